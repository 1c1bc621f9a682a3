"""Paged caches: the attention reads each sequence's pages through a block table
from a pool (exk_attention_compressed_paged / exk_attention_bf16_paged).

Three sequences of 1000, 513 and 260 tokens have their 16-token pages encoded
at random pages of a 256-page pool (the encoder writes any page of a cache:
encode_pages with that page's position). The paged call on the compressed
pool, the paged call on a bf16 pool with the same placement, and the
device-length call on the same sequences laid out contiguously agree bit for
bit, and each sequence is within tolerance of the float64 attention over its
own tokens. With 8 KV heads (8 consumer warps) and with 4 (4 warps).
"""
import numpy as np
import pytest
import torch

import exactkv_b200 as ekv
from exactkv_b200 import kernels, synthetic
from gpu_util import to_bits
from oracle import attention as oatt
from oracle.bf16 import bits_to_f32

pytestmark = pytest.mark.gpu

LENS = [1000, 513, 260]
MAX_PAGES = 64
POOL_B, POOL_TS = 4, 1024          # 256 pool pages


def _place(x, pool_c, pool_bf, perm):
    """Encode every page of x [B, MAX_PAGES*16, H, 128] that holds tokens at its
    pool page; returns the int32 block table [B, MAX_PAGES]."""
    B = x.shape[0]
    npp = POOL_TS // 16
    table = torch.zeros(B, MAX_PAGES, dtype=torch.int32)
    st = (x.stride(0), 16 * x.stride(1), x.stride(1), x.stride(2))
    i = 0
    for b, T in enumerate(LENS):
        for p in range(-(-T // 16)):
            phys = int(perm[i])
            i += 1
            table[b, p] = phys
            src = x[b:b + 1, p * 16:]
            kernels.encode_pages(src, st, pool_c.encoder_buffers(), phys // npp, phys % npp, 1, 1)
            pool_bf.view(-1, 16, x.shape[2], 128)[phys] = x[b, p * 16:(p + 1) * 16]
    assert int(pool_c.cnt.item()) <= pool_c.cap
    return table.cuda()


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (28, 4)])
def test_paged_attention_matches_contiguous(Hq, Hkv):
    B = len(LENS)
    TS = MAX_PAGES * 16
    k = synthetic.make_kv(B, TS, Hkv, seed=111, key=True, raw_frac=0.01)
    v = synthetic.make_kv(B, TS, Hkv, seed=112, key=False, raw_frac=0.01)
    q = synthetic.make_q(B, Hq, seed=113)
    perm = torch.randperm(POOL_B * POOL_TS // 16, generator=torch.Generator().manual_seed(114))
    kp, vp = (ekv.CompressedKV(POOL_B, POOL_TS, Hkv, 128, reserve=1.0) for _ in range(2))
    kbp, vbp = (torch.zeros(POOL_B, POOL_TS, Hkv, 128, dtype=torch.bfloat16, device="cuda") for _ in range(2))
    table = _place(k, kp, kbp, perm)
    assert torch.equal(_place(v, vp, vbp, perm), table)
    lens = torch.tensor(LENS, dtype=torch.int32, device="cuda")

    o_p = kernels.attention_paged(q, kp, vp, table, lens)
    o_r = kernels.attention_reference_paged(q, kbp, vbp, table, lens)
    assert torch.equal(o_p.view(torch.int16), o_r.view(torch.int16))

    kc, vc = (ekv.CompressedKV(B, TS, Hkv, 128, reserve=1.0) for _ in range(2))
    for b, T in enumerate(LENS):
        kc.prefill_slot(b, k[b:b + 1, :T].contiguous())
        vc.prefill_slot(b, v[b:b + 1, :T].contiguous())
    o_c = kernels.attention_compressed_devlen(q, kc, vc, lens, 0, num_warps=Hkv if Hkv < 8 else 8)
    assert torch.equal(o_p.view(torch.int16), o_c.view(torch.int16))

    for b, T in enumerate(LENS):
        qb, kb, vb = to_bits(q[b:b + 1]), to_bits(k[b:b + 1]), to_bits(v[b:b + 1])
        ref = oatt.attention_f64(qb, kb, vb, T)
        got = bits_to_f32(to_bits(o_p[b:b + 1])).astype(np.float64)
        assert (np.abs(got - ref) / oatt.tolerance(qb, kb, vb, T, ref)).max() <= 1.0, b
    kernels.check_status()


def test_paged_rejects_mismatched_warps_and_tables():
    """Host-side checks: a KV head count that is not a multiple of 4, and tables
    of the wrong shape or type, are refused before any launch."""
    B, Hq, Hkv = 1, 8, 2
    q = synthetic.make_q(B, Hq, seed=1)
    kp = ekv.CompressedKV(1, 256, Hkv, 128)
    table = torch.zeros(B, 16, dtype=torch.int32, device="cuda")
    lens = torch.full((B,), 100, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        kernels.attention_paged(q, kp, kp, table, lens)
    kp4 = ekv.CompressedKV(1, 256, 4, 128)
    q4 = synthetic.make_q(B, 16, seed=2)
    with pytest.raises(ValueError):
        kernels.attention_paged(q4, kp4, kp4, table.long(), lens)
    with pytest.raises(ValueError):
        kernels.attention_paged(q4, kp4, kp4, table[:, :8].t().contiguous(), lens)
