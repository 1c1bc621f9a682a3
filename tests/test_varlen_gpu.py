"""Variable-length batches: one token count per sequence on the device.

Sequences of 1000, 777, 512 and 33 tokens in one batch: the compressed and
the bf16 attention with per-sequence lengths agree bit for bit and each
sequence is within tolerance of the float64 attention over its own tokens;
then 40 decode steps through the device-length append (each sequence fills
its pages on its own steps) keep every stored value exact and the two
attentions identical.
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

LENS = [1000, 777, 512, 33]


def _check_seq(o, q, k, v, b, T):
    qb, kb, vb = to_bits(q[b:b + 1]), to_bits(k[b:b + 1]), to_bits(v[b:b + 1])
    ref = oatt.attention_f64(qb, kb, vb, T)
    got = bits_to_f32(to_bits(o[b:b + 1])).astype(np.float64)
    assert (np.abs(got - ref) / oatt.tolerance(qb, kb, vb, T, ref)).max() <= 1.0, b


def test_varlen_batch_prefill_and_steps():
    B, Hq, Hkv, TS, steps = len(LENS), 16, 4, 1088, 40
    k = synthetic.make_kv(B, TS, Hkv, seed=91, key=True, raw_frac=0.01)
    v = synthetic.make_kv(B, TS, Hkv, seed=92, key=False, raw_frac=0.01)
    kc = ekv.CompressedKV(B, TS, Hkv, 128)
    vc = ekv.CompressedKV(B, TS, Hkv, 128)
    for b, T in enumerate(LENS):
        kc.prefill_slot(b, k[b:b + 1, :T])
        vc.prefill_slot(b, v[b:b + 1, :T])
    lens = kc.lengths()
    assert lens.tolist() == LENS

    q = synthetic.make_q(B, Hq, seed=93)
    o_c = kernels.attention_compressed_devlen(q, kc, vc, lens, 0)
    o_r = kernels.attention_reference_devlen(q, k, v, lens, 0)
    assert torch.equal(o_c.view(torch.int16), o_r.view(torch.int16))
    for b, T in enumerate(LENS):
        _check_seq(o_c, q, k, v, b, T)

    for c in (kc, vc):
        c.ensure_headroom(steps // 16 + 2)
    for i in range(steps):
        pos = lens.long()
        bi = torch.arange(B, device="cuda")
        kc.append_dev(k[bi, pos].contiguous(), lens)
        vc.append_dev(v[bi, pos].contiguous(), lens)
        lens += 1
        kc.note_appended(1)
        vc.note_appended(1)
        if i % 13 == 12:
            qi = synthetic.make_q(B, Hq, seed=200 + i)
            a = kernels.attention_compressed_devlen(qi, kc, vc, lens, 0)
            r = kernels.attention_reference_devlen(qi, k, v, lens, 0)
            assert torch.equal(a.view(torch.int16), r.view(torch.int16)), i
    assert lens.tolist() == [T + steps for T in LENS] == kc.lens
    Tmax = max(kc.lens)
    for c, x in ((kc, k), (vc, v)):
        dec = kernels.decode_to_bf16(c.buffers(), Tmax)
        for b, T in enumerate(c.lens):
            assert torch.equal(dec[b, :T], x[b, :T]), b
    kernels.check_status()
