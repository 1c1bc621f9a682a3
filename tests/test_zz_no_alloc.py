"""exk_attention_compressed_noalloc: compressed decode attention for callers that
cannot allocate device memory when they call (a runtime that plans all device
memory up front, a plugin whose enqueue must not call cudaMalloc). It keeps its
split partials in a fixed array inside the library instead of a workspace.

Checked through the C ABI against the allocating entry points
(exk_attn_split_compressed + exk_attn_merge with a torch workspace) on two calls in
a row — the second reuses the array the first left behind — within the tolerance
the attention tests use (oracle.attention.tolerance), and bit for bit, since both
run the same kernels on the same split plan. Also: a request whose partials do not
fit the array is refused with EXK_ESCRATCH. This file is named to be collected
last; it passes on its own in a fresh process as well.
"""
import ctypes

import numpy as np
import pytest
import torch

import exactkv_b200 as ekv
from exactkv_b200 import kernels
from exactkv_b200._lib import lib
from gpu_util import to_bits
from oracle import attention as oatt
from oracle.bf16 import bits_to_f32

pytestmark = pytest.mark.gpu

EXK_ESCRATCH = -6
SCALE = 128 ** -0.5 * kernels.LOG2E


def _call_noalloc(q, kc, vc, T, out, num_warps=8):
    dev = q.device.index
    stream = torch.cuda.current_stream(q.device).cuda_stream
    return lib.exk_attention_compressed_noalloc(
        q.data_ptr(), ctypes.byref(kc.kernel_view()), ctypes.byref(vc.kernel_view()), q.shape[0], kc.TS, kc.H,
        q.shape[1], T, num_warps, SCALE, out.data_ptr(), kernels.status_tensor(dev).data_ptr(), dev, stream)


def _cache(x):
    B, TS, H, D = x.shape
    c = ekv.CompressedKV(B, TS, H, D)
    for b in range(B):
        c.prefill_slot(b, x[b:b + 1].contiguous())
    return c


@pytest.mark.parametrize("B,T,Hq,Hkv", [(4, 1000, 32, 8), (2, 2048, 28, 4)])
def test_noalloc_matches_allocating_entry_point(B, T, Hq, Hkv):
    g = torch.Generator().manual_seed(31 + T)
    TS = -(-T // 16) * 16
    scale = torch.exp(torch.randn(Hkv, 128, generator=g) * 0.7)
    k = (torch.randn(B, TS, Hkv, 128, generator=g) * scale).to(torch.bfloat16)
    v = torch.randn(B, TS, Hkv, 128, generator=g).to(torch.bfloat16)
    k[:, 5::61, :, 9] = 1e-30                                  # some raw rows
    kc, vc = _cache(k.cuda()), _cache(v.cuda())
    qs = [torch.randn(B, Hq, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(2)]
    kb, vb = to_bits(k), to_bits(v)
    for q in qs:                                               # two calls in a row
        out = torch.empty_like(q)
        assert _call_noalloc(q, kc, vc, T, out) == 0
        # the allocating entry points on the same (uniform) plan: exk_attn_split_compressed
        # over every split into a torch workspace, then exk_attn_merge
        ns, sl = kernels.plan_splits(B, Hkv, T)
        ws = kernels._workspace(q.device, 3, B * Hq, ns, sl)       # a private workspace key
        kernels.attention_split(q, kc, vc, T, ws, 0, ns)
        ref = kernels.merge_partials(ws, B * Hq, torch.empty_like(q))
        got = bits_to_f32(to_bits(out)).astype(np.float64)
        want = bits_to_f32(to_bits(ref)).astype(np.float64)
        tol = oatt.tolerance(to_bits(q), kb, vb, T, want)
        assert (np.abs(got - want) <= tol).all()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    kernels.check_status()


def test_noalloc_rejects_requests_beyond_its_scratch():
    # 16 query heads per KV head: B*Hq x splits x 130 fp32 outgrows the 4 MiB array
    for B, T, Hq, Hkv in [(64, 4096, 16, 1), (128, 4096, 16, 1), (256, 4096, 16, 1), (512, 2048, 16, 1)]:
        ns, _ = kernels.plan_splits(B, Hkv, T)
        if B * Hq * ns * 130 * 4 > 4 << 20:
            break
    else:
        pytest.fail("no candidate shape exceeds the scratch")
    kc = ekv.CompressedKV(B, T, Hkv, 128)
    q = torch.zeros(B, Hq, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(q)
    assert _call_noalloc(q, kc, kc, T, out) == EXK_ESCRATCH
    assert b"fixed scratch" in lib.exk_error_string(EXK_ESCRATCH)
