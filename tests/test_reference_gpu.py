"""Parity against the reference implementation itself, run on the same B200.

When the unmodified reference package is installed in baseline/_ref (git-ignored;
`pip install --no-deps --target baseline/_ref <reference checkout>`), its Triton
kernels run here beside ours on the same inputs:

  * its GPU encoder and ours write the same sm, code, base and rowmask bytes
    (raw-pool slot order differs: the reference takes slots with an atomic per
    page-head), and both caches decode to the source bits;
  * its compressed attention and ours agree within the stated tolerance of
    oracle.attention.tolerance, and each is within it of float64.

Skipped when baseline/_ref is absent (the package is not part of this
repository) or Triton cannot compile for this GPU.
"""
import os
import sys

import numpy as np
import pytest
import torch

import exactkv_b200 as ekv
from exactkv_b200 import kernels, synthetic
from gpu_util import to_bits
from oracle import attention as oatt
from oracle.bf16 import bits_to_f32

pytestmark = pytest.mark.gpu

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def _reference():
    if not os.path.isdir(os.path.join(REF, "exactkv")):
        pytest.skip("reference package not installed in baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import exactkv  # the reference
    return exactkv


def _f64_ratio(o, q, k, v, T):
    qb, kb, vb = to_bits(q), to_bits(k), to_bits(v)
    f64 = oatt.attention_f64(qb, kb, vb, T)
    got = bits_to_f32(to_bits(o)).astype(np.float64)
    return (np.abs(got - f64) / oatt.tolerance(qb, kb, vb, T, f64)).max()


@pytest.mark.parametrize("B,T,Hq,Hkv,theta", [(4, 1000, 32, 8, 5e5), (1, 4096, 28, 4, 1e6)])
def test_against_the_reference_kernels(B, T, Hq, Hkv, theta):
    ref = _reference()
    TS = -(-T // 16) * 16
    k = synthetic.make_kv(B, TS, Hkv, seed=201, theta=theta, key=True)
    v = synthetic.make_kv(B, TS, Hkv, seed=202, theta=theta, key=False)
    q = synthetic.make_q(B, Hq, seed=203)
    rk, rv = ref.CompressedKV(B, TS, Hkv, 128, reserve=1.0), ref.CompressedKV(B, TS, Hkv, 128, reserve=1.0)
    ok, ov = ekv.CompressedKV(B, TS, Hkv, 128, reserve=1.0), ekv.CompressedKV(B, TS, Hkv, 128, reserve=1.0)
    try:
        for b in range(B):
            rk.prefill_slot(b, k[b:b + 1, :T].contiguous())
            rv.prefill_slot(b, v[b:b + 1, :T].contiguous())
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001 - Triton cannot build the reference here
        pytest.skip(f"reference kernels unavailable: {type(e).__name__}: {str(e)[:120]}")
    for b in range(B):
        ok.prefill_slot(b, k[b:b + 1, :T].contiguous())
        ov.prefill_slot(b, v[b:b + 1, :T].contiguous())

    full = T // 16
    for r, o, x in ((rk, ok, k), (rv, ov, v)):
        for f in ("sm", "code"):
            assert torch.equal(getattr(r, f)[:, :full * 16], getattr(o, f)[:, :full * 16]), f
        for f in ("base", "rowmask"):
            assert torch.equal(getattr(r, f)[:, :full], getattr(o, f)[:, :full]), f
        assert int(r.cnt.item()) == int(o.cnt.item())
        assert torch.equal(ref.decode_to_bf16(r.buffers(), T), x[:, :T])
        assert torch.equal(kernels.decode_to_bf16(o.buffers(), T), x[:, :T])

    o_ref = ref.attention_compressed(q, rk, rv, T)
    o_ours = ekv.decode_attention(q, ok, ov)
    torch.cuda.synchronize()
    qb, kb, vb = to_bits(q), to_bits(k), to_bits(v)
    base = bits_to_f32(to_bits(o_ref)).astype(np.float64)
    got = bits_to_f32(to_bits(o_ours)).astype(np.float64)
    assert (np.abs(got - base) / oatt.tolerance(qb, kb, vb, T, base)).max() <= 1.0
    assert _f64_ratio(o_ours, q, k, v, T) <= 1.0
    assert _f64_ratio(o_ref, q, k, v, T) <= 1.0
    kernels.check_status()


# ---------------------------------------------------------------------------- absolute error vs the reference
#
# The stated bound for floating point: max |ours - reference| <= 2e-3 on the
# attention outputs (V ~ N(0, 1): the reference test's own recipe,
# tests/test_exactkv.py:61-78 of the reference). Both kernels end by rounding
# to bf16, whose step is 2^-8 = 3.9e-3 for outputs in [0.5, 1); two correct
# kernels that block the softmax differently (the reference: 64-token blocks
# and choose_split's splits; here: 16-token pages and the SM-balanced plan)
# round a few such outputs to neighbouring bf16 values. So each config reports
#   f32   max |ours - ref| of the outputs before the final bf16 rounding (both
#         merged in float64 from the kernels' own fp32 split partials), and
#   bf16  max |ours - ref| of the returned bf16 outputs, with the largest
#         difference in units of the output's bf16 step,
# and asserts, per element, bf16 |ours - ref| <= max(2e-3, one bf16 step of the
# output), and at the f32 level <= 2e-3 on N(0, 1) data. For the synthetic
# configs, whose V channels are scaled by up to 2^3 (outputs up to ~17, where
# one bf16 step is 2^-3), the reference's own error sets the f32 bound:
# max |ours - ref| <= max |ref - float64|.

def _merged64(o, m, l):
    """float64 out [rows, 128] from split partials o [rows, ns, 128], m, l [rows, ns]."""
    o, m, l = o.double(), m.double(), l.double()
    M = m.max(-1, keepdim=True).values
    w = torch.where(torch.isinf(m), torch.zeros_like(m), torch.exp2(m - M))
    return (o * w[..., None]).sum(1) / (l * w).sum(-1, keepdim=True)


def _f64_attention(q, k, v, T):
    """softmax(q k^T / sqrt(D)) v in float64 on the GPU (GQA head sharing)."""
    B, Hq, D = q.shape
    G = Hq // k.shape[2]
    kf = k[:, :T].double().repeat_interleave(G, 2)
    s = torch.einsum("bhd,bthd->bht", q.double(), kf) / D ** 0.5
    del kf
    p = s.softmax(-1)
    return torch.einsum("bht,bthd->bhd", p, v[:, :T].double().repeat_interleave(G, 2))


def _bf16_step(x):
    """The bf16 rounding step (ulp) at |x| (float64 tensor), 2^-133 floor."""
    e = torch.floor(torch.log2(x.abs().clamp_min(2.0 ** -126)))
    return torch.exp2(e - 7)


def _ref_cache(ref, x, T):
    B, TS, H, _ = x.shape
    c = ref.CompressedKV(B, TS, H, 128, reserve=1.0)
    for b in range(B):
        c.prefill_slot(b, x[b:b + 1, :T].contiguous())
    return c


def _our_cache(x, T):
    B, TS, H, _ = x.shape
    c = ekv.CompressedKV(B, TS, H, 128, reserve=0.05)
    for b in range(B):
        c.prefill_slot(b, x[b:b + 1, :T].contiguous())
    return c


def _recipe(B, T, Hq, Hkv, seed):
    """The reference test's inputs (its test_attention_bit_identical), from a CPU generator."""
    g = torch.Generator().manual_seed(seed)
    TS = -(-T // 16) * 16
    scale = torch.exp(torch.randn(Hkv, 128, generator=g) * 0.7)
    k = (torch.randn(B, TS, Hkv, 128, generator=g) * scale).to(torch.bfloat16)
    v = torch.randn(B, TS, Hkv, 128, generator=g).to(torch.bfloat16)
    k[:, ::97, :, 3] = 0.0
    q = (torch.randn(B, Hq, 128, generator=g) * 0.3).to(torch.bfloat16)
    return q.cuda(), k.cuda(), v.cuda()


def _synthetic(B, T, Hq, Hkv, theta, raw_frac, seed):
    k = synthetic.make_kv(B, T, Hkv, seed=seed, theta=theta, key=True, raw_frac=raw_frac)
    v = synthetic.make_kv(B, T, Hkv, seed=seed + 1, theta=theta, key=False, raw_frac=raw_frac)
    return synthetic.make_q(B, Hq, seed=seed + 2), k, v


CASES = [
    # name, kind, B, T, Hq, Hkv, theta, raw_frac
    ("reference recipe 1x4096 28q/4kv", "recipe", 1, 4096, 28, 4, None, None),
    ("reference recipe 3x1000 32q/8kv", "recipe", 3, 1000, 32, 8, None, None),
    ("reference recipe 2x333 32q/32kv", "recipe", 2, 333, 32, 32, None, None),
    ("reference recipe 4x17 16q/2kv", "recipe", 4, 17, 16, 2, None, None),
    ("config 2: Qwen2.5-7B 1x32768 28q/4kv", "synthetic", 1, 32768, 28, 4, 1e6, 3e-3),
    ("config 3: Llama-3.1-8B 4x4096 32q/8kv", "synthetic", 4, 4096, 32, 8, 5e5, 3e-3),
    ("config 3: Llama-3.1-8B 2x8192 32q/8kv", "synthetic", 2, 8192, 32, 8, 5e5, 3e-3),
    ("config 4: 1x131072 32q/8kv, 2% raw rows", "synthetic", 1, 131072, 32, 8, 1e6, 2e-2),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_absolute_error_against_the_reference(case):
    name, kind, B, T, Hq, Hkv, theta, raw_frac = case
    ref = _reference()
    if kind == "recipe":
        q, k, v = _recipe(B, T, Hq, Hkv, seed=7 + T)
    else:
        q, k, v = _synthetic(B, T, Hq, Hkv, theta, raw_frac, seed=300 + T % 1000)
    try:
        rk, rv = _ref_cache(ref, k, T), _ref_cache(ref, v, T)
        o_ref = ref.attention_compressed(q, rk, rv, T)
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001 - Triton cannot build the reference here
        pytest.skip(f"reference kernels unavailable: {type(e).__name__}: {str(e)[:120]}")
    ns_r, _ = ref.kernels.choose_split(B, Hkv, T, 64)
    stream = torch.cuda.current_stream().cuda_stream
    wr = ref.kernels._WS[(q.device.index, stream, B * Hq, ns_r, 128)]
    ref32 = _merged64(*wr)
    ok, ov = _our_cache(k, T), _our_cache(v, T)
    o_ours = kernels.attention_compressed(q, ok, ov, T)
    ns_o, _ = kernels.call_plan(B, Hkv, T)
    wo = kernels._WS[(q.device.index, stream, B * Hq, ns_o)]
    ours32 = _merged64(*wo[:3])
    assert torch.equal(o_ours.view(torch.int16), kernels.attention_reference(q, k, v, T).view(torch.int16))
    f64 = _f64_attention(q, k, v, T).reshape(B * Hq, 128)
    a, r = o_ours.double().reshape(B * Hq, 128), o_ref.double().reshape(B * Hq, 128)
    d16 = (a - r).abs()
    d32 = (ours32 - ref32).abs().max().item()
    worst = int(d16.argmax())
    w_out = r.flatten()[worst].abs().item()
    # per element: 2e-3, or one bf16 step of the larger output where that step is coarser
    allowed16 = torch.clamp(_bf16_step(torch.maximum(a.abs(), r.abs())), min=2e-3)
    ref_err16 = (r - f64).abs().max().item()
    ref_err32 = (ref32 - f64).abs().max().item()
    ours_err16 = (a - f64).abs().max().item()
    line = (f"[parity] {name}: max|ours-ref| bf16 {d16.max().item():.3g} (worst at |out| {w_out:.3g}, "
            f"bf16 step there {_bf16_step(torch.tensor(w_out, dtype=torch.float64)).item():.3g}), "
            f"f32 {d32:.3g}; max|ref-f64| bf16 {ref_err16:.3g} f32 {ref_err32:.3g}; max|ours-f64| bf16 "
            f"{ours_err16:.3g}; max|out| {r.abs().max().item():.3g}; splits ours {ns_o} ref {ns_r}")
    print(line)
    log = os.environ.get("EXK_PARITY_LOG")
    if log:
        with open(log, "a") as f:
            f.write(line + "\n")
    assert (d16 <= allowed16).all(), line
    if kind == "recipe":
        assert d32 <= 2e-3, line
    else:
        assert d32 <= max(ref_err32, 2e-3), line
    kernels.check_status()
