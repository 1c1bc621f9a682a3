"""Decode attention on the B200 kernels.

  * compressed == bf16 sibling, bit for bit (reference tests/test_exactkv.py:61-78,
    same shapes and data recipe, both consumer-warp counts);
  * both within oracle.attention.tolerance of the CPU restatement of the
    reference's split-K attention and of the float64 attention;
  * config 1 (golden float64 attention from the reference's test formula).
"""
import numpy as np
import pytest
import torch

import exactkv_b200 as ekv
from exactkv_b200 import kernels, synthetic
from gpu_util import same_bits, to_bits, to_dev
from oracle import attention as oatt
from oracle.bf16 import bits_to_f32
from synth_np import CONFIG1, config1_inputs

pytestmark = pytest.mark.gpu

REF_SHAPES = [(1, 4096, 28, 4), (3, 1000, 32, 8), (2, 333, 32, 32), (4, 17, 16, 2),
              (2, 1, 32, 8), (1, 16, 28, 4)]   # a single token; exactly one full page


def _compress(x):
    """[B, TS, H, D] bf16 -> a CompressedKV holding all TS tokens (prefill path)."""
    B, TS, H, D = x.shape
    c = ekv.CompressedKV(B, TS, H, D, reserve=1.0)
    for b in range(B):
        c.prefill_slot(b, x[b:b + 1].contiguous())
    return c


def _ref_test_data(B, T, Hq, Hkv, seed):
    """The reference test's recipe (tests/test_exactkv.py:64-69) on a CPU generator."""
    g = torch.Generator().manual_seed(seed)
    TS = -(-T // 16) * 16
    scale = torch.exp(torch.randn(Hkv, 128, generator=g) * 0.7)
    k = (torch.randn(B, TS, Hkv, 128, generator=g) * scale).to(torch.bfloat16)
    v = torch.randn(B, TS, Hkv, 128, generator=g).to(torch.bfloat16)
    k[:, ::97, :, 3] = 0.0
    q = (torch.randn(B, Hq, 128, generator=g) * 0.3).to(torch.bfloat16)
    return q.cuda(), k.cuda(), v.cuda()


def _check_close(o, q, k, v, T, ref=None):
    qb, kb, vb = to_bits(q), to_bits(k), to_bits(v)
    ref = oatt.attention_f64(qb, kb, vb, T) if ref is None else ref
    tol = oatt.tolerance(qb, kb, vb, T, ref)
    got = bits_to_f32(to_bits(o)).astype(np.float64)
    ratio = np.abs(got - ref) / tol
    assert ratio.max() <= 1.0, f"max err/tol {ratio.max():.3f}"
    orc = bits_to_f32(oatt.attention(qb, kb, vb, T)).astype(np.float64)
    ratio_o = np.abs(got - orc) / oatt.tolerance(qb, kb, vb, T, orc)
    assert ratio_o.max() <= 1.0, f"vs oracle: max err/tol {ratio_o.max():.3f}"
    return ratio.max()


@pytest.mark.parametrize("B,T,Hq,Hkv", REF_SHAPES)
def test_attention_bit_identical_and_close(B, T, Hq, Hkv):
    q, k, v = _ref_test_data(B, T, Hq, Hkv, seed=1 + B + T)
    kc, vc = _compress(k), _compress(v)
    for nw in (4, 8):
        o_c = kernels.attention_compressed(q, kc.buffers(), vc.buffers(), T, num_warps=nw)
        o_r = kernels.attention_reference(q, k, v, T, num_warps=nw)
        assert same_bits(o_c, o_r), (B, T, Hq, Hkv, nw)
        o_obj = kernels.attention_compressed(q, kc, vc, T, num_warps=nw)
        assert same_bits(o_obj, o_c)
        _check_close(o_c, q, k, v, T)
    kernels.check_status()


@pytest.mark.parametrize("case", CONFIG1, ids=[c["name"] for c in CONFIG1])
def test_attention_config1(golden, case):
    qn, kn, vn = config1_inputs(case)
    T = case["T"]
    q, k, v = to_dev(qn), to_dev(kn), to_dev(vn)
    # prefill exactly T tokens: full pages encoded, the tail page raw in the pool
    B, TS, H, D = k.shape
    kc, vc = ekv.CompressedKV(B, TS, H, D), ekv.CompressedKV(B, TS, H, D)
    for b in range(B):
        kc.prefill_slot(b, k[b:b + 1, :T].contiguous())
        vc.prefill_slot(b, v[b:b + 1, :T].contiguous())
    o_c = ekv.decode_attention(q, kc, vc)
    o_r = kernels.attention_reference(q, k, v, T)
    assert same_bits(o_c, o_r)
    _check_close(o_c, q, k, v, T, ref=golden["config1"][f"{case['name']}/attn_f64"])
    kernels.check_status()


@pytest.mark.parametrize("B,T,Hq,Hkv", [(1, 700, 12, 1), (2, 300, 16, 1), (2, 257, 9, 1), (1, 64, 1, 1)])
def test_attention_head_groups(B, T, Hq, Hkv):
    """G > 8 uses two n-tiles of heads; G = 1 pads seven."""
    q, k, v = _ref_test_data(B, T, Hq, Hkv, seed=7)
    kc, vc = _compress(k), _compress(v)
    o_c = kernels.attention_compressed(q, kc, vc, T)
    o_r = kernels.attention_reference(q, k, v, T)
    assert same_bits(o_c, o_r)
    _check_close(o_c, q, k, v, T)
    kernels.check_status()


def test_attention_llama_shaped_synthetic():
    """Llama-3.1-8B head layout (32 q / 8 kv) on the benchmark distribution
    (RoPE theta 5e5, 0.04% zeros, 0.3% forced raw rows), several splits per sequence."""
    B, T, Hq, Hkv = 4, 4096, 32, 8
    k = synthetic.make_kv(B, T, Hkv, seed=11, theta=5e5, key=True)
    v = synthetic.make_kv(B, T, Hkv, seed=12, theta=5e5, key=False)
    q = synthetic.make_q(B, Hq, seed=13)
    kc, vc = _compress(k), _compress(v)
    assert int(kc.cnt.item()) > 0 and int(vc.cnt.item()) > 0
    ns, _ = kernels.plan_splits(B, Hkv, T)
    assert ns > 1
    o_c = ekv.decode_attention(q, kc, vc)
    o_r = kernels.attention_reference(q, k, v, T)
    assert same_bits(o_c, o_r)
    _check_close(o_c, q, k, v, T)
    kernels.check_status()


@pytest.mark.parametrize("nw", [4, 8])
def test_attention_zero_groups_in_values(nw):
    """Exact zeros (and a denormal) in V make zero groups in V pages, which the kernels
    decode with the code-0 rule on a separate page body; some pages also carry
    raw rows, some end partly filled."""
    B, T, Hq, Hkv = 2, 1500, 32, 8
    TS = -(-T // 16) * 16
    k = synthetic.make_kv(B, TS, Hkv, seed=41, key=True)
    v = synthetic.make_kv(B, TS, Hkv, seed=42, key=False)
    g = torch.Generator(device="cuda").manual_seed(43)
    v = torch.where(torch.rand(v.shape, generator=g, device="cuda") < 2e-3, torch.zeros_like(v), v)
    v[:, 100:116, 3, 5] = 0.0                       # a whole page-channel of zeros
    v[1, 517, 6, 77] = torch.tensor(2.0 ** -130).to(torch.bfloat16)   # denormal in a zero group
    q = synthetic.make_q(B, Hq, seed=44)
    kc, vc = _compress(k), _compress(v)
    zg = (vc.base[:, :, :, :] >= 128).any(-1).float().mean().item()
    assert zg > 0.1, zg                             # a good share of V pages has a zero group
    o_c = kernels.attention_compressed(q, kc, vc, T, num_warps=nw)
    o_r = kernels.attention_reference(q, k, v, T, num_warps=nw)
    assert same_bits(o_c, o_r)
    _check_close(o_c, q, k, v, T)
    kernels.check_status()


def test_attention_split_subsets_match_full_run():
    """Running the plan's splits in two launches ([0, s) and [s, ns)) writes the same
    partials as one launch — the per-GPU step of a KV-sequence split."""
    B, T, Hq, Hkv = 1, 8192, 32, 8
    k = synthetic.make_kv(B, T, Hkv, seed=21, key=True)
    v = synthetic.make_kv(B, T, Hkv, seed=22, key=False)
    q = synthetic.make_q(B, Hq, seed=23)
    kc, vc = _compress(k), _compress(v)
    ns, sl = kernels.plan_splits(B, Hkv, T)
    assert ns >= 2
    ws_a = kernels._workspace(q.device, 1, B * Hq, ns, sl)   # private keys: not shared with other calls
    ws_b = kernels._workspace(q.device, 2, B * Hq, ns, sl)
    kernels.attention_split(q, kc, vc, T, ws_a, 0, ns)
    s = ns // 2
    kernels.attention_split(q, kc, vc, T, ws_b, 0, s)
    kernels.attention_split(q, kc, vc, T, ws_b, s, ns)
    for x, y in zip(ws_a[:3], ws_b[:3]):
        assert torch.equal(x, y)
    out = torch.empty_like(q)
    kernels.merge_partials(ws_b, B * Hq, out)
    assert same_bits(out, kernels.merge_partials(ws_a, B * Hq, torch.empty_like(q)))
    _check_close(out, q, k, v, T)
    kernels.check_status()


@pytest.mark.parametrize("heads", [1, 2, 4, 8])
def test_attention_heads_per_item(heads):
    """A plan may set the KV heads per work item (exk_partials.heads): 1, 2 and 4
    heads split each item's pages over the consumer warps and merge them inside
    the CTA. Compressed == bf16 partials bit for bit, the output within
    tolerance; T ends inside a page and the cache has forced raw rows."""
    B, T, Hq, Hkv = 1, 20000, 32, 8
    TS = -(-T // 16) * 16
    k = synthetic.make_kv(B, TS, Hkv, seed=61, key=True, raw_frac=0.02)
    v = synthetic.make_kv(B, TS, Hkv, seed=62, key=False, raw_frac=0.02)
    q = synthetic.make_q(B, Hq, seed=63)
    kc, vc = _compress(k), _compress(v)
    ns, sl = 37, 544
    ws_c = kernels._workspace(q.device, 11, B * Hq, ns, sl, heads)     # private keys
    ws_r = kernels._workspace(q.device, 12, B * Hq, ns, sl, heads)
    kernels.attention_split(q, kc, vc, T, ws_c, 0, ns)
    kernels.attention_split_bf16(q, k, v, T, ws_r, 0, ns)
    for x, y in zip(ws_c[:3], ws_r[:3]):
        assert torch.equal(x, y)
    out = kernels.merge_partials(ws_c, B * Hq, torch.empty_like(q))
    _check_close(out, q, k, v, T)
    kernels.check_status()


def test_attention_qwen_1x32k():
    """Qwen2.5-7B shape (28 q / 4 kv), one sequence of 32,768 tokens,
    RoPE theta 1e6: compressed == bf16 bit for bit, within tolerance of float64."""
    B, T, Hq, Hkv = 1, 32768, 28, 4
    k = synthetic.make_kv(B, T, Hkv, seed=51, theta=1e6, key=True)
    v = synthetic.make_kv(B, T, Hkv, seed=52, theta=1e6, key=False)
    q = synthetic.make_q(B, Hq, seed=53)
    kc, vc = _compress(k), _compress(v)
    o_c = ekv.decode_attention(q, kc, vc)
    o_r = kernels.attention_reference(q, k, v, T)
    assert same_bits(o_c, o_r)
    _check_close(o_c, q, k, v, T)
    kernels.check_status()


def test_attention_1x128k_raw_pool_stress():
    """BASELINE config 4 on one GPU: 32 q / 8 kv, 131,072 tokens with 2% forced raw rows,
    written page by page through the append path into a pool that starts too small
    (it must grow); compressed == bf16 bit for bit."""
    B, T, Hq, Hkv = 1, 131072, 32, 8
    k = synthetic.make_kv(B, T, Hkv, seed=61, theta=1e6, key=True, raw_frac=0.02)
    v = synthetic.make_kv(B, T, Hkv, seed=62, theta=1e6, key=False, raw_frac=0.02)
    q = synthetic.make_q(B, Hq, seed=63)
    T0 = T - 48
    kc = ekv.CompressedKV(B, T, Hkv, 128, reserve=0.005)
    vc = ekv.CompressedKV(B, T, Hkv, 128, reserve=0.005)
    kc.prefill_slot(0, k[:, :T0].contiguous())
    vc.prefill_slot(0, v[:, :T0].contiguous())
    for t in range(T0, T):
        kc.append(k[:, t])
        vc.append(v[:, t])
        if kc.T % 16 == 0:
            ekv.check_overflow([kc, vc])
    assert kc.grows + vc.grows > 0
    o_c = ekv.decode_attention(q, kc, vc)
    o_r = kernels.attention_reference(q, k, v, T)
    assert same_bits(o_c, o_r)
    assert same_bits(kernels.decode_to_bf16(kc.buffers(), T), k)
    kernels.check_status()


@pytest.mark.parametrize("B,T,Hq,Hkv,nw", [(40, 300, 32, 8, 8), (2, 8190, 32, 8, 8), (3, 1000, 28, 4, 8),
                                           (6, 777, 16, 2, 4), (5, 4096, 32, 8, 8)])
def test_balanced_plan(B, T, Hq, Hkv, nw):
    """The balanced plan (exk_partials.split_len = 0): every CTA gets an equal
    run of the call's stages, across sequence boundaries (many units per CTA at
    40 x 300; a unit cut into ~70 pieces at 2 x 8190, which takes the wide
    merge). The workspace has more columns than any unit needs, so the unit's
    last piece must close the rest with empty partials. Compressed == bf16 bit
    for bit, within tolerance of float64 and of the oracle, and within
    tolerance of the uniform plan's output."""
    TS = -(-T // 16) * 16
    k = synthetic.make_kv(B, TS, Hkv, seed=91, key=True, raw_frac=0.01)
    v = synthetic.make_kv(B, TS, Hkv, seed=92, key=False, raw_frac=0.01)
    q = synthetic.make_q(B, Hq, seed=93)
    kc, vc = _compress(k), _compress(v)
    ns = 160
    ws_c = kernels._workspace(q.device, 11, B * Hq, ns, 0)
    ws_r = kernels._workspace(q.device, 12, B * Hq, ns, 0)
    for ws in (ws_c, ws_r):                      # stale values in every column: all must be rewritten
        ws[0].fill_(float("nan"))
        ws[1].fill_(float("nan"))
        ws[2].fill_(float("nan"))
    kernels.attention_split(q, kc, vc, T, ws_c, 0, ns, num_warps=nw)
    kernels.attention_split_bf16(q, k, v, T, ws_r, 0, ns, num_warps=nw)
    o_c = kernels.merge_partials(ws_c, B * Hq, torch.empty_like(q))
    o_r = kernels.merge_partials(ws_r, B * Hq, torch.empty_like(q))
    assert same_bits(o_c, o_r)
    assert not torch.isnan(o_c.float()).any()
    _check_close(o_c, q, k, v, T)
    ns_u, sl_u = kernels.plan_splits(B, Hkv, T)
    ws_u = kernels._workspace(q.device, 13, B * Hq, ns_u, sl_u)
    kernels.attention_split(q, kc, vc, T, ws_u, 0, ns_u, num_warps=nw)
    o_u = kernels.merge_partials(ws_u, B * Hq, torch.empty_like(q))
    qb, kb, vb = to_bits(q), to_bits(k), to_bits(v)
    want = bits_to_f32(to_bits(o_u)).astype(np.float64)
    got = bits_to_f32(to_bits(o_c)).astype(np.float64)
    assert (np.abs(got - want) <= oatt.tolerance(qb, kb, vb, T, want)).all()
    kernels.check_status()


def test_whole_call_uses_the_balanced_plan_where_it_balances():
    """At the headline shape (32 x 4096, 8 KV heads, 148 SMs) equal splits leave
    the busiest CTAs 58 pages against an average of 55.35: the whole-call plan
    is the balanced one there, and the uniform one where items fill the waves."""
    assert kernels.call_plan(32, 8, 4096, num_ctas=148)[1] == 0
    assert kernels.call_plan(8, 8, 8192, num_ctas=148)[1] > 0
    assert kernels.call_plan(1, 4, 32768, num_ctas=148)[1] > 0


def _devlen_call(q, kc, vc, T_dev, ws, nw, bf16=False):
    """exk_attention_{compressed,bf16}_devlen (one length for the batch, T_add 0)
    over the given workspace: the kernels' own entry points with a chosen plan."""
    import ctypes
    from exactkv_b200._lib import lib
    B, Hq, _ = q.shape
    dev = q.device.index
    stream = torch.cuda.current_stream(q.device).cuda_stream
    out = torch.empty_like(q)
    common = (T_dev.data_ptr(), 0, 0, 0, ctypes.byref(ws[3]), out.data_ptr(), nw, 128 ** -0.5 * kernels.LOG2E,
              kernels.status_tensor(dev).data_ptr(), dev, stream)
    if bf16:
        TS, Hkv = kc.shape[1], kc.shape[2]
        rc = lib.exk_attention_bf16_devlen(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), B, TS, Hkv, Hq, TS, *common)
    else:
        ka, TS, Hkv = kernels._cache_args(kc)
        va, _, _ = kernels._cache_args(vc)
        rc = lib.exk_attention_compressed_devlen(q.data_ptr(), ctypes.byref(ka), ctypes.byref(va), B, TS, Hkv, Hq,
                                                 TS, *common)
    kernels.check(rc, "devlen")
    return out


@pytest.mark.parametrize("B,TS,Hq,Hkv,nw", [(32, 4096, 32, 8, 8), (3, 1008, 16, 2, 8), (5, 2048, 28, 4, 4)])
def test_devlen_balanced_plan_follows_the_device_length(B, TS, Hq, Hkv, nw):
    """A device-length call with one length for the batch over a balanced plan
    (split_len 0): the kernel cuts the stages of the length it reads into one
    equal run per SM, with ceil(SMs / units) + 1 workspace columns (the bound
    for every length; 51 at 3 x 1008 with 4 page phases per head, which takes
    the wide merge). At each length (fewer stages than SMs, ragged, the
    capacity) the output equals, bit for bit, the host-length call with the
    balanced plan at that length over the same columns, and the bf16 sibling's;
    at length 0 every column is closed with an empty partial. At the headline
    shape this is the plan the public device-length call picks."""
    sms = kernels.num_sms(0)
    hg = min(max(h for h in (1, 2, 4, 8) if Hkv % h == 0), nw)
    units = B * (Hkv // hg)
    ns = -(-sms // units) + 1
    if (B, TS) == (32, 4096):
        assert kernels.devlen_plan(B, Hkv, TS, torch.zeros(1, dtype=torch.int32, device="cuda"), num_warps=nw) == (ns, 0)
    k = synthetic.make_kv(B, TS, Hkv, seed=95, key=True, raw_frac=0.01)
    v = synthetic.make_kv(B, TS, Hkv, seed=96, key=False, raw_frac=0.01)
    q = synthetic.make_q(B, Hq, seed=97)
    kc, vc = _compress(k), _compress(v)
    ws_d = kernels._workspace(q.device, 21, B * Hq, ns, 0)
    ws_h = kernels._workspace(q.device, 22, B * Hq, ns, 0)
    ws_r = kernels._workspace(q.device, 23, B * Hq, ns, 0)
    T_dev = torch.zeros(1, dtype=torch.int32, device="cuda")
    for ws in (ws_d, ws_h, ws_r):
        for t in ws[:3]:
            t.fill_(float("nan"))
    _devlen_call(q, kc, vc, T_dev, ws_d, nw)
    torch.cuda.synchronize()
    assert torch.all(ws_d[1] == float("-inf")) and torch.all(ws_d[2] == 0) and torch.all(ws_d[0] == 0)
    for T in (1, 16, 100, TS // 2 + 37, TS - 1, TS):
        T_dev.fill_(T)
        o_d = _devlen_call(q, kc, vc, T_dev, ws_d, nw)
        o_r = _devlen_call(q, k, v, T_dev, ws_r, nw, bf16=True)
        kernels.attention_split(q, kc, vc, T, ws_h, 0, ns, num_warps=nw)
        o_h = kernels.merge_partials(ws_h, B * Hq, torch.empty_like(q))
        assert same_bits(o_d, o_h), T
        assert same_bits(o_d, o_r), T
        assert not torch.isnan(o_d.float()).any(), T
        if T == 100:
            _check_close(o_d, q, k, v, T)
    kernels.check_status()
