"""GPU page encoder and decoder against the reference's bytes (golden vectors)
and the CPU oracle. Mirrors tests/test_exactkv.py:46-58 of the reference, and
extends it: rowoff and raw are compared too (the encoder is deterministic)."""
import numpy as np
import pytest
import torch

import exactkv_b200 as ekv
from exactkv_b200 import kernels
from gpu_util import same_bits, to_bits, to_dev
from oracle import codec as ocodec
from synth_np import CONFIG1, config1_inputs, digest

pytestmark = pytest.mark.gpu

FIELDS = ("sm", "code", "base", "rowmask", "rowoff", "raw")
CASES = ("patterns", "specials", "constant", "zeros")


def _np(c, f):
    t = c[f]
    return to_bits(t) if f == "raw" else t.cpu().numpy()


@pytest.mark.parametrize("name", CASES)
def test_gpu_encoder_matches_reference_bytes(golden, name):
    g = golden["codec"]
    x = to_dev(g[f"{name}/input"])
    c = ekv.encode_reference(x)
    for f in FIELDS:
        assert np.array_equal(_np(c, f), g[f"{name}/{f}"]), (name, f)
    kernels.check_status()


@pytest.mark.parametrize("name", CASES)
def test_gpu_decode_roundtrip(golden, name):
    x = to_dev(golden["codec"][f"{name}/input"])
    c = ekv.encode_reference(x)
    assert same_bits(ekv.decode_reference(c), x)
    kernels.check_status()


@pytest.mark.parametrize("case", CONFIG1, ids=[c["name"] for c in CONFIG1])
def test_gpu_encoder_config1_digests(golden, case):
    g = golden["config1"]
    _, k, v = config1_inputs(case)
    Tf = case["T"] // 16 * 16
    for tag, x in (("k", k), ("v", v)):
        c = ekv.encode_reference(to_dev(x[:, :Tf]))
        for f in FIELDS:
            assert digest(_np(c, f)) == str(g[f"{case['name']}/{tag}/digest_{f}"]), (case["name"], tag, f)
    kernels.check_status()


def _codable_patterns():
    """Every sign|mantissa byte with every exponent the format codes without a raw
    row (0..142), in pages whose 16 tokens share one exponent per channel; plus pages
    where exponent 0 sits in a group with exponents up to 15 steps above (zero groups)."""
    exps = np.arange(0, 143)
    smb = np.arange(256)
    # group = (exponent, block of 16 sign|mantissa bytes): 143 * 16 groups of 16 tokens
    groups = [(e, blk) for e in exps for blk in range(16)]
    n_ch = 128
    n_pages = -(-len(groups) // n_ch)
    x = np.zeros((1, n_pages * 16, 1, 128), np.uint16)
    for gi, (e, blk) in enumerate(groups):
        p, ch = divmod(gi, n_ch)
        s = smb[blk * 16:(blk + 1) * 16]
        x[0, p * 16:(p + 1) * 16, 0, ch] = ((s & 0x80) << 8) | (e << 7) | (s & 0x7F)
    # zero groups: token 0 exponent 0 (any mantissa), tokens 1..15 exponents e0-14..e0
    z = np.zeros((1, 16 * 8, 1, 128), np.uint16)
    rng = np.random.default_rng(5)
    for p in range(8):
        for ch in range(128):
            e0 = 16 + (p * 128 + ch) % 112
            es = np.concatenate([[0], e0 - rng.integers(0, 15, size=15)])
            s = rng.integers(0, 256, size=16)
            z[0, p * 16:(p + 1) * 16, 0, ch] = ((s & 0x80) << 8) | (es << 7) | (s & 0x7F)
    return np.concatenate([x, z], axis=1)


def test_gpu_codec_exhaustive_codable_values():
    x = _codable_patterns()
    ref = ocodec.encode(x)
    assert ref["raw"].shape[0] == 0, "construction must not need raw rows"
    c = ekv.encode_reference(to_dev(x))
    for f in FIELDS:
        assert np.array_equal(_np(c, f), ref[f]), f
    assert np.array_equal(to_bits(ekv.decode_reference(c)), x)
    # every sign|mantissa byte and every exponent 0..142 occurs
    e = (x.astype(np.int32) >> 7) & 0xFF
    assert set(np.unique(e)) == set(range(143))
    kernels.check_status()


def test_gpu_encoder_strided_and_unaligned_sources():
    """Source views with head-major strides ([1, H, T, D] transposed, the HF prefill
    layout) and a 2-byte-offset start (the scalar-load path) give the same bytes."""
    _, k, _ = config1_inputs(CONFIG1[0])
    x = to_dev(k[:1, :512])                             # [1, 512, 2, 128]
    ref = ocodec.encode(k[:1, :512])
    hf = x.transpose(1, 2).contiguous().transpose(1, 2)  # same values, strides (T*H*D, D, T*D, 1)
    assert hf.stride(1) == 128
    flat = torch.empty(hf.numel() + 1, dtype=torch.bfloat16, device="cuda")
    shifted = flat[1:].view(1, 512, 2, 128)
    shifted.copy_(x)
    for src in (hf, shifted):
        B, T, H, D = src.shape
        c = ekv.CompressedKV(B, T, H, D, reserve=1.0)
        st = (src.stride(0), 16 * src.stride(1), src.stride(1), src.stride(2))
        kernels.encode_pages(src, st, c.encoder_buffers(), 0, 0, B, T // 16)
        n = int(c.cnt.item())
        for f in ("sm", "code", "base", "rowmask", "rowoff"):
            assert np.array_equal(getattr(c, f).cpu().numpy(), ref[f]), f
        assert np.array_equal(to_bits(c.raw[:n]), ref["raw"])
    kernels.check_status()


def test_gpu_encoder_pool_overflow_counts_and_skips():
    """With a pool smaller than the raw rows, cnt still counts every raw row and no
    slot at or past cap is written (the host then grows and re-encodes)."""
    x = np.full((1, 64, 4, 128), 0x3F80, np.uint16)      # 1.0
    x[0, ::3, :, 7] = 0x0080                              # 2^-126: escapes, row raw
    ref = ocodec.encode(x)
    nraw = ref["raw"].shape[0]
    assert nraw > 8
    c = ekv.CompressedKV(1, 64, 4, 128)
    buf = c.encoder_buffers()
    buf["cap"] = 8                                        # a pool smaller than needed
    sentinel = torch.full_like(c.raw, 7.0)
    c.raw.copy_(sentinel)
    xs = to_dev(x)
    kernels.encode_pages(xs, (xs.stride(0), 16 * xs.stride(1), xs.stride(1), xs.stride(2)), buf, 0, 0, 1, 4)
    assert int(c.cnt.item()) == nraw
    assert np.array_equal(to_bits(c.raw[:8]), ref["raw"][:8])
    assert same_bits(c.raw[8:], sentinel[8:])
    for f in ("sm", "code", "base", "rowmask", "rowoff"):
        assert np.array_equal(getattr(c, f).cpu().numpy(), ref[f]), f
    kernels.check_status()


def test_bounded_wait_reports_timeout():
    """Failure detection without a fault: a wait on a barrier that nothing completes
    gives up after its limit and reports EXK_S_FULL_TIMEOUT in the status word;
    the context stays usable (a kernel call right after works)."""
    import time
    from exactkv_b200 import _lib
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    rc = _lib.lib.exk_selftest_wait_timeout(st.data_ptr(), 5_000_000, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert int(st.item()) == 1                       # EXK_S_FULL_TIMEOUT
    assert time.perf_counter() - t0 < 2.0
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum().item()) == 8.0
