"""The CPU oracle against golden vectors made by the reference implementation
(tests/golden/make_golden.py). No GPU needed."""
import numpy as np
import pytest

from oracle import attention as oatt
from oracle import codec as ocodec
from oracle.bf16 import bits_to_f32, f32_to_bits
from synth_np import CONFIG1, config1_inputs, digest

FIELDS = ("sm", "code", "base", "rowmask", "rowoff", "raw")
CASES = ("patterns", "specials", "constant", "zeros")


@pytest.mark.parametrize("name", CASES)
def test_oracle_encode_matches_reference_bytes(golden, name):
    g = golden["codec"]
    x = g[f"{name}/input"]
    c = ocodec.encode(x)
    for f in FIELDS:
        assert np.array_equal(c[f], g[f"{name}/{f}"]), (name, f)


@pytest.mark.parametrize("name", CASES)
def test_oracle_roundtrip(golden, name):
    x = golden["codec"][f"{name}/input"]
    assert np.array_equal(ocodec.decode(ocodec.encode(x)), x)


def test_all_65536_patterns_present(golden):
    x = golden["codec"]["patterns/input"]
    assert np.array_equal(np.sort(x.ravel()), np.arange(65536, dtype=np.uint16))


@pytest.mark.parametrize("case", CONFIG1, ids=[c["name"] for c in CONFIG1])
def test_oracle_config1_digests(golden, case):
    g = golden["config1"]
    q, k, v = config1_inputs(case)
    assert str(g[f"{case['name']}/digest_q"]) == digest(q), "numpy generator changed: regenerate fixtures"
    Tf = case["T"] // 16 * 16
    for tag, x in (("k", k), ("v", v)):
        assert str(g[f"{case['name']}/digest_{tag}"]) == digest(x), "numpy generator changed"
        c = ocodec.encode(x[:, :Tf])
        for f in FIELDS:
            assert str(g[f"{case['name']}/{tag}/digest_{f}"]) == digest(c[f]), (case["name"], tag, f)
        assert np.array_equal(c["rowmask"], g[f"{case['name']}/{tag}/rowmask"])
        assert np.array_equal(ocodec.decode(c), x[:, :Tf])


@pytest.mark.parametrize("case", CONFIG1, ids=[c["name"] for c in CONFIG1])
def test_oracle_attention_vs_reference_f64(golden, case):
    """The fp32 restatement of the reference's split-K attention against the float64
    attention of the reference's test (tests/test_exactkv.py:75-78).

    Tolerance (oracle.attention.tolerance): |o - ref| <= 2^-8 sum_t p_t|v_t| +
    2^-8 |ref| — one bf16 rounding step of each P.V product plus one of the output.
    Config-1 outputs reach |o| ~ 15 (V channels scaled up to 2^3), where one bf16
    ulp is 2^-4, so a fixed 2e-3 absolute bound cannot hold for any bf16 output."""
    q, k, v = config1_inputs(case)
    o = bits_to_f32(oatt.attention(q, k, v, case["T"])).astype(np.float64)
    ref = golden["config1"][f"{case['name']}/attn_f64"]
    tol = oatt.tolerance(q, k, v, case["T"], ref)
    assert (np.abs(o - ref) <= tol).all()
    assert (np.abs(o - ref) / tol).max() < 0.75   # with margin at these inputs


def test_oracle_choose_split_rule():
    # exactkv/kernels.py:273-277 at the shapes the survey lists
    assert oatt.choose_split(32, 8, 4096, 64) == (2, 2048)
    assert oatt.choose_split(8, 8, 8192, 64) == (8, 1024)
    assert oatt.choose_split(1, 8, 131072, 64) == (64, 2048)
    assert oatt.choose_split(1, 4, 32768, 64) == (128, 256)


def test_bf16_conversion_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, np.inf, -np.inf, 0.0, -0.0], np.float32)
    assert np.array_equal(bits_to_f32(f32_to_bits(x)), np.array([1.0, 1.0, 1.015625, -2.5, np.inf, -np.inf, 0.0, -0.0],
                                                                  np.float32))
    assert np.isnan(bits_to_f32(f32_to_bits(np.array([np.nan], np.float32))))[0]


@pytest.mark.parametrize("case", CONFIG1, ids=lambda c: c["name"])
def test_oracle_two_level_merge(case):
    """The KV-sequence split's two-level merge (oracle.attention.merge_group per run
    of splits, then merge over the runs) against the float64 attention, with the
    same tolerance as the one-level merge; a run of one split is that split's
    partial unchanged, and empty splits (m = -inf) weigh nothing."""
    q, k, v = config1_inputs(case)
    T = case["T"]
    B, Hq, D = q.shape
    ns = 7
    per = -(-T // ns)
    sl = -(-per // 16) * 16              # ns splits of whole pages covering T
    o, m, l = oatt.split_partials(q, k, v, T, splits=(ns, sl))
    rows = B * Hq
    o, m, l = o.reshape(rows, ns, D), m.reshape(rows, ns), l.reshape(rows, ns)
    for bounds in ([0, 3, 7], [0, 1, 2, 4, 7], [0, 7]):
        groups = [oatt.merge_group(o[:, a:b], m[:, a:b], l[:, a:b]) for a, b in zip(bounds, bounds[1:])]
        go = np.stack([g[0] for g in groups], 1)
        gm = np.stack([g[1] for g in groups], 1)
        gl = np.stack([g[2] for g in groups], 1)
        out = bits_to_f32(f32_to_bits(oatt.merge(go, gm, gl))).reshape(B, Hq, D).astype(np.float64)
        ref = oatt.attention_f64(q, k, v, T)
        assert (np.abs(out - ref) <= oatt.tolerance(q, k, v, T, ref)).all(), bounds
    g1 = oatt.merge_group(o[:, 2:3], m[:, 2:3], l[:, 2:3])
    assert np.array_equal(g1[0], o[:, 2]) and np.array_equal(g1[1], m[:, 2]) and np.array_equal(g1[2], l[:, 2])
    m2 = m.copy()
    m2[:, 5] = -np.inf
    ge = oatt.merge_group(np.where(np.isneginf(m2)[..., None], 0, o), m2, np.where(np.isneginf(m2), 0, l))
    gd = oatt.merge_group(np.delete(o, 5, 1), np.delete(m, 5, 1), np.delete(l, 5, 1))
    assert all(np.array_equal(a, b) for a, b in zip(ge, gd))


def test_torch_attention_restatement_matches_the_numpy_oracle():
    """bench.py's CPU baseline states the reference attention in torch
    (oracle/torch_attention.py); it agrees with the numpy oracle within the
    stated tolerance, partial last pages and several splits included."""
    import torch

    from oracle import torch_attention
    rng = np.random.default_rng(5)
    for B, T, Hq, Hkv in [(2, 1000, 8, 2), (1, 777, 28, 4), (3, 100, 16, 2)]:
        TS = -(-T // 16) * 16
        k = (rng.standard_normal((B, TS, Hkv, 128)) * np.exp(rng.standard_normal((Hkv, 128)))).astype(np.float32)
        v = rng.standard_normal((B, TS, Hkv, 128)).astype(np.float32)
        q = rng.standard_normal((B, Hq, 128)).astype(np.float32)
        kb, vb, qb = (f32_to_bits(x) for x in (k, v, q))
        tk = lambda b: torch.from_numpy(b.view(np.int16).copy()).view(torch.bfloat16)  # noqa: E731
        got = torch_attention.attention(tk(qb), tk(kb), tk(vb), T)
        got = bits_to_f32(got.view(torch.int16).numpy().view(np.uint16)).astype(np.float64)
        want = bits_to_f32(oatt.attention(qb, kb, vb, T)).astype(np.float64)
        tol = oatt.tolerance(qb, kb, vb, T, want)
        assert (np.abs(got - want) <= tol).all(), (B, T, Hq, Hkv)
