"""Generates tests/golden/*.npz from the REFERENCE implementation (run in a
container that has the reference checkout; the fixtures are committed so the
tests never need it).

    python tests/golden/make_golden.py --reference /path/to/exactkv

What it records:
  codec_cases.npz   full input bit patterns and the reference encode_reference
                    outputs (exactkv/codec.py:31-55) for: all 65,536 bf16
                    patterns, Gaussian data with an outlier channel and
                    +-0 / 1e-30 / inf / NaN, a constant page, all zeros.
                    Each case is also run through the reference's Triton page
                    encoder (exactkv/kernels.py:233-268) under TRITON_INTERPRET=1
                    and must write the same bytes; decode_reference must
                    round-trip it.
  config1.npz       for config 1 (batch 2, T = 1000 and 777, 8 q / 2 kv heads,
                    RoPE theta 1e6, 0.04% zeros, 0.3% forced raw rows): SHA-256
                    of the seeded inputs and of every encode_reference output
                    over the full pages, rowmask/rowoff in full, and the float64
                    attention of the reference's test (tests/test_exactkv.py:75-77).
"""
import argparse
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")  # before triton is imported

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))
sys.path.insert(0, HERE)
from synth_np import CONFIG1, config1_inputs, digest  # noqa: E402
from oracle.bf16 import bits_to_f32, f32_to_bits  # noqa: E402

FIELDS = ("sm", "code", "base", "rowmask", "rowoff", "raw")


def codec_inputs():
    rng = np.random.default_rng(0)
    yield "patterns", rng.permutation(65536).astype(np.uint16).reshape(4, 128, 1, 128)
    scale = np.exp(rng.standard_normal((4, 128))).astype(np.float32)
    scale[0, 5] = 300.0
    x = rng.standard_normal((2, 64, 4, 128)).astype(np.float32) * scale
    x[0, 7, 1, 3] = 0.0
    x[1, 9, 2, 5] = -0.0
    x[1, 40, 2, :] = 1e-30
    x[0, 50, 3, 64] = np.inf
    x[1, 60, 0, 1] = np.nan
    yield "specials", f32_to_bits(x)
    yield "constant", f32_to_bits(np.full((1, 64, 2, 128), 1.5, np.float32))
    yield "zeros", np.zeros((1, 64, 2, 128), np.uint16)


def ref_encode(codec, bits):
    x = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
    c = codec.encode_reference(x)
    out = {k: (c[k].view(torch.int16).numpy().view(np.uint16) if k == "raw" else c[k].numpy()) for k in FIELDS}
    back = codec.decode_reference(c).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(back, bits), "reference decode_reference did not round-trip"
    return out


def interp_encode(exactkv, bits):
    """The reference's Triton encoder, interpreted on the CPU, into fresh buffers."""
    B, T, H, D = bits.shape
    x = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
    c = exactkv.CompressedKV(B, T, H, D, device="cpu", reserve=1.0)
    st = (x.stride(0), 16 * x.stride(1), x.stride(1), x.stride(2))
    exactkv.kernels.encode_pages(x, st, c._buf(), 0, 0, B, T // 16)
    n = int(c.cnt.item())
    return {"sm": c.sm.numpy(), "code": c.code.numpy(), "base": c.base.numpy(), "rowmask": c.rowmask.numpy(),
            "rowoff": c.rowoff.numpy(), "raw": c.raw[:n].view(torch.int16).numpy().view(np.uint16)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the exactkv checkout")
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    import exactkv  # noqa: E402
    from exactkv import codec  # noqa: E402

    store = {}
    for name, bits in codec_inputs():
        ref = ref_encode(codec, bits)
        itp = interp_encode(exactkv, bits)
        for k in FIELDS:
            assert np.array_equal(ref[k], itp[k]), f"{name}: reference Triton encoder differs on {k}"
        store[f"{name}/input"] = bits
        for k in FIELDS:
            store[f"{name}/{k}"] = ref[k]
        print(f"{name}: {bits.shape}, raw rows {ref['raw'].shape[0]}; Triton encoder (interpreted) identical")
    np.savez_compressed(os.path.join(HERE, "codec_cases.npz"), **store)

    cfg = {}
    for case in CONFIG1:
        q, k, v = config1_inputs(case)
        T = case["T"]
        Tf = T // 16 * 16
        cfg[f"{case['name']}/digest_q"] = np.array(digest(q))
        for tag, x in (("k", k), ("v", v)):
            cfg[f"{case['name']}/digest_{tag}"] = np.array(digest(x))
            ref = ref_encode(codec, np.ascontiguousarray(x[:, :Tf]))
            itp = interp_encode(exactkv, np.ascontiguousarray(x[:, :Tf]))
            for f in FIELDS:
                assert np.array_equal(ref[f], itp[f]), f"{case['name']} {tag}: Triton encoder differs on {f}"
                cfg[f"{case['name']}/{tag}/digest_{f}"] = np.array(digest(ref[f]))
            cfg[f"{case['name']}/{tag}/rowmask"] = ref["rowmask"]
            cfg[f"{case['name']}/{tag}/rowoff"] = ref["rowoff"]
            cfg[f"{case['name']}/{tag}/raw_rows"] = np.array(ref["raw"].shape[0])
            print(f"{case['name']} {tag}: full pages {Tf // 16}, raw rows {ref['raw'].shape[0]}")
        # float64 attention as in the reference test (tests/test_exactkv.py:75-77)
        G = case["Hq"] // case["Hkv"]
        qd = torch.from_numpy(bits_to_f32(q)).double()
        kd = torch.from_numpy(bits_to_f32(k[:, :T])).double().repeat_interleave(G, 2)
        vd = torch.from_numpy(bits_to_f32(v[:, :T])).double().repeat_interleave(G, 2)
        o64 = torch.einsum("bht,bthd->bhd",
                           (torch.einsum("bhd,bthd->bht", qd, kd) / 128 ** 0.5).softmax(-1), vd)
        cfg[f"{case['name']}/attn_f64"] = o64.numpy()
    np.savez_compressed(os.path.join(HERE, "config1.npz"), **cfg)
    print("wrote", os.path.join(HERE, "codec_cases.npz"), os.path.join(HERE, "config1.npz"))


if __name__ == "__main__":
    main()
