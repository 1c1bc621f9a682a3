"""The C-ABI library loads and exports every function include/exactkv_b200.h
declares; host-only entry points (split planner, error strings) behave. No GPU."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "exactkv_b200.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(exk_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = header_functions()
    for n in ("exk_attn_split_compressed", "exk_attn_split_bf16", "exk_attn_merge", "exk_encode_pages",
              "exk_decode_to_bf16", "exk_plan_splits"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from exactkv_b200 import _lib
    so = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in header_functions() if not hasattr(so, n)]
    assert not missing, missing
    # and the Python binding knows a signature for each of them
    assert sorted(header_functions()) == _lib.declared_symbols()


def test_library_is_built_for_sm100a():
    from exactkv_b200 import _lib
    # the build recipe compiles sm_100a only; the flag is part of the recipe
    from exactkv_b200 import build
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.NVCC_FLAGS)
    assert os.path.getsize(_lib.LIB_PATH) > 100_000


def test_error_strings():
    from exactkv_b200._lib import lib
    assert lib.exk_error_string(0) == b"ok"
    assert b"aligned" in lib.exk_error_string(-2)
    assert b"16 query heads" in lib.exk_error_string(-5)
    assert b"raw pool" in lib.exk_status_string(3)


def _plan(B, Hkv, T, ctas):
    from exactkv_b200._lib import lib
    ns, sl = ctypes.c_int32(), ctypes.c_int32()
    rc = lib.exk_plan_splits(B, Hkv, T, ctas, ctypes.byref(ns), ctypes.byref(sl))
    assert rc == 0
    return ns.value, sl.value


@pytest.mark.parametrize("B,Hkv,T", [(32, 8, 4096), (8, 8, 8192), (1, 4, 32768), (1, 8, 131072), (2, 2, 1000),
                                     (2, 2, 777), (1, 4, 4096), (3, 8, 1000), (2, 32, 333), (4, 2, 17), (1, 1, 1)])
def test_plan_covers_tokens_in_pages(B, Hkv, T):
    ns, sl = _plan(B, Hkv, T, 148)
    assert sl % 16 == 0 and sl > 0
    assert (ns - 1) * sl < T <= ns * sl          # every split holds at least one token
    assert ns <= 4096


def test_plan_balances_llama_shape():
    # 32 x 4096, 8 KV heads (one head group) over 148 SMs: 9 splits of 29 pages -> 288 items, 2 waves
    assert _plan(32, 8, 4096, 148) == (9, 464)


def test_plan_rejects_bad_arguments():
    from exactkv_b200._lib import lib
    ns, sl = ctypes.c_int32(), ctypes.c_int32()
    assert lib.exk_plan_splits(0, 8, 4096, 148, ctypes.byref(ns), ctypes.byref(sl)) == -1
    assert lib.exk_plan_splits(1, 8, 0, 148, ctypes.byref(ns), ctypes.byref(sl)) == -1


def test_entry_points_reject_bad_arguments_before_any_launch():
    """Argument errors come back as negative codes from the host-side checks that
    run before any CUDA call (fake, never dereferenced device addresses)."""
    from exactkv_b200._lib import lib, CView, Partials
    EARG, EALIGN, EHEADS = -1, -2, -5
    dev_addr = 1 << 40                     # 16-byte aligned, never touched
    ws = Partials(dev_addr, dev_addr + (1 << 20), dev_addr + (2 << 20), 4, 64, 0)
    cv = CView(dev_addr, dev_addr, dev_addr, dev_addr, dev_addr, dev_addr, 1024)
    st = ctypes.c_void_p(0)

    def split(q=dev_addr, k=cv, B=1, TS=256, Hkv=8, Hq=32, T=200, s0=0, s1=4, w=ws, nwc=8):
        return lib.exk_attn_split_compressed(q, ctypes.byref(k) if k is not None else None,
                                             ctypes.byref(cv), B, TS, Hkv, Hq, T, s0, s1,
                                             ctypes.byref(w) if w is not None else None, nwc, 0.1, st, 0, None)

    assert split(k=None) == EARG                       # null cache view
    assert split(w=None) == EARG                       # no workspace
    assert split(Hkv=1, Hq=32) == EHEADS               # 32 query heads per KV head
    assert split(Hq=30) == EARG                        # Hq not a multiple of Hkv
    assert split(nwc=6) == EARG                        # 4, 8 consumer warps only
    assert split(T=300) == EARG                        # T past the capacity TS
    assert split(s0=3, s1=3) == EARG                   # empty split range
    assert split(q=dev_addr + 8) == EALIGN             # q not 16-byte aligned
    short = Partials(dev_addr, dev_addr, dev_addr, 2, 64, 0)
    assert split(w=short, s1=2) == EARG                # the plan does not cover T
    bad_heads = Partials(dev_addr, dev_addr, dev_addr, 4, 64, 3)
    assert split(w=bad_heads) == EARG                  # heads per item must be 1, 2, 4 or 8
    counts = (ctypes.c_int32 * 2)(1, 1)
    flags = (ctypes.c_void_p * 2)(dev_addr, dev_addr)
    assert lib.exk_attn_merge_peers(flags, 2, 2, counts, 1, 32, dev_addr, flags, 1, dev_addr, None, 0, None) == EARG
    assert lib.exk_attn_merge_partial(ctypes.byref(ws), 32, 3, 3, dev_addr, dev_addr, dev_addr, 0, None) == EARG
    assert lib.exk_attn_merge_partial(ctypes.byref(ws), 32, 0, 5, dev_addr, dev_addr, dev_addr, 0, None) == EARG
    assert lib.exk_copy_from_host(dev_addr, dev_addr, 0, 0, None) == EARG           # nothing to copy
    assert lib.exk_copy_from_host(None, dev_addr, 64, 0, None) == EARG
    assert lib.exk_copy_from_host(dev_addr, dev_addr + 8, 64, 0, None) == EALIGN    # source not 16-byte aligned
    assert lib.exk_copy_from_host(dev_addr, dev_addr, 24, 0, None) == EALIGN        # not whole 16-byte words
    for code in (EARG, EALIGN, -3, -4, EHEADS, -6):
        assert lib.exk_error_string(code).startswith(b"exactkv_b200:")
    assert b"peer" in lib.exk_status_string(6)


def test_every_status_code_has_a_description():
    """Each EXK_S_* code the header defines has its own text (the host reads the
    device status word and raises with it)."""
    import re
    from exactkv_b200._lib import lib
    codes = {int(v) for v in re.findall(r"#define EXK_S_\w+\s+(\d+)", open(HEADER).read())}
    assert codes == set(range(len(codes)))
    texts = [lib.exk_status_string(c) for c in sorted(codes)]
    assert len(set(texts)) == len(texts) and all(t != b"unknown device status" for t in texts)
    assert lib.exk_status_string(max(codes) + 1) == b"unknown device status"


def test_noalloc_rejects_bad_arguments_before_any_launch():
    """The allocation-free entry point runs the shape and output checks of the
    allocating ones first: an over-wide GQA ratio is EXK_EHEADS (not the scratch
    limit), a bad output is refused before the split kernel could be queued."""
    from exactkv_b200._lib import lib, CView
    EARG, EALIGN, EHEADS = -1, -2, -5
    dev_addr = 1 << 40
    cv = CView(dev_addr, dev_addr, dev_addr, dev_addr, dev_addr, dev_addr, 1024)

    def call(B=1, TS=256, Hkv=8, Hq=32, T=200, out=dev_addr, q=dev_addr):
        return lib.exk_attention_compressed_noalloc(q, ctypes.byref(cv), ctypes.byref(cv), B, TS, Hkv, Hq, T, 8,
                                                    0.1, out, None, 0, None)

    assert call(B=4096, Hkv=1, Hq=32, TS=4096, T=4096) == EHEADS   # would also overflow the scratch
    assert call(Hq=30) == EARG
    assert call(TS=250, T=200) == EARG
    assert call(T=300) == EARG
    assert call(out=0) == EARG
    assert call(out=dev_addr + 2) == EALIGN
    assert call(q=0) == EARG


def test_balanced_plan_host_side():
    """exk_plan_balanced: the balanced plan's split count where it beats equal
    splits (32 x 4096 on 148 CTAs), 0 where the uniform plan is as good, and
    argument errors. For a device-length call (any_length) the split count is
    the bound for every length: ceil(148 / 32 units) + 1."""
    from exactkv_b200._lib import lib
    ns = ctypes.c_int32()
    assert lib.exk_plan_balanced(32, 8, 4096, 148, 8, 0, ctypes.byref(ns)) == 0 and 2 <= ns.value <= 16
    assert lib.exk_plan_balanced(32, 8, 4096, 148, 8, 1, ctypes.byref(ns)) == 0 and ns.value == 6
    assert lib.exk_plan_balanced(40, 8, 1024, 148, 8, 1, ctypes.byref(ns)) == 0 and ns.value == 5
    assert lib.exk_plan_balanced(8, 8, 8192, 148, 8, 0, ctypes.byref(ns)) == 0 and ns.value == 0
    assert lib.exk_plan_balanced(1, 4, 32768, 148, 8, 0, ctypes.byref(ns)) == 0 and ns.value == 0
    assert lib.exk_plan_balanced(1, 4, 32768, 148, 8, 1, ctypes.byref(ns)) == 0 and ns.value == 0
    assert lib.exk_plan_balanced(0, 8, 4096, 148, 8, 0, ctypes.byref(ns)) == -1
    assert lib.exk_plan_balanced(32, 8, 4096, 148, 6, 0, ctypes.byref(ns)) == -1


def test_balanced_plan_quotients_are_exact_in_double():
    """The attention kernel computes the balanced plan's run bounds floor(c W / G)
    and owners ceil((x + 1) G / W) - 1 with IEEE double division (W < 2^31
    stages, G <= 1024 CTAs): they equal the integer formulas, also next to the
    limits."""
    import numpy as np
    rng = np.random.default_rng(5)
    Ws = np.concatenate([rng.integers(1, 2 ** 31, 4000), [2 ** 31 - 1, 2 ** 31 - 2, 1, 2, 147, 148, 149]])
    for W in Ws.tolist():
        for G in (148, 1024, 1023, 7):
            cs = np.unique(np.concatenate([rng.integers(0, G + 1, 16), [0, 1, G - 1, G]]))
            for c in cs.tolist():
                assert int(c * W / G) == (c * W) // G
            xs = np.unique(np.concatenate([rng.integers(0, W, 16), [0, W - 1]]))
            for x in xs.tolist():
                import math
                assert math.ceil((x + 1) * G / W) - 1 == ((x + 1) * G + W - 1) // W - 1
