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
