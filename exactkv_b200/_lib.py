"""ctypes binding of libexactkv_b200.so (the C ABI declared in include/exactkv_b200.h).

The library is the product: there is no CPU or Triton fallback. Importing this
module without the built library raises ImportError; every entry point turns a
nonzero return code into RuntimeError.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libexactkv_b200.so")

c_void_p, c_int, c_int32, c_int64, c_float = ctypes.c_void_p, ctypes.c_int, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
c_uint32 = ctypes.c_uint32

# Every symbol the header declares, with its ctypes signature (restype, argtypes).
_SIGNATURES = {}


class CView(ctypes.Structure):
    """exk_cview: one compressed cache (the six buffers of the format)."""
    _fields_ = [("sm", c_void_p), ("code", c_void_p), ("base", c_void_p), ("rowmask", c_void_p),
                ("rowoff", c_void_p), ("raw", c_void_p), ("raw_rows", c_int64)]


class Partials(ctypes.Structure):
    """exk_partials: split-K workspace (o [rows, ns, 128], m, l [rows, ns]) and the split plan."""
    _fields_ = [("o", c_void_p), ("m", c_void_p), ("l", c_void_p), ("ns", c_int32), ("split_len", c_int32),
                ("heads", c_int32)]


_P = ctypes.POINTER
_SIGNATURES.update({
    "exk_plan_splits": (c_int, [c_int, c_int, c_int, c_int, _P(c_int32), _P(c_int32)]),
    "exk_plan_balanced": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, _P(c_int32)]),
    "exk_num_sms": (c_int, [c_int]),
    "exk_attn_split_compressed": (c_int, [c_void_p, _P(CView), _P(CView), c_int, c_int, c_int, c_int, c_int,
                                          c_int, c_int, _P(Partials), c_int, c_float, c_void_p, c_int, c_void_p]),
    "exk_attn_split_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                    _P(Partials), c_int, c_float, c_void_p, c_int, c_void_p]),
    "exk_attn_merge": (c_int, [_P(Partials), c_int, c_void_p, c_int, c_void_p]),
    "exk_attention_compressed_paged": (c_int, [c_void_p, _P(CView), _P(CView), c_int, c_int, c_int, c_int, c_void_p,
                                               c_int, c_void_p, _P(Partials), c_void_p, c_int, c_float, c_void_p,
                                               c_int, c_void_p]),
    "exk_attention_bf16_paged": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int,
                                         c_void_p, _P(Partials), c_void_p, c_int, c_float, c_void_p, c_int,
                                         c_void_p]),
    "exk_attn_merge_partial": (c_int, [_P(Partials), c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int,
                                       c_void_p]),
    "exk_attn_merge_gathered": (c_int, [c_void_p, c_int, _P(c_int32), c_int, c_int, c_void_p, c_int, c_void_p]),
    "exk_attn_merge_peers": (c_int, [_P(c_void_p), c_int, c_int, _P(c_int32), c_int, c_int, c_void_p, _P(c_void_p),
                                     c_uint32, c_void_p, c_void_p, c_int, c_void_p]),
    "exk_attention_compressed": (c_int, [c_void_p, _P(CView), _P(CView), c_int, c_int, c_int, c_int, c_int,
                                         _P(Partials), c_void_p, c_int, c_float, c_void_p, c_int, c_void_p]),
    "exk_attention_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, _P(Partials),
                                   c_void_p, c_int, c_float, c_void_p, c_int, c_void_p]),
    "exk_encode_pages": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int, c_int, c_int,
                                 c_int, c_int, c_int, c_void_p, c_int, c_void_p]),
    "exk_decode_to_bf16": (c_int, [_P(CView), c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p]),
    "exk_attention_compressed_devlen": (c_int, [c_void_p, _P(CView), _P(CView), c_int, c_int, c_int, c_int, c_int,
                                                c_void_p, c_int, c_int, c_int, _P(Partials), c_void_p, c_int, c_float,
                                                c_void_p, c_int, c_void_p]),
    "exk_attention_bf16_devlen": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                          c_void_p, c_int, c_int, c_int, _P(Partials), c_void_p, c_int, c_float,
                                          c_void_p, c_int, c_void_p]),
    "exk_append_token": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_int,
                                 c_void_p]),
    "exk_advance_length": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "exk_copy_from_host": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "exk_selftest_wait_timeout": (c_int, [c_void_p, ctypes.c_uint64, c_int, c_void_p]),
    "exk_attention_compressed_noalloc": (c_int, [c_void_p, _P(CView), _P(CView), c_int, c_int, c_int, c_int, c_int,
                                                 c_int, c_float, c_void_p, c_void_p, c_int, c_void_p]),
    "exk_error_string": (ctypes.c_char_p, [c_int]),
    "exk_status_string": (ctypes.c_char_p, [c_int]),
})


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"exactkv_b200: {LIB_PATH} is not built; run `python exactkv_b200/build.py` "
                          "(there is no CPU or Triton fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def declared_symbols():
    return sorted(_SIGNATURES)


def check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what}: {lib.exk_error_string(rc).decode()} (code {rc})")
