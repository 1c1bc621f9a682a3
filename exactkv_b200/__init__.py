"""exactkv_b200: a B200-native (sm_100a) implementation of exactkv's hot path —
split-K decode attention that reads the lossless exponent-coded bf16 KV cache,
and the page encoder that writes it — behind the reference's Python API.

Same public names as the reference package (exactkv/__init__.py:3-12).
"""
from .cache import CompressedKV, BF16KV, check_overflow
from .attention import decode_attention
from .codec import encode_reference, decode_reference, bits_per_value
from .kernels import attention_compressed, attention_reference, decode_to_bf16, encode_pages
from . import kernels

__version__ = "0.1.0"
__all__ = ["CompressedKV", "BF16KV", "check_overflow", "decode_attention", "Engine",
           "encode_reference", "decode_reference", "bits_per_value",
           "attention_compressed", "attention_reference", "decode_to_bf16", "encode_pages", "kernels"]


def __getattr__(name):
    # the engine pulls in transformers; load it on first use
    if name == "Engine":
        from .engine import Engine
        return Engine
    raise AttributeError(name)
