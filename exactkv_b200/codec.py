"""The storage format's whole-tensor functions (reference: exactkv/codec.py),
computed on the GPU by the sm_100a page encoder and decoder.

encode_reference(x) returns the same dict as the reference's CPU function —
raw rows in (sequence, page, head) order, so every field matches it byte for
byte — and decode_reference(c) inverts it. Inputs must be CUDA tensors: there
is no CPU path in this package.

Format, per 16-token page x KV head x channel (D = 128):
  sm      uint8 [B, T, H, D]      sign and mantissa, unchanged
  code    uint8 [B, T, H, D/2]    4-bit exponent offsets; byte j holds channels j and j + D/2
  base    uint8 [B, T/16, H, D]   < 128: exponent = base + code;  >= 128: a group with
                                  zeros: code 0 means exponent 0, else base - 128 + code
  rowmask int32 [B, T/16, H]      bit p set: token p of the page is stored raw
  rowoff  int32 [B, T/16, H]      index of the page's first raw row in `raw`
  raw     bf16  [N_raw, D]        rows holding a value more than 2^15 below its group's max
"""
import torch

from . import kernels
from .kernels import P


def encode_reference(x):
    """x: [B, T, H, D] bf16 CUDA tensor, T a multiple of 16. Returns a dict of tensors
    (raw rows in page order), as the reference's encode_reference."""
    B, T, H, D = x.shape
    if T % P or x.dtype != torch.bfloat16 or D != kernels.D:
        raise ValueError("x must be bf16 [B, T, H, 128] with T a multiple of 16")
    x = x.contiguous()
    dev = x.device
    NP = T // P
    u8, i32 = dict(dtype=torch.uint8, device=dev), dict(dtype=torch.int32, device=dev)
    buf = dict(sm=torch.empty(B, T, H, D, **u8), code=torch.empty(B, T, H, D // 2, **u8),
               base=torch.empty(B, NP, H, D, **u8), rowmask=torch.empty(B, NP, H, **i32),
               rowoff=torch.empty(B, NP, H, **i32), raw=torch.empty(B * T * H, D, dtype=torch.bfloat16, device=dev),
               cnt=torch.zeros(1, **i32), cap=B * T * H, TS=T, H=H, D=D)
    kernels.encode_pages(x, (x.stride(0), P * x.stride(1), x.stride(1), x.stride(2)), buf, 0, 0, B, NP)
    n = int(buf["cnt"].item())
    return dict(shape=(B, T, H, D), sm=buf["sm"], code=buf["code"], base=buf["base"], rowmask=buf["rowmask"],
                rowoff=buf["rowoff"], raw=buf["raw"][:n].clone())


def decode_reference(c):
    """Inverse of encode_reference."""
    return kernels.decode_to_bf16(c, c["shape"][1])


def bits_per_value(c):
    n = c["sm"].numel()
    return sum(c[k].numel() * c[k].element_size() for k in ("sm", "code", "base", "rowmask", "rowoff", "raw")) * 8 / n
