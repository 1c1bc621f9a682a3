"""Numpy restatement of the exactkv storage format (test infrastructure only).

Follows exactkv/codec.py: encode_reference (lines 31-55), decode_reference
(lines 58-73) and bits_per_value (lines 76-78). Inputs and outputs are numpy
arrays; bf16 values travel as uint16 bit patterns.

Per 16-token page x KV head x channel, with e = the 8-bit exponent of each
value and emax its maximum over the page:
  b      = max(emax - 15, 0)                       (the 16-step window's base)
  zgroup = some e == 0 and b > 0                   (zeros the window cannot hold)
  code   = 0 for a zero in a zero group, else e - b, clamped to 0..15
  escape = code below the group's floor (1 in a zero group, else 0) for a
           non-zero value, or b >= 128
  base   = min(b + 128 if zgroup else b, 255)
A (token, head) row with any escaping channel is stored raw.
"""
import numpy as np

PAGE = 16


def encode(bits):
    """bits: uint16 [B, T, H, D], T a multiple of 16. Returns the six format arrays
    (sm, code, base, rowmask, rowoff, raw) with raw rows in (b, page, head, token) order."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    B, T, H, D = bits.shape
    if T % PAGE:
        raise ValueError("T must be a multiple of 16")
    NP = T // PAGE
    u = bits.astype(np.int32)
    exp = (u >> 7) & 0xFF
    sm = (((u >> 8) & 0x80) | (u & 0x7F)).astype(np.uint8)

    ep = exp.reshape(B, NP, PAGE, H, D)
    base_exp = np.maximum(ep.max(axis=2) - 15, 0)                  # [B, NP, H, D]
    zgroup = (ep == 0).any(axis=2) & (base_exp > 0)
    b_b = base_exp[:, :, None]
    z_b = zgroup[:, :, None]
    zero_here = z_b & (ep == 0)
    code = np.where(zero_here, 0, ep - b_b)
    floor = z_b.astype(np.int32)
    escapes = ((code < floor) & ~zero_here) | (b_b >= 128)
    code = np.clip(code, 0, 15).reshape(B, T, H, D)
    half = D // 2
    packed = (code[..., :half] | (code[..., half:] << 4)).astype(np.uint8)
    base = np.minimum(np.where(zgroup, base_exp + 128, base_exp), 255).astype(np.uint8)

    raw_row = escapes.any(axis=-1).transpose(0, 1, 3, 2)          # [B, NP, H, PAGE]
    weights = (np.int64(1) << np.arange(PAGE, dtype=np.int64))
    rowmask = (raw_row.astype(np.int64) * weights).sum(-1).astype(np.int32)
    counts = raw_row.sum(-1).reshape(-1).astype(np.int64)
    rowoff = (np.cumsum(counts) - counts).astype(np.int32).reshape(B, NP, H)
    raw = bits.reshape(B, NP, PAGE, H, D).transpose(0, 1, 3, 2, 4)[raw_row]
    return dict(shape=(B, T, H, D), sm=sm, code=packed, base=base, rowmask=rowmask, rowoff=rowoff,
                raw=np.ascontiguousarray(raw))


def decode(c, T=None):
    """Inverse of encode (raw rows in page order); returns uint16 [B, T, H, D].
    With T < the stored length, only the first T tokens are rebuilt."""
    B, TS, H, D = c["shape"]
    NP = TS // PAGE
    code = c["code"].astype(np.int32)
    codes = np.concatenate([code & 15, code >> 4], axis=-1)
    bb = np.repeat(c["base"].astype(np.int32), PAGE, axis=1)
    exp = (bb & 127) + codes
    exp = np.where((bb >= 128) & (codes == 0), 0, exp)
    s = c["sm"].astype(np.int32)
    bits = (((s & 0x80) << 8) | ((exp & 0xFF) << 7) | (s & 0x7F)).astype(np.uint16)
    paged = bits.reshape(B, NP, PAGE, H, D).transpose(0, 1, 3, 2, 4)
    raw_row = ((c["rowmask"][..., None] >> np.arange(PAGE)) & 1).astype(bool)
    # rows are taken from `raw` at rowoff + rank within the page (what the kernels do)
    rank = np.cumsum(raw_row, axis=-1) - raw_row
    idx = (c["rowoff"][..., None] + rank)[raw_row]
    paged[raw_row] = c["raw"][idx]
    out = paged.transpose(0, 1, 3, 2, 4).reshape(B, TS, H, D)
    return out if T is None else out[:, :T]


def bits_per_value(c):
    n = c["sm"].size
    return sum(c[k].size * c[k].itemsize for k in ("sm", "code", "base", "rowmask", "rowoff", "raw")) * 8 / n
