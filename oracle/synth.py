"""Seeded numpy generator of the synthetic KV distribution (test infrastructure only).

x = 2^c[h, ch] * N(0, 1) with c ~ U{-4..3} per (KV head, channel), rounded
to bf16; keys are RoPE-rotated first (rotate-half pairing j <-> j + 64, the
same pairing as the format's code nibbles). Keys get `zero_frac` exact zeros;
a `raw_frac` share of rows has one channel scaled by 2^-20, which forces those
rows into the raw pool. The golden fixtures store a SHA-256 of each generated
input, so a changed generator is caught rather than silently accepted.
"""
import hashlib

import numpy as np

from .bf16 import bits_to_f32, f32_to_bits


def rope_np(x, theta):
    """Rotate [B, T, H, D] float32 by position t along axis 1 (rotate_half convention)."""
    B, T, H, D = x.shape
    half = D // 2
    inv = (1.0 / (theta ** (np.arange(0, half, dtype=np.float64) * 2.0 / D))).astype(np.float32)
    ang = np.arange(T, dtype=np.float32)[:, None] * inv[None, :]
    cos = np.cos(ang).astype(np.float32)[None, :, None, :]
    sin = np.sin(ang).astype(np.float32)[None, :, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1).astype(np.float32)


def synth_kv(seed, B, T, H, D=128, theta=1e6, key=True, zero_frac=4e-4, raw_frac=3e-3):
    """bf16 bit patterns uint16 [B, T, H, D]."""
    rng = np.random.default_rng(seed)
    c = rng.integers(-4, 4, size=(H, D))
    x = rng.standard_normal((B, T, H, D), dtype=np.float32) * np.exp2(c).astype(np.float32)
    if key:
        x = rope_np(x, theta)
    bits = f32_to_bits(x)
    if key and zero_frac > 0:
        bits[rng.random((B, T, H, D)) < zero_frac] = 0
    if raw_frac > 0:
        rows = rng.random((B, T, H)) < raw_frac
        ch = rng.integers(0, D, size=(B, T, H))
        b_i, t_i, h_i = np.nonzero(rows)
        c_i = ch[rows]
        vals = bits_to_f32(bits[b_i, t_i, h_i, c_i]) * np.float32(2.0 ** -20)
        bits[b_i, t_i, h_i, c_i] = f32_to_bits(vals)
    return bits


def synth_q(seed, B, Hq, D=128):
    rng = np.random.default_rng(seed)
    return f32_to_bits(rng.standard_normal((B, Hq, D), dtype=np.float32))


def digest(a):
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.tobytes()).hexdigest()
