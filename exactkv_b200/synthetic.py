"""Seeded synthetic KV and query tensors with the benchmark distribution, built
with torch on any device (the GPU for the full-size benchmark shapes).

x = 2^c[h, ch] * N(0, 1), c ~ U{-4..3} per (KV head, channel), rounded to
bf16. Keys are RoPE-rotated with the given theta (rotate-half pairing j <-> j+64)
and get `zero_frac` exact zeros (after RoPE about 0.04% of real keys are 0).
A `raw_frac` share of (token, head) rows has one channel scaled by 2^-20,
which forces those rows into the raw pool. Queries are N(0, 1).
There are no model checkpoints or datasets in this environment; these tensors
stand in for the real-model KV the reference benchmarks on.
"""
import torch


def rope_(x, theta, pos0=0):
    """In-place RoPE over axis 1 (tokens) of [B, T, H, D] float32."""
    B, T, H, D = x.shape
    half = D // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64, device=x.device) * 2.0 / D))
    ang = torch.arange(pos0, pos0 + T, dtype=torch.float32, device=x.device)[:, None] * inv.float()[None, :]
    cos, sin = torch.cos(ang)[None, :, None, :], torch.sin(ang)[None, :, None, :]
    x1, x2 = x[..., :half].clone(), x[..., half:].clone()
    x[..., :half] = x1 * cos - x2 * sin
    x[..., half:] = x2 * cos + x1 * sin
    return x


def make_kv(B, T, H, *, seed, theta=5e5, key=True, zero_frac=4e-4, raw_frac=3e-3, device="cuda", D=128):
    """bf16 [B, T, H, D]."""
    g = torch.Generator(device=device).manual_seed(seed)
    c = torch.randint(-4, 4, (H, D), generator=g, device=device)
    x = torch.randn(B, T, H, D, generator=g, device=device)
    x.mul_(torch.exp2(c.float()))
    if key:
        rope_(x, theta)
    x = x.to(torch.bfloat16)
    if key and zero_frac > 0:
        x.masked_fill_(torch.rand(B, T, H, D, generator=g, device=device) < zero_frac, 0.0)
    if raw_frac > 0:
        rows = torch.rand(B, T, H, generator=g, device=device) < raw_frac
        ch = torch.randint(0, D, (B, T, H), generator=g, device=device)
        sel = torch.zeros(B, T, H, D, dtype=torch.bool, device=device)
        sel.scatter_(3, ch[..., None], rows[..., None])
        x = torch.where(sel, (x.float() * 2.0 ** -20).to(torch.bfloat16), x)
    return x


def make_q(B, Hq, *, seed, device="cuda", D=128):
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(B, Hq, D, generator=g, device=device).to(torch.bfloat16)
