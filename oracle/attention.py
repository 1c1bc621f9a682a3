"""Numpy restatement of the reference's split-K decode attention (test infrastructure only).

Follows exactkv/kernels.py: choose_split (lines 273-277), the split kernel's
loop over BLOCK_N-token blocks (lines 142-165) with the online-softmax block
_attn_block (lines 46-59) — scores in base 2 with qk_scale = D^-0.5 log2(e)
(line 316), P rounded to bf16 before the PV product, fp32 accumulation — and
the split merge _reduce_kernel (lines 33-43). Also the float64 einsum the
reference's test uses as its truth bound (tests/test_exactkv.py:75-77).

All arithmetic is float32 numpy; matrix products sum in numpy's order, so the
result agrees with the GPU kernels to fp32 rounding, not bit for bit.
"""
import numpy as np

from .bf16 import bits_to_f32, f32_to_bits, round_f32

LOG2E = 1.4426950408889634


def choose_split(B, Hkv, T, block_n=64, target=512):
    """(number of splits, split length): at most `target` programs in total, the
    split length rounded up to a multiple of block_n (exactkv/kernels.py:273-277)."""
    blocks = -(-T // block_n)
    ns = max(1, min(blocks, target // max(1, B * Hkv)))
    per_split = -(-T // ns)
    split_len = -(-per_split // block_n) * block_n
    return -(-T // split_len), split_len


def split_partials(q_bits, k_bits, v_bits, T, block_n=64, splits=None):
    """Partials (o, m, l) of every split: o [B, Hq, ns, D], m, l [B, Hq, ns]."""
    q = bits_to_f32(q_bits)
    B, Hq, D = q.shape
    Hkv = k_bits.shape[2]
    G = Hq // Hkv
    ns, sl = splits if splits is not None else choose_split(B, Hkv, T, block_n)
    k = bits_to_f32(k_bits[:, :T]).reshape(B, T, Hkv, D)
    v = bits_to_f32(v_bits[:, :T]).reshape(B, T, Hkv, D)
    qg = q.reshape(B, Hkv, G, D)
    scale = np.float32(D ** -0.5 * LOG2E)
    h = D // 2
    o = np.zeros((B, Hkv, G, ns, D), np.float32)
    m_out = np.full((B, Hkv, G, ns), -np.inf, np.float32)
    l_out = np.zeros((B, Hkv, G, ns), np.float32)
    for s in range(ns):
        lo_t, hi_t = s * sl, min(s * sl + sl, T)
        m = np.full((B, Hkv, G), -np.inf, np.float32)
        l = np.zeros((B, Hkv, G), np.float32)
        acc = np.zeros((B, Hkv, G, D), np.float32)
        for n0 in range(lo_t, hi_t, block_n):
            n1 = min(n0 + block_n, hi_t)
            kb = k[:, n0:n1].transpose(0, 2, 3, 1)                 # [B, Hkv, D, n]
            vb = v[:, n0:n1].transpose(0, 2, 1, 3)                 # [B, Hkv, n, D]
            s_lo = np.matmul(qg[..., :h], kb[:, :, :h])            # two halves, as the kernel
            sc = (s_lo + np.matmul(qg[..., h:], kb[:, :, h:])) * scale
            m_new = np.maximum(m, sc.max(-1))
            alpha = np.exp2(m - m_new)
            p = np.exp2(sc - m_new[..., None])
            l = l * alpha + p.sum(-1)
            acc = acc * alpha[..., None] + np.matmul(round_f32(p), vb)
            m = m_new
        o[:, :, :, s] = acc
        m_out[:, :, :, s] = m
        l_out[:, :, :, s] = l
    return o.reshape(B, Hq, ns, D), m_out.reshape(B, Hq, ns), l_out.reshape(B, Hq, ns)


def merge(o, m, l):
    """out = sum_s o_s 2^(m_s - M) / sum_s l_s 2^(m_s - M) as float32."""
    M = m.max(-1, keepdims=True)
    w = np.exp2(m - M)
    return (o * w[..., None]).sum(-2) / (l * w).sum(-1)[..., None]


def merge_group(o, m, l):
    """The partial of a run of splits (the last axis of m, l; o [..., n, D]):
    M = max_s m_s, o_g = sum_s o_s 2^(m_s - M), l_g = sum_s l_s 2^(m_s - M), in
    the layout of one split's partial, so merge() combines groups like splits
    (the two-level merge of a KV-sequence split; no counterpart in the
    reference, whose merge is _reduce_kernel, exactkv/kernels.py:33-43)."""
    M = m.max(-1)
    w = np.where(np.isneginf(m), np.float32(0), np.exp2(m - M[..., None]))
    return (o * w[..., None]).sum(-2).astype(np.float32), M.astype(np.float32), (l * w).sum(-1).astype(np.float32)


def attention(q_bits, k_bits, v_bits, T, block_n=64):
    """Reference split-K decode attention; returns bf16 bit patterns [B, Hq, D]."""
    o, m, l = split_partials(q_bits, k_bits, v_bits, T, block_n)
    return f32_to_bits(merge(o, m, l))


def _softmax_f64(q_bits, k_bits, T):
    q = bits_to_f32(q_bits).astype(np.float64)
    B, Hq, D = q.shape
    G = Hq // k_bits.shape[2]
    k = np.repeat(bits_to_f32(k_bits[:, :T]).astype(np.float64), G, axis=2)
    s = np.einsum("bhd,bthd->bht", q, k) / np.sqrt(D)
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    return p / p.sum(-1, keepdims=True), G


def attention_f64(q_bits, k_bits, v_bits, T):
    """softmax(q k^T / sqrt(D)) v in float64 with GQA head sharing."""
    p, G = _softmax_f64(q_bits, k_bits, T)
    v = np.repeat(bits_to_f32(v_bits[:, :T]).astype(np.float64), G, axis=2)
    return np.einsum("bht,bthd->bhd", p, v)


def tolerance(q_bits, k_bits, v_bits, T, ref):
    """Per-output bound used by every attention comparison:
        |a - b| <= 2^-8 * sum_t p_t |v_t| + 2^-8 * |ref| + 1e-6
    i.e. one bf16 rounding step of each P.V product (P is rounded to bf16 before
    the product, and two kernels that block the softmax differently round P
    against different running maxima) plus one rounding step of the bf16 output.
    For V ~ N(0, 1) the first term is about 3e-3, the 2e-3 scale the reference
    test uses; it grows with |V| because the rounding error does."""
    p, G = _softmax_f64(q_bits, k_bits, T)
    vabs = np.repeat(np.abs(bits_to_f32(v_bits[:, :T]).astype(np.float64)), G, axis=2)
    return 2.0 ** -8 * np.einsum("bht,bthd->bhd", p, vabs) + 2.0 ** -8 * np.abs(ref) + 1e-6
