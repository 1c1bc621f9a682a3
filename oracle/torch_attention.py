"""PyTorch (CPU) restatement of the reference's split-K decode attention, for
bench.py's CPU baseline only (test/benchmark infrastructure, never the product).

The reference has no CPU attention: its attention is the Triton pair
_split_c_kernel/_split_ref_kernel + _reduce_kernel. This module states the same
algorithm in torch so that the reference's own PyTorch codec (decode_reference,
run unmodified) can be timed end to end on the host cores beside it:
  * choose_split (exactkv/kernels.py:273-277): at most 512 programs, split
    length a multiple of BLOCK_N = 64;
  * per split, the block loop of the split kernel (exactkv/kernels.py:142-165)
    with the online-softmax block _attn_block (exactkv/kernels.py:46-59):
    base-2 scores with qk_scale = D^-0.5 log2(e) (exactkv/kernels.py:316),
    running max, P rounded to bf16 before the PV product, fp32 accumulation;
  * the split merge _reduce_kernel (exactkv/kernels.py:33-43).
Vectorised over sequences, KV heads and splits; the loop runs over the blocks
of a split. float32 throughout (torch's matmul order, not the kernel's).
"""
import math

import torch

LOG2E = 1.4426950408889634


def choose_split(B, Hkv, T, block_n=64, target=512):
    ns = max(1, min(-(-T // block_n), target // max(1, B * Hkv)))
    split_len = -(-(-(-T // ns)) // block_n) * block_n
    return -(-T // split_len), split_len


def attention(q, k, v, T, block_n=64):
    """q [B, Hq, D] bf16, k, v [B, >=T, Hkv, D] bf16 (CPU). Returns bf16 [B, Hq, D]."""
    B, Hq, D = q.shape
    Hkv = k.shape[2]
    G = Hq // Hkv
    ns, sl = choose_split(B, Hkv, T, block_n)
    pad = ns * sl
    kf = torch.zeros(B, pad, Hkv, D, dtype=torch.float32)
    vf = torch.zeros(B, pad, Hkv, D, dtype=torch.float32)
    kf[:, :T] = k[:, :T].float()
    vf[:, :T] = v[:, :T].float()
    # [B, Hkv, ns, split_len, D]
    kf = kf.view(B, ns, sl, Hkv, D).permute(0, 3, 1, 2, 4)
    vf = vf.view(B, ns, sl, Hkv, D).permute(0, 3, 1, 2, 4)
    qg = q.float().view(B, Hkv, 1, G, D)
    valid = (torch.arange(pad) < T).view(ns, sl)
    scale = D ** -0.5 * LOG2E
    m = torch.full((B, Hkv, ns, G), -math.inf)
    l = torch.zeros(B, Hkv, ns, G)
    acc = torch.zeros(B, Hkv, ns, G, D)
    for n0 in range(0, sl, block_n):
        kb = kf[:, :, :, n0:n0 + block_n]                            # [B, Hkv, ns, n, D]
        vb = vf[:, :, :, n0:n0 + block_n]
        s = torch.matmul(qg, kb.transpose(-1, -2)) * scale             # [B, Hkv, ns, G, n]
        s = s.masked_fill(~valid[:, n0:n0 + block_n].view(1, 1, ns, 1, -1), -math.inf)
        m_new = torch.maximum(m, s.amax(-1))
        alpha = torch.exp2(m - m_new)
        p = torch.exp2(s - m_new[..., None])
        p = torch.nan_to_num(p, nan=0.0)                               # blocks past T in a split
        alpha = torch.nan_to_num(alpha, nan=1.0)
        l = l * alpha + p.sum(-1)
        acc = acc * alpha[..., None] + torch.matmul(p.to(torch.bfloat16).float(), vb)
        m = m_new
    M = m.amax(2, keepdim=True)
    w = torch.exp2(m - M)
    w = torch.nan_to_num(w, nan=0.0)
    out = (acc * w[..., None]).sum(2) / (l * w).sum(2)[..., None]   # [B, Hkv, G, D]
    return out.reshape(B, Hq, D).to(torch.bfloat16)
