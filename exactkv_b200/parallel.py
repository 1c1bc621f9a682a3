"""Multi-GPU decode attention: batch sharding and the KV-sequence split.

Batch sharding needs no code here: sequences are independent, so every GPU
runs its own batch slice (one replica per GPU, no collective).

KV-sequence split (one long sequence over N GPUs). A global split plan
(ns splits of split_len tokens, chosen for N x SMs persistent CTAs) is cut
into N contiguous runs of whole splits; rank r keeps the pages of its run,
tokens [s0 * split_len, min(s1 * split_len, T)), in its own cache. Each rank
computes the (o, m, l) partials of its splits with the split kernel, one
all-gather (NCCL over NVLink) exchanges them, and every rank merges all ns
partials in global split order. Partials depend only on their split's tokens,
so the result is bit-identical to a single GPU running the same plan.

The reference has no multi-GPU path; the partials and the merge are those of
its split-K decode (exactkv/kernels.py:33-43, 142-165).
"""
import torch

from . import kernels
from .kernels import D, P

PACK = D + 2  # per (row, split): o[0:D], m, l


class KVSplitPlan:
    """Global split plan and each rank's run of splits.

    bounds[r] .. bounds[r+1] are rank r's splits; token range of rank r:
    [bounds[r] * split_len, min(bounds[r+1] * split_len, T))."""

    def __init__(self, B, Hkv, T, world, ns, split_len):
        if world < 1 or ns < 1 or split_len % P != 0 or ns * split_len < T:
            raise ValueError("invalid KV-split plan")
        self.B, self.Hkv, self.T, self.world = B, Hkv, T, world
        self.ns, self.split_len = ns, split_len
        self.bounds = [(r * ns) // world for r in range(world + 1)]

    @classmethod
    def make(cls, B, Hkv, T, world, device=None):
        """The split kernel's own planner, sized for world x (SMs of one GPU) CTAs."""
        ns, sl = kernels.plan_splits(B, Hkv, T, device, num_ctas=world * kernels.num_sms(device))
        return cls(B, Hkv, T, world, ns, sl)

    def splits(self, rank):
        return self.bounds[rank], self.bounds[rank + 1]

    def tokens(self, rank):
        s0, s1 = self.splits(rank)
        return min(s0 * self.split_len, self.T), min(s1 * self.split_len, self.T)

    @property
    def max_local(self):
        return max(self.bounds[r + 1] - self.bounds[r] for r in range(self.world))


def local_partials(q, kc, vc, plan, rank, num_warps=None):
    """Rank `rank`'s partials, packed [B*Hq, max_local, D+2] fp32 (columns past the
    rank's own splits are padding). kc, vc hold the rank's tokens from position 0."""
    B, Hq, _ = q.shape
    rows = B * Hq
    s0, s1 = plan.splits(rank)
    t0, t1 = plan.tokens(rank)
    packed = torch.zeros(rows, plan.max_local, PACK, dtype=torch.float32, device=q.device)
    nloc = s1 - s0
    if nloc > 0 and t1 > t0:
        nloc = -(-(t1 - t0) // plan.split_len)  # splits that hold tokens
        stream = torch.cuda.current_stream(q.device).cuda_stream
        ws = kernels._workspace(q.device, stream, rows, nloc, plan.split_len)
        kernels.attention_split(q, kc, vc, t1 - t0, ws, 0, nloc, num_warps=num_warps)
        packed[:, :nloc, :D] = ws[0]
        packed[:, :nloc, D] = ws[1]
        packed[:, :nloc, D + 1] = ws[2]
    return packed


def assemble(gathered, plan):
    """Per-rank packed partials (a list in rank order) -> (o [rows, ns, D], m, l
    [rows, ns]) in global split order."""
    cols = []
    for r, g in enumerate(gathered):
        s0, s1 = plan.splits(r)
        t0, t1 = plan.tokens(r)
        n = -(-(t1 - t0) // plan.split_len) if t1 > t0 else 0
        if n:
            cols.append(g[:, :n])
    full = torch.cat(cols, dim=1)
    if full.shape[1] != -(-plan.T // plan.split_len):
        raise RuntimeError("gathered partials do not cover the sequence")
    return full[..., :D].contiguous(), full[..., D].contiguous(), full[..., D + 1].contiguous()


def merge(o, m, l, out):
    """Merge in split order with the split merge kernel; out: bf16 [B, Hq, D]."""
    rows, ns, _ = o.shape
    ws = (o, m, l, kernels.Partials(o.data_ptr(), m.data_ptr(), l.data_ptr(), ns, 0))
    return kernels.merge_partials(ws, rows, out)


def all_gather_packed(packed, group=None):
    """All-gather of equal-shaped packed partials; returns the list in rank order."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    bufs = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(bufs, packed, group=group)
    return bufs


def attention_kv_split(q, kc, vc, plan, rank, group=None, num_warps=None):
    """One decode-attention call over a sequence split across the ranks of `group`.
    q: bf16 [B, Hq, 128] (the same on every rank); kc, vc: this rank's caches.
    Returns bf16 [B, Hq, 128] on every rank."""
    packed = local_partials(q, kc, vc, plan, rank, num_warps=num_warps)
    o, m, l = assemble(all_gather_packed(packed, group), plan)
    return merge(o, m, l, torch.empty_like(q))
