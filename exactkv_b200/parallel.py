"""Multi-GPU decode attention: batch sharding and the KV-sequence split.

Batch sharding needs no code here: sequences are independent, so every GPU
runs its own batch slice (one replica per GPU, no collective).

KV-sequence split (one long sequence over N GPUs). A global split plan
(ns splits of split_len tokens, chosen for N x SMs persistent CTAs) is cut
into N contiguous runs of whole splits; rank r keeps the pages of its run,
tokens [s0 * split_len, min(s1 * split_len, T)), in its own cache. The merge
has two levels:

1. each rank's split kernel writes the (o, m, l) partials of its splits into a
   local workspace, and exk_attn_merge_partial reduces them to ONE partial per
   (sequence, query head) row — the partial of the rank's whole run, in the
   layout of a single split's (o [rows, 128] unnormalised, m, l [rows]);
2. the ranks exchange those group partials (rows x 130 floats per rank, 16.6 KB
   at 32 query heads) and every rank merges them in rank order.

Partials depend only on their split's tokens and each level's order only on
the plan, so the result is bit-identical to one GPU running the same plan and
the same two levels (merge_two_level). Two exchanges: attention_kv_split
all-gathers the group partials with NCCL (all_gather_into_tensor);
PeerExchange keeps them in symmetric memory and the final merge kernel reads
the peers' partials in place over NVLink after a flag handshake (no collective
call).

Block layout (fp32, `block_floats(rows)` floats per rank): o [rows, 128], then
m [rows], then l [rows], padded to a multiple of 4 floats; a rank whose run
holds no tokens has group count 0 and its block is not read.

The reference has no multi-GPU path; the partials and the merge are those of
its split-K decode (exactkv/kernels.py:33-43, 142-165).
"""
import ctypes

import torch

from . import kernels
from ._lib import Partials, check, lib
from .kernels import D, P

MAX_RANKS = 16  # ranks the gathered and peer merges take


def block_floats(rows, nmax=1):
    """Floats of one rank's block: o [rows, nmax, D], m, l [rows, nmax], padded to 16 bytes."""
    return (rows * nmax * (D + 2) + 3) // 4 * 4


def block_views(flat, rows, nmax=1):
    """(o [rows, nmax, D], m [rows, nmax], l [rows, nmax]) views of one rank block."""
    n = rows * nmax
    return flat[: n * D].view(rows, nmax, D), flat[n * D: n * (D + 1)].view(rows, nmax), \
        flat[n * (D + 1): n * (D + 2)].view(rows, nmax)


class KVSplitPlan:
    """Global split plan and each rank's run of splits.

    bounds[r] .. bounds[r+1] are rank r's splits; token range of rank r:
    [bounds[r] * split_len, min(bounds[r+1] * split_len, T))."""

    def __init__(self, B, Hkv, T, world, ns, split_len, heads=0):
        if world < 1 or ns < 1 or split_len % P != 0 or ns * split_len < T:
            raise ValueError("invalid KV-split plan")
        if heads not in (0, 1, 2, 4, 8) or (heads and Hkv % heads):
            raise ValueError("heads per work item must be 0 (default) or 1, 2, 4, 8 dividing Hkv")
        self.B, self.Hkv, self.T, self.world = B, Hkv, T, world
        self.ns, self.split_len, self.heads = ns, split_len, heads
        self.bounds = [(r * ns) // world for r in range(world + 1)]

    MIN_ITEM_PAGES = 24  # pages per work item below which a smaller head group pays

    @classmethod
    def make(cls, B, Hkv, T, world, device=None):
        """The split kernel's own planner, sized for world x (SMs of one GPU) CTAs.
        When that leaves work items of fewer than MIN_ITEM_PAGES pages (one long
        sequence over many GPUs), halve the KV heads per item (each item then
        takes more pages and the ranks fewer splits), down to 2, until items
        reach that length: measured at 1 x 131072 per rank (split kernel + group
        merge), 8 GPUs 35.6 -> 26.7 us with 2 heads per item; 4 GPUs unchanged;
        on 1 and 2 GPUs the default head group is the fastest and is kept."""
        sms = kernels.num_sms(device)
        ns, sl = kernels.plan_splits(B, Hkv, T, device, num_ctas=world * sms)
        if sl // P >= cls.MIN_ITEM_PAGES:
            return cls(B, Hkv, T, world, ns, sl)
        hg = 8
        while Hkv % hg:
            hg //= 2
        best = None
        while hg >= 2:
            units = B * (Hkv // hg)
            per_rank = max(1, sms // units)          # splits per rank: one wave of items
            quantum = P * (8 // hg)                  # whole stages of 8 / hg pages per warp
            sl_h = -(-T // (world * per_rank))
            sl_h = -(-sl_h // quantum) * quantum
            best = (hg, sl_h)
            if sl_h // P >= cls.MIN_ITEM_PAGES:
                break
            hg //= 2
        if best is None:
            return cls(B, Hkv, T, world, ns, sl)
        hg, sl_h = best
        return cls(B, Hkv, T, world, -(-T // sl_h), sl_h, hg)

    def splits(self, rank):
        return self.bounds[rank], self.bounds[rank + 1]

    def tokens(self, rank):
        s0, s1 = self.splits(rank)
        return min(s0 * self.split_len, self.T), min(s1 * self.split_len, self.T)

    def count(self, rank):
        """Splits of rank `rank` that hold tokens."""
        t0, t1 = self.tokens(rank)
        return -(-(t1 - t0) // self.split_len) if t1 > t0 else 0

    @property
    def counts(self):
        return [self.count(r) for r in range(self.world)]

    @property
    def group_counts(self):
        """Columns of each rank's block the final merge reads: 1, or 0 for an empty run."""
        return [1 if self.count(r) else 0 for r in range(self.world)]

    @property
    def max_local(self):
        return max(1, max(self.bounds[r + 1] - self.bounds[r] for r in range(self.world)))

    def partials(self, o, m, l, ns):
        """exk_partials over o, m, l with ns columns and this plan's split length and heads."""
        return Partials(o.data_ptr(), m.data_ptr(), l.data_ptr(), ns, self.split_len, self.heads)


_BUF = {}  # (device, stream, rows, nmax, world) -> (workspace, local block, gathered blocks)


def _buffers(device, stream, rows, plan):
    nmax = plan.max_local
    key = (device.index, stream, rows, nmax, plan.world)
    bufs = _BUF.get(key)
    if bufs is None:
        f32 = dict(dtype=torch.float32, device=device)
        o, m, l = torch.empty(rows, nmax, D, **f32), torch.empty(rows, nmax, **f32), torch.empty(rows, nmax, **f32)
        ws = (o, m, l, Partials(o.data_ptr(), m.data_ptr(), l.data_ptr(), nmax, 0, 0))
        nb = block_floats(rows)
        bufs = _BUF[key] = (ws, torch.empty(nb, **f32), torch.empty(plan.world, nb, **f32))
    bufs[0][3].split_len = plan.split_len
    bufs[0][3].heads = plan.heads
    return bufs


def merge_partial(ws, rows, s0, s1, block):
    """exk_attn_merge_partial: splits [s0, s1) of workspace ws into the group
    partial of a flat block (block_floats(rows) floats), on the current stream."""
    o, m, l = block_views(block, rows)
    stream = torch.cuda.current_stream(block.device).cuda_stream
    check(lib.exk_attn_merge_partial(ctypes.byref(ws[3]), rows, s0, s1, o.data_ptr(), m.data_ptr(), l.data_ptr(),
                                     block.device.index, stream), "exk_attn_merge_partial")
    return block


def local_partials(q, kc, vc, plan, rank, num_warps=None, out=None):
    """Level 1 on rank `rank`: its split kernel over its splits, then their group
    partial in a flat block (`out`, or a buffer reused by the next call on the
    same stream and shapes). kc, vc hold the rank's tokens from position 0. A
    rank without tokens leaves the block unwritten (its group count is 0)."""
    rows = q.shape[0] * q.shape[1]
    stream = torch.cuda.current_stream(q.device).cuda_stream
    ws, local, _ = _buffers(q.device, stream, rows, plan)
    block = local if out is None else out
    n = plan.count(rank)
    if n:
        t0, t1 = plan.tokens(rank)
        kernels.attention_split(q, kc, vc, t1 - t0, ws, 0, n, num_warps=num_warps)
        merge_partial(ws, rows, 0, n, block)
    return block


def all_gather_blocks(local, world, group=None, out=None):
    """All-gather of the ranks' flat blocks into [world, block] (rank order):
    one all_gather_into_tensor on NCCL, the list form elsewhere (gloo)."""
    import torch.distributed as dist

    if out is None:
        out = torch.empty(world, local.numel(), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), local, group=group)
    return out


def assemble(gathered, plan, rows):
    """Gathered blocks [world, block] -> the group partials (o [rows, g, D], m, l
    [rows, g]) of the ranks with tokens, in rank order (a copy; the merge kernels
    read the blocks in place)."""
    if sum(plan.counts) != -(-plan.T // plan.split_len):
        raise RuntimeError("the ranks' splits do not cover the sequence")
    cols = [[], [], []]
    for r in range(plan.world):
        if plan.count(r):
            for c, x in zip(cols, block_views(gathered[r], rows)):
                c.append(x)
    return tuple(torch.cat(c, dim=1).contiguous() for c in cols)


def merge_gathered(gathered, plan, out):
    """Level 2 from gathered blocks [world, block]: the group partials merged in
    rank order into bf16 out [B, Hq, D] (exk_attn_merge_gathered)."""
    if plan.world > MAX_RANKS:
        raise ValueError(f"the gathered merge takes at most {MAX_RANKS} ranks")
    rows = out.shape[0] * out.shape[1]
    if gathered.shape != (plan.world, block_floats(rows)):
        raise ValueError("gathered blocks do not match the plan")
    counts = (ctypes.c_int32 * plan.world)(*plan.group_counts)
    stream = torch.cuda.current_stream(gathered.device).cuda_stream
    check(lib.exk_attn_merge_gathered(gathered.data_ptr(), plan.world, counts, 1, rows, out.data_ptr(),
                                      gathered.device.index, stream), "exk_attn_merge_gathered")
    return out


def merge(o, m, l, out):
    """Merge of partials already in order (splits or group partials); out: bf16 [B, Hq, D]."""
    rows, ns, _ = o.shape
    ws = (o, m, l, Partials(o.data_ptr(), m.data_ptr(), l.data_ptr(), ns, 0, 0))
    return kernels.merge_partials(ws, rows, out)


def merge_two_level(ws, plan, rows, out):
    """One GPU running the plan's two levels over a workspace that holds every
    split of the plan: each rank's run reduced to its group partial, then the
    groups merged in rank order — the same bits as the plan run on plan.world
    GPUs."""
    gathered = torch.empty(plan.world, block_floats(rows), dtype=torch.float32, device=ws[0].device)
    for r in range(plan.world):
        n = plan.count(r)
        if n:
            merge_partial(ws, rows, plan.bounds[r], plan.bounds[r] + n, gathered[r])
    return merge_gathered(gathered, plan, out)


def attention_kv_split(q, kc, vc, plan, rank, group=None, num_warps=None, out=None):
    """One decode-attention call over a sequence split across the ranks of `group`:
    the rank's split kernel and group partial, one NCCL all-gather of the group
    partials, the final merge. q: bf16 [B, Hq, 128] (the same on every rank);
    kc, vc: this rank's caches. Returns bf16 [B, Hq, 128] on every rank."""
    rows = q.shape[0] * q.shape[1]
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _, _, gathered = _buffers(q.device, stream, rows, plan)
    local = local_partials(q, kc, vc, plan, rank, num_warps=num_warps)
    all_gather_blocks(local, plan.world, group, out=gathered)
    return merge_gathered(gathered, plan, torch.empty_like(q) if out is None else out)


FLAG_BYTES = 256  # head of a PeerExchange buffer: uint32 flag words, one per rank


def merge_peers(blocks, plan, rank, flags, peer_flags, epoch, out):
    """exk_attn_merge_peers over group-partial blocks with explicit device
    addresses (ints): blocks[r] rank r's block, flags this GPU's flag words,
    peer_flags[p] word `rank` of peer p's flags (PeerExchange builds these from
    symmetric memory)."""
    w = plan.world
    dev = torch.cuda.current_device() if not out.is_cuda else out.device.index
    stream = torch.cuda.current_stream(dev).cuda_stream
    check(lib.exk_attn_merge_peers((ctypes.c_void_p * w)(*blocks), w, rank, (ctypes.c_int32 * w)(*plan.group_counts),
                                   1, out.shape[0] * out.shape[1], flags, (ctypes.c_void_p * w)(*peer_flags), epoch,
                                   out.data_ptr(), kernels.status_tensor(dev).data_ptr(), dev, stream),
          "exk_attn_merge_peers")
    return out


class PeerExchange:
    """KV-sequence split whose final merge reads the peers' group partials in place.

    One symmetric-memory buffer per rank (torch.distributed._symmetric_memory:
    every rank maps every peer's buffer): [flags | block 0 | block 1]. Call e
    (counted from 1 on every rank) runs this rank's split kernel into a local
    workspace and reduces it into block e % 2, then exk_attn_merge_peers
    signals the peers and merges all ranks' blocks of that parity over NVLink.
    Every rank must make the same calls in the same order. close() (or deleting
    the object) before destroy_process_group."""

    def __init__(self, plan, rows, group=None, device=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        if plan.world > MAX_RANKS:
            raise ValueError(f"the peer merge takes at most {MAX_RANKS} ranks")
        self.group = group if group is not None else dist.group.WORLD
        self.rank, self.world = dist.get_rank(self.group), dist.get_world_size(self.group)
        if self.world != plan.world:
            raise ValueError("the plan's world size differs from the group's")
        self.plan, self.rows = plan, rows
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        nb = block_floats(rows)
        head = FLAG_BYTES // 4
        self.buf = symm_mem.empty(head + 2 * nb, dtype=torch.float32, device=self.device)
        self.buf[:head].view(torch.int32).zero_()
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)                     # every rank's flags are zero before any signal
        ptrs = self.handle.buffer_ptrs
        self._flags = ptrs[self.rank]
        self._peer_flags = (ctypes.c_void_p * self.world)(*[ptrs[p] + 4 * self.rank for p in range(self.world)])
        self._blocks = [(ctypes.c_void_p * self.world)(*[ptrs[p] + FLAG_BYTES + par * nb * 4
                                                         for p in range(self.world)]) for par in (0, 1)]
        self._local = [self.buf[head + par * nb: head + (par + 1) * nb] for par in (0, 1)]
        f32 = dict(dtype=torch.float32, device=self.device)
        n = plan.max_local
        o, m, l = torch.empty(rows, n, D, **f32), torch.empty(rows, n, **f32), torch.empty(rows, n, **f32)
        self._ws = (o, m, l, plan.partials(o, m, l, n))
        self._counts = (ctypes.c_int32 * self.world)(*plan.group_counts)
        self.epoch = 0

    def attention(self, q, kc, vc, out=None, num_warps=None):
        """One decode-attention call: q bf16 [B, Hq, 128] (the same on every rank),
        kc, vc this rank's caches; returns bf16 [B, Hq, 128] on every rank."""
        self.split(q, kc, vc, num_warps=num_warps)
        return self.merge(torch.empty_like(q) if out is None else out)

    def split(self, q, kc, vc, num_warps=None):
        """First half of a call: the next epoch; this rank's split kernel and its
        group partial, written into its block of the epoch's parity."""
        if self.handle is None:
            raise RuntimeError("PeerExchange is closed")
        if q.shape[0] * q.shape[1] != self.rows:
            raise ValueError("q does not match the exchange's rows")
        self.epoch += 1
        n = self.plan.count(self.rank)
        if n:
            t0, t1 = self.plan.tokens(self.rank)
            kernels.attention_split(q, kc, vc, t1 - t0, self._ws, 0, n, num_warps=num_warps)
            merge_partial(self._ws, self.rows, 0, n, self._local[self.epoch & 1])

    def merge(self, out):
        """Second half: signal the peers, wait for theirs, merge every rank's group
        partial of this epoch into bf16 out [B, Hq, 128]."""
        dev = self.device.index
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(lib.exk_attn_merge_peers(self._blocks[self.epoch & 1], self.world, self.rank, self._counts, 1,
                                       self.rows, self._flags, self._peer_flags, self.epoch & 0xFFFFFFFF,
                                       out.data_ptr(), kernels.status_tensor(dev).data_ptr(), dev, stream),
              "exk_attn_merge_peers")
        return out

    def close(self):
        """Waits for this rank's work and releases the symmetric buffer (no peer
        reads it afterwards once every rank has closed at the same call count)."""
        if self.handle is not None:
            torch.cuda.synchronize(self.device)
            self.handle = None
            self.buf = None
            self._local = None
