"""Multi-GPU decode attention: batch sharding and the KV-sequence split.

Batch sharding needs no code here: sequences are independent, so every GPU
runs its own batch slice (one replica per GPU, no collective).

KV-sequence split (one long sequence over N GPUs). A global split plan
(ns splits of split_len tokens, chosen for N x SMs persistent CTAs) is cut
into N contiguous runs of whole splits; rank r keeps the pages of its run,
tokens [s0 * split_len, min(s1 * split_len, T)), in its own cache. Each rank's
split kernel writes the (o, m, l) partials of its splits straight into one
flat block, one all-gather (NCCL over NVLink) exchanges the blocks, and the
gathered-merge kernel merges all ns partials in global split order from the
gathered buffer. Partials depend only on their split's tokens, so the result
is bit-identical to a single GPU running the same plan.

Rank block layout (fp32, `block_floats(rows, nmax)` floats, nmax = the longest
run of splits): o [rows, nmax, 128], then m [rows, nmax], then l [rows, nmax],
padded to a multiple of 4 floats; rank r's first counts[r] columns are valid.

Two exchanges: attention_kv_split all-gathers the blocks with NCCL
(all_gather_into_tensor) and merges the gathered copy; PeerExchange keeps each
rank's blocks in symmetric memory and its merge kernel reads the peers' blocks
in place over NVLink after a flag handshake (no collective call; the merge is
the only kernel that touches another GPU).

The reference has no multi-GPU path; the partials and the merge are those of
its split-K decode (exactkv/kernels.py:33-43, 142-165).
"""
import ctypes

import torch

from . import kernels
from ._lib import Partials, check, lib
from .kernels import D, P

MAX_RANKS = 16  # ranks the gathered merge takes


def block_floats(rows, nmax):
    """Floats of one rank's block (o, m, l padded to 16 bytes)."""
    return (rows * nmax * (D + 2) + 3) // 4 * 4


def block_views(flat, rows, nmax):
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

    @classmethod
    def make(cls, B, Hkv, T, world, device=None):
        """The split kernel's own planner, sized for world x (SMs of one GPU) CTAs,
        with the default KV heads per work item (fewer heads per item need fewer
        splits, but measured slower at 1 x 131072 on one and on two GPUs)."""
        ns, sl = kernels.plan_splits(B, Hkv, T, device, num_ctas=world * kernels.num_sms(device))
        return cls(B, Hkv, T, world, ns, sl)

    def partials(self, o, m, l, ns):
        """exk_partials over o, m, l with ns columns and this plan's split length and heads."""
        return Partials(o.data_ptr(), m.data_ptr(), l.data_ptr(), ns, self.split_len, self.heads)

    def splits(self, rank):
        return self.bounds[rank], self.bounds[rank + 1]

    def tokens(self, rank):
        s0, s1 = self.splits(rank)
        return min(s0 * self.split_len, self.T), min(s1 * self.split_len, self.T)

    def count(self, rank):
        """Splits of rank `rank` that hold tokens (the valid columns of its block)."""
        t0, t1 = self.tokens(rank)
        return -(-(t1 - t0) // self.split_len) if t1 > t0 else 0

    @property
    def counts(self):
        return [self.count(r) for r in range(self.world)]

    @property
    def max_local(self):
        return max(1, max(self.bounds[r + 1] - self.bounds[r] for r in range(self.world)))


_BUF = {}  # (device, stream, rows, nmax, world) -> (local block, gathered blocks, Partials)


def _buffers(device, stream, rows, plan):
    nmax = plan.max_local
    key = (device.index, stream, rows, nmax, plan.world)
    bufs = _BUF.get(key)
    if bufs is None:
        n = block_floats(rows, nmax)
        gathered = torch.empty(plan.world, n, dtype=torch.float32, device=device)
        local = torch.empty(n, dtype=torch.float32, device=device)
        o, m, l = block_views(local, rows, nmax)
        bufs = _BUF[key] = (local, gathered, Partials(o.data_ptr(), m.data_ptr(), l.data_ptr(), nmax, 0, 0))
    bufs[2].split_len = plan.split_len
    bufs[2].heads = plan.heads
    return bufs


def local_partials(q, kc, vc, plan, rank, num_warps=None):
    """Rank `rank`'s partials as one flat block (columns past plan.count(rank) are
    left unwritten). kc, vc hold the rank's tokens from position 0. The block is
    a buffer reused by the next call on the same stream and shapes."""
    rows = q.shape[0] * q.shape[1]
    stream = torch.cuda.current_stream(q.device).cuda_stream
    local, _, part = _buffers(q.device, stream, rows, plan)
    n = plan.count(rank)
    if n:
        t0, t1 = plan.tokens(rank)
        o, m, l = block_views(local, rows, plan.max_local)
        kernels.attention_split(q, kc, vc, t1 - t0, (o, m, l, part), 0, n, num_warps=num_warps)
    return local


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
    """Gathered blocks [world, block] -> (o [rows, ns, D], m, l [rows, ns]) in global
    split order (a copy; the merge kernel reads the blocks in place)."""
    cols = [[], [], []]
    for r in range(plan.world):
        n = plan.count(r)
        if n:
            for c, x in zip(cols, block_views(gathered[r], rows, plan.max_local)):
                c.append(x[:, :n])
    o, m, l = (torch.cat(c, dim=1).contiguous() for c in cols)
    if o.shape[1] != -(-plan.T // plan.split_len):
        raise RuntimeError("gathered partials do not cover the sequence")
    return o, m, l


def merge_gathered(gathered, plan, out):
    """Merge of the gathered blocks in global split order into bf16 out [B, Hq, D]
    (exk_attn_merge_gathered, on the current stream)."""
    if plan.world > MAX_RANKS:
        raise ValueError(f"the gathered merge takes at most {MAX_RANKS} ranks")
    rows = out.shape[0] * out.shape[1]
    if gathered.shape != (plan.world, block_floats(rows, plan.max_local)):
        raise ValueError("gathered blocks do not match the plan")
    counts = (ctypes.c_int32 * plan.world)(*plan.counts)
    stream = torch.cuda.current_stream(out.device).cuda_stream
    check(lib.exk_attn_merge_gathered(gathered.data_ptr(), plan.world, counts, plan.max_local, rows,
                                      out.data_ptr(), out.device.index, stream), "exk_attn_merge_gathered")
    return out


def merge(o, m, l, out):
    """Merge of partials already in global split order; out: bf16 [B, Hq, D]."""
    rows, ns, _ = o.shape
    ws = (o, m, l, Partials(o.data_ptr(), m.data_ptr(), l.data_ptr(), ns, 0))
    return kernels.merge_partials(ws, rows, out)


def attention_kv_split(q, kc, vc, plan, rank, group=None, num_warps=None, out=None):
    """One decode-attention call over a sequence split across the ranks of `group`:
    the rank's split kernel, one all-gather, the gathered merge.
    q: bf16 [B, Hq, 128] (the same on every rank); kc, vc: this rank's caches.
    Returns bf16 [B, Hq, 128] on every rank."""
    rows = q.shape[0] * q.shape[1]
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _, gathered, _ = _buffers(q.device, stream, rows, plan)
    local = local_partials(q, kc, vc, plan, rank, num_warps=num_warps)
    all_gather_blocks(local, plan.world, group, out=gathered)
    return merge_gathered(gathered, plan, torch.empty_like(q) if out is None else out)


FLAG_BYTES = 256  # head of a PeerExchange buffer: uint32 flag words, one per rank


def merge_peers(blocks, plan, rank, flags, peer_flags, epoch, out):
    """exk_attn_merge_peers with explicit device addresses (ints): blocks[r] rank
    r's block, flags this GPU's flag words, peer_flags[p] word `rank` of peer p's
    flags (PeerExchange builds these from symmetric memory)."""
    w = plan.world
    dev = out.device.index
    stream = torch.cuda.current_stream(out.device).cuda_stream
    check(lib.exk_attn_merge_peers((ctypes.c_void_p * w)(*blocks), w, rank, (ctypes.c_int32 * w)(*plan.counts),
                                   plan.max_local, out.shape[0] * out.shape[1], flags,
                                   (ctypes.c_void_p * w)(*peer_flags), epoch, out.data_ptr(),
                                   kernels.status_tensor(dev).data_ptr(), dev, stream), "exk_attn_merge_peers")
    return out


class PeerExchange:
    """KV-sequence split whose merge reads the peers' partial blocks in place.

    One symmetric-memory buffer per rank (torch.distributed._symmetric_memory:
    every rank maps every peer's buffer): [flags | block 0 | block 1]. Call e
    (counted from 1 on every rank) writes this rank's partials into block e % 2
    with the split kernel, then exk_attn_merge_peers signals the peers and
    merges all ranks' blocks of that parity over NVLink. Every rank must make
    the same calls in the same order. close() (or deleting the object) before
    destroy_process_group."""

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
        nb = block_floats(rows, plan.max_local)
        head = FLAG_BYTES // 4
        self.buf = symm_mem.empty(head + 2 * nb, dtype=torch.float32, device=self.device)
        self.buf[:head].view(torch.int32).zero_()
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)                     # every rank's flags are zero before any signal
        ptrs = self.handle.buffer_ptrs
        self._flags = ptrs[self.rank]
        self._peer_flags = (ctypes.c_void_p * self.world)(*[ptrs[p] + 4 * self.rank for p in range(self.world)])
        self._blocks, self._ws = [], []
        for par in (0, 1):
            off = FLAG_BYTES + par * nb * 4
            self._blocks.append((ctypes.c_void_p * self.world)(*[ptrs[p] + off for p in range(self.world)]))
            o, m, l = block_views(self.buf[head + par * nb: head + (par + 1) * nb], rows, plan.max_local)
            self._ws.append((o, m, l, plan.partials(o, m, l, plan.max_local)))
        self._counts = (ctypes.c_int32 * self.world)(*plan.counts)
        self.epoch = 0

    def attention(self, q, kc, vc, out=None, num_warps=None):
        """One decode-attention call: q bf16 [B, Hq, 128] (the same on every rank),
        kc, vc this rank's caches; returns bf16 [B, Hq, 128] on every rank."""
        self.split(q, kc, vc, num_warps=num_warps)
        return self.merge(torch.empty_like(q) if out is None else out)

    def split(self, q, kc, vc, num_warps=None):
        """First half of a call: the next epoch; this rank's split kernel writes
        its partials into its block of the epoch's parity."""
        if self.handle is None:
            raise RuntimeError("PeerExchange is closed")
        if q.shape[0] * q.shape[1] != self.rows:
            raise ValueError("q does not match the exchange's rows")
        self.epoch += 1
        n = self.plan.count(self.rank)
        if n:
            t0, t1 = self.plan.tokens(self.rank)
            kernels.attention_split(q, kc, vc, t1 - t0, self._ws[self.epoch & 1], 0, n, num_warps=num_warps)

    def merge(self, out):
        """Second half: signal the peers, wait for theirs, merge every rank's block
        of this epoch into bf16 out [B, Hq, 128]."""
        dev = out.device.index
        stream = torch.cuda.current_stream(out.device).cuda_stream
        check(lib.exk_attn_merge_peers(self._blocks[self.epoch & 1], self.world, self.rank, self._counts,
                                       self.plan.max_local, self.rows, self._flags, self._peer_flags,
                                       self.epoch & 0xFFFFFFFF, out.data_ptr(),
                                       kernels.status_tensor(dev).data_ptr(), dev, stream), "exk_attn_merge_peers")
        return out

    def close(self):
        """Waits for this rank's work and releases the symmetric buffer (no peer
        reads it afterwards once every rank has closed at the same call count)."""
        if self.handle is not None:
            torch.cuda.synchronize(self.device)
            self.handle = None
            self.buf = None
