"""KV caches behind the reference's cache interface (exactkv/cache.py: prefill_slot,
append, T, nbytes, buffers, kernel_args, check_overflow), built around a token
count that lives on the device.

Buffers (the format the kernels read; include/exactkv_b200.h):
  sm, code   u8  [B, TS, H, 128] / [B, TS, H, 64]
  base       u8  [B, TS/16, H, 128]
  rowmask    i32 [B, TS/16, H]        bit r: token r of the page is a raw row
  rowoff     i32 [B, TS/16, H]        pool row of the page's first raw row
  raw        bf16 [cap + B*H*16, 128] pool rows [0, cnt) for encoded pages,
                                      then one 16-row open page per (sequence, head)

The newest, partly filled page of every sequence lives in its open-page rows and
is marked all-raw (rowmask 0xFFFF, rowoff at those rows), so attention reads it
like any other page; when it fills, the device append kernel encodes it in place
and opens the next one (exk_append_token).

Pool policy, this package's own: every append goes through that device kernel,
and at each page boundary the host makes one check (check_overflow(), one sync
for all caches) that keeps at least one worst-case page (every row raw, B*H*16
rows) free in every pool. So an append can never overflow and no page is ever
encoded twice. Only a prefill, whose raw rows have no useful bound, can
overflow: its pages are then encoded again into a grown pool.
"""
import torch

from . import kernels
from ._lib import CView
from .kernels import P

_GROW_ALIGN = 256   # pool capacities are multiples of this many rows


class RawPool:
    """The raw bf16 rows of one cache: `cap` slots for encoded pages followed by
    the open-page area of `nseq` x `H` pages of 16 rows."""

    def __init__(self, nseq, H, D, cap, device):
        self.nseq, self.H, self.D, self.device = nseq, H, D, device
        self.cap = cap
        self.rows = torch.zeros(cap + nseq * H * P, D, dtype=torch.bfloat16, device=device)
        self.moves = 0

    def open_pages(self):
        """The open-page area as [nseq, H, 16, D]."""
        return self.rows[self.cap:].view(self.nseq, self.H, P, self.D)

    def open_page_rows(self):
        """int32 [nseq, H]: pool row of each open page's first row."""
        first = self.cap + P * torch.arange(self.nseq * self.H, dtype=torch.int32, device=self.device)
        return first.view(self.nseq, self.H)

    def enlarge(self, used, need):
        """Re-allocates with room for at least `need` slots, keeping slots [0, used)
        and the open pages. Capacity grows by half at least, so a cache that keeps
        overflowing pays a logarithmic number of copies."""
        cap = max(need, self.cap + self.cap // 2)
        cap = -(-cap // _GROW_ALIGN) * _GROW_ALIGN
        rows = torch.empty(cap + self.nseq * self.H * P, self.D, dtype=torch.bfloat16, device=self.device)
        if used:
            rows[:used].copy_(self.rows[:used])
        rows[cap:].copy_(self.rows[self.cap:])
        self.rows, self.cap = rows, cap
        self.moves += 1


class CompressedKV:
    """One layer's keys (or values) for B sequences of up to TS tokens, H KV heads,
    head dim 128. `reserve`: initial pool slots as a fraction of all rows."""

    def __init__(self, B, TS, H, D, device="cuda", reserve=0.01):
        if TS % P != 0 or D != 128:
            raise ValueError("TS must be a multiple of 16 and D = 128 (Qwen2/2.5/3, Llama-3 family)")
        self.B, self.TS, self.H, self.D = B, TS, H, D
        self.dev = torch.device(device)
        u8 = dict(dtype=torch.uint8, device=self.dev)
        i32 = dict(dtype=torch.int32, device=self.dev)
        npages = TS // P
        self.sm = torch.zeros(B, TS, H, D, **u8)
        self.code = torch.zeros(B, TS, H, D // 2, **u8)
        self.base = torch.zeros(B, npages, H, D, **u8)
        self.rowmask = torch.zeros(B, npages, H, **i32)
        self.rowoff = torch.zeros(B, npages, H, **i32)
        self.cnt = torch.zeros(1, **i32)                 # pool slots taken by encoded pages
        self.pool = RawPool(B, H, D, max(64, int(B * TS * H * reserve)), self.dev)
        self.lens = [0] * B                              # tokens per sequence
        self.T = 0                                       # tokens of the batch (the last prefilled slot's, as the reference)
        self._t_dev = torch.zeros(1, **i32)              # T on the device, for the append kernel
        self._t_dev_stale = False                        # T moved by device-length steps
        self._checked = True                             # headroom verified since the last page boundary
        self._bind()

    # ------------------------------------------------------------------ views
    @property
    def raw(self):
        return self.pool.rows

    @property
    def cap(self):
        return self.pool.cap

    @property
    def grows(self):
        return self.pool.moves

    def _bind(self):
        """Descriptors that name the pool's storage; rebuilt when it moves."""
        self._kargs = (self.sm, self.code, self.base, self.rowmask, self.rowoff, self.pool.rows.view(torch.int16))
        self._view = CView(self.sm.data_ptr(), self.code.data_ptr(), self.base.data_ptr(), self.rowmask.data_ptr(),
                           self.rowoff.data_ptr(), self.pool.rows.data_ptr(), self.pool.rows.shape[0])

    def kernel_args(self):
        return self._kargs

    def kernel_view(self):
        return self._view

    def tail_offsets(self):
        return self.pool.open_page_rows()

    def encoder_buffers(self):
        """The dict kernels.encode_pages writes into."""
        return dict(sm=self.sm, code=self.code, base=self.base, rowmask=self.rowmask, rowoff=self.rowoff,
                    raw=self.pool.rows, cnt=self.cnt, cap=self.pool.cap, TS=self.TS, H=self.H, D=self.D)

    def buffers(self):
        return dict(shape=(self.B, self.TS, self.H, self.D), sm=self.sm, code=self.code, base=self.base,
                    rowmask=self.rowmask, rowoff=self.rowoff, raw=self.pool.rows)

    def nbytes(self):
        return sum(t.numel() * t.element_size()
                   for t in (self.sm, self.code, self.base, self.rowmask, self.rowoff, self.pool.rows))

    # ------------------------------------------------------------------ pool
    def _relocate(self, used, need):
        """Moves the pool (keeping slots [0, used)) and re-points every open page."""
        self.pool.enlarge(used, need)
        self._bind()
        first = self.pool.open_page_rows()
        for b, t in enumerate(self.lens):
            if t < self.TS:
                self.rowoff[b, t // P] = first[b]

    def headroom_rows(self, pages=1):
        """Slots that `pages` pages of the whole batch need when every row is raw."""
        return pages * self.B * self.H * P

    def ensure_headroom(self, pages):
        """Before `pages` more pages are appended: one sync to read the slot counter,
        then grow so that even `pages` pages of nothing but raw rows fit. Returns
        True when the pool moved (work enqueued with the old buffers, such as a
        captured graph, must be rebuilt)."""
        return self._make_room(int(self.cnt.item()), pages)

    def _make_room(self, used, pages):
        need = used + self.headroom_rows(pages)
        self._checked = True
        if need <= self.pool.cap:
            return False
        # a quarter window of slack: the next check, after `pages` pages that
        # escaped a few per cent of their rows as usual, must not find the pool
        # short again (each growth moves the pool and invalidates captured work)
        self._relocate(used, need + self.headroom_rows(pages) // 4)
        return True

    # ------------------------------------------------------------------ filling
    def prefill_slot(self, b, x):
        """x: [1, T, H, D] bf16 (any strides, channels contiguous) for sequence slot b.
        Full pages are encoded (raw-pool slots follow the slot order of the calls);
        the rest goes to the slot's open page. Syncs once (the pool counter) and,
        if the pool overflowed, encodes the slot's pages again into a larger pool."""
        T = x.shape[1]
        if not 0 < T <= self.TS:
            raise ValueError(f"prefill of {T} tokens into a cache of {self.TS}")
        npg = T // P
        if npg:
            strides = (x.stride(0), P * x.stride(1), x.stride(1), x.stride(2))
            start = self.cnt.clone()
            kernels.encode_pages(x, strides, self.encoder_buffers(), b, 0, 1, npg)
            used = int(self.cnt.item())
            if used > self.pool.cap:
                self._relocate(int(start.item()), used)
                self.cnt.copy_(start)
                kernels.encode_pages(x, strides, self.encoder_buffers(), b, 0, 1, npg)
                if int(self.cnt.item()) > self.pool.cap:
                    raise RuntimeError("raw pool still too small after growing")
        self.lens[b] = T
        if npg < self.TS // P:
            self.rowmask[b, npg] = (1 << P) - 1
            self.rowoff[b, npg] = self.pool.open_page_rows()[b]
            self.pool.open_pages()[b, :, : T - npg * P] = x[0, npg * P:].transpose(0, 1)
        self.T = T
        self._t_dev.fill_(T)
        self._t_dev_stale = False
        self._checked = False

    def append(self, x):
        """x: [B, H, D] bf16, one new token per sequence (every sequence at the
        same length T). The device append kernel writes it and, when the page
        fills, encodes the page and opens the next. A boundary that the host has
        not checked since the previous one is checked here first."""
        if any(t != self.T for t in self.lens):
            raise RuntimeError("append needs every sequence at the same length (use append_dev for varlen)")
        if self.T >= self.TS:
            raise RuntimeError("cache full")
        if self.T % P == P - 1 and not self._checked:
            self.ensure_headroom(1)
        if self._t_dev_stale:                            # device-length steps moved T since
            self._t_dev.fill_(self.T)
            self._t_dev_stale = False
        kernels.append_token(x, self, self._t_dev)
        kernels.advance_length(self._t_dev, 1)
        self._count(1)
        if self.T % P == 0:
            self._checked = False

    # ------------------------------------------------------------------ device-length steps
    def append_dev(self, x, T_dev):
        """Enqueues the append of one token per sequence at the device-side length
        *T_dev (no host bookkeeping; see kernels.append_token). The host's count
        is advanced with note_appended() once the step is enqueued."""
        kernels.append_token(x, self, T_dev)

    def note_appended(self, n=1):
        """Records n tokens appended by device-length steps (append_dev)."""
        self._count(n)
        self._t_dev_stale = True

    def _count(self, n):
        self.T += n
        self.lens = [t + n for t in self.lens]

    def lengths(self):
        """The sequences' token counts as a device int32 tensor (the T_dev of a
        variable-length batch for the device-length calls)."""
        return torch.tensor(self.lens, dtype=torch.int32, device=self.dev)


class BF16KV:
    """Uncompressed bf16 cache [B, TS, H, D] with the same interface."""

    def __init__(self, B, TS, H, D, device="cuda"):
        self.buf = torch.zeros(B, TS, H, D, dtype=torch.bfloat16, device=device)
        self.T = 0
        self.cnt = None

    def prefill_slot(self, b, x):
        T = x.shape[1]
        self.buf[b, :T].copy_(x[0])
        self.T = T

    def append(self, x):
        self.buf[:, self.T].copy_(x)
        self.T += 1

    def nbytes(self):
        return self.buf.numel() * self.buf.element_size()


def check_overflow(caches):
    """The host check after a page boundary: one sync reads the slot counters of
    all compressed caches (and the kernels' status word, raising on a fault), then
    every pool with less than one worst-case page free grows. Returns the number
    of caches that grew."""
    cs = [c for c in caches if isinstance(c, CompressedKV) and not c._checked]
    if not cs:
        return 0
    status = kernels.status_tensor(cs[0].dev)
    vals = torch.cat([c.cnt for c in cs] + [status]).tolist()
    if vals[-1] != 0:
        kernels.check_status(cs[0].dev)
    return sum(int(c._make_room(used, 1)) for c, used in zip(cs, vals[:-1]))
