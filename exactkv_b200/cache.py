"""KV caches with the reference's interface (exactkv/cache.py): prefill_slot(b, x),
append(x), T, nbytes(), plus check_overflow().

CompressedKV holds one layer's keys (or values) in the exponent-coded format.
Full pages are encoded on the GPU by the sm_100a page encoder as they fill.
The newest, partly filled page lives as bf16 in a fixed area at the end of the
raw pool ([rows that did not fit | tail area]), with all its rows marked raw,
so attention reads it like any other page. Rows that do not fit have no hard
bound, so the pool grows on demand: after each page, check_overflow() makes
one host sync for all caches, and a page that overflowed is encoded again into
a pool at least twice as large. Data is never silently dropped.
"""
import torch

from . import kernels
from ._lib import CView
from .kernels import P, encode_pages


class CompressedKV:
    def __init__(self, B, TS, H, D, device="cuda", reserve=0.01):
        """B sequences of up to TS tokens (multiple of 16), H KV heads, head dim D (128).
        reserve: initial raw-row capacity as a fraction of all rows (grows on demand)."""
        if TS % P != 0 or D != 128:
            raise ValueError("TS must be a multiple of 16 and D = 128 (Qwen2/2.5/3, Llama-3 family)")
        NP = TS // P
        self.B, self.TS, self.H, self.D, self.dev = B, TS, H, D, torch.device(device)
        u8, i32 = dict(dtype=torch.uint8, device=device), dict(dtype=torch.int32, device=device)
        self.sm = torch.zeros(B, TS, H, D, **u8)
        self.code = torch.zeros(B, TS, H, D // 2, **u8)
        self.base = torch.zeros(B, NP, H, D, **u8)
        self.rowmask = torch.zeros(B, NP, H, **i32)
        self.rowoff = torch.zeros(B, NP, H, **i32)
        self.cnt = torch.zeros(1, **i32)        # raw-pool rows taken (may exceed cap: overflow)
        self._before = torch.zeros(1, **i32)    # counter before the last encoded page
        self.cap = max(64, int(B * TS * H * reserve))
        self.raw = torch.zeros(self.cap + B * H * P, D, dtype=torch.bfloat16, device=device)
        self.T = 0
        self.lens = [0] * B                     # tokens per sequence (all equal unless filled slot by slot)
        self.grows = 0
        self._pending = None                    # (strides, page) waiting for check_overflow
        self._rebind()

    # ------------------------------------------------------------------ internals
    def _rebind(self):
        """Views and the C-ABI descriptor that depend on the raw pool (rebuilt only when it grows)."""
        self._tailv = self.raw[self.cap:].view(self.B, self.H, P, self.D)
        self._toff = (self.cap + P * torch.arange(self.B * self.H, dtype=torch.int32, device=self.dev)
                      ).view(self.B, self.H)
        self._kargs = (self.sm, self.code, self.base, self.rowmask, self.rowoff, self.raw.view(torch.int16))
        self._cview = CView(self.sm.data_ptr(), self.code.data_ptr(), self.base.data_ptr(),
                            self.rowmask.data_ptr(), self.rowoff.data_ptr(), self.raw.data_ptr(),
                            self.raw.shape[0])

    def kernel_args(self):
        return self._kargs

    def kernel_view(self):
        return self._cview

    def _open_tail(self, pg):
        """Page pg becomes the open tail: all 16 rows raw, read from the tail area."""
        self.rowmask[:, pg] = (1 << P) - 1
        self.rowoff[:, pg] = self._toff

    def _buf(self):
        return dict(sm=self.sm, code=self.code, base=self.base, rowmask=self.rowmask, rowoff=self.rowoff,
                    raw=self.raw, cnt=self.cnt, cap=self.cap, TS=self.TS, H=self.H, D=self.D)

    def _grow(self, need):
        new_cap = max(2 * self.cap, need + self.cap // 4)
        raw = torch.zeros(new_cap + self.B * self.H * P, self.D, dtype=torch.bfloat16, device=self.dev)
        raw[: self.cap] = self.raw[: self.cap]
        raw[new_cap:] = self.raw[self.cap:]
        self.raw, self.cap = raw, new_cap
        self.grows += 1
        self._rebind()
        for b, t in enumerate(self.lens):                   # every open tail page moved with the pool
            if t < self.TS:
                self.rowoff[b, t // P] = self._toff[b]

    def _encode(self, src, strides, b0, pg0, nb, npg):
        self._before.copy_(self.cnt)
        encode_pages(src, strides, self._buf(), b0, pg0, nb, npg)

    def _redo(self, src, strides, b0, pg0, nb, npg):
        need = int(self.cnt.item())
        if need <= self.cap:
            return
        self._grow(need)
        self.cnt.copy_(self._before)
        encode_pages(src, strides, self._buf(), b0, pg0, nb, npg)
        if int(self.cnt.item()) > self.cap:
            raise RuntimeError("raw pool still too small after growing")

    # ------------------------------------------------------------------ interface
    def prefill_slot(self, b, x):
        """x: [1, T, H, D] bf16 (any strides, channels contiguous) for sequence slot b.
        The host-side append path needs every slot at the same T; slots of different
        lengths (a variable-length batch) are served by the device-length calls."""
        T = x.shape[1]
        full = T // P * P
        self.lens[b] = T
        if full:
            st = (x.stride(0), P * x.stride(1), x.stride(1), x.stride(2))
            self._encode(x, st, b, 0, 1, full // P)
            self._redo(x, st, b, 0, 1, full // P)          # one sync per prefilled sequence
        if full < self.TS:                                 # this slot's open tail page
            self.rowmask[b, full // P] = (1 << P) - 1
            self.rowoff[b, full // P] = self._toff[b]
        self._tailv[b, :, : T - full] = x[0, full:].transpose(0, 1)
        self.T = T

    def append(self, x):
        """x: [B, H, D] bf16, one new token per sequence."""
        if self._pending is not None:
            raise RuntimeError("call check_overflow() after a page boundary before appending again")
        self._tailv[:, :, self.T % P] = x
        self.T += 1
        self.lens = [self.T] * self.B
        if self.T % P == 0:
            pg = self.T // P - 1
            t = self._tailv
            st = (t.stride(0), 0, t.stride(2), t.stride(1))
            self._encode(t, st, 0, pg, self.B, 1)
            self._pending = (st, pg)
            if self.T < self.TS:
                self._open_tail(pg + 1)

    # ------------------------------------------------------------------ device-length steps
    def append_dev(self, x, T_dev):
        """Enqueue the append of one token per sequence at the device-side length
        *T_dev (no host bookkeeping; see kernels.append_token). The host's T is
        advanced with note_appended() once the step is enqueued."""
        kernels.append_token(x, self, T_dev)

    def note_appended(self, n=1):
        self.T += n
        self.lens = [t + n for t in self.lens]

    def lengths(self):
        """The sequences' token counts as a device int32 tensor (the T_dev of a
        variable-length batch for the device-length calls)."""
        return torch.tensor(self.lens, dtype=torch.int32, device=self.dev)

    def ensure_headroom(self, pages):
        """Before `pages` more pages are appended on the device: read the pool
        counter (one sync) and grow the pool so that even a page of nothing but
        raw rows always fits. Returns True when the pool moved (work enqueued
        with the old buffers, such as a captured graph, must be rebuilt)."""
        need = int(self.cnt.item()) + pages * self.B * self.H * P
        if need <= self.cap:
            return False
        self._grow(need)
        return True

    def finish_page(self, overflowed):
        """Called by check_overflow with this cache's result."""
        if self._pending is not None and overflowed:
            st, pg = self._pending
            self._redo(self._tailv, st, 0, pg, self.B, 1)
        self._pending = None

    def buffers(self):
        return dict(shape=(self.B, self.TS, self.H, self.D), sm=self.sm, code=self.code, base=self.base,
                    rowmask=self.rowmask, rowoff=self.rowoff, raw=self.raw)

    def nbytes(self):
        return sum(t.numel() * t.element_size()
                   for t in (self.sm, self.code, self.base, self.rowmask, self.rowoff, self.raw))


class BF16KV:
    """Plain bf16 cache [B, TS, H, D] with the same interface (the uncompressed sibling)."""

    def __init__(self, B, TS, H, D, device="cuda"):
        self.buf = torch.zeros(B, TS, H, D, dtype=torch.bfloat16, device=device)
        self.T = 0
        self.cnt = None

    def prefill_slot(self, b, x):
        self.buf[b, : x.shape[1]] = x[0]
        self.T = x.shape[1]

    def append(self, x):
        self.buf[:, self.T] = x
        self.T += 1

    def nbytes(self):
        return self.buf.numel() * 2


def check_overflow(caches):
    """After a page boundary: one host sync for all compressed caches, then re-encode
    any page that overflowed its raw pool. Returns the number of caches that grew.
    The same sync reads the kernels' device status word and raises on a fault."""
    cs = [c for c in caches if isinstance(c, CompressedKV) and c._pending is not None]
    if not cs:
        return 0
    counts = torch.cat([c.cnt for c in cs] + [kernels.status_tensor(cs[0].dev)]).cpu().tolist()
    if counts[-1] != 0:
        kernels.check_status(cs[0].dev)
    over = [n > c.cap for n, c in zip(counts, cs)]
    for c, o in zip(cs, over):
        c.finish_page(o)
    return sum(over)
