"""Decode steps captured once as a CUDA graph and replayed.

A step built from the device-length calls (CompressedKV.append_dev,
kernels.attention_compressed_devlen, kernels.advance_length) reads the token
count from a device tensor, so the same enqueued work serves every step of a
growing cache and no step needs the host. Host synchronisation is left to one
check every `check_pages` pages: it keeps every raw pool at least
`check_pages + 1` worst-case pages ahead (so the device never runs out of
slots: nothing has to be re-encoded, unlike the reference's
overflow-and-redo, exactkv/cache.py:149-158), reads the kernels' status word,
and captures the graph again when a pool had to grow (its buffers moved).
"""
import torch

from . import kernels
from .kernels import P


class DeviceLength:
    """The token count of a set of equally long caches, held on the device."""

    def __init__(self, caches):
        self.caches = list(caches)
        T = self.caches[0].T
        if any(c.T != T for c in self.caches):
            raise ValueError("the caches must hold the same number of tokens")
        self.t = torch.tensor([T], dtype=torch.int32, device=self.caches[0].sm.device)

    @property
    def T(self):
        return self.caches[0].T

    def advance(self, n=1):
        """Enqueue *t += n (the end of a step)."""
        kernels.advance_length(self.t, n)

    def note(self, n=1):
        for c in self.caches:
            c.note_appended(n)


class GraphedStep:
    """step(): replays `body` — a function that enqueues one decode step on the
    current stream using `length.t` and ends by advancing it (length.advance(),
    or attention_compressed_devlen(..., advance=1)); it may fork work onto other
    streams that join the current one — from a CUDA graph. The first call, and
    any call after a pool grew, captures it."""

    def __init__(self, body, length, check_pages=8):
        self.body, self.length, self.check_pages = body, length, check_pages
        self.graph = None
        self.captures = 0
        self._next_check = length.T

    def _check(self):
        moved = False
        for c in self.length.caches:
            moved |= c.ensure_headroom(self.check_pages + 1)
        kernels.check_status(self.length.t.device)
        self._next_check = (self.length.T // P + self.check_pages) * P
        return moved

    def _capture(self):
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.body()
        self.graph = g
        self.captures += 1

    def step(self):
        if self.length.T >= self._next_check:
            if self._check() or self.graph is None:
                self._capture()
        elif self.graph is None:
            self._capture()
        self.graph.replay()
        self.length.note(1)

    def close(self):
        self.graph = None
