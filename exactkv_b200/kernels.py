"""Drop-in replacement of the reference's exactkv/kernels.py, backed by the
sm_100a kernels of libexactkv_b200.so through its C ABI.

Same public names and argument meanings as the reference module
(exactkv/kernels.py:273-346): P, LOG2E, choose_split, attention_compressed,
attention_reference, decode_to_bf16, encode_pages. Everything runs on the
caller's current CUDA stream and nothing synchronises the host, except
check_status(). There is no CPU or Triton fallback: without the library this
module fails to import.

Differences from the reference, all invisible to callers of the reference API:
  * the split layout comes from call_plan() (persistent CTAs over the SMs:
    equal-length splits, or one equal run of pages per CTA when that balances
    better) instead of choose_split(); choose_split() is kept for compatibility;
  * BLOCK_N and num_stages are accepted and ignored (pages are 16 tokens and
    the TMA ring depth is fixed); num_warps selects 4 or 8 consumer warps
    (default 8) — the compressed and bf16 kernels called with the same value
    stay bit-identical, as in the reference;
  * the page encoder assigns raw-pool slots in (sequence, page, head) order,
    so rowoff/raw match encode_reference byte for byte as well.
"""
import ctypes

import torch

from ._lib import CView, Partials, check, lib

LOG2E = 1.4426950408889634
P = 16          # tokens per page
D = 128         # head dimension

_I32 = ctypes.c_int32


def choose_split(B, Hkv, T, BLOCK_N, target=512):
    """The reference's split rule (exactkv/kernels.py:273-277): at most `target`
    programs, split length a multiple of BLOCK_N. Returns (splits, split length)."""
    def cdiv(a, b):
        return (a + b - 1) // b

    ns = max(1, min(cdiv(T, BLOCK_N), target // max(1, B * Hkv)))
    split_len = cdiv(cdiv(T, ns), BLOCK_N) * BLOCK_N
    return cdiv(T, split_len), split_len


_SMS = {}


def num_sms(device=None):
    """SM count of a CUDA device (the number of persistent attention CTAs)."""
    dev = _device_index(device)
    if dev not in _SMS:
        n = lib.exk_num_sms(dev)
        if n <= 0:
            check(n if n < 0 else -1, "exk_num_sms")
        _SMS[dev] = n
    return _SMS[dev]


def plan_splits(B, Hkv, T, device=None, num_ctas=None):
    """(splits, split length in tokens) of the attention plan."""
    ns, sl = _I32(), _I32()
    ctas = num_ctas if num_ctas is not None else num_sms(device)
    check(lib.exk_plan_splits(B, Hkv, T, ctas, ctypes.byref(ns), ctypes.byref(sl)), "exk_plan_splits")
    return ns.value, sl.value


def call_plan(B, Hkv, T, device=None, num_warps=None, num_ctas=None, any_length=False):
    """(splits, split length) for one whole decode-attention call with host-side T:
    the balanced plan (split length 0: every CTA gets an equal run of the call's
    pages across sequence boundaries; exk_plan_balanced) when it is estimated
    faster than the uniform plan of plan_splits(), else the uniform one. The
    compressed and bf16 calls with the same arguments get the same plan.
    any_length: the plan of a device-length call with one length for the batch
    and capacity T (the balanced plan's kernel cuts the length it reads)."""
    ns = _I32()
    ctas = num_ctas if num_ctas is not None else num_sms(device)
    check(lib.exk_plan_balanced(B, Hkv, T, ctas, _consumer_warps(num_warps), int(bool(any_length)),
                                ctypes.byref(ns)), "exk_plan_balanced")
    if ns.value > 0:
        return ns.value, 0
    return plan_splits(B, Hkv, T, device, num_ctas)


def _device_index(device):
    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, int):
        return device
    device = torch.device(device)
    return device.index if device.index is not None else torch.cuda.current_device()


# ----------------------------------------------------------------------------- status word and scratch

_STATUS = {}   # device index -> int32[1] status word written by the kernels


def status_tensor(device):
    dev = _device_index(device)
    t = _STATUS.get(dev)
    if t is None:
        t = _STATUS[dev] = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
    return t


def check_status(device=None, reset=True):
    """Synchronises with the device and raises RuntimeError if a kernel recorded a
    fault (a timed-out wait or an out-of-range raw index) since the last check."""
    t = status_tensor(device)
    code = int(t.item())
    if code != 0:
        if reset:
            t.zero_()
        raise RuntimeError(f"exactkv_b200 device status {code}: {lib.exk_status_string(code).decode()}")
    return 0


# ----------------------------------------------------------------------------- split workspaces

_WS = {}  # (device, stream, rows, ns) -> (o, m, l, Partials); reused by calls on the same stream


def _workspace(device, stream, rows, ns, split_len, heads=0):
    """Split partials o [rows, ns, 128], m, l [rows, ns], for a plan of ns splits
    of split_len tokens and `heads` KV heads per work item (0: the default)."""
    key = (device.index, stream, rows, ns)
    ws = _WS.get(key)
    if ws is None:
        f32 = dict(device=device, dtype=torch.float32)
        o, m, l = torch.empty(rows, ns, D, **f32), torch.empty(rows, ns, **f32), torch.empty(rows, ns, **f32)
        ws = _WS[key] = (o, m, l, Partials(o.data_ptr(), m.data_ptr(), l.data_ptr(), ns, split_len))
    ws[3].split_len = split_len
    ws[3].heads = heads
    return ws


def _consumer_warps(num_warps):
    return 4 if num_warps is not None and num_warps <= 4 else 8


def _view_from_dict(c):
    raw = c["raw"]
    cv = CView(c["sm"].data_ptr(), c["code"].data_ptr(), c["base"].data_ptr(), c["rowmask"].data_ptr(),
               c["rowoff"].data_ptr(), raw.data_ptr(), raw.shape[0])
    return cv, c["shape"][1], c["shape"][2]


_ARGS_VIEWS = {}  # id(kernel_args() tuple) -> (the tuple, its exk_cview)


def _view_from_args(kargs):
    """exk_cview of a kernel_args() tuple (sm, code, base, rowmask, rowoff, raw as
    int16 [rows, 128]), the form a reference CompressedKV hands its kernels
    (exactkv/cache.py:39-47). A cache rebuilds that tuple only when its raw pool
    grows, so the view is kept per tuple object."""
    hit = _ARGS_VIEWS.get(id(kargs))
    if hit is not None and hit[0] is kargs:
        return hit[1]
    sm, code, base, rowmask, rowoff, raw = kargs
    cv = CView(sm.data_ptr(), code.data_ptr(), base.data_ptr(), rowmask.data_ptr(), rowoff.data_ptr(),
               raw.data_ptr(), raw.shape[0])
    if len(_ARGS_VIEWS) > 256:
        _ARGS_VIEWS.clear()
    _ARGS_VIEWS[id(kargs)] = (kargs, cv)
    return cv


def _cache_args(c):
    """(exk_cview, TS, Hkv) from a cache object or from its .buffers() dict, as the
    reference's _cache_args takes them (exactkv/kernels.py:302-307): this package's
    CompressedKV (its view is kept on the cache), or any cache with the reference's
    kernel_args() / .TS / .H, the reference's own CompressedKV included."""
    if isinstance(c, dict):
        return _view_from_dict(c)
    view = getattr(c, "kernel_view", None)
    if view is not None:
        return view(), c.TS, c.H
    return _view_from_args(c.kernel_args()), c.TS, c.H


def _check_q(q, T, TS):
    if q.dim() != 3 or q.shape[2] != D or q.dtype != torch.bfloat16 or not q.is_contiguous() or not q.is_cuda:
        raise ValueError("q must be a contiguous CUDA bf16 tensor [B, Hq, 128]")
    if not 0 < T <= TS:
        raise ValueError(f"T={T} out of range (1..{TS})")


def _check_out(out, q):
    """An output for q's shape: a CUDA tensor, or pinned host memory that the merge
    kernel writes directly (a zero-copy device-to-host result)."""
    if out.shape != q.shape or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 tensor shaped like q")
    if not out.is_cuda and not out.is_pinned():
        raise ValueError("out must be a CUDA tensor or pinned host memory")
    return out


def attention_split(q, kc, vc, T, ws, s0, s1, num_warps=None):
    """Split partials of the compressed attention for splits [s0, s1) of ws's plan
    (the per-GPU step of a KV-sequence split). ws: (o, m, l, Partials)."""
    ka, TS, Hkv = _cache_args(kc)
    va, _, _ = _cache_args(vc)
    _check_q(q, T, TS)
    B, Hq, _ = q.shape
    dev = q.device.index
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = lib.exk_attn_split_compressed(q.data_ptr(), ctypes.byref(ka), ctypes.byref(va), B, TS, Hkv, Hq, T, s0, s1,
                                       ctypes.byref(ws[3]), _consumer_warps(num_warps), D ** -0.5 * LOG2E,
                                       status_tensor(dev).data_ptr(), dev, stream)
    check(rc, "exk_attn_split_compressed")


def attention_split_bf16(q, k, v, T, ws, s0, s1, num_warps=None):
    """attention_split on uncompressed bf16 K, V [B, TS, Hkv, 128] (contiguous):
    the same partials as the compressed kernel for the same values and plan."""
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16 or not (k.is_contiguous() and v.is_contiguous()):
        raise ValueError("k and v must be contiguous bf16 [B, TS, Hkv, 128]")
    TS, Hkv = k.shape[1], k.shape[2]
    _check_q(q, T, TS)
    B, Hq, _ = q.shape
    dev = q.device.index
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = lib.exk_attn_split_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), B, TS, Hkv, Hq, T, s0, s1,
                                 ctypes.byref(ws[3]), _consumer_warps(num_warps), D ** -0.5 * LOG2E,
                                 status_tensor(dev).data_ptr(), dev, stream)
    check(rc, "exk_attn_split_bf16")


def merge_partials(ws, rows, out):
    """Merge of the workspace's splits into bf16 out [rows, 128] (a CUDA tensor or
    pinned host memory), on the workspace device's current stream."""
    dev = ws[0].device
    stream = torch.cuda.current_stream(dev).cuda_stream
    check(lib.exk_attn_merge(ctypes.byref(ws[3]), rows, out.data_ptr(), dev.index, stream), "exk_attn_merge")
    return out


def attention_compressed(q, kc, vc, T, BLOCK_N=64, num_warps=None, num_stages=1):
    """q [B, Hq, D] bf16 contiguous; kc, vc: CompressedKV objects (or their .buffers()
    dicts); T: valid tokens. Returns bf16 [B, Hq, D]. Bit-identical to
    attention_reference called with the same num_warps."""
    ka, TS, Hkv = _cache_args(kc)
    va, _, _ = _cache_args(vc)
    _check_q(q, T, TS)
    B, Hq, _ = q.shape
    dev = q.device.index
    stream = torch.cuda.current_stream(q.device).cuda_stream
    ns, sl = call_plan(B, Hkv, T, dev, num_warps)
    ws = _workspace(q.device, stream, B * Hq, ns, sl)
    out = torch.empty_like(q)
    rc = lib.exk_attention_compressed(q.data_ptr(), ctypes.byref(ka), ctypes.byref(va), B, TS, Hkv, Hq, T,
                                      ctypes.byref(ws[3]), out.data_ptr(), _consumer_warps(num_warps),
                                      D ** -0.5 * LOG2E, status_tensor(dev).data_ptr(), dev, stream)
    check(rc, "exk_attention_compressed")
    return out


def attention_reference(q, k, v, T, BLOCK_N=64, num_warps=None, num_stages=1):
    """The same computation on uncompressed bf16 K, V of shape [B, TS, Hkv, D] (contiguous)."""
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16 or not (k.is_contiguous() and v.is_contiguous()):
        raise ValueError("k and v must be contiguous bf16 [B, TS, Hkv, 128]")
    TS, Hkv = k.shape[1], k.shape[2]
    _check_q(q, T, TS)
    B, Hq, _ = q.shape
    dev = q.device.index
    stream = torch.cuda.current_stream(q.device).cuda_stream
    ns, sl = call_plan(B, Hkv, T, dev, num_warps)
    ws = _workspace(q.device, stream, B * Hq, ns, sl)
    out = torch.empty_like(q)
    rc = lib.exk_attention_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), B, TS, Hkv, Hq, T, ctypes.byref(ws[3]),
                                out.data_ptr(), _consumer_warps(num_warps), D ** -0.5 * LOG2E,
                                status_tensor(dev).data_ptr(), dev, stream)
    check(rc, "exk_attention_bf16")
    return out


def decode_to_bf16(c, T):
    """Compressed buffers (a .buffers() dict) -> bf16 [B, T, H, D] through the same
    decoder the attention kernel uses."""
    cv, TS, H = _view_from_dict(c)
    B = c["shape"][0]
    dev = c["sm"].device
    out = torch.empty(B, T, H, D, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    check(lib.exk_decode_to_bf16(ctypes.byref(cv), B, TS, H, T, out.data_ptr(),
                                 status_tensor(dev.index).data_ptr(), dev.index, stream), "exk_decode_to_bf16")
    return out


def encode_pages(src, strides, buf, b0, pg0, nb, npg):
    """Encode nb sequences x npg pages. src points at sequence b0's first page to
    encode; strides = (seq, page, token, head) in elements. buf: dict with sm, code,
    base, rowmask, rowoff, raw, cnt, cap, TS, H, D."""
    if buf["D"] != D or src.dtype != torch.bfloat16 or src.stride(-1) != 1:
        raise ValueError("src must be bf16 with contiguous channels; D = 128 only")
    dev = src.device
    stream = torch.cuda.current_stream(dev).cuda_stream
    s_b, s_pg, s_p, s_h = (int(s) for s in strides)
    rc = lib.exk_encode_pages(src.data_ptr(), s_b, s_pg, s_p, s_h, buf["sm"].data_ptr(), buf["code"].data_ptr(),
                              buf["base"].data_ptr(), buf["rowmask"].data_ptr(), buf["rowoff"].data_ptr(),
                              buf["raw"].data_ptr(), int(buf["cap"]), buf["cnt"].data_ptr(),
                              b0, pg0, nb, npg, buf["H"], buf["TS"], status_tensor(dev.index).data_ptr(),
                              dev.index, stream)
    check(rc, "exk_encode_pages")


# ----------------------------------------------------------------------------- device-length decode steps
#
# One decode step whose token count lives on the device (an int32 tensor, the
# tokens held before the step), so the whole step can be enqueued once and
# replayed (CUDA graphs): append_token writes and, at page boundaries, encodes;
# attention_compressed_devlen reads T from the device with the plan for the
# caches' capacity; advance_length moves the count on. No host synchronisation.

def _stride_of(T_dev, B):
    """0: one length for the batch (a 1-element tensor); 1: one per sequence."""
    if T_dev.dtype != torch.int32 or not T_dev.is_contiguous() or T_dev.numel() not in (1, B):
        raise ValueError("T_dev must be a contiguous int32 tensor of 1 or B lengths")
    return 0 if T_dev.numel() == 1 else 1


def devlen_plan(B, Hkv, TS, T_dev, device=None, num_warps=None):
    """(splits, split length) of a device-length call over caches of capacity
    TS: with one length for the batch the balanced plan where it is estimated
    faster (call_plan(any_length=True)), else plan_splits() for the capacity."""
    if _stride_of(T_dev, B) == 0:
        return call_plan(B, Hkv, TS, device, num_warps, any_length=True)
    return plan_splits(B, Hkv, TS, device)


def append_token(x, c, T_dev):
    """x [B, H, 128] bf16 (channels contiguous): the step's token for every
    sequence of CompressedKV `c`, appended at row T_dev (one length for the
    batch, or one per sequence)."""
    if x.dtype != torch.bfloat16 or x.stride(-1) != 1 or tuple(x.shape) != (c.B, c.H, D):
        raise ValueError("x must be bf16 [B, H, 128] with contiguous channels")
    dev = x.device
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.exk_append_token(x.data_ptr(), x.stride(0), x.stride(1), c.sm.data_ptr(), c.code.data_ptr(),
                              c.base.data_ptr(), c.rowmask.data_ptr(), c.rowoff.data_ptr(), c.raw.data_ptr(), c.cap,
                              c.cnt.data_ptr(), c.B, c.H, c.TS, T_dev.data_ptr(), _stride_of(T_dev, c.B),
                              status_tensor(dev.index).data_ptr(), dev.index, stream)
    check(rc, "exk_append_token")


def copy_from_host(dst, src):
    """dst (a contiguous CUDA tensor) <- src (a contiguous pinned CPU tensor of
    the same byte size): a kernel on the current stream reads the pinned
    memory over PCIe (exk_copy_from_host), so the copy needs no hand-off
    between the copy engine and the step's kernels. Returns dst."""
    if not (dst.is_cuda and dst.is_contiguous() and src.is_contiguous() and not src.is_cuda and src.is_pinned()):
        raise ValueError("dst must be a contiguous CUDA tensor and src a contiguous pinned host tensor")
    n = dst.numel() * dst.element_size()
    if src.numel() * src.element_size() != n:
        raise ValueError("dst and src must hold the same number of bytes")
    dev = dst.device
    check(lib.exk_copy_from_host(dst.data_ptr(), src.data_ptr(), n, dev.index,
                                 torch.cuda.current_stream(dev).cuda_stream), "exk_copy_from_host")
    return dst


def advance_length(T_dev, n=1):
    dev = T_dev.device
    check(lib.exk_advance_length(T_dev.data_ptr(), n, dev.index, torch.cuda.current_stream(dev).cuda_stream),
          "exk_advance_length")


def attention_compressed_devlen(q, kc, vc, T_dev, T_add=1, out=None, num_warps=None, advance=0):
    """Decode attention over the first min(TS, T_dev + T_add) tokens of the caches
    (T_dev: one int32 length for the batch or one per sequence), with the split
    plan's number of splits for their capacity TS, each sequence cut into that many
    equal page runs of its current length (see exk_attention_compressed_devlen); advance != 0
    then adds it to the batch length on the device (the end of a step)."""
    ka, TS, Hkv = _cache_args(kc)
    va, _, _ = _cache_args(vc)
    _check_q(q, TS, TS)
    B, Hq, _ = q.shape
    dev = q.device.index
    stream = torch.cuda.current_stream(q.device).cuda_stream
    ns, sl = devlen_plan(B, Hkv, TS, T_dev, dev, num_warps)
    ws = _workspace(q.device, stream, B * Hq, ns, sl)
    out = torch.empty_like(q) if out is None else _check_out(out, q)
    rc = lib.exk_attention_compressed_devlen(q.data_ptr(), ctypes.byref(ka), ctypes.byref(va), B, TS, Hkv, Hq, TS,
                                             T_dev.data_ptr(), T_add, _stride_of(T_dev, B), advance,
                                             ctypes.byref(ws[3]), out.data_ptr(), _consumer_warps(num_warps),
                                             D ** -0.5 * LOG2E, status_tensor(dev).data_ptr(), dev, stream)
    check(rc, "exk_attention_compressed_devlen")
    return out


# ----------------------------------------------------------------------------- paged caches

def _paged_warps(Hkv):
    """Consumer warps for a paged call: the head group (one page per head per stage)."""
    if Hkv % 8 == 0:
        return 8
    if Hkv % 4 == 0:
        return 4
    raise ValueError("paged attention needs a KV head count that is a multiple of 4")


def _paged_check(q, block_table, seq_lens):
    B = q.shape[0]
    for t, name in ((block_table, "block_table"), (seq_lens, "seq_lens")):
        if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous CUDA int32 tensor")
    if block_table.dim() != 2 or block_table.shape[0] != B or seq_lens.shape != (B,):
        raise ValueError("block_table must be [B, max_pages] and seq_lens [B]")
    return block_table.shape[1]


def attention_paged(q, kc, vc, block_table, seq_lens, out=None):
    """Decode attention over paged caches: kc, vc are CompressedKV objects (or
    their .buffers() dicts) used as page pools — their [B', TS'] buffers seen as
    B' * TS' / 16 pages — block_table int32 [B, max_pages] names each
    sequence's pages in the pool, seq_lens int32 [B] its tokens (both on the
    device). Same results as attention_compressed_devlen over the same pages
    laid out contiguously (exk_attention_compressed_paged)."""
    ka, TS, Hkv = _cache_args(kc)
    va, _, _ = _cache_args(vc)
    Bp = kc["shape"][0] if isinstance(kc, dict) else kc.B
    max_pages = _paged_check(q, block_table, seq_lens)
    _check_q(q, max_pages * P, max_pages * P)
    B, Hq, _ = q.shape
    dev = q.device.index
    stream = torch.cuda.current_stream(q.device).cuda_stream
    ns, sl = plan_splits(B, Hkv, max_pages * P, dev)
    ws = _workspace(q.device, stream, B * Hq, ns, sl)
    out = torch.empty_like(q) if out is None else _check_out(out, q)
    rc = lib.exk_attention_compressed_paged(q.data_ptr(), ctypes.byref(ka), ctypes.byref(va), Bp * TS // P, Hkv, B,
                                            Hq, block_table.data_ptr(), max_pages, seq_lens.data_ptr(),
                                            ctypes.byref(ws[3]), out.data_ptr(), _paged_warps(Hkv),
                                            D ** -0.5 * LOG2E, status_tensor(dev).data_ptr(), dev, stream)
    check(rc, "exk_attention_compressed_paged")
    return out


def attention_reference_paged(q, k, v, block_table, seq_lens, out=None):
    """The bf16 sibling of attention_paged over bf16 pools k, v of shape
    [B', TS', Hkv, 128] (contiguous; pages of 16 rows), bit-identical for the
    same values."""
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16 or not (k.is_contiguous() and v.is_contiguous()):
        raise ValueError("k and v must be contiguous bf16 [B', TS', Hkv, 128]")
    Hkv = k.shape[-2]
    pool_pages = k.numel() // (Hkv * D * P)
    max_pages = _paged_check(q, block_table, seq_lens)
    _check_q(q, max_pages * P, max_pages * P)
    B, Hq, _ = q.shape
    dev = q.device.index
    stream = torch.cuda.current_stream(q.device).cuda_stream
    ns, sl = plan_splits(B, Hkv, max_pages * P, dev)
    ws = _workspace(q.device, stream, B * Hq, ns, sl)
    out = torch.empty_like(q) if out is None else _check_out(out, q)
    rc = lib.exk_attention_bf16_paged(q.data_ptr(), k.data_ptr(), v.data_ptr(), pool_pages, Hkv, B, Hq,
                                      block_table.data_ptr(), max_pages, seq_lens.data_ptr(), ctypes.byref(ws[3]),
                                      out.data_ptr(), _paged_warps(Hkv), D ** -0.5 * LOG2E,
                                      status_tensor(dev).data_ptr(), dev, stream)
    check(rc, "exk_attention_bf16_paged")
    return out


def attention_reference_devlen(q, k, v, T_dev, T_add=0, out=None, num_warps=None):
    """The bf16 sibling of attention_compressed_devlen on k, v [B, TS, Hkv, 128]
    (bit-identical for the same values, lengths and num_warps)."""
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16 or not (k.is_contiguous() and v.is_contiguous()):
        raise ValueError("k and v must be contiguous bf16 [B, TS, Hkv, 128]")
    TS, Hkv = k.shape[1], k.shape[2]
    _check_q(q, TS, TS)
    B, Hq, _ = q.shape
    dev = q.device.index
    stream = torch.cuda.current_stream(q.device).cuda_stream
    ns, sl = devlen_plan(B, Hkv, TS, T_dev, dev, num_warps)
    ws = _workspace(q.device, stream, B * Hq, ns, sl)
    out = torch.empty_like(q) if out is None else _check_out(out, q)
    rc = lib.exk_attention_bf16_devlen(q.data_ptr(), k.data_ptr(), v.data_ptr(), B, TS, Hkv, Hq, TS, T_dev.data_ptr(),
                                       T_add, _stride_of(T_dev, B), 0, ctypes.byref(ws[3]), out.data_ptr(),
                                       _consumer_warps(num_warps), D ** -0.5 * LOG2E,
                                       status_tensor(dev).data_ptr(), dev, stream)
    check(rc, "exk_attention_bf16_devlen")
    return out
