"""Device-length decode steps replayed from a CUDA graph (exactkv_b200.graph).

Two identical cache pairs take the same tokens: one through the host path
(append, check_overflow at every page), one through a captured step (append
at the device-side length, attention with the capacity's plan, advance). The
graph's pools start too small, so it must grow them ahead of time and
capture again. Every step's output equals the host path's attention with the
same split plan bit for bit, and at the end both caches hold the same bytes.
"""
import pytest
import torch

import exactkv_b200 as ekv
from exactkv_b200 import kernels, synthetic
from exactkv_b200.graph import DeviceLength, GraphedStep

pytestmark = pytest.mark.gpu


def _pair(k, v, T0, TS, reserve):
    B, _, H, D = k.shape
    kc = ekv.CompressedKV(B, TS, H, D, reserve=reserve)
    vc = ekv.CompressedKV(B, TS, H, D, reserve=reserve)
    for b in range(B):
        kc.prefill_slot(b, k[b:b + 1, :T0].contiguous())
        vc.prefill_slot(b, v[b:b + 1, :T0].contiguous())
    return kc, vc


def _host_attention(q, kc, vc, T, ns_cap):
    """What the device-length call computes: the capacity plan's number of splits,
    each ceil(ceil(T / 16) / ns_cap) pages long, run over the splits that hold
    tokens."""
    sl = -(-(-(-T // 16)) // ns_cap) * 16
    n = -(-T // sl)
    B, Hq, _ = q.shape
    o = torch.empty(B * Hq, n, 128, device="cuda")
    m = torch.empty(B * Hq, n, device="cuda")
    l = torch.empty(B * Hq, n, device="cuda")
    ws = (o, m, l, kernels.Partials(o.data_ptr(), m.data_ptr(), l.data_ptr(), n, sl))
    kernels.attention_split(q, kc, vc, T, ws, 0, n)
    return kernels.merge_partials(ws, B * Hq, torch.empty_like(q))


def test_graphed_steps_match_host_path():
    B, Hq, Hkv, T0, TS, steps = 2, 16, 4, 700, 1024, 90
    k = synthetic.make_kv(B, TS, Hkv, seed=71, key=True, raw_frac=0.02)
    v = synthetic.make_kv(B, TS, Hkv, seed=72, key=False, raw_frac=0.02)
    qs = torch.stack([synthetic.make_q(B, Hq, seed=100 + i) for i in range(steps)])
    ka, va = _pair(k, v, T0, TS, reserve=1.0)
    kg, vg = _pair(k, v, T0, TS, reserve=0.002)
    ns, _ = kernels.plan_splits(B, Hkv, TS)
    ekv.decode_attention(qs[0], kg, vg)          # configures the kernels before any capture

    length = DeviceLength([kg, vg])
    q_in = torch.empty_like(qs[0])
    k_in = torch.empty(B, Hkv, 128, dtype=torch.bfloat16, device="cuda")
    v_in = torch.empty_like(k_in)
    out = torch.empty_like(q_in)

    def body():
        kg.append_dev(k_in, length.t)
        vg.append_dev(v_in, length.t)
        kernels.attention_compressed_devlen(q_in, kg, vg, length.t, 1, out=out)
        length.advance(1)

    gs = GraphedStep(body, length, check_pages=2)
    for i in range(steps):
        t = T0 + i
        if i == steps // 2:
            grows = kg.grows + vg.grows
            gs.check_pages = 40          # a wider window: the next check must grow the pools and capture again
        q_in.copy_(qs[i])
        k_in.copy_(k[:, t])
        v_in.copy_(v[:, t])
        gs.step()
        ka.append(k[:, t])
        va.append(v[:, t])
        if ka.T % 16 == 0:
            ekv.check_overflow([ka, va])
        ref = _host_attention(qs[i], ka, va, ka.T, ns)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), i
    torch.cuda.synchronize()
    assert gs.captures >= 2 and kg.grows + vg.grows > grows
    assert int(length.t.item()) == kg.T == ka.T == T0 + steps
    for a, g in ((ka, kg), (va, vg)):
        for f in ("sm", "code", "base", "rowmask"):
            assert torch.equal(getattr(a, f), getattr(g, f)), f
        # encoded pages share pool slots; the open tail page points into each pool's own tail area
        assert torch.equal(a.rowoff[:, :a.T // 16], g.rowoff[:, :g.T // 16])
        assert torch.equal(g.rowoff[:, g.T // 16], g.tail_offsets())
        n = int(a.cnt.item())
        assert n == int(g.cnt.item())
        assert torch.equal(a.raw[:n], g.raw[:n])
        assert torch.equal(kernels.decode_to_bf16(a.buffers(), a.T), kernels.decode_to_bf16(g.buffers(), g.T))
    assert torch.equal(kernels.decode_to_bf16(kg.buffers(), kg.T), k[:, :kg.T])
    kernels.check_status()
    gs.close()


def test_output_to_pinned_host_memory():
    """The merge writes straight into pinned host memory (a zero-copy result, also
    from a replayed graph): the same bits as a device output; pageable host
    memory is refused before any launch."""
    B, T, Hq, Hkv = 4, 1000, 32, 8
    TS = 1024
    k = synthetic.make_kv(B, TS, Hkv, seed=81, key=True)
    v = synthetic.make_kv(B, TS, Hkv, seed=82, key=False)
    q = synthetic.make_q(B, Hq, seed=83)
    kc, vc = _pair(k, v, T, TS, 0.05)
    lens = torch.full((1,), T, dtype=torch.int32, device="cuda")
    ref = kernels.attention_compressed_devlen(q, kc, vc, lens, 0)
    host = torch.empty(B, Hq, 128, dtype=torch.bfloat16).pin_memory()
    kernels.attention_compressed_devlen(q, kc, vc, lens, 0, out=host)
    torch.cuda.synchronize()
    assert torch.equal(host.view(torch.int16), ref.cpu().view(torch.int16))
    host.zero_()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        kernels.attention_compressed_devlen(q, kc, vc, lens, 0, out=host)   # warm the workspace on this stream
        with torch.cuda.graph(g, stream=s):
            kernels.attention_compressed_devlen(q, kc, vc, lens, 0, out=host)
    host.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(host.view(torch.int16), ref.cpu().view(torch.int16))
    del g
    with pytest.raises(ValueError):
        kernels.attention_compressed_devlen(q, kc, vc, lens, 0, out=torch.empty(B, Hq, 128, dtype=torch.bfloat16))
    kernels.check_status()


@pytest.mark.parametrize("nbytes", [16, 393216, 5 * 2 ** 20 + 16])
def test_copy_from_host(nbytes):
    """kernels.copy_from_host: a kernel copies pinned host memory into device
    memory (one grid-stride pass of 16-byte loads, several in flight per thread
    for large copies), byte for byte; pageable host memory is refused before any
    launch."""
    import ctypes
    from exactkv_b200._lib import lib
    g = torch.Generator().manual_seed(nbytes)
    src = torch.randint(-2 ** 31, 2 ** 31 - 1, (nbytes // 4,), generator=g, dtype=torch.int32).pin_memory()
    dst = torch.zeros(nbytes // 4, dtype=torch.int32, device="cuda")
    kernels.copy_from_host(dst, src)
    torch.cuda.synchronize()
    assert torch.equal(dst.cpu(), src)
    pageable = torch.zeros(64, dtype=torch.int32)
    assert lib.exk_copy_from_host(dst.data_ptr(), pageable.data_ptr(), 256, 0, None) == -1
    with pytest.raises(ValueError):
        kernels.copy_from_host(dst[:64], pageable)
    kernels.check_status()
