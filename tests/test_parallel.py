"""KV-sequence split over ranks (exactkv_b200.parallel): two-level merge.

CPU (gloo, world size 2 and 3): each rank computes its splits' partials and
their group partial with the oracle, the blocks go through the real all-gather
and assemble code, and the merge of the gathered group partials must equal the
single-process oracle running the same two levels bit for bit (partials depend
only on their split's tokens).
GPU: ranks emulated one after another on one GPU (every rank's cache holds only
its own pages) must be bit-identical to one kernel run over the whole cache
with the same plan and the same two levels, through the gathered merge and
through the peer merge (flags already set, so nothing waits), and within
tolerance of float64 attention; the peer merge's wait on a flag that nothing
sets gives up with its status code; with two or more GPUs, the same through
NCCL and through symmetric-memory peer reads.
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from exactkv_b200 import parallel
from exactkv_b200.parallel import KVSplitPlan, block_floats, block_views
from oracle import attention as oatt
from oracle.bf16 import bits_to_f32, f32_to_bits
from oracle.synth import synth_kv, synth_q

D = 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_plan_partition_covers_every_split_once():
    for (ns, sl, T, world) in [(9, 464, 4096, 2), (9, 464, 4096, 4), (3, 48, 130, 8), (128, 1024, 131072, 8),
                               (5, 16, 70, 3)]:
        plan = KVSplitPlan(1, 8, T, world, ns, sl)
        assert plan.bounds[0] == 0 and plan.bounds[-1] == ns
        assert all(a <= b for a, b in zip(plan.bounds, plan.bounds[1:]))
        toks = [plan.tokens(r) for r in range(world)]
        assert toks[0][0] == 0 and toks[-1][1] == T
        assert all(toks[r][1] == toks[r + 1][0] for r in range(world - 1))
        assert all(t0 % 16 == 0 for t0, _ in toks)
    with pytest.raises(ValueError):
        KVSplitPlan(1, 8, 4096, 2, 4, 464)     # splits do not cover T


def test_plan_head_groups_for_short_items(monkeypatch):
    """KVSplitPlan.make keeps the default head group while items hold >= 24 pages
    and halves it (down to 2) otherwise; every rank's items still fit one wave
    of its SMs and the splits cover the sequence."""
    from exactkv_b200 import kernels
    monkeypatch.setattr(kernels, "num_sms", lambda device=None: 148)
    for world, heads in [(1, 0), (2, 0), (4, 4), (8, 2)]:
        plan = KVSplitPlan.make(1, 8, 131072, world)
        assert plan.heads == heads, world
        assert plan.ns * plan.split_len >= 131072 and plan.split_len % 16 == 0
        units = 8 // (plan.heads or 8)
        assert all(units * n <= 148 for n in plan.counts), (world, plan.counts)
        if plan.heads:
            assert plan.split_len // 16 >= KVSplitPlan.MIN_ITEM_PAGES
            assert (plan.split_len // 16) % (8 // plan.heads) == 0   # whole stages per warp


def _oracle_block(qb, kb, vb, plan, rank):
    """One rank's flat block: the group partial of its splits, by the oracle over
    the rank's tokens only."""
    t0, t1 = plan.tokens(rank)
    B, Hq, _ = qb.shape
    rows = B * Hq
    flat = torch.zeros(block_floats(rows), dtype=torch.float32)
    n = plan.count(rank)
    if n:
        o, m, l = oatt.split_partials(qb, kb[:, t0:t1], vb[:, t0:t1], t1 - t0, splits=(n, plan.split_len))
        go, gm, gl = oatt.merge_group(o.reshape(rows, n, D), m.reshape(rows, n), l.reshape(rows, n))
        bo, bm, bl = block_views(flat, rows)
        bo[:, 0] = torch.from_numpy(go)
        bm[:, 0] = torch.from_numpy(gm)
        bl[:, 0] = torch.from_numpy(gl)
    return flat


def _oracle_two_level(qb, kb, vb, T, plan):
    """The single-process oracle: all splits, each rank's run merged to its group
    partial, the groups merged in rank order."""
    B, Hq, _ = qb.shape
    rows = B * Hq
    o, m, l = oatt.split_partials(qb, kb, vb, T, splits=(plan.ns, plan.split_len))
    o, m, l = o.reshape(rows, plan.ns, D), m.reshape(rows, plan.ns), l.reshape(rows, plan.ns)
    groups = [oatt.merge_group(o[:, a:a + n], m[:, a:a + n], l[:, a:a + n])
              for a, n in zip(plan.bounds, plan.counts) if n]
    go = np.stack([g[0] for g in groups], 1)
    gm = np.stack([g[1] for g in groups], 1)
    gl = np.stack([g[2] for g in groups], 1)
    return f32_to_bits(oatt.merge(go, gm, gl)).reshape(B, Hq, D)


def _gloo_rank(rank, world, port, args, outdir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        B, T, Hq, Hkv, ns, sl = args
        qb, kb, vb = synth_q(11, B, Hq), synth_kv(12, B, T, Hkv), synth_kv(13, B, T, Hkv, key=False)
        plan = KVSplitPlan(B, Hkv, T, world, ns, sl)
        gathered = parallel.all_gather_blocks(_oracle_block(qb, kb, vb, plan, rank), world)
        o, m, l = parallel.assemble(gathered, plan, B * Hq)
        out = oatt.merge(o.numpy(), m.numpy(), l.numpy())
        np.save(os.path.join(outdir, f"out{rank}.npy"), f32_to_bits(out).reshape(B, Hq, D))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,B,T,Hq,Hkv,ns,sl", [(2, 2, 1000, 8, 2, 5, 208), (3, 1, 700, 4, 1, 7, 112)])
def test_kv_split_gloo_bit_identical(world, B, T, Hq, Hkv, ns, sl):
    args = (B, T, Hq, Hkv, ns, sl)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_gloo_rank, args=(world, _free_port(), args, d), nprocs=world, join=True,
                           start_method="spawn")
        outs = [np.load(os.path.join(d, f"out{r}.npy")) for r in range(world)]
    qb, kb, vb = synth_q(11, B, Hq), synth_kv(12, B, T, Hkv), synth_kv(13, B, T, Hkv, key=False)
    plan = KVSplitPlan(B, Hkv, T, world, ns, sl)
    ref = _oracle_two_level(qb, kb, vb, T, plan)
    for out in outs:
        assert np.array_equal(out, ref)
    # and the two-level result is the attention: within tolerance of float64
    f64 = oatt.attention_f64(qb, kb, vb, T)
    got = bits_to_f32(ref).astype(np.float64)
    assert (np.abs(got - f64) / oatt.tolerance(qb, kb, vb, T, f64)).max() <= 1.0


# ------------------------------------------------------------------ GPU

def _rank_caches(k, v, plan, rank):
    import exactkv_b200 as ekv
    t0, t1 = plan.tokens(rank)
    caches = []
    for x in (k, v):
        B, _, H, _ = x.shape
        TS = max(16, -(-(t1 - t0) // 16) * 16)
        c = ekv.CompressedKV(B, TS, H, D, reserve=1.0)
        for b in range(B):
            if t1 > t0:
                c.prefill_slot(b, x[b:b + 1, t0:t1].contiguous())
        caches.append(c)
    return caches


def _full_run(q, k, v, T, plan):
    """One GPU, the whole cache: every split of the plan, then its two levels."""
    import exactkv_b200 as ekv
    from exactkv_b200 import kernels
    B, _, H, _ = k.shape
    TS = -(-T // 16) * 16
    kc, vc = ekv.CompressedKV(B, TS, H, D, reserve=1.0), ekv.CompressedKV(B, TS, H, D, reserve=1.0)
    for b in range(B):
        kc.prefill_slot(b, k[b:b + 1, :T].contiguous())
        vc.prefill_slot(b, v[b:b + 1, :T].contiguous())
    Hq = q.shape[1]
    ns = plan.ns
    o = torch.empty(B * Hq, ns, D, device="cuda")
    m = torch.empty(B * Hq, ns, device="cuda")
    l = torch.empty(B * Hq, ns, device="cuda")
    ws = (o, m, l, plan.partials(o, m, l, ns))
    kernels.attention_split(q, kc, vc, T, ws, 0, ns)
    return parallel.merge_two_level(ws, plan, B * Hq, torch.empty_like(q))


def _check_f64(out, q, k, v, T):
    from gpu_util import to_bits
    qb, kb, vb = to_bits(q), to_bits(k[:, :T]), to_bits(v[:, :T])
    f64 = oatt.attention_f64(qb, kb, vb, T)
    got = bits_to_f32(to_bits(out)).astype(np.float64)
    assert (np.abs(got - f64) / oatt.tolerance(qb, kb, vb, T, f64)).max() <= 1.0


@pytest.mark.gpu
@pytest.mark.parametrize("world,B,T,Hq,Hkv", [(2, 1, 8192, 32, 8), (4, 2, 3000, 28, 4), (8, 1, 131072, 32, 8),
                                              (8, 1, 50, 32, 8)])   # most ranks hold no tokens
def test_kv_split_emulated_ranks_bit_identical(world, B, T, Hq, Hkv):
    from exactkv_b200 import kernels, synthetic
    k = synthetic.make_kv(B, T, Hkv, seed=21, device="cuda")
    v = synthetic.make_kv(B, T, Hkv, seed=22, key=False, device="cuda")
    q = synthetic.make_q(B, Hq, seed=23, device="cuda")
    plan = KVSplitPlan.make(B, Hkv, T, world)
    rows = B * Hq
    gathered = torch.full((world, block_floats(rows)), float("nan"), device="cuda")
    for r in range(world):
        kc, vc = _rank_caches(k, v, plan, r)
        parallel.local_partials(q, kc, vc, plan, r, out=gathered[r])
    out = parallel.merge_gathered(gathered, plan, torch.empty_like(q))
    o, m, l = parallel.assemble(gathered, plan, rows)
    out2 = parallel.merge(o, m, l, torch.empty_like(q))
    ref = _full_run(q, k, v, T, plan)
    kernels.check_status()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    assert torch.equal(out2.view(torch.int16), ref.view(torch.int16))
    if T <= 8192:
        _check_f64(out, q, k, v, T)


@pytest.mark.gpu
@pytest.mark.parametrize("world,B,T,Hq,Hkv", [(2, 1, 8192, 32, 8), (3, 2, 3000, 28, 4), (8, 1, 131072, 32, 8),
                                              (8, 1, 50, 32, 8)])
def test_peer_merge_emulated_ranks_bit_identical(world, B, T, Hq, Hkv):
    from exactkv_b200 import kernels, synthetic
    k = synthetic.make_kv(B, T, Hkv, seed=41, device="cuda")
    v = synthetic.make_kv(B, T, Hkv, seed=42, key=False, device="cuda")
    q = synthetic.make_q(B, Hq, seed=43, device="cuda")
    plan = KVSplitPlan.make(B, Hkv, T, world)
    blocks = []
    for r in range(world):
        kc, vc = _rank_caches(k, v, plan, r)
        blocks.append(parallel.local_partials(q, kc, vc, plan, r).clone())
    ref = _full_run(q, k, v, T, plan)
    epoch = 5
    for rank in range(world):                       # every rank's view: all peers already signalled
        flags = torch.full((world,), epoch, dtype=torch.int32, device="cuda")
        sink = torch.zeros(world, dtype=torch.int32, device="cuda")   # stands in for the peers' flag words
        out = parallel.merge_peers([b.data_ptr() for b in blocks], plan, rank, flags.data_ptr(),
                                   [sink.data_ptr() + 4 * p for p in range(world)], epoch, torch.empty_like(q))
        kernels.check_status()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), rank
        assert all(sink[p].item() == (epoch if p != rank else 0) for p in range(world))


@pytest.mark.gpu
def test_peer_merge_wait_gives_up():
    """A peer that never signals: the merge's bounded wait (2 s) ends with
    EXK_S_PEER_TIMEOUT in the status word and the context stays usable."""
    from exactkv_b200 import kernels, synthetic
    B, T, Hq, Hkv, world = 1, 2048, 32, 8, 2
    k = synthetic.make_kv(B, T, Hkv, seed=51, device="cuda")
    v = synthetic.make_kv(B, T, Hkv, seed=52, key=False, device="cuda")
    q = synthetic.make_q(B, Hq, seed=53, device="cuda")
    plan = KVSplitPlan.make(B, Hkv, T, world)
    kc, vc = _rank_caches(k, v, plan, 0)
    block = parallel.local_partials(q, kc, vc, plan, 0).clone()
    flags = torch.zeros(world, dtype=torch.int32, device="cuda")       # nothing will set flags[1]
    sink = torch.zeros(world, dtype=torch.int32, device="cuda")
    parallel.merge_peers([block.data_ptr()] * world, plan, 0, flags.data_ptr(),
                         [sink.data_ptr() + 4 * p for p in range(world)], 1, torch.empty_like(q))
    torch.cuda.synchronize()
    st = kernels.status_tensor(torch.device("cuda", 0))
    assert st.item() == 6                              # EXK_S_PEER_TIMEOUT
    with pytest.raises(RuntimeError, match="peer merge"):
        kernels.check_status()
    assert st.item() == 0
    # the context is intact: a whole merge with the flag set now runs
    flags[1] = 1
    out = parallel.merge_peers([block.data_ptr()] * world, plan, 0, flags.data_ptr(),
                               [sink.data_ptr() + 4 * p for p in range(world)], 1, torch.empty_like(q))
    torch.cuda.synchronize()
    kernels.check_status()
    assert torch.isfinite(out.float()).all()


def _nccl_rank(rank, world, port, outdir):
    import torch.distributed as dist
    from exactkv_b200 import kernels, synthetic
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        B, T, Hq, Hkv = 1, 16384, 32, 8
        k = synthetic.make_kv(B, T, Hkv, seed=31, device="cuda")
        v = synthetic.make_kv(B, T, Hkv, seed=32, key=False, device="cuda")
        q = synthetic.make_q(B, Hq, seed=33, device="cuda")
        plan = KVSplitPlan.make(B, Hkv, T, world)
        kc, vc = _rank_caches(k, v, plan, rank)
        out = parallel.attention_kv_split(q, kc, vc, plan, rank)
        ref = _full_run(q, k, v, T, plan)
        kernels.check_status()
        ok = torch.equal(out.view(torch.int16), ref.view(torch.int16))
        # the peer merge over symmetric memory: several calls (both blocks of
        # each rank in turn), each against its own single-GPU run
        ex = parallel.PeerExchange(plan, B * Hq)
        for i in range(5):
            qi = synthetic.make_q(B, Hq, seed=300 + i, device="cuda")
            got = ex.attention(qi, kc, vc)
            want = _full_run(qi, k, v, T, plan)
            kernels.check_status()
            ok = ok and torch.equal(got.view(torch.int16), want.view(torch.int16))
        ex.close()
        dist.barrier()
        open(os.path.join(outdir, f"ok{rank}"), "w").write("1" if ok else "0")
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_kv_split_nccl_bit_identical():
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_nccl_rank, args=(world, _free_port(), d), nprocs=world, join=True, start_method="spawn")
        assert all(open(os.path.join(d, f"ok{r}")).read() == "1" for r in range(world))
