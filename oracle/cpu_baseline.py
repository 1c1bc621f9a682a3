"""CPU timing of the oracle path (test/benchmark infrastructure only).

Used by bench.py for its `cpu_baseline` field and its `--impl reference` arm:
the numpy restatement of the reference's codec (decode) plus its split-K
attention, run over (sequence, KV head) tasks in a process pool started with
`spawn`, one process per host core. Inputs are made on the CPU from the same
synthetic distribution as the GPU benchmark and encoded with the oracle
encoder; workers read them from memory-mapped .npy files.
"""
import os
import tempfile
import time

import numpy as np

from . import attention as oatt
from . import codec as ocodec

FIELDS = ("sm", "code", "base", "rowmask", "rowoff", "raw")


def build_sample(nseq, T, Hkv, Hq, theta, seed, make_kv, make_q):
    """Encodes nseq sequences of T tokens (K and V) with the oracle; writes the arrays
    to a temporary directory and returns (dir, compressed bytes per sequence)."""
    d = tempfile.mkdtemp(prefix="exk_cpu_")
    TS = -(-T // 16) * 16
    nbytes = 0
    for tag, key in (("k", True), ("v", False)):
        x = make_kv(seed + (0 if key else 1), nseq, TS, Hkv, theta=theta, key=key)
        c = ocodec.encode(x)
        for f in FIELDS:
            np.save(os.path.join(d, f"{tag}_{f}.npy"), c[f])
        raw_rows = int(sum(bin(int(m)).count("1") for m in c["rowmask"].ravel()))
        nbytes += nseq * TS * Hkv * 192 + c["base"].size + 8 * c["rowmask"].size + raw_rows * 256
    np.save(os.path.join(d, "q.npy"), make_q(seed + 2, nseq, Hq))
    meta = np.array([nseq, T, Hkv, Hq], np.int64)
    np.save(os.path.join(d, "meta.npy"), meta)
    return d, nbytes // nseq


def _load(d):
    arr = {k: np.load(os.path.join(d, f"{k}.npy"), mmap_mode="r") for k in ("q", "meta")}
    for tag in ("k", "v"):
        arr[tag] = {f: np.load(os.path.join(d, f"{tag}_{f}.npy"), mmap_mode="r") for f in FIELDS}
    return arr


def head_task(args):
    """Decode K and V of one (sequence, KV head) and run the reference attention for
    its query heads. Returns the elapsed seconds."""
    d, b, h = args
    t0 = time.perf_counter()
    a = _load(d)
    nseq, T, Hkv, Hq = (int(x) for x in a["meta"])
    G = Hq // Hkv
    TS = a["k"]["sm"].shape[1]
    dec = {}
    for tag in ("k", "v"):
        c = a[tag]
        one = dict(shape=(1, TS, 1, 128), sm=np.asarray(c["sm"][b:b + 1, :, h:h + 1]),
                   code=np.asarray(c["code"][b:b + 1, :, h:h + 1]), base=np.asarray(c["base"][b:b + 1, :, h:h + 1]),
                   rowmask=np.asarray(c["rowmask"][b:b + 1, :, h:h + 1]),
                   rowoff=np.asarray(c["rowoff"][b:b + 1, :, h:h + 1]), raw=c["raw"])
        dec[tag] = ocodec.decode(one, T)
    q = np.asarray(a["q"][b:b + 1, h * G:(h + 1) * G])
    oatt.attention(q, dec["k"], dec["v"], T)
    return time.perf_counter() - t0


def make_pool(procs=None):
    import multiprocessing as mp
    procs = procs or os.cpu_count() or 1
    return mp.get_context("spawn").Pool(procs), procs


def run_step(pool, d, seqs, Hkv):
    """One step = every (sequence, KV head) of `seqs`, spread over the pool. Returns wall seconds."""
    tasks = [(d, b, h) for b in seqs for h in range(Hkv)]
    t0 = time.perf_counter()
    pool.map(head_task, tasks, chunksize=1)
    return time.perf_counter() - t0
