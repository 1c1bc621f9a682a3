#!/usr/bin/env python
"""Benchmark of the exactkv hot path on B200: compressed split-K decode attention.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the config the headline metric is quoted
on): Llama-3.1-8B-shaped decode attention, 32 q / 8 kv heads, head dim 128,
page 16, batch 32 x 4096 context per GPU, synthetic KV (RoPE theta 5e5, 0.04%
zero keys, 0.3% forced raw rows; seeded, see exactkv_b200/synthetic.py). A
step is one decode-attention call over the whole batch: the split kernel plus
the merge kernel. Multi-GPU: one process per GPU, each with its own 32-sequence
batch (batch sharding: no collective on the data path), weak scaling.

value: compressed bytes the attention must read (algorithmic, below) x K
steps x ranks / device time of the K steps (max over ranks), in TB/s.
Algorithmic bytes per call, per K and V cache: 192 B per token row (sign|mantissa
128 + codes 64) + 136 B per page (base 128 + rowmask/rowoff 8) + 256 B per raw row
read; plus q (2 B x 128 per head) and the split partials written (fp32). The
bf16-equivalent bytes are 2 x B x T x Hkv x 256.

Timing: W warm-up steps, then K steps between two barriers + synchronize,
timed with CUDA events on the launching stream; the cache (~425 MB) exceeds the
126 MB L2, and a second pass with the L2 evicted between launches (a 256 MB read) is
reported as a cross-check of the per-launch kernel time. SM clocks and throttle
reasons are sampled through NVML every 5 ms during warm-up and timing.

e2e: the same metric through the public API with host buffers: each step
copies q [B, Hq, 128] and the new token's K and V [B, Hkv, 128] from pinned
host memory into the step's device buffers (kernels.copy_from_host: the SMs
read the pinned memory over PCIe; a copy-engine transfer of the same 384 KB
took 18.5 us plus ~19 us of hand-off to and from the kernels around it),
replays a captured CUDA graph of
the device-length decode step (exactkv_b200.graph: append, page encode at
page boundaries, decode attention, length advance; the raw pools are kept
ahead with one host sync per 8 pages instead of a sync per page), whose merge
kernel writes the output straight into pinned host memory (zero-copy over
PCIe: a separate 256 KB device-to-host copy took ~40 µs on the box); the
context grows by one token per step.

other_configs: BASELINE configs[1] (Qwen 1 x 32768) and Llama 8 x 8192 (the second
shape of configs[2]): per-call µs, compressed TB/s and the bf16 sibling's µs,
with the L2 evicted before each call.

other_configs.paged: the headline batch read through a block table that places
every page at a random page of the cache (exactkv_b200.kernels.attention_paged)
against the contiguous device-length call.

reference_triton_compressed_us_per_call: the reference's own Triton
compressed decode attention on this GPU (same K/V, its own encoder), when the
unmodified reference package is installed in baseline/_ref; a comparison only.

FlashInfer (installed library, comparison only): its TRT-LLM-gen bf16 paged
decode on the same bf16 K/V (16-token pages), timed like our calls.

kv_split: configs[3] (1 x 131072 split by KV sequence over the ranks).

engine: BASELINE configs[4] through exactkv_b200.Engine (CUDA-graphed decode
step) on a random-init Llama-3.1-8B (32 layers, hidden 4096, 32 q / 8 kv heads,
FFN 14336, vocab 128256, bf16 weights ~ N(0, 0.02)). The bf16-cache engine and
the compressed engine each run at the batch that fills the KV budget (free HBM
minus 1.6 GiB, the activations and the synthetic context's scratch), then the
compressed engine at the bf16 batch — the reference's own E2E comparison
(bench/e2e.py of the reference). Per engine, the first --engine-real-prompts
sequences are prefilled from 4096-token uniform-random-id prompts through
Engine.prefill (the model's forward pass) and the rest of the batch from the
synthetic KV through the prefill encoder; then --engine-gen (256) greedy
tokens, all but the first 4 timed with CUDA events; tok/s summed over ranks.
attn_ms_per_step: the 32 layers' decode-attention calls of one step timed
alone on the same caches, and attn_share its fraction of the step.

--impl reference: the reference's own CPU path on the host cores — its PyTorch
codec (exactkv.codec.decode_reference, loaded unmodified from baseline/_ref)
plus its split-K attention restated in torch (the reference has no CPU
attention; oracle/torch_attention.py), every host core as a torch thread — a
bounded sample per step (one sequence of the batch); rank 0 only. Without
baseline/_ref, the numpy oracle port of the same path. cpu_baseline (our arm)
reports the same reference path with the numpy port beside it.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "compressed decode-attn µs & HBM TB/s (% of peak) at 32×4K, 32q/8kv; engine tok/s"
UNIT = "TB/s"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
WORKLOAD = dict(workload="llama3.1-8b decode attention, compressed KV", batch_per_gpu=32, context=4096, q_heads=32,
                kv_heads=8, head_dim=128, page=16, rope_theta=5e5, zero_keys=4e-4, forced_raw_rows=3e-3)
TRAFFIC_RECORD = os.path.join(ROOT, "profiles", "attn_split_compressed__llama_32x4096.traffic.json")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-engine", action="store_true")
    ap.add_argument("--no-kv-split", action="store_true")
    ap.add_argument("--no-configs", action="store_true")
    ap.add_argument("--engine-gen", type=int, default=256, help="tokens generated per engine run")
    ap.add_argument("--engine-real-prompts", type=int, default=16,
                    help="sequences per engine prefilled from random-id prompts through the model")
    ap.add_argument("--num-warps", type=int, default=8)
    ap.add_argument("--only-config", choices=("qwen2.5-7b_1x32768", "llama3.1-8b_8x8192"),
                    help="run only that config's calls (a short command to profile) and exit")
    ap.add_argument("--record-traffic", metavar="NCU_REP",
                    help="write the split kernel's per-launch DRAM bytes from an ncu report and exit")
    ap.add_argument("--traffic-batch", type=int, default=16, help="batch of the --record-traffic capture")
    ap.add_argument("--quick", action="store_true",
                    help="few launches for profiling: no warm loop, L2-flushed pass, e2e or CPU baseline")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def load_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """(dram bytes per launch of the split kernel at this workload, record) from the
    data file `python bench.py --record-traffic <capture>.ncu-rep` writes, or
    (None, None) when no capture of the current source has been recorded."""
    try:
        with open(TRAFFIC_RECORD) as f:
            rec = json.load(f)
    except (OSError, ValueError):
        return None, None
    if rec.get("source_sha256") != kernel_source_digest():
        return None, "stale: recorded for other kernel source"
    return int(rec["traffic_bytes_per_launch"]), rec


def kernel_source_digest():
    """SHA-256 of the attention kernel's sources (a recorded capture is used only
    for the source it measured)."""
    import hashlib
    h = hashlib.sha256()
    for f in ("exk_attention.cu", "exk_device.cuh"):
        with open(os.path.join(ROOT, "exactkv_b200", "csrc", f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def record_traffic(rep, batch, scale):
    """Reads dram__bytes_read.sum + dram__bytes_write.sum of the split kernel's
    launches from an ncu report (ncu -i <rep> --page raw --csv) and writes the
    per-launch mean, scaled by `scale` (the headline batch over the captured
    batch; traffic grows with the pages read), to TRAFFIC_RECORD."""
    import csv
    import io
    import subprocess
    out = subprocess.run(["ncu", "-i", rep, "--page", "raw", "--csv"], capture_output=True, text=True,
                         check=True).stdout
    rows = list(csv.reader(io.StringIO(out)))
    hdr, units = rows[0], rows[1]
    col = {h: i for i, h in enumerate(hdr)}
    mult = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    per_launch = []
    for r in rows[2:]:
        name = r[col["Kernel Name"]]
        # the compressed instantiation: <1, ...> demangled, ILb1 mangled, <true, ...> with bool names
        if "attn_split_kernel" not in name or not any(k in name for k in ("<1,", "ILb1", "<true")):
            continue
        tot = 0.0
        for m in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            tot += float(r[col[m]].replace(",", "")) * mult[units[col[m]]]
        per_launch.append(tot)
    if not per_launch:
        raise SystemExit(f"no compressed split-kernel launch with dram byte counts in {rep}")
    rec = {"traffic_bytes_per_launch": int(statistics.mean(per_launch) * scale),
           "captured_bytes_per_launch": int(statistics.mean(per_launch)), "launches": len(per_launch),
           "captured_batch": batch, "scale": scale, "source_sha256": kernel_source_digest(),
           "report": os.path.basename(rep)}
    with open(TRAFFIC_RECORD, "w") as f:
        json.dump(rec, f, indent=1)
    print(json.dumps(rec))


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML in a thread (read-only)."""

    def __init__(self, dev, interval=0.005):
        self.samples, self.reasons, self.ok = [], set(), False
        self.interval, self._stop = interval, threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(dev)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.max_mhz = None

    def _names(self, bits):
        nv, out = self.nv, []
        table = {"sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
                 "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
                 "sync_boost": getattr(nv, "nvmlClocksEventReasonSyncBoost", 0x10),
                 "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
                 "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
                 "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
                 "applications_clocks_setting": 0x2, "gpu_idle": 0x1}
        for k, v in table.items():
            if bits & v:
                out.append(k)
        return out

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                self.reasons.update(self._names(fn(self.h)))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.interval)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples),
                "window": "warm-up + timed steps"}


# ----------------------------------------------------------------------------- our arm

def algorithmic_bytes(kc, vc, B, Hkv, Hq, T, ns):
    import torch
    npt = -(-T // 16)
    full = T // 16
    total = 0
    raw_rows = 0
    for c in (kc, vc):
        rm = c.rowmask[:, :npt].to(torch.int64)
        pop = torch.zeros_like(rm)
        for bit in range(16):
            pop += (rm >> bit) & 1
        if npt > full:                       # the partial tail page: only rows < T are read
            keep = (1 << (T - full * 16)) - 1
            pop[:, full] = 0
            tail = (rm[:, full] & keep)
            for bit in range(16):
                pop[:, full] += (tail >> bit) & 1
        r = int(pop.sum().item())
        raw_rows += r
        total += B * npt * 16 * Hkv * 192 + B * npt * Hkv * 136 + r * 256
    total += B * Hq * 128 * 2 + B * Hq * ns * (128 + 2) * 4
    return total, raw_rows


def l2_flush(buf):
    """Evicts the L2 (126 MB) by reading a 256 MB buffer: the lines it leaves are
    clean, so no write-back lands in the next timed kernel (a write flush would)."""
    buf.view(-1, 1 << 20).amax(dim=1)


def flashinfer_decode(q, k, v, T):
    """FlashInfer's TRT-LLM-gen bf16 paged decode (B200 kernels shipped prebuilt
    with flashinfer) over the same bf16 K, V viewed as 16-token pages in NHD
    layout; a speed comparison only, never part of the product. Returns a
    zero-argument call, or None with the reason when FlashInfer is unavailable."""
    import torch
    try:
        import flashinfer
        B, TS, Hkv, D = k.shape
        npg = TS // 16
        kp, vp = k.view(B * npg, 16, Hkv, D), v.view(B * npg, 16, Hkv, D)
        tables = torch.arange(B * npg, dtype=torch.int32, device=q.device).view(B, npg)
        lens = torch.full((B,), T, dtype=torch.int32, device=q.device)
        ws = torch.zeros(128 << 20, dtype=torch.uint8, device=q.device)

        def call():
            return flashinfer.decode.trtllm_batch_decode_with_kv_cache(q, (kp, vp), ws, tables, lens, T,
                                                                       bmm1_scale=D ** -0.5, bmm2_scale=1.0,
                                                                       kv_layout="NHD")
        call()
        torch.cuda.synchronize(q.device)
        return call, None
    except Exception as e:  # noqa: BLE001 - reported as unavailable
        return None, f"{type(e).__name__}: {str(e)[:160]}"


def reference_triton_decode(q, k, v, B, T, Hkv):
    """The reference's own compressed decode attention (its Triton kernels, JIT
    for this GPU) on caches built by its own encoder from the same K/V, when the
    unmodified reference package is installed in baseline/_ref (git-ignored).
    A speed comparison on the same box only. Returns a zero-argument call, or
    None with the reason."""
    import torch
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "exactkv")):
        return None, "reference package not installed in baseline/_ref"
    try:
        if ref_dir not in sys.path:
            sys.path.insert(0, ref_dir)
        import exactkv as ref
        rk, rv = ref.CompressedKV(B, T, Hkv, 128, device=q.device), ref.CompressedKV(B, T, Hkv, 128, device=q.device)
        for b in range(B):
            rk.prefill_slot(b, k[b:b + 1, :T])
            rv.prefill_slot(b, v[b:b + 1, :T])

        def call():
            return ref.attention_compressed(q, rk, rv, T)
        call()
        torch.cuda.synchronize(q.device)
        return call, None
    except Exception as e:  # noqa: BLE001 - reported as unavailable
        return None, f"{type(e).__name__}: {str(e)[:160]}"


def run_ours(a, rank, world, local):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))

    import exactkv_b200 as ekv
    from exactkv_b200 import kernels, synthetic

    B, T, Hq, Hkv = a.batch, a.context, 32, 8
    TS = T + max(256, -(-(a.steps + a.warmup + 16) // 16) * 16)
    seed = 1000 + 17 * rank
    k = synthetic.make_kv(B, T, Hkv, seed=seed, theta=5e5, key=True, device=dev)
    v = synthetic.make_kv(B, T, Hkv, seed=seed + 1, theta=5e5, key=False, device=dev)
    q = synthetic.make_q(B, Hq, seed=seed + 2, device=dev)
    kc, vc = ekv.CompressedKV(B, TS, Hkv, 128, device=dev), ekv.CompressedKV(B, TS, Hkv, 128, device=dev)
    for b in range(B):
        kc.prefill_slot(b, k[b:b + 1])
        vc.prefill_slot(b, v[b:b + 1])
    kbf = torch.zeros(B, TS, Hkv, 128, dtype=torch.bfloat16, device=dev)
    vbf = torch.zeros_like(kbf)
    kbf[:, :T] = k
    vbf[:, :T] = v
    del k, v
    kernels.check_status(dev)

    ns, sl = kernels.call_plan(B, Hkv, T, dev, a.num_warps)   # the plan decode_attention uses
    stream = torch.cuda.current_stream(dev)
    nbytes, raw_rows = algorithmic_bytes(kc, vc, B, Hkv, Hq, T, ns)
    bf16_bytes = 2 * B * T * Hkv * 256
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    ws = kernels._workspace(dev, stream.cuda_stream, B * Hq, ns, sl)
    out = torch.empty_like(q)

    def step(ev_a=None, ev_b=None):
        if ev_a is None:
            # the headline: one public-API call (split kernel + merge kernel)
            ekv.decode_attention(q, kc, vc, num_warps=a.num_warps)
            return
        # the dominant kernel's own duration: events around the split launch only
        ev_a.record(stream)
        kernels.attention_split(q, kc, vc, T, ws, 0, ns, num_warps=a.num_warps)
        ev_b.record(stream)
        kernels.merge_partials(ws, B * Hq, out)

    def sibling_step():
        kernels.attention_reference(q, kbf, vbf, T, num_warps=a.num_warps)

    def timed(fn, K, per_launch=False, flush_between=False):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)] \
            if per_launch else None
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(K):
            if flush_between:
                l2_flush(flush)
            if per_launch:
                fn(*evs[i])
            else:
                fn()
        t1.record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        total = t0.elapsed_time(t1)
        launches = [e[0].elapsed_time(e[1]) for e in evs] if per_launch else None
        return total, launches

    clocks = ClockSampler(local)
    with clocks:
        for _ in range(a.warmup):
            step()
        warm_until = time.perf_counter() + (0.0 if a.quick else 0.3)   # long enough for clock samples
        while time.perf_counter() < warm_until:
            step()
        total_ms, _ = timed(step, a.steps)
        # the kernel's own duration: events around every launch, in a second pass
        # (the events add a few us of their own to a step, so not in the headline)
        _, launch_ms = timed(step, a.steps, per_launch=True)
    kernels.check_status(dev)
    t = torch.tensor([total_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / a.steps
    kernel_us = statistics.mean(launch_ms) * 1e3

    kernel_us_flushed = None
    if not a.quick:
        _, flushed = timed(step, min(a.steps, 50), per_launch=True, flush_between=True)
        kernel_us_flushed = round(statistics.median(flushed) * 1e3, 2)
    for _ in range(3):
        sibling_step()
    sib_ms, _ = timed(sibling_step, a.steps)
    sib_us = sib_ms / a.steps * 1e3
    fi_call, fi_why = flashinfer_decode(q, kbf, vbf, T) if not a.quick else (None, "skipped (--quick)")
    fi_us = None
    if fi_call is not None:
        for _ in range(3):
            fi_call()
        fi_ms, _ = timed(fi_call, a.steps)
        fi_us = round(fi_ms / a.steps * 1e3, 2)
    fi_call = None                       # holds views of the bf16 cache, freed before the engine leg
    ref_call, ref_why = reference_triton_decode(q, kbf, vbf, B, T, Hkv) if not a.quick else \
        (None, "skipped (--quick)")
    ref_us = None
    if ref_call is not None:
        for _ in range(3):
            ref_call()
        ref_ms, _ = timed(ref_call, a.steps)
        ref_us = round(ref_ms / a.steps * 1e3, 2)
    ref_call = None                      # its caches are freed before the engine leg

    value = nbytes * a.steps * world / (total_ms * 1e-3) / 1e12
    peak, peak_src = load_peak()
    achieved_gbs = nbytes / (kernel_us * 1e-6) / 1e9      # all algorithmic bytes are this kernel's
    traffic, traffic_rec = profiled_traffic()

    encoder = None if a.quick else time_encoder(kbf, B, T, Hkv, dev)

    configs = None
    if not (a.no_configs or a.quick):
        configs = run_configs(a, dev, world)
        configs["paged"] = time_paged(q, kc, vc, B, T, dev, a.steps)

    kv_split = None
    if not (a.no_kv_split or a.quick):
        kv_split = run_kv_split(a, dev, rank, world)

    engine = None
    if not (a.no_engine or a.quick):
        del kbf, vbf
        engine = run_engine(a, dev, world)

    e2e = None
    if not (a.no_e2e or a.quick):
        e2e = run_e2e(a, kc, vc, B, Hq, Hkv, T, dev, world, raw_rows, ns)

    cpu = None
    if rank == 0 and world == 1 and not (a.no_cpu_baseline or a.quick):
        cpu = cpu_baselines(T, Hkv, Hq)
    rec = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8 codes -> bf16 mma, fp32 softmax", "data": "synthetic",
        "config": dict(WORKLOAD, global_batch=B * world, parallelism=f"batch-shard x{world} (independent replicas)",
                       l2="cache 425 MB > 126 MB L2; flushed pass reported separately", splits=ns, split_len=sl,
                       consumer_warps=a.num_warps),
        "attn_us_per_call": round(ms_per_step * 1e3, 2),
        "kernel_us": round(kernel_us, 2),
        "kernel_us_l2_flushed": kernel_us_flushed,
        "kernel_timing": "CUDA events around each split-kernel launch, second pass of K steps (the headline pass "
                         "times whole decode_attention calls without per-launch events)",
        "compressed_bytes_per_call": nbytes, "raw_rows": raw_rows,
        "raw_row_fraction": round(raw_rows / (2 * B * T * Hkv), 5),
        "bits_per_value": round(8 * nbytes / (2 * B * T * Hkv * 128), 3),
        "bf16_equiv_tbs": round(bf16_bytes * a.steps * world / (total_ms * 1e-3) / 1e12, 4),
        "frac_of_nominal_8tbs": round(value / world / (NOMINAL_HBM_GBS / 1e3), 4),
        "bf16_sibling_us_per_call": round(sib_us, 2),
        "speedup_vs_bf16_sibling": round(sib_us / (ms_per_step * 1e3), 3),
        "reference_triton_compressed_us_per_call": ref_us if ref_us is not None else ref_why,
        "speedup_vs_reference_triton": round(ref_us / (ms_per_step * 1e3), 3) if ref_us is not None else None,
        "flashinfer_trtllm_bf16_us_per_call": fi_us if fi_us is not None else fi_why,
        "speedup_vs_flashinfer_bf16": round(fi_us / (ms_per_step * 1e3), 3) if fi_us is not None else None,
        "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved_gbs / peak, 4), "peak_source": f"{peak_src} hbm_gbs (copy, read+write)",
                     "traffic": traffic, "kernel": "exk::attn_split_kernel<compressed>",
                     "traffic_source": traffic_rec if not isinstance(traffic_rec, dict) else
                     f"ncu capture {traffic_rec['report']} at batch {traffic_rec['captured_batch']}, "
                     f"x{traffic_rec['scale']} to the headline batch (recorded for this kernel source)"},
        "gpu_launches": 2 * a.steps,
        "encoder": encoder,
        "clocks": clocks.summary(),
        "e2e": e2e,
        "engine": engine,
        "other_configs": configs,
        "kv_split": kv_split,
        "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def time_paged(q, kc, vc, B, T, dev, reps):
    """The headline batch read through a block table that scatters every
    sequence's pages over the whole cache (a random permutation of its pages),
    against the same device-length call on the contiguous layout: what paging
    costs the attention."""
    import torch

    from exactkv_b200 import kernels
    npg = T // 16
    pool_pages = kc.B * kc.TS // 16
    g = torch.Generator().manual_seed(5)
    perm = torch.randperm(pool_pages, generator=g)[: B * npg].to(torch.int32)
    table = perm.view(B, npg).to(dev)
    lens = torch.full((B,), T, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return round(e0.elapsed_time(e1) / reps * 1e3, 2)

    paged = timed(lambda: kernels.attention_paged(q, kc, vc, table, lens, out=out))
    # the contiguous device-length call with the same plan (T_cap = T)
    contiguous = timed(lambda: kernels.attention_compressed_devlen(q, kc, vc, lens, 0, out=out))
    kernels.check_status(dev)
    return {"paged_us_per_call": paged, "contiguous_devlen_us_per_call": contiguous,
            "what": f"{B} x {T} through a block table over a {pool_pages}-page pool (pages randomly placed) "
                    "vs the contiguous device-length call; back-to-back calls, cache > L2"}


# GPU cycles (~0.5 ms) of a spin kernel enqueued before a single timed call, so
# that the host has enqueued the whole call before its start event runs: the
# events then time the device work and not the host's launch overhead.
HOST_AHEAD_CYCLES = 1_000_000


def reference_encode_us(src, st, B, T, Hkv, dev, reps):
    """The reference's own encode_pages (Triton) over the same source, when the
    reference package is installed in baseline/_ref (see reference_triton_decode);
    else the reason it is not timed."""
    import torch
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "exactkv")):
        return "reference package not installed in baseline/_ref"
    try:
        if ref_dir not in sys.path:
            sys.path.insert(0, ref_dir)
        import exactkv as ref
        c = ref.CompressedKV(B, T, Hkv, 128, device=dev, reserve=0.05)
        times = []
        for i in range(reps + 2):
            c.cnt.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda._sleep(HOST_AHEAD_CYCLES)
            e0.record()
            ref.encode_pages(src, st, c._buf(), 0, 0, B, T // 16)
            e1.record()
            torch.cuda.synchronize(dev)
            if i >= 2:
                times.append(e0.elapsed_time(e1) * 1e3)
        return round(statistics.median(times), 2)
    except Exception as e:  # noqa: BLE001 - reported as unavailable
        return f"{type(e).__name__}: {str(e)[:160]}"


def time_encoder(kbf, B, T, Hkv, dev, reps=5):
    """The page encoder over the whole batch's keys in one encode_pages call (a
    prefill of B sequences): bf16 bytes read and compressed bytes written per us."""
    import torch

    import exactkv_b200 as ekv
    from exactkv_b200 import kernels
    c = ekv.CompressedKV(B, T, Hkv, 128, device=dev, reserve=0.05)
    src = kbf[:, :T]
    st = (src.stride(0), 16 * src.stride(1), src.stride(1), src.stride(2))
    times = []
    for i in range(reps + 2):
        c.cnt.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(HOST_AHEAD_CYCLES)
        e0.record()
        kernels.encode_pages(src, st, c.encoder_buffers(), 0, 0, B, T // 16)
        e1.record()
        torch.cuda.synchronize(dev)
        if i >= 2:
            times.append(e0.elapsed_time(e1) * 1e3)
    n = int(c.cnt.item())
    us = statistics.median(times)
    rows = B * T * Hkv
    written = rows * 192 + (rows // 16) * 136 + n * 256
    ref_us = reference_encode_us(src, st, B, T, Hkv, dev, reps)
    return {"us": round(us, 2), "bf16_read_gbs": round(rows * 256 / us / 1e3, 1),
            "compressed_written_gbs": round(written / us / 1e3, 1), "raw_rows": n,
            "reference_triton_encode_pages_us": ref_us,
            "what": f"encode_pages over {B} x {T} tokens x {Hkv} heads of keys (4 launches: encode, chunk sums, "
                    "chunk scan, slot placement + raw copy; each call enqueued behind a spin kernel so the events "
                    "time the device work, the reference's call likewise)"}


def run_e2e(a, kc, vc, B, Hq, Hkv, T0, dev, world, raw_rows0, ns0):
    """Public-API decode steps with host buffers (see module docstring): each step
    copies its inputs from pinned host memory, replays the captured device-length
    step (exactkv_b200.graph) and copies the output back to pinned memory."""
    import torch
    import torch.distributed as dist

    import exactkv_b200 as ekv
    from exactkv_b200 import kernels
    from exactkv_b200.graph import DeviceLength, GraphedStep

    K = a.steps
    g = torch.Generator().manual_seed(77)
    n_all = K + 2
    nq, nk = B * Hq * 128, B * Hkv * 128
    # one pinned row per step: q, the new K token, the new V token (one H2D copy per step)
    inp_h = torch.randn(n_all, nq + 2 * nk, generator=g).to(torch.bfloat16).pin_memory()
    # the step's output: pinned host memory that the merge kernel writes directly
    # over PCIe (the device -> host read of the result, with no separate copy)
    out = torch.empty(B, Hq, 128, dtype=torch.bfloat16).pin_memory()
    stream = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)
    length = DeviceLength([kc, vc])
    inp = torch.empty(nq + 2 * nk, dtype=torch.bfloat16, device=dev)
    q_in = inp[:nq].view(B, Hq, 128)
    k_in = inp[nq:nq + nk].view(B, Hkv, 128)
    v_in = inp[nq + nk:].view(B, Hkv, 128)

    def body():
        main = torch.cuda.current_stream(dev)
        side.wait_stream(main)
        with torch.cuda.stream(side):             # the two caches' appends overlap
            vc.append_dev(v_in, length.t)
        kc.append_dev(k_in, length.t)
        main.wait_stream(side)
        kernels.attention_compressed_devlen(q_in, kc, vc, length.t, 1, out=out, advance=1)

    gs = GraphedStep(body, length, check_pages=8)
    ns_cap, _ = kernels.devlen_plan(B, Hkv, kc.TS, length.t, dev)

    def one(i):
        kernels.copy_from_host(inp, inp_h[i])     # the SMs read the step's inputs over PCIe
        gs.step()                                 # ends with the output written to host memory

    for i in range(2):                            # untimed: the first step captures the graph
        one(K + i)
    nbytes_total = 0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        one(i)
        T = kc.T
        npt = -(-T // 16)
        # as algorithmic_bytes(): full-page rows, page metadata, the prefill's raw rows and the
        # raw tail rows (pages encoded during these steps add a few more raw rows, not counted)
        nbytes_total += (2 * (B * npt * 16 * Hkv * 192 + B * npt * Hkv * 136)
                         + (raw_rows0 + 2 * B * Hkv * (T % 16)) * 256 + B * Hq * 256 + B * Hq * ns_cap * 520)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t0
    ms = e0.elapsed_time(e1)
    gs.close()
    kernels.check_status(dev)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    h2d = (B * Hq + 2 * B * Hkv) * 128 * 2
    d2h = B * Hq * 128 * 2
    return {"value": round(nbytes_total * world / (ms * 1e-3) / 1e12, 4), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms / K, 4),
            "wall_ms_per_step": round(wall / K * 1e3, 4), "graph_captures": gs.captures,
            "what": "per step: H2D q + new K/V token from pinned memory (read over PCIe by a copy kernel, "
                    "exk_copy_from_host), a replayed CUDA graph of the "
                    "device-length step (append + page encode at boundaries, decode attention, length advance; "
                    "pools kept ahead with one sync per 8 pages) whose merge kernel writes the output straight "
                    "into pinned host memory over PCIe (the D2H bytes); context grows from 4096"}


CONFIGS = {"qwen2.5-7b_1x32768": (1, 32768, 28, 4, 1e6), "llama3.1-8b_8x8192": (8, 8192, 32, 8, 5e5)}


def run_one_config(a, dev):
    """--only-config NAME: that config's compressed call (split + merge) a.steps
    times after a.warmup, nothing else (a short command for ncu captures)."""
    import torch

    import exactkv_b200 as ekv
    from exactkv_b200 import kernels, synthetic
    B, T, Hq, Hkv, theta = CONFIGS[a.only_config]
    k = synthetic.make_kv(B, T, Hkv, seed=700, theta=theta, key=True, device=dev)
    v = synthetic.make_kv(B, T, Hkv, seed=701, theta=theta, key=False, device=dev)
    q = synthetic.make_q(B, Hq, seed=702, device=dev)
    kc, vc = ekv.CompressedKV(B, T, Hkv, 128, device=dev), ekv.CompressedKV(B, T, Hkv, 128, device=dev)
    for b in range(B):
        kc.prefill_slot(b, k[b:b + 1])
        vc.prefill_slot(b, v[b:b + 1])
    del k, v
    for _ in range(a.warmup):
        ekv.decode_attention(q, kc, vc, num_warps=a.num_warps)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(a.steps):
        ekv.decode_attention(q, kc, vc, num_warps=a.num_warps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    kernels.check_status(dev)
    print(json.dumps({"config": a.only_config, "us_per_call": round(e0.elapsed_time(e1) * 1e3 / a.steps, 2),
                      "note": "back-to-back calls (cache in L2 when it fits); for profiling"}))


def run_configs(a, dev, world, reps=30):
    """BASELINE configs[1] (Qwen2.5-7B 1 x 32768, 28 q / 4 kv, RoPE theta 1e6) and
    the second shape of configs[2] (Llama 8 x 8192, 32 q / 8 kv): one
    decode-attention call through the public API, compressed and on the bf16
    sibling, each call's device time with a 256 MB L2 flush before it (the Qwen
    cache fits in L2); median over reps, this rank's replica."""
    import torch
    import torch.distributed as dist

    import exactkv_b200 as ekv
    from exactkv_b200 import kernels, synthetic

    peak, _ = load_peak()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    out = {}
    for name, (B, T, Hq, Hkv, theta) in CONFIGS.items():
        k = synthetic.make_kv(B, T, Hkv, seed=700, theta=theta, key=True, device=dev)
        v = synthetic.make_kv(B, T, Hkv, seed=701, theta=theta, key=False, device=dev)
        q = synthetic.make_q(B, Hq, seed=702, device=dev)
        kc, vc = ekv.CompressedKV(B, T, Hkv, 128, device=dev), ekv.CompressedKV(B, T, Hkv, 128, device=dev)
        for b in range(B):
            kc.prefill_slot(b, k[b:b + 1])
            vc.prefill_slot(b, v[b:b + 1])
        ns, _ = kernels.call_plan(B, Hkv, T, dev, a.num_warps)
        nbytes, raw_rows = algorithmic_bytes(kc, vc, B, Hkv, Hq, T, ns)

        def per_call(fn):
            for _ in range(3):
                fn()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize(dev)
            for e0, e1 in ev:
                l2_flush(flush)
                e0.record(stream)
                fn()
                e1.record(stream)
            torch.cuda.synchronize(dev)
            return statistics.median(e0.elapsed_time(e1) for e0, e1 in ev) * 1e3

        us_c = per_call(lambda: ekv.decode_attention(q, kc, vc, num_warps=a.num_warps))
        us_r = per_call(lambda: kernels.attention_reference(q, k, v, T, num_warps=a.num_warps))
        fi_call, fi_why = flashinfer_decode(q, k, v, T)
        us_f = per_call(fi_call) if fi_call is not None else None
        fi_call = None
        rf_call, rf_why = reference_triton_decode(q, k, v, B, T, Hkv)
        us_rf = per_call(rf_call) if rf_call is not None else None
        rf_call = None
        kernels.check_status(dev)
        tbs = nbytes / (us_c * 1e-6) / 1e12
        out[name] = {"batch": B, "context": T, "q_heads": Hq, "kv_heads": Hkv, "splits": ns,
                     "us_per_call": round(us_c, 2), "compressed_tbs": round(tbs, 3),
                     "frac_of_measured_peak": round(tbs * 1e3 / peak, 4),
                     "bf16_equiv_tbs": round(2 * B * T * Hkv * 256 / (us_c * 1e-6) / 1e12, 3),
                     "bf16_sibling_us_per_call": round(us_r, 2), "speedup_vs_bf16_sibling": round(us_r / us_c, 3),
                     "flashinfer_trtllm_bf16_us_per_call": round(us_f, 2) if us_f is not None else fi_why,
                     "reference_triton_compressed_us_per_call": round(us_rf, 2) if us_rf is not None else rf_why,
                     "speedup_vs_flashinfer_bf16": round(us_f / us_c, 3) if us_f is not None else None,
                     "raw_row_fraction": round(raw_rows / (2 * B * T * Hkv), 5)}
        del k, v, q, kc, vc
        torch.cuda.empty_cache()
    out["timing"] = ("CUDA events around each call (ours: split + merge), L2 evicted before each by reading a "
                     "256 MB buffer, median")
    return out


def run_kv_split(a, dev, rank, world, T=131072, Hq=32, Hkv=8, reps=20):
    """one sequence of 131072 tokens (2% forced raw rows) split
    over the ranks by KV sequence; per call: the split kernel, the rank's group
    partial (one per row) written into symmetric memory, then the peer merge
    reading every rank's group partial over NVLink
    (exactkv_b200.parallel.PeerExchange); the NCCL all-gather variant is timed
    beside it."""
    import torch
    import torch.distributed as dist

    import exactkv_b200 as ekv
    from exactkv_b200 import kernels, parallel, synthetic

    plan = parallel.KVSplitPlan.make(1, Hkv, T, world, dev)
    t0, t1 = plan.tokens(rank)
    n = t1 - t0
    TS = max(16, -(-n // 16) * 16)
    caches = []
    for j, key in enumerate((True, False)):
        x = synthetic.make_kv(1, T, Hkv, seed=500 + j, theta=1e6, key=key, raw_frac=0.02, device=dev)[:, t0:t1]
        c = ekv.CompressedKV(1, TS, Hkv, 128, device=dev, reserve=0.03)
        if n:
            c.prefill_slot(0, x.contiguous())
        caches.append(c)
        del x
    q = synthetic.make_q(1, Hq, seed=502, device=dev)
    kc, vc = caches

    out = torch.empty_like(q)
    ex, peer_err = None, None
    if world > 1:
        try:
            ex = parallel.PeerExchange(plan, Hq)
        except Exception as e:  # noqa: BLE001 - symmetric memory unavailable: NCCL numbers only
            peer_err = f"{type(e).__name__}: {str(e)[:160]}"
    peer = world == 1 or ex is not None

    def call_peer():
        if ex is not None:
            return ex.attention(q, kc, vc, out)
        local = parallel.local_partials(q, kc, vc, plan, 0)
        return parallel.merge_gathered(local.view(1, -1), plan, out)

    def call_nccl():
        return parallel.attention_kv_split(q, kc, vc, plan, rank, out=out)

    stream = torch.cuda.current_stream(dev)

    def timed(call):
        for _ in range(3):
            call()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            call()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) / reps * 1e3], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    us = timed(call_peer) if peer else None
    us_nccl = timed(call_nccl) if world > 1 else None

    # the peer path again with an event between the split kernel and the merge
    # (which includes the wait for the peers): this rank's average per phase
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(reps if peer else 0)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    for e in ev:
        e[0].record(stream)
        if ex is not None:
            ex.split(q, kc, vc)
            e[1].record(stream)
            ex.merge(out)
        else:
            local = parallel.local_partials(q, kc, vc, plan, 0)
            e[1].record(stream)
            parallel.merge_gathered(local.view(1, -1), plan, out)
        e[2].record(stream)
    torch.cuda.synchronize(dev)
    phases = {name: round(sum(e[i].elapsed_time(e[i + 1]) for e in ev) / reps * 1e3, 2)
              for i, name in enumerate(("split", "merge"))} if peer else None
    if ex is not None:
        dist.barrier()
        ex.close()
    kernels.check_status(dev)
    nbytes = sum(c.nbytes() for c in caches)        # this rank's compressed cache (an upper bound of what it reads)
    return {"us_per_call": round(us if us is not None else us_nccl, 2),
            "nccl_all_gather_us_per_call": None if us_nccl is None else round(us_nccl, 2),
            "peer_merge_unavailable": peer_err, "phases_us_rank0": phases, "context": T, "ranks": world, "splits": plan.ns,
            "split_len": plan.split_len, "tokens_per_rank": n, "compressed_mb_per_rank": round(nbytes / 1e6, 1),
            "what": "1 x 131072 decode attention (32 q / 8 kv, 2% raw rows) split by KV sequence over the ranks: "
                    "split kernel, the rank's splits merged to one group partial per row in its symmetric-memory "
                    "block, then the peer merge reading every rank's group partial over NVLink in rank order (max "
                    "over ranks); nccl_all_gather_us_per_call: the same with NCCL all_gather_into_tensor of the "
                    "group partials and the gathered merge"}


def _engine_model(dev):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=5e5,
                      max_position_embeddings=8192, rms_norm_eps=1e-5, initializer_range=0.02,
                      tie_word_embeddings=False)
    torch.manual_seed(1234)
    with torch.device(dev):
        return LlamaForCausalLM._from_config(cfg, dtype=torch.bfloat16).eval()


def _engine_run(model, backend, B, context, gen, warm, real, dev, world):
    """One engine at batch B: `real` sequences prefilled from uniform-random-id
    prompts of `context` tokens through Engine.prefill (the model's forward pass),
    the rest from the synthetic KV through the prefill encoder; then `gen` greedy
    tokens, the last gen - warm timed with CUDA events. Also the 32 layers'
    decode-attention calls of one step, timed alone at the end."""
    import torch
    import torch.distributed as dist

    import exactkv_b200 as ekv
    from exactkv_b200 import kernels, synthetic
    eng = ekv.Engine(model, B, context + gen + 16, backend=backend)
    g = torch.Generator(device=dev).manual_seed(77)
    ids = torch.randint(0, model.config.vocab_size, (real, context), generator=g, device=dev)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    tok = torch.empty(B, dtype=torch.long, device=dev)
    tok[:real] = eng.prefill(ids)
    torch.cuda.synchronize(dev)
    prefill_s = time.perf_counter() - t0
    chunk = 16
    for b0 in range(real, B, chunk):
        n = min(chunk, B - b0)
        k = synthetic.make_kv(n, context, 8, seed=900 + b0, theta=5e5, key=True, device=dev)
        v = synthetic.make_kv(n, context, 8, seed=901 + b0, theta=5e5, key=False, device=dev)
        for kc, vc in eng.kv:
            for j in range(n):
                kc.prefill_slot(b0 + j, k[j:j + 1])
                vc.prefill_slot(b0 + j, v[j:j + 1])
        del k, v
    tok[real:] = torch.randint(0, model.config.vocab_size, (B - real,), generator=g, device=dev)
    eng.sync_length()
    for _ in range(warm):
        tok = eng.step_greedy(tok)
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(gen - warm):
        tok = eng.step_greedy(tok)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    steps = gen - warm
    # the attention share of a step: the 32 layers' decode-attention calls alone,
    # on the same caches at the final length (after the graph's last step)
    q = synthetic.make_q(B, 32, seed=5, device=dev)
    length = torch.full((1,), eng.T - 1, dtype=torch.int32, device=dev)
    def attn_calls():
        for kc, vc in eng.kv:
            if eng.compressed:
                kernels.attention_compressed_devlen(q, kc, vc, length, 1)
            else:
                kernels.attention_reference_devlen(q, kc.buf, vc.buf, length, 1)
    attn_calls()
    torch.cuda.synchronize(dev)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(5):
        attn_calls()
    a1.record(stream)
    torch.cuda.synchronize(dev)
    attn_ms = a0.elapsed_time(a1) / 5
    res = {"backend": backend, "batch_per_gpu": int(B), "tok_s": round(B * steps * world / (ms * 1e-3), 1),
           "ms_per_step": round(ms / steps, 3), "attn_ms_per_step": round(attn_ms, 3),
           "attn_share": round(attn_ms / (ms / steps), 3), "prefill_s_real_prompts": round(prefill_s, 2),
           "pool_grows": int(eng.grows), "graph_captures": int(eng.captures)}
    eng.close()
    del eng
    return res


def run_engine(a, dev, world, context=4096, warm=4):
    """BASELINE configs[4] on each GPU: the bf16-cache engine and the compressed
    engine, each at the batch that fills the KV budget (free HBM minus 1.6 GiB and
    the activations), then the compressed engine at the bf16 batch (the
    reference's own E2E comparison, bench/e2e.py:52-90 of the reference)."""
    import gc
    import torch

    import exactkv_b200 as ekv

    gc.collect()
    torch.cuda.empty_cache()
    model = _engine_model(dev)
    gen = a.engine_gen
    TM = context + gen + 16
    per_seq = {}
    for be in ("bf16", "exactkv"):
        e1, e2 = ekv.Engine(model, 1, TM, backend=be), ekv.Engine(model, 2, TM, backend=be)
        per_seq[be] = e2.kv_bytes() - e1.kv_bytes()
        del e1, e2
        torch.cuda.empty_cache()
    chunk = 16
    scratch = 2 * chunk * context * 8 * 128 * 2 * 2           # the synthetic K/V chunk (and its copy)
    budget = torch.cuda.mem_get_info(dev)[0] - int(1.6 * 2 ** 30) - scratch - (3 << 30)   # activations, graph
    rows = []
    for be in ("bf16", "exactkv"):
        B = max(1, min(2048, budget // per_seq[be]))
        rows.append(_engine_run(model, be, B, context, gen, warm, min(a.engine_real_prompts, B), dev, world))
        gc.collect()
        torch.cuda.empty_cache()
    same = _engine_run(model, "exactkv", rows[0]["batch_per_gpu"], context, gen, warm,
                       min(a.engine_real_prompts, rows[0]["batch_per_gpu"]), dev, world)
    res = {"tok_s_exactkv": rows[1]["tok_s"], "tok_s_bf16": rows[0]["tok_s"],
           "throughput_ratio": round(rows[1]["tok_s"] / rows[0]["tok_s"], 3),
           "batch_exactkv": rows[1]["batch_per_gpu"], "batch_bf16": rows[0]["batch_per_gpu"],
           "step_time_ratio_same_batch": round(rows[0]["ms_per_step"] / same["ms_per_step"], 3),
           "attn_share_exactkv": rows[1]["attn_share"], "attn_share_bf16": rows[0]["attn_share"],
           "kv_mib_per_seq": {be: round(v / 2 ** 20, 1) for be, v in per_seq.items()},
           "kv_budget_gib": round(budget / 2 ** 30, 2), "context": context, "generated": gen,
           "timed_steps": gen - warm, "rows": rows + [same],
           "model": "random-init Llama-3.1-8B (bf16 weights ~ N(0, 0.02))",
           "what": f"greedy decode through exactkv_b200.Engine (HF modules, CUDA-graphed step). Per engine: "
                   f"{a.engine_real_prompts} sequences prefilled from {context}-token uniform-random-id prompts "
                   f"through Engine.prefill (model forward), the rest of the batch from the synthetic KV "
                   f"through the prefill encoder; {gen} generated tokens, the last {gen - warm} timed"}
    del model
    gc.collect()
    torch.cuda.empty_cache()
    return res


# ----------------------------------------------------------------------------- CPU (oracle) legs

def _cpu_setup(T, Hkv, Hq, nseq):
    from oracle import cpu_baseline
    from oracle.synth import synth_kv, synth_q
    d, per_seq = cpu_baseline.build_sample(nseq, T, Hkv, Hq, 5e5, 4242, synth_kv, synth_q)
    pool, procs = cpu_baseline.make_pool()
    return cpu_baseline, d, per_seq, pool, procs


def cpu_sample(T, Hkv, Hq, seconds=10.0, nseq=4):
    """Oracle decode + attention timed on a bounded sample: an `nseq`-sequence slice of
    the batch (all 8 KV heads, K and V), repeated for about `seconds`, over every host core."""
    cb, d, per_seq, pool, procs = _cpu_setup(T, Hkv, Hq, nseq)
    seqs = list(range(nseq))
    try:
        cb.run_step(pool, d, seqs[:1], Hkv)             # warm the workers
        secs = []
        t_end = time.perf_counter() + seconds
        while time.perf_counter() < t_end or len(secs) < 2:
            secs.append(cb.run_step(pool, d, seqs, Hkv))
    finally:
        pool.close()
        pool.join()
    s = sum(secs)
    return {"value": round(per_seq * nseq * len(secs) / s / 1e12, 8), "unit": UNIT, "cores": procs, "kind": "port",
            "sample": f"{len(secs)} passes over {nseq} of the 32 sequences (4096 tokens x 8 KV heads, K and V): "
                      f"numpy oracle decode + split-K attention, {s / len(secs) / nseq * 1e3:.1f} ms per sequence "
                      f"with {procs} processes"}


def _reference_codec():
    """The reference's own codec module (exactkv/codec.py, plain PyTorch), loaded by
    file path from the unmodified install in baseline/_ref; None when absent. Only
    codec.py is loaded (it imports torch alone), not the package with its Triton
    kernels."""
    import importlib.util
    path = os.path.join(ROOT, "baseline", "_ref", "exactkv", "codec.py")
    if not os.path.isfile(path):
        return None
    spec = importlib.util.spec_from_file_location("exactkv_reference_codec", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _reference_cpu_setup(T, Hkv, Hq):
    """One sequence (T tokens x Hkv heads, K and V) encoded by the reference's
    encode_reference on the CPU; returns (codec, (ck, cv, q), compressed bytes)."""
    import torch

    from exactkv_b200 import synthetic
    codec = _reference_codec()
    if codec is None:
        return None
    TS = -(-T // 16) * 16
    k = synthetic.make_kv(1, TS, Hkv, seed=4242, theta=5e5, key=True, device="cpu")
    v = synthetic.make_kv(1, TS, Hkv, seed=4243, theta=5e5, key=False, device="cpu")
    q = synthetic.make_q(1, Hq, seed=4244, device="cpu")
    ck, cv = codec.encode_reference(k), codec.encode_reference(v)
    nbytes = 0
    for c in (ck, cv):
        raw_rows = int(c["raw"].shape[0])
        nbytes += TS * Hkv * 192 + c["base"].numel() + 8 * c["rowmask"].numel() + raw_rows * 256
    torch.set_num_threads(os.cpu_count() or 1)
    return codec, (ck, cv, q), nbytes


def _reference_cpu_step(codec, data, T):
    """The reference's PyTorch decode_reference of K and V, then the split-K
    attention restated in torch (oracle/torch_attention.py)."""
    from oracle import torch_attention
    ck, cv, q = data
    return torch_attention.attention(q, codec.decode_reference(ck), codec.decode_reference(cv), T)


def cpu_reference_sample(T, Hkv, Hq, seconds=10.0):
    """The reference's own CPU codec (decode_reference, unmodified) + the torch
    attention restatement, on one sequence of the batch, repeated for about
    `seconds` with every host core as a torch thread. None without baseline/_ref."""
    import torch
    setup = _reference_cpu_setup(T, Hkv, Hq)
    if setup is None:
        return None
    codec, data, nbytes = setup
    _reference_cpu_step(codec, data, T)                  # warm
    secs = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(secs) < 2:
        t0 = time.perf_counter()
        _reference_cpu_step(codec, data, T)
        secs.append(time.perf_counter() - t0)
    s = sum(secs)
    threads = torch.get_num_threads()
    return {"value": round(nbytes * len(secs) / s / 1e12, 8), "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"{len(secs)} passes over 1 of the 32 sequences ({T} tokens x {Hkv} KV heads, K and V): "
                      f"the reference's exactkv.codec.decode_reference (PyTorch, unmodified, from baseline/_ref) "
                      f"+ its split-K attention restated in torch (oracle/torch_attention.py), "
                      f"{s / len(secs) * 1e3:.1f} ms per sequence with {threads} torch threads"}


def cpu_baselines(T, Hkv, Hq):
    """cpu_baseline: the reference's own CPU codec path when baseline/_ref is
    installed (kind "reference"), with the numpy port beside it; else the port."""
    ref = cpu_reference_sample(T, Hkv, Hq)
    port = cpu_sample(T, Hkv, Hq)
    if ref is None:
        return port
    ref["port"] = port
    return ref


def run_reference(a, rank, world):
    if rank != 0:
        return
    T, Hkv, Hq = a.context, 8, 32
    setup = _reference_cpu_setup(T, Hkv, Hq)
    if setup is not None:
        import torch
        codec, data, per_seq = setup
        kind, procs = "reference", torch.get_num_threads()
        for _ in range(max(1, a.warmup)):
            _reference_cpu_step(codec, data, T)
        t0 = time.perf_counter()
        for _ in range(a.steps):
            _reference_cpu_step(codec, data, T)
        total = time.perf_counter() - t0
        sample = (f"each step: 1 sequence of the 32 x 4096 batch (8 KV heads, K and V): the reference's own "
                  f"exactkv.codec.decode_reference (PyTorch, unmodified, from baseline/_ref) + its split-K "
                  f"attention restated in torch (oracle/torch_attention.py), {procs} torch threads")
    else:
        cb, d, per_seq, pool, procs = _cpu_setup(T, Hkv, Hq, 1)
        kind = "port"
        try:
            for _ in range(max(1, a.warmup)):
                cb.run_step(pool, d, [0], Hkv)
            t0 = time.perf_counter()
            for _ in range(a.steps):
                cb.run_step(pool, d, [0], Hkv)
            total = time.perf_counter() - t0
        finally:
            pool.close()
            pool.join()
        sample = (f"each step: 1 sequence of the 32 x 4096 batch (8 KV heads, K and V), numpy oracle restatement "
                  f"of the reference codec decode + split-K attention over {procs} processes (baseline/_ref absent)")
    value = per_seq * a.steps / total / 1e12
    rec = {"metric": METRIC, "value": round(value, 8), "unit": UNIT, "n_gpus": world, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": round(total / a.steps * 1e3, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "u8 codes -> fp32", "data": "synthetic",
           "config": dict(WORKLOAD, global_batch=32, parallelism="host CPU"), "impl": "reference",
           "cpu_baseline": {"value": round(value, 8), "unit": UNIT, "cores": procs, "kind": kind,
                            "sample": sample},
           "e2e": {"value": round(value, 8), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(rec), flush=True)


def main():
    a = parse_args()
    if a.record_traffic:
        record_traffic(a.record_traffic, a.traffic_batch, 32 / a.traffic_batch)
        return 0
    rank, world, local = dist_env()
    if a.only_config:
        import torch
        torch.cuda.set_device(local)
        run_one_config(a, torch.device("cuda", local))
        return 0
    if a.impl == "reference":
        run_reference(a, rank, world)
        return 0
    run_ours(a, rank, world, local)
    return 0


if __name__ == "__main__":
    sys.exit(main())
