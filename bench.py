#!/usr/bin/env python3
"""Benchmark of the fused token-sampling path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (per GPU, weak scaling): the bandwidth configuration, 65536 rows x
3072 f32 logits ~ N(0, 1), top_k 50, top_p 1.0, temperature 1.0, no penalty;
one step = one fused sampling launch over the 65536 rows.  The logits (805 MB)
exceed the 126 MB L2, so consecutive steps stream them from HBM.  Launches go
through a prepared q3s_batch (one C call per step), so the host keeps the
stream full and the per-step CUDA events time the kernel, not the host.

`value` is whole-job rows/s with the inputs resident in HBM.  `e2e` is the same
metric through the C ABI with host buffers: each step copies the logits and
the per-row seeds from pinned host memory and the tokens and status bytes
back.  `results.hetero_decode_step` is the heterogeneous full decode step
(4096 streams x 16 rows in total, whole streams sharded over the N GPUs, L2
flushed between launches), checked against the oracle on every rank.
`--impl reference` times the CPU restatement of the reference sampler
(src/talker/sampling.rs, with glibc expf as Rust's f32::exp uses on Linux) on
the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qwen3tts-rs_b200"))

METRIC = "sampled rows/sec at vocab 3072, B=1024 and 65536 (1/2/4/8 B200); % HBM roofline"
ROWS = 65536
VOCAB = 3072
TOP_K = 50
HETERO_STREAMS = 4096
# Algorithmic bytes per row of the bandwidth workload: 3072 f32 logits,
# the Philox seed and subsequence (8 + 8), the token (4) and the status (1).
BYTES_PER_ROW = 4 * VOCAB + 16 + 4 + 1
# DRAM bytes (read + write) per 65,536-row launch of the sampling kernel: an
# ncu capture of a 16,384-row launch (dram__bytes_read.sum +
# dram__bytes_write.sum = 201.810176 + 6.509312 MB) scaled by the rows, since
# every row is read from HBM exactly once.
NCU_TRAFFIC_PER_LAUNCH = 208.319488e6 * 4
FALLBACK_HBM_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20


def measured_peak_gbs():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """Samples the SM clock and throttle reasons of the given GPUs (NVML, one
    thread in one process) while running."""

    REASONS = {
        "hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
        "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, bus_ids, period_s: float = 0.02):
        self.samples = {i: [] for i in range(len(bus_ids))}
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = []
        self.period = period_s
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            for k, bus in enumerate(bus_ids):
                try:
                    h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
                except Exception:
                    h = pynvml.nvmlDeviceGetHandleByIndex(k)
                self._h.append(h)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h[0], pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = []
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            for i, h in enumerate(self._h):
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples[i].append((mhz, reasons))
                except Exception:
                    pass
            time.sleep(self.period)

    def __enter__(self):
        if self._h:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._h:
            self._t.join()

    def summary(self):
        allm = [s[0] for v in self.samples.values() for s in v]
        if not allm:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        active = 0
        for v in self.samples.values():
            for s in v:
                active |= s[1]
        reasons = [name for name, bit in self.REASONS.items() if active & bit]
        per_gpu = [statistics.median([s[0] for s in v]) if v else None
                   for v in self.samples.values()]
        return {"sm_mhz": statistics.median(allm), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(allm), "per_gpu_sm_mhz": per_gpu}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def oracle_mod():
    """The oracle (CPU restatement of the reference): the checker and the CPU
    baseline, always outside the timed regions."""
    for p in (ROOT / "oracle",):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))
    import oracle
    return oracle


def cpu_rows_per_s(oracle, logits, vocab, params, target_s: float, threads: int):
    """Times the CPU restatement (glibc expf) over a sample of rows."""
    import numpy as np
    R = logits.shape[0]
    flat = np.ascontiguousarray(logits.reshape(-1))
    off = np.arange(R, dtype=np.int64) * vocab
    voc = np.full(R, vocab, np.int32)
    seeds = np.arange(R, dtype=np.uint64)
    sub = np.zeros(R, np.uint64)
    probe = min(R, max(64, 16 * threads))
    t0 = time.perf_counter()
    oracle.sample_rows(flat, off[:probe], voc[:probe], params, seeds[:probe], sub[:probe],
                       exp_mode=oracle.EXP_LIBM, nthreads=threads)
    rate = probe / max(time.perf_counter() - t0, 1e-6)
    n = int(min(R, max(probe, rate * target_s)))
    t0 = time.perf_counter()
    oracle.sample_rows(flat, off[:n], voc[:n], params, seeds[:n], sub[:n],
                       exp_mode=oracle.EXP_LIBM, nthreads=threads)
    dt = time.perf_counter() - t0
    return n / dt, n


def run_reference(args, world, rank):
    """CPU arm: the restated reference sampler on every host thread."""
    import numpy as np
    if rank != 0:
        return 0
    oracle = oracle_mod()
    import q3s
    threads = cpu_threads()
    rng = np.random.default_rng(3)
    sample = 8192
    logits = rng.standard_normal((sample, VOCAB), dtype=np.float32)
    params = q3s.make_params(1, top_k=TOP_K, top_p=1.0, temperature=1.0)
    flat = logits.reshape(-1)
    off = np.arange(sample, dtype=np.int64) * VOCAB
    voc = np.full(sample, VOCAB, np.int32)
    seeds = np.arange(sample, dtype=np.uint64)
    sub = np.zeros(sample, np.uint64)
    # Rows per step: about 50 ms of work so K + W steps end within minutes.
    t0 = time.perf_counter()
    oracle.sample_rows(flat, off[:256], voc[:256], params, seeds[:256], sub[:256],
                       exp_mode=oracle.EXP_LIBM, nthreads=threads)
    rate = 256 / max(time.perf_counter() - t0, 1e-6)
    per_step = int(min(sample, max(256, rate * 0.05)))

    def step(i):
        s = (i * per_step) % (sample - per_step + 1)
        oracle.sample_rows(flat, off[s:s + per_step], voc[s:s + per_step], params,
                           seeds[s:s + per_step], sub[s:s + per_step],
                           exp_mode=oracle.EXP_LIBM, nthreads=threads)
    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    dt = time.perf_counter() - t0
    value = per_step * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / max(args.steps, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "sample": f"{per_step} rows of 3072 f32 N(0,1) per step, k=50, "
                                   f"CPU restatement of src/talker/sampling.rs with glibc expf"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(rows: int = ROWS):
    mb = rows * 4 * VOCAB / 1e6
    return {"workload": f"bandwidth: {rows} rows x 3072 f32 logits ~N(0,1) per GPU, top_k 50, "
                        "top_p 1.0, temperature 1.0, no penalty",
            "rows_per_gpu": rows, "vocab": VOCAB, "top_k": TOP_K, "global_batch": None,
            "l2": f"inputs {mb:.0f} MB per step > 126 MB L2 (no flush needed)",
            "parallelism": "row shards, no collective"}


class L2Flush:
    """Writes a buffer larger than L2 (between timed launches whose inputs
    would otherwise stay cached)."""

    def __init__(self, torch, dev):
        self.buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def __call__(self):
        self.buf.fill_(1.0)


def time_each(torch, launch, iters, flush=None, stream=None):
    """Mean device time of `launch` in ms: CUDA events around each launch on
    `stream`, with an optional L2 flush before each (outside the events)."""
    stream = stream or torch.cuda.current_stream()
    for _ in range(3):
        if flush:
            flush()
        launch()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(iters)]
    for a, b in ev:
        if flush:
            flush()
        a.record(stream)
        launch()
        b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in ev) / iters


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--hetero-steps", type=int, default=100,
                    help="timed launches of the heterogeneous leg (0 skips the leg)")
    ap.add_argument("--hetero-streams", type=int, default=HETERO_STREAMS,
                    help="streams of the heterogeneous leg (smaller cases are for profiler "
                         "captures only)")
    ap.add_argument("--rows", type=int, default=ROWS,
                    help="rows per GPU (smaller cases are for profiler captures only)")
    args = ap.parse_args()
    world, rank, local = dist_setup()
    if args.impl == "reference":
        return run_reference(args, world, rank)
    rows = args.rows

    import numpy as np
    import torch
    import torch.distributed as dist

    import q3s
    from q3s import shard, workloads

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        return shard.max_over_ranks(v, device=dev)

    def gather(obj):
        if world == 1:
            return [obj]
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    ctx = q3s.Context(local)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    w = workloads.bandwidth(dev, rows=rows, top_k=TOP_K, seed=3 + rank)
    a = w.device_args(dev)
    params, seeds, subseqs = a["params"], a["seeds"], a["subseqs"]
    tokens = torch.empty(rows, dtype=torch.int32, device=dev)
    status = torch.empty(rows, dtype=torch.uint8, device=dev)
    launch = q3s.prepare_batch(w.logits, params, seeds, subseqs, ctx=ctx, out=(tokens, status))

    # Untimed pre-warm before the counted warm-up steps: keep the GPU busy for
    # at least 0.3 s so its clocks have ramped before the timed region, on
    # every rank alike (a short timed region otherwise picks up the slowest
    # rank's ramp).
    t_warm = time.perf_counter()
    while time.perf_counter() - t_warm < 0.3:
        for _ in range(50):
            launch(sh)
        torch.cuda.synchronize()
    for _ in range(max(args.warmup, 3)):
        launch(sh)
    torch.cuda.synchronize()
    if not bool((status == 0).all()):
        raise RuntimeError("sampling failed on the benchmark workload")

    props = torch.cuda.get_device_properties(dev)
    bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
    buses = gather(bus)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    host_ns = 0
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(buses) if rank == 0 else contextlib.nullcontext()
    with sampler as clocks:
        t_begin.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            h0 = time.perf_counter_ns()
            launch(sh)
            host_ns += time.perf_counter_ns() - h0
            ends[i].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    my_elapsed = t_begin.elapsed_time(t_end)
    ks = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    gaps = [ends[i].elapsed_time(starts[i + 1]) for i in range(args.steps - 1)]
    my_kernel = sum(ks) / max(args.steps, 1)
    elapsed_ms = max_over_ranks(my_elapsed)
    kernel_ms = max_over_ranks(my_kernel)
    value = shard.whole_job_rate(rows, world, args.steps, elapsed_ms)
    peak, peak_kind = measured_peak_gbs()
    achieved = rows * BYTES_PER_ROW / (kernel_ms / 1e3) / 1e9
    per_rank = gather({
        "rank": rank, "elapsed_ms": my_elapsed, "kernel_ms_mean": my_kernel,
        "kernel_ms_median": statistics.median(ks), "kernel_ms_max": max(ks),
        "gap_ms_mean": (sum(gaps) / len(gaps)) if gaps else 0.0,
        "host_enqueue_us_mean": host_ns / 1e3 / max(args.steps, 1)})

    # Parity on every rank, outside the timed region: a row sample of this
    # rank's shard against the oracle (bit-exact tokens and statuses).
    oracle = oracle_mod()
    sel = np.sort(np.random.default_rng(100 + rank).choice(rows, min(rows, 256),
                                                             replace=False))
    ref = oracle.sample_rows(*w.oracle_layout(sel), nthreads=max(1, cpu_threads() // world))
    my_ok = bool(np.array_equal(status.cpu().numpy()[sel], ref["status"]) and
                 np.array_equal(tokens.cpu().numpy().view(np.uint32)[sel], ref["tokens"]))
    parity = gather(my_ok)

    # End to end through the C ABI with host buffers.
    e2e = None
    if args.e2e_steps > 0:
        host_logits = torch.empty((rows, VOCAB), dtype=torch.float32, pin_memory=True)
        host_logits.copy_(w.logits)
        host_seeds = seeds.cpu().pin_memory()
        host_sub = subseqs.cpu().pin_memory()
        host_tok = torch.empty(rows, dtype=torch.int32, pin_memory=True)
        host_st = torch.empty(rows, dtype=torch.uint8, pin_memory=True)
        dev_logits = torch.empty_like(w.logits)
        dev_seeds = torch.empty_like(seeds)
        dev_sub = torch.empty_like(subseqs)
        chunks = 8
        cr = rows // chunks
        streams = [torch.cuda.Stream(dev) for _ in range(2)]
        chunk_launch = []
        for c in range(chunks):
            sl = slice(c * cr, (c + 1) * cr)
            chunk_launch.append(q3s.prepare_batch(dev_logits[sl], params, dev_seeds[sl],
                                                  dev_sub[sl], ctx=ctx,
                                                  out=(tokens[sl], status[sl])))

        def e2e_step():
            ev0 = torch.cuda.Event()
            ev0.record(stream)
            for c in range(chunks):
                s = streams[c % 2]
                s.wait_event(ev0)
                with torch.cuda.stream(s):
                    sl = slice(c * cr, (c + 1) * cr)
                    dev_logits[sl].copy_(host_logits[sl], non_blocking=True)
                    dev_seeds[sl].copy_(host_seeds[sl], non_blocking=True)
                    dev_sub[sl].copy_(host_sub[sl], non_blocking=True)
                    chunk_launch[c](s.cuda_stream)
                    host_tok[sl].copy_(tokens[sl], non_blocking=True)
                    host_st[sl].copy_(status[sl], non_blocking=True)
            for s in streams:
                stream.wait_stream(s)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.e2e_steps
        if not bool((host_st == 0).all()):
            raise RuntimeError("end-to-end sampling failed")
        e2e = {"value": world * rows / (e2e_ms / 1e3), "unit": "rows/s",
               "h2d_bytes_per_step": rows * (4 * VOCAB + 16),
               "d2h_bytes_per_step": rows * 5, "ms_per_step": e2e_ms}
        del host_logits, dev_logits, chunk_launch

    del w, launch
    torch.cuda.empty_cache()
    hetero = None
    if args.hetero_steps > 0:
        hetero = hetero_leg(args, world, rank, dev, ctx, q3s, workloads, shard, np, torch, oracle,
                            peak, max_over_ranks, gather)

    results = {"hetero_decode_step": hetero}
    cpu = None
    exact = None
    if rank == 0 and world == 1 and not args.no_secondary:
        results.update(secondary(ctx, dev, q3s, workloads, np, torch))
        exact = exactness_counts(dev, q3s, workloads, np, torch, oracle)
        sample_rows = 16384
        wb = workloads.bandwidth(dev, rows=sample_rows, top_k=TOP_K, seed=3)
        x = wb.logits.cpu().numpy()
        threads = cpu_threads()
        p1 = q3s.make_params(1, top_k=TOP_K)
        rate, n = cpu_rows_per_s(oracle, x, VOCAB, p1, 10.0, threads)
        rate1, n1 = cpu_rows_per_s(oracle, x, VOCAB, p1, 5.0, 1)
        cpu = {"value": rate, "unit": "rows/s", "cores": threads, "kind": "port",
               "sample": f"{n} rows of the bandwidth workload (k=50), CPU restatement of "
                         f"src/talker/sampling.rs with glibc expf, {threads} threads",
               "single_thread": {"value": rate1, "unit": "rows/s", "cores": 1,
                                 "sample": f"{n1} rows, 1 thread (the reference samples one "
                                           f"row at a time on one thread)"}}

    if not all(parity):
        raise RuntimeError(f"parity failed on ranks {[i for i, p in enumerate(parity) if not p]}")
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": dict(workload_config(rows), global_batch=rows * world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": NCU_TRAFFIC_PER_LAUNCH * rows / ROWS,
                         "traffic_unit": "bytes per launch (ncu, scaled from 16384 rows)",
                         "bytes_per_row": BYTES_PER_ROW, "kernel_ms": kernel_ms},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            "per_rank": per_rank,
            "parity_rows_checked_per_rank": int(sel.size),
            "exactness": exact,
            "results": results,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def hetero_leg(args, world, rank, dev, ctx, q3s, workloads, shard, np, torch, oracle, peak,
               max_over_ranks, gather):
    """The heterogeneous full decode step: 4096 streams x (1 talker row of
    3072 + 15 code-predictor rows of 2048), whole streams sharded over the
    ranks; L2 flushed between launches.  Every rank checks a row sample of
    its shard against the oracle."""
    streams = args.hetero_streams
    w = workloads.hetero(dev, streams=streams)
    r0, r1 = shard.stream_range(streams, 16, world, rank)
    a = w.device_args(dev)
    R = r1 - r0
    hoff = a["history_offsets"]
    launch = q3s.prepare_batch(
        w.logits, a["params"][r0 * 48:r1 * 48], a["seeds"][r0:r1], a["subseqs"][r0:r1],
        row_offsets=a["row_offsets"][r0:r1], row_vocab=a["row_vocab"][r0:r1], vocab=a["vocab"],
        history=a["history"], history_offsets=hoff[r0:r1 + 1], ctx=ctx)
    sh = torch.cuda.current_stream(dev).cuda_stream
    flush = L2Flush(torch, dev)
    ms = time_each(torch, lambda: launch(sh), args.hetero_steps, flush)
    ms_max = max_over_ranks(ms)
    rows = np.arange(r0, r1)
    H = (w.history_offsets[r0 + 1:r1 + 1] - w.history_offsets[r0:r1]).astype(np.int64)
    V = w.row_vocab[r0:r1].astype(np.int64)
    # logits + history ids + params (48) + seed + subseq + history offset +
    # row offset (8 each) + row vocabulary (4) + token and status (5).
    my_bytes = int((4 * V + 2 * H).sum()) + R * (48 + 8 + 8 + 8 + 8 + 4 + 5)
    sel = np.sort(np.random.default_rng(200 + rank).choice(R, min(R, 512), replace=False))
    ref = oracle.sample_rows(*w.oracle_layout(rows[sel]), nthreads=max(1, os.cpu_count() // world))
    ok = bool(np.array_equal(launch.status.cpu().numpy()[sel], ref["status"]) and
              np.array_equal(launch.tokens.cpu().numpy().view(np.uint32)[sel], ref["tokens"]))
    per = gather({"rank": rank, "rows": R, "ms": ms, "bytes": my_bytes, "parity_ok": ok})
    if not all(p["parity_ok"] for p in per):
        raise RuntimeError(f"hetero parity failed: {per}")
    total_rows = sum(p["rows"] for p in per)
    gbs = [p["bytes"] / (p["ms"] / 1e3) / 1e9 for p in per]
    del w, launch, flush
    torch.cuda.empty_cache()
    return {"streams": streams, "rows_total": total_rows, "n_gpus": world,
            "rows_per_s": total_rows / (ms_max / 1e3), "ms_per_launch_max": ms_max,
            "gbs_per_gpu": gbs, "hbm_frac_per_gpu": [g / peak for g in gbs],
            "l2": "flushed between launches", "parity_rows_checked_per_rank": int(sel.size),
            "per_rank": per}


def exactness_counts(dev, q3s, workloads, np, torch, oracle):
    """Tokens and statuses of every row of the five configurations against
    the oracle with glibc expf (the reference's f32::exp on Linux): rows,
    rows within 1e-6 of a CDF boundary, and mismatching rows."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import exactness
    out = {}
    cases = [("talker_single_1000", lambda: workloads.talker_single(dev, steps=1000)),
             ("cp_frame_64x15", lambda: workloads.cp_frame(dev)),
             ("talker_batch_1024", lambda: workloads.talker_batch(dev, rows=1024)),
             ("bandwidth_65536_k1", lambda: workloads.bandwidth(dev, rows=65536, top_k=1)),
             ("bandwidth_65536_k50", lambda: workloads.bandwidth(dev, rows=65536, top_k=50)),
             ("bandwidth_65536_k256", lambda: workloads.bandwidth(dev, rows=65536, top_k=256)),
             ("hetero_4096x16", lambda: workloads.hetero(dev, streams=4096))]
    for name, make in cases:
        w = make()
        a = w.device_args(dev)
        t, s = q3s.sample_batch(w.logits, a.pop("params"), a.pop("seeds"), a.pop("subseqs"), **a)
        torch.cuda.synchronize()
        rep = exactness.libm_report(w.oracle_layout(), t.cpu().numpy(), s.cpu().numpy(),
                                    nthreads=cpu_threads())
        out[name] = {k: rep[k] for k in ("rows", "boundary_rows", "draw_boundary_rows",
                                         "topp_boundary_rows", "libm_mismatch_rows",
                                         "status_mismatch_rows", "violations")}
        del w, t, s
    torch.cuda.empty_cache()
    return out


def secondary(ctx, dev, q3s, workloads, np, torch):
    """Other configurations, device-resident, timed with CUDA events around
    each launch; inputs smaller than L2 are flushed from it before each."""
    out = {}
    flush = L2Flush(torch, dev)
    sh = torch.cuda.current_stream(dev).cuda_stream

    # B=1024 talker batch (penalty over histories, suppression, top-p 0.8).
    wb = workloads.talker_batch(dev, rows=1024)
    ab = wb.device_args(dev)
    lb = q3s.prepare_batch(wb.logits, ab.pop("params"), ab.pop("seeds"), ab.pop("subseqs"),
                           ctx=ctx, **ab)
    ms = time_each(torch, lambda: lb(sh), 50, flush)
    hist_bytes = int(wb.history_offsets[-1]) * 2
    out["talker_batch_1024"] = {
        "rows_per_s": 1024 / (ms / 1e3), "ms_per_launch": ms, "l2": "flushed",
        "gbs": (1024 * (4 * 3072 + 16 + 8 + 5) + hist_bytes) / (ms / 1e3) / 1e9}
    for k in (1, 256):
        wk = workloads.bandwidth(dev, rows=65536, top_k=k, seed=9)
        ak = wk.device_args(dev)
        lk = q3s.prepare_batch(wk.logits, ak.pop("params"), ak.pop("seeds"), ak.pop("subseqs"),
                               ctx=ctx)
        ms = time_each(torch, lambda: lk(sh), 50)
        out[f"bandwidth_k{k}"] = {"rows_per_s": 65536 / (ms / 1e3), "ms_per_launch": ms,
                                  "gbs": 65536 * BYTES_PER_ROW / (ms / 1e3) / 1e9}
        del wk, lk
    # Code-predictor frame: 15 dependent bf16 [64, 2048] launches.
    wc = workloads.cp_frame(dev)
    ac = wc.device_args(dev)
    pc = ac.pop("params")
    sc, uc = ac.pop("seeds"), ac.pop("subseqs")
    x = wc.logits.view(15, 64, 2048)
    groups = [q3s.prepare_batch(x[g], pc, sc[g * 64:(g + 1) * 64], uc[g * 64:(g + 1) * 64],
                                ctx=ctx) for g in range(15)]

    def frame():
        for g in range(15):
            groups[g](sh)
    ms = time_each(torch, frame, 20, flush)
    kms = time_each(torch, lambda: groups[0](sh), 50, flush)
    out["cp_frame_64x15"] = {"us_per_group": ms * 1e3 / 15, "rows_per_s": 960 / (ms / 1e3),
                             "kernel_us_one_group": kms * 1e3, "l2": "flushed per frame"}
    # The same frame kept on the device (q3s_commit_rows after each group:
    # ids into the frame's codes, counters advanced) and captured once in a
    # CUDA graph, replayed per frame.
    cs = torch.cuda.Stream(dev)
    seeds_f = torch.arange(64, dtype=torch.int64, device=dev)
    sub_f = torch.zeros(64, dtype=torch.int64, device=dev)
    codes_f = torch.zeros((64, 16), dtype=torch.int32, device=dev)
    fstat_f = torch.zeros(64, dtype=torch.uint8, device=dev)
    tok_f = torch.empty(64, dtype=torch.int32, device=dev)
    st_f = torch.empty(64, dtype=torch.uint8, device=dev)

    def dev_frame():
        fstat_f.zero_()
        for g in range(15):
            q3s.sample_commit(x[g], pc, seeds_f, sub_f, codes=codes_f, group=g + 1,
                              frame_status=fstat_f, ctx=ctx, stream=cs.cuda_stream,
                              out=(tok_f, st_f))
    with torch.cuda.stream(cs):
        dev_frame()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cs):
        dev_frame()
    with torch.cuda.stream(cs):
        ms_eager = time_each(torch, dev_frame, 20, flush, stream=cs)
        ms_graph = time_each(torch, graph.replay, 20, flush, stream=cs)
    if int(fstat_f.sum().item()) != 0:
        raise RuntimeError("device-resident frame failed")
    out["cp_frame_64x15_device_resident"] = {
        "us_per_group_eager": ms_eager * 1e3 / 15, "us_per_group_cuda_graph": ms_graph * 1e3 / 15,
        "note": "15 x q3s_sample_commit (sampling and commit in one launch), ids and counters "
                "kept on the device; "
                "eager launches against one CUDA graph replay per frame; L2 flushed per frame"}
    del graph
    # Codebook embedding sum after sampling: 4096 streams, 16 codebooks
    # (3072 + 15 x 2048 ids), hidden 2048, bf16, a text row per stream.
    R, H = 4096, 2048
    g = torch.Generator(device=dev).manual_seed(5)
    vocabs = [3072] + [2048] * 15
    tables = [(torch.randn((v, H), device=dev, generator=g) * 0.05).to(torch.bfloat16)
              for v in vocabs]
    codes = torch.stack([torch.randint(0, v, (R,), device=dev, generator=g, dtype=torch.int32)
                         for v in vocabs], 1)
    text = torch.randn((R, H), device=dev, generator=g).to(torch.bfloat16)
    eout = (torch.empty((R, H), device=dev, dtype=torch.bfloat16),
            torch.empty(R, device=dev, dtype=torch.uint8))
    ebytes = R * (16 * H * 2 + H * 2 + H * 2 + 16 * 4 + 1)
    res = {"tables_mb": sum(v * H * 2 for v in vocabs) / 1e6}
    for label, fl in (("l2_flushed", flush), ("l2_warm", None)):
        ms = time_each(torch, lambda: q3s.embed_sum(codes, tables, text, ctx=ctx, out=eout), 50,
                       fl)
        res[label] = {"us_per_launch": ms * 1e3, "rows_per_s": R / (ms / 1e3),
                      "algorithmic_gbs": ebytes / (ms / 1e3) / 1e9}
    if not bool((eout[1] == 0).all()):
        raise RuntimeError("embedding sum failed")
    out["embed_sum_4096x16_h2048_bf16"] = res
    del tables, text, eout
    # Producer fusion: the talker's codec_head projection (3072 x 1024 bf16)
    # and the sampling of its rows in one launch, against the matmul followed
    # by the sampling launch; L2 flushed before each (the weights are not
    # assumed resident).
    hg = torch.Generator(device=dev).manual_seed(21)
    weight = (torch.randn((3072, 1024), generator=hg, device=dev) * 0.05).to(torch.bfloat16)
    head = {}
    for R in (1, 16):
        hidden = torch.randn((R, 1024), generator=hg, device=dev).to(torch.bfloat16)
        hp = q3s.make_params(R, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.0,
                             suppress_from=2048, allow_token=2150)
        dp = torch.from_numpy(hp.view(np.uint8).copy()).to(dev)
        ds = torch.arange(R, dtype=torch.int64, device=dev)
        du = torch.zeros(R, dtype=torch.int64, device=dev)
        hout = (torch.empty(R, dtype=torch.int32, device=dev),
                torch.empty(R, dtype=torch.uint8, device=dev),
                torch.empty((R, 3072), dtype=torch.float32, device=dev))
        fused = time_each(torch, lambda: q3s.head_sample(hidden, weight, dp, ds, du, ctx=ctx,
                                                         out=hout), 50, flush)
        lg = torch.empty((R, 3072), dtype=torch.bfloat16, device=dev)
        sout = (torch.empty(R, dtype=torch.int32, device=dev),
                torch.empty(R, dtype=torch.uint8, device=dev))

        def unfused():
            torch.matmul(hidden, weight.t(), out=lg)  # bf16 logits, as the model's linear
            q3s.sample_batch(lg, dp, ds, du, ctx=ctx, out=sout)
        sep = time_each(torch, unfused, 50, flush)
        head[f"rows_{R}"] = {"fused_us": fused * 1e3, "matmul_then_sample_us": sep * 1e3}
    out["head_sample_3072x1024_bf16"] = dict(head, note="q3s_head_sample (projection and "
                                             "sampling in one launch) against torch.matmul "
                                             "(bf16 logits) followed by q3s_sample_batch; "
                                             "CUDA events, L2 flushed before each launch")
    del weight
    # Single-stream talker step through the stateful Sampler (host round trip),
    # broken down: the binding call, the bare C call, the kernel alone.
    import ctypes
    ws = workloads.talker_single(dev, steps=400)
    s = q3s.Sampler(42, ctx)
    o = q3s.SamplingOptions(0.9, 50, 1.0, 1.05)
    hist = np.ascontiguousarray(ws.history[:256])
    for i in range(5):
        s.sample_with_mode(ws.logits[i], o, True, 2048, 2150, hist)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(200):
        s.sample_with_mode(ws.logits[i], o, True, 2048, 2150, hist)
    dt = time.perf_counter() - t0
    grow = list(hist)
    t0 = time.perf_counter()
    for i in range(200):
        tok = s.sample_with_mode(ws.logits[200 + i], o, True, 2048, 2150,
                                 np.array(grow, np.uint16))
        grow.append(tok % 2048)
    dt_grow = time.perf_counter() - t0
    L = q3s.load()
    copt = o._c()
    tok_c, st_c = ctypes.c_uint32(0), ctypes.c_int32(0)
    cb = q3s.TRANSFER_CALLBACK(0)
    hp = hist.ctypes.data_as(ctypes.c_void_p)
    ptrs = [ctypes.c_void_p(ws.logits[i].data_ptr()) for i in range(200)]
    stream_c = ctypes.c_void_p(sh)
    t0 = time.perf_counter()
    for i in range(200):
        L.q3s_sampler_sample_with_mode(s._h, ptrs[i], q3s.DTYPE_F32, 3072, ctypes.byref(copt), 1,
                                       2048, 2150, hp, 256, cb, None, ctypes.byref(tok_c),
                                       ctypes.byref(st_c), stream_c)
    dt_c = time.perf_counter() - t0
    aw = ws.device_args(dev)
    one = q3s.prepare_batch(ws.logits[0:1], aw["params"], aw["seeds"][:1], aw["subseqs"][:1],
                            history=aw["history"], history_offsets=aw["history_offsets"][:2],
                            ctx=ctx)
    kms = time_each(torch, lambda: one(sh), 50, flush)
    kms_warm = time_each(torch, lambda: one(sh), 50)
    t0 = time.perf_counter()
    for _ in range(200):
        one(sh)
    enq = (time.perf_counter() - t0) / 200
    torch.cuda.synchronize()
    out["talker_single_step"] = {
        "us_per_step": dt * 1e6 / 200,
        "us_per_step_growing_history": dt_grow * 1e6 / 200,
        "c_call_us": dt_c * 1e6 / 200,
        "kernel_us_l2_warm": kms_warm * 1e3,
        "kernel_us_l2_flushed": kms * 1e3,
        "launch_enqueue_us": enq * 1e6,
        "note": "us_per_step: stateful Sampler call through the Python binding (256-id "
                "history, host wall clock, includes the sync and the token read); "
                "growing: the history grows by one id per step as the talker's does; "
                "c_call_us: the same C entry point called with prebuilt arguments; "
                "kernel_us: the 1-row launch alone (CUDA events)"}
    return out


if __name__ == "__main__":
    sys.exit(main())
