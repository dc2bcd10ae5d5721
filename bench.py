"""Benchmark of the batched token sampler (franzvill/quasar sample.c rebuilt for B200).

Workload (the headline): per GPU, B=4096 rows of
V=151936 fp32 logits ~N(0,3) (synthetic, seeded), per-row temperature
U[0.2,1.5], top_k off, top_p 0.95, min_p 0.05, repeat_penalty 1.1 over a
256-id history ring per row, row-indexed PRNG seeds, record on.
One step = one quasar_sampler_pick_batch call over the B rows. Rows are
independent, so N GPUs run N shards with no collective ("scaling": "weak").

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0. `value` is device-timed (CUDA events, inputs
resident in HBM, 2.49 GB per step > L2); `e2e` times the same call through the
public API with the logits copied from pinned host memory every step and the
ids read back. `--impl reference` times the reference sample.c (compiled
unmodified into oracle/_ref) on the host cores on bounded row samples.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

V = 151936
B = 4096
H = 256
SEED_LOGITS, SEED_HIST, SEED_TEMP, SEED_RNG = 3, 33, 3, 5000
METRIC = "sampled rows/s at V=151936, B=4096; % HBM roofline at 1/2/4/8 B200"
# algorithmic bytes per row: logits V*4 + history H*4 + ring len/head 8 + params 24
# + rng read/write 16 + id 4 + ring append 8
BYTES_PER_ROW = V * 4 + H * 4 + 60
FALLBACK_HBM_GBS = 6650.0


# Rows-mode workloads: 3 is the headline, 5 the
# full-vocab softmax + multinomial case.
CONFIGS = {
    "3": dict(rows=4096, hist=256, kind=0, scale=3.0, temp=(0.2, 1.5), top_p=0.95, min_p=0.05, rp=1.1, top_k=0,
              text="config3: N(0,3) logits, per-row T~U[0.2,1.5], top_p 0.95, min_p 0.05, "
                   "repeat_penalty 1.1 over 256 history ids, record on"),
    "5": dict(rows=16384, hist=2048, kind=2, scale=1.1, temp=(1.0, 1.0), top_p=1.0, min_p=0.1, rp=1.3, top_k=0,
              text="config5: Zipf(1.1) logits (-1.1 ln rank, per-row rank permutation), T 1.0, min_p 0.1, "
                   "repeat_penalty 1.3 over 2048 history ids, record on"),
    "2": dict(rows=256, hist=0, kind=1, scale=1.0, temp=(0.0, 0.0), top_p=1.0, min_p=0.0, rp=1.0, top_k=0,
              text="config2: Gumbel(0,1) logits with a planted +8 peak per row, greedy (temperature 0)"),
    "2k": dict(rows=256, hist=0, kind=1, scale=1.0, temp=(1.0, 1.0), top_p=1.0, min_p=0.0, rp=1.0, top_k=1,
               text="config2: Gumbel(0,1) logits with a planted +8 peak per row, top_k 1 at temperature 1"),
    # rows that only cut by top-p take the exact radix-select path (whole-row passes)
    "topp": dict(rows=4096, hist=256, kind=0, scale=3.0, temp=(0.2, 1.5), top_p=0.95, min_p=0.0, rp=1.1, top_k=0,
                 text="select path: config-3 logits and temperatures, top_k 0, min_p 0, top_p 0.95, "
                      "repeat_penalty 1.1 over 256 history ids, record on"),
}
CFG = CONFIGS["3"]


def workload_config(n_gpus: int) -> dict:
    return {"workload": CFG["text"], "rows_per_gpu": B, "vocab": V, "history": H, "global_batch": B * n_gpus,
            "parallelism": f"rows x{n_gpus}",
            "l2": "inputs larger than L2 (%.2f GB of logits per step per GPU)" % (B * V * 4 / 1e9)}


def peak_hbm() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic_per_launch() -> float | None:
    """DRAM bytes per launch of the sampler kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "sample_rows_config3_traffic.txt")
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch_full_size="):
                    return float(line.split("=", 1)[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while GPU work runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: str):
        self.gpus = gpus
        self.rows: list[list[str]] = []
        self.proc = None
        self.th = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpus, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.th = threading.Thread(target=self._read, daemon=True)
        self.th.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict | None:
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.th:
            self.th.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_rows(n_rows: int, row0: int = 0):
    """Workload rows [row0, row0+n_rows) generated on the CPU (same bits as the GPU)."""
    from oracle import oracle as O
    logits = O.synth_logits(CFG["kind"], SEED_LOGITS, row0, n_rows, V, CFG["scale"])
    hist = O.synth_hist(SEED_HIST, row0, n_rows, H, V)
    temps = O.synth_uniform(SEED_TEMP, row0, n_rows, *CFG["temp"])
    prm = O.make_params(n_rows, temperature=temps, top_p=CFG["top_p"], min_p=CFG["min_p"],
                        repeat_penalty=CFG["rp"], top_k=CFG["top_k"])
    seeds = np.arange(row0, row0 + n_rows, dtype=np.uint64) + np.uint64(SEED_RNG)
    return logits, (hist if H else None), prm, seeds


def time_cpu_reference(n_rows: int, threads: int, row0: int = 0):
    """(rows/s, backend kind) of the reference sampler on host cores."""
    from oracle import oracle as O
    backend = O.best_backend()
    logits, hist, prm, seeds = cpu_rows(n_rows, row0)
    t0 = time.perf_counter()
    O.pick_rows(logits, prm, seeds, hist=hist, backend=backend, nthreads=threads)
    dt = time.perf_counter() - t0
    return n_rows / dt, ("reference" if backend == "ref" else "port"), dt


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    if not O.available("ref") and not O.available("oracle"):
        O.build()
    threads = cpu_threads()
    sample = 8 * threads
    backend = O.best_backend()
    for w in range(args.warmup):
        time_cpu_reference(min(sample, 2 * threads), threads, row0=w * sample)
    rates, total_rows, total_t = [], 0, 0.0
    for k in range(args.steps):
        logits, hist, prm, seeds = cpu_rows(sample, row0=k * sample)
        t0 = time.perf_counter()
        O.pick_rows(logits, prm, seeds, hist=hist, backend=backend, nthreads=threads)
        dt = time.perf_counter() - t0
        rates.append(sample / dt)
        total_rows += sample
        total_t += dt
    value = total_rows / total_t
    kind = "reference" if backend == "ref" else "port"
    line = {"metric": METRIC, "value": value, "unit": "rows/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * total_t / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args.gpus),
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": kind,
                             "sample": f"{sample} {CFG['text'].split(':')[0]} rows per step (rows [k*{sample}, "
                                       f"(k+1)*{sample}) of the workload), one sampler object "
                                       f"per row, {threads} pthreads"},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    import quasar_b200 as q

    row0 = rank * B  # each rank samples its own rows of the synthetic batch
    logits = torch.empty(B, V, dtype=torch.float32, device=dev)
    q.synth_logits(CFG["kind"], SEED_LOGITS, row0, B, V, CFG["scale"], logits)
    hist = hist_len = hist_head = None
    if H:
        hist = torch.empty(B, H, dtype=torch.int32, device=dev)
        q.synth_hist(SEED_HIST, row0, B, H, V, hist)
        hist_len = torch.full((B,), H, dtype=torch.int32, device=dev)
        hist_head = torch.zeros(B, dtype=torch.int32, device=dev)
    temps = torch.empty(B, dtype=torch.float32, device=dev)
    q.synth_uniform(SEED_TEMP, row0, B, *CFG["temp"], temps)
    prm = q.make_params(B, temperature=temps.cpu().numpy(), top_p=CFG["top_p"], min_p=CFG["min_p"],
                        repeat_penalty=CFG["rp"], top_k=CFG["top_k"])
    d_params = q.params_to_device(prm, dev)
    seeds = np.arange(row0, row0 + B, dtype=np.uint64) + np.uint64(SEED_RNG)
    rng = torch.from_numpy(seeds.view(np.int64).copy()).to(dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    ws_bytes = q.workspace_bytes(B, H)
    ws_buf = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=dev)
    ws = ws_buf[(-ws_buf.data_ptr()) % 256:][:ws_bytes]

    def step(src=logits):
        q.pick_batch(src, rng, d_params=d_params, hist=hist, hist_len=hist_len,
                     hist_head=hist_head, record=H > 0, out=out, workspace=ws, flags=args.flags, stream=stream)

    def stream_only():
        # the streaming kernel alone (kernel A, the same instance pick_batch
        # launches for these rows): quasar_shard_stats over the whole rows
        check(q.lib().quasar_shard_stats(
            ctypes.c_void_p(logits.data_ptr()), logits.stride(0), B, V, 0, ctypes.c_void_p(d_params.data_ptr()),
            None, None if hist is None else ctypes.c_void_p(hist.data_ptr()), H,
            None if hist is None else ctypes.c_void_p(hist_len.data_ptr()),
            None if hist is None else ctypes.c_void_p(hist_head.data_ptr()), ctypes.c_void_p(stats.data_ptr()),
            ctypes.c_void_p(ws.data_ptr()), ws_bytes, args.flags, ctypes.c_void_p(stream.cuda_stream)),
            "quasar_shard_stats")

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)

    clocks = ClockSampler(",".join(str(i) for i in range(world)) if world > 1 else str(local))
    if rank == 0:
        clocks.start()
        time.sleep(0.2)
    # ---- device-timed region: inputs resident in HBM ----
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # ---- end to end through the public API, host buffers ----
    e2e_steps = 0 if args.no_e2e else max(1, min(args.steps, 5))
    if e2e_steps:
        host = torch.empty(B, V, dtype=torch.float32, pin_memory=True)
        host.copy_(logits)
        ids_host = torch.empty(B, dtype=torch.int32, pin_memory=True)
        stage = torch.empty_like(logits)
    h2d = B * V * 4
    d2h = B * 4
    barrier()
    torch.cuda.synchronize(dev)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e2e_steps):
        stage.copy_(host, non_blocking=True)
        step(stage)
        ids_host.copy_(out, non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    t2 = torch.tensor([f0.elapsed_time(f1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_ms = float(t2.item())

    # ---- the dominant kernel alone: kernel A (the streaming pass), CUDA
    # events on the stream it is launched on, inputs resident in HBM ----
    from quasar_b200._lib import check
    stats = torch.empty(B * 16, dtype=torch.uint8, device=dev)
    for _ in range(3):
        stream_only()
    torch.cuda.synchronize(dev)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(args.steps):
        stream_only()
    g1.record(stream)
    torch.cuda.synchronize(dev)
    a_ms = g0.elapsed_time(g1) / args.steps
    clk = clocks.stop() if rank == 0 else None

    rows_total = B * world * args.steps
    value = rows_total / (ms_max / 1e3)
    call_s = (ms / 1e3) / args.steps  # both kernels of one pick_batch call
    achieved = B * BYTES_PER_ROW / (a_ms / 1e3) / 1e9
    peak, peak_kind = peak_hbm()
    # the committed ncu summary covers the headline workload only
    traffic = ncu_traffic_per_launch() if CFG is CONFIGS["3"] and B == CONFIGS["3"]["rows"] else None
    line = {"metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload_config(world),
            "roofline": {"bound": "hbm", "kernel": "sample_rows_tma (kernel A, the streaming pass)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": peak_kind, "kernel_ms": a_ms,
                         "algorithmic_bytes_per_launch": B * BYTES_PER_ROW,
                         # the whole pick_batch call (kernel A + kernel B) against the same bytes
                         "call_achieved": B * BYTES_PER_ROW / call_s / 1e9,
                         "call_frac": B * BYTES_PER_ROW / call_s / 1e9 / peak},
            "e2e": None if not e2e_steps else {
                    "value": B * world * e2e_steps / (e2e_ms / 1e3), "unit": "rows/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps * q.lib().quasar_sampler_pick_batch_launches(),
            "clocks": clk}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = cpu_threads()
        rows = max(64, min(1024, 32 * threads))
        rate, kind, dt = time_cpu_reference(rows, threads)
        line["cpu_baseline"] = {"value": rate, "unit": "rows/s", "cores": threads, "kind": kind,
                                "sample": f"first {rows} rows of the {CFG['text'].split(':')[0]} workload "
                                          f"({dt:.1f} s wall on {threads} threads)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_latency(args) -> None:
    """BASELINE.json config 1, the latency case: one row (V=151936 N(0,3),
    seed 42), temperature 0.7, top_k 20, top_p 0.8, repeat_penalty 1.1 over
    the last 64 ids, seed 42. Timed three ways: the sample.h drop-in
    (quasar_sampler_pick) on a host row and on a device row (wall clock per
    call: each call blocks until the id is on the host), and
    quasar_sampler_pick_batch with B=1 on device-resident state (CUDA events
    over back-to-back calls), the last also at B = 4 and 16 and with each
    row on one CTA (QUASAR_FLAG_NO_SPLIT) beside the default fused cluster
    kernel of small batches.
    The reference sample.c, one core, on the same row is the CPU figure."""
    import torch
    import quasar_b200 as q
    from oracle import oracle as O
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    row = torch.empty(1, V, dtype=torch.float32, device=dev)
    q.synth_logits(q.SYNTH_NORMAL, 42, 0, 1, V, 3.0, row)
    host = row.cpu().numpy()[0].copy()
    kw = dict(temperature=0.7, top_p=0.8, top_k=20, min_p=0.0, repeat_penalty=1.1)
    steps = max(args.steps, 20)

    def drop_in(src):
        smp = q.Sampler()
        smp.config(kw["temperature"], kw["top_p"], kw["top_k"], kw["min_p"], kw["repeat_penalty"], 64, 42)
        for _ in range(max(args.warmup, 3)):
            smp.pick(src)
        ts = []
        for _ in range(steps):
            t0 = time.perf_counter()
            smp.pick(src)
            ts.append((time.perf_counter() - t0) * 1e3)
        smp.close()
        ts.sort()
        return ts[len(ts) // 2], ts[int(len(ts) * 0.9)]

    host_ms, host_p90 = drop_in(host)
    dev_ms, dev_p90 = drop_in(row[0])
    prm = q.make_params(1, **kw)
    stream = torch.cuda.current_stream(dev)

    def batch_ms(B, flags):
        """pick_batch over B rows (config 1's parameters), state on the
        device, calls back to back: CUDA events per call."""
        rows = torch.empty(B, V, dtype=torch.float32, device=dev)
        q.synth_logits(q.SYNTH_NORMAL, 42, 0, B, V, 3.0, rows)
        hist = torch.empty(B, 64, dtype=torch.int32, device=dev)
        q.synth_hist(42, 0, B, 64, V, hist)
        hl = torch.full((B,), 64, dtype=torch.int32, device=dev)
        hh = torch.zeros(B, dtype=torch.int32, device=dev)
        rng = torch.arange(42, 42 + B, dtype=torch.int64, device=dev)
        out = torch.empty(B, dtype=torch.int32, device=dev)
        nb = q.workspace_bytes(B, 64)
        ws = torch.empty(nb + 256, dtype=torch.uint8, device=dev)
        wsv = ws[(-ws.data_ptr()) % 256:][:nb]
        for _ in range(max(args.warmup, 3)):
            q.pick_batch(rows, rng, params=prm, hist=hist, hist_len=hl, hist_head=hh, record=True, out=out,
                         workspace=wsv, flags=flags, stream=stream)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            q.pick_batch(rows, rng, params=prm, hist=hist, hist_len=hl, hist_head=hh, record=True, out=out,
                         workspace=wsv, flags=flags, stream=stream)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps

    small = {}
    for B in (1, 4, 16):
        small[f"pick_batch_B{B}_split{q.split_shards(B, V, params=prm, hist_cap=64)}_per_call"] = batch_ms(B, 0)
        small[f"pick_batch_B{B}_one_cta_per_row_per_call"] = batch_ms(B, q.FLAG_NO_SPLIT)
    batch_ms1 = small["pick_batch_B1_split%d_per_call" % q.split_shards(1, V, params=prm, hist_cap=64)]
    # the reference sample.c on one core, the same row and parameters
    n_ref = 10
    t0 = time.perf_counter()
    O.ref_sequence(np.tile(host, (n_ref, 1)), O.make_params(1, **kw), 64, 42)
    ref_ms = (time.perf_counter() - t0) * 1e3 / n_ref
    line = {"metric": "config1: single-row pick latency (sample.h drop-in, host row)", "value": host_ms,
            "unit": "ms", "n_gpus": 1, "steps": steps, "warmup": args.warmup, "ms_per_step": host_ms,
            "higher_is_better": False, "scaling": "none", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "config1: 1 row, V=151936 N(0,3) seed 42, T 0.7, top_k 20, top_p 0.8, "
                                   "repeat_penalty 1.1 over the last 64 ids, seed 42"},
            "latency_ms": {"drop_in_host_row_p50": host_ms, "drop_in_host_row_p90": host_p90,
                           "drop_in_device_row_p50": dev_ms, "drop_in_device_row_p90": dev_p90,
                           "pick_batch_B1_device_per_call": batch_ms1, **small},
            "split_shards_B1": q.split_shards(1, V, params=prm, hist_cap=64),
            "e2e": {"value": host_ms, "unit": "ms", "h2d_bytes_per_step": V * 4, "d2h_bytes_per_step": 4},
            "gpu_launches": steps * (1 if q.split_shards(1, V, params=prm, hist_cap=64) else 2),
            "cpu_baseline": {"value": ref_ms, "unit": "ms", "cores": 1, "kind": "reference",
                             "sample": f"{n_ref} picks of the same row through one reference sampler object"}}
    print(json.dumps(line), flush=True)


def run_vocab_emulated(args) -> None:
    """Config 4's kernels on one GPU: the 8192 rows split into G column shards
    of V/G (18,992 at G=8), every shard's phase 1 and phase 2 run one after
    another and the merge once, the gathers done by placement (no exchange).
    Reports each phase's device time per shard (CUDA events between the
    phases): what one rank of a G-way split spends in kernels."""
    import torch
    import quasar_b200 as q
    from quasar_b200.sharded import STAT_BYTES, CudaShardPhases
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    G, rows, K = args.emulate_shards, args.rows or 8192, 40
    vs = V // G
    logits = torch.empty(rows, V, dtype=torch.float32, device=dev)
    q.synth_logits(q.SYNTH_NORMAL, SEED_LOGITS, 0, rows, V, 3.0, logits)
    shards = [logits[:, g * vs:(g + 1) * vs].contiguous() for g in range(G)]
    del logits
    torch.cuda.empty_cache()
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(SEED_RNG)
    rng = torch.from_numpy(seeds.view(np.int64).copy()).to(dev)
    prm = q.make_params(1, temperature=0.8, top_k=K, top_p=0.9)
    from quasar_b200.sharded import _host_params
    hp = _host_params(prm)
    ph = CudaShardPhases()
    stream = torch.cuda.current_stream(dev)
    wsb = q.workspace_bytes(rows, 0)
    wss = [torch.empty(wsb + 256, dtype=torch.uint8, device=dev) for _ in range(G)]
    wss = [w[(-w.data_ptr()) % 256:][:wsb] for w in wss]
    all_stats = torch.empty(G * rows * STAT_BYTES, dtype=torch.uint8, device=dev)
    all_cand = torch.empty(G * rows * K, dtype=torch.int64, device=dev)
    out = torch.empty(rows, dtype=torch.int32, device=dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    acc = [0.0, 0.0, 0.0]

    def step(timed):
        if timed:
            ev[0].record(stream)
        for g in range(G):
            ph.stats(shards[g], g * vs, hp, None, None, None, None,
                     all_stats[g * rows * STAT_BYTES:(g + 1) * rows * STAT_BYTES], wss[g], stream)
        if timed:
            ev[1].record(stream)
        for g in range(G):
            ph.candidates(shards[g], g * vs, hp, None, None, None, None, all_stats, G, g, K,
                          all_cand[g * rows * K:(g + 1) * rows * K], wss[g], stream)
        if timed:
            ev[2].record(stream)
        ph.finish(all_cand, all_stats, G, K, rows, hp, None, rng, None, None, None, False, out, None, stream)
        if timed:
            ev[3].record(stream)
            torch.cuda.synchronize(dev)
            for i in range(3):
                acc[i] += ev[i].elapsed_time(ev[i + 1])

    for _ in range(max(args.warmup, 3)):
        step(False)
    torch.cuda.synchronize(dev)
    for _ in range(args.steps):
        step(True)
    stats_ms, cand_ms, merge_ms = (x / args.steps for x in acc)
    per_rank = stats_ms / G + cand_ms / G + merge_ms
    peak, peak_kind = peak_hbm()
    shard_bytes = rows * (vs * 4 + 24)
    line = {"metric": "config4 kernels per rank of a %d-way vocab split (emulated on one GPU)" % G,
            "value": rows / (per_rank / 1e3), "unit": "rows/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": per_rank, "higher_is_better": True, "scaling": "none",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config4: 8192 rows, %d shards of %d columns, N(0,3), top_k 40, top_p 0.9, T 0.8"
                                   % (G, vs), "parallelism": "vocab x%d emulated" % G},
            "phases_ms_per_rank": {"stats (kernel A on one shard)": stats_ms / G,
                                   "candidates (kernel B on one shard)": cand_ms / G,
                                   "merge (every rank, all rows)": merge_ms},
            "roofline": {"bound": "hbm", "kernel": "sample_rows_tma on one %d-column shard" % vs,
                         "achieved": shard_bytes / (stats_ms / G / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": shard_bytes / (stats_ms / G / 1e3) / 1e9 / peak, "traffic": None,
                         "peak_source": peak_kind, "algorithmic_bytes_per_launch": shard_bytes},
            "gpu_launches": args.steps * (2 * G + 1)}
    print(json.dumps(line), flush=True)


def run_vocab_sharded(args) -> None:
    """Config 4: the vocab split over the ranks (tensor-parallel LM head).

    Every rank holds V/N columns of the same 8192 rows (N(0,3), seeded);
    top_k 40, top_p 0.9, temperature 0.8, no history. One step = one
    quasar_shard_pick call (NcclShardedSampler.pick): per-shard stats, an
    NCCL all-gather, per-shard top-40 candidates, a second all-gather,
    merge/cut/draw on every rank.
    `value` = rows per second of the whole job (all ranks sample the same
    rows together); the roofline counts each rank's shard bytes against one
    GPU's measured bandwidth."""
    import datetime

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev, world_size=world,
                            rank=rank, init_method=None if world > 1 else "tcp://127.0.0.1:29611")
    import quasar_b200 as q
    rows, K = 8192, 40
    vs = V // world
    full = torch.empty(rows, V, dtype=torch.float32, device=dev)
    q.synth_logits(q.SYNTH_NORMAL, SEED_LOGITS, 0, rows, V, 3.0, full)
    shard = full[:, rank * vs:(rank + 1) * vs].contiguous()
    del full
    torch.cuda.empty_cache()
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(SEED_RNG)
    rng = torch.from_numpy(seeds.view(np.int64).copy()).to(dev)
    out = torch.empty(rows, dtype=torch.int32, device=dev)
    # the C entry (quasar_shard_pick) over the library's own NCCL communicator;
    # torch.distributed only hands out its id and times the step
    uid = [q.NcclCommunicator.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    comm = q.NcclCommunicator(world, rank, uid[0], timeout_ms=60000)
    smp = q.NcclShardedSampler(comm, K)
    prm = {"temperature": 0.8, "top_k": K, "top_p": 0.9}
    stream = torch.cuda.current_stream(dev)

    def step():
        smp.pick(shard, rank * vs, rng, params=prm, out=out, stream=stream)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(",".join(str(i) for i in range(world)))
    if rank == 0:
        clocks.start()
        time.sleep(0.2)
    dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    clk = clocks.stop() if rank == 0 else None
    comm.wait(stream, timeout_ms=60000)
    # where a step's device time goes: one traced step (CUPTI through
    # torch.profiler), device time per kernel, the NCCL all-gathers included
    phases = None
    if args.trace_phases:
        from torch.profiler import ProfilerActivity, profile
        dist.barrier()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(3):
                step()
            torch.cuda.synchronize(dev)
        phases = {}
        for ev in prof.key_averages():
            dt = getattr(ev, "device_time_total", None) or getattr(ev, "cuda_time_total", 0)
            if dt and ev.count:
                phases[ev.key[:80]] = round(dt / 3.0, 2)  # us per step
        dist.barrier()
    per_step = ms / 1e3 / args.steps
    shard_bytes = rows * (vs * 4 + 24)
    peak, peak_kind = peak_hbm()
    line = {"metric": "sampled rows/s, vocab-sharded (config 4)", "value": rows / per_step, "unit": "rows/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "config4: %d rows x %d columns per GPU, N(0,3), top_k 40, top_p 0.9, T 0.8"
                                   % (rows, vs), "global_batch": rows, "parallelism": "vocab x%d" % world},
            "roofline": {"bound": "hbm", "achieved": shard_bytes / per_step / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": shard_bytes / per_step / 1e9 / peak, "traffic": None, "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": shard_bytes},
            "gpu_launches": args.steps * 3, "clocks": clk,
            "exchange": "quasar_shard_pick: two in-place NCCL all-gathers (libquasar_cuda communicator, "
                        "non-blocking, 60 s limit)"}
    if phases is not None:
        line["phases_us_per_step_rank0"] = phases
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", default="3", choices=sorted(CONFIGS) + ["1"],
                    help="workload: BASELINE.json config 3 (headline), 5, 2 (greedy) / 2k (top_k 1), "
                         "1 (single-row latency), or topp (top-p-only rows: the select path)")
    ap.add_argument("--emulate-shards", type=int, default=0,
                    help="vocab mode on one GPU: the phases of G shards of config 4 run one after another "
                         "(kernel costs of a G-way split, no exchange)")
    ap.add_argument("--rows", type=int, default=None, help="rows per GPU (default: the config's; profiling "
                                                          "runs use fewer)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg (profiling)")
    ap.add_argument("--flags", type=int, default=0, help="quasar_sampler_pick_batch flags (A/B runs)")
    ap.add_argument("--trace-phases", action="store_true",
                    help="vocab mode: trace one step per kernel (torch.profiler / CUPTI) after the timed region")
    ap.add_argument("--mode", default="rows", choices=["rows", "vocab"],
                    help="rows: config 3, rows split over GPUs (default); vocab: config 4, vocab split")
    args = ap.parse_args()
    cfg = CONFIGS[args.config] if args.config != "1" else CONFIGS["3"]
    globals()["CFG"] = cfg
    globals()["B"] = args.rows or cfg["rows"]
    globals()["H"] = cfg["hist"]
    globals()["BYTES_PER_ROW"] = V * 4 + cfg["hist"] * 4 + 60
    if args.config == "1" and args.impl == "ours":
        run_latency(args)
    elif args.mode == "vocab" and args.impl == "ours" and args.emulate_shards:
        run_vocab_emulated(args)
    elif args.mode == "vocab" and args.impl == "ours":
        run_vocab_sharded(args)
    elif args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
