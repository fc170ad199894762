#!/usr/bin/env python
"""Benchmark: q4_K batch-1 matvec HBM GB/s on B200 (BASELINE cfg0 shape).

One step = one pass of the quantized matvec path over one batch: for each of
C=6 distinct q4_K weight matrices of 17408 x 5120 (the config-0 shape; 6 x
50.1 MB = 301 MB rotate so the working set exceeds the 126 MB L2), quantize a
5120-long fp32 activation to q8_K and multiply.  Steps are replayed through
CUDA graphs of the C-ABI calls (m27b_act_quant + m27b_qmv), timed with CUDA
events on the launching stream, bracketed by a barrier and a synchronize.

value  = algorithmic bytes of all ranks' steps / max-over-ranks time, where a
         matvec's algorithmic bytes are W 50,135,040 + x 20,480 + y 69,632.
e2e    = the same through the C ABI with host buffers: per matvec a pinned
         host->device copy of x and a device->host copy of y inside the
         timed region.
roofline = the matvec kernel alone (graphs of m27b_qmv over the rotating
         weights), bytes per launch / mean launch time, against the measured
         HBM copy bandwidth in MEASURED_PEAKS.json.
cpu_baseline = the CPU oracle (restatement of ggml's vec_dot_q4_K_q8_K,
         OpenMP over rows) timed on this host's cores on a bounded sample.

--impl reference times that CPU path (the reference ships no CPU path of its
own and its ggml dependency is absent) on the same metric.

Multi-GPU (torchrun): each rank runs its own replica (the matvec shards by
matrix with no exchange), scaling "weak", value summed over ranks.
"""
import argparse
import json
import os
import re
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mono-qwen27_b200")
for _p in (ROOT, PKG, os.path.join(ROOT, "tests")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

ROWS, K = 17408, 5120
Q4_K = 12
W_BYTES = ROWS * (K // 256) * 144          # 50,135,040
X_BYTES = K * 4                            # fp32 activation in
Y_BYTES = ROWS * 4                         # fp32 output
MV_BYTES = W_BYTES + X_BYTES + Y_BYTES     # 50,225,152 algorithmic bytes per matvec
COPIES = 6
GRAPH_STEPS = 16
METRIC = "q4_K matvec HBM GB/s"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=40000)
    p.add_argument("--warmup", type=int, default=200)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def random_q4K(seed):
    import numpy as np
    from _data import random_valid_blocks
    return random_valid_blocks(Q4_K, ROWS, K, seed)


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic_per_launch():
    """DRAM bytes per launch of the q4_K matvec from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "qmv_q4K_cfg0.md")
    try:
        m = re.search(r"dram_bytes_per_launch:\s*([0-9]+)", open(path).read())
        return int(m.group(1)) if m else None
    except OSError:
        return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.lines = []

    def start(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.uuid, f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.5)
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [s.strip() for s in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_oracle_gbs(w_host, seconds, nthreads=0, rows=None):
    """GB/s of the CPU oracle's q4_K.q8_K matvec on (a row sample of) w_host."""
    import numpy as np
    from oracle import oracle as orc
    from _data import gauss_act
    w = w_host if rows is None else w_host[:rows]
    n = w.shape[0]
    xq = orc.quantize_q8_K(gauss_act(1, K, 1))
    orc.matvec(Q4_K, w, K, xq, nthreads)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        orc.matvec(Q4_K, w, K, xq, nthreads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds and reps >= 3:
            break
    bytes_per = n * (K // 256) * 144 + X_BYTES + n * 4
    return bytes_per * reps / el / 1e9, reps, n, (nthreads or orc.max_threads())


def run_reference(args, world, rank):
    """CPU reference arm: the ggml-semantics CPU path on all host threads."""
    if rank != 0:
        return 0
    from oracle import oracle as orc
    w = random_q4K(0)
    threads = orc.max_threads()
    # calibrate one full matvec, then size each step's row sample so that
    # warmup + steps take about a minute of CPU time in total
    t0 = time.perf_counter()
    cpu_oracle_gbs(w, 0.0)
    full = max(1e-4, (time.perf_counter() - t0) / 4)
    budget = 60.0 / max(1, args.steps + args.warmup)
    rows = int(min(ROWS, max(64, ROWS * budget / full)))
    from _data import gauss_act
    xq = orc.quantize_q8_K(gauss_act(1, K, 1))
    ws = w[:rows]
    for _ in range(args.warmup):
        orc.matvec(Q4_K, ws, K, xq)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.matvec(Q4_K, ws, K, xq)
    el = time.perf_counter() - t0
    step_bytes = rows * (K // 256) * 144 + X_BYTES + rows * 4
    gbs = step_bytes * args.steps / el / 1e9
    sample = f"{rows} of {ROWS} rows of one cfg0 q4_K matrix per step, x quantized to q8_K"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4_K*q8_K int32->f32",
        "data": "synthetic (seeded random valid q4_K blocks)",
        "config": {"workload": "cfg0: q4_K matvec 17408x5120, batch 1", "rows": ROWS, "k": K},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU restatement of ggml's vec_dot_q4_K_q8_K (ggml itself is absent from the reference checkout)",
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import numpy as np
    import torch
    import m27b

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))

    def barrier():
        if dist:
            dist.barrier()

    # ---- inputs resident in HBM
    host_w0 = None
    Ws = []
    for c in range(COPIES):
        wh = random_q4K(1000 * rank + c)
        if c == 0:
            host_w0 = wh
        Ws.append(m27b.QWeight(wh, Q4_K, K, ROWS))
    gen = np.random.default_rng(7 + rank)
    xs = [torch.from_numpy(gen.standard_normal((1, K)).astype(np.float32)).to(dev) for _ in range(COPIES)]
    xq = [torch.empty(m27b.act_bytes(m27b.Q8_K, K), dtype=torch.uint8, device=dev) for _ in range(COPIES)]
    ys = [torch.empty((1, ROWS), dtype=torch.float32, device=dev) for _ in range(COPIES)]
    # host buffers for the end-to-end variant
    xh = [x.cpu().pin_memory() for x in xs]
    yh = [torch.empty((1, ROWS), dtype=torch.float32).pin_memory() for _ in range(COPIES)]

    def step_dev():
        for c in range(COPIES):
            m27b.act_quant(xs[c], m27b.Q8_K, out=xq[c])
            m27b.qmv(Ws[c], xq[c], 1, ys[c])

    def step_qmv_only():
        for c in range(COPIES):
            m27b.qmv(Ws[c], xq[c], 1, ys[c])

    def step_e2e():
        for c in range(COPIES):
            xs[c].copy_(xh[c], non_blocking=True)
            m27b.act_quant(xs[c], m27b.Q8_K, out=xq[c])
            m27b.qmv(Ws[c], xq[c], 1, ys[c])
            yh[c].copy_(ys[c], non_blocking=True)

    # eager pass: validates the calls and warms per-kernel state before capture
    step_e2e()
    torch.cuda.synchronize()

    def capture(fn, n):
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for _ in range(n):
                    fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        return g

    graphs = {}

    def run_steps(fn, n):
        full, rem = divmod(n, GRAPH_STEPS)
        if full and (fn, GRAPH_STEPS) not in graphs:
            graphs[(fn, GRAPH_STEPS)] = capture(fn, GRAPH_STEPS)
        if rem and (fn, rem) not in graphs:
            graphs[(fn, rem)] = capture(fn, rem)
        for _ in range(full):
            graphs[(fn, GRAPH_STEPS)].replay()
        if rem:
            graphs[(fn, rem)].replay()

    def timed(fn, steps, warmup, sampler=None):
        run_steps(fn, warmup)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        if sampler:
            sampler.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run_steps(fn, steps)
        e1.record()
        torch.cuda.synchronize()
        clocks = sampler.stop() if sampler else None
        barrier()
        ms = e0.elapsed_time(e1)
        if dist:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, clocks

    warm = max(3, args.warmup)
    # pre-capture all graphs outside the timed regions
    for fn in (step_dev, step_qmv_only, step_e2e):
        run_steps(fn, GRAPH_STEPS + (args.steps % GRAPH_STEPS))
    torch.cuda.synchronize()

    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    ms, clocks = timed(step_dev, args.steps, warm, ClockSampler(uuid))
    ms_k, _ = timed(step_qmv_only, args.steps, warm)
    ms_e2e, _ = timed(step_e2e, args.steps, warm)

    step_bytes = COPIES * MV_BYTES
    value = world * step_bytes * args.steps / (ms / 1e3) / 1e9
    e2e = world * step_bytes * args.steps / (ms_e2e / 1e3) / 1e9
    kern_us = ms_k * 1e3 / (args.steps * COPIES)
    achieved = MV_BYTES / (kern_us * 1e-6) / 1e9
    peak, peak_kind = measured_peak()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, reps, nrows, threads = cpu_oracle_gbs(host_w0, 10.0)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{reps} full cfg0 matvecs (17408x5120 q4_K . q8_K), OpenMP over rows"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4_K*q8_K int8 dp4a, f32 accumulate",
            "data": "synthetic (seeded random valid q4_K blocks, N(0,1) activations)",
            "config": {"workload": "cfg0: q4_K matvec 17408x5120, batch 1, q8_K activations", "rows": ROWS, "k": K,
                       "matvecs_per_step": COPIES, "bytes_per_matvec": MV_BYTES,
                       "l2": f"inputs larger than L2: {COPIES} rotating weight matrices ({COPIES * W_BYTES / 1e6:.0f} MB)",
                       "parallelism": f"replica x{world}", "pct_of_8TBps": round(100 * value / world / 8000, 1)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": ncu_traffic_per_launch(),
                         "kernel": "k_qmv<W_Q4K,1,STORE>", "mean_launch_us": round(kern_us, 3),
                         "peak_kind": peak_kind},
            "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": COPIES * X_BYTES,
                    "d2h_bytes_per_step": COPIES * Y_BYTES},
            "gpu_launches": 2 * COPIES * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    for g in graphs.values():
        del g
    graphs.clear()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
