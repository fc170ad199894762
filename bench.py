#!/usr/bin/env python
"""Benchmark: quantized weight-streaming matvec on B200, HBM GB/s.

Default workload (the driver's line) — cfg0, the q4_K matvec BASELINE's
metric is quoted on: one step = one pass of the matvec path over one batch:
for each of C=6 distinct q4_K weight matrices of 17408 x 5120 (6 x 50.1 MB =
301 MB rotate, so the working set exceeds the 126 MB L2), quantize a
5120-long fp32 activation to q8_K and multiply — one launch of
m27b_qmv_f32 (the reference's l_mv_quant seam), whose kernel quantizes the
activation in its prologue.  Steps are replayed through CUDA graphs of the
C-ABI calls, timed with CUDA events on the launching stream, bracketed by a
barrier and a synchronize.

  value    algorithmic bytes of all ranks' steps / max-over-ranks time; a
           matvec's algorithmic bytes are W 50,135,040 + x 20,480 + y 69,632.
  e2e      the same through the C ABI with host buffers: per matvec a pinned
           host->device copy of x and a device->host copy of y are inside the
           timed region, on a copy stream beside the kernels (the inputs go
           out at the start of the step, each result comes back while the
           next matvec computes).
  roofline the step's kernel (for cfg0 the step is that one kernel; for
           cfg2 the matvec without the separate quantizer): bytes per launch
           / mean launch time, against the measured HBM copy bandwidth in
           MEASURED_PEAKS.json.
  cpu_baseline  the CPU oracle (restatement of ggml's vec_dot_q4_K_q8_K,
           OpenMP over rows) on this host's cores, a bounded sample.

Other workloads (--workload, for profiling and the design notes; not the
driver's line): cfg1 = q6_K lm_head 248320 x 5120 with fused argmax; cfg3 =
the FFN block down(silu(gate.x) * up.x) with RMSNormed input.

--impl reference times the ggml-semantics CPU path on the same metric (the
reference has no CPU path of its own and its ggml dependency is absent).

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

Q8_0, Q4_K, Q6_K, Q8_K = 8, 12, 14, 15
BLOCK = {Q4_K: (256, 144), Q6_K: (256, 210), Q8_0: (32, 34)}
GRAPH_STEPS = 16
# read-probe copy shapes: (warps per CTA, copies in flight per warp, bytes per
# copy, CTAs per SM); the first is the matvec kernel's own (8 warps, two
# 4608-byte q4_K items each, two CTAs per SM)
PROBE_SHAPES = [(8, 2, 4608, 2), (8, 3, 4608, 2), (8, 3, 8192, 1), (4, 3, 8192, 2), (16, 2, 4096, 1),
                (8, 6, 4096, 1), (1, 6, 32768, 1), (2, 6, 16384, 1)]


def wbytes(qt, rows, k):
    be, bb = BLOCK[qt]
    return rows * (k // be) * bb


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None)
    p.add_argument("--warmup", type=int, default=200)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["cfg0", "cfg1", "cfg2", "cfg3", "decode", "spec"], default="cfg0")
    p.add_argument("--rows", type=int, default=None, help="override the row count (smaller profiling cases)")
    p.add_argument("--ntok", type=int, default=None, help="tokens per matvec (cfg2: 16, cfg3: 1)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-decode", action="store_true", help="skip the whole-model decode figures of the default line")
    p.add_argument("--prompt", type=int, default=512, help="decode: prompt tokens before generation")
    p.add_argument("--gen", type=int, default=256, help="decode: generated tokens (timed)")
    p.add_argument("--layers", type=int, default=64, help="decode: layers (64 = the Qwen-27B shape)")
    p.add_argument("--hybrid", action="store_true",
                   help="decode: the hybrid layout (every 4th layer attention, the rest Gated DeltaNet; 1 GPU)")
    p.add_argument("--k", type=int, default=7, help="spec: tokens the draft proposes per round")
    p.add_argument("--comm", choices=["p2p", "nccl"], default="p2p",
                   help="decode, N>1: fused NVLink all-reduce (p2p) or NCCL all-reduce")
    a = p.parse_args()
    if a.steps is None:
        a.steps = {"cfg0": 40000, "cfg1": 2000, "cfg2": 20000, "cfg3": 8000, "decode": a.gen, "spec": a.gen}[a.workload]
    if a.ntok is None:
        a.ntok = 16 if a.workload == "cfg2" else 1
    return a


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic_per_launch(name):
    """DRAM bytes per launch of the named kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", name)
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


# --------------------------------------------------------------------------
# workloads


class Workload:
    """A step made of C-ABI calls; bytes are the algorithmic bytes per step."""

    def __init__(self, args, dev, rank):
        import numpy as np
        import torch
        import m27b
        from _data import random_valid_blocks
        self.m27b, self.torch, self.dev = m27b, torch, dev
        gen = np.random.default_rng(7 + rank)
        w = args.workload
        self.name = w
        if w in ("cfg0", "cfg2"):
            n = args.ntok if w == "cfg2" else 1
            rows, k, copies = args.rows or 17408, 5120, 6
            self.host_w0 = random_valid_blocks(Q4_K, rows, k, 1000 * rank)
            self.W = [m27b.QWeight(self.host_w0 if c == 0 else random_valid_blocks(Q4_K, rows, k, 1000 * rank + c),
                                   Q4_K, k, rows) for c in range(copies)]
            # the step's activations in one buffer (one host->device copy per step)
            self.x_all = torch.from_numpy(gen.standard_normal((copies, n, k)).astype(np.float32)).to(dev)
            self.x = list(self.x_all.unbind(0))
            self.xq = [torch.empty(n * m27b.act_bytes(Q8_K, k), dtype=torch.uint8, device=dev) for _ in range(copies)]
            self.y = [torch.empty((n, rows), dtype=torch.float32, device=dev) for _ in range(copies)]
            self.mv_bytes = wbytes(Q4_K, rows, k) + n * (k * 4 + rows * 4)
            self.step_bytes = copies * self.mv_bytes
            self.n = n
            l2 = (f"inputs larger than L2: {copies} rotating weight matrices ({copies * wbytes(Q4_K, rows, k) / 1e6:.0f} "
                  "MB); the kernel-only timing (roofline.achieved) reads one activation buffer for the rotation, "
                  "L2-resident as in a decode step")
            if w == "cfg0":
                self.metric = "q4_K matvec HBM GB/s"
                self.config = {"workload": f"cfg0: q4_K matvec {rows}x{k}, batch 1, q8_K activations", "rows": rows,
                               "k": k, "matvecs_per_step": copies, "bytes_per_matvec": self.mv_bytes, "l2": l2,
                               "data": (f"W: seeded random valid q4_K blocks (seeds {1000 * rank}..{1000 * rank + 5}, "
                                        f"d/dmin for sigma ~0.02); x: N(0,1), seed {7 + rank}.  The kernel has no "
                                        "data-dependent branch; BASELINE's Gaussian-quantized cfg0 (W seed 0, x seed 1) "
                                        "is the full-size parity test")}
                self.kernel = "k_qmv_q4k_blk<1,STORE> (q8_K quantization in the prologue)"
                self.profile = "qmv_q4K_cfg0.md"
            else:
                self.metric = f"q4_K verify matvec HBM GB/s ({n} tokens)"
                self.config = {"workload": f"cfg2: q4_K matvec {rows}x{k}, {n} tokens per matvec, q8_K activations",
                               "rows": rows, "k": k, "ntok": n, "matvecs_per_step": copies,
                               "bytes_per_matvec": self.mv_bytes, "l2": l2,
                               "int_ops_per_matvec": 2 * rows * k * n}
                self.kernel = ("k_qmv_q4k_mma<%d> (tcgen05 kind::i8, K split across CTAs: m27b_qmv_mma_split, "
                               "the verify pass's entry)" % (8 if n <= 8 else 16)) if n >= 5 else \
                    "k_qmv_q4k_blk<%d,STORE>" % n
                self.profile = "qmv_q4K_mma_cfg2.md"
                if n >= 5:
                    L = m27b.lib()
                    self.split = [(torch.empty(L.m27b_qmv_mma_split_part_bytes(m27b.ctypes.byref(W.view), n),
                                               dtype=torch.uint8, device=dev),
                                   torch.zeros(L.m27b_qmv_mma_split_count_bytes(m27b.ctypes.byref(W.view)),
                                               dtype=torch.uint8, device=dev)) for W in self.W]
            self.fused = w == "cfg0"  # quantize in the matvec prologue (m27b_qmv_f32)
            self.launches_per_step = copies if self.fused else 2 * copies
            self.copies, self.rows, self.k = copies, rows, k
            self.h2d = copies * n * k * 4
            self.d2h = copies * n * rows * 4
        elif w == "cfg1":
            rows, k = args.rows or 248320, 5120
            self.W = [m27b.QWeight(random_valid_blocks(Q6_K, rows, k, 2 + 1000 * rank), Q6_K, k, rows)]
            self.x = [torch.from_numpy(gen.standard_normal((1, k)).astype(np.float32)).to(dev)]
            self.xq = [torch.empty(m27b.act_bytes(Q8_K, k), dtype=torch.uint8, device=dev)]
            self.y = [torch.empty((1, rows), dtype=torch.float32, device=dev)]
            self.best = torch.empty(1, dtype=torch.int64, device=dev)
            self.mv_bytes = wbytes(Q6_K, rows, k) + k * 4 + rows * 4
            self.step_bytes = self.mv_bytes
            self.metric = "q6_K lm_head matvec+argmax HBM GB/s"
            self.config = {"workload": f"cfg1: q6_K lm_head {rows}x{k} with fused argmax, batch 1", "rows": rows, "k": k,
                           "l2": f"inputs larger than L2: {wbytes(Q6_K, rows, k) / 1e6:.0f} MB of weights"}
            self.kernel = "k_qmv_q6k_tile<1,ARGMAX>"
            self.profile = "qmv_q6K_lm_head.md"
            self.launches_per_step = 2
            self.copies, self.rows, self.k = 1, rows, k
            self.h2d, self.d2h = k * 4, rows * 4 + 8
            self.n = 1
        else:  # cfg3
            H, F, n = 5120, args.rows or 17408, args.ntok
            self.sets = []
            for c in range(2):
                G = m27b.QWeight(random_valid_blocks(Q4_K, F, H, 10 + 3 * c + 1000 * rank), Q4_K, H, F)
                U = m27b.QWeight(random_valid_blocks(Q4_K, F, H, 11 + 3 * c + 1000 * rank), Q4_K, H, F)
                D = m27b.QWeight(random_valid_blocks(Q6_K, H, F, 12 + 3 * c + 1000 * rank), Q6_K, F, H)
                self.sets.append((G, U, D))
            self.h = [torch.from_numpy(gen.standard_normal((n, H)).astype(np.float32)).to(dev) for _ in range(2)]
            self.hq = torch.empty(n * m27b.act_bytes(Q8_K, H), dtype=torch.uint8, device=dev)
            self.a = torch.empty((n, F), dtype=torch.float32, device=dev)
            self.aq = torch.empty(n * m27b.act_bytes(Q8_K, F), dtype=torch.uint8, device=dev)
            self.out = [torch.empty((n, H), dtype=torch.float32, device=dev) for _ in range(2)]
            self.n, self.H, self.F = n, H, F
            self.mv_bytes = 2 * wbytes(Q4_K, F, H) + wbytes(Q6_K, H, F) + n * (H * 4 * 2 + F * 4 * 2)
            self.step_bytes = 2 * self.mv_bytes
            self.metric = "q4_k_m FFN block HBM GB/s"
            self.config = {"workload": f"cfg3: FFN block gate/up {F}x{H} q4_K, down {H}x{F} q6_K, {n} token(s)",
                           "hidden": H, "ffn": F, "ntok": n, "l2": "inputs larger than L2: 2 rotating FFN weight sets "
                           f"({2 * (2 * wbytes(Q4_K, F, H) + wbytes(Q6_K, H, F)) / 1e6:.0f} MB)"}
            self.kernel = "k_qmv_q4k_blk<n,SWIGLU> + k_qmv_q6k_tile<n,STORE>"
            self.profile = "ffn_block_cfg3.md"
            self.launches_per_step = 8
            self.copies = 2
            self.hh = [x.cpu().pin_memory() for x in self.h]
            self.oh = [torch.empty((n, H), dtype=torch.float32).pin_memory() for _ in range(2)]
            self.h2d, self.d2h = 2 * n * H * 4, 2 * n * H * 4
            self.n = n
        if w in ("cfg0", "cfg2"):
            self.xh_all = self.x_all.cpu().pin_memory()
        if w in ("cfg0", "cfg1", "cfg2"):
            self.xh = [x.cpu().pin_memory() for x in self.x]
            self.yh = [torch.empty_like(y, device="cpu").pin_memory() for y in self.y]

    def _mv(self, c, xc=None):
        m = self.m27b
        xq = self.xq[c if xc is None else xc]
        if self.name == "cfg1":
            m.qmv_argmax(self.W[c], xq, 1, self.best, logits=self.y[c])
        elif getattr(self, "split", None):
            part, count = self.split[c]
            m.qmv_mma_split(self.W[c], xq, self.n, self.y[c], part=part, count=count)
        else:
            m.qmv(self.W[c], xq, self.n, self.y[c])

    def step(self):
        m = self.m27b
        if self.name == "cfg3":
            for c in range(2):
                self._ffn(c)
            return
        for c in range(self.copies):
            if getattr(self, "fused", False):
                m.qmv_f32(self.W[c], self.x[c], self.n, self.y[c])
                continue
            m.act_quant(self.x[c], Q8_K, out=self.xq[c])
            self._mv(c)

    def _ffn(self, c):
        m = self.m27b
        G, U, D = self.sets[c]
        m.act_quant(self.h[c], Q8_K, out=self.hq, eps=1e-6)
        m.qmv_swiglu(G, U, self.hq, self.n, self.a)
        m.act_quant(self.a, Q8_K, out=self.aq)
        m.qmv(D, self.aq, self.n, self.out[c])

    def kernel_only(self):
        if self.name == "cfg3":
            m = self.m27b
            for c in range(2):
                G, U, D = self.sets[c]
                m.qmv_swiglu(G, U, self.hq, self.n, self.a)
                m.qmv(D, self.aq, self.n, self.out[c])
            return
        # the kernel alone, as a decode step runs it: its activations are the
        # ones the previous kernel just wrote (L2-resident), here one buffer
        # the rotation shares; the weights stream from HBM (6 rotating copies)
        for c in range(self.copies):
            if getattr(self, "fused", False):
                self.m27b.qmv_f32(self.W[c], self.x[0], self.n, self.y[c])
            else:
                self._mv(c, xc=0)

    def step_e2e(self):
        if self.name == "cfg3":
            for c in range(2):
                self.h[c].copy_(self.hh[c], non_blocking=True)
                self._ffn(c)
                self.oh[c].copy_(self.out[c], non_blocking=True)
            return
        # the host copies run on a copy stream beside the kernels, as a
        # serving loop overlaps them: the step's activations go to the device
        # in one copy at its start (cfg0/cfg2: one pinned buffer; cfg1 has
        # one activation), and the copy of y[c] back to the host runs while
        # matvec c+1 computes; the step ends when the last result is on the
        # host
        torch = self.torch
        cur = torch.cuda.current_stream()
        if not hasattr(self, "copy_st"):
            self.copy_st = torch.cuda.Stream()
            self.ev_in = torch.cuda.Event()
            self.ev_out = [torch.cuda.Event() for _ in range(self.copies)]
        cs = self.copy_st
        cs.wait_stream(cur)
        with torch.cuda.stream(cs):
            if hasattr(self, "xh_all"):
                self.x_all.copy_(self.xh_all, non_blocking=True)
            else:
                for c in range(self.copies):
                    self.x[c].copy_(self.xh[c], non_blocking=True)
            self.ev_in.record(cs)
        cur.wait_event(self.ev_in)
        for c in range(self.copies):
            if getattr(self, "fused", False):
                self.m27b.qmv_f32(self.W[c], self.x[c], self.n, self.y[c])
            else:
                self.m27b.act_quant(self.x[c], Q8_K, out=self.xq[c])
                self._mv(c)
            self.ev_out[c].record(cur)
            cs.wait_event(self.ev_out[c])
            with torch.cuda.stream(cs):
                self.yh[c].copy_(self.y[c], non_blocking=True)
        cur.wait_stream(cs)

    def kernel_bytes(self):
        return self.step_bytes / (1 if self.name == "cfg3" else self.copies)

    def kernel_launches(self):
        # cfg3: the step's matvec kernels are timed as one unit
        return 1 if self.name == "cfg3" else self.copies


# --------------------------------------------------------------------------
# whole-model decode (cfg4): the engine's tensor-parallel greedy decode


def decode_bench(args, world, rank, dev, dist, uuid):
    """Qwen-27B-shaped synthetic model (seeded random valid q4_K / q6_K blocks,
    norms 1), tensor-parallel over `world` ranks.  The prompt is fed token by
    token (untimed), then args.gen tokens are generated twice from the same
    state: on the device (m27b_engine_generate: graph replays with no host
    round trip) and through m27b_engine_decode_step (one host call per token:
    16 B host->device, 8 B device->host).  Both are timed with CUDA events on
    the engine's stream, max over ranks; the two token sequences must agree."""
    import numpy as np
    import torch
    import m27b
    hybrid = bool(getattr(args, "hybrid", False))
    if hybrid and world > 1:
        raise SystemExit("--hybrid runs on one GPU")
    cfg = m27b.model_config(max_ctx=args.prompt + args.gen + 8, tp_rank=rank, tp_size=world, n_layers=args.layers,
                            **(m27b.HYBRID if hybrid else {}))
    e = m27b.Engine(cfg)
    try:
        if world > 1:
            uid = torch.zeros(128, dtype=torch.uint8, device=dev)
            if rank == 0:
                uid.copy_(torch.frombuffer(bytearray(m27b.nccl_unique_id()), dtype=torch.uint8))
            dist.broadcast(uid, 0)
            e.set_nccl(bytes(uid.cpu().numpy()))
            if args.comm == "p2p":
                e.enable_p2p()
        t0 = time.perf_counter()
        e.random_weights(seed=0, sigma=0.02)
        t_load = time.perf_counter() - t0
        prompt = np.random.default_rng(4).integers(0, cfg.vocab, args.prompt)

        def feed():
            # the prompt, token by token (untimed); a hybrid model's DeltaNet
            # state starts over, attention positions are simply rewritten
            if hybrid:
                e.reset()
            for pos in range(args.prompt - 1):
                e.decode_step(int(prompt[pos]), pos)

        feed()
        start, p0 = int(prompt[-1]), args.prompt - 1
        st = torch.cuda.ExternalStream(e.stream(), device=dev)
        warm = max(3, min(args.warmup, 16))
        e.generate(start, p0, warm)  # warm-up (rewritten by the timed runs)
        if hybrid:
            feed()

        def timed(fn, sampler=None):
            torch.cuda.synchronize()
            if dist:
                dist.barrier()
            torch.cuda.synchronize()
            if sampler:
                sampler.start()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            out = fn()
            b.record(st)
            b.synchronize()
            clk = sampler.stop() if sampler else None
            ms = a.elapsed_time(b)
            if dist:
                t = torch.tensor([ms], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            return ms, out, clk

        ms, gen, clocks = timed(lambda: e.generate(start, p0, args.gen), ClockSampler(uuid))
        if hybrid:
            feed()

        def host_loop():
            tok, out = start, []
            for i in range(args.gen):
                tok = e.decode_step(tok, p0 + i)
                out.append(tok)
            return out

        ms_e2e, gen_e2e, _ = timed(host_loop)
        # speculative verification: one pass over n drafted tokens (tensor cores for the q4_K matrices)
        verify = {}
        if not hybrid:
            vt = [int(t) for t in np.random.default_rng(5).integers(0, cfg.vocab, 16)]
            for n in (8, 16):
                e.verify(vt[:n], p0)  # capture
                reps = 5
                vms, _, _ = timed(lambda: [e.verify(vt[:n], p0) for _ in range(reps)])
                verify[str(n)] = {"ms_per_pass": round(vms / reps, 4), "tokens_per_s": round(n * reps / (vms / 1e3), 1)}
        wb = e.weight_bytes_per_token()
        n_attn = sum((l + 1) % 4 == 0 for l in range(args.layers)) if hybrid else args.layers
        kv_bytes = 2 * n_attn * (p0 + 1 + args.gen / 2) * e_kv_heads(cfg) * cfg.head_dim * 4
        tps = args.gen / (ms / 1e3)
        peak, peak_kind = measured_peak()
        per_rank_gbs = wb * tps / 1e9
        return {
            "tokens_per_s": round(tps, 2), "ms_per_token": round(ms / args.gen, 4), "tp": world,
            "e2e_tokens_per_s": round(args.gen / (ms_e2e / 1e3), 2),
            "weight_bytes_per_token_per_rank": wb, "kv_bytes_per_token_per_rank": int(kv_bytes),
            "weight_gbs_per_rank": round(per_rank_gbs, 1), "weight_gbs_total": round(per_rank_gbs * world, 1),
            "roofline_frac": round(per_rank_gbs / peak, 4), "peak_gbs": peak, "peak_kind": peak_kind,
            "tokens_match": list(map(int, gen)) == list(map(int, gen_e2e)),
            "verify": verify,
            "hybrid": (dict(m27b.HYBRID, deltanet_layers=sum((l + 1) % 4 != 0 for l in range(args.layers)))
                       if hybrid else None),
            "layers": args.layers, "prompt": args.prompt, "gen": args.gen, "weights_init_s": round(t_load, 1),
            "allreduce": "none" if world == 1 else ("fused NVLink push (P2P stores + release flags)" if args.comm == "p2p"
                                                   else "NCCL all-reduce"),
            "clocks": clocks,
        }
    finally:
        e.close()


def decode_launches_per_token(layers, p2p, hybrid):
    """This library's kernel launches in one decode step (NCCL's own kernels
    not counted).  Per attention layer: the qkv projection (RMSNorm + q8_K in
    its prologue), the two attention kernels (norm/RoPE/KV append/split
    attention; reduction + gate + q8_K), o_proj, gate/up (SwiGLU and the
    down projection's q8_K input in its epilogue), down = 6; with the fused
    NVLink all-reduce, o_proj and down push into the peers' windows and a
    consumer kernel follows each = 8.  Per DeltaNet layer (one GPU): RMSNorm,
    three projections, conv, delta rule, ssm_out, gate/up, down = 9.  Per
    step: the embedding row, the rotary table, the output RMSNorm + q8_K
    (before the first layer's projection with the fused all-reduce), lm_head
    + argmax, the token/position advance = 5."""
    n_attn = sum((l + 1) % 4 == 0 for l in range(layers)) if hybrid else layers
    return (8 if p2p else 6) * n_attn + 9 * (layers - n_attn) + 5


def decode_main(args, world, rank, dev, dist, uuid, tp_parity=None):
    """--workload decode: the decode figures as the line's own metric."""
    import m27b
    d = decode_bench(args, world, rank, dev, dist, uuid)
    if rank == 0:
        line = {
            "metric": "decode tokens/s", "value": d["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.gen, "warmup": max(3, min(args.warmup, 16)), "ms_per_step": d["ms_per_token"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "q4_K/q6_K * q8_K, int8 dp4a, f32 accumulate; fp32 KV cache",
            "data": "synthetic (seeded random valid q4_K/q6_K blocks, random 512-token prompt, seed 4)",
            "config": {"workload": f"cfg4: {args.layers}-layer Qwen-27B-shaped decode, TP={world}, "
                                   f"{args.prompt}-token prompt, {args.gen} generated tokens",
                       "parallelism": f"tp{world}", "l2": "weights per token >> L2 (16 GB / TP)"},
            "roofline": {"bound": "hbm", "achieved": d["weight_gbs_per_rank"], "peak": d["peak_gbs"], "unit": "GB/s",
                         "frac": d["roofline_frac"], "traffic": None, "kernel": "whole decode step (weight bytes / time)",
                         "peak_kind": d["peak_kind"]},
            "e2e": {"value": d["e2e_tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 8},
            "gpu_launches": decode_launches_per_token(args.layers, world > 1 and args.comm == "p2p",
                                                      bool(getattr(args, "hybrid", False))) * args.gen,
            "clocks": d["clocks"], "cpu_baseline": None,
            "device_status": m27b.device_status(clear=True), "decode": d, "tp_parity": tp_parity,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if tp_parity is None or tp_parity["pass"] else 1


# --------------------------------------------------------------------------
# tensor-parallel self-check (every N > 1 run, before anything is timed)

TP_PARITY_CFG = dict(n_layers=2, hidden=512, ffn=2048, n_head=8, n_kv_head=2, head_dim=256, vocab=1001, n_rot=64,
                     rope_theta=1e7, rms_eps=1e-6)
TP_PARITY_TOKENS = [7, 500, 3, 44, 999, 0, 123, 64]
TP_PARITY_TOL = 1e-3  # relative L2 of the hidden state, TP=N against TP=1


def _tp_trace(cfg_kw, rank, world, dist, dev, comm):
    """Hidden state and greedy token after every step of TP_PARITY_TOKENS,
    teacher-forced, on a small model with seeded weights generated on the
    device in global coordinates (the same tensors at every tp_size)."""
    import numpy as np
    import torch
    import m27b
    e = m27b.Engine(m27b.model_config(max_ctx=len(TP_PARITY_TOKENS) + 4, tp_rank=rank, tp_size=world, **cfg_kw))
    try:
        if world > 1:
            uid = torch.zeros(128, dtype=torch.uint8, device=dev)
            if rank == 0:
                uid.copy_(torch.frombuffer(bytearray(m27b.nccl_unique_id()), dtype=torch.uint8))
            dist.broadcast(uid, 0)
            e.set_nccl(bytes(uid.cpu().numpy()))
            if comm == "p2p":
                e.enable_p2p()
        e.random_weights(seed=11, sigma=0.02)
        hid, toks = [], []
        for pos, t in enumerate(TP_PARITY_TOKENS):
            toks.append(e.decode_step(t, pos))
            hid.append(e.hidden())
        return np.array(hid), np.array(toks)
    finally:
        e.close()


def tp_parity_check(world, rank, dev, dist):
    """Decode the small model at TP=world with the fused NVLink all-reduce and
    with NCCL, and on rank 0 at TP=1 (one GPU, no exchange): the replicated
    hidden states must agree within TP_PARITY_TOL and every rank must return
    the same tokens as TP=1.  (The TP=1 engine itself is held to the CPU
    oracle by the GPU test suite.)  Returns the summary every rank agrees on."""
    import numpy as np
    import torch
    import m27b
    d = dict(m27b.QWEN27)
    d.update(TP_PARITY_CFG)
    ref = _tp_trace(d, 0, 1, None, dev, None) if rank == 0 else None
    out = {}
    ok_all = True
    for comm in ("p2p", "nccl"):
        hid, toks = _tp_trace(d, rank, world, dist, dev, comm)
        # every rank's tokens and hidden states must equal rank 0's
        t = torch.from_numpy(toks.astype(np.int64)).to(dev)
        tmax, tmin = t.clone(), t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(tmin, op=dist.ReduceOp.MIN)
        ranks_agree = bool(torch.equal(tmax, tmin))
        h = torch.from_numpy(hid.astype(np.float32)).to(dev)
        hmax, hmin = h.clone(), h.clone()
        dist.all_reduce(hmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(hmin, op=dist.ReduceOp.MIN)
        ranks_agree = ranks_agree and bool(torch.equal(hmax, hmin))
        res = torch.zeros(3, dtype=torch.float64, device=dev)
        if rank == 0:
            rel = max(float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)) for a, b in zip(hid, ref[0]))
            res[0] = rel
            res[1] = float((toks == ref[1]).all())
            res[2] = float(ranks_agree)
        dist.broadcast(res, 0)
        rel, teq, agree = float(res[0]), bool(res[1] > 0.5), bool(res[2] > 0.5) and ranks_agree
        passed = rel <= TP_PARITY_TOL and teq and agree
        ok_all = ok_all and passed
        out[comm] = {"max_rel_l2": rel, "tokens_equal": teq, "ranks_agree": agree, "pass": passed}
    out["tol"] = TP_PARITY_TOL
    out["model"] = dict(TP_PARITY_CFG, steps=len(TP_PARITY_TOKENS), reference="TP=1 on rank 0's GPU")
    out["pass"] = ok_all
    return out


# --------------------------------------------------------------------------
# speculative decoding (cfg4 target + q8_0 draft), one GPU


def spec_main(args, dev, uuid):
    """--workload spec: the 64-layer target and the BASELINE cfg4 q8_0 draft
    (28 layers, hidden 1024, FFN 3072), seeded random weights, 512-token
    prompt.  Measured with CUDA events on the engines' streams: the target's
    plain greedy decode, the draft's generation per token, the target's verify
    pass of k + 1 tokens, and the whole speculative loop
    (m27b_engine_speculative_generate, C++) with this draft.  Random weights
    give two unrelated models, so the measured acceptance is ~0; the line also
    gives the tokens/s the measured costs imply at acceptance rates a trained
    draft reaches (expected tokens per round (1 - a^(k+1)) / (1 - a), one
    round = k draft tokens + one verify pass)."""
    import numpy as np
    import torch
    import m27b
    k = args.k
    ctx = args.prompt + args.gen + 2 * k + 8
    tc = m27b.model_config(max_ctx=ctx, n_layers=args.layers)
    d = dict(m27b.DRAFT)
    dc = m27b.model_config(max_ctx=ctx, **d)
    target, draft = m27b.Engine(tc), m27b.Engine(dc)
    try:
        target.random_weights(seed=0, sigma=0.02)
        draft.random_weights(seed=1, sigma=0.02)
        prompt = [int(t) for t in np.random.default_rng(4).integers(0, tc.vocab, args.prompt)]
        sts = [torch.cuda.ExternalStream(e.stream(), device=dev) for e in (target, draft)]

        def timed(fn):
            torch.cuda.synchronize()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in sts]
            for (a, _), s in zip(evs, sts):
                a.record(s)
            t0 = time.perf_counter()
            out = fn()
            host_ms = (time.perf_counter() - t0) * 1e3
            for (_, b), s in zip(evs, sts):
                b.record(s)
            torch.cuda.synchronize()
            return out, host_ms, [a.elapsed_time(b) for a, b in evs]

        def feed(e, n):
            for pos in range(n):
                e.decode_step(prompt[pos], pos)

        p0 = args.prompt - 1
        feed(target, p0)
        feed(draft, p0)
        target.generate(prompt[-1], p0, 4)  # warm-up (graphs captured; rewritten below)
        draft.generate(prompt[-1], p0, 4)
        _, _, (t_ms, _) = timed(lambda: target.generate(prompt[-1], p0, args.gen))
        _, _, (_, d_ms) = timed(lambda: draft.generate(prompt[-1], p0, args.gen))
        vt = [prompt[-1]] + [int(t) for t in np.random.default_rng(5).integers(0, tc.vocab, k)]
        target.verify(vt, p0)  # capture
        reps = 5
        _, _, (v_ms, _) = timed(lambda: [target.verify(vt, p0) for _ in range(reps)])
        v_ms /= reps
        # the whole loop from an empty cache, prompt included (the prompt's
        # share is reported apart, from the loop's own host clocks)
        (toks, st), host_ms, _ = timed(lambda: m27b.speculative_generate(target, draft, prompt, args.gen, k=k))
        loop_ms = st["draft_ms"] + st["verify_ms"]
        spec_tps = args.gen / (loop_ms / 1e3)
        plain_tps = args.gen / (t_ms / 1e3)
        d_tok = d_ms / args.gen
        proj = {}
        for a in (0.5, 0.7, 0.8, 0.9):
            per_round = (1 - a ** (k + 1)) / (1 - a)
            proj[str(a)] = round(per_round / ((k * d_tok + v_ms) / 1e3), 1)
        line = {
            "metric": "speculative decode tokens/s", "value": round(spec_tps, 2), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.gen, "warmup": 4, "ms_per_step": round(loop_ms / args.gen, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "target q4_K/q6_K, draft q8_0, * q8_K / q8_0 activations, f32 accumulate",
            "data": "synthetic (seeded random valid blocks for both models: unrelated, acceptance ~0)",
            "config": {"workload": f"cfg4 speculative: {args.layers}-layer target + 28-layer q8_0 draft "
                                   f"(hidden 1024, FFN 3072), k={k}, {args.prompt}-token prompt, {args.gen} tokens",
                       "k": k, "parallelism": "tp1"},
            "spec": {"acceptance": round(st["accepted"] / max(1, st["proposed"]), 4), "rounds": st["iterations"],
                     "loop_host_ms": round(loop_ms, 2), "prefill_host_ms": round(st["prefill_ms"], 1),
                     "target_plain_tokens_per_s": round(plain_tps, 2), "target_ms_per_token": round(t_ms / args.gen, 4),
                     "draft_ms_per_token": round(d_tok, 4), "draft_tokens_per_s": round(args.gen / (d_ms / 1e3), 1),
                     "verify_ms_per_pass": round(v_ms, 4), "verify_tokens": k + 1,
                     "verify_over_step": round(v_ms / (t_ms / args.gen), 3),
                     "projected_tokens_per_s_at_acceptance": proj,
                     "draft_weight_bytes_per_token": draft.weight_bytes_per_token()},
            "e2e": {"value": round(args.gen / (host_ms / 1e3), 2), "unit": "tokens/s (prompt feeding included)",
                    "h2d_bytes_per_step": 4 * (k + 1), "d2h_bytes_per_step": 4 * (2 * k + 1)},
            "device_status": m27b.device_status(clear=True), "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
        return 0 if line["device_status"] == 0 else 1
    finally:
        target.close()
        draft.close()


def e_kv_heads(cfg):
    import m27b
    return m27b.partition(cfg).n_kv


def cpu_oracle_gbs(w_host, k, seconds, nthreads=0):
    """GB/s of the CPU q4_K.q8_K matvec on w_host (rows x row bytes): the
    vectorised restatement of ggml's x86 path (AVX-512 VNNI or AVX2, bit for
    bit the scalar oracle's results), OpenMP over rows on all host threads.
    Returns (GB/s, full matvecs timed, threads, instruction set)."""
    from oracle import oracle as orc
    from _data import gauss_act
    n = w_host.shape[0]
    xq = orc.quantize_q8_K(gauss_act(1, k, 1))
    _, level = orc.matvec_q4K_simd(w_host, k, xq, nthreads)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        orc.matvec_q4K_simd(w_host, k, xq, nthreads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds and reps >= 3:
            break
    bytes_per = wbytes(Q4_K, n, k) + k * 4 + n * 4
    return bytes_per * reps / el / 1e9, reps, (nthreads or orc.max_threads()), orc.SIMD_NAMES[level]


def reference_gpu_leg(steps=20, warmup=5):
    """The reference executor's own q8_1 quantizer + dp4a matvec kernels,
    compiled for sm_100a from the reference checkout (oracle/_ref/, a
    comparison arm), timed on this GPU the way the GPU arm is timed: cfg0
    (6 rotating 17408 x 5120 q4_K matrices, one quantize + matvec each, CUDA
    graph, CUDA events), plus the q6_K lm_head (cfg1 shape) and ffn_down
    shapes.  None without a GPU or without the built harness."""
    try:
        import torch
        from oracle import ref_gpu
        if not torch.cuda.is_available() or not ref_gpu.available():
            return None
    except Exception:
        return None
    from _data import random_valid_blocks
    import numpy as np
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    out = {"kernels": "k_quant_q8_1 + k_q4k_mv_q8_dp4a / k_q6k_mv_q8_dp4a (reference src/mono27b_executor.cu, "
                      "sm_100a, --use_fast_math)"}

    def run(qtype, rows, k, copies):
        be = 256
        rb = k // be
        Ws = [torch.from_numpy(random_valid_blocks(qtype, rows, k, 100 + c).reshape(-1)).to(dev) for c in range(copies)]
        xs = [torch.from_numpy(np.random.default_rng(7 + c).standard_normal(k).astype(np.float32)).to(dev)
              for c in range(copies)]
        q8 = [torch.empty(ref_gpu.q8_1_bytes(k), dtype=torch.uint8, device=dev) for _ in range(copies)]
        ys = [torch.empty(rows, dtype=torch.float32, device=dev) for _ in range(copies)]
        s = torch.cuda.Stream()

        def step(kernel_only=False):
            h = s.cuda_stream
            for c in range(copies):
                if not kernel_only:
                    ref_gpu.quant_q8_1(xs[c].data_ptr(), q8[c].data_ptr(), k, h)
                ref_gpu.matvec(qtype, Ws[c].data_ptr(), q8[c].data_ptr(), ys[c].data_ptr(), rb, rows, h)

        res = {}
        for ko in (False, True):
            with torch.cuda.stream(s):
                step(ko)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    step(ko)
            for _ in range(warmup):
                g.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(steps):
                g.replay()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / steps
            mv_bytes = rows * rb * (144 if qtype == Q4_K else 210) + k * 4 + rows * 4
            res["kernel_gbs" if ko else "gbs"] = round(copies * mv_bytes / (ms / 1e3) / 1e9, 1)
            if ko:
                res["matvec_us"] = round(ms * 1e3 / copies, 2)
            del g
        return res

    peak, _ = measured_peak()
    r = run(Q4_K, 17408, 5120, 6)
    r["frac_of_peak"] = round(r["kernel_gbs"] / peak, 4)
    out["cfg0_q4K_17408x5120"] = r
    out["q6K_ffn_down_5120x17408"] = run(Q6_K, 5120, 17408, 4)
    out["q6K_lm_head_248320x5120"] = run(Q6_K, 248320, 5120, 1)
    torch.cuda.synchronize()
    return out


REF_TIMED_S = 10.0   # CPU seconds the reference arm's timed steps add up to
REF_WARM_S = 2.0


def run_reference(args, world, rank):
    """CPU reference arm: the ggml-semantics CPU path (vectorised q4_K.q8_K,
    all host threads) on cfg0.  Each step runs `reps` full 17408 x 5120
    matvecs, sized from a calibration so that the K timed steps add up to
    about REF_TIMED_S seconds (warm-up steps about REF_WARM_S), the same
    amount of work per second as the cpu_baseline leg of the GPU arm."""
    if rank != 0:
        return 0
    from oracle import oracle as orc
    from _data import gauss_act, random_valid_blocks
    rows, k = args.rows or 17408, 5120
    w = random_valid_blocks(Q4_K, rows, k, 0)
    threads = orc.max_threads()
    xq = orc.quantize_q8_K(gauss_act(1, k, 1))
    _, level = orc.matvec_q4K_simd(w, k, xq)
    t0 = time.perf_counter()
    n_cal = 0
    while time.perf_counter() - t0 < 1.0 or n_cal < 3:
        orc.matvec_q4K_simd(w, k, xq)
        n_cal += 1
    full = (time.perf_counter() - t0) / n_cal
    reps = max(1, int(round(REF_TIMED_S / max(1, args.steps) / full)))
    warm_reps = max(1, int(round(REF_WARM_S / max(1, args.warmup) / full)))
    for _ in range(args.warmup):
        for _ in range(warm_reps):
            orc.matvec_q4K_simd(w, k, xq)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(reps):
            orc.matvec_q4K_simd(w, k, xq)
    el = time.perf_counter() - t0
    step_bytes = reps * (wbytes(Q4_K, rows, k) + k * 4 + rows * 4)
    gbs = step_bytes * args.steps / el / 1e9
    sample = (f"{reps} full cfg0 matvecs ({rows}x{k} q4_K . q8_K) per step, {args.steps} steps = "
              f"{el:.1f} s timed, {orc.SIMD_NAMES[level]}, OpenMP over rows")
    line = {
        "impl": "reference", "metric": "q4_K matvec HBM GB/s", "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4_K*q8_K int32->f32",
        "data": "synthetic (seeded random valid q4_K blocks, seed 0; x N(0,1) seed 1)",
        "config": {"workload": f"cfg0: q4_K matvec {rows}x{k}, batch 1", "rows": rows, "k": k,
                   "matvecs_per_step": reps},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("CPU restatement of ggml's vec_dot_q4_K_q8_K in its x86 SIMD form (bit for bit the scalar "
                 "restatement); ggml itself is absent from the reference checkout"),
        "reference_gpu": reference_gpu_leg(),
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    # stdout carries exactly one JSON line: NCCL's own log lines (e.g. its
    # version banner under NCCL_DEBUG=VERSION) go to stderr unless a log file is set
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import torch

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

    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    tp_parity = tp_parity_check(world, rank, dev, dist) if world > 1 else None
    if args.workload == "decode":
        return decode_main(args, world, rank, dev, dist, uuid, tp_parity)
    if args.workload == "spec":
        if world > 1:
            raise SystemExit("--workload spec runs on one GPU")
        return spec_main(args, dev, uuid)

    wl = Workload(args, dev, rank)
    # eager pass: validates the calls and warms per-kernel state before capture
    wl.step_e2e()
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
    # graphs are replayed, and timed, on a stream of their own (not the legacy
    # default stream)
    run_st = torch.cuda.Stream()

    def ensure_graphs(fn, n):
        full, rem = divmod(n, GRAPH_STEPS)
        if full and (fn, GRAPH_STEPS) not in graphs:
            graphs[(fn, GRAPH_STEPS)] = capture(fn, GRAPH_STEPS)
        if rem and (fn, rem) not in graphs:
            graphs[(fn, rem)] = capture(fn, rem)

    def run_steps(fn, n):
        ensure_graphs(fn, n)
        full, rem = divmod(n, GRAPH_STEPS)
        with torch.cuda.stream(run_st):
            for _ in range(full):
                graphs[(fn, GRAPH_STEPS)].replay()
            if rem:
                graphs[(fn, rem)].replay()

    def timed(fn, steps, warmup, sampler=None):
        ensure_graphs(fn, steps)  # no capture inside the timed region
        run_steps(fn, warmup)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        if sampler:
            sampler.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(run_st)
        run_steps(fn, steps)
        e1.record(run_st)
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
    for fn in (wl.step, wl.kernel_only, wl.step_e2e):  # capture every graph outside the timed regions
        run_steps(fn, GRAPH_STEPS + (args.steps % GRAPH_STEPS))
    torch.cuda.synchronize()

    ms, clocks = timed(wl.step, args.steps, warm, ClockSampler(uuid))
    ms_k, _ = timed(wl.kernel_only, args.steps, warm)
    ms_e2e, _ = timed(wl.step_e2e, args.steps, warm)

    value = world * wl.step_bytes * args.steps / (ms / 1e3) / 1e9
    e2e = world * wl.step_bytes * args.steps / (ms_e2e / 1e3) / 1e9
    kern_us = ms_k * 1e3 / (args.steps * wl.kernel_launches())
    achieved = wl.kernel_bytes() / (kern_us * 1e-6) / 1e9
    peak, peak_kind = measured_peak()
    status = wl.m27b.device_status(clear=True)
    wl_config, wl_metric, wl_profile, wl_kernel = wl.config, wl.metric, wl.profile, wl.kernel
    wl_h2d, wl_d2h, wl_launches = wl.h2d, wl.d2h, wl.launches_per_step

    # the read ceiling for launches of this size: the same bytes per launch
    # streamed into shared memory by bulk copies, nothing computed, same
    # rotation and graph structure; the fastest of several copy shapes
    probe = None
    if wl.name == "cfg0":
        bufs = [torch.empty(wbytes(Q4_K, wl.rows, wl.k), dtype=torch.uint8, device=dev) for _ in range(wl.copies)]
        shapes = []
        for shape in PROBE_SHAPES:
            fn = lambda shape=shape: [wl.m27b.hbm_read_probe(b, shape) for b in bufs]
            run_steps(fn, GRAPH_STEPS)
            pms, _ = timed(fn, args.steps, warm)
            us = pms * 1e3 / (args.steps * wl.copies)
            shapes.append({"shape": list(shape), "launch_us": round(us, 3),
                           "gbs": round(bufs[0].numel() / (us * 1e-6) / 1e9, 1)})
        best = max(shapes, key=lambda r: r["gbs"])
        probe = {"gbs": best["gbs"], "launch_us": best["launch_us"], "bytes_per_launch": bufs[0].numel(),
                 "shape": best["shape"], "shape_keys": "warps per CTA, copies in flight per warp, bytes per copy, "
                                                       "CTAs per SM",
                 "shapes": shapes,
                 "kernel": "m27b_hbm_read_probe_shape (bulk copies into shared memory, nothing computed)"}
        del bufs
        graphs.clear()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and wl.name == "cfg0":
        gbs, reps, threads, isa = cpu_oracle_gbs(wl.host_w0, wl.k, 10.0)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{reps} full cfg0 matvecs ({wl.rows}x{wl.k} q4_K . q8_K) in 10 s, {isa}, OpenMP over rows"}

    graphs.clear()
    decode = None
    if not args.no_decode and wl.name == "cfg0":
        del wl  # release the matvec workload's buffers before the model is loaded
        torch.cuda.empty_cache()
        decode = decode_bench(args, world, rank, dev, dist, uuid)

    if rank == 0:
        cfg = dict(wl_config)
        cfg["parallelism"] = f"replica x{world}"
        cfg["pct_of_8TBps"] = round(100 * value / world / 8000, 1)
        line = {
            "metric": wl_metric, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4_K/q6_K * q8_K, int8 dp4a, f32 accumulate",
            "data": "synthetic (seeded random valid k-quant blocks, N(0,1) activations)",
            "config": cfg,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": ncu_traffic_per_launch(wl_profile),
                         "traffic_source": f"profiles/{wl_profile} (dram__bytes_read.sum + dram__bytes_write.sum of "
                                           "one ncu capture of this kernel)",
                         "kernel": wl_kernel, "mean_launch_us": round(kern_us, 3), "peak_kind": peak_kind,
                         "read_probe": probe,
                         "frac_of_read_probe": round(achieved / probe["gbs"], 4) if probe else None},
            "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": wl_h2d, "d2h_bytes_per_step": wl_d2h},
            "gpu_launches": wl_launches * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "device_status": status,
            "decode": decode,
            "tp_parity": tp_parity,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if status == 0 and (tp_parity is None or tp_parity["pass"]) else 1


if __name__ == "__main__":
    sys.exit(main())
