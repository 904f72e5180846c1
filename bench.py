"""Benchmark of the WiSP decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl wisp|reference] [--bits 4]

Workload (``config.workload``): the bs=1 decode hot path of a Qwen3-30B-A3B-shaped model, 48 MoE layers
(H=2048, I=768, 128 experts, top-8, group 128), all 6144 packed experts resident in HBM (15.4 GB at
4 bit).  One step = one token through the 48 layers: RMSNorm with the residual add fused, then the
fused dequant+GEMV MoE (gate/up + SwiGLU, down, weighted combine) over that layer's seeded top-8.
Attention is not part of this workload; the metric is therefore reported as "moe decode tok/s".
Synthetic seeded data (weights N(0, 0.02), router logits N(0,1)); the per-token working set (962 MB
of expert bytes) is far larger than L2, so no flush is needed between steps.

One JSON line is printed by rank 0.  ``--impl reference`` times the CPU restatement of the reference
path (dequantize then fp32 matmul, the oracle) on the host cores on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "wisp-runtime_b200"))
sys.path.insert(0, ROOT)

H, I, E, K_TOP, L, G = 2048, 768, 128, 8, 48, 128
N_ROUTES = 16  # distinct seeded routings (tokens) cycled through by the timed steps
# dram__bytes_read.sum + dram__bytes_write.sum of one gate/up + one down launch (4-bit, this shape),
# from the ncu capture summarised in profiles/moe_decode_q4_qwen3_gate_up_down_full.md
NCU_TRAFFIC_PER_CALL = 13_405_696 + 6_746_368


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="wisp", choices=["wisp", "reference"])
    ap.add_argument("--bits", type=int, default=4, choices=[4, 3, 2])
    ap.add_argument("--layers", type=int, default=48, help="MoE layers (48 = the model; fewer = a small ncu case)")
    a = ap.parse_args()
    global L
    L = a.layers
    return a


def metric_name():
    return "moe decode tok/s"


def workload_config(a, n):
    return {
        "workload": f"qwen3-30b-a3b moe stack: {L} layers x {E} experts, top-{K_TOP}, bs=1, {a.bits}-bit g{G}, "
        "all experts resident, rmsnorm+residual between layers (no attention)",
        "model": "Qwen3-30B-A3B-shaped (random init)",
        "global_batch": n,
        "seq_len": 1,
        "parallelism": "replicas" if n > 1 else "single",
        "l2": "working set 962 MB/token >> 126 MB L2; no flush",
    }


# ------------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 50 ms.  start() returns once the first sample
    has arrived (NVML initialised), so the sampler's start-up does not land inside a timed region;
    window() marks the timed regions and stop() summarises the samples taken inside them (or, when
    the regions are shorter than the sampling period, the samples taken around them)."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )
    PERIOD_MS = 50

    def __init__(self, index):
        self.index, self.proc, self.lines, self.windows = index, None, [], []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.PERIOD_MS)],
                stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL,
                text=True,
            )
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.perf_counter()
            while not self.lines and time.perf_counter() - t0 < 10 and self.proc.poll() is None:
                time.sleep(0.01)
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def window(self, t0, t1):
        self.windows.append((t0, t1))

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(2 * self.PERIOD_MS / 1e3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        slack = self.PERIOD_MS / 1e3
        inside = [ln for t, ln in self.lines if any(a <= t <= b for a, b in self.windows)]
        around = [ln for t, ln in self.lines if any(a - slack <= t <= b + slack for a, b in self.windows)]
        use, where = (inside, "inside") if inside else (around, "within one period of")
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in use:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": mx,
            "reasons": sorted(reasons),
            "samples": len(sm),
            "period_ms": self.PERIOD_MS,
            "samples_taken": f"{where} the timed regions",
        }


# ------------------------------------------------------------------------------------------------
# workload construction (GPU)
# ------------------------------------------------------------------------------------------------
def build_workload(bits, device, seed=0):
    import torch

    from wisp import quant

    n = H * I
    nb = quant.expert_nbytes(n, bits, G)
    pool = torch.empty((L * E, nb), dtype=torch.uint8, device=device)
    gen = torch.Generator(device=device).manual_seed(seed)
    for l in range(L):
        w3 = (torch.randn(E, 3, n, device=device, generator=gen) * 0.02).to(torch.bfloat16)
        pool[l * E : (l + 1) * E].copy_(quant.quantize_batch(w3, bits, G))
        del w3
    norm_w = (1.0 + 0.1 * torch.randn(L, H, device=device, generator=gen)).to(torch.bfloat16)
    # seeded router: softmax -> top-8 -> renormalise -> bf16 (wisp/moe.py:67-72), slot = l*E + e
    logits = torch.randn(N_ROUTES, L, E, device=device, generator=gen).to(torch.bfloat16)
    p = torch.softmax(logits.float(), -1)
    rw, sel = torch.topk(p, K_TOP, -1)
    rw = (rw / rw.sum(-1, keepdim=True)).to(torch.bfloat16).float()
    slots = sel + (torch.arange(L, device=device) * E)[None, :, None]
    meta = torch.cat([slots.float(), rw], -1).contiguous()  # [N_ROUTES, L, 2k]
    x0 = torch.randn(N_ROUTES, H, device=device, generator=gen).to(torch.bfloat16)
    return dict(pool=pool, nbytes=nb, norm_w=norm_w, meta=meta, x0=x0, n=n, bits=bits)


class MoEStack:
    """One token through the 48-layer MoE stack, captured as one CUDA graph per routing."""

    def __init__(self, W):
        import torch

        from wisp import kernels

        self.W = W
        dev = W["pool"].device
        self.h = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        self.xn = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        self.moe = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        self.scratch = kernels.moe_scratch(K_TOP, I, dev)
        self.meta_in = torch.zeros(L, 2 * K_TOP, dtype=torch.float32, device=dev)  # e2e routing input
        self.x_in = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        self.graphs = []

    def _layer_loop(self, meta, x0):
        from wisp import kernels

        W = self.W
        self.h.copy_(x0)
        self.moe.zero_()
        for l in range(L):
            # h = h + moe_{l-1};  xn = rmsnorm(h)
            kernels.rmsnorm(self.h, W["norm_w"][l], 1e-6, delta=self.moe, sum_out=self.h, out=self.xn)
            kernels.moe_decode_fast(
                W["pool"], meta[l], self.xn, K_TOP, W["n"], H, I, W["bits"], G, out=self.moe, scratch=self.scratch
            )
        self.h.add_(self.moe)

    def launches_per_step(self):
        return 3 * L  # rmsnorm, gate/up, down per layer (torch copy/add nodes not counted)

    def capture(self):
        import torch

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self._layer_loop(self.W["meta"][0], self.W["x0"][0])
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        pool = torch.cuda.graph_pool_handle()
        for r in range(N_ROUTES + 1):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                if r < N_ROUTES:
                    self._layer_loop(self.W["meta"][r], self.W["x0"][r])
                else:  # the e2e graph reads its inputs from the staging buffers
                    self._layer_loop(self.meta_in, self.x_in)
            self.graphs.append(g)
        torch.cuda.synchronize()

    def step(self, t):
        self.graphs[t % N_ROUTES].replay()

    def step_e2e(self, x_host, meta_host, out_host):
        """Public-API step from host buffers: H2D of the token's input and routing, the captured
        48-layer graph, D2H of the result."""
        self.x_in.copy_(x_host, non_blocking=True)
        self.meta_in.copy_(meta_host, non_blocking=True)
        self.graphs[N_ROUTES].replay()
        out_host.copy_(self.h, non_blocking=True)


def time_moe_kernel(W, reps=20, variant=0):
    """Average duration of one fused MoE decode call (gate/up + down kernels), rotated over the 48
    layers' distinct experts (962 MB per sweep), measured with CUDA events on the launching stream."""
    import torch

    from wisp import kernels

    dev = W["pool"].device
    x = torch.randn(L, H, device=dev).to(torch.bfloat16)
    out = torch.empty(L, H, dtype=torch.bfloat16, device=dev)
    scratch = kernels.moe_scratch(K_TOP, I, dev)

    def sweep():
        for l in range(L):
            kernels.moe_decode_fast(
                W["pool"], W["meta"][0, l], x[l], K_TOP, W["n"], H, I, W["bits"], G, out=out[l], scratch=scratch, variant=variant
            )

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        sweep()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        sweep()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / (reps * L)
    del g
    return ms


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs"), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------------------------------------
# CPU legs (oracle): cpu_baseline on rank 0, and the --impl reference arm
# ------------------------------------------------------------------------------------------------
def cpu_layer_sample(bits, seed=0):
    """One MoE layer, one token, on the CPU with the oracle (dequantize -> fp32 matmul), experts in
    parallel over the host cores.  Returns (seconds, threads)."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor

    from oracle import wisp_oracle as O

    rng = np.random.default_rng(seed)
    n = H * I
    pool = np.stack([O.quantize((rng.standard_normal((3, n)) * 0.02).astype(np.float32), bits, G) for _ in range(K_TOP)])
    x = rng.standard_normal(H).astype(np.float32)
    w = np.full(K_TOP, 1.0 / K_TOP, np.float32)
    threads = os.cpu_count() or 1

    def one(j):
        gm, um, dm = O.expert_weights(pool, j, n, bits, G, H, I)
        return w[j] * (dm @ (O.silu(gm @ x) * (um @ x)))

    with ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(one, range(K_TOP)))  # warm
        t0 = time.perf_counter()
        out = sum(ex.map(one, range(K_TOP)))
        dt = time.perf_counter() - t0
    assert np.isfinite(out).all()
    return dt, threads


def run_reference(a, rank):
    if rank != 0:
        return
    times = []
    threads = os.cpu_count() or 1
    for i in range(a.warmup + a.steps):
        dt, threads = cpu_layer_sample(a.bits, seed=i)
        if i >= a.warmup:
            times.append(dt)
    per_layer = statistics.mean(times)
    tok_s = 1.0 / (per_layer * L)
    line = {
        "impl": "reference",
        "metric": metric_name(),
        "value": tok_s,
        "unit": "tok/s",
        "n_gpus": a.gpus,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": per_layer * L * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(a, 1),
        "cpu_baseline": {
            "value": tok_s,
            "unit": "tok/s",
            "cores": threads,
            "kind": "port",
            "sample": f"1 MoE layer (8 experts, 1 token) per step, extrapolated x{L} layers",
        },
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if a.impl == "reference":
        run_reference(a, rank)
        return
    import torch
    import torch.distributed as dist

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    W = build_workload(a.bits, dev, seed=rank)
    stack = MoEStack(W)
    stack.capture()
    for t in range(a.warmup):
        stack.step(t)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record(st)
    for t in range(a.steps):
        stack.step(t)
    e1.record(st)
    barrier()
    clocks.window(w0, time.perf_counter())
    ms = e0.elapsed_time(e1)
    # e2e: host buffers, copies inside the timed region
    x_host = W["x0"].cpu().pin_memory()
    meta_host = W["meta"].cpu().pin_memory()
    out_host = torch.empty(H, dtype=torch.bfloat16).pin_memory()
    for t in range(3):
        stack.step_e2e(x_host[t % N_ROUTES], meta_host[t % N_ROUTES], out_host)
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e2.record(st)
    for t in range(a.steps):
        stack.step_e2e(x_host[t % N_ROUTES], meta_host[t % N_ROUTES], out_host)
    e3.record(st)
    barrier()
    clocks.window(w0, time.perf_counter())
    ms_e2e = e2.elapsed_time(e3)
    clk = clocks.stop()
    # roofline of the fused MoE decode (algorithmic bytes: 8 experts + x + out per call)
    per_call_ms = time_moe_kernel(W)
    v1_ms = time_moe_kernel(W, variant=1)
    alg_bytes = K_TOP * W["nbytes"] + 2 * H * 2
    achieved = alg_bytes / (per_call_ms * 1e-3) / 1e9
    peak, peak_kind = load_peaks()
    t = torch.tensor([ms, ms_e2e, per_call_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e, per_call_ms = t.tolist()
    if rank == 0:
        cpu_s, cores = cpu_layer_sample(a.bits)
        cpu_tok_s = 1.0 / (cpu_s * L)
        tok = a.steps * world
        line = {
            "metric": metric_name(),
            "value": tok / (ms * 1e-3),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": a.steps,
            "warmup": a.warmup,
            "ms_per_step": ms / a.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": f"u{a.bits}->f32",
            "data": "synthetic",
            "config": workload_config(a, world),
            "e2e": {
                "value": tok / (ms_e2e * 1e-3),
                "unit": "tok/s",
                "h2d_bytes_per_step": H * 2 + L * 2 * K_TOP * 4,
                "d2h_bytes_per_step": H * 2,
            },
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": NCU_TRAFFIC_PER_CALL if a.bits == 4 else None,
                "kernel": "wisp_moe_decode (gate/up + down)",
                "bytes_per_call": alg_bytes,
                "us_per_call": per_call_ms * 1e3,
                "us_per_call_cuda_core_variant": v1_ms * 1e3,
                "peak_source": peak_kind,
            },
            "cpu_baseline": {
                "value": cpu_tok_s,
                "unit": "tok/s",
                "cores": cores,
                "kind": "port",
                "sample": f"1 MoE layer (8 experts, 1 token) on the oracle, extrapolated x{L} layers",
            },
            "gpu_launches": stack.launches_per_step() * a.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        stack.graphs = []
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
