"""Benchmark of the WiSP decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl wisp|reference] [--bits 4]
                    [--workload decoder|moe-stack] [--layers 48]

Workload ``decoder`` (default; the Qwen3-30B-A3B bs=1 decode benchmark, expert cache capped at
``--cache-frac`` 0.4 of the experts with device-side paging): greedy bs=1 decode of a
Qwen3-30B-A3B-shaped random-init model (48 layers, hidden 2048, 32 query / 4 KV heads x 128, rotary
base 1e6, RMSNorm eps 1e-6, vocab 151936, 128 experts top-8, intermediate 768, 4-bit g128 experts,
bf16 attention and embeddings).  A 512-token seeded prompt is run first; one step = one generated
token through the whole-token CUDA graph (embedding, 48 x [attention block, router, fused MoE], final
norm, lm_head, argmax, position update).  The per-token working set (3.4 GB of weights) is far larger
than L2, so no flush is needed between steps.  Workload ``moe-stack``: the 48 fused MoE layers alone
with RMSNorm + residual between them (the MoE part of the same step).

One JSON line is printed by rank 0.  ``--impl reference`` times the CPU restatement of the reference
path (oracle: dequantize then fp32 matmul, fp32 attention) on the host cores on a bounded sample.
With N > 1 GPUs every rank runs an independent replica (bs=1 decode does not shard).
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
HQ, HK, D, VOCAB = 32, 4, 128, 151936
N_ROUTES = 16  # moe-stack: distinct seeded routings (tokens) cycled through by the timed steps
EP_BATCH = 64  # moe-ep: tokens per step over all ranks (config 4 batch)
# dram__bytes_read.sum + dram__bytes_write.sum of one gate/up + one down launch (4-bit, this shape),
# from one ncu capture of the fused decode kernels
NCU_TRAFFIC_PER_CALL = 13_419_008 + 6_755_328
# DRAM read + write of the batched gate/up and down grids for one 64-token Zipf(1.1) layer (ncu)
NCU_TRAFFIC_BATCHED_LAYER = 96_768_256 + 3_038_720 + 48_437_504 + 489_472
# DRAM bytes of the two gpt-oss GEMVs (gate_up + down) of one 20b layer at one token (4 experts), one ncu capture
NCU_TRAFFIC_GPTOSS_LAYER_BS1 = 35_287_552 + 17_679_872


GO_L, GO_H, GO_I, GO_E, GO_K = 24, 2880, 2880, 32, 4  # gpt-oss-20b MoE shape (config 5)
QB_CONTEXT = 4096  # qwen-batched: KV context of every sequence when the timed steps start (config 4)
GO_PROMPT, GO_VOCAB, GO_HQ, GO_HK, GO_D, GO_WINDOW = 256, 201088, 64, 8, 64, 128  # gpt-oss-20b decoder (config 5)
TIMELINE_TOKENS = 24  # decoder with device paging: untimed steps traced with CUDA events after the timed ones


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="wisp", choices=["wisp", "reference"])
    ap.add_argument("--bits", type=int, default=4, choices=[4, 3, 2])
    ap.add_argument("--workload", default="decoder",
                    choices=["decoder", "moe-stack", "moe-ep", "gptoss-moe", "gptoss", "qwen-batched"])
    ap.add_argument("--batch", type=int, default=1, help="gptoss, gptoss-moe: sequences (tokens) per step (config 5: 1 or 32)")
    ap.add_argument("--layers", type=int, default=48, help="layers (48 = the model; fewer = a small ncu case)")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--cache-frac", type=float, default=0.4,
                    help="decoder: fraction of the L*E experts resident in the GPU slot pool (config 3: 0.4; 1 = all)")
    ap.add_argument("--paging", default="device", choices=["device", "host"],
                    help="decoder with a capped cache: device slot table, misses read from the pinned host store by "
                    "the MoE kernels, page-ins one token behind (device), or the reference's per-layer host "
                    "decision with page-in before use (host)")
    ap.add_argument("--no-prefetch", action="store_true", help="host paging: no next-layer expert prefetch")
    ap.add_argument("--tokens", default="forced", choices=["forced", "greedy"],
                    help="decoder: the token each step decodes -- a seeded random token stream (teacher forcing, so "
                    "routing keeps moving the way a real prompt stream does) or the model's own greedy choice (a "
                    "random-init model settles into a fixed loop and hardly pages)")
    ap.add_argument("--admit", default="lfu", choices=["all", "hot", "lfu", "none"],
                    help="decoder, device paging: page every miss in (all), only experts whose decayed use "
                    "frequency reached the cache's admit threshold (hot), only experts used more often than the "
                    "one they would evict (lfu), or none; misses are read from the pinned host store either way")
    ap.add_argument("--profile-one-step", action="store_true",
                    help="after the warm-up, one extra untimed step between cudaProfilerStart / Stop (for "
                    "ncu --profile-from-start off)")
    ap.add_argument("--kernel-shares", type=int, default=0,
                    help="after the timed regions, run this many steps under the torch profiler (CUPTI) and print "
                    "each kernel's device time and share to stderr")
    ap.add_argument("--batched-path", default="auto", choices=["auto", "mma", "tcgen05"],
                    help="moe-ep: the batched MoE kernels (auto = tcgen05 for 4/2-bit codes; mma = the warp-level path)")
    ap.add_argument("--transport", default="auto", choices=["auto", "nccl", "p2p"],
                    help="moe-ep exchange: NCCL all-to-alls or kernel stores into peer memory (auto: p2p when N > 1)")
    a = ap.parse_args()
    global L
    L = a.layers
    return a


def metric_name(a):
    return {"decoder": "decode tok/s", "moe-stack": "moe decode tok/s", "moe-ep": "batched moe tok/s",
            "gptoss-moe": "moe decode tok/s", "gptoss": "decode tok/s", "qwen-batched": "decode tok/s"}[a.workload]


def workload_config(a, n):
    if a.workload == "decoder":
        paged = a.cache_frac < 1.0
        if not paged:
            res, graph = "all experts resident", "(whole-token CUDA graph)"
        elif a.paging == "device":
            res = (f"expert cache capped at {a.cache_frac:.0%} of the {L * E} experts (LRU; residency in a device slot "
                   "table, non-resident experts read by the MoE kernels from the pinned host store, page-ins "
                   f"({dict(all='every miss', hot='experts that turned hot', lfu='misses used more often than the expert they would evict', none='none')[a.admit]}) decided one token behind and "
                   "copied with cudaMemcpyAsync on a side stream)")
            graph = "(whole-token CUDA graph)"
        else:
            res = (f"expert cache capped at {a.cache_frac:.0%} of the {L * E} experts (LRU, pinned host store, "
                   f"per-layer host decision, cudaMemcpyAsync on a side stream{'' if a.no_prefetch else ', next-layer prefetch'})")
            graph = "(one CUDA graph per layer segment)"
        return {
            "workload": f"qwen3-30b-a3b greedy decode bs=1: {L} layers, 32q/4kv heads x 128, {E} experts top-{K_TOP}, "
            f"{a.bits}-bit g{G} experts, {res}, bf16 attention/embeddings, vocab {VOCAB}, "
            f"{a.prompt}-token seeded prompt (chunked prefill) then one token per step, "
            + ("teacher-forced from a seeded random token stream " if a.tokens == "forced" else "greedy ") + graph,
            "model": "Qwen3-30B-A3B-shaped (random init; o_proj and expert down at std 0.02/sqrt(2L))",
            "global_batch": n,
            "seq_len": a.prompt,
            "parallelism": "replicas" if n > 1 else "single",
            "l2": "working set 3.4 GB/token >> 126 MB L2; no flush",
        }
    if a.workload == "gptoss-moe":
        return {
            "workload": f"gpt-oss-20b moe stack (config 5 MoE): {a.batch} token(s) per step, {GO_L} layers x {GO_E} experts "
            f"top-{GO_K}, hidden = intermediate = {GO_H}, clamped SwiGLU with biases, {a.bits}-bit g{G} experts (input-major "
            "gate_up/down), all experts resident, top-k then softmax routing, rmsnorm+residual between layers (no attention)",
            "model": "gpt-oss-20b-shaped (random init)",
            "global_batch": a.batch * n,
            "seq_len": 1,
            "parallelism": "replicas" if n > 1 else "single",
            "l2": f"expert working set {GO_L * GO_E * 13.2:.0f} MB >> 126 MB L2; no flush",
        }
    if a.workload == "qwen-batched":
        return {
            "workload": f"qwen3-30b-a3b batched greedy decode (config 4): {EP_BATCH} sequences in total, KV context "
            f"{QB_CONTEXT} each (seeded synthetic K/V, then one token per sequence per step), {L} layers, 32q/4kv heads x 128, "
            f"{E} experts top-{K_TOP}, {a.bits}-bit g{G} experts all resident, router logits biased to Zipf(1.1) expert "
            f"popularity, experts sharded expert-parallel over {n} GPU(s) ({E // n} per layer each)"
            + (", dispatch / combine as kernel stores into peer memory" if n > 1 and a.transport in ("auto", "p2p")
               else (", NCCL all-to-all dispatch / combine" if n > 1 else ""))
            + f", attention data-parallel ({EP_BATCH // n} sequences per GPU), whole-step CUDA graph",
            "model": "Qwen3-30B-A3B-shaped (random init; o_proj and expert down at std 0.02/sqrt(2L))",
            "global_batch": EP_BATCH,
            "seq_len": QB_CONTEXT,
            "parallelism": f"ep{n}+dp{n}",
            "l2": "KV cache read per step (537 MB per layer at 64 x 4096) >> 126 MB L2; no flush",
        }
    if a.workload == "gptoss":
        return {
            "workload": f"gpt-oss-20b greedy decode, {a.batch} sequence(s) per step: {GO_L} layers, hidden {GO_H}, "
            f"{GO_HQ}q/{GO_HK}kv heads x {GO_D} with biases and per-head attention sinks, sliding window {GO_WINDOW} on "
            f"alternate layers, YaRN rotary, {GO_E} experts top-{GO_K} of intermediate {GO_I} (clamped SwiGLU, biases), "
            f"{a.bits}-bit g{G} experts all resident, bf16 attention/embeddings, vocab {GO_VOCAB}, {GO_PROMPT}-token seeded "
            "prompt per sequence, then one greedy token per sequence per step (whole-step CUDA graph)",
            "model": "gpt-oss-20b-shaped (random init; o_proj and expert down at std 0.02/sqrt(2L))",
            "global_batch": a.batch * n,
            "seq_len": GO_PROMPT,
            "parallelism": "replicas" if n > 1 else "single",
            "l2": "working set per step (lm_head 1.16 GB + experts) >> 126 MB L2; no flush",
        }
    if a.workload == "moe-ep":
        return {
            "workload": f"qwen3-30b-a3b batched moe stack (config 4 MoE): {EP_BATCH} tokens in total, {L} layers x {E} "
            f"experts top-{K_TOP}, Zipf(1.1) expert popularity, {a.bits}-bit g{G}, experts sharded expert-parallel "
            f"over {n} GPU(s) ({E // n} per layer each), "
            + ("dispatch and combine as kernel stores into peer memory (CUDA IPC over NVLink, flags)"
               if (a.transport == "p2p" or (a.transport == "auto" and n > 1)) else "NCCL all-to-all dispatch and combine")
            + ", rmsnorm+residual between layers (no attention), batched expert products on "
            + ("tcgen05 (TMEM accumulators)" if a.batched_path == "tcgen05" else "the warp-level tensor-core kernels"),
            "model": "Qwen3-30B-A3B-shaped (random init)",
            "global_batch": EP_BATCH,
            "seq_len": 1,
            "parallelism": f"ep{n}",
            "l2": "expert working set per layer >> 126 MB L2; no flush",
        }
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


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs"), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------------------------------------
# the fused MoE call in isolation (roofline of the dominant kernel pair)
# ------------------------------------------------------------------------------------------------
def time_moe_kernel(pool, nbytes, bits, reps=20, variant=0):
    """Average duration of one fused MoE decode call (gate/up + down kernels), rotated over L layers'
    distinct experts (L*8 experts per sweep, 962 MB at 48 layers and 4 bits), CUDA events on the
    launching stream around a graph of the sweep."""
    import torch

    from wisp import kernels

    dev = pool.device
    g = torch.Generator(device=dev).manual_seed(99)
    x = torch.randn(L, H, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(L, H, dtype=torch.bfloat16, device=dev)
    scratch = kernels.moe_scratch(K_TOP, I, dev, H, bits, G)
    metas = []
    nslots = pool.shape[0]
    for l in range(L):
        # distinct slots per call; with a full pool, layer l's experts (l*E ..), else any slots
        sel = torch.randperm(E, device=dev, generator=g)[:K_TOP] + l * E if nslots >= L * E else \
            torch.randperm(nslots, device=dev, generator=g)[:K_TOP]
        metas.append(torch.cat([sel.float(), torch.full((K_TOP,), 1.0 / K_TOP, device=dev)]))

    def sweep():
        for l in range(L):
            kernels.moe_decode_fast(pool, metas[l], x[l], K_TOP, H * I, H, I, bits, G, out=out[l], scratch=scratch, variant=variant)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        sweep()
    torch.cuda.current_stream().wait_stream(s)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        sweep()
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        gr.replay()
    e1.record(st)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / (reps * L)
    del gr
    return ms


def moe_roofline(pool, nbytes, bits):
    per_call_ms = time_moe_kernel(pool, nbytes, bits)
    v1_ms = time_moe_kernel(pool, nbytes, bits, variant=1)
    alg = K_TOP * nbytes + 2 * H * 2
    achieved = alg / (per_call_ms * 1e-3) / 1e9
    peak, kind = load_peaks()
    return {
        "bound": "hbm",
        "achieved": achieved,
        "peak": peak,
        "unit": "GB/s",
        "frac": achieved / peak,
        "traffic": NCU_TRAFFIC_PER_CALL if bits == 4 else None,
        "kernel": "wisp_moe_decode (gate/up + down), one layer's 8 routed experts",
        "bytes_per_call": alg,
        "us_per_call": per_call_ms * 1e3,
        "us_per_call_cuda_core_variant": v1_ms * 1e3,
        "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured" else "fallback",
    }, per_call_ms


# ------------------------------------------------------------------------------------------------
# CPU legs (oracle): cpu_baseline on rank 0, and the --impl reference arm
# ------------------------------------------------------------------------------------------------
_CPU_WEIGHTS = {}


def _cpu_weights(bits, attention, context):
    """Seeded host copies of one layer's weights (built once per process)."""
    import numpy as np

    from oracle import wisp_oracle as O

    key = (bits, attention, context)
    if key not in _CPU_WEIGHTS:
        rng = np.random.default_rng(1234)
        n = H * I
        wt = dict(pool=np.stack([O.quantize((rng.standard_normal((3, n)) * 0.02).astype(np.float32), bits, G) for _ in range(K_TOP)]))
        if attention:
            wt.update(
                wqkv=(rng.standard_normal(((HQ + 2 * HK) * D, H)) * 0.02).astype(np.float32),
                wo=(rng.standard_normal((H, HQ * D)) * 0.02).astype(np.float32),
                wr=(rng.standard_normal((E, H)) * 0.02).astype(np.float32),
                kc=rng.standard_normal((HK, context, D)).astype(np.float32),
                vc=rng.standard_normal((HK, context, D)).astype(np.float32),
            )
        _CPU_WEIGHTS[key] = wt
    return _CPU_WEIGHTS[key]


_CPU_POOL = None


def cpu_pool():
    """One thread per host core, kept for the whole run (numpy releases the GIL in its kernels)."""
    global _CPU_POOL
    if _CPU_POOL is None:
        from concurrent.futures import ThreadPoolExecutor

        _CPU_POOL = ThreadPoolExecutor(max_workers=os.cpu_count() or 1)
    return _CPU_POOL


def cpu_layer_sample(bits, seed=0, attention=False, context=512):
    """One layer, one token, on the CPU with the oracle (dequantize -> fp32 matmul; experts in
    parallel over the host cores): the fused MoE, plus (attention=True) RMSNorm, q/k/v/o projections,
    GQA attention over ``context`` cached positions and the router.  Returns (seconds, threads)."""
    import numpy as np

    from oracle import wisp_oracle as O

    wt = _cpu_weights(bits, attention, context)
    rng = np.random.default_rng(seed)
    n = H * I
    x = rng.standard_normal(H).astype(np.float32)
    w = np.full(K_TOP, 1.0 / K_TOP, np.float32)
    nw = np.ones(H, np.float32)

    def one(j):
        gm, um, dm = O.expert_weights(wt["pool"], j, n, bits, G, H, I)
        return w[j] * (dm @ (O.silu(gm @ x) * (um @ x)))

    ex = cpu_pool()
    t0 = time.perf_counter()
    if attention:
        xn = O.rmsnorm(x, nw)
        qkv = wt["wqkv"] @ xn
        q = qkv[: HQ * D].reshape(HQ, D)
        att = O.gqa_decode_attention(q, wt["kc"], wt["vc"], context - 1, D**-0.5)
        hm = x + wt["wo"] @ att.reshape(-1)
        O.router_topk((wt["wr"] @ O.rmsnorm(hm, nw))[None], K_TOP)
    out = sum(ex.map(one, range(K_TOP)))
    dt = time.perf_counter() - t0
    assert np.isfinite(out).all()
    return dt, os.cpu_count() or 1


def cpu_head_sample(seed=0, frac=16):
    """lm_head GEMV (fp32) over 1/frac of the vocabulary rows; returns the extrapolated seconds."""
    import numpy as np

    rng = np.random.default_rng(seed)
    rows = VOCAB // frac
    W = (rng.standard_normal((rows, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal(H).astype(np.float32)
    W @ x
    t0 = time.perf_counter()
    y = W @ x
    dt = time.perf_counter() - t0
    assert np.isfinite(y).all()
    return dt * frac


def _parallel_expert_cost(fn, m):
    """Wall time of m expert computations run in parallel on the host cores, per expert."""
    ex = cpu_pool()
    t0 = time.perf_counter()
    list(ex.map(fn, range(m)))
    return (time.perf_counter() - t0) / m


def cpu_sample(a, seed=0, distinct=60.0):
    """One bounded sample of the workload on the CPU path (the reference's algorithm restated in numpy:
    dequantize, then fp32 products), on every host core.  Returns (sample seconds, tokens/s that the
    sample implies for the whole step, cores, what the sample was)."""
    import numpy as np

    from oracle import wisp_oracle as O

    threads = os.cpu_count() or 1
    if a.workload == "decoder":
        dt, _ = cpu_layer_sample(a.bits, seed=seed, attention=True, context=a.prompt)
        head = cpu_head_sample(seed)
        return dt, 1.0 / (dt * L + head), threads, (
            f"one decoder layer of one token (RMSNorm, q/k/v/o projections, GQA attention over {a.prompt} positions, "
            f"router, 8 experts in parallel) per sample; token time = {L} x the layer + lm_head (1/16 of its rows timed, x16)")
    if a.workload == "moe-stack":
        dt, _ = cpu_layer_sample(a.bits, seed=seed)
        return dt, 1.0 / (dt * L), threads, f"one MoE layer (8 experts in parallel, 1 token) per sample; token time = {L} x the layer"
    rng = np.random.default_rng(seed)
    if a.workload == "moe-ep":
        n = H * I
        toks = max(1, int(round(EP_BATCH * K_TOP / distinct)))
        wt = _cpu_weights(a.bits, False, 0)
        x = rng.standard_normal((toks, H)).astype(np.float32)

        def one(j):
            gm, um, dm = O.expert_weights(wt["pool"], j % K_TOP, n, a.bits, G, H, I)
            return (O.silu(x @ gm.T) * (x @ um.T)) @ dm.T

        m = max(K_TOP, threads)
        per = _parallel_expert_cost(one, m)
        return per * m, EP_BATCH / (per * distinct * L), threads, (
            f"{m} experts in parallel (dequantize + fp32 MLP of the {toks} tokens an expert receives on average) per "
            f"sample; step time = per-expert time x {distinct:.0f} distinct experts per layer x {L} layers, {EP_BATCH} tokens")
    if a.workload == "gptoss":
        return cpu_gptoss_sample(a, seed, distinct)
    if a.workload == "qwen-batched":
        return cpu_batched_sample(a, seed, distinct)
    # gptoss-moe
    n = GO_H * GO_I
    dist_go = distinct if distinct < 60.0 else float(min(GO_E, a.batch * GO_K))
    toks = max(1, int(round(a.batch * GO_K / dist_go)))
    if "gptoss" not in _CPU_WEIGHTS:
        _CPU_WEIGHTS["gptoss"] = O.quantize((np.random.default_rng(77).standard_normal((3, n)) * 0.02).astype(np.float32),
                                            a.bits, G)[None]
    pool = _CPU_WEIGHTS["gptoss"]
    gub, db = np.zeros((1, 2 * GO_I), np.uint16), np.zeros((1, GO_H), np.uint16)
    x = rng.standard_normal((toks, GO_H)).astype(np.float32)

    def one(j):
        return O.gptoss_ref(pool, np.zeros((toks, 1), np.int64), np.ones((toks, 1), np.float32), x, GO_H, GO_I, a.bits, G,
                            gub, db)

    m = max(GO_K, threads)
    per = _parallel_expert_cost(one, m)
    return per * m, a.batch / (per * dist_go * GO_L), threads, (
        f"{m} gpt-oss experts in parallel (dequantize + fp32 MLP of {toks} token(s)) per sample; step time = per-expert "
        f"time x {dist_go:.1f} distinct experts per layer x {GO_L} layers, {a.batch} token(s) per step")


def cpu_batched_sample(a, seed, distinct, seqs=4):
    """Config 4 on the host cores: the attention part of one layer (RMSNorm, q/k/v projections, GQA over
    QB_CONTEXT positions, o projection, router) for ``seqs`` of the 64 sequences, scaled to 64; the
    distinct experts of a layer (dequantize + fp32 MLP of the tokens one expert receives on average) in
    parallel; step time = L x (attention part + experts) + the lm_head of 64 tokens (1/16 of its rows)."""
    import numpy as np

    from oracle import wisp_oracle as O

    wt = _cpu_weights(a.bits, True, QB_CONTEXT)
    rng = np.random.default_rng(seed)
    n = H * I
    nw = np.ones(H, np.float32)
    ex = cpu_pool()
    x = rng.standard_normal((seqs, H)).astype(np.float32)

    def attn(b):
        xn = O.rmsnorm(x[b], nw)
        q = (wt["wqkv"] @ xn)[: HQ * D].reshape(HQ, D)
        att = O.gqa_decode_attention(q, wt["kc"], wt["vc"], QB_CONTEXT - 1, D ** -0.5)
        hm = x[b] + wt["wo"] @ att.reshape(-1)
        O.router_topk((wt["wr"] @ O.rmsnorm(hm, nw))[None], K_TOP)

    t0 = time.perf_counter()
    list(ex.map(attn, range(seqs)))
    dense = (time.perf_counter() - t0) * EP_BATCH / seqs
    toks = max(1, int(round(EP_BATCH * K_TOP / distinct)))
    xe = rng.standard_normal((toks, H)).astype(np.float32)

    def one(j):
        gm, um, dm = O.expert_weights(wt["pool"], j % K_TOP, n, a.bits, G, H, I)
        return (O.silu(xe @ gm.T) * (xe @ um.T)) @ dm.T

    m = max(K_TOP, os.cpu_count() or 1)
    per = _parallel_expert_cost(one, m)
    head = cpu_head_sample(seed) * EP_BATCH
    step = L * (dense + per * distinct) + head
    return step, EP_BATCH / step, os.cpu_count() or 1, (
        f"per sample: the attention part of one layer for {seqs} sequences at context {QB_CONTEXT} (x {EP_BATCH // seqs}), "
        f"{m} experts in parallel (dequantize + fp32 MLP of {toks} tokens); step time = {L} x (attention part + per-expert "
        f"time x {distinct:.0f} distinct experts) + the lm_head of {EP_BATCH} tokens")


def cpu_gptoss_sample(a, seed, distinct):
    """One gpt-oss decoder layer for ``a.batch`` sequences on the host cores: RMSNorm, q/k/v projections with
    biases, GQA attention with sinks over the context (the window on sliding layers), o projection, router,
    the distinct experts of the layer (dequantize + fp32 clamped-SwiGLU MLP) in parallel; step time =
    24 x the layer + the lm_head over the vocabulary (1/16 of its rows timed)."""
    import numpy as np

    from oracle import wisp_oracle as O

    rng = np.random.default_rng(seed)
    B = a.batch
    n = GO_H * GO_I
    if "gptoss_dec" not in _CPU_WEIGHTS:
        r = np.random.default_rng(78)
        qkv = (GO_HQ + 2 * GO_HK) * GO_D
        _CPU_WEIGHTS["gptoss_dec"] = dict(
            pool=O.quantize((r.standard_normal((3, n)) * 0.02).astype(np.float32), a.bits, G)[None],
            wqkv=(r.standard_normal((qkv, GO_H)) * 0.02).astype(np.float32), bqkv=np.zeros(qkv, np.float32),
            wo=(r.standard_normal((GO_H, GO_HQ * GO_D)) * 0.02).astype(np.float32),
            wr=(r.standard_normal((GO_E, GO_H)) * 0.02).astype(np.float32),
            kc=r.standard_normal((GO_HK, GO_PROMPT, GO_D)).astype(np.float32),
            vc=r.standard_normal((GO_HK, GO_PROMPT, GO_D)).astype(np.float32),
            head=(r.standard_normal((GO_VOCAB // 16, GO_H)) * 0.02).astype(np.float32))
    wt = _CPU_WEIGHTS["gptoss_dec"]
    dist_go = distinct if distinct < 60.0 else float(min(GO_E, B * GO_K))
    toks = max(1, int(round(B * GO_K / dist_go)))
    gub, db = np.zeros((1, 2 * GO_I), np.uint16), np.zeros((1, GO_H), np.uint16)
    x = rng.standard_normal((B, GO_H)).astype(np.float32)
    xe = rng.standard_normal((toks, GO_H)).astype(np.float32)
    nw = np.ones(GO_H, np.float32)
    ex = cpu_pool()

    def attn(b, window):
        xn = O.rmsnorm(x[b], nw)
        q = (wt["wqkv"] @ xn + wt["bqkv"])[: GO_HQ * GO_D].reshape(GO_HQ, GO_D)
        lo = GO_PROMPT - window if window else 0
        att = O.gqa_decode_attention(q, wt["kc"][:, lo:], wt["vc"][:, lo:], GO_PROMPT - lo - 1, GO_D ** -0.5)
        hm = x[b] + wt["wo"] @ att.reshape(-1)
        O.router_topk((wt["wr"] @ O.rmsnorm(hm, nw))[None], GO_K)

    def expert(j):
        return O.gptoss_ref(wt["pool"], np.zeros((toks, 1), np.int64), np.ones((toks, 1), np.float32), xe, GO_H, GO_I, a.bits,
                            G, gub, db)

    t0 = time.perf_counter()
    for window in (GO_WINDOW, 0):  # one sliding and one full layer
        list(ex.map(lambda b: attn(b, window), range(B)))
    dense = (time.perf_counter() - t0) / 2
    m = max(GO_K, min(int(round(dist_go)), os.cpu_count() or 1))
    per = _parallel_expert_cost(expert, m)
    t0 = time.perf_counter()
    wt["head"] @ O.rmsnorm(x, nw).T
    head = (time.perf_counter() - t0) * 16
    step = GO_L * (dense + per * dist_go) + head
    return step, B / step, os.cpu_count() or 1, (
        f"per sample: {B} sequence(s) through the attention part of one sliding and one full layer (context "
        f"{GO_PROMPT}), {m} experts in parallel (dequantize + fp32 MLP of {toks} token(s)), lm_head over 1/16 of the vocabulary; "
        f"step time = {GO_L} x (attention part + per-expert time x {dist_go:.1f} distinct experts) + 16 x the lm_head share")


def cpu_tok_s(a, seed=0, distinct=60.0, samples=2):
    """The CPU baseline of the wisp arm's line: one warm-up sample, then the mean of ``samples``."""
    cpu_sample(a, seed, distinct)
    got = [cpu_sample(a, seed + 1 + i, distinct) for i in range(samples)]
    return statistics.mean(g[1] for g in got), got[0][2], got[0][3] + f"; mean of {samples} samples after 1 warm-up"


CPU_SAMPLES = 8  # most timed CPU samples per reference run (a decoder-layer sample takes about a second)


def run_reference(a, rank):
    """The reference arm: the CPU path on every host core, ``--warmup`` (at most 2) untimed samples, then
    ``--steps`` (at most CPU_SAMPLES) timed samples; each sample is one bounded piece of a step (a
    decoder layer, an MoE layer, a batch of experts), and ``value`` is the tokens/s those samples imply
    for whole steps.  ``steps`` and ``ms_per_step`` report the samples actually timed."""
    if rank != 0:
        return
    warm = max(1, min(a.warmup, 2))
    nt = max(1, min(a.steps, CPU_SAMPLES))
    for i in range(warm):
        cpu_sample(a, seed=i)
    t0 = time.perf_counter()
    got = [cpu_sample(a, seed=warm + i) for i in range(nt)]
    wall = time.perf_counter() - t0
    tok_s = statistics.mean(g[1] for g in got)
    threads, sample = got[0][2], got[0][3] + f"; mean of {nt} timed samples after {warm} untimed"
    line = {
        "impl": "reference",
        "metric": metric_name(a),
        "value": tok_s,
        "unit": "tok/s",
        "n_gpus": a.gpus,
        "steps": nt,
        "warmup": warm,
        "ms_per_step": 1e3 * statistics.mean(g[0] for g in got),
        "step_is_sample": True,
        "timed_s": wall,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(a, 1),
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# moe-stack workload
# ------------------------------------------------------------------------------------------------
def build_moe_workload(bits, device, seed=0):
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
    """One token through the MoE layers, captured as one CUDA graph per routing."""

    def __init__(self, W):
        import torch

        from wisp import kernels

        self.W = W
        dev = W["pool"].device
        self.h = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        self.xn = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        self.moe = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        self.scratch = kernels.moe_scratch(K_TOP, I, dev, H, W["bits"], G)
        self.meta_in = torch.zeros(L, 2 * K_TOP, dtype=torch.float32, device=dev)  # e2e routing input
        self.x_in = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        self.graphs = []

    def _layer_loop(self, meta, x0):
        from wisp import kernels

        W = self.W
        self.h.copy_(x0)
        self.moe.zero_()
        for l in range(L):
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

    def e2e_inputs(self):
        import torch

        return (self.W["x0"].cpu().pin_memory(), self.W["meta"].cpu().pin_memory(),
                torch.empty(H, dtype=torch.bfloat16).pin_memory())

    def step_e2e(self, t, inp):
        x_host, meta_host, out_host = inp
        self.x_in.copy_(x_host[t % N_ROUTES], non_blocking=True)
        self.meta_in.copy_(meta_host[t % N_ROUTES], non_blocking=True)
        self.graphs[N_ROUTES].replay()
        out_host.copy_(self.h, non_blocking=True)

    def e2e_bytes(self):
        return H * 2 + L * 2 * K_TOP * 4, H * 2

    def release(self):
        self.graphs = []


# ------------------------------------------------------------------------------------------------
# gptoss-moe workload (config 5 MoE part)
# ------------------------------------------------------------------------------------------------
class GptOssStack:
    """``a.batch`` tokens through the 24 gpt-oss-20b-shaped MoE layers, RMSNorm + residual between them,
    one CUDA graph per seeded routing (top-4 of the logits, then softmax over the selected,
    wisp/gptoss.py:116-118)."""

    def __init__(self, a, device, seed):
        import torch

        from wisp import kernels, quant

        self.N, self.bits = a.batch, a.bits
        n = GO_H * GO_I
        self.nb = quant.expert_nbytes(n, a.bits, G)
        bf = torch.bfloat16
        self.pool = torch.empty((GO_L * GO_E, self.nb), dtype=torch.uint8, device=device)
        gen = torch.Generator(device=device).manual_seed(seed)
        for l in range(GO_L):
            for e0 in range(0, GO_E, 8):
                w3 = (torch.randn(8, 3, n, device=device, generator=gen) * 0.02).to(bf)
                self.pool[l * GO_E + e0 : l * GO_E + e0 + 8].copy_(quant.quantize_batch(w3, a.bits, G))
                del w3
        self.gub = (torch.randn(GO_L, GO_E, 2 * GO_I, device=device, generator=gen) * 0.02).to(bf)
        self.db = (torch.randn(GO_L, GO_E, GO_H, device=device, generator=gen) * 0.02).to(bf)
        self.norm_w = (1.0 + 0.1 * torch.randn(GO_L, GO_H, device=device, generator=gen)).to(bf)
        logits = torch.randn(N_ROUTES, GO_L, self.N, GO_E, device=device, generator=gen).to(bf)
        tv, ti = torch.topk(logits.float(), GO_K, -1)
        sc = torch.softmax(tv, -1).to(bf).float()
        slots = ti + (torch.arange(GO_L, device=device) * GO_E)[None, :, None, None]
        self.meta = torch.cat([slots.float(), sc], -1).contiguous()  # [R, L, N, 2k]
        self.experts = ti.to(torch.int32).contiguous()  # [R, L, N, k]
        self.distinct = float(
            sum(torch.unique(ti[r, l]).numel() for r in range(N_ROUTES) for l in range(GO_L)) / (N_ROUTES * GO_L)
        )
        self.x0 = torch.randn(N_ROUTES, self.N, GO_H, device=device, generator=gen).to(bf)
        self.h = torch.zeros(self.N, GO_H, dtype=bf, device=device)
        self.xn = torch.zeros_like(self.h)
        self.moe = torch.zeros_like(self.h)
        from wisp import _lib

        self.ws = torch.empty(_lib.lib().wisp_moe_gptoss_workspace_bytes(self.N, GO_K, GO_H, GO_I), dtype=torch.uint8,
                              device=device)
        self.meta_in = torch.zeros_like(self.meta[0])
        self.exp_in = torch.zeros_like(self.experts[0])
        self.x_in = torch.zeros_like(self.h)
        self.graphs = []

    def _layer_loop(self, meta, experts, x0):
        from wisp import kernels

        self.h.copy_(x0)
        self.moe.zero_()
        for l in range(GO_L):
            kernels.rmsnorm(self.h, self.norm_w[l], 1e-5, delta=self.moe, sum_out=self.h, out=self.xn)
            kernels.moe_gptoss(self.pool, meta[l], experts[l], self.xn, GO_K, GO_H, GO_I, self.bits, self.gub[l], self.db[l],
                               group=G, out=self.moe, workspace=self.ws)
        self.h.add_(self.moe)

    def launches_per_step(self):
        return 6 * GO_L  # rmsnorm; grouping, gate_up GEMV, activation, down GEMV, combine

    def capture(self):
        import torch

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self._layer_loop(self.meta[0], self.experts[0], self.x0[0])
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        pool = torch.cuda.graph_pool_handle()
        for r in range(N_ROUTES + 1):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                if r < N_ROUTES:
                    self._layer_loop(self.meta[r], self.experts[r], self.x0[r])
                else:
                    self._layer_loop(self.meta_in, self.exp_in, self.x_in)
            self.graphs.append(g)
        torch.cuda.synchronize()

    def step(self, t):
        self.graphs[t % N_ROUTES].replay()

    def e2e_inputs(self):
        import torch

        return (self.x0.cpu().pin_memory(), self.meta.cpu().pin_memory(), self.experts.cpu().pin_memory(),
                torch.empty(self.N, GO_H, dtype=torch.bfloat16).pin_memory())

    def step_e2e(self, t, inp):
        x_host, meta_host, exp_host, out_host = inp
        r = t % N_ROUTES
        self.x_in.copy_(x_host[r], non_blocking=True)
        self.meta_in.copy_(meta_host[r], non_blocking=True)
        self.exp_in.copy_(exp_host[r], non_blocking=True)
        self.graphs[N_ROUTES].replay()
        out_host.copy_(self.h, non_blocking=True)

    def e2e_bytes(self):
        return self.x_in.numel() * 2 + self.meta_in.numel() * 4 + self.exp_in.numel() * 4, self.h.numel() * 2

    def roofline(self, ms_per_step, peak, peak_src):
        """Per layer: the distinct routed experts' bytes (+ activations in and out) over the step time
        per layer (RMSNorm included, so a lower bound on the MoE kernels' own rate)."""
        bytes_layer = self.distinct * self.nb + 2 * self.N * GO_H * 2
        us = ms_per_step / GO_L * 1e3
        ach = bytes_layer / (us * 1e-6) / 1e9
        traffic = NCU_TRAFFIC_GPTOSS_LAYER_BS1 if self.N == 1 and self.bits == 4 else None
        return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak, "traffic": traffic,
                "kernel": "wisp_moe_gptoss (grouping, gate_up GEMV, activation, down GEMV, combine) per layer, timed as "
                "the step time / layers (RMSNorm included)", "bytes_per_call": bytes_layer, "us_per_call": us,
                "peak_source": peak_src}

    def release(self):
        self.graphs = []


# ------------------------------------------------------------------------------------------------
# qwen-batched workload (config 4: 64 sequences at KV context 4096, experts expert-parallel)
# ------------------------------------------------------------------------------------------------
class QwenBatchedBench:
    """EP_BATCH sequences over all ranks (EP_BATCH / world each) decoded greedily through BatchedDecoder:
    every sequence's cache holds QB_CONTEXT seeded positions when the timed steps start; the router
    logits carry a Zipf(1.1) popularity bias; with world > 1 the experts are split over the ranks."""

    def __init__(self, a, device, rank, world):
        import torch

        from wisp.batched_decoder import BatchedDecoder, zipf_bias
        from wisp.ep import ExpertParallelMoE, batched_expert_fn
        from wisp.model import DecoderConfig, DecoderWeights

        assert EP_BATCH % world == 0 and E % world == 0
        self.B, self.El, self.world = EP_BATCH // world, E // world, world
        cfg = DecoderConfig(layers=L, bits=a.bits)
        local = None if world == 1 else (rank * self.El, self.El)
        self.w = DecoderWeights.random(cfg, device=device, seed=0, resid_scale=True, local_experts=local, router_std=H ** -0.5)
        self.nb = self.w.nbytes
        variant = {"auto": 0, "mma": 1, "tcgen05": 2}[a.batched_path]
        self.ep = None
        if world > 1:
            fn = batched_expert_fn(self.w.pool, lambda l, e: l * self.El + e, H * I, H, I, a.bits, G, variant=variant)
            transport = a.transport if a.transport != "auto" else "p2p"
            self.ep = ExpertParallelMoE(E, K_TOP, H, self.B, fn, device=device, slot_base=lambda l: l * self.El,
                                        transport=transport)
        tmax = QB_CONTEXT + 2 * (a.warmup + a.steps) + 64
        self.dec = BatchedDecoder(self.w, batch=self.B, tmax=tmax, ep=self.ep, expert_bias=zipf_bias(L, E, device=device),
                                  variant=variant)
        g = torch.Generator(device=device).manual_seed(100 + rank)
        for l in range(L):  # seeded synthetic context
            self.dec.kc[l, :, :, :QB_CONTEXT].normal_(generator=g)
            self.dec.vc[l, :, :, :QB_CONTEXT].normal_(generator=g)
        self.dec.pos.fill_(QB_CONTEXT)
        self.dec.tokens.copy_(torch.randint(0, VOCAB, (self.B,), device=device, generator=g))
        self.dec.next_token.copy_(self.dec.tokens)
        self.dec.capture()
        self.prefill_s = 0.0
        self.distinct_seen = []

    def step(self, t):
        self.dec.step()

    def record_routes(self):
        import torch

        r = self.dec.routes  # this rank's sequences; the distinct experts of the whole batch need every rank
        if self.world > 1:
            import torch.distributed as dist

            allr = [torch.empty_like(r) for _ in range(self.world)]
            dist.all_gather(allr, r.contiguous())
            r = torch.cat(allr, 1)
        self.distinct_seen.append(sum(torch.unique(r[l]).numel() for l in range(L)) / L)

    @property
    def distinct(self):
        return statistics.mean(self.distinct_seen) if self.distinct_seen else 50.0

    def launches_per_step(self):
        """This package's kernels per step (cuBLAS GEMMs, torch's adds, copies and argmax not counted): per
        layer RMSNorm, rotary + cache write, attention (2), router, and the batched MoE (grouping, permute,
        gate/up, down, combine: 5) or, expert-parallel, dispatch + batched MoE + combine (7, 9 with the
        peer-memory transport); the final RMSNorm."""
        per = 5 + (5 if self.world == 1 else (9 if self.ep.p2p is not None else 7))
        return L * per + 1

    def e2e_inputs(self):
        import torch

        return (torch.randint(0, VOCAB, (self.B,), generator=torch.Generator().manual_seed(9)).pin_memory(),
                torch.empty(self.B, dtype=torch.int64).pin_memory())

    def step_e2e(self, t, inp):
        tok_host, out_host = inp
        self.dec.tokens.copy_(tok_host, non_blocking=True)
        self.dec.graph.replay()
        out_host.copy_(self.dec.next_token, non_blocking=True)

    def e2e_bytes(self):
        return 8 * self.B, 8 * self.B

    def step_bytes(self, ctx):
        """Algorithmic bytes one GPU moves per step: every dense weight once, its share of the distinct
        experts of each layer, and its sequences' K/V over the context."""
        dense = L * 2 * ((HQ + 2 * HK) * D * H + H * HQ * D + E * H + 2 * H + 2 * D) + 2 * VOCAB * H + 2 * H
        kv = L * self.B * 2 * HK * D * 2 * ctx
        return dense + L * self.distinct / self.world * self.nb + kv

    def roofline(self, ms_per_step, peak, peak_src, ctx):
        b = self.step_bytes(ctx)
        ach = b / (ms_per_step * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak, "traffic": None,
                "kernel": "whole decode step on one GPU (every kernel of the graph): algorithmic bytes per step / step time",
                "bytes_per_call": b, "us_per_call": ms_per_step * 1e3, "peak_source": peak_src}

    def release(self):
        self.dec.release()
        if self.ep is not None:
            self.ep.close()


# ------------------------------------------------------------------------------------------------
# gptoss workload (config 5: the whole gpt-oss-20b-shaped decoder, bs 1 or 32)
# ------------------------------------------------------------------------------------------------
class GptOssDecodeBench:
    """``a.batch`` sequences decoded greedily through GptOssDecoder (one CUDA graph per step) after a
    256-token seeded prompt per sequence."""

    def __init__(self, a, device, seed):
        import torch

        from wisp.gptoss_decoder import GptOssDecoder, GptOssDecoderConfig, GptOssWeights

        self.a, self.B = a, a.batch
        cfg = GptOssDecoderConfig(bits=a.bits, group=G)
        t0 = time.perf_counter()
        self.w = GptOssWeights.random(cfg, device=device, seed=seed)
        torch.cuda.synchronize()
        self.build_s = time.perf_counter() - t0
        tmax = GO_PROMPT + 2 * a.warmup + 2 * a.steps + 16
        self.dec = GptOssDecoder(self.w, batch=self.B, tmax=tmax)
        self.nb = self.w.nbytes
        g = torch.Generator().manual_seed(1000 + seed)
        ids = torch.randint(0, cfg.vocab, (self.B, GO_PROMPT), generator=g).to(device)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        self.dec.prompt(ids)
        torch.cuda.synchronize()
        self.prefill_s = time.perf_counter() - t0
        self.distinct_seen = []

    def step(self, t):
        self.dec.step()

    def record_routes(self):
        import torch

        r = self.dec.routes
        self.distinct_seen.append(sum(torch.unique(r[l]).numel() for l in range(r.shape[0])) / r.shape[0])

    @property
    def distinct(self):
        return statistics.mean(self.distinct_seen) if self.distinct_seen else float(min(GO_E, self.B * GO_K))

    def launches_per_step(self):
        """This package's kernels per step (cuBLAS GEMMs, torch's adds and argmax at B > 1 not counted).
        Per layer: B = 1: two GEMVs, rotary + cache write, attention (2), router, wisp_moe_gptoss (4: the
        gate_up grid groups the pairs itself); B > 1: RMSNorm, rotary, attention (2), router, wisp_moe_gptoss
        (5 with its grouping grid).  Per step: embedding, final RMSNorm, lm_head GEMV, argmax (2) at B = 1;
        the final RMSNorm at B > 1."""
        return GO_L * 10 + (5 if self.B == 1 else 1)

    def e2e_inputs(self):
        import torch

        return (torch.randint(0, GO_VOCAB, (self.B,), generator=torch.Generator().manual_seed(9)).pin_memory(),
                torch.empty(self.B, dtype=torch.int64).pin_memory())

    def step_e2e(self, t, inp):
        tok_host, out_host = inp
        self.dec.tokens.copy_(tok_host, non_blocking=True)
        self.dec.graph.replay()
        out_host.copy_(self.dec.next_token, non_blocking=True)

    def e2e_bytes(self):
        return 8 * self.B, 8 * self.B

    def step_bytes(self, ctx):
        """Algorithmic bytes of one step: every dense weight once, the distinct experts of each layer,
        the embedding rows, and each sequence's cached K/V over its window."""
        d = GO_HQ * GO_D
        qkv = (GO_HQ + 2 * GO_HK) * GO_D
        dense = GO_L * 2 * (qkv * GO_H + qkv + GO_H * d + GO_H + GO_E * GO_H + GO_E + 4 * GO_H + GO_E * 3 * GO_I)
        dense += 2 * GO_VOCAB * GO_H + 2 * GO_H + self.B * 2 * GO_H
        kv = sum(self.B * 2 * GO_HK * GO_D * 2 * (min(ctx, GO_WINDOW) if l % 2 == 0 else ctx) for l in range(GO_L))
        return dense + GO_L * self.distinct * self.nb + kv

    def roofline(self, ms_per_step, peak, peak_src, ctx):
        b = self.step_bytes(ctx)
        ach = b / (ms_per_step * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak, "traffic": None,
                "kernel": "whole decode step (every kernel of the graph): algorithmic bytes per step / step time",
                "bytes_per_call": b, "us_per_call": ms_per_step * 1e3, "peak_source": peak_src}

    def release(self):
        self.dec.graph = None


# ------------------------------------------------------------------------------------------------
# decoder workload
# ------------------------------------------------------------------------------------------------
class DecodeBench:
    """Greedy or teacher-forced bs=1 decode: the whole-token graph (GraphDecoder / DevicePagedDecoder)
    or the segmented paged decoder (PagedGraphDecoder, the reference's per-layer host decision)."""

    def __init__(self, a, device, seed):
        import torch

        from wisp.graphdec import DevicePagedDecoder, GraphDecoder, PagedGraphDecoder
        from wisp.model import DecoderConfig, DecoderWeights

        cfg = DecoderConfig(layers=L, bits=a.bits)
        self.a = a
        # scaled residual init: with the plain init the residual stream of a random model grows a component
        # shared by every token and routing collapses onto ~20 experts per layer in the deep layers; scaled,
        # a token's routing follows the token (~110 of 128 experts per layer over 32 tokens)
        self.w = DecoderWeights.random(cfg, device=device, seed=seed, resid_scale=True)
        n_steps = a.warmup + 2 * a.steps + 3 + TIMELINE_TOKENS
        need = a.prompt + n_steps + 16
        self.paged = a.cache_frac < 1.0
        self.device_paged = self.paged and a.paging == "device"
        self.forced = a.tokens == "forced"
        if self.paged:
            from wisp.cache import ExpertCache
            from wisp.store import ExpertStore

            store = ExpertStore.from_pool(self.w.pool, H * I, a.bits, G, L, E)
            self.w.pool = None  # only the capped slot pool stays on the device
            torch.cuda.empty_cache()
            self.cache = ExpertCache(store, nslots=int(a.cache_frac * L * E), device=device)
            if self.device_paged:
                self.dec = DevicePagedDecoder(self.w, self.cache, tmax=need, admit=a.admit)
            else:
                self.dec = PagedGraphDecoder(self.w, self.cache, tmax=need, prefetch=not a.no_prefetch)
        else:
            self.dec = GraphDecoder(self.w, tmax=need)
        g = torch.Generator(device=device).manual_seed(seed)
        self.prompt = torch.randint(0, cfg.vocab, (a.prompt,), device=device, generator=g)
        # the token stream of the forced steps (seeded random ids, like a prompt being read)
        self.stream = torch.randint(0, cfg.vocab, (n_steps,), device=device, generator=g)
        self.stream_host = self.stream.cpu().pin_memory()
        self.i = 0
        t0 = time.perf_counter()
        self.dec.prefill(self.prompt)
        torch.cuda.synchronize()
        self.prefill_s = time.perf_counter() - t0
        self.tok = self.dec.logits.argmax().reshape(1)
        self.dec.ctl[0:1].copy_(self.tok)
        self.dec.ctl[1].fill_(self.dec.pos)
        if self.dec.graph is None:
            self.dec.capture()
        if self.paged:
            self.stats0 = dict(self.cache.stats), self.cache.bytes_h2d, self.cache.n_loads
        if self.device_paged:
            self.reads0 = self.dec.host_reads_total()
        self.tokens0 = self.dec.pos

    def launches_per_step(self):
        return self.dec.kernels_per_step()  # embed; per layer 3 GEMVs, attention, MoE x2; lm_head; argmax x2

    def step(self, t):
        """One decoded token: the step graph (teacher-forced: this step's token from the device stream;
        greedy: the previous step's choice, advanced inside the graph); paged decoders add their host
        work (the policy one token behind, or the L + 1 segments with per-layer decisions)."""
        if self.forced:
            self.dec.next(self.stream[self.i : self.i + 1])
            self.i += 1
        elif self.device_paged:
            self.dec.step_greedy()
        elif self.paged:
            self.dec.next(self.dec.next_token)
        else:
            self.dec.greedy_graph.replay()

    def e2e_inputs(self):
        import torch

        return self.stream_host, torch.zeros(1, dtype=torch.int64).pin_memory()

    def step_e2e(self, t, inp):
        """Public-API step from host buffers: the token H2D, one decode step, the chosen next token D2H."""
        tok_host, out_host = inp
        d = self.dec
        if self.forced:
            if self.paged and not self.device_paged:
                d.next(tok_host[self.i : self.i + 1].to(d.dev, non_blocking=True))
            else:
                d.ctl[0:1].copy_(tok_host[self.i : self.i + 1], non_blocking=True)
                d.ctl[1].fill_(d.pos)
                d.graph.replay()
                d.pos += 1
                if d.pager is not None:
                    d._after_replay()
            self.i += 1
        elif self.device_paged:
            d.ctl[0:1].copy_(tok_host[0:1], non_blocking=True)
            d.step_greedy()
        elif self.paged:
            d.next(tok_host[0:1].to(d.dev, non_blocking=True))
        else:
            d.ctl[0:1].copy_(tok_host[0:1], non_blocking=True)
            d.greedy_graph.replay()
        out_host.copy_(d.next_token, non_blocking=True)

    def e2e_bytes(self):
        return 8, 8

    def pool(self):
        return (self.cache.gpu if self.paged else self.w.pool), self.w.nbytes

    def paging_stats(self, value_tok_s):
        """Hit rate and PCIe traffic per token over the decode steps so far, the measured pinned H2D
        bandwidth and the PCIe floor it sets (bytes that must cross PCIe per token / H2D GB/s)."""
        if not self.paged:
            return None
        tokens = self.dec.pos - self.tokens0
        st0, b0, n0 = self.stats0
        st = self.cache.stats
        hits, misses = st["hits"] - st0["hits"], st["misses"] - st0["misses"]
        nb = self.w.nbytes
        page_ins = (self.cache.n_loads - n0) / tokens
        out = {
            "slots": self.cache.nslots,
            "tokens": tokens,
            "hit_rate": hits / max(1, hits + misses),
            "misses_per_token": misses / tokens,
            "page_ins_per_token": page_ins,
            "h2d_mb_per_token": (self.cache.bytes_h2d - b0) / tokens / 1e6,
            "mode": "device slot table" if self.device_paged else "per-layer host decision",
            "admit": self.a.admit if self.device_paged else "all",
            "token_stream": self.a.tokens,
        }
        pcie_bytes = (self.cache.bytes_h2d - b0) / tokens
        if self.device_paged:
            reads = (self.dec.host_reads_total() - self.reads0) / tokens
            out["host_store_expert_reads_per_token"] = reads
            out["host_read_mb_per_token"] = reads * nb / 1e6
            pcie_bytes += reads * nb
        gbs = measure_h2d_gbs()
        out["pcie_mb_per_token"] = pcie_bytes / 1e6
        out["pinned_h2d_gbs"] = gbs
        out["pcie_floor_tok_s"] = gbs * 1e9 / pcie_bytes if pcie_bytes > 0 else None
        out["frac_of_pcie_floor"] = value_tok_s / out["pcie_floor_tok_s"] if out["pcie_floor_tok_s"] else None
        return out

    def timeline(self, tokens=None):
        """CUDA-event timeline of ``tokens`` more forced decode steps (untimed): per step the compute
        stream's interval, per page-in batch the copy stream's; returns how much of the copy time ran
        while a step was computing."""
        import torch

        if not self.device_paged or not self.forced:
            return None
        tokens = tokens or TIMELINE_TOKENS
        cache = self.cache
        cache.timeline = []
        st = torch.cuda.current_stream()
        base = torch.cuda.Event(enable_timing=True)
        base.record(st)
        steps = []
        for _ in range(tokens):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            self.step(0)
            e1.record(st)
            steps.append((e0, e1))
        self.dec.flush()
        torch.cuda.synchronize()
        comp = [(base.elapsed_time(a), base.elapsed_time(b)) for a, b in steps]
        copies = [(base.elapsed_time(a), base.elapsed_time(b), nbytes) for a, b, nbytes in cache.timeline]
        cache.timeline = None
        copy_ms = sum(b - a for a, b, _ in copies)
        overl = 0.0
        for a, b, _ in copies:
            for c, d in comp:
                overl += max(0.0, min(b, d) - max(a, c))
        return {
            "tokens": tokens,
            "span_ms": comp[-1][1] - comp[0][0],
            "compute_ms": sum(d - c for c, d in comp),
            "page_in_batches": len(copies),
            "page_in_mb": sum(n for _, _, n in copies) / 1e6,
            "copy_ms": copy_ms,
            "copy_gbs": sum(n for _, _, n in copies) / (copy_ms * 1e-3) / 1e9 if copy_ms > 0 else None,
            "copy_overlapped_frac": overl / copy_ms if copy_ms > 0 else None,
            "steps_ms": [round(d - c, 3) for c, d in comp],
            "copies_ms": [(round(a, 3), round(b, 3)) for a, b, _ in copies],
        }

    def release(self):
        self.dec.graph = self.dec.greedy_graph = None
        if self.paged and not self.device_paged:
            self.dec.segs = None

    def bytes_per_token(self, ctx):
        cfg = self.w.cfg
        attn = (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim * cfg.hidden * 2 + cfg.hidden * cfg.heads * cfg.head_dim * 2
        router = cfg.experts * cfg.hidden * 2
        kv = 2 * cfg.kv_heads * ctx * cfg.head_dim * 2
        return L * (attn + router + K_TOP * self.w.nbytes + kv) + cfg.vocab * cfg.hidden * 2 + cfg.hidden * 2


def measure_h2d_gbs(mb=256, reps=5):
    """Pinned host -> device copy bandwidth (cudaMemcpyAsync of ``mb`` MB, best of ``reps``, CUDA events)."""
    import torch

    src = torch.empty(mb << 20, dtype=torch.uint8).pin_memory()
    dst = torch.empty(mb << 20, dtype=torch.uint8, device="cuda")
    best = 0.0
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dst.copy_(src, non_blocking=True)
        e1.record()
        e1.synchronize()
        best = max(best, src.numel() / (e0.elapsed_time(e1) * 1e-3) / 1e9)
    return best


# ------------------------------------------------------------------------------------------------
# moe-ep workload (config 4 MoE part, strong scaling over the ranks)
# ------------------------------------------------------------------------------------------------
class EPStack:
    """EP_BATCH tokens through the MoE layers with the experts sharded over the ranks; each rank keeps
    EP_BATCH / world tokens.  Routing: seeded logits biased to Zipf(1.1) popularity, softmax top-8."""

    def __init__(self, a, device, rank, world):
        import torch

        from wisp import kernels, quant
        from wisp.ep import ExpertParallelMoE, batched_expert_fn

        assert EP_BATCH % world == 0 and E % world == 0
        self.N, self.El = EP_BATCH // world, E // world
        n = H * I
        self.nb = quant.expert_nbytes(n, a.bits, G)
        # this rank's experts of every layer: slot l * El + e holds expert rank*El + e of layer l
        self.pool = torch.empty((L * self.El, self.nb), dtype=torch.uint8, device=device)
        gen = torch.Generator(device=device).manual_seed(1000 + rank)
        for l in range(L):
            w3 = (torch.randn(self.El, 3, n, device=device, generator=gen) * 0.02).to(torch.bfloat16)
            self.pool[l * self.El : (l + 1) * self.El].copy_(quant.quantize_batch(w3, a.bits, G))
            del w3
        g = torch.Generator(device=device).manual_seed(7)  # the same routing tables on every rank
        rank_pop = torch.randperm(E, device=device, generator=g).float() + 1
        bias = torch.log(rank_pop ** -1.1)
        logits = torch.randn(L, EP_BATCH, E, device=device, generator=g) + bias
        p = torch.softmax(logits.to(torch.bfloat16).float(), -1)
        rw, sel = torch.topk(p, K_TOP, -1)
        rw = (rw / rw.sum(-1, keepdim=True)).to(torch.bfloat16).float()
        lo = rank * self.N
        self.sel, self.rw = sel[:, lo : lo + self.N].contiguous(), rw[:, lo : lo + self.N].contiguous()
        self.distinct = float(torch.tensor([len(torch.unique(sel[l])) for l in range(L)]).float().mean())
        self.norm_w = (1.0 + 0.1 * torch.randn(L, H, device=device, generator=g)).to(torch.bfloat16)
        self.x0 = torch.randn(self.N, H, device=device, generator=gen).to(torch.bfloat16)
        fn = batched_expert_fn(self.pool, lambda l, e: l * self.El + e, n, H, I, a.bits, G,
                               variant={"auto": 0, "mma": 1, "tcgen05": 2}[a.batched_path])
        self.transport = a.transport if a.transport != "auto" else ("p2p" if world > 1 else "nccl")
        assert self.transport == "nccl" or L % 2 == 0, "the p2p buffer sets alternate per layer: use an even layer count"
        self.ep = ExpertParallelMoE(E, K_TOP, H, self.N, fn, device=device, slot_base=lambda l: l * self.El,
                                    transport=self.transport)
        self.h = torch.empty(self.N, H, dtype=torch.bfloat16, device=device)
        self.xn = torch.empty_like(self.h)
        self.kernels = kernels

    def launches_per_step(self):
        # rmsnorm, dispatch, the batched MoE (grouping, permute, gate/up, down, combine), combine per layer
        # (+ the dispatch wait and the return with the p2p transport)
        return L * (10 if self.transport == "p2p" else 8)

    def _body(self):
        self.h.copy_(self.x0)
        for l in range(L):
            self.kernels.rmsnorm(self.h, self.norm_w[l], 1e-6, out=self.xn)
            self.h.add_(self.ep.forward(self.xn, self.sel[l], self.rw[l], layer=l))

    def capture(self):
        """The whole step (all layers, NCCL exchanges included) as one CUDA graph."""
        import torch

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self._body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._body()
        torch.cuda.synchronize()

    def step(self, t):
        self.graph.replay()

    def e2e_inputs(self):
        import torch

        return self.x0.cpu().pin_memory(), torch.empty(self.N, H, dtype=torch.bfloat16).pin_memory()

    def step_e2e(self, t, inp):
        x_host, out_host = inp
        self.x0.copy_(x_host, non_blocking=True)
        self.step(t)
        out_host.copy_(self.h, non_blocking=True)

    def e2e_bytes(self):
        return self.N * H * 2, self.N * H * 2

    def roofline(self, ms_per_step, peak, peak_src, world):
        """Per layer on one GPU: its share of the distinct routed experts' bytes over the step time per
        layer (exchanges, grouping and combine included, so a lower bound on the grouped kernels' rate)."""
        bytes_layer = self.distinct / world * self.nb + 2 * self.N * H * 2
        us = ms_per_step / L * 1e3
        ach = bytes_layer / (us * 1e-6) / 1e9
        return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                # ncu, gate/up + down grids of one 64-token Zipf(1.1) layer
                "traffic": NCU_TRAFFIC_BATCHED_LAYER if world == 1 else None,
                "kernel": "batched MoE layer (dispatch, grouping, gate/up and down grids, combine) per GPU, timed as the "
                "step time / layers", "bytes_per_call": bytes_layer, "us_per_call": us, "peak_source": peak_src}

    def release(self):
        self.graph = None  # graphs holding NCCL calls go before the process group
        self.ep.close()


# ------------------------------------------------------------------------------------------------
def kernel_shares(bench, steps):
    """Device time per kernel over ``steps`` steps (torch profiler, CUDA activity) to stderr.  Kernels
    chained by programmatic dependent launch start before their predecessor ends and wait inside, so
    their durations overlap: the shares point at the heavy kernels, the step time is the bench's."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for t in range(steps):
            bench.step(t)
        torch.cuda.synchronize()
    rows = [(e.key, e.device_time_total, e.count) for e in prof.key_averages() if e.device_time_total > 0]
    tot = sum(r[1] for r in rows) or 1.0
    print(f"kernel shares over {steps} steps (device time, us; PDL-overlapped durations)", file=sys.stderr)
    for name, us, n in sorted(rows, key=lambda r: -r[1])[:25]:
        print(f"{us:12.1f} {n:6d}x {100 * us / tot:6.2f}%  {name[:110]}", file=sys.stderr)


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
    if a.workload == "decoder":
        bench = DecodeBench(a, dev, seed=rank)
        pool, nbytes = bench.pool()
    elif a.workload == "moe-ep":
        bench = EPStack(a, dev, rank, world)
        bench.capture()
        pool, nbytes = bench.pool, bench.nb
    elif a.workload == "gptoss":
        bench = GptOssDecodeBench(a, dev, seed=rank)
        pool, nbytes = None, bench.nb
    elif a.workload == "qwen-batched":
        bench = QwenBatchedBench(a, dev, rank, world)
        pool, nbytes = None, bench.nb
    elif a.workload == "gptoss-moe":
        bench = GptOssStack(a, dev, seed=rank)
        bench.capture()
        pool, nbytes = None, bench.nb
    else:
        W = build_moe_workload(a.bits, dev, seed=rank)
        bench = MoEStack(W)
        bench.capture()
        pool, nbytes = W["pool"], W["nbytes"]
    for t in range(a.warmup):
        bench.step(t)
    torch.cuda.synchronize()
    if a.profile_one_step:
        torch.cuda.cudart().cudaProfilerStart()
        bench.step(a.warmup)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()

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
        bench.step(t)
    e1.record(st)
    barrier()
    clocks.window(w0, time.perf_counter())
    ms = e0.elapsed_time(e1)
    if a.workload in ("gptoss", "qwen-batched"):
        bench.record_routes()
    # e2e: host buffers, copies inside the timed region
    inp = bench.e2e_inputs()
    for t in range(3):
        bench.step_e2e(t, inp)
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e2.record(st)
    for t in range(a.steps):
        bench.step_e2e(t, inp)
    e3.record(st)
    barrier()
    clocks.window(w0, time.perf_counter())
    ms_e2e = e2.elapsed_time(e3)
    clk = clocks.stop()
    if a.workload == "decoder" and bench.paged:
        paging = bench.paging_stats(a.steps / (ms * 1e-3))
        tl = bench.timeline()
        if tl is not None:
            paging["timeline"] = {k: v for k, v in tl.items() if k not in ("steps_ms", "copies_ms")}
            if os.environ.get("WISP_TIMELINE_OUT"):
                with open(os.environ["WISP_TIMELINE_OUT"], "w") as f:
                    json.dump(tl, f)
    if a.workload == "gptoss":
        peak, src = load_peaks()
        src = f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else src
        roof = bench.roofline(ms / a.steps, peak, src, GO_PROMPT + a.warmup + a.steps)
    elif a.workload == "qwen-batched":
        peak, src = load_peaks()
        src = f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else src
        roof = bench.roofline(ms / a.steps, peak, src, QB_CONTEXT + a.warmup + a.steps)
    elif a.workload in ("gptoss-moe", "moe-ep"):
        peak, src = load_peaks()
        src = f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else src
        roof = bench.roofline(ms / a.steps, peak, src) if a.workload == "gptoss-moe" else bench.roofline(ms / a.steps, peak, src, world)
    else:
        roof, _ = moe_roofline(pool, nbytes, a.bits) if pool.shape[0] >= K_TOP * L else (None, None)
    if a.workload == "decoder":
        ctx = bench.dec.pos + a.warmup + 2 * a.steps + 3  # context length at the end of the timed steps
        roof["step_bytes_per_token"] = bench.bytes_per_token(ctx)
        roof["step_achieved_gbs"] = bench.bytes_per_token(ctx) / (ms / a.steps * 1e-3) / 1e9
    if a.kernel_shares > 0:
        kernel_shares(bench, a.kernel_shares)
    t = torch.tensor([ms, ms_e2e], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e = t.tolist()
    if rank == 0:
        cpu_v, cores, sample = cpu_tok_s(
            a, distinct=bench.distinct if a.workload in ("moe-ep", "gptoss-moe", "gptoss", "qwen-batched") else 60.0)
        tok = a.steps * (EP_BATCH if a.workload in ("moe-ep", "qwen-batched")
                         else (a.batch * world if a.workload in ("gptoss-moe", "gptoss") else world))
        h2d, d2h = bench.e2e_bytes()
        line = {
            "metric": metric_name(a),
            "value": tok / (ms * 1e-3),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": a.steps,
            "warmup": a.warmup,
            "ms_per_step": ms / a.steps,
            "higher_is_better": True,
            "scaling": "strong" if a.workload in ("moe-ep", "qwen-batched") else "weak",
            "vs_baseline": None,
            "dtype": f"u{a.bits}->f32 experts, bf16 dense",
            "data": "synthetic",
            "config": workload_config(a, world),
            "e2e": {"value": tok / (ms_e2e * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": roof,
            "cpu_baseline": {"value": cpu_v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
            "gpu_launches": bench.launches_per_step() * a.steps,
            "clocks": clk,
        }
        if a.workload in ("decoder", "gptoss"):
            line["prefill_s"] = bench.prefill_s
        if a.workload == "gptoss":
            line["distinct_experts_per_layer"] = bench.distinct
            line["prefill"] = f"{GO_PROMPT} prompt tokens per sequence fed one position per graph step"
        if a.workload == "decoder" and bench.paged:
            line["paging"] = paging
        if a.workload == "gptoss-moe":
            line["distinct_experts_per_layer"] = bench.distinct
        if a.workload == "qwen-batched":
            line["distinct_experts_per_layer"] = bench.distinct
            line["context"] = f"{QB_CONTEXT} seeded K/V positions per sequence before the warm-up steps"
        if a.workload == "moe-ep":
            line["distinct_experts_per_layer"] = bench.distinct
            # expert bytes each GPU streams per layer (its share of the distinct experts) per layer time
            line["ep_weight_gbs_per_gpu"] = bench.distinct / world * nbytes / (ms / a.steps / L * 1e-3) / 1e9
        print(json.dumps(line), flush=True)
    bench.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
