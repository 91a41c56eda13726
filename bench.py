#!/usr/bin/env python
"""Batch-1 MoE expert-FFN decode benchmark, Qwen3-30B-A3B shape, on B200.

One step = one decode token through all 48 MoE layers, chained
(x_{l+1} = x_l + moe_l(RMSNorm(x_l)), tinygiant/engine.py:229-258 without
attention): per layer the FFN RMSNorm, the router (128 x 2048 fp32), top-8 +
softmax, the 8 chosen experts' gate/up (Q4_0) -> SwiGLU -> Q8_0 requant -> down,
weighted combine.  With --tokens T > 1 a step is T tokens through the batched
path (each expert's weights read once per layer for all its tokens).
Weights: 48 x 128 synthetic Q4_0 experts drawn from N(0, 0.02), all resident in
HBM (16.3 GB); routers N(0, 0.02); a fresh N(0, 1) hidden state per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  Under torchrun with N > 1 the ranks decode the
same token stream with the experts sharded over them (expert parallelism: rank r
holds experts [r*128/N, (r+1)*128/N) of every layer, one persistent kernel per rank
and token, the per-slot down values exchanged over NVLink inside it; strong
scaling); --replicas instead gives each rank its own full model (weak scaling).
Timings are max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
# stdout carries only the JSON result lines: they go to a private copy of the original
# stdout, and file descriptor 1 is pointed at stderr, so whatever libraries print there
# (NCCL's version line when NCCL_DEBUG is set, for one) lands in the log instead
_RESULT = os.fdopen(os.dup(1), "w")
os.dup2(2, 1)


def emit(obj) -> None:
    _RESULT.write(json.dumps(obj) + "\n")
    _RESULT.flush()

METRIC = "expert-FFN decode tok/s (Qwen3-30B-A3B shape) & Q4 weight-read HBM GB/s"
H, I, E, K_TOP, L = 2048, 768, 128, 8, 48
EXPERT_BYTES = 3 * I * (H // 32) * 18                      # 2,654,208
Q4_BYTES_PER_TOKEN = L * K_TOP * EXPERT_BYTES              # 1,019,215,872 (8 distinct experts per layer)
ROUTER_BYTES_PER_TOKEN = L * E * H * 4                     # 50,331,648
PUBLISHED_TOKS = 25.9   # reference README.md:13-23, Apple M1, same 48 x 8 expert decode


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--multi", action="store_true", help="three kernels per layer instead of the fused kernel")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: every rank decodes its own tokens on its own full model (weak scaling) instead "
                         "of the expert-parallel decode of one token stream")
    ap.add_argument("--single-expert", action="store_true",
                    help="configs[0]: single-expert Q4_0 FFN forwards (64 distinct resident experts per step)")
    ap.add_argument("--layers", type=int, default=L, help="fewer layers, for small profiling cases only")
    ap.add_argument("--tokens", type=str, default="1",
                    help="T > 1: T tokens per step through the batched path; with --ep a comma list runs each "
                         "batch size on one filled model (one JSON line each)")
    ap.add_argument("--tier", type=int, default=-1,
                    help="P >= 0: host tier with P experts per layer pinned in HBM, Zipf(1.1) routing (configs[3])")
    ap.add_argument("--cache-slots", type=int, default=24, help="HBM cache slots of the host tier")
    ap.add_argument("--layout", choices=["ggml", "rows"], default="ggml",
                    help="--tier: host bytes as ggml blobs (repacked after each copy) or a version-4 row-split "
                         "relayout (copied as they are)")
    ap.add_argument("--ep", action="store_true",
                    help="expert parallelism: under torchrun each rank holds E/N experts of every layer and "
                         "the ranks decode the same --tokens T tokens together (NCCL all-reduce per layer)")
    ap.add_argument("--p2p", action="store_true",
                    help="with --ep: exchange by direct NVLink stores and flags (tgx_ep_moe_layer_p2p) instead "
                         "of the NCCL all-reduce")
    ap.add_argument("--dispatch", action="store_true",
                    help="with --ep: token dispatch instead of replicated tokens: each rank holds T/N of the "
                         "tokens and sends each (token, slot) pair's Q8_0 row to its expert's holder and gets y "
                         "back (NCCL all-to-alls, tgx_ep_dispatch*)")
    ap.add_argument("--batched-kernels", choices=["auto", "dp4a", "mma", "mma-fast"], default="auto",
                    help="expert matmuls of the batched / EP path: auto (tensor cores from 16 pairs per expert), "
                         "dp4a, or mma (tcgen05), which give the same bits; mma-fast: tcgen05 with the one-fma "
                         "epilogue, within the accumulation-order tolerance instead of bit-identical")
    ap.add_argument("--shape", choices=["qwen3", "dsv3"], default="qwen3",
                    help="with --ep: qwen3 (configs[2]) or the DeepSeek-V3-like configs[4] (hidden 7168, "
                         "inter 2048, 256 routed + 1 shared expert, 58 layers, as many as fit per GPU)")
    ap.add_argument("--attention", action="store_true",
                    help="whole decode layers: the reference's attention step (Q4_K / f16 weights, fp32 KV cache) "
                         "then the MoE block, 48 layers per token in one CUDA graph")
    ap.add_argument("--pos", type=int, default=1024, help="--attention: rows already cached when timing starts")
    ap.add_argument("--head", action="store_true",
                    help="--attention: whole tokens (engine.DecodeEngine): embedding row, the layers, final RMSNorm "
                         "and the f16 output projection over the Qwen3 vocabulary")
    ap.add_argument("--format", choices=["q4_0", "q4_k", "q4_k_m"], default="q4_0",
                    help="q4_k / q4_k_m: the reference library's own formats (all-Q4_K experts, or Q4_K "
                         "gate/up with Q6_K down), expert FFN of 48 layers x top-8 per token")
    return ap.parse_args()


# ---------------------------------------------------------------- distributed

def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def init_dist(ws, backend):
    import torch.distributed as dist
    if ws > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group(backend=backend, timeout=timedelta(seconds=120))
    return dist


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def headline_parallelism(ws: int, replicas: bool) -> tuple[str, str]:
    """(parallelism, scaling) of the headline line at ws ranks."""
    if ws <= 1:
        return "single GPU", "weak"
    return ("replicas", "weak") if replicas else (f"ep{ws}", "strong")


def headline_config(n_layers: int, ws: int, replicas: bool = False) -> dict:
    """The workload of the headline line, printed identically by both arms."""
    return {"workload": f"qwen3-30b-a3b moe decode, batch 1, {n_layers} layers (configs[1])",
            "hidden": H, "inter": I, "experts": E, "top_k": K_TOP, "layers": n_layers,
            "weights": f"Q4_0 of N(0,0.02), {n_layers} layers x {E} experts",
            "hidden_states": "fresh N(0,1) per step",
            "l2": "inputs larger than L2 (1.02 GB of Q4 weights read per step)",
            "parallelism": headline_parallelism(ws, replicas)[0]}


# ---------------------------------------------------------------- CPU arm

def cpu_decode_rate(blobs, routers, seconds: float, threads: int, seed: int):
    """Oracle decode (all 48 layers, layer l uses pool entry l % len(blobs)) on host
    cores; returns (tok/s, tokens, elapsed)."""
    from oracle import oracle as O
    nl = len(blobs)
    lb = [blobs[l % nl] for l in range(L)]
    rs = [routers[l % nl] for l in range(L)]
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(H).astype(np.float32)
    O.decode_step_mt(lb, rs, x, K_TOP, H, I, 1, threads)          # warm-up token
    n, t0 = 0, time.perf_counter()
    while True:
        x = rng.standard_normal(H).astype(np.float32)
        O.decode_step_mt(lb, rs, x, K_TOP, H, I, 1, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 10000:
            return n / el, n, el


def host_pool(seed: int, n_layers: int = 2):
    """Two layers of Q4_0 experts + routers generated on the CPU by the oracle."""
    from oracle import oracle as O
    blobs, routers = [], []
    for l in range(n_layers):
        w = O.fill_normal(E * 3 * H * I, seed * 1000 + 2 * l, 0.02)
        blobs.append(O.quantize_q4_0(w))
        del w
        routers.append(O.fill_normal(E * H, seed * 1000 + 2 * l + 1, 0.02).reshape(E, H))
    return blobs, routers


def run_reference(args):
    """--impl reference: the reference's CPU path for this workload (the oracle port of
    csrc/libtinygiant.c's expert forward with the engine's routing, OpenMP over every
    host thread).  W untimed warm-up steps, then exactly K timed steps; a step is a
    bounded sample of the decode: m MoE layers of one token (48 layers make a token),
    m sized from the warm-up so that the K steps take about a minute at most.  tok/s =
    layers per second / 48.  Under torchrun only rank 0 runs."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import oracle as O
    threads = O.nproc()
    blobs, routers = host_pool(args.seed)
    nl = len(blobs)
    K, W = args.steps, args.warmup
    rng = np.random.default_rng(args.seed + 1)

    def layers(m):   # m chained MoE layers of one token, layer l from pool entry l % nl
        x = rng.standard_normal(H).astype(np.float32)
        O.decode_step_mt([blobs[l % nl] for l in range(m)], [routers[l % nl] for l in range(m)], x, K_TOP, H, I,
                         1, threads)

    layers(1)                                            # thread pool start, outside every count
    t0 = time.perf_counter()
    for _ in range(max(1, W)):
        layers(1)
    t_layer = (time.perf_counter() - t0) / max(1, W)
    budget = min(60.0, max(5.0, 0.02 * K))               # seconds for the K timed steps
    m = max(1, min(L, int(budget / K / t_layer)))
    t0 = time.perf_counter()
    for _ in range(K):
        layers(m)
    el = time.perf_counter() - t0
    rate = K * m / el / L
    sample = (f"{K} steps of {m} MoE layers of one token (48 layers = 1 token), top-{K_TOP} over a 2-layer x "
              f"128-expert Q4_0 pool (680 MB, cycled through the layers), {el:.1f} s, oracle port (C, OpenMP)")
    out = {
        "metric": METRIC, "value": rate, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": K, "warmup": W, "ms_per_step": 1000.0 * el / K, "higher_is_better": True,
        "scaling": headline_parallelism(ws, args.replicas)[1], "vs_baseline": rate / PUBLISHED_TOKS,
        "dtype": "int8", "data": "synthetic",
        "config": headline_config(L, ws, args.replicas),
        "layers_per_step": m,
        "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(out)
    return 0


# ---------------------------------------------------------------- GPU arm

def run_ours(args):
    import torch
    ws, rank, local = dist_env()
    if ws != args.gpus:
        args.gpus = ws
    torch.cuda.set_device(local)
    dist = init_dist(ws, "nccl")
    from tinygiant_b200.engine import MoEModel

    NL = args.layers
    model = MoEModel(H, I, E, K_TOP, NL, device=local)
    model.fill_synthetic(args.seed + 7919 * rank)
    ctas, smem, arena = model.fused_info()
    fused = ctas > 0 and not args.multi
    kernels_per_step = 1 if fused else 3 * NL
    q4_bytes = NL * K_TOP * EXPERT_BYTES
    K, W = args.steps, max(3, args.warmup)
    gen = torch.Generator(device="cuda").manual_seed(args.seed + rank)
    X = torch.randn(K + W, H, generator=gen, device="cuda", dtype=torch.float32)
    x = torch.empty(H, device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream()

    def barrier():
        if ws > 1:
            dist.barrier()

    # ---- device-resident timing (graph replay per step)
    for i in range(W):
        x.copy_(X[i])
        model.decode_step(x, stream, multi=args.multi)
    torch.cuda.synchronize()
    model.sync_status()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # per-launch events bracket the decode launch alone (not the input copy)
    ks = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ke = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev0.record(stream)
    for i in range(K):
        x.copy_(X[W + i])
        ks[i].record(stream)
        model.decode_step(x, stream, multi=args.multi)
        ke[i].record(stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.stop()
    model.sync_status()
    barrier()
    ms = ev0.elapsed_time(ev1)
    if ws > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step_ms = ms / K
    value = ws * K / (ms / 1000.0)

    kernel_ms = float(np.mean([a.elapsed_time(b) for a, b in zip(ks, ke)]))
    if ws > 1:
        t = torch.tensor([kernel_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        kernel_ms = float(t.item())

    # ---- end to end: pinned host input -> decode step -> host result, every step
    Xh = X.cpu().pin_memory()
    Yh = torch.empty_like(Xh).pin_memory()
    for i in range(W):
        x.copy_(Xh[i], non_blocking=True)
        model.decode_step(x, stream, multi=args.multi)
        Yh[i].copy_(x, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        x.copy_(Xh[W + i], non_blocking=True)
        model.decode_step(x, stream, multi=args.multi)
        Yh[W + i].copy_(x, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([ems], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    assert torch.isfinite(Yh[W:W + K]).all()
    e2e = ws * K / (ems / 1000.0)

    # ---- roofline of the dominant launch sequence (the decode step graph)
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    peak_gbs = peaks.get("hbm_gbs", 6650.0)
    # DRAM bytes per launch from the committed ncu summary (4-layer capture scaled to 48)
    traffic = None
    prof = ROOT / "profiles" / "k_decode_fused_qwen3.txt"
    if fused and NL == L and prof.exists():
        for line in prof.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                traffic = int(line.split(":")[1])
    achieved = q4_bytes / (kernel_ms / 1000.0) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s",
                "frac": achieved / peak_gbs, "traffic": traffic,
                "traffic_source": "ncu dram__bytes_read+write, profiles/k_decode_fused_qwen3.txt" if traffic else None,
                "kernel": ("k_decode_fused: one launch per token, all layers" if fused
                           else f"decode step, {kernels_per_step} launches (CUDA graph)"),
                "kernel_ms": kernel_ms,
                "algorithmic_bytes": q4_bytes,
                "algorithmic_bytes_def": "Q4_0 bytes of the k=8 distinct experts read per layer, x layers",
                "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks else "fallback",
                "router_gbs": NL * E * H * 4 / (kernel_ms / 1000.0) / 1e9,
                "fused_ctas": ctas, "fused_smem_bytes": smem}

    # ---- CPU baseline on rank 0 (oracle, all host cores, bounded sample)
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        threads = O.nproc()
        blobs = [model.read_experts(l, 0, E) for l in range(min(2, NL))]
        # host-drawn N(0, 0.02) routers: same distribution as the device ones; the
        # per-token work does not depend on which 8 experts a layer picks
        routers = [O.fill_normal(E * H, args.seed * 1000 + 2 * l + 1, 0.02).reshape(E, H) for l in range(len(blobs))]
        rate, n, el = cpu_decode_rate(blobs, routers, args.cpu_seconds, threads, args.seed)
        cpu = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{n} decode tokens (48 layers x top-8) cycling 2 of this run's Q4_0 layers "
                         f"(680 MB), {el:.1f} s, oracle C port with OpenMP"}

    model.close()
    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / PUBLISHED_TOKS, "dtype": "int8", "data": "synthetic",
            "config": headline_config(NL, ws, True),
            "path": "fused" if fused else "multi-kernel",
            "residency": f"{NL} x {E} experts resident in HBM ({NL * E * EXPERT_BYTES / 1e9:.1f} GB)",
            "q4_weight_gbs": achieved,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": H * 4},
            "gpu_launches": kernels_per_step * K,
            "clocks": clocks.summary(),
        }
        emit(out)
    if ws > 1:
        dist.destroy_process_group()
    return 0


def ep_split(stamps: np.ndarray) -> dict:
    """Per-layer phases of one traced expert-parallel step on one rank, from the kernel's
    globaltimer stamps ([layers][CTAs][32]), µs after the layer's first routing stamp,
    median over layers: partial = every CTA has stored its local slots' down values to
    every rank (routing, gate/up, h exchange, down), exchange = every CTA has received
    all k slots' values (the NVLink stores and the wait for the slowest rank), combine =
    every CTA has combined and sent the next layer's router sums."""
    ns = stamps[:, :, :16].astype(np.int64)
    t0 = ns[:, :, 0].min(axis=1)
    part = ns[:, :, 12].max(axis=1) - t0
    recv = ns[:, :, 13].max(axis=1) - t0
    done = ns[:, :, 7].max(axis=1) - t0
    nl = ns.shape[0]
    layer = np.diff(t0) if nl > 1 else done
    med = lambda a: float(np.median(a[: max(1, nl - 1)])) / 1000.0
    return {"layer_us": med(layer), "partial_us": med(part), "exchange_us": med(recv - part),
            "combine_us": med(done - recv)}


def run_ep_fused(args):
    """N > 1 ranks decode ONE token stream of the configs[1] model together: rank r holds
    experts [r*E/N, (r+1)*E/N) of every layer (tgx_ep_*), every rank routes every layer,
    and one persistent kernel per rank and token (tgx_ep_decode_step) computes the local
    slots and exchanges the per-slot down values over NVLink.  value = tokens of the one
    stream per second (strong scaling); e2e and the per-layer split as in the one-GPU
    line."""
    import torch
    ws, rank, local = dist_env()
    args.gpus = ws
    torch.cuda.set_device(local)
    dist = init_dist(ws, "nccl")
    from tinygiant_b200.ep import EPMoEModel

    NL = args.layers
    model = EPMoEModel(H, I, E, K_TOP, NL, rank=rank, size=ws, device=local)
    model.fill_synthetic(args.seed)          # one model, sharded: the same seed on every rank
    model.enable_fused()
    q4_bytes = NL * K_TOP * EXPERT_BYTES
    K, W = args.steps, max(3, args.warmup)
    gen = torch.Generator(device="cuda").manual_seed(args.seed)   # the same tokens on every rank
    X = torch.randn(K + W, H, generator=gen, device="cuda", dtype=torch.float32)
    x = torch.empty(H, device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream()

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing
    dist.barrier()
    for i in range(W):
        x.copy_(X[i])
        model.decode_step(x, stream)
    torch.cuda.synchronize()
    model.fused_status()
    dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ks = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ke = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev0.record(stream)
    for i in range(K):
        x.copy_(X[W + i])
        ks[i].record(stream)
        model.decode_step(x, stream)
        ke[i].record(stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.stop()
    model.fused_status()
    dist.barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    step_ms = ms / K
    value = K / (ms / 1000.0)
    kernel_ms = max_over_ranks(float(np.mean([a.elapsed_time(b) for a, b in zip(ks, ke)])))

    # ---- end to end: pinned host input -> decode step -> host result, every step, every rank
    Xh = X.cpu().pin_memory()
    Yh = torch.empty_like(Xh).pin_memory()
    dist.barrier()
    for i in range(W):
        x.copy_(Xh[i], non_blocking=True)
        model.decode_step(x, stream)
        Yh[i].copy_(x, non_blocking=True)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        x.copy_(Xh[W + i], non_blocking=True)
        model.decode_step(x, stream)
        Yh[W + i].copy_(x, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    model.fused_status()
    ems = max_over_ranks(e0.elapsed_time(e1))
    assert torch.isfinite(Yh[W:W + K]).all()
    e2e = K / (ems / 1000.0)
    # every rank ends every step with the same hidden state
    last = Yh[W + K - 1].cuda()
    got = [torch.empty_like(last) for _ in range(ws)]
    dist.all_gather(got, last)
    same_state = all(torch.equal(g.view(torch.int32), last.view(torch.int32)) for g in got)

    # ---- per-layer split from one traced step (not timed)
    dist.barrier()
    x.copy_(X[0])
    stamps = model.fused_trace(x, stream)
    model.fused_status()
    split = ep_split(stamps)
    splits = [None] * ws
    dist.all_gather_object(splits, split)
    worst = {kk: max(sp[kk] for sp in splits) for kk in split}
    limiter = max(("partial_us", "exchange_us", "combine_us"), key=lambda kk: worst[kk])

    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    peak_gbs = peaks.get("hbm_gbs", 6650.0)
    achieved = q4_bytes / (kernel_ms / 1000.0) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak_gbs * ws, "unit": "GB/s",
                "frac": achieved / (peak_gbs * ws), "traffic": None,
                "kernel": f"k_decode_fused (experts sharded): one launch per rank and token, all layers, {ws} ranks",
                "kernel_ms": kernel_ms, "algorithmic_bytes": q4_bytes,
                "algorithmic_bytes_def": "Q4_0 bytes of the k=8 distinct experts read per layer, x layers, "
                                         "summed over the ranks (each reads its local slots' experts)",
                "peak_source": ("measured (MEASURED_PEAKS.json hbm_gbs) x ranks" if "hbm_gbs" in peaks
                                else "fallback x ranks")}
    clk = clocks.summary()
    model.close()
    if rank == 0:
        par, scaling = headline_parallelism(ws, False)
        out = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": step_ms, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": value / PUBLISHED_TOKS, "dtype": "int8", "data": "synthetic",
            "config": headline_config(NL, ws),
            "path": "fused, experts sharded over the ranks (tgx_ep_decode_step)",
            "residency": f"{NL} x {E // ws} experts per rank resident in HBM "
                         f"({NL * E // ws * EXPERT_BYTES / 1e9:.1f} GB)",
            "q4_weight_gbs": achieved,
            "roofline": roofline,
            "cpu_baseline": None,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": ws * H * 4, "d2h_bytes_per_step": ws * H * 4},
            "gpu_launches": ws * K, "gpu_launches_per_rank": K,
            "ep_split": {"rank0": split, "max_over_ranks": worst, "limiter": limiter,
                         "nvlink_bytes_per_layer_per_rank": f"~{K_TOP // ws if ws <= K_TOP else 1} local slots x "
                                                            f"{H} rows x 8 B to each of {ws - 1} peers"},
            "ranks_agree": same_state,
            "clocks": clk,
        }
        emit(out)
    dist.destroy_process_group()
    return 0


def run_batched(args):
    """T tokens per step through all layers with the batched kernels (tgx_decode_batched)."""
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = init_dist(ws, "nccl") if ws > 1 else None
    from tinygiant_b200.engine import MoEModel

    T, NL = args.tokens, args.layers
    model = MoEModel(H, I, E, K_TOP, NL, device=local)
    model.fill_synthetic(args.seed + 7919 * rank)
    model.set_batched_kernels(KERNELS[args.batched_kernels])
    K, W = args.steps, max(3, args.warmup)
    gen = torch.Generator(device="cuda").manual_seed(args.seed + rank)
    pool = [torch.randn(T, H, generator=gen, device="cuda") for _ in range(4)]
    X = torch.empty(T, H, device="cuda")
    stream = torch.cuda.current_stream()
    for i in range(W):
        X.copy_(pool[i % 4])
        model.decode_batched(X, stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(K):
        X.copy_(pool[i % 4])                    # fresh hidden states (device copy, 8 KB per token)
        model.decode_batched(X, stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.stop()
    ms = ev0.elapsed_time(ev1)
    # e2e: host pinned tokens in, results out, every step
    Xh = pool[0].cpu().pin_memory()
    Yh = torch.empty_like(Xh).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ke = max(1, K // 4)
    e0.record(stream)
    for i in range(ke):
        X.copy_(Xh, non_blocking=True)
        model.decode_batched(X, stream)
        Yh.copy_(X, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms, ems], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ems = float(t[0]), float(t[1])
    model.close()
    if rank == 0:
        distinct = min(E, T * K_TOP)   # at most this many experts per layer are read
        out = {
            "metric": f"batched MoE decode tok/s (Qwen3-30B-A3B shape, {T} tokens per step)",
            "value": ws * T * K / (ms / 1000.0), "unit": "tok/s", "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"configs[2]: {T} tokens per step, {NL} layers, batched path",
                       "hidden": H, "inter": I, "experts": E, "top_k": K_TOP, "layers": NL, "tokens": T,
                       "batched_kernels": args.batched_kernels,
                       "parallelism": "replicas" if ws > 1 else "single GPU"},
            "weights_read_upper_bound_gbs": NL * distinct * EXPERT_BYTES / (ms / K / 1000.0) / 1e9,
            "e2e": {"value": ws * T * ke / (ems / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": T * H * 4,
                    "d2h_bytes_per_step": T * H * 4},
            "gpu_launches": 7 * NL * K,
            "clocks": clocks.summary(),
        }
        emit(out)
    if dist:
        dist.destroy_process_group()
    return 0


def zipf_routes(n_steps, n_layers, E, k, s, seed):
    """Per layer a seeded permutation of the experts ranked by Zipf(s); per step and
    layer k distinct experts drawn with probability ~ rank^-s.  Returns ids[step][layer][k]
    and the permutations (most popular first)."""
    rng = np.random.default_rng(seed)
    perms = [rng.permutation(E) for _ in range(n_layers)]
    p = 1.0 / np.arange(1, E + 1) ** s
    p /= p.sum()
    ids = np.empty((n_steps, n_layers, k), np.int64)
    for t in range(n_steps):
        for l in range(n_layers):
            ids[t, l] = perms[l][rng.choice(E, size=k, replace=False, p=p)]
    return ids, perms


def run_tier(args):
    """P experts per layer pinned in HBM, the rest copied on demand from a
    pinned host copy of the relayout bytes into HBM cache slots on a side stream, the
    next layer's misses prefetched while the current layer computes."""
    import ctypes
    import torch
    from tinygiant_b200.cache import HostTierCache
    from tinygiant_b200.engine import MoEModel
    torch.cuda.set_device(0)
    NL, P = args.layers, args.tier
    model = MoEModel(H, I, E, K_TOP, NL)
    model.fill_synthetic(args.seed)
    from tinygiant_b200 import relayout as RL
    host = []
    for l in range(NL):   # the relayout bytes of each layer in pinned host memory
        t = torch.empty(E * EXPERT_BYTES, dtype=torch.uint8, pin_memory=True)
        r = model.lib.tgx_read_experts(model.handle, l, 0, E, ctypes.c_void_p(t.data_ptr()))
        assert r == 0
        if args.layout == "rows":   # as a version-4 relayout stores them
            v = t.numpy()
            for e in range(E):
                v[e * EXPERT_BYTES:(e + 1) * EXPERT_BYTES] = RL.expert_convert(
                    v[e * EXPERT_BYTES:(e + 1) * EXPERT_BYTES], H, I, True)
        host.append(t)
    K, W = args.steps, max(3, args.warmup)
    ids, perms = zipf_routes(K + W, NL, E, K_TOP, 1.1, args.seed + 1)
    cache = HostTierCache(model, host, cache_slots=args.cache_slots, layout=args.layout)
    for l in range(NL):
        cache.pin(l, perms[l][:P])
    w = np.full(K_TOP, 1.0 / K_TOP, np.float32)
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    X = torch.randn(K + W, H, generator=gen, device="cuda")
    stream = torch.cuda.current_stream()

    def token(i):
        x = X[i]
        for l in range(NL):
            nl, ni = (l + 1, i) if l + 1 < NL else (0, i + 1)
            if ni < K + W:
                cache.prefetch(nl, ids[ni, nl])
            cache.forward(l, ids[i, l], w, x, stream)

    for i in range(W):
        token(i)
    torch.cuda.synchronize()
    h0, m0, b0 = cache.hits, cache.misses, cache.bytes_h2d
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    t0 = time.perf_counter()
    for i in range(W, W + K):
        token(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = ev0.elapsed_time(ev1)
    hits, misses, nbytes = cache.hits - h0, cache.misses - m0, cache.bytes_h2d - b0
    model.close()
    emit(({
        "metric": f"host-tier expert decode tok/s (Qwen3-30B-A3B shape, {P} experts per layer pinned in HBM)",
        "value": K / (ms / 1000.0), "unit": "tok/s", "n_gpus": 1, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"configs[3]: {NL} layers, top-{K_TOP} by Zipf(1.1) routing, {P} pinned per layer, "
                               f"{args.cache_slots} HBM cache slots, relayout bytes in pinned host memory "
                               f"({args.layout} layout)",
                   "layers": NL, "pinned_per_layer": P, "cache_slots": args.cache_slots, "layout": args.layout},
        "hit_rate": hits / max(1, hits + misses), "misses_per_token": misses / K,
        "h2d_gbs": nbytes / (ms / 1000.0) / 1e9, "wall_tok_s": K / wall,
    }))
    return 0


KERNELS = {"auto": 0, "dp4a": 1, "mma": 2, "mma-fast": 3}
Q4K_BLOCK, Q6K_BLOCK = 144, 210


def kq_sizes(fmt):
    gu = I * (H // 256) * Q4K_BLOCK                      # one Q4_K gate (or up) matrix
    down = H * (I // 256) * (Q6K_BLOCK if fmt == "q4_k_m" else Q4K_BLOCK)
    return gu, down


def run_kquant(args):
    """The reference's own kernel-library formats (csrc/libtinygiant.c:555-655) at the
    benchmark shape: per layer tg_moe_forward of the token's 8 experts (Q4_K gate/up,
    Q4_K or Q6_K down), x += sum_j w_j expert_j(x), 48 layers chained, one CUDA graph
    per token (96 launches).  Routes: uniformly drawn distinct experts per layer."""
    import ctypes
    import torch
    from tinygiant_b200._lib import check, get_lib
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = init_dist(ws, "nccl") if ws > 1 else None
    lib = get_lib()
    dev = torch.device("cuda", local)
    fmt = args.format
    NL = args.layers
    down_fmt = 2 if fmt == "q4_k_m" else 0
    gub, db = kq_sizes(fmt)
    expert_bytes = 2 * gub + db
    gen = torch.Generator(device="cuda").manual_seed(args.seed + 7919 * rank)
    s = torch.cuda.current_stream()
    sp = ctypes.c_void_p(s.cuda_stream)

    def fp16_bytes(n, lo, hi, scale=1.0):
        v = torch.empty(n, dtype=torch.float32, device=dev).uniform_(lo, hi, generator=gen)
        return (v * scale).half().view(torch.uint8), v

    def set_q4k_scales(blk):
        # dmin ~ 7.5 d keeps the dequantised weights near zero mean (bounded activations
        # over 48 chained layers); the values do not change the work
        d16, v = fp16_bytes(blk.shape[0], 5e-5, 1.5e-4)
        blk[:, 0:2] = d16.view(-1, 2)
        blk[:, 2:4] = (v * 7.5).half().view(torch.uint8).view(-1, 2)

    gu, dn = [], []
    raw = torch.empty(E * db, dtype=torch.uint8, device=dev) if down_fmt == 2 else None
    for l in range(NL):
        g = torch.randint(0, 256, (E * 2 * gub,), dtype=torch.uint8, device=dev, generator=gen)
        set_q4k_scales(g.view(-1, Q4K_BLOCK))
        d = torch.empty(E * db, dtype=torch.uint8, device=dev)
        if down_fmt == 0:
            d.random_(0, 256, generator=gen)
            set_q4k_scales(d.view(-1, Q4K_BLOCK))
        else:
            raw.random_(0, 256, generator=gen)
            b = raw.view(-1, Q6K_BLOCK)
            b[:, 208:210] = fp16_bytes(b.shape[0], 2e-5, 6e-5)[0].view(-1, 2)
            for e in range(E):
                check(lib.tgx_kq_prepare(2, ctypes.c_void_p(raw.data_ptr() + e * db),
                                         ctypes.c_void_p(d.data_ptr() + e * db), H, I, sp), lib)
        gu.append(g)
        dn.append(d)
    torch.cuda.synchronize()

    K, W = args.steps, max(3, args.warmup)
    S = min(K + W, 64)
    rng = np.random.default_rng(args.seed + rank)
    pool = np.empty((S, NL, 3, K_TOP), np.int64)
    for t in range(S):
        for l in range(NL):
            ids = rng.choice(E, size=K_TOP, replace=False)
            pool[t, l, 0] = gu[l].data_ptr() + ids * 2 * gub
            pool[t, l, 1] = gu[l].data_ptr() + ids * 2 * gub + gub
            pool[t, l, 2] = dn[l].data_ptr() + ids * db
    pool_d = torch.from_numpy(pool).to(dev)
    ptrs = torch.empty((NL, 3, K_TOP), dtype=torch.int64, device=dev)
    wts = torch.full((K_TOP,), 1.0 / K_TOP, dtype=torch.float32, device=dev)
    x = torch.empty(H, dtype=torch.float32, device=dev)
    sb = lib.tgx_kq_scratch_bytes(K_TOP, H, I)
    scratch = torch.zeros(sb, dtype=torch.uint8, device=dev)
    X = torch.randn(K + W, H, generator=gen, device=dev) * 0.05

    def token(stream_ptr):
        for l in range(NL):
            base = ptrs.data_ptr() + l * 3 * K_TOP * 8
            check(lib.tgx_kq_experts_forward(ctypes.c_void_p(base), ctypes.c_void_p(base + K_TOP * 8),
                                             ctypes.c_void_p(base + 2 * K_TOP * 8), down_fmt, K_TOP,
                                             ctypes.c_void_p(wts.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                             ctypes.c_void_p(x.data_ptr()), H, I, 1,
                                             ctypes.c_void_p(scratch.data_ptr()), sb, 1 if l else 0,
                                             stream_ptr), lib)

    ptrs.copy_(pool_d[0])
    x.copy_(X[0])
    token(sp)                                     # eager once (sets kernel attributes)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        token(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    for i in range(W):
        ptrs.copy_(pool_d[i % S])
        x.copy_(X[i])
        graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ks = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ke = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev0.record(s)
    for i in range(K):
        ptrs.copy_(pool_d[(W + i) % S])
        x.copy_(X[W + i])
        ks[i].record(s)
        graph.replay()
        ke[i].record(s)
    ev1.record(s)
    torch.cuda.synchronize()
    clocks.stop()
    ms = ev0.elapsed_time(ev1)
    graph_ms = float(np.mean([a.elapsed_time(b) for a, b in zip(ks, ke)]))
    assert torch.isfinite(x).all()
    # e2e: pinned host token in, result out, every step
    Xh = X.cpu().pin_memory()
    Yh = torch.empty_like(Xh).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(K):
        ptrs.copy_(pool_d[(W + i) % S])
        x.copy_(Xh[W + i], non_blocking=True)
        graph.replay()
        Yh[W + i].copy_(x, non_blocking=True)
    e1.record(s)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms, ems, graph_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ems, graph_ms = float(t[0]), float(t[1]), float(t[2])
    del graph

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        host_g = gu[0][:2 * gub].cpu().numpy()
        host_d = (raw[:db] if down_fmt == 2 else dn[0][:db]).cpu().numpy()
        xs = X[0].cpu().numpy()
        t0, n_ex = time.perf_counter(), 0
        while True:
            out = np.zeros(H, np.float32)
            O.expert_forward_k(host_g[:gub], host_g[gub:], host_d, down_fmt, xs, out, 0.125, H, I)
            n_ex += 1
            el = time.perf_counter() - t0
            if el >= min(args.cpu_seconds, 8.0) or n_ex >= 4000:
                break
        rate = n_ex / el / (NL * K_TOP)
        cpu = {"value": rate, "unit": "tok/s", "cores": 1, "kind": "port",
               "sample": f"{n_ex} expert forwards ({fmt}, one expert repeated), {el:.1f} s, oracle C port "
                         f"single-threaded, scaled by {NL * K_TOP} expert forwards per token"}
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    alg = NL * K_TOP * expert_bytes
    achieved = alg / (graph_ms / 1000.0) / 1e9
    if rank == 0:
        emit(({
            "metric": f"expert-FFN decode tok/s, reference formats ({fmt.upper()}, Qwen3-30B-A3B shape)",
            "value": ws * K / (ms / 1000.0), "unit": "tok/s", "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{NL} layers x top-{K_TOP} experts, {fmt} weights "
                                   f"({expert_bytes} B per expert), tg_moe_forward per layer, batch 1",
                       "hidden": H, "inter": I, "experts": E, "layers": NL, "format": fmt,
                       "l2": f"inputs larger than L2 ({alg / 1e9:.2f} GB of weights read per step)",
                       "parallelism": "replicas" if ws > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "kernel": f"token graph: {2 * NL} launches (k_kq gate/up, k_kq down)",
                         "graph_ms": graph_ms, "algorithmic_bytes": alg,
                         "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks else "fallback"},
            "cpu_baseline": cpu,
            "e2e": {"value": ws * K / (ems / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": H * 4,
                    "d2h_bytes_per_step": H * 4},
            "gpu_launches": 2 * NL * K,
            "clocks": clocks.summary(),
        }))
    if dist:
        dist.destroy_process_group()
    return 0


def run_layers(args):
    """Whole decode layers at the Qwen3-30B-A3B shape, as the reference engine runs them
    (tinygiant/engine.py:199-258): x += attention(RMSNorm(x)) by the tg_attention_decode_q4
    step (Q4_K wq / wk / wo, f16 wv, fp32 KV cache, 32 query / 4 kv heads of 128), then the
    MoE block (router, top-8, Q4_0 experts), for 48 layers; one CUDA graph per token, the
    cache position read on the device.  Every step is a new token at the next position."""
    import torch
    from tinygiant_b200.engine import AttentionModel, MoEModel
    from tinygiant_b200 import _constants as C
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = init_dist(ws, "nccl") if ws > 1 else None
    NL, K, W, P0 = args.layers, args.steps, max(3, args.warmup), args.pos
    kv_max = P0 + K + W + 2
    NH, NKV, HD = C.N_HEADS, C.N_KV_HEADS, C.HEAD_DIM
    moe = MoEModel(H, I, E, K_TOP, NL, device=local)
    moe.fill_synthetic(args.seed + 7919 * rank)
    am = AttentionModel(H, NH, NKV, HD, NL, kv_max=kv_max, q4=True, device=local)
    am.fill_synthetic(args.seed + 31 + 7919 * rank)
    gen = torch.Generator(device="cuda").manual_seed(args.seed + rank)
    X = torch.randn(K + W, H, generator=gen, device="cuda", dtype=torch.float32)
    x = torch.empty(H, device="cuda", dtype=torch.float32)
    s = torch.cuda.current_stream()
    eng = None
    if args.head:   # whole tokens: embedding row, the layers, final norm, output projection
        from tinygiant_b200.engine import DecodeEngine
        eng = DecodeEngine.synthetic(moe, am, C.VOCAB_SIZE, args.seed + 97 + rank)
        toks = np.random.default_rng(args.seed + rank).integers(0, C.VOCAB_SIZE, K + W)

    def step(i):   # token i of the run, at position P0 + i
        if eng is not None:
            eng.forward_one_token(int(toks[i]), P0 + i, s)
        else:
            am.decode_token(x, moe, s)

    am.reset(P0)
    for i in range(W):
        x.copy_(X[i])
        step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ks = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ke = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev0.record(s)
    for i in range(K):
        x.copy_(X[W + i])
        ks[i].record(s)
        step(W + i)
        ke[i].record(s)
    ev1.record(s)
    torch.cuda.synchronize()
    clocks.stop()
    assert am.status() == P0 + W + K
    moe.sync_status()
    assert torch.isfinite(x).all()
    ms = ev0.elapsed_time(ev1)
    tok_ms = float(np.mean([a.elapsed_time(b) for a, b in zip(ks, ke)]))
    # e2e: pinned host token in, hidden state out, every step, from the same position
    Xh = X.cpu().pin_memory()
    Yh = torch.empty_like(Xh).pin_memory()
    am.reset(P0 + W)
    if eng is not None:
        eng.next_pos = P0 + W
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(K):
        if eng is not None:   # the greedy token loop: the chosen token read back every step
            eng.forward_one_token(int(toks[W + i]), P0 + W + i, s)
            int(torch.argmax(eng.logits).item())
        else:
            x.copy_(Xh[W + i], non_blocking=True)
            am.decode_token(x, moe, s)
            Yh[W + i].copy_(x, non_blocking=True)
    e1.record(s)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    am.status()
    if dist:
        t = torch.tensor([ms, ems, tok_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ems, tok_ms = float(t[0]), float(t[1]), float(t[2])

    wq, wk, wv, wo = am.matrix_bytes()
    attn_w = wq + wk + wv + wo
    seq_mean = P0 + W + (K + 1) / 2.0                       # rows attended, averaged over the timed tokens
    kv_read = 2 * NKV * HD * 4 * seq_mean
    alg = NL * (attn_w + kv_read + K_TOP * EXPERT_BYTES)
    if eng is not None:
        alg += C.VOCAB_SIZE * H * 2 + H * 4                 # the f16 output projection, the embedding row
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        rng = np.random.default_rng(args.seed)
        qd, kvd = NH * HD, NKV * HD

        def q4k(nbytes):
            b = rng.integers(0, 256, size=(nbytes // 144, 144), dtype=np.uint8)
            b[:, 0:4] = np.asarray(rng.uniform(5e-5, 1.5e-4, (b.shape[0], 2)), np.float16).view(np.uint8)
            return b.ravel()

        Wh = (q4k(wq), q4k(wk), (rng.standard_normal(kvd * H) * 0.02).astype(np.float16).view(np.uint16), q4k(wo))
        ones = np.ones(HD, np.float32)
        seq = int(seq_mean)
        kk = np.zeros((NKV, seq + 1, HD), np.float32)
        vv = np.zeros((NKV, seq + 1, HD), np.float32)
        cos, sin = np.ones((1, HD // 2), np.float32), np.zeros((1, HD // 2), np.float32)
        blob = moe.read_experts(0, 0, E)
        R = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
        xs = X[0].cpu().numpy()
        t0, n_layers = time.perf_counter(), 0
        while True:
            nrm = O.rms_norm_k(xs, np.ones(H, np.float32), 1e-6)
            out = O.attention_decode(True, *Wh, ones, ones, kk, vv, seq, cos, sin, nrm, H, NH, NKV, HD, 0)
            xs = O.moe_block(blob, R, (xs + out).astype(np.float32), K_TOP, H, I)[0]
            n_layers += 1
            el = time.perf_counter() - t0
            if el >= min(args.cpu_seconds, 10.0) or n_layers >= 200:
                break
        cpu = {"value": n_layers / el / NL, "unit": "tok/s", "cores": 1, "kind": "port",
               "sample": f"{n_layers} whole layers (attention at {seq} cached rows + MoE block), {el:.1f} s, "
                         f"oracle C port single-threaded, scaled by {NL} layers per token"}
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = alg / (tok_ms / 1000.0) / 1e9
    if rank == 0:
        emit({
            "metric": ("decode tok/s, whole tokens (embedding, attention + MoE layers, output projection, "
                       "Qwen3-30B-A3B shape)") if eng is not None else
                      "decode tok/s, whole layers (attention + MoE, Qwen3-30B-A3B shape)",
            "value": ws * K / (ms / 1000.0), "unit": "tok/s", "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{NL} decode layers per token: attention (Q4_K / f16, fp32 KV cache, "
                                   f"positions {P0 + W}..{P0 + W + K - 1}) then the MoE block (top-{K_TOP} of {E} "
                                   f"Q4_0 experts)" + (f"; final RMSNorm and the f16 output projection over "
                                                       f"{C.VOCAB_SIZE} tokens" if eng is not None else ""),
                       "hidden": H, "inter": I, "experts": E, "layers": NL,
                       "heads": NH, "kv_heads": NKV, "head_dim": HD, "kv_max": kv_max,
                       "l2": f"inputs larger than L2 ({alg / 1e9:.2f} GB read per token)",
                       "parallelism": "replicas" if ws > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "kernel": f"token graph: {NL} x (RMSNorm, 6 attention kernels, fused MoE "
                                                    f"layer) + position advance", "token_ms": tok_ms,
                         "algorithmic_bytes": alg,
                         "algorithmic_bytes_def": "per layer: Q4_K/f16 attention weights + K and V rows read "
                                                  "(mean position) + Q4_0 bytes of the 8 experts"
                                                  + ("; + the f16 output matrix and one embedding row per token"
                                                     if eng is not None else ""),
                         "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks else "fallback"},
            "cpu_baseline": cpu,
            "e2e": {"value": ws * K / (ems / 1000.0), "unit": "tok/s",
                    "h2d_bytes_per_step": 0 if eng is not None else H * 4,   # a token id is a host scalar
                    "d2h_bytes_per_step": 8 if eng is not None else H * 4},  # the greedy token, or x
            "gpu_launches": (8 * NL + 1 + (2 if eng is not None else 0)) * K,
            "clocks": clocks.summary(),
        })
    am.close()
    moe.close()
    if dist:
        dist.destroy_process_group()
    return 0


def run_ep(args):
    """Expert parallelism (configs 3 / 5 at the Qwen3 shape): rank r holds experts
    [r*E/N, (r+1)*E/N) of all 48 layers; every rank routes the same T tokens, runs its
    local experts, the ranks all-reduce the per-(token, slot) outputs over NCCL and
    combine in slot order.  The job processes T tokens per step (strong scaling)."""
    import torch
    from tinygiant_b200.ep import EPMoEModel
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = init_dist(ws, "nccl") if ws > 1 else None
    T = args.tokens
    if args.shape == "dsv3":
        h, inter, e_all, n_sh, full_layers = 7168, 2048, 256, 1, 58
    else:
        h, inter, e_all, n_sh, full_layers = H, I, E, 0, L
    eb = 3 * inter * (h // 32) * 18
    per_layer = (e_all // ws + n_sh) * eb + e_all * h * 4
    if args.shape == "dsv3":   # per-layer subset: the layers that fit this GPU (all 58 from 8 GPUs up)
        free, _ = torch.cuda.mem_get_info()
        NL = max(1, min(full_layers, int(0.85 * (free - (8 << 30)) // per_layer)))
        if dist:
            t = torch.tensor([NL], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            NL = int(t.item())
        if args.layers != L:
            NL = min(NL, args.layers)
    else:
        NL = args.layers
    ep = EPMoEModel(h, inter, e_all, K_TOP, NL, rank=rank, size=ws, device=local, n_shared=n_sh)
    ep.fill_synthetic(args.seed)                          # one model, sharded: the same seed on every rank
    ep.set_kernels(KERNELS[args.batched_kernels])
    if args.p2p and not args.dispatch:
        ep.enable_p2p(max(args.token_list))
    if args.p2p and args.dispatch:   # device-side dispatch: regions sized for a rank's largest share
        ep.enable_dispatch_p2p(-(-max(args.token_list) // ws))
    for T in args.token_list:
        ep_measure(args, ep, T, NL, h, inter, e_all, n_sh, full_layers, eb, ws, rank, local, dist)
    ep.close()
    if dist:
        dist.destroy_process_group()
    return 0


def ep_measure(args, ep, T, NL, h, inter, e_all, n_sh, full_layers, eb, ws, rank, local, dist):
    import torch
    K, W = args.steps, max(3, args.warmup)
    gen = torch.Generator(device="cuda").manual_seed(args.seed + 1)
    disp = args.dispatch
    # token dispatch: this rank's share [lo, lo + Tl) of the step's T tokens
    sizes = [len(c) for c in torch.tensor_split(torch.arange(T), ws)] if disp else [T] * ws
    lo, Tl = sum(sizes[:rank]) if disp else 0, sizes[rank]
    pool = [torch.randn(T, h, generator=gen, device="cuda")[lo:lo + Tl].contiguous() for _ in range(4)]
    X = torch.empty(Tl, h, device="cuda")
    stream = torch.cuda.current_stream()
    X.copy_(pool[0])
    stats = {}
    dev_disp = disp and args.p2p                          # token dispatch through the IPC regions
    rb = ep.record_bytes()

    def one(Xs):
        if dev_disp:
            ep.decode_dispatch_p2p(Xs)
        elif disp:
            ep.decode_dispatch(Xs)
        else:
            ep.decode(Xs)

    if dev_disp:   # bytes received, layer by layer (untimed, synchronising)
        for layer in range(NL):
            ep.moe_layer_dispatch_p2p(layer, X)
            n_recv, n_sent = ep.dispatch_p2p_counts()
            stats["recv_bytes"] = stats.get("recv_bytes", 0) + n_recv * rb + n_sent * h * 4
            stats["layers"] = stats.get("layers", 0) + 1
        ep.dispatch_p2p_status()
    elif disp:
        ep.decode_dispatch(X, stats=stats)                # grows the buffers; counts the bytes received
    else:
        ep.decode(X)                                      # allocates scratch and the exchange buffer
    torch.cuda.synchronize()
    graph, graphed = torch.cuda.CUDAGraph(), False
    if disp and not dev_disp:
        graph = None                                      # the all-to-all sizes come from the host each layer
    else:
        try:
            with torch.cuda.graph(graph):
                one(X)
            graphed = True
        except Exception:                                 # eager launches otherwise (same kernels)
            graph = None
    torch.cuda.synchronize()

    def step():
        if graphed:
            graph.replay()
        else:
            one(X)

    for i in range(W):
        X.copy_(pool[i % 4])
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(K):
        X.copy_(pool[i % 4])
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.stop()
    ms = ev0.elapsed_time(ev1)
    recv_layer = stats.get("recv_bytes", 0) / max(1, stats.get("layers", 1))
    if dist and disp:
        t = torch.tensor([recv_layer], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        recv_layer = float(t.item())
    Xh = pool[1].cpu().pin_memory()
    Yh = torch.empty_like(Xh).pin_memory()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ke = max(1, K // 4)
    e0.record(stream)
    for i in range(ke):
        X.copy_(Xh, non_blocking=True)
        step()
        Yh.copy_(X, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms, ems], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ems = float(t[0]), float(t[1])
    if getattr(ep, "p2p", False) and not disp:
        ep.p2p_status()                                   # raises if a peer's flag wait expired
    if dev_disp:
        ep.dispatch_p2p_status()
    ep.status()
    assert torch.isfinite(Yh).all()
    del graph                                             # holds NCCL calls: released before the group
    if rank == 0:
        distinct = min(e_all, T * K_TOP)
        name = "DeepSeek-V3-like shape" if args.shape == "dsv3" else "Qwen3-30B-A3B shape"
        value = T * K / (ms / 1000.0)
        # expected distinct routed experts per layer under uniform routing, + the shared one
        exp_distinct = e_all * (1.0 - (1.0 - K_TOP / e_all) ** T) + n_sh
        alg = NL * exp_distinct * eb
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
        peak = peaks.get("hbm_gbs", 6650.0)
        achieved = alg / (ms / K / 1000.0) / 1e9
        emit(({
            "metric": f"expert-parallel MoE decode tok/s ({name}, {T} tokens per step, EP over {ws} GPUs)",
            "value": value, "unit": "tok/s", "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{'configs[4]' if args.shape == 'dsv3' else 'configs[2]'}: {T} tokens per step, "
                                   f"{NL} of {full_layers} layers, experts sharded {e_all // ws} per GPU"
                                   f"{' + the shared expert' if n_sh else ''}, "
                                   + ("tokens sharded, pairs dispatched to their experts' holders and back "
                                      + ("(NVLink stores into the ranks' regions, device-side)" if dev_disp
                                         else "(NCCL all-to-alls)") if disp else
                                      f"{'NVLink stores + flags' if args.p2p else 'NCCL all-reduce'} of y per layer"),
                       "hidden": h, "inter": inter, "experts": e_all, "shared_experts": n_sh, "top_k": K_TOP,
                       "layers": NL, "full_layers": full_layers, "tokens": T, "parallelism": f"ep{ws}",
                       "cuda_graph": graphed, "batched_kernels": args.batched_kernels,
                       "exchange": ("dispatch_p2p" if dev_disp else "dispatch") if disp else
                                   ("p2p" if args.p2p else "nccl_all_reduce")},
            "tok_s_full_depth": value * NL / full_layers,
            "exchange_bytes_per_layer": T * (K_TOP + n_sh) * h * 4,
            "recv_bytes_per_layer_per_rank": (recv_layer if disp else T * (K_TOP + n_sh) * h * 4),
            "recv_bytes_def": ("max over ranks of the records (16 B + Q8_0 row) and y rows (4 B x hidden) "
                               "a rank receives per layer" if disp else
                               "y of every (token, slot) pair, which every rank receives"),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak * ws, "unit": "GB/s",
                         "frac": achieved / (peak * ws), "traffic": None,
                         "algorithmic_bytes": alg,
                         "algorithmic_bytes_def": "expected distinct experts per layer (uniform routing) + shared, "
                                                  "x expert bytes x layers; peak = per-GPU peak x GPUs",
                         "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks else "fallback"},
            "e2e": {"value": T * ke / (ems / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": T * h * 4,
                    "d2h_bytes_per_step": T * h * 4},
            "gpu_launches": ((12 if dev_disp else 9 if disp else 6) + (1 if args.shape == "dsv3" else 0)) * NL * K,
            "clocks": clocks.summary(),
        }))


def run_single(args):
    """the single-expert fused Q4_0 x Q8_0 SwiGLU FFN (gate / up 768 x 2048,
    down 2048 x 768, N(0, 0.02) weights; x ~ N(0, 1)), out += w * expert(x) through
    tgx_expert_forward.  One expert is 2.65 MB, which fits the 126 MB L2, so a step is
    64 forwards over 64 distinct resident experts (170 MB; steps alternate between the
    two halves of a 128-expert layer), replayed from a CUDA graph."""
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = init_dist(ws, "nccl")
    from tinygiant_b200.engine import MoEModel
    B = 64
    model = MoEModel(H, I, E, K_TOP, 1, device=local)
    model.fill_synthetic(args.seed + 7919 * rank)
    K, W = args.steps, max(3, args.warmup)
    gen = torch.Generator(device="cuda").manual_seed(args.seed + rank)
    X = torch.randn(B, H, generator=gen, device="cuda")
    Y = torch.zeros(B, H, device="cuda")
    stream = torch.cuda.Stream()
    graphs = []
    with torch.cuda.stream(stream):
        for j in range(B):                       # the first call sets up the expert table
            model.expert_forward(0, j, X[j], Y[j], 0.125, stream)
        stream.synchronize()
        for half in range(2):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for j in range(B):
                    model.expert_forward(0, half * B + j, X[j], Y[j], 0.125, stream)
            graphs.append(g)
    torch.cuda.synchronize()

    def barrier():
        if ws > 1:
            dist.barrier()

    for i in range(W):
        with torch.cuda.stream(stream):
            graphs[i % 2].replay()
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * K + 2)]
    with torch.cuda.stream(stream):
        ev[0].record(stream)
        for i in range(K):
            ev[2 + 2 * i].record(stream)
            graphs[i % 2].replay()
            ev[3 + 2 * i].record(stream)
        ev[1].record(stream)
    torch.cuda.synchronize()
    clocks.stop()
    ms = ev[0].elapsed_time(ev[1])
    step_ms = float(np.mean([ev[2 + 2 * i].elapsed_time(ev[3 + 2 * i]) for i in range(K)]))
    if ws > 1:
        t = torch.tensor([ms, step_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, step_ms = float(t[0]), float(t[1])
    value = ws * K * B / (ms / 1000.0)
    # end to end: the step's inputs from pinned host memory, its outputs back
    Xh = X.cpu().pin_memory()
    Yh = torch.empty_like(Xh).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(K):
            X.copy_(Xh, non_blocking=True)
            graphs[i % 2].replay()
            Yh.copy_(Y, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([ems], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    assert torch.isfinite(Yh).all()
    e2e = ws * K * B / (ems / 1000.0)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = B * EXPERT_BYTES / (step_ms / 1000.0) / 1e9
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        n_pool = 64    # 170 MB of host experts: read from DRAM, not the CPU caches
        pool = O.quantize_q4_0(O.fill_normal(n_pool * 3 * H * I, args.seed, 0.02))
        x = O.fill_normal(H, args.seed + 1, 1.0)
        out = np.zeros(H, np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < min(args.cpu_seconds, 10.0):
            e = n % n_pool
            O.expert_forward(pool[e * EXPERT_BYTES:(e + 1) * EXPERT_BYTES], x, out, 0.125, H, I, 1)
            n += 1
        el = time.perf_counter() - t0
        cpu = {"value": n / el, "unit": "forwards/s", "cores": 1, "kind": "port",
               "sample": f"{n} expert forwards over {n_pool} host experts (170 MB), {el:.1f} s, oracle C port, "
                         f"one thread (the reference's expert forward is single-threaded)"}
    for g in graphs:
        del g
    model.close()
    if rank == 0:
        emit({
            "metric": "single-expert Q4_0 FFN forwards/s (configs[0]) & Q4 weight-read HBM GB/s", "value": value,
            "unit": "forwards/s", "n_gpus": ws, "steps": K, "warmup": W, "ms_per_step": ms / K,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": "single-expert fused Q4_0 x Q8_0 SwiGLU FFN (configs[0])", "hidden": H,
                       "inter": I, "forwards_per_step": B, "distinct_experts": 2 * B,
                       "weights": "Q4_0 of N(0,0.02)", "inputs": "N(0,1), resident",
                       "l2": f"each step reads {B} distinct experts ({B * EXPERT_BYTES / 1e6:.0f} MB > L2)",
                       "parallelism": "replicas" if ws > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None,
                         "kernel": "k_gateup + k_down_combine per expert (tgx_expert_forward), 64 per graph",
                         "kernel_ms": step_ms, "algorithmic_bytes": B * EXPERT_BYTES,
                         "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks
                         else "fallback"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e, "unit": "forwards/s", "h2d_bytes_per_step": B * H * 4,
                    "d2h_bytes_per_step": B * H * 4},
            "gpu_launches": 2 * B * K,
            "clocks": clocks.summary(),
        })
    if ws > 1:
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    token_list = [int(t) for t in str(args.tokens).split(",")]
    if len(token_list) > 1 and not args.ep:
        raise SystemExit("a list of --tokens needs --ep")
    args.token_list = token_list
    args.tokens = token_list[0]
    if args.impl == "reference":
        return run_reference(args)
    if args.single_expert:
        return run_single(args)
    if args.ep:
        return run_ep(args)
    if args.attention:
        return run_layers(args)
    if args.format != "q4_0":
        return run_kquant(args)
    if args.tier >= 0:
        return run_tier(args)
    if args.tokens > 1:
        return run_batched(args)
    if dist_env()[0] > 1 and not args.replicas and not args.multi:
        return run_ep_fused(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
