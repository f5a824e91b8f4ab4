"""Benchmark: batch-1 greedy decode of the Qwen3-30B-A3B-shaped MoE model (config 2).

Headline workload (the north star's target): 48
layers, d_model 2048, 32 query / 4 KV heads of 128, QK-RMSNorm, NeoX RoPE,
128 Q4_K experts top-8 renormalised (SwiGLU 768), Q8_0 attention, Q6_K
lm_head over 151936 tokens, an f16 KV cache of 4096 positions; a 32-token
seeded prompt, then 128 greedy tokens.  Weights are seeded synthetic bytes
with the config's distributions, generated on the device (48 distinct layers,
2.3 GB read per token, far beyond the 126 MB L2: no flush needed).

One bench step = one generation of that workload: 159 decode steps (the 32
prompt tokens and 127 sampled ones, each one token through the model, as the
reference's generate loop runs them), replayed as one captured CUDA graph per
token through the C++ host loop (llmtoy-zig_b200/host/decoder.cpp), whose
layers run as one persistent kernel per token (lt_stack_run).  value = decode
steps per second of device time; e2e = the same through lth_generate with the
prompt ids copied in and the token ids copied out every generation.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1: N independent replicas (batch-1 decode does not shard; weak scaling),
and the expert-parallel prefill line (config 4) shards its experts over the N
ranks.  `--impl reference` times the CPU restatement of the reference path
(oracle/, C, all host threads, built for the host CPU) on the same config-2
workload.  Extra keys: the config-1 MoE layer stack (T=1, 16 and 512), the
config-0 and config-3 decodes, and config 4.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

D_MODEL, N_EXPERTS, TOP_K, D_EXPERT = 2048, 128, 8, 768
Q4K_ROW = lambda cols: (cols // 256) * 144  # noqa: E731
EXPERT_BYTES = 2 * D_EXPERT * Q4K_ROW(D_MODEL) + D_MODEL * Q4K_ROW(D_EXPERT)  # 2,654,208
ROUTER_BYTES = N_EXPERTS * D_MODEL * 4
METRIC = "MoE decode tok/s (config 2: Qwen3-30B-A3B-shaped MoE, batch-1 greedy decode)"


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def measured_tflops() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except (KeyError, ValueError):
            pass
    return 1590.0, "fallback"


def ncu_traffic() -> dict | None:
    p = REPO / "profiles" / "ncu_summary.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return None
    return None


# ── clocks ───────────────────────────────────────────────────────────────────

class ClockSampler:
    """nvidia-smi every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        try:
            lines = Path(self.path).read_text().splitlines()
        except OSError:
            lines = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if self.path:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


# ── synthetic weights on the device ──────────────────────────────────────────

def q4k_bytes_device(torch, gen, rows: int, cols: int):
    nb = rows * (cols // 256)
    b = torch.randint(0, 256, (nb, 144), dtype=torch.uint8, device="cuda", generator=gen)
    d = (torch.rand(nb, device="cuda", generator=gen) * 3e-3 + 1e-3).half()
    dmin = (torch.rand(nb, device="cuda", generator=gen) * 2e-3).half()
    b[:, 0:2] = d.view(torch.uint8).view(nb, 2)
    b[:, 2:4] = dmin.view(torch.uint8).view(nb, 2)
    return b.view(-1)


def q8_0_bytes_device(torch, gen, rows: int, cols: int):
    """Q8_0 blocks: f16 d = 0.02/127 * U(0.5, 1.5), int8 quants uniform in [-127, 127]."""
    nb = rows * (cols // 32)
    b = torch.empty((nb, 34), dtype=torch.uint8, device="cuda")
    b[:, 2:] = torch.randint(-127, 128, (nb, 32), dtype=torch.int8, device="cuda", generator=gen).view(torch.uint8)
    d = ((torch.rand(nb, device="cuda", generator=gen) + 0.5) * (0.02 / 127)).half()
    b[:, 0:2] = d.view(torch.uint8).view(nb, 2)
    return b.view(-1)


def q6k_bytes_device(torch, gen, rows: int, cols: int):
    """Q6_K superblocks: uniform ql/qh/scale bytes, f16 d ~ U(1e-3, 4e-3) at the end."""
    nb = rows * (cols // 256)
    b = torch.randint(0, 256, (nb, 210), dtype=torch.uint8, device="cuda", generator=gen)
    d = (torch.rand(nb, device="cuda", generator=gen) * 3e-3 + 1e-3).half()
    b[:, 208:210] = d.view(torch.uint8).view(nb, 2)
    return b.view(-1)


class DeviceLayer:
    def __init__(self, pkg, ctx, torch, gen):
        router = torch.randn(N_EXPERTS, D_MODEL, device="cuda", generator=gen) * 0.02
        self.router = ctx.upload_device(router.view(torch.uint8).view(-1), pkg.F32, N_EXPERTS, D_MODEL)
        g = q4k_bytes_device(torch, gen, N_EXPERTS * D_EXPERT, D_MODEL)
        self.gate = ctx.upload_device(g, pkg.Q4_K, D_EXPERT, D_MODEL, N_EXPERTS)
        del g
        u = q4k_bytes_device(torch, gen, N_EXPERTS * D_EXPERT, D_MODEL)
        self.up = ctx.upload_device(u, pkg.Q4_K, D_EXPERT, D_MODEL, N_EXPERTS)
        del u
        dn = q4k_bytes_device(torch, gen, N_EXPERTS * D_MODEL, D_EXPERT)
        self.down = ctx.upload_device(dn, pkg.Q4_K, D_MODEL, D_EXPERT, N_EXPERTS)
        del dn
        self.norm = torch.ones(D_MODEL, device="cuda")



# ── CPU restatement (oracle) on the same workloads ───────────────────────────

NATIVE_FLAGS = "gcc -O3 -march=native -ffp-contract=off -fno-fast-math"


def oracle_module():
    """The CPU oracle's binding, built for this host's CPU (-march=native,
    as `zig build -Doptimize=ReleaseFast` targets the native CPU) when that
    build succeeds here, else the portable build; returns (module, flags).
    Both builds give the same bits: -ffp-contract=off and no fast-math keep
    every rounding of the restated Zig code."""
    sys.path.insert(0, str(REPO / "tests"))
    oracle = importlib.import_module("oracle_lib")
    flags = "gcc -O3 -march=x86-64-v2 -ffp-contract=off -fno-fast-math (portable build)"
    if oracle._lib is None:
        r = subprocess.run(["make", "-s", "-C", str(REPO / "oracle"), "native"], capture_output=True, text=True)
        native = REPO / "oracle" / "liboracle_native.so"
        if r.returncode == 0 and native.exists():
            oracle.use_library(native)
            flags = NATIVE_FLAGS
    elif str(oracle.LIB).endswith("liboracle_native.so"):
        flags = NATIVE_FLAGS
    oracle.lib()
    return oracle, flags


class CpuModel:
    """The reference CPU path (C restatement in oracle/, all host threads) on
    the config-2 model: forwardOneModel per token, 4 distinct host layer
    weight sets cycled through the 48 layers (each ~360 MB, far beyond the CPU
    caches), full vocabulary, f16-rounded KV values (the config's cache)."""

    def __init__(self, name: str = "config2"):
        self.oracle, self.flags = oracle_module()
        synth = importlib.import_module("llmtoy-zig_b200.synth")
        rng = np.random.Generator(np.random.PCG64(synth.config_seed(2 if name == "config2" else 0)))
        L = MODEL_CFG[name][0]
        m = synth.config2_model(rng, n_layers=4) if name == "config2" else synth.config0_model(rng, n_layers=4)
        self.m = synth.cycle_layers(m, L)
        self.threads = os.cpu_count() or 1
        self.pool = self.oracle.Pool(self.threads)
        self.dec = self.oracle.OracleDecoder(self.m, 4096, self.pool, kv_f16=name == "config2")
        self.prompt = np.random.Generator(np.random.PCG64(0x11A70000 + (2 if name == "config2" else 0))) \
            .integers(0, self.m.vocab, 32).tolist()
        self.pos = 0

    def tokens(self, n: int) -> None:
        """n decode steps of the workload, positions cycling over its 159."""
        for _ in range(n):
            tok = self.prompt[self.pos] if self.pos < len(self.prompt) else (7 * self.pos) % self.m.vocab
            self.dec.step(tok, self.pos)
            self.pos = (self.pos + 1) % 159

    def close(self) -> None:
        self.pool.close()


REF_TOKENS_PER_STEP = 8


def run_reference(args) -> None:
    rank, world, _ = env_rank()
    if rank != 0:
        return
    # per step: a bounded sample of the config-2 workload, 8 decode steps
    s = CpuModel()
    s.tokens(REF_TOKENS_PER_STEP * args.warmup)
    t0 = time.perf_counter()
    s.tokens(REF_TOKENS_PER_STEP * args.steps)
    dt = time.perf_counter() - t0
    s.close()
    n = REF_TOKENS_PER_STEP * args.steps
    rate = n / dt
    line = {
        "metric": METRIC, "value": rate, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (Q8_0/Q4_K/Q6_K weights dequantised per row)",
        "data": "synthetic (seeded, config-2 distributions)", "impl": "reference", "config": config_block(args, world),
        "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": s.threads, "kind": "port", "build": s.flags,
                         "sample": f"{n} decode steps of the 48-layer config-2 model (positions cycling over the "
                                   f"workload's 159, {REF_TOKENS_PER_STEP} per step), 4 distinct layer weight sets "
                                   f"cycled; C restatement of forwardOneModel (zig absent)"},
        "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_block(args, world: int) -> dict:
    return {"workload": "config 2: Qwen3-30B-A3B-shaped MoE model, batch-1 greedy decode -- 48 layers, d_model 2048, "
                        "32/4 heads of 128, QK-RMSNorm, NeoX RoPE, 128 Q4_K experts top-8 renormalised (SwiGLU 768), "
                        "Q8_0 attention, Q6_K lm_head (vocab 151936), f16 KV of 4096 positions; 32-token prompt + "
                        "128 greedy tokens = 159 decode steps per bench step",
            "global_batch": world, "seq_len": 160, "parallelism": f"replicas x{world}" if world > 1 else "single",
            "l2": "inputs larger than L2: 48 distinct layers, ~2.3 GB of weights read per decode step"}


# ── our path ─────────────────────────────────────────────────────────────────

def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5, help="generations of the config-2 workload (159 decode steps each)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU baseline work per line (rank 0, N=1)")
    ap.add_argument("--prefill-tokens", default="16,512",
                    help="comma list of T for the multi-token MoE layer measurement (config 1's T=16 and 512; 0: skip)")
    ap.add_argument("--prefill-layers", type=int, default=8)
    ap.add_argument("--ep-tokens", type=int, default=8 * 2048,
                    help="config 4: prompt tokens over all ranks, experts sharded 128/N (0: skip)")
    ap.add_argument("--ep-layers", type=int, default=2)
    ap.add_argument("--model-tokens", type=int, default=128, help="greedy tokens after the prompt (configs 2 and 0)")
    ap.add_argument("--models", default="config0,config3", help="extra whole-model decode lines ('none': skip)")
    ap.add_argument("--moe-stack", type=int, default=1, help="the config-1 MoE layer stack line (0: skip)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    pkg = importlib.import_module("llmtoy-zig_b200")
    ctx = pkg.Context(local)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream)
    ctx.reserve(1, TOP_K, D_MODEL, D_EXPERT)

    gen = torch.Generator(device="cuda")
    gen.manual_seed(0x11A70001 + 1000 * rank)
    layers = [DeviceLayer(pkg, ctx, torch, gen) for _ in range(args.layers)]
    torch.cuda.synchronize()

    # ---- headline: config-2 whole-model greedy decode ----
    head = measure_model_decode(args, pkg, ctx, torch, stream, layers, rank, world, dist, "config2",
                                runs=args.steps, warm=args.warmup, headline=True)

    moe_stack = measure_moe_stack(args, pkg, ctx, torch, stream, layers, rank, world, dist) if args.moe_stack else None

    prefill = None
    t_list = [int(t) for t in str(args.prefill_tokens).split(",") if int(t) > 0]
    if t_list:
        prefill = {f"T={T}": measure_prefill(args, pkg, ctx, torch, stream, gen, layers, rank, world, dist, T)
                   for T in t_list}

    model_decode = {}
    for name in [m for m in args.models.split(",") if m and m != "none"]:
        if name == "config3":
            model_decode[name] = measure_gemma_decode(args, pkg, ctx, torch, stream, rank, world, dist)
        else:
            model_decode[name] = measure_model_decode(args, pkg, ctx, torch, stream, layers, rank, world, dist, name)

    ep_prefill = None
    if args.ep_tokens > 0:
        ep_prefill = measure_ep_prefill(args, pkg, torch, stream, rank, world, local, dist)

    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4_k/q8_0/q6_k weights x int16+int8 activations (dp2a/dp4a), f32 accumulate",
            "data": "synthetic (seeded, config-2 distributions, generated on device)",
            "config": config_block(args, world),
            "ms_per_token": head["ms_per_token"], "decode_steps_per_step": head["steps_per_run"],
            "roofline": head["roofline"], "step_roofline": head["step_roofline"],
            "cpu_baseline": head.get("cpu_baseline"), "e2e": head["e2e"],
            "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
            "stack_kernel": head["uses_stack"], "deterministic_stream": head["deterministic_stream"],
            "kernels_per_token": head["kernels_per_token"],
            "moe_layer_stack": moe_stack, "prefill": prefill, "model_decode": model_decode,
            "ep_prefill": ep_prefill,
        }
        print(json.dumps(line), flush=True)

    for L in layers:
        for t in (L.router, L.gate, L.up, L.down):
            t.free()
    ctx.close()
    if dist is not None:
        dist.destroy_process_group()


def _barrier(torch, dist):
    if dist is not None:
        t = torch.zeros(1, device="cuda")
        dist.all_reduce(t)
    torch.cuda.synchronize()


def _max_over_ranks(torch, dist, v: float) -> float:
    if dist is None:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measure_moe_stack(args, pkg, ctx, torch, stream, layers, rank, world, dist) -> dict:
    """Config 1 at T=1: one token through the 48 chained MoE layers
    x <- x + moe(rmsnorm(x)) (one lt_moe_block per layer, a single persistent
    kernel each), replayed as one CUDA graph; 20 timed replays after the
    warm-up.  value = tokens per second through the 48-layer stack."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0x11A70101 + 1000 * rank)
    x0 = torch.randn(1, D_MODEL, device="cuda", generator=gen)
    xa = torch.empty(1, D_MODEL, device="cuda")

    def step():
        for L in layers:  # in place: xa <- xa + moe(rmsnorm(xa))
            ctx.moe_block(L.router, L.gate, L.up, L.down, pkg.ACT_SILU, True, None, L.norm, 1e-6, xa, 1, TOP_K, xa)

    with torch.cuda.stream(stream):
        xa.copy_(x0)
    step()
    ctx.sync()
    ctx.capture_begin()
    step()
    graph = ctx.capture_end()
    reps = 20
    for _ in range(args.warmup):
        graph.launch()
    _barrier(torch, dist)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(reps):
        graph.launch()
    ev1.record(stream)
    stream.synchronize()
    ms = _max_over_ranks(torch, dist, ev0.elapsed_time(ev1)) / reps
    graph.free()
    n = len(layers)
    kbytes = TOP_K * EXPERT_BYTES + ROUTER_BYTES + 3 * D_MODEL * 4
    peak, kind = measured_peaks()
    achieved = kbytes / (ms / n / 1e3) / 1e9
    out = {"metric": f"MoE decode tok/s (config-1 MoE layer, T=1, {n}-layer stack)", "value": world / (ms / 1e3),
           "unit": "tok/s", "ms_per_token": ms, "layers": n,
           "roofline": {"kernel": "moe_decode", "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                        "frac": achieved / peak, "peak_kind": kind, "algorithmic_bytes_per_launch": kbytes,
                        "us_per_launch": 1e3 * ms / n,
                        "note": "us_per_launch = graph replay time / launches (in-step, PDL hand-overs included)"}}
    if rank == 0 and world == 1 and args.cpu_budget > 0:
        out["cpu_baseline"] = cpu_stack_rate(n, min(args.cpu_budget, 10.0))
    return out


def cpu_stack_rate(n_layers: int, budget_s: float) -> dict:
    """The CPU restatement through n_layers config-1 MoE layers, 4 distinct
    host weight sets cycled, all host threads."""
    oracle, flags = oracle_module()
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(synth.config_seed(1)))
    sets = [synth.MoeLayer(rng, D_MODEL, N_EXPERTS, D_EXPERT) for _ in range(4)]
    norm = np.ones(D_MODEL, np.float32)
    threads = os.cpu_count() or 1
    pool = oracle.Pool(threads)
    x = rng.normal(0, 1, size=(1, D_MODEL)).astype(np.float32)
    L = oracle.lib()

    def token(xx):
        for li in range(n_layers):
            xn = np.empty_like(xx)
            L.orc_rmsnorm(xn.ctypes.data, xx.ctypes.data, norm.ctypes.data, D_MODEL, 1e-6)
            y, _, _ = oracle.moe_layer(sets[li % 4], xn, TOP_K, True, 0, None, pool)
            xx = (xx + y).astype(np.float32)
        return xx

    x = token(x)
    t0 = time.perf_counter()
    n = 0
    while n < 1 or time.perf_counter() - t0 < budget_s:
        x = token(x)
        n += 1
    dt = time.perf_counter() - t0
    pool.close()
    return {"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "port", "build": flags,
            "sample": f"{n} tokens x {n_layers} layers in {dt:.1f}s, 4 distinct host weight sets cycled"}


def measure_prefill(args, pkg, ctx, torch, stream, gen, layers, rank, world, dist, T: int) -> dict:
    """T tokens through `prefill_layers` MoE blocks in place (router, dispatch,
    gate/up and down -- the tensor-core GEMM from 64 tokens, the CUDA-core
    grouped kernels below -- combine, residual); value = tokens per second
    through one MoE layer, all ranks (replicas)."""
    nl = min(args.prefill_layers, len(layers))
    xp = torch.randn(T, D_MODEL, device="cuda", generator=gen)
    xp0 = xp.clone()

    def pstep():
        for L in layers[:nl]:
            ctx.moe_block(L.router, L.gate, L.up, L.down, pkg.ACT_SILU, True, None, L.norm, 1e-6, xp, T, TOP_K, xp)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            xp.copy_(xp0)
            pstep()
    ctx.sync()
    reps = max(1, args.steps // 10)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(reps):
        pstep()
    ev1.record(stream)
    stream.synchronize()
    ms = ev0.elapsed_time(ev1)
    if dist is not None:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_layer = ms / (reps * nl)
    ctx.sync()
    ctx.profile(True)
    ctx.profile_reset()
    pstep()
    ctx.sync()
    prof = ctx.profile_read()
    ctx.profile(False)
    ctx.profile_reset()
    k_us = {k: 1e3 * v["total_ms"] / v["count"] for k, v in prof.items()}
    gemm_us = k_us.get("moe_gemm_gate_up", 0.0) + k_us.get("moe_gemm_down", 0.0)
    flops = 2.0 * T * TOP_K * 3 * D_EXPERT * D_MODEL  # gate + up + down, algorithmic
    if gemm_us:  # tensor-core path: bound by the tensor pipe
        peak, kind = measured_tflops()
        achieved = flops / (gemm_us * 1e-6) / 1e12
        roofline = {"kernel": "moe_gemm_gate_up + moe_gemm_down", "bound": "tensor", "achieved": achieved,
                    "peak": peak, "unit": "TFLOP/s", "peak_kind": kind, "frac": achieved / peak,
                    "algorithmic_flops": flops, "traffic": None,
                    "note": "f16 tcgen05 MMAs; the activation's lo plane doubles the issued MMA work"}
    else:  # CUDA-core grouped kernels: bound by HBM (the distinct experts' bytes once each)
        L0 = layers[0]
        xn, ids, wts = torch.empty_like(xp0), torch.empty(T * TOP_K, dtype=torch.int32, device="cuda"), \
            torch.empty(T * TOP_K, device="cuda")
        ctx.rmsnorm(xp0, L0.norm, 1e-6, D_MODEL, T, xn)
        ctx.moe_route(L0.router, xn, T, TOP_K, True, None, ids, wts)
        ctx.sync()
        U = int(torch.unique(ids).numel())
        nbytes = U * EXPERT_BYTES + ROUTER_BYTES + 2 * T * D_MODEL * 4
        peak, kind = measured_peaks()
        achieved = nbytes / (ms_layer / 1e3) / 1e9
        roofline = {"kernel": "whole MoE layer (router, moe_gate_up, moe_down)", "bound": "hbm",
                    "achieved": achieved, "peak": peak, "unit": "GB/s", "peak_kind": kind, "frac": achieved / peak,
                    "algorithmic_bytes_per_layer": nbytes, "experts_selected": U, "traffic": None,
                    "note": "U distinct experts of the first layer's routing, each read once"}
    out = {
        "metric": f"MoE layer tok/s (config 1, T={T})", "value": world * T / (ms_layer / 1e3),
        "unit": "tok/s", "ms_per_layer": ms_layer, "layers_timed": nl, "reps": reps,
        "stack_equivalent_tok_s": world * T / (ms_layer / 1e3) / args.layers,
        "kernels_us": {k: round(v, 1) for k, v in k_us.items()},
        "roofline": roofline,
    }
    if rank == 0 and world == 1 and args.cpu_budget > 0:
        out["cpu_baseline"] = cpu_prefill_rate(min(args.cpu_budget, 10.0), T)
    return out


MODEL_CFG = {
    # name: (layers, d, heads, kv heads, head dim, vocab, d_ffn, lm type, qk norm, neox, MoE)
    "config2": (48, 2048, 32, 4, 128, 151936, 0, "q6_k", True, True, True),
    "config0": (24, 896, 14, 2, 64, 151936, 4864, "q8_0", False, False, False),
}


def model_layer_bytes(name: str, ctx_len: float) -> float:
    """Algorithmic HBM bytes of the decoder layers for one token: attention
    projections, router + 8 experts (or the dense FFN), the two norms and
    the KV cache read at ctx_len positions (f16 elements for config 2, whose
    cache the config specifies as f16)."""
    L, d, nh, nkv, hd, V, F, lm, _, _, moe = MODEL_CFG[name]
    q8 = lambda r, c: r * (c // 32) * 34  # noqa: E731
    attn = q8(nh * hd + 2 * nkv * hd, d) + q8(d, nh * hd)
    ffn = TOP_K * EXPERT_BYTES + ROUTER_BYTES if moe else 3 * q8(F, d)
    kv = 2 * ctx_len * nkv * hd * (2 if name == "config2" else 4)
    return L * (attn + ffn + kv + 2 * d * 4)


def model_bytes_per_token(name: str, ctx_len: float) -> float:
    """Algorithmic HBM bytes of one decode step: the layers, the lm_head and
    the embedding row."""
    L, d, nh, nkv, hd, V, F, lm, _, _, moe = MODEL_CFG[name]
    q8 = lambda r, c: r * (c // 32) * 34  # noqa: E731
    lm_bytes = V * (d // 256) * 210 if lm == "q6_k" else q8(V, d)
    return model_layer_bytes(name, ctx_len) + lm_bytes + q8(1, d) + d * 4


def measure_model_decode(args, pkg, ctx, torch, stream, moe_layers, rank, world, dist, name: str, runs: int = 1,
                         warm: int = 1, headline: bool = False) -> dict:
    """Greedy decode of a whole model through the C++ host loop
    (llmtoy-zig_b200/host/decoder.cpp): a 32-token prompt (config 0: 5
    tokens, its workload), then args.model_tokens tokens, one captured graph
    per token.  config2 reuses the stack's 48 MoE layers (router + experts)
    and adds Q8_0 attention with QK norm, NeoX RoPE, a Q8_0 embedding and the
    Q6_K lm_head; config0 is the dense Q8_0 Qwen2-0.5B shape.  `runs`
    generations are timed, each bracketed by a barrier and CUDA events on the
    context stream (the position reset between them is a host copy outside
    the timing); replicas on N > 1."""
    decoder = importlib.import_module("llmtoy-zig_b200.decoder")
    L, d, nh, nkv, hd, V, F, lm, qk, neox, moe = MODEL_CFG[name]
    n_prompt, n_gen = (32, args.model_tokens) if moe else (5, min(20, args.model_tokens))
    cap = 4096
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0x11A70002 + 1000 * rank if moe else 0x11A70000 + 1000 * rank)
    keep, tensors = [], []

    def up(b, t, r, c, e=0):
        tt = ctx.upload_device(b, t, r, c, e)
        tensors.append(tt)
        return tt

    ones = lambda n: keep.append(torch.ones(n, device="cuda")) or keep[-1]  # noqa: E731
    specs = []
    for li in range(L):
        ls = decoder.LayerSpec(attn_norm=ones(d), ffn_norm=ones(d),
                               wo=up(q8_0_bytes_device(torch, gen, d, nh * hd), pkg.Q8_0, d, nh * hd),
                               wqkv=up(q8_0_bytes_device(torch, gen, nh * hd + 2 * nkv * hd, d), pkg.Q8_0,
                                       nh * hd + 2 * nkv * hd, d),
                               q_norm=ones(hd) if qk else None, k_norm=ones(hd) if qk else None)
        if moe:
            ML = moe_layers[li % len(moe_layers)]
            ls.router, ls.exp_gate, ls.exp_up, ls.exp_down = ML.router, ML.gate, ML.up, ML.down
        else:
            ls.ffn_gate = up(q8_0_bytes_device(torch, gen, F, d), pkg.Q8_0, F, d)
            ls.ffn_up = up(q8_0_bytes_device(torch, gen, F, d), pkg.Q8_0, F, d)
            ls.ffn_down = up(q8_0_bytes_device(torch, gen, d, F), pkg.Q8_0, d, F)
        specs.append(ls)
    emb = up(q8_0_bytes_device(torch, gen, V, d), pkg.Q8_0, V, d)
    lmh = up(q6k_bytes_device(torch, gen, V, d), pkg.Q6_K, V, d) if lm == "q6_k" else \
        up(q8_0_bytes_device(torch, gen, V, d), pkg.Q8_0, V, d)
    spec = decoder.ModelSpec(d_model=d, n_heads=nh, n_kv_heads=nkv, head_dim=hd, vocab=V, token_emb=emb,
                             lm_head=lmh, out_norm=ones(d), layers=specs, n_used=TOP_K if moe else 0,
                             norm_topk=moe, rope_neox=neox, eps=1e-6, rope_theta=1e6, kv_cap=cap,
                             kv_f16=name == "config2")
    torch.cuda.synchronize()
    prompt = np.random.Generator(np.random.PCG64(0x11A70000 + (2 if moe else 0))).integers(0, V, n_prompt).tolist()
    steps = n_prompt + n_gen - 1
    dec = decoder.Decoder(ctx, spec)
    first = dec.generate(prompt, n_gen)  # warm-up: eager step, capture, replays
    for _ in range(max(0, warm - 1)):
        dec.generate(prompt, n_gen)

    # device time of `runs` whole generations (graph replays on the context stream)
    total_ms, deterministic = 0.0, True
    with ClockSampler(torch.cuda.current_device()) as clk:
        for _ in range(runs):
            dec.start(prompt)
            _barrier(torch, dist)
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            dec.replay(steps)
            ev1.record(stream)
            stream.synchronize()
            total_ms += _max_over_ranks(torch, dist, ev0.elapsed_time(ev1))
            deterministic = deterministic and dec.tokens(n_prompt + n_gen)[n_prompt:] == first
    clocks = clk.summary()
    ms_step = total_ms / (runs * steps)

    # end to end through the public entry point: host prompt in, host tokens out, every generation
    e2e_runs = max(1, runs if headline else 1)
    _barrier(torch, dist)
    t0 = time.perf_counter()
    for _ in range(e2e_runs):
        dec.generate(prompt, n_gen)
    e2e_s = _max_over_ranks(torch, dist, time.perf_counter() - t0)

    # the dominant kernel alone: the layer stack at the workload's mean context,
    # replayed as a graph (the position and caches stay put)
    mean_ctx = n_prompt + (n_gen - 1) / 2.0
    dec.start(prompt)
    dec.replay(int(mean_ctx))
    ctx.sync()
    ctx.capture_begin()
    dec.run_layers()
    lg = ctx.capture_end()
    for _ in range(3):
        lg.launch()
    _barrier(torch, dist)
    reps, batches = 10, 5  # the median of five batches of ten replays (single batches varied by a few percent)
    batch_ms = []
    for _ in range(batches):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(reps):
            lg.launch()
        ev1.record(stream)
        stream.synchronize()
        batch_ms.append(ev0.elapsed_time(ev1) / reps)
    layers_ms = _max_over_ranks(torch, dist, float(np.median(batch_ms)))
    lg.free()
    uses_stack = dec.uses_stack

    # per-kernel times and launches of one eager prompt step and one full step
    dec.start(prompt)
    ctx.profile(True)
    ctx.profile_reset()
    dec.step()
    ctx.sync()
    prof = ctx.profile_read()
    ctx.profile(False)
    ctx.profile_reset()
    launches_full = int(sum(v["count"] for v in prof.values()))
    # a prompt step skips the final norm, the lm_head matvec and the soft-cap
    launches_prompt = launches_full - int(sum(v["count"] for k, v in prof.items()
                                              if k.startswith(("rmsnorm", "qmv", "quantize", "softcap"))))
    dec.close()
    for tt in tensors:
        tt.free()
    peak, kind = measured_peaks()
    bpt = model_bytes_per_token(name, mean_ctx)
    achieved = bpt / (ms_step / 1e3) / 1e9
    lbytes = model_layer_bytes(name, mean_ctx)
    k_achieved = lbytes / (layers_ms / 1e3) / 1e9
    kname = "stack" if uses_stack else f"{L} x (attn_block + moe_decode)"
    step_roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                 "peak_kind": kind, "algorithmic_bytes_per_token": bpt, "ms_per_token": ms_step,
                 "note": "whole decode step (every kernel of one token, lm_head included) in graph replays; "
                         "weights + KV at the mean context"}
    roof = {"kernel": kname, "bound": "hbm", "achieved": k_achieved, "peak": peak, "unit": "GB/s",
            "frac": k_achieved / peak, "peak_kind": kind, "algorithmic_bytes_per_launch": lbytes,
            "avg_launch_ms": layers_ms, "traffic": (ncu_traffic() or {}).get(name, {}).get("dram_bytes_per_launch"),
            "note": f"the {L} decoder layers of one token at position {int(mean_ctx)} (the workload's mean "
                    f"context) as one graph: the median of {batches} batches of {reps} replays, CUDA events on the "
                    f"launching stream"}
    n_runs_launches = runs * ((n_prompt - 1) * launches_prompt + n_gen * launches_full)
    out = {
        "metric": f"greedy decode tok/s ({name}: {'Qwen3-30B-A3B' if moe else 'Qwen2-0.5B'} shape, {L} layers)",
        "value": world / (ms_step / 1e3), "unit": "tok/s", "ms_per_token": ms_step, "ms_per_step": total_ms / runs,
        "steps_per_run": steps, "runs": runs,
        "prompt_tokens": n_prompt, "generated_tokens": n_gen, "scaling": "weak",
        "kv_cache": {"dtype": "f16" if name == "config2" else "f32", "capacity": cap},
        "deterministic_stream": deterministic, "uses_stack": uses_stack,
        "roofline": roof, "step_roofline": step_roof,
        "e2e": {"value": world * e2e_runs * steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4 * n_prompt,
                "d2h_bytes_per_step": 4 * (n_prompt + n_gen), "runs": e2e_runs,
                "path": "lth_generate: host prompt ids in, host token ids out; decode steps per second"},
        "kernels_per_token": {k: {"count": v["count"], "us": round(1e3 * v["total_ms"], 1)} for k, v in prof.items()},
        "gpu_launches_per_token": launches_full, "gpu_launches": n_runs_launches,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and args.cpu_budget > 0:
        out["cpu_baseline"] = cpu_model_rate(name, min(args.cpu_budget, 10.0))
    return out


GEMMA = dict(n_layers=30, d=2816, n_heads=16, n_kv=8, hd=256, d_ffn=2112, E=128, k=8, F=704, vocab=262144,
             window=1024, period=6)


def gemma_types(seed: int) -> list[dict]:
    """The seeded per-tensor type mix of config 3 (60% Q4_K, 25% Q6_K, 15%
    Q8_0; Q8_0 where the columns are not a multiple of 256), per layer."""
    rng = np.random.Generator(np.random.PCG64(seed))
    g = GEMMA

    def pick(cols):
        if cols % 256:
            return 8
        u = rng.uniform()
        return 12 if u < 0.60 else 14 if u < 0.85 else 8

    out = []
    for _ in range(g["n_layers"]):
        t = {"wq": pick(g["d"]), "wk": pick(g["d"]), "wv": pick(g["d"]), "wo": pick(g["n_heads"] * g["hd"]),
             "gate": pick(g["d"]), "down": pick(g["d_ffn"]), "gate_up_exps": pick(g["d"]), "down_exps": pick(g["F"])}
        t["up"] = t["gate"]
        out.append(t)
    return out


def gemma_bytes_per_token(types: list[dict], ctx_len: float) -> float:
    """Algorithmic bytes of one config-3 step: every weight read (attention,
    dense FFN, router, the 8 selected experts, norms), the lm_head, the
    embedding row and the KV read (SWA layers see at most the window)."""
    g = GEMMA
    d, nq, nkv = g["d"], g["n_heads"] * g["hd"], g["n_kv"] * g["hd"]
    rb = lambda t, c: (c // 32) * 34 if t == 8 else (c // 256) * (144 if t == 12 else 210)  # noqa: E731
    total = 0.0
    for i, t in enumerate(types):
        swa = (i + 1) % g["period"] != 0
        total += nq * rb(t["wq"], d) + nkv * rb(t["wk"], d) + nkv * rb(t["wv"], d) + d * rb(t["wo"], nq)
        total += 2 * g["d_ffn"] * rb(t["gate"], d) + d * rb(t["down"], g["d_ffn"])
        total += g["E"] * d * 4 + g["k"] * (2 * g["F"] * rb(t["gate_up_exps"], d) + d * rb(t["down_exps"], g["F"]))
        win = min(ctx_len, g["window"]) if swa else ctx_len
        total += 2 * win * nkv * 4 + 10 * d * 4
    return total + g["vocab"] * (d // 256) * 210 + rb(12, d)


def measure_gemma_decode(args, pkg, ctx, torch, stream, rank, world, dist) -> dict:
    """Config 3: greedy decode of the Gemma-4-26B-A4B-like model through the
    C++ host loop (Gemma 4 family): a 64-token prompt, then 80 tokens (the
    config's workload; args.model_tokens caps it), weights generated on the
    device with the seeded per-tensor type mix, Q6_K lm_head."""
    decoder = importlib.import_module("llmtoy-zig_b200.decoder")
    g = GEMMA
    d, nq, nkv, E, F = g["d"], g["n_heads"] * g["hd"], g["n_kv"] * g["hd"], g["E"], g["F"]
    n_prompt, n_gen = 64, min(80, args.model_tokens)
    types = gemma_types(0x11A70003)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0x11A70003 + 1000 * rank)
    keep, tensors = [], []
    dev_gen = {8: q8_0_bytes_device, 12: q4k_bytes_device, 14: q6k_bytes_device}

    def up(t, r, c, e=0):
        tt = ctx.upload_device(dev_gen[t](torch, gen, r * max(1, e), c), t, r, c, e)
        tensors.append(tt)
        return tt

    def vec(n, v=1.0):
        keep.append(torch.full((n,), v, device="cuda"))
        return keep[-1]

    specs = []
    for i, t in enumerate(types):
        rw = torch.randn(E, d, device="cuda", generator=gen) * 0.02
        router = ctx.upload_device(rw.view(torch.uint8).view(-1), pkg.F32, E, d)
        tensors.append(router)
        del rw
        specs.append(decoder.LayerSpec(
            attn_norm=vec(d), ffn_norm=vec(d), wo=up(t["wo"], d, nq), wq=up(t["wq"], nq, d), wk=up(t["wk"], nkv, d),
            wv=up(t["wv"], nkv, d), q_norm=vec(g["hd"]), k_norm=vec(g["hd"]), ffn_gate=up(t["gate"], g["d_ffn"], d),
            ffn_up=up(t["up"], g["d_ffn"], d), ffn_down=up(t["down"], d, g["d_ffn"]), router=router,
            exp_gate=up(t["gate_up_exps"], 2 * F, d, E), exp_down=up(t["down_exps"], d, F, E),
            post_attention_norm=vec(d), pre_ffw_norm_2=vec(d), post_ffw_norm_1=vec(d), post_ffw_norm_2=vec(d),
            post_ffw_norm=vec(d), router_scale=vec(d), down_exps_scale=vec(E), layer_output_scale=1.0,
            is_swa=(i + 1) % g["period"] != 0, n_kv_heads=g["n_kv"], head_dim=g["hd"]))
    emb = up(12, g["vocab"], d)
    lmh = up(14, g["vocab"], d)
    spec = decoder.ModelSpec(d_model=d, n_heads=g["n_heads"], n_kv_heads=g["n_kv"], head_dim=g["hd"],
                             vocab=g["vocab"], token_emb=emb, lm_head=lmh, out_norm=vec(d), layers=specs, n_used=g["k"],
                             rope_neox=True, act=1, eps=1e-6, rope_theta=1e6, kv_cap=4096, family=decoder.GEMMA4,
                             rope_theta_swa=1e4, logit_softcap=30.0, sliding_window=g["window"])
    torch.cuda.synchronize()
    prompt = np.random.Generator(np.random.PCG64(0x11A70003)).integers(0, g["vocab"], n_prompt).tolist()
    steps = n_prompt + n_gen - 1
    dec = decoder.Decoder(ctx, spec)
    first = dec.generate(prompt, n_gen)
    dec.start(prompt)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        ev0.record(stream)
        dec.replay(steps)
        ev1.record(stream)
        stream.synchronize()
    ms = ev0.elapsed_time(ev1)
    deterministic = dec.tokens(n_prompt + n_gen)[n_prompt:] == first
    if dist is not None:
        tt = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ms_step = ms / steps
    t0 = time.perf_counter()
    dec.generate(prompt, n_gen)
    e2e_s = time.perf_counter() - t0
    dec.start(prompt)
    ctx.profile(True)
    ctx.profile_reset()
    dec.step()
    ctx.sync()
    prof = ctx.profile_read()
    ctx.profile(False)
    ctx.profile_reset()
    dec.close()
    for tt in tensors:
        tt.free()
    peak, kind = measured_peaks()
    bpt = gemma_bytes_per_token(types, n_prompt + (n_gen - 1) / 2.0)
    achieved = bpt / (ms_step / 1e3) / 1e9
    mix = {}
    for t in types:
        for v in t.values():
            mix[{8: "q8_0", 12: "q4_k", 14: "q6_k"}[v]] = mix.get({8: "q8_0", 12: "q4_k", 14: "q6_k"}[v], 0) + 1
    out = {
        "metric": "greedy decode tok/s (config3: Gemma-4-26B-A4B-like, 30 layers, 5 SWA : 1 global)",
        "value": world / (ms_step / 1e3), "unit": "tok/s", "ms_per_token": ms_step, "steps": steps,
        "prompt_tokens": n_prompt, "generated_tokens": n_gen, "scaling": "weak", "deterministic_stream": deterministic,
        "tensor_type_mix": mix,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": kind, "algorithmic_bytes_per_token": bpt},
        "e2e": {"value": world * n_gen / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4 * n_prompt / n_gen,
                "d2h_bytes_per_step": 4.0 * (n_prompt + n_gen) / n_gen,
                "path": "lth_generate: host prompt ids in, host token ids out (prompt steps included)"},
        "kernels_per_token": {k: {"count": v["count"], "us": round(1e3 * v["total_ms"], 1)} for k, v in prof.items()},
        "gpu_launches_per_token": int(sum(v["count"] for v in prof.values())),
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and args.cpu_budget > 0:
        out["cpu_baseline"] = cpu_gemma_rate(min(args.cpu_budget, 10.0))
    return out


def cpu_gemma_rate(budget_s: float) -> dict:
    """orc_gemma_step (all host threads) on the config-3 shape: 3 distinct host
    layer weight sets cycled through the 30 layers, full vocabulary."""
    oracle, flags = oracle_module()
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(synth.config_seed(3)))
    m = synth.cycle_layers(synth.GemmaModel(rng, n_layers=3), GEMMA["n_layers"], swa_period=GEMMA["period"])
    threads = os.cpu_count() or 1
    pool = oracle.Pool(threads)
    dec = oracle.OracleGemma(m, 64, pool)
    dec.step(1, 0)
    t0 = time.perf_counter()
    n = 0
    while n < 2 or time.perf_counter() - t0 < budget_s:
        dec.step(1 + n, (n + 1) % 64)
        n += 1
    dt = time.perf_counter() - t0
    pool.close()
    return {"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "port", "build": flags,
            "sample": f"{n} decode steps of the 30-layer model in {dt:.1f}s (3 distinct layer weight sets cycled; "
                      f"C restatement of gemma4 forwardOne, zig absent)"}


def cpu_model_rate(name: str, budget_s: float) -> dict:
    """The CPU restatement (orc_model_step, all host threads) on the same
    model shape: 4 distinct host layer sets cycled through all layers, full
    vocabulary (CpuModel)."""
    s = CpuModel(name)
    s.tokens(1)
    t0 = time.perf_counter()
    n = 0
    while n < 2 or time.perf_counter() - t0 < budget_s:
        s.tokens(1)
        n += 1
    dt = time.perf_counter() - t0
    s.close()
    return {"value": n / dt, "unit": "tok/s", "cores": s.threads, "kind": "port", "build": s.flags,
            "sample": f"{n} decode steps of the {s.m.n_layers}-layer model in {dt:.1f}s (4 distinct layer weight sets "
                      f"cycled; C restatement of forwardOneModel, zig absent)"}


def zipf_router(torch, n_experts: int, d: int, s: float, mu: float, seed: int):
    """Router weights (replicated: the same seed on every rank) whose logits
    carry a bias b_e = ln p_e, p_e proportional to rank_e^-s (Zipf), along a
    fixed unit direction u, with expert ranks a seeded permutation; hidden
    states get mu * u added, so after the RMSNorm each token's logit of
    expert e shifts by about b_e."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    base = torch.randn(n_experts, d, device="cuda", generator=g) * 0.02
    u = torch.randn(d, device="cuda", generator=g)
    u = u / u.norm()
    order = torch.randperm(n_experts, device="cuda", generator=g)
    ranks = torch.empty(n_experts, device="cuda")
    ranks[order] = torch.arange(1, n_experts + 1, device="cuda", dtype=torch.float32)
    b = -s * torch.log(ranks)  # ln p_e up to a constant
    b = b - b.mean()
    rms = (1.0 + mu * mu / d) ** 0.5
    return (base + (b * rms / mu)[:, None] * u[None, :]).contiguous(), u


def ep_expert_bytes(torch, layer: int, e: int):
    """Expert e of EP layer `layer`: gate, up and down GGUF bytes from a seed of
    their own, so every rank can rebuild any expert (the parity check needs the
    whole layer on each rank's host)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(0x11A74100 + 1000 * layer + e)
    return (q4k_bytes_device(torch, g, D_EXPERT, D_MODEL), q4k_bytes_device(torch, g, D_EXPERT, D_MODEL),
            q4k_bytes_device(torch, g, D_MODEL, D_EXPERT))


def ep_parity(torch, dist, moe, layer, x, mu: float, world: int, n_sample: int = 8) -> dict:
    """A seeded sample of this rank's tokens through the expert-parallel layer
    against orc_moe_layer on the whole layer (rebuilt on the host from the
    per-expert seeds): worst relative L2 of the MoE part over the sample, max
    over ranks."""
    import types
    oracle, _ = oracle_module()
    T = x.shape[0]
    rank = dist.get_rank() if dist is not None else 0
    idx = np.random.Generator(np.random.PCG64(0x11A7E000 + rank)).choice(T, size=min(n_sample, T), replace=False)
    out = moe.forward(layer, x)
    torch.cuda.synchronize()
    got = out[torch.from_numpy(idx).cuda()].cpu().numpy()
    xs = x[torch.from_numpy(idx).cuda()].cpu().numpy()
    gs, us, ds = [], [], []
    for e in range(N_EXPERTS):
        g, u, dn = ep_expert_bytes(torch, 0, e)
        gs.append(g.cpu().numpy())
        us.append(u.cpu().numpy())
        ds.append(dn.cpu().numpy())
    rw, _ = zipf_router(torch, N_EXPERTS, D_MODEL, 1.1, mu, 0x11A74000)
    full = types.SimpleNamespace(router=rw.cpu().numpy(), gate=np.concatenate(gs), up=np.concatenate(us),
                                 down=np.concatenate(ds), gate_type=12, down_type=12, d_model=D_MODEL,
                                 n_experts=N_EXPERTS, d_expert=D_EXPERT)
    norm = np.ones(D_MODEL, np.float32)
    xn = np.empty_like(xs)
    for t in range(xs.shape[0]):
        oracle.lib().orc_rmsnorm(xn[t].ctypes.data, xs[t].ctypes.data, norm.ctypes.data, D_MODEL, 1e-6)
    pool = oracle.Pool(max(1, (os.cpu_count() or 1) // world))
    ref, _, _ = oracle.moe_layer(full, xn, TOP_K, True, pool=pool)
    pool.close()
    worst = max(float(np.linalg.norm((got[t] - xs[t]) - ref[t]) / np.linalg.norm(ref[t])) for t in range(xs.shape[0]))
    worst = float(_max_over_ranks(torch, dist, worst))
    return {"worst_rel_l2": worst, "tokens_per_rank": int(len(idx)), "bar": 1e-4, "ok": worst < 1e-4,
            "against": "orc_moe_layer (router + 8 experts + renormalised combine) on the whole layer, the MoE part "
                       "of out = x + moe(rmsnorm(x))"}


def measure_ep_prefill(args, pkg, torch, stream, rank, world, local, dist) -> dict:
    """Config 4: args.ep_tokens prompt tokens (8 sequences x 2048) through
    args.ep_layers MoE blocks of the config-2 shape, tokens split evenly over
    the ranks, experts sharded 128/N, Zipf(1.1)-biased routing.  N = 1 runs
    the single-device path (no exchange); N > 1 the expert-parallel layer
    (llmtoy-zig_b200/ep.py: dispatch, NCCL all-to-all-v of rows, local
    grouped GEMM, all-to-all-v back, combine).  Each layer reads the same
    input (out = x + moe(rmsnorm(x))), so every step routes alike.  value =
    total tokens through one layer per second (strong scaling: the total is
    fixed)."""
    ep = importlib.import_module("llmtoy-zig_b200.ep")
    G = args.ep_tokens
    if G % world:
        return {"skipped": f"{G} tokens do not split over {world} ranks"}
    T = G // world
    lo, hi = ep.expert_range(N_EXPERTS, rank, world)
    ne = hi - lo
    mu = 4.0
    ctx = pkg.Context(local)
    out: dict = {}
    with torch.cuda.stream(stream):
        ops = ep.DeviceOps(ctx, f"cuda:{local}")
        gen = torch.Generator(device="cuda")
        gen.manual_seed(0x11A70004 + 1000 * rank)
        layers = []
        for li in range(args.ep_layers):
            rw, u = zipf_router(torch, N_EXPERTS, D_MODEL, 1.1, mu, 0x11A74000 + li)
            router = ctx.upload_device(rw.view(torch.uint8).view(-1), pkg.F32, N_EXPERTS, D_MODEL)
            del rw
            parts = [ep_expert_bytes(torch, li, e) for e in range(lo, hi)]
            gate = ctx.upload_device(torch.cat([q[0] for q in parts]), pkg.Q4_K, D_EXPERT, D_MODEL, ne)
            up = ctx.upload_device(torch.cat([q[1] for q in parts]), pkg.Q4_K, D_EXPERT, D_MODEL, ne)
            down = ctx.upload_device(torch.cat([q[2] for q in parts]), pkg.Q4_K, D_MODEL, D_EXPERT, ne)
            del parts
            layers.append((ep.EPLayer(router=router, gate=gate, up=up, down=down, n_experts=N_EXPERTS,
                                      d_model=D_MODEL, norm_w=torch.ones(D_MODEL, device="cuda")), u))
        x = torch.randn(T, D_MODEL, device="cuda", generator=gen) + mu * layers[0][1][None, :]
        moe = ep.ExpertParallelMoE(ops, TOP_K)

        a2a_ms = []

        def timed_a2a(o, i, os_=None, is_=None):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            dist.all_to_all_single(o, i, os_, is_)
            e1.record()
            a2a_ms.append((e0, e1, (o.numel() + i.numel()) * o.element_size()))

        def pstep():
            for L, _ in layers:
                moe.forward(L, x)

        for _ in range(args.warmup):
            pstep()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        reps = max(1, args.steps // 10)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(reps):
            pstep()
        ev1.record()
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        if dist is not None:
            t = torch.tensor([ms], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        ms_layer = ms / (reps * args.ep_layers)

        # one more pass with the kernel profiler and the exchanges timed alone
        ctx.profile(True)
        ctx.profile_reset()
        if world > 1:
            moe._a2a = timed_a2a
        for L, _ in layers:
            moe.forward(L, x)
        torch.cuda.synchronize()
        prof = ctx.profile_read()
        ctx.profile(False)
        k_us = {k: 1e3 * v["total_ms"] / v["count"] for k, v in prof.items()}
        k_layer_us = sum(v["total_ms"] for v in prof.values()) * 1e3 / args.ep_layers
        recv = torch.tensor([float(moe.last_stats.get("received_pairs", T * TOP_K))], device="cuda")
        if world > 1:
            a2a_us = sum(e0.elapsed_time(e1) for e0, e1, _ in a2a_ms) * 1e3 / args.ep_layers
            a2a_bytes = sum(b for _, _, b in a2a_ms) / args.ep_layers
            allr = [torch.zeros_like(recv) for _ in range(world)]
            dist.all_gather(allr, recv)
            loads = [float(t.item()) for t in allr]
        else:
            a2a_us, a2a_bytes, loads = 0.0, 0, [float(recv.item())]
        parity = ep_parity(torch, dist, moe, layers[0][0], x, mu, world)
        # expert popularity of the biased router over this rank's tokens
        xn = torch.empty_like(x)
        ctx.rmsnorm(x, layers[0][0].norm_w, 1e-6, D_MODEL, T, xn)
        ids = torch.empty(T, TOP_K, dtype=torch.int32, device="cuda")
        wts = torch.empty(T, TOP_K, device="cuda")
        ctx.moe_route(layers[0][0].router, xn, T, TOP_K, True, None, ids, wts)
        cnt = torch.bincount(ids.view(-1).long(), minlength=N_EXPERTS).float()
        if dist is not None:
            dist.all_reduce(cnt)
        torch.cuda.synchronize()
    gemm_us = k_us.get("moe_gemm_gate_up", 0.0) + k_us.get("moe_gemm_down", 0.0)
    flops_rank = 2.0 * max(loads) * 3 * D_EXPERT * D_MODEL
    peak, kind = measured_tflops()
    mean_load = sum(loads) / len(loads)
    out = {
        "metric": f"expert-parallel prefill tok/s (config 4: {G} tokens, 128 experts / {world} GPUs, Zipf 1.1)",
        "value": G / (ms_layer / 1e3), "unit": "tok/s", "n_gpus": world, "scaling": "strong",
        "ms_per_layer": ms_layer, "layers_timed": args.ep_layers, "reps": reps,
        "tokens_per_rank": T, "experts_per_rank": ne,
        "path": "single-device lt_moe_block" if world == 1 else "ExpertParallelMoE over NCCL all_to_all_single",
        "kernels_us": {k: round(v, 1) for k, v in k_us.items()}, "kernel_us_per_layer": k_layer_us,
        "load_pairs_per_rank": loads, "load_imbalance_max_over_mean": max(loads) / mean_load,
        "expert_popularity_max_over_mean": float(cnt.max() / cnt.mean()),
        "expert_popularity_top8_share": float(cnt.sort(descending=True).values[:8].sum() / cnt.sum()),
        "parity": parity,
        "roofline": {"kernel": "moe_gemm_gate_up + moe_gemm_down (busiest rank)", "bound": "tensor",
                     "achieved": flops_rank / (gemm_us * 1e-6) / 1e12 if gemm_us else None, "peak": peak,
                     "unit": "TFLOP/s", "peak_kind": kind,
                     "frac": flops_rank / (gemm_us * 1e-6) / 1e12 / peak if gemm_us else None},
    }
    if world > 1:
        out["all_to_all"] = {"us_per_layer": a2a_us, "bytes_per_layer_per_rank": a2a_bytes,
                             "gbs": a2a_bytes / (a2a_us * 1e-6) / 1e9 if a2a_us else None,
                             "nvlink_ref_gbs": 770.0,
                             "note": "rank-0 view: bytes sent + received per rank over the time of its four "
                                     "all_to_all_single calls (counts, rows, ids, results)"}
    for L, _ in layers:
        for t_ in (L.router, L.gate, L.up, L.down):
            t_.free()
    ctx.close()
    return out


def cpu_prefill_rate(budget_s: float, T: int) -> dict:
    """The CPU restatement on a bounded sample of the same workload: batches of
    min(T, 16) tokens through one MoE layer (router + experts), all host
    threads (the CPU path handles tokens one by one, so the rate does not
    depend on the batch)."""
    B = min(T, 16)
    oracle, flags = oracle_module()
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(synth.config_seed(1) + 77))
    L = synth.MoeLayer(rng, D_MODEL, N_EXPERTS, D_EXPERT)
    threads = os.cpu_count() or 1
    pool = oracle.Pool(threads)
    x = rng.normal(0, 1, size=(B, D_MODEL)).astype(np.float32)
    oracle.moe_layer(L, x, TOP_K, True, 0, None, pool)
    t0 = time.perf_counter()
    n = 0
    while n == 0 or time.perf_counter() - t0 < budget_s:
        oracle.moe_layer(L, x, TOP_K, True, 0, None, pool)
        n += 1
    dt = time.perf_counter() - t0
    pool.close()
    return {"value": B * n / dt, "unit": "tok/s", "cores": threads, "kind": "port", "build": flags,
            "sample": f"{n} batches of {B} tokens through one config-1 MoE layer in {dt:.1f}s"}


if __name__ == "__main__":
    main()
