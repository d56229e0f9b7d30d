"""Benchmark: Oasis-500M DiT forwards/s at T=32 on B200 (one process per GPU).

Workload (per GPU, weak scaling): one rollout session, full 32-frame sliding window,
DPM-Solver++ 2M with 5 solver steps per frame; a step = one full-window DiT forward
(4,608 tokens) + the DPM++ update of the newest frame.  The default 80 steps are the
16-frame x 5-step rollout.  Weights are random-init Oasis-500M (608M params, bf16 on
the tensor cores); latents/actions are seeded synthetic inputs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun every rank runs its own sessions; the timed region is bracketed by a
barrier + cuda synchronize and its device time is the max over ranks.  Rank 0 prints
ONE JSON line.  ``--impl reference`` times the CPU restatement of the reference forward
(the upstream DiT is not in the reference tree) on the host cores.
"""

from __future__ import annotations

import argparse
import datetime
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

PKG = "efficient-inference-world-models_b200"
TOKENS = 144
WINDOW = 32
DEPTH = 16
SOLVER_STEPS = 5
STAB_LEVEL = 15
FRAME = (16, 18, 32)
FRAME_ELEMS = 16 * 18 * 32
LINEAR_FLOP_PER_TOKEN = 2 * (3072 + 1024 + 4096 + 4096) * 1024 * 2 * DEPTH  # 0.805 GFLOP


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def load_traffic():
    """Per-launch DRAM traffic of the dominant kernel from the committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f)
    except Exception:
        return None


def max_over_ranks(x: float, dist=None, device="cpu") -> float:
    """Max of a per-rank scalar (device time of the timed region) over all ranks."""
    t = torch.tensor([float(x)], device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def whole_job_rate(units_per_rank: int, world: int, ms_max: float) -> float:
    """Whole-job throughput: every rank processed units_per_rank units; the job took
    the slowest rank's time."""
    return world * units_per_rank / (ms_max / 1000.0)


def synthetic_actions(g, B, T):
    a = torch.zeros(B, T, 25)
    a[..., :23] = (torch.rand(B, T, 23, generator=g) < 0.1).float()
    a[..., 23:] = torch.randn(B, T, 2, generator=g) * 0.3
    return a


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.thread.join(timeout=2)
        mhz, watts, mx, reasons = [], [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 10:
                continue
            if self.uuid and self.uuid not in parts[1]:
                continue
            try:
                mhz.append(float(parts[2]))
                mx = float(parts[3])
            except ValueError:
                continue
            try:
                watts.append(float(parts[4]))
            except ValueError:
                pass
            for n, val in zip(names, parts[6:10]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx,
                "power_w": statistics.median(watts) if watts else None,
                "reasons": sorted(reasons), "samples": len(mhz)}


# ------------------------------------------------------------------------------ CPU baseline
class CpuOracle:
    """The fp32 PyTorch restatement of the reference forward on the host cores, at the
    benchmark shape (B=1, T=32).  One sample = one SpatioTemporal block; a forward is
    embed + final layer (timed once) + 16 blocks."""

    def __init__(self, threads=None):
        from oracle.dit_ref import build_oracle
        pkg = importlib.import_module(PKG)
        if threads:
            torch.set_num_threads(threads)
        self.cores = torch.get_num_threads()
        self.m = build_oracle(pkg.random_state_dict(seed=0, depth=1), depth=1)
        g = torch.Generator().manual_seed(0)
        x = torch.randn(1, WINDOW, *FRAME, generator=g)
        t = torch.full((1, WINDOW), STAB_LEVEL - 1, dtype=torch.long)
        a = synthetic_actions(g, 1, WINDOW)
        with torch.no_grad():
            s = time.perf_counter()
            self.tok, self.c = self.m.embed(x, t, a)
            e = time.perf_counter() - s
            y = self.m.blocks[0](self.tok, self.c)  # warm-up
            s = time.perf_counter()
            self.m.unpatchify_out(y, self.c)
            self.embed_final_s = e + time.perf_counter() - s

    def block_seconds(self):
        with torch.no_grad():
            s = time.perf_counter()
            self.m.blocks[0](self.tok, self.c)
            return time.perf_counter() - s

    def rate(self, block_s):
        return 1.0 / (self.embed_final_s + DEPTH * block_s)


def cpu_oracle_rate(budget_s=12.0, threads=None):
    """Forwards/s of the CPU oracle from ~budget_s of block samples."""
    o = CpuOracle(threads)
    times, start = [], time.perf_counter()
    while len(times) < 2 or (time.perf_counter() - start < budget_s and len(times) < 64):
        times.append(o.block_seconds())
    blk = statistics.median(times)
    return {"value": o.rate(blk), "unit": "forwards/s", "cores": o.cores, "kind": "port",
            "sample": f"fp32 CPU oracle (PyTorch restatement of the reference forward): embed+final "
                      f"once, {len(times)} SpatioTemporal blocks of a B=1 T=32 window (median "
                      f"{blk:.3f} s each); forward = embed+final + 16 blocks"}


def workload_config(world, use_graph):
    """The workload both arms report: one session per GPU, full 32-frame window, the DPM++
    2M rollout of 16 frames x 5 solver steps."""
    return {
        "workload": "Oasis-500M DiT full-window forward + DPM-Solver++ 2M update, 1 session/GPU, "
                    "T=32 sliding window, 5 solver steps/frame (80 steps = 16-frame rollout)",
        "batch_per_gpu": 1, "frames": WINDOW, "tokens_per_forward": WINDOW * 144, "depth": DEPTH,
        "parallelism": f"replicas x{world} (sessions sharded by GPU, no collective on the hot path)",
        "l2": "inputs larger than L2: 1.21 GB of bf16 weights streamed per forward",
        "cuda_graph": use_graph}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    steps, warmup = max(1, args.steps), max(0, args.warmup)
    o = CpuOracle()
    for _ in range(warmup):
        o.block_seconds()
    times = [o.block_seconds() for _ in range(steps)]  # each step: one block sample
    blk = statistics.median(times)
    value = o.rate(blk)
    sample = (f"fp32 CPU oracle (PyTorch restatement of the reference forward; the upstream DiT is "
              f"not in the reference tree): each step one SpatioTemporal block of a B=1 T=32 window "
              f"(median {blk:.3f} s), forward = embed+final ({o.embed_final_s:.3f} s) + 16 blocks")
    line = {
        "impl": "reference", "metric": "Oasis-500M DiT forwards/s (T=32, bf16/FP8/INT4-KV)",
        "value": value, "unit": "forwards/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": 1000.0 / value, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(world, not args.no_graph),
        "cpu_baseline": {"value": value, "unit": "forwards/s", "cores": o.cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "forwards/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------ our arm
def gpu_launches_per_step(depth, chained=True, sampler=True):
    """Kernels of this library per step: im2col, patch GEMM, timestep/action prep, the two
    timestep-MLP GEMMs, the stacked adaLN GEMM and the first LayerNorm (7); then per
    sub-block attention + one chained launch (out-proj+LN, fc1, fc2+LN, next QKV) with the
    first QKV launched alone, or (separate launches, small windows) QKV, attention,
    out-proj, fc1, fc2; the final-layer GEMM; the DPM++ update."""
    head = 7
    if chained:
        body = 1 + 2 * depth * 2
    else:
        body = 2 * depth * 5
    return head + body + 1 + (1 if sampler else 0)


def run_ours(args, rank, world, local_rank):
    pkg = importlib.import_module(PKG)
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    peaks, peak_src = load_peaks()
    B, T = 1, WINDOW
    g = torch.Generator().manual_seed(1000 + rank)
    model = pkg.OasisDiTB200.random(seed=0, depth=DEPTH, device=dev)
    ab = pkg.alphas_cumprod()
    nr = torch.linspace(-1, 999, SOLVER_STEPS + 1)
    levels = []
    for k, idx in enumerate(reversed(range(1, SOLVER_STEPS + 1))):
        t_cur, t_nx = int(nr[idx]), int(nr[idx - 1])
        t_nx = t_cur if t_nx < 0 else t_nx
        levels.append((t_cur, float(ab[t_cur]), 1.0 if idx == 1 else float(ab[t_nx]), k == 0))

    # device-resident rollout state: sliding window of latents + actions
    x = torch.randn(B, T, *FRAME, generator=g).to(dev)
    acts = synthetic_actions(g, B, T).to(dev)
    t_bufs = []
    for (t_cur, _, _, _) in levels:
        tb = torch.full((B, T), STAB_LEVEL - 1, dtype=torch.long, device=dev)
        tb[:, -1] = t_cur
        t_bufs.append(tb)
    v = torch.empty(B, T, *FRAME, device=dev)
    eps_prev = torch.empty(B, FRAME_ELEMS, device=dev)
    noise = torch.randn(64, B, *FRAME, generator=g).clamp(-20, 20).to(dev)

    def step_body(k):
        t_cur, ab_t, ab_nx, first = levels[k]
        model(x, t_bufs[k], acts, out=v)
        pkg.dpmpp2m_update(x, v, eps_prev, ab_t, ab_nx, first)

    def next_frame(i):
        # slide the window by one frame and start a fresh noisy chunk
        x[:, :-1] = x[:, 1:].clone()
        x[:, -1] = noise[i % noise.shape[0]]

    # graphs: one per solver-step index (its t buffer and sampler scalars are baked in)
    use_graph = not args.no_graph
    graphs = []
    stream = torch.cuda.Stream(device=dev)
    for k in range(SOLVER_STEPS):  # eager warm-up of every code path
        step_body(k)
    torch.cuda.synchronize()
    if use_graph:
        with torch.cuda.stream(stream):
            for k in range(SOLVER_STEPS):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    step_body(k)
                graphs.append(gr)
        torch.cuda.synchronize()

    def run_step(s):
        k = s % SOLVER_STEPS
        if k == 0 and s > 0:
            next_frame(s // SOLVER_STEPS)
        if use_graph:
            graphs[k].replay()
        else:
            step_body(k)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for s in range(max(3, args.warmup)):
        run_step(s)
    barrier()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for s in range(args.steps):
        run_step(s)
    e1.record()
    barrier()
    clk = clocks.stop()
    ms_max = max_over_ranks(e0.elapsed_time(e1), dist, dev)
    value = whole_job_rate(B * args.steps, world, ms_max)

    # ---- e2e: public API, pinned host buffers, copies inside the timed region ----
    hx = torch.randn(B, T, *FRAME, generator=g).pin_memory()
    hts = []  # one pinned t buffer per solver step: never rewritten while a copy is in flight
    for (t_cur, _, _, _) in levels:
        ht = torch.full((B, T), STAB_LEVEL - 1, dtype=torch.long)
        ht[:, -1] = t_cur
        hts.append(ht.pin_memory())
    ha = synthetic_actions(g, B, T).pin_memory()
    hout = torch.empty(B, *FRAME).pin_memory()
    dx = torch.empty(B, T, *FRAME, device=dev)
    dt = torch.empty(B, T, dtype=torch.long, device=dev)
    da = torch.empty(B, T, 25, device=dev)
    e2e_steps = max(5, min(args.steps, 40))

    def e2e_step(s):
        k = s % SOLVER_STEPS
        t_cur, ab_t, ab_nx, first = levels[k]
        dx.copy_(hx, non_blocking=True)
        dt.copy_(hts[k], non_blocking=True)
        da.copy_(ha, non_blocking=True)
        model(dx, dt, da, out=v)
        pkg.dpmpp2m_update(dx, v, eps_prev, ab_t, ab_nx, first)
        hout.copy_(dx[:, -1], non_blocking=True)

    for s in range(3):
        e2e_step(s)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for s in range(e2e_steps):
        e2e_step(s)
    f1.record()
    barrier()
    e2e_value = whole_job_rate(B * e2e_steps, world, max_over_ranks(f0.elapsed_time(f1), dist, dev))
    h2d = hx.numel() * 4 + hts[0].numel() * 8 + ha.numel() * 4
    d2h = hout.numel() * 4

    # ---- live per-family kernel timing (CUDA events on the launching stream) ----
    model.set_timing(B, T, True)
    n_prof = 3
    for s in range(n_prof):
        step_body(s % SOLVER_STEPS)
    torch.cuda.synchronize()
    fam = model.get_timing(B, T)
    model.set_timing(B, T, False)
    gemm_ms, gemm_n = fam["gemm"]
    M = B * T * TOKENS
    gemm_flops = LINEAR_FLOP_PER_TOKEN * M * n_prof
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else None
    peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    traffic = load_traffic()
    per_fwd_ms = ms_max / args.steps
    kv = {}
    if rank == 0 and not args.skip_kv:
        kv = kv_configs(pkg, model, dev, g)

    if dist is not None:
        dist.barrier()
    if rank == 0:
        cpu = None
        if world == 1 and not args.skip_cpu:
            try:
                cpu = cpu_oracle_rate(budget_s=args.cpu_budget)
            except Exception as e:  # the baseline is reported, never required
                cpu = {"value": None, "unit": "forwards/s", "cores": None, "kind": "port",
                       "sample": f"failed: {e}"}
        line = {
            "metric": "Oasis-500M DiT forwards/s (T=32, bf16/FP8/INT4-KV)",
            "value": value, "unit": "forwards/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": per_fwd_ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) latents, Bernoulli(0.1)+N(0,0.3) actions, random-init weights)",
            "config": workload_config(world, use_graph),
            "e2e": {"value": e2e_value, "unit": "forwards/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps},
            "gpu_launches": gpu_launches_per_step(DEPTH) * args.steps,
            "roofline": {"bound": "tensor",
                         "kernel": "projection GEMMs: gemm_chain_kernel (per sub-block: out-proj + "
                                   "LayerNorm, fc1, fc2 + LayerNorm, next QKV on tcgen05 CTA pairs) "
                                   "+ the first QKV; their time includes the LayerNorm phases",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": (achieved / peak) if achieved else None,
                         "peak_source": f"{peak_src} bf16_tflops_sustained (kernel timed inside a long step)",
                         "traffic": traffic.get("bytes_per_launch") if traffic else None,
                         "traffic_note": traffic.get("note") if traffic else "no ncu capture committed",
                         "algorithmic_flop_per_launch": gemm_flops / max(1, gemm_n),
                         "launches_timed": gemm_n},
            "forward_tflops": LINEAR_FLOP_PER_TOKEN * M / (per_fwd_ms / 1000.0) / 1e12,
            "kernel_ms_per_forward": {k: round(vv[0] / n_prof, 4) for k, vv in fam.items()},
            "clocks": clk,
            "cpu_baseline": cpu,
            "kv_configs": kv,
        }
        print(json.dumps(line), flush=True)
    graphs.clear()
    if dist is not None:
        dist.destroy_process_group()
    return 0


def kv_configs(pkg, model, dev, g):
    """Secondary lines: incremental forwards/s with an FP8 cache (B=8) and a progressive
    INT4 cache (B=16, newest 8 frames bf16), T=32 (31 cached frames)."""
    out = {}
    for name, B, kinds in (("fp8_b8", 8, ["fp8"] * 31),
                           ("int4_b16", 16, ["int4"] * 23 + ["bf16"] * 8),
                           ("bf16_b8", 8, ["bf16"] * 31)):
        try:
            x = torch.randn(B, WINDOW, *FRAME, generator=g).to(dev)
            t = torch.full((B, WINDOW), STAB_LEVEL - 1, dtype=torch.long, device=dev)
            a = synthetic_actions(g, B, WINDOW).to(dev)
            cache = pkg.KVCacheB200(B, model.depth, kinds, device=dev)
            model(x, t, a, kv_cache=cache)  # prefill
            xn, tn, an = x[:, -1].contiguous(), torch.full((B,), 599, device=dev), a[:, -1].contiguous()
            vout = torch.empty(B, *FRAME, device=dev)
            for _ in range(3):
                model.forward_cached(xn, tn, an, cache, n_past=31, out=vout)
            gr = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(device=dev)
            with torch.cuda.stream(s):
                with torch.cuda.graph(gr, stream=s):
                    model.forward_cached(xn, tn, an, cache, n_past=31, out=vout)
            torch.cuda.synchronize()
            for _ in range(3):
                gr.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = 20
            e0.record()
            for _ in range(n):
                gr.replay()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / n
            out[name] = {"forwards_per_s": B / (ms / 1000.0), "ms_per_call": ms, "batch": B,
                         "cached_frames": 31, "kv_bytes": cache.nbytes,
                         "kv_bytes_bf16_equiv": cache.bf16_equivalent_bytes()}
            del gr, cache
        except Exception as e:
            out[name] = {"error": str(e)[:200]}
    return out


def run_isolated(args, local_rank):
    """Isolated kernels (one GPU): the attention sweep of the benchmark plan and single
    GEMM shapes for ncu captures.  Prints one JSON line per case."""
    pkg = importlib.import_module(PKG)
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    peaks, _ = load_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    g = torch.Generator(device=dev).manual_seed(0)
    stream = torch.cuda.current_stream()

    def timeit(fn, n):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    if args.isolated == "gemm":
        M, N, K = args.M, args.N, args.K
        A = torch.randn(M, K, device=dev, generator=g).bfloat16()
        Bw = torch.randn(N, K, device=dev, generator=g).bfloat16()
        D = torch.empty(M, N, device=dev).bfloat16()
        fn = lambda: pkg._native.call("oasis_gemm_bf16", A.data_ptr(), Bw.data_ptr(), D.data_ptr(),
                                      None, M, N, K, K, K, N, 0, stream.cuda_stream)
        ms = timeit(fn, args.steps)
        tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
        print(json.dumps({"case": f"gemm M={M} N={N} K={K}", "ms": ms, "tflops": tf,
                          "frac_burst": tf / peaks.get("bf16_tflops", 1590.0)}), flush=True)
        return 0
    # attention sweep: spatial (B*T frames of 144 tokens) and causal temporal with
    # bf16 / FP8 / INT4 K/V (every K/V frame read from the cache for the quantised kinds)
    for frames in (32, 256, 1024, 4096):
        qkv = torch.randn(frames * TOKENS, 3072, device=dev, generator=g).bfloat16()
        out = torch.empty(frames * TOKENS, 1024, device=dev).bfloat16()
        ms = timeit(lambda: pkg.attn_spatial(qkv, out=out), args.steps)
        byts = frames * TOKENS * 1024 * 2 * 4
        print(json.dumps({"case": f"spatial BT={frames}", "ms": ms, "GBps": byts / ms / 1e6,
                          "frac_hbm": byts / ms / 1e6 / hbm,
                          "tflops": 4 * 144 * 144 * 64 * 16 * frames / ms / 1e9}), flush=True)
        del qkv, out
    for T in (8, 16, 32):
        for B in (1, 8, 32):
            qkv = torch.randn(B * T * TOKENS, 3072, device=dev, generator=g).bfloat16()
            out = torch.empty(B * T * TOKENS, 1024, device=dev).bfloat16()
            for kind in ("bf16", "fp8", "int4"):
                if kind == "bf16":
                    fn = lambda: pkg.attn_temporal(qkv, batch=B, q_frames=T, out=out)
                    kv_bytes = B * T * TOKENS * 1024 * 2 * 2
                else:
                    cache = pkg.KVCacheB200.uniform(B, 1, T, kind, device=dev)
                    cache.store(qkv, layer=0)
                    fn = lambda: pkg.attn_temporal(qkv, batch=B, q_frames=T, n_past=T, n_kv=T,
                                                   cache=cache, layer=0, out=out)
                    per = 1 if kind == "fp8" else 0.5
                    kv_bytes = int(B * T * TOKENS * 1024 * 2 * per) + (
                        B * T * 16 * 2 * 2 if kind == "fp8" else B * T * TOKENS * 16 * 2 * 2 * 2)
                ms = timeit(fn, args.steps)
                byts = kv_bytes + B * T * TOKENS * 1024 * 2 * 2  # + Q read + O write
                print(json.dumps({"case": f"temporal T={T} B={B} kv={kind}", "ms": ms,
                                  "GBps": byts / ms / 1e6, "frac_hbm": byts / ms / 1e6 / hbm}), flush=True)
            del qkv, out
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=80)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-kv", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--isolated", choices=["attention", "gemm"], default=None)
    ap.add_argument("--M", type=int, default=36864)
    ap.add_argument("--N", type=int, default=1024)
    ap.add_argument("--K", type=int, default=4096)
    args = ap.parse_args()
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.isolated:
        return run_isolated(args, local_rank)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
