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
import platform
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
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"],
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


class NvmlClockSampler:
    """Clocks during the timed region from NVML, polled every `period_s` by a thread of
    this process (read-only queries: the SM clock, its maximum, power and the active
    clock-event reasons).  It starts without the ~0.1 s start-up of an nvidia-smi
    process, so a timed region of 20 steps (~90 ms) still gets tens of samples; samples
    outside [mark_begin(), mark_end()] are dropped."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, uuid, period_s=0.001):
        import pynvml
        self.nv = pynvml
        pynvml.nvmlInit()
        self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        self.period = period_s
        self.samples = []
        self.t0 = self.t1 = None
        self.stop_flag = threading.Event()

    def start(self):
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def _run(self):
        nv = self.nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        n, watts = 0, None
        while not self.stop_flag.is_set():
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                bits = int(get_reasons(self.h))
                if n % 10 == 0:  # the power reading is an average over a longer window anyway
                    watts = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                self.samples.append((time.perf_counter(), mhz, watts, bits))
                n += 1
            except Exception:
                pass
            time.sleep(self.period)

    def mark_begin(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def stop(self):
        self.stop_flag.set()
        self.thread.join(timeout=2)
        inside = [x for x in self.samples if self.t0 is not None and self.t0 <= x[0] <= (self.t1 or x[0])]
        reasons = set()
        for _, _, _, bits in inside:
            for name, const in self.REASONS:
                if bits & getattr(self.nv, const, 0):
                    reasons.add(name)
        mhz = [x[1] for x in inside]
        watts = [x[2] for x in inside if x[2] is not None]
        try:
            self.nv.nvmlShutdown()
        except Exception:
            pass
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "power_w": statistics.median(watts) if watts else None,
                "reasons": sorted(reasons), "samples": len(mhz), "source": "nvml",
                "sm_mhz_min": min(mhz) if mhz else None}


def clock_sampler(uuid):
    """The NVML sampler where NVML answers, else the nvidia-smi one."""
    try:
        return NvmlClockSampler(uuid)
    except Exception:
        return ClockSampler(uuid)


# ------------------------------------------------------------------------------ CPU baseline
def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


class CpuOracle:
    """The fp32 PyTorch restatement of the reference forward (the oracle) on the host
    cores, whole Oasis-500M forwards (depth 16) at B=1: the benchmark window (T=32) and
    the reference's CPU configuration (T=4)."""

    def __init__(self, threads=None):
        from oracle.dit_ref import build_oracle
        pkg = importlib.import_module(PKG)
        torch.set_num_threads(threads or os.cpu_count() or 1)
        self.cores = torch.get_num_threads()
        self.m = build_oracle(pkg.random_state_dict(seed=0, depth=DEPTH), depth=DEPTH)
        g = torch.Generator().manual_seed(0)
        self.inputs = {}
        for T in (WINDOW, 4):  # seeded N(0,1) latents, t ~ U{0..999}, actions as config 0
            self.inputs[T] = (torch.randn(1, T, *FRAME, generator=g),
                              torch.randint(0, 1000, (1, T), generator=g),
                              synthetic_actions(g, 1, T))

    def forward_seconds(self, T=WINDOW) -> float:
        x, t, a = self.inputs[T]
        with torch.no_grad():
            s = time.perf_counter()
            self.m(x, t, a)
            return time.perf_counter() - s


def cpu_oracle_rate(budget_s=15.0, threads=None):
    """Forwards/s of the CPU oracle: whole T=32 forwards for ~budget_s (at least 2), plus
    three whole forwards of the reference's CPU configuration (B=1, T=4)."""
    o = CpuOracle(threads)
    o.forward_seconds(4)
    o.forward_seconds()  # warm-up
    times, start = [], time.perf_counter()
    while len(times) < 2 or (time.perf_counter() - start < budget_s and len(times) < 20):
        times.append(o.forward_seconds())
    t4 = [o.forward_seconds(4) for _ in range(3)]
    med = statistics.median(times)
    return {"value": 1.0 / med, "unit": "forwards/s", "cores": o.cores, "kind": "port",
            "cpu": cpu_model(),
            "sample": f"{len(times)} whole fp32 forwards of the B=1 T=32 window (median {med:.3f} s) "
                      f"by the oracle (PyTorch restatement of the reference forward)",
            "config0_forwards_per_s": 1.0 / statistics.median(t4),
            "config0": "B=1, T=4, fp32, seed 0: 3 whole forwards"}


class TorchBf16DiT:
    """Same-box library comparator: the Oasis DiT-S/2 forward written directly in eager
    PyTorch bf16 (cuBLAS GEMMs, SDPA attention, axial / temporal RoPE tables on the GPU) on
    the same random weights.  A comparator only: nothing of it is on the product path."""

    def __init__(self, sd, depth, dev):
        bf = torch.bfloat16
        self.w = {k: v.to(dev, bf) for k, v in sd.items()}
        self.depth = depth

        def angles(pos, freqs):  # (n,) x (f,) -> (n, 2f), pairs interleaved
            return (pos[:, None] * freqs).repeat_interleave(2, dim=-1)

        # spatial: 16 "pixel" frequencies per axis over linspace(-1, 1) positions, H then W
        pf = torch.linspace(1.0, 128.0, 16, device=dev) * math.pi
        ah = angles(torch.linspace(-1.0, 1.0, 9, device=dev), pf)
        aw = angles(torch.linspace(-1.0, 1.0, 16, device=dev), pf)
        sp = torch.cat([ah[:, None, :].expand(9, 16, 32), aw[None, :, :].expand(9, 16, 32)], -1).reshape(144, 64)
        self.s_cos, self.s_sin = sp.cos().to(bf), sp.sin().to(bf)
        # temporal: 32 "lang" frequencies over frame positions 0..31
        lf = 1.0 / (10000.0 ** (torch.arange(0, 64, 2, device=dev).float() / 64))
        tp = angles(torch.arange(WINDOW, device=dev).float(), lf)
        self.t_cos, self.t_sin = tp.cos().to(bf), tp.sin().to(bf)

    @staticmethod
    def _rope(x, cos, sin):
        a, b = x.unflatten(-1, (-1, 2)).unbind(-1)
        return x * cos + torch.stack((-b, a), dim=-1).flatten(-2) * sin

    def _sub(self, x, c, i, kind):
        F = torch.nn.functional
        w, p = self.w, f"blocks.{i}.{kind}_"
        B, T = x.shape[:2]
        mod = F.linear(F.silu(c), w[p + "adaLN_modulation.1.weight"], w[p + "adaLN_modulation.1.bias"])
        sh1, sc1, g1, sh2, sc2, g2 = mod[:, :, None, :].chunk(6, dim=-1)
        h = F.layer_norm(x, (1024,), eps=1e-6) * (1 + sc1) + sh1
        q, k, v = F.linear(h, w[p + "attn.to_qkv.weight"]).view(B, T, 144, 3, 16, 64).unbind(3)
        if kind == "s":
            q, k, v = (z.reshape(B * T, 144, 16, 64).transpose(1, 2) for z in (q, k, v))
            q, k = self._rope(q, self.s_cos, self.s_sin), self._rope(k, self.s_cos, self.s_sin)
            o = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, T, 144, 1024)
        else:
            q, k, v = (z.permute(0, 2, 3, 1, 4).reshape(B * 144, 16, T, 64) for z in (q, k, v))
            cos, sin = self.t_cos[:T], self.t_sin[:T]
            q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            o = o.reshape(B, 144, 16, T, 64).permute(0, 3, 1, 2, 4).reshape(B, T, 144, 1024)
        x = x + g1 * F.linear(o, w[p + "attn.to_out.weight"], w[p + "attn.to_out.bias"])
        h = F.layer_norm(x, (1024,), eps=1e-6) * (1 + sc2) + sh2
        h = F.gelu(F.linear(h, w[p + "mlp.fc1.weight"], w[p + "mlp.fc1.bias"]), approximate="tanh")
        return x + g2 * F.linear(h, w[p + "mlp.fc2.weight"], w[p + "mlp.fc2.bias"])

    def __call__(self, x, t, a):
        F = torch.nn.functional
        w = self.w
        B, T = x.shape[:2]
        tok = F.conv2d(x.reshape(B * T, 16, 18, 32).to(torch.bfloat16), w["x_embedder.proj.weight"],
                       w["x_embedder.proj.bias"], stride=2)
        tok = tok.permute(0, 2, 3, 1).reshape(B, T, 144, 1024)
        half = 128
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=x.device).float() / half)
        args = t.reshape(-1, 1).float() * freqs[None]
        temb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1).to(torch.bfloat16)
        temb = F.linear(F.silu(F.linear(temb, w["t_embedder.mlp.0.weight"], w["t_embedder.mlp.0.bias"])),
                        w["t_embedder.mlp.2.weight"], w["t_embedder.mlp.2.bias"])
        c = temb.reshape(B, T, 1024) + F.linear(a.to(torch.bfloat16), w["external_cond.weight"], w["external_cond.bias"])
        for i in range(self.depth):
            tok = self._sub(self._sub(tok, c, i, "s"), c, i, "t")
        shift, scale = F.linear(F.silu(c), w["final_layer.adaLN_modulation.1.weight"],
                                w["final_layer.adaLN_modulation.1.bias"])[:, :, None, :].chunk(2, dim=-1)
        y = F.linear(F.layer_norm(tok, (1024,), eps=1e-6) * (1 + scale) + shift, w["final_layer.linear.weight"],
                     w["final_layer.linear.bias"])
        y = y.reshape(B * T, 9, 16, 2, 2, 16)
        return torch.einsum("nhwpqc->nchpwq", y).reshape(B, T, 16, 18, 32)


def library_bar(dev, model, steps=10):
    """Same-box library comparator (TorchBf16DiT), B=1 T=32 forwards/s, with the rel-L2 of
    its v against this package's forward on the same inputs."""
    try:
        pkg = importlib.import_module(PKG)
        m = TorchBf16DiT(pkg.random_state_dict(seed=0, depth=DEPTH), DEPTH, dev)
        g = torch.Generator().manual_seed(0)
        x = torch.randn(1, WINDOW, *FRAME, generator=g).to(dev)
        t = torch.full((1, WINDOW), STAB_LEVEL - 1, dtype=torch.long, device=dev)
        a = synthetic_actions(g, 1, WINDOW).to(dev)
        with torch.no_grad():
            for _ in range(3):
                v_lib = m(x, t, a)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                m(x, t, a)
            e1.record()
            torch.cuda.synchronize()
            v_ours = model(x, t, a)
            rel = ((v_lib.float() - v_ours.float()).norm() / v_ours.float().norm()).item()
        ms = e0.elapsed_time(e1) / steps
        del m
        torch.cuda.empty_cache()
        return {"value": 1000.0 / ms, "unit": "forwards/s", "ms_per_forward": ms, "rel_l2_vs_b200_path": rel,
                "what": "the same DiT forward in eager PyTorch bf16 on this GPU (cuBLAS + SDPA), B=1 T=32, "
                        "same random weights"}
    except Exception as e:  # a comparator, never required
        return {"value": None, "error": str(e)[:200]}


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
    """The reference arm: the oracle's whole fp32 forwards (B=1, T=32) on the host cores,
    one forward per step (the reference's own forward is not in its tree)."""
    if rank != 0:
        return 0
    steps, warmup = max(1, args.steps), max(0, args.warmup)
    o = CpuOracle(os.cpu_count() or 1)
    for _ in range(warmup):
        o.forward_seconds()
    times = [o.forward_seconds() for _ in range(steps)]
    total = sum(times)
    value = steps / total
    t4 = [o.forward_seconds(4) for _ in range(3)]
    sample = (f"fp32 CPU oracle (PyTorch restatement of the reference forward; the upstream DiT is "
              f"not in the reference tree): each step one whole B=1 T=32 forward "
              f"(mean {total / steps:.3f} s, median {statistics.median(times):.3f} s)")
    line = {
        "impl": "reference", "metric": "Oasis-500M DiT forwards/s (T=32, bf16/FP8/INT4-KV)",
        "value": value, "unit": "forwards/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": 1000.0 * total / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(world, not args.no_graph),
        "cpu_baseline": {"value": value, "unit": "forwards/s", "cores": o.cores, "kind": "port",
                         "cpu": cpu_model(), "sample": sample,
                         "config0_forwards_per_s": 1.0 / statistics.median(t4),
                         "config0": "B=1, T=4, fp32, seed 0: 3 whole forwards"},
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

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    # started before the warm-up steps, so it is polling steadily when the timed region
    # begins; only the samples taken between mark_begin and mark_end are kept
    clocks = clock_sampler(uuid)
    clocks.start()
    for s in range(max(3, args.warmup)):
        run_step(s)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    if hasattr(clocks, "mark_begin"):
        clocks.mark_begin()
    e0.record()
    for s in range(args.steps):
        run_step(s)
    e1.record()
    barrier()
    if hasattr(clocks, "mark_end"):
        clocks.mark_end()
    clk = clocks.stop()
    per_rank_ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(per_rank_ms, dist, dev)
    value = whole_job_rate(B * args.steps, world, ms_max)

    # ---- e2e: public API, pinned host buffers, copies inside the timed region ----
    # Every step copies its own inputs (window latents, t, actions) from pinned host memory
    # and reads its result (the updated newest frame) back.  The copies run on a copy
    # stream with two device input sets, as a serving loop pipelines them: step s+1's
    # inputs land while step s computes, and step s's result leaves while step s+1 computes.
    hx = torch.randn(B, T, *FRAME, generator=g).pin_memory()
    hts = []  # one pinned t buffer per solver step: never rewritten while a copy is in flight
    for (t_cur, _, _, _) in levels:
        ht = torch.full((B, T), STAB_LEVEL - 1, dtype=torch.long)
        ht[:, -1] = t_cur
        hts.append(ht.pin_memory())
    ha = synthetic_actions(g, B, T).pin_memory()
    hout = [torch.empty(B, *FRAME).pin_memory() for _ in range(2)]
    dx = [torch.empty(B, T, *FRAME, device=dev) for _ in range(2)]
    dt = [torch.empty(B, T, dtype=torch.long, device=dev) for _ in range(2)]
    da = [torch.empty(B, T, 25, device=dev) for _ in range(2)]
    e2e_steps = max(5, min(args.steps, 40))
    comp = torch.cuda.current_stream(dev)
    copy_s = torch.cuda.Stream(device=dev)
    ready = [torch.cuda.Event() for _ in range(2)]     # inputs of the set landed
    computed = [torch.cuda.Event() for _ in range(2)]  # the step using the set finished
    freed = [torch.cuda.Event() for _ in range(2)]     # its result left: the set may be refilled
    for ev in freed:
        ev.record(copy_s)

    def e2e_h2d(s):
        i = s % 2
        with torch.cuda.stream(copy_s):
            copy_s.wait_event(freed[i])
            dx[i].copy_(hx, non_blocking=True)
            dt[i].copy_(hts[s % SOLVER_STEPS], non_blocking=True)
            da[i].copy_(ha, non_blocking=True)
            ready[i].record(copy_s)

    def e2e_call(i, k):
        t_cur, ab_t, ab_nx, first = levels[k]
        model(dx[i], dt[i], da[i], out=v)
        pkg.dpmpp2m_update(dx[i], v, eps_prev, ab_t, ab_nx, first)

    # the API call of each (input set, solver step) captured once, as a serving loop replays
    # it; the copies stay outside the graphs, every step
    e2e_graphs = {}
    if use_graph:
        for i in range(2):
            for k in range(SOLVER_STEPS):
                e2e_call(i, k)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for i in range(2):
                for k in range(SOLVER_STEPS):
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr, stream=stream):
                        e2e_call(i, k)
                    e2e_graphs[(i, k)] = gr
        torch.cuda.synchronize()

    def e2e_step(s, last):
        i = s % 2
        k = s % SOLVER_STEPS
        if not last:
            e2e_h2d(s + 1)
        comp.wait_event(ready[i])
        if use_graph:
            e2e_graphs[(i, k)].replay()
        else:
            e2e_call(i, k)
        computed[i].record(comp)
        with torch.cuda.stream(copy_s):
            copy_s.wait_event(computed[i])
            hout[i].copy_(dx[i][:, -1], non_blocking=True)
            freed[i].record(copy_s)

    e2e_h2d(0)
    for s in range(3):
        e2e_step(s, s == 2)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(comp)
    copy_s.wait_event(f0)
    e2e_h2d(0)
    for s in range(e2e_steps):
        e2e_step(s, s == e2e_steps - 1)
    comp.wait_event(freed[(e2e_steps - 1) % 2])  # the last result has left
    f1.record(comp)
    barrier()
    e2e_value = whole_job_rate(B * e2e_steps, world, max_over_ranks(f0.elapsed_time(f1), dist, dev))
    h2d = hx.numel() * 4 + hts[0].numel() * 8 + ha.numel() * 4
    d2h = hout[0].numel() * 4

    # ---- per-family kernel time inside a graph-replayed step: a second capture of the same
    # step with timing events as graph nodes (the timed graphs carry none), replayed a few
    # times; the families' times come from the last replay ----
    M = B * T * TOKENS
    fam_src = "graph"
    n_prof = 5
    try:
        # five captures of the step (each with its own timing events), each replayed twice:
        # the family times are the mean over the second replays of the five graphs
        model.set_timing(B, T, True)
        gts = []
        for _ in range(n_prof):
            gt = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(gt, stream=stream):
                    step_body(1)
            gts.append(gt)
        for _ in range(2):
            for gt in gts:
                gt.replay()
        torch.cuda.synchronize()
        fam = model.get_timing(B, T)
        del gts
    except Exception:  # eager fallback: events on the launching stream
        fam_src = "eager"
        model.set_timing(B, T, True)
        n_prof = 3
        for s in range(n_prof):
            step_body(s % SOLVER_STEPS)
        torch.cuda.synchronize()
        fam = model.get_timing(B, T)
    model.set_timing(B, T, False)
    gemm_ms, gemm_n = fam["gemm"]
    gemm_flops = LINEAR_FLOP_PER_TOKEN * M * n_prof
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else None
    peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    traffic = load_traffic()
    per_fwd_ms = ms_max / args.steps
    kv, sweep, lib = {}, [], None
    if rank == 0 and not args.skip_kv:
        kv = kv_configs(pkg, model, dev, g, peaks)
    vae, rollout = {}, {}
    if rank == 0 and not args.skip_kv:
        rollout = rollout_bench(pkg, model, dev)
    if rank == 0 and not args.skip_sweep:
        sweep = attention_sweep(pkg, dev, peaks.get("hbm_gbs", 6650.0), reps=10)
        vae = vae_decode_bench(pkg, dev, peaks)
    if rank == 0 and world == 1 and not args.skip_cpu:
        lib = library_bar(dev, model)

    # every rank's own time and clocks, gathered outside the timed region
    mine = {"rank": rank, "ms_per_step": per_rank_ms / args.steps, "sm_mhz": clk.get("sm_mhz"),
            "power_w": clk.get("power_w"), "reasons": clk.get("reasons")}
    per_rank = [mine]
    if dist is not None:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, mine)
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
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "copies": "every step, on a copy stream with two device input sets (step s+1's "
                              "inputs land while step s computes)",
                    "launch": "graph replay of the API call" if use_graph else "eager"},
            "gpu_launches": gpu_launches_per_step(DEPTH) * args.steps,
            "roofline": {"bound": "tensor",
                         "kernel": "projection GEMMs: gemm_chain_kernel (per sub-block: out-proj + "
                                   "LayerNorm, fc1, fc2 + LayerNorm, next QKV on tcgen05 CTA pairs) "
                                   "+ the first QKV; their time includes the LayerNorm phases",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": (achieved / peak) if achieved else None,
                         "peak_source": f"{peak_src} bf16_tflops_sustained (kernel timed inside a long step)",
                         "timed_in": f"{fam_src}-replayed step (CUDA events on the launching stream)",
                         "traffic": traffic.get("bytes_per_launch") if traffic else None,
                         "traffic_note": traffic.get("note") if traffic else "no ncu capture committed",
                         "algorithmic_flop_per_launch": gemm_flops / max(1, gemm_n),
                         "launches_timed": gemm_n},
            "forward_tflops": LINEAR_FLOP_PER_TOKEN * M / (per_fwd_ms / 1000.0) / 1e12,
            "kernel_ms_per_forward": {k: round(vv[0] / n_prof, 4) for k, vv in fam.items()},
            "clocks": clk,
            "per_rank": per_rank,
            "cpu_baseline": cpu,
            "library_bar": lib,
            "kv_configs": kv,
            "attention_sweep": sweep,
            "vae_decode": vae,
            "rollout": rollout,
        }
        print(json.dumps(line), flush=True)
    graphs.clear()
    if dist is not None:
        dist.destroy_process_group()
    return 0


def _cached_call_flops(B):
    """Algorithmic FLOPs of one incremental forward of B sessions (144 new tokens each):
    the linear projections, the stacked adaLN GEMM, spatial attention over 144 tokens and
    temporal attention of the new frame over the 32-frame window."""
    tokens = B * TOKENS
    ada = 2.0 * B * 1024 * (2 * DEPTH * 6144 + 2048)
    spatial = 4.0 * TOKENS * TOKENS * 64 * 16 * B * DEPTH
    temporal = 4.0 * WINDOW * 64 * 16 * tokens * DEPTH
    return LINEAR_FLOP_PER_TOKEN * tokens + ada + spatial + temporal


def kv_configs(pkg, model, dev, g, peaks):
    """Incremental forwards/s with an FP8 cache (B=8), a progressive INT4 cache (B=16,
    newest 8 frames bf16) and a bf16 cache (B=8), T=32 (31 cached frames), each with its
    roofline: algorithmic bytes = every weight once + the whole cache, FLOPs as
    _cached_call_flops."""
    out = {}
    hbm = peaks.get("hbm_gbs", 6650.0)
    tpk = peaks.get("bf16_tflops_sustained", 1400.0)
    wbytes = model.weights.nbytes
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
            # three rounds of 20 replays, the median round: the calls follow the power-capped
            # main loop, and one round can catch a clock transient
            rounds = []
            for _ in range(3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                n = 20
                e0.record()
                for _ in range(n):
                    gr.replay()
                e1.record()
                torch.cuda.synchronize()
                rounds.append(e0.elapsed_time(e1) / n)
            ms = sorted(rounds)[1]
            byts = wbytes + cache.nbytes
            flops = _cached_call_flops(B)
            out[name] = {"forwards_per_s": B / (ms / 1000.0), "ms_per_call": ms, "ms_rounds": rounds, "batch": B,
                         "cached_frames": 31, "kv_bytes": cache.nbytes,
                         "kv_bytes_bf16_equiv": cache.bf16_equivalent_bytes(),
                         "roofline": {"bytes": byts, "GBps": byts / ms / 1e6,
                                      "frac_hbm": byts / ms / 1e6 / hbm, "flop": flops,
                                      "TFLOPs": flops / ms / 1e9, "frac_tensor": flops / ms / 1e9 / tpk,
                                      "note": "bytes = every weight once + the whole KV cache; "
                                              "of measured hbm_gbs / bf16_tflops_sustained"}}
            del gr, cache
        except Exception as e:
            out[name] = {"error": str(e)[:200]}
    return out


def rollout_bench(pkg, model, dev, frames=16, steps=SOLVER_STEPS):
    """The public rollout API (`rollout_dpmpp`, CUDA graphs per frame) over a full 32-frame
    window (31 prompt frames, then `frames` new ones, 5 DPM++ 2M steps each): every solver
    step a full-window forward, or the first step of each frame full-window (rebuilding the
    bf16 cache of the 31 past frames) and the other steps incremental forwards of the new
    frame.  Frames/s of the second of two calls (graphs are captured inside each call)."""
    out = {}
    try:
        g = torch.Generator().manual_seed(7)
        prompt = torch.randn(1, WINDOW - 1, *FRAME, generator=g).to(dev)
        acts = synthetic_actions(g, 1, WINDOW - 1 + frames).to(dev)
        for name, use_cache in (("full_window_steps", False), ("cached_steps", True)):
            ms = None
            for _ in range(2):
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                pkg.rollout_dpmpp(model, prompt, acts, num_frames=frames, solver_steps=steps,
                                  use_cache=use_cache, use_graph=True)
                e1.record()
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1)
            out[name] = {"frames_per_s": frames / (ms / 1000.0), "ms": ms, "frames": frames,
                         "solver_steps": steps}
        out["note"] = ("one session, window 32; causal temporal attention: the 31 context frames "
                       "never see the new frame, so their outputs are the same at every solver "
                       "step of a frame and the incremental steps skip only unused work")
    except Exception as e:
        out["error"] = str(e)[:200]
    return out


def replay_ms(fn, reps, dev):
    """Mean device ms of one `fn()` call: three warm-up calls, then `reps` calls captured in
    one CUDA graph and replayed once between CUDA events, so host launch cost (dozens of
    launches per VAE decode) stays out of the figure.  Falls back to timed eager calls if
    the capture fails.  Returns (ms, "graph" | "eager")."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=torch.cuda.Stream(device=dev)):
            for _ in range(reps):
                fn()
        gr.replay()
        torch.cuda.synchronize()
        e0.record()
        gr.replay()
        e1.record()
        torch.cuda.synchronize()
        del gr
        return e0.elapsed_time(e1) / reps, "graph"
    except RuntimeError:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps, "eager"


def vae_decode_bench(pkg, dev, peaks, reps=10):
    """Latent decoder (`vae.decode`): the newest frame of a session (1 frame) and a whole
    32-frame window, frames/s with the tensor roofline of its projections + attention."""
    out = {}
    try:
        dec = pkg.OasisVAEDecoderB200.random(seed=0, depth=12, device=dev)
        tpk = peaks.get("bf16_tflops_sustained", 1400.0)
        for F in (1, 32):
            z = torch.randn(F, 576, 16, device=dev, generator=torch.Generator(device=dev).manual_seed(F))
            o = torch.empty(F, 3, 360, 640, device=dev)
            ms, how = replay_ms(lambda: dec.decode(z, out=o), reps, dev)
            flop = F * 576 * 12 * 2 * (12 * 1024 * 1024) + F * 12 * 16 * 4 * 576 * 576 * 64
            out[f"frames_{F}"] = {"frames_per_s": F / (ms / 1e3), "ms": ms, "tflops": flop / ms / 1e9,
                                  "frac_tensor": flop / ms / 1e9 / tpk, "launch": how}
        del dec
        torch.cuda.empty_cache()
    except Exception as e:  # an extra line, never required
        out = {"error": str(e)[:200]}
    return out


def attention_sweep(pkg, dev, hbm, reps=20, only=None):
    """The isolated attention sweep (benchmark configuration 4): spatial attention over
    B*T frames of 144 tokens, causal temporal attention over T frames for B*144
    sequences with bf16 K/V (full-window kernel) or every K/V frame from an FP8 / INT4
    cache, and the one-query-frame kernel of the incremental forward (31 cached frames).
    Bytes: q, k, v read and o written once (k, v at their stored width).  `only`: run just
    the cases whose name contains it."""
    g = torch.Generator(device=dev).manual_seed(0)

    def wanted(case):
        return only is None or only in case

    def timeit(fn):
        return replay_ms(fn, reps, dev)[0]

    out = []
    for frames in (32, 256, 1024, 4096):
        if not wanted(f"spatial BT={frames}"):
            continue
        qkv = torch.randn(frames * TOKENS, 3072, device=dev, generator=g).bfloat16()
        o = torch.empty(frames * TOKENS, 1024, device=dev).bfloat16()
        ms = timeit(lambda: pkg.attn_spatial(qkv, out=o))
        byts = frames * TOKENS * 1024 * 2 * 4
        out.append({"case": f"spatial BT={frames}", "ms": ms, "GBps": byts / ms / 1e6,
                    "frac_hbm": byts / ms / 1e6 / hbm,
                    "tflops": 4 * 144 * 144 * 64 * 16 * frames / ms / 1e9})
        del qkv, o
    for T in (8, 16, 32):
        for B in (1, 8, 32):
            kinds = [k for k in ("bf16", "fp8", "int4") if wanted(f"temporal T={T} B={B} kv={k}")]
            if not kinds:
                continue
            qkv = torch.randn(B * T * TOKENS, 3072, device=dev, generator=g).bfloat16()
            o = torch.empty(B * T * TOKENS, 1024, device=dev).bfloat16()
            for kind in kinds:
                if kind == "bf16":
                    fn = lambda: pkg.attn_temporal(qkv, batch=B, q_frames=T, out=o)
                    kv_bytes = B * T * TOKENS * 1024 * 2 * 2
                else:
                    cache = pkg.KVCacheB200.uniform(B, 1, T, kind, device=dev)
                    cache.store(qkv, layer=0)
                    fn = lambda: pkg.attn_temporal(qkv, batch=B, q_frames=T, n_past=T, n_kv=T,
                                                   cache=cache, layer=0, out=o)
                    kv_bytes = cache.nbytes
                ms = timeit(fn)
                byts = kv_bytes + B * T * TOKENS * 1024 * 2 * 2  # + q read + o written
                out.append({"case": f"temporal T={T} B={B} kv={kind}", "ms": ms,
                            "GBps": byts / ms / 1e6, "frac_hbm": byts / ms / 1e6 / hbm})
            del qkv, o
    for B in (8, 32):
        kinds = [k for k in ("bf16", "fp8", "int4") if wanted(f"decode past=31 B={B} kv={k}")]
        if not kinds:
            continue
        new = torch.randn(B * TOKENS, 3072, device=dev, generator=g).bfloat16()
        o = torch.empty(B * TOKENS, 1024, device=dev).bfloat16()
        past = torch.randn(B * 31 * TOKENS, 3072, device=dev, generator=g).bfloat16()
        for kind in kinds:
            cache = pkg.KVCacheB200.uniform(B, 1, 31, kind, device=dev)
            cache.store(past, layer=0)
            ms = timeit(lambda: pkg.attn_temporal(new, batch=B, q_frames=1, q_pos0=31, n_past=31,
                                                  n_kv=32, cache=cache, layer=0, out=o))
            byts = cache.nbytes + B * TOKENS * 1024 * 2 * 4  # + live q, k, v read + o written
            out.append({"case": f"decode past=31 B={B} kv={kind}", "ms": ms, "GBps": byts / ms / 1e6,
                        "frac_hbm": byts / ms / 1e6 / hbm})
            del cache
        del new, o, past
    torch.cuda.empty_cache()
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
    if args.isolated == "vae":
        # the latent decoder (12 blocks, random init) on `--batch` frames, eager launches
        dec = pkg.OasisVAEDecoderB200.random(seed=0, depth=12, device=dev)
        F = args.batch
        z = torch.randn(F, 576, 16, device=dev, generator=g)
        o = torch.empty(F, 3, 360, 640, device=dev)
        ms = timeit(lambda: dec.decode(z, out=o), args.steps)
        print(json.dumps({"case": f"vae decode frames={F}", "ms": ms, "frames_per_s": F / (ms / 1e3)}), flush=True)
        return 0
    if args.isolated == "cached":
        # prefill of a B-session window into a cache of one kind, then `steps` incremental
        # forwards of the newest frame over the 31 cached frames (eager launches)
        B = args.batch
        model = pkg.OasisDiTB200.random(seed=0, depth=DEPTH, device=dev)
        gh = torch.Generator().manual_seed(0)
        x = torch.randn(B, WINDOW, *FRAME, generator=gh).to(dev)
        t = torch.full((B, WINDOW), STAB_LEVEL - 1, dtype=torch.long, device=dev)
        a = synthetic_actions(gh, B, WINDOW).to(dev)
        kinds = (["int4"] * 23 + ["bf16"] * 8) if args.kv == "progressive" else [args.kv] * (WINDOW - 1)
        cache = pkg.KVCacheB200(B, DEPTH, kinds, device=dev)
        model(x, t, a, kv_cache=cache)
        xn, an = x[:, -1].contiguous(), a[:, -1].contiguous()
        tn = torch.full((B,), 599, dtype=torch.long, device=dev)
        vout = torch.empty(B, *FRAME, device=dev)
        ms = timeit(lambda: model.forward_cached(xn, tn, an, cache, n_past=WINDOW - 1, out=vout), args.steps)
        print(json.dumps({"case": f"cached forward B={B} kv={args.kv} past=31", "ms": ms,
                          "forwards_per_s": B / (ms / 1e3), "launch": "eager"}), flush=True)
        return 0
    for line in attention_sweep(pkg, dev, hbm, reps=args.steps, only=args.case):
        print(json.dumps(line), flush=True)
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
    ap.add_argument("--skip-sweep", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--isolated", choices=["attention", "gemm", "cached", "vae"], default=None)
    ap.add_argument("--case", default=None, help="--isolated attention: cases whose name contains this")
    ap.add_argument("--batch", type=int, default=8, help="--isolated cached: sessions; --isolated vae: frames")
    ap.add_argument("--kv", default="fp8", choices=["bf16", "fp8", "int4", "progressive"],
                    help="--isolated cached: cache kind (progressive: 23 INT4 + 8 bf16 frames)")
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
