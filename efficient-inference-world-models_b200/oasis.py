"""Oasis autoregressive samplers on the B200 DiT (mirrors ``worldserve/models/oasis.py``
and the DPM-Solver++ 2M loop of ``benchmarks/optimised/oasis_dpmpp_modal.py``).

Semantics kept from the reference:
* sigmoid beta schedule over 1000 steps; ``noise_range = linspace(-1, 999, steps+1)``
  (``models/oasis.py:88-110``);
* DDIM-v update of the new frame only, past frames at t=0 (``models/oasis.py:174-235``);
* DPM++ 2M: context frames at ``stabilization_level - 1``, sliding window of
  ``max_frames`` (32), new chunk ~ N(0, 1) clamped to +-20, eps_prev reset per frame,
  only ``x[:, -1:]`` written back (``oasis_dpmpp_modal.py:118-164``).

``action_step_schedule`` is the action-magnitude difficulty schedule
(``benchmarks/optimised/oasis_difficulty_dpmpp_modal.py:93-101``): a frame whose action
L1 norm is below 0.5 gets 2 solver steps, below 1.5 gets 3, otherwise 5; rollout_dpmpp
accepts the per-frame list as ``solver_steps``.

``rollout_dpmpp(..., use_cache=True)`` runs the first solver step of each frame as a
full-window forward that also stores the window's temporal K/V, and the remaining steps
as incremental forwards of the new frame against that cache (the reference's
persistent past-frame reuse, ``kv_cache/oasis_temporal_persistent_wrapper.py``).
``rollout_dpmpp(..., use_graph=True)`` captures each frame's whole solver loop (its
forwards and latent updates) as one CUDA graph per (window length, step count) and
replays it for every later frame of the same shape.
The VAE decode (``models/oasis.py:237-245``) is outside this library.
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence, Union

import torch

from .kv_cache import KVCacheB200


def _window_cache(B: int, depth: int, n_past: int, kv_kinds, device) -> KVCacheB200:
    """Cache for the past frames of a window: ``kv_kinds(n_past)`` gives the slot kinds
    (one list for keys and values, or a ``(key kinds, value kinds)`` pair such as
    ``ProgressiveKVQuantizerB200.slot_kinds`` returns); bf16 when None."""
    kinds = kv_kinds(n_past) if kv_kinds is not None else ["bf16"] * n_past
    if isinstance(kinds, tuple):
        return KVCacheB200(B, depth, kinds[0], device=device, value_kinds=kinds[1])
    return KVCacheB200(B, depth, kinds, device=device)
from . import _native as N
from .samplers import FRAME_ELEMS, _stream_ptr, ddim_update

LATENT_C, LATENT_H, LATENT_W = 16, 18, 32
ACTION_DIM = 25
DDPM_T = 1000
DEFAULT_DDIM_STEPS = 10
N_PROMPT = 1
VAE_SCALE = 0.07843137255


def sigmoid_beta_schedule(timesteps: int = DDPM_T, start: float = -3.0, end: float = 3.0,
                          tau: float = 1.0) -> torch.Tensor:
    """Sigmoid schedule (Jabri et al. 2022, arXiv:2212.11972), float64, clipped to [0, 0.999]."""
    t = torch.linspace(0, timesteps, timesteps + 1, dtype=torch.float64) / timesteps
    v_start = torch.tensor(start / tau, dtype=torch.float64).sigmoid()
    v_end = torch.tensor(end / tau, dtype=torch.float64).sigmoid()
    ac = (-((t * (end - start) + start) / tau).sigmoid() + v_end) / (v_end - v_start)
    ac = ac / ac[0]
    return torch.clip(1 - ac[1:] / ac[:-1], 0, 0.999)


def alphas_cumprod(timesteps: int = DDPM_T) -> torch.Tensor:
    betas = sigmoid_beta_schedule(timesteps).float()
    return torch.cumprod(1.0 - betas, dim=0)


def _build_schedule(ddim_steps: int, alpha_bar_override: Optional[torch.Tensor] = None):
    ab = alpha_bar_override.float().cpu() if alpha_bar_override is not None else alphas_cumprod()
    noise_range = torch.linspace(-1, DDPM_T - 1, ddim_steps + 1)
    return ab, noise_range


@torch.no_grad()
def generate(model: Dict[str, Any], num_frames: int = 16, num_steps: int = DEFAULT_DDIM_STEPS,
             n_prompt: int = N_PROMPT, seed: int = 42, optimizations: Any = None) -> Dict[str, Any]:
    """DDIM-v autoregressive generation with ``model["dit"]`` (an ``OasisDiTB200``).

    Returns the latents (B, n_prompt + num_frames, 16, 18, 32); frames are decoded only
    if ``model`` carries a ``vae`` with ``decode``."""
    dit = model["dit"]
    device = model.get("device", "cuda")
    gen = torch.Generator(device=device).manual_seed(seed)
    B = 1
    total = n_prompt + num_frames
    ab, nr = _build_schedule(num_steps, model.get("alpha_bar_override"))
    x = torch.randn(B, n_prompt, LATENT_C, LATENT_H, LATENT_W, device=device, generator=gen)
    actions = torch.zeros(B, total, ACTION_DIM, device=device)
    step = 0
    for frame_i in range(n_prompt, total):
        chunk = torch.randn(B, 1, LATENT_C, LATENT_H, LATENT_W, device=device, generator=gen)
        x = torch.cat([x, chunk], dim=1)
        for noise_idx in reversed(range(1, num_steps + 1)):
            t_val = int(nr[noise_idx].long().clamp(0, DDPM_T - 1))
            t_in = torch.zeros(B, frame_i + 1, dtype=torch.long, device=device)
            t_in[:, -1] = t_val
            if optimizations is not None and optimizations.pre_step(step, num_frames * num_steps, x[:, -1:]):
                step += 1
                continue
            v = dit(x[:, -dit.max_frames:] if x.shape[1] > dit.max_frames else x,
                    t_in[:, -dit.max_frames:], actions[:, max(0, frame_i + 1 - dit.max_frames): frame_i + 1])
            t_prev = max(int(nr[noise_idx - 1]), 0)
            ddim_update(x, v, float(ab[t_val]), float(ab[t_prev]))
            if optimizations is not None:
                optimizations.post_step(step, num_frames * num_steps, x[:, -1:])
            step += 1
    out = {"latents": x, "num_frames": num_frames, "num_steps": num_steps, "n_prompt": n_prompt,
           "total_dit_fwd_passes": num_frames * num_steps}
    vae = model.get("vae")
    if vae is not None and hasattr(vae, "decode"):
        Bx, Tx = x.shape[:2]
        z = (x / VAE_SCALE).reshape(Bx * Tx, LATENT_C, LATENT_H * LATENT_W).permute(0, 2, 1)
        out["frames"] = vae.decode(z)
    return out


def steps_for_action_magnitude(mag: float, lo_threshold: float = 0.5, hi_threshold: float = 1.5,
                                reduced_steps: int = 2, mid_steps: int = 3, full_steps: int = 5) -> int:
    """Solver steps for one frame from its action L1 norm (the reference's bucket
    function, ``oasis_difficulty_dpmpp_modal.py:95-101``)."""
    if mag < lo_threshold:
        return reduced_steps
    if mag < hi_threshold:
        return mid_steps
    return full_steps


def action_step_schedule(actions: torch.Tensor, **thresholds) -> List[int]:
    """Per-frame solver steps for a rollout: the action magnitudes of the first session
    (``actions[0].abs().sum(-1)``, as the reference computes them) through
    ``steps_for_action_magnitude``.  actions (B, frames, 25)."""
    mags = actions[0].abs().sum(dim=-1).float().cpu().tolist()
    return [steps_for_action_magnitude(m, **thresholds) for m in mags]


@torch.no_grad()
def _solver_levels(steps: int, ab: torch.Tensor):
    """(t, alpha_bar(t), alpha_bar(next)) of each solver step of a frame, in order
    (``noise_range = linspace(-1, 999, steps + 1)`` walked backwards; the last step
    lands on alpha_bar = 1)."""
    nr = torch.linspace(-1, DDPM_T - 1, steps + 1)
    out = []
    for noise_idx in reversed(range(1, steps + 1)):
        t = int(nr[noise_idx])
        tn = int(nr[noise_idx - 1])
        tn = t if tn < 0 else tn
        out.append((t, float(ab[t]), 1.0 if noise_idx == 1 else float(ab[tn])))
    return out


class _FrameGraph:
    """One frame's solver loop for a window of T frames (B sessions, ``steps`` solver
    steps) as a CUDA graph over static buffers: the window latents and actions are copied
    in before a replay and the new frame is copied out after it.  The first call runs the
    loop eagerly (creating the forward plans and KV cache outside any capture); the
    second captures it, and every call from then on replays."""

    def __init__(self, dit, B: int, T: int, steps: int, ab: torch.Tensor, stabilization_level: int,
                 use_cache: bool, kv_kinds, device):
        self.dit, self.T = dit, T
        self.xw = torch.empty(B, T, LATENT_C, LATENT_H, LATENT_W, device=device)
        self.aw = torch.zeros(B, T, ACTION_DIM, device=device)
        self.eps = torch.empty(B, FRAME_ELEMS, device=device)
        self.v = torch.empty(B, T, LATENT_C, LATENT_H, LATENT_W, device=device)
        self.v1 = torch.empty(B, LATENT_C, LATENT_H, LATENT_W, device=device)
        self.cache = None
        if use_cache and T > 1:
            self.cache = _window_cache(B, dit.depth, T - 1, kv_kinds, device)
        self.levels = []
        for t, ab_t, ab_next in _solver_levels(steps, ab):
            tw = torch.full((B, T), stabilization_level - 1, dtype=torch.long, device=device)
            tw[:, -1] = t
            self.levels.append((tw, tw[:, -1].contiguous(), ab_t, ab_next))
        self.graph = None
        self.calls = 0

    def _body(self) -> None:
        T = self.T
        for k, (tw, t_new, ab_t, ab_next) in enumerate(self.levels):
            if self.cache is not None and k > 0:
                v = self.dit.forward_cached(self.xw[:, -1], t_new, self.aw[:, -1], self.cache,
                                            n_past=T - 1, out=self.v1)
            else:
                v = self.dit(self.xw, tw, self.aw, kv_cache=self.cache, out=self.v)
            _update_newest(self.xw, T - 1, v, self.eps, ab_t, ab_next, k == 0)

    def run(self, x: torch.Tensor, actions: torch.Tensor, start: int, i: int) -> None:
        self.xw.copy_(x[:, start: i + 1])
        self.aw.copy_(actions[:, start: i + 1])
        if self.calls == 0:
            self._body()
        else:
            if self.graph is None:
                side = torch.cuda.Stream(device=self.xw.device)
                side.wait_stream(torch.cuda.current_stream())
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.stream(side):
                    with torch.cuda.graph(graph, stream=side):
                        self._body()  # recorded, not run
                torch.cuda.current_stream().wait_stream(side)
                self.graph = graph
            self.graph.replay()
        self.calls += 1
        x[:, i].copy_(self.xw[:, -1])


def rollout_dpmpp(dit, prompt_latent: torch.Tensor, actions: torch.Tensor, num_frames: int,
                  solver_steps: Union[int, Sequence[int]] = 5, stabilization_level: int = 15,
                  noise_abs_max: float = 20.0,
                  seed: int = 42, use_cache: bool = False, kv_kinds=None,
                  alpha_bar: Optional[torch.Tensor] = None, step_callback=None,
                  use_graph: bool = False) -> torch.Tensor:
    """DPM-Solver++ 2M rollout of ``num_frames`` new frames for B sessions.

    prompt_latent (B, n_prompt, 16, 18, 32) on the device; actions (B, n_prompt +
    num_frames, 25).  ``solver_steps`` is one count for every frame or a per-frame list
    indexed by absolute frame (e.g. ``action_step_schedule(actions)``).  With
    ``use_graph`` each frame's solver loop is a replayed CUDA graph (no per-step
    ``step_callback`` then).  Returns all latents (B, n_prompt + num_frames, 16, 18, 32)."""
    if use_graph and step_callback is not None:
        raise ValueError("step_callback runs between solver steps; it cannot be used with use_graph")
    device = prompt_latent.device
    ab = (alpha_bar if alpha_bar is not None else alphas_cumprod()).float().cpu()
    max_frames = dit.max_frames
    B, n_prompt = prompt_latent.shape[:2]
    total = n_prompt + num_frames
    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.empty(B, total, LATENT_C, LATENT_H, LATENT_W, device=device)
    x[:, :n_prompt] = prompt_latent
    eps_prev = torch.empty(B, LATENT_C * LATENT_H * LATENT_W, device=device)
    cache = None
    graphs: Dict[Any, _FrameGraph] = {}
    for i in range(n_prompt, total):
        chunk = torch.randn((B, LATENT_C, LATENT_H, LATENT_W), device=device, generator=gen)
        x[:, i] = chunk.clamp(-noise_abs_max, noise_abs_max)
        start = max(0, i + 1 - max_frames)
        T = i + 1 - start
        steps_i = int(solver_steps) if isinstance(solver_steps, int) else int(solver_steps[i])
        if use_graph:
            if any(key[0] != T for key in graphs):  # the window grew: shorter shapes never recur
                graphs = {key: g for key, g in graphs.items() if key[0] == T}
            fg = graphs.get((T, steps_i))
            if fg is None:
                fg = graphs[(T, steps_i)] = _FrameGraph(dit, B, T, steps_i, ab, stabilization_level,
                                                        use_cache, kv_kinds, device)
            fg.run(x, actions, start, i)
            continue
        window = x[:, start: i + 1]
        act = actions[:, start: i + 1].contiguous()
        t_win = torch.full((B, T), stabilization_level - 1, dtype=torch.long, device=device)
        if use_cache and T > 1 and (cache is None or cache.n_slots != T - 1):
            cache = _window_cache(B, dit.depth, T - 1, kv_kinds, device)
        for k, (t, ab_t, ab_next) in enumerate(_solver_levels(steps_i, ab)):
            t_win[:, -1] = t
            if use_cache and T > 1 and k > 0:
                v = dit.forward_cached(x[:, i], t_win[:, -1], act[:, -1], cache, n_past=T - 1)
            else:
                v = dit(window.contiguous(), t_win, act,
                        kv_cache=cache if (use_cache and T > 1) else None)
            _update_newest(x, i, v, eps_prev, ab_t, ab_next, k == 0)
            if step_callback is not None:
                step_callback(i, k)
    return x


def _update_newest(x, i, v, eps_prev, ab_t, ab_next, first):
    """DPM++ 2M update of frame ``i`` of x in place (v: newest-frame prediction)."""
    B, total = x.shape[:2]
    vl = v[:, -1] if v.dim() == 5 else v
    v_stride = (v.shape[1] if v.dim() == 5 else 1) * FRAME_ELEMS
    N.call("oasis_dpmpp2m_update", x[:, i].data_ptr(), vl.data_ptr(), eps_prev.data_ptr(), B,
           FRAME_ELEMS, total * FRAME_ELEMS, v_stride, float(ab_t), float(ab_next), int(first),
           _stream_ptr())
