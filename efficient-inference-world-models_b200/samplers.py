"""Sampler latent updates on the GPU, behind the worldserve sampler APIs.

* :func:`dpmpp2m_update` / :func:`ddim_update` — the v-prediction updates of the
  Oasis loops (``benchmarks/optimised/oasis_dpmpp_modal.py:143-164``,
  ``worldserve/models/oasis.py:218-228``) as one elementwise kernel over the newest
  frame of every session.
* :class:`DPMSolverPPSampler` — same constructor / ``step`` / ``reset`` /
  ``pre_step`` / ``post_step`` / ``wrap_oasis_loop`` as
  ``optimizations/model_level/samplers/dpm_solver_pp.py:31-187``, with the Euler / AB2 /
  AB3 combination done by ``oasis_ab_update``.
"""

from __future__ import annotations

import math
from collections import deque
from typing import Callable, Optional

import torch

from . import _native as N

FRAME_ELEMS = 16 * 18 * 32


def _stream_ptr(stream=None) -> int:
    return (stream or torch.cuda.current_stream()).cuda_stream


def _check_f32(*ts):
    for t in ts:
        if t is not None and (t.dtype != torch.float32 or not t.is_cuda):
            raise ValueError("sampler tensors must be fp32 CUDA tensors")


def dpmpp2m_update(x: torch.Tensor, v: torch.Tensor, eps_prev: Optional[torch.Tensor],
                   ab_t: float, ab_next: float, first: bool, stream=None) -> None:
    """In-place DPM-Solver++ 2M v-step on the NEWEST frame of x (B, T, 16, 18, 32) from
    v (B, T', 16, 18, 32) (its newest frame is used); ``eps_prev`` (B, 16*18*32) is
    read unless ``first`` and always overwritten with this step's eps."""
    _check_f32(x, v, eps_prev)
    B, T = x.shape[:2]
    Tv = v.shape[1] if v.dim() == 5 else 1
    if not (x.is_contiguous() and v.is_contiguous()):
        raise ValueError("x and v must be contiguous")
    xl = x[:, -1]
    vl = v[:, -1] if v.dim() == 5 else v
    N.call("oasis_dpmpp2m_update", xl.data_ptr(), vl.data_ptr(),
           eps_prev.data_ptr() if eps_prev is not None else None, B, FRAME_ELEMS,
           T * FRAME_ELEMS, Tv * FRAME_ELEMS, float(ab_t), float(ab_next), int(first),
           _stream_ptr(stream))


def ddim_update(x: torch.Tensor, v: torch.Tensor, ab_t: float, ab_prev: float, stream=None) -> None:
    """In-place DDIM v-step of the newest frame of x (the reference's chunk update)."""
    dpmpp2m_update(x, v, None, ab_t, ab_prev, True, stream)


class DPMSolverPPSampler:
    """Multi-step sampler with the reference API; the update runs on the GPU."""

    _COEF = {1: (1.0, 0.0, 0.0), 2: (1.5, -0.5, 0.0), 3: (23.0 / 12.0, -4.0 / 3.0, 5.0 / 12.0)}

    def __init__(self, order: int = 2) -> None:
        if order not in (1, 2, 3):
            raise ValueError(f"order must be 1, 2, or 3; got {order}")
        self.order = order
        self._history: deque = deque(maxlen=max(1, order - 1))

    def pre_step(self, step_idx: int, total_steps: int, latents) -> bool:
        return False

    def post_step(self, step_idx: int, total_steps: int, latents) -> None:
        return

    def reset(self) -> None:
        self._history.clear()

    def step(self, latents: torch.Tensor, noise_pred: torch.Tensor, t_start, t_end) -> torch.Tensor:
        h = float(t_end) - float(t_start)
        hist = list(self._history)
        n_hist = len(hist)
        if self.order == 1 or n_hist == 0:
            c, d1, d2 = self._COEF[1], None, None
        elif self.order == 2 or n_hist == 1:
            c, d1, d2 = self._COEF[2], hist[-1], None
        else:
            c, d1, d2 = self._COEF[3], hist[-1], hist[-2]
        x = latents.contiguous().float()
        d0 = noise_pred.contiguous().float()
        _check_f32(x, d0)
        out = torch.empty_like(x)
        N.call("oasis_ab_update", x.data_ptr(), d0.data_ptr(),
               d1.data_ptr() if d1 is not None else None, d2.data_ptr() if d2 is not None else None,
               out.data_ptr(), x.numel(), h, c[0], c[1], c[2], _stream_ptr())
        self._history.append(d0.detach().clone())
        return out if latents.dtype == torch.float32 else out.to(latents.dtype)

    def wrap_oasis_loop(self, dit_fn: Callable, latents: torch.Tensor, timesteps: torch.Tensor):
        self.reset()
        for i in range(len(timesteps) - 1):
            t_start, t_end = timesteps[i], timesteps[i + 1]
            t_batch = t_start.expand(latents.shape[0], latents.shape[1])
            latents = self.step(latents, dit_fn(latents, t_batch), t_start, t_end)
        return latents


def euler_sampler() -> DPMSolverPPSampler:
    return DPMSolverPPSampler(order=1)


def dpm_solver_pp_2() -> DPMSolverPPSampler:
    return DPMSolverPPSampler(order=2)


def dpm_solver_pp_3() -> DPMSolverPPSampler:
    return DPMSolverPPSampler(order=3)
