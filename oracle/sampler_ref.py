"""numpy restatement of the Oasis samplers' latent updates — TEST INFRASTRUCTURE ONLY.

* ``ddim_vpred_step``   — ``worldserve/models/oasis.py:218-228``
  (x0 = sqrt(ab) x - sqrt(1-ab) v; eps = sqrt(1-ab) x + sqrt(ab) v;
  x' = sqrt(ab') x0 + sqrt(1-ab') eps).
* ``dpmpp2m_vpred_step`` — ``benchmarks/optimised/oasis_dpmpp_modal.py:143-164``
  (same x0/eps; D = eps on the first step of a frame, else (3 eps - eps_prev)/2;
  x' = sqrt(ab') x0 + sqrt(1-ab') D; eps_prev <- eps).
* ``ab_step``           — ``DPMSolverPPSampler.step``
  (``optimizations/model_level/samplers/dpm_solver_pp.py:111-141``): Euler / AB2 / AB3.
* ``sigmoid_beta_schedule`` — the published sigmoid schedule (Jabri et al. 2022,
  arXiv:2212.11972, fig. 8) that ``open-oasis/utils.py`` provides and the reference
  calls at ``models/oasis.py:102-106``: start -3, end 3, tau 1, clipped to [0, 0.999].
  Upstream is absent, so the schedule constants are unpinned.
"""

from __future__ import annotations

import numpy as np


def sigmoid_beta_schedule(timesteps: int = 1000, start: float = -3.0, end: float = 3.0,
                          tau: float = 1.0) -> np.ndarray:
    t = np.linspace(0, timesteps, timesteps + 1, dtype=np.float64) / timesteps
    sig = lambda z: 1.0 / (1.0 + np.exp(-z))
    v_start = sig(start / tau)
    v_end = sig(end / tau)
    ac = (-sig((t * (end - start) + start) / tau) + v_end) / (v_end - v_start)
    ac = ac / ac[0]
    betas = 1.0 - ac[1:] / ac[:-1]
    return np.clip(betas, 0.0, 0.999)


def alphas_cumprod(timesteps: int = 1000) -> np.ndarray:
    """Cumulative product of (1 - beta) as the reference computes it: ``betas.float()``,
    ``1 - betas`` in fp32, then ``torch.cumprod`` (whose CPU kernel accumulates in
    float64 and rounds each output to fp32)."""
    betas = sigmoid_beta_schedule(timesteps).astype(np.float32)
    alphas = (np.float32(1.0) - betas).astype(np.float32)
    return np.cumprod(alphas.astype(np.float64)).astype(np.float32)


def ddim_vpred_step(x, v, ab_t, ab_prev):
    x = np.asarray(x, np.float64)
    v = np.asarray(v, np.float64)
    x0 = np.sqrt(ab_t) * x - np.sqrt(1.0 - ab_t) * v
    eps = np.sqrt(1.0 - ab_t) * x + np.sqrt(ab_t) * v
    return np.sqrt(ab_prev) * x0 + np.sqrt(1.0 - ab_prev) * eps


def dpmpp2m_vpred_step(x, v, eps_prev, ab_t, ab_next, first: bool):
    x = np.asarray(x, np.float64)
    v = np.asarray(v, np.float64)
    x0 = np.sqrt(ab_t) * x - np.sqrt(1.0 - ab_t) * v
    eps = np.sqrt(1.0 - ab_t) * x + np.sqrt(ab_t) * v
    d = eps if first else (3.0 * eps - np.asarray(eps_prev, np.float64)) / 2.0
    return np.sqrt(ab_next) * x0 + np.sqrt(1.0 - ab_next) * d, eps


def ab_step(latents, d0, history, h: float, order: int):
    """One ``DPMSolverPPSampler.step``; ``history`` is oldest..newest past noise preds."""
    x = np.asarray(latents, np.float64)
    d0 = np.asarray(d0, np.float64)
    if order == 1 or len(history) == 0:
        return x + h * d0
    if order == 2 or len(history) == 1:
        return x + h * (1.5 * d0 - 0.5 * np.asarray(history[-1], np.float64))
    return x + h * ((23.0 / 12.0) * d0 - (4.0 / 3.0) * np.asarray(history[-1], np.float64)
                    + (5.0 / 12.0) * np.asarray(history[-2], np.float64))


def dpmpp_noise_levels(solver_steps: int, max_noise_level: int = 1000):
    """(t, t_next) integer pairs per step, as ``oasis_dpmpp_modal.py:105,126-133`` builds them:
    ``noise_range = linspace(-1, T-1, steps+1)``; ``t = int(noise_range[i])``,
    ``t_next = int(noise_range[i-1])`` with negative ``t_next`` replaced by ``t``."""
    nr = np.linspace(-1, max_noise_level - 1, solver_steps + 1, dtype=np.float32)
    out = []
    for idx in reversed(range(1, solver_steps + 1)):
        t = int(nr[idx])
        tn = int(nr[idx - 1])
        out.append((t, t if tn < 0 else tn, idx == 1))
    return out
