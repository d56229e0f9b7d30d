"""``OasisDiTB200`` — the drop-in for the open-oasis ``dit(x, t, external_cond)`` call.

The worldserve sampler calls the DiT as ``v = dit(x_in, t_in, actions)``
(``worldserve/models/oasis.py:216``, ``benchmarks/optimised/oasis_dpmpp_modal.py:141``)
with ``x`` (B, T, 16, 18, 32), ``t`` (B, T) int64 and actions (B, T, 25), and gets
``v`` with the shape of ``x``.  This module keeps that signature and runs the whole
forward through the C ABI (one ``oasis_dit_forward`` call per forward; the native
runtime launches every kernel).  Host tensors are accepted and copied in/out, which is
the end-to-end path; device tensors avoid the copies.
"""

from __future__ import annotations

import ctypes
from typing import Dict, Optional, Tuple

import torch

from . import _native as N
from .weights import DEPTH, DeviceWeights, pack_weights, random_state_dict

LATENT = (16, 18, 32)
FRAME_ELEMS = 16 * 18 * 32


def _stream_ptr(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class _Plan:
    """One native forward plan (fixed batch x frames) and its workspace."""

    def __init__(self, weights: DeviceWeights, batch: int, frames: int, device):
        self.batch, self.frames = batch, frames
        L = N.lib()
        nbytes = L.oasis_plan_workspace_size(batch, frames, weights.depth)
        if nbytes == 0:
            raise N.OasisError(1, "bad plan shape")
        self.workspace = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
        base = (self.workspace.data_ptr() + 255) & ~255
        handle = ctypes.c_void_p()
        N.check(L.oasis_plan_create(ctypes.byref(weights.struct), batch, frames,
                                    ctypes.c_void_p(base), nbytes, ctypes.byref(handle)))
        self.handle = handle
        self.weights = weights  # keep alive

    def __del__(self):
        try:
            if getattr(self, "handle", None) and self.handle.value:
                N.lib().oasis_plan_destroy(self.handle)
                self.handle = ctypes.c_void_p()
        except Exception:
            pass


class OasisDiTB200:
    """B200-native Oasis-500M DiT (bf16 tensor-core projections, fp32 residual stream).

    ``model = OasisDiTB200.from_state_dict(sd)`` or ``OasisDiTB200.random(seed)``;
    ``v = model(x, t, external_cond)``.
    """

    max_frames = N.MAX_FRAMES

    def __init__(self, weights: DeviceWeights, device="cuda"):
        if not torch.cuda.is_available():
            raise RuntimeError("OasisDiTB200 needs a CUDA device (B200, sm_100a); there is no CPU path")
        N.lib()  # fail loudly if the native library is missing
        self.weights = weights
        self.device = torch.device(device)
        self.depth = weights.depth
        self._plans: Dict[Tuple[int, int], _Plan] = {}
        self.kv_manager = None  # set by KVCacheManagerB200.wire_to_model

    # -- construction ----------------------------------------------------------
    @classmethod
    def from_state_dict(cls, sd, device="cuda", depth: Optional[int] = None) -> "OasisDiTB200":
        return cls(pack_weights(sd, device=device, depth=depth), device=device)

    @classmethod
    def random(cls, seed: int = 0, depth: int = DEPTH, device="cuda") -> "OasisDiTB200":
        return cls.from_state_dict(random_state_dict(seed, depth), device=device, depth=depth)

    def plan(self, batch: int, frames: int) -> _Plan:
        key = (batch, frames)
        p = self._plans.get(key)
        if p is None:
            p = _Plan(self.weights, batch, frames, self.device)
            self._plans[key] = p
        return p

    # -- helpers ---------------------------------------------------------------
    def _to_dev(self, t: torch.Tensor, dtype) -> torch.Tensor:
        t = t.to(device=self.device, dtype=dtype, non_blocking=True)
        return t.contiguous()

    # -- forwards --------------------------------------------------------------
    @torch.no_grad()
    def forward(self, x: torch.Tensor, t: torch.Tensor, external_cond: Optional[torch.Tensor] = None,
                kv_cache=None, out: Optional[torch.Tensor] = None,
                stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Full-window forward.  ``kv_cache`` (a :class:`KVCacheB200`) additionally
        receives the post-RoPE temporal K/V of frames 0..T-2 (prefill); without one, a
        wired KV manager (``KVCacheManagerB200.wire_to_model``) supplies its prefill cache."""
        if x.dim() != 5 or tuple(x.shape[2:]) != LATENT:
            raise ValueError(f"x must be (B, T, 16, 18, 32), got {tuple(x.shape)}")
        B, T = x.shape[:2]
        if t.shape != (B, T):
            raise ValueError(f"t must be (B, T) = {(B, T)}, got {tuple(t.shape)}")
        host_out = not x.is_cuda
        xd = self._to_dev(x, torch.float32)
        td = self._to_dev(t, torch.int64)
        ad = None
        if external_cond is not None:
            if tuple(external_cond.shape) != (B, T, 25):
                raise ValueError("external_cond must be (B, T, 25)")
            ad = self._to_dev(external_cond, torch.float32)
        v = out if out is not None else torch.empty((B, T) + LATENT, device=self.device, dtype=torch.float32)
        p = self.plan(B, T)
        if kv_cache is None and self.kv_manager is not None and T > 1:
            kv_cache = self.kv_manager.cache_for_window(T - 1)
        cache = ctypes.byref(kv_cache.struct) if kv_cache is not None else None
        N.call("oasis_dit_forward", p.handle, xd.data_ptr(), td.data_ptr(),
               ad.data_ptr() if ad is not None else None, v.data_ptr(), cache, _stream_ptr(stream))
        if host_out and out is None:
            return v.to("cpu", non_blocking=False)
        return v

    __call__ = forward

    @torch.no_grad()
    def forward_cached(self, x_new: torch.Tensor, t_new: torch.Tensor, a_new: Optional[torch.Tensor],
                       kv_cache, n_past: int, out: Optional[torch.Tensor] = None,
                       stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Incremental forward of the newest frame of each session: x_new (B, 16, 18, 32),
        t_new (B,), a_new (B, 25); temporal attention reads cache slots 0..n_past-1."""
        B = x_new.shape[0]
        xd = self._to_dev(x_new.reshape(B, 1, *LATENT), torch.float32)
        td = self._to_dev(t_new.reshape(B, 1), torch.int64)
        ad = self._to_dev(a_new.reshape(B, 1, 25), torch.float32) if a_new is not None else None
        v = out if out is not None else torch.empty((B,) + LATENT, device=self.device, dtype=torch.float32)
        p = self.plan(B, 1)
        N.call("oasis_dit_forward_cached", p.handle, xd.data_ptr(), td.data_ptr(),
               ad.data_ptr() if ad is not None else None, v.data_ptr(),
               ctypes.byref(kv_cache.struct), int(n_past), _stream_ptr(stream))
        return v

    # -- profiling -------------------------------------------------------------
    FAMILIES = ("gemm", "adaln_gemm", "spatial_attn", "temporal_attn", "ln_modulate",
                "embed_final", "kv_store")

    def set_timing(self, batch: int, frames: int, enable: bool) -> None:
        N.call("oasis_plan_set_timing", self.plan(batch, frames).handle, int(enable))

    def get_timing(self, batch: int, frames: int) -> Dict[str, Tuple[float, int]]:
        n = len(self.FAMILIES)
        ms = (ctypes.c_float * n)()
        cnt = (ctypes.c_int * n)()
        N.call("oasis_plan_get_timing", self.plan(batch, frames).handle, ms, cnt, n)
        return {f: (ms[i], cnt[i]) for i, f in enumerate(self.FAMILIES)}
