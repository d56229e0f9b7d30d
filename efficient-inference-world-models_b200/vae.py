"""Latent decoder of the Oasis rollout: ``vae.decode(z)`` (worldserve/models/oasis.py:237-245).

``decoder = OasisVAEDecoderB200.from_state_dict(sd)``; ``rgb = decoder.decode(z)`` with z
(frames, 576, 16) latents already divided by the VAE scale, rgb (frames, 3, 360, 640) fp32
in [-1, 1] (the reference maps it with ``(rgb + 1) / 2``).  The decoder is a ViT of width
1024 over the 18 x 32 latent grid with patch 20; its structure and parameter names are
the ones ``include/oasis_b200.h`` documents for ``oasis_vae_weights_t`` (upstream
open-oasis ``vae.py`` is not in the reference tree).  All compute runs in
``liboasis_b200.so`` (``oasis_vae_decode``).
"""

from __future__ import annotations

import ctypes
import math
from typing import Dict, List

import torch

from . import _native as N

DIM = 1024
MLP_HIDDEN = 4096
LATENT = 16
DEPTH = 12
TOKENS = 576
GRID_H, GRID_W = 18, 32
PATCH = 20
PATCH_DIM = PATCH * PATCH * 3  # 1200
IMG_H, IMG_W = 360, 640


def vae_param_shapes(depth: int = DEPTH) -> Dict[str, tuple]:
    shapes = {"post_quant_conv.weight": (DIM, LATENT), "post_quant_conv.bias": (DIM,)}
    for i in range(depth):
        p = f"decoder.{i}."
        shapes.update({
            p + "norm1.weight": (DIM,), p + "norm1.bias": (DIM,), p + "attn.qkv.weight": (3 * DIM, DIM),
            p + "attn.proj.weight": (DIM, DIM), p + "attn.proj.bias": (DIM,),
            p + "norm2.weight": (DIM,), p + "norm2.bias": (DIM,),
            p + "mlp.fc1.weight": (MLP_HIDDEN, DIM), p + "mlp.fc1.bias": (MLP_HIDDEN,),
            p + "mlp.fc2.weight": (DIM, MLP_HIDDEN), p + "mlp.fc2.bias": (DIM,),
        })
    shapes.update({"dec_norm.weight": (DIM,), "dec_norm.bias": (DIM,),
                   "predictor.weight": (PATCH_DIM, DIM), "predictor.bias": (PATCH_DIM,)})
    return shapes


def random_vae_state_dict(seed: int = 0, depth: int = DEPTH) -> Dict[str, torch.Tensor]:
    """Seeded fp32 CPU init: scaled normal weights, small biases, LayerNorm weights near 1."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape in vae_param_shapes(depth).items():
        if "norm" in name:
            t = torch.randn(shape, generator=g) * 0.1 + (1.0 if name.endswith("weight") else 0.0)
        elif name.endswith("bias"):
            t = torch.randn(shape, generator=g) * 0.02
        else:
            t = torch.randn(shape, generator=g) * math.sqrt(2.0 / (shape[0] + shape[1]))
        out[name] = t
    return out


def vae_rope_table() -> torch.Tensor:
    """[576][32][2] fp32 (cos, sin): 16 frequencies ``linspace(1, 128, 16) * pi`` per axis
    over ``linspace(-1, 1, n)`` positions; pairs 0..15 take the H angle, 16..31 the W angle."""
    f = torch.linspace(1.0, 128.0, 16) * math.pi
    ah = torch.linspace(-1, 1, GRID_H)[:, None] * f
    aw = torch.linspace(-1, 1, GRID_W)[:, None] * f
    ang = torch.cat([ah[:, None, :].expand(GRID_H, GRID_W, 16),
                     aw[None, :, :].expand(GRID_H, GRID_W, 16)], dim=-1).reshape(TOKENS, 32)
    return torch.stack([ang.cos(), ang.sin()], dim=-1).contiguous()


class _VaeDeviceWeights:
    def __init__(self, sd: Dict[str, torch.Tensor], device, depth: int):
        dev = torch.device(device)
        self.keep: List[torch.Tensor] = []

        def f32(t):
            t = t.detach().to(dev, torch.float32).contiguous()
            self.keep.append(t)
            return t.data_ptr()

        def bf16(t):
            t = t.detach().to(dev, torch.bfloat16).contiguous()
            self.keep.append(t)
            return t.data_ptr()

        w = N.VaeWeights()
        w.depth = depth
        post = torch.zeros(DIM, 64)
        post[:, :LATENT] = sd["post_quant_conv.weight"].float()
        w.post_w = bf16(post)
        w.post_b = f32(sd["post_quant_conv.bias"])
        for i in range(depth):
            p = f"decoder.{i}."
            b = w.blk[i]
            # affine LayerNorm as (1 + scale) * x_hat + shift
            b.ln1_shift = f32(sd[p + "norm1.bias"])
            b.ln1_scale = f32(sd[p + "norm1.weight"].float() - 1.0)
            b.qkv_w = bf16(sd[p + "attn.qkv.weight"])
            b.proj_w = bf16(sd[p + "attn.proj.weight"])
            b.proj_b = f32(sd[p + "attn.proj.bias"])
            b.ln2_shift = f32(sd[p + "norm2.bias"])
            b.ln2_scale = f32(sd[p + "norm2.weight"].float() - 1.0)
            b.fc1_w = bf16(sd[p + "mlp.fc1.weight"])
            b.fc1_b = f32(sd[p + "mlp.fc1.bias"])
            b.fc2_w = bf16(sd[p + "mlp.fc2.weight"])
            b.fc2_b = f32(sd[p + "mlp.fc2.bias"])
        w.norm_shift = f32(sd["dec_norm.bias"])
        w.norm_scale = f32(sd["dec_norm.weight"].float() - 1.0)
        pred = torch.zeros(N.VAE_PRED_LD, DIM)
        pred[:PATCH_DIM] = sd["predictor.weight"].float()
        w.pred_w = bf16(pred)
        pred_b = torch.zeros(N.VAE_PRED_LD)
        pred_b[:PATCH_DIM] = sd["predictor.bias"].float()
        w.pred_b = f32(pred_b)
        w.rope = f32(vae_rope_table())
        w.ones = f32(torch.ones(DIM))
        self.struct = w
        self.depth = depth


class _VaePlan:
    def __init__(self, weights: _VaeDeviceWeights, frames: int, device):
        nbytes = N.lib().oasis_vae_workspace_size(frames, weights.depth)
        if nbytes == 0:
            raise ValueError(f"oasis_vae_workspace_size({frames}, {weights.depth}) rejected the shape")
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.handle = ctypes.c_void_p()
        N.call("oasis_vae_plan_create", ctypes.byref(weights.struct), frames, self.ws.data_ptr(), nbytes,
               ctypes.byref(self.handle))

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                N.lib().oasis_vae_plan_destroy(h)
            except Exception:
                pass


class OasisVAEDecoderB200:
    """``decode(z)`` of the Oasis rollout on the B200: z (frames, 576, 16) -> (frames, 3, 360, 640)."""

    def __init__(self, sd: Dict[str, torch.Tensor], device="cuda", depth: int = None):
        if not torch.cuda.is_available():
            raise RuntimeError("OasisVAEDecoderB200 needs a CUDA device (B200, sm_100a); there is no CPU path")
        N.lib()
        if depth is None:
            depth = 1 + max(int(k.split(".")[1]) for k in sd if k.startswith("decoder."))
        if not 1 <= depth <= N.VAE_MAX_DEPTH:
            raise ValueError(f"depth {depth} outside 1..{N.VAE_MAX_DEPTH}")
        self.device = torch.device(device)
        self.weights = _VaeDeviceWeights(sd, self.device, depth)
        self.depth = depth
        self._plans: Dict[int, _VaePlan] = {}

    @classmethod
    def from_state_dict(cls, sd, device="cuda", depth: int = None) -> "OasisVAEDecoderB200":
        return cls(sd, device=device, depth=depth)

    @classmethod
    def random(cls, seed: int = 0, depth: int = DEPTH, device="cuda") -> "OasisVAEDecoderB200":
        return cls(random_vae_state_dict(seed, depth), device=device, depth=depth)

    def plan(self, frames: int) -> _VaePlan:
        p = self._plans.get(frames)
        if p is None:
            p = _VaePlan(self.weights, frames, self.device)
            self._plans[frames] = p
        return p

    def decode(self, z: torch.Tensor, out: torch.Tensor = None, stream=None) -> torch.Tensor:
        """z (frames, 576, 16) (host or device, any float dtype) -> fp32 (frames, 3, 360, 640)."""
        if z.dim() != 3 or z.shape[1:] != (TOKENS, LATENT):
            raise ValueError(f"z must be (frames, {TOKENS}, {LATENT}), got {tuple(z.shape)}")
        frames = z.shape[0]
        zd = z.to(device=self.device, dtype=torch.float32, non_blocking=True).contiguous()
        if out is None:
            out = torch.empty(frames, 3, IMG_H, IMG_W, device=self.device, dtype=torch.float32)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        N.call("oasis_vae_decode", self.plan(frames).handle, zd.data_ptr(), out.data_ptr(), s.cuda_stream)
        return out

    __call__ = decode
