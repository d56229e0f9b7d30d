"""Oasis-500M weights: seeded random init (upstream parameter names) and the device pack.

Parameter names follow open-oasis ``DiT-S/2`` exactly (``blocks.{i}.s_attn.to_qkv.weight``
etc.), so a real ``oasis500m.safetensors`` state dict loads through the same
:func:`pack_weights` (the reference loads it with ``load_state_dict(strict=False)``,
``worldserve/models/oasis.py:74-77``).

The random init is deliberately NOT adaLN-Zero: open-oasis zero-initialises the
adaLN and final layers, which would make every gate 0 and any parity check vacuous.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List

import torch

from . import _native as N

HIDDEN, HEADS, HEAD_DIM, MLP_HIDDEN = 1024, 16, 64, 4096
PATCH, IN_CH, LAT_H, LAT_W = 2, 16, 18, 32
GRID_H, GRID_W = LAT_H // PATCH, LAT_W // PATCH
ACTION_DIM, FREQ_EMB = 25, 256
DEPTH = 16


def param_shapes(depth: int = DEPTH) -> Dict[str, tuple]:
    s = {
        "x_embedder.proj.weight": (HIDDEN, IN_CH, PATCH, PATCH),
        "x_embedder.proj.bias": (HIDDEN,),
        "t_embedder.mlp.0.weight": (HIDDEN, FREQ_EMB),
        "t_embedder.mlp.0.bias": (HIDDEN,),
        "t_embedder.mlp.2.weight": (HIDDEN, HIDDEN),
        "t_embedder.mlp.2.bias": (HIDDEN,),
        "external_cond.weight": (HIDDEN, ACTION_DIM),
        "external_cond.bias": (HIDDEN,),
        "final_layer.linear.weight": (PATCH * PATCH * IN_CH, HIDDEN),
        "final_layer.linear.bias": (PATCH * PATCH * IN_CH,),
        "final_layer.adaLN_modulation.1.weight": (2 * HIDDEN, HIDDEN),
        "final_layer.adaLN_modulation.1.bias": (2 * HIDDEN,),
    }
    for i in range(depth):
        for a in ("s", "t"):
            p = f"blocks.{i}.{a}_"
            s[p + "attn.to_qkv.weight"] = (3 * HIDDEN, HIDDEN)
            s[p + "attn.to_out.weight"] = (HIDDEN, HIDDEN)
            s[p + "attn.to_out.bias"] = (HIDDEN,)
            s[p + "mlp.fc1.weight"] = (MLP_HIDDEN, HIDDEN)
            s[p + "mlp.fc1.bias"] = (MLP_HIDDEN,)
            s[p + "mlp.fc2.weight"] = (HIDDEN, MLP_HIDDEN)
            s[p + "mlp.fc2.bias"] = (HIDDEN,)
            s[p + "adaLN_modulation.1.weight"] = (6 * HIDDEN, HIDDEN)
            s[p + "adaLN_modulation.1.bias"] = (6 * HIDDEN,)
    return s


def random_state_dict(seed: int = 0, depth: int = DEPTH) -> Dict[str, torch.Tensor]:
    """Seeded fp32 CPU init: xavier-uniform-scaled normal weights, small biases, and
    adaLN/final weights at std 0.02 so shift/scale/gate are O(0.1-1)."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape in param_shapes(depth).items():
        if name.endswith("bias"):
            std = 0.1 if "adaLN" in name else 0.02
            t = torch.randn(shape, generator=g) * std
        elif "adaLN" in name:
            t = torch.randn(shape, generator=g) * 0.02
        else:
            fan_out = shape[0]
            fan_in = int(math.prod(shape[1:]))
            t = torch.randn(shape, generator=g) * math.sqrt(2.0 / (fan_in + fan_out))
        out[name] = t
    return out


def rope_tables() -> tuple:
    """(spatial [144][32][2], temporal [32][32][2]) fp32 cos/sin tables.

    Spatial: 16 frequencies ``linspace(1, 128, 16) * pi`` per axis, positions
    ``linspace(-1, 1, 9)`` (H) and ``linspace(-1, 1, 16)`` (W); pairs 0..15 use the H
    angle, 16..31 the W angle.  Temporal: ``1 / 10000^(2k/64)`` at positions 0..31.
    Angles and cos/sin are computed in fp32 like the upstream rotary module.
    """
    sf = torch.linspace(1.0, 128.0, 16) * math.pi
    ah = torch.linspace(-1, 1, GRID_H)[:, None] * sf              # (9, 16)
    aw = torch.linspace(-1, 1, GRID_W)[:, None] * sf              # (16, 16)
    ang_s = torch.cat([ah[:, None, :].expand(GRID_H, GRID_W, 16),
                       aw[None, :, :].expand(GRID_H, GRID_W, 16)], dim=-1).reshape(GRID_H * GRID_W, 32)
    tf = 1.0 / (10000.0 ** (torch.arange(0, HEAD_DIM, 2).float() / HEAD_DIM))
    ang_t = torch.arange(N.MAX_FRAMES).float()[:, None] * tf      # (32, 32)
    sp = torch.stack([ang_s.cos(), ang_s.sin()], dim=-1).contiguous()
    tp = torch.stack([ang_t.cos(), ang_t.sin()], dim=-1).contiguous()
    return sp, tp


@dataclass
class DeviceWeights:
    """Weights resident in HBM in the layout ``oasis_dit_weights_t`` describes."""
    depth: int
    tensors: List[torch.Tensor] = field(default_factory=list)
    struct: N.DiTWeights = None

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors)


def pack_weights(sd: Dict[str, torch.Tensor], device="cuda", depth: int = None) -> DeviceWeights:
    """Upload a state dict (upstream names) as bf16 GEMM weights + fp32 small weights."""
    if depth is None:
        depth = 1 + max(int(k.split(".")[1]) for k in sd if k.startswith("blocks."))
    if not 1 <= depth <= N.MAX_DEPTH:
        raise ValueError(f"depth {depth} outside 1..{N.MAX_DEPTH}")
    dev = torch.device(device)
    keep: List[torch.Tensor] = []

    def f32(name, shape=None):
        t = sd[name].detach().to(dev, torch.float32).contiguous()
        if shape is not None:
            t = t.reshape(shape)
        keep.append(t)
        return t.data_ptr()

    def bf16(t):
        t = t.detach().to(dev, torch.bfloat16).contiguous()
        keep.append(t)
        return t.data_ptr()

    w = N.DiTWeights()
    w.depth = depth
    w.patch_w = bf16(sd["x_embedder.proj.weight"].reshape(HIDDEN, IN_CH * PATCH * PATCH))
    w.patch_b = f32("x_embedder.proj.bias")
    w.t_fc1_w = bf16(sd["t_embedder.mlp.0.weight"])
    w.t_fc1_b = f32("t_embedder.mlp.0.bias")
    # second timestep linear and the action linear share one GEMM along K; the action
    # bias rides in column 1049 against an input that is 1 only when actions are given
    w2 = torch.zeros(HIDDEN, HIDDEN + 64)
    w2[:, :HIDDEN] = sd["t_embedder.mlp.2.weight"].float()
    w2[:, HIDDEN:HIDDEN + ACTION_DIM] = sd["external_cond.weight"].float()
    w2[:, HIDDEN + ACTION_DIM] = sd["external_cond.bias"].float()
    w.t_fc2_w = bf16(w2)
    w.t_fc2_b = f32("t_embedder.mlp.2.bias")
    ada_w, ada_b = [], []
    for i in range(depth):
        for a in ("s", "t"):
            ada_w.append(sd[f"blocks.{i}.{a}_adaLN_modulation.1.weight"])
            ada_b.append(sd[f"blocks.{i}.{a}_adaLN_modulation.1.bias"])
    ada_w.append(sd["final_layer.adaLN_modulation.1.weight"])
    ada_b.append(sd["final_layer.adaLN_modulation.1.bias"])
    w.ada_w = bf16(torch.cat([t.float() for t in ada_w], 0))
    tb = torch.cat([t.float() for t in ada_b], 0).to(dev).contiguous()
    keep.append(tb)
    w.ada_b = tb.data_ptr()
    w.final_w = bf16(sd["final_layer.linear.weight"])
    w.final_b = f32("final_layer.linear.bias")
    for i in range(depth):
        for j, a in enumerate(("s", "t")):
            p = f"blocks.{i}.{a}_"
            sw = w.sub[2 * i + j]
            sw.qkv_w = bf16(sd[p + "attn.to_qkv.weight"])
            sw.out_w = bf16(sd[p + "attn.to_out.weight"])
            sw.out_b = f32(p + "attn.to_out.bias")
            sw.fc1_w = bf16(sd[p + "mlp.fc1.weight"])
            sw.fc1_b = f32(p + "mlp.fc1.bias")
            sw.fc2_w = bf16(sd[p + "mlp.fc2.weight"])
            sw.fc2_b = f32(p + "mlp.fc2.bias")
    sp, tp = rope_tables()
    sp, tp = sp.to(dev), tp.to(dev)
    keep += [sp, tp]
    w.rope_spatial = sp.data_ptr()
    w.rope_temporal = tp.data_ptr()
    return DeviceWeights(depth=depth, tensors=keep, struct=w)
