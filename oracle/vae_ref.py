"""PyTorch fp32 CPU restatement of the ViT latent decoder behind Oasis's ``vae.decode``.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Parity with upstream open-oasis
is *unpinned*: the reference builds ``VAE_models["vit-l-20-shallow-encoder"]`` from an
unpinned open-oasis clone (``worldserve/models/oasis.py:60-82``) whose ``vae.py`` is not in
the reference tree, and ships no weights or outputs.  What the reference itself fixes, and
what this file follows:

* the call — ``vae.decode(z)`` with ``z`` of shape ``(frames, 576, 16)``: the DiT's
  ``(B, T, 16, 18, 32)`` latents divided by the VAE scale and laid out token-major
  (``oasis.py:237-242``); the result is an RGB frame per latent frame in [-1, 1]
  (``frames = (decoded + 1) / 2``, ``oasis.py:243-244``) at the 360 x 640 resolution the
  latent grid implies for a patch of 20 (``vit-l-20``: 18 x 32 tokens);
* ViT-L width: 1024 features, 16 heads of 64.

Choices that only upstream pins, fixed here once and used on both sides (the same family of
choices as the DiT restatement in ``oracle/dit_ref.py``): a Linear(16 -> 1024) latent
projection; 12 pre-norm transformer blocks (LayerNorm eps 1e-6 with affine; attention
with a bias-free QKV projection, axial RoPE on q and k over the 18 x 32 token grid — 16
"pixel" frequencies ``linspace(1, 128, 16)*pi`` per axis over ``linspace(-1, 1, n)``,
H axis on head dims 0..31, W axis on 32..63, pairs interleaved — non-causal softmax
attention and an output projection with bias; MLP 1024 -> 4096 -> 1024 with GELU(tanh));
a final affine LayerNorm; Linear(1024 -> 20*20*3) and an ``(h w) (p q c) -> c (h p) (w q)``
unpatchify.
"""

from __future__ import annotations

import math
from typing import Dict

import torch
import torch.nn.functional as F

DIM = 1024
HEADS = 16
HEAD_DIM = 64
DEPTH = 12
MLP_HIDDEN = 4096
LATENT = 16
GRID_H, GRID_W = 18, 32
TOKENS = GRID_H * GRID_W  # 576
PATCH = 20
OUT_CH = 3
PATCH_DIM = PATCH * PATCH * OUT_CH  # 1200
IMG_H, IMG_W = GRID_H * PATCH, GRID_W * PATCH  # 360, 640
LN_EPS = 1e-6


def param_shapes(depth: int = DEPTH) -> Dict[str, tuple]:
    """Parameter names and shapes of the decoder restated here."""
    shapes = {"post_quant_conv.weight": (DIM, LATENT), "post_quant_conv.bias": (DIM,)}
    for i in range(depth):
        p = f"decoder.{i}."
        shapes.update({
            p + "norm1.weight": (DIM,), p + "norm1.bias": (DIM,),
            p + "attn.qkv.weight": (3 * DIM, DIM),
            p + "attn.proj.weight": (DIM, DIM), p + "attn.proj.bias": (DIM,),
            p + "norm2.weight": (DIM,), p + "norm2.bias": (DIM,),
            p + "mlp.fc1.weight": (MLP_HIDDEN, DIM), p + "mlp.fc1.bias": (MLP_HIDDEN,),
            p + "mlp.fc2.weight": (DIM, MLP_HIDDEN), p + "mlp.fc2.bias": (DIM,),
        })
    shapes.update({"dec_norm.weight": (DIM,), "dec_norm.bias": (DIM,),
                   "predictor.weight": (PATCH_DIM, DIM), "predictor.bias": (PATCH_DIM,)})
    return shapes


def rope_table() -> torch.Tensor:
    """[576][32][2] fp32 (cos, sin) per token and rotated pair (pairs 0..15: H angle,
    16..31: W angle)."""
    f = torch.linspace(1.0, 128.0, 16) * math.pi
    ah = torch.linspace(-1, 1, GRID_H)[:, None] * f
    aw = torch.linspace(-1, 1, GRID_W)[:, None] * f
    ang = torch.cat([ah[:, None, :].expand(GRID_H, GRID_W, 16),
                     aw[None, :, :].expand(GRID_H, GRID_W, 16)], dim=-1).reshape(TOKENS, 32)
    return torch.stack([ang.cos(), ang.sin()], dim=-1).contiguous()


def _rope(x: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs (2i, 2i+1) of the last dim of x (..., 576, 64)."""
    cos, sin = table[..., 0], table[..., 1]  # (576, 32)
    a, b = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = a * cos - b * sin
    out[..., 1::2] = a * sin + b * cos
    return out


def decode(sd: Dict[str, torch.Tensor], z: torch.Tensor, depth: int = DEPTH) -> torch.Tensor:
    """``vae.decode``: z (frames, 576, 16) -> RGB (frames, 3, 360, 640), fp32 on the CPU."""
    w = {k: v.float() for k, v in sd.items()}
    n = z.shape[0]
    table = rope_table()
    x = F.linear(z.float(), w["post_quant_conv.weight"], w["post_quant_conv.bias"])
    for i in range(depth):
        p = f"decoder.{i}."
        h = F.layer_norm(x, (DIM,), w[p + "norm1.weight"], w[p + "norm1.bias"], eps=LN_EPS)
        q, k, v = F.linear(h, w[p + "attn.qkv.weight"]).view(n, TOKENS, 3, HEADS, HEAD_DIM).unbind(2)
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))  # (n, heads, 576, 64)
        q, k = _rope(q, table), _rope(k, table)
        o = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(n, TOKENS, DIM)
        x = x + F.linear(o, w[p + "attn.proj.weight"], w[p + "attn.proj.bias"])
        h = F.layer_norm(x, (DIM,), w[p + "norm2.weight"], w[p + "norm2.bias"], eps=LN_EPS)
        h = F.gelu(F.linear(h, w[p + "mlp.fc1.weight"], w[p + "mlp.fc1.bias"]), approximate="tanh")
        x = x + F.linear(h, w[p + "mlp.fc2.weight"], w[p + "mlp.fc2.bias"])
    x = F.layer_norm(x, (DIM,), w["dec_norm.weight"], w["dec_norm.bias"], eps=LN_EPS)
    y = F.linear(x, w["predictor.weight"], w["predictor.bias"])  # (n, 576, 1200)
    y = y.reshape(n, GRID_H, GRID_W, PATCH, PATCH, OUT_CH)
    return torch.einsum("nhwpqc->nchpwq", y).reshape(n, OUT_CH, IMG_H, IMG_W)
