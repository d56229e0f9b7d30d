"""PyTorch fp32 CPU restatement of the Oasis-500M (open-oasis ``DiT-S/2``) forward.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Parity with upstream
open-oasis is *unpinned*: the reference imports ``dit.DiT_models["DiT-S/2"]``
from an unpinned clone (``worldserve/models/oasis.py:66-77``,
``benchmarks/common.py:45-55``) that is not present, together with its
``rotary_embedding_torch`` module.  What the reference itself fixes, and what
this file follows:

* block structure — split spatial / temporal adaLN, 6-way chunk order
  shift, scale, gate (msa) then shift, scale, gate (mlp)
  (``benchmarks/optimised/oasis_custom_modal.py:395-431``);
* temporal attention — ``to_qkv`` without bias, ``to_out`` with bias,
  ``B T H W (h d) -> (B H W) h T d``, RoPE on q and k, causal SDPA, back-
  rearrange, ``to_out``
  (``kv_cache/oasis_temporal_persistent_wrapper.py:76-150``);
* the KV manager finds the attention modules by class name
  ``SpatialAxialAttention`` / ``TemporalAxialAttention``
  (``kv_cache/manager.py:947-961``) and the temporal wrapper by
  ``model.blocks[i].t_attn`` (``oasis_temporal_persistent_wrapper.py:160-167``);
* dims — hidden 1024, 16 heads x 64, depth 16 (``n_temporal_modules_wired: 16``
  in the reference's run JSONs), MLP ratio 4, patch 2, 16 latent channels on an
  18 x 32 latent, 25-dim action conditioning (``models/oasis.py:39-43,166-167``).

Choices that only upstream pins, fixed here once and used on both sides:
LayerNorm eps 1e-6 without affine; GELU(tanh); a 256-dim sinusoidal timestep
embedding (cos first, then sin; max period 10000) feeding Linear-SiLU-Linear;
final layer = LayerNorm + adaLN(shift, scale) + Linear(1024 -> 2*2*16) and an
``nhwpqc -> nchpwq`` unpatchify; temporal RoPE over all 64 head dims with
``1/10000^(2i/64)`` frequencies at window-relative positions 0..T-1; spatial
axial RoPE with 16 "pixel" frequencies ``linspace(1, 128, 16)*pi`` per axis over
``linspace(-1, 1, n)`` positions, H axis on head dims 0..31 and W axis on 32..63;
RoPE pairs are interleaved (dims 2i, 2i+1).
"""

from __future__ import annotations

import math
from typing import Dict, Optional

import torch
import torch.nn.functional as F
from torch import nn

HIDDEN = 1024
HEADS = 16
HEAD_DIM = 64
DEPTH = 16
MLP_HIDDEN = 4096
PATCH = 2
IN_CH = 16
LAT_H = 18
LAT_W = 32
GRID_H = LAT_H // PATCH  # 9
GRID_W = LAT_W // PATCH  # 16
TOKENS = GRID_H * GRID_W  # 144
ACTION_DIM = 25
FREQ_EMB = 256
LN_EPS = 1e-6


# ---------------------------------------------------------------------------
# Rotary embedding (restatement of the rotary_embedding_torch API the
# upstream attention modules call: rotate_queries_or_keys / get_axial_freqs)
# ---------------------------------------------------------------------------

def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """Interleaved rotation: (x0, x1, x2, x3, ...) -> (-x1, x0, -x3, x2, ...)."""
    pairs = x.unflatten(-1, (-1, 2))
    a, b = pairs.unbind(-1)
    return torch.stack((-b, a), dim=-1).flatten(-2)


def apply_rotary_emb(freqs: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
    """``t * cos(freqs) + rotate_half(t) * sin(freqs)`` over the last dim, cast back."""
    dtype = t.dtype
    out = t * freqs.cos() + rotate_half(t) * freqs.sin()
    return out.type(dtype)


class RotaryEmbedding(nn.Module):
    def __init__(self, dim: int, freqs_for: str = "lang", theta: float = 10000.0,
                 max_freq: float = 10.0) -> None:
        super().__init__()
        self.freqs_for = freqs_for
        if freqs_for == "lang":
            freqs = 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
        elif freqs_for == "pixel":
            freqs = torch.linspace(1.0, max_freq / 2, dim // 2) * math.pi
        else:
            raise ValueError(freqs_for)
        # upstream keeps the frequencies as a frozen parameter
        self.freqs = nn.Parameter(freqs, requires_grad=False)

    @staticmethod
    def _angles(pos: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
        ang = pos.type(freqs.dtype)[..., None] * freqs
        return ang.repeat_interleave(2, dim=-1)

    def rotate_queries_or_keys(self, t: torch.Tensor, freqs: torch.Tensor,
                               offset: int = 0) -> torch.Tensor:
        """Rotate along the sequence dim (-2) at positions ``offset .. offset+S-1``."""
        seq_len = t.shape[-2]
        pos = torch.arange(seq_len, dtype=t.dtype) + offset
        return apply_rotary_emb(self._angles(pos, freqs), t)

    def get_axial_freqs(self, *dims: int) -> torch.Tensor:
        parts = []
        for axis, n in enumerate(dims):
            pos = torch.linspace(-1, 1, steps=n) if self.freqs_for == "pixel" else torch.arange(n)
            ang = self._angles(pos, self.freqs)  # (n, 2*nf)
            shape = [1] * len(dims) + [ang.shape[-1]]
            shape[axis] = n
            parts.append(ang.reshape(shape))
        parts = torch.broadcast_tensors(*parts)
        return torch.cat(parts, dim=-1)


# ---------------------------------------------------------------------------
# Attention modules (class names are part of the reference's plug-in API)
# ---------------------------------------------------------------------------

class SpatialAxialAttention(nn.Module):
    def __init__(self, dim: int, heads: int, dim_head: int, rotary_emb: RotaryEmbedding) -> None:
        super().__init__()
        self.heads = heads
        self.head_dim = dim_head
        self.inner_dim = heads * dim_head
        self.to_qkv = nn.Linear(dim, 3 * self.inner_dim, bias=False)
        self.to_out = nn.Linear(self.inner_dim, dim)
        self.rotary_emb = rotary_emb

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, H, W, _ = x.shape
        q, k, v = self.to_qkv(x).chunk(3, dim=-1)

        def heads_first(z):  # B T H W (h d) -> (B T) h H W d
            return z.reshape(B * T, H, W, self.heads, self.head_dim).permute(0, 3, 1, 2, 4)

        q, k, v = heads_first(q), heads_first(k), heads_first(v)
        freqs = self.rotary_emb.get_axial_freqs(H, W)
        q = apply_rotary_emb(freqs, q)
        k = apply_rotary_emb(freqs, k)
        q, k, v = (z.reshape(B * T, self.heads, H * W, self.head_dim) for z in (q, k, v))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=False)
        o = o.reshape(B, T, self.heads, H, W, self.head_dim).permute(0, 1, 3, 4, 2, 5)
        o = o.reshape(B, T, H, W, self.inner_dim).to(q.dtype)
        return self.to_out(o)


class TemporalAxialAttention(nn.Module):
    def __init__(self, dim: int, heads: int, dim_head: int, rotary_emb: RotaryEmbedding,
                 is_causal: bool = True) -> None:
        super().__init__()
        self.heads = heads
        self.head_dim = dim_head
        self.inner_dim = heads * dim_head
        self.to_qkv = nn.Linear(dim, 3 * self.inner_dim, bias=False)
        self.to_out = nn.Linear(self.inner_dim, dim)
        self.rotary_emb = rotary_emb
        self.is_causal = is_causal

    def project(self, x: torch.Tensor):
        """Post-RoPE q, k, v in ``(B H W) h T d`` layout (what SDPA receives)."""
        B, T, H, W, _ = x.shape
        q, k, v = self.to_qkv(x).chunk(3, dim=-1)

        def seq_layout(z):  # B T H W (h d) -> (B H W) h T d
            z = z.reshape(B, T, H, W, self.heads, self.head_dim).permute(0, 2, 3, 4, 1, 5)
            return z.reshape(B * H * W, self.heads, T, self.head_dim)

        q, k, v = seq_layout(q), seq_layout(k), seq_layout(v)
        q = self.rotary_emb.rotate_queries_or_keys(q, self.rotary_emb.freqs)
        k = self.rotary_emb.rotate_queries_or_keys(k, self.rotary_emb.freqs)
        return q, k, v

    def finish(self, o: torch.Tensor, B: int, H: int, W: int) -> torch.Tensor:
        T = o.shape[2]
        o = o.reshape(B, H, W, self.heads, T, self.head_dim).permute(0, 4, 1, 2, 3, 5)
        o = o.reshape(B, T, H, W, self.inner_dim)
        return self.to_out(o)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, H, W, _ = x.shape
        q, k, v = self.project(x)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=self.is_causal).to(q.dtype)
        return self.finish(o, B, H, W)


# ---------------------------------------------------------------------------
# DiT
# ---------------------------------------------------------------------------

def modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """Per-frame modulation: shift/scale are (B, T, D), x is (B, T, H, W, D)."""
    while shift.dim() < x.dim():
        shift = shift.unsqueeze(-2)
        scale = scale.unsqueeze(-2)
    return x * (1 + scale) + shift


def gate(x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    while g.dim() < x.dim():
        g = g.unsqueeze(-2)
    return g * x


class Mlp(nn.Module):
    def __init__(self, dim: int, hidden: int) -> None:
        super().__init__()
        self.fc1 = nn.Linear(dim, hidden)
        self.fc2 = nn.Linear(hidden, dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc2(F.gelu(self.fc1(x), approximate="tanh"))


class PatchEmbed(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.proj = nn.Conv2d(IN_CH, HIDDEN, kernel_size=PATCH, stride=PATCH)

    def forward(self, x: torch.Tensor) -> torch.Tensor:  # (N, C, H, W) -> (N, h, w, D)
        return self.proj(x).permute(0, 2, 3, 1)


class TimestepEmbedder(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.mlp = nn.Sequential(nn.Linear(FREQ_EMB, HIDDEN), nn.SiLU(), nn.Linear(HIDDEN, HIDDEN))

    @staticmethod
    def timestep_embedding(t: torch.Tensor, dim: int = FREQ_EMB, max_period: float = 10000.0):
        half = dim // 2
        freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32) / half)
        args = t[:, None].float() * freqs[None]
        return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)

    def forward(self, t: torch.Tensor) -> torch.Tensor:
        return self.mlp(self.timestep_embedding(t))


class FinalLayer(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.norm_final = nn.LayerNorm(HIDDEN, elementwise_affine=False, eps=LN_EPS)
        self.linear = nn.Linear(HIDDEN, PATCH * PATCH * IN_CH)
        self.adaLN_modulation = nn.Sequential(nn.SiLU(), nn.Linear(HIDDEN, 2 * HIDDEN))

    def forward(self, x: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
        shift, scale = self.adaLN_modulation(c).chunk(2, dim=-1)
        return self.linear(modulate(self.norm_final(x), shift, scale))


class SpatioTemporalDiTBlock(nn.Module):
    def __init__(self, spatial_rotary: RotaryEmbedding, temporal_rotary: RotaryEmbedding) -> None:
        super().__init__()
        ln = lambda: nn.LayerNorm(HIDDEN, elementwise_affine=False, eps=LN_EPS)
        self.s_norm1, self.s_norm2 = ln(), ln()
        self.s_attn = SpatialAxialAttention(HIDDEN, HEADS, HEAD_DIM, spatial_rotary)
        self.s_mlp = Mlp(HIDDEN, MLP_HIDDEN)
        self.s_adaLN_modulation = nn.Sequential(nn.SiLU(), nn.Linear(HIDDEN, 6 * HIDDEN))
        self.t_norm1, self.t_norm2 = ln(), ln()
        self.t_attn = TemporalAxialAttention(HIDDEN, HEADS, HEAD_DIM, temporal_rotary, is_causal=True)
        self.t_mlp = Mlp(HIDDEN, MLP_HIDDEN)
        self.t_adaLN_modulation = nn.Sequential(nn.SiLU(), nn.Linear(HIDDEN, 6 * HIDDEN))

    def spatial(self, x, c):
        sh1, sc1, g1, sh2, sc2, g2 = self.s_adaLN_modulation(c).chunk(6, dim=-1)
        x = x + gate(self.s_attn(modulate(self.s_norm1(x), sh1, sc1)), g1)
        B, T, H, W, D = x.shape
        h = modulate(self.s_norm2(x), sh2, sc2).reshape(B * T, H * W, D)
        return x + gate(self.s_mlp(h).reshape(B, T, H, W, D), g2)

    def temporal(self, x, c, attn_fn=None):
        sh1, sc1, g1, sh2, sc2, g2 = self.t_adaLN_modulation(c).chunk(6, dim=-1)
        h = modulate(self.t_norm1(x), sh1, sc1)
        a = self.t_attn(h) if attn_fn is None else attn_fn(self.t_attn, h)
        x = x + gate(a, g1)
        B, T, H, W, D = x.shape
        h = modulate(self.t_norm2(x), sh2, sc2).reshape(B * T, H * W, D)
        return x + gate(self.t_mlp(h).reshape(B, T, H, W, D), g2)

    def forward(self, x, c):
        return self.temporal(self.spatial(x, c), c)


class DiT(nn.Module):
    """``DiT-S/2`` as the reference instantiates it (``DiT_models["DiT-S/2"]()``)."""

    def __init__(self, depth: int = DEPTH, max_frames: int = 32) -> None:
        super().__init__()
        self.max_frames = max_frames
        self.x_embedder = PatchEmbed()
        self.t_embedder = TimestepEmbedder()
        self.spatial_rotary_emb = RotaryEmbedding(HEAD_DIM // 2, freqs_for="pixel", max_freq=256)
        self.temporal_rotary_emb = RotaryEmbedding(HEAD_DIM)
        self.external_cond = nn.Linear(ACTION_DIM, HIDDEN)
        self.blocks = nn.ModuleList(
            [SpatioTemporalDiTBlock(self.spatial_rotary_emb, self.temporal_rotary_emb) for _ in range(depth)]
        )
        self.final_layer = FinalLayer()

    def embed(self, x, t, external_cond):
        B, T = x.shape[:2]
        tok = self.x_embedder(x.reshape(B * T, IN_CH, LAT_H, LAT_W)).reshape(B, T, GRID_H, GRID_W, HIDDEN)
        c = self.t_embedder(t.reshape(-1)).reshape(B, T, HIDDEN)
        if external_cond is not None:
            c = c + self.external_cond(external_cond)
        return tok, c

    def unpatchify_out(self, x, c):
        B, T = x.shape[:2]
        y = self.final_layer(x, c)  # (B, T, h, w, p*p*C)
        y = y.reshape(B * T, GRID_H, GRID_W, PATCH, PATCH, IN_CH)
        y = torch.einsum("nhwpqc->nchpwq", y).reshape(B, T, IN_CH, LAT_H, LAT_W)
        return y

    def forward(self, x: torch.Tensor, t: torch.Tensor, external_cond: Optional[torch.Tensor] = None):
        tok, c = self.embed(x, t, external_cond)
        for blk in self.blocks:
            tok = blk(tok, c)
        return self.unpatchify_out(tok, c)

    # -- cached incremental forward (persistent past-frame K/V) --------------

    def forward_capture_kv(self, x, t, external_cond=None):
        """Full-window forward that also returns, per block, the post-RoPE temporal
        K/V in ``(B H W) h T d`` layout (the tensors the reference's
        ``_capture_sdpa`` sees, ``kv_cache/manager.py:1048-1054``)."""
        tok, c = self.embed(x, t, external_cond)
        kvs = []

        def capture(attn, h):
            B, T, H, W, _ = h.shape
            q, k, v = attn.project(h)
            kvs.append((k, v))
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True).to(q.dtype)
            return attn.finish(o, B, H, W)

        for blk in self.blocks:
            tok = blk.temporal(blk.spatial(tok, c), c, attn_fn=capture)
        return self.unpatchify_out(tok, c), kvs

    def forward_incremental(self, x_new, t_new, a_new, past_kv, pos: int):
        """Forward of one new frame per session against cached past K/V.

        ``past_kv[i] = (k, v)`` are ``(B*H*W, heads, P, d)`` post-RoPE tensors of
        the ``P`` past frames for block ``i`` (possibly after a quantisation round
        trip); the new frame sits at window position ``pos`` (= P).  Equal to the
        last frame of a full-window forward when ``past_kv`` is exact
        (``kv_cache/oasis_persistent_kv_theory.py:24-112``).
        """
        tok, c = self.embed(x_new, t_new, a_new)  # T = 1

        for i, blk in enumerate(self.blocks):
            kp, vp = past_kv[i]

            def cached(attn, h, kp=kp, vp=vp):
                B, T, H, W, _ = h.shape
                q, k, v = attn.to_qkv(h).chunk(3, dim=-1)

                def seq_layout(z):
                    z = z.reshape(B, T, H, W, attn.heads, attn.head_dim).permute(0, 2, 3, 4, 1, 5)
                    return z.reshape(B * H * W, attn.heads, T, attn.head_dim)

                q, k, v = seq_layout(q), seq_layout(k), seq_layout(v)
                q = attn.rotary_emb.rotate_queries_or_keys(q, attn.rotary_emb.freqs, offset=pos)
                k = attn.rotary_emb.rotate_queries_or_keys(k, attn.rotary_emb.freqs, offset=pos)
                kk = torch.cat([kp.to(k.dtype), k], dim=2)
                vv = torch.cat([vp.to(v.dtype), v], dim=2)
                o = F.scaled_dot_product_attention(q, kk, vv, is_causal=False).to(q.dtype)
                return attn.finish(o, B, H, W)

            tok = blk.temporal(blk.spatial(tok, c), c, attn_fn=cached)
        return self.unpatchify_out(tok, c)


def DiT_S_2(**kw) -> DiT:
    return DiT(**kw)


def build_oracle(state_dict: Dict[str, torch.Tensor], depth: int = DEPTH) -> DiT:
    """fp32 CPU oracle loaded from a state dict with upstream parameter names."""
    m = DiT(depth=depth)
    missing, unexpected = m.load_state_dict(
        {k: v.float().cpu() for k, v in state_dict.items()}, strict=False)
    missing = [k for k in missing if not k.endswith("rotary_emb.freqs")]
    if missing or unexpected:
        raise KeyError(f"state dict mismatch: missing={missing[:5]} unexpected={unexpected[:5]}")
    return m.eval()
