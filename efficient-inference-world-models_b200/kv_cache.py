"""Temporal KV cache in HBM (bf16 / FP8-e4m3 / INT4 frame slots) and the worldserve
cache interfaces on top of it.

Storage (``oasis_kv_cache_t`` in include/oasis_b200.h): one slot per past window
frame, each slot a (session, layer) page of 144 tokens x 16 heads x 64 of post-RoPE K
and V in its slot's kind:

* bf16 — plain;
* FP8  — e4m3fn codes + one bf16 scale per (session, layer, frame, head, K|V)
  (``ProgressiveKVQuantizer.quantize_to_fp8`` applied per 144 x 64 frame-head slice,
  ``kv_cache/progressive_quant.py:113-138``);
* INT4 — packed nibbles (element 2i in the high nibble) + fp16 scale/zero per
  (token, head) group of 64 (``quantize_to_int4(group_size=64)``,
  ``progressive_quant.py:140-193``).

The temporal attention kernel dequantises codes while staging K/V into shared memory,
so a quantised cache is never expanded to bf16 in HBM.
"""

from __future__ import annotations

import ctypes
import math
from typing import Any, Dict, List, Optional, Sequence

import torch

from . import _native as N

TOKENS, HIDDEN, HEADS, HEAD_DIM = 144, 1024, 16, 64
KIND_NAMES = {"bf16": N.KV_BF16, "fp16": N.KV_BF16, "fp8": N.KV_FP8, "int4": N.KV_INT4}


def _stream_ptr(stream=None) -> int:
    return (stream or torch.cuda.current_stream()).cuda_stream


def _pool_map(kinds: Sequence[str]):
    """Per-kind frame counts and each slot's index inside its kind's pool."""
    counts = {N.KV_BF16: 0, N.KV_FP8: 0, N.KV_INT4: 0}
    index = []
    for k in kinds:
        c = KIND_NAMES[k]
        index.append(counts[c])
        counts[c] += 1
    return counts, index


class KVCacheB200:
    """Device pools for ``batch`` sessions x ``layers`` blocks x ``len(slot_kinds)`` slots.

    ``slot_kinds`` are the storage kinds of the key slots (slot 0 = oldest frame);
    ``value_kinds`` those of the value slots (default: the same).  Keys and values have
    their own pools, sized by their own kind counts, as the reference's progressive
    quantiser keeps each in its own precision tier."""

    def __init__(self, batch: int, layers: int, slot_kinds: Sequence[str], device="cuda",
                 value_kinds: Optional[Sequence[str]] = None):
        if not 1 <= len(slot_kinds) <= N.MAX_FRAMES:
            raise ValueError("need 1..32 slots")
        value_kinds = list(slot_kinds) if value_kinds is None else list(value_kinds)
        if len(value_kinds) != len(slot_kinds):
            raise ValueError("keys and values need the same number of slots")
        self.batch, self.layers = batch, layers
        self.device = torch.device(device)
        self.slot_kinds = [str(k) for k in slot_kinds]
        self.value_kinds = [str(k) for k in value_kinds]
        k_counts, k_index = _pool_map(self.slot_kinds)
        v_counts, v_index = _pool_map(self.value_kinds)
        self.counts = {"k": k_counts, "v": v_counts}
        self._alloc_pools(k_counts, v_counts)
        s = self._pool_struct()
        s.n_slots = len(self.slot_kinds)
        for i in range(s.n_slots):
            s.k.slot_kind[i], s.k.slot_index[i] = KIND_NAMES[self.slot_kinds[i]], k_index[i]
            s.v.slot_kind[i], s.v.slot_index[i] = KIND_NAMES[self.value_kinds[i]], v_index[i]
        self.struct = s

    _POOL_NAMES = ("bf16", "fp8", "fp8_scale", "int4", "i4_scale", "i4_zero")

    def _alloc_pools(self, k_counts: Dict[int, int], v_counts: Dict[int, int]) -> None:
        """Zeroed storage for ``counts[kind]`` frame slots of each kind, per tensor:
        attributes ``k_bf16``, ``k_fp8``, ``k_fp8_scale``, ``k_int4``, ``k_i4_scale``,
        ``k_i4_zero`` and the same with ``v_`` (None where a pool is empty)."""
        dev = self.device
        lead = (self.batch, self.layers)
        for which, counts in (("k", k_counts), ("v", v_counts)):
            for name in self._POOL_NAMES:
                setattr(self, f"{which}_{name}", None)
            n = counts[N.KV_BF16]
            if n:
                setattr(self, f"{which}_bf16", torch.zeros(lead + (n, TOKENS, HIDDEN), dtype=torch.bfloat16, device=dev))
            n = counts[N.KV_FP8]
            if n:
                setattr(self, f"{which}_fp8", torch.zeros(lead + (n, TOKENS, HIDDEN), dtype=torch.uint8, device=dev))
                setattr(self, f"{which}_fp8_scale", torch.zeros(lead + (n, HEADS), dtype=torch.bfloat16, device=dev))
            n = counts[N.KV_INT4]
            if n:
                setattr(self, f"{which}_int4", torch.zeros(lead + (n, TOKENS, HEADS, HEAD_DIM // 2), dtype=torch.uint8, device=dev))
                setattr(self, f"{which}_i4_scale", torch.zeros(lead + (n, TOKENS, HEADS), dtype=torch.float16, device=dev))
                setattr(self, f"{which}_i4_zero", torch.zeros(lead + (n, TOKENS, HEADS), dtype=torch.float16, device=dev))

    def _pool_struct(self) -> "N.KvCache":
        """A cache descriptor over this object's pools with no slots mapped yet."""
        s = N.KvCache()
        s.batch, s.layers, s.n_slots = self.batch, self.layers, 0

        def ptr(t):
            return t.data_ptr() if t is not None else None

        for which in ("k", "v"):
            t = getattr(s, which)
            counts = self.counts[which]
            t.n_bf16, t.n_fp8, t.n_int4 = counts[N.KV_BF16], counts[N.KV_FP8], counts[N.KV_INT4]
            for name in self._POOL_NAMES:
                setattr(t, name, ptr(getattr(self, f"{which}_{name}")))
        return s

    # -- configurations of the benchmark -----------------------------------------
    @classmethod
    def uniform(cls, batch, layers, n_slots, kind="bf16", device="cuda"):
        return cls(batch, layers, [kind] * n_slots, device)

    @classmethod
    def progressive(cls, batch, layers, n_slots, recent_bf16=8, old_kind="int4", device="cuda"):
        """Newest ``recent_bf16`` frames bf16, older frames ``old_kind`` (slot 0 = oldest)."""
        kinds = [old_kind] * max(0, n_slots - recent_bf16) + ["bf16"] * min(n_slots, recent_bf16)
        return cls(batch, layers, kinds, device)

    @property
    def n_slots(self) -> int:
        return len(self.slot_kinds)

    def tensors(self) -> List[torch.Tensor]:
        out = []
        for which in ("k", "v"):
            for name in self._POOL_NAMES:
                t = getattr(self, f"{which}_{name}")
                if t is not None:
                    out.append(t)
        return out

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors())

    def bf16_equivalent_bytes(self) -> int:
        return 2 * self.batch * self.layers * self.n_slots * TOKENS * HIDDEN * 2

    # -- native operators ------------------------------------------------------------
    def store(self, kv: torch.Tensor, layer: int, slot0: int = 0, k_col: int = HIDDEN,
              v_col: int = 2 * HIDDEN, stream=None) -> None:
        """Quantise rows of ``kv`` (bf16 [batch*frames*144][ld], K at ``k_col``, V at
        ``v_col``) into slots ``slot0..slot0+frames-1`` of ``layer``."""
        if kv.dtype != torch.bfloat16 or not kv.is_cuda or kv.dim() != 2 or not kv.is_contiguous():
            raise ValueError("kv must be a contiguous 2-D bf16 CUDA tensor")
        rows = kv.shape[0]
        if rows % (self.batch * TOKENS):
            raise ValueError("kv rows must be batch * frames * 144")
        frames = rows // (self.batch * TOKENS)
        N.call("oasis_kv_store", kv.data_ptr(), kv.shape[1], k_col, v_col, ctypes.byref(self.struct),
               layer, self.batch, frames, slot0, _stream_ptr(stream))

    def load(self, layer: int, slot0: int = 0, frames: Optional[int] = None, stream=None):
        """Dequantised K, V of ``frames`` slots: two bf16 [batch][frames][144][1024] tensors."""
        frames = self.n_slots - slot0 if frames is None else frames
        k = torch.empty((self.batch, frames, TOKENS, HIDDEN), dtype=torch.bfloat16, device=self.device)
        v = torch.empty_like(k)
        N.call("oasis_kv_load", ctypes.byref(self.struct), layer, slot0, frames, k.data_ptr(),
               v.data_ptr(), _stream_ptr(stream))
        return k, v


def attn_temporal(qkv: torch.Tensor, batch: int, q_frames: int, q_pos0: int = 0, n_past: int = 0,
                  n_kv: Optional[int] = None, cache: Optional[KVCacheB200] = None, layer: int = 0,
                  out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Causal temporal attention (see ``oasis_attn_temporal``): qkv bf16
    [batch*q_frames*144][3072] -> out bf16 [batch*q_frames*144][1024]."""
    n_kv = q_frames + n_past if n_kv is None else n_kv
    if out is None:
        out = torch.empty((qkv.shape[0], HIDDEN), dtype=torch.bfloat16, device=qkv.device)
    N.call("oasis_attn_temporal", qkv.data_ptr(), ctypes.byref(cache.struct) if cache else None,
           layer, out.data_ptr(), batch, q_frames, q_pos0, n_past, n_kv, _stream_ptr(stream))
    return out


def attn_spatial(qkv: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Spatial attention (see ``oasis_attn_spatial``): qkv bf16 [frames*144][3072]."""
    frames = qkv.shape[0] // TOKENS
    if out is None:
        out = torch.empty((qkv.shape[0], HIDDEN), dtype=torch.bfloat16, device=qkv.device)
    N.call("oasis_attn_spatial", qkv.data_ptr(), out.data_ptr(), frames, _stream_ptr(stream))
    return out
