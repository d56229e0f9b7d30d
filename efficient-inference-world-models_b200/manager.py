"""worldserve KV-cache manager / progressive quantiser interfaces over the B200 cache.

``KVCacheManagerB200`` keeps the method names of ``KVCacheManager``
(``kv_cache/manager.py``: ``create_cache`` :196, ``update`` :246,
``get_kv_for_attention`` :416, ``get_cache`` :482, ``snapshot``/``restore`` :555-588,
``get_memory_report`` :594, ``pre_step``/``post_step`` :682-688,
``set_current_frame_idx`` :734, ``wire_to_model`` :923) but its storage is the
HBM-resident :class:`KVCacheB200`: K/V are captured inside the DiT forward (the
temporal QKV epilogue writes post-RoPE K/V, ``oasis_kv_store`` quantises them), not by
swapping ``F.scaled_dot_product_attention`` at run time.

``ProgressiveKVQuantizerB200`` keeps the tier policy of ``ProgressiveKVQuantizer``
(``progressive_quant.py:67-98``: FP8 from ``fp8_age_threshold`` frames of age, INT4
from ``int4_age_threshold``, V thresholds x0.7 when ``key_value_asymmetry``) and maps
it to per-slot storage kinds.  The codes are produced by the CUDA store kernel with
the reference's arithmetic.
"""

from __future__ import annotations

import ctypes
from typing import Any, Dict, List, Optional, Tuple

import torch

from . import _native as N
from .kv_cache import HEAD_DIM, HEADS, HIDDEN, KIND_NAMES, TOKENS, KVCacheB200, _stream_ptr


class ProgressiveKVQuantizerB200:
    def __init__(self, fp8_age_threshold: int = 30, int4_age_threshold: int = 90,
                 key_value_asymmetry: bool = True) -> None:
        self.key_value_asymmetry = key_value_asymmetry
        self.k_fp8_age = fp8_age_threshold
        self.k_int4_age = int4_age_threshold
        scale = 0.7 if key_value_asymmetry else 1.0
        self.v_fp8_age = int(fp8_age_threshold * scale)
        self.v_int4_age = int(int4_age_threshold * scale)

    def precision_for_age(self, age: int) -> str:
        """Storage tier of a frame ``age`` frames old.  One kind serves K and V of a slot,
        so the coarser of the K and V tiers is used (as ``get_mixed_precision_cache``
        groups entries by the coarser precision, ``progressive_quant.py:473-484``)."""
        def tier(fp8_age, int4_age):
            if age >= int4_age:
                return 2
            if age >= fp8_age:
                return 1
            return 0
        t = max(tier(self.k_fp8_age, self.k_int4_age), tier(self.v_fp8_age, self.v_int4_age))
        return ("bf16", "fp8", "int4")[t]

    def slot_kinds(self, n_past: int) -> List[str]:
        """Kinds of slots 0..n_past-1 where slot s holds a frame of age n_past - s."""
        return [self.precision_for_age(n_past - s) for s in range(n_past)]


def _kv_rows(new_kv: Dict[str, torch.Tensor]) -> torch.Tensor:
    """One frame's K/V of one layer, ``{"key", "value"}`` each (batch, heads, tokens,
    head_dim) or (heads, tokens, head_dim), as bf16 rows [batch*144][K 1024 | V 1024]."""
    k, v = new_kv["key"], new_kv["value"]
    if k.dim() == 3:
        k, v = k.unsqueeze(0), v.unsqueeze(0)
    b = k.shape[0]
    rows = torch.cat([k.permute(0, 2, 1, 3).reshape(b * TOKENS, HIDDEN),
                      v.permute(0, 2, 1, 3).reshape(b * TOKENS, HIDDEN)], dim=1)
    return rows.to(torch.bfloat16).contiguous()


class RollingKVCacheB200(KVCacheB200):
    """A rolling window of at most ``capacity`` cached frames that ages like the
    reference's progressive cache: every ``append`` stores the new frame at full
    precision (bf16) with age 0, drops the oldest frame once the window is full
    (``manager.py:296-306``), adds one to every older frame's age and promotes the frames
    whose tier changed, oldest first: bf16 -> FP8, bf16 -> INT4 or FP8 -> INT4, the last
    through the fp16 dequantisation (``update_cache``, ``progressive_quant.py:263-350``,
    with one kind per frame for K and V as in ``ProgressiveKVQuantizerB200``).

    Frames live in per-kind pools sized for a full window (a promotion always finds the
    slot its predecessor freed); logical slots 0 (oldest) .. n_slots-1 (newest) are
    remapped on every append, so the object works wherever a :class:`KVCacheB200` does
    (``OasisDiTB200.forward_cached``, ``attn_temporal``, ``load``)."""

    def __init__(self, batch: int, layers: int, capacity: int,
                 quantizer: "ProgressiveKVQuantizerB200", device="cuda"):
        if not 1 <= capacity < N.MAX_FRAMES:
            raise ValueError(f"capacity must be 1..{N.MAX_FRAMES - 1} past frames")
        self.batch, self.layers, self.capacity = batch, layers, capacity
        self.quantizer = quantizer
        self.device = torch.device(device)
        # a full window: the newest frame (age 0, bf16) and ages 1..capacity-1 by tier
        tiers = ["bf16"] + [quantizer.precision_for_age(a) for a in range(1, capacity)]
        self.counts = {N.KV_BF16: tiers.count("bf16"), N.KV_FP8: tiers.count("fp8"),
                       N.KV_INT4: tiers.count("int4")}
        self._alloc_pools(self.counts)
        self._free = {k: list(range(n)) for k, n in self.counts.items()}
        self.frames: List[Dict[str, int]] = []  # oldest first: {"age", "kind", "index"}
        self._remap()

    # -- logical slots -----------------------------------------------------------------
    def _remap(self) -> None:
        s = self._pool_struct()
        s.n_slots = len(self.frames)
        for i, f in enumerate(self.frames):
            s.slot_kind[i] = f["kind"]
            s.slot_index[i] = f["index"]
        self.struct = s
        names = {v: k for k, v in KIND_NAMES.items() if k != "fp16"}
        self.slot_kinds = [names[f["kind"]] for f in self.frames]

    def frame_slots(self) -> List[Tuple[str, int, int]]:
        """(kind, pool index, age) of every cached frame, oldest first."""
        return [(self.slot_kinds[i], f["index"], f["age"]) for i, f in enumerate(self.frames)]

    def _take(self, kind: int) -> int:
        if not self._free[kind]:
            raise RuntimeError("rolling KV cache: no free slot of the promoted kind")
        return self._free[kind].pop(0)

    def _promote(self, f: Dict[str, int], kind: int, stream) -> None:
        pair = self._pool_struct()
        pair.n_slots = 2
        pair.slot_kind[0], pair.slot_index[0] = f["kind"], f["index"]
        dst = self._take(kind)
        pair.slot_kind[1], pair.slot_index[1] = kind, dst
        N.call("oasis_kv_migrate", ctypes.byref(pair), 0, 1, _stream_ptr(stream))
        self._free[f["kind"]].append(f["index"])
        f["kind"], f["index"] = kind, dst

    # -- the progressive update ------------------------------------------------------------
    def append(self, rows_per_layer, stream=None) -> None:
        """Add one frame: ``rows_per_layer[layer]`` is that layer's K/V as bf16 rows
        [batch*144][ld] with K in columns 0..1023 and V in 1024..2047, or a
        ``{"key", "value"}`` dict as ``KVCacheManager.update`` takes."""
        if len(rows_per_layer) != self.layers:
            raise ValueError("one entry per layer")
        if len(self.frames) == self.capacity:
            old = self.frames.pop(0)
            self._free[old["kind"]].append(old["index"])
        rank = {N.KV_BF16: 0, N.KV_FP8: 1, N.KV_INT4: 2}
        for f in self.frames:  # oldest first
            f["age"] += 1
            want = KIND_NAMES[self.quantizer.precision_for_age(f["age"])]
            if rank[want] > rank[f["kind"]]:
                self._promote(f, want, stream)
        self.frames.append({"age": 0, "kind": N.KV_BF16, "index": self._take(N.KV_BF16)})
        self._remap()
        for layer in range(self.layers):
            rows = rows_per_layer[layer]
            if isinstance(rows, dict):
                rows = _kv_rows(rows)
            self.store(rows, layer, slot0=self.n_slots - 1, k_col=0, v_col=HIDDEN, stream=stream)


class KVCacheManagerB200:
    def __init__(self, config: Dict[str, Any]) -> None:
        self.config = config
        self.num_layers = config.get("num_layers", 16)
        self.max_frames = config.get("max_frames", 32)
        self.batch = config.get("batch", 1)
        pq = config.get("progressive_quant", False)
        self.progressive_quantizer: Optional[ProgressiveKVQuantizerB200] = None
        if pq:
            kw = pq if isinstance(pq, dict) else {}
            self.progressive_quantizer = ProgressiveKVQuantizerB200(
                fp8_age_threshold=kw.get("fp8_age_threshold", 30),
                int4_age_threshold=kw.get("int4_age_threshold", 90),
                key_value_asymmetry=kw.get("key_value_asymmetry", True))
        self.fixed_kinds: Optional[List[str]] = config.get("slot_kinds")
        self.cache: Optional[KVCacheB200] = None
        self._current_frame_idx: Optional[int] = None
        self._step = 0
        self.device = config.get("device", "cuda")

    # -- lifecycle -----------------------------------------------------------------
    def create_cache(self, num_layers: Optional[int] = None, max_frames: Optional[int] = None) -> None:
        if num_layers is not None:
            self.num_layers = num_layers
        if max_frames is not None:
            self.max_frames = max_frames
        self.cache = None
        self._current_frame_idx = None
        self._step = 0

    def kinds_for(self, n_past: int) -> List[str]:
        if self.fixed_kinds is not None:
            return list(self.fixed_kinds[:n_past])
        if self.progressive_quantizer is not None:
            return self.progressive_quantizer.slot_kinds(n_past)
        return ["bf16"] * n_past

    def cache_for_window(self, n_past: int) -> KVCacheB200:
        """The cache a full-window forward of ``n_past + 1`` frames writes (prefill)."""
        kinds = self.kinds_for(n_past)
        if self.cache is None or self.cache.slot_kinds != kinds:
            self.cache = KVCacheB200(self.batch, self.num_layers, kinds, device=self.device)
        return self.cache

    def set_current_frame_idx(self, frame_idx: int) -> None:
        self._current_frame_idx = int(frame_idx)

    # -- updates / retrieval ----------------------------------------------------------
    def update(self, new_kv: Dict[int, Dict[str, torch.Tensor]], frame_idx: int,
               attention_weights=None, slot: Optional[int] = None) -> None:
        """Store one frame's post-RoPE K/V per layer: ``new_kv[layer] = {"key", "value"}``
        each (batch, heads, tokens, head_dim) or (heads, tokens, head_dim) bf16."""
        if self.cache is None:
            raise RuntimeError("no cache: call cache_for_window() (or run a prefill) first")
        s = self.cache.n_slots - 1 if slot is None else slot
        for layer, kv in new_kv.items():
            k, v = kv["key"], kv["value"]
            if k.dim() == 3:
                k, v = k.unsqueeze(0), v.unsqueeze(0)
            b = k.shape[0]
            # (B, heads, tokens, d) -> rows (B*tokens) x [K(1024) | V(1024)]
            rows = torch.cat([k.permute(0, 2, 1, 3).reshape(b * TOKENS, HIDDEN),
                              v.permute(0, 2, 1, 3).reshape(b * TOKENS, HIDDEN)], dim=1)
            self.cache.store(rows.to(torch.bfloat16).contiguous(), layer, slot0=s, k_col=0, v_col=HIDDEN)
        self._current_frame_idx = frame_idx

    def append(self, new_kv: Dict[int, Dict[str, torch.Tensor]], frame_idx: int) -> None:
        """The reference's progressive ``update`` (``manager.py:246-306`` with
        ``progressive_quant.py:263-350``): append one frame's post-RoPE K/V for every
        layer to a rolling window of ``max_frames - 1`` past frames (at most 31) that
        ages and promotes its frames (:class:`RollingKVCacheB200`)."""
        if not isinstance(self.cache, RollingKVCacheB200):
            q = self.progressive_quantizer or ProgressiveKVQuantizerB200(
                fp8_age_threshold=10 ** 6, int4_age_threshold=10 ** 6)
            self.cache = RollingKVCacheB200(self.batch, self.num_layers,
                                            min(self.max_frames - 1, N.MAX_FRAMES - 1), q,
                                            device=self.device)
        self.cache.append([new_kv[layer] for layer in range(self.num_layers)])
        self._current_frame_idx = frame_idx

    def get_kv_for_attention(self, layer_idx: int) -> Dict[str, torch.Tensor]:
        """Dequantised K/V of every slot: ``(batch, heads, slots*tokens, head_dim)`` bf16."""
        if self.cache is None:
            return {"key": torch.zeros(0), "value": torch.zeros(0)}
        k, v = self.cache.load(layer_idx)
        B, F = k.shape[:2]

        def heads(z):
            return z.reshape(B, F, TOKENS, HEADS, HEAD_DIM).permute(0, 3, 1, 2, 4).reshape(
                B, HEADS, F * TOKENS, HEAD_DIM)

        return {"key": heads(k), "value": heads(v)}

    def get_cache(self, precision: str = "fp16") -> Dict[int, Dict[str, torch.Tensor]]:
        return {l: self.get_kv_for_attention(l) for l in range(self.num_layers)} if self.cache else {}

    def snapshot(self):
        if self.cache is None:
            return None
        return [t.clone() for t in self.cache.tensors()]

    def restore(self, snap) -> None:
        if snap is None or self.cache is None:
            return
        for dst, src in zip(self.cache.tensors(), snap):
            dst.copy_(src)

    # -- reporting / hooks ------------------------------------------------------------
    def get_memory_report(self) -> Dict[str, Any]:
        if self.cache is None:
            return {"total_fp16_bytes": 0, "total_actual_bytes": 0, "savings_ratio": 0.0}
        full = self.cache.bf16_equivalent_bytes()
        actual = self.cache.nbytes
        return {"total_fp16_bytes": full, "total_actual_bytes": actual,
                "savings_ratio": 1.0 - actual / max(full, 1),
                "slot_kinds": list(self.cache.slot_kinds)}

    def get_stats(self) -> Dict[str, Any]:
        return self.get_memory_report()

    def pre_step(self, step_idx: int, total_steps: int, latents) -> bool:
        return False

    def post_step(self, step_idx: int, total_steps: int, latents) -> None:
        self._step = step_idx + 1

    def wire_to_model(self, model) -> int:
        """Attach to an ``OasisDiTB200``; returns the number of temporal layers served."""
        model.kv_manager = self
        self.num_layers = model.depth
        return model.depth
