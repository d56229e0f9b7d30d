"""worldserve KV-cache manager / progressive quantiser interfaces over the B200 cache.

``KVCacheManagerB200`` keeps the method names and the behaviour of ``KVCacheManager``
(``kv_cache/manager.py``: ``create_cache`` :196, ``update`` :246-306,
``get_kv_for_attention`` :416, ``get_cache`` :482, ``snapshot``/``restore`` :555-588,
``get_memory_report`` :594, ``pre_step``/``post_step`` :682-688,
``set_current_frame_idx`` :734, ``wire_to_model`` :923), but its storage is the
HBM-resident :class:`KVCacheB200`: K/V are captured inside the DiT forward (the
temporal QKV epilogue writes post-RoPE K/V, ``oasis_kv_store`` quantises them), not by
swapping ``F.scaled_dot_product_attention`` at run time, and a frame is kept only in
its current precision tier (the reference keeps a full-precision copy beside the
quantised store, which is what the quantised cache exists to avoid).

``ProgressiveKVQuantizerB200`` keeps the tier policy of ``ProgressiveKVQuantizer``
(``progressive_quant.py:67-98``): keys drop to FP8 at ``fp8_age_threshold`` frames of
age and to INT4 at ``int4_age_threshold``; values at ``int(0.7 x)`` those ages when
``key_value_asymmetry`` is set.  Keys and values are tiered separately, as
``update_cache`` promotes them (:310-322).  The codes are produced by the CUDA store
and migrate kernels with the reference's arithmetic.
"""

from __future__ import annotations

import ctypes
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch

from . import _native as N
from .kv_cache import HEAD_DIM, HEADS, HIDDEN, KIND_NAMES, TOKENS, KVCacheB200, _stream_ptr

_TIER_NAMES = ("bf16", "fp8", "int4")
_RANK = {N.KV_BF16: 0, N.KV_FP8: 1, N.KV_INT4: 2}


class ProgressiveKVQuantizerB200:
    def __init__(self, fp8_age_threshold: int = 30, int4_age_threshold: int = 90,
                 key_value_asymmetry: bool = True) -> None:
        self.key_value_asymmetry = key_value_asymmetry
        self.k_fp8_age = fp8_age_threshold
        self.k_int4_age = int4_age_threshold
        if key_value_asymmetry:
            self.v_fp8_age = int(fp8_age_threshold * 0.7)
            self.v_int4_age = int(int4_age_threshold * 0.7)
        else:
            self.v_fp8_age = fp8_age_threshold
            self.v_int4_age = int4_age_threshold

    def precision_for_age(self, age: int, tensor: str = "key") -> str:
        """Storage tier of a key (``tensor="key"``) or value (``"value"``) entry ``age``
        frames old, as ``update_cache`` leaves it (``progressive_quant.py:310-322``): the
        newest entry (age 0) is always full precision."""
        if tensor not in ("key", "value"):
            raise ValueError("tensor must be 'key' or 'value'")
        fp8_age, int4_age = ((self.k_fp8_age, self.k_int4_age) if tensor == "key"
                             else (self.v_fp8_age, self.v_int4_age))
        if age <= 0:
            return "bf16"
        if age >= int4_age:
            return "int4"
        if age >= fp8_age:
            return "fp8"
        return "bf16"

    def slot_kinds(self, n_past: int) -> Tuple[List[str], List[str]]:
        """(key kinds, value kinds) of slots 0..n_past-1, where slot s holds a frame of
        age n_past - s."""
        ages = [n_past - s for s in range(n_past)]
        return ([self.precision_for_age(a, "key") for a in ages],
                [self.precision_for_age(a, "value") for a in ages])


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


class _CacheView:
    """A cache descriptor over part of another cache's slots (same pools)."""

    def __init__(self, base: KVCacheB200, struct: "N.KvCache", slot_kinds, value_kinds):
        self.base, self.struct = base, struct
        self.batch, self.layers = base.batch, base.layers
        self.slot_kinds, self.value_kinds = list(slot_kinds), list(value_kinds)

    @property
    def n_slots(self) -> int:
        return len(self.slot_kinds)


class RollingKVCacheB200(KVCacheB200):
    """A rolling window of at most ``capacity`` cached frames that ages like the
    reference's progressive cache.  Every ``append`` drops the oldest frame once the
    window is full (``manager.py:296-306``), stores the new frame at full precision
    (bf16, age 0), adds one to every older frame's age and promotes, oldest first, the
    keys and the values whose tier changed, each on its own thresholds: bf16 -> FP8,
    bf16 -> INT4 or FP8 -> INT4, the last through the fp16 dequantisation
    (``update_cache``, ``progressive_quant.py:263-350``).

    Keys and values live in per-kind pools sized for a full window (a promotion always
    finds the slot its predecessor freed); logical slots 0 (oldest) .. n_slots-1
    (newest) are remapped on every append, so the object works wherever a
    :class:`KVCacheB200` does (``OasisDiTB200.forward_cached``, ``attn_temporal``,
    ``load``)."""

    def __init__(self, batch: int, layers: int, capacity: int,
                 quantizer: "ProgressiveKVQuantizerB200", device="cuda"):
        if not 1 <= capacity <= N.MAX_FRAMES:
            raise ValueError(f"capacity must be 1..{N.MAX_FRAMES} frames")
        self.batch, self.layers, self.capacity = batch, layers, capacity
        self.quantizer = quantizer
        self.device = torch.device(device)
        self.counts = {}
        for which, tensor in (("k", "key"), ("v", "value")):
            tiers = [quantizer.precision_for_age(a, tensor) for a in range(capacity)]
            self.counts[which] = {N.KV_BF16: tiers.count("bf16"), N.KV_FP8: tiers.count("fp8"),
                                  N.KV_INT4: tiers.count("int4")}
        self._alloc_pools(self.counts["k"], self.counts["v"])
        self._free = {w: {k: list(range(n)) for k, n in self.counts[w].items()} for w in ("k", "v")}
        # oldest first: {"age": a, "k": [kind, index], "v": [kind, index]}
        self.frames: List[Dict[str, Any]] = []
        self._seeded = False
        self._remap()

    # -- logical slots -----------------------------------------------------------------
    def _remap(self) -> None:
        s = self._pool_struct()
        s.n_slots = len(self.frames)
        for i, f in enumerate(self.frames):
            s.k.slot_kind[i], s.k.slot_index[i] = f["k"]
            s.v.slot_kind[i], s.v.slot_index[i] = f["v"]
        self.struct = s
        self.slot_kinds = [_TIER_NAMES[f["k"][0]] for f in self.frames]
        self.value_kinds = [_TIER_NAMES[f["v"][0]] for f in self.frames]

    def frame_slots(self) -> List[Dict[str, Any]]:
        """Every cached frame, oldest first: ``{"age", "key": (kind, pool index),
        "value": (kind, pool index)}``."""
        return [{"age": f["age"], "key": (_TIER_NAMES[f["k"][0]], f["k"][1]),
                 "value": (_TIER_NAMES[f["v"][0]], f["v"][1])} for f in self.frames]

    def _take(self, which: str, kind: int) -> int:
        if not self._free[which][kind]:
            raise RuntimeError("rolling KV cache: no free slot of the promoted kind")
        return self._free[which][kind].pop(0)

    def _promote(self, f: Dict[str, Any], want: Dict[str, int], stream) -> None:
        """One launch re-quantises the frame's keys and/or values into their new kinds:
        logical slot 0 of the pair descriptor is the current storage, slot 1 the new."""
        pair = self._pool_struct()
        pair.n_slots = 2
        mask = 0
        for which, bit in (("k", N.KV_KEYS), ("v", N.KV_VALUES)):
            t = getattr(pair, which)
            t.slot_kind[0], t.slot_index[0] = f[which]
            if which in want:
                mask |= bit
                t.slot_kind[1], t.slot_index[1] = want[which], self._take(which, want[which])
            else:  # not migrated: both slots name its current storage
                t.slot_kind[1], t.slot_index[1] = f[which]
        N.call("oasis_kv_migrate", ctypes.byref(pair), mask, 0, 1, _stream_ptr(stream))
        for which in want:
            self._free[which][f[which][0]].append(f[which][1])
            f[which] = [want[which], getattr(pair, which).slot_index[1]]

    # -- the progressive update ------------------------------------------------------------
    def append(self, rows_per_layer, stream=None) -> None:
        """Add one frame: ``rows_per_layer[layer]`` is that layer's K/V as bf16 rows
        [batch*144][ld] with K in columns 0..1023 and V in 1024..2047, or a
        ``{"key", "value"}`` dict as ``KVCacheManager.update`` takes."""
        if len(rows_per_layer) != self.layers:
            raise ValueError("one entry per layer")
        if len(self.frames) == self.capacity:
            old = self.frames.pop(0)
            for which in ("k", "v"):
                self._free[which][old[which][0]].append(old[which][1])
        seeded, self._seeded = self._seeded, False
        for f in self.frames:  # oldest first
            if seeded:  # seeded frames already carry their ages relative to this frame
                break
            f["age"] += 1
            want = {}
            for which, tensor in (("k", "key"), ("v", "value")):
                kind = KIND_NAMES[self.quantizer.precision_for_age(f["age"], tensor)]
                if _RANK[kind] > _RANK[f[which][0]]:
                    want[which] = kind
            if want:
                self._promote(f, want, stream)
        self.frames.append({"age": 0, "k": [N.KV_BF16, self._take("k", N.KV_BF16)],
                            "v": [N.KV_BF16, self._take("v", N.KV_BF16)]})
        self._remap()
        for layer in range(self.layers):
            rows = rows_per_layer[layer]
            if isinstance(rows, dict):
                rows = _kv_rows(rows)
            self.store(rows, layer, slot0=self.n_slots - 1, k_col=0, v_col=HIDDEN, stream=stream)

    def seed_from(self, cache: KVCacheB200, ages: Sequence[int]) -> None:
        """Start the window from the slots of another cache (e.g. the one a prefill wrote):
        slot s is copied page by page into a slot of the same kinds here.  ``ages[s]`` is
        its age relative to the NEXT appended frame (a prefill of window frames 0..T-2
        for frame T-1: ages T-1..1), so the next ``append`` adds its frame without ageing
        these; their kinds must be the tiers this window gives those ages."""
        if self.frames:
            raise RuntimeError("seed_from needs an empty window")
        # room for the frame the next append adds: at most capacity - 1 seeded frames
        keep = list(range(cache.n_slots))[max(0, cache.n_slots - (self.capacity - 1)):]
        for s in keep:
            f = {"age": int(ages[s])}
            for which, kinds in (("k", cache.slot_kinds), ("v", cache.value_kinds)):
                kind = KIND_NAMES[kinds[s]]
                tensor = "key" if which == "k" else "value"
                if kind != KIND_NAMES[self.quantizer.precision_for_age(f["age"], tensor)]:
                    raise ValueError("seed_from: slot kinds do not follow this window's tiers")
                src_idx = getattr(cache.struct, which).slot_index[s]
                dst_idx = self._take(which, kind)
                for name in {N.KV_BF16: ("bf16",), N.KV_FP8: ("fp8", "fp8_scale"),
                             N.KV_INT4: ("int4", "i4_scale", "i4_zero")}[kind]:
                    getattr(self, f"{which}_{name}")[:, :, dst_idx].copy_(
                        getattr(cache, f"{which}_{name}")[:, :, src_idx])
                f[which] = [kind, dst_idx]
            self.frames.append(f)
        self._seeded = bool(self.frames)
        self._remap()

    def newest(self, n: int) -> _CacheView:
        """A descriptor whose slots 0..n-1 are the newest ``n`` cached frames (oldest
        first): the past frames of a forward whose window holds fewer frames than this
        cache."""
        if not 0 < n <= self.n_slots:
            raise ValueError("newest(n): need 1 <= n <= n_slots")
        s = self._pool_struct()
        s.n_slots = n
        for i, f in enumerate(self.frames[-n:]):
            s.k.slot_kind[i], s.k.slot_index[i] = f["k"]
            s.v.slot_kind[i], s.v.slot_index[i] = f["v"]
        return _CacheView(self, s, self.slot_kinds[-n:], self.value_kinds[-n:])

    # -- snapshot ----------------------------------------------------------------------
    def state(self):
        return ([dict(age=f["age"], k=list(f["k"]), v=list(f["v"])) for f in self.frames],
                {w: {k: list(v) for k, v in d.items()} for w, d in self._free.items()}, self._seeded)

    def set_state(self, st) -> None:
        frames, free, self._seeded = st
        self.frames = [dict(age=f["age"], k=list(f["k"]), v=list(f["v"])) for f in frames]
        self._free = {w: {k: list(v) for k, v in d.items()} for w, d in free.items()}
        self._remap()


class KVCacheManagerB200:
    """The worldserve ``KVCacheManager`` interface over the B200 cache.

    ``update(new_kv, frame_idx)`` appends one frame's post-RoPE K/V (per layer
    ``{"key", "value"}``) to a rolling window of ``max_frames`` frames that ages and
    promotes keys and values on their own thresholds (:class:`RollingKVCacheB200`).
    ``cache_for_window(n_past)`` gives the cache a full-window forward writes (a
    prefill); the next ``update`` continues from it."""

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
        self._ages: List[int] = []  # age of every slot of a prefill cache, oldest first
        self._current_frame_idx: Optional[int] = None
        self._frame_count = 0
        self._step = 0
        self.device = config.get("device", "cuda")

    # -- lifecycle -----------------------------------------------------------------
    def create_cache(self, num_layers: Optional[int] = None, max_frames: Optional[int] = None) -> None:
        """Reset the managed cache (``manager.py:196-240``)."""
        if num_layers is not None:
            self.num_layers = num_layers
        if max_frames is not None:
            self.max_frames = max_frames
        self.cache = None
        self._ages = []
        self._current_frame_idx = None
        self._frame_count = 0
        self._step = 0

    def _quantizer(self) -> ProgressiveKVQuantizerB200:
        # no progressive quantisation: every frame stays full precision
        return self.progressive_quantizer or ProgressiveKVQuantizerB200(
            fp8_age_threshold=10 ** 6, int4_age_threshold=10 ** 6, key_value_asymmetry=False)

    def kinds_for(self, n_past: int) -> Tuple[List[str], List[str]]:
        """(key kinds, value kinds) of a prefill cache of ``n_past`` frames."""
        if self.fixed_kinds is not None:
            k = list(self.fixed_kinds[:n_past])
            return k, list(k)
        return self._quantizer().slot_kinds(n_past)

    def cache_for_window(self, n_past: int) -> KVCacheB200:
        """The cache a full-window forward of ``n_past + 1`` frames writes (prefill):
        slot s holds window frame s, of age ``n_past - s``, in its tier."""
        k_kinds, v_kinds = self.kinds_for(n_past)
        c = self.cache
        if (c is None or isinstance(c, RollingKVCacheB200) or c.slot_kinds != k_kinds
                or c.value_kinds != v_kinds):
            self.cache = KVCacheB200(self.batch, self.num_layers, k_kinds, device=self.device,
                                     value_kinds=v_kinds)
        self._ages = [n_past - s for s in range(n_past)]
        return self.cache

    def set_current_frame_idx(self, frame_idx: int) -> None:
        self._current_frame_idx = int(frame_idx)

    # -- updates / retrieval ----------------------------------------------------------
    def _rolling(self) -> RollingKVCacheB200:
        cap = min(self.max_frames, N.MAX_FRAMES)
        if isinstance(self.cache, RollingKVCacheB200):
            return self.cache
        r = RollingKVCacheB200(self.batch, self.num_layers, cap, self._quantizer(), device=self.device)
        if self.cache is not None and self.fixed_kinds is None:
            # continue from the prefill: its slots already sit in the tiers of their ages
            r.seed_from(self.cache, self._ages)
        self.cache = r
        return r

    def update(self, new_kv: Dict[int, Dict[str, torch.Tensor]], frame_idx: int,
               attention_weights=None) -> None:
        """Append one frame (``manager.py:246-306`` with ``update_cache``,
        ``progressive_quant.py:263-350``): ``new_kv[layer] = {"key", "value"}``, each
        (heads, tokens, head_dim) or (batch, heads, tokens, head_dim) post-RoPE K/V.
        The frame enters at full precision with age 0, older frames age by one and are
        promoted; the window keeps the newest ``max_frames`` frames (at most 32).
        ``attention_weights`` (importance tracking) is accepted and unused: importance
        tracking is off the benchmark path."""
        if len(new_kv) != self.num_layers:
            raise ValueError(f"update: need K/V for all {self.num_layers} layers")
        self._frame_count = frame_idx + 1
        self._rolling().append([new_kv[layer] for layer in range(self.num_layers)])
        self._current_frame_idx = frame_idx

    def append(self, new_kv: Dict[int, Dict[str, torch.Tensor]], frame_idx: int) -> None:
        """Same as :meth:`update`."""
        self.update(new_kv, frame_idx)

    def store_frame(self, new_kv: Dict[int, Dict[str, torch.Tensor]], slot: Optional[int] = None) -> None:
        """Overwrite one slot (default: the newest) of the current cache with given K/V,
        per layer, in that slot's kinds; no ageing."""
        if self.cache is None:
            raise RuntimeError("no cache: call cache_for_window() or update() first")
        s = self.cache.n_slots - 1 if slot is None else slot
        for layer, kv in new_kv.items():
            self.cache.store(_kv_rows(kv), layer, slot0=s, k_col=0, v_col=HIDDEN)

    def past_frames(self, n: Optional[int] = None):
        """The cache to pass as the past of an incremental forward: the newest ``n``
        frames (all when None)."""
        if self.cache is None:
            raise RuntimeError("no cache")
        if n is None or n == self.cache.n_slots:
            return self.cache
        if isinstance(self.cache, RollingKVCacheB200):
            return self.cache.newest(n)
        raise ValueError("past_frames(n) of a prefill cache needs n == n_slots")

    def _heads(self, z: torch.Tensor) -> torch.Tensor:
        """[batch][frames][144][1024] -> (heads, frames*144, d) for one session, else
        (batch, heads, frames*144, d)."""
        B, F = z.shape[:2]
        out = z.reshape(B, F, TOKENS, HEADS, HEAD_DIM).permute(0, 3, 1, 2, 4).reshape(
            B, HEADS, F * TOKENS, HEAD_DIM)
        return out[0] if B == 1 else out

    def get_kv_for_attention(self, layer_idx: int) -> Dict[str, torch.Tensor]:
        """Dequantised K/V of every cached frame, oldest first (``manager.py:416-480``):
        ``(heads, frames*tokens, head_dim)`` bf16 for one session, with a leading batch
        dimension for several."""
        if self.cache is None or self.cache.n_slots == 0:
            return {"key": torch.zeros(0), "value": torch.zeros(0)}
        k, v = self.cache.load(layer_idx)
        return {"key": self._heads(k), "value": self._heads(v)}

    def get_cache(self, precision: str = "fp16") -> Dict[int, Dict[str, torch.Tensor]]:
        """Every layer's cache at a precision tier, as float16 ``(frames, heads, tokens,
        head_dim)`` (with a leading batch dimension for several sessions), like
        ``manager.py:482-553``.  "fp16"/"bf16": the stored frames dequantised.  "fp8" /
        "int4": frames stored finer than that tier are quantised to it (the store
        kernel's FP8 / INT4 arithmetic on their stored values), coarser ones are
        returned as stored."""
        if precision not in ("fp16", "bf16", "fp8", "int4"):
            raise ValueError("precision must be fp16, bf16, fp8 or int4")
        if self.cache is None or self.cache.n_slots == 0:
            return {}
        n = self.cache.n_slots
        target = {"fp16": 0, "bf16": 0, "fp8": 1, "int4": 2}[precision]
        src = self.cache
        if target > 0:
            def coarse(kinds):
                return [_TIER_NAMES[max(target, _RANK[KIND_NAMES[k]])] for k in kinds]
            tmp = KVCacheB200(self.batch, self.num_layers, coarse(src.slot_kinds), device=self.device,
                              value_kinds=coarse(src.value_kinds))
            for layer in range(self.num_layers):
                k, v = src.load(layer)
                rows = torch.cat([k.reshape(-1, HIDDEN), v.reshape(-1, HIDDEN)], dim=1).contiguous()
                tmp.store(rows, layer, slot0=0, k_col=0, v_col=HIDDEN)
            src = tmp
        out = {}
        for layer in range(self.num_layers):
            k, v = src.load(layer)

            def frames(z):
                z = z.reshape(self.batch, n, TOKENS, HEADS, HEAD_DIM).permute(0, 1, 3, 2, 4).to(torch.float16)
                return z[0] if self.batch == 1 else z

            out[layer] = {"key": frames(k), "value": frames(v)}
        return out

    def snapshot(self):
        """Copy of the cache state (pools and slot maps); ``restore`` puts it back."""
        if self.cache is None:
            return None
        st = self.cache.state() if isinstance(self.cache, RollingKVCacheB200) else None
        return {"cache": self.cache, "tensors": [t.clone() for t in self.cache.tensors()],
                "state": st, "ages": list(self._ages)}

    def restore(self, snap) -> None:
        if snap is None:
            return
        self.cache = snap["cache"]
        for dst, src in zip(self.cache.tensors(), snap["tensors"]):
            dst.copy_(src)
        if snap["state"] is not None:
            self.cache.set_state(snap["state"])
        self._ages = list(snap["ages"])

    # -- reporting / hooks ------------------------------------------------------------
    def get_memory_report(self) -> Dict[str, Any]:
        if self.cache is None:
            return {"total_fp16_bytes": 0, "total_actual_bytes": 0, "savings_ratio": 0.0}
        full = self.cache.bf16_equivalent_bytes()
        actual = self.cache.nbytes
        return {"total_fp16_bytes": full, "total_actual_bytes": actual,
                "savings_ratio": 1.0 - actual / max(full, 1),
                "key_kinds": list(self.cache.slot_kinds),
                "value_kinds": list(self.cache.value_kinds)}

    def get_stats(self) -> Dict[str, Any]:
        return self.get_memory_report()

    def pre_step(self, step_idx: int, total_steps: int, latents) -> bool:
        return False

    def post_step(self, step_idx: int, total_steps: int, latents) -> None:
        self._step = step_idx + 1

    def wire_to_model(self, model) -> int:
        """Attach to an ``OasisDiTB200``: from now on every full-window forward of the
        model without an explicit ``kv_cache`` also writes the post-RoPE temporal K/V of
        its past frames into this manager's cache (``cache_for_window``), the analogue of
        the reference's capture at the attention call (``manager.py:923-1138``).
        Returns the number of temporal layers served."""
        model.kv_manager = self
        self.num_layers = model.depth
        return model.depth
