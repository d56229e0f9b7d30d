"""numpy restatement of the reference's progressive KV quantiser — TEST INFRASTRUCTURE ONLY.

Follows ``worldserve/optimizations/system_level/kv_cache/progressive_quant.py``:

* ``quantize_to_fp8``  (:113-138) per-tensor absmax scale, ``scale = amax.clamp(1e-12) / 448``,
  ``q = (x / scale).to(float8_e4m3fn)``.  With a bf16 input every step runs in bf16
  the way PyTorch's CPU kernels do it: the division is done in fp32 and rounded
  to bf16 (round-to-nearest-even), and the bf16 quotient is then rounded to
  e4m3fn (RNE; magnitudes above 464 become NaN, 464 itself ties to 448).
* ``quantize_to_int4`` (:140-193) group-wise asymmetric min/max in fp32:
  ``scale = (max - min).clamp(1e-12) / 15``, ``zero = min``,
  ``q = round((x - zero) / scale).clamp(0, 15)`` (round half to even); packed
  two codes per byte, element ``2i`` in the HIGH nibble, ``2i+1`` in the low one.
* ``dequantize_fp8`` (:195-212) ``q.to(dtype) * scale`` and ``dequantize_int4``
  (:214-257) ``q * scale + zero`` in the target dtype.

The granularity used by the B200 cache (one FP8 scale per frame-head slice of
144 x 64, one INT4 group per token-head row of 64) is obtained by calling these
per slice / with ``group_size=64``, exactly as the reference functions would be
called on those tensors.
"""

from __future__ import annotations

import numpy as np

FP8_MAX = 448.0


# ---------------------------------------------------------------- bf16 / fp16

def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); returns float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    out = b.astype(np.uint32).view(np.float32)
    return np.where(nan, np.float32(np.nan), out)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) of float32 values that are already bf16-exact."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- e4m3fn

def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn codes (uint8) with round-to-nearest-even."""
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    sign = np.signbit(x).astype(np.uint8) << 7
    a = np.abs(x)
    code = np.zeros(a.shape, dtype=np.int64)
    sub = a < 2.0 ** -6
    code[sub] = np.rint(a[sub] / 2.0 ** -9).astype(np.int64)  # 0..8 (8 == min normal)
    nrm = ~sub & np.isfinite(a)
    if np.any(nrm):
        an = a[nrm]
        e = np.floor(np.log2(an)).astype(np.int64)
        # guard log2 rounding at exact powers of two
        e = np.where(an < 2.0 ** e, e - 1, e)
        e = np.where(an >= 2.0 ** (e + 1), e + 1, e)
        m = np.rint((an / 2.0 ** e - 1.0) * 8.0).astype(np.int64)
        carry = m == 8
        e = np.where(carry, e + 1, e)
        m = np.where(carry, 0, m)
        code[nrm] = ((e + 7) << 3) | m
    code = np.where(np.isfinite(a) & (code <= 0x7E), code, 0x7F)
    return (code.astype(np.uint8) | sign).astype(np.uint8)


def e4m3_decode(code: np.ndarray) -> np.ndarray:
    code = np.asarray(code, dtype=np.uint8)
    sign = np.where(code & 0x80, -1.0, 1.0)
    e = (code >> 3) & 0xF
    m = (code & 0x7).astype(np.float64)
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * 2.0 ** (e.astype(np.float64) - 7))
    val = np.where((code & 0x7F) == 0x7F, np.nan, val)
    return (sign * val).astype(np.float32)


# ---------------------------------------------------------------- FP8 (bf16 input)

def quantize_to_fp8_bf16(x: np.ndarray):
    """Per-tensor FP8 quantisation of a bf16-valued array (given as float32).

    Returns ``(codes uint8, scale float32 holding a bf16 value)``.
    """
    x = np.asarray(x, dtype=np.float32)
    amax = np.float32(np.max(np.abs(x))) if x.size else np.float32(0.0)
    amax = max(amax, bf16_round(np.float32(1e-12)).item())
    scale = bf16_round(np.float32(np.float32(amax) / np.float32(FP8_MAX)))
    scaled = bf16_round((x / scale).astype(np.float32))
    return e4m3_encode(scaled), np.float32(scale)


def dequantize_fp8_bf16(codes: np.ndarray, scale) -> np.ndarray:
    return bf16_round((e4m3_decode(codes) * np.float32(scale)).astype(np.float32))


# ---------------------------------------------------------------- INT4

def quantize_to_int4(x: np.ndarray, group_size: int = 128):
    """Group-wise asymmetric INT4; returns ``(packed uint8, scale f32, zero f32)``."""
    flat = np.asarray(x, dtype=np.float32).reshape(-1)
    pad = (group_size - flat.size % group_size) % group_size
    if pad:
        flat = np.concatenate([flat, np.zeros(pad, np.float32)])
    g = flat.reshape(-1, group_size)
    gmin = g.min(axis=1)
    gmax = g.max(axis=1)
    scale = np.maximum(gmax - gmin, np.float32(1e-12)).astype(np.float32) / np.float32(15.0)
    scale = scale.astype(np.float32)
    zero = gmin
    q = ((g - zero[:, None]) / scale[:, None]).astype(np.float32)
    q = np.clip(np.rint(q), 0, 15).astype(np.uint8).reshape(-1)
    if q.size % 2:
        q = np.concatenate([q, np.zeros(1, np.uint8)])
    packed = ((q[0::2] << 4) | q[1::2]).astype(np.uint8)
    return packed, scale, zero


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    return np.stack([packed >> 4, packed & 0xF], axis=-1).reshape(-1)


def dequantize_int4(packed, scale, zero, group_size: int, numel: int) -> np.ndarray:
    """Float32 dequantisation ``q * scale + zero`` (target dtype float32)."""
    q = unpack_int4(packed)[: scale.size * group_size].reshape(-1, group_size).astype(np.float32)
    out = q * np.asarray(scale, np.float32)[:, None] + np.asarray(zero, np.float32)[:, None]
    return out.reshape(-1)[:numel]


# ---------------------------------------------------------------- cache-granularity helpers

def quantize_fp8_slices(kv: np.ndarray):
    """FP8 with one scale per ``(..., tokens, 64)`` slice: kv shape ``(S, tokens, 64)``."""
    codes = np.empty(kv.shape, np.uint8)
    scales = np.empty(kv.shape[0], np.float32)
    for s in range(kv.shape[0]):
        codes[s], scales[s] = quantize_to_fp8_bf16(kv[s])
    return codes, scales


def quantize_int4_rows(kv: np.ndarray):
    """INT4 with one group per 64-element row: kv ``(..., 64)`` -> packed ``(..., 32)``,
    fp16 scale/zero ``(...)`` (codes computed from the fp32 scale/zero)."""
    lead = kv.shape[:-1]
    packed, scale, zero = quantize_to_int4(kv.reshape(-1), group_size=kv.shape[-1])
    return (packed.reshape(*lead, kv.shape[-1] // 2),
            scale.astype(np.float16).reshape(lead), zero.astype(np.float16).reshape(lead),
            scale.reshape(lead), zero.reshape(lead))


# ---------------------------------------------------------------- age promotions

def promote_fp8_to_int4_rows(codes: np.ndarray, scale) -> tuple:
    """``_promote_to_int4`` of an FP8 entry (progressive_quant.py:334-350): the codes are
    dequantised with ``dequantize_fp8``'s default fp16 target, i.e. fp16(e4m3 x scale)
    with the product exact in fp32 and rounded once (RNE), and those values are quantised
    like ``quantize_int4_rows`` (one group per 64-element row)."""
    x = (e4m3_decode(codes) * np.float32(scale)).astype(np.float32)
    x16 = x.astype(np.float16).astype(np.float32)
    return quantize_int4_rows(x16)



# ---------------------------------------------------------------- update_cache

class UpdateCacheRef:
    """``ProgressiveKVQuantizer.update_cache`` (progressive_quant.py:263-350) for one
    stream of cache entries at the B200 cache's granularity (one 144 x 64 frame-head
    slice per append; FP8 one scale per slice, INT4 one group per 64-element row).

    Keys drop to FP8 at ``fp8_age`` and to INT4 at ``int4_age``; with
    ``key_value_asymmetry`` the values use ``int(0.7 x)`` those ages (:92-98).  Each
    append adds the new entries at full precision (age 0), then ages every older entry
    by one and promotes it, oldest first: ``age >= int4_age`` and not INT4 -> INT4 (from
    the entry's FP8 codes through the fp16 dequantisation, or from its full-precision
    values); otherwise ``age >= fp8_age`` and full precision -> FP8.  ``window`` keeps
    only the newest entries, as ``KVCacheManager.update`` trims its cache (manager.py:
    296-306)."""

    def __init__(self, fp8_age: int = 30, int4_age: int = 90, key_value_asymmetry: bool = True,
                 window: int = 0):
        self.thr = {"key": (fp8_age, int4_age)}
        if key_value_asymmetry:
            self.thr["value"] = (int(fp8_age * 0.7), int(int4_age * 0.7))
        else:
            self.thr["value"] = (fp8_age, int4_age)
        self.window = window
        self.entries = {"key": [], "value": []}
        self.ages = []

    def append(self, key: np.ndarray, value: np.ndarray) -> None:
        for t, x in (("key", key), ("value", value)):
            self.entries[t].append({"precision": "fp16", "x": np.asarray(x, np.float32).copy()})
        self.ages.append(0)
        for i in range(len(self.ages) - 1):
            self.ages[i] += 1
            for t in ("key", "value"):
                fp8_age, int4_age = self.thr[t]
                e = self.entries[t][i]
                if self.ages[i] >= int4_age and e["precision"] != "int4":
                    if e["precision"] == "fp8":
                        p, s16, z16, s, z = promote_fp8_to_int4_rows(e["codes"], e["scale"])
                    else:
                        p, s16, z16, s, z = quantize_int4_rows(e["x"])
                    e.update(precision="int4", packed=p, scale16=s16, zero16=z16, scale=s, zero=z)
                elif self.ages[i] >= fp8_age and e["precision"] == "fp16":
                    codes, scale = quantize_to_fp8_bf16(e["x"])
                    e.update(precision="fp8", codes=codes, scale=scale)
        if self.window and len(self.ages) > self.window:
            drop = len(self.ages) - self.window
            self.ages = self.ages[drop:]
            for t in ("key", "value"):
                self.entries[t] = self.entries[t][drop:]

    def precisions(self, tensor: str):
        return [e["precision"] for e in self.entries[tensor]]
