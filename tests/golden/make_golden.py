"""Generate the golden fixtures in this folder by running the REFERENCE's own code.

Run from the repository root in a container that has the reference checkout:

    PYTHONPATH=<reference checkout>:. python tests/golden/make_golden.py [maker ...]

(no argument: every fixture; otherwise only the named makers, e.g. ``update_cache``).

Only this script reads the reference; the fixtures it writes are committed so the
tests (CPU and GPU) never need the reference at run time.  Every fixture is
produced by calling the reference functions named below on seeded inputs:

* ``quant_golden.npz``   — ``ProgressiveKVQuantizer.quantize_to_fp8`` /
  ``dequantize_fp8`` on bf16 (144, 64) frame-head slices and
  ``quantize_to_int4(group_size=64)`` / ``dequantize_int4`` on the same slices,
  plus ``quantize_to_int4`` with its default group of 128 on a ragged flat tensor
  (``worldserve/optimizations/system_level/kv_cache/progressive_quant.py:113-257``).
* ``sampler_golden.npz`` — ``DPMSolverPPSampler(order=1,2,3).step`` sequences
  (``optimizations/model_level/samplers/dpm_solver_pp.py:85-143``) and the DDIM
  v-prediction updates made by ``worldserve.models.oasis.generate`` around a
  deterministic stand-in DiT (``worldserve/models/oasis.py:174-235``).
* ``temporal_attn_golden.npz`` — the reference's restated temporal attention
  ``PersistentTemporalAxialAttention`` (``kv_cache/oasis_temporal_persistent_wrapper.py``)
  built around the oracle's ``TemporalAxialAttention`` weights and RoPE, in full
  and in cached-prefix mode.
* ``cached_past_golden.npz`` — ``attention_with_cached_past``
  (``kv_cache/oasis_persistent_kv_theory.py:97-124``).
* ``promote_golden.npz`` — the age promotions of ``update_cache`` on the same bf16
  slices (``progressive_quant.py:263-350``): ``_promote_to_fp8`` (``quantize_to_fp8``),
  ``_promote_to_int4`` of an FP8 entry (``dequantize_fp8`` with its default fp16 target,
  then ``quantize_to_int4``) and of a full-precision entry (``quantize_to_int4``), with
  the cache's group of 64.
* ``update_cache_golden.npz`` — ``ProgressiveKVQuantizer.update_cache`` itself with
  ``key_value_asymmetry=True`` (values promoted at ``int(0.7 x)`` the key ages,
  ``progressive_quant.py:92-98,263-350``), fed one bf16 (144, 64) key slice and one
  value slice per frame; its INT4 group is set to the cache's 64 (one token-head row),
  the granularity of the benchmark's INT4 cache.  Recorded: every entry's precision
  after every append, and the final codes/scales/zeros of every entry, for thresholds
  (fp8 3, int4 8) over 12 frames and (2, 2) over 5 frames (bf16 -> INT4 directly); and
  the precisions alone for the reference defaults (30, 90) over 40 frames.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from worldserve.optimizations.system_level.kv_cache.progressive_quant import ProgressiveKVQuantizer  # noqa: E402
from worldserve.optimizations.model_level.samplers.dpm_solver_pp import DPMSolverPPSampler  # noqa: E402


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def quant_cases():
    g = torch.Generator().manual_seed(1234)
    xs = []
    for i in range(12):
        xs.append(torch.randn(144, 64, generator=g) * (0.05 * (i + 1)))
    xs.append(torch.zeros(144, 64))                              # all zero
    xs.append(torch.full((144, 64), 0.37))                       # constant
    x = torch.randn(144, 64, generator=g) * 0.01
    x[17, 5] = 40.0                                              # single outlier
    xs.append(x)
    xs.append(torch.randn(144, 64, generator=g) * 1e-6)          # tiny (FP8 subnormals)
    xs.append(torch.randn(144, 64, generator=g) * 300.0)         # large
    x = torch.randn(144, 64, generator=g)
    x[::3] = -x[::3].abs()                                       # skewed rows
    xs.append(x)
    return [z.bfloat16() for z in xs]


def make_quant():
    P = ProgressiveKVQuantizer
    xs = quant_cases()
    inp = np.stack([_bf16_bits(x) for x in xs])
    f8_codes, f8_scale, f8_deq = [], [], []
    i4_packed, i4_scale, i4_zero, i4_deq = [], [], [], []
    for x in xs:
        q, s = P.quantize_to_fp8(x)
        f8_codes.append(q.view(torch.uint8).numpy().copy())
        f8_scale.append(_bf16_bits(s.reshape(1))[0])
        f8_deq.append(_bf16_bits(P.dequantize_fp8(q, s, target_dtype=torch.bfloat16)))
        p, sc, z = P.quantize_to_int4(x, group_size=64)
        i4_packed.append(p.numpy().copy())
        i4_scale.append(sc.numpy().copy())
        i4_zero.append(z.numpy().copy())
        d = P.dequantize_int4(p, sc, z, 64, x.numel(), tuple(x.shape), target_dtype=torch.float32)
        i4_deq.append(d.numpy().copy())
    g = torch.Generator().manual_seed(99)
    flat = (torch.randn(1000, generator=g) * 2.0).bfloat16()     # ragged: pads to 1024
    p, sc, z = P.quantize_to_int4(flat)                          # default group_size=128
    np.savez_compressed(
        os.path.join(HERE, "quant_golden.npz"),
        inp_bf16=inp, fp8_codes=np.stack(f8_codes), fp8_scale_bf16=np.array(f8_scale, np.uint16),
        fp8_deq_bf16=np.stack(f8_deq), int4_packed=np.stack(i4_packed), int4_scale=np.stack(i4_scale),
        int4_zero=np.stack(i4_zero), int4_deq_f32=np.stack(i4_deq),
        flat_bf16=_bf16_bits(flat), flat_packed=p.numpy(), flat_scale=sc.numpy(), flat_zero=z.numpy(),
    )


def make_promote():
    P = ProgressiveKVQuantizer
    xs = quant_cases()
    fp8_codes, fp8_scale, from_fp8, from_full, deq_dtype = [], [], [], [], []
    for x in xs:
        q, s = P.quantize_to_fp8(x)                       # _promote_to_fp8
        fp8_codes.append(q.view(torch.uint8).numpy().copy())
        fp8_scale.append(_bf16_bits(s.reshape(1))[0])
        raw = P.dequantize_fp8(q, s)                      # _promote_to_int4, FP8 entry
        deq_dtype.append(str(raw.dtype))
        p, sc, z = P.quantize_to_int4(raw, group_size=64)
        from_fp8.append((p.numpy().copy(), sc.numpy().copy(), z.numpy().copy()))
        p, sc, z = P.quantize_to_int4(x, group_size=64)   # _promote_to_int4, full precision
        from_full.append((p.numpy().copy(), sc.numpy().copy(), z.numpy().copy()))
    assert len(set(deq_dtype)) == 1, deq_dtype
    np.savez_compressed(
        os.path.join(HERE, "promote_golden.npz"),
        inp_bf16=np.stack([_bf16_bits(x) for x in xs]), fp8_codes=np.stack(fp8_codes),
        fp8_scale_bf16=np.array(fp8_scale, np.uint16), dequant_dtype=np.array(deq_dtype[0]),
        i4_from_fp8_packed=np.stack([a for a, _, _ in from_fp8]),
        i4_from_fp8_scale=np.stack([b for _, b, _ in from_fp8]),
        i4_from_fp8_zero=np.stack([c for _, _, c in from_fp8]),
        i4_from_full_packed=np.stack([a for a, _, _ in from_full]),
        i4_from_full_scale=np.stack([b for _, b, _ in from_full]),
        i4_from_full_zero=np.stack([c for _, _, c in from_full]),
    )


class _StandInDiT:
    """Deterministic stand-in with the DiT call signature; records every call."""

    def __init__(self):
        self.calls = []

    def __call__(self, x, t, actions):
        v = 0.6 * torch.sin(x) - 0.25 * x + (t.float() / 1000.0)[..., None, None, None]
        self.calls.append((x.clone(), t.clone(), v.clone()))
        return v


class _StandInVAE:
    def decode(self, z):
        return z.unsqueeze(1).expand(-1, 3, -1, -1)


def make_sampler():
    out = {}
    g = torch.Generator().manual_seed(7)
    shape = (1, 2, 4, 6, 8)
    for order in (1, 2, 3):
        s = DPMSolverPPSampler(order=order)
        lat = torch.randn(shape, generator=g)
        ts = torch.linspace(1.0, 0.0, 6)
        lats, preds = [lat.numpy().copy()], []
        for i in range(5):
            v = torch.randn(shape, generator=g)
            preds.append(v.numpy().copy())
            lat = s.step(lat, v, ts[i], ts[i + 1])
            lats.append(lat.numpy().copy())
        out[f"ab{order}_latents"] = np.stack(lats)
        out[f"ab{order}_preds"] = np.stack(preds)
        out[f"ab{order}_ts"] = ts.numpy()

    # load models/oasis.py by path: the worldserve.models package __init__ pulls in
    # plotting dependencies that this container lacks
    import importlib.util
    import worldserve
    path = os.path.join(os.path.dirname(worldserve.__file__), "models", "oasis.py")
    spec = importlib.util.spec_from_file_location("_ref_oasis", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    generate = mod.generate
    from oracle.sampler_ref import alphas_cumprod
    ab = torch.from_numpy(alphas_cumprod(1000))
    dit = _StandInDiT()
    model = {"dit": dit, "vae": _StandInVAE(), "device": "cpu", "dtype": torch.float32,
             "alpha_bar_override": ab}
    generate(model, num_frames=2, num_steps=10, n_prompt=1, seed=5)
    out["ddim_x_in"] = np.stack([c[0][:, -1, :2].numpy() for c in dit.calls])  # 2 channels suffice
    out["ddim_t_in"] = np.stack([c[1][:, -1].numpy() for c in dit.calls])
    out["ddim_v"] = np.stack([c[2][:, -1, :2].numpy() for c in dit.calls])
    out["ddim_n_calls"] = np.array(len(dit.calls))
    out["ddim_steps"] = np.array(10)
    out["alphas_cumprod"] = ab.numpy()
    np.savez_compressed(os.path.join(HERE, "sampler_golden.npz"), **out)


def make_temporal_attn():
    from oracle.dit_ref import RotaryEmbedding, TemporalAxialAttention
    from worldserve.optimizations.system_level.kv_cache.oasis_temporal_persistent_wrapper import (
        PersistentTemporalAxialAttention, TemporalPersistentKVRuntime)
    torch.manual_seed(11)
    dim, heads, dh = 128, 2, 64
    rot = RotaryEmbedding(dh)
    base = TemporalAxialAttention(dim, heads, dh, rot, is_causal=True)
    with torch.no_grad():
        for p in base.parameters():
            if p.requires_grad:
                p.normal_(0, 0.05)
    rt = TemporalPersistentKVRuntime()
    ref = PersistentTemporalAxialAttention(base, layer_idx=0, runtime=rt)
    x0 = torch.randn(2, 5, 3, 4, dim)
    x1 = x0.clone()
    x1[:, -1] = torch.randn(2, 3, 4, dim)
    with torch.no_grad():
        y_full = ref(x0)
        rt.enable(True)
        rt.start_frame(4)
        y_step0 = ref(x0)
        rt.set_step(1)
        y_step1 = ref(x1)  # past prefix reused from step 0
    np.savez_compressed(
        os.path.join(HERE, "temporal_attn_golden.npz"),
        w_qkv=base.to_qkv.weight.detach().numpy(), w_out=base.to_out.weight.detach().numpy(),
        b_out=base.to_out.bias.detach().numpy(), x0=x0.numpy(), x1=x1.numpy(),
        y_full=y_full.numpy(), y_step0=y_step0.numpy(), y_step1=y_step1.numpy())


def make_cached_past():
    from worldserve.optimizations.system_level.kv_cache.oasis_persistent_kv_theory import (
        PersistentPastKVCache, attention_with_cached_past)
    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 4, 16, 64, generator=g)
    k = torch.randn(2, 4, 16 + 12, 64, generator=g)
    v = torch.randn(2, 4, 16 + 12, 64, generator=g)
    cache = PersistentPastKVCache()
    cache.start_frame(1)
    y = attention_with_cached_past(q, k, v, 12, cache, 0)
    np.savez_compressed(os.path.join(HERE, "cached_past_golden.npz"),
                        q=q.numpy(), k=k.numpy(), v=v.numpy(), n_past=np.array(12), y=y.numpy())


def _int4_group64(x, group_size=64):
    """The reference quantiser's INT4 at the cache's group of 64 (one token-head row)."""
    return ProgressiveKVQuantizer.quantize_to_int4(x, group_size=64)


UPDATE_CACHE_CONFIGS = (("a", 3, 8, 12), ("b", 2, 2, 5), ("d", 30, 90, 40))
PREC_CODE = {"fp16": 0, "fp8": 1, "int4": 2}


def make_update_cache():
    xs = quant_cases()
    out = {}
    for name, fp8_age, int4_age, n in UPDATE_CACHE_CONFIGS:
        q = ProgressiveKVQuantizer(fp8_age_threshold=fp8_age, int4_age_threshold=int4_age,
                                   key_value_asymmetry=True)
        q.quantize_to_int4 = _int4_group64
        hist = {t: np.full((n, n), -1, np.int8) for t in ("key", "value")}
        for f in range(n):
            if name == "d":  # precisions only: small entries
                k = v = torch.zeros(2, 64).bfloat16()
            else:
                k, v = xs[f % len(xs)], xs[(f + 7) % len(xs)]
            q.update_cache({}, {0: {"key": k, "value": v}}, f)
            for t, entries in (("key", q._cache_k[0]), ("value", q._cache_v[0])):
                hist[t][f, :f + 1] = [PREC_CODE[e.precision] for e in entries]
        for t, entries in (("key", q._cache_k[0]), ("value", q._cache_v[0])):
            out[f"{name}_{t}_hist"] = hist[t]
            if name == "d":
                continue
            fp8_codes = np.zeros((n, 144, 64), np.uint8)
            fp8_scale = np.zeros(n, np.uint16)
            i4_packed = np.zeros((n, 144 * 32), np.uint8)
            i4_scale = np.zeros((n, 144), np.float32)
            i4_zero = np.zeros((n, 144), np.float32)
            for i, e in enumerate(entries):
                if e.precision == "fp8":
                    fp8_codes[i] = e.data.view(torch.uint8).numpy()
                    fp8_scale[i] = _bf16_bits(e.scale.reshape(1))[0]
                elif e.precision == "int4":
                    i4_packed[i] = e.data.numpy()
                    i4_scale[i] = e.scale.numpy()
                    i4_zero[i] = e.zero_point.numpy()
            out.update({f"{name}_{t}_fp8_codes": fp8_codes, f"{name}_{t}_fp8_scale_bf16": fp8_scale,
                        f"{name}_{t}_i4_packed": i4_packed, f"{name}_{t}_i4_scale": i4_scale,
                        f"{name}_{t}_i4_zero": i4_zero})
        out[f"{name}_thresholds"] = np.array([fp8_age, int4_age, n])
    out["inputs"] = np.array("key of frame f: quant_golden inp_bf16[f % 18]; value: inp_bf16[(f + 7) % 18]")
    np.savez_compressed(os.path.join(HERE, "update_cache_golden.npz"), **out)


MAKERS = {"quant": make_quant, "sampler": make_sampler, "temporal_attn": make_temporal_attn,
          "cached_past": make_cached_past, "promote": make_promote, "update_cache": make_update_cache}

if __name__ == "__main__":
    for name in (sys.argv[1:] or list(MAKERS)):
        MAKERS[name]()
    print("golden fixtures written to", HERE)
