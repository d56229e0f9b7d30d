"""Pin the CPU oracle against fixtures produced by the reference's own code.

The fixtures in ``tests/golden`` were written by ``tests/golden/make_golden.py``
running the reference functions; these tests need no GPU and no reference checkout.
"""

import os

import numpy as np
import pytest
import torch

from oracle import quant_ref, sampler_ref
from oracle.dit_ref import RotaryEmbedding, TemporalAxialAttention

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


# ----------------------------------------------------------------- quantiser

def test_fp8_codes_and_scales_bit_exact():
    g = _load("quant_golden.npz")
    for i in range(g["inp_bf16"].shape[0]):
        x = quant_ref.bf16_from_bits(g["inp_bf16"][i])
        codes, scale = quant_ref.quantize_to_fp8_bf16(x)
        assert quant_ref.bf16_bits(np.float32(scale)) == g["fp8_scale_bf16"][i], i
        np.testing.assert_array_equal(codes, g["fp8_codes"][i], err_msg=f"case {i}")
        deq = quant_ref.dequantize_fp8_bf16(codes, scale)
        np.testing.assert_array_equal(quant_ref.bf16_bits(deq), g["fp8_deq_bf16"][i])


def test_int4_group64_bit_exact():
    g = _load("quant_golden.npz")
    for i in range(g["inp_bf16"].shape[0]):
        x = quant_ref.bf16_from_bits(g["inp_bf16"][i])
        packed, scale, zero = quant_ref.quantize_to_int4(x, group_size=64)
        np.testing.assert_array_equal(packed, g["int4_packed"][i], err_msg=f"case {i}")
        np.testing.assert_array_equal(scale.view(np.uint32), g["int4_scale"][i].view(np.uint32))
        np.testing.assert_array_equal(zero.view(np.uint32), g["int4_zero"][i].view(np.uint32))
        deq = quant_ref.dequantize_int4(packed, scale, zero, 64, x.size)
        np.testing.assert_array_equal(deq, g["int4_deq_f32"][i].reshape(-1))


def test_int4_default_group_ragged_bit_exact():
    g = _load("quant_golden.npz")
    x = quant_ref.bf16_from_bits(g["flat_bf16"])
    packed, scale, zero = quant_ref.quantize_to_int4(x)  # group 128, padded 1000 -> 1024
    np.testing.assert_array_equal(packed, g["flat_packed"])
    np.testing.assert_array_equal(scale, g["flat_scale"])
    np.testing.assert_array_equal(zero, g["flat_zero"])


def test_age_promotions_bit_exact():
    """bf16 -> FP8, FP8 -> INT4 (via the fp16 dequantisation) and bf16 -> INT4, as the
    reference's update_cache promotes entries, on the cache's 64-element groups."""
    g = _load("promote_golden.npz")
    assert str(g["dequant_dtype"]) == "torch.float16"
    xs = quant_ref.bf16_from_bits(g["inp_bf16"])
    for i in range(xs.shape[0]):
        codes, scale = quant_ref.quantize_to_fp8_bf16(xs[i])
        np.testing.assert_array_equal(codes, g["fp8_codes"][i])
        assert quant_ref.bf16_bits(np.array([scale], np.float32))[0] == g["fp8_scale_bf16"][i]
        p, _, _, s32, z32 = quant_ref.promote_fp8_to_int4_rows(codes, scale)
        np.testing.assert_array_equal(p.reshape(-1), g["i4_from_fp8_packed"][i])
        np.testing.assert_array_equal(s32, g["i4_from_fp8_scale"][i])
        np.testing.assert_array_equal(z32, g["i4_from_fp8_zero"][i])
        p, _, _, s32, z32 = quant_ref.quantize_int4_rows(xs[i])
        np.testing.assert_array_equal(p.reshape(-1), g["i4_from_full_packed"][i])
        np.testing.assert_array_equal(s32, g["i4_from_full_scale"][i])
        np.testing.assert_array_equal(z32, g["i4_from_full_zero"][i])


def test_e4m3_encoder_matches_torch_on_all_bf16_magnitudes():
    # every bf16 value in the e4m3 range and beyond, both signs
    bits = np.arange(0, 0x7F80, dtype=np.uint32)
    x = quant_ref.bf16_from_bits(bits)
    x = np.concatenate([x, -x])
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = quant_ref.e4m3_encode(x)
    nan_w = (want & 0x7F) == 0x7F
    nan_g = (got & 0x7F) == 0x7F
    np.testing.assert_array_equal(nan_w, nan_g)
    np.testing.assert_array_equal(got[~nan_w], want[~nan_w])


def test_bf16_round_matches_torch():
    x = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 37.0
    want = torch.from_numpy(x).bfloat16().float().numpy()
    np.testing.assert_array_equal(quant_ref.bf16_round(x), want)


# ----------------------------------------------------------------- samplers

@pytest.mark.parametrize("order", [1, 2, 3])
def test_ab_sampler_matches_reference(order):
    g = _load("sampler_golden.npz")
    lats, preds, ts = g[f"ab{order}_latents"], g[f"ab{order}_preds"], g[f"ab{order}_ts"]
    x, hist = lats[0], []
    for i in range(preds.shape[0]):
        h = float(np.float32(ts[i + 1]) - np.float32(ts[i]))
        x = sampler_ref.ab_step(x, preds[i], hist, h, order)
        hist.append(preds[i])
        np.testing.assert_allclose(x, lats[i + 1], rtol=1e-5, atol=1e-5)
        x = lats[i + 1]


def test_ddim_update_matches_reference_generate():
    g = _load("sampler_golden.npz")
    ab = g["alphas_cumprod"]
    np.testing.assert_allclose(ab, sampler_ref.alphas_cumprod(1000), rtol=0, atol=0)
    steps = int(g["ddim_steps"])
    nr = np.linspace(-1, 999, steps + 1, dtype=np.float32)
    xin, v = g["ddim_x_in"], g["ddim_v"]
    n = int(g["ddim_n_calls"])
    k = 0
    for frame in range(n // steps):
        for j, idx in enumerate(reversed(range(1, steps + 1))):
            t = int(np.clip(int(nr[idx]), 0, 999))
            tp = max(int(nr[idx - 1]), 0)
            assert int(g["ddim_t_in"][k].reshape(-1)[0]) == t
            if j < steps - 1:  # the next call sees the updated chunk
                want = xin[k + 1]
                got = sampler_ref.ddim_vpred_step(xin[k], v[k], float(ab[t]), float(ab[tp]))
                np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
            k += 1


def test_dpmpp_noise_levels():
    lv = sampler_ref.dpmpp_noise_levels(5)
    assert [a for a, _, _ in lv] == [999, 799, 599, 399, 199]
    assert [b for _, b, _ in lv] == [799, 599, 399, 199, 199]
    assert [f for _, _, f in lv] == [False, False, False, False, True]


# ----------------------------------------------------------------- attention structure

def _temporal_from_golden(g):
    dim, heads, dh = 128, 2, 64
    m = TemporalAxialAttention(dim, heads, dh, RotaryEmbedding(dh), is_causal=True)
    with torch.no_grad():
        m.to_qkv.weight.copy_(torch.from_numpy(g["w_qkv"]))
        m.to_out.weight.copy_(torch.from_numpy(g["w_out"]))
        m.to_out.bias.copy_(torch.from_numpy(g["b_out"]))
    return m


def test_temporal_attention_matches_reference_wrapper():
    g = _load("temporal_attn_golden.npz")
    m = _temporal_from_golden(g)
    with torch.no_grad():
        y = m(torch.from_numpy(g["x0"]))
    np.testing.assert_allclose(y.numpy(), g["y_full"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(y.numpy(), g["y_step0"], rtol=1e-5, atol=1e-6)


def test_temporal_attention_cached_prefix_matches_reference_wrapper():
    """Step>0 of the reference wrapper reuses the step-0 past q/k/v projections."""
    g = _load("temporal_attn_golden.npz")
    m = _temporal_from_golden(g)
    x0, x1 = torch.from_numpy(g["x0"]), torch.from_numpy(g["x1"])
    with torch.no_grad():
        q0, k0, v0 = m.to_qkv(x0).chunk(3, dim=-1)
        q1, k1, v1 = m.to_qkv(x1[:, -1:]).chunk(3, dim=-1)
        qkv = torch.cat([torch.cat([q0[:, :-1], q1], 1), torch.cat([k0[:, :-1], k1], 1),
                         torch.cat([v0[:, :-1], v1], 1)], dim=-1)
        # run the module's post-projection path on the mixed projections
        B, T, H, W, _ = x0.shape
        q, k, v = qkv.chunk(3, dim=-1)

        def seq(z):
            return z.reshape(B, T, H, W, 2, 64).permute(0, 2, 3, 4, 1, 5).reshape(B * H * W, 2, T, 64)

        q, k, v = seq(q), seq(k), seq(v)
        q = m.rotary_emb.rotate_queries_or_keys(q, m.rotary_emb.freqs)
        k = m.rotary_emb.rotate_queries_or_keys(k, m.rotary_emb.freqs)
        o = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
        y = m.finish(o, B, H, W)
    np.testing.assert_allclose(y.numpy(), g["y_step1"], rtol=1e-5, atol=1e-6)


def test_cached_past_attention_equals_reference():
    g = _load("cached_past_golden.npz")
    q, k, v = (torch.from_numpy(g[n]) for n in ("q", "k", "v"))
    y = torch.nn.functional.scaled_dot_product_attention(q, k, v)
    np.testing.assert_allclose(y.numpy(), g["y"], rtol=0, atol=1e-6)


# ----------------------------------------------------------------- update_cache (asymmetric)

PREC = {0: "fp16", 1: "fp8", 2: "int4"}


@pytest.mark.parametrize("name", ["a", "b", "d"])
def test_update_cache_oracle_matches_reference_asymmetric(name):
    """The oracle's update_cache, with the reference default key_value_asymmetry=True,
    against the reference's own update_cache: every entry's precision after every
    append, and (configs a, b) the final FP8 codes/scales and INT4 codes/scales/zeros."""
    g = np.load(os.path.join(GOLD, "update_cache_golden.npz"))
    xs = np.load(os.path.join(GOLD, "quant_golden.npz"))["inp_bf16"]
    fp8_age, int4_age, n = (int(v) for v in g[f"{name}_thresholds"])
    ref = quant_ref.UpdateCacheRef(fp8_age, int4_age, key_value_asymmetry=True)
    for f in range(n):
        if name == "d":
            k = v = np.zeros((2, 64), np.float32)
        else:
            k = quant_ref.bf16_from_bits(xs[f % len(xs)])
            v = quant_ref.bf16_from_bits(xs[(f + 7) % len(xs)])
        ref.append(k, v)
        for t in ("key", "value"):
            want = [PREC[int(c)] for c in g[f"{name}_{t}_hist"][f, :f + 1]]
            assert ref.precisions(t) == want, (name, f, t)
    if name == "d":
        return
    for t in ("key", "value"):
        for i, e in enumerate(ref.entries[t]):
            if e["precision"] == "fp8":
                np.testing.assert_array_equal(e["codes"], g[f"{name}_{t}_fp8_codes"][i])
                assert quant_ref.bf16_bits(np.float32(e["scale"])) == g[f"{name}_{t}_fp8_scale_bf16"][i]
            elif e["precision"] == "int4":
                np.testing.assert_array_equal(e["packed"].reshape(-1), g[f"{name}_{t}_i4_packed"][i])
                np.testing.assert_array_equal(e["scale"], g[f"{name}_{t}_i4_scale"][i])
                np.testing.assert_array_equal(e["zero"], g[f"{name}_{t}_i4_zero"][i])
