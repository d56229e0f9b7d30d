"""CPU-only checks of the host side: the C ABI library loads and exports every symbol
the header declares, argument validation fails cleanly, and the host-computed
constants (RoPE tables, schedule, parameter layout) agree with the oracle."""

import ctypes
import math
import os
import re

import numpy as np
import pytest
import torch

from oracle import sampler_ref
from oracle.dit_ref import DiT, RotaryEmbedding

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "oasis_b200.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(oasis_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol(pkg):
    L = pkg.lib()
    names = header_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), f"{n} declared in oasis_b200.h but not exported"
    # the ctypes signature table covers the same set
    assert sorted(pkg._native.SIGNATURES) == names


def test_version_and_no_error(pkg):
    assert "sm_100a" in pkg.version()
    assert pkg.lib().oasis_last_error() == b""


def test_invalid_arguments_are_reported_not_fatal(pkg):
    L = pkg.lib()
    h = ctypes.c_void_p()
    st = L.oasis_plan_create(None, 1, 4, None, 0, ctypes.byref(h))
    assert st == 1 and b"null" in L.oasis_last_error()
    w = pkg._native.DiTWeights()
    w.depth = 16
    st = L.oasis_plan_create(ctypes.byref(w), 1, 33, None, 0, ctypes.byref(h))
    assert st == 1 and b"frames" in L.oasis_last_error()
    st = L.oasis_plan_create(ctypes.byref(w), 1, 4, None, 0, ctypes.byref(h))
    assert st == 3  # workspace missing
    with pytest.raises(pkg.OasisError):
        pkg._native.check(st)
    st = L.oasis_attn_temporal(ctypes.c_void_p(16), None, 0, ctypes.c_void_p(16), 1, 4, 0, 2, 6, None)
    assert st == 1  # n_past > 0 without a cache
    st = L.oasis_dpmpp2m_update(ctypes.c_void_p(16), ctypes.c_void_p(16), None, 1, 8, 8, 8,
                                0.5, 0.5, 0, None)
    assert st == 1  # multistep without eps_prev


def test_workspace_size_formula(pkg):
    L = pkg.lib()
    ws = L.oasis_plan_workspace_size(1, 32, 16)
    M = 32 * 144
    act = M * 1024 * 4 + M * 1024 * 2 + M * 3072 * 2 + M * 1024 * 2 + M * 4096 * 2 + M * 64 * 2
    mod = 32 * (32 * 6144 + 2048) * 4
    assert act + mod <= ws <= act + mod + 2 * 1024 * 1024
    assert L.oasis_plan_workspace_size(0, 32, 16) == 0


def test_rope_tables_match_oracle_rotary(pkg):
    sp, tp = pkg.rope_tables()
    # spatial: oracle axial frequencies (9, 16, 64) interleaved -> pairs
    rot = RotaryEmbedding(32, freqs_for="pixel", max_freq=256)
    ang = rot.get_axial_freqs(9, 16).reshape(144, 64)[:, 0::2]
    np.testing.assert_array_equal(sp[..., 0].numpy(), ang.cos().numpy())
    np.testing.assert_array_equal(sp[..., 1].numpy(), ang.sin().numpy())
    rt = RotaryEmbedding(64)
    pos = torch.arange(32).float()
    ang_t = RotaryEmbedding._angles(pos, rt.freqs)[:, 0::2]
    np.testing.assert_array_equal(tp[..., 0].numpy(), ang_t.cos().numpy())
    np.testing.assert_array_equal(tp[..., 1].numpy(), ang_t.sin().numpy())


def test_state_dict_loads_into_oracle(pkg):
    sd = pkg.random_state_dict(seed=1, depth=2)
    m = DiT(depth=2)
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected
    assert all(k.endswith("rotary_emb.freqs") for k in missing)
    full = sum(math.prod(s) for s in pkg.param_shapes(16).values())
    assert 600e6 < full < 615e6  # Oasis-500M: ~608M parameters


def test_schedule_matches_oracle(pkg):
    # float64 schedule: the two restatements differ only in how sigmoid is evaluated
    np.testing.assert_allclose(pkg.sigmoid_beta_schedule(1000).numpy(),
                               sampler_ref.sigmoid_beta_schedule(1000), rtol=1e-12, atol=0)
    np.testing.assert_array_equal(pkg.alphas_cumprod().numpy(), sampler_ref.alphas_cumprod(1000))


def test_progressive_policy_matches_reference_thresholds(pkg):
    q = pkg.ProgressiveKVQuantizerB200(fp8_age_threshold=3, int4_age_threshold=10,
                                       key_value_asymmetry=True)
    assert (q.v_fp8_age, q.v_int4_age) == (2, 7)  # int(0.7 * threshold), progressive_quant.py:93-95
    keys, values = q.slot_kinds(12)  # slot s holds a frame of age 12 - s
    # keys: INT4 at ages 12..10, FP8 at 9..3, bf16 at 2..1; values: INT4 at 12..7, FP8 at 6..2
    assert keys == ["int4"] * 3 + ["fp8"] * 7 + ["bf16"] * 2
    assert values == ["int4"] * 6 + ["fp8"] * 5 + ["bf16"]
    assert q.precision_for_age(0, "value") == "bf16"  # a new entry is always full precision
    sym = pkg.ProgressiveKVQuantizerB200(fp8_age_threshold=3, int4_age_threshold=10,
                                         key_value_asymmetry=False)
    assert sym.slot_kinds(12)[0] == sym.slot_kinds(12)[1] == keys


def test_rolling_pool_sizes_follow_each_tensors_tiers(pkg):
    """A full window of 32 frames at the reference defaults: keys FP8 from age 30 (2
    frames), values FP8 from age 21 (11 frames); bf16 the rest, the newest frame included
    (pool sizes of the rolling cache)."""
    q = pkg.ProgressiveKVQuantizerB200()
    counts = {}
    for tensor in ("key", "value"):
        tiers = [q.precision_for_age(a, tensor) for a in range(32)]
        counts[tensor] = (tiers.count("bf16"), tiers.count("fp8"), tiers.count("int4"))
    assert counts == {"key": (30, 2, 0), "value": (21, 11, 0)}


def test_kv_struct_layout_matches_header(pkg):
    """The ctypes mirror of oasis_kv_tensor_t / oasis_kv_cache_t has the C layout: one
    slot map and six pool pointers per tensor, keys then values."""
    import ctypes
    N = pkg._native
    assert ctypes.sizeof(N.KvTensor) == 128
    assert (N.KvCache.k.offset, N.KvCache.v.offset, ctypes.sizeof(N.KvCache)) == (16, 144, 272)


def test_action_step_schedule_buckets(pkg):
    """steps(i) = 2 if ||a_i||_1 < 0.5, 3 if < 1.5, else 5 (the reference's bucket
    function, oasis_difficulty_dpmpp_modal.py:95-101; report eq. 'bucket')."""
    f = pkg.steps_for_action_magnitude
    assert [f(m) for m in (0.0, 0.49, 0.5, 1.49, 1.5, 7.0)] == [2, 2, 3, 3, 5, 5]
    assert f(0.7, lo_threshold=1.0, reduced_steps=1) == 1
    a = torch.zeros(2, 4, 25)
    a[0, 1, 0] = 1.0           # moderate
    a[0, 2, :3] = 1.0          # active (L1 = 3)
    a[0, 3, 23:] = -0.2        # camera only, idle (L1 = 0.4)
    a[1] = 9.0                 # other sessions do not change the schedule
    assert pkg.action_step_schedule(a) == [2, 3, 5, 2]


def test_vae_oracle_shapes_and_names(pkg):
    """The package's decoder parameters are the oracle's, and the oracle decodes
    (frames, 576, 16) latents into (frames, 3, 360, 640) frames."""
    from oracle import vae_ref
    sd = pkg.random_vae_state_dict(seed=0, depth=1)
    assert {k: tuple(v.shape) for k, v in sd.items()} == vae_ref.param_shapes(1)
    assert torch.allclose(pkg.vae.vae_rope_table(), vae_ref.rope_table())
    out = vae_ref.decode(sd, torch.randn(2, 576, 16), depth=1)
    assert out.shape == (2, 3, 360, 640) and torch.isfinite(out).all()
    assert pkg.lib().oasis_vae_workspace_size(1, 12) > 0
    assert pkg.lib().oasis_vae_workspace_size(1, 13) == 0


def test_vae_invalid_arguments_are_reported_not_fatal(pkg):
    L = pkg.lib()
    h = ctypes.c_void_p()
    assert L.oasis_vae_plan_create(None, 1, None, 0, ctypes.byref(h)) == 1
    w = pkg._native.VaeWeights()
    w.depth = 12
    assert L.oasis_vae_plan_create(ctypes.byref(w), 0, ctypes.c_void_p(256), 1 << 30, ctypes.byref(h)) == 1
    assert b"frames" in L.oasis_last_error()
    w.depth = 13
    assert L.oasis_vae_plan_create(ctypes.byref(w), 1, ctypes.c_void_p(256), 1 << 30, ctypes.byref(h)) == 1
    w.depth = 12
    need = L.oasis_vae_workspace_size(1, 12)
    assert L.oasis_vae_plan_create(ctypes.byref(w), 1, ctypes.c_void_p(256), need - 1, ctypes.byref(h)) == 3
    assert L.oasis_vae_decode(None, ctypes.c_void_p(16), ctypes.c_void_p(16), None) == 1
    assert not h.value  # no plan was handed out
