"""KV-cache manager interface (the worldserve method names and behaviour) over the B200
cache, with keys and values tiered on their own thresholds."""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_manager_prefill_retrieve_store_snapshot(pkg, cuda):
    depth, B, T = 2, 2, 5
    model = pkg.OasisDiTB200.random(seed=4, depth=depth, device=cuda)
    mgr = pkg.KVCacheManagerB200({"num_layers": depth, "batch": B,
                                  "progressive_quant": {"fp8_age_threshold": 3,
                                                        "int4_age_threshold": 4}})
    assert mgr.wire_to_model(model) == depth
    cache = mgr.cache_for_window(T - 1)
    # ages 4, 3, 2, 1: keys at the thresholds (FP8 3, INT4 4), values at int(0.7 x) = 2, 2
    assert cache.slot_kinds == ["int4", "fp8", "bf16", "bf16"]
    assert cache.value_kinds == ["int4", "int4", "int4", "bf16"]
    g = torch.Generator().manual_seed(0)
    x = torch.randn(B, T, 16, 18, 32, generator=g).to(cuda)
    t = torch.randint(0, 1000, (B, T), generator=g).to(cuda)
    model(x, t, None)  # wired: the forward writes its past frames into the manager's cache
    kv = mgr.get_kv_for_attention(1)
    assert kv["key"].shape == (B, 16, (T - 1) * 144, 64)
    assert torch.isfinite(kv["key"].float()).all() and kv["key"].abs().sum() > 0
    snap = mgr.snapshot()
    # store_frame(): overwrite the newest slot of layer 0 with given K/V, then restore
    k = torch.randn(B, 16, 144, 64, device=cuda).bfloat16()
    mgr.store_frame({0: {"key": k, "value": k}})
    got = mgr.get_kv_for_attention(0)["key"][:, :, -144:]
    assert torch.equal(got, k)  # bf16 slot stores exactly
    mgr.restore(snap)
    assert not torch.equal(mgr.get_kv_for_attention(0)["key"][:, :, -144:], k)
    rep = mgr.get_memory_report()
    assert 0.0 < rep["savings_ratio"] < 1.0
    assert rep["value_kinds"] == ["int4", "int4", "int4", "bf16"]


def _frame_rows(B, layers, seed, cuda):
    """One frame's K/V rows per layer: bf16 [B*144][K 1024 | V 1024], per-head scales
    spread over three decades so the FP8 scales differ."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(layers):
        z = torch.randn(B * 144, 2048, generator=g)
        z = z * (10.0 ** torch.empty(1, 32).uniform_(-2, 1, generator=g)).repeat_interleave(64, 1)
        out.append(z.bfloat16().to(cuda))
    return out


def _check_entry(cache, which, kind, idx, b, layer, h, e):
    """Stored codes of one (session, layer, head) slice of a cached frame == an oracle
    or fixture entry ``e`` (precision fp16/fp8/int4 with its payload)."""
    if kind == "bf16":
        assert e["precision"] == "fp16"
        got = getattr(cache, which + "_bf16")[b, layer, idx][:, h * 64:(h + 1) * 64].float().cpu().numpy()
        np.testing.assert_array_equal(got, e["x"])
    elif kind == "fp8":
        assert e["precision"] == "fp8"
        got = getattr(cache, which + "_fp8")[b, layer, idx][:, h * 64:(h + 1) * 64].cpu().numpy()
        np.testing.assert_array_equal(got, e["codes"])
        gs = getattr(cache, which + "_fp8_scale")[b, layer, idx, h].float().item()
        assert gs == float(e["scale"])
    else:
        assert e["precision"] == "int4"
        got = getattr(cache, which + "_int4")[b, layer, idx, :, h].cpu().numpy()
        np.testing.assert_array_equal(got, e["packed"].reshape(144, 32))
        gsc = getattr(cache, which + "_i4_scale")[b, layer, idx, :, h].cpu().numpy()
        gz = getattr(cache, which + "_i4_zero")[b, layer, idx, :, h].cpu().numpy()
        np.testing.assert_array_equal(gsc, np.asarray(e["scale"], np.float32).astype(np.float16))
        np.testing.assert_array_equal(gz, np.asarray(e["zero"], np.float32).astype(np.float16))


@pytest.mark.parametrize("name", ["a", "b"])
def test_rolling_cache_matches_reference_update_cache_asymmetric(pkg, cuda, name):
    """Keys and values each age and promote on their own thresholds, as the reference's
    own update_cache does with its default key_value_asymmetry=True: after every append
    each cached frame's key and value kinds equal the reference's precision history, and
    after the last append every stored code, scale and zero equals the reference's
    (tests/golden/update_cache_golden.npz; every head of every session and layer holds
    the fixture's slice of that frame)."""
    from oracle import quant_ref as Q
    g = np.load(os.path.join(GOLD, "update_cache_golden.npz"))
    xs = np.load(os.path.join(GOLD, "quant_golden.npz"))["inp_bf16"]
    fp8_age, int4_age, n = (int(v) for v in g[f"{name}_thresholds"])
    B, L = 2, 2
    q = pkg.ProgressiveKVQuantizerB200(fp8_age_threshold=fp8_age, int4_age_threshold=int4_age,
                                       key_value_asymmetry=True)
    cache = pkg.RollingKVCacheB200(B, L, n, q, device=cuda)
    names = {0: "bf16", 1: "fp8", 2: "int4"}
    raw = {}
    for f in range(n):
        k = Q.bf16_from_bits(xs[f % len(xs)])
        v = Q.bf16_from_bits(xs[(f + 7) % len(xs)])
        raw[f] = (k, v)
        row = torch.from_numpy(np.concatenate([np.tile(k, (1, 16)), np.tile(v, (1, 16))], axis=1))
        rows = [row.repeat(B, 1).bfloat16().to(cuda).contiguous() for _ in range(L)]
        cache.append(rows)
        assert cache.slot_kinds == [names[int(c)] for c in g[f"{name}_key_hist"][f, :f + 1]], f
        assert cache.value_kinds == [names[int(c)] for c in g[f"{name}_value_hist"][f, :f + 1]], f
    torch.cuda.synchronize()
    prec = {0: "fp16", 1: "fp8", 2: "int4"}
    for i, fr in enumerate(cache.frame_slots()):
        for which, tensor, col in (("k", "key", 0), ("v", "value", 1)):
            p = prec[int(g[f"{name}_{tensor}_hist"][n - 1, i])]
            e = {"precision": p, "x": raw[i][col]}
            if p == "fp8":
                e.update(codes=g[f"{name}_{tensor}_fp8_codes"][i],
                         scale=Q.bf16_from_bits(g[f"{name}_{tensor}_fp8_scale_bf16"][i]))
            elif p == "int4":
                e.update(packed=g[f"{name}_{tensor}_i4_packed"][i], scale=g[f"{name}_{tensor}_i4_scale"][i],
                         zero=g[f"{name}_{tensor}_i4_zero"][i])
            kind, idx = fr[tensor]
            for b in range(B):
                for layer in range(L):
                    for h in (0, 9, 15):
                        _check_entry(cache, which, kind, idx, b, layer, h, e)
    pkg._native.check(pkg.lib().oasis_check_device_error())


@pytest.mark.parametrize("fp8_age,int4_age,asym", [(2, 4, True), (3, 3, False), (2, 5, True)])
def test_rolling_window_matches_oracle_replay(pkg, cuda, fp8_age, int4_age, asym):
    """Nine appends into a 6-frame rolling window (the oldest frame leaves once the window
    is full): after each one, every cached frame's key and value codes equal the oracle's
    replay of the reference's manager window + update_cache, per head."""
    from oracle import quant_ref as Q
    B, L, C = 2, 2, 6
    q = pkg.ProgressiveKVQuantizerB200(fp8_age_threshold=fp8_age, int4_age_threshold=int4_age,
                                       key_value_asymmetry=asym)
    cache = pkg.RollingKVCacheB200(B, L, C, q, device=cuda)
    heads = (0, 7, 15)
    refs = {(b, layer, h): Q.UpdateCacheRef(fp8_age, int4_age, asym, window=C)
            for b in range(B) for layer in range(L) for h in heads}
    for n in range(9):
        rows = _frame_rows(B, L, 100 + n, cuda)
        cache.append(rows)
        host = [r.float().cpu().numpy() for r in rows]
        for (b, layer, h), ref in refs.items():
            z = host[layer][b * 144:(b + 1) * 144]
            ref.append(z[:, h * 64:(h + 1) * 64], z[:, 1024 + h * 64:1024 + (h + 1) * 64])
        torch.cuda.synchronize()
        slots = cache.frame_slots()
        assert [s["age"] for s in slots] == list(range(len(slots) - 1, -1, -1))
        assert len(slots) == min(n + 1, C)
        for (b, layer, h), ref in refs.items():
            for i, fr in enumerate(slots):
                for which, tensor in (("k", "key"), ("v", "value")):
                    kind, idx = fr[tensor]
                    _check_entry(cache, which, kind, idx, b, layer, h, ref.entries[tensor][i])
    # the window is a valid cache for the incremental forward
    model = pkg.OasisDiTB200.random(seed=3, depth=1, device=cuda)
    one = pkg.RollingKVCacheB200(B, model.depth, C, q, device=cuda)
    for n in range(C + 2):
        one.append(_frame_rows(B, model.depth, 200 + n, cuda))
    g = torch.Generator().manual_seed(1)
    v = model.forward_cached(torch.randn(B, 16, 18, 32, generator=g).to(cuda),
                             torch.full((B,), 500, device=cuda), None, one, n_past=one.n_slots)
    torch.cuda.synchronize()
    assert torch.isfinite(v).all()
    pkg._native.check(pkg.lib().oasis_check_device_error())


def test_manager_update_reference_thresholds_matches_oracle_replay(pkg, cuda):
    """KVCacheManagerB200.update, the reference's per-frame update (manager.py:246-306 +
    update_cache), at the reference's default thresholds (keys FP8 at age 30, values at
    21; INT4 at 90 / 63) and window (max_frames 32), for 40 frames: every cached frame's
    key and value codes equal the oracle replay; get_kv_for_attention returns the window
    oldest first in the reference's (heads, tokens, head_dim) layout."""
    from oracle import quant_ref as Q
    B, L = 1, 2
    mgr = pkg.KVCacheManagerB200({"num_layers": L, "batch": B, "max_frames": 32,
                                  "progressive_quant": True})
    heads = (0, 11)
    refs = {(layer, h): Q.UpdateCacheRef(30, 90, True, window=32) for layer in range(L) for h in heads}
    g = torch.Generator().manual_seed(5)
    for n in range(40):
        kv = {}
        for layer in range(L):
            k = torch.randn(16, 144, 64, generator=g).bfloat16()
            v = (torch.randn(16, 144, 64, generator=g) * 3).bfloat16()
            kv[layer] = {"key": k.to(cuda), "value": v.to(cuda)}
            for h in heads:
                refs[(layer, h)].append(k[h].float().numpy(), v[h].float().numpy())
        mgr.update(kv, frame_idx=n)
    torch.cuda.synchronize()
    cache = mgr.cache
    assert cache.n_slots == 32
    assert cache.slot_kinds == ["fp8"] * 2 + ["bf16"] * 30
    assert cache.value_kinds == ["fp8"] * 11 + ["bf16"] * 21
    for (layer, h), ref in refs.items():
        for i, fr in enumerate(cache.frame_slots()):
            for which, tensor in (("k", "key"), ("v", "value")):
                kind, idx = fr[tensor]
                _check_entry(cache, which, kind, idx, 0, layer, h, ref.entries[tensor][i])
    got = mgr.get_kv_for_attention(1)
    assert got["key"].shape == (16, 32 * 144, 64)
    assert torch.equal(got["key"][:, -144:].cpu(), kv[1]["key"].cpu())  # newest frame, bf16
    # the newest 31 frames are the past of a 32-frame window's incremental forward
    past = mgr.past_frames(31)
    assert past.n_slots == 31 and past.value_kinds == ["fp8"] * 10 + ["bf16"] * 21
    # get_cache honours its precision: INT4 everywhere is coarser than the stored tiers
    c4 = mgr.get_cache("int4")
    c16 = mgr.get_cache("fp16")
    assert c4[0]["key"].shape == (32, 16, 144, 64) and c4[0]["key"].dtype == torch.float16
    err = (c4[0]["key"].float() - c16[0]["key"].float()).abs().max().item()
    assert 0.0 < err < 1.0


def test_manager_update_continues_from_prefill(pkg, cuda):
    """A prefill (full-window forward into cache_for_window) followed by update(): the
    window keeps the prefill's frames, at the ages they have relative to the appended
    frame, and adds the new one."""
    depth, B, T = 1, 1, 6
    model = pkg.OasisDiTB200.random(seed=8, depth=depth, device=cuda)
    mgr = pkg.KVCacheManagerB200({"num_layers": depth, "batch": B, "max_frames": 8,
                                  "progressive_quant": {"fp8_age_threshold": 2,
                                                        "int4_age_threshold": 4}})
    cache = mgr.cache_for_window(T - 1)
    g = torch.Generator().manual_seed(2)
    x = torch.randn(B, T, 16, 18, 32, generator=g).to(cuda)
    t = torch.randint(0, 1000, (B, T), generator=g).to(cuda)
    model(x, t, None, kv_cache=cache)
    before_k, before_v = cache.load(0)
    k_new = torch.randn(16, 144, 64, generator=g).bfloat16().to(cuda)
    mgr.update({0: {"key": k_new, "value": k_new}}, frame_idx=T - 1)
    torch.cuda.synchronize()
    r = mgr.cache
    assert [s["age"] for s in r.frame_slots()] == [5, 4, 3, 2, 1, 0]
    assert r.slot_kinds[:-1] == cache.slot_kinds and r.value_kinds[:-1] == cache.value_kinds
    after_k, after_v = r.load(0)
    assert torch.equal(after_k[:, :T - 1], before_k) and torch.equal(after_v[:, :T - 1], before_v)
    assert torch.equal(after_k[0, -1].reshape(144, 16, 64).permute(1, 0, 2), k_new)
    # the next frame ages the window as update_cache does
    mgr.update({0: {"key": k_new, "value": k_new}}, frame_idx=T)
    assert [s["age"] for s in mgr.cache.frame_slots()] == [6, 5, 4, 3, 2, 1, 0]
    pkg._native.check(pkg.lib().oasis_check_device_error())
