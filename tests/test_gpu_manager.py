"""KV-cache manager interface (the worldserve method names) over the B200 cache."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_manager_prefill_retrieve_update_snapshot(pkg, cuda):
    depth, B, T = 2, 2, 5
    model = pkg.OasisDiTB200.random(seed=4, depth=depth, device=cuda)
    mgr = pkg.KVCacheManagerB200({"num_layers": depth, "batch": B,
                                  "progressive_quant": {"fp8_age_threshold": 3,
                                                        "int4_age_threshold": 4}})
    assert mgr.wire_to_model(model) == depth
    cache = mgr.cache_for_window(T - 1)
    # ages 4, 3, 2, 1; V thresholds are int(0.7x) = 2 (fp8) and 2 (int4): the coarser tier wins
    assert cache.slot_kinds == ["int4", "int4", "int4", "bf16"]
    g = torch.Generator().manual_seed(0)
    x = torch.randn(B, T, 16, 18, 32, generator=g).to(cuda)
    t = torch.randint(0, 1000, (B, T), generator=g).to(cuda)
    model(x, t, None, kv_cache=cache)
    kv = mgr.get_kv_for_attention(1)
    assert kv["key"].shape == (B, 16, (T - 1) * 144, 64)
    assert torch.isfinite(kv["key"].float()).all() and kv["key"].abs().sum() > 0
    snap = mgr.snapshot()
    # update(): overwrite the newest slot of layer 0 with given K/V, then restore
    k = torch.randn(B, 16, 144, 64, device=cuda).bfloat16()
    mgr.update({0: {"key": k, "value": k}}, frame_idx=T - 1)
    got = mgr.get_kv_for_attention(0)["key"][:, :, -144:]
    assert torch.equal(got, k)  # bf16 slot stores exactly
    mgr.restore(snap)
    assert not torch.equal(mgr.get_kv_for_attention(0)["key"][:, :, -144:], k)
    rep = mgr.get_memory_report()
    assert 0.0 < rep["savings_ratio"] < 1.0


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


@pytest.mark.parametrize("fp8_age,int4_age", [(2, 4), (3, 3)])
def test_rolling_cache_ages_and_promotes_like_update_cache(pkg, cuda, fp8_age, int4_age):
    """Nine appends into a 6-frame rolling window: after each one, every cached frame's
    stored codes equal the oracle's for its promotion history (bf16 exact; FP8 codes and
    bf16 scale; INT4 from the FP8 entry through the fp16 dequantisation, or straight from
    bf16 when the tiers jump), and the window holds the newest frames oldest first."""
    import numpy as np
    from oracle import quant_ref as Q

    B, L, C = 2, 2, 6
    q = pkg.ProgressiveKVQuantizerB200(fp8_age_threshold=fp8_age, int4_age_threshold=int4_age,
                                       key_value_asymmetry=False)
    cache = pkg.RollingKVCacheB200(B, L, C, q, device=cuda)
    frames = []
    for n in range(9):
        rows = _frame_rows(B, L, 100 + n, cuda)
        frames.append([r.float().cpu().numpy() for r in rows])
        cache.append(rows)
        torch.cuda.synchronize()
        slots = cache.frame_slots()
        assert [a for _, _, a in slots] == list(range(len(slots) - 1, -1, -1))
        assert len(slots) == min(n + 1, C)
        for s, (kind, idx, age) in enumerate(slots):
            data = frames[n - age]
            for layer in range(L):
                for b in range(B):
                    for which, col in (("k", 0), ("v", 1024)):
                        src = data[layer][b * 144:(b + 1) * 144, col:col + 1024]
                        if kind == "bf16":
                            got = getattr(cache, which + "_bf16")[b, layer, idx].float().cpu().numpy()
                            np.testing.assert_array_equal(got, src)
                            continue
                        for h in range(16):
                            sl = src[:, h * 64:(h + 1) * 64]
                            codes, scale = Q.quantize_to_fp8_bf16(sl)
                            if kind == "fp8":
                                got = getattr(cache, which + "_fp8")[b, layer, idx][:, h * 64:(h + 1) * 64]
                                np.testing.assert_array_equal(got.cpu().numpy(), codes)
                                gs = getattr(cache, which + "_fp8_scale")[b, layer, idx, h].float().item()
                                assert gs == scale
                                continue
                            via_fp8 = fp8_age < int4_age
                            p, s16, z16, _, _ = (Q.promote_fp8_to_int4_rows(codes, scale) if via_fp8
                                                 else Q.quantize_int4_rows(sl))
                            got = getattr(cache, which + "_int4")[b, layer, idx, :, h]
                            np.testing.assert_array_equal(got.cpu().numpy(), p)
                            gsc = getattr(cache, which + "_i4_scale")[b, layer, idx, :, h].cpu().numpy()
                            gz = getattr(cache, which + "_i4_zero")[b, layer, idx, :, h].cpu().numpy()
                            np.testing.assert_array_equal(gsc, s16)
                            np.testing.assert_array_equal(gz, z16)
    assert cache.slot_kinds[-1] == "bf16" and cache.slot_kinds[0] == "int4"
    # the window is a valid cache for the incremental forward
    model = pkg.OasisDiTB200.random(seed=3, depth=1, device=cuda)
    one = pkg.RollingKVCacheB200(B, model.depth, C, q, device=cuda)
    for n in range(C):
        one.append(_frame_rows(B, model.depth, 200 + n, cuda))
    g = torch.Generator().manual_seed(1)
    v = model.forward_cached(torch.randn(B, 16, 18, 32, generator=g).to(cuda),
                             torch.full((B,), 500, device=cuda), None, one, n_past=one.n_slots)
    torch.cuda.synchronize()
    assert torch.isfinite(v).all()
    pkg._native.check(pkg.lib().oasis_check_device_error())


def test_manager_append_keeps_a_rolling_progressive_window(pkg, cuda):
    """KVCacheManagerB200.append with the reference's per-layer dict input."""
    B, L = 1, 2
    mgr = pkg.KVCacheManagerB200({"num_layers": L, "batch": B, "max_frames": 5,
                                  "progressive_quant": {"fp8_age_threshold": 1,
                                                        "int4_age_threshold": 3,
                                                        "key_value_asymmetry": False}})
    g = torch.Generator().manual_seed(5)
    for n in range(7):
        kv = {l: {"key": torch.randn(B, 16, 144, 64, generator=g).bfloat16().to(cuda),
                  "value": torch.randn(B, 16, 144, 64, generator=g).bfloat16().to(cuda)}
              for l in range(L)}
        mgr.append(kv, frame_idx=n)
    assert mgr.cache.slot_kinds == ["int4", "fp8", "fp8", "bf16"]  # ages 3, 2, 1, 0
    newest = mgr.get_kv_for_attention(1)
    assert newest["key"].shape == (B, 16, 4 * 144, 64)
    assert torch.equal(newest["key"][:, :, -144:], kv[1]["key"])  # the new frame is bf16
    rep = mgr.get_memory_report()
    assert 0.0 < rep["savings_ratio"] < 1.0
