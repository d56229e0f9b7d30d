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
