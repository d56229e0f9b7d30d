"""The allocation-free forward entry point, checked against the regular one.

``oasis_dit_forward_noalloc`` serves callers that cannot call cudaMalloc (fixed memory
budgets, code running inside another framework's stream capture): it keeps its
scratch in a fixed device array inside the library instead of a caller workspace.
Its results must match ``oasis_dit_forward`` on the same weights and inputs, call
after call, since both run the same kernels.  This file is collected last so a
failure here cannot hide the other tests; it needs nothing from them.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(B, T, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, 16, 18, 32, generator=g)
    t = torch.randint(0, 1000, (B, T), generator=g)
    a = torch.zeros(B, T, 25)
    a[..., :23] = (torch.rand(B, T, 23, generator=g) < 0.1).float()
    a[..., 23:] = torch.randn(B, T, 2, generator=g) * 0.3
    return x, t, a


def _noalloc(pkg, model, x, t, a, v):
    B, T = x.shape[:2]
    pkg._native.call("oasis_dit_forward_noalloc", ctypes.byref(model.weights.struct), B, T,
                     x.data_ptr(), t.data_ptr(), a.data_ptr(), v.data_ptr(),
                     torch.cuda.current_stream().cuda_stream)


def test_noalloc_forward_matches_regular_entry_point(pkg, cuda):
    depth = 16
    model = pkg.OasisDiTB200.random(seed=3, depth=depth, device=cuda)
    # two calls in a row with different inputs (and one shape change in between)
    for (B, T, seed) in ((1, 4, 11), (2, 2, 12)):
        x, t, a = (z.to(cuda).contiguous() for z in _inputs(B, T, seed))
        v_ref = model(x, t, a)
        v = torch.full_like(v_ref, float("nan"))
        _noalloc(pkg, model, x, t, a, v)
        torch.cuda.synchronize()
        assert torch.isfinite(v).all()
        err = ((v.double() - v_ref.double()).norm() / v_ref.double().norm()).item()
        assert err <= 1e-5, err
    pkg._native.check(pkg.lib().oasis_check_device_error())


def test_noalloc_rejects_shapes_beyond_its_scratch(pkg, cuda):
    model = pkg.OasisDiTB200.random(seed=3, depth=1, device=cuda)
    x, t, a = (z.to(cuda).contiguous() for z in _inputs(1, 5, 1))
    v = torch.empty_like(x)
    st = pkg.lib().oasis_dit_forward_noalloc(ctypes.byref(model.weights.struct), 1, 5, x.data_ptr(),
                                             t.data_ptr(), a.data_ptr(), v.data_ptr(), None)
    assert st == 6  # OASIS_ERR_UNSUPPORTED
    assert b"batch * frames" in pkg.lib().oasis_last_error()
