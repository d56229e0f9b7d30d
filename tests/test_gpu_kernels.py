"""GPU parity of the individual kernels, called through the C ABI.

Float kernels are compared with a plain PyTorch fp32 reference of the same op on the
same bf16 inputs; the KV quantiser is compared bit-for-bit with the oracle's
restatement of the reference quantiser (itself pinned to fixtures from the reference)."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import quant_ref, sampler_ref

pytestmark = pytest.mark.gpu

TOK, HID = 144, 1024


def rel_l2(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


# ----------------------------------------------------------------- GEMM (tcgen05)

# (4608, 1024, 1024), (4500, 3072, 1024) and (4196, 4096, 256) run on CTA pairs (256-row
# tiles, from 4,096 rows on); in the last two the final tile is ragged, in (4196, ...) the
# second CTA of the last pair holds no valid row at all.  (1800, 4096, 256) and
# (2304, 1024, 4096) are single-CTA shapes of the incremental forward's size.
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 512, 1024), (576, 3072, 1024),
                                   (1000, 64, 4096), (4608, 1024, 1024), (130, 192, 128),
                                   (4500, 3072, 1024), (4196, 4096, 256), (1800, 4096, 256),
                                   (2304, 1024, 4096)])
def test_gemm_bf16_store(pkg, cuda, M, N, K):
    g = torch.Generator(device=cuda).manual_seed(M + N + K)
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    B = torch.randn(N, K, device=cuda, generator=g).bfloat16()
    D = torch.full((M, N), float("nan"), device=cuda).bfloat16()
    pkg._native.call("oasis_gemm_bf16", A.data_ptr(), B.data_ptr(), D.data_ptr(), None, M, N, K,
                     K, K, N, 0, torch.cuda.current_stream().cuda_stream)
    ref = A.float() @ B.float().T
    torch.cuda.synchronize()
    assert torch.isfinite(D.float()).all()
    assert rel_l2(D.float(), ref) < 4e-3  # bf16 output rounding


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (333, 128, 512), (1800, 4096, 256), (4196, 4096, 256)])
def test_gemm_f32_bias(pkg, cuda, M, N, K):
    g = torch.Generator(device=cuda).manual_seed(7)
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    B = torch.randn(N, K, device=cuda, generator=g).bfloat16()
    bias = torch.randn(N, device=cuda, generator=g)
    D = torch.empty(M, N, device=cuda)
    pkg._native.call("oasis_gemm_bf16", A.data_ptr(), B.data_ptr(), D.data_ptr(), bias.data_ptr(),
                     M, N, K, K, K, N, 1, torch.cuda.current_stream().cuda_stream)
    ref = A.float() @ B.float().T + bias
    torch.cuda.synchronize()
    assert rel_l2(D, ref) < 1e-5  # fp32 accumulate and store


# ----------------------------------------------------------------- attention

def _qkv(frames, cuda, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    return torch.randn(frames * TOK, 3 * HID, device=cuda, generator=g).bfloat16()


def _heads(z, frames):  # [frames*144][1024] -> (frames, 16, 144, 64)
    return z.float().reshape(frames, TOK, 16, 64).permute(0, 2, 1, 3)


@pytest.mark.parametrize("frames", [1, 3, 32])
def test_attn_spatial(pkg, cuda, frames):
    qkv = _qkv(frames, cuda, frames)
    out = pkg.attn_spatial(qkv)
    q, k, v = (_heads(qkv[:, i * HID:(i + 1) * HID], frames) for i in range(3))
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v)
    ref = ref.permute(0, 2, 1, 3).reshape(frames * TOK, HID)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2


def _temporal_ref(qkv, B, T, n_past_k=None, n_past_v=None, q_pos0=0):
    """fp32 causal attention over (B*144, 16, T, 64) from a [B*T*144][3072] buffer."""
    z = qkv.float().reshape(B, T, TOK, 3, 16, 64)
    q = z[:, :, :, 0].permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, T, 64)
    k = z[:, :, :, 1].permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, T, 64)
    v = z[:, :, :, 2].permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, T, 64)
    if n_past_k is not None:
        k = torch.cat([n_past_k, k], dim=2)
        v = torch.cat([n_past_v, v], dim=2)
    S = k.shape[2]
    pos_q = torch.arange(T, device=qkv.device) + q_pos0
    mask = torch.arange(S, device=qkv.device)[None, :] <= pos_q[:, None]
    o = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    return o.reshape(B, TOK, 16, T, 64).permute(0, 3, 1, 2, 4).reshape(B * T * TOK, HID)


@pytest.mark.parametrize("B,T", [(1, 1), (1, 5), (2, 8), (1, 32), (3, 17)])
def test_attn_temporal_bf16(pkg, cuda, B, T):
    qkv = _qkv(B * T, cuda, 100 + T)
    out = pkg.attn_temporal(qkv, batch=B, q_frames=T)
    ref = _temporal_ref(qkv, B, T)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2


@pytest.mark.parametrize("T,q_pos0,n_kv", [(8, 3, 5), (32, 0, 20), (17, 40, 17), (32, 7, 32)])
def test_attn_temporal_full_window_offsets(pkg, cuda, T, q_pos0, n_kv):
    """Full-window call (no cache) with the queries at window positions q_pos0.. and only
    the first n_kv frames as keys: the causal mask takes both into account."""
    B = 3
    qkv = _qkv(B * T, cuda, 400 + T + q_pos0)
    out = pkg.attn_temporal(qkv, batch=B, q_frames=T, q_pos0=q_pos0, n_kv=n_kv)
    z = qkv.float().reshape(B, T, TOK, 3, 16, 64)
    q, k, v = (z[:, :, :, i].permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, T, 64) for i in range(3))
    k, v = k[:, :, :n_kv].contiguous(), v[:, :, :n_kv].contiguous()
    mask = torch.arange(n_kv, device=cuda)[None, :] <= (torch.arange(T, device=cuda) + q_pos0)[:, None]
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    ref = ref.reshape(B, TOK, 16, T, 64).permute(0, 3, 1, 2, 4).reshape(B * T * TOK, HID)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2


# ----------------------------------------------------------------- KV cache quantisation

def _kv_rows(B, F, cuda, seed, scale_per_frame=True):
    g = torch.Generator(device=cuda).manual_seed(seed)
    z = torch.randn(B * F * TOK, 3 * HID, device=cuda, generator=g)
    if scale_per_frame:
        s = torch.rand(B * F, 1, 1, 16, 1, device=cuda, generator=g) * 3 + 0.01
        z = (z.reshape(B * F, TOK, 3, 16, 64) * s).reshape(B * F * TOK, 3 * HID)
    return z.bfloat16()


def _slice(kv_rows, b, f, F, col0, h):
    """bf16 (144, 64) slice of K (col0=1024) or V (2048) of head h, frame f, session b."""
    r0 = (b * F + f) * TOK
    return kv_rows[r0:r0 + TOK, col0 + h * 64: col0 + (h + 1) * 64].float().cpu().numpy()


def test_kv_store_fp8_bit_exact(pkg, cuda):
    B, F, L = 2, 3, 2
    rows = _kv_rows(B, F, cuda, 1)
    # plant the reference fixtures' edge cases (zeros, constant, outlier, tiny, large) in
    gold = np.load("tests/golden/quant_golden.npz")
    gi = torch.from_numpy(quant_ref.bf16_from_bits(gold["inp_bf16"][12:17])).to(cuda).bfloat16()
    for i in range(gi.shape[0]):
        rows[i * TOK:(i + 1) * TOK, HID + 64 * i: HID + 64 * (i + 1)] = gi[i]
    cache = pkg.KVCacheB200.uniform(B, L, F, "fp8", device=cuda)
    cache.store(rows, layer=1)
    torch.cuda.synchronize()
    for which, col0, codes_t, scale_t in (("k", HID, cache.k_fp8, cache.k_fp8_scale),
                                          ("v", 2 * HID, cache.v_fp8, cache.v_fp8_scale)):
        codes = codes_t[:, 1].cpu().numpy()          # (B, F, 144, 1024)
        scales = scale_t[:, 1].float().cpu().numpy()  # (B, F, 16)
        for b in range(B):
            for f in range(F):
                for h in range(16):
                    want_c, want_s = quant_ref.quantize_to_fp8_bf16(_slice(rows, b, f, F, col0, h))
                    assert scales[b, f, h] == want_s, (which, b, f, h)
                    np.testing.assert_array_equal(codes[b, f, :, h * 64:(h + 1) * 64], want_c)
    # untouched layer stays zero
    assert int(cache.k_fp8[:, 0].sum()) == 0


def test_kv_store_int4_bit_exact(pkg, cuda):
    B, F, L = 2, 2, 1
    rows = _kv_rows(B, F, cuda, 2)
    cache = pkg.KVCacheB200.uniform(B, L, F, "int4", device=cuda)
    cache.store(rows, layer=0)
    torch.cuda.synchronize()
    for col0, codes_t, sc_t, zp_t in ((HID, cache.k_int4, cache.k_i4_scale, cache.k_i4_zero),
                                      (2 * HID, cache.v_int4, cache.v_i4_scale, cache.v_i4_zero)):
        codes = codes_t[:, 0].cpu().numpy()   # (B, F, 144, 16, 32)
        sc = sc_t[:, 0].cpu().numpy()         # (B, F, 144, 16) fp16
        zp = zp_t[:, 0].cpu().numpy()
        for b in range(B):
            for f in range(F):
                for h in range(16):
                    x = _slice(rows, b, f, F, col0, h)
                    packed, s16, z16, _, _ = quant_ref.quantize_int4_rows(x)
                    np.testing.assert_array_equal(codes[b, f, :, h], packed)
                    np.testing.assert_array_equal(sc[b, f, :, h].view(np.uint16), s16.view(np.uint16))
                    np.testing.assert_array_equal(zp[b, f, :, h].view(np.uint16), z16.view(np.uint16))


def test_kv_load_matches_oracle_dequant(pkg, cuda):
    B, F = 1, 3
    rows = _kv_rows(B, F, cuda, 3)
    cache = pkg.KVCacheB200(B, 1, ["int4", "fp8", "bf16"], device=cuda)
    cache.store(rows, layer=0)
    k, v = cache.load(0)
    torch.cuda.synchronize()
    k = k.float().cpu().numpy()
    for f, kind in enumerate(["int4", "fp8", "bf16"]):
        for h in (0, 7, 15):
            x = _slice(rows, 0, f, F, HID, h)
            got = k[0, f, :, h * 64:(h + 1) * 64]
            if kind == "bf16":
                np.testing.assert_array_equal(got, x)
            elif kind == "fp8":
                c, s = quant_ref.quantize_to_fp8_bf16(x)
                np.testing.assert_array_equal(got, quant_ref.dequantize_fp8_bf16(c, s))
            else:
                p, s16, z16, _, _ = quant_ref.quantize_int4_rows(x)
                q = quant_ref.unpack_int4(p.reshape(-1)).reshape(144, 64).astype(np.float32)
                want = quant_ref.bf16_round(q * s16.astype(np.float32)[:, None] + z16.astype(np.float32)[:, None])
                np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("kinds", [["fp8"] * 7, ["int4"] * 5 + ["bf16"] * 2, ["bf16"] * 3 + ["fp8"] * 2])
def test_attn_temporal_incremental_quantized(pkg, cuda, kinds):
    """Newest-frame query against dequantised past slots + its own K/V (fused dequant)."""
    B, P = 2, len(kinds)
    past = _kv_rows(B, P, cuda, 11)
    cache = pkg.KVCacheB200(B, 1, kinds, device=cuda)
    cache.store(past, layer=0)
    new = _qkv(B, cuda, 12)  # one new frame per session
    out = pkg.attn_temporal(new, batch=B, q_frames=1, q_pos0=P, n_past=P, n_kv=P + 1, cache=cache, layer=0)
    k, v = cache.load(0)  # (B, P, 144, 1024) dequantised like the kernel does
    kp = k.float().reshape(B, P, TOK, 16, 64).permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, P, 64)
    vp = v.float().reshape(B, P, TOK, 16, 64).permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, P, 64)
    ref = _temporal_ref(new, B, 1, kp, vp, q_pos0=P)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2


@pytest.mark.parametrize("kind,T", [("fp8", 8), ("int4", 16), ("fp8", 32)])
def test_attn_temporal_full_from_quantized_cache(pkg, cuda, kind, T):
    """Isolated sweep case: causal T x T with every K/V frame read from the quantised cache."""
    B = 2
    qkv = _qkv(B * T, cuda, 200 + T)
    cache = pkg.KVCacheB200.uniform(B, 1, T, kind, device=cuda)
    cache.store(qkv, layer=0)
    out = pkg.attn_temporal(qkv, batch=B, q_frames=T, q_pos0=0, n_past=T, n_kv=T, cache=cache, layer=0)
    k, v = cache.load(0)
    deq = qkv.clone()
    deq[:, HID:2 * HID] = k.reshape(B * T * TOK, HID)
    deq[:, 2 * HID:] = v.reshape(B * T * TOK, HID)
    ref = _temporal_ref(deq, B, T)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2


@pytest.mark.parametrize("kinds,vkinds,q_frames,q_pos0", [
    (["bf16"] * 16, ["bf16"] * 16, 16, 0),
    (["fp8"] * 32, ["int4"] * 32, 8, 24),
    (["int4"] * 32, ["bf16"] * 32, 20, 12),
    (["int4"] * 16 + ["bf16"] * 16, ["int4"] * 16 + ["bf16"] * 16, 32, 0)])
def test_attn_window_from_cache(pkg, cuda, kinds, vkinds, q_frames, q_pos0):
    """Several query frames with every key and value from the cache: one kind per tensor runs
    the register-fragment window kernel, mixed kinds the staging kernel; vs fp32 SDPA over
    the dequantised cache, causal at window positions q_pos0.."""
    B, P = 3, len(kinds)
    past = _kv_rows(B, P, cuda, 400 + P)
    cache = pkg.KVCacheB200(B, 1, kinds, device=cuda, value_kinds=vkinds)
    cache.store(past, layer=0)
    new = _qkv(B * q_frames, cuda, 401)
    out = pkg.attn_temporal(new, batch=B, q_frames=q_frames, q_pos0=q_pos0, n_past=P, n_kv=P, cache=cache,
                            layer=0)
    k, v = cache.load(0)
    kp = k.float().reshape(B, P, TOK, 16, 64).permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, P, 64)
    vp = v.float().reshape(B, P, TOK, 16, 64).permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, P, 64)
    q = new.float().reshape(B, q_frames, TOK, 3, 16, 64)[:, :, :, 0]
    q = q.permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, q_frames, 64)
    pos_q = torch.arange(q_frames, device=cuda) + q_pos0
    mask = torch.arange(P, device=cuda)[None, :] <= pos_q[:, None]
    ref = torch.nn.functional.scaled_dot_product_attention(q, kp, vp, attn_mask=mask)
    ref = ref.reshape(B, TOK, 16, q_frames, 64).permute(0, 3, 1, 2, 4).reshape(B * q_frames * TOK, HID)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2


# keys and values in their own tiers (the reference's key/value asymmetry), one query frame
@pytest.mark.parametrize("kinds,vkinds", [
    (["int4"] * 3 + ["fp8"] * 3 + ["bf16"] * 2, ["int4"] * 5 + ["fp8"] * 2 + ["bf16"]),
    (["fp8"] * 31, ["fp8"] * 31),
    (["bf16"] * 31, ["fp8"] * 10 + ["bf16"] * 21),
    (["fp8"] * 2 + ["bf16"] * 29, ["fp8"] * 11 + ["bf16"] * 20),
    (["int4"] * 23 + ["bf16"] * 8, ["int4"] * 23 + ["bf16"] * 8),
    # every slot INT4, and fewer bf16 slots than a key tile: the 8-heads-per-warp kernel
    (["int4"] * 31, ["int4"] * 31),
    (["int4"] * 10 + ["bf16"] * 5, ["int4"] * 10 + ["bf16"] * 5),
    # kinds interleaved: the kernel regroups the slots into kind-uniform key tiles
    (["int4", "bf16"] * 8, ["int4", "bf16"] * 8),
    (["fp8", "int4"] * 10 + ["bf16"], ["fp8"] * 20 + ["bf16"])])
def test_attn_decode_keys_values_in_own_tiers(pkg, cuda, kinds, vkinds):
    """The one-query-frame kernel of the incremental forward: newest frame against cached
    slots whose keys and values sit in different tiers, plus its own K/V, vs fp32 SDPA on
    the dequantised cache."""
    B, P = 3, len(kinds)
    past = _kv_rows(B, P, cuda, 21)
    cache = pkg.KVCacheB200(B, 1, kinds, device=cuda, value_kinds=vkinds)
    cache.store(past, layer=0)
    new = _qkv(B, cuda, 22)
    out = pkg.attn_temporal(new, batch=B, q_frames=1, q_pos0=P, n_past=P, n_kv=P + 1, cache=cache, layer=0)
    k, v = cache.load(0)
    kp = k.float().reshape(B, P, TOK, 16, 64).permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, P, 64)
    vp = v.float().reshape(B, P, TOK, 16, 64).permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, P, 64)
    ref = _temporal_ref(new, B, 1, kp, vp, q_pos0=P)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2


@pytest.mark.parametrize("kinds,n_kv_extra", [(["int4"] * 31, 1), (["int4"] * 31, 0),
                                               (["int4"] * 23 + ["bf16"] * 8, 1)])
def test_attn_decode_int4_at_benchmark_batch(pkg, cuda, kinds, n_kv_extra):
    """The INT4 and progressive (23 INT4 + 8 bf16) one-query-frame cases at 16 sessions, the
    benchmark's batch (8 heads per warp, persistent grid with several items per warp), with
    and without the frame's own key, vs fp32 SDPA on the dequantised cache."""
    B, P = 16, len(kinds)
    past = _kv_rows(B, P, cuda, 41)
    cache = pkg.KVCacheB200(B, 1, kinds, device=cuda)
    cache.store(past, layer=0)
    new = _qkv(B, cuda, 42)
    q_pos0 = P if n_kv_extra else P - 1
    out = pkg.attn_temporal(new, batch=B, q_frames=1, q_pos0=q_pos0, n_past=P, n_kv=P + n_kv_extra, cache=cache,
                            layer=0)
    k, v = cache.load(0)
    kp = k.float().reshape(B, P, TOK, 16, 64).permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, P, 64)
    vp = v.float().reshape(B, P, TOK, 16, 64).permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, P, 64)
    if n_kv_extra:
        ref = _temporal_ref(new, B, 1, kp, vp, q_pos0=P)
    else:
        q = new.float().reshape(B, 1, TOK, 3, 16, 64)[:, :, :, 0].permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, 1, 64)
        ref = torch.nn.functional.scaled_dot_product_attention(q, kp, vp)
        ref = ref.reshape(B, TOK, 16, 1, 64).permute(0, 3, 1, 2, 4).reshape(B * TOK, HID)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert rel_l2(out.float(), ref) < 1e-2


def test_attn_decode_all_keys_cached(pkg, cuda):
    """One query frame whose keys all come from the cache (n_kv == n_past): the query at
    window position P-1 sees cached slots 0..P-1 and nothing of its own row."""
    B, P = 2, 9
    past = _kv_rows(B, P, cuda, 31)
    cache = pkg.KVCacheB200(B, 1, ["fp8"] * 4 + ["bf16"] * 5, device=cuda,
                            value_kinds=["int4"] * 6 + ["bf16"] * 3)
    cache.store(past, layer=0)
    new = _qkv(B, cuda, 32)
    out = pkg.attn_temporal(new, batch=B, q_frames=1, q_pos0=P - 1, n_past=P, n_kv=P, cache=cache, layer=0)
    k, v = cache.load(0)
    kp = k.float().reshape(B, P, TOK, 16, 64).permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, P, 64)
    vp = v.float().reshape(B, P, TOK, 16, 64).permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, P, 64)
    q = new.float().reshape(B, 1, TOK, 3, 16, 64)[:, :, :, 0].permute(0, 2, 3, 1, 4).reshape(B * TOK, 16, 1, 64)
    ref = torch.nn.functional.scaled_dot_product_attention(q, kp, vp)
    ref = ref.reshape(B, TOK, 16, 1, 64).permute(0, 3, 1, 2, 4).reshape(B * TOK, HID)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2


# the isolated attention sweep (benchmark configuration 4) at its own sizes
@pytest.mark.parametrize("frames", [256, 1024, 4096])
def test_attn_spatial_sweep_sizes(pkg, cuda, frames):
    qkv = _qkv(frames, cuda, 7 + frames)
    out = pkg.attn_spatial(qkv)
    q, k, v = (_heads(qkv[:, i * HID:(i + 1) * HID], frames) for i in range(3))
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v)
    ref = ref.permute(0, 2, 1, 3).reshape(frames * TOK, HID)
    del q, k, v
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2


@pytest.mark.parametrize("kind", ["bf16", "fp8", "int4"])
@pytest.mark.parametrize("T", [8, 16, 32])
@pytest.mark.parametrize("B", [8, 32])
def test_attn_temporal_sweep_sizes(pkg, cuda, B, T, kind):
    """Causal T x T over B*144 sequences with bf16 K/V (full-window kernel) or every K/V
    frame read from an FP8 / INT4 cache, vs fp32 SDPA on the (dequantised) inputs."""
    qkv = _qkv(B * T, cuda, 300 + B + T)
    if kind == "bf16":
        out = pkg.attn_temporal(qkv, batch=B, q_frames=T)
        ref = _temporal_ref(qkv, B, T)
    else:
        cache = pkg.KVCacheB200.uniform(B, 1, T, kind, device=cuda)
        cache.store(qkv, layer=0)
        out = pkg.attn_temporal(qkv, batch=B, q_frames=T, q_pos0=0, n_past=T, n_kv=T, cache=cache, layer=0)
        k, v = cache.load(0)
        deq = qkv.clone()
        deq[:, HID:2 * HID] = k.reshape(B * T * TOK, HID)
        deq[:, 2 * HID:] = v.reshape(B * T * TOK, HID)
        del k, v, cache
        ref = _temporal_ref(deq, B, T)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2


# ----------------------------------------------------------------- samplers

def test_dpmpp2m_and_ddim_update(pkg, cuda):
    B, T = 3, 4
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(B, T, 16, 18, 32, device=cuda, generator=g)
    v = torch.randn(B, T, 16, 18, 32, device=cuda, generator=g)
    eps_prev = torch.randn(B, 16 * 18 * 32, device=cuda, generator=g)
    x0, ep0 = x.clone(), eps_prev.clone()
    pkg.dpmpp2m_update(x, v, eps_prev, 0.3, 0.6, first=False)
    want, eps = sampler_ref.dpmpp2m_vpred_step(x0[:, -1].cpu().numpy(), v[:, -1].cpu().numpy(),
                                               ep0.reshape(B, 16, 18, 32).cpu().numpy(), 0.3, 0.6, False)
    torch.cuda.synchronize()
    np.testing.assert_allclose(x[:, -1].cpu().numpy(), want, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(eps_prev.reshape(B, 16, 18, 32).cpu().numpy(), eps, rtol=1e-5, atol=1e-5)
    assert torch.equal(x[:, :-1], x0[:, :-1])  # only the newest frame is written
    xd = x0.clone()
    pkg.ddim_update(xd, v, 0.2, 0.9)
    want = sampler_ref.ddim_vpred_step(x0[:, -1].cpu().numpy(), v[:, -1].cpu().numpy(), 0.2, 0.9)
    torch.cuda.synchronize()
    np.testing.assert_allclose(xd[:, -1].cpu().numpy(), want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("order", [1, 2, 3])
def test_ab_sampler_matches_reference_fixture(pkg, cuda, order):
    gold = np.load("tests/golden/sampler_golden.npz")
    lats, preds, ts = gold[f"ab{order}_latents"], gold[f"ab{order}_preds"], gold[f"ab{order}_ts"]
    s = pkg.DPMSolverPPSampler(order=order)
    x = torch.from_numpy(lats[0]).to(cuda)
    for i in range(preds.shape[0]):
        x = s.step(x, torch.from_numpy(preds[i]).to(cuda), torch.tensor(ts[i]), torch.tensor(ts[i + 1]))
        np.testing.assert_allclose(x.cpu().numpy(), lats[i + 1], rtol=1e-5, atol=1e-5)


def test_no_device_timeouts_recorded(pkg, cuda):
    torch.cuda.synchronize()
    pkg._native.check(pkg.lib().oasis_check_device_error())


def test_bounded_wait_gives_up_and_context_stays_usable(pkg, cuda):
    """A device-side wait on a flag that nothing sets runs out after its 2 s limit: the
    kernel records the timeout and returns, the host reads OASIS_ERR_DEVICE_TIMEOUT (5)
    once, and the next kernels on the same context give correct results."""
    L = pkg.lib()
    pkg._native.check(L.oasis_check_device_error())  # start from a clear error word
    assert L.oasis_selftest_bounded_wait(None) == 0
    assert L.oasis_check_device_error() == 5
    assert b"bounded wait" in L.oasis_last_error()
    assert L.oasis_check_device_error() == 0  # reading it cleared it
    qkv = _qkv(1 * 5, cuda, 77)
    out = pkg.attn_temporal(qkv, batch=1, q_frames=5)
    ref = _temporal_ref(qkv, 1, 5)
    torch.cuda.synchronize()
    assert rel_l2(out.float(), ref) < 1e-2
    pkg._native.check(L.oasis_check_device_error())
