// Forward plan: the native runtime that drives one Oasis DiT denoising forward.
//
// Per call (frames F = batch * frames_per_session, tokens M = F * 144):
//   patch im2col + fp32 linear -> residual x (fp32, [M][1024])
//   timestep sinusoid -> MLP (SiLU) + action linear -> c; bf16(SiLU(c))
//   ONE swap-AB tcgen05 GEMM for all 33 adaLN modulations -> mod [F][2*depth*6144 + 2048]
//   per sub-block (spatial, then temporal, x depth):
//     LN+modulate -> QKV GEMM (+RoPE epilogue) -> attention [-> KV store] ->
//     out GEMM (gate*(.+b) + residual epilogue) -> LN+modulate -> fc1 GEMM (+b, GELU) ->
//     fc2 GEMM (gate*(.+b) + residual epilogue)
//   final LN+modulate -> 1024->64 GEMM with the unpatchify store into v.
// All launches go to the caller's stream; nothing allocates or synchronises, so a
// forward can be captured into a CUDA graph.
#include <nvtx3/nvToolsExt.h>

#include <cstring>
#include <vector>

#include "gemm.cuh"
#include "launch.cuh"

namespace oasis {

namespace {

constexpr int kFamilies = 7;
enum Family { kFamGemm = 0, kFamAda, kFamSpatial, kFamTemporal, kFamLn, kFamEmbed, kFamKv };

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct Layout {
  size_t resid, hbuf, qkv, attn, mlp, cols, emb, h1a, silu, mod, cnt, total;
  size_t cnt_bytes;  // row-block counters of the residual GEMMs' LayerNorm tails
  // split-K ordering counters of the residual GEMMs, right after the row-block counters:
  // per sub-block two launches (out-proj, fc2) of at most ceil(M/128) x 8 tiles x 8 warps
  size_t flag_words_per_launch;
};

// Row-block counters (one per 128-row block), zeroed at the start of every forward.
// Per sub-block: 0 out-proj tiles, 1 rows normalised after it, 2 fc1 tiles (a bitmask
// of the finished N tiles), 3 fc2 tiles, 4 rows normalised after fc2 (the
// separate-launch path uses 0 and 3).
inline size_t row_blocks(size_t M) { return (M + 127) / 128; }
constexpr int kCountersPerSub = 5;

constexpr int kH1aLd = OASIS_HIDDEN + 64;  // [first-linear output | actions | zero pad]

Layout layout_for(int F, int depth) {
  const size_t M = static_cast<size_t>(F) * OASIS_TOKENS;
  const size_t mod_ld = static_cast<size_t>(2 * depth) * OASIS_ADA_PER_SUB + 2 * OASIS_HIDDEN;
  Layout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  L.resid = take(M * OASIS_HIDDEN * 4);
  L.hbuf = take(M * OASIS_HIDDEN * 2);
  L.qkv = take(M * 3 * OASIS_HIDDEN * 2);
  L.attn = take(M * OASIS_HIDDEN * 2);
  L.mlp = take(M * OASIS_MLP_HIDDEN * 2);
  L.cols = take(M * 64 * 2);
  L.emb = take(static_cast<size_t>(F) * 256 * 2);
  L.h1a = take(static_cast<size_t>(F) * kH1aLd * 2);
  L.silu = take(static_cast<size_t>(F) * OASIS_HIDDEN * 2);
  L.mod = take(static_cast<size_t>(F) * mod_ld * 4);
  L.cnt_bytes = static_cast<size_t>(2 * depth) * kCountersPerSub * row_blocks(M) * 4;
  L.flag_words_per_launch = row_blocks(M) * 8 * 8;  // splits use tiles N >= 128 (<= 8 of them)
  L.cnt = take(L.cnt_bytes + static_cast<size_t>(2 * depth) * 2 * L.flag_words_per_launch * 4);
  L.total = off;
  return L;
}

}  // namespace
}  // namespace oasis

struct oasis_plan {
  oasis_dit_weights_t w;
  int batch = 0, frames = 0, F = 0, M = 0, depth = 0;
  long long mod_ld = 0;
  uint8_t* ws = nullptr;
  oasis::Layout L{};
  // GEMM operand descriptors
  oasis::GemmOperands patch, temb1, temb2;  // embeddings
  oasis::GemmOperands ada;
  oasis::GemmOperands fin;
  oasis::GemmOperands qkv[2 * OASIS_MAX_DEPTH], out[2 * OASIS_MAX_DEPTH];  // per sub-block
  oasis::GemmOperands fc1[2 * OASIS_MAX_DEPTH], fc2[2 * OASIS_MAX_DEPTH];
  // out-proj, fc1, fc2 and the next QKV of a sub-block run as one chained launch
  // (gemm_chain_kernel) when all of them use CTA-pair 256-wide tiles
  bool chain = false;
  // bytes of row-block counters and split-K counters zeroed at the start of a forward
  size_t zero_bytes = 0;
  // timing
  bool timing = false;
  std::vector<cudaEvent_t> ev;
  std::vector<int> ev_family;
  int ev_used = 0;
  float fam_ms[oasis::kFamilies] = {};
  int fam_launches[oasis::kFamilies] = {};
};

namespace oasis {
namespace {

// NVTX range names of the kernel families (visible to Nsight tools; free otherwise).
const char* const kFamilyNames[kFamilies] = {"oasis/gemm", "oasis/adaln_gemm", "oasis/spatial_attn",
                                             "oasis/temporal_attn", "oasis/ln_modulate",
                                             "oasis/embed_final", "oasis/kv_store"};

// One launch group of a kernel family: an NVTX range around its host-side launches and,
// while the plan's timing is enabled, CUDA events around it on the stream.
struct Timer {
  oasis_plan* p;
  cudaStream_t s;
  int fam;
  int idx = -1;
  Timer(oasis_plan* p_, cudaStream_t s_, int fam_) : p(p_), s(s_), fam(fam_) {
    nvtxRangePushA(kFamilyNames[fam]);
    if (p->timing && p->ev_used + 2 <= static_cast<int>(p->ev.size())) {
      idx = p->ev_used;
      p->ev_used += 2;
      p->ev_family[idx] = fam;
      record(p->ev[idx]);
    }
  }
  ~Timer() {
    if (idx >= 0) record(p->ev[idx + 1]);
    nvtxRangePop();
  }
  // inside a stream capture the event becomes a record node of the graph, so the
  // family times come from the replayed graph
  void record(cudaEvent_t e) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cs);
    if (cs == cudaStreamCaptureStatusActive)
      cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
    else
      cudaEventRecord(e, s);
  }
};

template <typename T>
T* at(oasis_plan* p, size_t off) {
  return reinterpret_cast<T*>(p->ws + off);
}

// A projection GEMM over the M token rows: tile shape from choose_tiles; the residual
// GEMMs (out-proj, fc2) may split K.
int make_proj(GemmOperands* g, const void* A, long long lda, const void* B, long long ldb, int M,
              int N, int K, bool residual = false) {
  int bn = 256, ctas = 1, splits = 1;
  choose_tiles(M, N, K, residual, &bn, &ctas, &splits);
  if (int s = make_gemm_operands(g, A, lda, B, ldb, M, N, K, bn, ctas)) return s;
  g->splits = splits;
  return OASIS_OK;
}

int run_forward(oasis_plan* p, const float* x, const int64_t* t, const float* act, float* v,
                const oasis_kv_cache_t* cache, int n_past, bool cached, cudaStream_t s) {
  const int F = p->F, M = p->M;
  const oasis_dit_weights_t& w = p->w;
  float* resid = at<float>(p, p->L.resid);
  void* hbuf = at<void>(p, p->L.hbuf);
  void* qkv = at<void>(p, p->L.qkv);
  void* attn = at<void>(p, p->L.attn);
  void* mlp = at<void>(p, p->L.mlp);
  float* mod = at<float>(p, p->L.mod);
  const long long mld = p->mod_ld;

  unsigned int* counters = at<unsigned int>(p, p->L.cnt);
  const size_t nblk = row_blocks(static_cast<size_t>(M));
  {
    cudaError_t ce = cudaMemsetAsync(counters, 0, p->zero_bytes, s);
    if (ce != cudaSuccess) return cuda_status(ce, "cudaMemsetAsync(row-block counters)");
  }
  // the residual GEMMs (out-proj, fc2) end with the LayerNorm + modulate that feeds the
  // next GEMM: shift/scale rows and counter slice for launch k
  auto cnt = [&](int j, int c) { return counters + (static_cast<size_t>(j) * kCountersPerSub + c) * nblk; };
  // split-K counters of launch r (0 out-proj, 1 fc2) of sub-block j
  unsigned int* flags0 = counters + p->L.cnt_bytes / 4;
  auto flags = [&](int j, int r) { return flags0 + (static_cast<size_t>(j) * 2 + r) * p->L.flag_words_per_launch; };
  auto ln_tail = [&](EpiParams& ep, const float* shift, unsigned int* tiles_done) {
    ep.ln_out = static_cast<__nv_bfloat16*>(hbuf);
    ep.ln_shift = shift;
    ep.ln_scale = shift + OASIS_HIDDEN;
    ep.ln_mod_ld = mld;
    ep.ln_count = tiles_done;
  };
  const int T = p->frames;
  const int pos0 = cached ? n_past : 0;
  // QKV of sub-block j (RoPE on q and k: axial over the 144 tokens for spatial
  // sub-blocks, over the window position for temporal ones)
  auto qkv_params = [&](int j) {
    EpiParams ep{};
    ep.out = qkv;
    ep.ldd = 3 * OASIS_HIDDEN;
    ep.rope_cols = 2 * OASIS_HIDDEN;
    if (j % 2 == 0) {
      ep.rope = w.rope_spatial;
      ep.rope_div = 1;
      ep.rope_mod = OASIS_TOKENS;
      ep.rope_add = 0;
    } else {
      ep.rope = w.rope_temporal;
      ep.rope_div = OASIS_TOKENS;
      ep.rope_mod = T;
      ep.rope_add = pos0;
    }
    return ep;
  };

  // ---- embeddings (three small tcgen05 GEMMs) ----
  {
    Timer tm(p, s, kFamEmbed);
    if (int e = launch_patch_im2col(x, at<void>(p, p->L.cols), F, s)) return e;
    EpiParams pe{};
    pe.out = resid;
    pe.ldd = OASIS_HIDDEN;
    pe.bias = w.patch_b;
    if (int e = launch_gemm(p->patch, kEpiStoreF32Bias, pe, s)) return e;
    if (int e = launch_temb_prep(t, act, at<void>(p, p->L.emb), at<void>(p, p->L.h1a), F, s))
      return e;
    EpiParams e1{};  // h1 = SiLU(W1 emb + b1) -> h1a[:, 0:1024]
    e1.out = at<void>(p, p->L.h1a);
    e1.ldd = kH1aLd;
    e1.bias = w.t_fc1_b;
    e1.n_valid = F;
    if (int e = launch_gemm(p->temb1, kEpiAdaTSilu, e1, s)) return e;
    EpiParams e2{};  // SiLU(c), c = W2 h1 + Wa a + b2 + ba: the input of every adaLN linear
    e2.out = at<void>(p, p->L.silu);
    e2.ldd = OASIS_HIDDEN;
    e2.bias = w.t_fc2_b;
    e2.n_valid = F;
    if (int e = launch_gemm(p->temb2, kEpiAdaTSilu, e2, s)) return e;
  }
  // ---- all adaLN modulations in one swap-AB GEMM ----
  {
    Timer tm(p, s, kFamAda);
    EpiParams ep{};
    ep.out = mod;
    ep.ldd = mld;
    ep.bias = w.ada_b;
    ep.n_valid = F;
    if (int e = launch_gemm(p->ada, kEpiAdaT, ep, s)) return e;
  }

  KvView kvv;
  if (int e = make_kv_view(cached ? cache : nullptr, &kvv)) return e;

  const bool chain = p->chain;
  for (int j = 0; j < 2 * p->depth; ++j) {
    const bool spatial = (j % 2) == 0;
    const int blk = j / 2;
    const bool last = j == 2 * p->depth - 1;
    const oasis_sub_weights_t& sw = w.sub[j];
    const float* modj = mod + static_cast<long long>(j) * OASIS_ADA_PER_SUB;
    if (j == 0) {  // later LayerNorms are the tails of the residual GEMMs
      Timer tm(p, s, kFamLn);
      if (int e = launch_ln_modulate(resid, modj + 0 * OASIS_HIDDEN, modj + 1 * OASIS_HIDDEN, mld,
                                     hbuf, M, OASIS_TOKENS, s))
        return e;
    }
    if (j == 0 || !chain) {  // otherwise the previous sub-block's chain computed it
      Timer tm(p, s, kFamGemm);
      if (int e = launch_gemm(p->qkv[j], kEpiQkvRope, qkv_params(j), s)) return e;
    }
    if (spatial) {
      Timer tm(p, s, kFamSpatial);
      if (int e = launch_attn_spatial(qkv, attn, F, s)) return e;
    } else {
      if (cache && !cached && T > 1) {
        // post-RoPE K/V of window frames 0..T-2 -> cache slots 0..T-2
        Timer tm(p, s, kFamKv);
        if (int e = launch_kv_store(qkv, 3 * OASIS_HIDDEN, OASIS_HIDDEN, 2 * OASIS_HIDDEN, cache,
                                    blk, p->batch, T - 1, T, 0, s))
          return e;
      }
      Timer tm(p, s, kFamTemporal);
      if (cached) {
        // newest frame at window position n_past: cached slots 0..n_past-1 + its own K/V
        if (int e = launch_attn_temporal(qkv, kvv, blk, attn, p->batch, 1, n_past, n_past,
                                         n_past + 1, s))
          return e;
      } else {
        if (int e = launch_attn_temporal(qkv, kvv, blk, attn, p->batch, T, 0, 0, T, s)) return e;
      }
    }
    EpiParams eo{};  // resid += gate_msa * (attn W_out^T + b); then LayerNorm -> input of fc1
    eo.out = resid;
    eo.ldd = OASIS_HIDDEN;
    eo.bias = sw.out_b;
    eo.gate = modj + 2 * OASIS_HIDDEN;
    eo.gate_ld = mld;
    eo.split_flags = flags(j, 0);
    ln_tail(eo, modj + 3 * OASIS_HIDDEN, cnt(j, 0));
    EpiParams e1{};  // mlp = GELU(h W_1^T + b_1)
    e1.out = mlp;
    e1.ldd = OASIS_MLP_HIDDEN;
    e1.bias = sw.fc1_b;
    EpiParams e2{};  // resid += gate_mlp * (mlp W_2^T + b_2); then LayerNorm -> next QKV / final
    e2.out = resid;
    e2.ldd = OASIS_HIDDEN;
    e2.bias = sw.fc2_b;
    e2.gate = modj + 5 * OASIS_HIDDEN;
    e2.gate_ld = mld;
    e2.split_flags = flags(j, 1);
    ln_tail(e2, modj + OASIS_ADA_PER_SUB, cnt(j, 3));
    Timer tm(p, s, kFamGemm);
    if (chain) {
      ChainStep st[kMaxChainOps];
      // fc1 publishes a bitmask of its finished N tiles per row block; each k-block of fc2
      // waits only for the fc1 tile that produced its 64 columns, so fc2's main loop can
      // start on the tiles of earlier waves while the last fc1 wave is still in flight
      st[0] = ChainStep{&p->out[j], kEpiGateResid, eo, nullptr, 0, cnt(j, 0), cnt(j, 1), false, false};
      st[1] = ChainStep{&p->fc1[j], kEpiBiasGelu, e1, cnt(j, 1), 0, cnt(j, 2), nullptr, true, false};
      st[2] = ChainStep{&p->fc2[j], kEpiGateResid, e2, cnt(j, 2), 0, cnt(j, 3), cnt(j, 4), false, true};
      int n = 3;
      if (!last) st[n++] = ChainStep{&p->qkv[j + 1], kEpiQkvRope, qkv_params(j + 1), cnt(j, 4), 0,
                                     nullptr, nullptr, false, false};
      if (int e = launch_chain(st, n, s)) return e;
    } else {
      if (int e = launch_gemm(p->out[j], kEpiGateResid, eo, s)) return e;
      if (int e = launch_gemm(p->fc1[j], kEpiBiasGelu, e1, s)) return e;
      if (int e = launch_gemm(p->fc2[j], kEpiGateResid, e2, s)) return e;
    }
  }
  // ---- final layer (its LayerNorm + modulate was the last fc2's tail) ----
  {
    Timer tm(p, s, kFamEmbed);
    EpiParams ep{};
    ep.out = v;
    ep.bias = w.final_b;
    if (int e = launch_gemm(p->fin, kEpiFinal, ep, s)) return e;
  }
  return OASIS_OK;
}

}  // namespace
}  // namespace oasis

// ------------------------------------------------------------------ C ABI
using namespace oasis;

extern "C" size_t oasis_plan_workspace_size(int batch, int frames, int depth) {
  if (batch <= 0 || frames <= 0 || depth <= 0) return 0;
  return layout_for(batch * frames, depth).total;
}

namespace oasis {

// Validates the arguments and fills `p` (which may live in static storage): no device
// memory is allocated, only tensor maps are encoded on the host.
int plan_init(oasis_plan* p, const oasis_dit_weights_t* w, int batch, int frames, void* workspace,
              size_t workspace_bytes) {
  if (!w) return fail(OASIS_ERR_INVALID_ARG, "oasis_plan_create: null argument");
  if (batch <= 0 || frames <= 0 || frames > OASIS_MAX_FRAMES)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_plan_create: need batch > 0 and 1 <= frames <= 32");
  if (w->depth <= 0 || w->depth > OASIS_MAX_DEPTH)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_plan_create: depth must be 1..16");
  const int F = batch * frames;
  if (static_cast<long long>(F) * OASIS_TOKENS > (1LL << 30))
    return fail(OASIS_ERR_UNSUPPORTED, "oasis_plan_create: too many tokens");
  Layout L = layout_for(F, w->depth);
  if (!workspace || workspace_bytes < L.total)
    return fail(OASIS_ERR_WORKSPACE, "oasis_plan_create: workspace missing or smaller than "
                                     "oasis_plan_workspace_size()");
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(OASIS_ERR_ALIGNMENT, "oasis_plan_create: workspace must be 256-byte aligned");
  const void* req[] = {w->patch_w, w->patch_b, w->t_fc1_w, w->t_fc1_b, w->t_fc2_w, w->t_fc2_b,
                       w->ada_w,   w->ada_b,   w->final_w, w->final_b, w->rope_spatial,
                       w->rope_temporal};
  for (const void* q : req)
    if (!q) return fail(OASIS_ERR_INVALID_ARG, "oasis_plan_create: a weight pointer is NULL");
  for (int j = 0; j < 2 * w->depth; ++j) {
    const oasis_sub_weights_t& s = w->sub[j];
    if (!s.qkv_w || !s.out_w || !s.out_b || !s.fc1_w || !s.fc1_b || !s.fc2_w || !s.fc2_b)
      return fail(OASIS_ERR_INVALID_ARG, "oasis_plan_create: a sub-block weight pointer is NULL");
  }
  p->w = *w;
  p->batch = batch;
  p->frames = frames;
  p->F = F;
  p->M = F * OASIS_TOKENS;
  p->depth = w->depth;
  p->mod_ld = static_cast<long long>(2 * w->depth) * OASIS_ADA_PER_SUB + 2 * OASIS_HIDDEN;
  p->ws = static_cast<uint8_t*>(workspace);
  p->L = L;
  const int M = p->M;
  int st = OASIS_OK;
  // swap-AB GEMMs over the F conditioning rows: A = weights, B = per-frame vectors
  int bnf = 32;
  while (bnf < 256 && bnf < F) bnf <<= 1;
  st = make_gemm_operands(&p->ada, w->ada_w, OASIS_HIDDEN, p->ws + L.silu, OASIS_HIDDEN,
                          static_cast<int>(p->mod_ld), F, OASIS_HIDDEN, bnf);
  if (!st)
    st = make_gemm_operands(&p->temb1, w->t_fc1_w, 256, p->ws + L.emb, 256, OASIS_HIDDEN, F, 256,
                            bnf);
  if (!st)
    st = make_gemm_operands(&p->temb2, w->t_fc2_w, kH1aLd, p->ws + L.h1a, kH1aLd, OASIS_HIDDEN, F,
                            kH1aLd, bnf);
  if (!st)
    st = make_proj(&p->patch, p->ws + L.cols, 64, w->patch_w, 64, M, OASIS_HIDDEN, 64);
  if (!st) st = set_gemm_output(&p->patch, p->ws + L.resid, OASIS_HIDDEN, true);
  if (!st)
    st = make_gemm_operands(&p->fin, p->ws + L.hbuf, OASIS_HIDDEN, w->final_w, OASIS_HIDDEN, M, 64,
                            OASIS_HIDDEN, 64);
  for (int j = 0; j < 2 * w->depth && !st; ++j) {
    const oasis_sub_weights_t& s = w->sub[j];
    st = make_proj(&p->qkv[j], p->ws + L.hbuf, OASIS_HIDDEN, s.qkv_w, OASIS_HIDDEN, M,
                   3 * OASIS_HIDDEN, OASIS_HIDDEN);
    if (!st) st = set_gemm_output(&p->qkv[j], p->ws + L.qkv, 3 * OASIS_HIDDEN, false);
    if (!st)
      st = make_proj(&p->out[j], p->ws + L.attn, OASIS_HIDDEN, s.out_w, OASIS_HIDDEN, M, OASIS_HIDDEN,
                     OASIS_HIDDEN, true);
    if (!st) st = set_gemm_output(&p->out[j], p->ws + L.resid, OASIS_HIDDEN, true);
    if (!st)
      st = make_proj(&p->fc1[j], p->ws + L.hbuf, OASIS_HIDDEN, s.fc1_w, OASIS_HIDDEN, M,
                     OASIS_MLP_HIDDEN, OASIS_HIDDEN);
    if (!st) st = set_gemm_output(&p->fc1[j], p->ws + L.mlp, OASIS_MLP_HIDDEN, false);
    if (!st)
      st = make_proj(&p->fc2[j], p->ws + L.mlp, OASIS_MLP_HIDDEN, s.fc2_w, OASIS_MLP_HIDDEN, M,
                     OASIS_HIDDEN, OASIS_MLP_HIDDEN, true);
    if (!st) st = set_gemm_output(&p->fc2[j], p->ws + L.resid, OASIS_HIDDEN, true);
  }
  if (st) return st;
  // zeroed per forward: the row-block counters, and split-K counters if any launch splits
  p->zero_bytes = L.cnt_bytes;
  for (int j = 0; j < 2 * w->depth; ++j)
    if (p->out[j].splits > 1 || p->fc2[j].splits > 1) {
      if (split_flag_count(p->out[j]) > L.flag_words_per_launch ||
          split_flag_count(p->fc2[j]) > L.flag_words_per_launch)
        return fail(OASIS_ERR_UNSUPPORTED, "oasis_plan_create: split-K counters exceed their region");
      p->zero_bytes = L.cnt_bytes + static_cast<size_t>(2 * w->depth) * 2 * L.flag_words_per_launch * 4;
    }
  p->chain = true;
  for (int j = 0; j < 2 * w->depth; ++j)
    for (const GemmOperands* g : {&p->qkv[j], &p->out[j], &p->fc1[j], &p->fc2[j]})
      if (g->ctas != 2 || g->bn != 256) p->chain = false;
  // weights are the B operand of these GEMMs (swap-AB GEMMs read activations as B)
  p->patch.b_is_weight = true;
  p->ada.a_is_weight = p->temb1.a_is_weight = p->temb2.a_is_weight = true;
  p->fin.b_is_weight = true;
  for (int j = 0; j < 2 * w->depth; ++j)
    p->qkv[j].b_is_weight = p->out[j].b_is_weight = p->fc1[j].b_is_weight = p->fc2[j].b_is_weight = true;
  return OASIS_OK;
}

int plan_run(oasis_plan* p, const float* x, const int64_t* t, const float* act, float* v,
             const oasis_kv_cache_t* cache, int n_past, bool cached, cudaStream_t s) {
  return run_forward(p, x, t, act, v, cache, n_past, cached, s);
}

}  // namespace oasis

extern "C" int oasis_plan_create(const oasis_dit_weights_t* w, int batch, int frames,
                                 void* workspace, size_t workspace_bytes, oasis_plan_t** out) {
  if (!w || !out) return fail(OASIS_ERR_INVALID_ARG, "oasis_plan_create: null argument");
  *out = nullptr;
  oasis_plan* p = new oasis_plan();
  if (int st = plan_init(p, w, batch, frames, workspace, workspace_bytes)) {
    delete p;
    return st;
  }
  *out = p;
  return OASIS_OK;
}

extern "C" void oasis_plan_destroy(oasis_plan_t* plan) {
  if (!plan) return;
  for (cudaEvent_t e : plan->ev) cudaEventDestroy(e);
  delete plan;
}

static int check_cache_for_plan(const oasis_plan* p, const oasis_kv_cache_t* c, int n_slots_needed) {
  if (c->batch < p->batch || c->layers < p->depth)
    return fail(OASIS_ERR_INVALID_ARG, "KV cache batch/layers smaller than the plan's");
  return validate_slots(c, 0, n_slots_needed);
}

extern "C" int oasis_dit_forward(oasis_plan_t* plan, const float* x, const int64_t* t,
                                 const float* act, float* v, const oasis_kv_cache_t* cache,
                                 cudaStream_t stream) {
  if (!plan || !x || !t || !v) return fail(OASIS_ERR_INVALID_ARG, "oasis_dit_forward: null argument");
  if (!aligned16(x) || !aligned16(v)) return fail(OASIS_ERR_ALIGNMENT, "oasis_dit_forward: x/v alignment");
  if (cache && plan->frames > 1)
    if (int s = check_cache_for_plan(plan, cache, plan->frames - 1)) return s;
  return run_forward(plan, x, t, act, v, cache, 0, false, stream);
}

extern "C" int oasis_dit_forward_cached(oasis_plan_t* plan, const float* x, const int64_t* t,
                                        const float* act, float* v, const oasis_kv_cache_t* cache,
                                        int n_past, cudaStream_t stream) {
  if (!plan || !x || !t || !v || !cache)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_dit_forward_cached: null argument");
  if (plan->frames != 1)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_dit_forward_cached: plan must be built with frames == 1");
  if (n_past < 1 || n_past >= OASIS_MAX_FRAMES)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_dit_forward_cached: need 1 <= n_past <= 31");
  if (!aligned16(x) || !aligned16(v)) return fail(OASIS_ERR_ALIGNMENT, "oasis_dit_forward_cached: alignment");
  if (int s = check_cache_for_plan(plan, cache, n_past)) return s;
  return run_forward(plan, x, t, act, v, cache, n_past, true, stream);
}

extern "C" int oasis_plan_set_timing(oasis_plan_t* plan, int enable) {
  if (!plan) return fail(OASIS_ERR_INVALID_ARG, "oasis_plan_set_timing: null plan");
  if (enable && plan->ev.empty()) {
    const int n = 2 * 8 * (8 * 2 * plan->depth + 8);  // 8 forwards of timed launch groups
    plan->ev.resize(n);
    plan->ev_family.assign(n, 0);
    for (auto& e : plan->ev)
      if (cudaEventCreate(&e) != cudaSuccess) return fail(OASIS_ERR_CUDA, "cudaEventCreate");
  }
  plan->timing = enable != 0;
  plan->ev_used = 0;
  for (int i = 0; i < kFamilies; ++i) {
    plan->fam_ms[i] = 0.0f;
    plan->fam_launches[i] = 0;
  }
  return OASIS_OK;
}

static void harvest_timing(oasis_plan* p) {
  if (p->ev_used == 0) return;
  cudaEventSynchronize(p->ev[p->ev_used - 1]);
  for (int i = 0; i < p->ev_used; i += 2) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, p->ev[i], p->ev[i + 1]) == cudaSuccess) {
      p->fam_ms[p->ev_family[i]] += ms;
      p->fam_launches[p->ev_family[i]] += 1;
    }
  }
  p->ev_used = 0;
}

extern "C" int oasis_plan_get_timing(oasis_plan_t* plan, float* ms, int* launches, int n) {
  if (!plan || !ms || !launches) return fail(OASIS_ERR_INVALID_ARG, "oasis_plan_get_timing: null");
  harvest_timing(plan);
  for (int i = 0; i < n && i < kFamilies; ++i) {
    ms[i] = plan->fam_ms[i];
    launches[i] = plan->fam_launches[i];
  }
  return OASIS_OK;
}
