// oasis_dit_forward_noalloc: the full-window DiT forward for callers that cannot
// allocate device memory.
//
// Some hosts of this library may not call cudaMalloc at all: a process embedding the
// forward inside a real-time loop whose memory budget is fixed up front, a plug-in
// that runs inside another framework's stream capture (where a cudaMalloc would
// break the capture), or a runtime that forbids allocator calls after start-up.
// For them this entry point takes only inputs and outputs; its scratch (the
// activations of the forward) lives in a file-scope device array of fixed size,
// so every GPU that loads this library holds those bytes until the process exits.
#include <mutex>

#include "gemm.cuh"
#include "launch.cuh"

namespace oasis {

int plan_init(oasis_plan* p, const oasis_dit_weights_t* w, int batch, int frames, void* workspace,
              size_t workspace_bytes);
int plan_run(oasis_plan* p, const float* x, const int64_t* t, const float* act, float* v,
             const oasis_kv_cache_t* cache, int n_past, bool cached, cudaStream_t s);

namespace {

// 17 MiB: the workspace of a depth-16 forward of batch * frames = 4 (16.3 MB), rounded up.
constexpr size_t kNoAllocScratchBytes = 17u << 20;
constexpr int kMaxDevices = 16;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocState {
  void* scratch = nullptr;          // device address of g_noalloc_scratch on this device
  oasis_plan plan;                  // descriptors for the last (weights, batch, frames)
  oasis_dit_weights_t key_w{};
  int key_batch = 0, key_frames = 0;
  bool plan_valid = false;
};

std::mutex g_noalloc_mutex;
NoAllocState g_noalloc[kMaxDevices];

}  // namespace
}  // namespace oasis

using namespace oasis;

extern "C" int oasis_dit_forward_noalloc(const oasis_dit_weights_t* w, int batch, int frames,
                                         const float* x, const int64_t* t, const float* act,
                                         float* v, cudaStream_t stream) {
  if (!w || !x || !t || !v) return fail(OASIS_ERR_INVALID_ARG, "oasis_dit_forward_noalloc: null argument");
  if (batch <= 0 || frames <= 0 || batch * frames > OASIS_NOALLOC_MAX_FRAMES)
    return fail(OASIS_ERR_UNSUPPORTED,
                "oasis_dit_forward_noalloc: batch * frames must be 1.." +
                    std::to_string(OASIS_NOALLOC_MAX_FRAMES) + " (its scratch is a fixed " +
                    std::to_string(kNoAllocScratchBytes >> 20) + " MiB device array)");
  if (w->depth <= 0 || w->depth > OASIS_MAX_DEPTH)
    return fail(OASIS_ERR_INVALID_ARG, "oasis_dit_forward_noalloc: depth must be 1..16");
  const size_t need = oasis_plan_workspace_size(batch, frames, w->depth);
  if (need == 0 || need > kNoAllocScratchBytes)
    return fail(OASIS_ERR_UNSUPPORTED, "oasis_dit_forward_noalloc: shape needs more scratch than "
                                       "the fixed device array");
  if (!aligned16(x) || !aligned16(v)) return fail(OASIS_ERR_ALIGNMENT, "oasis_dit_forward_noalloc: x/v alignment");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "oasis_dit_forward_noalloc(cudaGetDevice)");
  if (dev < 0 || dev >= kMaxDevices) return fail(OASIS_ERR_UNSUPPORTED, "oasis_dit_forward_noalloc: device index");

  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoAllocState& st = g_noalloc[dev];
  {
    // the array's device address on this device (current here); the host-side name of a
    // __device__ array is not a device pointer.  Looked up on every call: after a device
    // reset or in a new context the array can live elsewhere, and the cached plan's
    // tensor maps point into it, so a changed address rebuilds the plan.
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "oasis_dit_forward_noalloc(cudaGetSymbolAddress)");
    if (addr != st.scratch) {
      st.scratch = addr;
      st.plan_valid = false;
    }
  }
  if (!st.plan_valid || st.key_batch != batch || st.key_frames != frames ||
      std::memcmp(&st.key_w, w, sizeof(*w)) != 0) {
    st.plan_valid = false;
    if (int s = plan_init(&st.plan, w, batch, frames, st.scratch, kNoAllocScratchBytes)) return s;
    st.key_w = *w;
    st.key_batch = batch;
    st.key_frames = frames;
    st.plan_valid = true;
  }
  return plan_run(&st.plan, x, t, act, v, nullptr, 0, false, stream);
}
