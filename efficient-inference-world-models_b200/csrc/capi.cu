// Status plumbing shared by every entry point of the C ABI.
#include <cstdio>
#include <string>

#include "launch.cuh"

namespace oasis {

namespace {
thread_local std::string t_last_error;
}

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return OASIS_ERR_CUDA;
}

}  // namespace oasis

extern "C" const char* oasis_last_error(void) { return oasis::t_last_error.c_str(); }

extern "C" const char* oasis_version(void) { return "oasis_b200 0.1 (sm_100a)"; }

extern "C" int oasis_check_device_error(void) {
  unsigned int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return oasis::cuda_status(e, "oasis_check_device_error(sync)");
  e = cudaMemcpyFromSymbol(&v, oasis::g_dev_error, sizeof(v));
  if (e != cudaSuccess) return oasis::cuda_status(e, "oasis_check_device_error(read)");
  if (v) {
    const unsigned int zero = 0;
    cudaMemcpyToSymbol(oasis::g_dev_error, &zero, sizeof(zero));
    return oasis::fail(OASIS_ERR_DEVICE_TIMEOUT, "a device-side bounded wait gave up");
  }
  return OASIS_OK;
}
