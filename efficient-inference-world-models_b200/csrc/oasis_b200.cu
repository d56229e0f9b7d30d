// Unity build of liboasis_b200.so: one translation unit so that the device-side
// error word (g_dev_error) is a single object shared by every kernel.
#include "capi.cu"
#include "gemm.cu"
#include "attention.cu"
#include "kv.cu"
#include "elementwise.cu"
#include "forward.cu"
#include "vae.cu"
#include "noalloc.cu"
