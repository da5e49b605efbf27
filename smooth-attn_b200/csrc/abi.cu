// C-ABI utilities: version, status strings, last CUDA error (per thread).
#include <stdio.h>
#include <string.h>

#include "sa_common.cuh"

static thread_local char g_last_err[256] = "";

int sa_record_cuda_error(cudaError_t e) {
  if (e == cudaSuccess) return SA_OK;
  snprintf(g_last_err, sizeof(g_last_err), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return SA_ERR_LAUNCH;
}

namespace sa {
int norm_timeouts(int reset);  // norm.cu
int flash_timeouts(int reset);      // flash_fwd.cu
int flash_bwd_timeouts(int reset);  // flash_bwd.cu
int paged_timeouts(int reset);      // paged.cu
int paged_bad_pages(int reset);     // paged.cu
int paged_tc_timeouts(int reset);   // paged_tc.cu
int paged_tc_bad_pages(int reset);  // paged_tc.cu
}  // namespace sa

extern "C" int sa_device_status(int reset) {
  if (cudaDeviceSynchronize() != cudaSuccess) return sa_record_cuda_error(cudaGetLastError());
  const int n = sa::norm_timeouts(reset) + sa::flash_timeouts(reset) + sa::flash_bwd_timeouts(reset) +
                sa::paged_timeouts(reset) + sa::paged_tc_timeouts(reset);
  const int bad = sa::paged_bad_pages(reset) + sa::paged_tc_bad_pages(reset);
  return n ? SA_ERR_TIMEOUT : bad ? SA_ERR_ARG : SA_OK;
}

extern "C" int sa_version(void) { return (0 << 16) | 1; }

extern "C" const char* sa_last_cuda_error(void) { return g_last_err; }

extern "C" const char* sa_status_string(int status) {
  switch (status) {
    case SA_OK: return "ok";
    case SA_ERR_ARG: return "invalid argument";
    case SA_ERR_ALIGN: return "unsupported pointer or stride alignment";
    case SA_ERR_UNSUPPORTED: return "unsupported dtype, head dim or shape";
    case SA_ERR_LAUNCH: return "CUDA launch failed";
    case SA_ERR_TIMEOUT: return "device-side wait timed out";
    case SA_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}
