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
int norm_timeouts(int reset, cudaStream_t st);       // norm.cu
int flash_timeouts(int reset, cudaStream_t st);      // flash_fwd.cu
int flash_bwd_timeouts(int reset, cudaStream_t st);  // flash_bwd.cu
int paged_timeouts(int reset, cudaStream_t st);      // paged.cu
int paged_bad_pages(int reset, cudaStream_t st);     // paged.cu
int paged_tc_timeouts(int reset, cudaStream_t st);   // paged_tc.cu
int paged_tc_bad_pages(int reset, cudaStream_t st);  // paged_tc.cu
int proj_timeouts(int reset, cudaStream_t st);       // proj.cu
// index checks that failed, per file (debug library; always 0 in release)
int norm_bounds(int reset, cudaStream_t st);
int flash_fwd_bounds(int reset, cudaStream_t st);
int flash_bwd_bounds(int reset, cudaStream_t st);
int paged_bounds(int reset, cudaStream_t st);
int paged_tc_bounds(int reset, cudaStream_t st);
int rope_bounds(int reset, cudaStream_t st);
int fp8_bounds(int reset, cudaStream_t st);
int proj_bounds(int reset, cudaStream_t st);

// Waits that the probe kernel below gave up on.
__device__ unsigned g_probe_timeouts;

int probe_timeouts(int reset, cudaStream_t st) {
  unsigned v = 0;
  cudaMemcpyFromSymbolAsync(&v, g_probe_timeouts, sizeof(v), 0, cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  if (reset) {
    const unsigned z = 0;
    cudaMemcpyToSymbolAsync(g_probe_timeouts, &z, sizeof(z), 0, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
  }
  return (int)v;
}

// One warp waits, with the library's bounded mbarrier wait, on a barrier
// that nothing arrives on: the wait gives up after limit_ns, the timeout is
// counted like any kernel's, and the kernel returns normally.  No copy or
// MMA is in flight, so nothing else needs to drain.
__global__ void __launch_bounds__(32) bounded_wait_probe(uint64_t limit_ns, int* done) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  const bool ok = mbar_wait(&bar, 0, limit_ns);
  if (threadIdx.x == 0) {
    if (!ok) atomicAdd(&g_probe_timeouts, 1u);
    *done = ok ? 2 : 1;
  }
}

static int collect(int reset, cudaStream_t st) {
  const int n = norm_timeouts(reset, st) + flash_timeouts(reset, st) + flash_bwd_timeouts(reset, st) +
                paged_timeouts(reset, st) + paged_tc_timeouts(reset, st) + probe_timeouts(reset, st) +
                proj_timeouts(reset, st);
  const int bad = paged_bad_pages(reset, st) + paged_tc_bad_pages(reset, st);
  const int oob = norm_bounds(reset, st) + flash_fwd_bounds(reset, st) + flash_bwd_bounds(reset, st) +
                  paged_bounds(reset, st) + paged_tc_bounds(reset, st) + rope_bounds(reset, st) +
                  fp8_bounds(reset, st) + proj_bounds(reset, st);
  return n ? SA_ERR_TIMEOUT : oob ? SA_ERR_BOUNDS : bad ? SA_ERR_ARG : SA_OK;
}
}  // namespace sa

extern "C" int sa_device_status(int reset) {
  if (cudaDeviceSynchronize() != cudaSuccess) return sa_record_cuda_error(cudaGetLastError());
  return sa::collect(reset, nullptr);
}

extern "C" int sa_stream_status(void* stream, int reset) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return sa_record_cuda_error(e);
  return sa::collect(reset, st);
}

extern "C" int sa_probe_bounded_wait(int64_t limit_ns, int* done, void* stream) {
  if (limit_ns <= 0 || limit_ns > 2000000000ll || done == nullptr) return SA_ERR_ARG;
  sa::bounded_wait_probe<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>((uint64_t)limit_ns, done);
  return sa_record_cuda_error(cudaGetLastError());
}

extern "C" int sa_version(void) { return (0 << 16) | 1; }

extern "C" int sa_debug_checks(void) {
#ifdef SA_DEBUG_CHECKS
  return 1;
#else
  return 0;
#endif
}

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
    case SA_ERR_BOUNDS: return "device-side index check failed (debug build)";
    default: return "unknown status";
  }
}
