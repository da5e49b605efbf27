// C-ABI utilities: version, status strings, last CUDA error (per thread),
// and the host-buffer helpers of the causal norm's host path.
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>
#if defined(__x86_64__)
#include <emmintrin.h>
#endif

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

extern "C" int sa_copy_causal_bands(void* dst, const void* src, int64_t nmat, int64_t L, int64_t elem_bytes,
                                    int64_t band, int to_device, int64_t* bytes_out, void* stream) {
  if (bytes_out != nullptr) *bytes_out = 0;
  if (nmat < 0 || L < 0 || band <= 0 || band % 8 != 0 || (elem_bytes != 2 && elem_bytes != 4)) return SA_ERR_ARG;
  if (nmat == 0 || L == 0) return SA_OK;
  if (dst == nullptr || src == nullptr) return SA_ERR_ARG;
  const int64_t vec = 16 / elem_bytes;
  const size_t pitch = (size_t)(L * elem_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t moved = 0;
  for (int64_t r0 = 0; r0 < L; r0 += band) {
    const int64_t r1 = r0 + band < L ? r0 + band : L;
    int64_t w = (r1 + vec - 1) / vec * vec;
    if (w > L) w = L;
    cudaMemcpy3DParms cp = {};
    // pitched pointers whose "height" is L rows, so one depth step is one whole matrix
    cp.srcPtr = make_cudaPitchedPtr(const_cast<char*>(static_cast<const char*>(src)) + r0 * pitch, pitch,
                                    (size_t)(w * elem_bytes), (size_t)L);
    cp.dstPtr = make_cudaPitchedPtr(static_cast<char*>(dst) + r0 * pitch, pitch, (size_t)(w * elem_bytes), (size_t)L);
    cp.extent = make_cudaExtent((size_t)(w * elem_bytes), (size_t)(r1 - r0), (size_t)nmat);
    cp.kind = to_device ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost;
    const cudaError_t e = cudaMemcpy3DAsync(&cp, st);
    if (e != cudaSuccess) return sa_record_cuda_error(e);
    moved += (r1 - r0) * w * elem_bytes * nmat;
  }
  if (bytes_out != nullptr) *bytes_out = moved;
  return SA_OK;
}

// Zeros [p, p + bytes): 16-byte non-temporal stores for the aligned middle
// (no read-for-ownership of lines that are only overwritten), memset around it.
static void zero_bytes(char* p, size_t bytes) {
#if defined(__x86_64__)
  char* a = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15));
  if (a > p + bytes) a = p + bytes;
  memset(p, 0, (size_t)(a - p));
  const size_t mid = (bytes - (size_t)(a - p)) & ~size_t(15);
  const __m128i z = _mm_setzero_si128();
  for (size_t i = 0; i < mid; i += 16) _mm_stream_si128(reinterpret_cast<__m128i*>(a + i), z);
  memset(a + mid, 0, bytes - (size_t)(a - p) - mid);
#else
  memset(p, 0, bytes);
#endif
}

extern "C" int sa_host_zero_causal_tail(void* out, int64_t nmat, int64_t L, int64_t elem_bytes, int64_t band,
                                        int nthreads) {
  if (nmat < 0 || L < 0 || band <= 0 || band % 8 != 0 || (elem_bytes != 2 && elem_bytes != 4)) return SA_ERR_ARG;
  if (nmat == 0 || L == 0) return SA_OK;
  if (out == nullptr) return SA_ERR_ARG;
  int nt = nthreads > 0 ? nthreads : (int)std::thread::hardware_concurrency();
  nt = std::max(1, std::min(nt, 32));
  nt = (int)std::min<int64_t>(nt, nmat);
  const int64_t vec = 16 / elem_bytes;
  auto work = [&](int64_t m0, int64_t m1) {
    for (int64_t m = m0; m < m1; ++m) {
      char* base = static_cast<char*>(out) + (size_t)m * (size_t)(L * L * elem_bytes);
      for (int64_t r0 = 0; r0 < L; r0 += band) {
        const int64_t r1 = std::min(L, r0 + band);
        const int64_t w = std::min(L, (r1 + vec - 1) / vec * vec);
        if (w >= L) continue;
        for (int64_t r = r0; r < r1; ++r)
          zero_bytes(base + (size_t)(r * L + w) * (size_t)elem_bytes, (size_t)((L - w) * elem_bytes));
      }
    }
#if defined(__x86_64__)
    _mm_sfence();  // the streaming stores are globally visible before this thread is joined
#endif
  };
  std::vector<std::thread> th;
  for (int t = 1; t < nt; ++t) th.emplace_back(work, nmat * t / nt, nmat * (t + 1) / nt);
  work(0, nmat / nt);
  for (auto& x : th) x.join();
  return SA_OK;
}

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
