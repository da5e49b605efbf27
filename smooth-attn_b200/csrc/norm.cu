// Squareplus normalization, forward and fused backward (memory-bound SIMT).
//
// Reference algorithm: src/smooth_attn/kernels.py
//   forward   :494-531 (row-wise), :565-676 (causal generic / winner / tiered)
//   backward  :679-849 (causal generic / winner / tiered), :1197-1230 (dispatch)
//
// B200 design (not a translation of the Triton kernels):
//   * a "row group" of G threads (G = 1..512, a power of two) owns one row;
//     thread t of the group owns the 16-byte vectors t, t+G, t+2G, ... so a
//     warp's loads and stores are fully coalesced 128-bit transactions;
//   * the whole visible part of the row is loaded into registers with
//     streaming (evict-first) loads before any arithmetic, which keeps
//     CHUNKS x 16 B per thread in flight;
//   * causal rows skip the masked triangle on read (vectors wholly above the
//     diagonal are never loaded) but still write their zeros, so no separate
//     out.zero_() pass and no multi-tier launches are needed;
//   * fp32 accumulation; warp shuffles, then shared memory when G > 32;
//   * one launch per call, grid = ceil(rows / rows-per-CTA).
#include "sa_common.cuh"

namespace sa {

// Sum over the G threads of a row group.  All threads of the CTA call this.
__device__ __forceinline__ float group_sum(float v, int G, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    if (o < G) v += __shfl_xor_sync(0xffffffffu, v, o);
  }
  if (G <= 32) return v;
  const int warp = threadIdx.x >> 5;
  const int wpg = G >> 5;  // warps per group
  __syncthreads();         // red[] may still be read from a previous call
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  const int first = (warp / wpg) * wpg;
  float s = 0.f;
  for (int w = 0; w < wpg; ++w) s += red[first + w];
  return s;
}

__device__ __forceinline__ float family_y(float x, float alpha, float theta, int power) {
  // a = alpha * (x - theta) keeps the reference's rounding order
  // (kernels.py:590); for alpha=2, theta=0.5 it equals the winner's x+x-1.
  const float a = alpha * (x - theta);
  const float u = fmaf(a, a, 4.0f);
  const float sp = 0.5f * (a + fast_sqrt(u));
  float y = sp;
  if (power >= 2) y *= sp;
  if (power == 3) y *= sp;
  return y;
}

template <typename T, int VEC, int CHUNKS, bool CAUSAL>
__global__ void __launch_bounds__(512) norm_fwd_kernel(const T* __restrict__ x, T* __restrict__ out,
                                                       float* __restrict__ rowsum, int64_t rows, int cols,
                                                       int64_t ldx, int64_t ldo, float alpha, float theta,
                                                       int power, int G) {
  __shared__ float red[16];
  const int lane = threadIdx.x & (G - 1);
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / G) + threadIdx.x / G;
  const bool row_ok = row < rows;
  const int nvec = cols / VEC;
  const int q = CAUSAL ? (int)(row % cols) : cols - 1;  // last visible column
  const int nvis = CAUSAL ? (q + VEC) / VEC : nvec;      // vectors holding visible columns

  const T* xr = x + (row_ok ? row : 0) * ldx;
  Pack<T, VEC> in[CHUNKS];
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int v = lane + c * G;
    if (row_ok && v < nvis) load_stream(in[c], xr + (int64_t)v * VEC);
  }

  float y[CHUNKS][VEC];
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int v = lane + c * G;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const int col = v * VEC + e;
      const bool vis = row_ok && v < nvis && col <= q;
      const float yy = vis ? family_y(in[c].get(e), alpha, theta, power) : 0.f;
      y[c][e] = yy;
      sum += yy;
    }
  }
  sum = group_sum(sum, G, red);
  const float S = sum + SA_EPS;
  const float inv = 1.0f / S;
  if (!row_ok) return;
  if (rowsum != nullptr && lane == 0) rowsum[row] = S;

  T* orow = out + row * ldo;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int v = lane + c * G;
    if (v < nvec) {
      Pack<T, VEC> o;
#pragma unroll
      for (int e = 0; e < VEC; ++e) o.set(e, y[c][e] * inv);
      store_stream(orow + (int64_t)v * VEC, o);
    }
  }
}

// VEC consecutive elements of TG held as floats-on-demand: 16-byte vectors
// when VEC * sizeof(TG) is a multiple of 16, scalar loads otherwise.
template <typename TG, int VEC>
struct GradPack {
  static constexpr bool VECTOR = VEC > 1 && (VEC * (int)sizeof(TG)) % 16 == 0;
  static constexpr int PER = VECTOR ? 16 / (int)sizeof(TG) : 1;
  static constexpr int NV = VECTOR ? VEC / PER : VEC;
  Pack<TG, PER> p[NV];
  __device__ __forceinline__ void load(const TG* ptr) {
#pragma unroll
    for (int i = 0; i < NV; ++i) load_stream(p[i], ptr + i * PER);
  }
  __device__ __forceinline__ float get(int e) const { return p[e / PER].get(e % PER); }
};

template <typename T, typename TG, int VEC, int CHUNKS, bool CAUSAL>
__global__ void __launch_bounds__(512) norm_bwd_kernel(const T* __restrict__ x, const TG* __restrict__ g,
                                                       const float* __restrict__ rowsum, T* __restrict__ dx,
                                                       int64_t rows, int cols, int64_t ldx, int64_t ldg,
                                                       int64_t ldd, float alpha, float theta, int power, int G) {
  __shared__ float red[16];
  const int lane = threadIdx.x & (G - 1);
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / G) + threadIdx.x / G;
  const bool row_ok = row < rows;
  const int nvec = cols / VEC;
  const int q = CAUSAL ? (int)(row % cols) : cols - 1;
  const int nvis = CAUSAL ? (q + VEC) / VEC : nvec;
  const int64_t r0 = row_ok ? row : 0;

  Pack<T, VEC> xin[CHUNKS];
  GradPack<TG, VEC> gin[CHUNKS];
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int v = lane + c * G;
    if (row_ok && v < nvis) {
      load_stream(xin[c], x + r0 * ldx + (int64_t)v * VEC);
      gin[c].load(g + r0 * ldg + (int64_t)v * VEC);
    }
  }

  // pass 1: sum y (unless the forward saved it) and sum g*y
  float sum_y = 0.f, sum_gy = 0.f;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int v = lane + c * G;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const int col = v * VEC + e;
      if (row_ok && v < nvis && col <= q) {
        const float yy = family_y(xin[c].get(e), alpha, theta, power);
        sum_y += yy;
        sum_gy += gin[c].get(e) * yy;
      }
    }
  }
  float S;
  if (rowsum != nullptr) {
    S = row_ok ? __ldg(rowsum + r0) : 1.f;
  } else {
    S = group_sum(sum_y, G, red) + SA_EPS;
  }
  sum_gy = group_sum(sum_gy, G, red);
  if (!row_ok) return;
  const float invS = 1.0f / S;
  const float dot = sum_gy * invS;  // sum_k g_k p_k
  const float ap = alpha * (float)power;

  // pass 2: dx = (dy/dx / S) * (g - dot)
  T* drow = dx + row * ldd;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int v = lane + c * G;
    if (v < nvec) {
      Pack<T, VEC> o;
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int col = v * VEC + e;
        float d = 0.f;
        if (v < nvis && col <= q) {
          const float a = alpha * (xin[c].get(e) - theta);
          const float u = fmaf(a, a, 4.0f);
          const float r = rsqrtf(u);
          const float sp = 0.5f * (a + u * r);
          const float spp = 0.5f * fmaf(a, r, 1.0f);
          float dydx = ap * spp;
          if (power >= 2) dydx *= sp;
          if (power == 3) dydx *= sp;
          d = (dydx * invS) * (gin[c].get(e) - dot);
        }
        o.set(e, d);
      }
      store_stream(drow + (int64_t)v * VEC, o);
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static int next_pow2(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static size_t dtype_size(int dt) { return dt == SA_F32 ? 4 : 2; }

struct LaunchShape {
  int G, chunks, threads;
  unsigned grid;
};

static LaunchShape pick_shape(int64_t rows, int cols, int vec, int max_chunks) {
  const int nvec = cols / vec;
  LaunchShape s;
  s.G = next_pow2((nvec + max_chunks - 1) / max_chunks);
  if (s.G < 1) s.G = 1;
  s.chunks = next_pow2((nvec + s.G - 1) / s.G);
  s.threads = s.G > 256 ? s.G : 256;
  const int64_t rpc = s.threads / s.G;
  s.grid = (unsigned)((rows + rpc - 1) / rpc);
  return s;
}

template <typename T, int VEC, bool CAUSAL>
static void launch_fwd_c(const LaunchShape& s, const void* x, void* out, float* rowsum, int64_t rows, int cols,
                         int64_t ldx, int64_t ldo, float alpha, float theta, int power, cudaStream_t st) {
  auto xs = static_cast<const T*>(x);
  auto os = static_cast<T*>(out);
#define SA_FWD(CH)                                                                                      \
  norm_fwd_kernel<T, VEC, CH, CAUSAL><<<s.grid, s.threads, 0, st>>>(xs, os, rowsum, rows, cols, ldx, ldo, \
                                                                     alpha, theta, power, s.G)
  switch (s.chunks) {
    case 1: SA_FWD(1); break;
    case 2: SA_FWD(2); break;
    case 4: SA_FWD(4); break;
    case 8: SA_FWD(8); break;
    default: SA_FWD(16); break;
  }
#undef SA_FWD
}

template <typename T>
static void launch_fwd_t(int vec, bool causal, const LaunchShape& s, const void* x, void* out, float* rowsum,
                         int64_t rows, int cols, int64_t ldx, int64_t ldo, float alpha, float theta, int power,
                         cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  if (vec == V) {
    if (causal) launch_fwd_c<T, V, true>(s, x, out, rowsum, rows, cols, ldx, ldo, alpha, theta, power, st);
    else launch_fwd_c<T, V, false>(s, x, out, rowsum, rows, cols, ldx, ldo, alpha, theta, power, st);
  } else {
    if (causal) launch_fwd_c<T, 1, true>(s, x, out, rowsum, rows, cols, ldx, ldo, alpha, theta, power, st);
    else launch_fwd_c<T, 1, false>(s, x, out, rowsum, rows, cols, ldx, ldo, alpha, theta, power, st);
  }
}

template <typename T, typename TG, int VEC, bool CAUSAL>
static void launch_bwd_c(const LaunchShape& s, const void* x, const void* g, const float* rowsum, void* dx,
                         int64_t rows, int cols, int64_t ldx, int64_t ldg, int64_t ldd, float alpha, float theta,
                         int power, cudaStream_t st) {
  auto xs = static_cast<const T*>(x);
  auto gs = static_cast<const TG*>(g);
  auto ds = static_cast<T*>(dx);
#define SA_BWD(CH)                                                                                          \
  norm_bwd_kernel<T, TG, VEC, CH, CAUSAL><<<s.grid, s.threads, 0, st>>>(xs, gs, rowsum, ds, rows, cols, ldx, \
                                                                         ldg, ldd, alpha, theta, power, s.G)
  switch (s.chunks) {
    case 1: SA_BWD(1); break;
    case 2: SA_BWD(2); break;
    case 4: SA_BWD(4); break;
    default: SA_BWD(8); break;
  }
#undef SA_BWD
}

template <typename T, typename TG>
static void launch_bwd_t(int vec, bool causal, const LaunchShape& s, const void* x, const void* g,
                         const float* rowsum, void* dx, int64_t rows, int cols, int64_t ldx, int64_t ldg,
                         int64_t ldd, float alpha, float theta, int power, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  if (vec == V) {
    if (causal) launch_bwd_c<T, TG, V, true>(s, x, g, rowsum, dx, rows, cols, ldx, ldg, ldd, alpha, theta, power, st);
    else launch_bwd_c<T, TG, V, false>(s, x, g, rowsum, dx, rows, cols, ldx, ldg, ldd, alpha, theta, power, st);
  } else {
    if (causal) launch_bwd_c<T, TG, 1, true>(s, x, g, rowsum, dx, rows, cols, ldx, ldg, ldd, alpha, theta, power, st);
    else launch_bwd_c<T, TG, 1, false>(s, x, g, rowsum, dx, rows, cols, ldx, ldg, ldd, alpha, theta, power, st);
  }
}

}  // namespace sa

int sa_record_cuda_error(cudaError_t e);  // defined in abi.cu

extern "C" int sa_norm_fwd(const void* x, void* out, float* rowsum, int64_t rows, int64_t cols, int64_t ld_x,
                           int64_t ld_out, int dtype, int causal, float alpha, float theta, int power,
                           void* stream) {
  using namespace sa;
  if (dtype != SA_F32 && dtype != SA_F16 && dtype != SA_BF16) return SA_ERR_UNSUPPORTED;
  if (rows < 0 || cols < 1 || cols > 4096) return SA_ERR_ARG;
  if (power < 1 || power > 3) return SA_ERR_ARG;
  if (ld_x < cols || ld_out < cols) return SA_ERR_ARG;
  if (causal && (rows % cols) != 0) return SA_ERR_ARG;
  if (rows == 0) return SA_OK;
  if (x == nullptr || out == nullptr) return SA_ERR_ARG;
  const size_t es = dtype_size(dtype);
  const int V = (int)(16 / es);
  const bool vec_ok = aligned16(x) && aligned16(out) && (cols % V) == 0 && ((ld_x * es) % 16) == 0 &&
                      ((ld_out * es) % 16) == 0;
  const int vec = vec_ok ? V : 1;
  const LaunchShape s = pick_shape(rows, (int)cols, vec, vec == 1 ? 16 : 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SA_F32: launch_fwd_t<float>(vec, causal, s, x, out, rowsum, rows, (int)cols, ld_x, ld_out, alpha, theta, power, st); break;
    case SA_F16: launch_fwd_t<__half>(vec, causal, s, x, out, rowsum, rows, (int)cols, ld_x, ld_out, alpha, theta, power, st); break;
    default: launch_fwd_t<__nv_bfloat16>(vec, causal, s, x, out, rowsum, rows, (int)cols, ld_x, ld_out, alpha, theta, power, st); break;
  }
  return sa_record_cuda_error(cudaGetLastError());
}

extern "C" int sa_norm_bwd(const void* x, const void* g, const float* rowsum, void* dx, int64_t rows, int64_t cols,
                           int64_t ld_x, int64_t ld_g, int64_t ld_dx, int dtype, int g_dtype, int causal,
                           float alpha, float theta, int power, void* stream) {
  using namespace sa;
  if (dtype != SA_F32 && dtype != SA_F16 && dtype != SA_BF16) return SA_ERR_UNSUPPORTED;
  if (g_dtype != SA_F32 && g_dtype != SA_F16 && g_dtype != SA_BF16) return SA_ERR_UNSUPPORTED;
  if (rows < 0 || cols < 1 || cols > 4096) return SA_ERR_ARG;
  if (power < 1 || power > 3) return SA_ERR_ARG;
  if (ld_x < cols || ld_g < cols || ld_dx < cols) return SA_ERR_ARG;
  if (causal && (rows % cols) != 0) return SA_ERR_ARG;
  if (rows == 0) return SA_OK;
  if (x == nullptr || g == nullptr || dx == nullptr) return SA_ERR_ARG;
  const size_t es = dtype_size(dtype), gs = dtype_size(g_dtype);
  const int V = (int)(16 / es);
  const bool vec_ok = aligned16(x) && aligned16(dx) && aligned16(g) && (cols % V) == 0 &&
                      ((ld_x * es) % 16) == 0 && ((ld_dx * es) % 16) == 0 && ((ld_g * gs) % 16) == 0 &&
                      ((size_t)V * gs) % 16 == 0;
  const int vec = vec_ok ? V : 1;
  const LaunchShape s = pick_shape(rows, (int)cols, vec, vec == 1 ? 8 : 4);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int c = (int)cols;
#define SA_BWD_G(T)                                                                                           \
  switch (g_dtype) {                                                                                          \
    case SA_F32: launch_bwd_t<T, float>(vec, causal, s, x, g, rowsum, dx, rows, c, ld_x, ld_g, ld_dx, alpha, theta, power, st); break; \
    case SA_F16: launch_bwd_t<T, __half>(vec, causal, s, x, g, rowsum, dx, rows, c, ld_x, ld_g, ld_dx, alpha, theta, power, st); break; \
    default: launch_bwd_t<T, __nv_bfloat16>(vec, causal, s, x, g, rowsum, dx, rows, c, ld_x, ld_g, ld_dx, alpha, theta, power, st); break; \
  }
  switch (dtype) {
    case SA_F32: SA_BWD_G(float); break;
    case SA_F16: SA_BWD_G(__half); break;
    default: SA_BWD_G(__nv_bfloat16); break;
  }
#undef SA_BWD_G
  return sa_record_cuda_error(cudaGetLastError());
}
