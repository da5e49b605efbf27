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
// Bulk-copy pipelined kernels (16-byte aligned rows: the fast path)
//
// Every warp is an independent persistent worker with a private ring of NST
// shared-memory row slots.  Lane 0 streams the visible bytes of the warp's
// upcoming rows into the ring with 1-D cp.async.bulk copies (completion
// counted on one mbarrier per slot), so up to NST rows per warp are in flight
// without holding registers; the lanes then read the row from shared memory
// with conflict-free 16-byte loads, reduce with warp shuffles and store the
// full output row (zeros included) with 16-byte streaming stores.
// ---------------------------------------------------------------------------

static __device__ unsigned g_norm_timeouts;  // bounded-wait failures (never traps)

constexpr int kBulkWarps = 4;     // warps per CTA
constexpr int kMaxStages = 8;     // slots per warp (upper bound)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Wait (bounded) on a slot; warp-uniform result.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t phase) {
  const bool ok = __all_sync(0xffffffffu, mbar_wait(bar, phase));
  if (!ok && (threadIdx.x & 31) == 0) atomicAdd(&g_norm_timeouts, 1u);
  return ok;
}

// 2^p * squareplus(a)^p with a = c1*x + c0 (c1 = alpha, c0 = -alpha*theta).
// t = a + sqrt(a^2+4) is exactly 2*squareplus(a); carrying y' = t^p = 2^p y
// instead of y drops the two 0.5 factors and scales every y, the row sum and
// EPS by the same power of two, so out = y'/S' equals y/S to the rounding.
// (For the default family, fma(x, 2, -1) is bit-identical to the
// reference's x + x - 1.)
template <bool P2>
__device__ __forceinline__ float y_scaled(float x, float c1, float c0, int power) {
  const float a = fmaf(x, c1, c0);
  const float u = fmaf(a, a, 4.0f);
  const float t = fmaf(u, rsqrt_approx(u), a);
  if (P2) return t * t;
  float y = t;
  if (power >= 2) y *= t;
  if (power == 3) y *= t;
  return y;
}

// fwd: CH = 16-byte vectors per lane held in registers, or 0 for rows too
// long to hold (then y is recomputed from shared memory in a second pass).
template <typename T, int CH, bool CAUSAL, bool P2>
__global__ void __launch_bounds__(kBulkWarps * 32) norm_fwd_bulk(const T* __restrict__ x, T* __restrict__ out,
                                                                 float* __restrict__ rowsum, int64_t rows, int cols,
                                                                 int64_t ldx, int64_t ldo, float c1, float c0,
                                                                 int power, float eps_s, float s_unscale, int nst,
                                                                 int sb) {
  constexpr int VEC = 16 / sizeof(T);
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kMaxStages;
  uint8_t* ring = smem + kBulkWarps * kMaxStages * 8 + (size_t)warp * nst * sb;
  const int64_t nw = (int64_t)gridDim.x * kBulkWarps;
  const int64_t first = (int64_t)blockIdx.x * kBulkWarps + warp;
  const int nvec = cols / VEC;

  auto issue = [&](int64_t row, int s) {
    const int q = CAUSAL ? (int)(row % cols) : cols - 1;
    uint32_t bytes = (uint32_t)((q + VEC) / VEC) * 16u;
    if (!SA_DCHECK(bytes <= (uint32_t)sb && row < rows)) bytes = 16u;  // the row must fit its ring slot
    mbar_arrive_expect_tx(&bars[s], bytes);
    bulk_g2s(ring + (size_t)s * sb, x + row * ldx, bytes, &bars[s]);
  };
  if (lane == 0) {
    for (int s = 0; s < nst; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    for (int s = 0; s < nst; ++s) {
      const int64_t r = first + s * nw;
      if (r < rows) issue(r, s);
    }
  }
  __syncwarp();

  int k = 0;
  for (int64_t row = first; row < rows; row += nw, ++k) {
    const int s = k % nst;
    if (!warp_wait(&bars[s], (uint32_t)(k / nst) & 1u)) return;
    const int q = CAUSAL ? (int)(row % cols) : cols - 1;
    const int nvis = (q + VEC) / VEC;
    const int qe = q - (nvis - 1) * VEC;  // last visible element inside the diagonal vector
    const uint8_t* slot = ring + (size_t)s * sb;
    T* orow = out + row * ldo;
    float sum = 0.f;
    if constexpr (CH > 0) {
      float y[CH][VEC];
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int v = lane + 32 * c;
        if (32 * c < nvis) {  // warp-uniform
          if (v < nvis) {
            float xf[VEC];
            unpack<T, VEC>(slot + (size_t)v * 16, xf);
            if constexpr (P2 && VEC % 2 == 0) {  // pairs per packed fp32x2 instruction
#pragma unroll
              for (int e = 0; e < VEC; e += 2) {
                const float2 a = ffma2(make_float2(xf[e], xf[e + 1]), make_float2(c1, c1), make_float2(c0, c0));
                const float2 u = ffma2(a, a, make_float2(4.0f, 4.0f));
                const float2 t = ffma2(u, make_float2(rsqrt_approx(u.x), rsqrt_approx(u.y)), a);
                const float2 yy = fmul2(t, t);
                y[c][e] = yy.x;
                y[c][e + 1] = yy.y;
              }
            } else {
#pragma unroll
              for (int e = 0; e < VEC; ++e) y[c][e] = y_scaled<P2>(xf[e], c1, c0, power);
            }
            if (CAUSAL && v == nvis - 1) {
#pragma unroll
              for (int e = 0; e < VEC; ++e) y[c][e] = e > qe ? 0.f : y[c][e];
            }
#pragma unroll
            for (int e = 0; e < VEC; ++e) sum += y[c][e];
          }
        }
      }
      __syncwarp();
      if (lane == 0 && row + nst * nw < rows) issue(row + nst * nw, s);  // slot consumed
      const float S = warp_sum(sum) + eps_s;
      const float inv = 1.0f / S;
      if (rowsum != nullptr && lane == 0) rowsum[row] = S * s_unscale;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int v = lane + 32 * c;
        if (v < nvec) {
          Pack<T, VEC> o;
          if (32 * c < nvis && v < nvis) {
#pragma unroll
            for (int e = 0; e < VEC; e += 2) {
              const float2 r = fmul2(make_float2(y[c][e], y[c][e + 1]), make_float2(inv, inv));
              o.set(e, r.x);
              o.set(e + 1, r.y);
            }
          } else {
            o.zero();
          }
          store_stream(orow + (int64_t)v * VEC, o);
        }
      }
    } else {
      const int nfull = CAUSAL ? nvis - 1 : nvis;  // vectors with no masked element
      for (int v = lane; v < nfull; v += 32) {
        float xf[VEC];
        unpack<T, VEC>(slot + (size_t)v * 16, xf);
#pragma unroll
        for (int e = 0; e < VEC; ++e) sum += y_scaled<P2>(xf[e], c1, c0, power);
      }
      if (CAUSAL && lane == (nvis - 1) % 32) {
        float xf[VEC];
        unpack<T, VEC>(slot + (size_t)(nvis - 1) * 16, xf);
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (e <= qe) sum += y_scaled<P2>(xf[e], c1, c0, power);
      }
      const float S = warp_sum(sum) + eps_s;
      const float inv = 1.0f / S;
      if (rowsum != nullptr && lane == 0) rowsum[row] = S * s_unscale;
      for (int v = lane; v < nvec; v += 32) {
        Pack<T, VEC> o;
        if (v < nvis) {
          float xf[VEC];
          unpack<T, VEC>(slot + (size_t)v * 16, xf);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const float yy = y_scaled<P2>(xf[e], c1, c0, power);
            o.set(e, (CAUSAL && v == nvis - 1 && e > qe) ? 0.f : yy * inv);
          }
        } else {
          o.zero();
        }
        store_stream(orow + (int64_t)v * VEC, o);
      }
      __syncwarp();
      if (lane == 0 && row + nst * nw < rows) issue(row + nst * nw, s);
    }
  }
}

// bwd: a slot holds the visible part of the x row followed (at offset gofs)
// by the visible part of the g row; y is recomputed in the second pass.
//   t = 2 sp, w = 2 sp' = 1 + a rsqrt(a^2+4)
//   dy/dx = alpha p sp^(p-1) sp' = kp t^(p-1) w,   kp = alpha p / 2^p
template <typename T, typename TG, bool CAUSAL, bool P2>
__global__ void __launch_bounds__(kBulkWarps * 32) norm_bwd_bulk(const T* __restrict__ x, const TG* __restrict__ g,
                                                                 const float* __restrict__ rowsum, T* __restrict__ dx,
                                                                 int64_t rows, int cols, int64_t ldx, int64_t ldg,
                                                                 int64_t ldd, float c1, float c0, int power,
                                                                 float eps_s, float s_scale, float kp, int nst, int sb,
                                                                 int gofs) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int GB = VEC * (int)sizeof(TG);  // bytes of g per x vector (8, 16 or 32)
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kMaxStages;
  uint8_t* ring = smem + kBulkWarps * kMaxStages * 8 + (size_t)warp * nst * sb;
  const int64_t nw = (int64_t)gridDim.x * kBulkWarps;
  const int64_t first = (int64_t)blockIdx.x * kBulkWarps + warp;
  const int nvec = cols / VEC;

  auto issue = [&](int64_t row, int s) {
    const int q = CAUSAL ? (int)(row % cols) : cols - 1;
    const int nv = (q + VEC) / VEC;
    uint32_t bx = (uint32_t)nv * 16u;
    uint32_t bg = ((uint32_t)nv * GB + 15u) & ~15u;  // in-row: cols*sizeof(TG) % 16 == 0
    if (!SA_DCHECK(bx <= (uint32_t)gofs && (uint32_t)gofs + bg <= (uint32_t)sb && row < rows)) bx = bg = 16u;  // x and dY fit the slot
    mbar_arrive_expect_tx(&bars[s], bx + bg);
    bulk_g2s(ring + (size_t)s * sb, x + row * ldx, bx, &bars[s]);
    bulk_g2s(ring + (size_t)s * sb + gofs, g + row * ldg, bg, &bars[s]);
  };
  if (lane == 0) {
    for (int s = 0; s < nst; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    for (int s = 0; s < nst; ++s) {
      const int64_t r = first + s * nw;
      if (r < rows) issue(r, s);
    }
  }
  __syncwarp();

  int k = 0;
  for (int64_t row = first; row < rows; row += nw, ++k) {
    const int s = k % nst;
    if (!warp_wait(&bars[s], (uint32_t)(k / nst) & 1u)) return;
    const int q = CAUSAL ? (int)(row % cols) : cols - 1;
    const int nvis = (q + VEC) / VEC;
    const int qe = q - (nvis - 1) * VEC;
    const uint8_t* sx = ring + (size_t)s * sb;
    const uint8_t* sg = sx + gofs;
    float sum_y = 0.f, sum_gy = 0.f;
    for (int v = lane; v < nvis; v += 32) {
      float xf[VEC], gf[VEC];
      unpack<T, VEC>(sx + (size_t)v * 16, xf);
      unpack<TG, VEC>(sg + (size_t)v * GB, gf);
      const int lim = (CAUSAL && v == nvis - 1) ? qe : VEC - 1;
      if constexpr (P2 && VEC % 2 == 0) {
        // power 2: pairs of elements per packed fp32x2 instruction
        // (bit-identical per element; the sums keep two partial lanes)
        float2 sy2 = make_float2(0.f, 0.f), sgy2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int e = 0; e < VEC; e += 2) {
          const float2 a = ffma2(make_float2(xf[e], xf[e + 1]), make_float2(c1, c1), make_float2(c0, c0));
          const float2 u = ffma2(a, a, make_float2(4.0f, 4.0f));
          const float2 t = ffma2(u, make_float2(rsqrt_approx(u.x), rsqrt_approx(u.y)), a);
          float2 yy = fmul2(t, t);
          yy.x = e <= lim ? yy.x : 0.f;
          yy.y = e + 1 <= lim ? yy.y : 0.f;
          sy2 = fadd2(sy2, yy);
          sgy2 = ffma2(make_float2(gf[e], gf[e + 1]), yy, sgy2);
        }
        sum_y += sy2.x + sy2.y;
        sum_gy += sgy2.x + sgy2.y;
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float yy = e <= lim ? y_scaled<P2>(xf[e], c1, c0, power) : 0.f;
          sum_y += yy;
          sum_gy = fmaf(gf[e], yy, sum_gy);
        }
      }
    }
    const float Sp = rowsum != nullptr ? __ldg(rowsum + row) * s_scale : warp_sum(sum_y) + eps_s;  // S' = 2^p S
    const float invSp = 1.0f / Sp;
    const float dot = warp_sum(sum_gy) * invSp;  // sum_k g_k p_k
    const float kr = kp * (invSp * s_scale);     // kp / S
    T* drow = dx + row * ldd;
    for (int v = lane; v < nvec; v += 32) {
      Pack<T, VEC> o;
      if (v < nvis) {
        float xf[VEC], gf[VEC];
        unpack<T, VEC>(sx + (size_t)v * 16, xf);
        unpack<TG, VEC>(sg + (size_t)v * GB, gf);
        const int lim = (CAUSAL && v == nvis - 1) ? qe : VEC - 1;
        if constexpr (P2 && VEC % 2 == 0) {
#pragma unroll
          for (int e = 0; e < VEC; e += 2) {
            const float2 a = ffma2(make_float2(xf[e], xf[e + 1]), make_float2(c1, c1), make_float2(c0, c0));
            const float2 u = ffma2(a, a, make_float2(4.0f, 4.0f));
            const float2 r = make_float2(rsqrt_approx(u.x), rsqrt_approx(u.y));
            const float2 w = ffma2(a, r, make_float2(1.0f, 1.0f));
            const float2 dydx = fmul2(fmul2(make_float2(kr, kr), w), ffma2(u, r, a));
            const float2 res = fmul2(dydx, fsub2(make_float2(gf[e], gf[e + 1]), make_float2(dot, dot)));
            o.set(e, e <= lim ? res.x : 0.f);
            o.set(e + 1, e + 1 <= lim ? res.y : 0.f);
          }
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const float a = fmaf(xf[e], c1, c0);
            const float u = fmaf(a, a, 4.0f);
            const float r = rsqrt_approx(u);
            const float w = fmaf(a, r, 1.0f);
            float dydx = kr * w;
            if (P2) {
              dydx *= fmaf(u, r, a);
            } else if (power >= 2) {
              const float t = fmaf(u, r, a);
              dydx *= t;
              if (power == 3) dydx *= t;
            }
            o.set(e, e <= lim ? dydx * (gf[e] - dot) : 0.f);
          }
        }
      } else {
        o.zero();
      }
      store_stream(drow + (int64_t)v * VEC, o);
    }
    __syncwarp();
    if (lane == 0 && row + nst * nw < rows) issue(row + nst * nw, s);
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


static int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// Ring slots per warp: rows of 8 KB and more get one slot; shorter rows get
// 2..8 slots within ~6 KB per warp.  Small rings leave room for more CTAs
// (warps) per SM, which this latency-bound per-row loop needs more than deep
// per-warp prefetch (measured on B200: bf16 L=1024 3.6 -> 5.1 TB/s, L=2048
// 5.8 -> 5.85 TB/s against a 14 KB-per-warp ring).

struct BulkShape {
  int nst, sb;
  size_t smem;
};

static BulkShape bulk_shape(int slot_bytes) {
  BulkShape b;
  b.sb = (slot_bytes + 127) & ~127;
  b.nst = b.sb >= 8192 ? 1 : 6144 / b.sb;
  if (b.sb < 8192 && b.nst < 2) b.nst = 2;
  if (b.nst > kMaxStages) b.nst = kMaxStages;
  b.smem = (size_t)kBulkWarps * kMaxStages * 8 + (size_t)kBulkWarps * b.nst * b.sb;
  return b;
}

template <typename K>
static unsigned bulk_grid(K kernel, size_t smem, int64_t rows) {
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kBulkWarps * 32, smem);
  if (occ < 1) occ = 1;
  const int64_t want = (rows + kBulkWarps - 1) / kBulkWarps;
  const int64_t cap = (int64_t)sm_count() * occ;
  return (unsigned)(want < cap ? want : cap);
}

struct FamConst {
  float c1, c0, eps_s, s_scale, s_unscale, kp;
  bool p2;
};

static FamConst fam_const(float alpha, float theta, int power) {
  FamConst f;
  const float two_p = (float)(1 << power);
  f.c1 = alpha;
  f.c0 = -alpha * theta;
  f.eps_s = SA_EPS * two_p;
  f.s_scale = two_p;
  f.s_unscale = 1.0f / two_p;
  f.kp = alpha * (float)power / two_p;
  f.p2 = power == 2;
  return f;
}

template <typename T, int CH, bool CAUSAL, bool P2>
static void fwd_bulk_launch(const void* x, void* out, float* rowsum, int64_t rows, int cols, int64_t ldx,
                            int64_t ldo, const FamConst& f, int power, cudaStream_t st) {
  const BulkShape b = bulk_shape(cols * (int)sizeof(T));
  auto k = norm_fwd_bulk<T, CH, CAUSAL, P2>;
  const unsigned grid = bulk_grid(k, b.smem, rows);
  k<<<grid, kBulkWarps * 32, b.smem, st>>>(static_cast<const T*>(x), static_cast<T*>(out), rowsum, rows, cols,
                                            ldx, ldo, f.c1, f.c0, power, f.eps_s, f.s_unscale, b.nst, b.sb);
}

template <typename T, bool CAUSAL>
static void fwd_bulk_t(const void* x, void* out, float* rowsum, int64_t rows, int cols, int64_t ldx, int64_t ldo,
                       float alpha, float theta, int power, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  const FamConst f = fam_const(alpha, theta, power);
  const int nvec = cols / VEC;
  int ch = next_pow2((nvec + 31) / 32);
  if (ch * VEC > 64) ch = 0;
#define SA_FB(CH)                                                                                        \
  do {                                                                                                   \
    if (f.p2) fwd_bulk_launch<T, CH, CAUSAL, true>(x, out, rowsum, rows, cols, ldx, ldo, f, power, st);  \
    else fwd_bulk_launch<T, CH, CAUSAL, false>(x, out, rowsum, rows, cols, ldx, ldo, f, power, st);      \
  } while (0)
  switch (ch) {
    case 1: SA_FB(1); break;
    case 2: SA_FB(2); break;
    case 4: SA_FB(4); break;
    case 8: SA_FB(8); break;
    case 16: if constexpr (VEC <= 4) { SA_FB(16); } else { SA_FB(0); } break;
    default: SA_FB(0); break;
  }
#undef SA_FB
}

template <typename T, typename TG, bool CAUSAL, bool P2>
static void bwd_bulk_launch(const void* x, const void* g, const float* rowsum, void* dx, int64_t rows, int cols,
                            int64_t ldx, int64_t ldg, int64_t ldd, const FamConst& f, int power, cudaStream_t st) {
  const int gofs = (cols * (int)sizeof(T) + 15) & ~15;
  const int gbytes = (cols * (int)sizeof(TG) + 15) & ~15;
  const BulkShape b = bulk_shape(gofs + gbytes);
  auto k = norm_bwd_bulk<T, TG, CAUSAL, P2>;
  const unsigned grid = bulk_grid(k, b.smem, rows);
  k<<<grid, kBulkWarps * 32, b.smem, st>>>(static_cast<const T*>(x), static_cast<const TG*>(g), rowsum,
                                            static_cast<T*>(dx), rows, cols, ldx, ldg, ldd, f.c1, f.c0, power,
                                            f.eps_s, f.s_scale, f.kp, b.nst, b.sb, gofs);
}

template <typename T, typename TG>
static void bwd_bulk_t(bool causal, const void* x, const void* g, const float* rowsum, void* dx, int64_t rows,
                       int cols, int64_t ldx, int64_t ldg, int64_t ldd, float alpha, float theta, int power,
                       cudaStream_t st) {
  const FamConst f = fam_const(alpha, theta, power);
#define SA_BB(C, P) bwd_bulk_launch<T, TG, C, P>(x, g, rowsum, dx, rows, cols, ldx, ldg, ldd, f, power, st)
  if (causal) {
    if (f.p2) SA_BB(true, true); else SA_BB(true, false);
  } else {
    if (f.p2) SA_BB(false, true); else SA_BB(false, false);
  }
#undef SA_BB
}

int norm_timeouts(int reset, cudaStream_t st) {
  unsigned v = 0;
  cudaMemcpyFromSymbolAsync(&v, g_norm_timeouts, sizeof(v), 0, cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  if (reset) {
    const unsigned z = 0;
    cudaMemcpyToSymbolAsync(g_norm_timeouts, &z, sizeof(z), 0, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
  }
  return (int)v;
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
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (vec_ok) {
    const int c = (int)cols;
#define SA_FWD_BULK(T)                                                                               \
    if (causal) fwd_bulk_t<T, true>(x, out, rowsum, rows, c, ld_x, ld_out, alpha, theta, power, st); \
    else fwd_bulk_t<T, false>(x, out, rowsum, rows, c, ld_x, ld_out, alpha, theta, power, st);
    switch (dtype) {
      case SA_F32: SA_FWD_BULK(float); break;
      case SA_F16: SA_FWD_BULK(__half); break;
      default: SA_FWD_BULK(__nv_bfloat16); break;
    }
#undef SA_FWD_BULK
    return sa_record_cuda_error(cudaGetLastError());
  }
  const LaunchShape s = pick_shape(rows, (int)cols, vec, 16);
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
                      ((ld_x * es) % 16) == 0 && ((ld_dx * es) % 16) == 0 && ((ld_g * gs) % 16) == 0;
  const int vec = vec_ok ? V : 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int c = (int)cols;
  if (vec_ok && ((size_t)cols * gs) % 16 == 0) {
#define SA_BWD_BULK_G(T)                                                                                            \
    switch (g_dtype) {                                                                                              \
      case SA_F32: bwd_bulk_t<T, float>(causal, x, g, rowsum, dx, rows, c, ld_x, ld_g, ld_dx, alpha, theta, power, st); break; \
      case SA_F16: bwd_bulk_t<T, __half>(causal, x, g, rowsum, dx, rows, c, ld_x, ld_g, ld_dx, alpha, theta, power, st); break; \
      default: bwd_bulk_t<T, __nv_bfloat16>(causal, x, g, rowsum, dx, rows, c, ld_x, ld_g, ld_dx, alpha, theta, power, st); break; \
    }
    switch (dtype) {
      case SA_F32: SA_BWD_BULK_G(float); break;
      case SA_F16: SA_BWD_BULK_G(__half); break;
      default: SA_BWD_BULK_G(__nv_bfloat16); break;
    }
#undef SA_BWD_BULK_G
    return sa_record_cuda_error(cudaGetLastError());
  }
  const LaunchShape s = pick_shape(rows, (int)cols, vec, 8);
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
SA_BOUNDS_ACCESSOR(norm_bounds)
