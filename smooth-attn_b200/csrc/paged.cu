// Paged-KV decode attention with the squareplus^2 normalizer (one query token
// per sequence), sm_100a.
//
// Reference: _sp2norm_paged_attention_kernel / sp2norm_paged_attention
// (src/smooth_attn/kernels.py:2681-2829).  Per sequence b and query head hq,
// over the context_lens[b] cached tokens j (no causal mask):
//   s_j = (q . k_j) * scale,  a_j = 2 s_j - 1,
//   y_j = squareplus(a_j)^2 = ((a_j + sqrt(a_j^2 + 4)) / 2)^2,
//   out = (sum_j y_j v_j) / (sum_j y_j + 1e-12)          (bf16 output)
// with k_j / v_j read from page block_table[b, j / block_size] of the cache
// [num_blocks, H_kv, block_size, D], row j % block_size.
//
// Design.  Decode is bound by the HBM read of the cache.  The work is the
// flattened sequence of "chunks" of every unit, where a unit is a (sequence,
// KV head, group of GT query heads) triple and a chunk is CR consecutive rows
// of one page of one KV head: a contiguous CR*D*2-byte span of K and the same
// of V.  Every cache byte is read once for all GT query heads of the group
// (the reference launches one program per QUERY head and rereads K/V G
// times).  A persistent grid (one resident wave of CTAs) splits the
// flattened chunks into equal contiguous ranges, so the load is balanced
// whatever the batch / context / head shape, with no tail wave.  Inside a
// CTA range the 4 warps interleave over chunks; each warp streams its chunks
// with two 1-D bulk async copies per chunk into its own shared-memory ring
// (no register staging, several chunks in flight per warp).  Inside a warp,
// L = D/(8*VPL) lanes hold one cache row (VPL 16-byte vectors each) so a
// warp consumes R = 32/L rows per step; the GT partial dot products of a lane are reduced
// across the L lanes by a reduce-scatter (each halving step exchanges half
// of the remaining heads), after which every lane owns the score of one
// (row, head) pair.  P.V uses packed fp32x2 FMAs.  All arithmetic is fp32,
// as in the reference.
//
// Combining.  At the end of each unit segment the warps of a CTA add their
// sums through shared memory.  A CTA whose range covers a whole unit writes
// the output directly.  Otherwise it writes the partial (sum y v, sum y) of
// its segment to a slot of the workspace: because the normalizer is a plain
// sum (no running max), partials combine by addition, in a fixed order (the
// result is deterministic).  The CTAs that touch a unit are a contiguous
// range known by arithmetic; the last of them to arrive (atomic ticket, no
// waiting) adds the partials, divides and writes the output, then resets the
// ticket to zero for the next call.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "paged_tc.h"
#include "sa_common.cuh"
#include "smooth_attn_b200.h"

int sa_record_cuda_error(cudaError_t e);

namespace sa {

static __device__ unsigned g_paged_timeouts;  // bounded-wait failures (never traps)
static __device__ unsigned g_paged_bad_pages; // block_table entries outside [0, num_blocks)

constexpr int kPgWarps = 4;       // warps per CTA
constexpr int kPgMaxStages = 8;   // ring slots per warp (upper bound)
constexpr int kPgRingBytes = 16384;  // per-warp ring target
constexpr int kPgChunkBytes = 4096;  // K bytes per chunk target

struct PagedArgs {
  const void* q;
  const void* kc;
  const void* vc;
  __nv_bfloat16* out;
  const int32_t* bt;
  const int32_t* cl;
  float* part;       // [units][slots][rec] fp32 partials
  int32_t* tickets;  // [units] arrival tickets, zero between calls
  int64_t num_blocks;
  int64_t W;         // total chunks = units * M
  int Hq, Hkv, G, bs, max_blocks;
  int CR;       // rows per chunk (divides bs)
  int cpp;      // chunks per page = bs / CR
  int M;        // chunks per unit = max_blocks * cpp
  int nhc;      // head groups per KV head = G / GT
  int nst;      // ring slots per warp
  int stage;    // bytes per ring slot (K + V, rows padded to R)
  int slots;    // partial slots per unit
  float qscale; // 2 * scale, folded into q
};

// 8 packed 16-bit values -> 4 float pairs (element order preserved).
template <typename T>
__device__ __forceinline__ void unpack8(const uint4 w, float2 (&f)[4]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      f[i].x = __uint_as_float(u[i] << 16);
      f[i].y = __uint_as_float(u[i] & 0xffff0000u);
    } else {
      f[i].x = __half2float(__ushort_as_half((unsigned short)(u[i] & 0xffffu)));
      f[i].y = __half2float(__ushort_as_half((unsigned short)(u[i] >> 16)));
    }
  }
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
}

// Record of one partial: GT*D sums of 4*y*v, then GT sums of 4*y, padded so
// every record starts 16-byte aligned.
__host__ __device__ constexpr int paged_rec_floats(int GT, int D) { return GT * D + 8; }

// Vectors per lane: two (fewer lanes per row, so a cheaper cross-lane
// reduction per score) unless the q / accumulator registers of 8 heads or a
// 32-wide row make one the better choice.
__host__ __device__ constexpr int paged_vpl(int D, int GT) { return (GT <= 4 && D >= 64) ? 2 : 1; }

template <typename T, int D, int GT>
__global__ void __launch_bounds__(kPgWarps * 32) paged_decode_kernel(const PagedArgs a) {
  constexpr int VPL = paged_vpl(D, GT);  // 16-byte vectors of a row per lane
  constexpr int L = D / (8 * VPL);        // lanes per cache row
  constexpr int R = 32 / L;               // rows per warp step
  constexpr int HS = L / GT;              // lanes sharing one head after the reduce-scatter
  constexpr int ROWB = D * (int)sizeof(T);
  constexpr int REC = paged_rec_floats(GT, D);
  constexpr int NT = kPgWarps * 32;
  static_assert(GT >= 1 && GT <= L && (L % GT) == 0, "head group must fit the row lanes");

  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(16) float red[kPgWarps][REC];  // per-warp (sum 4yv, sum 4y) of a segment
  __shared__ int last_cta;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = lane % L, r = lane / L;
  const int64_t NC = gridDim.x;
  const int64_t cta = blockIdx.x;
  const int64_t x0 = cta * a.W / NC, x1 = (cta + 1) * a.W / NC;
  if (x0 >= x1) return;  // whole CTA

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kPgMaxStages;
  uint8_t* ring = smem + kPgWarps * kPgMaxStages * 8 + (size_t)warp * a.nst * a.stage;
  const int CRp = (a.CR + R - 1) / R * R;
  const uint32_t chunk_bytes = (uint32_t)a.CR * ROWB;
  const int upb = a.Hkv * a.nhc;  // units per sequence
  const int ctx_max = a.max_blocks * a.bs;

  auto ctx_of = [&](int u) {
    const int n = __ldg(a.cl + u / upb);
    return max(0, min(n, ctx_max));
  };
  auto issue = [&](int u, int ci, int s) {
    const int b = u / upb;
    const int h = (u - b * upb) / a.nhc;
    const int page = ci / a.cpp;
    const int sub = ci - page * a.cpp;
    int phys = __ldg(a.bt + (int64_t)b * a.max_blocks + page);
    if (phys < 0 || phys >= a.num_blocks) {
      atomicAdd(&g_paged_bad_pages, 1u);
      phys = 0;
    }
    // the chunk lies inside its page and the KV head exists
    if (!SA_DCHECK(h < a.Hkv && sub < a.cpp && (int64_t)(sub + 1) * a.CR <= a.bs)) return;  // wait then gives up
    const int64_t off = (((int64_t)phys * a.Hkv + h) * a.bs + (int64_t)sub * a.CR) * D;
    uint8_t* slot = ring + (size_t)s * a.stage;
    mbar_arrive_expect_tx(&bars[s], 2u * chunk_bytes);
    bulk_g2s(slot, static_cast<const T*>(a.kc) + off, chunk_bytes, &bars[s]);
    bulk_g2s(slot + (size_t)CRp * ROWB, static_cast<const T*>(a.vc) + off, chunk_bytes, &bars[s]);
  };

  // The CTA's range is cut into unit segments; inside a segment warp w takes
  // chunks ci_lo + w, ci_lo + w + 4, ...  Producer cursor (lane 0): chunk pci
  // of unit pu, always a chunk with context tokens, or pmore = false.
  const int u_first = (int)(x0 / a.M);
  const int u_last = (int)((x1 - 1) / a.M);
  auto seg_hi = [&](int u) { return (int)(min(x1, (int64_t)(u + 1) * a.M) - (int64_t)u * a.M); };
  int pu = u_first, pci = (int)(x0 - (int64_t)u_first * a.M) + warp, pn = -1;
  bool pmore = false;
  auto p_seek = [&]() {
    while (pu <= u_last) {
      if (pn < 0) pn = min(seg_hi(pu), (ctx_of(pu) + a.CR - 1) / a.CR);
      if (pci < pn) return true;
      ++pu;
      pci = warp;
      pn = -1;
    }
    return false;
  };
  if (lane == 0) {
    for (int s = 0; s < a.nst; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    pmore = p_seek();
    for (int s = 0; s < a.nst && pmore; ++s) {
      issue(pu, pci, s);
      pci += kPgWarps;
      pmore = p_seek();
    }
  }
  __syncwarp();

  const float eps4 = 4.0f * SA_EPS;
  bool ok = true;
  int k = 0;  // chunks consumed by this warp
  for (int u = u_first; u <= u_last; ++u) {
    const int64_t ubase = (int64_t)u * a.M;
    const int ci_lo = (int)(max(x0, ubase) - ubase), ci_hi = seg_hi(u);
    const int b = u / upb;
    const int hq0 = (u - b * upb) * GT;  // = h * G + hc * GT
    const int ctx = ctx_of(u);
    const int ci_act = min(ci_hi, (ctx + a.CR - 1) / a.CR);

    // q of the GT heads, this lane's 8 columns, pre-scaled by 2*scale.
    // Lane column vectors are c, c + L, ... (16 bytes each), so the lanes of
    // a row read one contiguous span per shared-memory load.
    float2 q2[GT][VPL][4];
#pragma unroll
    for (int g = 0; g < GT; ++g)
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const T* qp = static_cast<const T*>(a.q) + ((int64_t)b * a.Hq + hq0 + g) * D + (j * L + c) * 8;
        unpack8<T>(__ldg(reinterpret_cast<const uint4*>(qp)), q2[g][j]);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          q2[g][j][i] = make_float2(q2[g][j][i].x * a.qscale, q2[g][j][i].y * a.qscale);
      }
    float2 o2[GT][VPL][4];
#pragma unroll
    for (int g = 0; g < GT; ++g)
#pragma unroll
      for (int j = 0; j < VPL; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) o2[g][j][i] = make_float2(0.f, 0.f);
    float ysum = 0.f;  // 4*y of this lane's (row, head) scores

    for (int ci = ci_lo + warp; ci < ci_act && ok; ci += kPgWarps, ++k) {
      const int s = k % a.nst;
      if (!__all_sync(0xffffffffu, mbar_wait(&bars[s], (uint32_t)(k / a.nst) & 1u))) {
        if (lane == 0) atomicAdd(&g_paged_timeouts, 1u);
        ok = false;  // reported by sa_device_status; keep joining the CTA barriers
        break;
      }
      const uint8_t* Ks = ring + (size_t)s * a.stage;
      const uint8_t* Vs = Ks + (size_t)CRp * ROWB;
      const int nvalid = min(a.CR, ctx - ci * a.CR);
      const int steps = (a.CR + R - 1) / R;
      auto step = [&](int st, auto masked) {
        constexpr bool MASK = decltype(masked)::value;
        const bool valid = !MASK || st * R + r < nvalid;
        const uint8_t* kr = Ks + (size_t)(st * R + r) * ROWB + c * 16;
        const uint8_t* vr = Vs + (size_t)(st * R + r) * ROWB + c * 16;
        float2 kf[VPL][4];
#pragma unroll
        for (int j = 0; j < VPL; ++j) unpack8<T>(lds128(kr + j * L * 16), kf[j]);
        float sc[GT];
#pragma unroll
        for (int g = 0; g < GT; ++g) {
          float2 d = make_float2(q2[g][0][0].x * kf[0][0].x, q2[g][0][0].y * kf[0][0].y);
#pragma unroll
          for (int j = 0; j < VPL; ++j)
#pragma unroll
            for (int i = (j == 0 ? 1 : 0); i < 4; ++i) d = ffma2(q2[g][j][i], kf[j][i], d);
          sc[g] = d.x + d.y;
        }
        // Reduce-scatter over the L lanes of the row: at each halving step a
        // lane keeps the lower or upper half of its remaining heads (by the
        // lane bit) and adds its partner's copy of that half.
#pragma unroll
        for (int m = L / 2, n = GT; m >= 1; m >>= 1) {
          if (n > 1) {
            const bool up = (c & m) != 0;
#pragma unroll
            for (int i = 0; i < GT / 2; ++i) {
              if (i < n / 2) {
                const float send = up ? sc[i] : sc[i + n / 2];
                const float keep = up ? sc[i + n / 2] : sc[i];
                sc[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
              }
            }
            n >>= 1;
          } else {
            sc[0] += __shfl_xor_sync(0xffffffffu, sc[0], m);
          }
        }
        // The lane now holds 2 s (scale folded into q) for head c / HS of its row.
        const float av = sc[0] - 1.0f;
        const float uu = fmaf(av, av, 4.0f);
        const float t = fmaf(uu, rsqrt_approx(uu), av);  // 2 * squareplus(a)
        const float y4 = valid ? t * t : 0.f;            // 4 * y
        ysum += y4;
        float2 vf[VPL][4];
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
          uint4 vw = lds128(vr + j * L * 16);
          if (MASK && !valid) vw = make_uint4(0u, 0u, 0u, 0u);  // rows past the context may hold NaN
          unpack8<T>(vw, vf[j]);
        }
#pragma unroll
        for (int g = 0; g < GT; ++g) {
          const float yg = __shfl_sync(0xffffffffu, y4, r * L + g * HS);
          const float2 y2 = make_float2(yg, yg);
#pragma unroll
          for (int j = 0; j < VPL; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) o2[g][j][i] = ffma2(y2, vf[j][i], o2[g][j][i]);
        }
      };
      if (nvalid == steps * R) {  // every row of every step holds a token
#pragma unroll 2
        for (int st = 0; st < steps; ++st) step(st, std::false_type{});
      } else {
        for (int st = 0; st < steps; ++st) step(st, std::true_type{});
      }
      __syncwarp();
      if (lane == 0 && pmore) {  // slot s consumed: refill it
        issue(pu, pci, s);
        pci += kPgWarps;
        pmore = p_seek();
      }
    }

    // Fold the R rows of the warp (lanes with equal c hold the same columns),
    // then the warps of the CTA through shared memory.
#pragma unroll
    for (int m = L; m < 32; m <<= 1) {
      ysum += __shfl_xor_sync(0xffffffffu, ysum, m);
#pragma unroll
      for (int g = 0; g < GT; ++g)
#pragma unroll
        for (int j = 0; j < VPL; ++j)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            o2[g][j][i].x += __shfl_xor_sync(0xffffffffu, o2[g][j][i].x, m);
            o2[g][j][i].y += __shfl_xor_sync(0xffffffffu, o2[g][j][i].y, m);
          }
    }
    __syncthreads();  // red[] of the previous segment fully read
    if (r == 0) {
#pragma unroll
      for (int g = 0; g < GT; ++g)
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
          float* dst = &red[warp][g * D + (j * L + c) * 8];
          *reinterpret_cast<float4*>(dst) = make_float4(o2[g][j][0].x, o2[g][j][0].y, o2[g][j][1].x, o2[g][j][1].y);
          *reinterpret_cast<float4*>(dst + 4) =
              make_float4(o2[g][j][2].x, o2[g][j][2].y, o2[g][j][3].x, o2[g][j][3].y);
        }
      if (c % HS == 0) red[warp][GT * D + c / HS] = ysum;
    }
    __syncthreads();

    if (ci_lo == 0 && ci_hi == a.M) {  // this CTA holds the whole unit
      for (int e = threadIdx.x; e < GT * D; e += NT) {
        const int g = e / D;
        float o = 0.f, sy = 0.f;
#pragma unroll
        for (int w = 0; w < kPgWarps; ++w) {
          o += red[w][e];
          sy += red[w][GT * D + g];
        }
        a.out[((int64_t)b * a.Hq + hq0) * D + e] = __float2bfloat16_rn(o / (sy + eps4));
      }
      continue;
    }

    // CTAs i0..i1 touch unit u; this CTA fills slot cta - i0.
    const int64_t i0 = ((ubase + 1) * NC - 1) / a.W;
    const int64_t i1 = (min(a.W, ubase + a.M) * NC - 1) / a.W;
    float* base = a.part + (int64_t)u * a.slots * REC;
    float* rec = base + (cta - i0) * REC;
    for (int e = threadIdx.x; e < GT * D + GT; e += NT) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kPgWarps; ++w) v += red[w][e];
      __stcg(rec + e, v);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_cta = atomicAdd(a.tickets + u, 1) == (int)(i1 - i0);
    __syncthreads();
    if (!last_cta) continue;
    __threadfence();
    const int nsl = (int)(i1 - i0 + 1);
    float* sy = &red[0][0];  // reuse: GT sums of 4y
    __syncthreads();
    if (threadIdx.x < 32) {  // one warp: lanes stride the slots, then a shuffle sum per head
      float t[GT];
#pragma unroll
      for (int g = 0; g < GT; ++g) t[g] = 0.f;
      for (int sl = threadIdx.x; sl < nsl; sl += 32)
#pragma unroll
        for (int g = 0; g < GT; ++g) t[g] += __ldcg(base + (int64_t)sl * REC + GT * D + g);
#pragma unroll
      for (int g = 0; g < GT; ++g) {
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) t[g] += __shfl_xor_sync(0xffffffffu, t[g], m);
        if (threadIdx.x == 0) sy[GT * D + g] = t[g] + eps4;
      }
    }
    __syncthreads();
    for (int e4 = threadIdx.x; e4 < GT * D / 4; e4 += NT) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      int sl = 0;
      for (; sl + 4 <= nsl; sl += 4) {
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __ldcg(reinterpret_cast<const float4*>(base + (int64_t)(sl + j) * REC) + e4);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc.x += v[j].x;
          acc.y += v[j].y;
          acc.z += v[j].z;
          acc.w += v[j].w;
        }
      }
      for (; sl < nsl; ++sl) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(base + (int64_t)sl * REC) + e4);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const float inv = 1.0f / sy[GT * D + (4 * e4) / D];
      uint2 w;
      w.x = pack_bf16x2(acc.x * inv, acc.y * inv);
      w.y = pack_bf16x2(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(a.out + ((int64_t)b * a.Hq + hq0) * D + 4 * e4) = w;
    }
    if (threadIdx.x == 0) a.tickets[u] = 0;  // ready for the next call
  }
}

int paged_timeouts(int reset, cudaStream_t st) {
  unsigned t = 0;
  cudaMemcpyFromSymbolAsync(&t, g_paged_timeouts, sizeof(t), 0, cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  if (reset) {
    const unsigned z = 0;
    cudaMemcpyToSymbolAsync(g_paged_timeouts, &z, sizeof(z), 0, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
  }
  return (int)t;
}

int paged_bad_pages(int reset, cudaStream_t st) {
  unsigned bad = 0;
  cudaMemcpyFromSymbolAsync(&bad, g_paged_bad_pages, sizeof(bad), 0, cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  if (reset) {
    const unsigned z = 0;
    cudaMemcpyToSymbolAsync(g_paged_bad_pages, &z, sizeof(z), 0, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
  }
  return (int)bad;
}

// ---- host side ---------------------------------------------------------------

namespace {

std::mutex g_sm_mu;
int g_sm_count[64] = {0};

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(g_sm_mu);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

struct Plan {
  int GT, nhc, CR, cpp, M, nst, stage, slots;
  int64_t units, W, grid;
  size_t smem;
  int64_t ticket_bytes, part_bytes;
  bool tc;  // tensor-core kernel (paged_tc.cu) instead of paged_decode_kernel
  PtcPlan ptc;
};

// SA_PAGED_DECODE_KERNEL=simt forces the CUDA-core kernel, =tc the
// tensor-core one where the shape allows it; default: tensor cores for GQA
// groups of bf16 D=128 caches with block_size a multiple of 8 dividing 128.
int kernel_choice() {
  const char* v = getenv("SA_PAGED_DECODE_KERNEL");
  if (v && strcmp(v, "simt") == 0) return 0;
  return 1;
}

// Resident CTAs per SM of one instantiation at one dynamic smem size, and
// the one-time opt-in to that much dynamic shared memory, cached per device
// (the per-call cost of the two runtime queries is several microseconds,
// comparable to a whole short decode).
struct OccEntry {
  const void* fn;
  size_t smem;
  int dev;
  int occ;
};
std::mutex g_occ_mu;
OccEntry g_occ[256];
int g_nocc = 0;

template <typename T, int D, int GT>
int occupancy(size_t smem) {
  auto kfn = paged_decode_kernel<T, D, GT>;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_occ_mu);
  for (int i = 0; i < g_nocc; ++i)
    if (g_occ[i].fn == (const void*)kfn && g_occ[i].smem == smem && g_occ[i].dev == dev) return g_occ[i].occ;
  int n = 0;
  bool cached = true;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kfn, kPgWarps * 32, smem) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = std::max<int>(1, std::min<int>(8, (int)((227 * 1024) / (smem + 1024))));
    cached = false;  // no device here: estimate, retry next time
  }
  if (cached && g_nocc < 256) g_occ[g_nocc++] = {(const void*)kfn, smem, dev, n};
  return n;
}

template <typename T, int D>
int occupancy_d(int GT, size_t smem) {
  switch (GT) {
    case 1: return occupancy<T, D, 1>(smem);
    case 2: return occupancy<T, D, 2>(smem);
    case 4: return occupancy<T, D, 4>(smem);
    default:
      if constexpr (D / 8 >= 8) return occupancy<T, D, 8>(smem);
      return 1;
  }
}

int occupancy_any(int dtype, int64_t D, int GT, size_t smem) {
  if (dtype == SA_BF16) {
    switch (D) {
      case 32: return occupancy_d<__nv_bfloat16, 32>(GT, smem);
      case 64: return occupancy_d<__nv_bfloat16, 64>(GT, smem);
      case 128: return occupancy_d<__nv_bfloat16, 128>(GT, smem);
      default: return occupancy_d<__nv_bfloat16, 256>(GT, smem);
    }
  }
  switch (D) {
    case 32: return occupancy_d<__half, 32>(GT, smem);
    case 64: return occupancy_d<__half, 64>(GT, smem);
    case 128: return occupancy_d<__half, 128>(GT, smem);
    default: return occupancy_d<__half, 256>(GT, smem);
  }
}

// Every size choice of a launch, shared by the workspace query and the launch.
int make_plan(int64_t B, int64_t Hq, int64_t Hkv, int64_t max_blocks, int64_t bs, int64_t D, int dtype, Plan* p) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || max_blocks <= 0 || bs <= 0 || D <= 0) return SA_ERR_ARG;
  if (Hq % Hkv != 0) return SA_ERR_ARG;
  if (dtype != SA_BF16 && dtype != SA_F16) return SA_ERR_UNSUPPORTED;
  if (D != 32 && D != 64 && D != 128 && D != 256) return SA_ERR_UNSUPPORTED;
  if (B > (1 << 24) || Hq > (1 << 20) || bs > (1 << 16) || max_blocks * bs > ((int64_t)1 << 30))
    return SA_ERR_UNSUPPORTED;
  p->tc = kernel_choice() == 1 && paged_tc_plan(B, Hq, Hkv, max_blocks, bs, D, dtype, sm_count(), &p->ptc);
  if (p->tc) {
    p->ticket_bytes = p->ptc.ticket_bytes;
    p->part_bytes = p->ptc.part_bytes;
    return SA_OK;
  }
  const int G = (int)(Hq / Hkv);
  int GT = G & -G;  // largest power of two dividing G
  GT = std::min(GT, std::min(8, (int)D / 8));
  const int L = (int)D / (8 * paged_vpl((int)D, GT)), R = 32 / L;
  p->GT = GT;
  p->nhc = G / GT;
  const int64_t rowb = D * 2;
  int CR = (int)bs;
  if (CR * rowb > kPgChunkBytes) {
    CR = std::max<int>(1, (int)(kPgChunkBytes / rowb));
    while (bs % CR != 0) --CR;
  }
  p->CR = CR;
  p->cpp = (int)(bs / CR);
  if (max_blocks * p->cpp > INT32_MAX) return SA_ERR_UNSUPPORTED;
  p->M = (int)(max_blocks * p->cpp);
  const int CRp = (CR + R - 1) / R * R;
  p->stage = (int)(2 * CRp * rowb);
  p->nst = std::max(2, std::min(kPgMaxStages, kPgRingBytes / p->stage));
  p->smem = kPgWarps * kPgMaxStages * 8 + (size_t)kPgWarps * p->nst * p->stage;
  p->units = B * Hkv * p->nhc;
  if (p->units > INT32_MAX / 2) return SA_ERR_UNSUPPORTED;
  p->W = p->units * p->M;
  if (p->W > ((int64_t)1 << 40)) return SA_ERR_UNSUPPORTED;
  // One resident wave of CTAs, but at least ~4 chunks per warp.
  const int64_t wave = (int64_t)sm_count() * occupancy_any(dtype, D, GT, p->smem);
  p->grid = std::max<int64_t>(1, std::min<int64_t>(wave, (p->W + 4 * kPgWarps - 1) / (4 * kPgWarps)));
  const int64_t share = std::max<int64_t>(1, p->W / p->grid);  // fewest chunks a non-empty CTA holds
  p->slots = (int)std::min<int64_t>(p->grid, (p->M + share - 1) / share + 2);
  p->ticket_bytes = (p->units * 4 + 255) / 256 * 256;
  p->part_bytes = p->units * p->slots * (int64_t)paged_rec_floats(GT, (int)D) * 4;
  return SA_OK;
}

template <typename T, int D, int GT>
int launch_t(const PagedArgs& a, const Plan& p, cudaStream_t st) {
  auto kfn = paged_decode_kernel<T, D, GT>;  // smem opt-in done by make_plan's occupancy()
  kfn<<<(unsigned)p.grid, kPgWarps * 32, p.smem, st>>>(a);
  return sa_record_cuda_error(cudaGetLastError());
}

template <typename T, int D>
int launch_d(const PagedArgs& a, const Plan& p, cudaStream_t st) {
  switch (p.GT) {
    case 1: return launch_t<T, D, 1>(a, p, st);
    case 2: return launch_t<T, D, 2>(a, p, st);
    case 4: return launch_t<T, D, 4>(a, p, st);
    case 8:
      if constexpr (D / 8 >= 8) return launch_t<T, D, 8>(a, p, st);
      return SA_ERR_UNSUPPORTED;
    default: return SA_ERR_UNSUPPORTED;
  }
}

template <typename T>
int launch_dt(int64_t D, const PagedArgs& a, const Plan& p, cudaStream_t st) {
  switch (D) {
    case 32: return launch_d<T, 32>(a, p, st);
    case 64: return launch_d<T, 64>(a, p, st);
    case 128: return launch_d<T, 128>(a, p, st);
    case 256: return launch_d<T, 256>(a, p, st);
    default: return SA_ERR_UNSUPPORTED;
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace sa

extern "C" int64_t sa_paged_decode_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t max_blocks,
                                                  int64_t block_size, int64_t D, int dtype) {
  sa::Plan p;
  const int rc = sa::make_plan(B, Hq, Hkv, max_blocks, block_size, D, dtype, &p);
  if (rc != SA_OK) return rc;
  return p.ticket_bytes + p.part_bytes;
}

extern "C" int sa_paged_decode(const void* q, const void* k_cache, const void* v_cache, void* out,
                               const int32_t* block_table, const int32_t* context_lens, void* workspace,
                               int64_t workspace_bytes, int64_t B, int64_t Hq, int64_t Hkv, int64_t num_blocks,
                               int64_t block_size, int64_t max_blocks, int64_t D, float scale, int dtype,
                               void* stream) {
  sa::Plan p;
  const int rc = sa::make_plan(B, Hq, Hkv, max_blocks, block_size, D, dtype, &p);
  if (rc != SA_OK) return rc;
  if (!q || !k_cache || !v_cache || !out || !block_table || !context_lens || num_blocks <= 0) return SA_ERR_ARG;
  if (!(scale == scale)) return SA_ERR_ARG;
  if (!sa::al16(q) || !sa::al16(k_cache) || !sa::al16(v_cache) || !sa::al16(out)) return SA_ERR_ALIGN;
  if (!workspace || workspace_bytes < p.ticket_bytes + p.part_bytes) return SA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return SA_ERR_ALIGN;
  if (p.tc)
    return sa::paged_tc_launch(q, k_cache, v_cache, out, block_table, context_lens, workspace, B, Hq, Hkv,
                               num_blocks, block_size, max_blocks, scale, p.ptc, static_cast<cudaStream_t>(stream));
  sa::PagedArgs a;
  a.q = q;
  a.kc = k_cache;
  a.vc = v_cache;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.bt = block_table;
  a.cl = context_lens;
  a.tickets = static_cast<int32_t*>(workspace);
  a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + p.ticket_bytes);
  a.num_blocks = num_blocks;
  a.W = p.W;
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.G = (int)(Hq / Hkv);
  a.bs = (int)block_size;
  a.max_blocks = (int)max_blocks;
  a.CR = p.CR;
  a.cpp = p.cpp;
  a.M = p.M;
  a.nhc = p.nhc;
  a.nst = p.nst;
  a.stage = p.stage;
  a.slots = p.slots;
  a.qscale = 2.0f * scale;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == SA_BF16 ? sa::launch_dt<__nv_bfloat16>(D, a, p, st) : sa::launch_dt<__half>(D, a, p, st);
}
SA_BOUNDS_ACCESSOR(paged_bounds)
