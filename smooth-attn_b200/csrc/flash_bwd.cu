// Fused causal squareplus attention, backward, on tcgen05 tensor cores.
//
// Reference algorithm: src/smooth_attn/kernels.py:1680-1909
// (_sp2norm_flash_bwd_dq_kernel, _sp2norm_flash_bwd_dkv_kernel) and the host
// wrapper :1934-1989:
//   delta = rowsum(dO * O);  s = (q . k) * scale;  a = 2 s - 1;
//   sp = (a + sqrt(a^2+4)) / 2;  y = sp^2;  sp' = (1 + a / sqrt(a^2+4)) / 2
//   P = y / R;  dP = dO V^T;  dY = (dP - delta) / R;  dS = dY * 4 sp sp' * scale
//   dQ = dS K;  dK = dS^T Q;  dV = P^T dO   (bf16 operands, fp32 accumulate)
//
// B200 design (three launches):
//   1. sp2_bwd_prep: delta = rowsum(dO * O) per query row (fp32) and zero
//      the fp32 dQ accumulator (memory-bound, 16-byte vector loads);
//   2. sp2_bwd_kernel: one CTA per 128-row KV tile of one (batch, kv head),
//      looping over the query heads of its GQA group and the 128-row query
//      tiles that can see it.  K and V stay resident in shared memory; Q / dO
//      tiles stream through a 2-stage TMA ring.  Per query tile:
//        MMA   S^T = K Q^T,  dP^T = V dO^T         (TMEM, 128 cols each)
//        warps 2..5 (thread = KV row): P -> TMEM (over S^T, bf16),
//              dS -> shared memory (bf16, 128 B swizzle)
//        MMA   dV += P^T dO (P from TMEM), dK += dS^T Q, dQ = dS K (into the
//              dP^T columns)
//        warps 2..5 (thread = query row): dQ rows -> fp32 vector atomics
//      dK / dV accumulate in TMEM over the whole loop (GQA heads summed
//      in-CTA like the reference) and are written once at the end.
//   3. sp2_bwd_dq_convert: dQ accumulator -> dq (bf16/fp16, caller strides).
// The dS tile in shared memory is laid out once (rows = KV, 64-wide query
// chunks, 128 B swizzle) and read by two MMAs with two descriptors: as a
// K-major A for dK and as an MN-major A for dQ.
// D = 128 uses sp2_bwd128_kernel instead (64-row query tiles, double-buffered
// S^T / dP^T, dQ^T drained by four warps).  The deterministic path
// (deterministic != 0) runs the key-major kernel without dQ
// (sp2_bwd_dkv128_kernel for D = 128) and then the query-major
// sp2_bwd_dq_kernel, which sums every dQ row in one CTA in a fixed order.
#include <cudaTypedefs.h>

#include <type_traits>

#include "sa_sm100.cuh"

static inline int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

namespace sa {
namespace sqattn {

using namespace sm100;

static __device__ unsigned g_flash_bwd_timeouts;

bool make_map_4d(CUtensorMap* map, const void* base, bool bf16, int64_t B, int64_t H, int64_t T, int64_t D,
                 const int64_t* strides, int chunk, int rows, bool u8 = false);

namespace {

__device__ __forceinline__ bool b_wait(uint64_t* bar, uint32_t phase, bool& failed) {
  if (failed) return false;
  if (!mbar_wait_spin(bar, phase)) {
    failed = true;
    atomicAdd(&g_flash_bwd_timeouts, 1u);
    return false;
  }
  return true;
}

__device__ __forceinline__ bool b_warp_wait_spin(uint64_t* bar, uint32_t phase, bool& failed) {
  const bool ok = __all_sync(0xffffffffu, !failed && mbar_wait_spin(bar, phase));
  if (!ok) {
    if (!failed && (threadIdx.x & 31) == 0) atomicAdd(&g_flash_bwd_timeouts, 1u);
    failed = true;
  }
  return ok;
}

__device__ __forceinline__ bool b_warp_wait(uint64_t* bar, uint32_t phase, bool& failed) {
  const bool ok = __all_sync(0xffffffffu, !failed && mbar_wait(bar, phase));
  if (!ok) {
    if (!failed && (threadIdx.x & 31) == 0) atomicAdd(&g_flash_bwd_timeouts, 1u);
    failed = true;
  }
  return ok;
}

// Named barrier over the 128 threads of warps 2..5.
__device__ __forceinline__ void compute_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

}  // namespace

// One 32-column chunk (query columns [32c, 32c+32)) of the backward
// elementwise stage for the KV row held by this thread: P -> TMEM (over S^T),
// dS -> the swizzled shared-memory tile.
template <bool BF16, bool EXACT, bool MASK>
__device__ __forceinline__ void bwd_chunk(uint32_t tl, int c, uint8_t* sDS, int r, const float* sInvR,
                                          const float* sDelta, float scale2, float c4s, int n, int q0, int qend,
                                          int Tk, int window) {
  uint32_t sv[32], dv[32];
  tmem_ld32(tl + c * 32, sv);
  tmem_ld32(tl + 128 + c * 32, dv);
  tmem_ld_wait();
  uint32_t pk[16], dk[16];
  const float2 half = make_float2(0.5f, 0.5f), c4s2 = make_float2(c4s, c4s);
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    // two query columns per packed fp32x2 instruction (bit-identical to scalar)
    const int m = c * 32 + e;
    const float2 a = ffma2(make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])),
                           make_float2(scale2, scale2), make_float2(-1.0f, -1.0f));
    const float2 w = ffma2(a, a, make_float2(4.0f, 4.0f));
    const float2 rs = make_float2(rsqrt_approx(w.x), rsqrt_approx(w.y));
    const float2 sq = EXACT ? make_float2(sqrtf(w.x), sqrtf(w.y)) : fmul2(w, rs);
    const float2 sp = fmul2(half, fadd2(a, sq));
    const float2 spp = fmul2(half, ffma2(a, rs, make_float2(1.0f, 1.0f)));
    const float2 invR = *reinterpret_cast<const float2*>(sInvR + m);
    const float2 dl = *reinterpret_cast<const float2*>(sDelta + m);
    float2 pp = fmul2(fmul2(sp, sp), invR);
    float2 ds = fmul2(fmul2(fsub2(make_float2(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])), dl), invR),
                      fmul2(fmul2(c4s2, sp), spp));
    if (MASK) {
      const int q = q0 + m;  // global query position (q0 global); qend = one past the last query
      const bool ok0 = (n <= q) && (q < qend) && (n < Tk) && (window <= 0 || q - n < window);
      const bool ok1 = (n <= q + 1) && (q + 1 < qend) && (n < Tk) && (window <= 0 || q + 1 - n < window);
      pp.x = ok0 ? pp.x : 0.f;
      ds.x = ok0 ? ds.x : 0.f;
      pp.y = ok1 ? pp.y : 0.f;
      ds.y = ok1 ? ds.y : 0.f;
    }
    pk[e / 2] = BF16 ? pack2_bf16(pp.x, pp.y) : pack2_f16(pp.x, pp.y);
    dk[e / 2] = BF16 ? pack2_bf16(ds.x, ds.y) : pack2_f16(ds.x, ds.y);
  }
  tmem_st16(tl + c * 16, pk);
  uint8_t* row = sDS + (c >> 1) * (128 * 128) + r * 128;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int piece = ((c & 1) * 4 + j) ^ (r & 7);
    *reinterpret_cast<uint4*>(row + piece * 16) = make_uint4(dk[4 * j], dk[4 * j + 1], dk[4 * j + 2], dk[4 * j + 3]);
  }
}

template <int D>
struct BwdCfg {
  static constexpr int BN = 128, BQ = 128;
  static constexpr int CHUNK = D >= 64 ? 64 : D;
  static constexpr int NCHUNK = D / CHUNK;
  static constexpr int ROWB = CHUNK * 2;
  static constexpr uint32_t SWZ = ROWB == 128 ? SW_128B : SW_64B;
  static constexpr int SBO = 8 * ROWB;
  static constexpr int TILE = 128 * D * 2;  // K, V, Q or dO tile bytes
  static constexpr int DS_BYTES = BQ * BN * 2;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE;
  static constexpr int OFF_Q = OFF_V + TILE;  // 2 stages
  static constexpr int OFF_DO = OFF_Q + 2 * TILE;  // 2 stages
  static constexpr int OFF_DS = OFF_DO + 2 * TILE;
  static constexpr int OFF_VEC = OFF_DS + DS_BYTES;  // invR[128], delta[128]
  static constexpr int OFF_BAR = OFF_VEC + 2 * 128 * 4;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr int TMEM_COLS = 512;  // S^T @0, dP^T / dQ @128, dK @256, dV @256+D
};

struct BwdParams {
  void* dk;
  void* dv;
  const float* rowsum;  // R  [B, Hq, T]
  const float* delta;   // [B, Hq, T]
  float* dq_acc;        // [B, Hq, T, D] fp32
  const float* rvec;    // per 128-row query tile: [2][128] = 1/R, -delta scale/R (D = 128 kernel)
  int64_t sdk_b, sdk_h, sdk_s;
  int64_t sdv_b, sdv_h, sdv_s;
  int B, Hq, Hkv, T, window;  // T: query rows
  int Tk, qoff;                 // key rows; global position of query row 0 (keys start at 0)
  float scale;
};

// Query tiles [qt_first, qt_last] (local, BQ rows each) that see some key of
// the KV tile [n0, n0 + BN): query rows at global positions >= n0 and, with a
// window, < n0 + BN - 1 + window.  Empty when qt_last < qt_first.
__device__ __forceinline__ void query_tile_range(const BwdParams& p, int n0, int BN, int BQ, int& qt_first,
                                                 int& qt_last) {
  const int first_local = n0 - p.qoff;
  qt_first = first_local > 0 ? first_local / BQ : 0;
  qt_last = (p.T + BQ - 1) / BQ - 1;
  if (p.window > 0) {
    const int last_local = n0 + BN - 1 + p.window - 1 - p.qoff;
    const int l = last_local >= 0 ? last_local / BQ : -1;
    if (l < qt_last) qt_last = l;
  }
}

template <int D, int BN>
__device__ void zero_dkdv(const BwdParams& p, int b, int kvh, int n0) {
  for (int i = threadIdx.x; i < 2 * BN * (D / 8); i += blockDim.x) {
    const int which = i / (BN * (D / 8));
    const int rem = i - which * BN * (D / 8);
    const int n = n0 + rem / (D / 8), c = rem % (D / 8);
    if (n >= p.Tk) continue;
    uint8_t* base = static_cast<uint8_t*>(which ? p.dv : p.dk) +
                    2 * (which ? ((int64_t)b * p.sdv_b + (int64_t)kvh * p.sdv_h + (int64_t)n * p.sdv_s)
                               : ((int64_t)b * p.sdk_b + (int64_t)kvh * p.sdk_h + (int64_t)n * p.sdk_s));
    reinterpret_cast<uint4*>(base)[c] = make_uint4(0u, 0u, 0u, 0u);
  }
}

struct BwdBars {
  uint64_t kv_full;
  uint64_t qdo_full[2];
  uint64_t qdo_empty[2];
  uint64_t s_full;
  uint64_t ds_ready;
  uint64_t mm2_done;
  uint64_t dq_free;
  uint64_t all_done;
  uint32_t tmem_base;
};

template <int D, bool BF16, bool EXACT, bool WITH_DQ = true>
__global__ void __launch_bounds__(192, 1)
    sp2_bwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                     const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmdo,
                     BwdParams p) {
  using C = BwdCfg<D>;
  // Declared 1024-byte aligned (the swizzled tiles need it; the kernel has no
  // static shared data, so dynamic shared memory starts on such a boundary):
  // the compiler then folds the tile addresses (measured 4 % on the D = 128
  // backward).  A misaligned start is counted as a timeout and every thread leaves.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicAdd(&g_flash_bwd_timeouts, 1u);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sDO = smem + C::OFF_DO;
  uint8_t* sDS = smem + C::OFF_DS;
  float* sInvR = reinterpret_cast<float*>(smem + C::OFF_VEC);
  float* sDelta = sInvR + 128;
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + C::OFF_BAR);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int kvt, bhk;  // KV tile (0 = most query tiles) and (batch, kv head)
  // one head at a time (group of 1): measured faster here than the grouped
  // order the forward uses, which lengthened this kernel's step
  grouped_longest_first((int)blockIdx.x, (p.Tk + C::BN - 1) / C::BN, p.B * p.Hkv, 1, kvt, bhk);
  const int n0 = kvt * C::BN;
  const int b = bhk / p.Hkv, kvh = bhk % p.Hkv;
  const int G = p.Hq / p.Hkv;
  int qt_first, qt_last;
  query_tile_range(p, n0, C::BN, C::BQ, qt_first, qt_last);
  const int per_head = qt_last - qt_first + 1;
  const int ntiles = per_head > 0 ? G * per_head : 0;
  if (ntiles == 0) {  // no query sees these keys: dK = dV = 0 (before any barrier)
    zero_dkdv<D, C::BN>(p, b, kvh, n0);
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->qdo_full[i], 1);
      mbar_init(&bars->qdo_empty[i], 1);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->ds_ready, 128);
    mbar_init(&bars->mm2_done, 1);
    mbar_init(&bars->dq_free, 128);
    mbar_init(&bars->all_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  bool failed = false;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      tma_prefetch_desc(&tmdo);
      mbar_arrive_expect_tx(&bars->kv_full, 2 * C::TILE);
      for (int c = 0; c < C::NCHUNK; ++c) {
        tma_load_4d(sK + c * 128 * C::ROWB, &tmk, c * C::CHUNK, n0, kvh, b, &bars->kv_full);
        tma_load_4d(sV + c * 128 * C::ROWB, &tmv, c * C::CHUNK, n0, kvh, b, &bars->kv_full);
      }
      for (int it = 0; it < ntiles; ++it) {
        const int st = it & 1;
        if (it >= 2 && !b_wait(&bars->qdo_empty[st], ((it >> 1) - 1) & 1, failed)) break;
        const int h = kvh * G + it / per_head;
        const int q0 = (qt_first + it % per_head) * C::BQ;
        mbar_arrive_expect_tx(&bars->qdo_full[st], 2 * C::TILE);
        for (int c = 0; c < C::NCHUNK; ++c) {
          tma_load_4d(sQ + st * C::TILE + c * 128 * C::ROWB, &tmq, c * C::CHUNK, q0, h, b, &bars->qdo_full[st]);
          tma_load_4d(sDO + st * C::TILE + c * 128 * C::ROWB, &tmdo, c * C::CHUNK, q0, h, b, &bars->qdo_full[st]);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr int ab = BF16 ? 1 : 0;
      constexpr uint32_t id_s = idesc_f16(128, C::BQ, ab, 0, 0);   // S^T, dP^T: A K-major, B K-major
      constexpr uint32_t id_kv = idesc_f16(128, D, ab, 0, 1);      // dV, dK: B (dO / Q) MN-major
      constexpr uint32_t id_dq = idesc_f16(128, D, ab, 1, 1);      // dQ: A (dS) MN-major, B (K) MN-major
      const uint32_t tS = tbase, tP = tbase + 128, tDK = tbase + 256, tDV = tbase + 256 + D;
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aQ = smem_u32(sQ), aDO = smem_u32(sDO);
      const uint32_t aDS = smem_u32(sDS);
      if (b_wait(&bars->kv_full, 0, failed)) {
        for (int it = 0; it < ntiles; ++it) {
          const int st = it & 1;
          if (!b_wait(&bars->qdo_full[st], (it >> 1) & 1, failed)) break;
          if (WITH_DQ && it > 0 && !b_wait(&bars->dq_free, (it - 1) & 1, failed)) break;
          tc_fence_after();
          const uint32_t q_s = aQ + st * C::TILE, do_s = aDO + st * C::TILE;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int c = (kk * 16) / C::CHUNK;
            const uint32_t off = c * 128 * C::ROWB + ((kk * 16) % C::CHUNK) * 2;
            mma_ss(tS, smem_desc(aK + off, 16, C::SBO, C::SWZ), smem_desc(q_s + off, 16, C::SBO, C::SWZ), id_s, kk > 0);
            mma_ss(tP, smem_desc(aV + off, 16, C::SBO, C::SWZ), smem_desc(do_s + off, 16, C::SBO, C::SWZ), id_s, kk > 0);
          }
          mma_commit(&bars->s_full);
          if (!b_wait(&bars->ds_ready, it & 1, failed)) break;
          tc_fence_after();
          // dV += P^T dO ; dK += dS^T Q   (K = 128 query rows, 8 steps of 16)
#pragma unroll
          for (int kk = 0; kk < C::BQ / 16; ++kk) {
            const uint64_t b_do = smem_desc(do_s + kk * 16 * C::ROWB, 128 * C::ROWB, C::SBO, C::SWZ);
            const uint64_t b_q = smem_desc(q_s + kk * 16 * C::ROWB, 128 * C::ROWB, C::SBO, C::SWZ);
            const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
            mma_ts(tDV, tS + kk * 8, b_do, id_kv, acc);
            // dS^T as K-major A: rows = KV, 64-wide query chunks of 128 B
            const uint64_t a_ds = smem_desc(aDS + (kk / 4) * (128 * 128) + (kk % 4) * 32, 16, 1024, SW_128B);
            mma_ss(tDK, a_ds, b_q, id_kv, acc);
          }
          // dQ = dS K   (M = query rows, K = 128 KV rows)
#pragma unroll
          for (int kk = 0; kk < (WITH_DQ ? C::BN / 16 : 0); ++kk) {
            const uint64_t a_ds = smem_desc(aDS + kk * 16 * 128, 128 * 128, 1024, SW_128B);
            const uint64_t b_k = smem_desc(aK + kk * 16 * C::ROWB, 128 * C::ROWB, C::SBO, C::SWZ);
            mma_ss(tP, a_ds, b_k, id_dq, kk > 0);
          }
          mma_commit(&bars->mm2_done);
          mma_commit(&bars->qdo_empty[st]);
        }
      }
      mma_commit(&bars->all_done);
    }
  } else {
    // ------------------------------------------------------------ compute warps
    const int g = warp & 3;
    const int r = 32 * g + lane;  // TMEM lane: KV row for S/dP/dK/dV, query row for dQ
    const int tid = threadIdx.x - 64;
    const uint32_t tl = tbase + ((uint32_t)(32 * g) << 16);
    const int n = n0 + r;
    const float scale2 = 2.0f * p.scale, c4s = 4.0f * p.scale;
    // R^-1 and delta of the next query tile are prefetched into registers one
    // tile ahead, so their global-load latency hides behind the current tile.
    float pre_invR = 0.f, pre_delta = 0.f;
    auto prefetch = [&](int it) {
      const int h = kvh * G + it / per_head;
      const int qq = (qt_first + it % per_head) * C::BQ + tid;
      const int64_t idx = ((int64_t)b * p.Hq + h) * p.T + qq;
      const bool ok = it < ntiles && qq < p.T;
      pre_invR = ok ? __ldg(p.rowsum + idx) : 0.f;  // inverted when stored (no stall here)
      pre_delta = ok ? __ldg(p.delta + idx) : 0.f;
    };
    prefetch(0);
    for (int it = 0; it < ntiles && !failed; ++it) {
      const int h = kvh * G + it / per_head;
      const int q0 = (qt_first + it % per_head) * C::BQ;
      const int64_t rbase = ((int64_t)b * p.Hq + h) * p.T;
      compute_sync();  // everyone done with the previous tile's invR / delta
      sInvR[tid] = pre_invR > 0.f ? 1.0f / pre_invR : 0.f;
      sDelta[tid] = pre_delta;
      compute_sync();
      prefetch(it + 1);
      if (!b_warp_wait(&bars->s_full, it & 1, failed)) break;
      tc_fence_after();
      const int q0g = q0 + p.qoff, qend = p.qoff + p.T;  // global query positions
      const bool need_mask = (q0g < n0 + C::BN - 1) || (q0 + C::BQ > p.T) || (n0 + C::BN > p.Tk) ||
                             (p.window > 0 && q0g + C::BQ - 1 - n0 >= p.window);
      if (need_mask) {
#pragma unroll 1
        for (int c = 0; c < C::BQ / 32; ++c)
          bwd_chunk<BF16, EXACT, true>(tl, c, sDS, r, sInvR, sDelta, scale2, c4s, n, q0g, qend, p.Tk, p.window);
      } else {
#pragma unroll 1
        for (int c = 0; c < C::BQ / 32; ++c)
          bwd_chunk<BF16, EXACT, false>(tl, c, sDS, r, sInvR, sDelta, scale2, c4s, n, q0g, qend, p.Tk, p.window);
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->ds_ready);
      if (!WITH_DQ) continue;  // dQ comes from the query-major kernel
      // drain dQ (TMEM lane = query row) with fp32 vector atomics
      if (!b_warp_wait(&bars->mm2_done, it & 1, failed)) break;
      tc_fence_after();
      const int q = q0 + r;
      float4* dst = reinterpret_cast<float4*>(p.dq_acc + (rbase + q) * D);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tl + 128 + c * 32, v);
        tmem_ld_wait();
        if (q < p.T) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            atomicAdd(dst + c * 8 + j, make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                                   __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3])));
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->dq_free);
    }
    // epilogue: dK, dV rows (TMEM lane = KV row)
    if (b_warp_wait(&bars->all_done, 0, failed)) {
      tc_fence_after();
      const bool live = n < p.Tk;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        uint8_t* base = static_cast<uint8_t*>(which ? p.dv : p.dk) +
                        2 * (which ? ((int64_t)b * p.sdv_b + (int64_t)kvh * p.sdv_h + (int64_t)n * p.sdv_s)
                                   : ((int64_t)b * p.sdk_b + (int64_t)kvh * p.sdk_h + (int64_t)n * p.sdk_s));
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tl + 256 + which * D + c * 32, v);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            pk[e / 2] = BF16 ? pack2_bf16(__uint_as_float(v[e]), __uint_as_float(v[e + 1]))
                             : pack2_f16(__uint_as_float(v[e]), __uint_as_float(v[e + 1]));
          if (live) {
            uint4* dst = reinterpret_cast<uint4*>(base + c * 64);
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// D = 128 backward: 64-row query tiles, double-buffered S^T / dP^T in TMEM.
//
// TMEM (512 columns): S^T_b @ 64b and dP^T_b @ 128 + 64b (both double-
// buffered), dK @ 256, dV @ 384.  dQ is produced transposed, dQ^T = K^T dS^T
// (M = the 128 head-dim rows, N = 64 query columns), into the dP^T buffer of
// its own tile after the elementwise stage consumed it, so everything fits.
// S^T and dP^T of tile i+2 are issued while tile i+1's elementwise stage runs.
// Warps: 0-7 elementwise (two warpgroups, 32 query columns each), 8-11 dQ
// drain (TMEM lane = head-dim index: coalesced fp32 atomics), 12 TMA, 13 MMA.
// ---------------------------------------------------------------------------
struct Bwd128 {
  static constexpr int D = 128, BN = 128, BQ = 64, NS = 3;
  static constexpr int KV_TILE = 128 * D * 2;  // 2 chunks of 128 rows x 128 B
  static constexpr int Q_TILE = BQ * D * 2;    // 2 chunks of 64 rows x 128 B
  static constexpr int DS_TILE = BN * BQ * 2;  // [128 kv][64 q], 128 B swizzle
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + KV_TILE;
  static constexpr int OFF_Q = OFF_V + KV_TILE;
  static constexpr int OFF_DO = OFF_Q + NS * Q_TILE;
  static constexpr int OFF_DS = OFF_DO + NS * Q_TILE;
  static constexpr int OFF_VEC = OFF_DS + 2 * DS_TILE;  // [2 buffers][3][64] per-column constants
  static constexpr int OFF_BAR = OFF_VEC + 2 * 3 * 64 * 4;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr int THREADS = 448;
};

struct Bwd128Bars {
  uint64_t kv_full;
  uint64_t q_full[3], q_empty[3];
  uint64_t s_full[2];   // S^T of tile j ready in buffer j&1
  uint64_t dp_full[2];  // dP^T of tile j ready in buffer j&1
  uint64_t p_ready;    // elementwise stage of tile j done (256 arrivals)
  // dK(j), dQ^T(j) complete, in barrier j&1.  The drain releases dq_free
  // before its atomics, so the MMA can finish tile j+2 before the drain waits
  // for tile j+1; one barrier per tile parity keeps each barrier at most one
  // phase ahead of its waiter (a single barrier could complete twice).
  uint64_t mm2_done[2];
  uint64_t dq_free;    // dQ^T(j) read out of TMEM (128 arrivals): dP^T buffer j&1 free
  uint64_t all_done;
  uint32_t tmem_base;
};

__device__ __forceinline__ void ew_sync() { asm volatile("bar.sync 2, 256;" ::: "memory"); }

// AND of `v` over the 256 elementwise threads (also a barrier among them).
__device__ __forceinline__ bool ew_all(bool v) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 2, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)v)
      : "memory");
  return out != 0;
}

// Per query column m the loader stores c4[m] = 1/(4R), cs[m] = scale/R and
// -cd[m] = -delta*scale/R, so with t = a + sqrt(a^2+4) = 2 sp and
// h = 1 + a rsqrt(a^2+4) = 2 sp':
//   P  = sp^2 / R                      = t*t*c4
//   dS = (dP - delta)/R * 4 sp sp' s   = (dP*cs - cd) * t*h = (dP*cs - cd) * t*t*rsqrt(a^2+4)
// Both 32-column TMEM loads are issued together (one latency); results are
// packed and stored 16 columns at a time to keep register use low.
template <bool BF16, bool EXACT, bool MASK>
__device__ __forceinline__ void bwd128_chunk(uint32_t tS, uint32_t tP, int w2, uint8_t* dsrow, int r,
                                             const float* vec, float scale2, int n, int q0, int qend, int Tk,
                                             int window) {
  uint32_t sv[32], dv[32];
  tmem_ld32(tS + 32 * w2, sv);
  tmem_ld32(tP + 32 * w2, dv);
  tmem_ld_wait(sv);
  tmem_ld_wait(dv);
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int col = 32 * w2 + 16 * hf;
    uint32_t pk[8], dk[8];
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      const float4 c4v = *reinterpret_cast<const float4*>(vec + col + e);
      const float4 csv = *reinterpret_cast<const float4*>(vec + 64 + col + e);
      const float4 cdv = *reinterpret_cast<const float4*>(vec + 128 + col + e);  // -cd
      const float2 c4p[2] = {make_float2(c4v.x, c4v.y), make_float2(c4v.z, c4v.w)};
      const float2 csp[2] = {make_float2(csv.x, csv.y), make_float2(csv.z, csv.w)};
      const float2 cdp[2] = {make_float2(cdv.x, cdv.y), make_float2(cdv.z, cdv.w)};
      float pv[4], dsv[4];
      // two query columns per packed fp32x2 instruction (bit-identical to the
      // scalar ops; the elementwise stage bounds this kernel's issue slots)
#pragma unroll
      for (int u = 0; u < 4; u += 2) {
        const int idx = 16 * hf + e + u;
        const float2 a = ffma2(make_float2(__uint_as_float(sv[idx]), __uint_as_float(sv[idx + 1])),
                               make_float2(scale2, scale2), make_float2(-1.0f, -1.0f));
        const float2 w = ffma2(a, a, make_float2(4.0f, 4.0f));
        const float2 rs = make_float2(rsqrt_approx(w.x), rsqrt_approx(w.y));
        const float2 t = EXACT ? make_float2(a.x + sqrtf(w.x), a.y + sqrtf(w.y)) : ffma2(w, rs, a);
        // 4 sp sp' = t (1 + a rsqrt(w)) = t^2 rsqrt(w): one multiply fewer, and
        // no cancellation in 1 + a rsqrt(w) for very negative a
        const float2 tt = fmul2(t, t);
        float2 pp = fmul2(tt, c4p[u / 2]);
        float2 ds = fmul2(ffma2(make_float2(__uint_as_float(dv[idx]), __uint_as_float(dv[idx + 1])), csp[u / 2],
                                cdp[u / 2]),
                          fmul2(tt, rs));
        if (MASK) {
          const int q = q0 + col + e + u;  // global query position
          const bool ok0 = (n <= q) && (q < qend) && (n < Tk) && (window <= 0 || q - n < window);
          const bool ok1 = (n <= q + 1) && (q + 1 < qend) && (n < Tk) && (window <= 0 || q + 1 - n < window);
          pp.x = ok0 ? pp.x : 0.f;
          ds.x = ok0 ? ds.x : 0.f;
          pp.y = ok1 ? pp.y : 0.f;
          ds.y = ok1 ? ds.y : 0.f;
        }
        pv[u] = pp.x;
        pv[u + 1] = pp.y;
        dsv[u] = ds.x;
        dsv[u + 1] = ds.y;
      }
      pk[e / 2] = BF16 ? pack2_bf16(pv[0], pv[1]) : pack2_f16(pv[0], pv[1]);
      pk[e / 2 + 1] = BF16 ? pack2_bf16(pv[2], pv[3]) : pack2_f16(pv[2], pv[3]);
      dk[e / 2] = BF16 ? pack2_bf16(dsv[0], dsv[1]) : pack2_f16(dsv[0], dsv[1]);
      dk[e / 2 + 1] = BF16 ? pack2_bf16(dsv[2], dsv[3]) : pack2_f16(dsv[2], dsv[3]);
    }
    // P of query columns [32 w2, 32 w2 + 32) goes over this warpgroup's own,
    // already-read S^T columns [32 w2, 32 w2 + 16): no cross-warpgroup hazard.
    tmem_st8(tS + 32 * w2 + 8 * hf, pk);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int piece = (w2 * 4 + hf * 2 + j) ^ (r & 7);
      *reinterpret_cast<uint4*>(dsrow + piece * 16) = make_uint4(dk[4 * j], dk[4 * j + 1], dk[4 * j + 2], dk[4 * j + 3]);
    }
  }
}

template <bool BF16, bool EXACT>
__global__ void __launch_bounds__(448, 1)
    sp2_bwd128_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmdo,
                        BwdParams p) {
  using C = Bwd128;
  constexpr int D = C::D;
  // Declared 1024-byte aligned (the swizzled tiles need it; the kernel has no
  // static shared data, so dynamic shared memory starts on such a boundary):
  // the compiler then folds the tile addresses (measured 4 % on the D = 128
  // backward).  A misaligned start is counted as a timeout and every thread leaves.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicAdd(&g_flash_bwd_timeouts, 1u);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sDO = smem + C::OFF_DO;
  uint8_t* sDS = smem + C::OFF_DS;
  float* vVec = reinterpret_cast<float*>(smem + C::OFF_VEC);  // [2][3][64]
  Bwd128Bars* bars = reinterpret_cast<Bwd128Bars*>(smem + C::OFF_BAR);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int kvt, bhk;  // KV tile (0 = most query tiles) and (batch, kv head)
  // one head at a time (group of 1): measured faster here than the grouped
  // order the forward uses, which lengthened this kernel's step
  grouped_longest_first((int)blockIdx.x, (p.Tk + C::BN - 1) / C::BN, p.B * p.Hkv, 1, kvt, bhk);
  const int n0 = kvt * C::BN;
  const int b = bhk / p.Hkv, kvh = bhk % p.Hkv;
  const int G = p.Hq / p.Hkv;
  int qt_first, qt_last;
  query_tile_range(p, n0, C::BN, C::BQ, qt_first, qt_last);
  const int per_head = qt_last - qt_first + 1;
  const int ntiles = per_head > 0 ? G * per_head : 0;
  if (ntiles == 0) {  // no query sees these keys: dK = dV = 0 (before any barrier)
    zero_dkdv<D, C::BN>(p, b, kvh, n0);
    return;
  }
  // Tiles run head-major: (head kvh*G + g, query tile qt_first .. qt_last).
  // Each role walks them with an incremental cursor (no integer division).
  struct Cursor {
    int h, qt;
  };
  auto advance = [&](Cursor& c) {
    if (++c.qt > qt_last) {
      c.qt = qt_first;
      ++c.h;
    }
  };

  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&bars->q_full[i], 1);
      mbar_init(&bars->q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&bars->s_full[i], 1);
    for (int i = 0; i < 2; ++i) mbar_init(&bars->dp_full[i], 1);
    mbar_init(&bars->p_ready, 256);
    for (int i = 0; i < 2; ++i) mbar_init(&bars->mm2_done[i], 1);
    mbar_init(&bars->dq_free, 128);
    mbar_init(&bars->all_done, 1);
    fence_mbar_init();
  }
  if (warp == 13) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  bool failed = false;

  if (warp == 12) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      tma_prefetch_desc(&tmdo);
      mbar_arrive_expect_tx(&bars->kv_full, 2 * C::KV_TILE);
      for (int c = 0; c < 2; ++c) {
        tma_load_4d(sK + c * 128 * 128, &tmk, c * 64, n0, kvh, b, &bars->kv_full);
        tma_load_4d(sV + c * 128 * 128, &tmv, c * 64, n0, kvh, b, &bars->kv_full);
      }
      Cursor cur{kvh * G, qt_first};
      for (int it = 0; it < ntiles && !failed; ++it, advance(cur)) {
        const int st = it % C::NS;
        if (it >= C::NS && !b_wait(&bars->q_empty[st], ((it / C::NS) - 1) & 1, failed)) break;
        const int h = cur.h;
        const int q0 = cur.qt * C::BQ;
        mbar_arrive_expect_tx(&bars->q_full[st], 2 * C::Q_TILE);
        for (int c = 0; c < 2; ++c) {
          tma_load_4d(sQ + st * C::Q_TILE + c * C::BQ * 128, &tmq, c * 64, q0, h, b, &bars->q_full[st]);
          tma_load_4d(sDO + st * C::Q_TILE + c * C::BQ * 128, &tmdo, c * 64, q0, h, b, &bars->q_full[st]);
        }
      }
    }
  } else if (warp == 13) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr int ab = BF16 ? 1 : 0;
      constexpr uint32_t id_s = idesc_f16(128, C::BQ, ab, 0, 0);  // S^T, dP^T
      constexpr uint32_t id_kv = idesc_f16(128, D, ab, 0, 1);     // dV, dK: B (dO / Q) MN-major
      constexpr uint32_t id_dq = idesc_f16(128, C::BQ, ab, 1, 1); // dQ^T: A = K^T MN-major, B = dS^T MN-major
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aQ = smem_u32(sQ), aDO = smem_u32(sDO);
      const uint32_t aDS = smem_u32(sDS);
      const uint32_t tDK = tbase + 256, tDV = tbase + 384;
      // descriptors are built once and advanced with plain adds in the MMA loops
      const uint64_t dK0 = smem_desc(aK, 16, 1024, SW_128B), dV0 = smem_desc(aV, 16, 1024, SW_128B);
      const uint64_t dKt0 = smem_desc(aK, 128 * 128, 1024, SW_128B);  // K as MN-major A (K^T)
      auto issue_s = [&](int it) {  // S^T(it) = K Q^T -> buffer it&1
        const uint64_t dq0 = smem_desc(aQ + (it % C::NS) * C::Q_TILE, 16, 1024, SW_128B);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t koff = (kk / 4) * 128 * 128 + (kk % 4) * 32;  // K: 128-row chunks
          const uint32_t qoff = (kk / 4) * C::BQ * 128 + (kk % 4) * 32;  // Q: 64-row chunks
          mma_ss(tbase + (it & 1) * 64, desc_add(dK0, koff), desc_add(dq0, qoff), id_s, kk > 0);
        }
        mma_commit(&bars->s_full[it & 1]);
      };
      auto issue_dp = [&](int it) {  // dP^T(it) = V dO^T -> dP^T buffer it&1
        const uint64_t ddo0 = smem_desc(aDO + (it % C::NS) * C::Q_TILE, 16, 1024, SW_128B);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t koff = (kk / 4) * 128 * 128 + (kk % 4) * 32;
          const uint32_t qoff = (kk / 4) * C::BQ * 128 + (kk % 4) * 32;
          mma_ss(tbase + 128 + (it & 1) * 64, desc_add(dV0, koff), desc_add(ddo0, qoff), id_s, kk > 0);
        }
        mma_commit(&bars->dp_full[it & 1]);
      };
      // Per tile j, once its elementwise stage is done: dV(j), dK(j), dQ^T(j)
      // into the dP^T buffer elementwise(j) consumed, then for tile j+2: S^T
      // (in issue order after dV(j), which reads P(j) from the same columns)
      // and, once dQ^T(j) is drained, dP^T.  S^T and dP^T of tile j+1 were
      // issued a tile earlier, so elementwise(j+1) starts without waiting.
      if (b_wait(&bars->kv_full, 0, failed) && ntiles > 0 && b_wait(&bars->q_full[0], 0, failed)) {
        tc_fence_after();
        issue_s(0);
        issue_dp(0);
        if (ntiles > 1 && b_wait(&bars->q_full[1], 0, failed)) {
          tc_fence_after();
          issue_s(1);
          issue_dp(1);
        }
        for (int it = 0; it < ntiles && !failed; ++it) {
          const int bb = it & 1, st = it % C::NS;
          if (!b_wait(&bars->p_ready, it & 1, failed)) break;
          tc_fence_after();
          const uint32_t q_s = aQ + st * C::Q_TILE, do_s = aDO + st * C::Q_TILE;
          const uint32_t ds_s = aDS + bb * C::DS_TILE;
          const uint64_t bdo0 = smem_desc(do_s, C::BQ * 128, 1024, SW_128B);
          const uint64_t bq0 = smem_desc(q_s, C::BQ * 128, 1024, SW_128B);
          const uint64_t ads0 = smem_desc(ds_s, 16, 1024, SW_128B);
          const uint64_t bds0 = smem_desc(ds_s, C::DS_TILE, 1024, SW_128B);
#pragma unroll
          for (int kk = 0; kk < C::BQ / 16; ++kk) {  // dV += P^T dO, K = 64 query rows
            const uint64_t b_do = desc_add(bdo0, kk * 16 * 128);
            // P of query rows [16 kk, 16 kk + 16) sits at columns 32 (kk / 2) + 8 (kk % 2)
            mma_ts(tDV, tbase + bb * 64 + (kk >> 1) * 32 + (kk & 1) * 8, b_do, id_kv, (it > 0 || kk > 0) ? 1u : 0u);
          }
#pragma unroll
          for (int kk = 0; kk < C::BQ / 16; ++kk) {  // dK += dS^T Q
            mma_ss(tDK, desc_add(ads0, kk * 32), desc_add(bq0, kk * 16 * 128), id_kv, (it > 0 || kk > 0) ? 1u : 0u);
          }
#pragma unroll
          for (int kk = 0; kk < C::BN / 16; ++kk) {  // dQ^T = K^T dS^T into dP^T buffer bb (consumed)
            mma_ss(tbase + 128 + bb * 64, desc_add(dKt0, kk * 16 * 128), desc_add(bds0, kk * 16 * 128), id_dq, kk > 0);
          }
          mma_commit(&bars->mm2_done[bb]);
          mma_commit(&bars->q_empty[st]);
          if (it + 2 < ntiles) {
            const int nx = it + 2;
            if (!b_wait(&bars->q_full[nx % C::NS], (nx / C::NS) & 1, failed)) break;
            tc_fence_after();
            // S^T(nx) overwrites the columns dV(it) reads P from: tcgen05.mma
            // ops of one thread execute in issue order, so no wait is needed.
            issue_s(nx);
            if (!b_wait(&bars->dq_free, it & 1, failed)) break;
            tc_fence_after();
            issue_dp(nx);
          }
        }
      }
      mma_commit(&bars->all_done);
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ dQ drain
    const int g = warp & 3;
    const int d = 32 * g + lane;  // TMEM lane = head-dim index of dQ^T
    const uint32_t tl = tbase + ((uint32_t)(32 * g) << 16);
    Cursor cur{kvh * G, qt_first};
    for (int it = 0; it < ntiles && !failed; ++it, advance(cur)) {
      // polling (not suspending): the drain's reaction time gates the next dP^T
      if (!b_warp_wait_spin(&bars->mm2_done[it & 1], (it >> 1) & 1, failed)) break;
      tc_fence_after();
      uint32_t v0[32], v1[32];
      tmem_ld32(tl + 128 + (it & 1) * 64, v0);  // dQ^T(it) sits in dP^T buffer it&1
      tmem_ld32(tl + 128 + (it & 1) * 64 + 32, v1);
      tmem_ld_wait(v0);
      tmem_ld_wait(v1);
      tc_fence_before();
      mbar_arrive(&bars->dq_free);
      const int h = cur.h;
      const int q0 = cur.qt * C::BQ;
      if (!SA_DCHECK(h < p.Hq && q0 < p.T)) continue;  // the dQ rows of a query tile that exists
      float* dst = p.dq_acc + (((int64_t)b * p.Hq + h) * p.T + q0) * D + d;
      const int lim = p.T - q0;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < lim) atomicAdd(dst + (int64_t)j * D, __uint_as_float(v0[j]));
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (32 + j < lim) atomicAdd(dst + (int64_t)(32 + j) * D, __uint_as_float(v1[j]));
    }
  } else {
    // ------------------------------------------------------------ elementwise warpgroups
    const int w2 = warp >> 2;  // query-column half
    const int g = warp & 3;
    const int r = 32 * g + lane;  // TMEM lane = KV row
    const int n = n0 + r;
    const int tid = threadIdx.x;  // 0..255
    const uint32_t tl = tbase + ((uint32_t)(32 * g) << 16);
    const float scale2 = 2.0f * p.scale;
    // R and delta of the next tile's query column `tid` (threads 0..63) are
    // loaded a tile ahead into registers.  The loads are unconditional (from a
    // valid index) and the validity flag is applied when the values are used,
    // so nothing waits on the load before the tile's barrier.
    float pre_r = 0.f, pre_d = 0.f;
    bool pre_ok = false;
    Cursor nxt{kvh * G, qt_first};  // tile the next prefetch loads
    auto prefetch = [&](int it) {  // threads 0..63: R and delta of query column tid
      const Cursor c = nxt;
      advance(nxt);
      if (tid >= 64) return;
      const int h = it < ntiles ? c.h : kvh * G;
      const int qq = c.qt * C::BQ + tid;
      pre_ok = it < ntiles && qq < p.T;
      const int64_t idx = ((int64_t)b * p.Hq + h) * p.T + (qq < p.T ? qq : 0);
      pre_r = __ldg(p.rowsum + idx);
      pre_d = __ldg(p.delta + idx);
    };
    prefetch(0);
    Cursor cur{kvh * G, qt_first};
    for (int it = 0; it < ntiles && !failed; ++it, advance(cur)) {
      const int bb = it & 1;
      const int q0 = cur.qt * C::BQ;
      // buffer bb was last read in tile it-2; every thread finished that
      // before the barrier below of tile it-1, so no barrier is needed here
      if (tid < 64) {
        const float ir = pre_ok ? 1.0f / pre_r : 0.f;
        float* vb = vVec + bb * 192;
        vb[tid] = 0.25f * ir;
        vb[64 + tid] = p.scale * ir;
        vb[128 + tid] = -(pre_d * p.scale * ir);  // stored negated: dP*cs - cd is one fma
      }
      ew_sync();
      prefetch(it + 1);
      // all 256 threads leave together on a timeout (the chunk below has a named barrier)
      if (!ew_all(mbar_wait(&bars->s_full[bb], (it >> 1) & 1) && mbar_wait(&bars->dp_full[bb], (it >> 1) & 1))) {
        if (tid == 0) atomicAdd(&g_flash_bwd_timeouts, 1u);
        failed = true;
        break;
      }
      tc_fence_after();
      const int q0g = q0 + p.qoff, qend = p.qoff + p.T;  // global query positions
      const bool need_mask = (q0g < n0 + C::BN - 1) || (q0 + C::BQ > p.T) || (n0 + C::BN > p.Tk) ||
                             (p.window > 0 && q0g + C::BQ - 1 - n0 >= p.window);
      uint8_t* dsrow = sDS + bb * C::DS_TILE + r * 128;
      if (need_mask)
        bwd128_chunk<BF16, EXACT, true>(tl + bb * 64, tl + 128 + bb * 64, w2, dsrow, r, vVec + bb * 192, scale2,
                                        n, q0g, qend, p.Tk, p.window);
      else
        bwd128_chunk<BF16, EXACT, false>(tl + bb * 64, tl + 128 + bb * 64, w2, dsrow, r, vVec + bb * 192, scale2,
                                         n, q0g, qend, p.Tk, p.window);
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_ready);
    }
    // epilogue: warpgroup 0 writes dK, warpgroup 1 writes dV (TMEM lane = KV row)
    if (b_warp_wait(&bars->all_done, 0, failed)) {
      tc_fence_after();
      const bool live = n < p.Tk;
      uint8_t* base = static_cast<uint8_t*>(w2 ? p.dv : p.dk) +
                      2 * (w2 ? ((int64_t)b * p.sdv_b + (int64_t)kvh * p.sdv_h + (int64_t)n * p.sdv_s)
                              : ((int64_t)b * p.sdk_b + (int64_t)kvh * p.sdk_h + (int64_t)n * p.sdk_s));
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tl + 256 + w2 * 128 + c * 32, v);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          pk[e / 2] = BF16 ? pack2_bf16(__uint_as_float(v[e]), __uint_as_float(v[e + 1]))
                           : pack2_f16(__uint_as_float(v[e]), __uint_as_float(v[e + 1]));
        if (live) {
          uint4* dst = reinterpret_cast<uint4*>(base + c * 64);
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------------------
// D = 128 backward, dK and dV only (the deterministic path): one CTA per 128-row KV tile of one (b, kv head),
// 128-row query tiles, so every tcgen05.mma is 128 x 128 x 16 (an N = 64 MMA
// takes 48 tensor cycles for half the work of a 64-cycle N = 128 one).  K and
// V stay in shared memory; Q / dO stream through two stages.  dQ comes from
// the query-major kernel below (sp2_bwd_dq_kernel), which sums it in a fixed
// order.  (Summing dQ here, with 128-row query tiles, took fp32 atomics of
// twice the partials per CTA and ran slower than the 64-row kernel above.)
//
// TMEM (512 columns): S^T @0 (P is written over it), dP^T @128, dK @256,
// dV @384.  With S^T and dP^T single-buffered, the elementwise stage runs in
// two halves so that it overlaps the MMAs:
//   P half  (needs S^T(i)):  P = sp^2 / R -> TMEM (16-bit, over S^T);
//                            g = 4 sp sp' = t^2 rsqrt(a^2 + 4) stays in registers
//   dS half (needs dP^T(i)): dS = (dP scale/R - delta scale/R) g -> shared memory
// Tensor-pipe order per tile: dV(i) += P^T dO, S^T(i+1) = K Q^T,
// dK(i) += dS^T Q, dP^T(i+1) = V dO^T.  The P half of tile i+1 runs under
// dK(i) and dP^T(i+1), the dS half of tile i under dV(i) and S^T(i+1).
// Warps: 0-15 elementwise (four warpgroups of 32 query columns; thread = KV
// row: four warps per scheduler hide the TMEM-load and MUFU latencies),
// 16 TMA, 17 MMA.
// ---------------------------------------------------------------------------
struct DkvCfg {
  static constexpr int D = 128, BN = 128, BQ = 128, NS = 2;
  static constexpr int TILE = 128 * D * 2;     // 32 KB: two 64-column chunks of 128 rows x 128 B
  static constexpr int CH = 128 * 128;         // one chunk
  static constexpr int VEC_TILE = 2 * BQ * 4;  // per query column: 1/R, -delta scale/R
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE;
  static constexpr int OFF_Q = OFF_V + TILE;
  static constexpr int OFF_DO = OFF_Q + NS * TILE;
  static constexpr int OFF_DS = OFF_DO + NS * TILE;  // dS [kv 128][q 128] as two 64-query chunks
  static constexpr int OFF_VEC = OFF_DS + TILE;
  static constexpr int OFF_BAR = OFF_VEC + NS * VEC_TILE;
  // no alignment slack: the kernel checks that dynamic shared memory starts
  // on a 1024-byte boundary (it does when the kernel has no static shared data)
  static constexpr int SMEM = OFF_BAR + 128;
  static constexpr int EW = 512;  // elementwise threads
  static constexpr int THREADS = EW + 64;
  static_assert(SMEM <= 227 * 1024, "shared memory plan");
};

struct DkvBars {
  uint64_t kv_full;
  uint64_t q_full[2], q_empty[2];
  uint64_t s_full;    // S^T(i) in TMEM
  uint64_t dp_full;   // dP^T(i) in TMEM (and every earlier MMA done)
  uint64_t p_ready;   // P(i) in TMEM (512 arrivals)
  uint64_t ds_ready;  // dS(i) in shared memory and dP^T(i) read (512 arrivals)
  uint64_t all_done;
  uint32_t tmem_base;
};
static_assert(sizeof(DkvBars) <= 128, "barrier block");

// P half for the 32 query columns [32 w4, 32 w4 + 32) of KV row `n`.  P
// (16-bit) goes over the first 16 of these 32 S^T columns; g is returned.
// ir[m] = 1/R of query column m; the products round as P = t*t*(ir/4) and
// g = t*t*rsqrt(a^2+4).
template <bool BF16, bool EXACT, bool MASK>
__device__ __forceinline__ void dkv_p(uint32_t tS, int w4, const float* ir, float scale2, float (&g)[32],
                                         int n, int q0, int qend, int Tk, int window) {
  uint32_t sv[32];
  tmem_ld32(tS + 32 * w4, sv);
  tmem_ld_wait(sv);
  uint32_t pk[16];
#pragma unroll
  for (int e = 0; e < 32; e += 4) {
    const int col = 32 * w4 + e;
    const float4 irv = *reinterpret_cast<const float4*>(ir + col);
    const float2 irp[2] = {make_float2(irv.x, irv.y), make_float2(irv.z, irv.w)};
#pragma unroll
    for (int u = 0; u < 4; u += 2) {
      const float2 a = ffma2(make_float2(__uint_as_float(sv[e + u]), __uint_as_float(sv[e + u + 1])),
                             make_float2(scale2, scale2), make_float2(-1.0f, -1.0f));
      const float2 w = ffma2(a, a, make_float2(4.0f, 4.0f));
      const float2 rs = make_float2(rsqrt_approx(w.x), rsqrt_approx(w.y));
      const float2 t = EXACT ? make_float2(a.x + sqrtf(w.x), a.y + sqrtf(w.y)) : ffma2(w, rs, a);
      const float2 tt = fmul2(t, t);
      float2 pp = fmul2(tt, fmul2(make_float2(0.25f, 0.25f), irp[u / 2]));
      float2 gg = fmul2(tt, rs);
      if (MASK) {
        const int q = q0 + col + u;  // global query position
        const bool ok0 = (n <= q) && (q < qend) && (n < Tk) && (window <= 0 || q - n < window);
        const bool ok1 = (n <= q + 1) && (q + 1 < qend) && (n < Tk) && (window <= 0 || q + 1 - n < window);
        pp.x = ok0 ? pp.x : 0.f;
        gg.x = ok0 ? gg.x : 0.f;
        pp.y = ok1 ? pp.y : 0.f;
        gg.y = ok1 ? gg.y : 0.f;
      }
      g[e + u] = gg.x;
      g[e + u + 1] = gg.y;
      pk[(e + u) / 2] = BF16 ? pack2_bf16(pp.x, pp.y) : pack2_f16(pp.x, pp.y);
    }
  }
  tmem_st8(tS + 32 * w4, *reinterpret_cast<const uint32_t(*)[8]>(&pk[0]));
  tmem_st8(tS + 32 * w4 + 8, *reinterpret_cast<const uint32_t(*)[8]>(&pk[8]));
}

// dS half: dS = (dP * scale/R - delta scale/R) * g for the same 32 columns,
// 16-bit, into row r of the 128-byte-swizzled dS chunk of 64 query columns
// (dsrow); these columns are the 64-byte half w4 & 1 of that row.
template <bool BF16, bool MASK>
__device__ __forceinline__ void dkv_ds(uint32_t tP, int w4, uint8_t* dsrow, int r, const float* ir,
                                          const float* ncd, float scale, const float (&g)[32], int n, int q0,
                                          int qend, int Tk, int window) {
  uint32_t dv[32];
  tmem_ld32(tP + 32 * w4, dv);
  tmem_ld_wait(dv);
  uint32_t dk[16];
#pragma unroll
  for (int e = 0; e < 32; e += 4) {
    const int col = 32 * w4 + e;
    const float4 irv = *reinterpret_cast<const float4*>(ir + col);
    const float4 cdv = *reinterpret_cast<const float4*>(ncd + col);
    const float2 irp[2] = {make_float2(irv.x, irv.y), make_float2(irv.z, irv.w)};
    const float2 cdp[2] = {make_float2(cdv.x, cdv.y), make_float2(cdv.z, cdv.w)};
#pragma unroll
    for (int u = 0; u < 4; u += 2) {
      const float2 cs = fmul2(make_float2(scale, scale), irp[u / 2]);
      float2 ds = fmul2(ffma2(make_float2(__uint_as_float(dv[e + u]), __uint_as_float(dv[e + u + 1])), cs,
                              cdp[u / 2]),
                        make_float2(g[e + u], g[e + u + 1]));
      if (MASK) {  // g is 0 there already; the select keeps garbage constants of padded columns out
        const int q = q0 + col + u;
        const bool ok0 = (n <= q) && (q < qend) && (n < Tk) && (window <= 0 || q - n < window);
        const bool ok1 = (n <= q + 1) && (q + 1 < qend) && (n < Tk) && (window <= 0 || q + 1 - n < window);
        ds.x = ok0 ? ds.x : 0.f;
        ds.y = ok1 ? ds.y : 0.f;
      }
      dk[(e + u) / 2] = BF16 ? pack2_bf16(ds.x, ds.y) : pack2_f16(ds.x, ds.y);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int piece = (4 * (w4 & 1) + j) ^ (r & 7);
    *reinterpret_cast<uint4*>(dsrow + piece * 16) = make_uint4(dk[4 * j], dk[4 * j + 1], dk[4 * j + 2], dk[4 * j + 3]);
  }
}

template <bool BF16, bool EXACT>
__global__ void __launch_bounds__(DkvCfg::THREADS, 1)
    sp2_bwd_dkv128_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmdo,
                      BwdParams p) {
  using C = DkvCfg;
  constexpr int D = C::D;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // never expected; all threads leave before any barrier
    if (threadIdx.x == 0) atomicAdd(&g_flash_bwd_timeouts, 1u);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sDO = smem + C::OFF_DO;
  uint8_t* sDS = smem + C::OFF_DS;
  float* vVec = reinterpret_cast<float*>(smem + C::OFF_VEC);  // [NS][2][128]
  DkvBars* bars = reinterpret_cast<DkvBars*>(smem + C::OFF_BAR);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int kvt, bhk;  // KV tile (0 = most query tiles) and (batch, kv head)
  grouped_longest_first((int)blockIdx.x, (p.Tk + C::BN - 1) / C::BN, p.B * p.Hkv, 1, kvt, bhk);
  const int n0 = kvt * C::BN;
  const int b = bhk / p.Hkv, kvh = bhk % p.Hkv;
  const int G = p.Hq / p.Hkv;
  int qt_first, qt_last;
  query_tile_range(p, n0, C::BN, C::BQ, qt_first, qt_last);
  const int per_head = qt_last - qt_first + 1;
  const int ntiles = per_head > 0 ? G * per_head : 0;
  if (ntiles == 0) {  // no query sees these keys: dK = dV = 0 (before any barrier)
    zero_dkdv<D, C::BN>(p, b, kvh, n0);
    return;
  }
  const int ntq = (p.T + C::BQ - 1) / C::BQ;  // query tiles per (b, h) in the constants array
  // Tiles run head-major: (head kvh*G + g, query tile qt_first .. qt_last).
  struct Cursor {
    int h, qt;
  };
  auto advance = [&](Cursor& c) {
    if (++c.qt > qt_last) {
      c.qt = qt_first;
      ++c.h;
    }
  };

  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->q_full[i], 1);
      mbar_init(&bars->q_empty[i], 1);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->dp_full, 1);
    mbar_init(&bars->p_ready, C::EW);
    mbar_init(&bars->ds_ready, C::EW);
    mbar_init(&bars->all_done, 1);
    fence_mbar_init();
  }
  if (warp == 17) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const uint32_t tS = tbase, tP = tbase + 128, tDK = tbase + 256, tDV = tbase + 384;
  bool failed = false;

  if (warp == 16) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      tma_prefetch_desc(&tmdo);
      mbar_arrive_expect_tx(&bars->kv_full, 2 * C::TILE);
      for (int c = 0; c < 2; ++c) {
        tma_load_4d(sK + c * C::CH, &tmk, c * 64, n0, kvh, b, &bars->kv_full);
        tma_load_4d(sV + c * C::CH, &tmv, c * 64, n0, kvh, b, &bars->kv_full);
      }
      Cursor cur{kvh * G, qt_first};
      for (int it = 0; it < ntiles && !failed; ++it, advance(cur)) {
        const int st = it & 1;
        if (it >= 2 && !b_wait(&bars->q_empty[st], ((it >> 1) - 1) & 1, failed)) break;
        const int h = cur.h;
        const int q0 = cur.qt * C::BQ;
        mbar_arrive_expect_tx(&bars->q_full[st], 2 * C::TILE + C::VEC_TILE);
        for (int c = 0; c < 2; ++c) {
          tma_load_4d(sQ + st * C::TILE + c * C::CH, &tmq, c * 64, q0, h, b, &bars->q_full[st]);
          tma_load_4d(sDO + st * C::TILE + c * C::CH, &tmdo, c * 64, q0, h, b, &bars->q_full[st]);
        }
        (void)SA_DCHECK(h < p.Hq && cur.qt < ntq);  // a constants block the prep kernel wrote
        bulk_g2s(vVec + st * 256, p.rvec + (((int64_t)b * p.Hq + h) * ntq + cur.qt) * 256, C::VEC_TILE,
                 &bars->q_full[st]);
      }
    }
  } else if (warp == 17) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr int ab = BF16 ? 1 : 0;
      constexpr uint32_t id_s = idesc_f16(128, 128, ab, 0, 0);  // S^T, dP^T: both K-major
      constexpr uint32_t id_kv = idesc_f16(128, D, ab, 0, 1);   // dV, dK: B (dO / Q) MN-major
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aQ = smem_u32(sQ), aDO = smem_u32(sDO);
      const uint64_t dK0 = smem_desc(aK, 16, 1024, SW_128B), dV0 = smem_desc(aV, 16, 1024, SW_128B);
      const uint64_t dSk0 = smem_desc(smem_u32(sDS), 16, 1024, SW_128B);  // dS^T as a K-major A (dK)
      // K-major operands: 16-element k-steps, 64-element chunks CH bytes apart
      auto koff = [](int kk) { return (uint32_t)((kk / 4) * C::CH + (kk % 4) * 32); };
      auto issue_s = [&](int it) {  // S^T(it) = K Q^T
        const uint64_t dq0 = smem_desc(aQ + (it & 1) * C::TILE, 16, 1024, SW_128B);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma_ss(tS, desc_add(dK0, koff(kk)), desc_add(dq0, koff(kk)), id_s, kk > 0);
        mma_commit(&bars->s_full);
      };
      auto issue_dp = [&](int it) {  // dP^T(it) = V dO^T
        const uint64_t ddo0 = smem_desc(aDO + (it & 1) * C::TILE, 16, 1024, SW_128B);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(tP, desc_add(dV0, koff(kk)), desc_add(ddo0, koff(kk)), id_s, kk > 0);
        mma_commit(&bars->dp_full);
      };
      if (b_wait(&bars->kv_full, 0, failed) && b_wait(&bars->q_full[0], 0, failed)) {
        tc_fence_after();
        issue_s(0);
        issue_dp(0);
        for (int it = 0; it < ntiles && !failed; ++it) {
          const int st = it & 1;
          const uint32_t q_s = aQ + st * C::TILE, do_s = aDO + st * C::TILE;
          const uint32_t acc0 = it > 0 ? 1u : 0u;
          if (!b_wait(&bars->p_ready, it & 1, failed)) break;
          tc_fence_after();
          // dV += P^T dO: P of query rows [16 kk, 16 kk + 16) sits at columns 32 (kk / 2) + 8 (kk % 2)
          const uint64_t bdo0 = smem_desc(do_s, C::CH, 1024, SW_128B);
#pragma unroll
          for (int kk = 0; kk < C::BQ / 16; ++kk)
            mma_ts(tDV, tS + (kk >> 1) * 32 + (kk & 1) * 8, desc_add(bdo0, kk * 16 * 128), id_kv, (acc0 | kk) ? 1u : 0u);
          if (it + 1 < ntiles) {
            // S^T(it+1) overwrites the columns dV(it) reads P from: tcgen05.mma
            // ops of one thread execute in issue order, so no wait is needed.
            if (!b_wait(&bars->q_full[(it + 1) & 1], ((it + 1) >> 1) & 1, failed)) break;
            tc_fence_after();
            issue_s(it + 1);
          }
          if (!b_wait(&bars->ds_ready, it & 1, failed)) break;
          tc_fence_after();
          const uint64_t bq0 = smem_desc(q_s, C::CH, 1024, SW_128B);
#pragma unroll
          for (int kk = 0; kk < C::BQ / 16; ++kk)  // dK += dS^T Q
            mma_ss(tDK, desc_add(dSk0, koff(kk)), desc_add(bq0, kk * 16 * 128), id_kv, (acc0 | kk) ? 1u : 0u);
          mma_commit(&bars->q_empty[st]);
          // dP^T(it) was read before ds_ready; dp_full(it+1) also tells the
          // elementwise warps that dK(it) is done with the dS tile
          if (it + 1 < ntiles) issue_dp(it + 1);
        }
      }
      mma_commit(&bars->all_done);
    }
  } else {
    // ------------------------------------------------------------ elementwise warpgroups
    const int w4 = warp >> 2;  // query-column quarter
    const int g = warp & 3;
    const int r = 32 * g + lane;  // TMEM lane = KV row
    const int n = n0 + r;
    const uint32_t tl = tbase + ((uint32_t)(32 * g) << 16);
    const float scale2 = 2.0f * p.scale;
    uint8_t* dsrow = sDS + (w4 >> 1) * C::CH + r * 128;
    Cursor cur{kvh * G, qt_first};
    for (int it = 0; it < ntiles && !failed; ++it, advance(cur)) {
      const int st = it & 1;
      const int q0 = cur.qt * C::BQ;
      if (!b_warp_wait(&bars->s_full, it & 1, failed)) break;
      // the constants landed with Q(it); stage st is refilled only after dK(it)
      if (!b_warp_wait(&bars->q_full[st], (it >> 1) & 1, failed)) break;
      tc_fence_after();
      const int q0g = q0 + p.qoff, qend = p.qoff + p.T;  // global query positions
      const bool need_mask = (q0g < n0 + C::BN - 1) || (q0 + C::BQ > p.T) || (n0 + C::BN > p.Tk) ||
                             (p.window > 0 && q0g + C::BQ - 1 - n0 >= p.window);
      const float* ir = vVec + st * 256;
      float gv[32];
      if (need_mask)
        dkv_p<BF16, EXACT, true>(tl, w4, ir, scale2, gv, n, q0g, qend, p.Tk, p.window);
      else
        dkv_p<BF16, EXACT, false>(tl, w4, ir, scale2, gv, n, q0g, qend, p.Tk, p.window);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->p_ready);
      if (!b_warp_wait(&bars->dp_full, it & 1, failed)) break;
      tc_fence_after();
      if (need_mask)
        dkv_ds<BF16, true>(tl + 128, w4, dsrow, r, ir, ir + 128, p.scale, gv, n, q0g, qend, p.Tk, p.window);
      else
        dkv_ds<BF16, false>(tl + 128, w4, dsrow, r, ir, ir + 128, p.scale, gv, n, q0g, qend, p.Tk, p.window);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->ds_ready);
    }
    // epilogue: warpgroups 0-1 write dK, 2-3 write dV, 64 columns each (TMEM lane = KV row)
    if (b_warp_wait(&bars->all_done, 0, failed)) {
      tc_fence_after();
      const bool live = n < p.Tk;
      const int which = w4 >> 1, half = w4 & 1;
      uint8_t* base = static_cast<uint8_t*>(which ? p.dv : p.dk) +
                      2 * (which ? ((int64_t)b * p.sdv_b + (int64_t)kvh * p.sdv_h + (int64_t)n * p.sdv_s)
                                 : ((int64_t)b * p.sdk_b + (int64_t)kvh * p.sdk_h + (int64_t)n * p.sdk_s));
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {
        uint32_t v[32];
        tmem_ld32(tl + 256 + which * 128 + c * 32, v);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          pk[e / 2] = BF16 ? pack2_bf16(__uint_as_float(v[e]), __uint_as_float(v[e + 1]))
                           : pack2_f16(__uint_as_float(v[e]), __uint_as_float(v[e + 1]));
        if (live) {
          uint4* dst = reinterpret_cast<uint4*>(base + c * 64);
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 17) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------------------
// Deterministic dQ: one CTA per 128-row query tile of one (batch, query head),
// the reference's query-major order (src/smooth_attn/kernels.py:1680-1784).
// Every dQ element is summed inside one CTA's TMEM accumulator over the key
// tiles in a fixed order and written once, so the result is bitwise the same
// run to run (the key-major kernel's fp32 atomics are not).  Per key tile j:
//   S_j = Q K_j^T  (TMEM, double-buffered),  dP_j = dO V_j^T  (TMEM),
//   elementwise (thread = query row, 1/R and delta folded into registers):
//   dS = (dP scale/R - delta scale/R) * t^2 rsqrt(a^2+4), rounded to 16 bits
//   over S_j's own columns (the forward's P layout),
//   dQ += dS K_j  (A = dS from TMEM, B = K_j as an N-major operand).
// dP_{j+1} is issued as soon as the elementwise warps have read dP_j into
// registers, and S_{j+2} right after dQ_j, so the tensor pipe runs under the
// elementwise stage.  TMEM: S_0 @0, S_1 @128, dP @256, dQ @384 (D columns).
// Warps 0-15: elementwise (four warpgroups, 32 key columns each: four warps per
// scheduler hide the TMEM-load and MUFU latencies); warp 16: TMA; warp 17: MMA.
// ---------------------------------------------------------------------------
template <int D>
struct DqCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int CHUNK = D >= 64 ? 64 : D;  // elements per swizzled smem row
  static constexpr int NCHUNK = D / CHUNK;
  static constexpr int ROWB = CHUNK * 2;
  static constexpr uint32_t SWZ = ROWB == 128 ? SW_128B : SW_64B;
  static constexpr int SBO = 8 * ROWB;
  static constexpr int TILE = 128 * D * 2;  // one Q / dO / K / V tile
  static constexpr int NK = 3, NV = 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = OFF_Q + TILE;
  static constexpr int OFF_K = OFF_DO + TILE;
  static constexpr int OFF_V = OFF_K + NK * TILE;
  static constexpr int OFF_BAR = OFF_V + NV * TILE;
  // at least half an SM's shared memory: one CTA per SM, so a second CTA
  // never waits in tcgen05.alloc for the first one's 512 TMEM columns
  static constexpr int SMEM = OFF_BAR + 512 + 1024 > 116 * 1024 ? OFF_BAR + 512 + 1024 : 116 * 1024;
  static constexpr int EW = 512;  // elementwise threads
  static constexpr int THREADS = EW + 64;
  static_assert(SMEM <= 227 * 1024, "shared memory plan");
};

struct DqBars {
  uint64_t q_full;
  uint64_t k_full[3], k_empty[3];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];   // S_j ready in buffer j & 1
  uint64_t dp_full;     // dP_j ready
  uint64_t dp_read;     // dP_j read into registers (512 arrivals): the buffer is free
  uint64_t ds_full[2];  // dS_j written over S buffer j & 1 (512 arrivals)
  uint64_t dq_full;
  uint32_t tmem_base;
};

struct DqParams {
  void* dq;
  const float* rowsum;  // R  [B, Hq, T]
  const float* delta;   // [B, Hq, T]
  int64_t sdq_b, sdq_h, sdq_s;
  int B, Hq, Hkv, T, ntiles, window;
  int Tk, qoff;
  float scale;
};

// KV tile range [j0, j1) seen by the 128 query rows at local row q0.
__device__ __forceinline__ void dq_kv_range(int q0, int Tq, int qoff, int Tk, int window, int& j0, int& j1) {
  const int q0g = q0 + qoff;
  const int nkv = (Tk + 127) / 128;
  j1 = (q0g + 128 + 127) / 128;
  if (j1 > nkv) j1 = nkv;
  j0 = 0;
  if (window > 0) {
    const int first = q0g - window + 1;
    j0 = first > 0 ? first / 128 : 0;
  }
  if (q0 >= Tq || j1 < j0) j1 = j0;
}

// dS for 32 key columns of one query row already in registers (s: scores,
// g: dP); writes the 16-bit dS pairs (16 columns) at taddr and taddr + 8.
template <bool BF16, bool EXACT, bool MASK>
__device__ __forceinline__ void dq_ds32(const uint32_t (&s)[32], const uint32_t (&g)[32], uint32_t taddr,
                                        float scale2, float cs, float ncd, int kbase, int q, int Tk, int window) {
  uint32_t pk[16];
  const float2 sc2 = make_float2(scale2, scale2), m1 = make_float2(-1.0f, -1.0f), four = make_float2(4.0f, 4.0f);
  const float2 cs2 = make_float2(cs, cs), ncd2 = make_float2(ncd, ncd);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float2 a = ffma2(make_float2(__uint_as_float(s[2 * k]), __uint_as_float(s[2 * k + 1])), sc2, m1);
    const float2 w = ffma2(a, a, four);
    const float2 rs = make_float2(rsqrt_approx(w.x), rsqrt_approx(w.y));
    const float2 t = EXACT ? make_float2(a.x + sqrtf(w.x), a.y + sqrtf(w.y)) : ffma2(w, rs, a);
    // 4 sp sp' = t^2 rsqrt(w); dS = (dP scale/R - delta scale/R) * 4 sp sp'
    float2 ds = fmul2(ffma2(make_float2(__uint_as_float(g[2 * k]), __uint_as_float(g[2 * k + 1])), cs2, ncd2),
                      fmul2(fmul2(t, t), rs));
    if (MASK) {
      const int kk = kbase + 2 * k;
      const bool ok0 = (kk <= q) && (kk < Tk) && (window <= 0 || q - kk < window);
      const bool ok1 = (kk + 1 <= q) && (kk + 1 < Tk) && (window <= 0 || q - kk - 1 < window);
      ds.x = ok0 ? ds.x : 0.f;
      ds.y = ok1 ? ds.y : 0.f;
    }
    pk[k] = BF16 ? pack2_bf16(ds.x, ds.y) : pack2_f16(ds.x, ds.y);
  }
  tmem_st8(taddr, *reinterpret_cast<const uint32_t(*)[8]>(&pk[0]));
  tmem_st8(taddr + 8, *reinterpret_cast<const uint32_t(*)[8]>(&pk[8]));
}

template <int D, bool BF16, bool EXACT>
__global__ void __launch_bounds__(DqCfg<D>::THREADS, 1)
    sp2_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmdo,
                      DqParams p) {
  using C = DqCfg<D>;
  // Declared 1024-byte aligned (the swizzled tiles need it; the kernel has no
  // static shared data, so dynamic shared memory starts on such a boundary):
  // the compiler then folds the tile addresses (measured 4 % on the D = 128
  // backward).  A misaligned start is counted as a timeout and every thread leaves.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicAdd(&g_flash_bwd_timeouts, 1u);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sDO = smem + C::OFF_DO;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  DqBars* bars = reinterpret_cast<DqBars*>(smem + C::OFF_BAR);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int xr, bh;
  grouped_longest_first((int)blockIdx.x, p.ntiles, p.B * p.Hq, kHeadGroup, xr, bh);
  const int qt = p.ntiles - 1 - xr;  // x = 0: the tile with the most key tiles
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int kvh = h / (p.Hq / p.Hkv);
  const int q0 = qt * C::BM;
  int j0, j1;
  dq_kv_range(q0, p.T, p.qoff, p.Tk, p.window, j0, j1);
  const int n = j1 - j0;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->ds_full[i], C::EW);
    }
    mbar_init(&bars->dp_full, 1);
    mbar_init(&bars->dp_read, C::EW);
    mbar_init(&bars->dq_full, 1);
    fence_mbar_init();
  }
  if (warp == 17) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  bool failed = false;

  if (warp == 16) {
    // ------------------------------------------------------------ TMA producer
    // order of need: K_0, V_0, K_1, then V_{j+1} and K_{j+2} for j = 0, 1, ...
    if (elect_one()) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      tma_prefetch_desc(&tmdo);
      if (n > 0) mbar_arrive_expect_tx(&bars->q_full, 2 * C::TILE);  // no copy in flight when there is no work
      for (int c = 0; c < (n > 0 ? C::NCHUNK : 0); ++c) {
        tma_load_4d(sQ + c * 128 * C::ROWB, &tmq, c * C::CHUNK, q0, h, b, &bars->q_full);
        tma_load_4d(sDO + c * 128 * C::ROWB, &tmdo, c * C::CHUNK, q0, h, b, &bars->q_full);
      }
      auto load_k = [&](int i) {
        const int ks = i % C::NK;
        if (i >= C::NK && !b_wait(&bars->k_empty[ks], ((i / C::NK) - 1) & 1, failed)) return;
        mbar_arrive_expect_tx(&bars->k_full[ks], C::TILE);
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_load_4d(sK + ks * C::TILE + c * 128 * C::ROWB, &tmk, c * C::CHUNK, (j0 + i) * C::BN, kvh, b,
                      &bars->k_full[ks]);
      };
      auto load_v = [&](int i) {
        const int vs = i % C::NV;
        if (i >= C::NV && !b_wait(&bars->v_empty[vs], ((i / C::NV) - 1) & 1, failed)) return;
        mbar_arrive_expect_tx(&bars->v_full[vs], C::TILE);
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_load_4d(sV + vs * C::TILE + c * 128 * C::ROWB, &tmv, c * C::CHUNK, (j0 + i) * C::BN, kvh, b,
                      &bars->v_full[vs]);
      };
      if (n > 0) load_k(0);
      if (n > 0) load_v(0);
      if (n > 1) load_k(1);
      for (int j = 0; j < n && !failed; ++j) {
        if (j + 1 < n) load_v(j + 1);
        if (j + 2 < n) load_k(j + 2);
      }
    }
  } else if (warp == 17) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr int ab = BF16 ? 1 : 0;
      constexpr uint32_t id_sp = idesc_f16(128, C::BN, ab, 0, 0);  // S, dP: A, B K-major
      constexpr uint32_t id_dq = idesc_f16(128, D, ab, 0, 1);      // dQ: A (dS, TMEM), B = K N-major
      const uint64_t dQ0 = smem_desc(smem_u32(sQ), 16, C::SBO, C::SWZ);
      const uint64_t dDO0 = smem_desc(smem_u32(sDO), 16, C::SBO, C::SWZ);
      const uint64_t dK0 = smem_desc(smem_u32(sK), 16, C::SBO, C::SWZ);
      const uint64_t dV0 = smem_desc(smem_u32(sV), 16, C::SBO, C::SWZ);
      const uint64_t dKn0 = smem_desc(smem_u32(sK), 128 * C::ROWB, C::SBO, C::SWZ);  // K as N-major B
      auto gemm_kmajor = [&](uint32_t dst, uint64_t a0, uint64_t b0) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk * 16) / C::CHUNK) * 128 * C::ROWB + ((kk * 16) % C::CHUNK) * 2;
          mma_ss(dst, desc_add(a0, off), desc_add(b0, off), id_sp, kk > 0);
        }
      };
      auto issue_s = [&](int i) {
        const int ks = i % C::NK;
        if (!b_wait(&bars->k_full[ks], (i / C::NK) & 1, failed)) return;
        tc_fence_after();
        gemm_kmajor(tbase + (i & 1) * 128, dQ0, desc_add(dK0, ks * C::TILE));
        mma_commit(&bars->s_full[i & 1]);
      };
      auto issue_dp = [&](int i) {
        const int vs = i % C::NV;
        if (!b_wait(&bars->v_full[vs], (i / C::NV) & 1, failed)) return;
        tc_fence_after();
        gemm_kmajor(tbase + 256, dDO0, desc_add(dV0, vs * C::TILE));
        mma_commit(&bars->dp_full);
        mma_commit(&bars->v_empty[vs]);
      };
      if (n > 0 && b_wait(&bars->q_full, 0, failed)) {
        issue_s(0);
        issue_dp(0);
        if (n > 1) issue_s(1);
        for (int j = 0; j < n && !failed; ++j) {
          const int sb = j & 1;
          if (j + 1 < n) {
            // dP_{j+1} into the one dP buffer once dP_j is in the elementwise warps' registers
            if (!b_wait(&bars->dp_read, j & 1, failed)) break;
            issue_dp(j + 1);
          }
          if (!b_wait(&bars->ds_full[sb], (j >> 1) & 1, failed)) break;
          tc_fence_after();
          const uint64_t dk = desc_add(dKn0, (j % C::NK) * C::TILE);
#pragma unroll
          for (int kk = 0; kk < C::BN / 16; ++kk)
            mma_ts(tbase + 384, tbase + sb * 128 + (kk >> 1) * 32 + (kk & 1) * 8, desc_add(dk, kk * 16 * C::ROWB),
                   id_dq, (j > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&bars->k_empty[j % C::NK]);
          // S_{j+2} reuses the buffer dQ_j reads dS_j from: tcgen05.mma ops of
          // one thread execute in issue order
          if (j + 2 < n) issue_s(j + 2);
        }
      }
      mma_commit(&bars->dq_full);  // also when there was no work
    }
  } else {
    // ------------------------------------------------------------ elementwise warps
    const int qr = warp >> 2;  // key-column quarter
    const int g = warp & 3;
    const int row = 32 * g + lane;
    const int q = q0 + row;
    const int q0g = q0 + p.qoff, qg = q + p.qoff;
    const uint32_t tl = tbase + ((uint32_t)(32 * g) << 16);
    const float scale2 = 2.0f * p.scale;
    float cs = 0.f, ncd = 0.f;
    if (q < p.T) {
      const int64_t idx = ((int64_t)b * p.Hq + h) * p.T + q;
      const float ir = 1.0f / __ldg(p.rowsum + idx);
      cs = p.scale * ir;
      ncd = -(__ldg(p.delta + idx) * p.scale * ir);
    }
    for (int j = 0; j < n; ++j) {
      const int sb = j & 1;
      if (!b_warp_wait(&bars->dp_full, j & 1, failed)) break;
      if (!b_warp_wait(&bars->s_full[sb], (j >> 1) & 1, failed)) break;
      tc_fence_after();
      // dP_j and S_j load together: one TMEM-load latency per key tile
      const int col = qr * 32;  // first score column of this warp's 32-column chunk
      uint32_t gd[32], sv[32];
      tmem_ld32(tl + 256 + qr * 32, gd);
      tmem_ld32(tl + sb * 128 + col, sv);
      tmem_ld_wait(gd);
      tmem_ld_wait(sv);
      tc_fence_before();
      mbar_arrive(&bars->dp_read);
      {
        const int kc = (j0 + j) * C::BN + col;
        const bool need_mask = (kc + 31 > q0g) || (kc + 32 > p.Tk) ||
                               (p.window > 0 && q0g + C::BM - 1 - kc >= p.window) || q0 + C::BM > p.T;
        // need_mask is the same for the whole warp: dq_ds32's tcgen05.st is
        // a warp-collective (.sync.aligned) and must not run diverged
        // dS of keys [col, col + 32) -> columns 32 (m / 2) + 8 (m % 2) for the
        // two 16-key slices m = col / 16, col / 16 + 1: inside this chunk's
        // own, already-read first 16 columns
        const uint32_t tds = tl + sb * 128 + col;
        const uint32_t(&gc)[32] = gd;
        if (need_mask)
          dq_ds32<BF16, EXACT, true>(sv, gc, tds, scale2, cs, ncd, kc, q < p.T ? qg : -1, p.Tk, p.window);
        else
          dq_ds32<BF16, EXACT, false>(sv, gc, tds, scale2, cs, ncd, 0, 0, 0, 0);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->ds_full[sb]);
    }
    if (b_warp_wait(&bars->dq_full, 0, failed) && n > 0) {
      tc_fence_after();
      const bool live = q < p.T;
      uint8_t* drow = static_cast<uint8_t*>(p.dq) + 2 * ((int64_t)b * p.sdq_b + (int64_t)h * p.sdq_h + (int64_t)q * p.sdq_s);
#pragma unroll 1
      for (int c = qr; c < D / 16; c += 4) {  // 16 columns at a time, shared by the four warpgroups
        uint32_t r[16];
        tmem_ld16(tl + 384 + c * 16, r);
        tmem_ld_wait(r);
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2)
          pk[e / 2] = BF16 ? pack2_bf16(__uint_as_float(r[e]), __uint_as_float(r[e + 1]))
                           : pack2_f16(__uint_as_float(r[e]), __uint_as_float(r[e + 1]));
        if (live) {
          uint4* dst = reinterpret_cast<uint4*>(drow + c * 32);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
    } else if (n == 0 && !failed && q < p.T) {  // no visible key: dq = 0
      uint8_t* drow = static_cast<uint8_t*>(p.dq) + 2 * ((int64_t)b * p.sdq_b + (int64_t)h * p.sdq_h + (int64_t)q * p.sdq_s);
      for (int c = qr; c < D / 8; c += 4) reinterpret_cast<uint4*>(drow)[c] = make_uint4(0u, 0u, 0u, 0u);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 17) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// delta = rowsum(dO * O) (fp32) and dq_acc = 0.  One warp per query row.
template <typename T, int D>
__global__ void __launch_bounds__(256) sp2_bwd_prep(const T* __restrict__ o, const T* __restrict__ o_lo,
                                                    const T* __restrict__ dout,
                                                      float* __restrict__ delta, float* __restrict__ dq_acc,
                                                      int64_t rows, int Hq, int Tlen, int64_t so_b, int64_t so_h,
                                                      int64_t so_s, int64_t sd_b, int64_t sd_h, int64_t sd_s,
                                                      const float* __restrict__ rowsum, float* __restrict__ rvec,
                                                      float scale) {
  // delta = rowsum(dO * O) and a zeroed fp32 dQ accumulator.  LPR lanes per
  // row (16 bytes each of O and dO); two rows per lane group per pass so four
  // 16-byte loads are in flight per thread; grid-stride over the rows.
  constexpr int VEC = 8;  // 16 bytes of 16-bit elements
  constexpr int LPR = D / VEC;
  constexpr int RPB = 256 / LPR;  // rows per block per pass
  const int sub = threadIdx.x % LPR;
  const int64_t stride = (int64_t)gridDim.x * RPB;
  auto addr = [&](int64_t row, const T* base, int64_t sb, int64_t sh, int64_t ss) {
    const int t = (int)(row % Tlen);
    const int64_t bh = row / Tlen;
    return base + (bh / Hq) * sb + (bh % Hq) * sh + (int64_t)t * ss + sub * VEC;
  };
  for (int64_t r0 = (int64_t)blockIdx.x * RPB + threadIdx.x / LPR; r0 < rows; r0 += 2 * stride) {
    const int64_t r1 = r0 + stride;
    const bool two = r1 < rows;
    Pack<T, VEC> a0, c0, a1, c1, l0, l1;
    a0.u = *reinterpret_cast<const uint4*>(addr(r0, o, so_b, so_h, so_s));
    c0.u = *reinterpret_cast<const uint4*>(addr(r0, dout, sd_b, sd_h, sd_s));
    if (two) {
      a1.u = *reinterpret_cast<const uint4*>(addr(r1, o, so_b, so_h, so_s));
      c1.u = *reinterpret_cast<const uint4*>(addr(r1, dout, sd_b, sd_h, sd_s));
    }
    l0.zero();
    l1.zero();
    if (o_lo != nullptr) {  // o + o_lo = the forward's fp32 output to ~16 mantissa bits (exact in fp32)
      l0.u = *reinterpret_cast<const uint4*>(addr(r0, o_lo, so_b, so_h, so_s));
      if (two) l1.u = *reinterpret_cast<const uint4*>(addr(r1, o_lo, so_b, so_h, so_s));
    }
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc0 += (a0.get(e) + l0.get(e)) * c0.get(e);
    if (two) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc1 += (a1.get(e) + l1.get(e)) * c1.get(e);
    }
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) {
      acc0 += __shfl_xor_sync(0xffffffffu, acc0, off);
      acc1 += __shfl_xor_sync(0xffffffffu, acc1, off);
    }
    if (sub == 0) {
      delta[r0] = acc0;
      if (two) delta[r1] = acc1;
      if (rvec != nullptr) {  // the D = 128 kernel's per-column constants, one [2][128] block per query tile
        const int ntq = (Tlen + 127) / 128;
        auto put = [&](int64_t row, float dl) {
          const int t = (int)(row % Tlen);
          const int64_t bh = row / Tlen;
          float* blk = rvec + (bh * ntq + t / 128) * 256 + (t % 128);
          const float ir = 1.0f / rowsum[row];
          blk[0] = ir;
          blk[128] = -(dl * scale * ir);  // stored negated: dP*cs - cd is one fma
        };
        put(r0, acc0);
        if (two) put(r1, acc1);
      }
    }
    if (dq_acc == nullptr) continue;  // deterministic path: no accumulator
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = sub; i < D / 4; i += LPR) {
      reinterpret_cast<float4*>(dq_acc + r0 * D)[i] = z;
      if (two) reinterpret_cast<float4*>(dq_acc + r1 * D)[i] = z;
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(256) sp2_bwd_dq_convert(const float* __restrict__ dq_acc, T* __restrict__ dq,
                                                            int64_t rows, int Hq, int Tlen, int64_t s_b, int64_t s_h,
                                                            int64_t s_s) {
  constexpr int VEC = 8;
  constexpr int NV = D / VEC;  // vectors per row
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = idx / NV;
  const int v = (int)(idx % NV);
  if (row >= rows) return;
  const int t = (int)(row % Tlen);
  const int64_t bh = row / Tlen;
  const int b = (int)(bh / Hq), h = (int)(bh % Hq);
  const float4* src = reinterpret_cast<const float4*>(dq_acc + row * D + v * VEC);
  const float4 a = src[0], c = src[1];
  Pack<T, VEC> out;
  out.set(0, a.x); out.set(1, a.y); out.set(2, a.z); out.set(3, a.w);
  out.set(4, c.x); out.set(5, c.y); out.set(6, c.z); out.set(7, c.w);
  *reinterpret_cast<uint4*>(dq + (int64_t)b * s_b + (int64_t)h * s_h + (int64_t)t * s_s + v * VEC) = out.u;
}

template <int D, bool BF16, bool EXACT>
static int launch_bwd(const void* q, const void* k, const void* v, const void* o, const void* o_lo, const void* dout,
                      const float* rowsum, void* dq, void* dk, void* dv, float* dq_acc, float* delta, int64_t B,
                      int64_t Hq, int64_t Hkv, int64_t T, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                      const int64_t* os, const int64_t* dos, const int64_t* dqs, const int64_t* dks,
                      const int64_t* dvs, float scale, int64_t window, cudaStream_t st, int64_t Tk = -1,
                      int64_t qoff = 0, bool det = false) {
  using C = BwdCfg<D>;
  if (det) dq_acc = nullptr;  // dQ comes from the query-major kernel: no accumulator
  if (Tk < 0) Tk = T;
  if (((Tk + C::BN - 1) / C::BN) * B * Hkv > INT32_MAX) return SA_ERR_UNSUPPORTED;  // 1-D grid, before any launch
  using T16 = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int64_t rows = B * Hq * T;
  // [B*Hq][ceil(T/64)][3][64] fp32 after delta (sa_flash_bwd_workspace_size counts it)
  float* rvec = D == 128 && det ? delta + align256(rows * 4) / 4 : nullptr;
  int prep_dev = 0, prep_sms = 148;
  if (cudaGetDevice(&prep_dev) == cudaSuccess)
    cudaDeviceGetAttribute(&prep_sms, cudaDevAttrMultiProcessorCount, prep_dev);
  const int64_t prep_rpb = 256 / (D / 8);
  sp2_bwd_prep<T16, D><<<(unsigned)std::max<int64_t>(1, std::min<int64_t>((rows + prep_rpb - 1) / prep_rpb,
                                                                              (int64_t)prep_sms * 8)),
                           256, 0, st>>>(
      static_cast<const T16*>(o), static_cast<const T16*>(o_lo), static_cast<const T16*>(dout), delta, dq_acc, rows, (int)Hq, (int)T, os[0], os[1],
      os[2], dos[0], dos[1], dos[2], rowsum, rvec, scale);
  CUtensorMap mq, mk, mv, mdo;
  if (!make_map_4d(&mq, q, BF16, B, Hq, T, D, qs, C::CHUNK, C::BQ) ||
      !make_map_4d(&mk, k, BF16, B, Hkv, Tk, D, ks, C::CHUNK, C::BN) ||
      !make_map_4d(&mv, v, BF16, B, Hkv, Tk, D, vs, C::CHUNK, C::BN) ||
      !make_map_4d(&mdo, dout, BF16, B, Hq, T, D, dos, C::CHUNK, C::BQ))
    return SA_ERR_ALIGN;
  BwdParams p;
  p.dk = dk;
  p.dv = dv;
  p.rowsum = rowsum;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.rvec = rvec;
  p.sdk_b = dks[0]; p.sdk_h = dks[1]; p.sdk_s = dks[2];
  p.sdv_b = dvs[0]; p.sdv_h = dvs[1]; p.sdv_s = dvs[2];
  p.B = (int)B;
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.T = (int)T;
  p.Tk = (int)Tk;
  p.qoff = (int)qoff;
  p.window = (int)window;
  p.scale = scale;
  dim3 grid((unsigned)(((Tk + C::BN - 1) / C::BN) * B * Hkv));
  if constexpr (D == 128) {
    if (det) {
      auto kern = sp2_bwd_dkv128_kernel<BF16, EXACT>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DkvCfg::SMEM);
      kern<<<grid, DkvCfg::THREADS, DkvCfg::SMEM, st>>>(mq, mk, mv, mdo, p);
    } else {
      CUtensorMap mq64, mdo64;
      if (!make_map_4d(&mq64, q, BF16, B, Hq, T, D, qs, 64, Bwd128::BQ) ||
          !make_map_4d(&mdo64, dout, BF16, B, Hq, T, D, dos, 64, Bwd128::BQ))
        return SA_ERR_ALIGN;
      auto kern = sp2_bwd128_kernel<BF16, EXACT>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Bwd128::SMEM);
      kern<<<grid, Bwd128::THREADS, Bwd128::SMEM, st>>>(mq64, mk, mv, mdo64, p);
    }
  } else {
    auto kern = det ? sp2_bwd_kernel<D, BF16, EXACT, false> : sp2_bwd_kernel<D, BF16, EXACT, true>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    kern<<<grid, 192, C::SMEM, st>>>(mq, mk, mv, mdo, p);
  }
  if (det) {
    using DC = DqCfg<D>;
    DqParams dp;
    dp.dq = dq;
    dp.rowsum = rowsum;
    dp.delta = delta;
    dp.sdq_b = dqs[0];
    dp.sdq_h = dqs[1];
    dp.sdq_s = dqs[2];
    dp.B = (int)B;
    dp.Hq = (int)Hq;
    dp.Hkv = (int)Hkv;
    dp.T = (int)T;
    dp.Tk = (int)Tk;
    dp.qoff = (int)qoff;
    dp.window = (int)window;
    dp.scale = scale;
    dp.ntiles = (int)((T + DC::BM - 1) / DC::BM);
    if ((int64_t)dp.ntiles * B * Hq > INT32_MAX) return SA_ERR_UNSUPPORTED;
    auto kq = sp2_bwd_dq_kernel<D, BF16, EXACT>;
    cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, DC::SMEM);
    kq<<<(unsigned)(dp.ntiles * B * Hq), DC::THREADS, DC::SMEM, st>>>(mq, mk, mv, mdo, dp);
    return SA_OK;
  }
  const int64_t nthreads = rows * (D / 8);
  sp2_bwd_dq_convert<T16, D><<<(unsigned)((nthreads + 255) / 256), 256, 0, st>>>(
      dq_acc, static_cast<T16*>(dq), rows, (int)Hq, (int)T, dqs[0], dqs[1], dqs[2]);
  return SA_OK;
}

}  // namespace sqattn

int flash_bwd_timeouts(int reset, cudaStream_t st) {
  unsigned v = 0;
  cudaMemcpyFromSymbolAsync(&v, sqattn::g_flash_bwd_timeouts, sizeof(v), 0, cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  if (reset) {
    const unsigned z = 0;
    cudaMemcpyToSymbolAsync(sqattn::g_flash_bwd_timeouts, &z, sizeof(z), 0, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
  }
  return (int)v;
}

}  // namespace sa

int sa_record_cuda_error(cudaError_t e);

static bool bwd_strides_ok(const int64_t* s) {
  return s != nullptr && s[3] == 1 && s[0] % 8 == 0 && s[1] % 8 == 0 && s[2] % 8 == 0 && s[0] >= 0 && s[1] >= 0 &&
         s[2] > 0;
}


// 0 for empty problems and for sizes whose byte count does not fit in an
// int64 (every product below is checked before it is formed).
extern "C" int64_t sa_flash_bwd_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D) {
  (void)Hkv;
  if (B <= 0 || Hq <= 0 || T <= 0 || D <= 0) return 0;
  int64_t rows, elems, acc_bytes, total;
  if (__builtin_mul_overflow(B, Hq, &rows) || __builtin_mul_overflow(rows, T, &rows) ||
      __builtin_mul_overflow(rows, D, &elems) || __builtin_mul_overflow(elems, (int64_t)4, &acc_bytes) ||
      acc_bytes > INT64_MAX / 2 - 1024)
    return 0;
  // + the D = 128 kernel's per-query-tile constants: 1 KB per 128 query rows of each (b, h)
  int64_t bh, tiles, vec_bytes;
  if (__builtin_mul_overflow(B, Hq, &bh) || __builtin_mul_overflow(bh, (T + 127) / 128, &tiles) ||
      __builtin_mul_overflow(tiles, (int64_t)1024, &vec_bytes) || vec_bytes > INT64_MAX / 4)
    return 0;
  total = align256(acc_bytes) + align256(rows * 4) + align256(vec_bytes);
  return total;
}

extern "C" int sa_flash_bwd(const void* q, const void* k, const void* v, const void* o,
                            const void* o_lo, const void* dout,
                            const float* rowsum, void* dq, void* dk, void* dv, void* workspace,
                            int64_t workspace_bytes, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D,
                            const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                            const int64_t* o_strides, const int64_t* do_strides, const int64_t* dq_strides,
                            const int64_t* dk_strides, const int64_t* dv_strides, float scale, int64_t window_size,
                            int exact_math, int dtype, int deterministic, void* stream) {
  if (dtype != SA_BF16 && dtype != SA_F16) return SA_ERR_UNSUPPORTED;
  if (D != 32 && D != 64 && D != 128) return SA_ERR_UNSUPPORTED;
  if (B < 0 || Hq < 1 || Hkv < 1 || T < 0 || Hq % Hkv != 0 || window_size < 0) return SA_ERR_ARG;
  if (B == 0 || T == 0) return SA_OK;
  if (T > (1ll << 30) || B > INT32_MAX || Hq > INT32_MAX || B * Hq > INT32_MAX ||
      sa_flash_bwd_workspace_size(B, Hq, Hkv, T, D) <= 0)
    return SA_ERR_UNSUPPORTED;
  if (!q || !k || !v || !o || !dout || !rowsum || !dq || !dk || !dv || !workspace) return SA_ERR_ARG;
  if (workspace_bytes < sa_flash_bwd_workspace_size(B, Hq, Hkv, T, D)) return SA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return SA_ERR_ALIGN;
  const int64_t* all[8] = {q_strides, k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides};
  for (auto s : all)
    if (!bwd_strides_ok(s)) return SA_ERR_ALIGN;
  const void* ptrs[10] = {q, k, v, o, o_lo, dout, dq, dk, dv, rowsum};
  for (auto p : ptrs)
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return SA_ERR_ALIGN;
  float* dq_acc = static_cast<float*>(workspace);
  float* delta = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align256(B * Hq * T * D * 4));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  using namespace sa::sqattn;
  int rc;
#define SA_BWD_CASE(DD, BF, EX)                                                                                  \
  rc = launch_bwd<DD, BF, EX>(q, k, v, o, o_lo, dout, rowsum, dq, dk, dv, dq_acc, delta, B, Hq, Hkv, T, q_strides,     \
                              k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, \
                              scale, window_size, st, -1, 0, deterministic != 0)
#define SA_BWD_D(DD)                              \
  if (dtype == SA_BF16) {                         \
    if (exact_math) SA_BWD_CASE(DD, true, true);  \
    else SA_BWD_CASE(DD, true, false);            \
  } else {                                        \
    if (exact_math) SA_BWD_CASE(DD, false, true); \
    else SA_BWD_CASE(DD, false, false);           \
  }
  if (D == 32) {
    SA_BWD_D(32)
  } else if (D == 64) {
    SA_BWD_D(64)
  } else {
    SA_BWD_D(128)
  }
#undef SA_BWD_D
#undef SA_BWD_CASE
  if (rc != SA_OK) return rc;
  return sa_record_cuda_error(cudaGetLastError());
}

extern "C" int sa_flash_bwd_chunk(const void* q, const void* k, const void* v, const void* o,
                                  const void* o_lo, const void* dout,
                                  const float* rowsum, void* dq, void* dk, void* dv, void* workspace,
                                  int64_t workspace_bytes, int64_t B, int64_t Hq, int64_t Hkv, int64_t Tq, int64_t Tk,
                                  int64_t q_offset, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                                  const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
                                  const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                                  float scale, int64_t window_size, int exact_math, int dtype, int deterministic, void* stream) {
  if (dtype != SA_BF16 && dtype != SA_F16) return SA_ERR_UNSUPPORTED;
  if (D != 32 && D != 64 && D != 128) return SA_ERR_UNSUPPORTED;
  if (B < 0 || Hq < 1 || Hkv < 1 || Tq < 0 || Tk < 0 || q_offset < 0 || Hq % Hkv != 0 || window_size < 0)
    return SA_ERR_ARG;
  if (B == 0 || Tq == 0 || Tk == 0) return Tk == 0 && Tq > 0 ? SA_ERR_ARG : SA_OK;
  if (Tq > (1ll << 30) || Tk > (1ll << 30) || q_offset > (1ll << 30) || B > INT32_MAX || Hq > INT32_MAX ||
      B * Hq > INT32_MAX || sa_flash_bwd_workspace_size(B, Hq, Hkv, Tq, D) <= 0)
    return SA_ERR_UNSUPPORTED;
  if (!q || !k || !v || !o || !dout || !rowsum || !dq || !dk || !dv || !workspace) return SA_ERR_ARG;
  if (workspace_bytes < sa_flash_bwd_workspace_size(B, Hq, Hkv, Tq, D)) return SA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return SA_ERR_ALIGN;
  const int64_t* all[8] = {q_strides, k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides};
  for (auto s : all)
    if (!bwd_strides_ok(s)) return SA_ERR_ALIGN;
  const void* ptrs[10] = {q, k, v, o, o_lo, dout, dq, dk, dv, rowsum};
  for (auto p : ptrs)
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return SA_ERR_ALIGN;
  float* dq_acc = static_cast<float*>(workspace);
  float* delta = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align256(B * Hq * Tq * D * 4));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  using namespace sa::sqattn;
  int rc;
#define SA_BWDC_CASE(DD, BF, EX)                                                                                 \
  rc = launch_bwd<DD, BF, EX>(q, k, v, o, o_lo, dout, rowsum, dq, dk, dv, dq_acc, delta, B, Hq, Hkv, Tq, q_strides,   \
                              k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, \
                              scale, window_size, st, Tk, q_offset, deterministic != 0)
#define SA_BWDC_D(DD)                              \
  if (dtype == SA_BF16) {                          \
    if (exact_math) SA_BWDC_CASE(DD, true, true);  \
    else SA_BWDC_CASE(DD, true, false);            \
  } else {                                         \
    if (exact_math) SA_BWDC_CASE(DD, false, true); \
    else SA_BWDC_CASE(DD, false, false);           \
  }
  if (D == 32) {
    SA_BWDC_D(32)
  } else if (D == 64) {
    SA_BWDC_D(64)
  } else {
    SA_BWDC_D(128)
  }
#undef SA_BWDC_D
#undef SA_BWDC_CASE
  if (rc != SA_OK) return rc;
  return sa_record_cuda_error(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Allocation-free variant of sa_flash_bwd.
//
// Some callers cannot call cudaMalloc: code running inside a CUDA-graph
// capture that must not allocate, plugins whose host framework owns all
// device memory and forbids allocation, or real-time loops where an
// allocator call could stall.  For them the backward's scratch (the fp32 dQ
// accumulator and the per-row delta) lives in a fixed, file-scope device
// array instead of a caller-provided workspace.  Every GPU that loads this
// library holds the array (SA_NOALLOC_SCRATCH_BYTES) until the process exits.
// ---------------------------------------------------------------------------

#define SA_NOALLOC_SCRATCH_BYTES (32ll << 20)  // 32 MiB

static __device__ __align__(256) unsigned char g_bwd_noalloc_scratch[SA_NOALLOC_SCRATCH_BYTES];

#include <algorithm>
#include <mutex>

// Device address of the scratch array for the current device.  In host code
// the array's name is only a host-side handle; the real device address is
// looked up once per device (with that device current) and cached together
// with the CUDA context it belongs to.  A device reset or a new primary
// context reloads the module, possibly at another address, so a cached entry
// whose context is no longer the current one is looked up again.
static int noalloc_scratch(void** out) {
  using CtxGetCurrent = CUresult (*)(CUcontext*);
  static CtxGetCurrent ctx_get = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      ctx_get = reinterpret_cast<CtxGetCurrent>(fn);
  });
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  static CUcontext ctx[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return sa_record_cuda_error(e);
  if (dev < 0 || dev >= 64) return SA_ERR_UNSUPPORTED;
  CUcontext cur = nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] != nullptr && ctx_get != nullptr && ctx_get(&cur) == CUDA_SUCCESS && cur == ctx[dev]) {
    *out = addr[dev];
    return SA_OK;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_bwd_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) return sa_record_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
  cur = nullptr;
  if (ctx_get != nullptr && ctx_get(&cur) != CUDA_SUCCESS) cur = nullptr;
  addr[dev] = p;
  ctx[dev] = cur;
  *out = p;
  return SA_OK;
}

extern "C" int64_t sa_flash_bwd_noalloc_max_bytes(void) { return SA_NOALLOC_SCRATCH_BYTES; }

extern "C" int sa_flash_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                                    const void* o_lo, const void* dout,
                                    const float* rowsum, void* dq, void* dk, void* dv, int64_t B, int64_t Hq,
                                    int64_t Hkv, int64_t T, int64_t D, const int64_t* q_strides,
                                    const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                    const int64_t* do_strides, const int64_t* dq_strides, const int64_t* dk_strides,
                                    const int64_t* dv_strides, float scale, int64_t window_size, int exact_math,
                                    int dtype, void* stream) {
  const int64_t need = sa_flash_bwd_workspace_size(B, Hq, Hkv, T, D);
  // too large for the fixed scratch, or so large that the size overflows (0)
  if (need > SA_NOALLOC_SCRATCH_BYTES || (need == 0 && B > 0 && Hq > 0 && T > 0 && D > 0)) return SA_ERR_ARG;
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = noalloc_scratch(&scratch);
    if (rc != SA_OK) return rc;
  }
  return sa_flash_bwd(q, k, v, o, o_lo, dout, rowsum, dq, dk, dv, scratch, SA_NOALLOC_SCRATCH_BYTES, B, Hq, Hkv, T, D,
                      q_strides, k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides,
                      scale, window_size, exact_math, dtype, 0, stream);
}
SA_BOUNDS_ACCESSOR(flash_bwd_bounds)
