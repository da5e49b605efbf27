// Paged-KV decode attention on tcgen05 tensor cores (GQA groups, D = 128,
// bf16), sm_100a.  Same result as paged_decode_kernel (paged.cu) and the
// reference _sp2norm_paged_attention_kernel (src/smooth_attn/kernels.py:
// 2681-2773); this file only changes where the arithmetic runs.
//
// Why.  With G query heads per KV head the CUDA-core kernel spends 2 FMAs per
// cache element per head; at G = 4 that FP32 work, not HBM, bounds it.  Here
// the two products are MMAs and the CUDA cores only evaluate squareplus once
// per (token, head):
//   S^T[tok, g]  = K_tile[tok, :] . q_g            M = 128 tokens, N = 16 heads
//   O^T[d, g']  += V_tile^T[d, tok] . P[tok, g']   M = 128 = D,   N = 32
// P holds y as a hi + lo bf16 pair (columns g and 16 + g), so the product
// carries ~16 mantissa bits of y, close to the reference's fp32 y . v; O^T's
// two halves are added in fp32 at the end.  Heads past the group are zero
// columns.
//
// Pipeline (one CTA per SM, 7 warps): warps 0 and 6 stream the K and V pages
// of 128-token tiles with 4-D TMA boxes (one page of one KV head = 64 x block_size
// per box, 128-byte swizzle, the operand layout of both MMAs: K as a K-major
// A, V as an MN-major A) into a 3-stage ring, one page per lane (block-table
// entry and boxes), so a tile's boxes go out in one warp instruction; warp 1 issues S^T for tile i+1 before
// O^T += V.P for tile i, so the squareplus of one tile overlaps the MMAs of
// the next; warps 2-5 (one token row per thread) read S^T from TMEM, write P
// to shared memory in the swizzled K-major layout, zero V rows past the
// context on the last tile (rows that were never loaded may hold NaN bits),
// and at the end of a unit read O^T (one head-dim row per thread).
// Work split, partial records, tickets and the last-arriver combine are those
// of paged.cu, over (unit, tile) instead of (unit, chunk).  Every wait is
// bounded; a timeout is counted and the CTA leaves through the teardown.
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <algorithm>

#include "paged_tc.h"
#include "sa_sm100.cuh"
#include "smooth_attn_b200.h"

int sa_record_cuda_error(cudaError_t e);

namespace sa {
namespace sqattn {
bool make_map_4d(CUtensorMap* map, const void* base, bool bf16, int64_t B, int64_t H, int64_t T, int64_t D,
                 const int64_t* strides, int chunk, int rows, bool u8 = false);
}

namespace ptc {

using namespace sm100;

static __device__ unsigned g_ptc_timeouts;
static __device__ unsigned g_ptc_bad_pages;

constexpr int D = 128, TOK = 128, NH = 16, NS = 3;
constexpr int KT = TOK * D * 2;      // one K (or V) tile: 32 KB, two 16 KB D-halves
constexpr int HALF = TOK * 128;      // one D-half of a tile (128 rows x 128 B)
constexpr int OFF_K = 0;
constexpr int OFF_V = NS * KT;
constexpr int OFF_Q = 2 * NS * KT;   // 2 D-halves x 16 head rows x 128 B
constexpr int OFF_P = OFF_Q + 4096;  // 2 buffers x 2 token-halves x 32 rows x 128 B
constexpr int OFF_RED = OFF_P + 2 * 8192;
constexpr int OFF_BAR = OFF_RED + 1024;
constexpr int SMEM = OFF_BAR + 512 + 1024;  // + alignment slack
constexpr int THREADS = 224;  // K producer, MMA, 4 squareplus warps, V producer
constexpr uint32_t TMEM_COLS = 64;  // S^T x2 @0/@16, O^T @32

struct Args {
  const __nv_bfloat16* q;
  __nv_bfloat16* out;
  const int32_t* bt;
  const int32_t* cl;
  float* part;
  int32_t* tickets;
  int64_t num_blocks, W;
  int Hq, Hkv, G, GT, nhc, bs, max_blocks, M, slots;
  float scale2;
};

constexpr int IQ = 4;  // item queue entries

struct Bars {
  uint64_t k_full[NS], k_empty[NS], v_full[NS], v_empty[NS];
  uint64_t s_full[2], p_full[2], p_free[2];
  uint64_t q_full, o_full;
  uint64_t it_full[IQ], it_empty[IQ];
  int itq[IQ];
  uint32_t tmem_base;
  int last;
};
static_assert(sizeof(Bars) <= 512, "barrier block");

// All waits poll (test_wait) instead of suspending: every tile passes four
// hand-offs (TMA -> MMA -> squareplus -> MMA -> TMA) and a suspended
// thread's wake-up latency would add to each.  Still bounded (2 s).
__device__ __forceinline__ bool wait_uni(uint64_t* bar, uint32_t phase, bool& failed) {
  const bool ok = __all_sync(0xffffffffu, !failed && mbar_wait_spin(bar, phase));
  if (!ok) {
    if (!failed && (threadIdx.x & 31) == 0) atomicAdd(&g_ptc_timeouts, 1u);
    failed = true;
  }
  return ok;
}

// Single-thread bounded wait (TMA / MMA issuing threads).
__device__ __forceinline__ bool wait_or(uint64_t* bar, uint32_t phase, bool& failed) {
  if (failed) return false;
  if (!mbar_wait_spin(bar, phase)) {
    failed = true;
    atomicAdd(&g_ptc_timeouts, 1u);
    return false;
  }
  return true;
}

__device__ __forceinline__ void ew_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// A work item is one unit segment: tiles [t_lo, t_hi) of unit u (t_hi cut at
// the context) inside the CTA's contiguous range of the flattened (unit,
// tile) space, with its partial-record slot among the unit's nslots
// contributing CTAs.  (Handing out unit-aligned chunks from an atomic counter
// instead was measured slower on every shape: per-chunk epilogues and more
// partials cost more than the static split's imbalance.)
struct Unit {
  int u, b, h, hq0, ctx, t_lo, t_hi, slot, nslots;
  bool whole;  // the item covers the unit's every tile: output written directly
};

__device__ __forceinline__ Unit item_of(const Args& a, int id, int64_t x0, int64_t x1) {
  Unit r;
  r.u = id;
  const int64_t ub = (int64_t)id * a.M;
  const int64_t lo = max(x0, ub) - ub, hi = min(x1, ub + a.M) - ub;
  const int64_t NC = gridDim.x;
  const int64_t i0 = ((ub + 1) * NC - 1) / a.W;  // CTAs i0..i1 cover unit u
  const int64_t i1 = (min(a.W, ub + a.M) * NC - 1) / a.W;
  r.slot = (int)(blockIdx.x - i0);
  r.nslots = (int)(i1 - i0 + 1);
  const int upb = a.Hkv * a.nhc;
  r.b = r.u / upb;
  const int rem = r.u - r.b * upb;
  r.h = rem / a.nhc;
  r.hq0 = r.h * a.G + (rem - r.h * a.nhc) * a.GT;
  r.ctx = max(0, min(__ldg(a.cl + r.b), a.max_blocks * a.bs));
  r.whole = lo == 0 && hi == a.M;
  r.t_lo = (int)lo;
  r.t_hi = (int)min(hi, (int64_t)((r.ctx + TOK - 1) / TOK));
  return r;
}

__global__ void __launch_bounds__(THREADS, 1)
    paged_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, const Args a) {
  // Declared 1024-byte aligned (the kernel has no static shared data, so
  // dynamic shared memory starts on such a boundary; the swizzled tiles need
  // it).  A misaligned start is counted as a timeout and every thread leaves.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicAdd(&g_ptc_timeouts, 1u);
    return;
  }
  uint8_t* smem = smem_raw;
  Bars* bars = reinterpret_cast<Bars*>(smem + OFF_BAR);
  float* red = reinterpret_cast<float*>(smem + OFF_RED);  // [4][NH] warp sums, [NH] totals
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t NC = gridDim.x, cta = blockIdx.x;
  const int64_t x0 = cta * a.W / NC, x1 = (cta + 1) * a.W / NC;
  if (x0 >= x1) return;  // empty range, before any barrier
  const int u_first = (int)(x0 / a.M), u_last = (int)((x1 - 1) / a.M);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 128);
      mbar_init(&bars->p_free[i], 1);
    }
    for (int i = 0; i < IQ; ++i) {
      mbar_init(&bars->it_full[i], 1);
      mbar_init(&bars->it_empty[i], 3);  // V producer, MMA issuer, epilogue warps
    }
    mbar_init(&bars->q_full, 128);
    mbar_init(&bars->o_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  // zero both P buffers once: head rows past the group stay zero
  for (int i = threadIdx.x; i < 2 * 8192 / 16; i += THREADS)
    reinterpret_cast<uint4*>(smem + OFF_P)[i] = make_uint4(0u, 0u, 0u, 0u);
  // The producers start their first unit's context-length and block-table
  // loads now, so those DRAM round trips overlap the setup barrier.
  int pre_wu = -1, pre_wp = 0, pre_win = 0;
  if (warp == 0 || warp == 6) {
    const Unit U0 = item_of(a, u_first, x0, x1);
    pre_wu = u_first;
    pre_wp = U0.t_lo * (TOK / a.bs);
    if (pre_wp + lane < a.max_blocks) pre_win = __ldg(a.bt + (int64_t)U0.b * a.max_blocks + pre_wp + lane);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  bool failed = false;
  const int np = TOK / a.bs;  // pages per tile

  // Item queue: warp 0 publishes the ids of the CTA's units in order into a
  // 4-entry ring; every role walks the same ring.
  // take(k): the k-th item id of this CTA, -1 when there is no more work.
  auto take = [&](int k, bool release) -> int {
    const int sl = k % IQ;
    if (!wait_uni(&bars->it_full[sl], (k / IQ) & 1, failed)) return -1;
    const int id = bars->itq[sl];
    __syncwarp();
    if (release && lane == 0) mbar_arrive(&bars->it_empty[sl]);
    return id;
  };

  if (warp == 0 || warp == 6) {
    // ------------------------------------------------------------ TMA producers
    // warp 0 streams K (stage freed by the S^T MMA), warp 6 streams V (freed
    // by the P.V MMA), so K runs ahead of V instead of waiting behind it.
    const bool isv = warp == 6;
    const CUtensorMap* map = isv ? &tmv : &tmk;
    uint64_t* full = isv ? bars->v_full : bars->k_full;
    uint64_t* empty = isv ? bars->v_empty : bars->k_empty;
    uint8_t* ring = smem + (isv ? OFF_V : OFF_K);
    if (lane == 0) tma_prefetch_desc(map);
    int n = 0;
    int wu = pre_wu, wp = pre_wp, win = pre_win;  // block-table window: lane l holds page wp + l of unit wu
    for (int k = 0; !failed; ++k) {
      int id;
      if (!isv) {  // warp 0 publishes the k-th item
        const int sl = k % IQ;
        if (k >= IQ && !wait_uni(&bars->it_empty[sl], ((k / IQ) - 1) & 1, failed)) break;
        if (lane == 0) {
          bars->itq[sl] = u_first + k <= u_last ? u_first + k : -1;
          mbar_arrive(&bars->it_full[sl]);
        }
        id = __shfl_sync(0xffffffffu, lane == 0 ? bars->itq[sl] : 0, 0);
      } else {
        id = take(k, true);
      }
      if (id < 0) break;
      const Unit U = item_of(a, id, x0, x1);
      for (int ti = U.t_lo; ti < U.t_hi && !failed; ++ti, ++n) {
        const int s = n % NS;
        const int nload = min(np, (U.ctx - ti * TOK + a.bs - 1) / a.bs);
        const int p0 = ti * np;
        if (wu != U.u || p0 < wp || p0 + nload > wp + 32) {  // refill: one load covers 32 / np tiles
          wu = U.u;
          wp = p0;
          win = 0;
          if (wp + lane < a.max_blocks) win = __ldg(a.bt + (int64_t)U.b * a.max_blocks + wp + lane);
        }
        int phys = __shfl_sync(0xffffffffu, win, (p0 - wp + lane) & 31);
        if (lane < nload && (phys < 0 || phys >= a.num_blocks)) {
          if (!isv) atomicAdd(&g_ptc_bad_pages, 1u);
          phys = 0;
        }
        (void)SA_DCHECK(nload >= 1 && nload <= np && p0 + nload <= a.max_blocks);  // pages of this tile
        if (n >= NS && !wait_uni(&empty[s], ((n / NS) - 1) & 1, failed)) break;
        if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)nload * a.bs * D * 2);
        __syncwarp();
        if (lane < nload)  // one page per lane: the warp issues the tile's boxes together
          for (int c = 0; c < 2; ++c)
            tma_load_4d(ring + s * KT + c * HALF + lane * a.bs * 128, map, c * 64, 0, U.h, phys, &full[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = idesc_f16(128, NH, 1, 0, 0);
    constexpr uint32_t idesc_o = idesc_f16(128, 2 * NH, 1, 1, 0);
    const uint64_t dK0 = smem_desc(smem_u32(smem + OFF_K), 16, 1024, SW_128B);
    const uint64_t dV0 = smem_desc(smem_u32(smem + OFF_V), HALF, 1024, SW_128B);
    const uint64_t dQ0 = smem_desc(smem_u32(smem + OFF_Q), 16, 1024, SW_128B);
    const uint64_t dP0 = smem_desc(smem_u32(smem + OFF_P), 16, 1024, SW_128B);
    const bool leader = elect_one();
    const int leader_lane = __ffs(__ballot_sync(0xffffffffu, leader)) - 1;
    auto pv = [&](int m, bool first) {  // O^T += V_m^T . P_m
      const int s = m % NS;
      if (!wait_or(&bars->p_full[m & 1], (m >> 1) & 1, failed)) return;
      if (!wait_or(&bars->v_full[s], (m / NS) & 1, failed)) return;
      tc_fence_after();
      const uint64_t dv = desc_add(dV0, s * KT), dp = desc_add(dP0, (m & 1) * 8192);
#pragma unroll
      for (int kk = 0; kk < TOK / 16; ++kk)
        mma_ss(tbase + 32, desc_add(dv, kk * 16 * 128), desc_add(dp, (kk / 4) * 4096 + (kk % 4) * 32), idesc_o,
               (!first || kk > 0) ? 1u : 0u);
      mma_commit(&bars->v_empty[s]);
      mma_commit(&bars->p_free[m & 1]);
    };
    int n = 0, seg = 0;
    for (int k = 0; !failed; ++k) {
      const int id = take(k, true);  // whole warp: keeps the queue walk warp-uniform
      if (id < 0) break;
      const Unit U = item_of(a, id, x0, x1);
      if (U.t_hi <= U.t_lo) continue;
      if (leader && wait_or(&bars->q_full, seg & 1, failed)) {  // no early exit here: lanes stay converged
        const int n0 = n;
        for (int ti = U.t_lo; ti < U.t_hi && !failed; ++ti, ++n) {
          const int s = n % NS;
          if (!wait_or(&bars->k_full[s], (n / NS) & 1, failed)) break;
          tc_fence_after();
          const uint64_t dk = desc_add(dK0, s * KT);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk / 4) * HALF + (kk % 4) * 32;
            mma_ss(tbase + (n & 1) * NH, desc_add(dk, off), desc_add(dQ0, (kk / 4) * 2048 + (kk % 4) * 32),
                   idesc_s, kk > 0 ? 1u : 0u);
          }
          mma_commit(&bars->k_empty[s]);
          mma_commit(&bars->s_full[n & 1]);
          if (n > n0) pv(n - 1, n - 1 == n0);
        }
        if (!failed) pv(n - 1, n - 1 == n0);
        mma_commit(&bars->o_full);
      }
      if (!leader) n += U.t_hi - U.t_lo;
      ++seg;
      failed = __shfl_sync(0xffffffffu, failed, leader_lane) || failed;
    }
  } else if (warp >= 2 && warp <= 5) {
    // ------------------------------------------------------------ squareplus / epilogue warps
    const int e = threadIdx.x - 64;       // 0..127
    const int quad = warp & 3;            // TMEM lane quadrant of this warp
    const int row = 32 * quad + lane;     // token row of S^T, head-dim row of O^T
    const uint32_t tl = tbase + ((uint32_t)(32 * quad) << 16);
    const float eps4 = 4.0f * SA_EPS;
    // Item k+1's q goes in as soon as item k's O is out of TMEM (before k's
    // epilogue), so the MMAs of k+1 overlap the partial write / combine of k.
    auto take_ew = [&](int k) {
      const int id = take(k, false);
      ew_sync();  // every epilogue thread has read the entry
      if (e == 0 && !failed) mbar_arrive(&bars->it_empty[k % IQ]);
      return id;
    };
    auto write_q = [&](const Unit& U) {
      const int r = e >> 3, j = e & 7;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < a.GT)
          v = __ldg(reinterpret_cast<const uint4*>(a.q + ((int64_t)U.b * a.Hq + U.hq0 + r) * D + c * 64 + j * 8));
        *reinterpret_cast<uint4*>(smem + OFF_Q + c * 2048 + r * 128 + ((j ^ (r & 7)) * 16)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->q_full);
    };
    int n = 0, seg = 0;
    int id = take_ew(0);
    if (id >= 0) {
      const Unit U0 = item_of(a, id, x0, x1);
      if (U0.t_hi > U0.t_lo) write_q(U0);
    }
    for (int k = 0; id >= 0; ++k) {
      const Unit U = item_of(a, id, x0, x1);
      const bool busy = U.t_hi > U.t_lo;
      float ysum[NH];
#pragma unroll
      for (int g = 0; g < NH; ++g) ysum[g] = 0.f;
      float o[NH];
#pragma unroll
      for (int g = 0; g < NH; ++g) o[g] = 0.f;
      for (int ti = U.t_lo; ti < U.t_hi; ++ti, ++n) {
        const bool ok = wait_uni(&bars->s_full[n & 1], (n >> 1) & 1, failed);
        uint32_t sr[16];
        if (ok) {
          tc_fence_after();
          tmem_ld16(tl + (n & 1) * NH, sr);
          tmem_ld_wait(sr);
        }
        const int tok = ti * TOK + row;
        const bool valid = tok < U.ctx;
        float yh[NH], yl[NH];
#pragma unroll
        for (int g = 0; g < NH; ++g) {
          float y4 = 0.f;
          if (g < a.GT) {
            const float av = fmaf(__uint_as_float(sr[g]), a.scale2, -1.0f);
            const float uu = fmaf(av, av, 4.0f);
            const float t = fmaf(uu, rsqrt_approx(uu), av);  // 2 * squareplus(a)
            y4 = valid ? t * t : 0.f;                         // 4 * y
          }
          ysum[g] += y4;
          const __nv_bfloat16 hb = __float2bfloat16_rn(y4);
          yh[g] = __bfloat162float(hb);
          yl[g] = y4 - yh[g];
        }
        if (n >= 2) wait_uni(&bars->p_free[n & 1], ((n - 2) >> 1) & 1, failed);
        // P (K-major B of the P.V MMA): rows g (hi) and 16 + g (lo), token column `row`
        uint8_t* pb = smem + OFF_P + (n & 1) * 8192 + (row >> 6) * 4096;
        const int tt = row & 63;
#pragma unroll
        for (int g = 0; g < NH; ++g) {
          if (g < a.GT) {
            const int rh = g, rl = NH + g;
            *reinterpret_cast<__nv_bfloat16*>(pb + rh * 128 + (((tt >> 3) ^ (rh & 7)) << 4) + (tt & 7) * 2) =
                __float2bfloat16_rn(yh[g]);
            *reinterpret_cast<__nv_bfloat16*>(pb + rl * 128 + (((tt >> 3) ^ (rl & 7)) << 4) + (tt & 7) * 2) =
                __float2bfloat16_rn(yl[g]);
          }
        }
        if ((ti + 1) * TOK > U.ctx) {  // last tile: V rows past the context become zeros
          const int s = n % NS;
          if (wait_uni(&bars->v_full[s], (n / NS) & 1, failed) && !valid) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              uint4* vr = reinterpret_cast<uint4*>(smem + OFF_V + s * KT + c * HALF + row * 128);
#pragma unroll
              for (int i = 0; i < 8; ++i) vr[i] = make_uint4(0u, 0u, 0u, 0u);
            }
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars->p_full[n & 1]);
      }
      if (busy) {
        if (wait_uni(&bars->o_full, seg & 1, failed)) {
          tc_fence_after();
          uint32_t orr[32];
          tmem_ld32(tl + 32, orr);
          tmem_ld_wait(orr);
#pragma unroll
          for (int g = 0; g < NH; ++g) o[g] = __uint_as_float(orr[g]) + __uint_as_float(orr[NH + g]);
        }
        tc_fence_before();
        ++seg;
      }
      const int id_next = take_ew(k + 1);
      if (id_next >= 0) {
        const Unit Un = item_of(a, id_next, x0, x1);
        if (Un.t_hi > Un.t_lo) write_q(Un);
      }
      // sum of 4y per head over the 128 token rows of every tile
#pragma unroll
      for (int g = 0; g < NH; ++g) {
        if (g < a.GT) {
#pragma unroll
          for (int m = 16; m > 0; m >>= 1) ysum[g] += __shfl_xor_sync(0xffffffffu, ysum[g], m);
        }
      }
      ew_sync();  // red[] of the previous item fully read
      if (lane == 0) {
#pragma unroll
        for (int g = 0; g < NH; ++g)
          if (g < a.GT) red[(warp - 2) * NH + g] = ysum[g];
      }
      ew_sync();
      float tot[NH];
#pragma unroll
      for (int g = 0; g < NH; ++g) tot[g] = red[g] + red[NH + g] + red[2 * NH + g] + red[3 * NH + g];
      const int d = row;  // head-dim row of O^T held by this thread
      if (U.whole) {
#pragma unroll
        for (int g = 0; g < NH; ++g)
          if (g < a.GT)
            a.out[((int64_t)U.b * a.Hq + U.hq0 + g) * D + d] = __float2bfloat16_rn(o[g] / (tot[g] + eps4));
        id = id_next;
        continue;
      }
      const int REC = a.GT * D + NH;  // o[GT][D], then up to 16 head sums
      float* base = a.part + (int64_t)U.u * a.slots * REC;
      float* rec = base + (int64_t)U.slot * REC;
#pragma unroll
      for (int g = 0; g < NH; ++g)
        if (g < a.GT) __stcg(rec + g * D + d, o[g]);
      if (e < a.GT) __stcg(rec + a.GT * D + e, red[e] + red[NH + e] + red[2 * NH + e] + red[3 * NH + e]);
      __threadfence();
      ew_sync();
      if (e == 0) bars->last = atomicAdd(a.tickets + U.u, 1) == U.nslots - 1;
      ew_sync();
      if (!bars->last) {
        id = id_next;
        continue;
      }
      __threadfence();
      const int nsl = U.nslots;
      // Thread e owns float4 groups f = e, e + 128, ... of the GT x D block and
      // adds, slot by slot in index order (deterministic), both its O values
      // and its head's sum: one pass, up to 16 slots of independent loads in
      // flight, no barrier.
      const int nf = a.GT * D / 4;
      for (int f = e; f < nf; f += 128) {
        const int g = (4 * f) / D;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        float sy = 0.f;
        int sl = 0;
        for (; sl + 16 <= nsl; sl += 16) {
          float4 v[16];
          float w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v[j] = __ldcg(reinterpret_cast<const float4*>(base + (int64_t)(sl + j) * REC) + f);
            w[j] = __ldcg(base + (int64_t)(sl + j) * REC + a.GT * D + g);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            acc.x += v[j].x, acc.y += v[j].y, acc.z += v[j].z, acc.w += v[j].w;
            sy += w[j];
          }
        }
        for (; sl < nsl; ++sl) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(base + (int64_t)sl * REC) + f);
          sy += __ldcg(base + (int64_t)sl * REC + a.GT * D + g);
          acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
        }
        const float inv = 1.0f / (sy + eps4);
        uint2 wo;
        wo.x = pack2_bf16(acc.x * inv, acc.y * inv);
        wo.y = pack2_bf16(acc.z * inv, acc.w * inv);
        *reinterpret_cast<uint2*>(a.out + ((int64_t)U.b * a.Hq + U.hq0) * D + 4 * f) = wo;
      }
      if (e == 0) a.tickets[U.u] = 0;  // ready for the next call
      id = id_next;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

}  // namespace ptc

// ---- host side ---------------------------------------------------------------

int paged_tc_timeouts(int reset, cudaStream_t st) {
  unsigned t = 0;
  cudaMemcpyFromSymbolAsync(&t, ptc::g_ptc_timeouts, sizeof(t), 0, cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  if (reset) {
    const unsigned z = 0;
    cudaMemcpyToSymbolAsync(ptc::g_ptc_timeouts, &z, sizeof(z), 0, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
  }
  return (int)t;
}

int paged_tc_bad_pages(int reset, cudaStream_t st) {
  unsigned t = 0;
  cudaMemcpyFromSymbolAsync(&t, ptc::g_ptc_bad_pages, sizeof(t), 0, cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  if (reset) {
    const unsigned z = 0;
    cudaMemcpyToSymbolAsync(ptc::g_ptc_bad_pages, &z, sizeof(z), 0, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
  }
  return (int)t;
}

// Tensor-core plan: eligible shapes, schedule, slots and workspace bytes.
bool paged_tc_plan(int64_t B, int64_t Hq, int64_t Hkv, int64_t max_blocks, int64_t bs, int64_t D, int dtype,
                   int sms, PtcPlan* p) {
  if (dtype != SA_BF16 || D != ptc::D || Hq % Hkv != 0) return false;
  const int64_t G = Hq / Hkv;
  if (G < 2) return false;  // one head per KV row: the CUDA-core kernel is already HBM-bound
  if (bs % 8 != 0 || ptc::TOK % bs != 0) return false;
  int gt = (int)std::min<int64_t>(G, ptc::NH);
  while (G % gt != 0) --gt;
  if (gt < 2) return false;  // e.g. a prime group above 16: one head per MMA column is the CUDA-core case
  const int64_t units = B * Hkv * (G / gt);
  const int64_t M = (max_blocks * bs + ptc::TOK - 1) / ptc::TOK;
  if (units > INT32_MAX / 2 || M > INT32_MAX / 2) return false;
  const int64_t W = units * M;
  p->GT = gt;
  p->grid = std::max<int64_t>(1, std::min<int64_t>(sms, W));
  const int64_t share = std::max<int64_t>(1, W / p->grid);  // fewest tiles a non-empty CTA holds
  p->slots = (int)std::min<int64_t>(p->grid, (M + share - 1) / share + 2);
  p->ticket_bytes = (units * 4 + 255) / 256 * 256;
  p->part_bytes = units * (int64_t)p->slots * (gt * ptc::D + ptc::NH) * 4;
  return true;
}

int paged_tc_launch(const void* q, const void* k_cache, const void* v_cache, void* out, const int32_t* bt,
                    const int32_t* cl, void* workspace, int64_t B, int64_t Hq, int64_t Hkv, int64_t num_blocks,
                    int64_t bs, int64_t max_blocks, float scale, const PtcPlan& pl, cudaStream_t st) {
  using namespace ptc;
  CUtensorMap mk, mv;
  const int64_t strides[4] = {Hkv * bs * D, bs * D, D, 1};
  if (!sqattn::make_map_4d(&mk, k_cache, true, num_blocks, Hkv, bs, D, strides, 64, (int)bs) ||
      !sqattn::make_map_4d(&mv, v_cache, true, num_blocks, Hkv, bs, D, strides, 64, (int)bs))
    return SA_ERR_ALIGN;
  Args a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.bt = bt;
  a.cl = cl;
  const int64_t units = B * Hkv * (Hq / Hkv / pl.GT);
  a.tickets = static_cast<int32_t*>(workspace);
  a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + pl.ticket_bytes);
  a.num_blocks = num_blocks;
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.G = (int)(Hq / Hkv);
  a.GT = pl.GT;
  a.nhc = a.G / pl.GT;
  a.bs = (int)bs;
  a.max_blocks = (int)max_blocks;
  a.M = (int)((max_blocks * bs + TOK - 1) / TOK);
  a.W = units * (int64_t)a.M;
  a.slots = pl.slots;
  a.scale2 = 2.0f * scale;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(paged_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return sa_record_cuda_error(e);
    if (dev >= 0 && dev < 64) attr_done[dev] = true;
  }
  paged_tc_kernel<<<(unsigned)pl.grid, THREADS, SMEM, st>>>(mk, mv, a);
  return sa_record_cuda_error(cudaGetLastError());
}

}  // namespace sa
SA_BOUNDS_ACCESSOR(paged_tc_bounds)
