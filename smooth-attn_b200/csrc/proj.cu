// Output projection of the RoPE attention: out[M, N] = A[M, K] W[K, N] on
// tcgen05 tensor cores, bf16 / fp16 operands, fp32 accumulation, 16-bit output.
//
// Reference: the W_o stage of _sp2norm_rope_flash_proj_fwd_kernel
// (src/smooth_attn/kernels.py:2233-2370), which multiplies each head's
// [BLOCK_Q, D] attention output by W_o[h] ([D, D_model]) and adds the per-head
// bf16 partials into `out` with atomic_add.  Here the attention writes its
// output as [B, T, H, D], so A = [B*T, H*D] and the sum over heads is the
// contraction of one GEMM, accumulated in fp32 inside the tensor core and
// rounded once (no arrival-order-dependent bf16 partial sums).
//
// B200 design: persistent CTAs (one per SM) walk the 128 x 256 output tiles.
//   warp 0      TMA producer: A tiles [128 rows x 64 K] (128 B swizzle,
//               K-major) and W tiles [64 K x 256 N] as four 64-column chunks
//               (128 B swizzle, N-major) into a 4-stage ring;
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//               (M = 128, N = 256, K = 16 per instruction) into one of two
//               256-column fp32 accumulators;
//   warps 2..5  epilogue: TMEM -> registers -> 16-bit -> global, one output
//               row per thread, while the MMA warp already accumulates the
//               next tile into the other accumulator.
// Every mbarrier wait is bounded (2 s); a timeout is counted and the CTA
// leaves through the normal teardown.
#include <cudaTypedefs.h>

#include "sa_sm100.cuh"

namespace sa {
namespace proj {

using namespace sm100;

__device__ unsigned g_proj_timeouts;

constexpr int BM = 128, BN = 256, BK = 64, NST = 4;
constexpr int A_TILE = BM * BK * 2;      // 16 KB
constexpr int W_CHUNK = BK * 64 * 2;     // one 64-column chunk of a W tile: 8 KB
constexpr int W_TILE = 4 * W_CHUNK;      // 32 KB
constexpr int STAGE = A_TILE + W_TILE;   // 48 KB
constexpr int OFF_BAR = NST * STAGE;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr int THREADS = 192;

struct Bars {
  uint64_t full[NST], empty[NST];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
};

struct ProjParams {
  void* out;
  int64_t ldo;
  int M, N, K;
  int tiles_m, tiles_n;
};

__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t phase, bool& failed) {
  if (failed) return false;
  if (!mbar_wait(bar, phase)) {
    failed = true;
    atomicAdd(&g_proj_timeouts, 1u);
    return false;
  }
  return true;
}

__device__ __forceinline__ bool warp_wait_or_flag(uint64_t* bar, uint32_t phase, bool& failed) {
  const bool ok = __all_sync(0xffffffffu, !failed && mbar_wait(bar, phase));
  if (!ok) {
    if (!failed && (threadIdx.x & 31) == 0) atomicAdd(&g_proj_timeouts, 1u);
    failed = true;
  }
  return ok;
}

template <bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    proj_gemm_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmw, ProjParams p) {
  // Declared 1024-byte aligned (the kernel has no static shared data, so
  // dynamic shared memory starts on such a boundary; the swizzled tiles need
  // it).  A misaligned start is counted as a timeout and every thread leaves.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicAdd(&g_proj_timeouts, 1u);
    return;
  }
  uint8_t* smem = smem_raw;
  Bars* bars = reinterpret_cast<Bars*>(smem + OFF_BAR);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = p.tiles_m * p.tiles_n;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->acc_full[i], 1);
      mbar_init(&bars->acc_empty[i], 128);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  bool failed = false;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&tma);
      tma_prefetch_desc(&tmw);
      int it = 0;  // ring position over all (tile, k-step) pairs of this CTA
      for (int t = blockIdx.x; t < ntiles && !failed; t += gridDim.x) {
        const int m0 = (t % p.tiles_m) * BM, n0 = (t / p.tiles_m) * BN;
        (void)SA_DCHECK(m0 < p.M && n0 < p.N);  // the tile starts inside the output
        for (int kb = 0; kb < nk && !failed; ++kb, ++it) {
          const int s = it % NST;
          if (it >= NST && !wait_or_flag(&bars->empty[s], ((it / NST) - 1) & 1, failed)) break;
          uint8_t* st = smem + s * STAGE;
          mbar_arrive_expect_tx(&bars->full[s], STAGE);
          tma_load_4d(st, &tma, kb * BK, m0, 0, 0, &bars->full[s]);
          for (int c = 0; c < 4; ++c)
            tma_load_4d(st + A_TILE + c * W_CHUNK, &tmw, n0 + c * 64, kb * BK, 0, 0, &bars->full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_f16(BM, BN, BF16 ? 1 : 0, 0, 1);  // A K-major, W N-major
      const uint32_t s0 = smem_u32(smem);
      int it = 0, local = 0;
      for (int t = blockIdx.x; t < ntiles && !failed; t += gridDim.x, ++local) {
        const int ab = local & 1;
        // the epilogue must have drained this accumulator (used two tiles ago)
        if (local >= 2 && !wait_or_flag(&bars->acc_empty[ab], ((local >> 1) - 1) & 1, failed)) break;
        tc_fence_after();
        const uint32_t acc = tbase + ab * BN;
        for (int kb = 0; kb < nk && !failed; ++kb, ++it) {
          const int s = it % NST;
          if (!wait_or_flag(&bars->full[s], (it / NST) & 1, failed)) break;
          tc_fence_after();
          const uint32_t a_s = s0 + s * STAGE, w_s = a_s + A_TILE;
          const uint64_t da = smem_desc(a_s, 16, 1024, SW_128B);
          const uint64_t dw = smem_desc(w_s, W_CHUNK, 1024, SW_128B);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_ss(acc, desc_add(da, kk * 32), desc_add(dw, kk * 16 * 128), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&bars->empty[s]);
        }
        mma_commit(&bars->acc_full[ab]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int g = warp & 3;  // TMEM lane quarter of this warp (warps 2..5 -> 2, 3, 0, 1)
    const int row = 32 * g + lane;
    const uint32_t tl = tbase + ((uint32_t)(32 * g) << 16);
    int local = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++local) {
      const int ab = local & 1;
      if (!warp_wait_or_flag(&bars->acc_full[ab], (local >> 1) & 1, failed)) break;
      tc_fence_after();
      const int m = (t % p.tiles_m) * BM + row, n0 = (t / p.tiles_m) * BN;
      uint8_t* orow = static_cast<uint8_t*>(p.out) + 2 * ((int64_t)m * p.ldo + n0);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tl + ab * BN + c * 32, r);  // all lanes: .sync.aligned
        tmem_ld_wait(r);
        if (m < p.M) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int col = n0 + c * 32 + v * 8;
            if (col < p.N) {  // N % 8 == 0: whole 8-column vectors
              uint32_t pk[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float lo = __uint_as_float(r[v * 8 + 2 * e]), hi = __uint_as_float(r[v * 8 + 2 * e + 1]);
                pk[e] = BF16 ? pack2_bf16(lo, hi) : pack2_f16(lo, hi);
              }
              *reinterpret_cast<uint4*>(orow + 2 * (c * 32 + v * 8)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->acc_empty[ab]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace proj

int proj_timeouts(int reset, cudaStream_t st) {
  unsigned v = 0;
  cudaMemcpyFromSymbolAsync(&v, proj::g_proj_timeouts, sizeof(v), 0, cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  if (reset) {
    const unsigned z = 0;
    cudaMemcpyToSymbolAsync(proj::g_proj_timeouts, &z, sizeof(z), 0, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
  }
  return (int)v;
}

namespace sqattn {
bool make_map_4d(CUtensorMap* map, const void* base, bool bf16, int64_t B, int64_t H, int64_t T, int64_t D,
                 const int64_t* strides, int chunk, int rows, bool u8);
}  // namespace sqattn

}  // namespace sa

int sa_record_cuda_error(cudaError_t e);

extern "C" int sa_out_proj(const void* a, const void* w, void* out, int64_t M, int64_t K, int64_t N, int64_t lda,
                           int64_t ldw, int64_t ldo, int dtype, void* stream) {
  using namespace sa::proj;
  if (dtype != SA_BF16 && dtype != SA_F16) return SA_ERR_UNSUPPORTED;
  if (M < 0 || K < 0 || N < 0) return SA_ERR_ARG;
  if (M == 0 || N == 0) return SA_OK;
  if (K == 0) return SA_ERR_ARG;  // an empty contraction has no defined 16-bit result here; callers zero-fill
  if (!a || !w || !out) return SA_ERR_ARG;
  if (M > INT32_MAX || K > INT32_MAX || N > INT32_MAX) return SA_ERR_UNSUPPORTED;
  // TMA: 16-byte aligned bases and row strides; the epilogue stores 8-column vectors
  if ((reinterpret_cast<uintptr_t>(a) & 15u) || (reinterpret_cast<uintptr_t>(w) & 15u) ||
      (reinterpret_cast<uintptr_t>(out) & 15u) || lda % 8 || ldw % 8 || ldo % 8 || N % 8 || lda < K || ldw < N ||
      ldo < N)
    return SA_ERR_ALIGN;
  const bool bf16 = dtype == SA_BF16;
  CUtensorMap ma, mw;
  const int64_t sa_[4] = {M * lda, M * lda, lda, 1};
  const int64_t sw_[4] = {K * ldw, K * ldw, ldw, 1};
  if (!sa::sqattn::make_map_4d(&ma, a, bf16, 1, 1, M, K, sa_, BK, BM, false) ||
      !sa::sqattn::make_map_4d(&mw, w, bf16, 1, 1, K, N, sw_, 64, BK, false))
    return SA_ERR_ALIGN;
  ProjParams p;
  p.out = out;
  p.ldo = ldo;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.tiles_m = (int)((M + BM - 1) / BM);
  p.tiles_n = (int)((N + BN - 1) / BN);
  const int64_t ntiles = (int64_t)p.tiles_m * p.tiles_n;
  if (ntiles > INT32_MAX) return SA_ERR_UNSUPPORTED;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = (unsigned)(ntiles < sms ? ntiles : sms);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bf16) {
    cudaFuncSetAttribute(proj_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    proj_gemm_kernel<true><<<grid, THREADS, SMEM, st>>>(ma, mw, p);
  } else {
    cudaFuncSetAttribute(proj_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    proj_gemm_kernel<false><<<grid, THREADS, SMEM, st>>>(ma, mw, p);
  }
  return sa_record_cuda_error(cudaGetLastError());
}
SA_BOUNDS_ACCESSOR(proj_bounds)
