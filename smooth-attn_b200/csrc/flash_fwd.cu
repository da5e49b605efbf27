// Fused causal squareplus attention, forward, on tcgen05 tensor cores.
//
// Reference algorithm: src/smooth_attn/kernels.py:1549-1631
// (_sp2norm_flash_fwd_with_rowsum_kernel) and the host wrapper :1912-1931.
//   s = (q . k) * scale;  a = 2 s - 1;  y = 0.25 (a + sqrt(a^2 + 4))^2 on the
//   visible (causal, optionally windowed) prefix;  R = 1e-12 + sum y;
//   o = (sum bf16(y) v) / R;  R is saved for the backward.
//
// B200 design.  One CTA owns one 128-row query tile of one (batch, head) and
// runs a warp-specialised pipeline:
//   warp 0      TMA producer: Q once, then K/V tiles (128 x D) into an
//               NS-stage shared-memory ring (128 B / 64 B swizzled boxes);
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer:
//               S_b = Q K^T into one of two 128-column TMEM score buffers,
//               O += P V with P read straight from TMEM (the "TS" form);
//   warps 2..5  squareplus warps: one query row per thread; tcgen05.ld the
//               score row, y = t*t with t = a + u*rsqrt(u) (MUFU), masked
//               only on tiles that cross the diagonal / window / sequence
//               end, fp32 row sum, bf16 P written back over S (tcgen05.st);
//               epilogue O / R -> global, R -> rowsum.
// Because the normalizer is a plain sum (no running max), O accumulates in
// TMEM across all KV tiles with no rescaling: there is no correction stage.
// The constant 0.25 is folded out (y' = 4y): it cancels exactly in
// sum(y'V)/sum(y') and R = R'/4 is exact, so only EPS moves (4e-12 for R').
// Every mbarrier wait is bounded (2 s); a timeout is recorded in
// g_flash_timeouts and the CTA leaves through the normal teardown.
#include <cudaTypedefs.h>

#include <mutex>

#include "sa_sm100.cuh"

namespace sa {
namespace flash {

using namespace sm100;

__device__ unsigned g_flash_timeouts;

template <int D>
struct FwdCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int CHUNK = D >= 64 ? 64 : D;  // elements per swizzled smem row
  static constexpr int NCHUNK = D / CHUNK;
  static constexpr int ROWB = CHUNK * 2;  // bytes per smem row
  static constexpr uint32_t SWZ = ROWB == 128 ? SW_128B : SW_64B;
  static constexpr int SBO = 8 * ROWB;  // stride between 8-row groups
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int NS = D == 128 ? 2 : (D == 64 ? 3 : 4);
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NS * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + NS * KV_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;  // + barriers + alignment slack
  static constexpr int TMEM_COLS = 512;            // S0 @0, S1 @128, O @256
  static constexpr int THREADS = 192;
};

struct FwdParams {
  void* o;
  float* rowsum;
  int64_t so_b, so_h, so_s;
  int B, Hq, Hkv, T, nqt, window;
  float scale2;  // 2 * scale
};

struct Bars {
  uint64_t q_full;
  uint64_t o_full;
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t k_full[4];
  uint64_t v_full[4];
  uint64_t kv_empty[4];
  uint32_t tmem_base;
};

__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t phase, bool& failed) {
  if (failed) return false;
  if (!mbar_wait(bar, phase)) {
    failed = true;
    atomicAdd(&g_flash_timeouts, 1u);
    return false;
  }
  return true;
}

// Warp-uniform variant for warps that then run .sync.aligned tcgen05 ops.
__device__ __forceinline__ bool warp_wait_or_flag(uint64_t* bar, uint32_t phase, bool& failed) {
  const bool ok = __all_sync(0xffffffffu, !failed && mbar_wait(bar, phase));
  if (!ok) {
    if (!failed && (threadIdx.x & 31) == 0) atomicAdd(&g_flash_timeouts, 1u);
    failed = true;
  }
  return ok;
}

template <int D, bool BF16, bool EXACT>
__global__ void __launch_bounds__(192, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                     const __grid_constant__ CUtensorMap tmv, FwdParams p) {
  using C = FwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  Bars* bars = reinterpret_cast<Bars*>(smem + C::OFF_BAR);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.nqt - 1 - (int)blockIdx.x;  // longest (most KV tiles) first
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int kvh = h / (p.Hq / p.Hkv);
  const int q0 = qt * C::BM;
  const int nkv_total = (p.T + C::BN - 1) / C::BN;
  int j1 = (q0 + C::BM + C::BN - 1) / C::BN;
  if (j1 > nkv_total) j1 = nkv_total;
  int j0 = 0;
  if (p.window > 0) {
    const int first = q0 - p.window + 1;
    j0 = first > 0 ? first / C::BN : 0;
  }
  const int n = j1 - j0;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->o_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_free[i], 1);
      mbar_init(&bars->p_full[i], 128);
    }
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->kv_empty[i], 1);
    }
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
      mbar_arrive_expect_tx(&bars->q_full, C::Q_BYTES);
      for (int c = 0; c < C::NCHUNK; ++c)
        tma_load_4d(sQ + c * C::BM * C::ROWB, &tmq, c * C::CHUNK, q0, h, b, &bars->q_full);
      for (int i = 0; i < n; ++i) {
        const int st = i % C::NS;
        if (i >= C::NS && !wait_or_flag(&bars->kv_empty[st], ((i / C::NS) - 1) & 1, failed)) break;
        const int kv0 = (j0 + i) * C::BN;
        uint8_t* k_dst = sK + st * C::KV_BYTES;
        uint8_t* v_dst = sV + st * C::KV_BYTES;
        mbar_arrive_expect_tx(&bars->k_full[st], C::KV_BYTES);
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_load_4d(k_dst + c * C::BN * C::ROWB, &tmk, c * C::CHUNK, kv0, kvh, b, &bars->k_full[st]);
        mbar_arrive_expect_tx(&bars->v_full[st], C::KV_BYTES);
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_load_4d(v_dst + c * C::BN * C::ROWB, &tmv, c * C::CHUNK, kv0, kvh, b, &bars->v_full[st]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_s = idesc_f16(128, C::BN, BF16 ? 1 : 0, 0, 0);
      constexpr uint32_t idesc_o = idesc_f16(128, D, BF16 ? 1 : 0, 0, 1);
      const uint32_t tS = tbase, tO = tbase + 256;
      const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV);
      if (wait_or_flag(&bars->q_full, 0, failed)) {
        for (int i = 0; i <= n && !failed; ++i) {
          if (i < n) {
            const int st = i % C::NS, bb = i & 1;
            if (!wait_or_flag(&bars->k_full[st], (i / C::NS) & 1, failed)) break;
            if (i >= 2 && !wait_or_flag(&bars->s_free[bb], ((i / 2) - 1) & 1, failed)) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int c = (kk * 16) / C::CHUNK;
              const uint32_t off = ((kk * 16) % C::CHUNK) * 2;
              const uint64_t da = smem_desc(aQ + c * C::BM * C::ROWB + off, 16, C::SBO, C::SWZ);
              const uint64_t db = smem_desc(aK + st * C::KV_BYTES + c * C::BN * C::ROWB + off, 16, C::SBO, C::SWZ);
              mma_ss(tS + bb * 128, da, db, idesc_s, kk > 0);
            }
            mma_commit(&bars->s_full[bb]);
          }
          if (i >= 1) {
            const int ip = i - 1, stp = ip % C::NS, bp = ip & 1;
            if (!wait_or_flag(&bars->p_full[bp], (ip / 2) & 1, failed)) break;
            if (!wait_or_flag(&bars->v_full[stp], (ip / C::NS) & 1, failed)) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < C::BN / 16; ++kk) {
              const uint64_t db = smem_desc(aV + stp * C::KV_BYTES + kk * 16 * C::ROWB, C::BN * C::ROWB, C::SBO, C::SWZ);
              mma_ts(tO, tS + bp * 128 + kk * 8, db, idesc_o, (ip > 0 || kk > 0) ? 1u : 0u);
            }
            mma_commit(&bars->kv_empty[stp]);
            mma_commit(&bars->s_free[bp]);
          }
        }
        mma_commit(&bars->o_full);
      }
    }
  } else {
    // ------------------------------------------------------------ squareplus warps
    const int g = warp & 3;
    const int row = 32 * g + lane;
    const int q = q0 + row;
    const uint32_t tl = tbase + ((uint32_t)(32 * g) << 16);
    float rsum = 4e-12f;  // 4 * EPS (y is carried as 4y)
    for (int i = 0; i < n; ++i) {
      const int bb = i & 1;
      const int k0 = (j0 + i) * C::BN;
      if (!warp_wait_or_flag(&bars->s_full[bb], (i / 2) & 1, failed)) break;
      tc_fence_after();
      const bool need_mask = (k0 + C::BN - 1 > q0) || (k0 + C::BN > p.T) ||
                             (p.window > 0 && q0 + C::BM - 1 - k0 >= p.window);
#pragma unroll
      for (int c = 0; c < C::BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tl + bb * 128 + c * 32, r);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float yv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float a = fmaf(__uint_as_float(r[e + u]), p.scale2, -1.0f);
            const float w = fmaf(a, a, 4.0f);
            const float t = EXACT ? a + sqrtf(w) : fmaf(w, rsqrtf(w), a);
            float y = t * t;
            if (need_mask) {
              const int k = k0 + c * 32 + e + u;
              const bool ok = (k <= q) && (k < p.T) && (p.window <= 0 || q - k < p.window);
              y = ok ? y : 0.f;
            }
            yv[u] = y;
          }
          rsum += yv[0] + yv[1];
          pk[e / 2] = BF16 ? pack2_bf16(yv[0], yv[1]) : pack2_f16(yv[0], yv[1]);
        }
        tmem_st16(tl + bb * 128 + c * 16, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->p_full[bb]);
    }
    if (warp_wait_or_flag(&bars->o_full, 0, failed)) {
      tc_fence_after();
      const float inv = 1.0f / rsum;
      const bool live = q < p.T;
      uint8_t* orow = static_cast<uint8_t*>(p.o) + 2 * ((int64_t)b * p.so_b + (int64_t)h * p.so_h + (int64_t)q * p.so_s);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tl + 256 + c * 32, r);  // all lanes: .sync.aligned
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float lo = __uint_as_float(r[e]) * inv, hi = __uint_as_float(r[e + 1]) * inv;
          pk[e / 2] = BF16 ? pack2_bf16(lo, hi) : pack2_f16(lo, hi);
        }
        if (live) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
      if (live) p.rowsum[((int64_t)b * p.Hq + h) * p.T + q] = 0.25f * rsum;
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
// host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 4-D map over a [B, H, T, D] tensor (element strides), box {chunk, rows, 1, 1}.
bool make_map_4d(CUtensorMap* map, const void* base, bool bf16, int64_t B, int64_t H, int64_t T, int64_t D,
                 const int64_t* strides, int chunk, int rows) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t gstr[3] = {(cuuint64_t)strides[2] * 2, (cuuint64_t)strides[1] * 2, (cuuint64_t)strides[0] * 2};
  cuuint32_t box[4] = {(cuuint32_t)chunk, (cuuint32_t)rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle swz = chunk * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : chunk * 2 == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                   : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(base), dims, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int D, bool BF16, bool EXACT>
static int launch_fwd(const void* q, const void* k, const void* v, void* o, float* rowsum, int64_t B, int64_t Hq,
                      int64_t Hkv, int64_t T, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                      const int64_t* os, float scale, int64_t window, cudaStream_t st) {
  using C = FwdCfg<D>;
  CUtensorMap mq, mk, mv;
  if (!make_map_4d(&mq, q, BF16, B, Hq, T, D, qs, C::CHUNK, C::BM) ||
      !make_map_4d(&mk, k, BF16, B, Hkv, T, D, ks, C::CHUNK, C::BN) ||
      !make_map_4d(&mv, v, BF16, B, Hkv, T, D, vs, C::CHUNK, C::BN))
    return SA_ERR_ALIGN;
  FwdParams p;
  p.o = o;
  p.rowsum = rowsum;
  p.so_b = os[0];
  p.so_h = os[1];
  p.so_s = os[2];
  p.B = (int)B;
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.T = (int)T;
  p.nqt = (int)((T + C::BM - 1) / C::BM);
  p.window = (int)window;
  p.scale2 = 2.0f * scale;
  auto kern = flash_fwd_kernel<D, BF16, EXACT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  dim3 grid(p.nqt, (unsigned)(B * Hq));
  kern<<<grid, C::THREADS, C::SMEM, st>>>(mq, mk, mv, p);
  return SA_OK;
}

}  // namespace flash

int flash_timeouts(int reset) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, flash::g_flash_timeouts, sizeof(v));
  if (reset) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(flash::g_flash_timeouts, &z, sizeof(z));
  }
  return (int)v;
}

}  // namespace sa

int sa_record_cuda_error(cudaError_t e);

static bool strides_ok(const int64_t* s) {
  return s != nullptr && s[3] == 1 && s[0] % 8 == 0 && s[1] % 8 == 0 && s[2] % 8 == 0 && s[0] >= 0 && s[1] >= 0 &&
         s[2] > 0;
}

static bool ptr16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int sa_flash_fwd(const void* q, const void* k, const void* v, void* o, float* rowsum, int64_t B,
                            int64_t Hq, int64_t Hkv, int64_t T, int64_t D, const int64_t* q_strides,
                            const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                            float scale, int64_t window_size, int exact_math, int dtype, void* stream) {
  if (dtype != SA_BF16 && dtype != SA_F16) return SA_ERR_UNSUPPORTED;
  if (D != 32 && D != 64 && D != 128) return SA_ERR_UNSUPPORTED;
  if (B < 0 || Hq < 1 || Hkv < 1 || T < 0 || Hq % Hkv != 0 || window_size < 0) return SA_ERR_ARG;
  if (B == 0 || T == 0) return SA_OK;
  if (T > (1ll << 30) || B * Hq > 65535ll * 32768) return SA_ERR_UNSUPPORTED;
  if (!q || !k || !v || !o || !rowsum) return SA_ERR_ARG;
  if (!strides_ok(q_strides) || !strides_ok(k_strides) || !strides_ok(v_strides) || !strides_ok(o_strides))
    return SA_ERR_ALIGN;
  if (!ptr16(q) || !ptr16(k) || !ptr16(v) || !ptr16(o)) return SA_ERR_ALIGN;
  if (B * Hq > 65535) return SA_ERR_UNSUPPORTED;  // grid.y limit
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  using namespace sa::flash;
  int rc;
#define SA_FWD_CASE(DD, BF, EX) \
  rc = launch_fwd<DD, BF, EX>(q, k, v, o, rowsum, B, Hq, Hkv, T, q_strides, k_strides, v_strides, o_strides, scale, window_size, st)
#define SA_FWD_D(DD)                                    \
  if (dtype == SA_BF16) {                               \
    if (exact_math) SA_FWD_CASE(DD, true, true);        \
    else SA_FWD_CASE(DD, true, false);                  \
  } else {                                              \
    if (exact_math) SA_FWD_CASE(DD, false, true);       \
    else SA_FWD_CASE(DD, false, false);                 \
  }
  if (D == 32) {
    SA_FWD_D(32)
  } else if (D == 64) {
    SA_FWD_D(64)
  } else {
    SA_FWD_D(128)
  }
#undef SA_FWD_D
#undef SA_FWD_CASE
  if (rc != SA_OK) return rc;
  return sa_record_cuda_error(cudaGetLastError());
}
