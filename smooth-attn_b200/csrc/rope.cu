// Rotary position embedding (rotate-half form) for the fused RoPE attention
// forward, sm_100a.
//
// Reference: _sp2norm_rope_flash_fwd_kernel / sp2norm_rope_flash_attention
// (src/smooth_attn/kernels.py:2104-2222, :2373-2430), RoPE applied to the
// loaded Q / K tiles in fp32 and rounded to 16 bits before the QK^T dot:
//   x1 = x[..., :D/2], x2 = x[..., D/2:],  c = cos[t], s = sin[t]
//   rot = [x1 c - x2 s,  x2 c + x1 s]
// (the reference tests' apply_rope_eager, tests/test_rope_proj.py:15-30,
// states the same map as x * [c, c] + [-x2, x1] * [s, s]).
//
// Design.  K is read by every query tile of a head, so rotating it inside
// the attention kernel would repeat the rotation T/128 times per head and
// put elementwise work on the warps that bound the forward.  Instead one
// memory-bound pass rotates Q and K together (16-byte loads of both halves,
// cos/sin rows from L2) into a workspace, and the tcgen05 forward reads the
// rotated tiles by TMA.  Each product and the sum are rounded separately
// (no FMA contraction), as the reference's eager formula does, then rounded
// to the input's 16-bit type.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "sa_common.cuh"
#include "smooth_attn_b200.h"

int sa_record_cuda_error(cudaError_t e);

namespace sa {

struct RopeTensor {
  const void* x;
  void* out;  // contiguous [B, H, T, D]
  int64_t H;
  int64_t sb, sh, st;  // element strides of x (dim stride 1)
};

template <typename CS>
__device__ __forceinline__ void load8f(const CS* p, float (&f)[8]) {
  if constexpr (sizeof(CS) == 4) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
  } else {
    unpack<CS, 8>(p, f);
  }
}

// One thread: one row, one group of 8 pairs (x[i], x[i + D/2]).
template <typename E, typename CS>
__global__ void __launch_bounds__(256) rope_rotate_kernel(RopeTensor a, RopeTensor b, const CS* __restrict__ cosv,
                                                          const CS* __restrict__ sinv, int64_t B, int64_t T,
                                                          int D) {
  const int G = D / 16;  // 8-pair groups per row
  const int64_t na = B * a.H * T * G;
  const int64_t n = na + B * b.H * T * G;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const bool first = i < na;
    const RopeTensor& r = first ? a : b;
    const int64_t j = first ? i : i - na;
    const int g = (int)(j % G);
    const int64_t row = j / G;  // (bb * H + h) * T + t
    const int64_t t = row % T;
    const int64_t bh = row / T;
    const int64_t h = bh % r.H, bb = bh / r.H;
    if (!SA_DCHECK(bb < B && g * 8 + 8 <= D / 2)) continue;
    const E* xr = static_cast<const E*>(r.x) + bb * r.sb + h * r.sh + t * r.st;
    E* orow = static_cast<E*>(r.out) + row * D;
    float x1[8], x2[8], c[8], s[8];
    unpack<E, 8>(xr + g * 8, x1);
    unpack<E, 8>(xr + D / 2 + g * 8, x2);
    load8f<CS>(cosv + t * (D / 2) + g * 8, c);
    load8f<CS>(sinv + t * (D / 2) + g * 8, s);
    Pack<E, 8> o1, o2;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o1.set(e, __fsub_rn(__fmul_rn(x1[e], c[e]), __fmul_rn(x2[e], s[e])));
      o2.set(e, __fadd_rn(__fmul_rn(x2[e], c[e]), __fmul_rn(x1[e], s[e])));
    }
    *reinterpret_cast<uint4*>(orow + g * 8) = o1.u;
    *reinterpret_cast<uint4*>(orow + D / 2 + g * 8) = o2.u;
  }
}

template <typename E>
int launch_rope(const RopeTensor& a, const RopeTensor& b, const void* cosv, const void* sinv, int cs_dtype,
                int64_t B, int64_t T, int D, cudaStream_t st) {
  const int64_t n = (a.H + b.H) * B * T * (D / 16);
  if (n == 0) return SA_OK;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8);
  switch (cs_dtype) {
    case SA_F32:
      rope_rotate_kernel<E, float><<<(unsigned)blocks, 256, 0, st>>>(
          a, b, static_cast<const float*>(cosv), static_cast<const float*>(sinv), B, T, D);
      break;
    case SA_BF16:
      rope_rotate_kernel<E, __nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(
          a, b, static_cast<const __nv_bfloat16*>(cosv), static_cast<const __nv_bfloat16*>(sinv), B, T, D);
      break;
    default:
      rope_rotate_kernel<E, __half><<<(unsigned)blocks, 256, 0, st>>>(
          a, b, static_cast<const __half*>(cosv), static_cast<const __half*>(sinv), B, T, D);
      break;
  }
  return sa_record_cuda_error(cudaGetLastError());
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_rope_args(const void* x, const int64_t* s, const void* cosv, const void* sinv, int cs_dtype, int64_t T,
                    int64_t D, int dtype) {
  if (!x || !s || !cosv || !sinv) return SA_ERR_ARG;
  if (dtype != SA_BF16 && dtype != SA_F16) return SA_ERR_UNSUPPORTED;
  if (cs_dtype != SA_F32 && cs_dtype != SA_BF16 && cs_dtype != SA_F16) return SA_ERR_UNSUPPORTED;
  if (D <= 0 || D % 16 != 0 || T <= 0) return SA_ERR_UNSUPPORTED;
  if (s[3] != 1) return SA_ERR_ALIGN;
  for (int i = 0; i < 3; ++i)
    if (s[i] % 8 != 0) return SA_ERR_ALIGN;
  const int cs_size = cs_dtype == SA_F32 ? 4 : 2;
  if (!al16(x) || !al16(cosv) || !al16(sinv) || ((D / 2) * cs_size) % 16 != 0) return SA_ERR_ALIGN;
  return SA_OK;
}

}  // namespace sa

extern "C" int sa_rope_rotate(const void* x, void* out, const void* cos_table, const void* sin_table, int cs_dtype,
                              int64_t B, int64_t H, int64_t T, int64_t D, const int64_t* x_strides, int dtype,
                              void* stream) {
  if (B < 0 || H < 0) return SA_ERR_ARG;
  int rc = sa::check_rope_args(x, x_strides, cos_table, sin_table, cs_dtype, T, D, dtype);
  if (rc != SA_OK) return rc;
  if (!out) return SA_ERR_ARG;
  if (!sa::al16(out)) return SA_ERR_ALIGN;
  sa::RopeTensor a{x, out, H, x_strides[0], x_strides[1], x_strides[2]};
  sa::RopeTensor none{x, out, 0, 0, 0, 0};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == SA_BF16 ? sa::launch_rope<__nv_bfloat16>(a, none, cos_table, sin_table, cs_dtype, B, T, (int)D, st)
                          : sa::launch_rope<__half>(a, none, cos_table, sin_table, cs_dtype, B, T, (int)D, st);
}

extern "C" int64_t sa_rope_flash_fwd_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D) {
  if (B < 0 || Hq < 0 || Hkv < 0 || T < 0 || D < 0) return SA_ERR_ARG;
  const int64_t q = (B * Hq * T * D * 2 + 255) / 256 * 256;
  return q + B * Hkv * T * D * 2;
}

extern "C" int sa_rope_flash_fwd(const void* q, const void* k, const void* v, void* o, float* rowsum,
                                 const void* cos_table, const void* sin_table, int cs_dtype, void* workspace,
                                 int64_t workspace_bytes, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D,
                                 const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                 const int64_t* o_strides, float scale, int64_t window_size, int exact_math,
                                 int dtype, void* stream) {
  if (B < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0) return SA_ERR_ARG;
  int rc = sa::check_rope_args(q, q_strides, cos_table, sin_table, cs_dtype, T, D, dtype);
  if (rc != SA_OK) return rc;
  rc = sa::check_rope_args(k, k_strides, cos_table, sin_table, cs_dtype, T, D, dtype);
  if (rc != SA_OK) return rc;
  if (D != 32 && D != 64 && D != 128) return SA_ERR_UNSUPPORTED;  // the attention kernel's head dims
  const int64_t need = sa_rope_flash_fwd_workspace_size(B, Hq, Hkv, T, D);
  if (!workspace || workspace_bytes < need) return SA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return SA_ERR_ALIGN;
  uint8_t* qr = static_cast<uint8_t*>(workspace);
  uint8_t* kr = qr + (B * Hq * T * D * 2 + 255) / 256 * 256;
  sa::RopeTensor a{q, qr, Hq, q_strides[0], q_strides[1], q_strides[2]};
  sa::RopeTensor b{k, kr, Hkv, k_strides[0], k_strides[1], k_strides[2]};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = dtype == SA_BF16 ? sa::launch_rope<__nv_bfloat16>(a, b, cos_table, sin_table, cs_dtype, B, T, (int)D, st)
                        : sa::launch_rope<__half>(a, b, cos_table, sin_table, cs_dtype, B, T, (int)D, st);
  if (rc != SA_OK) return rc;
  const int64_t qs[4] = {Hq * T * D, T * D, D, 1};
  const int64_t ks[4] = {Hkv * T * D, T * D, D, 1};
  return sa_flash_fwd(qr, kr, v, o, nullptr, rowsum, B, Hq, Hkv, T, D, qs, ks, v_strides, o_strides, scale, window_size,
                      exact_math, dtype, stream);
}
SA_BOUNDS_ACCESSOR(rope_bounds)
