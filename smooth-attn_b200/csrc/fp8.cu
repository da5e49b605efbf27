// Per-tensor FP8 (E4M3) quantization of Q, K and V for the FP8 attention
// forward, sm_100a.
//
// Reference: _quantize_to_fp8 (src/smooth_attn/kernels.py:2592-2601), called
// three times by sp2norm_fp8_flash_attention (:2630-2673):
//   amax = max |x|;  scale = max(amax / 448, 1e-12)   (fp32)
//   x8 = e4m3(clamp(x / scale, -448, 448))             (round to nearest even)
// followed by scale.item(), a device-to-host synchronisation per tensor.
//
// Design.  Two launches cover all three tensors and nothing leaves the
// device: a grid-stride absmax over q, k and v together (warp max, one
// atomicMax per warp on the float bits, which order like unsigned integers
// for non-negative floats), then one quantize pass that derives the scales
// on the device, writes q8 and k8 as E4M3 bytes (the tensor-core operands of
// QK^T), v as bf16 holding exactly the E4M3-rounded values (the reference
// casts v8 to bf16 for its P.V dot; every E4M3 value is a bf16 value), and
// the three scales to a device array that the attention kernel reads.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "sa_common.cuh"
#include "smooth_attn_b200.h"

int sa_record_cuda_error(cudaError_t e);

namespace sa {

constexpr float kE4M3Max = 448.0f;

struct Fp8Src {
  const void* p[3];
  int64_t n[3];  // elements; each a multiple of 8
};

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
  } else {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(p));
    unpack<T, 8>(&w, f);
  }
}

// amax[3] (float bits) must be zero on entry.
template <typename T>
__global__ void __launch_bounds__(256) fp8_absmax_kernel(Fp8Src s, unsigned* __restrict__ amax) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int t = 0; t < 3; ++t) {
    const T* x = static_cast<const T*>(s.p[t]);
    float m = 0.f;
    const int64_t nv = s.n[t] / 8;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < nv; i += 4 * stride) {  // four independent 16-byte loads in flight
      float f[4][8];
#pragma unroll
      for (int j = 0; j < 4; ++j) load8<T>(x + (i + j * stride) * 8, f[j]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(f[j][e]));  // NaN inputs are dropped by fmaxf
    }
    for (; i < nv; i += stride) {
      float f[8];
      load8<T>(x + i * 8, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(f[e]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(amax + t, __float_as_uint(m));
  }
}

__device__ __forceinline__ float fp8_scale(unsigned amax_bits) {
  return fmaxf(__fdiv_rn(__uint_as_float(amax_bits), kE4M3Max), 1e-12f);
}

__device__ __forceinline__ uint8_t to_e4m3(float x, float scale) {
  const float v = fminf(fmaxf(__fdiv_rn(x, scale), -kE4M3Max), kE4M3Max);
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ float e4m3_to_f(uint8_t b) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

template <typename T>
__global__ void __launch_bounds__(256) fp8_quantize_kernel(Fp8Src s, const unsigned* __restrict__ amax,
                                                           uint8_t* __restrict__ q8, uint8_t* __restrict__ k8,
                                                           __nv_bfloat16* __restrict__ vq,
                                                           float* __restrict__ scales) {
  const float sc[3] = {fp8_scale(amax[0]), fp8_scale(amax[1]), fp8_scale(amax[2])};
  if (blockIdx.x == 0 && threadIdx.x < 3) scales[threadIdx.x] = sc[threadIdx.x];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int t = 0; t < 3; ++t) {
    const T* x = static_cast<const T*>(s.p[t]);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < s.n[t] / 8; i += stride) {
      float f[8];
      if (!SA_DCHECK(i * 8 + 8 <= s.n[t])) continue;
      load8<T>(x + i * 8, f);
      uint8_t b[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) b[e] = to_e4m3(f[e], sc[t]);
      if (t < 2) {
        uint2 w;
        w.x = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
        w.y = (uint32_t)b[4] | ((uint32_t)b[5] << 8) | ((uint32_t)b[6] << 16) | ((uint32_t)b[7] << 24);
        *reinterpret_cast<uint2*>((t == 0 ? q8 : k8) + i * 8) = w;
      } else {
        Pack<__nv_bfloat16, 8> o;
#pragma unroll
        for (int e = 0; e < 8; ++e) o.set(e, e4m3_to_f(b[e]));  // exact in bf16
        *reinterpret_cast<uint4*>(vq + i * 8) = o.u;
      }
    }
  }
}

template <typename T>
int launch_fp8_quantize(const Fp8Src& s, unsigned* amax, uint8_t* q8, uint8_t* k8, __nv_bfloat16* vq,
                        float* scales, cudaStream_t st) {
  const int64_t n = std::max(s.n[0], std::max(s.n[1], s.n[2])) / 8;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8));
  cudaError_t e = cudaMemsetAsync(amax, 0, 3 * sizeof(unsigned), st);
  if (e != cudaSuccess) return sa_record_cuda_error(e);
  fp8_absmax_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(s, amax);
  fp8_quantize_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(s, amax, q8, k8, vq, scales);
  return sa_record_cuda_error(cudaGetLastError());
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace sa

extern "C" int sa_fp8_quantize(const void* q, const void* k, const void* v, int64_t nq, int64_t nk, int64_t nv,
                               int dtype, void* q8, void* k8, void* vq, float* scales, void* workspace,
                               void* stream) {
  if (!q || !k || !v || !q8 || !k8 || !vq || !scales || !workspace) return SA_ERR_ARG;
  if (nq < 0 || nk < 0 || nv < 0) return SA_ERR_ARG;
  if (nq % 8 || nk % 8 || nv % 8) return SA_ERR_UNSUPPORTED;
  if (dtype != SA_F32 && dtype != SA_F16 && dtype != SA_BF16) return SA_ERR_UNSUPPORTED;
  if (!sa::al16(q) || !sa::al16(k) || !sa::al16(v) || !sa::al16(vq) ||
      (reinterpret_cast<uintptr_t>(q8) & 7u) || (reinterpret_cast<uintptr_t>(k8) & 7u) ||
      (reinterpret_cast<uintptr_t>(workspace) & 3u))
    return SA_ERR_ALIGN;
  sa::Fp8Src s{{q, k, v}, {nq, nk, nv}};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* amax = static_cast<unsigned*>(workspace);
  auto* q8p = static_cast<uint8_t*>(q8);
  auto* k8p = static_cast<uint8_t*>(k8);
  auto* vqp = static_cast<__nv_bfloat16*>(vq);
  switch (dtype) {
    case SA_F32: return sa::launch_fp8_quantize<float>(s, amax, q8p, k8p, vqp, scales, st);
    case SA_F16: return sa::launch_fp8_quantize<__half>(s, amax, q8p, k8p, vqp, scales, st);
    default: return sa::launch_fp8_quantize<__nv_bfloat16>(s, amax, q8p, k8p, vqp, scales, st);
  }
}
SA_BOUNDS_ACCESSOR(fp8_bounds)
