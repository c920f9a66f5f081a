// Direct distance sum_k (p_k - c_k)^2 for one pair, in each fallback arithmetic the
// reference uses.  Accumulation is sequential in k with a fused multiply-add, which
// is what nvcc emits for the reference's `acc += diff * diff` loops.
#pragma once
#include "common.cuh"
#include "engine.h"

namespace euc {

template <typename T> __device__ __forceinline__ double wide(T x);
template <> __device__ __forceinline__ double wide<float>(float x) { return static_cast<double>(x); }
template <> __device__ __forceinline__ double wide<double>(double x) { return x; }
template <> __device__ __forceinline__ double wide<__half>(__half x) { return static_cast<double>(__half2float(x)); }
template <> __device__ __forceinline__ double wide<__nv_bfloat16>(__nv_bfloat16 x) {
  return static_cast<double>(__bfloat162float(x));
}
template <typename T> __device__ __forceinline__ float narrow(T x);
template <> __device__ __forceinline__ float narrow<float>(float x) { return x; }
template <> __device__ __forceinline__ float narrow<double>(double x) { return static_cast<float>(x); }
template <> __device__ __forceinline__ float narrow<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float narrow<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// Returns the recomputed distance widened to double (exact for the fp32/fp16/bf16 results).
//   RC_F64        direct_on_list_rowmajor (euclidean_kernels_mix.cu:156-177),
//                 direct_on_list_fp16/_bf16/_fp64 (euclidean_kernels_advanced.cu:148-220)
//   RC_F32        direct_fp32_on_list (euclidean_kernels_mix.cu:481-504)
//   RC_F16_ARITH  direct_fp16_on_list (euclidean_kernels_mix.cu:412-439)
//   RC_BF16_ARITH direct_bf16_on_list (euclidean_kernels_mix.cu:442-469)
template <typename TIN, int REC>
__device__ __forceinline__ double direct_dist(const TIN* __restrict__ p, const TIN* __restrict__ c, int dim) {
  if constexpr (REC == RC_F64) {
    double acc = 0.0;
    for (int k = 0; k < dim; ++k) {
      const double diff = wide(p[k]) - wide(c[k]);
      acc = fma(diff, diff, acc);
    }
    return acc;
  } else if constexpr (REC == RC_F32) {
    float acc = 0.f;
    for (int k = 0; k < dim; ++k) {
      const float diff = __fsub_rn(narrow(p[k]), narrow(c[k]));
      acc = __fmaf_rn(diff, diff, acc);
    }
    return static_cast<double>(acc);
  } else if constexpr (REC == RC_F16_ARITH) {
    __half acc = __float2half(0.f);
    for (int k = 0; k < dim; ++k) {
      const __half d = __hsub(__float2half_rn(narrow(p[k])), __float2half_rn(narrow(c[k])));
      acc = __hadd(acc, __hmul(d, d));
    }
    return static_cast<double>(__half2float(acc));
  } else if constexpr (REC == RC_BF16_ARITH) {
    __nv_bfloat16 acc = __float2bfloat16(0.f);
    for (int k = 0; k < dim; ++k) {
      const __nv_bfloat16 d = __hsub(__float2bfloat16_rn(narrow(p[k])), __float2bfloat16_rn(narrow(c[k])));
      acc = __hadd(acc, __hmul(d, d));
    }
    return static_cast<double>(__bfloat162float(acc));
  } else {
    return 0.0;
  }
}

}  // namespace euc
