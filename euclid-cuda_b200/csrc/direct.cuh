// Direct distance sum_k (p_k - c_k)^2 for one pair, in each fallback arithmetic the
// reference uses.  Accumulation is sequential in k with a fused multiply-add, which
// is what nvcc emits for the reference's `acc += diff * diff` loops.
#pragma once
#include "common.cuh"
#include "engine.h"

#include <type_traits>

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
// The half-arithmetic loops `acc += d * d` compile to one fused multiply-add per
// element on sm_100 (a single rounding of d*d + acc); it is written as such here.
template <typename TIN, int REC>
__device__ __forceinline__ double direct_dist_scalar(const TIN* __restrict__ p, const TIN* __restrict__ c, int dim) {
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
      acc = __hfma(d, d, acc);
    }
    return static_cast<double>(__half2float(acc));
  } else if constexpr (REC == RC_BF16_ARITH) {
    __nv_bfloat16 acc = __float2bfloat16(0.f);
    for (int k = 0; k < dim; ++k) {
      const __nv_bfloat16 d = __hsub(__float2bfloat16_rn(narrow(p[k])), __float2bfloat16_rn(narrow(c[k])));
      acc = __hfma(d, d, acc);
    }
    return static_cast<double>(__bfloat162float(acc));
  } else {
    return 0.0;
  }
}

// One element of the direct sum for fp32 inputs, in each fallback arithmetic (the
// same operations as direct_dist_scalar<float, REC>).
template <int REC> struct DirectAcc;
template <> struct DirectAcc<RC_F64> {
  double a = 0.0;
  __device__ __forceinline__ void add(float p, float c) {
    const double d = static_cast<double>(p) - static_cast<double>(c);
    a = fma(d, d, a);
  }
  __device__ __forceinline__ double get() const { return a; }
};
template <> struct DirectAcc<RC_F32> {
  float a = 0.f;
  __device__ __forceinline__ void add(float p, float c) {
    const float d = __fsub_rn(p, c);
    a = __fmaf_rn(d, d, a);
  }
  __device__ __forceinline__ double get() const { return static_cast<double>(a); }
};
template <> struct DirectAcc<RC_F16_ARITH> {
  __half a = __float2half(0.f);
  __device__ __forceinline__ void add(float p, float c) {
    const __half d = __hsub(__float2half_rn(p), __float2half_rn(c));
    a = __hfma(d, d, a);
  }
  __device__ __forceinline__ double get() const { return static_cast<double>(__half2float(a)); }
};
template <> struct DirectAcc<RC_BF16_ARITH> {
  __nv_bfloat16 a = __float2bfloat16(0.f);
  __device__ __forceinline__ void add(float p, float c) {
    const __nv_bfloat16 d = __hsub(__float2bfloat16_rn(p), __float2bfloat16_rn(c));
    a = __hfma(d, d, a);
  }
  __device__ __forceinline__ double get() const { return static_cast<double>(__bfloat162float(a)); }
};

// Direct distance of one pair.  fp32 rows that are 16-byte aligned with dim % 4 == 0
// are read 16 elements at a time (the loads issue together, the sum stays in k order).
template <typename TIN, int REC>
__device__ __forceinline__ double direct_dist(const TIN* __restrict__ p, const TIN* __restrict__ c, int dim) {
  if constexpr (std::is_same<TIN, float>::value && REC >= RC_F64 && REC <= RC_BF16_ARITH) {
    if ((dim & 3) == 0 && ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(c)) & 15u) == 0) {
      DirectAcc<REC> acc;
      const float4* p4 = reinterpret_cast<const float4*>(p);
      const float4* c4 = reinterpret_cast<const float4*>(c);
      const int nv = dim >> 2;
      for (int v0 = 0; v0 < nv; v0 += 4) {
        float4 a[4], b[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (v0 + t < nv) {
            a[t] = __ldg(p4 + v0 + t);
            b[t] = __ldg(c4 + v0 + t);
          }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (v0 + t < nv) {
            acc.add(a[t].x, b[t].x);
            acc.add(a[t].y, b[t].y);
            acc.add(a[t].z, b[t].z);
            acc.add(a[t].w, b[t].w);
          }
        }
      }
      return acc.get();
    }
  }
  return direct_dist_scalar<TIN, REC>(p, c, dim);
}

// The reference's distance for one accumulator value: S rounded to the GEMM's
// output precision, then max((pp - 2 s) + cc, 0) (form_mixed_and_list_*,
// euclidean_kernels_mix.cu:203-204).
template <int SROUND>
__device__ __forceinline__ float exact_d(float s, float pp, float cc) {
  if constexpr (SROUND == SR_F16) s = round_f16(s);
  if constexpr (SROUND == SR_BF16) s = round_bf16(s);
  return fmaxf(__fadd_rn(__fmaf_rn(-2.f, s, pp), cc), 0.f);
}

}  // namespace euc
