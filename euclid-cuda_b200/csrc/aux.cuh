// The extra K block of the fast argmin screen (one 32-byte K block appended to every
// row of A and every center row of B).
//
// Center row j of B holds [c0, c1, c2, 2^E, 2^E, 2^E, 0 ...] and point row i of A holds
// [2^E, 2^E, 2^E, r0, r1, r2, 0 ...], where c0..c2 are cc_j / 2 * 2^-E and r0..r2 are
// Br_i / 2 * 2^-E (Br_i = 1.0625 pp_i), each split in three parts of the operand type
// (a part is the rounding of what the earlier parts left).  Products with 2^E are
// exact, so the MMA adds y0 = (cc_j + Br_i) / 2 to the accumulator of pair (i, j) to
// within the type's precision cubed.  With the centers stored negated the accumulator
// is y = y0 - s >= 0, because 2 s <= pp + cc <= Br + cc (Cauchy-Schwarz, with 1/16 of pp
// to spare for the rounding of the norms).
//
// E scales fp16 parts into fp16's range (0 for bf16 and tf32, whose range is fp32's);
// E = 16 means the norms do not fit even scaled and the screen is not used.
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>

namespace euc {

constexpr float kAuxRowScale = 1.0625f;  // Br = kAuxRowScale * pp
constexpr int kAuxNoScreen = 16;         // E value: norms out of range, every row is redone

// rounding of v to the operand type, as stored (fp16 / bf16: 16 bits; tf32: 32 bits)
template <int KIND> __device__ __forceinline__ uint32_t low_bits(float v);
template <> __device__ __forceinline__ uint32_t low_bits<0>(float v) { return __half_as_ushort(__float2half_rn(v)); }
template <> __device__ __forceinline__ uint32_t low_bits<1>(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
template <> __device__ __forceinline__ uint32_t low_bits<2>(float v) {
  uint32_t b;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b) : "f"(v));
  return b;
}
template <int KIND> __device__ __forceinline__ float low_value(uint32_t b);
template <> __device__ __forceinline__ float low_value<0>(uint32_t b) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(b)));
}
template <> __device__ __forceinline__ float low_value<1>(uint32_t b) {
  return __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(b)));
}
template <> __device__ __forceinline__ float low_value<2>(uint32_t b) { return __uint_as_float(b); }

// three parts of v: p0 = low(v), p1 = low(v - p0), p2 = low(v - p0 - p1)
template <int KIND> __device__ __forceinline__ void split3(float v, uint32_t p[3]) {
  float r = v;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    p[k] = low_bits<KIND>(r);
    r = r - low_value<KIND>(p[k]);
  }
}

// a 32-byte extra-K row from its first six elements (the rest zero), as two 16-byte
// chunks in memory order
template <int KIND> __device__ __forceinline__ void aux_pack(const uint32_t e[6], uint4& lo, uint4& hi) {
  if constexpr (KIND == 2) {
    lo = make_uint4(e[0], e[1], e[2], e[3]);
    hi = make_uint4(e[4], e[5], 0u, 0u);
  } else {
    lo = make_uint4(e[0] | (e[1] << 16), e[2] | (e[3] << 16), e[4] | (e[5] << 16), 0u);
    hi = make_uint4(0u, 0u, 0u, 0u);
  }
}

// E for the largest finite center norm: fp16 parts of cc / 2 * 2^-E stay <= 2^7, which
// leaves room for point norms up to about 2^8 times the largest center norm
template <int KIND> __device__ __forceinline__ int aux_exponent(float max_cc) {
  if constexpr (KIND != 0) return 0;
  if (!(max_cc > 0.f)) return 0;  // all center norms zero: no scale to follow
  int e = -24;
  while (e < kAuxNoScreen && 0.5f * max_cc > ldexpf(128.f, e)) ++e;
  return e;
}

}  // namespace euc
