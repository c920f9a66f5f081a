// Row preparation: squared norms with the reference's exact accumulation order and,
// for the tensor-core path, a zero-padded low-precision copy whose rows are a whole
// number of 128-byte TMA boxes.
//
// Norm recipes (all accumulate k = 0 .. dim-1 in order, one row per thread):
//   NM_LOW_F16 / NM_LOW_BF16: s = fmaf(h, h, s) over h = low(x), stored low
//                             (compute_norms_fp16_uniform, euclidean_kernels_mix.cu:106-135)
//   NM_F32_FMA:   s = fmaf(x, x, s)            (compute_norms_rowmajor_float, euclidean_kernels.cu:16-26)
//   NM_F32_SUMSQ: s = s + fl(x*x)              ((P*P).sum(1), euclidean_kernels_tiled.cu:338)
//   NM_F64_FMA:   s = fma(x, x, s) in fp64     (compute_norms_rowmajor_double, euclidean_kernels.cu:28-38)
//
// Layout: a warp owns 32 rows; 32-column slabs are read coalesced into a padded
// shared tile (33 words per row, conflict-free transposed reads), then lane r folds
// row r's slab into its running norm and the slab is written back out as the low copy.
#include "common.cuh"
#include "engine.h"
#include "aux.cuh"

#include <type_traits>
#include <algorithm>

namespace euc {

template <typename T> __device__ __forceinline__ double to_d(T x);
template <> __device__ __forceinline__ double to_d<float>(float x) { return static_cast<double>(x); }
template <> __device__ __forceinline__ double to_d<double>(double x) { return x; }
template <> __device__ __forceinline__ double to_d<__half>(__half x) { return static_cast<double>(__half2float(x)); }
template <> __device__ __forceinline__ double to_d<__nv_bfloat16>(__nv_bfloat16 x) {
  return static_cast<double>(__bfloat162float(x));
}
template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<double>(double x) { return static_cast<float>(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// LOWT: 0 none, 1 fp16, 2 bf16, 3 tf32 (fp32 storage, rounded to 10 mantissa bits)
// value of x rounded to the MMA operand type LOWT (1 fp16, 2 bf16, 3 tf32), as fp32
template <int LOWT> __device__ __forceinline__ float operand_value(float x) {
  if constexpr (LOWT == 1) return round_f16(x);
  else if constexpr (LOWT == 2) return round_bf16(x);
  else {
    uint32_t b;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b) : "f"(x));
    return __uint_as_float(b);
  }
}

template <typename TIN, int NORM, int LOWT>
__global__ void __launch_bounds__(128) prep_rows_kernel(const TIN* __restrict__ X, int64_t rows, int dim,
                                                        void* __restrict__ low, int ldl,
                                                        void* __restrict__ norms) {
  constexpr bool kDouble = (NORM == NM_F64_FMA);
  using TS = typename std::conditional<kDouble, double, float>::type;
  __shared__ TS tile[4][32][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * 4 + warp) * 32;
  if (row0 >= rows) return;
  TS (*t)[33] = tile[warp];
  TS acc = 0;
  const int64_t my_row = row0 + lane;
  for (int c0 = 0; c0 < dim; c0 += 32) {
    const int c = c0 + lane;
#pragma unroll 4
    for (int r = 0; r < 32; ++r) {
      const int64_t gr = row0 + r;
      TS v = 0;
      if (gr < rows && c < dim) {
        if constexpr (kDouble)
          v = to_d(X[gr * dim + c]);
        else
          v = to_f(X[gr * dim + c]);
      }
      t[r][lane] = v;
    }
    __syncwarp();
    const int cend = min(32, dim - c0);
    for (int cc = 0; cc < cend; ++cc) {
      TS x = t[lane][cc];
      if constexpr (NORM == NM_LOW_F16) {
        const float h = round_f16(x);
        acc = __fmaf_rn(h, h, acc);
      } else if constexpr (NORM == NM_LOW_BF16) {
        const float h = round_bf16(x);
        acc = __fmaf_rn(h, h, acc);
      } else if constexpr (NORM == NM_F32_FMA) {
        acc = __fmaf_rn(x, x, acc);
      } else if constexpr (NORM == NM_F32_SUMSQ) {
        acc = __fadd_rn(acc, __fmul_rn(x, x));
      } else if constexpr (NORM == NM_OPERAND) {
        const float h = operand_value<LOWT>(x);
        acc = __fmaf_rn(h, h, acc);
      } else {
        acc = fma(x, x, acc);
      }
    }
    if constexpr (LOWT != 0) {
#pragma unroll 4
      for (int r = 0; r < 32; ++r) {
        const int64_t gr = row0 + r;
        if (gr < rows) {
          const float x = static_cast<float>(t[r][lane]);
          if constexpr (LOWT == 1)
            static_cast<__half*>(low)[gr * ldl + c] = __float2half_rn(c < dim ? x : 0.f);
          else if constexpr (LOWT == 2)
            static_cast<__nv_bfloat16*>(low)[gr * ldl + c] = __float2bfloat16_rn(c < dim ? x : 0.f);
          else {
            uint32_t b;
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b) : "f"(c < dim ? x : 0.f));
            static_cast<uint32_t*>(low)[gr * ldl + c] = b;
          }
        }
      }
    }
    __syncwarp();
  }
  // zero padding up to the padded row length
  if constexpr (LOWT != 0) {
    const int cstart = ((dim + 31) / 32) * 32;
    for (int r = 0; r < 32; ++r) {
      const int64_t gr = row0 + r;
      if (gr >= rows) break;
      for (int c = cstart + lane; c < ldl; c += 32) {
        if constexpr (LOWT == 1)
          static_cast<__half*>(low)[gr * ldl + c] = __float2half_rn(0.f);
        else if constexpr (LOWT == 2)
          static_cast<__nv_bfloat16*>(low)[gr * ldl + c] = __float2bfloat16_rn(0.f);
        else
          static_cast<uint32_t*>(low)[gr * ldl + c] = 0u;
      }
    }
  }
  if (my_row < rows) {
    if constexpr (NORM == NM_LOW_F16)
      static_cast<float*>(norms)[my_row] = round_f16(acc);
    else if constexpr (NORM == NM_LOW_BF16)
      static_cast<float*>(norms)[my_row] = round_bf16(acc);
    else if constexpr (kDouble)
      static_cast<double*>(norms)[my_row] = acc;
    else
      static_cast<float*>(norms)[my_row] = acc;
  }
}

// fp32 rows with dim % 4 == 0 and 16-byte aligned rows: same results, vector traffic.
// A half-warp reads one row's 64-column slab with 16-byte loads (two rows per load
// instruction), writes the low copy straight from registers (8- or 16-byte stores,
// coalesced) and parks the slab in shared memory, from where lane r folds row r into
// its norm in column order.
template <int NORM, int LOWT>
__global__ void __launch_bounds__(128) prep_rows_v4_kernel(const float* __restrict__ X, int64_t rows, int dim,
                                                           void* __restrict__ low, int ldl,
                                                           float* __restrict__ norms) {
  __shared__ float tile[4][32][65];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * 4 + warp) * 32;
  if (row0 >= rows) return;
  float (*t)[65] = tile[warp];
  const int half = lane >> 4, hl = lane & 15;
  float acc = 0.f;
  for (int c0 = 0; c0 < dim; c0 += 64) {
    const int c = c0 + hl * 4;
    const bool cok = c < dim;  // dim % 4 == 0: the whole vector is inside the row
    float4 v[16];
#pragma unroll
    for (int it = 0; it < 16; ++it) {
      const int64_t gr = row0 + it * 2 + half;
      v[it] = (gr < rows && cok) ? __ldg(reinterpret_cast<const float4*>(X + gr * dim + c))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int it = 0; it < 16; ++it) {
      const int r = it * 2 + half;
      t[r][hl * 4 + 0] = v[it].x;
      t[r][hl * 4 + 1] = v[it].y;
      t[r][hl * 4 + 2] = v[it].z;
      t[r][hl * 4 + 3] = v[it].w;
      if constexpr (LOWT != 0) {
        const int64_t gr = row0 + r;
        if (gr < rows && c < ldl) {
          if constexpr (LOWT == 1) {
            const __half2 a = __floats2half2_rn(v[it].x, v[it].y), b = __floats2half2_rn(v[it].z, v[it].w);
            uint2 w;
            w.x = *reinterpret_cast<const uint32_t*>(&a);
            w.y = *reinterpret_cast<const uint32_t*>(&b);
            *reinterpret_cast<uint2*>(static_cast<__half*>(low) + gr * ldl + c) = w;
          } else if constexpr (LOWT == 2) {
            const __nv_bfloat162 a = __floats2bfloat162_rn(v[it].x, v[it].y);
            const __nv_bfloat162 b = __floats2bfloat162_rn(v[it].z, v[it].w);
            uint2 w;
            w.x = *reinterpret_cast<const uint32_t*>(&a);
            w.y = *reinterpret_cast<const uint32_t*>(&b);
            *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(low) + gr * ldl + c) = w;
          } else {
            uint4 w;
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(w.x) : "f"(v[it].x));
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(w.y) : "f"(v[it].y));
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(w.z) : "f"(v[it].z));
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(w.w) : "f"(v[it].w));
            *reinterpret_cast<uint4*>(static_cast<uint32_t*>(low) + gr * ldl + c) = w;
          }
        }
      }
    }
    __syncwarp();
    const int cend = min(64, dim - c0);
    for (int k = 0; k < cend; ++k) {
      const float x = t[lane][k];
      if constexpr (NORM == NM_LOW_F16) {
        const float h = round_f16(x);
        acc = __fmaf_rn(h, h, acc);
      } else if constexpr (NORM == NM_LOW_BF16) {
        const float h = round_bf16(x);
        acc = __fmaf_rn(h, h, acc);
      } else if constexpr (NORM == NM_F32_FMA) {
        acc = __fmaf_rn(x, x, acc);
      } else if constexpr (NORM == NM_OPERAND) {
        const float h = operand_value<LOWT>(x);
        acc = __fmaf_rn(h, h, acc);
      } else {
        acc = __fadd_rn(acc, __fmul_rn(x, x));
      }
    }
    __syncwarp();
  }
  const int64_t my_row = row0 + lane;
  if (my_row < rows) {
    if constexpr (NORM == NM_LOW_F16)
      norms[my_row] = round_f16(acc);
    else if constexpr (NORM == NM_LOW_BF16)
      norms[my_row] = round_bf16(acc);
    else
      norms[my_row] = acc;
  }
}

template <typename TIN, int NORM, int LOWT>
static cudaError_t go(const void* X, int64_t rows, int dim, void* low, int ldl, void* norms, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const int64_t blocks = (rows + 127) / 128;
  if constexpr (std::is_same<TIN, float>::value && NORM != NM_F64_FMA) {
    // the vector kernel's low stores need 8 (fp16/bf16) or 16 (tf32) byte aligned rows
    const bool vec_ok = (dim % 4 == 0) && (reinterpret_cast<uintptr_t>(X) % 16 == 0) &&
                        (LOWT == 0 || ((reinterpret_cast<uintptr_t>(low) % 16 == 0) && ldl % 4 == 0));
    if (vec_ok) {
      prep_rows_v4_kernel<NORM, LOWT><<<static_cast<unsigned>(blocks), 128, 0, st>>>(
          static_cast<const float*>(X), rows, dim, low, ldl, static_cast<float*>(norms));
      return cudaGetLastError();
    }
  }
  prep_rows_kernel<TIN, NORM, LOWT><<<static_cast<unsigned>(blocks), 128, 0, st>>>(
      static_cast<const TIN*>(X), rows, dim, low, ldl, norms);
  return cudaGetLastError();
}

// points=true prepares P (n rows), else C (m rows).
cudaError_t launch_prep(const DistJob& j, bool points, bool make_low) {
  const OpSpec* s = j.spec;
  const void* X = points ? j.P : j.C;
  const int64_t rows = points ? j.n : j.m;
  void* low = make_low ? (points ? j.Plow : j.Clow) : nullptr;
  void* nrm = points ? j.pp : j.cc;
  const int ldl = j.ldlow;
  int lowt = 0;
  if (make_low) lowt = (s->gemm == G_TC_F16) ? 1 : (s->gemm == G_TC_BF16 ? 2 : 3);
  cudaStream_t st = j.stream;

  // the certified screen takes the fp32 norms of the rounded operands instead
  const int norm = (j.cert && make_low) ? static_cast<int>(NM_OPERAND) : static_cast<int>(s->norm);
#define PREP(TIN_, NORM_, LOWT_)                                   \
  if (norm == NORM_ && lowt == LOWT_)                              \
    return go<TIN_, NORM_, LOWT_>(X, rows, j.dim, low, ldl, nrm, st);

  switch (s->in) {
    case IN_F32:
      PREP(float, NM_LOW_F16, 1)
      PREP(float, NM_LOW_BF16, 2)
      PREP(float, NM_F32_FMA, 3)
      PREP(float, NM_F32_FMA, 0)
      PREP(float, NM_F32_SUMSQ, 1)
      PREP(float, NM_F32_SUMSQ, 2)
      PREP(float, NM_F32_SUMSQ, 0)
      PREP(float, NM_F64_FMA, 0)
      PREP(float, NM_OPERAND, 1)
      PREP(float, NM_OPERAND, 2)
      PREP(float, NM_OPERAND, 3)
      break;
    case IN_F16:
      PREP(__half, NM_LOW_F16, 1)
      PREP(__half, NM_F32_FMA, 0)
      break;
    case IN_BF16:
      PREP(__nv_bfloat16, NM_LOW_BF16, 2)
      PREP(__nv_bfloat16, NM_F32_FMA, 0)
      break;
    case IN_F64:
      PREP(double, NM_F64_FMA, 0)
      break;
  }
#undef PREP
  return cudaErrorNotSupported;
}

// ------------------------------------------------ norm range check
// Sets *flag to 1 if some row's fp32 sum of squares is not finite or lies outside
// [lo, hi] (a NaN sum fails the test too).  One warp per row, grid-stride; the lanes
// read consecutive values, so a warp's loads of a row are coalesced.  Used to decide,
// before any distance is formed, whether the cancellation test provably flags every
// pair (api.cu, the all-flagged route).
__global__ void __launch_bounds__(256) norm_range_kernel(const float* __restrict__ X, int64_t rows, int dim,
                                                         float lo, float hi, int* flag) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * 8;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5); r < rows; r += warps) {
    const float* x = X + r * dim;
    float acc = 0.f;
    for (int k = lane; k < dim; k += 32) acc = __fmaf_rn(__ldg(x + k), __ldg(x + k), acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0 && !(acc >= lo && acc <= hi)) atomicOr(flag, 1);
  }
}

cudaError_t launch_norm_range_check(const float* X, int64_t rows, int dim, float lo, float hi, int* flag,
                                    cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const int64_t want = (rows + 7) / 8;
  const int blocks = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(num_sms()) * 8));
  norm_range_kernel<<<blocks, 256, 0, st>>>(X, rows, dim, lo, hi, flag);
  return cudaGetLastError();
}

// ------------------------------------------------ fast argmin: sorted centers
// Stable rank sort of the centers by norm (ties kept in index order, NaN as +inf):
// rank_j = #{i : key_i < key_j or (key_i == key_j and i < j)}.  One warp per center,
// its lanes counting over the norms staged in shared memory.  Every block also reduces
// the largest finite norm (all blocks see all norms, so they agree), derives E of the
// extra K block (aux.cuh) and block 0 stores both.  Sorted position r receives the
// norm, the original index, the low-precision row NEGATED (the screening MMA forms
// y0 - s) and the center's extra-K row [c0, c1, c2, 2^E, 2^E, 2^E] (all zero for a norm
// that is not finite); the padded positions m .. mpad-1 get +inf in c0, so their keys
// never win.
template <int KIND>
__global__ void __launch_bounds__(256) sort_centers_kernel(const float* __restrict__ cc, int m, int mpad,
                                                           const uint4* __restrict__ low, int row_u4,
                                                           float* __restrict__ cc_s, int* __restrict__ perm,
                                                           uint4* __restrict__ low_s, int* __restrict__ aux_e,
                                                           float* __restrict__ ccmax, uint4* __restrict__ b_aux) {
  constexpr int SLAB = 2048;
  __shared__ float tile[SLAB];
  __shared__ unsigned int s_max;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x * 8 + warp;
  const float kInf = __int_as_float(0x7f800000);
  float kj = 0.f;
  if (j < m) {
    kj = cc[j];
    if (kj != kj) kj = kInf;
  }
  if (threadIdx.x == 0) s_max = 0u;
  int rank = 0;
  float mc = 0.f;
  for (int base = 0; base < m; base += SLAB) {
    __syncthreads();
    for (int t = threadIdx.x; t < SLAB && base + t < m; t += blockDim.x) {
      const float v = cc[base + t];
      if (v < 3.0e38f && v > mc) mc = v;  // skips inf and NaN
      tile[t] = (v != v) ? kInf : v;
    }
    __syncthreads();
    const int lim = min(SLAB, m - base);
    if (j < m) {
      for (int t = lane; t < lim; t += 32) {
        const float ki = tile[t];
        const int i = base + t;
        rank += (ki < kj) || (ki == kj && i < j);
      }
    }
  }
  rank = __reduce_add_sync(0xffffffffu, rank);
  const unsigned int wm = __reduce_max_sync(0xffffffffu, __float_as_uint(mc));  // non-negative: bits order as values
  if (lane == 0) atomicMax(&s_max, wm);
  __syncthreads();
  const int E = aux_exponent<KIND>(__uint_as_float(s_max));
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *aux_e = E;
    *ccmax = __uint_as_float(s_max);
  }
  if (j >= m && j < mpad && lane == 0) {
    const uint32_t inf_bits = (KIND == 2) ? 0x7f800000u : (KIND == 1 ? 0x7f80u : 0x7c00u);
    b_aux[2 * static_cast<int64_t>(j)] = make_uint4(inf_bits, 0u, 0u, 0u);
    b_aux[2 * static_cast<int64_t>(j) + 1] = make_uint4(0u, 0u, 0u, 0u);
  }
  if (j < m) {
    const float c = cc[j];
    const uint4* src = low + static_cast<int64_t>(j) * row_u4;
    uint4* dst = low_s + static_cast<int64_t>(rank) * row_u4;
    const uint32_t neg = (KIND == 2) ? 0x80000000u : 0x80008000u;
    for (int t = lane; t < row_u4; t += 32) {
      const uint4 w = src[t];
      dst[t] = make_uint4(w.x ^ neg, w.y ^ neg, w.z ^ neg, w.w ^ neg);
    }
    if (lane == 0) {
      cc_s[rank] = c;
      perm[rank] = j;
      uint32_t e[6] = {0u, 0u, 0u, 0u, 0u, 0u};
      if (c < 3.0e38f && E < kAuxNoScreen) {
        split3<KIND>(ldexpf(0.5f * c, -E), e);
        e[3] = e[4] = e[5] = low_bits<KIND>(ldexpf(1.f, E));
      }
      uint4 lo, hi;
      aux_pack<KIND>(e, lo, hi);
      b_aux[2 * static_cast<int64_t>(rank)] = lo;
      b_aux[2 * static_cast<int64_t>(rank) + 1] = hi;
    }
  }
}

cudaError_t launch_sort_centers(const DistJob& j) {
  const int kind = (j.spec->gemm == G_TC_F16) ? 0 : (j.spec->gemm == G_TC_BF16 ? 1 : 2);
  const int es = (kind == 2) ? 4 : 2;
  const int row_u4 = j.ldlow * es / 16;
  const int m = static_cast<int>(j.m);
  const int mpad = (m + 255) & ~255;
  const unsigned grid = static_cast<unsigned>(mpad / 8);  // one warp per sorted position, padding included
  const float* cc = static_cast<const float*>(j.cc);
  const uint4* low = static_cast<const uint4*>(j.Clow);
  uint4* low_s = static_cast<uint4*>(j.Clow_sorted);
  uint4* ba = static_cast<uint4*>(j.b_aux_sorted);
  if (kind == 0)
    sort_centers_kernel<0><<<grid, 256, 0, j.stream>>>(cc, m, mpad, low, row_u4, j.cc_sorted, j.perm, low_s, j.aux_e,
                                                       j.ccmax, ba);
  else if (kind == 1)
    sort_centers_kernel<1><<<grid, 256, 0, j.stream>>>(cc, m, mpad, low, row_u4, j.cc_sorted, j.perm, low_s, j.aux_e,
                                                       j.ccmax, ba);
  else
    sort_centers_kernel<2><<<grid, 256, 0, j.stream>>>(cc, m, mpad, low, row_u4, j.cc_sorted, j.perm, low_s, j.aux_e,
                                                       j.ccmax, ba);
  return cudaGetLastError();
}

}  // namespace euc
