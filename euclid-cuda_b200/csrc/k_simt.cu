// CUDA-core distance kernels.
//
// simt_dist_kernel: S = P.C^T by sequential fused multiply-adds (fp32 or fp64),
//   64x64 output tile per CTA, 4x4 outputs per thread, 16-wide K slabs staged in
//   shared memory; the epilogue is the same form / cancellation test / store-or-argmin
//   logic as the tensor-core kernel.  It serves the operators whose S comes from an
//   fp32 or fp64 GEMM in the reference (torch::mm, euclidean_kernels.cu:107,142;
//   euclidean_kernels_mix.cu:949,1550; euclidean_kernels_uniform.cu:239;
//   euclidean_kernels_advanced.cu:253,311,370,426) and the fp32 tiled operators
//   (euclidean_kernels_tiled.cu:500-528).
// direct_kernel: D = sum_k (p_k - c_k)^2 for every pair, same tiling
//   (pairwise_distance_direct_*, euclidean_kernels_uniform.cu:262-505).
#include "common.cuh"
#include "engine.h"
#include "direct.cuh"

namespace euc {

struct SimtArgs {
  const void* P;
  const void* C;
  int64_t n, m;
  int dim;
  const void* pp;
  const void* cc;
  float kf;
  double kd;
  void* D;
  unsigned long long* row_key;
  double* row_val64;
  long long* row_idx64;
  unsigned long long* count;
  unsigned long long* list;
  unsigned long long cap;
  int32_t* tile_counts;
  int tile_T;
  int64_t tiles_j;
};

constexpr int SB = 64;   // tile edge
constexpr int SK = 16;   // K slab
enum SimtMode { SM_D = 0, SM_ARGMIN_KEY = 1, SM_ARGMIN_F64 = 2 };

template <typename TACC, typename TIN> __device__ __forceinline__ TACC cvt_in(TIN x);
template <> __device__ __forceinline__ float cvt_in<float, float>(float x) { return x; }
template <> __device__ __forceinline__ float cvt_in<float, double>(double x) { return __double2float_rn(x); }
template <> __device__ __forceinline__ double cvt_in<double, float>(float x) { return static_cast<double>(x); }
template <> __device__ __forceinline__ double cvt_in<double, double>(double x) { return x; }
template <> __device__ __forceinline__ double cvt_in<double, __half>(__half x) {
  return static_cast<double>(__half2float(x));
}
template <> __device__ __forceinline__ double cvt_in<double, __nv_bfloat16>(__nv_bfloat16 x) {
  return static_cast<double>(__bfloat162float(x));
}
template <> __device__ __forceinline__ float cvt_in<float, __half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float cvt_in<float, __nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

__device__ __forceinline__ float fma_t(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fma_t(double a, double b, double c) { return __fma_rn(a, b, c); }

template <typename T> __device__ __forceinline__ void store_out(T* p, double v);
template <> __device__ __forceinline__ void store_out<float>(float* p, double v) { *p = static_cast<float>(v); }
template <> __device__ __forceinline__ void store_out<double>(double* p, double v) { *p = v; }
template <> __device__ __forceinline__ void store_out<__half>(__half* p, double v) {
  *p = __float2half_rn(static_cast<float>(v));
}
template <> __device__ __forceinline__ void store_out<__nv_bfloat16>(__nv_bfloat16* p, double v) {
  *p = __float2bfloat16_rn(static_cast<float>(v));
}

// Stage a 64 x 16 slab of rows [r0, r0+64) x cols [k0, k0+16) transposed into s[k][r].
template <typename TACC, typename TIN>
__device__ __forceinline__ void load_slab(TACC (*s)[SB + 4], const TIN* __restrict__ X, int64_t rows, int dim,
                                          int64_t r0, int k0) {
  for (int t = threadIdx.x; t < SB * SK; t += 256) {
    const int r = t >> 4, kk = t & 15;
    const int64_t gr = r0 + r;
    const int gk = k0 + kk;
    TACC v = 0;
    if (gr < rows && gk < dim) v = cvt_in<TACC>(X[gr * dim + gk]);
    s[kk][r] = v;
  }
}

template <typename TIN, typename TACC, int FORM, int FLAG, int REC, typename TOUT, int MODE>
__global__ void __launch_bounds__(256) simt_dist_kernel(const SimtArgs a) {
  __shared__ TACC As[SK][SB + 4];
  __shared__ TACC Bs[SK][SB + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * SB;
  const TIN* P = static_cast<const TIN*>(a.P);
  const TIN* C = static_cast<const TIN*>(a.C);
  using TN = typename std::conditional<FORM == FM_F64, double, float>::type;  // norm storage
  const TN* ppv = static_cast<const TN*>(a.pp);
  const TN* ccv = static_cast<const TN*>(a.cc);

  TN pp[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t i = row0 + ty * 4 + r;
    pp[r] = (i < a.n) ? ppv[i] : TN(0);
  }
  unsigned long long bkey[4] = {~0ull, ~0ull, ~0ull, ~0ull};
  double bval[4];
  long long bidx[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) { bval[r] = __longlong_as_double(0x7ff0000000000000ll); bidx[r] = -1; }

  const int64_t n_ct = (a.m + SB - 1) / SB;
  const int64_t ct_begin = (MODE == SM_D) ? blockIdx.y : 0;
  const int64_t ct_end = (MODE == SM_D) ? blockIdx.y + 1 : n_ct;
  for (int64_t ct = ct_begin; ct < ct_end; ++ct) {
    const int64_t col0 = ct * SB;
    TACC acc[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[r][c] = 0;
    for (int k0 = 0; k0 < a.dim; k0 += SK) {
      load_slab<TACC, TIN>(As, P, a.n, a.dim, row0, k0);
      load_slab<TACC, TIN>(Bs, C, a.m, a.dim, col0, k0);
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < SK; ++kk) {
        TACC av[4], bv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) av[r] = As[kk][ty * 4 + r];
#pragma unroll
        for (int c = 0; c < 4; ++c) bv[c] = Bs[kk][tx * 4 + c];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[r][c] = fma_t(av[r], bv[c], acc[r][c]);
      }
      __syncthreads();
    }
    // epilogue
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int64_t i = row0 + ty * 4 + r;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int64_t j = col0 + tx * 4 + c;
        if (i >= a.n || j >= a.m) continue;
        const TN cc = ccv[j];
        double dval;  // distance as stored
        bool flag = false;
        if constexpr (FORM == FM_F32) {
          const float s = static_cast<float>(acc[r][c]);
          float d = __fadd_rn(__fmaf_rn(-2.f, s, static_cast<float>(pp[r])), static_cast<float>(cc));
          d = fmaxf(d, 0.f);
          if constexpr (FLAG == FL_F32)
            flag = d <= __fmul_rn(a.kf, __fadd_rn(static_cast<float>(pp[r]), static_cast<float>(cc)));
          dval = d;
        } else if constexpr (FORM == FM_F64) {
          const double s = static_cast<double>(acc[r][c]);
          double d = __dadd_rn(fma(-2.0, s, static_cast<double>(pp[r])), static_cast<double>(cc));
          d = fmax(d, 0.0);
          if constexpr (FLAG == FL_F64)
            flag = d <= a.kd * (static_cast<double>(pp[r]) + static_cast<double>(cc));
          dval = d;
        } else {  // FM_F64_TO_F32
          const double s = static_cast<double>(acc[r][c]);
          const double d64 = __dadd_rn(fma(-2.0, s, static_cast<double>(pp[r])), static_cast<double>(cc));
          const float d = static_cast<float>(fmax(d64, 0.0));
          if constexpr (FLAG == FL_F32)
            flag = d <= __fmul_rn(a.kf, __fadd_rn(static_cast<float>(pp[r]), static_cast<float>(cc)));
          dval = d;
        }
        if constexpr (MODE == SM_D) {
          store_out<TOUT>(static_cast<TOUT*>(a.D) + i * a.m + j, dval);
        } else if constexpr (MODE == SM_ARGMIN_KEY) {
          if (!flag) {
            const unsigned long long key = make_key(static_cast<float>(dval), static_cast<uint32_t>(j));
            bkey[r] = key < bkey[r] ? key : bkey[r];
          }
        } else {
          if (dval < bval[r] || (dval == bval[r] && j < bidx[r])) { bval[r] = dval; bidx[r] = j; }
        }
        if constexpr (FLAG != FL_NONE) {
          if (flag) {
            const unsigned long long pos = atomicAdd(a.count, 1ull);
            if (pos < a.cap) {
              a.list[pos] = (static_cast<unsigned long long>(i) << 32) | static_cast<unsigned long long>(j);
            } else if constexpr (MODE == SM_ARGMIN_KEY) {
              const float dd = static_cast<float>(direct_dist_scalar<TIN, REC>(P + i * a.dim, C + j * a.dim, a.dim));
              const unsigned long long key = make_key(dd, static_cast<uint32_t>(j));
              bkey[r] = key < bkey[r] ? key : bkey[r];
            }
            if (a.tile_counts != nullptr) atomicAdd(&a.tile_counts[(i / a.tile_T) * a.tiles_j + j / a.tile_T], 1);
          }
        }
      }
    }
  }
  if constexpr (MODE != SM_D) {
    // reduce over the 16 threads (tx) that share rows ty*4 .. ty*4+3
#pragma unroll
    for (int r = 0; r < 4; ++r) {
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) {
        if constexpr (MODE == SM_ARGMIN_KEY) {
          const unsigned long long o = __shfl_xor_sync(0xffffffffu, bkey[r], off);
          bkey[r] = o < bkey[r] ? o : bkey[r];
        } else {
          const double ov = __shfl_xor_sync(0xffffffffu, bval[r], off);
          const long long oi = __shfl_xor_sync(0xffffffffu, bidx[r], off);
          if (ov < bval[r] || (ov == bval[r] && oi < bidx[r])) { bval[r] = ov; bidx[r] = oi; }
        }
      }
      const int64_t i = row0 + ty * 4 + r;
      if (tx == 0 && i < a.n) {
        if constexpr (MODE == SM_ARGMIN_KEY)
          a.row_key[i] = bkey[r];
        else {
          a.row_val64[i] = bval[r];
          a.row_idx64[i] = bidx[r];
        }
      }
    }
  }
}

template <typename TIN, typename TACC, int FORM, int FLAG, int REC, typename TOUT, int MODE>
static cudaError_t go_simt(const DistJob& j) {
  SimtArgs a{};
  a.P = j.P;
  a.C = j.C;
  a.n = j.n;
  a.m = j.m;
  a.dim = j.dim;
  a.pp = j.pp;
  a.cc = j.cc;
  a.kf = j.kf;
  a.kd = j.kd;
  a.D = j.D;
  a.row_key = j.row_key;
  a.row_val64 = j.row_val64;
  a.row_idx64 = j.row_idx64;
  a.count = j.count;
  a.list = j.list;
  a.cap = j.list_cap;
  a.tile_counts = j.tile_counts;
  a.tile_T = j.tile_T > 0 ? j.tile_T : 1;
  a.tiles_j = j.tiles_j;
  const int64_t nrt = (j.n + SB - 1) / SB;
  const int64_t nct = (j.m + SB - 1) / SB;
  if (nrt == 0 || nct == 0) return cudaSuccess;
  if (nct > 65535 && MODE == SM_D) return cudaErrorInvalidConfiguration;
  dim3 grid(static_cast<unsigned>(nrt), MODE == SM_D ? static_cast<unsigned>(nct) : 1u);
  timing_begin(j.stream, "simt_dist_kernel");
  simt_dist_kernel<TIN, TACC, FORM, FLAG, REC, TOUT, MODE><<<grid, 256, 0, j.stream>>>(a);
  cudaError_t e = cudaGetLastError();
  timing_end(j.stream);
  return e;
}

cudaError_t launch_simt(const DistJob& j) {
  const OpSpec* s = j.spec;
  const bool argmin = (j.D == nullptr);
  const bool f64key = argmin && s->form == FM_F64;
  const int mode = !argmin ? SM_D : (f64key ? SM_ARGMIN_F64 : SM_ARGMIN_KEY);

#define SIMT_CASE(IN_, TIN_, GEMM_, TACC_, FORM_, FLAG_, REC_, OUT_, TOUT_, MODE_)                   \
  if (s->in == IN_ && s->gemm == GEMM_ && s->form == FORM_ && s->flag == FLAG_ && mode == MODE_ &&  \
      (MODE_ == SM_D ? s->out == OUT_ : true) && (FLAG_ == FL_NONE || s->rec == REC_))               \
    return go_simt<TIN_, TACC_, FORM_, FLAG_, REC_, TOUT_, MODE_>(j);

  // base single / uniform tf32: fp32 GEMM, no flag
  SIMT_CASE(IN_F32, float, G_SIMT_F32, float, FM_F32, FL_NONE, RC_NONE, OUT_F32, float, SM_D)
  SIMT_CASE(IN_F32, float, G_SIMT_F32, float, FM_F32, FL_NONE, RC_NONE, OUT_F32, float, SM_ARGMIN_KEY)
  // base double: fp64 GEMM, no flag
  SIMT_CASE(IN_F64, double, G_SIMT_F64, double, FM_F64, FL_NONE, RC_NONE, OUT_F64, double, SM_D)
  SIMT_CASE(IN_F64, double, G_SIMT_F64, double, FM_F64, FL_NONE, RC_NONE, OUT_F64, double, SM_ARGMIN_F64)
  // mix fp32_fp64 / fp32_fp32, tiled fp32_*
  SIMT_CASE(IN_F32, float, G_SIMT_F32, float, FM_F32, FL_F32, RC_F64, OUT_F32, float, SM_D)
  SIMT_CASE(IN_F32, float, G_SIMT_F32, float, FM_F32, FL_F32, RC_F32, OUT_F32, float, SM_D)
  SIMT_CASE(IN_F32, float, G_SIMT_F32, float, FM_F32, FL_F32, RC_F64, OUT_F32, float, SM_ARGMIN_KEY)
  SIMT_CASE(IN_F32, float, G_SIMT_F32, float, FM_F32, FL_F32, RC_F32, OUT_F32, float, SM_ARGMIN_KEY)
  // advanced fp64_fp16 / fp64_bf16: fp64 GEMM on low inputs, float distances
  SIMT_CASE(IN_F16, __half, G_SIMT_F64, double, FM_F64_TO_F32, FL_F32, RC_F64, OUT_F32, float, SM_D)
  SIMT_CASE(IN_BF16, __nv_bfloat16, G_SIMT_F64, double, FM_F64_TO_F32, FL_F32, RC_F64, OUT_F32, float, SM_D)
  // advanced fp64_tf32 (fp32 GEMM, fp64 form) / fp64_fp32_gemm (fp64 in, fp32 GEMM)
  SIMT_CASE(IN_F32, float, G_SIMT_F32, float, FM_F64, FL_F64, RC_F64, OUT_F64, double, SM_D)
  SIMT_CASE(IN_F64, double, G_SIMT_F32, float, FM_F64, FL_F64, RC_F64, OUT_F64, double, SM_D)
#undef SIMT_CASE
  return cudaErrorNotSupported;
}

// ------------------------------------------------------------------ direct

template <typename TIN, typename TACC, typename TOUT>
__global__ void __launch_bounds__(256) direct_kernel(const TIN* __restrict__ P, const TIN* __restrict__ C,
                                                     int64_t n, int64_t m, int dim, TOUT* __restrict__ D) {
  __shared__ TACC As[SK][SB + 4];
  __shared__ TACC Bs[SK][SB + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * SB;
  const int64_t col0 = static_cast<int64_t>(blockIdx.y) * SB;
  TACC acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0;
  for (int k0 = 0; k0 < dim; k0 += SK) {
    load_slab<TACC, TIN>(As, P, n, dim, row0, k0);
    load_slab<TACC, TIN>(Bs, C, m, dim, col0, k0);
    __syncthreads();
    const int kend = min(SK, dim - k0);  // padded columns must not contribute (p-c)^2 terms
    for (int kk = 0; kk < kend; ++kk) {
      TACC av[4], bv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) av[r] = As[kk][ty * 4 + r];
#pragma unroll
      for (int c = 0; c < 4; ++c) bv[c] = Bs[kk][tx * 4 + c];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const TACC d = av[r] - bv[c];
          acc[r][c] = fma_t(d, d, acc[r][c]);
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t i = row0 + ty * 4 + r;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int64_t j = col0 + tx * 4 + c;
      if (i < n && j < m) store_out<TOUT>(D + i * m + j, static_cast<double>(acc[r][c]));
    }
  }
}

template <typename TIN, typename TACC, typename TOUT>
static cudaError_t go_direct(const void* P, const void* C, int64_t n, int64_t m, int dim, void* D,
                             cudaStream_t st) {
  const int64_t nrt = (n + SB - 1) / SB, nct = (m + SB - 1) / SB;
  if (nrt == 0 || nct == 0) return cudaSuccess;
  if (nct > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid(static_cast<unsigned>(nrt), static_cast<unsigned>(nct));
  timing_begin(st, "direct_kernel");
  direct_kernel<TIN, TACC, TOUT><<<grid, 256, 0, st>>>(static_cast<const TIN*>(P), static_cast<const TIN*>(C), n,
                                                       m, dim, static_cast<TOUT*>(D));
  cudaError_t e = cudaGetLastError();
  timing_end(st);
  return e;
}

// ------------------------------------------------------------- small dim, D
// D for dim <= THIN_MAX_DIM, where the store of D is the whole cost (4 m bytes per row
// against 4 dim read).  The dimension is padded to DIM in {2, 4, 8, 16} with zeros
// (a zero term adds exactly nothing to any of the sums below), so every loop is unrolled.
// A block walks chunks of THIN_RB consecutive rows: the chunk's points arrive in shared
// memory with coalesced loads (the next chunk's are loaded into registers while the
// current one is formed), the centers sit in shared memory k-major (CsT[k][j]); each
// half-warp forms one row at a time, lane l the 4 columns 4 l .. 4 l + 3 of each
// 64-column pass, stored with one 16-byte store (256 contiguous bytes per half-warp).
// Every value is formed with the arithmetic of the tiled kernels above:
//   THIN_DIRECT  sum_k (p_k - c_k)^2, fused multiply-adds in k order (direct_kernel);
//   THIN_FORM    s = sum_k p_k c_k in k order, d = max((pp - 2 s) + cc, 0), pp the
//                row's fmaf norm in k order and cc the prepared center norm
//                (simt_dist_kernel, FM_F32), and with FLAG the cancellation test
//                d <= K (pp + cc): a flagged pair stores its direct distance in the REC
//                arithmetic here, and is counted (no list).
constexpr int THIN_MAX_DIM = 16;
constexpr int THIN_MAX_CF = 10240;  // m * padded dim floats of centers in shared memory (40 KB)
constexpr int THIN_RB = 128;       // rows per chunk
enum ThinMode { THIN_DIRECT = 0, THIN_FORM = 1 };

// DIM consecutive staged values of one row (16-byte loads where DIM allows)
template <int DIM>
__device__ __forceinline__ void ld_row(const float* src, float* v) {
  if constexpr (DIM % 4 == 0) {
#pragma unroll
    for (int k = 0; k < DIM; k += 4) {
      const float4 x = *reinterpret_cast<const float4*>(src + k);
      v[k] = x.x;
      v[k + 1] = x.y;
      v[k + 2] = x.z;
      v[k + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < DIM; k += 2) {
      const float2 x = *reinterpret_cast<const float2*>(src + k);
      v[k] = x.x;
      v[k + 1] = x.y;
    }
  }
}

// a flagged pair's direct distance from the staged row and the k-major center column
// (out of line: it is rare, and keeps the common path's registers free)
template <int DIM, int REC>
__device__ __noinline__ float thin_recompute(const float* prow, const float* ccol, int m) {
  DirectAcc<REC> r;
#pragma unroll
  for (int k = 0; k < DIM; ++k) r.add(prow[k], ccol[k * m]);
  return static_cast<float>(r.get());
}

template <int DIM, int MODE, bool FLAG, int REC>
__global__ void __launch_bounds__(256, 4) thin_d_kernel(const float* __restrict__ P, const float* __restrict__ C,
                                                        const float* __restrict__ cc, int64_t n, int m, int dim,
                                                        float kf, float* __restrict__ D,
                                                        unsigned long long* __restrict__ count) {
  constexpr int PER = THIN_RB * DIM / 256;  // a thread's share of a chunk's values, at most
  constexpr int R = DIM <= 8 ? 2 : 1;        // rows a half-warp forms together
  __shared__ __align__(16) float ps[THIN_RB * DIM];
  extern __shared__ __align__(16) float csT[];  // [DIM][m], rows dim .. DIM-1 zero
  for (int e = threadIdx.x; e < m * DIM; e += blockDim.x) {
    const int k = e / m, j = e % m;
    csT[e] = k < dim ? C[static_cast<int64_t>(j) * dim + k] : 0.f;
  }
  for (int e = threadIdx.x; e < THIN_RB * DIM; e += blockDim.x) ps[e] = 0.f;  // padding stays zero
  const int lane = threadIdx.x & 31, hl = lane & 15, hw = threadIdx.x >> 4;  // 16 half-warps
  const int64_t nchunk = (n + THIN_RB - 1) / THIN_RB;
  const int cvals = THIN_RB * dim;  // values of a whole chunk
  float pre[PER];
  auto load = [&](int64_t ch) {  // the chunk's values, coalesced (rows are contiguous)
    const int64_t base = ch * THIN_RB * dim, lim = n * dim;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = threadIdx.x + u * 256;
      pre[u] = (ch < nchunk && e < cvals && base + e < lim) ? __ldg(P + base + e) : 0.f;
    }
  };
  int64_t ch = blockIdx.x;
  load(ch);
  unsigned int flagged = 0;
  for (; ch < nchunk; ch += gridDim.x) {
    __syncthreads();  // the previous chunk is formed (the first time: centers and padding in)
    if (dim == DIM) {  // no padding: the chunk is a straight copy
#pragma unroll
      for (int u = 0; u < PER; ++u) ps[threadIdx.x + u * 256] = pre[u];
    } else {
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int e = threadIdx.x + u * 256;
        if (e < cvals) ps[(e / dim) * DIM + e % dim] = pre[u];
      }
    }
    __syncthreads();
    load(ch + gridDim.x);
    const int64_t row0 = ch * THIN_RB;
    const int nrows = static_cast<int>(n - row0 < THIN_RB ? n - row0 : THIN_RB);
    float* const dbase = D + row0 * m;
#pragma unroll 1
    for (int rr = hw; rr < THIN_RB; rr += 16 * R) {
      // R rows at a time (rr, rr + 16, ...): the centers' values are read once for all
      float p[R][DIM], pp[R];
      bool ok[R];
#pragma unroll
      for (int t = 0; t < R; ++t) {
        const int rt = rr + 16 * t;
        ok[t] = rt < nrows;
#pragma unroll
        for (int k = 0; k < DIM; k += 2) {
          const float2 v = *reinterpret_cast<const float2*>(ps + rt * DIM + k);
          p[t][k] = v.x;
          p[t][k + 1] = v.y;
        }
        pp[t] = 0.f;
        if constexpr (MODE == THIN_FORM) {
#pragma unroll
          for (int k = 0; k < DIM; ++k) pp[t] = __fmaf_rn(p[t][k], p[t][k], pp[t]);
        }
      }
      if (!ok[0]) break;
      // each row's values twice in a 64-bit pair, for the packed arithmetic below
      uint64_t pb[R][DIM];
#pragma unroll
      for (int t = 0; t < R; ++t)
#pragma unroll
        for (int k = 0; k < DIM; ++k) pb[t][k] = f2_pack(p[t][k], p[t][k]);
      for (int j0 = hl * 4; j0 < m; j0 += 64) {
        // four centers as two pairs (j0, j0+1), (j0+2, j0+3); every lane of a packed
        // operation is the scalar fused multiply-add / add of that pair, in the same order
        uint64_t acc[R][2];
#pragma unroll
        for (int t = 0; t < R; ++t) acc[t][0] = acc[t][1] = 0ull;
#pragma unroll
        for (int k = 0; k < DIM; ++k) {
          uint64_t c01, c23;
          lds_f2x2(csT + k * m + j0, c01, c23);
#pragma unroll
          for (int t = 0; t < R; ++t) {
            if constexpr (MODE == THIN_DIRECT) {
              const uint64_t d01 = f2_sub(pb[t][k], c01), d23 = f2_sub(pb[t][k], c23);
              acc[t][0] = f2_fma(d01, d01, acc[t][0]);
              acc[t][1] = f2_fma(d23, d23, acc[t][1]);
            } else {
              acc[t][0] = f2_fma(pb[t][k], c01, acc[t][0]);
              acc[t][1] = f2_fma(pb[t][k], c23, acc[t][1]);
            }
          }
        }
        uint64_t cc2[2] = {0ull, 0ull};
        if constexpr (MODE == THIN_FORM) {
          const float4 c4 = __ldg(reinterpret_cast<const float4*>(cc + j0));
          cc2[0] = f2_pack(c4.x, c4.y);
          cc2[1] = f2_pack(c4.z, c4.w);
        }
        uint32_t fmask = 0;  // flagged pairs (bit 4 t + c)
#pragma unroll
        for (int t = 0; t < R; ++t) {
          if (!ok[t]) continue;
          const int rt = rr + 16 * t;
          float v[4];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if constexpr (MODE == THIN_DIRECT) {
              f2_unpack(acc[t][h], v[2 * h], v[2 * h + 1]);
            } else {
              // d = max((pp - 2 s) + cc, 0) and the test d <= K (pp + cc), per lane
              const uint64_t pp2 = f2_pack(pp[t], pp[t]);
              const uint64_t e = f2_add(f2_fma(f2_pack(-2.f, -2.f), acc[t][h], pp2), cc2[h]);
              float d0, d1;
              f2_unpack(e, d0, d1);
              d0 = fmaxf(d0, 0.f);
              d1 = fmaxf(d1, 0.f);
              v[2 * h] = d0;
              v[2 * h + 1] = d1;
              if constexpr (FLAG) {
                float t0, t1;
                f2_unpack(f2_mul(f2_pack(kf, kf), f2_add(pp2, cc2[h])), t0, t1);
                fmask |= (static_cast<uint32_t>(d0 <= t0) << (4 * t + 2 * h)) |
                         (static_cast<uint32_t>(d1 <= t1) << (4 * t + 2 * h + 1));
              }
            }
          }
          *reinterpret_cast<float4*>(dbase + static_cast<int64_t>(rt) * m + j0) = make_float4(v[0], v[1], v[2], v[3]);
        }
        if constexpr (FLAG) {
          // flagged pairs (rare): their direct distance replaces the stored value
          while (fmask) {
            const int b = __ffs(fmask) - 1;
            fmask &= fmask - 1u;
            const int rt = rr + 16 * (b >> 2), c = b & 3;
            dbase[static_cast<int64_t>(rt) * m + j0 + c] = thin_recompute<DIM, REC>(ps + rt * DIM, csT + j0 + c, m);
            ++flagged;
          }
        }
      }
    }
  }
  if constexpr (FLAG) {
    const unsigned int tot = __reduce_add_sync(0xffffffffu, flagged);
    if (lane == 0 && tot) atomicAdd(count, static_cast<unsigned long long>(tot));
  }
}

// thin_d_kernel with the centers in registers (padded dim 8; the template takes 2 and 4
// too, where thin_d_kernel measured as fast or faster).  In thin_d_kernel every k step
// reads its four center values from shared memory for the 8 outputs a lane forms with
// them, and those loads fill the L1 data pipe before HBM is saturated.  Here the launch
// is cut into 64-column slices of D (block b takes slice b mod S of its chunks): lane l
// of each half-warp owns the columns 64 s + 4 l .. + 3 for the whole launch, with their
// DIM x 4 values as packed pairs (and their 4 norms) in registers, so a k step reads
// nothing from shared memory.  Warp w forms rows 16 w .. 16 w + 15 of each chunk, the two
// half-warps alternating (a warp's 16-byte stores cover two consecutive rows); lane l < 16
// forms the fmaf norm of row 16 w + l once per chunk and hands it on by shuffle.  The
// arithmetic is thin_d_kernel's, operation for operation, so D is bit-identical.
template <int DIM, int REC>
__device__ __noinline__ float thin_recompute_g(const float* prow, const float* __restrict__ crow, int dim) {
  DirectAcc<REC> r;
#pragma unroll
  for (int k = 0; k < DIM; ++k) r.add(prow[k], k < dim ? crow[k] : 0.f);
  return static_cast<float>(r.get());
}

template <int DIM, int MODE, bool FLAG, int REC>
__global__ void __launch_bounds__(256, 3) thin_dr_kernel(const float* __restrict__ P, const float* __restrict__ C,
                                                         const float* __restrict__ cc, int64_t n, int m, int dim,
                                                         float kf, float* __restrict__ D,
                                                         unsigned long long* __restrict__ count, int slices) {
  static_assert(DIM == 2 || DIM == 4 || DIM == 8, "register centers: dim <= 8");
  constexpr int PER = THIN_RB * DIM / 256;
  __shared__ __align__(16) float ps[THIN_RB * DIM];
  const int lane = threadIdx.x & 31, hl = lane & 15, h = lane >> 4, w = threadIdx.x >> 5;
  const int slice = static_cast<int>(blockIdx.x % slices);
  const int64_t cb = blockIdx.x / slices, nb = gridDim.x / slices;
  const int j0 = slice * 64 + hl * 4;
  const bool colok = j0 < m;  // m is a multiple of 4: a lane's columns are all in or all out
  uint64_t c01[DIM], c23[DIM];
#pragma unroll
  for (int k = 0; k < DIM; ++k) {
    float a[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) a[c] = colok && k < dim ? __ldg(C + static_cast<int64_t>(j0 + c) * dim + k) : 0.f;
    c01[k] = f2_pack(a[0], a[1]);
    c23[k] = f2_pack(a[2], a[3]);
  }
  uint64_t cc2[2] = {0ull, 0ull};
  if constexpr (MODE == THIN_FORM) {
    if (colok) {
      const float4 c4 = __ldg(reinterpret_cast<const float4*>(cc + j0));
      cc2[0] = f2_pack(c4.x, c4.y);
      cc2[1] = f2_pack(c4.z, c4.w);
    }
  }
  for (int e = threadIdx.x; e < THIN_RB * DIM; e += blockDim.x) ps[e] = 0.f;  // padding stays zero
  const int64_t nchunk = (n + THIN_RB - 1) / THIN_RB;
  const int cvals = THIN_RB * dim;
  float pre[PER];
  auto load = [&](int64_t ch) {
    const int64_t base = ch * THIN_RB * dim, lim = n * dim;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = threadIdx.x + u * 256;
      pre[u] = (ch < nchunk && e < cvals && base + e < lim) ? __ldg(P + base + e) : 0.f;
    }
  };
  int64_t ch = cb;
  load(ch);
  unsigned int flagged = 0;
  for (; ch < nchunk; ch += nb) {
    __syncthreads();
    if (dim == DIM) {
#pragma unroll
      for (int u = 0; u < PER; ++u) ps[threadIdx.x + u * 256] = pre[u];
    } else {
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int e = threadIdx.x + u * 256;
        if (e < cvals) ps[(e / dim) * DIM + e % dim] = pre[u];
      }
    }
    __syncthreads();
    load(ch + nb);
    const int64_t row0 = ch * THIN_RB;
    const int nrows = static_cast<int>(n - row0 < THIN_RB ? n - row0 : THIN_RB);  // rows of this chunk
    float* const dbase = D + row0 * m + j0;
    float q = 0.f;  // norm of row 16 w + (lane & 15), fmaf in k order
    if constexpr (MODE == THIN_FORM) {
      float pv[DIM];
      ld_row<DIM>(ps + (16 * w + hl) * DIM, pv);
#pragma unroll
      for (int k = 0; k < DIM; ++k) q = __fmaf_rn(pv[k], pv[k], q);
    }
#pragma unroll 2
    for (int i = 0; i < 8; ++i) {
      const int rt = 16 * w + 2 * i + h;
      float pp = 0.f;
      if constexpr (MODE == THIN_FORM) pp = __shfl_sync(0xffffffffu, q, 2 * i + h);
      // (a 32-bit row test and a row pointer off the chunk's base measured 6 % faster for
      // the form and 3 % slower for the direct sum, which keeps the 64-bit forms)
      if (!colok || (MODE == THIN_FORM ? rt >= nrows : row0 + rt >= n)) continue;
      float pv[DIM];
      ld_row<DIM>(ps + rt * DIM, pv);
      uint64_t acc0 = 0ull, acc1 = 0ull;
#pragma unroll
      for (int k = 0; k < DIM; ++k) {
        const uint64_t pk = f2_pack(pv[k], pv[k]);
        if constexpr (MODE == THIN_DIRECT) {
          const uint64_t d01 = f2_sub(pk, c01[k]), d23 = f2_sub(pk, c23[k]);
          acc0 = f2_fma(d01, d01, acc0);
          acc1 = f2_fma(d23, d23, acc1);
        } else {
          acc0 = f2_fma(pk, c01[k], acc0);
          acc1 = f2_fma(pk, c23[k], acc1);
        }
      }
      float v[4], t[4] = {0.f, 0.f, 0.f, 0.f};
      if constexpr (MODE == THIN_DIRECT) {
        f2_unpack(acc0, v[0], v[1]);
        f2_unpack(acc1, v[2], v[3]);
      } else {
        // d = max((pp - 2 s) + cc, 0) and the test threshold K (pp + cc), per lane
        const uint64_t pp2 = f2_pack(pp, pp), m2 = f2_pack(-2.f, -2.f);
        f2_unpack(f2_add(f2_fma(m2, acc0, pp2), cc2[0]), v[0], v[1]);
        f2_unpack(f2_add(f2_fma(m2, acc1, pp2), cc2[1]), v[2], v[3]);
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = fmaxf(v[c], 0.f);
        if constexpr (FLAG) {
          const uint64_t k2 = f2_pack(kf, kf);
          f2_unpack(f2_mul(k2, f2_add(pp2, cc2[0])), t[0], t[1]);
          f2_unpack(f2_mul(k2, f2_add(pp2, cc2[1])), t[2], t[3]);
        }
      }
      float* drow = MODE == THIN_FORM ? dbase + static_cast<int64_t>(rt) * m : D + (row0 + rt) * m + j0;
      *reinterpret_cast<float4*>(drow) = make_float4(v[0], v[1], v[2], v[3]);
      if constexpr (FLAG) {
        if ((v[0] <= t[0]) | (v[1] <= t[1]) | (v[2] <= t[2]) | (v[3] <= t[3])) {
          // flagged pairs (rare): their direct distance replaces the stored value
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (v[c] <= t[c]) {
              drow[c] = thin_recompute_g<DIM, REC>(ps + rt * DIM, C + static_cast<int64_t>(j0 + c) * dim, dim);
              ++flagged;
            }
          }
        }
      }
    }
  }
  if constexpr (FLAG) {
    const unsigned int tot = __reduce_add_sync(0xffffffffu, flagged);
    if (lane == 0 && tot) atomicAdd(count, static_cast<unsigned long long>(tot));
  }
}

// thin_dr_kernel's form for padded dim 16, where four columns' 16 values would take 64
// registers: lane l of a warp owns columns 64 s + 2 l, + 1 of its slice (16 packed pairs,
// 32 registers) and the warp forms one row of the slice at a time, the 32 lanes' 8-byte
// stores covering the row's 256 bytes.  Warp w takes rows 16 w .. 16 w + 15 of each
// chunk; lane l < 16 forms the fmaf norm of row 16 w + l once per chunk.  The
// arithmetic is thin_d_kernel's, operation for operation.
template <int DIM, int MODE, bool FLAG, int REC>
__global__ void __launch_bounds__(256, 3) thin_dr2_kernel(const float* __restrict__ P, const float* __restrict__ C,
                                                          const float* __restrict__ cc, int64_t n, int m, int dim,
                                                          float kf, float* __restrict__ D,
                                                          unsigned long long* __restrict__ count, int slices) {
  static_assert(DIM == 16, "two columns a lane: dim 16");
  constexpr int PER = THIN_RB * DIM / 256;
  __shared__ __align__(16) float ps[THIN_RB * DIM];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int slice = static_cast<int>(blockIdx.x % slices);
  const int64_t cb = blockIdx.x / slices, nb = gridDim.x / slices;
  const int j0 = slice * 64 + lane * 2;
  const bool colok = j0 < m;  // m is a multiple of 4: both columns are in or both out
  uint64_t c01[DIM];
#pragma unroll
  for (int k = 0; k < DIM; ++k) {
    const float a0 = colok && k < dim ? __ldg(C + static_cast<int64_t>(j0) * dim + k) : 0.f;
    const float a1 = colok && k < dim ? __ldg(C + static_cast<int64_t>(j0 + 1) * dim + k) : 0.f;
    c01[k] = f2_pack(a0, a1);
  }
  uint64_t cc2 = 0ull;
  if constexpr (MODE == THIN_FORM) {
    if (colok) {
      const float2 c2 = __ldg(reinterpret_cast<const float2*>(cc + j0));
      cc2 = f2_pack(c2.x, c2.y);
    }
  }
  for (int e = threadIdx.x; e < THIN_RB * DIM; e += blockDim.x) ps[e] = 0.f;  // padding stays zero
  const int64_t nchunk = (n + THIN_RB - 1) / THIN_RB;
  const int cvals = THIN_RB * dim;
  float pre[PER];
  auto load = [&](int64_t ch) {
    const int64_t base = ch * THIN_RB * dim, lim = n * dim;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = threadIdx.x + u * 256;
      pre[u] = (ch < nchunk && e < cvals && base + e < lim) ? __ldg(P + base + e) : 0.f;
    }
  };
  int64_t ch = cb;
  load(ch);
  unsigned int flagged = 0;
  for (; ch < nchunk; ch += nb) {
    __syncthreads();
    if (dim == DIM) {
#pragma unroll
      for (int u = 0; u < PER; ++u) ps[threadIdx.x + u * 256] = pre[u];
    } else {
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int e = threadIdx.x + u * 256;
        if (e < cvals) ps[(e / dim) * DIM + e % dim] = pre[u];
      }
    }
    __syncthreads();
    load(ch + nb);
    const int64_t row0 = ch * THIN_RB;
    const int nrows = static_cast<int>(n - row0 < THIN_RB ? n - row0 : THIN_RB);  // rows of this chunk
    float* const dbase = D + row0 * m + j0;
    float q = 0.f;  // norm of row 16 w + (lane & 15), fmaf in k order
    if constexpr (MODE == THIN_FORM) {
      float pv[DIM];
      ld_row<DIM>(ps + (16 * w + (lane & 15)) * DIM, pv);
#pragma unroll
      for (int k = 0; k < DIM; ++k) q = __fmaf_rn(pv[k], pv[k], q);
    }
#pragma unroll 2
    for (int i = 0; i < 16; ++i) {
      const int rt = 16 * w + i;
      float pp = 0.f;
      if constexpr (MODE == THIN_FORM) pp = __shfl_sync(0xffffffffu, q, i);
      if (!colok || rt >= nrows) continue;
      float pv[DIM];
      ld_row<DIM>(ps + rt * DIM, pv);
      uint64_t acc = 0ull;
#pragma unroll
      for (int k = 0; k < DIM; ++k) {
        const uint64_t pk = f2_pack(pv[k], pv[k]);
        if constexpr (MODE == THIN_DIRECT) {
          const uint64_t d01 = f2_sub(pk, c01[k]);
          acc = f2_fma(d01, d01, acc);
        } else {
          acc = f2_fma(pk, c01[k], acc);
        }
      }
      float v0, v1, t0 = 0.f, t1 = 0.f;
      if constexpr (MODE == THIN_DIRECT) {
        f2_unpack(acc, v0, v1);
      } else {
        // d = max((pp - 2 s) + cc, 0) and the test threshold K (pp + cc), per lane
        const uint64_t pp2 = f2_pack(pp, pp);
        f2_unpack(f2_add(f2_fma(f2_pack(-2.f, -2.f), acc, pp2), cc2), v0, v1);
        v0 = fmaxf(v0, 0.f);
        v1 = fmaxf(v1, 0.f);
        if constexpr (FLAG) f2_unpack(f2_mul(f2_pack(kf, kf), f2_add(pp2, cc2)), t0, t1);
      }
      float* drow = dbase + static_cast<int64_t>(rt) * m;
      *reinterpret_cast<float2*>(drow) = make_float2(v0, v1);
      if constexpr (FLAG) {
        if ((v0 <= t0) | (v1 <= t1)) {
          // flagged pairs (rare): their direct distance replaces the stored value
          if (v0 <= t0) {
            drow[0] = thin_recompute_g<DIM, REC>(ps + rt * DIM, C + static_cast<int64_t>(j0) * dim, dim);
            ++flagged;
          }
          if (v1 <= t1) {
            drow[1] = thin_recompute_g<DIM, REC>(ps + rt * DIM, C + static_cast<int64_t>(j0 + 1) * dim, dim);
            ++flagged;
          }
        }
      }
    }
  }
  if constexpr (FLAG) {
    const unsigned int tot = __reduce_add_sync(0xffffffffu, flagged);
    if (lane == 0 && tot) atomicAdd(count, static_cast<unsigned long long>(tot));
  }
}

// Whether thin_d_kernel serves this D-mode call: fp32 in and out, dim <= 16, m a multiple
// of 4 with the centers in 40 KB of shared memory, D 16-byte aligned.
bool thin_d_ok(const OpSpec* s, int64_t m, int dim, const void* D) {
  if (s->in != IN_F32 || s->out != OUT_F32 || D == nullptr) return false;
  if (dim < 1 || dim > THIN_MAX_DIM || m < 4 || (m & 3) != 0) return false;
  const int pd = dim <= 2 ? 2 : (dim <= 4 ? 4 : (dim <= 8 ? 8 : 16));
  if (m * pd > THIN_MAX_CF) return false;
  if ((reinterpret_cast<uintptr_t>(D) & 15u) != 0) return false;
  if (s->gemm == G_DIRECT) return true;
  // the fp32 form with fmaf norms: single, and the mix operators on an fp32 GEMM
  return s->gemm == G_SIMT_F32 && s->form == FM_F32 && s->norm == NM_F32_FMA &&
         (s->flag == FL_NONE || (s->flag == FL_F32 && (s->rec == RC_F32 || s->rec == RC_F64)));
}

cudaError_t launch_thin_d(const OpSpec* s, const void* P, const void* C, const void* cc, int64_t n, int64_t m,
                          int dim, float kf, void* D, unsigned long long* count, cudaStream_t st) {
  if (!thin_d_ok(s, m, dim, D)) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  const int64_t nchunk = (n + THIN_RB - 1) / THIN_RB;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(nchunk, num_sms() * 8)));
  const float* Pf = static_cast<const float*>(P);
  const float* Cf = static_cast<const float*>(C);
  const float* ccf = static_cast<const float*>(cc);
  float* Df = static_cast<float*>(D);
  const int mi = static_cast<int>(m);
  timing_begin(st, "thin_d_kernel");
  const int pd = dim <= 2 ? 2 : (dim <= 4 ? 4 : (dim <= 8 ? 8 : 16));
  const size_t smem = static_cast<size_t>(m) * pd * 4;
  // padded dim 8: centers in registers, one wave of 3 blocks per SM over the column slices
  // (at dim <= 4 the shared-memory form measured as fast or faster)
  const int slices = static_cast<int>((m + 63) / 64);
  const int64_t nbx = std::max<int64_t>(1, std::min<int64_t>(nchunk, (num_sms() * 3 + slices - 1) / slices));
  const int rblocks = static_cast<int>(nbx * slices);
#define THIN_RGO(DIM_)                                                                                        \
  if (pd == DIM_) {                                                                                           \
    if (s->gemm == G_DIRECT)                                                                                  \
      thin_dr_kernel<DIM_, THIN_DIRECT, false, RC_NONE><<<rblocks, 256, 0, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count, slices); \
    else if (s->flag == FL_NONE)                                                                              \
      thin_dr_kernel<DIM_, THIN_FORM, false, RC_NONE><<<rblocks, 256, 0, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count, slices);   \
    else if (s->rec == RC_F32)                                                                                \
      thin_dr_kernel<DIM_, THIN_FORM, true, RC_F32><<<rblocks, 256, 0, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count, slices);     \
    else                                                                                                      \
      thin_dr_kernel<DIM_, THIN_FORM, true, RC_F64><<<rblocks, 256, 0, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count, slices);     \
  }
#define THIN_R2GO(DIM_)                                                                                       \
  if (pd == DIM_) {                                                                                           \
    if (s->gemm == G_DIRECT)                                                                                  \
      thin_dr2_kernel<DIM_, THIN_DIRECT, false, RC_NONE><<<rblocks, 256, 0, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count, slices); \
    else if (s->flag == FL_NONE)                                                                              \
      thin_dr2_kernel<DIM_, THIN_FORM, false, RC_NONE><<<rblocks, 256, 0, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count, slices);   \
    else if (s->rec == RC_F32)                                                                                \
      thin_dr2_kernel<DIM_, THIN_FORM, true, RC_F32><<<rblocks, 256, 0, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count, slices);     \
    else                                                                                                      \
      thin_dr2_kernel<DIM_, THIN_FORM, true, RC_F64><<<rblocks, 256, 0, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count, slices);     \
  }
#define THIN_GO(DIM_)                                                                                         \
  if (pd == DIM_) {                                                                                           \
    if (s->gemm == G_DIRECT)                                                                                  \
      thin_d_kernel<DIM_, THIN_DIRECT, false, RC_NONE><<<blocks, 256, smem, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count); \
    else if (s->flag == FL_NONE)                                                                              \
      thin_d_kernel<DIM_, THIN_FORM, false, RC_NONE><<<blocks, 256, smem, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count);   \
    else if (s->rec == RC_F32)                                                                                \
      thin_d_kernel<DIM_, THIN_FORM, true, RC_F32><<<blocks, 256, smem, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count);     \
    else                                                                                                      \
      thin_d_kernel<DIM_, THIN_FORM, true, RC_F64><<<blocks, 256, smem, st>>>(Pf, Cf, ccf, n, mi, dim, kf, Df, count);     \
  }
  THIN_GO(2)
  THIN_GO(4)
  THIN_RGO(8)
  THIN_R2GO(16)
#undef THIN_GO
#undef THIN_RGO
#undef THIN_R2GO
  cudaError_t e = cudaGetLastError();
  timing_end(st);
  return e;
}

cudaError_t launch_direct(const OpSpec* s, const void* P, const void* C, int64_t n, int64_t m, int dim, void* D,
                          cudaStream_t st) {
  if (thin_d_ok(s, m, dim, D)) return launch_thin_d(s, P, C, nullptr, n, m, dim, 0.f, D, nullptr, st);
  switch (s->in) {
    case IN_F16: return go_direct<__half, float, __half>(P, C, n, m, dim, D, st);
    case IN_BF16: return go_direct<__nv_bfloat16, float, __nv_bfloat16>(P, C, n, m, dim, D, st);
    case IN_F32: return go_direct<float, float, float>(P, C, n, m, dim, D, st);
    case IN_F64: return go_direct<double, double, double>(P, C, n, m, dim, D, st);
  }
  return cudaErrorNotSupported;
}

}  // namespace euc
