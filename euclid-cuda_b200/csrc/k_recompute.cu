// Selective recompute of the pairs flagged by the cancellation test, as a compacted
// second pass (the reference launches N*M threads and lets all but `count` exit,
// euclidean_kernels_mix.cu:573-578; here the grid is sized to the machine and walks
// only the list).
//
// D mode    : D[i, j] = direct(i, j) for every listed pair.  If more pairs were flagged
//             than the list holds, the kernel instead sweeps all of D and re-derives
//             the flag from the stored distance and norms (bit-identical test), so no
//             flagged pair is ever lost.
// argmin mode: row_key[i] = min(row_key[i], (direct(i, j), j)) with a 64-bit atomicMin;
//             the distance epilogue already recomputed in place whatever did not fit.
#include "common.cuh"
#include "engine.h"
#include "direct.cuh"

#include <type_traits>

namespace euc {

struct RecArgs {
  const void* P;
  const void* C;
  int64_t n, m;
  int dim;
  const unsigned long long* list;
  const unsigned long long* count;
  unsigned long long cap;
  void* D;
  unsigned long long* row_key;
  const void* pp;
  const void* cc;
  float kf;
  double kd;
};

template <typename TIN, int REC, typename TOUT, int FLAG, bool ARGMIN>
__global__ void __launch_bounds__(256) recompute_kernel(const RecArgs a) {
  const TIN* P = static_cast<const TIN*>(a.P);
  const TIN* C = static_cast<const TIN*>(a.C);
  const unsigned long long cnt = *a.count;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  const uint64_t t0 = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  // argmin: the listed pairs always go through here (the distance epilogue folded the
  // ones beyond the list's capacity in place); D: an overflowing list is ignored and
  // the dense sweep below recomputes every flagged pair instead
  if (ARGMIN || cnt <= a.cap) {
    const unsigned long long nlist = cnt < a.cap ? cnt : a.cap;
    for (uint64_t t = t0; t < nlist; t += stride) {
      const unsigned long long e = a.list[t];
      const int64_t i = static_cast<int64_t>(e >> 32);
      const int64_t j = static_cast<int64_t>(e & 0xffffffffull);
      if (i >= a.n || j >= a.m) continue;
      const double v = direct_dist<TIN, REC>(P + i * a.dim, C + j * a.dim, a.dim);
      if constexpr (ARGMIN) {
        atomicMin(&a.row_key[i], make_key(static_cast<float>(v), static_cast<uint32_t>(j)));
      } else {
        static_cast<TOUT*>(a.D)[i * a.m + j] = static_cast<TOUT>(v);
      }
    }
  } else if constexpr (!ARGMIN && REC != RC_F32 && REC != RC_F64) {
    // overflow: dense sweep, flag re-derived from the stored (pre-recompute) distance
    // (fp32 and fp64 recomputes take recompute_dense_tiled_kernel instead)
    const uint64_t total = static_cast<uint64_t>(a.n) * static_cast<uint64_t>(a.m);
    for (uint64_t t = t0; t < total; t += stride) {
      const int64_t i = static_cast<int64_t>(t / static_cast<uint64_t>(a.m));
      const int64_t j = static_cast<int64_t>(t % static_cast<uint64_t>(a.m));
      TOUT* dp = static_cast<TOUT*>(a.D) + t;
      bool flag;
      if constexpr (FLAG == FL_F32) {
        const float pp = static_cast<const float*>(a.pp)[i], cc = static_cast<const float*>(a.cc)[j];
        flag = static_cast<float>(*dp) <= __fmul_rn(a.kf, __fadd_rn(pp, cc));
      } else {
        const double pp = static_cast<const double*>(a.pp)[i], cc = static_cast<const double*>(a.cc)[j];
        flag = static_cast<double>(*dp) <= a.kd * (pp + cc);
      }
      if (flag) *dp = static_cast<TOUT>(direct_dist<TIN, REC>(P + i * a.dim, C + j * a.dim, a.dim));
    }
  }
}

// Argmin mode with fp32 inputs, warp-cooperative: a warp takes 32 listed pairs and
// stages their P and C rows through shared memory 32 dimensions at a time with coalesced
// (16-byte) loads, all of a slab's loads in flight together; each lane then runs its
// pair's sum in the same arithmetic and the same k order as direct_dist.
constexpr int RW_WARPS = 4;
constexpr int RW_K = 32;

template <int REC>
__global__ void __launch_bounds__(RW_WARPS * 32, 4) recompute_argmin_rows_kernel(const RecArgs a) {
  __shared__ float sp[RW_WARPS][32][RW_K + 1];
  __shared__ float sc[RW_WARPS][32][RW_K + 1];
  const float* P = static_cast<const float*>(a.P);
  const float* C = static_cast<const float*>(a.C);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const unsigned long long cnt = *a.count;
  const unsigned long long nlist = cnt < a.cap ? cnt : a.cap;
  const int dim = a.dim;
  const bool vec = (dim % 4 == 0) && ((reinterpret_cast<uintptr_t>(P) | reinterpret_cast<uintptr_t>(C)) % 16 == 0);
  const uint64_t gw = static_cast<uint64_t>(blockIdx.x) * RW_WARPS + w;
  const uint64_t nw = static_cast<uint64_t>(gridDim.x) * RW_WARPS;
  for (uint64_t base = gw * 32; base < nlist; base += nw * 32) {
    const uint64_t t = base + lane;
    bool valid = t < nlist;
    const unsigned long long e = valid ? a.list[t] : 0ull;
    const long long i = static_cast<long long>(e >> 32);
    const long long j = static_cast<long long>(e & 0xffffffffull);
    valid = valid && i < a.n && j < a.m;
    DirectAcc<REC> acc;
    for (int k0 = 0; k0 < dim; k0 += RW_K) {
      const int kn = min(RW_K, dim - k0);
      if (vec) {
        const int quarter = lane >> 3, c4 = (lane & 7) * 4;  // 8 lanes x 16 bytes per row slab
#pragma unroll
        for (int rr = 0; rr < 32; rr += 4) {
          const int r = rr + quarter;
          const long long ir = __shfl_sync(0xffffffffu, i, r);
          const long long jr = __shfl_sync(0xffffffffu, j, r);
          const bool vr = __shfl_sync(0xffffffffu, valid, r);
          float4 pv = make_float4(0.f, 0.f, 0.f, 0.f), cv = pv;
          if (vr && c4 < kn) {
            pv = __ldg(reinterpret_cast<const float4*>(P + ir * dim + k0 + c4));
            cv = __ldg(reinterpret_cast<const float4*>(C + jr * dim + k0 + c4));
          }
          float* dp = &sp[w][r][c4];
          float* dc = &sc[w][r][c4];
          dp[0] = pv.x; dp[1] = pv.y; dp[2] = pv.z; dp[3] = pv.w;
          dc[0] = cv.x; dc[1] = cv.y; dc[2] = cv.z; dc[3] = cv.w;
        }
      } else {
        for (int r = 0; r < 32; ++r) {
          const long long ir = __shfl_sync(0xffffffffu, i, r);
          const long long jr = __shfl_sync(0xffffffffu, j, r);
          const bool vr = __shfl_sync(0xffffffffu, valid, r);
          for (int c = lane; c < kn; c += 32) {
            sp[w][r][c] = vr ? __ldg(P + ir * dim + k0 + c) : 0.f;
            sc[w][r][c] = vr ? __ldg(C + jr * dim + k0 + c) : 0.f;
          }
        }
      }
      __syncwarp();
      for (int kk = 0; kk < kn; ++kk) acc.add(sp[w][lane][kk], sc[w][lane][kk]);
      __syncwarp();
    }
    if (valid) atomicMin(&a.row_key[i], make_key(static_cast<float>(acc.get()), static_cast<uint32_t>(j)));
  }
}

// D mode, list overflowed (more flagged pairs than it holds), fp32 or fp64 recompute:
// every flagged pair recomputed by tiles.  A block takes 64 x 64 tiles of D (grid-stride);
// each thread re-derives the flags of its 4 x 4 elements from the stored distance and
// the norms (the test of the distance kernel, bit-identical), a tile without a flag is
// skipped, and otherwise the rows and centers are staged through shared memory 16
// dimensions at a time and every element's direct sum is formed in the operator's
// arithmetic and dimension order (direct_dist); flagged elements are stored.  The
// kernel returns at once when the list held every flagged pair.
constexpr int RT_B = 64, RT_K = 16;
constexpr int RT_LD = RT_B + 4;  // shared row stride: 16-byte aligned rows, staggered banks

// four consecutive shared values (16-byte aligned) into registers: one 16-byte load for
// fp32, two for fp64
template <typename T>
__device__ __forceinline__ void rt_lds4(const T* p, T (&v)[4]) {
  if constexpr (sizeof(T) == 4) {
    const float4 q = *reinterpret_cast<const float4*>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  } else {
    const double2 q0 = *reinterpret_cast<const double2*>(p), q1 = *reinterpret_cast<const double2*>(p + 2);
    v[0] = q0.x; v[1] = q0.y; v[2] = q1.x; v[3] = q1.y;
  }
}

template <typename TIN, int REC, typename TOUT, int FLAG>
__global__ void __launch_bounds__(256) recompute_dense_tiled_kernel(const RecArgs a) {
  using TACC = typename std::conditional<REC == RC_F64, double, float>::type;
  if (*a.count <= a.cap) return;  // the list path has done it
  __shared__ __align__(16) TACC As[RT_K][RT_LD];
  __shared__ __align__(16) TACC Bs[RT_K][RT_LD];
  const TIN* P = static_cast<const TIN*>(a.P);
  const TIN* C = static_cast<const TIN*>(a.C);
  TOUT* D = static_cast<TOUT*>(a.D);
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t nrt = (a.n + RT_B - 1) / RT_B, nct = (a.m + RT_B - 1) / RT_B;
  // fp32 rows with dim % 4 == 0 on 16-byte boundaries stage 4 dimensions per load
  bool vec = false;
  if constexpr (std::is_same<TIN, float>::value)
    vec = (a.dim % 4 == 0) && ((reinterpret_cast<uintptr_t>(P) | reinterpret_cast<uintptr_t>(C)) % 16 == 0);
  for (int64_t tile = blockIdx.x; tile < nrt * nct; tile += gridDim.x) {
    const int64_t row0 = (tile / nct) * RT_B, col0 = (tile % nct) * RT_B;
    uint32_t fmask = 0;  // bit 4 r + c: element (row0 + 4 ty + r, col0 + 4 tx + c) is flagged
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int64_t i = row0 + ty * 4 + r;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int64_t j = col0 + tx * 4 + c;
        if (i >= a.n || j >= a.m) continue;
        bool flag;
        if constexpr (FLAG == FL_F32) {
          const float pp = static_cast<const float*>(a.pp)[i], cc = static_cast<const float*>(a.cc)[j];
          flag = static_cast<float>(D[i * a.m + j]) <= __fmul_rn(a.kf, __fadd_rn(pp, cc));
        } else {
          const double pp = static_cast<const double*>(a.pp)[i], cc = static_cast<const double*>(a.cc)[j];
          flag = static_cast<double>(D[i * a.m + j]) <= a.kd * (pp + cc);
        }
        fmask |= static_cast<uint32_t>(flag) << (4 * r + c);
      }
    }
    if (!__syncthreads_or(fmask != 0)) continue;  // block-uniform
    TACC acc[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[r][c] = 0;
    uint64_t acc2[4][2];  // fp32: (columns 2h, 2h + 1) of row r
#pragma unroll
    for (int r = 0; r < 4; ++r) acc2[r][0] = acc2[r][1] = 0ull;
    // fp32 rows with dim % 4 == 0 on 16-byte boundaries: thread t holds dimensions
    // k0 + 4 (t % 4) .. + 3 of row / center t / 4 (a quad is whole or past the end),
    // fetched one slab ahead so that the loads are in flight while a slab is formed
    float4 pvn = make_float4(0.f, 0.f, 0.f, 0.f), cvn = pvn;
    auto fetch = [&](int k0) {
      if constexpr (std::is_same<TIN, float>::value) {
        const int rr = threadIdx.x >> 2, k4 = (threadIdx.x & 3) * 4;
        const int64_t gi = row0 + rr, gj = col0 + rr;
        const int gk = k0 + k4;
        pvn = make_float4(0.f, 0.f, 0.f, 0.f);
        cvn = pvn;
        if (gk < a.dim) {
          if (gi < a.n) pvn = __ldg(reinterpret_cast<const float4*>(P + gi * a.dim + gk));
          if (gj < a.m) cvn = __ldg(reinterpret_cast<const float4*>(C + gj * a.dim + gk));
        }
      }
    };
    if (vec) fetch(0);
    for (int k0 = 0; k0 < a.dim; k0 += RT_K) {
      if constexpr (std::is_same<TIN, float>::value) {
        if (vec) {
          const int rr = threadIdx.x >> 2, k4 = (threadIdx.x & 3) * 4;
          const float pq[4] = {pvn.x, pvn.y, pvn.z, pvn.w}, cq[4] = {cvn.x, cvn.y, cvn.z, cvn.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            As[k4 + q][rr] = static_cast<TACC>(pq[q]);
            Bs[k4 + q][rr] = static_cast<TACC>(cq[q]);
          }
          if (k0 + RT_K < a.dim) fetch(k0 + RT_K);
        }
      }
      for (int t = threadIdx.x; !vec && t < RT_B * RT_K; t += 256) {
        const int rr = t / RT_K, kk = t % RT_K;
        const int64_t gi = row0 + rr, gj = col0 + rr;
        const int gk = k0 + kk;
        TACC pv = 0, cv = 0;
        if (gk < a.dim) {
          if constexpr (REC == RC_F64) {
            if (gi < a.n) pv = wide(P[gi * a.dim + gk]);
            if (gj < a.m) cv = wide(C[gj * a.dim + gk]);
          } else {
            if (gi < a.n) pv = narrow(P[gi * a.dim + gk]);
            if (gj < a.m) cv = narrow(C[gj * a.dim + gk]);
          }
        }
        As[kk][rr] = pv;
        Bs[kk][rr] = cv;
      }
      __syncthreads();
      const int kend = min(RT_K, a.dim - k0);  // padded dimensions must not add a term
      if constexpr (REC == RC_F32) {
        // fp32: columns in pairs on packed arithmetic, each lane the scalar __fsub_rn /
        // __fmaf_rn of its pair in k order (the same bits as the loop below)
        for (int kk = 0; kk < kend; ++kk) {
          float av[4];
          rt_lds4(&As[kk][ty * 4], av);
          uint64_t b01, b23;
          lds_f2x2(&Bs[kk][tx * 4], b01, b23);
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint64_t ar = f2_pack(av[r], av[r]);
            const uint64_t d01 = f2_sub(ar, b01), d23 = f2_sub(ar, b23);
            acc2[r][0] = f2_fma(d01, d01, acc2[r][0]);
            acc2[r][1] = f2_fma(d23, d23, acc2[r][1]);
          }
        }
      } else {
        for (int kk = 0; kk < kend; ++kk) {
          TACC av[4], bv[4];
          rt_lds4(&As[kk][ty * 4], av);
          rt_lds4(&Bs[kk][tx * 4], bv);
#pragma unroll
          for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              if constexpr (REC == RC_F64) {
                const double d = av[r] - bv[c];
                acc[r][c] = fma(d, d, acc[r][c]);
              } else {
                const float d = __fsub_rn(av[r], bv[c]);
                acc[r][c] = __fmaf_rn(d, d, acc[r][c]);
              }
            }
        }
      }
      __syncthreads();
    }
    if constexpr (REC == RC_F32) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float lo, hi;
        f2_unpack(acc2[r][0], lo, hi);
        acc[r][0] = lo;
        acc[r][1] = hi;
        f2_unpack(acc2[r][1], lo, hi);
        acc[r][2] = lo;
        acc[r][3] = hi;
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if ((fmask >> (4 * r + c)) & 1u)
          D[(row0 + ty * 4 + r) * a.m + col0 + tx * 4 + c] = static_cast<TOUT>(static_cast<double>(acc[r][c]));
  }
}

// All-flagged argmin over few centers: every pair is flagged (the range test of the
// all-flagged route), so the label is the first index of the smallest direct distance
// over all m centers.  With few centers the certified screen's bounds separate
// nothing, and it would evaluate every group after two screens; here each block takes
// 64-row tiles and sweeps all center tiles with recompute_dense_tiled_kernel's staging
// and arithmetic (fp32: packed lanes, each the scalar __fsub_rn / __fmaf_rn in k order;
// fp64: fma in k order), keeping per thread the first-index minimum of its 4 rows over
// its columns in increasing order; the 16 threads of a row then take the (distance,
// index) minimum by shuffle.  The minimum is taken over the certified path's keys, the
// distance as the operator stores it (rounded to fp32) above the center index, so the
// outputs are the certified argmin's for any input (fp64 values that round alike tie
// and the first index wins; NaN distances sort last).
template <int REC>
__global__ void __launch_bounds__(256) dense_argmin_kernel(const float* __restrict__ P, const float* __restrict__ C,
                                                           int64_t n, int64_t m, int dim, int64_t* __restrict__ labels,
                                                           int32_t* __restrict__ labels32, float* __restrict__ md) {
  using TACC = typename std::conditional<REC == RC_F64, double, float>::type;
  __shared__ __align__(16) TACC As[RT_K][RT_LD];
  __shared__ __align__(16) TACC Bs[RT_K][RT_LD];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t nrt = (n + RT_B - 1) / RT_B, nct = (m + RT_B - 1) / RT_B;
  const bool vec = (dim % 4 == 0) && ((reinterpret_cast<uintptr_t>(P) | reinterpret_cast<uintptr_t>(C)) % 16 == 0);
  for (int64_t rtile = blockIdx.x; rtile < nrt; rtile += gridDim.x) {
    const int64_t row0 = rtile * RT_B;
    unsigned long long bk[4] = {~0ull, ~0ull, ~0ull, ~0ull};
    for (int64_t ct = 0; ct < nct; ++ct) {
      const int64_t col0 = ct * RT_B;
      TACC acc[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0;
      uint64_t acc2[4][2];  // fp32: (columns 2h, 2h + 1) of row r
#pragma unroll
      for (int r = 0; r < 4; ++r) acc2[r][0] = acc2[r][1] = 0ull;
      // the 16-byte staging fetches one slab ahead (as in recompute_dense_tiled_kernel)
      float4 pvn = make_float4(0.f, 0.f, 0.f, 0.f), cvn = pvn;
      auto fetch = [&](int k0) {
        const int rr = threadIdx.x >> 2, k4 = (threadIdx.x & 3) * 4;
        const int64_t gi = row0 + rr, gj = col0 + rr;
        const int gk = k0 + k4;
        pvn = make_float4(0.f, 0.f, 0.f, 0.f);
        cvn = pvn;
        if (gk < dim) {
          if (gi < n) pvn = __ldg(reinterpret_cast<const float4*>(P + gi * dim + gk));
          if (gj < m) cvn = __ldg(reinterpret_cast<const float4*>(C + gj * dim + gk));
        }
      };
      if (vec) fetch(0);
      for (int k0 = 0; k0 < dim; k0 += RT_K) {
        if (vec) {
          const int rr = threadIdx.x >> 2, k4 = (threadIdx.x & 3) * 4;
          const float pq[4] = {pvn.x, pvn.y, pvn.z, pvn.w}, cq[4] = {cvn.x, cvn.y, cvn.z, cvn.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            As[k4 + q][rr] = static_cast<TACC>(pq[q]);
            Bs[k4 + q][rr] = static_cast<TACC>(cq[q]);
          }
          if (k0 + RT_K < dim) fetch(k0 + RT_K);
        } else {
          for (int t = threadIdx.x; t < RT_B * RT_K; t += 256) {
            const int rr = t / RT_K, kk = t % RT_K;
            const int64_t gi = row0 + rr, gj = col0 + rr;
            const int gk = k0 + kk;
            TACC pv = 0, cv = 0;
            if (gk < dim) {
              if (gi < n) pv = static_cast<TACC>(P[gi * dim + gk]);
              if (gj < m) cv = static_cast<TACC>(C[gj * dim + gk]);
            }
            As[kk][rr] = pv;
            Bs[kk][rr] = cv;
          }
        }
        __syncthreads();
        const int kend = min(RT_K, dim - k0);  // padded dimensions must not add a term
        if constexpr (REC == RC_F32) {
          for (int kk = 0; kk < kend; ++kk) {
            float av[4];
            rt_lds4(&As[kk][ty * 4], av);
            uint64_t b01, b23;
            lds_f2x2(&Bs[kk][tx * 4], b01, b23);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const uint64_t ar = f2_pack(av[r], av[r]);
              const uint64_t d01 = f2_sub(ar, b01), d23 = f2_sub(ar, b23);
              acc2[r][0] = f2_fma(d01, d01, acc2[r][0]);
              acc2[r][1] = f2_fma(d23, d23, acc2[r][1]);
            }
          }
        } else {
          for (int kk = 0; kk < kend; ++kk) {
            double av[4], bw[4];
            rt_lds4(&As[kk][ty * 4], av);
            rt_lds4(&Bs[kk][tx * 4], bw);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                const double d = av[r] - bw[c];
                acc[r][c] = fma(d, d, acc[r][c]);
              }
          }
        }
        __syncthreads();
      }
      if constexpr (REC == RC_F32) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          f2_unpack(acc2[r][0], acc[r][0], acc[r][1]);
          f2_unpack(acc2[r][1], acc[r][2], acc[r][3]);
        }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int64_t j = col0 + tx * 4 + c;
          if (j < m) {
            const unsigned long long key = make_key(static_cast<float>(acc[r][c]), static_cast<uint32_t>(j));
            bk[r] = key < bk[r] ? key : bk[r];
          }
        }
    }
    // the row's 16 threads: (distance, index) minimum
#pragma unroll
    for (int r = 0; r < 4; ++r) {
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, bk[r], o);
        bk[r] = other < bk[r] ? other : bk[r];
      }
      const int64_t i = row0 + ty * 4 + r;
      if (tx == 0 && i < n) {
        const uint32_t j = static_cast<uint32_t>(bk[r] & 0xffffffffull);
        if (labels) labels[i] = static_cast<int64_t>(j);
        if (labels32) labels32[i] = static_cast<int32_t>(j);
        if (md) md[i] = __uint_as_float(static_cast<uint32_t>(bk[r] >> 32));
      }
    }
  }
}

cudaError_t launch_dense_argmin(const OpSpec* s, const void* P, const void* C, int64_t n, int64_t m, int dim,
                                int64_t* labels, int32_t* labels32, float* md, cudaStream_t st) {
  const int64_t nrt = (n + RT_B - 1) / RT_B;
  if (nrt == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(nrt, 0x7fffffff));
  const float* Pf = static_cast<const float*>(P);
  const float* Cf = static_cast<const float*>(C);
  if (s->rec != RC_F64 && s->rec != RC_F32) return cudaErrorNotSupported;
  timing_begin(st, "dense_argmin_kernel");
  if (s->rec == RC_F64)
    dense_argmin_kernel<RC_F64><<<blocks, 256, 0, st>>>(Pf, Cf, n, m, dim, labels, labels32, md);
  else
    dense_argmin_kernel<RC_F32><<<blocks, 256, 0, st>>>(Pf, Cf, n, m, dim, labels, labels32, md);
  cudaError_t e = cudaGetLastError();
  timing_end(st);
  return e;
}

template <typename TIN, int REC, typename TOUT, int FLAG, bool ARGMIN>
static cudaError_t go_rec(const DistJob& j) {
  RecArgs a{};
  a.P = j.P;
  a.C = j.C;
  a.n = j.n;
  a.m = j.m;
  a.dim = j.dim;
  a.list = j.list;
  a.count = j.count;
  a.cap = j.list_cap;
  a.D = j.D;
  a.row_key = j.row_key;
  a.pp = j.pp;
  a.cc = j.cc;
  a.kf = j.kf;
  a.kd = j.kd;
  if constexpr (ARGMIN && std::is_same<TIN, float>::value) {
    // one full wave: the kernel walks the list grid-stride, and a second, partial wave
    // of equal-work blocks would leave most SMs idle at the end
    static int per_sm = 0;
    if (per_sm == 0) {
      int v = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, recompute_argmin_rows_kernel<REC>, RW_WARPS * 32, 0) !=
              cudaSuccess || v < 1)
        v = 4;
      per_sm = v;
    }
    recompute_argmin_rows_kernel<REC><<<num_sms() * per_sm, RW_WARPS * 32, 0, j.stream>>>(a);
    return cudaGetLastError();
  }
  const int blocks = num_sms() * 8;
  recompute_kernel<TIN, REC, TOUT, FLAG, ARGMIN><<<blocks, 256, 0, j.stream>>>(a);
  if constexpr (!ARGMIN && (REC == RC_F32 || REC == RC_F64))
    recompute_dense_tiled_kernel<TIN, REC, TOUT, FLAG><<<blocks, 256, 0, j.stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_recompute(const DistJob& j) {
  const OpSpec* s = j.spec;
  if (s->flag == FL_NONE) return cudaSuccess;
  const bool argmin = (j.D == nullptr);
#define REC_CASE(IN_, TIN_, REC_, OUT_, TOUT_, FLAG_)                                                    \
  if (s->in == IN_ && s->rec == REC_ && s->flag == FLAG_ && (argmin || s->out == OUT_)) {                \
    if (argmin) return go_rec<TIN_, REC_, TOUT_, FLAG_, true>(j);                                        \
    return go_rec<TIN_, REC_, TOUT_, FLAG_, false>(j);                                                   \
  }
  REC_CASE(IN_F32, float, RC_F64, OUT_F32, float, FL_F32)
  REC_CASE(IN_F32, float, RC_F32, OUT_F32, float, FL_F32)
  REC_CASE(IN_F32, float, RC_F16_ARITH, OUT_F32, float, FL_F32)
  REC_CASE(IN_F32, float, RC_BF16_ARITH, OUT_F32, float, FL_F32)
  if (!argmin) {
    REC_CASE(IN_F16, __half, RC_F64, OUT_F32, float, FL_F32)
    REC_CASE(IN_BF16, __nv_bfloat16, RC_F64, OUT_F32, float, FL_F32)
    REC_CASE(IN_F32, float, RC_F64, OUT_F64, double, FL_F64)
    REC_CASE(IN_F64, double, RC_F64, OUT_F64, double, FL_F64)
  }
#undef REC_CASE
  return cudaErrorNotSupported;
}

// ------------------------------------------------------------------ helpers

__global__ void keys_to_labels_kernel(const unsigned long long* __restrict__ keys, int64_t n,
                                      int64_t* __restrict__ labels, int32_t* __restrict__ labels32,
                                      float* __restrict__ mind) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long k = keys[i];
    const uint32_t j = static_cast<uint32_t>(k & 0xffffffffull);
    if (labels) labels[i] = j;
    if (labels32) labels32[i] = static_cast<int32_t>(j);
    if (mind) mind[i] = __uint_as_float(static_cast<uint32_t>(k >> 32));
  }
}

cudaError_t launch_keys_to_labels(const unsigned long long* keys, int64_t n, int64_t* labels, int32_t* labels32,
                                  float* mind, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, num_sms() * 16));
  keys_to_labels_kernel<<<blocks, 256, 0, st>>>(keys, n, labels, labels32, mind);
  return cudaGetLastError();
}

__global__ void idx_to_labels_kernel(const long long* __restrict__ idx, int64_t n, int64_t* __restrict__ labels,
                                     int32_t* __restrict__ labels32) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (labels) labels[i] = idx[i];
    if (labels32) labels32[i] = static_cast<int32_t>(idx[i]);
  }
}

cudaError_t launch_f64_to_labels(const long long* idx, int64_t n, int64_t* labels, int32_t* labels32,
                                 cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, num_sms() * 16));
  idx_to_labels_kernel<<<blocks, 256, 0, st>>>(idx, n, labels, labels32);
  return cudaGetLastError();
}

__global__ void fill_u64_kernel(unsigned long long* p, int64_t n, unsigned long long v) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = v;
}

cudaError_t launch_fill_u64(unsigned long long* p, int64_t n, unsigned long long v, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, num_sms() * 16));
  fill_u64_kernel<<<blocks, 256, 0, st>>>(p, n, v);
  return cudaGetLastError();
}

}  // namespace euc
