// k-means++ seeding on the device, deterministic (the caller-side step before the Lloyd
// loop; the reference leaves it to the caller).
//
// Draw s of a run uses r_s = the top 53 bits of splitmix64(seed + (s + 1) * golden gamma)
// (the published SplitMix64 finaliser), a uniform integer in [0, 2^53).
//   * center 0 is row floor(r_0 * n / 2^53);
//   * for s >= 1, D[i] = min over chosen centers of |x_i - c|^2 (the direct fp64 sum in
//     dimension order, as the fp64 recompute forms it), and row i is chosen with
//     probability D[i] / sum D: the weights are turned into exact integers
//     q_i = floor(D[i] 2^S), S = 62 - ceil(log2 n) - (floor(log2 max D) + 1), so that
//     their sum fits 62 bits and every sum is order-independent; target
//     t = floor(r_s * sum q / 2^53) (exact 128-bit product) and the chosen row is the
//     first i whose running sum of q exceeds t.  If every weight is 0 the draw is
//     uniform over the rows, as for center 0.
// Three launches per center: update D (and its max), block sums of q, select.
#include "common.cuh"
#include "engine.h"

#include <algorithm>

namespace euc {

constexpr int SD_BLOCK = 1024;  // rows per q block

__host__ __device__ __forceinline__ uint64_t seed_draw53(uint64_t seed, uint64_t s) {
  uint64_t z = seed + (s + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return z >> 11;
}

// floor(r * v / 2^53) for r < 2^53, v < 2^63
__device__ __forceinline__ uint64_t scale53(uint64_t r, uint64_t v) {
  const uint64_t lo = r * v, hi = __umul64hi(r, v);
  return (hi << 11) | (lo >> 53);
}

__device__ __forceinline__ int q_shift(double maxd, int64_t n) {
  int l = 0;
  while ((1ll << l) < n) ++l;  // ceil(log2 n)
  return 62 - l - (ilogb(maxd) + 1);
}

__device__ __forceinline__ uint64_t q_of(double d, int S) { return __double2ull_rz(ldexp(d, S)); }

// D[i] <- (first ? |x_i - c|^2 : min(D[i], |x_i - c|^2)), c = row idx[s - 1]; the max of D
// into *maxbits (non-negative doubles order as their bit patterns).  A NaN distance
// counts as 0.  A warp takes 32 consecutive rows and stages them through shared memory
// 128 bytes of each row at a time (coalesced loads); lane r then continues row r's sum
// in dimension order.
template <typename TX>
__global__ void __launch_bounds__(256) seed_update_kernel(const TX* __restrict__ X, int64_t n, int dim,
                                                          const int64_t* __restrict__ idx, int s, double* __restrict__ D,
                                                          unsigned long long* __restrict__ maxbits) {
  constexpr int SL = 128 / static_cast<int>(sizeof(TX));  // elements per staged slab of a row
  constexpr int RPI = 32 / SL;                             // rows per load instruction
  __shared__ TX tile[8][32][SL + 1];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c = idx[s - 1];
  const TX* xc = X + c * dim;
  double mx = 0.0;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * 8;
  for (int64_t r0 = (static_cast<int64_t>(blockIdx.x) * 8 + w) * 32; r0 < n; r0 += nwarps * 32) {
    const int64_t i = r0 + lane;
    double acc = 0.0;
    for (int k0 = 0; k0 < dim; k0 += SL) {
      const int kn = min(SL, dim - k0);
      const int col = lane % SL, sub = lane / SL;
#pragma unroll 4
      for (int j = 0; j < 32; j += RPI) {
        const int64_t row = r0 + j + sub;
        tile[w][j + sub][col] = (row < n && col < kn) ? X[row * dim + k0 + col] : TX(0);
      }
      __syncwarp();
      for (int kk = 0; kk < kn; ++kk) {
        const double diff = static_cast<double>(tile[w][lane][kk]) - static_cast<double>(__ldg(xc + k0 + kk));
        acc = fma(diff, diff, acc);
      }
      __syncwarp();
    }
    if (i < n) {
      double d2 = acc;
      if (!(d2 == d2)) d2 = 0.0;
      const double v = (s == 1) ? d2 : fmin(D[i], d2);
      D[i] = v;
      mx = fmax(mx, v);
    }
  }
  unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(mx));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
    b = t > b ? t : b;
  }
  if (lane == 0) atomicMax(maxbits, b);
}

// blocksum[b] = sum of q over rows [b * SD_BLOCK, (b + 1) * SD_BLOCK)
__global__ void __launch_bounds__(SD_BLOCK) seed_blocksum_kernel(const double* __restrict__ D, int64_t n,
                                                                 const unsigned long long* __restrict__ maxbits,
                                                                 unsigned long long* __restrict__ blocksum) {
  __shared__ unsigned long long part[SD_BLOCK / 32];
  const double maxd = __longlong_as_double(static_cast<long long>(*maxbits));
  const int64_t i = static_cast<int64_t>(blockIdx.x) * SD_BLOCK + threadIdx.x;
  unsigned long long q = 0;
  if (maxd > 0.0 && i < n) q = q_of(D[i], q_shift(maxd, n));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = q;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long t = part[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) blocksum[blockIdx.x] = t;
  }
}

// inclusive prefix sums of v over the block (one value per thread), in shared memory
__device__ __forceinline__ unsigned long long block_incl_scan(unsigned long long v, unsigned long long* warp_tot) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) warp_tot[w] = v;
  __syncthreads();
  if (w == 0) {
    unsigned long long t = lane < static_cast<int>(blockDim.x >> 5) ? warp_tot[lane] : 0ull;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long u = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += u;
    }
    warp_tot[lane] = t;
  }
  __syncthreads();
  const unsigned long long r = v + (w > 0 ? warp_tot[w - 1] : 0ull);
  __syncthreads();
  return r;
}

// one block: picks row idx[s] from the block sums (or uniformly if every weight is 0)
__global__ void __launch_bounds__(SD_BLOCK) seed_select_kernel(const double* __restrict__ D, int64_t n,
                                                               const unsigned long long* __restrict__ maxbits,
                                                               const unsigned long long* __restrict__ blocksum,
                                                               int64_t nb, uint64_t seed, int s,
                                                               int64_t* __restrict__ idx) {
  __shared__ unsigned long long warp_tot[32];
  __shared__ unsigned long long s_base, s_total;
  __shared__ long long s_blk;
  const double maxd = __longlong_as_double(static_cast<long long>(*maxbits));
  const uint64_t r = seed_draw53(seed, static_cast<uint64_t>(s));
  // each thread sums a contiguous slice of the block sums
  const int64_t per = (nb + SD_BLOCK - 1) / SD_BLOCK;
  const int64_t b0 = static_cast<int64_t>(threadIdx.x) * per, b1 = std::min<int64_t>(nb, b0 + per);
  unsigned long long mine = 0;
  for (int64_t b = b0; b < b1; ++b) mine += blocksum[b];
  const unsigned long long incl = block_incl_scan(mine, warp_tot);
  if (threadIdx.x == SD_BLOCK - 1) s_total = incl;
  __syncthreads();
  const unsigned long long total = s_total;
  if (!(maxd > 0.0) || total == 0) {
    if (threadIdx.x == 0) idx[s] = static_cast<int64_t>(scale53(r, static_cast<uint64_t>(n)));
    return;
  }
  const unsigned long long t = scale53(r, total);
  // the slice, then the block, whose running sum passes t
  const unsigned long long excl = incl - mine;
  if (excl <= t && t < incl) {
    unsigned long long run = excl;
    for (int64_t b = b0; b < b1; ++b) {
      if (t < run + blocksum[b]) {
        s_blk = b;
        s_base = run;
        break;
      }
      run += blocksum[b];
    }
  }
  __syncthreads();
  const int64_t blk = s_blk;
  const int64_t i = blk * SD_BLOCK + threadIdx.x;
  const unsigned long long q = i < n ? q_of(D[i], q_shift(maxd, n)) : 0ull;
  const unsigned long long run = s_base + block_incl_scan(q, warp_tot);
  // the first row whose running sum exceeds t (q > 0 there, so exactly one thread)
  if (run > t && run - q <= t) idx[s] = i;
}

__global__ void seed_first_kernel(int64_t* __restrict__ idx, int64_t first) { idx[0] = first; }

template <typename TX>
__global__ void seed_gather_kernel(const TX* __restrict__ X, int dim, const int64_t* __restrict__ idx, int64_t k,
                                   TX* __restrict__ centers) {
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < k * dim;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = t / dim;
    centers[t] = X[idx[c] * dim + (t - c * dim)];
  }
}

static inline size_t al(size_t b) { return (b + 255) & ~size_t(255); }

size_t seed_ws_bytes(int64_t n) {
  const int64_t nb = (n + SD_BLOCK - 1) / SD_BLOCK;
  return al(static_cast<size_t>(n) * 8) + al(static_cast<size_t>(nb) * 8) + 256;
}

template <typename TX>
static cudaError_t seed_t(const TX* X, int64_t n, int dim, int64_t k, uint64_t seed, int64_t* idx, TX* centers,
                          void* ws, cudaStream_t st) {
  uint8_t* p = static_cast<uint8_t*>(ws);
  double* D = reinterpret_cast<double*>(p);
  p += al(static_cast<size_t>(n) * 8);
  const int64_t nb = (n + SD_BLOCK - 1) / SD_BLOCK;
  unsigned long long* blocksum = reinterpret_cast<unsigned long long*>(p);
  p += al(static_cast<size_t>(nb) * 8);
  unsigned long long* maxbits = reinterpret_cast<unsigned long long*>(p);
  // center 0: uniform over the rows
  const int64_t first = static_cast<int64_t>(
      (static_cast<unsigned __int128>(seed_draw53(seed, 0)) * static_cast<unsigned __int128>(n)) >> 53);
  seed_first_kernel<<<1, 1, 0, st>>>(idx, first);
  cudaError_t e = cudaGetLastError();
  const int ublocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(num_sms()) * 5));
  for (int64_t s = 1; s < k && e == cudaSuccess; ++s) {
    e = cudaMemsetAsync(maxbits, 0, 8, st);
    if (e != cudaSuccess) break;
    seed_update_kernel<TX><<<ublocks, 256, 0, st>>>(X, n, dim, idx, static_cast<int>(s), D, maxbits);
    seed_blocksum_kernel<<<static_cast<unsigned>(nb), SD_BLOCK, 0, st>>>(D, n, maxbits, blocksum);
    seed_select_kernel<<<1, SD_BLOCK, 0, st>>>(D, n, maxbits, blocksum, nb, seed, static_cast<int>(s), idx);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && centers) {
    const int gb = static_cast<int>(std::min<int64_t>((k * dim + 255) / 256, static_cast<int64_t>(num_sms()) * 8));
    seed_gather_kernel<TX><<<gb, 256, 0, st>>>(X, dim, idx, k, centers);
    e = cudaGetLastError();
  }
  return e;
}

cudaError_t launch_kmeanspp(const void* X, bool x_f64, int64_t n, int64_t dim, int64_t k, uint64_t seed,
                            int64_t* idx, void* centers, void* ws, cudaStream_t st) {
  const int d = static_cast<int>(dim);
  if (x_f64)
    return seed_t<double>(static_cast<const double*>(X), n, d, k, seed, idx, static_cast<double*>(centers), ws, st);
  return seed_t<float>(static_cast<const float*>(X), n, d, k, seed, idx, static_cast<float*>(centers), ws, st);
}

}  // namespace euc
