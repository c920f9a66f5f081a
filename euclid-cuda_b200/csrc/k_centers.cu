// Center update for Lloyd iterations.
//
// The reference (center_kernels.cu:37-95) gives every (cluster, dim) thread a scan
// over all N labels: O(K*N) label reads.  Here the points are read once:
//
//   stats[c, 0:dim] = sum of X[i, :] over rows with label c   (fp64 accumulation)
//   stats[c, dim]   = number of such rows                     (exact in fp64)
//
// Two strategies, chosen by the size of the k x (dim+1) table:
//   * table <= 48 KiB  -> per-CTA privatised table in shared memory (smem fp64
//     atomics), one flush of the table per CTA;
//   * larger tables    -> counting sort by label (histogram, scan, warp-aggregated
//     scatter with __match_any_sync) followed by a segmented reduction where each
//     warp walks 1024 label-sorted rows with coalesced row reads and flushes one
//     fp64 atomic per (segment, dim).
// stats is the unit of the data-parallel all-reduce; centers = stats / count
// (euc_center_finalize), empty clusters -> 0 as in center_kernels.cu:52,116.
#include "common.cuh"
#include "engine.h"

namespace euc {

template <typename TL> __device__ __forceinline__ int64_t load_label(const TL* p, int64_t i) {
  return static_cast<int64_t>(p[i]);
}

// ------------------------------------------------------- privatised strategy
template <typename TX, typename TL>
__global__ void __launch_bounds__(256) stats_smem_kernel(const TX* __restrict__ X, const TL* __restrict__ labels,
                                                         int64_t n, int dim, int k, double* __restrict__ stats,
                                                         int64_t rows_per_cta) {
  extern __shared__ double tab[];
  const int w = dim + 1;
  for (int t = threadIdx.x; t < k * w; t += blockDim.x) tab[t] = 0.0;
  __syncthreads();
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
  const int64_t r1 = min(n, r0 + rows_per_cta);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int64_t i = r0 + warp; i < r1; i += nw) {
    const int64_t c = load_label(labels, i);
    if (c < 0 || c >= k) continue;
    double* row = tab + c * w;
    for (int j = lane; j < dim; j += 32) atomicAdd(row + j, static_cast<double>(X[i * dim + j]));
    if (lane == 0) atomicAdd(row + dim, 1.0);
  }
  __syncthreads();
  for (int t = threadIdx.x; t < k * w; t += blockDim.x) {
    const double v = tab[t];
    if (v != 0.0) atomicAdd(stats + t, v);
  }
}

// ------------------------------------------------------- sort strategy
template <typename TL>
__global__ void hist_kernel(const TL* __restrict__ labels, int64_t n, int k, unsigned int* __restrict__ counts) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = load_label(labels, i);
    const bool ok = c >= 0 && c < k;
    const int key = ok ? static_cast<int>(c) : -1;
    const unsigned peers = __match_any_sync(__activemask(), key);
    const int leader = __ffs(peers) - 1;
    if (ok && (threadIdx.x & 31) == leader) atomicAdd(&counts[c], static_cast<unsigned>(__popc(peers)));
  }
}

// exclusive scan of counts -> offs[0..k], cursor copy, and the count column of stats
__global__ void __launch_bounds__(1024) scan_kernel(const unsigned int* __restrict__ counts, int k, int dim,
                                                    unsigned long long* __restrict__ offs,
                                                    unsigned long long* __restrict__ cursor,
                                                    double* __restrict__ stats) {
  __shared__ unsigned long long warp_sums[32];
  __shared__ unsigned long long carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < k; base += 1024) {
    const int c = base + threadIdx.x;
    const unsigned long long v = (c < k) ? counts[c] : 0ull;
    unsigned long long x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      unsigned long long s = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      warp_sums[lane] = s;
    }
    __syncthreads();
    const unsigned long long incl = x + (warp > 0 ? warp_sums[warp - 1] : 0ull) + carry;
    if (c < k) {
      offs[c] = incl - v;
      cursor[c] = incl - v;
      stats[static_cast<int64_t>(c) * (dim + 1) + dim] = static_cast<double>(v);
    }
    __syncthreads();
    if (threadIdx.x == 1023) carry = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) offs[k] = carry;
}

template <typename TL>
__global__ void scatter_kernel(const TL* __restrict__ labels, int64_t n, int k,
                               unsigned long long* __restrict__ cursor, unsigned int* __restrict__ perm) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = load_label(labels, i);
    const bool ok = c >= 0 && c < k;
    const int key = ok ? static_cast<int>(c) : -1;
    const unsigned peers = __match_any_sync(__activemask(), key);
    const int lane = threadIdx.x & 31;
    const int leader = __ffs(peers) - 1;
    unsigned long long base = 0;
    if (ok && lane == leader) base = atomicAdd(&cursor[c], static_cast<unsigned long long>(__popc(peers)));
    base = __shfl_sync(peers, base, leader);
    if (ok) perm[base + __popc(peers & ((1u << lane) - 1u))] = static_cast<unsigned int>(i);
  }
}

// Each warp reduces SEG label-sorted rows; NPL = dims per lane (ceil(dim/32)).
template <typename TX, int NPL>
__global__ void __launch_bounds__(256) segsum_kernel(const TX* __restrict__ X, int dim, int k,
                                                     const unsigned long long* __restrict__ offs,
                                                     const unsigned int* __restrict__ perm,
                                                     double* __restrict__ stats) {
  constexpr int SEG = 1024;
  const int64_t total = static_cast<int64_t>(offs[k]);  // rows with a label in [0, k)
  const int lane = threadIdx.x & 31;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t p0 = gw * SEG;
  if (p0 >= total) return;
  const int64_t p1 = min(total, p0 + SEG);
  // cluster containing position p0: largest c with offs[c] <= p0
  int lo = 0, hi = k;  // invariant offs[lo] <= p0 < offs[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (offs[mid] <= static_cast<unsigned long long>(p0)) lo = mid; else hi = mid;
  }
  int c = lo;
  unsigned long long cend = offs[c + 1];
  double acc[NPL];
#pragma unroll
  for (int q = 0; q < NPL; ++q) acc[q] = 0.0;
  const int w = dim + 1;
  for (int64_t p = p0; p < p1; ++p) {
    while (static_cast<unsigned long long>(p) >= cend) {
#pragma unroll
      for (int q = 0; q < NPL; ++q) {
        const int j = lane + 32 * q;
        if (j < dim && acc[q] != 0.0) atomicAdd(stats + static_cast<int64_t>(c) * w + j, acc[q]);
        acc[q] = 0.0;
      }
      ++c;
      cend = offs[c + 1];
    }
    const int64_t row = perm[p];
    const TX* xr = X + row * dim;
#pragma unroll
    for (int q = 0; q < NPL; ++q) {
      const int j = lane + 32 * q;
      if (j < dim) acc[q] += static_cast<double>(xr[j]);
    }
  }
#pragma unroll
  for (int q = 0; q < NPL; ++q) {
    const int j = lane + 32 * q;
    if (j < dim && acc[q] != 0.0) atomicAdd(stats + static_cast<int64_t>(c) * w + j, acc[q]);
  }
}

static inline size_t al(size_t b) { return (b + 255) & ~size_t(255); }

static bool use_smem(int64_t dim, int64_t k) { return k * (dim + 1) * 8 <= 48 * 1024; }

size_t center_ws_bytes(int64_t n, int64_t dim, int64_t k) {
  if (use_smem(dim, k)) return 256;
  return al(k * 4) + al((k + 1) * 8) + al(k * 8) + al(n * 4) + 256;
}

template <typename TX, typename TL>
static cudaError_t stats_t(const TX* X, const TL* labels, int64_t n, int dim, int k, double* stats, void* ws,
                           cudaStream_t st) {
  const int64_t w = dim + 1;
  cudaError_t e = cudaMemsetAsync(stats, 0, static_cast<size_t>(k) * w * sizeof(double), st);
  if (e != cudaSuccess || n == 0) return e;
  const int sms = num_sms();
  if (use_smem(dim, k)) {
    const size_t smem = static_cast<size_t>(k) * w * sizeof(double);
    int64_t ctas = std::min<int64_t>(static_cast<int64_t>(sms) * 4, (n + 255) / 256);
    if (ctas < 1) ctas = 1;
    const int64_t rpc = (n + ctas - 1) / ctas;
    stats_smem_kernel<TX, TL><<<static_cast<unsigned>(ctas), 256, smem, st>>>(X, labels, n, dim, k, stats, rpc);
    return cudaGetLastError();
  }
  uint8_t* p = static_cast<uint8_t*>(ws);
  unsigned int* counts = reinterpret_cast<unsigned int*>(p);
  p += al(static_cast<size_t>(k) * 4);
  unsigned long long* offs = reinterpret_cast<unsigned long long*>(p);
  p += al(static_cast<size_t>(k + 1) * 8);
  unsigned long long* cursor = reinterpret_cast<unsigned long long*>(p);
  p += al(static_cast<size_t>(k) * 8);
  unsigned int* perm = reinterpret_cast<unsigned int*>(p);
  e = cudaMemsetAsync(counts, 0, static_cast<size_t>(k) * 4, st);
  if (e != cudaSuccess) return e;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, sms * 8));
  hist_kernel<TL><<<blocks, 256, 0, st>>>(labels, n, k, counts);
  scan_kernel<<<1, 1024, 0, st>>>(counts, k, dim, offs, cursor, stats);
  scatter_kernel<TL><<<blocks, 256, 0, st>>>(labels, n, k, cursor, perm);
  // rows with a valid label = offs[k] <= n; the grid covers n positions and each warp
  // clamps to offs[k] on the device.
  const int64_t warps = (n + 1023) / 1024;
  const int64_t sblocks = (warps + 7) / 8;
  const int npl = (dim + 31) / 32;
#define SEG(NPL_)                                                                                        \
  if (npl <= NPL_) {                                                                                     \
    segsum_kernel<TX, NPL_><<<static_cast<unsigned>(sblocks), 256, 0, st>>>(X, dim, k, offs, perm, stats); \
    return cudaGetLastError();                                                                           \
  }
  SEG(1) SEG(2) SEG(4) SEG(8) SEG(16) SEG(32)
#undef SEG
  return cudaErrorNotSupported;
}

cudaError_t launch_center_stats(const void* X, bool x_f64, const void* labels, bool labels_i64, int64_t n,
                                int64_t dim, int64_t k, double* stats, void* ws, size_t ws_bytes,
                                cudaStream_t st) {
  if (ws_bytes < center_ws_bytes(n, dim, k)) return cudaErrorInvalidValue;
  if (dim > 1024) return cudaErrorNotSupported;
  const int d = static_cast<int>(dim), kk = static_cast<int>(k);
  if (x_f64) {
    if (labels_i64)
      return stats_t<double, long long>(static_cast<const double*>(X), static_cast<const long long*>(labels), n, d,
                                        kk, stats, ws, st);
    return stats_t<double, int>(static_cast<const double*>(X), static_cast<const int*>(labels), n, d, kk, stats, ws,
                                st);
  }
  if (labels_i64)
    return stats_t<float, long long>(static_cast<const float*>(X), static_cast<const long long*>(labels), n, d, kk,
                                     stats, ws, st);
  return stats_t<float, int>(static_cast<const float*>(X), static_cast<const int*>(labels), n, d, kk, stats, ws,
                             st);
}

template <typename T>
__global__ void finalize_kernel(const double* __restrict__ stats, int dim, int64_t k, T* __restrict__ centers,
                                const T* __restrict__ prev, int empty_policy) {
  const int64_t total = k * dim;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = t / dim;
    const int j = static_cast<int>(t - c * dim);
    const double cnt = stats[c * (dim + 1) + dim];
    T v;
    if (cnt > 0.0)
      v = static_cast<T>(stats[c * (dim + 1) + j] / cnt);
    else
      v = (empty_policy == 1 && prev != nullptr) ? prev[t] : static_cast<T>(0);
    centers[t] = v;
  }
}

cudaError_t launch_center_finalize(const double* stats, int64_t dim, int64_t k, void* centers, bool f64,
                                   const void* prev, int empty_policy, cudaStream_t st) {
  const int64_t total = k * dim;
  if (total <= 0) return cudaSuccess;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, num_sms() * 8));
  if (f64)
    finalize_kernel<double><<<blocks, 256, 0, st>>>(stats, static_cast<int>(dim), k, static_cast<double*>(centers),
                                                   static_cast<const double*>(prev), empty_policy);
  else
    finalize_kernel<float><<<blocks, 256, 0, st>>>(stats, static_cast<int>(dim), k, static_cast<float*>(centers),
                                                  static_cast<const float*>(prev), empty_policy);
  return cudaGetLastError();
}

}  // namespace euc
