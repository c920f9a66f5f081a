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
//   * larger tables    -> counting sort by label followed by a segmented reduction
//     where each warp walks 1024 label-sorted rows with coalesced row reads and
//     flushes one fp64 atomic per (segment, dim).  The sort counts per block of rows
//     in shared memory (k <= 16384): block histograms, per-label totals, a scan over
//     labels, per-(block, label) offsets, and a scatter with shared-memory cursors.
//     Larger k counts with warp-aggregated global atomics (__match_any_sync).
// stats is the unit of the data-parallel all-reduce; centers = stats / count
// (euc_center_finalize), empty clusters -> 0 as in center_kernels.cu:52,116.
#include "common.cuh"
#include "engine.h"

#include <type_traits>

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

// ------------------------------------------ sort strategy, block-private counting
// Rows [b * rpb, (b + 1) * rpb) belong to block b.  T[b * k + c] first holds the block's
// count of label c, then (priv_offsets_kernel) the position of its first such row.
template <typename TL>
__global__ void __launch_bounds__(512) priv_hist_kernel(const TL* __restrict__ labels, int64_t n, int k,
                                                        int64_t rpb, unsigned int* __restrict__ T) {
  extern __shared__ unsigned int cnt[];
  for (int c = threadIdx.x; c < k; c += blockDim.x) cnt[c] = 0u;
  __syncthreads();
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rpb;
  const int64_t r1 = min(n, r0 + rpb);
  for (int64_t i = r0 + threadIdx.x; i < r1; i += blockDim.x) {
    const int64_t c = load_label(labels, i);
    if (c >= 0 && c < k) atomicAdd(&cnt[c], 1u);
  }
  __syncthreads();
  unsigned int* row = T + static_cast<int64_t>(blockIdx.x) * k;
  for (int c = threadIdx.x; c < k; c += blockDim.x) row[c] = cnt[c];
}

// The block dimension of T is cut into kPrivSlices slices of consecutive blocks, one
// thread per (label, slice).  PS[s * k + c]: rows with label c in slice s.
constexpr int kPrivSlices = 32;

__global__ void priv_slice_sums_kernel(const unsigned int* __restrict__ T, int nb, int k,
                                       unsigned int* __restrict__ PS) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x, sl = blockIdx.y;
  if (c >= k) return;
  const int per = (nb + kPrivSlices - 1) / kPrivSlices;
  const int b0 = sl * per, b1 = min(nb, b0 + per);
  unsigned int t = 0u;
  int b = b0;
  for (; b + 8 <= b1; b += 8) {  // eight independent loads in flight
    unsigned int v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = T[static_cast<int64_t>(b + u) * k + c];
#pragma unroll
    for (int u = 0; u < 8; ++u) t += v[u];
  }
  for (; b < b1; ++b) t += T[static_cast<int64_t>(b) * k + c];
  PS[static_cast<int64_t>(sl) * k + c] = t;
}

// counts[c] = total over the slices; PS becomes the exclusive prefix over slices
__global__ void priv_slice_scan_kernel(unsigned int* __restrict__ PS, int k, unsigned int* __restrict__ counts) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= k) return;
  unsigned int run = 0u;
  for (int sl = 0; sl < kPrivSlices; ++sl) {
    const int64_t at = static_cast<int64_t>(sl) * k + c;
    const unsigned int t = PS[at];
    PS[at] = run;
    run += t;
  }
  counts[c] = run;
}

// T[b * k + c] <- offs[c] + rows with label c in blocks before b
__global__ void priv_offsets_kernel(unsigned int* __restrict__ T, int nb, int k,
                                    const unsigned long long* __restrict__ offs,
                                    const unsigned int* __restrict__ PS) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x, sl = blockIdx.y;
  if (c >= k) return;
  const int per = (nb + kPrivSlices - 1) / kPrivSlices;
  const int b0 = sl * per, b1 = min(nb, b0 + per);
  unsigned int run = static_cast<unsigned int>(offs[c]) + PS[static_cast<int64_t>(sl) * k + c];
  int b = b0;
  for (; b + 8 <= b1; b += 8) {  // eight loads issued before the stores that follow them
    unsigned int v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = T[static_cast<int64_t>(b + u) * k + c];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      T[static_cast<int64_t>(b + u) * k + c] = run;
      run += v[u];
    }
  }
  for (; b < b1; ++b) {
    const int64_t at = static_cast<int64_t>(b) * k + c;
    const unsigned int t = T[at];
    T[at] = run;
    run += t;
  }
}

template <typename TL>
__global__ void __launch_bounds__(512) priv_scatter_kernel(const TL* __restrict__ labels, int64_t n, int k,
                                                           int64_t rpb, const unsigned int* __restrict__ T,
                                                           unsigned int* __restrict__ perm) {
  extern __shared__ unsigned int cur[];
  const unsigned int* row = T + static_cast<int64_t>(blockIdx.x) * k;
  for (int c = threadIdx.x; c < k; c += blockDim.x) cur[c] = row[c];
  __syncthreads();
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rpb;
  const int64_t r1 = min(n, r0 + rpb);
  for (int64_t i = r0 + threadIdx.x; i < r1; i += blockDim.x) {
    const int64_t c = load_label(labels, i);
    if (c >= 0 && c < k) perm[atomicAdd(&cur[c], 1u)] = static_cast<unsigned int>(i);
  }
}

constexpr int kPrivMaxK = 16384;  // block-private counters: 64 KiB of shared memory

// blocks of the block-private counting sort: at least 8192 rows each, at most 2048
static int64_t priv_blocks(int64_t n) {
  int64_t nb = (n + 8191) / 8192;
  return nb < 1 ? 1 : (nb > 2048 ? 2048 : nb);
}

// Each warp reduces SEG label-sorted rows (segsum_rows: fewer when the rows are few, so
// the grid still fills the SMs); NPL = dims per lane (ceil(dim/32)).
template <typename TX, int NPL>
__global__ void __launch_bounds__(256) segsum_kernel(const TX* __restrict__ X, int dim, int k,
                                                     const unsigned long long* __restrict__ offs,
                                                     const unsigned int* __restrict__ perm,
                                                     double* __restrict__ stats, const int SEG) {
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
  // rows in batches of RB: their indices, then their values, are loaded before any is
  // folded, so a warp keeps RB row reads in flight
  constexpr int RB = NPL <= 2 ? 4 : (NPL <= 4 ? 2 : 1);
  for (int64_t pb = p0; pb < p1; pb += RB) {
    int64_t row[RB];
#pragma unroll
    for (int u = 0; u < RB; ++u) row[u] = (pb + u < p1) ? static_cast<int64_t>(perm[pb + u]) : -1;
    TX v[RB][NPL];
#pragma unroll
    for (int u = 0; u < RB; ++u) {
#pragma unroll
      for (int q = 0; q < NPL; ++q) {
        const int j = lane + 32 * q;
        v[u][q] = (row[u] >= 0 && j < dim) ? X[row[u] * dim + j] : static_cast<TX>(0);
      }
    }
#pragma unroll
    for (int u = 0; u < RB; ++u) {
      const int64_t p = pb + u;
      if (p >= p1) break;
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
#pragma unroll
      for (int q = 0; q < NPL; ++q) acc[q] += static_cast<double>(v[u][q]);
    }
  }
#pragma unroll
  for (int q = 0; q < NPL; ++q) {
    const int j = lane + 32 * q;
    if (j < dim && acc[q] != 0.0) atomicAdd(stats + static_cast<int64_t>(c) * w + j, acc[q]);
  }
}

// fp32 rows with dim = 64 NV, 16-byte aligned: each half-warp walks every other
// label-sorted position (lane l of a half holds float4s l, l + 16, ... of the row), so a
// load instruction brings two rows and a warp keeps 2 RB rows in flight; each half
// flushes its own sums per segment.
template <int NV>
__global__ void __launch_bounds__(256) segsum_h_kernel(const float* __restrict__ X, int dim, int k,
                                                       const unsigned long long* __restrict__ offs,
                                                       const unsigned int* __restrict__ perm,
                                                       double* __restrict__ stats, const int SEG) {
  constexpr int RB = 4;
  const int64_t total = static_cast<int64_t>(offs[k]);
  const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t p0 = gw * SEG;
  if (p0 >= total) return;
  const int64_t p1 = min(total, p0 + SEG);
  const int64_t q0 = p0 + half;  // this half's first position
  int c = 0;
  unsigned long long cend = 0;
  if (q0 < p1) {
    int lo = 0, hi = k;  // invariant offs[lo] <= q0 < offs[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (offs[mid] <= static_cast<unsigned long long>(q0)) lo = mid; else hi = mid;
    }
    c = lo;
    cend = offs[c + 1];
  }
  double acc[NV][4];
#pragma unroll
  for (int q = 0; q < NV; ++q)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[q][e] = 0.0;
  const int w = dim + 1;
  auto flush = [&]() {
#pragma unroll
    for (int q = 0; q < NV; ++q)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (acc[q][e] != 0.0) atomicAdd(stats + static_cast<int64_t>(c) * w + 64 * q + 4 * hl + e, acc[q][e]);
        acc[q][e] = 0.0;
      }
  };
  for (int64_t pb = q0; pb < p1; pb += 2 * RB) {
    int64_t row[RB];
#pragma unroll
    for (int u = 0; u < RB; ++u) row[u] = (pb + 2 * u < p1) ? static_cast<int64_t>(perm[pb + 2 * u]) : -1;
    float4 v[RB][NV];
#pragma unroll
    for (int u = 0; u < RB; ++u)
#pragma unroll
      for (int q = 0; q < NV; ++q)
        v[u][q] = row[u] >= 0 ? __ldg(reinterpret_cast<const float4*>(X + row[u] * dim + 64 * q) + hl)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < RB; ++u) {
      const int64_t p = pb + 2 * u;
      if (p >= p1) break;
      while (static_cast<unsigned long long>(p) >= cend) {
        flush();
        ++c;
        cend = offs[c + 1];
      }
#pragma unroll
      for (int q = 0; q < NV; ++q) {
        acc[q][0] += static_cast<double>(v[u][q].x);
        acc[q][1] += static_cast<double>(v[u][q].y);
        acc[q][2] += static_cast<double>(v[u][q].z);
        acc[q][3] += static_cast<double>(v[u][q].w);
      }
    }
  }
  if (q0 < p1) flush();
}

static inline size_t al(size_t b) { return (b + 255) & ~size_t(255); }

static bool use_smem(int64_t dim, int64_t k) { return k * (dim + 1) * 8 <= 48 * 1024; }

size_t center_ws_bytes(int64_t n, int64_t dim, int64_t k) {
  if (use_smem(dim, k)) return 256;
  const size_t tab = k <= kPrivMaxK ? al(static_cast<size_t>(priv_blocks(n)) * k * 4) + al(kPrivSlices * k * 4) : 0;
  return al(k * 4) + al((k + 1) * 8) + al(k * 8) + al(n * 4) + tab + 256;
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
  p += al(static_cast<size_t>(n) * 4);
  if (k <= kPrivMaxK) {
    unsigned int* T = reinterpret_cast<unsigned int*>(p);
    const int64_t nb = priv_blocks(n);
    unsigned int* PS = reinterpret_cast<unsigned int*>(p + al(static_cast<size_t>(nb) * k * 4));
    const int64_t rpb = (n + nb - 1) / nb;
    const size_t sm = static_cast<size_t>(k) * 4;
    if (sm > 48 * 1024) {
      e = cudaFuncSetAttribute(priv_hist_kernel<TL>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(priv_scatter_kernel<TL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sm));
      if (e != cudaSuccess) return e;
    }
    const unsigned kb = static_cast<unsigned>((k + 255) / 256);
    priv_hist_kernel<TL><<<static_cast<unsigned>(nb), 512, sm, st>>>(labels, n, k, rpb, T);
    const dim3 g2(kb, kPrivSlices);
    priv_slice_sums_kernel<<<g2, 256, 0, st>>>(T, static_cast<int>(nb), k, PS);
    priv_slice_scan_kernel<<<kb, 256, 0, st>>>(PS, k, counts);
    scan_kernel<<<1, 1024, 0, st>>>(counts, k, dim, offs, cursor, stats);
    priv_offsets_kernel<<<g2, 256, 0, st>>>(T, static_cast<int>(nb), k, offs, PS);
    priv_scatter_kernel<TL><<<static_cast<unsigned>(nb), 512, sm, st>>>(labels, n, k, rpb, T, perm);
  } else {
    e = cudaMemsetAsync(counts, 0, static_cast<size_t>(k) * 4, st);
    if (e != cudaSuccess) return e;
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, sms * 8));
    hist_kernel<TL><<<blocks, 256, 0, st>>>(labels, n, k, counts);
    scan_kernel<<<1, 1024, 0, st>>>(counts, k, dim, offs, cursor, stats);
    scatter_kernel<TL><<<blocks, 256, 0, st>>>(labels, n, k, cursor, perm);
  }
  // rows with a valid label = offs[k] <= n; the grid covers n positions and each warp
  // clamps to offs[k] on the device.  A warp walks its rows one dependent round trip
  // (label-sorted position, then row) at a time, so a segment of 1024 rows leaves a
  // small n with few warps per SM: the segment shrinks (to 256 at least) until about 64
  // warps per SM cover the rows.
  int seg = 1024;
  while (seg > 256 && (n + seg - 1) / seg < static_cast<int64_t>(num_sms()) * 64) seg >>= 1;
  const int64_t warps = (n + seg - 1) / seg;
  const int64_t sblocks = (warps + 7) / 8;
  if constexpr (std::is_same<TX, float>::value) {
    if (dim % 64 == 0 && dim <= 256 && (reinterpret_cast<uintptr_t>(X) & 15u) == 0) {
      const unsigned b = static_cast<unsigned>(sblocks);
      if (dim == 64) segsum_h_kernel<1><<<b, 256, 0, st>>>(X, dim, k, offs, perm, stats, seg);
      else if (dim == 128) segsum_h_kernel<2><<<b, 256, 0, st>>>(X, dim, k, offs, perm, stats, seg);
      else if (dim == 192) segsum_h_kernel<3><<<b, 256, 0, st>>>(X, dim, k, offs, perm, stats, seg);
      else segsum_h_kernel<4><<<b, 256, 0, st>>>(X, dim, k, offs, perm, stats, seg);
      return cudaGetLastError();
    }
  }
  const int npl = (dim + 31) / 32;
#define SEG(NPL_)                                                                                        \
  if (npl <= NPL_) {                                                                                     \
    segsum_kernel<TX, NPL_><<<static_cast<unsigned>(sblocks), 256, 0, st>>>(X, dim, k, offs, perm, stats, seg); \
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
