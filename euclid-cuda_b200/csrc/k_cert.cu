// Certified argmin: second pass after the screening kernel's CERT form (sm_100a).
//
// The label of row i is the first index of the smallest direct distance
// D_ij = direct(p_i, c_j) over all centers, in the operator's recompute arithmetic
// (fp32 or fp64 sequential sum of squared differences, direct.cuh) -- what the
// operator stores for a pair it flags, so the labels equal the reference's whenever
// every pair of the row is flagged.  Only the candidates that can win are recomputed.
//
// The screening kernel leaves, for each of its four epilogue groups (tile parity,
// column half), the group's best screened distance d with the sorted start of its
// center's group of 8 sorted centers, and the second-best screened distance outside
// that group.  Merged: d1 (the row's best), its group G, and m2 (smallest screened
// distance of any center outside G).  The screened distance of pair j is
// d^_j = 2 y_j - Br + pp with y_j the MMA accumulator (aux.cuh).  It differs from
// |p~ - c~_j|^2 (p~, c~ the operands rounded to the MMA type) by a row-common part rho
// (pp against |p~|^2, the split of Br) and a pair part e_j (cc_j against |c~_j|^2, the
// fp32 accumulation of the MMA, the key truncation, the fp32 adds of the formula); and
// |p~ - c~_j| differs from a_j = |p - c_j| by at most Delta = u (|p| + |c_j|) + 2 eta
// sqrt(dim) (unit roundoff u of the MMA type, eta its absolute rounding floor).  The
// direct sum is within gd = (dim + 4) 2^-24 of a_j^2.  Hence
//   D_j <= UB = (sqrt(d1 + rho + e) + Delta)^2 (1 + gd)          for the winner,
//   D_j >= LB = max(sqrt(max(m2 - rho - e, 0)) - Delta, 0)^2 (1 - gd)  outside G,
// with rho, e and Delta bounded from pp and the largest center norm.  If LB > UB no
// center outside G reaches the winner's distance: the 8 direct distances of G decide
// the row.  Otherwise a center j can only win if its screened distance is at most
//   T = (sqrt(UB / (1 - gd)) + Delta)^2 + rho + e,
// and a second screen over the row tiles holding such rows lists every group of 8 with
// a screened distance <= T; the direct distances of the listed groups decide the row.
// Rows the screen does not bound (norms not finite or out of the extra K block's range)
// and rows whose listed groups overflow the list take every center's direct distance.
//
// The direct distances of the groups (the decided rows' and the second screen's) are
// taken by group: the (row, group) entries are counted and sorted by group, and a block
// stages its group's 8 centers once for all its rows.  When the workspace has no room
// for that, the decided rows take theirs row by row and the listed groups entry by entry.
//
// d_count receives the number of direct distances evaluated.
#include "common.cuh"
#include "engine.h"
#include "direct.cuh"
#include "aux.cuh"

#include <cmath>

namespace euc {

struct CertArgs {
  const float* P;
  const float* C;
  int64_t n, m;
  int dim;
  const int* perm;               // sorted position -> center index
  const float* pp;               // the screen's point norms
  const float* ccmax;            // largest finite center norm (device scalar)
  uint8_t* redo;                 // rows the screen does not bound (2: entries overflowed)
  const unsigned long long* key; // [4][n] (best screened distance, sorted start of its group)
  const float* d2;               // [4][n] second-best screened distance outside that group
  float* thr;                    // per row: T of the second screen, -inf for a decided row
  uint8_t* tiles;                // per row tile: holds a row for the second screen
  unsigned long long* row_key;   // rows of the second screen: smallest (distance, index)
  const unsigned long long* glist;  // second screen: (row << 32 | sorted group start) entries
  unsigned long long region_cap;    //   in regions of region_cap entries,
  const uint32_t* region_cnt;       //   region_cnt[r] of them used
  int regions;
  uint32_t* rows;                // rows evaluated whole
  unsigned int* nrows;
  // by group (ng > 0): (row << 32 | sorted group start) entries of the decided rows and
  // of the second screen, counted per group of 8 sorted centers, then their rows sorted
  // by group
  int ng;
  unsigned long long* ent;
  unsigned int* ent_n;
  unsigned int ent_cap;
  unsigned int* gcnt;            // entries per group, then the scatter cursors
  unsigned int* goff;            // exclusive prefix over the groups, ng + 1
  unsigned int* boff;            // exclusive prefix of the groups' 32-row batches, ng + 1
  uint32_t* srow;
  // second screen over the undecided rows alone: their list F (nF of them), and per
  // listed row its norm, threshold and redo byte; its entries name list positions
  bool gather;
  uint32_t* F;
  unsigned int* nF;
  float* pg;
  float* thr_g;
  uint8_t* redo_g;
  void* plow;                    // the gathered low-precision rows (ldlow elements each)
  int ldlow;
  int lowkind;                   // 0 fp16, 1 bf16
  unsigned long long* count;
  int64_t* labels;
  int32_t* labels32;
  float* mind;
  // bound constants
  double u;      // unit roundoff of the MMA operand type
  double un;     // relative error of a norm against |p~|^2
  double eta_n;  // absolute error of a norm (subnormal range of its type)
  double gmma;   // relative error of the MMA's fp32 accumulation, against the sum of |terms|
  double gd;     // relative error of the direct sum
  double eta;    // absolute rounding floor of one operand element
  double sqd;    // sqrt(dim)
};

__device__ __forceinline__ float key_dist(unsigned long long k) {
  return __uint_as_float(static_cast<uint32_t>(k >> 32));
}

__device__ __forceinline__ void cert_write(const CertArgs& a, int64_t i, unsigned long long k) {
  const uint32_t j = static_cast<uint32_t>(k & 0xffffffffull);
  if (a.labels) a.labels[i] = j;
  if (a.labels32) a.labels32[i] = static_cast<int32_t>(j);
  if (a.mind) a.mind[i] = key_dist(k);
}

// 1 when every center outside the winning group has a direct distance above the
// winner's (LB > UB above); else 2 with the second screen's threshold T in *thr, or 0
// when the screen gives no bound.  fp64 throughout; the bounds are monotone in the
// norms, so the largest center norm stands in for each center's.
__device__ int cert_bounds(const CertArgs& a, float ppf, float d1f, float m2f, float* thr) {
  const float kInf = __int_as_float(0x7f800000);
  if (!(d1f < kInf)) return 0;
  if (!(m2f < kInf)) return 1;  // no other center
  const double pp = ppf, ccm = *a.ccmax, d1 = d1f, m2 = m2f;
  const double br = static_cast<double>(__fmul_rn(ppf, kAuxRowScale));
  // |p|, |c| (fp32 vectors) and |p~|, |c~| (rounded), upper bounds
  const double np = (sqrt((pp + a.eta_n) / (1.0 - a.un)) + a.eta * a.sqd) / (1.0 - a.u);
  const double nc = (sqrt((ccm + a.eta_n) / (1.0 - a.un)) + a.eta * a.sqd) / (1.0 - a.u);
  const double npt = (1.0 + a.u) * np + a.eta * a.sqd;
  const double nct = (1.0 + a.u) * nc + a.eta * a.sqd;
  const double delta = a.u * (np + nc) + 2.0 * a.eta * a.sqd;
  const double sterm = npt * nct + 0.505 * (ccm + br);  // sum of |terms| of one MMA accumulator
  const double rho = a.un * npt * npt + a.eta_n + 0x1p-24 * br;
  const double e = a.un * nct * nct + a.eta_n + 0x1p-24 * ccm + (2.0 * a.gmma + 0x1.1p-17) * sterm +
                   0x1p-23 * (2.0 * sterm + br + pp);
  const double slack = rho + e;
  const double ua = sqrt(d1 + slack) + delta;
  const double ub = ua * ua * (1.0 + a.gd);
  const double la = fmax(sqrt(fmax(m2 - slack, 0.0)) - delta, 0.0);
  const double lb = la * la * (1.0 - a.gd);
  if (lb > ub * (1.0 + 0x1p-30)) return 1;
  const double ta = sqrt(ub / (1.0 - a.gd)) + delta;
  const float t = __double2float_ru((ta * ta + slack) * (1.0 + 0x1p-30));
  if (!(t < kInf)) return 0;
  *thr = t;
  return 2;
}

// The four partial results of row i merged: the best key, and m2 = the other groups'
// best distances and the winner's second-best.
__device__ __forceinline__ float cert_merge(const CertArgs& a, int64_t i, unsigned long long& k1) {
  const float kInf = __int_as_float(0x7f800000);
  float m2 = kInf, d2w = kInf;
  k1 = ~0ull;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const unsigned long long k = __ldg(a.key + g * a.n + i);
    const float d2 = __ldg(a.d2 + g * a.n + i);
    if (k < k1) {
      if (k1 != ~0ull) m2 = fminf(m2, key_dist(k1));
      k1 = k;
      d2w = d2;
    } else {
      m2 = fminf(m2, key_dist(k));
    }
  }
  return fminf(m2, d2w);
}

// Row by row (no room to sort by group): four rows per warp, 8 lanes per row.  Rows the
// winning group decides take its 8 direct distances here; rows it does not decide get
// their threshold T and their row tile is switched on for the second screen; rows
// without bounds are listed for cert_whole_rows_kernel.
template <int REC>
__global__ void __launch_bounds__(256) cert_rows_kernel(const CertArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = lane & 7;
  const float kInf = __int_as_float(0x7f800000);
  const int64_t nq = (a.n + 3) / 4;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  unsigned long long evals = 0;
  for (int64_t qd = gw; qd < nq; qd += nw) {
    const int64_t i = qd * 4 + (lane >> 3);
    const bool valid = i < a.n;
    bool whole = valid;
    float thr = -kInf;
    unsigned long long k1 = ~0ull;
    if (valid && a.redo[i] == 0) {
      const float m2 = cert_merge(a, i, k1);
      const int r = cert_bounds(a, __ldg(a.pp + i), key_dist(k1), m2, &thr);
      whole = r == 0;
      if (r == 2 && t == 0) {  // to the second screen
        a.row_key[i] = ~0ull;
        a.tiles[i / 128] = 1;
      }
      if (r != 2) thr = -kInf;
    }
    // thr: the second screen's T, -inf for a row its group decides, NaN for a row
    // evaluated whole
    if (valid && t == 0) a.thr[i] = whole ? __int_as_float(0x7fc00000) : thr;
    const bool grp = valid && !whole && !(thr > -kInf);
    unsigned long long best = ~0ull;
    if (grp) {
      const int64_t s = static_cast<int64_t>(k1 & 0xffffffffull) + t;  // sorted position
      if (s < a.m) {
        const int j = __ldg(a.perm + s);
        const double v = direct_dist<float, REC>(a.P + i * a.dim, a.C + static_cast<int64_t>(j) * a.dim, a.dim);
        best = make_key(static_cast<float>(v), static_cast<uint32_t>(j));
        ++evals;
      }
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other < best ? other : best;
    }
    if (grp && t == 0) cert_write(a, i, best);
    // rows evaluated whole: one list entry each, one reservation per warp
    const bool push = whole && t == 0;
    const unsigned int bal = __ballot_sync(0xffffffffu, push);
    if (bal) {
      unsigned int base = 0;
      if (lane == 0) base = atomicAdd(a.nrows, static_cast<unsigned int>(__popc(bal)));
      base = __shfl_sync(0xffffffffu, base, 0);
      if (push) a.rows[base + __popc(bal & ((1u << lane) - 1u))] = static_cast<uint32_t>(i);
    }
  }
  evals = __reduce_add_sync(0xffffffffu, static_cast<unsigned int>(evals));
  if (lane == 0 && evals) atomicAdd(a.count, evals);
}

// Appends this thread's item (if `take`) to a list: one reservation per block and list
// (a warp-shared global counter would serialise a few hundred thousand atomics).
// Every thread of the block calls it.
__device__ __forceinline__ void block_append(bool take, unsigned int* counter, unsigned int* wcnt,
                                             unsigned int* sbase, unsigned int& pos) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const unsigned int bal = __ballot_sync(0xffffffffu, take);
  if (lane == 0) wcnt[w] = __popc(bal);
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int tot = 0;
    for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) {
      const unsigned int c = wcnt[k];
      wcnt[k] = tot;
      tot += c;
    }
    *sbase = tot ? atomicAdd(counter, tot) : 0u;
  }
  __syncthreads();
  pos = *sbase + wcnt[w] + __popc(bal & ((1u << lane) - 1u));
  __syncthreads();  // wcnt and sbase are reused by the next call
}

// By group, one thread per row: a row its group decides gets an entry (row, group); a
// row it does not decide its threshold T, and its row tile switched on for the second
// screen (or, gathering, the row goes to that screen's list); a row without bounds goes
// to the rows evaluated whole.  thr: T, -inf for a decided row, NaN for a row
// evaluated whole.
__global__ void __launch_bounds__(256) cert_decide_kernel(const CertArgs a) {
  __shared__ unsigned int wcnt[8];
  __shared__ unsigned int sbase;
  const float kInf = __int_as_float(0x7f800000);
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x; base < a.n;
       base += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = base + threadIdx.x;
    const bool valid = i < a.n;
    int r = 0;
    float thr = -kInf;
    unsigned long long k1 = ~0ull;
    if (valid && a.redo[i] == 0) {
      const float m2 = cert_merge(a, i, k1);
      r = cert_bounds(a, __ldg(a.pp + i), key_dist(k1), m2, &thr);
    }
    const bool whole = valid && r == 0, dec = valid && r == 1, und = valid && r == 2;
    if (valid) {
      if (und && !a.gather) a.tiles[i / 128] = 1;
      if (r != 0) a.row_key[i] = ~0ull;
      a.thr[i] = whole ? __int_as_float(0x7fc00000) : (und ? thr : -kInf);
    }
    unsigned int pos;
    if (a.gather) {  // block-uniform
      block_append(und, a.nF, wcnt, &sbase, pos);
      if (und) a.F[pos] = static_cast<uint32_t>(i);
    }
    block_append(dec, a.ent_n, wcnt, &sbase, pos);
    if (dec) a.ent[pos] = (static_cast<unsigned long long>(i) << 32) | (k1 & 0xffffffffull);
    block_append(whole, a.nrows, wcnt, &sbase, pos);
    if (whole) a.rows[pos] = static_cast<uint32_t>(i);
  }
}

// By group: the second screen's entries appended to the decided rows' (one reservation
// per block); a row whose entry finds no room is evaluated whole (redo 2).
__global__ void __launch_bounds__(256) cert_gather_kernel(const CertArgs a) {
  __shared__ unsigned int s_base;
  constexpr int kBlocksPerRegion = 8;
  const int r = blockIdx.x / kBlocksPerRegion, b = blockIdx.x % kBlocksPerRegion;
  unsigned long long cnt64 = a.region_cnt[r];
  if (cnt64 > a.region_cap) cnt64 = a.region_cap;
  const uint32_t cnt = static_cast<uint32_t>(cnt64);
  const uint32_t lo = static_cast<uint32_t>(static_cast<unsigned long long>(cnt) * b / kBlocksPerRegion);
  const uint32_t hi = static_cast<uint32_t>(static_cast<unsigned long long>(cnt) * (b + 1) / kBlocksPerRegion);
  if (lo >= hi) return;  // the whole block
  if (threadIdx.x == 0) s_base = atomicAdd(a.ent_n, hi - lo);
  __syncthreads();
  const unsigned long long* gl = a.glist + static_cast<unsigned long long>(r) * a.region_cap;
  const unsigned int nf = a.gather ? *a.nF : 0u;
  for (uint32_t q = lo + threadIdx.x; q < hi; q += blockDim.x) {
    unsigned long long e = gl[q];
    const unsigned long long pos = static_cast<unsigned long long>(s_base) + (q - lo);
    int64_t i = static_cast<int64_t>(e >> 32);
    if (a.gather) {  // the entry names a list position
      if (i >= nf) continue;
      i = a.F[i];
      e = (static_cast<unsigned long long>(i) << 32) | (e & 0xffffffffull);
    }
    if (i >= a.n) continue;
    if (pos < a.ent_cap)
      a.ent[pos] = e;
    else
      a.redo[i] = 2;
  }
}

// Listed rows whose groups did not fit the second screen's list (redo 2 at their list
// position) are evaluated whole.
__global__ void __launch_bounds__(256) cert_relay_redo_kernel(const CertArgs a) {
  const unsigned int nf = *a.nF;
  for (unsigned int f = blockIdx.x * blockDim.x + threadIdx.x; f < nf; f += gridDim.x * blockDim.x)
    if (a.redo_g[f] != 0) a.redo[a.F[f]] = 2;
}

// The undecided rows gathered for the second screen over whole 128-row tiles, one thread
// per 8 values of a list position f: row f of the low-precision copy (the operand
// rounding of the screen, zero beyond dim; the points are whole 16-byte vectors), and
// per position its norm, threshold and row tile; positions past the list get threshold
// -inf (no group is listed for them).
template <int LOWK>
__global__ void __launch_bounds__(256) cert_compact_kernel(const CertArgs a) {
  const unsigned int nf = *a.nF;
  const unsigned int nfp = (nf + 127u) & ~127u;
  const float kInf = __int_as_float(0x7f800000);
  const unsigned int per = static_cast<unsigned int>(a.ldlow) / 8u;  // 8-value pieces per row
  const unsigned long long items = static_cast<unsigned long long>(nfp) * per;
  for (unsigned long long t = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; t < items;
       t += static_cast<unsigned long long>(gridDim.x) * blockDim.x) {
    const unsigned int f = static_cast<unsigned int>(t / per), q = static_cast<unsigned int>(t % per);
    uint4 out = make_uint4(0u, 0u, 0u, 0u);
    if (f < nf) {
      const int64_t i = a.F[f];
      const int k = static_cast<int>(q) * 8;
      float x[8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k + 4 * h < a.dim) v = __ldg(reinterpret_cast<const float4*>(a.P + i * a.dim + k + 4 * h));
        x[4 * h] = v.x;
        x[4 * h + 1] = v.y;
        x[4 * h + 2] = v.z;
        x[4 * h + 3] = v.w;
      }
      uint32_t b[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        b[e] = LOWK == 0 ? __half_as_ushort(__float2half_rn(x[e])) : __bfloat16_as_ushort(__float2bfloat16_rn(x[e]));
      out = make_uint4(b[0] | (b[1] << 16), b[2] | (b[3] << 16), b[4] | (b[5] << 16), b[6] | (b[7] << 16));
      if (q == 0) {
        a.pg[f] = __ldg(a.pp + i);
        a.thr_g[f] = a.thr[i];
        a.tiles[f / 128] = 1;
      }
    } else if (q == 0) {
      a.pg[f] = 0.f;
      a.thr_g[f] = -kInf;
    }
    reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.plow) + static_cast<size_t>(f) * a.ldlow)[q] = out;
  }
}

// This block's contiguous share [lo, hi) of the entries.
__device__ __forceinline__ void cert_share(const CertArgs& a, unsigned int& lo, unsigned int& hi) {
  const unsigned int ne = min(*a.ent_n, a.ent_cap);
  lo = static_cast<unsigned int>(static_cast<unsigned long long>(ne) * blockIdx.x / gridDim.x);
  hi = static_cast<unsigned int>(static_cast<unsigned long long>(ne) * (blockIdx.x + 1) / gridDim.x);
}

// Entries per group: a shared-memory histogram per block, flushed once per group.
__global__ void __launch_bounds__(256) cert_count_kernel(const CertArgs a) {
  extern __shared__ unsigned int hist[];
  for (int g = threadIdx.x; g < a.ng; g += blockDim.x) hist[g] = 0;
  __syncthreads();
  unsigned int lo, hi;
  cert_share(a, lo, hi);
  for (unsigned int q = lo + threadIdx.x; q < hi; q += blockDim.x)
    atomicAdd(hist + (static_cast<uint32_t>(a.ent[q]) >> 3), 1u);
  __syncthreads();
  for (int g = threadIdx.x; g < a.ng; g += blockDim.x)
    if (hist[g]) atomicAdd(a.gcnt + g, hist[g]);
}

// Exclusive prefixes over the groups (one block): goff of the entry counts (the counts
// become the scatter cursors) and boff of the 32-row batches.
__global__ void __launch_bounds__(1024) cert_scan_kernel(unsigned int* __restrict__ gcnt,
                                                         unsigned int* __restrict__ goff,
                                                         unsigned int* __restrict__ boff, int ng) {
  __shared__ unsigned int wsum[2][32];
  const int per = (ng + 1023) / 1024;
  const int g0 = threadIdx.x * per, g1 = min(g0 + per, ng);
  unsigned int sum = 0, bsum = 0;
  for (int g = g0; g < g1; ++g) {
    sum += gcnt[g];
    bsum += (gcnt[g] + 31u) / 32u;
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned int incl = sum, bincl = bsum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned int v = __shfl_up_sync(0xffffffffu, incl, o);
    const unsigned int bv = __shfl_up_sync(0xffffffffu, bincl, o);
    if (lane >= o) {
      incl += v;
      bincl += bv;
    }
  }
  if (lane == 31) {
    wsum[0][w] = incl;
    wsum[1][w] = bincl;
  }
  __syncthreads();
  if (w < 2) {
    unsigned int x = wsum[w][lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned int v = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += v;
    }
    wsum[w][lane] = x;  // inclusive over the warps
  }
  __syncthreads();
  unsigned int run = incl - sum + (w > 0 ? wsum[0][w - 1] : 0u);
  unsigned int brun = bincl - bsum + (w > 0 ? wsum[1][w - 1] : 0u);
  for (int g = g0; g < g1; ++g) {
    const unsigned int c = gcnt[g];
    goff[g] = run;
    boff[g] = brun;
    gcnt[g] = run;
    run += c;
    brun += (c + 31u) / 32u;
  }
  if (threadIdx.x == 1023) {
    goff[ng] = wsum[0][31];
    boff[ng] = wsum[1][31];
  }
}

// Rows of the entries sorted by group (any order within a group; ~0 for a row evaluated
// whole): per block, a histogram of its share, one cursor reservation per group, then
// shared-memory cursors.
__global__ void __launch_bounds__(256) cert_scatter_kernel(const CertArgs a) {
  extern __shared__ unsigned int sm[];
  unsigned int* cur = sm;          // per group: this block's count, then its cursor
  unsigned int* gbase = sm + a.ng; // per group: this block's first position
  for (int g = threadIdx.x; g < a.ng; g += blockDim.x) cur[g] = 0;
  __syncthreads();
  unsigned int lo, hi;
  cert_share(a, lo, hi);
  for (unsigned int q = lo + threadIdx.x; q < hi; q += blockDim.x)
    atomicAdd(cur + (static_cast<uint32_t>(a.ent[q]) >> 3), 1u);
  __syncthreads();
  for (int g = threadIdx.x; g < a.ng; g += blockDim.x) {
    const unsigned int c = cur[g];
    gbase[g] = c ? atomicAdd(a.gcnt + g, c) : 0u;
    cur[g] = 0;
  }
  __syncthreads();
  for (unsigned int q = lo + threadIdx.x; q < hi; q += blockDim.x) {
    const unsigned long long e = a.ent[q];
    const uint32_t g = static_cast<uint32_t>(e) >> 3;
    const uint32_t i = static_cast<uint32_t>(e >> 32);
    // a row evaluated whole (redo, final here) is skipped by the group evaluation
    a.srow[gbase[g] + atomicAdd(cur + g, 1u)] = a.redo[i] != 0 ? 0xffffffffu : i;
  }
}

// Batches of up to 32 rows of one group, the batches of all groups in order and each
// block taking a contiguous share.  A batch is evaluated CB_KD dimensions (a slab) at a
// time: the group's 8 sorted centers and the rows are staged in shared memory (the
// centers once per group when dim <= CB_KD), and thread (row, center) runs the pair's
// direct sum in the arithmetic and dimension order of direct_dist.  The next slab's
// values are loaded into registers while the current one is summed, and the row ids
// come from a shared-memory window of the sorted rows, so no load waits on another.
// The 8 keys of a row fold into its key with one 64-bit atomicMin.
constexpr int CB_KD = 64;
constexpr int CB_WIN = 256;  // sorted row ids staged per window

template <int REC>
__global__ void __launch_bounds__(256) cert_bucket_kernel(const CertArgs a) {
  __shared__ float cs[8][CB_KD + 1];
  __shared__ float ps[32][CB_KD + 1];
  __shared__ uint32_t rs[CB_WIN];
  const int tid = threadIdx.x, r = tid >> 3, c = tid & 7;
  const int dim = a.dim;
  const int nk = (dim + CB_KD - 1) / CB_KD;
  const unsigned int nb = a.boff[a.ng], ntot = a.goff[a.ng];
  const unsigned int qlo = static_cast<unsigned int>(static_cast<unsigned long long>(nb) * blockIdx.x / gridDim.x);
  const unsigned int qhi = static_cast<unsigned int>(static_cast<unsigned long long>(nb) * (blockIdx.x + 1) / gridDim.x);
  if (qlo >= qhi) return;  // the whole block
  int g = 0;  // the group of batch qlo: the largest g with boff[g] <= qlo
  {
    int ghi = a.ng - 1;
    while (g < ghi) {
      const int mid = (g + ghi + 1) >> 1;
      if (a.boff[mid] <= qlo) g = mid; else ghi = mid - 1;
    }
  }
  unsigned int win0 = 0xffffffffu;
  auto window = [&](unsigned int p0) {  // every thread; a barrier must follow
    for (int t = tid; t < CB_WIN; t += 256) rs[t] = p0 + t < ntot ? a.srow[p0 + t] : 0xffffffffu;
    win0 = p0;
  };
  auto first = [&](unsigned int q, int gg) { return a.goff[gg] + (q - a.boff[gg]) * 32u; };
  // registers of the slab loaded ahead
  float pv[32 * CB_KD / 256], cv[8 * CB_KD / 256];
  bool cst = false;
  uint32_t row_n = 0xffffffffu;
  int jc_n = -1, g_cs = -1;
  auto issue = [&](unsigned int q, int gg, int kc) {
    const unsigned int q0 = first(q, gg), q1 = min(q0 + 32u, a.goff[gg + 1]);
    const int k0 = kc * CB_KD, kn = min(CB_KD, dim - k0);
#pragma unroll
    for (int u = 0; u < 32 * CB_KD / 256; ++u) {
      const int e = tid + u * 256, pr = e / CB_KD, kk = e % CB_KD;
      const uint32_t row = q0 + pr < q1 ? rs[q0 + pr - win0] : 0xffffffffu;
      pv[u] = (row != 0xffffffffu && kk < kn) ? __ldg(a.P + static_cast<int64_t>(row) * dim + k0 + kk) : 0.f;
    }
    cst = nk > 1 || gg != g_cs;
    if (cst) {
#pragma unroll
      for (int u = 0; u < 8 * CB_KD / 256; ++u) {
        const int e = tid + u * 256, cr = e / CB_KD, kk = e % CB_KD;
        const int64_t sp = static_cast<int64_t>(gg) * 8 + cr;
        const int jj = sp < a.m ? __ldg(a.perm + sp) : -1;
        cv[u] = (jj >= 0 && kk < kn) ? __ldg(a.C + static_cast<int64_t>(jj) * dim + k0 + kk) : 0.f;
      }
    }
    row_n = q0 + r < q1 ? rs[q0 + r - win0] : 0xffffffffu;
    const int64_t sc = static_cast<int64_t>(gg) * 8 + c;
    jc_n = sc < a.m ? __ldg(a.perm + sc) : -1;
  };

  unsigned int q = qlo;
  int kc = 0;
  window(first(q, g));
  __syncthreads();
  issue(q, g, kc);
  DirectAcc<REC> acc;
  unsigned long long evals = 0;
  while (true) {
    __syncthreads();  // the previous slab is summed: ps and cs are free
#pragma unroll
    for (int u = 0; u < 32 * CB_KD / 256; ++u) {
      const int e = tid + u * 256;
      ps[e / CB_KD][e % CB_KD] = pv[u];
    }
    if (cst) {
#pragma unroll
      for (int u = 0; u < 8 * CB_KD / 256; ++u) {
        const int e = tid + u * 256;
        cs[e / CB_KD][e % CB_KD] = cv[u];
      }
      g_cs = g;
    }
    const uint32_t row = row_n;
    const int jc = jc_n;
    const int kn = min(CB_KD, dim - kc * CB_KD);
    const bool last = kc == nk - 1;
    // the next slab, and the window of its rows
    unsigned int qn = q;
    int kcn = kc + 1, gn = g;
    if (kcn == nk) {
      kcn = 0;
      ++qn;
      while (qn < qhi && a.boff[gn + 1] <= qn) ++gn;
    }
    const bool more = qn < qhi;
    if (more && kcn == 0) {
      const unsigned int q0n = first(qn, gn), q1n = min(q0n + 32u, a.goff[gn + 1]);
      if (q0n < win0 || q1n > win0 + CB_WIN) window(q0n);
    }
    __syncthreads();  // the slab and the window are in shared memory
    if (more) issue(qn, gn, kcn);
    for (int kk = 0; kk < kn; ++kk) acc.add(ps[r][kk], cs[c][kk]);
    if (last) {
      unsigned long long key = ~0ull;
      if (row != 0xffffffffu && jc >= 0) {
        key = make_key(static_cast<float>(acc.get()), static_cast<uint32_t>(jc));
        ++evals;
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other < key ? other : key;
      }
      if (c == 0 && row != 0xffffffffu) atomicMin(a.row_key + row, key);
      acc = DirectAcc<REC>();
    }
    if (!more) break;
    q = qn;
    kc = kcn;
    g = gn;
  }
  evals = __reduce_add_sync(0xffffffffu, static_cast<unsigned int>(evals));
  if ((tid & 31) == 0 && evals) atomicAdd(a.count, evals);
}

// By group: every row's outputs from its key -- rows its group decided and rows of the
// second screen; rows whose entries overflowed (redo 2) or found no key go to the rows
// evaluated whole (thr NaN: listed already).
__global__ void __launch_bounds__(256) cert_out_kernel(const CertArgs a) {
  const int lane = threadIdx.x & 31;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x; base < a.n;
       base += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = base + threadIdx.x;
    bool push = false;
    if (i < a.n) {
      const float t = a.thr[i];
      if (t == t) {
        const unsigned long long k = a.row_key[i];
        push = a.redo[i] != 0 || k == ~0ull;
        if (!push) cert_write(a, i, k);
      }
    }
    const unsigned int bal = __ballot_sync(0xffffffffu, push);
    if (bal) {
      unsigned int b = 0;
      if (lane == 0) b = atomicAdd(a.nrows, static_cast<unsigned int>(__popc(bal)));
      b = __shfl_sync(0xffffffffu, b, 0);
      if (push) a.rows[b + __popc(bal & ((1u << lane) - 1u))] = static_cast<uint32_t>(i);
    }
  }
}

// Listed rows: one warp per row, lanes over the centers, first index of the minimum.
template <int REC>
__global__ void __launch_bounds__(256) cert_whole_rows_kernel(const CertArgs a) {
  const int lane = threadIdx.x & 31;
  const unsigned int nr = *a.nrows;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  unsigned long long evals = 0;
  for (int64_t r = gw; r < nr; r += nw) {
    const int64_t i = a.rows[r];
    const float* p = a.P + i * a.dim;
    unsigned long long best = ~0ull;
    for (int64_t j = lane; j < a.m; j += 32) {
      const double v = direct_dist<float, REC>(p, a.C + j * a.dim, a.dim);
      const unsigned long long k = make_key(static_cast<float>(v), static_cast<uint32_t>(j));
      best = k < best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other < best ? other : best;
    }
    if (lane == 0) {
      cert_write(a, i, best);
      evals += static_cast<unsigned long long>(a.m);
    }
  }
  if (lane == 0 && evals) atomicAdd(a.count, evals);
}

// The second screen's listed groups: 8 direct distances each (four entries per warp),
// folded into the row's key with one 64-bit atomicMin.
template <int REC>
__global__ void __launch_bounds__(256) cert_groups_kernel(const CertArgs a) {
  constexpr int kBlocksPerRegion = 8;
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int t = lane & 7;
  const int r = blockIdx.x / kBlocksPerRegion;
  const uint32_t wr = (blockIdx.x % kBlocksPerRegion) * 8 + wib;
  constexpr uint32_t kStride = kBlocksPerRegion * 8 * 4;
  unsigned long long cnt64 = a.region_cnt[r];
  if (cnt64 > a.region_cap) cnt64 = a.region_cap;
  const uint32_t cnt = static_cast<uint32_t>(cnt64);
  const unsigned long long* gl = a.glist + static_cast<unsigned long long>(r) * a.region_cap;
  unsigned long long evals = 0;
  for (uint32_t t0 = wr * 4; t0 < cnt; t0 += kStride) {
    const uint32_t q = t0 + (lane >> 3);
    unsigned long long best = ~0ull;
    int64_t i = -1;
    if (q < cnt) {
      const unsigned long long e = gl[q];
      i = static_cast<int64_t>(e >> 32);
      const int64_t s = static_cast<int64_t>(e & 0xffffffffull) + t;
      // a row whose entries overflowed (redo 2) is evaluated whole instead
      if (i < a.n && s < a.m && a.redo[i] == 0) {
        const int j = __ldg(a.perm + s);
        const double v = direct_dist<float, REC>(a.P + i * a.dim, a.C + static_cast<int64_t>(j) * a.dim, a.dim);
        best = make_key(static_cast<float>(v), static_cast<uint32_t>(j));
        ++evals;
      }
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other < best ? other : best;
    }
    if (t == 0 && i >= 0 && i < a.n && best != ~0ull) atomicMin(a.row_key + i, best);
  }
  evals = __reduce_add_sync(0xffffffffu, static_cast<unsigned int>(evals));
  if (lane == 0 && evals) atomicAdd(a.count, evals);
}

// Rows of the second screen: outputs from the key, or (list overflow, redo 2) to the
// rows evaluated whole.
__global__ void __launch_bounds__(256) cert_second_rows_kernel(const CertArgs a) {
  const float kInf = __int_as_float(0x7f800000);
  const int lane = threadIdx.x & 31;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x; base < a.n;
       base += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = base + threadIdx.x;
    bool push = false;
    if (i < a.n && a.thr[i] > -kInf) {
      const unsigned long long k = a.row_key[i];
      push = a.redo[i] != 0 || k == ~0ull;
      if (!push) cert_write(a, i, k);
    }
    const unsigned int bal = __ballot_sync(0xffffffffu, push);
    if (bal) {
      unsigned int b = 0;
      if (lane == 0) b = atomicAdd(a.nrows, static_cast<unsigned int>(__popc(bal)));
      b = __shfl_sync(0xffffffffu, b, 0);
      if (push) a.rows[b + __popc(bal & ((1u << lane) - 1u))] = static_cast<uint32_t>(i);
    }
  }
}

static CertArgs cert_args(const DistJob& j, int64_t* labels, int32_t* labels32, float* mind) {
  const OpSpec* s = j.spec;
  CertArgs a{};
  a.P = static_cast<const float*>(j.P);
  a.C = static_cast<const float*>(j.C);
  a.n = j.n;
  a.m = j.m;
  a.dim = j.dim;
  a.perm = j.perm;
  a.pp = static_cast<const float*>(j.pp);
  a.ccmax = j.ccmax;
  a.redo = j.redo;
  a.key = j.cert_key;
  a.d2 = j.cert_d2;
  a.thr = j.cert_thr;
  a.tiles = j.cert_tiles;
  a.row_key = j.row_key;
  a.glist = j.chunk_list;
  a.region_cap = j.regions > 0 ? j.chunk_cap / static_cast<unsigned long long>(j.regions) : 0;
  a.region_cnt = j.region_cnt;
  a.regions = j.regions;
  a.rows = j.cert_rows;
  a.nrows = j.cert_nrows;
  a.ng = j.cert_ng;
  a.ent = j.cert_ent;
  a.ent_n = j.cert_ent_n;
  a.ent_cap = j.cert_ent_cap;
  a.gcnt = j.cert_gcnt;
  a.goff = j.cert_goff;
  a.boff = j.cert_goff + (j.cert_ng + 1);
  a.srow = j.cert_srow;
  a.gather = j.cert_gather;
  a.F = j.cert_F;
  a.nF = j.cert_nF;
  a.pg = j.cert_pg;
  a.thr_g = j.cert_thr_g;
  a.redo_g = j.cert_redo_g;
  a.plow = j.Plow;
  a.ldlow = j.ldlow;
  a.lowkind = j.spec->gemm == G_TC_BF16 ? 1 : 0;
  a.count = j.count;
  a.labels = labels;
  a.labels32 = labels32;
  a.mind = mind;
  const bool bf16 = s->gemm == G_TC_BF16;
  const bool f16 = s->gemm == G_TC_F16;
  a.u = bf16 ? 0x1p-8 : 0x1p-11;  // fp16, tf32 (cvt.rna): 11 significant bits; bf16: 8
  // the screen's norms are fp32 sums of squares of the rounded operands (NM_OPERAND): the
  // products are exact, the sum's relative error is at most (dim + 2) 2^-24, and squares
  // below fp32's normal range lose at most 2^-149 each
  a.un = (static_cast<double>(j.dim) + 2.0) * 0x1p-24 * 1.01;
  a.eta_n = (static_cast<double>(j.dim) + 1.0) * 0x1p-149;
  a.gmma = (static_cast<double>(j.ldlow) + 32.0) * 0x1p-22;
  a.gd = (static_cast<double>(j.dim) + 4.0) * 0x1p-24 * 1.01 + 0x1p-24;
  a.eta = f16 ? 0x1p-25 : 0x1p-133;
  a.sqd = std::sqrt(static_cast<double>(j.dim));
  return a;
}

static bool cert_job_ok(const DistJob& j) {
  const OpSpec* s = j.spec;
  return s->in == IN_F32 && (s->rec == RC_F32 || s->rec == RC_F64) && j.cert_key && j.cert_d2 && j.cert_thr &&
         j.cert_tiles && j.ccmax && j.cert_rows && j.cert_nrows && j.redo && j.perm && j.row_key && j.chunk_list &&
         j.region_cnt && j.regions > 0;
}

cudaError_t launch_cert_rows(const DistJob& j, int64_t* labels, int32_t* labels32, float* mind) {
  if (!cert_job_ok(j)) return cudaErrorInvalidValue;
  const CertArgs a = cert_args(j, labels, labels32, mind);
  if (a.ng > 0) {
    const int blocks = static_cast<int>(std::min<int64_t>((j.n + 255) / 256, static_cast<int64_t>(num_sms()) * 8));
    cert_decide_kernel<<<blocks, 256, 0, j.stream>>>(a);
    return cudaGetLastError();
  }
  const int64_t nq = (j.n + 3) / 4;
  const int blocks = static_cast<int>(std::min<int64_t>((nq + 7) / 8, static_cast<int64_t>(num_sms()) * 8));
  if (j.spec->rec == RC_F32)
    cert_rows_kernel<RC_F32><<<blocks, 256, 0, j.stream>>>(a);
  else
    cert_rows_kernel<RC_F64><<<blocks, 256, 0, j.stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_cert_compact(const DistJob& j) {
  if (!cert_job_ok(j) || !j.cert_gather || j.spec->gemm == G_TC_TF32) return cudaErrorInvalidValue;
  const CertArgs a = cert_args(j, nullptr, nullptr, nullptr);
  const int blocks = num_sms() * 8;
  if (a.lowkind == 0)
    cert_compact_kernel<0><<<blocks, 256, 0, j.stream>>>(a);
  else
    cert_compact_kernel<1><<<blocks, 256, 0, j.stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_cert_finish(const DistJob& j, int64_t* labels, int32_t* labels32, float* mind) {
  if (!cert_job_ok(j)) return cudaErrorInvalidValue;
  const CertArgs a = cert_args(j, labels, labels32, mind);
  const int gblocks = j.regions * 8;
  const int sblocks = static_cast<int>(std::min<int64_t>((j.n + 255) / 256, static_cast<int64_t>(num_sms()) * 8));
  const int wblocks = num_sms() * 8;
  const bool f32 = j.spec->rec == RC_F32;
  if (a.ng > 0) {
    // by group: the second screen's entries join the decided rows', sorted by group
    const size_t hist = static_cast<size_t>(a.ng) * 4;
    cudaError_t e = cudaFuncSetAttribute(cert_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(hist));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(cert_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(2 * hist));
    if (e != cudaSuccess) return e;
    cert_gather_kernel<<<gblocks, 256, 0, j.stream>>>(a);
    if (a.gather) cert_relay_redo_kernel<<<wblocks, 256, 0, j.stream>>>(a);
    cert_count_kernel<<<wblocks, 256, hist, j.stream>>>(a);
    cert_scan_kernel<<<1, 1024, 0, j.stream>>>(a.gcnt, a.goff, a.boff, a.ng);
    cert_scatter_kernel<<<wblocks, 256, 2 * hist, j.stream>>>(a);
    if (f32)
      cert_bucket_kernel<RC_F32><<<wblocks, 256, 0, j.stream>>>(a);
    else
      cert_bucket_kernel<RC_F64><<<wblocks, 256, 0, j.stream>>>(a);
    cert_out_kernel<<<sblocks, 256, 0, j.stream>>>(a);
  } else {
    if (f32)
      cert_groups_kernel<RC_F32><<<gblocks, 256, 0, j.stream>>>(a);
    else
      cert_groups_kernel<RC_F64><<<gblocks, 256, 0, j.stream>>>(a);
    cert_second_rows_kernel<<<sblocks, 256, 0, j.stream>>>(a);
  }
  if (f32)
    cert_whole_rows_kernel<RC_F32><<<wblocks, 256, 0, j.stream>>>(a);
  else
    cert_whole_rows_kernel<RC_F64><<<wblocks, 256, 0, j.stream>>>(a);
  return cudaGetLastError();
}

}  // namespace euc
