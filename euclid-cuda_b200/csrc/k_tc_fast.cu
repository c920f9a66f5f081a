// Fused distance + argmin on the tensor cores, screening form (sm_100a).
//
// TMA -> 128B-swizzled smem -> tcgen05.mma -> TMEM, with an epilogue reduced to what
// an argmin needs, so that it keeps pace with the tensor cores:
//
//  * a CTA owns 128 rows at a time (A resident in shared memory, double-buffered) while
//    the 256-center tiles stream past, one M=128, N=256 MMA per K step;
//  * TMEM holds two 256-column accumulators (tile parity b); the 16 epilogue warps form
//    4 groups (b, column half), one warp per TMEM lane quadrant, so a group has two
//    tile times to drain its half of an accumulator while the next tile's MMAs proceed;
//  * centers arrive sorted by norm (stable); a 4-slot ring of 1-D bulk copies brings
//    each center tile's norms into shared memory ahead of use, and the tile's extra-K
//    rows ride in the stage of its last K block;
//  * one extra 32-byte K block (aux.cuh) adds y0 = (cc_j + Br_i)/2 to the accumulator of
//    pair (i, j) (Br_i = 1.0625 pp_i, centers stored negated), so the MMA yields
//    y = y0 - s >= 0 directly; per 32-column chunk an epilogue warp replaces the low 5
//    mantissa bits of y with the column (one LOP3) and takes the minimum with a
//    depth-4 tree of 3-way mins;
//  * two row warps build each row tile's extra-K rows and its norms; for the fp16/bf16
//    operators whose norms are those of the rounded values they also take the fp32
//    points themselves (FUSED): the next row tile's points arrive by TMA in a staging
//    buffer while the current one is used, and the row warps round them into the
//    128B-swizzled A tile, accumulating the norms in dimension order, so no
//    low-precision copy of the points is written to HBM;
//  * a chunk in which some pair could meet the cancellation test
//        d <= K (pp + cc)  <=>  2 s >= (1 - K)(pp + cc)  (up to rounding margins)
//    -- bounded with the chunk's smallest and largest norm, tight because norms are
//    sorted -- is not resolved here: its (row, chunk) and its 32 fp32 accumulators are
//    appended to a list that eval_chunks_kernel evaluates with the operator's exact
//    arithmetic on s = y0 - y (the same rounding of S, distance formula and cancellation
//    test as the exact epilogue; flagged pairs go to the direct-recompute list);
//  * every other chunk can hold no flagged pair and contributes its key minimum.
//
// Labels equal the exact epilogue's wherever the row's top-two distance gap exceeds
// the screen's resolution: 2^-10 (pp + max cc) for fp16 S (2^-7 for bf16 S) plus the
// key truncation, 2^-16 (max cc + Br).  If the candidate list is full, or the row's
// norm does not fit the extra K block, the row is marked for a complete exact redo.
//
// All waits are bounded (common.cuh); on expiry the CTA records an error, drains its
// copies and MMAs, frees TMEM and returns.
#include "common.cuh"
#include "engine.h"
#include "../../include/euclid_b200.h"
#include "direct.cuh"
#include "aux.cuh"

#include <cudaTypedefs.h>
#include <algorithm>
#include <atomic>

namespace euc {

static __device__ int s_tf_err;

// A CTA tile is 128 rows by 256 centers: one M=128, N=256 MMA per K step (on this part
// an MMA instruction costs the same time for N = 128 and N = 256, so N = 256 doubles the
// rate); TMEM holds 2 accumulators of 256 columns, one per tile parity b.
constexpr int TF_BM = 128;
constexpr int TF_BN = 256;
constexpr int TF_EPI_WARPS = 16;  // 4 groups (b, column half) x 4 TMEM lane quadrants
constexpr int TF_ROW_WARPS = 2;   // row preparation: one thread per two rows of the tile
constexpr int TF_ROW_THREADS = TF_ROW_WARPS * 32;
constexpr int TF_THREADS = (2 + TF_EPI_WARPS + TF_ROW_WARPS) * 32;
// warp roles; an epilogue warp reads TMEM lane quadrant warp % 4, so 16 consecutive
// epilogue warps give each (group, quadrant) pair one warp
constexpr int TF_W_PRODUCER = 0;
constexpr int TF_W_MMA = 1;
constexpr int TF_W_EPI0 = 2;
constexpr int TF_W_ROW0 = TF_W_EPI0 + TF_EPI_WARPS;
constexpr int TF_A_KB = TF_BM * 128;  // one 128-row x 128-byte K block of A
constexpr int TF_B_KB = TF_BN * 128;  // one 256-row x 128-byte K block of B
constexpr int TF_SLOTS = 4;             // center-metadata ring
constexpr int TF_BAUX_BYTES = TF_BN * 32;  // the tile's extra-K rows (32 bytes each)
constexpr int TF_META_BYTES = TF_BN * 4;  // the tile's sorted center norms
constexpr int TF_XBOX_BYTES = 32 * 4 * TF_BM;  // FUSED staging: 32 fp32 values of the 128 rows
constexpr int TF_AAUX_BYTES = TF_BM * 32;       // per A buffer: the rows' extra-K rows
constexpr int TF_ROWBUF_BYTES = 2 * TF_BM * 4;  // per A buffer: pp and Br of each row
constexpr int TF_BAR_BYTES = 512;

struct TfArgs {
  int64_t n, m;
  int kblocks, nst, a_res, n_ct;
  int64_t n_rt;
  float* pp;          // point norms (written here with FUSED)
  const float* X;     // FUSED: the fp32 points, dim % 4 == 0, 16-byte aligned
  int dim;
  const float* ccs;   // norms, sorted, padded to whole 256-center tiles
  const int* perm;    // sorted position -> original index, padded
  float omk, margin, ovf;
  float nlim;         // norms at or above this are not screened (their rows are redone)
  const int* aux_e;             // E of the extra K block (device scalar)
  unsigned long long* row_key;
  unsigned long long* list;     // candidate chunks: region r = list + r * region_cap
  float* sbuf;                  // their 32 accumulator values, same index
  unsigned long long region_cap;
  uint32_t* region_cnt;
  uint8_t* redo;
  unsigned long long* cert_key;  // certified: [4][n] (best screened distance, sorted start of its group)
  float* cert_d2;                // certified: [4][n] second-best screened distance outside that group
  const float* cert_thr;         // certified, second screen: per row, the largest screened distance of a
                                 // center that can win (-inf: the row is decided)
  const uint8_t* tile_on;        // null, or per row tile: whether it is screened
  unsigned long long wait_ns;    // bound of every wait of the pipeline
  int withhold;                  // failure injection: CTA 0's first epilogue warp keeps its first
                                 // accumulator (its MMA warp's wait then runs out)
};

// The CTA's next row tile at or after rt (same stride as the persistent loop), skipping
// the tiles switched off.  Every role walks the same sequence.
__device__ __forceinline__ int64_t tf_next_tile(const TfArgs& a, int64_t rt) {
  if (a.tile_on != nullptr)
    while (rt < a.n_rt && a.tile_on[rt] == 0) rt += gridDim.x;
  return rt;
}

// FUSED row preparation, one staged box: 32 fp32 values of row r of the row tile (TMA
// with the 128-byte swizzle: 16-byte chunk j of row r at r * 128 + ((j ^ r % 8) * 16))
// rounded to the operand type (fp16 / bf16, round to nearest even) into K block kq / 2,
// chunks 4 (kq % 2) .. + 3 of row r of A, K-major with the 128-byte swizzle the MMA
// descriptor names (chunk q of row r in K block kb at kb * 16K + (r / 8) * 1024 +
// (r % 8) * 128 + ((q ^ r % 8) * 16)); the row's norm continues over them: fused
// multiply-adds of the rounded values in dimension order (the NM_LOW_F16 /
// NM_LOW_BF16 recipes of the standalone preparation).
template <int KIND>
__device__ __forceinline__ float convert_box(const uint8_t* box, int r, uint8_t* sA, int kq, float acc) {
  static_assert(KIND == 0 || KIND == 1, "fp16 / bf16 operands");
  const uint8_t* src = box + r * 128;
  uint8_t* rowp = sA + (kq >> 1) * TF_A_KB + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const float4 p0 = *reinterpret_cast<const float4*>(src + (((2 * jj) ^ (r & 7)) << 4));
    const float4 p1 = *reinterpret_cast<const float4*>(src + (((2 * jj + 1) ^ (r & 7)) << 4));
    const float x[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      float lo, hi;
      if constexpr (KIND == 0) {
        const __half2 t = __floats2half2_rn(x[2 * h], x[2 * h + 1]);
        w[h] = *reinterpret_cast<const uint32_t*>(&t);
        lo = __low2float(t);
        hi = __high2float(t);
      } else {
        const __nv_bfloat162 t = __floats2bfloat162_rn(x[2 * h], x[2 * h + 1]);
        w[h] = *reinterpret_cast<const uint32_t*>(&t);
        lo = __low2float(t);
        hi = __high2float(t);
      }
      acc = __fmaf_rn(lo, lo, acc);
      acc = __fmaf_rn(hi, hi, acc);
    }
    const int q = 4 * (kq & 1) + jj;
    *reinterpret_cast<uint4*>(rowp + ((q ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  return acc;
}

// PAIR: the CTAs run in pairs (clusters of 2) with M = 256 MMAs across both SMs.  CTA
// rank r owns row tile 2 p + r of pair tile p and loads centers [128 r, 128 r + 128) of
// every 256-center tile, so each SM streams half of each center tile; rank 0 issues the
// MMAs and commits to both CTAs' barriers, and the barriers that collect both CTAs'
// events (stage full, A ready, accumulator read) are rank 0's.
template <int KIND, bool FUSED, int CERT, bool PAIR>
__global__ void __launch_bounds__(TF_THREADS, 1)
    dist_tc_fast_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmBaux, const TfArgs a) {
  static_assert(!PAIR || CERT == 0, "the certified passes run unpaired");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NST = a.nst;
  const bool a_res = a.a_res != 0;
  const int KB = a.kblocks;
  constexpr int BNL = PAIR ? TF_BN / 2 : TF_BN;        // center rows this CTA loads per tile
  constexpr uint32_t B_KB_L = BNL * 128;               // its part of one K block of B
  constexpr uint32_t BAUX_L = BNL * 32;                // its part of the tile's extra-K rows
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  const uint32_t a_bytes = static_cast<uint32_t>(KB) * TF_A_KB;                   // all K blocks of A
  // a stage: B  |  A B, then room for the tile's extra-K rows (used by its last K block)
  const uint32_t ab_bytes = a_res ? B_KB_L : static_cast<uint32_t>(TF_A_KB + B_KB_L);
  const uint32_t stage_bytes = ab_bytes + BAUX_L;
  uint8_t* stage_base = smem + (a_res ? 2 * a_bytes : 0);
  uint8_t* meta = stage_base + NST * stage_bytes;  // TF_SLOTS x 256 sorted norms
  const int nbox = (a.dim + 31) >> 5;              // FUSED: staged 32-value boxes per row
  uint8_t* xst = meta + TF_SLOTS * TF_META_BYTES;  // FUSED: the next row tile's fp32 points
  uint8_t* aaux = xst + (FUSED ? nbox * TF_XBOX_BYTES : 0);  // per A buffer: the A side of the extra K block
  float* rowbuf = reinterpret_cast<float*>(aaux + 2 * TF_AAUX_BYTES);  // per A buffer: pp[128], Br[128]
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(rowbuf) + 2 * TF_ROWBUF_BYTES);
  uint64_t* empty = full + NST;
  uint64_t* afull = empty + NST;
  uint64_t* aempty = afull + 2;
  uint64_t* accf = aempty + 2;   // per tile parity: the accumulator is complete
  uint64_t* acce = accf + 2;     // per tile parity: the accumulator was read
  uint64_t* metaf = acce + 2;
  uint64_t* metae = metaf + TF_SLOTS;
  uint64_t* pempty = metae + TF_SLOTS;  // per A buffer: every epilogue warp has read its rows' pp, Br
  uint64_t* xfull = pempty + 2;         // FUSED staging: the row tile's points have landed
  uint64_t* xempty = xfull + 1;         // FUSED staging: every row thread has read them
  uint64_t* drain = xempty + 1;
  unsigned long long* lcount = reinterpret_cast<unsigned long long*>(drain + 1);  // this CTA's list entries
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(lcount + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr uint32_t kCols = 2 * TF_BN;  // 512

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    // afull: the row warps' arrivals (rank 0's also the other CTA's), plus the producer's
    // A copy when A comes by TMA (rank 0's producer expects both CTAs' bytes)
    const uint32_t afull_count = (PAIR && leader ? 2u : 1u) * TF_ROW_THREADS + ((!FUSED && a_res && leader) ? 1u : 0u);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&afull[s], afull_count);
      mbar_init(&aempty[s], 1);
      mbar_init(&pempty[s], TF_EPI_WARPS);
      if (s == 0) {
        mbar_init(xfull, 1);
        mbar_init(xempty, TF_ROW_THREADS);
      }
      mbar_init(&accf[s], 1);
      mbar_init(&acce[s], (PAIR ? 2 : 1) * TF_EPI_WARPS / 2);
    }
    for (int s = 0; s < TF_SLOTS; ++s) {
      mbar_init(&metaf[s], 1);
      mbar_init(&metae[s], TF_EPI_WARPS / 2);
    }
    mbar_init(drain, 1);
    *lcount = 0;
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == TF_W_MMA) {
    if constexpr (PAIR)
      tmem_alloc_pair(tmem_slot, kCols);
    else
      tmem_alloc(tmem_slot, kCols);
  }
  if (warp == TF_W_PRODUCER && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmBaux);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers are initialised before any remote use
  tc_fence_after();
  // rank 0's copies of the barriers that collect both CTAs' events
  const uint32_t full_c0 = PAIR ? cluster_addr(full, 0) : 0u;
  const uint32_t afull_c0 = PAIR ? cluster_addr(afull, 0) : 0u;
  const uint32_t acce_c0 = PAIR ? cluster_addr(acce, 0) : 0u;
  const uint32_t tmem_base = *tmem_slot;

  if (warp == TF_W_PRODUCER) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, rt_i = 0, t = 0;
      uint32_t issued_mask = 0, last_phase = 0, a_issued = 0, a_last = 0, m_issued = 0, m_last = 0;
      bool ok = true;
      const int kelems = (KIND == 2) ? 32 : 64;
      for (int64_t rt = tf_next_tile(a, blockIdx.x); rt < a.n_rt && ok; rt = tf_next_tile(a, rt + gridDim.x), ++rt_i) {
        const uint32_t abuf = rt_i & 1u, ause = (rt_i >> 1) & 1u;
        const int row0 = static_cast<int>(rt * TF_BM);
        if (!FUSED && a_res) {
          if (!(PAIR ? mbar_wait_cluster(&aempty[abuf], ause ^ 1u, abort_flag, a.wait_ns)
                     : mbar_wait(&aempty[abuf], ause ^ 1u, abort_flag, a.wait_ns))) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + abuf * a_bytes;
          if constexpr (PAIR) {
            if (leader) mbar_arrive_expect_tx(&afull[abuf], 2 * a_bytes);
            for (int kb = 0; kb < KB; ++kb)
              tma_load_2d_pair(sA + kb * TF_A_KB, &tmA, afull_c0 + 8u * abuf, kb * kelems, row0);
          } else {
            mbar_arrive_expect_tx(&afull[abuf], a_bytes);
            for (int kb = 0; kb < KB; ++kb)
              tma_load_2d(sA + kb * TF_A_KB, &tmA, &afull[abuf], kb * kelems, row0);
          }
          a_issued |= 1u << abuf;
          a_last = (a_last & ~(1u << abuf)) | (ause << abuf);
        }
        for (int ct = 0; ct < a.n_ct && ok; ++ct, ++t) {
          const uint32_t slot = t & (TF_SLOTS - 1), su = (t / TF_SLOTS) & 1u;
          if (!mbar_wait(&metae[slot], su ^ 1u, abort_flag, a.wait_ns)) { ok = false; break; }
          uint8_t* ms = meta + slot * TF_META_BYTES;
          mbar_arrive_expect_tx(&metaf[slot], TF_META_BYTES);
          bulk_load_1d(ms, a.ccs + static_cast<int64_t>(ct) * TF_BN, TF_BN * 4, &metaf[slot]);
          m_issued |= 1u << slot;
          m_last = (m_last & ~(1u << slot)) | (su << slot);
          for (int kb = 0; kb < KB; ++kb) {
            if (!(PAIR ? mbar_wait_cluster(&empty[stage], phase ^ 1u, abort_flag, a.wait_ns)
                       : mbar_wait(&empty[stage], phase ^ 1u, abort_flag, a.wait_ns))) {
              ok = false;
              break;
            }
            uint8_t* st = stage_base + stage * stage_bytes;
            const bool last_kb = kb == KB - 1;
            if constexpr (PAIR) {
              // this CTA's half of the center tile, completing on rank 0's stage barrier
              const uint32_t fb = full_c0 + 8u * stage;
              const int yb = ct * TF_BN + static_cast<int>(rank) * BNL;
              if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (last_kb ? stage_bytes : ab_bytes));
              if (a_res) {
                tma_load_2d_pair(st, &tmB, fb, kb * kelems, yb);
              } else {
                tma_load_2d_pair(st, &tmA, fb, kb * kelems, row0);
                tma_load_2d_pair(st + TF_A_KB, &tmB, fb, kb * kelems, yb);
              }
              if (last_kb) tma_load_2d_pair(st + ab_bytes, &tmBaux, fb, 0, yb);
            } else {
              mbar_arrive_expect_tx(&full[stage], last_kb ? stage_bytes : ab_bytes);
              if (a_res) {
                tma_load_2d(st, &tmB, &full[stage], kb * kelems, ct * TF_BN);
              } else {
                tma_load_2d(st, &tmA, &full[stage], kb * kelems, row0);
                tma_load_2d(st + TF_A_KB, &tmB, &full[stage], kb * kelems, ct * TF_BN);
              }
              if (last_kb) tma_load_2d(st + ab_bytes, &tmBaux, &full[stage], 0, ct * TF_BN);
            }
            issued_mask |= 1u << stage;
            last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
            if (++stage == static_cast<uint32_t>(NST)) { stage = 0; phase ^= 1u; }
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(&s_tf_err, DEV_TIMEOUT_PRODUCER);
      }
      volatile int no_abort = 0;
      // copies in flight land before the CTA exits (rank 1's copies complete on rank 0's
      // barriers, which rank 0 drains before the closing cluster barrier)
      if (!PAIR || leader) {
        for (int s = 0; s < NST; ++s)
          if (issued_mask & (1u << s)) mbar_wait_cluster(&full[s], (last_phase >> s) & 1u, &no_abort);
        for (int s = 0; s < 2; ++s)
          if (a_issued & (1u << s)) mbar_wait_cluster(&afull[s], (a_last >> s) & 1u, &no_abort);
      }
      for (int s = 0; s < TF_SLOTS; ++s)
        if (m_issued & (1u << s)) mbar_wait(&metaf[s], (m_last >> s) & 1u, &no_abort);
    }
  } else if (warp == TF_W_MMA) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t fmt = (KIND == 0) ? 0u : (KIND == 1 ? 1u : 2u);
      constexpr uint32_t idesc = umma_idesc(fmt, PAIR ? 256 : 128, TF_BN);
      uint32_t stage = 0, phase = 0, t = 0, rt_i = 0;
      bool ok = true;
      for (int64_t rt = tf_next_tile(a, blockIdx.x); rt < a.n_rt && ok; rt = tf_next_tile(a, rt + gridDim.x), ++rt_i) {
        const uint32_t abuf = rt_i & 1u, ause = (rt_i >> 1) & 1u;
        const uint32_t sAres = smem_u32(smem + abuf * a_bytes);
        const uint64_t aux_ad = sw32_kmajor_desc(smem_u32(aaux + abuf * TF_AAUX_BYTES));
        // the row tile's extra-K rows (and its resident A), in both CTAs with PAIR
        if (!mbar_wait_cluster(&afull[abuf], ause, abort_flag, a.wait_ns)) { ok = false; break; }
        for (int ct = 0; ct < a.n_ct && ok; ++ct, ++t) {
          const uint32_t b = t & 1u, use = (t >> 1) & 1u;
          if (!mbar_wait_cluster(&acce[b], use ^ 1u, abort_flag, a.wait_ns)) { ok = false; break; }
          tc_fence_after();
          for (int kb = 0; kb < KB; ++kb) {
            if (!mbar_wait_cluster(&full[stage], phase, abort_flag, a.wait_ns)) { ok = false; break; }
            tc_fence_after();
            const uint32_t st = smem_u32(stage_base + stage * stage_bytes);
            const uint32_t sA = a_res ? sAres + kb * TF_A_KB : st;
            const uint32_t sB = a_res ? st : st + TF_A_KB;
            const uint32_t d_tmem = tmem_base + b * TF_BN;
            // K step kk starts 32 bytes further: +2 in the descriptor's address field (in
            // 16-byte units; shared addresses stay below 2^18, so the field never carries)
            const uint64_t ad0 = sw128_kmajor_desc(sA), bd0 = sw128_kmajor_desc(sB);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = ad0 + 2u * kk;
              const uint64_t bd = bd0 + 2u * kk;
              if constexpr (KIND == 2) {
                if constexpr (PAIR) umma_tf32_pair(d_tmem, ad, bd, idesc, (kb | kk) != 0);
                else umma_tf32(d_tmem, ad, bd, idesc, (kb | kk) != 0);
              } else {
                if constexpr (PAIR) umma_f16_pair(d_tmem, ad, bd, idesc, (kb | kk) != 0);
                else umma_f16(d_tmem, ad, bd, idesc, (kb | kk) != 0);
              }
            }
            if (kb == KB - 1) {
              // the extra K block: adds (cc_j + Br_i) / 2 to the accumulator of pair (i, j)
              const uint64_t bd = sw32_kmajor_desc(st + ab_bytes);
              if constexpr (KIND == 2) {
                if constexpr (PAIR) umma_tf32_pair(d_tmem, aux_ad, bd, idesc, 1u);
                else umma_tf32(d_tmem, aux_ad, bd, idesc, 1u);
              } else {
                if constexpr (PAIR) umma_f16_pair(d_tmem, aux_ad, bd, idesc, 1u);
                else umma_f16(d_tmem, aux_ad, bd, idesc, 1u);
              }
            }
            if constexpr (PAIR) umma_commit_pair(&empty[stage]);
            else umma_commit(&empty[stage]);
            if (++stage == static_cast<uint32_t>(NST)) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          if constexpr (PAIR) umma_commit_pair(&accf[b]);
          else umma_commit(&accf[b]);
        }
        if (ok) {
          if constexpr (PAIR) umma_commit_pair(&aempty[abuf]);
          else umma_commit(&aempty[abuf]);
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(&s_tf_err, DEV_TIMEOUT_MMA);
      }
      if constexpr (PAIR) umma_commit_pair(drain);
      else umma_commit(drain);
    }
    if (lane == 0) {
      // every MMA of the CTA (with PAIR: of the pair) has completed
      volatile int no_abort = 0;
      if (PAIR) mbar_wait_cluster(drain, 0, &no_abort);
      else mbar_wait(drain, 0, &no_abort);
    }
  } else if (warp >= TF_W_EPI0 && warp < TF_W_EPI0 + TF_EPI_WARPS) {
    // ------------------------------------------------------------ epilogue
    // The accumulators hold y = (cc + Br) / 2 - s >= 0 (the extra K block adds the first
    // term), so a row's smallest distance in a chunk is its smallest y: keys are y with
    // the column in the low 5 mantissa bits, reduced with 3-way mins.
    const int ew = warp - TF_W_EPI0;    // 0..15
    const int q = warp & 3;             // TMEM lane quadrant
    const int g = ew >> 2;              // group: tile parity b = g >> 1, column half hc = g & 1
    const int hc = g & 1;
    const uint32_t b = static_cast<uint32_t>(g >> 1);
    const int row_local = q * 32 + lane;
    const uint32_t tmem_acc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * TF_BN + hc * 128;
    unsigned long long* region = a.list + static_cast<unsigned long long>(blockIdx.x) * a.region_cap;
    float* region_s = a.sbuf + static_cast<unsigned long long>(blockIdx.x) * a.region_cap * 32;
    // screen: a pair can only be flagged (d <= K (pp + cc)) where
    //   y <= (cc + Br - (1 - K)(pp + cc)) / 2,
    // so a chunk is a candidate when its smallest y <= thr = U_c + V, with
    //   U_c = (max cc (1 + margin) - (1 - K) min cc) / 2 over the chunk,
    //   V   = (Br (1 + margin) + pp (margin - (1 - K))) / 2 per row
    // ~31 in a register the compiler cannot fold, so that the column insertion below is
    // one three-input logic op per element
    uint32_t kmask;
    asm volatile("mov.b32 %0, %1;" : "=r"(kmask) : "r"(~31u));
    const float kInf = __int_as_float(0x7f800000);
    uint32_t rt_i = 0, t = 0, uses = 0;
    bool ok = true;
    for (int64_t rt = tf_next_tile(a, blockIdx.x); rt < a.n_rt && ok; rt = tf_next_tile(a, rt + gridDim.x), ++rt_i) {
      const int64_t i = rt * TF_BM + row_local;
      // the row's norm and Br from the row warps (Br NaN: past n, or redone whole)
      const uint32_t abuf = rt_i & 1u;
      if (!mbar_wait(&afull[abuf], (rt_i >> 1) & 1u, abort_flag, a.wait_ns)) { ok = false; break; }
      const float pp = rowbuf[abuf * 2 * TF_BM + row_local];
      const float br = rowbuf[abuf * 2 * TF_BM + TF_BM + row_local];
      __syncwarp();
      if (lane == 0) mbar_arrive(&pempty[abuf]);
      const bool row_ok = i < a.n && br == br;
      const float vlane = 0.5f * __fmaf_rn(br, 1.f + a.margin, pp * (a.margin - a.omk));
      // certified, second screen: the row's threshold on y (a group is listed when its
      // smallest key is at or below), from its distance threshold T: y = (T + Br - pp) / 2,
      // raised by 2^-16 of the magnitudes for the key truncation and the fp32 roundings
      float yt = -kInf;
      if constexpr (CERT == 2) {
        const float T = row_ok ? __ldg(a.cert_thr + i) : -kInf;
        if (T > -kInf) {
          const float h = 0.5f * __fadd_rn(__fadd_rn(T, br), -pp);
          yt = h + (fabsf(h) + fabsf(T) + br + pp) * 0x1p-16f;
        }
      }
      // best screened key of the row: y with its column in the low 5 bits, and the first
      // sorted column of its chunk
      float best_y = kInf;
      float sec_y = kInf;  // certified: second-best group minimum of the row
      uint32_t best_c = 0;
      for (int ct = 0; ct < a.n_ct; ++ct, ++t) {
        if ((t & 1u) != b) continue;  // the other parity's groups take this tile
        const uint32_t use = uses & 1u;
        ++uses;
        const uint32_t slot = t & (TF_SLOTS - 1), su = (t / TF_SLOTS) & 1u;
        const int64_t jt = static_cast<int64_t>(ct) * TF_BN + hc * 128;  // first (sorted) column of this warp
        if (!mbar_wait(&metaf[slot], su, abort_flag, a.wait_ns)) { ok = false; break; }
        const float* mcc = reinterpret_cast<const float*>(meta + slot * TF_META_BYTES) + hc * 128;
        const int64_t remt = a.m - jt;
        const int nvt = remt <= 0 ? 0 : (remt >= 128 ? 128 : static_cast<int>(remt));
        float u_own = 0.f;  // lane L < 4: U of chunk L
        if (lane < 4 && lane * 32 < nvt) {
          const int last = min(lane * 32 + 31, nvt - 1);
          u_own = 0.5f * (mcc[last] * (1.f + a.margin) - a.omk * mcc[lane * 32]);
        }
        const float ccmax_t = nvt > 0 ? mcc[nvt - 1] : 0.f;
        // rows whose S may overflow its rounded format, or whose norms (or this tile's)
        // are not finite, list every chunk
        const bool lane_exact = !(pp < a.nlim && ccmax_t < a.nlim && pp * ccmax_t <= a.ovf);
        const float vl = row_ok ? vlane : -kInf;  // rows past n never list a chunk
        const bool force = row_ok && lane_exact;
        if constexpr (CERT != 0) {
          if (force) a.redo[i] = 1;  // the certified pass evaluates this row whole
        }
        const int nch = (nvt + 31) >> 5;
        if (!(PAIR ? mbar_wait_cluster(&accf[b], use, abort_flag, a.wait_ns)
                   : mbar_wait(&accf[b], use, abort_flag, a.wait_ns))) {
          ok = false;
          break;
        }
        tc_fence_after();

        uint32_t cmask = 0;  // this lane's candidate chunks of the tile
        uint32_t gmask = 0;  // certified, second screen: bit 4 ch + u for group u of chunk ch
#pragma unroll 1
        for (int ch = 0; ch < nch; ++ch) {
          float v[32];
          tmem_ld32(tmem_acc + ch * 32, v);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            uint32_t kb;
            asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(kb) : "r"(__float_as_uint(v[e])), "r"(kmask), "r"(static_cast<uint32_t>(e)));
            v[e] = __uint_as_float(kb);
          }
          float km;
          bool cand = false;
          if constexpr (CERT != 0) {
            // four groups of 8 columns: the chunk's minimum, its second-smallest group
            // minimum, and the row's best and second-best group minima.  Padded
            // centers give NaN keys: fminf skips them and max.NaN keeps them out of
            // the second-best (NaN acts as +inf).
            float gm[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              gm[u] = fmin3(fmin3(v[8 * u], v[8 * u + 1], v[8 * u + 2]), fmin3(v[8 * u + 3], v[8 * u + 4], v[8 * u + 5]),
                            fminf(v[8 * u + 6], v[8 * u + 7]));
            const float lo01 = fminf(gm[0], gm[1]), lo23 = fminf(gm[2], gm[3]);
            km = fminf(lo01, lo23);
            if constexpr (CERT == 1) {
              const float s2 = fminf(fmax_nan(lo01, lo23), fminf(fmax_nan(gm[0], gm[1]), fmax_nan(gm[2], gm[3])));
              sec_y = fmin3(sec_y, s2, fmax_nan(best_y, km));
            } else {
#pragma unroll
              for (int u = 0; u < 4; ++u) gmask |= static_cast<uint32_t>(gm[u] <= yt) << (4 * ch + u);
            }
          } else {
            const float thr = __shfl_sync(0xffffffffu, u_own, ch) + vl;
            float tt[11];
#pragma unroll
            for (int u = 0; u < 10; ++u) tt[u] = fmin3(v[3 * u], v[3 * u + 1], v[3 * u + 2]);
            tt[10] = fminf(v[30], v[31]);
            km = fmin3(fmin3(tt[0], tt[1], tt[2]), fmin3(tt[3], tt[4], tt[5]),
                       fmin3(fmin3(tt[6], tt[7], tt[8]), tt[9], tt[10]));
            cand = force || km <= thr;
          }
          const float kf = cand ? kInf : km;
          if (kf < best_y) {
            best_y = kf;
            best_c = static_cast<uint32_t>(jt) + ch * 32;
          }
          cmask |= static_cast<uint32_t>(cand) << ch;
        }

        if constexpr (CERT == 2) {
          // the tile's listed groups: (row << 32 | sorted start of the group) entries in
          // this CTA's list region, one shared-memory reservation per warp and tile; a row
          // whose entries do not fit is evaluated whole (redo 2)
          if (__any_sync(0xffffffffu, gmask != 0)) {
            const uint32_t cnt = static_cast<uint32_t>(__popc(gmask));
            uint32_t incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
              if (lane >= o) incl += v;
            }
            const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
            unsigned long long base = 0;
            if (lane == 31) base = atomicAdd(lcount, static_cast<unsigned long long>(total));
            base = __shfl_sync(0xffffffffu, base, 31) + (incl - cnt);
            bool lost = false;
            for (uint32_t gmk = gmask; gmk; gmk &= gmk - 1u, ++base) {
              const uint32_t bit = static_cast<uint32_t>(__ffs(gmk) - 1);
              if (base < a.region_cap)
                region[base] = (static_cast<unsigned long long>(i) << 32) |
                               static_cast<unsigned long long>(jt + (bit >> 2) * 32 + (bit & 3u) * 8);
              else
                lost = true;
            }
            if (lost) a.redo[i] = 2;
          }
        }
        // candidate chunks of this tile (some pair may be flagged): each goes, with its
        // accumulators y (read again from TMEM), to this CTA's list region for the exact
        // second pass; one shared-memory reservation per warp and tile
        if (__any_sync(0xffffffffu, cmask != 0)) {
          uint32_t bal[4];
          uint32_t total = 0;
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            bal[ch] = __ballot_sync(0xffffffffu, (cmask >> ch) & 1u);
            total += __popc(bal[ch]);
          }
          unsigned long long base = 0;
          if (lane == 0) base = atomicAdd(lcount, static_cast<unsigned long long>(total));
          base = __shfl_sync(0xffffffffu, base, 0);
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            if (bal[ch]) {
              const bool cand = (cmask >> ch) & 1u;
              const unsigned long long pos = base + __popc(bal[ch] & ((1u << lane) - 1u));
              base += __popc(bal[ch]);
              const bool store = cand && pos < a.region_cap;
              if (cand && !store) a.redo[i] = 1;
              if (store)
                region[pos] = (static_cast<unsigned long long>(i) << 32) | static_cast<unsigned long long>(jt + ch * 32);
              float* dst = region_s + pos * 32;  // 128-byte entries: 32-byte stores of whole sectors
#pragma unroll
              for (int half = 0; half < 2; ++half) {
                float raw[16];
                tmem_ld16(tmem_acc + ch * 32 + half * 16, raw);  // whole warp: the load is .sync.aligned
                if (store) {
#pragma unroll
                  for (int e = 0; e < 16; e += 8)
                    asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst + half * 16 + e),
                                 "f"(raw[e]), "f"(raw[e + 1]), "f"(raw[e + 2]), "f"(raw[e + 3]), "f"(raw[e + 4]),
                                 "f"(raw[e + 5]), "f"(raw[e + 6]), "f"(raw[e + 7])
                                 : "memory");
                }
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (!(a.withhold && blockIdx.x == 0 && ew == 0 && t == 0)) {
            if constexpr (PAIR) mbar_arrive_cluster(acce_c0 + 8u * b);  // rank 0's MMA waits for both CTAs
            else mbar_arrive(&acce[b]);
          }
          mbar_arrive(&metae[slot]);
        }
      }
      if (!ok) break;
      if constexpr (CERT == 2) continue;
      if constexpr (CERT == 1) {
        // this group's partial result: its best screened distance with the sorted start
        // of that center's group of 8, and its second-best screened distance
        if (row_ok) {
          float bestv = kInf, d2 = kInf;
          uint32_t gs = 0xffffffffu;
          if (best_y < kInf) {
            const uint32_t kb = __float_as_uint(best_y);
            bestv = fmaxf(__fadd_rn(__fadd_rn(2.f * __uint_as_float(kb & ~31u), -br), pp), 0.f);
            gs = best_c + (kb & 24u);
          }
          if (sec_y < kInf)
            d2 = fmaxf(__fadd_rn(__fadd_rn(2.f * __uint_as_float(__float_as_uint(sec_y) & ~31u), -br), pp), 0.f);
          a.cert_key[static_cast<int64_t>(g) * a.n + i] = make_key(bestv, gs);
          a.cert_d2[static_cast<int64_t>(g) * a.n + i] = d2;
        }
        continue;
      }
      // this group's screened minimum of the row: distance d = 2 y - Br + pp and original
      // center index
      float bestv = kInf;
      uint32_t besti = 0xffffffffu;
      if (row_ok && best_y < kInf) {
        const uint32_t kb = __float_as_uint(best_y);
        bestv = fmaxf(__fadd_rn(__fadd_rn(2.f * __uint_as_float(kb & ~31u), -br), pp), 0.f);
        besti = static_cast<uint32_t>(__ldg(a.perm + static_cast<int64_t>(best_c) + (kb & 31u)));
      }
      // the four groups' (parity, column half) partial minima of a row meet in its key:
      // a 64-bit atomic min of (distance bits, original index), the smaller index among
      // equal distances, with no barrier between the groups (the key starts at ~0)
      if (row_ok) atomicMin(&a.row_key[i], make_key(bestv, besti));
    }
    if (!ok) {
      *abort_flag = 1;
      if (lane == 0) atomicExch(&s_tf_err, DEV_TIMEOUT_EPILOGUE);
    }
  } else {
    // ------------------------------------------------------------ row preparation
    // Thread c owns rows c and c + 64 of each row tile: their pp and Br for the epilogue
    // and their extra-K rows [2^E, 2^E, 2^E, parts of Br / 2 * 2^-E] for the MMA; with
    // FUSED also the rows of A and pp itself, from the staged fp32 points (tmA maps
    // them in 32-value x 128-row boxes; thread 0 loads the CTA's next row tile into the
    // staging buffer once every row thread has read the current one, a row tile ahead
    // of its use).  A row whose norm is not finite or does not fit the extra K block
    // gets a zero row term and is marked for the exact redo.
    const int c = threadIdx.x - TF_W_ROW0 * 32;
    const int E = __ldg(a.aux_e);
    const bool screen = E < kAuxNoScreen;
    const float sc = screen ? ldexpf(1.f, -E) : 0.f;
    const uint32_t te = screen ? low_bits<KIND>(ldexpf(1.f, E)) : 0u;
    const float kNaN = __int_as_float(0x7fc00000);
    bool x_pending = false;  // FUSED: a staged load this thread issued is in flight
    if constexpr (FUSED) {
      const int64_t rt0 = tf_next_tile(a, blockIdx.x);
      if (c == 0 && rt0 < a.n_rt) {
        mbar_arrive_expect_tx(xfull, static_cast<uint32_t>(nbox * TF_XBOX_BYTES));
        for (int bx = 0; bx < nbox; ++bx)
          tma_load_2d(xst + bx * TF_XBOX_BYTES, &tmA, xfull, bx * 32, static_cast<int>(rt0 * TF_BM));
        x_pending = true;
      }
    }
    uint32_t rt_i = 0;
    bool ok = true;
    for (int64_t rt = tf_next_tile(a, blockIdx.x); rt < a.n_rt; rt = tf_next_tile(a, rt + gridDim.x), ++rt_i) {
      const uint32_t abuf = rt_i & 1u, ause = (rt_i >> 1) & 1u;
      // the MMAs of the buffer's previous row tile are done, and the epilogue has read
      // its pp and Br
      if (!(PAIR ? mbar_wait_cluster(&aempty[abuf], ause ^ 1u, abort_flag, a.wait_ns)
                 : mbar_wait(&aempty[abuf], ause ^ 1u, abort_flag, a.wait_ns)) ||
          !mbar_wait(&pempty[abuf], ause ^ 1u, abort_flag, a.wait_ns)) {
        ok = false;
        break;
      }
      float acc0 = 0.f, acc1 = 0.f;
      if constexpr (FUSED) {
        if (!mbar_wait(xfull, rt_i & 1u, abort_flag, a.wait_ns)) {
          ok = false;
          break;
        }
        if (c == 0) x_pending = false;
        uint8_t* sA = smem + abuf * a_bytes;
        for (int bx = 0; bx < nbox; ++bx) {
          acc0 = convert_box<KIND>(xst + bx * TF_XBOX_BYTES, c, sA, bx, acc0);
          acc1 = convert_box<KIND>(xst + bx * TF_XBOX_BYTES, c + 64, sA, bx, acc1);
        }
        if (nbox & 1) {  // an odd number of boxes leaves the upper half of the last K block
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int r = c + 64 * h;
            uint8_t* rowp = sA + (KB - 1) * TF_A_KB + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
            for (int q = 4; q < 8; ++q)
              *reinterpret_cast<uint4*>(rowp + ((q ^ (r & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        mbar_arrive(xempty);
        // the CTA's next row tile into the staging buffer, once every row thread is done
        const int64_t nrt = tf_next_tile(a, rt + gridDim.x);
        if (c == 0 && nrt < a.n_rt) {
          if (!mbar_wait(xempty, rt_i & 1u, abort_flag, a.wait_ns)) {
            ok = false;
            break;
          }
          fence_async_shared();
          mbar_arrive_expect_tx(xfull, static_cast<uint32_t>(nbox * TF_XBOX_BYTES));
          for (int bx = 0; bx < nbox; ++bx)
            tma_load_2d(xst + bx * TF_XBOX_BYTES, &tmA, xfull, bx * 32, static_cast<int>(nrt * TF_BM));
          x_pending = true;
        }
      }
      float* rb = rowbuf + abuf * 2 * TF_BM;
      uint8_t* ax = aaux + abuf * TF_AAUX_BYTES;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int r = c + 64 * h;
        const int64_t i = rt * TF_BM + r;
        const bool valid = i < a.n;
        float pp;
        if constexpr (FUSED) {
          const float ah = h ? acc1 : acc0;
          // the operator's norm, rounded to the operand type; the certified screen keeps
          // the fp32 norm of the rounded values
          pp = CERT != 0 ? ah : (KIND == 0 ? round_f16(ah) : round_bf16(ah));
          if (valid) a.pp[i] = pp;
        } else {
          pp = valid ? __ldg(a.pp + i) : 0.f;
        }
        const float br = __fmul_rn(pp, kAuxRowScale);
        const float w = 0.5f * br * sc;
        const bool fits = screen && br < 3.0e38f && (KIND != 0 || w < 32768.f);
        if (valid) a.redo[i] = fits ? 0 : 1;  // every row's byte: no clearing pass needed
        const bool use = valid && fits;
        rb[r] = pp;
        rb[TF_BM + r] = use ? br : kNaN;
        uint32_t e[6] = {te, te, te, 0u, 0u, 0u};
        if (use) split3<KIND>(w, e + 3);
        uint4 lo, hi;
        aux_pack<KIND>(e, lo, hi);
        // 32-byte rows with the 32-byte swizzle: 16-byte chunk q of row r at chunk
        // q ^ ((r / 4) % 2)
        const int sw = (r >> 2) & 1;
        *reinterpret_cast<uint4*>(ax + r * 32 + (sw << 4)) = lo;
        *reinterpret_cast<uint4*>(ax + r * 32 + ((sw ^ 1) << 4)) = hi;
      }
      fence_async_shared();  // the MMA reads A and the extra-K rows through the async proxy
      mbar_arrive(&afull[abuf]);
      if (PAIR && !leader) mbar_arrive_cluster(afull_c0 + 8u * abuf);  // for rank 0's MMA
    }
    if (!ok) {
      *abort_flag = 1;
      if (c == 0) atomicExch(&s_tf_err, DEV_TIMEOUT_ROWS);
    }
    // a staged load still in flight lands before the CTA exits
    if (x_pending) {
      volatile int no_abort = 0;
      mbar_wait(xfull, rt_i & 1u, &no_abort);
    }
  }

  tc_fence_before();
  __syncthreads();
  // PAIR: neither CTA leaves while the other may still read its shared memory (MMA
  // operands) or arrive on its barriers
  if constexpr (PAIR) cluster_sync();
  tc_fence_after();
  if (threadIdx.x == 0) {
    const unsigned long long c = *lcount;
    a.region_cnt[blockIdx.x] = static_cast<uint32_t>(c < a.region_cap ? c : a.region_cap);
  }
  if (warp == TF_W_MMA) {
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, kCols);
    else
      tmem_dealloc(tmem_base, kCols);
  }
}

// ------------------------------------------------------------------ host side

constexpr size_t TF_SMEM_LIMIT = 232448;
constexpr size_t TF_FIXED = 1024 + static_cast<size_t>(TF_SLOTS) * TF_META_BYTES + 2 * TF_AAUX_BYTES +
                            2 * TF_ROWBUF_BYTES + TF_BAR_BYTES;
constexpr size_t TF_STAGE_EXTRA = TF_BAUX_BYTES;  // a stage's room for the tile's extra-K rows

// FUSED staging: the row tile's fp32 points, 32 values of each row per box
static size_t tf_xstage_bytes(int dim) { return static_cast<size_t>((dim + 31) / 32) * TF_XBOX_BYTES; }

// one stage's B part (and the tile's extra-K rows): with CTA pairs each CTA holds half
static size_t tf_bstage_bytes(bool pair) { return (TF_B_KB + TF_STAGE_EXTRA) / (pair ? 2 : 1); }

// Resident A (the row tile, double-buffered) with B-only stages when that leaves room
// for 3 stages (2 when the staging buffer of FUSED takes its share), else streaming
// (A B) stages; FUSED needs resident A.
static void tf_pipeline(int kblocks, size_t xbytes, bool pair, int* nst, int* a_res) {
  const size_t abytes = static_cast<size_t>(kblocks) * TF_A_KB;
  if (TF_FIXED + xbytes > TF_SMEM_LIMIT) {  // the staging buffer alone does not fit (FUSED at large dim)
    *a_res = 0;
    *nst = 0;
    return;
  }
  const size_t avail = TF_SMEM_LIMIT - TF_FIXED - xbytes;
  const size_t bst = tf_bstage_bytes(pair);
  const size_t min_st = xbytes ? 2 : 3;
  if (2 * abytes + min_st * bst <= avail) {
    *a_res = 1;
    *nst = static_cast<int>(std::min<size_t>(8, (avail - 2 * abytes) / bst));
  } else {
    *a_res = 0;
    *nst = xbytes ? 0 : static_cast<int>(std::min<size_t>(8, avail / (TF_A_KB + bst)));
  }
}
static size_t tf_smem_bytes(int kblocks, int nst, int a_res, size_t xbytes, bool pair) {
  const size_t body = a_res ? 2 * static_cast<size_t>(kblocks) * TF_A_KB + nst * tf_bstage_bytes(pair)
                            : nst * (TF_A_KB + tf_bstage_bytes(pair));
  return TF_FIXED + xbytes + body;
}

// CTA pairs for the screen of the fast argmin: process-wide switch (euc_set_screen_pairs)
// and, per device, how many pairs of this kernel's size can be resident at once.
static std::atomic<int> g_pairs_on{1};
static int g_pair_slots[64];
static int tf_pair_slots() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (g_pair_slots[dev] == 0) {
    auto kern = dist_tc_fast_kernel<0, true, 0, true>;
    int clusters = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(TF_SMEM_LIMIT)) ==
        cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * 1024);
      cfg.blockDim = dim3(TF_THREADS);
      cfg.dynamicSmemBytes = TF_SMEM_LIMIT;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 2;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) clusters = 0;
    }
    cudaGetLastError();  // a failed query leaves no error behind
    g_pair_slots[dev] = clusters > 0 ? clusters : -1;
  }
  return g_pair_slots[dev] > 0 ? g_pair_slots[dev] : 0;
}

// Pairs halve each SM's share of the center tiles streamed from L2, but make one MMA
// issuer wait for both CTAs' epilogues.  Measured on one B200: at 16 K blocks per tile
// (d = 1024, fp16) the screen runs 6 % faster paired; at 1 or 2 K blocks (d = 64, 128),
// where the epilogue sets the pace, 18-26 % slower.  So only tiles of 8 or more K blocks
// (d >= 512 for 16-bit operands) pair.
constexpr int TF_PAIR_MIN_KBLOCKS = 8;

bool tc_fast_pairs(bool cert, int kblocks) {
  return !cert && kblocks >= TF_PAIR_MIN_KBLOCKS && g_pairs_on.load() != 0 && tf_pair_slots() > 0;
}

int tc_fast_regions(int64_t n, bool cert, int kblocks) {
  if (tc_fast_pairs(cert, kblocks)) {
    const int64_t n_pt = (n + 2 * TF_BM - 1) / (2 * TF_BM);
    const int64_t clusters = std::min<int64_t>(tf_pair_slots(), std::max<int64_t>(n_pt, 1));
    return static_cast<int>(2 * clusters);
  }
  const int64_t n_rt = (n + TF_BM - 1) / TF_BM;
  int grid = num_sms();
  if (static_cast<int64_t>(grid) > n_rt) grid = static_cast<int>(n_rt);
  return grid < 1 ? 1 : grid;
}

template <int KIND, bool FUSED, int CERT, bool PAIR>
static cudaError_t launch_tf_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tba,
                               const TfArgs& args, int grid, cudaStream_t st) {
  auto kern = dist_tc_fast_kernel<KIND, FUSED, CERT, PAIR>;
  const size_t smem =
      tf_smem_bytes(args.kblocks, args.nst, args.a_res, FUSED ? tf_xstage_bytes(args.dim) : 0, PAIR);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  // the kernel timing hook times the screen over all rows (not the certified second screen)
  if (CERT != 2) timing_begin(st, "dist_tc_fast_kernel");
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(TF_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tba, args);
  } else {
    kern<<<grid, TF_THREADS, smem, st>>>(ta, tb, tba, args);
    e = cudaGetLastError();
  }
  if (CERT != 2) timing_end(st);
  return e;
}

static int low_kind(const OpSpec* s) { return (s->gemm == G_TC_F16) ? 0 : (s->gemm == G_TC_BF16 ? 1 : 2); }

static int tf_kblocks(const DistJob& j) {
  const int esize = (low_kind(j.spec) == 2) ? 4 : 2;
  return static_cast<int>((static_cast<int64_t>(j.ldlow) * esize) / 128);
}

int tc_fast_job_regions(const DistJob& j) { return tc_fast_regions(j.n, j.cert, tf_kblocks(j)); }

// The row warps read the fp32 points themselves when the operator's norm is that of
// the fp16 / bf16 rounded values, the rows are whole 16-byte vectors, and A stays
// resident in shared memory.
bool tc_fast_can_fuse_rows(const DistJob& j) {
  const OpSpec* s = j.spec;
  const bool recipe = (s->gemm == G_TC_F16 && s->norm == NM_LOW_F16) || (s->gemm == G_TC_BF16 && s->norm == NM_LOW_BF16);
  if (!recipe || s->in != IN_F32) return false;
  if (j.dim % 4 != 0 || (reinterpret_cast<uintptr_t>(j.P) & 15u) != 0) return false;
  int nst = 0, a_res = 0;
  tf_pipeline(tf_kblocks(j), tf_xstage_bytes(j.dim), false, &nst, &a_res);  // unpaired stages are the larger
  return a_res != 0 && nst >= 2;
}

cudaError_t launch_tc_fast(const DistJob& j, int cert_pass) {
  const OpSpec* s = j.spec;
  const int kind = low_kind(s);
  const int esize = (kind == 2) ? 4 : 2;
  if (j.n > 0x7fffffffll - TF_BM) return cudaErrorInvalidValue;  // TMA row coordinates are 32-bit
  TfArgs a{};
  a.n = j.n;
  a.m = j.m;
  a.kblocks = tf_kblocks(j);
  a.n_ct = static_cast<int>((j.m + TF_BN - 1) / TF_BN);
  // the fast argmin's screen runs on CTA pairs (row tiles counted in whole pairs)
  const bool pair = cert_pass == 0 && tc_fast_pairs(j.cert, a.kblocks);
  a.n_rt = pair ? 2 * ((j.n + 2 * TF_BM - 1) / (2 * TF_BM)) : (j.n + TF_BM - 1) / TF_BM;
  tf_pipeline(a.kblocks, j.fused_rows ? tf_xstage_bytes(j.dim) : 0, pair, &a.nst, &a.a_res);
  if (a.nst < 2) return cudaErrorInvalidValue;
  if (j.fused_rows && !tc_fast_can_fuse_rows(j)) return cudaErrorInvalidValue;
  a.pp = static_cast<float*>(j.pp);
  a.X = static_cast<const float*>(j.P);
  a.dim = j.dim;
  a.ccs = j.cc_sorted;
  a.perm = j.perm;
  a.omk = 1.f - j.kf;
  // screen margin: the rounding of S to the GEMM's output format dominates
  a.margin = s->sround == SR_F16 ? 0x1p-10f : (s->sround == SR_BF16 ? 0x1p-7f : 0x1p-16f);
  // (65504 / 1.05)^2: no fp16 overflow of s (the certified pass never rounds s)
  a.ovf = (s->sround == SR_F16 && !j.cert) ? 3.9e9f : 1.0e36f;
  // certified: below 4e9 no element of an fp32 row exceeds fp16's range
  a.nlim = (j.cert && kind == 0) ? 4.0e9f : 3.0e38f;
  a.aux_e = j.aux_e;
  a.row_key = j.row_key;
  a.list = j.chunk_list;
  a.sbuf = j.chunk_s;
  a.region_cap = j.chunk_cap / static_cast<unsigned long long>(j.regions);
  a.region_cnt = j.region_cnt;
  a.redo = j.redo;
  a.cert_key = j.cert_key;
  a.cert_d2 = j.cert_d2;
  a.wait_ns = wait_limit_ns();
  a.withhold = (cert_pass == 0 && take_withhold()) ? 1 : 0;
  const int grid = j.regions;
  if (grid != tc_fast_regions(j.n, j.cert, a.kblocks) || (pair && (grid & 1))) return cudaErrorInvalidValue;
  const int bn_load = pair ? TF_BN / 2 : TF_BN;  // center rows one CTA loads per tile
  // A: the low-precision copy, or with FUSED the fp32 points in 32-value x 128-row boxes
  CUtensorMap ta, tb;
  if (j.fused_rows) {
    if (!tc_make_tmap(&ta, j.P, j.n, j.dim, 4, TF_BM, true, false)) return cudaErrorInvalidValue;
  } else if (!tc_make_tmap(&ta, j.Plow, j.n, j.ldlow, esize, TF_BM, kind == 2, kind == 1)) {
    return cudaErrorInvalidValue;
  }
  if (!tc_make_tmap(&tb, j.Clow_sorted, j.m, j.ldlow, esize, bn_load, kind == 2, kind == 1))
    return cudaErrorInvalidValue;
  CUtensorMap tba;
  const int64_t mpad = (j.m + TF_BN - 1) / TF_BN * TF_BN;
  if (!tc_make_tmap_sw32(&tba, j.b_aux_sorted, mpad, esize, bn_load, kind == 2, kind == 1))
    return cudaErrorInvalidValue;
#define TF_LAUNCH(CM_, PR_)                                                     \
  if (j.fused_rows) {                                                           \
    if (kind == 0) return launch_tf_t<0, true, CM_, PR_>(ta, tb, tba, a, grid, j.stream); \
    return launch_tf_t<1, true, CM_, PR_>(ta, tb, tba, a, grid, j.stream);      \
  }                                                                             \
  if (kind == 0) return launch_tf_t<0, false, CM_, PR_>(ta, tb, tba, a, grid, j.stream);  \
  if (kind == 1) return launch_tf_t<1, false, CM_, PR_>(ta, tb, tba, a, grid, j.stream);  \
  return launch_tf_t<2, false, CM_, PR_>(ta, tb, tba, a, grid, j.stream);
  if (cert_pass == 1) {
    if (!j.cert_key || !j.cert_d2) return cudaErrorInvalidValue;
    TF_LAUNCH(1, false)
  }
  if (cert_pass == 0 && j.row_key) {
    // the screen folds each group's row minimum into the key with an atomic min
    const cudaError_t e = cudaMemsetAsync(j.row_key, 0xff, static_cast<size_t>(j.n) * sizeof(unsigned long long), j.stream);
    if (e != cudaSuccess) return e;
  }
  if (cert_pass == 2) {
    if (!j.cert_thr || !j.cert_tiles) return cudaErrorInvalidValue;
    a.cert_thr = j.cert_thr;
    a.tile_on = j.cert_tiles;
    TF_LAUNCH(2, false)
  }
  if (pair) {
    TF_LAUNCH(0, true)
  }
  TF_LAUNCH(0, false)
#undef TF_LAUNCH
}

int tf_error_and_clear() {
  int v = 0, z = 0;
  cudaMemcpyFromSymbol(&v, s_tf_err, sizeof(int));
  if (v) cudaMemcpyToSymbol(s_tf_err, &z, sizeof(int));
  return v;
}

// s of one pair over the rounded operands the MMA consumes, summed in dimension order
// with fused multiply-adds: the fp32 point row rounded here (the rounding of its
// low-precision copy), the center row from its low-precision copy.  The copies' zero
// padding would add nothing, so the sum stops at dim.
template <int KIND>
__device__ __forceinline__ float low_dot(const float* __restrict__ p, const uint4* __restrict__ c, int dim) {
  constexpr int PER = (KIND == 2) ? 4 : 8;  // elements per 16-byte vector of the copy
  float acc = 0.f;
  for (int v = 0; v * PER < dim; ++v) {
    const uint4 yv = __ldg(c + v);
    const uint32_t ys[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const int k = v * PER + e;
      if (k < dim) {
        const float x = low_value<KIND>(low_bits<KIND>(__ldg(p + k)));
        float y;
        if constexpr (KIND == 2)
          y = __uint_as_float(ys[e]);
        else
          y = low_value<KIND>((ys[e >> 1] >> ((e & 1) * 16)) & 0xffffu);
        acc = __fmaf_rn(x, y, acc);
      }
    }
  }
  return acc;
}

__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long k) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, k, o);
    k = t < k ? t : k;
  }
  return k;
}

// ================================================================ second pass
//
// Candidate chunks, evaluated with the operator's exact arithmetic on the stored MMA
// accumulators: s rounded to the GEMM's output format, d = max((pp - 2 s) + cc, 0),
// flagged when d <= K (pp + cc) (euclidean_kernels_mix.cu:203-211), exactly as the
// exact epilogue forms them.  One warp per chunk, one lane per column.  Unflagged
// pairs fold into the row's 64-bit key with one atomicMin per chunk; flagged pairs are
// counted and appended (warp-buffered) to the direct-recompute list, which
// recompute_kernel then folds in.  If that list is full the pair is recomputed here.

struct EvArgs {
  const unsigned long long* clist;
  const float* sbuf;            // the chunk's accumulators y = y0 - s, y0 = (cc + Br) / 2 (0 for a non-finite cc)
  unsigned long long region_cap;
  const uint32_t* region_cnt;
  const float* pp;
  const float* cc_s;
  const int* perm;
  int64_t n, m;
  float K;
  const uint8_t* redo;
  unsigned long long* row_key;
  unsigned long long* count;
  unsigned long long* list;
  unsigned long long cap;
  const float* P;
  const float* C;
  int dim;
};

constexpr int EV_BLOCKS_PER_REGION = 8;
constexpr int EV_WBUF = 256;  // flagged pairs buffered per warp before one list reservation

template <int REC>
__device__ __noinline__ void fold_direct(const float* P, const float* C, int dim, unsigned long long* row_key,
                                         int64_t i, uint32_t jo) {
  const float d = static_cast<float>(direct_dist_scalar<float, REC>(P + i * dim, C + static_cast<int64_t>(jo) * dim, dim));
  atomicMin(&row_key[i], make_key(d, jo));
}

template <int REC>
__device__ __forceinline__ void flush_pairs(const EvArgs& a, unsigned long long* wbuf, int& wcnt, int lane) {
  unsigned long long base = 0;
  if (lane == 0) base = atomicAdd(a.count, static_cast<unsigned long long>(wcnt));
  base = __shfl_sync(0xffffffffu, base, 0);
  for (int q = lane; q < wcnt; q += 32) {
    const unsigned long long e = wbuf[q];
    if (base + q < a.cap)
      a.list[base + q] = e;
    else
      fold_direct<REC>(a.P, a.C, a.dim, a.row_key, static_cast<int64_t>(e >> 32),
                       static_cast<uint32_t>(e & 0xffffffffull));
  }
  __syncwarp();
  wcnt = 0;
}

template <int SROUND, int REC>
__global__ void __launch_bounds__(256) eval_chunks_kernel(const EvArgs a) {
  __shared__ unsigned long long s_buf[8][EV_WBUF];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  // a warp evaluates four entries at a time: the eight lanes sg * 8 .. sg * 8 + 7 take
  // entry sg, lane sl of them the four columns 4 sl .. 4 sl + 3 (16-byte loads of the
  // accumulators, norms and original indices)
  const int sg = lane >> 3, sl = lane & 7;
  unsigned long long* wbuf = s_buf[wib];
  int wcnt = 0;
  const int r = blockIdx.x / EV_BLOCKS_PER_REGION;
  const unsigned wr = (blockIdx.x % EV_BLOCKS_PER_REGION) * 8 + wib;
  constexpr unsigned kStride = EV_BLOCKS_PER_REGION * 8;
  unsigned long long cnt64 = a.region_cnt[r];
  if (cnt64 > a.region_cap) cnt64 = a.region_cap;
  // a region holds at most max(2n, 2^16) / regions entries: 32 times that fits 32 bits
  const uint32_t cnt = static_cast<uint32_t>(cnt64);
  const unsigned long long rbase = static_cast<unsigned long long>(r) * a.region_cap;
  const unsigned long long* cl = a.clist + rbase;
  const float4* sb = reinterpret_cast<const float4*>(a.sbuf + rbase * 32) + sl;
  const uint32_t n32 = static_cast<uint32_t>(a.n), m32 = static_cast<uint32_t>(a.m);
  // two sets of four entries per iteration: their loads are independent and issue together
  constexpr int U = 2;
  for (uint32_t t0 = wr * 4u * U; t0 < cnt; t0 += kStride * 4u * U) {
    unsigned long long e[U];
    float4 s4[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t t = t0 + u * 4u + sg;
      const bool in = t < cnt;
      e[u] = in ? cl[t] : ~0ull;
      s4[u] = in ? sb[t * 8u] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    uint32_t i[U], j0[U];
    bool skip[U];
    float pp[U];
    float4 c4[U];
    int4 p4[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      i[u] = static_cast<uint32_t>(e[u] >> 32);
      const bool iv = i[u] < n32;
      skip[u] = !iv || a.redo[iv ? i[u] : 0u] != 0;  // redo rows are evaluated whole
      // the chunk's first sorted column is a multiple of 32 and the norms and indices are
      // padded to whole 256-center tiles, so the 16-byte loads stay in bounds
      j0[u] = static_cast<uint32_t>(e[u]) + 4u * static_cast<uint32_t>(sl);
      pp[u] = 0.f;
      c4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      p4[u] = make_int4(0, 0, 0, 0);
      if (!skip[u]) {
        pp[u] = __ldg(a.pp + i[u]);
        c4[u] = __ldg(reinterpret_cast<const float4*>(a.cc_s + j0[u]));
        p4[u] = __ldg(reinterpret_cast<const int4*>(a.perm + j0[u]));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float sv[4] = {s4[u].x, s4[u].y, s4[u].z, s4[u].w};
      const float cc[4] = {c4[u].x, c4[u].y, c4[u].z, c4[u].w};
      const uint32_t jo[4] = {static_cast<uint32_t>(p4[u].x), static_cast<uint32_t>(p4[u].y),
                              static_cast<uint32_t>(p4[u].z), static_cast<uint32_t>(p4[u].w)};
      const float br = __fmul_rn(pp[u], kAuxRowScale);
      // row key of the chunk: smallest unflagged distance (d >= 0, so its bits order as
      // unsigned), then the smallest original index among the columns that reach it
      unsigned long long best = ~0ull;
      uint32_t flm = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const bool jv = !skip[u] && j0[u] + c < m32;
        const float y0 = cc[c] < 3.0e38f ? __fadd_rn(0.5f * cc[c], 0.5f * br) : 0.f;
        const float d = exact_d<SROUND>(y0 - sv[c], pp[u], cc[c]);
        const bool fl = jv && d <= __fmul_rn(a.K, __fadd_rn(pp[u], cc[c]));
        flm |= static_cast<uint32_t>(fl) << c;
        const unsigned long long k = (jv && !fl) ? ((static_cast<unsigned long long>(__float_as_uint(d)) << 32) | jo[c]) : ~0ull;
        best = k < best ? k : best;
      }
      if (__any_sync(0xffffffffu, flm != 0)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const bool fl = (flm >> c) & 1u;
          const unsigned bal = __ballot_sync(0xffffffffu, fl);
          if (fl) wbuf[wcnt + __popc(bal & ((1u << lane) - 1u))] = (static_cast<unsigned long long>(i[u]) << 32) | jo[c];
          wcnt += __popc(bal);
        }
        __syncwarp();
        if (wcnt > EV_WBUF - 128) flush_pairs<REC>(a, wbuf, wcnt, lane);
      }
#pragma unroll
      for (int o = 4; o >= 1; o >>= 1) {
        const unsigned long long x = __shfl_xor_sync(0xffffffffu, best, o);
        best = x < best ? x : best;
      }
      if (sl == 0 && best != ~0ull) atomicMin(&a.row_key[i[u]], best);
    }
  }
  // the warps' remaining pairs: one list reservation for the whole block (a reservation
  // per warp would queue thousands of atomics on the one counter)
  __shared__ unsigned int s_tot;
  __shared__ unsigned long long s_base;
  if (threadIdx.x == 0) s_tot = 0u;
  __syncthreads();
  unsigned int off = 0u;
  if (lane == 0 && wcnt > 0) off = atomicAdd(&s_tot, static_cast<unsigned int>(wcnt));
  off = __shfl_sync(0xffffffffu, off, 0);
  __syncthreads();
  if (threadIdx.x == 0) s_base = s_tot ? atomicAdd(a.count, static_cast<unsigned long long>(s_tot)) : 0ull;
  __syncthreads();
  const unsigned long long base = s_base + off;
  for (int q = lane; q < wcnt; q += 32) {
    const unsigned long long e = wbuf[q];
    if (base + q < a.cap)
      a.list[base + q] = e;
    else
      fold_direct<REC>(a.P, a.C, a.dim, a.row_key, static_cast<int64_t>(e >> 32),
                       static_cast<uint32_t>(e & 0xffffffffull));
  }
}

// Rows whose candidates overflowed their region, or whose norm did not fit the extra K
// block: every pair evaluated exactly, with s summed in fp32 (sequential fused
// multiply-adds) over the rounded operands the MMA consumes; flagged pairs take the
// direct distance here.  The same pass then turns every row's key into its outputs
// (label, int32 label, distance), as keys_to_labels_kernel does for the other paths.

struct RdArgs {
  const void* Clow;   // original order
  int nvec;           // 16-byte vectors per low row
  const float* P;
  const float* C;
  int dim;
  const float* pp;
  const float* cc;
  int64_t n, m;
  float K;
  const uint8_t* redo;
  unsigned long long* row_key;
  unsigned long long* count;
  int64_t* labels;    // nullable outputs
  int32_t* labels32;
  float* mind;
};

template <int KIND, int SROUND, int REC>
__global__ void __launch_bounds__(256) redo_rows_kernel(const RdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  unsigned long long nfl = 0;
  // G groups of 32 rows per step: their redo bytes, then their keys, load together
  constexpr int G = 4;
  for (int64_t base0 = gw * 32 * G; base0 < a.n; base0 += nw * 32 * G) {
    unsigned balg[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int64_t ii = base0 + g * 32 + lane;
      balg[g] = __ballot_sync(0xffffffffu, ii < a.n && a.redo[ii] != 0);
    }
#pragma unroll 1
    for (int g = 0; g < G; ++g) {
      const int64_t base = base0 + g * 32;
      unsigned bal = balg[g];
      while (bal) {
        const int64_t i = base + (__ffs(bal) - 1);
        bal &= bal - 1;
        unsigned long long best = ~0ull;
        const float pp = __ldg(a.pp + i);
        for (int64_t j0 = 0; j0 < a.m; j0 += 32) {
          const int64_t j = j0 + lane;
          bool fl = false;
          if (j < a.m) {
            const float sv = low_dot<KIND>(a.P + i * a.dim, static_cast<const uint4*>(a.Clow) + j * a.nvec, a.dim);
            const float cc = __ldg(a.cc + j);
            float d = exact_d<SROUND>(sv, pp, cc);
            fl = d <= __fmul_rn(a.K, __fadd_rn(pp, cc));
            if (fl) d = static_cast<float>(direct_dist_scalar<float, REC>(a.P + i * a.dim, a.C + j * a.dim, a.dim));
            const unsigned long long k = make_key(d, static_cast<uint32_t>(j));
            best = k < best ? k : best;
          }
          nfl += __popc(__ballot_sync(0xffffffffu, fl));
        }
        best = warp_min_u64(best);
        if (lane == 0) a.row_key[i] = best;
      }
    }
    __syncwarp();
    unsigned long long kg[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int64_t ii = base0 + g * 32 + lane;
      kg[g] = ii < a.n ? a.row_key[ii] : 0ull;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int64_t ii = base0 + g * 32 + lane;
      if (ii < a.n) {
        const uint32_t j = static_cast<uint32_t>(kg[g] & 0xffffffffull);
        if (a.labels) a.labels[ii] = j;
        if (a.labels32) a.labels32[ii] = static_cast<int32_t>(j);
        if (a.mind) a.mind[ii] = __uint_as_float(static_cast<uint32_t>(kg[g] >> 32));
      }
    }
  }
  if (lane == 0 && nfl) atomicAdd(a.count, nfl);
}

#define FAST_REC_CASES(X)     \
  X(0, SR_F16, RC_F64)        \
  X(0, SR_F16, RC_F32)        \
  X(0, SR_F16, RC_F16_ARITH)  \
  X(0, SR_NONE, RC_F64)       \
  X(0, SR_NONE, RC_F32)       \
  X(1, SR_BF16, RC_F64)       \
  X(1, SR_BF16, RC_F32)       \
  X(1, SR_BF16, RC_BF16_ARITH)\
  X(1, SR_NONE, RC_F64)       \
  X(1, SR_NONE, RC_F32)       \
  X(2, SR_NONE, RC_F64)

cudaError_t launch_eval_chunks(const DistJob& j) {
  const OpSpec* s = j.spec;
  const int kind = low_kind(s);
  EvArgs a{};
  a.clist = j.chunk_list;
  a.sbuf = j.chunk_s;
  a.region_cap = j.chunk_cap / static_cast<unsigned long long>(j.regions);
  a.region_cnt = j.region_cnt;
  a.pp = static_cast<const float*>(j.pp);
  a.cc_s = j.cc_sorted;
  a.perm = j.perm;
  a.n = j.n;
  a.m = j.m;
  a.K = j.kf;
  a.redo = j.redo;
  a.row_key = j.row_key;
  a.count = j.count;
  a.list = j.list;
  a.cap = j.list_cap;
  a.P = static_cast<const float*>(j.P);
  a.C = static_cast<const float*>(j.C);
  a.dim = j.dim;
  const unsigned grid = static_cast<unsigned>(j.regions * EV_BLOCKS_PER_REGION);
#define EV_CASE(KIND_, SR_, REC_)                                         \
  if (kind == KIND_ && s->sround == SR_ && s->rec == REC_) {              \
    eval_chunks_kernel<SR_, REC_><<<grid, 256, 0, j.stream>>>(a);         \
    return cudaGetLastError();                                            \
  }
  FAST_REC_CASES(EV_CASE)
#undef EV_CASE
  return cudaErrorNotSupported;
}

cudaError_t launch_redo_rows(const DistJob& j, int64_t* labels, int32_t* labels32, float* mind) {
  const OpSpec* s = j.spec;
  const int kind = low_kind(s);
  const int esize = (kind == 2) ? 4 : 2;
  RdArgs a{};
  a.Clow = j.Clow;
  a.nvec = static_cast<int>(static_cast<int64_t>(j.ldlow) * esize / 16);
  a.P = static_cast<const float*>(j.P);
  a.C = static_cast<const float*>(j.C);
  a.dim = j.dim;
  a.pp = static_cast<const float*>(j.pp);
  a.cc = static_cast<const float*>(j.cc);
  a.n = j.n;
  a.m = j.m;
  a.K = j.kf;
  a.redo = j.redo;
  a.row_key = j.row_key;
  a.count = j.count;
  a.labels = labels;
  a.labels32 = labels32;
  a.mind = mind;
  const int64_t warps = (j.n + 127) / 128;  // four groups of 32 rows per warp step
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((warps + 7) / 8, static_cast<int64_t>(num_sms()) * 8));
#define RD_CASE(KIND_, SR_, REC_)                                             \
  if (kind == KIND_ && s->sround == SR_ && s->rec == REC_) {                  \
    redo_rows_kernel<KIND_, SR_, REC_><<<blocks, 256, 0, j.stream>>>(a);      \
    return cudaGetLastError();                                                \
  }
  FAST_REC_CASES(RD_CASE)
#undef RD_CASE
  return cudaErrorNotSupported;
}

}  // namespace euc

extern "C" void euc_set_screen_pairs(int enable) { euc::g_pairs_on.store(enable != 0 ? 1 : 0); }
