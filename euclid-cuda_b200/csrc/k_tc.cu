// Fused distance kernel on the 5th-generation tensor cores (sm_100a).
//
// One persistent CTA per SM walks 128-row tiles of the points.  For each row tile
// it sweeps every center tile (bn = 64/128/256 centers):
//   warp 0  : TMA producer; the row tile's A K-blocks (128 x 64 fp16/bf16 | 128 x 32
//             tf32) stay resident (double-buffered) when they fit, else A streams with
//             B; B (bn x same) K-blocks stream through a ring of up to 8 stages of
//             128B-swizzled smem;
//   warp 1  : tcgen05.mma issuer (one elected lane), M=128 x N=bn x K=16|8 per
//             instruction, fp32 accumulators double-buffered in TMEM (2*bn columns);
//             also owns the TMEM allocation;
//   warps 2-9: epilogue, 2 per TMEM lane quadrant (each half of the tile's columns);
//             each thread owns one TMEM lane = one point row.  It reads 32 or 64
//             accumulator columns at a time (tcgen05.ld 32x32b), applies the
//             reference's S rounding, forms d = max((pp - 2s) + cc, 0), runs the
//             cancellation test d <= K (pp + cc) and either stores D or keeps the
//             running (min, first index) of the row (exact argmin).  Flagged pairs are
//             appended to a compact list with one atomic per warp (ballot + popc).
//
// This replaces the reference's chain  cast -> norms -> cuBLAS GEMM (S in HBM) ->
// form_mixed_and_list_* (euclidean_kernels_mix.cu:184-316, 322-407) and the WMMA
// kernel euclidean_tensorcore_generic_kernel (euclidean_kernels_tiled_tc.cu:79-212):
// S never leaves the chip.
//
// Every mbarrier wait is bounded (common.cuh); on expiry the CTA records an error,
// drains its own in-flight TMA copies and MMAs, frees TMEM and returns.
#include "common.cuh"
#include "engine.h"
#include "direct.cuh"

#include <cudaTypedefs.h>
#include <algorithm>

namespace euc {

static __device__ int s_tc_err;

constexpr int TC_BM = 128;
constexpr int TC_EPI_WARPS = 8;  // two warps per TMEM lane quadrant, each owning half of the columns
constexpr int TC_THREADS = (2 + TC_EPI_WARPS) * 32;
constexpr int TC_A_BYTES = TC_BM * 128;  // one K-block of A: 128 rows x 128 bytes
constexpr int TC_BAR_BYTES = 256;        // mbarriers, TMEM slot, abort flag
constexpr int TC_EPI_BYTES = TC_EPI_WARPS * 128 * 4;  // per-warp center norms

enum TcMode { TM_ARGMIN = 0, TM_D_F32 = 1, TM_D_F16 = 2, TM_D_BF16 = 3 };

struct TcArgs {
  int64_t n, m;
  int dim;
  int kblocks;  // K-blocks of 128 bytes
  int bn;
  int nst;      // pipeline stages
  int a_res;    // 1: the row tile's A stays resident (double-buffered); stages carry B only
  int n_ct;     // center tiles
  int64_t n_rt; // row tiles
  const float* pp;
  const float* cc;    // center norms
  float K;
  void* D;
  unsigned long long* row_key;
  unsigned long long* list;
  unsigned long long list_cap;
  unsigned long long* count;
  int32_t* tile_counts;
  int tile_T;
  int64_t tiles_j;
  const float* P;  // fp32 originals (inline recompute when the list is full)
  const float* C;
  unsigned long long wait_ns;  // bound of every wait of the pipeline
};

// a pair's direct distance when the recompute list is full (out of line: the epilogue's
// registers stay its own; 16-byte loads when the rows allow them)
template <int REC>
__device__ __noinline__ float overflow_direct(const float* p, const float* c, int dim) {
  return static_cast<float>(direct_dist<float, REC>(p, c, dim));
}

template <int KIND, int SROUND, int FLAG, int MODE, int REC>
__global__ void __launch_bounds__(TC_THREADS, 1)
    dist_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment of every stage (required by the 128B swizzle atoms)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bn = a.bn;
  const int NST = a.nst;
  const bool a_res = a.a_res != 0;
  const uint32_t b_bytes = static_cast<uint32_t>(bn) * 128u;
  // resident mode: [A buf 0 | A buf 1 | B stage 0..NST-1]; streaming mode: [A+B stage 0..NST-1]
  const uint32_t a_bytes = static_cast<uint32_t>(a.kblocks) * TC_A_BYTES;
  const uint32_t stage_bytes = a_res ? b_bytes : (TC_A_BYTES + b_bytes);
  uint8_t* stage_base = smem + (a_res ? 2 * a_bytes : 0);
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_base + NST * stage_bytes);
  uint64_t* empty = full + NST;
  uint64_t* afull = empty + NST;
  uint64_t* aempty = afull + 2;
  uint64_t* accf = aempty + 2;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* epi = reinterpret_cast<float*>(stage_base + NST * stage_bytes + TC_BAR_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ncols = 2u * static_cast<uint32_t>(bn);  // power of two >= 128

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
      mbar_init(&accf[s], 1);
      mbar_init(&acce[s], TC_EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, ncols);
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, rt_i = 0;
      uint32_t issued_mask = 0, last_phase = 0, a_issued = 0, a_last = 0;
      bool ok = true;
      const int kelems = (KIND == 2) ? 32 : 64;  // elements per 128-byte K-block
      for (int64_t rt = blockIdx.x; rt < a.n_rt && ok; rt += gridDim.x, ++rt_i) {
        const uint32_t abuf = rt_i & 1u, ause = (rt_i >> 1) & 1u;
        if (a_res) {
          // the whole 128-row A tile once per row tile, into its own buffer
          if (!mbar_wait(&aempty[abuf], ause ^ 1u, abort_flag, a.wait_ns)) { ok = false; break; }
          mbar_arrive_expect_tx(&afull[abuf], a_bytes);
          uint8_t* sA = smem + abuf * a_bytes;
          for (int kb = 0; kb < a.kblocks; ++kb)
            tma_load_2d(sA + kb * TC_A_BYTES, &tmA, &afull[abuf], kb * kelems, static_cast<int>(rt * TC_BM));
          a_issued |= 1u << abuf;
          a_last = (a_last & ~(1u << abuf)) | (ause << abuf);
        }
        for (int ct = 0; ct < a.n_ct && ok; ++ct) {
          for (int kb = 0; kb < a.kblocks; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, a.wait_ns)) { ok = false; break; }
            uint8_t* st = stage_base + stage * stage_bytes;
            mbar_arrive_expect_tx(&full[stage], stage_bytes);
            if (a_res) {
              tma_load_2d(st, &tmB, &full[stage], kb * kelems, ct * bn);
            } else {
              tma_load_2d(st, &tmA, &full[stage], kb * kelems, static_cast<int>(rt * TC_BM));
              tma_load_2d(st + TC_A_BYTES, &tmB, &full[stage], kb * kelems, ct * bn);
            }
            issued_mask |= 1u << stage;
            last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
            if (++stage == static_cast<uint32_t>(NST)) { stage = 0; phase ^= 1u; }
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(&s_tc_err, DEV_TIMEOUT_PRODUCER);
      }
      // Drain: every issued copy must have landed before shared memory is released.
      volatile int no_abort = 0;
      for (int s = 0; s < NST; ++s)
        if (issued_mask & (1u << s)) mbar_wait(&full[s], (last_phase >> s) & 1u, &no_abort);
      for (int s = 0; s < 2; ++s)
        if (a_issued & (1u << s)) mbar_wait(&afull[s], (a_last >> s) & 1u, &no_abort);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = (KIND == 0) ? 0u : (KIND == 1 ? 1u : 2u);
      const uint32_t idesc = umma_idesc(fmt, TC_BM, static_cast<uint32_t>(bn));
      uint32_t stage = 0, phase = 0, acc_i = 0, rt_i = 0;
      bool ok = true;
      for (int64_t rt = blockIdx.x; rt < a.n_rt && ok; rt += gridDim.x, ++rt_i) {
        const uint32_t abuf = rt_i & 1u, ause = (rt_i >> 1) & 1u;
        const uint32_t sAres = smem_u32(smem + abuf * a_bytes);
        if (a_res) {
          if (!mbar_wait(&afull[abuf], ause, abort_flag, a.wait_ns)) { ok = false; break; }
        }
        for (int ct = 0; ct < a.n_ct && ok; ++ct) {
          const uint32_t buf = acc_i & 1u, use = (acc_i >> 1) & 1u;
          if (!mbar_wait(&acce[buf], use ^ 1u, abort_flag, a.wait_ns)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * static_cast<uint32_t>(bn);
          for (int kb = 0; kb < a.kblocks; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag, a.wait_ns)) { ok = false; break; }
            tc_fence_after();
            const uint32_t st = smem_u32(stage_base + stage * stage_bytes);
            const uint32_t sA = a_res ? sAres + kb * TC_A_BYTES : st;
            const uint32_t sB = a_res ? st : st + TC_A_BYTES;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {  // 4 x 32 bytes = one 128-byte swizzle row
              const uint64_t ad = sw128_kmajor_desc(sA + kk * 32);
              const uint64_t bd = sw128_kmajor_desc(sB + kk * 32);
              if constexpr (KIND == 2)
                umma_tf32(d_tmem, ad, bd, idesc, (kb | kk) != 0);
              else
                umma_f16(d_tmem, ad, bd, idesc, (kb | kk) != 0);
            }
            umma_commit(&empty[stage]);
            if (++stage == static_cast<uint32_t>(NST)) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          umma_commit(&accf[buf]);
          ++acc_i;
        }
        if (a_res && ok) umma_commit(&aempty[abuf]);  // A buffer free once this row tile's MMAs retire
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(&s_tc_err, DEV_TIMEOUT_MMA);
      }
      // Drain: wait until every MMA this thread issued has completed.
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    constexpr bool ARGMIN = (MODE == TM_ARGMIN);
    const int ew = warp - 2;             // 0..7
    const int q = warp & 3;              // TMEM lane quadrant this warp may access
    const int half = ew >> 2;            // which half of the tile's columns
    const int cols = bn >> 1;            // columns per warp: 32, 64 or 128
    const int nch = cols >> 5;           // 32-column chunks per warp and tile
    const int row_local = q * 32 + lane;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    float* cc_w = epi + ew * 128;        // this warp's columns: norms
    const float K = a.K;

    // Center metadata of the next tile this warp will process is loaded one tile ahead
    // (4 columns per lane at most), so the global-load latency overlaps the current tile.
    float pf_cc[4];
    auto prefetch = [&](int64_t rt_next, int ct_next) {
#pragma unroll
      for (int t = 0; t < 4; ++t) pf_cc[t] = 0.f;
      if (rt_next >= a.n_rt) return;
      const int64_t jw = static_cast<int64_t>(ct_next) * bn + half * cols;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int c = lane + 32 * t;
        if (c < cols && jw + c < a.m) pf_cc[t] = __ldg(a.cc + jw + c);
      }
    };

    uint32_t acc_i = 0, rt_i = 0;
    bool ok = true;
    prefetch(blockIdx.x, 0);
    for (int64_t rt = blockIdx.x; rt < a.n_rt && ok; rt += gridDim.x, ++rt_i) {
      const int64_t i = rt * TC_BM + row_local;
      const bool row_ok = i < a.n;
      const float pp = row_ok ? __ldg(a.pp + i) : 0.f;
      float bestv = __int_as_float(0x7f800000);
      uint32_t besti = 0xffffffffu;
      for (int ct = 0; ct < a.n_ct; ++ct) {
        const uint32_t buf = acc_i & 1u, use = (acc_i >> 1) & 1u;
        const int64_t jw = static_cast<int64_t>(ct) * bn + half * cols;  // first column of this warp
        // publish the prefetched metadata of this tile, then start fetching the next tile's
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int c = lane + 32 * t;
          if (c < cols) cc_w[c] = pf_cc[t];
        }
        __syncwarp();
        if (ct + 1 < a.n_ct)
          prefetch(rt, ct + 1);
        else
          prefetch(rt + gridDim.x, 0);
        if (!mbar_wait(&accf[buf], use, abort_flag, a.wait_ns)) { ok = false; break; }
        tc_fence_after();

        // one 32-column chunk: the reference's form and flag per pair
        auto process = [&](int ch, float (&v)[32]) {
          const int c0 = ch * 32;
          const int64_t j0 = jw + c0;
          const int64_t remc = a.m - j0;
          const int nvalid = remc <= 0 ? 0 : (remc >= 32 ? 32 : (int)remc);
          const uint32_t colmask = !row_ok ? 0u : (nvalid >= 32 ? 0xffffffffu : ((1u << nvalid) - 1u));
          {
            uint32_t fm = 0;
            // two columns at a time on packed fp32: each lane is the scalar operation of
            // exact_d and of the flag test (the same bits), the S rounding two at a time
            const uint64_t pp2 = f2_pack(pp, pp), m2 = f2_pack(-2.f, -2.f), K2 = f2_pack(K, K);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              uint64_t cc2;
              asm volatile("ld.shared.u64 %0, [%1];" : "=l"(cc2) : "r"(smem_u32(cc_w + c0 + e)));
              float s0 = v[e], s1 = v[e + 1];
              if constexpr (SROUND == SR_F16) {
                const float2 r = __half22float2(__floats2half2_rn(s0, s1));
                s0 = r.x;
                s1 = r.y;
              } else if constexpr (SROUND == SR_BF16) {
                const float2 r = __bfloat1622float2(__floats2bfloat162_rn(s0, s1));
                s0 = r.x;
                s1 = r.y;
              }
              float d2[2];
              f2_unpack(f2_add(f2_fma(m2, f2_pack(s0, s1), pp2), cc2), d2[0], d2[1]);
              float t2[2] = {0.f, 0.f};
              if constexpr (FLAG == FL_F32) f2_unpack(f2_mul(K2, f2_add(pp2, cc2)), t2[0], t2[1]);
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                const float d = fmaxf(d2[q], 0.f);
                bool fl = false;
                if constexpr (FLAG == FL_F32) fl = d <= t2[q];
                if constexpr (ARGMIN) {
                  if (((colmask >> (e + q)) & 1u) && !fl) {
                    if (d < bestv) { bestv = d; besti = static_cast<uint32_t>(j0 + e + q); }
                  }
                }
                if (fl) fm |= 1u << (e + q);
                v[e + q] = d;
              }
            }
            fm &= colmask;
            if constexpr (FLAG == FL_F32) {
              if (fm) {
                // append the flagged pairs of this row chunk to the recompute list
                unsigned long long pos = atomicAdd(a.count, static_cast<unsigned long long>(__popc(fm)));
                while (fm) {
                  const int e = __ffs(fm) - 1;
                  fm &= fm - 1;
                  const uint32_t jo = static_cast<uint32_t>(j0 + e);
                  if (pos < a.list_cap) {
                    a.list[pos] = (static_cast<unsigned long long>(i) << 32) | jo;
                  } else if constexpr (ARGMIN) {
                    // list full: recompute in place and fold into the row minimum
                    const float dd = overflow_direct<REC>(a.P + i * a.dim, a.C + static_cast<int64_t>(jo) * a.dim,
                                                          a.dim);
                    if (dd < bestv || (dd == bestv && jo < besti)) { bestv = dd; besti = jo; }
                  }
                  ++pos;
                  if (a.tile_counts != nullptr)
                    atomicAdd(&a.tile_counts[(i / a.tile_T) * a.tiles_j + static_cast<int64_t>(jo) / a.tile_T], 1);
                }
              }
            }
          }
          if constexpr (!ARGMIN) {
            if (row_ok) {
              if constexpr (MODE == TM_D_F32) {
                float* drow = static_cast<float*>(a.D) + i * a.m + j0;
                if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(drow) & 31u) == 0)) {
                  // 32-byte stores: each lane writes whole sectors of its row
#pragma unroll
                  for (int e = 0; e < 32; e += 8)
                    asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(drow + e), "f"(v[e]),
                                 "f"(v[e + 1]), "f"(v[e + 2]), "f"(v[e + 3]), "f"(v[e + 4]), "f"(v[e + 5]), "f"(v[e + 6]),
                                 "f"(v[e + 7])
                                 : "memory");
                } else if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(drow) & 15u) == 0)) {
#pragma unroll
                  for (int e = 0; e < 32; e += 4)
                    *reinterpret_cast<float4*>(drow + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                } else {
#pragma unroll
                  for (int e = 0; e < 32; ++e)
                    if (e < nvalid) drow[e] = v[e];
                }
              } else {
                // fp16 / bf16 output: D = round(d) (euclidean_kernels_uniform.cu:62,102)
                uint16_t* drow = static_cast<uint16_t*>(a.D) + i * a.m + j0;
                uint16_t hv[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                  if constexpr (MODE == TM_D_F16)
                    hv[e] = __half_as_ushort(__float2half_rn(v[e]));
                  else
                    hv[e] = __bfloat16_as_ushort(__float2bfloat16_rn(v[e]));
                }
                if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(drow) & 31u) == 0)) {
                  // 32-byte stores: each lane writes whole sectors of its row
#pragma unroll
                  for (int e = 0; e < 32; e += 16) {
                    uint32_t w[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) w[q] = hv[e + 2 * q] | (static_cast<uint32_t>(hv[e + 2 * q + 1]) << 16);
                    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(drow + e), "r"(w[0]),
                                 "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                                 : "memory");
                  }
                } else if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(drow) & 15u) == 0)) {
#pragma unroll
                  for (int e = 0; e < 32; e += 8) {
                    uint4 w;
                    w.x = hv[e] | (static_cast<uint32_t>(hv[e + 1]) << 16);
                    w.y = hv[e + 2] | (static_cast<uint32_t>(hv[e + 3]) << 16);
                    w.z = hv[e + 4] | (static_cast<uint32_t>(hv[e + 5]) << 16);
                    w.w = hv[e + 6] | (static_cast<uint32_t>(hv[e + 7]) << 16);
                    *reinterpret_cast<uint4*>(drow + e) = w;
                  }
                } else {
#pragma unroll
                  for (int e = 0; e < 32; ++e)
                    if (e < nvalid) drow[e] = hv[e];
                }
              }
            }
          }
        };

        const uint32_t tbase = lane_addr + buf * static_cast<uint32_t>(bn) + half * cols;
        for (int ch = 0; ch < nch; ch += 2) {
          float va[32], vb[32];
          if (ch + 1 < nch) {
            tmem_ld64(tbase + ch * 32, va, vb);  // two chunks per TMEM round trip
            process(ch, va);
            process(ch + 1, vb);
          } else {
            tmem_ld32(tbase + ch * 32, va);
            process(ch, va);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[buf]);
        ++acc_i;
      }
      if constexpr (ARGMIN) {
        if (!ok) break;
        // the two column halves' minima of a row meet in its key: a 64-bit atomic min of
        // (distance bits, original index), the smaller index among equal distances, with
        // no barrier between the halves (the key starts at ~0)
        if (row_ok) atomicMin(&a.row_key[i], make_key(bestv, besti));
      }
    }
    if (!ok) {
      *abort_flag = 1;
      if (lane == 0) atomicExch(&s_tc_err, DEV_TIMEOUT_EPILOGUE);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, ncols);
}

// ------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Row-major [rows x ld] matrix of `esize`-byte elements, box = 128 bytes x box_rows.
bool tc_make_tmap(CUtensorMap* map, const void* base, int64_t rows, int ld, int esize, int box_rows,
                      bool is_f32, bool is_bf16) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t gdim[2] = {static_cast<cuuint64_t>(ld), static_cast<cuuint64_t>(rows)};
  cuuint64_t gstride[1] = {static_cast<cuuint64_t>(ld) * esize};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esize), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapDataType dt = is_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : (is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Row-major [rows x (32 / esize)] matrix (32-byte rows), box = 32 bytes x box_rows,
// 32-byte swizzle.
bool tc_make_tmap_sw32(CUtensorMap* map, const void* base, int64_t rows, int esize, int box_rows, bool is_f32,
                       bool is_bf16) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t gdim[2] = {static_cast<cuuint64_t>(32 / esize), static_cast<cuuint64_t>(rows)};
  cuuint64_t gstride[1] = {32};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(32 / esize), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapDataType dt = is_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : (is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int pick_bn(int64_t m) {
  if (m <= 64) return 64;
  if (m <= 128) return 128;
  return 256;
}

constexpr size_t TC_SMEM_LIMIT = 232448;  // 227 KiB opt-in per block on sm_100
constexpr size_t TC_FIXED = 1024 /*alignment slack*/ + TC_BAR_BYTES + TC_EPI_BYTES;

// Pick the pipeline: resident A (double-buffered) with as many B stages as fit, or,
// when two A tiles do not fit next to 3 B stages, streaming (A + B) stages.
static void pick_pipeline(int bn, int kblocks, int* nst, int* a_res) {
  const size_t b = static_cast<size_t>(bn) * 128, abytes = static_cast<size_t>(kblocks) * TC_A_BYTES;
  const size_t avail = TC_SMEM_LIMIT - TC_FIXED;
  if (2 * abytes + 3 * b <= avail) {
    *a_res = 1;
    *nst = static_cast<int>(std::min<size_t>(8, (avail - 2 * abytes) / b));
  } else {
    *a_res = 0;
    *nst = static_cast<int>(std::min<size_t>(8, avail / (TC_A_BYTES + b)));
  }
}

size_t tc_smem_bytes(int bn, int kblocks, int nst, int a_res) {
  const size_t b = static_cast<size_t>(bn) * 128;
  const size_t body = a_res ? 2 * static_cast<size_t>(kblocks) * TC_A_BYTES + nst * b : nst * (TC_A_BYTES + b);
  return TC_FIXED + body;
}

template <int KIND, int SROUND, int FLAG, int MODE, int REC>
static cudaError_t launch_tc_t(const CUtensorMap& ta, const CUtensorMap& tb, const TcArgs& args,
                               cudaStream_t st) {
  auto kern = dist_tc_kernel<KIND, SROUND, FLAG, MODE, REC>;
  const size_t smem = tc_smem_bytes(args.bn, args.kblocks, args.nst, args.a_res);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int grid = num_sms();
  if (static_cast<int64_t>(grid) > args.n_rt) grid = static_cast<int>(args.n_rt);
  if (grid < 1) grid = 1;
  timing_begin(st, "dist_tc_kernel");
  kern<<<grid, TC_THREADS, smem, st>>>(ta, tb, args);
  e = cudaGetLastError();
  timing_end(st);
  return e;
}

cudaError_t launch_tc(const DistJob& j) {
  const OpSpec* s = j.spec;
  const int kind = (s->gemm == G_TC_F16) ? 0 : (s->gemm == G_TC_BF16 ? 1 : 2);
  const int esize = (kind == 2) ? 4 : 2;
  TcArgs a{};
  a.n = j.n;
  a.m = j.m;
  a.dim = j.dim;
  a.kblocks = static_cast<int>((static_cast<int64_t>(j.ldlow) * esize) / 128);
  a.bn = pick_bn(j.m);
  a.n_ct = static_cast<int>((j.m + a.bn - 1) / a.bn);
  a.n_rt = (j.n + TC_BM - 1) / TC_BM;
  pick_pipeline(a.bn, a.kblocks, &a.nst, &a.a_res);
  a.pp = static_cast<const float*>(j.pp);
  a.cc = static_cast<const float*>(j.cc);
  a.K = j.kf;
  a.D = j.D;
  a.row_key = j.row_key;
  a.list = j.list;
  a.list_cap = j.list_cap;
  a.count = j.count;
  a.tile_counts = j.tile_counts;
  a.tile_T = j.tile_T > 0 ? j.tile_T : 1;
  a.tiles_j = j.tiles_j;
  a.P = static_cast<const float*>(j.P);
  a.C = static_cast<const float*>(j.C);
  a.wait_ns = wait_limit_ns();

  CUtensorMap ta, tb;
  if (!tc_make_tmap(&ta, j.Plow, j.n, j.ldlow, esize, TC_BM, kind == 2, kind == 1)) return cudaErrorInvalidValue;
  if (!tc_make_tmap(&tb, j.Clow, j.m, j.ldlow, esize, a.bn, kind == 2, kind == 1))
    return cudaErrorInvalidValue;

  const bool argmin = (j.D == nullptr);
  int mode = TM_ARGMIN;
  if (!argmin) mode = (s->out == OUT_F16) ? TM_D_F16 : (s->out == OUT_BF16 ? TM_D_BF16 : TM_D_F32);
  const cudaStream_t st = j.stream;
  if (argmin && j.row_key) {
    // the two column halves fold their row minima into the key with an atomic min
    const cudaError_t e = cudaMemsetAsync(j.row_key, 0xff, static_cast<size_t>(j.n) * sizeof(unsigned long long), st);
    if (e != cudaSuccess) return e;
  }

#define TC_CASE1(KIND_, SR_, FL_, MODE_, REC_)                                                      \
  if (kind == KIND_ && s->sround == SR_ && s->flag == FL_ && mode == MODE_ &&                        \
      (MODE_ != TM_ARGMIN || s->rec == REC_))                                                         \
    return launch_tc_t<KIND_, SR_, FL_, MODE_, REC_>(ta, tb, a, st);
#define TC_CASE(KIND_, SR_, FL_, MODE_, REC_) TC_CASE1(KIND_, SR_, FL_, MODE_, REC_)
#define TC_CASE_A(KIND_, SR_, FL_, REC_) TC_CASE1(KIND_, SR_, FL_, TM_ARGMIN, REC_)

  // fp16 operands
  TC_CASE(0, SR_F16, FL_F32, TM_D_F32, RC_NONE)      // mix fp16_*
  TC_CASE(0, SR_NONE, FL_F32, TM_D_F32, RC_NONE)     // tiled / tensorcore fp16_*
  TC_CASE(0, SR_F16, FL_NONE, TM_D_F16, RC_NONE)     // uniform fp16
  TC_CASE_A(0, SR_F16, FL_F32, RC_F64)
  TC_CASE_A(0, SR_F16, FL_F32, RC_F32)
  TC_CASE_A(0, SR_F16, FL_F32, RC_F16_ARITH)
  TC_CASE_A(0, SR_NONE, FL_F32, RC_F64)
  TC_CASE_A(0, SR_NONE, FL_F32, RC_F32)
  // bf16 operands
  TC_CASE(1, SR_BF16, FL_F32, TM_D_F32, RC_NONE)
  TC_CASE(1, SR_NONE, FL_F32, TM_D_F32, RC_NONE)
  TC_CASE(1, SR_BF16, FL_NONE, TM_D_BF16, RC_NONE)
  TC_CASE_A(1, SR_BF16, FL_F32, RC_F64)
  TC_CASE_A(1, SR_BF16, FL_F32, RC_F32)
  TC_CASE_A(1, SR_BF16, FL_F32, RC_BF16_ARITH)
  TC_CASE_A(1, SR_NONE, FL_F32, RC_F64)
  TC_CASE_A(1, SR_NONE, FL_F32, RC_F32)
  // tf32 operands
  TC_CASE(2, SR_NONE, FL_F32, TM_D_F32, RC_NONE)
  TC_CASE_A(2, SR_NONE, FL_F32, RC_F64)
#undef TC_CASE
#undef TC_CASE_A
#undef TC_CASE1
  return cudaErrorNotSupported;
}

int tc_error_and_clear() {
  int v = 0, z = 0;
  cudaMemcpyFromSymbol(&v, s_tc_err, sizeof(int));
  if (v) cudaMemcpyToSymbol(s_tc_err, &z, sizeof(int));
  return v;
}

}  // namespace euc
