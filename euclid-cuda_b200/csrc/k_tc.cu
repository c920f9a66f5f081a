// Fused distance kernel on the 5th-generation tensor cores (sm_100a).
//
// One persistent CTA per SM walks 128-row tiles of the points.  For each row tile
// it sweeps every center tile (bn = 64/128/256 centers):
//   warp 0  : TMA producer, streams (A: 128 x 64 fp16/bf16 | 128 x 32 tf32) and
//             (B: bn x same) K-blocks into a 4-stage ring of 128B-swizzled smem;
//   warp 1  : tcgen05.mma issuer (one elected lane), M=128 x N=bn x K=16|8 per
//             instruction, fp32 accumulators double-buffered in TMEM (2*bn columns);
//             also owns the TMEM allocation;
//   warps 2-5: epilogue; each thread owns one TMEM lane = one point row.  It reads
//             32 accumulator columns at a time (tcgen05.ld 32x32b.x32), applies the
//             reference's S rounding, forms d = max((pp - 2s) + cc, 0), runs the
//             cancellation test d <= K (pp + cc) and either stores D or keeps the
//             running (min, first index) of the row.  Flagged pairs are appended to
//             a compact list with one atomic per warp (ballot + popc).
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

namespace euc {

static __device__ int s_tc_err;

constexpr int TC_BM = 128;
constexpr int TC_STAGES = 4;
constexpr int TC_EPI_WARPS = 4;
constexpr int TC_THREADS = (2 + TC_EPI_WARPS) * 32;
constexpr int TC_A_BYTES = TC_BM * 128;  // one K-block of A: 128 rows x 128 bytes

enum TcMode { TM_ARGMIN = 0, TM_D_F32 = 1, TM_D_F16 = 2, TM_D_BF16 = 3 };

struct TcArgs {
  int64_t n, m;
  int dim;
  int kblocks;  // K-blocks of 128 bytes
  int bn;
  int n_ct;     // center tiles
  int64_t n_rt; // row tiles
  const float* pp;
  const float* cc;
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
};

template <int KIND, int SROUND, int FLAG, int MODE, int REC>
__global__ void __launch_bounds__(TC_THREADS, 1)
    dist_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment of every stage (required by the 128B swizzle atoms)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bn = a.bn;
  const uint32_t b_bytes = static_cast<uint32_t>(bn) * 128u;
  const uint32_t stage_bytes = TC_A_BYTES + b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_STAGES * stage_bytes);
  uint64_t* empty = full + TC_STAGES;
  uint64_t* accf = empty + TC_STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ncols = 2u * static_cast<uint32_t>(bn);  // power of two >= 128

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
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

  const int64_t n_tiles = a.n_rt * a.n_ct;  // (row tile, center tile) pairs owned round-robin by row tile
  (void)n_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, last_phase = 0;
      bool ok = true;
      const int kelems = (KIND == 2) ? 32 : 64;  // elements per 128-byte K-block
      for (int64_t rt = blockIdx.x; rt < a.n_rt && ok; rt += gridDim.x) {
        for (int ct = 0; ct < a.n_ct && ok; ++ct) {
          for (int kb = 0; kb < a.kblocks; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
            uint8_t* sA = smem + stage * stage_bytes;
            uint8_t* sB = sA + TC_A_BYTES;
            mbar_arrive_expect_tx(&full[stage], stage_bytes);
            tma_load_2d(sA, &tmA, &full[stage], kb * kelems, static_cast<int>(rt * TC_BM));
            tma_load_2d(sB, &tmB, &full[stage], kb * kelems, ct * bn);
            issued_mask |= 1u << stage;
            last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
            if (++stage == TC_STAGES) { stage = 0; phase ^= 1u; }
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(&s_tc_err, DEV_TIMEOUT_PRODUCER);
      }
      // Drain: every issued stage's last load must have landed before smem is released.
      for (int s = 0; s < TC_STAGES; ++s)
        if (issued_mask & (1u << s)) {
          volatile int no_abort = 0;
          mbar_wait(&full[s], (last_phase >> s) & 1u, &no_abort);
        }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = (KIND == 0) ? 0u : (KIND == 1 ? 1u : 2u);
      const uint32_t idesc = umma_idesc(fmt, TC_BM, static_cast<uint32_t>(bn));
      uint32_t stage = 0, phase = 0, acc_i = 0;
      bool ok = true;
      for (int64_t rt = blockIdx.x; rt < a.n_rt && ok; rt += gridDim.x) {
        for (int ct = 0; ct < a.n_ct && ok; ++ct) {
          const uint32_t buf = acc_i & 1u, use = (acc_i >> 1) & 1u;
          if (!mbar_wait(&acce[buf], use ^ 1u, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * static_cast<uint32_t>(bn);
          for (int kb = 0; kb < a.kblocks; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sA = smem_u32(smem + stage * stage_bytes);
            const uint32_t sB = sA + TC_A_BYTES;
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
            if (++stage == TC_STAGES) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          umma_commit(&accf[buf]);
          ++acc_i;
        }
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
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_local = q * 32 + lane;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    const float K = a.K;
    uint32_t acc_i = 0;
    bool ok = true;
    for (int64_t rt = blockIdx.x; rt < a.n_rt && ok; rt += gridDim.x) {
      const int64_t i = rt * TC_BM + row_local;
      const bool row_ok = i < a.n;
      const float pp = row_ok ? __ldg(a.pp + i) : 0.f;
      unsigned long long best = ~0ull;
      for (int ct = 0; ct < a.n_ct; ++ct) {
        const uint32_t buf = acc_i & 1u, use = (acc_i >> 1) & 1u;
        if (!mbar_wait(&accf[buf], use, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int ch = 0; ch < bn / 32; ++ch) {
          float v[32];
          tmem_ld32(lane_addr + buf * static_cast<uint32_t>(bn) + ch * 32, v);
          const int64_t j0 = static_cast<int64_t>(ct) * bn + ch * 32;
          const bool full_chunk = (j0 + 32) <= a.m;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int64_t j = j0 + e;
            const bool valid = row_ok && (full_chunk || j < a.m);
            const float cc = (full_chunk || j < a.m) ? __ldg(a.cc + j) : 0.f;
            float s = v[e];
            if constexpr (SROUND == SR_F16) s = round_f16(s);
            if constexpr (SROUND == SR_BF16) s = round_bf16(s);
            float d = __fadd_rn(__fmaf_rn(-2.f, s, pp), cc);
            d = fmaxf(d, 0.f);
            bool flag = false;
            if constexpr (FLAG == FL_F32) flag = valid && (d <= __fmul_rn(K, __fadd_rn(pp, cc)));
            if constexpr (MODE == TM_ARGMIN) {
              if (valid && !flag) {
                const unsigned long long key = make_key(d, static_cast<uint32_t>(j));
                best = key < best ? key : best;
              }
            }
            v[e] = d;
            if constexpr (FLAG == FL_F32) {
              const unsigned msk = __ballot_sync(0xffffffffu, flag);
              if (msk) {
                const int leader = __ffs(msk) - 1;
                unsigned long long base = 0;
                if (lane == leader) base = atomicAdd(a.count, static_cast<unsigned long long>(__popc(msk)));
                base = __shfl_sync(0xffffffffu, base, leader);
                if (flag) {
                  const unsigned long long pos = base + __popc(msk & ((1u << lane) - 1u));
                  if (pos < a.list_cap) {
                    a.list[pos] = (static_cast<unsigned long long>(i) << 32) | static_cast<unsigned long long>(j);
                  } else if constexpr (MODE == TM_ARGMIN) {
                    // list full: recompute in place and fold into the row minimum
                    const float dd = static_cast<float>(direct_dist<float, REC>(a.P + i * a.dim, a.C + j * a.dim, a.dim));
                    const unsigned long long key = make_key(dd, static_cast<uint32_t>(j));
                    best = key < best ? key : best;
                  }
                  if (a.tile_counts != nullptr)
                    atomicAdd(&a.tile_counts[(i / a.tile_T) * a.tiles_j + j / a.tile_T], 1);
                }
              }
            }
          }
          if constexpr (MODE != TM_ARGMIN) {
            if (row_ok) {
              if constexpr (MODE == TM_D_F32) {
                float* drow = static_cast<float*>(a.D) + i * a.m + j0;
                if (full_chunk && ((reinterpret_cast<uintptr_t>(drow) & 15u) == 0)) {
#pragma unroll
                  for (int e = 0; e < 32; e += 4)
                    *reinterpret_cast<float4*>(drow + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                } else {
                  for (int e = 0; e < 32; ++e)
                    if (j0 + e < a.m) drow[e] = v[e];
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
                if (full_chunk && ((reinterpret_cast<uintptr_t>(drow) & 15u) == 0)) {
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
                  for (int e = 0; e < 32; ++e)
                    if (j0 + e < a.m) drow[e] = hv[e];
                }
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[buf]);
        ++acc_i;
      }
      if constexpr (MODE == TM_ARGMIN) {
        if (ok && row_ok) a.row_key[i] = best;
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
static bool make_tmap(CUtensorMap* map, const void* base, int64_t rows, int ld, int esize, int box_rows,
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

static int pick_bn(int64_t m) {
  if (m <= 64) return 64;
  if (m <= 128) return 128;
  return 256;
}

size_t tc_smem_bytes(int bn) {
  return 1024 /*alignment slack*/ + TC_STAGES * (TC_A_BYTES + bn * 128) + 256 /*barriers*/;
}

template <int KIND, int SROUND, int FLAG, int MODE, int REC>
static cudaError_t launch_tc_t(const CUtensorMap& ta, const CUtensorMap& tb, const TcArgs& args,
                               cudaStream_t st) {
  auto kern = dist_tc_kernel<KIND, SROUND, FLAG, MODE, REC>;
  const size_t smem = tc_smem_bytes(args.bn);
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

  CUtensorMap ta, tb;
  if (!make_tmap(&ta, j.Plow, j.n, j.ldlow, esize, TC_BM, kind == 2, kind == 1)) return cudaErrorInvalidValue;
  if (!make_tmap(&tb, j.Clow, j.m, j.ldlow, esize, a.bn, kind == 2, kind == 1)) return cudaErrorInvalidValue;

  const bool argmin = (j.D == nullptr);
  int mode = TM_ARGMIN;
  if (!argmin) mode = (s->out == OUT_F16) ? TM_D_F16 : (s->out == OUT_BF16 ? TM_D_BF16 : TM_D_F32);
  const cudaStream_t st = j.stream;

#define TC_CASE(KIND_, SR_, FL_, MODE_, REC_)                                                        \
  if (kind == KIND_ && s->sround == SR_ && s->flag == FL_ && mode == MODE_ && (MODE_ != TM_ARGMIN || \
                                                                             s->rec == REC_))       \
    return launch_tc_t<KIND_, SR_, FL_, MODE_, REC_>(ta, tb, a, st);

  // fp16 operands
  TC_CASE(0, SR_F16, FL_F32, TM_D_F32, RC_NONE)      // mix fp16_*
  TC_CASE(0, SR_NONE, FL_F32, TM_D_F32, RC_NONE)     // tiled / tensorcore fp16_*
  TC_CASE(0, SR_F16, FL_NONE, TM_D_F16, RC_NONE)     // uniform fp16
  TC_CASE(0, SR_F16, FL_F32, TM_ARGMIN, RC_F64)
  TC_CASE(0, SR_F16, FL_F32, TM_ARGMIN, RC_F32)
  TC_CASE(0, SR_F16, FL_F32, TM_ARGMIN, RC_F16_ARITH)
  TC_CASE(0, SR_NONE, FL_F32, TM_ARGMIN, RC_F64)
  TC_CASE(0, SR_NONE, FL_F32, TM_ARGMIN, RC_F32)
  // bf16 operands
  TC_CASE(1, SR_BF16, FL_F32, TM_D_F32, RC_NONE)
  TC_CASE(1, SR_NONE, FL_F32, TM_D_F32, RC_NONE)
  TC_CASE(1, SR_BF16, FL_NONE, TM_D_BF16, RC_NONE)
  TC_CASE(1, SR_BF16, FL_F32, TM_ARGMIN, RC_F64)
  TC_CASE(1, SR_BF16, FL_F32, TM_ARGMIN, RC_F32)
  TC_CASE(1, SR_BF16, FL_F32, TM_ARGMIN, RC_BF16_ARITH)
  TC_CASE(1, SR_NONE, FL_F32, TM_ARGMIN, RC_F64)
  TC_CASE(1, SR_NONE, FL_F32, TM_ARGMIN, RC_F32)
  // tf32 operands
  TC_CASE(2, SR_NONE, FL_F32, TM_D_F32, RC_NONE)
  TC_CASE(2, SR_NONE, FL_F32, TM_ARGMIN, RC_F64)
#undef TC_CASE
  return cudaErrorNotSupported;
}

int tc_error_and_clear() {
  int v = 0, z = 0;
  cudaMemcpyFromSymbol(&v, s_tc_err, sizeof(int));
  if (v) cudaMemcpyToSymbol(s_tc_err, &z, sizeof(int));
  return v;
}

}  // namespace euc
