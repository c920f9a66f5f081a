// C ABI of the distance engine (declared in include/euclid_b200.h).
//
// Each reference operator is one row of kOps: the numeric recipe it follows
// (input type, how S is produced and rounded, how the norms are accumulated, the
// cancellation threshold, the fallback arithmetic and the output type).  All
// distance entries go through run_distance(): prep (norms, low copies) ->
// tensor-core or CUDA-core distance kernel -> compacted recompute -> labels.
#include "engine.h"
#include "common.cuh"
#include "../../include/euclid_b200.h"

#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <algorithm>

namespace euc {

// clang-format off
static const OpSpec kOps[] = {
  // op                         name                                   in       gemm        sround   norm          form           flag    rec            out      kform u
  {EUC_OP_SINGLE,             "pairwise_euclidean_single",             IN_F32,  G_SIMT_F32, SR_NONE, NM_F32_FMA,   FM_F32,        FL_NONE, RC_NONE,      OUT_F32, 0, 0.0},
  {EUC_OP_DOUBLE,             "pairwise_euclidean_double",             IN_F64,  G_SIMT_F64, SR_NONE, NM_F64_FMA,   FM_F64,        FL_NONE, RC_NONE,      OUT_F64, 0, 0.0},
  {EUC_OP_MIX_FP16_FP64,      "pairwise_euclidean_fp16_fp64",          IN_F32,  G_TC_F16,   SR_F16,  NM_LOW_F16,   FM_F32,        FL_F32,  RC_F64,       OUT_F32, 0, 0x1p-11},
  {EUC_OP_MIX_BF16_FP64,      "pairwise_euclidean_bf16_fp64",          IN_F32,  G_TC_BF16,  SR_BF16, NM_LOW_BF16,  FM_F32,        FL_F32,  RC_F64,       OUT_F32, 0, 0x1p-7},
  {EUC_OP_MIX_TF32_FP64,      "pairwise_euclidean_tf32_fp64",          IN_F32,  G_TC_TF32,  SR_NONE, NM_F32_FMA,   FM_F32,        FL_F32,  RC_F64,       OUT_F32, 0, 0x1p-11},
  {EUC_OP_MIX_FP32_FP64,      "pairwise_euclidean_fp32_fp64",          IN_F32,  G_SIMT_F32, SR_NONE, NM_F32_FMA,   FM_F32,        FL_F32,  RC_F64,       OUT_F32, 1, 0x1p-23},
  {EUC_OP_MIX_FP16_FP16,      "pairwise_euclidean_fp16_fp16",          IN_F32,  G_TC_F16,   SR_F16,  NM_LOW_F16,   FM_F32,        FL_F32,  RC_F16_ARITH, OUT_F32, 0, 0x1p-11},
  {EUC_OP_MIX_FP16_FP32,      "pairwise_euclidean_fp16_fp32",          IN_F32,  G_TC_F16,   SR_F16,  NM_LOW_F16,   FM_F32,        FL_F32,  RC_F32,       OUT_F32, 0, 0x1p-11},
  {EUC_OP_MIX_BF16_BF16,      "pairwise_euclidean_bf16_bf16",          IN_F32,  G_TC_BF16,  SR_BF16, NM_LOW_BF16,  FM_F32,        FL_F32,  RC_BF16_ARITH,OUT_F32, 0, 0x1p-7},
  {EUC_OP_MIX_BF16_FP32,      "pairwise_euclidean_bf16_fp32",          IN_F32,  G_TC_BF16,  SR_BF16, NM_LOW_BF16,  FM_F32,        FL_F32,  RC_F32,       OUT_F32, 0, 0x1p-7},
  {EUC_OP_MIX_FP32_FP32,      "pairwise_euclidean_fp32_fp32",          IN_F32,  G_SIMT_F32, SR_NONE, NM_F32_FMA,   FM_F32,        FL_F32,  RC_F32,       OUT_F32, 0, 0x1p-23},
  {EUC_OP_TILED_FP16_FP64,    "pairwise_euclidean_tiled_fp16_fp64",    IN_F32,  G_TC_F16,   SR_NONE, NM_F32_SUMSQ, FM_F32,        FL_F32,  RC_F64,       OUT_F32, 0, 0x1p-11},
  {EUC_OP_TILED_FP16_FP32,    "pairwise_euclidean_tiled_fp16_fp32",    IN_F32,  G_TC_F16,   SR_NONE, NM_F32_SUMSQ, FM_F32,        FL_F32,  RC_F32,       OUT_F32, 0, 0x1p-11},
  {EUC_OP_TILED_BF16_FP64,    "pairwise_euclidean_tiled_bf16_fp64",    IN_F32,  G_TC_BF16,  SR_NONE, NM_F32_SUMSQ, FM_F32,        FL_F32,  RC_F64,       OUT_F32, 0, 0x1p-8},
  {EUC_OP_TILED_BF16_FP32,    "pairwise_euclidean_tiled_bf16_fp32",    IN_F32,  G_TC_BF16,  SR_NONE, NM_F32_SUMSQ, FM_F32,        FL_F32,  RC_F32,       OUT_F32, 0, 0x1p-8},
  {EUC_OP_TILED_FP32_FP64,    "pairwise_euclidean_tiled_fp32_fp64",    IN_F32,  G_SIMT_F32, SR_NONE, NM_F32_SUMSQ, FM_F32,        FL_F32,  RC_F64,       OUT_F32, 0, 0x1p-23},
  {EUC_OP_TILED_FP32_FP32,    "pairwise_euclidean_tiled_fp32_fp32",    IN_F32,  G_SIMT_F32, SR_NONE, NM_F32_SUMSQ, FM_F32,        FL_F32,  RC_F32,       OUT_F32, 0, 0x1p-23},
  {EUC_OP_TC_FP16_FP64,       "pairwise_euclidean_tensorcore_fp16_fp64", IN_F32, G_TC_F16,  SR_NONE, NM_F32_SUMSQ, FM_F32,        FL_F32,  RC_F64,       OUT_F32, 0, 0x1p-11},
  {EUC_OP_TC_FP16_FP32,       "pairwise_euclidean_tensorcore_fp16_fp32", IN_F32, G_TC_F16,  SR_NONE, NM_F32_SUMSQ, FM_F32,        FL_F32,  RC_F32,       OUT_F32, 0, 0x1p-11},
  {EUC_OP_TC_BF16_FP64,       "pairwise_euclidean_tensorcore_bf16_fp64", IN_F32, G_TC_BF16, SR_NONE, NM_F32_SUMSQ, FM_F32,        FL_F32,  RC_F64,       OUT_F32, 0, 0x1p-8},
  {EUC_OP_TC_BF16_FP32,       "pairwise_euclidean_tensorcore_bf16_fp32", IN_F32, G_TC_BF16, SR_NONE, NM_F32_SUMSQ, FM_F32,        FL_F32,  RC_F32,       OUT_F32, 0, 0x1p-8},
  {EUC_OP_UNI_FP16,           "pairwise_euclidean_uniform_fp16",       IN_F16,  G_TC_F16,   SR_F16,  NM_LOW_F16,   FM_F32,        FL_NONE, RC_NONE,      OUT_F16, 0, 0.0},
  {EUC_OP_UNI_BF16,           "pairwise_euclidean_uniform_bf16",       IN_BF16, G_TC_BF16,  SR_BF16, NM_LOW_BF16,  FM_F32,        FL_NONE, RC_NONE,      OUT_BF16,0, 0.0},
  {EUC_OP_UNI_TF32,           "pairwise_euclidean_uniform_tf32",       IN_F32,  G_SIMT_F32, SR_NONE, NM_F32_FMA,   FM_F32,        FL_NONE, RC_NONE,      OUT_F32, 0, 0.0},
  {EUC_OP_UNI_FP16_DIRECT,    "pairwise_euclidean_uniform_fp16_direct", IN_F16, G_DIRECT,   SR_NONE, NM_F32_FMA,   FM_F32,        FL_NONE, RC_NONE,      OUT_F16, 0, 0.0},
  {EUC_OP_UNI_BF16_DIRECT,    "pairwise_euclidean_uniform_bf16_direct", IN_BF16,G_DIRECT,   SR_NONE, NM_F32_FMA,   FM_F32,        FL_NONE, RC_NONE,      OUT_BF16,0, 0.0},
  {EUC_OP_UNI_TF32_DIRECT,    "pairwise_euclidean_uniform_tf32_direct", IN_F32, G_DIRECT,   SR_NONE, NM_F32_FMA,   FM_F32,        FL_NONE, RC_NONE,      OUT_F32, 0, 0.0},
  {EUC_OP_UNI_FP32_DIRECT,    "pairwise_euclidean_uniform_fp32_direct", IN_F32, G_DIRECT,   SR_NONE, NM_F32_FMA,   FM_F32,        FL_NONE, RC_NONE,      OUT_F32, 0, 0.0},
  {EUC_OP_UNI_FP64_DIRECT,    "pairwise_euclidean_uniform_fp64_direct", IN_F64, G_DIRECT,   SR_NONE, NM_F64_FMA,   FM_F64,        FL_NONE, RC_NONE,      OUT_F64, 0, 0.0},
  {EUC_OP_ADV_FP64_FP16,      "pairwise_euclidean_fp64_fp16",          IN_F16,  G_SIMT_F64, SR_NONE, NM_F32_FMA,   FM_F64_TO_F32, FL_F32,  RC_F64,       OUT_F32, 1, 0x1p-23},
  {EUC_OP_ADV_FP64_BF16,      "pairwise_euclidean_fp64_bf16",          IN_BF16, G_SIMT_F64, SR_NONE, NM_F32_FMA,   FM_F64_TO_F32, FL_F32,  RC_F64,       OUT_F32, 1, 0x1p-23},
  {EUC_OP_ADV_FP64_TF32,      "pairwise_euclidean_fp64_tf32",          IN_F32,  G_SIMT_F32, SR_NONE, NM_F64_FMA,   FM_F64,        FL_F64,  RC_F64,       OUT_F64, 2, 0x1p-52},
  {EUC_OP_ADV_FP64_FP32_GEMM, "pairwise_euclidean_fp64_fp32_gemm",     IN_F64,  G_SIMT_F32, SR_NONE, NM_F64_FMA,   FM_F64,        FL_F64,  RC_F64,       OUT_F64, 2, 0x1p-52},
};
// clang-format on

const OpSpec* find_op(int op) {
  for (const auto& s : kOps)
    if (s.op == op) return &s;
  return nullptr;
}

// ------------------------------------------------------------------ errors
static thread_local std::string g_err;
static int fail(int status, const std::string& msg) {
  g_err = msg;
  return status;
}
static int ok() { return EUC_OK; }
int set_error(int status, const char* msg) { return fail(status, msg); }
static int cuda_fail(cudaError_t e, const char* where) {
  return fail(EUC_ERR_LAUNCH, std::string(where) + ": " + cudaGetErrorString(e));
}

// ------------------------------------------------------------------ device info
static int g_sms[64];
int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (g_sms[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    g_sms[dev] = v > 0 ? v : 1;
  }
  return g_sms[dev];
}
int tc_error_and_clear();
int tf_error_and_clear();
int device_error_and_clear() {
  const int a = tc_error_and_clear(), b = tf_error_and_clear();
  return a ? a : b;
}

bool device_is_sm100() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  return major == 10;
}

// ------------------------------------------------------------------ wait limit
static std::atomic<unsigned long long> g_wait_ns{kWaitLimitNs};
static std::atomic<int> g_withhold{0};
unsigned long long wait_limit_ns() { return g_wait_ns.load(); }
bool take_withhold() { return g_withhold.exchange(0) != 0; }

// ------------------------------------------------------------------ timing
static bool g_timing = false;
static cudaEvent_t g_ev0 = nullptr, g_ev1 = nullptr;
static bool g_ev_recorded = false;
static const char* g_ev_name = "";
void timing_begin(cudaStream_t st, const char* name) {
  if (!g_timing) return;
  if (!g_ev0) {
    cudaEventCreate(&g_ev0);
    cudaEventCreate(&g_ev1);
  }
  g_ev_name = name;
  cudaEventRecord(g_ev0, st);
}
void timing_end(cudaStream_t st) {
  if (!g_timing || !g_ev1) return;
  cudaEventRecord(g_ev1, st);
  g_ev_recorded = true;
}

// ------------------------------------------------------------------ workspace
static inline size_t al(size_t b) { return (b + 255) & ~size_t(255); }

struct Layout {
  size_t hdr, pp, cc, plow, clow, clow_s, cc_s, perm, list, key, val64, idx64, rcnt, redo, clist, cs, baux, total;
  unsigned long long cap, ccap;
  int ldlow;
};

constexpr int kMaxRegions = 1024;  // CTAs of the fast argmin screen: at most one per SM

static int low_esize(const OpSpec* s) { return s->gemm == G_TC_TF32 ? 4 : 2; }
static bool is_tc(const OpSpec* s) { return s->gemm == G_TC_F16 || s->gemm == G_TC_BF16 || s->gemm == G_TC_TF32; }

// `prepared`: the points' low-precision copy and norms come from the caller
// (euc_argmin_prepared), so the workspace holds neither
static Layout layout_for(const OpSpec* s, int64_t n, int64_t m, int64_t dim, bool argmin, bool prepared = false) {
  Layout L{};
  const size_t nsz = (s->form == FM_F64) ? 8 : 4;
  const int es = low_esize(s);
  const int per_box = 128 / es;
  L.ldlow = static_cast<int>(((dim + per_box - 1) / per_box) * per_box);
  size_t off = 0;
  L.hdr = off; off += 256;
  L.pp = off; if (!prepared) off += al(static_cast<size_t>(n) * nsz);
  L.cc = off; off += al(static_cast<size_t>(m) * nsz);
  if (is_tc(s)) {
    L.plow = off; if (!prepared) off += al(static_cast<size_t>(n) * L.ldlow * es);
    L.clow = off; off += al(static_cast<size_t>(m) * L.ldlow * es);
    if (argmin && s->flag != FL_NONE) {  // norm-sorted centers for the fast argmin screen
      // norms and original indices padded to whole 256-center tiles (copied tile by tile)
      const size_t mpad = static_cast<size_t>((m + 255) / 256) * 256;
      L.clow_s = off; off += al(static_cast<size_t>(m) * L.ldlow * es);
      L.cc_s = off; off += al(mpad * 4);
      L.perm = off; off += al(mpad * 4);
      L.rcnt = off; off += al(static_cast<size_t>(kMaxRegions) * 4);
      L.redo = off; off += al(static_cast<size_t>(n));
      L.baux = off; off += al(mpad * 32);  // extra K block of the screening MMA: 32 bytes per center
    }
  }
  L.cap = 0;
  if (s->flag != FL_NONE) {
    const unsigned long long nm = static_cast<unsigned long long>(n) * static_cast<unsigned long long>(m);
    unsigned long long cap = nm / 256;
    cap = std::max<unsigned long long>(cap, 1ull << 16);
    cap = std::min<unsigned long long>(cap, 1ull << 26);
    cap = std::min<unsigned long long>(cap, nm);
    L.cap = cap;
    L.list = off; off += al(cap * 8);
    if (L.redo) {
      // fast argmin lists candidate 32-center chunks with their accumulators: room for two per row
      const unsigned long long chunks = static_cast<unsigned long long>(n) * static_cast<unsigned long long>((m + 31) / 32);
      L.ccap = std::min<unsigned long long>(chunks, std::max<unsigned long long>(2ull * n, 1ull << 16));
      L.clist = off; off += al(L.ccap * 8);
      L.cs = off; off += al(L.ccap * 128);
    }
  }
  if (argmin) {
    if (s->form == FM_F64 && s->flag == FL_NONE) {
      L.val64 = off; off += al(static_cast<size_t>(n) * 8);
      L.idx64 = off; off += al(static_cast<size_t>(n) * 8);
    } else {
      L.key = off; off += al(static_cast<size_t>(n) * 8);
    }
  }
  L.total = off;
  return L;
}

static double k_double(const OpSpec* s, float kappa, int64_t dim) {
  if (s->kform == 2) return (static_cast<double>(kappa) * 2.0) * (static_cast<double>(dim) * s->u);
  return 0.0;
}
static float k_float(const OpSpec* s, float kappa, int64_t dim) {
  const float u = static_cast<float>(s->u);
  if (s->kform == 0) {
    const int r = 2 * static_cast<int>(dim) + 4;
    const float gamma_r = static_cast<float>(r) * u;
    return kappa * gamma_r;
  }
  if (s->kform == 1) {
    const float gamma_n = static_cast<float>(static_cast<int>(dim)) * u;
    return (kappa * 2.f) * gamma_n;
  }
  return 0.f;
}

// K at or above which the cancellation test flags every pair with norms in the safe
// range (run_distance, the all-flagged route)
constexpr float kAllFlaggedK = 2.5f;

// the points' low-precision copy (n x ldlow) followed by their norms (fp32[n]), as
// euc_prepare_points writes them
static size_t prepared_plow_bytes(const OpSpec* s, int64_t n, int64_t dim) {
  const int es = low_esize(s);
  const int per_box = 128 / es;
  const int64_t ld = ((dim + per_box - 1) / per_box) * per_box;
  return al(static_cast<size_t>(n) * static_cast<size_t>(ld) * es);
}

struct RunOut {
  int mode = 0;                      // argmin mode: 0 screen, 1 exact epilogue, 2 certified
  const void* prep = nullptr;        // argmin: prepared points (euc_prepare_points)
  void* D = nullptr;                 // D mode
  int64_t* labels = nullptr;         // argmin mode
  int32_t* labels32 = nullptr;
  void* min_dist = nullptr;
  uint64_t* d_count = nullptr;
  int32_t* tile_counts = nullptr;
  int tile_T = 0;
};

// certified argmin whose bounds fail: at most this many centers take the dense sweep
constexpr int64_t kDenseArgminMaxM = 512;

static int run_distance(const OpSpec* s, const void* P, const void* C, int64_t n, int64_t m, int64_t dim,
                        float kappa, const RunOut& o, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (n < 0 || m < 0 || dim < 0) return fail(EUC_ERR_SHAPE, "negative size");
  if (dim > (1 << 20) || m > 0xffffffffll || n > 0xffffffffll)
    return fail(EUC_ERR_SHAPE, "shape too large");
  const bool argmin = (o.D == nullptr);
  if (!device_is_sm100()) return fail(EUC_ERR_DEVICE, "euclid_b200 requires an sm_100 (B200) device");
  if (n == 0 || m == 0) {
    if (o.d_count) cudaMemsetAsync(o.d_count, 0, 8, st);
    return ok();
  }
  if (!P || !C) return fail(EUC_ERR_ARG, "null input pointer");
  if (dim == 0) return fail(EUC_ERR_SHAPE, "dim must be >= 1");
  if (s->gemm == G_DIRECT) {
    if (argmin) return fail(EUC_ERR_UNSUPPORTED, "direct operators have no fused argmin");
    cudaError_t e = launch_direct(s, P, C, n, m, static_cast<int>(dim), o.D, st);
    return e == cudaSuccess ? ok() : cuda_fail(e, s->name);
  }
  const bool cert_capable = is_tc(s) && s->flag != FL_NONE && s->in == IN_F32 && (s->rec == RC_F32 || s->rec == RC_F64);
  bool cert = argmin && o.mode == 2;
  if (cert && !cert_capable)
    return fail(EUC_ERR_UNSUPPORTED,
                std::string(s->name) + ": no certified argmin (tensor-core operators with an fp32 or fp64 recompute)");
  const bool prepared = o.prep != nullptr;
  if (prepared && (!argmin || !is_tc(s) || s->in != IN_F32 || s->form != FM_F32 || o.mode == 2))
    return fail(EUC_ERR_UNSUPPORTED, std::string(s->name) +
                                         ": prepared points serve the tensor-core screen and exact argmin only");
  const Layout L = layout_for(s, n, m, dim, argmin, prepared);
  if (!ws || ws_bytes < L.total)
    return fail(EUC_ERR_WORKSPACE, std::string(s->name) + ": workspace of " + std::to_string(L.total) +
                                       " bytes required, got " + std::to_string(ws_bytes));
  uint8_t* w = static_cast<uint8_t*>(ws);
  // All-flagged route.  With K >= kAllFlaggedK the cancellation test flags every pair
  // whose norms lie in a safe range, and the reference's D is then the direct recompute
  // of every pair: its argmin (first index of the smallest stored value) is exactly what
  // the certified argmin computes, recomputing only the centers that can win, and the
  // flagged count is n * m.  Proof of "every pair": with e the low format's unit
  // roundoff (at most 2^-8), the rounded operands give |s| <= |p~||c~| (1 + d 2^-23)
  // (1 + e) <= (pp + cc) / 2 (1 + 2 d 2^-23 + 2e + ...) because pp and cc are the rounded
  // squared norms of the same operands, so d_exp = fl(fl(pp - 2s) + cc) <=
  // (pp + cc)(2 + 2 d 2^-23 + 2^-7 + 2^-22) < 2.5 (pp + cc) <= fl(K (pp + cc)) for
  // dim <= 2^20.  The range excludes what this bound does not cover: non-finite values
  // (NaN rows are never flagged), sums below 2^-13 (the absolute error of subnormal
  // fp16 S and norms, 2^-25, stays under 2^-12 of pp + cc), and for the operators that
  // round S or the norms to fp16, sums above 6.0e4 (fp16 overflows at 65520).  The
  // range test reads P and C once and costs one stream synchronisation; a call that
  // fails it takes the exact path below.
  bool all_flagged = false;
  if (argmin && !prepared && o.mode != 2 && cert_capable && k_float(s, kappa, dim) >= kAllFlaggedK) {
    Phase ph("euc:range_check");
    int* dflag = reinterpret_cast<int*>(w + L.hdr + 40);
    const bool f16 = s->sround == SR_F16 || s->norm == NM_LOW_F16;
    const float lo = 0x1p-13f, hi = f16 ? 6.0e4f : 1.0e37f;
    int bad = 1;
    cudaError_t e = cudaMemsetAsync(dflag, 0, sizeof(int), st);
    if (e == cudaSuccess) e = launch_norm_range_check(static_cast<const float*>(P), n, static_cast<int>(dim), lo, hi,
                                                      dflag, st);
    if (e == cudaSuccess) e = launch_norm_range_check(static_cast<const float*>(C), m, static_cast<int>(dim), lo, hi,
                                                      dflag, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&bad, dflag, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "range check");
    if (bad == 0) all_flagged = cert = true;
  }
  DistJob j{};
  j.spec = s;
  j.P = P;
  j.C = C;
  j.n = n;
  j.m = m;
  j.dim = static_cast<int>(dim);
  j.kf = k_float(s, kappa, dim);
  j.kd = k_double(s, kappa, dim);
  j.D = o.D;
  j.count = o.d_count ? reinterpret_cast<unsigned long long*>(o.d_count)
                      : reinterpret_cast<unsigned long long*>(w + L.hdr);
  j.list = s->flag != FL_NONE ? reinterpret_cast<unsigned long long*>(w + L.list) : nullptr;
  j.list_cap = L.cap;
  j.tile_counts = o.tile_counts;
  j.tile_T = o.tile_T;
  j.tiles_j = o.tile_T > 0 ? (m + o.tile_T - 1) / o.tile_T : 0;
  j.pp = w + L.pp;
  j.cc = w + L.cc;
  j.Plow = is_tc(s) ? w + L.plow : nullptr;
  if (prepared) {
    j.Plow = const_cast<void*>(o.prep);
    j.pp = static_cast<uint8_t*>(const_cast<void*>(o.prep)) + prepared_plow_bytes(s, n, dim);
  }
  j.Clow = is_tc(s) ? w + L.clow : nullptr;
  j.ldlow = L.ldlow;
  // the screen bounds flagged pairs through 1 - K > 0
  j.fast_argmin = argmin && is_tc(s) && s->flag != FL_NONE && ((o.mode == 0 && j.kf < 1.f) || cert);
  j.cert = cert;
  j.Clow_sorted = L.clow_s ? w + L.clow_s : nullptr;
  j.cc_sorted = L.cc_s ? reinterpret_cast<float*>(w + L.cc_s) : nullptr;
  j.perm = L.perm ? reinterpret_cast<int*>(w + L.perm) : nullptr;
  j.row_key = (argmin && L.key) ? reinterpret_cast<unsigned long long*>(w + L.key) : nullptr;
  j.row_val64 = (argmin && L.val64) ? reinterpret_cast<double*>(w + L.val64) : nullptr;
  j.row_idx64 = (argmin && L.idx64) ? reinterpret_cast<long long*>(w + L.idx64) : nullptr;
  j.chunk_list = L.clist ? reinterpret_cast<unsigned long long*>(w + L.clist) : nullptr;
  j.chunk_s = L.cs ? reinterpret_cast<float*>(w + L.cs) : nullptr;
  j.chunk_cap = L.ccap;
  j.regions = j.fast_argmin ? tc_fast_job_regions(j) : 0;
  j.b_aux_sorted = L.baux ? w + L.baux : nullptr;
  j.aux_e = reinterpret_cast<int*>(w + L.hdr + 16);
  j.ccmax = reinterpret_cast<float*>(w + L.hdr + 20);
  const int64_t n_rt = (n + 127) / 128;
  if (cert) {
    // the accumulator region of the candidate chunks (ccap >= n entries of 128 bytes) is
    // unused: [4][n] keys, [4][n] second distances, per row the second screen's threshold
    // and the list of rows evaluated whole, per 128-row tile its switch (56 n + n / 128
    // bytes); the second screen lists its groups in the entry region
    uint8_t* c = w + L.cs;
    j.cert_key = reinterpret_cast<unsigned long long*>(c);
    j.cert_d2 = reinterpret_cast<float*>(c + static_cast<size_t>(n) * 32);
    j.cert_thr = reinterpret_cast<float*>(c + static_cast<size_t>(n) * 48);
    j.cert_rows = reinterpret_cast<uint32_t*>(c + static_cast<size_t>(n) * 52);
    j.cert_tiles = c + static_cast<size_t>(n) * 56;
    // by group, where the region has room: 4 n entries and their sorted rows, and three
    // tables of ng + 1 counters (ng <= 16384: the block histograms fit shared memory);
    // then, for the second screen over the undecided rows alone, their list, norms,
    // thresholds and redo bytes (13 n)
    const size_t nb = static_cast<size_t>(n);
    const size_t cs_bytes = al(L.ccap * 128);
    const int64_t ng = (m + 7) / 8;
    const size_t b0 = (nb * 56 + static_cast<size_t>(n_rt) + 15) & ~size_t(15);
    const size_t need = b0 + nb * 48 + 12 * static_cast<size_t>(ng + 1);
    j.cert_ng = (ng <= 16384 && 4 * nb <= 0xffffffffull && need <= cs_bytes) ? static_cast<int>(ng) : 0;
    if (j.cert_ng > 0) {
      j.cert_ent = reinterpret_cast<unsigned long long*>(c + b0);
      j.cert_ent_cap = static_cast<unsigned int>(4 * nb);
      j.cert_srow = reinterpret_cast<uint32_t*>(c + b0 + nb * 32);
      j.cert_gcnt = reinterpret_cast<unsigned int*>(c + b0 + nb * 48);
      j.cert_goff = j.cert_gcnt + (ng + 1);
      j.cert_ent_n = reinterpret_cast<unsigned int*>(w + L.hdr + 28);
      const size_t g0 = (need + 15) & ~size_t(15);
      if (g0 + nb * 13 <= cs_bytes) {
        j.cert_F = reinterpret_cast<uint32_t*>(c + g0);
        j.cert_pg = reinterpret_cast<float*>(c + g0 + nb * 4);
        j.cert_thr_g = reinterpret_cast<float*>(c + g0 + nb * 8);
        j.cert_redo_g = c + g0 + nb * 12;
        j.cert_nF = reinterpret_cast<unsigned int*>(w + L.hdr + 32);
      }
    }
    j.cert_nrows = reinterpret_cast<unsigned int*>(w + L.hdr + 24);
    // the flagged-pair list is unused too: the second screen lists its groups in the
    // larger of the two entry regions
    if (L.cap > L.ccap) {
      j.chunk_list = reinterpret_cast<unsigned long long*>(w + L.list);
      j.chunk_cap = L.cap;
    }
  }
  j.region_cnt = L.rcnt ? reinterpret_cast<uint32_t*>(w + L.rcnt) : nullptr;
  j.redo = L.redo ? w + L.redo : nullptr;
  j.stream = st;
  if (j.fast_argmin && j.regions > kMaxRegions) return fail(EUC_ERR_UNSUPPORTED, "more SMs than list regions");
  // the screening kernel prepares the points itself where it can (no low-precision copy)
  j.fused_rows = j.fast_argmin && !prepared && tc_fast_can_fuse_rows(j);
  // certified, points read by the screen itself: the second screen runs on a gathered
  // low-precision copy of the undecided rows (the copy region is free)
  j.cert_gather = cert && j.cert_ng > 0 && j.fused_rows && j.cert_F != nullptr && j.Plow != nullptr;

  cudaError_t e = cudaMemsetAsync(j.count, 0, 8, st);
  if (e == cudaSuccess && o.tile_counts) {
    const int64_t nt = ((n + o.tile_T - 1) / o.tile_T) * j.tiles_j;
    e = cudaMemsetAsync(o.tile_counts, 0, static_cast<size_t>(nt) * 4, st);
  }
  if (e == cudaSuccess && cert) e = cudaMemsetAsync(j.cert_nrows, 0, 4, st);
  if (e == cudaSuccess && cert) e = cudaMemsetAsync(j.cert_tiles, 0, static_cast<size_t>(n_rt), st);
  if (e == cudaSuccess && j.cert_gather) e = cudaMemsetAsync(j.cert_nF, 0, 4, st);
  if (e == cudaSuccess && cert && j.cert_ng > 0) {
    e = cudaMemsetAsync(j.cert_ent_n, 0, 4, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(j.cert_gcnt, 0, static_cast<size_t>(j.cert_ng) * 4, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "memset");
  if (!argmin && !is_tc(s) && thin_d_ok(s, m, j.dim, o.D)) {
    // D of a small dim: the centers' norms, then one kernel that forms, tests, recomputes
    // the flagged pairs in place and stores (the rows' norms are formed in it)
    e = launch_prep(j, false, false);
    if (e == cudaSuccess) e = launch_thin_d(s, P, C, j.cc, n, m, j.dim, j.kf, o.D, j.count, st);
    return e == cudaSuccess ? ok() : cuda_fail(e, s->name);
  }
  {
    Phase ph("euc:prep");
    if (!j.fused_rows && !prepared) e = launch_prep(j, true, is_tc(s));
    if (e == cudaSuccess) e = launch_prep(j, false, is_tc(s));
    if (e == cudaSuccess && j.fast_argmin) e = launch_sort_centers(j);
  }
  if (e != cudaSuccess) return cuda_fail(e, "prep");
  {
    Phase ph(j.fast_argmin ? "euc:screen" : "euc:distance");
    e = j.fast_argmin ? launch_tc_fast(j, cert ? 1 : 0) : (is_tc(s) ? launch_tc(j) : launch_simt(j));
  }
  if (e != cudaSuccess) return cuda_fail(e, s->name);
  if (cert) {
    Phase ph("euc:certified");
    // rows the first screen decides; a second screen lists the candidate groups of the
    // others; their direct distances, and the rows evaluated whole
    float* md = static_cast<float*>(o.min_dist);
    e = launch_cert_rows(j, o.labels, o.labels32, md);
    // few centers: when the first screen's bounds decide fewer than half of the rows
    // (norms far larger than the distances, as in C3's offset points), the rest would go
    // through a second screen and every group; one dense sweep of all pairs, minimum of
    // the same keys, gives the same labels and distances sooner (C3, 2^22 x 256 x 64
    // bf16_fp64: 68.0 ms certified).  It rewrites every row's outputs; the count is the
    // n m direct distances it takes (the all-flagged route's count too).
    if (e == cudaSuccess && m <= kDenseArgminMaxM && j.cert_ng > 0 && j.cert_ent_n) {
      unsigned int decided = 0;
      e = cudaMemcpyAsync(&decided, j.cert_ent_n, sizeof(decided), cudaMemcpyDeviceToHost, st);
      if (e == cudaSuccess) e = cudaStreamSynchronize(st);
      if (e == cudaSuccess && 2 * static_cast<int64_t>(decided) < n) {
        Phase ph2("euc:dense_argmin");
        e = launch_dense_argmin(s, P, C, n, m, static_cast<int>(dim), o.labels, o.labels32, md, st);
        if (e == cudaSuccess)
          e = launch_fill_u64(j.count, 1, static_cast<unsigned long long>(n) * static_cast<unsigned long long>(m), st);
        return e == cudaSuccess ? ok() : cuda_fail(e, "dense argmin");
      }
    }
    if (e == cudaSuccess && j.cert_gather) {
      // the undecided rows gathered into whole row tiles of a low-precision copy, with
      // their norms, thresholds and redo bytes; the second screen reads that copy
      e = launch_cert_compact(j);
      DistJob j2 = j;
      j2.fused_rows = false;
      j2.pp = j.cert_pg;
      j2.redo = j.cert_redo_g;
      j2.cert_thr = j.cert_thr_g;
      if (e == cudaSuccess) e = launch_tc_fast(j2, 2);
    } else if (e == cudaSuccess) {
      e = launch_tc_fast(j, 2);
    }
    if (e == cudaSuccess) e = launch_cert_finish(j, o.labels, o.labels32, md);
    // all-flagged route: the count is that of the reference's list, every pair
    if (e == cudaSuccess && all_flagged)
      e = launch_fill_u64(j.count, 1, static_cast<unsigned long long>(n) * static_cast<unsigned long long>(m), st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "certified rows");
  }
  if (j.fast_argmin) {
    Phase ph("euc:eval_chunks");
    e = launch_eval_chunks(j);
  }
  if (e == cudaSuccess) {
    Phase ph("euc:recompute");
    e = launch_recompute(j);
  }
  if (e == cudaSuccess && j.fast_argmin) {
    Phase ph("euc:redo_rows");
    e = launch_redo_rows(j, o.labels, o.labels32, static_cast<float*>(o.min_dist));
  }
  if (e != cudaSuccess) return cuda_fail(e, "recompute");
  if (argmin && !j.fast_argmin) {  // the fast path's redo pass has written the outputs
    if (j.row_key) {
      e = launch_keys_to_labels(j.row_key, n, o.labels, o.labels32, static_cast<float*>(o.min_dist), st);
    } else {
      e = launch_f64_to_labels(j.row_idx64, n, o.labels, o.labels32, st);
      if (e == cudaSuccess && o.min_dist)
        e = cudaMemcpyAsync(o.min_dist, j.row_val64, static_cast<size_t>(n) * 8, cudaMemcpyDeviceToDevice, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "labels");
  }
  return ok();
}

static int run_named(int op, const void* P, const void* C, int64_t n, int64_t m, int64_t dim, float kappa,
                     const RunOut& o, void* ws, size_t ws_bytes, void* stream) {
  const OpSpec* s = find_op(op);
  if (!s) return fail(EUC_ERR_ARG, "unknown operator id");
  if (!o.D && n > 0 && m > 0) return fail(EUC_ERR_ARG, std::string(s->name) + ": null output D");
  if (!o.D) return EUC_OK;  // empty output
  return run_distance(s, P, C, n, m, dim, kappa, o, ws, ws_bytes, static_cast<cudaStream_t>(stream));
}

}  // namespace euc

using namespace euc;

// ==================================================================== C ABI
extern "C" {

const char* euc_version(void) { return "euclid_b200 0.1 (sm_100a)"; }

const char* euc_status_string(int s) {
  switch (s) {
    case EUC_OK: return "ok";
    case EUC_ERR_SHAPE: return "bad shape";
    case EUC_ERR_DTYPE: return "bad dtype";
    case EUC_ERR_UNSUPPORTED: return "unsupported argument";
    case EUC_ERR_LAUNCH: return "CUDA launch error";
    case EUC_ERR_TIMEOUT: return "device wait timed out";
    case EUC_ERR_WORKSPACE: return "workspace too small";
    case EUC_ERR_ARG: return "invalid argument";
    case EUC_ERR_DEVICE: return "unsupported device";
  }
  return "unknown status";
}

const char* euc_last_error(void) { return g_err.c_str(); }

int euc_device_check(void) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "device_check");
  const int v = device_error_and_clear();
  if (v != 0) return fail(EUC_ERR_TIMEOUT, "a bounded device wait expired (code " + std::to_string(v) + ")");
  return EUC_OK;
}

size_t euc_workspace_bytes(int op, int64_t n, int64_t m, int64_t dim) {
  if (op == EUC_OP_CENTERS_FP32 || op == EUC_OP_CENTERS_FP64)
    return al(static_cast<size_t>(m) * (dim + 1) * 8) + center_ws_bytes(n, dim, m);
  const OpSpec* s = find_op(op);
  if (!s) return 0;
  if (s->gemm == G_DIRECT) return 0;
  return layout_for(s, n, m, dim, false).total;
}

size_t euc_argmin_workspace_bytes(int op, int64_t n, int64_t m, int64_t dim) {
  const OpSpec* s = find_op(op);
  if (!s || s->gemm == G_DIRECT) return 0;
  return layout_for(s, n, m, dim, true).total;
}

void euc_set_kernel_timing(int enable) { g_timing = enable != 0; }

void euc_set_wait_limit_ns(uint64_t ns) { g_wait_ns.store(ns ? ns : kWaitLimitNs); }

void euc_test_withhold_arrival(void) { g_withhold.store(1); }

float euc_last_kernel_ms(void) {
  if (!g_ev_recorded) return -1.f;
  float ms = -1.f;
  if (cudaEventSynchronize(g_ev1) != cudaSuccess) return -1.f;
  cudaEventElapsedTime(&ms, g_ev0, g_ev1);
  return ms;
}

const char* euc_last_kernel_name(void) { return g_ev_name; }

int euc_pairwise_single(const float* P, const float* C, int64_t n, int64_t m, int64_t dim, float* D, void* ws,
                        size_t ws_bytes, void* stream) {
  RunOut o;
  o.D = D;
  return run_named(EUC_OP_SINGLE, P, C, n, m, dim, 0.f, o, ws, ws_bytes, stream);
}
int euc_pairwise_double(const double* P, const double* C, int64_t n, int64_t m, int64_t dim, double* D, void* ws,
                        size_t ws_bytes, void* stream) {
  RunOut o;
  o.D = D;
  return run_named(EUC_OP_DOUBLE, P, C, n, m, dim, 0.f, o, ws, ws_bytes, stream);
}

#define EUC_MIX_DEF(fname, OPID)                                                                        \
  int fname(const float* P, const float* C, int64_t n, int64_t m, int64_t dim, float kappa, float* D,   \
            uint64_t* d_count, void* ws, size_t ws_bytes, void* stream) {                               \
    RunOut o;                                                                                            \
    o.D = D;                                                                                             \
    o.d_count = d_count;                                                                                 \
    return run_named(OPID, P, C, n, m, dim, kappa, o, ws, ws_bytes, stream);                             \
  }
EUC_MIX_DEF(euc_mix_fp16_fp64, EUC_OP_MIX_FP16_FP64)
EUC_MIX_DEF(euc_mix_bf16_fp64, EUC_OP_MIX_BF16_FP64)
EUC_MIX_DEF(euc_mix_tf32_fp64, EUC_OP_MIX_TF32_FP64)
EUC_MIX_DEF(euc_mix_fp32_fp64, EUC_OP_MIX_FP32_FP64)
EUC_MIX_DEF(euc_mix_fp16_fp16, EUC_OP_MIX_FP16_FP16)
EUC_MIX_DEF(euc_mix_fp16_fp32, EUC_OP_MIX_FP16_FP32)
EUC_MIX_DEF(euc_mix_bf16_bf16, EUC_OP_MIX_BF16_BF16)
EUC_MIX_DEF(euc_mix_bf16_fp32, EUC_OP_MIX_BF16_FP32)
EUC_MIX_DEF(euc_mix_fp32_fp32, EUC_OP_MIX_FP32_FP32)
#undef EUC_MIX_DEF

// tile_size rules of euclidean_kernels_tiled.cu:331-336
static int tiled_tile(int tile_size, int64_t dim, int* T) {
  if (tile_size <= 0) tile_size = dim <= 128 ? 32 : 16;
  if (tile_size != 16 && tile_size != 32) return fail(EUC_ERR_UNSUPPORTED, "Supported tile_size: 16 or 32");
  if (dim > 512) return fail(EUC_ERR_UNSUPPORTED, "D too large for full caching (max 512)");
  *T = tile_size;
  return EUC_OK;
}

#define EUC_TILED_DEF(fname, OPID)                                                                          \
  int fname(const float* P, const float* C, int64_t n, int64_t m, int64_t dim, float kappa, int tile_size,  \
            float* D, int32_t* d_tile_counts, uint64_t* d_count, void* ws, size_t ws_bytes, void* stream) { \
    int T = 0;                                                                                               \
    int rc = tiled_tile(tile_size, dim, &T);                                                                 \
    if (rc != EUC_OK) return rc;                                                                             \
    RunOut o;                                                                                                \
    o.D = D;                                                                                                 \
    o.d_count = d_count;                                                                                     \
    o.tile_counts = d_tile_counts;                                                                           \
    o.tile_T = T;                                                                                            \
    return run_named(OPID, P, C, n, m, dim, kappa, o, ws, ws_bytes, stream);                                 \
  }
EUC_TILED_DEF(euc_tiled_fp16_fp64, EUC_OP_TILED_FP16_FP64)
EUC_TILED_DEF(euc_tiled_fp16_fp32, EUC_OP_TILED_FP16_FP32)
EUC_TILED_DEF(euc_tiled_bf16_fp64, EUC_OP_TILED_BF16_FP64)
EUC_TILED_DEF(euc_tiled_bf16_fp32, EUC_OP_TILED_BF16_FP32)
EUC_TILED_DEF(euc_tiled_fp32_fp64, EUC_OP_TILED_FP32_FP64)
EUC_TILED_DEF(euc_tiled_fp32_fp32, EUC_OP_TILED_FP32_FP32)
#undef EUC_TILED_DEF

// tile_size / dim rules of euclidean_kernels_tiled_tc.cu:246-248
#define EUC_TC_DEF(fname, OPID)                                                                             \
  int fname(const float* P, const float* C, int64_t n, int64_t m, int64_t dim, float kappa, int tile_size,  \
            float* D, uint64_t* d_count, void* ws, size_t ws_bytes, void* stream) {                         \
    if (tile_size <= 0) tile_size = 32;                                                                      \
    if (tile_size != 32) return fail(EUC_ERR_UNSUPPORTED, "This fixed kernel supports tile_size=32 only");   \
    if (dim % 16 != 0)                                                                                       \
      return fail(EUC_ERR_UNSUPPORTED, "For WMMA path, D must be multiple of 16 (pad input if needed)");     \
    RunOut o;                                                                                                \
    o.D = D;                                                                                                 \
    o.d_count = d_count;                                                                                     \
    return run_named(OPID, P, C, n, m, dim, kappa, o, ws, ws_bytes, stream);                                 \
  }
EUC_TC_DEF(euc_tensorcore_fp16_fp64, EUC_OP_TC_FP16_FP64)
EUC_TC_DEF(euc_tensorcore_fp16_fp32, EUC_OP_TC_FP16_FP32)
EUC_TC_DEF(euc_tensorcore_bf16_fp64, EUC_OP_TC_BF16_FP64)
EUC_TC_DEF(euc_tensorcore_bf16_fp32, EUC_OP_TC_BF16_FP32)
#undef EUC_TC_DEF

int euc_uniform_fp16(const uint16_t* P, const uint16_t* C, int64_t n, int64_t m, int64_t dim, uint16_t* D, void* ws,
                     size_t ws_bytes, void* stream) {
  RunOut o;
  o.D = D;
  return run_named(EUC_OP_UNI_FP16, P, C, n, m, dim, 0.f, o, ws, ws_bytes, stream);
}
int euc_uniform_bf16(const uint16_t* P, const uint16_t* C, int64_t n, int64_t m, int64_t dim, uint16_t* D, void* ws,
                     size_t ws_bytes, void* stream) {
  RunOut o;
  o.D = D;
  return run_named(EUC_OP_UNI_BF16, P, C, n, m, dim, 0.f, o, ws, ws_bytes, stream);
}
int euc_uniform_tf32(const float* P, const float* C, int64_t n, int64_t m, int64_t dim, float* D, void* ws,
                     size_t ws_bytes, void* stream) {
  RunOut o;
  o.D = D;
  return run_named(EUC_OP_UNI_TF32, P, C, n, m, dim, 0.f, o, ws, ws_bytes, stream);
}

#define EUC_DIRECT_DEF(fname, OPID, T)                                                                  \
  int fname(const T* P, const T* C, int64_t n, int64_t m, int64_t dim, T* D, void* stream) {            \
    RunOut o;                                                                                            \
    o.D = D;                                                                                             \
    return run_named(OPID, P, C, n, m, dim, 0.f, o, nullptr, 0, stream);                                 \
  }
EUC_DIRECT_DEF(euc_uniform_fp16_direct, EUC_OP_UNI_FP16_DIRECT, uint16_t)
EUC_DIRECT_DEF(euc_uniform_bf16_direct, EUC_OP_UNI_BF16_DIRECT, uint16_t)
EUC_DIRECT_DEF(euc_uniform_tf32_direct, EUC_OP_UNI_TF32_DIRECT, float)
EUC_DIRECT_DEF(euc_uniform_fp32_direct, EUC_OP_UNI_FP32_DIRECT, float)
EUC_DIRECT_DEF(euc_uniform_fp64_direct, EUC_OP_UNI_FP64_DIRECT, double)
#undef EUC_DIRECT_DEF

int euc_advanced_fp64_fp16(const uint16_t* P, const uint16_t* C, int64_t n, int64_t m, int64_t dim, float kappa,
                           float* D, uint64_t* d_count, void* ws, size_t ws_bytes, void* stream) {
  RunOut o;
  o.D = D;
  o.d_count = d_count;
  return run_named(EUC_OP_ADV_FP64_FP16, P, C, n, m, dim, kappa, o, ws, ws_bytes, stream);
}
int euc_advanced_fp64_bf16(const uint16_t* P, const uint16_t* C, int64_t n, int64_t m, int64_t dim, float kappa,
                           float* D, uint64_t* d_count, void* ws, size_t ws_bytes, void* stream) {
  RunOut o;
  o.D = D;
  o.d_count = d_count;
  return run_named(EUC_OP_ADV_FP64_BF16, P, C, n, m, dim, kappa, o, ws, ws_bytes, stream);
}
int euc_advanced_fp64_tf32(const float* P, const float* C, int64_t n, int64_t m, int64_t dim, float kappa,
                           double* D, uint64_t* d_count, void* ws, size_t ws_bytes, void* stream) {
  RunOut o;
  o.D = D;
  o.d_count = d_count;
  return run_named(EUC_OP_ADV_FP64_TF32, P, C, n, m, dim, kappa, o, ws, ws_bytes, stream);
}
int euc_advanced_fp64_fp32_gemm(const double* P, const double* C, int64_t n, int64_t m, int64_t dim, float kappa,
                                double* D, uint64_t* d_count, void* ws, size_t ws_bytes, void* stream) {
  RunOut o;
  o.D = D;
  o.d_count = d_count;
  return run_named(EUC_OP_ADV_FP64_FP32_GEMM, P, C, n, m, dim, kappa, o, ws, ws_bytes, stream);
}

int euc_read_count_i32(const int32_t* d_counter, int32_t* host_out) {
  if (!d_counter || !host_out) return fail(EUC_ERR_ARG, "null pointer");
  cudaError_t e = cudaMemcpy(host_out, d_counter, sizeof(int32_t), cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? EUC_OK : cuda_fail(e, "read_count");
}
int euc_read_count_u64(const uint64_t* d_counter, uint64_t* host_out) {
  if (!d_counter || !host_out) return fail(EUC_ERR_ARG, "null pointer");
  cudaError_t e = cudaMemcpy(host_out, d_counter, sizeof(uint64_t), cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? EUC_OK : cuda_fail(e, "read_count");
}

// ------------------------------------------------------------------ centers
static int centers_impl(const void* X, bool f64, const int64_t* labels, int64_t n, int64_t dim, int64_t k,
                        void* centers, int64_t* d_counts, void* ws, size_t ws_bytes, void* stream) {
  if (n < 0 || dim < 0 || k < 0) return fail(EUC_ERR_SHAPE, "negative size");
  if (k == 0 || dim == 0) return EUC_OK;
  if (dim > 1024) return fail(EUC_ERR_UNSUPPORTED, "dim > 1024 not supported by the center update");
  if (k > 0x7fffffffll) return fail(EUC_ERR_SHAPE, "too many clusters");
  if (!device_is_sm100()) return fail(EUC_ERR_DEVICE, "euclid_b200 requires an sm_100 (B200) device");
  if (!centers || (n > 0 && (!X || !labels))) return fail(EUC_ERR_ARG, "null pointer");
  const size_t stats_b = al(static_cast<size_t>(k) * (dim + 1) * 8);
  const size_t need = stats_b + center_ws_bytes(n, dim, k);
  if (!ws || ws_bytes < need)
    return fail(EUC_ERR_WORKSPACE, "update_centers: workspace of " + std::to_string(need) + " bytes required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  double* stats = static_cast<double*>(ws);
  cudaError_t e = launch_center_stats(X, f64, labels, true, n, dim, k, stats, static_cast<uint8_t*>(ws) + stats_b,
                                      ws_bytes - stats_b, st);
  if (e == cudaSuccess) e = launch_center_finalize(stats, dim, k, centers, f64, nullptr, 0, st);
  if (e == cudaSuccess && d_counts) {
    // counts column -> int64 (strided copy: one element per (dim+1)-wide row)
    e = cudaMemcpy2DAsync(d_counts, sizeof(int64_t), stats + dim, (dim + 1) * sizeof(double), sizeof(double), k,
                          cudaMemcpyDeviceToDevice, st);
  }
  return e == cudaSuccess ? EUC_OK : cuda_fail(e, "update_centers");
}

int euc_update_centers_fp32(const float* X, const int64_t* labels, int64_t n, int64_t dim, int64_t k, float* centers,
                            int64_t* d_counts, void* ws, size_t ws_bytes, void* stream) {
  return centers_impl(X, false, labels, n, dim, k, centers, d_counts, ws, ws_bytes, stream);
}
int euc_update_centers_fp64(const double* X, const int64_t* labels, int64_t n, int64_t dim, int64_t k,
                            double* centers, int64_t* d_counts, void* ws, size_t ws_bytes, void* stream) {
  return centers_impl(X, true, labels, n, dim, k, centers, d_counts, ws, ws_bytes, stream);
}

size_t euc_center_stats_workspace_bytes(int64_t n, int64_t dim, int64_t k) { return center_ws_bytes(n, dim, k); }

int euc_center_stats(const void* X, int x_is_f64, const void* labels, int labels_are_i64, int64_t n, int64_t dim,
                     int64_t k, double* stats, void* ws, size_t ws_bytes, void* stream) {
  if (n < 0 || dim <= 0 || k <= 0) return fail(EUC_ERR_SHAPE, "bad size");
  if (dim > 1024) return fail(EUC_ERR_UNSUPPORTED, "dim > 1024 not supported by the center update");
  if (!stats || (n > 0 && (!X || !labels))) return fail(EUC_ERR_ARG, "null pointer");
  if (!device_is_sm100()) return fail(EUC_ERR_DEVICE, "euclid_b200 requires an sm_100 (B200) device");
  if (ws_bytes < center_ws_bytes(n, dim, k) || !ws)
    return fail(EUC_ERR_WORKSPACE, "center_stats: workspace too small");
  Phase ph("euc:center_stats");
  cudaError_t e = launch_center_stats(X, x_is_f64 != 0, labels, labels_are_i64 != 0, n, dim, k, stats, ws, ws_bytes,
                                      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? EUC_OK : cuda_fail(e, "center_stats");
}

int euc_center_finalize(const double* stats, int64_t dim, int64_t k, void* centers, int centers_are_f64,
                        const void* prev, int empty_policy, void* stream) {
  if (dim <= 0 || k <= 0) return fail(EUC_ERR_SHAPE, "bad size");
  if (!stats || !centers) return fail(EUC_ERR_ARG, "null pointer");
  if (empty_policy == 1 && !prev) return fail(EUC_ERR_ARG, "empty_policy 1 needs prev centers");
  Phase ph("euc:center_finalize");
  cudaError_t e = launch_center_finalize(stats, dim, k, centers, centers_are_f64 != 0, prev, empty_policy,
                                         static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? EUC_OK : cuda_fail(e, "center_finalize");
}

// ------------------------------------------------------------------ seeding
size_t euc_kmeanspp_workspace_bytes(int64_t n, int64_t dim, int64_t k) {
  (void)dim;
  (void)k;
  return n > 0 ? seed_ws_bytes(n) : 0;
}

int euc_kmeanspp(const void* X, int x_is_f64, int64_t n, int64_t dim, int64_t k, uint64_t seed, int64_t* indices,
                 void* centers, void* ws, size_t ws_bytes, void* stream) {
  if (n <= 0 || dim <= 0 || k <= 0 || k > n) return fail(EUC_ERR_SHAPE, "kmeanspp: need 1 <= k <= n and dim >= 1");
  if (dim > (1 << 20) || n > (1ll << 40) || k > 0x7fffffffll) return fail(EUC_ERR_SHAPE, "kmeanspp: shape too large");
  if (!X || !indices) return fail(EUC_ERR_ARG, "null pointer");
  if (!device_is_sm100()) return fail(EUC_ERR_DEVICE, "euclid_b200 requires an sm_100 (B200) device");
  if (!ws || ws_bytes < seed_ws_bytes(n)) return fail(EUC_ERR_WORKSPACE, "kmeanspp: workspace too small");
  cudaError_t e = launch_kmeanspp(X, x_is_f64 != 0, n, dim, k, seed, indices, centers, ws,
                                  static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? EUC_OK : cuda_fail(e, "kmeanspp");
}

// ------------------------------------------------------------------ fused argmin
// ------------------------------------------------------------------ prepared points
size_t euc_prepared_points_bytes(int op, int64_t n, int64_t dim) {
  const OpSpec* s = find_op(op);
  if (!s || !is_tc(s) || n < 0 || dim <= 0) return 0;
  return prepared_plow_bytes(s, n, dim) + al(static_cast<size_t>(n) * 4);
}

int euc_prepare_points(int op, const float* P, int64_t n, int64_t dim, void* prep, size_t prep_bytes, void* stream) {
  const OpSpec* s = find_op(op);
  if (!s) return fail(EUC_ERR_ARG, "unknown operator id");
  if (!is_tc(s) || s->in != IN_F32 || s->form != FM_F32)
    return fail(EUC_ERR_UNSUPPORTED, std::string(s->name) + ": no prepared points (tensor-core operators only)");
  if (n < 0 || dim <= 0) return fail(EUC_ERR_SHAPE, "bad size");
  if (dim > (1 << 20) || n > 0xffffffffll) return fail(EUC_ERR_SHAPE, "shape too large");
  if (!device_is_sm100()) return fail(EUC_ERR_DEVICE, "euclid_b200 requires an sm_100 (B200) device");
  if (n == 0) return ok();
  if (!P || !prep) return fail(EUC_ERR_ARG, "null pointer");
  if (prep_bytes < euc_prepared_points_bytes(op, n, dim))
    return fail(EUC_ERR_WORKSPACE, std::string(s->name) + ": prepared-points buffer too small");
  DistJob j{};
  j.spec = s;
  j.P = P;
  j.n = n;
  j.dim = static_cast<int>(dim);
  j.ldlow = layout_for(s, n, 1, dim, true).ldlow;
  j.Plow = prep;
  j.pp = static_cast<uint8_t*>(prep) + prepared_plow_bytes(s, n, dim);
  j.stream = static_cast<cudaStream_t>(stream);
  Phase ph("euc:prepare_points");
  const cudaError_t e = launch_prep(j, true, true);
  return e == cudaSuccess ? ok() : cuda_fail(e, "prepare_points");
}

size_t euc_argmin_prepared_workspace_bytes(int op, int64_t n, int64_t m, int64_t dim) {
  const OpSpec* s = find_op(op);
  if (!s || !is_tc(s)) return 0;
  return layout_for(s, n, m, dim, true, true).total;
}

int euc_argmin_prepared(int op, const float* P, const void* prep, const float* C, int64_t n, int64_t m, int64_t dim,
                        float kappa, int exact, int64_t* labels, int32_t* labels32, void* min_dist, uint64_t* d_count,
                        void* ws, size_t ws_bytes, void* stream) {
  const OpSpec* s = find_op(op);
  if (!s) return fail(EUC_ERR_ARG, "unknown operator id");
  if (!is_tc(s)) return fail(EUC_ERR_UNSUPPORTED, std::string(s->name) + ": no prepared points (tensor-core operators only)");
  if (exact == EUC_ARGMIN_CERTIFIED)
    return fail(EUC_ERR_UNSUPPORTED, "prepared points serve the screen and the exact argmin, not the certified mode");
  if (n > 0 && m > 0 && !prep) return fail(EUC_ERR_ARG, "null prepared points");
  RunOut o;
  o.mode = exact != 0 ? 1 : 0;
  o.prep = prep;
  o.labels = labels;
  o.labels32 = labels32;
  o.min_dist = min_dist;
  o.d_count = d_count;
  return run_distance(s, P, C, n, m, dim, kappa, o, ws, ws_bytes, static_cast<cudaStream_t>(stream));
}

int euc_argmin(int op, const void* P, const void* C, int64_t n, int64_t m, int64_t dim, float kappa, int exact,
               int64_t* labels, int32_t* labels32, void* min_dist, uint64_t* d_count, void* ws, size_t ws_bytes,
               void* stream) {
  const OpSpec* s = find_op(op);
  if (!s) return fail(EUC_ERR_ARG, "unknown operator id");
  const bool allowed = op == EUC_OP_SINGLE || op == EUC_OP_DOUBLE || (op >= EUC_OP_MIX_FP16_FP64 && op <= EUC_OP_MIX_FP32_FP32) ||
                       (op >= EUC_OP_TILED_FP16_FP64 && op <= EUC_OP_TILED_FP32_FP32) ||
                       (op >= EUC_OP_TC_FP16_FP64 && op <= EUC_OP_TC_BF16_FP32);
  if (!allowed) return fail(EUC_ERR_UNSUPPORTED, std::string(s->name) + ": no fused argmin form");
  if (m > 0xffffffffll) return fail(EUC_ERR_SHAPE, "too many centers");
  RunOut o;
  o.mode = exact == EUC_ARGMIN_CERTIFIED ? 2 : (exact != 0 ? 1 : 0);
  o.labels = labels;
  o.labels32 = labels32;
  o.min_dist = min_dist;
  o.d_count = d_count;
  return run_distance(s, P, C, n, m, dim, kappa, o, ws, ws_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
