// Internal interface of the distance engine: the per-operator numeric recipe
// (which rounding, which GEMM, which cancellation test, which recompute) and the
// launchers of the individual kernels.  The C ABI (api.cu) maps every reference
// entry point onto one OpSpec row and runs it through run_distance().
#pragma once
#include <cuda_runtime.h>
#include <cuda.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>
#include <stddef.h>

namespace euc {

// NVTX range over the host-side enqueue of one phase (a profiler attributes the kernels
// launched inside it to the phase); without an attached tool a push/pop costs a check.
struct Phase {
  explicit Phase(const char* name) { nvtxRangePushA(name); }
  ~Phase() { nvtxRangePop(); }
  Phase(const Phase&) = delete;
  Phase& operator=(const Phase&) = delete;
};

enum InType { IN_F32 = 0, IN_F16 = 1, IN_BF16 = 2, IN_F64 = 3 };
// How S = P.C^T is produced.
enum Gemm {
  G_TC_F16 = 0,    // tcgen05 kind::f16, fp16 operands, fp32 accumulate
  G_TC_BF16 = 1,   // tcgen05 kind::f16, bf16 operands, fp32 accumulate
  G_TC_TF32 = 2,   // tcgen05 kind::tf32, fp32 operands rounded to tf32, fp32 accumulate
  G_SIMT_F32 = 3,  // CUDA-core fp32 FMA, inputs rounded to fp32
  G_SIMT_F64 = 4,  // CUDA-core fp64 FMA, inputs widened to fp64
  G_DIRECT = 5     // no GEMM: direct sum of squared differences
};
// Rounding applied to S before the distance is formed (the reference's cuBLAS
// GEMM writes S in the low precision, euclidean_kernels_mix.cu:538).
enum SRound { SR_NONE = 0, SR_F16 = 1, SR_BF16 = 2 };
enum Norm {
  NM_LOW_F16 = 0,   // fp32 fmaf over fp16-rounded values, result stored as fp16 (mix.cu:106-119)
  NM_LOW_BF16 = 1,  // same for bf16 (mix.cu:122-135)
  NM_F32_FMA = 2,   // fp32 fmaf over fp32 values (euclidean_kernels.cu:16-26)
  NM_F32_SUMSQ = 3, // sum of fp32-rounded squares: (P*P).sum(1) (tiled.cu:338)
  NM_F64_FMA = 4,   // fp64 fma over fp64 values (euclidean_kernels.cu:28-38)
  NM_OPERAND = 5    // fp32 fmaf over the values rounded to the MMA operand type, kept in fp32
                    // (the certified screen's norms: |p~|^2 to fp32 accuracy)
};
enum Form {
  FM_F32 = 0,        // d = max((pp - 2s) + cc, 0) in fp32
  FM_F64 = 1,        // same in fp64
  FM_F64_TO_F32 = 2  // fp64 formula on fp32 norms, result rounded to fp32 (advanced.cu:103-115)
};
enum Flag { FL_NONE = 0, FL_F32 = 1, FL_F64 = 2 };
// Recompute of flagged pairs (the "fallback" kernels).
enum Rec {
  RC_NONE = 0,
  RC_F64 = 1,        // direct formula, fp64 FMA, on the inputs widened to fp64 (mix.cu:156-177)
  RC_F32 = 2,        // direct formula, fp32 FMA on fp32 inputs (mix.cu:481-504)
  RC_F16_ARITH = 3,  // direct formula in fp16 arithmetic on the fp16-rounded inputs (mix.cu:412-439)
  RC_BF16_ARITH = 4  // same in bf16 arithmetic (mix.cu:442-469)
};
enum Out { OUT_F32 = 0, OUT_F16 = 1, OUT_BF16 = 2, OUT_F64 = 3 };

struct OpSpec {
  int op;
  const char* name;
  InType in;
  Gemm gemm;
  SRound sround;
  Norm norm;
  Form form;
  Flag flag;
  Rec rec;
  Out out;
  // Cancellation threshold: eps = K * (pp + cc) with K built exactly as the
  // reference's float expression, either
  //   kform 0: K = kappa * ((float)(2*dim+4) * u)            (mix.cu:207-211, tiled.cu:133,201)
  //   kform 1: K = (kappa * 2) * ((float)dim * u)            (euclidean_kernels.cu:71, mix.cu:930-931)
  //   kform 2: K = ((double)kappa * 2.0) * ((double)dim * u) (advanced.cu:138,353)
  int kform;
  double u;
};

const OpSpec* find_op(int op);

// Distance job: everything the launchers need, resolved from an OpSpec.
struct DistJob {
  const OpSpec* spec;
  const void* P;
  const void* C;
  int64_t n, m;
  int dim;
  float kf;    // flag constant (fp32 forms)
  double kd;   // flag constant (fp64 forms)
  // outputs
  void* D;                       // D mode (null in argmin mode)
  unsigned long long* row_key;   // argmin mode (fp32 distances)
  double* row_val64;             // argmin mode, fp64 distances (no flag ops)
  long long* row_idx64;          // argmin mode, fp64 distances
  unsigned long long* count;     // flagged-pair counter (device)
  unsigned long long* list;      // flagged (i<<32|j) entries
  unsigned long long list_cap;
  int32_t* tile_counts;          // nullable
  int tile_T;
  int64_t tiles_j;
  // workspace-resident intermediates
  void* pp;                      // fp32 or fp64 norms
  void* cc;
  void* Plow;                    // padded low-precision copies (tcgen05 path)
  void* Clow;
  int ldlow;                     // padded row length (elements)
  // fast argmin: centers sorted by norm (stable), their norms and original indices
  bool fast_argmin;
  void* Clow_sorted;
  float* cc_sorted;
  int* perm;
  // fast argmin: candidate chunks, (row << 32 | first sorted column) entries and their
  // 32 fp32 accumulator values, kept in one region of chunk_cap / regions entries per
  // CTA of the screening kernel
  unsigned long long* chunk_list;
  float* chunk_s;
  unsigned long long chunk_cap;
  int regions;
  uint32_t* region_cnt;          // entries per region (written by the screening kernel)
  uint8_t* redo;                 // rows whose candidates did not fit: recomputed whole
  // fast argmin: the MMA also adds (cc_j + Br_i) / 2 to pair (i, j) through one extra
  // K block (32-byte rows, aux.cuh); b_aux holds the sorted centers' rows, the point
  // rows are built in the screening kernel from pp
  void* b_aux_sorted;
  int* aux_e;                    // E (device scalar)
  // fast argmin: the screening kernel reads the fp32 points itself (rounding, norms and
  // the extra-K rows in shared memory) instead of a prepared low-precision copy
  bool fused_rows;
  // certified argmin: the screen keeps, per row and column group of 8 sorted centers, the
  // best and second-best screened distance; every (parity, column half) group of the
  // epilogue writes its partial result ([4][n] keys and second distances); ccmax is the
  // largest finite center norm (device scalar, written by the center sort)
  bool cert;
  unsigned long long* cert_key;
  float* cert_d2;
  float* ccmax;
  float* cert_thr;               // per row: threshold of the second screen (-inf: decided)
  uint8_t* cert_tiles;           // per row tile: whether the second screen visits it
  uint32_t* cert_rows;           // rows evaluated whole
  unsigned int* cert_nrows;
  // direct distances by group of 8 sorted centers (cert_ng groups; 0: row by row)
  int cert_ng;
  unsigned long long* cert_ent;  // (row << 32 | sorted group start) entries
  unsigned int* cert_ent_n;
  unsigned int cert_ent_cap;
  unsigned int* cert_gcnt;
  unsigned int* cert_goff;
  uint32_t* cert_srow;
  // second screen over the undecided rows alone (FUSED points): their list, and per
  // listed row its norm, threshold and redo byte; the low-precision copy goes to Plow
  bool cert_gather;
  uint32_t* cert_F;
  unsigned int* cert_nF;
  float* cert_pg;
  float* cert_thr_g;
  uint8_t* cert_redo_g;
  cudaStream_t stream;
};

// Launchers (return cudaError_t of the launch).
cudaError_t launch_prep(const DistJob& j, bool points, bool make_low);
cudaError_t launch_sort_centers(const DistJob& j);
cudaError_t launch_tc(const DistJob& j);
// fast argmin: screening kernel, exact evaluation of the candidate chunks (flagged pairs
// go to the recompute list), and rows whose candidates did not fit
// cert_pass: 0 the screen of the fast argmin, 1 the certified screen, 2 its second
// screen over the rows the first did not decide
cudaError_t launch_tc_fast(const DistJob& j, int cert_pass = 0);
cudaError_t launch_eval_chunks(const DistJob& j);
// ... and writes every row's outputs from its key (labels, labels32, mind nullable)
cudaError_t launch_redo_rows(const DistJob& j, int64_t* labels, int32_t* labels32, float* mind);
// CTAs (= list regions) of the screening kernel; the fast argmin's screen (not the
// certified passes) runs on CTA pairs where the device can hold them
int tc_fast_regions(int64_t n, bool cert, int kblocks);
bool tc_fast_pairs(bool cert, int kblocks);
int tc_fast_job_regions(const DistJob& j);  // the above for a prepared job (spec, n, ldlow, cert)
bool tc_make_tmap(CUtensorMap* map, const void* base, int64_t rows, int ld, int esize, int box_rows, bool is_f32,
                  bool is_bf16);
bool tc_make_tmap_sw32(CUtensorMap* map, const void* base, int64_t rows, int esize, int box_rows, bool is_f32,
                       bool is_bf16);
// whether the screening kernel can prepare the points itself for this job
bool tc_fast_can_fuse_rows(const DistJob& j);
// certified argmin (k_cert.cu): every row's outputs from the screen's partial results,
// with the direct distances of its candidates (labels, labels32, mind nullable)
cudaError_t launch_cert_rows(const DistJob& j, int64_t* labels, int32_t* labels32, float* mind);
// the undecided rows gathered for the second screen (cert_gather)
cudaError_t launch_cert_compact(const DistJob& j);
// ... and, after the second screen, its listed groups and the rows evaluated whole
cudaError_t launch_cert_finish(const DistJob& j, int64_t* labels, int32_t* labels32, float* mind);
cudaError_t launch_simt(const DistJob& j);
// D of small dim (k_simt.cu): whether thin_d_kernel serves the call, and its launch
bool thin_d_ok(const OpSpec* s, int64_t m, int dim, const void* D);
cudaError_t launch_thin_d(const OpSpec* s, const void* P, const void* C, const void* cc, int64_t n, int64_t m,
                          int dim, float kf, void* D, unsigned long long* count, cudaStream_t st);
cudaError_t launch_direct(const OpSpec* s, const void* P, const void* C, int64_t n, int64_t m, int dim,
                          void* D, cudaStream_t st);
cudaError_t launch_recompute(const DistJob& j);
// every pair flagged, few centers: first-index argmin of the direct distances of all pairs
cudaError_t launch_dense_argmin(const OpSpec* s, const void* P, const void* C, int64_t n, int64_t m, int dim,
                                int64_t* labels, int32_t* labels32, float* md, cudaStream_t st);
cudaError_t launch_keys_to_labels(const unsigned long long* keys, int64_t n, int64_t* labels, int32_t* labels32,
                                  float* mind, cudaStream_t st);
cudaError_t launch_f64_to_labels(const long long* idx, int64_t n, int64_t* labels, int32_t* labels32,
                                 cudaStream_t st);
cudaError_t launch_fill_u64(unsigned long long* p, int64_t n, unsigned long long v, cudaStream_t st);
// *flag |= 1 if some row's fp32 sum of squares is not finite or outside [lo, hi] (k_prep.cu)
cudaError_t launch_norm_range_check(const float* X, int64_t rows, int dim, float lo, float hi, int* flag,
                                    cudaStream_t st);

// Center statistics (k x (dim+1) fp64 rows: sums then count).
size_t center_ws_bytes(int64_t n, int64_t dim, int64_t k);
cudaError_t launch_center_stats(const void* X, bool x_f64, const void* labels, bool labels_i64, int64_t n,
                                int64_t dim, int64_t k, double* stats, void* ws, size_t ws_bytes,
                                cudaStream_t st);
cudaError_t launch_center_finalize(const double* stats, int64_t dim, int64_t k, void* centers, bool f64,
                                   const void* prev, int empty_policy, cudaStream_t st);

// k-means++ seeding (k_seed.cu): indices (int64[k]) and, if non-null, the chosen rows.
size_t seed_ws_bytes(int64_t n);
cudaError_t launch_kmeanspp(const void* X, bool x_f64, int64_t n, int64_t dim, int64_t k, uint64_t seed,
                            int64_t* idx, void* centers, void* ws, cudaStream_t st);

// Bound of the pipeline waits of the tensor-core kernels (api.cu, euc_set_wait_limit_ns),
// and the one-shot failure injection of euc_test_withhold_arrival: true once per arming.
unsigned long long wait_limit_ns();
bool take_withhold();

// Kernel timing hook (api.cu).
void timing_begin(cudaStream_t st, const char* name);
void timing_end(cudaStream_t st);

int num_sms();
bool device_is_sm100();
// records `msg` as the calling thread's euc_last_error() text and returns `status`
int set_error(int status, const char* msg);
int device_error_and_clear();

}  // namespace euc
