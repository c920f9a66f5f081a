/*
 * euclid_b200.h -- C ABI of the B200 (sm_100a) k-means distance engine.
 *
 * Every function takes plain device pointers, element counts and a CUDA stream
 * (passed as void*, NULL = legacy default stream).  No torch types cross this
 * boundary.  Functions are asynchronous on `stream` unless stated otherwise and
 * return an euc_status; euc_last_error() gives a readable message for the last
 * failing call on the calling host thread.
 *
 * Scratch memory: each distance / center entry point takes a caller-owned device
 * workspace (`ws`, `ws_bytes`).  Query the size with euc_workspace_bytes(); a
 * smaller workspace is rejected with EUC_ERR_WORKSPACE.  The library itself
 * never allocates device memory on these paths.
 *
 * Shapes follow the reference: P is n x dim (points, row-major, contiguous),
 * C is m x dim (centers), D is n x m (row-major).  Index arithmetic is 64-bit
 * throughout; unlike the reference there is no N*M <= 2^32 limit.
 *
 * Reference citations are file:line in inEXASCALE/euclid-cuda.
 */
#ifndef EUCLID_B200_H
#define EUCLID_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EUC_API __attribute__((visibility("default")))
#else
#define EUC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
typedef enum {
  EUC_OK = 0,
  EUC_ERR_SHAPE = 1,       /* bad or mismatched sizes (reference: "Dimension mismatch", ...) */
  EUC_ERR_DTYPE = 2,       /* unsupported element type for this entry point                  */
  EUC_ERR_UNSUPPORTED = 3, /* argument value the operator does not support (e.g. tile_size)  */
  EUC_ERR_LAUNCH = 4,      /* CUDA launch / runtime error                                     */
  EUC_ERR_TIMEOUT = 5,     /* a bounded device-side wait expired; the kernel returned early   */
  EUC_ERR_WORKSPACE = 6,   /* workspace missing or smaller than euc_workspace_bytes()         */
  EUC_ERR_ARG = 7,         /* null pointer or invalid argument                                */
  EUC_ERR_DEVICE = 8       /* current device is not sm_100                                    */
} euc_status;

EUC_API const char* euc_version(void);
EUC_API const char* euc_status_string(int status);
/* Message of the last failing call on this host thread ("" if none). */
EUC_API const char* euc_last_error(void);
/* Synchronising check of the device-side error word: returns EUC_ERR_TIMEOUT if a
 * bounded wait inside a kernel expired since the previous check (and clears it),
 * EUC_OK otherwise. */
EUC_API int euc_device_check(void);

/* No counterpart in the reference (it bounds no device wait).  Bound, in nanoseconds,
 * of every pipeline wait of the tensor-core kernels launched after this call (default
 * 2e9; 0 restores it).  A wait that runs out makes the kernel record the error, stop
 * its pipeline, let its copies and MMAs in flight land, free its tensor memory and
 * return; euc_device_check() then reports EUC_ERR_TIMEOUT and the context stays
 * usable.  Process-wide. */
EUC_API void euc_set_wait_limit_ns(uint64_t ns);
/* No counterpart in the reference.  Failure injection for tests, made on the host: the
 * next launch of the screening kernel (euc_argmin's default mode) runs with one
 * arrival withheld (its first CTA's first epilogue warp keeps its first accumulator),
 * so that CTA's MMA warp waits until the wait limit and the launch ends as above.
 * One-shot; the outputs of that call are not meaningful. */
EUC_API void euc_test_withhold_arrival(void);
/* No counterpart in the reference.  Whether the screening kernel of euc_argmin's
 * default mode runs on pairs of SMs (1, the default: clusters of two CTAs, each SM
 * streaming half of every 256-center tile into one M = 256 tensor-core MMA) or on
 * single SMs (0).  Both give the same outputs; process-wide. */
EUC_API void euc_set_screen_pairs(int enable);

/* Operator identifiers, used by euc_workspace_bytes() and the generic entries. */
typedef enum {
  /* euclidean_cuda.cpp:26-32 */
  EUC_OP_SINGLE = 0, EUC_OP_DOUBLE = 1,
  /* euclidean_cuda_mix.cpp:13-83 */
  EUC_OP_MIX_FP16_FP64 = 10, EUC_OP_MIX_BF16_FP64 = 11, EUC_OP_MIX_TF32_FP64 = 12,
  EUC_OP_MIX_FP32_FP64 = 13, EUC_OP_MIX_FP16_FP16 = 14, EUC_OP_MIX_FP16_FP32 = 15,
  EUC_OP_MIX_BF16_BF16 = 16, EUC_OP_MIX_BF16_FP32 = 17, EUC_OP_MIX_FP32_FP32 = 18,
  /* euclidean_cuda_tiled.cpp:12-45 */
  EUC_OP_TILED_FP16_FP64 = 20, EUC_OP_TILED_FP16_FP32 = 21, EUC_OP_TILED_BF16_FP64 = 22,
  EUC_OP_TILED_BF16_FP32 = 23, EUC_OP_TILED_FP32_FP64 = 24, EUC_OP_TILED_FP32_FP32 = 25,
  /* euclidean_cuda_tiled.cpp:51-62 */
  EUC_OP_TC_FP16_FP64 = 30, EUC_OP_TC_FP16_FP32 = 31, EUC_OP_TC_BF16_FP64 = 32,
  EUC_OP_TC_BF16_FP32 = 33,
  /* euclidean_cuda_uniform.cpp:9-40 */
  EUC_OP_UNI_FP16 = 40, EUC_OP_UNI_BF16 = 41, EUC_OP_UNI_TF32 = 42,
  EUC_OP_UNI_FP16_DIRECT = 43, EUC_OP_UNI_BF16_DIRECT = 44, EUC_OP_UNI_TF32_DIRECT = 45,
  EUC_OP_UNI_FP32_DIRECT = 46, EUC_OP_UNI_FP64_DIRECT = 47,
  /* euclidean_cuda_advanced.cpp:10-27 */
  EUC_OP_ADV_FP64_FP16 = 50, EUC_OP_ADV_FP64_BF16 = 51, EUC_OP_ADV_FP64_TF32 = 52,
  EUC_OP_ADV_FP64_FP32_GEMM = 53,
  /* center_kernels.cu:255-262 */
  EUC_OP_CENTERS_FP32 = 60, EUC_OP_CENTERS_FP64 = 61
} euc_op;

/* Device workspace (bytes) needed by `op` at this size.  For the fused argmin
 * entry (euc_argmin) pass the distance op it is built on. */
EUC_API size_t euc_workspace_bytes(int op, int64_t n, int64_t m, int64_t dim);
EUC_API size_t euc_argmin_workspace_bytes(int op, int64_t n, int64_t m, int64_t dim);

/* Optional per-call timing of the dominant distance kernel (CUDA events on the
 * launching stream).  euc_last_kernel_ms() synchronises on the stop event. */
EUC_API void euc_set_kernel_timing(int enable);
EUC_API float euc_last_kernel_ms(void);
/* Name of the kernel that euc_last_kernel_ms() timed. */
EUC_API const char* euc_last_kernel_name(void);

/* ------------------------------------------------------- base op (fp32/fp64)
 * pairwise_euclidean_single / _double, euclidean_kernels.cu:83,120
 * (bound at euclidean_cuda.cpp:26,30).  D = max(|p|^2 - 2 p.c + |c|^2, 0). */
EUC_API int euc_pairwise_single(const float* P, const float* C, int64_t n, int64_t m, int64_t dim,
                        float* D, void* ws, size_t ws_bytes, void* stream);
EUC_API int euc_pairwise_double(const double* P, const double* C, int64_t n, int64_t m, int64_t dim,
                        double* D, void* ws, size_t ws_bytes, void* stream);

/* ------------------------------------------------ mixed precision + fallback
 * One entry per pairwise_euclidean_<low>_<fallback> of euclidean_kernels_mix.cu.
 * P, C are fp32; D is fp32 n x m.  `d_count` (nullable, device uint64) receives
 * the number of pairs flagged by the cancellation test; it replaces the
 * `_with_stats` twins (euclidean_kernels_mix.cu:713-912, 1099-1626), which read
 * the same counter back to the host. */
#define EUC_MIX_DECL(name)                                                                 \
  EUC_API int name(const float* P, const float* C, int64_t n, int64_t m, int64_t dim, float kappa, \
           float* D, uint64_t* d_count, void* ws, size_t ws_bytes, void* stream)
EUC_MIX_DECL(euc_mix_fp16_fp64); /* euclidean_kernels_mix.cu:515  */
EUC_MIX_DECL(euc_mix_bf16_fp64); /* euclidean_kernels_mix.cu:584  */
EUC_MIX_DECL(euc_mix_tf32_fp64); /* euclidean_kernels_mix.cu:648  */
EUC_MIX_DECL(euc_mix_fp32_fp64); /* euclidean_kernels_mix.cu:918  */
EUC_MIX_DECL(euc_mix_fp16_fp16); /* euclidean_kernels_mix.cu:1041 */
EUC_MIX_DECL(euc_mix_fp16_fp32); /* euclidean_kernels_mix.cu:1163 */
EUC_MIX_DECL(euc_mix_bf16_bf16); /* euclidean_kernels_mix.cu:1284 */
EUC_MIX_DECL(euc_mix_bf16_fp32); /* euclidean_kernels_mix.cu:1405 */
EUC_MIX_DECL(euc_mix_fp32_fp32); /* euclidean_kernels_mix.cu:1525 */
#undef EUC_MIX_DECL

/* ---------------------------------------------------------- tiled operators
 * pairwise_euclidean_tiled_<low>_<high>[_with_stats], euclidean_kernels_tiled.cu:440-528.
 * tile_size must be 16 or 32 (<= 0 selects 32 for dim <= 128, else 16) and dim <= 512,
 * as in euclidean_kernels_tiled.cu:331-336.  `d_tile_counts` (nullable, device int32,
 * ceil(n/T)*ceil(m/T) entries, zeroed by the call) receives the per-tile flag counts
 * in the reference's tile order (tile_i * ceil(m/T) + tile_j). */
#define EUC_TILED_DECL(name)                                                                 \
  EUC_API int name(const float* P, const float* C, int64_t n, int64_t m, int64_t dim, float kappa,   \
           int tile_size, float* D, int32_t* d_tile_counts, uint64_t* d_count, void* ws,     \
           size_t ws_bytes, void* stream)
EUC_TILED_DECL(euc_tiled_fp16_fp64); /* euclidean_kernels_tiled.cu:440 */
EUC_TILED_DECL(euc_tiled_fp16_fp32); /* euclidean_kernels_tiled.cu:447 */
EUC_TILED_DECL(euc_tiled_bf16_fp64); /* euclidean_kernels_tiled.cu:470 */
EUC_TILED_DECL(euc_tiled_bf16_fp32); /* euclidean_kernels_tiled.cu:477 */
EUC_TILED_DECL(euc_tiled_fp32_fp64); /* euclidean_kernels_tiled.cu:500 */
EUC_TILED_DECL(euc_tiled_fp32_fp32); /* euclidean_kernels_tiled.cu:507 */
#undef EUC_TILED_DECL

/* pairwise_euclidean_tensorcore_<low>_<high>, euclidean_kernels_tiled_tc.cu:274-300.
 * tile_size must be 32 (<= 0 selects 32) and dim % 16 == 0, as in
 * euclidean_kernels_tiled_tc.cu:246-248. */
#define EUC_TC_DECL(name)                                                                   \
  EUC_API int name(const float* P, const float* C, int64_t n, int64_t m, int64_t dim, float kappa,  \
           int tile_size, float* D, uint64_t* d_count, void* ws, size_t ws_bytes, void* stream)
EUC_TC_DECL(euc_tensorcore_fp16_fp64); /* euclidean_kernels_tiled_tc.cu:274 */
EUC_TC_DECL(euc_tensorcore_fp16_fp32); /* euclidean_kernels_tiled_tc.cu:281 */
EUC_TC_DECL(euc_tensorcore_bf16_fp64); /* euclidean_kernels_tiled_tc.cu:288 */
EUC_TC_DECL(euc_tensorcore_bf16_fp32); /* euclidean_kernels_tiled_tc.cu:295 */
#undef EUC_TC_DECL

/* -------------------------------------------------------- uniform precision
 * pairwise_euclidean_uniform_*, euclidean_kernels_uniform.cu:138-532.  fp16/bf16
 * tensors are passed as uint16_t bit patterns; D has the input's type. */
EUC_API int euc_uniform_fp16(const uint16_t* P, const uint16_t* C, int64_t n, int64_t m, int64_t dim,
                     uint16_t* D, void* ws, size_t ws_bytes, void* stream);          /* :138 */
EUC_API int euc_uniform_bf16(const uint16_t* P, const uint16_t* C, int64_t n, int64_t m, int64_t dim,
                     uint16_t* D, void* ws, size_t ws_bytes, void* stream);          /* :177 */
EUC_API int euc_uniform_tf32(const float* P, const float* C, int64_t n, int64_t m, int64_t dim,
                     float* D, void* ws, size_t ws_bytes, void* stream);             /* :215 */
EUC_API int euc_uniform_fp16_direct(const uint16_t* P, const uint16_t* C, int64_t n, int64_t m,
                            int64_t dim, uint16_t* D, void* stream);                  /* :288 */
EUC_API int euc_uniform_bf16_direct(const uint16_t* P, const uint16_t* C, int64_t n, int64_t m,
                            int64_t dim, uint16_t* D, void* stream);                  /* :345 */
EUC_API int euc_uniform_tf32_direct(const float* P, const float* C, int64_t n, int64_t m,
                            int64_t dim, float* D, void* stream);                     /* :398 */
EUC_API int euc_uniform_fp32_direct(const float* P, const float* C, int64_t n, int64_t m,
                            int64_t dim, float* D, void* stream);                     /* :453 */
EUC_API int euc_uniform_fp64_direct(const double* P, const double* C, int64_t n, int64_t m,
                            int64_t dim, double* D, void* stream);                    /* :507 */

/* ------------------------------------------------------- advanced operators
 * euclidean_kernels_advanced.cu:225-453 (bound at euclidean_cuda_advanced.cpp:10-27). */
EUC_API int euc_advanced_fp64_fp16(const uint16_t* P, const uint16_t* C, int64_t n, int64_t m,
                           int64_t dim, float kappa, float* D, uint64_t* d_count, void* ws,
                           size_t ws_bytes, void* stream);                           /* :225 */
EUC_API int euc_advanced_fp64_bf16(const uint16_t* P, const uint16_t* C, int64_t n, int64_t m,
                           int64_t dim, float kappa, float* D, uint64_t* d_count, void* ws,
                           size_t ws_bytes, void* stream);                           /* :283 */
EUC_API int euc_advanced_fp64_tf32(const float* P, const float* C, int64_t n, int64_t m,
                           int64_t dim, float kappa, double* D, uint64_t* d_count, void* ws,
                           size_t ws_bytes, void* stream);                           /* :341 */
EUC_API int euc_advanced_fp64_fp32_gemm(const double* P, const double* C, int64_t n, int64_t m,
                                int64_t dim, float kappa, double* D, uint64_t* d_count,
                                void* ws, size_t ws_bytes, void* stream);            /* :398 */

/* get_fallback_count_low / get_last_fallback_count (euclidean_kernels_mix.cu:1028,
 * euclidean_kernels_advanced.cu:455): synchronous read of a device int32 counter. */
EUC_API int euc_read_count_i32(const int32_t* d_counter, int32_t* host_out);
/* Synchronous read of a device uint64 counter written by d_count above. */
EUC_API int euc_read_count_u64(const uint64_t* d_counter, uint64_t* host_out);

/* ---------------------------------------------------------- center update
 * update_centers_fp32 / _fp64, center_kernels.cu:101-139 (bound at :255-262):
 * centers[c] = mean of the rows of X whose label is c; labels outside [0, k) are
 * ignored; an empty cluster's center is 0.  Sums are accumulated in fp64.
 * `d_counts` (nullable, device int64[k]) receives the cluster sizes; the
 * `_with_reinit` twins (center_kernels.cu:195-246) are composed from these counts
 * and the caller's RNG by the binding layer. */
EUC_API int euc_update_centers_fp32(const float* X, const int64_t* labels, int64_t n, int64_t dim,
                            int64_t k, float* centers, int64_t* d_counts, void* ws,
                            size_t ws_bytes, void* stream);
EUC_API int euc_update_centers_fp64(const double* X, const int64_t* labels, int64_t n, int64_t dim,
                            int64_t k, double* centers, int64_t* d_counts, void* ws,
                            size_t ws_bytes, void* stream);

/* ============================================================ new entries
 * No counterpart in the reference: the k-means caller composes these instead of
 * materialising D (the Lloyd hot path: distances -> argmin -> center update). */

/* `exact` value of euc_argmin selecting the certified mode (no counterpart in the
 * reference). */
#define EUC_ARGMIN_CERTIFIED 2

/* Fused distance + row argmin for distance operator `op` (an EUC_OP_MIX_*,
 * EUC_OP_TILED_*, EUC_OP_TC_*, EUC_OP_SINGLE or EUC_OP_DOUBLE id), without
 * materialising D.  Flagged pairs take their recomputed value, as in the reference.
 *   exact == EUC_ARGMIN_CERTIFIED (tensor-core operators whose recompute is fp32 or
 *               fp64): the label is the first index of the smallest direct distance
 *               direct(p, c_j) over all centers, in the operator's recompute
 *               arithmetic (the value `op` stores for a pair it flags), and min_dist is
 *               that distance -- the reference's labels when every pair of the row is
 *               flagged.  The tensor-core screen bounds every pair; only the
 *               centers that can win are recomputed: the 8 of the best group of 8
 *               norm-sorted centers when the bounds separate it from the rest, else
 *               those of every group a second screen finds within reach (all of the
 *               row's when the norms give no bound).  d_count receives the number of
 *               direct distances evaluated.  Other operators return
 *               EUC_ERR_UNSUPPORTED.
 *   exact != 0 (other values): every pair's distance is formed exactly as `op` forms
 *               D, and the label is torch.argmin(D, 1) of that D (first index of the
 *               minimum).
 *   exact == 0: tensor-core operators screen each 32-center chunk: the MMA itself
 *               yields y = (|c|^2 + Br)/2 - p.c (Br = 1.0625 |p|^2 of the row), and per
 *               pair one key (y with the column in its low 5 bits) and half a 3-way min
 *               remain; the exact path runs only on chunks where a pair could be
 *               flagged.  Labels equal the exact ones whenever the row's top-two
 *               distance gap exceeds 2^-10 (|p|^2 + max|c|^2) + 2^-16 (max|c|^2 + Br)
 *               (2^-7 for bf16 S); min_dist then carries about 18 significant bits
 *               relative to max|c|^2 + Br.  For the fp16/bf16 mix operators with
 *               dim % 4 == 0 and a 16-byte aligned P, the screen reads the fp32 points
 *               itself (no low-precision copy of P is made).
 * P/C element type follows `op` (fp64 for EUC_OP_DOUBLE, fp32 otherwise).  Outputs
 * are nullable: labels (int64[n]), labels32 (int32[n]), min_dist (fp32[n]; fp64[n]
 * for EUC_OP_DOUBLE). */
EUC_API int euc_argmin(int op, const void* P, const void* C, int64_t n, int64_t m, int64_t dim,
               float kappa, int exact, int64_t* labels, int32_t* labels32, void* min_dist,
               uint64_t* d_count, void* ws, size_t ws_bytes, void* stream);

/* Prepared points.  The reference casts the fp32 points to the GEMM's low precision on
 * every call (euclidean_kernels_mix.cu:531-532, P.to(torch::kFloat16)); a caller that
 * screens the same points many times (Lloyd iterations) can keep that low-precision
 * copy instead: euc_prepare_points writes, for a tensor-core operator `op`, the points
 * rounded to its operand type (rows padded to whole 128-byte boxes) followed by their
 * norms in the operator's recipe, into a caller buffer of euc_prepared_points_bytes().
 * euc_argmin_prepared then screens from that copy (2 bytes a value for fp16/bf16) and
 * reads the fp32 points P only for the pairs it recomputes; its outputs equal
 * euc_argmin's for the same P (modes 0 and 1; the certified mode is rejected).  Its
 * workspace is euc_argmin_prepared_workspace_bytes(), smaller than euc_argmin's by the
 * copy and the norms.  No counterpart in the reference beyond the cast it replaces. */
EUC_API size_t euc_prepared_points_bytes(int op, int64_t n, int64_t dim);
EUC_API int euc_prepare_points(int op, const float* P, int64_t n, int64_t dim, void* prep, size_t prep_bytes,
                       void* stream);
EUC_API size_t euc_argmin_prepared_workspace_bytes(int op, int64_t n, int64_t m, int64_t dim);
EUC_API int euc_argmin_prepared(int op, const float* P, const void* prep, const float* C, int64_t n, int64_t m,
                        int64_t dim, float kappa, int exact, int64_t* labels, int32_t* labels32, void* min_dist,
                        uint64_t* d_count, void* ws, size_t ws_bytes, void* stream);

/* No counterpart in the reference.  euc_argmin without a workspace, for callers that
 * cannot allocate device memory (a host binding with no device allocator, or a
 * process whose memory pool already holds the device's memory): the scratch is one
 * static device array of euc_argmin_noalloc_max_bytes() (32 MiB) per device and
 * context; nothing is allocated.  The array takes its device memory when its module
 * loads into a context: on the first call on that device under CUDA's default lazy
 * loading, at context creation under CUDA_MODULE_LOADING=EAGER (then in every process
 * that loads this library, whether or not it calls this entry); it holds it until the
 * context ends.  The first call on each device should come before any stream capture.
 * Every call takes the array's address in the current context, so it follows a reset
 * or a caller's own context.  Arguments are checked first (unknown op EUC_ERR_ARG,
 * negative sizes EUC_ERR_SHAPE, no sm_100 device EUC_ERR_DEVICE); a shape whose
 * euc_argmin_workspace_bytes() exceeds the array is rejected with EUC_ERR_WORKSPACE
 * before any launch.  Calls that overlap in time in one context race on the shared
 * scratch. */
EUC_API size_t euc_argmin_noalloc_max_bytes(void);
EUC_API int euc_argmin_noalloc(int op, const void* P, const void* C, int64_t n, int64_t m, int64_t dim,
                       float kappa, int exact, int64_t* labels, int32_t* labels32, void* min_dist,
                       uint64_t* d_count, void* stream);

/* Partial center statistics for data-parallel Lloyd iterations: for the n local
 * rows, stats[c*(dim+1) + j] = sum of X[i, j] over rows with label c (j < dim) and
 * stats[c*(dim+1) + dim] = number of such rows, all fp64 (exact integer counts).
 * `x_is_f64` selects fp64 X (else fp32); labels are int32 (labels_are_i64 = 0)
 * or int64.  One all-reduce(sum) of `stats` combines ranks. */
EUC_API size_t euc_center_stats_workspace_bytes(int64_t n, int64_t dim, int64_t k);
EUC_API int euc_center_stats(const void* X, int x_is_f64, const void* labels, int labels_are_i64,
                     int64_t n, int64_t dim, int64_t k, double* stats, void* ws,
                     size_t ws_bytes, void* stream);
/* centers[c, j] = stats[c, j] / stats[c, dim]; an empty cluster becomes 0
 * (empty_policy 0, the reference's behaviour) or keeps `prev` (empty_policy 1). */
EUC_API int euc_center_finalize(const double* stats, int64_t dim, int64_t k, void* centers,
                        int centers_are_f64, const void* prev, int empty_policy, void* stream);

/* No counterpart in the reference: k-means++ seeding, the caller-side step before the
 * Lloyd loop, on the device and deterministic for a given `seed`.  Row 0 of the
 * chosen set is uniform over the n rows; each next row is drawn with probability
 * proportional to its squared distance to the nearest chosen row (the fp64 direct sum
 * in dimension order), the weights scaled to exact 62-bit integers so that the draw
 * does not depend on summation order; draw s uses the top 53 bits of
 * SplitMix64(seed + (s + 1) * 0x9E3779B97F4A7C15).  Writes indices (int64[k], device)
 * and, if non-null, centers (k x dim rows of X, X's type).  One host-side launch
 * sequence of 3 kernels per center; `ws` of euc_kmeanspp_workspace_bytes(). */
EUC_API size_t euc_kmeanspp_workspace_bytes(int64_t n, int64_t dim, int64_t k);
EUC_API int euc_kmeanspp(const void* X, int x_is_f64, int64_t n, int64_t dim, int64_t k, uint64_t seed,
                 int64_t* indices, void* centers, void* ws, size_t ws_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* EUCLID_B200_H */
