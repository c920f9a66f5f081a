// Selective recompute of the pairs flagged by the cancellation test, as a compacted
// second pass (the reference launches N*M threads and lets all but `count` exit,
// euclidean_kernels_mix.cu:573-578; here the grid is sized to the machine and walks
// only the list).
//
// D mode    : D[i, j] = direct(i, j) for every listed pair.  If more pairs were flagged
//             than the list holds, the kernel instead sweeps all of D and re-derives
//             the flag from the stored distance and norms (bit-identical test), so no
//             flagged pair is ever lost.
// argmin mode: row_key[i] = min(row_key[i], (direct(i, j), j)) with a 64-bit atomicMin;
//             the distance epilogue already recomputed in place whatever did not fit.
#include "common.cuh"
#include "engine.h"
#include "direct.cuh"

namespace euc {

struct RecArgs {
  const void* P;
  const void* C;
  int64_t n, m;
  int dim;
  const unsigned long long* list;
  const unsigned long long* count;
  unsigned long long cap;
  void* D;
  unsigned long long* row_key;
  const void* pp;
  const void* cc;
  float kf;
  double kd;
};

template <typename TIN, int REC, typename TOUT, int FLAG, bool ARGMIN>
__global__ void __launch_bounds__(256) recompute_kernel(const RecArgs a) {
  const TIN* P = static_cast<const TIN*>(a.P);
  const TIN* C = static_cast<const TIN*>(a.C);
  const unsigned long long cnt = *a.count;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  const uint64_t t0 = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  // argmin: the listed pairs always go through here (the distance epilogue folded the
  // ones beyond the list's capacity in place); D: an overflowing list is ignored and
  // the dense sweep below recomputes every flagged pair instead
  if (ARGMIN || cnt <= a.cap) {
    const unsigned long long nlist = cnt < a.cap ? cnt : a.cap;
    for (uint64_t t = t0; t < nlist; t += stride) {
      const unsigned long long e = a.list[t];
      const int64_t i = static_cast<int64_t>(e >> 32);
      const int64_t j = static_cast<int64_t>(e & 0xffffffffull);
      if (i >= a.n || j >= a.m) continue;
      const double v = direct_dist<TIN, REC>(P + i * a.dim, C + j * a.dim, a.dim);
      if constexpr (ARGMIN) {
        atomicMin(&a.row_key[i], make_key(static_cast<float>(v), static_cast<uint32_t>(j)));
      } else {
        static_cast<TOUT*>(a.D)[i * a.m + j] = static_cast<TOUT>(v);
      }
    }
  } else if constexpr (!ARGMIN) {
    // overflow: dense sweep, flag re-derived from the stored (pre-recompute) distance
    const uint64_t total = static_cast<uint64_t>(a.n) * static_cast<uint64_t>(a.m);
    for (uint64_t t = t0; t < total; t += stride) {
      const int64_t i = static_cast<int64_t>(t / static_cast<uint64_t>(a.m));
      const int64_t j = static_cast<int64_t>(t % static_cast<uint64_t>(a.m));
      TOUT* dp = static_cast<TOUT*>(a.D) + t;
      bool flag;
      if constexpr (FLAG == FL_F32) {
        const float pp = static_cast<const float*>(a.pp)[i], cc = static_cast<const float*>(a.cc)[j];
        flag = static_cast<float>(*dp) <= __fmul_rn(a.kf, __fadd_rn(pp, cc));
      } else {
        const double pp = static_cast<const double*>(a.pp)[i], cc = static_cast<const double*>(a.cc)[j];
        flag = static_cast<double>(*dp) <= a.kd * (pp + cc);
      }
      if (flag) *dp = static_cast<TOUT>(direct_dist<TIN, REC>(P + i * a.dim, C + j * a.dim, a.dim));
    }
  }
}

template <typename TIN, int REC, typename TOUT, int FLAG, bool ARGMIN>
static cudaError_t go_rec(const DistJob& j) {
  RecArgs a{};
  a.P = j.P;
  a.C = j.C;
  a.n = j.n;
  a.m = j.m;
  a.dim = j.dim;
  a.list = j.list;
  a.count = j.count;
  a.cap = j.list_cap;
  a.D = j.D;
  a.row_key = j.row_key;
  a.pp = j.pp;
  a.cc = j.cc;
  a.kf = j.kf;
  a.kd = j.kd;
  const int blocks = num_sms() * 8;
  recompute_kernel<TIN, REC, TOUT, FLAG, ARGMIN><<<blocks, 256, 0, j.stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_recompute(const DistJob& j) {
  const OpSpec* s = j.spec;
  if (s->flag == FL_NONE) return cudaSuccess;
  const bool argmin = (j.D == nullptr);
#define REC_CASE(IN_, TIN_, REC_, OUT_, TOUT_, FLAG_)                                                    \
  if (s->in == IN_ && s->rec == REC_ && s->flag == FLAG_ && (argmin || s->out == OUT_)) {                \
    if (argmin) return go_rec<TIN_, REC_, TOUT_, FLAG_, true>(j);                                        \
    return go_rec<TIN_, REC_, TOUT_, FLAG_, false>(j);                                                   \
  }
  REC_CASE(IN_F32, float, RC_F64, OUT_F32, float, FL_F32)
  REC_CASE(IN_F32, float, RC_F32, OUT_F32, float, FL_F32)
  REC_CASE(IN_F32, float, RC_F16_ARITH, OUT_F32, float, FL_F32)
  REC_CASE(IN_F32, float, RC_BF16_ARITH, OUT_F32, float, FL_F32)
  if (!argmin) {
    REC_CASE(IN_F16, __half, RC_F64, OUT_F32, float, FL_F32)
    REC_CASE(IN_BF16, __nv_bfloat16, RC_F64, OUT_F32, float, FL_F32)
    REC_CASE(IN_F32, float, RC_F64, OUT_F64, double, FL_F64)
    REC_CASE(IN_F64, double, RC_F64, OUT_F64, double, FL_F64)
  }
#undef REC_CASE
  return cudaErrorNotSupported;
}

// ------------------------------------------------------------------ helpers

__global__ void keys_to_labels_kernel(const unsigned long long* __restrict__ keys, int64_t n,
                                      int64_t* __restrict__ labels, int32_t* __restrict__ labels32,
                                      float* __restrict__ mind) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long k = keys[i];
    const uint32_t j = static_cast<uint32_t>(k & 0xffffffffull);
    if (labels) labels[i] = j;
    if (labels32) labels32[i] = static_cast<int32_t>(j);
    if (mind) mind[i] = __uint_as_float(static_cast<uint32_t>(k >> 32));
  }
}

cudaError_t launch_keys_to_labels(const unsigned long long* keys, int64_t n, int64_t* labels, int32_t* labels32,
                                  float* mind, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, num_sms() * 16));
  keys_to_labels_kernel<<<blocks, 256, 0, st>>>(keys, n, labels, labels32, mind);
  return cudaGetLastError();
}

__global__ void idx_to_labels_kernel(const long long* __restrict__ idx, int64_t n, int64_t* __restrict__ labels,
                                     int32_t* __restrict__ labels32) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (labels) labels[i] = idx[i];
    if (labels32) labels32[i] = static_cast<int32_t>(idx[i]);
  }
}

cudaError_t launch_f64_to_labels(const long long* idx, int64_t n, int64_t* labels, int32_t* labels32,
                                 cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, num_sms() * 16));
  idx_to_labels_kernel<<<blocks, 256, 0, st>>>(idx, n, labels, labels32);
  return cudaGetLastError();
}

__global__ void fill_u64_kernel(unsigned long long* p, int64_t n, unsigned long long v) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = v;
}

cudaError_t launch_fill_u64(unsigned long long* p, int64_t n, unsigned long long v, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, num_sms() * 16));
  fill_u64_kernel<<<blocks, 256, 0, st>>>(p, n, v);
  return cudaGetLastError();
}

}  // namespace euc
