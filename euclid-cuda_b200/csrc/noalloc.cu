// Fused distance + argmin for callers that cannot allocate device memory.
//
// euc_argmin_noalloc runs exactly the kernels of euc_argmin, but instead of a
// caller-owned workspace it uses one file-scope __device__ array of NOALLOC_SCRATCH_BYTES
// (one instance per device).  Nothing here calls cudaMalloc, cudaFree or any
// allocating routine.
//
// Set-up: the first call on each device (with that device current) takes the array's
// address with cudaGetSymbolAddress, which also loads this module onto the device,
// and caches it.  That first call should come before any stream capture.
//
// What must start at zero: the flag counter inside the scratch; euc_argmin clears it
// with cudaMemsetAsync on `stream` at the start of every call.  Every other scratch
// word is written before it is read within the call, so the scratch needs no zeroing
// at set-up.
//
// All calls on one device share the one scratch: calls that overlap in time (on
// different streams, or from different host threads without ordering) race on it.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/euclid_b200.h"
#include "engine.h"

namespace euc {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(32) << 20;
constexpr int NOALLOC_MAX_DEVICES = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[NOALLOC_MAX_DEVICES];

// address of this device's scratch array, taken once per device
static int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(EUC_ERR_DEVICE, cudaGetErrorString(e));
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return set_error(EUC_ERR_DEVICE, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(EUC_ERR_LAUNCH, (std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e)).c_str());
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return EUC_OK;
}

}  // namespace euc

extern "C" {

size_t euc_argmin_noalloc_max_bytes(void) { return euc::NOALLOC_SCRATCH_BYTES; }

int euc_argmin_noalloc(int op, const void* P, const void* C, int64_t n, int64_t m, int64_t dim, float kappa,
                       int exact, int64_t* labels, int32_t* labels32, void* min_dist, uint64_t* d_count,
                       void* stream) {
  const size_t need = euc_argmin_workspace_bytes(op, n, m, dim);
  if (need > euc::NOALLOC_SCRATCH_BYTES)
    return euc::set_error(EUC_ERR_WORKSPACE,
                          ("euc_argmin_noalloc: this shape needs " + std::to_string(need) +
                           " bytes of scratch; the static scratch holds " +
                           std::to_string(euc::NOALLOC_SCRATCH_BYTES) + " (use euc_argmin with a workspace)")
                              .c_str());
  void* ws = nullptr;
  const int rc = euc::noalloc_scratch(&ws);
  if (rc != EUC_OK) return rc;
  return euc_argmin(op, P, C, n, m, dim, kappa, exact, labels, labels32, min_dist, d_count, ws,
                    euc::NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
