// Fused distance + argmin for callers that cannot allocate device memory.
//
// euc_argmin_noalloc runs exactly the kernels of euc_argmin, but instead of a
// caller-owned workspace it uses one file-scope __device__ array of NOALLOC_SCRATCH_BYTES
// (one instance per device and context).  Nothing here calls cudaMalloc, cudaFree or any
// allocating routine.
//
// Set-up: this file's module holds no kernel, only the array, so it is loaded into a
// context the first time the array's address is taken there: lazily (CUDA's default
// module loading) on the first call on each device, with that device current, or at
// context creation under CUDA_MODULE_LOADING=EAGER.  From then on the array holds its
// 32 MiB of that device's memory until the context ends, in every process that loads
// it.  The first call on a device should come before any stream capture.
//
// Every call takes the array's address in the current context with
// cudaGetSymbolAddress (a host-side lookup that allocates nothing), so the address
// follows the context: a cudaDeviceReset, or a caller's own driver-API context, gets
// its own array rather than a stale address.
//
// What must start at zero: the flag counter inside the scratch; euc_argmin clears it
// with cudaMemsetAsync on `stream` at the start of every call (and clears the certified
// mode's counters and switches the same way).  Every other scratch word is written
// before it is read within the call, so the scratch needs no zeroing at set-up.
//
// All calls in one context share the one scratch: calls that overlap in time (on
// different streams, or from different host threads without ordering) race on it.
#include <cuda_runtime.h>

#include <string>

#include "../../include/euclid_b200.h"
#include "engine.h"

namespace euc {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// address of the scratch array in the current context
static int noalloc_scratch(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p)
    return set_error(EUC_ERR_LAUNCH, (std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e)).c_str());
  *out = p;
  return EUC_OK;
}

}  // namespace euc

extern "C" {

size_t euc_argmin_noalloc_max_bytes(void) { return euc::NOALLOC_SCRATCH_BYTES; }

int euc_argmin_noalloc(int op, const void* P, const void* C, int64_t n, int64_t m, int64_t dim, float kappa,
                       int exact, int64_t* labels, int32_t* labels32, void* min_dist, uint64_t* d_count,
                       void* stream) {
  // the argument checks euc_argmin makes, before the size test and the array's address
  // (a negative size must not read as a huge workspace, a wrong device must not try to
  // load the module)
  if (!euc::find_op(op)) return euc::set_error(EUC_ERR_ARG, "unknown operator id");
  if (n < 0 || m < 0 || dim < 0) return euc::set_error(EUC_ERR_SHAPE, "negative size");
  if (!euc::device_is_sm100())
    return euc::set_error(EUC_ERR_DEVICE, "euclid_b200 requires an sm_100 (B200) device");
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
