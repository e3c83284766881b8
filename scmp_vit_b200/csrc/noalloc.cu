// scmp_sc_matmul_noalloc: the SC matmul for callers that cannot allocate.
//
// scmp_sc_matmul needs device scratch (quantised codes, scales, the stream
// table) and takes it from the caller.  Some callers have no way to provide
// it: a host that binds the C ABI from plain C or another language's FFI has
// no caching allocator, and a cudaMalloc/cudaFree pair per call would
// synchronise the device and stall every other stream; a runtime that
// reserves the whole device memory budget at start-up does not let a plug-in
// allocate at all.  This entry point takes its scratch from a fixed array
// compiled into the library instead, so it allocates nothing.
//
// Limits and rules (also stated in include/scmp_b200.h):
//  * The array holds SCMP_NOALLOC_SCRATCH_BYTES (32 MiB) on every device that
//    loads the library, for the life of the process.  Problems whose scratch
//    (scmp_sc_matmul_workspace_size) exceeds it are rejected with
//    SCMP_EWORKSPACE and a message naming both sizes.
//  * All calls on a device share the one array and it keeps whatever the last
//    call left there.  The engine writes every scratch byte it reads before
//    reading it, so nothing needs clearing between calls -- but two calls
//    whose kernels overlap on the GPU (different streams, no ordering) race on
//    the array and corrupt each other.  Order such calls on one stream.
//  * The first call on each device (and in each further driver context a
//    host makes current on it) looks up the array's device address
//    (cudaGetSymbolAddress) with that device current, and caches it per
//    (device, context).  Make that first call before any stream capture
//    begins.
#include <cstdio>
#include <mutex>

#include "sc_common.cuh"

namespace {

constexpr size_t kScratchBytes = (size_t)SCMP_NOALLOC_SCRATCH_BYTES;

// The scratch array.  In host code `g_noalloc_scratch` names a host-side
// stand-in, not device memory: pass only the address from
// cudaGetSymbolAddress to kernels.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
scmp::SymbolCache g_scratch_ptr[scmp::kMaxCachedDevices];

// Device address of the scratch array in the current context (set-up on the
// first call per device and context).
int scratch_for_current_device(void **out) {
  const cudaError_t e = scmp::cached_symbol_address(g_scratch_ptr, g_mu, g_noalloc_scratch, out);
  if (e != cudaSuccess) {
    scmp::set_last_error(e == cudaErrorInvalidDevice
                             ? "device ordinal out of range for the no-alloc scratch table"
                             : cudaGetErrorString(e));
    return e == cudaErrorInvalidDevice ? SCMP_EUNSUPPORTED : SCMP_ECUDA;
  }
  return SCMP_OK;
}

}  // namespace

extern "C" SCMP_API int scmp_sc_matmul_noalloc(const scmp_matmul_args *args, void *stream) {
  if (!args) {
    scmp::set_last_error("args is NULL");
    return SCMP_EINVAL;
  }
  const size_t need = scmp_sc_matmul_workspace_size(args);
  if (need == 0) return scmp_sc_matmul(args, stream);  // invalid: reports the reason
  if (need > kScratchBytes) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "problem needs %zu bytes of scratch; the no-alloc entry point has %zu "
             "(SCMP_NOALLOC_SCRATCH_BYTES); use scmp_sc_matmul with a caller workspace",
             need, kScratchBytes);
    scmp::set_last_error(buf);
    return SCMP_EWORKSPACE;
  }
  void *scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != SCMP_OK) return rc;
  scmp_matmul_args local = *args;
  local.workspace = scratch;
  local.workspace_bytes = kScratchBytes;
  return scmp_sc_matmul(&local, stream);
}
