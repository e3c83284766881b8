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
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current, and caches it.  Make
//    that first call before any stream capture begins.
#include <cstdio>
#include <mutex>

#include "sc_common.cuh"

namespace scmp {
void set_last_error(const char *msg);
}

namespace {

constexpr size_t kScratchBytes = (size_t)SCMP_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The scratch array.  In host code `g_noalloc_scratch` names a host-side
// stand-in, not device memory: pass only the address from
// cudaGetSymbolAddress to kernels.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void *g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up on the
// first call per device).
int scratch_for_current_device(void **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    scmp::set_last_error(cudaGetErrorString(e));
    return SCMP_ECUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    scmp::set_last_error("device ordinal out of range for the no-alloc scratch table");
    return SCMP_EUNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      scmp::set_last_error(e != cudaSuccess ? cudaGetErrorString(e)
                                            : "cudaGetSymbolAddress returned NULL");
      return SCMP_ECUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
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
