// sas_fwd_noalloc: the forward for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc at the point where they
// run attention: code inside a pre-planned memory arena, a runtime whose
// allocator is frozen during a step, or a host that forbids device
// allocations after start-up.  sas_fwd needs a caller-sized workspace (the
// work plan plus the fp32 split-KV partials).  This entry point keeps that
// workspace in a file-scope device array instead, so a call needs nothing
// beyond the caller's inputs and outputs.
//
// * Limit: SAS_NOALLOC_SCRATCH_BYTES (16 MiB).  A problem whose plan and
//   partials need more is rejected with SAS_ERR_WORKSPACE; fewer workers
//   (SasFwdParams.num_sms) means fewer split rows and smaller partials.
// * Every GPU that loads libsas.so holds the array until the process exits.
// * In host code the array's name is only a host-side stand-in; its device
//   address is looked up with cudaGetSymbolAddress once per device, on that
//   device's first call (with that device current).  Make that first call
//   before any stream capture.
// * Each call builds its work plan on the host and copies it into the array
//   with a stream-ordered copy from host memory, then launches the kernels.
// * All calls on a device share the array and it keeps the last call's
//   contents.  Nothing in it has to start at zero: the plan is rewritten by
//   every call and each partial is written before it is read.  Calls that
//   overlap on the GPU (concurrent streams or host threads on one device)
//   race on the array: serialise them.
// * No cudaMalloc, cudaFree or other allocating device call is made.

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <vector>

#include "sas.h"
#include "sas_internal.h"
#include "sas_kernels.h"

namespace {

constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[SAS_NOALLOC_SCRATCH_BYTES];

std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up once).
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SAS_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return SAS_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return SAS_OK;
}

}  // namespace

extern "C" int sas_fwd_noalloc(const SasProblem* prob, const SasFwdParams* params,
                               void* stream) {
  if (!prob || !params) return SAS_ERR_INVALID;
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != SAS_OK) return rc;
  // sas_fwd_prepare plans once and returns SAS_ERR_WORKSPACE, before copying
  // anything, when the plan and partials need more than the array holds.
  SasPlanInfo info;
  rc = sas_fwd_prepare(prob, params, scratch, SAS_NOALLOC_SCRATCH_BYTES, stream, &info);
  if (rc != SAS_OK) return rc;
  return sas_fwd_execute(prob, params, &info, scratch, SAS_NOALLOC_SCRATCH_BYTES, stream,
                         SAS_PHASE_ALL);
}
