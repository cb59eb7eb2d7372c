// ssm_noalloc.cu — ssm_scan_bwd_noalloc: the backward scan without a caller workspace.
//
// Some callers cannot hand the backward a scratch buffer: a serving or training process whose
// memory pool is fixed after start-up and forbids cudaMalloc on the hot path, or a plugin whose
// host application owns all device memory and gives the plugin no allocator.  For them the
// library carries a fixed scratch area in the module itself: every GPU that loads the library
// holds SSM_NOALLOC_SCRATCH_BYTES of device memory until the process exits.
//
// The scratch is a file-scope __device__ array.  Host code must not pass the array's name to a
// kernel (in host code it is only a host-side stand-in); every call looks up its device address
// on the current device through cudaGetSymbolAddress (cheap once the module is loaded; not cached,
// so a cudaDeviceReset, after which the array can sit elsewhere, leaves no stale address behind).
#include <cuda_runtime.h>

#include <cstdio>

#include "ssm_b200.h"

namespace ssm {
int report_error(int code, const char* msg);   // sets the message ssm_last_error_message returns
}  // namespace ssm

namespace {

static __device__ __align__(256) unsigned char g_ssm_noalloc_scratch[SSM_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array on the current device.
int scratch_address(void** out) {
  char msg[256];
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_ssm_noalloc_scratch);
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "cudaGetSymbolAddress of the scratch array: %s", cudaGetErrorString(e));
    return ssm::report_error(SSM_ERR_CUDA, msg);
  }
  *out = p;
  return SSM_OK;
}

}  // namespace

extern "C" int ssm_scan_bwd_noalloc(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view u,
                                    ssm_view delta, const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip,
                                    ssm_view z, const float* h0, const float* chunk_states, ssm_view ygate,
                                    ssm_view dy, const float* dlast, ssm_view du, ssm_view ddelta, float* dA,
                                    ssm_view dBm, ssm_view dCm, float* dDskip, ssm_view dz, float* dh0,
                                    void* stream) {
  size_t need = 0;
  int rc = ssm_scan_bwd_workspace_size(B, L, D, N, &need);
  if (rc != SSM_OK) return rc;
  if (need > (size_t)SSM_NOALLOC_SCRATCH_BYTES) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "ssm_scan_bwd_noalloc: this shape needs %zu bytes of scratch; the built-in scratch holds %zu "
             "(call ssm_scan_bwd with a workspace instead)",
             need, (size_t)SSM_NOALLOC_SCRATCH_BYTES);
    return ssm::report_error(SSM_ERR_WORKSPACE, msg);
  }
  void* scratch = nullptr;
  rc = scratch_address(&scratch);
  if (rc != SSM_OK) return rc;
  // The backward writes every scratch word it reads (per-CTA partials, then their sums), so the
  // contents left by an earlier call need no clearing.
  return ssm_scan_bwd(B, L, D, N, method, u, delta, A, Bm, Cm, Dskip, z, h0, chunk_states, ygate, dy, dlast, du,
                      ddelta, dA, dBm, dCm, dDskip, dz, dh0, scratch, (size_t)SSM_NOALLOC_SCRATCH_BYTES, stream);
}
