// ipc_weight_update_noalloc: the split-K weight update with its fp32 partial
// tiles in a fixed scratch array of this library rather than caller memory.
//
// The array is a file-scope __device__ variable, so the CUDA runtime places it
// (one copy per device) when it loads this library's device code; the entry
// point looks its address up once per device and hands it to the
// ipc_fused_gemm_ws path as the workspace.  No device memory is allocated by
// the call.  Nothing in the array needs initialising: each split writes its
// whole partial tile before the reduce pass reads it.
#include <cuda_runtime.h>

#include <mutex>

#include "ipc_b200.h"
#include "ipc_common.cuh"

namespace {

constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[IPC_NOALLOC_SCRATCH_BYTES / sizeof(float)];

std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Address of this device's scratch (the current device); looked up on first use.
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return ipc::set_error(IPC_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices)
    return ipc::set_error(IPC_ERR_UNSUPPORTED, "device ordinal %d above %d", dev, kMaxDevices - 1);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr)
      return ipc::set_error(IPC_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev,
                            cudaGetErrorString(err));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return IPC_OK;
}

}  // namespace

extern "C" int ipc_weight_update_noalloc(int mode, const void* e, const void* a_up, void* out, int M, int K, int B,
                                         int groups, float alpha, int flags, int act, int dtype, int algo,
                                         void* stream) {
  if (mode != IPC_MODE_WEIGHT && mode != IPC_MODE_WDELTA)
    return ipc::set_error(IPC_ERR_ARG, "ipc_weight_update_noalloc: mode %d is not IPC_MODE_WEIGHT / IPC_MODE_WDELTA",
                          mode);
  if (M < 0 || K < 0 || B < 0 || groups < 0)
    return ipc::set_error(IPC_ERR_ARG, "ipc_weight_update_noalloc: negative size (M=%d K=%d B=%d groups=%d)", M, K,
                          B, groups);
  const long long elems = (long long)groups * M * K;
  if (elems > (long long)IPC_NOALLOC_MAX_OUT_ELEMS)
    return ipc::set_error(IPC_ERR_ARG,
                          "ipc_weight_update_noalloc: groups*M*K = %lld exceeds the static scratch limit %u "
                          "(IPC_NOALLOC_MAX_OUT_ELEMS); use ipc_fused_gemm_ws with a caller workspace",
                          elems, (unsigned)IPC_NOALLOC_MAX_OUT_ELEMS);
  int rc = ipc::require_sm100();
  if (rc) return rc;
  void* scratch = nullptr;
  rc = scratch_address(&scratch);
  if (rc) return rc;
  return ipc_fused_gemm_ws(mode, e, a_up, out, nullptr, nullptr, M, K, B, groups, alpha, flags, act, dtype, algo,
                           scratch, IPC_NOALLOC_SCRATCH_BYTES, stream);
}
