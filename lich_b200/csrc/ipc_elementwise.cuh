#pragma once
#include <cuda_runtime.h>

#include "ipc_generic.cuh"

namespace ipc {
// opt (may be null): an optimizer step instead of W += alpha * acc (non-delta updates only).
int launch_outer(void* out, const void* e, const void* x, int M, int K, int B, int groups, float alpha,
                 bool bact, bool delta, int accumulate, int act, int dtype, cudaStream_t s,
                 const OptParams* opt = nullptr);
int launch_opt_apply(void* w, const float* dw, long long n, int dtype, const OptParams& opt, cudaStream_t s);
int launch_activate(void* a, const void* x, long long n, int act, int dtype, cudaStream_t s);
int launch_apply(void* w, const float* dw, long long n, int dtype, cudaStream_t s);
int launch_count_correct(const void* logits, int C, int B, const long long* labels, int* count, int dtype,
                         cudaStream_t s);
}  // namespace ipc
