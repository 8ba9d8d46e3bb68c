#pragma once
#include <cuda_runtime.h>

namespace ipc {
int launch_outer(void* out, const void* e, const void* x, int M, int K, int B, int groups, float alpha,
                 bool bact, bool delta, int accumulate, int act, int dtype, cudaStream_t s);
int launch_activate(void* a, const void* x, long long n, int act, int dtype, cudaStream_t s);
int launch_apply(void* w, const float* dw, long long n, int dtype, cudaStream_t s);
}  // namespace ipc
