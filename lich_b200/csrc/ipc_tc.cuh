// tcgen05 / TMEM / TMA tensor-core path of the fused P / I / W GEMMs.
#pragma once
#include "ipc_generic.cuh"

namespace ipc {
// True when the tensor-core kernel serves this request (16-bit storage,
// TMA-aligned shapes, large enough to fill 128-row tiles).
bool tc_eligible(int mode, int M, int K, int B, int dtype, int algo);
int launch_tc(const GemmArgs& p, int mode, bool bact, int act, int dtype, cudaStream_t s);
}  // namespace ipc
