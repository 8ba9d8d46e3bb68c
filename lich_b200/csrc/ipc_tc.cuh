// tcgen05 / TMEM / TMA tensor-core path of the fused P / I / W / forward GEMMs.
#pragma once
#include "ipc_generic.cuh"

namespace ipc {
// True when the tensor-core kernel serves this request: 16-bit storage, inner
// dimensions multiples of 8, no activation to apply to the B operand, and (for
// IPC_ALGO_AUTO) large enough to fill 128 x 256 tiles.
bool tc_eligible(int mode, int M, int K, int B, int dtype, int algo, bool b_activated);
int launch_tc(const GemmArgs& p, int mode, int act, int dtype, cudaStream_t s);
// Device status word written by bounded waits (0 = fine); clear != 0 resets it.
int read_device_status(int* status, int clear);
}  // namespace ipc
