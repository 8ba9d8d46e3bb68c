// tcgen05 / TMEM / TMA tensor-core path of the fused P / I / W / forward GEMMs.
#pragma once
#include "ipc_generic.cuh"

namespace ipc {
// True when the tensor-core kernel serves this request: 16-bit storage, inner
// dimensions multiples of 8, no activation to apply to the B operand, and (for
// IPC_ALGO_AUTO) large enough to fill 128 x 256 tiles.
// splitk: an fp32 workspace is available, so a weight update whose batch
// reduction is long and whose output has few tiles may be split over the SMs.
bool tc_eligible(int mode, int M, int K, int B, int dtype, int algo, bool b_activated, bool splitk = false);
// Per-call overrides of the kernel's launch heuristics (0 = the heuristic's choice); ipc_gemm_tune_t.
struct TcTune {
  int bn;        // output tile width: 128 or 256
  int splits;    // weight modes: 1 = no split-K, >= 2 = that many batch ranges (bounded by the workspace)
  int raster;    // M-tiles per raster band of the persistent tile walk
  int max_ctas;  // persistent CTAs (further bounded by ipc_set_max_ctas and the SM count)
  int pair;      // 2: CTA pairs (cta_group::2, 256 x 256 tiles); 0 / 1: single CTAs
};
// ws / ws_bytes: optional fp32 workspace for split-K partial tiles (weight modes).
int launch_tc(const GemmArgs& p, int mode, int act, int dtype, cudaStream_t s, float* ws = nullptr,
              size_t ws_bytes = 0, const TcTune* tune = nullptr);
// Cap on the CTAs of a persistent tensor-core launch (0 = one per SM); see ipc_set_max_ctas.
int set_max_ctas(int max_ctas);
// Device status word written by bounded waits (0 = fine); clear != 0 resets it.
int read_device_status(int* status, int clear);
// The same for the bounded grid barriers of the wide small-batch step kernel (ipc_widenet.cu).
int read_wide_status(int* status, int clear);
// The same for the bounded mbarrier waits of the persistent cluster kernel (ipc_net.cu).
int read_net_status(int* status, int clear);
// Launch the barrier-timeout self-test (ipc_widenet.cu).
int wide_selftest_timeout(void* sync, int limit_us, cudaStream_t s);
}  // namespace ipc
