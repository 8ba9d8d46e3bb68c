#include "ipc_common.cuh"
#include "ipc_tc.cuh"

namespace ipc {
bool tc_eligible(int, int, int, int, int, int) { return false; }
int launch_tc(const GemmArgs&, int, bool, int, int, cudaStream_t) {
  return set_error(IPC_ERR_UNSUPPORTED, "tcgen05 path not built");
}
}  // namespace ipc
