// 4-bit MatMulNBits prefill GEMM on sm_100a tcgen05 tensor cores (in progress: not yet
// selected by the planner; prefill rows run the generic kernel until it is enabled).
#include "mmnb_common.cuh"

namespace xrgpu {

bool gemm_supported(const Problem&) { return false; }
uint64_t gemm_workspace_bytes(const Problem&) { return 0; }
cudaError_t launch_gemm(const Problem&, void*, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace xrgpu
