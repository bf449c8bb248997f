// tc_stub.cu — placeholder until the tcgen05 kernels land: nothing is eligible.
#include "tc.cuh"

namespace bozo {
bool tc_fwd_eligible(const FwdP&) { return false; }
cudaError_t launch_tc_fwd(const FwdP&, cudaStream_t, int*) { return cudaErrorNotSupported; }
bool tc_bwd_eligible(const BwdP&) { return false; }
cudaError_t launch_tc_bwd(const BwdP&, cudaStream_t, int*) { return cudaErrorNotSupported; }
}  // namespace bozo
