// tc.cuh — entry points of the tcgen05 / TMA / TMEM kernels (sm_100a).
#pragma once
#include "common.cuh"

namespace bozo {

// True when the forward arguments qualify for the tensor-core kernel.
bool tc_fwd_eligible(const FwdP& p);
cudaError_t launch_tc_fwd(const FwdP& p, cudaStream_t st, int* launches);

bool tc_bwd_eligible(const BwdP& p);
cudaError_t launch_tc_bwd(const BwdP& p, cudaStream_t st, int* launches);

}  // namespace bozo
