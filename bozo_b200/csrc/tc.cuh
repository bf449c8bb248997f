// tc.cuh — entry points of the tcgen05 / TMA / TMEM kernels (sm_100a).
#pragma once
#include "common.cuh"

namespace bozo {

// True when the forward arguments qualify for the tensor-core kernel.
bool tc_fwd_eligible(const FwdP& p);
cudaError_t launch_tc_fwd(const FwdP& p, cudaStream_t st, int* launches);

bool tc_bwd_eligible(const BwdP& p);
cudaError_t launch_tc_bwd(const BwdP& p, cudaStream_t st, int* launches);

// Backward coefficient pre-pass: α/2, α·c, β·c (c = 1/(4·scale)) per query row
// into three padded planes [B·H, tpad] at coef (tc_bwd.cu).
cudaError_t launch_alpha_beta(const BwdP& p, int tpad, float ds_scale, float* coef,
                              cudaStream_t st);

// Global full-causal block (tc_global.cu).
bool tc_global_fwd_eligible(const FwdP& p);
cudaError_t launch_tc_global_fwd(const FwdP& p, cudaStream_t st, int* launches);
bool tc_global_bwd_eligible(const BwdP& p);
cudaError_t launch_tc_global_bwd(const BwdP& p, cudaStream_t st, int* launches);
// Bytes of the dSᵀ scratch that lets the key-tile backward skip recomputing
// S and dP for dQ (0 when the key-tile kernels do not serve the shape).
size_t tc_global_ds_bytes(int B, int T, int H, int mode, int W);

// Bounded-wait self-test kernel (wait_selftest.cu): one wait on an mbarrier
// nothing arrives on, limited to limit_ns; result (device int[4] or null).
cudaError_t launch_wait_selftest(uint64_t limit_ns, int* err, int* result, cudaStream_t st);

}  // namespace bozo
