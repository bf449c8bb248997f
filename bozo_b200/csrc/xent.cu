// xent.cu — cross-entropy over the vocabulary (the training loss of
// train.py:920, nn.CrossEntropyLoss: mean over rows whose target is not
// −100) computed straight from the bf16 (or fp32) logits: the forward reads
// each row once for its logsumexp and the target's logit, the backward reads
// it once more and writes (softmax − onehot)·g in the logits' dtype.  The
// framework path under autocast instead makes an fp32 copy of the logits,
// a log-softmax of it, and casts the gradient back — several passes over
// [rows, vocab].
//
// One 256-thread block per row; each thread keeps an online (max, Σ exp)
// pair over its 16-byte vectors (exp as exp2f of the log2e-scaled
// difference), combined across the block with shuffles and shared memory.
#include <cuda_bf16.h>

#include "bozo_block_ops.h"
#include "common.cuh"

namespace bozo {
namespace {

constexpr int kXentThreads = 256;
constexpr float kLog2e = 1.44269504f;

template <typename T> struct XVec;
template <> struct XVec<float> { static constexpr int n = 4; };
template <> struct XVec<__nv_bfloat16> { static constexpr int n = 8; };

__device__ __forceinline__ void xload(const float* p, float* v) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
__device__ __forceinline__ void xload(const __nv_bfloat16* p, float* v) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void xstore(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void xstore(__nv_bfloat16* p, const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ float xf(float v) { return v; }
__device__ __forceinline__ float xf(__nv_bfloat16 v) { return __bfloat162float(v); }

// (m, s) ⊕ (m', s') = (max, s·2^{(m−max)log2e} + s'·2^{(m'−max)log2e})
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float mx = fmaxf(m, m2);
  if (mx == -INFINITY) return;
  s = s * exp2f((m - mx) * kLog2e) + s2 * exp2f((m2 - mx) * kLog2e);
  m = mx;
}

template <typename T>
__global__ void __launch_bounds__(kXentThreads)
    xent_fwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ targets, int V,
                    float* __restrict__ row_lse, float* __restrict__ row_loss) {
  constexpr int NV = XVec<T>::n;
  const long long r = blockIdx.x;
  const T* row = logits + r * V;
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x * NV; i < V; i += kXentThreads * NV) {
    float x[NV];
    xload(row + i, x);
    float vm = x[0];
#pragma unroll
    for (int k = 1; k < NV; ++k) vm = fmaxf(vm, x[k]);
    float vs = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) vs += exp2f((x[k] - vm) * kLog2e);
    lse_merge(m, s, vm, vs);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
  }
  __shared__ float sm[kXentThreads / 32], ss[kXentThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss[0];
    for (int w = 1; w < kXentThreads / 32; ++w) lse_merge(M, S, sm[w], ss[w]);
    const float lse = M + logf(S);
    row_lse[r] = lse;
    const int64_t t = targets[r];
    row_loss[r] = (t >= 0 && t < V) ? lse - xf(row[t]) : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(kXentThreads)
    xent_bwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ targets, int V,
                    const float* __restrict__ row_lse, const float* __restrict__ g_ptr,
                    T* __restrict__ d_logits) {
  constexpr int NV = XVec<T>::n;
  const long long r = blockIdx.x;
  const T* row = logits + r * V;
  T* drow = d_logits + r * V;
  const int64_t t = targets[r];
  const bool live = t >= 0 && t < V;
  const float g = live ? __ldg(g_ptr) : 0.f;  // ignored rows get a zero gradient
  const float lse = row_lse[r];
  for (int i = threadIdx.x * NV; i < V; i += kXentThreads * NV) {
    float x[NV], d[NV];
    xload(row + i, x);
#pragma unroll
    for (int k = 0; k < NV; ++k) d[k] = (exp2f((x[k] - lse) * kLog2e) - (i + k == t ? 1.f : 0.f)) * g;
    xstore(drow + i, d);
  }
}

}  // namespace

bool xent_shape_ok(int V, int dt) {
  const int nv = dt == BOZO_DT_BF16 ? 8 : 4;
  return V > 0 && V % nv == 0;
}

cudaError_t launch_xent(const bozo_cross_entropy_args& a, bool backward, cudaStream_t st) {
  const dim3 grid((unsigned)a.rows);
  if (a.logits_dtype == BOZO_DT_BF16) {
    using T = __nv_bfloat16;
    if (backward)
      xent_bwd_kernel<T><<<grid, kXentThreads, 0, st>>>(static_cast<const T*>(a.logits), a.targets, a.vocab,
                                                        a.row_lse, a.d_scale, static_cast<T*>(a.d_logits));
    else
      xent_fwd_kernel<T><<<grid, kXentThreads, 0, st>>>(static_cast<const T*>(a.logits), a.targets, a.vocab,
                                                        a.row_lse, a.row_loss);
  } else {
    if (backward)
      xent_bwd_kernel<float><<<grid, kXentThreads, 0, st>>>(static_cast<const float*>(a.logits), a.targets,
                                                            a.vocab, a.row_lse, a.d_scale,
                                                            static_cast<float*>(a.d_logits));
    else
      xent_fwd_kernel<float><<<grid, kXentThreads, 0, st>>>(static_cast<const float*>(a.logits), a.targets,
                                                            a.vocab, a.row_lse, a.row_loss);
  }
  return cudaGetLastError();
}

}  // namespace bozo
