// common.cuh — shared device helpers and the internal parameter blocks that
// the C ABI (abi.cu) hands to the kernel launchers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "bozo_block_ops.h"
#include "bozo_graph_bias.h"
#include "bozo_tau_aux.h"
#include "bozo_tension.h"

namespace bozo {

constexpr float kMassEps = 1e-6f;  // model.py:227/257/281 clamp(min=1e-6)

struct DevT4 {
  const void* p;
  int dt;
  long long sb, st, sh, sd;
};

inline DevT4 dev_t4(const bozo_tensor4& t) {
  return DevT4{t.ptr, t.dtype, t.stride[0], t.stride[1], t.stride[2], t.stride[3]};
}

// Everything a forward kernel needs, in device-friendly form.
struct FwdP {
  int B, T, H, HD, mode, W, norm;
  float scale, inv_scale;
  const float* cos;
  const float* sin;    // NULL when no RoPE
  const float* theta;  // [HD/2] frequencies of cos/sin, NULL if not supplied
  DevT4 q, k, v;
  const float* bias;
  long long bs0, bs1, bs2;
  void* out;
  int out_dt;
  void* tau;
  int tau_dt;
  float* row_mass;
  void* q_rot;  // optional rotated copies (dtype of q / k)
  void* k_rot;
  void* q_lp;   // bf16 operand copies of fp32 q / k (tensor-core path)
  void* k_lp;
  int* err;  // device error word
};

struct BwdP {
  int B, T, H, HD, mode, W, norm;
  float scale, inv_scale;
  const float* cos;
  const float* sin;
  const float* theta;
  DevT4 q, k, v, dout, out;
  const float* row_mass;
  const float* bias;
  long long bs0, bs1, bs2;
  const void* dtau;
  int dtau_dt;
  void* dq;
  void* dk;
  void* dv;
  int dq_dt, dk_dt, dv_dt;
  float* alpha;  // [B,H,T] workspace (CUDA-core path)
  float* beta;   // [B,H,T] workspace
  float* coef;   // [3][B·H, Tpad] workspace (tensor-core path)
  void* dout_lp;  // workspace room for a bf16 copy of an fp32 dO (tensor-core path) or null
  void* ds_scratch;  // key-tile path: dSᵀ tiles stored by DKV for the dQ pass, or null
  int qk_rotated;  // q, k are RoPE-rotated already
  const float* aux_row;  // [3][B·H·T] per-row τ cotangent (a1, a0, inv_d) or null
  int* err;
};

__device__ __forceinline__ float ldf(const void* p, long long i, int dt) {
  if (dt == BOZO_DT_F32) return static_cast<const float*>(p)[i];
  if (dt == BOZO_DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void stf(void* p, long long i, int dt, float v) {
  if (dt == BOZO_DT_F32) {
    static_cast<float*>(p)[i] = v;
  } else if (dt == BOZO_DT_BF16) {
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half*>(p)[i] = __float2half_rn(v);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Exact logistic sigmoid in fp32 (the CUDA-core path's definition).
__device__ __forceinline__ float sigmoid_exact(float x) { return 1.0f / (1.0f + expf(-x)); }

// Launchers (simt.cu)
cudaError_t launch_simt_fwd(const FwdP& p, cudaStream_t st, int* launches);
cudaError_t launch_simt_bwd(const BwdP& p, cudaStream_t st, int* launches);
// Write RoPE(q), RoPE(k) into p.q_rot / p.k_rot (dtype of q / k).
cudaError_t launch_rope_copy(const FwdP& p, cudaStream_t st, int* launches);
// fp32 (any strides) → contiguous bf16 [B,T,H,HD] copy (convert.cu)
cudaError_t launch_to_bf16(const DevT4& src, int B, int T, int H, int HD, void* dst, int sms,
                           cudaStream_t st);

// One decode step (decode.cu): the new token's projections against ring
// caches [B, C, H, HD] of rotated keys and values.
struct DecodeP {
  int B, H, HD, mode, W, norm, C, tw, rope_len;
  float inv_scale;
  const int* pos;  // device: absolute position t of the new token
  const float* cos;
  const float* sin;
  DevT4 q, k, v;   // [B, ·, H, HD] views (T stride unused)
  void* kc;
  int kc_dt;
  void* vc;
  int vc_dt;
  void* out;
  int out_dt;
  void* tau;
  int tau_dt;
  int* err;
};
size_t decode_smem_bytes(const DecodeP& p);
cudaError_t launch_decode(const DecodeP& p, cudaStream_t st);

// Fused add + RMSNorm and SwiGLU (norm.cu).
struct NormP {
  long long N;
  int D;
  float eps;
  int sms;
  const void* x;
  int x_dt;
  const void* y;
  int y_dt;
  const void* scale;
  void* out;
  float* rstd;
  const void* dout;
  void* dx;
  void* dy;
  void* dscale;
  float* part;  // backward: [blocks][D] partial sums of dscale
  void* out_lp;         // forward: bf16 copy of out, or null (fp32 x only)
  const void* dout_lp;  // backward: bf16 cotangent of out_lp, or null
};
int norm_partial_blocks(long long N, int sms);
bool norm_width_ok(int D);
cudaError_t launch_add_rmsnorm(const NormP& p, bool backward, cudaStream_t st);
// wo projection + residual add + RMSNorm, forward (wo_norm.cu): cluster size
// for a width (0 = unsupported) and the launch
int wo_norm_cluster(int width, bool x_bf16);
cudaError_t launch_wo_norm(const bozo_wo_add_rmsnorm_args& a, int* err, cudaStream_t st);
// width 0: flat tensors; else g/v/dg/dv rows of `width` elements `stride` apart
cudaError_t launch_swiglu(const void* g, const void* v, void* h, const void* dh, void* dg, void* dv,
                          long long n, int width, long long stride, int dt, int sms, cudaStream_t st);

// Token-embedding weight gradient (embed.cu).
cudaError_t launch_embedding_bwd(const bozo_embedding_bwd_args& a, int sms, cudaStream_t st);

// Cross-entropy from the logits (xent.cu).
bool xent_shape_ok(int V, int dt);
cudaError_t launch_xent(const bozo_cross_entropy_args& a, bool backward, cudaStream_t st);

// Graph bias on the device (graph_bias.cu).
cudaError_t launch_graph_bias(const bozo_graph_bias_args& a, int sms, cudaStream_t st);

// Fused τ-field consumer (tau_aux.cu).  Shape of one call's fields and the
// consistency extents: m = min(W−2, 4) slots (0: the layer is skipped),
// t_out queries per slot.
// Unsigned 32-bit division by an invariant divisor as a multiply-high and
// two shifts (Granlund & Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, Fig. 4.1): l = ⌈log2 d⌉,
// m = ⌊2^32·(2^l − d)/d⌋ + 1, q = (t + ((n − t) >> min(l,1))) >> max(l−1,0)
// with t = mulhi(m, n); exact for every 32-bit n.
struct FastDiv {
  uint32_t m, s1, s2;
};
inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
  return FastDiv{(uint32_t)m, l < 1 ? l : 1u, l > 1 ? l - 1 : 0u};
}
__device__ __forceinline__ uint32_t fast_div(uint32_t n, FastDiv f) {
  const uint32_t t = __umulhi(f.m, n);
  return (t + ((n - t) >> f.s1)) >> f.s2;
}

struct AuxShape {
  int B, T, H, W;
  long long N;  // rows B·T·H (< 2^31)
  int m, t_out;
  float inv_n, inv_w, inv_cons;
  FastDiv div_h, div_t;  // row → (b·T + t) → b
};
AuxShape aux_shape(int B, int T, int H, int W);
int aux_blocks(const AuxShape& s, int n_layers, int sms);
cudaError_t launch_tau_aux_fwd(const bozo_tau_aux_fwd_args& a, int nblk, float* partial,
                               cudaStream_t st);
cudaError_t launch_tau_aux_bwd(const bozo_tau_aux_bwd_args& a, int nblk, cudaStream_t st);
bool tau_aux_row_mode_ok(const bozo_tau_aux_bwd_args& a);

}  // namespace bozo
