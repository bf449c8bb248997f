// torch_ext.cpp — PyTorch C++ extension over the C ABI (include/bozo_tension.h).
//
// The autograd functions in bozo_b200/ops.py call these two entry points for
// every forward / backward.  They fill the ABI argument blocks straight from
// at::Tensor metadata, allocate the outputs (and the backward's coefficient
// workspace) with the caching allocator on the tensors' device, and launch on
// the caller's current stream — the same work the reference's
// _CausalTensionFn.forward/backward do around their Triton launches
// (triton_tension/ops.py:75-124, 126-187), in C++ so a call costs a few
// microseconds of host time instead of a Python-level struct build.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "bozo_block_ops.h"
#include "bozo_graph_bias.h"
#include "bozo_tau_aux.h"
#include "bozo_tension.h"

namespace {

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return BOZO_DT_F32;
    case at::kBFloat16: return BOZO_DT_BF16;
    case at::kHalf: return BOZO_DT_F16;
    default:
      throw pybind11::type_error(std::string("bozo tension: unsupported dtype ") +
                                  c10::toString(t) +
                                  " (float32, bfloat16 and float16 are supported)");
  }
}

at::ScalarType scalar_type(int64_t code) {
  switch (code) {
    case BOZO_DT_F32: return at::kFloat;
    case BOZO_DT_BF16: return at::kBFloat16;
    case BOZO_DT_F16: return at::kHalf;
    default: throw pybind11::type_error("bozo tension: bad dtype code");
  }
}

bozo_tensor4 t4(const at::Tensor& t) {
  bozo_tensor4 s{};
  if (!t.defined()) return s;
  s.ptr = t.data_ptr();
  s.dtype = dtype_code(t.scalar_type());
  for (int i = 0; i < 4; ++i) s.stride[i] = t.stride(i);
  return s;
}

void check(int status, const char* what) {
  if (status == BOZO_OK) return;
  std::string msg = std::string(what) + " failed: " + bozo_status_string(status) +
                    " (status " + std::to_string(status) + ")";
  if (status == BOZO_ERR_CUDA) msg += std::string(" [") + bozo_tension_last_cuda_error() + "]";
  throw std::runtime_error(msg);
}

template <typename A>
void fill_common(A& a, const at::Tensor& q, int64_t mode, int64_t window, int64_t norm,
                 double scale, int64_t path, const c10::optional<at::Tensor>& cos,
                 const c10::optional<at::Tensor>& sin, const c10::optional<at::Tensor>& theta) {
  a.B = (int32_t)q.size(0);
  a.T = (int32_t)q.size(1);
  a.H = (int32_t)q.size(2);
  a.HD = (int32_t)q.size(3);
  a.mode = (int32_t)mode;
  a.window = (int32_t)window;
  a.normalize = (int32_t)norm;
  a.path = (int32_t)path;
  a.scale = (float)scale;
  if (cos && cos->defined()) {
    a.rope_len = (int32_t)cos->size(0);
    a.rope_cos = cos->data_ptr<float>();
    a.rope_sin = sin->data_ptr<float>();
    a.rope_theta = (theta && theta->defined()) ? theta->data_ptr<float>() : nullptr;
  }
}

void fill_bias(const c10::optional<at::Tensor>& bias, const float** ptr, int64_t* stride) {
  if (bias && bias->defined()) {
    *ptr = bias->data_ptr<float>();
    for (int i = 0; i < 3; ++i) stride[i] = bias->stride(i);
  }
}

// Returns [out, tau, row_mass, q_rot, k_rot, q_lp, k_lp]; absent ones are
// None.  With want_lp, fp32 q/k get bf16 operand copies (q_lp, k_lp): the
// tensor-core kernels compute from them when the call qualifies, and the
// backward takes them as its q/k in every case.
std::vector<at::Tensor> tension_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                    int64_t mode, int64_t window, int64_t norm, double scale,
                                    int64_t path, const c10::optional<at::Tensor>& cos,
                                    const c10::optional<at::Tensor>& sin,
                                    const c10::optional<at::Tensor>& theta,
                                    const c10::optional<at::Tensor>& bias, int64_t tau_width,
                                    int64_t out_dtype, int64_t tau_dtype, bool want_mass,
                                    bool want_rotated, bool want_lp) {
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t B = q.size(0), T = q.size(1), H = q.size(2), HD = q.size(3);
  auto opts = q.options();
  at::Tensor out = at::empty({B, T, H, HD}, opts.dtype(scalar_type(out_dtype)));
  at::Tensor tau, mass, q_rot, k_rot;
  if (tau_width > 0) tau = at::empty({B, T, H, tau_width}, opts.dtype(scalar_type(tau_dtype)));
  if (want_mass) mass = at::empty({B, H, T}, opts.dtype(at::kFloat));
  if (want_rotated && cos && cos->defined()) {
    q_rot = at::empty({B, T, H, HD}, opts);
    k_rot = at::empty({B, T, H, HD}, k.options());
  }
  bozo_tension_fwd_args a{};
  fill_common(a, q, mode, window, norm, scale, path, cos, sin, theta);
  a.q = t4(q);
  a.k = t4(k);
  a.v = t4(v);
  fill_bias(bias, &a.bias, a.bias_stride);
  a.out = out.data_ptr();
  a.out_dtype = (int32_t)out_dtype;
  if (tau.defined()) {
    a.tau = tau.data_ptr();
    a.tau_dtype = (int32_t)tau_dtype;
  }
  if (mass.defined()) a.row_mass = mass.data_ptr<float>();
  if (q_rot.defined()) {
    a.q_rot = q_rot.data_ptr();
    a.k_rot = k_rot.data_ptr();
  }
  at::Tensor q_lp, k_lp;
  if (want_lp && q.scalar_type() == at::kFloat && k.scalar_type() == at::kFloat) {
    q_lp = at::empty({B, T, H, HD}, opts.dtype(at::kBFloat16));
    k_lp = at::empty({B, T, H, HD}, opts.dtype(at::kBFloat16));
    a.q_lp = q_lp.data_ptr();
    a.k_lp = k_lp.data_ptr();
  }
  check(bozo_tension_fwd(&a, at::cuda::getCurrentCUDAStream(q.device().index()).stream()),
        "bozo_tension_fwd");
  return {out, tau, mass, q_rot, k_rot, q_lp, k_lp};
}

// Returns [dq, dk, dv] in the dtypes of q, k, v.
std::vector<at::Tensor> tension_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                    const at::Tensor& d_out, int64_t mode, int64_t window,
                                    int64_t norm, double scale, int64_t path,
                                    const c10::optional<at::Tensor>& cos,
                                    const c10::optional<at::Tensor>& sin,
                                    const c10::optional<at::Tensor>& theta,
                                    const c10::optional<at::Tensor>& bias,
                                    const c10::optional<at::Tensor>& out,
                                    const c10::optional<at::Tensor>& mass,
                                    const c10::optional<at::Tensor>& d_tau, bool qk_rotated,
                                    const c10::optional<at::Tensor>& aux_row, int64_t dq_dtype,
                                    int64_t dk_dtype) {
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t B = q.size(0), T = q.size(1), H = q.size(2), HD = q.size(3);
  // gradient dtypes: q's and k's unless given (the bf16 operand copies of an
  // fp32 forward still owe fp32 gradients)
  at::Tensor dq = at::empty({B, T, H, HD}, dq_dtype >= 0 ? q.options().dtype(scalar_type(dq_dtype)) : q.options());
  at::Tensor dk = at::empty({B, T, H, HD}, dk_dtype >= 0 ? k.options().dtype(scalar_type(dk_dtype)) : k.options());
  at::Tensor dv = at::empty({B, T, H, HD}, v.options());
  bozo_tension_bwd_args a{};
  fill_common(a, q, mode, window, norm, scale, path, cos, sin, theta);
  a.q = t4(q);
  a.k = t4(k);
  a.v = t4(v);
  a.d_out = t4(d_out);
  if (out && out->defined()) a.out = t4(*out);
  if (mass && mass->defined()) a.row_mass = mass->data_ptr<float>();
  fill_bias(bias, &a.bias, a.bias_stride);
  if (d_tau && d_tau->defined()) {
    a.d_tau = d_tau->data_ptr();
    a.d_tau_dtype = dtype_code(d_tau->scalar_type());
  }
  a.grad_dtype[0] = dtype_code(dq.scalar_type());
  a.grad_dtype[1] = dtype_code(dk.scalar_type());
  a.grad_dtype[2] = dtype_code(v.scalar_type());
  a.qk_rotated = qk_rotated ? 1 : 0;
  if (aux_row && aux_row->defined()) {
    if (aux_row->scalar_type() != at::kFloat || !aux_row->is_contiguous() ||
        aux_row->numel() != 3 * B * T * H)
      throw std::invalid_argument("tension_bwd: aux_row must be a contiguous fp32 [3, B·H·T] tensor");
    a.aux_row = aux_row->data_ptr<float>();
  }
  a.dq = dq.data_ptr();
  a.dk = dk.data_ptr();
  a.dv = dv.data_ptr();
  const size_t ws_bytes = bozo_tension_bwd_workspace(&a);
  at::Tensor ws;
  if (ws_bytes) {
    ws = at::empty({(int64_t)ws_bytes}, q.options().dtype(at::kByte));
    a.workspace = ws.data_ptr();
    a.workspace_bytes = ws_bytes;
  }
  check(bozo_tension_bwd(&a, at::cuda::getCurrentCUDAStream(q.device().index()).stream()),
        "bozo_tension_bwd");
  return {dq, dk, dv};
}

// One decode step (bozo_tension_decode): q, k, v are the new token's
// projections [B, H, HD] (any strides, unit HD stride not required); the ring
// caches [B, C, H, HD] are updated in place.  Returns [out, tau] (tau
// undefined unless tau_width > 0).
std::vector<at::Tensor> tension_decode(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                       const at::Tensor& k_cache, const at::Tensor& v_cache,
                                       const at::Tensor& pos, int64_t mode, int64_t window,
                                       int64_t norm, double scale,
                                       const c10::optional<at::Tensor>& cos,
                                       const c10::optional<at::Tensor>& sin, int64_t tau_width,
                                       int64_t out_dtype, int64_t tau_dtype) {
  const c10::cuda::CUDAGuard guard(q.device());
  if (q.dim() != 3 || k.dim() != 3 || v.dim() != 3)
    throw std::invalid_argument("tension_decode: q, k, v must be [B, H, HD]");
  if (k_cache.dim() != 4 || !k_cache.is_contiguous() || !v_cache.is_contiguous() ||
      v_cache.sizes() != k_cache.sizes())
    throw std::invalid_argument("tension_decode: caches must be contiguous [B, C, H, HD]");
  if (pos.scalar_type() != at::kInt || pos.numel() != 1 || !pos.is_cuda())
    throw std::invalid_argument("tension_decode: pos must be a one-element int32 CUDA tensor");
  const int64_t B = q.size(0), H = q.size(1), HD = q.size(2);
  at::Tensor out = at::empty({B, H, HD}, q.options().dtype(scalar_type(out_dtype)));
  at::Tensor tau;
  if (tau_width > 0) tau = at::empty({B, H, tau_width}, q.options().dtype(scalar_type(tau_dtype)));
  auto t4_3 = [](const at::Tensor& t) {
    bozo_tensor4 s{};
    s.ptr = t.data_ptr();
    s.dtype = dtype_code(t.scalar_type());
    s.stride[0] = t.stride(0);
    s.stride[1] = 0;
    s.stride[2] = t.stride(1);
    s.stride[3] = t.stride(2);
    return s;
  };
  bozo_tension_decode_args a{};
  a.B = (int32_t)B; a.H = (int32_t)H; a.HD = (int32_t)HD;
  a.mode = (int32_t)mode; a.window = (int32_t)window; a.normalize = (int32_t)norm;
  a.capacity = (int32_t)k_cache.size(1);
  a.tau_width = (int32_t)tau_width;
  a.scale = (float)scale;
  a.pos = pos.data_ptr<int32_t>();
  if (cos && cos->defined()) {
    a.rope_len = (int32_t)cos->size(0);
    a.rope_cos = cos->data_ptr<float>();
    a.rope_sin = sin->data_ptr<float>();
  }
  a.q = t4_3(q); a.k = t4_3(k); a.v = t4_3(v);
  a.k_cache = k_cache.data_ptr(); a.k_cache_dtype = dtype_code(k_cache.scalar_type());
  a.v_cache = v_cache.data_ptr(); a.v_cache_dtype = dtype_code(v_cache.scalar_type());
  a.out = out.data_ptr(); a.out_dtype = (int32_t)out_dtype;
  if (tau.defined()) {
    a.tau = tau.data_ptr();
    a.tau_dtype = (int32_t)tau_dtype;
  }
  check(bozo_tension_decode(&a, at::cuda::getCurrentCUDAStream(q.device().index()).stream()),
        "bozo_tension_decode");
  return {out, tau};
}

// Graph bias [T, W] (window > 0) or [T, T] (window 0) from the context's
// content ids and the sorted edge table; stats [3] (pairs, Σ weight, max)
// as float64.  Returns [bias, stats].
std::vector<at::Tensor> graph_bias(const at::Tensor& ctx_content, const at::Tensor& keys,
                                   const at::Tensor& weights, int64_t window, double alpha) {
  const c10::cuda::CUDAGuard guard(ctx_content.device());
  if (ctx_content.scalar_type() != at::kInt || ctx_content.dim() != 1 || !ctx_content.is_contiguous() ||
      keys.scalar_type() != at::kLong || weights.scalar_type() != at::kDouble ||
      keys.numel() != weights.numel() || !keys.is_contiguous() || !weights.is_contiguous())
    throw std::invalid_argument("graph_bias: int32 [T] content ids, int64 keys, float64 weights");
  const int64_t T = ctx_content.size(0);
  at::Tensor out = at::empty({T, window > 0 ? window : T}, ctx_content.options().dtype(at::kFloat));
  at::Tensor stats = at::zeros({3}, ctx_content.options().dtype(at::kDouble));
  bozo_graph_bias_args a{};
  a.T = (int32_t)T;
  a.window = (int32_t)window;
  a.alpha = alpha;
  a.ctx_content = ctx_content.data_ptr<int32_t>();
  a.n_edges = keys.numel();
  if (a.n_edges > 0) {
    a.edge_keys = reinterpret_cast<const uint64_t*>(keys.data_ptr<int64_t>());
    a.edge_weights = weights.data_ptr<double>();
  }
  a.out = out.data_ptr<float>();
  a.stats = stats.data_ptr<double>();
  check(bozo_graph_bias_build(&a, at::cuda::getCurrentCUDAStream(out.device().index()).stream()),
        "bozo_graph_bias_build");
  return {out, stats};
}

// add + RMSNorm forward: x [N, D] (+ y [N, D]) → (out [N, D] in x's dtype, rstd [N] fp32,
// and with want_lp a bf16 copy of out, else an undefined tensor).
std::vector<at::Tensor> add_rmsnorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& y,
                                        const at::Tensor& scale, double eps, bool want_lp) {
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor out = at::empty_like(x), out_lp;
  at::Tensor rstd = at::empty({x.size(0)}, x.options().dtype(at::kFloat));
  bozo_add_rmsnorm_args a{};
  if (want_lp) {
    out_lp = at::empty_like(x, x.options().dtype(at::kBFloat16));
    a.out_lp = out_lp.data_ptr();
  }
  a.rows = x.size(0); a.width = (int32_t)x.size(1); a.eps = (float)eps;
  a.x = x.data_ptr(); a.x_dtype = dtype_code(x.scalar_type());
  if (y && y->defined()) { a.y = y->data_ptr(); a.y_dtype = dtype_code(y->scalar_type()); }
  a.scale = scale.data_ptr(); a.out = out.data_ptr(); a.rstd = rstd.data_ptr<float>();
  check(bozo_add_rmsnorm_fwd(&a, at::cuda::getCurrentCUDAStream(x.device().index()).stream()),
        "bozo_add_rmsnorm_fwd");
  return {out, rstd, out_lp};
}

// add + RMSNorm backward → (dx, dy (undefined without y), dscale).
std::vector<at::Tensor> add_rmsnorm_bwd(const at::Tensor& d_out, const at::Tensor& x,
                                        const c10::optional<at::Tensor>& y, const at::Tensor& scale,
                                        const at::Tensor& rstd, const c10::optional<at::Tensor>& d_out_lp) {
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor dx = at::empty_like(x), dy, dscale = at::empty_like(scale);
  bozo_add_rmsnorm_args a{};
  if (d_out_lp && d_out_lp->defined()) a.d_out_lp = d_out_lp->data_ptr();
  a.rows = x.size(0); a.width = (int32_t)x.size(1);
  a.x = x.data_ptr(); a.x_dtype = dtype_code(x.scalar_type());
  if (y && y->defined()) {
    a.y = y->data_ptr(); a.y_dtype = dtype_code(y->scalar_type());
    dy = at::empty_like(*y);
    a.dy = dy.data_ptr();
  }
  a.scale = scale.data_ptr(); a.rstd = rstd.data_ptr<float>();
  a.d_out = d_out.data_ptr(); a.dx = dx.data_ptr(); a.d_scale = dscale.data_ptr();
  const size_t ws_bytes = bozo_add_rmsnorm_workspace(&a);
  at::Tensor ws = at::empty({(int64_t)std::max<size_t>(ws_bytes, 1)}, x.options().dtype(at::kByte));
  a.workspace = ws.data_ptr(); a.workspace_bytes = ws_bytes;
  check(bozo_add_rmsnorm_bwd(&a, at::cuda::getCurrentCUDAStream(x.device().index()).stream()),
        "bozo_add_rmsnorm_bwd");
  return {dx, dy, dscale};
}

// wo projection + residual add + RMSNorm forward: msg [N, D] bf16, wo [D, D] bf16,
// x [N, D] → (out [N, D] in x's dtype, rstd [N] fp32).
std::vector<at::Tensor> wo_add_rmsnorm_fwd(const at::Tensor& msg, const at::Tensor& wo,
                                           const at::Tensor& x, const at::Tensor& scale, double eps) {
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor out = at::empty_like(x);
  at::Tensor rstd = at::empty({x.size(0)}, x.options().dtype(at::kFloat));
  bozo_wo_add_rmsnorm_args a{};
  a.rows = x.size(0); a.width = (int32_t)x.size(1); a.eps = (float)eps;
  a.msg = msg.data_ptr(); a.wo = wo.data_ptr();
  a.x = x.data_ptr(); a.x_dtype = dtype_code(x.scalar_type());
  a.scale = scale.data_ptr(); a.out = out.data_ptr(); a.rstd = rstd.data_ptr<float>();
  TORCH_CHECK(msg.scalar_type() == at::kBFloat16 && wo.scalar_type() == at::kBFloat16,
              "wo_add_rmsnorm_fwd: msg and wo must be bf16");
  check(bozo_wo_add_rmsnorm_fwd(&a, at::cuda::getCurrentCUDAStream(x.device().index()).stream()),
        "bozo_wo_add_rmsnorm_fwd");
  return {out, rstd};
}

// SwiGLU over packed rows gv [N, 2F] = [gate | value] (one GEMM's output):
// forward → h [N, F]; backward → d_gv [N, 2F] in the same packed layout.
at::Tensor swiglu_packed_fwd(const at::Tensor& gv) {
  const c10::cuda::CUDAGuard guard(gv.device());
  const int64_t F = gv.size(1) / 2;
  at::Tensor h = at::empty({gv.size(0), F}, gv.options());
  bozo_swiglu_args a{};
  a.n = gv.size(0) * F; a.dtype = dtype_code(gv.scalar_type());
  a.width = F; a.row_stride = gv.stride(0);
  a.gate = gv.data_ptr();
  a.value = static_cast<char*>(gv.data_ptr()) + F * gv.element_size();
  a.out = h.data_ptr();
  check(bozo_swiglu_fwd(&a, at::cuda::getCurrentCUDAStream(gv.device().index()).stream()), "bozo_swiglu_fwd");
  return h;
}

at::Tensor swiglu_packed_bwd(const at::Tensor& dh, const at::Tensor& gv) {
  const c10::cuda::CUDAGuard guard(gv.device());
  const int64_t F = gv.size(1) / 2;
  at::Tensor dgv = at::empty({gv.size(0), 2 * F}, gv.options());
  bozo_swiglu_args a{};
  a.n = gv.size(0) * F; a.dtype = dtype_code(gv.scalar_type());
  a.width = F; a.row_stride = gv.stride(0);
  a.gate = gv.data_ptr();
  a.value = static_cast<char*>(gv.data_ptr()) + F * gv.element_size();
  a.d_out = dh.data_ptr();
  a.d_gate = dgv.data_ptr();
  a.d_value = static_cast<char*>(dgv.data_ptr()) + F * dgv.element_size();
  TORCH_CHECK(dgv.stride(0) == gv.stride(0), "swiglu_packed_bwd: gv must be contiguous");
  check(bozo_swiglu_bwd(&a, at::cuda::getCurrentCUDAStream(gv.device().index()).stream()), "bozo_swiglu_bwd");
  return dgv;
}

at::Tensor swiglu_fwd(const at::Tensor& g, const at::Tensor& v) {
  const c10::cuda::CUDAGuard guard(g.device());
  at::Tensor h = at::empty_like(g);
  bozo_swiglu_args a{};
  a.n = g.numel(); a.dtype = dtype_code(g.scalar_type());
  a.gate = g.data_ptr(); a.value = v.data_ptr(); a.out = h.data_ptr();
  check(bozo_swiglu_fwd(&a, at::cuda::getCurrentCUDAStream(g.device().index()).stream()), "bozo_swiglu_fwd");
  return h;
}

std::vector<at::Tensor> swiglu_bwd(const at::Tensor& dh, const at::Tensor& g, const at::Tensor& v) {
  const c10::cuda::CUDAGuard guard(g.device());
  at::Tensor dg = at::empty_like(g), dv = at::empty_like(v);
  bozo_swiglu_args a{};
  a.n = g.numel(); a.dtype = dtype_code(g.scalar_type());
  a.gate = g.data_ptr(); a.value = v.data_ptr(); a.d_out = dh.data_ptr();
  a.d_gate = dg.data_ptr(); a.d_value = dv.data_ptr();
  check(bozo_swiglu_bwd(&a, at::cuda::getCurrentCUDAStream(g.device().index()).stream()), "bozo_swiglu_bwd");
  return {dg, dv};
}

// Token-embedding weight gradient from the stably sorted ids (int32) and
// their positions (int64): [vocab, dim] fp32, every row written.
at::Tensor embedding_bwd(const at::Tensor& sorted_ids, const at::Tensor& order, const at::Tensor& d_out,
                         int64_t vocab) {
  const c10::cuda::CUDAGuard guard(d_out.device());
  TORCH_CHECK(sorted_ids.scalar_type() == at::kInt && order.scalar_type() == at::kLong,
              "embedding_bwd: int32 keys and int64 positions");
  TORCH_CHECK(d_out.scalar_type() == at::kFloat && d_out.dim() == 2 && d_out.is_contiguous(),
              "embedding_bwd: d_out must be contiguous fp32 [n, dim]");
  TORCH_CHECK(sorted_ids.is_contiguous() && order.is_contiguous() && sorted_ids.numel() == d_out.size(0) &&
              order.numel() == d_out.size(0), "embedding_bwd: one key and one position per d_out row");
  at::Tensor dw = at::empty({vocab, d_out.size(1)}, d_out.options());
  at::Tensor scratch = at::empty({2 * vocab}, d_out.options().dtype(at::kInt));
  bozo_embedding_bwd_args a{};
  a.n = d_out.size(0); a.dim = (int32_t)d_out.size(1); a.vocab = (int32_t)vocab;
  a.sorted_ids = sorted_ids.data_ptr<int32_t>(); a.order = order.data_ptr<int64_t>();
  a.d_out = d_out.data_ptr<float>(); a.d_weight = dw.data_ptr<float>();
  a.scratch = scratch.data_ptr<int32_t>();
  check(bozo_embedding_bwd(&a, at::cuda::getCurrentCUDAStream(d_out.device().index()).stream()),
        "bozo_embedding_bwd");
  return dw;
}

// Cross-entropy: forward → (row_loss, row_lse); backward → d_logits.
std::vector<at::Tensor> cross_entropy_fwd(const at::Tensor& logits, const at::Tensor& targets) {
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t R = logits.size(0);
  at::Tensor loss = at::empty({R}, logits.options().dtype(at::kFloat));
  at::Tensor lse = at::empty({R}, logits.options().dtype(at::kFloat));
  bozo_cross_entropy_args a{};
  a.rows = R; a.vocab = (int32_t)logits.size(1);
  a.logits = logits.data_ptr(); a.logits_dtype = dtype_code(logits.scalar_type());
  a.targets = targets.data_ptr<int64_t>(); a.row_lse = lse.data_ptr<float>();
  a.row_loss = loss.data_ptr<float>();
  check(bozo_cross_entropy_fwd(&a, at::cuda::getCurrentCUDAStream(logits.device().index()).stream()),
        "bozo_cross_entropy_fwd");
  return {loss, lse};
}

at::Tensor cross_entropy_bwd(const at::Tensor& logits, const at::Tensor& targets, const at::Tensor& lse,
                             const at::Tensor& g) {
  const c10::cuda::CUDAGuard guard(logits.device());
  at::Tensor d = at::empty_like(logits);
  bozo_cross_entropy_args a{};
  a.rows = logits.size(0); a.vocab = (int32_t)logits.size(1);
  a.logits = logits.data_ptr(); a.logits_dtype = dtype_code(logits.scalar_type());
  a.targets = targets.data_ptr<int64_t>(); a.row_lse = lse.data_ptr<float>();
  a.d_scale = g.data_ptr<float>(); a.d_logits = d.data_ptr();
  check(bozo_cross_entropy_bwd(&a, at::cuda::getCurrentCUDAStream(logits.device().index()).stream()),
        "bozo_cross_entropy_bwd");
  return d;
}

// τ fields of one τ-consumer call: same shape, dtype and device, contiguous.
void check_fields(const std::vector<at::Tensor>& taus) {
  if (taus.empty()) throw std::invalid_argument("tau_aux: no τ fields");
  const at::Tensor& t0 = taus[0];
  for (const auto& t : taus) {
    if (!t.is_cuda()) throw std::invalid_argument("tau_aux: τ fields must be CUDA tensors");
    if (t.dim() != 4 || t.sizes() != t0.sizes() || t.scalar_type() != t0.scalar_type() ||
        t.device() != t0.device())
      throw std::invalid_argument("tau_aux: τ fields must share one [B,T,H,W] shape, dtype and device");
    if (!t.is_contiguous()) throw std::invalid_argument("tau_aux: τ fields must be contiguous");
  }
}

template <typename A>
void fill_aux(A& a, const std::vector<at::Tensor>& taus, size_t i0, size_t n) {
  const at::Tensor& t0 = taus[0];
  a.n_layers = (int32_t)n;
  a.dtype = dtype_code(t0.scalar_type());
  a.B = (int32_t)t0.size(0);
  a.T = (int32_t)t0.size(1);
  a.H = (int32_t)t0.size(2);
  a.W = (int32_t)t0.size(3);
  for (size_t i = 0; i < n; ++i) a.tau[i] = taus[i0 + i].data_ptr();
}

// Per-layer statistics [L, 3] fp32 of the τ fields (bozo_tau_aux_fwd), in
// chunks of BOZO_TAU_AUX_MAX_LAYERS fields.
at::Tensor tau_aux_fwd(const std::vector<at::Tensor>& taus) {
  check_fields(taus);
  const c10::cuda::CUDAGuard guard(taus[0].device());
  const auto stream = at::cuda::getCurrentCUDAStream(taus[0].device().index()).stream();
  const int64_t L = (int64_t)taus.size();
  at::Tensor stats = at::empty({L, 3}, taus[0].options().dtype(at::kFloat));
  for (size_t i0 = 0; i0 < taus.size(); i0 += BOZO_TAU_AUX_MAX_LAYERS) {
    const size_t n = std::min<size_t>(BOZO_TAU_AUX_MAX_LAYERS, taus.size() - i0);
    bozo_tau_aux_fwd_args a{};
    fill_aux(a, taus, i0, n);
    a.stats = stats.data_ptr<float>() + 3 * i0;
    const size_t ws_bytes = bozo_tau_aux_workspace(&a);
    at::Tensor ws = at::empty({(int64_t)std::max<size_t>(ws_bytes, 1)},
                              taus[0].options().dtype(at::kByte));
    a.workspace = ws.data_ptr();
    a.workspace_bytes = ws_bytes;
    check(bozo_tau_aux_fwd(&a, stream), "bozo_tau_aux_fwd");
  }
  return stats;
}

// Per-row entropies [L, B·T·H] of the τ fields (bozo_tau_aux_fwd's row_ent).
at::Tensor tau_row_entropy(const std::vector<at::Tensor>& taus) {
  check_fields(taus);
  const c10::cuda::CUDAGuard guard(taus[0].device());
  const auto stream = at::cuda::getCurrentCUDAStream(taus[0].device().index()).stream();
  const int64_t L = (int64_t)taus.size();
  const int64_t rows = taus[0].size(0) * taus[0].size(1) * taus[0].size(2);
  at::Tensor stats = at::empty({L, 3}, taus[0].options().dtype(at::kFloat));
  at::Tensor ent = at::empty({L, rows}, taus[0].options().dtype(at::kFloat));
  for (size_t i0 = 0; i0 < taus.size(); i0 += BOZO_TAU_AUX_MAX_LAYERS) {
    const size_t n = std::min<size_t>(BOZO_TAU_AUX_MAX_LAYERS, taus.size() - i0);
    bozo_tau_aux_fwd_args a{};
    fill_aux(a, taus, i0, n);
    a.stats = stats.data_ptr<float>() + 3 * i0;
    a.row_ent = ent.data_ptr<float>() + rows * (int64_t)i0;
    const size_t ws_bytes = bozo_tau_aux_workspace(&a);
    at::Tensor ws = at::empty({(int64_t)std::max<size_t>(ws_bytes, 1)},
                              taus[0].options().dtype(at::kByte));
    a.workspace = ws.data_ptr();
    a.workspace_bytes = ws_bytes;
    check(bozo_tau_aux_fwd(&a, stream), "bozo_tau_aux_fwd (row entropies)");
  }
  return ent;
}

// Cotangents of the τ fields from the cotangent [L, 3] of their statistics.
std::vector<at::Tensor> tau_aux_bwd(const std::vector<at::Tensor>& taus, const at::Tensor& d_stats) {
  check_fields(taus);
  const int64_t L = (int64_t)taus.size();
  if (d_stats.scalar_type() != at::kFloat || d_stats.numel() != 3 * L || !d_stats.is_contiguous() ||
      d_stats.device() != taus[0].device())
    throw std::invalid_argument("tau_aux: d_stats must be a contiguous fp32 [L,3] tensor on the fields' device");
  const c10::cuda::CUDAGuard guard(taus[0].device());
  const auto stream = at::cuda::getCurrentCUDAStream(taus[0].device().index()).stream();
  std::vector<at::Tensor> out;
  out.reserve(taus.size());
  for (const auto& t : taus) out.push_back(at::empty_like(t));
  for (size_t i0 = 0; i0 < taus.size(); i0 += BOZO_TAU_AUX_MAX_LAYERS) {
    const size_t n = std::min<size_t>(BOZO_TAU_AUX_MAX_LAYERS, taus.size() - i0);
    bozo_tau_aux_bwd_args a{};
    fill_aux(a, taus, i0, n);
    a.d_stats = d_stats.data_ptr<float>() + 3 * i0;
    for (size_t i = 0; i < n; ++i) a.d_tau[i] = out[i0 + i].data_ptr();
    check(bozo_tau_aux_bwd(&a, stream), "bozo_tau_aux_bwd");
  }
  return out;
}

// Row mode of the τ consumer's cotangent: per field the per-query-row
// coefficients [3, B·H·T] (a1, a0, 1/D) the tension backward takes as aux_row.
at::Tensor tau_aux_rowcoef(const std::vector<at::Tensor>& taus, const at::Tensor& d_stats) {
  check_fields(taus);
  const int64_t L = (int64_t)taus.size();
  if (d_stats.scalar_type() != at::kFloat || d_stats.numel() != 3 * L || !d_stats.is_contiguous() ||
      d_stats.device() != taus[0].device())
    throw std::invalid_argument("tau_aux: d_stats must be a contiguous fp32 [L,3] tensor on the fields' device");
  const c10::cuda::CUDAGuard guard(taus[0].device());
  const auto stream = at::cuda::getCurrentCUDAStream(taus[0].device().index()).stream();
  const int64_t rows = taus[0].size(0) * taus[0].size(1) * taus[0].size(2);
  at::Tensor out = at::empty({L, 3, rows}, taus[0].options().dtype(at::kFloat));
  for (size_t i0 = 0; i0 < taus.size(); i0 += BOZO_TAU_AUX_MAX_LAYERS) {
    const size_t n = std::min<size_t>(BOZO_TAU_AUX_MAX_LAYERS, taus.size() - i0);
    bozo_tau_aux_bwd_args a{};
    fill_aux(a, taus, i0, n);
    a.d_stats = d_stats.data_ptr<float>() + 3 * i0;
    for (size_t i = 0; i < n; ++i) a.row_coef[i] = out[i0 + i].data_ptr<float>();
    check(bozo_tau_aux_bwd(&a, stream), "bozo_tau_aux_bwd (row mode)");
  }
  return out;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "PyTorch binding of the bozo tension C ABI";
  m.def("tension_fwd", &tension_fwd, "forward through bozo_tension_fwd");
  m.def("tension_bwd", &tension_bwd, "backward through bozo_tension_bwd");
  m.def("tension_decode", &tension_decode, "one decode step through bozo_tension_decode");
  m.def("graph_bias", &graph_bias, "graph bias through bozo_graph_bias_build");
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd, "residual add + RMSNorm through bozo_add_rmsnorm_fwd");
  m.def("add_rmsnorm_bwd", &add_rmsnorm_bwd, "its backward through bozo_add_rmsnorm_bwd");
  m.def("wo_add_rmsnorm_fwd", &wo_add_rmsnorm_fwd,
        "wo projection + residual add + RMSNorm through bozo_wo_add_rmsnorm_fwd");
  m.def("embedding_bwd", &embedding_bwd, "token-embedding weight gradient through bozo_embedding_bwd");
  m.def("swiglu_fwd", &swiglu_fwd, "SwiGLU through bozo_swiglu_fwd");
  m.def("cross_entropy_fwd", &cross_entropy_fwd, "cross-entropy through bozo_cross_entropy_fwd");
  m.def("cross_entropy_bwd", &cross_entropy_bwd, "its backward through bozo_cross_entropy_bwd");
  m.def("swiglu_bwd", &swiglu_bwd, "its backward through bozo_swiglu_bwd");
  m.def("swiglu_packed_fwd", &swiglu_packed_fwd, "SwiGLU over packed [gate | value] rows");
  m.def("swiglu_packed_bwd", &swiglu_packed_bwd, "its backward, packed [d_gate | d_value] rows");
  m.def("tau_aux_fwd", &tau_aux_fwd, "τ-field statistics through bozo_tau_aux_fwd");
  m.def("tau_aux_bwd", &tau_aux_bwd, "τ-field cotangents through bozo_tau_aux_bwd");
  m.def("tau_row_entropy", &tau_row_entropy, "per-row τ entropies through bozo_tau_aux_fwd");
  m.def("tau_aux_rowcoef", &tau_aux_rowcoef,
        "per-query-row τ cotangent coefficients through bozo_tau_aux_bwd (row mode)");
}
