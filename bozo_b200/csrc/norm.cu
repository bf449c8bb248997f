// norm.cu — the elementwise work around the tension operator in a TensionLM
// block, fused: residual add + RMSNorm (model.py:86-98, the
// `norm(x + wo(msg))` of model.py:259 and `norm(x + proj(h))` of
// model.py:330) and SwiGLU (model.py:328-329), forward and backward.
//
// add + RMSNorm, rows of width D (a multiple of 128): one warp per row, lane
// ℓ holding elements 4(ℓ + 32k) … +3 (one 16-byte load of x and one 8- or
// 16-byte load of y per k), so every warp load is a whole contiguous span of
// the row.  s = x + y (rounded to X when X is bf16, as a bf16 add is),
// rstd = rsqrt(mean(s²) + eps), out = s·rstd·scale.  The backward recomputes
// s from x and y: with g = dout·scale and ŝ = s·rstd,
//   ds = rstd·(g − ŝ·mean(g·ŝ)),  dx = ds,  dy = ds (in y's dtype),
//   dscale = Σ_rows dout·ŝ
// — the last as fixed-order per-block partial sums (each lane keeps its own
// columns' sums across the block's rows) reduced by a second kernel, instead
// of a column reduction over the whole [N, D] gradient.  For an fp32 stream
// under bf16 autocast the forward can also write a bf16 copy of out (the
// operand of the projections that read it, made once instead of one cast per
// projection), and the backward then adds that copy's bf16 cotangent to
// dout as it loads it.
//
// SwiGLU: h = silu(g)·v, dg = dh·v·σ(g)·(1 + g·(1 − σ(g))), dv = dh·silu(g),
// in fp32 per element, one read and one write of each tensor; g and v may be
// the two halves of packed [g | v] rows (one GEMM's output), and dg, dv then
// land in the same packed layout.
#include <cuda_bf16.h>

#include "bozo_block_ops.h"
#include "common.cuh"

namespace bozo {
namespace {

constexpr int kNormWarps = 8;

__device__ __forceinline__ void load4(const float* p, float* v) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float* v) {
  const uint2 a = *reinterpret_cast<const uint2*>(p);
  v[0] = __uint_as_float(a.x << 16); v[1] = __uint_as_float(a.x & 0xffff0000u);
  v[2] = __uint_as_float(a.y << 16); v[3] = __uint_as_float(a.y & 0xffff0000u);
}
__device__ __forceinline__ void store4(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float* v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<const uint32_t*>(&a),
                                            *reinterpret_cast<const uint32_t*>(&b));
}
__device__ __forceinline__ float round_to(float v, float*) { return v; }
__device__ __forceinline__ float round_to(float v, __nv_bfloat16*) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// K = D/128 chunks of 4 per lane
template <typename X, typename Y, int K>
__global__ void __launch_bounds__(kNormWarps * 32)
    add_rmsnorm_fwd_kernel(const X* __restrict__ x, const Y* __restrict__ y, const X* __restrict__ scale,
                           X* __restrict__ out, __nv_bfloat16* __restrict__ out_lp,
                           float* __restrict__ rstd_out, long long N, float eps) {
  constexpr int D = K * 128;
  const int lane = threadIdx.x & 31;
  float sc[K][4];
#pragma unroll
  for (int k = 0; k < K; ++k) load4(scale + 4 * (lane + 32 * k), sc[k]);
  for (long long r = (long long)blockIdx.x * kNormWarps + (threadIdx.x >> 5); r < N;
       r += (long long)gridDim.x * kNormWarps) {
    float s[K][4], ss = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const long long e = r * D + 4 * (lane + 32 * k);
      load4(x + e, s[k]);
      if (y) {
        float yv[4];
        load4(y + e, yv);
#pragma unroll
        for (int i = 0; i < 4; ++i) s[k][i] = round_to(s[k][i] + yv[i], (X*)nullptr);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) ss = fmaf(s[k][i], s[k][i], ss);
    }
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss * (1.f / D) + eps);
    if (lane == 0) rstd_out[r] = rstd;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = s[k][i] * rstd * sc[k][i];
      store4(out + r * D + 4 * (lane + 32 * k), o);
      if (out_lp) store4(out_lp + r * D + 4 * (lane + 32 * k), o);
    }
  }
}

template <typename X, typename Y, int K>
__global__ void __launch_bounds__(kNormWarps * 32)
    add_rmsnorm_bwd_kernel(const X* __restrict__ dout, const __nv_bfloat16* __restrict__ dout_lp,
                           const X* __restrict__ x, const Y* __restrict__ y,
                           const X* __restrict__ scale, const float* __restrict__ rstd_in,
                           X* __restrict__ dx, Y* __restrict__ dy, float* __restrict__ dscale_part,
                           long long N) {
  constexpr int D = K * 128;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float sc[K][4], acc[K][4];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    load4(scale + 4 * (lane + 32 * k), sc[k]);
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[k][i] = 0.f;
  }
  for (long long r = (long long)blockIdx.x * kNormWarps + warp; r < N; r += (long long)gridDim.x * kNormWarps) {
    const float rstd = rstd_in[r];
    float sh[K][4], g[K][4], dot = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const long long e = r * D + 4 * (lane + 32 * k);
      float dv[4];
      load4(x + e, sh[k]);
      if (y) {
        float yv[4];
        load4(y + e, yv);
#pragma unroll
        for (int i = 0; i < 4; ++i) sh[k][i] = round_to(sh[k][i] + yv[i], (X*)nullptr);
      }
      load4(dout + e, dv);
      if (dout_lp) {
        float dl[4];
        load4(dout_lp + e, dl);
#pragma unroll
        for (int i = 0; i < 4; ++i) dv[i] += dl[i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sh[k][i] *= rstd;
        g[k][i] = dv[i] * sc[k][i];
        dot = fmaf(g[k][i], sh[k][i], dot);
        acc[k][i] = fmaf(dv[i], sh[k][i], acc[k][i]);
      }
    }
    dot = warp_sum(dot) * (1.f / D);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float d[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] = rstd * (g[k][i] - sh[k][i] * dot);
      const long long e = r * D + 4 * (lane + 32 * k);
      store4(dx + e, d);
      if (dy) store4(dy + e, d);
    }
  }
  // block partial of dscale: the warps' column sums, added in warp order
  __shared__ float red[kNormWarps][D];
#pragma unroll
  for (int k = 0; k < K; ++k)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][4 * (lane + 32 * k) + i] = acc[k][i];
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kNormWarps; ++w) v += red[w][c];
    dscale_part[(long long)blockIdx.x * D + c] = v;
  }
}

// dscale[c] = Σ_blocks part[b][c] in a fixed order (deterministic): one CTA
// per 32 columns, lane = column (each warp reads whole 128-byte rows), warp w
// sums blocks w, w + 32, … in four interleaved chains, then the 32 warp sums
// are added in warp order.
constexpr int kReduceWarps = 32;
template <typename X>
__global__ void __launch_bounds__(kReduceWarps * 32)
    dscale_reduce_kernel(const float* __restrict__ part, int nblk, int D, X* __restrict__ dscale) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (c < D) {
    int b = warp;
#pragma unroll 1
    for (; b + 3 * kReduceWarps < nblk; b += 4 * kReduceWarps) {
#pragma unroll
      for (int z = 0; z < 4; ++z) v[z] += __ldg(part + (long long)(b + z * kReduceWarps) * D + c);
    }
    for (int z = 0; b < nblk; b += kReduceWarps, ++z) v[z] += __ldg(part + (long long)b * D + c);
  }
  __shared__ float red[kReduceWarps][32];
  red[warp][lane] = (v[0] + v[1]) + (v[2] + v[3]);
  __syncthreads();
  if (warp == 0 && c < D) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kReduceWarps; ++w) s += red[w][lane];
    dscale[c] = (X)s;
  }
}

// Offset of element e of h in the gate/value (and their gradients') layout:
// the same index for flat tensors (width 0), else row e / width at `stride`.
__device__ __forceinline__ long long gv_off(long long e, int width, long long stride) {
  if (width == 0) return e;
  const long long r = e / width;
  return r * stride + (e - r * width);
}

template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ g, const T* __restrict__ v, T* __restrict__ h,
                                  long long n, int width, long long stride) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n / 4;
       i += (long long)gridDim.x * blockDim.x) {
    float gv[4], vv[4], o[4];
    const long long a = gv_off(4 * i, width, stride);
    load4(g + a, gv);
    load4(v + a, vv);
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = gv[k] / (1.f + expf(-gv[k])) * vv[k];
    store4(h + 4 * i, o);
  }
}

template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ dh, const T* __restrict__ g, const T* __restrict__ v,
                                  T* __restrict__ dg, T* __restrict__ dv, long long n, int width,
                                  long long stride) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n / 4;
       i += (long long)gridDim.x * blockDim.x) {
    float d[4], gv[4], vv[4], og[4], ov[4];
    const long long a = gv_off(4 * i, width, stride);
    load4(dh + 4 * i, d);
    load4(g + a, gv);
    load4(v + a, vv);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float sig = 1.f / (1.f + expf(-gv[k]));
      ov[k] = d[k] * gv[k] * sig;
      og[k] = d[k] * vv[k] * sig * (1.f + gv[k] * (1.f - sig));
    }
    store4(dg + a, og);
    store4(dv + a, ov);
  }
}

// bf16 SwiGLU, 8 elements (16 bytes) per thread and step.  Chunk c of h is
// row c / w8, columns 8·(c mod w8) … +7 of the gate/value layout (a flat
// tensor is one row: w8 = chunks, stride unused); a 32-bit division per 8
// elements instead of a 64-bit one per 4.  σ(g) = 1/(1 + e^−g) with the
// hardware exponential and a correctly rounded reciprocal (e^−g = ∞ gives
// σ = 0); the products round once more, to bf16, on the way out.
__device__ __forceinline__ void unpack8(uint4 q, float* f) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    f[2 * k] = __uint_as_float(w[k] << 16);
    f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
    w[k] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ float sigmoid_fast(float x) { return __frcp_rn(1.f + __expf(-x)); }

__global__ void swiglu_fwd_bf16x8(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ v,
                                  __nv_bfloat16* __restrict__ h, int chunks, int w8, long long stride) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < chunks; c += gridDim.x * blockDim.x) {
    const int row = c / w8;
    const long long a = (long long)row * stride + 8 * (c - row * w8);
    float gf[8], vf[8], o[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(g + a)), gf);
    unpack8(__ldg(reinterpret_cast<const uint4*>(v + a)), vf);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = gf[k] * sigmoid_fast(gf[k]) * vf[k];
    reinterpret_cast<uint4*>(h)[c] = pack8(o);
  }
}

__global__ void swiglu_bwd_bf16x8(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ g,
                                  const __nv_bfloat16* __restrict__ v, __nv_bfloat16* __restrict__ dg,
                                  __nv_bfloat16* __restrict__ dv, int chunks, int w8, long long stride) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < chunks; c += gridDim.x * blockDim.x) {
    const int row = c / w8;
    const long long a = (long long)row * stride + 8 * (c - row * w8);
    float d[8], gf[8], vf[8], og[8], ov[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(dh) + c), d);
    unpack8(__ldg(reinterpret_cast<const uint4*>(g + a)), gf);
    unpack8(__ldg(reinterpret_cast<const uint4*>(v + a)), vf);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float sig = sigmoid_fast(gf[k]);
      ov[k] = d[k] * gf[k] * sig;
      og[k] = d[k] * vf[k] * sig * (1.f + gf[k] * (1.f - sig));
    }
    *reinterpret_cast<uint4*>(dg + a) = pack8(og);
    *reinterpret_cast<uint4*>(dv + a) = pack8(ov);
  }
}

int norm_grid(long long N, int sms) {
  const long long want = (N + kNormWarps - 1) / kNormWarps;
  const long long cap = (long long)sms * 4;
  return (int)(want < cap ? (want < 1 ? 1 : want) : cap);
}

template <typename X, typename Y>
cudaError_t fwd_t(const NormP& p, cudaStream_t st) {
  const int grid = norm_grid(p.N, p.sms);
  const X* x = static_cast<const X*>(p.x);
  const Y* y = static_cast<const Y*>(p.y);
  const X* sc = static_cast<const X*>(p.scale);
  X* out = static_cast<X*>(p.out);
  __nv_bfloat16* olp = static_cast<__nv_bfloat16*>(p.out_lp);
  switch (p.D / 128) {
    case 1: add_rmsnorm_fwd_kernel<X, Y, 1><<<grid, kNormWarps * 32, 0, st>>>(x, y, sc, out, olp, p.rstd, p.N, p.eps); break;
    case 2: add_rmsnorm_fwd_kernel<X, Y, 2><<<grid, kNormWarps * 32, 0, st>>>(x, y, sc, out, olp, p.rstd, p.N, p.eps); break;
    case 4: add_rmsnorm_fwd_kernel<X, Y, 4><<<grid, kNormWarps * 32, 0, st>>>(x, y, sc, out, olp, p.rstd, p.N, p.eps); break;
    case 6: add_rmsnorm_fwd_kernel<X, Y, 6><<<grid, kNormWarps * 32, 0, st>>>(x, y, sc, out, olp, p.rstd, p.N, p.eps); break;
    case 8: add_rmsnorm_fwd_kernel<X, Y, 8><<<grid, kNormWarps * 32, 0, st>>>(x, y, sc, out, olp, p.rstd, p.N, p.eps); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename X, typename Y>
cudaError_t bwd_t(const NormP& p, cudaStream_t st) {
  const int grid = norm_grid(p.N, p.sms);
  const X* dout = static_cast<const X*>(p.dout);
  const __nv_bfloat16* dlp = static_cast<const __nv_bfloat16*>(p.dout_lp);
  const X* x = static_cast<const X*>(p.x);
  const Y* y = static_cast<const Y*>(p.y);
  const X* sc = static_cast<const X*>(p.scale);
  X* dx = static_cast<X*>(p.dx);
  Y* dy = static_cast<Y*>(p.dy);
  switch (p.D / 128) {
    case 1: add_rmsnorm_bwd_kernel<X, Y, 1><<<grid, kNormWarps * 32, 0, st>>>(dout, dlp, x, y, sc, p.rstd, dx, dy, p.part, p.N); break;
    case 2: add_rmsnorm_bwd_kernel<X, Y, 2><<<grid, kNormWarps * 32, 0, st>>>(dout, dlp, x, y, sc, p.rstd, dx, dy, p.part, p.N); break;
    case 4: add_rmsnorm_bwd_kernel<X, Y, 4><<<grid, kNormWarps * 32, 0, st>>>(dout, dlp, x, y, sc, p.rstd, dx, dy, p.part, p.N); break;
    case 6: add_rmsnorm_bwd_kernel<X, Y, 6><<<grid, kNormWarps * 32, 0, st>>>(dout, dlp, x, y, sc, p.rstd, dx, dy, p.part, p.N); break;
    case 8: add_rmsnorm_bwd_kernel<X, Y, 8><<<grid, kNormWarps * 32, 0, st>>>(dout, dlp, x, y, sc, p.rstd, dx, dy, p.part, p.N); break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  dscale_reduce_kernel<X><<<(p.D + 31) / 32, kReduceWarps * 32, 0, st>>>(p.part, grid, p.D,
                                                                      static_cast<X*>(p.dscale));
  return cudaGetLastError();
}

}  // namespace

int norm_partial_blocks(long long N, int sms) { return norm_grid(N, sms); }

bool norm_width_ok(int D) {
  const int k = D / 128;
  return D % 128 == 0 && (k == 1 || k == 2 || k == 4 || k == 6 || k == 8);
}

cudaError_t launch_add_rmsnorm(const NormP& p, bool backward, cudaStream_t st) {
  const bool xb = p.x_dt == BOZO_DT_BF16;
  const int yk = p.y ? p.y_dt : -1;
  if (!backward) {
    if (!xb && yk == BOZO_DT_BF16) return fwd_t<float, __nv_bfloat16>(p, st);
    if (!xb) return fwd_t<float, float>(p, st);
    return fwd_t<__nv_bfloat16, __nv_bfloat16>(p, st);
  }
  if (!xb && yk == BOZO_DT_BF16) return bwd_t<float, __nv_bfloat16>(p, st);
  if (!xb) return bwd_t<float, float>(p, st);
  return bwd_t<__nv_bfloat16, __nv_bfloat16>(p, st);
}

cudaError_t launch_swiglu(const void* g, const void* v, void* h, const void* dh, void* dg, void* dv,
                          long long n, int width, long long stride, int dt, int sms, cudaStream_t st) {
  const long long want = (n / 4 + 255) / 256;
  const int grid = (int)(want < (long long)sms * 8 ? (want < 1 ? 1 : want) : (long long)sms * 8);
  if (dt == BOZO_DT_BF16) {
    using T = __nv_bfloat16;
    auto a16 = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (n % 8 == 0 && n / 8 <= 0x7fffffffLL && width % 8 == 0 && stride % 8 == 0 && a16(g) && a16(v) &&
        a16(h) && a16(dh) && a16(dg) && a16(dv)) {
      const int chunks = (int)(n / 8);
      const int w8 = width ? width / 8 : chunks;
      const long long want8 = (chunks + 255) / 256;
      const int grid8 = (int)(want8 < (long long)sms * 8 ? (want8 < 1 ? 1 : want8) : (long long)sms * 8);
      if (dh)
        swiglu_bwd_bf16x8<<<grid8, 256, 0, st>>>((const T*)dh, (const T*)g, (const T*)v, (T*)dg, (T*)dv,
                                                 chunks, w8, stride);
      else
        swiglu_fwd_bf16x8<<<grid8, 256, 0, st>>>((const T*)g, (const T*)v, (T*)h, chunks, w8, stride);
      return cudaGetLastError();
    }
    if (dh)
      swiglu_bwd_kernel<T><<<grid, 256, 0, st>>>((const T*)dh, (const T*)g, (const T*)v, (T*)dg, (T*)dv, n,
                                                  width, stride);
    else
      swiglu_fwd_kernel<T><<<grid, 256, 0, st>>>((const T*)g, (const T*)v, (T*)h, n, width, stride);
  } else {
    if (dh)
      swiglu_bwd_kernel<float><<<grid, 256, 0, st>>>((const float*)dh, (const float*)g, (const float*)v,
                                                      (float*)dg, (float*)dv, n, width, stride);
    else
      swiglu_fwd_kernel<float><<<grid, 256, 0, st>>>((const float*)g, (const float*)v, (float*)h, n, width,
                                                      stride);
  }
  return cudaGetLastError();
}

}  // namespace bozo
