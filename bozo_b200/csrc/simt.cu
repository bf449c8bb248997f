// simt.cu — exact-fp32 CUDA-core kernels for every flag combination of the
// tension operator (any HD ≤ 128, any dtype mix, local or global, bias, τ
// export, RoPE, all three normalisations).  This is the parity path for fp32
// callers (rtol 1e-5) and the fallback for shapes the tcgen05 kernels do not
// take.  Semantics follow triton_tension/kernel.py:41-126 (forward),
// kernel.py:130-228 (dQ) and kernel.py:232-341 (dK/dV), widened by the
// model.py normalisation (257-258, 261-264) and global path (217-237).
//
// Structure: a CTA owns 32 rows (queries for fwd/dQ, keys for dK/dV) of one
// (b, h); 8 warps × 4 rows.  The partner rows are streamed through shared
// memory in chunks of 32 with lane = partner index, so the score of a
// (row, partner) pair lives in one lane and the HD-wide accumulations use
// warp shuffles.  All arithmetic is fp32.
#include <algorithm>

#include "common.cuh"

namespace bozo {
namespace {

constexpr int kRows = 32;     // rows owned by a CTA
constexpr int kChunk = 32;    // partner rows per shared-memory chunk
constexpr int kThreads = 256; // 8 warps × 4 rows

// Stage rows [t_begin, t_begin + n) of x[b, :, h, :] into dst (row pitch ld),
// applying the half-split rotation of model.py:75-81 when cos/sin are given.
// Out-of-range rows read as zero.
__device__ void stage_rows(float* dst, int ld, const DevT4& x, int b, int h,
                           int t_begin, int n, int T, int HD, const float* cos,
                           const float* sin) {
  const int half = HD / 2;
  const bool rope = cos != nullptr;
  const int per_row = rope ? half : HD;
  for (int idx = threadIdx.x; idx < n * per_row; idx += blockDim.x) {
    const int r = idx / per_row, d = idx % per_row;
    const int t = t_begin + r;
    float* row = dst + r * ld;
    if (t < 0 || t >= T) {
      row[d] = 0.f;
      if (rope) row[d + half] = 0.f;
      continue;
    }
    const long long base = (long long)b * x.sb + (long long)t * x.st + (long long)h * x.sh;
    if (rope) {
      const float x1 = ldf(x.p, base + (long long)d * x.sd, x.dt);
      const float x2 = ldf(x.p, base + (long long)(d + half) * x.sd, x.dt);
      const float c = cos[(long long)t * half + d], s = sin[(long long)t * half + d];
      row[d] = x1 * c - x2 * s;
      row[d + half] = x1 * s + x2 * c;
    } else {
      row[d] = ldf(x.p, base + (long long)d * x.sd, x.dt);
    }
  }
}

// Stage per-row scalars alpha/beta for query rows [t_begin, t_begin+n).
__device__ void stage_scalars(float* a_dst, float* b_dst, const float* alpha,
                              const float* beta, long long row_base, int t_begin,
                              int n, int T) {
  for (int r = threadIdx.x; r < n; r += blockDim.x) {
    const int t = t_begin + r;
    const bool ok = t >= 0 && t < T;
    a_dst[r] = ok ? alpha[row_base + t] : 0.f;
    b_dst[r] = ok ? beta[row_base + t] : 0.f;
  }
}

// Key validity and the bias / τ slot for the pair (query t, key s).
struct Pair {
  bool valid;
  int slot;       // local: window slot w; global: key position s
  int tau_slot;   // exported τ column, -1 if not exported
};

__device__ __forceinline__ Pair pair_of(int mode, int W, int T, int t, int s) {
  Pair pr;
  if (mode == BOZO_MODE_LOCAL) {
    pr.slot = s - t + W;
    pr.valid = s >= 0 && t < T && pr.slot >= 0 && pr.slot < W;
    pr.tau_slot = pr.valid ? pr.slot : -1;
  } else {
    pr.slot = s;
    pr.valid = s >= 0 && s <= t && t < T;
    const int j = T - 1 - s;  // model.py:236 flip: column j holds key T-1-j
    pr.tau_slot = (pr.valid && j < W) ? j : -1;
  }
  return pr;
}

__device__ __forceinline__ float row_dot(const float* a, const float* b, int HD) {
  float acc = 0.f;
  for (int d = 0; d < HD; ++d) acc = fmaf(a[d], b[d], acc);
  return acc;
}

// ───────────────────────────── forward ─────────────────────────────
template <int NJ>
__global__ void __launch_bounds__(kThreads) simt_fwd_kernel(FwdP p) {
  extern __shared__ float sm[];
  constexpr int LD = 32 * NJ + 1;
  float* Qs = sm;
  float* Ks = Qs + kRows * LD;
  float* Vs = Ks + kChunk * LD;
  const int b = blockIdx.z, h = blockIdx.y, t0 = blockIdx.x * kRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = p.T, HD = p.HD, W = p.W;
  const bool local = p.mode == BOZO_MODE_LOCAL;

  stage_rows(Qs, LD, p.q, b, h, t0, kRows, T, HD, p.cos, p.sin);
  if (!local && p.tau != nullptr) {
    // global export: zero the exported window for this tile first
    for (int idx = threadIdx.x; idx < kRows * W; idx += blockDim.x) {
      const int t = t0 + idx / W, j = idx % W;
      if (t < T) stf(p.tau, (((long long)b * T + t) * p.H + h) * W + j, p.tau_dt, 0.f);
    }
  }
  const int s_lo = local ? t0 - W : 0;
  const int s_hi = local ? min(t0 + kRows - 1, T) : min(t0 + kRows, T);

  float acc[4][NJ];
  float mass[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mass[i] = 0.f;
#pragma unroll
    for (int n = 0; n < NJ; ++n) acc[i][n] = 0.f;
  }

  for (int c0 = s_lo; c0 < s_hi; c0 += kChunk) {
    __syncthreads();
    stage_rows(Ks, LD, p.k, b, h, c0, kChunk, T, HD, p.cos, p.sin);
    stage_rows(Vs, LD, p.v, b, h, c0, kChunk, T, HD, nullptr, nullptr);
    __syncthreads();
    const int s = c0 + lane;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = warp * 4 + i, t = t0 + r;
      if (t >= T) continue;  // warp-uniform
      const Pair pr = pair_of(p.mode, W, T, t, s);
      float tau = 0.f;
      if (pr.valid && s < s_hi) {
        float x = row_dot(Qs + r * LD, Ks + lane * LD, HD) / p.scale;
        if (p.bias) x += p.bias[(long long)b * p.bs0 + (long long)t * p.bs1 + (long long)pr.slot * p.bs2];
        tau = sigmoid_exact(x);
      }
      if (p.tau != nullptr && s < s_hi) {
        if (local) {
          if (pr.slot >= 0 && pr.slot < W)
            stf(p.tau, (((long long)b * T + t) * p.H + h) * W + pr.slot, p.tau_dt, tau);
        } else if (pr.tau_slot >= 0) {
          stf(p.tau, (((long long)b * T + t) * p.H + h) * W + pr.tau_slot, p.tau_dt, tau);
        }
      }
      mass[i] += tau;
      for (int jj = 0; jj < kChunk; ++jj) {
        const float tj = __shfl_sync(0xffffffffu, tau, jj);
        if (tj == 0.f) continue;  // uniform across the warp
#pragma unroll
        for (int n = 0; n < NJ; ++n) acc[i][n] = fmaf(tj, Vs[jj * LD + lane + 32 * n], acc[i][n]);
      }
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp * 4 + i, t = t0 + r;
    const float m = warp_sum(mass[i]);
    if (t >= T) continue;
    float denom = 1.f;
    if (p.norm == BOZO_NORM_MASS) denom = fmaxf(m, kMassEps);
    if (p.norm == BOZO_NORM_COUNT) denom = (float)max(min(t, W), 1);
    const long long ob = (((long long)b * T + t) * p.H + h) * HD;
#pragma unroll
    for (int n = 0; n < NJ; ++n) {
      const int d = lane + 32 * n;
      if (d < HD) stf(p.out, ob + d, p.out_dt, p.norm == BOZO_NORM_NONE ? acc[i][n] : acc[i][n] / denom);
    }
    if (lane == 0 && p.row_mass) p.row_mass[((long long)b * p.H + h) * T + t] = m;
  }
}

// ───────────────────────── backward: dQ (+α, β) ─────────────────────────
// dτ(t,s) = α_t·(dO_t·V_s) + β_t + dTau(t,slot);  ds = dτ·τ(1−τ)/scale
//   NONE : α = 1,            β = 0
//   COUNT: α = 1/count_t,    β = 0
//   MASS : α = 1/max(m,ε),   β = −(dO_t·out_t)/max(m,ε) if m ≥ ε else 0
template <int NJ>
__global__ void __launch_bounds__(kThreads) simt_bwd_dq_kernel(BwdP p) {
  extern __shared__ float sm[];
  constexpr int LD = 32 * NJ + 1;
  float* Qs = sm;
  float* dOs = Qs + kRows * LD;
  float* Ks = dOs + kRows * LD;
  float* Vs = Ks + kChunk * LD;
  const int b = blockIdx.z, h = blockIdx.y, t0 = blockIdx.x * kRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = p.T, HD = p.HD, W = p.W;
  const bool local = p.mode == BOZO_MODE_LOCAL;
  const long long row_base = ((long long)b * p.H + h) * T;

  // inputs already rotated by the forward need no rotation here
  const float* rc = p.qk_rotated ? nullptr : p.cos;
  const float* rs = p.qk_rotated ? nullptr : p.sin;
  stage_rows(Qs, LD, p.q, b, h, t0, kRows, T, HD, rc, rs);
  stage_rows(dOs, LD, p.dout, b, h, t0, kRows, T, HD, nullptr, nullptr);
  __syncthreads();

  float alpha[4], beta[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp * 4 + i, t = t0 + r;
    alpha[i] = 1.f;
    beta[i] = 0.f;
    if (t >= T) continue;
    if (p.norm == BOZO_NORM_MASS) {
      const float m = p.row_mass[row_base + t];
      const float denom = fmaxf(m, kMassEps);
      float dd = 0.f;
      const long long ob = (long long)b * p.out.sb + (long long)t * p.out.st + (long long)h * p.out.sh;
      for (int d = lane; d < HD; d += 32) dd = fmaf(dOs[r * LD + d], ldf(p.out.p, ob + (long long)d * p.out.sd, p.out.dt), dd);
      dd = warp_sum(dd);
      alpha[i] = 1.f / denom;
      beta[i] = (m >= kMassEps) ? -dd / denom : 0.f;
    } else if (p.norm == BOZO_NORM_COUNT) {
      alpha[i] = 1.f / (float)max(min(t, W), 1);
    }
    if (lane == 0) {
      p.alpha[row_base + t] = alpha[i];
      p.beta[row_base + t] = beta[i];
    }
  }

  const int s_lo = local ? t0 - W : 0;
  const int s_hi = local ? min(t0 + kRows - 1, T) : min(t0 + kRows, T);
  float acc[4][NJ];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int n = 0; n < NJ; ++n) acc[i][n] = 0.f;

  for (int c0 = s_lo; c0 < s_hi; c0 += kChunk) {
    __syncthreads();
    stage_rows(Ks, LD, p.k, b, h, c0, kChunk, T, HD, rc, rs);
    stage_rows(Vs, LD, p.v, b, h, c0, kChunk, T, HD, nullptr, nullptr);
    __syncthreads();
    const int s = c0 + lane;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = warp * 4 + i, t = t0 + r;
      if (t >= T) continue;
      const Pair pr = pair_of(p.mode, W, T, t, s);
      float ds = 0.f;
      if (pr.valid && s < s_hi) {
        float x = row_dot(Qs + r * LD, Ks + lane * LD, HD) / p.scale;
        if (p.bias) x += p.bias[(long long)b * p.bs0 + (long long)t * p.bs1 + (long long)pr.slot * p.bs2];
        const float tau = sigmoid_exact(x);
        float dtau = fmaf(alpha[i], row_dot(dOs + r * LD, Vs + lane * LD, HD), beta[i]);
        if (p.dtau && pr.tau_slot >= 0)
          dtau += ldf(p.dtau, (((long long)b * T + t) * p.H + h) * W + pr.tau_slot, p.dtau_dt);
        ds = dtau * tau * (1.f - tau) / p.scale;
      }
      for (int jj = 0; jj < kChunk; ++jj) {
        const float dj = __shfl_sync(0xffffffffu, ds, jj);
        if (dj == 0.f) continue;
#pragma unroll
        for (int n = 0; n < NJ; ++n) acc[i][n] = fmaf(dj, Ks[jj * LD + lane + 32 * n], acc[i][n]);
      }
    }
  }

  // inverse RoPE (transpose rotation) through a shared-memory row, then store
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp * 4 + i;
#pragma unroll
    for (int n = 0; n < NJ; ++n) {
      const int d = lane + 32 * n;
      if (d < HD) Qs[r * LD + d] = acc[i][n];
    }
  }
  __syncwarp();
  const int half = HD / 2;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp * 4 + i, t = t0 + r;
    if (t >= T) continue;
    const long long ob = (((long long)b * T + t) * p.H + h) * HD;
    for (int d = lane; d < HD; d += 32) {
      float g = Qs[r * LD + d];
      if (p.cos) {
        const int dd = d < half ? d : d - half;
        const float c = p.cos[(long long)t * half + dd], sn = p.sin[(long long)t * half + dd];
        const float g1 = Qs[r * LD + dd], g2 = Qs[r * LD + dd + half];
        g = d < half ? (g1 * c + g2 * sn) : (g2 * c - g1 * sn);
      }
      stf(p.dq, ob + d, p.dq_dt, g);
    }
  }
}

// ─────────────────────── backward: dK, dV (key-centric) ───────────────────────
template <int NJ>
__global__ void __launch_bounds__(kThreads) simt_bwd_dkv_kernel(BwdP p) {
  extern __shared__ float sm[];
  constexpr int LD = 32 * NJ + 1;
  float* Ks = sm;
  float* Vs = Ks + kRows * LD;
  float* Qc = Vs + kRows * LD;
  float* dOc = Qc + kChunk * LD;
  float* Ac = dOc + kChunk * LD;
  float* Bc = Ac + kChunk;
  const int b = blockIdx.z, h = blockIdx.y, s0 = blockIdx.x * kRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = p.T, HD = p.HD, W = p.W;
  const bool local = p.mode == BOZO_MODE_LOCAL;
  const long long row_base = ((long long)b * p.H + h) * T;

  const float* rc = p.qk_rotated ? nullptr : p.cos;
  const float* rs = p.qk_rotated ? nullptr : p.sin;
  stage_rows(Ks, LD, p.k, b, h, s0, kRows, T, HD, rc, rs);
  stage_rows(Vs, LD, p.v, b, h, s0, kRows, T, HD, nullptr, nullptr);

  const int t_lo = local ? s0 + 1 : s0;
  const int t_hi = local ? min(s0 + kRows - 1 + W + 1, T) : T;

  float dk[4][NJ], dv[4][NJ];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int n = 0; n < NJ; ++n) dk[i][n] = dv[i][n] = 0.f;

  for (int c0 = t_lo; c0 < t_hi; c0 += kChunk) {
    __syncthreads();
    stage_rows(Qc, LD, p.q, b, h, c0, kChunk, T, HD, rc, rs);
    stage_rows(dOc, LD, p.dout, b, h, c0, kChunk, T, HD, nullptr, nullptr);
    stage_scalars(Ac, Bc, p.alpha, p.beta, row_base, c0, kChunk, T);
    __syncthreads();
    const int t = c0 + lane;
    const float a_t = Ac[lane], b_t = Bc[lane];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = warp * 4 + i, s = s0 + r;
      if (s >= T) continue;
      const Pair pr = pair_of(p.mode, W, T, t, s);
      float ds = 0.f, pa = 0.f;
      if (pr.valid && t < t_hi) {
        float x = row_dot(Qc + lane * LD, Ks + r * LD, HD) / p.scale;
        if (p.bias) x += p.bias[(long long)b * p.bs0 + (long long)t * p.bs1 + (long long)pr.slot * p.bs2];
        const float tau = sigmoid_exact(x);
        float dtau = fmaf(a_t, row_dot(dOc + lane * LD, Vs + r * LD, HD), b_t);
        if (p.dtau && pr.tau_slot >= 0)
          dtau += ldf(p.dtau, (((long long)b * T + t) * p.H + h) * W + pr.tau_slot, p.dtau_dt);
        ds = dtau * tau * (1.f - tau) / p.scale;
        pa = tau * a_t;
      }
      for (int jj = 0; jj < kChunk; ++jj) {
        const float dj = __shfl_sync(0xffffffffu, ds, jj);
        const float pj = __shfl_sync(0xffffffffu, pa, jj);
        if (dj == 0.f && pj == 0.f) continue;
#pragma unroll
        for (int n = 0; n < NJ; ++n) {
          dk[i][n] = fmaf(dj, Qc[jj * LD + lane + 32 * n], dk[i][n]);
          dv[i][n] = fmaf(pj, dOc[jj * LD + lane + 32 * n], dv[i][n]);
        }
      }
    }
  }

  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp * 4 + i;
#pragma unroll
    for (int n = 0; n < NJ; ++n) {
      const int d = lane + 32 * n;
      if (d < HD) Ks[r * LD + d] = dk[i][n];
    }
  }
  __syncwarp();
  const int half = HD / 2;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp * 4 + i, s = s0 + r;
    if (s >= T) continue;
    const long long ob = (((long long)b * T + s) * p.H + h) * HD;
#pragma unroll
    for (int n = 0; n < NJ; ++n) {
      const int d = lane + 32 * n;
      if (d < HD) stf(p.dv, ob + d, p.dv_dt, dv[i][n]);
    }
    for (int d = lane; d < HD; d += 32) {
      float g = Ks[r * LD + d];
      if (p.cos) {
        const int dd = d < half ? d : d - half;
        const float c = p.cos[(long long)s * half + dd], sn = p.sin[(long long)s * half + dd];
        const float g1 = Ks[r * LD + dd], g2 = Ks[r * LD + dd + half];
        g = d < half ? (g1 * c + g2 * sn) : (g2 * c - g1 * sn);
      }
      stf(p.dk, ob + d, p.dk_dt, g);
    }
  }
}

// RoPE(q) → q_rot, RoPE(k) → k_rot (half-split rotation, model.py:75-81),
// one thread per (row, pair), output contiguous in the input's dtype.
__global__ void rope_copy_kernel(FwdP p) {
  const int half = p.HD / 2;
  const long long n = (long long)p.B * p.T * p.H * half;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(idx % half);
    const long long row = idx / half;  // (b·T + t)·H + h
    const int h = (int)(row % p.H);
    const long long bt = row / p.H;
    const int t = (int)(bt % p.T), b = (int)(bt / p.T);
    const float c = p.cos[(long long)t * half + d], s = p.sin[(long long)t * half + d];
    const DevT4* src[2] = {&p.q, &p.k};
    void* dst[2] = {p.q_rot, p.k_rot};
#pragma unroll
    for (int z = 0; z < 2; ++z) {
      if (!dst[z]) continue;
      const DevT4& x = *src[z];
      const long long base = (long long)b * x.sb + (long long)t * x.st + (long long)h * x.sh;
      const float x1 = ldf(x.p, base + (long long)d * x.sd, x.dt);
      const float x2 = ldf(x.p, base + (long long)(d + half) * x.sd, x.dt);
      stf(dst[z], row * p.HD + d, x.dt, x1 * c - x2 * s);
      stf(dst[z], row * p.HD + d + half, x.dt, x1 * s + x2 * c);
    }
  }
}

// bf16 rows of HD 64 with unit innermost stride: four threads per row, each
// rotating eight frequency pairs with 16-byte loads and stores (columns
// [8c, 8c+8) with [32+8c, 32+8c+8)), one index division per row — the same
// arithmetic as rope_copy_kernel, at HBM speed instead of instruction-bound.
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[2 * e] = __uint_as_float(w[e] << 16);
    f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__global__ void __launch_bounds__(256) rope_copy_bf16_hd64(FwdP p) {
  const long long n = (long long)p.B * p.T * p.H * 4;
  const int TH = p.T * p.H;
  for (long long gi = blockIdx.x * (long long)blockDim.x + threadIdx.x; gi < n;
       gi += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(gi >> 2), c = (int)(gi & 3);
    const int b = row / TH, rem = row - b * TH, t = rem / p.H, h = rem - t * p.H;
    float cs[8], sn[8];
    {
      const float4* c4 = reinterpret_cast<const float4*>(p.cos + (long long)t * 32 + 8 * c);
      const float4* s4 = reinterpret_cast<const float4*>(p.sin + (long long)t * 32 + 8 * c);
      const float4 c0 = __ldg(c4), c1 = __ldg(c4 + 1), s0 = __ldg(s4), s1 = __ldg(s4 + 1);
      cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w; cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
      sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
    }
#pragma unroll
    for (int z = 0; z < 2; ++z) {
      const DevT4& x = z == 0 ? p.q : p.k;
      __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(z == 0 ? p.q_rot : p.k_rot);
      if (!dst) continue;
      const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(x.p) + (long long)b * x.sb +
                                 (long long)t * x.st + (long long)h * x.sh;
      float x1[8], x2[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(src + 8 * c)), x1);
      unpack8(__ldg(reinterpret_cast<const uint4*>(src + 32 + 8 * c)), x2);
      uint32_t r1[4], r2[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        r1[e] = pack2(x1[2 * e] * cs[2 * e] - x2[2 * e] * sn[2 * e],
                      x1[2 * e + 1] * cs[2 * e + 1] - x2[2 * e + 1] * sn[2 * e + 1]);
        r2[e] = pack2(x1[2 * e] * sn[2 * e] + x2[2 * e] * cs[2 * e],
                      x1[2 * e + 1] * sn[2 * e + 1] + x2[2 * e + 1] * cs[2 * e + 1]);
      }
      __nv_bfloat16* drow = dst + (long long)row * 64;
      *reinterpret_cast<uint4*>(drow + 8 * c) = make_uint4(r1[0], r1[1], r1[2], r1[3]);
      *reinterpret_cast<uint4*>(drow + 32 + 8 * c) = make_uint4(r2[0], r2[1], r2[2], r2[3]);
    }
  }
}

bool rope_copy_vec_ok(const FwdP& p) {
  if (p.HD != 64 || (long long)p.B * p.T * p.H >= (1ll << 29)) return false;
  if ((reinterpret_cast<uintptr_t>(p.cos) | reinterpret_cast<uintptr_t>(p.sin)) & 15) return false;
  const DevT4* xs[2] = {&p.q, &p.k};
  void* ds[2] = {p.q_rot, p.k_rot};
  for (int z = 0; z < 2; ++z) {
    if (!ds[z]) continue;
    const DevT4& x = *xs[z];
    if (x.dt != BOZO_DT_BF16 || x.sd != 1 || ((reinterpret_cast<uintptr_t>(x.p) | reinterpret_cast<uintptr_t>(ds[z])) & 15))
      return false;
    if ((x.sb | x.st | x.sh) & 7) return false;
  }
  return true;
}

template <int NJ>
cudaError_t fwd_nj(const FwdP& p, cudaStream_t st) {
  constexpr int LD = 32 * NJ + 1;
  const size_t smem = sizeof(float) * (kRows * LD + 2 * kChunk * LD);
  cudaError_t e = cudaFuncSetAttribute(simt_fwd_kernel<NJ>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.T + kRows - 1) / kRows, p.H, p.B);
  simt_fwd_kernel<NJ><<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <int NJ>
cudaError_t bwd_nj(const BwdP& p, cudaStream_t st) {
  constexpr int LD = 32 * NJ + 1;
  const size_t smem_dq = sizeof(float) * (2 * kRows * LD + 2 * kChunk * LD);
  const size_t smem_dkv = sizeof(float) * (2 * kRows * LD + 2 * kChunk * LD + 2 * kChunk);
  cudaError_t e = cudaFuncSetAttribute(simt_bwd_dq_kernel<NJ>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_dq);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(simt_bwd_dkv_kernel<NJ>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_dkv);
  if (e != cudaSuccess) return e;
  dim3 grid((p.T + kRows - 1) / kRows, p.H, p.B);
  simt_bwd_dq_kernel<NJ><<<grid, kThreads, smem_dq, st>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  simt_bwd_dkv_kernel<NJ><<<grid, kThreads, smem_dkv, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rope_copy(const FwdP& p, cudaStream_t st, int* launches) {
  *launches += 1;
  if (rope_copy_vec_ok(p)) {
    const long long n = (long long)p.B * p.T * p.H * 4;
    const int grid = (int)std::min<long long>((n + 255) / 256, 148 * 16);
    rope_copy_bf16_hd64<<<grid, 256, 0, st>>>(p);
    return cudaGetLastError();
  }
  const long long n = (long long)p.B * p.T * p.H * (p.HD / 2);
  const int grid = (int)std::min<long long>((n + 255) / 256, 148 * 16);
  rope_copy_kernel<<<grid, 256, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_simt_fwd(const FwdP& p, cudaStream_t st, int* launches) {
  *launches = 1;
  if (p.HD <= 32) return fwd_nj<1>(p, st);
  if (p.HD <= 64) return fwd_nj<2>(p, st);
  return fwd_nj<4>(p, st);
}

cudaError_t launch_simt_bwd(const BwdP& p, cudaStream_t st, int* launches) {
  *launches = 2;
  if (p.HD <= 32) return bwd_nj<1>(p, st);
  if (p.HD <= 64) return bwd_nj<2>(p, st);
  return bwd_nj<4>(p, st);
}

}  // namespace bozo
