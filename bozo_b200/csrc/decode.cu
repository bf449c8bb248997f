// decode.cu — one decode step of the tension operator (bozo_tension_decode):
// the new token's query against ring caches of rotated keys and values.
// Per step and (b, h) this reads the W cached keys of a local layer (all
// cached keys of a global one) once, instead of model.py:718-768's
// generate_cached, which re-runs every layer over the whole context for
// each new token.
//
// Step at position t (read from device memory, so a captured CUDA graph of
// the whole step can be replayed for every token):
//   1. RoPE(k_t) and v_t go into ring row t mod C; RoPE(q_t) into shared
//      memory (half-split rotation, model.py:75-81, tables [rope_len, HD/2]);
//   2. keys: LOCAL s ∈ [max(0, t−W), t−1] (self excluded, ops.py:29-63),
//      GLOBAL s ∈ [max(0, t−C+1), t] (self included, model.py:217-237; a
//      wrapped ring keeps the last C keys); one warp per key, lanes over the
//      head dimension, τ = σ(q·k/scale) with the exact fp32 sigmoid;
//   3. normaliser: τ-mass max(Σ τ, 1e-6) (model.py:257-258), valid count
//      max(min(t, W), 1) (model.py:261-264) or 1 (raw);
//   4. out[d] = Σ τ·v[d] / normaliser, one thread per head dimension reading
//      whole value rows;
//   5. optional τ row: LOCAL slot w = W − (t − s), GLOBAL column c = t − s
//      (model.py:233-236's flipped window), zero where no key exists.
// One 128-thread block per (b, h); the cache rows of a (b, h) are only
// touched by its block.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace bozo {
namespace {

constexpr int kDecThreads = 128;
constexpr int kErrDecode = 0x400;

__global__ void __launch_bounds__(kDecThreads) decode_kernel(DecodeP p) {
  extern __shared__ float sm[];
  float* sq = sm;           // rotated q [HD]
  float* stau = sm + p.HD;  // τ per key [n]
  __shared__ float red[kDecThreads / 32];
  const int b = blockIdx.x / p.H, h = blockIdx.x - b * p.H;
  const int HD = p.HD, half = HD / 2;
  const int t = __ldg(p.pos);
  if (t < 0 || (p.cos && t >= p.rope_len)) {  // no table row for this position
    if (threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, kErrDecode | 1);
    return;
  }
  const long long qo = (long long)b * p.q.sb + (long long)h * p.q.sh;
  const long long ko = (long long)b * p.k.sb + (long long)h * p.k.sh;
  const long long vo = (long long)b * p.v.sb + (long long)h * p.v.sh;
  const long long crow = (((long long)b * p.C + (t % p.C)) * p.H + h) * HD;
  // 1. rotate q and k; k, v into ring row t mod C
  if (p.cos) {
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const float c = p.cos[(long long)t * half + i], s = p.sin[(long long)t * half + i];
      const float q1 = ldf(p.q.p, qo + (long long)i * p.q.sd, p.q.dt);
      const float q2 = ldf(p.q.p, qo + (long long)(i + half) * p.q.sd, p.q.dt);
      const float k1 = ldf(p.k.p, ko + (long long)i * p.k.sd, p.k.dt);
      const float k2 = ldf(p.k.p, ko + (long long)(i + half) * p.k.sd, p.k.dt);
      sq[i] = q1 * c - q2 * s;
      sq[i + half] = q1 * s + q2 * c;
      stf(p.kc, crow + i, p.kc_dt, k1 * c - k2 * s);
      stf(p.kc, crow + i + half, p.kc_dt, k1 * s + k2 * c);
    }
  } else {
    for (int i = threadIdx.x; i < HD; i += blockDim.x) {
      sq[i] = ldf(p.q.p, qo + (long long)i * p.q.sd, p.q.dt);
      stf(p.kc, crow + i, p.kc_dt, ldf(p.k.p, ko + (long long)i * p.k.sd, p.k.dt));
    }
  }
  for (int i = threadIdx.x; i < HD; i += blockDim.x)
    stf(p.vc, crow + i, p.vc_dt, ldf(p.v.p, vo + (long long)i * p.v.sd, p.v.dt));
  __syncthreads();  // the block's own cache writes and sq are visible below

  // 2. τ of every key: key j is s = t − 1 − j (local) or s = t − j (global)
  const bool local = p.mode == BOZO_MODE_LOCAL;
  const int n = local ? min(t, p.W) : min(t + 1, p.C);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = warp; j < n; j += kDecThreads / 32) {
    const int s = local ? t - 1 - j : t - j;
    const long long row = (((long long)b * p.C + (s % p.C)) * p.H + h) * HD;
    float dot = 0.f;
    for (int d = lane; d < HD; d += 32) dot = fmaf(sq[d], ldf(p.kc, row + d, p.kc_dt), dot);
    dot = warp_sum(dot);
    if (lane == 0) stau[j] = sigmoid_exact(dot * p.inv_scale);
  }
  __syncthreads();

  // 3. normaliser
  float den = 1.f;
  if (p.norm == BOZO_NORM_MASS) {
    float m = 0.f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) m += stau[j];
    m = warp_sum(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = 0.f;
    for (int w = 0; w < kDecThreads / 32; ++w) m += red[w];
    den = fmaxf(m, kMassEps);
  } else if (p.norm == BOZO_NORM_COUNT) {
    den = (float)max(n, 1);
  }
  const float inv_den = 1.f / den;

  // 4. out = Σ τ·v / normaliser
  const long long oo = ((long long)b * p.H + h) * HD;
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < n; ++j) {
      const int s = local ? t - 1 - j : t - j;
      const long long row = (((long long)b * p.C + (s % p.C)) * p.H + h) * HD;
      acc = fmaf(stau[j], ldf(p.vc, row + d, p.vc_dt), acc);
    }
    stf(p.out, oo + d, p.out_dt, acc * inv_den);
  }

  // 5. this row of the exported τ field
  if (p.tau) {
    const long long to = ((long long)b * p.H + h) * p.tw;
    for (int c = threadIdx.x; c < p.tw; c += blockDim.x) {
      // LOCAL slot c holds key t − (W − c), i.e. key index j = W − 1 − c;
      // GLOBAL column c holds key t − c, i.e. j = c
      const int j = local ? p.W - 1 - c : c;
      stf(p.tau, to + c, p.tau_dt, (j >= 0 && j < n) ? stau[j] : 0.f);
    }
  }
}

// ─────────────── vector path: caches of one dtype E, HD ∈ {32, 64, 128} ───────────────
// Steps 2 and 4 with whole-row vector loads: G = HD·sizeof(E)/16 lanes share
// one cached key row (one 16-byte load each), so a warp scores 32/G keys per
// load and four key groups are in flight per iteration; for the values each
// warp accumulates Σ τ·v over its share of the keys with each lane holding
// HD/32 consecutive dimensions (coalesced row loads, 8 keys in flight), and
// the warps' partial sums are added in shared memory.  The ring slot of each
// key comes from one division per CTA and a conditional wrap, and the
// sigmoid runs once per key over all threads after the dot products (not in
// one lane of G).  At B16 H12 with 1001 cached keys this took the kernel
// from 33.7 to 17.3 µs (16 warps per CTA for long caches: two CTAs per SM
// fit in the register file, so all 192 CTAs run in one wave; 32 warps gave
// 21.4 µs), and a 64-key window from 5.5 to 4.8 µs.
constexpr int kFastWarps = 8;
constexpr int kWideWarps = 16;

template <typename E> struct DecVec;
template <> struct DecVec<float> { static constexpr int n = 4; };
template <> struct DecVec<__nv_bfloat16> { static constexpr int n = 8; };
template <> struct DecVec<__half> { static constexpr int n = 8; };

__device__ __forceinline__ float dec_f(float v) { return v; }
__device__ __forceinline__ float dec_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float dec_f(__half v) { return __half2float(v); }

// N consecutive elements (N·sizeof(E) ∈ {2, 4, 8, 16} bytes, aligned) as floats
template <typename E, int N>
__device__ __forceinline__ void dec_load(const E* p, float* x) {
  constexpr int bytes = N * (int)sizeof(E);
  E e[N];
  if constexpr (bytes == 16) {
    *reinterpret_cast<uint4*>(e) = __ldg(reinterpret_cast<const uint4*>(p));
  } else if constexpr (bytes == 8) {
    *reinterpret_cast<uint2*>(e) = __ldg(reinterpret_cast<const uint2*>(p));
  } else if constexpr (bytes == 4) {
    *reinterpret_cast<uint32_t*>(e) = __ldg(reinterpret_cast<const uint32_t*>(p));
  } else {
#pragma unroll
    for (int k = 0; k < N; ++k) e[k] = p[k];
  }
#pragma unroll
  for (int k = 0; k < N; ++k) x[k] = dec_f(e[k]);
}

template <typename E, int HD, int kW>
__global__ void __launch_bounds__(kW * 32) decode_kernel_vec(DecodeP p) {
  constexpr int NV = DecVec<E>::n, G = HD / NV, KPW = 32 / G, DPL = HD / 32;
  static_assert(HD % NV == 0 && G <= 32 && (G & (G - 1)) == 0, "lanes per key");
  extern __shared__ float sm[];
  float* sq = sm;                      // rotated q [HD]
  float* part = sm + HD;               // per-warp Σ τ·v [warps][HD]
  float* stau = part + kW * HD;  // τ per key [n]
  __shared__ float red[kW];
  const int b = blockIdx.x / p.H, h = blockIdx.x - b * p.H;
  const int half = HD / 2;
  const int t = __ldg(p.pos);
  if (t < 0 || (p.cos && t >= p.rope_len)) {
    if (threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, kErrDecode | 1);
    return;
  }
  E* kc = static_cast<E*>(p.kc);
  E* vc = static_cast<E*>(p.vc);
  const long long qo = (long long)b * p.q.sb + (long long)h * p.q.sh;
  const long long ko = (long long)b * p.k.sb + (long long)h * p.k.sh;
  const long long vo = (long long)b * p.v.sb + (long long)h * p.v.sh;
  const long long crow = (((long long)b * p.C + (t % p.C)) * p.H + h) * HD;
  if (p.cos) {
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const float c = p.cos[(long long)t * half + i], s = p.sin[(long long)t * half + i];
      const float q1 = ldf(p.q.p, qo + (long long)i * p.q.sd, p.q.dt);
      const float q2 = ldf(p.q.p, qo + (long long)(i + half) * p.q.sd, p.q.dt);
      const float k1 = ldf(p.k.p, ko + (long long)i * p.k.sd, p.k.dt);
      const float k2 = ldf(p.k.p, ko + (long long)(i + half) * p.k.sd, p.k.dt);
      sq[i] = q1 * c - q2 * s;
      sq[i + half] = q1 * s + q2 * c;
      stf(kc, crow + i, p.kc_dt, k1 * c - k2 * s);
      stf(kc, crow + i + half, p.kc_dt, k1 * s + k2 * c);
    }
  } else {
    for (int i = threadIdx.x; i < HD; i += blockDim.x) {
      sq[i] = ldf(p.q.p, qo + (long long)i * p.q.sd, p.q.dt);
      stf(kc, crow + i, p.kc_dt, ldf(p.k.p, ko + (long long)i * p.k.sd, p.k.dt));
    }
  }
  for (int i = threadIdx.x; i < HD; i += blockDim.x)
    stf(vc, crow + i, p.vc_dt, ldf(p.v.p, vo + (long long)i * p.v.sd, p.v.dt));
  __syncthreads();

  const bool local = p.mode == BOZO_MODE_LOCAL;
  const int n = local ? min(t, p.W) : min(t + 1, p.C);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane % G, sub = lane / G;
  // ring slot of key j (0 = the newest key): one division per CTA, then a
  // conditional wrap (j < n ≤ C, so at most one)
  const int s_top = max(local ? t - 1 : t, 0) % p.C;
  const long long row0 = ((long long)b * p.C * p.H + h) * HD, rstride = (long long)p.H * HD;
  auto key_row = [&](int j) {
    int s = s_top - j;
    s += s < 0 ? p.C : 0;
    return row0 + s * rstride;
  };
  // 2. scores (scaled dot products) into stau: keys j = j0 + sub, four
  // groups per iteration
  float qv[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) qv[k] = sq[g * NV + k];
  constexpr int kStep = kW * KPW;
  constexpr int kGroups = 4;  // key groups in flight per iteration
  for (int j0 = warp * KPW; j0 < n; j0 += kGroups * kStep) {
    float x[kGroups][NV];
#pragma unroll
    for (int u = 0; u < kGroups; ++u) {
      const int jj = j0 + u * kStep + sub;
      if (jj < n) {
        dec_load<E, NV>(kc + key_row(jj) + g * NV, x[u]);
      } else {
#pragma unroll
        for (int k = 0; k < NV; ++k) x[u][k] = 0.f;
      }
    }
    float d[kGroups];
#pragma unroll
    for (int u = 0; u < kGroups; ++u) {
      d[u] = 0.f;
#pragma unroll
      for (int k = 0; k < NV; ++k) d[u] = fmaf(qv[k], x[u][k], d[u]);
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) d[u] += __shfl_xor_sync(0xffffffffu, d[u], o);
    }
    if (g == 0) {
#pragma unroll
      for (int u = 0; u < kGroups; ++u) {
        const int jj = j0 + u * kStep + sub;
        if (jj < n) stau[jj] = d[u] * p.inv_scale;
      }
    }
  }
  __syncthreads();

  // 3. τ = σ(score), one key per thread (not one lane in G), and the
  // normaliser
  float m = 0.f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float tau = sigmoid_exact(stau[j]);
    stau[j] = tau;
    m += tau;
  }
  __syncthreads();
  float den = 1.f;
  if (p.norm == BOZO_NORM_MASS) {
    m = warp_sum(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) m += red[w];
    den = fmaxf(m, kMassEps);
  } else if (p.norm == BOZO_NORM_COUNT) {
    den = (float)max(n, 1);
  }

  // 4. per-warp Σ τ·v over keys j ≡ warp (mod warps), lane = HD/32 dims
  float acc[DPL];
#pragma unroll
  for (int k = 0; k < DPL; ++k) acc[k] = 0.f;
  constexpr int kRowsInFlight = 8;
  int j = warp;
  for (; j + (kRowsInFlight - 1) * kW < n; j += kRowsInFlight * kW) {
    float v[kRowsInFlight][DPL];
#pragma unroll
    for (int r = 0; r < kRowsInFlight; ++r)
      dec_load<E, DPL>(vc + key_row(j + r * kW) + lane * DPL, v[r]);
#pragma unroll
    for (int r = 0; r < kRowsInFlight; ++r) {
      const float tr = stau[j + r * kW];
#pragma unroll
      for (int k = 0; k < DPL; ++k) acc[k] = fmaf(tr, v[r][k], acc[k]);
    }
  }
  for (; j < n; j += kW) {
    float v0[DPL];
    dec_load<E, DPL>(vc + key_row(j) + lane * DPL, v0);
    const float t0 = stau[j];
#pragma unroll
    for (int k = 0; k < DPL; ++k) acc[k] = fmaf(t0, v0[k], acc[k]);
  }
#pragma unroll
  for (int k = 0; k < DPL; ++k) part[warp * HD + lane * DPL + k] = acc[k];
  __syncthreads();
  const float inv_den = 1.f / den;
  const long long oo = ((long long)b * p.H + h) * HD;
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) o += part[w * HD + d];
    stf(p.out, oo + d, p.out_dt, o * inv_den);
  }
  if (p.tau) {
    const long long to = ((long long)b * p.H + h) * p.tw;
    for (int c = threadIdx.x; c < p.tw; c += blockDim.x) {
      const int jj = local ? p.W - 1 - c : c;
      stf(p.tau, to + c, p.tau_dt, (jj >= 0 && jj < n) ? stau[jj] : 0.f);
    }
  }
}

template <typename E>
cudaError_t launch_vec(const DecodeP& p, size_t smem, cudaStream_t st) {
  // a long cache (global layers, wide windows) gets 32 warps per (b, h):
  // four times the loads in flight per step of its short dependent chain
  const bool wide = (p.mode == BOZO_MODE_GLOBAL ? p.C : p.W) > 256;
  const int threads = (wide ? kWideWarps : kFastWarps) * 32;
  auto go = [&](auto kern) {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    kern<<<p.B * p.H, threads, smem, st>>>(p);
    return cudaGetLastError();
  };
  switch (p.HD) {
    case 32: return wide ? go(decode_kernel_vec<E, 32, kWideWarps>) : go(decode_kernel_vec<E, 32, kFastWarps>);
    case 64: return wide ? go(decode_kernel_vec<E, 64, kWideWarps>) : go(decode_kernel_vec<E, 64, kFastWarps>);
    default:
      return wide ? go(decode_kernel_vec<E, 128, kWideWarps>) : go(decode_kernel_vec<E, 128, kFastWarps>);
  }
}

bool vec_path_ok(const DecodeP& p) {
  if (p.HD != 32 && p.HD != 64 && p.HD != 128) return false;
  if (p.kc_dt != p.vc_dt) return false;
  if ((reinterpret_cast<uintptr_t>(p.kc) | reinterpret_cast<uintptr_t>(p.vc)) & 15) return false;
  return true;
}

}  // namespace

size_t decode_smem_bytes(const DecodeP& p) {
  const int n = p.mode == BOZO_MODE_LOCAL ? p.W : p.C;
  if (vec_path_ok(p)) return (size_t)(p.HD * (1 + kWideWarps) + n) * sizeof(float);
  return (size_t)(p.HD + n) * sizeof(float);
}

cudaError_t launch_decode(const DecodeP& p, cudaStream_t st) {
  const size_t smem = decode_smem_bytes(p);
  if (vec_path_ok(p)) {
    switch (p.kc_dt) {
      case BOZO_DT_F32: return launch_vec<float>(p, smem, st);
      case BOZO_DT_BF16: return launch_vec<__nv_bfloat16>(p, smem, st);
      default: return launch_vec<__half>(p, smem, st);
    }
  }
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  decode_kernel<<<p.B * p.H, kDecThreads, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace bozo
