// tau_aux.cu — the fused τ-field consumer (include/bozo_tau_aux.h): the
// three τ regularisers of the reference training loop (model.py:498-611) as
// one read of every exported τ field, and their cotangent as one read plus
// one write of it.
//
// A field is N = B·T·H rows of W values (row r = (b·T + t)·H + h).  Every
// statistic is a sum of per-row terms, so each kernel walks rows:
//   * vector path (W a multiple of the 16-byte vector and ≤ 32 vectors):
//     G = W/vec lanes share one row, one 16-byte load each, so a warp load
//     covers 32/G whole rows (two 128-byte rows per 8-lane group pair at
//     W = 64 bf16) and the row sums are 8-lane shuffle trees;
//   * scalar path (any other W): one warp per row, lanes strided over it,
//     the row re-read from L1/L2 for each pass.
// Per row (x = the row, S = Σx, D = S + 1e-8, p = x/D, model.py:527-528;
// one reciprocal per row, logs in base 2 with the row scale and ln 2 applied
// per row, log2 and 1/q by the fast hardware approximations, whose error
// stays far below the fp32 tolerance of the sums):
//   ent = −Σ p·log(p + 1e-8)                           diversity (model.py:528)
//   pen = relu(0.05 − S/W) + relu(S/W − 0.8)           entropy   (model.py:602-608)
//   hinge_i = relu(x[t,i]·x[t−1,0] − x[t,i+1]),  i < m  consistency (model.py:561-576)
// The backward (∂ent/∂x_w = g_w/D − (Σ_v g_v·x_v)/D², g = −(log(p+1e-8) +
// p/(p+1e-8))) recomputes S, D, p from the row it rewrites; the consistency
// terms that reach slot 0 of row t from row t+1 read the first m+1 values of
// that row (an L2 hit: the neighbouring rows are streamed by other warps).
//
// The statistics are reduced deterministically: fp32 per-block partial sums,
// then one block per layer adds them in a fixed order in fp64.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "bozo_tau_aux.h"
#include "common.cuh"

namespace bozo {
namespace {

constexpr int kAuxThreads = 256;
constexpr int kAuxWarps = kAuxThreads / 32;
constexpr float kAuxEps = 1e-8f;  // model.py:527-528

struct AuxPtrs {
  const void* tau[BOZO_TAU_AUX_MAX_LAYERS];
  void* dtau[BOZO_TAU_AUX_MAX_LAYERS];
};

// 16-byte vectors of each element type
template <typename E> struct VecOf;
template <> struct VecOf<float> { static constexpr int n = 4; };
template <> struct VecOf<__nv_bfloat16> { static constexpr int n = 8; };
template <> struct VecOf<__half> { static constexpr int n = 8; };

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
template <typename E> __device__ __forceinline__ E from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename E>
__device__ __forceinline__ void load_vec(const E* p, float* x) {
  constexpr int n = VecOf<E>::n;
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const E* e = reinterpret_cast<const E*>(&u);
#pragma unroll
  for (int k = 0; k < n; ++k) x[k] = to_f(e[k]);
}

template <typename E>
__device__ __forceinline__ void store_vec(E* p, const float* x) {
  constexpr int n = VecOf<E>::n;
  uint4 u;
  E* e = reinterpret_cast<E*>(&u);
#pragma unroll
  for (int k = 0; k < n; ++k) e[k] = from_f<E>(x[k]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Query position t of row r = (b·T + t)·H + h.
__device__ __forceinline__ int query_of(long long r, const AuxShape& s) {
  const uint32_t bt = fast_div((uint32_t)r, s.div_h);
  return (int)(bt - fast_div(bt, s.div_t) * (uint32_t)s.T);
}

// Sum over the G lanes of an aligned lane group (all 32 lanes take part).
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// The row entropy in base 2 with the row scale pulled out:
//   −Σ_w p_w·ln(p_w + 1e-8) = −ln2·(1/D)·Σ_w x_w·log2(x_w/D + 1e-8),
// so a value costs one FFMA, one MUFU lg2 and one FFMA.
constexpr float kLn2 = 0.69314718f;
constexpr float kInvLn2 = 1.44269504f;
__device__ __forceinline__ float ent2_term(float x, float invD, float acc) {
  return fmaf(x, __log2f(fmaf(x, invD, kAuxEps)), acc);
}
// ∂ent/∂p = −(ln q + p/q), q = p + 1e-8, as −ln2·h with
// h = log2 q + (p/ln2)·(1/q)  (invDl = invD/ln2): two MUFU ops and two FFMAs.
__device__ __forceinline__ float grad_h(float x, float invD, float invDl) {
  const float q = fmaf(x, invD, kAuxEps);
  return fmaf(x * invDl, __fdividef(1.f, q), __log2f(q));
}

// Consistency slot i is live for query t iff t ∈ [i+2, i+2+t_out) (model.py:561-571).
__device__ __forceinline__ bool cons_live(int t, int i, int t_out) {
  return t >= i + 2 && t < i + 2 + t_out;
}

// Sums the three per-block accumulators and writes this block's partials.
__device__ void block_partials(float a0, float a1, float a2, float* out) {
  __shared__ float red[3][kAuxWarps];
  a0 = warp_sum(a0);
  a1 = warp_sum(a1);
  a2 = warp_sum(a2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red[0][warp] = a0;
    red[1][warp] = a1;
    red[2][warp] = a2;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    float s = 0.f;
    for (int w = 0; w < kAuxWarps; ++w) s += red[threadIdx.x][w];
    out[threadIdx.x] = s;
  }
}

// ───────────────────────────── vector path ─────────────────────────────
// What one lane fetches for row r an iteration ahead of using it: its vector
// of the row and, on the group's first lane, the neighbour-row values of the
// consistency terms (slot 0 of row t−1; for the backward also the first
// slots of row t+1).  So every load of an iteration is issued together and
// none waits on another.
template <typename E, bool kNext>
struct RowFetch {
  float x[VecOf<E>::n];
  float prev0;
  float nxt[8];
  int t;
  bool live;
};

template <typename E, bool kNext>
__device__ __forceinline__ void fetch_row(const E* tau, long long r, const AuxShape& s, int g,
                                          RowFetch<E, kNext>& f) {
  constexpr int NV = VecOf<E>::n;
  f.live = r < s.N;
  // N < 2^31 (checked on the host): 32-bit index math
  f.t = f.live ? query_of(r, s) : 0;
  if (f.live) {
    load_vec(tau + r * s.W + g * NV, f.x);
  } else {
#pragma unroll
    for (int k = 0; k < NV; ++k) f.x[k] = 0.f;
  }
  const bool lead = g == 0 && f.live && s.m > 0;
  f.prev0 = lead && f.t >= 1 ? to_f(tau[(r - s.H) * s.W]) : 0.f;
  if constexpr (kNext) {
#pragma unroll
    for (int k = 0; k < 8; ++k) f.nxt[k] = 0.f;
    if (lead && f.t + 1 < s.T) {
      const E* nrow = tau + (r + s.H) * s.W;
      load_vec(nrow, f.nxt);
      if (NV == 4 && s.m >= 4) load_vec(nrow + 4, f.nxt + 4);
    }
  }
}

template <typename E, int G>
__global__ void __launch_bounds__(kAuxThreads)
    tau_aux_fwd_vec(AuxPtrs P, AuxShape s, float* __restrict__ partial, float* __restrict__ row_ent) {
  constexpr int NV = VecOf<E>::n, RPW = 32 / G;
  const int layer = blockIdx.y;
  const E* tau = static_cast<const E*>(P.tau[layer]);
  const int lane = threadIdx.x & 31, g = lane % G, sub = lane / G;
  const long long warp0 = (long long)blockIdx.x * kAuxWarps + (threadIdx.x >> 5);
  const long long step = (long long)gridDim.x * kAuxWarps * RPW;
  float acc_ent = 0.f, acc_hinge = 0.f, acc_pen = 0.f;
  RowFetch<E, false> cur, nx;
  fetch_row<E, false>(tau, warp0 * RPW + sub, s, g, nx);
  for (long long base = warp0 * RPW; base < s.N; base += step) {
    cur = nx;
    fetch_row<E, false>(tau, base + step + sub, s, g, nx);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) sum += cur.x[k];
    sum = group_sum<G>(sum);
    const float invD = __fdividef(1.f, sum + kAuxEps);
    float e = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) e = ent2_term(cur.x[k], invD, e);
    e = -kLn2 * invD * group_sum<G>(e);
    // slot 4 of a fp32 row sits in the group's second lane
    const float x4 = NV > 4 ? cur.x[NV > 4 ? 4 : 0] : __shfl_down_sync(0xffffffffu, cur.x[0], 1);
    if (cur.live && g == 0) {
      acc_ent += e;
      if (row_ent) row_ent[(long long)layer * s.N + base + sub] = e;
      const float mu = sum * s.inv_w;
      acc_pen += fmaxf(0.05f - mu, 0.f) + fmaxf(mu - 0.8f, 0.f);
      if (s.m > 0 && cur.t >= 1) {
        const float xe[5] = {cur.x[0], cur.x[1], cur.x[2], cur.x[3], x4};
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (i < s.m && cons_live(cur.t, i, s.t_out))
            acc_hinge += fmaxf(xe[i] * cur.prev0 - xe[i + 1], 0.f);
      }
    }
  }
  block_partials(acc_ent, acc_hinge, acc_pen,
                 partial + ((long long)layer * gridDim.x + blockIdx.x) * 3);
}

template <typename E, int G>
__global__ void __launch_bounds__(kAuxThreads)
    tau_aux_bwd_vec(AuxPtrs P, AuxShape s, const float* __restrict__ d_stats) {
  constexpr int NV = VecOf<E>::n, RPW = 32 / G;
  const int layer = blockIdx.y;
  const E* tau = static_cast<const E*>(P.tau[layer]);
  E* dtau = static_cast<E*>(P.dtau[layer]);
  const float gE = d_stats[layer * 3 + 0] * s.inv_n;
  const float gC = d_stats[layer * 3 + 1] * s.inv_cons;
  const float gP = d_stats[layer * 3 + 2] * s.inv_n * s.inv_w;
  const int lane = threadIdx.x & 31, g = lane % G, sub = lane / G;
  const long long warp0 = (long long)blockIdx.x * kAuxWarps + (threadIdx.x >> 5);
  const long long step = (long long)gridDim.x * kAuxWarps * RPW;
  RowFetch<E, true> cur, nx;
  fetch_row<E, true>(tau, warp0 * RPW + sub, s, g, nx);
  for (long long base = warp0 * RPW; base < s.N; base += step) {
    cur = nx;
    fetch_row<E, true>(tau, base + step + sub, s, g, nx);
    const long long r = base + sub;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) sum += cur.x[k];
    sum = group_sum<G>(sum);
    const float invD = __fdividef(1.f, sum + kAuxEps), invDl = invD * kInvLn2;
    float hq[NV], a = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      hq[k] = grad_h(cur.x[k], invD, invDl);
      a = fmaf(hq[k], cur.x[k], a);
    }
    a = group_sum<G>(a);
    const float mu = sum * s.inv_w;
    const float dpen = gP * ((0.05f - mu > 0.f ? -1.f : 0.f) + (mu - 0.8f > 0.f ? 1.f : 0.f));
    // dx = gE·(g/D − (Σ g·x)/D²) + dpen with g = −ln2·h
    const float c1 = -kLn2 * gE * invD, c0 = dpen + kLn2 * gE * a * invD * invD;
    float dx[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) dx[k] = fmaf(c1, hq[k], c0);
    // consistency: slots 0..m of this row, from this row's terms and row t+1's
    const float x4 = NV > 4 ? cur.x[NV > 4 ? 4 : 0] : __shfl_down_sync(0xffffffffu, cur.x[0], 1);
    float dc[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    if (cur.live && g == 0 && s.m > 0) {
      const float xe[5] = {cur.x[0], cur.x[1], cur.x[2], cur.x[3], x4};
      if (cur.t >= 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (i < s.m && cons_live(cur.t, i, s.t_out) && xe[i] * cur.prev0 - xe[i + 1] > 0.f) {
            dc[i] += gC * cur.prev0;
            dc[i + 1] -= gC;
          }
      }
      if (cur.t + 1 < s.T) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (i < s.m && cons_live(cur.t + 1, i, s.t_out) && cur.nxt[i] * xe[0] - cur.nxt[i + 1] > 0.f)
            dc[0] += gC * cur.nxt[i];
      }
    }
    if (g == 0) {
#pragma unroll
      for (int k = 0; k < (NV < 5 ? NV : 5); ++k) dx[k] += dc[k];
    }
    if (NV == 4) {  // slot 4 of a fp32 row belongs to the group's second lane
      const float d4 = __shfl_up_sync(0xffffffffu, dc[4], 1);
      if (g == 1) dx[0] += d4;
    }
    if (cur.live) store_vec(dtau + r * s.W + g * NV, dx);
  }
}

// ─────────────── wide path: 2-byte fields, W = 32·G (G = 1, 2, 4, 8) ───────────────
// Each lane holds 32 values of a row as four 16-byte chunks c = k·G + g
// (k < 4), so every warp load covers G consecutive chunks of each of its 32/G
// rows, and the per-row work (index math, consistency slots, reciprocal) is
// spread over 32 values per lane instead of 8.  Slots 0..7 — all the
// consistency terms touch — are chunk 0, on the group's first lane.
__device__ __forceinline__ float2 unpack2(uint32_t u, __nv_bfloat16*) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
__device__ __forceinline__ float2 unpack2(uint32_t u, __half*) {
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t word(const uint4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

template <bool kNext>
struct WideFetch {
  uint4 v[4];
  uint4 nxt;     // chunk 0 of row t+1 (backward, first lane of the group)
  float prev0;   // slot 0 of row t−1 (first lane of the group)
  int t;
  bool live;
};

template <typename E, int G, bool kNext>
__device__ __forceinline__ void fetch_wide(const E* tau, long long r, const AuxShape& s, int g,
                                           WideFetch<kNext>& f) {
  f.live = r < s.N;
  f.t = f.live ? query_of(r, s) : 0;
  const uint4 z = make_uint4(0, 0, 0, 0);
  const uint4* row = reinterpret_cast<const uint4*>(tau + r * s.W);
#pragma unroll
  for (int k = 0; k < 4; ++k) f.v[k] = f.live ? __ldg(row + k * G + g) : z;
  const bool lead = g == 0 && f.live && s.m > 0;
  f.prev0 = lead && f.t >= 1 ? to_f(tau[(r - s.H) * s.W]) : 0.f;
  if constexpr (kNext)
    f.nxt = lead && f.t + 1 < s.T ? __ldg(reinterpret_cast<const uint4*>(tau + (r + s.H) * s.W)) : z;
}

template <typename E, int G>
__global__ void __launch_bounds__(kAuxThreads)
    tau_aux_fwd_wide(AuxPtrs P, AuxShape s, float* __restrict__ partial, float* __restrict__ row_ent) {
  constexpr int RPW = 32 / G;
  const int layer = blockIdx.y;
  const E* tau = static_cast<const E*>(P.tau[layer]);
  const int lane = threadIdx.x & 31, g = lane % G, sub = lane / G;
  const long long warp0 = (long long)blockIdx.x * kAuxWarps + (threadIdx.x >> 5);
  const long long step = (long long)gridDim.x * kAuxWarps * RPW;
  float acc_ent = 0.f, acc_hinge = 0.f, acc_pen = 0.f;
  WideFetch<false> cur, nx;
  fetch_wide<E, G, false>(tau, warp0 * RPW + sub, s, g, nx);
  for (long long base = warp0 * RPW; base < s.N; base += step) {
    cur = nx;
    fetch_wide<E, G, false>(tau, base + step + sub, s, g, nx);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = unpack2(word(cur.v[k], j), (E*)nullptr);
        sum += a.x + a.y;
      }
    sum = group_sum<G>(sum);
    const float invD = __fdividef(1.f, sum + kAuxEps);
    float e = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = unpack2(word(cur.v[k], j), (E*)nullptr);
        e = ent2_term(a.x, invD, e);
        e = ent2_term(a.y, invD, e);
      }
    e = -kLn2 * invD * group_sum<G>(e);
    if (cur.live && g == 0) {
      acc_ent += e;
      if (row_ent) row_ent[(long long)layer * s.N + base + sub] = e;
      const float mu = sum * s.inv_w;
      acc_pen += fmaxf(0.05f - mu, 0.f) + fmaxf(mu - 0.8f, 0.f);
      if (s.m > 0 && cur.t >= 1) {
        const float2 a = unpack2(cur.v[0].x, (E*)nullptr), b = unpack2(cur.v[0].y, (E*)nullptr),
                     c = unpack2(cur.v[0].z, (E*)nullptr);
        const float xe[5] = {a.x, a.y, b.x, b.y, c.x};
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (i < s.m && cons_live(cur.t, i, s.t_out))
            acc_hinge += fmaxf(xe[i] * cur.prev0 - xe[i + 1], 0.f);
      }
    }
  }
  block_partials(acc_ent, acc_hinge, acc_pen,
                 partial + ((long long)layer * gridDim.x + blockIdx.x) * 3);
}

template <typename E, int G>
__global__ void __launch_bounds__(kAuxThreads)
    tau_aux_bwd_wide(AuxPtrs P, AuxShape s, const float* __restrict__ d_stats) {
  constexpr int RPW = 32 / G;
  const int layer = blockIdx.y;
  const E* tau = static_cast<const E*>(P.tau[layer]);
  E* dtau = static_cast<E*>(P.dtau[layer]);
  const float gE = d_stats[layer * 3 + 0] * s.inv_n;
  const float gC = d_stats[layer * 3 + 1] * s.inv_cons;
  const float gP = d_stats[layer * 3 + 2] * s.inv_n * s.inv_w;
  const int lane = threadIdx.x & 31, g = lane % G, sub = lane / G;
  const long long warp0 = (long long)blockIdx.x * kAuxWarps + (threadIdx.x >> 5);
  const long long step = (long long)gridDim.x * kAuxWarps * RPW;
  WideFetch<true> cur, nx;
  fetch_wide<E, G, true>(tau, warp0 * RPW + sub, s, g, nx);
  for (long long base = warp0 * RPW; base < s.N; base += step) {
    cur = nx;
    fetch_wide<E, G, true>(tau, base + step + sub, s, g, nx);
    const long long r = base + sub;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = unpack2(word(cur.v[k], j), (E*)nullptr);
        sum += a.x + a.y;
      }
    sum = group_sum<G>(sum);
    const float invD = __fdividef(1.f, sum + kAuxEps), invDl = invD * kInvLn2;
    // h_w (∂ent/∂p_w = −ln2·h_w), kept for the write pass
    float gq[32], a = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = unpack2(word(cur.v[k], j), (E*)nullptr);
        gq[8 * k + 2 * j] = grad_h(x.x, invD, invDl);
        gq[8 * k + 2 * j + 1] = grad_h(x.y, invD, invDl);
        a = fmaf(gq[8 * k + 2 * j], x.x, a);
        a = fmaf(gq[8 * k + 2 * j + 1], x.y, a);
      }
    a = group_sum<G>(a);
    const float mu = sum * s.inv_w;
    const float dpen = gP * ((0.05f - mu > 0.f ? -1.f : 0.f) + (mu - 0.8f > 0.f ? 1.f : 0.f));
    const float c1 = -kLn2 * gE * invD, c0 = dpen + kLn2 * gE * a * invD * invD;
    // consistency: slots 0..m of this row, from this row's terms and row t+1's
    float dc[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    if (cur.live && g == 0 && s.m > 0) {
      const float2 a0 = unpack2(cur.v[0].x, (E*)nullptr), a1 = unpack2(cur.v[0].y, (E*)nullptr),
                   a2 = unpack2(cur.v[0].z, (E*)nullptr);
      const float xe[5] = {a0.x, a0.y, a1.x, a1.y, a2.x};
      if (cur.t >= 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (i < s.m && cons_live(cur.t, i, s.t_out) && xe[i] * cur.prev0 - xe[i + 1] > 0.f) {
            dc[i] += gC * cur.prev0;
            dc[i + 1] -= gC;
          }
      }
      if (cur.t + 1 < s.T) {
        const float2 n0 = unpack2(cur.nxt.x, (E*)nullptr), n1 = unpack2(cur.nxt.y, (E*)nullptr),
                     n2 = unpack2(cur.nxt.z, (E*)nullptr);
        const float xn[5] = {n0.x, n0.y, n1.x, n1.y, n2.x};
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (i < s.m && cons_live(cur.t + 1, i, s.t_out) && xn[i] * xe[0] - xn[i + 1] > 0.f)
            dc[0] += gC * xn[i];
      }
    }
    if (cur.live) {
      uint4* out = reinterpret_cast<uint4*>(dtau + r * s.W);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float d0 = fmaf(c1, gq[8 * k + 2 * j], c0), d1 = fmaf(c1, gq[8 * k + 2 * j + 1], c0);
          if (k == 0 && j < 3) {  // slots 0..5 of chunk 0 (dc is zero off the first lane)
            d0 += dc[2 * j];
            if (2 * j + 1 < 5) d1 += dc[2 * j + 1];
          }
          w[j] = pack2(d0, d1, (E*)nullptr);
        }
        out[k * G + g] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

// Row mode of the cotangent: per query row the coefficients with which the
// tension backward forms the diversity + entropy cotangent itself,
//   dτ_w = c1·h_w + c0 = a1·(log2 q_w − 1e-8/(q_w·ln 2)) + a0,
//   a1 = c1, a0 = c0 + c1/ln 2, q_w = τ_w/D + 1e-8,
// written to [a1 | a0 | 1/D] planes at row (b·H + h)·T + t (the backward's
// per-query-row order).  The consistency cotangent is not per-row: callers
// use this mode only when it is zero.
template <typename E, int G>
__global__ void __launch_bounds__(kAuxThreads)
    tau_aux_rowcoef_wide(AuxPtrs P, AuxShape s, const float* __restrict__ d_stats) {
  constexpr int RPW = 32 / G;
  const int layer = blockIdx.y;
  const E* tau = static_cast<const E*>(P.tau[layer]);
  float* coef = static_cast<float*>(P.dtau[layer]);
  const float gE = d_stats[layer * 3 + 0] * s.inv_n;
  const float gP = d_stats[layer * 3 + 2] * s.inv_n * s.inv_w;
  const int lane = threadIdx.x & 31, g = lane % G, sub = lane / G;
  const long long warp0 = (long long)blockIdx.x * kAuxWarps + (threadIdx.x >> 5);
  const long long step = (long long)gridDim.x * kAuxWarps * RPW;
  WideFetch<false> cur, nx;
  fetch_wide<E, G, false>(tau, warp0 * RPW + sub, s, g, nx);
  for (long long base = warp0 * RPW; base < s.N; base += step) {
    cur = nx;
    fetch_wide<E, G, false>(tau, base + step + sub, s, g, nx);
    const long long r = base + sub;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = unpack2(word(cur.v[k], j), (E*)nullptr);
        sum += a.x + a.y;
      }
    sum = group_sum<G>(sum);
    const float invD = __fdividef(1.f, sum + kAuxEps), invDl = invD * kInvLn2;
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = unpack2(word(cur.v[k], j), (E*)nullptr);
        a = fmaf(grad_h(x.x, invD, invDl), x.x, a);
        a = fmaf(grad_h(x.y, invD, invDl), x.y, a);
      }
    a = group_sum<G>(a);
    if (cur.live && g == 0) {
      const float mu = sum * s.inv_w;
      const float dpen = gP * ((0.05f - mu > 0.f ? -1.f : 0.f) + (mu - 0.8f > 0.f ? 1.f : 0.f));
      const float c1 = -kLn2 * gE * invD, c0 = dpen + kLn2 * gE * a * invD * invD;
      const uint32_t bt = fast_div((uint32_t)r, s.div_h);
      const uint32_t h = (uint32_t)r - bt * (uint32_t)s.H;
      const uint32_t b = fast_div(bt, s.div_t);
      const uint32_t t = bt - b * (uint32_t)s.T;
      const long long o = ((long long)b * s.H + h) * s.T + t;
      coef[o] = c1;
      coef[s.N + o] = fmaf(c1, kInvLn2, c0);
      coef[2 * s.N + o] = invD;
    }
  }
}

// ───────────────────────────── scalar path ─────────────────────────────
// One warp per row, any W; the row is re-read for every pass.
template <typename E>
__global__ void __launch_bounds__(kAuxThreads)
    tau_aux_fwd_scalar(AuxPtrs P, AuxShape s, float* __restrict__ partial, float* __restrict__ row_ent) {
  const int layer = blockIdx.y;
  const E* tau = static_cast<const E*>(P.tau[layer]);
  const int lane = threadIdx.x & 31;
  const long long w0 = (long long)blockIdx.x * kAuxWarps + (threadIdx.x >> 5);
  const long long wstep = (long long)gridDim.x * kAuxWarps;
  float acc_ent = 0.f, acc_hinge = 0.f, acc_pen = 0.f;
  for (long long r = w0; r < s.N; r += wstep) {
    const E* row = tau + r * s.W;
    float sum = 0.f;
    for (int w = lane; w < s.W; w += 32) sum += to_f(row[w]);
    sum = warp_sum(sum);
    const float invD = __fdividef(1.f, sum + kAuxEps);
    float e = 0.f;
    for (int w = lane; w < s.W; w += 32) e = ent2_term(to_f(row[w]), invD, e);
    e = -kLn2 * invD * warp_sum(e);
    if (lane == 0) {
      acc_ent += e;
      if (row_ent) row_ent[(long long)layer * s.N + r] = e;
      const float mu = sum * s.inv_w;
      acc_pen += fmaxf(0.05f - mu, 0.f) + fmaxf(mu - 0.8f, 0.f);
      const int t = query_of(r, s);
      if (s.m > 0 && t >= 1) {
        const float prev0 = to_f(tau[(r - s.H) * s.W]);
        for (int i = 0; i < s.m; ++i)
          if (cons_live(t, i, s.t_out)) acc_hinge += fmaxf(to_f(row[i]) * prev0 - to_f(row[i + 1]), 0.f);
      }
    }
  }
  block_partials(acc_ent, acc_hinge, acc_pen,
                 partial + ((long long)layer * gridDim.x + blockIdx.x) * 3);
}

template <typename E>
__global__ void __launch_bounds__(kAuxThreads)
    tau_aux_bwd_scalar(AuxPtrs P, AuxShape s, const float* __restrict__ d_stats) {
  const int layer = blockIdx.y;
  const E* tau = static_cast<const E*>(P.tau[layer]);
  E* dtau = static_cast<E*>(P.dtau[layer]);
  const float gE = d_stats[layer * 3 + 0] * s.inv_n;
  const float gC = d_stats[layer * 3 + 1] * s.inv_cons;
  const float gP = d_stats[layer * 3 + 2] * s.inv_n * s.inv_w;
  const int lane = threadIdx.x & 31;
  const long long w0 = (long long)blockIdx.x * kAuxWarps + (threadIdx.x >> 5);
  const long long wstep = (long long)gridDim.x * kAuxWarps;
  for (long long r = w0; r < s.N; r += wstep) {
    const E* row = tau + r * s.W;
    float sum = 0.f;
    for (int w = lane; w < s.W; w += 32) sum += to_f(row[w]);
    sum = warp_sum(sum);
    const float invD = __fdividef(1.f, sum + kAuxEps), invDl = invD * kInvLn2;
    float a = 0.f;
    for (int w = lane; w < s.W; w += 32) {
      const float x = to_f(row[w]);
      a = fmaf(grad_h(x, invD, invDl), x, a);
    }
    a = warp_sum(a);
    const float mu = sum * s.inv_w;
    const float dpen = gP * ((0.05f - mu > 0.f ? -1.f : 0.f) + (mu - 0.8f > 0.f ? 1.f : 0.f));
    const float c1 = -kLn2 * gE * invD, c0 = dpen + kLn2 * gE * a * invD * invD;
    const int t = query_of(r, s);
    for (int w = lane; w < s.W; w += 32) {
      const float x = to_f(row[w]);
      float dx = fmaf(c1, grad_h(x, invD, invDl), c0);
      if (s.m > 0 && w <= s.m) {  // consistency terms of slot w
        if (t >= 1) {
          const float prev0 = to_f(tau[(r - s.H) * s.W]);
          for (int i = 0; i < s.m; ++i)
            if (cons_live(t, i, s.t_out) && to_f(row[i]) * prev0 - to_f(row[i + 1]) > 0.f) {
              if (w == i) dx += gC * prev0;
              if (w == i + 1) dx -= gC;
            }
        }
        if (w == 0 && t + 1 < s.T) {
          const E* nrow = tau + (r + s.H) * s.W;
          for (int i = 0; i < s.m; ++i) {
            const float xi = to_f(nrow[i]);
            if (cons_live(t + 1, i, s.t_out) && xi * x - to_f(nrow[i + 1]) > 0.f) dx += gC * xi;
          }
        }
      }
      dtau[r * s.W + w] = from_f<E>(dx);
    }
  }
}

// One block per layer: the fixed-order fp64 sum of that layer's partials.
__global__ void __launch_bounds__(kAuxThreads)
    tau_aux_finalize(const float* __restrict__ partial, int nblk, AuxShape s, float* __restrict__ stats) {
  const int layer = blockIdx.x;
  const float* pl = partial + (long long)layer * nblk * 3;
  double a[3] = {0.0, 0.0, 0.0};
  for (int i = threadIdx.x; i < nblk; i += kAuxThreads)
#pragma unroll
    for (int k = 0; k < 3; ++k) a[k] += (double)pl[i * 3 + k];
  __shared__ double red[3][kAuxWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    double v = a[k];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[k][warp] = v;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    double v = 0.0;
    for (int w = 0; w < kAuxWarps; ++w) v += red[threadIdx.x][w];
    const double den = threadIdx.x == 1 ? (double)s.m * s.B * s.t_out * s.H : (double)s.N;
    stats[layer * 3 + threadIdx.x] = threadIdx.x == 1 && s.m == 0 ? 0.f : (float)(v / den);
  }
}

// Lanes per row of the vector path, or 0 when the scalar path serves W.
template <typename E>
int vec_lanes(int W, const void* const* ptrs, int n) {
  constexpr int NV = VecOf<E>::n;
  if (W % NV != 0) return 0;
  const int g = W / NV;
  if (g > 32 || (g & (g - 1)) != 0) return 0;
  for (int i = 0; i < n; ++i)
    if (reinterpret_cast<uintptr_t>(ptrs[i]) & 15) return 0;
  return g;
}

// Lanes per row of the wide path (2-byte fields, W = 32·G), or 0.
template <typename E>
int wide_lanes(int W, const void* const* ptrs, int n) {
  if (sizeof(E) != 2 || W % 32 != 0) return 0;
  const int g = W / 32;
  if (g != 1 && g != 2 && g != 4 && g != 8) return 0;
  for (int i = 0; i < n; ++i)
    if (reinterpret_cast<uintptr_t>(ptrs[i]) & 15) return 0;
  return g;
}

template <typename E>
cudaError_t launch_fwd_narrow(const AuxPtrs& P, const AuxShape& s, int n_layers, int nblk,
                              float* partial, float* stats, float* row_ent, cudaStream_t st);

template <typename E>
cudaError_t launch_fwd_t(const AuxPtrs& P, const AuxShape& s, int n_layers, int nblk, float* partial,
                         float* stats, float* row_ent, cudaStream_t st) {
  const dim3 grid(nblk, n_layers);
  if constexpr (sizeof(E) != 2) {
    return launch_fwd_narrow<E>(P, s, n_layers, nblk, partial, stats, row_ent, st);
  } else {
    switch (wide_lanes<E>(s.W, P.tau, n_layers)) {
      case 1: tau_aux_fwd_wide<E, 1><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
      case 2: tau_aux_fwd_wide<E, 2><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
      case 4: tau_aux_fwd_wide<E, 4><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
      case 8: tau_aux_fwd_wide<E, 8><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
      default: return launch_fwd_narrow<E>(P, s, n_layers, nblk, partial, stats, row_ent, st);
    }
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  tau_aux_finalize<<<n_layers, kAuxThreads, 0, st>>>(partial, nblk, s, stats);
  return cudaGetLastError();
}

template <typename E>
cudaError_t launch_fwd_narrow(const AuxPtrs& P, const AuxShape& s, int n_layers, int nblk,
                              float* partial, float* stats, float* row_ent, cudaStream_t st) {
  const dim3 grid(nblk, n_layers);
  switch (vec_lanes<E>(s.W, P.tau, n_layers)) {
    case 1: tau_aux_fwd_vec<E, 1><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
    case 2: tau_aux_fwd_vec<E, 2><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
    case 4: tau_aux_fwd_vec<E, 4><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
    case 8: tau_aux_fwd_vec<E, 8><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
    case 16: tau_aux_fwd_vec<E, 16><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
    case 32: tau_aux_fwd_vec<E, 32><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
    default: tau_aux_fwd_scalar<E><<<grid, kAuxThreads, 0, st>>>(P, s, partial, row_ent); break;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  tau_aux_finalize<<<n_layers, kAuxThreads, 0, st>>>(partial, nblk, s, stats);
  return cudaGetLastError();
}

template <typename E>
cudaError_t launch_bwd_t(const AuxPtrs& P, const AuxShape& s, int n_layers, int nblk,
                         const float* d_stats, cudaStream_t st) {
  bool aligned = true;
  for (int i = 0; i < n_layers; ++i)
    if (reinterpret_cast<uintptr_t>(P.dtau[i]) & 15) aligned = false;
  const dim3 grid(nblk, n_layers);
  if constexpr (sizeof(E) == 2) {
    switch (aligned ? wide_lanes<E>(s.W, P.tau, n_layers) : 0) {
      case 1: tau_aux_bwd_wide<E, 1><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); return cudaGetLastError();
      case 2: tau_aux_bwd_wide<E, 2><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); return cudaGetLastError();
      case 4: tau_aux_bwd_wide<E, 4><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); return cudaGetLastError();
      case 8: tau_aux_bwd_wide<E, 8><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); return cudaGetLastError();
      default: break;
    }
  }
  switch (aligned ? vec_lanes<E>(s.W, P.tau, n_layers) : 0) {
    case 1: tau_aux_bwd_vec<E, 1><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); break;
    case 2: tau_aux_bwd_vec<E, 2><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); break;
    case 4: tau_aux_bwd_vec<E, 4><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); break;
    case 8: tau_aux_bwd_vec<E, 8><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); break;
    case 16: tau_aux_bwd_vec<E, 16><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); break;
    case 32: tau_aux_bwd_vec<E, 32><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); break;
    default: tau_aux_bwd_scalar<E><<<grid, kAuxThreads, 0, st>>>(P, s, d_stats); break;
  }
  return cudaGetLastError();
}

}  // namespace

AuxShape aux_shape(int B, int T, int H, int W) {
  AuxShape s{};
  s.B = B; s.T = T; s.H = H; s.W = W;
  s.N = (long long)B * T * H;
  // consistency: w1 ∈ [1, min(W−2, 4)], skipped when W < 3, T < 3 or the
  // last start m+1 reaches T (model.py:551-562)
  s.m = 0;
  if (W >= 3 && T >= 3) {
    const int m = W - 2 < 4 ? W - 2 : 4;
    if (m + 1 < T) {
      s.m = m;
      s.t_out = T - (m + 1);
    }
  }
  s.inv_n = 1.f / (float)s.N;
  s.inv_w = 1.f / (float)W;
  s.inv_cons = s.m > 0 ? 1.f / ((float)s.m * (float)B * (float)s.t_out * (float)H) : 0.f;
  s.div_h = make_fastdiv((uint32_t)H);
  s.div_t = make_fastdiv((uint32_t)T);
  return s;
}

// Blocks per layer: two 256-thread blocks per SM over all layers — the
// resident count of the wide kernels at their register use, so the grid is
// one wave — never more than the rows need.
int aux_blocks(const AuxShape& s, int n_layers, int sms) {
  const long long rows_per_block = (long long)kAuxWarps * 4;
  long long need = (s.N + rows_per_block - 1) / rows_per_block;
  long long cap = (long long)sms * 2 / n_layers;
  if (cap < 1) cap = 1;
  long long nb = need < cap ? need : cap;
  return (int)(nb < 1 ? 1 : nb);
}

cudaError_t launch_tau_aux_fwd(const bozo_tau_aux_fwd_args& a, int nblk, float* partial,
                               cudaStream_t st) {
  AuxPtrs P{};
  for (int i = 0; i < a.n_layers; ++i) P.tau[i] = a.tau[i];
  const AuxShape s = aux_shape(a.B, a.T, a.H, a.W);
  switch (a.dtype) {
    case BOZO_DT_F32: return launch_fwd_t<float>(P, s, a.n_layers, nblk, partial, a.stats, a.row_ent, st);
    case BOZO_DT_BF16: return launch_fwd_t<__nv_bfloat16>(P, s, a.n_layers, nblk, partial, a.stats, a.row_ent, st);
    default: return launch_fwd_t<__half>(P, s, a.n_layers, nblk, partial, a.stats, a.row_ent, st);
  }
}

// Row mode is served by the wide kernels only.
bool tau_aux_row_mode_ok(const bozo_tau_aux_bwd_args& a) {
  if (a.dtype == BOZO_DT_BF16) return wide_lanes<__nv_bfloat16>(a.W, a.tau, a.n_layers) != 0;
  if (a.dtype == BOZO_DT_F16) return wide_lanes<__half>(a.W, a.tau, a.n_layers) != 0;
  return false;
}

cudaError_t launch_tau_aux_bwd(const bozo_tau_aux_bwd_args& a, int nblk, cudaStream_t st) {
  AuxPtrs P{};
  const bool rows = a.row_coef[0] != nullptr;
  for (int i = 0; i < a.n_layers; ++i) {
    P.tau[i] = a.tau[i];
    P.dtau[i] = rows ? static_cast<void*>(a.row_coef[i]) : a.d_tau[i];
  }
  if (rows) {
    const AuxShape s = aux_shape(a.B, a.T, a.H, a.W);
    const dim3 grid(nblk, a.n_layers);
    const int g = a.dtype == BOZO_DT_BF16 ? wide_lanes<__nv_bfloat16>(a.W, a.tau, a.n_layers)
                                          : wide_lanes<__half>(a.W, a.tau, a.n_layers);
#define BOZO_ROWCOEF(E)                                                                          \
  switch (g) {                                                                                   \
    case 1: tau_aux_rowcoef_wide<E, 1><<<grid, kAuxThreads, 0, st>>>(P, s, a.d_stats); break;   \
    case 2: tau_aux_rowcoef_wide<E, 2><<<grid, kAuxThreads, 0, st>>>(P, s, a.d_stats); break;   \
    case 4: tau_aux_rowcoef_wide<E, 4><<<grid, kAuxThreads, 0, st>>>(P, s, a.d_stats); break;   \
    default: tau_aux_rowcoef_wide<E, 8><<<grid, kAuxThreads, 0, st>>>(P, s, a.d_stats); break;  \
  }
    if (a.dtype == BOZO_DT_BF16) {
      BOZO_ROWCOEF(__nv_bfloat16)
    } else {
      BOZO_ROWCOEF(__half)
    }
#undef BOZO_ROWCOEF
    return cudaGetLastError();
  }
  const AuxShape s = aux_shape(a.B, a.T, a.H, a.W);
  switch (a.dtype) {
    case BOZO_DT_F32: return launch_bwd_t<float>(P, s, a.n_layers, nblk, a.d_stats, st);
    case BOZO_DT_BF16: return launch_bwd_t<__nv_bfloat16>(P, s, a.n_layers, nblk, a.d_stats, st);
    default: return launch_bwd_t<__half>(P, s, a.n_layers, nblk, a.d_stats, st);
  }
}

}  // namespace bozo
