// tc_bwd.cu — tcgen05 / TMA / TMEM backward of the local tension operator
// for bf16 Q/K/V/dO with HD = 64 and W ≤ 128 (sm_100a).
//
// Math (τ = σ(x), x = Rq_t·Rk_s/scale + bias, valid band 1 ≤ t−s ≤ W):
//   dτ_ts = α_t·(dO_t·V_s) + β_t + dTau_ts
//   ds_ts = dτ_ts·τ_ts(1−τ_ts)/scale
//   dV_s  = Σ_t α_t τ_ts dO_t,  dK_s = R_sᵀ Σ_t ds_ts Rq_t,  dQ_t = R_tᵀ Σ_s ds_ts Rk_s
// with α/β from the normalisation: raw α=1, β=0 (triton_tension/kernel.py:
// 130-341); τ-mass α=1/max(m,ε), β=−α·(dO_t·out_t) if m ≥ ε else 0
// (autograd of model.py:257-258); count α=1/max(min(t,W),1), β=0
// (model.py:261-264).  α/β come from a small coalesced pre-pass
// (alpha_beta_kernel) and are bulk-copied into shared memory with each query
// tile.  Q and K arrive already rotated (the forward's RoPE copies), so RoPE
// appears here only as the inverse rotation of dQ and dK.
//
// Work decomposition: key tiles of 128 rows, flattened b-h-major; one
// persistent CTA per SM walks a contiguous range.  The queries that see key
// tile i are query tile i and the first W rows of query tile i+1; they are
// visited as 64-query sub-chunks (i,0-63) (i,64-127) (i+1,0-63) (i+1,64-127).
// Per sub-chunk:
//   Sᵀ = K_i·Q_hᵀ, dPᵀ = V_i·dO_hᵀ     TMEM, M = 128 keys, N = 64, double-buffered
//   epilogue → Pᵀ = α·τ, dSᵀ = ds      bf16 shared memory, double-buffered
//   dV += Pᵀ·dO_h, dK += dSᵀ·Q_h       TMEM, complete per key tile
// and after both halves of a query tile:
//   dQ_j += dS_j·K_i                   (A = both dSᵀ halves read MN-major)
// into one of two TMEM accumulators: query tile i+1 starts in iteration i and
// completes in i+1, so no partial sums leave the SM and no atomics are used.
// Two threads issue MMAs — one the Sᵀ/dPᵀ of every sub-chunk, one the
// consumers — so Sᵀ/dPᵀ run ahead of the consumers and tensor cores and the
// epilogue overlap.  A CTA whose range
// starts mid-sequence first runs a warm-up pass over key tile i−1 for dQ_i.
//
// Warps: 0 TMA; 1 MMA (Sᵀ/dPᵀ); 14 MMA (consumers); 2/3/12/13 output (dQ/dK/dV
// from TMEM → inverse RoPE → shared staging → TMA store); 4-11 epilogue.
// All waits are bounded
// (tc_ptx.cuh).
#include <algorithm>
#include <type_traits>

#include "tc.cuh"
#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace bozo {
namespace {

using namespace tc;

constexpr int kTile = kTcTile;
constexpr int kHD = kTcHD;
constexpr int kTileBytes = kTile * kHD * 2;  // 16 KiB
constexpr int kHalfBytes = kTileBytes;       // one [128 x 64] bf16 Pᵀ or dSᵀ buffer
constexpr int kThreads = 15 * 32;
constexpr int kErrBwd = 0x200;
constexpr float kEpsOverLn2 = 1.44269504e-8f;  // 1e-8 / ln 2

// TMEM columns: Sᵀ/dPᵀ buffer b at 128b (Sᵀ) and 128b+64 (dPᵀ)
constexpr uint32_t kColDK = 256, kColDV = 320, kColDQ = 384;

struct BwdTC {
  int B, T, H, W, Wr, nT, total, tpad;
  float half_inv_scale, ds_scale;  // 0.5/scale, 0.25/scale
  const float* theta;              // RoPE frequencies [32] or null (no RoPE)
  const float* bias;
  long long bs0, bs1, bs2;
  const void* dtau;                // [B,T,H,W] contiguous (bf16, fp32 with kF32) or null
  const float* coef;               // [3][B·H, tpad]: α/2, α·c, β·c
  void* dq;                        // [B,T,H,64] contiguous outputs (dQ/dK fp32 with kF32)
  void* dk;
  void* dv;
  int* err;
};

struct __align__(8) Bars {
  uint64_t kv_full[2], kv_empty[2];
  uint64_t q_full[2], q_empty[2];
  uint64_t sdp_full[2], sdp_free[2], p_full[2], p_free[2];
  uint64_t acc_full, dkv_free, dq_free[2];
  uint64_t aux_staged, aux_stored;
  uint32_t tmem_base;
};

struct Layout {
  uint32_t k, v, q, dout, pds, stage, ab, theta, bars, total;
};

// nplanes per-query-row coefficient planes per query slot: α/2, α·c, β·c
// (+ a1·c and 1/D of the per-row τ cotangent when kAux)
__host__ __device__ inline Layout bwd_layout(int nplanes) {
  Layout L;
  L.k = 0;
  L.v = L.k + 2 * kTileBytes;
  L.q = L.v + 2 * kTileBytes;
  L.dout = L.q + 2 * kTileBytes;
  L.pds = L.dout + 2 * kTileBytes;       // [P0][dS0][P1][dS1], 16 KiB each
  L.stage = L.pds + 4 * kHalfBytes;      // dQ output staging tile
  L.ab = L.stage + kTileBytes;           // coefficients: float[2 slots][nplanes][128]
  L.theta = L.ab + 2 * nplanes * kTile * 4;  // RoPE θ: float[32]
  L.bars = L.theta + 32 * 4;
  L.total = L.bars + (uint32_t)sizeof(Bars);
  return L;
}

// Per query row: the epilogue's coefficients α/2, α·c and β·c (c = 1/(4·scale))
// of the normalisation, into padded rows [B·H, tpad] (rows t ≥ T are 0).
// τ-mass needs D = dO·out per row: eight threads share one 128-byte bf16 row
// (one 16-byte chunk each) and rows are walked in memory order (t, h) within
// batch b = blockIdx.y, so every warp load is four whole rows and the index
// math is one 32-bit division per row.  The grid-stride step is a multiple of
// 32 threads, so the 8-lane shuffle groups stay whole and warp-uniform.
// With a per-row τ cotangent (aux_row: a1 | a0 | 1/D planes over B·H·T rows)
// its constant a0 joins β and a1·c, 1/D fill two more planes.
__global__ void alpha_beta_kernel(int B, int T, int H, int W, int tpad, int norm, float ds_scale,
                                  const float* __restrict__ row_mass, DevT4 dout, DevT4 out,
                                  float* __restrict__ a_half, float* __restrict__ a_ds,
                                  float* __restrict__ b_ds, const float* __restrict__ aux_row,
                                  float* __restrict__ a1_ds, float* __restrict__ inv_d) {
  const int bb = blockIdx.y;
  const int n8 = T * H * 8;  // threads needed for this batch row
  const int stride = gridDim.x * blockDim.x;
  const int c = threadIdx.x & 7;
  const __nv_bfloat16* dob = static_cast<const __nv_bfloat16*>(dout.p) + bb * dout.sb;
  const __nv_bfloat16* oub = static_cast<const __nv_bfloat16*>(out.p) + bb * out.sb;
  for (int base = blockIdx.x * blockDim.x; base < n8; base += stride) {
    const int idx = base + threadIdx.x;
    const bool live = idx < n8;
    const int rr = live ? idx >> 3 : 0;  // (t, h) row within the batch
    const int t = rr / H, h = rr - t * H;
    // the row's τ-mass is loaded with the row (one latency per iteration, not two)
    const float m = (norm == BOZO_NORM_MASS && live) ? __ldg(row_mass + (long long)(bb * H + h) * T + t) : 0.f;
    float dd = 0.f;
    if (norm == BOZO_NORM_MASS && live) {
      const uint4 x = __ldg(reinterpret_cast<const uint4*>(dob + (long long)t * dout.st + h * dout.sh) + c);
      const uint4 y = __ldg(reinterpret_cast<const uint4*>(oub + (long long)t * out.st + h * out.sh) + c);
      const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
      const uint32_t ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 u = *reinterpret_cast<const __nv_bfloat162*>(&xs[e]);
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&ys[e]);
        dd = fmaf(__low2float(u), __low2float(v), dd);
        dd = fmaf(__high2float(u), __high2float(v), dd);
      }
    }
    if (norm == BOZO_NORM_MASS) {
      dd += __shfl_xor_sync(0xffffffffu, dd, 4);
      dd += __shfl_xor_sync(0xffffffffu, dd, 2);
      dd += __shfl_xor_sync(0xffffffffu, dd, 1);
    }
    if (live && c == 0) {
      const int bh = bb * H + h;
      float a, b = 0.f;
      if (norm == BOZO_NORM_MASS) {
        a = 1.f / fmaxf(m, kMassEps);
        b = m >= kMassEps ? -dd * a : 0.f;
      } else if (norm == BOZO_NORM_COUNT) {
        a = 1.f / (float)max(min(t, W), 1);
      } else {
        a = 1.f;
      }
      const long long o = (long long)bh * tpad + t;
      if (aux_row) {
        const long long nr = (long long)B * H * T, ar = (long long)bh * T + t;
        b += aux_row[nr + ar];
        a1_ds[o] = aux_row[ar] * ds_scale;
        inv_d[o] = aux_row[2 * nr + ar];
      }
      a_half[o] = 0.5f * a;
      a_ds[o] = a * ds_scale;
      b_ds[o] = b * ds_scale;
    }
  }
  // padding rows t ∈ [T, tpad) of this batch's heads
  const int pad = tpad - T;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H * pad; i += stride) {
    const long long o = (long long)(bb * H + i / pad) * tpad + T + (i % pad);
    a_half[o] = 0.f;
    a_ds[o] = 0.f;
    b_ds[o] = 0.f;
    if (aux_row) {
      a1_ds[o] = 0.f;
      inv_d[o] = 0.f;
    }
  }
}

// Deterministic per-CTA schedule shared by every role.
struct Step {
  int bh, i;
  bool warm, first_of_seg, has_c1, last;
};

__device__ __forceinline__ Step step_of(int u, int u0, int u1, int nT) {
  Step s;
  s.bh = u / nT;
  s.i = u % nT;
  s.warm = (u == u0) && s.i >= 1;
  s.first_of_seg = (u == u0) || s.i == 0;
  s.has_c1 = s.i + 1 < nT;
  s.last = (u + 1 == u1);
  return s;
}

// A 64-query sub-chunk as the MMA issuer tracks it.
struct Sub {
  int n, it, ks, qs, hh, bq, kk0;
  int bh, ikey, c;  // key tile (bh, ikey) against query tile ikey + c
  int kidx, qidx;  // load index of a key / query tile first used here, else −1
  bool zero, warm, dq, dq_acc, kv_first, last_of_iter, rel_q, rel_k;
};

// Generates the CTA's sub-chunks in order (the same order the epilogue walks).
struct SubGen {
  int u, u0, u1, nT, Wr, idx, it, n, nk, nq, qslot, kslot;
  bool c1h1_zero;
  Step st;     // step of key tile u (recomputed only when u advances)
  int st_u = -1;
  __device__ bool next(Sub& s) {
    while (u < u1) {
      if (st_u != u) {
        st = step_of(u, u0, u1, nT);
        st_u = u;
      }
      const int kinds = (st.warm ? 2 : 0) + 2 + (st.has_c1 ? 2 : 0);
      if (idx >= kinds) {
        ++u;
        ++it;
        idx = 0;
        continue;
      }
      int kind = idx++;
      if (!st.warm) kind += 2;  // 0,1 warm · 2,3 chunk 0 · 4,5 chunk 1
      const int hh = kind & 1;
      s = Sub{};
      s.n = n++;
      s.it = it;
      s.hh = hh;
      s.bh = st.bh;
      s.ikey = kind < 2 ? st.i - 1 : st.i;
      s.c = (kind < 2 || kind >= 4) ? 1 : 0;
      s.kidx = s.qidx = -1;
      const int bq_i = st.i & 1;
      if (kind < 2) {  // warm-up over key tile i−1 for dQ_i
        if (hh == 0) {
          s.kidx = nk; kslot = nk & 1; ++nk;
          s.qidx = nq; qslot = nq & 1; ++nq;
        }
        s.ks = kslot; s.qs = qslot;
        s.zero = hh == 1 && c1h1_zero; s.warm = true;
        s.dq = true; s.dq_acc = false; s.bq = bq_i; s.kk0 = (kTcTile - Wr) / 16;
        s.rel_k = hh == 1;  // the warm-up key tile has no outputs: free it here
      } else if (kind < 4) {  // chunk 0: query tile i
        if (hh == 0) {
          if (!st.warm && st.first_of_seg) { s.qidx = nq; qslot = nq & 1; ++nq; }
          s.kidx = nk; kslot = nk & 1; ++nk;
        }
        s.ks = kslot; s.qs = qslot;
        s.kv_first = hh == 0;
        s.dq = true; s.dq_acc = st.warm || !st.first_of_seg; s.bq = bq_i; s.kk0 = 0;
        s.rel_q = hh == 1;
        s.last_of_iter = hh == 1 && !st.has_c1;
      } else {  // chunk 1: the first rows of query tile i+1
        if (hh == 0) { s.qidx = nq; qslot = nq & 1; ++nq; }
        s.ks = kslot; s.qs = qslot;
        s.zero = hh == 1 && c1h1_zero;
        s.dq = !st.last; s.dq_acc = false; s.bq = bq_i ^ 1; s.kk0 = (kTcTile - Wr) / 16;
        s.rel_q = hh == 1 && st.last;
        s.last_of_iter = hh == 1;
      }
      return true;
    }
    return false;
  }
};

// kF32: the τ cotangent arrives in fp32 and dQ/dK leave in fp32 (the
// reference's gradient dtypes for fp32 Q/K, ops.py:186-187), from bf16
// operand copies of Q/K; dV stays bf16.
template <bool kBias, bool kDTau, bool kAux, bool kF32>
__global__ void __launch_bounds__(kThreads, 1)
    tc_bwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmdo,
                  const __grid_constant__ CUtensorMap tmdq, const __grid_constant__ CUtensorMap tmdk,
                  const __grid_constant__ CUtensorMap tmdv, const BwdTC p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int NP = kAux ? 5 : 3;  // coefficient planes per query slot
  const Layout L = bwd_layout(NP);
  uint8_t* sK = smem + L.k;
  uint8_t* sV = smem + L.v;
  uint8_t* sQ = smem + L.q;
  uint8_t* sDO = smem + L.dout;
  uint8_t* sPDS = smem + L.pds;
  uint8_t* sStage = smem + L.stage;
  float* sAB = reinterpret_cast<float*>(smem + L.ab);
  float* sTheta = reinterpret_cast<float*>(smem + L.theta);
  Bars* bar = reinterpret_cast<Bars*>(smem + L.bars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = (int)((long long)blockIdx.x * p.total / gridDim.x);
  const int u1 = (int)((long long)(blockIdx.x + 1) * p.total / gridDim.x);
  const int nT = p.nT, Wr = p.Wr, H = p.H, W = p.W;
  // the second 64-query half of query tile i+1 is outside every band when Wr ≤ 64
  const bool c1h1_zero = Wr <= 64;

  if (threadIdx.x < 32) sTheta[threadIdx.x] = p.theta ? __ldg(p.theta + threadIdx.x) : 0.f;
  const float* th = p.theta ? sTheta : nullptr;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->kv_full[s], 1);
      mbar_init(&bar->kv_empty[s], 1);
      mbar_init(&bar->q_full[s], 1);
      mbar_init(&bar->q_empty[s], 1);
      mbar_init(&bar->sdp_full[s], 1);
      mbar_init(&bar->sdp_free[s], 8);
      mbar_init(&bar->p_full[s], 8);
      mbar_init(&bar->p_free[s], 1);
      mbar_init(&bar->dq_free[s], 4);
    }
    mbar_init(&bar->aux_staged, 4);
    mbar_init(&bar->aux_stored, 1);
    mbar_init(&bar->acc_full, 1);
    mbar_init(&bar->dkv_free, 4);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&bar->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bar->tmem_base;
  int* err = p.err;

  if (warp == 0) {
    // ─────────────────────────── TMA producer ───────────────────────────
    if (lane == 0) {
      prefetch_tmap(&tmq); prefetch_tmap(&tmk); prefetch_tmap(&tmv); prefetch_tmap(&tmdo);
      prefetch_tmap(&tmdq); prefetch_tmap(&tmdk); prefetch_tmap(&tmdv);
      int nk = 0, nq = 0;
      bool ok = true;
      auto load_key = [&](int bh, int jj) {
        const int s = nk & 1;
        if (nk >= 2) ok = ok && mbar_wait(&bar->kv_empty[s], ((nk >> 1) - 1) & 1, err, kErrBwd | 1);
        if (!ok) return;
        mbar_arrive_expect_tx(&bar->kv_full[s], 2 * kTileBytes);
        tma_load_4d(sK + s * kTileBytes, &tmk, &bar->kv_full[s], 0, bh % H, jj * kTile, bh / H);
        tma_load_4d(sV + s * kTileBytes, &tmv, &bar->kv_full[s], 0, bh % H, jj * kTile, bh / H);
        ++nk;
      };
      auto load_query = [&](int bh, int jj) {
        const int s = nq & 1;
        if (nq >= 2) ok = ok && mbar_wait(&bar->q_empty[s], ((nq >> 1) - 1) & 1, err, kErrBwd | 2);
        if (!ok) return;
        mbar_arrive_expect_tx(&bar->q_full[s], 2 * kTileBytes + NP * kTile * 4);
        tma_load_4d(sQ + s * kTileBytes, &tmq, &bar->q_full[s], 0, bh % H, jj * kTile, bh / H);
        tma_load_4d(sDO + s * kTileBytes, &tmdo, &bar->q_full[s], 0, bh % H, jj * kTile, bh / H);
        const long long ab_off = (long long)bh * p.tpad + jj * kTile;
        const long long plane = (long long)p.B * H * p.tpad;
#pragma unroll
        for (int z = 0; z < NP; ++z)
          bulk_load_1d(sAB + (s * NP + z) * kTile, p.coef + z * plane + ab_off, kTile * 4, &bar->q_full[s]);
        ++nq;
      };
      for (int u = u0; u < u1 && ok; ++u) {
        const Step st = step_of(u, u0, u1, nT);
        if (st.warm) load_key(st.bh, st.i - 1);
        if (st.first_of_seg) load_query(st.bh, st.i);
        load_key(st.bh, st.i);
        if (st.has_c1) load_query(st.bh, st.i + 1);
      }
    }
  } else if (warp == 1 || warp == 14) {
    // ──────────── MMA issuers: warp 1 Sᵀ/dPᵀ, warp 14 consumers ────────────
    // Two issuing threads: each walks the same sub-chunk sequence with a
    // short, wait-only loop, so neither waits behind the other's MMAs.  Each
    // commit covers only its own thread's MMAs; that suffices because the
    // consumers of a sub-chunk start after the epilogue consumed its Sᵀ/dPᵀ
    // (p_full), i.e. after every producer MMA that read the same tiles.
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(128, 64, false, false);   // Sᵀ/dPᵀ: A,B K-major
      const uint32_t id_kv = idesc_bf16(128, kHD, false, true);  // dV/dK: A K-major, B MN-major
      const uint32_t id_q = idesc_bf16(128, kHD, true, true);    // dQ: A (dSᵀ) MN-major
      constexpr uint64_t kTD = kTileBytes >> 4;
      constexpr uint64_t kHD16 = kHalfBytes >> 4;
      const uint64_t dK0 = sdesc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t dV0 = sdesc_sw128(smem_u32(sV), 16, 1024);
      const uint64_t dQ0 = sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t dDO0 = sdesc_sw128(smem_u32(sDO), 16, 1024);
      const uint64_t dPDS = sdesc_sw128(smem_u32(sPDS), 16, 1024);
      // both dSᵀ halves as the MN-major A operand of dQ (query blocks 32 KiB apart)
      const uint64_t dDSmn = sdesc_sw128(smem_u32(sPDS) + kHalfBytes, 2 * kHalfBytes, 1024);
      int dq_started[2] = {0, 0};
      bool ok = true;

      auto issue_sdp = [&](const Sub& s) {
        const int b = s.n & 1;
        if (!s.zero) {
          const uint64_t rowoff = (uint64_t)(64 * s.hh) * 8;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            mma_bf16(tbase + 128 * b, dK0 + s.ks * kTD + 2 * kk, dQ0 + s.qs * kTD + rowoff + 2 * kk, id_s, kk > 0);
            mma_bf16(tbase + 128 * b + 64, dV0 + s.ks * kTD + 2 * kk, dDO0 + s.qs * kTD + rowoff + 2 * kk, id_s, kk > 0);
          }
        }
        mma_commit(&bar->sdp_full[b]);
      };
      // consumer MMAs of a sub-chunk (its Pᵀ/dSᵀ are in shared buffer n&1)
      auto issue_consumers = [&](const Sub& s) {
        const int b = s.n & 1;
        if (!s.zero && !s.warm) {
          const uint64_t a_p = dPDS + (uint64_t)(2 * b) * kHD16;
          const uint64_t a_s = dPDS + (uint64_t)(2 * b + 1) * kHD16;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t rowoff = (uint64_t)(64 * s.hh + 16 * kk) * 8;  // 128 B rows in 16 B units
            const uint32_t acc = (s.kv_first && kk == 0) ? 0u : 1u;
            mma_bf16(tbase + kColDV, a_p + 2 * kk, dDO0 + s.qs * kTD + rowoff, id_kv, acc);
            mma_bf16(tbase + kColDK, a_s + 2 * kk, dQ0 + s.qs * kTD + rowoff, id_kv, acc);
          }
        }
        if (s.hh == 1) {
          if (s.dq) {
            if (!s.dq_acc) ++dq_started[s.bq];
            uint32_t acc = s.dq_acc ? 1u : 0u;
            for (int kk = s.kk0; kk < 8; ++kk) {
              mma_bf16(tbase + kColDQ + 64 * s.bq, dDSmn + kk * 128, dK0 + s.ks * kTD + kk * 128, id_q, acc);
              acc = 1;
            }
          }
          mma_commit(&bar->p_free[0]);
          mma_commit(&bar->p_free[1]);
          if (s.rel_q) mma_commit(&bar->q_empty[s.qs]);
        }
        if (s.last_of_iter) mma_commit(&bar->acc_full);
        if (s.rel_k) mma_commit(&bar->kv_empty[s.ks]);
      };

      SubGen gen{u0, u0, u1, nT, Wr, 0, 0, 0, 0, 0, 0, 0, c1h1_zero};
      Sub s{};
      if (warp == 1) {
        while (ok && gen.next(s)) {
          if (s.kidx >= 0) ok = mbar_wait(&bar->kv_full[s.kidx & 1], (s.kidx >> 1) & 1, err, kErrBwd | 16);
          if (ok && s.qidx >= 0) ok = mbar_wait(&bar->q_full[s.qidx & 1], (s.qidx >> 1) & 1, err, kErrBwd | 17);
          if (ok && s.n >= 2) ok = mbar_wait(&bar->sdp_free[s.n & 1], ((s.n >> 1) - 1) & 1, err, kErrBwd | 18);
          if (!ok) break;
          tc_fence_after();
          issue_sdp(s);
        }
      } else {
        while (ok && gen.next(s)) {
          ok = mbar_wait(&bar->p_full[s.n & 1], (s.n >> 1) & 1, err, kErrBwd | 19);
          if (ok && s.kv_first && s.it >= 1) ok = mbar_wait(&bar->dkv_free, (s.it - 1) & 1, err, kErrBwd | 20);
          if (ok && s.hh == 1 && s.dq && !s.dq_acc && dq_started[s.bq] >= 1)
            ok = mbar_wait(&bar->dq_free[s.bq], (dq_started[s.bq] - 1) & 1, err, kErrBwd | 21);
          if (!ok) break;
          tc_fence_after();
          issue_consumers(s);
        }
      }
    }
  } else if (warp < 4 || warp == 12 || warp == 13) {
    // ──────── output warps: dQ/dK/dV of each key tile ────────
    const int r = (warp & 3) * 32 + lane;  // == TMEM lane of this thread
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    bool ok = true;
    // key slot of each iteration's key tile, replaying the TMA load order
    int nk = 0;
    auto key_slot_of = [&](int u) {
      const Step st = step_of(u, u0, u1, nT);
      if (st.warm) ++nk;
      const int s = nk & 1;
      ++nk;
      return s;
    };
    for (int u = u0, it = 0; u < u1 && ok; ++u, ++it) {
      const Step st = step_of(u, u0, u1, nT);
      const int ks_cur = key_slot_of(u);
      ok = mbar_wait(&bar->acc_full, it & 1, err, kErrBwd | 25);
      if (!ok) break;
      __syncwarp();
      tc_fence_after();
      const int bq = st.i & 1, b = st.bh / H, h = st.bh % H;
      const int pos = st.i * kTile + r;
      const bool rope = th != nullptr && pos < p.T;
      // K_i / V_i slots are dead once acc_full fired: stage dK and dV there
      const uint32_t kst = smem_u32(sK + ks_cur * kTileBytes), vst = smem_u32(sV + ks_cur * kTileBytes);
      const uint32_t qst = smem_u32(sStage);
      uint32_t g[64];
      // dV, then dK leave TMEM first: the next key tile's dV/dK MMAs wait only
      // for that (dkv_free), not for the rotation and staging below
      tmem_ld32_wait(tbase + lane_off + kColDV, g);
      tmem_ld32_wait(tbase + lane_off + kColDV + 32, g + 32);
#pragma unroll
      for (int z = 0; z < 8; ++z) {
        uint32_t w4[4];
#pragma unroll
        for (int y = 0; y < 4; ++y)
          w4[y] = pack_bf16(__uint_as_float(g[8 * z + 2 * y]), __uint_as_float(g[8 * z + 2 * y + 1]));
        st_shared_v4(vst + sw128_off(r, z), w4[0], w4[1], w4[2], w4[3]);
      }
      tmem_ld32_wait(tbase + lane_off + kColDK, g);
      tmem_ld32_wait(tbase + lane_off + kColDK + 32, g + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->dkv_free);
      // dQ: the staging tile must have been read out by the previous store
      if (it >= 1) ok = mbar_wait(&bar->aux_stored, (it - 1) & 1, err, kErrBwd | 26);
      if (!ok) break;
      // inverse RoPE of dK (registers) and dQ (TMEM, 8 frequencies at a time):
      // frequency i pairs columns i and 32+i; one cos/sin serves both rows
      const uint32_t qc = tbase + lane_off + kColDQ + 64 * bq;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        uint32_t gq[16];
        tmem_ld8x2_wait(qc + 8 * c8, qc + 32 + 8 * c8, gq);  // columns [8c8, +8) and [32+8c8, +8)
        float ok8[16], oq8[16];
#pragma unroll
        for (int z = 0; z < 8; ++z) {
          float cs = 1.f, sn = 0.f;
          if (rope) rope_cs(pos, th[c8 * 8 + z], cs, sn);
          const float k1 = __uint_as_float(g[8 * c8 + z]), k2 = __uint_as_float(g[32 + 8 * c8 + z]);
          const float q1 = __uint_as_float(gq[z]), q2 = __uint_as_float(gq[8 + z]);
          ok8[z] = k1 * cs + k2 * sn;
          ok8[8 + z] = k2 * cs - k1 * sn;
          oq8[z] = q1 * cs + q2 * sn;
          oq8[8 + z] = q2 * cs - q1 * sn;
        }
        if constexpr (kF32) {
          // row pos of dK (key tile i) and of dQ (query tile i), columns
          // [8c8, 8c8+8) and [32+8c8, +8), straight to global memory
          if (pos < p.T) {
            const long long row = ((long long)(b * p.T + pos) * H + h) * kHD;
            float4* gk = reinterpret_cast<float4*>(static_cast<float*>(p.dk) + row);
            float4* gq = reinterpret_cast<float4*>(static_cast<float*>(p.dq) + row);
            gk[2 * c8] = make_float4(ok8[0], ok8[1], ok8[2], ok8[3]);
            gk[2 * c8 + 1] = make_float4(ok8[4], ok8[5], ok8[6], ok8[7]);
            gk[8 + 2 * c8] = make_float4(ok8[8], ok8[9], ok8[10], ok8[11]);
            gk[8 + 2 * c8 + 1] = make_float4(ok8[12], ok8[13], ok8[14], ok8[15]);
            gq[2 * c8] = make_float4(oq8[0], oq8[1], oq8[2], oq8[3]);
            gq[2 * c8 + 1] = make_float4(oq8[4], oq8[5], oq8[6], oq8[7]);
            gq[8 + 2 * c8] = make_float4(oq8[8], oq8[9], oq8[10], oq8[11]);
            gq[8 + 2 * c8 + 1] = make_float4(oq8[12], oq8[13], oq8[14], oq8[15]);
          }
        } else {
          st_shared_v4(kst + sw128_off(r, c8), pack_bf16(ok8[0], ok8[1]), pack_bf16(ok8[2], ok8[3]),
                       pack_bf16(ok8[4], ok8[5]), pack_bf16(ok8[6], ok8[7]));
          st_shared_v4(kst + sw128_off(r, 4 + c8), pack_bf16(ok8[8], ok8[9]), pack_bf16(ok8[10], ok8[11]),
                       pack_bf16(ok8[12], ok8[13]), pack_bf16(ok8[14], ok8[15]));
          st_shared_v4(qst + sw128_off(r, c8), pack_bf16(oq8[0], oq8[1]), pack_bf16(oq8[2], oq8[3]),
                       pack_bf16(oq8[4], oq8[5]), pack_bf16(oq8[6], oq8[7]));
          st_shared_v4(qst + sw128_off(r, 4 + c8), pack_bf16(oq8[8], oq8[9]), pack_bf16(oq8[10], oq8[11]),
                       pack_bf16(oq8[12], oq8[13]), pack_bf16(oq8[14], oq8[15]));
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar->dq_free[bq]);
        mbar_arrive(&bar->aux_staged);
      }
      if (warp == 2 && lane == 0) {
        ok = mbar_wait(&bar->aux_staged, it & 1, err, kErrBwd | 27);
        if (ok) {
          if constexpr (!kF32) tma_store_4d(&tmdk, sK + ks_cur * kTileBytes, 0, h, st.i * kTile, b);
          tma_store_4d(&tmdv, sV + ks_cur * kTileBytes, 0, h, st.i * kTile, b);
          if constexpr (!kF32) tma_store_4d(&tmdq, sStage, 0, h, st.i * kTile, b);
          bulk_commit_group();
          bulk_wait_group_read0();
          mbar_arrive(&bar->kv_empty[ks_cur]);  // the TMA may refill this key slot
          mbar_arrive(&bar->aux_stored);
        }
      }
      __syncwarp();
    }
    if (warp == 2 && lane == 0) bulk_wait_group0();
  } else {
    // ─────────────────────────── epilogue (8 warps) ───────────────────────────
    const int e = warp - 4;
    const int qd = warp & 3;
    const int hf = e >> 2;  // which 32 query columns of the 64-wide sub-chunk
    const int r = qd * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const uint32_t pds = smem_u32(sPDS);
    int n = 0;
    bool ok = true;

    // One 64-query sub-chunk: key tile i_key, query tile i_key+c, half hh.
    // Thread = key row r; this warp covers query columns 32·hf … 32·hf+31 in
    // two 16-column pieces.  Per element (c = 1/(4·scale), th = tanh(x/2)):
    //   τ·α = α/2 + α/2·th,  ds = (α·c·dP + β·c + c·dTau)·(1 − th²)
    // Without per-element inputs both pieces' Sᵀ/dPᵀ leave TMEM under one
    // completion wait and the TMEM buffer is handed back before the element
    // math; with bias / τ cotangent gathers each piece loads after its gathers
    // were issued, so their global latency overlaps the TMEM load (the per-row
    // τ cotangent also loads per piece: its two extra coefficient planes leave
    // no room for both pieces' registers).
    auto subchunk = [&](int bh, int i_key, int c, int hh, int qs, bool zero) {
      const int b = n & 1;
      ok = ok && mbar_wait(&bar->sdp_full[b], (n >> 1) & 1, err, kErrBwd | 30);
      if (!ok) return;
      __syncwarp();
      tc_fence_after();
      const int bb = bh / H, h = bh % H;
      const int tq0 = (i_key + c) * kTile;
      const float* cf = sAB + qs * NP * kTile;  // α/2 | α·c | β·c (| a1·c | 1/D)
      bool band[2];
      int lo[2], cnt[2];
#pragma unroll
      for (int ss = 0; ss < 2; ++ss) {
        const int cq0 = 64 * hh + 32 * hf + 16 * ss;  // first query column (in tile)
        const int dmax = kTile * c + cq0 + 15 - qd * 32, dmin = kTile * c + cq0 - qd * 32 - 31;
        band[ss] = !zero && dmax >= 1 && dmin <= W;
        // this row's valid columns e ∈ [lo, lo+cnt) of the 16: 1 ≤ t−s ≤ W, t < T
        lo[ss] = r + 1 - kTile * c - cq0;
        const int hi = min(r + W - kTile * c - cq0 + 1, p.T - tq0 - cq0);
        cnt[ss] = max(hi - max(lo[ss], 0), 0);
        lo[ss] = max(lo[ss], 0);
      }
      uint32_t pk[2][8], dk[2][8];
      // element math of piece ss from its Sᵀ (R[0,16)) and dPᵀ (R[16,32))
      auto piece = [&](int ss, const uint32_t* R, const float* gb, const float* gd) {
        const int cq0 = 64 * hh + 32 * hf + 16 * ss;
#pragma unroll
        for (int e4 = 0; e4 < 16; e4 += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(cf + cq0 + e4);
          const float4 d4 = *reinterpret_cast<const float4*>(cf + kTile + cq0 + e4);
          const float4 b4 = *reinterpret_cast<const float4*>(cf + 2 * kTile + cq0 + e4);
          const float ah[4] = {a4.x, a4.y, a4.z, a4.w};
          const float ad[4] = {d4.x, d4.y, d4.z, d4.w};
          const float bd[4] = {b4.x, b4.y, b4.z, b4.w};
          float a1[4] = {0.f, 0.f, 0.f, 0.f}, ivd[4] = {0.f, 0.f, 0.f, 0.f};
          if constexpr (kAux) {
            const float4 u4 = *reinterpret_cast<const float4*>(cf + 3 * kTile + cq0 + e4);
            const float4 v4 = *reinterpret_cast<const float4*>(cf + 4 * kTile + cq0 + e4);
            a1[0] = u4.x; a1[1] = u4.y; a1[2] = u4.z; a1[3] = u4.w;
            ivd[0] = v4.x; ivd[1] = v4.y; ivd[2] = v4.z; ivd[3] = v4.w;
          }
          float pv[4], dv[4];
#pragma unroll
          for (int z = 0; z < 4; ++z) {
            const int e = e4 + z;
            const bool valid = (unsigned)(e - lo[ss]) < (unsigned)cnt[ss];
            float x = __uint_as_float(R[e]) * p.half_inv_scale;
            float dt = fmaf(ad[z], __uint_as_float(R[16 + e]), bd[z]);
            if constexpr (kBias) x += gb[e];
            if constexpr (kDTau) dt += gd[e];
            const float th = tanh_approx(x);
            if constexpr (kAux) {
              // per-row τ cotangent a1·(log2 q − 1e-8/(q·ln 2)) (its a0 is in β),
              // q = τ/D + 1e-8 at the recomputed τ = (1 + th)/2
              const float q = fmaf(fmaf(0.5f, th, 0.5f), ivd[z], 1e-8f);
              dt = fmaf(a1[z], fmaf(-kEpsOverLn2, __fdividef(1.f, q), __log2f(q)), dt);
            }
            pv[z] = valid ? fmaf(ah[z], th, ah[z]) : 0.f;
            dv[z] = valid ? dt * fmaf(-th, th, 1.f) : 0.f;
          }
          pk[ss][e4 >> 1] = pack_bf16(pv[0], pv[1]);
          pk[ss][(e4 >> 1) + 1] = pack_bf16(pv[2], pv[3]);
          dk[ss][e4 >> 1] = pack_bf16(dv[0], dv[1]);
          dk[ss][(e4 >> 1) + 1] = pack_bf16(dv[2], dv[3]);
        }
      };
      if constexpr (!(kBias || kDTau || kAux)) {
        uint32_t R[64];  // piece ss: Sᵀ at R[32ss], dPᵀ at R[32ss+16]
        const uint32_t col = tbase + lane_off + 128 * b + 32 * hf;
        if (band[0] && band[1]) tmem_ld16x4_wait(col, col + 64, col + 16, col + 80, R);
        else if (band[0]) tmem_ld16x2_wait(col, col + 64, R);
        else if (band[1]) tmem_ld16x2_wait(col + 16, col + 80, R + 32);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->sdp_free[b]);
#pragma unroll
        for (int ss = 0; ss < 2; ++ss) {
          if (band[ss]) {
            piece(ss, R + 32 * ss, nullptr, nullptr);
          } else {
#pragma unroll
            for (int z = 0; z < 8; ++z) pk[ss][z] = dk[ss][z] = 0u;
          }
        }
      } else {
#pragma unroll
        for (int ss = 0; ss < 2; ++ss) {
          const int cq0 = 64 * hh + 32 * hf + 16 * ss;
          if (band[ss]) {
            uint32_t R[32];  // Sᵀ | dPᵀ of this 16-column piece
            const uint32_t col = tbase + lane_off + 128 * b + 32 * hf + 16 * ss;
            // the optional per-element inputs are gathered before the TMEM
            // load (a memory-clobbering asm the loads cannot move past); across
            // the warp each load reads 32 consecutive window slots of one query
            // row.  Element e of the piece is query t = tq0+cq0+e at window
            // slot w = W − (128c + cq0 + e − r): one base address per piece,
            // then a constant step per element; out-of-band elements load nothing.
            float gb[16], gd[16];
            const int t0 = tq0 + cq0, w0 = W - (kTile * c + cq0 - r);
            const float* b0 = nullptr;
            using DTauT = typename std::conditional<kF32, float, __nv_bfloat16>::type;
            const DTauT* d0 = nullptr;
            long long bstep = 0, dstep = 0;
            if constexpr (kBias) {
              b0 = p.bias + bb * p.bs0 + (long long)t0 * p.bs1 + (long long)w0 * p.bs2;
              bstep = p.bs1 - p.bs2;
            }
            if constexpr (kDTau) {
              d0 = static_cast<const DTauT*>(p.dtau) + (((long long)bb * p.T + t0) * H + h) * W + w0;
              dstep = (long long)H * W - 1;
            }
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const bool valid = (unsigned)(e - lo[ss]) < (unsigned)cnt[ss];
              if constexpr (kBias) gb[e] = valid ? 0.5f * __ldg(b0 + e * bstep) : 0.f;
              if constexpr (kDTau) {
                if constexpr (kF32) gd[e] = valid ? p.ds_scale * __ldg(d0 + e * dstep) : 0.f;
                else gd[e] = valid ? p.ds_scale * __bfloat162float(d0[e * dstep]) : 0.f;
              }
            }
            tmem_ld16x2_wait(col, col + 64, R);
            piece(ss, R, gb, gd);
          } else {
#pragma unroll
            for (int z = 0; z < 8; ++z) pk[ss][z] = dk[ss][z] = 0u;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->sdp_free[b]);
      }
      // shared buffer b is free once the consumers of sub-chunks n−2, n−1 ran
      if (n >= 2) ok = mbar_wait(&bar->p_free[b], ((n >> 1) - 1) & 1, err, kErrBwd | 31);
      if (!ok) return;
      const uint32_t pb = pds + (2 * b) * kHalfBytes, db = pb + kHalfBytes;
#pragma unroll
      for (int ss = 0; ss < 2; ++ss) {
        const int c16 = (32 * hf + 16 * ss) >> 3;
        st_shared_v4(pb + sw128_off(r, c16), pk[ss][0], pk[ss][1], pk[ss][2], pk[ss][3]);
        st_shared_v4(pb + sw128_off(r, c16 + 1), pk[ss][4], pk[ss][5], pk[ss][6], pk[ss][7]);
        st_shared_v4(db + sw128_off(r, c16), dk[ss][0], dk[ss][1], dk[ss][2], dk[ss][3]);
        st_shared_v4(db + sw128_off(r, c16 + 1), dk[ss][4], dk[ss][5], dk[ss][6], dk[ss][7]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->p_full[b]);
      ++n;
    };

    // the sub-chunks in the MMA issuers' order; one call site keeps the
    // element code inlined once (instruction-cache footprint).  α/β of a
    // query tile arrive with its TMA load (q_full).
    SubGen gen{u0, u0, u1, nT, Wr, 0, 0, 0, 0, 0, 0, 0, c1h1_zero};
    Sub sc{};
    while (ok && gen.next(sc)) {
      if (sc.qidx >= 0)
        ok = mbar_wait(&bar->q_full[sc.qidx & 1], (sc.qidx >> 1) & 1, err, kErrBwd | 35);
      subchunk(sc.bh, sc.ikey, sc.c, sc.hh, sc.qs, sc.zero);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

template <bool kBias, bool kDTau, bool kAux, bool kF32>
cudaError_t launch_bwd_variant(const CUtensorMap* m, const BwdTC& a, size_t smem, int grid,
                               cudaStream_t st) {
  auto kern = tc_bwd_kernel<kBias, kDTau, kAux, kF32>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], m[6], a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_alpha_beta(const BwdP& p, int tpad, float ds_scale, float* coef,
                              cudaStream_t st) {
  const long long n = (long long)p.B * p.H * tpad;
  // per batch row: T·H·8 threads; about 16 resident CTAs per SM over all rows
  const long long per_b = ((long long)p.T * p.H * 8 + 255) / 256;
  const int gx = (int)std::max<long long>(1, std::min<long long>(per_b, (num_sms() * 16LL + p.B - 1) / p.B));
  alpha_beta_kernel<<<dim3(gx, p.B), 256, 0, st>>>(p.B, p.T, p.H, p.W, tpad, p.norm, ds_scale,
                                                   p.row_mass, p.dout, p.out, coef, coef + n,
                                                   coef + 2 * n, p.aux_row, coef + 3 * n,
                                                   coef + 4 * n);
  return cudaGetLastError();
}

bool tc_bwd_eligible(const BwdP& p) {
  if (p.mode != BOZO_MODE_LOCAL || p.HD != kHD || p.W < 1 || p.W > 128) return false;
  if (p.B > 65535 || (long long)p.T * p.H * 8 > 0x7fffffffLL) return false;  // pre-pass grid
  // dQ/dK in bf16, or both in fp32 (the fp32-IO variant: fp32 τ cotangent,
  // an fp32 dO copied to bf16 in the workspace, no RoPE); dV in bf16
  const bool f32 = p.dq_dt == BOZO_DT_F32;
  if (p.dq_dt != p.dk_dt || (p.dq_dt != BOZO_DT_BF16 && !f32) || p.dv_dt != BOZO_DT_BF16) return false;
  if (f32 && (p.cos || (p.dtau && p.dtau_dt != BOZO_DT_F32))) return false;
  if (!f32 && p.dtau && p.dtau_dt != BOZO_DT_BF16) return false;
  if (!tma_view_ok(p.q, p.B, p.T, p.H) || !tma_view_ok(p.k, p.B, p.T, p.H) ||
      !tma_view_ok(p.v, p.B, p.T, p.H))
    return false;
  if (p.dout.dt == BOZO_DT_F32 ? !p.dout_lp : !tma_view_ok(p.dout, p.B, p.T, p.H)) return false;
  if (p.dtau && (reinterpret_cast<uintptr_t>(p.dtau) & 15) != 0) return false;
  if (p.norm == BOZO_NORM_MASS) {
    // out rows are read with 16-byte vector loads
    if (p.out.dt != BOZO_DT_BF16 || p.out.sd != 1 || (reinterpret_cast<uintptr_t>(p.out.p) & 15) ||
        (p.out.sb % 8) || (p.out.st % 8) || (p.out.sh % 8))
      return false;
  }
  for (const void* ptr : {p.dq, p.dk, p.dv})
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return false;
  // RoPE: Q/K must arrive rotated (the forward's copies); θ drives the
  // inverse rotation of dQ/dK
  if (p.cos && (!p.theta || !p.qk_rotated)) return false;
  if (!p.coef || (reinterpret_cast<uintptr_t>(p.coef) & 15)) return false;
  return tmap_encoder_available();
}

cudaError_t launch_tc_bwd(const BwdP& p, cudaStream_t st, int* launches) {
  BwdTC a{};
  a.B = p.B; a.T = p.T; a.H = p.H; a.W = p.W;
  a.Wr = (p.W + 15) / 16 * 16;
  a.nT = (p.T + kTile - 1) / kTile;
  a.total = p.B * p.H * a.nT;
  a.tpad = a.nT * kTile;
  a.half_inv_scale = 0.5f / p.scale;
  a.ds_scale = 0.25f / p.scale;
  a.theta = p.cos ? p.theta : nullptr;
  a.bias = p.bias; a.bs0 = p.bs0; a.bs1 = p.bs1; a.bs2 = p.bs2;
  a.dtau = p.dtau;
  a.coef = p.coef;
  a.dq = p.dq;
  a.dk = p.dk;
  a.dv = p.dv;
  a.err = p.err;
  const bool f32 = p.dq_dt == BOZO_DT_F32;
  int nl = 2;
  DevT4 dout = p.dout;
  if (p.dout.dt == BOZO_DT_F32) {  // a bf16 copy of the fp32 cotangent for the TMA tiles
    cudaError_t e = launch_to_bf16(p.dout, p.B, p.T, p.H, kHD, p.dout_lp, num_sms(), st);
    if (e != cudaSuccess) return e;
    dout = DevT4{p.dout_lp, BOZO_DT_BF16, (long long)p.T * p.H * kHD, (long long)p.H * kHD, kHD, 1};
    ++nl;
  }
  {  // coefficient pre-pass into the (padded) workspace rows
    cudaError_t e = launch_alpha_beta(p, a.tpad, a.ds_scale, p.coef, st);
    if (e != cudaSuccess) return e;
  }
  CUtensorMap m[7];
  const DevT4* in[4] = {&p.q, &p.k, &p.v, &dout};
  for (int i = 0; i < 4; ++i)
    if (!make_tmap_bthd(&m[i], in[i]->p, in[i]->sb, in[i]->st, in[i]->sh, p.B, p.T, p.H, kTile))
      return cudaErrorInvalidValue;
  const long long ob = (long long)p.T * p.H * kHD, ot = (long long)p.H * kHD, oh = kHD;
  // dQ/dK in fp32 leave from registers: their maps are placeholders
  void* outs[3] = {f32 ? p.dv : p.dq, f32 ? p.dv : p.dk, p.dv};
  for (int i = 0; i < 3; ++i)
    if (!make_tmap_bthd(&m[4 + i], outs[i], ob, ot, oh, p.B, p.T, p.H, kTile)) return cudaErrorInvalidValue;
  const bool has_aux = p.aux_row != nullptr;
  const Layout L = bwd_layout(has_aux ? 5 : 3);
  const size_t smem = L.total + 1024;
  const int grid = std::min(num_sms(), a.total);
  *launches = nl;
  const bool has_bias = p.bias != nullptr, has_dtau = p.dtau != nullptr;
  if (f32) {
    // the fp32-IO variant serves the reference's fp32-Q call, which has no
    // per-row τ cotangent (that is formed for bf16 fields only)
    if (has_aux) return cudaErrorInvalidValue;
    const int v = (has_bias ? 2 : 0) | (has_dtau ? 1 : 0);
    switch (v) {
      case 0: return launch_bwd_variant<false, false, false, true>(m, a, smem, grid, st);
      case 1: return launch_bwd_variant<false, true, false, true>(m, a, smem, grid, st);
      case 2: return launch_bwd_variant<true, false, false, true>(m, a, smem, grid, st);
      default: return launch_bwd_variant<true, true, false, true>(m, a, smem, grid, st);
    }
  }
  const int v = (has_bias ? 4 : 0) | (has_dtau ? 2 : 0) | (has_aux ? 1 : 0);
  switch (v) {
    case 0: return launch_bwd_variant<false, false, false, false>(m, a, smem, grid, st);
    case 1: return launch_bwd_variant<false, false, true, false>(m, a, smem, grid, st);
    case 2: return launch_bwd_variant<false, true, false, false>(m, a, smem, grid, st);
    case 3: return launch_bwd_variant<false, true, true, false>(m, a, smem, grid, st);
    case 4: return launch_bwd_variant<true, false, false, false>(m, a, smem, grid, st);
    case 5: return launch_bwd_variant<true, false, true, false>(m, a, smem, grid, st);
    case 6: return launch_bwd_variant<true, true, false, false>(m, a, smem, grid, st);
    default: return launch_bwd_variant<true, true, true, false>(m, a, smem, grid, st);
  }
}

}  // namespace bozo
