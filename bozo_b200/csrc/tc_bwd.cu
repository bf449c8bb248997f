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
// (model.py:261-264).
//
// Work decomposition: key tiles of 128 rows, flattened b-h-major; one
// persistent CTA per SM walks a contiguous range.  For key tile i the queries
// that see it are query tile i (chunk 0) and the first Wr = ⌈W/16⌉·16 rows of
// query tile i+1 (chunk 1).  Per chunk:
//   Sᵀ = K_i·Q_cᵀ, dPᵀ = V_i·dO_cᵀ            (TMEM, M = 128 keys)
//   epilogue → Pᵀ = α·τ, dSᵀ = ds (bf16, shared memory, K-major over queries)
//   dV += Pᵀ·dO_c, dK += dSᵀ·Q_c                (TMEM, complete per key tile)
//   dQ_c += dS_c·K_i  (A = dSᵀ read MN-major)   (TMEM, two ping-pong
//                                                  accumulators: query tile
//                                                  i+1 starts in iteration i
//                                                  and completes in i+1)
// so no atomics and no partial sums leave the SM.  A CTA whose range starts
// mid-sequence first runs a chunk-1-only warm-up on key tile i−1 for dQ_i.
// α/β come from row_mass and dO·out computed when each query tile lands.
//
// Warps: 0 TMA, 1 MMA, 2/3/12/13 RoPE + α/β, 4-11 epilogue.  All waits are
// bounded (tc_ptx.cuh).
#include <algorithm>

#include "tc.cuh"
#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace bozo {
namespace {

using namespace tc;

constexpr int kTile = kTcTile;
constexpr int kHD = kTcHD;
constexpr int kTileBytes = kTile * kHD * 2;  // 16 KiB
constexpr int kThreads = 14 * 32;
constexpr int kRotThreads = 128;
constexpr int kErrBwd = 0x200;

// TMEM columns
constexpr uint32_t kColS = 0, kColDP = 128, kColDK = 256, kColDV = 320, kColDQ = 384;

struct BwdTC {
  int B, T, H, W, Wr, nT, total, norm;
  float half_inv_scale, ds_scale;  // 0.5/scale, 0.25/scale
  const float* cos;
  const float* sin;
  const float* bias;
  long long bs0, bs1, bs2;
  const __nv_bfloat16* dtau;  // [B,T,H,W] contiguous or null
  const float* row_mass;      // [B,H,T]
  int* err;
};

struct __align__(8) Bars {
  uint64_t kv_full[2], k_ready[2], kv_empty[2];
  uint64_t q_full[2], q_ready[2], q_empty[2];
  uint64_t o_full, o_empty;
  uint64_t sdp_full, sdp_free, p_full, p_free;
  uint64_t acc_full, dkv_free, dq_free[2];
  uint64_t stage_full, stage_free;
  uint32_t tmem_base;
};

struct Layout {
  uint32_t k, v, q, dout, o, pt, dst, ab, bars, total;
};

__host__ __device__ inline Layout bwd_layout() {
  Layout L;
  L.k = 0;
  L.v = L.k + 2 * kTileBytes;
  L.q = L.v + 2 * kTileBytes;
  L.dout = L.q + 2 * kTileBytes;
  L.o = L.dout + 2 * kTileBytes;
  L.pt = L.o + kTileBytes;          // Pᵀ  [128 keys x 128 queries] = 2 blocks
  L.dst = L.pt + 2 * kTileBytes;    // dSᵀ [128 keys x 128 queries] = 2 blocks
  L.ab = L.dst + 2 * kTileBytes;    // α/β: float[2 slots][2][128]
  L.bars = L.ab + 2 * 2 * kTile * 4;
  L.total = L.bars + (uint32_t)sizeof(Bars);
  return L;
}

// ── RoPE on a 128B-swizzled [128 x 64] bf16 tile (positions t0 + r) ──
__device__ __forceinline__ void rope_chunk(uint32_t base, int r, int c, const float (&cs)[8],
                                           const float (&sn)[8]) {
  uint32_t a[4], b[4], ra[4], rb[4];
  ld_shared_v4(base + sw128_off(r, c), a[0], a[1], a[2], a[3]);
  ld_shared_v4(base + sw128_off(r, c + 4), b[0], b[1], b[2], b[3]);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __nv_bfloat162 x1 = *reinterpret_cast<const __nv_bfloat162*>(&a[e]);
    const __nv_bfloat162 x2 = *reinterpret_cast<const __nv_bfloat162*>(&b[e]);
    const float x1l = __low2float(x1), x1h = __high2float(x1);
    const float x2l = __low2float(x2), x2h = __high2float(x2);
    const float cl = cs[2 * e], ch = cs[2 * e + 1], sl = sn[2 * e], sh = sn[2 * e + 1];
    ra[e] = pack_bf16(x1l * cl - x2l * sl, x1h * ch - x2h * sh);
    rb[e] = pack_bf16(x1l * sl + x2l * cl, x1h * sh + x2h * ch);
  }
  st_shared_v4(base + sw128_off(r, c), ra[0], ra[1], ra[2], ra[3]);
  st_shared_v4(base + sw128_off(r, c + 4), rb[0], rb[1], rb[2], rb[3]);
}

__device__ __forceinline__ void load_cs8(const float* tab, int t, int c, float (&v)[8]) {
  const float4* p = reinterpret_cast<const float4*>(tab + (long long)t * 32 + c * 8);
  const float4 a = __ldg(p), b = __ldg(p + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ void rope_tile(uint8_t* tile, int t0, int T, const float* cos, const float* sin, int tid) {
  const uint32_t base = smem_u32(tile);
  for (int item = tid; item < kTile * 4; item += 2 * kRotThreads) {
    const int i0 = item, i1 = item + kRotThreads;
    const int r0 = i0 >> 2, c0 = i0 & 3, r1 = i1 >> 2, c1 = i1 & 3;
    const bool ok0 = t0 + r0 < T, ok1 = i1 < kTile * 4 && t0 + r1 < T;
    float cs0[8], sn0[8], cs1[8], sn1[8];
    load_cs8(cos, ok0 ? t0 + r0 : 0, c0, cs0);
    load_cs8(sin, ok0 ? t0 + r0 : 0, c0, sn0);
    load_cs8(cos, ok1 ? t0 + r1 : 0, c1, cs1);
    load_cs8(sin, ok1 ? t0 + r1 : 0, c1, sn1);
    if (ok0) rope_chunk(base, r0, c0, cs0, sn0);
    if (ok1) rope_chunk(base, r1, c1, cs1, sn1);
  }
}

// Row dot product of two 128B-swizzled bf16 tiles (row r, 64 elements).
__device__ __forceinline__ float row_dot_sw(uint32_t a, uint32_t b, int r) {
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t x[4], y[4];
    ld_shared_v4(a + sw128_off(r, c), x[0], x[1], x[2], x[3]);
    ld_shared_v4(b + sw128_off(r, c), y[0], y[1], y[2], y[3]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 u = *reinterpret_cast<const __nv_bfloat162*>(&x[e]);
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&y[e]);
      acc = fmaf(__low2float(u), __low2float(v), acc);
      acc = fmaf(__high2float(u), __high2float(v), acc);
    }
  }
  return acc;
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

template <bool kBias, bool kDTau>
__global__ void __launch_bounds__(kThreads, 1)
    tc_bwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmdo,
                  const __grid_constant__ CUtensorMap tmo, const __grid_constant__ CUtensorMap tmdq,
                  const __grid_constant__ CUtensorMap tmdk, const __grid_constant__ CUtensorMap tmdv,
                  const BwdTC p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = bwd_layout();
  uint8_t* sK = smem + L.k;
  uint8_t* sV = smem + L.v;
  uint8_t* sQ = smem + L.q;
  uint8_t* sDO = smem + L.dout;
  uint8_t* sO = smem + L.o;
  uint8_t* sPT = smem + L.pt;
  uint8_t* sDST = smem + L.dst;
  float* sAB = reinterpret_cast<float*>(smem + L.ab);
  Bars* bar = reinterpret_cast<Bars*>(smem + L.bars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = (int)((long long)blockIdx.x * p.total / gridDim.x);
  const int u1 = (int)((long long)(blockIdx.x + 1) * p.total / gridDim.x);
  const bool need_o = p.norm == BOZO_NORM_MASS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->kv_full[s], 1);
      mbar_init(&bar->k_ready[s], 4);
      mbar_init(&bar->kv_empty[s], 1);
      mbar_init(&bar->q_full[s], 1);
      mbar_init(&bar->q_ready[s], 4);
      mbar_init(&bar->q_empty[s], 1);
      mbar_init(&bar->dq_free[s], 4);
    }
    mbar_init(&bar->o_full, 1);
    mbar_init(&bar->o_empty, 4);
    mbar_init(&bar->sdp_full, 1);
    mbar_init(&bar->sdp_free, 8);
    mbar_init(&bar->p_full, 8);
    mbar_init(&bar->p_free, 1);
    mbar_init(&bar->acc_full, 1);
    mbar_init(&bar->dkv_free, 8);
    mbar_init(&bar->stage_full, 8);
    mbar_init(&bar->stage_free, 1);
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
  const int nT = p.nT, Wr = p.Wr, H = p.H;

  if (warp == 0) {
    // ─────────────────────────── TMA producer ───────────────────────────
    if (lane == 0) {
      prefetch_tmap(&tmq); prefetch_tmap(&tmk); prefetch_tmap(&tmv); prefetch_tmap(&tmdo);
      if (need_o) prefetch_tmap(&tmo);
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
        if (need_o && nq >= 1) ok = ok && mbar_wait(&bar->o_empty, (nq - 1) & 1, err, kErrBwd | 3);
        if (!ok) return;
        mbar_arrive_expect_tx(&bar->q_full[s], 2 * kTileBytes);
        tma_load_4d(sQ + s * kTileBytes, &tmq, &bar->q_full[s], 0, bh % H, jj * kTile, bh / H);
        tma_load_4d(sDO + s * kTileBytes, &tmdo, &bar->q_full[s], 0, bh % H, jj * kTile, bh / H);
        if (need_o) {
          mbar_arrive_expect_tx(&bar->o_full, kTileBytes);
          tma_load_4d(sO, &tmo, &bar->o_full, 0, bh % H, jj * kTile, bh / H);
        }
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
  } else if (warp == 1) {
    // ─────────────────────────── MMA issuer ───────────────────────────
    if (lane == 0) {
      const uint32_t id_s0 = idesc_bf16(128, 128, false, false);   // Sᵀ/dPᵀ chunk 0
      const uint32_t id_s1 = idesc_bf16(128, Wr, false, false);    // Sᵀ/dPᵀ chunk 1
      const uint32_t id_kv = idesc_bf16(128, kHD, false, true);    // dV/dK: A K-major, B MN-major
      const uint32_t id_q = idesc_bf16(128, kHD, true, true);      // dQ: A (dSᵀ) MN-major
      constexpr uint64_t kTD = kTileBytes >> 4;
      const uint64_t dK0 = sdesc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t dV0 = sdesc_sw128(smem_u32(sV), 16, 1024);
      const uint64_t dQ0 = sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t dDO0 = sdesc_sw128(smem_u32(sDO), 16, 1024);
      const uint64_t dPT = sdesc_sw128(smem_u32(sPT), 16, 1024);
      const uint64_t dDST = sdesc_sw128(smem_u32(sDST), 16, 1024);
      // dSᵀ as the MN-major A operand of dQ: 64-query blocks 16 KiB apart (LBO)
      const uint64_t dDSmn = sdesc_sw128(smem_u32(sDST), kTileBytes, 1024);
      const uint32_t tS = tbase + kColS, tDP = tbase + kColDP, tDK = tbase + kColDK,
                     tDV = tbase + kColDV;
      int nk = 0, nq = 0, nchunk = 0, dq_started[2] = {0, 0};
      int kslot_cur = 0, qslot_cur = 0;  // slot of query tile i (chunk 0)
      bool ok = true;
      int it = 0;

      // issue Sᵀ and dPᵀ for one chunk of N query rows
      auto sdp = [&](int ks, int qs, int N) {
        if (nchunk >= 1) ok = ok && mbar_wait(&bar->sdp_free, (nchunk - 1) & 1, err, kErrBwd | 10);
        if (!ok) return;
        tc_fence_after();
        const uint32_t id = N == 128 ? id_s0 : id_s1;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_bf16(tS, dK0 + ks * kTD + 2 * kk, dQ0 + qs * kTD + 2 * kk, id, kk > 0);
          mma_bf16(tDP, dV0 + ks * kTD + 2 * kk, dDO0 + qs * kTD + 2 * kk, id, kk > 0);
        }
        mma_commit(&bar->sdp_full);
        ok = ok && mbar_wait(&bar->p_full, nchunk & 1, err, kErrBwd | 11);
        tc_fence_after();
      };
      auto wait_key = [&]() {
        const int s = nk & 1;
        ok = ok && mbar_wait(&bar->k_ready[s], (nk >> 1) & 1, err, kErrBwd | 12);
        ++nk;
        return s;
      };
      auto wait_query = [&]() {
        const int s = nq & 1;
        ok = ok && mbar_wait(&bar->q_ready[s], (nq >> 1) & 1, err, kErrBwd | 13);
        ++nq;
        return s;
      };
      // dQ[b] (+)= dS·K over the keys of slot ks, first key k-step kk0
      auto dq_mma = [&](int b, int ks, int kk0, bool accumulate) {
        if (!accumulate) {
          if (dq_started[b] >= 1)
            ok = ok && mbar_wait(&bar->dq_free[b], (dq_started[b] - 1) & 1, err, kErrBwd | 14);
          ++dq_started[b];
          tc_fence_after();
        }
        if (!ok) return;
        uint32_t acc = accumulate ? 1u : 0u;
        for (int kk = kk0; kk < 8; ++kk) {
          mma_bf16(tbase + kColDQ + 64 * b, dDSmn + kk * 128, dK0 + ks * kTD + kk * 128, id_q, acc);
          acc = 1;
        }
      };

      for (int u = u0; u < u1 && ok; ++u, ++it) {
        const Step st = step_of(u, u0, u1, nT);
        const int bq = st.i & 1;  // dQ accumulator of query tile i
        if (st.warm) {
          const int ks = wait_key();
          qslot_cur = wait_query();
          sdp(ks, qslot_cur, Wr);  // chunk-1-type pass: key tile i−1 vs query tile i
          if (!ok) break;
          dq_mma(bq, ks, (kTile - Wr) / 16, false);
          mma_commit(&bar->p_free);
          mma_commit(&bar->kv_empty[ks]);
          ++nchunk;
        } else if (st.first_of_seg) {
          qslot_cur = wait_query();
        }
        kslot_cur = wait_key();
        if (!ok) break;
        // ── chunk 0: query tile i ──
        sdp(kslot_cur, qslot_cur, 128);
        if (!ok) break;
        if (it >= 1) ok = mbar_wait(&bar->dkv_free, (it - 1) & 1, err, kErrBwd | 15);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a_pt = dPT + (kk >> 2) * kTD + (kk & 3) * 2;
          const uint64_t a_ds = dDST + (kk >> 2) * kTD + (kk & 3) * 2;
          mma_bf16(tDV, a_pt, dDO0 + qslot_cur * kTD + kk * 128, id_kv, kk > 0);
          mma_bf16(tDK, a_ds, dQ0 + qslot_cur * kTD + kk * 128, id_kv, kk > 0);
        }
        dq_mma(bq, kslot_cur, 0, st.warm || !st.first_of_seg);
        mma_commit(&bar->p_free);
        mma_commit(&bar->q_empty[qslot_cur]);
        ++nchunk;
        // ── chunk 1: first Wr rows of query tile i+1 ──
        if (st.has_c1) {
          const int qs1 = wait_query();
          sdp(kslot_cur, qs1, Wr);
          if (!ok) break;
          for (int kk = 0; kk < Wr / 16; ++kk) {
            const uint64_t a_pt = dPT + (kk >> 2) * kTD + (kk & 3) * 2;
            const uint64_t a_ds = dDST + (kk >> 2) * kTD + (kk & 3) * 2;
            mma_bf16(tDV, a_pt, dDO0 + qs1 * kTD + kk * 128, id_kv, 1);
            mma_bf16(tDK, a_ds, dQ0 + qs1 * kTD + kk * 128, id_kv, 1);
          }
          if (!st.last) dq_mma(bq ^ 1, kslot_cur, (kTile - Wr) / 16, false);
          mma_commit(&bar->p_free);
          if (st.last) mma_commit(&bar->q_empty[qs1]);
          ++nchunk;
          qslot_cur = qs1;
        }
        mma_commit(&bar->acc_full);
        mma_commit(&bar->kv_empty[kslot_cur]);
      }
    }
  } else if (warp < 4 || warp >= 12) {
    // ───────────── RoPE of K / Q tiles and per-query α, β ─────────────
    const int tid = (warp < 4 ? warp - 2 : warp - 10) * 32 + lane;
    int nk = 0, nq = 0;
    bool ok = true;
    auto do_key = [&](int bh, int jj) {
      const int s = nk & 1;
      ok = ok && mbar_wait(&bar->kv_full[s], (nk >> 1) & 1, err, kErrBwd | 20);
      if (ok && p.cos) rope_tile(sK + s * kTileBytes, jj * kTile, p.T, p.cos, p.sin, tid);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->k_ready[s]);
      ++nk;
    };
    auto do_query = [&](int bh, int jj) {
      const int s = nq & 1;
      ok = ok && mbar_wait(&bar->q_full[s], (nq >> 1) & 1, err, kErrBwd | 21);
      if (ok && p.cos) rope_tile(sQ + s * kTileBytes, jj * kTile, p.T, p.cos, p.sin, tid);
      // α/β for query row r = tid
      const int t = jj * kTile + tid;
      float a = 0.f, b = 0.f;
      if (need_o) ok = ok && mbar_wait(&bar->o_full, nq & 1, err, kErrBwd | 22);
      if (ok && t < p.T) {
        if (p.norm == BOZO_NORM_MASS) {
          const float m = p.row_mass[(long long)bh * p.T + t];
          const float dd = row_dot_sw(smem_u32(sDO + s * kTileBytes), smem_u32(sO), tid);
          a = 1.f / fmaxf(m, kMassEps);
          b = m >= kMassEps ? -dd * a : 0.f;
        } else if (p.norm == BOZO_NORM_COUNT) {
          a = 1.f / (float)max(min(t, p.W), 1);
        } else {
          a = 1.f;
        }
      }
      sAB[(s * 2 + 0) * kTile + tid] = a;
      sAB[(s * 2 + 1) * kTile + tid] = b;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (need_o) mbar_arrive(&bar->o_empty);
        mbar_arrive(&bar->q_ready[s]);
      }
      ++nq;
    };
    for (int u = u0; u < u1 && ok; ++u) {
      const Step st = step_of(u, u0, u1, nT);
      if (st.warm) do_key(st.bh, st.i - 1);
      if (st.first_of_seg) do_query(st.bh, st.i);
      do_key(st.bh, st.i);
      if (st.has_c1) do_query(st.bh, st.i + 1);
    }
  } else {
    // ─────────────────────────── epilogue (8 warps) ───────────────────────────
    const int e = warp - 4;
    const int qd = warp & 3;
    const int hf = e >> 2;
    const int r = qd * 32 + lane;  // key row in the tile / query row for dQ
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const int W = p.W;
    const uint32_t pt_base = smem_u32(sPT), ds_base = smem_u32(sDST);
    int nchunk = 0, nq = 0, it = 0;
    int qslot_cur = 0;
    bool ok = true;

    // One chunk: query tile jq (slot qs), chunk type c (0: same tile, 1: next),
    // N query columns; if dq_only, Pᵀ is not needed (warm-up).
    auto chunk = [&](int bh, int i_key, int c, int qs, int N) {
      ok = ok && mbar_wait(&bar->sdp_full, nchunk & 1, err, kErrBwd | 30);
      if (!ok) return;
      __syncwarp();
      tc_fence_after();
      // Pᵀ/dSᵀ buffers: previous chunk's MMAs and the last staging store done
      if (nchunk >= 1) ok = mbar_wait(&bar->p_free, (nchunk - 1) & 1, err, kErrBwd | 31);
      if (ok && c == 0 && it >= 1) ok = mbar_wait(&bar->stage_free, (it - 1) & 1, err, kErrBwd | 32);
      if (!ok) return;
      __syncwarp();
      const int b = bh / H, h = bh % H;
      const int t0 = (i_key + c) * kTile;        // query position of column 0
      const float* ab = sAB + qs * 2 * kTile;
      // band of this quadrant: q ∈ [32qd + 1 − 128c, 32qd + 31 + W − 128c]
      const int q_lo = qd * 32 + 1 - kTile * c, q_hi = qd * 32 + 31 + W - kTile * c;
      const float* bias_b = nullptr;
      const __nv_bfloat16* dtau_b = nullptr;
      if constexpr (kBias) bias_b = p.bias + b * p.bs0;
      if constexpr (kDTau) dtau_b = p.dtau;
#pragma unroll 1
      for (int sc = hf * 4; sc < hf * 4 + 4; ++sc) {
        const int cq0 = sc * 16;
        const bool band = cq0 < N && cq0 + 15 >= q_lo && cq0 <= q_hi;
        uint32_t pk[8], dk[8];
        if (band) {
          uint32_t rs[16], rd[16];
          tmem_ld16_wait(tbase + lane_off + kColS + cq0, rs);
          tmem_ld16_wait(tbase + lane_off + kColDP + cq0, rd);
#pragma unroll
          for (int e2 = 0; e2 < 16; e2 += 2) {
            float pv[2], dv[2];
#pragma unroll
            for (int z = 0; z < 2; ++z) {
              const int q = cq0 + e2 + z;
              const int t = t0 + q;
              const int dlt = q + kTile * c - r;  // t − s
              const bool valid = dlt >= 1 && dlt <= W && t < p.T;
              const int w = W - dlt;              // window slot of (t, s)
              const int wc = valid ? w : 0;
              const int tc = valid ? t : 0;
              float x = __uint_as_float(rs[e2 + z]) * p.half_inv_scale;
              if constexpr (kBias) x = fmaf(0.5f, __ldg(bias_b + (long long)tc * p.bs1 + (long long)wc * p.bs2), x);
              const float th = tanh_approx(x);
              const float tau = fmaf(0.5f, th, 0.5f);
              const float g = fmaf(-th, th, 1.f);  // 4τ(1−τ)
              const float al = ab[q], be = ab[kTile + q];
              float dtau = fmaf(al, __uint_as_float(rd[e2 + z]), be);
              if constexpr (kDTau)
                dtau += __bfloat162float(dtau_b[(((long long)b * p.T + tc) * H + h) * W + wc]);
              pv[z] = valid ? tau * al : 0.f;
              dv[z] = valid ? dtau * g * p.ds_scale : 0.f;
            }
            pk[e2 >> 1] = pack_bf16(pv[0], pv[1]);
            dk[e2 >> 1] = pack_bf16(dv[0], dv[1]);
          }
        } else {
#pragma unroll
          for (int z = 0; z < 8; ++z) pk[z] = dk[z] = 0u;
        }
        const int blk = cq0 >> 6, c16 = (cq0 & 63) >> 3;
        st_shared_v4(pt_base + blk * kTileBytes + sw128_off(r, c16), pk[0], pk[1], pk[2], pk[3]);
        st_shared_v4(pt_base + blk * kTileBytes + sw128_off(r, c16 + 1), pk[4], pk[5], pk[6], pk[7]);
        st_shared_v4(ds_base + blk * kTileBytes + sw128_off(r, c16), dk[0], dk[1], dk[2], dk[3]);
        st_shared_v4(ds_base + blk * kTileBytes + sw128_off(r, c16 + 1), dk[4], dk[5], dk[6], dk[7]);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar->sdp_free);
        mbar_arrive(&bar->p_full);
      }
      ++nchunk;
    };

    // α/β of a query tile become visible through its q_ready phase
    auto take_query = [&]() {
      const int s = nq & 1;
      ok = ok && mbar_wait(&bar->q_ready[s], (nq >> 1) & 1, err, kErrBwd | 35);
      ++nq;
      return s;
    };
    for (int u = u0; u < u1 && ok; ++u, ++it) {
      const Step st = step_of(u, u0, u1, nT);
      const int b = st.bh / H, h = st.bh % H;
      if (st.warm) {
        qslot_cur = take_query();
        chunk(st.bh, st.i - 1, 1, qslot_cur, Wr);
      } else if (st.first_of_seg) {
        qslot_cur = take_query();
      }
      chunk(st.bh, st.i, 0, qslot_cur, 128);
      if (st.has_c1) {
        const int qs1 = take_query();
        chunk(st.bh, st.i, 1, qs1, Wr);
        qslot_cur = qs1;
      }
      if (!ok) break;
      // ── outputs of key tile i: dQ_i (query rows), dK_i, dV_i (key rows) ──
      ok = mbar_wait(&bar->acc_full, it & 1, err, kErrBwd | 33);
      if (!ok) break;
      __syncwarp();
      tc_fence_after();
      const int bq = st.i & 1;
      const int pos = st.i * kTile + r;  // query position (dQ) == key position (dK)
      uint32_t g[64];
      tmem_ld32_wait(tbase + lane_off + (hf == 0 ? kColDQ + 64 * bq : kColDK), g);
      tmem_ld32_wait(tbase + lane_off + (hf == 0 ? kColDQ + 64 * bq : kColDK) + 32, g + 32);
      // inverse RoPE: g1' = g1·c + g2·s, g2' = g2·c − g1·s
      if (p.cos && pos < p.T) {
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float cs[8], sn[8];
          load_cs8(p.cos, pos, c8, cs);
          load_cs8(p.sin, pos, c8, sn);
#pragma unroll
          for (int z = 0; z < 8; ++z) {
            const int d = c8 * 8 + z;
            const float g1 = __uint_as_float(g[d]), g2 = __uint_as_float(g[d + 32]);
            g[d] = __float_as_uint(g1 * cs[z] + g2 * sn[z]);
            g[d + 32] = __float_as_uint(g2 * cs[z] - g1 * sn[z]);
          }
        }
      }
      // stage: dQ → Pᵀ block 0, dK → Pᵀ block 1, dV → dSᵀ block 0
      const uint32_t gdst = pt_base + hf * kTileBytes;
#pragma unroll
      for (int z = 0; z < 8; ++z) {
        uint32_t w4[4];
#pragma unroll
        for (int y = 0; y < 4; ++y)
          w4[y] = pack_bf16(__uint_as_float(g[8 * z + 2 * y]), __uint_as_float(g[8 * z + 2 * y + 1]));
        st_shared_v4(gdst + sw128_off(r, z), w4[0], w4[1], w4[2], w4[3]);
      }
      {
        uint32_t vv[32];
        tmem_ld32_wait(tbase + lane_off + kColDV + 32 * hf, vv);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bar->dkv_free);
          if (hf == 0) mbar_arrive(&bar->dq_free[bq]);
        }
#pragma unroll
        for (int z = 0; z < 4; ++z) {
          uint32_t w4[4];
#pragma unroll
          for (int y = 0; y < 4; ++y)
            w4[y] = pack_bf16(__uint_as_float(vv[8 * z + 2 * y]), __uint_as_float(vv[8 * z + 2 * y + 1]));
          st_shared_v4(ds_base + sw128_off(r, hf * 4 + z), w4[0], w4[1], w4[2], w4[3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->stage_full);
      if (warp == 4 && lane == 0) {
        ok = mbar_wait(&bar->stage_full, it & 1, err, kErrBwd | 34);
        if (ok) {
          tma_store_4d(&tmdq, sPT, 0, h, st.i * kTile, b);
          tma_store_4d(&tmdk, sPT + kTileBytes, 0, h, st.i * kTile, b);
          tma_store_4d(&tmdv, sDST, 0, h, st.i * kTile, b);
          bulk_commit_group();
          bulk_wait_group_read0();
          mbar_arrive(&bar->stage_free);
        }
      }
      __syncwarp();
    }
    if (warp == 4 && lane == 0) bulk_wait_group0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

template <bool kBias, bool kDTau>
cudaError_t launch_bwd_variant(const CUtensorMap* m, const BwdTC& a, size_t smem, int grid,
                               cudaStream_t st) {
  auto kern = tc_bwd_kernel<kBias, kDTau>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], m[6], m[7], a);
  return cudaGetLastError();
}

}  // namespace

bool tc_bwd_eligible(const BwdP& p) {
  if (p.mode != BOZO_MODE_LOCAL || p.HD != kHD || p.W < 1 || p.W > 128) return false;
  if (p.dq_dt != BOZO_DT_BF16 || p.dk_dt != BOZO_DT_BF16 || p.dv_dt != BOZO_DT_BF16) return false;
  if (!tma_view_ok(p.q, p.B, p.T, p.H) || !tma_view_ok(p.k, p.B, p.T, p.H) ||
      !tma_view_ok(p.v, p.B, p.T, p.H) || !tma_view_ok(p.dout, p.B, p.T, p.H))
    return false;
  if (p.norm == BOZO_NORM_MASS && !tma_view_ok(p.out, p.B, p.T, p.H)) return false;
  if (p.dtau && p.dtau_dt != BOZO_DT_BF16) return false;
  for (const void* ptr : {p.dq, p.dk, p.dv})
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return false;
  if (p.cos && ((reinterpret_cast<uintptr_t>(p.cos) & 15) || (reinterpret_cast<uintptr_t>(p.sin) & 15)))
    return false;
  return tmap_encoder_available();
}

cudaError_t launch_tc_bwd(const BwdP& p, cudaStream_t st, int* launches) {
  BwdTC a{};
  a.B = p.B; a.T = p.T; a.H = p.H; a.W = p.W;
  a.Wr = (p.W + 15) / 16 * 16;
  a.nT = (p.T + kTile - 1) / kTile;
  a.total = p.B * p.H * a.nT;
  a.norm = p.norm;
  a.half_inv_scale = 0.5f / p.scale;
  a.ds_scale = 0.25f / p.scale;
  a.cos = p.cos; a.sin = p.sin;
  a.bias = p.bias; a.bs0 = p.bs0; a.bs1 = p.bs1; a.bs2 = p.bs2;
  a.dtau = static_cast<const __nv_bfloat16*>(p.dtau);
  a.row_mass = p.row_mass;
  a.err = p.err;
  CUtensorMap m[8];
  const long long ob = (long long)p.T * p.H * kHD, ot = (long long)p.H * kHD, oh = kHD;
  const DevT4* in[5] = {&p.q, &p.k, &p.v, &p.dout, &p.out};
  for (int i = 0; i < 5; ++i) {
    if (i == 4 && p.norm != BOZO_NORM_MASS) {
      m[4] = m[3];  // unused
      continue;
    }
    if (!make_tmap_bthd(&m[i], in[i]->p, in[i]->sb, in[i]->st, in[i]->sh, p.B, p.T, p.H, kTile))
      return cudaErrorInvalidValue;
  }
  void* outs[3] = {p.dq, p.dk, p.dv};
  for (int i = 0; i < 3; ++i)
    if (!make_tmap_bthd(&m[5 + i], outs[i], ob, ot, oh, p.B, p.T, p.H, kTile)) return cudaErrorInvalidValue;
  const Layout L = bwd_layout();
  const size_t smem = L.total + 1024;
  const int grid = std::min(num_sms(), a.total);
  *launches = 1;
  const bool has_bias = p.bias != nullptr, has_dtau = p.dtau != nullptr;
  if (has_bias && has_dtau) return launch_bwd_variant<true, true>(m, a, smem, grid, st);
  if (has_bias) return launch_bwd_variant<true, false>(m, a, smem, grid, st);
  if (has_dtau) return launch_bwd_variant<false, true>(m, a, smem, grid, st);
  return launch_bwd_variant<false, false>(m, a, smem, grid, st);
}

}  // namespace bozo
