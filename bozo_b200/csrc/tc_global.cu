// tc_global.cu — tcgen05 / TMA / TMEM kernels that stream whole key tiles:
// the GLOBAL full-causal tension block (model.py:217-237) and local windows
// too wide for the band kernels (W > 128), for bf16 Q/K/V with HD = 64.
//
// Semantics: τ[t,s] = σ(q_t·k_s/scale + bias) for every key s ≤ t (global,
// self included, bias[b,t,s]) or 1 ≤ t − s ≤ W (local, bias[b,t,w] at window
// slot w = W − (t − s), triton_tension/kernel.py:41-126); out_t = Σ_s τ·v_s
// normalised by τ-mass (model.py:257-258), by the position count
// (model.py:261-264) or raw; the exported τ (local [B,T,H,W]; global: the
// reference's window τ_x[t,c] = τ[t, T−1−c], c < tw, model.py:233-236); and
// the backward through all of it.  Q and K arrive RoPE-rotated (the forward
// writes the rotated copies first); the backward inverse-rotates dQ and dK.
//
// Three kernels share one pipeline skeleton.  A work unit is one 128-row
// "outer" tile held in shared memory while 128-row "inner" tiles stream
// through a TMA ring, each inner tile in two 64-row halves (sub-steps):
//
//   role  outer           inner (range)          producers (TMEM)        consumers (TMEM acc)
//   FWD   Q_j             K_i,V_i   (i ≤ j)      S = Q·K_hᵀ              O  += P·V_h
//   DKV   K_i,V_i         Q_j,dO_j  (j ≥ i)      Sᵀ = K·Q_hᵀ, dPᵀ=V·dO_hᵀ dV += (ατ)ᵀ·dO_h, dK += dSᵀ·Q_h
//   DQ    Q_j,dO_j        K_i,V_i   (i ≤ j)      S = Q·K_hᵀ, dP = dO·V_hᵀ dQ += dS·K_h
// (a local window limits the inner range to the tiles its band touches).
//
// All MMAs are M = 128, N = 64, K = 64 (kind::f16, bf16 in, fp32 accumulate).
// Producer results are double-buffered in TMEM, the epilogue's bf16 tiles
// double-buffered in shared memory, and the accumulators double-buffered in
// TMEM per unit, so the MMA of sub-step n+1 overlaps the epilogue of n and a
// unit's output overlaps the next unit.  dQ is computed per query tile by its
// own kernel so no partial sums leave an SM and no atomics are needed.  When
// the caller's workspace has room for it, DKV also stores each dSᵀ tile it
// formed (bf16, [128 keys × 64 queries], by TMA from the tile the dK MMA
// reads) and the dQ kernel is a pure MMA pass over them (role DQS):
//   DQS   (none)          K_i, dSᵀ(i,j) halves   —                      dQ += dS·K_h
// instead of recomputing S, dP and the element math (role DQ).  Units are
// dealt to persistent CTAs heaviest first.
//
// Warps: 0 TMA; 1 MMA (one thread); 2,3,12,13 output (TMEM accumulators →
// bf16 tile in the dead outer slot → TMA store); 4-11 epilogue.  Every
// mbarrier wait is bounded (tc_ptx.cuh).
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
constexpr int kTileBytes = kTile * kHD * 2;  // 16 KiB: [128 x 64] bf16, SW128
constexpr int kCoefBytes = 3 * kTile * 4;   // α/2, α·c, β·c of 128 query rows
constexpr int kThreads = 14 * 32;
constexpr int kErrG = 0x300;

enum Role : int { kFwd = 0, kDKV = 1, kDQ = 2, kDQS = 3 };

template <int R>
struct Traits {
  // DQS keeps one outer slot per unit only as the dQ staging tile
  static constexpr int kOuterTiles = (R == kFwd || R == kDQS) ? 1 : 2;
  static constexpr bool kOuterCoef = R == kDQ;
  static constexpr bool kInnerCoef = R == kDKV;
  static constexpr int kInnerStages = R == kDKV ? 2 : 3;
  static constexpr int kInnerTiles = R == kDQS ? 3 : 2;  // K_i (+ V_i | Q_j, dO_j | dSᵀ halves)
  static constexpr int kEpiTiles = R == kDKV ? 2 : (R == kDQS ? 0 : 1);  // bf16 tiles per sub-step
  static constexpr int kAccCols = R == kDKV ? 128 : 64;
};

struct GlobTC {
  int B, T, H, BH, nT, units, tpad, tw;
  int local, W;  // local: sliding window of W keys before each query (self excluded)
  float half_inv_scale, ds_scale;
  int norm;
  const float* theta;  // RoPE frequencies [32] (inverse rotation of dQ/dK) or null
  const float* bias;   // global [B,T,T] / local [B,T,W]
  long long bs0, bs1, bs2;
  __nv_bfloat16* tau;         // FWD: exported τ [B,T,H,tw], zero-filled before
  const __nv_bfloat16* dtau;  // DKV/DQ: its cotangent
  float* row_mass;            // FWD: [B,H,T]
  const float* coef;          // DKV/DQ: [3][B·H, tpad]
  int ds_store;               // DKV: store every dSᵀ tile for DQS
  int dsD;                    // dSᵀ tiles per (b·h, key tile): the longest inner range
  int* err;
};

// Index of the first of the two dSᵀ query-half tiles of key tile i and query
// tile j of head bh in the dense scratch [B·H][nT][dsD][2][128][64] (bf16).
__device__ __forceinline__ int ds_tile(int bh, int i, int j, int nT, int dsD) {
  return ((bh * nT + i) * dsD + (j - i)) * 2;
}

struct __align__(8) GBars {
  uint64_t outer_full[2], outer_empty[2];
  uint64_t inner_full[3], inner_empty[3];
  uint64_t s_full[2], s_free[2], p_full[2], p_free[2];
  uint64_t acc_full[2], acc_free[2];
  uint64_t mass_ready[2], staged;
  uint32_t tmem_base;
};

struct GLayout {
  uint32_t outer, ocoef, inner, icoef, epi, mass, bars, total;
};

template <int R>
__host__ __device__ inline GLayout glayout() {
  using Tr = Traits<R>;
  GLayout L;
  L.outer = 0;
  L.ocoef = L.outer + 2 * Tr::kOuterTiles * kTileBytes;
  L.inner = L.ocoef + (Tr::kOuterCoef ? 2 * kCoefBytes : 0);
  L.inner = (L.inner + 1023) & ~1023u;
  L.icoef = L.inner + Tr::kInnerStages * Tr::kInnerTiles * kTileBytes;
  L.epi = L.icoef + (Tr::kInnerCoef ? Tr::kInnerStages * kCoefBytes : 0);
  L.epi = (L.epi + 1023) & ~1023u;
  L.mass = L.epi + 2 * Tr::kEpiTiles * kTileBytes;
  L.bars = L.mass + (R == kFwd ? 2 * 2 * kTile * 4 : 0);
  L.total = L.bars + (uint32_t)sizeof(GBars);
  return L;
}

// Work unit k (heaviest first): FWD/DQ outer query tile j has key tiles
// [first, j] (first = 0 globally, the window's first tile locally), DKV outer
// key tile i has query tiles [i, last].
__device__ __forceinline__ void unit_of(int role, int k, int BH, int nT, int local, int W, int& bh,
                                        int& ot, int& first_inner, int& n_inner) {
  const int g = k / BH;
  bh = k % BH;
  if (role == kDKV) {
    ot = g;
    first_inner = g;
    const int last = local ? min(nT - 1, (g * kTile + kTile - 1 + W) / kTile) : nT - 1;
    n_inner = last - g + 1;
  } else {
    ot = nT - 1 - g;
    first_inner = local ? max(0, ot * kTile - W) / kTile : 0;
    n_inner = ot - first_inner + 1;
  }
}

template <int R, bool kBias, bool kExtra>
__global__ void __launch_bounds__(kThreads, 1)
    tc_global_kernel(const __grid_constant__ CUtensorMap tmo0, const __grid_constant__ CUtensorMap tmo1,
                     const __grid_constant__ CUtensorMap tmi0, const __grid_constant__ CUtensorMap tmi1,
                     const __grid_constant__ CUtensorMap tmout0, const __grid_constant__ CUtensorMap tmout1,
                     const __grid_constant__ CUtensorMap tmds, const GlobTC p) {
  using Tr = Traits<R>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const GLayout L = glayout<R>();
  uint8_t* sOuter = smem + L.outer;  // [slot][tile] 16 KiB each
  float* sOCoef = reinterpret_cast<float*>(smem + L.ocoef);
  uint8_t* sInner = smem + L.inner;  // [stage][2 tiles]
  float* sICoef = reinterpret_cast<float*>(smem + L.icoef);
  uint8_t* sEpi = smem + L.epi;      // [buffer][tile]
  float* sMass = reinterpret_cast<float*>(smem + L.mass);
  GBars* bar = reinterpret_cast<GBars*>(smem + L.bars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int H = p.H, T = p.T, nT = p.nT, BH = p.BH;
  constexpr int kStages = Tr::kInnerStages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->outer_full[s], 1);
      mbar_init(&bar->outer_empty[s], 1);
      mbar_init(&bar->s_full[s], 1);
      mbar_init(&bar->s_free[s], 8);
      mbar_init(&bar->p_full[s], 8);
      // DKV storing dSᵀ: the MMA thread also arrives once the tile's store
      // has read the buffer
      mbar_init(&bar->p_free[s], (R == kDKV && p.ds_store) ? 2 : 1);
      mbar_init(&bar->acc_full[s], 1);
      mbar_init(&bar->acc_free[s], 4);
      mbar_init(&bar->mass_ready[s], 8);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar->inner_full[s], 1);
      mbar_init(&bar->inner_empty[s], 1);
    }
    mbar_init(&bar->staged, 4);
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
      if (R != kDQS) prefetch_tmap(&tmo0);
      prefetch_tmap(&tmi0); prefetch_tmap(&tmi1); prefetch_tmap(&tmout0);
      if (Tr::kOuterTiles == 2) prefetch_tmap(&tmo1);
      if (R == kDKV) prefetch_tmap(&tmout1);
      if (R == kDQS) prefetch_tmap(&tmds);
      const long long plane = (long long)BH * p.tpad;
      bool ok = true;
      int ni = 0;
      for (int k = blockIdx.x, m = 0; k < p.units && ok; k += G, ++m) {
        int bh, ot, fi, nin;
        unit_of(R, k, BH, nT, p.local, p.W, bh, ot, fi, nin);
        const int b = bh / H, h = bh % H;
        const int os = m & 1;
        if (R != kDQS) {  // DQS has no outer operand (its outer slot is staging only)
          if (m >= 2) ok = mbar_wait(&bar->outer_empty[os], ((m >> 1) - 1) & 1, err, kErrG | 1);
          if (!ok) break;
          uint8_t* o = sOuter + os * Tr::kOuterTiles * kTileBytes;
          mbar_arrive_expect_tx(&bar->outer_full[os],
                                Tr::kOuterTiles * kTileBytes + (Tr::kOuterCoef ? kCoefBytes : 0));
          tma_load_4d(o, &tmo0, &bar->outer_full[os], 0, h, ot * kTile, b);
          if (Tr::kOuterTiles == 2)
            tma_load_4d(o + kTileBytes, &tmo1, &bar->outer_full[os], 0, h, ot * kTile, b);
        }
        if (Tr::kOuterCoef) {
          const long long off = (long long)bh * p.tpad + ot * kTile;
#pragma unroll
          for (int z = 0; z < 3; ++z)
            bulk_load_1d(sOCoef + (os * 3 + z) * kTile, p.coef + z * plane + off, kTile * 4,
                         &bar->outer_full[os]);
        }
        for (int x = 0; x < nin && ok; ++x) {
          const int it = fi + x;
          const int st = ni % kStages;
          if (ni >= kStages) ok = mbar_wait(&bar->inner_empty[st], ((ni / kStages) - 1) & 1, err, kErrG | 2);
          if (!ok) break;
          uint8_t* in = sInner + st * Tr::kInnerTiles * kTileBytes;
          mbar_arrive_expect_tx(&bar->inner_full[st],
                                Tr::kInnerTiles * kTileBytes + (Tr::kInnerCoef ? kCoefBytes : 0));
          tma_load_4d(in, &tmi0, &bar->inner_full[st], 0, h, it * kTile, b);
          if (R == kDQS) {  // the two dSᵀ query halves of (key tile it, query tile ot)
            const int t0 = ds_tile(bh, it, ot, nT, p.dsD);
            tma_load_2d(in + kTileBytes, &tmds, &bar->inner_full[st], 0, t0 * kTile);
            tma_load_2d(in + 2 * kTileBytes, &tmds, &bar->inner_full[st], 0, (t0 + 1) * kTile);
          } else {
            tma_load_4d(in + kTileBytes, &tmi1, &bar->inner_full[st], 0, h, it * kTile, b);
          }
          if (Tr::kInnerCoef) {
            const long long off = (long long)bh * p.tpad + it * kTile;
#pragma unroll
            for (int z = 0; z < 3; ++z)
              bulk_load_1d(sICoef + (st * 3 + z) * kTile, p.coef + z * plane + off, kTile * 4,
                           &bar->inner_full[st]);
          }
          ++ni;
        }
      }
    }
  } else if (warp == 1) {
    // ─────────────────────────── MMA issuer ───────────────────────────
    if (lane == 0) {
      const uint32_t id_p = idesc_bf16(128, 64, false, false);    // producers: A, B K-major
      const uint32_t id_c = idesc_bf16(128, kHD, false, true);    // consumers: B MN-major
      constexpr uint64_t kTD = kTileBytes >> 4;                   // one tile, 16 B units
      const uint64_t dOuter = sdesc_sw128(smem_u32(sOuter), 16, 1024);
      const uint64_t dInner = sdesc_sw128(smem_u32(sInner), 16, 1024);
      const uint64_t dEpi = sdesc_sw128(smem_u32(sEpi), 16, 1024);
      // DQS: both dSᵀ query halves of a stage as the MN-major A operand of
      // dQ (query blocks one tile apart), K_i as the MN-major B operand
      const uint32_t id_q = idesc_bf16(128, kHD, true, true);
      const uint64_t dDSmn = sdesc_sw128(smem_u32(sInner) + kTileBytes, kTileBytes, 1024);
      bool ok = true;

      // The CTA's sub-steps in order (the order the epilogue walks): unit m,
      // inner tile x of it (ring load ni, stage st), 64-row half hh.
      struct GSub {
        int n, m, ni, st, hh, bh, ot, x;
        bool unit_first, last;
      };
      int gk = blockIdx.x, gm = 0, gx = 0, ghh = 0, gn = 0, gni = 0, gnin = 0, gbh = 0, got = 0;
      bool in_unit = false;
      auto next_sub = [&](GSub& s) -> bool {
        for (;;) {
          if (!in_unit) {
            if (gk >= p.units) return false;
            int fi;
            unit_of(R, gk, BH, nT, p.local, p.W, gbh, got, fi, gnin);
            gx = 0;
            ghh = 0;
            in_unit = true;
          }
          if (gx < gnin) {
            s.n = gn++;
            s.m = gm;
            s.ni = gni;
            s.st = gni % kStages;
            s.hh = ghh;
            s.bh = gbh;
            s.ot = got;
            s.x = gx;
            s.unit_first = gx == 0 && ghh == 0;
            s.last = gx == gnin - 1 && ghh == 1;
            if (++ghh == 2) {
              ghh = 0;
              ++gx;
              ++gni;
            }
            return true;
          }
          in_unit = false;
          gk += G;
          ++gm;
        }
      };

      // Sᵀ/S (and dPᵀ/dP) of sub-step c into TMEM buffer c.n & 1
      auto producers = [&](const GSub& c) {
        const int b = c.n & 1;
        if (c.unit_first) ok = mbar_wait(&bar->outer_full[c.m & 1], (c.m >> 1) & 1, err, kErrG | 5);
        if (ok && c.hh == 0) ok = mbar_wait(&bar->inner_full[c.st], (c.ni / kStages) & 1, err, kErrG | 6);
        if (ok && c.n >= 2) ok = mbar_wait(&bar->s_free[b], ((c.n >> 1) - 1) & 1, err, kErrG | 7);
        if (!ok) return;
        tc_fence_after();
        const uint64_t o0 = dOuter + (uint64_t)((c.m & 1) * Tr::kOuterTiles) * kTD;
        const uint64_t o1 = o0 + kTD;
        const uint64_t in0 = dInner + (uint64_t)(c.st * 2) * kTD;
        const uint64_t in1 = in0 + kTD;
        const uint64_t half = (uint64_t)(64 * c.hh) * 8;
        const uint32_t sc = tbase + 128 * b;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          if (R == kFwd) {
            mma_bf16(sc, o0 + 2 * kk, in0 + half + 2 * kk, id_p, kk > 0);        // S = Q·Kᵀ
          } else if (R == kDKV) {
            mma_bf16(sc, o0 + 2 * kk, in0 + half + 2 * kk, id_p, kk > 0);        // Sᵀ = K·Qᵀ
            mma_bf16(sc + 64, o1 + 2 * kk, in1 + half + 2 * kk, id_p, kk > 0);   // dPᵀ = V·dOᵀ
          } else {
            mma_bf16(sc, o0 + 2 * kk, in0 + half + 2 * kk, id_p, kk > 0);        // S = Q·Kᵀ
            mma_bf16(sc + 64, o1 + 2 * kk, in1 + half + 2 * kk, id_p, kk > 0);   // dP = dO·Vᵀ
          }
        }
        mma_commit(&bar->s_full[b]);
      };

      // accumulator MMAs of sub-step c (its bf16 tiles in shared buffer c.n & 1)
      auto consumers = [&](const GSub& c) {
        const int b = c.n & 1, ub = c.m & 1;
        ok = mbar_wait(&bar->p_full[b], (c.n >> 1) & 1, err, kErrG | 3);
        if (ok && c.unit_first && c.m >= 2)
          ok = mbar_wait(&bar->acc_free[ub], ((c.m >> 1) - 1) & 1, err, kErrG | 4);
        if (!ok) return;
        tc_fence_after();
        const uint64_t in0 = dInner + (uint64_t)(c.st * 2) * kTD;   // K / Q / K
        const uint64_t in1 = in0 + kTD;                              // V / dO / V
        const uint64_t e0 = dEpi + (uint64_t)(b * Tr::kEpiTiles) * kTD;
        const uint32_t acc_col = tbase + 256 + ub * Tr::kAccCols;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t rows = (uint64_t)(64 * c.hh + 16 * kk) * 8;  // 16 B units
          const uint32_t acc = (c.unit_first && kk == 0) ? 0u : 1u;
          if (R == kFwd) {
            mma_bf16(acc_col, e0 + 2 * kk, in1 + rows, id_c, acc);            // O += P·V
          } else if (R == kDKV) {
            mma_bf16(acc_col + 64, e0 + 2 * kk, in1 + rows, id_c, acc);       // dV += (ατ)ᵀ·dO
            mma_bf16(acc_col, e0 + kTD + 2 * kk, in0 + rows, id_c, acc);      // dK += dSᵀ·Q
          } else {
            mma_bf16(acc_col, e0 + 2 * kk, in0 + rows, id_c, acc);            // dQ += dS·K
          }
        }
        mma_commit(&bar->p_free[b]);
        if (R == kDKV && p.ds_store) {
          // this sub-step's dSᵀ tile (the epilogue's second tile, fenced for
          // the async proxy before p_full) to the scratch, for DQS; the
          // buffer's second p_free arrival comes once the store has read it,
          // checked one sub-step later so the wait rarely blocks
          const int t = ds_tile(c.bh, c.ot, c.ot + c.x, nT, p.dsD) + c.hh;
          tma_store_2d(&tmds, sEpi + (b * 2 + 1) * kTileBytes, 0, t * kTile);
          bulk_commit_group();
          if (c.n >= 1) {
            bulk_wait_group_read1();
            mbar_arrive(&bar->p_free[(c.n - 1) & 1]);
          }
        }
        if (c.hh == 1) mma_commit(&bar->inner_empty[c.st]);
        if (c.last) mma_commit(&bar->acc_full[ub]);
      };

      // DQS: dQ += dS·K_h straight from the stored dSᵀ halves (no producers,
      // no element math)
      auto consumers_dqs = [&](const GSub& c) {
        const int ub = c.m & 1;
        if (c.hh == 0) ok = mbar_wait(&bar->inner_full[c.st], (c.ni / kStages) & 1, err, kErrG | 6);
        if (ok && c.unit_first && c.m >= 2)
          ok = mbar_wait(&bar->acc_free[ub], ((c.m >> 1) - 1) & 1, err, kErrG | 4);
        if (!ok) return;
        tc_fence_after();
        const uint64_t k0 = dInner + (uint64_t)(c.st * Tr::kInnerTiles) * kTD;
        const uint64_t ds = dDSmn + (uint64_t)(c.st * Tr::kInnerTiles) * kTD;
        const uint32_t acc_col = tbase + 256 + ub * Tr::kAccCols;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t rows = (uint64_t)(64 * c.hh + 16 * kk) * 8;  // key rows, 16 B units
          const uint32_t acc = (c.unit_first && kk == 0) ? 0u : 1u;
          mma_bf16(acc_col, ds + rows, k0 + rows, id_q, acc);
        }
        if (c.hh == 1) mma_commit(&bar->inner_empty[c.st]);
        if (c.last) mma_commit(&bar->acc_full[ub]);
      };

      // Producers of sub-step n are issued before the consumers of n − 1, so
      // the epilogue of n overlaps the accumulator MMAs of n − 1.  Each kind
      // of MMA has exactly one issue site: the consumer MMAs of a unit's last
      // sub-step, when issued from a second inlined copy of this code after
      // the loop, read their B tile with a corrupted layout (every 16-byte
      // column chunk of the product equal to the first) whenever the wait
      // before them ran out of line.
      if constexpr (R == kDQS) {
        GSub cur{};
        while (ok && next_sub(cur)) consumers_dqs(cur);
      } else {
        GSub cur{}, prev{};
        bool have_prev = false;
        while (ok) {
          const bool more = next_sub(cur);
          if (more) producers(cur);
          if (ok && have_prev) consumers(prev);
          if (!more) break;
          prev = cur;
          have_prev = true;
        }
        if (R == kDKV && p.ds_store) bulk_wait_group0();  // the dSᵀ stores have landed
      }
    }
  } else if (warp < 4 || warp >= 12) {
    // ─────────── output warps: accumulators → bf16 → TMA store ───────────
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // TMEM lane = tile row
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    float th[32];
#pragma unroll
    for (int z = 0; z < 32; ++z) th[z] = p.theta ? __ldg(p.theta + z) : 0.f;
    bool ok = true;
    for (int k = blockIdx.x, m = 0; k < p.units && ok; k += G, ++m) {
      int bh, ot, fi, nin;
      unit_of(R, k, BH, nT, p.local, p.W, bh, ot, fi, nin);
      const int b = bh / H, h = bh % H;
      const int ub = m & 1, os = m & 1;
      ok = mbar_wait(&bar->acc_full[ub], (m >> 1) & 1, err, kErrG | 8);
      if (R == kFwd && ok) ok = mbar_wait(&bar->mass_ready[ub], (m >> 1) & 1, err, kErrG | 9);
      // DQS loads nothing into its outer slots: the staging slot is free
      // again once the store from it two units back has read it
      if (R == kDQS && ok && m >= 2) ok = mbar_wait(&bar->outer_empty[os], ((m >> 1) - 1) & 1, err, kErrG | 16);
      if (!ok) break;
      __syncwarp();
      tc_fence_after();
      const int pos = ot * kTile + r;
      const uint32_t acc = tbase + lane_off + 256 + ub * Tr::kAccCols;
      uint8_t* o = sOuter + os * Tr::kOuterTiles * kTileBytes;  // dead outer slot
      const uint32_t st0 = smem_u32(o);
      if (R == kFwd) {
        // the τ-mass halves are read before acc_free is handed back: the
        // epilogue rewrites this mass slot (outer tile m+2) once acc_free fires
        const float mass = sMass[(ub * 2 + 0) * kTile + r] + sMass[(ub * 2 + 1) * kTile + r];
        uint32_t g[64];
        tmem_ld32_wait(acc, g);
        tmem_ld32_wait(acc + 32, g + 32);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->acc_free[ub]);
        float inv = 1.f;
        if (p.norm == BOZO_NORM_MASS) inv = 1.f / fmaxf(mass, kMassEps);
        else if (p.norm == BOZO_NORM_COUNT) inv = 1.f / (float)max(min(pos, p.W), 1);  // model.py:261-264
#pragma unroll
        for (int z = 0; z < 8; ++z) {
          uint32_t w4[4];
#pragma unroll
          for (int y = 0; y < 4; ++y)
            w4[y] = pack_bf16(__uint_as_float(g[8 * z + 2 * y]) * inv,
                              __uint_as_float(g[8 * z + 2 * y + 1]) * inv);
          st_shared_v4(st0 + sw128_off(r, z), w4[0], w4[1], w4[2], w4[3]);
        }
        if (p.row_mass && pos < T) p.row_mass[(long long)bh * T + pos] = mass;
      } else {
        // dK (DKV) / dQ (DQ): inverse RoPE at this row's position
        // dK (DKV) / dQ (DQ) in the accumulator's first 64 columns; frequency
        // group c8 pairs columns [8c8, 8c8+8) with [32+8c8, 32+8c8+8)
#pragma unroll
        for (int c8 = 0; c8 < 4; c8 += 2) {
          uint32_t g[32];
          tmem_ld8x4_wait(acc + 8 * c8, acc + 32 + 8 * c8, acc + 8 * c8 + 8, acc + 40 + 8 * c8, g);
#pragma unroll
          for (int hg = 0; hg < 2; ++hg) {
            const int grp = c8 + hg;
            float o8[16];
#pragma unroll
            for (int z = 0; z < 8; ++z) {
              float cs = 1.f, sn = 0.f;
              if (p.theta && pos < T) rope_cs(pos, th[grp * 8 + z], cs, sn);
              const float x1 = __uint_as_float(g[16 * hg + z]);
              const float x2 = __uint_as_float(g[16 * hg + 8 + z]);
              o8[z] = x1 * cs + x2 * sn;
              o8[8 + z] = x2 * cs - x1 * sn;
            }
            st_shared_v4(st0 + sw128_off(r, grp), pack_bf16(o8[0], o8[1]), pack_bf16(o8[2], o8[3]),
                         pack_bf16(o8[4], o8[5]), pack_bf16(o8[6], o8[7]));
            st_shared_v4(st0 + sw128_off(r, 4 + grp), pack_bf16(o8[8], o8[9]),
                         pack_bf16(o8[10], o8[11]), pack_bf16(o8[12], o8[13]),
                         pack_bf16(o8[14], o8[15]));
          }
        }
        if (R == kDKV) {
          uint32_t g[64];
          tmem_ld32_wait(acc + 64, g);
          tmem_ld32_wait(acc + 96, g + 32);
          const uint32_t st1 = st0 + kTileBytes;
#pragma unroll
          for (int z = 0; z < 8; ++z) {
            uint32_t w4[4];
#pragma unroll
            for (int y = 0; y < 4; ++y)
              w4[y] = pack_bf16(__uint_as_float(g[8 * z + 2 * y]), __uint_as_float(g[8 * z + 2 * y + 1]));
            st_shared_v4(st1 + sw128_off(r, z), w4[0], w4[1], w4[2], w4[3]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->acc_free[ub]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->staged);
      if (warp == 2 && lane == 0) {
        ok = mbar_wait(&bar->staged, m & 1, err, kErrG | 10);
        if (ok) {
          tma_store_4d(&tmout0, o, 0, h, ot * kTile, b);
          if (R == kDKV) tma_store_4d(&tmout1, o + kTileBytes, 0, h, ot * kTile, b);
          bulk_commit_group();
          bulk_wait_group_read0();
          mbar_arrive(&bar->outer_empty[os]);  // the TMA may refill this outer slot
        }
      }
      __syncwarp();
    }
    if (warp == 2 && lane == 0) bulk_wait_group0();
  } else {
    // ─────────────────────────── epilogue (8 warps) ───────────────────────────
    const int e = warp - 4;
    const int qd = warp & 3;
    const int hf = e >> 2;  // which 32 of the sub-step's 64 inner columns
    const int r = qd * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const uint32_t epi = smem_u32(sEpi);
    bool ok = true;
    int n = 0, ni = 0;
    // (DQS has no element math: its epilogue warps only reach the final sync)
    for (int k = blockIdx.x, m = 0; R != kDQS && k < p.units && ok; k += G, ++m) {
      int bh, ot, fi, nin;
      unit_of(R, k, BH, nT, p.local, p.W, bh, ot, fi, nin);
      const int b = bh / H, h = bh % H;
      const int os = m & 1;
      const int orow = ot * kTile + r;  // this thread's outer position
      float mass = 0.f;
      float row_ad = 0.f, row_bd = 0.f;
      if (R == kDQ) {
        ok = mbar_wait(&bar->outer_full[os], (m >> 1) & 1, err, kErrG | 11);
        if (!ok) break;
        row_ad = sOCoef[(os * 3 + 1) * kTile + r];
        row_bd = sOCoef[(os * 3 + 2) * kTile + r];
      }
      for (int x = 0; x < nin && ok; ++x) {
        const int it = fi + x;
        const int st = ni % kStages;
        if (R == kDKV) {
          ok = mbar_wait(&bar->inner_full[st], (ni / kStages) & 1, err, kErrG | 12);
          if (!ok) break;
        }
        const float* cf = sICoef + st * 3 * kTile;
        for (int hh = 0; hh < 2 && ok; ++hh) {
          const int bb = n & 1;
          ok = mbar_wait(&bar->s_full[bb], (n >> 1) & 1, err, kErrG | 13);
          if (!ok) break;
          __syncwarp();
          tc_fence_after();
          uint32_t pk[2][8], dk[2][8];
#pragma unroll
          for (int ss = 0; ss < 2; ++ss) {
            const int c0 = 64 * hh + 32 * hf + 16 * ss;  // first inner row (within tile) of the piece
            const int ipos0 = it * kTile + c0;          // its position
            // query / key positions of (row, column e): FWD/DQ row = query, DKV row = key
            uint32_t Rg[32];
            const uint32_t col = tbase + lane_off + 128 * bb + 32 * hf + 16 * ss;
            if (R == kFwd) {
              tmem_ld16_wait(col, Rg);
            } else {
              tmem_ld16x2_wait(col, col + 64, Rg);
            }
            // Does this piece touch the exported τ?  Local windows export every
            // valid element; the global block only the last tw keys
            // (model.py:233-236), i.e. pieces whose key positions reach T − tw
            // — uniform over the warp for FWD/DQ (keys = inner positions), per
            // thread for DKV (key = this row).  Only those pieces take the
            // element loop with the τ store / cotangent read.
            const bool pexp = kExtra && (p.local || (R == kDKV ? orow >= T - p.tw : ipos0 + 15 >= T - p.tw));
            auto piece = [&](auto exp_tag) {
              constexpr bool kExp = decltype(exp_tag)::value;
#pragma unroll
            for (int e4 = 0; e4 < 16; e4 += 2) {
              float pv[2], dv[2];
#pragma unroll
              for (int z = 0; z < 2; ++z) {
                const int ee = e4 + z;
                const int ipos = ipos0 + ee;
                const int tq = (R == kDKV) ? ipos : orow;  // query position
                const int sk = (R == kDKV) ? orow : ipos;  // key position
                // global: s ≤ t; local: 1 ≤ t − s ≤ W, window slot w = W − (t − s)
                const int dts = tq - sk;
                const bool valid = tq < T && (p.local ? (dts >= 1 && dts <= p.W) : dts >= 0);
                float x = __uint_as_float(Rg[ee]) * p.half_inv_scale;
                if constexpr (kBias) {
                  const int tqc = min(tq, T - 1);
                  const int col = p.local ? (valid ? p.W - dts : 0) : min(sk, T - 1);
                  x = fmaf(0.5f, __ldg(p.bias + b * p.bs0 + (long long)tqc * p.bs1 + (long long)col * p.bs2), x);
                }
                const float thv = tanh_approx(x);
                if (R == kFwd) {
                  const float tau = valid ? fmaf(0.5f, thv, 0.5f) : 0.f;
                  mass += tau;
                  pv[z] = tau;
                  if constexpr (kExp) {
                    // exported τ: local [B,T,H,W] at w; global window of the last
                    // tw keys, column T−1−s (model.py:233-236)
                    const int col = p.local ? p.W - dts : T - 1 - sk;
                    if (valid && (unsigned)col < (unsigned)p.tw)
                      p.tau[((long long)(b * T + tq) * H + h) * p.tw + col] = __float2bfloat16_rn(tau);
                  }
                } else {
                  float ad, bd, ah = 0.f;
                  if (R == kDKV) {
                    const int qi = c0 + ee;  // query row within the inner tile
                    ah = cf[qi];
                    ad = cf[kTile + qi];
                    bd = cf[2 * kTile + qi];
                  } else {
                    ad = row_ad;
                    bd = row_bd;
                  }
                  float dt = fmaf(ad, __uint_as_float(Rg[16 + ee]), bd);
                  if constexpr (kExp) {
                    const int col = p.local ? p.W - dts : T - 1 - sk;
                    if (valid && (unsigned)col < (unsigned)p.tw)
                      dt = fmaf(__bfloat162float(p.dtau[((long long)(b * T + tq) * H + h) * p.tw + col]),
                                p.ds_scale, dt);
                  }
                  dv[z] = valid ? dt * fmaf(-thv, thv, 1.f) : 0.f;
                  if (R == kDKV) pv[z] = valid ? fmaf(ah, thv, ah) : 0.f;
                }
              }
              if (R == kFwd || R == kDKV) pk[ss][e4 >> 1] = pack_bf16(pv[0], pv[1]);
              if (R != kFwd) dk[ss][e4 >> 1] = pack_bf16(dv[0], dv[1]);
            }
            };
            // Interior piece: every element valid for every row of the warp
            // (inside the causal triangle / the window band, rows and columns
            // below T) and nothing exported — no positions, mask or selects
            // per element, and DKV's per-query coefficients as 16-byte
            // broadcast loads.  Decided warp-uniformly.
            bool tfull;
            if (R == kDKV)  // row = key orow, columns = queries ipos0 … ipos0+15
              tfull = ipos0 + 15 < T && (p.local ? (ipos0 - orow >= 1 && ipos0 + 15 - orow <= p.W)
                                                 : ipos0 >= orow);
            else            // row = query orow, columns = keys
              tfull = orow < T && (p.local ? (orow - ipos0 - 15 >= 1 && orow - ipos0 <= p.W)
                                           : ipos0 + 15 <= orow);
            const bool full = __all_sync(0xffffffffu, tfull && !pexp);
            auto piece_full = [&]() {
              long long bbase = 0, bstep = 0;
              if constexpr (kBias) {
                // element ee: bias at (query, slot) — global slot = key, local
                // slot = W − (t − s); one base per piece, a constant step
                if (R == kDKV) {  // query varies with ee
                  bbase = b * p.bs0 + (long long)ipos0 * p.bs1 +
                          (long long)(p.local ? p.W - (ipos0 - orow) : orow) * p.bs2;
                  bstep = p.bs1 - (p.local ? p.bs2 : 0);
                } else {          // key varies with ee
                  bbase = b * p.bs0 + (long long)orow * p.bs1 +
                          (long long)(p.local ? p.W - (orow - ipos0) : ipos0) * p.bs2;
                  bstep = p.bs2;
                }
              }
#pragma unroll
              for (int e4 = 0; e4 < 16; e4 += 4) {
                float ah[4] = {0.f, 0.f, 0.f, 0.f}, ad[4], bd[4];
                if (R == kDKV) {
                  const float4 a4 = *reinterpret_cast<const float4*>(cf + c0 + e4);
                  const float4 d4 = *reinterpret_cast<const float4*>(cf + kTile + c0 + e4);
                  const float4 b4 = *reinterpret_cast<const float4*>(cf + 2 * kTile + c0 + e4);
                  ah[0] = a4.x; ah[1] = a4.y; ah[2] = a4.z; ah[3] = a4.w;
                  ad[0] = d4.x; ad[1] = d4.y; ad[2] = d4.z; ad[3] = d4.w;
                  bd[0] = b4.x; bd[1] = b4.y; bd[2] = b4.z; bd[3] = b4.w;
                } else {
#pragma unroll
                  for (int z = 0; z < 4; ++z) { ad[z] = row_ad; bd[z] = row_bd; }
                }
                float pv[4], dv[4];
#pragma unroll
                for (int z = 0; z < 4; ++z) {
                  const int ee = e4 + z;
                  float x = __uint_as_float(Rg[ee]) * p.half_inv_scale;
                  if constexpr (kBias) x = fmaf(0.5f, __ldg(p.bias + bbase + ee * bstep), x);
                  const float thv = tanh_approx(x);
                  if (R == kFwd) {
                    pv[z] = fmaf(0.5f, thv, 0.5f);
                    mass += pv[z];
                  } else {
                    const float dt = fmaf(ad[z], __uint_as_float(Rg[16 + ee]), bd[z]);
                    dv[z] = dt * fmaf(-thv, thv, 1.f);
                    if (R == kDKV) pv[z] = fmaf(ah[z], thv, ah[z]);
                  }
                }
                if (R == kFwd || R == kDKV) {
                  pk[ss][e4 >> 1] = pack_bf16(pv[0], pv[1]);
                  pk[ss][(e4 >> 1) + 1] = pack_bf16(pv[2], pv[3]);
                }
                if (R != kFwd) {
                  dk[ss][e4 >> 1] = pack_bf16(dv[0], dv[1]);
                  dk[ss][(e4 >> 1) + 1] = pack_bf16(dv[2], dv[3]);
                }
              }
            };
            if (full)
              piece_full();
            else if (pexp)
              piece(std::true_type{});
            else
              piece(std::false_type{});
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar->s_free[bb]);
          if (n >= 2) ok = mbar_wait(&bar->p_free[bb], ((n >> 1) - 1) & 1, err, kErrG | 14);
          if (!ok) break;
          const uint32_t t0 = epi + (bb * Tr::kEpiTiles) * kTileBytes;
#pragma unroll
          for (int ss = 0; ss < 2; ++ss) {
            const int c16 = (32 * hf + 16 * ss) >> 3;
            if (R == kFwd || R == kDKV) {
              st_shared_v4(t0 + sw128_off(r, c16), pk[ss][0], pk[ss][1], pk[ss][2], pk[ss][3]);
              st_shared_v4(t0 + sw128_off(r, c16 + 1), pk[ss][4], pk[ss][5], pk[ss][6], pk[ss][7]);
            }
            if (R != kFwd) {
              const uint32_t td = (R == kDKV) ? t0 + kTileBytes : t0;
              st_shared_v4(td + sw128_off(r, c16), dk[ss][0], dk[ss][1], dk[ss][2], dk[ss][3]);
              st_shared_v4(td + sw128_off(r, c16 + 1), dk[ss][4], dk[ss][5], dk[ss][6], dk[ss][7]);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar->p_full[bb]);
          ++n;
        }
        ++ni;
      }
      if (R == kFwd && ok) {
        // the output warps wait for both halves' τ-mass of every row
        const int ub = m & 1;
        if (m >= 2) ok = mbar_wait(&bar->acc_free[ub], ((m >> 1) - 1) & 1, err, kErrG | 15);
        if (!ok) break;
        sMass[(ub * 2 + hf) * kTile + r] = mass;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->mass_ready[ub]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

template <int R, bool kBias, bool kExtra>
cudaError_t launch_g(const CUtensorMap* m, const GlobTC& a, cudaStream_t st) {
  auto kern = tc_global_kernel<R, kBias, kExtra>;
  const size_t smem = glayout<R>().total + 1024;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int grid = std::min(num_sms(), a.units);
  kern<<<grid, kThreads, smem, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], m[6], a);
  return cudaGetLastError();
}

template <int R>
cudaError_t launch_role(const CUtensorMap* m, const GlobTC& a, bool bias, bool extra, cudaStream_t st) {
  if (bias && extra) return launch_g<R, true, true>(m, a, st);
  if (bias) return launch_g<R, true, false>(m, a, st);
  if (extra) return launch_g<R, false, true>(m, a, st);
  return launch_g<R, false, false>(m, a, st);
}

bool out_ok(const void* ptr) { return ptr && (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

// Longest inner range of a DKV unit: every query tile for the global block,
// the band's tiles for a local window.
int ds_depth(int nT, int mode, int W) {
  return mode == BOZO_MODE_GLOBAL ? nT : std::min(nT, (kTile - 1 + W) / kTile + 1);
}

}  // namespace

size_t tc_global_ds_bytes(int B, int T, int H, int mode, int W) {
  if (B <= 0 || T <= 0 || H <= 0) return 0;
  if (mode == BOZO_MODE_LOCAL && W <= 128) return 0;  // the band kernels serve it
  const int nT = (T + kTile - 1) / kTile;
  const long long tiles = (long long)B * H * nT * ds_depth(nT, mode, W) * 2;
  if (tiles * kTile > 0x7fffffffLL) return 0;  // beyond a tensor map's row coordinate
  return (size_t)tiles * kTileBytes;
}

bool tc_global_fwd_eligible(const FwdP& p) {
  if (p.HD != kHD || (p.mode == BOZO_MODE_LOCAL && p.W < 1)) return false;
  if (p.mode == BOZO_MODE_GLOBAL && p.norm == BOZO_NORM_COUNT) return false;
  if (p.out_dt != BOZO_DT_BF16 || !out_ok(p.out)) return false;
  if (p.tau && p.tau_dt != BOZO_DT_BF16) return false;
  if (!tma_view_ok(p.q, p.B, p.T, p.H) || !tma_view_ok(p.k, p.B, p.T, p.H) ||
      !tma_view_ok(p.v, p.B, p.T, p.H))
    return false;
  // RoPE: the kernel reads the rotated copies, which the caller must request
  if (p.cos && (!out_ok(p.q_rot) || !out_ok(p.k_rot))) return false;
  return tmap_encoder_available();
}

cudaError_t launch_tc_global_fwd(const FwdP& p, cudaStream_t st, int* launches) {
  *launches = 0;
  GlobTC a{};
  a.B = p.B; a.T = p.T; a.H = p.H; a.BH = p.B * p.H;
  a.nT = (p.T + kTile - 1) / kTile;
  a.units = a.BH * a.nT;
  a.tw = p.tau ? p.W : 0;
  a.local = p.mode == BOZO_MODE_LOCAL;
  a.W = p.W;
  a.half_inv_scale = 0.5f / p.scale;
  a.norm = p.norm;
  a.bias = p.bias; a.bs0 = p.bs0; a.bs1 = p.bs1; a.bs2 = p.bs2;
  a.tau = static_cast<__nv_bfloat16*>(p.tau);
  a.row_mass = p.row_mass;
  a.err = p.err;
  cudaError_t e;
  const long long ob = (long long)p.T * p.H * kHD, ot = (long long)p.H * kHD, oh = kHD;
  const void* qp = p.q.p;
  const void* kp = p.k.p;
  long long qs[3] = {p.q.sb, p.q.st, p.q.sh}, ks[3] = {p.k.sb, p.k.st, p.k.sh};
  if (p.cos) {
    if ((e = launch_rope_copy(p, st, launches)) != cudaSuccess) return e;
    qp = p.q_rot;
    kp = p.k_rot;
    qs[0] = ks[0] = ob; qs[1] = ks[1] = ot; qs[2] = ks[2] = oh;
  }
  if (p.tau) {
    e = cudaMemsetAsync(p.tau, 0, (size_t)p.B * p.T * p.H * p.W * sizeof(__nv_bfloat16), st);
    if (e != cudaSuccess) return e;
  }
  CUtensorMap m[7];
  if (!make_tmap_bthd(&m[0], qp, qs[0], qs[1], qs[2], p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&m[2], kp, ks[0], ks[1], ks[2], p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&m[3], p.v.p, p.v.sb, p.v.st, p.v.sh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&m[4], p.out, ob, ot, oh, p.B, p.T, p.H, kTile))
    return cudaErrorInvalidValue;
  m[1] = m[0];
  m[5] = m[4];
  m[6] = m[0];  // unused
  *launches += 1;
  return launch_role<kFwd>(m, a, p.bias != nullptr, p.tau != nullptr, st);
}

bool tc_global_bwd_eligible(const BwdP& p) {
  if (p.HD != kHD || (p.mode == BOZO_MODE_LOCAL && p.W < 1)) return false;
  if (p.B > 65535 || (long long)p.T * p.H * 8 > 0x7fffffffLL) return false;  // pre-pass grid
  if (p.mode == BOZO_MODE_GLOBAL && p.norm == BOZO_NORM_COUNT) return false;
  if (p.dq_dt != BOZO_DT_BF16 || p.dk_dt != BOZO_DT_BF16 || p.dv_dt != BOZO_DT_BF16) return false;
  if (!tma_view_ok(p.q, p.B, p.T, p.H) || !tma_view_ok(p.k, p.B, p.T, p.H) ||
      !tma_view_ok(p.v, p.B, p.T, p.H) || !tma_view_ok(p.dout, p.B, p.T, p.H))
    return false;
  if (p.norm == BOZO_NORM_MASS) {
    if (p.out.dt != BOZO_DT_BF16 || p.out.sd != 1 || (reinterpret_cast<uintptr_t>(p.out.p) & 15) ||
        (p.out.sb % 8) || (p.out.st % 8) || (p.out.sh % 8))
      return false;
  }
  if (p.dtau && p.dtau_dt != BOZO_DT_BF16) return false;
  if (!out_ok(p.dq) || !out_ok(p.dk) || !out_ok(p.dv)) return false;
  if (p.cos && (!p.theta || !p.qk_rotated)) return false;
  if (!out_ok(p.coef)) return false;
  return tmap_encoder_available();
}

cudaError_t launch_tc_global_bwd(const BwdP& p, cudaStream_t st, int* launches) {
  GlobTC a{};
  a.B = p.B; a.T = p.T; a.H = p.H; a.BH = p.B * p.H;
  a.nT = (p.T + kTile - 1) / kTile;
  a.units = a.BH * a.nT;
  a.tpad = a.nT * kTile;
  a.tw = p.dtau ? p.W : 0;
  a.local = p.mode == BOZO_MODE_LOCAL;
  a.W = p.W;
  a.half_inv_scale = 0.5f / p.scale;
  a.ds_scale = 0.25f / p.scale;
  a.norm = p.norm;
  a.theta = p.cos ? p.theta : nullptr;
  a.bias = p.bias; a.bs0 = p.bs0; a.bs1 = p.bs1; a.bs2 = p.bs2;
  a.dtau = static_cast<const __nv_bfloat16*>(p.dtau);
  a.coef = p.coef;
  a.err = p.err;
  cudaError_t e = launch_alpha_beta(p, a.tpad, a.ds_scale, p.coef, st);
  if (e != cudaSuccess) return e;
  CUtensorMap mq, mk, mv, mdo, mdq, mdk, mdv;
  const long long ob = (long long)p.T * p.H * kHD, ot = (long long)p.H * kHD, oh = kHD;
  if (!make_tmap_bthd(&mq, p.q.p, p.q.sb, p.q.st, p.q.sh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&mk, p.k.p, p.k.sb, p.k.st, p.k.sh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&mv, p.v.p, p.v.sb, p.v.st, p.v.sh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&mdo, p.dout.p, p.dout.sb, p.dout.st, p.dout.sh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&mdq, p.dq, ob, ot, oh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&mdk, p.dk, ob, ot, oh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&mdv, p.dv, ob, ot, oh, p.B, p.T, p.H, kTile))
    return cudaErrorInvalidValue;
  const bool bias = p.bias != nullptr, dt = p.dtau != nullptr;
  // with room for the dSᵀ scratch, DKV stores its dSᵀ tiles and the dQ pass
  // multiplies them by K (DQS); otherwise the dQ pass recomputes S and dP (DQ)
  CUtensorMap mds = mq;
  if (p.ds_scratch) {
    a.dsD = ds_depth(a.nT, p.mode, p.W);
    const long long rows = (long long)a.BH * a.nT * a.dsD * 2 * kTile;
    if (!make_tmap_2d(&mds, p.ds_scratch, false, kHD, (uint64_t)rows, kHD * 2, kHD, kTile))
      return cudaErrorInvalidValue;
    a.ds_store = 1;
  }
  {
    const CUtensorMap m[7] = {mk, mv, mq, mdo, mdk, mdv, mds};
    if ((e = launch_role<kDKV>(m, a, bias, dt, st)) != cudaSuccess) return e;
  }
  if (p.ds_scratch) {
    const CUtensorMap m[7] = {mq, mq, mk, mk, mdq, mdq, mds};
    if ((e = launch_g<kDQS, false, false>(m, a, st)) != cudaSuccess) return e;
  } else {
    const CUtensorMap m[7] = {mq, mdo, mk, mv, mdq, mdq, mds};
    if ((e = launch_role<kDQ>(m, a, bias, dt, st)) != cudaSuccess) return e;
  }
  *launches = 3;
  return cudaSuccess;
}

}  // namespace bozo
