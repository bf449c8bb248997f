// tc_fwd.cu — tcgen05 / TMA / TMEM forward of the local tension operator
// for bf16 Q/K/V with HD = 64 and W ≤ 128 (sm_100a).
//
// Semantics: triton_tension/kernel.py:41-126 (τ = σ(q·k/scale + bias) over the
// W keys before each query, self excluded, S = Σ τ·V, optional τ export)
// fused with RoPE (model.py:75-81) and the model's normalisation
// (τ-mass model.py:257-258 / count model.py:261-264).
//
// Design (one persistent CTA per SM, 14 warps):
//   * work = 128-row query tiles of one (b, h), flattened b-h-major; each CTA
//     streams a contiguous range, so the K/V tile of query tile j stays in
//     shared memory and serves as the W-key halo of tile j+1 (3-slot ring):
//     every Q/K/V byte is read from HBM once (plus one halo tile per CTA);
//   * warp 0  — TMA producer (4-D tensor maps, 128B swizzle);
//   * warp 1  — tcgen05 MMA issuer: S = Q·[K_{j-1} tail ; K_j]ᵀ (M=128,
//               N = Wr + 128, fp32 in TMEM), then O = P·[V_{j-1} tail ; V_j];
//   * warps 2,3,12,13 — RoPE: rotate Q_j and K_j in place (same positions,
//               one cos/sin fetch for both);
//   * warps 4-11 — epilogue: TMEM → registers, band mask, bias, sigmoid
//               (0.5·tanh(x/2)+0.5), τ-mass, optional τ export, bf16 P tile in
//               the UMMA K-major layout; then O/mass → bf16 tile → TMA store.
//   TMEM holds two (S, O) buffers when Wr ≤ 64 so tile j+1's QKᵀ overlaps
//   tile j's epilogue.  Optional inputs/outputs (bias, τ) are template
//   parameters so the common path has no per-element branches.  All
//   mbarrier waits are bounded (tc_ptx.cuh).
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
constexpr int kQSlots = 2;
constexpr int kKVSlots = 3;
constexpr int kThreads = 14 * 32;
constexpr int kRotThreads = 128;
constexpr int kErrFwd = 0x100;  // device error codes (| site)

struct FwdTC {
  int B, T, H, W, Wr, nT, total;
  int norm, nbuf, ncols, pblocks;
  float half_inv_scale;
  const float* theta;  // RoPE frequencies [32] or null (no RoPE)
  const float* bias;
  long long bs0, bs1, bs2;
  __nv_bfloat16* tau;
  float* row_mass;
  int store_rot;  // also TMA-store the rotated Q/K tiles (q_rot, k_rot)
  int* err;
};

struct __align__(8) Bars {
  uint64_t q_full[kQSlots], q_ready[kQSlots], q_empty[kQSlots];
  uint64_t kv_full[kKVSlots], k_ready[kKVSlots], kv_empty[kKVSlots];
  uint64_t s_full[2], o_full[2], tmem_empty[2];
  uint64_t p_full;
  uint64_t mass_ready[2];  // the 8 epilogue warps have published their τ-mass halves
  uint64_t ostage_full, ostage_empty;
  uint32_t tmem_base;
};

struct Layout {
  uint32_t q, k, v, p, o, mass, bars, total;
};

__host__ __device__ inline Layout fwd_layout(int pblocks) {
  Layout L;
  L.q = 0;
  L.k = L.q + kQSlots * kTileBytes;
  L.v = L.k + kKVSlots * kTileBytes;
  L.p = L.v + kKVSlots * kTileBytes;
  L.o = L.p + pblocks * kTileBytes;
  L.mass = L.o + kTileBytes;  // float[2][2][128]
  L.bars = L.mass + 2 * 2 * kTile * 4;
  L.total = L.bars + (uint32_t)sizeof(Bars);
  return L;
}

// Rotate one 16-byte chunk pair (elements 8c..8c+7 and 32+8c..) of row r of a
// 128B-swizzled [128 x 64] bf16 tile by the given cos/sin (8 frequencies).
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

// Rotate rows [0,128) of tiles a (and b, if non-null) — same positions t0+r.
// Thread tid always handles 16-byte chunk c = tid & 3, so it keeps the eight
// frequencies θ[8c..8c+7] in registers and evaluates cos/sin on the fly.
__device__ void rope_tiles(uint8_t* ta, uint8_t* tb, int t0, int T, const float (&th)[8], int tid) {
  const uint32_t ba = smem_u32(ta), bb = tb ? smem_u32(tb) : 0u;
  const int c = tid & 3;
  for (int item = tid; item < kTile * 4; item += kRotThreads) {
    const int r = item >> 2;
    const int t = t0 + r;
    if (t >= T) continue;
    float cs[8], sn[8];
#pragma unroll
    for (int z = 0; z < 8; ++z) rope_cs(t, th[z], cs[z], sn[z]);
    rope_chunk(ba, r, c, cs, sn);
    if (tb) rope_chunk(bb, r, c, cs, sn);
  }
}

template <bool kBias, bool kTau>
__global__ void __launch_bounds__(kThreads, 1)
    tc_fwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmo,
                  const __grid_constant__ CUtensorMap tmqr, const __grid_constant__ CUtensorMap tmkr,
                  const FwdTC p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = fwd_layout(p.pblocks);
  uint8_t* sQ = smem + L.q;
  uint8_t* sK = smem + L.k;
  uint8_t* sV = smem + L.v;
  uint8_t* sP = smem + L.p;
  uint8_t* sO = smem + L.o;
  float* sMass = reinterpret_cast<float*>(smem + L.mass);
  Bars* bar = reinterpret_cast<Bars*>(smem + L.bars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = (int)((long long)blockIdx.x * p.total / gridDim.x);
  const int u1 = (int)((long long)(blockIdx.x + 1) * p.total / gridDim.x);

  // zero the P tile once: chunks outside every quadrant's band stay zero
  for (int i = threadIdx.x; i < p.pblocks * kTileBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(sP)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kQSlots; ++i) {
      mbar_init(&bar->q_full[i], 1);
      mbar_init(&bar->q_ready[i], 4);
      mbar_init(&bar->q_empty[i], 1);
    }
    for (int i = 0; i < kKVSlots; ++i) {
      mbar_init(&bar->kv_full[i], 1);
      mbar_init(&bar->k_ready[i], 4);
      mbar_init(&bar->kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->o_full[i], 1);
      mbar_init(&bar->tmem_empty[i], 8);
      mbar_init(&bar->mass_ready[i], 8);
    }
    mbar_init(&bar->p_full, 8);
    mbar_init(&bar->ostage_full, 8);
    mbar_init(&bar->ostage_empty, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&bar->tmem_base, 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bar->tmem_base;
  int* err = p.err;
  const int nT = p.nT, Wr = p.Wr;

  if (warp == 0) {
    // ─────────────── TMA producer ───────────────
    if (lane == 0) {
      prefetch_tmap(&tmq);
      prefetch_tmap(&tmk);
      prefetch_tmap(&tmv);
      prefetch_tmap(&tmo);
      if (p.store_rot) {
        prefetch_tmap(&tmqr);
        prefetch_tmap(&tmkr);
      }
      int n = 0, n_cur = 0;
      bool ok = true, pending_stores = false;
      // rotated tiles are stored from the ring slots: a slot is refilled only
      // after every store issued so far has finished reading shared memory
      auto before_refill = [&]() {
        if (pending_stores) {
          bulk_wait_group_read0();
          pending_stores = false;
        }
      };
      auto load_key = [&](int bh, int jj) {
        const int s = n % kKVSlots;
        if (n >= kKVSlots)
          ok = ok && mbar_wait(&bar->kv_empty[s], ((n / kKVSlots) - 1) & 1, err, kErrFwd | 1);
        if (!ok) return;
        before_refill();
        mbar_arrive_expect_tx(&bar->kv_full[s], 2 * kTileBytes);
        const int b = bh / p.H, h = bh % p.H;
        tma_load_4d(sK + s * kTileBytes, &tmk, &bar->kv_full[s], 0, h, jj * kTile, b);
        tma_load_4d(sV + s * kTileBytes, &tmv, &bar->kv_full[s], 0, h, jj * kTile, b);
        ++n;
      };
      // store RoPE(Q), RoPE(K) of tile (bh, j) once the rotators are done
      auto store_rot = [&](int it_s, int bh, int j, int nk) {
        const int qs = it_s % kQSlots, ks = nk % kKVSlots;
        ok = ok && mbar_wait(&bar->q_ready[qs], (it_s / kQSlots) & 1, err, kErrFwd | 15);
        ok = ok && mbar_wait(&bar->k_ready[ks], (nk / kKVSlots) & 1, err, kErrFwd | 16);
        if (!ok) return;
        tma_store_4d(&tmqr, sQ + qs * kTileBytes, 0, bh % p.H, j * kTile, bh / p.H);
        tma_store_4d(&tmkr, sK + ks * kTileBytes, 0, bh % p.H, j * kTile, bh / p.H);
        bulk_commit_group();
        pending_stores = true;
      };
      int prev_bh = 0, prev_j = 0, prev_n = 0;
      for (int u = u0, it = 0; u < u1 && ok; ++u, ++it) {
        const int bh = u / nT, j = u % nT;
        const int qs = it % kQSlots;
        if (it >= kQSlots)
          ok = mbar_wait(&bar->q_empty[qs], ((it / kQSlots) - 1) & 1, err, kErrFwd | 2);
        if (!ok) break;
        before_refill();
        mbar_arrive_expect_tx(&bar->q_full[qs], kTileBytes);
        tma_load_4d(sQ + qs * kTileBytes, &tmq, &bar->q_full[qs], 0, bh % p.H, j * kTile, bh / p.H);
        if (j >= 1 && u == u0) load_key(bh, j - 1);
        n_cur = n;
        load_key(bh, j);
        if (p.store_rot && it >= 1) store_rot(it - 1, prev_bh, prev_j, prev_n);
        prev_bh = bh; prev_j = j; prev_n = n_cur;
      }
      if (ok && p.store_rot && u1 > u0) store_rot(u1 - u0 - 1, prev_bh, prev_j, prev_n);
      if (pending_stores) bulk_wait_group0();
    }
  } else if (warp == 1) {
    // ─────────────── MMA issuer ───────────────
    if (lane == 0) {
      const uint32_t id_s1 = idesc_bf16(128, Wr, false, false);
      const uint32_t id_s2 = idesc_bf16(128, 128, false, false);
      const uint32_t id_o = idesc_bf16(128, kHD, false, true);
      const uint64_t dq0 = sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t dk0 = sdesc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t dv0 = sdesc_sw128(smem_u32(sV), 16, 1024);
      const uint64_t dp0 = sdesc_sw128(smem_u32(sP), 16, 1024);
      constexpr uint64_t kTileD = kTileBytes >> 4;  // descriptor units (16 B)
      const uint64_t halo = (uint64_t)((kTile - Wr) * 128) >> 4;
      int n = 0, prev = -1;
      bool ok = true;
      for (int u = u0, it = 0; u < u1 && ok; ++u, ++it) {
        const int j = u % nT;
        const int bi = p.nbuf == 2 ? (it & 1) : 0;
        if (it >= p.nbuf)
          ok = mbar_wait(&bar->tmem_empty[bi], ((it / p.nbuf) - 1) & 1, err, kErrFwd | 3);
        if (ok && j >= 1 && u == u0) {
          prev = n % kKVSlots;
          ok = mbar_wait(&bar->k_ready[prev], (n / kKVSlots) & 1, err, kErrFwd | 4);
          ++n;
        }
        const int cur = n % kKVSlots;
        ok = ok && mbar_wait(&bar->k_ready[cur], (n / kKVSlots) & 1, err, kErrFwd | 5);
        ++n;
        const int qs = it % kQSlots;
        ok = ok && mbar_wait(&bar->q_ready[qs], (it / kQSlots) & 1, err, kErrFwd | 6);
        if (!ok) break;
        tc_fence_after();
        const bool has_prev = j >= 1;
        const uint32_t s_col = tbase + bi * 256;
        const uint32_t o_col = s_col + p.ncols;
        const uint64_t dq = dq0 + qs * kTileD;
        if (has_prev) {
          const uint64_t dk = dk0 + prev * kTileD + halo;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16(s_col, dq + 2 * kk, dk + 2 * kk, id_s1, kk > 0);
        }
        {
          const uint64_t dk = dk0 + cur * kTileD;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16(s_col + Wr, dq + 2 * kk, dk + 2 * kk, id_s2, kk > 0);
        }
        mma_commit(&bar->s_full[bi]);
        mma_commit(&bar->q_empty[qs]);
        ok = mbar_wait(&bar->p_full, it & 1, err, kErrFwd | 7);
        if (!ok) break;
        tc_fence_after();
        uint32_t acc = 0;
        if (has_prev) {
          const uint64_t dv = dv0 + prev * kTileD + halo;
          for (int kk = 0; kk < Wr / 16; ++kk) {
            mma_bf16(o_col, dp0 + (kk >> 2) * kTileD + (kk & 3) * 2, dv + kk * 128, id_o, acc);
            acc = 1;
          }
        }
        {
          const uint64_t dv = dv0 + cur * kTileD;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int pk = Wr / 16 + kk;
            mma_bf16(o_col, dp0 + (pk >> 2) * kTileD + (pk & 3) * 2, dv + kk * 128, id_o, acc);
            acc = 1;
          }
        }
        mma_commit(&bar->o_full[bi]);
        if (has_prev) mma_commit(&bar->kv_empty[prev]);
        const bool next_is_succ = (u + 1 < u1) && ((u + 1) % nT != 0);
        if (next_is_succ) {
          prev = cur;
        } else {
          mma_commit(&bar->kv_empty[cur]);
          prev = -1;
        }
      }
    }
  } else if (warp < 4 || warp >= 12) {
    // ─────────────── RoPE rotators (4 warps) ───────────────
    const int tid = (warp < 4 ? warp - 2 : warp - 10) * 32 + lane;
    float th[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (p.theta)
#pragma unroll
      for (int z = 0; z < 8; ++z) th[z] = __ldg(p.theta + (tid & 3) * 8 + z);
    int n = 0;
    bool ok = true;
    for (int u = u0, it = 0; u < u1 && ok; ++u, ++it) {
      const int j = u % nT;
      const int qs = it % kQSlots;
      if (j >= 1 && u == u0) {  // halo key tile loaded only at the start of a range
        const int s = n % kKVSlots;
        ok = mbar_wait(&bar->kv_full[s], (n / kKVSlots) & 1, err, kErrFwd | 8);
        if (!ok) break;
        if (p.theta) rope_tiles(sK + s * kTileBytes, nullptr, (j - 1) * kTile, p.T, th, tid);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->k_ready[s]);
        ++n;
      }
      const int s = n % kKVSlots;
      ok = mbar_wait(&bar->q_full[qs], (it / kQSlots) & 1, err, kErrFwd | 9);
      ok = ok && mbar_wait(&bar->kv_full[s], (n / kKVSlots) & 1, err, kErrFwd | 8);
      if (!ok) break;
      if (p.theta) rope_tiles(sQ + qs * kTileBytes, sK + s * kTileBytes, j * kTile, p.T, th, tid);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar->q_ready[qs]);
        mbar_arrive(&bar->k_ready[s]);
      }
      ++n;
    }
  } else {
    // ─────────────── epilogue (8 warps) ───────────────
    const int e = warp - 4;
    const int qd = warp & 3;  // TMEM lane quadrant this warp may access
    const int hf = e >> 2;    // column half
    const int i = qd * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const int W = p.W;
    // 16-column chunks holding this quadrant's band: c ∈ [32qd+Wr−W, 32qd+31+Wr)
    const int ch_lo = max(0, qd * 32 + Wr - W) / 16;
    const int ch_hi = (qd * 32 + 30 + Wr) / 16;
    const int nch = ch_hi - ch_lo + 1;
    const int my_lo = hf == 0 ? ch_lo : ch_lo + (nch + 1) / 2;
    const int my_hi = hf == 0 ? ch_lo + (nch + 1) / 2 : ch_hi + 1;
    const uint32_t p_base = smem_u32(sP);
    const uint32_t o_base = smem_u32(sO);
    bool ok = true;
    for (int u = u0, it = 0; u < u1 && ok; ++u, ++it) {
      const int bh = u / nT, j = u % nT;
      const int b = bh / p.H, h = bh % p.H;
      const int bi = p.nbuf == 2 ? (it & 1) : 0;
      const uint32_t par = (it / p.nbuf) & 1;
      ok = mbar_wait(&bar->s_full[bi], par, err, kErrFwd | 10);
      if (!ok) break;
      __syncwarp();  // tcgen05.ld below is .sync.aligned
      tc_fence_after();
      const int t = j * kTile + i;
      const bool row_ok = t < p.T;
      // column c ↔ key s = jT − Wr + c ↔ window slot w = c − i − Wr + W
      const int w_of_c0 = W - Wr - i;
      const int c_min = Wr - j * kTile;  // s ≥ 0  ⇔  c ≥ c_min
      float mass = 0.f;
      const float* bias_row = nullptr;
      __nv_bfloat16* tau_row = nullptr;
      if constexpr (kBias) bias_row = p.bias + b * p.bs0 + (long long)min(t, p.T - 1) * p.bs1;
      if constexpr (kTau) tau_row = p.tau + ((long long)(b * p.T + min(t, p.T - 1)) * p.H + h) * W;

      auto process16 = [&](int ch, const uint32_t* r) {
        uint32_t pk[8];
#pragma unroll
        for (int e2 = 0; e2 < 16; e2 += 2) {
          float tv[2];
#pragma unroll
          for (int z = 0; z < 2; ++z) {
            const int c = ch * 16 + e2 + z;
            const int w = c + w_of_c0;
            const bool in_win = (unsigned)w < (unsigned)W;
            const bool valid = row_ok && in_win && c >= c_min;
            float x = __uint_as_float(r[e2 + z]) * p.half_inv_scale;
            if constexpr (kBias) {
              const float bv = __ldg(bias_row + (long long)(in_win ? w : 0) * p.bs2);
              x = fmaf(0.5f, bv, x);
            }
            const float tau = valid ? fmaf(0.5f, tanh_approx(x), 0.5f) : 0.f;
            mass += tau;
            tv[z] = tau;
            if constexpr (kTau) {
              if (row_ok && in_win) tau_row[w] = __float2bfloat16_rn(tau);
            }
          }
          pk[e2 >> 1] = pack_bf16(tv[0], tv[1]);
        }
        const int blk = (ch * 16) >> 6, c16 = ((ch * 16) & 63) >> 3;
        const uint32_t rowb = p_base + blk * kTileBytes;
        st_shared_v4(rowb + sw128_off(i, c16), pk[0], pk[1], pk[2], pk[3]);
        st_shared_v4(rowb + sw128_off(i, c16 + 1), pk[4], pk[5], pk[6], pk[7]);
      };

      const uint32_t s_addr = tbase + lane_off + bi * 256;
      for (int ch = my_lo; ch < my_hi; ch += 2) {
        uint32_t r[32];
        if (ch + 1 < my_hi) {
          tmem_ld32_wait(s_addr + ch * 16, r);
          process16(ch, r);
          process16(ch + 1, r + 16);
        } else {
          tmem_ld16_wait(s_addr + ch * 16, r);
          process16(ch, r);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->p_full);
      sMass[((it & 1) * 2 + hf) * kTile + i] = mass;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->mass_ready[it & 1]);
      ok = mbar_wait(&bar->mass_ready[it & 1], (it >> 1) & 1, err, kErrFwd | 12);
      ok = ok && mbar_wait(&bar->o_full[bi], par, err, kErrFwd | 11);
      if (!ok) break;
      __syncwarp();
      tc_fence_after();
      const float m = sMass[((it & 1) * 2 + 0) * kTile + i] + sMass[((it & 1) * 2 + 1) * kTile + i];
      float inv = 1.f;
      if (p.norm == BOZO_NORM_MASS) inv = 1.f / fmaxf(m, kMassEps);
      else if (p.norm == BOZO_NORM_COUNT) inv = 1.f / (float)max(min(t, W), 1);
      uint32_t o[32];
      tmem_ld32_wait(tbase + lane_off + bi * 256 + p.ncols + hf * 32, o);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->tmem_empty[bi]);
      // stage the bf16 tile for one TMA store (the previous store must have
      // finished reading the staging buffer)
      if (it > 0) ok = mbar_wait(&bar->ostage_empty, (it - 1) & 1, err, kErrFwd | 13);
      if (!ok) break;
#pragma unroll
      for (int z = 0; z < 4; ++z) {
        uint32_t w4[4];
#pragma unroll
        for (int y = 0; y < 4; ++y)
          w4[y] = pack_bf16(__uint_as_float(o[8 * z + 2 * y]) * inv, __uint_as_float(o[8 * z + 2 * y + 1]) * inv);
        st_shared_v4(o_base + sw128_off(i, hf * 4 + z), w4[0], w4[1], w4[2], w4[3]);
      }
      if (hf == 0 && row_ok && p.row_mass) p.row_mass[(long long)bh * p.T + t] = m;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->ostage_full);
      if (warp == 4 && lane == 0) {
        ok = mbar_wait(&bar->ostage_full, it & 1, err, kErrFwd | 14);
        if (ok) {
          tma_store_4d(&tmo, sO, 0, h, j * kTile, b);
          bulk_commit_group();
          bulk_wait_group_read0();
          mbar_arrive(&bar->ostage_empty);
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

template <bool kBias, bool kTau>
cudaError_t launch_variant(const CUtensorMap* m, const FwdTC& a, size_t smem, int grid,
                           cudaStream_t st) {
  auto kern = tc_fwd_kernel<kBias, kTau>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], a);
  return cudaGetLastError();
}

}  // namespace

bool tc_fwd_eligible(const FwdP& p) {
  if (p.mode != BOZO_MODE_LOCAL || p.HD != kHD || p.W < 1 || p.W > 128) return false;
  if (p.out_dt != BOZO_DT_BF16) return false;
  if (p.tau && p.tau_dt != BOZO_DT_BF16) return false;
  if (!tma_view_ok(p.q, p.B, p.T, p.H) || !tma_view_ok(p.k, p.B, p.T, p.H) ||
      !tma_view_ok(p.v, p.B, p.T, p.H))
    return false;
  if ((reinterpret_cast<uintptr_t>(p.out) & 15) != 0) return false;
  for (const void* r : {p.q_rot, p.k_rot})
    if (r && (reinterpret_cast<uintptr_t>(r) & 15) != 0) return false;
  if (p.cos && !p.theta) return false;  // on-the-fly RoPE needs θ
  return tmap_encoder_available();
}

cudaError_t launch_tc_fwd(const FwdP& p, cudaStream_t st, int* launches) {
  FwdTC a{};
  a.B = p.B; a.T = p.T; a.H = p.H; a.W = p.W;
  a.Wr = (p.W + 15) / 16 * 16;
  a.nT = (p.T + kTile - 1) / kTile;
  a.total = p.B * p.H * a.nT;
  a.norm = p.norm;
  a.ncols = a.Wr + kTile;
  a.nbuf = (a.ncols + kHD <= 256) ? 2 : 1;
  a.pblocks = (a.ncols + 63) / 64;
  a.half_inv_scale = 0.5f / p.scale;
  a.theta = p.cos ? p.theta : nullptr;
  a.bias = p.bias; a.bs0 = p.bs0; a.bs1 = p.bs1; a.bs2 = p.bs2;
  a.tau = static_cast<__nv_bfloat16*>(p.tau);
  a.row_mass = p.row_mass;
  a.store_rot = (a.theta && p.q_rot && p.k_rot) ? 1 : 0;
  a.err = p.err;
  CUtensorMap m[6];
  const long long ob = (long long)p.T * p.H * kHD, ot = (long long)p.H * kHD, oh = kHD;
  if (!make_tmap_bthd(&m[0], p.q.p, p.q.sb, p.q.st, p.q.sh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&m[1], p.k.p, p.k.sb, p.k.st, p.k.sh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&m[2], p.v.p, p.v.sb, p.v.st, p.v.sh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&m[3], p.out, ob, ot, oh, p.B, p.T, p.H, kTile))
    return cudaErrorInvalidValue;
  if (a.store_rot) {
    if (!make_tmap_bthd(&m[4], p.q_rot, ob, ot, oh, p.B, p.T, p.H, kTile) ||
        !make_tmap_bthd(&m[5], p.k_rot, ob, ot, oh, p.B, p.T, p.H, kTile))
      return cudaErrorInvalidValue;
  } else {
    m[4] = m[3];  // unused
    m[5] = m[3];
  }
  const Layout L = fwd_layout(a.pblocks);
  const size_t smem = L.total + 1024;
  const int grid = std::min(num_sms(), a.total);
  *launches = 1;
  const bool has_bias = p.bias != nullptr, has_tau = p.tau != nullptr;
  if (has_bias && has_tau) return launch_variant<true, true>(m, a, smem, grid, st);
  if (has_bias) return launch_variant<true, false>(m, a, smem, grid, st);
  if (has_tau) return launch_variant<false, true>(m, a, smem, grid, st);
  return launch_variant<false, false>(m, a, smem, grid, st);
}

}  // namespace bozo
