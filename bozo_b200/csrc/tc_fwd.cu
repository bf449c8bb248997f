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
constexpr int kQSlots = 2;
constexpr int kKVSlots = 3;  // barrier array size; p.nkv ≤ this slots are used
constexpr int kThreads = 14 * 32;
constexpr int kRotThreads = 128;
constexpr int kErrFwd = 0x100;  // device error codes (| site)
constexpr size_t kMaxSmemPerBlock = 227 * 1024;  // sm_100 opt-in limit

struct FwdTC {
  int B, T, H, W, Wr, nT, total;
  int norm, nbuf, ncols, pblocks;
  int nkv;      // K/V ring slots (3, or 2 when the τ staging rows need the room)
  int tstride;  // bytes per row of the τ staging buffer (0: no τ export)
  float half_inv_scale;
  const float* theta;  // RoPE frequencies [32] or null (no RoPE)
  const float* bias;
  long long bs0, bs1, bs2;
  void* tau;      // bf16, or fp32 in the fp32-output variant
  float* out_f32;  // fp32-output variant: out [B,T,H,64] fp32, stored from registers
  float* row_mass;
  int store_rot;  // also TMA-store the rotated Q/K tiles (q_rot, k_rot)
  int* err;
};

struct __align__(8) Bars {
  uint64_t q_full[kQSlots], q_ready[kQSlots], q_empty[kQSlots];
  // K and V have separate ring barriers: a K slot is free after its last
  // QKᵀ, a V slot only after its last P·V
  uint64_t k_full[kKVSlots], k_ready[kKVSlots], k_empty[kKVSlots];
  uint64_t v_full[kKVSlots], v_empty[kKVSlots];
  uint64_t s_full[2], o_full[2], tmem_empty[2];
  uint64_t p_full;
  uint64_t mass_ready[2];  // the 8 epilogue warps have published their τ-mass halves
  uint64_t ostage_full, ostage_empty;
  uint64_t tau_free;  // every epilogue warp has copied its τ rows out
  uint32_t tmem_base;
};

struct Layout {
  uint32_t q, k, v, p, o, mass, tau, bars, total;
};

// f32_out: the fp32-output variant stores O from registers and needs no
// bf16 staging tile.
__host__ __device__ inline Layout fwd_layout(int pblocks, int nkv, int tstride, bool f32_out = false) {
  Layout L;
  L.q = 0;
  L.k = L.q + kQSlots * kTileBytes;
  L.v = L.k + nkv * kTileBytes;
  L.p = L.v + nkv * kTileBytes;
  L.o = L.p + pblocks * kTileBytes;
  L.mass = L.o + (f32_out ? 0 : kTileBytes);  // float[2][2][128]
  L.tau = L.mass + 2 * 2 * kTile * 4;  // τ rows [128][tstride bytes]
  L.bars = L.tau + kTile * tstride;
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
__device__ __noinline__ void rope_tiles(uint8_t* ta, uint8_t* tb, int t0, int T, const float (&th)[8],
                                       int tid) {
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

// kF32: out and the exported τ in fp32 (the reference's dtype contract when
// Q is fp32, ops.py:122-124), from bf16 operand copies of Q and K.
template <bool kBias, bool kTau, int kNKV, bool kF32>
__global__ void __launch_bounds__(kThreads, 1)
    tc_fwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmo,
                  const __grid_constant__ CUtensorMap tmqr, const __grid_constant__ CUtensorMap tmkr,
                  const FwdTC p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = fwd_layout(p.pblocks, p.nkv, p.tstride, kF32);
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
    for (int i = 0; i < kNKV; ++i) {
      mbar_init(&bar->k_full[i], 1);
      mbar_init(&bar->k_ready[i], 4);
      mbar_init(&bar->k_empty[i], 1);
      mbar_init(&bar->v_full[i], 1);
      mbar_init(&bar->v_empty[i], 1);
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
    mbar_init(&bar->tau_free, 8);
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
  constexpr int NKV = kNKV;  // K/V ring slots (compile time: cheap slot/phase math)

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
        const int s = n % NKV;
        const int b = bh / p.H, h = bh % p.H;
        if (n >= NKV)
          ok = ok && mbar_wait(&bar->k_empty[s], ((n / NKV) - 1) & 1, err, kErrFwd | 1);
        if (!ok) return;
        before_refill();
        mbar_arrive_expect_tx(&bar->k_full[s], kTileBytes);
        tma_load_4d(sK + s * kTileBytes, &tmk, &bar->k_full[s], 0, h, jj * kTile, b);
        if (n >= NKV)
          ok = ok && mbar_wait(&bar->v_empty[s], ((n / NKV) - 1) & 1, err, kErrFwd | 17);
        if (!ok) return;
        mbar_arrive_expect_tx(&bar->v_full[s], kTileBytes);
        tma_load_4d(sV + s * kTileBytes, &tmv, &bar->v_full[s], 0, h, jj * kTile, b);
        ++n;
      };
      // store RoPE(Q), RoPE(K) of tile (bh, j) once the rotators are done
      auto store_rot = [&](int it_s, int bh, int j, int nk) {
        const int qs = it_s % kQSlots, ks = nk % NKV;
        ok = ok && mbar_wait(&bar->q_ready[qs], (it_s / kQSlots) & 1, err, kErrFwd | 15);
        ok = ok && mbar_wait(&bar->k_ready[ks], (nk / NKV) & 1, err, kErrFwd | 16);
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
    // The order note: P·V of tile it is issued as soon as its P is complete,
    // the QKᵀ of tile it+1 right after it.  QKᵀ(it+1) waits for the RoPE
    // warps to rotate tile it+1; issued first, it held P·V(it) back behind
    // them (forward 51.4 → 47 µs at B8 H12 T2048 W64 when reordered).  With
    // two TMEM buffers (nbuf 2) QKᵀ(it+1) lands in the other buffer while the
    // epilogue reads O(it), so S(it+1) is ready when the epilogue is done
    // with tile it.  The single shared P tile stays safe: the epilogue writes
    // P(it+1) only after it has waited for P·V(it) (o_full) to normalise O(it).
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
      struct Rec {
        int it, bi, qs, prev, cur, prev_idx, cur_idx;
        bool has_prev, next_is_succ;
      };
      int n = 0, carry = -1, carry_idx = 0;  // K/V load index; halo slot carried over
      bool ok = true;
      // slots of tile u (in load order) and its waits before QKᵀ
      auto make = [&](int u, int it) {
        Rec r;
        const int j = u % nT;
        r.it = it;
        r.bi = p.nbuf == 2 ? (it & 1) : 0;
        r.qs = it % kQSlots;
        r.has_prev = j >= 1;
        r.prev = carry;
        r.prev_idx = carry_idx;
        if (r.has_prev && u == u0) {  // halo tile loaded only at the start of a range
          r.prev = n % NKV;
          r.prev_idx = n;
          ++n;
        }
        r.cur = n % NKV;
        r.cur_idx = n;
        ++n;
        r.next_is_succ = (u + 1 < u1) && ((u + 1) % nT != 0);
        carry = r.next_is_succ ? r.cur : -1;
        carry_idx = r.cur_idx;
        return r;
      };
      auto issue_s = [&](const Rec& r) {
        if (r.it >= p.nbuf)
          ok = ok && mbar_wait(&bar->tmem_empty[r.bi], ((r.it / p.nbuf) - 1) & 1, err, kErrFwd | 3);
        if (r.has_prev)
          ok = ok && mbar_wait(&bar->k_ready[r.prev], (r.prev_idx / NKV) & 1, err, kErrFwd | 4);
        ok = ok && mbar_wait(&bar->k_ready[r.cur], (r.cur_idx / NKV) & 1, err, kErrFwd | 5);
        ok = ok && mbar_wait(&bar->q_ready[r.qs], (r.it / kQSlots) & 1, err, kErrFwd | 6);
        if (!ok) return;
        tc_fence_after();
        const uint32_t s_col = tbase + r.bi * 256;
        const uint64_t dq = dq0 + r.qs * kTileD;
        if (r.has_prev) {
          const uint64_t dk = dk0 + r.prev * kTileD + halo;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16(s_col, dq + 2 * kk, dk + 2 * kk, id_s1, kk > 0);
        }
        {
          const uint64_t dk = dk0 + r.cur * kTileD;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16(s_col + Wr, dq + 2 * kk, dk + 2 * kk, id_s2, kk > 0);
        }
        mma_commit(&bar->s_full[r.bi]);
        mma_commit(&bar->q_empty[r.qs]);
        // K of the halo tile is done; the current tile's K still serves as
        // the next tile's halo unless that tile starts a new sequence
        if (r.has_prev) mma_commit(&bar->k_empty[r.prev]);
        if (!r.next_is_succ) mma_commit(&bar->k_empty[r.cur]);
      };
      auto issue_o = [&](const Rec& r) {
        // V first (loaded long before, so these waits overlap the epilogue)
        if (r.has_prev)
          ok = ok && mbar_wait(&bar->v_full[r.prev], (r.prev_idx / NKV) & 1, err, kErrFwd | 18);
        ok = ok && mbar_wait(&bar->v_full[r.cur], (r.cur_idx / NKV) & 1, err, kErrFwd | 19);
        ok = ok && mbar_wait(&bar->p_full, r.it & 1, err, kErrFwd | 7);
        if (!ok) return;
        tc_fence_after();
        const uint32_t o_col = tbase + r.bi * 256 + p.ncols;
        uint32_t acc = 0;
        if (r.has_prev) {
          const uint64_t dv = dv0 + r.prev * kTileD + halo;
          for (int kk = 0; kk < Wr / 16; ++kk) {
            mma_bf16(o_col, dp0 + (kk >> 2) * kTileD + (kk & 3) * 2, dv + kk * 128, id_o, acc);
            acc = 1;
          }
        }
        {
          const uint64_t dv = dv0 + r.cur * kTileD;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int pk = Wr / 16 + kk;
            mma_bf16(o_col, dp0 + (pk >> 2) * kTileD + (pk & 3) * 2, dv + kk * 128, id_o, acc);
            acc = 1;
          }
        }
        mma_commit(&bar->o_full[r.bi]);
        if (r.has_prev) mma_commit(&bar->v_empty[r.prev]);
        if (!r.next_is_succ) mma_commit(&bar->v_empty[r.cur]);
      };
      // The output tile of tile it, staged by the epilogue, is stored from
      // here (this thread would otherwise idle until the next P is ready):
      // issued before the next P·V, the staging buffer handed back after it,
      // by when the store has long finished reading it.
      auto store_o = [&](int u, int it) {
        if constexpr (kF32) return;  // the epilogue stored O itself
        ok = ok && mbar_wait(&bar->ostage_full, it & 1, err, kErrFwd | 14);
        if (!ok) return;
        const int bh = u / nT, j = u % nT;
        tma_store_4d(&tmo, sO, 0, bh % p.H, j * kTile, bh / p.H);
        bulk_commit_group();
      };
      auto release_o = [&]() {
        if constexpr (kF32) return;
        bulk_wait_group_read0();
        mbar_arrive(&bar->ostage_empty);
      };
      if (u0 < u1) {
        Rec cur = make(u0, 0);
        issue_s(cur);
        for (int u = u0, it = 0; u < u1 && ok; ++u, ++it) {
          Rec nxt{};
          const bool more = u + 1 < u1;
          if (more) nxt = make(u + 1, it + 1);
          if (it >= 1) store_o(u - 1, it - 1);     // staged while P(it) was formed
          issue_o(cur);
          if (it >= 1 && ok) release_o();
          if (more) issue_s(nxt);  // after P·V(it): see the order note above
          cur = nxt;
        }
        if (ok) store_o(u1 - 1, u1 - u0 - 1);
        bulk_wait_group0();
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
        const int s = n % NKV;
        ok = mbar_wait(&bar->k_full[s], (n / NKV) & 1, err, kErrFwd | 8);
        if (!ok) break;
        if (p.theta) rope_tiles(sK + s * kTileBytes, nullptr, (j - 1) * kTile, p.T, th, tid);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->k_ready[s]);
        ++n;
      }
      const int s = n % NKV;
      ok = mbar_wait(&bar->q_full[qs], (it / kQSlots) & 1, err, kErrFwd | 9);
      ok = ok && mbar_wait(&bar->k_full[s], (n / NKV) & 1, err, kErrFwd | 8);
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
    // τ staging rows (exported τ): row i holds τ[t, 0..W) in the output dtype
    using TauT = typename std::conditional<kF32, float, __nv_bfloat16>::type;
    TauT* const tau_s = reinterpret_cast<TauT*>(smem + L.tau);
    const int tau_pitch = p.tstride / (int)sizeof(TauT);  // elements per staging row
    bool ok = true;
    for (int u = u0, it = 0; u < u1 && ok; ++u, ++it) {
      const int bh = u / nT, j = u % nT;
      const int b = bh / p.H, h = bh % p.H;
      const int bi = p.nbuf == 2 ? (it & 1) : 0;
      const uint32_t par = (it / p.nbuf) & 1;
      ok = mbar_wait(&bar->s_full[bi], par, err, kErrFwd | 10);
      // the τ rows of the previous tile must have been copied out
      if constexpr (kTau) {
        if (ok && it >= 1) ok = mbar_wait(&bar->tau_free, (it - 1) & 1, err, kErrFwd | 20);
      }
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
      if constexpr (kBias) bias_row = p.bias + b * p.bs0 + (long long)min(t, p.T - 1) * p.bs1;
      TauT* const tau_row = tau_s + i * tau_pitch;

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
              if (in_win) {
                if constexpr (kF32) tau_row[w] = tau;
                else tau_row[w] = __float2bfloat16_rn(tau);
              }
            }
          }
          pk[e2 >> 1] = pack_bf16(tv[0], tv[1]);
        }
        const int blk = (ch * 16) >> 6, c16 = ((ch * 16) & 63) >> 3;
        const uint32_t rowb = p_base + blk * kTileBytes;
        st_shared_v4(rowb + sw128_off(i, c16), pk[0], pk[1], pk[2], pk[3]);
        st_shared_v4(rowb + sw128_off(i, c16 + 1), pk[4], pk[5], pk[6], pk[7]);
      };

      // one 16-column chunk per TMEM read: a single inlined copy of the
      // element code (instruction-cache footprint)
      const uint32_t s_addr = tbase + lane_off + bi * 256;
      for (int ch = my_lo; ch < my_hi; ++ch) {
        uint32_t r[16];
        tmem_ld16_wait(s_addr + ch * 16, r);
        process16(ch, r);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->p_full);
      sMass[((it & 1) * 2 + hf) * kTile + i] = mass;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->mass_ready[it & 1]);
      ok = mbar_wait(&bar->mass_ready[it & 1], (it >> 1) & 1, err, kErrFwd | 12);
      if constexpr (kTau) {
        // every warp is past its τ writes: copy 16 whole rows out, each row
        // contiguous in [B,T,H,W] (16-byte stores when a row is a multiple of
        // 16 bytes)
        if (ok) {
          const int r0 = e * 16;
          TauT* const gbase = static_cast<TauT*>(p.tau) + ((long long)b * p.T * p.H + h) * W;
          const long long gpitch = (long long)p.H * W;  // elements between rows t, t+1
          constexpr int kPer16 = 16 / (int)sizeof(TauT);  // elements per 16-byte chunk
          if ((W % kPer16) == 0) {
            const int vpr = W / kPer16;
            for (int idx = lane; idx < 16 * vpr; idx += 32) {
              const int rr = r0 + idx / vpr, cc = idx - (idx / vpr) * vpr;
              const int tt = j * kTile + rr;
              if (tt < p.T) {
                uint32_t a0, a1, a2, a3;
                ld_shared_v4(smem_u32(tau_s + rr * tau_pitch) + cc * 16, a0, a1, a2, a3);
                *reinterpret_cast<uint4*>(gbase + tt * gpitch + cc * kPer16) = make_uint4(a0, a1, a2, a3);
              }
            }
          } else {
            for (int idx = lane; idx < 16 * W; idx += 32) {
              const int rr = r0 + idx / W, cc = idx - (idx / W) * W;
              const int tt = j * kTile + rr;
              if (tt < p.T) gbase[tt * gpitch + cc] = tau_s[rr * tau_pitch + cc];
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar->tau_free);
        }
      }
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
      if (hf == 0 && row_ok && p.row_mass) p.row_mass[(long long)bh * p.T + t] = m;
      if constexpr (kF32) {
        // this thread's 32 fp32 values of row t, straight from registers (the
        // row's other half comes from the warp of the other column half)
        if (row_ok) {
          float4* dst = reinterpret_cast<float4*>(p.out_f32 + ((long long)(b * p.T + t) * p.H + h) * kHD +
                                                  hf * 32);
#pragma unroll
          for (int z = 0; z < 8; ++z)
            dst[z] = make_float4(__uint_as_float(o[4 * z]) * inv, __uint_as_float(o[4 * z + 1]) * inv,
                                 __uint_as_float(o[4 * z + 2]) * inv, __uint_as_float(o[4 * z + 3]) * inv);
        }
      } else {
        // stage the bf16 tile for one TMA store (issued by the MMA thread); the
        // previous store must have finished reading the staging buffer
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
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->ostage_full);
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

template <bool kBias, bool kTau, int kNKV, bool kF32>
cudaError_t launch_variant(const CUtensorMap* m, const FwdTC& a, size_t smem, int grid,
                           cudaStream_t st) {
  auto kern = tc_fwd_kernel<kBias, kTau, kNKV, kF32>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], a);
  return cudaGetLastError();
}

template <bool kF32>
cudaError_t launch_dtype(const CUtensorMap* m, const FwdTC& a, size_t smem, int grid, bool has_bias,
                         bool has_tau, cudaStream_t st) {
  const bool two = a.nkv == 2;  // only τ export narrows the ring
  if (has_bias && has_tau)
    return two ? launch_variant<true, true, 2, kF32>(m, a, smem, grid, st)
               : launch_variant<true, true, 3, kF32>(m, a, smem, grid, st);
  if (has_tau)
    return two ? launch_variant<false, true, 2, kF32>(m, a, smem, grid, st)
               : launch_variant<false, true, 3, kF32>(m, a, smem, grid, st);
  if (has_bias) return launch_variant<true, false, 3, kF32>(m, a, smem, grid, st);
  return launch_variant<false, false, 3, kF32>(m, a, smem, grid, st);
}

// Shared-memory plan of a call: τ staging pitch, K/V ring slots, total bytes.
struct FwdPlan {
  int Wr, ncols, pblocks, tstride, nkv;
  bool f32;
  size_t smem;
};

FwdPlan fwd_plan(const FwdP& p) {
  FwdPlan q{};
  q.f32 = p.out_dt == BOZO_DT_F32;
  q.Wr = (p.W + 15) / 16 * 16;
  q.ncols = q.Wr + kTile;
  q.pblocks = (q.ncols + 63) / 64;
  // τ export stages whole rows in shared memory (+16 bytes per row keeps the
  // rows' writes off one bank); the K/V ring drops to two slots when three
  // would not leave room for them
  q.tstride = p.tau ? p.W * (q.f32 ? 4 : 2) + 16 : 0;
  q.nkv = 3;
  if (fwd_layout(q.pblocks, 3, q.tstride, q.f32).total + 1024 > kMaxSmemPerBlock) q.nkv = 2;
  q.smem = fwd_layout(q.pblocks, q.nkv, q.tstride, q.f32).total + 1024;
  return q;
}

}  // namespace

bool tc_fwd_eligible(const FwdP& p) {
  if (p.mode != BOZO_MODE_LOCAL || p.HD != kHD || p.W < 1 || p.W > 128) return false;
  if (p.out_dt == BOZO_DT_F32) {
    // fp32 out and τ (the reference's dtypes for fp32 Q), from bf16 operand
    // copies of Q/K; no RoPE in this variant
    if (p.tau && p.tau_dt != BOZO_DT_F32) return false;
    if (p.cos || !p.out || (reinterpret_cast<uintptr_t>(p.out) & 15) != 0) return false;
  } else {
    if (p.out_dt != BOZO_DT_BF16) return false;
    if (p.tau && p.tau_dt != BOZO_DT_BF16) return false;
  }
  if (p.tau && (reinterpret_cast<uintptr_t>(p.tau) & 15) != 0) return false;
  if (!tma_view_ok(p.q, p.B, p.T, p.H) || !tma_view_ok(p.k, p.B, p.T, p.H) ||
      !tma_view_ok(p.v, p.B, p.T, p.H))
    return false;
  if ((reinterpret_cast<uintptr_t>(p.out) & 15) != 0) return false;
  for (const void* r : {p.q_rot, p.k_rot})
    if (r && (reinterpret_cast<uintptr_t>(r) & 15) != 0) return false;
  if (p.cos && !p.theta) return false;  // on-the-fly RoPE needs θ
  if (fwd_plan(p).smem > kMaxSmemPerBlock) return false;
  return tmap_encoder_available();
}

cudaError_t launch_tc_fwd(const FwdP& p, cudaStream_t st, int* launches) {
  const FwdPlan plan = fwd_plan(p);
  FwdTC a{};
  a.B = p.B; a.T = p.T; a.H = p.H; a.W = p.W;
  a.Wr = plan.Wr;
  a.nT = (p.T + kTile - 1) / kTile;
  a.total = p.B * p.H * a.nT;
  a.norm = p.norm;
  a.ncols = plan.ncols;
  a.nbuf = (a.ncols + kHD <= 256) ? 2 : 1;
  a.pblocks = plan.pblocks;
  a.half_inv_scale = 0.5f / p.scale;
  a.theta = p.cos ? p.theta : nullptr;
  a.bias = p.bias; a.bs0 = p.bs0; a.bs1 = p.bs1; a.bs2 = p.bs2;
  a.tau = p.tau;
  a.out_f32 = plan.f32 ? static_cast<float*>(p.out) : nullptr;
  a.row_mass = p.row_mass;
  a.store_rot = (a.theta && p.q_rot && p.k_rot) ? 1 : 0;
  a.err = p.err;
  a.tstride = plan.tstride;
  a.nkv = plan.nkv;
  CUtensorMap m[6];
  const long long ob = (long long)p.T * p.H * kHD, ot = (long long)p.H * kHD, oh = kHD;
  if (!make_tmap_bthd(&m[0], p.q.p, p.q.sb, p.q.st, p.q.sh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&m[1], p.k.p, p.k.sb, p.k.st, p.k.sh, p.B, p.T, p.H, kTile) ||
      !make_tmap_bthd(&m[2], p.v.p, p.v.sb, p.v.st, p.v.sh, p.B, p.T, p.H, kTile))
    return cudaErrorInvalidValue;
  if (plan.f32) {
    m[3] = m[0];  // unused: the fp32 output leaves from registers
  } else if (!make_tmap_bthd(&m[3], p.out, ob, ot, oh, p.B, p.T, p.H, kTile)) {
    return cudaErrorInvalidValue;
  }
  if (a.store_rot) {
    if (!make_tmap_bthd(&m[4], p.q_rot, ob, ot, oh, p.B, p.T, p.H, kTile) ||
        !make_tmap_bthd(&m[5], p.k_rot, ob, ot, oh, p.B, p.T, p.H, kTile))
      return cudaErrorInvalidValue;
  } else {
    m[4] = m[3];  // unused
    m[5] = m[3];
  }
  if (plan.smem > kMaxSmemPerBlock) return cudaErrorInvalidConfiguration;
  const int grid = std::min(num_sms(), a.total);
  *launches = 1;
  const bool has_bias = p.bias != nullptr, has_tau = p.tau != nullptr;
  return plan.f32 ? launch_dtype<true>(m, a, plan.smem, grid, has_bias, has_tau, st)
                  : launch_dtype<false>(m, a, plan.smem, grid, has_bias, has_tau, st);
}

}  // namespace bozo
