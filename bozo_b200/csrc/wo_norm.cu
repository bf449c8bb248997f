// wo_norm.cu — a TensionLM block's output projection fused with the residual
// add and RMSNorm that follow it, forward only (prefill, decode and
// evaluation run without gradients):
//
//     out = RMSNorm(x + msg·Woᵀ)·scale        (model.py:259 / 283, RMSNorm
//                                              model.py:86-98)
//
// so the projection's [rows, width] result never makes a round trip through
// HBM between the GEMM and the norm.
//
// A cluster of CN CTAs owns 128 rows; CTA c computes the Nc = width / CN
// columns [c·Nc, (c+1)·Nc) of y = msg·Woᵀ on the tensor cores (tcgen05,
// M = 128, N = Nc, bf16 operands, fp32 accumulator in TMEM), its operands
// TMA-loaded 64 K-columns at a time through a ring of 2-4 stages.  The CTA's
// [128, Nc] tile of x is TMA-loaded into shared memory at the start, so it
// arrives while the MMAs run.  Epilogue (all eight warps; warp w reads TMEM
// lanes 32·(w mod 4).. and half w / 4 of the columns, one row per thread):
//   pass 1  s = x + bf16(y) (rounded to x's dtype when that is bf16, as the
//           unfused add is), written over x in shared memory; Σ s² over the
//           thread's columns goes to every CTA of the cluster through
//           distributed shared memory;
//   pass 2  after one cluster barrier each row's sum is complete:
//           out = s·rstd·scale, written over s, and the tile leaves by TMA.
// Shared-memory tiles use the 128-byte swizzle (rows of 128 bytes, 16-byte
// chunks XOR row mod 8), so one row per thread reads and writes 16-byte
// chunks without bank conflicts.  No TMA multicast: every CTA loads its own
// tiles.
#include <algorithm>

#include "tc.cuh"
#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace bozo {
namespace {

using namespace tc;

constexpr int kRows = 128;        // rows per cluster
constexpr int kK = 64;            // K columns per stage (one 128-byte swizzle row)
constexpr int kMaxStages = 4;
constexpr int kThreads = 8 * 32;
constexpr int kMaxCluster = 8;
constexpr int kBox = kRows * 128;  // one swizzled [128 rows × 128 bytes] box
constexpr uint32_t kSmemLimit = 232448;  // 227 KB per CTA
constexpr int kErrWo = 0x500;

struct WoP {
  long long M;
  int D, Nc, CN, KT, stages;
  float eps;
  const void* scale;  // [D], x's dtype
  float* rstd;        // [M] or null
  int* err;
};

struct __align__(8) WoBars {
  uint64_t full[kMaxStages], empty[kMaxStages], acc_full, x_full;
  uint32_t tmem_base;
};

inline uint32_t stage_bytes(int Nc) { return (uint32_t)(kRows + Nc) * kK * 2; }
inline uint32_t tile_bytes(int Nc, int esz) { return (uint32_t)kRows * Nc * esz; }
inline uint32_t fixed_bytes() { return 2 * kMaxCluster * kRows * 4 + sizeof(WoBars) + 1024; }
inline int stages_for(int Nc, int esz) {
  const long long room = (long long)kSmemLimit - fixed_bytes() - tile_bytes(Nc, esz);
  return room <= 0 ? 0 : (int)std::min<long long>(kMaxStages, room / stage_bytes(Nc));
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of `local` (this CTA's shared memory) in CTA `rank`
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float lo_bf16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Shared-memory address of the 16-byte chunk holding columns [c, c + 16/esz)
// of row r of the staged tile (boxes of 128 bytes per row, swizzled).
template <bool kBf16>
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int r, int c) {
  constexpr int cpb = kBf16 ? 64 : 32;  // columns per box
  constexpr int cpc = kBf16 ? 8 : 4;    // columns per 16-byte chunk
  return base + (uint32_t)(c / cpb) * kBox + sw128_off(r, (c % cpb) / cpc);
}

// 16 columns of the staged tile (row r, from column c) to fp32 and back.
template <bool kBf16>
__device__ __forceinline__ void tile_ld16(uint32_t base, int r, int c, float* v) {
  if constexpr (kBf16) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t w[4];
      ld_shared_v4(tile_addr<true>(base, r, c + 8 * h), w[0], w[1], w[2], w[3]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[8 * h + 2 * e] = lo_bf16(w[e]);
        v[8 * h + 2 * e + 1] = hi_bf16(w[e]);
      }
    }
  } else {
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      uint32_t w[4];
      ld_shared_v4(tile_addr<false>(base, r, c + 4 * h), w[0], w[1], w[2], w[3]);
#pragma unroll
      for (int e = 0; e < 4; ++e) v[4 * h + e] = __uint_as_float(w[e]);
    }
  }
}
template <bool kBf16>
__device__ __forceinline__ void tile_st16(uint32_t base, int r, int c, const float* v) {
  if constexpr (kBf16) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
      st_shared_v4(tile_addr<true>(base, r, c + 8 * h), pack_bf16(v[8 * h], v[8 * h + 1]),
                   pack_bf16(v[8 * h + 2], v[8 * h + 3]), pack_bf16(v[8 * h + 4], v[8 * h + 5]),
                   pack_bf16(v[8 * h + 6], v[8 * h + 7]));
  } else {
#pragma unroll
    for (int h = 0; h < 4; ++h)
      st_shared_v4(tile_addr<false>(base, r, c + 4 * h), __float_as_uint(v[4 * h]),
                   __float_as_uint(v[4 * h + 1]), __float_as_uint(v[4 * h + 2]),
                   __float_as_uint(v[4 * h + 3]));
  }
}

template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    wo_norm_kernel(const __grid_constant__ CUtensorMap tm_msg, const __grid_constant__ CUtensorMap tm_wo,
                   const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_out,
                   const WoP p) {
  constexpr int esz = kBf16 ? 2 : 4;
  constexpr int cpb = 128 / esz;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbytes = (uint32_t)(kRows + p.Nc) * kK * 2;
  uint8_t* sX = smem + p.stages * sbytes;                              // [128, Nc] tile, x's dtype
  float* sPart = reinterpret_cast<float*>(sX + kRows * p.Nc * esz);    // [2·CN][128] row partial sums
  WoBars* bar = reinterpret_cast<WoBars*>(sPart + 2 * kMaxCluster * kRows);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const long long m0 = (long long)blockIdx.y * kRows;
  const int n0 = (int)rank * p.Nc;
  const int nbox = p.Nc / cpb;
  const uint32_t tcols = p.Nc <= 32 ? 32 : p.Nc <= 64 ? 64 : p.Nc <= 128 ? 128 : 256;
  int* err = p.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&bar->full[s], 1);
      mbar_init(&bar->empty[s], 1);
    }
    mbar_init(&bar->acc_full, 1);
    mbar_init(&bar->x_full, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&bar->tmem_base, tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bar->tmem_base;
  // Arrive now, wait before the first store into another CTA's shared memory:
  // that store must not land before its target CTA has started.
  cluster_arrive_relaxed();

  if (warp == 0 && lane == 0) {  // ─── TMA producer ───
    prefetch_tmap(&tm_msg);
    prefetch_tmap(&tm_wo);
    mbar_arrive_expect_tx(&bar->x_full, (uint32_t)kRows * p.Nc * esz);
    for (int j = 0; j < nbox; ++j) tma_load_2d(sX + j * kBox, &tm_x, &bar->x_full, n0 + j * cpb, (int)m0);
    bool ok = true;
    for (int k = 0; k < p.KT && ok; ++k) {
      const int s = k % p.stages;
      if (k >= p.stages) ok = mbar_wait(&bar->empty[s], ((k / p.stages) - 1) & 1, err, kErrWo | 1);
      if (!ok) break;
      uint8_t* st = smem + s * sbytes;
      mbar_arrive_expect_tx(&bar->full[s], sbytes);
      tma_load_2d(st, &tm_msg, &bar->full[s], k * kK, (int)m0);
      tma_load_2d(st + kRows * kK * 2, &tm_wo, &bar->full[s], k * kK, n0);
    }
  } else if (warp == 1 && lane == 0) {  // ─── MMA issuer ───
    const uint32_t idesc = idesc_bf16(kRows, p.Nc, false, false);  // A, B K-major
    bool ok = true;
    for (int k = 0; k < p.KT && ok; ++k) {
      const int s = k % p.stages;
      ok = mbar_wait(&bar->full[s], (k / p.stages) & 1, err, kErrWo | 2);
      if (!ok) break;
      tc_fence_after();
      const uint32_t st = smem_u32(smem + s * sbytes);
      const uint64_t da = sdesc_sw128(st, 16, 1024), db = sdesc_sw128(st + kRows * kK * 2, 16, 1024);
#pragma unroll
      for (int kk = 0; kk < kK / 16; ++kk)
        mma_bf16(tbase, da + 2 * kk, db + 2 * kk, idesc, (k > 0 || kk > 0) ? 1u : 0u);
      mma_commit(&bar->empty[s]);
    }
    if (ok) mma_commit(&bar->acc_full);
  }
  __syncwarp();

  // ─── epilogue: every warp ───
  const int q = warp & 3, h = warp >> 2;
  const int r = q * 32 + lane;
  const long long m = m0 + r;
  const uint32_t lane_off = (uint32_t)(q * 32) << 16;
  const int c_lo = h * (p.Nc / 2), c_hi = c_lo + p.Nc / 2;
  const uint32_t xs = smem_u32(sX);
  bool ok = mbar_wait(&bar->acc_full, 0u, err, kErrWo | 3);
  ok = ok && mbar_wait(&bar->x_full, 0u, err, kErrWo | 4);
  ok = __all_sync(~0u, ok);  // TMEM loads are warp-collective
  tc_fence_after();
  // pass 1: s = x + bf16(y) over this thread's columns, Σ s²
  float ss = 0.f;
  if (ok) {
    for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
      uint32_t a[16];
      tmem_ld16_wait(tbase + lane_off + c0, a);
      float v[16];
      tile_ld16<kBf16>(xs, r, c0, v);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        float s = v[e] + round_bf16(__uint_as_float(a[e]));
        if (kBf16) s = round_bf16(s);
        v[e] = s;
        ss = fmaf(s, s, ss);
      }
      tile_st16<kBf16>(xs, r, c0, v);
    }
  }
  // this thread's partial to slot [2·rank + h][r] of every CTA in the cluster
  cluster_wait();
  const uint32_t local = smem_u32(sPart + (2 * rank + h) * kRows + r);
  for (int j = 0; j < p.CN; ++j) st_cluster_f32(map_to_rank(local, (uint32_t)j), ss);
  cluster_sync_all();

  // pass 2: out = s·rstd·scale
  float tot = 0.f;
  for (int j = 0; j < 2 * p.CN; ++j) tot += sPart[j * kRows + r];
  const float rstd = rsqrtf(tot / (float)p.D + p.eps);
  if (ok && h == 0 && rank == 0 && p.rstd && m < p.M) p.rstd[m] = rstd;
  if (ok) {
    for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
      float v[16];
      tile_ld16<kBf16>(xs, r, c0, v);
#pragma unroll
      for (int g = 0; g < 16; g += 8) {
        float sc[8];
        if (kBf16) {
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.scale) +
                                                               n0 + c0 + g));
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            sc[2 * e] = lo_bf16(w[e]);
            sc[2 * e + 1] = hi_bf16(w[e]);
          }
        } else {
          const float4* f = reinterpret_cast<const float4*>(static_cast<const float*>(p.scale) + n0 + c0 + g);
          const float4 f0 = __ldg(f), f1 = __ldg(f + 1);
          sc[0] = f0.x; sc[1] = f0.y; sc[2] = f0.z; sc[3] = f0.w;
          sc[4] = f1.x; sc[5] = f1.y; sc[6] = f1.z; sc[7] = f1.w;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) v[g + e] = v[g + e] * rstd * sc[e];
      }
      tile_st16<kBf16>(xs, r, c0, v);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  const int bad = __syncthreads_or(!ok);
  if (threadIdx.x == 0 && !bad) {
    for (int j = 0; j < nbox; ++j) tma_store_2d(&tm_out, sX + j * kBox, n0 + j * cpb, (int)m0);
    bulk_commit_group();
    bulk_wait_group_read0();
  }
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, tcols);
  }
}

}  // namespace

// Cluster size for a width and x dtype: the fewest CTAs (≤ 8) whose column
// share Nc is at most 256 (the M = 128 MMA's N range), a whole number of
// 128-byte boxes of x, and leaves room for at least two operand stages beside
// the staged x tile; 0 if there is none.
int wo_norm_cluster(int D, bool x_bf16) {
  const int esz = x_bf16 ? 2 : 4, cpb = 128 / esz;
  if (D < 64 || D % kK) return 0;
  for (int cn = 1; cn <= kMaxCluster; ++cn) {
    if (D % cn) continue;
    const int nc = D / cn;
    if (nc > 256 || nc % cpb || nc % 32) continue;
    if (stages_for(nc, esz) >= 2) return cn;
  }
  return 0;
}

cudaError_t launch_wo_norm(const bozo_wo_add_rmsnorm_args& a, int* err, cudaStream_t st) {
  const bool bf = a.x_dtype == BOZO_DT_BF16;
  const int esz = bf ? 2 : 4, cpb = 128 / esz;
  WoP p{};
  p.M = a.rows;
  p.D = a.width;
  p.CN = wo_norm_cluster(a.width, bf);
  if (!p.CN) return cudaErrorInvalidValue;
  p.Nc = p.D / p.CN;
  p.KT = p.D / kK;
  p.stages = stages_for(p.Nc, esz);
  p.eps = a.eps;
  p.scale = a.scale;
  p.rstd = a.rstd;
  p.err = err;
  CUtensorMap tm_msg, tm_wo, tm_x, tm_out;
  const uint64_t D = (uint64_t)p.D, M = (uint64_t)p.M;
  if (!make_tmap_2d(&tm_msg, a.msg, false, D, M, D * 2, kK, kRows) ||
      !make_tmap_2d(&tm_wo, a.wo, false, D, D, D * 2, kK, p.Nc) ||
      !make_tmap_2d(&tm_x, a.x, !bf, D, M, D * esz, cpb, kRows) ||
      !make_tmap_2d(&tm_out, a.out, !bf, D, M, D * esz, cpb, kRows))
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)p.stages * stage_bytes(p.Nc) + tile_bytes(p.Nc, esz) + fixed_bytes();
  auto kern = bf ? wo_norm_kernel<true> : wo_norm_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.CN, (unsigned)((p.M + kRows - 1) / kRows), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.CN;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tm_msg, tm_wo, tm_x, tm_out, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace bozo
