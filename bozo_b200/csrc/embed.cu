// embed.cu — gradient of the token-embedding lookup with respect to its
// weight (the model's tok_emb, model.py: out[p] = weight[ids[p]], the weight
// tied to the output head): d_weight[v] = Σ_{p : ids[p] = v} d_out[p].
//
// The caller sorts the ids stably with their positions (keys ascending,
// equal keys in increasing position).  Pass 1 marks each key's run
// [start, end) in the sorted order; pass 2 gives every vocabulary row one
// warp that sums its run's d_out rows in that order — a fixed order, so the
// result is the same on every call — and writes the row (zeros where the
// token does not occur).  Every weight row is written exactly once: 4·V·D
// bytes out, 4·n·D bytes of d_out in, with no atomics and no zero-fill pass.
#include <cuda_runtime.h>
#include <stdint.h>

#include "bozo_block_ops.h"
#include "common.cuh"

namespace bozo {
namespace {

constexpr int kRowWarps = 8;    // warps (vocabulary rows) per block
constexpr int kColVecs = 8;     // float4 per lane per column block: 1024 floats per pass

__global__ void embed_runs_kernel(const int32_t* __restrict__ keys, long long n, int vocab,
                                  int32_t* __restrict__ start, int32_t* __restrict__ end) {
  for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < n;
       j += (long long)gridDim.x * blockDim.x) {
    const int k = keys[j];
    if ((unsigned)k >= (unsigned)vocab) continue;  // ids outside the table own no row
    if (j == 0 || keys[j - 1] != k) start[k] = (int32_t)j;
    if (j == n - 1 || keys[j + 1] != k) end[k] = (int32_t)(j + 1);
  }
}

__global__ void embed_rows_kernel(const int32_t* __restrict__ start, const int32_t* __restrict__ end,
                                  const int64_t* __restrict__ order, const float* __restrict__ d_out,
                                  int vocab, int dim, float* __restrict__ d_weight) {
  const int lane = threadIdx.x & 31;
  const int nv = dim >> 2;  // float4 per row
  for (int v = blockIdx.x * kRowWarps + (threadIdx.x >> 5); v < vocab; v += gridDim.x * kRowWarps) {
    const int s = start[v], e = end[v];
    float4* dst = reinterpret_cast<float4*>(d_weight + (long long)v * dim);
    for (int c0 = 0; c0 < nv; c0 += 32 * kColVecs) {
      float4 acc[kColVecs];
#pragma unroll
      for (int z = 0; z < kColVecs; ++z) acc[z] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = s; j < e; ++j) {
        const float4* src = reinterpret_cast<const float4*>(d_out + __ldg(order + j) * dim);
#pragma unroll
        for (int z = 0; z < kColVecs; ++z) {
          const int c = c0 + lane + 32 * z;
          if (c < nv) {
            const float4 x = __ldg(src + c);
            acc[z].x += x.x; acc[z].y += x.y; acc[z].z += x.z; acc[z].w += x.w;
          }
        }
      }
#pragma unroll
      for (int z = 0; z < kColVecs; ++z) {
        const int c = c0 + lane + 32 * z;
        if (c < nv) dst[c] = acc[z];
      }
    }
  }
}

}  // namespace

cudaError_t launch_embedding_bwd(const bozo_embedding_bwd_args& a, int sms, cudaStream_t st) {
  int32_t* start = a.scratch;
  int32_t* end = a.scratch + a.vocab;
  // empty runs for every row first (start = end = 0)
  cudaError_t e = cudaMemsetAsync(a.scratch, 0, sizeof(int32_t) * 2 * (size_t)a.vocab, st);
  if (e != cudaSuccess) return e;
  const long long want = (a.n + 255) / 256;
  const int g1 = (int)(want < (long long)sms * 8 ? (want < 1 ? 1 : want) : (long long)sms * 8);
  embed_runs_kernel<<<g1, 256, 0, st>>>(a.sorted_ids, a.n, a.vocab, start, end);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int rows_blocks = (a.vocab + kRowWarps - 1) / kRowWarps;
  const int g2 = rows_blocks < sms * 16 ? rows_blocks : sms * 16;
  embed_rows_kernel<<<g2, 32 * kRowWarps, 0, st>>>(start, end, a.order, a.d_out, a.vocab, a.dim,
                                                   a.d_weight);
  return cudaGetLastError();
}

}  // namespace bozo
