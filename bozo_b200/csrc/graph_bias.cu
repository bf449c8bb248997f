// graph_bias.cu — the graph bias built on the device (include/bozo_graph_bias.h):
// every (query t, key s) pair of the local window or the causal triangle
// looks up the edge weight content[s] → content[t] in a sorted table of
// 64-bit keys by binary search, and the pair's bias is α · weight where that
// weight is positive (ts_bridge/bias.py:153-167, 213-226).  Grid-stride over
// the T·W (or T·T) output elements, row-major, so consecutive threads write
// consecutive floats; the context's content ids (T int32) stay in L1/L2.
// The statistics are accumulated with one atomic per warp and quantity.
#include "bozo_graph_bias.h"
#include "common.cuh"

namespace bozo {
namespace {

// Largest weight as the bit pattern of a non-negative double: for those,
// unsigned integer order is numeric order.
__device__ __forceinline__ void atomic_max_nonneg(double* addr, double v) {
  atomicMax(reinterpret_cast<unsigned long long*>(addr), (unsigned long long)__double_as_longlong(v));
}

__device__ __forceinline__ double edge_weight(const uint64_t* keys, const double* w, long long n,
                                              uint64_t key) {
  long long lo = 0, hi = n;  // first index with keys[i] >= key
  while (lo < hi) {
    const long long mid = (lo + hi) >> 1;
    if (__ldg(keys + mid) < key) lo = mid + 1;
    else hi = mid;
  }
  return (lo < n && __ldg(keys + lo) == key) ? __ldg(w + lo) : 0.0;
}

__global__ void graph_bias_kernel(int T, int W, double alpha, const int* __restrict__ cid,
                                  const uint64_t* __restrict__ keys, const double* __restrict__ w,
                                  long long n_edges, float* __restrict__ out, double* stats) {
  const int cols = W > 0 ? W : T;
  const long long total = (long long)T * cols;
  const long long stride = (long long)gridDim.x * blockDim.x;
  double hits = 0.0, sum = 0.0, mx = 0.0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int t = (int)(i / cols), c = (int)(i - (long long)t * cols);
    const int s = W > 0 ? t - (W - c) : c;  // local slot c, or key column c
    const bool live = W > 0 ? s >= 0 : s < t;
    double wt = 0.0;
    if (live) {
      const int a = __ldg(cid + s), b = __ldg(cid + t);
      if (a >= 0 && b >= 0)
        wt = edge_weight(keys, w, n_edges, ((uint64_t)(uint32_t)a << 32) | (uint32_t)b);
    }
    if (wt > 0.0) {
      out[i] = (float)(alpha * wt);
      hits += 1.0;
      sum += wt;
      mx = fmax(mx, wt);
    } else {
      out[i] = 0.f;
    }
  }
  if (stats) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      hits += __shfl_xor_sync(0xffffffffu, hits, o);
      sum += __shfl_xor_sync(0xffffffffu, sum, o);
      mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if ((threadIdx.x & 31) == 0 && hits > 0.0) {
      atomicAdd(stats, hits);
      atomicAdd(stats + 1, sum);
      atomic_max_nonneg(stats + 2, mx);
    }
  }
}

}  // namespace

cudaError_t launch_graph_bias(const bozo_graph_bias_args& a, int sms, cudaStream_t st) {
  const long long total = (long long)a.T * (a.window > 0 ? a.window : a.T);
  const long long want = (total + 255) / 256;
  const int grid = (int)(want < (long long)sms * 8 ? (want < 1 ? 1 : want) : (long long)sms * 8);
  graph_bias_kernel<<<grid, 256, 0, st>>>(a.T, a.window, a.alpha, a.ctx_content, a.edge_keys,
                                          a.edge_weights, a.n_edges, a.out, a.stats);
  return cudaGetLastError();
}

}  // namespace bozo
