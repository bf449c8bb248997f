/*
 * bozo_graph_bias.h — C ABI of the device-side construction of the graph
 * bias the tension operator adds before the sigmoid.
 *
 * Reference interfaces replaced (BoggersTheFish/bozo, ts_bridge/bias.py):
 *   GraphBias.local_bias   bias.py:125-170  [B, T, W]: slot w of query t is
 *                          key s = t − (W − w) (s ≥ 0)
 *   GraphBias.global_bias  bias.py:172-233  [B, T, T]: key s < t
 * Both set bias = α · edge_weight(content[s] → content[t]) where the edge
 * map holds a positive weight, else 0, and report the number of such
 * pairs, their largest and their mean weight.  The reference fills the
 * tensors with O(T·W) / O(T²) Python loops over dictionary lookups; here the
 * host maps each context token to a content id once (O(T)) and one kernel
 * looks every (key, query) pair up in a sorted table of 64-bit
 * (src_content << 32 | dst_content) keys by binary search.
 *
 * α and the weights are kept in double and each product is rounded to fp32
 * once, as the reference's Python-float product stored into an fp32 tensor.
 */
#ifndef BOZO_GRAPH_BIAS_H
#define BOZO_GRAPH_BIAS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int32_t T;                    /* context length */
  int32_t window;               /* W ≥ 1: local bias [T, W]; 0: global bias [T, T] */
  double alpha;
  const int32_t* ctx_content;   /* [T] device: content id of each token, −1 = no edges */
  const uint64_t* edge_keys;    /* [n_edges] device, ascending: (src << 32) | dst content ids */
  const double* edge_weights;   /* [n_edges] device */
  int64_t n_edges;
  float* out;                   /* [T, W] or [T, T] fp32, device, row-major */
  double* stats;                /* optional [3] device, zeroed by the caller: pairs with a
                                   positive weight, Σ weight, max weight (accumulated) */
} bozo_graph_bias_args;

/* Fills `out` (every element) and accumulates `stats` on `stream`.
 * Returns a bozo_status (bozo_tension.h). */
int bozo_graph_bias_build(const bozo_graph_bias_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BOZO_GRAPH_BIAS_H */
