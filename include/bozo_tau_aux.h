/*
 * bozo_tau_aux.h — C ABI of the fused τ-field consumer: the three τ
 * regularisers of the reference training loop, computed on the device from
 * the τ fields the tension operator exports, plus their cotangent.
 *
 * Reference interfaces replaced (BoggersTheFish/bozo):
 *   tension_diversity_loss       model.py:498-532
 *   constraint_consistency_loss  model.py:535-577
 *   tension_entropy_loss         model.py:580-611
 * as train.py:1083-1087 calls them, one τ field [B,T,H,W] per tension layer,
 * and the per-row entropies behind train.py:411-447 uncertainty_gate.
 * The reference evaluates each as a chain of framework ops over stacked
 * copies of the fields; here one launch reads every field once and produces
 * per-layer statistics, and one launch writes each field's cotangent.
 *
 * Per layer (rows r = (b,t,h), N = B·T·H rows of W values x_r):
 *   stats[l][0] = (1/N) Σ_r ent_r,  ent_r = −Σ_w p_w·log(p_w + 1e-8),
 *                 p_w = x_w / (Σ_w x_w + 1e-8)
 *   stats[l][1] = mean over i ∈ [0,m), t ∈ [i+2, i+2+T−m−1), b, h of
 *                 relu(x[t,i]·x[t−1,0] − x[t,i+1]),  m = min(W−2, 4)
 *                 (0 when W < 3, T < 3 or m+1 ≥ T: the layer is skipped)
 *   stats[l][2] = (1/N) Σ_r relu(0.05 − μ_r) + relu(μ_r − 0.8),  μ_r = Σ_w x_w / W
 * in fp32 from the stored τ values.  The reference's scalar tails — the mean
 * of stats[·][0] per window group and relu(log W − ·), the count of
 * consistency layers, the averages — are a few scalar ops on the host side
 * (bozo_b200/aux.py); their gradient arrives here as d_stats.
 *
 * The backward writes, for every layer, d_tau = Σ_k d_stats[l][k] ·
 * ∂stats[l][k]/∂τ (the whole field; no accumulation into existing values).
 * d_stats is read on the device, so no host synchronisation is needed.
 */
#ifndef BOZO_TAU_AUX_H
#define BOZO_TAU_AUX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BOZO_TAU_AUX_MAX_LAYERS 64

typedef struct {
  int32_t n_layers;       /* τ fields in this call: 1..BOZO_TAU_AUX_MAX_LAYERS */
  int32_t dtype;          /* bozo_dtype (bozo_tension.h) of every field */
  int32_t B, T, H, W;     /* every field is [B,T,H,W], contiguous */
  const void* tau[BOZO_TAU_AUX_MAX_LAYERS];
  float* stats;           /* out: [n_layers][3] fp32, device */
  void* workspace;        /* device scratch of bozo_tau_aux_workspace() bytes */
  size_t workspace_bytes;
  /* Optional out: [n_layers][B·T·H] fp32, each row's entropy ent_r (the
   * per-row term of stats[l][0]; train.py:411-447 uncertainty_gate averages
   * it over heads and layers), or NULL. */
  float* row_ent;
} bozo_tau_aux_fwd_args;

typedef struct {
  int32_t n_layers;
  int32_t dtype;
  int32_t B, T, H, W;
  const void* tau[BOZO_TAU_AUX_MAX_LAYERS];
  const float* d_stats;   /* [n_layers][3] fp32 cotangent of stats, device */
  void* d_tau[BOZO_TAU_AUX_MAX_LAYERS]; /* out: same shape and dtype as tau */
  /* Row mode (every d_tau NULL, every row_coef set): instead of d_tau write
   * per query row r = (b·H + h)·T + t the coefficients [a1, a0, inv_d]
   * ([3][B·H·T] fp32) with which the tension backward forms the cotangent
   * a1·(log2 q − 1e-8/(q·ln 2)) + a0, q = τ·inv_d + 1e-8, itself
   * (bozo_tension_bwd_args.aux_row).  That is the diversity and entropy
   * terms' cotangent exactly, evaluated at the τ the backward recomputes; it
   * needs the consistency cotangent d_stats[l][1] to be zero (not a per-row
   * quantity).  2-byte fields with W = 32·G, G ∈ {1, 2, 4, 8}, only. */
  float* row_coef[BOZO_TAU_AUX_MAX_LAYERS];
} bozo_tau_aux_bwd_args;

/* Bytes of device scratch the forward needs (per-block partial sums). */
size_t bozo_tau_aux_workspace(const bozo_tau_aux_fwd_args* args);

/* Statistics of every field (asynchronous on `stream`, a cudaStream_t).
 * Returns a bozo_status (bozo_tension.h). */
int bozo_tau_aux_fwd(const bozo_tau_aux_fwd_args* args, void* stream);

/* Cotangent of every field from d_stats (or, in row mode, its per-row
 * coefficients). */
int bozo_tau_aux_bwd(const bozo_tau_aux_bwd_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BOZO_TAU_AUX_H */
