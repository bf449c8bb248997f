/*
 * bozo_block_ops.h — C ABI of the fused elementwise work around the tension
 * operator in a TensionLM block.
 *
 * Reference interfaces replaced (BoggersTheFish/bozo, model.py):
 *   RMSNorm after a residual add   model.py:86-98 applied to x + wo(msg)
 *                                  (model.py:259, 283) and x + proj(h)
 *                                  (model.py:330); plain RMSNorm (y NULL) for
 *                                  the pre-norm and final norm (model.py:376, 458)
 *   SwiGLU                         model.py:328-329, silu(gate(x)) · val(x)
 *   cross-entropy loss             train.py:920 nn.CrossEntropyLoss() (mean over
 *                                  rows whose target is not −100) of the logits
 * each with its backward, in place of the framework's separate add, norm,
 * silu and multiply kernels and its column reduction for the norm scale's
 * gradient.
 *
 * add + RMSNorm (rows × width, width a multiple of 128 with width/128 ∈
 * {1, 2, 4, 6, 8}; all tensors contiguous):
 *   s = x + y (rounded to x's dtype when that is bf16), rstd = rsqrt(mean(s²)
 *   + eps), out = s·rstd·scale in x's dtype.  x fp32 with y fp32 or bf16, or
 *   x bf16 with y bf16.  Backward: dx (x's dtype), dy (y's dtype, when y is
 *   given) = rstd·(g − ŝ·mean(g·ŝ)), g = d_out·scale, ŝ = s·rstd;
 *   d_scale = Σ_rows d_out·ŝ, summed in a fixed order (deterministic).
 * SwiGLU (n elements, n a multiple of 4, fp32 or bf16, fp32 arithmetic):
 *   out = silu(gate)·value; d_gate = d_out·value·σ(gate)·(1 + gate·(1 − σ(gate))),
 *   d_value = d_out·silu(gate).
 */
#ifndef BOZO_BLOCK_OPS_H
#define BOZO_BLOCK_OPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int64_t rows;
  int32_t width;
  float eps;
  const void* x;          /* [rows, width] residual stream */
  int32_t x_dtype;        /* bozo_dtype: F32 or BF16 */
  const void* y;          /* [rows, width] addend, or NULL (plain RMSNorm) */
  int32_t y_dtype;
  const void* scale;      /* [width], x's dtype */
  void* out;              /* forward: [rows, width], x's dtype */
  float* rstd;            /* [rows]: written by the forward, read by the backward */
  const void* d_out;      /* backward: cotangent of out, x's dtype */
  void* dx;               /* backward: x's dtype */
  void* dy;               /* backward: y's dtype (NULL when y is NULL) */
  void* d_scale;          /* backward: [width], x's dtype */
  void* workspace;        /* backward: bozo_add_rmsnorm_workspace() bytes */
  size_t workspace_bytes;
  /* Optional, fp32 x only: the forward also writes out rounded to bf16 here
   * (what bf16 autocast would cast out to for the projections that read it,
   * made once), and the backward adds this bf16 cotangent of that copy to
   * d_out.  NULL: not used. */
  void* out_lp;           /* forward: [rows, width] bf16 */
  const void* d_out_lp;   /* backward: [rows, width] bf16 */
} bozo_add_rmsnorm_args;

size_t bozo_add_rmsnorm_workspace(const bozo_add_rmsnorm_args* args);
int bozo_add_rmsnorm_fwd(const bozo_add_rmsnorm_args* args, void* stream);
int bozo_add_rmsnorm_bwd(const bozo_add_rmsnorm_args* args, void* stream);

typedef struct {
  int64_t n;              /* elements, a multiple of 4 */
  int32_t dtype;          /* bozo_dtype: F32 or BF16 (all tensors) */
  const void* gate;
  const void* value;
  void* out;              /* forward */
  const void* d_out;      /* backward */
  void* d_gate;
  void* d_value;
  /* 0: gate/value/d_gate/d_value are flat like out.  Otherwise out holds
   * rows of `width` elements (n / width rows, width a multiple of 4) and the
   * other four hold rows of `width` elements `row_stride` elements apart
   * (row_stride a multiple of 4) — e.g. the two halves of one GEMM's packed
   * [gate | value] rows: value = gate + width, row_stride = 2·width. */
  int64_t width;
  int64_t row_stride;
} bozo_swiglu_args;

int bozo_swiglu_fwd(const bozo_swiglu_args* args, void* stream);
int bozo_swiglu_bwd(const bozo_swiglu_args* args, void* stream);

/* The attention-output projection fused with the residual add and RMSNorm
 * that follow it, forward only:
 *   y = bf16(msg · woᵀ), s = x + y (rounded to x's dtype when that is bf16),
 *   rstd = rsqrt(mean(s²) + eps), out = s·rstd·scale in x's dtype
 * — the same numbers as a bf16 projection followed by bozo_add_rmsnorm_fwd,
 * without the projection's [rows, width] output going through device memory.
 * Replaces model.py:259 / 283 (`self.norm(x + self.wo(msg))`, RMSNorm
 * model.py:86-98) on paths without gradients (prefill, decode, evaluation).
 * msg [rows, width] and wo [width, width] (nn.Linear weight, out × in) bf16
 * contiguous and 16-byte aligned; x, scale, out as in bozo_add_rmsnorm_args;
 * rstd [rows] fp32 or NULL.  Widths: bozo_wo_add_rmsnorm_supported says
 * (64, 128, 256, 384, 512, 768, 1024 for both x dtypes, 2048 for bf16 x;
 * BOZO_ERR_UNSUPPORTED otherwise). */
typedef struct {
  int64_t rows;
  int32_t width;
  float eps;
  const void* msg;        /* [rows, width] bf16: the tension layer's normalised output */
  const void* wo;         /* [width, width] bf16: the projection's weight */
  const void* x;          /* [rows, width] residual stream */
  int32_t x_dtype;        /* bozo_dtype: F32 or BF16 */
  const void* scale;      /* [width], x's dtype */
  void* out;              /* [rows, width], x's dtype */
  float* rstd;            /* [rows] or NULL */
} bozo_wo_add_rmsnorm_args;

int bozo_wo_add_rmsnorm_fwd(const bozo_wo_add_rmsnorm_args* args, void* stream);
/* 1 if bozo_wo_add_rmsnorm_fwd takes this width with x of this dtype. */
int bozo_wo_add_rmsnorm_supported(int32_t width, int32_t x_dtype);

/* Cross-entropy from the logits in their own dtype (bf16 or fp32, fp32
 * arithmetic).  Forward: row_lse[r] = logsumexp(logits[r]) and row_loss[r] =
 * row_lse[r] − logits[r][targets[r]] (0 where the target is outside
 * [0, vocab), e.g. −100); the mean is the caller's sum of row_loss over the
 * live rows.  Backward: d_logits[r] = (softmax(logits[r]) − onehot)·g with
 * g = *d_scale (device scalar: the mean's cotangent ÷ live rows), zero rows
 * for ignored targets. */
typedef struct {
  int64_t rows;
  int32_t vocab;          /* a multiple of 8 (bf16) or 4 (fp32) */
  const void* logits;     /* [rows, vocab] contiguous */
  int32_t logits_dtype;
  const int64_t* targets; /* [rows] */
  float* row_lse;         /* [rows]: forward writes, backward reads */
  float* row_loss;        /* [rows]: forward */
  const float* d_scale;   /* backward: device scalar g */
  void* d_logits;         /* backward: [rows, vocab], logits' dtype */
} bozo_cross_entropy_args;

int bozo_cross_entropy_fwd(const bozo_cross_entropy_args* args, void* stream);
int bozo_cross_entropy_bwd(const bozo_cross_entropy_args* args, void* stream);

/* Gradient of a token-embedding lookup (out[p] = weight[ids[p]]) with
 * respect to the weight: d_weight[v] = Σ of d_out[p] over the positions p
 * with ids[p] = v, summed in increasing p (the same result on every call),
 * and zero rows for tokens that do not occur.  Replaces the weight gradient
 * of nn.Embedding (model.py's tok_emb, tied to the output head).  The caller
 * sorts the n ids stably: sorted_ids ascending (int32), order their positions
 * (int64) — e.g. torch.sort(ids.int(), stable=True).  Ids outside [0, vocab)
 * contribute nothing.  d_out [n, dim] and d_weight [vocab, dim] fp32
 * contiguous, 16-byte aligned, dim a multiple of 4; scratch holds
 * 2·vocab int32 (run bounds). */
typedef struct {
  int64_t n;              /* positions */
  int32_t dim;
  int32_t vocab;
  const int32_t* sorted_ids;
  const int64_t* order;
  const float* d_out;
  float* d_weight;        /* written in full */
  int32_t* scratch;       /* [2·vocab] int32 */
} bozo_embedding_bwd_args;

int bozo_embedding_bwd(const bozo_embedding_bwd_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BOZO_BLOCK_OPS_H */
