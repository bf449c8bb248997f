/*
 * bozo_tension.h — C ABI of the B200 (sm_100a) sigmoid-tension operator.
 *
 * Plain pointers, sizes and strides only: no framework types cross this
 * boundary.  Every call is asynchronous on the caller's CUDA stream, borrows
 * its inputs, writes caller-allocated outputs, keeps no state between calls
 * and is safe to call concurrently from several host threads (one stream
 * each).
 *
 * Semantics (Q,K,V,dO are [B,T,H,HD]; σ = logistic sigmoid; scale = √HD in
 * the reference model):
 *
 *   LOCAL  (window W ≥ 1): key slot w ∈ [0,W) of query t is position
 *          s = t − (W − w); valid iff s ≥ 0 (self excluded).
 *   GLOBAL (full causal):  keys s ∈ [0, t] (self included).
 *
 *   τ[t,s] = σ( Rq_t·Rk_s / scale + bias ) · valid     (R = optional RoPE)
 *   S_t    = Σ_s τ[t,s] · V_s
 *   out_t  = S_t                          (BOZO_NORM_NONE  — raw op)
 *          = S_t / max(Σ_s τ[t,s], 1e-6)  (BOZO_NORM_MASS  — τ-mass)
 *          = S_t / max(#valid slots, 1)   (BOZO_NORM_COUNT — position count)
 *
 * Reference interfaces replaced (BoggersTheFish/bozo):
 *   bozo_tension_fwd  ← triton_tension/ops.py:75-124 (_CausalTensionFn.forward,
 *                       the _fwd_kernel launch at ops.py:104) and, with
 *                       NORM_MASS / NORM_COUNT / rope / GLOBAL, the
 *                       surrounding model.py:200-237, 257-258, 261-264 code.
 *   bozo_tension_bwd  ← triton_tension/ops.py:126-187 (_CausalTensionFn.backward,
 *                       the _bwd_dq_kernel / _bwd_dkv_kernel launches at
 *                       ops.py:165 and ops.py:174) plus autograd of the
 *                       model.py normalisation and RoPE.
 */
#ifndef BOZO_TENSION_H
#define BOZO_TENSION_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BOZO_TENSION_ABI_VERSION 7

typedef enum {
  BOZO_OK = 0,
  BOZO_ERR_BAD_SHAPE = 1,      /* non-positive sizes, W < 1, bad bias/tau shape */
  BOZO_ERR_BAD_DTYPE = 2,      /* dtype code not in bozo_dtype */
  BOZO_ERR_UNSUPPORTED = 3,    /* e.g. HD > 128, odd HD with RoPE */
  BOZO_ERR_ALIGNMENT = 4,      /* a forced tensor-core path got unaligned data */
  BOZO_ERR_NULL = 5,           /* a required pointer is NULL */
  BOZO_ERR_DEVICE_TIMEOUT = 6, /* a bounded device-side wait gave up */
  BOZO_ERR_CUDA = 7,           /* a CUDA runtime call failed */
  BOZO_ERR_WORKSPACE = 8,      /* workspace NULL or smaller than required */
  BOZO_ERR_SCRATCH_LIMIT = 9   /* bozo_tension_bwd_noalloc: problem needs more
                                  than BOZO_NOALLOC_SCRATCH_BYTES of scratch */
} bozo_status;

/* Size of the library's fixed device scratch array used by
 * bozo_tension_bwd_noalloc (8 MiB per device). */
#define BOZO_NOALLOC_SCRATCH_BYTES (8u << 20)

typedef enum { BOZO_DT_F32 = 0, BOZO_DT_BF16 = 1, BOZO_DT_F16 = 2 } bozo_dtype;
typedef enum { BOZO_MODE_LOCAL = 0, BOZO_MODE_GLOBAL = 1 } bozo_mode;
typedef enum { BOZO_NORM_NONE = 0, BOZO_NORM_MASS = 1, BOZO_NORM_COUNT = 2 } bozo_norm;

/* Kernel-path selection (flags). AUTO picks the tcgen05 path whenever the
 * inputs qualify (bf16 Q/K/V with unit HD stride, 16-byte aligned rows,
 * HD = 64, LOCAL, W ≤ 128, RoPE given with rope_theta), else the
 * exact-fp32 SIMT path. */
enum {
  BOZO_PATH_AUTO = 0,
  BOZO_PATH_SIMT = 1,     /* force the fp32 CUDA-core path */
  BOZO_PATH_TCGEN05 = 2   /* force the tensor-core path; error if ineligible */
};

/* A strided 4-D view [B,T,H,HD] (element strides). */
typedef struct {
  const void* ptr;
  int32_t dtype;          /* bozo_dtype */
  int32_t _pad;
  int64_t stride[4];      /* b, t, h, d — in elements */
} bozo_tensor4;

typedef struct {
  int32_t B, T, H, HD;
  int32_t mode;           /* bozo_mode */
  int32_t window;         /* LOCAL: W. GLOBAL: width of the exported τ window
                             (min(local W, T) as model.py:235 takes it). */
  int32_t normalize;      /* bozo_norm */
  int32_t path;           /* BOZO_PATH_* */
  float scale;            /* divisor of the dot product (√HD in model.py:122) */
  int32_t rope_len;       /* rows of the RoPE tables (≥ T) or 0 for no RoPE */
  const float* rope_cos;  /* [rope_len, HD/2] fp32 contiguous, or NULL */
  const float* rope_sin;
  const float* rope_theta; /* [HD/2] fp32 frequencies θ_i of those tables
                              (cos[t][i] = cos(t·θ_i)); lets the tensor-core
                              kernels evaluate the rotation on the fly.
                              Optional: NULL keeps table lookups only. */
  bozo_tensor4 q, k, v;
  const float* bias;      /* LOCAL [B,T,W] / GLOBAL [B,T,T] fp32, or NULL */
  int64_t bias_stride[3];
  /* outputs */
  void* out;              /* [B,T,H,HD] contiguous, dtype out_dtype */
  int32_t out_dtype;
  int32_t tau_dtype;
  void* tau;              /* [B,T,H,window] contiguous or NULL (no export) */
  float* row_mass;        /* [B,H,T] fp32 Σ_s τ (unclamped) or NULL */
  void* q_rot;            /* optional [B,T,H,HD] contiguous copies of RoPE(q), */
  void* k_rot;            /* RoPE(k) in q/k's dtype (for a later backward)    */
  /* Optional room for bf16 operand copies of fp32 q and k ([B,T,H,HD]
   * contiguous, 16-byte aligned).  When both are set and q, k are fp32, the
   * forward always writes bf16(q), bf16(k) here; when
   * bozo_tension_fwd_needs_lp() is 1 it also runs the tensor-core kernels on
   * them (fp32 out and τ).  The caller keeps them and passes them to the
   * backward as q and k, with grad_dtype F32 for dq/dk.  NULL keeps an
   * fp32-q/k call on the exact fp32 path. */
  void* q_lp;
  void* k_lp;
} bozo_tension_fwd_args;

typedef struct {
  int32_t B, T, H, HD;
  int32_t mode, window, normalize, path;
  float scale;
  int32_t rope_len;
  const float* rope_cos;
  const float* rope_sin;
  const float* rope_theta;
  bozo_tensor4 q, k, v;   /* the forward inputs (pre-RoPE when RoPE is on) */
  bozo_tensor4 d_out;     /* cotangent of out */
  bozo_tensor4 out;       /* forward output — read only for NORM_MASS */
  const float* row_mass;  /* forward Σ τ [B,H,T] — required for NORM_MASS */
  const float* bias;
  int64_t bias_stride[3];
  const void* d_tau;      /* [B,T,H,window] contiguous cotangent of τ, or NULL */
  int32_t d_tau_dtype;
  int32_t grad_dtype[3];  /* dtypes of dq, dk, dv */
  int32_t qk_rotated;     /* 1: q, k above are already RoPE-rotated (the
                             forward's q_rot/k_rot); dq, dk are still
                             returned w.r.t. the pre-RoPE inputs */
  void* dq;               /* [B,T,H,HD] contiguous (gradient w.r.t. pre-RoPE q) */
  void* dk;
  void* dv;
  void* workspace;        /* device scratch of bozo_tension_bwd_workspace() bytes
                             (with bf16 q/k and an fp32 d_out it includes room
                             for a bf16 copy of d_out) */
  size_t workspace_bytes;
  /* Optional cotangent of τ given per query row instead of per element (the
   * fused τ consumer's diversity and entropy terms, bozo_tau_aux.h): for
   * every valid slot of query row r = (b·H + h)·T + t it adds
   *     a1·(log2 q − 1e-8/(q·ln 2)) + a0,   q = τ·inv_d + 1e-8,
   * a1 = aux_row[r], a0 = aux_row[n + r], inv_d = aux_row[2n + r]
   * (n = B·H·T) to the cotangent of τ, with τ as the backward recomputes
   * it.  fp32 [3][B·H·T] or NULL.  LOCAL windows on the tensor-core path
   * only (BOZO_ERR_UNSUPPORTED otherwise); combines with d_tau. */
  const float* aux_row;
} bozo_tension_bwd_args;

/* One decode step: the query of a new token at position t against ring
 * caches of the earlier tokens' RoPE-rotated keys and values, O(W) work per
 * (b, h) for a local layer (O(C) for a global one) instead of model.py:
 * 718-768's re-run of the whole context per generated token.  The step
 * first writes RoPE(k_t) and v_t into ring row t mod capacity, then
 *   LOCAL : keys s ∈ [max(0, t−W), t−1]             (self excluded)
 *   GLOBAL: keys s ∈ [max(0, t−capacity+1), t]      (self included; a wrapped
 *           ring keeps the last `capacity` keys, as a sliding context does)
 *   out    = Σ τ·v / (τ-mass | valid count | 1)   (normalize)
 *   τ row  = LOCAL slot w ↔ key t − (W − w); GLOBAL column c ↔ key t − c
 *           (row t of the exported field, model.py:233-236), 0 where no key.
 * t is read from device memory (`pos`), so the step can be captured in a
 * CUDA graph and replayed per token.  No bias.  A t outside [0, rope_len)
 * with RoPE sets the device error word (bozo_tension_poll_error). */
typedef struct {
  int32_t B, H, HD;
  int32_t mode;           /* bozo_mode */
  int32_t window;         /* LOCAL: W.  GLOBAL: unused (0) */
  int32_t normalize;      /* bozo_norm */
  int32_t capacity;       /* ring rows C: LOCAL ≥ W + 1 */
  int32_t tau_width;      /* columns of the τ row (LOCAL: W) when tau is set */
  float scale;            /* divisor of the dot product */
  const int32_t* pos;     /* device int32: position t of the new token */
  int32_t rope_len;       /* rows of the RoPE tables (> t) or 0 for no RoPE */
  const float* rope_cos;  /* [rope_len, HD/2] fp32 contiguous, or NULL */
  const float* rope_sin;
  bozo_tensor4 q, k, v;   /* the new token's projections as [B,1,H,HD] views */
  void* k_cache;          /* [B, capacity, H, HD] contiguous, RoPE(k) rows */
  int32_t k_cache_dtype;
  void* v_cache;          /* [B, capacity, H, HD] contiguous */
  int32_t v_cache_dtype;
  void* out;              /* [B, H, HD] contiguous */
  int32_t out_dtype;
  void* tau;              /* [B, H, tau_width] contiguous, or NULL */
  int32_t tau_dtype;
} bozo_tension_decode_args;

/* Reference interface replaced: model.py:718-768 (generate_cached: one full
 * forward over the last max_seq_len tokens per generated token) and the τ
 * row ts_bridge/streaming.py:100-194 (ingest_step) takes from such a
 * forward. */
int bozo_tension_decode(const bozo_tension_decode_args* args, void* stream);

/* 1 when this forward, given q_lp / k_lp, runs on the tensor-core kernels
 * from bf16 copies of fp32 q and k: the reference's mixed-dtype call
 * (model.py:248-264 under bf16 autocast — RoPE-promoted fp32 Q/K, bf16 V,
 * fp32 out and τ as ops.py:122-124 returns them; local window ≤ 128,
 * HD 64, no RoPE inside the call).  Depends only on the arguments, so a
 * caller can decide whether to allocate the copies before the call.
 * Replaces nothing in the reference (its Triton kernels load every dtype as
 * fp32, triton_tension/kernel.py:76). */
int bozo_tension_fwd_needs_lp(const bozo_tension_fwd_args* args);

/* Forward. Returns bozo_status; launches are asynchronous on `stream`
 * (a cudaStream_t, NULL = legacy default stream). */
int bozo_tension_fwd(const bozo_tension_fwd_args* args, void* stream);

/* Device scratch the backward uses for these arguments (bytes, 256-aligned
 * size; 0 is possible).  For the key-tile kernels (global block, windows
 * wider than 128, bf16 HD 64) it includes a dSᵀ scratch of
 * 2·B·H·nT·D·16 KiB (nT = ceil(T/128); D = nT for the global block, else
 * min(nT, floor((W+127)/128)+1)) that spares the dQ pass recomputing the
 * scores; a workspace of only the rest (what bozo_tension_bwd_noalloc
 * checks) still works, with that recomputation. */
size_t bozo_tension_bwd_workspace(const bozo_tension_bwd_args* args);

/* Backward: writes dq, dk, dv. */
int bozo_tension_bwd(const bozo_tension_bwd_args* args, void* stream);

/* Backward that allocates nothing. This entry point has no counterpart in the
 * reference. It is for callers that cannot allocate device memory per call: a plain C,
 * cgo or ctypes host with no caching allocator (a cudaMalloc/cudaFree pair per
 * backward would synchronise the device each step), or a service that reserves
 * all device memory at start-up and may not allocate afterwards.
 * Same arguments and results as bozo_tension_bwd, except that `workspace` and
 * `workspace_bytes` are ignored: the scratch is a fixed array of
 * BOZO_NOALLOC_SCRATCH_BYTES inside the library, one per device. Problems whose
 * bozo_tension_bwd_workspace() exceeds that size return
 * BOZO_ERR_SCRATCH_LIMIT before anything is launched.
 * The first call on a device looks up the array's device address (once per
 * device, with that device current); make that first call before any stream
 * capture begins. Calls that overlap in time on one device (two streams, two
 * threads) share the array and race; the array keeps the last call's contents
 * after it returns. */
int bozo_tension_bwd_noalloc(const bozo_tension_bwd_args* args, void* stream);

/* Synchronise `stream`, then read and clear the device error word that
 * bounded waits inside the tensor-core kernels set when they give up.
 * Returns BOZO_OK or BOZO_ERR_DEVICE_TIMEOUT (or BOZO_ERR_CUDA). */
int bozo_tension_poll_error(void* stream);

/* Enqueue on `stream` an asynchronous copy of the device error word of the
 * current device into host memory (pinned for a truly asynchronous copy), so
 * a caller can check it once the stream has passed that point without
 * synchronising every step.  A non-zero value means a bounded wait gave up in
 * some earlier launch: call bozo_tension_poll_error to read and clear it.
 * No counterpart in the reference (it has no device-side waits). */
int bozo_tension_error_async(int32_t* host_dst, void* stream);

/* Self-test of the bounded device waits; no counterpart in the reference (its
 * only timeout is the NCCL one train.py:561-564 comments on).  One CTA starts
 * a bulk copy and a tensor-core MMA, then waits on an mbarrier that nothing
 * arrives on, limited to limit_ns nanoseconds (1 µs … 1 s, else
 * BOZO_ERR_BAD_SHAPE) instead of the kernels' 4 s.  The wait gives up and
 * sets the device error word (bozo_tension_poll_error then returns
 * BOZO_ERR_DEVICE_TIMEOUT); the CTA drains the copy and the MMA with bounded
 * waits and releases its TMEM before it exits — the exit path of every
 * tensor-core kernel — so the context stays usable.  `result`: device
 * int32[4] or NULL — [0] 1 if the wait gave up, [1] 1 if the copy drained,
 * [2] 1 if the MMA drained, [3] microseconds the wait took. */
int bozo_tension_wait_selftest(uint64_t limit_ns, int32_t* result, void* stream);

/* Which kernel path the last successful call in this process ran:
 * BOZO_PATH_SIMT or BOZO_PATH_TCGEN05 (0 before any call). */
int bozo_tension_last_path(void);

/* Number of kernels the last successful call in this process launched. */
int bozo_tension_last_launches(void);

const char* bozo_status_string(int status);
int bozo_tension_abi_version(void);

/* Name of the CUDA runtime error behind the last BOZO_ERR_CUDA returned in
 * this process ("cudaSuccess" if none). */
const char* bozo_tension_last_cuda_error(void);

#ifdef __cplusplus
}
#endif

#endif /* BOZO_TENSION_H */
