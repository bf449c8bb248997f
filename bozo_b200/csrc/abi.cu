// abi.cu — the extern "C" boundary (include/bozo_tension.h): argument
// validation, kernel-path selection and launch bookkeeping.
//
// Validation mirrors the reference's asserts: bias must be [B,T,W]
// (triton_tension/ops.py:93-97), tensors are 4-D [B,T,H,HD] (ops.py:22-24).
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "tc.cuh"
#include "tc_host.cuh"

namespace bozo {
namespace {

__device__ int g_device_error;  // set by bounded device-side waits

// Last path / launch count, process-wide (autograd may run the backward on
// its own device thread, so these are not thread-local).
std::atomic<int> t_last_path{0};
std::atomic<int> t_last_launches{0};
std::atomic<int> t_last_cuda_error{0};

int cuda_fail(cudaError_t e) {
  t_last_cuda_error = (int)e;
  return BOZO_ERR_CUDA;
}

constexpr int kMaxDevices = 64;
int* g_err_ptr[kMaxDevices] = {nullptr};
std::mutex g_err_mu;

// Device address of the error word for the current device (looked up once
// per device; cudaGetSymbolAddress needs that device current).
int* error_word(cudaError_t* e) {
  int dev = 0;
  *e = cudaGetDevice(&dev);
  if (*e != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (!g_err_ptr[dev]) {
    void* ptr = nullptr;
    *e = cudaGetSymbolAddress(&ptr, g_device_error);
    if (*e != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(ptr);
  }
  return g_err_ptr[dev];
}

// Fixed backward scratch for bozo_tension_bwd_noalloc, for callers that may
// not allocate device memory per call (a C/cgo/ctypes host without a caching
// allocator, where cudaMalloc/cudaFree would synchronise the device every
// step, or a service that reserves its memory once at start-up).  The array
// is part of the module image, so using it allocates nothing.  No byte of it
// has to start at zero: the first kernel of either backward path writes every
// coefficient the later one reads.  Overlapping calls on one device share it
// and race; it keeps the last call's contents.
__device__ __align__(256) unsigned char g_noalloc_scratch[BOZO_NOALLOC_SCRATCH_BYTES];
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device, looked up once
// per device with that device current (the first call should come before any
// stream capture begins).
void* noalloc_scratch(cudaError_t* e) {
  int dev = 0;
  *e = cudaGetDevice(&dev);
  if (*e != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= kMaxDevices) {
    *e = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    *e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
    if (*e != cudaSuccess) return nullptr;
    g_scratch_ptr[dev] = ptr;
  }
  return g_scratch_ptr[dev];
}

// Make the device that owns `ptr` current on the calling thread, with its
// primary context bound.  Calls may arrive on threads that never touched CUDA
// through this library (e.g. an autograd worker thread); without this the
// driver-level tensor-map encoder sees no context and kernels would go to the
// runtime's default device.
//
// The caller's current device is put back when the entry point returns
// (DeviceRestore), so a call with data on another GPU does not switch the
// calling thread — and the framework that owns it — to that GPU.
struct DeviceRestore {
  int prev = -1;
  DeviceRestore() = default;
  DeviceRestore(const DeviceRestore&) = delete;
  DeviceRestore& operator=(const DeviceRestore&) = delete;
  ~DeviceRestore() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

cudaError_t bind_device(const void* ptr, DeviceRestore& restore) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
  if (e != cudaSuccess) return e;
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return cudaErrorInvalidDevicePointer;
  int cur = -1;
  if (cudaGetDevice(&cur) == cudaSuccess && cur != attr.device) restore.prev = cur;
  return cudaSetDevice(attr.device);
}

bool dtype_ok(int dt) { return dt == BOZO_DT_F32 || dt == BOZO_DT_BF16 || dt == BOZO_DT_F16; }

int check_common(int B, int T, int H, int HD, int mode, int W, int norm, float scale,
                 int rope_len, const float* cos, const float* sin) {
  if (B <= 0 || T <= 0 || H <= 0 || HD <= 0) return BOZO_ERR_BAD_SHAPE;
  if (HD > 128) return BOZO_ERR_UNSUPPORTED;
  if (mode != BOZO_MODE_LOCAL && mode != BOZO_MODE_GLOBAL) return BOZO_ERR_BAD_SHAPE;
  if (mode == BOZO_MODE_LOCAL && W < 1) return BOZO_ERR_BAD_SHAPE;
  if (mode == BOZO_MODE_GLOBAL && W < 0) return BOZO_ERR_BAD_SHAPE;
  if (norm != BOZO_NORM_NONE && norm != BOZO_NORM_MASS && norm != BOZO_NORM_COUNT)
    return BOZO_ERR_BAD_SHAPE;
  if (mode == BOZO_MODE_GLOBAL && norm == BOZO_NORM_COUNT) return BOZO_ERR_UNSUPPORTED;
  if (!(scale != 0.f)) return BOZO_ERR_BAD_SHAPE;
  if (rope_len != 0) {
    if (!cos || !sin) return BOZO_ERR_NULL;
    if (HD % 2 != 0) return BOZO_ERR_UNSUPPORTED;
    if (rope_len < T) return BOZO_ERR_BAD_SHAPE;
  }
  return BOZO_OK;
}

int check_t4(const bozo_tensor4& t) {
  if (!t.ptr) return BOZO_ERR_NULL;
  if (!dtype_ok(t.dtype)) return BOZO_ERR_BAD_DTYPE;
  return BOZO_OK;
}

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

// Shared checks of the two τ-consumer argument blocks.
template <typename A>
int check_aux(const A* a) {
  if (!a) return BOZO_ERR_NULL;
  if (a->n_layers < 1 || a->n_layers > BOZO_TAU_AUX_MAX_LAYERS) return BOZO_ERR_BAD_SHAPE;
  if (a->B <= 0 || a->T <= 0 || a->H <= 0 || a->W <= 0) return BOZO_ERR_BAD_SHAPE;
  if ((long long)a->B * a->T * a->H > 0x7fffffffLL) return BOZO_ERR_UNSUPPORTED;  // rows < 2^31
  if (!dtype_ok(a->dtype)) return BOZO_ERR_BAD_DTYPE;
  for (int i = 0; i < a->n_layers; ++i)
    if (!a->tau[i]) return BOZO_ERR_NULL;
  return BOZO_OK;
}

}  // namespace
}  // namespace bozo

using namespace bozo;

extern "C" {

int bozo_tension_abi_version(void) { return BOZO_TENSION_ABI_VERSION; }

const char* bozo_status_string(int s) {
  switch (s) {
    case BOZO_OK: return "ok";
    case BOZO_ERR_BAD_SHAPE: return "bad shape or size argument";
    case BOZO_ERR_BAD_DTYPE: return "unsupported dtype code";
    case BOZO_ERR_UNSUPPORTED: return "unsupported configuration";
    case BOZO_ERR_ALIGNMENT: return "tensor-core path needs 16-byte aligned rows with unit HD stride";
    case BOZO_ERR_NULL: return "required pointer is NULL";
    case BOZO_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait timed out";
    case BOZO_ERR_CUDA: return "CUDA runtime error";
    case BOZO_ERR_WORKSPACE: return "workspace missing or too small";
    case BOZO_ERR_SCRATCH_LIMIT:
      return "problem needs more than the fixed 8 MiB no-alloc scratch; use bozo_tension_bwd";
    default: return "unknown status";
  }
}

int bozo_tension_last_path(void) { return t_last_path.load(); }
const char* bozo_tension_last_cuda_error(void) {
  return cudaGetErrorName((cudaError_t)t_last_cuda_error.load());
}
int bozo_tension_last_launches(void) { return t_last_launches.load(); }

namespace {

// The fp32-Q/K call (model.py's autocast call site: RoPE-promoted fp32 Q/K,
// bf16 V, fp32 out and τ by the reference's dtype contract) runs on the
// tensor cores from bf16 copies of Q and K.  True when `a` is such a call
// and the band kernel takes it (judged with aligned contiguous stand-ins for
// the copies, which the caller allocates).
bool fwd_wants_lp(const bozo_tension_fwd_args* a) {
  if (!a || a->path == BOZO_PATH_SIMT || a->rope_len != 0 || a->mode != BOZO_MODE_LOCAL) return false;
  if (a->q.dtype != BOZO_DT_F32 || a->k.dtype != BOZO_DT_F32 || a->v.dtype != BOZO_DT_BF16) return false;
  if (a->out_dtype != BOZO_DT_F32 || (a->tau && a->tau_dtype != BOZO_DT_F32)) return false;
  if (a->HD != kTcHD || a->B <= 0 || a->T <= 0 || a->H <= 0) return false;
  FwdP p{};
  p.B = a->B; p.T = a->T; p.H = a->H; p.HD = a->HD; p.mode = a->mode; p.W = a->window;
  p.norm = a->normalize; p.scale = a->scale;
  const long long ob = (long long)a->T * a->H * a->HD, ot = (long long)a->H * a->HD;
  void* const aligned = reinterpret_cast<void*>(uintptr_t(256));
  p.q = DevT4{aligned, BOZO_DT_BF16, ob, ot, a->HD, 1};
  p.k = p.q;
  p.v = dev_t4(a->v);
  p.bias = a->bias;
  p.out = a->out ? a->out : aligned;
  p.out_dt = a->out_dtype;
  p.tau = a->tau;
  p.tau_dt = a->tau_dtype;
  return tc_fwd_eligible(p);
}

}  // namespace

int bozo_tension_fwd_needs_lp(const bozo_tension_fwd_args* a) { return fwd_wants_lp(a) ? 1 : 0; }

int bozo_tension_fwd(const bozo_tension_fwd_args* a, void* stream) {
  if (!a) return BOZO_ERR_NULL;
  int st = check_common(a->B, a->T, a->H, a->HD, a->mode, a->window, a->normalize, a->scale,
                        a->rope_len, a->rope_cos, a->rope_sin);
  if (st) return st;
  if ((st = check_t4(a->q)) || (st = check_t4(a->k)) || (st = check_t4(a->v))) return st;
  if (!a->out) return BOZO_ERR_NULL;
  if (!dtype_ok(a->out_dtype)) return BOZO_ERR_BAD_DTYPE;
  if (a->tau && !dtype_ok(a->tau_dtype)) return BOZO_ERR_BAD_DTYPE;
  if (a->mode == BOZO_MODE_GLOBAL && a->tau && a->window > a->T) return BOZO_ERR_BAD_SHAPE;

  DeviceRestore restore;
  cudaError_t e = bind_device(a->q.ptr, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  FwdP p{};
  p.B = a->B; p.T = a->T; p.H = a->H; p.HD = a->HD; p.mode = a->mode; p.W = a->window;
  p.norm = a->normalize; p.scale = a->scale; p.inv_scale = 1.0f / a->scale;
  p.cos = a->rope_len ? a->rope_cos : nullptr;
  p.sin = a->rope_len ? a->rope_sin : nullptr;
  p.theta = a->rope_len ? a->rope_theta : nullptr;
  p.q = dev_t4(a->q); p.k = dev_t4(a->k); p.v = dev_t4(a->v);
  p.bias = a->bias; p.bs0 = a->bias_stride[0]; p.bs1 = a->bias_stride[1]; p.bs2 = a->bias_stride[2];
  p.out = a->out; p.out_dt = a->out_dtype; p.tau = a->tau; p.tau_dt = a->tau_dtype;
  p.row_mass = a->row_mass;
  p.q_rot = p.cos ? a->q_rot : nullptr;
  p.k_rot = p.cos ? a->k_rot : nullptr;
  p.err = error_word(&e);
  if (!p.err) return cuda_fail(e);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int launches = 0;
  const bool lp_given = a->q_lp && a->k_lp && a->q.dtype == BOZO_DT_F32 && a->k.dtype == BOZO_DT_F32;
  if (lp_given) {
    // bf16 copies of fp32 q / k into the caller's q_lp / k_lp, whichever path
    // runs, so the caller can always hand them to the backward
    if ((reinterpret_cast<uintptr_t>(a->q_lp) | reinterpret_cast<uintptr_t>(a->k_lp)) & 7)
      return BOZO_ERR_ALIGNMENT;
    const int sms = num_sms();
    if ((e = launch_to_bf16(p.q, p.B, p.T, p.H, p.HD, a->q_lp, sms, s)) != cudaSuccess ||
        (e = launch_to_bf16(p.k, p.B, p.T, p.H, p.HD, a->k_lp, sms, s)) != cudaSuccess)
      return cuda_fail(e);
    launches += 2;
  }
  if (lp_given && fwd_wants_lp(a) &&
      ((reinterpret_cast<uintptr_t>(a->q_lp) | reinterpret_cast<uintptr_t>(a->k_lp)) & 15) == 0) {
    // fp32 Q/K: the band kernel on the bf16 copies, fp32 out and τ (without
    // the copies' room the call stays on the exact fp32 path below)
    const long long ob = (long long)p.T * p.H * p.HD, ot = (long long)p.H * p.HD;
    p.q = DevT4{a->q_lp, BOZO_DT_BF16, ob, ot, p.HD, 1};
    p.k = DevT4{a->k_lp, BOZO_DT_BF16, ob, ot, p.HD, 1};
    if (!tc_fwd_eligible(p)) return BOZO_ERR_ALIGNMENT;
    int nl = 0;
    if ((e = launch_tc_fwd(p, s, &nl)) != cudaSuccess) return cuda_fail(e);
    t_last_path = BOZO_PATH_TCGEN05;
    t_last_launches = launches + nl;
    return BOZO_OK;
  }
  // local windows up to 128 keys: the band kernel; global and wider local
  // windows: the key-tile streaming kernel
  const bool band = p.mode == BOZO_MODE_LOCAL && tc_fwd_eligible(p);
  const bool tc_ok = band || tc_global_fwd_eligible(p);
  if (a->path == BOZO_PATH_TCGEN05 && !tc_ok) return BOZO_ERR_ALIGNMENT;
  int path, nl = 0;
  if (tc_ok && a->path != BOZO_PATH_SIMT) {
    e = band ? launch_tc_fwd(p, s, &nl) : launch_tc_global_fwd(p, s, &nl);
    path = BOZO_PATH_TCGEN05;
  } else {
    e = launch_simt_fwd(p, s, &nl);
    // the CUDA-core forward does not stage whole tiles: rotated copies
    // come from a separate elementwise pass
    if (e == cudaSuccess && (p.q_rot || p.k_rot)) e = launch_rope_copy(p, s, &nl);
    path = BOZO_PATH_SIMT;
  }
  if (e != cudaSuccess) return cuda_fail(e);
  t_last_path = path;
  t_last_launches = launches + nl;
  return BOZO_OK;
}

// The workspace every backward needs (coefficient planes, a bf16 copy of an
// fp32 cotangent); the key-tile path's optional dSᵀ scratch follows it.
static size_t bwd_base_bytes(const bozo_tension_bwd_args* a) {
  if (!a || a->B <= 0 || a->T <= 0 || a->H <= 0) return 0;
  // three per-query-row coefficient planes (five with a per-row τ
  // cotangent); rows padded to a multiple of 128 so a 128-row slice starts
  // 16-byte aligned (tensor-core bulk copies)
  const size_t tpad = ((size_t)a->T + 127) / 128 * 128;
  const size_t rows = (size_t)a->B * a->H * tpad;
  size_t bytes = round256(rows * sizeof(float)) * (a->aux_row ? 5 : 3);
  // an fp32 cotangent with bf16 q/k (the fp32-Q call on the tensor cores):
  // room for its bf16 copy
  if (a->d_out.dtype == BOZO_DT_F32 && a->q.dtype == BOZO_DT_BF16 && a->HD > 0)
    bytes += round256((size_t)a->B * a->T * a->H * a->HD * 2);
  return bytes;
}

// The dSᵀ scratch of the key-tile backward (global block, windows > 128,
// bf16 HD 64): with it the dQ pass multiplies stored dSᵀ tiles by K instead
// of recomputing S, dP and the element math.
static size_t bwd_ds_bytes(const bozo_tension_bwd_args* a) {
  if (!a || a->HD != 64 || a->q.dtype != BOZO_DT_BF16 || a->path == BOZO_PATH_SIMT) return 0;
  return round256(tc_global_ds_bytes(a->B, a->T, a->H, a->mode, a->window));
}

size_t bozo_tension_bwd_workspace(const bozo_tension_bwd_args* a) {
  return bwd_base_bytes(a) + bwd_ds_bytes(a);
}

int bozo_tension_bwd(const bozo_tension_bwd_args* a, void* stream) {
  if (!a) return BOZO_ERR_NULL;
  int st = check_common(a->B, a->T, a->H, a->HD, a->mode, a->window, a->normalize, a->scale,
                        a->rope_len, a->rope_cos, a->rope_sin);
  if (st) return st;
  if ((st = check_t4(a->q)) || (st = check_t4(a->k)) || (st = check_t4(a->v)) ||
      (st = check_t4(a->d_out)))
    return st;
  if (a->normalize == BOZO_NORM_MASS) {
    if ((st = check_t4(a->out))) return st;
    if (!a->row_mass) return BOZO_ERR_NULL;
  }
  if (!a->dq || !a->dk || !a->dv) return BOZO_ERR_NULL;
  for (int i = 0; i < 3; ++i)
    if (!dtype_ok(a->grad_dtype[i])) return BOZO_ERR_BAD_DTYPE;
  if (a->d_tau && !dtype_ok(a->d_tau_dtype)) return BOZO_ERR_BAD_DTYPE;
  const size_t need = bwd_base_bytes(a);
  if (need && (!a->workspace || a->workspace_bytes < need)) return BOZO_ERR_WORKSPACE;

  DeviceRestore restore;
  cudaError_t e = bind_device(a->q.ptr, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  BwdP p{};
  p.B = a->B; p.T = a->T; p.H = a->H; p.HD = a->HD; p.mode = a->mode; p.W = a->window;
  p.norm = a->normalize; p.scale = a->scale; p.inv_scale = 1.0f / a->scale;
  p.cos = a->rope_len ? a->rope_cos : nullptr;
  p.sin = a->rope_len ? a->rope_sin : nullptr;
  p.theta = a->rope_len ? a->rope_theta : nullptr;
  p.q = dev_t4(a->q); p.k = dev_t4(a->k); p.v = dev_t4(a->v); p.dout = dev_t4(a->d_out);
  p.out = dev_t4(a->out);
  p.row_mass = a->row_mass;
  p.bias = a->bias; p.bs0 = a->bias_stride[0]; p.bs1 = a->bias_stride[1]; p.bs2 = a->bias_stride[2];
  p.dtau = a->d_tau; p.dtau_dt = a->d_tau_dtype;
  p.dq = a->dq; p.dk = a->dk; p.dv = a->dv;
  p.dq_dt = a->grad_dtype[0]; p.dk_dt = a->grad_dtype[1]; p.dv_dt = a->grad_dtype[2];
  p.qk_rotated = (a->qk_rotated && p.cos) ? 1 : 0;
  p.aux_row = a->aux_row;
  const size_t tpad = ((size_t)a->T + 127) / 128 * 128;
  const size_t rows = (size_t)a->B * a->H * tpad;
  p.alpha = static_cast<float*>(a->workspace);
  p.beta = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + round256(rows * sizeof(float)));
  // the tensor-core path uses the same bytes as three contiguous planes
  p.coef = static_cast<float*>(a->workspace);
  if (a->d_out.dtype == BOZO_DT_F32 && a->q.dtype == BOZO_DT_BF16)
    p.dout_lp = static_cast<char*>(a->workspace) + round256(rows * sizeof(float)) * (a->aux_row ? 5 : 3);
  // the dSᵀ scratch when the caller's workspace holds it (else dQ recomputes)
  const size_t ds = bwd_ds_bytes(a);
  if (ds && a->workspace_bytes >= need + ds) p.ds_scratch = static_cast<char*>(a->workspace) + need;
  p.err = error_word(&e);
  if (!p.err) return cuda_fail(e);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int launches = 0;
  const bool band = p.mode == BOZO_MODE_LOCAL && tc_bwd_eligible(p);
  const bool tc_ok = band || tc_global_bwd_eligible(p);
  if (a->path == BOZO_PATH_TCGEN05 && !tc_ok) return BOZO_ERR_ALIGNMENT;
  // the per-row τ cotangent is formed by the local tensor-core kernel only
  if (a->aux_row && (!band || a->path == BOZO_PATH_SIMT)) return BOZO_ERR_UNSUPPORTED;
  int path;
  if (tc_ok && a->path != BOZO_PATH_SIMT) {
    e = band ? launch_tc_bwd(p, s, &launches) : launch_tc_global_bwd(p, s, &launches);
    path = BOZO_PATH_TCGEN05;
  } else {
    e = launch_simt_bwd(p, s, &launches);
    path = BOZO_PATH_SIMT;
  }
  if (e != cudaSuccess) return cuda_fail(e);
  t_last_path = path;
  t_last_launches = launches;
  return BOZO_OK;
}

int bozo_tension_bwd_noalloc(const bozo_tension_bwd_args* a, void* stream) {
  if (!a) return BOZO_ERR_NULL;
  if (!a->q.ptr) return BOZO_ERR_NULL;
  if (bwd_base_bytes(a) > (size_t)BOZO_NOALLOC_SCRATCH_BYTES)
    return BOZO_ERR_SCRATCH_LIMIT;
  // the scratch address is per device: take it with the data's device current
  DeviceRestore restore;
  cudaError_t e = bind_device(a->q.ptr, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  void* scratch = noalloc_scratch(&e);
  if (!scratch) return cuda_fail(e);
  bozo_tension_bwd_args local = *a;
  local.workspace = scratch;
  local.workspace_bytes = BOZO_NOALLOC_SCRATCH_BYTES;
  return bozo_tension_bwd(&local, stream);
}

size_t bozo_tau_aux_workspace(const bozo_tau_aux_fwd_args* a) {
  if (check_aux(a) != BOZO_OK) return 0;
  const AuxShape s = aux_shape(a->B, a->T, a->H, a->W);
  return round256((size_t)a->n_layers * aux_blocks(s, a->n_layers, num_sms()) * 3 * sizeof(float));
}

int bozo_tau_aux_fwd(const bozo_tau_aux_fwd_args* a, void* stream) {
  int st = check_aux(a);
  if (st) return st;
  if (!a->stats) return BOZO_ERR_NULL;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->tau[0], restore);
  if (e != cudaSuccess) return cuda_fail(e);
  const size_t need = bozo_tau_aux_workspace(a);
  if (!a->workspace || a->workspace_bytes < need) return BOZO_ERR_WORKSPACE;
  const AuxShape s = aux_shape(a->B, a->T, a->H, a->W);
  e = launch_tau_aux_fwd(*a, aux_blocks(s, a->n_layers, num_sms()), static_cast<float*>(a->workspace),
                         static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_tau_aux_bwd(const bozo_tau_aux_bwd_args* a, void* stream) {
  int st = check_aux(a);
  if (st) return st;
  if (!a->d_stats) return BOZO_ERR_NULL;
  // every layer in one mode: all d_tau (cotangent) or all row_coef (row mode)
  const bool rows = a->row_coef[0] != nullptr;
  for (int i = 0; i < a->n_layers; ++i) {
    if (rows ? !a->row_coef[i] : !a->d_tau[i]) return BOZO_ERR_NULL;
    if (rows && a->d_tau[i]) return BOZO_ERR_BAD_SHAPE;
  }
  if (rows && !tau_aux_row_mode_ok(*a)) return BOZO_ERR_UNSUPPORTED;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->tau[0], restore);
  if (e != cudaSuccess) return cuda_fail(e);
  const AuxShape s = aux_shape(a->B, a->T, a->H, a->W);
  e = launch_tau_aux_bwd(*a, aux_blocks(s, a->n_layers, num_sms()), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_tension_decode(const bozo_tension_decode_args* a, void* stream) {
  if (!a) return BOZO_ERR_NULL;
  if (a->B <= 0 || a->H <= 0 || a->HD <= 0 || a->capacity <= 0) return BOZO_ERR_BAD_SHAPE;
  if (a->HD > 128) return BOZO_ERR_UNSUPPORTED;
  if (a->mode != BOZO_MODE_LOCAL && a->mode != BOZO_MODE_GLOBAL) return BOZO_ERR_BAD_SHAPE;
  if (a->mode == BOZO_MODE_LOCAL && (a->window < 1 || a->capacity < a->window + 1))
    return BOZO_ERR_BAD_SHAPE;
  if (a->normalize != BOZO_NORM_NONE && a->normalize != BOZO_NORM_MASS &&
      a->normalize != BOZO_NORM_COUNT)
    return BOZO_ERR_BAD_SHAPE;
  if (!(a->scale != 0.f)) return BOZO_ERR_BAD_SHAPE;
  if (!a->pos || !a->k_cache || !a->v_cache || !a->out) return BOZO_ERR_NULL;
  int st;
  if ((st = check_t4(a->q)) || (st = check_t4(a->k)) || (st = check_t4(a->v))) return st;
  for (int dt : {a->k_cache_dtype, a->v_cache_dtype, a->out_dtype})
    if (!dtype_ok(dt)) return BOZO_ERR_BAD_DTYPE;
  if (a->tau && (!dtype_ok(a->tau_dtype) || a->tau_width < 1)) return BOZO_ERR_BAD_SHAPE;
  if (a->mode == BOZO_MODE_LOCAL && a->tau && a->tau_width != a->window) return BOZO_ERR_BAD_SHAPE;
  if (a->rope_len != 0) {
    if (!a->rope_cos || !a->rope_sin) return BOZO_ERR_NULL;
    if (a->HD % 2 != 0) return BOZO_ERR_UNSUPPORTED;
  }
  DeviceRestore restore;
  cudaError_t e = bind_device(a->q.ptr, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  DecodeP p{};
  p.B = a->B; p.H = a->H; p.HD = a->HD; p.mode = a->mode; p.W = a->window;
  p.norm = a->normalize; p.C = a->capacity; p.tw = a->tau ? a->tau_width : 0;
  p.rope_len = a->rope_len; p.inv_scale = 1.0f / a->scale; p.pos = a->pos;
  p.cos = a->rope_len ? a->rope_cos : nullptr;
  p.sin = a->rope_len ? a->rope_sin : nullptr;
  p.q = dev_t4(a->q); p.k = dev_t4(a->k); p.v = dev_t4(a->v);
  p.kc = a->k_cache; p.kc_dt = a->k_cache_dtype;
  p.vc = a->v_cache; p.vc_dt = a->v_cache_dtype;
  p.out = a->out; p.out_dt = a->out_dtype;
  p.tau = a->tau; p.tau_dt = a->tau_dtype;
  p.err = error_word(&e);
  if (!p.err) return cuda_fail(e);
  if (decode_smem_bytes(p) > 200 * 1024) return BOZO_ERR_UNSUPPORTED;
  e = launch_decode(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e);
  t_last_path = BOZO_PATH_SIMT;
  t_last_launches = 1;
  return BOZO_OK;
}

int bozo_graph_bias_build(const bozo_graph_bias_args* a, void* stream) {
  if (!a) return BOZO_ERR_NULL;
  if (a->T <= 0 || a->window < 0 || a->n_edges < 0) return BOZO_ERR_BAD_SHAPE;
  if (!a->ctx_content || !a->out || (a->n_edges > 0 && (!a->edge_keys || !a->edge_weights)))
    return BOZO_ERR_NULL;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->out, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  e = launch_graph_bias(*a, num_sms(), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

static int check_norm(const bozo_add_rmsnorm_args* a) {
  if (!a) return BOZO_ERR_NULL;
  if (a->rows <= 0 || a->width <= 0) return BOZO_ERR_BAD_SHAPE;
  if (!norm_width_ok(a->width)) return BOZO_ERR_UNSUPPORTED;
  if (a->x_dtype != BOZO_DT_F32 && a->x_dtype != BOZO_DT_BF16) return BOZO_ERR_BAD_DTYPE;
  if (a->y && a->y_dtype != BOZO_DT_F32 && a->y_dtype != BOZO_DT_BF16) return BOZO_ERR_BAD_DTYPE;
  if (a->y && a->x_dtype == BOZO_DT_BF16 && a->y_dtype != BOZO_DT_BF16) return BOZO_ERR_UNSUPPORTED;
  if ((a->out_lp || a->d_out_lp) && a->x_dtype != BOZO_DT_F32) return BOZO_ERR_UNSUPPORTED;
  if (!a->x || !a->scale || !a->rstd) return BOZO_ERR_NULL;
  return BOZO_OK;
}

static NormP norm_params(const bozo_add_rmsnorm_args* a) {
  NormP p{};
  p.N = a->rows; p.D = a->width; p.eps = a->eps; p.sms = num_sms();
  p.x = a->x; p.x_dt = a->x_dtype; p.y = a->y; p.y_dt = a->y_dtype; p.scale = a->scale;
  p.out = a->out; p.rstd = a->rstd; p.dout = a->d_out; p.dx = a->dx; p.dy = a->dy;
  p.dscale = a->d_scale; p.part = static_cast<float*>(a->workspace);
  p.out_lp = a->out_lp; p.dout_lp = a->d_out_lp;
  return p;
}

size_t bozo_add_rmsnorm_workspace(const bozo_add_rmsnorm_args* a) {
  if (!a || a->rows <= 0 || a->width <= 0) return 0;
  return round256((size_t)norm_partial_blocks(a->rows, num_sms()) * a->width * sizeof(float));
}

int bozo_add_rmsnorm_fwd(const bozo_add_rmsnorm_args* a, void* stream) {
  int st = check_norm(a);
  if (st) return st;
  if (!a->out) return BOZO_ERR_NULL;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->x, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  e = launch_add_rmsnorm(norm_params(a), false, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_add_rmsnorm_bwd(const bozo_add_rmsnorm_args* a, void* stream) {
  int st = check_norm(a);
  if (st) return st;
  if (!a->d_out || !a->dx || !a->d_scale || (a->y && !a->dy)) return BOZO_ERR_NULL;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->x, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  if (!a->workspace || a->workspace_bytes < bozo_add_rmsnorm_workspace(a)) return BOZO_ERR_WORKSPACE;
  e = launch_add_rmsnorm(norm_params(a), true, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_wo_add_rmsnorm_fwd(const bozo_wo_add_rmsnorm_args* a, void* stream) {
  if (!a) return BOZO_ERR_NULL;
  if (a->rows <= 0 || a->width <= 0) return BOZO_ERR_BAD_SHAPE;
  if (a->x_dtype != BOZO_DT_F32 && a->x_dtype != BOZO_DT_BF16) return BOZO_ERR_BAD_DTYPE;
  if (!wo_norm_cluster(a->width, a->x_dtype == BOZO_DT_BF16)) return BOZO_ERR_UNSUPPORTED;
  if (!a->msg || !a->wo || !a->x || !a->scale || !a->out) return BOZO_ERR_NULL;
  const void* ptrs[5] = {a->msg, a->wo, a->x, a->out, a->scale};
  for (const void* ptr : ptrs)
    if (reinterpret_cast<uintptr_t>(ptr) & 15) return BOZO_ERR_ALIGNMENT;
  if (!tmap_encoder_available()) return BOZO_ERR_UNSUPPORTED;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->x, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  int* err = error_word(&e);
  if (!err) return cuda_fail(e);
  e = launch_wo_norm(*a, err, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_wo_add_rmsnorm_supported(int32_t width, int32_t x_dtype) {
  if (x_dtype != BOZO_DT_F32 && x_dtype != BOZO_DT_BF16) return 0;
  return wo_norm_cluster(width, x_dtype == BOZO_DT_BF16) ? 1 : 0;
}

static int check_swiglu(const bozo_swiglu_args* a) {
  if (!a) return BOZO_ERR_NULL;
  if (a->n <= 0 || a->n % 4 != 0) return BOZO_ERR_BAD_SHAPE;
  if (a->dtype != BOZO_DT_F32 && a->dtype != BOZO_DT_BF16) return BOZO_ERR_BAD_DTYPE;
  if (a->width < 0 || a->width % 4 != 0 || a->width > 0x7fffffff) return BOZO_ERR_BAD_SHAPE;
  if (a->width > 0 && (a->n % a->width != 0 || a->row_stride < a->width || a->row_stride % 4 != 0))
    return BOZO_ERR_BAD_SHAPE;
  if (!a->gate || !a->value) return BOZO_ERR_NULL;
  return BOZO_OK;
}

int bozo_swiglu_fwd(const bozo_swiglu_args* a, void* stream) {
  int st = check_swiglu(a);
  if (st) return st;
  if (!a->out) return BOZO_ERR_NULL;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->gate, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  e = launch_swiglu(a->gate, a->value, a->out, nullptr, nullptr, nullptr, a->n, (int)a->width,
                    a->row_stride, a->dtype, num_sms(), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_swiglu_bwd(const bozo_swiglu_args* a, void* stream) {
  int st = check_swiglu(a);
  if (st) return st;
  if (!a->d_out || !a->d_gate || !a->d_value) return BOZO_ERR_NULL;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->gate, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  e = launch_swiglu(a->gate, a->value, nullptr, a->d_out, a->d_gate, a->d_value, a->n, (int)a->width,
                    a->row_stride, a->dtype, num_sms(), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_embedding_bwd(const bozo_embedding_bwd_args* a, void* stream) {
  if (!a) return BOZO_ERR_NULL;
  if (a->n <= 0 || a->n > 0x7fffffffLL || a->vocab <= 0 || a->dim <= 0 || a->dim % 4 != 0)
    return BOZO_ERR_BAD_SHAPE;
  if (!a->sorted_ids || !a->order || !a->d_out || !a->d_weight || !a->scratch) return BOZO_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(a->d_out) & 15) || (reinterpret_cast<uintptr_t>(a->d_weight) & 15))
    return BOZO_ERR_ALIGNMENT;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->d_out, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  e = launch_embedding_bwd(*a, num_sms(), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

static int check_xent(const bozo_cross_entropy_args* a) {
  if (!a) return BOZO_ERR_NULL;
  if (a->rows <= 0 || a->rows > 0x7fffffffLL) return BOZO_ERR_BAD_SHAPE;
  if (a->logits_dtype != BOZO_DT_F32 && a->logits_dtype != BOZO_DT_BF16) return BOZO_ERR_BAD_DTYPE;
  if (!xent_shape_ok(a->vocab, a->logits_dtype)) return BOZO_ERR_UNSUPPORTED;
  if (!a->logits || !a->targets || !a->row_lse) return BOZO_ERR_NULL;
  return BOZO_OK;
}

int bozo_cross_entropy_fwd(const bozo_cross_entropy_args* a, void* stream) {
  int st = check_xent(a);
  if (st) return st;
  if (!a->row_loss) return BOZO_ERR_NULL;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->logits, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  e = launch_xent(*a, false, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_cross_entropy_bwd(const bozo_cross_entropy_args* a, void* stream) {
  int st = check_xent(a);
  if (st) return st;
  if (!a->d_scale || !a->d_logits) return BOZO_ERR_NULL;
  DeviceRestore restore;
  cudaError_t e = bind_device(a->logits, restore);
  if (e != cudaSuccess) return cuda_fail(e);
  e = launch_xent(*a, true, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_tension_wait_selftest(uint64_t limit_ns, int32_t* result, void* stream) {
  if (limit_ns < 1000ull || limit_ns > 1000000000ull) return BOZO_ERR_BAD_SHAPE;
  DeviceRestore restore;
  cudaError_t e = cudaSuccess;
  if (result && (e = bind_device(result, restore)) != cudaSuccess) return cuda_fail(e);
  int* err = error_word(&e);
  if (!err) return cuda_fail(e);
  e = launch_wait_selftest(limit_ns, err, result, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_tension_error_async(int32_t* host_dst, void* stream) {
  if (!host_dst) return BOZO_ERR_NULL;
  cudaError_t e = cudaSuccess;
  int* err = error_word(&e);
  if (!err) return cuda_fail(e);
  e = cudaMemcpyAsync(host_dst, err, sizeof(int), cudaMemcpyDeviceToHost,
                      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BOZO_OK : cuda_fail(e);
}

int bozo_tension_poll_error(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return BOZO_ERR_CUDA;
  int* ptr = error_word(&e);
  if (!ptr) return BOZO_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, ptr, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return BOZO_ERR_CUDA;
  if (v) {
    const int zero = 0;
    if (cudaMemcpy(ptr, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return BOZO_ERR_CUDA;
    return BOZO_ERR_DEVICE_TIMEOUT;
  }
  return BOZO_OK;
}

}  // extern "C"
