// tc_host.cu — TMA tensor-map construction (driver entry point fetched
// through the runtime, so the library needs no link-time libcuda).
#include <cudaTypedefs.h>

#include "tc_host.cuh"

namespace bozo {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

}  // namespace

bool tmap_encoder_available() { return get_encode() != nullptr; }

bool tma_view_ok(const DevT4& x, int B, int T, int H) {
  if (x.dt != BOZO_DT_BF16 || x.sd != 1) return false;
  if ((reinterpret_cast<uintptr_t>(x.p) & 15) != 0) return false;
  const long long s[3] = {x.sh, x.st, x.sb};
  const int n[3] = {H, T, B};
  for (int i = 0; i < 3; ++i)
    if (n[i] > 1 && (s[i] <= 0 || s[i] % 8 != 0 || s[i] >= (1ll << 38))) return false;
  if (H > 1 && x.sh < kTcHD) return false;
  return true;
}

bool make_tmap_bthd(CUtensorMap* m, const void* base, long long sb, long long st, long long sh,
                    int B, int T, int H, int box_t) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)kTcHD, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  // a size-1 dimension is never stepped: give it a harmless 16-byte-multiple stride
  const long long h_ = H > 1 ? sh : kTcHD, t_ = T > 1 ? st : 8, b_ = B > 1 ? sb : 8;
  cuuint64_t strides[3] = {(cuuint64_t)h_ * 2, (cuuint64_t)t_ * 2, (cuuint64_t)b_ * 2};
  cuuint32_t box[4] = {(cuuint32_t)kTcHD, 1, (cuuint32_t)box_t, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_2d(CUtensorMap* m, const void* base, bool f32, uint64_t inner, uint64_t outer,
                  uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(outer > 1 ? row_bytes : 16)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box,
                   es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return n;
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

}  // namespace bozo
