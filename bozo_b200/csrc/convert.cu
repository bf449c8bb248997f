// convert.cu — fp32 → bf16 operand copies for the tensor-core kernels.
//
// model.py's autocast call (model.py:200-204, 248-264) hands the operator
// fp32 Q/K (RoPE multiplies the bf16 projections by fp32 tables) and, in the
// backward, an fp32 cotangent of the fp32 output.  The tcgen05 kernels take
// bf16 tiles, so these tensors are copied to contiguous bf16 [B,T,H,HD] once
// per call: 16 bytes in / 8 bytes out per thread and step when the rows are
// unit-stride with HD a multiple of 4, element by element otherwise.
#include <algorithm>

#include "common.cuh"

namespace bozo {
namespace {

__global__ void to_bf16_vec4(const float* __restrict__ src, long long sb, long long st,
                             long long sh, int T, int H, int HD, long long n4,
                             __nv_bfloat16* __restrict__ dst) {
  const int q4 = HD / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    long long r = i / q4;
    const int c = (int)(i - r * q4) * 4;
    const int h = (int)(r % H);
    r /= H;
    const int t = (int)(r % T);
    const long long b = r / T;
    const float4 x = __ldg(reinterpret_cast<const float4*>(src + b * sb + t * st + h * sh + c));
    __nv_bfloat162 lo = __floats2bfloat162_rn(x.x, x.y), hi = __floats2bfloat162_rn(x.z, x.w);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&lo);
    w.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst + i * 4) = w;
  }
}

__global__ void to_bf16_any(DevT4 src, int T, int H, int HD, long long n,
                            __nv_bfloat16* __restrict__ dst) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    long long r = i / HD;
    const int d = (int)(i - r * HD);
    const int h = (int)(r % H);
    r /= H;
    const int t = (int)(r % T);
    const long long b = r / T;
    dst[i] = __float2bfloat16_rn(ldf(src.p, b * src.sb + t * src.st + h * src.sh + d * src.sd, src.dt));
  }
}

}  // namespace

cudaError_t launch_to_bf16(const DevT4& src, int B, int T, int H, int HD, void* dst, int sms,
                           cudaStream_t st) {
  const long long n = (long long)B * T * H * HD;
  auto* out = static_cast<__nv_bfloat16*>(dst);
  const bool vec = src.dt == BOZO_DT_F32 && src.sd == 1 && HD % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(src.p) & 15) == 0 && src.sb % 4 == 0 &&
                   src.st % 4 == 0 && src.sh % 4 == 0 && (reinterpret_cast<uintptr_t>(dst) & 7) == 0;
  const int threads = 256;
  if (vec) {
    const long long n4 = n / 4;
    const int grid = (int)std::min<long long>((n4 + threads - 1) / threads, (long long)sms * 8);
    to_bf16_vec4<<<grid, threads, 0, st>>>(static_cast<const float*>(src.p), src.sb, src.st, src.sh,
                                            T, H, HD, n4, out);
  } else {
    const int grid = (int)std::min<long long>((n + threads - 1) / threads, (long long)sms * 8);
    to_bf16_any<<<grid, threads, 0, st>>>(src, T, H, HD, n, out);
  }
  return cudaGetLastError();
}

}  // namespace bozo
