// wait_selftest.cu — a kernel that makes one bounded mbarrier wait run out on
// purpose, so a test can check the timeout path of the tensor-core kernels
// without hanging or faulting a GPU.
//
// One CTA of two warps: warp 0 allocates TMEM; its lane 0 starts a bulk copy
// into shared memory and one tcgen05 MMA (zero operands) into that TMEM, then
// waits with a short limit on an mbarrier that nothing ever arrives on.  The
// wait gives up through the same polling loop as every tensor-core kernel
// (mbar_wait_until), records its code in the device error word, and — with
// its limit far shorter than the kernels' 4 s — drains the copy and the MMA
// with bounded waits (drain_loads / drain_mma) before the TMEM is released
// and the CTA exits.  The optional result words say what
// happened: [0] the wait gave up, [1] the copy drained, [2] the MMA drained,
// [3] microseconds the wait took before it gave up.
#include "tc.cuh"
#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace bozo {
namespace {

using namespace tc;

constexpr int kErrSelftest = 0x400;
constexpr int kATile = 128 * 128;  // A: 128 rows × 64 bf16 (SW128), 16 KiB
constexpr int kBTile = 64 * 128;   // B: 64 rows × 64 bf16 (SW128), 8 KiB
constexpr int kCopy = 4096;        // bulk-copied bytes

// source of the bulk copy (zeros; 16-byte aligned as cp.async.bulk requires)
__device__ __align__(128) unsigned char g_selftest_src[kCopy];

__global__ void __launch_bounds__(64, 1)
    wait_selftest_kernel(uint64_t limit_ns, int* err, int* result) {
  __shared__ __align__(1024) uint8_t sA[kATile];
  __shared__ __align__(1024) uint8_t sB[kBTile];
  __shared__ __align__(16) uint8_t sCopy[kCopy];
  __shared__ __align__(8) uint64_t bars[3];  // [0] nothing arrives, [1] the copy, [2] MMA drain
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < (kATile + kBTile) / 16; i += blockDim.x) {
    uint4* dst = i < kATile / 16 ? reinterpret_cast<uint4*>(sA) + i
                                 : reinterpret_cast<uint4*>(sB) + (i - kATile / 16);
    *dst = make_uint4(0, 0, 0, 0);
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 64);
    tmem_relinquish();
  }
  fence_proxy_async_smem();  // the zeroed operands are read by the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bars[1], kCopy);
    bulk_load_1d(sCopy, g_selftest_src, kCopy, &bars[1]);
    const uint64_t da = sdesc_sw128(smem_u32(sA), 16, 1024);
    const uint64_t db = sdesc_sw128(smem_u32(sB), 16, 1024);
    mma_bf16(tmem_base, da, db, idesc_bf16(128, 64, false, false), 0u);
    const uint64_t t0 = globaltimer_ns();
    const bool done = mbar_wait_until(&bars[0], 0u, err, kErrSelftest | 1, limit_ns);
    const uint64_t waited = globaltimer_ns() - t0;
    // the exit path of every tensor-core kernel: nothing async left in flight
    drain_loads(&bars[1], 1, 1, err, kErrSelftest | 2);
    const bool copy_ok = mbar_test(&bars[1], 0u);
    drain_mma(&bars[2], err, kErrSelftest | 3);
    const bool mma_ok = mbar_test(&bars[2], 0u);
    if (result) {
      result[0] = done ? 0 : 1;
      result[1] = copy_ok ? 1 : 0;
      result[2] = mma_ok ? 1 : 0;
      result[3] = waited / 1000u > 0x7fffffffull ? 0x7fffffff : (int)(waited / 1000u);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 64);
  }
}

}  // namespace

cudaError_t launch_wait_selftest(uint64_t limit_ns, int* err, int* result, cudaStream_t st) {
  wait_selftest_kernel<<<1, 64, 0, st>>>(limit_ns, err, result);
  return cudaGetLastError();
}

}  // namespace bozo
