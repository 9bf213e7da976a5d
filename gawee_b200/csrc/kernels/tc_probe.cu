// gawee_probe_tf32_mma: the tensor cores' TF32 rate on this device, measured.
//
// One CTA per SM issues back-to-back tcgen05.mma.kind::tf32 instructions of
// M = 128, N = 128, K = 8 (both operands in shared memory, one accumulator in
// tensor memory) from a single thread, the shape and operand kinds the
// contraction kernels use; the launch is timed with CUDA events.  The fp32
// path issues three such products per multiply-add, so a third of this rate
// is its tensor ceiling.  Every wait is bounded: on expiry the kernel records
// ST_BARRIER_TIMEOUT in the status word and returns.

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "gawee_cuda.h"
#include "kernels.h"
#include "tc_common.cuh"

namespace gawee {
void set_thread_error(const std::string& msg);
namespace kern {
namespace {

constexpr int kProbeThreads = 128;
constexpr int kProbeSmem = 32 * 1024 + 1024;  // A and B tiles (16 KB each) + alignment

__global__ void __launch_bounds__(kProbeThreads, 1) tf32_mma_probe_kernel(int iters, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint32_t tmem_slot;
  __shared__ __align__(8) uint64_t done;
  __shared__ int abort_flag;
  for (int i = threadIdx.x; i < 32 * 1024 / 4; i += kProbeThreads) reinterpret_cast<float*>(smem)[i] = 0.0f;
  const int warp = threadIdx.x / 32;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(smem_u32(&tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&done), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the zeroed tiles, for the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    const uint64_t da = umma_desc_sw128(smem_u32(smem));
    const uint64_t db = umma_desc_sw128(smem_u32(smem + 16 * 1024));
    const uint32_t idesc = umma_idesc_tf32<128>();
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
            "l"(da + 2 * kk), "l"(db + 2 * kk), "r"(idesc), "r"((uint32_t)((it | kk) != 0))
            : "memory");
      }
    }
    umma_commit(smem_u32(&done));
    mbar_wait(smem_u32(&done), 0, &abort_flag, status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tmem) : "memory");
  }
}

}  // namespace
}  // namespace kern
}  // namespace gawee

extern "C" gawee_status gawee_probe_tf32_mma(int device, double* tflops) {
  using namespace gawee::kern;
  if (!tflops) return GAWEE_ERR_INVALID;
  *tflops = 0.0;
  auto fail = [](const char* what, cudaError_t e) {
    gawee::set_thread_error(std::string("gawee_probe_tf32_mma: ") + what + ": " + cudaGetErrorString(e));
    return GAWEE_ERR_CUDA;
  };
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail("cudaSetDevice", e);
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (sms <= 0) return fail("SM count", cudaErrorInvalidDevice);
  e = cudaFuncSetAttribute(tf32_mma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeSmem);
  if (e != cudaSuccess) return fail("cudaFuncSetAttribute", e);
  int* status = nullptr;
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  if ((e = cudaMalloc(&status, sizeof(int))) != cudaSuccess) return fail("cudaMalloc", e);
  gawee_status st = GAWEE_OK;
  const int iters = 8192;  // 32768 MMAs per SM: about a millisecond
  do {
    if ((e = cudaMemset(status, 0, sizeof(int))) != cudaSuccess) { st = fail("cudaMemset", e); break; }
    if ((e = cudaEventCreate(&t0)) != cudaSuccess || (e = cudaEventCreate(&t1)) != cudaSuccess) {
      st = fail("cudaEventCreate", e);
      break;
    }
    float best = 0.0f;
    for (int rep = 0; rep < 4; ++rep) {  // the first launch warms up; keep the fastest
      cudaEventRecord(t0, 0);
      tf32_mma_probe_kernel<<<sms, kProbeThreads, kProbeSmem, 0>>>(iters, status);
      cudaEventRecord(t1, 0);
      if ((e = cudaEventSynchronize(t1)) != cudaSuccess) { st = fail("probe launch", e); break; }
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, t0, t1);
      if (rep > 0 && (best == 0.0f || ms < best)) best = ms;
    }
    if (st != GAWEE_OK) break;
    int h = 0;
    if ((e = cudaMemcpy(&h, status, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess) {
      st = fail("cudaMemcpy", e);
      break;
    }
    if (h != 0) {
      gawee::set_thread_error("gawee_probe_tf32_mma: a wait in the probe kernel timed out");
      st = GAWEE_ERR_DEVICE;
      break;
    }
    const double flops = 2.0 * 128 * 128 * 8 * 4.0 * iters * sms;
    *tflops = best > 0.0f ? flops / (best * 1e-3) / 1e12 : 0.0;
  } while (false);
  if (t0) cudaEventDestroy(t0);
  if (t1) cudaEventDestroy(t1);
  cudaFree(status);
  return st;
}
