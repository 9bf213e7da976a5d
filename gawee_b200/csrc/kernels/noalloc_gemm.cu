// gawee_matmul_f32_noalloc: an fp32 matrix product on the tensor-core kernel
// that allocates no memory.
//
// The regular path (gawee_create + gawee_forward) allocates its buffers once,
// when the graph is planned.  Some callers cannot allocate device memory at
// the point they need a product: a host framework whose caching allocator
// owns the device memory and forbids allocations behind its back (a
// cudaMalloc there can fail, or fragment the pool the framework manages), a
// caller holding a fixed memory budget, or code on an error-recovery path
// after an allocation already failed.  cudaMalloc and cudaFree can also wait
// for the whole device, which a latency-sensitive caller cannot accept in
// the middle of its work.  They pass their own A, B and C; the only extra
// memory the product needs — the split-precision TF32 planes of B that the
// tensor cores read through TMA — lives in the file-scope array below, which
// the CUDA runtime creates when it loads this library on a device, next to a
// status word that the kernel's bounded waits report into.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../../include/gawee_cuda.h"
#include "kernels.h"

namespace gawee {
void set_thread_error(const std::string& msg);  // runtime.cpp: read back by gawee_last_error(NULL, ...)
}

namespace {

// 16 MiB per device: the hi and lo planes of B, n * round_up(k, 4) floats each.
constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr size_t kScratchFloats = kScratchBytes / sizeof(float);
__device__ __align__(256) float g_noalloc_scratch[kScratchFloats];
// First error a kernel of this entry point reported (kern::Status), read and
// cleared by gawee_synchronize(NULL, stream).  Shared by every call, like the
// scratch.
__device__ int g_noalloc_status;

constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct DeviceStatics {
  float* scratch = nullptr;
  int* status = nullptr;
};
DeviceStatics g_statics[kMaxDevices];

// Device addresses of the scratch array and the status word on the current
// device.  Their names are only host-side stand-ins in host code; the
// addresses come from cudaGetSymbolAddress, once per device, with that device
// current.
gawee_status statics_for_current_device(DeviceStatics* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    gawee::set_thread_error(std::string("gawee_matmul_f32_noalloc: cudaGetDevice: ") +
                            (e != cudaSuccess ? cudaGetErrorString(e) : "device index out of range"));
    return GAWEE_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceStatics& d = g_statics[dev];
  if (!d.scratch) {
    void* p = nullptr;
    void* q = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&q, g_noalloc_status);
    if (e != cudaSuccess || !p || !q) {
      gawee::set_thread_error(std::string("gawee_matmul_f32_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      return GAWEE_ERR_CUDA;
    }
    d.status = static_cast<int*>(q);
    d.scratch = static_cast<float*>(p);
  }
  *out = d;
  return GAWEE_OK;
}

}  // namespace

namespace gawee {
// gawee_synchronize(NULL, stream): waits for `stream`, then reads and clears
// the status word on the current device (no allocation: a pageable 4-byte
// copy and a memset on the caller's stream).  Returns the kern::Status code
// (0 = no error), or -1 with the thread's error message set on a CUDA failure.
int noalloc_take_status(cudaStream_t s) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  int* status = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    status = g_statics[dev].status;
  }
  cudaError_t e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && !status) return 0;  // no call of the entry point on this device yet
  int v = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&v, status, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && v != 0) e = cudaMemsetAsync(status, 0, sizeof(int), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_thread_error(std::string("gawee_synchronize: ") + cudaGetErrorString(e));
    return -1;
  }
  return v;
}
}  // namespace gawee

extern "C" gawee_status gawee_matmul_f32_noalloc(const float* a, const float* b, float* c, int64_t m, int64_t n,
                                                 int64_t k, void* stream) {
  using namespace gawee::kern;
  if (!a || !b || !c || m <= 0 || n <= 0 || k <= 0) {
    gawee::set_thread_error("gawee_matmul_f32_noalloc: null pointer or empty shape");
    return GAWEE_ERR_INVALID;
  }
  if (k % 4 != 0 || (reinterpret_cast<uintptr_t>(a) & 15) != 0) {
    gawee::set_thread_error("gawee_matmul_f32_noalloc: k must be a multiple of 4 and a 16-byte aligned");
    return GAWEE_ERR_INVALID;
  }
  const int64_t ldk = k;  // multiple of 4
  if (n > (int64_t)(kScratchFloats / 2) / ldk) {
    gawee::set_thread_error("gawee_matmul_f32_noalloc: n * k = " + std::to_string(n * k) + " exceeds the " +
                            std::to_string(kScratchFloats / 2) + " elements of the 16 MiB scratch (2 planes)");
    return GAWEE_ERR_INVALID;
  }
  DeviceStatics d;
  if (gawee_status st = statics_for_current_device(&d)) return st;
  float* hi = d.scratch;
  float* lo = d.scratch + n * ldk;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // B [k][n] row-major -> planes [n][ldk]; every element of both planes is
  // written (zeros past k), so nothing from an earlier call survives.
  PackBParams pp{};
  pp.src = b;
  pp.hi = hi;
  pp.lo = lo;
  pp.batch = 1;
  pp.K = k;
  pp.N = n;
  pp.ldk = ldk;
  pp.sn = 1;
  pp.k_rank = 1;
  pp.k_shape[0] = k;
  pp.k_st[0] = n;
  pp.k_valid[0] = k;
  pp.batch_rank = 0;
  launch_pack_b(pp, s);

  const int block_n = n <= 64 ? 64 : 128;
  alignas(64) unsigned char tm[2][128];
  if (!make_b_tensor_maps(hi, lo, 1, n, ldk, block_n, tm[0], tm[1])) {
    gawee::set_thread_error("gawee_matmul_f32_noalloc: cuTensorMapEncodeTiled failed");
    return GAWEE_ERR_CUDA;
  }
  ConvGemmParams p{};
  p.x = a;
  p.x_sn = 0;
  p.x_sh = m > 1 ? k : 0;
  p.x_sw = 0;
  p.H = m;
  p.W = 1;
  p.C = k;
  p.P = m;
  p.Q = 1;
  p.R = p.S = 1;
  p.sh = p.sw = 1;
  p.ph = p.pw = 0;
  p.dh = p.dw = 1;
  p.M = m;
  p.N = n;
  p.K = k;
  p.nb = 1;
  p.batch_rank = 0;
  p.out = c;
  p.ldc = n;
  p.ldc_n = 1;
  p.epi = EPI_NONE;
  p.status = d.status;  // a bounded wait that gives up records ST_BARRIER_TIMEOUT here
  if (!launch_conv_gemm_tc(p, tm[0], tm[1], block_n, s)) {
    gawee::set_thread_error("gawee_matmul_f32_noalloc: the tensor-core kernel rejected the shape");
    return GAWEE_ERR_UNSUPPORTED;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    gawee::set_thread_error(std::string("gawee_matmul_f32_noalloc: launch: ") + cudaGetErrorString(e));
    return GAWEE_ERR_CUDA;
  }
  return GAWEE_OK;
}
