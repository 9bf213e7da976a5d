// Memory-bound kernels of the gawee CUDA runtime: strided elementwise programs,
// reductions, softmax, gather, index remaps, pooling, top-k and the packing of
// tensor-core B operands.  Grids are sized as multiples of the SM count and
// use grid-stride loops.
#include <cuda_bf16.h>

#include <algorithm>
#include <cfloat>
#include <cstdio>

#include "kernels.h"
#include "program.cuh"

namespace gawee {
namespace kern {

namespace {

constexpr int kThreads = 256;

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// One wave of the blocks that fit on the SMs at once (a grid-stride kernel
// then has no partial last wave), or fewer when the work is smaller.
template <auto Kernel>
unsigned resident_grid(int64_t work) {
  static const int per_sm = [] {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, Kernel, kThreads, 0) != cudaSuccess || n < 1) n = 1;
    return n;
  }();
  int64_t g = (work + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)sm_count() * per_sm;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

unsigned grid_for(int64_t work, int per_block = kThreads, int waves = 8) {
  int64_t g = (work + per_block - 1) / per_block;
  int64_t cap = (int64_t)sm_count() * waves;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

__device__ __forceinline__ void set_status(int* st, int code) {
  if (st) atomicCAS(st, 0, code);
}

}  // namespace

// ---------------------------------------------------------------------------
// Elementwise: one program run per output element; operands addressed through
// per-dimension strides over the iteration space (0 = broadcast).
// ---------------------------------------------------------------------------
// Evaluates a recognised f32 program (EwParams::fast) on operand values v.
template <int N>
__device__ __forceinline__ float eval_fast(const EwParams& p, const float (&v)[kMaxIn][N], int e) {
  switch (p.fast) {
    case EW_COPY: return v[0][e];
    case EW_SQR: return __fmul_rn(v[0][e], v[0][e]);
    case EW_NEG: return -v[0][e];
    case EW_ADDC_SQRT: return __fsqrt_rn(__fadd_rn(v[0][e], p.fk));
    case EW_DIV_MUL: return __fmul_rn(__fdiv_rn(v[0][e], v[1][e]), v[2][e]);
    default: return __fadd_rn(__fmul_rn(v[0][e], v[1][e]), __fmul_rn(v[2][e], v[3][e]));
  }
}

__global__ void __launch_bounds__(kThreads) elementwise_kernel(const __grid_constant__ EwParams p) {
  Reg regs[kMaxRegs];
  int err = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < p.numel; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i;
    int64_t off_out = 0;
    int64_t off_in[kMaxIn];
#pragma unroll
    for (int k = 0; k < kMaxIn; ++k) off_in[k] = 0;
    for (int d = p.rank - 1; d >= 0; --d) {
      int64_t c = rem % p.shape[d];
      rem /= p.shape[d];
      off_out += c * p.out.st[d];
#pragma unroll
      for (int k = 0; k < kMaxIn; ++k)
        if (k < p.n_in) off_in[k] += c * p.in[k].st[d];
    }
#pragma unroll
    for (int k = 0; k < kMaxIn; ++k)
      if (k < p.n_in) regs[k] = load_dt(p.in[k].ptr, off_in[k], p.in[k].dt);
    Reg r = run_program(p.prog, regs, &err);
    store_dt(p.out.ptr, off_out, p.out.dt, r);
  }
  if (err) set_status(p.status, err);
}

// Contiguous float fast path: all operands f32 with identical dense layout or
// scalar broadcast, processed four elements at a time.
__global__ void __launch_bounds__(kThreads) elementwise_dense4_kernel(const __grid_constant__ EwParams p,
                                                                      unsigned scalar_mask) {
  Reg regs[kMaxRegs];
  int err = 0;
  const int64_t n4 = p.numel / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 v[kMaxIn];
#pragma unroll
    for (int k = 0; k < kMaxIn; ++k) {
      if (k < p.n_in) {
        if (scalar_mask & (1u << k)) {
          float s = static_cast<const float*>(p.in[k].ptr)[0];
          v[k] = make_float4(s, s, s, s);
        } else {
          v[k] = reinterpret_cast<const float4*>(p.in[k].ptr)[i];
        }
      }
    }
    float4 o;
    float* op = reinterpret_cast<float*>(&o);
    if (p.fast != EW_INTERP) {
      float w[kMaxIn][4];
#pragma unroll
      for (int k = 0; k < kMaxIn; ++k) {
        w[k][0] = v[k].x;
        w[k][1] = v[k].y;
        w[k][2] = v[k].z;
        w[k][3] = v[k].w;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) op[e] = eval_fast(p, w, e);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
#pragma unroll
        for (int k = 0; k < kMaxIn; ++k)
          if (k < p.n_in) regs[k].f = reinterpret_cast<float*>(&v[k])[e];
        op[e] = run_program(p.prog, regs, &err).f;
      }
    }
    reinterpret_cast<float4*>(p.out.ptr)[i] = o;
  }
  // tail
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < p.numel;
       i += (int64_t)gridDim.x * blockDim.x) {
#pragma unroll
    for (int k = 0; k < kMaxIn; ++k)
      if (k < p.n_in) regs[k].f = static_cast<const float*>(p.in[k].ptr)[(scalar_mask & (1u << k)) ? 0 : i];
    static_cast<float*>(p.out.ptr)[i] = run_program(p.prog, regs, &err).f;
  }
  if (err) set_status(p.status, err);
}

// All-f32 operands, output rows contiguous: each thread takes a run of four
// consecutive elements of one row (coordinates unravelled once per run),
// loads each operand as a float4 when its inner stride is 1 (and aligned),
// broadcasts it when the stride is 0, and stores a float4.
// Idx: type of the run index and coordinates (32-bit when the iteration
// space has < 2^31 elements: its divisions cost a fraction of 64-bit ones).
template <typename Idx>
__global__ void __launch_bounds__(kThreads) elementwise_rows4_kernel(const __grid_constant__ EwParams p,
                                                                     unsigned vec_mask, unsigned bcast_mask,
                                                                     int64_t rows, int64_t cols) {
  Reg regs[kMaxRegs];
  int err = 0;
  const Idx runs_per_row = (Idx)((cols + 3) / 4);
  const Idx runs = (Idx)rows * runs_per_row;
  const int inner = p.rank - 1;
  for (Idx u = blockIdx.x * (Idx)blockDim.x + threadIdx.x; u < runs; u += (Idx)gridDim.x * blockDim.x) {
    const Idx row = u / runs_per_row;
    const int64_t c0 = (int64_t)(u - row * runs_per_row) * 4;
    Idx rem = row;
    int64_t off_out = 0;
    int64_t off_in[kMaxIn];
#pragma unroll
    for (int k = 0; k < kMaxIn; ++k) off_in[k] = 0;
    for (int d = inner - 1; d >= 0; --d) {
      const Idx sh = (Idx)p.shape[d];
      const Idx qq = rem / sh;
      const int64_t c = (int64_t)(rem - qq * sh);
      rem = qq;
      off_out += c * p.out.st[d];
#pragma unroll
      for (int k = 0; k < kMaxIn; ++k)
        if (k < p.n_in) off_in[k] += c * p.in[k].st[d];
    }
    float* op = static_cast<float*>(p.out.ptr) + off_out + c0;
    const bool full = c0 + 4 <= cols;
    float v[kMaxIn][4];
#pragma unroll
    for (int k = 0; k < kMaxIn; ++k) {
      if (k >= p.n_in) continue;
      const float* ip = static_cast<const float*>(p.in[k].ptr) + off_in[k];
      if (bcast_mask & (1u << k)) {
        const float x = ip[0];
        v[k][0] = v[k][1] = v[k][2] = v[k][3] = x;
      } else if (full && (vec_mask & (1u << k))) {
        const float4 x = *reinterpret_cast<const float4*>(ip + c0);
        v[k][0] = x.x;
        v[k][1] = x.y;
        v[k][2] = x.z;
        v[k][3] = x.w;
      } else {
        const int64_t st = p.in[k].st[inner];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[k][e] = c0 + e < cols ? ip[(c0 + e) * st] : 0.f;
      }
    }
    float o[4];
    if (p.fast != EW_INTERP) {
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = eval_fast(p, v, e);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
#pragma unroll
        for (int k = 0; k < kMaxIn; ++k)
          if (k < p.n_in) regs[k].f = v[k][e];
        o[e] = run_program(p.prog, regs, &err).f;
      }
    }
    if (full && (vec_mask & (1u << 31))) {
      *reinterpret_cast<float4*>(op) = make_float4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (c0 + e < cols) op[e] = o[e];
    }
  }
  if (err) set_status(p.status, err);
}

void launch_elementwise(const EwParams& p, cudaStream_t s) {
  if (p.numel <= 0) return;
  // Rows fast path: every operand f32 and the output's inner stride 1
  // (operands with other inner strides are read element by element).
  if (p.rank >= 2 && p.out.dt == DT_F32 && p.out.st[p.rank - 1] == 1) {
    const int inner = p.rank - 1;
    bool ok = true;
    unsigned vec_mask = 0, bcast_mask = 0;
    const int64_t cols = p.shape[inner];
    for (int k = 0; k < p.n_in && ok; ++k) {
      if (p.in[k].dt != DT_F32) ok = false;
      else if (p.in[k].st[inner] == 0) bcast_mask |= 1u << k;
      else if (p.in[k].st[inner] == 1) {
        bool aligned = (reinterpret_cast<uintptr_t>(p.in[k].ptr) & 15) == 0;
        for (int d = 0; d < inner; ++d) aligned = aligned && (p.in[k].st[d] % 4 == 0);
        if (aligned) vec_mask |= 1u << k;
      }
    }
    bool out_aligned = (reinterpret_cast<uintptr_t>(p.out.ptr) & 15) == 0;
    for (int d = 0; d < inner; ++d) out_aligned = out_aligned && (p.out.st[d] % 4 == 0);
    if (out_aligned) vec_mask |= 1u << 31;
    if (ok && cols >= 4) {
      const int64_t rows = p.numel / cols;
      const int64_t runs = rows * ((cols + 3) / 4);
      if (p.numel < (int64_t(1) << 31))
        elementwise_rows4_kernel<uint32_t><<<grid_for(runs), kThreads, 0, s>>>(p, vec_mask, bcast_mask, rows, cols);
      else
        elementwise_rows4_kernel<int64_t><<<grid_for(runs), kThreads, 0, s>>>(p, vec_mask, bcast_mask, rows, cols);
      return;
    }
  }
  // Dense float fast path: rank-1 iteration, unit strides or scalars, 16-byte aligned.
  bool dense = p.rank == 1 && p.out.dt == DT_F32 && p.out.st[0] == 1 &&
               (reinterpret_cast<uintptr_t>(p.out.ptr) & 15) == 0;
  unsigned scalar_mask = 0;
  for (int k = 0; dense && k < p.n_in; ++k) {
    if (p.in[k].dt != DT_F32) dense = false;
    else if (p.in[k].st[0] == 0) scalar_mask |= 1u << k;
    else if (p.in[k].st[0] != 1 || (reinterpret_cast<uintptr_t>(p.in[k].ptr) & 15) != 0) dense = false;
  }
  if (dense) {
    elementwise_dense4_kernel<<<grid_for(p.numel / 4 + 1), kThreads, 0, s>>>(p, scalar_mask);
  } else {
    elementwise_kernel<<<grid_for(p.numel), kThreads, 0, s>>>(p);
  }
}

// ---------------------------------------------------------------------------
// Float sum / mean reductions: one warp per output row.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t unravel_off(int64_t idx, int rank, const int64_t* shape, const int64_t* st) {
  int64_t off = 0;
  for (int d = rank - 1; d >= 0; --d) {
    int64_t c = idx % shape[d];
    idx /= shape[d];
    off += c * st[d];
  }
  return off;
}

__global__ void __launch_bounds__(kThreads) reduce_f32_kernel(const __grid_constant__ ReduceParams p) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x & 31;
  for (int64_t row = blockIdx.x * (int64_t)warps + threadIdx.x / 32; row < p.rows; row += (int64_t)gridDim.x * warps) {
    const int64_t base = unravel_off(row, p.kept_rank, p.kept_shape, p.kept_st);
    float acc = 0.0f;
    if (p.red_rank == 1 && p.red_st[0] == 1) {
      const float* rp = p.in + base;
      for (int64_t c = lane; c < p.cols; c += 32) acc += rp[c];
    } else {
      for (int64_t c = lane; c < p.cols; c += 32) acc += p.in[base + unravel_off(c, p.red_rank, p.red_shape, p.red_st)];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      const int64_t oo = unravel_off(row, p.kept_rank, p.kept_shape, p.out_st);
      p.out[oo] = p.mode == 1 ? __fdiv_rn(acc, p.count) : acc;
    }
  }
}

// Rows that sit next to each other in memory while each row's elements are
// strided (a spatial mean over channels-last data): one thread per row, so
// the lanes of a warp read adjacent rows and every load is coalesced.  Each
// row is summed sequentially from 0 in row-major order over the reduced
// dimensions, the order of the reference's loop.
__global__ void __launch_bounds__(kThreads) reduce_f32_strided_kernel(const __grid_constant__ ReduceParams p) {
  const int64_t n0 = p.red_shape[0], s0 = p.red_st[0];
  const int64_t n1 = p.red_rank == 2 ? p.red_shape[1] : 1, s1 = p.red_rank == 2 ? p.red_st[1] : 0;
  for (int64_t row = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; row < p.rows;
       row += (int64_t)gridDim.x * blockDim.x) {
    const float* rp = p.in + unravel_off(row, p.kept_rank, p.kept_shape, p.kept_st);
    float acc = 0.0f;
    for (int64_t a = 0; a < n0; ++a) {
      const float* ra = rp + a * s0;
#pragma unroll 7
      for (int64_t b = 0; b < n1; ++b) acc = __fadd_rn(acc, __ldg(ra + b * s1));
    }
    p.out[unravel_off(row, p.kept_rank, p.kept_shape, p.out_st)] = p.mode == 1 ? __fdiv_rn(acc, p.count) : acc;
  }
}

void launch_reduce_f32(const ReduceParams& p, cudaStream_t s) {
  if (p.rows <= 0) return;
  const bool strided_rows = p.kept_rank >= 1 && p.kept_st[p.kept_rank - 1] == 1 && p.red_rank >= 1 &&
                            p.red_rank <= 2 && p.red_st[p.red_rank - 1] != 1 && p.cols <= 4096 &&
                            p.rows >= 32;
  if (strided_rows)
    reduce_f32_strided_kernel<<<grid_for(p.rows), kThreads, 0, s>>>(p);
  else
    reduce_f32_kernel<<<grid_for(p.rows, kThreads / 32), kThreads, 0, s>>>(p);
}

__global__ void __launch_bounds__(kThreads) generic_reduce_kernel(const __grid_constant__ GenericReduceParams p) {
  Reg regs[kMaxRegs];
  int err = 0;
  for (int64_t row = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; row < p.rows; row += (int64_t)gridDim.x * blockDim.x) {
    const int64_t base = unravel_off(row, p.kept_rank, p.kept_shape, p.kept_st);
    const int64_t oo = unravel_off(row, p.kept_rank, p.kept_shape, p.out_st);
    Reg acc = load_dt(p.out, oo, p.out_dt);
    for (int64_t c = 0; c < p.cols; ++c) {
      regs[0] = load_dt(p.in, base + unravel_off(c, p.red_rank, p.red_shape, p.red_st), p.in_dt);
      regs[1] = acc;
      acc = run_program(p.prog, regs, &err);
    }
    store_dt(p.out, oo, p.out_dt, acc);
  }
  if (err) set_status(p.status, err);
}

void launch_generic_reduce(const GenericReduceParams& p, cudaStream_t s) {
  if (p.rows <= 0) return;
  generic_reduce_kernel<<<grid_for(p.rows), kThreads, 0, s>>>(p);
}

// ---------------------------------------------------------------------------
// Softmax (linalg.softmax decomposition: max from the lowest finite float,
// exp(x - max), sum, divide).  One warp per row for short rows, a block per
// row for long ones.
// ---------------------------------------------------------------------------
template <int WARPS_PER_ROW>
__global__ void __launch_bounds__(kThreads) softmax_kernel(const __grid_constant__ SoftmaxParams p) {
  __shared__ float red[kThreads / 32];
  constexpr int kRowThreads = 32 * WARPS_PER_ROW;
  const int rows_per_block = kThreads / kRowThreads;
  const int t = threadIdx.x % kRowThreads;
  const int sub = threadIdx.x / kRowThreads;
  const int lane = threadIdx.x & 31;
  const int wid = t / 32;
  for (int64_t rb = blockIdx.x * (int64_t)rows_per_block; rb < p.rows; rb += (int64_t)gridDim.x * rows_per_block) {
    const int64_t row = rb + sub;
    const bool active = row < p.rows;
    const float* x = active ? p.in + unravel_off(row, p.rank, p.row_shape, p.in_row_st) : p.in;
    float* y = active ? p.out + unravel_off(row, p.rank, p.row_shape, p.out_row_st) : p.out;
    float m = -FLT_MAX;
    if (active)
      for (int64_t j = t; j < p.len; j += kRowThreads) m = fmaxf(m, x[j * p.in_axis_st]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (WARPS_PER_ROW > 1) {
      if (lane == 0) red[threadIdx.x / 32] = m;
      __syncthreads();
      m = -FLT_MAX;
      for (int w = 0; w < WARPS_PER_ROW; ++w) m = fmaxf(m, red[sub * WARPS_PER_ROW + w]);
      __syncthreads();
    }
    float ssum = 0.0f;
    if (active)
      for (int64_t j = t; j < p.len; j += kRowThreads) {
        float e = expf(__fsub_rn(x[j * p.in_axis_st], m));
        y[j * p.out_axis_st] = e;
        ssum += e;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    if (WARPS_PER_ROW > 1) {
      if (lane == 0) red[threadIdx.x / 32] = ssum;
      __syncthreads();
      ssum = 0.0f;
      for (int w = 0; w < WARPS_PER_ROW; ++w) ssum += red[sub * WARPS_PER_ROW + w];
      __syncthreads();
    }
    (void)wid;
    if (active)
      for (int64_t j = t; j < p.len; j += kRowThreads) y[j * p.out_axis_st] = __fdiv_rn(y[j * p.out_axis_st], ssum);
  }
}

// Rows of up to 32 * PER elements: one warp per row holds the row in
// registers (PER values per lane, float4 loads and stores when the axis is
// contiguous and aligned), so the row is read once and written once.  Same
// steps as the multi-pass kernel: max from -FLT_MAX, exp(x - max), sum, divide.
template <int PER>
__global__ void __launch_bounds__(kThreads) softmax_reg_kernel(const __grid_constant__ SoftmaxParams p, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
  for (int64_t row = blockIdx.x * (int64_t)(kThreads / 32) + threadIdx.x / 32; row < p.rows; row += warps) {
    const float* x = p.in + unravel_off(row, p.rank, p.row_shape, p.in_row_st);
    float* y = p.out + unravel_off(row, p.rank, p.row_shape, p.out_row_st);
    float v[PER];
    if (vec) {
#pragma unroll
      for (int c = 0; c < PER / 4; ++c) {
        const int64_t j = ((int64_t)c * 32 + lane) * 4;
        float4 t = make_float4(-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX);
        if (j < p.len) t = *reinterpret_cast<const float4*>(x + j);
        v[4 * c] = t.x;
        v[4 * c + 1] = t.y;
        v[4 * c + 2] = t.z;
        v[4 * c + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int c = 0; c < PER; ++c) {
        const int64_t j = (int64_t)c * 32 + lane;
        v[c] = j < p.len ? x[j * p.in_axis_st] : -FLT_MAX;
      }
    }
    float m = -FLT_MAX;
#pragma unroll
    for (int c = 0; c < PER; ++c) m = fmaxf(m, v[c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float ssum = 0.0f;
#pragma unroll
    for (int c = 0; c < PER; ++c) {
      const int64_t j = vec ? ((int64_t)(c / 4) * 32 + lane) * 4 + (c & 3) : (int64_t)c * 32 + lane;
      v[c] = j < p.len ? expf(__fsub_rn(v[c], m)) : 0.0f;
      ssum += v[c];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    if (vec) {
#pragma unroll
      for (int c = 0; c < PER / 4; ++c) {
        const int64_t j = ((int64_t)c * 32 + lane) * 4;
        if (j < p.len)
          *reinterpret_cast<float4*>(y + j) = make_float4(__fdiv_rn(v[4 * c], ssum), __fdiv_rn(v[4 * c + 1], ssum),
                                                          __fdiv_rn(v[4 * c + 2], ssum), __fdiv_rn(v[4 * c + 3], ssum));
      }
    } else {
#pragma unroll
      for (int c = 0; c < PER; ++c) {
        const int64_t j = (int64_t)c * 32 + lane;
        if (j < p.len) y[j * p.out_axis_st] = __fdiv_rn(v[c], ssum);
      }
    }
  }
}

void launch_softmax(const SoftmaxParams& p, cudaStream_t s) {
  if (p.rows <= 0) return;
  // float4 rows: contiguous axis, length a multiple of 4, every row 16-byte aligned
  bool vec = p.in_axis_st == 1 && p.out_axis_st == 1 && p.len % 4 == 0 &&
             (reinterpret_cast<uintptr_t>(p.in) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0;
  for (int d = 0; d < p.rank && vec; ++d) vec = p.in_row_st[d] % 4 == 0 && p.out_row_st[d] % 4 == 0;
  if (p.len <= 128) {
    softmax_reg_kernel<4><<<grid_for(p.rows, kThreads / 32), kThreads, 0, s>>>(p, vec);
  } else if (p.len <= 512) {
    softmax_reg_kernel<16><<<grid_for(p.rows, kThreads / 32), kThreads, 0, s>>>(p, vec);
  } else if (p.len <= 1024) {
    softmax_kernel<1><<<grid_for(p.rows, kThreads / 32), kThreads, 0, s>>>(p);
  } else {
    softmax_kernel<8><<<grid_for(p.rows, 1), kThreads, 0, s>>>(p);
  }
}

// ---------------------------------------------------------------------------
// Gather
// ---------------------------------------------------------------------------
__device__ __forceinline__ long long load_index(const void* idx, int64_t j, int dt) {
  return dt == DT_I32 ? (long long)static_cast<const int*>(idx)[j] : static_cast<const long long*>(idx)[j];
}

__global__ void __launch_bounds__(kThreads) gather_rows16_kernel(const __grid_constant__ GatherParams p) {
  // post * elem_bytes is a multiple of 16: copy 16-byte chunks
  const int64_t chunks = p.post * p.elem_bytes / 16;
  const int64_t total = p.pre * p.nidx * chunks;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = i % chunks;
    const int64_t j = (i / chunks) % p.nidx;
    const int64_t a = i / (chunks * p.nidx);
    long long v = load_index(p.idx, j, p.idx_dt);
    uint4 val = make_uint4(0, 0, 0, 0);
    if (v < 0 || v >= p.axis_len) {
      set_status(p.status, ST_GATHER_INDEX);
    } else {
      val = reinterpret_cast<const uint4*>(p.data)[(a * p.axis_len + v) * chunks + c];
    }
    reinterpret_cast<uint4*>(p.out)[i] = val;
  }
}

__global__ void __launch_bounds__(kThreads) gather_elems_kernel(const __grid_constant__ GatherParams p) {
  const int64_t total = p.pre * p.nidx * p.post;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t q = i % p.post;
    const int64_t j = (i / p.post) % p.nidx;
    const int64_t a = i / (p.post * p.nidx);
    long long v = load_index(p.idx, j, p.idx_dt);
    const unsigned char* src = static_cast<const unsigned char*>(p.data);
    unsigned char* dst = static_cast<unsigned char*>(p.out) + i * p.elem_bytes;
    if (v < 0 || v >= p.axis_len) {
      set_status(p.status, ST_GATHER_INDEX);
      for (int b = 0; b < p.elem_bytes; ++b) dst[b] = 0;
    } else {
      src += ((a * p.axis_len + v) * p.post + q) * p.elem_bytes;
      for (int b = 0; b < p.elem_bytes; ++b) dst[b] = src[b];
    }
  }
}

void launch_gather(const GatherParams& p, cudaStream_t s) {
  const int64_t total = p.pre * p.nidx * p.post;
  if (total <= 0) return;
  bool vec = (p.post * p.elem_bytes) % 16 == 0 && (reinterpret_cast<uintptr_t>(p.data) & 15) == 0 &&
             (reinterpret_cast<uintptr_t>(p.out) & 15) == 0;
  if (vec) gather_rows16_kernel<<<grid_for(total * p.elem_bytes / 16), kThreads, 0, s>>>(p);
  else gather_elems_kernel<<<grid_for(total), kThreads, 0, s>>>(p);
}

__global__ void __launch_bounds__(kThreads) gather_elements_kernel(const __grid_constant__ GatherElementsParams p) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < p.numel; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, off = 0;
    long long v = load_index(p.idx, i, p.idx_dt);
    bool ok = v >= 0 && v < p.data_axis_len;
    for (int d = p.rank - 1; d >= 0; --d) {
      int64_t c = rem % p.shape[d];
      rem /= p.shape[d];
      off += (d == p.axis ? (ok ? v : 0) : c) * p.data_st[d];
    }
    if (!ok) set_status(p.status, ST_GATHER_INDEX);
    const unsigned char* src = static_cast<const unsigned char*>(p.data) + off * p.elem_bytes;
    unsigned char* dst = static_cast<unsigned char*>(p.out) + i * p.elem_bytes;
    for (int b = 0; b < p.elem_bytes; ++b) dst[b] = ok ? src[b] : 0;
  }
}

void launch_gather_elements(const GatherElementsParams& p, cudaStream_t s) {
  if (p.numel <= 0) return;
  gather_elements_kernel<<<grid_for(p.numel), kThreads, 0, s>>>(p);
}

// ---------------------------------------------------------------------------
// Index remap (pad / tile / resize)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads) remap_kernel(const __grid_constant__ RemapParams p) {
  const T fill = *reinterpret_cast<const T*>(&p.fill_bits);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < p.numel; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, src = 0, dst = 0;
    bool inside = true;
    for (int d = p.rank - 1; d >= 0; --d) {
      const int64_t o = rem % p.out_shape[d];
      rem /= p.out_shape[d];
      dst += o * p.out_st[d];
      const int64_t c = ((o / p.div[d]) % p.mod[d]) - p.sub[d];
      if (c < 0 || c >= p.in_shape[d]) inside = false;
      src += c * p.in_st[d];
    }
    static_cast<T*>(p.out)[dst] = inside ? static_cast<const T*>(p.in)[src] : fill;
  }
}

void launch_remap(const RemapParams& p, cudaStream_t s) {
  if (p.numel <= 0) return;
  const unsigned g = grid_for(p.numel);
  switch (p.elem_bytes) {
    case 1: remap_kernel<uint8_t><<<g, kThreads, 0, s>>>(p); break;
    case 2: remap_kernel<uint16_t><<<g, kThreads, 0, s>>>(p); break;
    case 4: remap_kernel<uint32_t><<<g, kThreads, 0, s>>>(p); break;
    default: remap_kernel<uint64_t><<<g, kThreads, 0, s>>>(p); break;
  }
}

// NCHW -> NHWC with the channel dim padded (zeros) to C4, a multiple of 4:
// each thread writes one pixel's 4 channels with a 16-byte store; the reads
// of a warp stay within 4 channel planes at consecutive pixels.
__global__ void __launch_bounds__(kThreads) nchw_to_nhwc4_kernel(const float* __restrict__ in, float* __restrict__ out,
                                                                 int64_t N, int C, int C4, int64_t HW,
                                                                 int64_t in_sn, int64_t in_sc) {
  const int cg = C4 / 4;
  const int64_t total = N * HW * cg;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(i % cg);
    const int64_t pix = (i / cg) % HW;
    const int64_t n = i / (cg * HW);
    const float* src = in + n * in_sn + pix;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = g * 4 + k;
      v[k] = c < C ? __ldg(src + (int64_t)c * in_sc) : 0.0f;
    }
    reinterpret_cast<float4*>(out)[i] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// C <= 4 (an image input): four consecutive pixels per thread, one float4
// load per channel plane and four float4 stores (64 contiguous bytes);
// 32-bit indices.  Strides are in float4 units.
__global__ void __launch_bounds__(kThreads) nchw_to_nhwc4_px4_kernel(const float4* __restrict__ in,
                                                                     float4* __restrict__ out, uint32_t N, int C,
                                                                     uint32_t HW4, uint32_t in_sn4, uint32_t in_sc4) {
  const uint32_t total = N * HW4;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t n = i / HW4, q = i - n * HW4;
    const float4* src = in + (size_t)n * in_sn4 + q;
    float4 c[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) c[k] = k < C ? __ldg(src + (size_t)k * in_sc4) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4* dst = out + (size_t)i * 4;
    dst[0] = make_float4(c[0].x, c[1].x, c[2].x, c[3].x);
    dst[1] = make_float4(c[0].y, c[1].y, c[2].y, c[3].y);
    dst[2] = make_float4(c[0].z, c[1].z, c[2].z, c[3].z);
    dst[3] = make_float4(c[0].w, c[1].w, c[2].w, c[3].w);
  }
}

void launch_nchw_to_nhwc4(const float* in, float* out, int64_t N, int C, int C4, int64_t HW, int64_t in_sn,
                          int64_t in_sc, cudaStream_t s) {
  const int64_t total = N * HW * (C4 / 4);
  if (total <= 0) return;
  const bool px4 = C4 == 4 && HW % 4 == 0 && in_sn % 4 == 0 && in_sc % 4 == 0 && in_sn / 4 < (int64_t(1) << 32) &&
                   in_sc / 4 < (int64_t(1) << 32) && N * HW / 4 < (int64_t(1) << 31) &&
                   (reinterpret_cast<uintptr_t>(in) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  if (px4)
    nchw_to_nhwc4_px4_kernel<<<grid_for(N * HW / 4), kThreads, 0, s>>>(
        reinterpret_cast<const float4*>(in), reinterpret_cast<float4*>(out), (uint32_t)N, C, (uint32_t)(HW / 4),
        (uint32_t)(in_sn / 4), (uint32_t)(in_sc / 4));
  else
    nchw_to_nhwc4_kernel<<<grid_for(total), kThreads, 0, s>>>(in, out, N, C, C4, HW, in_sn, in_sc);
}

__global__ void range_kernel(const __grid_constant__ RangeParams p) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < p.n; i += (int64_t)gridDim.x * blockDim.x) {
    Reg r;
    r.i = 0;
    if (p.dt == DT_F32) r.f = __fadd_rn((float)p.fstart, __fmul_rn((float)i, (float)p.fdelta));
    else if (p.dt == DT_F64) r.d = p.fstart + (double)i * p.fdelta;
    else r.i = wrap_((long long)((unsigned long long)p.istart + (unsigned long long)i * (unsigned long long)p.idelta), p.dt);
    store_dt(p.out, i, p.dt, r);
  }
}

void launch_range(const RangeParams& p, cudaStream_t s) {
  if (p.n <= 0) return;
  range_kernel<<<grid_for(p.n), kThreads, 0, s>>>(p);
}

// ---------------------------------------------------------------------------
// Pooling: one thread per output element, iterated in the output's physical
// order so that NHWC tensors are read and written coalesced along channels.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) pool_kernel(const __grid_constant__ PoolParams p) {
  const int64_t total = p.N * p.C * p.OH * p.OW;
  const int64_t dims[4] = {p.N, p.C, p.OH, p.OW};
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, c4[4];
    for (int k = 3; k >= 0; --k) {
      int d = (int)p.iter_perm[k];
      c4[d] = rem % dims[d];
      rem /= dims[d];
    }
    const int64_t n = c4[0], c = c4[1], oh = c4[2], ow = c4[3];
    const float* base = p.in + n * p.in_st[0] + c * p.in_st[1];
    float acc = p.mode == 0 ? -INFINITY : 0.0f;
    for (int kh = 0; kh < p.kh; ++kh) {
      const int64_t ih = oh * p.sh + kh * p.dh - p.ph;
      for (int kw = 0; kw < p.kw; ++kw) {
        const int64_t iw = ow * p.sw + kw * p.dw - p.pw;
        const bool in = ih >= 0 && ih < p.H && iw >= 0 && iw < p.W;
        if (p.mode == 0) {
          const float v = in ? base[ih * p.in_st[2] + iw * p.in_st[3]] : -INFINITY;
          acc = maximumf_(acc, v);
        } else {
          const float v = in ? base[ih * p.in_st[2] + iw * p.in_st[3]] : 0.0f;
          acc = __fadd_rn(acc, v);
        }
      }
    }
    if (p.mode == 1) acc = __fdiv_rn(acc, p.count);
    p.out[n * p.out_st[0] + c * p.out_st[1] + oh * p.out_st[2] + ow * p.out_st[3]] = acc;
  }
}

// Dense NHWC on both sides with C % 4 == 0: one thread per 4 channels of an
// output pixel, 16-byte loads and stores, 32-bit spatial indices.  Idx is the
// type of the flat output index (32-bit when the output has < 2^31 groups:
// its divisions cost a fraction of 64-bit ones).
// KW > 0 fixes the window at compile time (KW x KW), so the window's loads are
// all issued before the first is used.
// arith.maximumf in one instruction: max.NaN.f32 (PTX ISA 7.0+, sm_80+)
// returns NaN when either input is NaN and orders -0 < +0.  Its NaN is
// canonicalised per output (nan_canon_) to the 0x7fc00000 that maximumf_
// returns, so the pool results keep the same bits.
__device__ __forceinline__ float max_nan_(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float nan_canon_(float x) { return isnan(x) ? __int_as_float(0x7fc00000) : x; }
__device__ __forceinline__ float4 max_nan4_(float4 a, float4 b) {
  return make_float4(max_nan_(a.x, b.x), max_nan_(a.y, b.y), max_nan_(a.z, b.z), max_nan_(a.w, b.w));
}
__device__ __forceinline__ float4 nan_canon4_(float4 a) {
  return make_float4(nan_canon_(a.x), nan_canon_(a.y), nan_canon_(a.z), nan_canon_(a.w));
}

template <typename Idx, int KW>
__global__ void __launch_bounds__(kThreads) pool_nhwc4_kernel(const __grid_constant__ PoolParams p) {
  const Idx cg = (Idx)(p.C / 4);
  const Idx OW = (Idx)p.OW, OH = (Idx)p.OH;
  const Idx total = (Idx)(p.N * p.OH * p.OW) * cg;
  for (Idx i = blockIdx.x * (Idx)blockDim.x + threadIdx.x; i < total; i += (Idx)gridDim.x * blockDim.x) {
    const int g = (int)(i % cg);
    Idx r = i / cg;
    const int ow = (int)(r % OW);
    r /= OW;
    const int oh = (int)(r % OH);
    const int64_t n = (int64_t)(r / OH);
    const float* base = p.in + n * p.in_st[0] + g * 4;
    float4 acc = p.mode == 0 ? make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY) : make_float4(0.f, 0.f, 0.f, 0.f);
    const int nkh = KW > 0 ? KW : p.kh, nkw = KW > 0 ? KW : p.kw;
#pragma unroll
    for (int kh = 0; kh < nkh; ++kh) {
      const int ih = oh * p.sh + kh * p.dh - p.ph;
#pragma unroll
      for (int kw = 0; kw < nkw; ++kw) {
        const int iw = ow * p.sw + kw * p.dw - p.pw;
        const bool in = ih >= 0 && ih < p.H && iw >= 0 && iw < p.W;
        float4 v;
        if (in) v = __ldg(reinterpret_cast<const float4*>(base + ih * p.in_st[2] + iw * p.in_st[3]));
        else v = p.mode == 0 ? make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.mode == 0) {
          acc = max_nan4_(acc, v);
        } else {
          acc.x = __fadd_rn(acc.x, v.x); acc.y = __fadd_rn(acc.y, v.y);
          acc.z = __fadd_rn(acc.z, v.z); acc.w = __fadd_rn(acc.w, v.w);
        }
      }
    }
    if (p.mode == 0) acc = nan_canon4_(acc);
    if (p.mode == 1) {
      acc.x = __fdiv_rn(acc.x, p.count); acc.y = __fdiv_rn(acc.y, p.count);
      acc.z = __fdiv_rn(acc.z, p.count); acc.w = __fdiv_rn(acc.w, p.count);
    }
    *reinterpret_cast<float4*>(p.out + n * p.out_st[0] + (int64_t)oh * p.out_st[2] + (int64_t)ow * p.out_st[3] + g * 4) = acc;
  }
}

// 3x3 window, stride 2, dilation 1 (the ResNet stem pool), dense NHWC,
// C % 4 == 0: one thread per 4 channels of a BH x BW block of outputs, which
// share a (2BH+1) x (2BW+1) input patch (a 1x2 block: 15 loads instead of
// 18).  Each output still folds its window in (kh, kw) order with the same
// padding values.
template <int BH, int BW>
__global__ void __launch_bounds__(kThreads) pool_nhwc4_3x3s2_kernel(const __grid_constant__ PoolParams p) {
  const uint32_t cg = (uint32_t)(p.C / 4);
  const uint32_t OW = (uint32_t)p.OW, OH = (uint32_t)p.OH;
  const uint32_t OW2 = (OW + BW - 1) / BW, OH2 = (OH + BH - 1) / BH;
  const uint32_t total = (uint32_t)p.N * OH2 * OW2 * cg;
  const float pad = p.mode == 0 ? -INFINITY : 0.f;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t g = i % cg;
    uint32_t r = i / cg;
    const uint32_t ow2 = r % OW2;
    r /= OW2;
    const uint32_t oh2 = r % OH2;
    const int64_t n = r / OH2;
    const int oh = BH * (int)oh2, ow = BW * (int)ow2;
    const float* base = p.in + n * p.in_st[0] + g * 4;
    float4 acc[BH][BW];
#pragma unroll
    for (int a = 0; a < BH; ++a)
#pragma unroll
      for (int b = 0; b < BW; ++b) acc[a][b] = make_float4(pad, pad, pad, pad);
#pragma unroll
    for (int dy = 0; dy < 2 * BH + 1; ++dy) {
      const int ih = oh * 2 - p.ph + dy;
#pragma unroll
      for (int dx = 0; dx < 2 * BW + 1; ++dx) {
        const int iw = ow * 2 - p.pw + dx;
        float4 v = make_float4(pad, pad, pad, pad);
        if (ih >= 0 && ih < p.H && iw >= 0 && iw < p.W)
          v = __ldg(reinterpret_cast<const float4*>(base + ih * p.in_st[2] + iw * p.in_st[3]));
#pragma unroll
        for (int a = 0; a < BH; ++a) {
          const int kh = dy - 2 * a;
          if (kh < 0 || kh > 2) continue;
#pragma unroll
          for (int b = 0; b < BW; ++b) {
            const int kw = dx - 2 * b;
            if (kw < 0 || kw > 2) continue;
            float4& o = acc[a][b];
            if (p.mode == 0) {
              o = max_nan4_(o, v);
            } else {
              o.x = __fadd_rn(o.x, v.x); o.y = __fadd_rn(o.y, v.y);
              o.z = __fadd_rn(o.z, v.z); o.w = __fadd_rn(o.w, v.w);
            }
          }
        }
      }
    }
#pragma unroll
    for (int a = 0; a < BH; ++a)
#pragma unroll
      for (int b = 0; b < BW; ++b) {
        if ((uint32_t)(oh + a) >= OH || (uint32_t)(ow + b) >= OW) continue;
        float4 o = acc[a][b];
        if (p.mode == 0) o = nan_canon4_(o);
        if (p.mode == 1) {
          o.x = __fdiv_rn(o.x, p.count); o.y = __fdiv_rn(o.y, p.count);
          o.z = __fdiv_rn(o.z, p.count); o.w = __fdiv_rn(o.w, p.count);
        }
        *reinterpret_cast<float4*>(p.out + n * p.out_st[0] + (int64_t)(oh + a) * p.out_st[2] +
                                   (int64_t)(ow + b) * p.out_st[3] + g * 4) = o;
      }
  }
}

void launch_pool(const PoolParams& p, cudaStream_t s) {
  const int64_t total = p.N * p.C * p.OH * p.OW;
  if (total <= 0) return;
  const bool nhwc4 = p.C % 4 == 0 && p.in_st[1] == 1 && p.out_st[1] == 1 && p.in_st[3] == p.C &&
                     p.out_st[3] == p.C && p.in_st[2] % 4 == 0 && p.out_st[2] % 4 == 0 && p.in_st[0] % 4 == 0 &&
                     p.out_st[0] % 4 == 0 && (reinterpret_cast<uintptr_t>(p.in) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(p.out) & 15) == 0;
  const bool small = total / 4 < (int64_t(1) << 31);
  if (nhwc4 && small && p.kh == 3 && p.kw == 3 && p.sh == 2 && p.sw == 2 && p.dh == 1 && p.dw == 1)
    pool_nhwc4_3x3s2_kernel<1, 2><<<resident_grid<pool_nhwc4_3x3s2_kernel<1, 2>>(total / 8 + 1), kThreads, 0, s>>>(p);
  else if (nhwc4 && small && p.kh == 3 && p.kw == 3)
    pool_nhwc4_kernel<uint32_t, 3><<<grid_for(total / 4), kThreads, 0, s>>>(p);
  else if (nhwc4 && small) pool_nhwc4_kernel<uint32_t, 0><<<grid_for(total / 4), kThreads, 0, s>>>(p);
  else if (nhwc4) pool_nhwc4_kernel<int64_t, 0><<<grid_for(total / 4), kThreads, 0, s>>>(p);
  else pool_kernel<<<grid_for(total), kThreads, 0, s>>>(p);
}

// ---------------------------------------------------------------------------
// Top-k: one block per row; each round is a block-wide first-strict-max scan
// over unused positions, as in the reference's selection loop.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) topk_kernel(const __grid_constant__ TopKParams p) {
  __shared__ float sv[kThreads];
  __shared__ long long si[kThreads];
  for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const float* x = p.in + row * p.len;
    unsigned char* used = p.used + row * p.len;
    for (int64_t j = threadIdx.x; j < p.len; j += blockDim.x) used[j] = 0;
    __syncthreads();
    for (int64_t ki = 0; ki < p.k; ++ki) {
      float bv = -INFINITY;
      long long bi = 0;
      bool found = false;
      for (int64_t j = threadIdx.x; j < p.len; j += blockDim.x) {
        float v = x[j];
        if (!used[j] && v > bv) { bv = v; bi = j; found = true; }
      }
      sv[threadIdx.x] = bv;
      si[threadIdx.x] = found ? bi : (long long)p.len;  // "none" sorts last
      __syncthreads();
      for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) {
          float v2 = sv[threadIdx.x + o];
          long long i2 = si[threadIdx.x + o];
          float v1 = sv[threadIdx.x];
          long long i1 = si[threadIdx.x];
          // earliest index with the strictly largest value wins; ties keep the first
          bool take = (i2 < p.len) && ((i1 >= p.len) || v2 > v1 || (v2 == v1 && i2 < i1));
          if (take) { sv[threadIdx.x] = v2; si[threadIdx.x] = i2; }
        }
        __syncthreads();
      }
      if (threadIdx.x == 0) {
        long long w = si[0];
        float wv = sv[0];
        if (w >= p.len) { w = 0; wv = -INFINITY; }
        p.vals[row * p.k + ki] = wv;
        p.idxs[row * p.k + ki] = w;
        used[w] = 1;
      }
      __syncthreads();
    }
  }
}

void launch_topk(const TopKParams& p, cudaStream_t s) {
  if (p.rows <= 0) return;
  topk_kernel<<<grid_for(p.rows, 1, 4), kThreads, 0, s>>>(p);
}

// ---------------------------------------------------------------------------
// Row normalisation: one warp per row.  Rows of at most kRowRegCols columns
// (float4-aligned) are loaded once into registers, all loads in flight
// together; longer or unaligned rows are read again per pass (the repeat
// reads hit L1).  Either way each lane adds its own elements in ascending
// column order and a shuffle tree adds the lanes, so both forms give the
// same bits.
// ---------------------------------------------------------------------------
constexpr int kRowRegVecs = 8;                  // float4 per lane
constexpr int kRowRegCols = kRowRegVecs * 128;  // 1024 columns

__device__ __forceinline__ void rownorm_row_regs(const RowNormParams& p, const float* x, float* y, int lane,
                                                 float count) {
  auto warp_sum = [](float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
  };
  float4 v[kRowRegVecs];
#pragma unroll
  for (int j = 0; j < kRowRegVecs; ++j) {
    const int64_t c = lane * 4 + 128 * j;
    v[j] = c < p.cols ? *reinterpret_cast<const float4*>(x + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float mu = 0.f;
  if (p.centered) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kRowRegVecs; ++j)
      if (lane * 4 + 128 * j < p.cols) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[j].x), v[j].y), v[j].z), v[j].w);
    mu = __fdiv_rn(warp_sum(s), count);
  }
  float s2 = 0.f;
#pragma unroll
  for (int j = 0; j < kRowRegVecs; ++j) {
    if (lane * 4 + 128 * j < p.cols) {
      const float a = __fsub_rn(v[j].x, mu), b = __fsub_rn(v[j].y, mu), d = __fsub_rn(v[j].z, mu),
                  e = __fsub_rn(v[j].w, mu);
      s2 = __fadd_rn(s2, __fmul_rn(a, a));
      s2 = __fadd_rn(s2, __fmul_rn(b, b));
      s2 = __fadd_rn(s2, __fmul_rn(d, d));
      s2 = __fadd_rn(s2, __fmul_rn(e, e));
    }
  }
  const float r = __fsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(s2), count), p.eps));
#pragma unroll
  for (int j = 0; j < kRowRegVecs; ++j) {
    const int64_t c = lane * 4 + 128 * j;
    if (c < p.cols) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(p.w + c));
      float4 o = make_float4(__fmul_rn(__fdiv_rn(__fsub_rn(v[j].x, mu), r), w.x),
                             __fmul_rn(__fdiv_rn(__fsub_rn(v[j].y, mu), r), w.y),
                             __fmul_rn(__fdiv_rn(__fsub_rn(v[j].z, mu), r), w.z),
                             __fmul_rn(__fdiv_rn(__fsub_rn(v[j].w, mu), r), w.w));
      if (p.b) {
        const float4 bb = __ldg(reinterpret_cast<const float4*>(p.b + c));
        o = make_float4(__fadd_rn(o.x, bb.x), __fadd_rn(o.y, bb.y), __fadd_rn(o.z, bb.z), __fadd_rn(o.w, bb.w));
      }
      *reinterpret_cast<float4*>(y + c) = o;
    }
  }
}

__global__ void __launch_bounds__(kThreads) rownorm_kernel(const __grid_constant__ RowNormParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const float count = (float)p.cols;  // the mean divides by it, as the reference does
  const bool vec = (p.cols & 3) == 0 && (p.x_rs & 3) == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 && p.w_st == 1 &&
                   (reinterpret_cast<uintptr_t>(p.w) & 15) == 0 &&
                   (!p.b || (p.b_st == 1 && (reinterpret_cast<uintptr_t>(p.b) & 15) == 0));
  auto warp_sum = [](float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
  };
  for (int64_t row = blockIdx.x * (int64_t)(blockDim.x / 32) + threadIdx.x / 32; row < p.rows; row += warps) {
    const float* x = p.x + row * p.x_rs;
    float* y = p.out + row * p.cols;
    if (vec && p.cols <= kRowRegCols) {
      rownorm_row_regs(p, x, y, lane, count);
      continue;
    }
    float mu = 0.f;
    if (p.centered) {
      float s = 0.f;
      if (vec) {
        for (int64_t c = lane * 4; c < p.cols; c += 128) {
          const float4 v = *reinterpret_cast<const float4*>(x + c);
          s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v.x), v.y), v.z), v.w);
        }
      } else {
        for (int64_t c = lane; c < p.cols; c += 32) s = __fadd_rn(s, x[c]);
      }
      mu = __fdiv_rn(warp_sum(s), count);
    }
    float s2 = 0.f;
    if (vec) {
      for (int64_t c = lane * 4; c < p.cols; c += 128) {
        const float4 v = *reinterpret_cast<const float4*>(x + c);
        const float a = __fsub_rn(v.x, mu), b = __fsub_rn(v.y, mu), d = __fsub_rn(v.z, mu), e = __fsub_rn(v.w, mu);
        s2 = __fadd_rn(s2, __fmul_rn(a, a));
        s2 = __fadd_rn(s2, __fmul_rn(b, b));
        s2 = __fadd_rn(s2, __fmul_rn(d, d));
        s2 = __fadd_rn(s2, __fmul_rn(e, e));
      }
    } else {
      for (int64_t c = lane; c < p.cols; c += 32) {
        const float a = __fsub_rn(x[c], mu);
        s2 = __fadd_rn(s2, __fmul_rn(a, a));
      }
    }
    const float r = __fsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(s2), count), p.eps));
    if (vec) {
      for (int64_t c = lane * 4; c < p.cols; c += 128) {
        const float4 v = *reinterpret_cast<const float4*>(x + c);
        const float4 w = __ldg(reinterpret_cast<const float4*>(p.w + c));
        float4 o = make_float4(__fmul_rn(__fdiv_rn(__fsub_rn(v.x, mu), r), w.x),
                               __fmul_rn(__fdiv_rn(__fsub_rn(v.y, mu), r), w.y),
                               __fmul_rn(__fdiv_rn(__fsub_rn(v.z, mu), r), w.z),
                               __fmul_rn(__fdiv_rn(__fsub_rn(v.w, mu), r), w.w));
        if (p.b) {
          const float4 bb = __ldg(reinterpret_cast<const float4*>(p.b + c));
          o = make_float4(__fadd_rn(o.x, bb.x), __fadd_rn(o.y, bb.y), __fadd_rn(o.z, bb.z), __fadd_rn(o.w, bb.w));
        }
        *reinterpret_cast<float4*>(y + c) = o;
      }
    } else {
      for (int64_t c = lane; c < p.cols; c += 32) {
        float o = __fmul_rn(__fdiv_rn(__fsub_rn(x[c], mu), r), __ldg(p.w + c * p.w_st));
        if (p.b) o = __fadd_rn(o, __ldg(p.b + c * p.b_st));
        y[c] = o;
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) rope_kernel(const __grid_constant__ RopeParams p) {
  const int r = p.rank;
  const int64_t d = p.shape[r - 1];
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < p.numel; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i / d;
    const int64_t col = i - rem * d;
    int64_t xo = 0, co = 0, so = 0;
    for (int k = r - 2; k >= 0; --k) {
      const int64_t c = rem % p.shape[k];
      rem /= p.shape[k];
      xo += c * p.x_st[k];
      co += c * p.c_st[k];
      so += c * p.s_st[k];
    }
    const int64_t xl = p.x_st[r - 1];
    const float xv = p.x[xo + col * xl];
    const float rot = col < p.half ? -p.x[xo + (col + p.half) * xl] : p.x[xo + (col - p.half) * xl];
    p.out[i] = __fadd_rn(__fmul_rn(xv, __ldg(p.cs + co + col * p.c_st[r - 1])),
                         __fmul_rn(rot, __ldg(p.sn + so + col * p.s_st[r - 1])));
  }
}

// Four consecutive columns of one row and their partners half a row away
// per thread (d / 2 a multiple of 4): out[c] = x[c] cos[c] + (-x[c + h]) sin[c]
// and out[c + h] = x[c + h] cos[c + h] + x[c] sin[c + h] read x[c] and
// x[c + h] once for both; 32-bit coordinates found once per eight outputs;
// float4 loads of x, cos and sin where their last stride is 1 and rows are
// aligned.
__global__ void __launch_bounds__(kThreads) rope4_kernel(const __grid_constant__ RopeParams p, unsigned vec_mask) {
  const int r = p.rank;
  const uint32_t d = (uint32_t)p.shape[r - 1], half = (uint32_t)p.half, h4 = half / 4;
  const uint32_t total = (uint32_t)(p.numel / 8);
  for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < total; u += gridDim.x * blockDim.x) {
    uint32_t rem = u / h4;
    const uint32_t col = (u - rem * h4) * 4;
    const uint32_t row = rem;
    int64_t xo = 0, co = 0, so = 0;
    for (int k = r - 2; k >= 0; --k) {
      const uint32_t sh = (uint32_t)p.shape[k];
      const uint32_t qq = rem / sh;
      const int64_t c = rem - qq * sh;
      rem = qq;
      xo += c * p.x_st[k];
      co += c * p.c_st[k];
      so += c * p.s_st[k];
    }
    float a[4], b[4], ca[4], cb[4], sa[4], sb[4];
    auto load4 = [&](const float* base, int64_t st, bool v, float (&o)[4]) {
      if (v) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(base));
        o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = __ldg(base + e * st);
      }
    };
    const int64_t xl = p.x_st[r - 1], cl = p.c_st[r - 1], sl = p.s_st[r - 1];
    load4(p.x + xo + col * xl, xl, vec_mask & 1, a);
    load4(p.x + xo + (col + half) * xl, xl, vec_mask & 1, b);
    load4(p.cs + co + col * cl, cl, vec_mask & 2, ca);
    load4(p.cs + co + (col + half) * cl, cl, vec_mask & 2, cb);
    load4(p.sn + so + col * sl, sl, vec_mask & 4, sa);
    load4(p.sn + so + (col + half) * sl, sl, vec_mask & 4, sb);
    float lo[4], hi[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      lo[e] = __fadd_rn(__fmul_rn(a[e], ca[e]), __fmul_rn(-b[e], sa[e]));
      hi[e] = __fadd_rn(__fmul_rn(b[e], cb[e]), __fmul_rn(a[e], sb[e]));
    }
    float* orow = p.out + (int64_t)row * d;
    *reinterpret_cast<float4*>(orow + col) = make_float4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<float4*>(orow + col + half) = make_float4(hi[0], hi[1], hi[2], hi[3]);
  }
}

void launch_rope(const RopeParams& p, cudaStream_t s) {
  if (p.numel <= 0) return;
  const int r = p.rank;
  const int64_t d = p.shape[r - 1];
  auto rows_aligned = [&](const float* b, const int64_t* st) {
    if (st[r - 1] != 1 || (reinterpret_cast<uintptr_t>(b) & 15)) return false;
    for (int k = 0; k < r - 1; ++k)
      if (st[k] % 4) return false;
    return true;
  };
  if (d % 8 == 0 && 2 * p.half == d && p.numel / 4 < (int64_t(1) << 31) &&
      (reinterpret_cast<uintptr_t>(p.out) & 15) == 0) {
    const unsigned mask = (rows_aligned(p.x, p.x_st) ? 1u : 0u) | (rows_aligned(p.cs, p.c_st) ? 2u : 0u) |
                          (rows_aligned(p.sn, p.s_st) ? 4u : 0u);
    rope4_kernel<<<resident_grid<rope4_kernel>(p.numel / 8), kThreads, 0, s>>>(p, mask);
    return;
  }
  rope_kernel<<<resident_grid<rope_kernel>(p.numel), kThreads, 0, s>>>(p);
}

void launch_rownorm(const RowNormParams& p, cudaStream_t s) {
  if (p.rows <= 0) return;
  rownorm_kernel<<<resident_grid<rownorm_kernel>(p.rows * 32), kThreads, 0, s>>>(p);
}

// ---------------------------------------------------------------------------
// B-operand packing into TF32 hi/lo planes [batch][N][ldk].
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) pack_b_kernel(const __grid_constant__ PackBParams p) {
  const int64_t total = p.batch * p.N * p.ldk;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = i % p.ldk;
    const int64_t n = (i / p.ldk) % p.N;
    const int64_t b = i / (p.ldk * p.N);
    float x = 0.0f;
    if (k < p.K) {
      int64_t off = n * p.sn, rem = b;
      for (int d = p.batch_rank - 1; d >= 0; --d) {
        off += (rem % p.batch_shape[d]) * p.batch_st[d];
        rem /= p.batch_shape[d];
      }
      bool valid = true;
      rem = k;
      for (int d = p.k_rank - 1; d >= 0; --d) {
        const int64_t c = rem % p.k_shape[d];
        rem /= p.k_shape[d];
        if (c >= p.k_valid[d]) valid = false;
        off += c * p.k_st[d];
      }
      if (valid) x = p.src[off];
    }
    const float hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
    p.hi[i] = hi;
    p.lo[i] = __fsub_rn(x, hi);
  }
}

// Four consecutive k of one (b, n) row per thread, 32-bit indices: the row's
// source offset is found once per four outputs, a single k dimension needs no
// division, contiguous k loads as a float4, and both planes store float4s
// (ldk is a multiple of 4).  Same values as pack_b_kernel.
__global__ void __launch_bounds__(kThreads) pack_b4_kernel(const __grid_constant__ PackBParams p, bool vec_src) {
  const uint32_t q4 = (uint32_t)(p.ldk / 4), N = (uint32_t)p.N, K = (uint32_t)p.K;
  const uint32_t total = (uint32_t)(p.batch * p.N) * q4;
  for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < total; u += gridDim.x * blockDim.x) {
    const uint32_t row = u / q4;
    const uint32_t k0 = (u - row * q4) * 4;
    const uint32_t b = row / N, n = row - b * N;
    int64_t base = (int64_t)n * p.sn;
    uint32_t rem = b;
    for (int d = p.batch_rank - 1; d >= 0; --d) {
      const uint32_t sh = (uint32_t)p.batch_shape[d];
      const uint32_t qq = rem / sh;
      base += (int64_t)(rem - qq * sh) * p.batch_st[d];
      rem = qq;
    }
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    if (vec_src && k0 + 4 <= K) {
      const float4 t = *reinterpret_cast<const float4*>(p.src + base + k0);
      x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t k = k0 + e;
        if (k >= K) continue;
        if (p.k_rank == 1) {
          if (k < (uint32_t)p.k_valid[0]) x[e] = p.src[base + (int64_t)k * p.k_st[0]];
        } else {
          int64_t off = base;
          bool valid = true;
          uint32_t r = k;
          for (int d = p.k_rank - 1; d >= 0; --d) {
            const uint32_t sh = (uint32_t)p.k_shape[d];
            const uint32_t qq = r / sh;
            const uint32_t c = r - qq * sh;
            r = qq;
            if (c >= (uint32_t)p.k_valid[d]) valid = false;
            off += (int64_t)c * p.k_st[d];
          }
          if (valid) x[e] = p.src[off];
        }
      }
    }
    float h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      h[e] = __uint_as_float(__float_as_uint(x[e]) & 0xffffe000u);
      l[e] = __fsub_rn(x[e], h[e]);
    }
    const int64_t i = (int64_t)u * 4;
    *reinterpret_cast<float4*>(p.hi + i) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(p.lo + i) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// Sources stored k-outer, n-contiguous ([k][n] rows, the layout of a
// gawee.matmul right operand): a 32 x 32 block of (k, n) goes through shared
// memory, so the loads run along n and the plane stores along k, both
// coalesced.  One k dimension; batch offsets as in pack_b_kernel.  Same values.
constexpr int kPackT = 32;
__global__ void __launch_bounds__(256) pack_b_kn_kernel(const __grid_constant__ PackBParams p) {
  __shared__ float tile[kPackT][kPackT + 1];
  const int64_t kt = (p.ldk + kPackT - 1) / kPackT, nt = (p.N + kPackT - 1) / kPackT;
  const int64_t tiles = p.batch * nt * kt;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t k0 = (t % kt) * kPackT;
    const int64_t n0 = ((t / kt) % nt) * kPackT;
    const int64_t b = t / (kt * nt);
    int64_t base = 0, rem = b;
    for (int d = p.batch_rank - 1; d >= 0; --d) {
      base += (rem % p.batch_shape[d]) * p.batch_st[d];
      rem /= p.batch_shape[d];
    }
    const int64_t n = n0 + tx;
#pragma unroll
    for (int j = 0; j < kPackT; j += 8) {
      const int64_t k = k0 + ty + j;
      float x = 0.f;
      if (n < p.N && k < p.K && k < p.k_valid[0]) x = p.src[base + k * p.k_st[0] + n];
      tile[ty + j][tx] = x;
    }
    __syncthreads();
    const int64_t k = k0 + tx;
#pragma unroll
    for (int j = 0; j < kPackT; j += 8) {
      const int64_t nn = n0 + ty + j;
      if (nn < p.N && k < p.ldk) {
        const float x = tile[tx][ty + j];
        const float hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
        const int64_t i = (b * p.N + nn) * p.ldk + k;
        p.hi[i] = hi;
        p.lo[i] = __fsub_rn(x, hi);
      }
    }
    __syncthreads();
  }
}

// The BF16 mode's B plane from the packed TF32 planes: hi + lo is the
// packed fp32 value exactly (lo = x - hi, exact), rounded to bf16 (nearest
// even); rows of ldk16 >= ldk values, zero past ldk.
__global__ void __launch_bounds__(kThreads) planes_to_bf16_kernel(const float* __restrict__ hi,
                                                                  const float* __restrict__ lo,
                                                                  __nv_bfloat16* __restrict__ out, int64_t rows,
                                                                  int64_t ldk, int64_t ldk16) {
  const int64_t total = rows * ldk16;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / ldk16, k = i - r * ldk16;
    float x = 0.f;
    if (k < ldk) x = __fadd_rn(hi[r * ldk + k], lo[r * ldk + k]);
    out[i] = __float2bfloat16_rn(x);
  }
}

void launch_planes_to_bf16(const float* hi, const float* lo, void* out, int64_t rows, int64_t ldk, int64_t ldk16,
                           cudaStream_t s) {
  if (rows <= 0 || ldk16 <= 0) return;
  planes_to_bf16_kernel<<<grid_for(rows * ldk16), kThreads, 0, s>>>(hi, lo, static_cast<__nv_bfloat16*>(out), rows,
                                                                    ldk, ldk16);
}

void launch_pack_b(const PackBParams& p, cudaStream_t s) {
  const int64_t total = p.batch * p.N * p.ldk;
  if (total <= 0) return;
  if (p.k_rank == 1 && p.sn == 1 && p.k_st[0] != 1) {
    const int64_t tiles = p.batch * ((p.N + kPackT - 1) / kPackT) * ((p.ldk + kPackT - 1) / kPackT);
    pack_b_kn_kernel<<<(unsigned)std::min<int64_t>(tiles, 148 * 8), 256, 0, s>>>(p);
    return;
  }
  const bool fits = total / 4 < (int64_t(1) << 31) && p.batch * p.N < (int64_t(1) << 31) && p.ldk % 4 == 0 &&
                    (reinterpret_cast<uintptr_t>(p.hi) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.lo) & 15) == 0;
  if (fits) {
    // k contiguous in the source, whole float4s valid, rows and batches 16-byte aligned
    bool vec = p.k_rank == 1 && p.k_st[0] == 1 && p.k_valid[0] >= p.K && p.sn % 4 == 0 &&
               (reinterpret_cast<uintptr_t>(p.src) & 15) == 0;
    for (int d = 0; d < p.batch_rank && vec; ++d) vec = p.batch_st[d] % 4 == 0;
    pack_b4_kernel<<<grid_for(total / 4), kThreads, 0, s>>>(p, vec);
    return;
  }
  pack_b_kernel<<<grid_for(total), kThreads, 0, s>>>(p);
}

}  // namespace kern
}  // namespace gawee
