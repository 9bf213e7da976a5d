// Device helpers shared by the tensor-core kernels (conv_gemm_tc.cu, the
// cp.async-gather kernel, and conv_gemm_tma.cu, the TMA kernel): mbarrier,
// cp.async, TMA and tcgen05 wrappers, the UMMA descriptors, and the epilogue
// that turns a tile's fp32 sums into the output (bias, ReLU, residual, or a
// scalar program over aux operands).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <climits>
#include <cstdint>

#include "kernels.h"
#include "program.cuh"

namespace gawee {
namespace kern {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;               // fp32 elements per k-block (one 128-byte swizzle row)
constexpr int kThreadsTC = 448;  // 4 A warps, 1 TMA, 1 MMA, 8 accumulator warps
constexpr unsigned long long kWaitNs = 4000000000ull;  // 4 s per barrier wait
// Epilogue staging: each accumulator warp transposes 16-column chunks of its
// 32 rows through shared memory (row pitch 20 floats: conflict-free float4
// writes by row, float4 reads by column group).
constexpr int kStagePitch = 20;
constexpr int kStageWarpFloats = 32 * kStagePitch;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of a phase (test_wait never suspends the thread).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false if the CTA is aborting or the wait timed out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitNs) {
      *abort_flag = 1;
      if (status) atomicCAS(status, 0, (int)ST_BARRIER_TIMEOUT);
      return false;
    }
  }
}


// The same bounded wait for warps off the critical path: between polls the
// thread sleeps `sleep_ns`, so a dozen waiting warps do not keep the
// shared-memory barrier unit busy while the MMA issuer polls its own barrier.
__device__ __forceinline__ bool mbar_wait_relaxed(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status,
                                                  unsigned sleep_ns) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (true) {
    __nanosleep(sleep_ns);
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitNs) {
      *abort_flag = 1;
      if (status) atomicCAS(status, 0, (int)ST_BARRIER_TIMEOUT);
      return false;
    }
  }
}

// 16-byte global -> shared copy that bypasses registers; `bytes` 0 writes zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ float4 lds128(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset
  d |= (uint64_t)1 << 46;                   // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::tf32, fp32 accumulate, K-major A and B, M = 128.
template <int BN>
__device__ __forceinline__ uint32_t umma_idesc_tf32() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}


// D (tensor memory) += A (tensor memory, lane = row, one column per k) . B (shared memory)
__device__ __forceinline__ void umma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}


__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }


// Epilogue of one output tile.  Called by each of the eight accumulator
// warps (warps 6-13: lane quarter warp % 4 is fixed by the hardware, two
// warps share a quarter and split the tile's columns in halves) with the
// row's fp32 sums of its half tile in `acc`; c_off is the tile's output
// offset (batch, or split slice), stage_all the 8 warps' staging buffers in
// shared memory, ok false when the tile's accumulation was aborted.
template <int BN, int EPI>
__device__ __forceinline__ void tile_epilogue(const ConvGemmParams& p, float (&acc)[BN / 2], int64_t m0, int n0,
                                              int z, int64_t c_off, int warp, int lane, float* stage_all, bool ok) {
  constexpr int HB = BN / 2;
  const int q = warp & 3;
  const int half = (warp - 6) / 4;
  const int cbase = half * HB;
  const int row = q * 32 + lane;
  if (EPI < EPI_PROGRAM) {
    // Coalesced epilogue: the warp writes its 32 rows 16 columns at a
    // time into shared memory, then stores them four lanes per row, so a
    // store instruction covers 8 rows x 64 contiguous bytes instead of 32
    // rows x 16 bytes; bias and residual come as whole float4 groups.
    const bool coal = p.ldc_n == 1 && (p.ldc & 3) == 0 && (c_off & 3) == 0 &&
                      (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
                      (EPI != EPI_BIAS_ADD_RELU || (reinterpret_cast<uintptr_t>(p.res) & 15) == 0);
    if (coal && __all_sync(0xffffffffu, ok)) {
      float* stage = stage_all + (warp - 6) * kStageWarpFloats;
      const int nb0 = n0 + cbase;
      const int c4 = lane & 3;
#pragma unroll
      for (int c0 = 0; c0 < HB; c0 += 16) {
        float* srow = stage + lane * kStagePitch;
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(srow + j) = make_float4(acc[c0 + j], acc[c0 + j + 1], acc[c0 + j + 2], acc[c0 + j + 3]);
        __syncwarp();
        const int64_t n = nb0 + c0 + c4 * 4;
        float b[4] = {0.f, 0.f, 0.f, 0.f};
        if (EPI >= EPI_BIAS) {
#pragma unroll
          for (int e = 0; e < 4; ++e) b[e] = n + e < p.N ? __ldg(p.bias + n + e) : 0.f;
        }
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int r = it * 8 + (lane >> 2);
          const int64_t m = m0 + q * 32 + r;
          const float4 v = *reinterpret_cast<const float4*>(stage + r * kStagePitch + c4 * 4);
          if (m < p.M && n < p.N) {
            float x[4] = {v.x, v.y, v.z, v.w};
            const bool full = n + 3 < p.N;
            float rv[4] = {0.f, 0.f, 0.f, 0.f};
            if (EPI == EPI_BIAS_ADD_RELU) {
              const float* rp = p.res + c_off + m * p.ldc + n;
              if (full) {
                const float4 t = __ldg(reinterpret_cast<const float4*>(rp));
                rv[0] = t.x; rv[1] = t.y; rv[2] = t.z; rv[3] = t.w;
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) rv[e] = n + e < p.N ? __ldg(rp + e) : 0.f;
              }
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (EPI >= EPI_BIAS) x[e] = __fadd_rn(x[e], b[e]);
              if (EPI == EPI_BIAS_ADD_RELU) x[e] = __fadd_rn(x[e], rv[e]);
              if (EPI == EPI_BIAS_RELU || EPI == EPI_BIAS_ADD_RELU) x[e] = maximumf_(x[e], 0.0f);
            }
            float* cp = p.out + c_off + m * p.ldc + n;
            if (full) {
              *reinterpret_cast<float4*>(cp) = make_float4(x[0], x[1], x[2], x[3]);
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                if (n + e < p.N) cp[e] = x[e];
            }
          }
        }
        __syncwarp();  // the staging rows are rewritten by the next chunk
      }
      return;
    }
  }
  if (EPI == EPI_FAST) {
    // Recognised programs: each thread loads its row's aux values (one
    // 16-column chunk ahead when there is a single aux operand), computes
    // the chunk, and the warp stores it through the shared-memory
    // transpose (8 rows x 64 bytes per store instead of 32 rows x 16 bytes).
    const bool two = p.fast == FAST_SIGMOID_MUL || p.fast == FAST_ADD_ADD;
    int64_t abase = 0, abase1 = 0;
    {
      uint32_t rem = (uint32_t)z;
      for (int d = p.batch_rank - 1; d >= 0; --d) {
        const uint32_t sh = (uint32_t)p.batch_shape[d];
        const uint32_t qq = rem / sh;
        abase += (int64_t)(rem - qq * sh) * p.aux_sb[0][d];
        if (two) abase1 += (int64_t)(rem - qq * sh) * p.aux_sb[1][d];
        rem = qq;
      }
    }
    const int nb0 = n0 + cbase;
    const bool coal = p.ldc_n == 1 && (p.ldc & 3) == 0 && (c_off & 3) == 0 &&
                      (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 && p.aux_sn[0] == 1 &&
                      (p.aux_sm[0] & 3) == 0 && ((reinterpret_cast<uintptr_t>(p.aux[0] + abase) & 15) == 0) &&
                      p.bias == nullptr && nb0 + HB <= p.N &&
                      (!two || (p.aux_sn[1] == 1 && (p.aux_sm[1] & 3) == 0 &&
                                ((reinterpret_cast<uintptr_t>(p.aux[1] + abase1) & 15) == 0)));
    if (coal && __all_sync(0xffffffffu, ok)) {
      float* stage = stage_all + (warp - 6) * kStageWarpFloats;
      const int64_t m = m0 + row;
      const bool mrow = m < p.M;
      const float* arow = p.aux[0] + abase + (mrow ? m : 0) * p.aux_sm[0] + nb0;
      const float* arow1 = two ? p.aux[1] + abase1 + (mrow ? m : 0) * p.aux_sm[1] + nb0 : arow;
      float4 an[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) an[j] = mrow ? __ldg(reinterpret_cast<const float4*>(arow) + j) : make_float4(0, 0, 0, 0);
      const int c4 = lane & 3;
#pragma unroll
      for (int c0 = 0; c0 < HB; c0 += 16) {
        float a[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          a[4 * j] = an[j].x; a[4 * j + 1] = an[j].y; a[4 * j + 2] = an[j].z; a[4 * j + 3] = an[j].w;
        }
        float o[16];
        if (two) {  // this chunk's second operand now; no prefetch (registers)
          if (p.fast == FAST_SIGMOID_MUL) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // four values of the second operand live at a time
              const float4 t = mrow ? __ldg(reinterpret_cast<const float4*>(arow1 + c0) + j) : make_float4(0, 0, 0, 0);
              const float b1[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-b1[e])));
                acc[c0 + 4 * j + e] = __fmul_rn(__fmul_rn(a[4 * j + e], sg), acc[c0 + 4 * j + e]);
              }
            }
          } else {  // FAST_ADD_ADD
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 t = mrow ? __ldg(reinterpret_cast<const float4*>(arow1 + c0) + j) : make_float4(0, 0, 0, 0);
              const float b1[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
              for (int e = 0; e < 4; ++e)
                acc[c0 + 4 * j + e] = __fadd_rn(__fadd_rn(acc[c0 + 4 * j + e], a[4 * j + e]), b1[e]);
            }
          }
          if (c0 + 16 < HB) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              an[j] = mrow ? __ldg(reinterpret_cast<const float4*>(arow + c0 + 16) + j) : make_float4(0, 0, 0, 0);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = acc[c0 + j];
        } else {
          // computed in place: this chunk's accumulators are not needed
          // afterwards, and the aux registers are free for the next chunk,
          // whose loads are then in flight while this one is stored
          // one loop per form: a form chosen per element let the compiler
          // evaluate the IEEE division for every element of every form
          if (p.fast == FAST_ADD) {
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[c0 + j] = __fadd_rn(acc[c0 + j], a[j]);
          } else if (p.fast == FAST_DIVC_ADD) {
            const float c = p.fast_c;
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[c0 + j] = __fadd_rn(__fdiv_rn(acc[c0 + j], c), a[j]);
          } else if (p.fast == FAST_MULC_ADD) {
            const float c = p.fast_c;
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[c0 + j] = __fadd_rn(__fmul_rn(acc[c0 + j], c), a[j]);
          } else {  // FAST_GELU
            const float c = p.fast_c;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float t = __fadd_rn(acc[c0 + j], a[j]);
              acc[c0 + j] = __fmul_rn(__fmul_rn(t, __fadd_rn(erff(__fdiv_rn(t, c)), 1.0f)), 0.5f);
            }
          }
          if (c0 + 16 < HB) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              an[j] = mrow ? __ldg(reinterpret_cast<const float4*>(arow + c0 + 16) + j) : make_float4(0, 0, 0, 0);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = acc[c0 + j];
        }
        float* srow = stage + lane * kStagePitch;
#pragma unroll
        for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(srow + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int r = it * 8 + (lane >> 2);
          const int64_t mm = m0 + q * 32 + r;
          const float4 v = *reinterpret_cast<const float4*>(stage + r * kStagePitch + c4 * 4);
          if (mm < p.M) *reinterpret_cast<float4*>(p.out + c_off + mm * p.ldc + nb0 + c0 + c4 * 4) = v;
        }
        __syncwarp();
      }
      return;
    }
  }
  const int64_t m = m0 + row;
  if (!ok || m >= p.M) return;
  float* crow = p.out + c_off + m * p.ldc;
  const int nb0 = n0 + cbase;  // first column of this thread's half tile
  if (EPI == EPI_PROGRAM || EPI == EPI_FAST) {
    // operand offsets of this row: the batch coordinate is fixed per tile
    int64_t aux_row[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      aux_row[a] = 0;
      if (a < p.n_aux) {
        int64_t o = m * p.aux_sm[a];
        uint32_t rem = (uint32_t)z;
        for (int d = p.batch_rank - 1; d >= 0; --d) {
          const uint32_t sh = (uint32_t)p.batch_shape[d];
          const uint32_t q = rem / sh;
          o += (int64_t)(rem - q * sh) * p.aux_sb[a][d];
          rem = q;
        }
        aux_row[a] = o;
      }
    }
    const bool vec = p.ldc_n == 1 && nb0 + HB <= p.N && ((reinterpret_cast<uintptr_t>(crow + nb0) & 15) == 0);
    auto store8 = [&](int c0, const float (&o)[8]) {
      if (vec) {
        *reinterpret_cast<float4*>(crow + nb0 + c0) = make_float4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<float4*>(crow + nb0 + c0 + 4) = make_float4(o[4], o[5], o[6], o[7]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (nb0 + c0 + j < p.N) crow[(int64_t)(nb0 + c0 + j) * p.ldc_n] = o[j];
      }
    };
    int err = 0;
    if (EPI == EPI_FAST) {
      // Fully unrolled: the accumulators stay in registers.  8 columns at
      // a time, their operand loads all in flight before they are used.
      bool aux_vec = p.aux_sn[0] == 1 && nb0 + HB <= p.N &&
                     ((reinterpret_cast<uintptr_t>(p.aux[0] + aux_row[0] + nb0) & 15) == 0);
      const bool two = p.fast == FAST_SIGMOID_MUL || p.fast == FAST_ADD_ADD;
      if (two)
        aux_vec = aux_vec && p.aux_sn[1] == 1 && ((reinterpret_cast<uintptr_t>(p.aux[1] + aux_row[1] + nb0) & 15) == 0);
#pragma unroll
      for (int c0 = 0; c0 < HB; c0 += 8) {
        float a0[8], a1[8], o[8];
        if (aux_vec) {  // unit column stride, 16-byte aligned rows, whole chunk in range
          const float4* q0 = reinterpret_cast<const float4*>(p.aux[0] + aux_row[0] + nb0 + c0);
          const float4 u = __ldg(q0), v = __ldg(q0 + 1);
          a0[0] = u.x; a0[1] = u.y; a0[2] = u.z; a0[3] = u.w;
          a0[4] = v.x; a0[5] = v.y; a0[6] = v.z; a0[7] = v.w;
          if (two) {
            const float4* q1 = reinterpret_cast<const float4*>(p.aux[1] + aux_row[1] + nb0 + c0);
            const float4 w = __ldg(q1), x = __ldg(q1 + 1);
            a1[0] = w.x; a1[1] = w.y; a1[2] = w.z; a1[3] = w.w;
            a1[4] = x.x; a1[5] = x.y; a1[6] = x.z; a1[7] = x.w;
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) a1[j] = 0.f;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int64_t n = nb0 + c0 + j;
            const bool in = n < p.N;
            a0[j] = in ? __ldg(p.aux[0] + aux_row[0] + n * p.aux_sn[0]) : 0.f;
            a1[j] = (in && two) ? __ldg(p.aux[1] + aux_row[1] + n * p.aux_sn[1]) : 0.f;
          }
        }
        float xs[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int64_t n = nb0 + c0 + j;
          xs[j] = p.bias ? __fadd_rn(acc[c0 + j], n < p.N ? __ldg(p.bias + n) : 0.f) : acc[c0 + j];
        }
        // one loop per form (see the coalesced path)
        if (p.fast == FAST_ADD) {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = __fadd_rn(xs[j], a0[j]);
        } else if (p.fast == FAST_DIVC_ADD) {
          const float c = p.fast_c;
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = __fadd_rn(__fdiv_rn(xs[j], c), a0[j]);
        } else if (p.fast == FAST_MULC_ADD) {
          const float c = p.fast_c;
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = __fadd_rn(__fmul_rn(xs[j], c), a0[j]);
        } else if (p.fast == FAST_ADD_ADD) {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = __fadd_rn(__fadd_rn(xs[j], a0[j]), a1[j]);
        } else if (p.fast == FAST_GELU) {
          const float c = p.fast_c;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float t = __fadd_rn(xs[j], a0[j]);
            o[j] = __fmul_rn(__fmul_rn(t, __fadd_rn(erff(__fdiv_rn(t, c)), 1.0f)), 0.5f);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a1[j])));
            o[j] = __fmul_rn(__fmul_rn(a0[j], sg), xs[j]);
          }
        }
        store8(c0, o);
      }
    } else {
      // Interpreter (its own instantiation, EPI_PROGRAM): the row's sums
      // go to a separate array first, so the dynamically indexed loop
      // below does not move `acc` itself out of registers.
      float accl[HB];
#pragma unroll
      for (int j = 0; j < HB; ++j) accl[j] = acc[j];
      Reg regs[kMaxRegs];
      for (int c0 = 0; c0 < HB; c0 += 8) {
        float av[4][8];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int64_t n = nb0 + c0 + j;
            av[a][j] = (a < p.n_aux && n < p.N) ? __ldg(p.aux[a] + aux_row[a] + n * p.aux_sn[a]) : 0.f;
          }
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int64_t n = nb0 + c0 + j;
          o[j] = 0.f;
          if (n < p.N) {
            regs[0].f = p.bias ? __fadd_rn(accl[c0 + j], __ldg(p.bias + n)) : accl[c0 + j];
#pragma unroll
            for (int a = 0; a < 4; ++a)
              if (a < p.n_aux) regs[1 + a].f = av[a][j];
            o[j] = run_program(p.prog, regs, &err).f;
          }
        }
        store8(c0, o);
      }
    }
    if (err && p.status) atomicCAS(p.status, 0, err);
  } else {
    const bool vec = p.ldc_n == 1 && nb0 + HB <= p.N && ((reinterpret_cast<uintptr_t>(crow + nb0) & 15) == 0);
    // 16 columns at a time keeps the bias / residual temporaries small
#pragma unroll
    for (int c0 = 0; c0 < HB; c0 += 16) {
      float o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int64_t n = nb0 + c0 + j;
        float x = acc[c0 + j];
        if (EPI >= EPI_BIAS) x = __fadd_rn(x, n < p.N ? __ldg(p.bias + n) : 0.f);
        if (EPI == EPI_BIAS_ADD_RELU) x = __fadd_rn(x, n < p.N ? __ldg(p.res + c_off + m * p.ldc + n * p.ldc_n) : 0.f);
        if (EPI == EPI_BIAS_RELU || EPI == EPI_BIAS_ADD_RELU) x = maximumf_(x, 0.0f);
        o[j] = x;
      }
      if (vec) {
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(crow + nb0 + c0 + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (nb0 + c0 + j < p.N) crow[(int64_t)(nb0 + c0 + j) * p.ldc_n] = o[j];
      }
    }
  }
}

__device__ __forceinline__ void sts128(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// Shared-memory address of 16-byte chunk `ch` (4 columns, 0 .. BN / 4 - 1) of
// row r of a staged aux tile: BN / 32 boxes of [128 rows][32 columns], box b
// 16 KB at b * 16 KB, 128-byte swizzled (chunk c of row r at c ^ (r & 7)).
__device__ __forceinline__ uint32_t aux_chunk(uint32_t tile, int r, int ch) {
  return tile + (uint32_t)((ch >> 3) * (kBM * kBK * 4) + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

// FAST_SIGMOID_MUL, ahead of the epilogue: 16-column chunk i of this
// thread's half row of the staged aux tile becomes aux * (1 / (1 + exp(-aux)))
// in place -- the epilogue's first product, which does not involve the
// accumulator -- so the epilogue that follows only multiplies by it.  The
// accumulator warps call it between round drains, while the tensor core
// works on the tile's remaining rounds.
template <int BN>
__device__ __forceinline__ void aux_sigmoid_chunk(uint32_t tile, int warp, int lane, int i) {
  constexpr int HB = BN / 2;
  const int row = (warp & 3) * 32 + lane;
  const int ch0 = (((warp - 6) / 4) * HB + i * 16) >> 2;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t addr = aux_chunk(tile, row, ch0 + j);
    const float4 v = lds128(addr);
    const float a[4] = {v.x, v.y, v.z, v.w};
    float t[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) t[e] = __fmul_rn(a[e], __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a[e]))));
    sts128(addr, t[0], t[1], t[2], t[3]);
  }
}

// Epilogue of one unsplit output tile whose aux operand is already in shared
// memory (`tile`: the residual of EPI_BIAS_ADD_RELU, or aux 0 of EPI_FAST,
// laid out as aux_chunk describes, zero past M and N; for FAST_SIGMOID_MUL
// this thread's first `pre` 16-column chunks already hold aux * sigmoid(aux),
// from aux_sigmoid_chunk).  Same warps, operations and order as tile_epilogue;
// each thread reads its row's aux values, writes its results over them, and
// the warp stores its 32 rows 8 at a time (4 lanes x 16 bytes per row) --
// both shared-memory patterns cover the 8 chunk positions of a 128-byte row
// evenly, so neither has bank conflicts.  Columns past N and rows past M are
// computed but not stored.
template <int BN, int EPI>
__device__ __forceinline__ void tile_epilogue_aux(const ConvGemmParams& p, float (&acc)[BN / 2], int64_t m0, int n0,
                                                  int warp, int lane, uint32_t tile, int pre) {
  static_assert(EPI == EPI_FAST || EPI == EPI_BIAS_ADD_RELU, "aux epilogue forms");
  constexpr int HB = BN / 2;
  const int q = warp & 3;
  const int cbase = ((warp - 6) / 4) * HB;
  const int row = q * 32 + lane;
  auto chunk = [tile](int r, int ch) -> uint32_t { return aux_chunk(tile, r, ch); };
  const int c4 = lane & 3;
#pragma unroll
  for (int c0 = 0; c0 < HB; c0 += 16) {
    const int ch0 = (cbase + c0) >> 2;
    float a[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = lds128(chunk(row, ch0 + j));
      a[4 * j] = v.x; a[4 * j + 1] = v.y; a[4 * j + 2] = v.z; a[4 * j + 3] = v.w;
    }
    float o[16];
    // one loop per form: a form chosen per element would have the compiler
    // evaluate the IEEE division for every element of every form
    if (EPI == EPI_BIAS_ADD_RELU) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = n0 + cbase + c0 + j;
        const float x = __fadd_rn(__fadd_rn(acc[c0 + j], n < p.N ? __ldg(p.bias + n) : 0.f), a[j]);
        o[j] = maximumf_(x, 0.0f);
      }
    } else if (p.fast == FAST_ADD) {
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = __fadd_rn(acc[c0 + j], a[j]);
    } else if (p.fast == FAST_DIVC_ADD) {
      const float c = p.fast_c;
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = __fadd_rn(__fdiv_rn(acc[c0 + j], c), a[j]);
    } else if (p.fast == FAST_MULC_ADD) {
      const float c = p.fast_c;
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = __fadd_rn(__fmul_rn(acc[c0 + j], c), a[j]);
    } else if (c0 / 16 < pre) {  // FAST_SIGMOID_MUL, the chunk already aux * sigmoid(aux)
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = __fmul_rn(a[j], acc[c0 + j]);
    } else {  // FAST_SIGMOID_MUL with both operands the aux tile
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a[j])));
        o[j] = __fmul_rn(__fmul_rn(a[j], sg), acc[c0 + j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) sts128(chunk(row, ch0 + j), o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
    __syncwarp();
    const int n = n0 + cbase + c0 + c4 * 4;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int r = q * 32 + it * 8 + (lane >> 2);
      const int64_t m = m0 + r;
      const float4 v = lds128(chunk(r, ch0 + c4));
      if (m < p.M && n < p.N) {
        float* cp = p.out + m * p.ldc + n;
        if (n + 3 < p.N) {
          *reinterpret_cast<float4*>(cp) = v;
        } else {
          const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (n + e < p.N) cp[e] = x[e];
        }
      }
    }
  }
  // the tile was written through the generic proxy; the next TMA load into
  // it comes through the async proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace
}  // namespace kern
}  // namespace gawee
