// Tensor-core implicit-GEMM convolution and GEMM with both operands fed by
// TMA (sm_100a).
//
// Same arithmetic as conv_gemm_tc.cu — fp32 results from three TF32
// tcgen05.mma per k-step (hi*hi + hi*lo + lo*hi; Ootomo & Yokota 2022), each
// 64-wide round summed alone in tensor memory and promoted into fp32
// registers with IEEE round-to-nearest — but the A operand is no longer
// gathered by warps:
//   * A arrives by TMA.  A convolution whose channel count is a multiple of
//     32 uses an im2col tensor map over the NHWC input: one load per k-block
//     brings 128 output pixels x 32 channels of one filter tap, with the
//     padding, stride and dilation applied by the copy engine (zero fill
//     outside the image).  A plain GEMM uses a tiled 2-D map over its rows.
//     Both land in the 128-byte-swizzled K-major layout the MMA reads.
//   * The four A warps read each staged A tile once and store its raw values
//     (the tensor core reads fp32 as TF32 by dropping the 13 low mantissa
//     bits, so raw is the high part) and remainders x - tf32(x) to tensor
//     memory; all three MMAs take A from there and only B from shared
//     memory.  (Measured: an MMA reading A from shared memory costs about
//     twice one reading it from tensor memory here, where TMA writes and
//     the A warps' reads share the shared-memory bandwidth.)
//   * Shared-memory stages (one k-block of A and of both B planes each) and
//     round accumulators (tensor memory) are separate pipelines: a stage is
//     refilled as soon as its MMAs complete, up to NS k-blocks ahead.
//
// Warp roles (448 threads), persistent over work units (tile, k split):
//   warps 0-3  A: wait for a stage, read its A rows, store raw values and
//              remainders into the stage's tensor-memory columns
//   warp 4     TMA for A and the B planes; owns the tensor-memory allocation
//   warp 5     lane 0 issues the MMAs and the commits that track them
//   warps 6-13 drain round sums and run the epilogue (tc_common.cuh)
// Every mbarrier wait is bounded in time (tc_common.cuh: mbar_wait); on
// expiry the CTA records ST_BARRIER_TIMEOUT in the status word, lets its
// copies land and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "kernels.h"
#include "program.cuh"
#include "tc_common.cuh"

namespace gawee {
namespace kern {

namespace {

// Stages per tile width: 4 x 48 KB (BN 128) or 4 x 32 KB (BN 64) of shared
// memory plus 20 KB of epilogue staging; tensor memory holds NS A stages of
// 64 columns (raw, remainder) beside the two round accumulators.  With the
// epilogue's aux operand staged by TMA (AUX), the [128][BN] aux tile takes
// the staging's place and BN 128 keeps 3 stages (3 x 48 + 64 KB).
template <int BN>
struct TmaConfig;
template <>
struct TmaConfig<64> {
  static constexpr int NS = 4;
  static constexpr int NS_AUX = 4;
};
template <>
struct TmaConfig<128> {
  static constexpr int NS = 4;
  static constexpr int NS_AUX = 3;
};

template <int BN, int NS, int AUX = 0, int PASSES = 3>
struct TmaSmem {
  // PASSES 2: the BF16 mode -- one B plane of bf16 values (64-byte rows,
  // 64-byte swizzled) and A as bf16 pairs in tensor memory
  static constexpr bool kBf16 = PASSES == 2;
  static constexpr int kATile = kBM * kBK * 4;          // 16 KB: raw A of one k-block
  static constexpr int kBTile = BN * kBK * (kBf16 ? 2 : 4);  // one B plane of one k-block
  static constexpr int kStage = kATile + (kBf16 ? 1 : 2) * kBTile;  // A, B hi[, B lo] (a multiple of 1024)
  static constexpr int kStageOff = NS * kStage;         // epilogue staging, or the aux tile
  // the aux tile: BN / 32 boxes of [128 rows][32 columns], 16 KB each, 128-byte swizzled
  static constexpr int kAuxBox = kBM * kBK * 4;
  static constexpr int kAuxBytes = AUX ? (BN / kBK) * kAuxBox : 0;
  static constexpr int kBarOff = kStageOff + (AUX ? kAuxBytes : 8 * kStageWarpFloats * 4);
  static constexpr int kNAcc = 2;                       // round accumulators in tensor memory
  // full, remainders-ready, empty per stage; full, empty per accumulator; all
  // MMAs done; with AUX the aux tile's full and empty
  static constexpr int kNumBars = 3 * NS + 2 * kNAcc + 1 + (AUX ? 2 : 0);
  static constexpr int kBytes = kBarOff + 8 * kNumBars + 16 + 1024;  // + alignment slack
  // BN 64 folds hi*hi and hi*lo into one N = 128 MMA (B stage: hi rows then lo rows)
  static constexpr bool kFold = BN == 64 && !kBf16;
  static constexpr int kAccCols = kFold ? 2 * BN : BN;
  static constexpr int kACol = kNAcc * kAccCols;          // first A column
  // per stage 32 raw and 32 remainder columns, or 16 columns of bf16 pairs
  static constexpr int kAStageCols = kBf16 ? kBK / 2 : 2 * kBK;
  static constexpr int kUsedCols = kACol + NS * kAStageCols;
  static constexpr int kTmemCols = kUsedCols <= 256 ? 256 : 512;
  static_assert(kStage % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");
  static_assert(kUsedCols <= 512, "tensor memory columns");
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// im2col load: 128 pixels x 32 channels starting at the window base (w, h)
// of image n, filter tap offsets (ow, oh); coordinates are (c, w, h, n).
__device__ __forceinline__ void tma_load_im2col_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c, int w,
                                                   int h, int n, uint16_t ow, uint16_t oh) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2], {%7, %8};" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n), "h"(ow), "h"(oh)
      : "memory");
}

// Shared-memory descriptor for the BF16 mode's B tile: K-major, 64-byte
// swizzle (rows of 32 bf16), 8-row groups 512 B apart.
__device__ __forceinline__ uint64_t umma_desc_sw64(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(512 >> 4) << 32;          // stride byte offset
  d |= (uint64_t)1 << 46;                   // descriptor version (sm_100)
  d |= (uint64_t)4 << 61;                   // SWIZZLE_64B
  return d;
}

// Instruction descriptor: kind::f16 with bf16 A and B, fp32 accumulate, K-major, M = 128.
template <int BN>
__device__ __forceinline__ uint32_t umma_idesc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

// D (tensor memory) += A (tensor memory, bf16 pairs: two k per column) . B (shared memory, bf16)
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st16_a(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Two fp32 values rounded to bf16 (round to nearest even), the first in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

}  // namespace

// Poll intervals of the waits off the MMA issuer's path (nanoseconds): the A
// warps and the TMA warp have thousands of cycles of slack per stage, the
// accumulator warps a whole round.
constexpr unsigned kSleepA = 64, kSleepTma = 32, kSleepAcc = 256;

// AUX: the epilogue's aux operand (the residual of EPI_BIAS_ADD_RELU, or
// aux 0 of EPI_FAST) is loaded per tile by the TMA warp through tm_x into
// shared memory while the tile's rounds run, instead of being read from
// global memory by the accumulator warps after the tile's last round (which
// held the MMA issuer up once it ran out of drained accumulators); for
// FAST_SIGMOID_MUL the accumulator warps also form aux * sigmoid(aux) in
// place between the last round drains.  Only unsplit launches (ksplit 1)
// use it.
// PASSES: 3 (fp32 from three TF32 products), 1 (one TF32 product) or 2 (the
// BF16 mode: one kind::f16 product of bf16 operands, B from a bf16 plane
// through tm_hi, A rounded to bf16 by the A warps).
template <int BN, int NS, int EPI, int PASSES, int AUX>
__global__ void __launch_bounds__(kThreadsTC, 1)
    conv_gemm_tma_kernel(const __grid_constant__ ConvGemmParams p, const __grid_constant__ CUtensorMap tm_a,
                         const __grid_constant__ CUtensorMap tm_hi, const __grid_constant__ CUtensorMap tm_lo,
                         const __grid_constant__ CUtensorMap tm_x) {
  using L = TmaSmem<BN, NS, AUX, PASSES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* full = bars;               // stage loaded (TMA transaction bytes)
  uint64_t* remr = bars + NS;          // stage's A in tensor memory, and for a round's first stage
                                       // the round's accumulator drained (4 A warps)
  uint64_t* empty = bars + 2 * NS;     // stage's MMAs completed (one commit)
  uint64_t* accf = bars + 3 * NS;      // round accumulator complete (one commit)
  uint64_t* acce = accf + L::kNAcc;    // round accumulator drained (8 accumulator warps)
  uint64_t* done = acce + L::kNAcc;    // every MMA of this CTA completed
  uint64_t* aux_full = done + 1;       // AUX: the tile's aux operand landed (TMA transaction bytes)
  uint64_t* aux_empty = done + 2;      // AUX: the aux tile's epilogue is done with it (8 accumulator warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  // fp32 from three TF32 products, or one (the single-pass TF32 mode): a
  // template parameter, so the three-pass kernel carries no test of it
  constexpr bool three = PASSES == 3;
  constexpr bool bf16 = PASSES == 2;
  const int num_kb = (int)((p.K + kBK - 1) / kBK);
  const int rk = p.rk;  // k-blocks per promotion round (the launcher fills it)
  const int num_rounds = (num_kb + rk - 1) / rk;
  auto round_kbs = [&](int r) { return min(rk, num_kb - r * rk); };
  const int64_t m_tiles = (p.M + kBM - 1) / kBM;
  const int64_t n_tiles = (p.N + BN - 1) / BN;
  const int64_t num_tiles = m_tiles * n_tiles;  // unbatched: the launcher requires nb == 1
  const uint32_t m_tiles32 = (uint32_t)m_tiles;
  // Work units (tile, k split) exactly as in conv_gemm_tc.cu: unit u covers
  // tile u % tiles over round range u / tiles; m tiles run fastest.
  const int ksplit = p.ksplit > 1 ? p.ksplit : 1;
  const int64_t num_units = num_tiles * ksplit;
  const uint32_t tiles32 = (uint32_t)num_tiles;
  auto unit_split = [&](int64_t u, int64_t& m0, int& n0, int& split, int& r_lo, int& nr) {
    const uint32_t uu = (uint32_t)u;
    const uint32_t sp = uu / tiles32;
    const uint32_t t = uu - sp * tiles32;
    const uint32_t nt = t / m_tiles32;
    m0 = (int64_t)(t - nt * m_tiles32) * kBM;
    n0 = (int)(nt * BN);
    split = (int)sp;
    r_lo = (int)(((int64_t)sp * num_rounds) / ksplit);
    nr = (int)(((int64_t)(sp + 1) * num_rounds) / ksplit) - r_lo;
  };
  // rounds of a unit start at (m tile mod its round count), spreading the
  // B-operand k-blocks that CTAs running together fetch
  auto r_rotation = [&](int64_t m0, int nr) -> int { return (int)((uint32_t)(m0 / kBM) % (uint32_t)nr); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&remr[s]), 4);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < L::kNAcc; ++b) {
      mbar_init(smem_u32(&accf[b]), 1);
      mbar_init(smem_u32(&acce[b]), 8);
    }
    mbar_init(smem_u32(done), 1);
    if (AUX) {
      mbar_init(smem_u32(aux_full), 1);
      mbar_init(smem_u32(aux_empty), 8);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 4) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)L::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
    // ------------------------------------------------------------------ remainders
    // Lane = row of the A tile = tensor-memory lane (warp w owns 32w..32w+31).
    const int row = warp * 32 + lane;
    const uint32_t tmem_rows = tmem_base + ((uint32_t)(warp * 32) << 16);
    const bool taps = p.a_tma == A_TMA_IM2COL_TAPS;
    // tap blocks: C / 4 16-byte chunks per row (C = 4, 8, 16 -> shift 0, 1, 2)
    const uint32_t tap_shift = taps ? (p.C == 4 ? 0u : p.C == 8 ? 1u : 2u) : 0u;
    const uint32_t tap_mask = (1u << tap_shift) - 1u;
    const uint32_t row_bytes = taps ? (uint32_t)p.C * 4u : 0u;
    const uint32_t tap_bytes = row_bytes * kBM;
    uint32_t g = 0;   // k-blocks consumed
    uint32_t ar = 0;  // rounds consumed
    bool alive = true;
    for (int64_t u = blockIdx.x; u < num_units && alive; u += gridDim.x) {
      int64_t m0;
      int n0, split, r_lo, nr;
      unit_split(u, m0, n0, split, r_lo, nr);
      for (int rr = 0; rr < nr && alive; ++rr, ++ar) {
        const int nk = round_kbs(r_lo + (r_rotation(m0, nr) + rr) % nr);
        for (int j = 0; j < nk; ++j, ++g) {
          const uint32_t st = g % NS;
          if (!mbar_wait_relaxed(smem_u32(&full[st]), (g / NS) & 1, abort_flag, p.status, kSleepA)) {
            alive = false;
            break;
          }
          // the stage's raw A row: 128-byte-swizzled (chunk c of row r sits at
          // c ^ (r & 7)), or for tap blocks chunk c at tap c / (C / 4) of
          // 128 rows x C * 4 bytes, byte (c % (C / 4)) * 16 of the row
          const uint32_t stage = smem_u32(smem + st * L::kStage);
          uint32_t x[32];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t addr = taps ? stage + (uint32_t)(c >> tap_shift) * tap_bytes + row * row_bytes +
                                             ((uint32_t)(c & tap_mask) << 4)
                                       : stage + row * 128 + ((c ^ (row & 7)) << 4);
            const float4 v = lds128(addr);
            x[4 * c] = __float_as_uint(v.x);
            x[4 * c + 1] = __float_as_uint(v.y);
            x[4 * c + 2] = __float_as_uint(v.z);
            x[4 * c + 3] = __float_as_uint(v.w);
          }
          const uint32_t acol = tmem_rows + (uint32_t)(L::kACol + st * L::kAStageCols);
          if constexpr (bf16) {
            uint32_t h[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) h[e] = pack_bf16x2(__uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1]));
            tmem_st16_a(acol, h);
          } else {
            tmem_st32(acol, x);
          }
          if (three) {
            uint32_t y[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float v = __uint_as_float(x[e]);
              y[e] = __float_as_uint(__fsub_rn(v, tf32_hi(v)));
            }
            tmem_st32(acol + kBK, y);
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          // A round's first stage also certifies that the accumulator buffer
          // the round overwrites has been drained, so the MMA issuer never
          // waits on the accumulator warps itself (every wait it makes is
          // idle tensor time: the tensor core queues only a few MMAs).
          if (j == 0 &&
              !__all_sync(0xffffffffu, mbar_wait_relaxed(smem_u32(&acce[ar & 1]), ((ar >> 1) & 1) ^ 1, abort_flag,
                                                         p.status, kSleepA))) {
            alive = false;
            break;
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&remr[st]));
        }
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------------ TMA (A and B)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_hi)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_lo)) : "memory");
      if (AUX) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x)) : "memory");
      const int C = (int)p.C, S = p.S;
      const uint32_t PQ = (uint32_t)(p.P * p.Q), Q = (uint32_t)p.Q;
      // AUX: the unit-local k-block after whose loads the aux tile is loaded
      // (an unsplit unit covers all num_kb k-blocks): late enough that the
      // previous tile's epilogue has released it, early enough that it lands
      // while the tile's last rounds are still to come
      const int aux_at = max(0, min(num_kb - 2 * NS, 3 * NS));
      uint32_t g = 0;
      uint32_t ua = 0;  // aux tiles loaded
      bool alive = true;
      for (int64_t u = blockIdx.x; u < num_units && alive; u += gridDim.x) {
        int64_t m0;
        int n0, split, r_lo, nr;
        unit_split(u, m0, n0, split, r_lo, nr);
        // im2col window base of the tile's first output pixel
        const uint32_t m32 = (uint32_t)m0;
        const uint32_t img = m32 / PQ, pq = m32 - img * PQ;
        const uint32_t pp = pq / Q, qq = pq - pp * Q;
        const int w0 = (int)(qq * p.sw) - p.pw, h0 = (int)(pp * p.sh) - p.ph;
        const int rot = r_rotation(m0, nr);
        int jj = 0;  // unit-local k-block
        for (int rr = 0; rr < nr && alive; ++rr) {
          const int r = r_lo + (rot + rr) % nr;
          const int nk = round_kbs(r);
          for (int j = 0; j < nk; ++j, ++g, ++jj) {
            const uint32_t st = g % NS;
            if (!mbar_wait_relaxed(smem_u32(&empty[st]), ((g / NS) & 1) ^ 1, abort_flag, p.status, kSleepTma)) {
              alive = false;
              break;
            }
            const uint32_t bar = smem_u32(&full[st]);
            mbar_arrive_tx(bar, three ? (uint32_t)L::kStage : (uint32_t)(L::kATile + L::kBTile));
            const uint32_t sa = smem_u32(smem + st * L::kStage);
            const int k0 = (r * rk + j) * kBK;
            if (p.a_tma == A_TMA_IM2COL) {
              const int tap = k0 / C, c0 = k0 - tap * C;  // C is a multiple of 32: one tap per k-block
              const int fr = tap / S, fs = tap - fr * S;
              tma_load_im2col_4d(sa, &tm_a, bar, c0, w0, h0, (int)img, (uint16_t)(fs * p.dw),
                                 (uint16_t)(fr * p.dh));
            } else if (p.a_tma == A_TMA_IM2COL_TAPS) {
              // 32 / C taps, each a dense [128][C] block; taps past the filter
              // repeat its last one (their B rows are the zero fill past K)
              const int tpk = kBK / C, last = p.R * S - 1;
              for (int t = 0; t < tpk; ++t) {
                const int tap = min(k0 / C + t, last);
                const int fr = tap / S, fs = tap - fr * S;
                tma_load_im2col_4d(sa + (uint32_t)(t * kBM * C * 4), &tm_a, bar, 0, w0, h0, (int)img,
                                   (uint16_t)(fs * p.dw), (uint16_t)(fr * p.dh));
              }
            } else {
              tma_load_2d(sa, &tm_a, bar, k0, (int)m0);
            }
            tma_load_3d(sa + L::kATile, &tm_hi, bar, k0, n0, 0);
            if (three) tma_load_3d(sa + L::kATile + L::kBTile, &tm_lo, bar, k0, n0, 0);
            if (AUX && jj == aux_at) {
              // the previous tile's epilogue has released the aux tile
              if (!mbar_wait_relaxed(smem_u32(aux_empty), (ua & 1) ^ 1, abort_flag, p.status, kSleepTma)) {
                alive = false;
                break;
              }
              const uint32_t xb = smem_u32(aux_full);
              mbar_arrive_tx(xb, (uint32_t)L::kAuxBytes);
              const uint32_t sx = smem_u32(smem + L::kStageOff);
#pragma unroll
              for (int b = 0; b < BN / kBK; ++b)
                tma_load_2d(sx + (uint32_t)(b * L::kAuxBox), &tm_x, xb, n0 + b * kBK, (int)m0);
              ++ua;
            }
          }
        }
      }
      if (*abort_flag && g > 0) {
        // copies already issued must land before the CTA retires (a stage
        // lands within microseconds); their phases may never be waited on
        const unsigned long long t0 = global_ns();
        while (global_ns() - t0 < 100000ull) {
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    const uint32_t idesc = bf16 ? umma_idesc_bf16<BN>() : umma_idesc_tf32<BN>();
    const uint32_t idesc2 = umma_idesc_tf32<2 * BN>();  // B's hi and lo planes as one operand
    const uint64_t desc0 = bf16 ? umma_desc_sw64(smem_u32(smem)) : umma_desc_sw128(smem_u32(smem));
    constexpr uint64_t kStageDesc = (uint64_t)(L::kStage >> 4);  // descriptor start-address units
    constexpr uint64_t kATileDesc = (uint64_t)(L::kATile >> 4);
    constexpr uint64_t kBTileDesc = (uint64_t)(L::kBTile >> 4);
    uint32_t g = 0, ar = 0;
    bool alive = true;
    for (int64_t u = blockIdx.x; u < num_units && alive; u += gridDim.x) {
      int64_t m0;
      int n0, split, r_lo, nr;
      unit_split(u, m0, n0, split, r_lo, nr);
      const int rot = r_rotation(m0, nr);
      for (int rr = 0; rr < nr && alive; ++rr, ++ar) {
        const int nk = round_kbs(r_lo + (rot + rr) % nr);
        // the round's first remr barrier includes the drain of buffer buf
        const uint32_t buf = ar & 1;
        const uint32_t tmem_d = tmem_base + buf * L::kAccCols;
        for (int j = 0; j < nk; ++j, ++g) {
          const uint32_t st = g % NS;
          if (!mbar_wait(smem_u32(&remr[st]), (g / NS) & 1, abort_flag, p.status)) {
            alive = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint64_t dbh = desc0 + (uint64_t)st * kStageDesc + kATileDesc;
            const uint64_t dbl = dbh + kBTileDesc;
            const uint32_t a_raw = tmem_base + (uint32_t)(L::kACol + st * L::kAStageCols);
            const uint32_t a_rem = a_raw + kBK;
            // a K-major SW128 descriptor advances 32 bytes (2 units) per
            // 8-wide k-step; an A column holds one k
            // the pass count is tested once per k-block, outside the issue
            // loop: the issuing thread is the kernel's critical path
            if constexpr (bf16) {
              // two 16-wide k-steps: 32 bytes of each 64-byte B row and 8 A columns (two k each) apart
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk)
                umma_bf16_ts(tmem_d, a_raw + 8 * kk, dbh + 2 * kk, idesc, (j | kk) != 0);
            } else if (three) {
#pragma unroll
              for (int kk = 0; kk < kBK / 8; ++kk) {
                const uint64_t o = (uint64_t)(2 * kk);
                const uint32_t ka = (uint32_t)(8 * kk);
                const uint32_t first = (j | kk) != 0;
                if (L::kFold) {
                  umma_tf32_ts(tmem_d, a_raw + ka, dbh + o, idesc2, first);  // [hi*hi | hi*lo]
                  umma_tf32_ts(tmem_d, a_rem + ka, dbh + o, idesc, 1);       // lo*hi
                } else {
                  umma_tf32_ts(tmem_d, a_raw + ka, dbh + o, idesc, first);
                  umma_tf32_ts(tmem_d, a_raw + ka, dbl + o, idesc, 1);
                  umma_tf32_ts(tmem_d, a_rem + ka, dbh + o, idesc, 1);
                }
              }
            } else {
#pragma unroll
              for (int kk = 0; kk < kBK / 8; ++kk)  // single pass: hi*hi
                umma_tf32_ts(tmem_d, a_raw + 8 * kk, dbh + 2 * kk, idesc, (j | kk) != 0);
            }
            umma_commit(smem_u32(&empty[st]));  // the stage may be refilled once these MMAs complete
          }
          __syncwarp();
        }
        if (!alive) break;
        if (lane == 0) umma_commit(smem_u32(&accf[buf]));  // the round's sum is complete
        __syncwarp();
      }
    }
    if (lane == 0) umma_commit(smem_u32(done));
  } else {
    // ------------------------------------------------------------------ accumulate + epilogue
    constexpr int HB = BN / 2;
    const int q = warp & 3;
    const int half = (warp - 6) / 4;
    const int cbase = half * HB;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
    uint32_t ar = 0;
    uint32_t ua = 0;  // AUX: aux tiles consumed
    bool ok = true;
    for (int64_t u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      int64_t m0;
      int n0, split, r_lo, nr;
      unit_split(u, m0, n0, split, r_lo, nr);
      const int64_t c_off = (int64_t)split * p.split_stride;  // split slice of the workspace (0 unsplit)
      float acc[HB];
#pragma unroll
      for (int j = 0; j < HB; ++j) acc[j] = 0.0f;
      int pre = 0;  // FAST_SIGMOID_MUL: 16-column chunks of the aux row already aux * sigmoid(aux)
      for (int r = 0; r < nr; ++r, ++ar) {
        const uint32_t buf = ar & 1;
        if (!__all_sync(0xffffffffu,
                        mbar_wait_relaxed(smem_u32(&accf[buf]), (ar >> 1) & 1, abort_flag, p.status, kSleepAcc))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < HB; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(lane_base + (uint32_t)(buf * L::kAccCols + cbase + c0), v);
          if (L::kFold && three) {  // the round's sum is split over the two halves
            uint32_t v2[32];
            tmem_ld32(lane_base + (uint32_t)(buf * L::kAccCols + BN + cbase + c0), v2);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              acc[c0 + j] = __fadd_rn(acc[c0 + j], __fadd_rn(__uint_as_float(v[j]), __uint_as_float(v2[j])));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[c0 + j] = __fadd_rn(acc[c0 + j], __uint_as_float(v[j]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&acce[buf]));
        if constexpr (AUX != 0 && EPI == EPI_FAST) {
          // one chunk after each of the last rounds but the final one, once
          // the aux tile has landed (tested without waiting): the tensor core
          // has two rounds of work queued meanwhile
          if (p.fast == FAST_SIGMOID_MUL && r + 1 < nr && r + 1 + (HB / 16) >= nr && pre < HB / 16 &&
              __all_sync(0xffffffffu, mbar_test(smem_u32(aux_full), ua & 1))) {
            aux_sigmoid_chunk<BN>(smem_u32(smem + L::kStageOff), warp, lane, pre);
            ++pre;
          }
        }
      }
      ok = __all_sync(0xffffffffu, ok && !*abort_flag);
      if constexpr (AUX != 0) {
        if (ok)
          ok = __all_sync(0xffffffffu,
                          mbar_wait_relaxed(smem_u32(aux_full), ua & 1, abort_flag, p.status, kSleepAcc));
        if (ok) tile_epilogue_aux<BN, EPI>(p, acc, m0, n0, warp, lane, smem_u32(smem + L::kStageOff), pre);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(aux_empty));
        ++ua;
      } else {
        tile_epilogue<BN, EPI>(p, acc, m0, n0, 0, c_off, warp, lane,
                               reinterpret_cast<float*>(smem + L::kStageOff), ok);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    // every MMA must have completed before the tensor memory is released
    volatile int never = 0;
    if (lane == 0) mbar_wait(smem_u32(done), 0, &never, p.status);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"((uint32_t)L::kTmemCols)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeIm2col_v12000 get_encode_im2col() {
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(ptr);
  });
  return fn;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

template <int BN, int EPI, int PASSES, int AUX>
bool launch_t(const ConvGemmParams& p, const void* tma, const void* tmh, const void* tml, const void* tmx,
              cudaStream_t s) {
  constexpr int NS = AUX ? TmaConfig<BN>::NS_AUX : TmaConfig<BN>::NS;
  auto kern = conv_gemm_tma_kernel<BN, NS, EPI, PASSES, AUX>;
  constexpr int smem = TmaSmem<BN, NS, AUX, PASSES>::kBytes;
  static_assert(smem <= 232448, "shared memory per CTA");
  static std::mutex mu;
  static uint64_t attr_devices = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !(attr_devices >> dev & 1)) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return false;
      attr_devices |= uint64_t(1) << dev;
    }
  }
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  const int64_t units = ((p.M + kBM - 1) / kBM) * ((p.N + BN - 1) / BN) * std::max(1, p.ksplit);
  dim3 grid((unsigned)std::min<int64_t>(units, sms), 1, 1);
  kern<<<grid, kThreadsTC, smem, s>>>(p, *static_cast<const CUtensorMap*>(tma), *static_cast<const CUtensorMap*>(tmh),
                                      *static_cast<const CUtensorMap*>(tml), *static_cast<const CUtensorMap*>(tmx));
  return true;
}

// tmx: the aux operand's tensor map, or nullptr (the epilogue reads it from
// global memory; the kernel's tm_x is then a copy of tm_a it never reads)
template <int BN, int PASSES>
bool launch_epi_p(const ConvGemmParams& p, const void* tma, const void* tmh, const void* tml, const void* tmx,
                  cudaStream_t s) {
  switch (p.epi) {
    case EPI_NONE: return launch_t<BN, EPI_NONE, PASSES, 0>(p, tma, tmh, tml, tma, s);
    case EPI_BIAS: return launch_t<BN, EPI_BIAS, PASSES, 0>(p, tma, tmh, tml, tma, s);
    case EPI_BIAS_RELU: return launch_t<BN, EPI_BIAS_RELU, PASSES, 0>(p, tma, tmh, tml, tma, s);
    case EPI_BIAS_ADD_RELU:
      return tmx ? launch_t<BN, EPI_BIAS_ADD_RELU, PASSES, 1>(p, tma, tmh, tml, tmx, s)
                 : launch_t<BN, EPI_BIAS_ADD_RELU, PASSES, 0>(p, tma, tmh, tml, tma, s);
    case EPI_PROGRAM: return launch_t<BN, EPI_PROGRAM, PASSES, 0>(p, tma, tmh, tml, tma, s);
    case EPI_FAST:
      return tmx ? launch_t<BN, EPI_FAST, PASSES, 1>(p, tma, tmh, tml, tmx, s)
                 : launch_t<BN, EPI_FAST, PASSES, 0>(p, tma, tmh, tml, tma, s);
    default: return false;
  }
}

template <int BN>
bool launch_epi(const ConvGemmParams& p, const void* tma, const void* tmh, const void* tml, const void* tmx,
                cudaStream_t s) {
  if (p.passes == 1) return launch_epi_p<BN, 1>(p, tma, tmh, tml, tmx, s);
  if (p.passes == 2) return launch_epi_p<BN, 2>(p, tma, tmh, tml, tmx, s);
  return launch_epi_p<BN, 3>(p, tma, tmh, tml, tmx, s);
}

// The aux operand of an unsplit launch as a tiled map over [M][N] (row
// stride ld), when the epilogue can take it from shared memory: the
// residual of EPI_BIAS_ADD_RELU, or the single aux tensor of an EPI_FAST
// form (FAST_SIGMOID_MUL when both of its operands are the same tensor);
// rows 16-byte aligned, unit column stride, and an output the epilogue
// stores in float4 rows.
bool make_aux_tensor_map(const ConvGemmParams& p, CUtensorMap* out) {
  if (p.ksplit > 1 || p.nb != 1 || p.ldc_n != 1 || p.ldc % 4 != 0 || (reinterpret_cast<uintptr_t>(p.out) & 15))
    return false;
  const float* src = nullptr;
  int64_t ld = 0;
  if (p.epi == EPI_BIAS_ADD_RELU && p.bias && p.res) {
    src = p.res;
    ld = p.ldc;
  } else if (p.epi == EPI_FAST && !p.bias && p.n_aux >= 1 && p.aux_sn[0] == 1 &&
             (p.fast == FAST_ADD || p.fast == FAST_DIVC_ADD || p.fast == FAST_MULC_ADD ||
              (p.fast == FAST_SIGMOID_MUL && p.n_aux >= 2 && p.aux[1] == p.aux[0] && p.aux_sm[1] == p.aux_sm[0] &&
               p.aux_sn[1] == 1))) {
    src = p.aux[0];
    ld = p.aux_sm[0];
  }
  if (!src || ld < p.N) return false;
  return make_a_tensor_map_2d(src, p.M, p.N, ld, out);
}

}  // namespace

bool conv_gemm_tma_aux_ok(const ConvGemmParams& p) {
  CUtensorMap m;
  return make_aux_tensor_map(p, &m);
}

int conv_gemm_tma_smem_bytes(int block_n) {
  return block_n == 64 ? TmaSmem<64, TmaConfig<64>::NS>::kBytes : TmaSmem<128, TmaConfig<128>::NS>::kBytes;
}

bool make_a_tensor_map_im2col(const float* x, int64_t images, int64_t H, int64_t W, int64_t C, int64_t x_sn,
                              int64_t x_sh, int64_t x_sw, int R, int S, int sh, int sw, int ph, int pw, int dh,
                              int dw, void* tmap_out, int* mode) {
  auto enc = get_encode_im2col();
  if (!enc) return false;
  const bool taps = C == 4 || C == 8 || C == 16;
  if ((C % kBK != 0 && !taps) || (reinterpret_cast<uintptr_t>(x) & 15)) return false;
  if (images == 1 && x_sn == 0) x_sn = x_sh * H;  // a size-1 dimension: any valid stride
  if (x_sw % 4 || x_sh % 4 || x_sn % 4 || x_sw <= 0 || x_sh <= 0 || x_sn <= 0) return false;
  // bounding box of the window bases: [-pad, dim - 1 + pad - dilation * (filter - 1)],
  // traversed with the convolution stride (one position per output pixel)
  const int lower[2] = {-pw, -ph};
  const int upper[2] = {pw - dw * (S - 1), ph - dh * (R - 1)};
  for (int i = 0; i < 2; ++i)
    if (lower[i] < -128 || lower[i] > 127 || upper[i] < -128 || upper[i] > 127) return false;
  if (dw * (S - 1) > 255 || dh * (R - 1) > 255 || sw > 8 || sh > 8 || sw < 1 || sh < 1) return false;
  cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)images};
  cuuint64_t strides[3] = {(cuuint64_t)(x_sw * 4), (cuuint64_t)(x_sh * 4), (cuuint64_t)(x_sn * 4)};
  cuuint32_t estr[4] = {1, (cuuint32_t)sw, (cuuint32_t)sh, 1};
  // a tap block of C channels is C * 4 bytes per pixel (16, 32 or 64): dense rows, no swizzle
  CUresult r = enc(static_cast<CUtensorMap*>(tmap_out), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(x),
                   dims, strides, lower, upper, (cuuint32_t)(taps ? C : kBK), (cuuint32_t)kBM, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, taps ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (mode) *mode = taps ? A_TMA_IM2COL_TAPS : A_TMA_IM2COL;
  return true;
}

bool make_a_tensor_map_2d(const float* x, int64_t M, int64_t K, int64_t ld, void* tmap_out) {
  auto enc = get_encode_tiled();
  if (!enc) return false;
  if (M == 1 && ld == 0) ld = (K + 3) / 4 * 4;
  if (ld % 4 || ld < K || (reinterpret_cast<uintptr_t>(x) & 15)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(static_cast<CUtensorMap*>(tmap_out), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x),
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool launch_conv_gemm_tma(const ConvGemmParams& p_in, const void* tmap_a, const void* tmap_hi, const void* tmap_lo,
                          int block_n, cudaStream_t s) {
  ConvGemmParams p = p_in;
  if (p.M <= 0 || p.N <= 0) return true;
  if (p.rk <= 0) p.rk = kRK;
  if (p.rk > 16) return false;
  if (p.passes == 0) p.passes = 3;
  if (p.passes < 1 || p.passes > 3) return false;
  if (p.K <= 0 || p.nb != 1 || (p.a_tma != A_TMA_2D && p.a_tma != A_TMA_IM2COL && p.a_tma != A_TMA_IM2COL_TAPS))
    return false;
  if (p.a_tma == A_TMA_IM2COL && p.C % kBK != 0) return false;
  if (p.a_tma == A_TMA_IM2COL_TAPS && p.C != 4 && p.C != 8 && p.C != 16) return false;
  if (p.ksplit > 1) {
    const int rounds = (int)(((p.K + kBK - 1) / kBK + p.rk - 1) / p.rk);
    if (!p.ws || p.epi > EPI_BIAS_ADD_RELU || p.ksplit > rounds) return false;
    p.out = p.ws;  // raw partial sums into the workspace slices
    p.ldc = p.N;
    p.ldc_n = 1;
    p.epi = EPI_NONE;
    p.split_stride = p.M * p.N;
  } else {
    p.ksplit = 1;
    p.split_stride = 0;
  }
  const int64_t units = ((p.M + kBM - 1) / kBM) * ((p.N + block_n - 1) / block_n) * p.ksplit;
  if (p.M >= (int64_t(1) << 31) || units >= (int64_t(1) << 31) || p.P * p.Q >= (int64_t(1) << 31)) return false;
  CUtensorMap xmap;
  const void* tmap_x = p.aux_tma && make_aux_tensor_map(p, &xmap) ? &xmap : nullptr;
  bool ok = false;
  if (block_n == 64) ok = launch_epi<64>(p, tmap_a, tmap_hi, tmap_lo, tmap_x, s);
  else if (block_n == 128) ok = launch_epi<128>(p, tmap_a, tmap_hi, tmap_lo, tmap_x, s);
  if (!ok) return false;
  if (p.ksplit > 1) launch_splitk_reduce(p_in, p.split_stride, s);
  return true;
}

}  // namespace kern
}  // namespace gawee
