// Tensor-core implicit-GEMM convolution and (batched) GEMM for sm_100a.
//
// One CTA computes a 128 x BN tile of C = A . B^T with fp32 accuracy from
// TF32 tensor cores: three tcgen05.mma per k-step (hi*hi + hi*lo + lo*hi; see
// Ootomo & Yokota, "Recovering single precision accuracy from Tensor Cores
// while surpassing the FP32 theoretical peak performance", 2022).  The tensor
// core reads an fp32 operand as TF32 by dropping its 13 low mantissa bits, so
// the raw value serves as the high part and only the remainder x - tf32(x)
// is formed explicitly.
//
// The tensor core's fp32 accumulation truncates (Fasi et al., "Numerical
// behavior of NVIDIA tensor cores", 2021), so over thousands of k-steps its
// error grows linearly with K.  Each 64-wide round (two k-blocks) is
// therefore accumulated alone in a tensor-memory buffer, and the accumulator
// warps add the round sums into fp32 registers with IEEE round-to-nearest
// while later rounds are multiplied into the other buffer.
//
// Operands: A (im2col rows of the NHWC input, or GEMM rows) lives in tensor
// memory, B (pre-split weight planes) in shared memory, so the MMAs read only
// B through the shared-memory port (tcgen05.mma with [a-tmem]).
//
// Warp roles (448 threads), persistent over output tiles (one CTA per SM):
//   warps 0-3  copy the A rows with cp.async into a shared-memory ring several
//              k-blocks ahead (zero padding and K tails by zero-fill), then
//              write raw values and remainders into the A stage in tensor
//              memory with tcgen05.st (warp w owns TMEM lanes 32w..32w+31)
//   warp 4     issues the TMA loads of the B planes; owns the TMEM allocation
//   warp 5     lane 0 issues tcgen05.mma and the tcgen05.commit that track them
//   warps 6-13 accumulate block sums from TMEM (two warps per TMEM lane
//              quarter, each owning half the tile's columns) and run the
//              epilogue of tile t while the MMAs of tile t+1 proceed
// Stage hand-off uses mbarriers; every wait is bounded in time and on expiry
// records ST_BARRIER_TIMEOUT in the status word and lets the CTA finish.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <cstdio>
#include <mutex>

#include "kernels.h"
#include "program.cuh"
#include "tc_common.cuh"

namespace gawee {
namespace kern {

namespace {

// Round slots: each of the kS slots holds one round's A stage (tensor
// memory), B stage (shared memory) and accumulator (tensor memory), so one
// barrier per slot says "everything for this round is ready".
constexpr int kS = 2;
// Raw A k-blocks in flight per tile width.  Shared memory: 2 x 32 KB + 8 x
// 16 KB for BN 64, 2 x 64 KB + 4 x 16 KB for BN 128, plus 20 KB of epilogue
// staging; tensor memory: 2 x 64 + 2 x 128 and 2 x 128 + 2 x 128 of its 512
// columns.
template <int BN>
struct TcConfig;
template <>
struct TcConfig<64> {
  static constexpr int RD = 8;
};
template <>
struct TcConfig<128> {
  static constexpr int RD = 4;
};
// Shared memory: kS B stages (per round: kRK k-blocks of hi and lo planes,
// TMA), RD raw A k-blocks (cp.async ring, 128 rows x 128 B, 16-byte chunks
// swizzled by row), then the barriers.  Tensor memory: kS round accumulators
// of BN columns, then kS A stages of kRK x 64 columns (per k-block 32 raw
// values and 32 remainders; lane = row).
template <int BN, int RD>
struct Smem {
  static constexpr int kATile = kBM * kBK * 4;  // 16 KB
  static constexpr int kBTile = BN * kBK * 4;
  static constexpr int kBStage = kRK * 2 * kBTile;
  static constexpr int kRawOff = kS * kBStage;
  static constexpr int kStageOff = kRawOff + RD * kATile;
  static constexpr int kBarOff = kStageOff + 8 * kStageWarpFloats * 4;
  static constexpr int kNumBars = 2 * kS + 1;  // ready, done per slot; all MMAs done
  static constexpr int kBytes = kBarOff + 8 * kNumBars + 16 + 1024;  // + alignment slack
  // BN 64 folds two passes into one N = 128 MMA (see the MMA issuer), so its
  // round accumulator spans 2 x BN columns.
  static constexpr bool kFold = BN == 64;
  static constexpr int kAccCols = kFold ? 2 * BN : BN;
  static constexpr int kACol = kS * kAccCols;
  static constexpr int kAStageCols = kRK * 2 * kBK;
  static constexpr int kUsedCols = kS * kAccCols + kS * kAStageCols;
  static constexpr int kTmemCols = kUsedCols <= 256 ? 256 : 512;
  static_assert(kUsedCols <= 512, "tensor memory columns");
};

// Arrivals that complete a slot's "ready" phase: 4 A producer warps, the TMA
// thread (plus the B transaction bytes) and 8 accumulator warps (the slot's
// accumulator has been drained).
constexpr int kReadyCount = 4 + 1 + 8;

}  // namespace

template <int BN, int RD, int EPI>
__global__ void __launch_bounds__(kThreadsTC, 1)
    conv_gemm_tc_kernel(const __grid_constant__ ConvGemmParams p, const __grid_constant__ CUtensorMap tm_hi,
                        const __grid_constant__ CUtensorMap tm_lo) {
  using L = Smem<BN, RD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  // Round g uses slot g % kS.  ready[s]: A written, B landed, accumulator
  // drained (kReadyCount arrivals + B bytes); done[s]: the round's MMAs have
  // completed (one tcgen05.commit), so its A stage, B stage and accumulator
  // may be read or reused.
  uint64_t* ready = bars;
  uint64_t* rdone = bars + kS;
  uint64_t* done = bars + 2 * kS;  // every MMA issued by this CTA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const bool three = p.passes != 1;  // fp32 from three TF32 products (else one)
  const int num_kb = (int)((p.K + kBK - 1) / kBK);
  const int num_rounds = (num_kb + kRK - 1) / kRK;
  auto round_kbs = [&](int r) { return min(kRK, num_kb - r * kRK); };
  const int64_t m_tiles = (p.M + kBM - 1) / kBM;
  const int64_t n_tiles = (p.N + BN - 1) / BN;
  const int64_t num_tiles = m_tiles * n_tiles * p.nb;
  // Work units: (tile, k split).  With p.ksplit = S > 1 the rounds of a tile
  // are cut into S contiguous ranges and unit u covers tile u % tiles over
  // range u / tiles, writing its partial sums to split slice u / tiles of the
  // output (a workspace the launcher reduces in split order).  Consecutive
  // units share their k range, so CTAs running together read the same part
  // of the B operand.
  const int ksplit = p.ksplit > 1 ? p.ksplit : 1;
  const int64_t num_units = num_tiles * ksplit;
  const uint32_t tiles32 = (uint32_t)num_tiles;
  auto unit_split = [&](int64_t u, int64_t& t, int& split, int& r_lo, int& nr) {
    const uint32_t uu = (uint32_t)u;
    const uint32_t sp = uu / tiles32;
    t = (int64_t)(uu - sp * tiles32);
    split = (int)sp;
    r_lo = (int)(((int64_t)sp * num_rounds) / ksplit);
    nr = (int)(((int64_t)(sp + 1) * num_rounds) / ksplit) - r_lo;
  };

  // Tile t -> (z, n tile, m tile), m fastest so CTAs running together share B.
  // Tile, row and batch coordinates fit in 32 bits (the launcher checks), so
  // their divisions use 32-bit arithmetic.
  const uint32_t m_tiles32 = (uint32_t)m_tiles, n_tiles32 = (uint32_t)n_tiles;
  auto tile_coords = [&](int64_t t, int64_t& m0, int& n0, int& z) {
    const uint32_t tt = (uint32_t)t;
    const uint32_t mn = tt / m_tiles32;
    m0 = (int64_t)(tt - mn * m_tiles32) * kBM;
    const uint32_t zz = mn / n_tiles32;
    n0 = (int)((mn - zz * n_tiles32) * BN);
    z = (int)zz;
  };
  // Each unit walks its rounds starting at (m tile index mod its round
  // count): CTAs that run side by side then fetch different k-blocks of the
  // shared B operand instead of all hitting the same L2 lines at once.
  auto r_rotation = [&](int64_t t, int nr) -> int { return (int)(((uint32_t)t % m_tiles32) % (uint32_t)nr); };
  auto batch_offsets = [&](int z, int64_t& a_off, int64_t& c_off, int& b_plane) {
    a_off = 0;
    c_off = 0;
    b_plane = 0;
    uint32_t rem = (uint32_t)z;
    for (int d = p.batch_rank - 1; d >= 0; --d) {
      const uint32_t sh = (uint32_t)p.batch_shape[d];
      const uint32_t q = rem / sh;
      const int64_t c = rem - q * sh;
      rem = q;
      a_off += c * p.a_bst[d];
      c_off += c * p.c_bst[d];
      b_plane += (int)(c * p.b_bst[d]);
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(smem_u32(&ready[s]), kReadyCount);
      mbar_init(smem_u32(&rdone[s]), 1);
    }
    mbar_init(smem_u32(done), 1);
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
    // ------------------------------------------------------------------ A producer
    // Warp w owns rows 32w..32w+31 of every A tile: the tensor-memory lanes
    // it may write.  Its lanes copy those rows with cp.async in 16-byte
    // chunks (lane -> chunk lane%8 of rows i*4 + lane/8, so each instruction
    // reads four whole 128-byte rows) into a ring of RD raw k-blocks that
    // only this warp touches, RD k-blocks ahead.  Then each lane takes its
    // own row, stores the raw values (the tensor core reads fp32 as TF32 by
    // dropping the low 13 mantissa bits, so raw is the high part) and the
    // remainders x - tf32(x) into the A stage in tensor memory.
    const int chunk = lane & 7;
    const int rsub = lane >> 3;
    const int64_t PQ = p.P * p.Q;
    const uint32_t raw_base = smem_u32(smem + L::kRawOff);
    const uint32_t tmem_rows = tmem_base + ((uint32_t)(warp * 32) << 16);

    // load cursor: unit, k-block, and the chunk's (c, r, s) within the filter window
    int64_t lu = blockIdx.x;  // unit being loaded
    int lkb = 0;              // k-blocks of the current unit issued so far
    int lka = 0;              // the k-block they are at (rotated order)
    int l_kb_lo = 0, l_kb_hi = 0;  // the unit's k-block range
    int64_t li = 0;
    int64_t rowoff[8];
    int ih0[8], iw0[8];
    int kc = 0, kr = 0, ks = 0;
    const int H = (int)p.H, W = (int)p.W, C = (int)p.C;
    // When C divides kBK (the 7x7 stem's four padded channels), a k-block
    // moves kBK / C whole filter taps and the channel offset stays put.
    const int tap_step = (C < kBK && kBK % C == 0) ? kBK / C : 0;
    auto decompose = [&](int k) {
      const int rs = k / C;
      kc = k - rs * C;
      kr = rs / p.S;
      ks = rs - kr * p.S;
    };
    auto start_tile = [&]() {
      int64_t m0, a_off, c_off, lt;
      int n0, z, b_plane, lsplit, lr_lo, lnr;
      unit_split(lu, lt, lsplit, lr_lo, lnr);
      l_kb_lo = lr_lo * kRK;
      l_kb_hi = min((lr_lo + lnr) * kRK, num_kb);
      tile_coords(lt, m0, n0, z);
      batch_offsets(z, a_off, c_off, b_plane);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t m = m0 + warp * 32 + i * 4 + rsub;
        if (m < p.M) {
          const uint32_t m32 = (uint32_t)m, PQ32 = (uint32_t)PQ, Q32 = (uint32_t)p.Q;
          const uint32_t img32 = m32 / PQ32, pq = m32 - img32 * PQ32;
          const uint32_t pp = pq / Q32, qq = pq - pp * Q32;
          const int64_t img = img32;
          ih0[i] = (int)(pp * p.sh - p.ph);
          iw0[i] = (int)(qq * p.sw - p.pw);
          rowoff[i] = a_off + img * p.x_sn + (int64_t)ih0[i] * p.x_sh + (int64_t)iw0[i] * p.x_sw;
        } else {
          ih0[i] = INT_MIN / 2;  // fails every bounds test
          iw0[i] = 0;
          rowoff[i] = 0;
        }
      }
      lka = l_kb_lo + r_rotation(lt, lnr) * kRK;
      decompose(lka * kBK + chunk * 4);
    };
    auto issue = [&]() {
      if (lu < num_units) {
        if (lkb == 0) start_tile();
        const uint32_t slot = raw_base + (uint32_t)((li % RD) * L::kATile);
        const bool kin = (int64_t)lka * kBK + chunk * 4 < p.K;
        const int dr = kr * p.dh, ds = ks * p.dw;
        const int64_t koff = (int64_t)dr * p.x_sh + (int64_t)ds * p.x_sw + kc;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int row = warp * 32 + i * 4 + rsub;
          const bool ok = kin && (unsigned)(ih0[i] + dr) < (unsigned)H && (unsigned)(iw0[i] + ds) < (unsigned)W;
          cp_async16(slot + row * 128 + ((chunk ^ (row & 7)) << 4),
                     ok ? (const void*)(p.x + rowoff[i] + koff) : (const void*)p.x, ok ? 16u : 0u);
        }
        // next k-block of the same chunk: k advances by 32 (wrapping to the
        // start of the unit's range)
        if (++lkb == l_kb_hi - l_kb_lo) {
          lkb = 0;
          lu += gridDim.x;
        } else if (++lka == l_kb_hi) {
          lka = l_kb_lo;
          decompose(lka * kBK + chunk * 4);
        } else if (tap_step) {
          ks += tap_step;
          while (ks >= p.S) {
            ks -= p.S;
            ++kr;
          }
        } else if (C < kBK) {
          decompose(lka * kBK + chunk * 4);  // k crosses several (r, s) positions: divide directly
        } else {
          kc += kBK;
          while (kc >= C) {
            kc -= C;
            if (++ks == p.S) {
              ks = 0;
              ++kr;
            }
          }
        }
      }
      cp_async_commit();  // empty groups past the end keep the group count uniform
      ++li;
    };

    const int row = warp * 32 + lane;
#pragma unroll
    for (int j = 0; j < RD; ++j) issue();
    int64_t g = 0;        // k-blocks consumed
    int sa = 0;           // round slot
    uint32_t free_ph = 1;  // parity of the slot's previous round completing (fresh: passes)
    bool alive = true;
    for (int64_t u = blockIdx.x; u < num_units && alive; u += gridDim.x) {
      int64_t t;
      int split, r_lo, nr;
      unit_split(u, t, split, r_lo, nr);
      const int rot = r_rotation(t, nr);
      for (int rr = 0; rr < nr && alive; ++rr) {
        int r = rot + rr;
        if (r >= nr) r -= nr;
        r += r_lo;
        const int nk = round_kbs(r);
        if (!mbar_wait(smem_u32(&rdone[sa]), free_ph, abort_flag, p.status)) {
          alive = false;
          break;
        }
        tc_fence_after();
        for (int j = 0; j < nk; ++j, ++g) {
          cp_async_wait<RD - 1>();  // this lane's copies of k-block g have landed
          __syncwarp();             // ... and every other lane's
          const uint32_t src = raw_base + (uint32_t)((g % RD) * L::kATile) + row * 128;
          uint32_t x[32];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 v = lds128(src + ((c ^ (row & 7)) << 4));
            x[4 * c] = __float_as_uint(v.x);
            x[4 * c + 1] = __float_as_uint(v.y);
            x[4 * c + 2] = __float_as_uint(v.z);
            x[4 * c + 3] = __float_as_uint(v.w);
          }
          const uint32_t acol = tmem_rows + (uint32_t)(L::kACol + sa * L::kAStageCols + j * 2 * kBK);
          tmem_st32(acol, x);
          uint32_t y[32];  // remainders (formed in both modes; stored for three passes)
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            const float v = __uint_as_float(x[q]);
            y[q] = __float_as_uint(__fsub_rn(v, tf32_hi(v)));
          }
          __syncwarp();  // every lane has read its row: the slot may be refilled
          issue();
          if (three) tmem_st32(acol + kBK, y);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ready[sa]));
        if (++sa == kS) {
          sa = 0;
          free_ph ^= 1;
        }
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // nothing of this thread in flight at exit
  } else if (warp == 4) {
    // ------------------------------------------------------------------ B producer (TMA)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_hi)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_lo)) : "memory");
      int64_t g = 0;
      int sb = 0;
      uint32_t free_ph = 1;
      bool alive = true;
      for (int64_t u = blockIdx.x; u < num_units && alive; u += gridDim.x) {
        int64_t m0, a_off, c_off, t;
        int n0, z, b_plane, split, r_lo, nr;
        unit_split(u, t, split, r_lo, nr);
        tile_coords(t, m0, n0, z);
        batch_offsets(z, a_off, c_off, b_plane);
        const int rot = r_rotation(t, nr);
        for (int rr = 0; rr < nr; ++rr) {
          int r = rot + rr;
          if (r >= nr) r -= nr;
          r += r_lo;
          const int nk = round_kbs(r);
          if (!mbar_wait(smem_u32(&rdone[sb]), free_ph, abort_flag, p.status)) {
            alive = false;
            break;
          }
          const uint32_t bar = smem_u32(&ready[sb]);
          mbar_arrive_tx(bar, (uint32_t)(nk * (three ? 2 : 1) * L::kBTile));
          for (int j = 0; j < nk; ++j) {
            uint8_t* b_hi = smem + sb * L::kBStage + j * 2 * L::kBTile;
            uint8_t* b_lo = b_hi + L::kBTile;
            const int kb = r * kRK + j;
            tma_load_3d(smem_u32(b_hi), &tm_hi, bar, kb * kBK, n0, b_plane);
            if (three) tma_load_3d(smem_u32(b_lo), &tm_lo, bar, kb * kBK, n0, b_plane);
          }
          ++g;
          if (++sb == kS) {
            sb = 0;
            free_ph ^= 1;
          }
        }
      }
      if (*abort_flag && g > 0) {
        // Copies already in flight must land before the CTA retires; their
        // barrier phase may never complete once other roles have stopped, so
        // wait a fixed 100 us (a B stage lands within microseconds).
        const unsigned long long t0 = global_ns();
        while (global_ns() - t0 < 100000ull) {
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (its values stay warp-uniform); lane 0
    // issues the MMAs and the commits that track them.  A comes from tensor
    // memory (raw and remainder columns), B from shared memory.
    const uint32_t idesc = umma_idesc_tf32<BN>();
    const uint32_t idesc2 = umma_idesc_tf32<2 * BN>();  // B's hi and lo planes as one operand
    const uint64_t desc0 = umma_desc_sw128(smem_u32(smem));
    constexpr uint64_t kBStageDesc = (uint64_t)(L::kBStage >> 4);  // descriptor start-address units
    constexpr uint64_t kBTileDesc = (uint64_t)(L::kBTile >> 4);
    int sl = 0;            // round slot
    uint32_t rdy_ph = 0;   // parity of the slot's ready phase for this round
    bool alive = true;
    for (int64_t u = blockIdx.x; u < num_units && alive; u += gridDim.x) {
      int64_t t;
      int split, r_lo, nr;
      unit_split(u, t, split, r_lo, nr);
      const int rot = r_rotation(t, nr);
      for (int rr = 0; rr < nr; ++rr) {
        int r = rot + rr;
        if (r >= nr) r -= nr;
        r += r_lo;
        const int nk = round_kbs(r);
        if (!mbar_wait(smem_u32(&ready[sl]), rdy_ph, abort_flag, p.status)) {
          alive = false;
          break;
        }
        tc_fence_after();
        // the start address of a K-major SW128 descriptor advances 32 bytes
        // (2 units) per 8-wide k-step; an A column holds one k
        const uint32_t tmem_d = tmem_base + (uint32_t)(sl * L::kAccCols);
        if (lane == 0) {
          for (int j = 0; j < nk; ++j) {
            const uint64_t dbh = desc0 + (uint64_t)sl * kBStageDesc + (uint64_t)j * 2 * kBTileDesc;
            const uint64_t dbl = dbh + kBTileDesc;
            const uint32_t a_raw = tmem_base + (uint32_t)(L::kACol + sl * L::kAStageCols + j * 2 * kBK);
            const uint32_t a_rem = a_raw + kBK;
            if (!three) {  // single pass: hi*hi (tested once per k-block, outside the issue loop)
#pragma unroll
              for (int kk = 0; kk < kBK / 8; ++kk)
                umma_tf32_ts(tmem_d, a_raw + 8 * kk, dbh + 2 * kk, idesc, (j | kk) != 0);
              continue;
            }
#pragma unroll
            for (int kk = 0; kk < kBK / 8; ++kk) {
              const uint64_t o = (uint64_t)(2 * kk);
              const uint32_t ka = (uint32_t)(8 * kk);
              if (L::kFold) {
                // The B stage holds the hi plane's BN rows directly followed by
                // the lo plane's, so one N = 2*BN MMA gives [hi*hi | hi*lo];
                // lo*hi (N = BN) accumulates into the first half.  An M = 128
                // MMA costs nearly the same for N = 64 and 128, so this issues
                // two MMAs per k-step instead of three.
                umma_tf32_ts(tmem_d, a_raw + ka, dbh + o, idesc2, (j | kk) != 0);
                umma_tf32_ts(tmem_d, a_rem + ka, dbh + o, idesc, 1);
              } else {
                umma_tf32_ts(tmem_d, a_rem + ka, dbh + o, idesc, (j | kk) != 0);
                umma_tf32_ts(tmem_d, a_raw + ka, dbl + o, idesc, 1);
                umma_tf32_ts(tmem_d, a_raw + ka, dbh + o, idesc, 1);
              }
            }
          }
          umma_commit(smem_u32(&rdone[sl]));
        }
        __syncwarp();
        if (++sl == kS) {
          sl = 0;
          rdy_ph ^= 1;
        }
      }
    }
    if (lane == 0) umma_commit(smem_u32(done));
  } else {
    // ------------------------------------------------------------------ accumulate + epilogue
    // warps 6..13: lane quarter (warp % 4) is fixed by the hardware; two
    // warps share a quarter and split the tile's columns in halves
    constexpr int HB = BN / 2;
    const int q = warp & 3;
    const int half = (warp - 6) / 4;
    const int cbase = half * HB;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
    int sl = 0;
    uint32_t done_ph = 0;
    bool ok = true;
    // every accumulator starts drained: count toward the first round of each slot
    if (lane == 0)
      for (int k = 0; k < kS; ++k) mbar_arrive(smem_u32(&ready[k]));
    for (int64_t u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      int64_t m0, a_off, c_off, t;
      int n0, z, b_plane, split, r_lo, nr;
      unit_split(u, t, split, r_lo, nr);
      tile_coords(t, m0, n0, z);
      batch_offsets(z, a_off, c_off, b_plane);
      c_off += (int64_t)split * p.split_stride;  // partial sums: this split's slice of the workspace
      float acc[HB];
#pragma unroll
      for (int j = 0; j < HB; ++j) acc[j] = 0.0f;
      for (int r = 0; r < nr; ++r) {
        const int buf = sl;
        // warp-uniform outcome: the epilogue below uses warp-collective steps
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&rdone[sl]), done_ph, abort_flag, p.status))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < HB; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(lane_base + (uint32_t)(buf * L::kAccCols + cbase + c0), r);
          if (L::kFold && three) {  // the round's sum is split over the two halves
            uint32_t r2[32];
            tmem_ld32(lane_base + (uint32_t)(buf * L::kAccCols + BN + cbase + c0), r2);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              acc[c0 + j] = __fadd_rn(acc[c0 + j], __fadd_rn(__uint_as_float(r[j]), __uint_as_float(r2[j])));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[c0 + j] = __fadd_rn(acc[c0 + j], __uint_as_float(r[j]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ready[sl]));  // the accumulator is free for round + kS
        if (++sl == kS) {
          sl = 0;
          done_ph ^= 1;
        }
      }
      ok = __all_sync(0xffffffffu, ok && !*abort_flag);
      tile_epilogue<BN, EPI>(p, acc, m0, n0, z, c_off, warp, lane,
                             reinterpret_cast<float*>(smem + L::kStageOff), ok);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    // every MMA must have completed before the accumulator memory is released
    volatile int never = 0;
    if (lane == 0) mbar_wait(smem_u32(done), 0, &never, p.status);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"((uint32_t)L::kTmemCols)
                 : "memory");
  }
}

// Split-K reduction: out = epilogue(sum over splits of ws[s]) in split order
// (deterministic), with the same epilogue operations as the tensor-core
// kernel: acc + bias[n], + res[m][n], max(., 0).  Four columns per thread.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const __grid_constant__ ConvGemmParams p) {
  const int64_t n4 = (p.N + 3) / 4;
  const int64_t total = p.M * n4;
  const bool vin = (p.N & 3) == 0;
  const bool vout = vin && p.ldc_n == 1 && (p.ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
                    (p.epi != EPI_BIAS_ADD_RELU || (reinterpret_cast<uintptr_t>(p.res) & 15) == 0);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / n4;
    const int64_t n = (i - m * n4) * 4;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    for (int sp = 0; sp < p.ksplit; ++sp) {
      const float* w = p.ws + sp * p.split_stride + m * p.N + n;
      if (vin) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(w));
        x[0] = __fadd_rn(x[0], v.x); x[1] = __fadd_rn(x[1], v.y);
        x[2] = __fadd_rn(x[2], v.z); x[3] = __fadd_rn(x[3], v.w);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (n + e < p.N) x[e] = __fadd_rn(x[e], __ldg(w + e));
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (n + e >= p.N) continue;
      if (p.epi >= EPI_BIAS) x[e] = __fadd_rn(x[e], __ldg(p.bias + n + e));
      if (p.epi == EPI_BIAS_ADD_RELU) x[e] = __fadd_rn(x[e], __ldg(p.res + m * p.ldc + (n + e) * p.ldc_n));
      if (p.epi == EPI_BIAS_RELU || p.epi == EPI_BIAS_ADD_RELU) x[e] = maximumf_(x[e], 0.0f);
    }
    float* o = p.out + m * p.ldc;
    if (vout) {
      *reinterpret_cast<float4*>(o + n) = make_float4(x[0], x[1], x[2], x[3]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (n + e < p.N) o[(n + e) * p.ldc_n] = x[e];
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

template <int BN, int EPI>
bool launch_t(const ConvGemmParams& p, const void* tmh, const void* tml, cudaStream_t s) {
  using Cfg = TcConfig<BN>;
  auto kern = conv_gemm_tc_kernel<BN, Cfg::RD, EPI>;
  constexpr int smem = Smem<BN, Cfg::RD>::kBytes;
  static_assert(smem <= 232448, "shared memory per CTA");
  // the shared-memory opt-in is per device
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
  const int64_t units = ((p.M + kBM - 1) / kBM) * ((p.N + BN - 1) / BN) * p.nb * std::max(1, p.ksplit);
  dim3 grid((unsigned)std::min<int64_t>(units, sms), 1, 1);
  kern<<<grid, kThreadsTC, smem, s>>>(p, *static_cast<const CUtensorMap*>(tmh), *static_cast<const CUtensorMap*>(tml));
  return true;
}

template <int BN>
bool launch_epi(const ConvGemmParams& p, const void* tmh, const void* tml, cudaStream_t s) {
  switch (p.epi) {
    case EPI_NONE: return launch_t<BN, EPI_NONE>(p, tmh, tml, s);
    case EPI_BIAS: return launch_t<BN, EPI_BIAS>(p, tmh, tml, s);
    case EPI_BIAS_RELU: return launch_t<BN, EPI_BIAS_RELU>(p, tmh, tml, s);
    case EPI_BIAS_ADD_RELU: return launch_t<BN, EPI_BIAS_ADD_RELU>(p, tmh, tml, s);
    case EPI_PROGRAM: return launch_t<BN, EPI_PROGRAM>(p, tmh, tml, s);
    case EPI_FAST: return launch_t<BN, EPI_FAST>(p, tmh, tml, s);
    default: return false;
  }
}

}  // namespace

int conv_gemm_smem_bytes(int block_n) {
  using C64 = TcConfig<64>;
  using C128 = TcConfig<128>;
  return block_n == 64 ? Smem<64, C64::RD>::kBytes : Smem<128, C128::RD>::kBytes;
}

bool make_b_tensor_maps(const float* hi, const float* lo, int64_t batch, int64_t N, int64_t ldk, int block_n,
                        void* tmap_hi_out, void* tmap_lo_out) {
  auto enc = get_encode();
  if (!enc) return false;
  if (ldk % 4 != 0 || (reinterpret_cast<uintptr_t>(hi) & 15) || (reinterpret_cast<uintptr_t>(lo) & 15)) return false;
  cuuint64_t dims[3] = {(cuuint64_t)ldk, (cuuint64_t)N, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ldk * 4), (cuuint64_t)(N * ldk * 4)};
  cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)block_n, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  for (int k = 0; k < 2; ++k) {
    CUtensorMap* m = static_cast<CUtensorMap*>(k == 0 ? tmap_hi_out : tmap_lo_out);
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(k == 0 ? hi : lo), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
  }
  return true;
}

bool make_b_tensor_map_bf16(const void* plane, int64_t batch, int64_t N, int64_t ldk16, int block_n,
                            void* tmap_out) {
  auto enc = get_encode();
  if (!enc) return false;
  if (ldk16 % 8 != 0 || (reinterpret_cast<uintptr_t>(plane) & 15)) return false;
  cuuint64_t dims[3] = {(cuuint64_t)ldk16, (cuuint64_t)N, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ldk16 * 2), (cuuint64_t)(N * ldk16 * 2)};
  cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)block_n, 1};  // 32 bf16: one 64-byte swizzled row
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(static_cast<CUtensorMap*>(tmap_out), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(plane),
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int choose_ksplit(int64_t M, int64_t N, int64_t K, int nb, int block_n, int epi, int sms, int rk) {
  if (nb != 1 || epi > EPI_BIAS_ADD_RELU || M <= 0 || N <= 0 || K <= 0 || sms <= 0 || rk <= 0) return 1;
  const int64_t tiles = ((M + kBM - 1) / kBM) * ((N + block_n - 1) / block_n);
  const int rounds = (int)(((K + kBK - 1) / kBK + rk - 1) / rk);
  // Estimated time in rounds: waves of units x (rounds per unit + the fixed
  // cost of a unit: pipeline fill and epilogue, about 1.5 rounds), plus the
  // reduce pass (about half a round per extra split of a tile's outputs).
  auto cost = [&](int S) {
    const int64_t units = tiles * S;
    const int64_t waves = (units + sms - 1) / sms;
    const double per = (double)((rounds + S - 1) / S) + 1.5;
    return (double)waves * per + (S > 1 ? 0.5 + 0.25 * S : 0.0);
  };
  int best = 1;
  double best_cost = cost(1);
  for (int S = 2; S <= std::min(rounds, 32); ++S) {
    const double c = cost(S);
    if (c < best_cost * 0.97) {  // a split must win clearly to pay for its workspace traffic
      best = S;
      best_cost = c;
    }
  }
  return best;
}

bool launch_conv_gemm_tc(const ConvGemmParams& p_in, const void* tmap_hi, const void* tmap_lo, int block_n,
                         cudaStream_t s) {
  ConvGemmParams p = p_in;
  if (p.M <= 0 || p.N <= 0 || p.nb <= 0) return true;
  if (p.passes == 0) p.passes = 3;
  if (p.passes != 1 && p.passes != 3) return false;
  if (p.ksplit > 1) {
    const int rounds = (int)(((p.K + kBK - 1) / kBK + kRK - 1) / kRK);
    if (!p.ws || p.nb != 1 || p.epi > EPI_BIAS_ADD_RELU || p.ksplit > rounds) return false;
    // the tensor-core pass writes raw partial sums into the workspace slices
    p.out = p.ws;
    p.ldc = p.N;
    p.ldc_n = 1;
    p.epi = EPI_NONE;
    p.split_stride = p.M * p.N;
  } else {
    p.ksplit = 1;
    p.split_stride = 0;
  }
  if (p.K <= 0) return false;  // an empty reduction would leave tensor memory unwritten
  // 16-byte A gathers need channel counts and strides in whole float4s
  if (p.C % 4 != 0 || p.x_sh % 4 != 0 || p.x_sw % 4 != 0 || p.x_sn % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(p.x) & 15))
    return false;
  for (int d = 0; d < p.batch_rank; ++d)
    if (p.a_bst[d] % 4 != 0) return false;
  if (p.nb > (1 << 30)) return false;
  // tile, row and batch coordinates use 32-bit arithmetic in the kernel
  const int64_t tiles = ((p.M + kBM - 1) / kBM) * ((p.N + block_n - 1) / block_n) * p.nb;
  if (p.M >= (int64_t(1) << 31) || tiles >= (int64_t(1) << 31) || p.P * p.Q >= (int64_t(1) << 31)) return false;
  const int64_t units = tiles * p.ksplit;
  if (units >= (int64_t(1) << 31)) return false;
  bool ok = false;
  if (block_n == 64) ok = launch_epi<64>(p, tmap_hi, tmap_lo, s);
  else if (block_n == 128) ok = launch_epi<128>(p, tmap_hi, tmap_lo, s);
  if (!ok) return false;
  if (p.ksplit > 1) launch_splitk_reduce(p_in, p.split_stride, s);
  return true;
}

void launch_splitk_reduce(const ConvGemmParams& p_in, int64_t split_stride, cudaStream_t s) {
  ConvGemmParams r = p_in;
  r.split_stride = split_stride;
  const int64_t work = r.M * ((r.N + 3) / 4);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, 148 * 16));
  splitk_reduce_kernel<<<grid, 256, 0, s>>>(r);
}

}  // namespace kern
}  // namespace gawee
