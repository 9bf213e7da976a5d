// Fused attention for sm_100a: softmax((Q . K^T) / c + mask) . V in one
// kernel, the scores never leaving the SM.
//
// It computes the reference's cluster  matmul(Q, K^T) -> div(c) -> add(mask)
// -> softmax(-1) -> matmul(., V)  (GaweeToLinalg.cpp:959-1112 for the two
// matmuls, 1377-1441 for div/add, 1885-1900 + DecomposeAggregatedLinalgOps.cpp:22-55
// for the softmax: max, exp(x - max), sum, divide) with the softmax taken
// online over 128-key tiles (running max m, running sum l, output rescaled
// by exp(m_old - m_new)), which is the same quantity evaluated in a
// different order.  Contractions are fp32-accurate split-precision TF32 on
// tcgen05 (hi*hi + hi*lo + lo*hi; the tensor core reads fp32 as TF32 by
// dropping the 13 low mantissa bits, so a raw value is its high part):
//   S  = Q.K^T : Q raw (smem, TMA) x K raw / K lo (smem), Q lo (tensor memory) x K raw
//   O += P.V   : P raw / P lo (tensor memory, written by the softmax warps)
//                x V^T raw / V^T lo (smem, K-major: the split warps transpose
//                each V tile as they form its remainders)
// GQA needs no expanded copy: query head h reads key/value head h / (H / Hkv).
// A key tile whose mask block is -inf for every row of the query tile adds
// exactly nothing (exp(-inf - m) = 0) and is skipped (flags precomputed per
// forward by attn_skip_kernel).
//
// One CTA per (batch, head, 128-query tile), heaviest query tiles first.
// Warp roles (448 threads):
//   warps 0-7  softmax rows, two warps per row quarter (lane = query row =
//              tensor-memory lane), each over half the keys of a tile and
//              half the output columns; the fp32 output accumulator in
//              registers, the final O / l store
//   warp 8     TMA (Q once, then K tiles into two buffers and V tiles into
//              one); owns the tensor-memory allocation
//   warp 9     lane 0 issues the MMAs and the commits that track them
//   warps 10-13 split: Q lo into tensor memory once, then per key tile K lo,
//              and V^T raw and V^T lo (transposed to K-major) in shared memory
// Every mbarrier wait is bounded (tc_common.cuh: mbar_wait); on expiry the
// CTA records ST_BARRIER_TIMEOUT and finishes without its result.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "kernels.h"
#include "program.cuh"
#include "tc_common.cuh"

namespace gawee {
namespace kern {

namespace {

constexpr int kAttnThreads = 448;
constexpr int kRowsQ = 128;       // query rows per CTA
constexpr int kKeys = 128;        // keys per tile
constexpr int kTile = 16384;      // 128 rows x 32 fp32: one 128-byte-swizzled half of a 64-wide head dim
constexpr int kMaxKeyTiles = 64;  // keys per sequence <= 8192
// shared memory (32 KB each): Q, K raw x2 buffers, K lo, V raw, V^T raw, V^T lo.
// Q and K are [rows][d] in two 128-byte-swizzled halves of the head dim; V^T
// is [d][keys] in four 8 KB k-blocks of 32 keys (64 rows x 128 bytes).
constexpr int kOffQ = 0;
constexpr int kOffK = 2 * kTile;
constexpr int kOffKlo = 6 * kTile;
constexpr int kOffV = 8 * kTile;
constexpr int kOffVt = 10 * kTile;
constexpr int kOffVtlo = 12 * kTile;
constexpr int kOffBar = 14 * kTile;
constexpr int kVtBlock = 8192;
enum Bar : int {
  BAR_Q, BAR_QLO, BAR_KF0, BAR_KF1, BAR_KE0, BAR_KE1, BAR_VF, BAR_VE, BAR_KLO_R, BAR_KLO_F, BAR_VT_R, BAR_VT_F,
  BAR_SF0, BAR_SF1, BAR_SE0, BAR_SE1, BAR_P_R, BAR_PLO_F, BAR_PV_F, BAR_PV_E, BAR_DONE, NUM_BARS
};
constexpr int kOffXch = kOffBar + 512;  // partial row maxima / sums of the two halves: [2][128] floats
constexpr int kAttnSmem = kOffXch + 2 * kRowsQ * 4 + 1024;
static_assert(NUM_BARS * 8 + 16 + kMaxKeyTiles * 4 <= 512, "barriers, flags and tile list");
// tensor memory columns: S buffers (P raw overwrites them), P lo, Q lo, P.V
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColPlo = 256, kColQlo = 384, kColPV = 448;

// (d, seq, head, batch) coordinates placed in the map's dim order
__device__ __forceinline__ void tma_load_attn(uint32_t dst, const CUtensorMap* map, uint32_t bar, const int8_t* cpos,
                                              int d, int sq, int hh, int bb) {
  int c[4];
  c[0] = d;
  c[cpos[0]] = sq;
  c[cpos[1]] = hh;
  c[cpos[2]] = bb;
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3])
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void umma_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::tf32, fp32 accumulate, K-major A and B, M = 128, N = n
__device__ __forceinline__ uint32_t idesc_tf32(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kRowsQ >> 4) << 24);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ float maxnan(float a, float b) { return a > b ? a : b; }

}  // namespace

// flags[mb][mh][qt][kt]: 1 when mask(b, h, i, j) is -inf for every query row i
// and key j of the tile pair (the tile is skipped), 2 when it is +0 or -0
// everywhere (adding it changes no score that reaches the softmax, so the
// kernel does not read it), 0 otherwise; rows / keys past the sequence ignored.
__global__ void __launch_bounds__(256) attn_skip_kernel(const __grid_constant__ AttnParams p, uint8_t* flags) {
  const int kt = blockIdx.x % p.KT;
  const int qt = (blockIdx.x / p.KT) % p.QT;
  const int mh = (blockIdx.x / (p.KT * p.QT)) % p.mh;
  const int mb = blockIdx.x / (p.KT * p.QT * p.mh);
  const float* base = p.mask + (int64_t)mb * p.m_st[0] + (int64_t)mh * p.m_st[1];
  int all_neg_inf = 1, all_zero = 1;
  for (int e = threadIdx.x; e < kRowsQ * kKeys; e += blockDim.x) {
    const int i = qt * kRowsQ + e / kKeys, j = kt * kKeys + e % kKeys;
    if (i >= p.S || j >= p.Skv) continue;
    const float v = base[(int64_t)i * p.m_st[2] + (int64_t)j * p.m_st[3]];
    if (!(v == -INFINITY)) all_neg_inf = 0;
    if (!(v == 0.0f)) all_zero = 0;
  }
  all_neg_inf = __syncthreads_and(all_neg_inf);
  all_zero = __syncthreads_and(all_zero);
  if (threadIdx.x == 0) flags[blockIdx.x] = (uint8_t)(all_neg_inf ? 1 : all_zero ? 2 : 0);
}

// Poll intervals (nanoseconds) of the waits outside the softmax warps.  The
// softmax warps are bound by instruction issue, and the TMA, MMA and split
// warps share their sub-partitions: polling those barriers in a tight loop
// took the issue slots the softmax needs.
constexpr unsigned kSleepTma = 64, kSleepMma = 32, kSleepSplit = 64;

template <int DV>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ AttnParams p, const __grid_constant__ CUtensorMap tq,
                   const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* ntiles = reinterpret_cast<int*>(tmem_slot + 2);
  int* tiles = reinterpret_cast<int*>(tmem_slot + 4);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  // heaviest (last) query tiles first
  const int BH = p.B * p.H;
  const int qt = p.QT - 1 - (int)(blockIdx.x / BH);
  const int bh = (int)(blockIdx.x % BH);
  const int b = bh / p.H, h = bh - b * p.H;
  const int hkv = h / (p.H / p.Hkv);
  const int q0 = qt * kRowsQ;

  if (warp == 8) {
    // the TMA warp sets up the barriers and issues Q at once: its latency
    // overlaps the tile list and the tensor-memory allocation
    if (lane == 0) {
      for (int i = 0; i < NUM_BARS; ++i) {
        uint32_t count = 1;
        if (i == BAR_QLO || i == BAR_KLO_R || i == BAR_VT_R || i == BAR_VE) count = 4;
        if (i == BAR_P_R || i == BAR_PV_E) count = 8;
        mbar_init(bar(i), count);
      }
      *abort_flag = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tq)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tk)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tv)) : "memory");
      mbar_arrive_tx(bar(BAR_Q), 2 * kTile);
      for (int hd = 0; hd < 2; ++hd)
        tma_load_attn(smem_u32(smem + kOffQ + hd * kTile), &tq, bar(BAR_Q), p.cpos[0], hd * 32, q0, h, b);
    }
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  } else if (warp == 0) {
    // the key tiles this query tile visits, ascending: one flag per lane
    // (all reads in flight together), compacted with ballots
    const uint8_t* fl = p.skip ? p.skip + ((int64_t)((p.mb > 1 ? b : 0) * p.mh + (p.mh > 1 ? h : 0)) * p.QT + qt) * p.KT
                               : nullptr;
    int n = 0;
    for (int base = 0; base < p.KT; base += 32) {
      const int kt = base + lane;
      const int f = (fl && kt < p.KT) ? (int)fl[kt] : 0;
      const bool keep = kt < p.KT && f != 1;
      const unsigned m = __ballot_sync(0xffffffffu, keep);
      if (keep) tiles[n + __popc(m & ((1u << lane) - 1u))] = kt | (f == 2 ? 0x10000 : 0);
      n += __popc(m);
    }
    if (lane == 0) *ntiles = n;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int T = *ntiles;

  if (warp < 8) {
    // ------------------------------------------------------------------ softmax rows
    // Two warps per lane quarter: warp w owns rows 32 (w % 4) .. + 31 (its
    // tensor-memory lanes) over key columns 64 hf .. + 63 and output
    // columns 32 hf .. (hf = w / 4).  The halves of a row exchange their
    // partial maxima per tile through shared memory (named barrier of the
    // two warps) and their partial sums once at the end.
    const int q = warp & 3, hf = warp >> 2;
    const int r = q * 32 + lane;
    const int qi = q0 + r;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    float* xch = reinterpret_cast<float*>(smem + kOffXch);  // [2][128]
    auto pair_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(1 + q), "r"(64) : "memory"); };
    const float* mrow = p.mask ? p.mask + (int64_t)b * p.m_st[0] + (int64_t)h * p.m_st[1] +
                                     (int64_t)min(qi, p.S - 1) * p.m_st[2]
                               : nullptr;
    constexpr int kO0 = DV < 32 ? DV : 32;        // output columns of half 0
    constexpr int kO1 = DV > 32 ? DV - 32 : 0;    // of half 1
    const int ocol0 = 32 * hf, ocols = hf ? kO1 : kO0;
    float o[32];
#pragma unroll
    for (int d = 0; d < 32; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    const bool mvec = mrow && p.m_st[3] == 1 && (reinterpret_cast<uintptr_t>(mrow) & 15) == 0;
    const float scale = p.scale;
    auto correct = [&](int u, float alpha) -> bool {  // O = O * alpha_u + (P_u . V_u), this half's columns
      if (!__all_sync(0xffffffffu, mbar_wait(bar(BAR_PV_F), u & 1, abort_flag, p.status))) return false;
      tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < 32; c0 += 16) {
        if (c0 < ocols) {
          uint32_t v[16];
          tmem_ld16(trow + kColPV + ocol0 + c0, v);
#pragma unroll
          for (int e = 0; e < 16; ++e) o[c0 + e] = __fadd_rn(__fmul_rn(o[c0 + e], alpha), __uint_as_float(v[e]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_PV_E));
      return true;
    };
    // The two warps of a row pair meet at a named barrier twice per tile and
    // once at the end, always: after a failed (bounded) wait a warp skips its
    // work but never a barrier, so neither can be left waiting at one.
    for (int t = 0; t < T; ++t) {
      const int sb = t & 1;
      const uint32_t scol = (sb ? kColS1 : kColS0) + 64 * hf;
      const int j0 = (tiles[t] & 0xffff) * kKeys + 64 * hf;
      const bool use_mask = mrow && !(tiles[t] & 0x10000);
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(sb ? BAR_SF1 : BAR_SF0), (t >> 1) & 1, abort_flag, p.status));
      tc_fence_after();
      // pass 1: scores (acc / c + mask, the reference's operations and
      // order; -inf past the sequence) written back over the accumulators,
      // and this half's row maximum
      float tmax = -INFINITY;
#pragma unroll
      for (int c0 = 0; c0 < 64 && ok; c0 += 16) {
        uint32_t x[16];
        float mk[16];
        if (use_mask) {
          if (mvec && j0 + c0 + 16 <= p.Skv) {
#pragma unroll
            for (int e = 0; e < 16; e += 4) {
              const float4 v = __ldg(reinterpret_cast<const float4*>(mrow + j0 + c0 + e));
              mk[e] = v.x; mk[e + 1] = v.y; mk[e + 2] = v.z; mk[e + 3] = v.w;
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              mk[e] = j0 + c0 + e < p.Skv ? __ldg(mrow + (int64_t)(j0 + c0 + e) * p.m_st[3]) : 0.f;
          }
        }
        tmem_ld16(trow + scol + c0, x);
        // the scale's form is chosen once per chunk, outside the element loop:
        // with the choice inside, the IEEE division ran for every element
        // (the compiler evaluated both arms), about 150 cycles per score
        const int valid = min(16, p.Skv - (j0 + c0));
        if (p.scale_mul) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float sc = __fmul_rn(__uint_as_float(x[e]), scale);
            if (use_mask) sc = __fadd_rn(sc, mk[e]);
            if (e >= valid) sc = -INFINITY;
            tmax = maxnan(tmax, sc);
            x[e] = __float_as_uint(sc);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float sc = __fdiv_rn(__uint_as_float(x[e]), scale);
            if (use_mask) sc = __fadd_rn(sc, mk[e]);
            if (e >= valid) sc = -INFINITY;
            tmax = maxnan(tmax, sc);
            x[e] = __float_as_uint(sc);
          }
        }
        tmem_st16(trow + scol + c0, x);
      }
      // the row's maximum over both halves
      xch[hf * kRowsQ + r] = tmax;
      pair_sync();
      tmax = maxnan(tmax, xch[(hf ^ 1) * kRowsQ + r]);
      pair_sync();  // both read before the next tile's writes
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      const float m_new = maxnan(m, tmax);
      const float alpha = m_new == -INFINITY ? 1.f : expf(__fsub_rn(m, m_new));
      // P lo of the previous tile must have been consumed by its P.V
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(BAR_PLO_F), (t & 1) ^ 1, abort_flag, p.status));
      if (!ok) continue;
      tc_fence_after();
      // pass 2: p = exp(s - m_new); P raw over the scores, P lo beside
      float lsum = 0.f;
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 16) {
        uint32_t x[16], y[16];
        tmem_ld16(trow + scol + c0, x);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float sv = __uint_as_float(x[e]);
          // __expf: relative error within a few ulp where p is not negligible
          // (s - m in [-20, 0]); the row's largest term is exactly 1
          const float pe = (sv == -INFINITY) ? 0.f : __expf(__fsub_rn(sv, m_new));
          lsum = __fadd_rn(lsum, pe);
          x[e] = __float_as_uint(pe);
          y[e] = __float_as_uint(__fsub_rn(pe, tf32_hi(pe)));
        }
        tmem_st16(trow + scol + c0, x);
        tmem_st16(trow + kColPlo + 64 * hf + c0, y);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_P_R));
      l = __fadd_rn(__fmul_rn(l, alpha), lsum);  // this half's partial sum
      m = m_new;
      if (t > 0) ok = correct(t - 1, alpha_prev);
      alpha_prev = alpha;
    }
    if (ok && T > 0) ok = correct(T - 1, alpha_prev);
    ok = __all_sync(0xffffffffu, ok && !*abort_flag);
    // the row's sum: both halves add the partials in the same order
    xch[hf * kRowsQ + r] = l;
    pair_sync();
    l = __fadd_rn(xch[r], xch[kRowsQ + r]);
    if (ok && qi < p.S) {
      float* orow = p.out + (int64_t)b * p.o_st[0] + (int64_t)h * p.o_st[1] + (int64_t)qi * p.o_st[2] +
                    (int64_t)ocol0 * p.o_st[3];
      // compile-time indices keep o[] in registers
      if (p.o_st[3] == 1 && (reinterpret_cast<uintptr_t>(orow) & 15) == 0 && p.D % 4 == 0) {
#pragma unroll
        for (int d = 0; d < 32; d += 4)
          if (d < ocols && ocol0 + d < p.D)
            *reinterpret_cast<float4*>(orow + d) = make_float4(__fdiv_rn(o[d], l), __fdiv_rn(o[d + 1], l),
                                                               __fdiv_rn(o[d + 2], l), __fdiv_rn(o[d + 3], l));
      } else {
#pragma unroll
        for (int d = 0; d < 32; ++d)
          if (d < ocols && ocol0 + d < p.D) orow[(int64_t)d * p.o_st[3]] = __fdiv_rn(o[d], l);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      for (int t = 0; t < T; ++t) {  // (Q was issued before the block-wide barrier)
        const int kb = t & 1;
        const int j0 = (tiles[t] & 0xffff) * kKeys;
        // K into its buffer once QK of tile t - 2 has completed
        if (!mbar_wait_relaxed(bar(kb ? BAR_KE1 : BAR_KE0), ((t >> 1) & 1) ^ 1, abort_flag, p.status, kSleepTma)) break;
        const uint32_t kf = bar(kb ? BAR_KF1 : BAR_KF0);
        mbar_arrive_tx(kf, 2 * kTile);
        for (int hd = 0; hd < 2; ++hd)
          tma_load_attn(smem_u32(smem + kOffK + (2 * kb + hd) * kTile), &tk, kf, p.cpos[1], hd * 32, j0, hkv, b);
        // V once the split warps have transposed tile t - 1
        if (!mbar_wait_relaxed(bar(BAR_VE), (t & 1) ^ 1, abort_flag, p.status, kSleepTma)) break;
        mbar_arrive_tx(bar(BAR_VF), 2 * kTile);
        for (int hd = 0; hd < 2; ++hd)
          tma_load_attn(smem_u32(smem + kOffV + hd * kTile), &tv, bar(BAR_VF), p.cpos[2], hd * 32, j0, hkv, b);
      }
      if (*abort_flag) {
        const unsigned long long t0 = global_ns();  // let issued copies land
        while (global_ns() - t0 < 100000ull) {
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const bool three = p.passes != 1;
      const uint32_t id_s = idesc_tf32(kKeys);  // S: N = 128 keys
      const uint32_t id_o = idesc_tf32(DV);     // O: N = head dim
      const uint32_t aq = smem_u32(smem + kOffQ);
      // Q lo is waited for just before the first lo products (tile 0)
      bool alive = mbar_wait_relaxed(bar(BAR_Q), 0, abort_flag, p.status, kSleepMma);
      tc_fence_after();
      auto pv = [&](int u) -> bool {
        const int sb = u & 1;
        if (!mbar_wait_relaxed(bar(BAR_P_R), u & 1, abort_flag, p.status, kSleepMma)) return false;
        if (!mbar_wait_relaxed(bar(BAR_VT_R), u & 1, abort_flag, p.status, kSleepMma)) return false;
        if (!mbar_wait_relaxed(bar(BAR_PV_E), (u & 1) ^ 1, abort_flag, p.status, kSleepMma)) return false;
        tc_fence_after();
        const uint32_t praw = tmem + (sb ? kColS1 : kColS0), plo = tmem + kColPlo, dpv = tmem + kColPV;
        const uint32_t vt = smem_u32(smem + kOffVt), vtl = smem_u32(smem + kOffVtlo);
        if (three) {
#pragma unroll 4
          for (int kk = 0; kk < kKeys / 8; ++kk) {  // 8 keys per step; a V^T k-block holds 32
            const uint32_t blk = (uint32_t)(kk >> 2) * kVtBlock;
            const uint64_t o = (uint64_t)(2 * (kk & 3));
            const uint64_t dv = umma_desc_sw128(vt + blk) + o, dvl = umma_desc_sw128(vtl + blk) + o;
            umma_tf32_ts(dpv, praw + 8 * kk, dv, id_o, kk != 0);
            umma_tf32_ts(dpv, praw + 8 * kk, dvl, id_o, 1);
            umma_tf32_ts(dpv, plo + 8 * kk, dv, id_o, 1);
          }
        } else {  // single pass: the lo operands' data flow stays, their products are skipped
#pragma unroll 4
          for (int kk = 0; kk < kKeys / 8; ++kk) {
            const uint64_t dv = umma_desc_sw128(vt + (uint32_t)(kk >> 2) * kVtBlock) + (uint64_t)(2 * (kk & 3));
            umma_tf32_ts(dpv, praw + 8 * kk, dv, id_o, kk != 0);
          }
        }
        umma_commit(bar(BAR_PV_F));
        umma_commit(bar(sb ? BAR_SE1 : BAR_SE0));
        umma_commit(bar(BAR_PLO_F));
        umma_commit(bar(BAR_VT_F));
        return true;
      };
      for (int t = 0; t < T && alive; ++t) {
        const int kb = t & 1;
        // the raw products need only K and a free score buffer; K lo (and,
        // for tile 0, Q lo) are waited for after them, so the split of K
        // overlaps the first eight MMAs
        alive = mbar_wait_relaxed(bar(kb ? BAR_KF1 : BAR_KF0), (t >> 1) & 1, abort_flag, p.status, kSleepMma) &&
                mbar_wait_relaxed(bar(kb ? BAR_SE1 : BAR_SE0), ((t >> 1) & 1) ^ 1, abort_flag, p.status, kSleepMma);
        if (!alive) break;
        tc_fence_after();
        const uint32_t ds = tmem + (kb ? kColS1 : kColS0);
        const uint32_t k_raw = smem_u32(smem + kOffK + 2 * kb * kTile);
#pragma unroll
        for (int hd = 0; hd < 2; ++hd) {  // K = 64: two 32-wide halves of the head dim
          const uint64_t dq = umma_desc_sw128(aq + hd * kTile);
          const uint64_t dk = umma_desc_sw128(k_raw + hd * kTile);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_ss(ds, dq + 2 * kk, dk + 2 * kk, id_s, (hd | kk) != 0);
        }
        alive = mbar_wait_relaxed(bar(BAR_KLO_R), t & 1, abort_flag, p.status, kSleepMma) &&
                (t > 0 || mbar_wait_relaxed(bar(BAR_QLO), 0, abort_flag, p.status, kSleepMma));
        if (!alive) break;
        tc_fence_after();
        if (three) {
#pragma unroll
          for (int hd = 0; hd < 2; ++hd) {
            const uint64_t dq = umma_desc_sw128(aq + hd * kTile);
            const uint64_t dk = umma_desc_sw128(k_raw + hd * kTile);
            const uint64_t dkl = umma_desc_sw128(smem_u32(smem + kOffKlo + hd * kTile));
            const uint32_t qlo = tmem + kColQlo + 32 * hd;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t o = (uint64_t)(2 * kk);
              umma_ss(ds, dq + o, dkl + o, id_s, 1);
              umma_tf32_ts(ds, qlo + 8 * kk, dk + o, id_s, 1);
            }
          }
        }
        umma_commit(bar(kb ? BAR_SF1 : BAR_SF0));
        umma_commit(bar(BAR_KLO_F));
        umma_commit(bar(kb ? BAR_KE1 : BAR_KE0));
        if (t > 0) alive = pv(t - 1);
      }
      if (alive && T > 0) pv(T - 1);
      umma_commit(bar(BAR_DONE));
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ split
    const int q4 = warp & 3;                 // tensor-memory lane quarter of this warp
    const int row = q4 * 32 + lane;          // Q row for Q lo
    const int tid = (warp - 10) * 32 + lane;  // 0..127 for the K / V tiles
    bool alive = mbar_wait_relaxed(bar(BAR_Q), 0, abort_flag, p.status, kSleepSplit);
    if (alive) {
      const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
      for (int hd = 0; hd < 2; ++hd) {
        const uint32_t src = smem_u32(smem + kOffQ + hd * kTile) + row * 128;
        uint32_t y[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 v = lds128(src + ((c ^ (row & 7)) << 4));
          y[4 * c] = __float_as_uint(__fsub_rn(v.x, tf32_hi(v.x)));
          y[4 * c + 1] = __float_as_uint(__fsub_rn(v.y, tf32_hi(v.y)));
          y[4 * c + 2] = __float_as_uint(__fsub_rn(v.z, tf32_hi(v.z)));
          y[4 * c + 3] = __float_as_uint(__fsub_rn(v.w, tf32_hi(v.w)));
        }
        tmem_st32(trow + kColQlo + 32 * hd, y);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_QLO));
    }
    // lo = x - tf32(x) of a 32 KB tile, element by element (layout-agnostic)
    auto split_tile = [&](uint32_t src, uint32_t dst) {
#pragma unroll 4
      for (int c = tid; c < 2 * kTile / 16; c += 128) {
        const float4 v = lds128(src + c * 16);
        const float4 w = make_float4(__fsub_rn(v.x, tf32_hi(v.x)), __fsub_rn(v.y, tf32_hi(v.y)),
                                     __fsub_rn(v.z, tf32_hi(v.z)), __fsub_rn(v.w, tf32_hi(v.w)));
        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst + c * 16), "f"(w.x), "f"(w.y), "f"(w.z),
                     "f"(w.w)
                     : "memory");
      }
      fence_async_smem();  // generic-proxy writes, read by the tensor core
      __syncwarp();
    };
    // V [keys][d] (two swizzled d halves) -> V^T [d][keys] (four swizzled
    // 32-key k-blocks), raw and lo; each thread moves 4 x 4 blocks: four
    // 16-byte reads (4 d of one key) and four 16-byte writes (4 keys of one d)
    const uint32_t v_in = smem_u32(smem + kOffV), vt_out = smem_u32(smem + kOffVt), vtl_out = smem_u32(smem + kOffVtlo);
    auto transpose_v = [&]() {
#pragma unroll 1
      for (int blk = tid; blk < (kKeys / 4) * (64 / 4); blk += 128) {
        const int j0 = (blk % (kKeys / 4)) * 4, d0 = (blk / (kKeys / 4)) * 4;
        float x[4][4];  // [key][d]
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const int j = j0 + a;
          const float4 v = lds128(v_in + (d0 >> 5) * kTile + j * 128 + ((((d0 & 31) >> 2) ^ (j & 7)) << 4));
          x[a][0] = v.x; x[a][1] = v.y; x[a][2] = v.z; x[a][3] = v.w;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int d = d0 + c;
          const uint32_t off = (uint32_t)(j0 >> 5) * kVtBlock + d * 128 + ((((j0 & 31) >> 2) ^ (d & 7)) << 4);
          const float r0 = x[0][c], r1 = x[1][c], r2 = x[2][c], r3 = x[3][c];
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(vt_out + off), "f"(r0), "f"(r1), "f"(r2),
                       "f"(r3)
                       : "memory");
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(vtl_out + off),
                       "f"(__fsub_rn(r0, tf32_hi(r0))), "f"(__fsub_rn(r1, tf32_hi(r1))),
                       "f"(__fsub_rn(r2, tf32_hi(r2))), "f"(__fsub_rn(r3, tf32_hi(r3)))
                       : "memory");
        }
      }
      fence_async_smem();  // generic-proxy writes, read by the tensor core
      __syncwarp();
    };
    // K lo of tile u once K(u) has landed and QK(u - 1) has read K lo(u - 1)
    auto k_lo = [&](int u) -> bool {
      const int kb = u & 1;
      if (!(mbar_wait_relaxed(bar(kb ? BAR_KF1 : BAR_KF0), (u >> 1) & 1, abort_flag, p.status, kSleepSplit) &&
            mbar_wait_relaxed(bar(BAR_KLO_F), (u & 1) ^ 1, abort_flag, p.status, kSleepSplit)))
        return false;
      split_tile(smem_u32(smem + kOffK + 2 * kb * kTile), smem_u32(smem + kOffKlo));
      if (lane == 0) mbar_arrive(bar(BAR_KLO_R));
      return true;
    };
    // K lo(t + 1) goes before the transpose of V(t): the transpose waits for
    // P.V(t - 1), and QK(t + 1) should not wait behind it
    if (T > 0) alive = k_lo(0);
    for (int t = 0; t < T && alive; ++t) {
      if (t + 1 < T && !k_lo(t + 1)) {
        alive = false;
        break;
      }
      alive = mbar_wait_relaxed(bar(BAR_VF), t & 1, abort_flag, p.status, kSleepSplit) &&
              mbar_wait_relaxed(bar(BAR_VT_F), (t & 1) ^ 1, abort_flag, p.status, kSleepSplit);
      if (!alive) break;
      transpose_v();
      if (lane == 0) {
        mbar_arrive(bar(BAR_VT_R));
        mbar_arrive(bar(BAR_VE));  // the V buffer may be refilled
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    volatile int never = 0;
    if (lane == 0) mbar_wait(bar(BAR_DONE), 0, &never, p.status);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
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

template <int DV>
bool launch_dv(const AttnParams& p, const void* tq, const void* tk, const void* tv, cudaStream_t s) {
  auto kern = attn_tc_kernel<DV>;
  static std::mutex mu;
  static uint64_t attr_devices = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !(attr_devices >> dev & 1)) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem) != cudaSuccess)
        return false;
      attr_devices |= uint64_t(1) << dev;
    }
  }
  const unsigned grid = (unsigned)(p.B * p.H * p.QT);
  kern<<<grid, kAttnThreads, kAttnSmem, s>>>(p, *static_cast<const CUtensorMap*>(tq),
                                              *static_cast<const CUtensorMap*>(tk),
                                              *static_cast<const CUtensorMap*>(tv));
  return true;
}

}  // namespace

bool make_attn_tensor_map(const float* base, int64_t batch, int64_t heads, int64_t seq, int64_t dim, int64_t st_b,
                          int64_t st_h, int64_t st_s, void* tmap_out, int8_t* cpos) {
  auto enc = encode_tiled();
  if (!enc) return false;
  // the map's outer dims (seq, head, batch) go in increasing stride order
  // (heads may be interleaved inside a row: st_h < st_s); size-1 dims last
  int64_t ext[3] = {seq, heads, batch}, st[3] = {st_s, st_h, st_b};
  int64_t big = 1;
  for (int i = 0; i < 3; ++i) big = std::max(big, std::abs(st[i]) * ext[i]);
  for (int i = 0; i < 3; ++i)
    if (ext[i] == 1) st[i] = big;  // never stepped: any valid stride
  if ((reinterpret_cast<uintptr_t>(base) & 15)) return false;
  int order[3] = {0, 1, 2};
  std::sort(order, order + 3, [&](int a, int b) { return st[a] < st[b] || (st[a] == st[b] && a < b); });
  cuuint64_t dims[4] = {(cuuint64_t)dim, 0, 0, 0};
  cuuint64_t strides[3];
  cuuint32_t box[4] = {32, 1, 1, 1};
  for (int k = 0; k < 3; ++k) {
    const int i = order[k];
    if (st[i] <= 0 || st[i] % 4) return false;
    dims[1 + k] = (cuuint64_t)ext[i];
    strides[k] = (cuuint64_t)(st[i] * 4);
    if (i == 0) box[1 + k] = (cuuint32_t)kRowsQ;
    cpos[i] = (int8_t)(1 + k);
  }
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(static_cast<CUtensorMap*>(tmap_out), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base),
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool attn_supported(int64_t D, int64_t Skv, int64_t H, int64_t Hkv) {
  return D >= 16 && D <= 64 && D % 16 == 0 && Skv >= 1 && (Skv + kKeys - 1) / kKeys <= kMaxKeyTiles && Hkv >= 1 &&
         H % Hkv == 0;
}

bool launch_attention(const AttnParams& p, const void* tq, const void* tk, const void* tv, uint8_t* skip_flags,
                      bool flags_current, cudaStream_t s) {
  if (!attn_supported(p.D, p.Skv, p.H, p.Hkv) || p.B <= 0 || p.S <= 0) return false;
  if (p.passes != 0 && p.passes != 1 && p.passes != 3) return false;
  AttnParams q = p;
  if (q.passes == 0) q.passes = 3;
  q.skip = nullptr;
  if (p.mask && skip_flags) {
    if (!flags_current) {
      const int blocks = p.mb * p.mh * p.QT * p.KT;
      attn_skip_kernel<<<blocks, 256, 0, s>>>(p, skip_flags);
    }
    q.skip = skip_flags;
  }
  switch ((p.D + 15) / 16 * 16) {
    case 16:
    case 32: return launch_dv<32>(q, tq, tk, tv, s);
    case 48: return launch_dv<48>(q, tq, tk, tv, s);
    case 64: return launch_dv<64>(q, tq, tk, tv, s);
    default: return false;
  }
}

}  // namespace kern
}  // namespace gawee
