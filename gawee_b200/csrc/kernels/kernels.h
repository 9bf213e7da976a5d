// Launch interfaces of the sm_100a kernels used by the gawee CUDA runtime.
// Plain structs passed by value as kernel parameters; no torch types.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace gawee {
namespace kern {

constexpr int kMaxRank = 8;
constexpr int kMaxIn = 8;
// Promotion granularity of the tensor-core kernels: each round of kRK
// 32-wide k-blocks is accumulated alone in a tensor-memory buffer, and the
// accumulator warps add the round sums into fp32 registers with IEEE
// round-to-nearest (the TMA kernel may take a longer round: ConvGemmParams::rk).
constexpr int kRK = 2;
constexpr int kMaxInstr = 40;
constexpr int kMaxRegs = 32;

// Device-side dtype codes (same numbering as gawee::DType).
enum DT : int8_t { DT_F32 = 0, DT_F64 = 1, DT_F16 = 2, DT_I64 = 3, DT_I32 = 4, DT_I1 = 5, DT_INDEX = 6 };

// Error codes written to the per-context device status word.
enum Status : int {
  ST_OK = 0,
  ST_GATHER_INDEX = 1,     // gather index outside the table
  ST_BARRIER_TIMEOUT = 2,  // a bounded mbarrier wait in a tensor-core kernel gave up
  ST_BAD_PROGRAM = 3,      // elementwise program with an unknown opcode
  ST_INT_DIV_ZERO = 4,
  ST_SLICE_BOUNDS = 5,
};

struct DInstr {
  uint8_t op, ty, rty;
  int8_t pred;
  int8_t dst, a, b, c;
  double fimm;
  long long iimm;
};

struct DProgram {
  int n_code;
  int n_args;
  int result;
  DInstr code[kMaxInstr];
};

// A strided operand over the iteration space of an elementwise launch.
struct EwOperand {
  void* ptr;
  int64_t st[kMaxRank];  // element strides per iteration dim (0 = broadcast)
  int8_t dt;
};

// Elementwise programs recognised on the host (all f32) and evaluated without
// the interpreter, with the same IEEE operations in the same order.
// The host reorders the operands so the fast form reads in[0..3].
enum FastEw : int {
  EW_INTERP = 0,
  EW_COPY = 1,        // in[0]
  EW_SQR = 2,         // in[0] * in[0]           (powf(x, 2) or x * x)
  EW_NEG = 3,         // -in[0]
  EW_ADDC_SQRT = 4,   // sqrt(in[0] + fk)
  EW_DIV_MUL = 5,     // (in[0] / in[1]) * in[2]
  EW_MUL_MUL_ADD = 6, // (in[0] * in[1]) + (in[2] * in[3])
};

struct EwParams {
  int rank;
  int n_in;
  int64_t numel;
  int64_t shape[kMaxRank];  // iteration space (output shape, dims ordered outer..inner)
  EwOperand out;
  EwOperand in[kMaxIn];
  DProgram prog;
  int fast;                  // FastEw
  float fk;                  // its constant
  int* status;
};

void launch_elementwise(const EwParams& p, cudaStream_t s);

// Reduction of `cols` elements per output row.  Input offset of (row, col) is
// unravel(row over kept dims) . kept strides + unravel(col over reduced dims) . red strides.
struct ReduceParams {
  const float* in;
  float* out;              // out[row]; contiguous rows in output order
  int64_t rows, cols;
  int kept_rank, red_rank;
  int64_t kept_shape[kMaxRank], kept_st[kMaxRank];
  int64_t red_shape[kMaxRank], red_st[kMaxRank];
  int64_t out_st[kMaxRank];  // output strides over kept dims
  int mode;                // 0 sum, 1 mean (sum / count)
  float count;
};
void launch_reduce_f32(const ReduceParams& p, cudaStream_t s);

// linalg.reduce with an arbitrary scalar body: one thread per output element,
// sequential over the reduced elements in input row-major order (the
// reference loop order).  The output already holds the init values.
struct GenericReduceParams {
  const void* in;
  void* out;
  int8_t in_dt, out_dt;
  int64_t rows, cols;
  int kept_rank, red_rank;
  int64_t kept_shape[kMaxRank], kept_st[kMaxRank];
  int64_t red_shape[kMaxRank], red_st[kMaxRank];
  int64_t out_st[kMaxRank];
  DProgram prog;  // registers 0 = input element, 1 = accumulator
  int* status;
};
void launch_generic_reduce(const GenericReduceParams& p, cudaStream_t s);

// Softmax along one axis: rows x len, element (row, j) at in + row_off(row) + j * axis_st.
struct SoftmaxParams {
  const float* in;
  float* out;
  int64_t rows, len;
  int rank;                       // rank of the row space
  int64_t row_shape[kMaxRank], in_row_st[kMaxRank], out_row_st[kMaxRank];
  int64_t in_axis_st, out_axis_st;
};
void launch_softmax(const SoftmaxParams& p, cudaStream_t s);

// out[pre, j, post] = data[pre, idx[j], post] with data contiguous [pre, axis, post].
struct GatherParams {
  const void* data;
  const void* idx;     // i64 or i32 index tensor, contiguous
  void* out;           // contiguous [pre, nidx, post]
  int8_t idx_dt;
  int elem_bytes;
  int64_t pre, axis_len, nidx, post;
  int* status;
};
void launch_gather(const GatherParams& p, cudaStream_t s);

// out[i] = data[i with dim `axis` replaced by idx[i]]; all contiguous.
struct GatherElementsParams {
  const void* data;
  const void* idx;
  void* out;
  int8_t idx_dt;
  int elem_bytes;
  int rank, axis;
  int64_t numel;
  int64_t shape[kMaxRank];       // output/index shape
  int64_t data_st[kMaxRank];     // data strides (elements)
  int64_t data_axis_len;
  int* status;
};
void launch_gather_elements(const GatherElementsParams& p, cudaStream_t s);

// Per-dim index remap copy: src coordinate = ((o / div) % mod) - sub; outside
// [0, src_dim) reads `fill`.  Used for pad, tile and nearest resize.
struct RemapParams {
  const void* in;
  void* out;
  int elem_bytes;
  int rank;
  int64_t numel;
  int64_t out_shape[kMaxRank], out_st[kMaxRank];
  int64_t in_shape[kMaxRank], in_st[kMaxRank];
  int64_t div[kMaxRank], mod[kMaxRank], sub[kMaxRank];
  uint64_t fill_bits;
};
void launch_remap(const RemapParams& p, cudaStream_t s);

// NCHW (channel stride in_sc, image stride in_sn, pixels contiguous) to dense
// NHWC with C4 >= C channels (multiple of 4), zero in the padding channels.
void launch_nchw_to_nhwc4(const float* in, float* out, int64_t N, int C, int C4, int64_t HW, int64_t in_sn,
                          int64_t in_sc, cudaStream_t s);

// out[i] = start + i * delta
struct RangeParams {
  void* out;
  int8_t dt;
  int64_t n;
  double fstart, fdelta;
  long long istart, idelta;
};
void launch_range(const RangeParams& p, cudaStream_t s);

// Row normalisation, the reference's RMSNorm / LayerNorm chains over the
// last dim in one pass per row: (centered: xc = x - mean(x), else xc = x)
//   out = (xc / sqrt(mean(xc * xc) + eps)) * w  [+ b]
// mean = sum / cols (ReduceMeanOpLowering: sum, then divide).  Row i starts at
// x + i * x_rs (elements, cols contiguous); w / b indexed by column with
// stride w_st / b_st (0 = broadcast scalar); out dense [rows][cols].
struct RowNormParams {
  const float* x;
  float* out;
  const float* w;
  const float* b;  // nullptr: no bias
  int64_t rows, cols, x_rs, w_st, b_st;
  float eps;
  int centered;
};
void launch_rownorm(const RowNormParams& p, cudaStream_t s);

// Rotary position embedding as the reference's graph computes it:
//   out = x * cos + rotate_half(x) * sin,  rotate_half(x)[i] = -x[i + d/2] (i < d/2), x[i - d/2] (else)
// over the last dim d (= 2 * half).  x, cos, sin are strided views over the
// output shape (stride 0 = broadcast); out is dense.
struct RopeParams {
  const float* x;
  const float* cs;
  const float* sn;
  float* out;
  int rank;  // <= 4
  int64_t numel, half;
  int64_t shape[4], x_st[4], c_st[4], s_st[4];
};
void launch_rope(const RopeParams& p, cudaStream_t s);

// Max / sum pooling over (n, c, oh, ow) with arbitrary strides on both sides.
struct PoolParams {
  const float* in;
  float* out;
  int64_t N, C, H, W, OH, OW;
  int64_t in_st[4], out_st[4];  // n, c, h, w strides
  int kh, kw, sh, sw, ph, pw, dh, dw;
  int mode;                      // 0 max (pad -inf), 1 sum / count (pad 0)
  float count;
  int64_t iter_perm[4];          // iteration order of output dims, outermost first
};
void launch_pool(const PoolParams& p, cudaStream_t s);

// Rank-2 top-k following the reference's selection loop.
struct TopKParams {
  const float* in;
  float* vals;
  int64_t* idxs;
  unsigned char* used;  // rows x len scratch flags
  int64_t rows, len, k;
};
void launch_topk(const TopKParams& p, cudaStream_t s);

// Pack a B operand for the tensor-core kernels into split-precision planes
// hi/lo of shape [batch][N][ldk] (row-major, zero for k >= K), where hi = x
// with the low 13 mantissa bits cleared (an exact TF32 value) and lo = x - hi.
// Source element (b, k, n) is read at
//   src + boff(b) + sum_d kc_d * k_st[d] + n * sn
// where k is unravelled over k_shape (outer..inner) into coordinates kc_d; a
// coordinate kc_d >= k_valid[d] reads zero (used for channel padding).
struct PackBParams {
  const float* src;
  float* hi;
  float* lo;
  int64_t batch, K, N, ldk;
  int64_t sn;
  int k_rank;
  int64_t k_shape[3], k_st[3], k_valid[3];
  int batch_rank;
  int64_t batch_shape[4], batch_st[4];
};
void launch_pack_b(const PackBParams& p, cudaStream_t s);
// The BF16 mode's B plane ([rows][ldk16] bf16, ldk16 a multiple of 8 >= ldk)
// from packed hi / lo planes ([rows][ldk] fp32): bf16(hi + lo), zero past ldk.
void launch_planes_to_bf16(const float* hi, const float* lo, void* out, int64_t rows, int64_t ldk, int64_t ldk16,
                           cudaStream_t s);

// ---------------------------------------------------------------------------
// Tensor-core contraction: implicit-GEMM convolution / (batched) GEMM.
// C[z][m][n] = sum_k A[z][m][k] * B[z][n][k]  (+ epilogue)
// The A operand is gathered: for row m = (img, p, q) and k = (r, s, c):
//   A = x[img*x_sn + (p*sh - ph + r*dh)*x_sh + (q*sw - pw + s*dw)*x_sw + c]
// with zero outside the image (implicit zero padding); a plain GEMM is the
// 1x1 case with P = rows, Q = 1.  The B operand is read from packed TF32
// hi/lo planes with TMA.  Products use three TF32 tcgen05 MMAs
// (hi*hi + hi*lo + lo*hi) accumulated in fp32 in tensor memory.
// ---------------------------------------------------------------------------
enum Epi : int {
  EPI_NONE = 0,       // C = acc
  EPI_BIAS = 1,       // C = acc + bias[n]
  EPI_BIAS_RELU = 2,  // C = max(acc + bias[n], 0)
  EPI_BIAS_ADD_RELU = 3,  // C = max((acc + bias[n]) + res[m][n], 0)
  EPI_PROGRAM = 4,    // C = program(acc, aux...) with aux operands indexed like C
  EPI_FAST = 5,       // a program recognised on the host (ConvGemmParams::fast), no interpreter
};

struct ConvGemmParams {
  // A gather
  const float* x;
  int64_t x_sn, x_sh, x_sw;     // c stride is 1
  int64_t H, W, C;              // input spatial size and channels
  int64_t P, Q;                 // output spatial size (GEMM: P = M, Q = 1)
  int R, S, sh, sw, ph, pw, dh, dw;
  int64_t M, N, K;              // M = imgs*P*Q, N = out channels, K = R*S*C
  // batching (GEMM only; conv uses nb = 1)
  int nb;
  int batch_rank;
  int64_t batch_shape[4];
  int64_t a_bst[4];             // A batch strides (elements)
  int64_t b_bst[4];             // B batch strides (planes)
  int64_t c_bst[4];             // C batch strides (elements)
  // output
  float* out;
  int64_t ldc;                  // row stride of C
  int64_t ldc_n;                // column stride of C (1 unless transposed output)
  int epi;
  const float* bias;            // [N]
  const float* res;             // residual, same indexing as C
  // EPI_PROGRAM operands: register 0 = accumulator, 1.. = aux loads
  int n_aux;
  const float* aux[4];
  int64_t aux_sm[4], aux_sn[4], aux_sb[4][4];
  DProgram prog;
  // Programs recognised on the host and evaluated without the interpreter
  // (same IEEE operations in the same order): see FastEpi.
  int fast;
  float fast_c;
  int* status;
  // Split-K (conv and unbatched GEMM with EPI_NONE .. EPI_BIAS_ADD_RELU):
  // ksplit > 1 cuts each tile's k range into ksplit parts whose partial sums
  // go to `ws` ([ksplit][M][N], dense), then a reduce kernel adds them in
  // split order and applies the epilogue.  The launcher fills split_stride.
  int ksplit;
  float* ws;
  int64_t split_stride;
  // A operand source for launch_conv_gemm_tma (ATma): an im2col tensor map
  // over the NHWC input (convolutions, C a multiple of 32) or a tiled map over
  // the GEMM rows.
  int a_tma;
  // launch_conv_gemm_tma only: k-blocks per promotion round (0 = kRK).
  int rk;
  // Tensor-core passes per product: 3 (fp32 from three TF32 products,
  // hi*hi + hi*lo + lo*hi; the default, also for 0) or 1 (one TF32 product
  // of the truncated operands: the single-pass TF32 precision mode); 2 is
  // the BF16 mode of launch_conv_gemm_tma only (one kind::f16 product of
  // bf16-rounded operands, B from the bf16 plane's map passed as tmap_hi).
  int passes;
  // launch_conv_gemm_tma only: nonzero lets the epilogue's aux operand (the
  // residual, or an EPI_FAST operand) come per tile through shared memory by
  // TMA when conv_gemm_tma_aux_ok accepts the launch; 0 reads it from global
  // memory in the epilogue.  Same results either way.
  int aux_tma;
};

enum ATma : int {
  A_TMA_NONE = 0,    // A gathered by warps (launch_conv_gemm_tc)
  A_TMA_2D = 1,      // tiled 2-D tensor map over rows [M][K] (row stride ld)
  A_TMA_IM2COL = 2,  // im2col tensor map over the NHWC convolution input
  // im2col with few channels (C = 4, 8 or 16): a k-block spans 32 / C filter
  // taps, each loaded as its own dense [128 pixels][C] block (no swizzle)
  A_TMA_IM2COL_TAPS = 3,
};

enum FastEpi : int {
  FAST_NONE = 0,
  FAST_ADD = 1,          // acc + aux0
  FAST_DIVC_ADD = 2,     // (acc / c) + aux0
  FAST_SIGMOID_MUL = 3,  // (aux0 * (1 / (1 + exp(-aux1)))) * acc
  FAST_MULC_ADD = 4,     // (acc * c) + aux0: acc / d with d a power of two, c = 1 / d (exact)
  FAST_ADD_ADD = 5,      // (acc + aux0) + aux1: bias and residual
  FAST_GELU = 6,         // (t * (erf(t / c) + 1)) * 0.5 with t = acc + aux0: bias and exact GELU
};

// ---------------------------------------------------------------------------
// Fused attention (attention_tc.cu): out = softmax((q . k^T) / c + mask) . v
// per (batch, head), q [B, H, S, D], k / v [B, Hkv, Skv, D] (query head h
// reads key/value head h / (H / Hkv)), d contiguous, D <= 64 and a multiple
// of 16.  The three operands are addressed by 4-D tensor maps
// (make_attn_tensor_map); the mask by strides (0 = broadcast).
// ---------------------------------------------------------------------------
struct AttnParams {
  int B, H, Hkv, S, Skv, D;
  int QT, KT;                 // 128-row query tiles, 128-key tiles
  float scale;
  int scale_mul;              // scores = acc * scale (scale = 1 / c, c a power of two) or acc / scale (scale = c)
  const float* mask;          // nullptr: no mask
  int64_t m_st[4];            // mask strides over (b, h, i, j)
  int mb, mh;                 // skip-flag extents over b and h (1 where the mask is broadcast)
  const uint8_t* skip;        // set by launch_attention
  float* out;
  int64_t o_st[4];            // output strides over (b, h, i, d)
  int* status;
  int8_t cpos[3][3];          // per operand (q, k, v): map dim of (seq, head, batch), from make_attn_tensor_map
  int passes;                 // 3 (default, also 0): fp32 from three TF32 products; 1: single TF32 pass
};

bool attn_supported(int64_t D, int64_t Skv, int64_t H, int64_t Hkv);
// 4-D tensor map (d, seq, head, batch) over a [batch, heads, seq, dim] view with d contiguous.
// The outer dims are ordered by stride; cpos[0..2] receives the map dim of (seq, head, batch).
bool make_attn_tensor_map(const float* base, int64_t batch, int64_t heads, int64_t seq, int64_t dim, int64_t st_b,
                          int64_t st_h, int64_t st_s, void* tmap_out, int8_t* cpos);
// skip_flags: mb * mh * QT * KT bytes of device scratch (used when p.mask is set).
// skip_flags: per (mask block, query tile, key tile) flags that
// attn_skip_kernel fills before the attention kernel runs, unless
// flags_current says they already hold this mask's flags (a mask that never
// changes after the forward that first filled them).
bool launch_attention(const AttnParams& p, const void* tq, const void* tk, const void* tv, uint8_t* skip_flags,
                      bool flags_current, cudaStream_t s);

// Returns false (and launches nothing) when the shape is not supported.
bool launch_conv_gemm_tc(const ConvGemmParams& p, const void* tmap_hi, const void* tmap_lo, int block_n,
                         cudaStream_t s);

// Number of k splits for a contraction of this shape on `sms` SMs (1 = no
// split): splitting pays when the output tiles leave SMs idle.  The
// workspace it needs is ksplit * M * N floats (0 when ksplit is 1).
int choose_ksplit(int64_t M, int64_t N, int64_t K, int nb, int block_n, int epi, int sms, int rk = kRK);

// The split-K reduction of launch_conv_gemm_tc / launch_conv_gemm_tma: out =
// epilogue(sum over splits of ws[s]) in split order; p as given to the launch.
void launch_splitk_reduce(const ConvGemmParams& p, int64_t split_stride, cudaStream_t s);

// The TMA-fed kernel (conv_gemm_tma.cu): A by TMA (ConvGemmParams::a_tma and
// the map below), B as for launch_conv_gemm_tc.  Unbatched (nb == 1) only.
bool launch_conv_gemm_tma(const ConvGemmParams& p, const void* tmap_a, const void* tmap_hi, const void* tmap_lo,
                          int block_n, cudaStream_t s);

// A-operand tensor maps for launch_conv_gemm_tma.  im2col: NHWC input with
// element strides x_sn, x_sh, x_sw (channel stride 1), the convolution's
// filter size, stride, padding and dilation; C a multiple of 32 gives the
// A_TMA_IM2COL map (32-channel boxes, 128-byte swizzle), C = 4, 8 or 16 the
// A_TMA_IM2COL_TAPS map (C-channel boxes, no swizzle); *mode receives which.
// 2d: rows [M][K] with row stride ld (elements).  Return false when TMA
// cannot express it.
bool make_a_tensor_map_im2col(const float* x, int64_t images, int64_t H, int64_t W, int64_t C, int64_t x_sn,
                              int64_t x_sh, int64_t x_sw, int R, int S, int sh, int sw, int ph, int pw, int dh,
                              int dw, void* tmap_out, int* mode);
bool make_a_tensor_map_2d(const float* x, int64_t M, int64_t K, int64_t ld, void* tmap_out);
int conv_gemm_tma_smem_bytes(int block_n);
// Whether launch_conv_gemm_tma can stage this launch's epilogue operand in
// shared memory: an unsplit launch, EPI_BIAS_ADD_RELU (the residual) or an
// EPI_FAST form with one distinct aux tensor, that operand a row-major
// [M][N] view with 16-byte aligned rows, and the output in float4 rows.
bool conv_gemm_tma_aux_ok(const ConvGemmParams& p);

// Build the TMA descriptors for packed B planes [batch][N][ldk] (fp32).
// The BF16 mode's B operand for launch_conv_gemm_tma (passes 2, as its tmap_hi):
// a tiled map over the bf16 plane, boxes of 32 k x block_n rows, 64-byte swizzle.
bool make_b_tensor_map_bf16(const void* plane, int64_t batch, int64_t N, int64_t ldk16, int block_n,
                            void* tmap_out);
bool make_b_tensor_maps(const float* hi, const float* lo, int64_t batch, int64_t N, int64_t ldk, int block_n,
                        void* tmap_hi_out, void* tmap_lo_out);

// Shared-memory bytes the tensor-core kernel requests for a given block_n.
int conv_gemm_smem_bytes(int block_n);

}  // namespace kern
}  // namespace gawee
