// Execution planning for a gawee graph on one GPU.
//
// The planner turns the graph into a static list of kernel launches:
//   * layout-only ops (reshape, transpose, squeeze/unsqueeze, flatten, slice,
//     split, expand) become strided views of existing buffers;
//   * elementwise ops (the gawee arithmetic/activation/compare/cast ops and
//     the emitter's linalg.generic forms) become scalar programs over strided
//     operands, and single-use chains are fused into one launch, following the
//     producer -> single-use elementwise consumer rule of the reference's
//     LinalgFusion pass (middle/mlir/lib/Conversion/LinalgFusion.cpp:54-67);
//   * conv / linear / matmul become tensor-core launches whose B operand is
//     packed once (weights) or per forward (activations), and whose single-use
//     elementwise consumers are fused into the epilogue;
//   * ops that depend only on constants run once (prologue), weight packing
//     runs when its weight argument changes, everything else runs per forward;
//   * per-forward intermediates share one arena by liveness.
#pragma once

#include <cstdint>
#include <functional>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "ir.h"

namespace gawee {

struct View {
  int buf = -1;
  int64_t off = 0;  // elements
  DType dt = DType::F32;
  std::vector<int64_t> shape, st;
  int rank() const { return (int)shape.size(); }
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
  bool dense_rowmajor() const;  // contiguous in row-major order (size-1 dims ignored)
};

enum class BufKind { ARG, CONST, PERSIST, ARENA };
enum class Phase { PROLOGUE = 0, PACK = 1, MAIN = 2 };

struct Buf {
  BufKind kind = BufKind::ARENA;
  DType dt = DType::F32;
  int64_t elems = 0;
  int arg = -1;            // ARG: argument index
  int const_value = -1;    // CONST: graph value id holding the payload
  std::vector<uint8_t> host_init;  // CONST payload built by the planner
  int producer = -1;       // first op writing it
  size_t offset = 0;       // within its region (arena or persistent)
  bool live = false;       // needs storage
  void* ptr = nullptr;
  size_t bytes() const { return (size_t)elems * dtype_size(dt); }
};

enum class OpKind { EW, REDUCE, GREDUCE, SOFTMAX, GATHER, GATHER_ELEMS, REMAP, RANGE, POOL, TOPK, PACK, TC, ATTN };

struct Runtime;  // execution state (device pointers), runtime.cpp

struct Op {
  OpKind kind = OpKind::EW;
  Phase phase = Phase::MAIN;
  std::string name;
  bool dead = false;
  std::vector<View> reads, writes;  // for liveness and phases
  std::set<int> dep_args;           // PACK: arguments whose change requires re-running

  // EW: output view over the iteration space; inputs as views over the same
  // iteration space (strides per output dim, 0 = broadcast).
  EProgram prog;
  View out;
  std::vector<View> ins;

  // TC: structured contraction (see plan.cpp)
  struct Tc {
    bool conv = false;
    View x;                  // A source (conv input NHWC / GEMM lhs)
    View out;                // C [batch..., M, N] (GEMM) or NHWC (conv)
    int hi = -1, lo = -1;    // packed B plane buffers
    int64_t b_batch = 1, ldk = 0;
    int block_n = 128;
    int epi = 0;             // kern::Epi
    View bias, res;          // optional
    std::vector<View> aux;   // EPI_PROGRAM operands (views over C's shape)
    EProgram prog;           // EPI_PROGRAM body: r0 = acc(+bias), r1.. = aux
    // geometry
    int64_t H = 1, W = 1, C = 0, P = 0, Q = 1, M = 0, N = 0, K = 0;
    int R = 1, S = 1, sh = 1, sw = 1, ph = 0, pw = 0, dh = 1, dw = 1;
    int batch_rank = 0;
    std::vector<int64_t> batch_shape, a_bst, b_bst;
    double flops = 0;        // algorithmic 2*M*N*K over every batch (unpadded K)
  } tc;

  // ATTN: the attention cluster matmul(Q, K^T) -> div(c) -> add(mask) ->
  // softmax(-1) -> matmul(., V) as one fused op.  k and v are the key/value
  // tensors before any GQA head expansion ([B, Hkv, Skv, D], d contiguous).
  struct Attn {
    View q, k, v, mask, out;   // q, out: [B, H, S, D]; mask broadcast to [B, H, S, Skv]
    bool has_mask = false;
    int64_t B = 0, H = 0, Hkv = 0, S = 0, Skv = 0, D = 0;
    double c = 1.0;            // the divisor
    double flops = 0;          // 4 * B * H * S * Skv * D (both products over the full score matrix)
  } attn;

  // Non-structured ops: launcher resolving device pointers at launch time.
  std::function<void(Runtime&, void* stream)> launch;
};

struct Plan {
  Graph g;
  std::vector<Buf> bufs;
  std::vector<Op> ops;
  std::vector<View> value_view;  // per graph value
  std::vector<int> arg_buf;      // per argument
  std::vector<View> result_view; // per result (dense row-major)
  std::vector<int> prologue, pack, main;  // op indices per phase, in order
  size_t arena_bytes = 0, persist_bytes = 0;
  std::string summary() const;  // one line per main op: its name and execution_note
};

// Build the plan (throws std::runtime_error with a message on unsupported input).
// Buffer offsets are assigned: persistent buffers packed one after another,
// per-forward buffers placed in the arena by live interval over `main`.
std::unique_ptr<Plan> build_plan(Graph g);

// " [interp]" when the op's scalar program runs on the device interpreter
// (dynamically indexed registers: the slow path) -- an elementwise program
// with no specialised form, a generic reduction, or a GEMM epilogue program
// that is not one of the recognised forms; "" otherwise (runtime.cpp).
std::string execution_note(const Op& op);

}  // namespace gawee
