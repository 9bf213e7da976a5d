// libgawee_cuda runtime: device memory, launches, CUDA-graph replay and the
// C ABI declared in include/gawee_cuda.h.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <array>
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../../include/gawee_cuda.h"
#include "../kernels/kernels.h"
#include "ir.h"
#include "launch.h"
#include "plan.h"

namespace gawee {

int noalloc_take_status(cudaStream_t s);  // noalloc_gemm.cu

struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct StatusError : std::runtime_error {
  gawee_status code;
  StatusError(gawee_status c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define GCHECK(expr)                                                                            \
  do {                                                                                          \
    cudaError_t e_ = (expr);                                                                    \
    if (e_ != cudaSuccess) throw ::gawee::CudaError(std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)

struct alignas(64) TMap {
  unsigned char b[128];
};

// ---------------------------------------------------------------------------
// NCCL, loaded on first use so that the library itself has no NCCL dependency.
// ---------------------------------------------------------------------------
struct NcclApi {
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*groupStart)() = nullptr;
  ncclResult_t (*groupEnd)() = nullptr;
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*errorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

static NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.getUniqueId = (decltype(api.getUniqueId))dlsym(h, "ncclGetUniqueId");
    api.commInitRank = (decltype(api.commInitRank))dlsym(h, "ncclCommInitRank");
    api.commDestroy = (decltype(api.commDestroy))dlsym(h, "ncclCommDestroy");
    api.send = (decltype(api.send))dlsym(h, "ncclSend");
    api.recv = (decltype(api.recv))dlsym(h, "ncclRecv");
    api.groupStart = (decltype(api.groupStart))dlsym(h, "ncclGroupStart");
    api.groupEnd = (decltype(api.groupEnd))dlsym(h, "ncclGroupEnd");
    api.allGather = (decltype(api.allGather))dlsym(h, "ncclAllGather");
    api.errorString = (decltype(api.errorString))dlsym(h, "ncclGetErrorString");
    api.ok = api.getUniqueId && api.commInitRank && api.commDestroy && api.send && api.recv && api.groupStart &&
             api.groupEnd && api.allGather && api.errorString;
  });
  return api;
}

static void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw StatusError(GAWEE_ERR_NCCL, std::string(what) + ": " + nccl().errorString(r));
}

// ---------------------------------------------------------------------------
// Runtime state
// ---------------------------------------------------------------------------
struct Runtime {
  std::unique_ptr<Plan> plan;
  int device = 0;
  cudaStream_t own_stream = nullptr;
  void* persist = nullptr;
  void* arena = nullptr;
  int* d_status = nullptr;
  std::vector<char> dirty;       // per argument
  std::vector<char> pack_done;   // per op
  bool prologue_done = false;
  bool graph_mode = true;
  int forwards = 0;
  cudaGraphExec_t gexec = nullptr;
  cudaGraph_t graph = nullptr;
  std::vector<std::array<TMap, 3>> tmaps;  // per op (TC only): B hi, B lo, A (TMA-fed kernel)
  std::vector<int> a_tma;                  // per op (TC only): kern::ATma, A_TMA_NONE = warp gather
  int tma_rk = kern::kRK;                  // TMA kernel: k-blocks per promotion round
  int passes = 3;                          // tensor-core passes per product (precision mode: 3 fp32, 1 tf32)
  // BF16 mode: TMA-kernel contractions in bf16 from a bf16 copy of their B
  // planes (the other tensor-core kernels run single-pass TF32, passes 1)
  bool bf16 = false;
  std::vector<void*> bf16_plane;           // per op (TMA-kernel TC ops): [b_batch * N][bf16_ldk] bf16
  std::vector<TMap> bf16_map;              // per op: its tensor map
  std::vector<int64_t> bf16_ldk;           // per op: row pitch, a multiple of 8
  std::vector<char> bf16_fresh;            // per op: the plane matches the packed planes
  std::vector<int> ksplit;                 // per op (TC only): k splits, 1 = none
  std::vector<char> aux_tma;               // per op (TC only): epilogue operand staged by TMA (TMA kernel)
  std::vector<uint8_t*> attn_skip;         // per op (ATTN only): skip flags of the mask tiles
  // per op (ATTN only): 1 when the mask is a constant or a prologue result
  // (fixed once the prologue has run), 2 once its flags have been filled
  std::vector<char> attn_skip_static;
  std::vector<std::array<std::array<int8_t, 3>, 3>> attn_cpos;  // per op (ATTN): tensor-map dim order
  float* splitk_ws = nullptr;              // partial sums of split contractions (ops run in order: shared)
  ncclComm_t comm = nullptr;
  int world = 1, rank = 0;
  // output bytes of every rank (rank-major, one entry per output), exchanged
  // at gawee_dp_init: shards may differ by a row, so rank 0 receives each
  // peer's own count at the running offset
  std::vector<int64_t> peer_bytes;

  char* ptr(const View& v) const {
    const Buf& b = plan->bufs[v.buf];
    if (!b.ptr) throw std::runtime_error("internal: buffer without storage");
    return static_cast<char*>(b.ptr) + v.off * (int64_t)dtype_size(v.dt);
  }
  int* status() const { return d_status; }

  ~Runtime() {
    if (gexec) cudaGraphExecDestroy(gexec);
    if (graph) cudaGraphDestroy(graph);
    if (comm && nccl().ok) nccl().commDestroy(comm);
    if (persist) cudaFree(persist);
    if (arena) cudaFree(arena);
    if (d_status) cudaFree(d_status);
    if (splitk_ws) cudaFree(splitk_ws);
    for (uint8_t* f : attn_skip)
      if (f) cudaFree(f);
    for (void* b : bf16_plane)
      if (b) cudaFree(b);
    if (own_stream) cudaStreamDestroy(own_stream);
  }

  void allocate();
  void build_tensor_maps();
  void enable_bf16();
  void run_op(int o, cudaStream_t s);
  void run_list(const std::vector<int>& ops, cudaStream_t s, bool check);
  void forward(cudaStream_t s);
};

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

void Runtime::allocate() {
  Plan& P = *plan;
  auto& bufs = P.bufs;
  size_t poff = P.persist_bytes, arena_bytes = P.arena_bytes;
  if (poff) {
    if (cudaMalloc(&persist, poff) != cudaSuccess)
      throw StatusError(GAWEE_ERR_OOM, "cudaMalloc of " + std::to_string(poff) + " persistent bytes failed");
  }
  if (arena_bytes) {
    if (cudaMalloc(&arena, arena_bytes) != cudaSuccess)
      throw StatusError(GAWEE_ERR_OOM, "cudaMalloc of " + std::to_string(arena_bytes) + " arena bytes failed");
  }
  GCHECK(cudaMalloc(&d_status, sizeof(int)));
  GCHECK(cudaMemset(d_status, 0, sizeof(int)));
  for (auto& B : bufs) {
    if (!B.live) continue;
    B.ptr = static_cast<char*>(B.kind == BufKind::ARENA ? arena : persist) + B.offset;
  }
  // constants
  for (auto& B : bufs) {
    if (B.kind != BufKind::CONST || !B.ptr) continue;
    if (B.const_value >= 0) {
      const Value& v = P.g.values[B.const_value];
      GCHECK(cudaMemcpy(B.ptr, v.data.data(), v.data.size(), cudaMemcpyHostToDevice));
    } else if (!B.host_init.empty()) {
      GCHECK(cudaMemcpy(B.ptr, B.host_init.data(), B.host_init.size(), cudaMemcpyHostToDevice));
    }
  }
  dirty.assign(P.g.args.size(), 1);
  pack_done.assign(P.ops.size(), 0);
}

// Batch dims of a GEMM that only continue its rows are merged into M: B is
// broadcast along them and every other operand's stride along them equals
// the rows so far times its row stride (A, C and the epilogue's aux
// operands), innermost batch dim first.  The kernels then see one larger
// product with fewer (usually no) batch dims, e.g. a [64, 512, 576] x
// [576, N] projection becomes a single 32768-row GEMM.
struct GemmRows {
  int64_t M;
  int batch_rank;  // outer batch dims left
};
static GemmRows merged_rows(const Op& op) {
  const auto& t = op.tc;
  GemmRows g{t.M, t.batch_rank};
  if (t.conv || t.M <= 1) return g;
  const int ra = t.x.rank(), rc = t.out.rank();
  while (g.batch_rank > 0) {
    const int d = g.batch_rank - 1;
    const int64_t bs = t.batch_shape[d];
    if (bs != 1) {
      if (t.b_bst[d] != 0) break;
      if (t.a_bst[d] != g.M * t.x.st[ra - 2]) break;
      if (t.out.st[d] != g.M * t.out.st[rc - 2]) break;
      bool aux_ok = true;
      for (const View& v : t.aux) {
        const int rv = v.rank();
        if (v.st[d] != g.M * v.st[rv - 2]) aux_ok = false;
      }
      if (!aux_ok) break;
    }
    g.M *= bs;
    --g.batch_rank;
  }
  return g;
}

kern::ConvGemmParams tc_params(Runtime& rt, int o, const Op& op);

void Runtime::build_tensor_maps() {
  Plan& P = *plan;
  tmaps.assign(P.ops.size(), {});
  ksplit.assign(P.ops.size(), 1);
  aux_tma.assign(P.ops.size(), 0);
  a_tma.assign(P.ops.size(), kern::A_TMA_NONE);
  // GAWEE_TC_TMA=0 keeps every contraction on the warp-gather kernel
  bool use_tma = true;
  if (const char* e = std::getenv("GAWEE_TC_TMA")) use_tma = std::atoi(e) != 0;
  // The TMA kernel stages its epilogue's residual or fast-epilogue operand in
  // shared memory by TMA where the layout allows; GAWEE_TC_TMA_AUX=0 has the
  // epilogue read it from global memory instead (the same bits, slower)
  bool use_aux = true;
  if (const char* e = std::getenv("GAWEE_TC_TMA_AUX")) use_aux = std::atoi(e) != 0;
  int sms = 0;
  GCHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  // GAWEE_MAX_KSPLIT caps the k splits of small contractions (1 disables them)
  int cap = 32;
  if (const char* e = std::getenv("GAWEE_MAX_KSPLIT")) cap = std::max(1, std::atoi(e));
  // GAWEE_TMA_ROUND_KB: k-blocks per promotion round of the TMA kernel (1..16).
  // Longer rounds accumulate more truncating tensor-memory additions: at 4 the
  // ResNet-18 logits left the reference tolerance (1.47x of it, 0.80x at 2).
  if (const char* e = std::getenv("GAWEE_TMA_ROUND_KB")) tma_rk = std::min(16, std::max(1, std::atoi(e)));
  if (const char* e = std::getenv("GAWEE_PRECISION")) {
    const std::string m(e);
    if (m == "tf32") passes = 1;
    else if (m == "bf16") passes = 1, bf16 = true;
    else if (m == "fp32" || m.empty()) passes = 3;
    else throw StatusError(GAWEE_ERR_INVALID, "GAWEE_PRECISION must be fp32, tf32 or bf16, not " + m);
  }
  size_t ws_floats = 0;
  attn_skip.assign(P.ops.size(), nullptr);
  attn_skip_static.assign(P.ops.size(), 0);
  attn_cpos.assign(P.ops.size(), {});
  for (size_t o = 0; o < P.ops.size(); ++o) {
    const Op& op = P.ops[o];
    if (op.dead) continue;
    if (op.kind == OpKind::ATTN) {
      const auto& a = op.attn;
      auto map = [&](const View& v, int64_t heads, int64_t seq, int which) {
        return kern::make_attn_tensor_map(reinterpret_cast<const float*>(ptr(v)), a.B, heads, seq, a.D, v.st[0],
                                          v.st[1], v.st[2], tmaps[o][which].b, attn_cpos[o][which].data());
      };
      if (!map(a.q, a.H, a.S, 0) || !map(a.k, a.Hkv, a.Skv, 1) || !map(a.v, a.Hkv, a.Skv, 2))
        throw StatusError(GAWEE_ERR_UNSUPPORTED, "attention operands cannot be addressed by TMA for op " + op.name);
      if (a.has_mask) {
        const int64_t mb = a.mask.st[0] ? a.B : 1, mh = a.mask.st[1] ? a.H : 1;
        const int64_t n = mb * mh * ((a.S + 127) / 128) * ((a.Skv + 127) / 128);
        if (cudaMalloc(&attn_skip[o], (size_t)n) != cudaSuccess)
          throw StatusError(GAWEE_ERR_OOM, "cudaMalloc of attention skip flags failed");
        // a constant mask, or a persistent one written only by prologue ops
        // (the causal mask): its flags, once filled, hold for every forward
        const Buf& mbuf = P.bufs[a.mask.buf];
        bool fixed = mbuf.kind == BufKind::CONST;
        if (mbuf.kind == BufKind::PERSIST) {
          fixed = true;
          for (const Op& w : P.ops)
            for (const View& v : w.writes)
              if (!w.dead && v.buf == a.mask.buf && w.phase != Phase::PROLOGUE) fixed = false;
        }
        attn_skip_static[o] = fixed ? 1 : 0;
      }
      continue;
    }
    if (op.kind != OpKind::TC) continue;
    const auto& t = op.tc;
    const float* hi = static_cast<const float*>(P.bufs[t.hi].ptr);
    const float* lo = static_cast<const float*>(P.bufs[t.lo].ptr);
    if (!kern::make_b_tensor_maps(hi, lo, t.b_batch, t.N, t.ldk, t.block_n, tmaps[o][0].b, tmaps[o][1].b))
      throw std::runtime_error("cuTensorMapEncodeTiled failed for op " + op.name);
    const GemmRows gr = merged_rows(op);
    int nb = 1;
    for (int d = 0; d < gr.batch_rank; ++d) nb *= (int)t.batch_shape[d];
    // A by TMA when the copy engine can address it: a convolution over whole
    // 32-channel k-blocks (im2col), or an unbatched GEMM with aligned rows
    if (use_tma && nb == 1) {
      const float* x = reinterpret_cast<const float*>(ptr(t.x));
      // tap blocks (C = 4, 8, 16) only on request: on the ResNet stem (C = 4,
      // 16-byte pixels) the im2col copies ran slower than the warp gather
      bool taps = false;
      if (const char* e = std::getenv("GAWEE_TC_TMA_TAPS")) taps = std::atoi(e) != 0;
      if (t.conv && (t.C % 32 == 0 || (taps && (t.C == 4 || t.C == 8 || t.C == 16)))) {
        int mode = kern::A_TMA_NONE;
        if (kern::make_a_tensor_map_im2col(x, t.x.shape[0], t.H, t.W, t.C, t.x.shape[0] > 1 ? t.x.st[0] : 0,
                                           t.x.st[2], t.x.st[3], t.R, t.S, t.sh, t.sw, t.ph, t.pw, t.dh, t.dw,
                                           tmaps[o][2].b, &mode))
          a_tma[o] = mode;
      } else if (!t.conv) {
        const int r = t.x.rank();
        if (t.x.st[r - 1] == 1 &&
            kern::make_a_tensor_map_2d(x, gr.M, t.K, gr.M > 1 ? t.x.st[r - 2] : 0, tmaps[o][2].b))
          a_tma[o] = kern::A_TMA_2D;
      }
    }
    const int k = std::min(cap, kern::choose_ksplit(gr.M, t.N, t.K, nb, t.block_n, t.epi, sms,
                                                    a_tma[o] != kern::A_TMA_NONE ? tma_rk : kern::kRK));
    ksplit[o] = k;
    if (k > 1) ws_floats = std::max(ws_floats, (size_t)k * (size_t)gr.M * (size_t)t.N);
    if (use_aux && a_tma[o] != kern::A_TMA_NONE && k == 1)
      aux_tma[o] = kern::conv_gemm_tma_aux_ok(tc_params(*this, (int)o, op)) ? 1 : 0;
  }
  if (ws_floats) {
    if (cudaMalloc(&splitk_ws, ws_floats * sizeof(float)) != cudaSuccess)
      throw StatusError(GAWEE_ERR_OOM, "cudaMalloc of the split-K workspace failed");
  }
  if (bf16) enable_bf16();
}

// The BF16 mode's per-op state: a bf16 B plane and its tensor map for every
// contraction on the TMA kernel (allocated once, on the first switch to the
// mode); an op whose plane cannot be mapped keeps single-pass TF32.  Planes
// are filled from the packed planes before the next forward's main phase.
void Runtime::enable_bf16() {
  Plan& P = *plan;
  bf16_plane.resize(P.ops.size(), nullptr);
  bf16_map.resize(P.ops.size());
  bf16_ldk.resize(P.ops.size(), 0);
  bf16_fresh.assign(P.ops.size(), 0);
  for (size_t o = 0; o < P.ops.size(); ++o) {
    const Op& op = P.ops[o];
    if (op.dead || op.kind != OpKind::TC || a_tma[o] == kern::A_TMA_NONE || bf16_plane[o]) continue;
    const auto& t = op.tc;
    const int64_t ldk16 = (t.ldk + 7) / 8 * 8;
    void* b = nullptr;
    if (cudaMalloc(&b, (size_t)(t.b_batch * t.N * ldk16) * 2) != cudaSuccess)
      throw StatusError(GAWEE_ERR_OOM, "cudaMalloc of a bf16 B plane failed");
    if (!kern::make_b_tensor_map_bf16(b, t.b_batch, t.N, ldk16, t.block_n, bf16_map[o].b)) {
      cudaFree(b);
      continue;
    }
    bf16_plane[o] = b;
    bf16_ldk[o] = ldk16;
  }
}

// ---------------------------------------------------------------------------
// Structured launches
// ---------------------------------------------------------------------------
static kern::DProgram to_device(const EProgram& p) {
  if ((int)p.code.size() > kern::kMaxInstr || (int)p.reg_types.size() > kern::kMaxRegs)
    throw std::runtime_error("scalar program too large for the device interpreter");
  kern::DProgram d{};
  d.n_code = (int)p.code.size();
  d.n_args = p.n_args;
  d.result = p.result;
  for (size_t k = 0; k < p.code.size(); ++k) {
    const EInstr& in = p.code[k];
    auto& o = d.code[k];
    o.op = (uint8_t)in.op;
    o.ty = (uint8_t)in.ty;
    o.rty = (uint8_t)in.rty;
    o.pred = in.pred;
    o.dst = (int8_t)in.dst;
    o.a = (int8_t)in.a;
    o.b = (int8_t)in.b;
    o.c = (int8_t)in.c;
    o.fimm = in.fimm;
    o.iimm = in.iimm;
  }
  return d;
}

// Recognises the GEMM epilogue programs the emitter's decoder blocks produce
// (residual add, score scale + mask, SiLU-gated product) so the kernel can
// evaluate them without the interpreter.  Registers: r0 = accumulator,
// r1.. = aux operands; every match checks the exact operation sequence, so
// the fast path computes the same IEEE operations in the same order.
// *swap_aux is set when the program adds aux 1 before aux 0 (FAST_ADD_ADD):
// the caller then swaps the two operands so the kernel's order is the program's.
static int match_fast_epilogue(const EProgram& p, float* c, bool* swap_aux = nullptr) {
  const auto& k = p.code;
  auto f32 = [&](const EInstr& in) { return in.ty == DType::F32 && in.rty == DType::F32; };
  auto uses = [](const EInstr& in, int x, int y) { return (in.a == x && in.b == y) || (in.a == y && in.b == x); };
  for (const auto& in : k)
    if (!f32(in)) return kern::FAST_NONE;
  if (p.n_args == 2 && k.size() == 1 && k[0].op == EOp::ADDF && uses(k[0], 0, 1) && p.result == k[0].dst)
    return kern::FAST_ADD;
  if (p.n_args == 2 && k.size() == 3 && k[0].op == EOp::CONST && k[1].op == EOp::DIVF && k[1].a == 0 &&
      k[1].b == k[0].dst && k[2].op == EOp::ADDF && uses(k[2], k[1].dst, 1) && p.result == k[2].dst) {
    *c = (float)k[0].fimm;
    // For c = 2^e, x / c and x * 2^-e are the same real number, and IEEE
    // division and multiplication both round that exact value, so the two
    // agree bit for bit (2^-e must itself be a normal float: e <= 126).
    int e = 0;
    const float mant = std::frexp(*c, &e);
    if (mant == 0.5f && e >= 1 && e <= 64) {
      *c = std::ldexp(1.0f, 1 - e);
      return kern::FAST_MULC_ADD;
    }
    return kern::FAST_DIVC_ADD;
  }
  if (p.n_args == 3 && k.size() == 7 && k[0].op == EOp::CONST && k[0].fimm == 1.0 && k[1].op == EOp::NEGF &&
      k[1].a == 2 && k[2].op == EOp::EXP && k[2].a == k[1].dst && k[3].op == EOp::ADDF &&
      uses(k[3], k[0].dst, k[2].dst) && k[4].op == EOp::DIVF && k[4].a == k[0].dst && k[4].b == k[3].dst &&
      k[5].op == EOp::MULF && uses(k[5], 1, k[4].dst) && k[6].op == EOp::MULF && uses(k[6], k[5].dst, 0) &&
      p.result == k[6].dst)
    return kern::FAST_SIGMOID_MUL;
  // (acc + aux0) + aux1, or (acc + aux1) + aux0: a bias and a residual
  if (p.n_args == 3 && k.size() == 2 && k[0].op == EOp::ADDF && k[1].op == EOp::ADDF && p.result == k[1].dst) {
    if (uses(k[0], 0, 1) && uses(k[1], k[0].dst, 2)) return kern::FAST_ADD_ADD;
    if (uses(k[0], 0, 2) && uses(k[1], k[0].dst, 1)) {
      if (swap_aux) *swap_aux = true;
      return kern::FAST_ADD_ADD;
    }
  }
  // exact GELU after a bias: t = acc + aux0, (t * (erf(t / c) + 1)) * 0.5, the
  // constants wherever the code holds them; traced back from the result
  if (p.n_args == 2 && k.size() == 9) {
    auto def = [&](int r) -> const EInstr* {
      for (const auto& in : k)
        if (in.dst == r) return &in;
      return nullptr;
    };
    auto is_const = [&](int r, double v) {
      const EInstr* d = def(r);
      return d && d->op == EOp::CONST && d->fimm == v;
    };
    const EInstr* R = def(p.result);
    if (!R || R->op != EOp::MULF) return kern::FAST_NONE;
    const int w = is_const(R->b, 0.5) ? R->a : is_const(R->a, 0.5) ? R->b : -1;
    const EInstr* W = def(w);
    if (!W || W->op != EOp::MULF) return kern::FAST_NONE;
    for (int side = 0; side < 2; ++side) {
      const EInstr* T = def(side ? W->b : W->a);
      const EInstr* V = def(side ? W->a : W->b);
      if (!T || !V || T->op != EOp::ADDF || !uses(*T, 0, 1) || V->op != EOp::ADDF) continue;
      const int e = is_const(V->b, 1.0) ? V->a : is_const(V->a, 1.0) ? V->b : -1;
      const EInstr* E = def(e);
      if (!E || E->op != EOp::ERF) continue;
      const EInstr* U = def(E->a);
      if (!U || U->op != EOp::DIVF || U->a != T->dst) continue;
      const EInstr* C = def(U->b);
      if (!C || C->op != EOp::CONST) continue;
      *c = (float)C->fimm;
      return kern::FAST_GELU;
    }
  }
  return kern::FAST_NONE;
}

// Recognises the small f32 elementwise programs decoder and normalisation
// blocks produce (copy, square, negate, sqrt(x + eps), x / r * w, a*b + c*d)
// so the kernels evaluate them without the interpreter; each match checks
// the exact operation sequence and records operand indices.
static void match_fast_ew(const EProgram& p, kern::EwParams& e) {
  const auto& k = p.code;
  int fast = kern::EW_INTERP;
  std::vector<int> sel;  // program arguments in the order the fast form reads them
  for (DType t : p.reg_types)
    if (t != DType::F32) return;
  for (const auto& in : k)
    if (in.ty != DType::F32 || in.rty != DType::F32) return;
  auto arg = [&](int r) { return r >= 0 && r < p.n_args; };
  if (k.empty() && arg(p.result)) {
    fast = kern::EW_COPY;
    sel = {p.result};
  } else if (k.size() == 1 && k[0].dst == p.result && k[0].op == EOp::NEGF && arg(k[0].a)) {
    fast = kern::EW_NEG;
    sel = {k[0].a};
  } else if (k.size() == 1 && k[0].dst == p.result && k[0].op == EOp::MULF && arg(k[0].a) && k[0].a == k[0].b) {
    fast = kern::EW_SQR;
    sel = {k[0].a};
  } else if (k.size() == 2 && k[0].op == EOp::CONST && k[1].op == EOp::POWF && k[0].fimm == 2.0 && arg(k[1].a) &&
             k[1].b == k[0].dst && k[1].dst == p.result) {
    fast = kern::EW_SQR;  // the interpreter evaluates powf(x, 2) as x * x
    sel = {k[1].a};
  } else if (k.size() == 2 && k[0].op == EOp::DIVF && arg(k[0].a) && arg(k[0].b) && k[1].op == EOp::MULF &&
             k[1].dst == p.result && ((k[1].a == k[0].dst && arg(k[1].b)) || (k[1].b == k[0].dst && arg(k[1].a)))) {
    fast = kern::EW_DIV_MUL;
    sel = {k[0].a, k[0].b, k[1].a == k[0].dst ? k[1].b : k[1].a};
  } else if (k.size() == 3 && k[0].op == EOp::CONST && k[1].op == EOp::ADDF && k[2].op == EOp::SQRT &&
             k[2].a == k[1].dst && k[2].dst == p.result &&
             ((k[1].a == k[0].dst && arg(k[1].b)) || (k[1].b == k[0].dst && arg(k[1].a)))) {
    fast = kern::EW_ADDC_SQRT;
    sel = {k[1].a == k[0].dst ? k[1].b : k[1].a};
    e.fk = (float)k[0].fimm;
  } else if (k.size() == 3 && k[0].op == EOp::MULF && k[1].op == EOp::MULF && k[2].op == EOp::ADDF &&
             arg(k[0].a) && arg(k[0].b) && arg(k[1].a) && arg(k[1].b) && k[2].dst == p.result &&
             ((k[2].a == k[0].dst && k[2].b == k[1].dst) || (k[2].a == k[1].dst && k[2].b == k[0].dst))) {
    fast = kern::EW_MUL_MUL_ADD;  // a*b + c*d: IEEE addition is commutative, so the product order is free
    sel = {k[0].a, k[0].b, k[1].a, k[1].b};
  } else {
    return;
  }
  kern::EwOperand orig[kern::kMaxIn];
  for (int i = 0; i < e.n_in; ++i) orig[i] = e.in[i];
  for (size_t i = 0; i < sel.size(); ++i) e.in[i] = orig[sel[i]];
  e.n_in = (int)sel.size();
  e.fast = fast;
}

std::string execution_note(const Op& op) {
  if (op.kind == OpKind::GREDUCE) return " [interp]";
  if (op.kind == OpKind::TC) {
    float c = 0.0f;
    return op.tc.epi == kern::EPI_PROGRAM && match_fast_epilogue(op.tc.prog, &c) == kern::FAST_NONE
               ? " [interp epilogue]"
               : "";
  }
  if (op.kind != OpKind::EW) return "";
  bool all_f32 = op.out.dt == DType::F32;
  for (const auto& v : op.ins) all_f32 = all_f32 && v.dt == DType::F32;
  kern::EwParams p{};
  p.fast = kern::EW_INTERP;
  p.n_in = (int)std::min<size_t>(op.ins.size(), kern::kMaxIn);
  if (all_f32) match_fast_ew(op.prog, p);
  return p.fast == kern::EW_INTERP ? " [interp]" : "";
}

static void launch_ew(Runtime& rt, const Op& op, cudaStream_t s) {
  const View& out = op.out;
  int r = out.rank();
  // iteration dims: drop size-1 dims, order by output stride (outermost first), merge contiguous
  std::vector<int> dims;
  for (int d = 0; d < r; ++d)
    if (out.shape[d] != 1) dims.push_back(d);
  std::stable_sort(dims.begin(), dims.end(), [&](int a, int b) { return out.st[a] > out.st[b]; });
  std::vector<int64_t> shape;
  std::vector<std::vector<int64_t>> st(op.ins.size() + 1);
  for (int d : dims) {
    shape.push_back(out.shape[d]);
    st[0].push_back(out.st[d]);
    for (size_t k = 0; k < op.ins.size(); ++k) st[k + 1].push_back(op.ins[k].st[d]);
  }
  // merge dim i into i-1 when every operand is contiguous across them
  for (int i = (int)shape.size() - 1; i > 0; --i) {
    bool ok = true;
    for (auto& s2 : st)
      if (s2[i - 1] != s2[i] * shape[i]) ok = false;
    if (!ok) continue;
    shape[i - 1] *= shape[i];
    shape.erase(shape.begin() + i);
    for (auto& s2 : st) {
      s2[i - 1] = s2[i];
      s2.erase(s2.begin() + i);
    }
  }
  if (shape.empty()) {
    shape.push_back(1);
    for (auto& s2 : st) s2.push_back(0);
  }
  if ((int)shape.size() > kern::kMaxRank) throw std::runtime_error("elementwise iteration rank too large");
  if ((int)op.ins.size() > kern::kMaxIn) throw std::runtime_error("too many elementwise operands");
  kern::EwParams p{};
  p.rank = (int)shape.size();
  p.n_in = (int)op.ins.size();
  p.numel = 1;
  for (size_t d = 0; d < shape.size(); ++d) {
    p.shape[d] = shape[d];
    p.numel *= shape[d];
    p.out.st[d] = st[0][d];
    for (size_t k = 0; k < op.ins.size(); ++k) p.in[k].st[d] = st[k + 1][d];
  }
  p.out.ptr = rt.ptr(out);
  p.out.dt = (int8_t)out.dt;
  for (size_t k = 0; k < op.ins.size(); ++k) {
    p.in[k].ptr = rt.ptr(op.ins[k]);
    p.in[k].dt = (int8_t)op.ins[k].dt;
  }
  p.prog = to_device(op.prog);
  bool all_f32 = out.dt == DType::F32;
  for (const auto& v : op.ins) all_f32 = all_f32 && v.dt == DType::F32;
  if (all_f32) match_fast_ew(op.prog, p);
  p.status = rt.status();
  kern::launch_elementwise(p, s);
}

// The contraction's launch parameters, from the op and the runtime's
// per-op choices (A source, k splits, aux staging).
kern::ConvGemmParams tc_params(Runtime& rt, int o, const Op& op) {
  const auto& t = op.tc;
  kern::ConvGemmParams p{};
  p.x = reinterpret_cast<const float*>(rt.ptr(t.x));
  // strides of size-1 dims are never stepped; zero them so alignment checks see only real strides
  if (t.conv) {
    p.x_sn = t.x.shape[0] > 1 ? t.x.st[0] : 0;
    p.x_sh = t.x.st[2];
    p.x_sw = t.x.st[3];
  } else {
    int r = t.x.rank();
    p.x_sn = 0;
    p.x_sh = t.M > 1 ? t.x.st[r - 2] : 0;
    p.x_sw = 0;
  }
  p.H = t.H; p.W = t.W; p.C = t.C; p.P = t.P; p.Q = t.Q;
  p.R = t.R; p.S = t.S; p.sh = t.sh; p.sw = t.sw; p.ph = t.ph; p.pw = t.pw; p.dh = t.dh; p.dw = t.dw;
  p.M = t.M; p.N = t.N; p.K = t.K;
  const GemmRows gr = merged_rows(op);
  if (gr.M != t.M) p.M = p.P = p.H = gr.M;  // batch dims merged into the rows (a GEMM: H = P = M, Q = 1)
  p.nb = 1;
  p.batch_rank = gr.batch_rank;
  for (int d = 0; d < gr.batch_rank; ++d) {
    p.batch_shape[d] = t.batch_shape[d];
    p.a_bst[d] = t.a_bst[d];
    p.b_bst[d] = t.b_bst[d];
    p.c_bst[d] = t.out.st[d];
    p.nb *= (int)t.batch_shape[d];
  }
  p.out = reinterpret_cast<float*>(rt.ptr(t.out));
  if (t.conv) {
    p.ldc = t.out.st[3];
    p.ldc_n = t.out.st[1];
  } else {
    int r = t.out.rank();
    p.ldc = t.out.st[r - 2];
    p.ldc_n = t.out.st[r - 1];
  }
  p.epi = t.epi;
  p.bias = t.bias.buf >= 0 ? reinterpret_cast<const float*>(rt.ptr(t.bias)) : nullptr;
  p.res = t.res.buf >= 0 ? reinterpret_cast<const float*>(rt.ptr(t.res)) : nullptr;
  p.n_aux = (int)t.aux.size();
  for (size_t a = 0; a < t.aux.size(); ++a) {
    const View& v = t.aux[a];
    int r = v.rank();
    p.aux[a] = reinterpret_cast<const float*>(rt.ptr(v));
    p.aux_sm[a] = v.st[r - 2];
    p.aux_sn[a] = v.st[r - 1];
    for (int d = 0; d < t.batch_rank; ++d) p.aux_sb[a][d] = v.st[d];
  }
  if (t.epi == kern::EPI_PROGRAM) {
    p.prog = to_device(t.prog);
    bool swap = false;
    p.fast = match_fast_epilogue(t.prog, &p.fast_c, &swap);
    if (p.fast != kern::FAST_NONE) p.epi = kern::EPI_FAST;
    if (swap) {  // the form adds aux 0 first
      std::swap(p.aux[0], p.aux[1]);
      std::swap(p.aux_sm[0], p.aux_sm[1]);
      std::swap(p.aux_sn[0], p.aux_sn[1]);
      for (int d = 0; d < 4; ++d) std::swap(p.aux_sb[0][d], p.aux_sb[1][d]);
    }
  }
  p.status = rt.status();
  p.passes = rt.passes;
  if (rt.bf16 && o < (int)rt.bf16_plane.size() && rt.bf16_plane[o]) p.passes = 2;
  if (rt.ksplit[o] > 1 && p.epi <= kern::EPI_BIAS_ADD_RELU) {
    p.ksplit = rt.ksplit[o];
    p.ws = rt.splitk_ws;
  }
  if (rt.a_tma[o] != kern::A_TMA_NONE) {
    p.a_tma = rt.a_tma[o];
    p.rk = rt.tma_rk;
    p.aux_tma = o < (int)rt.aux_tma.size() ? rt.aux_tma[o] : 0;
  }
  return p;
}

static void launch_tc(Runtime& rt, int o, const Op& op, cudaStream_t s) {
  const auto& t = op.tc;
  const kern::ConvGemmParams p = tc_params(rt, o, op);
  bool launched;
  if (rt.a_tma[o] != kern::A_TMA_NONE) {
    const void* b_map = p.passes == 2 ? static_cast<const void*>(rt.bf16_map[o].b) : rt.tmaps[o][0].b;
    launched = kern::launch_conv_gemm_tma(p, rt.tmaps[o][2].b, b_map, rt.tmaps[o][1].b, t.block_n, s);
  } else {
    launched = kern::launch_conv_gemm_tc(p, rt.tmaps[o][0].b, rt.tmaps[o][1].b, t.block_n, s);
  }
  if (!launched) throw StatusError(GAWEE_ERR_UNSUPPORTED, "tensor-core launch rejected the shape of op " + op.name);
}

static void launch_attn(Runtime& rt, int o, const Op& op, cudaStream_t s) {
  const auto& a = op.attn;
  kern::AttnParams p{};
  p.B = (int)a.B; p.H = (int)a.H; p.Hkv = (int)a.Hkv; p.S = (int)a.S; p.Skv = (int)a.Skv; p.D = (int)a.D;
  p.QT = (int)((a.S + 127) / 128);
  p.KT = (int)((a.Skv + 127) / 128);
  // (acc / c): a power-of-two c divides exactly as a multiply by 1 / c
  int e = 0;
  const double mant = std::frexp(a.c, &e);
  if (mant == 0.5 && e >= -100 && e <= 100) {
    p.scale = (float)std::ldexp(1.0, 1 - e);
    p.scale_mul = 1;
  } else {
    p.scale = (float)a.c;
    p.scale_mul = 0;
  }
  if (a.has_mask) {
    p.mask = reinterpret_cast<const float*>(rt.ptr(a.mask));
    for (int d = 0; d < 4; ++d) p.m_st[d] = a.mask.st[d];
    p.mb = a.mask.st[0] ? p.B : 1;
    p.mh = a.mask.st[1] ? p.H : 1;
  }
  p.out = reinterpret_cast<float*>(rt.ptr(a.out));
  for (int d = 0; d < 4; ++d) p.o_st[d] = a.out.st[d];
  for (int w = 0; w < 3; ++w)
    for (int i = 0; i < 3; ++i) p.cpos[w][i] = rt.attn_cpos[o][w][i];
  p.status = rt.status();
  p.passes = rt.passes;
  char& fixed = rt.attn_skip_static[o];
  if (!kern::launch_attention(p, rt.tmaps[o][0].b, rt.tmaps[o][1].b, rt.tmaps[o][2].b, rt.attn_skip[o], fixed == 2,
                              s))
    throw StatusError(GAWEE_ERR_UNSUPPORTED, "attention launch rejected the shape of op " + op.name);
  if (fixed == 1) fixed = 2;  // filled by this launch, valid for every later forward
}

void Runtime::run_op(int o, cudaStream_t s) {
  const Op& op = plan->ops[o];
  if (op.kind == OpKind::EW) launch_ew(*this, op, s);
  else if (op.kind == OpKind::TC) launch_tc(*this, o, op, s);
  else if (op.kind == OpKind::ATTN) launch_attn(*this, o, op, s);
  else op.launch(*this, s);
}

void Runtime::run_list(const std::vector<int>& ops, cudaStream_t s, bool check) {
  for (int o : ops) {
    run_op(o, s);
    if (check) {
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) throw CudaError("launch of " + plan->ops[o].name + ": " + cudaGetErrorString(e));
    }
  }
}

void Runtime::forward(cudaStream_t s) {
  if (!prologue_done) {
    run_list(plan->prologue, s, true);
    prologue_done = true;
  }
  bool repacked = false;
  for (int o : plan->pack) {
    const Op& op = plan->ops[o];
    bool need = !pack_done[o];
    for (int a : op.dep_args) need = need || dirty[a];
    if (need) {
      run_op(o, s);
      GCHECK(cudaGetLastError());
      pack_done[o] = 1;
      repacked = true;
    }
  }
  if (repacked) std::fill(bf16_fresh.begin(), bf16_fresh.end(), 0);
  if (bf16) {
    for (size_t o = 0; o < bf16_plane.size(); ++o) {
      if (!bf16_plane[o] || bf16_fresh[o]) continue;
      const auto& t = plan->ops[o].tc;
      kern::launch_planes_to_bf16(static_cast<const float*>(plan->bufs[t.hi].ptr),
                                  static_cast<const float*>(plan->bufs[t.lo].ptr), bf16_plane[o], t.b_batch * t.N,
                                  t.ldk, bf16_ldk[o], s);
      GCHECK(cudaGetLastError());
      bf16_fresh[o] = 1;
    }
  }
  // First forward runs eagerly (it also sets kernel attributes); later ones
  // replay a CUDA graph of the main sequence.
  if (graph_mode && forwards > 0 && s != nullptr) {
    if (!gexec) {
      GCHECK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      try {
        run_list(plan->main, s, false);
      } catch (...) {
        cudaGraph_t g;
        cudaStreamEndCapture(s, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      GCHECK(cudaStreamEndCapture(s, &graph));
      GCHECK(cudaGraphInstantiate(&gexec, graph, 0));
    }
    GCHECK(cudaGraphLaunch(gexec, s));
  } else {
    run_list(plan->main, s, true);
  }
  std::fill(dirty.begin(), dirty.end(), 0);
  ++forwards;
}

// ---------------------------------------------------------------------------
// Launch builders (launch.h)
// ---------------------------------------------------------------------------
namespace launch {

Fn remap(kern::RemapParams rp, const View& in, const View& out) {
  return [rp, in, out](Runtime& rt, void* s) mutable {
    rp.in = rt.ptr(in);
    rp.out = rt.ptr(out);
    kern::launch_remap(rp, static_cast<cudaStream_t>(s));
  };
}

Fn nchw_to_nhwc4(const View& in, const View& out, int64_t N, int C, int C4, int64_t HW, int64_t in_sn, int64_t in_sc) {
  return [=](Runtime& rt, void* s) {
    kern::launch_nchw_to_nhwc4(reinterpret_cast<const float*>(rt.ptr(in)), reinterpret_cast<float*>(rt.ptr(out)), N, C,
                               C4, HW, in_sn, in_sc, static_cast<cudaStream_t>(s));
  };
}

static void split_dims(const View& in, const std::vector<bool>& red, kern::ReduceParams* rp,
                       kern::GenericReduceParams* gp, const View& out) {
  std::vector<int64_t> ks, kst, rs, rst;
  for (int d = 0; d < in.rank(); ++d) {
    if (red[d]) { rs.push_back(in.shape[d]); rst.push_back(in.st[d]); }
    else { ks.push_back(in.shape[d]); kst.push_back(in.st[d]); }
  }
  // output strides over kept dims: the output is dense row-major over its own
  // shape, which equals the kept dims with unit dims inserted (keepdims)
  std::vector<int64_t> ost;
  {
    int k = 0;
    for (int d = 0; d < in.rank(); ++d) {
      if (red[d]) continue;
      (void)k;
      ost.push_back(0);
    }
    // strides over kept dims in row-major order of the kept shape
    int64_t acc = 1;
    for (int i = (int)ks.size() - 1; i >= 0; --i) {
      ost[i] = acc;
      acc *= ks[i];
    }
  }
  if (ks.size() > (size_t)kern::kMaxRank || rs.size() > (size_t)kern::kMaxRank)
    throw std::runtime_error("reduction rank too large");
  auto fill = [&](auto* p) {
    p->kept_rank = (int)ks.size();
    p->red_rank = (int)rs.size();
    p->rows = 1;
    p->cols = 1;
    for (size_t i = 0; i < ks.size(); ++i) {
      p->kept_shape[i] = ks[i];
      p->kept_st[i] = kst[i];
      p->out_st[i] = ost[i];
      p->rows *= ks[i];
    }
    for (size_t i = 0; i < rs.size(); ++i) {
      p->red_shape[i] = rs[i];
      p->red_st[i] = rst[i];
      p->cols *= rs[i];
    }
  };
  if (rp) fill(rp);
  if (gp) fill(gp);
  (void)out;
}

Fn reduce(const View& in, const View& out, const std::vector<bool>& red, bool mean, float count) {
  if (!out.dense_rowmajor()) throw std::runtime_error("reduce output must be dense");
  kern::ReduceParams rp{};
  split_dims(in, red, &rp, nullptr, out);
  rp.mode = mean ? 1 : 0;
  rp.count = count;
  return [rp, in, out](Runtime& rt, void* s) mutable {
    rp.in = reinterpret_cast<const float*>(rt.ptr(in));
    rp.out = reinterpret_cast<float*>(rt.ptr(out));
    kern::launch_reduce_f32(rp, static_cast<cudaStream_t>(s));
  };
}

Fn rope(const View& x, const View& cs, const View& sn, const View& out) {
  kern::RopeParams rp{};
  rp.rank = out.rank();
  if (rp.rank < 1 || rp.rank > 4) throw std::runtime_error("rope: rank must be 1..4");
  rp.numel = out.numel();
  rp.half = out.shape[rp.rank - 1] / 2;
  for (int d = 0; d < rp.rank; ++d) {
    rp.shape[d] = out.shape[d];
    rp.x_st[d] = x.st[d];
    rp.c_st[d] = cs.st[d];
    rp.s_st[d] = sn.st[d];
  }
  return [rp, x, cs, sn, out](Runtime& rt, void* s) mutable {
    rp.x = reinterpret_cast<const float*>(rt.ptr(x));
    rp.cs = reinterpret_cast<const float*>(rt.ptr(cs));
    rp.sn = reinterpret_cast<const float*>(rt.ptr(sn));
    rp.out = reinterpret_cast<float*>(rt.ptr(out));
    kern::launch_rope(rp, static_cast<cudaStream_t>(s));
  };
}

Fn rownorm(const View& x, int64_t rows, int64_t cols, int64_t x_rs, const View& w, int64_t w_st, const View& b,
           int64_t b_st, const View& out, float eps, bool centered) {
  kern::RowNormParams rp{};
  rp.rows = rows;
  rp.cols = cols;
  rp.x_rs = x_rs;
  rp.w_st = w_st;
  rp.b_st = b_st;
  rp.eps = eps;
  rp.centered = centered ? 1 : 0;
  return [rp, x, w, b, out](Runtime& rt, void* s) mutable {
    rp.x = reinterpret_cast<const float*>(rt.ptr(x));
    rp.w = reinterpret_cast<const float*>(rt.ptr(w));
    rp.b = b.buf >= 0 ? reinterpret_cast<const float*>(rt.ptr(b)) : nullptr;
    rp.out = reinterpret_cast<float*>(rt.ptr(out));
    kern::launch_rownorm(rp, static_cast<cudaStream_t>(s));
  };
}

Fn generic_reduce(const View& in, const View& out, const std::vector<bool>& red, const EProgram& body) {
  kern::GenericReduceParams gp{};
  split_dims(in, red, nullptr, &gp, out);
  gp.in_dt = (int8_t)in.dt;
  gp.out_dt = (int8_t)out.dt;
  gp.prog = to_device(body);
  return [gp, in, out](Runtime& rt, void* s) mutable {
    gp.in = rt.ptr(in);
    gp.out = rt.ptr(out);
    gp.status = rt.status();
    kern::launch_generic_reduce(gp, static_cast<cudaStream_t>(s));
  };
}

Fn pool(kern::PoolParams pp, const View& in, const View& out) {
  return [pp, in, out](Runtime& rt, void* s) mutable {
    pp.in = reinterpret_cast<const float*>(rt.ptr(in));
    pp.out = reinterpret_cast<float*>(rt.ptr(out));
    kern::launch_pool(pp, static_cast<cudaStream_t>(s));
  };
}

Fn softmax(const View& in, const View& out, int axis) {
  kern::SoftmaxParams sp{};
  sp.len = in.shape[axis];
  sp.in_axis_st = in.st[axis];
  sp.out_axis_st = out.st[axis];
  sp.rows = 1;
  int k = 0;
  for (int d = 0; d < in.rank(); ++d) {
    if (d == axis) continue;
    sp.row_shape[k] = in.shape[d];
    sp.in_row_st[k] = in.st[d];
    sp.out_row_st[k] = out.st[d];
    sp.rows *= in.shape[d];
    ++k;
  }
  sp.rank = k;
  return [sp, in, out](Runtime& rt, void* s) mutable {
    sp.in = reinterpret_cast<const float*>(rt.ptr(in));
    sp.out = reinterpret_cast<float*>(rt.ptr(out));
    kern::launch_softmax(sp, static_cast<cudaStream_t>(s));
  };
}

Fn gather(const View& data, const View& idx, const View& out, int64_t pre, int64_t axis_len, int64_t nidx,
          int64_t post) {
  kern::GatherParams gp{};
  gp.idx_dt = (int8_t)idx.dt;
  gp.elem_bytes = (int)dtype_size(data.dt);
  gp.pre = pre;
  gp.axis_len = axis_len;
  gp.nidx = nidx;
  gp.post = post;
  return [gp, data, idx, out](Runtime& rt, void* s) mutable {
    gp.data = rt.ptr(data);
    gp.idx = rt.ptr(idx);
    gp.out = rt.ptr(out);
    gp.status = rt.status();
    kern::launch_gather(gp, static_cast<cudaStream_t>(s));
  };
}

Fn gather_elements(const View& data, const View& idx, const View& out, int axis) {
  kern::GatherElementsParams gp{};
  gp.idx_dt = (int8_t)idx.dt;
  gp.elem_bytes = (int)dtype_size(data.dt);
  gp.rank = idx.rank();
  gp.axis = axis;
  gp.numel = idx.numel();
  for (int d = 0; d < idx.rank(); ++d) {
    gp.shape[d] = idx.shape[d];
    gp.data_st[d] = data.st[d];
  }
  gp.data_axis_len = data.shape[axis];
  return [gp, data, idx, out](Runtime& rt, void* s) mutable {
    gp.data = rt.ptr(data);
    gp.idx = rt.ptr(idx);
    gp.out = rt.ptr(out);
    gp.status = rt.status();
    kern::launch_gather_elements(gp, static_cast<cudaStream_t>(s));
  };
}

Fn range(kern::RangeParams rp, const View& out) {
  return [rp, out](Runtime& rt, void* s) mutable {
    rp.out = rt.ptr(out);
    kern::launch_range(rp, static_cast<cudaStream_t>(s));
  };
}

Fn topk(const View& in, const View& vals, const View& idxs, const View& used, int64_t k) {
  kern::TopKParams tp{};
  tp.rows = in.shape[0];
  tp.len = in.shape[1];
  tp.k = k;
  return [tp, in, vals, idxs, used](Runtime& rt, void* s) mutable {
    tp.in = reinterpret_cast<const float*>(rt.ptr(in));
    tp.vals = reinterpret_cast<float*>(rt.ptr(vals));
    tp.idxs = reinterpret_cast<int64_t*>(rt.ptr(idxs));
    tp.used = reinterpret_cast<unsigned char*>(rt.ptr(used));
    kern::launch_topk(tp, static_cast<cudaStream_t>(s));
  };
}

Fn pack(const PackSpec& ps, int64_t ldk, int hi, int lo) {
  kern::PackBParams pp{};
  pp.batch = ps.batch;
  pp.K = ps.K;
  pp.N = ps.N;
  pp.ldk = ldk;
  pp.sn = ps.sn;
  pp.k_rank = (int)ps.k_shape.size();
  for (int d = 0; d < pp.k_rank; ++d) {
    pp.k_shape[d] = ps.k_shape[d];
    pp.k_st[d] = ps.k_st[d];
    pp.k_valid[d] = ps.k_valid[d];
  }
  pp.batch_rank = (int)ps.batch_shape.size();
  for (int d = 0; d < pp.batch_rank; ++d) {
    pp.batch_shape[d] = ps.batch_shape[d];
    pp.batch_st[d] = ps.batch_st[d];
  }
  View src = ps.src;
  const int64_t off = ps.row_off * ldk;
  return [pp, src, hi, lo, off](Runtime& rt, void* s) mutable {
    pp.src = reinterpret_cast<const float*>(rt.ptr(src));
    pp.hi = static_cast<float*>(rt.plan->bufs[hi].ptr) + off;
    pp.lo = static_cast<float*>(rt.plan->bufs[lo].ptr) + off;
    kern::launch_pack_b(pp, static_cast<cudaStream_t>(s));
  };
}

}  // namespace launch
}  // namespace gawee

// ===========================================================================
// C ABI
// ===========================================================================
struct gawee_ctx {
  gawee::Runtime rt;
  std::string err;
};

namespace {

template <class F>
gawee_status guard(gawee_ctx* ctx, F&& f) {
  try {
    if (ctx) cudaSetDevice(ctx->rt.device);
    f();
    return GAWEE_OK;
  } catch (const gawee::StatusError& e) {
    if (ctx) ctx->err = e.what();
    return e.code;
  } catch (const gawee::ParseError& e) {
    if (ctx) ctx->err = e.what();
    return GAWEE_ERR_PARSE;
  } catch (const gawee::CudaError& e) {
    if (ctx) ctx->err = e.what();
    return GAWEE_ERR_CUDA;
  } catch (const std::exception& e) {
    if (ctx) ctx->err = e.what();
    std::string m = e.what();
    return m.rfind("unsupported", 0) == 0 || m.find(": unsupported") != std::string::npos ? GAWEE_ERR_UNSUPPORTED
                                                                                          : GAWEE_ERR_INVALID;
  } catch (...) {
    if (ctx) ctx->err = "unknown error";
    return GAWEE_ERR_INVALID;
  }
}

const char* device_status_name(int st) {
  static const char* names[] = {"ok", "gather index out of range", "tensor-core barrier wait timed out",
                                "invalid scalar program", "integer division by zero", "slice out of bounds"};
  return st >= 0 && st < 6 ? names[st] : "error";
}

// Reads and clears a device status word (after the work that writes it has
// completed); a non-zero code becomes GAWEE_ERR_DEVICE with its meaning.
void check_device_status(int* d_status) {
  int st = 0;
  GCHECK(cudaMemcpy(&st, d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (st) {
    GCHECK(cudaMemset(d_status, 0, sizeof(int)));
    throw gawee::StatusError(GAWEE_ERR_DEVICE, std::string("device reported: ") + device_status_name(st));
  }
}

cudaStream_t stream_of(gawee_ctx* ctx, void* s) {
  return s ? static_cast<cudaStream_t>(s) : ctx->rt.own_stream;
}

thread_local std::string g_create_error;

gawee_status create_impl(const std::string& text, const char* entry, int device, gawee_ctx** out) {
  if (!out) return GAWEE_ERR_INVALID;
  *out = nullptr;
  auto* ctx = new gawee_ctx();
  ctx->rt.device = device;
  gawee_status st = guard(ctx, [&] {
    int n = 0;
    GCHECK(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) throw gawee::StatusError(GAWEE_ERR_INVALID, "invalid device index");
    GCHECK(cudaSetDevice(device));
    gawee::Graph g = gawee::parse_mlir(text, entry ? entry : "forward");
    ctx->rt.plan = gawee::build_plan(std::move(g));
    GCHECK(cudaStreamCreateWithFlags(&ctx->rt.own_stream, cudaStreamNonBlocking));
    ctx->rt.allocate();
    ctx->rt.build_tensor_maps();
  });
  if (st != GAWEE_OK) {
    g_create_error = ctx->err;
    delete ctx;
    return st;
  }
  *out = ctx;
  return GAWEE_OK;
}

int value_info(const gawee::Value& v, int* dtype, int* rank, int64_t* shape) {
  if (dtype) *dtype = (int)v.type.dtype;
  if (rank) *rank = v.type.rank();
  if (shape)
    for (int d = 0; d < v.type.rank(); ++d) shape[d] = v.type.shape[d];
  return GAWEE_OK;
}

}  // namespace

namespace gawee {
// Error text for calls without a context (creation, context-free entry points).
void set_thread_error(const std::string& msg) { g_create_error = msg; }
}  // namespace gawee

extern "C" {

gawee_status gawee_create(const char* mlir_text, const char* entry, int device, gawee_ctx** out) {
  if (!mlir_text) return GAWEE_ERR_INVALID;
  return create_impl(mlir_text, entry, device, out);
}

gawee_status gawee_create_from_file(const char* path, const char* entry, int device, gawee_ctx** out) {
  if (!path) return GAWEE_ERR_INVALID;
  std::string text;
  try {
    text = gawee::read_text_file(path);
  } catch (const std::exception& e) {
    g_create_error = e.what();
    return GAWEE_ERR_INVALID;
  }
  return create_impl(text, entry, device, out);
}

void gawee_destroy(gawee_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->rt.device);
  if (ctx->rt.own_stream) cudaStreamSynchronize(ctx->rt.own_stream);
  delete ctx;
}

gawee_status gawee_last_error(const gawee_ctx* ctx, char* buf, size_t n) {
  if (!buf || n == 0) return GAWEE_ERR_INVALID;
  const std::string& m = ctx ? ctx->err : g_create_error;
  std::strncpy(buf, m.c_str(), n - 1);
  buf[n - 1] = 0;
  return GAWEE_OK;
}

int gawee_num_args(const gawee_ctx* ctx) { return ctx ? (int)ctx->rt.plan->g.args.size() : -1; }
int gawee_num_outputs(const gawee_ctx* ctx) { return ctx ? (int)ctx->rt.plan->g.results.size() : -1; }

gawee_status gawee_arg_info(const gawee_ctx* ctx, int i, int* dtype, int* rank, int64_t* shape) {
  if (!ctx || i < 0 || i >= gawee_num_args(ctx)) return GAWEE_ERR_INVALID;
  const auto& g = ctx->rt.plan->g;
  return value_info(g.values[g.args[i]], dtype, rank, shape);
}

gawee_status gawee_output_info(const gawee_ctx* ctx, int i, int* dtype, int* rank, int64_t* shape) {
  if (!ctx || i < 0 || i >= gawee_num_outputs(ctx)) return GAWEE_ERR_INVALID;
  const auto& g = ctx->rt.plan->g;
  return value_info(g.values[g.results[i]], dtype, rank, shape);
}

static gawee_status set_arg_impl(gawee_ctx* ctx, int i, const void* src, size_t bytes, void* stream,
                                 cudaMemcpyKind kind) {
  if (!ctx) return GAWEE_ERR_INVALID;
  return guard(ctx, [&] {
    auto& rt = ctx->rt;
    if (i < 0 || i >= (int)rt.plan->arg_buf.size()) throw gawee::StatusError(GAWEE_ERR_INVALID, "argument index out of range");
    const gawee::Buf& b = rt.plan->bufs[rt.plan->arg_buf[i]];
    if (bytes != b.bytes() || !src)
      throw gawee::StatusError(GAWEE_ERR_INVALID, "argument " + std::to_string(i) + " expects " +
                                                      std::to_string(b.bytes()) + " bytes, got " + std::to_string(bytes));
    if (!b.ptr) return;  // argument never read by the graph
    GCHECK(cudaMemcpyAsync(b.ptr, src, bytes, kind, stream_of(ctx, stream)));
    rt.dirty[i] = 1;
  });
}

gawee_status gawee_set_arg(gawee_ctx* ctx, int i, const void* host, size_t bytes, void* stream) {
  return set_arg_impl(ctx, i, host, bytes, stream, cudaMemcpyHostToDevice);
}

gawee_status gawee_set_arg_device(gawee_ctx* ctx, int i, const void* dev, size_t bytes, void* stream) {
  return set_arg_impl(ctx, i, dev, bytes, stream, cudaMemcpyDeviceToDevice);
}

gawee_status gawee_forward(gawee_ctx* ctx, void* stream) {
  if (!ctx) return GAWEE_ERR_INVALID;
  return guard(ctx, [&] { ctx->rt.forward(stream_of(ctx, stream)); });
}

gawee_status gawee_get_output(gawee_ctx* ctx, int i, void* host, size_t bytes, void* stream) {
  if (!ctx) return GAWEE_ERR_INVALID;
  return guard(ctx, [&] {
    auto& rt = ctx->rt;
    if (i < 0 || i >= (int)rt.plan->result_view.size()) throw gawee::StatusError(GAWEE_ERR_INVALID, "output index out of range");
    const gawee::View& v = rt.plan->result_view[i];
    size_t nb = (size_t)v.numel() * gawee::dtype_size(v.dt);
    if (bytes != nb || !host)
      throw gawee::StatusError(GAWEE_ERR_INVALID, "output " + std::to_string(i) + " has " + std::to_string(nb) + " bytes");
    GCHECK(cudaMemcpyAsync(host, rt.ptr(v), nb, cudaMemcpyDeviceToHost, stream_of(ctx, stream)));
  });
}

gawee_status gawee_output_device_ptr(gawee_ctx* ctx, int i, void** ptr) {
  if (!ctx || !ptr) return GAWEE_ERR_INVALID;
  return guard(ctx, [&] {
    auto& rt = ctx->rt;
    if (i < 0 || i >= (int)rt.plan->result_view.size()) throw gawee::StatusError(GAWEE_ERR_INVALID, "output index out of range");
    *ptr = rt.ptr(rt.plan->result_view[i]);
  });
}

gawee_status gawee_synchronize(gawee_ctx* ctx, void* stream) {
  if (!ctx) {
    // the allocation-free entry point's status word on the current device
    const int st = gawee::noalloc_take_status(static_cast<cudaStream_t>(stream));
    if (st < 0) return GAWEE_ERR_CUDA;
    if (st > 0) {
      g_create_error = std::string("device reported: ") + device_status_name(st);
      return GAWEE_ERR_DEVICE;
    }
    return GAWEE_OK;
  }
  return guard(ctx, [&] {
    GCHECK(cudaStreamSynchronize(stream_of(ctx, stream)));
    check_device_status(ctx->rt.d_status);
  });
}

gawee_status gawee_set_graph_mode(gawee_ctx* ctx, int enabled) {
  if (!ctx) return GAWEE_ERR_INVALID;
  ctx->rt.graph_mode = enabled != 0;
  return GAWEE_OK;
}

gawee_status gawee_set_precision(gawee_ctx* ctx, int mode) {
  if (!ctx || (mode != GAWEE_PRECISION_FP32 && mode != GAWEE_PRECISION_TF32 && mode != GAWEE_PRECISION_BF16))
    return GAWEE_ERR_INVALID;
  const int passes = mode == GAWEE_PRECISION_FP32 ? 3 : 1;
  const bool bf16 = mode == GAWEE_PRECISION_BF16;
  if (passes == ctx->rt.passes && bf16 == ctx->rt.bf16) return GAWEE_OK;
  cudaSetDevice(ctx->rt.device);
  if (bf16) {
    const gawee_status st = guard(ctx, [&] { ctx->rt.enable_bf16(); });
    if (st != GAWEE_OK) return st;
  }
  ctx->rt.bf16 = bf16;
  // the captured graph holds the old kernel parameters: capture again
  if (ctx->rt.gexec) cudaGraphExecDestroy(ctx->rt.gexec);
  if (ctx->rt.graph) cudaGraphDestroy(ctx->rt.graph);
  ctx->rt.gexec = nullptr;
  ctx->rt.graph = nullptr;
  ctx->rt.passes = passes;
  return GAWEE_OK;
}

int gawee_precision(const gawee_ctx* ctx) {
  if (!ctx) return -1;
  if (ctx->rt.bf16) return GAWEE_PRECISION_BF16;
  return ctx->rt.passes == 1 ? GAWEE_PRECISION_TF32 : GAWEE_PRECISION_FP32;
}

int gawee_num_kernels(const gawee_ctx* ctx) { return ctx ? (int)ctx->rt.plan->main.size() : -1; }

int gawee_num_launches(const gawee_ctx* ctx) {
  if (!ctx) return -1;
  int n = 0;
  for (int o : ctx->rt.plan->main) {
    const auto& op = ctx->rt.plan->ops[o];
    n += 1 + (o < (int)ctx->rt.ksplit.size() && ctx->rt.ksplit[o] > 1 ? 1 : 0);
    // the skip-flag pass, unless the mask is fixed and its flags are filled
    if (op.kind == gawee::OpKind::ATTN && op.attn.has_mask &&
        !(o < (int)ctx->rt.attn_skip_static.size() && ctx->rt.attn_skip_static[o] == 2))
      ++n;
  }
  return n;
}

gawee_status gawee_plan_summary(const gawee_ctx* ctx, char* buf, size_t n) {
  if (!ctx || !buf || n == 0) return GAWEE_ERR_INVALID;
  std::string s = ctx->rt.plan->summary();
  std::strncpy(buf, s.c_str(), n - 1);
  buf[n - 1] = 0;
  return GAWEE_OK;
}

gawee_status gawee_op_info(const gawee_ctx* ctx, int i, char* name, size_t n, int* is_tc, double* flops) {
  if (!ctx || i < 0 || i >= (int)ctx->rt.plan->main.size()) return GAWEE_ERR_INVALID;
  const int o = ctx->rt.plan->main[i];
  const gawee::Op& op = ctx->rt.plan->ops[o];
  if (name && n) {
    std::string nm = op.name;
    if (op.kind == gawee::OpKind::TC && o < (int)ctx->rt.a_tma.size() && ctx->rt.a_tma[o] != gawee::kern::A_TMA_NONE)
      nm += ctx->rt.a_tma[o] == gawee::kern::A_TMA_IM2COL        ? " [tma im2col]"
            : ctx->rt.a_tma[o] == gawee::kern::A_TMA_IM2COL_TAPS ? " [tma im2col taps]"
                                                                  : " [tma]";
    if (op.kind == gawee::OpKind::TC && o < (int)ctx->rt.ksplit.size() && ctx->rt.ksplit[o] > 1)
      nm += " [split-k " + std::to_string(ctx->rt.ksplit[o]) + "]";
    if (op.kind == gawee::OpKind::TC && o < (int)ctx->rt.aux_tma.size() && ctx->rt.aux_tma[o])
      nm += " [aux smem]";
    if (ctx->rt.bf16 && o < (int)ctx->rt.bf16_plane.size() && ctx->rt.bf16_plane[o]) nm += " [bf16]";
    std::strncpy(name, nm.c_str(), n - 1);
    name[n - 1] = 0;
  }
  if (is_tc) *is_tc = op.kind == gawee::OpKind::TC || op.kind == gawee::OpKind::ATTN;
  if (flops) *flops = op.kind == gawee::OpKind::TC ? op.tc.flops : op.kind == gawee::OpKind::ATTN ? op.attn.flops : 0.0;
  return GAWEE_OK;
}

gawee_status gawee_profile_forward(gawee_ctx* ctx, void* stream, float* ms, int n) {
  if (!ctx || !ms || n < (int)ctx->rt.plan->main.size()) return GAWEE_ERR_INVALID;
  return guard(ctx, [&] {
    auto& rt = ctx->rt;
    cudaStream_t s = stream_of(ctx, stream);
    rt.forward(s);  // prologue / packing as needed, then one regular forward
    const auto& main = rt.plan->main;
    std::vector<cudaEvent_t> ev(main.size() + 1);
    for (auto& e : ev) GCHECK(cudaEventCreate(&e));
    GCHECK(cudaEventRecord(ev[0], s));
    for (size_t k = 0; k < main.size(); ++k) {
      rt.run_op(main[k], s);
      GCHECK(cudaGetLastError());
      GCHECK(cudaEventRecord(ev[k + 1], s));
    }
    GCHECK(cudaStreamSynchronize(s));
    for (size_t k = 0; k < main.size(); ++k) GCHECK(cudaEventElapsedTime(&ms[k], ev[k], ev[k + 1]));
    for (auto& e : ev) cudaEventDestroy(e);
  });
}

gawee_status gawee_plan_text(const char* mlir_text, const char* entry, char* buf, size_t n) {
  if (!mlir_text || !buf || n == 0) return GAWEE_ERR_INVALID;
  gawee_status st = GAWEE_OK;
  std::string out;
  try {
    auto plan = gawee::build_plan(gawee::parse_mlir(mlir_text, entry ? entry : "forward"));
    out = plan->summary();
  } catch (const gawee::ParseError& e) {
    out = e.what();
    st = GAWEE_ERR_PARSE;
  } catch (const std::exception& e) {
    out = e.what();
    std::string m = out;
    st = m.find("unsupported") != std::string::npos ? GAWEE_ERR_UNSUPPORTED : GAWEE_ERR_INVALID;
  }
  std::strncpy(buf, out.c_str(), n - 1);
  buf[n - 1] = 0;
  g_create_error = st == GAWEE_OK ? "" : out;
  return st;
}

gawee_status gawee_ciface_forward(gawee_ctx* ctx, void* result_desc, void* const* arg_descs, int nargs) {
  if (!ctx) return GAWEE_ERR_INVALID;
  return guard(ctx, [&] {
    auto& rt = ctx->rt;
    const auto& g = rt.plan->g;
    if (nargs != (int)g.args.size()) throw gawee::StatusError(GAWEE_ERR_INVALID, "wrong number of memref arguments");
    if (g.results.size() != 1) throw gawee::StatusError(GAWEE_ERR_UNSUPPORTED, "the ciface entry supports one result");
    cudaStream_t s = rt.own_stream;
    for (int a = 0; a < nargs; ++a) {
      const auto& t = g.values[g.args[a]].type;
      const char* d = static_cast<const char*>(arg_descs[a]);
      const char* aligned;
      int64_t offset;
      std::memcpy(&aligned, d + sizeof(void*), sizeof(void*));
      std::memcpy(&offset, d + 2 * sizeof(void*), 8);
      const int64_t* sizes = reinterpret_cast<const int64_t*>(d + 2 * sizeof(void*) + 8);
      const int64_t* strides = sizes + t.rank();
      int64_t expect = 1;
      for (int k = t.rank() - 1; k >= 0; --k) {
        if (sizes[k] != t.shape[k]) throw gawee::StatusError(GAWEE_ERR_INVALID, "memref size mismatch on arg " + std::to_string(a));
        if (t.shape[k] != 1 && strides[k] != expect)
          throw gawee::StatusError(GAWEE_ERR_INVALID, "memref arg " + std::to_string(a) + " is not dense row-major");
        expect *= t.shape[k];
      }
      const gawee::Buf& b = rt.plan->bufs[rt.plan->arg_buf[a]];
      if (b.ptr)
        GCHECK(cudaMemcpyAsync(b.ptr, aligned + offset * (int64_t)gawee::dtype_size(t.dtype), b.bytes(),
                               cudaMemcpyHostToDevice, s));
      rt.dirty[a] = 1;
    }
    rt.forward(s);
    const gawee::View& v = rt.plan->result_view[0];
    size_t nb = (size_t)v.numel() * gawee::dtype_size(v.dt);
    void* host = std::malloc(nb ? nb : 1);  // owned by the caller, as in the reference ABI
    if (!host) throw gawee::StatusError(GAWEE_ERR_OOM, "malloc of the result failed");
    GCHECK(cudaMemcpyAsync(host, rt.ptr(v), nb, cudaMemcpyDeviceToHost, s));
    try {
      GCHECK(cudaStreamSynchronize(s));
      check_device_status(rt.d_status);
    } catch (...) {
      std::free(host);
      throw;
    }
    char* r = static_cast<char*>(result_desc);
    const auto& rtype = g.values[g.results[0]].type;
    int64_t zero = 0;
    std::memcpy(r, &host, sizeof(void*));
    std::memcpy(r + sizeof(void*), &host, sizeof(void*));
    std::memcpy(r + 2 * sizeof(void*), &zero, 8);
    int64_t* sizes = reinterpret_cast<int64_t*>(r + 2 * sizeof(void*) + 8);
    int64_t* strides = sizes + rtype.rank();
    int64_t acc = 1;
    for (int k = rtype.rank() - 1; k >= 0; --k) {
      sizes[k] = rtype.shape[k];
      strides[k] = acc;
      acc *= rtype.shape[k];
    }
  });
}

gawee_status gawee_embedded_forward(const char* mlir_text, int device, void* result_desc, void* const* arg_descs,
                                    int nargs) {
  struct Cache {
    std::mutex mu;
    std::vector<std::pair<std::pair<const char*, int>, gawee_ctx*>> ctxs;
  };
  static Cache* cache = new Cache();  // contexts live until process exit
  if (!mlir_text) return GAWEE_ERR_INVALID;
  gawee_ctx* ctx = nullptr;
  {
    std::lock_guard<std::mutex> lock(cache->mu);
    for (auto& e : cache->ctxs)
      if (e.first.first == mlir_text && e.first.second == device) ctx = e.second;
    if (!ctx) {
      gawee_status st = gawee_create(mlir_text, "forward", device, &ctx);
      if (st) return st;
      cache->ctxs.push_back({{mlir_text, device}, ctx});
    }
  }
  gawee_status st = gawee_ciface_forward(ctx, result_desc, arg_descs, nargs);
  // the caller holds no context: its message goes where gawee_last_error(NULL, ...) reads
  if (st != GAWEE_OK) g_create_error = ctx->err;
  return st;
}

gawee_status gawee_dp_unique_id(void* id) {
  if (!id) return GAWEE_ERR_INVALID;
  if (!gawee::nccl().ok) return GAWEE_ERR_NCCL;
  ncclUniqueId u;
  if (gawee::nccl().getUniqueId(&u) != ncclSuccess) return GAWEE_ERR_NCCL;
  static_assert(sizeof(ncclUniqueId) == GAWEE_NCCL_ID_BYTES, "nccl id size");
  std::memcpy(id, &u, sizeof(u));
  return GAWEE_OK;
}

gawee_status gawee_dp_init(gawee_ctx* ctx, int world, int rank, const void* id) {
  if (!ctx || !id || world < 1 || rank < 0 || rank >= world) return GAWEE_ERR_INVALID;
  return guard(ctx, [&] {
    if (!gawee::nccl().ok) throw gawee::StatusError(GAWEE_ERR_NCCL, "libnccl.so.2 could not be loaded");
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    auto& rt = ctx->rt;
    gawee::nccl_check(gawee::nccl().commInitRank(&rt.comm, world, u, rank), "ncclCommInitRank");
    rt.world = world;
    rt.rank = rank;
    // every rank learns every rank's output sizes (one all-gather of a few
    // int64s, once): the gather then moves each peer's own byte count
    const size_t nout = rt.plan->result_view.size();
    std::vector<int64_t> mine(nout);
    for (size_t i = 0; i < nout; ++i) {
      const gawee::View& v = rt.plan->result_view[i];
      mine[i] = v.numel() * (int64_t)gawee::dtype_size(v.dt);
    }
    rt.peer_bytes.assign((size_t)world * nout, 0);
    if (nout) {
      int64_t* d = nullptr;
      GCHECK(cudaMalloc(&d, sizeof(int64_t) * nout * (world + 1)));
      try {
        GCHECK(cudaMemcpyAsync(d, mine.data(), sizeof(int64_t) * nout, cudaMemcpyHostToDevice, rt.own_stream));
        gawee::nccl_check(gawee::nccl().allGather(d, d + nout, nout * sizeof(int64_t), ncclInt8, rt.comm,
                                                  rt.own_stream), "ncclAllGather");
        GCHECK(cudaMemcpyAsync(rt.peer_bytes.data(), d + nout, sizeof(int64_t) * nout * world,
                               cudaMemcpyDeviceToHost, rt.own_stream));
        GCHECK(cudaStreamSynchronize(rt.own_stream));
      } catch (...) {
        cudaFree(d);
        throw;
      }
      GCHECK(cudaFree(d));
    }
    for (int r = 0; r < world; ++r)
      for (size_t i = 0; i < nout; ++i) {
        const int64_t b = rt.peer_bytes[(size_t)r * nout + i];
        // every rank plans the same graph up to its batch size: a rank whose
        // row size differs from rank 0's cannot be gathered row-wise
        const int64_t rows0 = rt.plan->result_view[i].shape.empty() ? 1 : rt.plan->result_view[i].shape[0];
        const int64_t row_bytes = rows0 ? mine[i] / rows0 : 0;
        if (b < 0 || (row_bytes && b % row_bytes != 0))
          throw gawee::StatusError(GAWEE_ERR_INVALID, "rank " + std::to_string(r) + " output " + std::to_string(i) +
                                                          " is not a whole number of this rank's rows");
      }
  });
}

gawee_status gawee_dp_output_bytes(gawee_ctx* ctx, int i, size_t* total) {
  if (!ctx || !total) return GAWEE_ERR_INVALID;
  return guard(ctx, [&] {
    auto& rt = ctx->rt;
    if (!rt.comm) throw gawee::StatusError(GAWEE_ERR_INVALID, "gawee_dp_init was not called");
    const size_t nout = rt.plan->result_view.size();
    if (i < 0 || i >= (int)nout) throw gawee::StatusError(GAWEE_ERR_INVALID, "output index out of range");
    size_t t = 0;
    for (int r = 0; r < rt.world; ++r) t += (size_t)rt.peer_bytes[(size_t)r * nout + i];
    *total = t;
  });
}

gawee_status gawee_dp_gather_output(gawee_ctx* ctx, int i, void* dst, void* stream) {
  if (!ctx) return GAWEE_ERR_INVALID;
  return guard(ctx, [&] {
    auto& rt = ctx->rt;
    if (!rt.comm) throw gawee::StatusError(GAWEE_ERR_INVALID, "gawee_dp_init was not called");
    if (i < 0 || i >= (int)rt.plan->result_view.size()) throw gawee::StatusError(GAWEE_ERR_INVALID, "output index out of range");
    const gawee::View& v = rt.plan->result_view[i];
    size_t nb = (size_t)v.numel() * gawee::dtype_size(v.dt);
    const size_t nout = rt.plan->result_view.size();
    if ((int64_t)nb != rt.peer_bytes[(size_t)rt.rank * nout + i])
      throw gawee::StatusError(GAWEE_ERR_INVALID, "output size changed since gawee_dp_init");
    cudaStream_t s = stream_of(ctx, stream);
    auto& api = gawee::nccl();
    if (rt.rank == 0) {
      if (!dst) throw gawee::StatusError(GAWEE_ERR_INVALID, "rank 0 needs a destination buffer");
      GCHECK(cudaMemcpyAsync(dst, rt.ptr(v), nb, cudaMemcpyDeviceToDevice, s));
      size_t off = nb;
      gawee::nccl_check(api.groupStart(), "ncclGroupStart");
      for (int r = 1; r < rt.world; ++r) {
        const size_t rb = (size_t)rt.peer_bytes[(size_t)r * nout + i];
        if (rb)
          gawee::nccl_check(api.recv(static_cast<char*>(dst) + off, rb, ncclInt8, r, rt.comm, s), "ncclRecv");
        off += rb;
      }
      gawee::nccl_check(api.groupEnd(), "ncclGroupEnd");
    } else if (nb) {
      gawee::nccl_check(api.send(rt.ptr(v), nb, ncclInt8, 0, rt.comm, s), "ncclSend");
    }
  });
}

}  // extern "C"
