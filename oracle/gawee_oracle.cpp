// CPU oracle for gawee-dialect graphs — TEST INFRASTRUCTURE ONLY.
//
// This is a restatement, in plain C++, of what the reference's CPU pipeline
// computes for every op: the executable semantics are the conversion patterns
// of middle/mlir/lib/Conversion/GaweeToLinalg.cpp (cited per op below), plus
// the emitter's direct linalg forms (middle/mlir/lib/Emit/ONNXMLIREmitter.cpp).
// It exists to check the CUDA backend; nothing in the product links it.
//
// Numerical conventions follow the reference's lowered code:
//   * fp32 arithmetic with separate multiply and add (no FMA contraction:
//     built with -ffp-contract=off), accumulators zero-initialised and
//     reduced in the sequential loop order of the linalg op
//     (conv: c, kh, kw; matmul/linear: k; reductions: row-major input order);
//   * math functions are libm calls (MathToLibm in middle/mlir/tools/gawee-opt.cpp:174):
//     expf, erff, tanhf, sinf, cosf, powf, sqrtf;
//   * arith.maximumf / minimumf propagate NaN and order -0 < +0.
//
// Parity is unpinned against the reference binary itself: the reference needs
// an MLIR/LLVM 22 toolchain that is not available, and the reference repository
// ships no golden vectors.  The oracle is pinned instead by hand-computed
// known-answer tests and by independent torch-CPU models in tests/.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include <thread>

#include "../gawee_b200/csrc/host/ir.h"

namespace oracle {

// Work is split over host threads by output element only, so every output's
// accumulation order is the sequential order above whatever the thread count.
static int g_threads = 1;

template <class F>
static void parallel_for(int64_t n, F&& f) {
  int t = (int)std::min<int64_t>(g_threads, n);
  if (t <= 1) {
    for (int64_t i = 0; i < n; ++i) f(i);
    return;
  }
  std::vector<std::thread> pool;
  int64_t chunk = (n + t - 1) / t;
  for (int k = 0; k < t; ++k) {
    int64_t b = k * chunk, e = std::min(n, b + chunk);
    if (b >= e) break;
    pool.emplace_back([b, e, &f] { for (int64_t i = b; i < e; ++i) f(i); });
  }
  for (auto& th : pool) th.join();
}

using gawee::Attr;
using gawee::DType;
using gawee::EInstr;
using gawee::EOp;
using gawee::EProgram;
using gawee::Graph;
using gawee::Node;

struct Tensor {
  DType dt = DType::F32;
  std::vector<int64_t> shape;
  std::vector<uint8_t> buf;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
  void alloc(DType t, const std::vector<int64_t>& s) {
    dt = t;
    shape = s;
    buf.assign((size_t)numel() * gawee::dtype_size(t), 0);
  }
  template <class T> T* p() { return reinterpret_cast<T*>(buf.data()); }
  template <class T> const T* p() const { return reinterpret_cast<const T*>(buf.data()); }
};

static std::vector<int64_t> strides_of(const std::vector<int64_t>& s) {
  std::vector<int64_t> st(s.size(), 1);
  for (int i = (int)s.size() - 2; i >= 0; --i) st[i] = st[i + 1] * s[i + 1];
  return st;
}

// ---------------------------------------------------------------------------
// Scalar element model: one 64-bit slot per element, interpreted by dtype.
// ---------------------------------------------------------------------------
union Sc {
  float f;
  double d;
  int64_t i;
};

static Sc load(const Tensor& t, int64_t k) {
  Sc s;
  s.i = 0;
  switch (t.dt) {
    case DType::F32: s.f = t.p<float>()[k]; break;
    case DType::F64: s.d = t.p<double>()[k]; break;
    case DType::I64: case DType::INDEX: s.i = t.p<int64_t>()[k]; break;
    case DType::I32: s.i = t.p<int32_t>()[k]; break;
    case DType::I1: s.i = t.p<uint8_t>()[k] ? 1 : 0; break;
    default: throw std::runtime_error("oracle: unsupported dtype");
  }
  return s;
}

static void store(Tensor& t, int64_t k, Sc s) {
  switch (t.dt) {
    case DType::F32: t.p<float>()[k] = s.f; break;
    case DType::F64: t.p<double>()[k] = s.d; break;
    case DType::I64: case DType::INDEX: t.p<int64_t>()[k] = s.i; break;
    case DType::I32: t.p<int32_t>()[k] = (int32_t)s.i; break;
    case DType::I1: t.p<uint8_t>()[k] = (s.i & 1) ? 1 : 0; break;
    default: throw std::runtime_error("oracle: unsupported dtype");
  }
}

// arith.maximumf / arith.minimumf: NaN-propagating, -0 < +0.
static float maximumf(float a, float b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<float>::quiet_NaN();
  if (a == b) return std::signbit(a) ? b : a;
  return a > b ? a : b;
}
static float minimumf(float a, float b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<float>::quiet_NaN();
  if (a == b) return std::signbit(a) ? a : b;
  return a < b ? a : b;
}
static double maximumd(double a, double b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<double>::quiet_NaN();
  if (a == b) return std::signbit(a) ? b : a;
  return a > b ? a : b;
}
static double minimumd(double a, double b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<double>::quiet_NaN();
  if (a == b) return std::signbit(a) ? a : b;
  return a < b ? a : b;
}

static int64_t wrap_int(int64_t v, DType t) {
  if (t == DType::I32) return (int64_t)(int32_t)(uint32_t)(uint64_t)v;
  if (t == DType::I1) return v & 1;
  return v;
}

static bool cmpf(int pred, double a, double b) {
  bool uno = std::isnan(a) || std::isnan(b);
  switch (pred) {
    case gawee::CF_FALSE: return false;
    case gawee::CF_OEQ: return !uno && a == b;
    case gawee::CF_OGT: return !uno && a > b;
    case gawee::CF_OGE: return !uno && a >= b;
    case gawee::CF_OLT: return !uno && a < b;
    case gawee::CF_OLE: return !uno && a <= b;
    case gawee::CF_ONE: return !uno && a != b;
    case gawee::CF_ORD: return !uno;
    case gawee::CF_UEQ: return uno || a == b;
    case gawee::CF_UGT: return uno || a > b;
    case gawee::CF_UGE: return uno || a >= b;
    case gawee::CF_ULT: return uno || a < b;
    case gawee::CF_ULE: return uno || a <= b;
    case gawee::CF_UNE: return uno || a != b;
    case gawee::CF_UNO: return uno;
    default: return true;
  }
}

static bool cmpi(int pred, int64_t a, int64_t b, DType t) {
  uint64_t ua = (uint64_t)a, ub = (uint64_t)b;
  if (t == DType::I32) { ua &= 0xffffffffu; ub &= 0xffffffffu; }
  if (t == DType::I1) { ua &= 1; ub &= 1; }
  switch (pred) {
    case gawee::CI_EQ: return a == b;
    case gawee::CI_NE: return a != b;
    case gawee::CI_SLT: return a < b;
    case gawee::CI_SLE: return a <= b;
    case gawee::CI_SGT: return a > b;
    case gawee::CI_SGE: return a >= b;
    case gawee::CI_ULT: return ua < ub;
    case gawee::CI_ULE: return ua <= ub;
    case gawee::CI_UGT: return ua > ub;
    default: return ua >= ub;
  }
}

// Interpret one scalar op program (linalg.generic / linalg.reduce bodies).
static Sc run_program(const EProgram& pg, std::vector<Sc>& r) {
  for (const EInstr& in : pg.code) {
    Sc a = in.a >= 0 ? r[in.a] : Sc{}, b = in.b >= 0 ? r[in.b] : Sc{}, c = in.c >= 0 ? r[in.c] : Sc{};
    Sc o;
    o.i = 0;
    bool f32 = in.ty == DType::F32, f64 = in.ty == DType::F64;
    auto F = [&](auto ff, auto fd) {
      if (f32) o.f = ff(a.f, b.f);
      else if (f64) o.d = fd(a.d, b.d);
      else throw std::runtime_error("oracle: float op on non-float type");
    };
    switch (in.op) {
      case EOp::CONST:
        if (in.rty == DType::F32) o.f = (float)in.fimm;
        else if (in.rty == DType::F64) o.d = in.fimm;
        else o.i = wrap_int(in.iimm, in.rty);
        break;
      case EOp::ADDF: F([](float x, float y) { return x + y; }, [](double x, double y) { return x + y; }); break;
      case EOp::SUBF: F([](float x, float y) { return x - y; }, [](double x, double y) { return x - y; }); break;
      case EOp::MULF: F([](float x, float y) { return x * y; }, [](double x, double y) { return x * y; }); break;
      case EOp::DIVF: F([](float x, float y) { return x / y; }, [](double x, double y) { return x / y; }); break;
      case EOp::REMF: F([](float x, float y) { return std::fmod(x, y); }, [](double x, double y) { return std::fmod(x, y); }); break;
      case EOp::MAXIMUMF: F(maximumf, maximumd); break;
      case EOp::MINIMUMF: F(minimumf, minimumd); break;
      case EOp::MAXNUMF: F([](float x, float y) { return std::fmax(x, y); }, [](double x, double y) { return std::fmax(x, y); }); break;
      case EOp::MINNUMF: F([](float x, float y) { return std::fmin(x, y); }, [](double x, double y) { return std::fmin(x, y); }); break;
      case EOp::POWF: F([](float x, float y) { return powf(x, y); }, [](double x, double y) { return std::pow(x, y); }); break;
#define UNF(OP, FF, FD) case EOp::OP: if (f32) o.f = FF(a.f); else o.d = FD(a.d); break;
      UNF(NEGF, -, -)
      UNF(SQRT, sqrtf, std::sqrt)
      UNF(EXP, expf, std::exp)
      UNF(LOG, logf, std::log)
      UNF(ERF, erff, std::erf)
      UNF(TANH, tanhf, std::tanh)
      UNF(SIN, sinf, std::sin)
      UNF(COS, cosf, std::cos)
      UNF(ABSF, fabsf, std::fabs)
      UNF(FLOOR, floorf, std::floor)
      UNF(CEIL, ceilf, std::ceil)
#undef UNF
      case EOp::RSQRT: if (f32) o.f = 1.0f / sqrtf(a.f); else o.d = 1.0 / std::sqrt(a.d); break;
      case EOp::ADDI: o.i = wrap_int((int64_t)((uint64_t)a.i + (uint64_t)b.i), in.ty); break;
      case EOp::SUBI: o.i = wrap_int((int64_t)((uint64_t)a.i - (uint64_t)b.i), in.ty); break;
      case EOp::MULI: o.i = wrap_int((int64_t)((uint64_t)a.i * (uint64_t)b.i), in.ty); break;
      case EOp::DIVSI:
        if (b.i == 0) throw std::runtime_error("oracle: integer division by zero");
        o.i = wrap_int(a.i / b.i, in.ty);
        break;
      case EOp::REMSI:
        if (b.i == 0) throw std::runtime_error("oracle: integer remainder by zero");
        o.i = wrap_int(a.i % b.i, in.ty);
        break;
      case EOp::MAXSI: o.i = std::max(a.i, b.i); break;
      case EOp::MINSI: o.i = std::min(a.i, b.i); break;
      case EOp::ANDI: o.i = a.i & b.i; break;
      case EOp::ORI: o.i = a.i | b.i; break;
      case EOp::XORI: o.i = wrap_int(a.i ^ b.i, in.ty); break;
      case EOp::CMPF: o.i = cmpf(in.pred, f32 ? (double)a.f : a.d, f32 ? (double)b.f : b.d); break;
      case EOp::CMPI: o.i = cmpi(in.pred, a.i, b.i, in.ty); break;
      case EOp::SELECT: o = (a.i & 1) ? b : c; break;
      case EOp::SITOFP:
        if (in.rty == DType::F32) o.f = (float)a.i; else o.d = (double)a.i;
        break;
      case EOp::UITOFP: {
        uint64_t u = (uint64_t)a.i;
        if (in.ty == DType::I32) u &= 0xffffffffu;
        if (in.ty == DType::I1) u &= 1;
        if (in.rty == DType::F32) o.f = (float)u; else o.d = (double)u;
        break;
      }
      case EOp::FPTOSI: o.i = wrap_int(f32 ? (int64_t)a.f : (int64_t)a.d, in.rty); break;
      case EOp::EXTF: o.d = (double)a.f; break;
      case EOp::TRUNCF: o.f = (float)a.d; break;
      case EOp::EXTSI: o.i = a.i; break;
      case EOp::EXTUI: o.i = in.ty == DType::I1 ? (a.i & 1) : (in.ty == DType::I32 ? (int64_t)(uint32_t)a.i : a.i); break;
      case EOp::TRUNCI: o.i = wrap_int(a.i, in.rty); break;
      case EOp::INDEX_CAST: o.i = wrap_int(a.i, in.rty); break;
      case EOp::COPY: o = a; break;
      default: throw std::runtime_error("oracle: unsupported body op");
    }
    r[in.dst] = o;
  }
  return r[pg.result];
}

// ---------------------------------------------------------------------------
// Broadcast indexing (buildBroadcastMap, GaweeToLinalg.cpp:123-144): input dim i
// aligned to output dim (outRank - inRank + i); a static size-1 input dim that
// meets a non-1 output dim reads index 0.
// ---------------------------------------------------------------------------
struct BIndex {
  std::vector<int64_t> st;  // stride of each OUTPUT dim into the input (0 = broadcast)
  BIndex(const std::vector<int64_t>& in, const std::vector<int64_t>& out) {
    st.assign(out.size(), 0);
    auto is = strides_of(in);
    int lead = (int)out.size() - (int)in.size();
    if (lead < 0) throw std::runtime_error("oracle: broadcast input has higher rank than output");
    for (size_t i = 0; i < in.size(); ++i) {
      int od = lead + (int)i;
      if (in[i] == 1 && out[od] != 1) st[od] = 0;
      else {
        if (in[i] != out[od]) throw std::runtime_error("oracle: incompatible broadcast");
        st[od] = is[i];
      }
    }
  }
};

static void for_each_index(const std::vector<int64_t>& shape, const std::function<void(int64_t, const int64_t*)>& fn) {
  int r = (int)shape.size();
  int64_t n = 1;
  for (auto d : shape) n *= d;
  std::vector<int64_t> idx(r, 0);
  for (int64_t k = 0; k < n; ++k) {
    fn(k, idx.data());
    for (int d = r - 1; d >= 0; --d) {
      if (++idx[d] < shape[d]) break;
      idx[d] = 0;
    }
  }
}

class Interp {
 public:
  explicit Interp(Graph g) : g_(std::move(g)) {}
  const Graph& graph() const { return g_; }

  void run(const std::vector<const void*>& args, const std::vector<void*>& outs) {
    vals_.assign(g_.values.size(), Tensor());
    for (size_t v = 0; v < g_.values.size(); ++v) {
      const auto& gv = g_.values[v];
      if (gv.is_const) {
        vals_[v].alloc(gv.type.dtype, gv.type.is_tensor ? gv.type.shape : std::vector<int64_t>{});
        std::memcpy(vals_[v].buf.data(), gv.data.data(), gv.data.size());
      }
    }
    if (args.size() != g_.args.size()) throw std::runtime_error("oracle: wrong number of arguments");
    for (size_t a = 0; a < g_.args.size(); ++a) {
      const auto& gv = g_.values[g_.args[a]];
      Tensor& t = vals_[g_.args[a]];
      t.alloc(gv.type.dtype, gv.type.shape);
      std::memcpy(t.buf.data(), args[a], t.buf.size());
    }
    for (size_t n = 0; n < g_.nodes.size(); ++n) {
      try {
        exec(g_.nodes[n]);
      } catch (std::exception& e) {
        throw std::runtime_error("node " + std::to_string(n) + " (" + g_.nodes[n].op + "): " + e.what());
      }
      // free dead intermediates to bound memory on large graphs
      release_after(n);
    }
    for (size_t r = 0; r < g_.results.size(); ++r) {
      const Tensor& t = vals_[g_.results[r]];
      std::memcpy(outs[r], t.buf.data(), t.buf.size());
    }
  }

  void prepare_liveness() {
    last_use_.assign(g_.values.size(), -1);
    for (size_t n = 0; n < g_.nodes.size(); ++n)
      for (int v : g_.nodes[n].ins) last_use_[v] = (int)n;
    for (int v : g_.results) last_use_[v] = (int)g_.nodes.size();
  }

 private:
  Graph g_;
  std::vector<Tensor> vals_;
  std::vector<int> last_use_;

  void release_after(size_t n) {
    if (last_use_.empty()) return;
    for (int v : g_.nodes[n].ins)
      if (last_use_[v] == (int)n && !g_.values[v].is_const && g_.values[v].arg_index < 0) {
        std::vector<uint8_t>().swap(vals_[v].buf);
      }
  }

  Tensor& out_tensor(const Node& n, int k = 0) {
    const auto& gv = g_.values[n.outs[k]];
    Tensor& t = vals_[n.outs[k]];
    t.alloc(gv.type.dtype, gv.type.shape);
    return t;
  }
  const Tensor& in(const Node& n, int k) { return vals_[n.ins[k]]; }

  std::vector<int64_t> const_ints(const Node& n, int k) {
    const auto& gv = g_.values[n.ins[k]];
    if (!gv.is_const) throw std::runtime_error("expected a constant integer tensor operand");
    std::vector<int64_t> v;
    int64_t cnt = gv.type.is_tensor ? gv.type.numel() : 1;
    for (int64_t i = 0; i < cnt; ++i) v.push_back(gawee::const_as_int(gv, i));
    return v;
  }

  // -- elementwise helpers --------------------------------------------------
  void binary(const Node& n, const std::function<Sc(Sc, Sc, DType)>& f) {
    const Tensor& a = in(n, 0);
    const Tensor& b = in(n, 1);
    Tensor& o = out_tensor(n);
    BIndex ia(a.shape, o.shape), ib(b.shape, o.shape);
    DType t = a.dt;
    for_each_index(o.shape, [&](int64_t k, const int64_t* idx) {
      int64_t oa = 0, ob = 0;
      for (size_t d = 0; d < o.shape.size(); ++d) { oa += idx[d] * ia.st[d]; ob += idx[d] * ib.st[d]; }
      store(o, k, f(load(a, oa), load(b, ob), t));
    });
  }
  void unary_f32(const Node& n, const std::function<float(float)>& f) {
    const Tensor& a = in(n, 0);
    Tensor& o = out_tensor(n);
    if (a.dt != DType::F32) throw std::runtime_error("float op expects f32");
    const float* x = a.p<float>();
    float* y = o.p<float>();
    int64_t cnt = o.numel();
    parallel_for(cnt, [&](int64_t k) { y[k] = f(x[k]); });
  }

  void exec(const Node& n) {
    const std::string& op = n.op;
    if (op == "tensor.empty") { out_tensor(n); return; }
    if (op == "linalg.fill") { fill(n); return; }
    if (op == "linalg.generic") { generic(n); return; }
    if (op == "linalg.reduce") { linalg_reduce(n); return; }
    if (op.rfind("gawee.", 0) != 0) throw std::runtime_error("unsupported op");
    std::string k = op.substr(6);
    // -- elementwise (GaweeToLinalg.cpp:461-557, 1377-1441, 1902-2292) --------
    if (k == "add" || k == "sub" || k == "mul" || k == "div") {
      char c = k[0];
      binary(n, [c](Sc x, Sc y, DType t) {
        Sc r;
        r.i = 0;
        if (t == DType::F32) {
          r.f = c == 'a' ? x.f + y.f : c == 's' ? x.f - y.f : c == 'm' ? x.f * y.f : x.f / y.f;
        } else if (t == DType::F64) {
          r.d = c == 'a' ? x.d + y.d : c == 's' ? x.d - y.d : c == 'm' ? x.d * y.d : x.d / y.d;
        } else {
          if (c == 'd' && y.i == 0) throw std::runtime_error("integer division by zero");
          uint64_t ux = (uint64_t)x.i, uy = (uint64_t)y.i;
          r.i = wrap_int(c == 'a' ? (int64_t)(ux + uy) : c == 's' ? (int64_t)(ux - uy)
                         : c == 'm' ? (int64_t)(ux * uy) : x.i / y.i, t);
        }
        return r;
      });
      return;
    }
    if (k == "relu") { unary_f32(n, [](float x) { return maximumf(x, 0.0f); }); return; }
    if (k == "sqrt") { unary_f32(n, [](float x) { return sqrtf(x); }); return; }
    if (k == "tanh") { unary_f32(n, [](float x) { return tanhf(x); }); return; }
    if (k == "erf") { unary_f32(n, [](float x) { return erff(x); }); return; }
    if (k == "sigmoid") {  // 1 / (1 + exp(-x)), GaweeToLinalg.cpp:1976-1981
      unary_f32(n, [](float x) { return 1.0f / (1.0f + expf(-x)); });
      return;
    }
    if (k == "gelu") {  // 0.5 * (x * (1 + erf(x / sqrt2))), GaweeToLinalg.cpp:2128-2139
      unary_f32(n, [](float x) {
        float d = x / (float)1.4142135623730951;
        return 0.5f * (x * (1.0f + erff(d)));
      });
      return;
    }
    if (k == "hard_sigmoid") {
      float alpha = (float)n.attr("alpha").f, beta = (float)n.attr("beta").f;
      unary_f32(n, [=](float x) { return minimumf(maximumf(x * alpha + beta, 0.0f), 1.0f); });
      return;
    }
    if (k == "hard_swish") {
      unary_f32(n, [](float x) { return (x * minimumf(maximumf(x + 3.0f, 0.0f), 6.0f)) / 6.0f; });
      return;
    }
    if (k == "leaky_relu") {
      float alpha = (float)n.attr("alpha").f;
      unary_f32(n, [=](float x) {
        float s = x * alpha;
        float r = maximumf(x, s);
        return (x < 0.0f) ? s : r;
      });
      return;
    }
    if (k == "equal") {
      binary(n, [](Sc x, Sc y, DType t) {
        Sc r;
        r.i = t == DType::F32 ? (x.f == y.f) : t == DType::F64 ? (x.d == y.d) : (x.i == y.i);
        return r;
      });
      return;
    }
    if (k == "max" || k == "min") { maxmin(n, k == "max"); return; }
    if (k == "where") { where(n); return; }
    if (k == "cast") { cast(n); return; }
    if (k == "batch_norm") { batch_norm(n); return; }
    if (k == "expand") { expand(n); return; }
    // -- contractions ----------------------------------------------------------
    if (k == "conv") { conv(n); return; }
    if (k == "linear") { linear(n); return; }
    if (k == "matmul") { matmul(n); return; }
    // -- pooling / reductions --------------------------------------------------
    if (k == "max_pool") { max_pool(n); return; }
    if (k == "average_pool") { avg_pool(n); return; }
    if (k == "global_average_pool" || k == "ad_avg_pool") { global_avg(n); return; }
    if (k == "reduce_mean" || k == "reduce_sum") { reduce(n, k == "reduce_mean"); return; }
    if (k == "softmax") { softmax(n); return; }
    if (k == "topk") { topk(n); return; }
    // -- layout / index ----------------------------------------------------------
    if (k == "reshape" || k == "flatten" || k == "squeeze" || k == "unsqueeze") {
      Tensor& o = out_tensor(n);
      const Tensor& a = in(n, 0);
      if (a.buf.size() != o.buf.size()) throw std::runtime_error("reshape changes element count");
      std::memcpy(o.buf.data(), a.buf.data(), a.buf.size());
      return;
    }
    if (k == "transpose") { transpose(n); return; }
    if (k == "gather") { gather(n); return; }
    if (k == "gather_elements") { gather_elements(n); return; }
    if (k == "cat") { cat(n); return; }
    if (k == "split") { split(n); return; }
    if (k == "slice") { slice(n); return; }
    if (k == "tile") { tile(n); return; }
    if (k == "pad") { pad(n); return; }
    if (k == "range") { range(n); return; }
    if (k == "shape") { shape_op(n); return; }
    if (k == "resize") { resize(n); return; }
    throw std::runtime_error("unsupported gawee op");
  }

  // ---- linalg forms emitted directly by the ONNX emitter ----------------------
  void fill(const Node& n) {
    Tensor& o = out_tensor(n);
    Sc s = load(in(n, 0), 0);
    for (int64_t k = 0; k < o.numel(); ++k) store(o, k, s);
  }

  void generic(const Node& n) {
    for (bool p : n.parallel)
      if (!p) throw std::runtime_error("linalg.generic with reduction iterators is not supported");
    Tensor& o = out_tensor(n);
    if (!n.maps.back().is_identity()) throw std::runtime_error("linalg.generic output map must be identity");
    int nin = n.n_linalg_ins;
    std::vector<std::vector<int64_t>> st(n.ins.size());
    for (size_t k = 0; k < n.ins.size(); ++k) {
      const Tensor& t = in(n, (int)k);
      auto ts = strides_of(t.shape);
      const auto& m = n.maps[k];
      st[k].assign(o.shape.size() + 1, 0);  // last slot: constant offset
      for (size_t e = 0; e < m.exprs.size(); ++e) {
        if (m.exprs[e] >= 0) st[k][m.exprs[e]] += ts[e];
        else st[k].back() += (-1 - m.exprs[e]) * ts[e];
      }
    }
    std::vector<Sc> regs(n.body.reg_types.size());
    for_each_index(o.shape, [&](int64_t k, const int64_t* idx) {
      for (int a = 0; a < (int)n.ins.size(); ++a) {
        int64_t off = st[a].back();
        for (size_t d = 0; d < o.shape.size(); ++d) off += idx[d] * st[a][d];
        regs[a] = load(in(n, a), off);
      }
      (void)nin;
      store(o, k, run_program(n.body, regs));
    });
  }

  void linalg_reduce(const Node& n) {
    const Tensor& x = in(n, 0);
    const Tensor& init = in(n, 1);
    Tensor& o = out_tensor(n);
    std::memcpy(o.buf.data(), init.buf.data(), init.buf.size());
    std::vector<bool> red(x.shape.size(), false);
    for (auto d : n.dims) red[d] = true;
    auto ost = strides_of(o.shape);
    std::vector<Sc> regs(n.body.reg_types.size());
    for_each_index(x.shape, [&](int64_t k, const int64_t* idx) {
      int64_t off = 0, od = 0;
      for (size_t d = 0; d < x.shape.size(); ++d)
        if (!red[d]) off += idx[d] * ost[od++];
      regs[0] = load(x, k);
      regs[1] = load(o, off);
      store(o, off, run_program(n.body, regs));
    });
  }

  // ---- elementwise with special semantics -----------------------------------
  // gawee.max / gawee.min: pairwise NaN-propagating maximumf/minimumf (ints: maxsi/minsi),
  // each pair broadcast to the result type (GaweeToLinalg.cpp:2250-2292).
  void maxmin(const Node& n, bool is_max) {
    Tensor& o = out_tensor(n);
    Tensor cur = in(n, 0);
    for (size_t k = 1; k < n.ins.size(); ++k) {
      const Tensor& nx = in(n, (int)k);
      Tensor r;
      r.alloc(o.dt, o.shape);
      BIndex ia(cur.shape, o.shape), ib(nx.shape, o.shape);
      for_each_index(o.shape, [&](int64_t e, const int64_t* idx) {
        int64_t oa = 0, ob = 0;
        for (size_t d = 0; d < o.shape.size(); ++d) { oa += idx[d] * ia.st[d]; ob += idx[d] * ib.st[d]; }
        Sc x = load(cur, oa), y = load(nx, ob), z;
        z.i = 0;
        if (o.dt == DType::F32) z.f = is_max ? maximumf(x.f, y.f) : minimumf(x.f, y.f);
        else if (o.dt == DType::F64) z.d = is_max ? maximumd(x.d, y.d) : minimumd(x.d, y.d);
        else z.i = is_max ? std::max(x.i, y.i) : std::min(x.i, y.i);
        store(r, e, z);
      });
      cur = std::move(r);
    }
    o.buf = cur.buf;
  }

  void where(const Node& n) {  // GaweeToLinalg.cpp:2213-2248
    const Tensor& c = in(n, 0);
    const Tensor& a = in(n, 1);
    const Tensor& b = in(n, 2);
    Tensor& o = out_tensor(n);
    BIndex ic(c.shape, o.shape), ia(a.shape, o.shape), ib(b.shape, o.shape);
    for_each_index(o.shape, [&](int64_t k, const int64_t* idx) {
      int64_t oc = 0, oa = 0, ob = 0;
      for (size_t d = 0; d < o.shape.size(); ++d) {
        oc += idx[d] * ic.st[d]; oa += idx[d] * ia.st[d]; ob += idx[d] * ib.st[d];
      }
      store(o, k, (load(c, oc).i & 1) ? load(a, oa) : load(b, ob));
    });
  }

  // gawee.cast (GaweeToLinalg.cpp:2799-2863): i1->float uitofp, int->float sitofp,
  // float->int fptosi (truncation), int widen extsi / narrow trunci.
  void cast(const Node& n) {
    const Tensor& a = in(n, 0);
    Tensor& o = out_tensor(n);
    for (int64_t k = 0; k < o.numel(); ++k) {
      Sc x = load(a, k), y;
      y.i = 0;
      bool sf = gawee::is_float(a.dt), df = gawee::is_float(o.dt);
      if (a.dt == o.dt) y = x;
      else if (sf && df) {
        if (o.dt == DType::F64) y.d = (double)x.f; else y.f = (float)x.d;
      } else if (!sf && df) {
        int64_t v = a.dt == DType::I1 ? (x.i & 1) : x.i;
        if (o.dt == DType::F32) y.f = (float)v; else y.d = (double)v;
      } else if (sf && !df) {
        y.i = wrap_int(a.dt == DType::F32 ? (int64_t)x.f : (int64_t)x.d, o.dt);
      } else {
        y.i = wrap_int(x.i, o.dt);
      }
      store(o, k, y);
    }
  }

  // (x - mean) / sqrt(var + eps) * w + b per channel (GaweeToLinalg.cpp:1122-1173)
  void batch_norm(const Node& n) {
    const Tensor& x = in(n, 0);
    const float* w = in(n, 1).p<float>();
    const float* b = in(n, 2).p<float>();
    const float* mean = in(n, 3).p<float>();
    const float* var = in(n, 4).p<float>();
    float eps = (float)n.attr("eps").f;
    Tensor& o = out_tensor(n);
    int64_t N = x.shape[0], C = x.shape[1], HW = x.shape[2] * x.shape[3];
    for (int64_t i = 0; i < N; ++i)
      for (int64_t c = 0; c < C; ++c)
        for (int64_t s = 0; s < HW; ++s) {
          int64_t k = (i * C + c) * HW + s;
          float denom = sqrtf(var[c] + eps);
          o.p<float>()[k] = ((x.p<float>()[k] - mean[c]) / denom) * w[c] + b[c];
        }
  }

  // linalg.generic broadcast copy: a size-1 input dim meeting a non-1 output dim
  // reads index 0 (GaweeToLinalg.cpp:2294-2332).
  void expand(const Node& n) {
    const Tensor& a = in(n, 0);
    Tensor& o = out_tensor(n);
    BIndex ia(a.shape, o.shape);
    for_each_index(o.shape, [&](int64_t k, const int64_t* idx) {
      int64_t off = 0;
      for (size_t d = 0; d < o.shape.size(); ++d) off += idx[d] * ia.st[d];
      store(o, k, load(a, off));
    });
  }

  // ---- contractions ------------------------------------------------------------
  // gawee.conv (GaweeToLinalg.cpp:322-455): zero-pad H by padding[0] and W by
  // padding[1] on both sides, linalg.conv_2d_nchw_fchw (reduction c, kh, kw),
  // then a separate bias add indexed by channel.
  void conv(const Node& n) {
    const Tensor& x = in(n, 0);
    const Tensor& w = in(n, 1);
    const Tensor& bias = in(n, 2);
    Tensor& o = out_tensor(n);
    auto st = n.attr("strides").ints, pd = n.attr("padding").ints, dl = n.attr("dilation").ints;
    int64_t N = x.shape[0], C = x.shape[1], H = x.shape[2], W = x.shape[3];
    int64_t F = w.shape[0], KH = w.shape[2], KW = w.shape[3];
    int64_t OH = o.shape[2], OW = o.shape[3];
    int64_t ph = pd[0], pw = pd[1];
    if (w.shape[1] != C) throw std::runtime_error("conv channel mismatch (groups are not supported)");
    const float* xp = x.p<float>();
    const float* wp = w.p<float>();
    const float* bp = bias.p<float>();
    float* op = o.p<float>();
    parallel_for(N * F, [&](int64_t nf) {
        int64_t i = nf / F, f = nf % F;
        std::vector<float> acc((size_t)(OH * OW), 0.0f);
        for (int64_t c = 0; c < C; ++c)
          for (int64_t kh = 0; kh < KH; ++kh)
            for (int64_t kw = 0; kw < KW; ++kw) {
              float wv = wp[((f * C + c) * KH + kh) * KW + kw];
              for (int64_t oh = 0; oh < OH; ++oh) {
                int64_t ih = oh * st[0] + kh * dl[0] - ph;
                float* arow = acc.data() + oh * OW;
                if (ih < 0 || ih >= H) {  // padded row: adds x*w with x = 0
                  for (int64_t ow = 0; ow < OW; ++ow) arow[ow] = arow[ow] + 0.0f * wv;
                  continue;
                }
                const float* xrow = xp + ((i * C + c) * H + ih) * W;
                for (int64_t ow = 0; ow < OW; ++ow) {
                  int64_t iw = ow * st[1] + kw * dl[1] - pw;
                  float xv = (iw >= 0 && iw < W) ? xrow[iw] : 0.0f;
                  arow[ow] = arow[ow] + xv * wv;
                }
              }
            }
        float* orow = op + (i * F + f) * OH * OW;
        for (int64_t s = 0; s < OH * OW; ++s) orow[s] = acc[s] + bp[f];
      });
  }

  // gawee.linear (GaweeToLinalg.cpp:877-957): matmul_transpose_b then bias on dim 1.
  void linear(const Node& n) {
    const Tensor& x = in(n, 0);
    const Tensor& w = in(n, 1);
    const Tensor& b = in(n, 2);
    Tensor& o = out_tensor(n);
    if (x.shape.size() != 2) throw std::runtime_error("linear expects a rank-2 input");
    int64_t M = x.shape[0], K = x.shape[1], N = w.shape[0];
    const float* xp = x.p<float>();
    const float* wp = w.p<float>();
    const float* bp = b.p<float>();
    float* op = o.p<float>();
    parallel_for(M, [&](int64_t m) {
      for (int64_t j = 0; j < N; ++j) {
        float acc = 0.0f;
        for (int64_t k = 0; k < K; ++k) acc = acc + xp[m * K + k] * wp[j * K + k];
        op[m * N + j] = acc + bp[j];
      }
    });
  }

  // gawee.matmul (GaweeToLinalg.cpp:959-1112): batch dims broadcast (size 1 -> 0),
  // reduction innermost, acc = a*b + acc from zero.
  void matmul(const Node& n) {
    const Tensor& a = in(n, 0);
    const Tensor& b = in(n, 1);
    Tensor& o = out_tensor(n);
    int ra = (int)a.shape.size(), rb = (int)b.shape.size(), ro = (int)o.shape.size();
    if (ra < 2 || rb < 2) throw std::runtime_error("matmul expects rank >= 2 operands");
    int64_t M = a.shape[ra - 2], K = a.shape[ra - 1], N = b.shape[rb - 1];
    if (b.shape[rb - 2] != K) throw std::runtime_error("matmul K mismatch");
    std::vector<int64_t> bshape(o.shape.begin(), o.shape.end() - 2);
    std::vector<int64_t> ash(a.shape.begin(), a.shape.end() - 2), bsh(b.shape.begin(), b.shape.end() - 2);
    BIndex ia(ash, bshape), ib(bsh, bshape);
    int64_t nb = 1;
    for (auto d : bshape) nb *= d;
    std::vector<int64_t> boff_a(nb), boff_b(nb);
    for_each_index(bshape, [&](int64_t k, const int64_t* idx) {
      int64_t x = 0, y = 0;
      for (size_t d = 0; d < bshape.size(); ++d) { x += idx[d] * ia.st[d]; y += idx[d] * ib.st[d]; }
      boff_a[k] = x * M * K;
      boff_b[k] = y * K * N;
    });
    (void)ro;
    const float* ap = a.p<float>();
    const float* bp = b.p<float>();
    float* op = o.p<float>();
    parallel_for(nb * M, [&](int64_t bm) {
        int64_t bi = bm / M, m = bm % M;
        float* orow = op + (bi * M + m) * N;
        for (int64_t j = 0; j < N; ++j) orow[j] = 0.0f;
        const float* arow = ap + boff_a[bi] + m * K;
        const float* bmat = bp + boff_b[bi];
        for (int64_t k = 0; k < K; ++k) {
          float av = arow[k];
          const float* brow = bmat + k * N;
          for (int64_t j = 0; j < N; ++j) orow[j] = av * brow[j] + orow[j];
        }
      });
  }

  // ---- pooling -----------------------------------------------------------------
  // gawee.max_pool (GaweeToLinalg.cpp:565-706): pad with -inf using padding[0..1],
  // ceilMode ignored, linalg.pooling_nchw_max over an output pre-filled with -inf.
  void max_pool(const Node& n) {
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    auto ks = n.attr("kernelSize").ints, st = n.attr("strides").ints, pd = n.attr("padding").ints,
         dl = n.attr("dilation").ints;
    int64_t N = x.shape[0], C = x.shape[1], H = x.shape[2], W = x.shape[3];
    int64_t OH = o.shape[2], OW = o.shape[3];
    const float* xp = x.p<float>();
    float* op = o.p<float>();
    const float ninf = -std::numeric_limits<float>::infinity();
    parallel_for(N * C, [&](int64_t nc) {
      int64_t i = nc / C, c = nc % C;
        for (int64_t oh = 0; oh < OH; ++oh)
          for (int64_t ow = 0; ow < OW; ++ow) {
            float m = ninf;
            for (int64_t kh = 0; kh < ks[0]; ++kh)
              for (int64_t kw = 0; kw < ks[1]; ++kw) {
                int64_t ih = oh * st[0] + kh * dl[0] - pd[0];
                int64_t iw = ow * st[1] + kw * dl[1] - pd[1];
                float v = (ih >= 0 && ih < H && iw >= 0 && iw < W) ? xp[((i * C + c) * H + ih) * W + iw] : ninf;
                m = maximumf(m, v);
              }
            op[((i * C + c) * OH + oh) * OW + ow] = m;
          }
    });
  }

  // gawee.average_pool (GaweeToLinalg.cpp:1175-1258): zero pad, sum pool
  // (dilation 1), divide by kernel count (count_include_pad semantics).
  void avg_pool(const Node& n) {
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    auto ks = n.attr("kernelSize").ints, st = n.attr("strides").ints, pd = n.attr("padding").ints;
    if (!n.attr("countIncludePad").b && (pd[0] != 0 || pd[1] != 0))
      throw std::runtime_error("average_pool with padding requires count_include_pad=true");
    int64_t N = x.shape[0], C = x.shape[1], H = x.shape[2], W = x.shape[3];
    int64_t OH = o.shape[2], OW = o.shape[3];
    float cnt = (float)(ks[0] * ks[1]);
    const float* xp = x.p<float>();
    float* op = o.p<float>();
    for (int64_t i = 0; i < N; ++i)
      for (int64_t c = 0; c < C; ++c)
        for (int64_t oh = 0; oh < OH; ++oh)
          for (int64_t ow = 0; ow < OW; ++ow) {
            float s = 0.0f;
            for (int64_t kh = 0; kh < ks[0]; ++kh)
              for (int64_t kw = 0; kw < ks[1]; ++kw) {
                int64_t ih = oh * st[0] + kh - pd[0], iw = ow * st[1] + kw - pd[1];
                float v = (ih >= 0 && ih < H && iw >= 0 && iw < W) ? xp[((i * C + c) * H + ih) * W + iw] : 0.0f;
                s = s + v;
              }
            op[((i * C + c) * OH + oh) * OW + ow] = s / cnt;
          }
  }

  // gawee.global_average_pool / gawee.ad_avg_pool (GaweeToLinalg.cpp:1327-1375,
  // 713-806): sum over the whole H x W plane, then divide by h*w.
  void global_avg(const Node& n) {
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    int64_t N = x.shape[0], C = x.shape[1], HW = x.shape[2] * x.shape[3];
    float cnt = (float)HW;
    const float* xp = x.p<float>();
    float* op = o.p<float>();
    for (int64_t i = 0; i < N * C; ++i) {
      float s = 0.0f;
      for (int64_t k = 0; k < HW; ++k) s = s + xp[i * HW + k];
      op[i] = s / cnt;
    }
  }

  // gawee.reduce_mean / reduce_sum (GaweeToLinalg.cpp:1443-1572): linalg.reduce sum
  // from zero in input row-major order, then (mean) a separate divide by the count.
  void reduce(const Node& n, bool mean) {
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    int r = (int)x.shape.size();
    std::vector<bool> red(r, false);
    int64_t count = 1;
    for (auto a : n.attr("axes").ints) {
      int64_t ax = a < 0 ? a + r : a;
      if (!red[ax]) count *= x.shape[ax];
      red[ax] = true;
    }
    // output laid out over kept dims (keepDims only inserts unit dims)
    std::vector<int64_t> kept;
    for (int d = 0; d < r; ++d) if (!red[d]) kept.push_back(x.shape[d]);
    auto kst = strides_of(kept);
    if (x.dt != DType::F32) throw std::runtime_error("reduce expects f32");
    std::vector<float> acc((size_t)o.numel(), 0.0f);
    const float* xp = x.p<float>();
    for_each_index(x.shape, [&](int64_t k, const int64_t* idx) {
      int64_t off = 0, kd = 0;
      for (int d = 0; d < r; ++d) if (!red[d]) off += idx[d] * kst[kd++];
      acc[off] = acc[off] + xp[k];
    });
    float c = (float)count;
    for (int64_t k = 0; k < o.numel(); ++k) o.p<float>()[k] = mean ? acc[k] / c : acc[k];
  }

  // gawee.softmax -> linalg.softmax, decomposed as upstream MLIR does
  // (DecomposeAggregatedLinalgOps.cpp:22-55): max-reduce (maxnumf from the
  // lowest finite float), exp(x - max), sum-reduce from zero, divide.
  void softmax(const Node& n) {
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    int r = (int)x.shape.size();
    int64_t ax = n.attr("axis").i;
    if (ax < 0) ax += r;
    int64_t L = x.shape[ax], inner = 1, outer = 1;
    for (int d = ax + 1; d < r; ++d) inner *= x.shape[d];
    for (int d = 0; d < ax; ++d) outer *= x.shape[d];
    const float* xp = x.p<float>();
    float* op = o.p<float>();
    parallel_for(outer * inner, [&](int64_t ab) {
        int64_t a = ab / inner, b = ab % inner;
        const float* row = xp + a * L * inner + b;
        float* orow = op + a * L * inner + b;
        float m = -std::numeric_limits<float>::max();
        for (int64_t j = 0; j < L; ++j) m = std::fmax(m, row[j * inner]);
        float s = 0.0f;
        for (int64_t j = 0; j < L; ++j) {
          float e = expf(row[j * inner] - m);
          orow[j * inner] = e;
          s = s + e;
        }
        for (int64_t j = 0; j < L; ++j) orow[j * inner] = orow[j * inner] / s;
      });
  }

  // gawee.topk (GaweeToLinalg.cpp:1577-1680): rank-2, axis 1; k rounds of a
  // first-strict-maximum scan over unused positions starting from (-inf, 0).
  void topk(const Node& n) {
    const Tensor& x = in(n, 0);
    Tensor& vals = out_tensor(n, 0);
    Tensor& idxs = out_tensor(n, 1);
    int64_t B = x.shape[0], L = x.shape[1], K = n.attr("k").i;
    const float* xp = x.p<float>();
    for (int64_t b = 0; b < B; ++b) {
      std::vector<uint8_t> used((size_t)L, 0);
      for (int64_t ki = 0; ki < K; ++ki) {
        float bv = -std::numeric_limits<float>::infinity();
        int64_t bi = 0;
        for (int64_t j = 0; j < L; ++j) {
          float v = xp[b * L + j];
          if (!used[j] && v > bv) { bv = v; bi = j; }
        }
        vals.p<float>()[b * K + ki] = bv;
        idxs.p<int64_t>()[b * K + ki] = bi;
        used[bi] = 1;
      }
    }
  }

  // ---- layout / index ----------------------------------------------------------
  void transpose(const Node& n) {  // linalg.transpose, GaweeToLinalg.cpp:1735-1751
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    auto perm = n.attr("perm").ints;
    auto xs = strides_of(x.shape);
    size_t es = gawee::dtype_size(x.dt);
    for_each_index(o.shape, [&](int64_t k, const int64_t* idx) {
      int64_t off = 0;
      for (size_t d = 0; d < o.shape.size(); ++d) off += idx[d] * xs[perm[d]];
      std::memcpy(o.buf.data() + k * es, x.buf.data() + off * es, es);
    });
  }

  // gawee.gather (GaweeToLinalg.cpp:2334-2396): out[pre, idx..., post] =
  // data[pre, indices[idx...], post]; the reference neither wraps negative
  // indices nor checks bounds, so an out-of-range index is undefined there and
  // an error here.
  void gather(const Node& n) {
    const Tensor& data = in(n, 0);
    const Tensor& ind = in(n, 1);
    Tensor& o = out_tensor(n);
    int rd = (int)data.shape.size();
    int64_t ax = n.attr("axis").i;
    if (ax < 0) ax += rd;
    int ri = (int)ind.shape.size();
    auto ds = strides_of(data.shape);
    size_t es = gawee::dtype_size(data.dt);
    for_each_index(o.shape, [&](int64_t k, const int64_t* idx) {
      int64_t off = 0;
      for (int d = 0; d < rd; ++d) {
        int64_t v;
        if (d < ax) v = idx[d];
        else if (d == ax) {
          int64_t ioff = 0;
          auto is = strides_of(ind.shape);
          for (int e = 0; e < ri; ++e) ioff += idx[ax + e] * is[e];
          v = load(ind, ioff).i;
          if (v < 0 || v >= data.shape[ax]) throw std::runtime_error("gather index out of range");
        } else v = idx[d + ri - 1];
        off += v * ds[d];
      }
      std::memcpy(o.buf.data() + k * es, data.buf.data() + off * es, es);
    });
  }

  void gather_elements(const Node& n) {  // GaweeToLinalg.cpp:2398-2437
    const Tensor& data = in(n, 0);
    const Tensor& ind = in(n, 1);
    Tensor& o = out_tensor(n);
    int r = (int)ind.shape.size();
    int64_t ax = n.attr("axis").i;
    if (ax < 0) ax += r;
    auto ds = strides_of(data.shape);
    size_t es = gawee::dtype_size(data.dt);
    for_each_index(o.shape, [&](int64_t k, const int64_t* idx) {
      int64_t off = 0;
      for (int d = 0; d < r; ++d) {
        int64_t v = d == ax ? load(ind, k).i : idx[d];
        if (d == ax && (v < 0 || v >= data.shape[d])) throw std::runtime_error("gather_elements index out of range");
        off += v * ds[d];
      }
      std::memcpy(o.buf.data() + k * es, data.buf.data() + off * es, es);
    });
  }

  void cat(const Node& n) {  // tensor.insert_slice per input, GaweeToLinalg.cpp:1260-1325
    Tensor& o = out_tensor(n);
    int r = (int)o.shape.size();
    int64_t ax = n.attr("axis").i;
    if (ax < 0) ax += r;
    size_t es = gawee::dtype_size(o.dt);
    auto os = strides_of(o.shape);
    int64_t base = 0;
    for (size_t k = 0; k < n.ins.size(); ++k) {
      const Tensor& x = in(n, (int)k);
      for_each_index(x.shape, [&](int64_t e, const int64_t* idx) {
        int64_t off = 0;
        for (int d = 0; d < r; ++d) off += (idx[d] + (d == ax ? base : 0)) * os[d];
        std::memcpy(o.buf.data() + off * es, x.buf.data() + e * es, es);
      });
      base += x.shape[ax];
    }
  }

  void split(const Node& n) {  // extract_slice per result, GaweeToLinalg.cpp:2554-2592
    const Tensor& x = in(n, 0);
    int r = (int)x.shape.size();
    int64_t ax = n.attr("axis").i;
    if (ax < 0) ax += r;
    auto xs = strides_of(x.shape);
    size_t es = gawee::dtype_size(x.dt);
    int64_t base = 0;
    auto sizes = n.attr("splitSizes").ints;
    for (size_t k = 0; k < n.outs.size(); ++k) {
      Tensor& o = out_tensor(n, (int)k);
      for_each_index(o.shape, [&](int64_t e, const int64_t* idx) {
        int64_t off = 0;
        for (int d = 0; d < r; ++d) off += (idx[d] + (d == ax ? base : 0)) * xs[d];
        std::memcpy(o.buf.data() + e * es, x.buf.data() + off * es, es);
      });
      base += sizes[k];
    }
  }

  // gawee.slice (GaweeToLinalg.cpp:2594-2715): constant axes/steps (steps > 0),
  // negative starts wrapped once by the dim size, sizes from the result type,
  // offsets not clamped.
  void slice(const Node& n) {
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    auto starts = const_ints(n, 1), axes = const_ints(n, 3), steps = const_ints(n, 4);
    int r = (int)x.shape.size();
    std::vector<int64_t> off(r, 0), step(r, 1);
    for (size_t k = 0; k < axes.size(); ++k) {
      int64_t ax = axes[k] < 0 ? axes[k] + r : axes[k];
      if (steps[k] <= 0) throw std::runtime_error("slice supports positive steps only");
      int64_t s = starts[k];
      if (s < 0) s += x.shape[ax];
      off[ax] = s;
      step[ax] = steps[k];
    }
    auto xs = strides_of(x.shape);
    size_t es = gawee::dtype_size(x.dt);
    for_each_index(o.shape, [&](int64_t e, const int64_t* idx) {
      int64_t src = 0;
      for (int d = 0; d < r; ++d) {
        int64_t v = off[d] + idx[d] * step[d];
        if (v < 0 || v >= x.shape[d]) throw std::runtime_error("slice reads out of bounds");
        src += v * xs[d];
      }
      std::memcpy(o.buf.data() + e * es, x.buf.data() + src * es, es);
    });
  }

  void tile(const Node& n) {  // out[i] = in[i mod dim], GaweeToLinalg.cpp:2717-2752
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    auto xs = strides_of(x.shape);
    size_t es = gawee::dtype_size(x.dt);
    for_each_index(o.shape, [&](int64_t e, const int64_t* idx) {
      int64_t src = 0;
      for (size_t d = 0; d < o.shape.size(); ++d) src += (idx[d] % x.shape[d]) * xs[d];
      std::memcpy(o.buf.data() + e * es, x.buf.data() + src * es, es);
    });
  }

  void pad(const Node& n) {  // constant mode tensor.pad, GaweeToLinalg.cpp:2754-2797
    if (n.attr("mode").s != "constant") throw std::runtime_error("pad supports constant mode only");
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    auto pads = const_ints(n, 1);
    Sc cv = load(in(n, 2), 0);
    int r = (int)x.shape.size();
    auto xs = strides_of(x.shape);
    for_each_index(o.shape, [&](int64_t e, const int64_t* idx) {
      int64_t src = 0;
      bool inside = true;
      for (int d = 0; d < r; ++d) {
        int64_t v = idx[d] - pads[d];
        if (v < 0 || v >= x.shape[d]) { inside = false; break; }
        src += v * xs[d];
      }
      store(o, e, inside ? load(x, src) : cv);
    });
  }

  void range(const Node& n) {  // start + i * delta, GaweeToLinalg.cpp:2439-2496
    Tensor& o = out_tensor(n);
    Sc start = load(in(n, 0), 0), delta = load(in(n, 2), 0);
    for (int64_t i = 0; i < o.numel(); ++i) {
      Sc v;
      v.i = 0;
      if (o.dt == DType::F32) v.f = start.f + (float)i * delta.f;
      else if (o.dt == DType::F64) v.d = start.d + (double)i * delta.d;
      else v.i = wrap_int((int64_t)((uint64_t)start.i + (uint64_t)i * (uint64_t)delta.i), o.dt);
      store(o, i, v);
    }
  }

  void shape_op(const Node& n) {  // GaweeToLinalg.cpp:1851-1883
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    int r = (int)x.shape.size();
    int64_t s = n.attr("start").i, e = n.attr("end").i;
    if (s < 0) s += r;
    if (e < 0) e += r;
    e = std::min<int64_t>(e, r);
    for (int64_t d = s; d < e; ++d) {
      Sc v;
      v.i = x.shape[d];
      store(o, d - s, v);
    }
  }

  // gawee.resize (GaweeToLinalg.cpp:2498-2552): nearest / asymmetric / floor with
  // integer scales: source index = output index / scale.
  void resize(const Node& n) {
    const Tensor& x = in(n, 0);
    Tensor& o = out_tensor(n);
    const auto& sv = g_.values[n.ins[1]];
    std::vector<int64_t> scale;
    for (int64_t k = 0; k < sv.type.numel(); ++k) scale.push_back((int64_t)gawee::const_as_double(sv, k));
    auto xs = strides_of(x.shape);
    size_t es = gawee::dtype_size(x.dt);
    for_each_index(o.shape, [&](int64_t e, const int64_t* idx) {
      int64_t src = 0;
      for (size_t d = 0; d < o.shape.size(); ++d) src += (idx[d] / scale[d]) * xs[d];
      std::memcpy(o.buf.data() + e * es, x.buf.data() + src * es, es);
    });
  }
};

}  // namespace oracle

// ---------------------------------------------------------------------------
// C interface (loaded by the tests through ctypes).
// ---------------------------------------------------------------------------
namespace {
void set_err(char* err, int n, const std::string& msg) {
  if (err && n > 0) {
    std::strncpy(err, msg.c_str(), (size_t)n - 1);
    err[n - 1] = 0;
  }
}
}  // namespace

extern "C" {

void* gawee_oracle_load(const char* mlir_text, const char* entry, char* err, int errlen) {
  try {
    auto g = gawee::parse_mlir(mlir_text, entry ? entry : "forward");
    auto* it = new oracle::Interp(std::move(g));
    it->prepare_liveness();
    return it;
  } catch (std::exception& e) {
    set_err(err, errlen, e.what());
    return nullptr;
  }
}

void gawee_oracle_free(void* h) { delete static_cast<oracle::Interp*>(h); }

int gawee_oracle_num_args(void* h) { return (int)static_cast<oracle::Interp*>(h)->graph().args.size(); }
int gawee_oracle_num_outputs(void* h) { return (int)static_cast<oracle::Interp*>(h)->graph().results.size(); }

static int info(const gawee::Value& v, int* dtype, int* rank, int64_t* shape) {
  *dtype = (int)v.type.dtype;
  *rank = v.type.rank();
  for (int d = 0; d < v.type.rank() && d < 8; ++d) shape[d] = v.type.shape[d];
  return v.type.rank() > 8 ? 1 : 0;
}

int gawee_oracle_arg_info(void* h, int i, int* dtype, int* rank, int64_t* shape) {
  const auto& g = static_cast<oracle::Interp*>(h)->graph();
  if (i < 0 || i >= (int)g.args.size()) return 1;
  return info(g.values[g.args[i]], dtype, rank, shape);
}

int gawee_oracle_output_info(void* h, int i, int* dtype, int* rank, int64_t* shape) {
  const auto& g = static_cast<oracle::Interp*>(h)->graph();
  if (i < 0 || i >= (int)g.results.size()) return 1;
  return info(g.values[g.results[i]], dtype, rank, shape);
}

int gawee_oracle_run(void* h, const void* const* args, void* const* outs, int threads, char* err, int errlen) {
  auto* it = static_cast<oracle::Interp*>(h);
  try {
    oracle::g_threads = threads > 0 ? threads : (int)std::max(1u, std::thread::hardware_concurrency());
    std::vector<const void*> a(args, args + it->graph().args.size());
    std::vector<void*> o(outs, outs + it->graph().results.size());
    it->run(a, o);
    return 0;
  } catch (std::exception& e) {
    set_err(err, errlen, e.what());
    return 1;
  }
}

}  // extern "C"
