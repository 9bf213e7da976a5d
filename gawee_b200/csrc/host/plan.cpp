// Planner: gawee graph -> views, fused ops, phases and buffers. See plan.h.
#include "plan.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <map>
#include <numeric>
#include <set>
#include <sstream>
#include <stdexcept>

#include "../kernels/kernels.h"
#include "launch.h"

namespace gawee {

namespace {

[[noreturn]] void unsupported(const std::string& msg) { throw std::runtime_error("unsupported: " + msg); }

std::vector<int64_t> rowmajor_strides(const std::vector<int64_t>& shape) {
  std::vector<int64_t> st(shape.size(), 1);
  for (int i = (int)shape.size() - 2; i >= 0; --i) st[i] = st[i + 1] * shape[i + 1];
  return st;
}

// strides for a dense layout whose dims are stored in `order` (outermost first)
std::vector<int64_t> strides_in_order(const std::vector<int64_t>& shape, const std::vector<int>& order) {
  std::vector<int64_t> st(shape.size(), 0);
  int64_t acc = 1;
  for (int i = (int)order.size() - 1; i >= 0; --i) {
    st[order[i]] = acc;
    acc *= shape[order[i]];
  }
  return st;
}

// Small helper to build scalar programs for the gawee elementwise ops.
struct PB {
  EProgram p;
  explicit PB(std::vector<DType> args) {
    for (auto t : args) p.add_reg(t);
    p.n_args = (int)args.size();
  }
  int cf(double v, DType t = DType::F32) {
    EInstr in;
    in.op = EOp::CONST;
    in.ty = in.rty = t;
    in.fimm = v;
    in.iimm = (int64_t)v;
    in.dst = (int16_t)p.add_reg(t);
    p.code.push_back(in);
    return in.dst;
  }
  int ci(int64_t v, DType t) {
    EInstr in;
    in.op = EOp::CONST;
    in.ty = in.rty = t;
    in.iimm = v;
    in.fimm = (double)v;
    in.dst = (int16_t)p.add_reg(t);
    p.code.push_back(in);
    return in.dst;
  }
  int op(EOp o, DType ty, int a, int b = -1, int c = -1, DType rty = DType(-1), int pred = 0) {
    EInstr in;
    in.op = o;
    in.ty = ty;
    in.rty = (int)rty < 0 ? ty : rty;
    in.a = (int16_t)a;
    in.b = (int16_t)b;
    in.c = (int16_t)c;
    in.pred = (int8_t)pred;
    in.dst = (int16_t)p.add_reg(in.rty);
    p.code.push_back(in);
    return in.dst;
  }
  EProgram done(int result) {
    p.result = result;
    return p;
  }
};

bool same_view(const View& a, const View& b) {
  return a.buf == b.buf && a.off == b.off && a.shape == b.shape && a.st == b.st && a.dt == b.dt;
}

}  // namespace

bool View::dense_rowmajor() const {
  int64_t expect = 1;
  for (int i = rank() - 1; i >= 0; --i) {
    if (shape[i] == 1) continue;
    if (st[i] != expect) return false;
    expect *= shape[i];
  }
  return true;
}

std::string Plan::summary() const {
  std::ostringstream o;
  int live = 0;
  for (auto& op : ops) live += !op.dead;
  o << "ops=" << live << " prologue=" << prologue.size() << " pack=" << pack.size() << " main=" << main.size()
    << " arena_bytes=" << arena_bytes << " persist_bytes=" << persist_bytes << "\n";
  for (int i : main) o << "  " << ops[i].name << execution_note(ops[i]) << "\n";
  return o.str();
}

namespace {

class Planner {
 public:
  explicit Planner(Graph g) { plan_ = std::make_unique<Plan>(); plan_->g = std::move(g); }

  std::unique_ptr<Plan> run() {
    Graph& g = plan_->g;
    plan_->value_view.assign(g.values.size(), View());
    has_view_.assign(g.values.size(), false);
    // arguments
    for (size_t a = 0; a < g.args.size(); ++a) {
      const Value& v = g.values[g.args[a]];
      if (!v.type.is_tensor) unsupported("scalar function arguments");
      int b = new_buf(v.type.dtype, v.type.numel(), BufKind::ARG);
      plan_->bufs[b].arg = (int)a;
      plan_->arg_buf.push_back(b);
      set_view(g.args[a], dense_view(b, v.type.dtype, v.type.shape));
    }
    find_attention_clusters();
    find_norm_clusters();
    find_rope_clusters();
    find_merged_matmuls();
    for (size_t n = 0; n < g.nodes.size(); ++n) {
      if (skip_node_.count((int)n)) continue;  // folded into a fused op
      try {
        auto at = attn_at_.find((int)n);
        if (at != attn_at_.end()) {
          plan_attention(at->second);
          continue;
        }
        auto nt = norm_at_.find((int)n);
        if (nt != norm_at_.end()) {
          plan_rownorm(nt->second);
          continue;
        }
        auto rt = rope_at_.find((int)n);
        if (rt != rope_at_.end()) {
          plan_rope(rt->second);
          continue;
        }
        auto mt = merge_at_.find((int)n);
        if (mt != merge_at_.end()) {
          plan_matmul_merged(mt->second);
          continue;
        }
        plan_node(g.nodes[n]);
      } catch (std::exception& e) {
        throw std::runtime_error("node " + std::to_string(n) + " (" + g.nodes[n].op + "): " + e.what());
      }
    }
    // results must be dense row-major in buffers that survive the forward
    for (int r : g.results) {
      View v = value_view(r);
      const Buf& b = plan_->bufs[v.buf];
      if (!v.dense_rowmajor() || b.kind == BufKind::ARG || b.kind == BufKind::CONST || v.off != 0 ||
          v.numel() != b.elems)
        v = copy_to_new(v, "result_copy");
      plan_->result_view.push_back(v);
    }
    assign_phases();
    fuse_elementwise();
    fuse_epilogues();
    finalize_kinds();
    for (const Op& op : plan_->ops)
      if (!op.dead && op.kind == OpKind::TC) validate_tc(op);
    return std::move(plan_);
  }

 private:
  std::unique_ptr<Plan> plan_;
  std::vector<bool> has_view_;

  // ---------------------------------------------------------------- attention clusters
  // matmul(Q, KT) -> div(A, c) [-> add(., mask)] -> softmax(-1) -> matmul(P, V),
  // every intermediate used once (GaweeToLinalg.cpp:959-1112, 1377-1441,
  // 1885-1900).  K and V may come through the GQA head expansion
  // unsqueeze(x, [2]) -> expand([B, Hkv, rep, S, D]) -> reshape([B, H, S, D]),
  // which the fused op replaces by reading head h / rep.
  struct AttnMatch {
    int q = -1, kt = -1, k_base = -1, v = -1, v_base = -1, mask = -1;
    double c = 1.0;
    int out_transpose = -1;  // the node permuting the output to [B, S, H, D], if that is its only use
    int pv_out = -1;         // the cluster's result value
  };
  std::map<int, AttnMatch> attn_at_;  // PV matmul node -> cluster
  std::set<int> skip_node_;
  std::vector<int> uses_;

  int def_node(int v) const { return plan_->g.values[v].def_node; }
  const Node* node_of(int v) const {
    int d = def_node(v);
    return d >= 0 ? &plan_->g.nodes[d] : nullptr;
  }
  static bool is_op(const Node* n, const char* op) { return n && n->op == op; }

  // x = reshape(expand(unsqueeze(base, [2]), [B, Hkv, rep, S, D]), [B, Hkv * rep, S, D]) -> base
  int gqa_base(int x, std::vector<int>& nodes) {
    const Node* r = node_of(x);
    if (!is_op(r, "gawee.reshape") || uses_[x] != 1) return -1;
    const Node* e = node_of(r->ins[0]);
    if (!is_op(e, "gawee.expand") || uses_[r->ins[0]] != 1) return -1;
    const Node* u = node_of(e->ins[0]);
    if (!is_op(u, "gawee.unsqueeze") || uses_[e->ins[0]] != 1) return -1;
    if (!u->has_attr("axes") || u->attr("axes").ints != std::vector<int64_t>{2}) return -1;
    const auto& es = val(r->ins[0]).type.shape;  // [B, Hkv, rep, S, D]
    const auto& bs = val(u->ins[0]).type.shape;  // [B, Hkv, S, D]
    const auto& xs = val(x).type.shape;          // [B, H, S, D]
    if (es.size() != 5 || bs.size() != 4 || xs.size() != 4) return -1;
    if (es[0] != bs[0] || es[1] != bs[1] || es[3] != bs[2] || es[4] != bs[3]) return -1;
    if (xs[0] != bs[0] || xs[1] != es[1] * es[2] || xs[2] != bs[2] || xs[3] != bs[3]) return -1;
    nodes.push_back(def_node(x));
    return u->ins[0];
  }

  void find_attention_clusters() {
    Graph& g = plan_->g;
    uses_.assign(g.values.size(), 0);
    for (const Node& n : g.nodes)
      for (int v : n.ins) uses_[v]++;
    for (int r : g.results) uses_[r] += 2;  // a result is never folded away
    for (size_t e = 0; e < g.nodes.size(); ++e) {
      const Node& E = g.nodes[e];
      if (E.op != "gawee.matmul" || E.ins.size() != 2) continue;
      const Node* P = node_of(E.ins[0]);
      if (!is_op(P, "gawee.softmax") || uses_[E.ins[0]] != 1) continue;
      const int rank = val(E.ins[0]).type.rank();
      int64_t axis = P->has_attr("axis") ? P->attr("axis").i : -1;
      if (axis < 0) axis += rank;
      if (rank != 4 || axis != 3) continue;
      // softmax input: add(div(.), mask), or the div itself (no mask)
      const Node* C = node_of(P->ins[0]);
      if (uses_[P->ins[0]] != 1) continue;
      const Node* Bn = nullptr;
      int mask = -1;
      if (is_op(C, "gawee.div")) {
        Bn = C;
      } else if (is_op(C, "gawee.add")) {
        for (int side = 0; side < 2; ++side) {
          const Node* D = node_of(C->ins[side]);
          if (is_op(D, "gawee.div") && uses_[C->ins[side]] == 1) {
            Bn = D;
            mask = C->ins[1 - side];
            break;
          }
        }
      }
      if (!Bn) continue;
      double c = 0;
      int64_t ci = 0;
      if (!scalar_const(Bn->ins[1], c, ci) || val(Bn->ins[1]).type.dtype != DType::F32 || !(c > 0)) continue;
      const Node* A = node_of(Bn->ins[0]);
      if (!is_op(A, "gawee.matmul") || uses_[Bn->ins[0]] != 1) continue;
      const auto& qs = val(A->ins[0]).type.shape;   // [B, H, S, D]
      const auto& kts = val(A->ins[1]).type.shape;  // [B, H, D, Skv]
      const auto& vs = val(E.ins[1]).type.shape;    // [B, H, Skv, D]
      if (qs.size() != 4 || kts.size() != 4 || vs.size() != 4) continue;
      if (kts[0] != qs[0] || kts[1] != qs[1] || kts[2] != qs[3] || vs[0] != qs[0] || vs[1] != qs[1] ||
          vs[2] != kts[3] || vs[3] != qs[3])
        continue;
      if (val(A->ins[0]).type.dtype != DType::F32 || val(A->ins[1]).type.dtype != DType::F32 ||
          val(E.ins[1]).type.dtype != DType::F32)
        continue;
      if (mask >= 0) {
        const Value& ms = val(mask);
        if (ms.type.dtype != DType::F32 || ms.type.rank() > 4) continue;
        const std::vector<int64_t> sshape = {qs[0], qs[1], qs[2], kts[3]};
        bool bcast_ok = true;  // the mask broadcasts to the score shape
        for (int d = 0; d < ms.type.rank(); ++d) {
          const int64_t md = ms.type.shape[ms.type.rank() - 1 - d], sd = sshape[3 - d];
          if (md != 1 && md != sd) bcast_ok = false;
        }
        if (!bcast_ok) continue;
      }
      if (!kern::attn_supported(qs[3], kts[3], qs[1], qs[1])) continue;
      AttnMatch m;
      m.q = A->ins[0];
      m.kt = A->ins[1];
      m.v = E.ins[1];
      m.mask = mask;
      m.c = c;
      m.pv_out = E.outs[0];
      std::vector<int> skip = {def_node(E.ins[0]), def_node(P->ins[0]), def_node(Bn->ins[0])};
      if (Bn != C) skip.push_back(def_node(C->ins[C->ins[0] == mask ? 1 : 0]));  // the div under the add
      // K: the transpose of a GQA expansion, if any
      const Node* Tk = node_of(m.kt);
      if (is_op(Tk, "gawee.transpose") && uses_[m.kt] == 1 && Tk->attr("perm").ints == std::vector<int64_t>{0, 1, 3, 2}) {
        std::vector<int> kn;
        int kb = gqa_base(Tk->ins[0], kn);
        if (kb >= 0) {
          m.k_base = kb;
          skip.push_back(def_node(m.kt));
          skip.insert(skip.end(), kn.begin(), kn.end());
        }
      }
      std::vector<int> vn;
      m.v_base = gqa_base(m.v, vn);
      if (m.v_base >= 0) skip.insert(skip.end(), vn.begin(), vn.end());
      // K and V must agree on the head grouping
      const int64_t hk = m.k_base >= 0 ? val(m.k_base).type.shape[1] : qs[1];
      const int64_t hv = m.v_base >= 0 ? val(m.v_base).type.shape[1] : qs[1];
      if (hk != hv || !kern::attn_supported(qs[3], kts[3], qs[1], hk)) continue;
      // an output used only by transpose(perm [0, 2, 1, 3]) is written in [B, S, H, D] order
      const int out = E.outs[0];
      if (uses_[out] == 1) {
        for (size_t n2 = e + 1; n2 < g.nodes.size(); ++n2) {
          const Node& X = g.nodes[n2];
          if (X.op == "gawee.transpose" && X.ins.size() == 1 && X.ins[0] == out &&
              X.attr("perm").ints == std::vector<int64_t>{0, 2, 1, 3})
            m.out_transpose = (int)n2;
        }
      }
      for (int sn : skip) skip_node_.insert(sn);
      attn_at_[(int)e] = m;
    }
  }

  // ---------------------------------------------------------------- normalisation chains
  // RMSNorm:   pow(x, 2) -> reduce_mean(-1, keepdims) -> add(eps) -> sqrt -> div(x, .) -> mul(., w) [-> add(., b)]
  // LayerNorm: the same over xc = sub(x0, reduce_mean(x0, -1)), as the emitter decomposes them
  // (ReduceMeanOpLowering GaweeToLinalg.cpp:1443-1514, Pow ONNXMLIREmitter.cpp:846-871,
  // Sqrt / Div 1902-1927 / 1421-1441, Mul / Add 532-557, 1377-1419).
  struct NormMatch {
    int x = -1, x0 = -1, w = -1, b = -1, out = -1;
    double eps = 0;
    bool centered = false;
  };
  std::map<int, NormMatch> norm_at_;  // final node of the chain -> match

  bool is_square_of(const Node* P, int x) {
    if (!P) return false;
    if (P->op == "gawee.mul") return P->ins.size() == 2 && P->ins[0] == x && P->ins[1] == x;
    if (P->op != "linalg.generic" || P->ins.empty() || P->ins[0] != x || P->outs.size() != 1) return false;
    if (!P->maps.empty() && !P->maps[0].is_identity()) return false;
    const EProgram& b = P->body;
    if (P->n_linalg_ins == 2) {  // powf(in, c) with c a scalar constant 2
      double f;
      int64_t i;
      if (!scalar_const(P->ins[1], f, i) || f != 2.0) return false;
      return b.code.size() == 1 && b.code[0].op == EOp::POWF && b.code[0].a == 0 && b.code[0].b == 1 &&
             b.result == b.code[0].dst;
    }
    if (P->n_linalg_ins != 1) return false;
    if (b.code.size() == 1 && b.code[0].op == EOp::MULF && b.code[0].a == 0 && b.code[0].b == 0)
      return b.result == b.code[0].dst;
    return b.code.size() == 2 && b.code[0].op == EOp::CONST && b.code[0].fimm == 2.0 && b.code[1].op == EOp::POWF &&
           b.code[1].a == 0 && b.code[1].b == b.code[0].dst && b.result == b.code[1].dst;
  }

  bool is_last_dim_mean(const Node* M) {
    if (!is_op(M, "gawee.reduce_mean") || M->ins.size() != 1) return false;
    const int rank = val(M->ins[0]).type.rank();
    const auto& ax = M->attr("axes").ints;
    const bool keep = !M->has_attr("keepDims") || M->attr("keepDims").b || M->attr("keepDims").i != 0;
    return keep && ax.size() == 1 && (ax[0] == -1 || ax[0] == rank - 1);
  }

  // w (or b) broadcasts over every dim of `shape` but the last
  bool per_column(int v, const std::vector<int64_t>& shape) {
    const auto& ws = val(v).type.shape;
    if (val(v).type.dtype != DType::F32 || ws.size() > shape.size()) return false;
    for (size_t d = 0; d + 1 < ws.size(); ++d)
      if (ws[d] != 1) return false;
    return ws.empty() || ws.back() == 1 || ws.back() == shape.back();
  }

  void find_norm_clusters() {
    Graph& g = plan_->g;
    for (size_t f = 0; f < g.nodes.size(); ++f) {
      const Node& F = g.nodes[f];
      if (F.op != "gawee.mul" || F.ins.size() != 2 || skip_node_.count((int)f)) continue;
      for (int side = 0; side < 2; ++side) {
        const int dv = F.ins[side], w = F.ins[1 - side];
        const Node* D = node_of(dv);
        if (!is_op(D, "gawee.div") || uses_[dv] != 1) continue;
        const int x = D->ins[0];
        const Node* Q = node_of(D->ins[1]);
        if (!is_op(Q, "gawee.sqrt") || uses_[D->ins[1]] != 1) continue;
        const Node* A = node_of(Q->ins[0]);
        if (!is_op(A, "gawee.add") || uses_[Q->ins[0]] != 1) continue;
        int mi = -1;
        double eps = 0;
        int64_t ei = 0;
        for (int k = 0; k < 2; ++k)
          if (is_last_dim_mean(node_of(A->ins[k])) && scalar_const(A->ins[1 - k], eps, ei)) mi = k;
        if (mi < 0 || uses_[A->ins[mi]] != 1) continue;
        const Node* M = node_of(A->ins[mi]);
        const Node* P = node_of(M->ins[0]);
        if (!is_square_of(P, x) || uses_[M->ins[0]] != 1) continue;
        const auto& xs = val(x).type.shape;
        if (val(x).type.dtype != DType::F32 || xs.empty() || val(F.outs[0]).type.shape != xs ||
            !per_column(w, xs))
          continue;
        NormMatch m;
        m.x = x;
        m.w = w;
        m.eps = eps;
        std::vector<int> skip = {def_node(dv), def_node(D->ins[1]), def_node(Q->ins[0]), def_node(A->ins[mi]),
                                 def_node(M->ins[0])};
        // LayerNorm: x = sub(x0, mean(x0)), used only by the square and the divide
        const Node* X = node_of(x);
        if (is_op(X, "gawee.sub") && uses_[x] == 2 && X->ins.size() == 2) {
          const Node* MU = node_of(X->ins[1]);
          if (is_last_dim_mean(MU) && MU->ins[0] == X->ins[0] && uses_[X->ins[1]] == 1 &&
              val(X->ins[0]).type.shape == xs) {
            m.centered = true;
            m.x0 = X->ins[0];
            skip.push_back(def_node(x));
            skip.push_back(def_node(X->ins[1]));
          }
        }
        // a trailing per-column add (LayerNorm's beta)
        int last = (int)f;
        m.out = F.outs[0];
        if (uses_[F.outs[0]] == 1) {
          for (size_t n2 = f + 1; n2 < g.nodes.size(); ++n2) {
            const Node& B = g.nodes[n2];
            if (B.op != "gawee.add" || B.ins.size() != 2) continue;
            const int k = B.ins[0] == F.outs[0] ? 0 : B.ins[1] == F.outs[0] ? 1 : -1;
            if (k < 0) continue;
            if (per_column(B.ins[1 - k], xs) && val(B.outs[0]).type.shape == xs) {
              m.b = B.ins[1 - k];
              m.out = B.outs[0];
              skip.push_back(last);
              last = (int)n2;
            }
            break;
          }
        }
        for (int sn : skip) skip_node_.insert(sn);
        norm_at_[last] = m;
        break;
      }
    }
  }

  void plan_rownorm(const NormMatch& m) {
    View x = value_view(m.centered ? m.x0 : m.x);
    const int r = x.rank();
    const int64_t cols = x.shape[r - 1], rows = x.numel() / std::max<int64_t>(cols, 1);
    // rows with one stride and contiguous columns, else a dense copy
    bool ok = x.st[r - 1] == 1 || cols == 1;
    int64_t x_rs = cols;
    if (ok && !x.dense_rowmajor()) {
      int64_t expect = -1;
      for (int d = r - 2; d >= 0 && ok; --d) {
        if (x.shape[d] == 1) continue;
        if (expect < 0) {
          x_rs = x.st[d];
          expect = x.st[d] * x.shape[d];
        } else if (x.st[d] != expect) {
          ok = false;
        } else {
          expect *= x.shape[d];
        }
      }
    }
    if (!ok) {
      x = copy_to_new(x, "rownorm_in");
      x_rs = cols;
    }
    View w = broadcast_to(value_view(m.w), x.shape);
    View b;
    if (m.b >= 0) b = broadcast_to(value_view(m.b), x.shape);
    View out = alloc(DType::F32, x.shape);
    Op op;
    op.kind = OpKind::REDUCE;
    op.name = m.centered ? "layer_norm" : "rms_norm";
    op.reads = {x, w};
    if (m.b >= 0) op.reads.push_back(b);
    op.writes = {out};
    op.launch = launch::rownorm(x, rows, cols, x_rs, w, w.st[r - 1], b, m.b >= 0 ? b.st[r - 1] : 0, out,
                                (float)m.eps, m.centered);
    add_op(std::move(op));
    set_view(m.out, out);
  }

  // ---------------------------------------------------------------- rotary embedding
  // add(mul(x, cos), mul(cat([neg(slice(x, d/2..d)), slice(x, 0..d/2)], -1), sin)), the rotate-half
  // form the emitter produces from Slice / Neg / Concat / Mul / Add (ONNXMLIREmitter.cpp:873-903,
  // 2074-2124; SliceOpLowering GaweeToLinalg.cpp:2594-2715, CatOpLowering 1260-1325).
  struct RopeMatch {
    int x = -1, cs = -1, sn = -1, out = -1;
  };
  std::map<int, RopeMatch> rope_at_;

  // the slice [start, start + len) of `data` along its last axis, step 1
  bool last_axis_slice(const Node* n, int data, int64_t start, int64_t len) {
    if (!is_op(n, "gawee.slice") || n->ins.size() < 5 || n->ins[0] != data) return false;
    const Value& v = val(data);
    const int r = v.type.rank();
    const Value& o = val(n->outs[0]);
    if (!val(n->ins[1]).is_const || !val(n->ins[3]).is_const || !val(n->ins[4]).is_const) return false;
    auto starts = const_ints(n->ins[1]), axes = const_ints(n->ins[3]), steps = const_ints(n->ins[4]);
    if (axes.size() != 1 || starts.size() != 1 || steps.size() != 1 || steps[0] != 1) return false;
    if (!(axes[0] == -1 || axes[0] == r - 1)) return false;
    int64_t st = starts[0] < 0 ? starts[0] + v.type.shape[r - 1] : starts[0];
    return st == start && o.type.shape.size() == (size_t)r && o.type.shape[r - 1] == len;
  }

  bool is_negation(const Node* n) {
    if (!n) return false;
    if (n->op == "gawee.neg") return n->ins.size() == 1;
    if (n->op != "linalg.generic" || n->n_linalg_ins != 1 || n->outs.size() != 1) return false;
    if (!n->maps.empty() && !n->maps[0].is_identity()) return false;
    const EProgram& b = n->body;
    return b.code.size() == 1 && b.code[0].op == EOp::NEGF && b.code[0].a == 0 && b.result == b.code[0].dst;
  }

  void find_rope_clusters() {
    Graph& g = plan_->g;
    for (size_t i = 0; i < g.nodes.size(); ++i) {
      const Node& R = g.nodes[i];
      if (R.op != "gawee.add" || R.ins.size() != 2 || skip_node_.count((int)i)) continue;
      const auto& os = val(R.outs[0]).type.shape;
      if (os.empty() || os.size() > 4 || os.back() % 2 || val(R.outs[0]).type.dtype != DType::F32) continue;
      const int64_t d = os.back(), half = d / 2;
      for (int k = 0; k < 2; ++k) {
        const Node* M1 = node_of(R.ins[k]);
        const Node* M2 = node_of(R.ins[1 - k]);
        if (!is_op(M1, "gawee.mul") || !is_op(M2, "gawee.mul") || uses_[R.ins[k]] != 1 || uses_[R.ins[1 - k]] != 1)
          continue;
        // M2 = rotate_half(x) * sin
        int rhi = -1;
        for (int j = 0; j < 2; ++j)
          if (is_op(node_of(M2->ins[j]), "gawee.cat")) rhi = j;
        if (rhi < 0 || uses_[M2->ins[rhi]] != 1) continue;
        const Node* C = node_of(M2->ins[rhi]);
        int64_t ax = C->attr("axis").i;
        if (ax < 0) ax += (int64_t)os.size();
        if (C->ins.size() != 2 || ax != (int64_t)os.size() - 1) continue;
        const Node* N = node_of(C->ins[0]);
        if (!is_negation(N) || uses_[C->ins[0]] != 1 || uses_[C->ins[1]] != 1 || uses_[N->ins[0]] != 1) continue;
        const Node* S2 = node_of(N->ins[0]);
        const Node* S1 = node_of(C->ins[1]);
        if (!S2 || !S1) continue;
        const int x = S2->ins[0];
        if (!last_axis_slice(S2, x, half, half) || !last_axis_slice(S1, x, 0, half)) continue;
        // M1 = x * cos
        int xi = -1;
        for (int j = 0; j < 2; ++j)
          if (M1->ins[j] == x) xi = j;
        if (xi < 0 || val(x).type.shape != os) continue;
        const int cs = M1->ins[1 - xi], sn = M2->ins[1 - rhi];
        auto bcast_ok = [&](int v) {
          const auto& vs = val(v).type.shape;
          if (val(v).type.dtype != DType::F32 || vs.size() > os.size()) return false;
          for (size_t q = 0; q < vs.size(); ++q)
            if (vs[vs.size() - 1 - q] != 1 && vs[vs.size() - 1 - q] != os[os.size() - 1 - q]) return false;
          return true;
        };
        if (!bcast_ok(cs) || !bcast_ok(sn)) continue;
        RopeMatch m{x, cs, sn, R.outs[0]};
        for (int sn2 : {def_node(R.ins[k]), def_node(R.ins[1 - k]), def_node(M2->ins[rhi]), def_node(C->ins[0]),
                        def_node(N->ins[0]), def_node(C->ins[1])})
          skip_node_.insert(sn2);
        rope_at_[(int)i] = m;
        break;
      }
    }
  }

  void plan_rope(const RopeMatch& m) {
    const auto& os = val(m.out).type.shape;
    View x = value_view(m.x);
    View cs = broadcast_to(value_view(m.cs), os);
    View sn = broadcast_to(value_view(m.sn), os);
    View out = alloc(DType::F32, os);
    Op op;
    op.kind = OpKind::REMAP;
    op.name = "rope";
    op.reads = {x, cs, sn};
    op.writes = {out};
    op.launch = launch::rope(x, cs, sn, out);
    add_op(std::move(op));
    set_view(m.out, out);
  }

  void plan_attention(const AttnMatch& m) {
    View q = value_view(m.q);
    View k, v;
    if (m.k_base >= 0) {
      k = value_view(m.k_base);
    } else {  // K^T [B, H, D, Skv] -> K [B, H, Skv, D]
      View kt = value_view(m.kt);
      k = kt;
      std::swap(k.shape[2], k.shape[3]);
      std::swap(k.st[2], k.st[3]);
    }
    v = value_view(m.v_base >= 0 ? m.v_base : m.v);
    const int64_t B = q.shape[0], H = q.shape[1], S = q.shape[2], D = q.shape[3], Skv = k.shape[2];
    auto dense_inner = [](View& x) {  // d contiguous; strides of size-1 dims are never stepped
      return x.st[3] == 1 || x.shape[3] == 1;
    };
    if (!dense_inner(q)) q = copy_to_new(q, "attn_q_copy");
    if (!dense_inner(k)) k = copy_to_new(k, "attn_k_copy");
    if (!dense_inner(v)) v = copy_to_new(v, "attn_v_copy");
    Op op;
    op.kind = OpKind::ATTN;
    op.name = "attention";
    auto& a = op.attn;
    a.q = q;
    a.k = k;
    a.v = v;
    a.B = B; a.H = H; a.Hkv = k.shape[1]; a.S = S; a.Skv = Skv; a.D = D;
    a.c = m.c;
    a.has_mask = m.mask >= 0;
    if (a.has_mask) a.mask = broadcast_to(value_view(m.mask), {B, H, S, Skv});
    a.flops = 4.0 * (double)B * (double)H * (double)S * (double)Skv * (double)D;
    View out;
    if (m.out_transpose >= 0) {
      out = alloc(DType::F32, {B, S, H, D});  // dense [B, S, H, D], seen as [B, H, S, D]
      std::swap(out.shape[1], out.shape[2]);
      std::swap(out.st[1], out.st[2]);
    } else {
      out = alloc(DType::F32, {B, H, S, D});
    }
    a.out = out;
    op.reads = {q, k, v};
    if (a.has_mask) op.reads.push_back(a.mask);
    op.writes = {out};
    add_op(std::move(op));
    set_view(m.pv_out, out);
  }

  // ---------------------------------------------------------------- buffers / views
  int new_buf(DType dt, int64_t elems, BufKind kind = BufKind::ARENA) {
    Buf b;
    b.kind = kind;
    b.dt = dt;
    b.elems = std::max<int64_t>(elems, 1);
    plan_->bufs.push_back(b);
    return (int)plan_->bufs.size() - 1;
  }

  View dense_view(int buf, DType dt, const std::vector<int64_t>& shape) {
    View v;
    v.buf = buf;
    v.dt = dt;
    v.shape = shape;
    v.st = rowmajor_strides(shape);
    return v;
  }

  View alloc(DType dt, const std::vector<int64_t>& shape, const std::vector<int>& order = {}) {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    int b = new_buf(dt, n);
    View v;
    v.buf = b;
    v.dt = dt;
    v.shape = shape;
    if (order.empty()) v.st = rowmajor_strides(shape);
    else v.st = strides_in_order(shape, order);
    return v;
  }

  void set_view(int value, const View& v) {
    plan_->value_view[value] = v;
    has_view_[value] = true;
  }

  View value_view(int value) {
    if (has_view_[value]) return plan_->value_view[value];
    const Value& gv = plan_->g.values[value];
    if (gv.is_const) {
      int b = new_buf(gv.type.dtype, gv.type.is_tensor ? gv.type.numel() : 1, BufKind::CONST);
      plan_->bufs[b].const_value = value;
      View v = dense_view(b, gv.type.dtype, gv.type.is_tensor ? gv.type.shape : std::vector<int64_t>{});
      set_view(value, v);
      return v;
    }
    throw std::runtime_error("value " + gv.name + " has no producer");
  }

  const Value& val(int id) const { return plan_->g.values[id]; }

  // Scalar payload of a constant with one element, if any.
  bool scalar_const(int value, double& f, int64_t& i) {
    const Value& v = val(value);
    if (!v.is_const) return false;
    if (v.type.is_tensor && v.type.numel() != 1) return false;
    f = const_as_double(v, 0);
    i = const_as_int(v, 0);
    return true;
  }

  std::vector<int64_t> const_ints(int value) {
    const Value& v = val(value);
    if (!v.is_const) unsupported("expected a constant integer tensor operand (" + v.name + ")");
    std::vector<int64_t> out;
    int64_t n = v.type.is_tensor ? v.type.numel() : 1;
    for (int64_t k = 0; k < n; ++k) out.push_back(const_as_int(v, k));
    return out;
  }

  // numpy/buildBroadcastMap broadcast of a view to `out` (GaweeToLinalg.cpp:123-144)
  View broadcast_to(const View& v, const std::vector<int64_t>& out) {
    View r = v;
    r.shape = out;
    r.st.assign(out.size(), 0);
    int lead = (int)out.size() - v.rank();
    if (lead < 0) unsupported("broadcast of a higher-rank operand");
    for (int i = 0; i < v.rank(); ++i) {
      int od = lead + i;
      if (v.shape[i] == 1 && out[od] != 1) r.st[od] = 0;
      else {
        if (v.shape[i] != out[od]) unsupported("incompatible broadcast");
        r.st[od] = v.st[i];
      }
    }
    return r;
  }

  // dims order for an elementwise output: follow the first input that spans the
  // whole output (non-zero strides on every non-unit dim), else row-major
  std::vector<int> layout_like(const std::vector<View>& ins, const std::vector<int64_t>& out_shape) {
    std::vector<int> order(out_shape.size());
    std::iota(order.begin(), order.end(), 0);
    for (const View& v : ins) {
      bool full = true;
      for (size_t d = 0; d < out_shape.size(); ++d)
        if (out_shape[d] != 1 && v.st[d] == 0) full = false;
      if (!full) continue;
      std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
        if (out_shape[a] == 1 || out_shape[b] == 1) return false;
        return v.st[a] > v.st[b];
      });
      return order;
    }
    return order;
  }

  // ---------------------------------------------------------------- op creation
  int add_op(Op op) {
    for (const View& w : op.writes)
      if (plan_->bufs[w.buf].producer < 0) plan_->bufs[w.buf].producer = (int)plan_->ops.size();
    plan_->ops.push_back(std::move(op));
    return (int)plan_->ops.size() - 1;
  }

  // Drop argument registers no instruction reads (e.g. a linalg.generic `outs`
  // operand whose block argument is unused).
  static EProgram prune_args(const EProgram& p, std::vector<View>& ins) {
    std::vector<char> used(p.reg_types.size(), 0);
    for (const EInstr& in : p.code) {
      if (in.a >= 0) used[in.a] = 1;
      if (in.b >= 0) used[in.b] = 1;
      if (in.c >= 0) used[in.c] = 1;
    }
    if (p.result >= 0) used[p.result] = 1;
    EProgram q;
    std::vector<int> map(p.reg_types.size(), -1);
    std::vector<View> kept;
    for (int a = 0; a < p.n_args; ++a) {
      if (!used[a]) continue;
      map[a] = q.add_reg(p.reg_types[a]);
      kept.push_back(ins[a]);
    }
    q.n_args = (int)q.reg_types.size();
    for (const EInstr& in0 : p.code) {
      EInstr in = in0;
      if (in.a >= 0) in.a = (int16_t)map[in.a];
      if (in.b >= 0) in.b = (int16_t)map[in.b];
      if (in.c >= 0) in.c = (int16_t)map[in.c];
      in.dst = (int16_t)q.add_reg(p.reg_types[in0.dst]);
      map[in0.dst] = in.dst;
      q.code.push_back(in);
    }
    q.result = map[p.result];
    ins = kept;
    return q;
  }

  // Elementwise op writing `out` from `ins` (views over out's shape).
  int add_ew(const std::string& name, const View& out, std::vector<View> ins, EProgram prog) {
    if ((int)ins.size() != prog.n_args) throw std::runtime_error("internal: operand count != program arguments");
    prog = prune_args(prog, ins);
    // inline scalar constants as immediates
    for (int k = (int)ins.size() - 1; k >= 0; --k) {
      const Buf& b = plan_->bufs[ins[k].buf];
      if (b.kind != BufKind::CONST || b.const_value < 0) continue;
      const Value& cv = val(b.const_value);
      int64_t cnt = cv.type.is_tensor ? cv.type.numel() : 1;
      if (cnt != 1) continue;
      EInstr c;
      c.op = EOp::CONST;
      c.ty = c.rty = cv.type.dtype;
      c.fimm = const_as_double(cv, 0);
      c.iimm = const_as_int(cv, 0);
      prog = substitute_arg(prog, k, c);
      ins.erase(ins.begin() + k);
    }
    Op op;
    op.kind = OpKind::EW;
    op.name = name;
    op.out = out;
    op.ins = ins;
    op.prog = prog;
    op.reads = ins;
    op.writes = {out};
    return add_op(std::move(op));
  }

  // Replace argument register `k` of a program by an instruction computing it.
  static EProgram substitute_arg(const EProgram& p, int k, EInstr def) {
    EProgram q;
    // new args: old args without k
    std::vector<int> map(p.reg_types.size(), -1);
    for (int a = 0; a < p.n_args; ++a) {
      if (a == k) continue;
      map[a] = q.add_reg(p.reg_types[a]);
    }
    q.n_args = p.n_args - 1;
    def.dst = (int16_t)q.add_reg(p.reg_types[k]);
    map[k] = def.dst;
    q.code.push_back(def);
    for (const EInstr& in0 : p.code) {
      EInstr in = in0;
      if (in.a >= 0) in.a = (int16_t)map[in.a];
      if (in.b >= 0) in.b = (int16_t)map[in.b];
      if (in.c >= 0) in.c = (int16_t)map[in.c];
      in.dst = (int16_t)q.add_reg(p.reg_types[in0.dst]);
      map[in0.dst] = in.dst;
      q.code.push_back(in);
    }
    q.result = map[p.result];
    return q;
  }

  View copy_to_new(const View& src, const std::string& name, const std::vector<int>& order = {}) {
    View out = alloc(src.dt, src.shape, order);
    PB pb({src.dt});
    add_ew(name, out, {src}, pb.done(0));
    return out;
  }

  // ---------------------------------------------------------------- view ops
  // Reshape without copying when strides allow (merge/split of compatible dims).
  bool reshape_view(const View& v, const std::vector<int64_t>& ns, View& out) {
    out = v;
    out.shape = ns;
    // drop size-1 dims of the source
    std::vector<int64_t> os, ost;
    for (int i = 0; i < v.rank(); ++i)
      if (v.shape[i] != 1) { os.push_back(v.shape[i]); ost.push_back(v.st[i]); }
    std::vector<int64_t> nst(ns.size(), 0);
    size_t oi = 0;
    size_t ni = 0;
    while (ni < ns.size()) {
      if (ns[ni] == 1) { nst[ni] = 1; ++ni; continue; }
      if (oi >= os.size()) return false;
      // group: accumulate old dims until products match
      int64_t op = os[oi], np = ns[ni];
      size_t ob = oi, nb = ni;
      while (op != np) {
        if (op < np) { if (++oi >= os.size()) return false; op *= os[oi]; }
        else {
          do { if (++ni >= ns.size()) return false; } while (ns[ni] == 1 && false);
          np *= ns[ni];
        }
      }
      // old dims ob..oi must be mergeable (contiguous with each other)
      for (size_t k = ob; k < oi; ++k)
        if (ost[k] != ost[k + 1] * os[k + 1]) return false;
      // assign new strides inner to outer within the group
      int64_t acc = ost[oi];
      for (size_t k = ni + 1; k-- > nb;) {
        nst[k] = ns[k] == 1 ? acc : acc;
        acc *= ns[k];
      }
      ++oi;
      ++ni;
    }
    if (oi != os.size()) return false;
    out.st = nst;
    return true;
  }

  View reshape(const View& v, const std::vector<int64_t>& ns) {
    int64_t n = 1;
    for (auto d : ns) n *= d;
    if (n != v.numel()) unsupported("reshape changes the element count");
    View out;
    if (reshape_view(v, ns, out)) return out;
    View c = copy_to_new(v, "reshape_copy");
    return dense_view_like(c, ns);
  }

  View dense_view_like(const View& c, const std::vector<int64_t>& ns) {
    View r = c;
    r.shape = ns;
    r.st = rowmajor_strides(ns);
    return r;
  }

  // ---------------------------------------------------------------- node planning
  void plan_node(const Node& n) {
    const std::string& op = n.op;
    if (op == "tensor.empty") {
      const Value& o = val(n.outs[0]);
      set_view(n.outs[0], alloc(o.type.dtype, o.type.shape));
      return;
    }
    if (op == "linalg.fill") return plan_fill(n);
    if (op == "linalg.generic") return plan_generic(n);
    if (op == "linalg.reduce") return plan_linalg_reduce(n);
    if (op.rfind("gawee.", 0) != 0) unsupported("op " + op);
    const std::string k = op.substr(6);
    if (k == "add" || k == "sub" || k == "mul" || k == "div" || k == "equal") return plan_binary(n, k);
    if (k == "relu" || k == "sigmoid" || k == "gelu" || k == "erf" || k == "sqrt" || k == "tanh" ||
        k == "hard_sigmoid" || k == "hard_swish" || k == "leaky_relu")
      return plan_unary(n, k);
    if (k == "where") return plan_where(n);
    if (k == "max" || k == "min") return plan_maxmin(n, k == "max");
    if (k == "cast") return plan_cast(n);
    if (k == "batch_norm") return plan_batch_norm(n);
    if (k == "expand") {
      View v = value_view(n.ins[0]);
      set_view(n.outs[0], broadcast_to(v, val(n.outs[0]).type.shape));
      return;
    }
    if (k == "reshape" || k == "flatten" || k == "squeeze" || k == "unsqueeze") {
      set_view(n.outs[0], reshape(value_view(n.ins[0]), val(n.outs[0]).type.shape));
      return;
    }
    if (k == "transpose") {
      View v = value_view(n.ins[0]);
      auto perm = n.attr("perm").ints;
      View r = v;
      for (size_t d = 0; d < perm.size(); ++d) {
        r.shape[d] = v.shape[perm[d]];
        r.st[d] = v.st[perm[d]];
      }
      set_view(n.outs[0], r);
      return;
    }
    if (k == "slice") return plan_slice(n);
    if (k == "split") return plan_split(n);
    if (k == "cat") return plan_cat(n);
    if (k == "conv") return plan_conv(n);
    if (k == "linear") return plan_linear(n);
    if (k == "matmul") return plan_matmul(n);
    if (k == "reduce_mean" || k == "reduce_sum") return plan_reduce(n, k == "reduce_mean");
    if (k == "global_average_pool" || k == "ad_avg_pool") return plan_global_avg(n);
    if (k == "max_pool" || k == "average_pool") return plan_pool(n, k == "max_pool");
    if (k == "softmax") return plan_softmax(n);
    if (k == "gather") return plan_gather(n);
    if (k == "gather_elements") return plan_gather_elements(n);
    if (k == "range") return plan_range(n);
    if (k == "shape") return plan_shape(n);
    if (k == "tile" || k == "pad" || k == "resize") return plan_remap(n, k);
    if (k == "topk") return plan_topk(n);
    unsupported("gawee op " + k);
  }

  void plan_fill(const Node& n) {
    double f;
    int64_t i;
    if (!scalar_const(n.ins[0], f, i)) unsupported("linalg.fill with a non-constant value");
    const Value& o = val(n.outs[0]);
    View out = alloc(o.type.dtype, o.type.shape);
    PB pb({});
    int r = is_float(o.type.dtype) ? pb.cf(f, o.type.dtype) : pb.ci(i, o.type.dtype);
    add_ew("fill", out, {}, pb.done(r));
    set_view(n.outs[0], out);
  }

  void plan_generic(const Node& n) {
    for (bool p : n.parallel)
      if (!p) unsupported("linalg.generic with reduction iterators");
    if (n.outs.size() != 1) unsupported("linalg.generic with several results");
    const Value& o = val(n.outs[0]);
    const auto& out_shape = o.type.shape;
    if (!n.maps.back().is_identity()) unsupported("linalg.generic with a non-identity output map");
    std::vector<View> ins;
    for (size_t a = 0; a < n.ins.size(); ++a) {
      View v = value_view(n.ins[a]);
      const AffineMapIR& m = n.maps[a];
      View r = v;
      r.shape = out_shape;
      r.st.assign(out_shape.size(), 0);
      for (size_t e = 0; e < m.exprs.size(); ++e) {
        if (m.exprs[e] >= 0) r.st[m.exprs[e]] += v.st[e];
        else r.off += (-1 - m.exprs[e]) * v.st[e];
      }
      ins.push_back(r);
    }
    View out = alloc(o.type.dtype, out_shape, layout_like(ins, out_shape));
    add_ew("generic", out, ins, n.body);
    set_view(n.outs[0], out);
  }

  void plan_linalg_reduce(const Node& n) {
    View in = value_view(n.ins[0]);
    View init = value_view(n.ins[1]);
    const Value& o = val(n.outs[0]);
    View out = alloc(o.type.dtype, o.type.shape);
    PB pb({init.dt});
    add_ew("reduce_init", out, {init}, pb.done(0));
    std::vector<bool> red(in.rank(), false);
    for (auto d : n.dims) red[d] = true;
    Op op;
    op.kind = OpKind::GREDUCE;
    op.name = "linalg_reduce";
    op.reads = {in, out};
    op.writes = {out};
    op.launch = launch::generic_reduce(in, out, red, n.body);
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  void plan_binary(const Node& n, const std::string& k) {
    View a = value_view(n.ins[0]), b = value_view(n.ins[1]);
    const Value& o = val(n.outs[0]);
    auto shape = o.type.shape;
    View ba = broadcast_to(a, shape), bb = broadcast_to(b, shape);
    DType t = a.dt;
    PB pb({a.dt, b.dt});
    int r;
    bool f = is_float(t);
    if (k == "add") r = pb.op(f ? EOp::ADDF : EOp::ADDI, t, 0, 1);
    else if (k == "sub") r = pb.op(f ? EOp::SUBF : EOp::SUBI, t, 0, 1);
    else if (k == "mul") r = pb.op(f ? EOp::MULF : EOp::MULI, t, 0, 1);
    else if (k == "div") r = pb.op(f ? EOp::DIVF : EOp::DIVSI, t, 0, 1);
    else r = pb.op(f ? EOp::CMPF : EOp::CMPI, t, 0, 1, -1, DType::I1, f ? CF_OEQ : CI_EQ);
    View out = alloc(o.type.dtype, shape, layout_like({ba, bb}, shape));
    add_ew(k, out, {ba, bb}, pb.done(r));
    set_view(n.outs[0], out);
  }

  void plan_unary(const Node& n, const std::string& k) {
    View a = value_view(n.ins[0]);
    const Value& o = val(n.outs[0]);
    if (a.dt != DType::F32) unsupported(k + " on non-f32 input");
    const DType F = DType::F32;
    PB pb({F});
    int r;
    if (k == "relu") r = pb.op(EOp::MAXIMUMF, F, 0, pb.cf(0.0));  // GaweeToLinalg.cpp:513-514
    else if (k == "sigmoid") {  // 1 / (1 + exp(-x)), GaweeToLinalg.cpp:1976-1981
      int one = pb.cf(1.0);
      int e = pb.op(EOp::EXP, F, pb.op(EOp::NEGF, F, 0));
      r = pb.op(EOp::DIVF, F, one, pb.op(EOp::ADDF, F, one, e));
    } else if (k == "gelu") {  // 0.5 * (x * (1 + erf(x / sqrt2))), GaweeToLinalg.cpp:2128-2139
      int d = pb.op(EOp::DIVF, F, 0, pb.cf((float)1.4142135623730951));
      int e = pb.op(EOp::ERF, F, d);
      int plus = pb.op(EOp::ADDF, F, pb.cf(1.0), e);
      int sc = pb.op(EOp::MULF, F, 0, plus);
      r = pb.op(EOp::MULF, F, pb.cf(0.5), sc);
    } else if (k == "erf") r = pb.op(EOp::ERF, F, 0);
    else if (k == "sqrt") r = pb.op(EOp::SQRT, F, 0);
    else if (k == "tanh") r = pb.op(EOp::TANH, F, 0);
    else if (k == "hard_sigmoid") {  // GaweeToLinalg.cpp:2000-2030
      int s = pb.op(EOp::MULF, F, 0, pb.cf((float)n.attr("alpha").f));
      int sh = pb.op(EOp::ADDF, F, s, pb.cf((float)n.attr("beta").f));
      r = pb.op(EOp::MINIMUMF, F, pb.op(EOp::MAXIMUMF, F, sh, pb.cf(0.0)), pb.cf(1.0));
    } else if (k == "hard_swish") {  // GaweeToLinalg.cpp:2041-2056
      int sh = pb.op(EOp::ADDF, F, 0, pb.cf(3.0));
      int hi = pb.op(EOp::MINIMUMF, F, pb.op(EOp::MAXIMUMF, F, sh, pb.cf(0.0)), pb.cf(6.0));
      r = pb.op(EOp::DIVF, F, pb.op(EOp::MULF, F, 0, hi), pb.cf(6.0));
    } else {  // leaky_relu, GaweeToLinalg.cpp:2079-2090
      int s = pb.op(EOp::MULF, F, 0, pb.cf((float)n.attr("alpha").f));
      int m = pb.op(EOp::MAXIMUMF, F, 0, s);
      int neg = pb.op(EOp::CMPF, F, 0, pb.cf(0.0), -1, DType::I1, CF_OLT);
      r = pb.op(EOp::SELECT, F, neg, s, m);
    }
    View out = alloc(o.type.dtype, o.type.shape, layout_like({a}, o.type.shape));
    add_ew(k, out, {a}, pb.done(r));
    set_view(n.outs[0], out);
  }

  void plan_where(const Node& n) {  // GaweeToLinalg.cpp:2213-2248
    const Value& o = val(n.outs[0]);
    auto shape = o.type.shape;
    View c = broadcast_to(value_view(n.ins[0]), shape);
    View a = broadcast_to(value_view(n.ins[1]), shape);
    View b = broadcast_to(value_view(n.ins[2]), shape);
    PB pb({c.dt, a.dt, b.dt});
    int r = pb.op(EOp::SELECT, a.dt, 0, 1, 2);
    View out = alloc(o.type.dtype, shape, layout_like({a, b, c}, shape));
    add_ew("where", out, {c, a, b}, pb.done(r));
    set_view(n.outs[0], out);
  }

  void plan_maxmin(const Node& n, bool is_max) {  // GaweeToLinalg.cpp:2250-2292
    const Value& o = val(n.outs[0]);
    auto shape = o.type.shape;
    std::vector<View> ins;
    std::vector<DType> tys;
    for (int v : n.ins) {
      ins.push_back(broadcast_to(value_view(v), shape));
      tys.push_back(ins.back().dt);
    }
    PB pb(tys);
    DType t = o.type.dtype;
    int cur = 0;
    for (size_t k = 1; k < ins.size(); ++k)
      cur = pb.op(is_float(t) ? (is_max ? EOp::MAXIMUMF : EOp::MINIMUMF) : (is_max ? EOp::MAXSI : EOp::MINSI), t, cur,
                  (int)k);
    if (ins.size() == 1) cur = pb.op(EOp::COPY, t, 0);
    View out = alloc(t, shape, layout_like(ins, shape));
    add_ew(is_max ? "max" : "min", out, ins, pb.done(cur));
    set_view(n.outs[0], out);
  }

  void plan_cast(const Node& n) {  // GaweeToLinalg.cpp:2799-2863
    View a = value_view(n.ins[0]);
    const Value& o = val(n.outs[0]);
    DType s = a.dt, d = o.type.dtype;
    if (s == d) {
      set_view(n.outs[0], a);
      return;
    }
    PB pb({s});
    int r;
    if (is_float(s) && is_float(d)) r = pb.op(dtype_size(d) > dtype_size(s) ? EOp::EXTF : EOp::TRUNCF, s, 0, -1, -1, d);
    else if (!is_float(s) && is_float(d)) r = pb.op(s == DType::I1 ? EOp::UITOFP : EOp::SITOFP, s, 0, -1, -1, d);
    else if (is_float(s) && !is_float(d)) r = pb.op(EOp::FPTOSI, s, 0, -1, -1, d);
    else {
      size_t ws = s == DType::I1 ? 0 : dtype_size(s), wd = d == DType::I1 ? 0 : dtype_size(d);
      r = pb.op(wd > ws ? EOp::EXTSI : (wd < ws ? EOp::TRUNCI : EOp::COPY), s, 0, -1, -1, d);
    }
    View out = alloc(d, o.type.shape, layout_like({a}, o.type.shape));
    add_ew("cast", out, {a}, pb.done(r));
    set_view(n.outs[0], out);
  }

  void plan_batch_norm(const Node& n) {  // GaweeToLinalg.cpp:1122-1173
    View x = value_view(n.ins[0]);
    const Value& o = val(n.outs[0]);
    if (x.rank() != 4) unsupported("batch_norm on a non-4D tensor");
    auto chan = [&](int v) {
      View c = value_view(v);
      View r = c;
      r.shape = x.shape;
      r.st = {0, c.st[0], 0, 0};
      return r;
    };
    View w = chan(n.ins[1]), b = chan(n.ins[2]), mean = chan(n.ins[3]), var = chan(n.ins[4]);
    const DType F = DType::F32;
    PB pb({F, F, F, F, F});
    int denom = pb.op(EOp::SQRT, F, pb.op(EOp::ADDF, F, 4, pb.cf((float)n.attr("eps").f)));
    int normd = pb.op(EOp::DIVF, F, pb.op(EOp::SUBF, F, 0, 3), denom);
    int r = pb.op(EOp::ADDF, F, pb.op(EOp::MULF, F, normd, 1), 2);
    View out = alloc(F, o.type.shape, layout_like({x}, o.type.shape));
    add_ew("batch_norm", out, {x, w, b, mean, var}, pb.done(r));
    set_view(n.outs[0], out);
  }

  void plan_slice(const Node& n) {  // GaweeToLinalg.cpp:2594-2715
    View v = value_view(n.ins[0]);
    const Value& o = val(n.outs[0]);
    auto starts = const_ints(n.ins[1]);
    auto axes = const_ints(n.ins[3]);
    auto steps = const_ints(n.ins[4]);
    View r = v;
    r.shape = o.type.shape;
    for (size_t k = 0; k < axes.size(); ++k) {
      int64_t ax = axes[k] < 0 ? axes[k] + v.rank() : axes[k];
      if (steps[k] <= 0) unsupported("slice with non-positive step");
      int64_t s = starts[k];
      if (s < 0) s += v.shape[ax];
      if (s < 0 || (r.shape[ax] > 0 && s + (r.shape[ax] - 1) * steps[k] >= v.shape[ax]))
        throw std::runtime_error("slice reads outside its input");
      r.off += s * v.st[ax];
      r.st[ax] = v.st[ax] * steps[k];
    }
    set_view(n.outs[0], r);
  }

  void plan_split(const Node& n) {  // GaweeToLinalg.cpp:2554-2592
    View v = value_view(n.ins[0]);
    int64_t ax = n.attr("axis").i;
    if (ax < 0) ax += v.rank();
    int64_t base = 0;
    for (size_t k = 0; k < n.outs.size(); ++k) {
      View r = v;
      r.shape = val(n.outs[k]).type.shape;
      r.off += base * v.st[ax];
      base += r.shape[ax];
      set_view(n.outs[k], r);
    }
  }

  void plan_cat(const Node& n) {  // GaweeToLinalg.cpp:1260-1325
    const Value& o = val(n.outs[0]);
    int64_t ax = n.attr("axis").i;
    if (ax < 0) ax += (int64_t)o.type.shape.size();
    View out = alloc(o.type.dtype, o.type.shape);
    int64_t base = 0;
    for (int v : n.ins) {
      View src = value_view(v);
      View dst = out;
      dst.shape = src.shape;
      dst.off += base * out.st[ax];
      base += src.shape[ax];
      PB pb({src.dt});
      add_ew("cat_copy", dst, {src}, pb.done(0));
    }
    set_view(n.outs[0], out);
  }

  // ---------------------------------------------------------------- contractions
  std::pair<int, int> add_pack(const PackSpec& ps, int64_t ldk, const std::string& name) {
    int hi = new_buf(DType::F32, ps.batch * ps.N * ldk);
    int lo = new_buf(DType::F32, ps.batch * ps.N * ldk);
    Op op;
    op.kind = OpKind::PACK;
    op.name = name;
    op.reads = {ps.src};
    View vh = dense_view(hi, DType::F32, {ps.batch * ps.N * ldk});
    View vl = dense_view(lo, DType::F32, {ps.batch * ps.N * ldk});
    op.writes = {vh, vl};
    op.launch = launch::pack(ps, ldk, hi, lo);
    add_op(std::move(op));
    return {hi, lo};
  }

  static int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

  static int pick_block_n(int64_t N) { return N <= 64 ? 64 : 128; }

  void plan_conv(const Node& n) {  // GaweeToLinalg.cpp:322-455
    View x = value_view(n.ins[0]);
    View w = value_view(n.ins[1]);
    View bias = value_view(n.ins[2]);
    const Value& o = val(n.outs[0]);
    if (x.rank() != 4 || w.rank() != 4) unsupported("conv expects NCHW input and FCHW weight");
    auto st = n.attr("strides").ints, pd = n.attr("padding").ints, dl = n.attr("dilation").ints;
    if (st.size() < 2 || pd.size() < 2 || dl.size() < 2) unsupported("conv attributes");
    int64_t N = x.shape[0], C = x.shape[1], H = x.shape[2], W = x.shape[3];
    int64_t F = w.shape[0], R = w.shape[2], S = w.shape[3];
    if (w.shape[1] != C) unsupported("grouped convolution");
    int64_t P = o.type.shape[2], Q = o.type.shape[3];
    int64_t C4 = round_up(C, 4);
    // input must be NHWC with unit channel stride, channels a multiple of 4
    bool nhwc = C == C4 && x.st[1] == 1 && x.st[3] == C && x.st[2] == W * C && x.st[0] == H * W * C &&
                (x.off % 4) == 0;
    View xin = x;
    if (!nhwc) {
      // NCHW (or any) -> NHWC with the channel dim zero-padded to a multiple of 4
      View out = alloc(DType::F32, {N, C4, H, W}, {0, 2, 3, 1});
      Op op;
      op.kind = OpKind::REMAP;
      op.name = "to_nhwc";
      op.reads = {x};
      op.writes = {out};
      if (x.dt == DType::F32 && x.st[3] == 1 && x.st[2] == W) {  // NCHW planes: pixel-vectorised kernel
        op.launch = launch::nchw_to_nhwc4(x, out, N, (int)C, (int)C4, H * W, N > 1 ? x.st[0] : 0, x.st[1]);
        add_op(std::move(op));
        xin = out;
        goto packed;
      }
      kern::RemapParams rp{};
      rp.elem_bytes = 4;
      rp.rank = 4;
      rp.numel = N * C4 * H * W;
      int perm[4] = {0, 2, 3, 1};  // iterate in NHWC order for coalesced writes
      for (int d = 0; d < 4; ++d) {
        int s = perm[d];
        rp.out_shape[d] = out.shape[s];
        rp.out_st[d] = out.st[s];
        rp.in_shape[d] = x.shape[s];
        rp.in_st[d] = x.st[s];
        rp.div[d] = 1;
        rp.mod[d] = std::numeric_limits<int64_t>::max();
        rp.sub[d] = 0;
      }
      rp.fill_bits = 0;
      op.launch = launch::remap(rp, x, out);
      add_op(std::move(op));
      xin = out;
    }
  packed:
    PackSpec ps;
    ps.src = w;
    ps.batch = 1;
    ps.K = R * S * C4;
    ps.N = F;
    ps.sn = w.st[0];
    ps.k_shape = {R, S, C4};
    ps.k_st = {w.st[2], w.st[3], w.st[1]};
    ps.k_valid = {R, S, C};
    int64_t ldk = round_up(ps.K, 4);
    auto hl = add_pack(ps, ldk, "pack_conv_w");
    View out = alloc(DType::F32, o.type.shape, {0, 2, 3, 1});
    Op op;
    op.kind = OpKind::TC;
    op.name = "conv";
    auto& t = op.tc;
    t.conv = true;
    t.x = xin;
    t.out = out;
    t.hi = hl.first;
    t.lo = hl.second;
    t.b_batch = 1;
    t.ldk = ldk;
    t.H = H; t.W = W; t.C = C4; t.P = P; t.Q = Q;
    t.R = (int)R; t.S = (int)S;
    t.sh = (int)st[0]; t.sw = (int)st[1];
    t.ph = (int)pd[0]; t.pw = (int)pd[1];
    t.dh = (int)dl[0]; t.dw = (int)dl[1];
    t.M = N * P * Q;
    t.N = F;
    t.K = R * S * C4;
    t.block_n = pick_block_n(F);
    t.epi = kern::EPI_BIAS;
    t.bias = bias;
    t.flops = 2.0 * (double)(N * P * Q) * (double)F * (double)(R * S * C);
    op.reads = {xin, dense_view(hl.first, DType::F32, {1}), dense_view(hl.second, DType::F32, {1}), bias};
    op.writes = {out};
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  // A operand of a GEMM: rows with unit k stride and 16-byte aligned rows.
  View gemm_operand_a(const View& a) {
    int r = a.rank();
    int64_t K = a.shape[r - 1];
    bool ok = a.dt == DType::F32 && (a.st[r - 1] == 1 || K == 1) && K % 4 == 0 && a.off % 4 == 0;
    for (int d = 0; d < r - 1 && ok; ++d)
      if (a.shape[d] != 1 && a.st[d] % 4 != 0) ok = false;
    if (ok) return a;
    if (K % 4 == 0) return copy_to_new(a, "gemm_a_copy");
    // pad K to a multiple of 4 with zeros
    std::vector<int64_t> ps = a.shape;
    ps[r - 1] = round_up(K, 4);
    View out = alloc(DType::F32, ps);
    Op op;
    op.kind = OpKind::REMAP;
    op.name = "gemm_a_pad";
    op.reads = {a};
    op.writes = {out};
    kern::RemapParams rp{};
    rp.elem_bytes = 4;
    rp.rank = r;
    rp.numel = out.numel();
    for (int d = 0; d < r; ++d) {
      rp.out_shape[d] = out.shape[d];
      rp.out_st[d] = out.st[d];
      rp.in_shape[d] = a.shape[d];
      rp.in_st[d] = a.st[d];
      rp.div[d] = 1;
      rp.mod[d] = std::numeric_limits<int64_t>::max();
      rp.sub[d] = 0;
    }
    op.launch = launch::remap(rp, a, out);
    add_op(std::move(op));
    View v = out;
    v.shape[r - 1] = K;  // logical K stays; padding is zero and read as k >= K by the kernel anyway
    return out;
  }

  void plan_linear(const Node& n) {  // GaweeToLinalg.cpp:877-957: X . W^T + b
    View x = value_view(n.ins[0]);
    View w = value_view(n.ins[1]);
    View bias = value_view(n.ins[2]);
    const Value& o = val(n.outs[0]);
    if (x.rank() != 2 || w.rank() != 2) unsupported("linear expects rank-2 operands");
    int64_t M = x.shape[0], K = x.shape[1], Nn = w.shape[0];
    View a = gemm_operand_a(x);
    PackSpec ps;
    ps.src = w;
    ps.K = K;
    ps.N = Nn;
    ps.sn = w.st[0];
    ps.k_shape = {K};
    ps.k_st = {w.st[1]};
    ps.k_valid = {K};
    int64_t ldk = round_up(K, 4);
    auto hl = add_pack(ps, ldk, "pack_linear_w");
    View out = alloc(DType::F32, o.type.shape);
    Op op;
    op.kind = OpKind::TC;
    op.name = "linear";
    auto& t = op.tc;
    t.x = a;
    t.out = out;
    t.hi = hl.first;
    t.lo = hl.second;
    t.ldk = ldk;
    t.H = M; t.W = 1; t.C = a.shape[1]; t.P = M; t.Q = 1;
    t.M = M; t.N = Nn; t.K = K;
    t.block_n = pick_block_n(Nn);
    t.epi = kern::EPI_BIAS;
    t.bias = bias;
    t.flops = 2.0 * (double)M * (double)Nn * (double)K;
    op.reads = {a, dense_view(hl.first, DType::F32, {1}), dense_view(hl.second, DType::F32, {1}), bias};
    op.writes = {out};
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  void plan_matmul(const Node& n) {  // GaweeToLinalg.cpp:959-1112
    View lhs = value_view(n.ins[0]);
    View rhs = value_view(n.ins[1]);
    const Value& o = val(n.outs[0]);
    int ro = (int)o.type.shape.size(), ra = lhs.rank(), rb = rhs.rank();
    if (ra < 2 || rb < 2) unsupported("matmul with rank < 2 operands");
    if (o.type.dtype != DType::F32) unsupported("non-f32 matmul");
    int64_t M = lhs.shape[ra - 2], K = lhs.shape[ra - 1], Nn = rhs.shape[rb - 1];
    int br = ro - 2;
    if (br > 4) unsupported("matmul with more than 4 batch dims");
    std::vector<int64_t> bshape(o.type.shape.begin(), o.type.shape.begin() + br);
    View a = gemm_operand_a(lhs);
    // A batch strides over output batch dims (size-1 -> 0)
    std::vector<int64_t> a_bst(br, 0), b_bst(br, 0), c_bst(br, 0);
    int la = br - (ra - 2), lb = br - (rb - 2);
    for (int d = 0; d < br; ++d) {
      int ia = d - la;
      // a size-1 dim is never stepped: its stride is irrelevant and left 0
      if (ia >= 0 && a.shape[ia] != 1) a_bst[d] = a.st[ia];
    }
    // B planes are packed for B's own batch dims
    PackSpec ps;
    ps.src = rhs;
    ps.K = K;
    ps.N = Nn;
    ps.sn = rhs.st[rb - 1];
    ps.k_shape = {K};
    ps.k_st = {rhs.st[rb - 2]};
    ps.k_valid = {K};
    int64_t bb = 1;
    for (int d = 0; d < rb - 2; ++d) {
      ps.batch_shape.push_back(rhs.shape[d]);
      ps.batch_st.push_back(rhs.st[d]);
      bb *= rhs.shape[d];
    }
    ps.batch = bb;
    // plane index strides of B's batch dims (row-major over B's batch shape)
    {
      int64_t acc = 1;
      for (int d = rb - 3; d >= 0; --d) {
        int od = lb + d;
        if (rhs.shape[d] != 1) b_bst[od] = acc;
        acc *= rhs.shape[d];
      }
    }
    if (ps.batch_shape.size() > 4) unsupported("matmul rhs with more than 4 batch dims");
    int64_t ldk = round_up(K, 4);
    auto hl = add_pack(ps, ldk, "pack_matmul_b");
    View out = alloc(DType::F32, o.type.shape);
    for (int d = 0; d < br; ++d) c_bst[d] = out.st[d];
    Op op;
    op.kind = OpKind::TC;
    op.name = "matmul";
    auto& t = op.tc;
    t.x = a;
    t.out = out;
    t.hi = hl.first;
    t.lo = hl.second;
    t.b_batch = bb;
    t.ldk = ldk;
    t.H = M; t.W = 1; t.C = round_up(K, 4); t.P = M; t.Q = 1;
    t.M = M; t.N = Nn; t.K = K;
    t.block_n = pick_block_n(Nn);
    t.epi = kern::EPI_NONE;
    t.batch_rank = br;
    t.batch_shape = bshape;
    t.a_bst = a_bst;
    t.b_bst = b_bst;
    {
      double nbt = 1;
      for (auto d : bshape) nbt *= (double)d;
      t.flops = 2.0 * nbt * (double)M * (double)Nn * (double)K;
    }
    op.reads = {a, dense_view(hl.first, DType::F32, {1}), dense_view(hl.second, DType::F32, {1})};
    op.writes = {out};
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  // ---------------------------------------------------------------- merged contractions
  // Matmuls that share their left operand (the same value) and whose right
  // operands are 2-D arguments or constants -- the Q, K and V projections of
  // an attention block -- run as one GEMM over the concatenated weights: A is
  // read once and the N = 192 projections of a GQA block stop wasting half a
  // 128-wide tile.  Each result is a column slice of the shared output, so
  // only results that feed views (reshape, transpose) are merged: a result
  // feeding an elementwise op keeps its own GEMM and the fused epilogue.
  // GAWEE_MERGE_GEMMS=0 turns the merge off.
  std::map<int, std::vector<int>> merge_at_;  // first matmul node -> the group's nodes, in order

  void find_merged_matmuls() {
    if (const char* e = std::getenv("GAWEE_MERGE_GEMMS"))
      if (std::atoi(e) == 0) return;
    Graph& g = plan_->g;
    std::vector<std::vector<int>> consumers(g.values.size());
    for (size_t k = 0; k < g.nodes.size(); ++k)
      for (int v : g.nodes[k].ins) consumers[v].push_back((int)k);
    std::set<int> results(g.results.begin(), g.results.end());
    std::map<int, std::vector<int>> by_lhs;  // lhs value -> candidate nodes
    for (size_t k = 0; k < g.nodes.size(); ++k) {
      const Node& n = g.nodes[k];
      if (n.op != "gawee.matmul" || n.ins.size() != 2 || n.outs.size() != 1) continue;
      if (skip_node_.count((int)k) || attn_at_.count((int)k) || norm_at_.count((int)k) || rope_at_.count((int)k))
        continue;
      const Value& a = val(n.ins[0]);
      const Value& b = val(n.ins[1]);
      const Value& o = val(n.outs[0]);
      if (!a.type.is_tensor || !b.type.is_tensor || b.type.shape.size() != 2 || a.type.shape.size() < 2) continue;
      if (b.def_node >= 0) continue;  // weights: function arguments or constants
      if (o.type.dtype != DType::F32 || a.type.dtype != DType::F32 || b.type.dtype != DType::F32) continue;
      if (b.type.shape[1] % 4 != 0 || results.count(n.outs[0])) continue;
      bool views_only = !consumers[n.outs[0]].empty();
      for (int c : consumers[n.outs[0]])
        if (g.nodes[c].op != "gawee.reshape" && g.nodes[c].op != "gawee.transpose") views_only = false;
      if (!views_only) continue;
      by_lhs[n.ins[0]].push_back((int)k);
    }
    for (auto& [lhs, nodes] : by_lhs) {
      (void)lhs;
      if (nodes.size() < 2) continue;
      merge_at_[nodes[0]] = nodes;
      for (size_t i = 1; i < nodes.size(); ++i) skip_node_.insert(nodes[i]);
    }
  }

  void plan_matmul_merged(const std::vector<int>& nodes) {  // GaweeToLinalg.cpp:959-1112, per member
    Graph& g = plan_->g;
    const Node& n0 = g.nodes[nodes[0]];
    View lhs = value_view(n0.ins[0]);
    const int ra = lhs.rank();
    const int64_t M = lhs.shape[ra - 2], K = lhs.shape[ra - 1];
    std::vector<int64_t> widths;
    int64_t Ntot = 0;
    for (int k : nodes) {
      const View rhs = value_view(g.nodes[k].ins[1]);
      if (rhs.rank() != 2 || rhs.shape[0] != K) unsupported("merged matmul operands");
      widths.push_back(rhs.shape[1]);
      Ntot += rhs.shape[1];
    }
    const int64_t ldk = round_up(K, 4);
    const int hi = new_buf(DType::F32, Ntot * ldk);
    const int lo = new_buf(DType::F32, Ntot * ldk);
    int64_t row = 0;
    for (size_t i = 0; i < nodes.size(); ++i) {
      const View rhs = value_view(g.nodes[nodes[i]].ins[1]);
      PackSpec ps;
      ps.src = rhs;
      ps.K = K;
      ps.N = widths[i];
      ps.sn = rhs.st[1];
      ps.k_shape = {K};
      ps.k_st = {rhs.st[0]};
      ps.k_valid = {K};
      ps.batch = 1;
      ps.row_off = row;
      row += widths[i];
      Op op;
      op.kind = OpKind::PACK;
      op.name = "pack_matmul_b";
      op.reads = {rhs};
      op.writes = {dense_view(hi, DType::F32, {Ntot * ldk}), dense_view(lo, DType::F32, {Ntot * ldk})};
      op.launch = launch::pack(ps, ldk, hi, lo);
      add_op(std::move(op));
    }
    const Value& o0 = val(n0.outs[0]);
    std::vector<int64_t> oshape = o0.type.shape;
    oshape.back() = Ntot;
    const int br = (int)oshape.size() - 2;
    if (br > 4) unsupported("matmul with more than 4 batch dims");
    View a = gemm_operand_a(lhs);
    std::vector<int64_t> a_bst(br, 0), b_bst(br, 0);
    const int la = br - (ra - 2);
    for (int d = 0; d < br; ++d) {
      const int ia = d - la;
      if (ia >= 0 && a.shape[ia] != 1) a_bst[d] = a.st[ia];
    }
    View out = alloc(DType::F32, oshape);
    Op op;
    op.kind = OpKind::TC;
    op.name = "matmul" + std::to_string(nodes.size());
    auto& t = op.tc;
    t.x = a;
    t.out = out;
    t.hi = hi;
    t.lo = lo;
    t.b_batch = 1;
    t.ldk = ldk;
    t.H = M; t.W = 1; t.C = round_up(K, 4); t.P = M; t.Q = 1;
    t.M = M; t.N = Ntot; t.K = K;
    t.block_n = pick_block_n(Ntot);
    t.epi = kern::EPI_NONE;
    t.batch_rank = br;
    t.batch_shape.assign(oshape.begin(), oshape.begin() + br);
    t.a_bst = a_bst;
    t.b_bst = b_bst;
    {
      double nbt = 1;
      for (auto d : t.batch_shape) nbt *= (double)d;
      t.flops = 2.0 * nbt * (double)M * (double)Ntot * (double)K;
    }
    op.reads = {a, dense_view(hi, DType::F32, {1}), dense_view(lo, DType::F32, {1})};
    op.writes = {out};
    add_op(std::move(op));
    // each member's result: its column slice of the shared output
    int64_t col = 0;
    for (size_t i = 0; i < nodes.size(); ++i) {
      View v = out;
      v.shape.back() = widths[i];
      v.off += col;
      col += widths[i];
      set_view(g.nodes[nodes[i]].outs[0], v);
    }
  }

  // ---------------------------------------------------------------- reductions / pools
  void plan_reduce(const Node& n, bool mean) {  // GaweeToLinalg.cpp:1443-1572
    View in = value_view(n.ins[0]);
    const Value& o = val(n.outs[0]);
    if (in.dt != DType::F32) unsupported("reduce on non-f32");
    std::vector<bool> red(in.rank(), false);
    int64_t count = 1;
    for (auto a : n.attr("axes").ints) {
      int64_t ax = a < 0 ? a + in.rank() : a;
      if (!red[ax]) count *= in.shape[ax];
      red[ax] = true;
    }
    View out = alloc(DType::F32, o.type.shape);
    Op op;
    op.kind = OpKind::REDUCE;
    op.name = mean ? "reduce_mean" : "reduce_sum";
    op.reads = {in};
    op.writes = {out};
    op.launch = launch::reduce(in, out, red, mean, (float)count);
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  void plan_global_avg(const Node& n) {  // GaweeToLinalg.cpp:1327-1375, 713-806
    View in = value_view(n.ins[0]);
    const Value& o = val(n.outs[0]);
    std::vector<bool> red = {false, false, true, true};
    View out = alloc(DType::F32, o.type.shape);
    Op op;
    op.kind = OpKind::REDUCE;
    op.name = "global_avg_pool";
    op.reads = {in};
    op.writes = {out};
    op.launch = launch::reduce(in, out, red, true, (float)(in.shape[2] * in.shape[3]));
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  void plan_pool(const Node& n, bool is_max) {  // GaweeToLinalg.cpp:565-706, 1175-1258
    View in = value_view(n.ins[0]);
    const Value& o = val(n.outs[0]);
    auto ks = n.attr("kernelSize").ints, st = n.attr("strides").ints, pd = n.attr("padding").ints;
    std::vector<int64_t> dl = {1, 1};
    if (is_max && n.has_attr("dilation")) dl = n.attr("dilation").ints;
    if (!is_max && !n.attr("countIncludePad").b && (pd[0] != 0 || pd[1] != 0))
      unsupported("average_pool with padding and count_include_pad = false");
    View out = alloc(DType::F32, o.type.shape, layout_like({in}, o.type.shape));
    kern::PoolParams pp{};
    pp.N = in.shape[0]; pp.C = in.shape[1]; pp.H = in.shape[2]; pp.W = in.shape[3];
    pp.OH = out.shape[2]; pp.OW = out.shape[3];
    for (int d = 0; d < 4; ++d) { pp.in_st[d] = in.st[d]; pp.out_st[d] = out.st[d]; }
    pp.kh = (int)ks[0]; pp.kw = (int)ks[1];
    pp.sh = (int)st[0]; pp.sw = (int)st[1];
    pp.ph = (int)pd[0]; pp.pw = (int)pd[1];
    pp.dh = (int)dl[0]; pp.dw = (int)dl[1];
    pp.mode = is_max ? 0 : 1;
    pp.count = (float)(ks[0] * ks[1]);
    std::vector<int> order = {0, 1, 2, 3};
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return out.st[a] > out.st[b]; });
    for (int d = 0; d < 4; ++d) pp.iter_perm[d] = order[d];
    Op op;
    op.kind = OpKind::POOL;
    op.name = is_max ? "max_pool" : "avg_pool";
    op.reads = {in};
    op.writes = {out};
    op.launch = launch::pool(pp, in, out);
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  void plan_softmax(const Node& n) {  // GaweeToLinalg.cpp:1885-1900
    View in = value_view(n.ins[0]);
    const Value& o = val(n.outs[0]);
    int64_t ax = n.attr("axis").i;
    if (ax < 0) ax += in.rank();
    View out = alloc(DType::F32, o.type.shape);
    Op op;
    op.kind = OpKind::SOFTMAX;
    op.name = "softmax";
    op.reads = {in};
    op.writes = {out};
    op.launch = launch::softmax(in, out, (int)ax);
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  void plan_gather(const Node& n) {  // GaweeToLinalg.cpp:2334-2396
    View data = value_view(n.ins[0]);
    View idx = value_view(n.ins[1]);
    const Value& o = val(n.outs[0]);
    int64_t ax = n.attr("axis").i;
    if (ax < 0) ax += data.rank();
    if (!data.dense_rowmajor() || data.off % 4 != 0) data = copy_to_new(data, "gather_data_copy");
    if (!idx.dense_rowmajor()) idx = copy_to_new(idx, "gather_index_copy");
    if (idx.dt != DType::I64 && idx.dt != DType::I32) unsupported("gather indices must be i32/i64");
    int64_t pre = 1, post = 1;
    for (int d = 0; d < ax; ++d) pre *= data.shape[d];
    for (int d = (int)ax + 1; d < data.rank(); ++d) post *= data.shape[d];
    View out = alloc(o.type.dtype, o.type.shape);
    Op op;
    op.kind = OpKind::GATHER;
    op.name = "gather";
    op.reads = {data, idx};
    op.writes = {out};
    op.launch = launch::gather(data, idx, out, pre, data.shape[ax], idx.numel(), post);
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  void plan_gather_elements(const Node& n) {  // GaweeToLinalg.cpp:2398-2437
    View data = value_view(n.ins[0]);
    View idx = value_view(n.ins[1]);
    const Value& o = val(n.outs[0]);
    int64_t ax = n.attr("axis").i;
    if (ax < 0) ax += idx.rank();
    if (!idx.dense_rowmajor()) idx = copy_to_new(idx, "gather_index_copy");
    View out = alloc(o.type.dtype, o.type.shape);
    Op op;
    op.kind = OpKind::GATHER_ELEMS;
    op.name = "gather_elements";
    op.reads = {data, idx};
    op.writes = {out};
    op.launch = launch::gather_elements(data, idx, out, (int)ax);
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  void plan_range(const Node& n) {  // GaweeToLinalg.cpp:2439-2496
    const Value& o = val(n.outs[0]);
    double fs, fd, fl;
    int64_t is, id, il;
    if (!scalar_const(n.ins[0], fs, is) || !scalar_const(n.ins[1], fl, il) || !scalar_const(n.ins[2], fd, id))
      unsupported("range with non-constant operands");
    View out = alloc(o.type.dtype, o.type.shape);
    kern::RangeParams rp{};
    rp.dt = (int8_t)o.type.dtype;
    rp.n = out.numel();
    rp.fstart = fs; rp.fdelta = fd; rp.istart = is; rp.idelta = id;
    Op op;
    op.kind = OpKind::RANGE;
    op.name = "range";
    op.reads = {value_view(n.ins[0]), value_view(n.ins[2])};
    op.writes = {out};
    op.launch = launch::range(rp, out);
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  void plan_shape(const Node& n) {  // GaweeToLinalg.cpp:1851-1883: static dims
    View in = value_view(n.ins[0]);
    const Value& o = val(n.outs[0]);
    int r = in.rank();
    int64_t s = n.attr("start").i, e = n.attr("end").i;
    if (s < 0) s += r;
    if (e < 0) e += r;
    e = std::min<int64_t>(e, r);
    int b = new_buf(o.type.dtype, o.type.numel(), BufKind::CONST);
    auto& hb = plan_->bufs[b].host_init;
    hb.assign((size_t)o.type.numel() * dtype_size(o.type.dtype), 0);
    for (int64_t d = s; d < e; ++d) {
      if (o.type.dtype == DType::I64) { int64_t x = in.shape[d]; std::memcpy(hb.data() + 8 * (d - s), &x, 8); }
      else if (o.type.dtype == DType::I32) { int32_t x = (int32_t)in.shape[d]; std::memcpy(hb.data() + 4 * (d - s), &x, 4); }
      else unsupported("shape result type");
    }
    set_view(n.outs[0], dense_view(b, o.type.dtype, o.type.shape));
  }

  void plan_remap(const Node& n, const std::string& k) {  // tile / pad / resize
    View in = value_view(n.ins[0]);
    const Value& o = val(n.outs[0]);
    View out = alloc(o.type.dtype, o.type.shape);
    kern::RemapParams rp{};
    rp.elem_bytes = (int)dtype_size(in.dt);
    rp.rank = in.rank();
    rp.numel = out.numel();
    std::vector<int64_t> pads;
    std::vector<double> scales;
    uint64_t fill = 0;
    if (k == "pad") {
      if (n.attr("mode").s != "constant") unsupported("pad mode " + n.attr("mode").s);
      pads = const_ints(n.ins[1]);
      const Value& cv = val(n.ins[2]);
      if (!cv.is_const) unsupported("pad with a non-constant value");
      std::memcpy(&fill, cv.data.data(), std::min<size_t>(8, cv.data.size()));
    } else if (k == "resize") {  // GaweeToLinalg.cpp:2498-2552
      if (n.attr("mode").s != "nearest" || n.attr("coordinateTransformationMode").s != "asymmetric" ||
          n.attr("nearestMode").s != "floor")
        unsupported("resize mode");
      const Value& sv = val(n.ins[1]);
      if (!sv.is_const) unsupported("resize with non-constant scales");
      for (int64_t q = 0; q < sv.type.numel(); ++q) {
        double sc = const_as_double(sv, q);
        if (sc != std::floor(sc) || sc < 1) unsupported("resize with non-integer scales");
        scales.push_back(sc);
      }
    }
    for (int d = 0; d < rp.rank; ++d) {
      rp.out_shape[d] = out.shape[d];
      rp.out_st[d] = out.st[d];
      rp.in_shape[d] = in.shape[d];
      rp.in_st[d] = in.st[d];
      rp.div[d] = 1;
      rp.mod[d] = std::numeric_limits<int64_t>::max();
      rp.sub[d] = 0;
      if (k == "tile") rp.mod[d] = in.shape[d];                    // GaweeToLinalg.cpp:2733-2747
      if (k == "pad") rp.sub[d] = pads[d];                         // GaweeToLinalg.cpp:2754-2797
      if (k == "resize") rp.div[d] = (int64_t)scales[d];
    }
    rp.fill_bits = fill;
    Op op;
    op.kind = OpKind::REMAP;
    op.name = k;
    op.reads = {in};
    op.writes = {out};
    op.launch = launch::remap(rp, in, out);
    add_op(std::move(op));
    set_view(n.outs[0], out);
  }

  void plan_topk(const Node& n) {  // GaweeToLinalg.cpp:1577-1680
    View in = value_view(n.ins[0]);
    int64_t k = n.attr("k").i, ax = n.attr("axis").i;
    if (ax < 0) ax += in.rank();
    if (in.rank() != 2 || ax != 1) unsupported("topk supports rank-2 inputs along axis 1");
    if (!in.dense_rowmajor()) in = copy_to_new(in, "topk_copy");
    View vals = alloc(DType::F32, val(n.outs[0]).type.shape);
    View idxs = alloc(DType::I64, val(n.outs[1]).type.shape);
    View used = alloc(DType::I1, in.shape);
    Op op;
    op.kind = OpKind::TOPK;
    op.name = "topk";
    op.reads = {in};
    op.writes = {vals, idxs, used};
    op.launch = launch::topk(in, vals, idxs, used, k);
    add_op(std::move(op));
    set_view(n.outs[0], vals);
    set_view(n.outs[1], idxs);
  }

  // The tensor-core kernel gathers A with 16-byte loads: every stepped A
  // stride, the channel count and the base offset must be whole float4s.
  static void validate_tc(const Op& op) {
    const auto& t = op.tc;
    auto bad = [&](const std::string& why) { throw std::runtime_error("internal: " + op.name + ": " + why); };
    if (t.K <= 0 || t.M <= 0 || t.N <= 0) bad("empty contraction");
    if (t.C % 4 != 0) bad("channel count not a multiple of 4");
    if (t.x.off % 4 != 0) bad("A operand offset not 16-byte aligned");
    if (t.conv) {
      if (t.x.st[1] != 1 || t.x.st[3] % 4 || t.x.st[2] % 4 || (t.x.shape[0] > 1 && t.x.st[0] % 4))
        bad("conv input not NHWC with 16-byte aligned pixels");
    } else {
      int r = t.x.rank();
      if (t.x.shape[r - 1] > 1 && t.x.st[r - 1] != 1) bad("A rows not unit-stride");
      if (t.M > 1 && t.x.st[r - 2] % 4) bad("A row stride not a multiple of 4");
      for (int d = 0; d < t.batch_rank; ++d)
        if (t.a_bst[d] % 4) bad("A batch stride not a multiple of 4");
    }
    if (t.ldk % 4) bad("packed B row pitch not a multiple of 4");
  }

  // ---------------------------------------------------------------- phases
  void assign_phases() {
    auto& ops = plan_->ops;
    auto& bufs = plan_->bufs;
    std::vector<int> buf_phase(bufs.size(), -1);  // -1 none, 0 const, else producing phase
    for (size_t b = 0; b < bufs.size(); ++b)
      if (bufs[b].kind == BufKind::CONST) buf_phase[b] = (int)Phase::PROLOGUE;
    for (auto& op : ops) {
      bool only_const = true, only_static = true;
      std::set<int> args;
      for (const View& r : op.reads) {
        const Buf& b = bufs[r.buf];
        if (b.kind == BufKind::ARG) {
          only_const = false;
          args.insert(b.arg);
          continue;
        }
        int ph = buf_phase[r.buf];
        if (ph == (int)Phase::PROLOGUE) continue;
        only_const = false;
        only_static = false;
      }
      if (only_const) op.phase = Phase::PROLOGUE;
      else if (op.kind == OpKind::PACK && only_static) {
        op.phase = Phase::PACK;
        op.dep_args = args;
      } else op.phase = Phase::MAIN;
      for (const View& w : op.writes) {
        int& bp = buf_phase[w.buf];
        bp = std::max(bp, (int)op.phase);
      }
    }
  }

  // ---------------------------------------------------------------- fusion
  // readers[b] = list of (op, slot) reading buffer b; -1 op = graph result
  std::vector<std::vector<std::pair<int, int>>> readers() {
    std::vector<std::vector<std::pair<int, int>>> r(plan_->bufs.size());
    for (size_t o = 0; o < plan_->ops.size(); ++o) {
      const Op& op = plan_->ops[o];
      if (op.dead) continue;
      for (size_t s = 0; s < op.reads.size(); ++s) r[op.reads[s].buf].push_back({(int)o, (int)s});
    }
    for (const View& v : plan_->result_view) r[v.buf].push_back({-1, 0});
    return r;
  }

  static int count_writers(const std::vector<Op>& ops, int buf) {
    int c = 0;
    for (const auto& op : ops)
      if (!op.dead)
        for (const View& w : op.writes) c += w.buf == buf;
    return c;
  }

  // Merge producer program P (whose result feeds argument slots `slots` of C).
  static bool merge_programs(const EProgram& P, const EProgram& C, const std::vector<int>& slots, EProgram& out,
                             std::vector<int>& c_arg_map_out) {
    // new args: C args not in slots, then P args
    EProgram q;
    std::vector<int> cmap(C.reg_types.size(), -1), pmap(P.reg_types.size(), -1);
    std::vector<int> kept;
    for (int a = 0; a < C.n_args; ++a) {
      if (std::find(slots.begin(), slots.end(), a) != slots.end()) continue;
      cmap[a] = q.add_reg(C.reg_types[a]);
      kept.push_back(a);
    }
    for (int a = 0; a < P.n_args; ++a) pmap[a] = q.add_reg(P.reg_types[a]);
    q.n_args = (int)q.reg_types.size();
    for (const EInstr& in0 : P.code) {
      EInstr in = in0;
      if (in.a >= 0) in.a = (int16_t)pmap[in.a];
      if (in.b >= 0) in.b = (int16_t)pmap[in.b];
      if (in.c >= 0) in.c = (int16_t)pmap[in.c];
      in.dst = (int16_t)q.add_reg(P.reg_types[in0.dst]);
      pmap[in0.dst] = in.dst;
      q.code.push_back(in);
    }
    int pres = pmap[P.result];
    for (int s : slots) cmap[s] = pres;
    for (const EInstr& in0 : C.code) {
      EInstr in = in0;
      if (in.a >= 0) in.a = (int16_t)cmap[in.a];
      if (in.b >= 0) in.b = (int16_t)cmap[in.b];
      if (in.c >= 0) in.c = (int16_t)cmap[in.c];
      in.dst = (int16_t)q.add_reg(C.reg_types[in0.dst]);
      cmap[in0.dst] = in.dst;
      q.code.push_back(in);
    }
    q.result = cmap[C.result];
    if ((int)q.code.size() > kern::kMaxInstr || (int)q.reg_types.size() > kern::kMaxRegs) return false;
    out = q;
    c_arg_map_out = kept;
    return true;
  }

  void fuse_elementwise() {
    auto& ops = plan_->ops;
    bool changed = true;
    while (changed) {
      changed = false;
      auto rd = readers();
      for (size_t c = 0; c < ops.size(); ++c) {
        Op& C = ops[c];
        if (C.dead || C.kind != OpKind::EW) continue;
        for (size_t s = 0; s < C.ins.size(); ++s) {
          int b = C.ins[s].buf;
          int p = plan_->bufs[b].producer;
          if (p < 0 || p >= (int)c) continue;
          Op& P = ops[p];
          if (P.dead || P.kind != OpKind::EW || P.phase != C.phase) continue;
          if (count_writers(ops, b) != 1) continue;
          // every read of b must be C reading exactly P's output view over C's space
          if (!same_view(P.out, C.ins[s]) || P.out.shape != C.out.shape) continue;
          bool ok = true;
          std::vector<int> slots;
          for (auto& r : rd[b]) {
            if (r.first != (int)c) { ok = false; break; }
            if (!same_view(C.reads[r.second], P.out)) { ok = false; break; }
          }
          if (!ok) continue;
          for (size_t k = 0; k < C.ins.size(); ++k)
            if (C.ins[k].buf == b) slots.push_back((int)k);
          if ((int)(C.ins.size() - slots.size() + P.ins.size()) > kern::kMaxIn) continue;
          EProgram merged;
          std::vector<int> kept;
          if (!merge_programs(P.prog, C.prog, slots, merged, kept)) continue;
          std::vector<View> nins;
          for (int k : kept) nins.push_back(C.ins[k]);
          for (const View& v : P.ins) nins.push_back(v);
          C.ins = nins;
          C.reads = nins;
          C.prog = merged;
          C.name = P.name + "+" + C.name;
          P.dead = true;
          changed = true;
          break;
        }
        if (changed) break;
      }
    }
  }

  // Recognise the conv epilogue shapes relu(acc) and relu(acc + res).
  static int match_conv_epilogue(const EProgram& p, int acc_slot) {
    // expect: [const 0], maximumf(x, 0) with x = acc (relu) or x = addf(acc, other)
    const EInstr* last = nullptr;
    for (const auto& in : p.code)
      if (in.dst == p.result) last = &in;
    if (!last || last->op != EOp::MAXIMUMF || last->ty != DType::F32) return -1;
    auto is_zero = [&](int reg) {
      for (const auto& in : p.code)
        if (in.dst == reg) return in.op == EOp::CONST && in.fimm == 0.0 && !std::signbit(in.fimm);
      return false;
    };
    int x = -1;
    if (is_zero(last->b)) x = last->a;
    else return -1;
    if (x == acc_slot && p.code.size() == 2) return kern::EPI_BIAS_RELU;
    for (const auto& in : p.code)
      if (in.dst == x && in.op == EOp::ADDF && (in.a == acc_slot || in.b == acc_slot) && in.a != in.b &&
          p.code.size() == 3 && p.n_args == 2)
        return kern::EPI_BIAS_ADD_RELU;
    return -1;
  }

  void fuse_epilogues() {
    auto& ops = plan_->ops;
    auto rd = readers();
    for (size_t t = 0; t < ops.size(); ++t) {
      Op& T = ops[t];
      if (T.dead || T.kind != OpKind::TC) continue;
      if (T.tc.epi != kern::EPI_NONE && T.tc.epi != kern::EPI_BIAS) continue;  // already fused
      int b = T.tc.out.buf;
      if (rd[b].size() != 1 || rd[b][0].first < 0) continue;
      int c = rd[b][0].first;
      Op& C = ops[c];
      if (C.dead || C.kind != OpKind::EW || C.phase != T.phase) continue;
      if (C.out.dt != DType::F32 || C.out.shape != T.tc.out.shape) continue;
      std::vector<int> slots;
      for (size_t k = 0; k < C.ins.size(); ++k)
        if (C.ins[k].buf == b) {
          if (!same_view(C.ins[k], T.tc.out)) slots.clear(), slots.push_back(-1);
          else slots.push_back((int)k);
        }
      if (slots.size() != 1 || slots[0] < 0) continue;
      int acc_slot = slots[0];
      // output of C must be addressable like T's output
      const View& co = C.out;
      if (T.tc.conv) {
        // NHWC dense output: pixel stride uniform
        if (!(co.st[1] == 1 && co.st[3] == co.shape[1] && co.st[2] == co.shape[3] * co.shape[1] &&
              co.st[0] == co.shape[2] * co.shape[3] * co.shape[1]))
          continue;
        int epi = match_conv_epilogue(C.prog, acc_slot);
        if (epi == kern::EPI_BIAS_RELU) {
          T.tc.epi = epi;
        } else if (epi == kern::EPI_BIAS_ADD_RELU) {
          const View& res = C.ins[1 - acc_slot];
          if (res.st != co.st || res.dt != DType::F32) continue;
          T.tc.epi = epi;
          T.tc.res = res;
        } else {
          continue;
        }
      } else {
        // GEMM: C's output must be row-major over [batch..., M, N] with unit column stride
        int r = co.rank();
        if (co.st[r - 1] != 1 || co.off != 0) continue;
        if ((int)C.ins.size() - 1 > 4) continue;
        // aux operands: all other inputs must be f32
        bool ok = true;
        for (size_t k = 0; k < C.ins.size(); ++k)
          if ((int)k != acc_slot && C.ins[k].dt != DType::F32) ok = false;
        if (!ok || C.prog.reg_types[acc_slot] != DType::F32) continue;
        // program with the accumulator as register 0, aux 1..
        EProgram q;
        std::vector<int> map(C.prog.reg_types.size(), -1);
        map[acc_slot] = q.add_reg(DType::F32);
        std::vector<View> aux;
        for (size_t k = 0; k < C.ins.size(); ++k)
          if ((int)k != acc_slot) {
            map[k] = q.add_reg(C.prog.reg_types[k]);
            aux.push_back(C.ins[k]);
          }
        q.n_args = (int)q.reg_types.size();
        for (const EInstr& in0 : C.prog.code) {
          EInstr in = in0;
          if (in.a >= 0) in.a = (int16_t)map[in.a];
          if (in.b >= 0) in.b = (int16_t)map[in.b];
          if (in.c >= 0) in.c = (int16_t)map[in.c];
          in.dst = (int16_t)q.add_reg(C.prog.reg_types[in0.dst]);
          map[in0.dst] = in.dst;
          q.code.push_back(in);
        }
        q.result = map[C.prog.result];
        if (T.tc.epi == kern::EPI_BIAS) {
          // keep the bias add as the first step of the program: acc + bias[n]
          // (expressed by passing bias through the kernel's bias pointer)
        }
        T.tc.epi = kern::EPI_PROGRAM;
        T.tc.prog = q;
        T.tc.aux = aux;
      }
      // T now writes C's output, at C's position in the sequence (C's other
      // operands, e.g. a residual from a later downsample conv, exist there)
      const View out_view = co;  // copy: `co` refers into ops[c], which is replaced below
      T.tc.out = out_view;
      T.writes = {out_view};
      for (const View& v : C.ins)
        if (v.buf != b) T.reads.push_back(v);
      T.name = T.name + "+" + C.name;
      Op fused = std::move(T);
      ops[t] = Op();
      ops[t].dead = true;
      ops[c] = std::move(fused);
      for (auto& buf : plan_->bufs)
        if (buf.producer == (int)t) buf.producer = c;
      plan_->bufs[out_view.buf].producer = c;
    }
  }

  void finalize_kinds() {
    for (size_t o = 0; o < plan_->ops.size(); ++o) {
      const Op& op = plan_->ops[o];
      if (op.dead) continue;
      if (op.phase == Phase::PROLOGUE) plan_->prologue.push_back((int)o);
      else if (op.phase == Phase::PACK) plan_->pack.push_back((int)o);
      else plan_->main.push_back((int)o);
    }
    // buffers written outside MAIN persist; so do result buffers
    for (size_t o = 0; o < plan_->ops.size(); ++o) {
      const Op& op = plan_->ops[o];
      if (op.dead || op.phase == Phase::MAIN) continue;
      for (const View& w : op.writes)
        if (plan_->bufs[w.buf].kind == BufKind::ARENA) plan_->bufs[w.buf].kind = BufKind::PERSIST;
    }
    for (const View& v : plan_->result_view)
      if (plan_->bufs[v.buf].kind == BufKind::ARENA) plan_->bufs[v.buf].kind = BufKind::PERSIST;
  }

};

}  // namespace

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

static void assign_offsets(Plan& P) {
  auto& bufs = P.bufs;
  std::vector<int> first(bufs.size(), -1), last(bufs.size(), -1);
  std::vector<char> touched(bufs.size(), 0);
  for (size_t i = 0; i < P.main.size(); ++i) {
    const Op& op = P.ops[P.main[i]];
    auto touch = [&](const View& v) {
      touched[v.buf] = 1;
      if (first[v.buf] < 0) first[v.buf] = (int)i;
      last[v.buf] = std::max(last[v.buf], (int)i);
    };
    for (const View& v : op.reads) touch(v);
    for (const View& v : op.writes) touch(v);
  }
  for (const auto* list : {&P.prologue, &P.pack})
    for (int o : *list) {
      for (const View& v : P.ops[o].writes) touched[v.buf] = 1;
      for (const View& v : P.ops[o].reads) touched[v.buf] = 1;
    }
  for (const View& v : P.result_view) touched[v.buf] = 1;
  size_t poff = 0;
  for (size_t b = 0; b < bufs.size(); ++b) {
    Buf& B = bufs[b];
    if (B.kind == BufKind::ARENA) continue;
    if (!touched[b] && B.kind != BufKind::ARG) continue;
    B.offset = poff;
    B.live = true;
    poff = align_up(poff + B.bytes(), 256);
  }
  // arena: largest first, lowest offset free over the buffer's live interval
  std::vector<int> order;
  for (size_t b = 0; b < bufs.size(); ++b)
    if (bufs[b].kind == BufKind::ARENA && touched[b] && first[b] >= 0) order.push_back((int)b);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return bufs[a].bytes() > bufs[b].bytes(); });
  struct Placed { size_t off, size; int f, l; };
  std::vector<Placed> placed;
  size_t arena = 0;
  for (int b : order) {
    size_t sz = align_up(bufs[b].bytes(), 256);
    std::vector<std::pair<size_t, size_t>> busy;
    for (const auto& p : placed)
      if (!(p.l < first[b] || last[b] < p.f)) busy.push_back({p.off, p.off + p.size});
    std::sort(busy.begin(), busy.end());
    size_t off = 0;
    for (const auto& r : busy) {
      if (off + sz <= r.first) break;
      off = std::max(off, r.second);
    }
    bufs[b].offset = off;
    bufs[b].live = true;
    placed.push_back({off, sz, first[b], last[b]});
    arena = std::max(arena, off + sz);
  }
  P.persist_bytes = poff;
  P.arena_bytes = arena;
}

std::unique_ptr<Plan> build_plan(Graph g) {
  Planner p(std::move(g));
  auto plan = p.run();
  assign_offsets(*plan);
  return plan;
}

}  // namespace gawee
