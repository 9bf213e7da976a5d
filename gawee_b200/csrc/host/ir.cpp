// MLIR-text parser for gawee-dialect `forward` functions. See ir.h.
#include "ir.h"

#include <cctype>
#include <cmath>
#include <cstring>
#include <fstream>
#include <sstream>
#include <unordered_map>

namespace gawee {

size_t dtype_size(DType t) {
  switch (t) {
    case DType::F32: return 4;
    case DType::F64: return 8;
    case DType::F16: return 2;
    case DType::I64: return 8;
    case DType::I32: return 4;
    case DType::I1: return 1;
    case DType::INDEX: return 8;
  }
  return 0;
}

const char* dtype_name(DType t) {
  switch (t) {
    case DType::F32: return "f32";
    case DType::F64: return "f64";
    case DType::F16: return "f16";
    case DType::I64: return "i64";
    case DType::I32: return "i32";
    case DType::I1: return "i1";
    case DType::INDEX: return "index";
  }
  return "?";
}

int64_t TensorType::numel() const {
  int64_t n = 1;
  for (int64_t d : shape) n *= d;
  return n;
}

std::string TensorType::str() const {
  if (!is_tensor) return dtype_name(dtype);
  std::string s = "tensor<";
  for (int64_t d : shape) s += std::to_string(d) + "x";
  return s + dtype_name(dtype) + ">";
}

bool AffineMapIR::is_identity() const {
  if ((int)exprs.size() != n_dims) return false;
  for (int i = 0; i < n_dims; ++i)
    if (exprs[i] != i) return false;
  return true;
}

const Attr& Node::attr(const std::string& k) const {
  auto it = attrs.find(k);
  if (it == attrs.end()) throw std::runtime_error(op + ": missing attribute '" + k + "'");
  return it->second;
}

const char* eop_name(EOp op) {
  static const char* names[] = {
      "const", "addf", "subf", "mulf", "divf", "remf", "maximumf", "minimumf", "maxnumf", "minnumf",
      "powf", "negf", "sqrt", "rsqrt", "exp", "log", "erf", "tanh", "sin", "cos", "absf", "floor",
      "ceil", "addi", "subi", "muli", "divsi", "remsi", "maxsi", "minsi", "andi", "ori", "xori",
      "cmpf", "cmpi", "select", "sitofp", "uitofp", "fptosi", "extf", "truncf", "extsi", "extui",
      "trunci", "index_cast", "copy"};
  static_assert(sizeof(names) / sizeof(names[0]) == (size_t)EOp::COUNT_, "eop names");
  return names[(int)op];
}

std::string EProgram::str() const {
  std::ostringstream o;
  o << "args=" << n_args << " regs=" << reg_types.size() << " result=r" << result << "\n";
  for (const auto& in : code) {
    o << "  r" << in.dst << " = " << eop_name(in.op) << "." << dtype_name(in.ty);
    if (in.op == EOp::CONST) {
      if (is_float(in.rty)) o << " " << in.fimm; else o << " " << in.iimm;
    }
    if (in.a >= 0) o << " r" << in.a;
    if (in.b >= 0) o << " r" << in.b;
    if (in.c >= 0) o << " r" << in.c;
    if (in.op == EOp::CMPF || in.op == EOp::CMPI) o << " pred=" << int(in.pred);
    o << "\n";
  }
  return o.str();
}

std::string read_text_file(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw std::runtime_error("could not open " + path);
  std::ostringstream ss;
  ss << in.rdbuf();
  return ss.str();
}

double const_as_double(const Value& v, int64_t i) {
  const uint8_t* p = v.data.data();
  switch (v.type.dtype) {
    case DType::F32: { float x; std::memcpy(&x, p + 4 * i, 4); return x; }
    case DType::F64: { double x; std::memcpy(&x, p + 8 * i, 8); return x; }
    case DType::I64: case DType::INDEX: { int64_t x; std::memcpy(&x, p + 8 * i, 8); return (double)x; }
    case DType::I32: { int32_t x; std::memcpy(&x, p + 4 * i, 4); return (double)x; }
    case DType::I1: return p[i] ? 1.0 : 0.0;
    default: throw std::runtime_error("const_as_double: unsupported dtype");
  }
}

int64_t const_as_int(const Value& v, int64_t i) {
  const uint8_t* p = v.data.data();
  switch (v.type.dtype) {
    case DType::I64: case DType::INDEX: { int64_t x; std::memcpy(&x, p + 8 * i, 8); return x; }
    case DType::I32: { int32_t x; std::memcpy(&x, p + 4 * i, 4); return x; }
    case DType::I1: return p[i] ? 1 : 0;
    case DType::F32: { float x; std::memcpy(&x, p + 4 * i, 4); return (int64_t)x; }
    case DType::F64: { double x; std::memcpy(&x, p + 8 * i, 8); return (int64_t)x; }
    default: throw std::runtime_error("const_as_int: unsupported dtype");
  }
}

namespace {

struct Cursor {
  const std::string& s;
  size_t p = 0;
  explicit Cursor(const std::string& str) : s(str) {}

  [[noreturn]] void fail(const std::string& msg) const {
    size_t line = 1, col = 1;
    for (size_t i = 0; i < p && i < s.size(); ++i) {
      if (s[i] == '\n') { ++line; col = 1; } else { ++col; }
    }
    size_t e = s.find('\n', p);
    std::string ctx = s.substr(p, std::min<size_t>(60, (e == std::string::npos ? s.size() : e) - p));
    throw ParseError("parse error at line " + std::to_string(line) + ":" + std::to_string(col) + ": " + msg +
                     " near '" + ctx + "'");
  }
  void ws() {
    while (p < s.size()) {
      char c = s[p];
      if (std::isspace((unsigned char)c)) { ++p; continue; }
      if (c == '/' && p + 1 < s.size() && s[p + 1] == '/') {
        while (p < s.size() && s[p] != '\n') ++p;
        continue;
      }
      break;
    }
  }
  bool eof() { ws(); return p >= s.size(); }
  char peek() { ws(); return p < s.size() ? s[p] : '\0'; }
  bool starts(const char* t) {
    ws();
    return s.compare(p, std::strlen(t), t) == 0;
  }
  bool accept(const char* t) {
    if (starts(t)) { p += std::strlen(t); return true; }
    return false;
  }
  void expect(const char* t) {
    if (!accept(t)) fail(std::string("expected '") + t + "'");
  }
  static bool idch(char c) { return std::isalnum((unsigned char)c) || c == '_' || c == '.' || c == '$' || c == '-'; }
  std::string ident() {
    ws();
    size_t b = p;
    while (p < s.size() && (std::isalnum((unsigned char)s[p]) || s[p] == '_' || s[p] == '.' || s[p] == '$')) ++p;
    if (b == p) fail("expected identifier");
    return s.substr(b, p - b);
  }
  // %name, %name#k (use), %name:N handled by caller
  std::string ssa() {
    ws();
    if (p >= s.size() || s[p] != '%') fail("expected SSA value");
    size_t b = p++;
    while (p < s.size() && (std::isalnum((unsigned char)s[p]) || s[p] == '_' || s[p] == '.' || s[p] == '$' || s[p] == '-')) ++p;
    if (p < s.size() && s[p] == '#') {
      ++p;
      while (p < s.size() && std::isdigit((unsigned char)s[p])) ++p;
    }
    return s.substr(b, p - b);
  }
  std::string string_lit() {
    ws();
    if (s[p] != '"') fail("expected string literal");
    ++p;
    std::string out;
    while (p < s.size() && s[p] != '"') {
      if (s[p] == '\\' && p + 1 < s.size()) { out.push_back(s[p + 1]); p += 2; continue; }
      out.push_back(s[p++]);
    }
    if (p >= s.size()) fail("unterminated string");
    ++p;
    return out;
  }
  // integer or float literal (decimal, hex integer, inf/nan spelled by MLIR as hex)
  bool number(double& f, int64_t& i, bool& is_int, bool& is_hex) {
    ws();
    size_t b = p;
    is_hex = false;
    if (s.compare(p, 2, "0x") == 0 || s.compare(p, 3, "-0x") == 0) {
      bool neg = s[p] == '-';
      p += neg ? 3 : 2;
      size_t hb = p;
      while (p < s.size() && std::isxdigit((unsigned char)s[p])) ++p;
      if (hb == p) { p = b; return false; }
      uint64_t u = std::stoull(s.substr(hb, p - hb), nullptr, 16);
      i = neg ? -(int64_t)u : (int64_t)u;
      f = (double)i;
      is_int = true;
      is_hex = true;
      return true;
    }
    if (p < s.size() && (s[p] == '-' || s[p] == '+')) ++p;
    bool digits = false, fl = false;
    while (p < s.size() && std::isdigit((unsigned char)s[p])) { ++p; digits = true; }
    if (p < s.size() && s[p] == '.') { fl = true; ++p; while (p < s.size() && std::isdigit((unsigned char)s[p])) { ++p; digits = true; } }
    if (digits && p < s.size() && (s[p] == 'e' || s[p] == 'E')) {
      size_t q = p + 1;
      if (q < s.size() && (s[q] == '-' || s[q] == '+')) ++q;
      if (q < s.size() && std::isdigit((unsigned char)s[q])) {
        fl = true;
        p = q;
        while (p < s.size() && std::isdigit((unsigned char)s[p])) ++p;
      }
    }
    if (!digits) { p = b; return false; }
    std::string t = s.substr(b, p - b);
    if (fl) { f = std::strtod(t.c_str(), nullptr); i = (int64_t)f; is_int = false; }
    else { i = std::stoll(t); f = (double)i; is_int = true; }
    return true;
  }
  int64_t integer() {
    double f; int64_t i; bool ii, hx;
    if (!number(f, i, ii, hx) || !ii) fail("expected integer");
    return i;
  }
};

DType parse_scalar_type(Cursor& c) {
  std::string t = c.ident();
  if (t == "f32") return DType::F32;
  if (t == "f64") return DType::F64;
  if (t == "f16") return DType::F16;
  if (t == "i64" || t == "si64") return DType::I64;
  if (t == "i32" || t == "si32") return DType::I32;
  if (t == "i1") return DType::I1;
  if (t == "index") return DType::INDEX;
  c.fail("unsupported element type '" + t + "'");
}

TensorType parse_type(Cursor& c) {
  TensorType tt;
  if (c.accept("tensor<") || c.accept("memref<")) {
    // dims "AxBx...xT" or just "T"
    while (true) {
      c.ws();
      if (c.s[c.p] == '?') c.fail("dynamic dimensions are not supported (static shapes only)");
      if (std::isdigit((unsigned char)c.s[c.p])) {
        size_t b = c.p;
        while (std::isdigit((unsigned char)c.s[c.p])) ++c.p;
        tt.shape.push_back(std::stoll(c.s.substr(b, c.p - b)));
        if (c.s[c.p] != 'x') c.fail("expected 'x' in shaped type");
        ++c.p;
        continue;
      }
      break;
    }
    tt.dtype = parse_scalar_type(c);
    // memref layouts / tensor encodings are not expected; skip to '>'
    c.ws();
    if (c.s[c.p] == ',') {
      int depth = 0;
      while (c.p < c.s.size()) {
        char ch = c.s[c.p];
        if (ch == '<') ++depth;
        if (ch == '>') { if (depth == 0) break; --depth; }
        ++c.p;
      }
    }
    c.expect(">");
    tt.is_tensor = true;
    return tt;
  }
  tt.dtype = parse_scalar_type(c);
  tt.is_tensor = false;
  return tt;
}

// Fill `out` (row-major, storage dtype) from a dense<...> payload.
void parse_dense_payload(Cursor& c, const TensorType& tt, std::vector<uint8_t>& out) {
  int64_t n = tt.is_tensor ? tt.numel() : 1;
  size_t es = dtype_size(tt.dtype);
  out.assign((size_t)n * es, 0);
  auto store = [&](int64_t idx, double f, int64_t i, bool is_int, bool is_hex) {
    uint8_t* p = out.data() + idx * es;
    switch (tt.dtype) {
      case DType::F32: {
        float x;
        if (is_hex) { uint32_t u = (uint32_t)i; std::memcpy(&x, &u, 4); }
        else x = is_int ? (float)i : (float)f;
        std::memcpy(p, &x, 4); break;
      }
      case DType::F64: {
        double x;
        if (is_hex) { uint64_t u = (uint64_t)i; std::memcpy(&x, &u, 8); }
        else x = is_int ? (double)i : f;
        std::memcpy(p, &x, 8); break;
      }
      case DType::I64: case DType::INDEX: { int64_t x = is_int ? i : (int64_t)f; std::memcpy(p, &x, 8); break; }
      case DType::I32: { int32_t x = (int32_t)(is_int ? i : (int64_t)f); std::memcpy(p, &x, 4); break; }
      case DType::I1: { p[0] = (is_int ? i : (int64_t)f) != 0; break; }
      default: c.fail("unsupported dense element type");
    }
  };
  auto scalar = [&](int64_t idx) {
    c.ws();
    if (c.accept("true")) { store(idx, 1, 1, true, false); return; }
    if (c.accept("false")) { store(idx, 0, 0, true, false); return; }
    double f; int64_t i; bool ii, hx;
    if (c.accept("inf")) { store(idx, INFINITY, 0, false, false); return; }
    if (c.accept("-inf")) { store(idx, -INFINITY, 0, false, false); return; }
    if (c.accept("nan")) { store(idx, NAN, 0, false, false); return; }
    if (!c.number(f, i, ii, hx)) c.fail("expected dense element");
    store(idx, f, i, ii, hx && is_float(tt.dtype));
  };
  c.ws();
  if (c.s[c.p] == '"') {
    std::string hex = c.string_lit();
    if (hex.size() < 2 || hex[0] != '0' || (hex[1] != 'x' && hex[1] != 'X')) c.fail("bad hex dense payload");
    size_t nbytes = (hex.size() - 2) / 2;
    std::vector<uint8_t> raw(nbytes);
    for (size_t k = 0; k < nbytes; ++k) raw[k] = (uint8_t)std::stoul(hex.substr(2 + 2 * k, 2), nullptr, 16);
    if (raw.size() == out.size()) { out = raw; return; }
    if (raw.size() == es) {  // hex splat
      for (int64_t k = 0; k < n; ++k) std::memcpy(out.data() + k * es, raw.data(), es);
      return;
    }
    c.fail("hex dense payload size does not match the type");
  }
  if (c.peek() != '[') {  // splat
    scalar(0);
    for (int64_t k = 1; k < n; ++k) std::memcpy(out.data() + k * es, out.data(), es);
    return;
  }
  int64_t idx = 0;
  int depth = 0;
  while (true) {
    c.ws();
    char ch = c.s[c.p];
    if (ch == '[') { ++depth; ++c.p; continue; }
    if (ch == ']') { --depth; ++c.p; if (depth == 0) break; continue; }
    if (ch == ',') { ++c.p; continue; }
    if (idx >= n) c.fail("too many dense elements");
    scalar(idx++);
  }
  if (idx != n) c.fail("dense element count " + std::to_string(idx) + " != " + std::to_string(n));
}

AffineMapIR parse_affine_map_body(Cursor& c) {
  // (d0, d1, ...) -> (exprs)
  AffineMapIR m;
  std::unordered_map<std::string, int> dimidx;
  c.expect("(");
  if (!c.accept(")")) {
    while (true) {
      std::string d = c.ident();
      dimidx[d] = m.n_dims++;
      if (c.accept(")")) break;
      c.expect(",");
    }
  }
  if (c.accept("[")) {  // symbols are not supported
    c.fail("affine map symbols are not supported");
  }
  c.expect("->");
  c.expect("(");
  if (!c.accept(")")) {
    while (true) {
      c.ws();
      if (std::isdigit((unsigned char)c.s[c.p]) || c.s[c.p] == '-') {
        int64_t v = c.integer();
        m.exprs.push_back(AffineMapIR::constant(v));
      } else {
        std::string d = c.ident();
        auto it = dimidx.find(d);
        if (it == dimidx.end()) c.fail("unknown affine dim " + d);
        m.exprs.push_back(it->second);
      }
      if (c.accept(")")) break;
      if (!c.accept(",")) c.fail("only plain dims and constants are supported in affine maps");
    }
  }
  return m;
}

struct Parser {
  Cursor c;
  Graph g;
  std::unordered_map<std::string, AffineMapIR> map_aliases;
  std::unordered_map<std::string, int> scope;  // ssa name -> value id

  explicit Parser(const std::string& text) : c(text) {}

  int lookup(const std::string& name) {
    auto it = scope.find(name);
    if (it == scope.end()) c.fail("use of undefined value " + name);
    return it->second;
  }

  Attr parse_attr_value() {
    Attr a;
    c.ws();
    if (c.accept("array<")) {
      DType t = parse_scalar_type(c);
      if (c.accept(":")) {
        while (true) {
          double f; int64_t i; bool ii, hx;
          if (!c.number(f, i, ii, hx)) c.fail("expected array element");
          if (is_float(t)) a.floats.push_back(ii ? (double)i : f); else a.ints.push_back(i);
          if (!c.accept(",")) break;
        }
      }
      c.expect(">");
      a.kind = is_float(t) ? Attr::FLOATS : Attr::INTS;
      return a;
    }
    if (c.accept("true")) { a.kind = Attr::BOOL; a.b = true; a.ty = DType::I1; return a; }
    if (c.accept("false")) { a.kind = Attr::BOOL; a.b = false; a.ty = DType::I1; return a; }
    if (c.peek() == '"') {
      a.kind = Attr::STR;
      a.s = c.string_lit();
      if (c.accept(":")) parse_type(c);
      return a;
    }
    if (c.accept("unit")) { a.kind = Attr::UNIT; return a; }
    if (c.peek() == '[') {
      // list: ints, strings ("parallel"), #linalg.iterator_type<...>, #map refs
      ++c.p;
      a.kind = Attr::INTS;
      std::vector<std::string> strs;
      if (!c.accept("]")) {
        while (true) {
          c.ws();
          if (c.s[c.p] == '"') {
            strs.push_back(c.string_lit());
          } else if (c.accept("#linalg.iterator_type<")) {
            strs.push_back(c.ident());
            c.expect(">");
          } else if (c.starts("affine_map<")) {
            c.expect("affine_map<");
            parse_affine_map_body(c);
            c.expect(">");
          } else if (c.s[c.p] == '#') {
            ++c.p;
            strs.push_back("#" + c.ident());
          } else {
            double f; int64_t i; bool ii, hx;
            if (!c.number(f, i, ii, hx)) c.fail("unsupported list element");
            if (ii) a.ints.push_back(i); else { a.kind = Attr::FLOATS; a.floats.push_back(f); }
            if (c.accept(":")) parse_scalar_type(c);
          }
          if (c.accept("]")) break;
          c.expect(",");
        }
      }
      if (!strs.empty()) {
        a.kind = Attr::STR;
        for (size_t k = 0; k < strs.size(); ++k) a.s += (k ? "," : "") + strs[k];
      }
      return a;
    }
    if (c.accept("dense<")) {
      // payload parsed after we know the type; remember the position
      size_t pos = c.p;
      int depth = 1;
      bool in_str = false;
      while (c.p < c.s.size() && depth > 0) {
        char ch = c.s[c.p];
        if (ch == '"') in_str = !in_str;
        if (!in_str) { if (ch == '<') ++depth; else if (ch == '>') --depth; }
        ++c.p;
      }
      c.expect(":");
      TensorType tt = parse_type(c);
      size_t end = c.p;
      c.p = pos;
      std::vector<uint8_t> data;
      parse_dense_payload(c, tt, data);
      c.expect(">");
      c.p = end;
      a.kind = Attr::DENSE;
      a.s.assign((const char*)data.data(), data.size());
      a.ints = tt.shape;
      a.i = (int64_t)tt.dtype;
      return a;
    }
    double f; int64_t i; bool ii, hx;
    if (c.number(f, i, ii, hx)) {
      a.kind = ii ? Attr::INT : Attr::FLOAT;
      a.i = i; a.f = ii ? (double)i : f;
      if (c.accept(":")) {
        DType t = parse_scalar_type(c);
        a.typed = true;
        a.ty = t;
        if (is_float(t)) {
          a.kind = Attr::FLOAT;
          if (hx) {
            if (t == DType::F32) { uint32_t u = (uint32_t)i; float x; std::memcpy(&x, &u, 4); a.f = x; }
            else { uint64_t u = (uint64_t)i; double x; std::memcpy(&x, &u, 8); a.f = x; }
          } else if (ii) a.f = (double)i;
        }
      }
      return a;
    }
    if (c.peek() == '#') {
      ++c.p;
      std::string id = c.ident();
      a.kind = Attr::STR;
      a.s = "#" + id;
      if (c.accept("<")) {  // e.g. #linalg.iterator_type<parallel>
        a.s += "<" + c.ident() + ">";
        c.expect(">");
      }
      return a;
    }
    if (c.starts("affine_map<")) {
      c.expect("affine_map<");
      parse_affine_map_body(c);
      c.expect(">");
      a.kind = Attr::STR;
      a.s = "affine_map";
      return a;
    }
    c.fail("unsupported attribute value");
  }

  void parse_attr_dict(std::map<std::string, Attr>& out, const char* close) {
    if (c.accept(close)) return;
    while (true) {
      std::string key;
      c.ws();
      if (c.s[c.p] == '"') key = c.string_lit(); else key = c.ident();
      if (c.accept("=")) out[key] = parse_attr_value();
      else { Attr u; u.kind = Attr::UNIT; out[key] = u; }
      if (c.accept(close)) break;
      c.expect(",");
    }
  }

  int new_value(const std::string& name, const TensorType& t, int def_node, int def_result) {
    Value v;
    v.name = name;
    v.type = t;
    v.def_node = def_node;
    v.def_result = def_result;
    int id = g.add_value(v);
    scope[name] = id;
    return id;
  }

  // results: "%a" or "%a:N" or "%a, %b"
  std::vector<std::string> parse_result_names() {
    std::vector<std::string> names;
    while (true) {
      std::string r = c.ssa();
      if (c.accept(":")) {
        int64_t n = c.integer();
        for (int64_t k = 0; k < n; ++k) names.push_back(r + "#" + std::to_string(k));
      } else {
        names.push_back(r);
      }
      if (!c.accept(",")) break;
    }
    c.expect("=");
    return names;
  }

  void bind_results(const std::vector<std::string>& names, int node, const std::vector<TensorType>& types) {
    if (names.size() != types.size()) c.fail("result count does not match the result types");
    for (size_t k = 0; k < names.size(); ++k) {
      int id = new_value(names[k], types[k], node, (int)k);
      g.nodes[node].outs.push_back(id);
      if (names.size() > 1 && names[k].find('#') == std::string::npos) scope[names[k]] = id;
    }
    if (names.size() > 1) {
      // also bind "%r#k" spellings when results were declared as "%r:N"
      for (size_t k = 0; k < names.size(); ++k) scope[names[k]] = g.nodes[node].outs[k];
    }
  }

  std::vector<TensorType> parse_type_list_paren() {
    std::vector<TensorType> ts;
    c.expect("(");
    if (c.accept(")")) return ts;
    while (true) {
      ts.push_back(parse_type(c));
      if (c.accept(")")) break;
      c.expect(",");
    }
    return ts;
  }

  std::vector<TensorType> parse_result_types() {
    if (c.peek() == '(') return parse_type_list_paren();
    return {parse_type(c)};
  }

  // ---- scalar region bodies ------------------------------------------------
  // Parses `^bb0(%a: T, ...):` (or a bare `(%a: T, ...)` header for
  // linalg.reduce) and the ops up to linalg.yield into an EProgram.
  void parse_body(EProgram& prog, bool header_has_bb) {
    std::unordered_map<std::string, int> regs;
    std::unordered_map<std::string, DType> outer_scalars;
    if (header_has_bb) {
      c.expect("{");
      c.expect("^");
      c.ident();
    }
    c.expect("(");
    if (!c.accept(")")) {
      while (true) {
        std::string n = c.ssa();
        c.expect(":");
        TensorType t = parse_type(c);
        regs[n] = prog.add_reg(t.dtype);
        if (c.accept(")")) break;
        c.expect(",");
      }
    }
    prog.n_args = (int)prog.reg_types.size();
    if (header_has_bb) c.expect(":"); else c.expect("{");

    auto reg_of = [&](const std::string& name) -> int {
      auto it = regs.find(name);
      if (it != regs.end()) return it->second;
      // captured outer scalar constant
      auto sit = scope.find(name);
      if (sit != scope.end()) {
        const Value& v = g.values[sit->second];
        if (v.is_const && (!v.type.is_tensor || v.type.numel() == 1)) {
          EInstr in;
          in.op = EOp::CONST;
          in.ty = in.rty = v.type.dtype;
          if (is_float(v.type.dtype)) in.fimm = const_as_double(v, 0); else in.iimm = const_as_int(v, 0);
          in.dst = (int16_t)prog.add_reg(v.type.dtype);
          prog.code.push_back(in);
          regs[name] = in.dst;
          return in.dst;
        }
      }
      c.fail("body uses unsupported value " + name);
    };

    while (true) {
      c.ws();
      if (c.accept("linalg.yield")) {
        std::string y = c.ssa();
        prog.result = reg_of(y);
        c.expect(":");
        parse_type(c);
        c.expect("}");
        break;
      }
      std::string res = c.ssa();
      c.expect("=");
      std::string opn = c.ident();
      EInstr in;
      auto bin = [&](EOp op) {
        std::string a = c.ssa(); c.expect(","); std::string b = c.ssa();
        if (c.accept("fastmath<")) { c.ident(); c.expect(">"); }
        c.expect(":");
        DType t = parse_scalar_type(c);
        in.op = op; in.ty = in.rty = t; in.a = (int16_t)reg_of(a); in.b = (int16_t)reg_of(b);
      };
      auto un = [&](EOp op) {
        std::string a = c.ssa();
        if (c.accept("fastmath<")) { c.ident(); c.expect(">"); }
        c.expect(":");
        DType t = parse_scalar_type(c);
        in.op = op; in.ty = in.rty = t; in.a = (int16_t)reg_of(a);
      };
      auto cast = [&](EOp op) {
        std::string a = c.ssa();
        c.expect(":");
        DType t = parse_scalar_type(c);
        c.expect("to");
        DType r = parse_scalar_type(c);
        in.op = op; in.ty = t; in.rty = r; in.a = (int16_t)reg_of(a);
      };
      static const std::unordered_map<std::string, EOp> binops = {
          {"arith.addf", EOp::ADDF}, {"arith.subf", EOp::SUBF}, {"arith.mulf", EOp::MULF},
          {"arith.divf", EOp::DIVF}, {"arith.remf", EOp::REMF}, {"arith.maximumf", EOp::MAXIMUMF},
          {"arith.minimumf", EOp::MINIMUMF}, {"arith.maxnumf", EOp::MAXNUMF}, {"arith.minnumf", EOp::MINNUMF},
          {"math.powf", EOp::POWF}, {"arith.addi", EOp::ADDI}, {"arith.subi", EOp::SUBI},
          {"arith.muli", EOp::MULI}, {"arith.divsi", EOp::DIVSI}, {"arith.remsi", EOp::REMSI},
          {"arith.maxsi", EOp::MAXSI}, {"arith.minsi", EOp::MINSI}, {"arith.andi", EOp::ANDI},
          {"arith.ori", EOp::ORI}, {"arith.xori", EOp::XORI}};
      static const std::unordered_map<std::string, EOp> unops = {
          {"arith.negf", EOp::NEGF}, {"math.sqrt", EOp::SQRT}, {"math.rsqrt", EOp::RSQRT},
          {"math.exp", EOp::EXP}, {"math.log", EOp::LOG}, {"math.erf", EOp::ERF}, {"math.tanh", EOp::TANH},
          {"math.sin", EOp::SIN}, {"math.cos", EOp::COS}, {"math.absf", EOp::ABSF},
          {"math.floor", EOp::FLOOR}, {"math.ceil", EOp::CEIL}};
      static const std::unordered_map<std::string, EOp> castops = {
          {"arith.sitofp", EOp::SITOFP}, {"arith.uitofp", EOp::UITOFP}, {"arith.fptosi", EOp::FPTOSI},
          {"arith.extf", EOp::EXTF}, {"arith.truncf", EOp::TRUNCF}, {"arith.extsi", EOp::EXTSI},
          {"arith.extui", EOp::EXTUI}, {"arith.trunci", EOp::TRUNCI}, {"arith.index_cast", EOp::INDEX_CAST}};
      if (binops.count(opn)) {
        bin(binops.at(opn));
      } else if (unops.count(opn)) {
        un(unops.at(opn));
      } else if (castops.count(opn)) {
        cast(castops.at(opn));
      } else if (opn == "arith.cmpf" || opn == "arith.cmpi") {
        std::string pr = c.ident();
        c.expect(",");
        static const char* fp[] = {"false", "oeq", "ogt", "oge", "olt", "ole", "one", "ord",
                                   "ueq", "ugt", "uge", "ult", "ule", "une", "uno", "true"};
        static const char* ip[] = {"eq", "ne", "slt", "sle", "sgt", "sge", "ult", "ule", "ugt", "uge"};
        int pi = -1;
        if (opn == "arith.cmpf") { for (int k = 0; k < 16; ++k) if (pr == fp[k]) pi = k; }
        else { for (int k = 0; k < 10; ++k) if (pr == ip[k]) pi = k; }
        if (pi < 0) c.fail("unknown predicate " + pr);
        bin(opn == "arith.cmpf" ? EOp::CMPF : EOp::CMPI);
        in.rty = DType::I1;
        in.pred = (int8_t)pi;
      } else if (opn == "arith.select") {
        std::string a = c.ssa(); c.expect(","); std::string b = c.ssa(); c.expect(","); std::string d = c.ssa();
        c.expect(":");
        DType t = parse_scalar_type(c);
        in.op = EOp::SELECT; in.ty = in.rty = t;
        in.a = (int16_t)reg_of(a); in.b = (int16_t)reg_of(b); in.c = (int16_t)reg_of(d);
      } else if (opn == "arith.constant") {
        Attr a = parse_attr_value();
        DType t = DType::F32;
        if (a.kind == Attr::BOOL) { t = DType::I1; in.iimm = a.b; }
        else if (a.typed) t = a.ty;
        else if (c.accept(":")) t = parse_scalar_type(c);
        else c.fail("untyped constant in linalg body");
        in.op = EOp::CONST; in.ty = in.rty = t;
        if (a.kind == Attr::FLOAT) { in.fimm = a.f; in.iimm = (int64_t)a.f; }
        else if (a.kind == Attr::INT) { in.iimm = a.i; in.fimm = (double)a.i; if (is_float(t)) in.fimm = a.f; }
        if (a.kind == Attr::FLOAT && !is_float(t)) c.fail("float constant with integer type");
        if (a.kind == Attr::INT && is_float(t)) in.fimm = a.f;
      } else {
        c.fail("unsupported op in linalg body: " + opn);
      }
      in.dst = (int16_t)prog.add_reg(in.rty);
      prog.code.push_back(in);
      regs[res] = in.dst;
    }
  }

  void parse_ins_outs(Node& n, const char* kw, bool is_ins) {
    c.expect(kw);
    c.expect("(");
    std::vector<std::string> names;
    if (!c.accept(")")) {
      while (true) {
        names.push_back(c.ssa());
        if (c.accept(":")) break;
        c.expect(",");
      }
      for (size_t k = 0; k < names.size(); ++k) {
        parse_type(c);
        if (k + 1 < names.size()) c.expect(",");
      }
      c.expect(")");
    }
    for (auto& nm : names) n.ins.push_back(lookup(nm));
    if (is_ins) n.n_linalg_ins = (int)names.size();
  }

  AffineMapIR resolve_map(const std::string& ref) {
    auto it = map_aliases.find(ref);
    if (it == map_aliases.end()) c.fail("unknown affine map alias " + ref);
    return it->second;
  }

  void parse_op_stmt() {
    std::vector<std::string> results = parse_result_names();
    c.ws();
    int node = (int)g.nodes.size();
    if (c.peek() == '"') {
      // generic operation form
      Node n;
      n.op = c.string_lit();
      c.expect("(");
      if (!c.accept(")")) {
        while (true) {
          n.ins.push_back(lookup(c.ssa()));
          if (c.accept(")")) break;
          c.expect(",");
        }
      }
      if (c.accept("<{")) parse_attr_dict(n.attrs, "}>");
      if (c.accept("{")) parse_attr_dict(n.attrs, "}");
      c.expect(":");
      parse_type_list_paren();
      c.expect("->");
      std::vector<TensorType> rt = parse_result_types();
      if (n.op == "arith.constant") {
        const Attr& a = n.attrs.at("value");
        make_constant(results, a, rt.at(0));
        return;
      }
      g.nodes.push_back(n);
      bind_results(results, node, rt);
      return;
    }
    std::string opn = c.ident();
    if (opn == "arith.constant") {
      Attr a = parse_attr_value();
      TensorType t;
      if (a.kind == Attr::DENSE) {
        t.dtype = (DType)a.i;
        t.shape = a.ints;
        t.is_tensor = true;
      } else if (a.kind == Attr::BOOL) {
        t.dtype = DType::I1;
        t.is_tensor = false;
        if (c.accept(":")) t = parse_type(c);
      } else if (a.typed) {
        t.dtype = a.ty;
        t.is_tensor = false;
      } else {
        c.expect(":");
        t = parse_type(c);
      }
      make_constant(results, a, t);
      return;
    }
    Node n;
    n.op = opn;
    if (opn == "tensor.empty") {
      c.expect("(");
      c.expect(")");
      c.expect(":");
      TensorType t = parse_type(c);
      g.nodes.push_back(n);
      bind_results(results, node, {t});
      return;
    }
    if (opn == "linalg.fill") {
      parse_ins_outs(n, "ins", true);
      parse_ins_outs(n, "outs", false);
      c.expect("->");
      TensorType t = parse_type(c);
      g.nodes.push_back(n);
      bind_results(results, node, {t});
      return;
    }
    if (opn == "linalg.generic") {
      std::map<std::string, Attr> attrs;
      c.expect("{");
      // indexing_maps / iterator_types: keep the raw alias list
      while (true) {
        std::string key = c.ident();
        c.expect("=");
        if (key == "indexing_maps") {
          c.expect("[");
          while (true) {
            c.ws();
            if (c.starts("affine_map<")) {
              c.expect("affine_map<");
              n.maps.push_back(parse_affine_map_body(c));
              c.expect(">");
            } else {
              c.expect("#");
              n.maps.push_back(resolve_map("#" + c.ident()));
            }
            if (c.accept("]")) break;
            c.expect(",");
          }
        } else if (key == "iterator_types") {
          Attr it = parse_attr_value();
          std::stringstream ss(it.s);
          std::string item;
          while (std::getline(ss, item, ',')) n.parallel.push_back(item.find("parallel") != std::string::npos);
        } else {
          parse_attr_value();
        }
        if (c.accept("}")) break;
        c.expect(",");
      }
      parse_ins_outs(n, "ins", true);
      parse_ins_outs(n, "outs", false);
      if (c.starts("attrs")) { c.expect("attrs"); c.expect("="); c.expect("{"); parse_attr_dict(n.attrs, "}"); }
      parse_body(n.body, true);
      c.expect("->");
      std::vector<TensorType> rt = parse_result_types();
      if (n.maps.size() != n.ins.size()) c.fail("indexing_maps count does not match operands");
      g.nodes.push_back(n);
      bind_results(results, node, rt);
      return;
    }
    if (opn == "linalg.reduce") {
      parse_ins_outs(n, "ins", true);
      parse_ins_outs(n, "outs", false);
      c.expect("dimensions");
      c.expect("=");
      Attr d = parse_attr_value();
      n.dims = d.ints;
      parse_body(n.body, false);
      std::vector<TensorType> rt;
      for (size_t k = n.n_linalg_ins; k < n.ins.size(); ++k) rt.push_back(g.values[n.ins[k]].type);
      g.nodes.push_back(n);
      bind_results(results, node, rt);
      return;
    }
    c.fail("unsupported operation '" + opn + "'");
  }

  void make_constant(const std::vector<std::string>& results, const Attr& a, const TensorType& t) {
    if (results.size() != 1) c.fail("arith.constant has one result");
    Value v;
    v.name = results[0];
    v.type = t;
    v.is_const = true;
    size_t es = dtype_size(t.dtype);
    int64_t n = t.is_tensor ? t.numel() : 1;
    v.data.assign((size_t)n * es, 0);
    if (a.kind == Attr::DENSE) {
      if (a.s.size() != v.data.size()) c.fail("dense payload size mismatch");
      std::memcpy(v.data.data(), a.s.data(), a.s.size());
    } else {
      for (int64_t k = 0; k < n; ++k) {
        uint8_t* p = v.data.data() + k * es;
        switch (t.dtype) {
          case DType::F32: { float x = (float)(a.kind == Attr::INT ? (double)a.i : a.f); std::memcpy(p, &x, 4); break; }
          case DType::F64: { double x = a.kind == Attr::INT ? (double)a.i : a.f; std::memcpy(p, &x, 8); break; }
          case DType::I64: case DType::INDEX: { int64_t x = a.kind == Attr::BOOL ? a.b : a.i; std::memcpy(p, &x, 8); break; }
          case DType::I32: { int32_t x = (int32_t)a.i; std::memcpy(p, &x, 4); break; }
          case DType::I1: p[0] = a.kind == Attr::BOOL ? a.b : (a.i != 0); break;
          default: c.fail("unsupported constant type");
        }
      }
    }
    int id = g.add_value(v);
    scope[results[0]] = id;
  }

  void parse_function_body() {
    c.expect("{");
    while (true) {
      c.ws();
      if (c.accept("}")) break;
      if (c.starts("return") || c.starts("func.return")) {
        if (!c.accept("func.return")) c.expect("return");
        std::vector<std::string> names;
        if (c.peek() == '%') {
          while (true) {
            names.push_back(c.ssa());
            if (!c.accept(",")) break;
          }
          c.expect(":");
          for (size_t k = 0; k < names.size(); ++k) {
            parse_type(c);
            if (k + 1 < names.size()) c.expect(",");
          }
        }
        for (auto& nm : names) g.results.push_back(lookup(nm));
        continue;
      }
      if (c.starts("\"func.return\"")) {
        c.string_lit();
        c.expect("(");
        if (!c.accept(")")) {
          while (true) {
            g.results.push_back(lookup(c.ssa()));
            if (c.accept(")")) break;
            c.expect(",");
          }
        }
        c.expect(":");
        parse_type_list_paren();
        c.expect("->");
        c.expect("(");
        c.expect(")");
        continue;
      }
      parse_op_stmt();
    }
  }

  void skip_balanced(char open, char close) {
    c.ws();
    if (c.s[c.p] != open) c.fail(std::string("expected '") + open + "'");
    int depth = 0;
    bool in_str = false;
    while (c.p < c.s.size()) {
      char ch = c.s[c.p++];
      if (ch == '"') in_str = !in_str;
      if (in_str) continue;
      if (ch == open) ++depth;
      else if (ch == close && --depth == 0) return;
    }
    c.fail("unbalanced block");
  }

  Graph run(const std::string& entry) {
    g.entry = entry;
    bool found = false;
    while (!c.eof()) {
      c.ws();
      if (c.s[c.p] == '#') {
        ++c.p;
        std::string alias = "#" + c.ident();
        c.expect("=");
        if (c.accept("affine_map<")) {
          map_aliases[alias] = parse_affine_map_body(c);
          c.expect(">");
        } else {
          // other attribute aliases are not needed by the forward function
          while (c.p < c.s.size() && c.s[c.p] != '\n') ++c.p;
        }
        continue;
      }
      if (c.accept("{-#")) {  // dialect resources: skip
        size_t e = c.s.find("#-}", c.p);
        if (e == std::string::npos) c.fail("unterminated resource block");
        c.p = e + 3;
        continue;
      }
      if (c.accept("module")) {
        if (c.starts("@")) { ++c.p; c.ident(); }
        if (c.accept("attributes")) skip_balanced('{', '}');
        c.expect("{");
        continue;
      }
      if (c.accept("}")) continue;
      if (c.accept("func.func")) {
        c.accept("private");
        c.expect("@");
        std::string name = c.ident();
        if (name != entry) {
          // skip signature + body of other functions
          skip_balanced('(', ')');
          while (c.p < c.s.size() && c.s[c.p] != '{' && c.s[c.p] != '\n') ++c.p;
          c.ws();
          if (c.s[c.p] == '{') skip_balanced('{', '}');
          continue;
        }
        found = true;
        c.expect("(");
        if (!c.accept(")")) {
          while (true) {
            std::string an = c.ssa();
            c.expect(":");
            TensorType t = parse_type(c);
            if (c.peek() == '{') skip_balanced('{', '}');  // argument attributes
            Value v;
            v.name = an;
            v.type = t;
            v.arg_index = (int)g.args.size();
            int id = g.add_value(v);
            scope[an] = id;
            g.args.push_back(id);
            if (c.accept(")")) break;
            c.expect(",");
          }
        }
        if (c.accept("->")) {
          c.ws();
          if (c.s[c.p] == '(') parse_type_list_paren(); else parse_type(c);
        }
        if (c.accept("attributes")) {
          std::map<std::string, Attr> fa;
          c.expect("{");
          parse_attr_dict(fa, "}");
          auto it = fa.find("gawee.onnx_source");
          if (it != fa.end()) g.onnx_source = it->second.s;
        }
        parse_function_body();
        continue;
      }
      c.fail("unexpected top-level text");
    }
    if (!found) throw ParseError("function @" + entry + " not found");
    if (g.results.empty()) throw ParseError("function @" + entry + " returns nothing");
    return std::move(g);
  }
};

}  // namespace

Graph parse_mlir(const std::string& text, const std::string& entry) {
  Parser p(text);
  return p.run(entry);
}

}  // namespace gawee
