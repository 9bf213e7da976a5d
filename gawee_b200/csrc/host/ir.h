// Graph IR for one `func.func @forward` of the gawee dialect, and the parser
// that reads it from MLIR text.
//
// The parser accepts what `gawee-onnx-translate` prints
// (middle/mlir/lib/Emit/ONNXMLIREmitter.cpp): `gawee.*` ops in MLIR's generic
// operation syntax (inherent attributes either as `<{...}>` properties or as a
// `{...}` attribute dictionary, as in middle/mlir/test/*.mlir), `arith.constant`,
// `tensor.empty`, `linalg.fill`, `linalg.generic` and `linalg.reduce` with
// scalar arith/math bodies, and `return`.  Shapes must be static, as the
// reference AOT runner also requires (back/eval_priority_models.py:232-239).
#pragma once

#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace gawee {

enum class DType : int32_t { F32 = 0, F64 = 1, F16 = 2, I64 = 3, I32 = 4, I1 = 5, INDEX = 6 };

size_t dtype_size(DType t);       // storage bytes (i1 is one byte, index is 8)
const char* dtype_name(DType t);  // "f32", "i64", ...
inline bool is_float(DType t) { return t == DType::F32 || t == DType::F64 || t == DType::F16; }

struct TensorType {
  DType dtype = DType::F32;
  std::vector<int64_t> shape;
  bool is_tensor = true;  // false for scalar SSA values (body args, scalar constants)
  int64_t numel() const;
  int rank() const { return (int)shape.size(); }
  std::string str() const;
};

// ---------------------------------------------------------------------------
// Scalar expression programs: the bodies of linalg.generic / linalg.reduce and
// the per-element semantics of every elementwise gawee op.
// ---------------------------------------------------------------------------
enum class EOp : uint8_t {
  CONST,
  // float
  ADDF, SUBF, MULF, DIVF, REMF, MAXIMUMF, MINIMUMF, MAXNUMF, MINNUMF, POWF,
  NEGF, SQRT, RSQRT, EXP, LOG, ERF, TANH, SIN, COS, ABSF, FLOOR, CEIL,
  // integer
  ADDI, SUBI, MULI, DIVSI, REMSI, MAXSI, MINSI, ANDI, ORI, XORI,
  // comparisons (predicate in `pred`)
  CMPF, CMPI,
  SELECT,
  // conversions (source type in `ty`, result type in `rty`)
  SITOFP, UITOFP, FPTOSI, EXTF, TRUNCF, EXTSI, EXTUI, TRUNCI, INDEX_CAST,
  COPY,
  COUNT_
};
const char* eop_name(EOp op);

// arith.cmpf predicates (MLIR arith::CmpFPredicate numbering)
enum CmpF : int8_t { CF_FALSE = 0, CF_OEQ, CF_OGT, CF_OGE, CF_OLT, CF_OLE, CF_ONE, CF_ORD,
                     CF_UEQ, CF_UGT, CF_UGE, CF_ULT, CF_ULE, CF_UNE, CF_UNO, CF_TRUE };
// arith.cmpi predicates (MLIR arith::CmpIPredicate numbering)
enum CmpI : int8_t { CI_EQ = 0, CI_NE, CI_SLT, CI_SLE, CI_SGT, CI_SGE, CI_ULT, CI_ULE, CI_UGT, CI_UGE };

struct EInstr {
  EOp op = EOp::COPY;
  DType ty = DType::F32;   // operand type
  DType rty = DType::F32;  // result type
  int8_t pred = 0;
  int16_t dst = -1, a = -1, b = -1, c = -1;  // registers
  double fimm = 0.0;       // CONST float payload
  int64_t iimm = 0;        // CONST integer payload
};

// Registers [0, n_args) hold the block arguments (linalg: inputs then outputs).
struct EProgram {
  int n_args = 0;
  std::vector<DType> reg_types;  // size = number of registers
  std::vector<EInstr> code;
  int result = -1;               // register yielded
  int add_reg(DType t) { reg_types.push_back(t); return (int)reg_types.size() - 1; }
  std::string str() const;
};

// Affine map restricted to what the emitter and lowering produce: each result
// expression is a loop dimension or an integer constant.
struct AffineMapIR {
  int n_dims = 0;
  std::vector<int64_t> exprs;  // >= 0: dimension index; < 0: constant (-1 - value)
  static int64_t constant(int64_t v) { return -1 - v; }
  bool is_identity() const;
};

struct Attr {
  enum Kind { NONE, INT, FLOAT, BOOL, STR, INTS, FLOATS, DENSE, UNIT } kind = NONE;
  int64_t i = 0;
  double f = 0.0;
  bool b = false;
  std::string s;
  std::vector<int64_t> ints;
  std::vector<double> floats;
  bool typed = false;        // a `: type` suffix was present on a scalar literal
  DType ty = DType::F32;
};

struct Value {
  std::string name;
  TensorType type;
  int def_node = -1;     // producing node, -1 for arguments and constants
  int def_result = 0;
  int arg_index = -1;    // >= 0 for func arguments
  bool is_const = false; // arith.constant (payload below, row-major)
  std::vector<uint8_t> data;
};

struct Node {
  std::string op;            // "gawee.conv", "linalg.generic", "linalg.fill", "tensor.empty", ...
  std::vector<int> ins;      // value ids
  std::vector<int> outs;     // value ids (results)
  std::map<std::string, Attr> attrs;
  // linalg.generic / linalg.reduce payload
  int n_linalg_ins = 0;      // first n of `ins` are `ins(...)`, the rest `outs(...)`
  std::vector<AffineMapIR> maps;
  std::vector<bool> parallel;  // iterator types
  std::vector<int64_t> dims;   // linalg.reduce dimensions
  EProgram body;
  bool has_attr(const std::string& k) const { return attrs.count(k) != 0; }
  const Attr& attr(const std::string& k) const;
};

struct Graph {
  std::string entry;
  std::string onnx_source;
  std::vector<Value> values;
  std::vector<Node> nodes;
  std::vector<int> args;     // value ids of func arguments, in order
  std::vector<int> results;  // value ids returned
  int add_value(const Value& v) { values.push_back(v); return (int)values.size() - 1; }
};

struct ParseError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// Parse the function `entry` out of MLIR module text. Throws ParseError.
Graph parse_mlir(const std::string& text, const std::string& entry = "forward");

// Read a whole file; throws std::runtime_error.
std::string read_text_file(const std::string& path);

// Constant payload helpers (row-major, storage dtype of the value).
double const_as_double(const Value& v, int64_t i);
int64_t const_as_int(const Value& v, int64_t i);

}  // namespace gawee
