// Device interpreter for scalar op programs (gawee::EProgram lowered to
// kern::DProgram).  Semantics follow the MLIR arith/math ops the reference
// lowers to: IEEE fp32 add/sub/mul/div/sqrt (no fast-math), NaN-propagating
// maximumf/minimumf, CUDA libdevice expf/erff/tanhf/sinf/cosf/powf for the
// libm calls, wrapping integer arithmetic, truncating fp->int conversion.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "kernels.h"

namespace gawee {
namespace kern {

union Reg {
  float f;
  double d;
  long long i;
};

// Opcode numbering: must match gawee::EOp.
enum DOp : uint8_t {
  O_CONST = 0,
  O_ADDF, O_SUBF, O_MULF, O_DIVF, O_REMF, O_MAXIMUMF, O_MINIMUMF, O_MAXNUMF, O_MINNUMF, O_POWF,
  O_NEGF, O_SQRT, O_RSQRT, O_EXP, O_LOG, O_ERF, O_TANH, O_SIN, O_COS, O_ABSF, O_FLOOR, O_CEIL,
  O_ADDI, O_SUBI, O_MULI, O_DIVSI, O_REMSI, O_MAXSI, O_MINSI, O_ANDI, O_ORI, O_XORI,
  O_CMPF, O_CMPI,
  O_SELECT,
  O_SITOFP, O_UITOFP, O_FPTOSI, O_EXTF, O_TRUNCF, O_EXTSI, O_EXTUI, O_TRUNCI, O_INDEX_CAST,
  O_COPY
};

__device__ __forceinline__ float maximumf_(float a, float b) {
  if (isnan(a) || isnan(b)) return __int_as_float(0x7fc00000);
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
__device__ __forceinline__ float minimumf_(float a, float b) {
  if (isnan(a) || isnan(b)) return __int_as_float(0x7fc00000);
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}
__device__ __forceinline__ double maximumd_(double a, double b) {
  if (isnan(a) || isnan(b)) return __longlong_as_double(0x7ff8000000000000ll);
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
__device__ __forceinline__ double minimumd_(double a, double b) {
  if (isnan(a) || isnan(b)) return __longlong_as_double(0x7ff8000000000000ll);
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}

__device__ __forceinline__ long long wrap_(long long v, int t) {
  if (t == DT_I32) return (long long)(int)(unsigned)(unsigned long long)v;
  if (t == DT_I1) return v & 1;
  return v;
}

__device__ __forceinline__ bool cmpf_(int pred, double a, double b) {
  bool uno = isnan(a) || isnan(b);
  switch (pred) {
    case 0: return false;
    case 1: return !uno && a == b;
    case 2: return !uno && a > b;
    case 3: return !uno && a >= b;
    case 4: return !uno && a < b;
    case 5: return !uno && a <= b;
    case 6: return !uno && a != b;
    case 7: return !uno;
    case 8: return uno || a == b;
    case 9: return uno || a > b;
    case 10: return uno || a >= b;
    case 11: return uno || a < b;
    case 12: return uno || a <= b;
    case 13: return uno || a != b;
    case 14: return uno;
    default: return true;
  }
}

__device__ __forceinline__ bool cmpi_(int pred, long long a, long long b, int t) {
  unsigned long long ua = (unsigned long long)a, ub = (unsigned long long)b;
  if (t == DT_I32) { ua &= 0xffffffffull; ub &= 0xffffffffull; }
  if (t == DT_I1) { ua &= 1; ub &= 1; }
  switch (pred) {
    case 0: return a == b;
    case 1: return a != b;
    case 2: return a < b;
    case 3: return a <= b;
    case 4: return a > b;
    case 5: return a >= b;
    case 6: return ua < ub;
    case 7: return ua <= ub;
    case 8: return ua > ub;
    default: return ua >= ub;
  }
}

__device__ __forceinline__ Reg load_dt(const void* base, long long off, int dt) {
  Reg r;
  r.i = 0;
  switch (dt) {
    case DT_F32: r.f = static_cast<const float*>(base)[off]; break;
    case DT_F64: r.d = static_cast<const double*>(base)[off]; break;
    case DT_I64: case DT_INDEX: r.i = static_cast<const long long*>(base)[off]; break;
    case DT_I32: r.i = static_cast<const int*>(base)[off]; break;
    case DT_I1: r.i = static_cast<const unsigned char*>(base)[off] ? 1 : 0; break;
    default: break;
  }
  return r;
}

__device__ __forceinline__ void store_dt(void* base, long long off, int dt, Reg r) {
  switch (dt) {
    case DT_F32: static_cast<float*>(base)[off] = r.f; break;
    case DT_F64: static_cast<double*>(base)[off] = r.d; break;
    case DT_I64: case DT_INDEX: static_cast<long long*>(base)[off] = r.i; break;
    case DT_I32: static_cast<int*>(base)[off] = (int)r.i; break;
    case DT_I1: static_cast<unsigned char*>(base)[off] = (r.i & 1) ? 1 : 0; break;
    default: break;
  }
}

// Runs `prog` over the register file; returns the result register.
// `err` receives a status code on integer division by zero / bad opcode.
__device__ __forceinline__ Reg run_program(const DProgram& pg, Reg* r, int* err) {
  for (int k = 0; k < pg.n_code; ++k) {
    const DInstr in = pg.code[k];
    Reg a = in.a >= 0 ? r[in.a] : Reg{0}, b = in.b >= 0 ? r[in.b] : Reg{0};
    Reg o;
    o.i = 0;
    const bool f32 = in.ty == DT_F32;
    switch (in.op) {
      case O_CONST:
        if (in.rty == DT_F32) o.f = (float)in.fimm;
        else if (in.rty == DT_F64) o.d = in.fimm;
        else o.i = wrap_(in.iimm, in.rty);
        break;
      case O_ADDF: if (f32) o.f = __fadd_rn(a.f, b.f); else o.d = __dadd_rn(a.d, b.d); break;
      case O_SUBF: if (f32) o.f = __fsub_rn(a.f, b.f); else o.d = __dsub_rn(a.d, b.d); break;
      case O_MULF: if (f32) o.f = __fmul_rn(a.f, b.f); else o.d = __dmul_rn(a.d, b.d); break;
      case O_DIVF: if (f32) o.f = __fdiv_rn(a.f, b.f); else o.d = __ddiv_rn(a.d, b.d); break;
      case O_REMF: if (f32) o.f = fmodf(a.f, b.f); else o.d = fmod(a.d, b.d); break;
      case O_MAXIMUMF: if (f32) o.f = maximumf_(a.f, b.f); else o.d = maximumd_(a.d, b.d); break;
      case O_MINIMUMF: if (f32) o.f = minimumf_(a.f, b.f); else o.d = minimumd_(a.d, b.d); break;
      case O_MAXNUMF: if (f32) o.f = fmaxf(a.f, b.f); else o.d = fmax(a.d, b.d); break;
      case O_MINNUMF: if (f32) o.f = fminf(a.f, b.f); else o.d = fmin(a.d, b.d); break;
      case O_POWF:
        if (f32) o.f = (b.f == 2.0f) ? __fmul_rn(a.f, a.f) : powf(a.f, b.f);
        else o.d = pow(a.d, b.d);
        break;
      case O_NEGF: if (f32) o.f = -a.f; else o.d = -a.d; break;
      case O_SQRT: if (f32) o.f = __fsqrt_rn(a.f); else o.d = __dsqrt_rn(a.d); break;
      case O_RSQRT: if (f32) o.f = __fdiv_rn(1.0f, __fsqrt_rn(a.f)); else o.d = 1.0 / __dsqrt_rn(a.d); break;
      case O_EXP: if (f32) o.f = expf(a.f); else o.d = exp(a.d); break;
      case O_LOG: if (f32) o.f = logf(a.f); else o.d = log(a.d); break;
      case O_ERF: if (f32) o.f = erff(a.f); else o.d = erf(a.d); break;
      case O_TANH: if (f32) o.f = tanhf(a.f); else o.d = tanh(a.d); break;
      case O_SIN: if (f32) o.f = sinf(a.f); else o.d = sin(a.d); break;
      case O_COS: if (f32) o.f = cosf(a.f); else o.d = cos(a.d); break;
      case O_ABSF: if (f32) o.f = fabsf(a.f); else o.d = fabs(a.d); break;
      case O_FLOOR: if (f32) o.f = floorf(a.f); else o.d = floor(a.d); break;
      case O_CEIL: if (f32) o.f = ceilf(a.f); else o.d = ceil(a.d); break;
      case O_ADDI: o.i = wrap_((long long)((unsigned long long)a.i + (unsigned long long)b.i), in.ty); break;
      case O_SUBI: o.i = wrap_((long long)((unsigned long long)a.i - (unsigned long long)b.i), in.ty); break;
      case O_MULI: o.i = wrap_((long long)((unsigned long long)a.i * (unsigned long long)b.i), in.ty); break;
      case O_DIVSI:
        if (b.i == 0) { *err = ST_INT_DIV_ZERO; o.i = 0; } else o.i = wrap_(a.i / b.i, in.ty);
        break;
      case O_REMSI:
        if (b.i == 0) { *err = ST_INT_DIV_ZERO; o.i = 0; } else o.i = wrap_(a.i % b.i, in.ty);
        break;
      case O_MAXSI: o.i = a.i > b.i ? a.i : b.i; break;
      case O_MINSI: o.i = a.i < b.i ? a.i : b.i; break;
      case O_ANDI: o.i = a.i & b.i; break;
      case O_ORI: o.i = a.i | b.i; break;
      case O_XORI: o.i = wrap_(a.i ^ b.i, in.ty); break;
      case O_CMPF: o.i = cmpf_(in.pred, f32 ? (double)a.f : a.d, f32 ? (double)b.f : b.d); break;
      case O_CMPI: o.i = cmpi_(in.pred, a.i, b.i, in.ty); break;
      case O_SELECT: o = (a.i & 1) ? b : r[in.c]; break;
      case O_SITOFP: if (in.rty == DT_F32) o.f = (float)a.i; else o.d = (double)a.i; break;
      case O_UITOFP: {
        unsigned long long u = (unsigned long long)a.i;
        if (in.ty == DT_I32) u &= 0xffffffffull;
        if (in.ty == DT_I1) u &= 1;
        if (in.rty == DT_F32) o.f = (float)u; else o.d = (double)u;
        break;
      }
      case O_FPTOSI: o.i = wrap_(f32 ? (long long)a.f : (long long)a.d, in.rty); break;
      case O_EXTF: o.d = (double)a.f; break;
      case O_TRUNCF: o.f = (float)a.d; break;
      case O_EXTSI: o.i = a.i; break;
      case O_EXTUI:
        o.i = in.ty == DT_I1 ? (a.i & 1) : (in.ty == DT_I32 ? (long long)(unsigned)a.i : a.i);
        break;
      case O_TRUNCI: case O_INDEX_CAST: o.i = wrap_(a.i, in.rty); break;
      case O_COPY: o = a; break;
      default: *err = ST_BAD_PROGRAM; break;
    }
    r[in.dst] = o;
  }
  return r[pg.result];
}

}  // namespace kern
}  // namespace gawee
