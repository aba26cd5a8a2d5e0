// Elementwise bytecode shared by the fused elementwise, gather-RMW and
// generic-path kernels.
//
// A program is a straight-line list of KtirInstr over KTIR_NREG 64-bit
// registers.  Float registers (f16 / f32 results) hold a float; integer and
// boolean registers hold an int64.  Every float result whose dtype is f16 is
// rounded to f16 after the operation, which is what NumPy's float16 loops do
// (compute, then one rounding per op), so + - * / on f16 tiles match the
// reference bit for bit; transcendental ops run in f32 and are then rounded,
// as ktir_cpu/ops/math_ops.py does.
#pragma once

#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "../../include/ktir_b200.h"

namespace ktir {

enum Op : uint8_t {
  OP_NOP = 0, OP_LD = 1, OP_ST = 2, OP_IMM = 3, OP_IOTA = 4, OP_CAST = 5, OP_BITCAST = 6,
  OP_FADD = 10, OP_FSUB, OP_FMUL, OP_FDIV, OP_FMOD, OP_FMAXNUM, OP_FMINNUM, OP_FMAXIMUM,
  OP_FMINIMUM, OP_FPOW,
  OP_FNEG = 20, OP_FABS, OP_FEXP, OP_FSQRT, OP_FRSQRT, OP_FLOG, OP_FLOG2, OP_FLOG1P, OP_FTANH,
  OP_FSIN, OP_FCOS, OP_FCEIL, OP_FFLOOR, OP_FERF,
  OP_FFMA = 34, OP_FCMP = 35, OP_SELECT = 36,
  OP_IADD = 40, OP_ISUB, OP_IMUL, OP_IFLOORDIV, OP_IMOD, OP_ITRUNCDIV, OP_ITRUNCREM, OP_ICEILDIV,
  OP_IAND, OP_IOR, OP_IXOR, OP_ISHL, OP_ISHR, OP_ISHRU, OP_IMAX, OP_IMIN, OP_INEG, OP_IABS,
  OP_ICMP = 58,
};

union Reg {
  float f;
  long long i;
};

__device__ __forceinline__ bool is_float(int dt) { return dt == KTIR_F16 || dt == KTIR_F32; }

__device__ __forceinline__ float round_to(float x, int dt) {
  return dt == KTIR_F16 ? __half2float(__float2half_rn(x)) : x;
}

__device__ __forceinline__ long long wrap_to(long long v, int dt) {
  if (dt == KTIR_I32) return (long long)(int)v;
  if (dt == KTIR_U32) return (long long)(unsigned)v;
  if (dt == KTIR_BOOL) return v != 0;
  return v;
}

// element load with the reference's zero fill past the end of the buffer
__device__ __forceinline__ Reg load_elem(const KtirBuffers& b, int slot, int dt, int64_t off) {
  Reg r;
  r.i = 0;
  if (off < 0 || off >= b.numel[slot]) {
    if (is_float(dt)) r.f = 0.f;
    return r;
  }
  const void* p = b.base[slot];
  switch (dt) {
    case KTIR_F16: r.f = __half2float(((const __half*)p)[off]); break;
    case KTIR_F32: r.f = ((const float*)p)[off]; break;
    case KTIR_I32: r.i = ((const int*)p)[off]; break;
    case KTIR_I64: r.i = ((const long long*)p)[off]; break;
    case KTIR_BOOL: r.i = ((const uint8_t*)p)[off] != 0; break;
    case KTIR_U32: r.i = ((const unsigned*)p)[off]; break;
  }
  return r;
}

// element store (register of type reg_dt) with truncation past the buffer end
__device__ __forceinline__ void store_elem(const KtirBuffers& b, int slot, int dt, int64_t off,
                                           Reg v, int reg_dt) {
  if (off < 0 || off >= b.numel[slot]) return;
  void* p = b.base[slot];
  bool fsrc = is_float(reg_dt);
  switch (dt) {
    case KTIR_F16:
      ((__half*)p)[off] = __float2half_rn(fsrc ? v.f : (float)v.i);
      break;
    case KTIR_F32:
      ((float*)p)[off] = fsrc ? v.f : (float)v.i;
      break;
    case KTIR_I32:
      ((int*)p)[off] = fsrc ? (int)v.f : (int)v.i;
      break;
    case KTIR_I64:
      ((long long*)p)[off] = fsrc ? (long long)v.f : v.i;
      break;
    case KTIR_BOOL:
      ((uint8_t*)p)[off] = fsrc ? (v.f != 0.f) : (v.i != 0);
      break;
    case KTIR_U32:
      ((unsigned*)p)[off] = fsrc ? (unsigned)(long long)v.f : (unsigned)v.i;
      break;
  }
}

// NumPy np.remainder for floats: sign of the divisor
__device__ __forceinline__ float py_fmod(float a, float b) {
  float m = fmodf(a, b);
  if (b == 0.f) return m;
  if (m != 0.f) {
    if ((b < 0.f) != (m < 0.f)) m += b;
  } else {
    m = copysignf(0.f, b);
  }
  return m;
}

__device__ __forceinline__ long long py_floordiv(long long a, long long b) {
  if (b == 0) return 0;
  long long q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) --q;
  return q;
}

__device__ __forceinline__ long long py_mod(long long a, long long b) {
  if (b == 0) return 0;
  long long m = a % b;
  if (m != 0 && ((m < 0) != (b < 0))) m += b;
  return m;
}

// Abramowitz-Stegun 7.1.26, the formula ktir_cpu/ops/math_ops.py:220-241 evaluates in f32
__device__ __forceinline__ float as_erf(float x) {
  float a = fabsf(x);
  float t = 1.0f / (1.0f + 0.3275911f * a);
  float poly = t * (0.254829592f + t * (-0.284496736f + t * (1.421413741f +
               t * (-1.453152027f + t * 1.061405429f))));
  float s = (x > 0.f) ? 1.f : ((x < 0.f) ? -1.f : 0.f);
  return s * (1.0f - poly * expf(-a * a));
}

__device__ __forceinline__ bool fcmp(int pred, float x, float y) {
  bool nan = isnan(x) || isnan(y);
  switch (pred) {
    case 0: return false;
    case 1: return x == y;
    case 2: return x > y;
    case 3: return x >= y;
    case 4: return x < y;
    case 5: return x <= y;
    case 6: return (x != y) && !nan;
    case 7: return !nan;
    case 8: return (x == y) || nan;
    case 9: return (x > y) || nan;
    case 10: return (x >= y) || nan;
    case 11: return (x < y) || nan;
    case 12: return (x <= y) || nan;
    case 13: return x != y;
    case 14: return nan;
    default: return true;
  }
}

__device__ __forceinline__ bool icmp(int pred, long long x, long long y) {
  switch (pred) {
    case 0: return x == y;
    case 1: return x != y;
    case 2: case 6: return x < y;
    case 3: case 7: return x <= y;
    case 4: case 8: return x > y;
    default: return x >= y;
  }
}

__device__ __forceinline__ Reg convert(Reg v, int from, int to) {
  Reg r;
  r.i = 0;
  if (is_float(from)) {
    if (is_float(to)) {
      r.f = round_to(v.f, to);
    } else if (to == KTIR_BOOL) {
      r.i = v.f != 0.f;
    } else if (to == KTIR_I32) {
      // NumPy's float -> int32 cast (x86): truncation toward zero, and the
      // integer-indefinite value INT32_MIN for NaN and out-of-range inputs
      r.i = (v.f > -2147483904.f && v.f < 2147483648.f) ? (long long)(int)v.f : (long long)INT32_MIN;
    } else if (to == KTIR_U32) {
      // NumPy's float -> uint32 cast (x86): values below 2^31 go through a
      // signed int32 (negative inputs wrap), [2^31, 2^32) convert directly;
      // other inputs are invalid casts (NumPy warns), given 2^31 here
      r.i = (v.f > -2147483904.f && v.f < 2147483648.f)
                ? (long long)(unsigned)(int)v.f
                : ((v.f >= 2147483648.f && v.f < 4294967296.f) ? (long long)(unsigned)v.f
                                                                 : 2147483648ll);
    } else {
      r.i = wrap_to((long long)v.f, to);
    }
  } else {
    if (is_float(to)) {
      r.f = (to == KTIR_F16) ? __half2float(__ll2half_rn(v.i)) : (float)v.i;
    } else {
      r.i = wrap_to(v.i, to);
    }
  }
  return r;
}

__device__ __forceinline__ float binf(int op, float x, float y) {
  switch (op) {
    case OP_FADD: return x + y;
    case OP_FSUB: return x - y;
    case OP_FMUL: return x * y;
    case OP_FDIV: return x / y;
    case OP_FMOD: return py_fmod(x, y);
    case OP_FMAXNUM: return fmaxf(x, y);
    case OP_FMINNUM: return fminf(x, y);
    case OP_FMAXIMUM: return (isnan(x) || isnan(y)) ? __int_as_float(0x7fc00000) : fmaxf(x, y);
    case OP_FMINIMUM: return (isnan(x) || isnan(y)) ? __int_as_float(0x7fc00000) : fminf(x, y);
    case OP_FPOW: return powf(x, y);
  }
  return 0.f;
}

__device__ __forceinline__ float unf(int op, float x) {
  switch (op) {
    case OP_FNEG: return -x;
    case OP_FABS: return fabsf(x);
    case OP_FEXP: return expf(x);
    case OP_FSQRT: return sqrtf(x);
    case OP_FRSQRT: return 1.0f / sqrtf(x);
    case OP_FLOG: return logf(x);
    case OP_FLOG2: return log2f(x);
    case OP_FLOG1P: return log1pf(x);
    case OP_FTANH: return tanhf(x);
    case OP_FSIN: return sinf(x);
    case OP_FCOS: return cosf(x);
    case OP_FCEIL: return ceilf(x);
    case OP_FFLOOR: return floorf(x);
    case OP_FERF: return as_erf(x);
  }
  return 0.f;
}

__device__ __forceinline__ long long bini(int op, long long x, long long y) {
  switch (op) {
    case OP_IADD: return x + y;
    case OP_ISUB: return x - y;
    case OP_IMUL: return x * y;
    case OP_IFLOORDIV: return py_floordiv(x, y);
    case OP_IMOD: return py_mod(x, y);
    case OP_ITRUNCDIV: return y == 0 ? 0 : x / y;
    case OP_ITRUNCREM: return y == 0 ? 0 : x % y;
    case OP_ICEILDIV: return y == 0 ? 0 : -py_floordiv(-x, y);
    case OP_IAND: return x & y;
    case OP_IOR: return x | y;
    case OP_IXOR: return x ^ y;
    case OP_ISHL: return x << (y & 63);
    case OP_ISHR: return x >> (y & 63);
    case OP_ISHRU: return (long long)((unsigned long long)x >> (y & 63));
    case OP_IMAX: return x > y ? x : y;
    case OP_IMIN: return x < y ? x : y;
  }
  return 0;
}

// Execute one arithmetic instruction (not LD/ST/IOTA, which need the iteration
// context).  `r` is the register file.
__device__ __forceinline__ void exec_arith(const KtirInstr& in, Reg* r) {
  const int op = in.op;
  const int dt = in.dt;
  Reg out;
  out.i = 0;
  if (op == OP_IMM) {
    if (is_float(dt)) {
      double d = __longlong_as_double(in.imm);
      out.f = (dt == KTIR_F16) ? __half2float(__double2half(d)) : (float)d;
    } else {
      out.i = wrap_to(in.imm, dt);
    }
  } else if (op == OP_CAST) {
    out = convert(r[in.a], in.aux, dt);
  } else if (op == OP_BITCAST) {
    out = r[in.a];
  } else if (op >= OP_FADD && op <= OP_FPOW) {
    out.f = round_to(binf(op, r[in.a].f, r[in.b].f), dt);
  } else if (op >= OP_FNEG && op <= OP_FERF) {
    out.f = round_to(unf(op, r[in.a].f), dt);
  } else if (op == OP_FFMA) {
    out.f = round_to(r[in.a].f * r[in.b].f + r[in.c].f, dt);
  } else if (op == OP_FCMP) {
    out.i = fcmp(in.aux, r[in.a].f, r[in.b].f);
  } else if (op == OP_SELECT) {
    out = r[in.a].i ? r[in.b] : r[in.c];
  } else if (op >= OP_IADD && op <= OP_IMIN) {
    out.i = wrap_to(bini(op, r[in.a].i, r[in.b].i), dt);
  } else if (op == OP_INEG) {
    out.i = wrap_to(-r[in.a].i, dt);
  } else if (op == OP_IABS) {
    long long v = r[in.a].i;
    out.i = wrap_to(v < 0 ? -v : v, dt);
  } else if (op == OP_ICMP) {
    out.i = icmp(in.aux, r[in.a].i, r[in.b].i);
  }
  r[in.dst] = out;
}

}  // namespace ktir
