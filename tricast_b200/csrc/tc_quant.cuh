// Quantize internals shared by the quantize translation units: spec parameters, element and scale
// codes, scale selection and the per-element rounding (TriCast src/tricast/reference/quantize.py).
#pragma once

#include <cmath>
#include <cstring>
#include <string>

#include "tc_common.cuh"
#include "tc_lean.cuh"

namespace tc {

enum { GRAN_TENSOR = 0, GRAN_ROW = 1, GRAN_GROUP = 2, GRAN_BLOCK = 3 };
enum { M_ABSMAX = 0, M_POW2_FLOOR = 1, M_POW2_CEIL = 2, M_MSE = 3, M_PERCENTILE = 4 };
enum { ZP_NONE = 0, ZP_INT = 1, ZP_FLOAT = 2 };

struct QParams {
  Fmt ef, sf;
  int64_t rows, K;
  int64_t dr, dc, nr, nc;  // nominal domain rect and domain grid
  int has_scale, method, srnd, two_level, zp, rnd, sr_bits, saturate;
  float max_elem;          // element max_normal (exact in fp32)
  double max_elem_d;
  int emax_elem;
  uint32_t min_scale_bits;  // scale format min_subnormal (pow2: min_normal) as fp32
  double qmin_d, qmax_d;
  float qrange;             // qmax - qmin
  int x_dtype, v_dtype;
  int code_bits;            // 0, 4 or 8
  int scode;                // 0 none, 1 byte code of the scale format
  double prod_max_d;        // element max * scale max (two-level global scale)
  int pow2_div;             // every divisor is a power of two (pow2 methods, one level)
};

// ------------------------------------------------------------------ element codes
// Bit encoding of a grid value in a <= 8-bit format (sign | exponent field | fraction field, or
// two's complement k for integers). NaN uses the format's NaN encoding where it has one.
__device__ __forceinline__ uint32_t element_code(float v, const Fmt &f, int total_bits) {
  uint32_t u = f2u(v);
  uint32_t sign = u >> 31;
  uint32_t a = u & 0x7FFFFFFFu;
  if (f.kind == 1) {
    if (a > kInf) return 0u;
    double k = ldexp((double)fabsf(v), f.frac_bits);
    int64_t ki = (int64_t)k;
    if (sign && a) ki = -ki;
    return (uint32_t)ki & ((1u << total_bits) - 1u);
  }
  int mb = f.mbits;
  uint32_t mmask = (1u << mb) - 1u;
  uint32_t top_field = (1u << f.ebits) - 1u;
  uint32_t code;
  if (a > kInf) {
    if (f.special == 1) code = (top_field << mb) | mmask;                // fn: all ones
    else if (f.special == 2) return 1u << (total_bits - 1);              // fnuz: the "-0" pattern
    else if (f.special == 0) code = (top_field << mb) | (mb ? (1u << (mb - 1)) : 0u);
    else code = 0u;
    sign = 0;
  } else if (a == kInf) {
    code = top_field << mb;
  } else if (a == 0) {
    code = 0u;
  } else {
    int field = (int)(a >> 23);
    int e32 = field ? field - 127 : -126;
    uint32_t sig = field ? ((a & 0x7FFFFFu) | 0x800000u) : a;
    if (e32 >= f.emin) {
      code = ((uint32_t)(e32 + f.bias) << mb) | ((sig >> (23 - mb)) & mmask);
    } else {
      int s = 23 - mb + (f.emin - e32);   // fraction of a subnormal in units of 2**(emin - mbits)
      code = s >= 32 ? 0u : (sig >> s);
    }
  }
  if (f.is_signed) code |= sign << (f.ebits + mb);
  return code & ((1u << total_bits) - 1u);
}

__device__ __forceinline__ uint32_t scale_code(float s, const Fmt &f) {
  if (f.kind == 2) {
    uint32_t a = f2u(s);
    if ((a & 0x7FFFFFFFu) > kInf) return 0xFFu;
    int e;
    frexpf(s, &e);
    return (uint32_t)(e - 1 + f.bias) & 0xFFu;
  }
  return element_code(s, f, f.ebits + f.mbits + (f.is_signed ? 1 : 0));
}

// ------------------------------------------------------------------ scale selection
__device__ __forceinline__ float amax_scale(float amax, float d2, bool has_d2, const QParams &p, uint32_t noise) {
  float t = __fdiv_rn(amax, p.max_elem);
  if (has_d2) t = __fdiv_rn(t, d2);
  float s = cast_to(t, p.sf, p.srnd, true, noise, 32);
  if (s == 0.0f) s = u2f(p.min_scale_bits);
  if (amax == 0.0f) s = 1.0f;
  return s;
}

__device__ __forceinline__ float pow2_scale(float amax, const QParams &p) {
  double a = amax == 0.0f ? ldexp(1.0, -126) : (double)amax;
  int ex;
  frexp(a, &ex);
  int e = ex - 1 - p.emax_elem;
  if (p.method == M_POW2_CEIL && ldexp(p.max_elem_d, e) < a) e += 1;
  bool overflow = e > p.sf.emax || !isfinite(a);
  e = e < p.sf.emin ? p.sf.emin : (e > p.sf.emax ? p.sf.emax : e);
  float s = __double2float_rn(ldexp(1.0, e));
  return overflow ? u2f(kQNaN) : s;
}

// One exact binary32 rounding of amax / P, P = element max * scale max, as TriCast's
// _global_scale (src/tricast/reference/quantize.py:195-219): the fp64 quotient gives a candidate
// and the midpoints to its neighbours are tested exactly with fma (the sign of m*P - amax).
__device__ inline float global_scale(float amax, double P) {
  if (!isfinite(amax)) return amax;
  if (amax == 0.0f) return 1.0f;
  double A = (double)amax;
  float r = __double2float_rn(A / P);
  for (int it = 0; it < 2; ++it) {
    float up = nextafterf(r, INFINITY);
    double mid = 0.5 * ((double)r + (double)up);
    double s = fma(mid, P, -A);
    if (s < 0 || (s == 0 && (f2u(r) & 1u))) r = up;
    float dn = nextafterf(r, -INFINITY);
    mid = 0.5 * ((double)r + (double)dn);
    s = fma(mid, P, -A);
    if (s > 0 || (s == 0 && (f2u(r) & 1u))) r = dn;
  }
  return r == 0.0f ? 1.0f : r;
}

// Affine scale and zero point from the domain range (src/tricast/reference/quantize.py:176-192).
__device__ __forceinline__ void zp_scale(float lo, float hi, const QParams &p, uint32_t noise, float &s, float &z) {
  if (p.zp == ZP_INT) {
    if (lo > 0.0f) lo = 0.0f;  // clamp(max=0): keeps -0 and NaN
    if (hi < 0.0f) hi = 0.0f;
  }
  float raw = __fdiv_rn(__fsub_rn(hi, lo), p.qrange);
  s = cast_to(raw, p.sf, p.srnd, true, noise, 32);
  if (s == 0.0f) s = u2f(p.min_scale_bits);
  if (hi == lo) s = 1.0f;
  z = lo;
  if (p.zp == ZP_INT) {
    float t = rintf(__fsub_rn((float)p.qmin_d, __fdiv_rn(lo, s)));
    if (t < (float)p.qmin_d) t = (float)p.qmin_d;
    if (t > (float)p.qmax_d) t = (float)p.qmax_d;
    z = t;  // NaN stays NaN (both comparisons false)
  }
}

// Order-preserving keys: -0 sorts below +0.
__device__ __forceinline__ uint32_t fkey(float v) {
  uint32_t u = f2u(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unkey(uint32_t k) { return u2f((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k); }

// ------------------------------------------------------------------ element rounding
// Integer rounding for zero-point specs on the unbounded integer grid, then + z and clamp
// (src/tricast/reference/quantize.py:325-332).
__device__ __forceinline__ float zp_round(float xq, float z, const QParams &p, uint32_t noise) {
  if (p.rnd != TC_SR && p.qmax_d < 16777216.0 && p.qmin_d > -16777216.0) {
    // Deterministic modes in fp32 (integer grids inside +-2**24): rint / trunc / ceil / floor / round
    // give the integer the reference forms on |xq| (its direction rules per sign are exactly these),
    // NaN and Inf pass through; an integer zero point then adds exactly (both integers below 2**24;
    // any larger sum lies beyond the clamp and clamps to the same bound), and the compare-and-select
    // clamp keeps NaN as the reference's does.
    const float k = p.rnd == TC_RNE ? rintf(xq)
                    : p.rnd == TC_RTZ ? truncf(xq)
                    : p.rnd == TC_RUP ? ceilf(xq)
                    : p.rnd == TC_RDN ? floorf(xq)
                                      : roundf(xq);
    float r = p.zp == ZP_INT ? __fadd_rn(k, z) : k;
    const float lo = (float)p.qmin_d, hi = (float)p.qmax_d;
    if (r < lo) r = lo;
    if (r > hi) r = hi;
    return r;
  }
  uint32_t u = f2u(xq);
  uint32_t a = u & 0x7FFFFFFFu;
  double r;
  if (a > kInf) {
    r = (double)xq;
  } else if (a == kInf) {
    r = (double)xq;
  } else {
    bool neg = (u >> 31) && a;
    uint32_t field = a >> 23;
    uint32_t sig = field ? ((a & 0x7FFFFFu) | 0x800000u) : a;
    int e32 = field ? (int)field - 127 : -126;
    int shift = 23 - e32;  // quantum 2**0
    double k;
    if (shift <= 0) {
      k = (double)fabsf(xq);
    } else {
      uint32_t kept = shift >= 32 ? 0u : (sig >> shift);
      uint32_t rem = shift >= 32 ? sig : (sig & ((1u << shift) - 1u));
      kept += round_inc(kept, rem, shift, neg, p.rnd, noise, p.sr_bits) ? 1u : 0u;
      k = (double)kept;
    }
    r = (u >> 31) ? -k : k;
  }
  if (p.zp == ZP_INT) r = r + (double)z;
  if (r < p.qmin_d) r = p.qmin_d;
  if (r > p.qmax_d) r = p.qmax_d;
  return (float)r;
}

struct ElemOut {
  float value;
  float dequant;
};

// The divisor of a domain: s (one level) or RN(s * d2) (two-level), and, when it is a power of two,
// its exact reciprocal: RN(x / 2**e) == RN(x * 2**-e) for every fp32 x, 2**-e being representable.
struct Divisor {
  float eff, inv;
  bool by_inv;
};

__device__ __forceinline__ Divisor make_divisor(float s, float d2, bool has_d2, const QParams &p) {
  Divisor d;
  d.eff = has_d2 ? __fmul_rn(s, d2) : s;
  d.by_inv = p.pow2_div != 0;
  d.inv = d.by_inv ? __frcp_rn(d.eff) : 0.0f;
  return d;
}

__device__ __forceinline__ ElemOut quant_elem_d(float x, float s, float z, const Divisor &dv, float d2, bool has_d2,
                                                const QParams &p, uint32_t noise) {
  float xq = x;
  if (p.zp == ZP_FLOAT) xq = __fsub_rn(xq, z);
  if (p.has_scale) xq = dv.by_inv ? __fmul_rn(xq, dv.inv) : __fdiv_rn(xq, dv.eff);
  ElemOut o;
  o.value = p.zp ? zp_round(xq, z, p, noise) : cast_to(xq, p.ef, p.rnd, p.saturate, noise, p.sr_bits);
  float d = o.value;
  if (p.zp == ZP_INT) d = __fsub_rn(d, z);
  if (p.has_scale) d = __fmul_rn(d, s);
  if (p.zp == ZP_FLOAT) d = __fadd_rn(d, z);
  if (has_d2) d = __fmul_rn(d, d2);
  o.dequant = d;
  return o;
}

// ------------------------------------------------------------------ MSE scale search
// Candidate ratios of an MSE search (src/tricast/reference/quantize.py:286-301): the spec's search
// list or linspace(1.0, 0.5, mse_grid), both as fp32, computed by the caller exactly as TriCast does.
constexpr int kMaxRatios = 256;
struct Ratios {
  int n;
  float r[kMaxRatios];
};

// Squared error of one element quantized with candidate scale s (the divisor dv of s): the
// reference's (x - restored)**2 with restored = (q * s) [* d2], differences and squares in fp64.
__device__ __forceinline__ double cand_sq_error(float x, float s, const Divisor &dv, float d2, bool has_d2,
                                                const QParams &p, uint32_t noise);

__device__ __forceinline__ ElemOut quant_elem(float x, float s, float z, float d2, bool has_d2, const QParams &p,
                                              uint32_t noise) {
  return quant_elem_d(x, s, z, make_divisor(s, d2, has_d2, p), d2, has_d2, p, noise);
}

__device__ __forceinline__ double cand_sq_error(float x, float s, const Divisor &dv, float d2, bool has_d2,
                                                const QParams &p, uint32_t noise) {
  const ElemOut o = quant_elem_d(x, s, 0.0f, dv, d2, has_d2, p, noise);
  const double d = __dsub_rn((double)x, (double)o.dequant);
  return __dmul_rn(d, d);
}

}  // namespace tc
