// Lean cast of fp32 values onto a narrow float grid, used by the streaming quantize and cast kernels
// when the format and rounding allow it; results equal cast_float() bit for bit.
//
// For a finite magnitude a whose exponent is e, the grid quantum is 2**qe with
// qe = max(e, emin) - mbits. With M = 2**(qe + 23) and mbits <= 22, a < M, so a + M lies in
// [M, 2M) where fp32's spacing is exactly 2**qe: one fp32 addition in the wanted direction rounds a
// to the grid (nearest-even: the parity of (M + k 2**qe) / 2**qe is the parity of k) and the
// subtraction of M is exact (both operands lie within a factor of two). The sign is handled on the
// side: RUP rounds a positive magnitude up and a negative one toward zero, RDN the reverse.
//
// Element codes come from one exact multiply: r * 2**(-126 - emin) maps the format's normals onto
// fp32 normals with exponent field (e - emin + 1), i.e. the format's biased exponent, and its
// subnormals onto fp32 subnormals whose fraction is the format's fraction, so the code magnitude is
// that product's bit pattern shifted right by 23 - mbits.
#pragma once

#include <cstring>

#include "tc_common.cuh"

namespace tc {

struct Lean {
  int ok;           // format and rounding are handled by the lean path
  int mshift;       // 23 - mbits
  int qlo, qhi;     // bounds of M's exponent field: emin + 127 + mshift, emax + 128 + mshift
  float min_norm;   // 2**emin
  float top_pow;    // 2**(emax + 1)
  float m_mul;      // 2**(23 - mbits)
  float maxv;       // max_normal
  float code_mul;   // 2**(-126 - emin)
  int sign_pos;     // ebits + mbits: sign bit of the element code
  int sat_only;     // every overflow becomes max_normal (saturate, or a format without Inf/NaN)
  uint32_t ovf_pos, ovf_neg;  // overflow magnitude bits otherwise (by sign of the value)
};

// Host: constants of the lean cast, ok = 0 when the generic cast must be used.
inline Lean make_lean(const tc_format &f, const Fmt &d, int rounding, int saturate) {
  Lean l;
  memset(&l, 0, sizeof(l));
  if (f.kind != 0 || !f.is_signed || !f.subnormals) return l;
  if (f.special == 2) return l;                                      // fnuz: no negative zero
  if (f.mbits > 22 || d.emin < -126 || d.emax + 128 + 23 - f.mbits > 254) return l;
  if (rounding != TC_RNE && rounding != TC_RTZ && rounding != TC_RUP && rounding != TC_RDN) return l;
  l.mshift = 23 - f.mbits;
  l.qlo = d.emin + 127 + l.mshift;
  l.qhi = d.emax + 128 + l.mshift;
  auto pow2f = [](int e) { uint32_t b = (uint32_t)(e + 127) << 23; float v; memcpy(&v, &b, 4); return v; };
  l.min_norm = pow2f(d.emin);
  l.top_pow = pow2f(d.emax + 1);
  l.m_mul = pow2f(l.mshift);
  uint32_t mb = d.max_bits;
  memcpy(&l.maxv, &mb, 4);
  uint32_t cm = (uint32_t)(-126 - d.emin + 127) << 23;
  memcpy(&l.code_mul, &cm, 4);
  l.sign_pos = f.ebits + f.mbits;
  l.sat_only = saturate || f.special == 3;
  auto ovf = [&](bool neg) -> uint32_t {
    if (l.sat_only) return d.max_bits;
    if (f.special == 1) return kQNaN;
    bool away = rounding == TC_RTZ ? false : rounding == TC_RUP ? !neg : rounding == TC_RDN ? neg : true;
    return away ? kInf : d.max_bits;
  };
  l.ovf_pos = ovf(false);
  l.ovf_neg = ovf(true);
  l.ok = 1;
  return l;
}

// Grid magnitude of x (finite or infinite, not NaN) rounded in direction RND. CLAMP bounds M for
// magnitudes above the format's range (infinite or huge x), which only ever overflow.
template <int RND, bool CLAMP>
__device__ __forceinline__ float lean_mag(float x, const Lean &l) {
  const uint32_t u = f2u(x);
  const uint32_t a = u & 0x7FFFFFFFu;
  int mf = max((int)(a >> 23) + l.mshift, l.qlo);
  if (CLAMP) mf = min(mf, l.qhi);
  const float M = u2f((uint32_t)mf << 23);
  const float af = u2f(a);
  float s;
  if (RND == TC_RNE) {
    s = __fadd_rn(af, M);
  } else if (RND == TC_RTZ) {
    s = __fadd_rz(af, M);
  } else {
    const bool neg = (u >> 31) != 0;
    const bool up = RND == TC_RUP ? !neg : neg;
    s = up ? __fadd_ru(af, M) : __fadd_rz(af, M);
  }
  return __fsub_rn(s, M);
}

// The same rounding with M built by float min/max and an exponent mask (2**max(e, emin) scaled by
// 2**(23 - mbits)). Without CLAMP the caller guarantees |x| < 2**(emax + 1) or that x is only ever
// rounded into overflow with CLAMP's bound. RNDC 0: nearest-even; 1: RTZ / RUP / RDN chosen at run
// time by `rnd`.
template <int RNDC, bool CLAMP>
__device__ __forceinline__ float lean_mag2(float x, const Lean &l, int rnd) {
  const float ax = fabsf(x);
  float e = fmaxf(ax, l.min_norm);
  if (CLAMP) e = fminf(e, l.top_pow);
  const float M = __fmul_rn(u2f(f2u(e) & 0x7F800000u), l.m_mul);
  float s;
  if (RNDC == 0) {
    s = __fadd_rn(ax, M);
  } else {
    const bool neg = (f2u(x) >> 31) != 0;
    const bool up = rnd == TC_RUP ? !neg : (rnd == TC_RDN && neg);
    s = rnd == TC_RNE ? __fadd_rn(ax, M) : up ? __fadd_ru(ax, M) : __fadd_rz(ax, M);
  }
  return __fsub_rn(s, M);
}

// Overflow rule applied to a rounded magnitude r of a value with sign bit `sign`.
__device__ __forceinline__ float lean_overflow(float r, uint32_t sign, const Lean &l) {
  if (l.sat_only) return fminf(r, l.maxv);
  return r > l.maxv ? u2f(sign ? l.ovf_neg : l.ovf_pos) : r;
}

// Code magnitude of a finite grid magnitude r.
__device__ __forceinline__ uint32_t lean_code(float r, const Lean &l) {
  return f2u(__fmul_rn(r, l.code_mul)) >> l.mshift;
}

}  // namespace tc
