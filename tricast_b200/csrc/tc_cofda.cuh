// CoFDA building blocks shared by the tiled kernel (tc_gemm_cofda.cu) and the small-M kernel
// (tc_gemv_cofda.cu): element decoding, the running value's FDA term, truncation of a scaled product
// and the fp32 / fp64 accumulator arithmetic.
#pragma once

#include "tc_gemm.cuh"

namespace tc {
namespace cofda {

constexpr int kZeroExp = -8192;  // exponent label of a zero element (int16)

// A grid element's decoded exponent label (mma.py:75-91): false for NaN / Inf, values off the
// format's grid and values beyond its largest exponent.
__device__ __forceinline__ bool decode_elem(float v, const Fmt &f, int &e) {
  uint32_t u = f2u(v);
  uint32_t a = u & 0x7FFFFFFFu;
  if (a >= kInf) return false;
  if (a == 0) {
    e = kZeroExp;
    return true;
  }
  Term t = decode_term(v, f);
  // On-grid check: the decoded significand must reproduce |v| exactly (mbits <= 3 here).
  if (t.sig == 0 || t.sig >= (1ull << (f.mbits + 1))) return false;
  float back = ldexpf((float)t.sig, t.exp - f.mbits);
  if (back != fabsf(v)) return false;
  if (t.exp > f.emax) return false;  // beyond the format's range: products could leave fp32's
  e = t.exp;
  return true;
}

__device__ __forceinline__ int running_exp(float c) {
  uint32_t a = f2u(c) & 0x7FFFFFFFu;
  if (a == 0 || a >= kInf) return kZeroExp;
  uint32_t field = a >> 23;
  return field ? (int)field - 127 : ilog2_u32(a) - 149;
}

// The running value as an FDA term at radix F <= 23, aligned to emax with truncation: its 24-bit
// significand shifted right by (23 - F) + (emax - ec) (mma.py:85-91 then the alignment shift).
// Exact integer below 2**(F+1), returned as fp32.
__device__ __forceinline__ float running_term(float c, int F, int emax) {
  const uint32_t a = f2u(c) & 0x7FFFFFFFu;
  if (a == 0 || a >= kInf) return 0.0f;
  const uint32_t field = a >> 23;
  const uint32_t sig = field ? ((a & 0x7FFFFFu) | 0x800000u) : a;
  const int lead = ilog2_u32(sig);
  const int ec = (field ? (int)field - 127 : -126) + lead - 23;
  const uint32_t norm = sig << (23 - lead);
  const int sh = (23 - F) + (emax - ec);
  const uint32_t v = sh >= 32 ? 0u : (norm >> sh);
  return (f2u(c) >> 31) ? -(float)v : (float)v;
}

// 2**e as fp32 for e in [-126, 127] (callers clamp).
__device__ __forceinline__ float pow2f(int e) { return u2f((uint32_t)(e + 127) << 23); }

// floor(|x| * s) with x's sign, exact for |x * s| < 2**23 (x * s exact or not).
__device__ __forceinline__ float trunc_scaled(float x, float s) {
  const float m = u2f((f2u(x) & 0x80000000u) | 0x4B000000u);
  return __fadd_rn(__fmaf_rz(x, s, m), -m);
}

// The accumulator arithmetic of one precision: powers of two, truncation of a scaled product and
// the running value's term. fp32 serves F + 2 + log2(CS + 1) <= 24, fp64 up to 53.
template <class T>
struct Acc;

template <>
struct Acc<float> {
  static __device__ __forceinline__ float pow2(int e) { return pow2f(e > 127 ? 127 : (e < -126 ? -126 : e)); }
  static __device__ __forceinline__ float trunc(float x, float s) { return trunc_scaled(x, s); }
  static __device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
  static __device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
  static __device__ __forceinline__ float fma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
  // copysign(2**23, b), the rounding magic of every product |a| * b; floor(|p * s|) with p's sign for
  // such a magic m of p's sign (exact for |p * s| < 2**23, as trunc).
  static __device__ __forceinline__ float magic(float b) { return u2f((f2u(b) & 0x80000000u) | 0x4B000000u); }
  static __device__ __forceinline__ float trunc_m(float p, float s, float m) { return __fadd_rn(__fmaf_rz(p, s, m), -m); }
  // floor(|c| * 2**(F - emax)) with c's sign (c's significand cut to F fraction bits, then aligned):
  // |c| < 2**(emax + 1), so the product is below 2**(F + 1) <= 2**22 and the fma.rz truncation is exact.
  // When every product of the chunk is zero emax is c's own exponent, which can sit below
  // F - 127 (s clamped): that case takes the integer shift.
  static __device__ __forceinline__ float running(float c, int F, int emax, float s) {
    const uint32_t a = f2u(c) & 0x7FFFFFFFu;
    if (a == 0 || a >= kInf) return 0.0f;
    return F - emax <= 127 ? trunc_scaled(c, s) : running_term(c, F, emax);
  }
  // fixed_to_fp32(tot, emax, F, rne, true) for the exact integer tot (|tot| < 2**24): the fp32 pattern
  // of |tot| rounded to min(F, 23) fraction bits (toward zero, or to nearest even by the carry-add
  // on the pattern), its exponent moved by emax - F. Results outside the normal range take the
  // general routine (subnormal truncation, overflow to Inf).
  static __device__ __forceinline__ float finish(float tot, int emax, int F, bool rne) {
    const uint32_t a = f2u(tot) & 0x7FFFFFFFu;
    if (a == 0) return 0.0f;
    const int drop = F < 23 ? 23 - F : 0;
    uint32_t r = a;
    if (rne && drop > 0) r += ((1u << drop) >> 1) - 1u + ((a >> drop) & 1u);
    r &= ~((1u << drop) - 1u);
    const int field = (int)(r >> 23) + emax - F;
    if (field < 1 || field > 254) return fixed_to_fp32((int64_t)tot, emax, F, rne, true);
    return u2f(((uint32_t)field << 23) | (r & 0x7FFFFFu) | (f2u(tot) & 0x80000000u));
  }
  // Branch-free forms for the per-output steps of a chunk: the common case is computed with selects
  // and `rare` reports an output that needs the general routine above (running: F - emax > 127;
  // finish: a result outside the normal range), which the caller redoes for the few that set it.
  static __device__ __forceinline__ float running_fast(float c, float s, int F, int emax, bool &rare) {
    const uint32_t a = f2u(c) & 0x7FFFFFFFu;
    const bool live = (a != 0) & (a < kInf);
    rare = live & (F - emax > 127);
    const float t = trunc_scaled(c, s);
    return live ? t : 0.0f;
  }
  static __device__ __forceinline__ float finish_fast(float tot, int emax, int F, bool rne, bool &rare) {
    const uint32_t a = f2u(tot) & 0x7FFFFFFFu;
    const int drop = F < 23 ? 23 - F : 0;
    const uint32_t up = (rne && drop > 0) ? ((1u << drop) >> 1) - 1u + ((a >> drop) & 1u) : 0u;
    const uint32_t r = (a + up) & ~((1u << drop) - 1u);
    const int field = (int)(r >> 23) + emax - F;
    rare = (a != 0) & ((field < 1) | (field > 254));
    const float v = u2f(((uint32_t)field << 23) | (r & 0x7FFFFFu) | (f2u(tot) & 0x80000000u));
    return a == 0 ? 0.0f : v;
  }
};

template <>
struct Acc<double> {
  static __device__ __forceinline__ double pow2(int e) {
    e = e > 1023 ? 1023 : (e < -1022 ? -1022 : e);
    return __hiloint2double((e + 1023) << 20, 0);
  }
  // floor(|x| * s) with x's sign, exact for |x * s| < 2**52: fma.rz into the binade of 2**52.
  static __device__ __forceinline__ double trunc(double x, double s) {
    const double m = __hiloint2double((int)(((uint32_t)__double2hiint(x) & 0x80000000u) | 0x43300000u), 0);
    return __dadd_rn(__fma_rz(x, s, m), -m);
  }
  static __device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
  static __device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
  static __device__ __forceinline__ double fma(double a, double b, double c) { return __fma_rn(a, b, c); }
  // As Acc<float>: copysign(2**52, b), and floor(|p * s|) with p's sign for |p * s| < 2**52.
  static __device__ __forceinline__ double magic(double b) {
    return __hiloint2double((int)(((uint32_t)__double2hiint(b) & 0x80000000u) | 0x43300000u), 0);
  }
  static __device__ __forceinline__ double trunc_m(double p, double s, double m) { return __dadd_rn(__fma_rz(p, s, m), -m); }
  // floor(|c| * 2**(F - emax)) with c's sign; |c| < 2**(emax + 1), so the product is below 2**(F + 1).
  static __device__ __forceinline__ double running(float c, int, int, double s) {
    const uint32_t a = f2u(c) & 0x7FFFFFFFu;
    return (a == 0 || a >= kInf) ? 0.0 : trunc((double)c, s);
  }
  // As Acc<float>::finish for |tot| < 2**53, on the fp64 pattern.
  static __device__ __forceinline__ float finish(double tot, int emax, int F, bool rne) {
    const uint64_t bits = (uint64_t)__double_as_longlong(tot);
    const uint64_t a = bits & 0x7FFFFFFFFFFFFFFFull;
    if (a == 0) return 0.0f;
    const int drop = 52 - (F < 23 ? F : 23);
    uint64_t r = a;
    if (rne) r += ((1ull << drop) >> 1) - 1ull + ((a >> drop) & 1ull);
    r &= ~((1ull << drop) - 1ull);
    const int field = (int)(r >> 52) - 1023 + 127 + emax - F;
    if (field < 1 || field > 254) return fixed_to_fp32((int64_t)tot, emax, F, rne, true);
    return u2f(((uint32_t)field << 23) | (uint32_t)((r >> 29) & 0x7FFFFFu) | (uint32_t)(bits >> 32 & 0x80000000u));
  }
  // Branch-free forms, as for fp32 (the fp64 running term has no rare case).
  static __device__ __forceinline__ double running_fast(float c, double s, int F, int emax, bool &rare) {
    rare = false;
    return running(c, F, emax, s);
  }
  static __device__ __forceinline__ float finish_fast(double tot, int emax, int F, bool rne, bool &rare) {
    const uint64_t bits = (uint64_t)__double_as_longlong(tot);
    const uint64_t a = bits & 0x7FFFFFFFFFFFFFFFull;
    const int drop = 52 - (F < 23 ? F : 23);
    const uint64_t up = rne ? ((1ull << drop) >> 1) - 1ull + ((a >> drop) & 1ull) : 0ull;
    const uint64_t r = (a + up) & ~((1ull << drop) - 1ull);
    const int field = (int)(r >> 52) - 1023 + 127 + emax - F;
    rare = (a != 0) & ((field < 1) | (field > 254));
    const float v = u2f(((uint32_t)field << 23) | (uint32_t)((r >> 29) & 0x7FFFFFu) | (uint32_t)(bits >> 32 & 0x80000000u));
    return a == 0 ? 0.0f : v;
  }
};

// Decoupled CoFDA (mma.py:296-301): the chunk's partial p, normalised at radix F from a zero running
// value, joins the running value c in a two-term FDA at radix F2: emax is the larger exponent label,
// each term is floor(|v| * 2**(F2 - emax)) (the value's significand cut to F2 fraction bits, then
// aligned; exact in fp64 for F2 <= 50, and so is their sum), normalised at F2. NaN or opposite
// infinities give NaN, an infinity wins otherwise, and two zero terms keep c.
__device__ __forceinline__ float merge_decoupled(float pv, float c, int F2, bool rne) {
  const uint32_t ap = f2u(pv) & 0x7FFFFFFFu, ac = f2u(c) & 0x7FFFFFFFu;
  if (ap >= kInf || ac >= kInf) {
    if (ap > kInf || ac > kInf) return u2f(kQNaN);
    if (ap == kInf && ac == kInf) return f2u(pv) == f2u(c) ? pv : u2f(kQNaN);
    return ap == kInf ? pv : c;
  }
  if (ap == 0 && ac == 0) return c;
  const int emax = max(running_exp(pv), running_exp(c));
  const double s = Acc<double>::pow2(F2 - emax);
  const double t = Acc<double>::add(Acc<double>::running(pv, 0, 0, s), Acc<double>::running(c, 0, 0, s));
  return Acc<double>::finish(t, emax, F2, rne);
}

template <class T>
__device__ __forceinline__ void load4(const T *src, T (&o)[4]) {
  if (sizeof(T) == 4) {
    const float4 v = *reinterpret_cast<const float4 *>(src);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  } else {
    const double2 v0 = *reinterpret_cast<const double2 *>(src), v1 = *reinterpret_cast<const double2 *>(src + 2);
    o[0] = v0.x; o[1] = v0.y; o[2] = v1.x; o[3] = v1.y;
  }
}

}  // namespace cofda
}  // namespace tc
