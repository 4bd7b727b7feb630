// Exact integer datapath primitives of TriCast's emulated MMA (src/tricast/reference/mma.py):
// terms (sign, exponent, significand at an explicit radix, zero/nan/inf flags), decoding grid
// values, product and scale combination, the truncating alignment sum and the fixed-point to fp32
// normalisation. Used by the generic per-output kernel and by the fast kernels' epilogues.
#pragma once

#include "tc_common.cuh"

namespace tc {

struct Term {
  uint64_t sig;
  int exp;
  bool neg, zero, nan, inf;
};

constexpr int kNoExp = -4096;  // exponent of "no active term" (reference: -4096)

__device__ __forceinline__ uint64_t shift_u64(uint64_t x, int amount) {
  if (amount >= 64 || amount <= -64) return 0ull;
  return amount >= 0 ? (x << amount) : (x >> (-amount));
}

// Shift right with round-half-even on the discarded bits (mma.py:46-52).
__device__ __forceinline__ uint64_t rounded_shift_u64(uint64_t x, int amount) {
  uint64_t kept = shift_u64(x, amount);
  if (amount < 0 && amount > -64) {
    int discard = -amount;
    uint64_t rem = x - (kept << discard);
    uint64_t half = 1ull << (discard - 1);
    if (rem > half || (rem == half && (kept & 1ull))) kept += 1;
  }
  return kept;
}

// value = sig * 2**(e0) with sig a 24-bit fp32 significand: |v| split exactly.
__device__ __forceinline__ void split_f32(uint32_t a, uint32_t &m, int &e0) {
  uint32_t field = a >> 23;
  m = field ? ((a & 0x7FFFFFu) | 0x800000u) : (a & 0x7FFFFFu);
  e0 = field ? (int)field - 150 : -149;
}

__device__ __forceinline__ int floor_log2_f32(uint32_t a) {  // a > 0 finite
  uint32_t field = a >> 23;
  return field ? (int)field - 127 : ilog2_u32(a) - 149;
}

// Format-native decode (src/tricast/reference/cast.py:186-222; mma.py:75-82): exponent =
// max(floor log2 |v|, emin) with significand at radix mbits for floats; exponent 0 and |k| at
// radix frac_bits for ints; log2 v with significand 1 for powers of two. Specials get sig 0.
__device__ __forceinline__ Term decode_term(float v, const Fmt &f) {
  Term t;
  uint32_t u = f2u(v);
  uint32_t a = u & 0x7FFFFFFFu;
  t.neg = (u >> 31) != 0;
  t.zero = a == 0;
  t.nan = a > kInf;
  t.inf = a == kInf;
  t.sig = 0;
  t.exp = 0;
  if (t.zero || t.nan || t.inf) return t;
  uint32_t m;
  int e0;
  split_f32(a, m, e0);
  if (f.kind == 0) {
    int fl = floor_log2_f32(a);
    t.exp = fl > f.emin ? fl : f.emin;
    t.sig = shift_u64(m, e0 + f.mbits - t.exp);
  } else if (f.kind == 1) {
    t.sig = shift_u64(m, e0 + f.frac_bits);
  } else {
    t.exp = floor_log2_f32(a);
    t.sig = 1;
  }
  if (t.sig == 0) t.exp = 0;
  return t;
}

__device__ __forceinline__ int radix_of(const Fmt &f) { return f.kind == 0 ? f.mbits : (f.kind == 1 ? f.frac_bits : 0); }

// The running fp32 value as a term at `radix`, subnormals normalised (mma.py:85-91).
__device__ __forceinline__ Term c_term(float c, int radix) {
  Term t;
  uint32_t u = f2u(c);
  uint32_t a = u & 0x7FFFFFFFu;
  t.neg = (u >> 31) != 0;
  t.zero = a == 0;
  t.nan = a > kInf;
  t.inf = a == kInf;
  t.sig = 0;
  t.exp = 0;
  if (t.zero || t.nan || t.inf) return t;
  uint32_t field = a >> 23;
  uint32_t sig = field ? ((a & 0x7FFFFFu) | 0x800000u) : (a & 0x7FFFFFu);
  int exp = field ? (int)field - 127 : -126;
  int lead = ilog2_u32(sig);
  t.exp = exp + lead - 23;
  t.sig = shift_u64(sig, radix - lead);
  return t;
}

// Flags and exponent of a product of two terms (mma.py:94-97); the caller sets sig.
__device__ __forceinline__ Term combine(const Term &a, const Term &b) {
  Term t;
  t.nan = a.nan || b.nan || (a.inf && b.zero) || (b.inf && a.zero);
  t.inf = (a.inf || b.inf) && !t.nan;
  t.zero = a.zero || b.zero;
  t.neg = a.neg != b.neg;
  t.exp = a.exp + b.exp;
  t.sig = 0;
  return t;
}

// (a * b) shifted by `amount` (mma.py:55-72): 128-bit product, result assumed to fit 64 bits.
__device__ __forceinline__ uint64_t mul_shift(uint64_t a, uint64_t b, int amount) {
  unsigned __int128 p = (unsigned __int128)a * b;
  if (amount >= 0) return (uint64_t)(p << (amount > 127 ? 127 : amount));
  int r = -amount;
  if (r >= 128) return 0ull;
  return (uint64_t)(p >> r);
}

__device__ __forceinline__ bool active(const Term &t) { return !(t.zero || t.nan || t.inf); }

// Accumulates the alignment sum over terms in two passes (mma.py:104-115).
struct FdaState {
  int emax;
  bool any_nan, pos_inf, neg_inf, all_zero;
};

__device__ __forceinline__ void fda_scan(FdaState &s, const Term &t) {
  if (active(t) && t.exp > s.emax) s.emax = t.exp;
  s.any_nan |= t.nan;
  if (t.inf) {
    if (t.neg) s.neg_inf = true;
    else s.pos_inf = true;
  }
  s.all_zero &= t.zero;
}

__device__ __forceinline__ int64_t fda_aligned(const Term &t, int emax) {
  if (!active(t)) return 0;
  int64_t m = (int64_t)shift_u64(t.sig, t.exp - emax);
  return t.neg ? -m : m;
}

// Normalise an exact fixed-point sum into fp32 (mma.py:118-137).
__device__ __forceinline__ float fixed_to_fp32(int64_t total, int exponent, int radix, bool rne, bool fda) {
  if (total == 0) return 0.0f;
  uint64_t mag = total < 0 ? (uint64_t)(-total) : (uint64_t)total;
  int lead = ilog2_u64(mag);
  int biased = lead + exponent - radix + 127;
  int precision = fda ? (radix < 23 ? radix : 23) : 23;
  uint32_t bits;
  if (biased <= 0) {
    int sub_shift = 149 + exponent - radix;
    uint64_t sub = fda ? shift_u64(mag, sub_shift) : rounded_shift_u64(mag, sub_shift);
    bits = (uint32_t)sub;
  } else {
    int amount = precision - lead;
    uint64_t kept = rne ? rounded_shift_u64(mag, amount) : shift_u64(mag, amount);
    int carry = kept >= (1ull << (precision + 1)) ? 1 : 0;
    if (carry) kept >>= 1;
    int nexp = biased + carry;
    bits = nexp >= 255 ? kInf : (((uint32_t)nexp << 23) | ((uint32_t)(kept << (23 - precision)) & 0x7FFFFFu));
  }
  if (total < 0) bits |= 0x80000000u;
  return u2f(bits);
}

__device__ __forceinline__ float fda_finish(const FdaState &s, int64_t total, int radix, bool rne, float c) {
  float r = fixed_to_fp32(total, s.emax, radix, rne, true);
  if (s.all_zero) r = c;
  bool nan = s.any_nan || (s.pos_inf && s.neg_inf);
  if (nan) return u2f(kQNaN);
  if (s.neg_inf) return -INFINITY;
  if (s.pos_inf) return INFINITY;
  return r;
}

// One fused dot-add of `count` terms produced by term(i) with running value c at `radix`
// (mma.py:140-151). term(i) is evaluated twice (scan, then sum).
template <class TermFn>
__device__ __forceinline__ float fda(int count, TermFn term, float c, int radix, bool rne) {
  Term ct = c_term(c, radix);
  FdaState s{kNoExp, false, false, false, true};
  fda_scan(s, ct);
  for (int i = 0; i < count; ++i) fda_scan(s, term(i));
  int64_t total = fda_aligned(ct, s.emax);
  for (int i = 0; i < count; ++i) total += fda_aligned(term(i), s.emax);
  return fda_finish(s, total, radix, rne, c);
}

}  // namespace tc
