// The exact generic GEMM output: one output computed in TriCast's order (src/tricast/reference/
// mma.py:286-384) for every operand format, scale layout, accumulation model and Inf/NaN rule. Used by
// the generic kernel (tc_gemm.cu) and, for its fallback, by the small-M scan kernel (tc_gemv.cu).
#pragma once

#include "tc_gemm.cuh"

namespace tc {

__device__ __forceinline__ float op_value(const OpDesc &o, int64_t r, int64_t k) {
  return load_as_float(o.v, o.dt, r * o.K + k);
}

// K-scale of operand o at row r, element k, as a term; standard E8M0 2**-127 is a zero scale
// (mma.py:241-252).
__device__ __forceinline__ Term kscale_term(const OpDesc &o, int64_t r, int64_t k, float &raw) {
  raw = o.scale[r * o.nkd + k / o.kd];
  Term t = decode_term(raw, o.sf);
  if (o.field0 && f2u(raw) == 0x00400000u) {
    t.zero = true;
    t.sig = 0;
  }
  return t;
}

struct ScaleFactor {
  Term t;          // the combined scale (both sides multiplied when both have K scales)
  int radix;
  bool present;
  bool fnan, fzero;  // NaN / zero of any individual factor (the GDFS group rule reads these)
};

__device__ __forceinline__ ScaleFactor scale_factor(const GemmDesc &g, int64_t m, int64_t n, int64_t k) {
  ScaleFactor s;
  s.present = false;
  s.radix = 0;
  s.fnan = s.fzero = false;
  float raw;
  bool ha = g.a.skind == SK_K, hb = g.b.skind == SK_K;
  if (ha) {
    s.t = kscale_term(g.a, m, k, raw);
    s.radix = g.a.srad;
    s.present = true;
    s.fnan = s.t.nan;
    s.fzero = s.t.zero;
  }
  if (hb) {
    Term tb = kscale_term(g.b, n, k, raw);
    s.fnan |= tb.nan;
    s.fzero |= tb.zero;
    if (ha) {
      Term c = combine(s.t, tb);
      c.sig = s.t.sig * tb.sig;
      s.t = c;
      s.radix += g.b.srad;
    } else {
      s.t = tb;
      s.radix = g.b.srad;
    }
    s.present = true;
  }
  return s;
}

__device__ __forceinline__ Term product(const GemmDesc &g, int64_t m, int64_t n, int64_t k) {
  Term ta = decode_term(op_value(g.a, m, k), g.a.f);
  Term tb = decode_term(op_value(g.b, n, k), g.b.f);
  Term t = combine(ta, tb);
  t.sig = ta.sig * tb.sig;
  return t;
}

// A product moved to radix F, with product-level K scales when scale_apply == product
// (mma.py:295-299, 255-269).
__device__ __forceinline__ Term product_at_f(const GemmDesc &g, int64_t m, int64_t n, int64_t k) {
  Term t = product(g, m, n, k);
  int rr = g.a.radix + g.b.radix;
  if (g.apply == AP_PRODUCT) {
    ScaleFactor s = scale_factor(g, m, n, k);
    if (s.present) {
      Term r = combine(t, s.t);
      r.sig = mul_shift(t.sig, s.t.sig, g.F - rr - s.radix);
      return r;
    }
  }
  t.sig = shift_u64(t.sig, g.F - rr);
  return t;
}

// One GDFS group: products summed exactly at G, then group-level scales (mma.py:323-332).
__device__ __forceinline__ Term gdfs_group(const GemmDesc &g, int64_t m, int64_t n, int64_t start, int64_t end) {
  int rr = g.a.radix + g.b.radix;
  FdaState s{kNoExp, false, false, false, true};
  for (int64_t k = start; k < end; ++k) {
    Term t = product(g, m, n, k);
    t.sig = shift_u64(t.sig, g.G - rr);
    fda_scan(s, t);
  }
  int64_t total = 0;
  for (int64_t k = start; k < end; ++k) {
    Term t = product(g, m, n, k);
    t.sig = shift_u64(t.sig, g.G - rr);
    total += fda_aligned(t, s.emax);
  }
  bool nan = s.any_nan || (s.pos_inf && s.neg_inf);
  bool inf = !nan && (s.pos_inf || s.neg_inf);
  bool exceptional = nan || inf;
  Term t;
  t.exp = s.emax;
  t.sig = total < 0 ? (uint64_t)(-total) : (uint64_t)total;
  t.zero = total == 0 && !exceptional;
  t.nan = nan;
  t.inf = inf;
  t.neg = inf ? s.neg_inf : total < 0;
  if (g.apply != AP_GROUP) {
    t.sig = shift_u64(t.sig, g.F - g.G);
    return t;
  }
  ScaleFactor sf = scale_factor(g, m, n, start);
  if (!sf.present) {
    t.sig = shift_u64(t.sig, g.F - g.G);
    return t;
  }
  // Group rule: an explicit zero precedes Inf, but never masks NaN (mma.py:270-276).
  Term r;
  bool any_nan = t.nan || sf.fnan;
  bool any_zero = t.zero || sf.fzero;
  r.nan = any_nan;
  r.zero = any_zero && !any_nan;
  r.inf = (t.inf || sf.t.inf) && !(any_nan || any_zero);
  r.neg = t.neg != sf.t.neg;
  r.exp = t.exp + sf.t.exp;
  r.sig = mul_shift(t.sig, sf.t.sig, g.F - g.G - sf.radix);
  return r;
}

// only_if_flag, when given, points at the fast path's {fallback flag, timeout status} pair: the
// exact kernel runs behind a fast kernel only if the fast kernel declined the operands or one of its
// bounded waits gave up, so a timeout still ends in the exact result.
// One output of the exact product, any algorithm (src/tricast/reference/mma.py:339-384).
__device__ __forceinline__ void generic_output(const GemmDesc &g, int64_t m, int64_t n) {
  const int64_t K = g.K;
  float acc = 0.0f;
  if (g.alg == ALG_COFDA) {
    int64_t interval = g.PI ? g.PI : (K > 0 ? K : 1);
    for (int64_t begin = 0; begin < K; begin += interval) {
      float partial = g.PI ? 0.0f : acc;
      int64_t stop = begin + interval < K ? begin + interval : K;
      for (int64_t start = begin; start < stop; start += g.CS) {
        int64_t end = start + g.CS < stop ? start + g.CS : stop;
        int cnt = (int)(end - start);
        auto term = [&](int i) { return product_at_f(g, m, n, start + i); };
        if (g.decoupled && !g.PI) {
          float p = fda(cnt, term, 0.0f, g.F, g.rne);
          Term pt = c_term(p, g.F2);
          partial = fda(1, [&](int) { return pt; }, partial, g.F2, g.rne);
        } else {
          partial = fda(cnt, term, partial, g.F, g.rne);
        }
      }
      if (g.PI) {
        float w = 1.0f;
        if (g.a.skind == SK_K) w = __fmul_rn(w, g.a.scale[m * g.a.nkd + begin / g.a.kd]);
        if (g.b.skind == SK_K) w = __fmul_rn(w, g.b.scale[n * g.b.nkd + begin / g.b.kd]);
        acc = __fmaf_rn(partial, w, acc);
      } else {
        acc = partial;
      }
    }
  } else if (g.alg == ALG_GDFS) {
    for (int64_t tile = 0; tile < K; tile += g.KT) {
      Term groups[8];
      int ng = 0;
      int64_t tend = tile + g.KT < K ? tile + g.KT : K;
      for (int64_t start = tile; start < tend; start += g.GS) {
        int64_t end = start + g.GS < K ? start + g.GS : K;
        groups[ng++] = gdfs_group(g, m, n, start, end);
      }
      acc = fda(ng, [&](int i) { return groups[i]; }, acc, g.F, g.rne);
    }
  } else if (g.alg == ALG_INT_EXACT) {
    int64_t total = 0;
    for (int64_t k = 0; k < K; ++k) {
      Term t = product(g, m, n, k);
      total += t.neg ? -(int64_t)t.sig : (int64_t)t.sig;
    }
    acc = fixed_to_fp32(total, -(g.a.radix + g.b.radix), 0, true, false);
  } else if (g.alg == ALG_FP64) {
    double accd = 0.0;
    for (int64_t k = 0; k < K; ++k) {
      float av = op_value(g.a, m, k), bv = op_value(g.b, n, k);
      if (g.apply == AP_OPERAND) {
        if (g.a.skind == SK_K) av = __fmul_rn(av, g.a.scale[m * g.a.nkd + k / g.a.kd]);
        if (g.b.skind == SK_K) bv = __fmul_rn(bv, g.b.scale[n * g.b.nkd + k / g.b.kd]);
      }
      accd = __fma_rn((double)av, (double)bv, accd);
    }
    acc = __double2float_rn(accd);
  } else {
    for (int64_t k = 0; k < K; ++k) {
      float av = op_value(g.a, m, k), bv = op_value(g.b, n, k);
      if (g.apply == AP_OPERAND) {
        if (g.a.skind == SK_K) av = __fmul_rn(av, g.a.scale[m * g.a.nkd + k / g.a.kd]);
        if (g.b.skind == SK_K) bv = __fmul_rn(bv, g.b.scale[n * g.b.nkd + k / g.b.kd]);
      }
      acc = __fmaf_rn(av, bv, acc);
    }
  }
  store_out(g, m, n, epilogue(g, m, n, acc));
}

}  // namespace tc
