// Emulated GEMM entry point and the exact generic kernel.
//
// The generic kernel computes one output per thread in TriCast's order (src/tricast/reference/
// mma.py:286-384): CoFDA chunks from k = 0 (fused, decoupled or promoted), GDFS tiles of groups,
// exact integer sums, or IEEE fp32 / fp64 FMA chains, then the epilogue. It handles every
// operand format, scale layout and Inf/NaN rule, and is the path for anything the fast kernels
// (tc_gemm_fast.cu) do not claim.
#include <cstring>
#include <string>

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

// 16 x 16 output tiles, grid-stride, one output per thread. Behind a fast kernel the grid is small, so
// the common case (flag clear) costs a few hundred blocks that read two words and exit.
// Runs of the exact kernel behind a fast kernel that declined its operands (or timed out), per device.
__device__ unsigned long long g_exact_fallbacks;

__global__ void __launch_bounds__(256) gemm_generic_kernel(GemmDesc g, const int32_t *only_if_flag) {
  if (only_if_flag && only_if_flag[0] == 0 && only_if_flag[1] == 0) return;  // the fast kernel took it
  if (only_if_flag && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(&g_exact_fallbacks, 1ull);
  const int64_t tiles_n = (g.N + 15) / 16, tiles = tiles_n * ((g.M + 15) / 16);
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t n = (tile % tiles_n) * 16 + (threadIdx.x & 15);
    const int64_t m = (tile / tiles_n) * 16 + (threadIdx.x >> 4);
    if (m < g.M && n < g.N) generic_output(g, m, n);
  }
}

// Device-side finiteness check (int_exact operands).
__global__ void any_nonfinite_kernel(const void *v, int dt, int64_t n, int32_t *flag) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  bool bad = false;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float x = load_as_float(v, dt, i);
    bad |= (f2u(x) & 0x7F800000u) == 0x7F800000u;
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicExch(flag, 1);
}

static std::string check_operand(const tc_operand &o, const char *side) {
  std::string s(side);
  if (o.rows < 0 || o.K < 0) return s + ": negative shape";
  if (o.rows * o.K > 0 && !o.values) return s + ": null values";
  if (o.values_dtype < 0 || o.values_dtype > 2) return s + ": unsupported values dtype";
  std::string e = fmt_error(o.fmt);
  if (!e.empty()) return s + " format: " + e;
  if (o.scale_kind < 0 || o.scale_kind > 3) return s + ": unknown scale_kind";
  if (o.scale_kind != SK_NONE && !o.scale) return s + ": scale_kind set without a scale";
  if (o.scale_kind == SK_K) {
    if (o.k_domain <= 0) return s + ": K-varying scales need k_domain > 0";
    if (o.has_scale_fmt) {
      e = fmt_error(o.scale_fmt);
      if (!e.empty()) return s + " scale format: " + e;
    }
  }
  return "";
}

static OpDesc make_op(const tc_operand &o) {
  OpDesc d;
  std::memset(&d, 0, sizeof(d));
  d.v = o.values;
  d.dt = o.values_dtype;
  d.rows = o.rows;
  d.K = o.K;
  d.f = derive(o.fmt);
  d.radix = o.fmt.kind == 0 ? o.fmt.mbits : (o.fmt.kind == 1 ? o.fmt.frac_bits : 0);
  d.scale = o.scale;
  d.skind = o.scale_kind;
  d.kd = o.k_domain > 0 ? o.k_domain : 1;
  d.nkd = o.scale_kind == SK_K ? (o.K + d.kd - 1) / d.kd : 1;
  tc_format sf = o.fmt;
  if (o.scale_kind == SK_K && o.has_scale_fmt) {
    sf = o.scale_fmt;
  } else {
    std::memset(&sf, 0, sizeof(sf));
    sf.kind = 0; sf.ebits = 8; sf.mbits = 23; sf.bias = 127; sf.special = 0; sf.is_signed = 1; sf.subnormals = 1;
  }
  d.sf = derive(sf);
  d.srad = sf.kind == 0 ? sf.mbits : (sf.kind == 1 ? sf.frac_bits : 0);
  d.field0 = o.scale_kind == SK_K && sf.kind == 2 && sf.ebits == 8 && sf.bias == 127;
  d.alpha = o.alpha;
  return d;
}

int build_desc(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec, const float *bias, void *out,
               GemmDesc &g) {
  if (!a || !b || !spec) return set_error("tc_gemm: null argument"), TC_INVALID_ARGUMENT;
  std::string e = check_operand(*a, "a");
  if (e.empty()) e = check_operand(*b, "b");
  if (!e.empty()) return set_error("tc_gemm: " + e), TC_INVALID_ARGUMENT;
  if (a->K != b->K) return set_error("operands must have the same K"), TC_INVALID_ARGUMENT;
  if (spec->algorithm < 0 || spec->algorithm > 4) return set_error("unknown algorithm"), TC_INVALID_ARGUMENT;
  if (spec->out_format.kind != 0) return set_error("out_format must be a float format"), TC_INVALID_ARGUMENT;
  if (a->rows * b->rows > 0 && !out) return set_error("tc_gemm: null output"), TC_INVALID_ARGUMENT;
  if (spec->algorithm == ALG_COFDA && spec->chunk_size < 1) return set_error("chunk_size must be >= 1"), TC_INVALID_ARGUMENT;
  if (spec->algorithm == ALG_GDFS && (spec->group_size < 1 || spec->k_tile % spec->group_size ||
                                      spec->k_tile / spec->group_size > 8 || spec->k_tile < 1))
    return set_error("k_tile must be a positive multiple of group_size with at most 8 groups"), TC_INVALID_ARGUMENT;
  std::memset(&g, 0, sizeof(g));
  g.a = make_op(*a);
  g.b = make_op(*b);
  g.M = a->rows;
  g.N = b->rows;
  g.K = a->K;
  g.alg = spec->algorithm;
  g.F = spec->f_bits;
  g.CS = spec->chunk_size;
  g.decoupled = spec->c_mode == 1;
  g.F2 = spec->f2_bits;
  g.G = spec->g_bits;
  g.GS = spec->group_size;
  g.KT = spec->k_tile;
  g.rne = spec->norm_rounding == 1;
  g.apply = spec->scale_apply;
  g.PI = spec->promote_interval;
  g.of = derive(spec->out_format);
  g.out_dt = spec->out_dtype;
  const tc_format &of = spec->out_format;
  g.out_is_plain = of.ebits == 8 && of.mbits == 23 && of.bias == 127 && of.special == 0 && of.is_signed && of.subnormals;
  g.bias = bias;
  g.out = out;
  return TC_OK;
}

void launch_generic(const GemmDesc &g, const int32_t *only_if_flag, cudaStream_t s) {
  const int64_t tiles = ((g.N + 15) / 16) * ((g.M + 15) / 16);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t cap = (int64_t)sms * 8;
  gemm_generic_kernel<<<(unsigned)(tiles < cap ? tiles : cap), 256, 0, s>>>(g, only_if_flag);
  count_launch();
}

}  // namespace tc

using namespace tc;

extern "C" size_t tc_gemm_workspace(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec) {
  GemmDesc g;
  if (build_desc(a, b, spec, nullptr, (void *)1, g)) return 0;
  return fast_workspace(g);
}

extern "C" int tc_gemm(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec, const float *bias,
                       void *out, void *workspace, size_t workspace_bytes, tc_stream stream) {
  GemmDesc g;
  int st = build_desc(a, b, spec, bias, out, g);
  if (st) return st;
  if (g.M == 0 || g.N == 0) return TC_OK;
  cudaStream_t s = (cudaStream_t)stream;
  st = launch_fast(g, workspace, workspace_bytes, s);
  if (st != TC_UNSUPPORTED) return st;
  if ((g.M + 15) / 16 > 65535) return set_error("tc_gemm: too many rows for the generic kernel"), TC_INVALID_ARGUMENT;
  launch_generic(g, nullptr, s);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

extern "C" int tc_exact_fallbacks(uint64_t *count) {
  if (!count) return set_error("tc_exact_fallbacks: null argument"), TC_INVALID_ARGUMENT;
  unsigned long long v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_exact_fallbacks, sizeof(v));
  if (e != cudaSuccess) return set_error(std::string("tc_exact_fallbacks: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  *count = (uint64_t)v;
  return TC_OK;
}

extern "C" int tc_any_nonfinite(const void *values, int32_t dtype, int64_t n, int32_t *flag, tc_stream stream) {
  if (n <= 0) return TC_OK;
  if (!values || !flag || dtype < 0 || dtype > 2) return set_error("tc_any_nonfinite: bad argument"), TC_INVALID_ARGUMENT;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  any_nonfinite_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(values, dtype, n, flag);
  ::tc::count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_any_nonfinite: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}
