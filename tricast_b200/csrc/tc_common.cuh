// Shared device code: derived format constants, the bit-level cast onto a format grid, container
// conversions and error reporting. Semantics follow TriCast's reference cast
// (src/tricast/reference/cast.py:18-179); the arithmetic here is integer work on the fp32 bit
// pattern (sign, exponent field, 24-bit significand), so no floating rescale is ever rounded.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "tricast_b200.h"

namespace tc {

// Derived constants of one format, computed on the host and passed by value to kernels.
struct Fmt {
  int kind;          // 0 float, 1 int, 2 pow2
  int mbits;         // float: fraction bits
  int emin, emax;    // float/pow2: exponent range of normals
  int special;       // 0 ieee, 1 fn, 2 fnuz, 3 none
  int is_signed;
  int subnormals;
  uint32_t max_bits;       // fp32 bits of max_normal (floats, pow2)
  uint32_t min_normal_bits;
  uint32_t min_sub_bits;   // fp32 bits of min_subnormal (floats) or min_normal (pow2)
  int frac_bits;           // int
  int64_t qmin, qmax;      // int
  int int_double;          // int: results can leave fp32's exact range -> compute in fp64
  int bias, ebits;         // pow2 / float field layout (codes)
};

// ---------------------------------------------------------------- host-side derivation
std::string fmt_error(const tc_format &f);
Fmt derive(const tc_format &f);
double fmt_max_normal(const tc_format &f);
double fmt_min_scale(const tc_format &f);   // min_subnormal (floats) / min_normal (pow2)
int fmt_emax_elem(const tc_format &f);      // floor(log2(max_normal))
void set_error(const std::string &msg);
void count_launch();  // every kernel launch of the library; read by tc_launch_count()
// Multiprocessor count of the current device (queried once per device ordinal); grid-stride
// kernels cap their grids at a multiple of it.
int sm_count();
// Poll limit of the staged kernels' pipeline waits for the next launches (negative = the kernels'
// defaults); set by tc_set_wait_limit, read at every launch.
int wait_polls();

// ---------------------------------------------------------------- small device helpers
__host__ __device__ __forceinline__ uint32_t f2u(float v) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(v);
#else
  uint32_t u; memcpy(&u, &v, 4); return u;
#endif
}
__host__ __device__ __forceinline__ float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float v; memcpy(&v, &u, 4); return v;
#endif
}

constexpr uint32_t kQNaN = 0x7FC00000u;
constexpr uint32_t kInf = 0x7F800000u;

__device__ __forceinline__ int ilog2_u64(uint64_t v) { return 63 - __clzll((long long)v); }  // v > 0
__device__ __forceinline__ int ilog2_u32(uint32_t v) { return 31 - __clz((int)v); }         // v > 0

// k * 2**q as fp32 bits for 0 <= k < 2**25 and q >= -149 (results below 2**-126 are exact
// subnormals because q >= -149). Magnitudes >= 2**128 give +Inf bits.
__device__ __forceinline__ uint32_t encode_scaled(uint32_t k, int q) {
  if (k == 0) return 0u;
  int lead = ilog2_u32(k);
  int e = lead + q;
  if (e >= -126) {
    if (e > 127) return kInf;
    uint32_t frac = lead <= 23 ? (k << (23 - lead)) : (k >> (lead - 23));
    return ((uint32_t)(e + 127) << 23) | (frac & 0x7FFFFFu);
  }
  return k << (q + 149);
}

// Whether stochastic rounding rounds a truncated magnitude up: u < rem / 2**shift with
// u = floor(noise / 2**(32 - sr_bits)) / 2**sr_bits (src/tricast/reference/cast.py:125-134),
// evaluated exactly in integers. rem < 2**24, shift > 0.
__device__ __forceinline__ bool sr_up(uint32_t rem, int shift, uint32_t noise, int sr_bits) {
  if (rem == 0) return false;
  uint64_t r = (uint64_t)(noise >> (32 - sr_bits));
  if (shift <= sr_bits) return r < ((uint64_t)rem << (sr_bits - shift));
  int d = shift - sr_bits;
  uint64_t lim = d >= 32 ? 0ull : ((uint64_t)(rem - 1) >> d);
  return r <= lim;
}

// Increment decision for a magnitude truncated by `shift` bits with remainder `rem`
// (src/tricast/reference/cast.py:112-135).
__device__ __forceinline__ bool round_inc(uint32_t kept, uint32_t rem, int shift, bool neg, int rounding,
                                          uint32_t noise, int sr_bits) {
  if (shift <= 0 || rem == 0) return false;
  switch (rounding) {
    case TC_RNE: {
      if (shift > 24) return false;  // rem < 2**24 <= half
      uint32_t half = 1u << (shift - 1);
      return rem > half || (rem == half && (kept & 1u));
    }
    case TC_RNA: {
      if (shift > 24) return false;
      return rem >= (1u << (shift - 1));
    }
    case TC_RTZ: return false;
    case TC_RUP: return !neg;
    case TC_RDN: return neg;
    default: return sr_up(rem, shift, noise, sr_bits);
  }
}

// Overflow value of a float format (src/tricast/reference/cast.py:138-147), magnitude bits.
__device__ __forceinline__ uint32_t overflow_bits(const Fmt &f, bool neg, int rounding, bool saturate) {
  if (saturate || f.special == 3) return f.max_bits;
  if (f.special == 1 || f.special == 2) return kQNaN;
  bool away = rounding == TC_RTZ ? false : rounding == TC_RUP ? !neg : rounding == TC_RDN ? neg : true;
  return away ? kInf : f.max_bits;
}

// Power-of-two formats (E8M0): round the value, ties up; clamp below; NaN for negatives, NaN and
// non-saturating overflow (src/tricast/reference/cast.py:156-179).
__device__ __forceinline__ float cast_pow2(uint32_t bits, const Fmt &f, int rounding, bool saturate) {
  uint32_t a = bits & 0x7FFFFFFFu;
  bool neg = (bits >> 31) != 0;
  if (a > kInf || (neg && a != 0)) return u2f(kQNaN);
  if (a == 0) return u2f(f.min_sub_bits);
  bool over;
  int e;
  if (a == kInf) {
    over = true;
    e = f.emax;
  } else {
    uint32_t field = a >> 23;
    uint32_t sig = field ? ((a & 0x7FFFFFu) | 0x800000u) : a;
    int lead = ilog2_u32(sig);                          // 23 for normals
    e = field ? (int)field - 127 : lead - 149;          // exact floor(log2 |x|)
    uint32_t below = sig & ((1u << lead) - 1u);          // bits under the leading one
    bool up = false;
    if (rounding == TC_RNE || rounding == TC_RNA) up = lead > 0 && (below >> (lead - 1)) != 0;
    else if (rounding == TC_RUP) up = below != 0;
    e += up;
    if (e < f.emin) e = f.emin;
    over = e > f.emax;
  }
  if (over) return saturate ? u2f(f.max_bits) : u2f(kQNaN);
  // 2**e for e in [emin, emax]; values below fp32's subnormal range round like fp64 -> fp32 RNE.
  if (e >= -126) return u2f((uint32_t)(e + 127) << 23);
  if (e >= -149) return u2f(1u << (e + 149));
  return 0.0f;  // 2**-150 ties to the even 0; smaller powers round to 0
}

// Integer (fixed-point) formats: k * 2**-frac_bits with k clamped to [qmin, qmax]
// (src/tricast/reference/cast.py:53-73).
__device__ __forceinline__ float cast_int(uint32_t bits, const Fmt &f, int rounding, uint32_t noise, int sr_bits) {
  uint32_t a = bits & 0x7FFFFFFFu;
  bool neg = (bits >> 31) != 0 && a != 0;    // -0 is not "< 0"
  uint32_t sign = bits & 0x80000000u;
  if (a > kInf) return u2f(bits);
  int64_t bound = neg ? -f.qmin : f.qmax;
  if (!f.is_signed && neg) bound = 0;
  uint64_t k;
  if (a == kInf) {
    k = (uint64_t)bound;
  } else {
    uint32_t field = a >> 23;
    uint32_t sig = field ? ((a & 0x7FFFFFu) | 0x800000u) : a;
    int e32 = field ? (int)field - 127 : -126;
    int q = -f.frac_bits;
    int shift = q - e32 + 23;
    if (shift <= 0) {
      k = (-shift) >= 40 ? ~0ull : ((uint64_t)sig << (-shift));
    } else {
      uint32_t kept = shift >= 32 ? 0u : (sig >> shift);
      uint32_t rem = shift >= 32 ? sig : (sig & ((1u << shift) - 1u));
      k = kept + (round_inc(kept, rem, shift, neg, rounding, noise, sr_bits) ? 1u : 0u);
    }
    if (k > (uint64_t)bound) k = (uint64_t)bound;
  }
  float mag;
  if (f.int_double) {
    mag = __double2float_rn(ldexp((double)k, -f.frac_bits));
  } else {
    mag = u2f(encode_scaled((uint32_t)k, -f.frac_bits));
  }
  if (!f.is_signed) return mag;                 // unsigned grids carry no sign, not even -0
  return u2f(f2u(mag) | sign);
}

// Float (ExMy) formats (src/tricast/reference/cast.py:43-83).
__device__ __forceinline__ float cast_float(uint32_t bits, const Fmt &f, int rounding, bool saturate,
                                            uint32_t noise, int sr_bits) {
  uint32_t a = bits & 0x7FFFFFFFu;
  uint32_t sign = bits & 0x80000000u;
  if (a > kInf) return u2f(bits);
  if (!f.subnormals && a < f.min_normal_bits) a = 0;  // flushed to a signed zero
  bool neg = sign != 0 && a != 0;                     // "x < 0" after the flush
  uint32_t mag;
  if (a == kInf) {
    mag = overflow_bits(f, neg, rounding, saturate);
  } else {
    uint32_t field = a >> 23;
    uint32_t sig = field ? ((a & 0x7FFFFFu) | 0x800000u) : a;
    int e32 = field ? (int)field - 127 : -126;
    int q = (e32 > f.emin ? e32 : f.emin) - f.mbits;
    int shift = q - e32 + 23;
    if (shift <= 0) {
      mag = a;  // already on the grid
    } else {
      uint32_t kept = shift >= 32 ? 0u : (sig >> shift);
      uint32_t rem = shift >= 32 ? sig : (sig & ((1u << shift) - 1u));
      kept += round_inc(kept, rem, shift, neg, rounding, noise, sr_bits) ? 1u : 0u;
      mag = encode_scaled(kept, q);
    }
    if (mag > f.max_bits) mag = overflow_bits(f, neg, rounding, saturate);
  }
  uint32_t out = mag | sign;
  if ((f.special == 2 || !f.is_signed) && (mag == 0)) out = 0;
  if (!f.is_signed && neg) out = saturate ? 0u : kQNaN;
  return u2f(out);
}

__device__ __forceinline__ float cast_to(float x, const Fmt &f, int rounding, bool saturate, uint32_t noise,
                                         int sr_bits) {
  uint32_t bits = f2u(x);
  if (f.kind == 0) return cast_float(bits, f, rounding, saturate, noise, sr_bits);
  if (f.kind == 1) return cast_int(bits, f, rounding, noise, sr_bits);
  return cast_pow2(bits, f, rounding, saturate);
}

// ---------------------------------------------------------------- containers
__device__ __forceinline__ float load_as_float(const void *p, int dtype, int64_t i) {
  if (dtype == TC_F32) return static_cast<const float *>(p)[i];
  if (dtype == TC_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

// Exact store of a grid value into its container. NaN becomes the canonical quiet NaN that
// PyTorch's own conversions produce (bf16 0x7FC0, fp16 0x7E00).
__device__ __forceinline__ void store_container(void *p, int dtype, int64_t i, float v) {
  if (dtype == TC_F32) {
    static_cast<float *>(p)[i] = v;
  } else if (dtype == TC_BF16) {
    uint32_t u = f2u(v);
    uint16_t h = ((u & 0x7FFFFFFFu) > kInf) ? (uint16_t)0x7FC0 : (uint16_t)(u >> 16);
    static_cast<uint16_t *>(p)[i] = h;
  } else {
    __half h = (v != v) ? __ushort_as_half((unsigned short)0x7E00) : __float2half_rn(v);
    static_cast<__half *>(p)[i] = h;
  }
}

}  // namespace tc
