// E2M1 x E2M1 GDFS building blocks shared by the tiled kernel (tc_gemm_fast.cu) and the small-M
// kernel (tc_gemv.cu): the operand record encoder, the scale word, exponent-class labels, DP4A group
// dot products and the running value's FDA term.
#pragma once

#include "tc_gemm.cuh"

namespace tc {
namespace fp4 {

constexpr int kGS = 16;          // GDFS group size of the fast path
constexpr int kNone = -(1 << 28);  // "no active term" exponent
constexpr int kBig = 1 << 28;

// Scale word: es (int16, biased by 0x8000 in bits 0..15), ms (bits 16..23), sign (bit 24), the
// group's largest exponent class (bits 25..26) and "every code of the group is zero" (bit 27).
__host__ __device__ __forceinline__ uint32_t pack_scale(int es, uint32_t ms, uint32_t neg) {
  return ((uint32_t)(es + 0x8000) & 0xFFFFu) | ((ms & 0xFFu) << 16) | ((neg & 1u) << 24);
}

// Doubled E2M1 codes of one group (int8 lanes of q; elements j >= valid are zero), the exponent-class
// masks (c0: non-zero, c1: |v| >= 2, c2: |v| >= 4) and whether any value is off the E2M1 grid
// (NaN / Inf included).
__device__ __forceinline__ void e2m1_codes(const float (&vin)[kGS], int valid, uint4 &q, uint32_t &c0, uint32_t &c1,
                                           uint32_t &c2, bool &bad) {
  uint32_t codes[4] = {0, 0, 0, 0};
  c0 = c1 = c2 = 0;
#pragma unroll
  for (int j = 0; j < kGS; ++j) {
    int qv = 0;
    if (j < valid) {
      const float t = 2.0f * vin[j];  // exact for finite values
      const int ti = (int)t;
      const int at = ti < 0 ? -ti : ti;
      const bool on_grid = (float)ti == t && (at <= 4 || at == 6 || at == 8 || at == 12);
      if (!on_grid) bad = true;
      qv = ti;
      if (at) {
        c0 |= 1u << j;
        if (at >= 4) c1 |= 1u << j;
        if (at >= 8) c2 |= 1u << j;
      }
    }
    codes[j >> 2] |= ((uint32_t)(qv & 0xFF)) << (8 * (j & 3));
  }
  q = make_uint4(codes[0], codes[1], codes[2], codes[3]);
}

// The doubled E2M1 code of one container element from its bit pattern, without float <-> int
// conversions: |v| in {0.5, 1, 1.5, 2, 3, 4, 6} sits at (bits - bits(0.5)) >> (fraction bits - 1) in
// {0, 2, 3, 4, 5, 6, 7} with the lower fraction bits zero, and the code's magnitude is the nibble
// of 0xC8643201 at that index (index 1 is 0.75, off the grid). Zero (either sign) is code 0. Anything
// else (off-grid values, NaN, Inf) clears ok.
template <int DT>
__device__ __forceinline__ int e2m1_code_bits(uint32_t bits, bool &ok) {
  constexpr uint32_t kAbs = DT == TC_F32 ? 0x7FFFFFFFu : 0x7FFFu;
  constexpr int kHalf = DT == TC_F32 ? 0x3F000000 : (DT == TC_BF16 ? 0x3F00 : 0x3800);
  constexpr int kShift = DT == TC_F32 ? 22 : (DT == TC_BF16 ? 6 : 9);
  constexpr int kLow = (1 << kShift) - 1;
  constexpr uint32_t kSign = DT == TC_F32 ? 0x80000000u : 0x8000u;
  const uint32_t a = bits & kAbs;
  const int d = (int)a - kHalf;
  const int r = d >> kShift;
  const bool on = a == 0u || ((d & kLow) == 0 && (unsigned)r <= 7u && r != 1);
  ok &= on;
  const int mag = a == 0u ? 0 : (int)((0xC8643201u >> ((4 * r) & 31)) & 0xFu);
  return (bits & kSign) ? -mag : mag;
}

// PTX prmt in its default mode: result byte k is byte c[k] & 7 of {b, a}, sign-replicated when bit 3 of
// the selector nibble is set.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Doubled E2M1 codes of four bf16 container values (w0 holds elements 0 and 1, element 0 in the low
// half; w1 elements 2 and 3) as int8 lanes, four at a time:
//   * bits 8..6 of a bf16 E2M1 value (the exponent's low bit and the top two fraction bits) index
//     its magnitude: 2.0, 3.0, 4.0, 6.0, 0.5, 0.75, 1.0, 1.5 for indices 0..7, so one byte permute
//     of a table gives the four |2v| (0.75 is off the grid and maps to 0);
//   * zero elements (+-0) are masked out through bit 15 of each half of (|w| + 0x7FFF);
//   * the grid check rebuilds each magnitude's bf16 pattern from its code and compares it with the
//     input, which rejects everything else (other fraction bits, other exponents, NaN, Inf, 0.75);
//   * signs become byte masks by sign-replicating permutes, and a negative code is (m ^ 0xFF) + 1
//     per byte (no carry: m >= 1 where the mask is set).
// mag returns the four code magnitudes |2v|, one byte each: bit 3 of a byte marks |v| >= 4, bits
// 2..3 |v| >= 2. e2m1_codes4_bf16 collects them into orm across calls.
__device__ __forceinline__ uint32_t e2m1_codes4_bf16_mag(uint32_t w0, uint32_t w1, bool &ok, uint32_t &mag) {
  const uint32_t x0 = w0 & 0x7FFF7FFFu, x1 = w1 & 0x7FFF7FFFu;
  const uint32_t nz = prmt(x0 + 0x7FFF7FFFu, x1 + 0x7FFF7FFFu, 0xFDB9u);
  const uint32_t t0 = (w0 >> 6) & 0x00070007u, t1 = (w1 >> 6) & 0x00070007u;
  const uint32_t sel = ((t0 | (t0 >> 12)) & 0xFFu) | (((t1 | (t1 >> 12)) & 0xFFu) << 8);
  mag = prmt(0x0C080604u, 0x03020001u, sel) & nz;
  const uint32_t live8 = mag + 0x7F7F7F7Fu;  // bit 7 of byte k: element k has a code
  const uint32_t lo = prmt(0xC0804000u, 0xC0804000u, sel), hi = prmt(0x40404040u, 0x3F3F3F3Fu, sel);
  const uint32_t r0 = prmt(lo, hi, 0x5140u) & prmt(live8, live8, 0x9988u);
  const uint32_t r1 = prmt(lo, hi, 0x7362u) & prmt(live8, live8, 0xBBAAu);
  ok &= (r0 == x0) & (r1 == x1);
  const uint32_t smask = prmt(w0, w1, 0xFDB9u) & prmt(live8, live8, 0xBA98u);
  return (mag ^ smask) + (smask & 0x01010101u);
}

__device__ __forceinline__ uint32_t e2m1_codes4_bf16(uint32_t w0, uint32_t w1, bool &ok, uint32_t &orm) {
  uint32_t mag;
  const uint32_t codes = e2m1_codes4_bf16_mag(w0, w1, ok, mag);
  orm |= mag;
  return codes;
}

// Bit 7 of byte k of x to bit k (k = 0..3): the four terms of the product land on distinct bits
// below bit 28 or on bits 28..31, so no carry reaches the result.
__device__ __forceinline__ uint32_t byte_msb4(uint32_t x) { return ((x & 0x80808080u) * 0x00204081u) >> 28; }

// The exponent-class masks of four elements from their code magnitudes (bytes of 2|v|, at most 12):
// c0 non-zero, c1 |v| >= 2 (magnitude >= 4), c2 |v| >= 4 (magnitude >= 8), one bit per element.
__device__ __forceinline__ void class_masks4(uint32_t mag, uint32_t &c0, uint32_t &c1, uint32_t &c2) {
  c0 = byte_msb4(mag + 0x7F7F7F7Fu);
  c1 = byte_msb4((mag & 0x0C0C0C0Cu) + 0x7F7F7F7Fu);
  c2 = byte_msb4((mag & 0x08080808u) << 4);
}

// A group's K scale as (es, ms, sign) at the scale format's radix, or zero (the group becomes a zero
// term, mma.py:270-276). Scale significands up to 4 bits (UE4M3, E4M3, E8M0) keep
// |D| * ms_a * ms_b < 2**20; |es| <= 400 keeps every fp64 power 2**(es_a + es_b - srad - 2) normal.
__device__ __forceinline__ uint32_t group_scale_word(float s, const Fmt &sf, int field0, bool &zero, bool &bad) {
  const Term t = decode_term(s, sf);
  if (t.nan || t.inf || t.sig > 15 || t.exp < -400 || t.exp > 400) bad = true;
  zero = t.zero || (field0 && f2u(s) == 0x00400000u);
  return zero ? pack_scale(0, 0, 0) : pack_scale(t.exp, (uint32_t)t.sig, t.neg ? 1u : 0u);
}

// group_scale_word for a normal fp32 scale value of a float or power-of-two scale format, on the bit
// pattern (decode_term's exponent max(floor log2 |s|, emin) and truncated significand at the format's
// radix); zero, subnormal and non-finite scales and integer scale formats take group_scale_word.
__device__ __forceinline__ uint32_t group_scale_word_fast(float s, const Fmt &sf, int field0, bool &zero, bool &bad) {
  const uint32_t u = f2u(s), a = u & 0x7FFFFFFFu, field = a >> 23;
  if (field == 0u || field == 255u || sf.kind == 1) return group_scale_word(s, sf, field0, zero, bad);
  zero = false;
  const int fl = (int)field - 127;
  int e = fl;
  uint32_t sig = 1;
  if (sf.kind == 0) {
    e = fl > sf.emin ? fl : sf.emin;
    const int r = 23 - sf.mbits + e - fl;
    sig = r >= 24 ? 0u : (((a & 0x7FFFFFu) | 0x800000u) >> r);
    if (sig == 0u) e = 0;
  }
  if (sig > 15u) bad = true;  // |e| <= 127 here
  return pack_scale(e, sig, u >> 31);
}

struct EncodeArgs {
  const void *v;
  int dt;
  int64_t rows, K, rows_pad, ntiles;
  int ng;                 // groups per K tile
  const float *scale;     // K scales or nullptr
  int64_t nkd;
  int kd;
  Fmt sf;
  int field0;
  uint4 *q;               // [ntiles * ng][rows_pad]
  uint4 *m;
  uint32_t *s;            // scale words [ntiles * ng][rows_pad]
  int32_t *flag;          // set when the fast path cannot take this operand
  int side;               // 0: A record layout, 1: B record layout
  int vec;                // rows start 16-byte aligned: whole groups load as vectors
};

// Encodes an operand into records [ntiles * ng][rows_pad] (tc_gemm_fast.cu).
__global__ void __launch_bounds__(256) encode_fp4_kernel(EncodeArgs e);

// Exponent-class masks of one group in the record layouts exp_class_max pairs up (A: side 0, B: side 1).
__device__ __forceinline__ uint4 a_masks(uint32_t c0, uint32_t c1, uint32_t c2) {
  return make_uint4(c0 | (c1 << 16), c2 | (c1 << 16), c2, c2);
}
__device__ __forceinline__ uint4 b_masks(uint32_t c0, uint32_t c1, uint32_t c2) {
  return make_uint4(c1 | (c0 << 16), c1 | (c2 << 16), c0, c2 | (c1 << 16));
}

__device__ __forceinline__ int exp_class_max(const uint4 &a, const uint4 &b) {
  // a = {A0|A1<<16, A2|A1<<16, A2, A2}, b = {B1|B0<<16, B1|B2<<16, B0, B2|B1<<16}
  uint32_t t1 = a.x & b.x;                  // A0&B1 | A1&B0        (sum >= 1)
  uint32_t t2 = (a.x & b.w) | (a.z & b.z);  // A0&B2 | A1&B1 | A2&B0 (sum >= 2)
  uint32_t t3 = a.y & b.y;                  // A2&B1 | A1&B2        (sum >= 3)
  uint32_t t4 = a.w & b.w;                  // A2&B2                (sum = 4; a.w has no high half)
  return (int)(t1 != 0) + (int)(t2 != 0) + (int)(t3 != 0) + (int)(t4 != 0);
}

__device__ __forceinline__ int dot16(const uint4 &a, const uint4 &b) {
  int d = __dp4a((int)a.x, (int)b.x, 0);
  d = __dp4a((int)a.y, (int)b.y, d);
  d = __dp4a((int)a.z, (int)b.z, d);
  return __dp4a((int)a.w, (int)b.w, d);
}

__device__ __forceinline__ int scale_exp(uint32_t w) { return (int)(w & 0xFFFFu) - 0x8000; }

// Exponent of the running value as an FDA term (mma.py:85-91); kNone for 0 / Inf / NaN.
__device__ __forceinline__ int running_exp(float c) {
  uint32_t a = f2u(c) & 0x7FFFFFFFu;
  if (a == 0 || a >= kInf) return kNone;
  uint32_t field = a >> 23;
  if (field) return (int)field - 127;
  return ilog2_u32(a) - 149;
}

// The running value's significand at radix F, aligned to emax with truncation, signed.
__device__ __forceinline__ int64_t running_term(float c, int F, int emax) {
  uint32_t a = f2u(c) & 0x7FFFFFFFu;
  if (a == 0 || a >= kInf) return 0;
  uint32_t field = a >> 23;
  uint32_t sig = field ? ((a & 0x7FFFFFu) | 0x800000u) : a;
  int lead = ilog2_u32(sig);
  int ec = (field ? (int)field - 127 : -126) + lead - 23;
  uint64_t m = (uint64_t)(sig << (23 - lead));  // 24-bit, leading one at bit 23
  int sh = (F - 23) - (emax - ec);
  uint64_t v = sh >= 0 ? (m << sh) : (sh <= -64 ? 0ull : (m >> -sh));
  return (f2u(c) >> 31) ? -(int64_t)v : (int64_t)v;
}

// Arguments of the GDFS-FP4 GEMM kernels (tiled DP4A and tensor-core): the encoded records of both
// operands, the GDFS radices and the epilogue.
struct GemmArgs {
  const uint4 *aq, *am, *bq, *bm;
  const uint32_t *as, *bs;        // scale words (exact path)
  const int32_t *amul, *bmul;     // multipliers [ntiles * ng][rows_pad]
  const int2 *atw, *btw;          // tile words [ntiles][rows_pad]
  const int4 *atc, *btc;          // the tensor-core kernel's tile words [ntiles][rows_pad] (tile_words_kernel)
  int64_t a_rows_pad, b_rows_pad;
  int64_t M, N, ntiles;
  int F, shift0;       // shift0 = F - 2 - srad (srad = radix of the combined scale)
  int srad2;           // srad + 2: a group value is sx * 2**(es_a + es_b - srad2)
  int pexp;            // 1023 - srad2: fp64 exponent field offset of those powers of two
  int rne;
  const float *alpha_a, *alpha_b, *bias;
  Fmt of;
  int out_plain, out_dt;
  void *out;
  const int32_t *flag;   // nonzero: the fast path is not valid for these operands
  int32_t *status;       // set to 1 when a bounded wait gives up
  int wait_polls;        // poll limit of the pipeline waits (negative: default)
};

}  // namespace fp4
}  // namespace tc
