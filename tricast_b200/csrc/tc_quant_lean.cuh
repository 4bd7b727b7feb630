// Lean fused group quantize (granularity "group", float element formats, absmax / pow2 scales,
// nearest-even or directed rounding, no zero point, no stochastic rounding): one pass over x with
// LG = group_size / E lanes per group and E consecutive elements per lane.
//  * The group statistic is a float max of |x| plus a finiteness probe fma(x, 0, acc), which stays
//    +0 for finite inputs and turns NaN for any Inf or NaN. Groups with a non-finite element redo
//    the NaN-propagating integer amax over the group's lanes.
//  * The power-of-two scale 2**e comes from the amax bit pattern in integers
//    (e = floor(log2 amax) - emax_elem, +1 for pow2_ceil when the amax significand exceeds
//    max_normal's, clamped to the scale format), so x / 2**e is the exact multiply by 2**-e and
//    |x / 2**e| < 2**(emax_elem + 1) needs no clamp in the lean rounding.
//  * Elements use the lean cast (tc_lean.cuh); codes use multiply-high arithmetic (fma_code).
//  * A group the lean path does not cover (non-finite inputs or divisor, or a non-saturating overflow,
//    detected up front by rounding the largest magnitude upward) is handed whole to lean_fallback,
//    a separate routine that re-reads its elements and applies the generic definition
//    (quant_elem_d, element_code), so the common path computes none of it.
#pragma once

#include "tc_quant.cuh"

namespace tc {

struct LeanPow2 {
  uint32_t max_sig;   // 24-bit significand of the element max_normal
  int emax_elem;
  int emin, emax;     // scale format exponent range
  int bias;
  int e8m0_code;      // scale format is power-of-two: code = e + bias
};

__device__ __forceinline__ uint32_t pow2_bits(int e) {  // 2**e for -149 <= e <= 127
  return e >= -126 ? (uint32_t)(e + 127) << 23 : 1u << (e + 149);
}

// Code of a finite grid value q (sign-magnitude float format): b = bits(q * 2**(-126 - emin)) holds
// sign << 31 | magnitude << mshift, so t = b >> mshift has the magnitude in its low bits and the sign
// at bit 31 - mshift, which moves to bit sign_pos by adding sign * -(2**(31 - mshift) - 2**sign_pos).
// The shifts are multiply-highs by run-time powers of two.
struct CodeMul {
  uint32_t hi;      // 2**(32 - mshift): umulhi(b, hi) == b >> mshift
  uint32_t two;     // 2: umulhi(b, two) == b >> 31
  uint32_t neg_k;   // -(2**(31 - mshift) - 2**sign_pos) mod 2**32
  uint32_t radix;   // 16 (4-bit codes) or 256 (8-bit codes): Horner packing
};

__device__ __forceinline__ uint32_t fma_code(float q, const Lean &ln, const CodeMul &cm) {
  const uint32_t b = f2u(__fmul_rn(q, ln.code_mul));
  return __umulhi(b, cm.two) * cm.neg_k + __umulhi(b, cm.hi);
}

struct LeanArgs {
  const void *x;
  QParams p;
  Lean ln;
  LeanPow2 lp;
  CodeMul cm;
  const float *d2;
  const uint32_t *scale_noise;
  void *values;
  float *scale;
  uint8_t *codes;
  uint8_t *scodes;
  float *dequant;
};

// Where one lane's outputs go: element oi of the bases (global memory, or a warp's shared-memory
// staging slice that a bulk copy writes out afterwards).
struct LaneOut {
  void *values;
  float *dequant;
  uint8_t *codes;
  int64_t oi;
};

// The generic definition for the E elements of one lane (rare groups only): it re-reads its inputs
// (x elements i0 ..) and shares no values with the lean path, which therefore stays free of it.
template <int E>
__device__ __forceinline__ void lean_fallback(const void *x, int64_t i0, float sc, float d2, const QParams &p,
                                              const LaneOut &o) {
  const Divisor dv = make_divisor(sc, d2, p.two_level, p);
  uint32_t cw[2] = {0u, 0u};
#pragma unroll 1
  for (int j = 0; j < E; ++j) {
    const float v = load_as_float(x, p.x_dtype, i0 + j);
    const ElemOut e = quant_elem_d(v, sc, 0.0f, dv, d2, p.two_level, p, 0u);
    if (o.values) store_container(o.values, p.v_dtype, o.oi + j, e.value);
    if (o.dequant) o.dequant[o.oi + j] = e.dequant;
    if (o.codes) {
      const uint32_t c = element_code(e.value, p.ef, p.code_bits == 4 ? 4 : 8);
      if (p.code_bits == 4) cw[j >> 3] |= (c & 0xFu) << (4 * (j & 7));
      else o.codes[o.oi + j] = (uint8_t)c;
    }
  }
  if (o.codes && p.code_bits == 4)
    for (int k = 0; k < E / 8; ++k) reinterpret_cast<uint32_t *>(o.codes + (o.oi >> 1))[k] = cw[k];
}

// The work of one lane on its E elements v of group g (elements i0 .. i0 + E - 1; lane `sub` of the
// group's LG lanes, whose mask is gmask): group amax and scale, lean elements, all stores (scale and
// scale code to global memory, the element outputs to `o`). FAST:
// nearest-even rounding with saturating overflow (the MX / NVFP4 default); otherwise rounding and
// overflow rule are read at run time. CB: element code width written (0 none, 4 or 8). OUT: 0 any
// outputs (read at run time), 1 dequant only, 2 bf16 values only.
template <int E, int LG, bool POW2, bool FAST, int CB, int OUT>
__device__ __forceinline__ void lean_lane(const LeanArgs &a, const float (&v)[E], int64_t g, int64_t i0, int sub,
                                          unsigned gmask, const LaneOut &o) {
  const QParams &p = a.p;
  const bool two_level = !POW2 && p.two_level;
  const float d2 = two_level ? *a.d2 : 1.0f;
  const bool has_values = OUT == 0 ? a.values != nullptr : OUT == 2;
  const bool has_dequant = OUT == 0 ? a.dequant != nullptr : OUT == 1;
  const Lean &ln = a.ln;
  const CodeMul &cm = a.cm;
  const LeanPow2 &lp = a.lp;
  float amf = 0.0f, probe = 0.0f;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    amf = fmaxf(amf, fabsf(v[j]));
    probe = __fmaf_rn(v[j], 0.0f, probe);
  }
#pragma unroll
  for (int m = 1; m < LG; m <<= 1) {
    amf = fmaxf(amf, __shfl_xor_sync(0xFFFFFFFFu, amf, m));
    probe = __fadd_rn(probe, __shfl_xor_sync(0xFFFFFFFFu, probe, m));
  }
  const bool finite = probe == 0.0f;
  uint32_t am = f2u(amf);
  if (!finite) {  // every lane of this group is here: shuffles over the group's lanes only
    am = 0;
#pragma unroll
    for (int j = 0; j < E; ++j) am = max(am, f2u(v[j]) & 0x7FFFFFFFu);
#pragma unroll
    for (int m = 1; m < LG; m <<= 1) am = max(am, __shfl_xor_sync(gmask, am, m));
  }
  float sc, mul = 0.0f, eff = 1.0f;
  uint32_t scode = 0;
  bool lean_ok;
  if (POW2) {
    const bool nrm = am >= 0x00800000u;
    const int lead = ilog2_u32(am | 1u);
    int e = (nrm ? (int)(am >> 23) - 127 : am ? lead - 149 : -126) - lp.emax_elem;
    const uint32_t sig = nrm ? ((am & 0x7FFFFFu) | 0x800000u) : am ? am << (23 - lead) : 0x800000u;
    if (p.method == M_POW2_CEIL && sig > lp.max_sig) e += 1;
    lean_ok = finite && e <= lp.emax;
    e = max(e, lp.emin);
    sc = u2f(pow2_bits(e));
    mul = u2f(pow2_bits(-e));
    scode = (uint32_t)(e + lp.bias) & 0xFFu;
  } else {
    const uint32_t sn = a.scale_noise ? a.scale_noise[g] : 0u;
    sc = amax_scale(u2f(am), d2, two_level, p, sn);
    eff = two_level ? __fmul_rn(sc, d2) : sc;
    const uint32_t eb = f2u(eff) & 0x7FFFFFFFu;
    lean_ok = finite && eb != 0 && eb < kInf;
  }
  if (!FAST && lean_ok && !ln.sat_only) {
    // Non-saturating overflow is the generic path's: no element overflows if the largest
    // magnitude rounded upward stays within max_normal.
    const float top = POW2 ? __fmul_rn(amf, mul) : __fdiv_rn(amf, eff);
    lean_ok = lean_mag2<1, !POW2>(top, ln, TC_RUP) <= ln.maxv;
  }
  if (!lean_ok) {
    if (POW2) sc = pow2_scale(u2f(am), p);
    if (sub == 0) {
      a.scale[g] = sc;
      if (a.scodes) a.scodes[g] = (uint8_t)scale_code(sc, p.sf);
    }
    LaneOut fo = o;
    if (!has_values) fo.values = nullptr;
    if (!has_dequant) fo.dequant = nullptr;
    lean_fallback<E>(a.x, i0, sc, d2, a.p, fo);
    return;
  }
  if (a.scodes && !(POW2 && lp.e8m0_code)) scode = scale_code(sc, p.sf);
  if (sub == 0) {
    a.scale[g] = sc;
    if (a.scodes) a.scodes[g] = (uint8_t)scode;
  }
  uint32_t cw[CB == 8 ? E / 4 : E / 8 + 1];
#pragma unroll
  for (int h = 0; h < E / 8; ++h) {
    float q[8], dq[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float xq = POW2 ? __fmul_rn(v[8 * h + j], mul) : __fdiv_rn(v[8 * h + j], eff);
      float r = lean_mag2<FAST ? 0 : 1, !POW2>(xq, ln, p.rnd);
      if (FAST || ln.sat_only) r = fminf(r, ln.maxv);
      q[j] = u2f(f2u(r) | (f2u(xq) & 0x80000000u));
      float d = __fmul_rn(q[j], sc);
      if (two_level) d = __fmul_rn(d, d2);
      dq[j] = d;
    }
    const int64_t ih = o.oi + 8 * h;
    if (has_values) {
      if (OUT == 2 || p.v_dtype == TC_BF16) {
        uint4 w;  // grid values are exact in bf16: keep the high halves
        w.x = __byte_perm(f2u(q[0]), f2u(q[1]), 0x7632);
        w.y = __byte_perm(f2u(q[2]), f2u(q[3]), 0x7632);
        w.z = __byte_perm(f2u(q[4]), f2u(q[5]), 0x7632);
        w.w = __byte_perm(f2u(q[6]), f2u(q[7]), 0x7632);
        *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(o.values) + ih) = w;
      } else if (p.v_dtype == TC_F32) {
        float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(o.values) + ih);
        dst[0] = make_float4(q[0], q[1], q[2], q[3]);
        dst[1] = make_float4(q[4], q[5], q[6], q[7]);
      } else {
        uint4 w;
        w.x = __half_as_ushort(__float2half_rn(q[0])) | ((uint32_t)__half_as_ushort(__float2half_rn(q[1])) << 16);
        w.y = __half_as_ushort(__float2half_rn(q[2])) | ((uint32_t)__half_as_ushort(__float2half_rn(q[3])) << 16);
        w.z = __half_as_ushort(__float2half_rn(q[4])) | ((uint32_t)__half_as_ushort(__float2half_rn(q[5])) << 16);
        w.w = __half_as_ushort(__float2half_rn(q[6])) | ((uint32_t)__half_as_ushort(__float2half_rn(q[7])) << 16);
        *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(o.values) + ih) = w;
      }
    }
    if (has_dequant) {
      float4 *dst = reinterpret_cast<float4 *>(o.dequant + ih);
      dst[0] = make_float4(dq[0], dq[1], dq[2], dq[3]);
      dst[1] = make_float4(dq[4], dq[5], dq[6], dq[7]);
    }
    // Horner packing, last element first, so element j lands at bits CB * j of its word.
    if (CB == 4) {
      uint32_t w = 0;
#pragma unroll
      for (int j = 7; j >= 0; --j) w = w * cm.radix + fma_code(q[j], ln, cm);
      cw[h] = w;
    } else if (CB == 8) {
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int j = 3; j >= 0; --j) {
        w1 = w1 * cm.radix + fma_code(q[4 + j], ln, cm);
        w0 = w0 * cm.radix + fma_code(q[j], ln, cm);
      }
      cw[2 * h] = w0;
      cw[2 * h + 1] = w1;
    }
  }
  if (CB == 4) {
    if (E == 16) *reinterpret_cast<uint2 *>(o.codes + (o.oi >> 1)) = make_uint2(cw[0], cw[1]);
    else *reinterpret_cast<uint32_t *>(o.codes + (o.oi >> 1)) = cw[0];
  } else if (CB == 8) {
    if (E == 16) *reinterpret_cast<uint4 *>(o.codes + o.oi) = make_uint4(cw[0], cw[1], cw[2], cw[3]);
    else *reinterpret_cast<uint2 *>(o.codes + o.oi) = make_uint2(cw[0], cw[1]);
  }
}

// Decode a lane's E elements from 16-byte chunks (E/4 for fp32, E/8 for 16-bit inputs).
template <int E>
__device__ __forceinline__ void lean_decode(const uint4 (&raw)[E / 4], int x_dtype, float (&v)[E]) {
  if (x_dtype == TC_F32) {
#pragma unroll
    for (int k = 0; k < E / 4; ++k) {
      v[4 * k] = u2f(raw[k].x); v[4 * k + 1] = u2f(raw[k].y);
      v[4 * k + 2] = u2f(raw[k].z); v[4 * k + 3] = u2f(raw[k].w);
    }
  } else {
#pragma unroll
    for (int k = 0; k < E / 8; ++k) {
      const uint32_t w[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (x_dtype == TC_BF16) {
          v[8 * k + 2 * j] = u2f(w[j] << 16);
          v[8 * k + 2 * j + 1] = u2f(w[j] & 0xFFFF0000u);
        } else {
          v[8 * k + 2 * j] = __half2float(__ushort_as_half((unsigned short)(w[j] & 0xFFFF)));
          v[8 * k + 2 * j + 1] = __half2float(__ushort_as_half((unsigned short)(w[j] >> 16)));
        }
      }
    }
  }
}

// Register-staged kernel: E elements per lane, LG lanes per group (group size E * LG). Each
// iteration issues the loads of the next one first (the address is clamped to the last group, so no
// branch guards it). The kernel covers the first ngroups - ngroups % (32 / LG) groups, so every warp
// iteration is full; the host hands the few remaining groups to the four-elements-per-lane pass.
template <int E, int LG, bool POW2, bool FAST, int CB, int OUT>
__global__ void __launch_bounds__(256, 4) group_lean_kernel(const LeanArgs a) {
  constexpr int G = E * LG;
  constexpr int kGroupsPerWarp = 32 / LG;
  const QParams &p = a.p;
  const int64_t ngroups = (p.rows * p.K) / G / kGroupsPerWarp * kGroupsPerWarp;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LG;
  const unsigned gmask = LG == 32 ? 0xFFFFFFFFu : (((1u << LG) - 1u) << (lane & ~(LG - 1)));
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t step = (((int64_t)gridDim.x * blockDim.x) >> 5) * kGroupsPerWarp;
  const bool x32 = p.x_dtype == TC_F32;
  uint4 raw[E / 4];
  auto fetch = [&](int64_t gg) {
    gg = gg < ngroups ? gg : ngroups - 1;
    const int64_t off = gg * G + sub * E;
    const uint4 *src = x32 ? reinterpret_cast<const uint4 *>(static_cast<const float *>(a.x) + off)
                           : reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(a.x) + off);
#pragma unroll
    for (int k = 0; k < E / 4; ++k)
      if (x32 || k < E / 8) raw[k] = __ldcs(src + k);  // read once: evict-first (measured 33.7 -> 32.7 us on cfg1)
  };
  int64_t base = warp * kGroupsPerWarp;
  fetch(base + lane / LG);
  for (; base < ngroups; base += step) {
    const int64_t g = base + lane / LG;
    float v[E];
    lean_decode<E>(raw, p.x_dtype, v);
    fetch(g + step);  // the next iteration's loads are in flight while this one computes
    const int64_t i0 = g * G + sub * E;
    lean_lane<E, LG, POW2, FAST, CB, OUT>(a, v, g, i0, sub, gmask, LaneOut{a.values, a.dequant, a.codes, i0});
  }
}

// Launch for one code width; gi selects the group size (8, 16, 32, 64, 128): 8 elements per lane for
// groups of 8, 16 otherwise.
template <int CB>
void launch_group_lean_cb(const LeanArgs &a, int grid, int gi, bool pow2, bool fast, int out, cudaStream_t s) {
  const int key = (gi * 4 + (pow2 ? 2 : 0) + (fast ? 1 : 0)) * 3 + out;
  switch (key) {
#define TC_LEAN_CASE(LGV, GI, P2, FA, OU)                                                     \
  case (GI * 4 + (P2 ? 2 : 0) + (FA ? 1 : 0)) * 3 + OU:                                      \
    group_lean_kernel<(GI == 0 ? 8 : 16), LGV, P2, FA, CB, OU><<<grid, 256, 0, s>>>(a);  \
    break;
#define TC_LEAN_O(LGV, GI, P2, FA) TC_LEAN_CASE(LGV, GI, P2, FA, 0) TC_LEAN_CASE(LGV, GI, P2, FA, 1) TC_LEAN_CASE(LGV, GI, P2, FA, 2)
#define TC_LEAN_P(LGV, GI, P2) TC_LEAN_O(LGV, GI, P2, false) TC_LEAN_O(LGV, GI, P2, true)
#define TC_LEAN_G(LGV, GI) TC_LEAN_P(LGV, GI, false) TC_LEAN_P(LGV, GI, true)
    TC_LEAN_G(1, 0)
    TC_LEAN_G(1, 1)
    TC_LEAN_G(2, 2)
    TC_LEAN_G(4, 3)
    TC_LEAN_G(8, 4)
#undef TC_LEAN_G
#undef TC_LEAN_P
#undef TC_LEAN_O
#undef TC_LEAN_CASE
    default: break;
  }
}

void launch_group_lean_c0(const LeanArgs &a, int grid, int gi, bool pow2, bool fast, int out, cudaStream_t s);
void launch_group_lean_c4(const LeanArgs &a, int grid, int gi, bool pow2, bool fast, int out, cudaStream_t s);
void launch_group_lean_c8(const LeanArgs &a, int grid, int gi, bool pow2, bool fast, int out, cudaStream_t s);


}  // namespace tc
