// Cast and quantize kernels (TriCast round_to_format / quantize, src/tricast/reference/cast.py and
// src/tricast/reference/quantize.py), and the host dispatch of tc_cast / tc_quantize.
//
// Quantize runs one of these pipelines:
//  * lean group pass (tc_quant_lean.cuh) — granularity "group" with a float element format, absmax or
//    power-of-two scale, nearest-even or directed rounding, no zero point: one pass over x with 16
//    elements per lane (8 for groups of 8), the next iteration's loads in flight while the current
//    one computes; the last few groups take the four-elements-per-lane pass below;
//  * fused group pass — any other group spec with group_size in {4,...,128} dividing K: each group is
//    owned by group_size/4 adjacent lanes that load 4 elements each with one vector load, reduce the
//    domain statistic with warp shuffles, compute the scale, and write values / scale / codes /
//    dequant in the same pass, so x is read from HBM once;
//  * row pass, tensor pass (statistic kernel + element kernel) and the general pass — any
//    granularity: (A) per-domain partial statistics, (B) one warp per domain combines partials and
//    derives scale and zero point, (C) element rounding.
// Two-level specs first reduce the tensor amax and derive the global decode scale d2 on the device.
// The direct cast and the tensor pass use the lean cast (tc_lean.cuh) where the format allows.
#include <algorithm>

#include "tc_quant.cuh"
#include "tc_quant_lean.cuh"

namespace tc {

// ------------------------------------------------------------------ cast kernel
__global__ void __launch_bounds__(256) cast_kernel(const float *__restrict__ x, float *__restrict__ y,
                                                   const uint32_t *__restrict__ noise, int64_t n, Fmt f, int rnd,
                                                   int saturate, int sr_bits, int vec) {
  int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    int64_t n4 = n >> 2;
    for (int64_t i = tid; i < n4; i += stride) {
      float4 v = reinterpret_cast<const float4 *>(x)[i];
      uint4 r = noise ? reinterpret_cast<const uint4 *>(noise)[i] : make_uint4(0, 0, 0, 0);
      float4 o;
      o.x = cast_to(v.x, f, rnd, saturate, r.x, sr_bits);
      o.y = cast_to(v.y, f, rnd, saturate, r.y, sr_bits);
      o.z = cast_to(v.z, f, rnd, saturate, r.z, sr_bits);
      o.w = cast_to(v.w, f, rnd, saturate, r.w, sr_bits);
      reinterpret_cast<float4 *>(y)[i] = o;
    }
    for (int64_t i = (n4 << 2) + tid; i < n; i += stride)
      y[i] = cast_to(x[i], f, rnd, saturate, noise ? noise[i] : 0u, sr_bits);
  } else {
    for (int64_t i = tid; i < n; i += stride) y[i] = cast_to(x[i], f, rnd, saturate, noise ? noise[i] : 0u, sr_bits);
  }
}

// Lean cast of one value of any class: NaN passes through, Inf and huge magnitudes overflow.
template <int RND>
__device__ __forceinline__ float lean_cast(float v, const Lean &l) {
  const uint32_t u = f2u(v);
  const uint32_t sign = u & 0x80000000u;
  const float r = lean_overflow(lean_mag<RND, true>(v, l), sign, l);
  return (u & 0x7FFFFFFFu) > kInf ? v : u2f(f2u(r) | sign);
}

// round_to_format for the lean-eligible formats and roundings, 8 elements per thread.
template <int RND>
__global__ void __launch_bounds__(256) cast_lean_kernel(const float *__restrict__ x, float *__restrict__ y, int64_t n,
                                                        Lean l) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n8 = n >> 3;
  for (int64_t i = tid; i < n8; i += stride) {
    const float4 *src = reinterpret_cast<const float4 *>(x) + 2 * i;
    float4 a = src[0], b = src[1];
    a.x = lean_cast<RND>(a.x, l); a.y = lean_cast<RND>(a.y, l); a.z = lean_cast<RND>(a.z, l); a.w = lean_cast<RND>(a.w, l);
    b.x = lean_cast<RND>(b.x, l); b.y = lean_cast<RND>(b.y, l); b.z = lean_cast<RND>(b.z, l); b.w = lean_cast<RND>(b.w, l);
    float4 *dst = reinterpret_cast<float4 *>(y) + 2 * i;
    dst[0] = a;
    dst[1] = b;
  }
  for (int64_t i = (n8 << 3) + tid; i < n; i += stride) y[i] = lean_cast<RND>(x[i], l);
}

static int grid_for(int64_t work, int threads, int per_sm = 8) {
  int64_t blocks = (work + threads - 1) / threads;
  int64_t cap = (int64_t)sm_count() * per_sm;
  if (blocks > cap) blocks = cap;
  return (int)(blocks < 1 ? 1 : blocks);
}

static int launch_status(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return TC_CUDA_ERROR;
  }
  return TC_OK;
}

// ------------------------------------------------------------------ general pass (A): statistics
// Partial statistic of one (domain, part): amax bits (NaN-propagating max of |x| bits) or
// (min key, max key, nan flag).
struct Stat {
  uint32_t amax, lo, hi, nan;
};

__device__ __forceinline__ void stat_init(Stat &s) {
  s.amax = 0;
  s.lo = 0xFFFFFFFFu;
  s.hi = 0;
  s.nan = 0;
}
__device__ __forceinline__ void stat_add(Stat &s, float v) {
  uint32_t a = f2u(v) & 0x7FFFFFFFu;
  s.amax = max(s.amax, a);
  if (a > kInf) {
    s.nan = 1;
  } else {
    uint32_t k = fkey(v);
    s.lo = min(s.lo, k);
    s.hi = max(s.hi, k);
  }
}
__device__ __forceinline__ void stat_merge(Stat &s, const Stat &o) {
  s.amax = max(s.amax, o.amax);
  s.lo = min(s.lo, o.lo);
  s.hi = max(s.hi, o.hi);
  s.nan |= o.nan;
}
__device__ __forceinline__ Stat stat_shfl(const Stat &s, int lane_mask) {
  Stat o;
  o.amax = __shfl_xor_sync(0xFFFFFFFFu, s.amax, lane_mask);
  o.lo = __shfl_xor_sync(0xFFFFFFFFu, s.lo, lane_mask);
  o.hi = __shfl_xor_sync(0xFFFFFFFFu, s.hi, lane_mask);
  o.nan = __shfl_xor_sync(0xFFFFFFFFu, s.nan, lane_mask);
  return o;
}

// Domain d as a rectangle of x; element e of it in row-major order.
__device__ __forceinline__ void domain_rect(const QParams &p, int64_t d, int64_t &r0, int64_t &c0, int64_t &h,
                                            int64_t &w) {
  int64_t dri = d / p.nc, dci = d % p.nc;
  r0 = dri * p.dr;
  c0 = dci * p.dc;
  h = min(p.dr, p.rows - r0);
  w = min(p.dc, p.K - c0);
}

__global__ void __launch_bounds__(256) stats_kernel(const void *__restrict__ x, QParams p, int64_t nd, int parts,
                                                    int64_t chunk, Stat *__restrict__ partial) {
  int64_t d = blockIdx.x / parts;
  int part = blockIdx.x % parts;
  if (d >= nd) return;
  int64_t r0, c0, h, w;
  domain_rect(p, d, r0, c0, h, w);
  int64_t n = h * w;
  int64_t beg = part * chunk, end = min(n, beg + chunk);
  Stat s;
  stat_init(s);
  for (int64_t e = beg + threadIdx.x; e < end; e += blockDim.x) {
    int64_t r = r0 + e / w, c = c0 + e % w;
    stat_add(s, load_as_float(x, p.x_dtype, r * p.K + c));
  }
  for (int m = 16; m; m >>= 1) stat_merge(s, stat_shfl(s, m));
  __shared__ Stat warp_stat[8];
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) warp_stat[warp] = s;
  __syncthreads();
  if (warp == 0) {
    if (lane < (int)(blockDim.x >> 5)) s = warp_stat[lane];
    else stat_init(s);
    for (int m = 16; m; m >>= 1) stat_merge(s, stat_shfl(s, m));
    if (lane == 0) partial[d * parts + part] = s;
  }
}

// ------------------------------------------------------------------ general pass (B): scales
// One warp per domain combines its partials and derives scale / zero point (and, for the
// tensor-amax pre-pass of two-level specs, the global scale d2).
__global__ void scale_kernel(QParams p, int64_t nd, int parts, const Stat *__restrict__ partial,
                             const float *__restrict__ amax_override, float *__restrict__ d2_slot,
                             const uint32_t *__restrict__ scale_noise, float *__restrict__ scale,
                             float *__restrict__ zero, uint8_t *__restrict__ scodes, int global_only) {
  int lane = threadIdx.x & 31;
  int64_t d = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (d >= nd) return;
  Stat s;
  stat_init(s);
  for (int i = lane; i < parts; i += 32) stat_merge(s, partial[d * parts + i]);
  for (int m = 16; m; m >>= 1) stat_merge(s, stat_shfl(s, m));
  if (lane) return;
  float amax = amax_override ? *amax_override : u2f(s.amax);
  if (global_only) {
    *d2_slot = global_scale(amax, p.prod_max_d);
    return;
  }
  uint32_t noise = scale_noise ? scale_noise[d] : 0u;
  float sc, z = 0.0f;
  if (p.zp) {
    float lo = s.nan ? u2f(kQNaN) : unkey(s.lo);
    float hi = s.nan ? u2f(kQNaN) : unkey(s.hi);
    zp_scale(lo, hi, p, noise, sc, z);
    zero[d] = z;
  } else if (p.two_level || p.method == M_ABSMAX) {
    sc = amax_scale(amax, p.two_level ? *d2_slot : 1.0f, p.two_level, p, noise);
  } else {
    sc = pow2_scale(amax, p);
  }
  scale[d] = sc;
  if (scodes) scodes[d] = (uint8_t)scale_code(sc, p.sf);
}

// ------------------------------------------------------------------ general pass (C): elements
__device__ __forceinline__ void store_codes(uint8_t *codes, int bits, int64_t i, uint32_t c, uint32_t c_next,
                                            bool pair) {
  if (bits == 8) {
    codes[i] = (uint8_t)c;
  } else if (pair) {
    codes[i >> 1] = (uint8_t)((c & 0xF) | ((c_next & 0xF) << 4));
  }
}

__global__ void __launch_bounds__(256) element_kernel(const void *__restrict__ x, QParams p,
                                                      const float *__restrict__ scale, const float *__restrict__ zero,
                                                      const float *__restrict__ d2p, const uint32_t *__restrict__ noise,
                                                      void *__restrict__ values, uint8_t *__restrict__ codes,
                                                      float *__restrict__ dequant) {
  int64_t n = p.rows * p.K;
  int64_t npairs = (n + 1) >> 1;
  float d2 = p.two_level ? *d2p : 1.0f;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t pi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; pi < npairs; pi += stride) {
    uint32_t cc[2] = {0, 0};
    for (int j = 0; j < 2; ++j) {
      int64_t i = 2 * pi + j;
      if (i >= n) break;
      int64_t r = i / p.K, c = i % p.K;
      float s = 1.0f, z = 0.0f;
      if (p.has_scale) {
        int64_t d = (r / p.dr) * p.nc + c / p.dc;
        s = scale[d];
        if (p.zp) z = zero[d];
      }
      ElemOut o = quant_elem(load_as_float(x, p.x_dtype, i), s, z, d2, p.two_level, p, noise ? noise[i] : 0u);
      if (values) store_container(values, p.v_dtype, i, o.value);
      if (dequant) dequant[i] = o.dequant;
      if (codes) cc[j] = element_code(o.value, p.ef, p.code_bits == 4 ? 4 : 8);
    }
    if (codes) {
      if (p.code_bits == 8) {
        codes[2 * pi] = (uint8_t)cc[0];
        if (2 * pi + 1 < n) codes[2 * pi + 1] = (uint8_t)cc[1];
      } else {
        codes[pi] = (uint8_t)((cc[0] & 0xF) | ((cc[1] & 0xF) << 4));
      }
    }
  }
}

// ------------------------------------------------------------------ fused group pass
// L = group_size / 4 lanes own one group; each lane handles 4 consecutive elements.
// MSE specs (rt.n > 0) try every candidate scale on the group before the inactive lanes of the
// last iteration leave, so the error sums' shuffles see the full warp.
template <int L>
__global__ void __launch_bounds__(256) group_kernel(const void *__restrict__ x, QParams p,
                                                    const float *__restrict__ d2p, const uint32_t *__restrict__ noise,
                                                    const uint32_t *__restrict__ scale_noise, void *__restrict__ values,
                                                    float *__restrict__ scale, float *__restrict__ zero,
                                                    uint8_t *__restrict__ codes, uint8_t *__restrict__ scodes,
                                                    float *__restrict__ dequant, const Ratios rt) {
  const int64_t n = p.rows * p.K;
  const int64_t ngroups = n / (4 * L);
  const float d2 = p.two_level ? *d2p : 1.0f;
  const int lane = threadIdx.x & 31;
  const int sub = lane % L;                    // position inside the group
  constexpr int kGroupsPerWarp = 32 / L;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  // The trip count depends only on the warp, so every shuffle below sees the full warp.
  for (int64_t base = warp * kGroupsPerWarp; base < ngroups; base += nwarps * kGroupsPerWarp) {
    const int64_t g = base + lane / L;
    const bool active = g < ngroups;
    const int64_t i0 = g * (4 * L) + sub * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (active) {
      if (p.x_dtype == TC_F32) {
        float4 t = *reinterpret_cast<const float4 *>(static_cast<const float *>(x) + i0);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      } else {
        uint2 t = *reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(x) + i0);
        uint16_t h[4] = {(uint16_t)(t.x & 0xFFFF), (uint16_t)(t.x >> 16), (uint16_t)(t.y & 0xFFFF),
                         (uint16_t)(t.y >> 16)};
        for (int j = 0; j < 4; ++j)
          v[j] = p.x_dtype == TC_BF16 ? __bfloat162float(__ushort_as_bfloat16(h[j]))
                                      : __half2float(__ushort_as_half(h[j]));
      }
    }
    Stat s;
    stat_init(s);
    if (active)
      for (int j = 0; j < 4; ++j) stat_add(s, v[j]);
    for (int m = 1; m < L; m <<= 1) stat_merge(s, stat_shfl(s, m));
    const uint32_t sn = (active && scale_noise) ? scale_noise[g] : 0u;
    uint32_t nn[4] = {0u, 0u, 0u, 0u};
    if (noise && active)
      for (int j = 0; j < 4; ++j) nn[j] = noise[i0 + j];
    float sc = 0.0f, z = 0.0f;
    if (rt.n > 0) {
      // Candidates in order; a later one wins only with a strictly smaller error (ties keep the first).
      double best = 0.0;
      for (int c = 0; c < rt.n; ++c) {
        const float cs = amax_scale(__fmul_rn(u2f(s.amax), rt.r[c]), d2, p.two_level, p, sn);
        const Divisor cdv = make_divisor(cs, d2, p.two_level, p);
        double e = 0.0;
        if (active)
          for (int j = 0; j < 4; ++j) e = __dadd_rn(e, cand_sq_error(v[j], cs, cdv, d2, p.two_level, p, nn[j]));
        for (int m = 1; m < L; m <<= 1) e = __dadd_rn(e, __shfl_xor_sync(0xFFFFFFFFu, e, m));
        if (c == 0 || e < best) {
          best = e;
          sc = cs;
        }
      }
    }
    if (!active) continue;  // only in the last iteration; no shuffle follows
    if (rt.n > 0) {
    } else if (p.zp) {
      float lo = s.nan ? u2f(kQNaN) : unkey(s.lo);
      float hi = s.nan ? u2f(kQNaN) : unkey(s.hi);
      zp_scale(lo, hi, p, sn, sc, z);
    } else if (p.two_level || p.method == M_ABSMAX) {
      sc = amax_scale(u2f(s.amax), d2, p.two_level, p, sn);
    } else {
      sc = pow2_scale(u2f(s.amax), p);
    }
    if (sub == 0) {
      scale[g] = sc;
      if (p.zp) zero[g] = z;
      if (scodes) scodes[g] = (uint8_t)scale_code(sc, p.sf);
    }
    float q[4], dq[4];
    uint32_t cd[4];
    const Divisor dv = make_divisor(sc, d2, p.two_level, p);
    for (int j = 0; j < 4; ++j) {
      ElemOut o = quant_elem_d(v[j], sc, z, dv, d2, p.two_level, p, nn[j]);
      q[j] = o.value;
      dq[j] = o.dequant;
      cd[j] = codes ? element_code(o.value, p.ef, p.code_bits == 4 ? 4 : 8) : 0u;
    }
    if (!values) {
    } else if (p.v_dtype == TC_F32) {
      *reinterpret_cast<float4 *>(static_cast<float *>(values) + i0) = make_float4(q[0], q[1], q[2], q[3]);
    } else {
      uint16_t h[4];
      for (int j = 0; j < 4; ++j) {
        uint32_t u = f2u(q[j]);
        if (p.v_dtype == TC_BF16) h[j] = ((u & 0x7FFFFFFFu) > kInf) ? (uint16_t)0x7FC0 : (uint16_t)(u >> 16);
        else h[j] = (q[j] != q[j]) ? (uint16_t)0x7E00 : __half_as_ushort(__float2half_rn(q[j]));
      }
      *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(values) + i0) =
          make_uint2((uint32_t)h[0] | ((uint32_t)h[1] << 16), (uint32_t)h[2] | ((uint32_t)h[3] << 16));
    }
    if (dequant) *reinterpret_cast<float4 *>(dequant + i0) = make_float4(dq[0], dq[1], dq[2], dq[3]);
    if (codes) {
      if (p.code_bits == 4) {
        *reinterpret_cast<uint16_t *>(codes + (i0 >> 1)) =
            (uint16_t)((cd[0] & 0xF) | ((cd[1] & 0xF) << 4) | ((cd[2] & 0xF) << 8) | ((cd[3] & 0xF) << 12));
      } else {
        *reinterpret_cast<uint32_t *>(codes + i0) = (cd[0] & 0xFF) | ((cd[1] & 0xFF) << 8) |
                                                    ((cd[2] & 0xFF) << 16) | ((cd[3] & 0xFF) << 24);
      }
    }
  }
}

// ------------------------------------------------------------------ tensor statistics
// One Stat for the whole tensor, reduced with atomics into a workspace slot that the host cleared
// to the identity (amax 0, lo 0xFFFFFFFF, hi 0, nan 0). 16-byte loads when aligned.
template <bool AMAX_ONLY>
__device__ __forceinline__ void tstat_add(Stat &s, float v) {
  if (AMAX_ONLY) s.amax = max(s.amax, f2u(v) & 0x7FFFFFFFu);  // NaN bits sort above Inf: NaN-propagating
  else stat_add(s, v);
}

// AMAX_ONLY: only the NaN-propagating amax (two-level specs and absmax / pow2 tensor scales); the
// full statistic adds the signed range for zero points.
// With AMAX_ONLY and amax_bits given, the amax goes to *amax_bits instead of out->amax.
template <bool AMAX_ONLY>
__global__ void __launch_bounds__(256) tensor_stats_kernel(const void *__restrict__ x, int dt, int64_t n, int vec,
                                                           Stat *__restrict__ out, uint32_t *amax_bits = nullptr) {
  Stat s;
  stat_init(s);
  int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t done = 0;
  if (vec && dt == TC_F32) {
    int64_t n4 = n >> 2;
    for (int64_t i = tid; i < n4; i += stride) {
      float4 v = reinterpret_cast<const float4 *>(x)[i];
      tstat_add<AMAX_ONLY>(s, v.x); tstat_add<AMAX_ONLY>(s, v.y);
      tstat_add<AMAX_ONLY>(s, v.z); tstat_add<AMAX_ONLY>(s, v.w);
    }
    done = n4 << 2;
  } else if (vec) {
    const int64_t n8 = n >> 3;
    auto add8 = [&](const uint4 &u) {
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint16_t lo = (uint16_t)(w[j] & 0xFFFF), hi = (uint16_t)(w[j] >> 16);
        if (dt == TC_BF16) {
          tstat_add<AMAX_ONLY>(s, u2f((uint32_t)lo << 16));
          tstat_add<AMAX_ONLY>(s, u2f((uint32_t)hi << 16));
        } else {
          tstat_add<AMAX_ONLY>(s, __half2float(__ushort_as_half(lo)));
          tstat_add<AMAX_ONLY>(s, __half2float(__ushort_as_half(hi)));
        }
      }
    };
    // Four independent 16-byte loads in flight per thread, then the grid-stride remainder.
    const uint4 *x8 = reinterpret_cast<const uint4 *>(x);
    int64_t i = tid;
    for (; i + 3 * stride < n8; i += 4 * stride) {
      const uint4 u0 = x8[i], u1 = x8[i + stride], u2 = x8[i + 2 * stride], u3 = x8[i + 3 * stride];
      add8(u0);
      add8(u1);
      add8(u2);
      add8(u3);
    }
    for (; i < n8; i += stride) add8(x8[i]);
    done = n8 << 3;
  }
  for (int64_t i = done + tid; i < n; i += stride) tstat_add<AMAX_ONLY>(s, load_as_float(x, dt, i));
  if (AMAX_ONLY) {
    for (int m = 16; m; m >>= 1) s.amax = max(s.amax, __shfl_xor_sync(0xFFFFFFFFu, s.amax, m));
    if ((threadIdx.x & 31) == 0) atomicMax(amax_bits ? amax_bits : &out->amax, s.amax);
  } else {
    for (int m = 16; m; m >>= 1) stat_merge(s, stat_shfl(s, m));
    if ((threadIdx.x & 31) == 0) {
      atomicMax(&out->amax, s.amax);
      atomicMin(&out->lo, s.lo);
      atomicMax(&out->hi, s.hi);
      if (s.nan) atomicExch(&out->nan, 1u);
    }
  }
}

// ------------------------------------------------------------------ row-resident pass
// Granularity "row": one block per row (grid-stride over rows). Pass 1 reduces the row's statistic,
// thread 0 derives the scale, pass 2 re-reads the row (now in L1/L2) and writes every output.
__global__ void __launch_bounds__(256) row_kernel(const void *__restrict__ x, QParams p,
                                                  const float *__restrict__ d2p, const uint32_t *__restrict__ noise,
                                                  const uint32_t *__restrict__ scale_noise, void *__restrict__ values,
                                                  float *__restrict__ scale, float *__restrict__ zero,
                                                  uint8_t *__restrict__ codes, uint8_t *__restrict__ scodes,
                                                  float *__restrict__ dequant) {
  __shared__ Stat warp_stat[8];
  __shared__ float sh_scale, sh_zero;
  const float d2 = p.two_level ? *d2p : 1.0f;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
    const int64_t base = r * p.K;
    Stat s;
    stat_init(s);
    for (int64_t c = threadIdx.x; c < p.K; c += blockDim.x) stat_add(s, load_as_float(x, p.x_dtype, base + c));
    for (int m = 16; m; m >>= 1) stat_merge(s, stat_shfl(s, m));
    if (lane == 0) warp_stat[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w) stat_merge(s, warp_stat[w]);
      uint32_t sn = scale_noise ? scale_noise[r] : 0u;
      float sc, z = 0.0f;
      if (p.zp) {
        float lo = s.nan ? u2f(kQNaN) : unkey(s.lo);
        float hi = s.nan ? u2f(kQNaN) : unkey(s.hi);
        zp_scale(lo, hi, p, sn, sc, z);
        zero[r] = z;
      } else if (p.two_level || p.method == M_ABSMAX) {
        sc = amax_scale(u2f(s.amax), d2, p.two_level, p, sn);
      } else {
        sc = pow2_scale(u2f(s.amax), p);
      }
      scale[r] = sc;
      if (scodes) scodes[r] = (uint8_t)scale_code(sc, p.sf);
      sh_scale = sc;
      sh_zero = z;
    }
    __syncthreads();
    const float sc = sh_scale, z = sh_zero;
    const Divisor dv = make_divisor(sc, d2, p.two_level, p);
    // Pairs of elements so 4-bit codes pack into whole bytes (K even is required for codes).
    for (int64_t c = 2 * threadIdx.x; c < p.K; c += 2 * blockDim.x) {
      uint32_t cc[2] = {0, 0};
      for (int j = 0; j < 2 && c + j < p.K; ++j) {
        int64_t i = base + c + j;
        ElemOut o = quant_elem_d(load_as_float(x, p.x_dtype, i), sc, z, dv, d2, p.two_level, p,
                                 noise ? noise[i] : 0u);
        if (values) store_container(values, p.v_dtype, i, o.value);
        if (dequant) dequant[i] = o.dequant;
        if (codes) cc[j] = element_code(o.value, p.ef, p.code_bits == 4 ? 4 : 8);
      }
      if (codes) {
        if (p.code_bits == 8) {
          codes[base + c] = (uint8_t)cc[0];
          if (c + 1 < p.K) codes[base + c + 1] = (uint8_t)cc[1];
        } else {
          codes[(base + c) >> 1] = (uint8_t)((cc[0] & 0xF) | ((cc[1] & 0xF) << 4));
        }
      }
    }
    __syncthreads();  // warp_stat / sh_scale are reused by the next row
  }
}

// One thread: the scale (or d2) of a single-domain spec from the reduced tensor statistic.
__global__ void tensor_scale_kernel(QParams p, const Stat *__restrict__ st, const float *__restrict__ amax_override,
                                    float *__restrict__ d2_slot, const uint32_t *__restrict__ scale_noise,
                                    float *__restrict__ scale, float *__restrict__ zero, uint8_t *__restrict__ scodes,
                                    int global_only) {
  Stat s = *st;
  float amax = amax_override ? *amax_override : u2f(s.amax);
  if (global_only) {
    *d2_slot = global_scale(amax, p.prod_max_d);
    return;
  }
  uint32_t noise = scale_noise ? scale_noise[0] : 0u;
  float sc, z = 0.0f;
  if (p.zp) {
    float lo = s.nan ? u2f(kQNaN) : unkey(s.lo);
    float hi = s.nan ? u2f(kQNaN) : unkey(s.hi);
    zp_scale(lo, hi, p, noise, sc, z);
    zero[0] = z;
  } else if (p.two_level || p.method == M_ABSMAX) {
    sc = amax_scale(amax, p.two_level ? *d2_slot : 1.0f, p.two_level, p, noise);
  } else {
    sc = pow2_scale(amax, p);
  }
  scale[0] = sc;
  if (scodes) scodes[0] = (uint8_t)scale_code(sc, p.sf);
}

// Elements of a single-domain (tensor) spec, or of a direct cast: 4 consecutive elements per thread.
// RND >= 0 selects the lean cast for that rounding (float formats, no zero point, no noise).
template <int RND>
__global__ void __launch_bounds__(256) flat_kernel(const void *__restrict__ x, QParams p, Lean ln,
                                                   const float *__restrict__ scale, const float *__restrict__ zero,
                                                   const float *__restrict__ d2p, const uint32_t *__restrict__ noise,
                                                   void *__restrict__ values, uint8_t *__restrict__ codes,
                                                   float *__restrict__ dequant) {
  const int64_t n = p.rows * p.K;
  const float d2 = p.two_level ? *d2p : 1.0f;
  const float sc = p.has_scale ? scale[0] : 1.0f;
  const float z = p.zp ? zero[0] : 0.0f;
  const Divisor dv = make_divisor(sc, d2, p.two_level, p);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q * 4 < n; q += stride) {
    const int64_t i0 = q * 4;
    float v[4];
    const bool full = i0 + 4 <= n;
    if (full && p.x_dtype == TC_F32 && (((uintptr_t)x & 15) == 0)) {
      float4 t = reinterpret_cast<const float4 *>(x)[q];
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
      for (int j = 0; j < 4; ++j) v[j] = i0 + j < n ? load_as_float(x, p.x_dtype, i0 + j) : 0.0f;
    }
    float o[4], dq[4];
    uint32_t cd[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (RND >= 0) {
        float xq = v[j];
        if (p.has_scale) xq = dv.by_inv ? __fmul_rn(xq, dv.inv) : __fdiv_rn(xq, dv.eff);
        const float val = lean_cast<RND < 0 ? 0 : RND>(xq, ln);
        float d = val;
        if (p.has_scale) d = __fmul_rn(d, sc);
        if (p.two_level) d = __fmul_rn(d, d2);
        o[j] = val;
        dq[j] = d;
        if (codes) {
          const float mag = fabsf(val);
          cd[j] = mag <= ln.maxv ? lean_code(mag, ln) | ((f2u(val) >> 31) << ln.sign_pos)
                                 : element_code(val, p.ef, p.code_bits == 4 ? 4 : 8);
        }
      } else {
        ElemOut e = quant_elem_d(v[j], sc, z, dv, d2, p.two_level, p, noise && i0 + j < n ? noise[i0 + j] : 0u);
        o[j] = e.value;
        dq[j] = e.dequant;
        if (codes) cd[j] = element_code(e.value, p.ef, p.code_bits == 4 ? 4 : 8);
      }
    }
    for (int j = 0; j < 4 && i0 + j < n; ++j) {
      if (values) store_container(values, p.v_dtype, i0 + j, o[j]);
      if (dequant) dequant[i0 + j] = dq[j];
      if (codes && p.code_bits == 8) codes[i0 + j] = (uint8_t)cd[j];
    }
    if (codes && p.code_bits == 4) {
      codes[i0 >> 1] = (uint8_t)((cd[0] & 0xF) | ((cd[1] & 0xF) << 4));
      if (i0 + 2 < n) codes[(i0 >> 1) + 1] = (uint8_t)((cd[2] & 0xF) | ((cd[3] & 0xF) << 4));
    }
  }
}

static void launch_flat(int grid, cudaStream_t s, const void *x, const QParams &p, const Lean &ln, int lean_rnd,
                        const float *scale, const float *zero, const float *d2, const uint32_t *noise, void *values,
                        uint8_t *codes, float *dequant) {
  switch (lean_rnd) {
    case TC_RNE: flat_kernel<TC_RNE><<<grid, 256, 0, s>>>(x, p, ln, scale, zero, d2, noise, values, codes, dequant); break;
    case TC_RTZ: flat_kernel<TC_RTZ><<<grid, 256, 0, s>>>(x, p, ln, scale, zero, d2, noise, values, codes, dequant); break;
    case TC_RUP: flat_kernel<TC_RUP><<<grid, 256, 0, s>>>(x, p, ln, scale, zero, d2, noise, values, codes, dequant); break;
    case TC_RDN: flat_kernel<TC_RDN><<<grid, 256, 0, s>>>(x, p, ln, scale, zero, d2, noise, values, codes, dequant); break;
    default: flat_kernel<-1><<<grid, 256, 0, s>>>(x, p, ln, scale, zero, d2, noise, values, codes, dequant); break;
  }
}

// ------------------------------------------------------------------ MSE and percentile scales
// Sum over a 256-thread block in a fixed order: butterflies within each warp, then the eight warp
// sums in index order by thread 0 (valid in thread 0 only).
__device__ __forceinline__ double block_sum_fixed(double v, double *warp_sums) {
  for (int m = 16; m; m >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, m));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) warp_sums[warp] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = __dadd_rn(t, warp_sums[w]);
  return t;
}

// Per-domain amax (NaN-propagating) from the statistic partials, one warp per domain.
__global__ void domain_amax_kernel(int64_t nd, int parts, const Stat *__restrict__ partial, float *__restrict__ amax) {
  const int lane = threadIdx.x & 31;
  const int64_t d = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (d >= nd) return;
  uint32_t a = 0;
  for (int i = lane; i < parts; i += 32) a = max(a, partial[d * parts + i].amax);
  for (int m = 16; m; m >>= 1) a = max(a, __shfl_xor_sync(0xFFFFFFFFu, a, m));
  if (lane == 0) amax[d] = u2f(a);
}

// MSE search, pass 1 (src/tricast/reference/quantize.py:286-301): one block per (domain, part); for
// every candidate ratio r the scale absmax_scale(RN(amax * r)) and the part's sum of squared errors
// of the elements quantized and restored with it (fp64, element noise reused for every candidate).
__global__ void __launch_bounds__(256) mse_partial_kernel(const void *__restrict__ x, QParams p, int64_t nd, int parts,
                                                          int64_t chunk, const float *__restrict__ amax,
                                                          const float *__restrict__ d2p,
                                                          const uint32_t *__restrict__ noise,
                                                          const uint32_t *__restrict__ scale_noise, const Ratios rt,
                                                          double *__restrict__ err) {
  __shared__ double warp_sums[8];
  const int64_t d = blockIdx.x / parts;
  const int part = blockIdx.x % parts;
  if (d >= nd) return;
  int64_t r0, c0, h, w;
  domain_rect(p, d, r0, c0, h, w);
  const int64_t n = h * w;
  const int64_t beg = part * chunk, end = min(n, beg + chunk);
  const float d2 = p.two_level ? *d2p : 1.0f;
  const uint32_t sn = scale_noise ? scale_noise[d] : 0u;
  for (int c = 0; c < rt.n; ++c) {
    const float cs = amax_scale(__fmul_rn(amax[d], rt.r[c]), d2, p.two_level, p, sn);
    const Divisor dv = make_divisor(cs, d2, p.two_level, p);
    double e = 0.0;
    for (int64_t i = beg + threadIdx.x; i < end; i += blockDim.x) {
      const int64_t idx = (r0 + i / w) * p.K + c0 + i % w;
      e = __dadd_rn(e, cand_sq_error(load_as_float(x, p.x_dtype, idx), cs, dv, d2, p.two_level, p,
                                     noise ? noise[idx] : 0u));
    }
    const double t = block_sum_fixed(e, warp_sums);
    if (threadIdx.x == 0) err[(d * parts + part) * rt.n + c] = t;
  }
}

// MSE search, pass 2: per domain, each candidate's error summed over the parts in order; a later
// candidate replaces the best only with a strictly smaller error (ties keep the first).
__global__ void mse_select_kernel(QParams p, int64_t nd, int parts, const Ratios rt, const float *__restrict__ amax,
                                  const float *__restrict__ d2p, const uint32_t *__restrict__ scale_noise,
                                  const double *__restrict__ err, float *__restrict__ scale,
                                  uint8_t *__restrict__ scodes) {
  const int64_t d = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= nd) return;
  const float d2 = p.two_level ? *d2p : 1.0f;
  const uint32_t sn = scale_noise ? scale_noise[d] : 0u;
  double best = 0.0;
  int pick = 0;
  for (int c = 0; c < rt.n; ++c) {
    double e = 0.0;
    for (int part = 0; part < parts; ++part) e = __dadd_rn(e, err[(d * parts + part) * rt.n + c]);
    if (c == 0 || e < best) {
      best = e;
      pick = c;
    }
  }
  const float sc = amax_scale(__fmul_rn(amax[d], rt.r[pick]), d2, p.two_level, p, sn);
  scale[d] = sc;
  if (scodes) scodes[d] = (uint8_t)scale_code(sc, p.sf);
}

// The order statistic of rank r (0-based, ascending) among the |x| bit patterns of a domain: radix
// select over four 8-bit digits, most significant first (non-negative floats order like their bits).
__device__ uint32_t domain_select(const void *x, const QParams &p, int64_t r0, int64_t c0, int64_t w, int64_t n,
                                  int64_t r, unsigned *hist, uint32_t *s_prefix, long long *s_rank) {
  uint32_t prefix = 0, mask = 0;
  long long rr = r;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t key = f2u(load_as_float(x, p.x_dtype, (r0 + i / w) * p.K + c0 + i % w)) & 0x7FFFFFFFu;
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFFu], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      long long cum = 0;
      for (int b = 0; b < 256; ++b) {
        if (cum + hist[b] > rr) {
          *s_prefix = prefix | ((uint32_t)b << shift);
          *s_rank = rr - cum;
          break;
        }
        cum += hist[b];
      }
    }
    __syncthreads();
    prefix = *s_prefix;
    rr = *s_rank;
    mask |= 0xFFu << shift;
    __syncthreads();
  }
  return prefix;
}

// Percentile scale (src/tricast/reference/quantize.py:233-241, 282-283): per domain the linear
// quantile of |x| at rank (n - 1) * percentile / 100 between the two neighbouring order statistics
// (torch.lerp's two-sided form in fp64, then one rounding to fp32), NaN if the domain holds a NaN;
// the scale is the absmax scale of that value. One block per domain.
__global__ void __launch_bounds__(256) percentile_kernel(const void *__restrict__ x, QParams p, int64_t nd, double pct,
                                                         const float *__restrict__ d2p,
                                                         const uint32_t *__restrict__ scale_noise,
                                                         float *__restrict__ scale, uint8_t *__restrict__ scodes) {
  __shared__ unsigned hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ long long s_rank;
  for (int64_t d = blockIdx.x; d < nd; d += gridDim.x) {
    int64_t r0, c0, h, w;
    domain_rect(p, d, r0, c0, h, w);
    const int64_t n = h * w;
    int nan = 0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
      nan |= (f2u(load_as_float(x, p.x_dtype, (r0 + i / w) * p.K + c0 + i % w)) & 0x7FFFFFFFu) > kInf;
    float value;
    if (__syncthreads_or(nan)) {
      value = u2f(kQNaN);
    } else {
      const double rank = __dmul_rn((double)(n - 1), pct);
      const int64_t below = (int64_t)floor(rank), above = (int64_t)ceil(rank);
      const double lo = (double)u2f(domain_select(x, p, r0, c0, w, n, below, hist, &s_prefix, &s_rank));
      const double hi = (double)u2f(domain_select(x, p, r0, c0, w, n, above, hist, &s_prefix, &s_rank));
      const double wt = __dsub_rn(rank, (double)below);
      const double diff = __dsub_rn(hi, lo);
      const double v = wt < 0.5 ? __dadd_rn(lo, __dmul_rn(wt, diff)) : __dsub_rn(hi, __dmul_rn(diff, __dsub_rn(1.0, wt)));
      value = __double2float_rn(v);
    }
    if (threadIdx.x == 0) {
      const float d2 = p.two_level ? *d2p : 1.0f;
      const float sc = amax_scale(value, d2, p.two_level, p, scale_noise ? scale_noise[d] : 0u);
      scale[d] = sc;
      if (scodes) scodes[d] = (uint8_t)scale_code(sc, p.sf);
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ host side
static int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

static int stats_parts(int64_t domain_elems) {
  int64_t parts = cdiv(domain_elems, 8192);
  if (parts > 4096) parts = 4096;
  return (int)(parts < 1 ? 1 : parts);
}

enum { PATH_FLAT = 0, PATH_GROUP = 1, PATH_ROW = 2, PATH_TENSOR = 3, PATH_GENERAL = 4, PATH_GROUP_LEAN = 5 };

struct Plan {
  QParams p;
  Lean ln;
  LeanPow2 lp;
  Ratios rt;          // MSE candidates (rt.n == 0: no search)
  double pct;         // percentile / 100 (percentile method)
  int64_t nd;
  int parts;          // per-domain partials of the general path
  int path;
  size_t ws_stats, total;  // general-path partials; plus one tensor Stat slot
  size_t off_amax, off_err;  // MSE / percentile: per-domain amax, per-(domain, part, candidate) errors
};

static int make_plan(const void *x, int32_t x_dtype, int64_t rows, int64_t K, const tc_quant_spec *spec,
                     const tc_quant_out *out, Plan &pl) {
  std::memset(&pl, 0, sizeof(pl));
  QParams &p = pl.p;
  std::string err = fmt_error(spec->format);
  if (!err.empty()) return set_error("element format: " + err), TC_INVALID_ARGUMENT;
  if (spec->format.kind == 2) return set_error("e8m0 is a scale format, not an element format"), TC_INVALID_ARGUMENT;
  if (rows <= 0 || K <= 0) return set_error("quantization needs a nonempty tensor of shape [..., K]"), TC_INVALID_ARGUMENT;
  if (rows * K >= (1ll << 40)) return set_error("tensor too large"), TC_INVALID_ARGUMENT;
  if (x_dtype < 0 || x_dtype > 2) return set_error("unsupported input dtype"), TC_INVALID_ARGUMENT;
  if (spec->sr_bits < 1 || spec->sr_bits > 32) return set_error("sr_bits must be in [1, 32]"), TC_INVALID_ARGUMENT;
  p.ef = derive(spec->format);
  pl.ln = make_lean(spec->format, p.ef, spec->rounding, spec->saturate);
  p.rows = rows;
  p.K = K;
  p.has_scale = spec->has_scale;
  p.method = spec->scale_method;
  p.srnd = spec->scale_rounding;
  p.two_level = spec->has_scale && spec->two_level;
  p.zp = spec->zero_point;
  p.rnd = spec->rounding;
  p.sr_bits = spec->sr_bits;
  p.saturate = spec->saturate;
  p.x_dtype = x_dtype;
  p.v_dtype = out->values_dtype;
  p.max_elem_d = fmt_max_normal(spec->format);
  p.max_elem = (float)p.max_elem_d;
  p.emax_elem = fmt_emax_elem(spec->format);
  if (spec->format.kind == 1) {
    p.qmin_d = (double)p.ef.qmin;
    p.qmax_d = (double)p.ef.qmax;
    p.qrange = (float)(p.ef.qmax - p.ef.qmin);
  }
  int total_bits = spec->format.kind == 0 ? spec->format.ebits + spec->format.mbits + (spec->format.is_signed ? 1 : 0)
                                          : spec->format.bits;
  if (out->codes) {
    if (total_bits > 8) return set_error("element codes need a format of at most 8 bits"), TC_INVALID_ARGUMENT;
    p.code_bits = total_bits <= 4 ? 4 : 8;
    if (p.code_bits == 4 && ((rows * K) & 1)) return set_error("4-bit codes need an even element count"), TC_INVALID_ARGUMENT;
  }
  if (!spec->has_scale) {
    if (spec->granularity != GRAN_TENSOR) return set_error("a direct cast (scale=None) has no granularity"), TC_INVALID_ARGUMENT;
    if (spec->zero_point) return set_error("zero points need a scale"), TC_INVALID_ARGUMENT;
    p.dr = rows; p.dc = K; p.nr = 1; p.nc = 1;
    pl.nd = 0;
    pl.path = PATH_FLAT;
    pl.total = 256;
    return TC_OK;
  }
  err = fmt_error(spec->scale_format);
  if (!err.empty()) return set_error("scale format: " + err), TC_INVALID_ARGUMENT;
  p.sf = derive(spec->scale_format);
  p.min_scale_bits = p.sf.min_sub_bits;
  if (spec->scale_format.kind == 0) {
    uint32_t u;
    float m = (float)fmt_min_scale(spec->scale_format);
    std::memcpy(&u, &m, 4);
    p.min_scale_bits = u;
  }
  p.prod_max_d = fmt_max_normal(spec->format) * fmt_max_normal(spec->scale_format);
  if (out->scale_codes) {
    int sbits = spec->scale_format.kind == 2 ? 8
              : spec->scale_format.kind == 0 ? spec->scale_format.ebits + spec->scale_format.mbits + (spec->scale_format.is_signed ? 1 : 0)
                                             : 99;
    if (sbits > 8) return set_error("scale codes need a scale format of at most 8 bits"), TC_INVALID_ARGUMENT;
    p.scode = 1;
  }
  if (spec->scale_method == M_MSE) {
    if (spec->n_search < 1 || !spec->mse_search)
      return set_error("mse scale selection needs its candidate ratios (n_search >= 1)"), TC_INVALID_ARGUMENT;
    if (spec->n_search > kMaxRatios)
      return set_error("mse scale selection supports at most 256 candidates"), TC_UNSUPPORTED;
    pl.rt.n = spec->n_search;
    for (int c = 0; c < spec->n_search; ++c) pl.rt.r[c] = spec->mse_search[c];
  }
  if (spec->scale_method == M_PERCENTILE) {
    if (!(spec->percentile > 0.0f && spec->percentile <= 100.0f))
      return set_error("percentile must be in (0, 100]"), TC_INVALID_ARGUMENT;
    pl.pct = (double)spec->percentile / 100.0;
  }
  switch (spec->granularity) {
    case GRAN_TENSOR: p.dr = rows; p.dc = K; break;
    case GRAN_ROW: p.dr = 1; p.dc = K; break;
    case GRAN_GROUP:
      if (spec->group_size <= 0) return set_error("granularity 'group' needs group_size > 0"), TC_INVALID_ARGUMENT;
      p.dr = 1; p.dc = spec->group_size; break;
    case GRAN_BLOCK:
      if (spec->block_rows <= 0 || spec->block_cols <= 0)
        return set_error("granularity 'block' needs block=(rows, cols) > 0"), TC_INVALID_ARGUMENT;
      p.dr = spec->block_rows; p.dc = spec->block_cols; break;
    default: return set_error("unknown granularity"), TC_INVALID_ARGUMENT;
  }
  if (p.dr > rows) p.dr = rows;
  if (p.dc > K) p.dc = K;
  p.nr = cdiv(rows, p.dr);
  p.nc = cdiv(K, p.dc);
  pl.nd = p.nr * p.nc;
  // Power-of-two divisors (one-level pow2 methods) are applied by an exact reciprocal multiply.
  p.pow2_div = !p.two_level && !p.zp && (p.method == M_POW2_FLOOR || p.method == M_POW2_CEIL);
  int gs = (int)p.dc;
  bool aligned = ((uintptr_t)x % (x_dtype == TC_F32 ? 16 : 8)) == 0;
  bool group_ok = spec->granularity == GRAN_GROUP && p.dr == 1 && K % gs == 0 && gs % 4 == 0 &&
                  (gs == 4 || gs == 8 || gs == 16 || gs == 32 || gs == 64 || gs == 128) && aligned &&
                  (!out->values || ((uintptr_t)out->values % 16) == 0) &&
                  (!out->dequant || ((uintptr_t)out->dequant % 16) == 0) &&
                  (!out->codes || ((uintptr_t)out->codes % 4) == 0);
  // The lean group pass: float elements with a nearest-even or directed rounding, no zero point,
  // 8 elements per lane (group sizes 8..128), absmax or power-of-two scales.
  const bool pow2_method = !p.two_level && (p.method == M_POW2_FLOOR || p.method == M_POW2_CEIL);
  const bool searched = p.method == M_MSE || p.method == M_PERCENTILE;
  bool lean_ok = group_ok && !searched && pl.ln.ok && !p.zp && gs % 8 == 0 &&
                 (p.two_level || p.method == M_ABSMAX || pow2_method) &&
                 (!out->codes || ((uintptr_t)out->codes % (p.code_bits == 4 ? 8 : 16)) == 0);
  if (pow2_method) {
    float mx = (float)p.max_elem_d;
    uint32_t mb;
    std::memcpy(&mb, &mx, 4);
    pl.lp.max_sig = (mb & 0x7FFFFFu) | 0x800000u;
    pl.lp.emax_elem = p.emax_elem;
    pl.lp.emin = p.sf.emin;
    pl.lp.emax = p.sf.emax;
    pl.lp.bias = p.sf.bias;
    pl.lp.e8m0_code = spec->scale_format.kind == 2;
    lean_ok = lean_ok && (spec->scale_format.kind == 2 || spec->scale_format.kind == 0) && p.sf.emin >= -127 &&
              p.sf.emax <= 127 && (mb >> 23) != 0;
  }
  if (lean_ok) pl.path = PATH_GROUP_LEAN;
  else if (group_ok && p.method != M_PERCENTILE) pl.path = PATH_GROUP;  // MSE searches inside the group pass
  else if (searched) pl.path = PATH_GENERAL;
  // A single domain of more than a few thousand elements (a whole tensor, or the one row of a decode
  // step's activation) takes the grid-wide tensor pipeline; the row pass runs one block per row.
  else if (p.nr == 1 && p.nc == 1 && rows * K >= 2048 && (!out->codes || p.code_bits == 8 || (rows * K) % 2 == 0))
    pl.path = PATH_TENSOR;  // (the flat element pass packs 4-bit codes in pairs)
  else if (p.dr == 1 && p.dc == K && (!out->codes || p.code_bits == 8 || K % 2 == 0)) pl.path = PATH_ROW;
  else if (p.nr == 1 && p.nc == 1) pl.path = PATH_TENSOR;
  else pl.path = PATH_GENERAL;
  pl.parts = stats_parts(p.dr * p.dc);
  pl.ws_stats = pl.path == PATH_GENERAL ? sizeof(Stat) * (size_t)pl.nd * pl.parts : 0;
  size_t off = ((pl.ws_stats + 255) & ~(size_t)255) + 256;  // + tensor Stat slot
  if (pl.path == PATH_GENERAL && searched) {
    pl.off_amax = off;
    off += ((size_t)pl.nd * sizeof(float) + 255) & ~(size_t)255;
    pl.off_err = off;
    off += ((size_t)pl.nd * pl.parts * (size_t)(pl.rt.n > 0 ? pl.rt.n : 0) * sizeof(double) + 255) & ~(size_t)255;
  }
  pl.total = off;
  return TC_OK;
}

}  // namespace tc

using namespace tc;

extern "C" int tc_cast(const float *x, float *y, const uint32_t *noise, int64_t n, const tc_format *fmt,
                       int32_t rounding, int32_t saturate, int32_t sr_bits, tc_stream stream) {
  if (!fmt || (n > 0 && (!x || !y))) return set_error("tc_cast: null argument"), TC_INVALID_ARGUMENT;
  std::string err = fmt_error(*fmt);
  if (!err.empty()) return set_error("tc_cast: " + err), TC_INVALID_ARGUMENT;
  if (rounding < 0 || rounding > 5) return set_error("tc_cast: unknown rounding"), TC_INVALID_ARGUMENT;
  if (fmt->kind == 2 && rounding == TC_SR)
    return set_error("stochastic rounding is not defined for power-of-two formats"), TC_INVALID_ARGUMENT;
  if (sr_bits < 1 || sr_bits > 32) return set_error("sr_bits must be in [1, 32]"), TC_INVALID_ARGUMENT;
  if (n <= 0) return TC_OK;
  Fmt f = derive(*fmt);
  const Lean ln = make_lean(*fmt, f, rounding, saturate);
  if (ln.ok && (uintptr_t)x % 16 == 0 && (uintptr_t)y % 16 == 0) {
    const int grid = grid_for((n + 7) / 8, 256);
    cudaStream_t s = (cudaStream_t)stream;
    switch (rounding) {
      case TC_RNE: cast_lean_kernel<TC_RNE><<<grid, 256, 0, s>>>(x, y, n, ln); break;
      case TC_RTZ: cast_lean_kernel<TC_RTZ><<<grid, 256, 0, s>>>(x, y, n, ln); break;
      case TC_RUP: cast_lean_kernel<TC_RUP><<<grid, 256, 0, s>>>(x, y, n, ln); break;
      default: cast_lean_kernel<TC_RDN><<<grid, 256, 0, s>>>(x, y, n, ln); break;
    }
    ::tc::count_launch();
    return launch_status("tc_cast");
  }
  int vec = ((uintptr_t)x % 16 == 0) && ((uintptr_t)y % 16 == 0) && (!noise || (uintptr_t)noise % 16 == 0);
  cast_kernel<<<grid_for(vec ? (n + 3) / 4 : n, 256), 256, 0, (cudaStream_t)stream>>>(x, y, noise, n, f, rounding,
                                                                                   saturate, sr_bits, vec);
  ::tc::count_launch();
  return launch_status("tc_cast");
}

extern "C" size_t tc_quantize_workspace(int64_t rows, int64_t K, const tc_quant_spec *spec) {
  if (!spec) return 0;
  Plan pl;
  tc_quant_out dummy;
  std::memset(&dummy, 0, sizeof(dummy));
  // Upper bound independent of pointer alignment: size the general path's partials as well.
  static float probe[4] __attribute__((aligned(16)));
  if (make_plan(probe, TC_F32, rows, K, spec, &dummy, pl) != TC_OK) return 256;
  size_t stats = pl.nd ? sizeof(Stat) * (size_t)pl.nd * pl.parts : 0;
  size_t total = ((stats + 255) & ~(size_t)255) + 256;
  if (spec->has_scale && (spec->scale_method == M_MSE || spec->scale_method == M_PERCENTILE)) {
    total += ((size_t)pl.nd * sizeof(float) + 255) & ~(size_t)255;
    total += ((size_t)pl.nd * pl.parts * (size_t)pl.rt.n * sizeof(double) + 255) & ~(size_t)255;
  }
  return total;
}

extern "C" int tc_quantize(const void *x, int32_t x_dtype, int64_t rows, int64_t K, const tc_quant_spec *spec,
                           const float *amax, const uint32_t *noise, const uint32_t *scale_noise,
                           const tc_quant_out *out, void *workspace, size_t workspace_bytes, tc_stream stream) {
  if (!x || !spec || !out) return set_error("tc_quantize: null argument"), TC_INVALID_ARGUMENT;
  if (!out->values && !out->codes && !out->dequant)
    return set_error("tc_quantize: no element output (values, codes or dequant)"), TC_INVALID_ARGUMENT;
  // For tensor granularity an amax override replaces the statistic, so MSE and percentile specs
  // search nothing: TriCast uses the absmax scale of the override (src/tricast/reference/quantize.py:
  // 282-285). For a two-level spec of finer granularity it is the tensor amax that the global decode
  // scale d2 is derived from (a tensor sharded across devices, whose amax the caller reduced); the
  // per-domain scales still come from the data, MSE and percentile searches included.
  const bool d2_amax = amax && spec->granularity != GRAN_TENSOR;
  if (d2_amax && !(spec->has_scale && spec->two_level))
    return set_error("amax override requires tensor granularity and a scalar"), TC_INVALID_ARGUMENT;
  tc_quant_spec eff = *spec;
  if (amax && !d2_amax && spec->has_scale && (spec->scale_method == M_MSE || spec->scale_method == M_PERCENTILE))
    eff.scale_method = M_ABSMAX;
  spec = &eff;
  Plan pl;
  int st = make_plan(x, x_dtype, rows, K, spec, out, pl);
  if (st) return st;
  QParams &p = pl.p;
  if (p.has_scale && (!out->scale || (p.zp && !out->zero_point) || (p.two_level && !out->global_scale)))
    return set_error("tc_quantize: missing scale / zero_point / global_scale output"), TC_INVALID_ARGUMENT;
  if (pl.total > workspace_bytes || !workspace)
    return set_error("tc_quantize: workspace too small"), TC_WORKSPACE_TOO_SMALL;
  cudaStream_t s = (cudaStream_t)stream;
  char *ws = static_cast<char *>(workspace);
  Stat *stats = reinterpret_cast<Stat *>(ws);
  Stat *tstat = reinterpret_cast<Stat *>(ws + ((pl.ws_stats + 255) & ~(size_t)255));
  float *d2 = out->global_scale;
  const int64_t n = rows * K;
  const int lean_rnd = (pl.ln.ok && !p.zp && !noise) ? spec->rounding : -1;
  const int vec = ((uintptr_t)x % 16) == 0;
  if (pl.path == PATH_FLAT) {
    launch_flat(grid_for((n + 3) / 4, 256, 8), s, x, p, pl.ln, lean_rnd, nullptr, nullptr, nullptr, noise,
                out->values, out->codes, out->dequant);
    ::tc::count_launch();
    return launch_status("tc_quantize elements");
  }
  // Tensor statistic: needed for two-level d2, and as the single domain of tensor granularity.
  const bool need_tensor_stat = (p.two_level || pl.path == PATH_TENSOR) && !(amax && !p.zp);
  if (need_tensor_stat) {
    cudaMemsetAsync(tstat, 0, sizeof(Stat), s);
    cudaMemsetAsync(&tstat->lo, 0xFF, sizeof(uint32_t), s);
    if (p.zp)
      tensor_stats_kernel<false><<<grid_for((n + 7) / 8, 256, 8), 256, 0, s>>>(x, x_dtype, n, vec, tstat);
    else
      tensor_stats_kernel<true><<<grid_for((n + 7) / 8, 256, 8), 256, 0, s>>>(x, x_dtype, n, vec, tstat);
    ::tc::count_launch();
  }
  if (p.two_level) {
    tensor_scale_kernel<<<1, 1, 0, s>>>(p, tstat, amax, d2, nullptr, nullptr, nullptr, nullptr, 1);
    ::tc::count_launch();
  }
  if ((st = launch_status("tc_quantize tensor statistic"))) return st;
  if (pl.path == PATH_GROUP_LEAN) {
    const int gs = (int)p.dc;
    const bool pow2 = !p.two_level && p.method != M_ABSMAX;
    const bool fast = spec->rounding == TC_RNE && pl.ln.sat_only;
    const int outs = (!out->values && out->dequant) ? 1 : (out->values && !out->dequant && p.v_dtype == TC_BF16) ? 2 : 0;
    LeanArgs la;
    std::memset(&la, 0, sizeof(la));
    la.x = x;
    la.p = p;
    la.ln = pl.ln;
    la.lp = pl.lp;
    la.cm.hi = 1u << (32 - pl.ln.mshift);
    la.cm.two = 2u;
    la.cm.neg_k = 0u - ((1u << (31 - pl.ln.mshift)) - (1u << pl.ln.sign_pos));
    la.cm.radix = p.code_bits == 4 ? 16u : 256u;
    la.d2 = d2;
    la.scale_noise = scale_noise;
    la.values = out->values;
    la.scale = out->scale;
    la.codes = out->codes;
    la.scodes = out->scale_codes;
    la.dequant = out->dequant;
    // The register-staged kernel over whole warp iterations, then the four-elements-per-lane pass
    // over the last few groups (pointers offset to that range).
    int64_t done = 0;
    {
      const int esz = x_dtype == TC_F32 ? 4 : 2;
      const int vsz = out->values_dtype == TC_F32 ? 4 : 2;
      auto shifted = [&](int64_t off, int64_t count) {
        LeanArgs r = la;
        r.p.rows = 1;
        r.p.K = count;
        r.x = static_cast<const char *>(x) + off * esz;
        r.values = out->values ? static_cast<char *>(out->values) + off * vsz : nullptr;
        r.codes = out->codes ? out->codes + (p.code_bits == 4 ? off / 2 : off) : nullptr;
        r.scodes = out->scale_codes ? out->scale_codes + off / gs : nullptr;
        r.dequant = out->dequant ? out->dequant + off : nullptr;
        r.scale = out->scale + off / gs;
        r.scale_noise = scale_noise ? scale_noise + off / gs : nullptr;
        return r;
      };
      const int64_t rest_groups = (n - done) / gs;
      const int lanes_per_group = gs == 8 ? 1 : gs / 16;  // 8 elements per lane for gs 8, else 16
      const int64_t per_warp = 32 / lanes_per_group;
      const int64_t main_groups = rest_groups / per_warp * per_warp;
      if (main_groups > 0) {
        const LeanArgs r = shifted(done, main_groups * gs);
        // Up to 16 CTAs per SM (two resident waves): the cfg1 cast measured 4.585 TB/s against 4.54 with
        // one wave of 8, 4.41 with 4 and 4.32 with 32.
        const int grid = grid_for(main_groups * lanes_per_group, 256, 16);
        const int gi = gs == 8 ? 0 : gs == 16 ? 1 : gs == 32 ? 2 : gs == 64 ? 3 : 4;
        if (!out->codes) launch_group_lean_c0(r, grid, gi, pow2, fast, outs, s);
        else if (p.code_bits == 4) launch_group_lean_c4(r, grid, gi, pow2, fast, outs, s);
        else launch_group_lean_c8(r, grid, gi, pow2, fast, outs, s);
        ::tc::count_launch();
        done += main_groups * gs;
      }
      if (done < n) {
        const LeanArgs r = shifted(done, n - done);
        Ratios no_search;
        no_search.n = 0;
        const int L = gs / 4;
        const int tgrid = grid_for((n - done) / gs * L, 256, 16);
#define TC_TAIL_CASE(LL)                                                                                   \
  case LL:                                                                                                 \
    group_kernel<LL><<<tgrid, 256, 0, s>>>(r.x, r.p, d2, nullptr, r.scale_noise, r.values, r.scale, nullptr, \
                                           r.codes, r.scodes, r.dequant, no_search);                       \
    break;
        switch (L) {
          TC_TAIL_CASE(2)
          TC_TAIL_CASE(4)
          TC_TAIL_CASE(8)
          TC_TAIL_CASE(16)
          TC_TAIL_CASE(32)
        }
#undef TC_TAIL_CASE
        ::tc::count_launch();
      }
    }
    return launch_status("tc_quantize lean group pass");
  }
  if (pl.path == PATH_GROUP) {
    int L = (int)(p.dc / 4);
    int64_t ngroups = n / p.dc;
    int grid = grid_for(ngroups * L, 256, 16);
#define TC_GROUP_CASE(LL)                                                                                         \
  case LL:                                                                                                        \
    group_kernel<LL><<<grid, 256, 0, s>>>(x, p, d2, noise, scale_noise, out->values, out->scale, out->zero_point, \
                                          out->codes, out->scale_codes, out->dequant, pl.rt);                     \
    ::tc::count_launch();                                                                                         \
    break;
    switch (L) {
      TC_GROUP_CASE(1)
      TC_GROUP_CASE(2)
      TC_GROUP_CASE(4)
      TC_GROUP_CASE(8)
      TC_GROUP_CASE(16)
      TC_GROUP_CASE(32)
    }
#undef TC_GROUP_CASE
    return launch_status("tc_quantize group pass");
  }
  if (pl.path == PATH_ROW) {
    int grid = (int)(rows < (int64_t)sm_count() * 8 ? rows : (int64_t)sm_count() * 8);
    row_kernel<<<grid, 256, 0, s>>>(x, p, d2, noise, scale_noise, out->values, out->scale, out->zero_point,
                                    out->codes, out->scale_codes, out->dequant);
    ::tc::count_launch();
    return launch_status("tc_quantize row pass");
  }
  if (pl.path == PATH_TENSOR) {
    tensor_scale_kernel<<<1, 1, 0, s>>>(p, tstat, (amax && !p.zp) ? amax : nullptr, d2, scale_noise, out->scale,
                                        out->zero_point, out->scale_codes, 0);
    ::tc::count_launch();
    launch_flat(grid_for((n + 3) / 4, 256, 8), s, x, p, pl.ln, lean_rnd, out->scale, out->zero_point, d2, noise,
                out->values, out->codes, out->dequant);
    ::tc::count_launch();
    return launch_status("tc_quantize tensor pass");
  }
  int64_t chunk = cdiv(p.dr * p.dc, pl.parts);
  if (p.method == M_PERCENTILE) {
    const int grid = (int)std::min<int64_t>(pl.nd, (int64_t)sm_count() * 8);
    percentile_kernel<<<grid, 256, 0, s>>>(x, p, pl.nd, pl.pct, d2, scale_noise, out->scale, out->scale_codes);
    ::tc::count_launch();
  } else {
    stats_kernel<<<(unsigned)(pl.nd * pl.parts), 256, 0, s>>>(x, p, pl.nd, pl.parts, chunk, stats);
    ::tc::count_launch();
    if (pl.rt.n > 0) {
      float *dom_amax = reinterpret_cast<float *>(ws + pl.off_amax);
      double *err = reinterpret_cast<double *>(ws + pl.off_err);
      domain_amax_kernel<<<(unsigned)cdiv(pl.nd * 32, 256), 256, 0, s>>>(pl.nd, pl.parts, stats, dom_amax);
      ::tc::count_launch();
      mse_partial_kernel<<<(unsigned)(pl.nd * pl.parts), 256, 0, s>>>(x, p, pl.nd, pl.parts, chunk, dom_amax, d2, noise,
                                                                      scale_noise, pl.rt, err);
      ::tc::count_launch();
      mse_select_kernel<<<(unsigned)cdiv(pl.nd, 256), 256, 0, s>>>(p, pl.nd, pl.parts, pl.rt, dom_amax, d2,
                                                                  scale_noise, err, out->scale, out->scale_codes);
      ::tc::count_launch();
    } else {
      scale_kernel<<<(unsigned)cdiv(pl.nd * 32, 256), 256, 0, s>>>(p, pl.nd, pl.parts, stats, nullptr, d2, scale_noise,
                                                                  out->scale, out->zero_point, out->scale_codes, 0);
      ::tc::count_launch();
    }
  }
  if ((st = launch_status("tc_quantize scales"))) return st;
  element_kernel<<<grid_for((n + 1) / 2, 256), 256, 0, s>>>(x, p, out->scale, out->zero_point, d2, noise, out->values,
                                                           out->codes, out->dequant);
  ::tc::count_launch();
  return launch_status("tc_quantize elements");
}

// Tensor amax of a shard, as the bit pattern of the fp32 |x| maximum (NaN-propagating: NaN bits sort
// above Inf's), max-reduced into *bits (accumulating: the caller clears it, and may reduce several
// shards or ranks into it with an integer max).
extern "C" int tc_tensor_amax_bits(const void *x, int32_t x_dtype, int64_t n, uint32_t *bits, tc_stream stream) {
  if (n <= 0) return TC_OK;
  if (!x || !bits || x_dtype < 0 || x_dtype > 2) return set_error("tc_tensor_amax_bits: bad argument"), TC_INVALID_ARGUMENT;
  const int vec = ((uintptr_t)x % 16) == 0;
  tensor_stats_kernel<true><<<grid_for((n + 7) / 8, 256, 8), 256, 0, (cudaStream_t)stream>>>(x, x_dtype, n, vec,
                                                                                             nullptr, bits);
  ::tc::count_launch();
  return launch_status("tc_tensor_amax_bits");
}
