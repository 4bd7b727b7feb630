// Small-M emulated GEMM kernels (M <= 16, the decode shapes TriCast routes to its _gemv kernel,
// src/tricast/kernels/mma.py:483-485,663-720,845-847). The tiled kernels stage 64-row tiles; with a
// handful of rows most of that work would be padding, and the operand encoders would write several
// bytes per element of the (large) B operand for a single use. These kernels read B straight from
// its container and scales, once, and keep every row of A in the same CTA.
//
// GDFS, E2M1 x E2M1 (gdfs_fp4_gemv_kernel). The arithmetic is the tiled kernel's (tc_gemm_fast.cu):
// a group of 16 contributes D * ms_a * ms_b * 2**(es_a + es_b - srad - 2) with D the DP4A dot product
// of the doubled codes, and a K tile whose every group value is a multiple of 2**(emax'' - F), with
// the running value's bits kept, is summed exactly and normalised by one fp64 -> fp32 rounding. Here
// the bounds are taken per output and per tile over the groups whose D is non-zero:
//     emax'' = max(e_c, max_g (es_a + es_b + class_a + class_b)) >= emax,
//     E = min_g (es_a + es_b),  safe iff  emax'' <= E - srad - 2 + F  and  emax'' - e_c <= F - 23,
// and the tile's value sum_g D ms_a ms_b 2**(es_a + es_b - srad - 2) is formed in fp64, exact while
// the exponent spread of its groups is at most 30 (|D ms_a ms_b| < 2**20, at most 8 groups). A tile
// that fails runs the reference's exact two-pass step for that output (exponent-class labels, aligned
// truncated integer terms, fixed-point normalisation).
//
// Work split: a CTA owns 16 columns (rows of B) and all M rows. K advances in chunks of 32 groups
// (512 elements): warp w loads the chunk of columns w and w + 8, lane = group, so each warp reads
// two contiguous 1 KB (bf16) row segments; the raw values of the next chunk are loaded into registers
// before the current chunk is scanned. Each lane encodes its group, forms D against every row of A
// (A encoded once by encode_fp4_kernel, rows padded to 16) and writes it to shared memory; then thread
// (m, column) runs the sequential tile scan of its output over the chunk. One barrier per chunk: the
// product table is double-buffered.
//
// Operands or scales the fast path cannot take (off-grid or non-finite values, wide scale
// significands) raise the device flag; the exact generic kernel queued behind this one then
// recomputes every output.
#include <algorithm>
#include <cstring>
#include <string>

#include "tc_bulk.cuh"
#include "tc_fp4.cuh"
#include "tc_generic.cuh"

namespace tc {
namespace gemv {

constexpr int kThreads = 256;
constexpr int kGroups = 32;  // groups per chunk: one per lane

// Per (column, K tile, row of A): the tile's value over its groups with D != 0 (exact when their
// exponent spread is at most 30), the largest label bound and the smallest scale exponent sum.
struct TileRec {
  double sum;
  int lmax, emin;
};

// Slabs whose small-M kernels fell back to the exact routine, per device (reported with the generic
// kernel's count by tc_exact_fallbacks).
__device__ unsigned long long g_gemv_fallbacks;

struct Fp4Args {
  const uint4 *aq, *am;      // A records [groups][mp] (codes, exponent-class masks), padded to whole chunks
  const uint32_t *as;        // A scale words [groups][mp]
  int mp;                    // A rows padded to a power of two
  const void *bv;            // B values [N][K] in their container
  const float *bscale;       // B K scales [N][nkd] or nullptr
  int64_t b_nkd;
  int b_kd, b_field0, bvec;  // bvec: B rows start 16-byte aligned (whole groups load as vectors)
  Fmt bsf;
  int64_t M, N, K, ngroups;  // ngroups = ceil(K / 16)
  int ng;                    // groups per K tile
  int F, shift0, srad2;
  const float *alpha_a, *alpha_b, *bias;
  Fmt of;
  int out_plain, out_dt;
  void *out;
  GemmDesc g;                // the whole product, for the exact fallback
  int64_t ngroups_pad;       // groups rounded up to whole chunks
  TileRec *rec;              // [ns][ntiles][M]
  int64_t ntiles, n_base, ns;  // K tiles; the slab of columns [n_base, n_base + ns)
  int32_t *flag;             // nonzero: the fast path cannot take the operands
};

// Raw bytes of one group (16 elements) of a B row: 2 (bf16 / fp16) or 4 (fp32) 16-byte vectors.
template <int DT>
struct Raw {
  static constexpr int kVec = DT == TC_F32 ? 4 : 2;
  uint4 u[kVec];
};

template <int DT>
__device__ __forceinline__ void raw_load(const Fp4Args &p, int64_t n, int64_t gi, Raw<DT> &r) {
  constexpr int esz = DT == TC_F32 ? 4 : 2;
  const int64_t k0 = gi * fp4::kGS;
  if (n < p.N && gi < p.ngroups && p.bvec && k0 + fp4::kGS <= p.K) {
    const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const char *>(p.bv) + (n * p.K + k0) * esz);
#pragma unroll
    for (int w = 0; w < Raw<DT>::kVec; ++w) r.u[w] = __ldcs(src + w);  // streamed once
  }
}

template <int DT>
__device__ __forceinline__ void raw_values(const Fp4Args &p, int64_t n, int64_t gi, const Raw<DT> &r,
                                           float (&v)[fp4::kGS]) {
  const int64_t k0 = gi * fp4::kGS;
  if (p.bvec && k0 + fp4::kGS <= p.K) {
#pragma unroll
    for (int w = 0; w < Raw<DT>::kVec; ++w) {
      const uint32_t uu[4] = {r.u[w].x, r.u[w].y, r.u[w].z, r.u[w].w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        if (DT == TC_F32) {
          v[4 * w + h] = u2f(uu[h]);
        } else if (DT == TC_BF16) {
          v[8 * w + 2 * h] = u2f(uu[h] << 16);
          v[8 * w + 2 * h + 1] = u2f(uu[h] & 0xFFFF0000u);
        } else {
          v[8 * w + 2 * h] = __half2float(__ushort_as_half((unsigned short)(uu[h] & 0xFFFF)));
          v[8 * w + 2 * h + 1] = __half2float(__ushort_as_half((unsigned short)(uu[h] >> 16)));
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < fp4::kGS; ++j) v[j] = k0 + j < p.K ? load_as_float(p.bv, DT, n * p.K + k0 + j) : 0.0f;
  }
}

// Codes, scale word and exponent-class masks of B's group (n, gi), as encode_fp4_kernel would make
// them (zero-scale groups become all-zero groups).
template <int DT>
__device__ __forceinline__ void b_group(const Fp4Args &p, int64_t n, int64_t gi, const Raw<DT> &r, uint4 &q,
                                        uint32_t &sword, uint4 &masks, bool &bad) {
  float v[fp4::kGS];
  raw_values<DT>(p, n, gi, r, v);
  const int64_t left = p.K - gi * fp4::kGS;
  uint32_t c0, c1, c2;
  fp4::e2m1_codes(v, left < fp4::kGS ? (int)left : fp4::kGS, q, c0, c1, c2, bad);
  bool zero = false;
  sword = p.bscale ? fp4::group_scale_word(p.bscale[n * p.b_nkd + gi * fp4::kGS / p.b_kd], p.bsf, p.b_field0, zero, bad)
                   : fp4::pack_scale(0, 1, 0);
  if (zero) {
    q = make_uint4(0, 0, 0, 0);
    c0 = c1 = c2 = 0;
  }
  const uint32_t gemax = c2 ? 2u : c1 ? 1u : 0u;
  sword |= (gemax << 25) | ((c0 == 0 ? 1u : 0u) << 27);
  masks = fp4::b_masks(c0, c1, c2);
}

// b_group without the exponent-class masks, for whole in-range groups loaded as vectors: codes from
// the container bit patterns (e2m1_code_bits), the group's largest exponent class from the largest
// code magnitude. Other groups take b_group.
template <int DT>
__device__ __forceinline__ void b_group_fast(const Fp4Args &p, int64_t n, int64_t gi, const Raw<DT> &r, uint4 &q,
                                             uint32_t &sword, bool &bad) {
  const int64_t k0 = gi * fp4::kGS;
  if (!(p.bvec && k0 + fp4::kGS <= p.K)) {
    uint4 masks;
    b_group<DT>(p, n, gi, r, q, sword, masks, bad);
    return;
  }
  uint32_t codes[4] = {0, 0, 0, 0};
  int maxmag = 0;
  bool ok = true;
  if (DT == TC_BF16) {
    uint32_t orm = 0;
    codes[0] = fp4::e2m1_codes4_bf16(r.u[0].x, r.u[0].y, ok, orm);
    codes[1] = fp4::e2m1_codes4_bf16(r.u[0].z, r.u[0].w, ok, orm);
    codes[2] = fp4::e2m1_codes4_bf16(r.u[1].x, r.u[1].y, ok, orm);
    codes[3] = fp4::e2m1_codes4_bf16(r.u[1].z, r.u[1].w, ok, orm);
    maxmag = (orm & 0x08080808u) ? 8 : (orm & 0x0C0C0C0Cu) ? 4 : (orm ? 1 : 0);
  }
#pragma unroll
  for (int j = 0; j < (DT == TC_BF16 ? 0 : fp4::kGS); ++j) {
    uint32_t bits;
    if (DT == TC_F32) {
      const uint4 &u = r.u[j >> 2];
      bits = (j & 3) == 0 ? u.x : (j & 3) == 1 ? u.y : (j & 3) == 2 ? u.z : u.w;
    } else {
      const uint4 &u = r.u[j >> 3];
      const int h = (j & 7) >> 1;
      const uint32_t w = h == 0 ? u.x : h == 1 ? u.y : h == 2 ? u.z : u.w;
      bits = (j & 1) ? (w >> 16) : (w & 0xFFFFu);
    }
    const int code = fp4::e2m1_code_bits<DT>(bits, ok);
    maxmag = max(maxmag, code < 0 ? -code : code);
    codes[j >> 2] |= ((uint32_t)code & 0xFFu) << (8 * (j & 3));
  }
  if (!ok) bad = true;
  bool zero = false;
  sword = p.bscale ? fp4::group_scale_word_fast(p.bscale[n * p.b_nkd + k0 / p.b_kd], p.bsf, p.b_field0, zero, bad)
                   : fp4::pack_scale(0, 1, 0);
  if (zero) {
    codes[0] = codes[1] = codes[2] = codes[3] = 0;
    maxmag = 0;
  }
  q = make_uint4(codes[0], codes[1], codes[2], codes[3]);
  // Doubled codes: |v| >= 4 is |code| >= 8 (class 2), |v| >= 2 is |code| >= 4 (class 1).
  const uint32_t gemax = maxmag >= 8 ? 2u : maxmag >= 4 ? 1u : 0u;
  sword |= (gemax << 25) | ((maxmag == 0 ? 1u : 0u) << 27);
}

__device__ __forceinline__ double pow2d(int e) { return __hiloint2double((e + 1023) << 20, 0); }

// Phase 1. CTA = two chunks of 32 groups (lane = group) x 8 columns (warp = column). Each lane decodes
// its B groups from the container, forms D against every row of A (the chunks' A records staged in
// shared memory) and each group's value and bounds; lanes of a K tile combine them with xor shuffles
// and the tile's first lane writes the record.
constexpr int kChunksPerCta = 2;

template <int DT>
__global__ void __launch_bounds__(kThreads) gdfs_fp4_tiles_kernel(Fp4Args p) {
  if (*p.flag) return;  // A could not be encoded: the scan kernel computes every output exactly
  __shared__ uint4 saq[kChunksPerCta][kGroups * 16];
  __shared__ uint32_t sas[kChunksPerCta][kGroups * 16];
  const int mp = p.mp, M = (int)p.M, ng = p.ng;
  const int64_t nchunks = p.ngroups_pad / kGroups;
  const int64_t ch0 = (int64_t)blockIdx.x * kChunksPerCta;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.y * 8 + warp;  // column within the slab
  const int64_t n = p.n_base + col;
  const int nc = (int)(nchunks - ch0 < kChunksPerCta ? nchunks - ch0 : kChunksPerCta);
  {
    const int nq = kGroups * mp, ns = nq / 4;
    for (int c = 0; c < nc; ++c)
      for (int i = threadIdx.x; i < nq + ns; i += kThreads) {
        if (i < nq) cp_async16(&saq[c][i], p.aq + (ch0 + c) * nq + i);
        else cp_async16(&sas[c][4 * (i - nq)], p.as + (ch0 + c) * nq + 4 * (i - nq));
      }
    cp_async_commit();
  }
  uint4 bq[kChunksPerCta];
  uint32_t swb[kChunksPerCta];
  bool bad = false;
  {
    Raw<DT> r[kChunksPerCta];
#pragma unroll
    for (int c = 0; c < kChunksPerCta; ++c) raw_load<DT>(p, n, (ch0 + c) * kGroups + lane, r[c]);
#pragma unroll
    for (int c = 0; c < kChunksPerCta; ++c) {
      const int64_t gi = (ch0 + c) * kGroups + lane;
      bq[c] = make_uint4(0, 0, 0, 0);
      swb[c] = fp4::pack_scale(0, 0, 0) | (1u << 27);
      if (col < p.ns && n < p.N && gi < p.ngroups) b_group_fast<DT>(p, n, gi, r[c], bq[c], swb[c], bad);
    }
  }
  cp_async_wait_all();
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kChunksPerCta; ++c) {
    if (c >= nc) break;
    const int64_t tile = ((ch0 + c) * kGroups + lane) / ng;
    const bool writer = (lane % ng) == 0 && col < p.ns && n < p.N && tile < p.ntiles;
    const int eb = fp4::scale_exp(swb[c]), cb = (int)((swb[c] >> 25) & 3u);
    const uint32_t msb = (swb[c] >> 16) & 0xFFu;
    for (int m = 0; m < M; ++m) {
      const uint32_t swa = sas[c][lane * mp + m];
      const int d = fp4::dot16(saq[c][lane * mp + m], bq[c]);
      double v = 0.0;
      int lmax = fp4::kNone, emin = fp4::kBig;
      if (d != 0) {
        const int e = fp4::scale_exp(swa) + eb;
        lmax = e + (int)((swa >> 25) & 3u) + cb;
        emin = e;
        const int x = d * (int)(((swa >> 16) & 0xFFu) * msb);  // |x| < 2**20
        v = (double)((((swa ^ swb[c]) >> 24) & 1u) ? -x : x) * pow2d(e - p.srad2);
      }
      for (int o = 1; o < ng; o <<= 1) {
        // Exact while the tile's exponent spread is at most 30 (checked by the scan before use).
        v = __dadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
        lmax = max(lmax, __shfl_xor_sync(0xFFFFFFFFu, lmax, o));
        emin = min(emin, __shfl_xor_sync(0xFFFFFFFFu, emin, o));
      }
      if (writer) p.rec[(col * p.ntiles + tile) * M + m] = TileRec{v, lmax, emin};
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicExch(p.flag, 1);
}

// The reference's exact two-pass tile step for output (m, n) (mma.py:318-336), everything recomputed
// from global memory: exponent labels from the exponent-class masks, then the aligned, truncated
// integer terms and the fixed-point normalisation. Taken by the rare tiles that fail the bounds.
template <int DT, bool RNE>
__device__ __noinline__ float exact_tile(const Fp4Args *pp, float c, int m, int64_t n, int64_t t) {
  const Fp4Args &p = *pp;
  const int64_t g0 = t * p.ng, g1 = min(g0 + p.ng, p.ngroups);
  int emax = fp4::running_exp(c);
  for (int pass = 0; pass < 2; ++pass) {
    int64_t total = pass ? fp4::running_term(c, p.F, emax) : 0;
    for (int64_t gi = g0; gi < g1; ++gi) {
      Raw<DT> rr;
      raw_load<DT>(p, n, gi, rr);
      uint4 bq, bm;
      uint32_t swb;
      bool ignored = false;
      b_group<DT>(p, n, gi, rr, bq, swb, bm, ignored);
      const uint32_t swa = p.as[gi * p.mp + m];
      const int d = fp4::dot16(p.aq[gi * p.mp + m], bq);
      if (d == 0) continue;
      if (pass == 0) {
        const int label = fp4::exp_class_max(p.am[gi * p.mp + m], bm) + fp4::scale_exp(swa) + fp4::scale_exp(swb);
        emax = max(emax, label);
      } else {
        const uint32_t x = (uint32_t)(d < 0 ? -d : d) * (((swa >> 16) & 0xFFu) * ((swb >> 16) & 0xFFu));
        const int sh = p.shift0 + fp4::scale_exp(swa) + fp4::scale_exp(swb) - emax;
        // x < 2**20 and sh <= shift0 <= 40 (a label is at least its scale exponents).
        const int rs = max(40 - sh, 0);
        const uint64_t v = rs >= 64 ? 0ull : (((uint64_t)x << 40) >> rs);
        const bool neg = (d < 0) != (((swa ^ swb) >> 24) & 1u);
        total += neg ? -(int64_t)v : (int64_t)v;
      }
    }
    if (pass) return fixed_to_fp32(total, emax, p.F, RNE, true);
  }
  return c;
}

// Phase 2. One thread per output (m fastest): the K tiles in order, eight records in flight.
template <int DT, bool RNE>
__global__ void __launch_bounds__(128) gdfs_fp4_scan_kernel(const __grid_constant__ Fp4Args p) {
  const int M = (int)p.M;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= p.ns * M) return;
  const int m = (int)(idx % M);
  const int64_t col = idx / M, n = p.n_base + col;
  if (n >= p.N) return;
  if (*p.flag) {  // an operand the fast path cannot take: this output by the exact generic routine
    if (idx == 0) atomicAdd(&g_gemv_fallbacks, 1ull);
    generic_output(p.g, m, n);
    return;
  }
  const TileRec *rec = p.rec + col * p.ntiles * M + m;
  float c = 0.0f;
  constexpr int kBatch = 8;
  TileRec nxt[kBatch];
#pragma unroll
  for (int i = 0; i < kBatch; ++i)
    if (i < p.ntiles) nxt[i] = rec[(int64_t)i * M];
  for (int64_t t0 = 0; t0 < p.ntiles; t0 += kBatch) {
    TileRec cur[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) cur[i] = nxt[i];
#pragma unroll
    for (int i = 0; i < kBatch; ++i)
      if (t0 + kBatch + i < p.ntiles) nxt[i] = rec[(t0 + kBatch + i) * M];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int64_t t = t0 + i;
      if (t >= p.ntiles) break;
      const uint32_t cb = f2u(c) & 0x7FFFFFFFu;
      if (cb >= kInf) break;                         // an Inf / NaN running value is sticky
      const TileRec r = cur[i];
      if (r.lmax == fp4::kNone) continue;            // every group sum is zero: c stays
      const int be = (int)(cb >> 23);
      const int lo = max(r.lmax - (p.F - 23) + 127, 1);
      const int hi = r.emin + p.F - p.srad2 + 127;
      const bool safe = r.lmax - r.emin <= 30 && r.lmax <= r.emin - p.srad2 + p.F &&
                        (cb == 0 || (be >= lo && be <= hi));
      if (safe) {
        // Exact: both are multiples of 2**(emax'' - F) and |v| < 2**(emax'' + 4).
        const double v = __dadd_rn(r.sum, (double)c);
        const float rr = (RNE && fabs(v) >= 0x1p-126) ? __double2float_rn(v) : __double2float_rz(v);
        c = fabs(v) >= 0x1p128 ? __int_as_float((int)((f2u(rr) & 0x80000000u) | kInf)) : rr;
      } else {
        c = exact_tile<DT, RNE>(&p, c, m, n, t);
      }
    }
  }
  // Epilogue: alpha, bias, output rounding (src/tricast/reference/mma.py:376-384).
  float acc = c;
  if (p.alpha_a || p.alpha_b) {
    float alpha = p.alpha_a ? *p.alpha_a : 1.0f;
    if (p.alpha_b) alpha = p.alpha_a ? __fmul_rn(alpha, *p.alpha_b) : *p.alpha_b;
    acc = __fmul_rn(alpha, acc);
  }
  if (p.bias) acc = __fadd_rn(acc, p.bias[n]);
  if (!p.out_plain) acc = cast_to(acc, p.of, TC_RNE, false, 0u, 32);
  store_container(p.out, p.out_dt, (int64_t)m * p.N + n, acc);
}

}  // namespace gemv

// ---------------------------------------------------------------- host side
struct Fp4GemvPlan {
  int64_t ngroups, ngroups_pad, ntiles, slab;
  int mp;
  size_t off_q, off_m, off_s, off_rec, off_flag, total;
};

// Records of at most this many bytes per slab of columns (phase 1 and 2 run once per slab).
constexpr size_t kRecordBytes = (size_t)64 << 20;

static Fp4GemvPlan plan_fp4_gemv(const GemmDesc &g, int ng) {
  Fp4GemvPlan p;
  p.ngroups = (g.K + fp4::kGS - 1) / fp4::kGS;
  p.ngroups_pad = (p.ngroups + gemv::kGroups - 1) / gemv::kGroups * gemv::kGroups;
  p.ntiles = (p.ngroups + ng - 1) / ng;
  p.mp = 1;
  while (p.mp < g.M) p.mp *= 2;
  const size_t per_col = (size_t)std::max<int64_t>(p.ntiles, 1) * g.M * sizeof(gemv::TileRec);
  p.slab = std::max<int64_t>(8, (int64_t)(kRecordBytes / per_col) / 8 * 8);
  p.slab = std::min<int64_t>(p.slab, (int64_t)65535 * 8);
  p.slab = std::min<int64_t>(p.slab, (g.N + 7) / 8 * 8);
  const size_t recs = (size_t)p.ngroups_pad * p.mp;
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  p.off_q = 0;
  p.off_m = up(recs * 16);
  p.off_s = p.off_m + up(recs * 16);
  p.off_rec = p.off_s + up(recs * 4);
  p.off_flag = p.off_rec + up((size_t)p.slab * per_col);
  p.total = p.off_flag + 256;
  return p;
}

size_t fp4_gemv_workspace(const GemmDesc &g, int ng) { return plan_fp4_gemv(g, ng).total; }

uint64_t gemv_exact_fallbacks() {
  unsigned long long v = 0;
  return cudaMemcpyFromSymbol(&v, gemv::g_gemv_fallbacks, sizeof(v)) == cudaSuccess ? (uint64_t)v : 0;
}

template <int DT, bool RNE>
static int launch_fp4_gemv_slabs(gemv::Fp4Args a, int64_t nchunks, int64_t slab, cudaStream_t s) {
  for (int64_t n0 = 0; n0 < a.N; n0 += slab) {
    a.n_base = n0;
    a.ns = std::min<int64_t>(slab, a.N - n0);
    if (nchunks > 0) {
      dim3 grid((unsigned)((nchunks + gemv::kChunksPerCta - 1) / gemv::kChunksPerCta), (unsigned)((a.ns + 7) / 8));
      gemv::gdfs_fp4_tiles_kernel<DT><<<grid, gemv::kThreads, 0, s>>>(a);
      count_launch();
    }
    const int64_t threads = a.ns * a.M;
    gemv::gdfs_fp4_scan_kernel<DT, RNE><<<(unsigned)((threads + 127) / 128), 128, 0, s>>>(a);
    count_launch();
  }
  return TC_OK;
}

template <int DT>
static int launch_fp4_gemv_dt(const gemv::Fp4Args &a, bool rne, int64_t nchunks, int64_t slab, cudaStream_t s) {
  return rne ? launch_fp4_gemv_slabs<DT, true>(a, nchunks, slab, s) : launch_fp4_gemv_slabs<DT, false>(a, nchunks, slab, s);
}

// GDFS-FP4 for M <= 16 (the caller checked the tiled kernel's preconditions: E2M1 operands, G >= 6,
// group size 16, K scales per multiple of 16, 23 <= F <= 48).
int launch_fp4_gemv(const GemmDesc &g, int ng, void *workspace, size_t workspace_bytes, cudaStream_t s) {
  const Fp4GemvPlan p = plan_fp4_gemv(g, ng);
  if (!workspace || workspace_bytes < p.total) return set_error("tc_gemm: workspace too small"), TC_WORKSPACE_TOO_SMALL;
  char *ws = static_cast<char *>(workspace);
  int32_t *flag = reinterpret_cast<int32_t *>(ws + p.off_flag);
  cudaMemsetAsync(flag, 0, 2 * sizeof(int32_t), s);  // [0] operands rejected, [1] timeout: both gate the generic kernel
  if (p.ngroups > 0) {
    fp4::EncodeArgs e;
    std::memset(&e, 0, sizeof(e));
    e.v = g.a.v;
    e.dt = g.a.dt;
    e.rows = g.a.rows;
    e.K = g.a.K;
    e.rows_pad = p.mp;
    e.ntiles = p.ngroups_pad;  // one group per "tile"; groups past K encode as zero
    e.ng = 1;
    e.scale = g.a.skind == SK_K ? g.a.scale : nullptr;
    e.nkd = g.a.nkd;
    e.kd = g.a.kd;
    e.sf = g.a.sf;
    e.field0 = g.a.field0;
    e.q = reinterpret_cast<uint4 *>(ws + p.off_q);
    e.m = reinterpret_cast<uint4 *>(ws + p.off_m);
    e.s = reinterpret_cast<uint32_t *>(ws + p.off_s);
    e.flag = flag;
    e.side = 0;
    const int esz = g.a.dt == TC_F32 ? 4 : 2;
    e.vec = ((uintptr_t)g.a.v % 16 == 0) && ((g.a.K * esz) % 16 == 0);
    const int64_t work = p.ngroups_pad * p.mp;
    const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 16);
    fp4::encode_fp4_kernel<<<(unsigned)blocks, 256, 0, s>>>(e);
    count_launch();
  }
  gemv::Fp4Args a;
  std::memset(&a, 0, sizeof(a));
  a.aq = reinterpret_cast<const uint4 *>(ws + p.off_q);
  a.am = reinterpret_cast<const uint4 *>(ws + p.off_m);
  a.as = reinterpret_cast<const uint32_t *>(ws + p.off_s);
  a.mp = p.mp;
  a.bv = g.b.v;
  a.bscale = g.b.skind == SK_K ? g.b.scale : nullptr;
  a.b_nkd = g.b.nkd;
  a.b_kd = g.b.kd;
  a.b_field0 = g.b.field0;
  a.bsf = g.b.sf;
  const int besz = g.b.dt == TC_F32 ? 4 : 2;
  a.bvec = ((uintptr_t)g.b.v % 16 == 0) && ((g.b.K * besz) % 16 == 0);
  a.M = g.M;
  a.N = g.N;
  a.K = g.K;
  a.ngroups = p.ngroups;
  a.ng = ng;
  a.ntiles = p.ntiles;
  const int srad = (g.a.skind == SK_K ? g.a.srad : 0) + (g.b.skind == SK_K ? g.b.srad : 0);
  a.F = g.F;
  a.shift0 = g.F - 2 - srad;
  a.srad2 = srad + 2;
  a.alpha_a = g.a.alpha;
  a.alpha_b = g.b.alpha;
  a.bias = g.bias;
  a.of = g.of;
  a.out_plain = g.out_is_plain;
  a.out_dt = g.out_dt;
  a.out = g.out;
  a.rec = reinterpret_cast<gemv::TileRec *>(ws + p.off_rec);
  a.g = g;
  a.ngroups_pad = p.ngroups_pad;
  a.flag = flag;
  const int64_t nchunks = p.ngroups_pad / gemv::kGroups;
  int st;
  switch (g.b.dt) {
    case TC_F32: st = launch_fp4_gemv_dt<TC_F32>(a, g.rne, nchunks, p.slab, s); break;
    case TC_BF16: st = launch_fp4_gemv_dt<TC_BF16>(a, g.rne, nchunks, p.slab, s); break;
    default: st = launch_fp4_gemv_dt<TC_F16>(a, g.rne, nchunks, p.slab, s); break;
  }
  if (st) return st;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm gemv: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

}  // namespace tc
