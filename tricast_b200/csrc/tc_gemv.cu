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

namespace tc {
namespace gemv {

constexpr int kThreads = 256;
constexpr int kCols = 16;                  // columns (rows of B) per CTA
constexpr int kGroups = 32;                // groups per chunk: one per lane
constexpr int kDCol = kCols + 1;           // padded column stride of the product table (words)
constexpr int kDRow = kGroups * kDCol + 16;  // padded row stride: rows m and m + 1 hit other banks

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
#pragma unroll
  for (int j = 0; j < fp4::kGS; ++j) {
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
  sword = p.bscale ? fp4::group_scale_word(p.bscale[n * p.b_nkd + k0 / p.b_kd], p.bsf, p.b_field0, zero, bad)
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

template <int DT, bool RNE>
__global__ void __launch_bounds__(kThreads) gdfs_fp4_gemv_kernel(Fp4Args p) {
  if (*p.flag) return;  // A could not be encoded: the generic kernel takes over
  // Dynamic shared memory: products D [2][M][kDRow] (int32), then A's records of three chunks (a ring:
  // codes [3][kGroups * mp] uint4, scale words [3][kGroups * mp] uint32).
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ uint32_t bsw[2][kGroups][kDCol];  // B scale words of the chunk
  const int M = (int)p.M, mp = p.mp;
  int32_t *dsm = reinterpret_cast<int32_t *>(smem_raw);
  uint4 *saq = reinterpret_cast<uint4 *>(smem_raw + (size_t)2 * M * kDRow * sizeof(int32_t));
  uint32_t *sas = reinterpret_cast<uint32_t *>(saq + 3 * kGroups * mp);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t n0 = (int64_t)blockIdx.x * kCols;
  const int64_t nchunks = (p.ngroups + kGroups - 1) / kGroups;
  // Scan role: thread (m, col) for m < M.
  const int sm = threadIdx.x / kCols, scol = threadIdx.x % kCols;
  const bool scanner = sm < M;
  const int64_t sn = n0 + scol;
  float c = 0.0f;
  bool bad = false;

  // A's records of one chunk (contiguous: the arrays are padded to whole chunks) into a ring slot.
  auto copy_a = [&](int64_t ch) {
    const int slot = (int)(ch % 3);
    const int nq = kGroups * mp, ns = kGroups * mp / 4;
    for (int i = threadIdx.x; i < nq + ns; i += kThreads) {
      if (i < nq) cp_async16(saq + slot * nq + i, p.aq + ch * nq + i);
      else cp_async16(sas + slot * nq + 4 * (i - nq), p.as + ch * nq + 4 * (i - nq));
    }
    cp_async_commit();
  };
  copy_a(0);
  Raw<DT> raw[2];
  raw_load<DT>(p, n0 + warp, lane, raw[0]);
  raw_load<DT>(p, n0 + warp + 8, lane, raw[1]);
  cp_async_wait_all();
  __syncthreads();
  for (int64_t ch = 0; ch < nchunks; ++ch) {
    const int buf = (int)(ch & 1), slot = (int)(ch % 3);
    if (ch + 1 < nchunks) copy_a(ch + 1);  // lands during this chunk; the ring slot was last read two chunks ago
    const int64_t gi = ch * kGroups + lane;
    int32_t *dbuf = dsm + buf * M * kDRow;
    // Encode this lane's group of both columns and form D against every row of A.
    uint4 bq[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int col = warp + 8 * j;
      const int64_t n = n0 + col;
      uint32_t sword = fp4::pack_scale(0, 0, 0) | (1u << 27);
      bq[j] = make_uint4(0, 0, 0, 0);
      if (n < p.N && gi < p.ngroups) b_group_fast<DT>(p, n, gi, raw[j], bq[j], sword, bad);
      bsw[buf][lane][col] = sword;
    }
    // Next chunk's raw values are in flight while this one is multiplied and scanned.
    if (ch + 1 < nchunks) {
      raw_load<DT>(p, n0 + warp, gi + kGroups, raw[0]);
      raw_load<DT>(p, n0 + warp + 8, gi + kGroups, raw[1]);
    }
    const uint4 *arow = saq + slot * kGroups * mp + lane * mp;
    for (int m = 0; m < M; ++m) {
      const uint4 aq = arow[m];  // zero codes past K (the encoder pads)
      dbuf[m * kDRow + lane * kDCol + warp] = fp4::dot16(aq, bq[0]);
      dbuf[m * kDRow + lane * kDCol + warp + 8] = fp4::dot16(aq, bq[1]);
    }
    cp_async_wait_all();
    __syncthreads();
    if (scanner && sn < p.N) {
      const int32_t *drow = dbuf + sm * kDRow;
      const uint32_t *swa_row = sas + slot * kGroups * mp + sm;
      const int ng = p.ng, tiles = kGroups / ng;
      for (int t = 0; t < tiles; ++t) {
        const int64_t g0 = ch * kGroups + t * ng;
        if (g0 >= p.ngroups) break;
        const uint32_t cb = f2u(c) & 0x7FFFFFFFu;
        if (cb >= kInf) break;  // an Inf / NaN running value is sticky
        int d[8];
        uint32_t swa[8], swb[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (q < ng) {
            const int l = t * ng + q;
            d[q] = drow[l * kDCol + scol];
            swa[q] = swa_row[l * mp];
            swb[q] = bsw[buf][l][scol];
          } else {
            d[q] = 0;
            swa[q] = swb[q] = 0;
          }
        }
        // Bounds and fp64 value of the tile over its groups with D != 0.
        double sum = 0.0;
        int lmax = fp4::kNone, emin = fp4::kBig;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int e = fp4::scale_exp(swa[q]) + fp4::scale_exp(swb[q]);
          const int x = d[q] * (int)(((swa[q] >> 16) & 0xFFu) * ((swb[q] >> 16) & 0xFFu));
          const bool neg = ((swa[q] ^ swb[q]) >> 24) & 1u;
          if (d[q] != 0) {
            lmax = max(lmax, e + (int)((swa[q] >> 25) & 3u) + (int)((swb[q] >> 25) & 3u));
            emin = min(emin, e);
            sum = __fma_rn((double)(neg ? -x : x), pow2d(e - p.srad2), sum);
          }
        }
        if (lmax == fp4::kNone) continue;  // every group sum is zero: the tile leaves c as it is
        const int be = (int)(cb >> 23);
        const int lo = max(lmax - (p.F - 23) + 127, 1);
        const int hi = emin + p.F - p.srad2 + 127;
        const bool safe = lmax - emin <= 30 && lmax <= emin - p.srad2 + p.F && (cb == 0 || (be >= lo && be <= hi));
        if (safe) {
          const double v = __dadd_rn(sum, (double)c);  // exact: both are multiples of 2**(emax'' - F), |v| < 2**(emax'' + 4)
          float r = (RNE && fabs(v) >= 0x1p-126) ? __double2float_rn(v) : __double2float_rz(v);
          c = fabs(v) >= 0x1p128 ? __int_as_float((int)((f2u(r) & 0x80000000u) | kInf)) : r;
          continue;
        }
        // Exact two-pass step (mma.py:318-336): exponent labels from the exponent-class masks (A's
        // from its records, B's recomputed from the raw group), then the aligned, truncated integer
        // terms and the fixed-point normalisation. Rare; the operands are read again from shared memory.
        int emax = fp4::running_exp(c);
        for (int q = 0; q < ng; ++q) {
          const int l = t * ng + q;
          if (drow[l * kDCol + scol] == 0) continue;
          Raw<DT> rr;
          raw_load<DT>(p, sn, g0 + q, rr);
          uint4 q4, bm;
          uint32_t sw;
          bool ignored = false;
          b_group<DT>(p, sn, g0 + q, rr, q4, sw, bm, ignored);
          const int label = fp4::exp_class_max(__ldg(p.am + (g0 + q) * mp + sm), bm) + fp4::scale_exp(swa_row[l * mp]) +
                            fp4::scale_exp(sw);
          emax = max(emax, label);
        }
        int64_t total = fp4::running_term(c, p.F, emax);
        for (int q = 0; q < ng; ++q) {
          const int l = t * ng + q;
          const int dq = drow[l * kDCol + scol];
          if (dq == 0) continue;
          const uint32_t wa = swa_row[l * mp], wb = bsw[buf][l][scol];
          const uint32_t x = (uint32_t)(dq < 0 ? -dq : dq) * (((wa >> 16) & 0xFFu) * ((wb >> 16) & 0xFFu));
          const int sh = p.shift0 + fp4::scale_exp(wa) + fp4::scale_exp(wb) - emax;
          // x < 2**20 and sh <= shift0 <= 40 (a label is at least its scale exponents).
          const int rs = max(40 - sh, 0);
          const uint64_t v = rs >= 64 ? 0ull : (((uint64_t)x << 40) >> rs);
          const bool neg = (dq < 0) != (((wa ^ wb) >> 24) & 1u);
          total += neg ? -(int64_t)v : (int64_t)v;
        }
        c = fixed_to_fp32(total, emax, p.F, RNE, true);
      }
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicExch(p.flag, 1);
  if (!scanner || sn >= p.N) return;
  // Epilogue: alpha, bias, output rounding (src/tricast/reference/mma.py:376-384).
  float acc = c;
  if (p.alpha_a || p.alpha_b) {
    float alpha = p.alpha_a ? *p.alpha_a : 1.0f;
    if (p.alpha_b) alpha = p.alpha_a ? __fmul_rn(alpha, *p.alpha_b) : *p.alpha_b;
    acc = __fmul_rn(alpha, acc);
  }
  if (p.bias) acc = __fadd_rn(acc, p.bias[sn]);
  if (!p.out_plain) acc = cast_to(acc, p.of, TC_RNE, false, 0u, 32);
  store_container(p.out, p.out_dt, (int64_t)sm * p.N + sn, acc);
}

}  // namespace gemv

// ---------------------------------------------------------------- host side
struct Fp4GemvPlan {
  int64_t ngroups, ngroups_pad;
  int mp;
  size_t off_q, off_m, off_s, off_flag, total;
};

static Fp4GemvPlan plan_fp4_gemv(const GemmDesc &g) {
  Fp4GemvPlan p;
  p.ngroups = (g.K + fp4::kGS - 1) / fp4::kGS;
  p.ngroups_pad = (p.ngroups + gemv::kGroups - 1) / gemv::kGroups * gemv::kGroups;
  p.mp = 1;
  while (p.mp < g.M) p.mp *= 2;
  const size_t recs = (size_t)p.ngroups_pad * p.mp;
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  p.off_q = 0;
  p.off_m = up(recs * 16);
  p.off_s = p.off_m + up(recs * 16);
  p.off_flag = p.off_s + up(recs * 4);
  p.total = p.off_flag + 256;
  return p;
}

size_t fp4_gemv_workspace(const GemmDesc &g) { return plan_fp4_gemv(g).total; }

template <int DT, bool RNE>
static int launch_fp4_gemv_kernel(const gemv::Fp4Args &a, cudaStream_t s) {
  const size_t smem = 2 * (size_t)a.M * gemv::kDRow * sizeof(int32_t) + 3 * (size_t)gemv::kGroups * a.mp * 20;
  cudaError_t e = cudaFuncSetAttribute(gemv::gdfs_fp4_gemv_kernel<DT, RNE>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(std::string("gdfs fp4 gemv: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  const unsigned grid = (unsigned)((a.N + gemv::kCols - 1) / gemv::kCols);
  gemv::gdfs_fp4_gemv_kernel<DT, RNE><<<grid, gemv::kThreads, smem, s>>>(a);
  count_launch();
  return TC_OK;
}

template <int DT>
static int launch_fp4_gemv_dt(const gemv::Fp4Args &a, bool rne, cudaStream_t s) {
  return rne ? launch_fp4_gemv_kernel<DT, true>(a, s) : launch_fp4_gemv_kernel<DT, false>(a, s);
}

// GDFS-FP4 for M <= 16 (the caller checked the tiled kernel's preconditions: E2M1 operands, G >= 6,
// group size 16, K scales per multiple of 16, 23 <= F <= 48).
int launch_fp4_gemv(const GemmDesc &g, int ng, void *workspace, size_t workspace_bytes, cudaStream_t s) {
  const Fp4GemvPlan p = plan_fp4_gemv(g);
  if (!workspace || workspace_bytes < p.total) return set_error("tc_gemm: workspace too small"), TC_WORKSPACE_TOO_SMALL;
  if (g.N > ((int64_t)1 << 36)) return TC_UNSUPPORTED;
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
    const int64_t blocks = std::min<int64_t>((work + 255) / 256, 148 * 16);
    fp4::encode_fp4_kernel<<<(unsigned)blocks, 256, 0, s>>>(e);
    count_launch();
  }
  gemv::Fp4Args a;
  std::memset(&a, 0, sizeof(a));
  a.aq = reinterpret_cast<const uint4 *>(ws + p.off_q);
  a.am = reinterpret_cast<const uint4 *>(ws + p.off_m);
  a.as = reinterpret_cast<const uint32_t *>(ws + p.off_s);
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
  a.mp = p.mp;
  a.ng = ng;
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
  a.flag = flag;
  int st;
  switch (g.b.dt) {
    case TC_F32: st = launch_fp4_gemv_dt<TC_F32>(a, g.rne, s); break;
    case TC_BF16: st = launch_fp4_gemv_dt<TC_BF16>(a, g.rne, s); break;
    default: st = launch_fp4_gemv_dt<TC_F16>(a, g.rne, s); break;
  }
  if (st) return st;
  launch_generic(g, flag, s);  // runs only when an operand raised the flag
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm gemv: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

}  // namespace tc
