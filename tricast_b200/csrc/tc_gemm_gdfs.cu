// Fast GDFS kernel for narrow float grids (FP8 / FP6 operands, or FP4 outside the E2M1 tensor-core
// path), e.g. TriCast's own benchmark row "GDFS G=32 F=25 GS=16" on FP8 E4M3
// (scripts/bench/bench_mma_vs_nadpe.py:31-32).
//
// Reference: TriCast src/tricast/reference/mma.py:318-336 (_gdfs) with _sum_terms (:104-115),
// _apply_scales (:255-277) and _fda (:140-151). Per K tile of KT = NG * GS elements and output (m, n):
//   * each group g of GS products is summed at radix G, aligned to its largest exponent label
//     emax_g (the labels of its non-zero products) with truncation:
//         S_g = sum_k sign_k * floor(|a_k b_k| * 2**(G - emax_g))
//     (the product significand shifted from radix ra + rb to G, then right by emax_g - e_k: two
//     truncating shifts of a non-negative integer compose into one floor);
//   * the group becomes a term (sign, exponent emax_g, |S_g|) re-radixed to F by a truncating shift,
//     and the tile's FDA at radix F aligns the group terms and the running value c to their largest
//     exponent emax_t (zero terms take no part) with truncation:
//         total = sign_c * floor(|c| * 2**(F - emax_t)) + sum_g sign_g * floor(|S_g| * 2**(F - G + emax_g - emax_t))
//     (again the re-radix and the alignment compose into one floor);
//   * total is normalised by the fixed-point -> fp32 rule at radix F.
//
// Every quantity is an exact fp64 value: products of two narrow grid values have at most 8
// significant bits; each aligned product is below 2**(G + 2) and their sum below GS * 2**(G + 2) <=
// 2**53, each aligned group term below GS * 2**(F + 2) and the total below 2**53 (the plan checks
// G + 2 + log2 GS <= 53 and F + 3 + log2(NG * GS) <= 53). Each floor is the fma.rz magic of
// Acc<double>::trunc. emax_t is taken from the running value and from every group that has a non-zero
// product; a group whose aligned sum cancels to exactly zero takes no part in the reference's FDA, so
// an output where that changes emax_t redoes its tile step with the true emax_t (rare).
//
// No truncation: a non-zero product is sig * 2**(e_k - ma - mb) with an integer significand product
// (ma, mb the operands' mantissa bits), so floor(|P_k| * 2**(G - emax_g)) drops nothing when
// emax_g - e_k <= G - ma - mb. A thread checks that bound for each of its outputs and groups from the
// group's largest product label and the smallest non-zero labels of its rows and columns (kept per
// (row, group) by min_label_kernel); when all 32 lanes pass, the group's sum is the exact fp64 sum of
// its products (one FMA each: at most G + 2 + log2 GS <= 53 significant bits), and its tile term
// floor(|sum| * 2**(F - emax_t)) is the same as that of the aligned sum. Otherwise every product is
// truncated as above.
//
// Operands are staged as the CoFDA kernel's are (tc_cofda_tile.cuh) with one chunk per group: values
// in fp64 and packed int16 labels, power-of-two K scales constant over a group folded in at encode
// time (equal to GDFS's group-level exponent add). Anything else goes to the exact generic kernel.
#include <cstring>
#include <string>

#include "tc_cofda_tile.cuh"

namespace tc {
namespace gdfs {

using cofda::Acc;
using cofda::kTile;
using cofda::kZeroExp;
using cofda::load4;

constexpr int kNoLabel = 0x7FFF;  // smallest label of a row or column with no non-zero element

// One group's stage: the tile layout's values and labels, plus each row's and column's smallest
// non-zero label in the group.
template <int GS>
struct GStage {
  double av[GS][kTile];
  double bv[GS][kTile];
  uint32_t be[GS][kTile];
  uint32_t ae[GS][kTile / 2];
  int16_t amin[kTile];
  int16_t bmin[kTile];
};

// Per (row tile, chunk, row): the smallest label among the row's non-zero elements of the chunk
// (kNoLabel when it has none), from the encoded labels (A: row pairs, B: duplicated halves).
__global__ void __launch_bounds__(256) min_label_kernel(const uint32_t *__restrict__ exp, int side, int64_t rows_pad,
                                                        int64_t nchunks, int CS, int16_t *__restrict__ out) {
  const int64_t total = rows_pad * nchunks;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(idx % kTile);
    const int64_t tc = idx / kTile;  // row tile * nchunks + chunk
    int mn = kNoLabel;
    for (int kk = 0; kk < CS; ++kk) {
      const int64_t base = (tc * CS + kk) * kTile;
      const uint32_t w = side == 0 ? exp[base / 2 + r / 2] >> ((r & 1) * 16) : exp[base + r];
      const int lab = (int)(int16_t)(w & 0xFFFFu);
      if (lab != kZeroExp) mn = min(mn, lab);
    }
    out[idx] = (int16_t)mn;
  }
}

// Output (i, j)'s label from the packed pair of rows (2q, 2q + 1) of pass 1. A product with a zero
// element carries kZeroExp plus the other element's label (at most a few hundred above kZeroExp,
// far below any real label): a group with no non-zero product reads as kZeroExp.
__device__ __forceinline__ int emax_of(const uint32_t (&e)[2][4], int i, int j) {
  const uint32_t w = e[i >> 1][j];
  const int v = (int)(int16_t)((i & 1) ? (w >> 16) : (w & 0xFFFFu));
  return v < kZeroExp / 2 ? kZeroExp : v;
}

// The tile step of one output redone with the true tile exponent (a group whose aligned sum cancelled
// to zero had set it): every group's sum recomputed from the staged operands, only the non-zero ones
// and the running value taking part. Rare, so kept out of line.
template <int GS, int NG, bool RNE>
__device__ __noinline__ float redo_tile(const GStage<GS> *stages, int64_t c0, int i, int j, int tx, int ty,
                                        float c, int4 egs, int F, int G) {
  constexpr int kSt = 2 * NG;
  const int egv[4] = {egs.x, egs.y, egs.z, egs.w};
  double sums[NG];
  int et = cofda::running_exp(c);
  for (int gg = 0; gg < NG; ++gg) {
    const GStage<GS> &st = stages[(c0 + gg) % kSt];
    const int eg = egv[gg];
    const double S = Acc<double>::pow2(G - eg);
    double sum = 0.0;
    for (int kk = 0; kk < GS; ++kk)
      sum = __dadd_rn(sum, Acc<double>::trunc(__dmul_rn(st.av[kk][ty * 4 + i], st.bv[kk][cofda::bcol<double>(tx * 4 + j)]), S));
    sums[gg] = sum;
    if (sum != 0.0) et = max(et, eg);
  }
  if (et == kZeroExp) return c;  // no term takes part: the running value stays
  double total = Acc<double>::running(c, F, et, Acc<double>::pow2(F - et));
  for (int gg = 0; gg < NG; ++gg)
    total = __dadd_rn(total, Acc<double>::trunc(sums[gg], Acc<double>::pow2(F - G + egv[gg] - et)));
  return Acc<double>::finish(total, et, F, RNE);
}

struct Args {
  const double *av, *bv;
  const uint32_t *ae, *be;
  const int16_t *amin, *bmin;  // [tile][chunk][kTile]: smallest non-zero label per row / column
  int64_t M, N, ntiles;
  int F, G, span;              // span = G - ma - mb: the label distance below emax_g kept exactly
  GemmDesc g;
  const int32_t *flag;
  int32_t *status;
  int wait_polls;
};

template <int GS, int NG, bool RNE>
__global__ void __launch_bounds__(256) gdfs_kernel(Args p) {
  if (*p.flag) return;
  constexpr int kSt = 2 * NG;  // the stages of two K tiles: one being scanned, one in flight
  using Stage = GStage<GS>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Stage *stages = reinterpret_cast<Stage *>(smem_raw);
  __shared__ __align__(8) uint64_t full[kSt];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t mt = blockIdx.y, nt = blockIdx.x;
  const int64_t m0 = mt * kTile, n0 = nt * kTile;
  constexpr uint32_t kValBytes = GS * kTile * 8;
  constexpr uint32_t kBexpBytes = GS * kTile * 4;
  constexpr uint32_t kAexpBytes = GS * (kTile / 2) * 4;
  constexpr uint32_t kMinBytes = kTile * 2;
  constexpr uint32_t kStageBytes = 2 * kValBytes + kBexpBytes + kAexpBytes + 2 * kMinBytes;
  const int64_t nchunks = p.ntiles * NG;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSt; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int64_t c) {
    const int s = (int)(c % kSt);
    Stage &st = stages[s];
    mbar_expect_tx(&full[s], kStageBytes);
    const int64_t a_off = (mt * nchunks + c) * GS * kTile;
    const int64_t b_off = (nt * nchunks + c) * GS * kTile;
    bulk_g2s(&st.av[0][0], p.av + a_off, kValBytes, &full[s]);
    bulk_g2s(&st.ae[0][0], p.ae + a_off / 2, kAexpBytes, &full[s]);
    bulk_g2s(&st.bv[0][0], p.bv + b_off, kValBytes, &full[s]);
    bulk_g2s(&st.be[0][0], p.be + b_off, kBexpBytes, &full[s]);
    bulk_g2s(&st.amin[0], p.amin + (mt * nchunks + c) * kTile, kMinBytes, &full[s]);
    bulk_g2s(&st.bmin[0], p.bmin + (nt * nchunks + c) * kTile, kMinBytes, &full[s]);
  };
  if (threadIdx.x == 0)
    for (int64_t c = 0; c < kSt && c < nchunks; ++c) issue(c);

  float c[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0.0f;
  const int F = p.F, G = p.G;

  for (int64_t t = 0; t < p.ntiles; ++t) {
    const int64_t c0 = t * NG;
    bool timed_out = false;
#pragma unroll
    for (int gg = 0; gg < NG; ++gg)
      if (!mbar_wait(&full[(c0 + gg) % kSt], (uint32_t)(((c0 + gg) / kSt) & 1), p.wait_polls)) timed_out = true;
    if (__syncthreads_or(timed_out)) {
      if (threadIdx.x == 0) {
        atomicExch(p.status, 1);
        // Chunks c0 .. c0 + kSt - 1 may still be in flight: they land before the CTA exits.
        for (int64_t u = c0; u < c0 + kSt && u < nchunks; ++u) mbar_wait(&full[u % kSt], (uint32_t)((u / kSt) & 1));
      }
      return;
    }
    // Pass 1: each group's largest label, two rows per 16-bit half.
    uint32_t em2[NG][2][4];
#pragma unroll
    for (int gg = 0; gg < NG; ++gg) {
      const Stage &st = stages[(c0 + gg) % kSt];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int j = 0; j < 4; ++j) em2[gg][q][j] = ((uint32_t)kZeroExp & 0xFFFFu) | ((uint32_t)kZeroExp << 16);
#pragma unroll 8
      for (int kk = 0; kk < GS; ++kk) {
        const uint2 ea = *reinterpret_cast<const uint2 *>(&st.ae[kk][ty * 2]);
        const uint4 eb = *reinterpret_cast<const uint4 *>(&st.be[kk][tx * 4]);
        const uint32_t ebs[4] = {eb.x, eb.y, eb.z, eb.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          em2[gg][0][j] = __viaddmax_s16x2(ea.x, ebs[j], em2[gg][0][j]);
          em2[gg][1][j] = __viaddmax_s16x2(ea.y, ebs[j], em2[gg][1][j]);
        }
      }
    }
    // The tile's exponent, taking every group with a non-zero product and the running value.
    int et[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        int e = cofda::running_exp(c[i][j]);
#pragma unroll
        for (int gg = 0; gg < NG; ++gg) e = max(e, emax_of(em2[gg], i, j));
        et[i][j] = e;
      }
    // Pass 2: each group's exact aligned sum at radix G, folded into the tile total at radix F.
    double total[4][4];
    // Bit i * 4 + j: output (i, j)'s tile exponent is attained by a term that takes part (its running
    // value, or a group whose sum is non-zero); otherwise the true exponent is smaller (a redo).
    uint32_t held = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        total[i][j] = Acc<double>::running(c[i][j], F, et[i][j], Acc<double>::pow2(F - et[i][j]));
        held |= (uint32_t)(cofda::running_exp(c[i][j]) == et[i][j]) << (i * 4 + j);
      }
#pragma unroll
    for (int gg = 0; gg < NG; ++gg) {
      const Stage &st = stages[(c0 + gg) % kSt];
      double sum[4][4];
      bool exact = true;  // no product of this thread's outputs is truncated at radix G
      {
        const uint2 am = *reinterpret_cast<const uint2 *>(&st.amin[ty * 4]);
        const uint2 bm = *reinterpret_cast<const uint2 *>(&st.bmin[tx * 4]);
        const int ra[4] = {(int)(int16_t)(am.x & 0xFFFFu), (int)(int16_t)(am.x >> 16), (int)(int16_t)(am.y & 0xFFFFu),
                           (int)(int16_t)(am.y >> 16)};
        const int cb[4] = {(int)(int16_t)(bm.x & 0xFFFFu), (int)(int16_t)(bm.x >> 16), (int)(int16_t)(bm.y & 0xFFFFu),
                           (int)(int16_t)(bm.y >> 16)};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) exact &= emax_of(em2[gg], i, j) - ra[i] - cb[j] <= p.span;
      }
      if (__all_sync(0xFFFFFFFFu, exact)) {
        // The exact sum of the products: the aligned sum at radix G times 2**(emax_g - G).
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) sum[i][j] = 0.0;
#pragma unroll 4
        for (int kk = 0; kk < GS; ++kk) {
          double as[4], bs[4];
          load4<double>(&st.av[kk][ty * 4], as);
          cofda::load_b4<double>(&st.bv[kk][0], tx, bs);
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sum[i][j] = __fma_rn(as[i], bs[j], sum[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int eg = emax_of(em2[gg], i, j);
            total[i][j] = __dadd_rn(total[i][j], Acc<double>::trunc(sum[i][j], Acc<double>::pow2(F - et[i][j])));
            held |= (uint32_t)((sum[i][j] != 0.0) & (eg == et[i][j])) << (i * 4 + j);
          }
      } else {
        double S[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            S[i][j] = Acc<double>::pow2(G - emax_of(em2[gg], i, j));
            sum[i][j] = 0.0;
          }
#pragma unroll 4
        for (int kk = 0; kk < GS; ++kk) {
          double as[4], bs[4];
          load4<double>(&st.av[kk][ty * 4], as);
          cofda::load_b4<double>(&st.bv[kk][0], tx, bs);
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
              sum[i][j] = __dadd_rn(sum[i][j], Acc<double>::trunc(__dmul_rn(as[i], bs[j]), S[i][j]));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int eg = emax_of(em2[gg], i, j);
            total[i][j] = __dadd_rn(total[i][j], Acc<double>::trunc(sum[i][j], Acc<double>::pow2(F - G + eg - et[i][j])));
            held |= (uint32_t)((sum[i][j] != 0.0) & (eg == et[i][j])) << (i * 4 + j);
          }
      }
    }
    // Normalise; an output whose tile exponent came only from groups that cancelled to zero redoes
    // its step with the true exponent. An overflowed running value is sticky (operands are finite).
    uint32_t redo = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool same_et = (held >> (i * 4 + j)) & 1u;
        const bool sticky = (f2u(c[i][j]) & 0x7FFFFFFFu) >= kInf;
        redo |= (uint32_t)(!same_et && !sticky) << (i * 4 + j);
        if (!sticky && same_et && et[i][j] != kZeroExp)
          c[i][j] = Acc<double>::finish(total[i][j], et[i][j], F, RNE);
      }
    if (redo) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if ((redo >> (i * 4 + j)) & 1u) {
            int eg[4] = {kZeroExp, kZeroExp, kZeroExp, kZeroExp};
#pragma unroll
            for (int gg = 0; gg < NG; ++gg) eg[gg] = emax_of(em2[gg], i, j);
            c[i][j] = redo_tile<GS, NG, RNE>(stages, c0, i, j, tx, ty, c[i][j], make_int4(eg[0], eg[1], eg[2], eg[3]), F,
                                             G);
          }
    }
    __syncthreads();
    // The stages of this tile are free: refill them with tile t + 2.
    if (threadIdx.x == 0)
      for (int gg = 0; gg < NG; ++gg)
        if (c0 + kSt + gg < nchunks) issue(c0 + kSt + gg);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m >= p.M || n >= p.N) continue;
      store_out(p.g, m, n, epilogue(p.g, m, n, c[i][j]));
    }
}

}  // namespace gdfs

// ---------------------------------------------------------------- host side
using cofda::kTile;

struct GdfsPlan {
  bool ok;
  int GS, NG;
  int64_t ntiles, a_pad, b_pad;
  size_t off[6], flag_off, total;  // A values, A labels, B values, B labels, A / B smallest labels
};

static int bit_length(int64_t v) {
  int b = 0;
  while (v >> b) ++b;
  return b;
}

static GdfsPlan plan_gdfs(const GemmDesc &g) {
  GdfsPlan p;
  std::memset(&p, 0, sizeof(p));
  if (g.alg != ALG_GDFS) return p;
  if (!cofda::narrow_float(g.a.f) || !cofda::narrow_float(g.b.f)) return p;
  if (g.GS != 8 && g.GS != 16 && g.GS != 32) return p;
  if (g.KT % g.GS) return p;
  const int ng = g.KT / g.GS;
  if (ng != 1 && ng != 2 && ng != 4) return p;
  if ((size_t)2 * ng * (sizeof(gdfs::GStage<32>) * g.GS / 32 + 256) > 200 * 1024) return p;
  if (g.G < 1 || g.G + 2 + bit_length(g.GS) > 53) return p;           // exact group sums in fp64
  if (g.F < 1 || g.F + 3 + bit_length(ng * g.GS) > 53) return p;      // exact tile totals in fp64
  if (g.apply == AP_GROUP) {
    // K scales: powers of two constant over each group fold into the operands (the group-level
    // exponent add of mma.py:268-277); scale significands would multiply the group sums.
    for (const OpDesc *o : {&g.a, &g.b})
      if (o->skind == SK_K && (o->sf.kind != 2 || o->kd % g.GS)) return p;
  } else if (g.apply != AP_EPILOGUE) {
    return p;
  }
  p.GS = g.GS;
  p.NG = ng;
  p.ntiles = (g.K + g.KT - 1) / g.KT;
  p.a_pad = (g.M + kTile - 1) / kTile * kTile;
  p.b_pad = (g.N + kTile - 1) / kTile * kTile;
  const int64_t nchunks = p.ntiles * ng;
  const size_t ka = (size_t)p.a_pad * nchunks * g.GS, kb = (size_t)p.b_pad * nchunks * g.GS;
  const size_t sizes[6] = {ka * 8, ka * 2, kb * 8, kb * 4, (size_t)p.a_pad * nchunks * 2, (size_t)p.b_pad * nchunks * 2};
  size_t off = 0;
  for (int i = 0; i < 6; ++i) {
    p.off[i] = off;
    off += (sizes[i] + 255) & ~(size_t)255;
  }
  p.flag_off = off;
  p.total = off + 256;
  p.ok = true;
  return p;
}

size_t gdfs_workspace(const GemmDesc &g) {
  const GdfsPlan p = plan_gdfs(g);
  return p.ok ? p.total : 0;
}

template <int GS, int NG, bool RNE>
static int launch_gdfs_kernel(const gdfs::Args &a, cudaStream_t s) {
  const size_t smem = sizeof(gdfs::GStage<GS>) * 2 * NG;
  cudaError_t e = cudaFuncSetAttribute(gdfs::gdfs_kernel<GS, NG, RNE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return set_error(std::string("gdfs: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  dim3 grid((unsigned)((a.N + kTile - 1) / kTile), (unsigned)((a.M + kTile - 1) / kTile));
  gdfs::gdfs_kernel<GS, NG, RNE><<<grid, 256, smem, s>>>(a);
  count_launch();
  return TC_OK;
}

template <int GS, bool RNE>
static int launch_gdfs_ng(const gdfs::Args &a, int ng, cudaStream_t s) {
  if (ng == 1) return launch_gdfs_kernel<GS, 1, RNE>(a, s);
  if (ng == 2) return launch_gdfs_kernel<GS, 2, RNE>(a, s);
  return launch_gdfs_kernel<GS, 4, RNE>(a, s);
}

template <bool RNE>
static int launch_gdfs_gs(const gdfs::Args &a, int gs, int ng, cudaStream_t s) {
  if (gs == 8) return launch_gdfs_ng<8, RNE>(a, ng, s);
  if (gs == 16) return launch_gdfs_ng<16, RNE>(a, ng, s);
  return launch_gdfs_ng<32, RNE>(a, ng, s);
}

int launch_gdfs(const GemmDesc &g, void *workspace, size_t workspace_bytes, cudaStream_t s) {
  const GdfsPlan p = plan_gdfs(g);
  if (!p.ok) return TC_UNSUPPORTED;
  if (!workspace || workspace_bytes < p.total) return set_error("tc_gemm: workspace too small"), TC_WORKSPACE_TOO_SMALL;
  if ((g.M + kTile - 1) / kTile > 65535) return TC_UNSUPPORTED;
  char *ws = static_cast<char *>(workspace);
  int32_t *flag = reinterpret_cast<int32_t *>(ws + p.flag_off);
  cudaMemsetAsync(flag, 0, 2 * sizeof(int32_t), s);  // [0] operands rejected, [1] a wait ran out
  const int64_t nchunks = p.ntiles * p.NG;
  for (int side = 0; side < 2; ++side) {
    const OpDesc &o = side ? g.b : g.a;
    cofda::EncodeArgs e;
    std::memset(&e, 0, sizeof(e));
    e.v = o.v;
    e.dt = o.dt;
    e.rows = o.rows;
    e.K = o.K;
    e.rows_pad = side ? p.b_pad : p.a_pad;
    e.nchunks = nchunks;
    e.CS = p.GS;
    e.f = o.f;
    e.scale = (g.apply == AP_GROUP && o.skind == SK_K) ? o.scale : nullptr;
    e.nkd = o.nkd;
    e.kd = o.kd;
    e.sf = o.sf;
    e.field0 = o.field0;
    e.val = ws + p.off[side * 2];
    e.exp = reinterpret_cast<uint32_t *>(ws + p.off[side * 2 + 1]);
    e.side = side;
    e.flag = flag;
    const int64_t work = e.rows_pad / 2 * nchunks * p.GS;
    const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 16);
    cofda::encode_kernel<double><<<(unsigned)blocks, 256, 0, s>>>(e);
    count_launch();
    const int64_t rows = e.rows_pad * nchunks;
    const int64_t mblocks = std::min<int64_t>((rows + 255) / 256, (int64_t)sm_count() * 16);
    gdfs::min_label_kernel<<<(unsigned)mblocks, 256, 0, s>>>(e.exp, side, e.rows_pad, nchunks, p.GS,
                                                             reinterpret_cast<int16_t *>(ws + p.off[4 + side]));
    count_launch();
  }
  gdfs::Args a;
  std::memset(&a, 0, sizeof(a));
  a.av = reinterpret_cast<const double *>(ws + p.off[0]);
  a.ae = reinterpret_cast<const uint32_t *>(ws + p.off[1]);
  a.bv = reinterpret_cast<const double *>(ws + p.off[2]);
  a.be = reinterpret_cast<const uint32_t *>(ws + p.off[3]);
  a.amin = reinterpret_cast<const int16_t *>(ws + p.off[4]);
  a.bmin = reinterpret_cast<const int16_t *>(ws + p.off[5]);
  a.M = g.M;
  a.N = g.N;
  a.ntiles = p.ntiles;
  a.F = g.F;
  a.G = g.G;
  a.span = g.G - g.a.f.mbits - g.b.f.mbits;
  a.g = g;
  a.flag = flag;
  a.status = flag + 1;
  a.wait_polls = wait_polls();
  const int st = g.rne ? launch_gdfs_gs<true>(a, p.GS, p.NG, s) : launch_gdfs_gs<false>(a, p.GS, p.NG, s);
  if (st) return st;
  launch_generic(g, flag, s);  // runs only when an operand raised the flag or a wait ran out
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm gdfs: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

}  // namespace tc
