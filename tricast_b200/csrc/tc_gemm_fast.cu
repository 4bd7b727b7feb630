// Fast emulated-GEMM kernels for the accumulation models the benchmark configurations use.
//
// GDFS with E2M1 x E2M1 operands and G >= 6 (the nvidia_blackwell_fp4 preset on NVFP4 / MXFP4
// operands). Exactness argument (TriCast src/tricast/reference/mma.py:318-336): an E2M1 value is
// m * 2**(e - 1) with m in {1, 2, 3} and e in {0, 1, 2}, so a product's decoded exponent is
// ea + eb in [0, 4] and its significand m_a*m_b sits at radix 2. Moved to radix G and aligned to the
// group maximum ge with a truncating right shift of ge - e <= 4 <= G - 2 bits, no product loses a
// bit. The group sum is therefore S = 2**(G - 2 - ge) * D with D = sum (2a)(2b) the exact integer
// dot product of the doubled codes (DP4A on int8 codes), and the group's aligned contribution to
// the tile FDA at radix F is
//     floor(|D| * ms_a * ms_b * 2**(F - 2 - srad + es_a + es_b - emax))
// where (es, ms) are the decoded K-scale terms at radix srad and emax is the largest exponent
// label ge + es_a + es_b over the tile's non-zero groups and the running value. ge itself only
// enters through emax; it is the largest i + j such that some k has an A element of exponent
// class >= i and a B element of class >= j, found with a few 16-bit mask ANDs per group.
//
// One pass. Bound the labels from above per row and column of the tile: L = es + (largest exponent
// class of that operand's group), emax'' = max(running exponent, max_g L_a + max_g L_b) >= emax. If
// every group's value sx * 2**(es_a + es_b - srad - 2) (sx = D * ms_a * ms_b, |sx| < 2**20) is a
// multiple of 2**(emax'' - F) (min_g es_a + min_g es_b - srad - 2 >= emax'' - F) and the running
// value's bits survive the alignment (emax'' - e_c <= F - 23), then no term is truncated under
// emax'' nor under emax, and the radix-F sum is the exact sum of the values. That sum is formed in
// integers: relative to the row's and column's smallest scale exponents each group contributes
// D * (ms_a << (es_a - min es_a)) * (ms_b << (es_b - min es_b)), two multiply-adds into an int64
// (the exponent spread is checked to keep it below 2**45); once per tile the int64 becomes an fp64
// (exact), is scaled by 2**(min es_a + min es_b - srad - 2) and added to the running value (exact for
// F <= 48), and the result rounded toward zero to fp32 is the FDA normalisation (min(F, 23) = 23
// fraction bits, subnormals truncated). A thread whose tile fails a check redoes its outputs for that
// tile with the exact two-pass integer labels and sums (mask records read from global memory), so the
// result is always the reference's.
//
// Operands are first encoded (encode_fp4_kernel) into 16-byte records per (K tile, group, row):
// the sixteen int8 codes, the exponent-class masks, and the scale word. The GEMM kernel stages the
// records of a 64-row x 64-column CTA tile through shared memory with 1-D TMA bulk copies
// (cp.async.bulk, no multicast) completing on mbarriers, in a multi-stage ring. Every wait is
// bounded; a timeout sets the device status word and the kernel returns.
//
// Any operand value or scale the fast path cannot take (NaN/Inf, off-grid values, wide scale
// significands) raises a device flag during encoding; the fast kernel then writes nothing and the
// exact generic kernel, launched behind it on the same stream, computes the product instead.
#include <algorithm>
#include <cstring>
#include <string>

#include "tc_bulk.cuh"
#include "tc_fp4.cuh"

namespace tc {

namespace fp4 {

constexpr int kTileRows = 64;    // rows (A) / columns (B) per CTA
constexpr int kStages = 4;

__global__ void __launch_bounds__(256) encode_fp4_kernel(EncodeArgs e) {
  int64_t ngroups_row = e.ntiles * e.ng;
  int64_t total = ngroups_row * e.rows_pad;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  bool bad = false;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    int64_t gi = idx / e.rows_pad;       // group index along K
    int64_t r = idx % e.rows_pad;        // consecutive threads take consecutive rows
    int64_t k0 = gi * kGS;
    uint32_t codes[4] = {0, 0, 0, 0};
    uint32_t c0 = 0, c1 = 0, c2 = 0;     // exponent-class masks: >= 0 (nonzero), >= 1, >= 2
    uint32_t sword = pack_scale(0, 0, 0);
    if (r < e.rows && e.vec && k0 + kGS <= e.K && e.dt == TC_BF16) {
      // Whole group in bf16 containers: codes and exponent-class masks four elements at a time from
      // the bit patterns (e2m1_codes4_bf16_mag), no float conversion.
      const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(e.v) + r * e.K + k0);
      const uint4 u0 = src[0], u1 = src[1];
      const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      bool ok = true;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t mag, m0, m1, m2;
        codes[q] = e2m1_codes4_bf16_mag(w[2 * q], w[2 * q + 1], ok, mag);
        class_masks4(mag, m0, m1, m2);
        c0 |= m0 << (4 * q);
        c1 |= m1 << (4 * q);
        c2 |= m2 << (4 * q);
      }
      if (!ok) bad = true;
      bool zero = false;
      sword = e.scale ? group_scale_word(e.scale[r * e.nkd + k0 / e.kd], e.sf, e.field0, zero, bad) : pack_scale(0, 1, 0);
      if (zero) {
        codes[0] = codes[1] = codes[2] = codes[3] = 0;
        c0 = c1 = c2 = 0;
      }
      const uint32_t gemax = c2 ? 2u : c1 ? 1u : 0u;
      sword |= (gemax << 25) | ((c0 == 0 ? 1u : 0u) << 27);
    } else if (r < e.rows) {
      // The group's 16 inputs: vector loads when the whole group is in range and 16-byte aligned.
      float vin[kGS];
      if (e.vec && k0 + kGS <= e.K) {
        if (e.dt == TC_F32) {
          const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(e.v) + r * e.K + k0);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const float4 t4 = src[w];
            vin[4 * w] = t4.x; vin[4 * w + 1] = t4.y; vin[4 * w + 2] = t4.z; vin[4 * w + 3] = t4.w;
          }
        } else {
          const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(e.v) + r * e.K + k0);
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const uint4 u4 = src[w];
            const uint32_t uu[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              if (e.dt == TC_BF16) {
                vin[8 * w + 2 * h] = u2f(uu[h] << 16);
                vin[8 * w + 2 * h + 1] = u2f(uu[h] & 0xFFFF0000u);
              } else {
                vin[8 * w + 2 * h] = __half2float(__ushort_as_half((unsigned short)(uu[h] & 0xFFFF)));
                vin[8 * w + 2 * h + 1] = __half2float(__ushort_as_half((unsigned short)(uu[h] >> 16)));
              }
            }
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < kGS; ++j) vin[j] = k0 + j < e.K ? load_as_float(e.v, e.dt, r * e.K + k0 + j) : 0.0f;
      }
      uint4 qq;
      const int64_t left = e.K - k0;
      e2m1_codes(vin, left < kGS ? (int)left : kGS, qq, c0, c1, c2, bad);
      codes[0] = qq.x; codes[1] = qq.y; codes[2] = qq.z; codes[3] = qq.w;
      bool zero = false;
      // No K scale: es = 0, ms = 1. Groups past K (padding of the last tile) read no scale.
      sword = (e.scale && k0 < e.K) ? group_scale_word(e.scale[r * e.nkd + k0 / e.kd], e.sf, e.field0, zero, bad)
                                    : pack_scale(0, 1, 0);
      if (zero) {
        // A zero scale makes the whole group a zero term (the group rule of mma.py:270-276);
        // zero codes give D = 0 for every partner, so the group never enters emax.
        codes[0] = codes[1] = codes[2] = codes[3] = 0;
        c0 = c1 = c2 = 0;
      }
      const uint32_t gemax = c2 ? 2u : c1 ? 1u : 0u;
      sword |= (gemax << 25) | ((c0 == 0 ? 1u : 0u) << 27);
    } else {
      sword |= 1u << 27;  // padding rows are all-zero groups
    }
    uint4 q4 = make_uint4(codes[0], codes[1], codes[2], codes[3]);
    const uint4 m4 = e.side == 0 ? a_masks(c0, c1, c2) : b_masks(c0, c1, c2);
    e.q[idx] = q4;
    e.m[idx] = m4;
    e.s[idx] = sword;
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicExch(e.flag, 1);
}

// Per (K tile, row): the multipliers D is scaled by and the tile's bounds. For the tile's non-zero
// groups let minE = min es and L = max(es + largest exponent class); a group's multiplier is
// +-(ms << (es - minE)) (0 for an all-zero group). tw = {minE, L}: {kBig, kNone} when every group is
// zero, L = kBig when the exponent spread exceeds 11 (the multiplier bound), which forces the exact
// path for every output that uses the row.
//
// tcw (optional, for the tensor-core kernel): the tile words re-expressed so that the per-output tile
// step is a handful of adds and compares. For an output (row of A with {ea, la}, column of B with
// {eb, lb}) the single-pass conditions and the fp64 power are sums of a row part and a column part:
//   lo   = la + lb - (F - 23) + 127         row: la - (F - 23) + 127   column: lb
//   hi   = ea + eb + F - srad2 + 127        (stored as the span hi - lo, a row part plus a column part)
//   d    = (ea - la) + (eb - lb) - (srad2 - F)   row: ea - la - (srad2 - F)   column: eb - lb
//   p2   = 2**(ea + eb - srad2), its fp64 high word ((ea + eb - srad2 + 1023) << 20):
//          row: (ea' - srad2 + 1023) << 20   column: eb' << 20, with ea', eb' clamped to [-500, 500]
// so words are {lo part, span part, d part, p2 part}. The biased exponent be of the running value
// passes lo <= be <= hi iff (unsigned)(be - lo) <= (unsigned)(hi - lo) whenever d >= 0 (then
// hi - lo = d + F - 23 >= 0), which the step also requires. Scale exponents are within +-400 except
// for the all-zero sentinel, whose acc is 0, so the clamp changes no result and keeps the power a
// normal double.
__global__ void __launch_bounds__(256) tile_words_kernel(const uint32_t *__restrict__ sw, int64_t rows_pad,
                                                         int64_t ntiles, int ng, int32_t *__restrict__ mult,
                                                         int2 *__restrict__ tw, int4 *__restrict__ tcw, int side,
                                                         int F, int srad2) {
  const int64_t total = ntiles * rows_pad;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = idx / rows_pad, r = idx % rows_pad;
    int min_e = kBig, max_e = kNone, max_l = kNone;
    for (int gg = 0; gg < ng; ++gg) {
      const uint32_t w = sw[(t * ng + gg) * rows_pad + r];
      if ((w >> 27) & 1u) continue;
      const int es = (int)(w & 0xFFFFu) - 0x8000;
      min_e = min(min_e, es);
      max_e = max(max_e, es);
      max_l = max(max_l, es + (int)((w >> 25) & 3u));
    }
    const bool wide = min_e != kBig && max_e - min_e > 11;
    for (int gg = 0; gg < ng; ++gg) {
      const int64_t gi = (t * ng + gg) * rows_pad + r;
      const uint32_t w = sw[gi];
      int m = 0;
      if (!((w >> 27) & 1u) && !wide) {
        m = (int)((w >> 16) & 0xFFu) << ((int)(w & 0xFFFFu) - 0x8000 - min_e);
        if ((w >> 24) & 1u) m = -m;
      }
      mult[gi] = m;
    }
    const int ea = min_e, la = wide ? kBig : max_l;
    tw[idx] = make_int2(ea, la);
    if (tcw) {
      const int ec = min(max(ea, -500), 500);
      tcw[idx] = side == 0 ? make_int4(la - (F - 23) + 127, (ea + F - srad2 + 127) - (la - (F - 23) + 127),
                                       ea - la - (srad2 - F), (ec - srad2 + 1023) << 20)
                           : make_int4(la, ea - la, ea - la, ec << 20);
    }
  }
}

template <int NG>
struct Stage {
  uint4 aq[NG][kTileRows];
  uint4 bq[NG][kTileRows];
  int32_t amul[NG][kTileRows];
  int32_t bmul[NG][kTileRows];
  int2 atw[kTileRows];
  int2 btw[kTileRows];
};


// 256 threads as 16 x 16; thread (ty, tx) owns rows ty*4 + i and columns tx + 16*j of the tile.
template <int NG, bool RNE>
__global__ void __launch_bounds__(256, 2) gdfs_fp4_kernel(GemmArgs g) {
  if (*g.flag) return;  // the generic kernel takes over
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Stage<NG> *stages = reinterpret_cast<Stage<NG> *>(smem_raw);
  __shared__ __align__(8) uint64_t full[kStages];   // stage landed (bulk copies complete)
  __shared__ __align__(8) uint64_t empty[kStages];  // every warp is done with the stage
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * kTileRows, n0 = (int64_t)blockIdx.x * kTileRows;
  constexpr uint32_t kRec = kTileRows * sizeof(uint4);
  constexpr uint32_t kSw = kTileRows * sizeof(uint32_t);
  constexpr uint32_t kTw = kTileRows * sizeof(int2);
  constexpr uint32_t kStageBytes = NG * (2 * kRec + 2 * kSw) + 2 * kTw;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    fence_barrier_init();
  }
  __syncthreads();

  int64_t issued = 0;  // tiles handed to the copy engine (thread 0's count)
  auto issue = [&](int64_t t, int s) {
    issued = t + 1;
    Stage<NG> &st = stages[s];
    mbar_expect_tx(&full[s], kStageBytes);
    for (int gg = 0; gg < NG; ++gg) {
      int64_t ga = (t * NG + gg) * g.a_rows_pad + m0;
      int64_t gb = (t * NG + gg) * g.b_rows_pad + n0;
      bulk_g2s(st.aq[gg], g.aq + ga, kRec, &full[s]);
      bulk_g2s(st.amul[gg], g.amul + ga, kSw, &full[s]);
      bulk_g2s(st.bq[gg], g.bq + gb, kRec, &full[s]);
      bulk_g2s(st.bmul[gg], g.bmul + gb, kSw, &full[s]);
    }
    bulk_g2s(st.atw, g.atw + t * g.a_rows_pad + m0, kTw, &full[s]);
    bulk_g2s(st.btw, g.btw + t * g.b_rows_pad + n0, kTw, &full[s]);
  };
  if (threadIdx.x == 0)
    for (int s = 0; s < kStages && s < g.ntiles; ++s) issue(s, s);

  float c[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0.0f;

  // Warps run independently through the ring: a warp releases a stage on empty[s]; thread 0 refills
  // the stage of tile t - 1 once all eight warps have released it. Every wait is bounded; a warp
  // whose wait runs out sets the status word (the exact kernel behind this one then recomputes the
  // product) and leaves the loop.
  bool producer_ok = true;
  int64_t t = 0;
  for (; t < g.ntiles; ++t) {
    const int s = (int)(t % kStages);
    const bool landed = mbar_wait(&full[s], (uint32_t)((t / kStages) & 1), g.wait_polls);
    if (__any_sync(0xFFFFFFFFu, !landed)) {
      if ((threadIdx.x & 31) == 0) atomicExch(g.status, 1);
      break;
    }
    const Stage<NG> &st = stages[s];
    // Bounds from the tile words: rows i (A) and columns j (B) of this thread.
    int min_ea[4], max_la[4], min_eb[4], max_lb[4];
    int sep = kBig;  // min_i (min es_a - L_a) + min_j (min es_b - L_b), separable part of the check
    {
      int da = kBig, db = kBig;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int2 wa = st.atw[ty * 4 + k], wb = st.btw[tx + 16 * k];
        min_ea[k] = wa.x; max_la[k] = wa.y;
        min_eb[k] = wb.x; max_lb[k] = wb.y;
        da = min(da, wa.x - wa.y);
        db = min(db, wb.x - wb.y);
      }
      sep = da + db;
    }
    // No term truncated under emax'' = max(e_c, L_a + L_b): every group's value is a multiple of
    // 2**(emax'' - F) and the running value keeps its bits, i.e. (with e_c the running exponent)
    //   min es_a + min es_b - srad - 2 >= L_a + L_b - F      (separable: sep >= srad + 2 - F)
    //   L_a + L_b - (F - 23) <= e_c <= min es_a + min es_b + F - srad - 2   (running value non-zero)
    bool safe = sep >= g.srad2 - g.F;
    int64_t acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // In biased form: lo <= biased exponent of c <= hi, or c is zero / Inf / NaN. A subnormal
        // running value (biased exponent 0 < lo) takes the exact path.
        const uint32_t cb = f2u(c[i][j]) & 0x7FFFFFFFu;
        const int be = (int)(cb >> 23);
        const int lo = max(max_la[i] + max_lb[j] - (g.F - 23) + 127, 1);
        const int hi = min_ea[i] + min_eb[j] + g.F - g.srad2 + 127;
        safe &= (cb == 0) | (cb >= kInf) | ((be >= lo) & (be <= hi));
        acc[i][j] = 0;
      }
#pragma unroll 1
    for (int gg = 0; gg < NG; ++gg) {
      uint4 bq[4];
      int mb[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        bq[j] = st.bq[gg][tx + 16 * j];
        mb[j] = st.bmul[gg][tx + 16 * j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 aq = st.aq[gg][ty * 4 + i];
        const int ma = st.amul[gg][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += (int64_t)dot16(aq, bq[j]) * (int64_t)(ma * mb[j]);
      }
    }
    if (!safe) {
      // Exact two-pass labels and sums for this thread's outputs (mask records from global memory).
      int emax[4][4];
      int64_t total[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) emax[i][j] = running_exp(c[i][j]);
#pragma unroll 1
      for (int gg = 0; gg < NG; ++gg) {
        const int64_t grow = (t * NG + gg);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 aq = st.aq[gg][ty * 4 + i];
          const uint4 am = g.am[grow * g.a_rows_pad + m0 + ty * 4 + i];
          const int ea = scale_exp(g.as[grow * g.a_rows_pad + m0 + ty * 4 + i]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 bm = g.bm[grow * g.b_rows_pad + n0 + tx + 16 * j];
            const int d = dot16(aq, st.bq[gg][tx + 16 * j]);
            const int label = exp_class_max(am, bm) + ea + scale_exp(g.bs[grow * g.b_rows_pad + n0 + tx + 16 * j]);
            if (d != 0 && label > emax[i][j]) emax[i][j] = label;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) total[i][j] = running_term(c[i][j], g.F, emax[i][j]);
#pragma unroll 1
      for (int gg = 0; gg < NG; ++gg) {
        const int64_t grow = (t * NG + gg);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 aq = st.aq[gg][ty * 4 + i];
          const uint32_t sa = g.as[grow * g.a_rows_pad + m0 + ty * 4 + i];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t sbj = g.bs[grow * g.b_rows_pad + n0 + tx + 16 * j];
            const int d = dot16(aq, st.bq[gg][tx + 16 * j]);
            const uint32_t x = (uint32_t)(d < 0 ? -d : d) * (((sa >> 16) & 0xFFu) * ((sbj >> 16) & 0xFFu));
            const int sh = g.shift0 + scale_exp(sa) + scale_exp(sbj) - emax[i][j];
            // x < 2**20 and sh <= shift0 <= 40: (x << 40) >> (40 - sh) is the exact truncation.
            const int r = max(40 - sh, 0);  // sh > 40 only for d == 0 (x == 0)
            const uint64_t v = r >= 64 ? 0ull : (((uint64_t)x << 40) >> r);
            const bool neg = (d < 0) != (((sa ^ sbj) >> 24) & 1u);
            total[i][j] += neg ? -(int64_t)v : (int64_t)v;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t cb = f2u(c[i][j]) & 0x7FFFFFFFu;
          if (cb >= kInf || emax[i][j] == kNone) continue;  // sticky Inf/NaN; every term zero keeps c
          c[i][j] = fixed_to_fp32(total[i][j], emax[i][j], g.F, RNE, true);
        }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // c + acc * 2**(min es_a + min es_b - srad - 2), exact in fp64 (the clamp only matters for an
          // all-zero row or column, whose acc is 0).
          const int e2 = min(max(min_ea[i] + min_eb[j] - g.srad2, -1000), 1000);
          const double p2 = __hiloint2double((e2 + 1023) << 20, 0);
          const double v = __fma_rn((double)acc[i][j], p2, (double)c[i][j]);
          float r = (RNE && fabs(v) >= 0x1p-126) ? __double2float_rn(v) : __double2float_rz(v);
          r = fabs(v) >= 0x1p128 ? __int_as_float((int)((f2u(r) & 0x80000000u) | kInf)) : r;
          c[i][j] = (f2u(c[i][j]) & 0x7FFFFFFFu) >= kInf ? c[i][j] : r;  // Inf / NaN running value is sticky
        }
    }
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[s]);
    if (threadIdx.x == 0 && producer_ok && t >= 1 && t - 1 + kStages < g.ntiles) {
      const int sp = (int)((t - 1) % kStages);
      if (mbar_wait(&empty[sp], (uint32_t)(((t - 1) / kStages) & 1), g.wait_polls)) {
        issue(t - 1 + kStages, sp);
      } else {
        atomicExch(g.status, 1);
        producer_ok = false;
      }
    }
  }
  if (threadIdx.x == 0)
    for (int64_t u = t; u < issued; ++u)  // copies still in flight land before the CTA exits
      mbar_wait(&full[u % kStages], (uint32_t)((u / kStages) & 1));
  if (t < g.ntiles) return;  // a wait ran out: the exact kernel recomputes every output
  // Epilogue: alpha, bias, output rounding (src/tricast/reference/mma.py:376-384).
  float alpha = 1.0f;
  bool has_alpha = g.alpha_a || g.alpha_b;
  if (g.alpha_a) alpha = *g.alpha_a;
  if (g.alpha_b) alpha = g.alpha_a ? __fmul_rn(alpha, *g.alpha_b) : *g.alpha_b;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t m = m0 + ty * 4 + i, n = n0 + tx + 16 * j;
      if (m >= g.M || n >= g.N) continue;
      float acc = c[i][j];
      if (has_alpha) acc = __fmul_rn(alpha, acc);
      if (g.bias) acc = __fadd_rn(acc, g.bias[n]);
      if (!g.out_plain) acc = cast_to(acc, g.of, TC_RNE, false, 0u, 32);
      store_container(g.out, g.out_dt, m * g.N + n, acc);
    }
}

}  // namespace fp4

// ---------------------------------------------------------------- dispatch
struct Fp4Plan {
  bool ok;
  int ng;
  int64_t ntiles, a_pad, b_pad;
  // per side (A then B): codes, masks, scale words, multipliers, tile words; then the tensor-core
  // kernel's tile words of A and of B
  size_t off[12], bytes[12], flag_off, total;
};

static bool is_e2m1(const Fmt &f) { return f.kind == 0 && f.mbits == 1 && f.emin == 0 && f.emax == 2 && f.is_signed; }

static Fp4Plan plan_fp4(const GemmDesc &g) {
  Fp4Plan p;
  std::memset(&p, 0, sizeof(p));
  if (g.alg != ALG_GDFS || g.GS != fp4::kGS || g.G < 6 || g.KT % fp4::kGS) return p;
  if (!is_e2m1(g.a.f) || !is_e2m1(g.b.f)) return p;
  if (g.apply != AP_GROUP && (g.a.skind == SK_K || g.b.skind == SK_K)) return p;
  if (g.a.skind == SK_TENSOR || g.a.skind == SK_ROW || g.b.skind == SK_TENSOR || g.b.skind == SK_ROW) return p;
  if ((g.a.skind == SK_K && g.a.kd % fp4::kGS) || (g.b.skind == SK_K && g.b.kd % fp4::kGS)) return p;
  int srad = (g.a.skind == SK_K ? g.a.srad : 0) + (g.b.skind == SK_K ? g.b.srad : 0);
  int shift0 = g.F - 2 - srad;
  if (shift0 > 40 || shift0 < -20) return p;
  if (g.F < 23 || g.F > 48) return p;  // the fp64 single pass needs 23 <= F (normalisation) and F <= 48
  p.ng = g.KT / fp4::kGS;
  if (p.ng != 1 && p.ng != 2 && p.ng != 4 && p.ng != 8) return p;
  p.ntiles = (g.K + g.KT - 1) / g.KT;
  p.a_pad = (g.M + 127) / 128 * 128;  // whole 128-row tiles for the tensor-core kernel (64 for the DP4A one)
  p.b_pad = (g.N + fp4::kTileRows - 1) / fp4::kTileRows * fp4::kTileRows;
  int64_t ga = p.ntiles * p.ng * p.a_pad, gb = p.ntiles * p.ng * p.b_pad;
  size_t sizes[12] = {(size_t)ga * 16, (size_t)ga * 16, (size_t)ga * 4, (size_t)ga * 4, (size_t)(p.ntiles * p.a_pad) * 8,
                      (size_t)gb * 16, (size_t)gb * 16, (size_t)gb * 4, (size_t)gb * 4, (size_t)(p.ntiles * p.b_pad) * 8,
                      (size_t)(p.ntiles * p.a_pad) * 16, (size_t)(p.ntiles * p.b_pad) * 16};
  size_t off = 0;
  for (int i = 0; i < 12; ++i) {
    p.off[i] = off;
    p.bytes[i] = sizes[i];
    off += (sizes[i] + 255) & ~(size_t)255;
  }
  p.flag_off = off;
  p.total = off + 256;
  p.ok = true;
  return p;
}

size_t cofda_workspace(const GemmDesc &g);
int launch_cofda(const GemmDesc &g, void *workspace, size_t workspace_bytes, cudaStream_t s);

size_t int_workspace(const GemmDesc &g);
int launch_fma(const GemmDesc &g, cudaStream_t s);
size_t gdfs_workspace(const GemmDesc &g);
int launch_gdfs(const GemmDesc &g, void *workspace, size_t workspace_bytes, cudaStream_t s);
int launch_int(const GemmDesc &g, void *workspace, size_t workspace_bytes, cudaStream_t s);

int launch_fp4_gemm_tc(const fp4::GemmArgs &args, int ng, cudaStream_t s);
size_t fp4_gemv_workspace(const GemmDesc &g, int ng);
int launch_fp4_gemv(const GemmDesc &g, int ng, void *workspace, size_t workspace_bytes, cudaStream_t s);

// Decode shapes (at most this many rows of A) take the small-M kernels (tc_gemv.cu).
constexpr int64_t kGemvMaxM = 16;

size_t fast_workspace(const GemmDesc &g) {
  if (g.K == 0) return 0;  // no products: the generic kernel writes the epilogue of a zero sum
  Fp4Plan p = plan_fp4(g);
  if (p.ok) return g.M <= kGemvMaxM ? fp4_gemv_workspace(g, p.ng) : p.total;
  size_t w = int_workspace(g);
  if (!w) w = cofda_workspace(g);
  return w ? w : gdfs_workspace(g);
}

template <int NG, bool RNE>
static int launch_fp4_gemm_r(const fp4::GemmArgs &args, int64_t M, int64_t N, cudaStream_t s) {
  size_t smem = sizeof(fp4::Stage<NG>) * fp4::kStages;
  cudaError_t e =
      cudaFuncSetAttribute(fp4::gdfs_fp4_kernel<NG, RNE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(std::string("gdfs fp4: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  dim3 grid((unsigned)((N + fp4::kTileRows - 1) / fp4::kTileRows), (unsigned)((M + fp4::kTileRows - 1) / fp4::kTileRows));
  fp4::gdfs_fp4_kernel<NG, RNE><<<grid, 256, smem, s>>>(args);
  count_launch();
  return TC_OK;
}

template <int NG>
static int launch_fp4_gemm(const fp4::GemmArgs &args, int64_t M, int64_t N, cudaStream_t s) {
  return args.rne ? launch_fp4_gemm_r<NG, true>(args, M, N, s) : launch_fp4_gemm_r<NG, false>(args, M, N, s);
}

// One operand's GDFS-FP4 records: the encoder (codes, class masks, scale words) and the tile words
// (multipliers, tile bounds, the tensor-core kernel's tile words), into the given arrays.
static void encode_fp4_side(const GemmDesc &g, const Fp4Plan &p, int side, char *q, char *m, char *sw, char *mult,
                            char *tw, char *tcw, int32_t *flag, int srad2, cudaStream_t s) {
  const OpDesc &o = side ? g.b : g.a;
  fp4::EncodeArgs e;
  e.v = o.v;
  e.dt = o.dt;
  e.rows = o.rows;
  e.K = o.K;
  e.rows_pad = side ? p.b_pad : p.a_pad;
  e.ntiles = p.ntiles;
  e.ng = p.ng;
  e.scale = o.skind == SK_K ? o.scale : nullptr;
  e.nkd = o.nkd;
  e.kd = o.kd;
  e.sf = o.sf;
  e.field0 = o.field0;
  e.q = reinterpret_cast<uint4 *>(q);
  e.m = reinterpret_cast<uint4 *>(m);
  e.s = reinterpret_cast<uint32_t *>(sw);
  e.flag = flag;
  e.side = side;
  const int esz = o.dt == TC_F32 ? 4 : 2;
  e.vec = ((uintptr_t)o.v % 16 == 0) && ((o.K * esz) % 16 == 0);
  const int64_t work = p.ntiles * p.ng * e.rows_pad;
  const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 16);
  fp4::encode_fp4_kernel<<<(unsigned)blocks, 256, 0, s>>>(e);
  count_launch();
  const int64_t twork = p.ntiles * e.rows_pad;
  const int64_t tblocks = std::min<int64_t>((twork + 255) / 256, (int64_t)sm_count() * 16);
  fp4::tile_words_kernel<<<(unsigned)tblocks, 256, 0, s>>>(e.s, e.rows_pad, p.ntiles, p.ng,
                                                           reinterpret_cast<int32_t *>(mult), reinterpret_cast<int2 *>(tw),
                                                           reinterpret_cast<int4 *>(tcw), side, g.F, srad2);
  count_launch();
}

// A pre-encoded B of the tiled GDFS-FP4 path: B's records and tile words (the plan's B arrays and the
// tensor-core tile words of B), each 256-byte aligned, then a flag word set when B cannot be encoded.
struct Fp4BLayout {
  size_t off[6], flag_off, total;
};

static Fp4BLayout fp4_b_layout(const Fp4Plan &p) {
  Fp4BLayout l;
  const int idx[6] = {5, 6, 7, 8, 9, 11};
  size_t off = 0;
  for (int i = 0; i < 6; ++i) {
    l.off[i] = off;
    off += (p.bytes[idx[i]] + 255) & ~(size_t)255;
  }
  l.flag_off = off;
  l.total = off + 256;
  return l;
}

size_t cofda_encoded_b_bytes(const GemmDesc &g);
int cofda_encode_b(const GemmDesc &g, void *enc, cudaStream_t s);
int launch_cofda_encoded(const GemmDesc &g, const void *benc, void *workspace, size_t workspace_bytes,
                         cudaStream_t s);

static bool fp4_tiled_encodable(const GemmDesc &g, const Fp4Plan &p) {
  return p.ok && g.M > kGemvMaxM && p.ntiles * fp4::kTileRows <= ((int64_t)1 << 40);
}

size_t encoded_b_bytes(const GemmDesc &g) {
  if (g.K == 0) return 0;
  const Fp4Plan p = plan_fp4(g);
  if (p.ok) return fp4_tiled_encodable(g, p) ? fp4_b_layout(p).total : 0;
  if (int_workspace(g)) return 0;  // integer operands: encoded per call
  return cofda_encoded_b_bytes(g);
}

int encode_b(const GemmDesc &g, void *enc, size_t enc_bytes, cudaStream_t s) {
  const size_t need = encoded_b_bytes(g);
  if (!need) return set_error("tc_encode_b: this operand pair has no path that takes a pre-encoded B"), TC_UNSUPPORTED;
  if (!enc || enc_bytes < need) return set_error("tc_encode_b: buffer too small"), TC_INVALID_ARGUMENT;
  const Fp4Plan p = plan_fp4(g);
  if (!p.ok) return cofda_encode_b(g, enc, s);
  const Fp4BLayout l = fp4_b_layout(p);
  char *e = static_cast<char *>(enc);
  int32_t *flag = reinterpret_cast<int32_t *>(e + l.flag_off);
  cudaMemsetAsync(flag, 0, sizeof(int32_t), s);
  const int srad = (g.a.skind == SK_K ? g.a.srad : 0) + (g.b.skind == SK_K ? g.b.srad : 0);
  encode_fp4_side(g, p, 1, e + l.off[0], e + l.off[1], e + l.off[2], e + l.off[3], e + l.off[4], e + l.off[5], flag,
                  srad + 2, s);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(std::string("tc_encode_b: ") + cudaGetErrorString(err)), TC_CUDA_ERROR;
  return TC_OK;
}

int launch_fast_encoded(const GemmDesc &g, const void *benc, size_t enc_bytes, void *workspace, size_t workspace_bytes,
                        cudaStream_t s) {
  const size_t need = encoded_b_bytes(g);
  if (!need || enc_bytes != need || !benc)
    return set_error("tc_gemm_encoded: the encoded B was made for another operand pair, spec or row count"),
           TC_INVALID_ARGUMENT;
  const Fp4Plan p = plan_fp4(g);
  if (!p.ok) return launch_cofda_encoded(g, benc, workspace, workspace_bytes, s);
  return launch_fast(g, workspace, workspace_bytes, s, benc);
}

int launch_fast(const GemmDesc &g, void *workspace, size_t workspace_bytes, cudaStream_t s, const void *benc) {
  if (g.K == 0) return TC_UNSUPPORTED;  // bias-only outputs: the generic kernel
  Fp4Plan p = plan_fp4(g);
  if (!p.ok) {
    int st = launch_int(g, workspace, workspace_bytes, s);
    if (st != TC_UNSUPPORTED) return st;
    st = launch_cofda(g, workspace, workspace_bytes, s);
    if (st != TC_UNSUPPORTED) return st;
    st = launch_gdfs(g, workspace, workspace_bytes, s);
    if (st != TC_UNSUPPORTED) return st;
    return launch_fma(g, s);
  }
  if (g.M <= kGemvMaxM) return launch_fp4_gemv(g, p.ng, workspace, workspace_bytes, s);
  if (!workspace || workspace_bytes < p.total) return set_error("tc_gemm: workspace too small"), TC_WORKSPACE_TOO_SMALL;
  if (p.ntiles * fp4::kTileRows > (int64_t)1 << 40) return TC_UNSUPPORTED;
  char *ws = static_cast<char *>(workspace);
  int32_t *flag = reinterpret_cast<int32_t *>(ws + p.flag_off);
  cudaMemsetAsync(flag, 0, 2 * sizeof(int32_t), s);
  if (benc)  // a B the encoder could not take gates this product like one rejected now
    cudaMemcpyAsync(flag, static_cast<const char *>(benc) + fp4_b_layout(p).flag_off, sizeof(int32_t),
                    cudaMemcpyDeviceToDevice, s);
  const int srad = (g.a.skind == SK_K ? g.a.srad : 0) + (g.b.skind == SK_K ? g.b.srad : 0);
  const int srad2 = srad + 2;
  // A is encoded on every call; B too unless the caller passed it pre-encoded (tc_encode_b).
  for (int side = 0; side < (benc ? 1 : 2); ++side)
    encode_fp4_side(g, p, side, ws + p.off[side * 5 + 0], ws + p.off[side * 5 + 1], ws + p.off[side * 5 + 2],
                    ws + p.off[side * 5 + 3], ws + p.off[side * 5 + 4], ws + p.off[10 + side], flag, srad2, s);
  const char *bsrc[6] = {ws + p.off[5], ws + p.off[6], ws + p.off[7], ws + p.off[8], ws + p.off[9], ws + p.off[11]};
  if (benc) {
    const Fp4BLayout l = fp4_b_layout(p);
    for (int i = 0; i < 6; ++i) bsrc[i] = static_cast<const char *>(benc) + l.off[i];
  }
  fp4::GemmArgs a;
  a.aq = reinterpret_cast<const uint4 *>(ws + p.off[0]);
  a.am = reinterpret_cast<const uint4 *>(ws + p.off[1]);
  a.as = reinterpret_cast<const uint32_t *>(ws + p.off[2]);
  a.amul = reinterpret_cast<const int32_t *>(ws + p.off[3]);
  a.atw = reinterpret_cast<const int2 *>(ws + p.off[4]);
  a.bq = reinterpret_cast<const uint4 *>(bsrc[0]);
  a.bm = reinterpret_cast<const uint4 *>(bsrc[1]);
  a.bs = reinterpret_cast<const uint32_t *>(bsrc[2]);
  a.bmul = reinterpret_cast<const int32_t *>(bsrc[3]);
  a.btw = reinterpret_cast<const int2 *>(bsrc[4]);
  a.atc = reinterpret_cast<const int4 *>(ws + p.off[10]);
  a.btc = reinterpret_cast<const int4 *>(bsrc[5]);
  a.a_rows_pad = p.a_pad;
  a.b_rows_pad = p.b_pad;
  a.M = g.M;
  a.N = g.N;
  a.ntiles = p.ntiles;
  a.F = g.F;
  a.shift0 = g.F - 2 - srad;
  a.srad2 = srad + 2;
  a.pexp = 1023 - (srad + 2);
  a.rne = g.rne;
  a.alpha_a = g.a.alpha;
  a.alpha_b = g.b.alpha;
  a.bias = g.bias;
  a.of = g.of;
  a.out_plain = g.out_is_plain;
  a.out_dt = g.out_dt;
  a.out = g.out;
  a.flag = flag;
  a.status = flag + 1;
  a.wait_polls = wait_polls();
  int st = launch_fp4_gemm_tc(a, p.ng, s);  // tensor cores for NG <= 4
  if (st == TC_UNSUPPORTED) switch (p.ng) {
    case 1: st = launch_fp4_gemm<1>(a, g.M, g.N, s); break;
    case 2: st = launch_fp4_gemm<2>(a, g.M, g.N, s); break;
    case 4: st = launch_fp4_gemm<4>(a, g.M, g.N, s); break;
    default: st = launch_fp4_gemm<8>(a, g.M, g.N, s); break;
  }
  if (st) return st;
  launch_generic(g, flag, s);  // runs only when the encoder raised the flag
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm fast: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

}  // namespace tc
