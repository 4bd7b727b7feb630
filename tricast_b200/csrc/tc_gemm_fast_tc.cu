// GDFS for E2M1 x E2M1 (the nvidia_blackwell_fp4 preset on NVFP4 / MXFP4) with the group dot
// products on the 5th-generation tensor cores.
//
// The arithmetic is the tiled DP4A kernel's (tc_gemm_fast.cu): a group of 16 contributes
// D * ms_a * ms_b * 2**(es_a + es_b - srad - 2), D = sum (2a)(2b) the exact integer dot product of
// the doubled codes; a K tile that passes the single-pass bounds is summed exactly in int64
// (D times the two multipliers) and normalised by one fp64 -> fp32 rounding, and a tile that fails
// redoes that output with the exact two-pass labels. Only D moves: tcgen05.mma kind::i8 computes it
// for a 128 x 64 block of outputs per group, one MMA of K = 32 per group whose second 16-byte K half
// is a zero block (the descriptor's leading byte offset points there), so each group lands in its own
// int32 TMEM accumulator, exact (|D| <= 16 * 144).
//
// CTA: 128 rows of A (TMEM lanes) x 64 columns of B, K tiles of NG <= 4 groups. Warp 16 is the
// producer and MMA issuer: 1-D bulk copies (no multicast) bring a tile's records (16-byte code rows,
// the encoder's layout, which is UMMA's K-major no-swizzle layout; multipliers; tile words) into a
// 4-stage ring; one thread issues NG MMAs per tile into one of two TMEM buffers (NG x 64 columns each)
// and commits them to mbarriers. Warps 0..15 are the epilogue: warp w owns rows 32 (w % 4) .. +31 and
// columns 16 (w / 4) .. +15, reads the group sums with tcgen05.ld, forms the int64 tile sum and runs
// the tile step. A stage is released when its MMAs and all sixteen epilogue warps are done with it;
// an accumulator buffer when the epilogue has read it. Every wait is bounded; on a timeout the
// status word is set, outstanding copies and MMAs are waited for (bounded), TMEM is freed, and the
// exact generic kernel queued behind recomputes the product.
#include <algorithm>
#include <cstring>
#include <string>

#include "tc_fp4.cuh"
#include "tc_tcgen05.cuh"

namespace tc {
namespace fp4tc {

// (output, K tile) pairs that failed the single-pass bounds and took the exact two-pass step, summed
// over every launch on this device (one warp-aggregated atomic per round of the rare path).
__device__ unsigned long long g_exact_tile_steps;

constexpr int kM = 128;  // rows of A per CTA (TMEM lanes)
constexpr int kN = 64;   // columns of B per CTA
constexpr int kStages = 4;
constexpr int kEpiWarps = 16;
constexpr int kCols = kN / (kEpiWarps / 4);  // columns per epilogue thread
constexpr int kChunk = 4;                    // columns per tile-step pass (bounds the live int64 sums)
constexpr int kThreads = (kEpiWarps + 1) * 32;
constexpr uint32_t kTmemCols = 512;  // two buffers of NG (<= 4) groups x 64 columns

template <int NG>
struct Stage {
  uint4 aq[NG][kM];  // 16-byte code rows (2 KB per group)
  uint4 bq[NG][kN];
  int32_t amul[NG][kM];
  int32_t bmul[NG][kN];
  int4 atc[kM];      // row parts of the tile-step bounds and power (tile_words_kernel)
  int4 btc[kN];      // column parts
};

// The exact two-pass tile step for one output whose tile failed the single-pass bounds (rare). Called
// by the whole warp (the TMEM loads are warp-collective); lanes with j < 0 only take part in the loads.
template <int NG, bool RNE>
__device__ __noinline__ float exact_tile_step(const fp4::GemmArgs &g, uint32_t buf_addr, int j, float cj, int64_t t,
                                              int64_t m, int64_t ncol0) {
  int dj[NG];
#pragma unroll
  for (int gg = 0; gg < NG; ++gg) {
    int v = 0;
#pragma unroll
    for (int h = 0; h < kCols / 8; ++h) {
      uint32_t d[8];
      tc5::tmem_ld8(buf_addr + (uint32_t)(gg * kN + h * 8), d);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) v = h * 8 + jj == j ? (int)d[jj] : v;
    }
    dj[gg] = v;
  }
  if (j < 0) return cj;
  const int64_t n = ncol0 + j;
  int emax = fp4::running_exp(cj);
#pragma unroll
  for (int gg = 0; gg < NG; ++gg) {
    const int64_t grow = t * NG + gg;
    if (dj[gg] == 0) continue;
    const int label = fp4::exp_class_max(g.am[grow * g.a_rows_pad + m], g.bm[grow * g.b_rows_pad + n]) +
                      fp4::scale_exp(g.as[grow * g.a_rows_pad + m]) + fp4::scale_exp(g.bs[grow * g.b_rows_pad + n]);
    emax = max(emax, label);
  }
  int64_t total = fp4::running_term(cj, g.F, emax);
#pragma unroll
  for (int gg = 0; gg < NG; ++gg) {
    const int64_t grow = t * NG + gg;
    const int d = dj[gg];
    const uint32_t sa = g.as[grow * g.a_rows_pad + m], sb = g.bs[grow * g.b_rows_pad + n];
    const uint32_t x = (uint32_t)(d < 0 ? -d : d) * (((sa >> 16) & 0xFFu) * ((sb >> 16) & 0xFFu));
    const int sh = g.shift0 + fp4::scale_exp(sa) + fp4::scale_exp(sb) - emax;
    // x < 2**20 and sh <= shift0 <= 40: (x << 40) >> (40 - sh) is the exact truncation.
    const int rs = max(40 - sh, 0);  // sh > 40 only for d == 0 (x == 0)
    const uint64_t v = rs >= 64 ? 0ull : (((uint64_t)x << 40) >> rs);
    const bool neg = (d < 0) != (((sa ^ sb) >> 24) & 1u);
    total += neg ? -(int64_t)v : (int64_t)v;
  }
  const uint32_t cb = f2u(cj) & 0x7FFFFFFFu;
  if (cb < kInf && emax != fp4::kNone) cj = fixed_to_fp32(total, emax, g.F, RNE, true);
  return cj;
}

template <int NG, bool RNE>
__global__ void __launch_bounds__(kThreads, 1) gdfs_fp4_tc_kernel(const __grid_constant__ fp4::GemmArgs g) {
  if (*g.flag) return;  // an operand the encoder rejected: the generic kernel takes over
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Stage<NG> *stages = reinterpret_cast<Stage<NG> *>(smem_raw);
  uint4 *zeros = reinterpret_cast<uint4 *>(smem_raw + kStages * sizeof(Stage<NG>));  // kM x 16 zero bytes
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], tfull[2], tempty[2];
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = (int64_t)blockIdx.y * kM, n0 = (int64_t)blockIdx.x * kN;
  constexpr uint32_t kIdesc = tc5::idesc_i8(kM, kN);

  for (int i = threadIdx.x; i < kM; i += kThreads) zeros[i] = make_uint4(0, 0, 0, 0);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the zero block is read by the MMAs
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + kEpiWarps);  // the MMAs' commit and every epilogue warp
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == 0) tc5::tmem_alloc(&tmem_base, kTmemCols);
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tbase = tmem_base;

  if (warp == kEpiWarps) {
    if (lane == 0) {
      // Producer and MMA issuer (one thread).
      constexpr uint32_t kStageBytes = NG * (kM * 16 + kN * 16 + kM * 4 + kN * 4) + kM * 16 + kN * 16;
      bool ok = true;
      int64_t issued = 0, waited_full = 0, last = -1;
      auto issue = [&](int64_t t) {
        Stage<NG> &st = stages[t % kStages];
        uint64_t *bar = &full[t % kStages];
        mbar_expect_tx(bar, kStageBytes);
        for (int gg = 0; gg < NG; ++gg) {
          const int64_t ga = (t * NG + gg) * g.a_rows_pad + m0, gb = (t * NG + gg) * g.b_rows_pad + n0;
          bulk_g2s(st.aq[gg], g.aq + ga, kM * 16, bar);
          bulk_g2s(st.bq[gg], g.bq + gb, kN * 16, bar);
          bulk_g2s(st.amul[gg], g.amul + ga, kM * 4, bar);
          bulk_g2s(st.bmul[gg], g.bmul + gb, kN * 4, bar);
        }
        bulk_g2s(st.atc, g.atc + t * g.a_rows_pad + m0, kM * 16, bar);
        bulk_g2s(st.btc, g.btc + t * g.b_rows_pad + n0, kN * 16, bar);
        issued = t + 1;
      };
      for (int64_t t = 0; t < kStages && t < g.ntiles; ++t) issue(t);
      for (int64_t t = 0; t < g.ntiles; ++t) {
        const int s = (int)(t % kStages), b = (int)(t & 1);
        if (t >= 2 && !mbar_wait_sleep(&tempty[b], (uint32_t)(((t - 2) >> 1) & 1), g.wait_polls)) { ok = false; break; }
        if (!mbar_wait_sleep(&full[s], (uint32_t)((t / kStages) & 1), g.wait_polls)) { ok = false; break; }
        waited_full = t + 1;
        tc5::fence_after_sync();
        const Stage<NG> &st = stages[s];
#pragma unroll
        for (int gg = 0; gg < NG; ++gg) {
          // K = 32: the group's 16 code bytes, then 16 zero bytes (leading byte offset to the zero block).
          const uint64_t da = tc5::smem_desc(st.aq[gg], (uint32_t)(smem_addr(zeros) - smem_addr(st.aq[gg])), 128);
          const uint64_t db = tc5::smem_desc(st.bq[gg], (uint32_t)(smem_addr(zeros) - smem_addr(st.bq[gg])), 128);
          tc5::mma_i8(tbase + (uint32_t)((b * NG + gg) * kN), da, db, kIdesc, 0u);
        }
        tc5::mma_commit(&empty[s]);
        tc5::mma_commit(&tfull[b]);
        last = t;
        // Refill the stage of tile t - 1 (released by its MMAs and the epilogue) with tile t - 1 + kStages.
        const int64_t prev = t - 1;
        if (prev >= 0 && prev + kStages < g.ntiles) {
          if (!mbar_wait_sleep(&empty[prev % kStages], (uint32_t)((prev / kStages) & 1), g.wait_polls)) { ok = false; break; }
          issue(prev + kStages);
        }
      }
      if (!ok) atomicExch(g.status, 1);
      for (int64_t u = waited_full; u < issued; ++u) mbar_wait_sleep(&full[u % kStages], (uint32_t)((u / kStages) & 1));
      if (last >= 0) mbar_wait_sleep(&tfull[last & 1], (uint32_t)((last >> 1) & 1));
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3, part = warp >> 2;
    const int row = quarter * 32 + lane, col0 = part * kCols;
    const int64_t m = m0 + row;
    const uint32_t lane_addr = tbase + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col0;
    float c[kCols];
#pragma unroll
    for (int j = 0; j < kCols; ++j) c[j] = 0.0f;
    bool ok = true;
    for (int64_t t = 0; t < g.ntiles; ++t) {
      const int s = (int)(t % kStages), b = (int)(t & 1);
      ok = mbar_wait_sleep(&tfull[b], (uint32_t)((t >> 1) & 1), g.wait_polls);
      if (!__all_sync(0xFFFFFFFFu, ok)) {
        if (lane == 0) atomicExch(g.status, 1);
        ok = false;
        break;
      }
      tc5::fence_after_sync();
      const Stage<NG> &st = stages[s];
      // Tile step per output (the tiled kernel's single-pass bounds): the int64 tile sum of the group
      // sums times their multipliers, then c + sum * 2**(ea + eb - srad2) in fp64 (exact under the
      // bounds) and one rounding to fp32. The bounds and the power are a row part (this thread's) plus
      // a column part (tile_words_kernel). TMEM is read kChunk columns x NG groups at a time with one
      // wait per chunk. (17 warps leave 96 registers a thread: five warps share one sub-partition's
      // register file, so the chunk's loads are not double-buffered.)
      const int4 rw = st.atc[row];
      const int nd = -rw.z;  // d = rw.z + cw.z >= 0  <=>  cw.z >= -rw.z
      int ma[NG];
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) ma[gg] = st.amul[gg][row];
      const uint32_t buf = lane_addr + (uint32_t)(b * NG * kN);
      uint32_t unsafe = 0;
#pragma unroll
      for (int h = 0; h < kCols / kChunk; ++h) {
        uint32_t dh[NG * kChunk];
#pragma unroll
        for (int gg = 0; gg < NG; ++gg)
          tc5::tmem_ld4_nowait(buf + (uint32_t)(gg * kN + h * kChunk), *reinterpret_cast<uint32_t(*)[4]>(&dh[gg * kChunk]));
        tc5::tmem_wait_ld<NG * kChunk>(dh);
        int4 bm[NG];
#pragma unroll
        for (int gg = 0; gg < NG; ++gg) bm[gg] = *reinterpret_cast<const int4 *>(&st.bmul[gg][col0 + h * kChunk]);
#pragma unroll
        for (int jj = 0; jj < kChunk; ++jj) {
          const int j = h * kChunk + jj;
          int64_t acc = 0;
#pragma unroll
          for (int gg = 0; gg < NG; ++gg) {
            const int mb = jj == 0 ? bm[gg].x : jj == 1 ? bm[gg].y : jj == 2 ? bm[gg].z : bm[gg].w;
            acc += (int64_t)(int)dh[gg * kChunk + jj] * (int64_t)(ma[gg] * mb);
          }
          const int4 cw = st.btc[col0 + j];
          const uint32_t cb = f2u(c[j]) & 0x7FFFFFFFu;
          const int be = max((int)(cb >> 23), 1);  // a subnormal c has the lsb and exponent of field 1
          // The terms' quanta allow one pass (d >= 0), and c keeps its bits at the tile's radix (its
          // lsb and magnitude within the window) or is zero.
          const bool keeps = ((uint32_t)(be - rw.x - cw.x) <= (uint32_t)(rw.y + cw.y)) | (cb == 0u);
          const bool safe = (cw.z >= nd) & keeps;
          const double p2 = __hiloint2double(rw.w + cw.w, 0);
          const double v = __fma_rn((double)acc, p2, (double)c[j]);
          const float r = (RNE && fabs(v) >= 0x1p-126) ? __double2float_rn(v) : __double2float_rz(v);
          // |v| >= 2**128 overflows the fixed-point normalisation: the exact step decides.
          const bool fits = fabs(v) < 0x1p128;
          const bool take = safe & fits & (cb < kInf);  // an Inf / NaN running value is sticky
          c[j] = take ? r : c[j];
          unsafe |= (!take & (cb < kInf)) ? 1u << j : 0u;
        }
      }
      // Exact two-pass tile step for the outputs that failed the bounds (rare): each round, every lane
      // takes its lowest pending column and the warp runs the step together. It is a separate
      // (non-inlined) function so that its registers do not count against this loop's.
      while (__any_sync(0xFFFFFFFFu, unsafe != 0)) {
        const int j = unsafe ? __ffs(unsafe) - 1 : -1;
        const unsigned pending = __ballot_sync(0xFFFFFFFFu, j >= 0);
        if (lane == 0) atomicAdd(&g_exact_tile_steps, (unsigned long long)__popc(pending));
        float cj = 0.0f;
#pragma unroll
        for (int jj = 0; jj < kCols; ++jj) cj = jj == j ? c[jj] : cj;
        cj = exact_tile_step<NG, RNE>(g, lane_addr + (uint32_t)(b * NG * kN), j, cj, t, m, n0 + col0);
        if (j >= 0) unsafe &= unsafe - 1;
#pragma unroll
        for (int jj = 0; jj < kCols; ++jj) c[jj] = jj == j ? cj : c[jj];
      }
      tc5::fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tempty[b]);  // the accumulator buffer may take tile t + 2
        mbar_arrive(&empty[s]);   // this warp is done with the stage's multipliers and tile words
      }
    }
    if (ok && m < g.M) {
      // Epilogue: alpha, bias, output rounding (src/tricast/reference/mma.py:376-384).
      float alpha = 1.0f;
      const bool has_alpha = g.alpha_a || g.alpha_b;
      if (g.alpha_a) alpha = *g.alpha_a;
      if (g.alpha_b) alpha = g.alpha_a ? __fmul_rn(alpha, *g.alpha_b) : *g.alpha_b;
#pragma unroll
      for (int j = 0; j < kCols; ++j) {
        const int64_t n = n0 + col0 + j;
        if (n >= g.N) continue;
        float v = c[j];
        if (has_alpha) v = __fmul_rn(alpha, v);
        if (g.bias) v = __fadd_rn(v, g.bias[n]);
        if (!g.out_plain) v = cast_to(v, g.of, TC_RNE, false, 0u, 32);
        store_container(g.out, g.out_dt, m * g.N + n, v);
      }
    }
  }
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  if (warp == 0) tc5::tmem_dealloc(tbase, kTmemCols);
}

}  // namespace fp4tc

template <int NG, bool RNE>
static int launch_tc(const fp4::GemmArgs &args, cudaStream_t s) {
  // At least 120 KB: one CTA per SM, so the 512 TMEM columns it allocates are always free.
  const size_t smem = std::max<size_t>(sizeof(fp4tc::Stage<NG>) * fp4tc::kStages + fp4tc::kM * 16, 120 * 1024);
  cudaError_t e = cudaFuncSetAttribute(fp4tc::gdfs_fp4_tc_kernel<NG, RNE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return set_error(std::string("gdfs fp4 tc: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  dim3 grid((unsigned)((args.N + fp4tc::kN - 1) / fp4tc::kN), (unsigned)((args.M + fp4tc::kM - 1) / fp4tc::kM));
  fp4tc::gdfs_fp4_tc_kernel<NG, RNE><<<grid, fp4tc::kThreads, smem, s>>>(args);
  count_launch();
  return TC_OK;
}

int exact_tile_steps(unsigned long long *count) {
  cudaError_t e = cudaMemcpyFromSymbol(count, fp4tc::g_exact_tile_steps, sizeof(*count));
  if (e != cudaSuccess) return set_error(std::string("tc_exact_tile_steps: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

// The GDFS-FP4 GEMM on tensor cores for NG in {1, 2, 4} groups per K tile (A rows padded to 128, B
// rows to 64); TC_UNSUPPORTED otherwise.
int launch_fp4_gemm_tc(const fp4::GemmArgs &args, int ng, cudaStream_t s) {
  if (args.a_rows_pad % fp4tc::kM || args.b_rows_pad % fp4tc::kN || args.ntiles == 0) return TC_UNSUPPORTED;
  if ((args.M + fp4tc::kM - 1) / fp4tc::kM > 65535) return TC_UNSUPPORTED;
  switch (ng) {
    case 1: return args.rne ? launch_tc<1, true>(args, s) : launch_tc<1, false>(args, s);
    case 2: return args.rne ? launch_tc<2, true>(args, s) : launch_tc<2, false>(args, s);
    case 4: return args.rne ? launch_tc<4, true>(args, s) : launch_tc<4, false>(args, s);
    default: return TC_UNSUPPORTED;
  }
}

}  // namespace tc
