// Integer-operand GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8): promoted CoFDA with
// exact intervals (the cfg4 mapping) and int_exact.
//
// Exactness is the DP4A kernel's argument (tc_gemm_int.cu): with PI * max|ka| * max|kb| < 2**(p+1),
// p = min(F, 23), every promote interval's partial is the exact integer dot product D of the int8
// codes, and the reference's promotion is acc = fma(float(D), (1 * sa) * sb, acc) in IEEE fp32. An
// int8 x int8 MMA accumulating in int32 produces exactly these integers (|D| < 2**24 here), so the
// tensor cores change nothing in the arithmetic. int_exact needs the integer sum over all of K; the
// tensor cores accumulate it in TMEM when max|ka| * max|kb| * K < 2**31 and it is normalised once.
//
// CTA: 128 x 128 outputs, K in spans of 128 (one promote interval). Warp 16 is the producer and MMA
// issuer: 1-D bulk copies (cp.async.bulk, no multicast) bring a span of A and B (16 KB each, already
// in the UMMA canonical K-major layout written by the encoder) into a 3-stage ring; one elected
// thread issues four M128 N128 K32 MMAs per span into a double-buffered int32 accumulator in TMEM
// and commits them to mbarriers. Warps 0..15 are the epilogue: warp w reads TMEM lanes 32 (w % 4)
// (rows) and columns 32 (w / 4) .. +31 with tcgen05.ld and applies the promotion. Every mbarrier wait
// is bounded; on a timeout the status word is set, in-flight MMAs are waited for (bounded), TMEM is
// freed, and the exact generic kernel queued behind recomputes the product.
//
// Shared-memory operand layout (UMMA K-major, no swizzle): element (row r, k) of a span sits at byte
// (k / 16) * 2048 + r * 16 + k % 16, i.e. 8-row x 16-byte core matrices, 128 bytes apart along M
// (stride byte offset) and 2048 bytes apart along K (leading byte offset).
#include <algorithm>
#include <cstring>
#include <string>

#include "tc_bulk.cuh"
#include "tc_gemm.cuh"
#include "tc_tcgen05.cuh"

namespace tc {
namespace itc {

constexpr int kTile = 128;    // rows of A / columns of B per CTA
constexpr int kSpan = 128;    // K per stage
constexpr int kStages = 3;
constexpr int kSpanBytes = kTile * kSpan;  // 16 KB of int8 codes per operand and span
constexpr int kEpilogueWarps = 16;
constexpr int kThreads = (kEpilogueWarps + 1) * 32;
constexpr uint32_t kTmemCols = 256;        // two 128-column int32 accumulators

struct EncodeArgs {
  const void *v;
  int dt;
  int64_t rows, K, rows_pad, nspans;
  int frac;
  uint4 *out;     // [tile][span][k / 16][row in tile] 16-byte groups of int8 codes
  int32_t *flag;
};

// One thread per (tile, span, k/16, row): 16 codes k = v * 2**frac (|k| <= 127, on the grid).
__global__ void __launch_bounds__(256) encode_kernel(EncodeArgs e) {
  const int64_t total = e.rows_pad * e.nspans * (kSpan / 16);
  bool bad = false;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rr = idx % kTile;
    int64_t rest = idx / kTile;
    const int64_t k16 = rest % (kSpan / 16);
    rest /= (kSpan / 16);
    const int64_t span = rest % e.nspans;
    const int64_t tile = rest / e.nspans;
    const int64_t r = tile * kTile + rr;
    uint32_t w[4] = {0, 0, 0, 0};
    if (r < e.rows) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int64_t k = span * kSpan + k16 * 16 + j;
        int q = 0;
        if (k < e.K) {
          const float t = ldexpf(load_as_float(e.v, e.dt, r * e.K + k), e.frac);
          q = (int)t;
          if (!((float)q == t) || q > 127 || q < -127) bad = true;  // also NaN / Inf / off-grid
        }
        w[j >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (j & 3));
      }
    }
    e.out[idx] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicExch(e.flag, 1);
}

// The promote interval scales of one operand, span-major: dst[sp][r] = src[r][sp * kSpan / kd] (1 for
// padding rows), so an epilogue thread reads its 32 columns' weights with 16-byte loads.
__global__ void __launch_bounds__(256) span_scales_kernel(const float *src, int64_t nkd, int kd, int64_t rows,
                                                          int64_t rows_pad, int64_t nspans, float *dst) {
  const int64_t total = nspans * rows_pad;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t sp = idx / rows_pad, r = idx % rows_pad;
    dst[idx] = r < rows ? src[r * nkd + sp * kSpan / kd] : 1.0f;
  }
}

struct Args {
  const uint8_t *aw, *bw;   // encoded operands [tile][span][kSpanBytes]
  int64_t M, N, nspans;
  int promote;              // 1: per-span promotion; 0: int_exact (TMEM accumulates all of K)
  int exp_out;              // int_exact exponent -(frac_a + frac_b)
  const float *sa_t, *sb_t; // promote K scales per span, span-major [nspans][rows_pad], or nullptr
  int64_t a_pad, b_pad;
  GemmDesc g;
  const int32_t *flag;
  int32_t *status;
  int wait_polls;  // poll limit of the pipeline waits (negative: default)
};

// Instruction descriptor: kind::i8, D int32, A and B signed int8, both K-major, M = 128, N = 128.
constexpr uint32_t kIdesc = tc5::idesc_i8(kTile, kTile);

template <bool PROMOTE>
__global__ void __launch_bounds__(kThreads, 1) int_tc_kernel(Args p) {
  if (*p.flag) return;  // an operand the encoder rejected: the generic kernel takes over
  extern __shared__ __align__(1024) unsigned char smem_raw[];  // [kStages][A, B][kSpanBytes]
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], tfull[2], tempty[2];
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t mt = blockIdx.y, nt = blockIdx.x;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpilogueWarps);
    }
    fence_barrier_init();
  }
  if (warp == 0) tc5::tmem_alloc(&tmem_base, kTmemCols);
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tbase = tmem_base;

  if (warp == kEpilogueWarps) {
    if (lane == 0) {
      // Producer and MMA issuer (one thread).
      bool ok = true;
      int64_t issued = 0, waited_full = 0, last = -1;
      auto issue = [&](int64_t sp) {
        const int s = (int)(sp % kStages);
        unsigned char *st = smem_raw + (size_t)s * 2 * kSpanBytes;
        mbar_expect_tx(&full[s], 2 * kSpanBytes);
        bulk_g2s(st, p.aw + (mt * p.nspans + sp) * kSpanBytes, kSpanBytes, &full[s]);
        bulk_g2s(st + kSpanBytes, p.bw + (nt * p.nspans + sp) * kSpanBytes, kSpanBytes, &full[s]);
        issued = sp + 1;
      };
      for (int64_t sp = 0; sp < kStages && sp < p.nspans; ++sp) issue(sp);
      for (int64_t sp = 0; sp < p.nspans; ++sp) {
        const int s = (int)(sp % kStages);
        const int b = PROMOTE ? (int)(sp & 1) : 0;
        // The accumulator buffer is free once the epilogue has read span sp - 2 from it.
        if (PROMOTE && sp >= 2 && !mbar_wait_sleep(&tempty[b], (uint32_t)(((sp - 2) >> 1) & 1), p.wait_polls)) { ok = false; break; }
        if (!mbar_wait_sleep(&full[s], (uint32_t)((sp / kStages) & 1), p.wait_polls)) { ok = false; break; }
        waited_full = sp + 1;
        tc5::fence_after_sync();
        const unsigned char *sa = smem_raw + (size_t)s * 2 * kSpanBytes, *sb = sa + kSpanBytes;
#pragma unroll
        for (int kk = 0; kk < kSpan / 32; ++kk) {
          const uint64_t da = tc5::smem_desc(sa + kk * 2 * (kTile * 16), kTile * 16, 128);
          const uint64_t db = tc5::smem_desc(sb + kk * 2 * (kTile * 16), kTile * 16, 128);
          tc5::mma_i8(tbase + (uint32_t)(b * kTile), da, db, kIdesc, (PROMOTE ? kk > 0 : (sp > 0 || kk > 0)) ? 1u : 0u);
        }
        tc5::mma_commit(&empty[s]);                          // the stage is free once these MMAs finish
        if (PROMOTE || sp == p.nspans - 1) tc5::mma_commit(&tfull[b]);  // the partial is ready
        last = sp;
        // Refill the stage of span sp - 1 (its MMAs run ahead of the ones just queued) with the span
        // kStages after it, so the tensor pipe always has the next span's MMAs queued.
        const int64_t prev = sp - 1;
        if (prev >= 0 && prev + kStages < p.nspans) {
          if (!mbar_wait_sleep(&empty[prev % kStages], (uint32_t)((prev / kStages) & 1), p.wait_polls)) { ok = false; break; }
          issue(prev + kStages);
        }
      }
      if (!ok) atomicExch(p.status, 1);
      // Nothing of this CTA may still be in flight when it exits: copies issued but not waited for,
      // and the MMAs up to the last commit (bounded waits).
      for (int64_t u = waited_full; u < issued; ++u) mbar_wait_sleep(&full[u % kStages], (uint32_t)((u / kStages) & 1));
      if (last >= 0) mbar_wait_sleep(&empty[last % kStages], (uint32_t)((last / kStages) & 1));
    }
    __syncwarp();
  } else {
    // Epilogue: thread = row 32 (warp % 4) + lane, columns 32 (warp / 4) .. +31 of the tile.
    const int quarter = warp & 3, part = warp >> 2;
    const int64_t m = mt * kTile + quarter * 32 + lane;
    const int64_t n0 = nt * kTile + part * 32;
    const uint32_t lane_addr = tbase + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(part * 32);
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
    bool ok = true;
    const int64_t rounds = PROMOTE ? p.nspans : 1;
    for (int64_t sp = 0; sp < rounds; ++sp) {
      const int b = PROMOTE ? (int)(sp & 1) : 0;
      ok = mbar_wait_sleep(&tfull[b], PROMOTE ? (uint32_t)((sp >> 1) & 1) : 0u, p.wait_polls);
      if (!__all_sync(0xFFFFFFFFu, ok)) {
        if (lane == 0) atomicExch(p.status, 1);
        ok = false;
        break;
      }
      tc5::fence_after_sync();
      uint32_t d[32];
      tc5::tmem_ld32(lane_addr + (uint32_t)(b * kTile), d);
      tc5::fence_before_sync();
      __syncwarp();
      if (PROMOTE && lane == 0) mbar_arrive(&tempty[b]);  // the buffer may take span sp + 2
      if (PROMOTE) {
        // weight = (1 * sa) * sb, each an fp32 RN multiply; the interval's exact partial as fp32.
        const float wa = p.sa_t ? __ldg(p.sa_t + sp * p.a_pad + m) : 1.0f;
        const float4 *src = reinterpret_cast<const float4 *>(p.sb_t + sp * p.b_pad + n0);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 v = p.sb_t ? __ldg(src + q) : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
          const float wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int j = 4 * q + t;
            const float w = p.sb_t ? (p.sa_t ? __fmul_rn(wa, wv[t]) : wv[t]) : wa;
            acc[j] = __fmaf_rn(__int2float_rn((int)d[j]), w, acc[j]);
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = fixed_to_fp32((int64_t)(int)d[j], p.exp_out, 0, true, false);
      }
    }
    if (ok && m < p.M) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int64_t n = n0 + j;
        if (n < p.N) store_out(p.g, m, n, epilogue(p.g, m, n, acc[j]));
      }
    }
  }
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  if (warp == 0) tc5::tmem_dealloc(tbase, kTmemCols);
}

}  // namespace itc

// ---------------------------------------------------------------- dispatch
// The caller (launch_int) established the exactness conditions of the promoted path, or int_exact's.
bool int_tc_eligible(const GemmDesc &g, bool promote, int64_t max_a, int64_t max_b) {
  if (promote) return g.PI == itc::kSpan;
  return (double)max_a * (double)max_b * (double)((g.K + itc::kSpan - 1) / itc::kSpan * itc::kSpan) < 2147483647.0;
}

struct IntTcPlan {
  int64_t nspans, a_pad, b_pad;
  size_t off_a, off_b, off_sa, off_sb, off_flag, total;
};

static IntTcPlan plan_int_tc(const GemmDesc &g) {
  IntTcPlan p;
  p.nspans = (g.K + itc::kSpan - 1) / itc::kSpan;
  p.a_pad = (g.M + itc::kTile - 1) / itc::kTile * itc::kTile;
  p.b_pad = (g.N + itc::kTile - 1) / itc::kTile * itc::kTile;
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  p.off_a = 0;
  p.off_b = up((size_t)p.a_pad * p.nspans * itc::kSpan);
  p.off_sa = p.off_b + up((size_t)p.b_pad * p.nspans * itc::kSpan);
  p.off_sb = p.off_sa + up((size_t)p.a_pad * p.nspans * sizeof(float));
  p.off_flag = p.off_sb + up((size_t)p.b_pad * p.nspans * sizeof(float));
  p.total = p.off_flag + 256;
  return p;
}

size_t int_tc_workspace(const GemmDesc &g) { return plan_int_tc(g).total; }

int launch_int_tc(const GemmDesc &g, bool promote, void *workspace, size_t workspace_bytes, cudaStream_t s) {
  const IntTcPlan p = plan_int_tc(g);
  if (!workspace || workspace_bytes < p.total) return set_error("tc_gemm: workspace too small"), TC_WORKSPACE_TOO_SMALL;
  if (p.a_pad / itc::kTile > 65535 || p.nspans == 0) return TC_UNSUPPORTED;
  char *ws = static_cast<char *>(workspace);
  int32_t *flag = reinterpret_cast<int32_t *>(ws + p.off_flag);
  cudaMemsetAsync(flag, 0, 2 * sizeof(int32_t), s);  // [0] operands rejected, [1] timeout
  for (int side = 0; side < 2; ++side) {
    const OpDesc &o = side ? g.b : g.a;
    itc::EncodeArgs e;
    e.v = o.v;
    e.dt = o.dt;
    e.rows = o.rows;
    e.K = o.K;
    e.rows_pad = side ? p.b_pad : p.a_pad;
    e.nspans = p.nspans;
    e.frac = o.f.frac_bits;
    e.out = reinterpret_cast<uint4 *>(ws + (side ? p.off_b : p.off_a));
    e.flag = flag;
    const int64_t work = e.rows_pad * p.nspans * (itc::kSpan / 16);
    const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 16);
    itc::encode_kernel<<<(unsigned)blocks, 256, 0, s>>>(e);
    count_launch();
    if (promote && o.skind == SK_K) {
      const int64_t n = e.rows_pad * p.nspans;
      float *dst = reinterpret_cast<float *>(ws + (side ? p.off_sb : p.off_sa));
      itc::span_scales_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 8), 256, 0, s>>>(
          o.scale, o.nkd, o.kd, o.rows, e.rows_pad, p.nspans, dst);
      count_launch();
    }
  }
  itc::Args a;
  std::memset(&a, 0, sizeof(a));
  a.aw = reinterpret_cast<const uint8_t *>(ws + p.off_a);
  a.bw = reinterpret_cast<const uint8_t *>(ws + p.off_b);
  a.M = g.M;
  a.N = g.N;
  a.nspans = p.nspans;
  a.promote = promote;
  a.exp_out = -(g.a.f.frac_bits + g.b.f.frac_bits);
  a.a_pad = p.a_pad;
  a.b_pad = p.b_pad;
  if (promote && g.a.skind == SK_K) a.sa_t = reinterpret_cast<const float *>(ws + p.off_sa);
  if (promote && g.b.skind == SK_K) a.sb_t = reinterpret_cast<const float *>(ws + p.off_sb);
  a.g = g;
  a.flag = flag;
  a.status = flag + 1;
  a.wait_polls = wait_polls();
  const size_t smem = (size_t)itc::kStages * 2 * itc::kSpanBytes;
  auto kern = promote ? itc::int_tc_kernel<true> : itc::int_tc_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(std::string("int tc gemm: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  dim3 grid((unsigned)(p.b_pad / itc::kTile), (unsigned)(p.a_pad / itc::kTile));
  kern<<<grid, itc::kThreads, smem, s>>>(a);
  count_launch();
  launch_generic(g, flag, s);  // runs only when an operand was rejected or a wait ran out
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm int tc: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

}  // namespace tc
