// Fast kernels for integer operands: promoted CoFDA with exact intervals, and int_exact.
//
// Promoted CoFDA (TriCast src/tricast/reference/mma.py:286-315 with promote_interval > 0) on two
// integer formats without fraction bits: every product has exponent 0 and significand |ka*kb| at
// radix 0. Inside one interval the partial starts at +0; if every prefix sum P satisfies
// |P| < 2**(p+1), p = min(F, 23), then at each chunk (by induction) the running value's exponent L
// is at most p <= F, so emax = max(0, L) <= F, every alignment shift of a product (|ka*kb| << F)
// >> emax is exact, the sum is the exact integer, and normalisation to p + 1 bits keeps it whole.
// PI * max|ka| * max|kb| < 2**(p+1) guarantees this for any data, so each interval's partial is the
// exact integer dot product D (DP4A on int8 codes), and the reference's promotion is
// acc = fma(float(D), (1 * sa) * sb, acc) in IEEE fp32.
//
// int_exact (mma.py:348-358): the exact integer sum over all of K, normalised once with RNE
// (fda=False) at exponent -(frac_a + frac_b).
//
// Operands are encoded to int8 codes k = v * 2**frac in [interval][k/4][row] 32-bit words so that a
// CTA's stage is one contiguous 1-D bulk copy; off-grid values or |k| > 127 raise the device flag
// and the exact generic kernel runs instead.
#include <cstring>
#include <string>

#include "tc_gemm.cuh"

namespace tc {
namespace intk {

constexpr int kTile = 128;   // rows / columns per CTA (16 x 16 threads, 8 x 8 outputs each)
constexpr int kSpan = 128;   // K elements per stage (one promote interval of 128, or 128 of K)
constexpr int kStages = 3;

struct EncodeArgs {
  const void *v;
  int dt;
  int64_t rows, K, rows_pad, nspans;
  int frac;
  uint32_t *out;  // [tile][span][kSpan/4][kTile] words of 4 int8 codes
  int32_t *flag;
};

__global__ void __launch_bounds__(256) encode_kernel(EncodeArgs e) {
  const int64_t total = e.rows_pad * e.nspans * (kSpan / 4);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  bool bad = false;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int64_t rr = idx % kTile;
    int64_t rest = idx / kTile;
    const int64_t k4 = rest % (kSpan / 4);
    rest /= (kSpan / 4);
    const int64_t span = rest % e.nspans;
    const int64_t tile = rest / e.nspans;
    const int64_t r = tile * kTile + rr;
    uint32_t word = 0;
    if (r < e.rows) {
      for (int j = 0; j < 4; ++j) {
        const int64_t k = span * kSpan + k4 * 4 + j;
        int q = 0;
        if (k < e.K) {
          float v = load_as_float(e.v, e.dt, r * e.K + k);
          float t = ldexpf(v, e.frac);
          q = (int)t;
          if (!((float)q == t) || q > 127 || q < -127) bad = true;  // also NaN / Inf / off-grid
        }
        word |= ((uint32_t)q & 0xFFu) << (8 * j);
      }
    }
    e.out[idx] = word;
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicExch(e.flag, 1);
}

struct Args {
  const uint32_t *aw, *bw;
  int64_t M, N, nspans;
  int promote;               // 1: per-span fma promotion; 0: int_exact
  int exp_out;               // int_exact exponent -(frac_a + frac_b)
  const float *sa, *sb;      // promote K scales or nullptr
  int64_t sa_nkd, sb_nkd;
  int sa_kd, sb_kd;
  GemmDesc g;
  const int32_t *flag;
  int32_t *status;
  int wait_polls;  // poll limit of the pipeline waits (negative: default)
};

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: ~2**22 polls, or `polls` when that is not negative (0: gives up at once).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int polls = -1) {
  const int limit = polls < 0 ? (1 << 22) : polls;
  for (int i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

struct Stage {
  uint32_t a[kSpan / 4][kTile];
  uint32_t b[kSpan / 4][kTile];
};

// Thread (ty, tx): rows ty*4 + {0..3} and 64 + ty*4 + {0..3}; columns likewise with tx, so the
// 16-byte shared loads of a warp fall on distinct banks.
template <bool PROMOTE>
__global__ void __launch_bounds__(256) int_kernel(Args p) {
  if (*p.flag) return;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Stage *stages = reinterpret_cast<Stage *>(smem_raw);
  __shared__ __align__(8) uint64_t full[kStages];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t mt = blockIdx.y, nt = blockIdx.x;
  constexpr uint32_t kBytes = (kSpan / 4) * kTile * 4;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  auto issue = [&](int64_t sp, int s) {
    mbar_expect_tx(&full[s], 2 * kBytes);
    bulk_g2s(&stages[s].a[0][0], p.aw + (mt * p.nspans + sp) * (kSpan / 4) * kTile, kBytes, &full[s]);
    bulk_g2s(&stages[s].b[0][0], p.bw + (nt * p.nspans + sp) * (kSpan / 4) * kTile, kBytes, &full[s]);
  };
  if (threadIdx.x == 0)
    for (int s = 0; s < kStages && s < p.nspans; ++s) issue(s, s);

  // PROMOTE: fp32 accumulators; int_exact: int64 totals (only one of the two is live).
  float acc[8][8];
  int64_t total[PROMOTE ? 1 : 8][PROMOTE ? 1 : 8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      acc[i][j] = 0.0f;
      if (!PROMOTE) total[PROMOTE ? 0 : i][PROMOTE ? 0 : j] = 0;
    }
  bool timed_out = false;
  for (int64_t sp = 0; sp < p.nspans; ++sp) {
    const int s = (int)(sp % kStages);
    if (!mbar_wait(&full[s], (uint32_t)((sp / kStages) & 1), p.wait_polls)) timed_out = true;
    if (__syncthreads_or(timed_out)) {
      if (threadIdx.x == 0) {
        atomicExch(p.status, 1);
        // Spans sp .. sp + kStages - 1 may still be in flight: they land before the CTA exits.
        for (int64_t u = sp; u < sp + kStages && u < p.nspans; ++u) mbar_wait(&full[u % kStages], (uint32_t)((u / kStages) & 1));
      }
      return;
    }
    const Stage &st = stages[s];
    int d[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) d[i][j] = 0;
#pragma unroll 4
    for (int k4 = 0; k4 < kSpan / 4; ++k4) {
      const uint4 a0 = *reinterpret_cast<const uint4 *>(&st.a[k4][ty * 4]);
      const uint4 a1 = *reinterpret_cast<const uint4 *>(&st.a[k4][64 + ty * 4]);
      const uint4 b0 = *reinterpret_cast<const uint4 *>(&st.b[k4][tx * 4]);
      const uint4 b1 = *reinterpret_cast<const uint4 *>(&st.b[k4][64 + tx * 4]);
      const int av[8] = {(int)a0.x, (int)a0.y, (int)a0.z, (int)a0.w, (int)a1.x, (int)a1.y, (int)a1.z, (int)a1.w};
      const int bv[8] = {(int)b0.x, (int)b0.y, (int)b0.z, (int)b0.w, (int)b1.x, (int)b1.y, (int)b1.z, (int)b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) d[i][j] = __dp4a(av[i], bv[j], d[i][j]);
    }
    if (PROMOTE) {
      // This interval's scale columns (one division per span, not per output).
      const int64_t begin = sp * kSpan;
      const float *sac = p.sa ? p.sa + begin / p.sa_kd : nullptr;
      const float *sbc = p.sb ? p.sb + begin / p.sb_kd : nullptr;
      float wa[8], wb[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t m = mt * kTile + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        wa[i] = (sac && m < p.M) ? sac[m * p.sa_nkd] : 1.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t n = nt * kTile + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
        wb[j] = (sbc && n < p.N) ? sbc[n * p.sb_nkd] : 1.0f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // weight = (1 * sa) * sb, each an fp32 RN multiply; the interval's exact partial as fp32.
          float w = p.sa ? wa[i] : 1.0f;
          if (p.sb) w = __fmul_rn(w, wb[j]);
          acc[i][j] = __fmaf_rn((float)d[i][j], w, acc[i][j]);
        }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) total[PROMOTE ? 0 : i][PROMOTE ? 0 : j] += d[i][j];
    }
    __syncthreads();
    if (threadIdx.x == 0 && sp + kStages < p.nspans) issue(sp + kStages, s);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t m = mt * kTile + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
      const int64_t n = nt * kTile + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (m >= p.M || n >= p.N) continue;
      float v = PROMOTE ? acc[i][j] : fixed_to_fp32(total[PROMOTE ? 0 : i][PROMOTE ? 0 : j], p.exp_out, 0, true, false);
      store_out(p.g, m, n, epilogue(p.g, m, n, v));
    }
}

}  // namespace intk

struct IntPlan {
  bool ok, promote;
  int64_t nspans, a_pad, b_pad;
  size_t off[2], flag_off, total;
};

static int64_t int_max_abs(const Fmt &f) { return f.qmax > -f.qmin ? f.qmax : -f.qmin; }

static IntPlan plan_int(const GemmDesc &g) {
  IntPlan p;
  std::memset(&p, 0, sizeof(p));
  if (g.a.f.kind != 1 || g.b.f.kind != 1) return p;
  const int64_t ma = int_max_abs(g.a.f), mb = int_max_abs(g.b.f);
  if (ma > 127 || mb > 127) return p;
  if (g.alg == ALG_COFDA && g.apply == AP_PROMOTE && g.PI == intk::kSpan) {
    if (g.a.f.frac_bits != 0 || g.b.f.frac_bits != 0) return p;
    const int prec = g.F < 23 ? g.F : 23;
    if ((double)g.PI * (double)ma * (double)mb >= (double)(1ll << (prec + 1))) return p;
    for (const OpDesc *o : {&g.a, &g.b})
      if (o->skind == SK_K && o->kd % intk::kSpan) return p;
    p.promote = true;
  } else if (g.alg == ALG_INT_EXACT && g.apply == AP_EPILOGUE) {
    if ((double)ma * (double)mb * (double)intk::kSpan >= 2147483647.0) return p;
    p.promote = false;
  } else {
    return p;
  }
  p.nspans = (g.K + intk::kSpan - 1) / intk::kSpan;
  p.a_pad = (g.M + intk::kTile - 1) / intk::kTile * intk::kTile;
  p.b_pad = (g.N + intk::kTile - 1) / intk::kTile * intk::kTile;
  size_t sa = (size_t)p.a_pad * p.nspans * intk::kSpan, sb = (size_t)p.b_pad * p.nspans * intk::kSpan;
  p.off[0] = 0;
  p.off[1] = (sa + 255) & ~(size_t)255;
  p.flag_off = p.off[1] + ((sb + 255) & ~(size_t)255);
  p.total = p.flag_off + 256;
  p.ok = true;
  return p;
}

// Tensor-core version (tc_gemm_int_tc.cu): the same exact integers from tcgen05.mma kind::i8.
bool int_tc_eligible(const GemmDesc &g, bool promote, int64_t max_a, int64_t max_b);
size_t int_tc_workspace(const GemmDesc &g);
int launch_int_tc(const GemmDesc &g, bool promote, void *workspace, size_t workspace_bytes, cudaStream_t s);

static bool use_tc(const GemmDesc &g, const IntPlan &p) {
  return p.nspans > 0 && int_tc_eligible(g, p.promote, int_max_abs(g.a.f), int_max_abs(g.b.f));
}

size_t int_workspace(const GemmDesc &g) {
  IntPlan p = plan_int(g);
  if (!p.ok) return 0;
  return use_tc(g, p) ? int_tc_workspace(g) : p.total;
}

int launch_int(const GemmDesc &g, void *workspace, size_t workspace_bytes, cudaStream_t s) {
  IntPlan p = plan_int(g);
  if (!p.ok) return TC_UNSUPPORTED;
  if (use_tc(g, p)) {
    const int st = launch_int_tc(g, p.promote, workspace, workspace_bytes, s);
    if (st != TC_UNSUPPORTED) return st;
  }
  if (!workspace || workspace_bytes < p.total) return set_error("tc_gemm: workspace too small"), TC_WORKSPACE_TOO_SMALL;
  if ((g.M + intk::kTile - 1) / intk::kTile > 65535) return TC_UNSUPPORTED;
  char *ws = static_cast<char *>(workspace);
  int32_t *flag = reinterpret_cast<int32_t *>(ws + p.flag_off);
  cudaMemsetAsync(flag, 0, 2 * sizeof(int32_t), s);
  for (int side = 0; side < 2; ++side) {
    const OpDesc &o = side ? g.b : g.a;
    intk::EncodeArgs e;
    e.v = o.v;
    e.dt = o.dt;
    e.rows = o.rows;
    e.K = o.K;
    e.rows_pad = side ? p.b_pad : p.a_pad;
    e.nspans = p.nspans;
    e.frac = o.f.frac_bits;
    e.out = reinterpret_cast<uint32_t *>(ws + p.off[side]);
    e.flag = flag;
    int64_t work = e.rows_pad * p.nspans * (intk::kSpan / 4);
    int64_t blocks = (work + 255) / 256;
    if (blocks > (int64_t)sm_count() * 16) blocks = (int64_t)sm_count() * 16;
    intk::encode_kernel<<<(unsigned)blocks, 256, 0, s>>>(e);
    count_launch();
  }
  intk::Args a;
  std::memset(&a, 0, sizeof(a));
  a.aw = reinterpret_cast<const uint32_t *>(ws + p.off[0]);
  a.bw = reinterpret_cast<const uint32_t *>(ws + p.off[1]);
  a.M = g.M;
  a.N = g.N;
  a.nspans = p.nspans;
  a.promote = p.promote;
  a.exp_out = -(g.a.f.frac_bits + g.b.f.frac_bits);
  if (p.promote) {
    if (g.a.skind == SK_K) { a.sa = g.a.scale; a.sa_nkd = g.a.nkd; a.sa_kd = g.a.kd; }
    if (g.b.skind == SK_K) { a.sb = g.b.scale; a.sb_nkd = g.b.nkd; a.sb_kd = g.b.kd; }
  }
  a.g = g;
  a.flag = flag;
  a.status = flag + 1;
  a.wait_polls = wait_polls();
  size_t smem = sizeof(intk::Stage) * intk::kStages;
  auto kern = p.promote ? intk::int_kernel<true> : intk::int_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(std::string("int gemm: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  dim3 grid((unsigned)((g.N + intk::kTile - 1) / intk::kTile), (unsigned)((g.M + intk::kTile - 1) / intk::kTile));
  kern<<<grid, 256, smem, s>>>(a);
  count_launch();
  launch_generic(g, flag, s);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm int: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

}  // namespace tc
