// Small-M CoFDA kernel (M <= 16) for narrow float operands: the decode shapes of the FP8 presets
// (nvidia_hopper_fp8, nvidia_ada_fp8, nvidia_blackwell_fp8, deepseek_fp8_promote128), TriCast's
// _gemv (src/tricast/kernels/mma.py:663-720) in its cofda mode.
//
// Arithmetic: the tiled kernel's (tc_gemm_cofda.cu). For a chunk of CS products and running value c,
// emax is the largest exponent label, each product's aligned term is fma.rz(P, 2**(F - emax), +-2**23)
// -+ 2**23 (2**52 in fp64 for wide radices), the partial sums are exact, and the exact integer total is
// normalised by the reference's fixed-point rule.
//
// Work split: LG lanes share one output (m, n); a chunk's CS products are split CS / LG per lane, the
// label maximum and the exact term sum are combined with xor shuffles. A CTA owns `cols` columns and
// all M rows; K advances in steps of 4096 / cols elements. B is read once, straight from its
// container: each thread decodes 16 consecutive elements of one column (on-grid check, exponent
// label, folded power-of-two K scale) into a double-buffered shared-memory stage, and the raw values
// of the next step are loaded into registers before the current step is scanned. A is decoded once
// by prep_a_kernel into [M][Kp] values and int16 labels (read through the L1).
//
// Elements the fast path cannot take (NaN / Inf, off-grid, beyond the format's exponent range,
// non-power-of-two or out-of-range product scales) raise the device flag; the exact generic kernel
// queued behind this one then recomputes every output.
#include <algorithm>
#include <cstring>
#include <string>

#include "tc_bulk.cuh"
#include "tc_cofda.cuh"

namespace tc {
namespace cgemv {

constexpr int kThreads = 256;
constexpr int kPerThread = 16;     // B elements decoded per thread and step
constexpr int kMaxKC = 1024;       // K elements per step (at least 4 columns per CTA)
constexpr int kPad = 8;            // column padding of the stage (elements)

template <class T>
struct Args {
  const T *aval;             // A decoded values, folded power-of-two K scales [M][Kp]
  const int16_t *aexp;       // A exponent labels [M][Kp]
  int64_t Kp;
  const void *bv;            // B values [N][K] in their container
  int bdt, bvec;             // bvec: B rows start 16-byte aligned
  Fmt bf;
  const float *bscale;       // B product-mode K scales (folded) or nullptr; b_kd % 16 == 0
  int64_t b_nkd;
  int b_kd, b_field0;
  Fmt bsf;
  int64_t M, N, K, nchunks;
  int F, cols, KC, rne, PI_chunks;
  int dec, F2;               // decoupled accumulator (no promotion) and its merge radix
  const float *sa, *sb;      // promote K scales or nullptr
  int64_t sa_nkd, sb_nkd;
  int sa_kd, sb_kd;
  GemmDesc g;                // epilogue
  int32_t *flag;             // nonzero: the fast path cannot take the operands
  const T *bval_enc;         // pre-encoded B (tc_encode_b): values [N][Kp] as prep_a_kernel writes them
  const int16_t *bexp_enc;   // and labels
};

struct PrepArgs {
  const void *v;
  int dt;
  int64_t rows, K, Kp;
  Fmt f;
  const float *scale;        // product-mode K scales or nullptr
  int64_t nkd;
  int kd;
  Fmt sf;
  int field0;
  void *val;                 // [rows][Kp], float or double
  int16_t *exp;
  int32_t *flag;
};

// A's elements decoded as the tiled kernel's encoder does (tc_gemm_cofda.cu encode_kernel).
template <class T>
__global__ void __launch_bounds__(256) prep_a_kernel(PrepArgs e) {
  const int64_t total = e.rows * e.Kp;
  bool bad = false;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / e.Kp, k = idx % e.Kp;
    float v = 0.0f;
    int ex = cofda::kZeroExp;
    if (k < e.K) {
      v = load_as_float(e.v, e.dt, r * e.K + k);
      if (!cofda::decode_elem(v, e.f, ex)) bad = true;
      if (e.scale) {
        const float s = e.scale[r * e.nkd + k / e.kd];
        const Term ts = decode_term(s, e.sf);
        const bool zero = ts.zero || (e.field0 && f2u(s) == 0x00400000u);
        if (ts.nan || ts.inf || (!zero && (ts.sig != 1 || ts.neg))) bad = true;  // pow2 scales only
        if (zero || ex == cofda::kZeroExp) {
          v = 0.0f;
          ex = cofda::kZeroExp;
        } else {
          if (ts.exp < -60 || ts.exp > 60 || ex + ts.exp < -50 || ex + ts.exp > 60) bad = true;
          v = ldexpf(v, ts.exp);
          ex += ts.exp;
        }
      }
    }
    if (ex == cofda::kZeroExp) v = 0.0f;
    static_cast<T *>(e.val)[idx] = (T)v;
    e.exp[idx] = (int16_t)(bad ? cofda::kZeroExp : ex);
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicExch(e.flag, 1);
}

// One B element: value with its folded scale (exponent s_exp, or zero) and exponent label. A value
// the fast path cannot take sets bad (its outputs are then recomputed by the exact kernel).
__device__ __forceinline__ void decode_b(float x, const Fmt &f, int s_exp, bool s_zero, float &v, int &e, bool &bad) {
  // Branch-free: every test is evaluated and folded into `bad` (a rejected element sends the whole
  // product to the exact kernel, so its value and label do not matter). Zero elements and elements
  // under a zero K scale are zero product terms; fp32 subnormals (below every narrow grid), NaN / Inf,
  // off-grid values, exponents beyond the format and folded exponents outside [-50, 60] are rejected.
  const uint32_t u = f2u(x), a = u & 0x7FFFFFFFu;
  const uint32_t field = a >> 23;
  const int fl = (int)field - 127;
  const int ee = fl > f.emin ? fl : f.emin;
  const int sh = 23 - f.mbits + (ee - fl);  // fraction bits below the grid, all zero on the grid
  const uint32_t below = sh > 23 ? 0xFFFFFFFFu : (1u << sh) - 1u;
  const bool nz = a != 0;
  const bool live = nz & !s_zero;
  const int ef = ee + s_exp;
  bad |= nz & ((field == 0) | (field == 255));
  bad |= live & ((ee > f.emax) | ((a & below) != 0u) | (ef < -50) | (ef > 60));
  e = live ? ef : cofda::kZeroExp;
  v = live ? u2f(u + ((uint32_t)s_exp << 23)) : 0.0f;  // exact: the folded value stays a normal fp32 number
}

template <class T, int N>
__device__ __forceinline__ void load_vec(const T *p, T (&o)[N]) {
  if (N * sizeof(T) >= 16) {
#pragma unroll
    for (int i = 0; i < N * (int)sizeof(T) / 16; ++i) {
      const uint4 w = *reinterpret_cast<const uint4 *>(reinterpret_cast<const char *>(p) + 16 * i);
      memcpy(reinterpret_cast<char *>(o) + 16 * i, &w, 16);
    }
  } else if (N * sizeof(T) == 8) {
    const uint2 w = *reinterpret_cast<const uint2 *>(p);
    memcpy(o, &w, 8);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) o[i] = p[i];
  }
}

template <int N>
__device__ __forceinline__ void load_labels(const int16_t *p, int (&o)[N]) {
  int16_t t[N];
  if (N * 2 >= 16) {
#pragma unroll
    for (int i = 0; i < N * 2 / 16; ++i) {
      const uint4 w = *reinterpret_cast<const uint4 *>(p + 8 * i);
      memcpy(t + 8 * i, &w, 16);
    }
  } else if (N * 2 == 8) {
    const uint2 w = *reinterpret_cast<const uint2 *>(p);
    memcpy(t, &w, 8);
  } else if (N * 2 == 4) {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(p);
    memcpy(t, &w, 4);
  } else {
    t[0] = p[0];
  }
#pragma unroll
  for (int i = 0; i < N; ++i) o[i] = t[i];
}

template <int LG, class T>
__device__ __forceinline__ T group_sum(T v) {
#pragma unroll
  for (int o = LG / 2; o > 0; o >>= 1) v = cofda::Acc<T>::add(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

template <int LG>
__device__ __forceinline__ int group_max(int v) {
#pragma unroll
  for (int o = LG / 2; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// BENC: B arrives pre-encoded (values and labels [N][Kp], prep_a_kernel's layout) and is staged with
// asynchronous copies one step ahead, like A, instead of being loaded and decoded here.
template <int CS, int LG, class T, bool BENC>
__global__ void __launch_bounds__(kThreads) cofda_gemv_kernel(Args<T> p) {
  constexpr int PL = CS / LG;  // products per lane per chunk
  if (*p.flag) return;         // A could not be decoded: the generic kernel takes over
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int stride = p.KC + kPad;  // row stride of a stage (elements)
  // Dynamic shared memory: B values [2][cols][stride], B labels (same shape), A values [2][M][stride],
  // A labels (same shape).
  T *bval = reinterpret_cast<T *>(smem_raw);
  int16_t *bexp = reinterpret_cast<int16_t *>(bval + 2 * (size_t)p.cols * stride);
  T *aval_s = reinterpret_cast<T *>(bexp + 2 * (size_t)p.cols * stride);
  int16_t *aexp_s = reinterpret_cast<int16_t *>(aval_s + 2 * (size_t)p.M * stride);
  const int64_t n0 = (int64_t)blockIdx.x * p.cols;
  const int M = (int)p.M;
  // Load role: 16 consecutive elements of one column.
  const int le = threadIdx.x * kPerThread;
  const bool loader = le < p.cols * p.KC;  // the stage holds cols x KC elements of B
  const int lcol = loader ? le / p.KC : 0, lk = loader ? le % p.KC : 0;
  const int64_t ln = loader ? n0 + lcol : p.N;  // idle loaders decode nothing
  // Scan role: LG lanes per slot, slot -> (row, column).
  const int slot = threadIdx.x / LG, j = threadIdx.x % LG;
  const int sm = slot % M, scol = slot / M;
  const bool active = scol < p.cols && n0 + scol < p.N;
  const int scol_c = scol < p.cols ? scol : 0;  // idle slots scan column 0 and store nothing
  const int64_t sn = n0 + scol;
  const int esz = p.bdt == TC_F32 ? 4 : 2;
  const int64_t nsteps = (p.K + p.KC - 1) / p.KC;
  const int chunks_per_step = p.KC / CS;
  float c = 0.0f, acc = 0.0f;
  bool bad = false;

  uint4 raw[4];
  auto fetch = [&](int64_t step) {
    const int64_t k = step * p.KC + lk;
    if (ln < p.N && p.bvec && k + kPerThread <= p.K) {
      const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const char *>(p.bv) + (ln * p.K + k) * esz);
      raw[0] = __ldcs(src);
      raw[1] = __ldcs(src + 1);
      if (esz == 4) {
        raw[2] = __ldcs(src + 2);
        raw[3] = __ldcs(src + 3);
      }
    }
  };
  // A's values and labels of one step into slot step & 1 (rows padded to whole steps in global memory).
  auto copy_a = [&](int64_t step) {
    const int slot = (int)(step & 1);
    const int vpr = p.KC * (int)sizeof(T) / 16, epr = p.KC * 2 / 16;  // 16-byte pieces per row
    for (int i = threadIdx.x; i < M * (vpr + epr); i += kThreads) {
      const int m = i / (vpr + epr), r = i % (vpr + epr);
      if (r < vpr)
        cp_async16(reinterpret_cast<char *>(aval_s + ((size_t)slot * M + m) * stride) + 16 * r,
                   reinterpret_cast<const char *>(p.aval + m * p.Kp + step * p.KC) + 16 * r);
      else
        cp_async16(reinterpret_cast<char *>(aexp_s + ((size_t)slot * M + m) * stride) + 16 * (r - vpr),
                   reinterpret_cast<const char *>(p.aexp + m * p.Kp + step * p.KC) + 16 * (r - vpr));
    }
    cp_async_commit();
  };
  // B's values and labels of one step into slot step & 1 (pre-encoded B only).
  auto copy_b = [&](int64_t step) {
    const int slot = (int)(step & 1);
    const int vpr = p.KC * (int)sizeof(T) / 16, epr = p.KC * 2 / 16;
    for (int i = threadIdx.x; i < p.cols * (vpr + epr); i += kThreads) {
      const int c = i / (vpr + epr), r = i % (vpr + epr);
      if (n0 + c >= p.N) continue;  // columns past N are scanned by idle slots only
      if (r < vpr)
        cp_async16(reinterpret_cast<char *>(bval + ((size_t)slot * p.cols + c) * stride) + 16 * r,
                   reinterpret_cast<const char *>(p.bval_enc + (n0 + c) * p.Kp + step * p.KC) + 16 * r);
      else
        cp_async16(reinterpret_cast<char *>(bexp + ((size_t)slot * p.cols + c) * stride) + 16 * (r - vpr),
                   reinterpret_cast<const char *>(p.bexp_enc + (n0 + c) * p.Kp + step * p.KC) + 16 * (r - vpr));
    }
    cp_async_commit();
  };
  copy_a(0);
  if constexpr (BENC) copy_b(0);
  else fetch(0);
  for (int64_t step = 0; step < nsteps; ++step) {
    const int buf = (int)(step & 1);
    T *sv = bval + (size_t)buf * p.cols * stride;
    int16_t *se = bexp + (size_t)buf * p.cols * stride;
    if constexpr (!BENC) {
      const int64_t k = step * p.KC + lk;
      float x[kPerThread];
      if (ln < p.N && p.bvec && k + kPerThread <= p.K) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const uint32_t uu[4] = {raw[w].x, raw[w].y, raw[w].z, raw[w].w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            if (esz == 4) {
              x[4 * w + h] = u2f(uu[h]);
            } else if (w < 2) {
              const int i = 8 * w + 2 * h;
              if (p.bdt == TC_BF16) {
                x[i] = u2f(uu[h] << 16);
                x[i + 1] = u2f(uu[h] & 0xFFFF0000u);
              } else {
                x[i] = __half2float(__ushort_as_half((unsigned short)(uu[h] & 0xFFFF)));
                x[i + 1] = __half2float(__ushort_as_half((unsigned short)(uu[h] >> 16)));
              }
            }
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < kPerThread; ++i)
          x[i] = (ln < p.N && k + i < p.K) ? load_as_float(p.bv, p.bdt, ln * p.K + k + i) : 0.0f;
      }
      int s_exp = 0;
      bool s_zero = false;
      if (p.bscale && ln < p.N && k < p.K) {
        const float s = p.bscale[ln * p.b_nkd + k / p.b_kd];
        const Term ts = decode_term(s, p.bsf);
        s_zero = ts.zero || (p.b_field0 && f2u(s) == 0x00400000u);
        if (ts.nan || ts.inf || (!s_zero && (ts.sig != 1 || ts.neg || ts.exp < -60 || ts.exp > 60))) bad = true;
        s_exp = s_zero ? 0 : ts.exp;
      }
      T vals[kPerThread];
      int16_t labs[kPerThread];
#pragma unroll
      for (int i = 0; i < kPerThread; ++i) {
        float v;
        int e;
        decode_b(x[i], p.bf, s_exp, s_zero, v, e, bad);
        vals[i] = (T)v;
        labs[i] = (int16_t)e;
      }
      if (loader) {
#pragma unroll
        for (int i = 0; i < kPerThread * (int)sizeof(T) / 16; ++i)
          *reinterpret_cast<uint4 *>(reinterpret_cast<char *>(sv + (size_t)lcol * stride + lk) + 16 * i) =
              *reinterpret_cast<const uint4 *>(reinterpret_cast<const char *>(vals) + 16 * i);
        *reinterpret_cast<uint4 *>(se + (size_t)lcol * stride + lk) = *reinterpret_cast<const uint4 *>(labs);
        *reinterpret_cast<uint4 *>(se + (size_t)lcol * stride + lk + 8) = *reinterpret_cast<const uint4 *>(labs + 8);
      }
    }
    if constexpr (!BENC)
      if (step + 1 < nsteps) fetch(step + 1);  // in flight while this step is scanned
    cp_async_wait_all();                       // this step's A (and pre-encoded B), issued one step earlier
    __syncthreads();
    // The other slots were last read by the previous step's scan, which every thread has finished.
    if (step + 1 < nsteps) {
      copy_a(step + 1);
      if constexpr (BENC) copy_b(step + 1);
    }
    const T *bv_col = sv + (size_t)scol_c * stride + j * PL;
    const int16_t *be_col = se + (size_t)scol_c * stride + j * PL;
    const T *av_row = aval_s + ((size_t)(step & 1) * M + sm) * stride + j * PL;
    const int16_t *ae_row = aexp_s + ((size_t)(step & 1) * M + sm) * stride + j * PL;
    for (int cl = 0; cl < chunks_per_step; ++cl) {
      const int64_t gch = step * chunks_per_step + cl;
      if (gch >= p.nchunks) break;  // uniform across the CTA
      T a[PL], b[PL];
      int ea[PL], eb[PL];
      load_vec<T, PL>(av_row + cl * CS, a);
      load_labels<PL>(ae_row + cl * CS, ea);
      load_vec<T, PL>(bv_col + cl * CS, b);
      load_labels<PL>(be_col + cl * CS, eb);
      int pe = cofda::kZeroExp;
#pragma unroll
      for (int i = 0; i < PL; ++i) pe = max(pe, ea[i] + eb[i]);
      pe = group_max<LG>(pe);
      const int emax = p.dec ? pe : max(cofda::running_exp(c), pe);  // decoupled: c is not in the chunk
      const T S = cofda::Acc<T>::pow2(p.F - emax);
      T tot = (T)0;
#pragma unroll
      for (int i = 0; i < PL; ++i) tot = cofda::Acc<T>::add(tot, cofda::Acc<T>::trunc(cofda::Acc<T>::mul(a[i], b[i]), S));
      tot = group_sum<LG, T>(tot);
      if (!p.dec) tot = cofda::Acc<T>::add(tot, cofda::Acc<T>::running(c, p.F, emax, S));
      const float nc = cofda::Acc<T>::finish(tot, emax, p.F, p.rne != 0);
      if (p.dec) c = cofda::merge_decoupled(nc, c, p.F2, p.rne != 0);
      else c = (f2u(c) & 0x7FFFFFFFu) >= kInf ? c : nc;  // an overflowed running value is sticky
      if (p.PI_chunks && ((gch + 1) % p.PI_chunks == 0 || gch + 1 == p.nchunks)) {
        // End of a promote interval: acc = fma(partial, (1 * sa) * sb, acc), partial restarts at 0.
        const int64_t begin = (gch / p.PI_chunks) * (int64_t)p.PI_chunks * CS;
        float w = 1.0f;
        if (active) {
          if (p.sa) w = __fmul_rn(w, p.sa[sm * p.sa_nkd + begin / p.sa_kd]);
          if (p.sb) w = __fmul_rn(w, p.sb[sn * p.sb_nkd + begin / p.sb_kd]);
        }
        acc = __fmaf_rn(c, w, acc);
        c = 0.0f;
      }
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicExch(p.flag, 1);
  if (active && j == 0) store_out(p.g, sm, sn, epilogue(p.g, sm, sn, p.PI_chunks ? acc : c));
}

}  // namespace cgemv

// ---------------------------------------------------------------- host side
struct CofdaGemvPlan {
  int64_t Kp;
  size_t off_val, off_exp, off_flag, total;
};

static CofdaGemvPlan plan_cofda_gemv(const GemmDesc &g, bool wide) {
  CofdaGemvPlan p;
  p.Kp = (g.K + cgemv::kMaxKC - 1) / cgemv::kMaxKC * cgemv::kMaxKC;
  const size_t n = (size_t)g.M * p.Kp;
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  p.off_val = 0;
  p.off_exp = up(n * (wide ? 8 : 4));
  p.off_flag = p.off_exp + up(n * 2);
  p.total = p.off_flag + 256;
  return p;
}

// The caller (launch_cofda) checked the tiled kernel's preconditions; the small-M kernel also needs
// B's folded product scales to change at most every 16 elements.
bool cofda_gemv_eligible(const GemmDesc &g) {
  if (g.M > 16) return false;
  if (g.apply == AP_PRODUCT && g.b.skind == SK_K && g.b.kd % 16) return false;
  return true;
}

size_t cofda_gemv_workspace(const GemmDesc &g, bool wide) { return plan_cofda_gemv(g, wide).total; }

// A pre-encoded B of the small-M path: B's elements decoded as A's are (values with the folded
// power-of-two product scales, and labels), [N][Kp] each, then a flag word set when B cannot be taken.
struct CofdaGemvBLayout {
  int64_t Kp;
  size_t off_val, off_exp, off_flag, total;
};

static CofdaGemvBLayout cofda_gemv_b_layout(const GemmDesc &g, bool wide) {
  CofdaGemvBLayout l;
  l.Kp = (g.K + cgemv::kMaxKC - 1) / cgemv::kMaxKC * cgemv::kMaxKC;
  const size_t n = (size_t)g.N * l.Kp;
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  l.off_val = 0;
  l.off_exp = up(n * (wide ? 8 : 4));
  l.off_flag = l.off_exp + up(n * 2);
  l.total = l.off_flag + 256;
  return l;
}

size_t cofda_gemv_b_bytes(const GemmDesc &g, bool wide) { return cofda_gemv_b_layout(g, wide).total; }

int encode_cofda_gemv_b(const GemmDesc &g, bool wide, void *enc, cudaStream_t s) {
  const CofdaGemvBLayout l = cofda_gemv_b_layout(g, wide);
  char *e = static_cast<char *>(enc);
  int32_t *flag = reinterpret_cast<int32_t *>(e + l.off_flag);
  cudaMemsetAsync(flag, 0, sizeof(int32_t), s);
  if (g.N > 0 && l.Kp > 0) {
    cgemv::PrepArgs pa;
    std::memset(&pa, 0, sizeof(pa));
    pa.v = g.b.v;
    pa.dt = g.b.dt;
    pa.rows = g.N;
    pa.K = g.K;
    pa.Kp = l.Kp;
    pa.f = g.b.f;
    pa.scale = (g.apply == AP_PRODUCT && g.b.skind == SK_K) ? g.b.scale : nullptr;
    pa.nkd = g.b.nkd;
    pa.kd = g.b.kd;
    pa.sf = g.b.sf;
    pa.field0 = g.b.field0;
    pa.val = e + l.off_val;
    pa.exp = reinterpret_cast<int16_t *>(e + l.off_exp);
    pa.flag = flag;
    const int64_t work = g.N * l.Kp;
    const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 8);
    if (wide) cgemv::prep_a_kernel<double><<<(unsigned)blocks, 256, 0, s>>>(pa);
    else cgemv::prep_a_kernel<float><<<(unsigned)blocks, 256, 0, s>>>(pa);
    count_launch();
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(std::string("tc_encode_b: ") + cudaGetErrorString(err)), TC_CUDA_ERROR;
  return TC_OK;
}

template <int CS, int LG, class T, bool BENC>
static int launch_cofda_gemv_b(const cgemv::Args<T> &a, cudaStream_t s) {
  const size_t smem = 2 * (size_t)(a.cols + a.M) * (a.KC + cgemv::kPad) * (sizeof(T) + 2);
  cudaError_t e = cudaFuncSetAttribute(cgemv::cofda_gemv_kernel<CS, LG, T, BENC>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(std::string("cofda gemv: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  const unsigned grid = (unsigned)((a.N + a.cols - 1) / a.cols);
  cgemv::cofda_gemv_kernel<CS, LG, T, BENC><<<grid, cgemv::kThreads, smem, s>>>(a);
  count_launch();
  return TC_OK;
}

template <int CS, int LG, class T>
static int launch_cofda_gemv_t(const cgemv::Args<T> &a, cudaStream_t s) {
  return a.bval_enc ? launch_cofda_gemv_b<CS, LG, T, true>(a, s) : launch_cofda_gemv_b<CS, LG, T, false>(a, s);
}

template <int LG, class T>
static int launch_cofda_gemv_cs(const cgemv::Args<T> &a, int CS, cudaStream_t s) {
  if (CS == 32) return launch_cofda_gemv_t<32, LG, T>(a, s);
  if (CS == 16) return launch_cofda_gemv_t<16, LG, T>(a, s);
  return launch_cofda_gemv_t<8, LG, T>(a, s);
}

template <class T>
static int launch_cofda_gemv_typed(const GemmDesc &g, const CofdaGemvPlan &p, char *ws, int32_t *flag,
                                   const char *benc, cudaStream_t s) {
  if (g.M > 0 && p.Kp > 0) {
    cgemv::PrepArgs e;
    std::memset(&e, 0, sizeof(e));
    e.v = g.a.v;
    e.dt = g.a.dt;
    e.rows = g.M;
    e.K = g.K;
    e.Kp = p.Kp;
    e.f = g.a.f;
    e.scale = (g.apply == AP_PRODUCT && g.a.skind == SK_K) ? g.a.scale : nullptr;
    e.nkd = g.a.nkd;
    e.kd = g.a.kd;
    e.sf = g.a.sf;
    e.field0 = g.a.field0;
    e.val = ws + p.off_val;
    e.exp = reinterpret_cast<int16_t *>(ws + p.off_exp);
    e.flag = flag;
    const int64_t work = g.M * p.Kp;
    const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 8);
    cgemv::prep_a_kernel<T><<<(unsigned)blocks, 256, 0, s>>>(e);
    count_launch();
  }
  cgemv::Args<T> a;
  std::memset(&a, 0, sizeof(a));
  a.aval = reinterpret_cast<const T *>(ws + p.off_val);
  a.aexp = reinterpret_cast<const int16_t *>(ws + p.off_exp);
  a.Kp = p.Kp;
  a.bv = g.b.v;
  a.bdt = g.b.dt;
  const int besz = g.b.dt == TC_F32 ? 4 : 2;
  a.bvec = ((uintptr_t)g.b.v % 16 == 0) && ((g.b.K * besz) % 16 == 0);
  a.bf = g.b.f;
  if (g.apply == AP_PRODUCT && g.b.skind == SK_K) {
    a.bscale = g.b.scale;
    a.b_nkd = g.b.nkd;
    a.b_kd = g.b.kd;
    a.bsf = g.b.sf;
    a.b_field0 = g.b.field0;
  }
  a.M = g.M;
  a.N = g.N;
  a.K = g.K;
  a.nchunks = (g.K + g.CS - 1) / g.CS;
  a.F = g.F;
  a.rne = g.rne;
  a.PI_chunks = g.apply == AP_PROMOTE ? g.PI / g.CS : 0;
  a.dec = g.decoupled && !g.PI;  // with a promote interval the reference accumulates fused
  a.F2 = g.F2;
  if (g.apply == AP_PROMOTE) {
    if (g.a.skind == SK_K) { a.sa = g.a.scale; a.sa_nkd = g.a.nkd; a.sa_kd = g.a.kd; }
    if (g.b.skind == SK_K) { a.sb = g.b.scale; a.sb_nkd = g.b.nkd; a.sb_kd = g.b.kd; }
  }
  a.g = g;
  a.flag = flag;
  if (benc) {
    const CofdaGemvBLayout l = cofda_gemv_b_layout(g, sizeof(T) == 8);
    a.bval_enc = reinterpret_cast<const T *>(benc + l.off_val);
    a.bexp_enc = reinterpret_cast<const int16_t *>(benc + l.off_exp);
  }
  // Lanes per output: 16 for a single row (twice the CTAs of 8 lanes: 256 for N = 4096), 8 while few
  // rows leave the GPU short of threads, else 4; at least two products per lane and chunk. Columns
  // per CTA: the largest power of two whose M x cols slots fit the CTA.
  const int LG = (g.M == 1 && g.CS >= 32) ? 16 : (g.M <= 4 ? 8 : 4);
  const int slots = cgemv::kThreads / LG;
  int cols = 1;
  while (cols * 2 * g.M <= slots) cols *= 2;
  a.cols = cols;
  // K elements per step: stages of at most 4096 (fp32) / 2048 (fp64) elements of B and of A.
  int mp = 1;
  while (mp < g.M) mp *= 2;
  a.KC = (sizeof(T) == 4 ? 4096 : 2048) / std::max(cols, mp);
  if (LG == 16) return launch_cofda_gemv_t<32, 16, T>(a, s);
  return LG == 8 ? launch_cofda_gemv_cs<8, T>(a, g.CS, s) : launch_cofda_gemv_cs<4, T>(a, g.CS, s);
}

int launch_cofda_gemv(const GemmDesc &g, bool wide, void *workspace, size_t workspace_bytes, cudaStream_t s,
                      const void *benc) {
  const CofdaGemvPlan p = plan_cofda_gemv(g, wide);
  if (!workspace || workspace_bytes < p.total) return set_error("tc_gemm: workspace too small"), TC_WORKSPACE_TOO_SMALL;
  char *ws = static_cast<char *>(workspace);
  int32_t *flag = reinterpret_cast<int32_t *>(ws + p.off_flag);
  cudaMemsetAsync(flag, 0, 2 * sizeof(int32_t), s);  // [0] operands rejected, [1] timeout: both gate the generic kernel
  const char *b = static_cast<const char *>(benc);
  if (b)  // a B the encoder rejected gates this product like an A rejected now
    cudaMemcpyAsync(flag, b + cofda_gemv_b_layout(g, wide).off_flag, sizeof(int32_t), cudaMemcpyDeviceToDevice, s);
  const int st = wide ? launch_cofda_gemv_typed<double>(g, p, ws, flag, b, s)
                      : launch_cofda_gemv_typed<float>(g, p, ws, flag, b, s);
  if (st) return st;
  launch_generic(g, flag, s);  // runs only when an operand raised the flag
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm cofda gemv: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

}  // namespace tc
