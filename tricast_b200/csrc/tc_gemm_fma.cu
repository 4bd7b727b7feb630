// Fast FMA-chain kernels: the fp64 and fp32_fma algorithms (TriCast src/tricast/reference/mma.py:
// 359-371). Each output is one sequential chain over K in order, acc = fma(a_k, b_k, acc), in fp64
// (one rounding to fp32 at the end) or in IEEE fp32; with scale_apply == operand every element is
// first multiplied by its K scale in fp32.
//
// A CTA computes 128 rows x 64 columns; each of its 256 threads owns 8 rows x 4 columns (rows
// 8 ty .. 8 ty + 7, columns tx + 16 j), so one K step costs it 32 FMAs against 8 shared loads.
// Operands pass through shared memory in 16-wide K slices already converted to the accumulator
// type, double-buffered: the next slice's 16-byte global loads are in flight while the current one
// is computed. A partial last slice stops at K, so every chain is exactly the reference's.
#include <cstring>
#include <string>

#include "tc_gemm.cuh"

namespace tc {
namespace fmak {

constexpr int kRows = 128;  // rows of A per CTA
constexpr int kCols = 64;   // columns (rows of B) per CTA
constexpr int kKs = 16;     // K elements per slice

template <class T>
struct Slices {
  T a[2][kKs][kRows];
  T b[2][kKs][kCols];
};

// 8 consecutive elements of one row (k0 .. k0 + 7) as floats: one or two 16-byte loads when the row
// slice is whole and aligned, else element by element with zeros past K; scaled by the K scale
// first under scale_apply == operand.
struct Load8 {
  uint4 raw[2];
  bool vec;
};

__device__ __forceinline__ void fetch8(const OpDesc &o, int64_t row, int64_t nrows, int64_t k0, bool aligned,
                                       Load8 &l) {
  l.vec = aligned && row < nrows && k0 + 8 <= o.K;
  if (l.vec) {
    const int esz = o.dt == TC_F32 ? 4 : 2;
    const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const char *>(o.v) + (row * o.K + k0) * esz);
    l.raw[0] = src[0];
    if (esz == 4) l.raw[1] = src[1];
  }
}

__device__ __forceinline__ void unpack8(const OpDesc &o, int64_t row, int64_t nrows, int64_t k0, bool operand,
                                        const Load8 &l, float (&x)[8]) {
  if (l.vec) {
    if (o.dt == TC_F32) {
      const uint32_t w[8] = {l.raw[0].x, l.raw[0].y, l.raw[0].z, l.raw[0].w,
                             l.raw[1].x, l.raw[1].y, l.raw[1].z, l.raw[1].w};
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = u2f(w[i]);
    } else {
      const uint32_t w[4] = {l.raw[0].x, l.raw[0].y, l.raw[0].z, l.raw[0].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (o.dt == TC_BF16) {
          x[2 * i] = u2f(w[i] << 16);
          x[2 * i + 1] = u2f(w[i] & 0xFFFF0000u);
        } else {
          x[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xFFFFu)));
          x[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
        }
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      x[i] = (row < nrows && k0 + i < o.K) ? load_as_float(o.v, o.dt, row * o.K + k0 + i) : 0.0f;
  }
  if (operand && o.skind == SK_K && row < nrows) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (k0 + i < o.K) x[i] = __fmul_rn(x[i], o.scale[row * o.nkd + (k0 + i) / o.kd]);
  }
}

template <class T>
__global__ void __launch_bounds__(256, 2) fma_kernel(GemmDesc g) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Slices<T> &sl = *reinterpret_cast<Slices<T> *>(smem_raw);
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * kRows, n0 = (int64_t)blockIdx.x * kCols;
  const bool operand = g.apply == AP_OPERAND;
  // Load role: thread t stages row t / 2 of A and (t < 128) row t / 2 of B, elements 8 (t & 1) .. + 7
  // of the slice.
  const int lr = threadIdx.x >> 1, lh = (threadIdx.x & 1) * 8;
  const bool loads_b = threadIdx.x < 2 * kCols;
  const int esz_a = g.a.dt == TC_F32 ? 4 : 2, esz_b = g.b.dt == TC_F32 ? 4 : 2;
  const bool align_a = (uintptr_t)g.a.v % 16 == 0 && (g.K * esz_a) % 16 == 0;
  const bool align_b = (uintptr_t)g.b.v % 16 == 0 && (g.K * esz_b) % 16 == 0;
  Load8 la, lb;
  auto fetch = [&](int64_t k0) {
    fetch8(g.a, m0 + lr, g.M, k0 + lh, align_a, la);
    if (loads_b) fetch8(g.b, n0 + lr, g.N, k0 + lh, align_b, lb);
  };
  auto stage = [&](int buf, int64_t k0) {
    float x[8];
    unpack8(g.a, m0 + lr, g.M, k0 + lh, operand, la, x);
#pragma unroll
    for (int i = 0; i < 8; ++i) sl.a[buf][lh + i][lr] = (T)x[i];
    if (loads_b) {
      unpack8(g.b, n0 + lr, g.N, k0 + lh, operand, lb, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) sl.b[buf][lh + i][lr] = (T)x[i];
    }
  };

  T acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = (T)0;
  const int64_t nslices = (g.K + kKs - 1) / kKs;
  if (nslices > 0) {
    fetch(0);
    stage(0, 0);
  }
  __syncthreads();
  for (int64_t sidx = 0; sidx < nslices; ++sidx) {
    const int buf = (int)(sidx & 1);
    const int64_t k0 = sidx * kKs;
    if (sidx + 1 < nslices) fetch(k0 + kKs);  // in flight while this slice is computed
    const int kn = (int)(g.K - k0 < kKs ? g.K - k0 : kKs);
    for (int kk = 0; kk < kn; ++kk) {
      T a[8], b[4];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = sl.a[buf][kk][ty * 8 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sl.b[buf][kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if constexpr (sizeof(T) == 8) acc[i][j] = __fma_rn(a[i], b[j], acc[i][j]);
          else acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
    }
    // The other buffer was last read by the previous slice's computation, which every thread
    // finished before the barrier that ended it.
    if (sidx + 1 < nslices) stage(buf ^ 1, k0 + kKs);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t m = m0 + ty * 8 + i, n = n0 + tx + 16 * j;
      if (m >= g.M || n >= g.N) continue;
      float v;
      if constexpr (sizeof(T) == 8) v = __double2float_rn(acc[i][j]);
      else v = acc[i][j];
      store_out(g, m, n, epilogue(g, m, n, v));
    }
}

}  // namespace fmak

int launch_fma(const GemmDesc &g, cudaStream_t s) {
  if (g.alg != ALG_FP64 && g.alg != ALG_FP32_FMA) return TC_UNSUPPORTED;
  if ((g.M + fmak::kRows - 1) / fmak::kRows > 65535) return TC_UNSUPPORTED;
  dim3 grid((unsigned)((g.N + fmak::kCols - 1) / fmak::kCols), (unsigned)((g.M + fmak::kRows - 1) / fmak::kRows));
  cudaError_t e;
  if (g.alg == ALG_FP64) {
    const int smem = (int)sizeof(fmak::Slices<double>);
    e = cudaFuncSetAttribute(fmak::fma_kernel<double>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) fmak::fma_kernel<double><<<grid, 256, smem, s>>>(g);
  } else {
    const int smem = (int)sizeof(fmak::Slices<float>);
    e = cudaFuncSetAttribute(fmak::fma_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) fmak::fma_kernel<float><<<grid, 256, smem, s>>>(g);
  }
  if (e != cudaSuccess) return set_error(std::string("tc_gemm fma: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  count_launch();
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm fma: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

}  // namespace tc
