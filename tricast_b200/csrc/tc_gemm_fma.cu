// Fast FMA-chain kernels: the fp64 and fp32_fma algorithms (TriCast src/tricast/reference/mma.py:
// 359-371). Each output is one sequential chain over K in order, acc = fma(a_k, b_k, acc), in fp64
// (one rounding to fp32 at the end) or in IEEE fp32; with scale_apply == operand every element is
// first multiplied by its K scale in fp32. A 64 x 64 CTA tile stages 32-wide K slices of both
// operands through shared memory already converted to the accumulator type, so a thread's chain
// over its 4 x 4 outputs runs on registers and shared memory only, in the reference's K order.
#include <cstring>
#include <string>

#include "tc_gemm.cuh"

namespace tc {
namespace fmak {

constexpr int kTile = 64;
constexpr int kSlice = 32;

template <class T>
__global__ void __launch_bounds__(256) fma_kernel(GemmDesc g) {
  __shared__ T as[kSlice][kTile + 1];
  __shared__ T bs[kSlice][kTile + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * kTile, n0 = (int64_t)blockIdx.x * kTile;
  T acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = (T)0;
  const bool operand = g.apply == AP_OPERAND;
  for (int64_t k0 = 0; k0 < g.K; k0 += kSlice) {
    // Stage: thread t loads 8 elements of A and 8 of B (64 rows x 32 k each); consecutive threads
    // read consecutive k of one row.
    for (int e = threadIdx.x; e < kTile * kSlice; e += blockDim.x) {
      const int r = e / kSlice, kk = e % kSlice;
      const int64_t k = k0 + kk;
      float av = 0.0f, bv = 0.0f;
      const int64_t m = m0 + r, n = n0 + r;
      if (k < g.K) {
        if (m < g.M) {
          av = load_as_float(g.a.v, g.a.dt, m * g.K + k);
          if (operand && g.a.skind == SK_K) av = __fmul_rn(av, g.a.scale[m * g.a.nkd + k / g.a.kd]);
        }
        if (n < g.N) {
          bv = load_as_float(g.b.v, g.b.dt, n * g.K + k);
          if (operand && g.b.skind == SK_K) bv = __fmul_rn(bv, g.b.scale[n * g.b.nkd + k / g.b.kd]);
        }
      }
      as[kk][r] = (T)av;
      bs[kk][r] = (T)bv;
    }
    __syncthreads();
    const int kn = (int)(g.K - k0 < kSlice ? g.K - k0 : kSlice);
    for (int kk = 0; kk < kn; ++kk) {
      T a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = as[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if constexpr (sizeof(T) == 8) acc[i][j] = __fma_rn(a[i], b[j], acc[i][j]);
          else acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t m = m0 + ty * 4 + i, n = n0 + tx + 16 * j;
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
  if ((g.M + fmak::kTile - 1) / fmak::kTile > 65535) return TC_UNSUPPORTED;
  dim3 grid((unsigned)((g.N + fmak::kTile - 1) / fmak::kTile), (unsigned)((g.M + fmak::kTile - 1) / fmak::kTile));
  if (g.alg == ALG_FP64) fmak::fma_kernel<double><<<grid, 256, 0, s>>>(g);
  else fmak::fma_kernel<float><<<grid, 256, 0, s>>>(g);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm fma: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

}  // namespace tc
