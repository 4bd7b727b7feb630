// Per-layer error sums (TriCast analysis._ErrorStats.update, src/tricast/analysis.py:37-50):
// fp64 sum x^2, sum y^2, sum (x-y)^2, sum x*y and max |x-y| of a reference / emulated pair,
// added into a caller-owned device array so several slabs of one layer can be accumulated.
#include <string>

#include "tc_common.cuh"

namespace tc {

__device__ __forceinline__ void atomic_max_nonneg(double *addr, double v) {
  // Non-negative doubles order like their bit patterns.
  atomicMax(reinterpret_cast<unsigned long long *>(addr), (unsigned long long)__double_as_longlong(v));
}

__global__ void __launch_bounds__(256) error_stats_kernel(const void *__restrict__ ref, int rdt,
                                                          const void *__restrict__ emu, int edt, int64_t n,
                                                          double *__restrict__ sums) {
  double sx = 0, sy = 0, se = 0, sd = 0, mx = 0, bad = 0;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    double x = (double)load_as_float(ref, rdt, i);
    double y = (double)load_as_float(emu, edt, i);
    if (!isfinite(x) || !isfinite(y)) {
      bad += 1;
      continue;
    }
    double d = x - y;
    sx = __fma_rn(x, x, sx);
    sy = __fma_rn(y, y, sy);
    se = __fma_rn(d, d, se);
    sd = __fma_rn(x, y, sd);
    mx = fmax(mx, fabs(d));
  }
  for (int m = 16; m; m >>= 1) {
    sx += __shfl_xor_sync(0xFFFFFFFFu, sx, m);
    sy += __shfl_xor_sync(0xFFFFFFFFu, sy, m);
    se += __shfl_xor_sync(0xFFFFFFFFu, se, m);
    sd += __shfl_xor_sync(0xFFFFFFFFu, sd, m);
    mx = fmax(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, m));
    bad += __shfl_xor_sync(0xFFFFFFFFu, bad, m);
  }
  __shared__ double part[8][6];
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    part[w][0] = sx; part[w][1] = sy; part[w][2] = se; part[w][3] = sd; part[w][4] = mx; part[w][5] = bad;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double t[6] = {0, 0, 0, 0, 0, 0};
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
      for (int j = 0; j < 6; ++j) t[j] = j == 4 ? fmax(t[j], part[i][j]) : t[j] + part[i][j];
    }
    atomicAdd(&sums[0], t[0]);
    atomicAdd(&sums[1], t[1]);
    atomicAdd(&sums[2], t[2]);
    atomicAdd(&sums[3], t[3]);
    atomic_max_nonneg(&sums[4], t[4]);
    atomicAdd(&sums[5], t[5]);
  }
}

}  // namespace tc

extern "C" int tc_error_stats(const void *ref, int32_t ref_dtype, const void *emu, int32_t emu_dtype, int64_t n,
                              double *sums, tc_stream stream) {
  if (n <= 0) return TC_OK;
  if (!ref || !emu || !sums || ref_dtype < 0 || ref_dtype > 2 || emu_dtype < 0 || emu_dtype > 2) {
    tc::set_error("tc_error_stats: bad argument");
    return TC_INVALID_ARGUMENT;
  }
  int64_t blocks = (n + 255) / 256;
  if (blocks > (int64_t)tc::sm_count() * 4) blocks = (int64_t)tc::sm_count() * 4;
  tc::error_stats_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(ref, ref_dtype, emu, emu_dtype, n, sums);
  ::tc::count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    tc::set_error(std::string("tc_error_stats: ") + cudaGetErrorString(e));
    return TC_CUDA_ERROR;
  }
  return TC_OK;
}
