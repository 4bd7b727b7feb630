// Silicon probe: the B200's own FP8 tensor-core MMA (tcgen05.mma kind::f8f6f4, fp32 accumulation in
// TMEM) on raw E4M3 / E5M2 codes, so that its results can be compared bit for bit with the emulated
// accumulation models (does a preset reproduce the silicon?). It computes D = A * B^T with no scales:
// the MMA is issued over K in slabs of 32 (one instruction each, in K order), accumulating into one
// fp32 accumulator, which is what a kernel on this hardware would do.
//
// CTA: 128 rows of A x 64 columns of B, 128 threads. K advances in stages of 128: the threads copy the
// stage's codes into shared memory in the UMMA K-major no-swizzle layout (element (r, k) at byte
// (k / 16) * rows * 16 + r * 16 + k % 16), fence them for the tensor core, and thread 0 issues four
// M128 N64 K32 MMAs and commits them to an mbarrier; every thread waits (bounded) before the stage is
// overwritten. Warp w then reads TMEM lanes 32 w .. +31 (rows) with tcgen05.ld. A wait that runs out
// sets the status word and the kernel frees TMEM and returns; the host reports an error.
#include <algorithm>
#include <cstring>
#include <string>

#include "tc_bulk.cuh"
#include "tc_common.cuh"
#include "tc_tcgen05.cuh"

namespace tc {
namespace probe {

constexpr int kM = 128, kN = 64, kKS = 128;  // tile rows, columns, K per stage
constexpr uint32_t kTmemCols = 64;

// Instruction descriptor, kind::f8f6f4: D fp32 (bits 4-5 = 1), A and B format (bits 7-9, 10-12:
// 0 E4M3, 1 E5M2), both K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_f8(int fmt, int M, int N) {
  return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %4, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(accumulate), "r"(idesc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__global__ void __launch_bounds__(128, 1) mma_fp8_kernel(const uint8_t *__restrict__ a, const uint8_t *__restrict__ b,
                                                         int64_t M, int64_t N, int64_t K, int fmt,
                                                         float *__restrict__ out, int32_t *status) {
  __shared__ __align__(1024) uint8_t sa[kM * kKS];
  __shared__ __align__(1024) uint8_t sb[kN * kKS];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = (int64_t)blockIdx.y * kM, n0 = (int64_t)blockIdx.x * kN;
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    fence_barrier_init();
  }
  if (warp == 0) tc5::tmem_alloc(&tmem_base, kTmemCols);
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tbase = tmem_base;
  const uint32_t idesc = idesc_f8(fmt, kM, kN);
  bool ok = true;
  const int64_t nstages = (K + kKS - 1) / kKS;
  int64_t st = 0;
  for (; st < nstages && ok; ++st) {
    // Stage the codes (zero beyond M, N and K) in the canonical layout, 16 bytes per thread and step.
    for (int i = threadIdx.x; i < (kM + kN) * (kKS / 16); i += blockDim.x) {
      const bool isa = i < kM * (kKS / 16);
      const int j = isa ? i : i - kM * (kKS / 16);
      const int rows = isa ? kM : kN;
      const int r = j % rows, c16 = j / rows;
      const int64_t row = (isa ? m0 : n0) + r, rows_total = isa ? M : N;
      const uint8_t *src = isa ? a : b;
      uint8_t bytes[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int64_t k = st * kKS + c16 * 16 + t;
        bytes[t] = (row < rows_total && k < K) ? src[row * K + k] : (uint8_t)0;
      }
      uint4 w;
      memcpy(&w, bytes, 16);
      *reinterpret_cast<uint4 *>((isa ? sa : sb) + (size_t)c16 * rows * 16 + (size_t)r * 16) = w;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy stores seen by the MMA
    __syncthreads();
    if (threadIdx.x == 0) {
      tc5::fence_after_sync();
#pragma unroll
      for (int kk = 0; kk < kKS / 32; ++kk) {
        const uint64_t da = tc5::smem_desc(sa + kk * 2 * (kM * 16), kM * 16, 128);
        const uint64_t db = tc5::smem_desc(sb + kk * 2 * (kN * 16), kN * 16, 128);
        mma_f8(tbase, da, db, idesc, (st > 0 || kk > 0) ? 1u : 0u);
      }
      tc5::mma_commit(&done);
    }
    // Everyone waits for this stage's MMAs before the codes are overwritten (and before the readout).
    ok = mbar_wait_sleep(&done, (uint32_t)(st & 1));
    ok = __syncthreads_and(ok);
    tc5::fence_after_sync();
  }
  if (!ok) {
    // The last commit has not arrived: wait once more (bounded) for those MMAs before TMEM is freed.
    if (threadIdx.x == 0) atomicExch(status, 1);
    mbar_wait_sleep(&done, (uint32_t)((st - 1) & 1));
  } else {
    uint32_t d[32];
    const int64_t m = m0 + warp * 32 + lane;
#pragma unroll
    for (int h = 0; h < kN / 32; ++h) {
      tc5::tmem_ld32(tbase + ((uint32_t)(warp * 32) << 16) + (uint32_t)(h * 32), d);
      if (m < M)
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int64_t n = n0 + h * 32 + j;
          if (n < N) out[m * N + n] = __uint_as_float(d[j]);
        }
    }
  }
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  if (warp == 0) tc5::tmem_dealloc(tbase, kTmemCols);
}

}  // namespace probe
}  // namespace tc

using namespace tc;

extern "C" int tc_probe_mma_fp8(const uint8_t *a, const uint8_t *b, int64_t M, int64_t N, int64_t K, int32_t fmt,
                                float *out, int32_t *status, tc_stream stream) {
  if (M < 0 || N < 0 || K < 0 || (M * N > 0 && (!a || !b || !out)) || !status)
    return set_error("tc_probe_mma_fp8: bad argument"), TC_INVALID_ARGUMENT;
  if (fmt != 0 && fmt != 1) return set_error("tc_probe_mma_fp8: fmt must be 0 (E4M3) or 1 (E5M2)"), TC_INVALID_ARGUMENT;
  if (M == 0 || N == 0) return TC_OK;
  if ((M + probe::kM - 1) / probe::kM > 65535) return set_error("tc_probe_mma_fp8: too many rows"), TC_INVALID_ARGUMENT;
  cudaStream_t s = (cudaStream_t)stream;
  cudaMemsetAsync(status, 0, sizeof(int32_t), s);
  if (K == 0) {
    cudaMemsetAsync(out, 0, (size_t)M * N * sizeof(float), s);
  } else {
    dim3 grid((unsigned)((N + probe::kN - 1) / probe::kN), (unsigned)((M + probe::kM - 1) / probe::kM));
    probe::mma_fp8_kernel<<<grid, 128, 0, s>>>(a, b, M, N, K, fmt, out, status);
    count_launch();
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_probe_mma_fp8: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}
