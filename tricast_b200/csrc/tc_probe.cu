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
// Unused dynamic shared memory that caps the CTAs resident on one SM (228 KB of shared memory) so that
// their TMEM allocations never exceed the SM's 512 columns: at most 6 CTAs x 64 columns here.
constexpr int kPadSmem8 = 12 * 1024;

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

// ---------------------------------------------------------------------------------------------------
// Block-scaled FP4: tcgen05.mma kind::mxf4nvf4 on packed E2M1 codes (two a byte, element 2i in the low
// nibble) with one scale byte per 16 elements (UE4M3, scale_vec::4X: NVFP4) or per 32 (E8M0,
// scale_vec::2X: MXFP4), K = 64 per instruction. The scale factors live in TMEM: for an M- or N-extent
// of 32 c + t, 32-bit column c of lane 32 r + t (every sub-partition r holds a copy) carries that row's
// scale bytes for the instruction's 64 elements, byte j for the j-th scale block. Each warp writes its
// own lane quarter with tcgen05.st before the MMAs of the stage are issued.
constexpr int kKS4 = 256;               // E2M1 elements of K per stage (128 bytes a row)
constexpr uint32_t kTmemCols4 = 128;    // D in columns 0..63, SFA at 64 + 4 kk, SFB at 80 + 2 kk
constexpr uint32_t kSfaCol = 64, kSfbCol = 80;
constexpr int kPadSmem4 = 22 * 1024;    // 24.6 + 22 KB a CTA: at most 4 CTAs x 128 TMEM columns an SM

__host__ __device__ constexpr uint32_t idesc_fp4(bool e8m0, int M, int N) {
  // A and B E2M1 (MXF4 format 1, bits 7-9 and 10-12), K-major, N >> 3 in bits 17-22, scale type in bit
  // 23 (0 UE4M3, 1 E8M0), M >> 4 in bits 24-28; D is always fp32 for block-scaled kinds.
  return (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((e8m0 ? 1u : 0u) << 23) | ((uint32_t)(M >> 4) << 24);
}

template <bool E8M0>
__device__ __forceinline__ void mma_fp4(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate,
                                        uint32_t tsfa, uint32_t tsfb) {
  if constexpr (E8M0)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
            tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
            tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
}

__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v) : "memory");
}

// The scale bytes of one row for one K = 64 instruction, packed little-endian (0 beyond the rows).
template <bool E8M0>
__device__ __forceinline__ uint32_t sf_word(const uint8_t *sf, int64_t row, int64_t rows, int64_t K, int64_t k0) {
  constexpr int kVS = E8M0 ? 32 : 16, kNSF = 64 / kVS;
  if (row >= rows) return 0u;
  const uint8_t *p = sf + row * (K / kVS) + k0 / kVS;
  uint32_t w = 0;
#pragma unroll
  for (int j = 0; j < kNSF; ++j) w |= (uint32_t)p[j] << (8 * j);
  return w;
}

template <bool E8M0>
__global__ void __launch_bounds__(128, 1) mma_fp4_kernel(const uint8_t *__restrict__ a, const uint8_t *__restrict__ b,
                                                         const uint8_t *__restrict__ sfa,
                                                         const uint8_t *__restrict__ sfb, int64_t M, int64_t N,
                                                         int64_t K, float *__restrict__ out, int32_t *status) {
  constexpr int kRowBytes = kKS4 / 2;
  __shared__ __align__(1024) uint8_t sa[kM * kRowBytes];
  __shared__ __align__(1024) uint8_t sb[kN * kRowBytes];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = (int64_t)blockIdx.y * kM, n0 = (int64_t)blockIdx.x * kN;
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    fence_barrier_init();
  }
  if (warp == 0) tc5::tmem_alloc(&tmem_base, kTmemCols4);
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tbase = tmem_base, lane_base = tbase + ((uint32_t)(warp * 32) << 16);
  const uint32_t idesc = idesc_fp4(E8M0, kM, kN);
  const int64_t row_bytes = K / 2;  // K is a multiple of 64: whole 16-byte chunks
  bool ok = true;
  const int64_t nstages = (K + kKS4 - 1) / kKS4;
  int64_t st = 0;
  for (; st < nstages && ok; ++st) {
    for (int i = threadIdx.x; i < (kM + kN) * (kRowBytes / 16); i += blockDim.x) {
      const bool isa = i < kM * (kRowBytes / 16);
      const int j = isa ? i : i - kM * (kRowBytes / 16);
      const int rows = isa ? kM : kN;
      const int r = j % rows, c16 = j / rows;
      const int64_t row = (isa ? m0 : n0) + r, kb = st * kRowBytes + c16 * 16;
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (row < (isa ? M : N) && kb < row_bytes)
        w = *reinterpret_cast<const uint4 *>((isa ? a : b) + row * row_bytes + kb);
      *reinterpret_cast<uint4 *>((isa ? sa : sb) + (size_t)c16 * rows * 16 + (size_t)r * 16) = w;
    }
    const int nmma = (int)((K - st * kKS4) / 64 < kKS4 / 64 ? (K - st * kKS4) / 64 : kKS4 / 64);
    for (int kk = 0; kk < nmma; ++kk) {
      const int64_t k0 = st * kKS4 + kk * 64;
#pragma unroll
      for (int c = 0; c < kM / 32; ++c)
        tmem_st1(lane_base + kSfaCol + 4 * kk + c, sf_word<E8M0>(sfa, m0 + 32 * c + lane, M, K, k0));
#pragma unroll
      for (int c = 0; c < kN / 32; ++c)
        tmem_st1(lane_base + kSfbCol + 2 * kk + c, sf_word<E8M0>(sfb, n0 + 32 * c + lane, N, K, k0));
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc5::fence_before_sync();
    __syncthreads();
    if (threadIdx.x == 0) {
      tc5::fence_after_sync();
      for (int kk = 0; kk < nmma; ++kk) {
        const uint64_t da = tc5::smem_desc(sa + kk * 2 * (kM * 16), kM * 16, 128);
        const uint64_t db = tc5::smem_desc(sb + kk * 2 * (kN * 16), kN * 16, 128);
        mma_fp4<E8M0>(tbase, da, db, idesc, (st > 0 || kk > 0) ? 1u : 0u, tbase + kSfaCol + 4 * kk,
                      tbase + kSfbCol + 2 * kk);
      }
      tc5::mma_commit(&done);
    }
    ok = mbar_wait_sleep(&done, (uint32_t)(st & 1));
    ok = __syncthreads_and(ok);
    tc5::fence_after_sync();
  }
  if (!ok) {
    if (threadIdx.x == 0) atomicExch(status, 1);
    mbar_wait_sleep(&done, (uint32_t)((st - 1) & 1));
  } else {
    uint32_t d[32];
    const int64_t m = m0 + warp * 32 + lane;
#pragma unroll
    for (int h = 0; h < kN / 32; ++h) {
      tc5::tmem_ld32(lane_base + (uint32_t)(h * 32), d);
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
  if (warp == 0) tc5::tmem_dealloc(tbase, kTmemCols4);
}

}  // namespace probe
}  // namespace tc

using namespace tc;

extern "C" int tc_probe_mma_fp8(const uint8_t *a, const uint8_t *b, int64_t M, int64_t N, int64_t K, int32_t fmt,
                                float *out, int32_t *status, tc_stream stream) {
  if (M < 0 || N < 0 || K < 0 || (M * N > 0 && (!out || (K > 0 && (!a || !b)))) || !status)
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
    probe::mma_fp8_kernel<<<grid, 128, probe::kPadSmem8, s>>>(a, b, M, N, K, fmt, out, status);
    count_launch();
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_probe_mma_fp8: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

extern "C" int tc_probe_mma_fp4(const uint8_t *a, const uint8_t *b, const uint8_t *sfa, const uint8_t *sfb, int64_t M,
                                int64_t N, int64_t K, int32_t scale_fmt, float *out, int32_t *status,
                                tc_stream stream) {
  if (M < 0 || N < 0 || K < 0 || K % 64 || !status || (M * N > 0 && (!out || (K > 0 && (!a || !b || !sfa || !sfb)))))
    return set_error("tc_probe_mma_fp4: bad argument (K must be a multiple of 64)"), TC_INVALID_ARGUMENT;
  if (scale_fmt != 0 && scale_fmt != 1)
    return set_error("tc_probe_mma_fp4: scale_fmt must be 0 (UE4M3 per 16) or 1 (E8M0 per 32)"), TC_INVALID_ARGUMENT;
  if (((uintptr_t)a | (uintptr_t)b) & 15) return set_error("tc_probe_mma_fp4: codes must be 16-byte aligned"), TC_INVALID_ARGUMENT;
  if (M == 0 || N == 0) return TC_OK;
  if ((M + probe::kM - 1) / probe::kM > 65535) return set_error("tc_probe_mma_fp4: too many rows"), TC_INVALID_ARGUMENT;
  cudaStream_t s = (cudaStream_t)stream;
  cudaMemsetAsync(status, 0, sizeof(int32_t), s);
  if (K == 0) {
    cudaMemsetAsync(out, 0, (size_t)M * N * sizeof(float), s);
  } else {
    dim3 grid((unsigned)((N + probe::kN - 1) / probe::kN), (unsigned)((M + probe::kM - 1) / probe::kM));
    if (scale_fmt == 1)
      probe::mma_fp4_kernel<true><<<grid, 128, probe::kPadSmem4, s>>>(a, b, sfa, sfb, M, N, K, out, status);
    else
      probe::mma_fp4_kernel<false><<<grid, 128, probe::kPadSmem4, s>>>(a, b, sfa, sfb, M, N, K, out, status);
    count_launch();
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_probe_mma_fp4: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}
