// tc_gemm_noalloc: the emulated GEMM for callers that cannot allocate device memory.
//
// tc_gemm asks its caller for a workspace (the fast kernels encode both operands into it). Some
// callers have no way to provide one: a host that reaches this library only through a plain C
// FFI and owns no CUDA allocator, a serving process whose device memory is fully reserved up front
// by its own pool, or code that must not allocate at all between set-up and teardown. For them this
// entry point takes its scratch from a fixed array that lives inside the library itself.
//
// The array is a file-scope __device__ object of kScratchBytes (32 MiB). Every GPU on which the
// library's device code is loaded holds it until the process exits. In host code its name is only a
// host-side stand-in, so the first call on each device resolves its real device address with
// cudaGetSymbolAddress (with that device current) and caches it; that first call should therefore
// come before any stream capture. Nothing here calls cudaMalloc, cudaFree or an allocating library
// routine.
//
// Every call shares the one array and it keeps whatever the previous call left in it: the fast
// path's status words are cleared on the stream at the start of each call, and everything else is
// fully rewritten before it is read. Calls whose GPU work overlaps (different streams, or other host
// threads, without ordering between them) race on the array and must not be issued.
//
// The array used is the current device's, so the output (and the stream) must belong to the device
// that is current on the calling thread; a call whose output lives on another device is rejected
// with TC_INVALID_ARGUMENT before anything is launched.
#include <mutex>
#include <string>

#include "tc_gemm.cuh"

namespace tc {

constexpr size_t kScratchBytes = 32ull << 20;
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

static std::mutex g_scratch_mu;
static void *g_scratch_ptr[128];  // per device ordinal

// Device address of g_scratch on the current device (set up once per device).
static int scratch_on_current_device(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(std::string("tc_gemm_noalloc: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  if (dev < 0 || dev >= 128) return set_error("tc_gemm_noalloc: device ordinal out of range"), TC_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || !p)
      return set_error(std::string("tc_gemm_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e)),
             TC_CUDA_ERROR;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TC_OK;
}

// The output must be memory of the current device (the scratch array resolved above is that
// device's): a device pointer of another device is refused.
static int out_on_current_device(const void *out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(std::string("tc_gemm_noalloc: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  cudaPointerAttributes attr;
  e = cudaPointerGetAttributes(&attr, out);
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error of a pointer CUDA does not know
    return set_error("tc_gemm_noalloc: the output is not CUDA memory"), TC_INVALID_ARGUMENT;
  }
  if (attr.type == cudaMemoryTypeDevice && attr.device != dev)
    return set_error("tc_gemm_noalloc: the output lives on device " + std::to_string(attr.device) +
                     " but device " + std::to_string(dev) + " is current; make the output's device current"),
           TC_INVALID_ARGUMENT;
  return TC_OK;
}

}  // namespace tc

using namespace tc;

extern "C" int tc_gemm_noalloc(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec, const float *bias,
                               void *out, tc_stream stream) {
  GemmDesc g;
  int st = build_desc(a, b, spec, bias, out, g);
  if (st) return st;
  if (g.M == 0 || g.N == 0) return TC_OK;
  size_t need = fast_workspace(g);
  if (need > kScratchBytes)
    return set_error("tc_gemm_noalloc: these operands need " + std::to_string(need) +
                     " bytes of scratch, more than the fixed " + std::to_string(kScratchBytes) +
                     "-byte array; call tc_gemm with a workspace instead"),
           TC_INVALID_ARGUMENT;
  cudaStream_t s = (cudaStream_t)stream;
  if ((st = out_on_current_device(out))) return st;
  // Kernels that need no scratch (fp64 / fp32_fma chains) take the fast path with no workspace, as
  // tc_gemm does; the others get the fixed array.
  void *scratch = nullptr;
  if (need > 0 && (st = scratch_on_current_device(&scratch))) return st;
  st = launch_fast(g, scratch, need > 0 ? kScratchBytes : 0, s);
  if (st != TC_UNSUPPORTED) return st;
  if ((g.M + 15) / 16 > 65535) return set_error("tc_gemm_noalloc: too many rows for the generic kernel"), TC_INVALID_ARGUMENT;
  launch_generic(g, nullptr, s);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm_noalloc: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}
