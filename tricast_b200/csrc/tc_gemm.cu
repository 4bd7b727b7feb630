// Emulated GEMM entry point and the exact generic kernel.
//
// The generic kernel computes one output per thread in TriCast's order (src/tricast/reference/
// mma.py:286-384): CoFDA chunks from k = 0 (fused, decoupled or promoted), GDFS tiles of groups,
// exact integer sums, or IEEE fp32 / fp64 FMA chains, then the epilogue. It handles every
// operand format, scale layout and Inf/NaN rule, and is the path for anything the fast kernels
// (tc_gemm_fast.cu) do not claim.
#include <cstring>
#include <string>

#include "tc_generic.cuh"

namespace tc {

// 16 x 16 output tiles, grid-stride, one output per thread. Behind a fast kernel the grid is small, so
// the common case (flag clear) costs a few hundred blocks that read two words and exit.
// Runs of the exact kernel behind a fast kernel that declined its operands (or timed out), per device.
__device__ unsigned long long g_exact_fallbacks;
// Of those, the runs whose fast kernel reported a bounded wait that ran out (its status word).
__device__ unsigned long long g_wait_timeouts;

__global__ void __launch_bounds__(256) gemm_generic_kernel(GemmDesc g, const int32_t *only_if_flag) {
  if (only_if_flag && only_if_flag[0] == 0 && only_if_flag[1] == 0) return;  // the fast kernel took it
  if (only_if_flag && blockIdx.x == 0 && threadIdx.x == 0) {
    atomicAdd(&g_exact_fallbacks, 1ull);
    if (only_if_flag[1]) atomicAdd(&g_wait_timeouts, 1ull);
  }
  const int64_t tiles_n = (g.N + 15) / 16, tiles = tiles_n * ((g.M + 15) / 16);
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t n = (tile % tiles_n) * 16 + (threadIdx.x & 15);
    const int64_t m = (tile / tiles_n) * 16 + (threadIdx.x >> 4);
    if (m < g.M && n < g.N) generic_output(g, m, n);
  }
}

// Device-side finiteness check (int_exact operands).
__global__ void any_nonfinite_kernel(const void *v, int dt, int64_t n, int32_t *flag) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  bool bad = false;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float x = load_as_float(v, dt, i);
    bad |= (f2u(x) & 0x7F800000u) == 0x7F800000u;
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicExch(flag, 1);
}

static std::string check_operand(const tc_operand &o, const char *side) {
  std::string s(side);
  if (o.rows < 0 || o.K < 0) return s + ": negative shape";
  if (o.rows * o.K > 0 && !o.values) return s + ": null values";
  if (o.values_dtype < 0 || o.values_dtype > 2) return s + ": unsupported values dtype";
  std::string e = fmt_error(o.fmt);
  if (!e.empty()) return s + " format: " + e;
  if (o.scale_kind < 0 || o.scale_kind > 3) return s + ": unknown scale_kind";
  if (o.scale_kind != SK_NONE && !o.scale) return s + ": scale_kind set without a scale";
  if (o.scale_kind == SK_K) {
    if (o.k_domain <= 0) return s + ": K-varying scales need k_domain > 0";
    if (o.has_scale_fmt) {
      e = fmt_error(o.scale_fmt);
      if (!e.empty()) return s + " scale format: " + e;
    }
  }
  return "";
}

static OpDesc make_op(const tc_operand &o) {
  OpDesc d;
  std::memset(&d, 0, sizeof(d));
  d.v = o.values;
  d.dt = o.values_dtype;
  d.rows = o.rows;
  d.K = o.K;
  d.f = derive(o.fmt);
  d.radix = o.fmt.kind == 0 ? o.fmt.mbits : (o.fmt.kind == 1 ? o.fmt.frac_bits : 0);
  d.scale = o.scale;
  d.skind = o.scale_kind;
  d.kd = o.k_domain > 0 ? o.k_domain : 1;
  d.nkd = o.scale_kind == SK_K ? (o.K + d.kd - 1) / d.kd : 1;
  tc_format sf = o.fmt;
  if (o.scale_kind == SK_K && o.has_scale_fmt) {
    sf = o.scale_fmt;
  } else {
    std::memset(&sf, 0, sizeof(sf));
    sf.kind = 0; sf.ebits = 8; sf.mbits = 23; sf.bias = 127; sf.special = 0; sf.is_signed = 1; sf.subnormals = 1;
  }
  d.sf = derive(sf);
  d.srad = sf.kind == 0 ? sf.mbits : (sf.kind == 1 ? sf.frac_bits : 0);
  d.field0 = o.scale_kind == SK_K && sf.kind == 2 && sf.ebits == 8 && sf.bias == 127;
  d.alpha = o.alpha;
  return d;
}

int build_desc(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec, const float *bias, void *out,
               GemmDesc &g) {
  if (!a || !b || !spec) return set_error("tc_gemm: null argument"), TC_INVALID_ARGUMENT;
  std::string e = check_operand(*a, "a");
  if (e.empty()) e = check_operand(*b, "b");
  if (!e.empty()) return set_error("tc_gemm: " + e), TC_INVALID_ARGUMENT;
  if (a->K != b->K) return set_error("operands must have the same K"), TC_INVALID_ARGUMENT;
  if (spec->algorithm < 0 || spec->algorithm > 4) return set_error("unknown algorithm"), TC_INVALID_ARGUMENT;
  if (spec->out_format.kind != 0) return set_error("out_format must be a float format"), TC_INVALID_ARGUMENT;
  if (a->rows * b->rows > 0 && !out) return set_error("tc_gemm: null output"), TC_INVALID_ARGUMENT;
  if (spec->algorithm == ALG_COFDA && spec->chunk_size < 1) return set_error("chunk_size must be >= 1"), TC_INVALID_ARGUMENT;
  if (spec->algorithm == ALG_GDFS && (spec->group_size < 1 || spec->k_tile % spec->group_size ||
                                      spec->k_tile / spec->group_size > 8 || spec->k_tile < 1))
    return set_error("k_tile must be a positive multiple of group_size with at most 8 groups"), TC_INVALID_ARGUMENT;
  std::memset(&g, 0, sizeof(g));
  g.a = make_op(*a);
  g.b = make_op(*b);
  g.M = a->rows;
  g.N = b->rows;
  g.K = a->K;
  g.alg = spec->algorithm;
  g.F = spec->f_bits;
  g.CS = spec->chunk_size;
  g.decoupled = spec->c_mode == 1;
  g.F2 = spec->f2_bits;
  g.G = spec->g_bits;
  g.GS = spec->group_size;
  g.KT = spec->k_tile;
  g.rne = spec->norm_rounding == 1;
  g.apply = spec->scale_apply;
  g.PI = spec->promote_interval;
  g.of = derive(spec->out_format);
  g.out_dt = spec->out_dtype;
  const tc_format &of = spec->out_format;
  g.out_is_plain = of.ebits == 8 && of.mbits == 23 && of.bias == 127 && of.special == 0 && of.is_signed && of.subnormals;
  g.bias = bias;
  g.out = out;
  return TC_OK;
}

void launch_generic(const GemmDesc &g, const int32_t *only_if_flag, cudaStream_t s) {
  const int64_t tiles = ((g.N + 15) / 16) * ((g.M + 15) / 16);
  const int64_t cap = (int64_t)sm_count() * 8;
  gemm_generic_kernel<<<(unsigned)(tiles < cap ? tiles : cap), 256, 0, s>>>(g, only_if_flag);
  count_launch();
}

}  // namespace tc

using namespace tc;

extern "C" size_t tc_gemm_workspace(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec) {
  GemmDesc g;
  if (build_desc(a, b, spec, nullptr, (void *)1, g)) return 0;
  return fast_workspace(g);
}

extern "C" int tc_gemm(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec, const float *bias,
                       void *out, void *workspace, size_t workspace_bytes, tc_stream stream) {
  GemmDesc g;
  int st = build_desc(a, b, spec, bias, out, g);
  if (st) return st;
  if (g.M == 0 || g.N == 0) return TC_OK;
  cudaStream_t s = (cudaStream_t)stream;
  st = launch_fast(g, workspace, workspace_bytes, s);
  if (st != TC_UNSUPPORTED) return st;
  if ((g.M + 15) / 16 > 65535) return set_error("tc_gemm: too many rows for the generic kernel"), TC_INVALID_ARGUMENT;
  launch_generic(g, nullptr, s);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_gemm: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}

extern "C" size_t tc_encode_b_bytes(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec) {
  GemmDesc g;
  if (build_desc(a, b, spec, nullptr, (void *)1, g)) return 0;
  return encoded_b_bytes(g);
}

extern "C" int tc_encode_b(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec, void *enc,
                           size_t enc_bytes, tc_stream stream) {
  GemmDesc g;
  int st = build_desc(a, b, spec, nullptr, (void *)1, g);
  if (st) return st;
  return encode_b(g, enc, enc_bytes, (cudaStream_t)stream);
}

extern "C" int tc_gemm_encoded(const tc_operand *a, const tc_operand *b, const void *b_enc, size_t b_enc_bytes,
                               const tc_mma_spec *spec, const float *bias, void *out, void *workspace,
                               size_t workspace_bytes, tc_stream stream) {
  GemmDesc g;
  int st = build_desc(a, b, spec, bias, out, g);
  if (st) return st;
  if (g.M == 0 || g.N == 0) return TC_OK;
  return launch_fast_encoded(g, b_enc, b_enc_bytes, workspace, workspace_bytes, (cudaStream_t)stream);
}

namespace tc {
uint64_t gemv_exact_fallbacks();
}

extern "C" int tc_exact_fallbacks(uint64_t *count) {
  if (!count) return set_error("tc_exact_fallbacks: null argument"), TC_INVALID_ARGUMENT;
  unsigned long long v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_exact_fallbacks, sizeof(v));
  if (e != cudaSuccess) return set_error(std::string("tc_exact_fallbacks: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  *count = (uint64_t)v + tc::gemv_exact_fallbacks();
  return TC_OK;
}

namespace tc {
int exact_tile_steps(unsigned long long *count);
}

extern "C" int tc_exact_tile_steps(uint64_t *count) {
  if (!count) return set_error("tc_exact_tile_steps: null argument"), TC_INVALID_ARGUMENT;
  unsigned long long v = 0;
  int st = tc::exact_tile_steps(&v);
  *count = (uint64_t)v;
  return st;
}

extern "C" int tc_wait_timeouts(uint64_t *count) {
  if (!count) return set_error("tc_wait_timeouts: null argument"), TC_INVALID_ARGUMENT;
  unsigned long long v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v));
  if (e != cudaSuccess) return set_error(std::string("tc_wait_timeouts: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  *count = (uint64_t)v;
  return TC_OK;
}

extern "C" int tc_any_nonfinite(const void *values, int32_t dtype, int64_t n, int32_t *flag, tc_stream stream) {
  if (n <= 0) return TC_OK;
  if (!values || !flag || dtype < 0 || dtype > 2) return set_error("tc_any_nonfinite: bad argument"), TC_INVALID_ARGUMENT;
  int64_t blocks = (n + 255) / 256;
  if (blocks > (int64_t)sm_count() * 8) blocks = (int64_t)sm_count() * 8;
  any_nonfinite_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(values, dtype, n, flag);
  ::tc::count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(std::string("tc_any_nonfinite: ") + cudaGetErrorString(e)), TC_CUDA_ERROR;
  return TC_OK;
}
