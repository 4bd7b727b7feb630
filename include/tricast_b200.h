/*
 * tricast_b200.h — C ABI of the B200 (sm_100a) backend for TriCast's emulation hot path.
 *
 * The library replaces TriCast's Triton backend module by module. Every entry point takes plain
 * device pointers, sizes and small POD descriptors; the caller (PyTorch in the Python shim, or any
 * C/ctypes caller) owns every buffer. Entry points are asynchronous on the given stream, never
 * allocate device memory except where a comment says so, and return a tc_status; the message of
 * the last failure on the calling host thread is available from tc_last_error().
 *
 * Reference interfaces each entry point replaces (paths inside the TriCast checkout):
 *   tc_cast              <- round_to_format_triton   src/tricast/kernels/quantize.py:161-178
 *                           (semantics: src/tricast/reference/cast.py:18-83)
 *   tc_quantize          <- quantize_triton          src/tricast/kernels/quantize.py:192-275
 *                           (semantics: src/tricast/reference/quantize.py:244-350)
 *   tc_gemm              <- gemm_triton              src/tricast/kernels/mma.py:821-886
 *                           (semantics: src/tricast/reference/mma.py:339-384)
 *   tc_error_stats       <- analysis._ErrorStats.update  src/tricast/analysis.py:37-50
 */
#ifndef TRICAST_B200_H
#define TRICAST_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; 0 is the legacy default stream. */
typedef struct CUstream_st *tc_stream;

typedef enum tc_status {
  TC_OK = 0,
  TC_INVALID_ARGUMENT = 1,  /* bad shape, pointer, descriptor or size limit */
  TC_UNSUPPORTED = 2,       /* a valid TriCast spec this build does not implement */
  TC_CUDA_ERROR = 3,        /* a CUDA launch or runtime call failed */
  TC_WORKSPACE_TOO_SMALL = 4,
  TC_NONFINITE = 5          /* int_exact saw a NaN/Inf operand (reported by tc_gemm_check) */
} tc_status;

/* Container dtypes of values, inputs and outputs. */
typedef enum tc_dtype { TC_F32 = 0, TC_BF16 = 1, TC_F16 = 2 } tc_dtype;

/* Rounding codes (src/tricast/rounding.py:39). */
typedef enum tc_rounding { TC_RNE = 0, TC_RNA = 1, TC_RTZ = 2, TC_RUP = 3, TC_RDN = 4, TC_SR = 5 } tc_rounding;

/* A TriCast number format (src/tricast/formats.py:29-201): primary fields only; the library
 * derives emin/emax/max_normal itself. kind: 0 float (ExMy), 1 int (fixed point), 2 pow2 (E8M0).
 * special (floats): 0 ieee, 1 fn, 2 fnuz, 3 none. */
typedef struct tc_format {
  int32_t kind;
  int32_t ebits;       /* float, pow2 */
  int32_t mbits;       /* float */
  int32_t bias;        /* float, pow2 */
  int32_t special;     /* float */
  int32_t is_signed;   /* float, int */
  int32_t subnormals;  /* float */
  int32_t bits;        /* int */
  int32_t symmetric;   /* int */
  int32_t frac_bits;   /* int */
} tc_format;

/* QuantSpec (src/tricast/quant/spec.py:167-234). granularity: 0 tensor, 1 row, 2 group, 3 block.
 * scale_method: 0 absmax, 1 pow2_floor, 2 pow2_ceil, 3 mse, 4 percentile. zero_point: 0 none,
 * 1 int, 2 float. mse_search holds the MSE candidate ratios (already rounded to fp32) on the host. */
typedef struct tc_quant_spec {
  tc_format format;
  int32_t granularity;
  int32_t group_size;
  int32_t block_rows;
  int32_t block_cols;
  int32_t has_scale;
  tc_format scale_format;
  int32_t scale_method;
  int32_t scale_rounding;
  int32_t two_level;
  int32_t zero_point;
  int32_t rounding;
  int32_t sr_bits;
  int32_t saturate;
  float percentile;
  int32_t n_search;
  const float *mse_search;
} tc_quant_spec;

/* Outputs of tc_quantize. values (container dtype) and, when the spec has them, scale /
 * zero_point (scale layout, fp32) and global_scale (one fp32) are required; the rest are optional
 * extras written in the same pass (NULL to skip):
 *   codes       element codes: 4-bit formats two per byte (low nibble = even element), else one byte
 *   scale_codes scale-format codes, one byte per scale (E8M0: exponent + 127)
 *   dequant     fp32 dequantized values ((v - z) * s [+ z]) * d2, TriCast's QTensor.dequantize order */
typedef struct tc_quant_out {
  void *values;
  int32_t values_dtype;
  float *scale;
  float *zero_point;
  float *global_scale;
  uint8_t *codes;
  uint8_t *scale_codes;
  float *dequant;
} tc_quant_out;

/* One MMA operand (src/tricast/mma/operand.py:28-57): values [rows, K] row-major and contiguous.
 * scale_kind: 0 none, 1 tensor (scalar), 2 row ([rows]), 3 k ([rows, ceil(K / k_domain)]).
 * scale_fmt is used for scale_kind 3 only (has_scale_fmt 0 means fp32). alpha: device scalar or NULL. */
typedef struct tc_operand {
  const void *values;
  int32_t values_dtype;
  int64_t rows;
  int64_t K;
  tc_format fmt;
  const float *scale;
  int32_t scale_kind;
  int32_t has_scale_fmt;
  tc_format scale_fmt;
  int32_t k_domain;
  const float *alpha;
} tc_operand;

/* MMASpec (src/tricast/mma/spec.py:223-270) with scale_apply already resolved (TriCast's
 * resolve_scale_apply, src/tricast/reference/mma.py:184-202): 0 epilogue, 1 product, 2 group,
 * 3 promote, 4 operand. algorithm: 0 cofda, 1 gdfs, 2 fp32_fma, 3 fp64, 4 int_exact.
 * c_mode: 0 fused, 1 decoupled. norm_rounding: 0 rtz, 1 rne. out_dtype: container of out_format. */
typedef struct tc_mma_spec {
  int32_t algorithm;
  int32_t f_bits;
  int32_t chunk_size;
  int32_t c_mode;
  int32_t f2_bits;
  int32_t g_bits;
  int32_t group_size;
  int32_t k_tile;
  int32_t norm_rounding;
  int32_t scale_apply;
  int32_t promote_interval;
  tc_format out_format;
  int32_t out_dtype;
} tc_mma_spec;

/* Cast n fp32 values onto fmt's grid (TriCast round_to_format). noise: NULL or n uint32 values
 * (stochastic rounding). y may alias x. */
int tc_cast(const float *x, float *y, const uint32_t *noise, int64_t n, const tc_format *fmt,
            int32_t rounding, int32_t saturate, int32_t sr_bits, tc_stream stream);

/* Bytes of scratch tc_quantize needs for this shape and spec (0 when none). */
size_t tc_quantize_workspace(int64_t rows, int64_t K, const tc_quant_spec *spec);

/* Quantize x [rows, K] (x_dtype: TC_F32 / TC_BF16 / TC_F16) under spec, writing out. amax: NULL,
 * or a device fp32 scalar: for tensor granularity it overrides the tensor amax (TriCast's
 * quantize(amax=...)); for a two-level spec of finer granularity (NVFP4) it is the tensor amax the
 * global scale d2 is derived from, so that a shard of a larger tensor quantizes exactly as the same
 * rows of the whole tensor would (an extension: TriCast accepts amax for tensor granularity only);
 * other specs reject it. noise: NULL or rows*K uint32; scale_noise: NULL or one uint32 per scale. */
int tc_quantize(const void *x, int32_t x_dtype, int64_t rows, int64_t K, const tc_quant_spec *spec,
                const float *amax, const uint32_t *noise, const uint32_t *scale_noise,
                const tc_quant_out *out, void *workspace, size_t workspace_bytes, tc_stream stream);

/* The amax of x (n elements of x_dtype) as the bits of the fp32 |x| maximum, NaN-propagating (NaN
 * bits sort above Inf's), max-reduced into *bits (device uint32, cleared by the caller). A rank
 * holding a row shard of a tensor reduces its shard's bits with the other ranks' (integer max) and
 * passes the result, viewed as fp32, as tc_quantize's amax of a two-level spec. No counterpart in
 * TriCast, whose tensors are never sharded. */
int tc_tensor_amax_bits(const void *x, int32_t x_dtype, int64_t n, uint32_t *bits, tc_stream stream);

/* Bytes of scratch tc_gemm needs for these operands and spec. */
size_t tc_gemm_workspace(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec);

/* out [a.rows, b.rows] (spec.out_dtype) = a @ b^T under spec's accumulation rule, bias ([b.rows]
 * fp32) optional. Validation of TriCast's int64 headroom rules is the caller's (the Python shim
 * does it with TriCast's messages); this call checks pointers, shapes and size limits. */
int tc_gemm(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec, const float *bias, void *out,
            void *workspace, size_t workspace_bytes, tc_stream stream);

/* Pre-encoded B operands (weights). TriCast keeps a weight operand's packed K-major copy between
 * calls (src/tricast/mma/operand.py:66-75, nn/linear.py:216-224); these keep the fast path's own
 * encoding of B instead, so repeated GEMMs against one weight skip re-encoding it.
 * tc_encode_b_bytes: bytes of B's encoding for GEMMs of A operands like a (same format and scale
 * layout, and a row count on the same side of 16: more than 16 rows take the tiled kernels, at most
 * 16 the small-M ones) under spec; 0 when that path takes no pre-encoded B (the tiled GDFS-FP4 path
 * and the small-M CoFDA path take one). a's values are not read.
 * tc_encode_b: writes it into enc (device memory the caller owns, at least that many bytes); B's
 * values and scales are read, asynchronously on stream. A B the fast path cannot take is recorded in
 * the encoding and sends every GEMM on it to the exact kernel, as tc_gemm does.
 * tc_gemm_encoded: tc_gemm with B given by its encoding (b still describes B: shape, format, scales
 * for the exact kernel); workspace as tc_gemm_workspace(a, b, spec). The encoding must come from
 * tc_encode_b for this b, spec and an A like a; an encoding of another size is rejected with
 * TC_INVALID_ARGUMENT. */
size_t tc_encode_b_bytes(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec);
int tc_encode_b(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec, void *enc, size_t enc_bytes,
                tc_stream stream);
int tc_gemm_encoded(const tc_operand *a, const tc_operand *b, const void *b_enc, size_t b_enc_bytes,
                    const tc_mma_spec *spec, const float *bias, void *out, void *workspace, size_t workspace_bytes,
                    tc_stream stream);

/* tc_gemm for callers that cannot allocate device memory. No counterpart in TriCast: this entry point
 * exists for hosts that reach the library through a bare C FFI without a CUDA allocator of their own,
 * or that reserve all device memory up front, and so cannot hand tc_gemm a workspace. Same
 * arguments and result as tc_gemm minus the workspace; the scratch comes from a fixed 32 MiB array
 * inside the library (held on every GPU that loads the library, until exit). Operands whose
 * tc_gemm_workspace() exceeds 32 MiB are rejected with TC_INVALID_ARGUMENT. The first call on a
 * device looks up that array's device address, so make it before any stream capture. The array used is
 * the current device's: call with the device of out (and of stream) current; an out on another
 * device is rejected with TC_INVALID_ARGUMENT. All calls share the array: calls whose GPU work can
 * overlap race and must not be issued. Allocates nothing. */
int tc_gemm_noalloc(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec, const float *bias,
                    void *out, tc_stream stream);

/* Device-side check used before int_exact: writes 1 to *flag (device int32) when any value of the
 * operand is NaN/Inf, else leaves it unchanged. */
int tc_any_nonfinite(const void *values, int32_t dtype, int64_t n, int32_t *flag, tc_stream stream);

/* fp64 error sums of ref vs emu (n elements each, dtypes as tc_dtype) added into sums[6] on the
 * device: {sum x^2, sum y^2, sum (x-y)^2, sum x*y, max |x-y|, count of non-finite elements}. */
int tc_error_stats(const void *ref, int32_t ref_dtype, const void *emu, int32_t emu_dtype, int64_t n,
                   double *sums, tc_stream stream);

/* Message of the last failed call on this host thread ("" if none). */
const char *tc_last_error(void);

/* Number of kernels this library has launched in the process (all threads, all devices). */
uint64_t tc_launch_count(void);

/* How many times, on the current device, the exact generic GEMM kernel queued behind a fast kernel
 * has actually run (the fast kernel declined the operands or one of its waits ran out). Waits for the
 * device. */
int tc_exact_fallbacks(uint64_t *count);

/* Of those runs, how many followed a fast kernel whose bounded wait ran out (it set its status word,
 * drained its own copies and MMAs, freed its TMEM and returned). Waits for the device. No counterpart
 * in TriCast, whose Triton kernels have no bounded waits. */
int tc_wait_timeouts(uint64_t *count);

/* How many (output, K tile) steps of the tensor-core GDFS-FP4 kernel, on the current device, failed
 * the single-pass bounds and ran the exact two-pass step instead (exact either way; this counts how
 * often the slow step runs). Waits for the device. No counterpart in TriCast. */
int tc_exact_tile_steps(uint64_t *count);

/* Poll limit of the pipeline waits (on shared-memory barriers) of the staged GEMM kernels launched
 * from now on, process-wide; polls < 0 restores the defaults (about 2**16 suspended or 2**22 plain
 * polls, seconds). With polls = 0 every such wait gives up at once: the kernel takes its timeout path
 * and the exact kernel queued behind it recomputes the product, so results stay exact. The waits that
 * drain a kernel's own copies and MMAs before it exits keep the default limit. No counterpart in
 * TriCast: it exists to test the timeout path without hanging or faulting a GPU. */
int tc_set_wait_limit(int32_t polls);

/* Silicon probe, not part of the emulation API: out[M][N] = sum_k A[m][k] * B[n][k] computed by the
 * B200's own FP8 tensor-core MMA (tcgen05.mma kind::f8f6f4, fp32 accumulator, K issued 32 at a time
 * in order, no scales). a [M][K] and b [N][K] are row-major 8-bit codes, fmt 0 = E4M3, 1 = E5M2;
 * out is fp32 [M][N]. *status (device) is set non-zero if a wait inside the kernel ran out. Used to
 * test whether an emulated accumulation model reproduces the hardware; no reference interface. */
int tc_probe_mma_fp8(const uint8_t *a, const uint8_t *b, int64_t M, int64_t N, int64_t K, int32_t fmt, float *out,
                     int32_t *status, tc_stream stream);

/* Silicon probe, block-scaled FP4: out[M][N] = sum_k A[m][k] sA[m][k / V] * B[n][k] sB[n][k / V] by the
 * tensor core's tcgen05.mma kind::mxf4nvf4 (fp32 accumulator, K issued 64 at a time in order).
 * a [M][K/2] and b [N][K/2] are packed E2M1 codes (element 2i in the low nibble, 16-byte aligned);
 * sfa [M][K/V] and sfb [N][K/V] are scale bytes: scale_fmt 0 = UE4M3 with V = 16 (NVFP4),
 * 1 = E8M0 with V = 32 (MXFP4). K must be a multiple of 64. *status as for tc_probe_mma_fp8. */
int tc_probe_mma_fp4(const uint8_t *a, const uint8_t *b, const uint8_t *sfa, const uint8_t *sfb, int64_t M, int64_t N,
                     int64_t K, int32_t scale_fmt, float *out, int32_t *status, tc_stream stream);

/* Library version string. */
const char *tc_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TRICAST_B200_H */
