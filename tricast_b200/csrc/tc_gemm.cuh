// Descriptors shared by the GEMM kernels.
#pragma once

#include "tc_mma_exact.cuh"

namespace tc {

enum { ALG_COFDA = 0, ALG_GDFS = 1, ALG_FP32_FMA = 2, ALG_FP64 = 3, ALG_INT_EXACT = 4 };
enum { AP_EPILOGUE = 0, AP_PRODUCT = 1, AP_GROUP = 2, AP_PROMOTE = 3, AP_OPERAND = 4 };
enum { SK_NONE = 0, SK_TENSOR = 1, SK_ROW = 2, SK_K = 3 };

struct OpDesc {
  const void *v;
  int dt;
  int64_t rows, K;
  Fmt f;
  int radix;
  const float *scale;
  int skind;
  Fmt sf;
  int srad;
  int kd;
  int64_t nkd;
  int field0;  // standard E8M0 K scale: 2**-127 counts as zero
  const float *alpha;
};

struct GemmDesc {
  OpDesc a, b;
  int64_t M, N, K;
  int alg, F, CS, decoupled, F2, G, GS, KT, rne, apply, PI;
  Fmt of;
  int out_dt;
  int out_is_plain;  // out_format is fp32 itself: no output cast
  const float *bias;
  void *out;
};

// Epilogue (src/tricast/reference/mma.py:372-384): tensor/row scales of b then a, alpha_a*alpha_b,
// bias, each one fp32 RN step, then the out_format rounding into the container.
__device__ __forceinline__ float epilogue(const GemmDesc &g, int64_t m, int64_t n, float acc) {
  if (g.b.skind == SK_TENSOR) acc = __fmul_rn(g.b.scale[0], acc);
  else if (g.b.skind == SK_ROW) acc = __fmul_rn(g.b.scale[n], acc);
  if (g.a.skind == SK_TENSOR) acc = __fmul_rn(g.a.scale[0], acc);
  else if (g.a.skind == SK_ROW) acc = __fmul_rn(g.a.scale[m], acc);
  if (g.a.alpha || g.b.alpha) {
    float al = g.a.alpha ? *g.a.alpha : 1.0f;
    if (g.b.alpha) al = g.a.alpha ? __fmul_rn(al, *g.b.alpha) : *g.b.alpha;
    acc = __fmul_rn(al, acc);
  }
  if (g.bias) acc = __fadd_rn(acc, g.bias[n]);
  return acc;
}

__device__ __forceinline__ void store_out(const GemmDesc &g, int64_t m, int64_t n, float acc) {
  float v = g.out_is_plain ? acc : cast_to(acc, g.of, TC_RNE, false, 0u, 32);
  store_container(g.out, g.out_dt, m * g.N + n, v);
}

int build_desc(const tc_operand *a, const tc_operand *b, const tc_mma_spec *spec, const float *bias, void *out,
               GemmDesc &g);

// Fast kernels (tc_gemm_fast.cu): return TC_UNSUPPORTED when the case is not theirs.
size_t fast_workspace(const GemmDesc &g);
int launch_fast(const GemmDesc &g, void *workspace, size_t workspace_bytes, cudaStream_t s,
                const void *benc = nullptr);

// Pre-encoded B operands (tc_encode_b): bytes of B's encoding for this operand pair and spec (0: the
// pair's fast path takes none), the encoder, and the GEMM on an encoded B. The tiled GDFS-FP4 path
// (A of more than 16 rows) and the small-M CoFDA path (at most 16) take one.
size_t encoded_b_bytes(const GemmDesc &g);
int encode_b(const GemmDesc &g, void *enc, size_t enc_bytes, cudaStream_t s);
int launch_fast_encoded(const GemmDesc &g, const void *benc, size_t enc_bytes, void *workspace,
                        size_t workspace_bytes, cudaStream_t s);

// The exact generic kernel; with only_if_flag it runs only when *only_if_flag != 0.
void launch_generic(const GemmDesc &g, const int32_t *only_if_flag, cudaStream_t s);

}  // namespace tc
