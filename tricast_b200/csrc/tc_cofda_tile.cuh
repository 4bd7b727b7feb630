// The tiled layout shared by the CoFDA kernel (tc_gemm_cofda.cu) and the GDFS kernel for narrow
// float grids (tc_gemm_gdfs.cu): each operand's elements decoded once into per (row tile of 64,
// chunk, k) values (the grid value with any power-of-two K scale folded in, fp32 or fp64) and int16
// exponent labels, so that a CTA's stage for one chunk is four contiguous bulk copies.
#pragma once

#include "tc_bulk.cuh"
#include "tc_cofda.cuh"

namespace tc {
namespace cofda {

constexpr int kTile = 64;     // rows of A and columns of B per CTA

// Float grids whose products are exact fp32 values well inside fp32's normal range (FP8 / FP6 / FP4).
inline bool narrow_float(const Fmt &f) { return f.kind == 0 && f.mbits <= 3 && f.emax <= 15 && f.emin >= -14; }

struct EncodeArgs {
  const void *v;
  int dt;
  int64_t rows, K, rows_pad, nchunks;
  int CS;
  Fmt f;
  const float *scale;  // product-mode pow2 K scales folded into the values, or nullptr
  int64_t nkd;
  int kd;
  Fmt sf;
  int field0;
  void *val;           // [tile][chunk][k][kTile], float or double
  uint32_t *exp;       // A: [tile][chunk][k][kTile/2] (pairs of rows); B: [tile][chunk][k][kTile] (duplicated)
  void *sgn;           // optional, laid out as val: val then holds |value| and sgn its sign as +-1
  int side;
  int32_t *flag;
};

// Position of column c of a 64-wide tile among the staged B values. fp32 keeps the natural order (a
// thread's four columns are one 16-byte load, 16 threads read 256 contiguous bytes); fp64 puts columns
// 4t, 4t + 1 at 2t, 2t + 1 and 4t + 2, 4t + 3 at 32 + 2t, 33 + 2t, so each of a thread's two 16-byte
// loads is again one of 16 contiguous pairs (no shared-memory bank conflicts).
template <class T>
__host__ __device__ __forceinline__ int bcol(int c) {
  return sizeof(T) == 8 ? ((c & 2) << 4) + ((c >> 2) << 1) + (c & 1) : c;
}

// Thread tx's four B values (columns 4 tx .. 4 tx + 3) of one k from the staged row.
template <class T>
__device__ __forceinline__ void load_b4(const T *row, int tx, T (&o)[4]) {
  if constexpr (sizeof(T) == 4) {
    load4<T>(row + tx * 4, o);
  } else {
    const double2 v0 = *reinterpret_cast<const double2 *>(row + tx * 2);
    const double2 v1 = *reinterpret_cast<const double2 *>(row + 32 + tx * 2);
    o[0] = v0.x; o[1] = v0.y; o[2] = v1.x; o[3] = v1.y;
  }
}

template <class T>
__global__ void __launch_bounds__(256) encode_kernel(EncodeArgs e) {
  const int64_t pairs = e.rows_pad / 2;
  const int64_t total = pairs * e.nchunks * e.CS;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  bool bad = false;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int64_t rp = idx % (kTile / 2);            // row pair inside the tile
    int64_t rest = idx / (kTile / 2);
    const int64_t kk = rest % e.CS;
    rest /= e.CS;
    const int64_t chunk = rest % e.nchunks;
    const int64_t tile = rest / e.nchunks;
    const int64_t k = chunk * e.CS + kk;
    float vals[2];
    int exps[2];
    for (int h = 0; h < 2; ++h) {
      const int64_t r = tile * kTile + rp * 2 + h;
      float v = 0.0f;
      int ex = kZeroExp;
      if (r < e.rows && k < e.K) {
        v = load_as_float(e.v, e.dt, r * e.K + k);
        if (!decode_elem(v, e.f, ex)) bad = true;
        if (e.scale) {
          float s = e.scale[r * e.nkd + k / e.kd];
          Term ts = decode_term(s, e.sf);
          bool zero = ts.zero || (e.field0 && f2u(s) == 0x00400000u);
          if (ts.nan || ts.inf || (!zero && (ts.sig != 1 || ts.neg))) bad = true;  // pow2 scales only
          if (zero || ex == kZeroExp) {
            v = 0.0f;
            ex = kZeroExp;
          } else {
            // Folded labels in [-50, 60]: products stay normal fp32 values, and a chunk with a non-zero
            // product has emax >= -100, so its scale 2**(F - emax) is a normal fp32 power.
            if (ts.exp < -60 || ts.exp > 60 || ex + ts.exp < -50 || ex + ts.exp > 60) bad = true;
            v = ldexpf(v, ts.exp);
            ex += ts.exp;
          }
        }
      }
      if (ex == kZeroExp) v = 0.0f;
      vals[h] = v;
      exps[h] = ex;
    }
    const int64_t base = ((tile * e.nchunks + chunk) * e.CS + kk) * kTile;
    if (e.sgn) {
      static_cast<T *>(e.sgn)[base + rp * 2] = signbit(vals[0]) ? (T)-1 : (T)1;
      static_cast<T *>(e.sgn)[base + rp * 2 + 1] = signbit(vals[1]) ? (T)-1 : (T)1;
      vals[0] = fabsf(vals[0]);
      vals[1] = fabsf(vals[1]);
    }
    const int c0 = e.side ? bcol<T>((int)rp * 2) : (int)rp * 2;  // B: the loads' column order
    const int c1 = e.side ? bcol<T>((int)rp * 2 + 1) : (int)rp * 2 + 1;
    static_cast<T *>(e.val)[base + c0] = (T)vals[0];
    static_cast<T *>(e.val)[base + c1] = (T)vals[1];
    if (e.side == 0) {
      e.exp[base / 2 + rp] = ((uint32_t)exps[0] & 0xFFFFu) | ((uint32_t)exps[1] << 16);
    } else {
      e.exp[base + rp * 2] = ((uint32_t)exps[0] & 0xFFFFu) | ((uint32_t)exps[0] << 16);
      e.exp[base + rp * 2 + 1] = ((uint32_t)exps[1] & 0xFFFFu) | ((uint32_t)exps[1] << 16);
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicExch(e.flag, 1);
}

template <int CS, class T>
struct Stage {
  T av[CS][kTile];
  T bv[CS][kTile];
  uint32_t be[CS][kTile];
  uint32_t ae[CS][kTile / 2];
};

}  // namespace cofda
}  // namespace tc
