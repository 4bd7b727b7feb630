// Host-side support of the C ABI: format derivation, thread-local error messages, version.
#include <atomic>
#include <cmath>
#include <cstring>
#include <string>

#include "tc_common.cuh"

namespace tc {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const std::string &msg) { g_last_error = msg; }

static std::atomic<int> g_wait_polls{-1};
int wait_polls() { return g_wait_polls.load(std::memory_order_relaxed); }

int sm_count() {
  static std::atomic<int> counts[128];
  int dev = 0;
  // A failed query leaves a grid of one block per 'SM' of a one-SM device: slower, never wrong (the
  // kernels are grid-stride), and the launch reports the CUDA error anyway.
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 1;
  int c = counts[dev].load(std::memory_order_relaxed);
  if (c <= 0) {
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) return 1;
    counts[dev].store(c, std::memory_order_relaxed);
  }
  return c;
}

static uint32_t host_f2u(float v) {
  uint32_t u;
  std::memcpy(&u, &v, 4);
  return u;
}

// Float-format range (src/tricast/formats.py:74-99).
static void float_range(const tc_format &f, int &emin, int &emax, double &maxn) {
  emin = 1 - f.bias;
  int top = (1 << f.ebits) - 1 - (f.special == 0 ? 1 : 0);
  emax = top - f.bias;
  int kept = f.special == 1 ? f.mbits - 1 : f.mbits;
  maxn = (2.0 - std::ldexp(1.0, -kept)) * std::ldexp(1.0, emax);
}

std::string fmt_error(const tc_format &f) {
  if (f.kind == 0) {
    if (f.ebits < 1 || f.ebits > 8 || f.mbits < 0 || f.mbits > 23 || f.special < 0 || f.special > 3)
      return "float format fields out of range";
    int emin, emax;
    double m;
    float_range(f, emin, emax, m);
    if (emin < -126 || emax > 127) return "float format exponent range exceeds fp32";
    return "";
  }
  if (f.kind == 1) {
    if (f.bits < 1 || f.bits > 24 || (f.is_signed && f.bits < 2)) return "int format bits out of range";
    return "";
  }
  if (f.kind == 2) {
    if (f.ebits < 1 || f.ebits > 8) return "pow2 format ebits out of range";
    return "";
  }
  return "unknown format kind";
}

double fmt_max_normal(const tc_format &f) {
  if (f.kind == 0) {
    int emin, emax;
    double m;
    float_range(f, emin, emax, m);
    return m;
  }
  if (f.kind == 1) {
    int64_t qmax = f.is_signed ? (1ll << (f.bits - 1)) - 1 : (1ll << f.bits) - 1;
    return std::ldexp((double)qmax, -f.frac_bits);
  }
  return std::ldexp(1.0, (1 << f.ebits) - 2 - f.bias);
}

double fmt_min_scale(const tc_format &f) {
  if (f.kind == 0) {
    int emin = 1 - f.bias;
    return f.subnormals ? std::ldexp(1.0, emin - f.mbits) : std::ldexp(1.0, emin);
  }
  if (f.kind == 1) return std::ldexp(1.0, -f.frac_bits);
  return std::ldexp(1.0, -f.bias);
}

int fmt_emax_elem(const tc_format &f) {
  int e;
  std::frexp(fmt_max_normal(f), &e);
  return e - 1;
}

Fmt derive(const tc_format &f) {
  Fmt d;
  std::memset(&d, 0, sizeof(d));
  d.kind = f.kind;
  d.is_signed = f.is_signed;
  if (f.kind == 0) {
    double m;
    float_range(f, d.emin, d.emax, m);
    d.mbits = f.mbits;
    d.special = f.special;
    d.subnormals = f.subnormals;
    d.max_bits = host_f2u((float)m);
    d.min_normal_bits = host_f2u((float)std::ldexp(1.0, d.emin));
    d.min_sub_bits = host_f2u((float)fmt_min_scale(f));
    d.bias = f.bias;
    d.ebits = f.ebits;
  } else if (f.kind == 1) {
    d.frac_bits = f.frac_bits;
    d.qmin = !f.is_signed ? 0 : -(1ll << (f.bits - 1)) + (f.symmetric ? 1 : 0);
    d.qmax = f.is_signed ? (1ll << (f.bits - 1)) - 1 : (1ll << f.bits) - 1;
    d.max_bits = host_f2u((float)fmt_max_normal(f));
    d.min_normal_bits = host_f2u((float)std::ldexp(1.0, -f.frac_bits));
    d.min_sub_bits = d.min_normal_bits;
    // k * 2**-frac is exact in fp32 when the finest step is >= 2**-149 and the top fits.
    d.int_double = (-f.frac_bits < -149) || (25 - f.frac_bits > 127);
    d.subnormals = 1;
    d.special = 3;
  } else {
    d.emin = -f.bias;
    d.emax = (1 << f.ebits) - 2 - f.bias;
    d.max_bits = host_f2u((float)std::ldexp(1.0, d.emax));
    d.min_normal_bits = host_f2u((float)std::ldexp(1.0, d.emin));
    d.min_sub_bits = d.min_normal_bits;
    d.bias = f.bias;
    d.ebits = f.ebits;
    d.special = 3;
  }
  return d;
}

}  // namespace tc

extern "C" const char *tc_last_error(void) { return tc::g_last_error.c_str(); }

extern "C" uint64_t tc_launch_count(void) { return tc::g_launches.load(std::memory_order_relaxed); }

extern "C" int tc_set_wait_limit(int32_t polls) {
  tc::g_wait_polls.store(polls < 0 ? -1 : polls, std::memory_order_relaxed);
  return TC_OK;
}

extern "C" const char *tc_version(void) { return "tricast_b200 0.1.0 (sm_100a)"; }
