// Lean group-quantize kernels writing 4-bit element codes (one translation unit per code width,
// compiled in parallel).
#include "tc_quant_lean.cuh"

namespace tc {

void launch_group_lean_c4(const LeanArgs &a, int grid, int gi, bool pow2, bool fast, int out, cudaStream_t s) {
  launch_group_lean_cb<4>(a, grid, gi, pow2, fast, out, s);
}

}  // namespace tc
