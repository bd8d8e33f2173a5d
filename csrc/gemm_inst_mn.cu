// Instantiations of the tcgen05 GEMM kernel with MN-major operands: dgrad
// against the frozen weight as stored (B = W [N_out, K_in] read MN-major, no
// transposed copy) and LoRA gradients contracted over tokens (both operands
// MN-major, split-K fp32 atomics into the gradient).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>

#include "gemm_tc.cuh"

namespace gb {

GemmLauncher gemm_launcher_mn(int bn, int epi, bool swap, int layout) {
  if (layout == 1 && !swap && epi == kStoreBF16) {
    switch (bn) {
      case 256: return &launch_gemm<256, kStoreBF16, false, 1>;
      case 128: return &launch_gemm<128, kStoreBF16, false, 1>;
      case 64: return &launch_gemm<64, kStoreBF16, false, 1>;
      default: return nullptr;
    }
  }
  if (layout == 3 && bn == 64 && epi == kAtomicF32) {
    return swap ? &launch_gemm<64, kAtomicF32, true, 3> : &launch_gemm<64, kAtomicF32, false, 3>;
  }
  return nullptr;
}

}  // namespace gb
