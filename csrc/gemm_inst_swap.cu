// Instantiations of the tcgen05 GEMM kernel: transposed store (swap-AB decode GEMMs), N tiles 32/64/128.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>

#include "gemm_tc.cuh"

namespace gb {

template <int BN>
static GemmLauncher swap_for(int epi) {
  switch (epi) {
    case kStoreBF16: return &launch_gemm<BN, kStoreBF16, true>;
    case kSwiGLU: return &launch_gemm<BN, kSwiGLU, true>;
    case kAtomicF32: return &launch_gemm<BN, kAtomicF32, true>;
    case kStoreF32: return &launch_gemm<BN, kStoreF32, true>;
    default: return nullptr;
  }
}

GemmLauncher gemm_launcher_swap(int bn, int epi) {
  switch (bn) {
    case 32: return swap_for<32>(epi);
    case 64: return swap_for<64>(epi);
    case 128: return swap_for<128>(epi);
    default: return nullptr;
  }
}
}  // namespace gb
