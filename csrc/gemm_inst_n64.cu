// Instantiations of the tcgen05 GEMM kernel: non-transposed store, N tile 64.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>

#include "gemm_tc.cuh"

namespace gb {

GemmLauncher gemm_launcher_n64(int epi) {
  switch (epi) {
    case kStoreBF16: return &launch_gemm<64, kStoreBF16, false>;
    case kSwiGLU: return &launch_gemm<64, kSwiGLU, false>;
    case kAtomicF32: return &launch_gemm<64, kAtomicF32, false>;
    case kLSE: return &launch_gemm<64, kLSE, false>;
    case kStoreF32: return &launch_gemm<64, kStoreF32, false>;
    case kSoftmaxGrad: return &launch_gemm<64, kSoftmaxGrad, false>;
    default: return nullptr;
  }
}
}  // namespace gb
