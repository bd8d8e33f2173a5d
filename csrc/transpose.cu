// Tiled bf16 matrix transpose through shared memory (32x32 tiles, padded to
// avoid bank conflicts).  Used to present activations / output gradients
// K-major to the tensor-core GEMM for the LoRA weight-gradient reductions,
// where the reduction runs over tokens.

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "sm100_common.cuh"

namespace gb {

namespace {
__global__ void transpose_bf16_kernel(const __nv_bfloat16* __restrict__ in, long ldin,
                                      __nv_bfloat16* __restrict__ out, long ldout, int rows, int cols) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = in[static_cast<long>(r) * ldin + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[static_cast<long>(c) * ldout + r] = tile[threadIdx.x][i];
  }
}
}  // namespace

// out[c, r] = in[r, c]
void transpose_bf16(torch::Tensor in, torch::Tensor out) {
  const c10::cuda::CUDAGuard guard(in.device());
  TORCH_CHECK(in.dim() == 2 && out.dim() == 2 && in.stride(1) == 1 && out.stride(1) == 1, "2-D row-major tensors");
  TORCH_CHECK(in.scalar_type() == torch::kBFloat16 && out.scalar_type() == torch::kBFloat16, "bf16 only");
  const int rows = static_cast<int>(in.size(0)), cols = static_cast<int>(in.size(1));
  TORCH_CHECK(out.size(0) == cols && out.size(1) == rows, "shape mismatch");
  if (rows == 0 || cols == 0) return;
  dim3 grid((cols + 31) / 32, (rows + 31) / 32);
  transpose_bf16_kernel<<<grid, dim3(32, 8), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(in.data_ptr()), in.stride(0),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), rows, cols);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace gb
