// Elementwise / short-window kernels of the Qwen3.5 hybrid (gated DeltaNet +
// gated attention) decoder, forward and backward.
// Reference counterparts (PyTorch there): the causal depthwise conv1d + SiLU of
// the DeltaNet mixer, the gated RMSNorm of its output and the sigmoid output
// gate of the gated attention (src/graspo/backends/graspoflow/models/common/
// layers.py:358-633, tensor_utils.py:490-646).
//
// * conv_silu_fwd   y[b, t, c] = silu(sum_j w[c, j] * x[b, t - (K-1) + j, c]),
//                   channels-last [B, S, C] in and out (no transposes), the
//                   K-1 positions before t = 0 read from an optional carried
//                   state [B, C, K-1] (zeros without one); fp32 accumulation.
// * conv_silu_bwd   dx[b, t, c] = sum_j w[c, j] * dpre[b, t + (K-1) - j, c] with
//                   dpre = dy * silu'(pre) recomputed from x (the conv weight
//                   is frozen: no weight gradient).
// * gated_rmsnorm_fwd / _bwd  y = w * bf16(rmsnorm(x)) * silu(z) per row of D
//                   (fp32 statistics), gradients for x and z (w frozen).
// * sigmoid_gate_fwd / _bwd   y = o * sigmoid(g), gradients for o and g.

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>

#include "sm100_common.cuh"

namespace gb {

namespace {

constexpr int kMaxK = 8;

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) {
  if constexpr (sizeof(T) == 2) return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
  else return static_cast<float>(*p);
}

template <typename T>
__device__ __forceinline__ void st_f(T* p, float v) {
  if constexpr (sizeof(T) == 2) *reinterpret_cast<__nv_bfloat16*>(p) = __float2bfloat16(v);
  else *p = v;
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }

// input at (b, t, c) for t in [-(K-1), S): the carried state before t = 0
template <typename T>
__device__ __forceinline__ float conv_in(const T* x, const T* prev, int b, int t, int c, int S, int C, int K) {
  if (t >= 0) return ld_f(x + (static_cast<long>(b) * S + t) * C + c);
  if (prev == nullptr) return 0.f;
  return ld_f(prev + (static_cast<long>(b) * C + c) * (K - 1) + (K - 1 + t));
}

template <typename T>
__global__ void conv_silu_fwd_kernel(const T* __restrict__ x, const T* __restrict__ prev,
                                     const T* __restrict__ w, T* __restrict__ y, int B, int S, int C, int K) {
  const long n = static_cast<long>(B) * S * C;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % C);
    const long bt = i / C;
    const int t = static_cast<int>(bt % S), b = static_cast<int>(bt / S);
    float acc = 0.f;
    for (int j = 0; j < K; ++j) acc = fmaf(ld_f(w + static_cast<long>(c) * K + j),
                                           conv_in(x, prev, b, t - (K - 1) + j, c, S, C, K), acc);
    st_f(y + i, acc * sigmoid_f(acc));
  }
}

template <typename T>
__global__ void conv_silu_bwd_kernel(const T* __restrict__ x, const T* __restrict__ prev,
                                     const T* __restrict__ w, const T* __restrict__ dy, T* __restrict__ dx,
                                     int B, int S, int C, int K) {
  const long n = static_cast<long>(B) * S * C;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % C);
    const long bt = i / C;
    const int t = static_cast<int>(bt % S), b = static_cast<int>(bt / S);
    float wc[kMaxK];
    for (int j = 0; j < K; ++j) wc[j] = ld_f(w + static_cast<long>(c) * K + j);
    float acc = 0.f;
    // x[t] feeds outputs u = t + (K-1) - j for j = 0..K-1 (u < S)
    for (int j = 0; j < K; ++j) {
      const int u = t + (K - 1) - j;
      if (u >= S) continue;
      float pre = 0.f;
      for (int jj = 0; jj < K; ++jj) pre = fmaf(wc[jj], conv_in(x, prev, b, u - (K - 1) + jj, c, S, C, K), pre);
      const float s = sigmoid_f(pre);
      const float dsilu = s * (1.f + pre * (1.f - s));
      acc = fmaf(wc[j], ld_f(dy + (static_cast<long>(b) * S + u) * C + c) * dsilu, acc);
    }
    st_f(dx + i, acc);
  }
}

// one warp per row of D (D <= 1024)
template <typename T>
__global__ void gated_rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                         const T* __restrict__ w, T* __restrict__ y, long rows, int D, float eps) {
  const long row = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * D;
  float ss = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float v = ld_f(xr + d);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / D + eps);
  for (int d = lane; d < D; d += 32) {
    // the normalised value is rounded to the activation type before the gate, as in the eager model
    float nv = ld_f(xr + d) * rstd;
    if constexpr (sizeof(T) == 2) nv = __bfloat162float(__float2bfloat16(nv));
    const float zv = ld_f(z + row * D + d);
    st_f(y + row * D + d, ld_f(w + d) * nv * (zv * sigmoid_f(zv)));
  }
}

template <typename T>
__global__ void gated_rmsnorm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                         const T* __restrict__ w, const T* __restrict__ dy, T* __restrict__ dx,
                                         T* __restrict__ dz, long rows, int D, float eps) {
  const long row = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * D;
  float ss = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float v = ld_f(xr + d);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / D + eps);
  // g = dL/d(normalised x) = dy * w * silu(z); dx = rstd * (g - xhat * mean(g * xhat))
  float gx = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float zv = ld_f(z + row * D + d);
    const float g = ld_f(dy + row * D + d) * ld_f(w + d) * (zv * sigmoid_f(zv));
    gx = fmaf(g, ld_f(xr + d) * rstd, gx);
  }
  gx = warp_sum(gx) / D;
  for (int d = lane; d < D; d += 32) {
    const float xv = ld_f(xr + d);
    const float zv = ld_f(z + row * D + d);
    const float s = sigmoid_f(zv);
    const float dyv = ld_f(dy + row * D + d);
    const float wv = ld_f(w + d);
    const float xhat = xv * rstd;
    float nv = xhat;
    if constexpr (sizeof(T) == 2) nv = __bfloat162float(__float2bfloat16(nv));
    const float g = dyv * wv * (zv * s);
    st_f(dx + row * D + d, rstd * (g - xhat * gx));
    st_f(dz + row * D + d, dyv * wv * nv * s * (1.f + zv * (1.f - s)));
  }
}

template <typename T>
__global__ void sigmoid_gate_fwd_kernel(const T* __restrict__ o, const T* __restrict__ g, T* __restrict__ y, long n) {
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    st_f(y + i, ld_f(o + i) * sigmoid_f(ld_f(g + i)));
}

template <typename T>
__global__ void sigmoid_gate_bwd_kernel(const T* __restrict__ o, const T* __restrict__ g, const T* __restrict__ dy,
                                        T* __restrict__ dout, T* __restrict__ dg, long n) {
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float s = sigmoid_f(ld_f(g + i));
    const float d = ld_f(dy + i);
    st_f(dout + i, d * s);
    st_f(dg + i, d * ld_f(o + i) * s * (1.f - s));
  }
}

int grid_for(long n, int threads, const torch::Tensor& t) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, t.get_device());
  return static_cast<int>(std::max<long>(1, std::min<long>((n + threads - 1) / threads, 16L * sms)));
}

void check_act(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() &&
                  (t.scalar_type() == torch::kBFloat16 || t.scalar_type() == torch::kFloat32),
              name, " must be a contiguous bf16 or fp32 CUDA tensor");
}

}  // namespace

#define GB_DISPATCH(T_, ...)                                        \
  if ((T_).scalar_type() == torch::kBFloat16) {                    \
    using scalar = __nv_bfloat16;                                   \
    __VA_ARGS__;                                                    \
  } else {                                                          \
    using scalar = float;                                           \
    __VA_ARGS__;                                                    \
  }

// x [B, S, C], prev optional [B, C, K-1], w [C, K] -> y [B, S, C]
void conv_silu_fwd(torch::Tensor x, c10::optional<torch::Tensor> prev, torch::Tensor w, torch::Tensor y) {
  check_act(x, "x");
  check_act(w, "w");
  check_act(y, "y");
  TORCH_CHECK(x.dim() == 3 && w.dim() == 2 && w.size(0) == x.size(2) && w.size(1) <= kMaxK && w.size(1) >= 1,
              "x [B, S, C] and w [C, K <= 8]");
  TORCH_CHECK(w.scalar_type() == x.scalar_type() && y.scalar_type() == x.scalar_type() && y.sizes() == x.sizes(),
              "x, w and y share dtype; y matches x");
  const int B = static_cast<int>(x.size(0)), S = static_cast<int>(x.size(1)), C = static_cast<int>(x.size(2));
  const int K = static_cast<int>(w.size(1));
  const bool hp = prev.has_value() && prev->defined();
  if (hp) {
    check_act(*prev, "prev");
    TORCH_CHECK(prev->scalar_type() == x.scalar_type() && prev->dim() == 3 && prev->size(0) == B &&
                    prev->size(1) == C && prev->size(2) == K - 1, "prev must be [B, C, K-1]");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  const long n = static_cast<long>(B) * S * C;
  if (n == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  GB_DISPATCH(x, conv_silu_fwd_kernel<scalar><<<grid_for(n, 256, x), 256, 0, stream>>>(
                     reinterpret_cast<const scalar*>(x.data_ptr()),
                     hp ? reinterpret_cast<const scalar*>(prev->data_ptr()) : nullptr,
                     reinterpret_cast<const scalar*>(w.data_ptr()), reinterpret_cast<scalar*>(y.data_ptr()), B, S, C, K));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void conv_silu_bwd(torch::Tensor x, c10::optional<torch::Tensor> prev, torch::Tensor w, torch::Tensor dy,
                   torch::Tensor dx) {
  check_act(x, "x");
  check_act(dy, "dy");
  check_act(dx, "dx");
  TORCH_CHECK(dy.sizes() == x.sizes() && dx.sizes() == x.sizes() && dy.scalar_type() == x.scalar_type() &&
                  dx.scalar_type() == x.scalar_type() && w.scalar_type() == x.scalar_type() &&
                  w.size(0) == x.size(2) && w.size(1) <= kMaxK, "shapes / dtypes of the conv backward");
  const int B = static_cast<int>(x.size(0)), S = static_cast<int>(x.size(1)), C = static_cast<int>(x.size(2));
  const int K = static_cast<int>(w.size(1));
  const bool hp = prev.has_value() && prev->defined();
  const c10::cuda::CUDAGuard guard(x.device());
  const long n = static_cast<long>(B) * S * C;
  if (n == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  GB_DISPATCH(x, conv_silu_bwd_kernel<scalar><<<grid_for(n, 256, x), 256, 0, stream>>>(
                     reinterpret_cast<const scalar*>(x.data_ptr()),
                     hp ? reinterpret_cast<const scalar*>(prev->data_ptr()) : nullptr,
                     reinterpret_cast<const scalar*>(w.data_ptr()), reinterpret_cast<const scalar*>(dy.data_ptr()),
                     reinterpret_cast<scalar*>(dx.data_ptr()), B, S, C, K));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// x, z [rows, D], w [D] -> y [rows, D]
void gated_rmsnorm_fwd(torch::Tensor x, torch::Tensor z, torch::Tensor w, torch::Tensor y, double eps) {
  check_act(x, "x");
  check_act(z, "z");
  check_act(w, "w");
  check_act(y, "y");
  const int D = static_cast<int>(x.size(-1));
  TORCH_CHECK(z.sizes() == x.sizes() && y.sizes() == x.sizes() && w.numel() == D &&
                  z.scalar_type() == x.scalar_type() && y.scalar_type() == x.scalar_type() &&
                  w.scalar_type() == x.scalar_type(), "gated RMSNorm operands must match");
  const long rows = x.numel() / D;
  const c10::cuda::CUDAGuard guard(x.device());
  if (rows == 0) return;
  const int blocks = static_cast<int>((rows * 32 + 255) / 256);
  GB_DISPATCH(x, gated_rmsnorm_fwd_kernel<scalar><<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
                     reinterpret_cast<const scalar*>(x.data_ptr()), reinterpret_cast<const scalar*>(z.data_ptr()),
                     reinterpret_cast<const scalar*>(w.data_ptr()), reinterpret_cast<scalar*>(y.data_ptr()), rows, D,
                     static_cast<float>(eps)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gated_rmsnorm_bwd(torch::Tensor x, torch::Tensor z, torch::Tensor w, torch::Tensor dy, torch::Tensor dx,
                       torch::Tensor dz, double eps) {
  check_act(x, "x");
  check_act(dy, "dy");
  const int D = static_cast<int>(x.size(-1));
  TORCH_CHECK(z.sizes() == x.sizes() && dy.sizes() == x.sizes() && dx.sizes() == x.sizes() &&
                  dz.sizes() == x.sizes() && w.numel() == D, "gated RMSNorm backward operands must match");
  const long rows = x.numel() / D;
  const c10::cuda::CUDAGuard guard(x.device());
  if (rows == 0) return;
  const int blocks = static_cast<int>((rows * 32 + 255) / 256);
  GB_DISPATCH(x, gated_rmsnorm_bwd_kernel<scalar><<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
                     reinterpret_cast<const scalar*>(x.data_ptr()), reinterpret_cast<const scalar*>(z.data_ptr()),
                     reinterpret_cast<const scalar*>(w.data_ptr()), reinterpret_cast<const scalar*>(dy.data_ptr()),
                     reinterpret_cast<scalar*>(dx.data_ptr()), reinterpret_cast<scalar*>(dz.data_ptr()), rows, D,
                     static_cast<float>(eps)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void sigmoid_gate_fwd(torch::Tensor o, torch::Tensor g, torch::Tensor y) {
  check_act(o, "o");
  check_act(g, "g");
  check_act(y, "y");
  TORCH_CHECK(g.sizes() == o.sizes() && y.sizes() == o.sizes() && g.scalar_type() == o.scalar_type() &&
                  y.scalar_type() == o.scalar_type(), "gate operands must match");
  const c10::cuda::CUDAGuard guard(o.device());
  const long n = o.numel();
  if (n == 0) return;
  GB_DISPATCH(o, sigmoid_gate_fwd_kernel<scalar><<<grid_for(n, 256, o), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
                     reinterpret_cast<const scalar*>(o.data_ptr()), reinterpret_cast<const scalar*>(g.data_ptr()),
                     reinterpret_cast<scalar*>(y.data_ptr()), n));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void sigmoid_gate_bwd(torch::Tensor o, torch::Tensor g, torch::Tensor dy, torch::Tensor dout, torch::Tensor dg) {
  check_act(o, "o");
  check_act(dy, "dy");
  TORCH_CHECK(g.sizes() == o.sizes() && dy.sizes() == o.sizes() && dout.sizes() == o.sizes() &&
                  dg.sizes() == o.sizes(), "gate backward operands must match");
  const c10::cuda::CUDAGuard guard(o.device());
  const long n = o.numel();
  if (n == 0) return;
  GB_DISPATCH(o, sigmoid_gate_bwd_kernel<scalar><<<grid_for(n, 256, o), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
                     reinterpret_cast<const scalar*>(o.data_ptr()), reinterpret_cast<const scalar*>(g.data_ptr()),
                     reinterpret_cast<const scalar*>(dy.data_ptr()), reinterpret_cast<scalar*>(dout.data_ptr()),
                     reinterpret_cast<scalar*>(dg.data_ptr()), n));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

#undef GB_DISPATCH

}  // namespace gb
