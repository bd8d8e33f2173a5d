// Consumer half of the fused tensor-parallel all-reduce / reduce-scatter of
// prefill and training (the producer half is the GEMM epilogue's slot push,
// GemmArgs::out_push in gemm_tc.cuh).
//
// Reference counterpart: the NCCL all-reduce after the row-parallel o_proj /
// down_proj (src/graspo/backends/graspoflow/tensor_utils.py:146-164, called from
// models/common/layers_qwen3.py:263-264, 333-335) and its backward conjugate.
//
// Every rank's GEMM stores its bf16 partial tiles into the receive slot that
// belongs to it in every destination rank's symmetric buffer (its own slot in
// its own buffer included) and adds the element counts to the remote
// destinations' 64-bit arrival counters.  tp_reduce waits (bounded) until this
// rank's counter has reached the cumulative count expected after this site,
// then writes out = residual + sum over ranks of slot[q], adding the slots in
// rank order with fp32 arithmetic, so every rank of the group produces the same
// bits.  The counter is never reset: the host keeps the cumulative expectation.
//
// Wait bound: `spin_limit` SM clock cycles (0: 10 x kSpinLimitCycles, about
// 10 s); when it runs out the kernel records kErrPeerTimeout in the error word,
// writes nothing and returns, and the host raises KernelTimeout.

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>

#include "sm100_common.cuh"

namespace gb {

namespace {

constexpr int kReduceThreads = 256;
constexpr int kMaxRanks = 8;
// Kernels that spin on arrival counters keep their grid to two 256-thread CTAs
// per SM, so a kernel that signals a peer (sent from this GPU's side stream) is
// never starved of an SM by them: the peers' waits can only end once this
// GPU's own signals have run.
constexpr long kWaitCtasPerSm = 2;

struct ReduceArgs {
  const __nv_bfloat16* src[kMaxRanks];
  int nsrc;
  const unsigned long long* counter;
  unsigned long long expected;
  const __nv_bfloat16* residual;  // may be null
  long ld_res;
  __nv_bfloat16* out;
  long ld_out;
  long ld_src;
  int rows, cols;                 // cols a multiple of 8
  int* err;
  long long spin_limit;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kReduceThreads) tp_reduce_kernel(ReduceArgs a) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int good = 1;
    if (a.counter != nullptr) {
      const long long t0 = clock64();
      while (ld_acquire_sys_u64(a.counter) < a.expected) {
        if (clock64() - t0 > a.spin_limit) {
          record_error(a.err, kErrPeerTimeout);
          good = 0;
          break;
        }
        __nanosleep(128);
      }
    }
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const int vec_per_row = a.cols / 8;
  const long total = static_cast<long>(a.rows) * vec_per_row;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long r = i / vec_per_row;
    const int c = static_cast<int>(i - r * vec_per_row) * 8;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int q = 0; q < a.nsrc; ++q) {
      // L2 loads: the slots were written by peers over NVLink after this kernel may have started
      const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(a.src[q] + r * a.ld_src + c));
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += __bfloat162float(b[e]);
    }
    if (a.residual != nullptr) {
      const uint4 raw = *reinterpret_cast<const uint4*>(a.residual + r * a.ld_res + c);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += __bfloat162float(b[e]);
    }
    uint4 pk;
    __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
    for (int e = 0; e < 4; ++e) p2[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
    *reinterpret_cast<uint4*>(a.out + r * a.ld_out + c) = pk;
  }
}

// ---------------------------------------------------------------------------
// Vocab-parallel selected-token log-prob: every rank holds the LM-head logits
// of its vocabulary shard.  lse_push merges the shard's per-tile (max,
// sum-exp) partials of row t into the shard's log-sum-exp and stores the pair
// (lse_q, target logit or 0) into slot q of every rank (float2 per row), then
// signals the remote ranks; lse_merge waits for the pairs of all ranks and
// writes lse = log sum_q exp(lse_q) and logp = sum_q tgt_q - lse, in rank
// order on every rank.
struct PairPushArgs {
  const float2* part;  // [T, ld] partials of this shard
  long ld;
  int nblk;
  const float* tgt;    // [T] target logit where the target is in this shard, else 0
  float2* dst[kMaxRanks];
  unsigned long long* sig[kMaxRanks];
  int nranks, self, T;
};

__global__ void lse_push_kernel(PairPushArgs a) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t < a.T) {
    float m = -INFINITY, s = 0.f;
    for (int b = lane; b < a.nblk; b += 32) {
      const float2 p = a.part[static_cast<long>(t) * a.ld + b];
      if (p.x == -INFINITY) continue;
      const float mn = fmaxf(m, p.x);
      s = s * __expf(m - mn) + p.y * __expf(p.x - mn);
      m = mn;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const float os = __shfl_xor_sync(0xffffffffu, s, o);
      const float mn = fmaxf(m, om);
      if (mn == -INFINITY) continue;
      s = s * __expf(m - mn) + os * __expf(om - mn);
      m = mn;
    }
    if (lane < a.nranks) a.dst[lane][t] = make_float2(m + logf(s), a.tgt[t]);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int first = blockIdx.x * (blockDim.x >> 5);
    const int rows = max(0, min(a.T, first + static_cast<int>(blockDim.x >> 5)) - first);
    for (int q = 0; q < a.nranks; ++q)
      if (q != a.self && rows > 0)
        asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(a.sig[q]),
                     "l"(static_cast<unsigned long long>(rows)) : "memory");
  }
}

struct PairMergeArgs {
  const float2* src[kMaxRanks];
  int nranks, T;
  const unsigned long long* counter;
  unsigned long long expected;
  float* lse;
  float* logp;
  int* err;
  long long spin_limit;
};

__global__ void lse_merge_kernel(PairMergeArgs a) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int good = 1;
    const long long t0 = clock64();
    while (ld_acquire_sys_u64(a.counter) < a.expected) {
      if (clock64() - t0 > a.spin_limit) {
        record_error(a.err, kErrPeerTimeout);
        good = 0;
        break;
      }
      __nanosleep(128);
    }
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < a.T; t += gridDim.x * blockDim.x) {
    float m = -INFINITY, tg = 0.f;
    float2 v[kMaxRanks];
    for (int q = 0; q < a.nranks; ++q) {
      v[q] = __ldcg(a.src[q] + t);
      m = fmaxf(m, v[q].x);
    }
    float s = 0.f;
    for (int q = 0; q < a.nranks; ++q) {
      s += __expf(v[q].x - m);
      tg += v[q].y;
    }
    const float l = m + logf(s);
    a.lse[t] = l;
    a.logp[t] = tg - l;
  }
}

// ---------------------------------------------------------------------------
// Data-parallel LoRA-gradient all-reduce.  During the backward each layer's
// finished gradient slices are copied into every DP peer's receive slot by the
// copy engines on a side stream (cudaMemcpyAsync to the CUDA-IPC mapped
// address, overlapping the remaining layers' backward), followed by
// signal_kernel, which adds the copied element count to the peers' 64-bit
// arrival counters.  dp_reduce_kernel then waits (bounded) for all peers'
// slices and writes g = scale * sum over ranks of g_q, in rank order (this
// rank's own term read from its gradient buffer), so every DP replica holds the
// same bits.
struct SignalArgs {
  unsigned long long* ctr[kMaxRanks];
  int n;
  unsigned long long count;
};

__global__ void signal_kernel(SignalArgs a) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  for (int q = 0; q < a.n; ++q)
    if (a.ctr[q] != nullptr)
      asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(a.ctr[q]), "l"(a.count) : "memory");
}

struct DPReduceArgs {
  float* grads;                     // this rank's gradients (its own term, overwritten with the result)
  const float* src[kMaxRanks];      // per rank: receive slot, or nullptr for this rank
  int nranks;
  long n;
  float scale;
  const unsigned long long* counter;
  unsigned long long expected;
  int* err;
  long long spin_limit;
};

__global__ void __launch_bounds__(256) dp_reduce_kernel(DPReduceArgs a) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int good = 1;
    const long long t0 = clock64();
    while (ld_acquire_sys_u64(a.counter) < a.expected) {
      if (clock64() - t0 > a.spin_limit) {
        record_error(a.err, kErrPeerTimeout);
        good = 0;
        break;
      }
      __nanosleep(128);
    }
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const long n4 = a.n / 4;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < a.nranks; ++q) {
      const float4 v = a.src[q] != nullptr ? __ldcg(reinterpret_cast<const float4*>(a.src[q]) + i)
                                           : reinterpret_cast<const float4*>(a.grads)[i];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    reinterpret_cast<float4*>(a.grads)[i] =
        make_float4(acc.x * a.scale, acc.y * a.scale, acc.z * a.scale, acc.w * a.scale);
  }
  for (long i = n4 * 4 + blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < a.n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    float acc = 0.f;
    for (int q = 0; q < a.nranks; ++q) acc += a.src[q] != nullptr ? __ldcg(a.src[q] + i) : a.grads[i];
    a.grads[i] = acc * a.scale;
  }
}

}  // namespace

// Copy `nbytes` from a local tensor (at a byte offset) to a device address on
// the current stream -- a CUDA-IPC mapped peer buffer -- with the copy engines.
void peer_copy(int64_t dst, torch::Tensor src, int64_t src_offset_bytes, int64_t nbytes) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous(), "peer_copy source must be a contiguous CUDA tensor");
  TORCH_CHECK(src_offset_bytes >= 0 && nbytes >= 0 &&
                  src_offset_bytes + nbytes <= static_cast<int64_t>(src.numel() * src.element_size()),
              "peer_copy range outside the source");
  if (nbytes == 0) return;
  const c10::cuda::CUDAGuard guard(src.device());
  C10_CUDA_CHECK(cudaMemcpyAsync(reinterpret_cast<void*>(dst),
                                 static_cast<const uint8_t*>(src.data_ptr()) + src_offset_bytes,
                                 static_cast<size_t>(nbytes), cudaMemcpyDeviceToDevice,
                                 at::cuda::getCurrentCUDAStream()));
}

// Add `count` to each 64-bit counter of the CPU int64 address table (0 entries are skipped).
void signal_counters(torch::Tensor counters, int64_t count) {
  TORCH_CHECK(counters.device().is_cpu() && counters.scalar_type() == torch::kInt64 && counters.numel() <= kMaxRanks,
              "counters: CPU int64 address table of <= 8 entries");
  SignalArgs a{};
  auto c = counters.contiguous();
  a.n = static_cast<int>(c.numel());
  for (int q = 0; q < a.n; ++q) a.ctr[q] = reinterpret_cast<unsigned long long*>(c.data_ptr<int64_t>()[q]);
  a.count = static_cast<unsigned long long>(count);
  signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_CHECK(cudaGetLastError());
}

// grads = scale * sum_q slot_q in rank order (srcs[q] == 0 for this rank: its grads), after a
// bounded wait until this rank's counter reaches `expected`.
void dp_reduce(torch::Tensor grads, torch::Tensor srcs, int64_t counter, int64_t expected, double scale,
               torch::Tensor err, int64_t spin_limit) {
  TORCH_CHECK(grads.is_cuda() && grads.scalar_type() == torch::kFloat32 && grads.is_contiguous(),
              "grads must be a contiguous fp32 CUDA tensor");
  TORCH_CHECK(srcs.device().is_cpu() && srcs.scalar_type() == torch::kInt64 && srcs.numel() >= 1 &&
                  srcs.numel() <= kMaxRanks, "srcs: CPU int64 table of 1..8 addresses");
  const c10::cuda::CUDAGuard guard(grads.device());
  DPReduceArgs a{};
  a.grads = grads.data_ptr<float>();
  auto s = srcs.contiguous();
  a.nranks = static_cast<int>(s.numel());
  for (int q = 0; q < a.nranks; ++q) {
    a.src[q] = reinterpret_cast<const float*>(s.data_ptr<int64_t>()[q]);
    TORCH_CHECK(reinterpret_cast<uintptr_t>(a.src[q]) % 16 == 0, "16-byte aligned slots");
  }
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.grads) % 16 == 0, "16-byte aligned gradients");
  a.n = grads.numel();
  a.scale = static_cast<float>(scale);
  a.counter = reinterpret_cast<const unsigned long long*>(counter);
  a.expected = static_cast<unsigned long long>(expected);
  a.err = err.data_ptr<int>();
  a.spin_limit = spin_limit > 0 ? spin_limit : 10 * kSpinLimitCycles;
  if (a.n == 0) return;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, grads.get_device());
  // two waiting CTAs per SM at most: the side stream's signal kernel must find room (see tp_reduce)
  const int blocks = static_cast<int>(std::min<long>((a.n / 4 + 255) / 256 + 1, kWaitCtasPerSm * sms));
  dp_reduce_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_CHECK(cudaGetLastError());
}

// Vocab-parallel log-prob exchange, producer half (see lse_push_kernel).
void lse_push(torch::Tensor partials, torch::Tensor tgt, torch::Tensor dst, torch::Tensor sig, int64_t self) {
  TORCH_CHECK(partials.is_cuda() && partials.scalar_type() == torch::kFloat32 && partials.dim() == 3 &&
                  partials.size(2) == 2 && partials.stride(2) == 1 && partials.stride(1) == 2,
              "partials: fp32 [T, nblk, 2] with contiguous pairs");
  TORCH_CHECK(tgt.is_cuda() && tgt.scalar_type() == torch::kFloat32 && tgt.is_contiguous() &&
                  tgt.numel() == partials.size(0), "tgt: fp32 [T]");
  TORCH_CHECK(dst.device().is_cpu() && sig.device().is_cpu() && dst.scalar_type() == torch::kInt64 &&
                  sig.scalar_type() == torch::kInt64 && dst.numel() == sig.numel() && dst.numel() >= 1 &&
                  dst.numel() <= kMaxRanks, "dst / sig: CPU int64 tables of 1..8 entries");
  const c10::cuda::CUDAGuard guard(partials.device());
  PairPushArgs a{};
  a.part = reinterpret_cast<const float2*>(partials.data_ptr<float>());
  a.ld = partials.stride(0) / 2;
  a.nblk = static_cast<int>(partials.size(1));
  a.tgt = tgt.data_ptr<float>();
  a.nranks = static_cast<int>(dst.numel());
  a.self = static_cast<int>(self);
  a.T = static_cast<int>(partials.size(0));
  TORCH_CHECK(a.self >= 0 && a.self < a.nranks, "self must index the tables");
  auto d = dst.contiguous(), g = sig.contiguous();
  for (int q = 0; q < a.nranks; ++q) {
    a.dst[q] = reinterpret_cast<float2*>(d.data_ptr<int64_t>()[q]);
    a.sig[q] = reinterpret_cast<unsigned long long*>(g.data_ptr<int64_t>()[q]);
    TORCH_CHECK(a.dst[q] != nullptr && reinterpret_cast<uintptr_t>(a.dst[q]) % 8 == 0, "8-byte aligned slots");
  }
  if (a.T == 0) return;
  constexpr int kThreads = 256;
  const int blocks = (a.T * 32 + kThreads - 1) / kThreads;
  lse_push_kernel<<<blocks, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_CHECK(cudaGetLastError());
}

// Consumer half: bounded wait on this rank's counter, then the merge.
void lse_merge(torch::Tensor srcs, int64_t counter, int64_t expected, torch::Tensor lse, torch::Tensor logp,
               torch::Tensor err, int64_t spin_limit) {
  TORCH_CHECK(srcs.device().is_cpu() && srcs.scalar_type() == torch::kInt64 && srcs.numel() >= 1 &&
                  srcs.numel() <= kMaxRanks, "srcs: CPU int64 table of 1..8 slot addresses");
  TORCH_CHECK(lse.is_cuda() && logp.is_cuda() && lse.scalar_type() == torch::kFloat32 &&
                  logp.scalar_type() == torch::kFloat32 && lse.is_contiguous() && logp.is_contiguous() &&
                  lse.numel() == logp.numel(), "lse / logp: fp32 [T]");
  const c10::cuda::CUDAGuard guard(lse.device());
  PairMergeArgs a{};
  auto s = srcs.contiguous();
  a.nranks = static_cast<int>(s.numel());
  for (int q = 0; q < a.nranks; ++q) a.src[q] = reinterpret_cast<const float2*>(s.data_ptr<int64_t>()[q]);
  a.T = static_cast<int>(lse.numel());
  a.counter = reinterpret_cast<const unsigned long long*>(counter);
  a.expected = static_cast<unsigned long long>(expected);
  a.lse = lse.data_ptr<float>();
  a.logp = logp.data_ptr<float>();
  a.err = err.data_ptr<int>();
  a.spin_limit = spin_limit > 0 ? spin_limit : 10 * kSpinLimitCycles;
  if (a.T == 0) return;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, lse.get_device());
  const int blocks = std::min((a.T + 255) / 256, static_cast<int>(kWaitCtasPerSm) * sms);
  lse_merge_kernel<<<std::max(blocks, 1), 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_CHECK(cudaGetLastError());
}

// srcs: CPU int64 table of slot addresses in rank order (all in this rank's
// buffer); counter: device address of this rank's arrival counter (0: no
// wait); expected: the cumulative count that completes this site.
void tp_reduce(torch::Tensor srcs, int64_t counter, int64_t expected, c10::optional<torch::Tensor> residual,
               torch::Tensor out, int64_t ld_src, torch::Tensor err, int64_t spin_limit) {
  TORCH_CHECK(srcs.device().is_cpu() && srcs.scalar_type() == torch::kInt64 && srcs.numel() >= 1 &&
                  srcs.numel() <= kMaxRanks,
              "srcs: CPU int64 table of 1..8 slot addresses");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kBFloat16 && out.dim() == 2 && out.stride(1) == 1,
              "out must be a 2-D bf16 CUDA tensor with unit inner stride");
  const int rows = static_cast<int>(out.size(0)), cols = static_cast<int>(out.size(1));
  TORCH_CHECK(cols % 8 == 0 && (out.stride(0) % 8) == 0 && ld_src % 8 == 0 && ld_src >= cols,
              "tp_reduce works on 16-byte vectors: cols, strides multiples of 8");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == torch::kInt32, "err must be the int32 device error word");
  const c10::cuda::CUDAGuard guard(out.device());
  ReduceArgs a{};
  auto s = srcs.contiguous();
  a.nsrc = static_cast<int>(s.numel());
  for (int q = 0; q < a.nsrc; ++q) {
    a.src[q] = reinterpret_cast<const __nv_bfloat16*>(s.data_ptr<int64_t>()[q]);
    TORCH_CHECK(a.src[q] != nullptr && reinterpret_cast<uintptr_t>(a.src[q]) % 16 == 0, "16-byte aligned slots");
  }
  a.counter = reinterpret_cast<const unsigned long long*>(counter);
  a.expected = static_cast<unsigned long long>(expected);
  if (residual.has_value() && residual->defined()) {
    TORCH_CHECK(residual->scalar_type() == torch::kBFloat16 && residual->dim() == 2 && residual->size(0) == rows &&
                    residual->size(1) == cols && residual->stride(1) == 1 && residual->stride(0) % 8 == 0,
                "residual must match out");
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    a.ld_res = residual->stride(0);
  }
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ld_out = out.stride(0);
  a.ld_src = ld_src;
  a.rows = rows;
  a.cols = cols;
  a.err = err.data_ptr<int>();
  a.spin_limit = spin_limit > 0 ? spin_limit : 10 * kSpinLimitCycles;
  if (rows == 0) return;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, out.get_device());
  const long vecs = static_cast<long>(rows) * (cols / 8);
  // at most two waiting CTAs per SM: the peers' arrivals may come from a signal kernel on this
  // GPU's side stream, which needs room on an SM while these CTAs spin
  const int blocks = static_cast<int>(std::min<long>((vecs + kReduceThreads - 1) / kReduceThreads, kWaitCtasPerSm * sms));
  tp_reduce_kernel<<<std::max(blocks, 1), kReduceThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_CHECK(cudaGetLastError());
}

}  // namespace gb
