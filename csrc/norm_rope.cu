// Normalisation, rotary-embedding and small fused elementwise kernels.
// Reference counterparts (all ATen eager there), under src/graspo/backends/graspoflow/:
//   RMSNorm            models/common/layers_qwen3.py:338-351
//   QK-norm            models/common/layers_qwen3.py:193-204, 231-236
//   RoPE cache + apply tensor_utils.py:361-374, 403-449
//   SwiGLU             models/common/layers_qwen3.py:334
//   embedding          models/qwen3/model.py:262-269
//
// * add_rmsnorm      h' = h + delta (bf16 or fp32 delta; an fp32 delta is a
//                    split-K workspace and is zeroed after it is read), then
//                    y = rmsnorm(h') * w, optionally U = s * y A^T (the LoRA
//                    "down" projection, CUDA cores, for decode-sized batches).
// * rmsnorm_bwd      dx = rstd * (g - xhat * mean(g * xhat)), g = dy * w
//                    (norm weights are frozen: no weight gradient).
// * qk_norm_rope     per-head RMSNorm of q and k, rotate-half RoPE, and the
//                    scatter of q / k / v to their destinations (contiguous
//                    tensors, or the paged KV cache through a block table).
// * qk_norm_rope_bwd the inverse rotation followed by the per-head norm backward.
// * swiglu_bwd       from interleaved (g, u) pre-activations and dh.
// * lora_down        U = s * x A^T on CUDA cores (decode-sized M).
// * embedding        row gather.
//
// Numerics: fp32 math, one rounding to bf16 per stored value.  Rotary
// frequencies come from a host-computed fp32 table so they match the
// PyTorch formulation bit for bit.

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "sm100_common.cuh"

namespace gb {

namespace {

constexpr int kNormThreads = 256;
constexpr int kStageBytes = 64 * 1024;   // one slot of the LoRA weight-row ring
constexpr int kMaxLoraRows = 128;        // LoRA-down outputs per row (2 r for gate/up, r <= 64)

template <int VEC>
struct BF16Vec {
  __nv_bfloat16 v[VEC];
};

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (warp == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

// One CTA per row; H <= 8 * 256 * 8 (each thread holds up to 8 chunks of 8).
// Tensor-parallel sum of an fp32 delta whose peer partials were pushed into
// this rank's receive slots by the producing GEMM (see GemmArgs::push_dst).
struct PeerSum {
  const float* src[8];  // per rank: receive slot, or nullptr for this rank (the local delta)
  int n;                // ranks (<= 1: the local delta alone)
  int* arrivals;        // grows by the pushed element count; this kernel takes `expected` back off
  int* done;            // CTAs finished (the last resets it)
  int expected;
  int* err;
};

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait (about 10 s) for the peers' pushes of this step.
__device__ __forceinline__ void peer_wait(const PeerSum& ps) {
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    while (ld_acquire_sys(ps.arrivals) < ps.expected) {
      if (clock64() - t0 > 10 * kSpinLimitCycles) {
        record_error(ps.err, kErrPeerTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void peer_release(const PeerSum& ps) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(ps.done, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      *ps.done = 0;
      atomicSub_system(ps.arrivals, ps.expected);
    }
  }
}

// Row `row` of the tensor-parallel sum at columns [col, col + 8): partials
// added in rank order, so every rank gets the same bits.
__device__ __forceinline__ void peer_sum8(const PeerSum& ps, const float* local, long off, float (&d)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) d[e] = 0.f;
  for (int q = 0; q < ps.n; ++q) {
    const float* src = ps.src[q] != nullptr ? ps.src[q] + off : local + off;
    const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(src + 4));
    d[0] += a.x; d[1] += a.y; d[2] += a.z; d[3] += a.w;
    d[4] += b.x; d[5] += b.y; d[6] += b.z; d[7] += b.w;
  }
}

template <bool DELTA_F32, bool HAS_DELTA, bool LORA>
__global__ void add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ h, const void* delta,
                                   __nv_bfloat16* __restrict__ h_out,
                                   const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out,
                                   const __nv_bfloat16* __restrict__ lora_a,
                                   __nv_bfloat16* __restrict__ lora_u, int H, int R, int ldu,
                                   float scale, float eps, long ldd,
                                   const __nv_bfloat16* __restrict__ dlb, int ldb, int dlr, PeerSum ps,
                                   float* __restrict__ zero_tail, long zero_ld, int zero_n) {
  constexpr int MAXC = 4;  // chunks of 8 per thread: H <= 256*8*4 = 8192
  __shared__ float red[32];
  __shared__ float ured[8][kMaxLoraRows];
  __shared__ float dus[64];
  __shared__ uint64_t stage_bar[2];
  extern __shared__ __align__(16) uint8_t stage_smem[];   // 2 x kStageBytes when LoRA rows are staged
  const long row = blockIdx.x;
  const __nv_bfloat16* hr = h + row * H;
  // LoRA weight rows (B^T of the delta's LoRA, then A of this norm's LoRA-down)
  // stream through a two-slot shared-memory ring as 1-D bulk copies of whole
  // rows: every thread then reads its columns from shared memory instead of
  // waiting on one global load per rank row.
  const int pass_rows = kStageBytes / (H * 2);
  const int b_rows = (HAS_DELTA && DELTA_F32 && dlb != nullptr) ? dlr : 0;
  const int a_rows = LORA ? R : 0;
  const int b_passes = (b_rows + pass_rows - 1) / pass_rows;
  const int n_passes = b_passes + (a_rows + pass_rows - 1) / pass_rows;
  auto pass_src = [&](int k, int& r0, int& nr) -> const __nv_bfloat16* {
    if (k < b_passes) {
      r0 = k * pass_rows;
      nr = min(pass_rows, b_rows - r0);
      return dlb + static_cast<long>(r0) * H;
    }
    r0 = (k - b_passes) * pass_rows;
    nr = min(pass_rows, a_rows - r0);
    return lora_a + static_cast<long>(r0) * H;
  };
  auto issue = [&](int k) {
    if (threadIdx.x == 0 && k < n_passes) {
      int r0, nr;
      const __nv_bfloat16* src = pass_src(k, r0, nr);
      const uint32_t bytes = static_cast<uint32_t>(nr) * H * 2;
      mbar_arrive_expect_tx(&stage_bar[k & 1], bytes);
      bulk_copy_g2s(stage_smem + (k & 1) * kStageBytes, src, bytes, &stage_bar[k & 1]);
    }
  };
  if (n_passes > 0) {
    if (threadIdx.x == 0) {
      mbar_init(&stage_bar[0], 1);
      mbar_init(&stage_bar[1], 1);
      fence_mbar_init();
    }
    __syncthreads();
    issue(0);  // frozen weights: fetched before waiting on the producing kernel
    issue(1);
  }
  pdl_trigger();
  pdl_wait();
  const bool peers = HAS_DELTA && DELTA_F32 && ps.n > 1;
  if (peers) peer_wait(ps);
  if constexpr (HAS_DELTA && DELTA_F32) {
    // U = s * A x of the producing GEMM sits after the H delta columns; take it
    // and zero it (the workspace is accumulated by atomics on the next step)
    if (dlb != nullptr) {
      float* ur = static_cast<float*>(const_cast<void*>(delta)) + row * ldd + H;
      if (threadIdx.x < dlr) {
        float u = 0.f;
        if (peers) {
          for (int q = 0; q < ps.n; ++q)
            u += __ldcg((ps.src[q] != nullptr ? ps.src[q] + row * ldd + H : ur) + threadIdx.x);
        } else {
          u = ur[threadIdx.x];
        }
        dus[threadIdx.x] = u;
      }
      __syncthreads();
      // the whole U region (padding columns included) starts the next step at zero
      for (long j = threadIdx.x; j < ldd - H; j += blockDim.x) ur[j] = 0.f;
    }
  }
  float x[MAXC][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int col = (threadIdx.x + c * kNormThreads) * 8;
    if (col < H) {
      uint4 raw = *reinterpret_cast<const uint4*>(hr + col);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[c][e] = __bfloat162float(b[e]);
      if constexpr (HAS_DELTA) {
        if constexpr (DELTA_F32) {
          float* d = static_cast<float*>(const_cast<void*>(delta)) + row * ldd + col;
          if (peers) {
            float ds[8];
            peer_sum8(ps, static_cast<const float*>(delta), row * ldd + col, ds);
#pragma unroll
            for (int e = 0; e < 8; ++e) x[c][e] += ds[e];
          } else {
            float4 d0 = *reinterpret_cast<float4*>(d);
            float4 d1 = *reinterpret_cast<float4*>(d + 4);
            x[c][0] += d0.x; x[c][1] += d0.y; x[c][2] += d0.z; x[c][3] += d0.w;
            x[c][4] += d1.x; x[c][5] += d1.y; x[c][6] += d1.z; x[c][7] += d1.w;
          }
          *reinterpret_cast<float4*>(d) = make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(d + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
          const __nv_bfloat16* d = static_cast<const __nv_bfloat16*>(delta) + row * ldd + col;
          uint4 draw = *reinterpret_cast<const uint4*>(d);
          const __nv_bfloat16* db = reinterpret_cast<const __nv_bfloat16*>(&draw);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[c][e] += __bfloat162float(db[e]);
        }
      }
    }
  }
  // B^T [r, H] rows (rank row j holds every column): x += B U, in rank order
  bool staged_ok = true;
  for (int k = 0; k < b_passes; ++k) {
    int r0, nr;
    pass_src(k, r0, nr);
    staged_ok = staged_ok && mbar_wait(&stage_bar[k & 1], (k >> 1) & 1, ps.err, kErrTmaFullTimeout);
    const uint8_t* st = stage_smem + (k & 1) * kStageBytes;
    for (int jj = 0; jj < nr && staged_ok; ++jj) {
      const float u = dus[r0 + jj];
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
        const int col = (threadIdx.x + c * kNormThreads) * 8;
        if (col < H) {
          const uint4 raw = *reinterpret_cast<const uint4*>(st + (static_cast<long>(jj) * H + col) * 2);
          const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[c][e] += __bfloat162float(bb[e]) * u;
        }
      }
    }
    __syncthreads();  // slot k & 1 is free again
    if (staged_ok) issue(k + 2);
  }
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int col = (threadIdx.x + c * kNormThreads) * 8;
    if (col < H) {
      if constexpr (HAS_DELTA) {
        // the residual stream is stored in bf16: round the sum once
        uint4 out;
        __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ob[e] = __float2bfloat16(x[c][e]);
          x[c][e] = __bfloat162float(ob[e]);
        }
        *reinterpret_cast<uint4*>(h_out + row * H + col) = out;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += x[c][e] * x[c][e];
    }
  }
  const float total = block_sum(ss, red);
  const float rstd = rsqrtf(total / static_cast<float>(H) + eps);
  if (rstd_out != nullptr && threadIdx.x == 0) rstd_out[row] = rstd;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int col = (threadIdx.x + c * kNormThreads) * 8;
    if (col < H) {
      uint4 wraw = *reinterpret_cast<const uint4*>(w + col);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wraw);
      uint4 out;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ob[e] = __float2bfloat16(x[c][e] * rstd * __bfloat162float(wb[e]));
        x[c][e] = __bfloat162float(ob[e]);
      }
      *reinterpret_cast<uint4*>(y + row * H + col) = out;
    }
  }
  if constexpr (LORA) {
    // U[row, j] = scale * sum_k y[k] * A[j, k]   for j < R; zero for R <= j < ldu
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int k = b_passes; k < n_passes; ++k) {
      int r0, nr;
      pass_src(k, r0, nr);
      staged_ok = staged_ok && mbar_wait(&stage_bar[k & 1], (k >> 1) & 1, ps.err, kErrTmaFullTimeout);
      const uint8_t* st = stage_smem + (k & 1) * kStageBytes;
      for (int jj = 0; jj < nr && staged_ok; ++jj) {
        float p = 0.f;
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
          const int col = (threadIdx.x + c * kNormThreads) * 8;
          if (col < H) {
            const uint4 raw = *reinterpret_cast<const uint4*>(st + (static_cast<long>(jj) * H + col) * 2);
            const __nv_bfloat16* ab = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
            for (int e = 0; e < 8; ++e) p += x[c][e] * __bfloat162float(ab[e]);
          }
        }
        p = warp_sum(p);
        if (lane == 0) ured[warp][r0 + jj] = p;
      }
      __syncthreads();  // slot k & 1 is free again; ured rows of this pass are complete
      if (staged_ok) issue(k + 2);
    }
    for (int j = threadIdx.x; j < R; j += blockDim.x) {
      float s = 0.f;
      for (int wi = 0; wi < kNormThreads / 32; ++wi) s += ured[wi][j];
      lora_u[row * ldu + j] = __float2bfloat16(staged_ok ? s * scale : 0.f);
    }
    for (int j = R + threadIdx.x; j < ldu; j += blockDim.x) lora_u[row * ldu + j] = __float2bfloat16(0.f);
  }
  // another kernel's per-row fp32 columns to clear for the next step (the LoRA
  // U of the q/k/v projection, read by qk_norm_rope earlier in this step)
  if (zero_tail != nullptr)
    for (int j = threadIdx.x; j < zero_n; j += blockDim.x) zero_tail[row * zero_ld + j] = 0.f;
  if (peers) peer_release(ps);
}

__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                   const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ w,
                                   const float* __restrict__ rstd_in,
                                   const __nv_bfloat16* __restrict__ dres,
                                   __nv_bfloat16* __restrict__ dx, int H, float eps) {
  constexpr int MAXC = 4;
  __shared__ float red[32];
  const long row = blockIdx.x;
  float xv[MAXC][8], gv[MAXC][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int col = (threadIdx.x + c * kNormThreads) * 8;
    if (col < H) {
      uint4 xr = *reinterpret_cast<const uint4*>(x + row * H + col);
      uint4 dr = *reinterpret_cast<const uint4*>(dy + row * H + col);
      uint4 wr = *reinterpret_cast<const uint4*>(w + col);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xr);
      const __nv_bfloat16* db = reinterpret_cast<const __nv_bfloat16*>(&dr);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wr);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        xv[c][e] = __bfloat162float(xb[e]);
        gv[c][e] = __bfloat162float(db[e]) * __bfloat162float(wb[e]);
        ss += xv[c][e] * xv[c][e];
      }
    }
  }
  float rstd;
  if (rstd_in != nullptr) {
    rstd = rstd_in[row];
  } else {
    rstd = rsqrtf(block_sum(ss, red) / static_cast<float>(H) + eps);
  }
  float dot = 0.f;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int col = (threadIdx.x + c * kNormThreads) * 8;
    if (col < H) {
#pragma unroll
      for (int e = 0; e < 8; ++e) dot += gv[c][e] * xv[c][e] * rstd;
    }
  }
  const float mean_gx = block_sum(dot, red) / static_cast<float>(H);
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int col = (threadIdx.x + c * kNormThreads) * 8;
    if (col < H) {
      float add[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (dres != nullptr) {
        uint4 rr = *reinterpret_cast<const uint4*>(dres + row * H + col);
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rr);
#pragma unroll
        for (int e = 0; e < 8; ++e) add[e] = __bfloat162float(rb[e]);
      }
      uint4 out;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xhat = xv[c][e] * rstd;
        ob[e] = __float2bfloat16(rstd * (gv[c][e] - xhat * mean_gx) + add[e]);
      }
      *reinterpret_cast<uint4*>(dx + row * H + col) = out;
    }
  }
}

// ------------------------------------------------------------------- rope
// One warp per (token, head).  head_dim == 128: lane owns elements
// [4*lane, 4*lane+4); the rotate-half partner lives 16 lanes away.
struct RopeArgs {
  const void* qkv;          // [T, (nq + 2 nkv) * D], bf16 or fp32 (split-K workspace)
  long ld_qkv;
  int qkv_f32;              // 1 if qkv is fp32 (then zeroed after reading)
  const __nv_bfloat16* q_w; // [D]
  const __nv_bfloat16* k_w; // [D]
  const float* inv_freq;    // [D/2]
  const int64_t* pos;       // [T]
  __nv_bfloat16* q_out;     // [T, nq, D]
  __nv_bfloat16* k_out;     // contiguous [T, nkv, D] (if block_table == nullptr)
  __nv_bfloat16* v_out;
  // paged cache: pool [num_pages, nkv, page, D]
  const int* block_table;   // [rows, max_pages]
  int max_pages;
  int page_size;
  int num_pages;            // pool pages (kernel-checks builds validate block-table entries)
  int* err;
  const int64_t* row_of_token;  // token -> cache row (paged)
  const int64_t* slot;          // token -> cache slot (paged); the rope position differs
                                // from the slot when the row is left-padded
  int T, nq, nkv;
  float eps;
  // LoRA on q/k/v computed by the projection GEMM itself: the fp32 workspace
  // row holds, after the (nq + 2 nkv) * D projection columns, U = s * A x in
  // u_width columns (q, k, v blocks of lora_r each); this kernel adds B U
  // (lora_b = B^T [3 r, (nq + 2 nkv) * D] of the block-diagonal q/k/v B).
  const __nv_bfloat16* lora_b;
  int ldb, lora_r, u_width;
};

// One warp per (token, head).  The LoRA U columns are only read here; the
// residual-add + RMSNorm kernel after the attention zeroes them for the next
// step (see add_rmsnorm's zero_tail).
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(RopeArgs a) {
  constexpr int D = 128;
  const int lane = threadIdx.x & 31;
  const int heads = a.nq + 2 * a.nkv;
  const long wg = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  pdl_trigger();
  pdl_wait();
  if (wg >= static_cast<long>(a.T) * heads) return;
  const int t = static_cast<int>(wg / heads);
  const bool lora = a.qkv_f32 && a.lora_b != nullptr;
  const float* us = lora ? static_cast<const float*>(a.qkv) + static_cast<long>(t) * a.ld_qkv +
                               static_cast<long>(heads) * D
                         : nullptr;
  {
  const int hd = static_cast<int>(wg - static_cast<long>(t) * heads);
  float x[4];
  const long base = static_cast<long>(t) * a.ld_qkv + static_cast<long>(hd) * D + lane * 4;
  if (a.qkv_f32) {
    float* src = static_cast<float*>(const_cast<void*>(a.qkv)) + base;
    float4 f = *reinterpret_cast<float4*>(src);
    x[0] = f.x; x[1] = f.y; x[2] = f.z; x[3] = f.w;
    *reinterpret_cast<float4*>(src) = make_float4(0.f, 0.f, 0.f, 0.f);
    // round like a bf16 GEMM output would be
    if (lora) {
      const int blk = hd < a.nq ? 0 : (hd < a.nq + a.nkv ? 1 : 2);
      const float* u = us + blk * a.lora_r;  // L1/L2-served broadcast reads
      // B^T [3r, W]: rank row (blk r + j) holds this lane's 4 columns contiguously
      for (int j = 0; j < a.lora_r; ++j) {
        const uint2 raw = __ldg(reinterpret_cast<const uint2*>(
            a.lora_b + static_cast<long>(blk * a.lora_r + j) * a.ldb + hd * D + lane * 4));
        const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&raw);
        const float uj = u[j];
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] += __bfloat162float(bb[e]) * uj;
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = __bfloat162float(__float2bfloat16(x[e]));
  } else {
    const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(a.qkv) + base;
    uint2 raw = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = __bfloat162float(b[e]);
  }
  const bool is_q = hd < a.nq;
  const bool is_k = !is_q && hd < a.nq + a.nkv;
  __nv_bfloat16* dst;
  if (is_q) {
    dst = a.q_out + (static_cast<long>(t) * a.nq + hd) * D;
  } else {
    const int kvh = is_k ? hd - a.nq : hd - a.nq - a.nkv;
    __nv_bfloat16* pool = is_k ? a.k_out : a.v_out;
    if (a.block_table != nullptr) {
      const long row = a.row_of_token[t];
      const long p = a.slot[t];
      const int page = checked_index(a.block_table[row * a.max_pages + p / a.page_size], a.num_pages, a.err);
      const int off = static_cast<int>(p % a.page_size);
      dst = pool + ((static_cast<long>(page) * a.nkv + kvh) * a.page_size + off) * D;
    } else {
      dst = pool + (static_cast<long>(t) * a.nkv + kvh) * D;
    }
  }
  if (is_q || is_k) {
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss / D + a.eps);
    const __nv_bfloat16* wn = is_q ? a.q_w : a.k_w;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      x[e] = __bfloat162float(__float2bfloat16(x[e] * rstd * __bfloat162float(wn[lane * 4 + e])));
    const float p = static_cast<float>(a.pos[t]);
    float partner[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const bool first_half = lane < 16;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = (lane & 15) * 4 + e;  // frequency index
      float s, c;
      sincosf(p * a.inv_freq[i], &s, &c);
      // first half: x*cos - x[i+D/2]*sin ; second half: x*cos + x[i-D/2]*sin
      x[e] = first_half ? (x[e] * c - partner[e] * s) : (x[e] * c + partner[e] * s);
    }
  }
  uint2 out;
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
  for (int e = 0; e < 4; ++e) ob[e] = __float2bfloat16(x[e]);
  *reinterpret_cast<uint2*>(dst + lane * 4) = out;
  }
}

// Backward: inputs dq [T,nq,D], dk/dv [T,nkv,D], the pre-norm qkv [T, ...] (bf16);
// output d(qkv) [T, (nq+2nkv)*D] bf16.
__global__ void qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dq,
                                        const __nv_bfloat16* __restrict__ dk,
                                        const __nv_bfloat16* __restrict__ dv,
                                        const __nv_bfloat16* __restrict__ qkv, long ld_qkv,
                                        const __nv_bfloat16* __restrict__ q_w,
                                        const __nv_bfloat16* __restrict__ k_w,
                                        const float* __restrict__ inv_freq,
                                        const int64_t* __restrict__ pos,
                                        __nv_bfloat16* __restrict__ dqkv, int T, int nq, int nkv,
                                        float eps) {
  constexpr int D = 128;
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = nq + 2 * nkv;
  if (warp_global >= T * heads) return;
  const int t = warp_global / heads;
  const int hd = warp_global - t * heads;
  const bool is_q = hd < nq;
  const bool is_k = !is_q && hd < nq + nkv;
  const __nv_bfloat16* g_src =
      is_q ? dq + (static_cast<long>(t) * nq + hd) * D
           : (is_k ? dk + (static_cast<long>(t) * nkv + (hd - nq)) * D
                   : dv + (static_cast<long>(t) * nkv + (hd - nq - nkv)) * D);
  float g[4];
  {
    uint2 raw = *reinterpret_cast<const uint2*>(g_src + lane * 4);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) g[e] = __bfloat162float(b[e]);
  }
  if (is_q || is_k) {
    // inverse rotation (transpose of the forward rotation)
    const float p = static_cast<float>(pos[t]);
    float partner[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, g[e], 16);
    const bool first_half = lane < 16;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = (lane & 15) * 4 + e;
      float s, c;
      sincosf(p * inv_freq[i], &s, &c);
      g[e] = first_half ? (g[e] * c + partner[e] * s) : (g[e] * c - partner[e] * s);
    }
    // per-head rmsnorm backward
    const __nv_bfloat16* xs = qkv + static_cast<long>(t) * ld_qkv + static_cast<long>(hd) * D + lane * 4;
    uint2 raw = *reinterpret_cast<const uint2*>(xs);
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&raw);
    float x[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = __bfloat162float(xb[e]);
    const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
    const float rstd = rsqrtf(ss / D + eps);
    const __nv_bfloat16* wn = is_q ? q_w : k_w;
    float gw[4];
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      gw[e] = g[e] * __bfloat162float(wn[lane * 4 + e]);
      dot += gw[e] * x[e] * rstd;
    }
    const float mean = warp_sum(dot) / D;
#pragma unroll
    for (int e = 0; e < 4; ++e) g[e] = rstd * (gw[e] - x[e] * rstd * mean);
  }
  uint2 out;
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
  for (int e = 0; e < 4; ++e) ob[e] = __float2bfloat16(g[e]);
  *reinterpret_cast<uint2*>(dqkv + static_cast<long>(t) * heads * D + static_cast<long>(hd) * D + lane * 4) = out;
}

// d(gate, up) interleaved from dh and the stored interleaved (g, u).
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                  const __nv_bfloat16* __restrict__ dh,
                                  __nv_bfloat16* __restrict__ dgu, long n_pairs) {
  const long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x;
  if (i >= n_pairs) return;
  const __nv_bfloat162 p = reinterpret_cast<const __nv_bfloat162*>(gu)[i];
  const float g = __bfloat162float(p.x), u = __bfloat162float(p.y);
  const float d = __bfloat162float(dh[i]);
  const float sig = 1.f / (1.f + __expf(-g));
  const float silu = g * sig;
  const float dg = d * u * sig * (1.f + g * (1.f - sig));
  const float du = d * silu;
  reinterpret_cast<__nv_bfloat162*>(dgu)[i] = __floats2bfloat162_rn(dg, du);
}

// U[row, j] = scale * x[row, :] . A[j, :]  for j < R (zero-padded to ldu).
// One CTA per row; the first 16384 columns of x are held in registers.
__global__ void __launch_bounds__(256) lora_down_kernel(const __nv_bfloat16* __restrict__ x, long ldx,
                                                         const __nv_bfloat16* __restrict__ A,
                                                         __nv_bfloat16* __restrict__ U, int K, int R, int ldu,
                                                         float scale) {
  constexpr int MAXC = 8;  // chunks of 8 per thread: K <= 256 * 8 * 8
  __shared__ float part[8][64];
  const long row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float xv[MAXC][8];
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int col = (threadIdx.x + c * 256) * 8;
    if (col < K) {
      uint4 xr = *reinterpret_cast<const uint4*>(x + row * ldx + col);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xr);
#pragma unroll
      for (int e = 0; e < 8; ++e) xv[c][e] = __bfloat162float(xb[e]);
    }
  }
  for (int j0 = 0; j0 < R; j0 += 64) {
    const int jn = min(64, R - j0);
    for (int j = 0; j < jn; j += 4) {
      float p[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        p[jj] = 0.f;
        if (j + jj < jn) {
          const __nv_bfloat16* arow = A + static_cast<long>(j0 + j + jj) * K;
#pragma unroll
          for (int c = 0; c < MAXC; ++c) {
            const int col = (threadIdx.x + c * 256) * 8;
            if (col < K) {
              uint4 ar = __ldg(reinterpret_cast<const uint4*>(arow + col));
              const __nv_bfloat16* ab = reinterpret_cast<const __nv_bfloat16*>(&ar);
#pragma unroll
              for (int e = 0; e < 8; ++e) p[jj] += xv[c][e] * __bfloat162float(ab[e]);
            }
          }
          // columns beyond the register-held prefix (K > 16384)
          for (int col = (threadIdx.x + MAXC * 256) * 8; col < K; col += 256 * 8) {
            uint4 xr = *reinterpret_cast<const uint4*>(x + row * ldx + col);
            uint4 ar = __ldg(reinterpret_cast<const uint4*>(arow + col));
            const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xr);
            const __nv_bfloat16* ab = reinterpret_cast<const __nv_bfloat16*>(&ar);
#pragma unroll
            for (int e = 0; e < 8; ++e) p[jj] += __bfloat162float(xb[e]) * __bfloat162float(ab[e]);
          }
        }
      }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const float v = warp_sum(p[jj]);
        if (lane == 0 && j + jj < jn) part[warp][j + jj] = v;
      }
    }
    __syncthreads();
    if (threadIdx.x < jn) {
      float s = 0.f;
      for (int wi = 0; wi < 8; ++wi) s += part[wi][threadIdx.x];
      U[row * ldu + j0 + threadIdx.x] = __float2bfloat16(s * scale);
    }
    __syncthreads();
  }
  for (int j = R + threadIdx.x; j < ldu; j += blockDim.x) U[row * ldu + j] = __float2bfloat16(0.f);
}

__global__ void embedding_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int H, long vocab) {
  const long row = blockIdx.x;
  pdl_trigger();
  pdl_wait();
  long id = ids[row];
  if (id < 0 || id >= vocab) id = 0;
  const uint4* src = reinterpret_cast<const uint4*>(table + id * H);
  uint4* dst = reinterpret_cast<uint4*>(out + row * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

}  // namespace

// ===================================================================== host
static void check_bf16(const torch::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.is_contiguous(), n,
              " must be a contiguous CUDA bf16 tensor");
}

void add_rmsnorm(torch::Tensor h, c10::optional<torch::Tensor> delta,
                 c10::optional<torch::Tensor> h_out, torch::Tensor w, torch::Tensor y,
                 c10::optional<torch::Tensor> rstd, c10::optional<torch::Tensor> lora_a,
                 c10::optional<torch::Tensor> lora_u, double scale, double eps,
                 c10::optional<torch::Tensor> delta_lora_b, int64_t delta_lora_r,
                 c10::optional<torch::Tensor> peer_src, c10::optional<torch::Tensor> peer_sync,
                 int64_t peer_expected, c10::optional<torch::Tensor> err,
                 c10::optional<torch::Tensor> zero_tail) {
  check_bf16(h, "h");
  check_bf16(y, "y");
  const c10::cuda::CUDAGuard guard(h.device());
  const int H = static_cast<int>(h.size(-1));
  const long rows = h.numel() / H;
  TORCH_CHECK(H % 8 == 0 && H <= 8192, "hidden size must be a multiple of 8 and <= 8192");
  const bool has_delta = delta.has_value() && delta->defined();
  const bool delta_f32 = has_delta && delta->scalar_type() == torch::kFloat32;
  const bool lora = lora_a.has_value() && lora_a->defined();
  auto stream = at::cuda::getCurrentCUDAStream();
  const void* dptr = has_delta ? delta->data_ptr() : nullptr;
  __nv_bfloat16* hout = (h_out.has_value() && h_out->defined())
                            ? reinterpret_cast<__nv_bfloat16*>(h_out->data_ptr())
                            : nullptr;
  TORCH_CHECK(!has_delta || hout != nullptr, "delta requires h_out");
  float* rp = (rstd.has_value() && rstd->defined()) ? rstd->data_ptr<float>() : nullptr;
  const __nv_bfloat16* ap = lora ? reinterpret_cast<const __nv_bfloat16*>(lora_a->data_ptr()) : nullptr;
  __nv_bfloat16* up = lora ? reinterpret_cast<__nv_bfloat16*>(lora_u->data_ptr()) : nullptr;
  const int R = lora ? static_cast<int>(lora_a->size(0)) : 0;
  const int ldu = lora ? static_cast<int>(lora_u->size(-1)) : 0;
  auto hp = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr());
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  long ldd = H;
  if (has_delta) {
    TORCH_CHECK(delta->stride(-1) == 1 && delta->numel() / delta->size(-1) == rows && delta->size(-1) >= H,
                "delta must be row-major [rows, >= H]");
    ldd = delta->stride(0);
  }
  const __nv_bfloat16* dlb = nullptr;
  int ldb = 0, dlr = 0;
  if (delta_lora_b.has_value() && delta_lora_b->defined()) {
    TORCH_CHECK(delta_f32, "the LoRA B.U term needs an fp32 delta workspace");
    check_bf16(*delta_lora_b, "delta_lora_b");
    dlb = reinterpret_cast<const __nv_bfloat16*>(delta_lora_b->data_ptr());
    ldb = static_cast<int>(delta_lora_b->size(1));
    dlr = static_cast<int>(delta_lora_r);
    TORCH_CHECK(delta_lora_b->size(1) == H && delta_lora_b->size(0) >= dlr && dlr <= 64 && ldb % 8 == 0 &&
                    delta->size(-1) >= H + dlr,
                "delta LoRA: B^T must be [>= r, H] with r <= 64, U after the H delta columns");
  }
  PeerSum ps{};
  if (peer_src.has_value() && peer_src->defined()) {
    TORCH_CHECK(delta_f32, "the tensor-parallel sum needs an fp32 delta workspace");
    TORCH_CHECK(peer_src->device().is_cpu() && peer_src->scalar_type() == torch::kInt64 && peer_src->numel() <= 8,
                "peer_src must be a CPU int64 address table (<= 8 ranks)");
    TORCH_CHECK(peer_sync.has_value() && peer_sync->device().is_cpu() && peer_sync->numel() == 2,
                "peer_sync must hold the arrival and done counter addresses");
    auto src = peer_src->contiguous();
    auto sy = peer_sync->contiguous();
    ps.n = static_cast<int>(src.numel());
    for (int q = 0; q < ps.n; ++q) ps.src[q] = reinterpret_cast<const float*>(src.data_ptr<int64_t>()[q]);
    ps.arrivals = reinterpret_cast<int*>(sy.data_ptr<int64_t>()[0]);
    ps.done = reinterpret_cast<int*>(sy.data_ptr<int64_t>()[1]);
    ps.expected = static_cast<int>(peer_expected);
    TORCH_CHECK(ldd % 4 == 0, "peer sum needs 16-byte aligned rows");
  }
  // error word for the bounded waits (peer sums, staged LoRA rows)
  ps.err = (err.has_value() && err->defined()) ? err->data_ptr<int>() : nullptr;
  float* zt = nullptr;
  long zld = 0;
  int zn = 0;
  if (zero_tail.has_value() && zero_tail->defined()) {
    TORCH_CHECK(zero_tail->scalar_type() == torch::kFloat32 && zero_tail->dim() == 2 && zero_tail->stride(1) == 1 &&
                    zero_tail->size(0) == rows,
                "zero_tail must be an fp32 [rows, n] view with unit inner stride");
    zt = zero_tail->data_ptr<float>();
    zld = zero_tail->stride(0);
    zn = static_cast<int>(zero_tail->size(1));
  }
  const bool staged = dlb != nullptr || lora;
  TORCH_CHECK(R <= kMaxLoraRows && (!lora || ldu >= R), "LoRA-down: at most 128 rows, U at least that wide");
  const int dyn_smem = staged ? 2 * kStageBytes : 0;
  if (staged) {
    TORCH_CHECK(reinterpret_cast<uintptr_t>(dlb) % 16 == 0 && reinterpret_cast<uintptr_t>(ap) % 16 == 0,
                "LoRA weight rows must be 16-byte aligned");
    TORCH_CHECK(dlb == nullptr || ldb == H, "B^T rows must be contiguous [r, H]");
    TORCH_CHECK(!lora || (lora_a->stride(0) == H && lora_a->stride(1) == 1), "LoRA A rows must be contiguous [R, H]");
  }
#define GB_LAUNCH_NORM(DF, HD, LR)                                                                           \
  do {                                                                                                       \
    static bool configured[64] = {};                                                                         \
    const int dev = h.get_device();                                                                          \
    if (!configured[dev]) {                                                                                  \
      C10_CUDA_CHECK(cudaFuncSetAttribute(add_rmsnorm_kernel<DF, HD, LR>,                                    \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * kStageBytes));   \
      configured[dev] = true;                                                                                \
    }                                                                                                        \
    C10_CUDA_CHECK(launch_kernel(add_rmsnorm_kernel<DF, HD, LR>, dim3(rows), dim3(kNormThreads), dyn_smem,  \
                                 stream, hp, dptr, hout, wp, yp, rp, ap, up, H, R, ldu, (float)scale,        \
                                 (float)eps, ldd, dlb, ldb, dlr, ps, zt, zld, zn));                          \
  } while (0)
  if (!has_delta) {
    if (lora) GB_LAUNCH_NORM(false, false, true); else GB_LAUNCH_NORM(false, false, false);
  } else if (delta_f32) {
    if (lora) GB_LAUNCH_NORM(true, true, true); else GB_LAUNCH_NORM(true, true, false);
  } else {
    if (lora) GB_LAUNCH_NORM(false, true, true); else GB_LAUNCH_NORM(false, true, false);
  }
#undef GB_LAUNCH_NORM
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> rstd,
                 c10::optional<torch::Tensor> dres, torch::Tensor dx, double eps) {
  check_bf16(dy, "dy");
  check_bf16(x, "x");
  check_bf16(dx, "dx");
  const c10::cuda::CUDAGuard guard(x.device());
  const int H = static_cast<int>(x.size(-1));
  const long rows = x.numel() / H;
  TORCH_CHECK(H % 8 == 0 && H <= 8192, "hidden size must be a multiple of 8 and <= 8192");
  rmsnorm_bwd_kernel<<<rows, kNormThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      (rstd.has_value() && rstd->defined()) ? rstd->data_ptr<float>() : nullptr,
      (dres.has_value() && dres->defined()) ? reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr()) : nullptr,
      reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), H, static_cast<float>(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qk_norm_rope(torch::Tensor qkv, torch::Tensor q_w, torch::Tensor k_w, torch::Tensor inv_freq,
                  torch::Tensor pos, torch::Tensor q_out, torch::Tensor k_out, torch::Tensor v_out,
                  c10::optional<torch::Tensor> block_table, c10::optional<torch::Tensor> row_of_token,
                  c10::optional<torch::Tensor> slot, int64_t nq, int64_t nkv, int64_t page_size, double eps,
                  c10::optional<torch::Tensor> lora_b, int64_t lora_r, c10::optional<torch::Tensor> err) {
  const c10::cuda::CUDAGuard guard(qkv.device());
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1, "qkv must be 2-D row-major");
  RopeArgs a{};
  a.err = (err.has_value() && err->defined()) ? err->data_ptr<int>() : nullptr;
  a.num_pages = static_cast<int>(k_out.size(0));
  a.qkv = qkv.data_ptr();
  a.ld_qkv = qkv.stride(0);
  a.qkv_f32 = qkv.scalar_type() == torch::kFloat32 ? 1 : 0;
  a.q_w = reinterpret_cast<const __nv_bfloat16*>(q_w.data_ptr());
  a.k_w = reinterpret_cast<const __nv_bfloat16*>(k_w.data_ptr());
  a.inv_freq = inv_freq.data_ptr<float>();
  a.pos = pos.data_ptr<int64_t>();
  a.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  a.k_out = reinterpret_cast<__nv_bfloat16*>(k_out.data_ptr());
  a.v_out = reinterpret_cast<__nv_bfloat16*>(v_out.data_ptr());
  if (block_table.has_value() && block_table->defined()) {
    a.block_table = block_table->data_ptr<int>();
    a.max_pages = static_cast<int>(block_table->size(1));
    TORCH_CHECK(row_of_token.has_value() && slot.has_value(), "paged KV write needs row_of_token and slot");
    a.row_of_token = row_of_token->data_ptr<int64_t>();
    a.slot = slot->data_ptr<int64_t>();
    a.page_size = static_cast<int>(page_size);
  }
  a.T = static_cast<int>(qkv.size(0));
  a.nq = static_cast<int>(nq);
  a.nkv = static_cast<int>(nkv);
  a.eps = static_cast<float>(eps);
  TORCH_CHECK(qkv.size(1) >= (nq + 2 * nkv) * 128, "qkv width / head_dim mismatch (head_dim must be 128)");
  if (lora_b.has_value() && lora_b->defined()) {
    TORCH_CHECK(a.qkv_f32, "the LoRA B.U term applies to the fp32 split-K workspace");
    check_bf16(*lora_b, "lora_b");
    a.lora_b = reinterpret_cast<const __nv_bfloat16*>(lora_b->data_ptr());
    a.ldb = static_cast<int>(lora_b->size(1));
    a.lora_r = static_cast<int>(lora_r);
    a.u_width = static_cast<int>(qkv.size(1) - (nq + 2 * nkv) * 128);
    TORCH_CHECK(3 * lora_r <= a.u_width && lora_r <= 64 && a.ldb % 4 == 0,
                "LoRA rank at most 64, with U columns after the projection");
    TORCH_CHECK(lora_b->size(1) == (nq + 2 * nkv) * 128 && lora_b->size(0) >= 3 * lora_r,
                "lora_b must be B^T [3r, projection width]");
  }
  const long warps = static_cast<long>(a.T) * (nq + 2 * nkv);
  if (warps > 0)
    C10_CUDA_CHECK(launch_kernel(qk_norm_rope_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0,
                                 at::cuda::getCurrentCUDAStream(), a));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qk_norm_rope_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv,
                      torch::Tensor q_w, torch::Tensor k_w, torch::Tensor inv_freq, torch::Tensor pos,
                      torch::Tensor dqkv, int64_t nq, int64_t nkv, double eps) {
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int T = static_cast<int>(qkv.size(0));
  const long warps = static_cast<long>(T) * (nq + 2 * nkv);
  const int threads = 256;
  const long blocks = (warps * 32 + threads - 1) / threads;
  if (blocks > 0)
    qk_norm_rope_bwd_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dq.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(dk.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(dv.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(q_w.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(k_w.data_ptr()), inv_freq.data_ptr<float>(),
        pos.data_ptr<int64_t>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), T,
        static_cast<int>(nq), static_cast<int>(nkv), static_cast<float>(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_bwd(torch::Tensor gu, torch::Tensor dh, torch::Tensor dgu) {
  check_bf16(gu, "gu");
  check_bf16(dh, "dh");
  check_bf16(dgu, "dgu");
  const c10::cuda::CUDAGuard guard(gu.device());
  const long n = dh.numel();
  if (n == 0) return;
  swiglu_bwd_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lora_down(torch::Tensor x, torch::Tensor A, torch::Tensor U, double scale) {
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be 2-D row-major");
  check_bf16(A, "A");
  check_bf16(U, "U");
  const c10::cuda::CUDAGuard guard(x.device());
  const int K = static_cast<int>(x.size(1));
  TORCH_CHECK(K % 8 == 0 && A.size(1) == K, "K mismatch");
  const long rows = x.size(0);
  if (rows == 0) return;
  lora_down_kernel<<<rows, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(A.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(U.data_ptr()), K, static_cast<int>(A.size(0)),
      static_cast<int>(U.size(1)), static_cast<float>(scale));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out) {
  check_bf16(table, "table");
  check_bf16(out, "out");
  const c10::cuda::CUDAGuard guard(table.device());
  const long rows = ids.numel();
  const int H = static_cast<int>(table.size(1));
  TORCH_CHECK(H % 8 == 0, "hidden must be a multiple of 8");
  if (rows == 0) return;
  C10_CUDA_CHECK(launch_kernel(embedding_kernel, dim3(rows), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
      ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), H, table.size(0)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


}  // namespace gb
