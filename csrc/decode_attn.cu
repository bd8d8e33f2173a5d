// Decode-step attention over the paged KV cache.
//
// Cache layout: k_pool / v_pool [num_pages, n_kv_heads, page_size, 128] bf16,
// block_table [rows, max_pages] maps a row's logical page to a physical page.
// Rows that share a prompt (the G completions of one GRASPO group) point at
// the same physical prompt pages, so the prompt KV is stored once per group.
// A row attends to key positions [start[row], len[row]) (left padding is
// skipped, the newest token at len-1 is included).
//
// One CTA per (row, kv_head) handles all G = nq / nkv query heads of that KV
// head (GQA packing: every K/V element is read once for the whole group).  Each
// of the 4 warps walks a quarter of every page; a lane owns 4 of the 128 head
// dims; per-warp online-softmax states are merged through shared memory at the
// end.  This kernel is bandwidth-bound: the figure of merit is KV bytes / time.

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "sm100_common.cuh"

namespace gb {

namespace {

constexpr int kD = 128;
constexpr int kMaxGroup = 8;

template <int G>
__global__ void __launch_bounds__(128) paged_decode_attn_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_pool,
    const __nv_bfloat16* __restrict__ v_pool, const int* __restrict__ block_table,
    const int* __restrict__ start, const int* __restrict__ len, __nv_bfloat16* __restrict__ out,
    int nq, int nkv, int page_size, int max_pages, float scale_log2) {
  const int row = blockIdx.x / nkv;
  const int kvh = blockIdx.x - row * nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s0 = start[row], s1 = len[row];

  float qv[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const __nv_bfloat16* qp = q + (static_cast<long>(row) * nq + kvh * G + g) * kD + lane * 4;
    uint2 raw = *reinterpret_cast<const uint2*>(qp);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) qv[g][e] = __bfloat162float(b[e]) * scale_log2;
  }
  float m[G], l[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
  }

  const int first_page = s0 / page_size;
  const int last_page = (s1 - 1) / page_size;
  const int per_warp = page_size / 4;
  for (int lp = first_page; lp <= last_page && s1 > s0; ++lp) {
    const int phys = block_table[static_cast<long>(row) * max_pages + lp];
    const long page_base = (static_cast<long>(phys) * nkv + kvh) * page_size;
    const int t_begin = lp * page_size + warp * per_warp;
#pragma unroll 2
    for (int i = 0; i < per_warp; ++i) {
      const int t = t_begin + i;
      if (t < s0 || t >= s1) continue;  // uniform across the warp
      const long off = (page_base + (t - lp * page_size)) * kD + lane * 4;
      uint2 kr = *reinterpret_cast<const uint2*>(k_pool + off);
      uint2 vr = *reinterpret_cast<const uint2*>(v_pool + off);
      const __nv_bfloat16* kb = reinterpret_cast<const __nv_bfloat16*>(&kr);
      const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(&vr);
      float kf[4], vf[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        kf[e] = __bfloat162float(kb[e]);
        vf[e] = __bfloat162float(vb[e]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float s = qv[g][0] * kf[0] + qv[g][1] * kf[1] + qv[g][2] * kf[2] + qv[g][3] * kf[3];
        s = warp_sum(s);
        const float mn = fmaxf(m[g], s);
        const float corr = exp2f(m[g] - mn);
        const float p = exp2f(s - mn);
        l[g] = l[g] * corr + p;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[g][e] = acc[g][e] * corr + p * vf[e];
        m[g] = mn;
      }
    }
  }

  // merge the 4 warps
  __shared__ float sm_m[4][kMaxGroup], sm_l[4][kMaxGroup];
  __shared__ float sm_acc[4][kMaxGroup][kD];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      sm_m[warp][g] = m[g];
      sm_l[warp][g] = l[g];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) sm_acc[warp][g][lane * 4 + e] = acc[g][e];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * kD; idx += blockDim.x) {
    const int g = idx / kD, d = idx - g * kD;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mx = fmaxf(mx, sm_m[w][g]);
    float lsum = 0.f, o = 0.f;
    if (mx > -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float c = exp2f(sm_m[w][g] - mx);
        lsum += sm_l[w][g] * c;
        o += sm_acc[w][g][d] * c;
      }
    }
    const float res = lsum > 0.f ? o / lsum : 0.f;
    out[(static_cast<long>(row) * nq + kvh * G + g) * kD + d] = __float2bfloat16(res);
  }
}

}  // namespace

void paged_decode_attention(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool,
                            torch::Tensor block_table, torch::Tensor start, torch::Tensor len,
                            torch::Tensor out, double scale) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && q.is_contiguous(), "q must be contiguous bf16");
  TORCH_CHECK(k_pool.dim() == 4 && k_pool.size(3) == kD, "k_pool must be [pages, nkv, page, 128]");
  const int rows = static_cast<int>(q.size(0));
  const int nq = static_cast<int>(q.size(1));
  const int nkv = static_cast<int>(k_pool.size(1));
  const int page = static_cast<int>(k_pool.size(2));
  TORCH_CHECK(page % 4 == 0, "page size must be a multiple of 4");
  TORCH_CHECK(nq % nkv == 0, "nq must be a multiple of nkv");
  const int G = nq / nkv;
  const float scale_log2 = static_cast<float>(scale) * 1.4426950408889634f;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int blocks = rows * nkv;
  if (blocks == 0) return;
#define GB_ATT(GV)                                                                                   \
  paged_decode_attn_kernel<GV><<<blocks, 128, 0, stream>>>(                                          \
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()),                                          \
      reinterpret_cast<const __nv_bfloat16*>(k_pool.data_ptr()),                                     \
      reinterpret_cast<const __nv_bfloat16*>(v_pool.data_ptr()), block_table.data_ptr<int>(),        \
      start.data_ptr<int>(), len.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), \
      nq, nkv, page, static_cast<int>(block_table.size(1)), scale_log2)
  switch (G) {
    case 1: GB_ATT(1); break;
    case 2: GB_ATT(2); break;
    case 4: GB_ATT(4); break;
    case 8: GB_ATT(8); break;
    default: TORCH_CHECK(false, "unsupported GQA group size ", G);
  }
#undef GB_ATT
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace gb
