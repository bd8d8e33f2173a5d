// Decode-step attention over the paged KV cache (flash-decoding).
//
// Cache layout: k_pool / v_pool [num_pages, n_kv_heads, page_size, 128] bf16,
// block_table [rows, max_pages] maps a row's logical page to a physical page.
// Rows that share a prompt (the G completions of one GRASPO group) point at
// the same physical prompt pages, so the prompt KV is stored once per group;
// CTAs of one group are launched next to each other, so those pages are
// read from DRAM once and served from L2 to the other rows.  A row attends to
// key positions [start[row], len[row]).
//
// Grid: (split, kv head, row), row fastest.  A CTA handles all G = nq / nkv
// query heads of one KV head (GQA packing) over one contiguous slice of the
// key range.  Inside a CTA each warp walks 32-key chunks:
//   * QK: lane t owns key t of the chunk and computes its G dot products
//     (q broadcast from shared memory) -- no per-key shuffles;
//   * online softmax per head with one warp max / sum per chunk;
//   * PV: lane l owns head dims [4l, 4l+4); probabilities are broadcast by
//     shuffle, V rows are read coalesced.
// With more than one split, every CTA writes its (max, sum, acc) partial to a
// scratch buffer and bumps a per-(row, kv head) counter; the CTA that arrives
// last merges the partials and writes the output (no CTA ever waits on
// another).  The counter is reset by that last CTA, so the scratch buffer is
// reusable by the next launch without clearing.

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>

#include "graspo_noalloc.h"
#include "sm100_common.cuh"

namespace gb {

namespace {

constexpr int kD = 128;
constexpr int kWarps = 4;

struct DecodeAttnArgs {
  const __nv_bfloat16* q;       // [rows, nq, D]
  const __nv_bfloat16* k_pool;  // [pages, nkv, page, D]
  const __nv_bfloat16* v_pool;
  const int* block_table;       // [rows, max_pages]
  const int* start;             // [rows]
  const int* len;               // [rows]
  __nv_bfloat16* out;           // [rows, nq * D]
  float* part_acc;              // [rows, nq, splits, D]    (splits > 1)
  float* part_ml;               // [rows, nq, splits, 2]
  int* counters;                // [rows, nkv]
  int nq, nkv, page_size, max_pages, splits, keys_per_split;
  float scale_log2;
  // Shared-prefix mode (prefix_len > 0): consecutive groups of group_rows rows
  // share the pages of key positions [start, prefix_len).  Those keys are
  // handled by paged_prefix_attn_kernel for all rows of a group at once
  // (prefix_splits key slices, one partial slot each); the split kernels then
  // cover [prefix_len, len) and merge prefix_slots + splits partials per row.
  int prefix_len, group_rows, prefix_splits, prefix_kps, prefix_slots;
  int num_pages;  // pages in the pools (kernel-checks builds validate block-table entries)
  int* err;
};

template <int G>
__global__ void __launch_bounds__(kWarps * 32) paged_decode_attn_kernel(DecodeAttnArgs a) {
  const int rows_total = gridDim.x / (a.nkv * a.splits);
  const int row = blockIdx.x % rows_total;
  const int rest = blockIdx.x / rows_total;
  const int kvh = rest % a.nkv;
  const int split = rest / a.nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  __shared__ __align__(16) float q_s[G][kD];
  __shared__ float m_s[kWarps][G], l_s[kWarps][G];
  __shared__ float acc_s[kWarps][G][kD];
  __shared__ int is_last;

  for (int i = threadIdx.x; i < G * kD; i += blockDim.x) {
    const int g = i / kD, d = i - g * kD;
    q_s[g][d] = __bfloat162float(a.q[(static_cast<long>(row) * a.nq + kvh * G + g) * kD + d]) * a.scale_log2;
  }
  __syncthreads();

  const int s0 = a.start[row], s1 = a.len[row];
  const int k_begin = max(s0, split * a.keys_per_split);
  // keys beyond the row's block table are never read, whatever len says
  const int k_end = min(min(s1, a.max_pages * a.page_size), (split + 1) * a.keys_per_split);

  float m[G], l[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
  }

  const int* bt = a.block_table + static_cast<long>(row) * a.max_pages;
  // chunks of 32 keys, aligned to 32; warps take chunks round-robin
  const int first_chunk = k_begin >> 5;
  const int last_chunk = (k_end - 1) >> 5;
  for (int c = first_chunk + warp; c <= last_chunk && k_end > k_begin; c += kWarps) {
    const int t = c * 32 + lane;
    const bool valid = t >= k_begin && t < k_end;
    const int page = checked_index(valid ? bt[t / a.page_size] : bt[(c * 32) / a.page_size], a.num_pages, a.err);
    const long kv_off = ((static_cast<long>(page) * a.nkv + kvh) * a.page_size + (t % a.page_size)) * kD;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    if (valid) {
      const uint4* kr = reinterpret_cast<const uint4*>(a.k_pool + kv_off);
#pragma unroll 4
      for (int q8 = 0; q8 < kD / 8; ++q8) {
        const uint4 raw = kr[q8];
        const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f2 = __bfloat1622float2(k2[e]);
          kf[2 * e] = f2.x;
          kf[2 * e + 1] = f2.y;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 qa = *reinterpret_cast<const float4*>(&q_s[g][q8 * 8]);
          const float4 qb = *reinterpret_cast<const float4*>(&q_s[g][q8 * 8 + 4]);
          s[g] = fmaf(qa.x, kf[0], s[g]);
          s[g] = fmaf(qa.y, kf[1], s[g]);
          s[g] = fmaf(qa.z, kf[2], s[g]);
          s[g] = fmaf(qa.w, kf[3], s[g]);
          s[g] = fmaf(qb.x, kf[4], s[g]);
          s[g] = fmaf(qb.y, kf[5], s[g]);
          s[g] = fmaf(qb.z, kf[6], s[g]);
          s[g] = fmaf(qb.w, kf[7], s[g]);
        }
      }
    }
    float p[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sv = valid ? s[g] : -INFINITY;
      const float cmax = warp_max(sv);
      const float mn = fmaxf(m[g], cmax);
      const float corr = exp2f(m[g] - mn);  // m = -inf at first: exp2(-inf) = 0
      p[g] = valid ? exp2f(sv - mn) : 0.f;
      l[g] = l[g] * corr + warp_sum(p[g]);
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[g][e] *= corr;
      m[g] = mn;
    }
    // PV: lane owns dims [4*lane, 4*lane+4)
    const int n_valid_hi = min(32, k_end - c * 32);
    const int n_valid_lo = max(0, k_begin - c * 32);
    for (int j = n_valid_lo; j < n_valid_hi; ++j) {
      const int tj = c * 32 + j;
      const int pg = checked_index(bt[tj / a.page_size], a.num_pages, a.err);
      const long off = ((static_cast<long>(pg) * a.nkv + kvh) * a.page_size + (tj % a.page_size)) * kD + lane * 4;
      const uint2 vr = *reinterpret_cast<const uint2*>(a.v_pool + off);
      const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&vr);
      const float2 v01 = __bfloat1622float2(v2[0]);
      const float2 v23 = __bfloat1622float2(v2[1]);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pj = __shfl_sync(0xffffffffu, p[g], j);
        acc[g][0] = fmaf(pj, v01.x, acc[g][0]);
        acc[g][1] = fmaf(pj, v01.y, acc[g][1]);
        acc[g][2] = fmaf(pj, v23.x, acc[g][2]);
        acc[g][3] = fmaf(pj, v23.y, acc[g][3]);
      }
    }
  }

  // ---- merge warps
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      m_s[warp][g] = m[g];
      l_s[warp][g] = l[g];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) acc_s[warp][g][lane * 4 + e] = acc[g][e];
  }
  __syncthreads();
  const long head_base = static_cast<long>(row) * a.nq + kvh * G;
  for (int i = threadIdx.x; i < G * kD; i += blockDim.x) {
    const int g = i / kD, d = i - g * kD;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, m_s[w][g]);
    float ls = 0.f, o = 0.f;
    if (mx > -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float cf = exp2f(m_s[w][g] - mx);
        ls += l_s[w][g] * cf;
        o += acc_s[w][g][d] * cf;
      }
    }
    if (a.splits == 1) {
      a.out[(head_base + g) * kD + d] = __float2bfloat16(ls > 0.f ? o / ls : 0.f);
    } else {
      const long pidx = (head_base + g) * a.splits + split;
      a.part_acc[pidx * kD + d] = o;
      if (d == 0) {
        a.part_ml[pidx * 2] = mx;
        a.part_ml[pidx * 2 + 1] = ls;
      }
    }
  }
  if (a.splits == 1) return;

  // ---- last CTA of this (row, kv head) merges the splits
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* ctr = a.counters + static_cast<long>(row) * a.nkv + kvh;
    const int prev = atomicAdd(ctr, 1);
    is_last = (prev == a.splits - 1);
    if (is_last) *ctr = 0;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < G * kD; i += blockDim.x) {
    const int g = i / kD, d = i - g * kD;
    const long pbase = (head_base + g) * a.splits;
    float mx = -INFINITY;
    for (int sp = 0; sp < a.splits; ++sp) mx = fmaxf(mx, __ldcg(a.part_ml + (pbase + sp) * 2));
    float ls = 0.f, o = 0.f;
    if (mx > -INFINITY) {
      for (int sp = 0; sp < a.splits; ++sp) {
        const float ms = __ldcg(a.part_ml + (pbase + sp) * 2);
        if (ms == -INFINITY) continue;
        const float cf = exp2f(ms - mx);
        ls += __ldcg(a.part_ml + (pbase + sp) * 2 + 1) * cf;
        o += __ldcg(a.part_acc + (pbase + sp) * kD + d) * cf;
      }
    }
    a.out[(head_base + g) * kD + d] = __float2bfloat16(ls > 0.f ? o / ls : 0.f);
  }
}


// ---------------------------------------------------------------------------
// Tensor-core variant for page_size % 64 == 0.  Per CTA and 64-key tile:
// K and V tiles are copied to shared memory with cp.async (double buffered,
// 16-byte chunks XOR-swizzled by row so ldmatrix reads are conflict-free);
// each of the 4 warps owns 16 keys of the tile.  S = Q K^T uses
// mma.sync.m16n8k16 (bf16 in, fp32 out) with the G query heads as the first G
// of 16 MMA rows; P (the softmax numerators, re-packed to bf16 in registers)
// multiplies V loaded with ldmatrix.trans.  Per-warp online-softmax states are
// merged exactly as in the CUDA-core kernel.
constexpr int kTile = 64;
constexpr int kRowBytes = kD * 2;                    // 256 B per key row
constexpr int kTileBytes = kTile * kRowBytes;         // 16 KiB per K or V tile
constexpr int kPrefStages = 4;                          // prefix kernel: 3 tiles in flight
constexpr int kTcSmem = kPrefStages * 2 * kTileBytes;   // stages x (K, V) (prefix kernel)
constexpr int kTcStages = 3;                            // split kernel: 3 tiles in flight
constexpr int kTcSmemSplit = kTcStages * 2 * kTileBytes;
constexpr int kBtCache = 128;                           // block-table entries kept in shared memory

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  // byte offset of 16-byte chunk `chunk` (0..15) of key row `row` in a tile
  return static_cast<uint32_t>(row * kRowBytes + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Shared-prefix decode attention.  CTA = (group, kv head, prefix split); its
// 4 * MT warps take the group's R rows x G query heads (R * G <= 16 * MT) as MT
// MMA row tiles of 16 -- the prompt K/V tiles are loaded once for the whole
// group instead of once per row, and the MMA rows are full instead of G of 16.
// Warp w handles row tile w / 4 and keys [16 (w % 4), +16) of each 64-key
// tile, and writes its own partial (max, sum, acc) into slot
// split * 4 + w % 4 of every (row, head) it holds; the split kernel that runs
// next merges them with the partials of the generated keys.
template <int G, int MT>
__global__ void __launch_bounds__(MT * 4 * 32) paged_prefix_attn_kernel(DecodeAttnArgs a) {
  extern __shared__ __align__(128) uint8_t tc_smem[];
  constexpr int kThreadsP = MT * 4 * 32;
  const int groups = gridDim.x / (a.nkv * a.prefix_splits);
  const int grp = blockIdx.x % groups;
  const int rest = blockIdx.x / groups;
  const int kvh = rest % a.nkv;
  const int split = rest / a.nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = warp >> 2, kw = warp & 3;
  const int g = lane >> 2, c = (lane & 3) * 2;
  pdl_trigger();
  pdl_wait();
  const int R = a.group_rows;
  const int row0 = grp * R;
  const int s0 = a.start[row0];
  const int k_begin = max(s0, split * a.prefix_kps);
  const int k_end = min(min(a.prefix_len, a.max_pages * a.page_size), (split + 1) * a.prefix_kps);
  const int* bt = a.block_table + static_cast<long>(row0) * a.max_pages;
  const uint32_t sbase = smem_addr(tc_smem);
  const int total = a.prefix_slots + a.splits;

  // this thread's two MMA rows (g and g + 8 of row tile mt) -> (row, head)
  const int qr0 = mt * 16 + g, qr1 = qr0 + 8;
  const bool ok0 = qr0 < R * G, ok1 = qr1 < R * G;
  uint32_t qa[8][4];
  {
    const __nv_bfloat16* q0 = a.q + ((static_cast<long>(row0 + qr0 / G)) * a.nq + kvh * G + qr0 % G) * kD;
    const __nv_bfloat16* q1 = a.q + ((static_cast<long>(row0 + qr1 / G)) * a.nq + kvh * G + qr1 % G) * kD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int d0 = ks * 16 + c;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
      if (ok0) {
        v[0] = __bfloat162float(q0[d0]) * a.scale_log2;
        v[1] = __bfloat162float(q0[d0 + 1]) * a.scale_log2;
        v[4] = __bfloat162float(q0[d0 + 8]) * a.scale_log2;
        v[5] = __bfloat162float(q0[d0 + 9]) * a.scale_log2;
      }
      if (ok1) {
        v[2] = __bfloat162float(q1[d0]) * a.scale_log2;
        v[3] = __bfloat162float(q1[d0 + 1]) * a.scale_log2;
        v[6] = __bfloat162float(q1[d0 + 8]) * a.scale_log2;
        v[7] = __bfloat162float(q1[d0 + 9]) * a.scale_log2;
      }
      qa[ks][0] = pack_bf16(v[0], v[1]);
      qa[ks][1] = pack_bf16(v[2], v[3]);
      qa[ks][2] = pack_bf16(v[4], v[5]);
      qa[ks][3] = pack_bf16(v[6], v[7]);
    }
  }

  auto load_tile = [&](int tile, int stage) {
    const int t0 = tile * kTile;
    const int phys = checked_index(bt[t0 / a.page_size], a.num_pages, a.err);
    const long base = ((static_cast<long>(phys) * a.nkv + kvh) * a.page_size + (t0 % a.page_size)) * kD;
    const uint8_t* ksrc = reinterpret_cast<const uint8_t*>(a.k_pool + base);
    const uint8_t* vsrc = reinterpret_cast<const uint8_t*>(a.v_pool + base);
    const uint32_t kdst = sbase + stage * 2 * kTileBytes;
    const uint32_t vdst = kdst + kTileBytes;
#pragma unroll
    for (int i = 0; i < (kTileBytes / 16) / kThreadsP; ++i) {
      const int chunk_id = threadIdx.x + i * kThreadsP;
      const int r = chunk_id >> 4, ch = chunk_id & 15;
      cp_async16(kdst + swz(r, ch), ksrc + r * kRowBytes + ch * 16);
      cp_async16(vdst + swz(r, ch), vsrc + r * kRowBytes + ch * 16);
    }
  };

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const bool any = k_end > k_begin;
  const int t_first = any ? k_begin / kTile : 0, t_last = any ? (k_end - 1) / kTile : -1;
  // kPrefStages-deep cp.async ring: one commit group per tile (empty groups past the end)
#pragma unroll
  for (int sidx = 0; sidx < kPrefStages - 1; ++sidx) {
    if (t_first + sidx <= t_last) load_tile(t_first + sidx, sidx);
    cp_async_commit();
  }
  for (int tile = t_first; tile <= t_last; ++tile) {
    const int stage = (tile - t_first) % kPrefStages;
    cp_async_wait<kPrefStages - 2>();
    __syncthreads();
    const uint32_t kt = sbase + stage * 2 * kTileBytes;
    const uint32_t vt = kt + kTileBytes;
    const int key0 = kw * 16;
    float s[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int mi = lane >> 3, rr = lane & 7;
      const int key = key0 + rr + ((mi >> 1) << 3);
      const int chunk = ks * 2 + (mi & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kt + swz(key, chunk), b0, b1, b2, b3);
      mma_bf16(s[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
      mma_bf16(s[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
    }
    const int tbase = tile * kTile + key0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tbase + j * 8 + c + e;
        if (t < k_begin || t >= k_end) {
          s[j][e] = -INFINITY;
          s[j][2 + e] = -INFINITY;
        }
      }
    }
    // online softmax, rows g (elements 0,1) and g + 8 (elements 2,3)
    float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float c0 = n0 == -INFINITY ? 1.f : exp2f(m0 - n0);
    const float c1 = n1 == -INFINITY ? 1.f : exp2f(m1 - n1);
    float p[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        p[j][e] = n0 == -INFINITY ? 0.f : exp2f(s[j][e] - n0);
        p[j][2 + e] = n1 == -INFINITY ? 0.f : exp2f(s[j][2 + e] - n1);
      }
    }
    float ps0 = p[0][0] + p[0][1] + p[1][0] + p[1][1];
    float ps1 = p[0][2] + p[0][3] + p[1][2] + p[1][3];
    ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
    ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
    ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
    ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
    l0 = l0 * c0 + ps0;
    l1 = l1 * c1 + ps1;
    m0 = n0;
    m1 = n1;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= c0;
      o[n][1] *= c0;
      o[n][2] *= c1;
      o[n][3] *= c1;
    }
    const uint32_t pa0 = pack_bf16(p[0][0], p[0][1]), pa1 = pack_bf16(p[0][2], p[0][3]);
    const uint32_t pa2 = pack_bf16(p[1][0], p[1][1]), pa3 = pack_bf16(p[1][2], p[1][3]);
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      const int mi = lane >> 3, rr = lane & 7;
      const int key = key0 + rr + ((mi & 1) << 3);
      const int chunk = nd * 2 + (mi >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vt + swz(key, chunk), b0, b1, b2, b3);
      mma_bf16(o[2 * nd], pa0, pa1, pa2, pa3, b0, b1);
      mma_bf16(o[2 * nd + 1], pa0, pa1, pa2, pa3, b2, b3);
    }
    __syncthreads();  // the stage read above is refilled below
    if (tile + kPrefStages - 1 <= t_last)
      load_tile(tile + kPrefStages - 1, (tile + kPrefStages - 1 - t_first) % kPrefStages);
    cp_async_commit();
  }
  cp_async_wait<0>();
  // ---- the four key-warps of each row tile merge inside the CTA (their K/V
  // staging memory holds the exchange), so each split leaves one partial slot
  __shared__ float xm[2][4][16], xl[2][4][16];
  float* xo = reinterpret_cast<float*>(tc_smem);          // [2 tiles][4 key-warps][16 rows][kD]
  __syncthreads();                                        // no warp reads K / V any more
  for (int mt0 = 0; mt0 < MT; mt0 += 2) {
    if (mt >= mt0 && mt < mt0 + 2) {
      const int lt = mt - mt0;
      float* dst = xo + static_cast<long>((lt * 4 + kw) * 16) * kD;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        dst[g * kD + n * 8 + c] = o[n][0];
        dst[g * kD + n * 8 + c + 1] = o[n][1];
        dst[(g + 8) * kD + n * 8 + c] = o[n][2];
        dst[(g + 8) * kD + n * 8 + c + 1] = o[n][3];
      }
      if ((lane & 3) == 0) {
        xm[lt][kw][g] = m0;
        xl[lt][kw][g] = l0;
        xm[lt][kw][g + 8] = m1;
        xl[lt][kw][g + 8] = l1;
      }
    }
    __syncthreads();
    const int nlt = min(2, MT - mt0);
    for (int i = threadIdx.x; i < nlt * 16 * kD; i += kThreadsP) {
      const int lt = i / (16 * kD), rr = (i / kD) % 16, d = i % kD;
      const int qr = (mt0 + lt) * 16 + rr;
      if (qr >= R * G) continue;
      float mm = -INFINITY;
#pragma unroll
      for (int k = 0; k < 4; ++k) mm = fmaxf(mm, xm[lt][k][rr]);
      float ll = 0.f, oo = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float w = mm == -INFINITY ? 0.f : exp2f(xm[lt][k][rr] - mm);
        ll += xl[lt][k][rr] * w;
        oo += xo[static_cast<long>((lt * 4 + k) * 16 + rr) * kD + d] * w;
      }
      const long head_idx = static_cast<long>(row0 + qr / G) * a.nq + kvh * G + qr % G;
      const long pidx = head_idx * total + split;
      a.part_acc[pidx * kD + d] = oo;
      if (d == 0) {
        a.part_ml[pidx * 2] = mm;
        a.part_ml[pidx * 2 + 1] = ll;
      }
    }
    __syncthreads();
  }
}

template <int G>
__global__ void __launch_bounds__(kWarps * 32) paged_decode_attn_tc_kernel(DecodeAttnArgs a) {
  extern __shared__ __align__(128) uint8_t tc_smem[];
  __shared__ float m_s[kWarps][16], l_s[kWarps][16];
  __shared__ float acc_s[kWarps][G][kD];
  __shared__ int is_last;
  const int rows_total = gridDim.x / (a.nkv * a.splits);
  const int row = blockIdx.x % rows_total;
  const int rest = blockIdx.x / rows_total;
  const int kvh = rest % a.nkv;
  const int split = rest / a.nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = (lane & 3) * 2;
  pdl_trigger();
  pdl_wait();

  const int s0 = a.start[row], s1 = a.len[row];
  const int P = a.prefix_len;  // 0 unless the shared prefix is handled separately
  const int total = a.prefix_slots + a.splits;
  const int k_begin = max(max(s0, P), P + split * a.keys_per_split);
  // keys beyond the row's block table are never read, whatever len says
  const int k_end = min(min(s1, a.max_pages * a.page_size), P + (split + 1) * a.keys_per_split);
  const int t_first = k_begin / kTile, t_last = (k_end - 1) / kTile;
  const int* bt = a.block_table + static_cast<long>(row) * a.max_pages;
  const uint32_t sbase = smem_addr(tc_smem);

  // Q fragments (A operand, rows = heads; rows >= G are zero), pre-scaled
  uint32_t qa[8][4];
  {
    const __nv_bfloat16* qr = a.q + (static_cast<long>(row) * a.nq + kvh * G) * kD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
      if (g < G) {
        const int d0 = ks * 16 + c;
        v[0] = __bfloat162float(qr[g * kD + d0]) * a.scale_log2;
        v[1] = __bfloat162float(qr[g * kD + d0 + 1]) * a.scale_log2;
        v[4] = __bfloat162float(qr[g * kD + d0 + 8]) * a.scale_log2;
        v[5] = __bfloat162float(qr[g * kD + d0 + 9]) * a.scale_log2;
      }
      qa[ks][0] = pack_bf16(v[0], v[1]);
      qa[ks][1] = pack_bf16(v[2], v[3]);  // row g + 8: zero
      qa[ks][2] = pack_bf16(v[4], v[5]);
      qa[ks][3] = pack_bf16(v[6], v[7]);  // row g + 8: zero
    }
  }

  // block-table entries of this split's pages, read once
  __shared__ int bt_s[kBtCache];
  const int page_first = k_end > k_begin ? (t_first * kTile) / a.page_size : 0;
  const int page_count = k_end > k_begin ? ((t_last + 1) * kTile - 1) / a.page_size - page_first + 1 : 0;
  for (int i = threadIdx.x; i < min(page_count, kBtCache); i += blockDim.x) bt_s[i] = bt[page_first + i];
  __syncthreads();
  auto page_of = [&](int t0) {
    const int pg = t0 / a.page_size - page_first;
    return pg < kBtCache ? bt_s[pg] : bt[page_first + pg];
  };

  auto load_tile = [&](int tile, int stage) {
    const int t0 = tile * kTile;
    const int phys = checked_index(page_of(t0), a.num_pages, a.err);
    const long base = ((static_cast<long>(phys) * a.nkv + kvh) * a.page_size + (t0 % a.page_size)) * kD;
    const uint8_t* ksrc = reinterpret_cast<const uint8_t*>(a.k_pool + base);
    const uint8_t* vsrc = reinterpret_cast<const uint8_t*>(a.v_pool + base);
    const uint32_t kdst = sbase + stage * 2 * kTileBytes;
    const uint32_t vdst = kdst + kTileBytes;
#pragma unroll
    for (int i = 0; i < (kTileBytes / 16) / (kWarps * 32); ++i) {
      const int chunk_id = threadIdx.x + i * kWarps * 32;  // 0..1023
      const int r = chunk_id >> 4, ch = chunk_id & 15;
      cp_async16(kdst + swz(r, ch), ksrc + r * kRowBytes + ch * 16);
      cp_async16(vdst + swz(r, ch), vsrc + r * kRowBytes + ch * 16);
    }
  };

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // for row g (rows g+8 are padding)

  // kTcStages-deep cp.async ring: one commit group per tile (empty groups past the end)
  const bool any_keys = k_end > k_begin;
#pragma unroll
  for (int sidx = 0; sidx < kTcStages - 1; ++sidx) {
    if (any_keys && t_first + sidx <= t_last) load_tile(t_first + sidx, sidx);
    cp_async_commit();
  }
  for (int tile = t_first; tile <= t_last && any_keys; ++tile) {
    const int stage = (tile - t_first) % kTcStages;
    cp_async_wait<kTcStages - 2>();
    __syncthreads();
    const uint32_t kt = sbase + stage * 2 * kTileBytes;
    const uint32_t vt = kt + kTileBytes;
    const int key0 = warp * 16;  // this warp's 16 keys inside the tile
    // ---- S = Q K^T for 16 keys (two n-tiles of 8)
    float s[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      // matrices: (keys 0-7, dims 0-7), (keys 0-7, dims 8-15), (keys 8-15, dims 0-7), (keys 8-15, dims 8-15)
      const int mi = lane >> 3, rr = lane & 7;
      const int key = key0 + rr + ((mi >> 1) << 3);
      const int chunk = ks * 2 + (mi & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kt + swz(key, chunk), b0, b1, b2, b3);
      mma_bf16(s[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
      mma_bf16(s[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
    }
    // ---- mask keys outside [k_begin, k_end)
    const int tbase = tile * kTile + key0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tbase + j * 8 + c + e;
        if (t < k_begin || t >= k_end) s[j][e] = -INFINITY;
        s[j][2 + e] = -INFINITY;  // padding rows
      }
    }
    // ---- online softmax for row g over this warp's 16 keys
    float mx = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    float p[2][2];
    float corr = 1.f;
    if (m_new == -INFINITY) {
      p[0][0] = p[0][1] = p[1][0] = p[1][1] = 0.f;
    } else {
      corr = exp2f(m_run - m_new);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) p[j][e] = exp2f(s[j][e] - m_new);
    }
    float ps = p[0][0] + p[0][1] + p[1][0] + p[1][1];
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l_run = l_run * corr + ps;
    m_run = m_new;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= corr;
      o[n][1] *= corr;
    }
    // ---- O += P V  (P: 16 rows x 16 keys as the A operand)
    const uint32_t pa0 = pack_bf16(p[0][0], p[0][1]);
    const uint32_t pa2 = pack_bf16(p[1][0], p[1][1]);
    const uint32_t zero = 0u;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      // matrices: (keys 0-7, dims 16nd..+7), (keys 8-15, dims 16nd..), (keys 0-7, dims 16nd+8..), (keys 8-15, ...)
      const int mi = lane >> 3, rr = lane & 7;
      const int key = key0 + rr + ((mi & 1) << 3);
      const int chunk = nd * 2 + (mi >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vt + swz(key, chunk), b0, b1, b2, b3);
      mma_bf16(o[2 * nd], pa0, zero, pa2, zero, b0, b1);
      mma_bf16(o[2 * nd + 1], pa0, zero, pa2, zero, b2, b3);
    }
    __syncthreads();  // the stage read above is refilled below
    if (tile + kTcStages - 1 <= t_last) load_tile(tile + kTcStages - 1, (tile + kTcStages - 1 - t_first) % kTcStages);
    cp_async_commit();
  }
  cp_async_wait<0>();

  // ---- merge warps (rows g < G hold data)
  if ((lane & 3) == 0 && g < G) {
    m_s[warp][g] = m_run;
    l_s[warp][g] = l_run;
  }
  if (g < G) {
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      acc_s[warp][g][n * 8 + c] = o[n][0];
      acc_s[warp][g][n * 8 + c + 1] = o[n][1];
    }
  }
  __syncthreads();
  const long head_base = static_cast<long>(row) * a.nq + kvh * G;
  for (int i = threadIdx.x; i < G * kD; i += blockDim.x) {
    const int gg = i / kD, d = i - gg * kD;
    float mxx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mxx = fmaxf(mxx, m_s[w][gg]);
    float ls = 0.f, ov = 0.f;
    if (mxx > -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (m_s[w][gg] == -INFINITY) continue;
        const float cf = exp2f(m_s[w][gg] - mxx);
        ls += l_s[w][gg] * cf;
        ov += acc_s[w][gg][d] * cf;
      }
    }
    if (total == 1) {
      a.out[(head_base + gg) * kD + d] = __float2bfloat16(ls > 0.f ? ov / ls : 0.f);
    } else if (a.splits == 1) {
      // one key split besides the shared-prefix slots, which the prefix kernel
      // (earlier in stream order) has completed: merge them here directly
      const long pbase = (head_base + gg) * total;
      float mm = mxx;
      for (int sp = 0; sp < a.prefix_slots; ++sp) mm = fmaxf(mm, __ldcg(a.part_ml + (pbase + sp) * 2));
      float lt = 0.f, ot = 0.f;
      if (mm > -INFINITY) {
        if (mxx > -INFINITY) {
          const float cf = exp2f(mxx - mm);
          lt = ls * cf;
          ot = ov * cf;
        }
        for (int sp = 0; sp < a.prefix_slots; ++sp) {
          const float ms = __ldcg(a.part_ml + (pbase + sp) * 2);
          if (ms == -INFINITY) continue;
          const float cf = exp2f(ms - mm);
          lt += __ldcg(a.part_ml + (pbase + sp) * 2 + 1) * cf;
          ot += __ldcg(a.part_acc + (pbase + sp) * kD + d) * cf;
        }
      }
      a.out[(head_base + gg) * kD + d] = __float2bfloat16(lt > 0.f ? ot / lt : 0.f);
    } else {
      const long pidx = (head_base + gg) * total + a.prefix_slots + split;
      a.part_acc[pidx * kD + d] = ov;
      if (d == 0) {
        a.part_ml[pidx * 2] = mxx;
        a.part_ml[pidx * 2 + 1] = ls;
      }
    }
  }
  if (total == 1 || a.splits == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* ctr = a.counters + static_cast<long>(row) * a.nkv + kvh;
    const int prev = atomicAdd(ctr, 1);
    is_last = (prev == a.splits - 1);
    if (is_last) *ctr = 0;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < G * kD; i += blockDim.x) {
    const int gg = i / kD, d = i - gg * kD;
    const long pbase = (head_base + gg) * total;
    float mxx = -INFINITY;
    for (int sp = 0; sp < total; ++sp) mxx = fmaxf(mxx, __ldcg(a.part_ml + (pbase + sp) * 2));
    float ls = 0.f, ov = 0.f;
    if (mxx > -INFINITY) {
      for (int sp = 0; sp < total; ++sp) {
        const float ms = __ldcg(a.part_ml + (pbase + sp) * 2);
        if (ms == -INFINITY) continue;
        const float cf = exp2f(ms - mxx);
        ls += __ldcg(a.part_ml + (pbase + sp) * 2 + 1) * cf;
        ov += __ldcg(a.part_acc + (pbase + sp) * kD + d) * cf;
      }
    }
    a.out[(head_base + gg) * kD + d] = __float2bfloat16(ls > 0.f ? ov / ls : 0.f);
  }
}

}  // namespace

// scratch: optional fp32 buffer of at least rows*nq*splits*(D+2) floats plus
// rows*nkv ints for the counters (zero-initialised once); required when the
// launch is split.
bool kernel_checks() { return kKernelChecks; }

void paged_decode_attention(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool,
                            torch::Tensor block_table, torch::Tensor start, torch::Tensor len,
                            torch::Tensor out, double scale, int64_t splits,
                            c10::optional<torch::Tensor> scratch, int64_t prefix_len, int64_t group_rows,
                            int64_t prefix_splits, c10::optional<torch::Tensor> err) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && q.is_contiguous(), "q must be contiguous bf16");
  TORCH_CHECK(k_pool.dim() == 4 && k_pool.size(3) == kD, "k_pool must be [pages, nkv, page, 128]");
  const int rows = static_cast<int>(q.size(0));
  const int nq = static_cast<int>(q.size(1));
  const int nkv = static_cast<int>(k_pool.size(1));
  const int page = static_cast<int>(k_pool.size(2));
  TORCH_CHECK(nq % nkv == 0, "nq must be a multiple of nkv");
  const int G = nq / nkv;
  const int max_pages = static_cast<int>(block_table.size(1));
  DecodeAttnArgs a{};
  a.num_pages = static_cast<int>(k_pool.size(0));
  a.err = (err.has_value() && err->defined()) ? err->data_ptr<int>() : nullptr;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k_pool = reinterpret_cast<const __nv_bfloat16*>(k_pool.data_ptr());
  a.v_pool = reinterpret_cast<const __nv_bfloat16*>(v_pool.data_ptr());
  a.block_table = block_table.data_ptr<int>();
  a.start = start.data_ptr<int>();
  a.len = len.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.nq = nq;
  a.nkv = nkv;
  a.page_size = page;
  a.max_pages = max_pages;
  a.splits = static_cast<int>(std::max<int64_t>(1, splits));
  const int capacity = max_pages * page;
  const bool use_tc = (page % kTile) == 0 && G <= 8;
  const int align = use_tc ? kTile : 32;
  const int P = static_cast<int>(prefix_len);
  int MT = 0;
  if (P > 0) {
    const int R = static_cast<int>(group_rows);
    TORCH_CHECK(use_tc, "shared-prefix decode attention needs pages that are a multiple of 64 keys");
    TORCH_CHECK(R > 0 && rows % R == 0 && R * G <= 64, "rows must form groups of group_rows with R * G <= 64");
    TORCH_CHECK(P % kTile == 0 && P <= capacity && prefix_splits > 0, "prefix length must be 64-aligned");
    MT = (R * G + 15) / 16;
    MT = MT <= 1 ? 1 : (MT <= 2 ? 2 : 4);
    a.prefix_len = P;
    a.group_rows = R;
    a.prefix_splits = static_cast<int>(prefix_splits);
    a.prefix_kps = ((P + a.prefix_splits - 1) / a.prefix_splits + kTile - 1) / kTile * kTile;
    a.prefix_slots = a.prefix_splits;
  }
  a.keys_per_split = ((capacity - P + a.splits - 1) / a.splits + align - 1) / align * align;
  a.scale_log2 = static_cast<float>(scale) * 1.4426950408889634f;
  const int total = a.prefix_slots + a.splits;
  if (total > 1) {
    TORCH_CHECK(scratch.has_value() && scratch->defined() && scratch->scalar_type() == torch::kFloat32,
                "split decode attention needs an fp32 scratch buffer");
    const long need_f = static_cast<long>(rows) * nq * total * (kD + 2);
    const long need = need_f + static_cast<long>(rows) * nkv;
    TORCH_CHECK(scratch->numel() >= need, "decode-attention scratch too small: need ", need, " floats");
    float* base = scratch->data_ptr<float>();
    a.part_acc = base;
    a.part_ml = base + static_cast<long>(rows) * nq * total * kD;
    a.counters = reinterpret_cast<int*>(base + need_f);
  }
  const int blocks = rows * nkv * a.splits;
  if (blocks == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (P > 0) {
    static bool pconf[64][4][3] = {};
    const int dev = q.get_device();
    const int pblocks = (rows / a.group_rows) * nkv * a.prefix_splits;
    const int gi = G == 1 ? 0 : (G == 2 ? 1 : (G == 4 ? 2 : 3));
    const int mi = MT == 1 ? 0 : (MT == 2 ? 1 : 2);
#define GB_PF(GV, MV)                                                                                         \
  do {                                                                                                        \
    if (!pconf[dev][gi][mi]) {                                                                                \
      cudaFuncSetAttribute(paged_prefix_attn_kernel<GV, MV>, cudaFuncAttributeMaxDynamicSharedMemorySize,     \
                           kTcSmem);                                                                          \
      pconf[dev][gi][mi] = true;                                                                              \
    }                                                                                                         \
    C10_CUDA_CHECK(launch_kernel(paged_prefix_attn_kernel<GV, MV>, dim3(pblocks), dim3(MV * 128), kTcSmem,   \
                                 stream, a));                                                                 \
  } while (0)
#define GB_PF_G(GV)                   \
  switch (MT) {                       \
    case 1: GB_PF(GV, 1); break;      \
    case 2: GB_PF(GV, 2); break;      \
    default: GB_PF(GV, 4); break;     \
  }
    switch (G) {
      case 1: GB_PF_G(1); break;
      case 2: GB_PF_G(2); break;
      case 4: GB_PF_G(4); break;
      default: GB_PF_G(8); break;
    }
#undef GB_PF_G
#undef GB_PF
  }
  if (use_tc) {
    static bool configured[64][4] = {};
    const int dev = q.get_device();
#define GB_TC(GV, IDX)                                                                                       \
  if (!configured[dev][IDX]) {                                                                               \
    cudaFuncSetAttribute(paged_decode_attn_tc_kernel<GV>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemSplit); \
    configured[dev][IDX] = true;                                                                             \
  }                                                                                                          \
  C10_CUDA_CHECK(launch_kernel(paged_decode_attn_tc_kernel<GV>, dim3(blocks), dim3(kWarps * 32), kTcSmemSplit, stream, a))
    switch (G) {
      case 1: GB_TC(1, 0); break;
      case 2: GB_TC(2, 1); break;
      case 4: GB_TC(4, 2); break;
      case 8: GB_TC(8, 3); break;
      default: TORCH_CHECK(false, "unsupported GQA group size ", G);
    }
#undef GB_TC
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  switch (G) {
    case 1: paged_decode_attn_kernel<1><<<blocks, kWarps * 32, 0, stream>>>(a); break;
    case 2: paged_decode_attn_kernel<2><<<blocks, kWarps * 32, 0, stream>>>(a); break;
    case 4: paged_decode_attn_kernel<4><<<blocks, kWarps * 32, 0, stream>>>(a); break;
    case 8: paged_decode_attn_kernel<8><<<blocks, kWarps * 32, 0, stream>>>(a); break;
    default: TORCH_CHECK(false, "unsupported GQA group size ", G);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace gb

// ===========================================================================
// Allocation-free entry point (C ABI).
//
// This entry point has no counterpart in the reference implementation.
//
// Some callers cannot allocate device memory when they call into this library:
// a serving process whose whole HBM budget is carved up up front by its own
// arena allocator (and which forbids any other cudaMalloc), C or C++ hosts that
// have no PyTorch caching allocator to borrow a scratch tensor from, and code
// on a latency-critical path where cudaMalloc's implicit device
// synchronisation is unacceptable.  For them the split decode attention can
// run with its scratch (per-split partial results plus the per-(row, kv head)
// arrival counters) taken from a fixed array compiled into this library
// instead of from a caller-provided buffer.
//
// Limits and contract:
//  * The array holds kNoAllocScratchFloats floats (4 MiB) and
//    kNoAllocMaxCounters counters (32 KiB); every GPU that loads this library
//    keeps that memory until the process exits.  A call whose
//    rows * nq * splits * (128 + 2) floats or rows * nkv counters do not fit is
//    rejected with GB_NOALLOC_TOO_LARGE before anything is launched.
//  * The caller passes inputs and outputs as device pointers plus the stream.
//    Nothing is allocated: no cudaMalloc / cudaFree, no library allocator.
//  * The first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (host code cannot use the array's name as a device
//    address).  Make that first call on each device before any stream capture.
//  * Every call uses the same array and the array keeps the last call's
//    contents; the counters are cleared (cudaMemsetAsync on the call's stream)
//    before each launch.  Calls that can overlap on the GPU (different streams
//    without ordering) race on the array and must not be issued.
// ===========================================================================

constexpr long kNoAllocScratchFloats = GRASPO_NOALLOC_SCRATCH_FLOATS;
constexpr int kNoAllocMaxCounters = GRASPO_NOALLOC_MAX_COUNTERS;

// File-scope scratch for the allocation-free entry point (see above).  In host
// code these names are host-side stand-ins, not device addresses: the device
// addresses come from cudaGetSymbolAddress.
static __device__ __align__(256) float g_decode_attn_scratch[kNoAllocScratchFloats];
static __device__ __align__(256) int g_decode_attn_counters[kNoAllocMaxCounters];

namespace gb {
namespace noalloc {

struct DeviceSlots {
  float* scratch = nullptr;
  int* counters = nullptr;
  bool ready = false;
};

static DeviceSlots g_slots[64];
static std::mutex g_slots_mutex;

// Resolve the device addresses of the two arrays for the current device.
static int resolve_slots(int device, DeviceSlots** out) {
  if (device < 0 || device >= 64) return 5;
  std::lock_guard<std::mutex> lock(g_slots_mutex);
  DeviceSlots& s = g_slots[device];
  if (!s.ready) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_attn_scratch) != cudaSuccess || p == nullptr) return 3;
    s.scratch = static_cast<float*>(p);
    p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_attn_counters) != cudaSuccess || p == nullptr) return 3;
    s.counters = static_cast<int*>(p);
    s.ready = true;
  }
  *out = &s;
  return 0;
}

}  // namespace noalloc
}  // namespace gb

// Paged decode attention, split over the key range, scratch from the library's
// fixed array.  Same layouts and semantics as paged_decode_attention(); the
// declaration and its contract are in graspo_noalloc.h.
extern "C" int graspo_paged_decode_attention_noalloc(const void* q, const void* k_pool, const void* v_pool,
                                                     const int* block_table, const int* start, const int* len,
                                                     void* out, int rows, int nq, int nkv, int page_size,
                                                     int max_pages, int num_pages, int splits, float scale, int* err,
                                                     cudaStream_t stream) {
  using namespace gb;
  if (q == nullptr || k_pool == nullptr || v_pool == nullptr || block_table == nullptr || start == nullptr ||
      len == nullptr || out == nullptr || rows <= 0 || nq <= 0 || nkv <= 0 || nq % nkv != 0 || page_size <= 0 ||
      max_pages <= 0 || num_pages <= 0 || splits < 2) {
    return GB_NOALLOC_BAD_ARGUMENT;
  }
  const int G = nq / nkv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return GB_NOALLOC_BAD_ARGUMENT;
  const long need_floats = static_cast<long>(rows) * nq * splits * (kD + 2);
  const long need_counters = static_cast<long>(rows) * nkv;
  if (need_floats > kNoAllocScratchFloats || need_counters > kNoAllocMaxCounters) {
    return GB_NOALLOC_TOO_LARGE;
  }
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return GB_NOALLOC_BAD_DEVICE;
  noalloc::DeviceSlots* slots = nullptr;
  const int rc = noalloc::resolve_slots(device, &slots);
  if (rc != 0) return rc;
  if (cudaMemsetAsync(slots->counters, 0, need_counters * sizeof(int), stream) != cudaSuccess) {
    return GB_NOALLOC_LAUNCH_FAILED;
  }
  DecodeAttnArgs a{};
  a.num_pages = num_pages;
  a.err = err;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k_pool = static_cast<const __nv_bfloat16*>(k_pool);
  a.v_pool = static_cast<const __nv_bfloat16*>(v_pool);
  a.block_table = block_table;
  a.start = start;
  a.len = len;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.part_acc = slots->scratch;
  a.part_ml = slots->scratch + static_cast<long>(rows) * nq * splits * kD;
  a.counters = slots->counters;
  a.nq = nq;
  a.nkv = nkv;
  a.page_size = page_size;
  a.max_pages = max_pages;
  a.splits = splits;
  const int capacity = max_pages * page_size;
  a.keys_per_split = ((capacity + splits - 1) / splits + 31) / 32 * 32;
  a.scale_log2 = scale * 1.4426950408889634f;
  const int blocks = rows * nkv * splits;
  switch (G) {
    case 1: paged_decode_attn_kernel<1><<<blocks, kWarps * 32, 0, stream>>>(a); break;
    case 2: paged_decode_attn_kernel<2><<<blocks, kWarps * 32, 0, stream>>>(a); break;
    case 4: paged_decode_attn_kernel<4><<<blocks, kWarps * 32, 0, stream>>>(a); break;
    default: paged_decode_attn_kernel<8><<<blocks, kWarps * 32, 0, stream>>>(a); break;
  }
  return cudaGetLastError() == cudaSuccess ? GB_NOALLOC_OK : GB_NOALLOC_LAUNCH_FAILED;
}
