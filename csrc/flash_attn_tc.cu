// Flash attention forward on the 5th-generation tensor cores (tcgen05 + TMEM).
// Reference counterpart: SDPA with an explicit boolean causal + padding mask and
// repeat_interleave for GQA (src/graspo/backends/graspoflow/models/common/layers_qwen3.py:252-257,
// src/graspo/backends/graspoflow/tensor_utils.py:452-468).
//
// Same contract as flash_attn_fwd (csrc/flash_attn.cu): q [T, nq, 128], k / v
// [T, nkv, 128] bf16, T = B * S tokens, row b attends causally inside its
// valid range [start[b], end[b]); outputs O (bf16) and the row log-sum-exp
// (log2 domain).  CTA = 128 query rows of one head, key tiles of 128.
//
// Warp roles (320 threads):
//   warp 0     TMA producer: Q once, then K and V tiles into 2-stage rings;
//   warp 1     TMEM owner (512 columns: S double buffer at 0 / 128, O at 256)
//              and MMA issuer: S_j = Q K_j^T (M=128, N=128, K=128) into
//              S[j % 2], then O += P_{j-1} V_{j-1} (A = P from shared memory,
//              B = V read MN-major) -- so QK^T of tile j overlaps the softmax
//              of tile j-1;
//   warps 2-9  softmax, two threads per query row: warps w and w + 4 read the
//              same TMEM lanes (row = their lane) and take 64 of the 128 key
//              columns each (and 64 of the 128 head-dim columns of O).  The
//              pair swaps its partial row maxima through shared memory
//              (barrier.red also agrees on the error state), then each thread
//              computes p = 2^(s * scale - m) for its half, keeps its own
//              partial row sum (both halves see the same rescale factors, so
//              the sums add at the end) and writes its 64-key atom column of P
//              (bf16, 128B-swizzled K-major).  Only tiles that touch a range
//              boundary or the causal diagonal evaluate the mask.  O is
//              rescaled in TMEM only when the running max grows by more than
//              2^8 (otherwise the stale max is kept: P stays <= 256, exact in
//              fp32 accumulation), and normalised once at the end.
// Every wait is bounded (an error word is set and the kernel drains); the
// pair barriers are reached the same number of times by both warps of a pair
// on every path.

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "sm100_common.cuh"

namespace gb {

CUtensorMap make_tmap_bf16(const void* ptr, long rows, long cols, long ld, int box_rows);

namespace {

constexpr int kBM = 128;           // query rows per CTA
constexpr int kBN = 128;           // keys per tile
constexpr int kHD = 128;           // head dim
constexpr int kAtom = kBM * 128;   // one 128-row x 128-byte swizzle-atom column: 16 KiB
constexpr int kTile = 2 * kAtom;   // 128 rows x 128 bf16: 32 KiB
constexpr int kStages = 2;
constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.f;

// smem layout (offsets from a 1024-aligned base)
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTile;
constexpr int kOffV = kOffK + kStages * kTile;
constexpr int kOffP = kOffV + kStages * kTile;
constexpr int kOffBar = kOffP + kTile;
constexpr int kOffX = kOffBar + 256;          // pair exchange: [2 parity][2 half][128 rows] fp32
constexpr int kSmem = kOffX + 2 * 2 * kBM * 4 + 1024;

struct FwdTcArgs {
  __nv_bfloat16* o;
  float* lse;
  const int *start, *end;
  int S, nq, nkv;
  float scale_log2;
  int* err;
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// barrier over the 64 threads of a softmax warp pair that also ANDs a predicate
__device__ __forceinline__ bool pair_and(int id, bool p) {
  uint32_t out;
  asm volatile(
      "{\n .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n"
      " barrier.red.and.pred po, %2, 64, pi;\n selp.u32 %0, 1, 0, po;\n}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(p)), "r"(id)
      : "memory");
  return out != 0;
}

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32; 2^-inf = +0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, FwdTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* sm = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;    // [2]
  uint64_t* k_empty = bar + 3;   // [2]
  uint64_t* v_full = bar + 5;    // [2]
  uint64_t* v_empty = bar + 7;   // [2]
  uint64_t* s_full = bar + 9;    // [2]
  uint64_t* s_free = bar + 11;   // [2]
  uint64_t* p_full = bar + 13;
  uint64_t* o_done = bar + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // heaviest (latest) query blocks first
  const int qb = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);
  const int h = blockIdx.y, b = blockIdx.z;
  const int G = a.nq / a.nkv, hk = h / G;
  const int q0 = qb * kBM;
  const int s0 = a.start[b], s1 = a.end[b];
  const int q_last = min(q0 + kBM, s1) - 1;
  const bool any = q_last >= s0 && q0 < s1;
  const int j_first = any ? s0 / kBN : 0;
  const int j_last = any ? q_last / kBN : -1;
  const int n_tiles = j_last - j_first + 1;
  const long tok0 = static_cast<long>(b) * a.S;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(k_full + i, 1);
      mbar_init(k_empty + i, 1);
      mbar_init(v_full + i, 1);
      mbar_init(v_empty + i, 1);
      mbar_init(s_full + i, 1);
      mbar_init(s_free + i, kSoftmaxThreads);
    }
    mbar_init(p_full, kSoftmaxThreads);
    mbar_init(o_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = smem_addr(sm + kOffQ), sK = smem_addr(sm + kOffK), sV = smem_addr(sm + kOffV),
                 sP = smem_addr(sm + kOffP);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, kTile);
      for (int c = 0; c < 2; ++c)
        tma_load_2d(sm + kOffQ + c * kAtom, &tmQ, q_full, h * kHD + c * 64, static_cast<int>(tok0 + q0));
      for (int i = 0; i < n_tiles; ++i) {
        const int st = i & 1;
        const int key0 = (j_first + i) * kBN;
        if (i >= 2 && !mbar_wait(k_empty + st, ((i - 2) >> 1) & 1, a.err, kErrSmemEmptyTimeout)) break;
        mbar_arrive_expect_tx(k_full + st, kTile);
        for (int c = 0; c < 2; ++c)
          tma_load_2d(sm + kOffK + st * kTile + c * kAtom, &tmK, k_full + st, hk * kHD + c * 64,
                      static_cast<int>(tok0 + key0));
        if (i >= 2 && !mbar_wait(v_empty + st, ((i - 2) >> 1) & 1, a.err, kErrSmemEmptyTimeout)) break;
        mbar_arrive_expect_tx(v_full + st, kTile);
        for (int c = 0; c < 2; ++c)
          tma_load_2d(sm + kOffV + st * kTile + c * kAtom, &tmV, v_full + st, hk * kHD + c * 64,
                      static_cast<int>(tok0 + key0));
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kBM, kBN, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kBM, kHD, false, true);
      const uint32_t o_tmem = tmem + 256;
      bool ok = mbar_wait(q_full, 0, a.err, kErrTmaFullTimeout);
      auto mma_pv = [&](int t) {
        if (!ok) return;
        ok = mbar_wait(p_full, t & 1, a.err, kErrTmaFullTimeout) &&
             mbar_wait(v_full + (t & 1), (t >> 1) & 1, a.err, kErrTmaFullTimeout);
        if (!ok) return;
        tc_fence_after();
        const uint32_t vbase = sV + (t & 1) * kTile;
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          // A = P (K-major: key atom k / 4, +32 B per 16 keys inside it)
          const uint64_t pd = umma_desc_k_sw128(sP + (k >> 2) * kAtom) + 2 * (k & 3);
          // B = V (MN-major: head-dim atom columns 16 KiB apart, 16-key step = two 8-row groups)
          const uint64_t vd = umma_desc_mn_sw128(vbase + k * 2048, kAtom, 1024);
          umma_bf16(o_tmem, pd, vd, idesc_pv, (t > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(v_empty + (t & 1));
        umma_commit(o_done);
      };
      for (int i = 0; i < n_tiles && ok; ++i) {
        const int st = i & 1;
        ok = mbar_wait(k_full + st, (i >> 1) & 1, a.err, kErrTmaFullTimeout);
        if (ok && i >= 2) ok = mbar_wait(s_free + st, ((i - 2) >> 1) & 1, a.err, kErrTmemEmptyTimeout);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kbase = sK + st * kTile;
#pragma unroll
        for (int k = 0; k < kHD / 16; ++k) {
          const uint64_t qd = umma_desc_k_sw128(sQ + (k >> 2) * kAtom) + 2 * (k & 3);
          const uint64_t kd = umma_desc_k_sw128(kbase + (k >> 2) * kAtom) + 2 * (k & 3);
          umma_bf16(tmem + st * kBN, qd, kd, idesc_qk, k > 0 ? 1u : 0u);
        }
        umma_commit(k_empty + st);
        umma_commit(s_full + st);
        if (i >= 1) mma_pv(i - 1);
      }
      mma_pv(n_tiles - 1);
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    const int half = (warp - 2) >> 2;           // key / head-dim columns [64 half, 64 half + 64)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;          // query row inside the tile (TMEM lane)
    const int qi = q0 + r;
    const bool row_ok = qi >= s0 && qi < s1 && qi < a.S;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t col0 = static_cast<uint32_t>(half * 64);
    const int pair_bar = 1 + quarter;           // named barrier of warps (w, w + 4)
    float* xch = reinterpret_cast<float*>(sm + kOffX);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      const int st = i & 1;
      const int key0 = (j_first + i) * kBN;
      // every key of the tile valid and causal for every row of the CTA: no mask
      // (rows outside the valid range compute values that are never stored)
      const bool interior = key0 >= s0 && key0 + kBN <= s1 && key0 + kBN - 1 <= q0;
      bool got = ok && __all_sync(0xffffffffu, mbar_wait(s_full + st, (i >> 1) & 1, a.err, kErrTmemFullTimeout));
      float s[64];
      float mx = -INFINITY;
      if (got) {
        tc_fence_after();
        tmem_ld32(tmem + lane_off + st * kBN + col0, *reinterpret_cast<float(*)[32]>(s));
        tmem_ld32(tmem + lane_off + st * kBN + col0 + 32, *reinterpret_cast<float(*)[32]>(s + 32));
        tc_fence_before();
        mbar_arrive(s_free + st);
        if (!interior) {
          const int kb = key0 + half * 64;
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const int kj = kb + e;
            if (!(row_ok && kj >= s0 && kj < s1 && kj <= qi)) s[e] = -INFINITY;
          }
        }
        float m4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
        for (int e = 4; e < 64; ++e) m4[e & 3] = fmaxf(m4[e & 3], s[e]);
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      }
      xch[((i & 1) * 2 + half) * kBM + r] = mx;
      ok = pair_and(pair_bar, got);
      if (!ok) break;
      mx = fmaxf(mx, xch[((i & 1) * 2 + (half ^ 1)) * kBM + r]);
      // the log2-domain max is max * scale (scale > 0); both threads of a row
      // take identical decisions from identical inputs
      const float m_new = fmaxf(m, mx * a.scale_log2);
      float alpha = 1.f;
      const bool need = m != -INFINITY && m_new > m + kRescaleLog2;
      if (m == -INFINITY) {
        m = m_new;                               // first finite max: nothing accumulated yet
      } else if (need) {
        alpha = ex2(m - m_new);
        m = m_new;
      }
      const bool rescale = __any_sync(0xffffffffu, need);
      // a row with no valid key so far has m = -inf and only -inf scores: p = 2^-inf = 0
      const float neg_m = m == -INFINITY ? 0.f : -m;
      float p4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int e = 0; e < 64; ++e) {
        s[e] = ex2(fmaf(s[e], a.scale_log2, neg_m));
        p4[e & 3] += s[e];
      }
      l = l * alpha + ((p4[0] + p4[1]) + (p4[2] + p4[3]));
      // P(i) overwrites P(i-1) and O may be rescaled: O += P(i-1) V(i-1) must be done
      bool ready = true;
      if (i >= 1) {
        ready = __all_sync(0xffffffffu, mbar_wait(o_done, (i - 1) & 1, a.err, kErrTmemFullTimeout));
        tc_fence_after();
      }
      if (!ready) {
        ok = false;                              // reported at the next pair barrier (or the epilogue's)
        continue;
      }
      if (rescale && i >= 1) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v[32];
          tmem_ld32(tmem + lane_off + 256 + col0 + c * 32, v);
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] *= alpha;
          tmem_st32(tmem + lane_off + 256 + col0 + c * 32, v);
        }
        tmem_wait_st();
      }
      // this thread's 64 keys are atom column `half` of the K-major P tile
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t addr = sP + half * kAtom + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4);
        const uint32_t w0 = pack2(s[c * 8 + 0], s[c * 8 + 1]), w1 = pack2(s[c * 8 + 2], s[c * 8 + 3]);
        const uint32_t w2 = pack2(s[c * 8 + 4], s[c * 8 + 5]), w3 = pack2(s[c * 8 + 6], s[c * 8 + 7]);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                     : "memory");
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // ---- epilogue: O / l -> bf16, log-sum-exp (the pair adds its partial sums)
    bool got = ok;
    if (n_tiles > 0 && got) {
      got = __all_sync(0xffffffffu, mbar_wait(o_done, (n_tiles - 1) & 1, a.err, kErrTmemFullTimeout));
      tc_fence_after();
    }
    xch[((n_tiles & 1) * 2 + half) * kBM + r] = l;
    got = pair_and(pair_bar, got);
    const float l_tot = l + xch[((n_tiles & 1) * 2 + (half ^ 1)) * kBM + r];
    const bool valid = row_ok && n_tiles > 0 && got && l_tot > 0.f;
    const float inv = valid ? 1.f / l_tot : 0.f;
    __nv_bfloat16* orow = a.o + ((tok0 + min(qi, a.S - 1)) * a.nq + h) * kHD + col0;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float v[32];
      if (n_tiles > 0 && got) {
        tmem_ld32(tmem + lane_off + 256 + col0 + c * 32, v);   // every lane of the warp takes part
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
      }
      if (qi < a.S) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint4 pkt;
          pkt.x = pack2(valid ? v[q4 * 8 + 0] * inv : 0.f, valid ? v[q4 * 8 + 1] * inv : 0.f);
          pkt.y = pack2(valid ? v[q4 * 8 + 2] * inv : 0.f, valid ? v[q4 * 8 + 3] * inv : 0.f);
          pkt.z = pack2(valid ? v[q4 * 8 + 4] * inv : 0.f, valid ? v[q4 * 8 + 5] * inv : 0.f);
          pkt.w = pack2(valid ? v[q4 * 8 + 6] * inv : 0.f, valid ? v[q4 * 8 + 7] * inv : 0.f);
          *reinterpret_cast<uint4*>(orow + c * 32 + q4 * 8) = pkt;
        }
      }
    }
    if (qi < a.S && half == 0) a.lse[(tok0 + qi) * a.nq + h] = valid ? m + log2f(l_tot) : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

void flash_attn_fwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                       torch::Tensor start, torch::Tensor end, int64_t B, int64_t S, double scale, torch::Tensor err) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && out.is_contiguous(), "contiguous inputs");
  TORCH_CHECK(q.size(-1) == kHD && q.scalar_type() == torch::kBFloat16, "bf16 q/k/v with head_dim 128");
  const long T = q.size(0);
  const int nq = static_cast<int>(q.size(1)), nkv = static_cast<int>(k.size(1));
  FwdTcArgs a{};
  a.o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.start = start.data_ptr<int>();
  a.end = end.data_ptr<int>();
  a.S = static_cast<int>(S);
  a.nq = nq;
  a.nkv = nkv;
  a.scale_log2 = static_cast<float>(scale) * 1.4426950408889634f;
  a.err = err.data_ptr<int>();
  CUtensorMap tq = make_tmap_bf16(q.data_ptr(), T, static_cast<long>(nq) * kHD, static_cast<long>(nq) * kHD, kBM);
  CUtensorMap tk = make_tmap_bf16(k.data_ptr(), T, static_cast<long>(nkv) * kHD, static_cast<long>(nkv) * kHD, kBN);
  CUtensorMap tv = make_tmap_bf16(v.data_ptr(), T, static_cast<long>(nkv) * kHD, static_cast<long>(nkv) * kHD, kBN);
  static bool configured[64] = {};
  const int dev = q.get_device();
  if (!configured[dev]) {
    cudaFuncSetAttribute(flash_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    configured[dev] = true;
  }
  dim3 grid(static_cast<unsigned>((S + kBM - 1) / kBM), static_cast<unsigned>(nq), static_cast<unsigned>(B));
  flash_fwd_tc_kernel<<<grid, kThreads, kSmem, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


// ===========================================================================
// Flash attention backward on tcgen05.
//
// CTA = one tile of 128 keys of one KV head; it walks every (query head of the
// GQA group, 128-query tile) pair j that can see those keys and accumulates
// dK and dV in TMEM.  Products (rows = TMEM lanes):
//   S^T_j  = K Q_j^T            [keys x queries]   TMEM cols [0, 128)
//   dP^T_j = V dO_j^T           [keys x queries]   same columns, after S^T_j is read
//   P^T = 2^(S^T * scale - lse_q), dS^T = scale * P^T (dP^T - delta_q)  (registers,
//         two threads per key row, 64 query columns each; written to shared
//         memory as bf16 128B-swizzled K-major tiles)
//   dV += P^T dO_j             cols [256, 384)   (dO read MN-major)
//   dK += dS^T Q_j             cols [384, 512)   (Q read MN-major)
//   dQ_j = dS K                cols [128, 256)   (the dS^T tile read MN-major is dS;
//                                                 K read MN-major), then added to
//                                                 the fp32 dQ buffer with vector
//                                                 atomics by the softmax warps.
// Warp 0: TMA (K, V once; Q_j + lse_j and dO_j + delta_j per step); warp 1: TMEM
// owner and MMA issuer; warps 2-9: elementwise work, dQ drain and the dK / dV
// epilogue.  lse and delta arrive as [B * nq, S_pad] rows (bulk copies of 512 B).
// Every wait is bounded.
// ===========================================================================
namespace {

constexpr int kBOffK = 0;
constexpr int kBOffV = kBOffK + kTile;
constexpr int kBOffQ = kBOffV + kTile;        // 2 buffers: Q_{j+1} loads while step j runs
constexpr int kBOffDO = kBOffQ + 2 * kTile;
constexpr int kBOffP = kBOffDO + kTile;
constexpr int kBOffDS = kBOffP + kTile;
constexpr int kBOffLse = kBOffDS + kTile;     // 2 x 128 fp32 (with the Q buffers)
constexpr int kBOffDel = kBOffLse + 1024;     // 128 fp32
constexpr int kBOffBar = kBOffDel + 512;
constexpr int kBSmem = kBOffBar + 256 + 1024;
static_assert(kBSmem <= 227 * 1024, "backward shared memory budget");

struct BwdTcArgs {
  const float *lse_t, *delta_t;   // [B * nq, S_pad]
  float* dq;                      // fp32 [T, nq, 128], accumulated
  __nv_bfloat16 *dk, *dv;         // [T, nkv, 128]
  const int *start, *end;
  int S, S_pad, nq, nkv;
  float scale_log2, scale;
  int* err;
};

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    flash_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        BwdTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* sm = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kBOffBar);
  uint64_t* kv_full = bar + 0;
  uint64_t* q_full = bar + 1;     // [2]
  uint64_t* q_empty = bar + 3;    // [2]
  uint64_t* do_full = bar + 5;
  uint64_t* do_empty = bar + 6;
  uint64_t* s_full = bar + 7;
  uint64_t* s_loaded = bar + 8;
  uint64_t* dp_full = bar + 9;
  uint64_t* dp_loaded = bar + 10;
  uint64_t* ds_ready = bar + 11;
  uint64_t* dq_full = bar + 12;
  uint64_t* dq_free = bar + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 14);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.nq / a.nkv;
  const int k0 = kb * kBN;
  const int s0 = a.start[b], s1 = a.end[b];
  const long tok0 = static_cast<long>(b) * a.S;
  // query tiles that can see a key of this tile (queries >= keys, both in [s0, s1))
  const bool live = k0 < s1 && k0 + kBN > s0;
  const int qt_first = max(kb, s0 / kBM);
  const int qt_last = live ? (s1 - 1) / kBM : qt_first - 1;
  const int n_qt = max(0, qt_last - qt_first + 1);
  const int n_steps = G * n_qt;                 // j = head_in_group * n_qt + (qt - qt_first)

  if (threadIdx.x == 0) {
    for (int i = 0; i < 14; ++i) mbar_init(bar + i, 1);
    mbar_init(s_loaded, kSoftmaxThreads);
    mbar_init(dp_loaded, kSoftmaxThreads);
    mbar_init(ds_ready, kSoftmaxThreads);
    mbar_init(dq_free, kSoftmaxThreads);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sK = smem_addr(sm + kBOffK), sV = smem_addr(sm + kBOffV), sQ = smem_addr(sm + kBOffQ),
                 sDO = smem_addr(sm + kBOffDO), sP = smem_addr(sm + kBOffP), sDS = smem_addr(sm + kBOffDS);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && n_steps > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(kv_full, 2 * kTile);
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(sm + kBOffK + c * kAtom, &tmK, kv_full, hk * kHD + c * 64, static_cast<int>(tok0 + k0));
        tma_load_2d(sm + kBOffV + c * kAtom, &tmV, kv_full, hk * kHD + c * 64, static_cast<int>(tok0 + k0));
      }
      for (int j = 0; j < n_steps; ++j) {
        const int h = hk * G + j / n_qt;
        const int q0 = (qt_first + j % n_qt) * kBM;
        const long vec = (static_cast<long>(b) * a.nq + h) * a.S_pad + q0;
        const int qs = j & 1;
        if (j >= 2 && !mbar_wait(q_empty + qs, ((j - 2) >> 1) & 1, a.err, kErrSmemEmptyTimeout)) break;
        mbar_arrive_expect_tx(q_full + qs, kTile + 512);
        for (int c = 0; c < 2; ++c)
          tma_load_2d(sm + kBOffQ + qs * kTile + c * kAtom, &tmQ, q_full + qs, h * kHD + c * 64,
                      static_cast<int>(tok0 + q0));
        bulk_load(smem_addr(sm + kBOffLse + qs * 512), a.lse_t + vec, 512, q_full + qs);
        if (j >= 1 && !mbar_wait(do_empty, (j - 1) & 1, a.err, kErrSmemEmptyTimeout)) break;
        mbar_arrive_expect_tx(do_full, kTile + 512);
        for (int c = 0; c < 2; ++c)
          tma_load_2d(sm + kBOffDO + c * kAtom, &tmDO, do_full, h * kHD + c * 64, static_cast<int>(tok0 + q0));
        bulk_load(smem_addr(sm + kBOffDel), a.delta_t + vec, 512, do_full);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_steps > 0) {
      constexpr uint32_t id_kk = umma_idesc_bf16(kBN, kBM, false, false);   // S^T, dP^T
      constexpr uint32_t id_kmn = umma_idesc_bf16(kBN, kHD, false, true);   // dV, dK: B MN-major
      constexpr uint32_t id_mnmn = umma_idesc_bf16(kBM, kHD, true, true);   // dQ: A and B MN-major
      const uint32_t t_sd = tmem, t_dq = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 384;
      bool ok = mbar_wait(kv_full, 0, a.err, kErrTmaFullTimeout);
      for (int j = 0; j < n_steps && ok; ++j) {
        const uint32_t par = j & 1;
        const uint32_t sQj = sQ + (j & 1) * kTile;
        ok = mbar_wait(q_full + (j & 1), (j >> 1) & 1, a.err, kErrTmaFullTimeout);
        if (ok && j >= 1) ok = mbar_wait(dp_loaded, par ^ 1u, a.err, kErrTmemEmptyTimeout);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kHD / 16; ++k) {
          const uint64_t ad = umma_desc_k_sw128(sK + (k >> 2) * kAtom) + 2 * (k & 3);
          const uint64_t bd = umma_desc_k_sw128(sQj + (k >> 2) * kAtom) + 2 * (k & 3);
          umma_bf16(t_sd, ad, bd, id_kk, k > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        ok = mbar_wait(do_full, par, a.err, kErrTmaFullTimeout) &&
             mbar_wait(s_loaded, par, a.err, kErrTmemEmptyTimeout);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kHD / 16; ++k) {
          const uint64_t ad = umma_desc_k_sw128(sV + (k >> 2) * kAtom) + 2 * (k & 3);
          const uint64_t bd = umma_desc_k_sw128(sDO + (k >> 2) * kAtom) + 2 * (k & 3);
          umma_bf16(t_sd, ad, bd, id_kk, k > 0 ? 1u : 0u);
        }
        umma_commit(dp_full);
        ok = mbar_wait(ds_ready, par, a.err, kErrTmaFullTimeout);
        if (!ok) break;
        tc_fence_after();
        // dV += P^T dO  (K = queries: 16 per step, +32 B in the K-major P^T row, two 8-row groups down dO)
#pragma unroll
        for (int k = 0; k < kBM / 16; ++k) {
          const uint64_t ad = umma_desc_k_sw128(sP + (k >> 2) * kAtom) + 2 * (k & 3);
          const uint64_t bd = umma_desc_mn_sw128(sDO + k * 2048, kAtom, 1024);
          umma_bf16(t_dv, ad, bd, id_kmn, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(do_empty);
        // dK += dS^T Q
#pragma unroll
        for (int k = 0; k < kBM / 16; ++k) {
          const uint64_t ad = umma_desc_k_sw128(sDS + (k >> 2) * kAtom) + 2 * (k & 3);
          const uint64_t bd = umma_desc_mn_sw128(sQj + k * 2048, kAtom, 1024);
          umma_bf16(t_dk, ad, bd, id_kmn, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(q_empty + (j & 1));
        // dQ_j = dS K  (K = keys: the dS^T tile read MN-major, K read MN-major)
        if (j >= 1) ok = mbar_wait(dq_free, par ^ 1u, a.err, kErrTmemEmptyTimeout);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          const uint64_t ad = umma_desc_mn_sw128(sDS + k * 2048, kAtom, 1024);
          const uint64_t bd = umma_desc_mn_sw128(sK + k * 2048, kAtom, 1024);
          umma_bf16(t_dq, ad, bd, id_mnmn, k > 0 ? 1u : 0u);
        }
        umma_commit(dq_full);
      }
    }
  } else {
    // ------------------------------------------------------------ elementwise / drains / epilogue
    const int half = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;          // TMEM lane: key row (S^T, dP^T, dK, dV) or query row (dQ)
    const int kr = k0 + r;
    const bool key_ok = kr >= s0 && kr < s1;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t col0 = static_cast<uint32_t>(half * 64);
    const float* lse_s = reinterpret_cast<const float*>(sm + kBOffLse) + half * 64;
    const float* del_s = reinterpret_cast<const float*>(sm + kBOffDel) + half * 64;
    bool ok = true;
    for (int j = 0; j < n_steps && ok; ++j) {
      const uint32_t par = j & 1;
      const int h = hk * G + j / n_qt;
      const int q0 = (qt_first + j % n_qt) * kBM;
      const bool interior = k0 >= s0 && q0 >= s0 && q0 + kBM <= s1 && q0 >= k0 + kBN - 1;
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, par, a.err, kErrTmemFullTimeout) &&
                                       mbar_wait(q_full + (j & 1), (j >> 1) & 1, a.err, kErrTmaFullTimeout));
      const float* lse_j = lse_s + (j & 1) * 128;
      if (!ok) break;
      tc_fence_after();
      float p[64];
      tmem_ld32(tmem + lane_off + col0, *reinterpret_cast<float(*)[32]>(p));
      tmem_ld32(tmem + lane_off + col0 + 32, *reinterpret_cast<float(*)[32]>(p + 32));
      tc_fence_before();
      mbar_arrive(s_loaded);
      const int qc = q0 + half * 64;            // first query column of this thread
#pragma unroll
      for (int e = 0; e < 64; ++e) {
        const float v = ex2(fmaf(p[e], a.scale_log2, -lse_j[e]));
        const int qq = qc + e;
        p[e] = (interior || (key_ok && qq >= kr && qq < s1)) ? v : 0.f;
      }
      ok = __all_sync(0xffffffffu, mbar_wait(dp_full, par, a.err, kErrTmemFullTimeout) &&
                                       mbar_wait(do_full, par, a.err, kErrTmaFullTimeout));
      if (!ok) break;
      tc_fence_after();
      float d[64];
      tmem_ld32(tmem + lane_off + col0, *reinterpret_cast<float(*)[32]>(d));
      tmem_ld32(tmem + lane_off + col0 + 32, *reinterpret_cast<float(*)[32]>(d + 32));
      tc_fence_before();
      mbar_arrive(dp_loaded);
#pragma unroll
      for (int e = 0; e < 64; ++e) d[e] = p[e] != 0.f ? p[e] * (d[e] - del_s[e]) * a.scale : 0.f;
      // P^T and dS^T rows: this thread's 64 queries are atom column `half`
      // (the previous step's MMAs finished reading both tiles: dq_full(j - 1) was awaited)
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t off = half * kAtom + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(sP + off),
                     "r"(pack2(p[c * 8 + 0], p[c * 8 + 1])), "r"(pack2(p[c * 8 + 2], p[c * 8 + 3])),
                     "r"(pack2(p[c * 8 + 4], p[c * 8 + 5])), "r"(pack2(p[c * 8 + 6], p[c * 8 + 7]))
                     : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(sDS + off),
                     "r"(pack2(d[c * 8 + 0], d[c * 8 + 1])), "r"(pack2(d[c * 8 + 2], d[c * 8 + 3])),
                     "r"(pack2(d[c * 8 + 4], d[c * 8 + 5])), "r"(pack2(d[c * 8 + 6], d[c * 8 + 7]))
                     : "memory");
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(ds_ready);
      // dQ_j rows (lane = query row): add into the fp32 buffer
      ok = __all_sync(0xffffffffu, mbar_wait(dq_full, par, a.err, kErrTmemFullTimeout));
      if (!ok) break;
      tc_fence_after();
      const int qr = q0 + r;
      const bool q_ok = qr >= s0 && qr < s1;
      float* dst = a.dq + ((tok0 + min(qr, a.S - 1)) * a.nq + h) * kHD + col0;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v[32];
        tmem_ld32(tmem + lane_off + 128 + col0 + c * 32, v);
        if (q_ok) {
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4)
            red_add_v4(dst + c * 32 + q4 * 4, v[q4 * 4 + 0], v[q4 * 4 + 1], v[q4 * 4 + 2], v[q4 * 4 + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(dq_free);
    }
    // ---- epilogue: dK, dV rows (zero where the key is outside the valid range);
    // the TMEM loads are warp-uniform, only the stores depend on the row
    const bool have = n_steps > 0 && ok;
    const bool keep = have && key_ok;
    const long row = (tok0 + min(kr, a.S - 1)) * a.nkv + hk;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      __nv_bfloat16* out = (which == 0 ? a.dv : a.dk) + row * kHD + col0;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v[32];
        if (have) {
          tmem_ld32(tmem + lane_off + (which == 0 ? 256 : 384) + col0 + c * 32, v);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = 0.f;
        }
        if (kr < a.S) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 pkt;
            pkt.x = pack2(keep ? v[q4 * 8 + 0] : 0.f, keep ? v[q4 * 8 + 1] : 0.f);
            pkt.y = pack2(keep ? v[q4 * 8 + 2] : 0.f, keep ? v[q4 * 8 + 3] : 0.f);
            pkt.z = pack2(keep ? v[q4 * 8 + 4] : 0.f, keep ? v[q4 * 8 + 5] : 0.f);
            pkt.w = pack2(keep ? v[q4 * 8 + 6] : 0.f, keep ? v[q4 * 8 + 7] : 0.f);
            *reinterpret_cast<uint4*>(out + c * 32 + q4 * 8) = pkt;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// delta[b, h, s] = sum_d dO * O and lse copied into [B * nq, S_pad] rows (one warp per (t, h))
__global__ void flash_bwd_tc_pre_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                        const float* __restrict__ lse, float* __restrict__ delta_t,
                                        float* __restrict__ lse_t, long n_rows, int nq, int S, int S_pad) {
  const long w = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= n_rows) return;
  const uint2 ov = *reinterpret_cast<const uint2*>(o + w * kHD + lane * 4);
  const uint2 dv = *reinterpret_cast<const uint2*>(dout + w * kHD + lane * 4);
  const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&ov);
  const __nv_bfloat16* db = reinterpret_cast<const __nv_bfloat16*>(&dv);
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) s += __bfloat162float(ob[e]) * __bfloat162float(db[e]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) {
    const long t = w / nq;
    const int h = static_cast<int>(w - t * nq);
    const long b = t / S, pos = t - b * S;
    const long dst = (b * nq + h) * S_pad + pos;
    delta_t[dst] = s;
    lse_t[dst] = lse[w];
  }
}

__global__ void dq_to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, long n) {
  const long i = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(src + i);
    uint2 out;
    out.x = pack2(v.x, v.y);
    out.y = pack2(v.z, v.w);
    *reinterpret_cast<uint2*>(dst + i) = out;
  } else {
    for (long k = i; k < n; ++k) dst[k] = __float2bfloat16(src[k]);
  }
}

}  // namespace

void flash_attn_bwd_tc(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out,
                       torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor start,
                       torch::Tensor end, int64_t B, int64_t S, double scale, torch::Tensor err) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(dout.is_contiguous() && q.is_contiguous() && k.is_contiguous() && v.is_contiguous() &&
                  out.is_contiguous() && lse.is_contiguous(), "contiguous inputs");
  TORCH_CHECK(q.size(-1) == kHD && q.scalar_type() == torch::kBFloat16, "bf16 q/k/v with head_dim 128");
  const long T = q.size(0);
  TORCH_CHECK(T == B * S, "q must hold B * S tokens");
  const int nq = static_cast<int>(q.size(1)), nkv = static_cast<int>(k.size(1));
  TORCH_CHECK(nq % nkv == 0, "query heads must be a multiple of KV heads");
  auto stream = at::cuda::getCurrentCUDAStream();
  auto opts = q.options().dtype(torch::kFloat32);
  const int S_pad = static_cast<int>((S + kBM - 1) / kBM * kBM);
  // padding columns (positions >= S) are read by boundary tiles and masked: keep them finite
  torch::Tensor delta_t = torch::zeros({B * nq, S_pad}, opts);
  torch::Tensor lse_t = torch::zeros({B * nq, S_pad}, opts);
  torch::Tensor dq32 = torch::zeros({T, nq, kHD}, opts);
  const long rows = T * nq;
  flash_bwd_tc_pre_kernel<<<(rows * 32 + 255) / 256, 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      lse.data_ptr<float>(), delta_t.data_ptr<float>(), lse_t.data_ptr<float>(), rows, nq, static_cast<int>(S), S_pad);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  BwdTcArgs a{};
  a.lse_t = lse_t.data_ptr<float>();
  a.delta_t = delta_t.data_ptr<float>();
  a.dq = dq32.data_ptr<float>();
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  a.start = start.data_ptr<int>();
  a.end = end.data_ptr<int>();
  a.S = static_cast<int>(S);
  a.S_pad = S_pad;
  a.nq = nq;
  a.nkv = nkv;
  a.scale = static_cast<float>(scale);
  a.scale_log2 = static_cast<float>(scale) * 1.4426950408889634f;
  a.err = err.data_ptr<int>();
  CUtensorMap tq = make_tmap_bf16(q.data_ptr(), T, static_cast<long>(nq) * kHD, static_cast<long>(nq) * kHD, kBM);
  CUtensorMap tdo = make_tmap_bf16(dout.data_ptr(), T, static_cast<long>(nq) * kHD, static_cast<long>(nq) * kHD, kBM);
  CUtensorMap tk = make_tmap_bf16(k.data_ptr(), T, static_cast<long>(nkv) * kHD, static_cast<long>(nkv) * kHD, kBN);
  CUtensorMap tv = make_tmap_bf16(v.data_ptr(), T, static_cast<long>(nkv) * kHD, static_cast<long>(nkv) * kHD, kBN);
  static bool configured[64] = {};
  const int dev = q.get_device();
  if (!configured[dev]) {
    cudaFuncSetAttribute(flash_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBSmem);
    configured[dev] = true;
  }
  dim3 grid(static_cast<unsigned>(S_pad / kBN), static_cast<unsigned>(nkv), static_cast<unsigned>(B));
  flash_bwd_tc_kernel<<<grid, kThreads, kBSmem, stream>>>(tq, tk, tv, tdo, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const long n = dq32.numel();
  dq_to_bf16_kernel<<<(n / 4 + 255) / 256 + 1, 256, 0, stream>>>(dq32.data_ptr<float>(),
                                                                  reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace gb
