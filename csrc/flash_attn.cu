// Flash attention for prefill and training (forward + backward), head_dim 128.
// Reference counterpart: SDPA with a boolean mask (src/graspo/backends/graspoflow/models/
// common/layers_qwen3.py:252-257); this mma.sync version is the fallback of csrc/flash_attn_tc.cu.
//
// Layout: q [T, nq, 128], k / v [T, nkv, 128] bf16 with T = B * S tokens of a
// padded batch.  Row b's valid tokens are the contiguous range
// [start[b], end[b]) (left padding before the prompt, right padding after
// EOS); query i attends to keys j with start <= j <= i.  Queries outside the
// valid range produce zeros and take no part in the backward pass.
//
// Forward (Dao, "FlashAttention-2", 2023; written here for this layout):
// CTA = (64 query rows, q head, batch row), 4 warps x 16 rows.  K/V tiles of
// 64 keys are streamed by cp.async into XOR-swizzled shared memory (double
// buffered); S = Q K^T and O += P V run on mma.sync.m16n8k16 (bf16 in, fp32
// accumulate) with P reused from registers; online softmax in the log2
// domain.  Writes O (bf16) and the row log-sum-exp (log2 domain, fp32).
//
// Backward: CTA = (64 keys, kv head, batch row), looping over the G query
// heads of the KV head and the query blocks at or after the key block.  Each
// warp owns 16 keys and accumulates their dK / dV in registers:
//   S^T = K Q^T, P^T = exp2(S^T - lse), dV += P^T dO, dP^T = V dO^T,
//   dS^T = P^T * (dP^T - D), dK += dS^T Q,
// dS^T goes through shared memory so that dQ += dS K is computed per query
// row block and accumulated with fp32 atomics.  D = rowsum(dO * O) comes from
// a small pre-pass.

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "sm100_common.cuh"

namespace gb {
namespace {

constexpr int kD = 128;
constexpr int kBlk = 64;
constexpr int kRowB = kD * 2;          // bytes per row
constexpr int kTileB = kBlk * kRowB;   // 16 KiB
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * kRowB + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void ldsm4(uint32_t a, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm4t(uint32_t a, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pk(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Copy rows [r0, r0 + 64) of one head (row stride `ld` elements) into a
// swizzled tile; rows beyond `rows_valid` are zero-filled.
__device__ __forceinline__ void load_tile(uint32_t dst, const __nv_bfloat16* base, long ld, int r0, int rows_valid) {
#pragma unroll
  for (int i = 0; i < (kTileB / 16) / 128; ++i) {
    const int id = threadIdx.x + i * 128;
    const int r = id >> 4, ch = id & 15;
    if (r0 + r < rows_valid) {
      cp16(dst + swz(r, ch), base + static_cast<long>(r0 + r) * ld + ch * 8);
    } else {
      asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(dst + swz(r, ch)), "r"(0u) : "memory");
    }
  }
}

struct FwdArgs {
  const __nv_bfloat16 *q, *k, *v;
  __nv_bfloat16* o;
  float* lse;  // [T, nq] log2-domain
  const int *start, *end;
  int S, nq, nkv;
  float scale_log2;
};

__global__ void __launch_bounds__(128) flash_fwd_kernel(FwdArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int G = a.nq / a.nkv, hk = h / G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = (lane & 3) * 2;
  const int s0 = a.start[b], s1 = a.end[b];
  const int q0 = qb * kBlk;
  const long ldq = static_cast<long>(a.nq) * kD, ldk = static_cast<long>(a.nkv) * kD;
  const __nv_bfloat16* qbase = a.q + (static_cast<long>(b) * a.S) * ldq + h * kD;
  const __nv_bfloat16* kbase = a.k + (static_cast<long>(b) * a.S) * ldk + hk * kD;
  const __nv_bfloat16* vbase = a.v + (static_cast<long>(b) * a.S) * ldk + hk * kD;
  const uint32_t sq = smem_addr(sm), skv = sq + kTileB;  // then 2 stages x (K, V)

  const int row_lo = q0 + warp * 16;  // this warp's first query row
  // queries of this CTA that can have keys
  const int q_last = min(q0 + kBlk, s1) - 1;
  const bool any = (q_last >= s0) && (q0 < s1);
  int kb_first = s0 / kBlk, kb_last = any ? q_last / kBlk : -1;

  load_tile(sq, qbase, ldq, q0, a.S);
  cp_commit();
  if (any) {
    load_tile(skv, kbase, ldk, kb_first * kBlk, a.S);
    load_tile(skv + kTileB, vbase, ldk, kb_first * kBlk, a.S);
  }
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  uint32_t qf[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int mi = lane >> 3;
    ldsm4(sq + swz(warp * 16 + (mi & 1) * 8 + (lane & 7), ks * 2 + (mi >> 1)), qf[ks]);
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g, g+8
  const int r0 = row_lo + g, r1 = row_lo + g + 8;

  for (int kb = kb_first; kb <= kb_last; ++kb) {
    const int stage = (kb - kb_first) & 1;
    const uint32_t kt = skv + stage * 2 * kTileB, vt = kt + kTileB;
    if (kb < kb_last) {
      const uint32_t nk = skv + (stage ^ 1) * 2 * kTileB;
      load_tile(nk, kbase, ldk, (kb + 1) * kBlk, a.S);
      load_tile(nk + kTileB, vbase, ldk, (kb + 1) * kBlk, a.S);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of 8-key n-tiles
        const int mi = lane >> 3;
        uint32_t bfr[4];
        ldsm4(kt + swz(np * 16 + (mi >> 1) * 8 + (lane & 7), ks * 2 + (mi & 1)), bfr);
        mma(s[2 * np], qf[ks], bfr[0], bfr[1]);
        mma(s[2 * np + 1], qf[ks], bfr[2], bfr[3]);
      }
    }
    // mask + scale (log2 domain)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = kb * kBlk + n * 8 + c + e;
        const bool kv_ok = j >= s0 && j < s1;
        s[n][e] = (kv_ok && j <= r0) ? s[n][e] * a.scale_log2 : -INFINITY;
        s[n][2 + e] = (kv_ok && j <= r1) ? s[n][2 + e] * a.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, s[n][e]);
        mx1 = fmaxf(mx1, s[n][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float c0 = (n0 == -INFINITY) ? 1.f : exp2f(m0 - n0);
    const float c1 = (n1 == -INFINITY) ? 1.f : exp2f(m1 - n1);
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[n][e] = (n0 == -INFINITY) ? 0.f : exp2f(s[n][e] - n0);
        s[n][2 + e] = (n1 == -INFINITY) ? 0.f : exp2f(s[n][2 + e] - n1);
        ps0 += s[n][e];
        ps1 += s[n][2 + e];
      }
    }
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
    // O += P V: k = keys (4 steps of 16), n = dims (16 tiles of 8)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4] = {pk(s[2 * kk][0], s[2 * kk][1]), pk(s[2 * kk][2], s[2 * kk][3]),
                        pk(s[2 * kk + 1][0], s[2 * kk + 1][1]), pk(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
      for (int nd = 0; nd < 8; ++nd) {
        const int mi = lane >> 3;
        uint32_t bfr[4];
        ldsm4t(vt + swz(kk * 16 + (mi & 1) * 8 + (lane & 7), nd * 2 + (mi >> 1)), bfr);
        mma(o[2 * nd], pa, bfr[0], bfr[1]);
        mma(o[2 * nd + 1], pa, bfr[2], bfr[3]);
      }
    }
    __syncthreads();
  }
  // write O and lse
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const bool ok0 = r0 >= s0 && r0 < s1 && r0 < a.S, ok1 = r1 >= s0 && r1 < s1 && r1 < a.S;
  __nv_bfloat16* obase = a.o + (static_cast<long>(b) * a.S) * ldq + h * kD;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    if (r0 < a.S)
      *reinterpret_cast<uint32_t*>(obase + static_cast<long>(r0) * ldq + n * 8 + c) =
          ok0 ? pk(o[n][0] * inv0, o[n][1] * inv0) : 0u;
    if (r1 < a.S)
      *reinterpret_cast<uint32_t*>(obase + static_cast<long>(r1) * ldq + n * 8 + c) =
          ok1 ? pk(o[n][2] * inv1, o[n][3] * inv1) : 0u;
  }
  if ((lane & 3) == 0) {
    if (r0 < a.S) a.lse[(static_cast<long>(b) * a.S + r0) * a.nq + h] = ok0 ? m0 + log2f(l0) : 0.f;
    if (r1 < a.S) a.lse[(static_cast<long>(b) * a.S + r1) * a.nq + h] = ok1 ? m1 + log2f(l1) : 0.f;
  }
}

// D[t, h] = sum_d dO[t, h, d] * O[t, h, d]   (one warp per (t, h))
__global__ void flash_bwd_pre_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                     float* __restrict__ dvec, long n_rows) {
  const long w = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= n_rows) return;
  const uint2 ov = *reinterpret_cast<const uint2*>(o + w * kD + lane * 4);
  const uint2 dv = *reinterpret_cast<const uint2*>(dout + w * kD + lane * 4);
  const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&ov);
  const __nv_bfloat16* db = reinterpret_cast<const __nv_bfloat16*>(&dv);
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) s += __bfloat162float(ob[e]) * __bfloat162float(db[e]);
  s = warp_sum(s);
  if (lane == 0) dvec[w] = s;
}

struct BwdArgs {
  const __nv_bfloat16 *q, *k, *v, *dout;
  const float *lse, *dvec;  // [T, nq]
  float* dq;                // fp32 [T, nq, 128], accumulated atomically
  __nv_bfloat16 *dk, *dv;   // [T, nkv, 128]
  const int *start, *end;
  int S, nq, nkv;
  float scale_log2, scale;
};

__global__ void __launch_bounds__(128) flash_bwd_kernel(BwdArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int kb = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.nq / a.nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = (lane & 3) * 2;
  const int s0 = a.start[b], s1 = a.end[b];
  const int k0 = kb * kBlk;
  const long ldq = static_cast<long>(a.nq) * kD, ldk = static_cast<long>(a.nkv) * kD;
  const long tok0 = static_cast<long>(b) * a.S;
  // shared: K tile, V tile, 2 x (Q tile, dO tile), dS^T [64 keys x 64 q] bf16
  const uint32_t sk = smem_addr(sm), sv = sk + kTileB;
  const uint32_t sqd = sv + kTileB;          // stage s: Q at sqd + s*2*kTileB, dO at +kTileB
  const uint32_t sds = sqd + 4 * kTileB;     // dS^T, rows = keys, 64 q cols (128 B per row)
  __nv_bfloat16* ds_ptr = reinterpret_cast<__nv_bfloat16*>(sm + 6 * kTileB);

  float dk[16][4], dv[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[n][e] = dv[n][e] = 0.f;

  const bool keys_live = k0 < s1 && k0 + kBlk > s0;
  const int qb_first = k0 / kBlk;            // causal: queries >= keys
  const int qb_last = (s1 - 1) / kBlk;
  if (keys_live) {
    load_tile(sk, a.k + tok0 * ldk + hk * kD, ldk, k0, a.S);
    load_tile(sv, a.v + tok0 * ldk + hk * kD, ldk, k0, a.S);
    cp_commit();
    cp_wait<0>();
    __syncthreads();
  }
  const int key_r0 = k0 + warp * 16 + g, key_r1 = key_r0 + 8;  // rows of the S^T fragments
  const int n_iter = keys_live ? G * (qb_last - qb_first + 1) : 0;
  auto issue = [&](int it, int stage) {
    const int hq = hk * G + it / (qb_last - qb_first + 1);
    const int qb = qb_first + it % (qb_last - qb_first + 1);
    const uint32_t dst = sqd + stage * 2 * kTileB;
    load_tile(dst, a.q + tok0 * ldq + hq * kD, ldq, qb * kBlk, a.S);
    load_tile(dst + kTileB, a.dout + tok0 * ldq + hq * kD, ldq, qb * kBlk, a.S);
    cp_commit();
  };
  if (n_iter > 0) issue(0, 0);
  for (int it = 0; it < n_iter; ++it) {
    const int stage = it & 1;
    const int hq = hk * G + it / (qb_last - qb_first + 1);
    const int qb = qb_first + it % (qb_last - qb_first + 1);
    const int q0 = qb * kBlk;
    if (it + 1 < n_iter) {
      issue(it + 1, stage ^ 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint32_t tq = sqd + stage * 2 * kTileB, tdo = tq + kTileB;
    // S^T [16 keys x 64 q] = K_w Q^T ;  dP^T = V_w dO^T
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[n][e] = dpt[n][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      // this warp's 16 keys as A fragments, re-read from shared memory to keep
      // registers for the dK / dV accumulators
      uint32_t kf[4], vf[4];
      {
        const int mi = lane >> 3;
        ldsm4(sk + swz(warp * 16 + (mi & 1) * 8 + (lane & 7), ks * 2 + (mi >> 1)), kf);
        ldsm4(sv + swz(warp * 16 + (mi & 1) * 8 + (lane & 7), ks * 2 + (mi >> 1)), vf);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int mi = lane >> 3;
        uint32_t bq[4], bo[4];
        ldsm4(tq + swz(np * 16 + (mi >> 1) * 8 + (lane & 7), ks * 2 + (mi & 1)), bq);
        ldsm4(tdo + swz(np * 16 + (mi >> 1) * 8 + (lane & 7), ks * 2 + (mi & 1)), bo);
        mma(st[2 * np], kf, bq[0], bq[1]);
        mma(st[2 * np + 1], kf, bq[2], bq[3]);
        mma(dpt[2 * np], vf, bo[0], bo[1]);
        mma(dpt[2 * np + 1], vf, bo[2], bo[3]);
      }
    }
    // P^T, dS^T (columns = queries)
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int qi = q0 + n * 8 + c + e;
        const bool q_ok = qi >= s0 && qi < s1 && qi < a.S;
        const long li = (tok0 + min(qi, a.S - 1)) * a.nq + hq;
        const float L = a.lse[li], Dq = a.dvec[li];
        const bool ok0 = q_ok && key_r0 >= s0 && key_r0 < s1 && key_r0 <= qi;
        const bool ok1 = q_ok && key_r1 >= s0 && key_r1 < s1 && key_r1 <= qi;
        const float p0 = ok0 ? exp2f(st[n][e] * a.scale_log2 - L) : 0.f;
        const float p1 = ok1 ? exp2f(st[n][2 + e] * a.scale_log2 - L) : 0.f;
        st[n][e] = p0;
        st[n][2 + e] = p1;
        dpt[n][e] = p0 * (dpt[n][e] - Dq) * a.scale;
        dpt[n][2 + e] = p1 * (dpt[n][2 + e] - Dq) * a.scale;
      }
    }
    // dV += P^T dO ; dK += dS^T Q   (k = queries: 4 steps of 16)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t pa[4] = {pk(st[2 * kk][0], st[2 * kk][1]), pk(st[2 * kk][2], st[2 * kk][3]),
                              pk(st[2 * kk + 1][0], st[2 * kk + 1][1]), pk(st[2 * kk + 1][2], st[2 * kk + 1][3])};
      const uint32_t da[4] = {pk(dpt[2 * kk][0], dpt[2 * kk][1]), pk(dpt[2 * kk][2], dpt[2 * kk][3]),
                              pk(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]), pk(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3])};
#pragma unroll
      for (int nd = 0; nd < 8; ++nd) {
        const int mi = lane >> 3;
        uint32_t bo[4], bq[4];
        ldsm4t(tdo + swz(kk * 16 + (mi & 1) * 8 + (lane & 7), nd * 2 + (mi >> 1)), bo);
        ldsm4t(tq + swz(kk * 16 + (mi & 1) * 8 + (lane & 7), nd * 2 + (mi >> 1)), bq);
        mma(dv[2 * nd], pa, bo[0], bo[1]);
        mma(dv[2 * nd + 1], pa, bo[2], bo[3]);
        mma(dk[2 * nd], da, bq[0], bq[1]);
        mma(dk[2 * nd + 1], da, bq[2], bq[3]);
      }
    }
    // dS^T -> shared (rows = keys, 64 query columns, 128 B rows, 16-byte chunks swizzled)
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int kr0 = warp * 16 + g, kr1 = kr0 + 8;
      const int col = n * 8 + c;
      const int ch = col >> 3, within = col & 7;
      *reinterpret_cast<uint32_t*>(ds_ptr + kr0 * 64 + (((ch ^ (kr0 & 7)) << 3) + within)) = pk(dpt[n][0], dpt[n][1]);
      *reinterpret_cast<uint32_t*>(ds_ptr + kr1 * 64 + (((ch ^ (kr1 & 7)) << 3) + within)) = pk(dpt[n][2], dpt[n][3]);
    }
    __syncthreads();
    // dQ[16 q rows of this warp] += dS [q x 64 keys] K [64 keys x 128]
    {
      float dq[16][4];
#pragma unroll
      for (int n = 0; n < 16; ++n) dq[n][0] = dq[n][1] = dq[n][2] = dq[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // keys 16 at a time
        // A = dS (rows = queries warp*16.., k = keys) = transpose of dS^T tile
        uint32_t af[4];
        {
          const int mi = lane >> 3;
          const int key = kk * 16 + (mi >> 1) * 8 + (lane & 7);
          const int qcol_chunk = (warp * 16 + (mi & 1) * 8) >> 3;
          ldsm4t(sds + key * 128 + ((qcol_chunk ^ (key & 7)) << 4), af);
          // ldmatrix.trans of (keys x q) 8x8 blocks gives the (q x keys) A layout:
          // matrices ordered (q 0-7,k 0-7), (q 8-15,k 0-7), (q 0-7,k 8-15), (q 8-15,k 8-15)
        }
#pragma unroll
        for (int nd = 0; nd < 8; ++nd) {
          const int mi = lane >> 3;
          uint32_t bk[4];
          ldsm4t(sk + swz(kk * 16 + (mi & 1) * 8 + (lane & 7), nd * 2 + (mi >> 1)), bk);
          mma(dq[2 * nd], af, bk[0], bk[1]);
          mma(dq[2 * nd + 1], af, bk[2], bk[3]);
        }
      }
      const int qr0 = q0 + warp * 16 + g, qr1 = qr0 + 8;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        if (qr0 < a.S) {
          float* p = a.dq + ((tok0 + qr0) * a.nq + hq) * kD + n * 8 + c;
          atomicAdd(p, dq[n][0]);
          atomicAdd(p + 1, dq[n][1]);
        }
        if (qr1 < a.S) {
          float* p = a.dq + ((tok0 + qr1) * a.nq + hq) * kD + n * 8 + c;
          atomicAdd(p, dq[n][2]);
          atomicAdd(p + 1, dq[n][3]);
        }
      }
    }
    __syncthreads();
  }
  // write dK, dV for this warp's 16 keys
  const int kr0 = k0 + warp * 16 + g, kr1 = kr0 + 8;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    if (kr0 < a.S) {
      const long off = (tok0 + kr0) * ldk + hk * kD + n * 8 + c;
      *reinterpret_cast<uint32_t*>(a.dk + off) = pk(dk[n][0], dk[n][1]);
      *reinterpret_cast<uint32_t*>(a.dv + off) = pk(dv[n][0], dv[n][1]);
    }
    if (kr1 < a.S) {
      const long off = (tok0 + kr1) * ldk + hk * kD + n * 8 + c;
      *reinterpret_cast<uint32_t*>(a.dk + off) = pk(dk[n][2], dk[n][3]);
      *reinterpret_cast<uint32_t*>(a.dv + off) = pk(dv[n][2], dv[n][3]);
    }
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long n) {
  const long i = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(x + i);
    uint2 out;
    out.x = pk(v.x, v.y);
    out.y = pk(v.z, v.w);
    *reinterpret_cast<uint2*>(y + i) = out;
  } else {
    for (long j = i; j < n; ++j) y[j] = __float2bfloat16(x[j]);
  }
}

constexpr int kFwdSmem = 5 * kTileB;             // Q + 2 x (K, V)
constexpr int kBwdSmem = 6 * kTileB + kBlk * 128;  // K, V, 2 x (Q, dO), dS^T

}  // namespace

void flash_attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                    torch::Tensor start, torch::Tensor end, int64_t B, int64_t S, double scale) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && out.is_contiguous(), "contiguous inputs");
  TORCH_CHECK(q.size(-1) == kD, "head_dim must be 128");
  FwdArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.start = start.data_ptr<int>();
  a.end = end.data_ptr<int>();
  a.S = static_cast<int>(S);
  a.nq = static_cast<int>(q.size(1));
  a.nkv = static_cast<int>(k.size(1));
  a.scale_log2 = static_cast<float>(scale) * kLog2e;
  static bool configured[64] = {};
  const int dev = q.get_device();
  if (!configured[dev]) {
    cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem);
    configured[dev] = true;
  }
  dim3 grid((S + kBlk - 1) / kBlk, a.nq, B);
  flash_fwd_kernel<<<grid, 128, kFwdSmem, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void flash_attn_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out,
                    torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor start,
                    torch::Tensor end, int64_t B, int64_t S, double scale) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(dout.is_contiguous() && q.is_contiguous() && out.is_contiguous(), "contiguous inputs");
  const long T = q.size(0);
  const int nq = static_cast<int>(q.size(1)), nkv = static_cast<int>(k.size(1));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto opts = q.options().dtype(torch::kFloat32);
  torch::Tensor dvec = torch::empty({T, nq}, opts);
  torch::Tensor dq32 = torch::zeros({T, nq, kD}, opts);
  const long rows = T * nq;
  flash_bwd_pre_kernel<<<(rows * 32 + 255) / 256, 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      dvec.data_ptr<float>(), rows);
  BwdArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.dvec = dvec.data_ptr<float>();
  a.dq = dq32.data_ptr<float>();
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  a.start = start.data_ptr<int>();
  a.end = end.data_ptr<int>();
  a.S = static_cast<int>(S);
  a.nq = nq;
  a.nkv = nkv;
  a.scale = static_cast<float>(scale);
  a.scale_log2 = static_cast<float>(scale) * kLog2e;
  static bool configured[64] = {};
  const int dev = q.get_device();
  if (!configured[dev]) {
    cudaFuncSetAttribute(flash_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem);
    configured[dev] = true;
  }
  dim3 grid((S + kBlk - 1) / kBlk, nkv, B);
  flash_bwd_kernel<<<grid, 128, kBwdSmem, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const long n = dq32.numel();
  f32_to_bf16_kernel<<<(n / 4 + 255) / 256 + 1, 256, 0, stream>>>(dq32.data_ptr<float>(),
                                                                   reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace gb
