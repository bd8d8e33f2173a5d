// Sampling, log-prob reductions, the GRPO loss, dropout and the fused AdamW.
// Reference counterparts, under src/graspo/backends/graspoflow/ unless noted: sampling
// tensor_utils.py:649-683, selected-token log-prob tensor_utils.py:167-186, GRPO loss
// src/graspo/core/graspo_loss.py:45-63, clip + AdamW models/qwen35_36/training.py:435-441,
// recurrent gated delta rule tensor_utils.py:592-646.
//
// Random numbers come from Philox4x32-10 (Salmon, Moraes, Dror, Shaw:
// "Parallel random numbers: as easy as 1, 2, 3", SC'11), implemented here
// from the paper: counter-based, so a (seed, counter) pair always produces the
// same numbers -- dropout masks are regenerated in the backward pass instead of
// being stored, and sampling inside a replayed CUDA graph draws fresh numbers
// because the counter includes the row's cache slot, which advances every step.
//
// * sample_append   Gumbel-max sampling from logits / T (exact categorical
//                   sampling in one pass; temperature 0 -> argmax), optional
//                   nucleus (top-p) restriction found by bisection on the
//                   probability threshold, then the decode-state update:
//                   record the token, stop rows at EOS, advance slot/pos/len.
// * lse_combine     merge per-tile (max, sum-exp) partials of the LM-head GEMM
//                   into log-sum-exp and selected-token log-probs.
// * grpo_loss       PPO-clip loss with per-sequence masked mean, and its
//                   gradient w.r.t. the token log-probs, in one kernel.
// * dropout         x * mask / (1 - p) with a Philox mask.
// * grad_sumsq / adamw   global grad-norm (sum of squares) and a flat-buffer
//                   AdamW with clipping and non-finite skip decided on device.

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>
#include <cmath>

#include "sm100_common.cuh"

namespace gb {

namespace {

struct U4 {
  uint32_t x, y, z, w;
};

// Philox4x32 with 10 rounds; multipliers and Weyl key increments from the paper.
__device__ __forceinline__ U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;
  constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kM0, c.x), lo0 = kM0 * c.x;
    const uint32_t hi1 = __umulhi(kM1, c.z), lo1 = kM1 * c.z;
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += kW0;
    k1 += kW1;
  }
  return c;
}

// uniform in the open interval (0, 1)
__device__ __forceinline__ float u01(uint32_t x) {
  return (static_cast<float>(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ float gumbel(uint32_t x) { return -logf(-logf(u01(x))); }

struct ArgMax {
  float v;
  int i;
};

__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ ArgMax block_argmax(ArgMax a) {
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax other{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
    a = better(a, other);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) {
    sv[warp] = a.v;
    si[warp] = a.i;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    ArgMax b{lane < nw ? sv[lane] : -INFINITY, lane < nw ? si[lane] : 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax other{__shfl_xor_sync(0xffffffffu, b.v, o), __shfl_xor_sync(0xffffffffu, b.i, o)};
      b = better(b, other);
    }
    if (lane == 0) {
      sv[0] = b.v;
      si[0] = b.i;
    }
  }
  __syncthreads();
  return ArgMax{sv[0], si[0]};
}

__device__ float block_reduce_sum(float v) {
  __shared__ float s[32];
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) s[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = threadIdx.x < nw ? s[threadIdx.x] : 0.f;
  if (warp == 0) t = warp_sum(t);
  if (threadIdx.x == 0) s[0] = t;
  __syncthreads();
  return s[0];
}

__device__ float block_reduce_max(float v) {
  __shared__ float s[32];
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) s[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = threadIdx.x < nw ? s[threadIdx.x] : -INFINITY;
  if (warp == 0) t = warp_max(t);
  if (threadIdx.x == 0) s[0] = t;
  __syncthreads();
  return s[0];
}

struct SampleArgs {
  const float* logits;  // [rows, V]
  long ld;
  int V;
  float inv_temp;       // 0 => greedy
  float top_p;          // >= 1 => no nucleus restriction
  uint32_t seed_lo, seed_hi;
  // decode state
  int64_t* next_ids;    // [rows]
  int64_t* slot;        // [rows] cache slot of the token just processed
  int64_t* pos;         // [rows]
  int* kv_len;          // [rows]
  uint8_t* finished;    // [rows]
  int64_t* out_tokens;  // [rows, max_new]
  int max_new;
  int64_t prompt_slots; // P: generated token j sits at slot P + j
  int64_t eos_id, pad_id;
  int ignore_eos;
  const uint8_t* active; // optional [rows] mask of rows still generating
};

__global__ void sample_append_kernel(SampleArgs a) {
  const int row = blockIdx.x;
  pdl_trigger();
  pdl_wait();
  const float* lg = a.logits + static_cast<long>(row) * a.ld;
  const int64_t slot = a.slot[row];
  float thresh = -INFINITY;  // in units of logit/T
  if (a.inv_temp > 0.f && a.top_p < 1.f) {
    float mx = -INFINITY;
    for (int v = threadIdx.x; v < a.V; v += blockDim.x) mx = fmaxf(mx, lg[v] * a.inv_temp);
    mx = block_reduce_max(mx);
    float z = 0.f;
    for (int v = threadIdx.x; v < a.V; v += blockDim.x) z += __expf(lg[v] * a.inv_temp - mx);
    z = block_reduce_sum(z);
    // largest s with mass(x >= s) >= top_p, by bisection on s in [mx - 60, mx]
    float lo = mx - 60.f, hi = mx;
    for (int it = 0; it < 32; ++it) {
      const float mid = 0.5f * (lo + hi);
      float mass = 0.f;
      for (int v = threadIdx.x; v < a.V; v += blockDim.x) {
        const float x = lg[v] * a.inv_temp;
        if (x >= mid) mass += __expf(x - mx);
      }
      mass = block_reduce_sum(mass) / z;
      if (mass >= a.top_p) lo = mid; else hi = mid;
    }
    thresh = lo;
  }
  ArgMax best{-INFINITY, 0x7fffffff};
  const int n4 = (a.V + 3) / 4;
  for (int q = threadIdx.x; q < n4; q += blockDim.x) {
    U4 r{0, 0, 0, 0};
    if (a.inv_temp > 0.f) {
      r = philox4x32_10(U4{static_cast<uint32_t>(q), static_cast<uint32_t>(slot),
                           static_cast<uint32_t>(row), 0x5A3F1u},
                        a.seed_lo, a.seed_hi);
    }
    const uint32_t bits[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int v = q * 4 + e;
      if (v >= a.V) break;
      float key;
      if (a.inv_temp > 0.f) {
        const float x = lg[v] * a.inv_temp;
        if (x < thresh) continue;
        key = x + gumbel(bits[e]);
      } else {
        key = lg[v];
      }
      best = better(best, ArgMax{key, v});
    }
  }
  best = block_argmax(best);
  if (threadIdx.x == 0) {
    const bool live = (a.active == nullptr || a.active[row]) && !a.finished[row];
    int64_t tok = live ? static_cast<int64_t>(best.i) : a.pad_id;
    const int64_t col = slot + 1 - a.prompt_slots;
    if (col >= 0 && col < a.max_new) a.out_tokens[static_cast<long>(row) * a.max_new + col] = tok;
    if (live && !a.ignore_eos && tok == a.eos_id) a.finished[row] = 1;
    a.next_ids[row] = tok;
    a.slot[row] = slot + 1;
    a.pos[row] = a.pos[row] + 1;
    a.kv_len[row] = static_cast<int>(slot + 2);
  }
}

// ---------------------------------------------------------------------------
// Split sampler (top-p = 1): the vocabulary of each row is cut into chunks, one
// CTA per (chunk, row) draws the same Gumbel noise as sample_append (Philox
// counter = global vocabulary index / 4, the row's cache slot and the row) and
// keeps its chunk's best (key, index); the CTA that completes a row (arrival
// counter) takes the best chunk.  With one vocabulary shard it then updates the
// decode state; with several (vocab-parallel LM head), it stores the shard's
// winner into every rank's exchange slot over NVLink and signals the peers, and
// sample_exchange_kernel picks the best of all shards -- the same token on
// every rank, without gathering the logits.
struct SplitSampleArgs {
  SampleArgs s;           // logits = this shard's [rows, V_local], V = V_local
  int vocab_start;        // global index of this shard's first entry (a multiple of 4)
  int chunk;              // entries per CTA (a multiple of 4)
  int nchunks;
  float2* part;           // [rows, nchunks]: (key, index as float bits)
  int* counters;          // [rows], left at zero
  // exchange (ntp > 1): this shard's winner -> slot `self` of every rank
  float2* xdst[8];        // per rank: its exchange slots + rank `self`'s block ([rows] float2)
  int* xsig[8];           // per rank: its arrival counters [rows] (nullptr for this rank)
  int ntp, self;
};

__device__ __forceinline__ void sample_update(const SampleArgs& a, int row, int64_t best_i) {
  const int64_t slot = a.slot[row];
  const bool live = (a.active == nullptr || a.active[row]) && !a.finished[row];
  const int64_t tok = live ? best_i : a.pad_id;
  const int64_t col = slot + 1 - a.prompt_slots;
  if (col >= 0 && col < a.max_new) a.out_tokens[static_cast<long>(row) * a.max_new + col] = tok;
  if (live && !a.ignore_eos && tok == a.eos_id) a.finished[row] = 1;
  a.next_ids[row] = tok;
  a.slot[row] = slot + 1;
  a.pos[row] = a.pos[row] + 1;
  a.kv_len[row] = static_cast<int>(slot + 2);
}

__global__ void __launch_bounds__(256) sample_chunk_kernel(SplitSampleArgs x) {
  const SampleArgs& a = x.s;
  const int c = blockIdx.x, row = blockIdx.y;
  __shared__ int last;
  pdl_wait();
  const float* lg = a.logits + static_cast<long>(row) * a.ld;
  const int64_t slot = a.slot[row];
  const int v0 = c * x.chunk, v1 = min(a.V, v0 + x.chunk);
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int v4 = v0 + 4 * threadIdx.x; v4 < v1; v4 += 4 * blockDim.x) {
    const int g4 = x.vocab_start + v4;  // global index of the group's first entry
    U4 r{0, 0, 0, 0};
    if (a.inv_temp > 0.f) {
      r = philox4x32_10(U4{static_cast<uint32_t>(g4 >> 2), static_cast<uint32_t>(slot), static_cast<uint32_t>(row),
                           0x5A3F1u},
                        a.seed_lo, a.seed_hi);
    }
    const uint32_t bits[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int v = v4 + e;
      if (v >= v1) break;
      const float key = a.inv_temp > 0.f ? lg[v] * a.inv_temp + gumbel(bits[e]) : lg[v];
      best = better(best, ArgMax{key, x.vocab_start + v});
    }
  }
  best = block_argmax(best);
  if (threadIdx.x == 0) {
    x.part[static_cast<long>(row) * x.nchunks + c] = make_float2(best.v, __int_as_float(best.i));
    __threadfence();
    const int prev = atomicAdd(x.counters + row, 1);
    last = prev == x.nchunks - 1;
    if (last) x.counters[row] = 0;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  ArgMax w{-INFINITY, 0x7fffffff};
  for (int k = 0; k < x.nchunks; ++k) {
    const float2 p = __ldcg(x.part + static_cast<long>(row) * x.nchunks + k);
    w = better(w, ArgMax{p.x, __float_as_int(p.y)});
  }
  if (x.ntp <= 1) {
    sample_update(a, row, w.i);
    return;
  }
  const float2 mine = make_float2(w.v, __int_as_float(w.i));
  for (int q = 0; q < x.ntp; ++q) x.xdst[q][row] = mine;
  __threadfence_system();
  for (int q = 0; q < x.ntp; ++q)
    if (x.xsig[q] != nullptr) asm volatile("red.release.sys.global.add.s32 [%0], 1;" ::"l"(x.xsig[q] + row) : "memory");
}

// One thread per row: bounded wait for the other shards' winners, the best of
// all shards (ties -> smaller index, as in a single full-vocabulary pass), the
// decode-state update, and the arrival counter back to zero for the next step.
struct ExchangeArgs {
  SampleArgs s;
  const float2* slots;   // this rank's [ntp, rows] exchange slots
  int* arrivals;         // this rank's [rows] counters
  int ntp, rows;
  int* err;
  long long spin_limit;
};

__global__ void sample_exchange_kernel(ExchangeArgs x) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  if (row >= x.rows) return;
  const long long t0 = clock64();
  bool ok = true;
  for (;;) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(x.arrivals + row) : "memory");
    if (v >= x.ntp - 1) break;
    if (clock64() - t0 > x.spin_limit) {
      record_error(x.err, kErrPeerTimeout);
      ok = false;
      break;
    }
    __nanosleep(64);
  }
  ArgMax w{-INFINITY, 0x7fffffff};
  for (int q = 0; q < x.ntp; ++q) {
    const float2 p = __ldcg(x.slots + static_cast<long>(q) * x.rows + row);
    w = better(w, ArgMax{p.x, __float_as_int(p.y)});
  }
  if (ok) x.arrivals[row] = 0;
  sample_update(x.s, row, ok ? w.i : x.s.pad_id);
}

// one warp per token
__global__ void lse_combine_kernel(const float2* __restrict__ part, long ld, int nblk,
                                   const float* __restrict__ tgt, float* __restrict__ lse,
                                   float* __restrict__ logp, int T) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float m = -INFINITY, s = 0.f;
  for (int b = lane; b < nblk; b += 32) {
    const float2 p = part[static_cast<long>(t) * ld + b];
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
  if (lane == 0) {
    const float l = m + logf(s);
    lse[t] = l;
    logp[t] = tgt[t] - l;
  }
}

// One CTA per sequence.  loss += mean_b( sum_t m*l / max(1, sum_t m) );
// dlogp = grad_scale * m * dl/dlogp / (max(1, cnt) * B).
__global__ void grpo_loss_kernel(const float* __restrict__ logp, const float* __restrict__ old_logp,
                                 const float* __restrict__ adv, const uint8_t* __restrict__ mask,
                                 int S, int B, float clip_eps, float grad_scale,
                                 float* __restrict__ loss, float* __restrict__ dlogp,
                                 float* __restrict__ stats) {
  const long base = static_cast<long>(blockIdx.x) * S;
  float sum = 0.f, cnt = 0.f, clipped = 0.f, ratio_sum = 0.f;
  for (int t = threadIdx.x; t < S; t += blockDim.x) {
    if (!mask[base + t]) continue;
    const float r = __expf(logp[base + t] - old_logp[base + t]);
    const float A = adv[base + t];
    const float u1 = r * A;
    const float u2 = fminf(fmaxf(r, 1.f - clip_eps), 1.f + clip_eps) * A;
    sum += -fminf(u1, u2);
    cnt += 1.f;
    clipped += (u2 < u1) ? 1.f : 0.f;
    ratio_sum += r;
  }
  sum = block_reduce_sum(sum);
  cnt = block_reduce_sum(cnt);
  clipped = block_reduce_sum(clipped);
  ratio_sum = block_reduce_sum(ratio_sum);
  const float denom = fmaxf(cnt, 1.f);
  if (threadIdx.x == 0) {
    atomicAdd(loss, sum / denom / static_cast<float>(B));
    if (stats != nullptr) {
      atomicAdd(stats + 0, clipped);
      atomicAdd(stats + 1, ratio_sum);
      atomicAdd(stats + 2, cnt);
    }
  }
  const float g = grad_scale / (denom * static_cast<float>(B));
  for (int t = threadIdx.x; t < S; t += blockDim.x) {
    float d = 0.f;
    if (mask[base + t]) {
      const float r = __expf(logp[base + t] - old_logp[base + t]);
      const float A = adv[base + t];
      const float u1 = r * A;
      const float u2 = fminf(fmaxf(r, 1.f - clip_eps), 1.f + clip_eps) * A;
      d = (u1 <= u2) ? -r * A * g : 0.f;
    }
    dlogp[base + t] = d;
  }
}

// y = (add ? add : 0) + x * mask / (1 - p).  One Philox4x32-10 draw per 8
// elements: each 32-bit output word supplies two 16-bit uniforms, and an element
// is kept when its uniform is >= round(p * 2^16) (keep probability within 2^-17
// of 1 - p).  Threads move 16-byte vectors (8 bf16); the mask of element i
// depends only on (seed, stream_id, i), so the backward recomputes the forward's
// mask exactly.  Any tail of n % 8 elements goes through the same draw.
__global__ void dropout_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* y,
                               const __nv_bfloat16* add, long n, uint32_t thresh16, float keep_scale,
                               uint32_t seed_lo, uint32_t seed_hi, uint32_t stream_id) {
  const long groups = (n + 7) / 8;
  for (long q = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; q < groups;
       q += static_cast<long>(gridDim.x) * blockDim.x) {
    const U4 r = philox4x32_10(U4{static_cast<uint32_t>(q), static_cast<uint32_t>(q >> 32), stream_id, 0xD1u},
                               seed_lo, seed_hi);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
    const long i0 = q * 8;
    float v[8];
    const bool full = i0 + 8 <= n;
    if (full) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + i0);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __bfloat162float(b[e]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = i0 + e < n ? __bfloat162float(x[i0 + e]) : 0.f;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t u16 = (w[e >> 1] >> ((e & 1) * 16)) & 0xFFFFu;
      v[e] = u16 >= thresh16 ? v[e] * keep_scale : 0.f;
    }
    if (add != nullptr) {
      if (full) {
        const uint4 raw = *reinterpret_cast<const uint4*>(add + i0);
        const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] += __bfloat162float(b[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (i0 + e < n) v[e] += __bfloat162float(add[i0 + e]);
      }
    }
    if (full) {
      uint4 pk;
      __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
      for (int e = 0; e < 4; ++e) p2[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
      *reinterpret_cast<uint4*>(y + i0) = pk;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (i0 + e < n) y[i0 + e] = __float2bfloat16(v[e]);
    }
  }
}

__global__ void grad_sumsq_kernel(const float* __restrict__ g, long n, float* __restrict__ out) {
  float s = 0.f;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    s += g[i] * g[i];
  s = block_reduce_sum(s);
  if (threadIdx.x == 0) atomicAdd(out, s);
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, long n, float lr, float b1, float b2, float eps,
                             float wd, float bc1, float bc2_sqrt, const float* __restrict__ sumsq,
                             float max_norm, const float* __restrict__ loss, int* __restrict__ skipped) {
  const float ss = *sumsq;
  const bool finite = isfinite(ss) && (loss == nullptr || isfinite(*loss));
  if (!finite) {
    if (blockIdx.x == 0 && threadIdx.x == 0 && skipped != nullptr) atomicAdd(skipped, 1);
    return;
  }
  float coef = 1.f;
  if (max_norm > 0.f) coef = fminf(1.f, max_norm / (sqrtf(ss) + 1e-6f));
  const float step = lr / bc1;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float gi = g[i] * coef;
    float pi = p[i] * (1.f - lr * wd);
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    pi -= step * mi / (sqrtf(vi) / bc2_sqrt + eps);
    p[i] = pi;
  }
}

}  // namespace

void sample_append(torch::Tensor logits, double temperature, double top_p, int64_t seed,
                   torch::Tensor next_ids, torch::Tensor slot, torch::Tensor pos, torch::Tensor kv_len,
                   torch::Tensor finished, torch::Tensor out_tokens, int64_t prompt_slots,
                   int64_t eos_id, int64_t pad_id, bool ignore_eos,
                   c10::optional<torch::Tensor> active) {
  const c10::cuda::CUDAGuard guard(logits.device());
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.stride(1) == 1, "logits must be fp32 row-major");
  SampleArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.V = static_cast<int>(logits.size(1));
  a.inv_temp = temperature > 0 ? static_cast<float>(1.0 / std::max(temperature, 1e-6)) : 0.f;
  a.top_p = static_cast<float>(top_p);
  a.seed_lo = static_cast<uint32_t>(seed & 0xffffffff);
  a.seed_hi = static_cast<uint32_t>((seed >> 32) & 0xffffffff);
  a.next_ids = next_ids.data_ptr<int64_t>();
  a.slot = slot.data_ptr<int64_t>();
  a.pos = pos.data_ptr<int64_t>();
  a.kv_len = kv_len.data_ptr<int>();
  a.finished = finished.data_ptr<uint8_t>();
  a.out_tokens = out_tokens.data_ptr<int64_t>();
  a.max_new = static_cast<int>(out_tokens.size(1));
  a.prompt_slots = prompt_slots;
  a.eos_id = eos_id;
  a.pad_id = pad_id;
  a.ignore_eos = ignore_eos ? 1 : 0;
  a.active = (active.has_value() && active->defined()) ? active->data_ptr<uint8_t>() : nullptr;
  const int rows = static_cast<int>(logits.size(0));
  if (rows == 0) return;
  C10_CUDA_CHECK(launch_kernel(sample_append_kernel, dim3(rows), dim3(1024), 0, at::cuda::getCurrentCUDAStream(), a));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Split sampler (temperature > 0 or greedy, no nucleus): see sample_chunk_kernel.
// scratch: int32 [rows] counters (zeroed once, left zeroed) followed by fp32
// [rows * nchunks * 2] partials.  exch_dst / exch_sig: CPU int64 tables (one
// entry per rank) for the vocab-parallel exchange; exch_slots / exch_arrivals:
// this rank's own exchange slots and counters.
void sample_append_split(torch::Tensor logits, double temperature, int64_t seed, torch::Tensor next_ids,
                         torch::Tensor slot, torch::Tensor pos, torch::Tensor kv_len, torch::Tensor finished,
                         torch::Tensor out_tokens, int64_t prompt_slots, int64_t eos_id, int64_t pad_id,
                         bool ignore_eos, int64_t vocab_start, torch::Tensor scratch, int64_t chunk,
                         torch::Tensor err, c10::optional<torch::Tensor> exch_dst,
                         c10::optional<torch::Tensor> exch_sig, int64_t exch_self, int64_t exch_slots,
                         int64_t exch_arrivals, int64_t spin_limit) {
  const c10::cuda::CUDAGuard guard(logits.device());
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.stride(1) == 1, "logits must be fp32 row-major");
  TORCH_CHECK(vocab_start % 4 == 0 && chunk % 4 == 0 && chunk > 0, "vocab_start and chunk must be multiples of 4");
  SplitSampleArgs x{};
  SampleArgs& a = x.s;
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.V = static_cast<int>(logits.size(1));
  a.inv_temp = temperature > 0 ? static_cast<float>(1.0 / std::max(temperature, 1e-6)) : 0.f;
  a.top_p = 1.f;
  a.seed_lo = static_cast<uint32_t>(seed & 0xffffffff);
  a.seed_hi = static_cast<uint32_t>((seed >> 32) & 0xffffffff);
  a.next_ids = next_ids.data_ptr<int64_t>();
  a.slot = slot.data_ptr<int64_t>();
  a.pos = pos.data_ptr<int64_t>();
  a.kv_len = kv_len.data_ptr<int>();
  a.finished = finished.data_ptr<uint8_t>();
  a.out_tokens = out_tokens.data_ptr<int64_t>();
  a.max_new = static_cast<int>(out_tokens.size(1));
  a.prompt_slots = prompt_slots;
  a.eos_id = eos_id;
  a.pad_id = pad_id;
  a.ignore_eos = ignore_eos ? 1 : 0;
  const int rows = static_cast<int>(logits.size(0));
  if (rows == 0) return;
  x.vocab_start = static_cast<int>(vocab_start);
  x.chunk = static_cast<int>(chunk);
  x.nchunks = (a.V + x.chunk - 1) / x.chunk;
  TORCH_CHECK(scratch.is_cuda() && scratch.scalar_type() == torch::kFloat32 &&
                  scratch.numel() >= static_cast<long>(rows) * (1 + 2L * x.nchunks),
              "sampler scratch: fp32 with rows * (1 + 2 * chunks) entries");
  x.counters = reinterpret_cast<int*>(scratch.data_ptr<float>());
  x.part = reinterpret_cast<float2*>(scratch.data_ptr<float>() + ((rows + 1) / 2) * 2);
  x.ntp = 1;
  if (exch_dst.has_value() && exch_dst->defined()) {
    TORCH_CHECK(exch_sig.has_value() && exch_dst->device().is_cpu() && exch_sig->device().is_cpu() &&
                    exch_dst->numel() == exch_sig->numel() && exch_dst->numel() <= 8,
                "exchange tables: CPU int64, one entry per rank (<= 8)");
    x.ntp = static_cast<int>(exch_dst->numel());
    x.self = static_cast<int>(exch_self);
    auto d = exch_dst->contiguous(), g = exch_sig->contiguous();
    for (int q = 0; q < x.ntp; ++q) {
      x.xdst[q] = reinterpret_cast<float2*>(d.data_ptr<int64_t>()[q]);
      x.xsig[q] = reinterpret_cast<int*>(g.data_ptr<int64_t>()[q]);
    }
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(launch_kernel(sample_chunk_kernel, dim3(x.nchunks, rows), dim3(256), 0, stream, x));
  if (x.ntp > 1) {
    ExchangeArgs e{};
    e.s = a;
    e.slots = reinterpret_cast<const float2*>(exch_slots);
    e.arrivals = reinterpret_cast<int*>(exch_arrivals);
    e.ntp = x.ntp;
    e.rows = rows;
    e.err = err.data_ptr<int>();
    e.spin_limit = spin_limit > 0 ? spin_limit : 10 * kSpinLimitCycles;
    C10_CUDA_CHECK(launch_kernel(sample_exchange_kernel, dim3((rows + 127) / 128), dim3(128), 0, stream, e));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lse_combine(torch::Tensor partials, torch::Tensor tgt, torch::Tensor lse, torch::Tensor logp) {
  const c10::cuda::CUDAGuard guard(partials.device());
  TORCH_CHECK(partials.scalar_type() == torch::kFloat32 && partials.dim() == 3 && partials.size(2) == 2,
              "partials must be fp32 [T, nblk, 2]");
  const int T = static_cast<int>(partials.size(0));
  if (T == 0) return;
  const int threads = 256;
  const int blocks = (T * 32 + threads - 1) / threads;
  lse_combine_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float2*>(partials.data_ptr<float>()), partials.stride(0) / 2,
      static_cast<int>(partials.size(1)), tgt.data_ptr<float>(), lse.data_ptr<float>(),
      logp.data_ptr<float>(), T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void grpo_loss(torch::Tensor logp, torch::Tensor old_logp, torch::Tensor adv, torch::Tensor mask,
               double clip_eps, double grad_scale, torch::Tensor loss, torch::Tensor dlogp,
               c10::optional<torch::Tensor> stats) {
  const c10::cuda::CUDAGuard guard(logp.device());
  TORCH_CHECK(logp.is_contiguous() && old_logp.is_contiguous() && adv.is_contiguous() && mask.is_contiguous(),
              "grpo_loss inputs must be contiguous");
  TORCH_CHECK(mask.scalar_type() == torch::kUInt8 || mask.scalar_type() == torch::kBool, "mask must be uint8/bool");
  const int B = static_cast<int>(logp.size(0));
  const int S = static_cast<int>(logp.size(1));
  if (B == 0) return;
  grpo_loss_kernel<<<B, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      logp.data_ptr<float>(), old_logp.data_ptr<float>(), adv.data_ptr<float>(),
      reinterpret_cast<const uint8_t*>(mask.data_ptr()), S, B, static_cast<float>(clip_eps),
      static_cast<float>(grad_scale), loss.data_ptr<float>(), dlogp.data_ptr<float>(),
      (stats.has_value() && stats->defined()) ? stats->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dropout(torch::Tensor x, torch::Tensor y, double p, int64_t seed, int64_t stream_id,
             c10::optional<torch::Tensor> add) {
  const c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous(), "dropout tensors must be contiguous");
  const long n = x.numel();
  if (n == 0) return;
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && y.scalar_type() == torch::kBFloat16 && y.numel() == n,
              "dropout takes bf16 tensors of equal size");
  const bool has_add = add.has_value() && add->defined();
  if (has_add) TORCH_CHECK(add->is_contiguous() && add->numel() == n && add->scalar_type() == torch::kBFloat16,
                           "dropout add must match x");
  for (const void* ptr : {x.data_ptr(), y.data_ptr(), has_add ? add->data_ptr() : x.data_ptr()})
    TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "dropout tensors must be 16-byte aligned");
  TORCH_CHECK(p >= 0.0 && p < 1.0, "dropout probability must be in [0, 1)");
  const long groups = (n + 7) / 8;
  const uint32_t thresh16 = static_cast<uint32_t>(std::lround(p * 65536.0));
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x.get_device());
  const int blocks = static_cast<int>(std::min<long>((groups + 255) / 256, 16L * sms));
  dropout_kernel<<<std::max(blocks, 1), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
      has_add ? reinterpret_cast<const __nv_bfloat16*>(add->data_ptr()) : nullptr, n, thresh16,
      static_cast<float>(1.0 / (1.0 - p)), static_cast<uint32_t>(seed & 0xffffffff),
      static_cast<uint32_t>((seed >> 32) & 0xffffffff), static_cast<uint32_t>(stream_id));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void grad_sumsq(torch::Tensor g, torch::Tensor out) {
  const c10::cuda::CUDAGuard guard(g.device());
  const long n = g.numel();
  if (n == 0) return;
  const int blocks = static_cast<int>(std::min<long>((n + 1023) / 1024, 1184));
  grad_sumsq_kernel<<<blocks, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(g.data_ptr<float>(), n,
                                                                          out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, double lr, double b1,
           double b2, double eps, double wd, int64_t step, torch::Tensor sumsq, double max_norm,
           c10::optional<torch::Tensor> loss, c10::optional<torch::Tensor> skipped) {
  const c10::cuda::CUDAGuard guard(p.device());
  const long n = p.numel();
  if (n == 0) return;
  const float bc1 = 1.f - static_cast<float>(std::pow(b1, static_cast<double>(step)));
  const float bc2s = static_cast<float>(std::sqrt(1.0 - std::pow(b2, static_cast<double>(step))));
  const int blocks = static_cast<int>(std::min<long>((n + 255) / 256, 148 * 8));
  adamw_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), n,
      static_cast<float>(lr), static_cast<float>(b1), static_cast<float>(b2), static_cast<float>(eps),
      static_cast<float>(wd), bc1, bc2s, sumsq.data_ptr<float>(), static_cast<float>(max_norm),
      (loss.has_value() && loss->defined()) ? loss->data_ptr<float>() : nullptr,
      (skipped.has_value() && skipped->defined()) ? skipped->data_ptr<int>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace gb

// ---------------------------------------------------------------------------
// One decoding step of the gated delta rule (Gated DeltaNet, Yang et al. 2024)
// for every (row, head):
//   S <- exp(g) S;  u = beta (v - S^T k);  S <- S + k u^T;  o = S^T q
// S [dk, dv] fp32 is read twice (the second pass mostly from cache) and
// written once.  One CTA per (row, head); thread j owns column j of S, so
// S^T k and S^T q are thread-local dot products and the rank-1 update needs
// no communication; a warp touches 32 consecutive columns (coalesced).
namespace gb {
namespace {
template <int DK>
__global__ void __launch_bounds__(128) gated_delta_step_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                               const float* __restrict__ v, const float* __restrict__ g,
                                                               const float* __restrict__ beta, float* __restrict__ state,
                                                               float* __restrict__ out, int dv) {
  __shared__ float ks[DK], qs[DK];
  const long bh = blockIdx.x;
  for (int i = threadIdx.x; i < DK; i += blockDim.x) {
    ks[i] = k[bh * DK + i];
    qs[i] = q[bh * DK + i];
  }
  __syncthreads();
  const float decay = __expf(g[bh]);
  const float b = beta[bh];
  for (int j = threadIdx.x; j < dv; j += blockDim.x) {
    float* col = state + bh * DK * dv + j;
    float mem = 0.f;
#pragma unroll 8
    for (int i = 0; i < DK; ++i) mem += col[static_cast<long>(i) * dv] * ks[i];
    const float u = b * (v[bh * dv + j] - mem * decay);
    float o = 0.f;
#pragma unroll 8
    for (int i = 0; i < DK; ++i) {
      const float sn = col[static_cast<long>(i) * dv] * decay + ks[i] * u;
      col[static_cast<long>(i) * dv] = sn;
      o += sn * qs[i];
    }
    out[bh * dv + j] = o;
  }
}
}  // namespace

void gated_delta_step(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                      torch::Tensor state, torch::Tensor out) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(state.scalar_type() == torch::kFloat32 && state.is_contiguous() && state.dim() == 4,
              "state must be contiguous fp32 [B, h, dk, dv]");
  const int dk = static_cast<int>(state.size(2)), dv = static_cast<int>(state.size(3));
  const long bh = state.size(0) * state.size(1);
  for (auto* t : {&q, &k, &v, &g, &beta, &out})
    TORCH_CHECK(t->scalar_type() == torch::kFloat32 && t->is_contiguous(), "fp32 contiguous operands");
  TORCH_CHECK(q.numel() == bh * dk && k.numel() == bh * dk && v.numel() == bh * dv && g.numel() == bh &&
                  beta.numel() == bh && out.numel() == bh * dv,
              "shape mismatch");
  if (bh == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
#define GB_GDS(DKV)                                                                                        \
  gated_delta_step_kernel<DKV><<<bh, 128, 0, stream>>>(q.data_ptr<float>(), k.data_ptr<float>(),           \
                                                       v.data_ptr<float>(), g.data_ptr<float>(),           \
                                                       beta.data_ptr<float>(), state.data_ptr<float>(),    \
                                                       out.data_ptr<float>(), dv)
  switch (dk) {
    case 64: GB_GDS(64); break;
    case 128: GB_GDS(128); break;
    case 256: GB_GDS(256); break;
    default: TORCH_CHECK(false, "gated_delta_step supports key head dims 64, 128, 256");
  }
#undef GB_GDS
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
}  // namespace gb
