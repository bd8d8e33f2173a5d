// Decode-step attention over the paged KV cache on the 5th-generation tensor
// cores: TMA page tiles into a shared-memory ring, S = Q K^T and O += P V as
// tcgen05.mma with the accumulators in TMEM, one softmax thread per query row.
//
// Reference counterpart: the decode attention of the reference's generation
// loop (src/graspo/backends/graspoflow/models/common/layers_qwen3.py:248-251,
// SDPA over a concatenated KV cache; models/qwen35_36/generation.py:249-276).
//
// Cache layout: k_pool / v_pool [num_pages, nkv, page, 128] bf16; block_table
// [rows, max_pages]; row r attends to key positions [start[r], len[r]).
//
// Work units (one CTA each, grid = units):
//   * prompt units (prefix_len > 0): the rows of a GRASPO group share the pages
//     of key positions [start, prefix_len).  One unit takes a slice of those
//     keys for ALL group_rows x G query heads of one KV head (up to 128 query
//     rows of the MMA tile), so the prompt keys are read from DRAM once per
//     group instead of once per row.
//   * row units: one row's own keys [max(start, prefix_len), len) -- all of its
//     keys without a prefix -- split into `splits` slices; G query rows.
// Every unit stores per query row an unnormalised partial (O, running max m,
// sum l) into the scratch slots; a per-(row, KV head) arrival counter lets the
// CTA that completes a row's last slot merge all of its slots and write the
// output (no CTA ever waits on another).  The counter is reset by the merger.
//
// CTA: 6 warps.  Warp 0 issues TMA loads of 64-key K and V tiles (128-byte
// swizzle, one box of up to 64 keys x 64 dims per page piece) into a 3-stage
// ring; warp 1 owns TMEM (256 columns: two S buffers of 64 + O of 128) and
// issues the MMAs (M = 128 query rows, of which the unit's valid ones are
// real); warps 2-5 load Q into swizzled shared memory, run the online softmax
// in the log2 domain with lazy O rescaling (only when the running max grows by
// more than 2^8), write P (bf16, K-major) for the PV MMA, and store the
// partials.  Every wait is bounded; a wait that gives up records an error code
// and the kernel drains and exits.
//
// No TMA multicast is used (each CTA loads its own tiles of this GPU's pool).

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>

#include "sm100_common.cuh"

namespace gb {

namespace {

constexpr int kHD = 128;             // head dim
constexpr int kKeys = 64;            // keys per tile
constexpr int kRows = 128;           // query rows of the MMA tile
constexpr int kStages = 3;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 256;  // S0 [0, 64), S1 [64, 128), O [128, 256)
constexpr float kRescaleLog2 = 8.f;

constexpr int kQAtom = kRows * 128;      // 128 rows x 128 B: 16 KiB (one 64-dim half of Q)
constexpr int kKVAtom = kKeys * 128;     // 64 keys x 128 B: 8 KiB (one 64-dim half of a K / V tile)
constexpr int kKVTile = 2 * kKVAtom;     // 16 KiB
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kQAtom;
constexpr int kOffV = kOffK + kStages * kKVTile;
constexpr int kOffP = kOffV + kStages * kKVTile;   // 128 rows x 64 keys bf16: 16 KiB
constexpr int kOffBar = kOffP + kQAtom;
constexpr int kOffMisc = kOffBar + 256;
constexpr int kSmem = kOffMisc + 256 + 1024;

struct DecodeTcArgs {
  const __nv_bfloat16* q;  // [rows, nq, 128]
  const int* block_table;  // [rows, max_pages]
  const int* start;        // [rows]
  const int* len;          // [rows]
  __nv_bfloat16* out;      // [rows, nq * 128]
  float* part_acc;         // [rows, nq, slots, 128]
  float* part_ml;          // [rows, nq, slots, 2]
  int* counters;           // [rows, nkv]
  int rows, nq, nkv, G, page, max_pages, num_pages;
  int prefix_len, group_rows, prefix_splits, prefix_kps;  // prompt units (prefix_len > 0)
  int splits, kps;                                       // row units: key slices of kps keys
  int prompt_units;                                      // groups * nkv * prefix_splits
  int slots;                                             // prefix_splits (if prefix) + splits
  float scale_log2;
  int* err;
};

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

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

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// The unit a CTA works on.
struct Unit {
  bool prompt;     // prompt unit (all rows of a group) or row unit
  int row0;        // first row (prompt: the group's first row)
  int nrows;       // rows whose queries are in the tile (prompt: group_rows, row unit: 1)
  int kvh;
  int slot;        // partial slot of every query row of the unit
  int k_begin, k_end;  // key positions of the unit (may be empty)
};

__device__ __forceinline__ Unit decode_unit(const DecodeTcArgs& a, int b) {
  Unit u;
  if (b < a.prompt_units) {
    const int ps = b % a.prefix_splits;
    const int rest = b / a.prefix_splits;
    u.kvh = rest % a.nkv;
    const int grp = rest / a.nkv;
    u.prompt = true;
    u.row0 = grp * a.group_rows;
    u.nrows = a.group_rows;
    u.slot = ps;
    const int s0 = a.start[u.row0];
    u.k_begin = max(s0, ps * a.prefix_kps);
    u.k_end = min(a.prefix_len, (ps + 1) * a.prefix_kps);
  } else {
    const int c = b - a.prompt_units;
    const int s = c % a.splits;
    const int rest = c / a.splits;
    u.kvh = rest % a.nkv;
    u.row0 = rest / a.nkv;
    u.prompt = false;
    u.nrows = 1;
    u.slot = (a.prefix_len > 0 ? a.prefix_splits : 0) + s;
    const int lo = max(a.start[u.row0], a.prefix_len);
    const int hi = min(a.len[u.row0], a.max_pages * a.page);
    u.k_begin = max(lo, a.prefix_len + s * a.kps);
    u.k_end = min(hi, a.prefix_len + (s + 1) * a.kps);
  }
  return u;
}

__global__ void __launch_bounds__(kThreads, 1)
    paged_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           DecodeTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* sm = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint64_t* k_full = bar + 0;                 // [kStages]
  uint64_t* k_empty = bar + kStages;          // [kStages]
  uint64_t* v_full = bar + 2 * kStages;       // [kStages]
  uint64_t* v_empty = bar + 3 * kStages;      // [kStages]
  uint64_t* s_full = bar + 4 * kStages;       // [2]
  uint64_t* s_free = s_full + 2;              // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 1;
  uint64_t* q_full = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffMisc);
  int* merge_list = reinterpret_cast<int*>(sm + kOffMisc + 16);   // rows this CTA must merge (<= 64)
  int* merge_n = reinterpret_cast<int*>(sm + kOffMisc + 8);
  const uint32_t sQ = smem_addr(sm + kOffQ), sK = smem_addr(sm + kOffK), sV = smem_addr(sm + kOffV),
                 sP = smem_addr(sm + kOffP);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();  // q, the lengths and the pool belong to the preceding kernels
  const Unit u = decode_unit(a, blockIdx.x);
  const int t_first = u.k_end > u.k_begin ? u.k_begin / kKeys : 0;
  const int n_tiles = u.k_end > u.k_begin ? (u.k_end - 1) / kKeys - t_first + 1 : 0;
  const int* bt = a.block_table + static_cast<long>(u.row0) * a.max_pages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(s_full + s, 1);
      mbar_init(s_free + s, 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(q_full, 128);
    *merge_n = 0;
    fence_mbar_init();
  }
  if (warp == 1 && n_tiles > 0) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = n_tiles > 0 ? *tmem_slot : 0u;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const int box = a.page < kKeys ? a.page : kKeys;   // keys per TMA box
      auto load_tile = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* b, int key0) {
        // 64 keys from one or more pages (box rows each), both 64-dim halves; a
        // page index past the pool reads the tensor map's zero fill
        for (int kk = 0; kk < kKeys; kk += box) {
          const int key = key0 + kk;
          const int lp = min(key / a.page, a.max_pages - 1);
          const int phys = checked_index(bt[lp], a.num_pages, a.err);
          const int y = (phys * a.nkv + u.kvh) * a.page + (key - lp * a.page);
#pragma unroll
          for (int c = 0; c < 2; ++c) tma_load_2d(dst + c * kKVAtom + kk * 128, map, b, c * 64, y);
        }
      };
      for (int i = 0; i < n_tiles; ++i) {
        const int st = i % kStages;
        const uint32_t ph = (i / kStages) & 1;
        const int key0 = (t_first + i) * kKeys;
        if (i >= kStages && !mbar_wait(k_empty + st, ph ^ 1u, a.err, kErrSmemEmptyTimeout)) break;
        mbar_arrive_expect_tx(k_full + st, kKVTile);
        load_tile(&tmK, sm + kOffK + st * kKVTile, k_full + st, key0);
        if (i >= kStages && !mbar_wait(v_empty + st, ph ^ 1u, a.err, kErrSmemEmptyTimeout)) break;
        mbar_arrive_expect_tx(v_full + st, kKVTile);
        load_tile(&tmV, sm + kOffV + st * kKVTile, v_full + st, key0);
      }
      // drain: no TMA write may still target this CTA's shared memory at exit
      for (int i = max(0, n_tiles - kStages); i < n_tiles; ++i) {
        const int st = i % kStages;
        const uint32_t ph = (i / kStages) & 1;
        if (!mbar_wait(k_empty + st, ph, a.err, kErrSmemEmptyTimeout)) break;
        if (!mbar_wait(v_empty + st, ph, a.err, kErrSmemEmptyTimeout)) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kRows, kKeys, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kRows, kHD, false, true);
      const uint32_t o_tmem = tmem + 128;
      bool ok = mbar_wait(q_full, 0, a.err, kErrTmaFullTimeout);
      auto mma_pv = [&](int t) {
        if (!ok) return;
        const int st = t % kStages;
        ok = mbar_wait(p_full, t & 1, a.err, kErrTmaFullTimeout) &&
             mbar_wait(v_full + st, (t / kStages) & 1, a.err, kErrTmaFullTimeout);
        if (!ok) return;
        tc_fence_after();
        const uint32_t vbase = sV + st * kKVTile;
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k) {
          // A = P (K-major, one atom; +32 B per 16 keys), B = V (MN-major: the two 64-dim atom
          // columns are 8 KiB apart, a 16-key step is two 8-row groups = 2 KiB)
          const uint64_t pd = umma_desc_k_sw128(sP) + 2 * k;
          const uint64_t vd = umma_desc_mn_sw128(vbase + k * 2048, kKVAtom, 1024);
          umma_bf16(o_tmem, pd, vd, idesc_pv, (t > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(v_empty + st);
        umma_commit(o_done);
      };
      for (int i = 0; i < n_tiles && ok; ++i) {
        const int st = i % kStages;
        const int sb = i & 1;
        ok = mbar_wait(k_full + st, (i / kStages) & 1, a.err, kErrTmaFullTimeout);
        if (ok && i >= 2) ok = mbar_wait(s_free + sb, ((i - 2) >> 1) & 1, a.err, kErrTmemEmptyTimeout);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kbase = sK + st * kKVTile;
#pragma unroll
        for (int k = 0; k < kHD / 16; ++k) {
          const uint64_t qd = umma_desc_k_sw128(sQ + (k >> 2) * kQAtom) + 2 * (k & 3);
          const uint64_t kd = umma_desc_k_sw128(kbase + (k >> 2) * kKVAtom) + 2 * (k & 3);
          umma_bf16(tmem + sb * kKeys, qd, kd, idesc_qk, k > 0 ? 1u : 0u);
        }
        umma_commit(k_empty + st);
        umma_commit(s_full + sb);
        if (i >= 1) mma_pv(i - 1);
      }
      mma_pv(n_tiles - 1);
    }
  } else {
    // ------------------------------------------------------------ softmax / partials
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;            // query row of the tile = TMEM lane
    const int heads = a.G;
    const int nvalid = u.nrows * heads;
    const bool row_ok = r < nvalid;
    const int qrow = u.row0 + (row_ok ? r / heads : 0);        // decode row of this query
    const int qhead = u.kvh * heads + (row_ok ? r % heads : 0);
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    // Q row -> swizzled K-major tile (zeros for the padding rows)
    if (n_tiles > 0) {
      const uint4* src = reinterpret_cast<const uint4*>(a.q + (static_cast<long>(qrow) * a.nq + qhead) * kHD);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v = row_ok ? src[c] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t addr = sQ + (c >> 3) * kQAtom + (r >> 3) * 1024 + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
      }
      fence_async_smem();
      mbar_arrive(q_full);
    }
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      const int sb = i & 1;
      const int key0 = (t_first + i) * kKeys;
      const bool interior = key0 >= u.k_begin && key0 + kKeys <= u.k_end;
      bool got = ok && __all_sync(0xffffffffu, mbar_wait(s_full + sb, (i >> 1) & 1, a.err, kErrTmemFullTimeout));
      if (!got) {
        ok = false;
        break;
      }
      float s[64];
      tc_fence_after();
      tmem_ld32(tmem + lane_off + sb * kKeys, *reinterpret_cast<float(*)[32]>(s));
      tmem_ld32(tmem + lane_off + sb * kKeys + 32, *reinterpret_cast<float(*)[32]>(s + 32));
      tc_fence_before();
      mbar_arrive(s_free + sb);
      if (!interior) {
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          const int kj = key0 + e;
          if (kj < u.k_begin || kj >= u.k_end) s[e] = -INFINITY;
        }
      }
      float m4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
      for (int e = 4; e < 64; ++e) m4[e & 3] = fmaxf(m4[e & 3], s[e]);
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      const float m_new = fmaxf(m, mx * a.scale_log2);
      float alpha = 1.f;
      const bool need = m != -INFINITY && m_new > m + kRescaleLog2;
      if (m == -INFINITY) {
        m = m_new;
      } else if (need) {
        alpha = ex2(m - m_new);
        m = m_new;
      }
      const bool rescale = __any_sync(0xffffffffu, need);
      const float neg_m = m == -INFINITY ? 0.f : -m;
      float p4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int e = 0; e < 64; ++e) {
        s[e] = ex2(fmaf(s[e], a.scale_log2, neg_m));
        p4[e & 3] += s[e];
      }
      l = l * alpha + ((p4[0] + p4[1]) + (p4[2] + p4[3]));
      // P(i) overwrites P(i-1), and O may be rescaled: O += P(i-1) V(i-1) must be complete
      if (i >= 1) {
        if (!__all_sync(0xffffffffu, mbar_wait(o_done, (i - 1) & 1, a.err, kErrTmemFullTimeout))) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (rescale && i >= 1) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tmem + lane_off + 128 + c * 32, v);
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] *= alpha;
          tmem_st32(tmem + lane_off + 128 + c * 32, v);
        }
        tmem_wait_st();
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t addr = sP + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4);
        const uint32_t w0 = pack2(s[c * 8 + 0], s[c * 8 + 1]), w1 = pack2(s[c * 8 + 2], s[c * 8 + 3]);
        const uint32_t w2 = pack2(s[c * 8 + 4], s[c * 8 + 5]), w3 = pack2(s[c * 8 + 6], s[c * 8 + 7]);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                     : "memory");
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // ---- partial of this unit for every valid query row: O (unnormalised), m, l
    if (ok && n_tiles > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(o_done, (n_tiles - 1) & 1, a.err, kErrTmemFullTimeout));
      tc_fence_after();
    }
    const long pidx = (static_cast<long>(qrow) * a.nq + qhead) * a.slots + u.slot;
    if (ok && n_tiles > 0) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tmem + lane_off + 128 + c * 32, v);   // every lane of the warp takes part
        if (row_ok) {
          float4* dst = reinterpret_cast<float4*>(a.part_acc + pidx * kHD + c * 32);
#pragma unroll
          for (int e = 0; e < 8; ++e) __stcg(dst + e, make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]));
        }
      }
    }
    if (row_ok) {
      // an empty or failed unit contributes nothing (m = -inf)
      const bool have = ok && n_tiles > 0;
      __stcg(reinterpret_cast<float2*>(a.part_ml) + pidx, make_float2(have ? m : -INFINITY, have ? l : 0.f));
    }
  }

  // ---- arrivals: the CTA that completes a (row, KV head) merges its slots
  __threadfence();
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int rr = 0; rr < u.nrows; ++rr) {
      int* ctr = a.counters + static_cast<long>(u.row0 + rr) * a.nkv + u.kvh;
      const int prev = atomicAdd(ctr, 1);
      if (prev == a.slots - 1) {
        *ctr = 0;
        merge_list[(*merge_n)++] = u.row0 + rr;
      }
    }
  }
  __syncthreads();
  const int nm = *merge_n;
  if (nm > 0) {
    __threadfence();
    for (int i = threadIdx.x; i < nm * a.G * kHD; i += blockDim.x) {
      const int d = i % kHD;
      const int hh = (i / kHD) % a.G;
      const int row = merge_list[i / (kHD * a.G)];
      const long head = static_cast<long>(row) * a.nq + u.kvh * a.G + hh;
      const long pbase = head * a.slots;
      float mm = -INFINITY;
      for (int sp = 0; sp < a.slots; ++sp) mm = fmaxf(mm, __ldcg(a.part_ml + (pbase + sp) * 2));
      float ls = 0.f, ov = 0.f;
      if (mm > -INFINITY) {
        for (int sp = 0; sp < a.slots; ++sp) {
          const float ms = __ldcg(a.part_ml + (pbase + sp) * 2);
          if (ms == -INFINITY) continue;
          const float cf = exp2f(ms - mm);
          ls += __ldcg(a.part_ml + (pbase + sp) * 2 + 1) * cf;
          ov += __ldcg(a.part_acc + (pbase + sp) * kHD + d) * cf;
        }
      }
      a.out[head * kHD + d] = __float2bfloat16(ls > 0.f ? ov / ls : 0.f);
    }
  }
  if (warp == 1 && n_tiles > 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

CUtensorMap make_tmap_bf16(const void* ptr, long rows, long cols, long ld, int box_rows);

// Decode attention on tcgen05 over the paged cache (see the file comment).
// scratch: fp32, at least rows*nq*slots*130 floats + rows*nkv counters (zeroed once;
// the kernel leaves the counters zeroed).  slots = splits (+ prefix_splits when
// prefix_len > 0).
void paged_decode_attention_tc(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool,
                               torch::Tensor block_table, torch::Tensor start, torch::Tensor len,
                               torch::Tensor out, double scale, int64_t splits, torch::Tensor scratch,
                               int64_t prefix_len, int64_t group_rows, int64_t prefix_splits,
                               torch::Tensor err) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && q.is_contiguous() && q.dim() == 3 && q.size(2) == kHD,
              "q must be contiguous bf16 [rows, nq, 128]");
  TORCH_CHECK(k_pool.dim() == 4 && k_pool.size(3) == kHD && k_pool.is_contiguous() && v_pool.is_contiguous() &&
                  v_pool.sizes() == k_pool.sizes() && k_pool.scalar_type() == torch::kBFloat16,
              "k_pool / v_pool must be contiguous bf16 [pages, nkv, page, 128]");
  const int rows = static_cast<int>(q.size(0)), nq = static_cast<int>(q.size(1));
  const int pages = static_cast<int>(k_pool.size(0)), nkv = static_cast<int>(k_pool.size(1));
  const int page = static_cast<int>(k_pool.size(2));
  TORCH_CHECK(nq % nkv == 0, "nq must be a multiple of nkv");
  TORCH_CHECK(page % 16 == 0 && (page % kKeys == 0 || kKeys % page == 0),
              "page size must divide 64 or be a multiple of 64 (and a multiple of 16)");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && block_table.is_contiguous() &&
                  block_table.size(0) == rows, "block_table must be int32 [rows, max_pages]");
  DecodeTcArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.block_table = block_table.data_ptr<int>();
  a.start = start.data_ptr<int>();
  a.len = len.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.rows = rows;
  a.nq = nq;
  a.nkv = nkv;
  a.G = nq / nkv;
  a.page = page;
  a.max_pages = static_cast<int>(block_table.size(1));
  a.num_pages = pages;
  a.err = err.data_ptr<int>();
  a.scale_log2 = static_cast<float>(scale) * 1.4426950408889634f;
  const int capacity = a.max_pages * page;
  a.prefix_len = static_cast<int>(prefix_len);
  if (a.prefix_len > 0) {
    a.group_rows = static_cast<int>(group_rows);
    a.prefix_splits = static_cast<int>(std::max<int64_t>(1, prefix_splits));
    TORCH_CHECK(a.group_rows > 0 && rows % a.group_rows == 0 && a.group_rows * a.G <= kRows && a.group_rows <= 64,
                "rows must form groups of group_rows with group_rows * G <= 128");
    TORCH_CHECK(a.prefix_len % kKeys == 0 && a.prefix_len <= capacity, "prefix length must be 64-aligned");
    a.prefix_kps = ((a.prefix_len + a.prefix_splits - 1) / a.prefix_splits + kKeys - 1) / kKeys * kKeys;
    a.prompt_units = (rows / a.group_rows) * nkv * a.prefix_splits;
  } else {
    TORCH_CHECK(a.G <= kRows, "too many query heads per KV head");
    a.prefix_splits = 0;
    a.prompt_units = 0;
  }
  a.splits = static_cast<int>(std::max<int64_t>(1, splits));
  a.kps = ((capacity - a.prefix_len + a.splits - 1) / a.splits + kKeys - 1) / kKeys * kKeys;
  a.slots = a.prefix_splits + a.splits;
  const long need_f = static_cast<long>(rows) * nq * a.slots * (kHD + 2);
  TORCH_CHECK(scratch.scalar_type() == torch::kFloat32 && scratch.is_contiguous() &&
                  scratch.numel() >= need_f + static_cast<long>(rows) * nkv,
              "decode-attention scratch too small: need ", need_f + static_cast<long>(rows) * nkv, " floats");
  float* base = scratch.data_ptr<float>();
  a.part_acc = base;
  a.part_ml = base + static_cast<long>(rows) * nq * a.slots * kHD;
  a.counters = reinterpret_cast<int*>(base + need_f);
  const int units = a.prompt_units + rows * nkv * a.splits;
  if (units == 0) return;
  // both pools viewed as [pages * nkv * page, 128] rows; boxes of min(page, 64) keys x 64 dims
  const int box = page < kKeys ? page : kKeys;
  const long krows = static_cast<long>(pages) * nkv * page;
  const CUtensorMap tk = make_tmap_bf16(k_pool.data_ptr(), krows, kHD, kHD, box);
  const CUtensorMap tv = make_tmap_bf16(v_pool.data_ptr(), krows, kHD, kHD, box);
  static bool configured[64] = {false};
  const int dev = q.get_device();
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(paged_decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    configured[dev] = true;
  }
  C10_CUDA_CHECK(launch_kernel(paged_decode_tc_kernel, dim3(units), dim3(kThreads), kSmem,
                               at::cuda::getCurrentCUDAStream(), tk, tv, a));
}

}  // namespace gb
