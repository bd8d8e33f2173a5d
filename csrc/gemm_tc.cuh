#pragma once
// Persistent, warp-specialised bf16 GEMM on the 5th-generation tensor cores.
// Reference counterparts: the LoRA linears (src/graspo/backends/graspoflow/lora.py:208-213,
// models/common/layers_qwen3.py:148-192, 287-316, 333-335), SwiGLU (layers_qwen3.py:334),
// the LM head and selected-token log-prob (tensor_utils.py:167-186) -- cuBLAS + ATen there.
//
//   C[M, N] = A[M, K] * B[N, K]^T  (+ A2[M, K2] * B2[N, K2]^T)   fp32 accumulate
//
// Both operands are K-major (row-major with K contiguous).  The optional
// second pair (A2, B2) extends the reduction: this is how a rank-r LoRA update
// s * (x A^T) B^T is folded into the frozen base GEMM x W^T -- the caller passes
// U = s * x A^T as A2 and the LoRA B factor as B2, so the adapter costs one or
// two extra K-blocks of MMA instead of a separate GEMM and an extra pass over
// the output.
//
// Structure (one CTA per SM, 6 warps):
//   warp 0      TMA producer: streams 128x64 A tiles and BNx64 B tiles into a
//               STAGES-deep shared-memory ring (128-byte swizzle).
//   warp 1      TMEM allocator + MMA issuer: one elected thread issues
//               tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM
//               accumulators and commits completion to mbarriers.
//   warps 2-5   epilogue: tcgen05.ld the finished accumulator (each warp owns
//               its 32-lane TMEM quarter), apply the fused epilogue, store.
// Double-buffered accumulators let the epilogue of tile i overlap the
// main loop of tile i+1.  Work units are (tile, K-split) pairs walked in a
// grouped raster so concurrently running CTAs share A and B tiles in L2.
//
// Epilogues:
//   kStoreBF16     C = acc (+ R)                        bf16
//   kSwiGLU        B rows interleave (gate_j, up_j): C[:, j] = silu(g) * u,
//                  optionally also stores the raw (g, u) pairs to `aux`
//   kAtomicF32     C += acc (fp32 red.add; split-K partial sums)
//   kLSE           per row: (max, sum exp) of this tile's columns < N into
//                  aux[row, n_block]; logit of targets[row] if it falls here
//   kStoreF32      C = acc fp32
//   kSoftmaxGrad   C = g[row] * (onehot(targets[row]) - exp(acc - lse[row]))  bf16;
//                  the gradient of selected-token log-probs w.r.t. the logits,
//                  produced without materialising the logits
// SWAP=true stores the transpose (C[n, m]); used for small-M decode GEMMs
// that run "swap-AB" (weights as the 128-row operand, tokens as N).
//
// No TMA multicast is used anywhere (every CTA loads its own tiles).

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>

#include "sm100_common.cuh"

namespace gb {

enum Epilogue : int { kStoreBF16 = 0, kSwiGLU = 1, kAtomicF32 = 2, kLSE = 3, kStoreF32 = 4, kSoftmaxGrad = 5 };

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kGroupM = 8;
constexpr int kMaxPeers = 8;

struct GemmArgs {
  int M, N;
  int kb_main;   // K-blocks from (A, B)
  int kb_ext;    // K-blocks from (A2, B2)
  int splits;    // split-K factor (kAtomicF32 only)
  void* C;
  long ldc;
  const __nv_bfloat16* R;  // optional residual for kStoreBF16
  long ldr;
  void* aux;
  long ldaux;
  const int64_t* targets;  // kLSE, kSoftmaxGrad
  float* tgt_logit;        // kLSE
  const float* row_lse;    // kSoftmaxGrad
  const float* row_scale;  // kSoftmaxGrad
  int* err;
  // Tensor-parallel all-reduce inside a swap kAtomicF32 GEMM: when the last
  // split of an output tile has added its partial sums, the complete fp32 tile
  // is stored into every peer's receive slot (push_dst[q], same layout as C)
  // and push_flag[q] (the peer's arrival counter) grows by the tile's element
  // count.  tile_ctr counts finished splits per tile (zeroed by the last).
  float* push_dst[kMaxPeers];
  int* push_flag[kMaxPeers];
  int npeers;              // ranks in the group (0: no push)
  int* tile_ctr;
  int nonempty_splits;     // splits that own at least one K-block
  // Tiles [0, full_tiles) run with the whole K range (one unit each); only the
  // remaining tiles are split `splits` ways (split-K SwiGLU: the last wave of a
  // persistent grid is filled without splitting every tile).  0: all tiles split.
  int full_tiles;
  // Tensor-parallel all-reduce / reduce-scatter of a non-swap bf16 GEMM
  // (prefill and training, row-parallel projections and column-parallel
  // dgrads).  With npush > 0 the epilogue stores every finished bf16 tile
  // straight into the receive slot out_push[q] of each destination rank q
  // (this rank's own slot included; row stride ldc) instead of C, and after
  // the tile the 64-bit arrival counter sig_push[q] of each remote
  // destination grows by the number of elements it received (release at
  // system scope).  push_rows > 0 selects reduce-scatter: row m goes only to
  // rank m / push_rows, at row m % push_rows of its slot; push_rows == 0 is
  // all-reduce (every rank receives every row).  The consumer kernel
  // (tp_reduce) waits for the counters and sums the slots in rank order.
  __nv_bfloat16* out_push[kMaxPeers];
  unsigned long long* sig_push[kMaxPeers];
  int npush;
  int push_self;
  int push_rows;
  int push_fence_once;  // 1: one system fence per tile by the signalling thread (after the barrier)
};

template <int BN_>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN >= 256) ? 4 : (BN >= 128 ? 6 : 8);
  static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

struct Unit {
  int m_block, n_block, kb_begin, kb_end;
  int split;      // K-split index inside its tile
  bool partial;   // the tile is split (its units write partial results)
};

__host__ __device__ __forceinline__ int unit_count(int tiles, int splits, int full_tiles) {
  return full_tiles + (tiles - full_tiles) * splits;
}

__device__ __forceinline__ Unit decode_unit(int u, int num_m, int num_n, int splits, int kb_total,
                                            int full_tiles = 0) {
  int tile, split, nsplit;
  if (u < full_tiles) {
    tile = u;
    split = 0;
    nsplit = 1;
  } else {
    const int v = u - full_tiles;
    tile = full_tiles + v / splits;
    split = v - (v / splits) * splits;
    nsplit = splits;
  }
  const int group = kGroupM * num_n;
  const int g = tile / group;
  const int first_m = g * kGroupM;
  const int gm = min(num_m - first_m, kGroupM);
  const int in_group = tile - g * group;
  Unit r;
  r.m_block = first_m + in_group % gm;
  r.n_block = in_group / gm;
  const int per = (kb_total + nsplit - 1) / nsplit;
  r.kb_begin = split * per;
  r.kb_end = min(kb_total, r.kb_begin + per);
  r.split = split;
  r.partial = nsplit > 1;
  return r;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Called by the 128 epilogue threads after they issued a unit's atomics
// (swap layout: thread <-> output feature m, C[n, m] with n = token).
template <int BN>
__device__ __forceinline__ void push_tile_impl(const GemmArgs& args, const Unit& w, int num_n, int m, int row_in_tile) {
  __shared__ int last_split;
  __threadfence();
  epi_bar();
  const int tile = w.m_block * num_n + w.n_block;
  if (row_in_tile == 0) {
    const int prev = atomicAdd(args.tile_ctr + tile, 1);
    const int last = prev == args.nonempty_splits - 1;
    if (last) args.tile_ctr[tile] = 0;
    last_split = last;
  }
  epi_bar();
  const bool last = last_split != 0;
  if (last) {
    __threadfence();
    const int n0 = w.n_block * BN;
    const int nn = min(BN, args.N - n0);
    if (m < args.M) {
      // 32 loads in flight per batch, then the stores to every peer
      const float* __restrict__ src = static_cast<const float*>(args.C);
      for (int j0 = 0; j0 < nn; j0 += 32) {
        float v[32];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          v[jj] = (j0 + jj < nn) ? __ldcg(src + static_cast<long>(n0 + j0 + jj) * args.ldc + m) : 0.f;
        for (int q = 0; q < args.npeers; ++q) {
          float* __restrict__ dst = args.push_dst[q];
          if (dst == nullptr) continue;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj)
            if (j0 + jj < nn) __stcg(dst + static_cast<long>(n0 + j0 + jj) * args.ldc + m, v[jj]);
        }
      }
    }
    __threadfence_system();
    epi_bar();
    if (row_in_tile == 0) {
      const int mm = min(BM, args.M - w.m_block * BM);
      for (int q = 0; q < args.npeers; ++q)
        if (args.push_flag[q] != nullptr)
          asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(args.push_flag[q]), "r"(mm * nn) : "memory");
    }
  }
  epi_bar();  // last_split is rewritten by the next unit
}

// One 32-column chunk of output row m (fp32 values v) to its destination
// slot(s) of the fused all-reduce / reduce-scatter (see GemmArgs::out_push).
__device__ __forceinline__ void push_chunk_bf16(const GemmArgs& args, int m, int nc, bool full_chunk,
                                                const float (&v)[32]) {
  int q0 = 0, q1 = args.npush;
  long row = m;
  if (args.push_rows > 0) {
    q0 = m / args.push_rows;
    q1 = q0 + 1;
    row = m - static_cast<long>(q0) * args.push_rows;
  }
  uint4 pk[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk[q]);
#pragma unroll
    for (int e = 0; e < 4; ++e) p2[e] = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
  }
  for (int q = q0; q < q1; ++q) {
    __nv_bfloat16* D = args.out_push[q] + row * args.ldc + nc;
    if (full_chunk) {
#pragma unroll
      for (int c = 0; c < 4; ++c) reinterpret_cast<uint4*>(D)[c] = pk[c];
    } else {
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(pk);
      for (int j = 0; j < 32; ++j)
        if (nc + j < args.N) D[j] = b[j];
    }
  }
}

// After the 128 epilogue threads stored a tile to its destinations: make the
// stores visible system-wide, then one thread adds the element counts to the
// remote destinations' arrival counters (release).  Every epilogue thread
// reaches the barrier, also after a timed-out accumulator wait, so the peers'
// consumers are never left waiting on a tile that will not be signalled.
template <int BN>
__device__ __forceinline__ void push_signal(const GemmArgs& args, const Unit& w, int row_in_tile) {
  if (!args.push_fence_once) __threadfence_system();
  epi_bar();
  if (row_in_tile == 0) {
    // the barrier orders the other epilogue threads' stores before this thread's
    // release (release is cumulative); the fence makes them visible system-wide
    if (args.push_fence_once) __threadfence_system();
    const int m0 = w.m_block * BM;
    const int mm = min(BM, args.M - m0);
    const int nn = min(BN, args.N - w.n_block * BN);
    for (int q = 0; q < args.npush; ++q) {
      if (q == args.push_self || args.sig_push[q] == nullptr) continue;
      long rows_q = mm;
      if (args.push_rows > 0) {
        const long lo = max(static_cast<long>(m0), static_cast<long>(q) * args.push_rows);
        const long hi = min(static_cast<long>(m0 + mm), static_cast<long>(q + 1) * args.push_rows);
        rows_q = hi > lo ? hi - lo : 0;
      }
      if (rows_q > 0) {
        const unsigned long long cnt = static_cast<unsigned long long>(rows_q) * nn;
        asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(args.sig_push[q]), "l"(cnt) : "memory");
      }
    }
  }
}

// Split-K SwiGLU (swap layout): every split stores its fp32 partial tile into
// its own slice of the workspace `aux` ([splits][N][ldaux]); the split that
// finishes last (tile counter) sums the slices, applies silu(gate) * up and
// writes the bf16 output -- no atomics and no workspace clearing.
constexpr int kMaxSwigluSplits = 4;

template <int BN>
__device__ __forceinline__ void swiglu_fixup_impl(const GemmArgs& args, const Unit& w, int num_n, int m,
                                                  int row_in_tile) {
  __shared__ int last_split_sw;
  // the 128 epilogue threads' partial stores are ordered before one thread's
  // acq_rel arrival by the named barrier (release is cumulative); the last
  // arrival's acquire orders the slice reads of every thread after the next barrier
  epi_bar();
  const int tile = w.m_block * num_n + w.n_block;
  if (row_in_tile == 0) {
    int prev;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(args.tile_ctr + tile) : "memory");
    const int last = prev == args.nonempty_splits - 1;
    if (last) args.tile_ctr[tile] = 0;
    last_split_sw = last;
  }
  epi_bar();
  if (last_split_sw != 0) {
    const int n0 = w.n_block * BN;
    const int nn = min(BN, args.N - n0);
    const float* __restrict__ ws = static_cast<const float*>(args.aux);
    const long slice = args.ldaux * static_cast<long>(args.N);
    __nv_bfloat16* C = static_cast<__nv_bfloat16*>(args.C);
    const int lane = threadIdx.x & 31;
    const bool live = m < args.M;
    const int ns = args.nonempty_splits;
    for (int j0 = 0; j0 < nn; j0 += 32) {
      // 32 token rows x every split: all loads in flight together
      float part[kMaxSwigluSplits][32];
#pragma unroll
      for (int q = 0; q < kMaxSwigluSplits; ++q)
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          part[q][jj] = (live && q < ns && j0 + jj < nn)
                            ? __ldcg(ws + q * slice + static_cast<long>(n0 + j0 + jj) * args.ldaux + m)
                            : 0.f;
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const float acc = (part[0][jj] + part[1][jj]) + (part[2][jj] + part[3][jj]);
        const float partner = __shfl_xor_sync(0xffffffffu, acc, 1);  // (gate, up) sit in adjacent lanes
        if ((lane & 1) == 0 && live && j0 + jj < nn)
          C[static_cast<long>(n0 + j0 + jj) * args.ldc + (m >> 1)] = __float2bfloat16(silu_f(acc) * partner);
      }
    }
  }
  epi_bar();  // last_split_sw is rewritten by the next unit
}

// LAYOUT bit 0: B (and B2) are MN-major -- given as [K, N] row-major; bit 1:
// A (and A2) are MN-major -- given as [K, M].  MN-major tiles are loaded as
// 64-wide column blocks of 64 K-rows (one swizzle atom column each).
constexpr int kMnAtomBytes = 64 * 64 * 2;

template <int BN, int EPI, bool SWAP, int LAYOUT = 0>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB2, GemmArgs args) {
  static_assert((LAYOUT & 1) == 0 || BN % 64 == 0, "MN-major B needs whole 64-wide atom columns");
  using C_ = Cfg<BN>;
  constexpr int STAGES = C_::STAGES;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment is required by the 128-byte swizzle atoms.
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * C_::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C_::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int num_m = (args.M + BM - 1) / BM;
  const int num_n = (args.N + BN - 1) / BN;
  const int kb_total = args.kb_main + args.kb_ext;
  const int units = unit_count(num_m * num_n, args.splits, args.full_tiles);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C_::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      if (args.kb_ext > 0) {
        tma_prefetch_desc(&tmA2);
        tma_prefetch_desc(&tmB2);
      }
      constexpr bool A_MN = (LAYOUT & 2) != 0;
      constexpr bool B_MN = (LAYOUT & 1) != 0;
      auto load_a = [&](uint8_t* dst, const CUtensorMap* map, int kc, int m_block, uint64_t* bar) {
        if constexpr (A_MN) {
#pragma unroll
          for (int j = 0; j < BM / 64; ++j) tma_load_2d(dst + j * kMnAtomBytes, map, bar, m_block * BM + j * 64, kc);
        } else {
          tma_load_2d(dst, map, bar, kc, m_block * BM);
        }
      };
      auto load_b = [&](uint8_t* dst, const CUtensorMap* map, int kc, int n_block, uint64_t* bar) {
        if constexpr (B_MN) {
#pragma unroll
          for (int j = 0; j < (BN + 63) / 64; ++j)
            tma_load_2d(dst + j * kMnAtomBytes, map, bar, n_block * BN + j * 64, kc);
        } else {
          tma_load_2d(dst, map, bar, kc, n_block * BN);
        }
      };
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // Swap (decode) GEMMs: the A operand is a frozen weight that no kernel
      // writes, so the first ring stages are filled with it before waiting on
      // the preceding kernel; their B halves follow after the wait.
      int early = 0;
      if constexpr (SWAP) {
        if (blockIdx.x < units) {
          const Unit w = decode_unit(blockIdx.x, num_m, num_n, args.splits, kb_total, args.full_tiles);
          for (int kb = w.kb_begin; kb < w.kb_end && early < STAGES; ++kb, ++early) {
            mbar_arrive_expect_tx(&full[early], C_::STAGE_BYTES);
            uint8_t* a_dst = smA + early * C_::A_BYTES;
            if (kb < args.kb_main) {
              load_a(a_dst, &tmA, kb * BK, w.m_block, &full[early]);
            } else {
              load_a(a_dst, &tmA2, (kb - args.kb_main) * BK, w.m_block, &full[early]);
            }
          }
        }
      }
      pdl_wait();
      int issued = 0;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit w = decode_unit(u, num_m, num_n, args.splits, kb_total, args.full_tiles);
        for (int kb = w.kb_begin; kb < w.kb_end; ++kb, ++issued) {
          uint8_t* a_dst = smA + stage * C_::A_BYTES;
          uint8_t* b_dst = smB + stage * C_::B_BYTES;
          if (issued < early) {
            // A half already in flight on this stage
            if (kb < args.kb_main) {
              load_b(b_dst, &tmB, kb * BK, w.n_block, &full[stage]);
            } else {
              load_b(b_dst, &tmB2, (kb - args.kb_main) * BK, w.n_block, &full[stage]);
            }
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1u, args.err, kErrSmemEmptyTimeout)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], C_::STAGE_BYTES);
            if (kb < args.kb_main) {
              load_a(a_dst, &tmA, kb * BK, w.m_block, &full[stage]);
              load_b(b_dst, &tmB, kb * BK, w.n_block, &full[stage]);
            } else {
              const int ke = kb - args.kb_main;
              load_a(a_dst, &tmA2, ke * BK, w.m_block, &full[stage]);
              load_b(b_dst, &tmB2, ke * BK, w.n_block, &full[stage]);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: wait (bounded) until every stage we filled has been consumed so
      // no TMA write into this CTA's shared memory is still in flight at exit.
      for (int s = 0; s < STAGES; ++s) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, args.err, kErrSmemEmptyTimeout)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool A_MN = (LAYOUT & 2) != 0;
      constexpr bool B_MN = (LAYOUT & 1) != 0;
      constexpr uint32_t idesc = umma_idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc_iter = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit w = decode_unit(u, num_m, num_n, args.splits, kb_total, args.full_tiles);
        if (w.kb_end <= w.kb_begin) continue;
        const int acc = acc_iter & 1;
        const uint32_t acc_phase = (acc_iter >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, args.err, kErrTmemEmptyTimeout)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = w.kb_begin; kb < w.kb_end; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrTmaFullTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smA + stage * C_::A_BYTES);
          const uint32_t b_addr = smem_addr(smB + stage * C_::B_BYTES);
          const uint64_t a_desc = A_MN ? umma_desc_mn_sw128(a_addr, kMnAtomBytes, 1024) : umma_desc_k_sw128(a_addr);
          const uint64_t b_desc = B_MN ? umma_desc_mn_sw128(b_addr, kMnAtomBytes, 1024) : umma_desc_k_sw128(b_addr);
          // K-step of 16: +32 bytes inside a K-major swizzled row, or two
          // 8-row atoms (2048 bytes) down an MN-major atom column
          constexpr uint64_t a_step = A_MN ? (2048 >> 4) : 2;
          constexpr uint64_t b_step = B_MN ? (2048 >> 4) : 2;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // advance 16 elements (32 bytes) along K inside the swizzled row
            umma_bf16(d_tmem, a_desc + a_step * k, b_desc + b_step * k, idesc,
                      (kb > w.kb_begin || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma_commit(&tfull[acc]);
        ++acc_iter;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;          // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    pdl_wait();  // outputs (and residual / target inputs) belong to neighbouring kernels
    int acc_iter = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const Unit w = decode_unit(u, num_m, num_n, args.splits, kb_total, args.full_tiles);
      if (w.kb_end <= w.kb_begin) continue;
      const int acc = acc_iter & 1;
      const uint32_t acc_phase = (acc_iter >> 1) & 1;
      // on a timeout the unit is skipped but the loop goes on, so every
      // epilogue warp reaches the same named barriers of the tile push
      const bool have_acc = mbar_wait(&tfull[acc], acc_phase, args.err, kErrTmemFullTimeout);
      tc_fence_after();
      const int m = w.m_block * BM + row_in_tile;
      const int n0 = w.n_block * BN;
      const uint32_t t_row = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      float run_max = -INFINITY, run_sum = 0.f;
#pragma unroll 1
      for (int c = 0; c < (have_acc ? BN / 32 : 0); ++c) {
        float v[32];
        tmem_ld32(t_row + c * 32, v);
        const int nc = n0 + c * 32;
        if constexpr (SWAP) {
          // lane <-> output feature m, column <-> token n; store C[n, m]
          if constexpr (EPI == kAtomicF32) {
            float* C = static_cast<float*>(args.C);
            if (m < args.M) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (nc + j < args.N) atomicAdd(C + static_cast<long>(nc + j) * args.ldc + m, v[j]);
            }
          } else if constexpr (EPI == kStoreBF16) {
            __nv_bfloat16* C = static_cast<__nv_bfloat16*>(args.C);
            if (m < args.M) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (nc + j < args.N) {
                  float x = v[j];
                  if (args.R != nullptr) x += __bfloat162float(args.R[static_cast<long>(nc + j) * args.ldr + m]);
                  C[static_cast<long>(nc + j) * args.ldc + m] = __float2bfloat16(x);
                }
              }
            }
          } else if constexpr (EPI == kSwiGLU) {
            if (w.partial) {
              // split-K: the partial tile goes to this split's workspace slice
              float* P = static_cast<float*>(args.aux) +
                         static_cast<long>(w.split) * args.ldaux * static_cast<long>(args.N);
              if (m < args.M) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (nc + j < args.N) __stcg(P + static_cast<long>(nc + j) * args.ldaux + m, v[j]);
              }
            } else {
              // adjacent lanes hold (gate_j, up_j); even lanes write silu(g)*u
              __nv_bfloat16* C = static_cast<__nv_bfloat16*>(args.C);
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float partner = __shfl_xor_sync(0xffffffffu, v[j], 1);
                if ((lane & 1) == 0 && m < args.M && nc + j < args.N) {
                  C[static_cast<long>(nc + j) * args.ldc + (m >> 1)] =
                      __float2bfloat16(silu_f(v[j]) * partner);
                }
              }
            }
          } else if constexpr (EPI == kStoreF32) {
            float* C = static_cast<float*>(args.C);
            if (m < args.M) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (nc + j < args.N) C[static_cast<long>(nc + j) * args.ldc + m] = v[j];
            }
          }
        } else {
          if (m >= args.M) {
            if constexpr (EPI == kLSE) { /* keep tcgen05.ld convergent; nothing to write */ }
            continue;
          }
          const bool full_chunk = (nc + 32 <= args.N);
          if constexpr (EPI == kStoreBF16) {
            if (args.npush > 0) {
              if (args.R != nullptr) {
                const __nv_bfloat16* R = args.R + static_cast<long>(m) * args.ldr + nc;
                if (full_chunk) {
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    uint4 rv = *reinterpret_cast<const uint4*>(R + q * 8);
                    const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[q * 8 + e] += __bfloat162float(rb[e]);
                  }
                } else {
                  for (int j = 0; j < 32; ++j)
                    if (nc + j < args.N) v[j] += __bfloat162float(R[j]);
                }
              }
              push_chunk_bf16(args, m, nc, full_chunk, v);
              continue;
            }
            __nv_bfloat16* C = static_cast<__nv_bfloat16*>(args.C) + static_cast<long>(m) * args.ldc + nc;
            if (args.R != nullptr) {
              const __nv_bfloat16* R = args.R + static_cast<long>(m) * args.ldr + nc;
              if (full_chunk) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  uint4 rv = *reinterpret_cast<const uint4*>(R + q * 8);
                  const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
                  for (int e = 0; e < 8; ++e) v[q * 8 + e] += __bfloat162float(rb[e]);
                }
              } else {
                for (int j = 0; j < 32; ++j)
                  if (nc + j < args.N) v[j] += __bfloat162float(R[j]);
              }
            }
            if (full_chunk) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 pk;
                __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int e = 0; e < 4; ++e) p2[e] = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
                *reinterpret_cast<uint4*>(C + q * 8) = pk;
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (nc + j < args.N) C[j] = __float2bfloat16(v[j]);
            }
          } else if constexpr (EPI == kStoreF32) {
            float* C = static_cast<float*>(args.C) + static_cast<long>(m) * args.ldc + nc;
            if (full_chunk) {
#pragma unroll
              for (int q = 0; q < 8; ++q)
                *reinterpret_cast<float4*>(C + q * 4) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            } else {
              for (int j = 0; j < 32; ++j)
                if (nc + j < args.N) C[j] = v[j];
            }
          } else if constexpr (EPI == kAtomicF32) {
            float* C = static_cast<float*>(args.C) + static_cast<long>(m) * args.ldc + nc;
            for (int j = 0; j < 32; ++j)
              if (nc + j < args.N) atomicAdd(C + j, v[j]);
          } else if constexpr (EPI == kSwiGLU) {
            // columns (2i, 2i+1) = (gate_i, up_i) -> out column (nc/2 + i)
            __nv_bfloat16* C = static_cast<__nv_bfloat16*>(args.C) + static_cast<long>(m) * args.ldc + (nc >> 1);
            if (args.aux != nullptr) {
              __nv_bfloat16* G = static_cast<__nv_bfloat16*>(args.aux) + static_cast<long>(m) * args.ldaux + nc;
              if (full_chunk) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  uint4 pk;
                  __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                  for (int e = 0; e < 4; ++e) p2[e] = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
                  *reinterpret_cast<uint4*>(G + q * 8) = pk;
                }
              } else {
                for (int j = 0; j < 32; ++j)
                  if (nc + j < args.N) G[j] = __float2bfloat16(v[j]);
              }
            }
            if (full_chunk) {
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                uint4 pk;
                __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int i0 = q * 16 + 4 * e;
                  // the GEMM accumulates in fp32; the activation is applied to
                  // the bf16-rounded pre-activations so forward and backward see
                  // the same (g, u) values that are stored to `aux`
                  const float g0 = __bfloat162float(__float2bfloat16(v[i0]));
                  const float u0 = __bfloat162float(__float2bfloat16(v[i0 + 1]));
                  const float g1 = __bfloat162float(__float2bfloat16(v[i0 + 2]));
                  const float u1 = __bfloat162float(__float2bfloat16(v[i0 + 3]));
                  p2[e] = __floats2bfloat162_rn(silu_f(g0) * u0, silu_f(g1) * u1);
                }
                *reinterpret_cast<uint4*>(C + q * 8) = pk;
              }
            } else {
              for (int j = 0; j + 1 < 32; j += 2)
                if (nc + j + 1 < args.N) {
                  const float g = __bfloat162float(__float2bfloat16(v[j]));
                  const float uu = __bfloat162float(__float2bfloat16(v[j + 1]));
                  C[j >> 1] = __float2bfloat16(silu_f(g) * uu);
                }
            }
          } else if constexpr (EPI == kSoftmaxGrad) {
            __nv_bfloat16* C = static_cast<__nv_bfloat16*>(args.C) + static_cast<long>(m) * args.ldc + nc;
            const float l = args.row_lse[m];
            const float gs = args.row_scale[m];
            const long tgt = args.targets[m];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = gs * (((nc + j) == tgt ? 1.f : 0.f) - __expf(v[j] - l));
            if (full_chunk) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 pk;
                __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int e = 0; e < 4; ++e) p2[e] = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
                *reinterpret_cast<uint4*>(C + q * 8) = pk;
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (nc + j < args.N) C[j] = __float2bfloat16(v[j]);
            }
          } else if constexpr (EPI == kLSE) {
            float cmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nc + j < args.N) cmax = fmaxf(cmax, v[j]);
            if (cmax > -INFINITY) {
              const float new_max = fmaxf(run_max, cmax);
              float s = 0.f;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (nc + j < args.N) s += __expf(v[j] - new_max);
              run_sum = run_sum * __expf(run_max - new_max) + s;
              run_max = new_max;
            }
            const long tgt = args.targets[m];
            if (tgt >= nc && tgt < nc + 32) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (tgt == nc + j) args.tgt_logit[m] = v[j];
            }
          }
        }
      }
      if constexpr (EPI == kLSE && !SWAP) {
        if (m < args.M && have_acc) {
          float2* P = static_cast<float2*>(args.aux) + static_cast<long>(m) * args.ldaux + w.n_block;
          *P = make_float2(run_max, run_sum);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      ++acc_iter;
      if constexpr (SWAP && EPI == kAtomicF32) {
        if (args.npeers > 1) push_tile_impl<BN>(args, w, num_n, m, row_in_tile);
      }
      if constexpr (SWAP && EPI == kSwiGLU) {
        if (w.partial) swiglu_fixup_impl<BN>(args, w, num_n, m, row_in_tile);
      }
      if constexpr (!SWAP && EPI == kStoreBF16) {
        if (args.npush > 0) push_signal<BN>(args, w, row_in_tile);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C_::TMEM_COLS);
  }
}

inline int num_sms(int device) {
  static int cached[64] = {0};
  if (cached[device] == 0) {
    cudaDeviceGetAttribute(&cached[device], cudaDevAttrMultiProcessorCount, device);
  }
  return cached[device];
}

template <int BN, int EPI, bool SWAP, int LAYOUT = 0>
void launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& a2,
                        const CUtensorMap& b2, const GemmArgs& args, int max_ctas,
                        cudaStream_t stream, int device) {
  auto kern = gemm_tc_kernel<BN, EPI, SWAP, LAYOUT>;
  // MN-major instantiations get 16 KiB of unused tail so that every address a
  // stage descriptor can reach stays inside the allocation
  constexpr int smem = Cfg<BN>::SMEM_BYTES + (LAYOUT != 0 ? 16384 : 0);
  static_assert(smem <= 227 * 1024, "shared memory budget");
  static bool configured[64] = {false};
  if (!configured[device]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured[device] = true;
  }
  const int num_m = (args.M + BM - 1) / BM;
  const int num_n = (args.N + BN - 1) / BN;
  const int units = unit_count(num_m * num_n, args.splits, args.full_tiles);
  int grid = std::min(units, num_sms(device));
  if (max_ctas > 0) grid = std::min(grid, max_ctas);
  grid = std::max(grid, 1);
  C10_CUDA_CHECK(launch_kernel(kern, dim3(grid), dim3(kThreads), smem, stream, a, b, a2, b2, args));
}


using GemmLauncher = void (*)(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                              const GemmArgs&, int, cudaStream_t, int);

// Defined in the gemm_inst_*.cu translation units (compiled in parallel).
GemmLauncher gemm_launcher_n256(int epi);
GemmLauncher gemm_launcher_n128(int epi);
GemmLauncher gemm_launcher_n64(int epi);
GemmLauncher gemm_launcher_swap(int bn, int epi);
GemmLauncher gemm_launcher_mn(int bn, int epi, bool swap, int layout);

}  // namespace gb
