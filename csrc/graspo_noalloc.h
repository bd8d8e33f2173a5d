/* Allocation-free entry points of the graspo_b200 kernel library (C ABI).
 *
 * This header has no counterpart in the reference implementation.
 *
 * Who needs it: callers that cannot allocate device memory at the moment
 * they call into the library -- a serving process whose whole HBM budget is
 * carved up up front by its own arena allocator and which forbids any other
 * cudaMalloc, a C or C++ host that has no PyTorch caching allocator to borrow
 * a scratch buffer from, and code on a latency-critical path that cannot take
 * cudaMalloc's implicit device synchronisation.  The entry points below take
 * their scratch memory from a fixed array compiled into the library instead
 * of from the caller.
 *
 * Link against graspo_b200/_C*.so (the symbol is exported with C linkage).
 *
 * Contract of graspo_paged_decode_attention_noalloc:
 *   - Inputs and outputs are device pointers on the current device; the work
 *     is queued on `stream`.  Nothing is allocated: no cudaMalloc, cudaFree or
 *     allocating library routine is called.
 *   - Scratch limit: rows * nq * splits * (128 + 2) floats must not exceed
 *     GRASPO_NOALLOC_SCRATCH_FLOATS (2^20 floats, 4 MiB) and rows * nkv must
 *     not exceed GRASPO_NOALLOC_MAX_COUNTERS (8192); larger requests return
 *     GB_NOALLOC_TOO_LARGE and launch nothing.  Every GPU that loads the
 *     library holds this memory until the process exits.
 *   - The first call on a device resolves the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.
 *   - All calls share the one array, which keeps the last call's contents
 *     (the arrival counters are cleared on `stream` before every launch).
 *     Calls that can overlap on the GPU (unordered streams) race on the
 *     array: issue them on one stream or order them.
 *   - Block-table entries must lie in [0, num_pages); builds compiled with
 *     GRASPO_KERNEL_CHECKS report an entry outside that range in `err`
 *     (kErrBadIndex) and clamp it.  `err` may be NULL.
 */
#ifndef GRASPO_NOALLOC_H_
#define GRASPO_NOALLOC_H_

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GRASPO_NOALLOC_SCRATCH_FLOATS (1L << 20)
#define GRASPO_NOALLOC_MAX_COUNTERS 8192

typedef enum GbNoAllocStatus {
  GB_NOALLOC_OK = 0,
  GB_NOALLOC_TOO_LARGE = 1,     /* scratch or counters beyond the fixed array */
  GB_NOALLOC_BAD_ARGUMENT = 2,  /* null pointer, non-positive size, nq % nkv != 0, G not in {1,2,4,8}, splits < 2 */
  GB_NOALLOC_SETUP_FAILED = 3,  /* cudaGetSymbolAddress failed */
  GB_NOALLOC_LAUNCH_FAILED = 4, /* the counter clear or the kernel launch failed */
  GB_NOALLOC_BAD_DEVICE = 5,    /* no current device, or a device index >= 64 */
} GbNoAllocStatus;

/* Split-KV paged decode attention (one query token per row).
 *   q           [rows, nq, 128] bf16
 *   k_pool      [num_pages, nkv, page_size, 128] bf16 (v_pool alike)
 *   block_table [rows, max_pages] int32 page indices
 *   start, len  [rows] int32: row r attends its keys [start[r], len[r])
 *   out         [rows, nq * 128] bf16
 * Query head h reads key/value head h / (nq / nkv).  Returns a GbNoAllocStatus;
 * nothing is queued unless it returns GB_NOALLOC_OK. */
int graspo_paged_decode_attention_noalloc(const void* q, const void* k_pool, const void* v_pool,
                                          const int* block_table, const int* start, const int* len, void* out,
                                          int rows, int nq, int nkv, int page_size, int max_pages, int num_pages,
                                          int splits, float scale, int* err, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GRASPO_NOALLOC_H_ */
