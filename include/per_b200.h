/*
 * per_b200.h - C ABI of the B200 prioritized-replay engine.
 *
 * The engine keeps the two-level priority store of triton-per
 * (src/triton_per/buffer.py:20-63: float32 leaf priorities padded to
 * BLOCK_P = 1024 per block, plus one float32 partial sum per block) and widens
 * it into a 32-ary sum tree whose fan-out equals the warp width:
 *
 *   level 0   leaf priorities                       float32[capacity_padded]
 *   level 1   sums of 32 leaves ("chunks")          float32
 *   level 2   sums of 32 chunks = 1024-leaf blocks  float32   (== block_sums)
 *   level k   sums of 32 level k-1 nodes            float32   (only when needed)
 *
 * Each level step of a sample is one coalesced 128-byte warp load plus a warp
 * scan; the highest level the sampler needs ("top level", at most
 * PER_TOP_MAX nodes) is staged as a float64 prefix in shared memory.
 *
 * Conventions of every entry point:
 *   - plain device pointers and sizes; no framework types;
 *   - the caller allocates every buffer (per_layout() gives the sizes) and
 *     keeps ownership; the library never allocates or frees device memory in
 *     these entry points and never synchronises the host;
 *   - all work is enqueued on `stream` (a cudaStream_t passed as void*,
 *     NULL = legacy default stream), in stream order, like the reference's
 *     kernels on the caller's current stream;
 *   - return 0 (PER_OK) or a PER_ERR_* code; per_error_string() names it and
 *     per_last_cuda_error() gives the CUDA error code behind PER_ERR_CUDA;
 *   - calls on one store must not overlap on the GPU (one stream, or events);
 *     the reference buffer is single-threaded in the same way.
 *
 * Device-side events that the host cannot see at launch time (barrier
 * timeouts, indices out of range, rounding fallbacks) are counted in the
 * store's `status` words; see PER_STATUS_*.
 */
#ifndef PER_B200_H
#define PER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PER_ABI_VERSION 2

#define PER_BLOCK_P 1024   /* leaves per block: reference buffer.py:20 BLOCK_P */
#define PER_FANOUT 32      /* children per tree node (= warp width) */
#define PER_LOG_FANOUT 5
#define PER_MAX_LEVELS 7   /* levels 0..6: up to 2^30 leaves */
#define PER_TOP_MAX 4096   /* max nodes of the level staged in shared memory */
#define PER_MAX_FIELDS 16  /* max fields of one add() call */
#define PER_STATUS_WORDS 16
#define PER_MAX_GRID 4096  /* max CTAs of one grid-synchronised launch */
#define PER_SCRATCH_BYTES (256 + 4 * PER_MAX_GRID)
#define PER_MAX_SHARDS 64  /* shards of one sharded buffer */
#define PER_MAILBOX_BYTES 8192  /* peer-memory mailbox of one rank */
#define PER_IPC_HANDLE_BYTES 64

/* return codes */
#define PER_OK 0
#define PER_ERR_INVALID_ARGUMENT 1
#define PER_ERR_NULL_POINTER 2
#define PER_ERR_EMPTY 3
#define PER_ERR_TOO_LARGE 4
#define PER_ERR_MISALIGNED 5
#define PER_ERR_CUDA 6
#define PER_ERR_NO_DEVICE 7

/* status[] word indices (device uint32 counters / bit sets) */
#define PER_STATUS_ERRORS 0        /* bit set of PER_EVT_* error bits */
#define PER_STATUS_FALLBACKS 1     /* draws that met a rounding / overflow fallback in the tree walk */
#define PER_STATUS_ZERO_WALKS 2    /* draws whose clamped slot had p == 0 and walked back */
#define PER_STATUS_CLAMPS 3        /* draws clamped to size-1 */
#define PER_STATUS_BAD_INDICES 4   /* update indices outside [0, capacity) (skipped) */
#define PER_STATUS_TIMEOUTS 5      /* grid-barrier waits that gave up */
#define PER_STATUS_FOREIGN 6       /* sharded: indices owned by another shard (skipped) */

#define PER_EVT_BARRIER_TIMEOUT 0x1u
#define PER_EVT_EMPTY_BUFFER 0x2u
#define PER_EVT_BAD_INDEX 0x4u
#define PER_EVT_INCONSISTENT_TREE 0x8u
#define PER_EVT_PEER_TIMEOUT 0x10u

/* Sizes of every array of a store of `capacity` slots. */
typedef struct per_layout {
  int64_t capacity;
  int64_t capacity_padded;              /* ceil(capacity / 1024) * 1024 */
  int64_t num_blocks;                   /* ceil(capacity / 1024) */
  int32_t num_levels;                   /* levels maintained, >= 3 */
  int32_t top_level;                    /* level staged in shared memory by the sampler */
  int64_t level_nodes[PER_MAX_LEVELS];  /* live nodes per level: ceil(capacity / 32^k) */
  int64_t level_len[PER_MAX_LEVELS];    /* allocated float32 entries per level (padded) */
  int64_t scratch_bytes;                /* bytes of `scratch` */
} per_layout_t;

/* One replay store: device pointers owned by the caller. */
typedef struct per_store {
  float* levels[PER_MAX_LEVELS];    /* levels[0] = priorities, levels[2] = block sums */
  uint32_t* claims[PER_MAX_LEVELS]; /* zeroed scratch, level_len[k] words each, for k < num_levels */
  int64_t level_len[PER_MAX_LEVELS];
  int32_t num_levels;
  int32_t top_level;
  int64_t capacity;
  float* storage;          /* float32 rows, row i at storage + i * row_stride */
  int64_t row_dim;
  int64_t row_stride;      /* elements, >= row_dim */
  int64_t* size_cursor;    /* device int64[2]: live size, ring cursor */
  float* max_priority;     /* device float32 scalar, already ^alpha (buffer.py:59) */
  uint32_t* status;        /* device uint32[PER_STATUS_WORDS] */
  void* scratch;           /* device, scratch_bytes, zeroed once at creation */
  int64_t scratch_bytes;
  float alpha;             /* buffer.py:29 */
  float eps;               /* buffer.py:30 */
  /* bytes per row element: 4 (or 0) = float32 rows as in the reference;
   * 2 = 16-bit rows (bfloat16 / float16, stored and gathered bit for bit,
   * half the row bytes; not in the reference, whose rows are float32,
   * buffer.py:52). With 2: row_dim, row_stride, every out_stride and every
   * field's dim, stride and col_offset must be even (elements move in
   * pairs), and `out` / field data point at 16-bit elements. */
  int32_t elem_bytes;
} per_store_t;

/* One field of an add() batch: rows [n, dim] of the store's element type
 * (float32, or 16-bit with elem_bytes 2) with a row stride. */
typedef struct per_field {
  const float* data;
  int64_t dim;
  int64_t stride;      /* elements between consecutive rows of `data` */
  int64_t col_offset;  /* first column of this field inside a storage row */
} per_field_t;

/* Storage row stride (elements) the engine recommends for rows of
 * `row_dim` float32 values: a multiple of 4 (16-byte rows, so rows can be
 * copied by the Tensor Memory Accelerator) and, when it costs at most 1/8
 * more memory, of 16 (64-byte rows, fewer DRAM lines per row).
 * Replaces the packed row layout of reference buffer.py:41,52. */
int64_t per_row_stride(int64_t row_dim);

/* Fill `out` with the array sizes for a store of `capacity` slots.
 * Replaces the sizing in reference buffer.py:48-54. */
int per_layout(int64_t capacity, per_layout_t* out);

/* Fused prioritized sample: tree search + row gather + importance weights
 * normalised by the batch maximum, in one launch.
 * For j < batch: u_j = rand[j] * total (float32), idx[j] = first slot whose
 * inclusive priority prefix exceeds u_j, clamped to size-1; out row j =
 * storage row idx[j]; w[j] = (size * p / total)^-beta / max_j(...).
 * Replaces reference buffer.py:82-94 (sample, w / w.max()), buffer.py:107-130
 * (_sample_triton) and kernels/fused.py:16-52 (fused_sample_kernel) with
 * kernels/sampling.py:16-56 (_find_index).
 * `out_stride` is in elements (>= row_dim). */
int per_sample_fused(const per_store_t* store, const float* rand, int64_t batch,
                     float beta, float* out, int64_t out_stride, int64_t* idx,
                     float* w, void* stream);

/* per_sample_fused() with the uniforms drawn inside the kernel instead of
 * read from `rand`: rand[j] = Philox4x32-10 (Salmon et al., SC 2011) with key
 * `seed` and counter *counter + j (first output word, top 24 bits * 2^-24);
 * the kernel then advances the device word *counter by `batch`, so repeated
 * calls (and CUDA-graph replays) continue the stream. Replaces the
 * torch.rand(batch) launch of reference buffer.py:85. */
int per_sample_fused_rng(const per_store_t* store, uint64_t seed, uint64_t* counter,
                         int64_t batch, float beta, float* out, int64_t out_stride,
                         int64_t* idx, float* w, void* stream);

/* p_i <- (|td_i| + eps)^alpha for every i, max-priority tracking, and exact
 * recomputation of every touched chunk / block / upper node. Duplicate
 * indices resolve deterministically: the last occurrence wins.
 * Replaces reference buffer.py:133-162 (update_priorities, including the
 * periodic exact refresh) and kernels/update.py:14-35 (update_kernel). */
int per_update_priorities(const per_store_t* store, const int64_t* idx,
                          const float* td, int64_t n, void* stream);

/* Ring insert of n transitions at the device cursor: rows are written from
 * the field arrays, new leaves get the current max priority, touched tree
 * nodes are recomputed exactly, and size/cursor advance on the device.
 * Replaces reference buffer.py:66-79 (add) without its host synchronisation. */
int per_add(const per_store_t* store, const per_field_t* fields,
            int32_t n_fields, int64_t n, void* stream);

/* Allocation-free variant of per_update_priorities(), for callers that cannot
 * allocate device memory (an application that fixes the library's device
 * memory at start-up and forbids later allocations, or a latency-critical
 * path where cudaMalloc would synchronise the device). No counterpart in the
 * reference: triton-per allocates through PyTorch.
 * The claim words and grid-barrier words that per_update_priorities() takes
 * from store->claims and store->scratch come instead from a scratch array
 * compiled into the library (PER_NOALLOC_SCRATCH_BYTES, held on every GPU
 * that loads the library until exit); store->claims and store->scratch may be
 * NULL. Stores of more than PER_NOALLOC_MAX_CAPACITY slots are rejected with
 * PER_ERR_TOO_LARGE. The first call on a device resolves the array's device
 * address (cudaGetSymbolAddress, with that device current): make it before
 * any stream capture; after cudaDeviceReset() on that device the cached
 * address is stale, so do not call it there again. Batches of up to 2048
 * indices use none of the array; larger ones first clear, on `stream`, the
 * words they use. Calls that overlap on the GPU share the array and race:
 * serialise them.
 * Calls no cudaMalloc, cudaFree or allocating library routine. */
#define PER_NOALLOC_MAX_CAPACITY 1048576
#define PER_NOALLOC_SCRATCH_BYTES 4346368
int per_update_priorities_noalloc(const per_store_t* store, const int64_t* idx,
                                  const float* td, int64_t n, void* stream);

/* Recompute every tree level above the leaves from the leaves and clear the
 * claim scratch. Call after writing priorities directly.
 * Replaces the exact refresh of reference buffer.py:156-162. */
int per_rebuild_sums(const per_store_t* store, void* stream);

/* ---- sharded mode (no counterpart in the reference, which has no
 * multi-GPU code). Shard g of `world` owns global slots
 * [g * shard_capacity, (g + 1) * shard_capacity) in its own store. All shards
 * draw the same global uniforms; a draw belongs to the shard whose range of
 * the global priority prefix holds u = rand * total, so the union of the
 * shards' draws equals the draw of one buffer holding every slot. */

/* stats[0] = total priority of this shard (float64), stats[1] = its live
 * size; the caller all-gathers these into a [world][2] array. */
int per_shard_stats(const per_store_t* store, double* stats, void* stream);

/* per_sample_fused() for shard `rank` of `world`: `stats` is the all-gathered
 * [world][2] array, `rand` the `batch` global uniforms (identical on every
 * shard). The draws this shard owns are searched, gathered and weighted with
 * the global size and total, then compacted into out/idx/w/pos (pos = global
 * draw position; the order of the compacted draws is unspecified; idx
 * entries past them are set to -1); *count receives their number and
 * *local_max their max unnormalised weight. The
 * caller reduces local_max over the shards (max) and calls per_normalize().
 * Replaces, per shard, reference buffer.py:82-105 and fused.py:16-52. */
int per_sample_sharded(const per_store_t* store, int32_t rank, int32_t world,
                       int64_t shard_base, const double* stats, const float* rand,
                       int64_t batch, float beta, float* out, int64_t out_stride,
                       int64_t* idx, float* w, int32_t* pos, int64_t* count,
                       float* local_max, void* stream);

/* per_sample_sharded() with in-kernel Philox uniforms (as per_sample_fused_rng;
 * the same seed and counter on every shard give every shard the same draws). */
int per_sample_sharded_rng(const per_store_t* store, int32_t rank, int32_t world,
                           int64_t shard_base, const double* stats, uint64_t seed,
                           uint64_t* counter, int64_t batch, float beta, float* out,
                           int64_t out_stride, int64_t* idx, float* w, int32_t* pos,
                           int64_t* count, float* local_max, void* stream);

/* Peer-memory exchange (one process per GPU, GPUs connected by NVLink):
 * each rank creates one mailbox, exports it as a CUDA IPC handle, and maps the
 * handles of all peers. per_mailbox_create also zeroes the mailbox. These are
 * set-up / tear-down calls (they allocate and map device memory). */
int per_mailbox_create(void** mailbox, void* ipc_handle);
int per_mailbox_open(const void* ipc_handle, void** mailbox);
int per_mailbox_close(void* peer_mailbox);
int per_mailbox_destroy(void* mailbox);

/* per_sample_sharded() with both exchanges done inside the kernel over peer
 * memory instead of by the caller: the shard statistics and the max weight
 * are written into slot `rank` of every rank's mailbox (`mailboxes`: a device
 * array of `world` mailbox pointers as mapped in this process, own included)
 * with system-scope release stores, and read back from this rank's mailbox
 * after bounded waits; the weights come out normalised. Every rank must make
 * the same sequence of calls (collective). batch must fit one wave of the
 * kernel (PER_ERR_TOO_LARGE otherwise: use per_sample_sharded()). A peer that
 * does not publish within about a second sets PER_EVT_PEER_TIMEOUT; the
 * ranks' sequence numbers then disagree and the mailboxes must be destroyed
 * and created again before the next call. The ranks' kernels wait on one
 * another, so each rank must run on its own GPU. No counterpart in the
 * reference (single GPU); the exchange it replaces is the host-side
 * all-gather / all-reduce around per_sample_sharded(). */
int per_sample_sharded_p2p(const per_store_t* store, int32_t rank, int32_t world,
                           int64_t shard_base, void* const* mailboxes, const float* rand,
                           int64_t batch, float beta, float* out, int64_t out_stride,
                           int64_t* idx, float* w, int32_t* pos, int64_t* count,
                           void* stream);

/* per_sample_sharded_p2p() with in-kernel Philox uniforms. */
int per_sample_sharded_p2p_rng(const per_store_t* store, int32_t rank, int32_t world,
                               int64_t shard_base, void* const* mailboxes, uint64_t seed,
                               uint64_t* counter, int64_t batch, float beta, float* out,
                               int64_t out_stride, int64_t* idx, float* w, int32_t* pos,
                               int64_t* count, void* stream);

/* per_sample_sharded_p2p_rng() with each rank's weights normalised by the
 * largest weight among the draws that rank owns, instead of the largest of
 * the whole global batch: the second exchange (the max weight, one more
 * NVLink round trip per call) is left out. Indices, rows and the unnormalised
 * weights are those of per_sample_sharded_p2p_rng(); only the scale of each
 * rank's weights differs (a per-rank constant), as when each rank normalises
 * its own batch. No counterpart in the reference (single GPU; buffer.py:92
 * normalises by the batch max). Ranks may run one call apart; the mailbox
 * keeps the statistics of two consecutive calls. */
int per_sample_sharded_p2p_local_rng(const per_store_t* store, int32_t rank, int32_t world,
                                     int64_t shard_base, void* const* mailboxes, uint64_t seed,
                                     uint64_t* counter, int64_t batch, float beta, float* out,
                                     int64_t out_stride, int64_t* idx, float* w, int32_t* pos,
                                     int64_t* count, void* stream);

/* Largest batch per_sample_sharded_p2p() accepts for this store on the
 * current device (one wave of co-resident CTAs, one tile per warp). */
int per_sample_sharded_p2p_max_batch(const per_store_t* store, int64_t* max_batch);

/* w[j] /= *gmax for j < min(*count, cap) (device count and max). */
int per_normalize(float* w, const int64_t* count, const float* gmax, int64_t cap, void* stream);

/* per_update_priorities() with global indices: slot = idx - base; indices
 * owned by other shards (or negative padding) are skipped and counted in
 * status[PER_STATUS_FOREIGN]. Replaces, per shard, reference
 * buffer.py:133-162. */
int per_update_priorities_shard(const per_store_t* store, int64_t base, const int64_t* idx,
                                const float* td, int64_t n, void* stream);

/* per_update_priorities_shard() applied to the first min(n, *count) entries
 * only (`count` is a device int64, e.g. the count written by a sharded
 * sample, whose idx array is padded with -1 past it): the host sizes the
 * launch for n without reading the device count. */
int per_update_priorities_shard_count(const per_store_t* store, int64_t base, const int64_t* idx,
                                      const float* td, int64_t n, const int64_t* count,
                                      void* stream);

/* Human-readable name of a PER_* return code. */
const char* per_error_string(int code);

/* cudaError_t value behind the last PER_ERR_CUDA returned on this thread. */
int per_last_cuda_error(void);

/* PER_ABI_VERSION of the loaded library. */
int per_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PER_B200_H */
