// extern "C" entry points: argument checks, layout, launch plumbing.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "per_b200.h"
#include "per_internal.h"

#include <nvtx3/nvToolsExt.h>

namespace {

// NVTX range around an entry point (profilers show each call; without a
// profiler attached this is a few tens of nanoseconds)
struct PerRange {
  explicit PerRange(const char* name) { nvtxRangePushA(name); }
  ~PerRange() { nvtxRangePop(); }
};


thread_local int g_last_cuda = 0;

struct OccEntry {
  int device;
  const void* fn;
  int threads;
  size_t smem;
  int ctas;
};
constexpr int kOccSlots = 256;
OccEntry g_occ[kOccSlots];
int g_occ_n = 0;
std::mutex g_occ_mu;

// Grid-synchronising kernels never exceed the co-resident CTA count of an
// idle GPU and bound every wait, so they are launched like the others (with
// the programmatic dependency), in graphs and eagerly. PER_COOPERATIVE=1
// launches them cooperatively outside stream capture instead: the runtime then
// guarantees co-residency even next to other streams' kernels, at about 1 us
// more host and device time per launch.
bool cooperative_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("PER_COOPERATIVE");
    v = (s && s[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

// Launches carry a programmatic dependency on the previous kernel of the
// stream (the kernel may start early and waits with griddepcontrol.wait),
// except cooperative launches; PER_PDL=0 turns it off.
bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("PER_PDL");
    v = (s && s[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

}  // namespace

PerTree per_tree_of(const per_store_t* s) {
  PerTree t;
  for (int k = 0; k < PER_MAX_LEVELS; ++k) {
    t.levels[k] = s->levels[k];
    t.claims[k] = s->claims[k];
    t.level_len[k] = s->level_len[k];
  }
  t.num_levels = s->num_levels;
  t.top_level = s->top_level;
  t.capacity = s->capacity;
  // 16-bit rows travel as pairs of elements in 4-byte words: the kernels see
  // float32-sized words (row sizes and strides in words)
  t.storage = s->storage;
  t.row_dim = s->elem_bytes == 2 ? s->row_dim / 2 : s->row_dim;
  t.row_stride = s->elem_bytes == 2 ? s->row_stride / 2 : s->row_stride;
  t.size_cursor = s->size_cursor;
  t.max_priority = s->max_priority;
  t.status = s->status;
  t.scratch = reinterpret_cast<PerScratch*>(s->scratch);
  t.alpha = s->alpha;
  t.eps = s->eps;
  return t;
}

int per_check_store(const per_store_t* s, bool with_scratch) {
  if (!s) return PER_ERR_NULL_POINTER;
  per_layout_t l;
  int rc = per_layout(s->capacity, &l);
  if (rc) return rc;
  if (s->num_levels != l.num_levels || s->top_level != l.top_level) return PER_ERR_INVALID_ARGUMENT;
  for (int k = 0; k < l.num_levels; ++k) {
    if (!s->levels[k] || (with_scratch && !s->claims[k])) return PER_ERR_NULL_POINTER;
    if (s->level_len[k] != l.level_len[k]) return PER_ERR_INVALID_ARGUMENT;
    if (((uintptr_t)s->levels[k]) % 16) return PER_ERR_MISALIGNED;
  }
  if (!s->storage || !s->size_cursor || !s->max_priority || !s->status)
    return PER_ERR_NULL_POINTER;
  if (with_scratch) {
    if (!s->scratch) return PER_ERR_NULL_POINTER;
    if (s->scratch_bytes < PER_SCRATCH_BYTES) return PER_ERR_INVALID_ARGUMENT;
    if (((uintptr_t)s->scratch) % 16) return PER_ERR_MISALIGNED;
  }
  if (((uintptr_t)s->storage) % 4) return PER_ERR_MISALIGNED;
  if (s->row_dim < 1 || s->row_stride < s->row_dim) return PER_ERR_INVALID_ARGUMENT;
  if (!(s->eps >= 0.f) || !(s->alpha == s->alpha)) return PER_ERR_INVALID_ARGUMENT;
  if (s->elem_bytes != 0 && s->elem_bytes != 4 && s->elem_bytes != 2) return PER_ERR_INVALID_ARGUMENT;
  if (s->elem_bytes == 2 && (s->row_dim % 2 || s->row_stride % 2)) return PER_ERR_INVALID_ARGUMENT;
  return PER_OK;
}

namespace {

PerTree tree_of(const per_store_t* s) { return per_tree_of(s); }

// Checks that a store descriptor is self-consistent with per_layout().
int check_store(const per_store_t* s) { return per_check_store(s, true); }

// out_stride (elements of the store) in the kernels' 4-byte words; -1 if a
// 16-bit store gets an odd stride
int64_t out_words(const per_store_t* s, int64_t out_stride) {
  if (s->elem_bytes != 2) return out_stride;
  return out_stride % 2 ? -1 : out_stride / 2;
}

}  // namespace

int per_record_cuda(cudaError_t e) {
  g_last_cuda = (int)e;
  return PER_ERR_CUDA;
}

int per_coresident_ctas(const void* fn, int threads, size_t smem, int* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return per_record_cuda(e);
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    for (int i = 0; i < g_occ_n; ++i) {
      const OccEntry& o = g_occ[i];
      if (o.device == dev && o.fn == fn && o.threads == threads && o.smem == smem) {
        *out = o.ctas;
        return PER_OK;
      }
    }
  }
  int sms = 0, per_sm = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return per_record_cuda(e);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
  if (e != cudaSuccess) return per_record_cuda(e);
  if (per_sm < 1) return PER_ERR_TOO_LARGE;
  const int ctas = sms * per_sm;
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    if (g_occ_n < kOccSlots) g_occ[g_occ_n++] = OccEntry{dev, fn, threads, smem, ctas};
  }
  *out = ctas;
  return PER_OK;
}

int per_set_smem(const void* fn, size_t smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return per_record_cuda(e);
  static std::mutex mu;
  static struct {
    int device;
    const void* fn;
    size_t smem;
  } done[64];
  static int n_done = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n_done; ++i)
    if (done[i].device == dev && done[i].fn == fn && done[i].smem >= smem) return PER_OK;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return per_record_cuda(e);
  // prefer the largest shared-memory carveout, so that several CTAs fit per SM
  e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return per_record_cuda(e);
  for (int i = 0; i < n_done; ++i)
    if (done[i].device == dev && done[i].fn == fn) {
      done[i].smem = smem;
      return PER_OK;
    }
  if (n_done < 64) done[n_done++] = {dev, fn, smem};
  return PER_OK;
}

cudaError_t per_launch(const void* fn, unsigned grid, unsigned threads, size_t smem,
                       cudaStream_t stream, void** args, bool grid_sync) {
  bool coop = grid_sync && cooperative_enabled();
  if (coop) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(stream, &cs);
    if (e != cudaSuccess) return e;
    if (cs != cudaStreamCaptureStatusNone) coop = false;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (coop) {
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  } else {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = (coop || pdl_enabled()) ? 1 : 0;
  cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

extern "C" {

int per_abi_version(void) { return PER_ABI_VERSION; }

int per_last_cuda_error(void) { return g_last_cuda; }

const char* per_error_string(int code) {
  switch (code) {
    case PER_OK: return "ok";
    case PER_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PER_ERR_NULL_POINTER: return "null pointer";
    case PER_ERR_EMPTY: return "empty input";
    case PER_ERR_TOO_LARGE: return "size exceeds a supported maximum";
    case PER_ERR_MISALIGNED: return "misaligned pointer or stride";
    case PER_ERR_CUDA: return "CUDA error (see per_last_cuda_error)";
    case PER_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown error";
  }
}

int64_t per_row_stride(int64_t row_dim) {
  if (row_dim < 1) return 0;
  if (row_dim < 4) return row_dim;
  const int64_t s16 = (row_dim + 15) / 16 * 16;
  if ((s16 - row_dim) * 8 <= row_dim) return s16;
  return (row_dim + 3) / 4 * 4;
}

int per_layout(int64_t capacity, per_layout_t* out) {
  if (!out) return PER_ERR_NULL_POINTER;
  if (capacity < 1) return PER_ERR_INVALID_ARGUMENT;
  if (capacity > ((int64_t)1 << 30)) return PER_ERR_TOO_LARGE;
  memset(out, 0, sizeof(*out));
  out->capacity = capacity;
  out->num_blocks = (capacity + PER_BLOCK_P - 1) / PER_BLOCK_P;
  out->capacity_padded = out->num_blocks * PER_BLOCK_P;
  int top = -1;
  for (int k = 0; k < PER_MAX_LEVELS; ++k) {
    const int64_t span = (int64_t)1 << (PER_LOG_FANOUT * k);
    out->level_nodes[k] = (capacity + span - 1) / span;
    if (top < 0 && k >= 1 && out->level_nodes[k] <= PER_TOP_MAX) top = k;
  }
  if (top < 0) return PER_ERR_TOO_LARGE;
  out->top_level = top;
  out->num_levels = top + 1 > 3 ? top + 1 : 3;
  out->level_len[0] = out->capacity_padded;
  for (int k = 1; k < out->num_levels; ++k)
    out->level_len[k] = (out->level_nodes[k] + PER_FANOUT - 1) / PER_FANOUT * PER_FANOUT;
  out->scratch_bytes = PER_SCRATCH_BYTES;
  return PER_OK;
}

namespace {

// rand XOR rng: caller-provided uniforms, or the in-kernel Philox stream
int sample_fused(const per_store_t* store, const float* rand, const PerRng* rng, int64_t batch,
                 float beta, float* out, int64_t out_stride, int64_t* idx, float* w,
                 void* stream) {
  int rc = check_store(store);
  if (rc) return rc;
  if ((!rand && !rng) || !out || !idx || !w) return PER_ERR_NULL_POINTER;
  if (rng && !rng->counter) return PER_ERR_NULL_POINTER;
  if (batch < 1) return PER_ERR_EMPTY;
  if (batch > ((int64_t)1 << 31)) return PER_ERR_TOO_LARGE;
  if (out_stride < store->row_dim) return PER_ERR_INVALID_ARGUMENT;
  const int64_t ow = out_words(store, out_stride);
  if (ow < 0) return PER_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)out) % 4 || ((uintptr_t)idx) % 8 || ((uintptr_t)w) % 4 || ((uintptr_t)rand) % 4 ||
      (rng && ((uintptr_t)rng->counter) % 8))
    return PER_ERR_MISALIGNED;
  return per_launch_sample(tree_of(store), rand, rng, batch, beta, out, ow, idx, w,
                           (cudaStream_t)stream);
}

int sample_sharded(const per_store_t* store, int32_t rank, int32_t world, int64_t shard_base,
                   const double* stats, const float* rand, const PerRng* rng, int64_t batch,
                   float beta, float* out, int64_t out_stride, int64_t* idx, float* w,
                   int32_t* pos, int64_t* count, float* local_max, void* stream) {
  int rc = check_store(store);
  if (rc) return rc;
  if (!stats || (!rand && !rng) || !out || !idx || !w || !pos || !count || !local_max)
    return PER_ERR_NULL_POINTER;
  if (rng && !rng->counter) return PER_ERR_NULL_POINTER;
  if (world < 1 || world > PER_MAX_SHARDS || rank < 0 || rank >= world || shard_base < 0)
    return PER_ERR_INVALID_ARGUMENT;
  if (batch < 1) return PER_ERR_EMPTY;
  if (batch > ((int64_t)1 << 31)) return PER_ERR_TOO_LARGE;
  if (out_stride < store->row_dim) return PER_ERR_INVALID_ARGUMENT;
  const int64_t ow = out_words(store, out_stride);
  if (ow < 0) return PER_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)out) % 4 || ((uintptr_t)idx) % 8 || ((uintptr_t)w) % 4 || ((uintptr_t)rand) % 4 ||
      ((uintptr_t)stats) % 8 || ((uintptr_t)pos) % 4 || ((uintptr_t)count) % 8 ||
      (rng && ((uintptr_t)rng->counter) % 8))
    return PER_ERR_MISALIGNED;
  return per_launch_sample_sharded(tree_of(store), rank, world, shard_base, stats, rand, rng,
                                   batch, beta, out, ow, idx, w, pos, count, local_max,
                                   (cudaStream_t)stream);
}

int sample_sharded_p2p(const per_store_t* store, int32_t rank, int32_t world, int64_t shard_base,
                       void* const* mailboxes, const float* rand, const PerRng* rng, int64_t batch,
                       float beta, float* out, int64_t out_stride, int64_t* idx, float* w,
                       int32_t* pos, int64_t* count, int32_t local_norm, void* stream) {
  int rc = check_store(store);
  if (rc) return rc;
  if (!mailboxes || (!rand && !rng) || !out || !idx || !w || !pos || !count)
    return PER_ERR_NULL_POINTER;
  if (rng && !rng->counter) return PER_ERR_NULL_POINTER;
  if (world < 1 || world > PER_MAX_SHARDS || rank < 0 || rank >= world || shard_base < 0)
    return PER_ERR_INVALID_ARGUMENT;
  if (batch < 1) return PER_ERR_EMPTY;
  if (batch > ((int64_t)1 << 31)) return PER_ERR_TOO_LARGE;
  if (out_stride < store->row_dim) return PER_ERR_INVALID_ARGUMENT;
  const int64_t ow = out_words(store, out_stride);
  if (ow < 0) return PER_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)out) % 4 || ((uintptr_t)idx) % 8 || ((uintptr_t)w) % 4 || ((uintptr_t)rand) % 4 ||
      ((uintptr_t)pos) % 4 || ((uintptr_t)count) % 8 || ((uintptr_t)mailboxes) % 8 ||
      (rng && ((uintptr_t)rng->counter) % 8))
    return PER_ERR_MISALIGNED;
  return per_launch_sample_sharded_p2p(tree_of(store), rank, world, shard_base,
                                       reinterpret_cast<PerMailbox* const*>(mailboxes), rand, rng,
                                       batch, beta, out, ow, idx, w, pos, count, local_norm,
                                       (cudaStream_t)stream);
}

}  // namespace

int per_sample_fused(const per_store_t* store, const float* rand, int64_t batch, float beta,
                     float* out, int64_t out_stride, int64_t* idx, float* w, void* stream) {
  PerRange range("per_sample_fused");
  if (!rand) return PER_ERR_NULL_POINTER;
  return sample_fused(store, rand, nullptr, batch, beta, out, out_stride, idx, w, stream);
}

int per_sample_fused_rng(const per_store_t* store, uint64_t seed, uint64_t* counter, int64_t batch,
                         float beta, float* out, int64_t out_stride, int64_t* idx, float* w,
                         void* stream) {
  PerRange range("per_sample_fused_rng");
  const PerRng rng{(unsigned long long)seed, reinterpret_cast<unsigned long long*>(counter)};
  return sample_fused(store, nullptr, &rng, batch, beta, out, out_stride, idx, w, stream);
}

int per_update_priorities(const per_store_t* store, const int64_t* idx, const float* td, int64_t n,
                          void* stream) {
  PerRange range("per_update_priorities");
  int rc = check_store(store);
  if (rc) return rc;
  if (!idx || !td) return PER_ERR_NULL_POINTER;
  if (n < 1) return PER_ERR_EMPTY;
  if (n >= (int64_t)0xffffffffLL) return PER_ERR_TOO_LARGE;
  return per_launch_update(tree_of(store), idx, td, n, (cudaStream_t)stream);
}

int per_add(const per_store_t* store, const per_field_t* fields, int32_t n_fields, int64_t n,
            void* stream) {
  PerRange range("per_add");
  int rc = check_store(store);
  if (rc) return rc;
  if (n < 0) return PER_ERR_INVALID_ARGUMENT;
  if (n == 0) return PER_OK;
  if (!fields) return PER_ERR_NULL_POINTER;
  if (n_fields < 1 || n_fields > PER_MAX_FIELDS) return PER_ERR_INVALID_ARGUMENT;
  int64_t covered = 0;
  for (int f = 0; f < n_fields; ++f) {
    const per_field_t& fd = fields[f];
    if (!fd.data) return PER_ERR_NULL_POINTER;
    if (fd.dim < 1 || fd.stride < fd.dim || fd.col_offset < 0 ||
        fd.col_offset + fd.dim > store->row_dim)
      return PER_ERR_INVALID_ARGUMENT;
    covered += fd.dim;
  }
  if (covered != store->row_dim) return PER_ERR_INVALID_ARGUMENT;
  if (store->elem_bytes == 2) {  // 16-bit rows: fields move as pairs of elements (words)
    per_field_t words[PER_MAX_FIELDS];
    for (int f = 0; f < n_fields; ++f) {
      const per_field_t& fd = fields[f];
      if (fd.dim % 2 || fd.stride % 2 || fd.col_offset % 2) return PER_ERR_INVALID_ARGUMENT;
      if (((uintptr_t)fd.data) % 4) return PER_ERR_MISALIGNED;
      words[f] = per_field_t{fd.data, fd.dim / 2, fd.stride / 2, fd.col_offset / 2};
    }
    return per_launch_add(tree_of(store), words, n_fields, n, (cudaStream_t)stream);
  }
  return per_launch_add(tree_of(store), fields, n_fields, n, (cudaStream_t)stream);
}

int per_shard_stats(const per_store_t* store, double* out, void* stream) {
  PerRange range("per_shard_stats");
  int rc = check_store(store);
  if (rc) return rc;
  if (!out) return PER_ERR_NULL_POINTER;
  if (((uintptr_t)out) % 8) return PER_ERR_MISALIGNED;
  return per_launch_shard_stats(tree_of(store), out, (cudaStream_t)stream);
}

int per_sample_sharded(const per_store_t* store, int32_t rank, int32_t world, int64_t shard_base,
                       const double* stats, const float* rand, int64_t batch, float beta,
                       float* out, int64_t out_stride, int64_t* idx, float* w, int32_t* pos,
                       int64_t* count, float* local_max, void* stream) {
  PerRange range("per_sample_sharded");
  if (!rand) return PER_ERR_NULL_POINTER;
  return sample_sharded(store, rank, world, shard_base, stats, rand, nullptr, batch, beta, out,
                        out_stride, idx, w, pos, count, local_max, stream);
}

int per_sample_sharded_rng(const per_store_t* store, int32_t rank, int32_t world,
                           int64_t shard_base, const double* stats, uint64_t seed,
                           uint64_t* counter, int64_t batch, float beta, float* out,
                           int64_t out_stride, int64_t* idx, float* w, int32_t* pos,
                           int64_t* count, float* local_max, void* stream) {
  PerRange range("per_sample_sharded_rng");
  const PerRng rng{(unsigned long long)seed, reinterpret_cast<unsigned long long*>(counter)};
  return sample_sharded(store, rank, world, shard_base, stats, nullptr, &rng, batch, beta, out,
                        out_stride, idx, w, pos, count, local_max, stream);
}

int per_mailbox_create(void** mailbox, void* ipc_handle) {
  if (!mailbox || !ipc_handle) return PER_ERR_NULL_POINTER;
  static_assert(sizeof(cudaIpcMemHandle_t) == PER_IPC_HANDLE_BYTES, "ipc handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, PER_MAILBOX_BYTES);
  if (e != cudaSuccess) return per_record_cuda(e);
  e = cudaMemset(p, 0, PER_MAILBOX_BYTES);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return per_record_cuda(e);
  }
  *mailbox = p;
  return PER_OK;
}

int per_mailbox_open(const void* ipc_handle, void** mailbox) {
  if (!mailbox || !ipc_handle) return PER_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(mailbox, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}

int per_mailbox_close(void* peer_mailbox) {
  if (!peer_mailbox) return PER_ERR_NULL_POINTER;
  cudaError_t e = cudaIpcCloseMemHandle(peer_mailbox);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}

int per_mailbox_destroy(void* mailbox) {
  if (!mailbox) return PER_ERR_NULL_POINTER;
  cudaError_t e = cudaFree(mailbox);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}

int per_sample_sharded_p2p(const per_store_t* store, int32_t rank, int32_t world,
                           int64_t shard_base, void* const* mailboxes, const float* rand,
                           int64_t batch, float beta, float* out, int64_t out_stride,
                           int64_t* idx, float* w, int32_t* pos, int64_t* count, void* stream) {
  PerRange range("per_sample_sharded_p2p");
  if (!rand) return PER_ERR_NULL_POINTER;
  return sample_sharded_p2p(store, rank, world, shard_base, mailboxes, rand, nullptr, batch, beta,
                            out, out_stride, idx, w, pos, count, 0, stream);
}

int per_sample_sharded_p2p_rng(const per_store_t* store, int32_t rank, int32_t world,
                               int64_t shard_base, void* const* mailboxes, uint64_t seed,
                               uint64_t* counter, int64_t batch, float beta, float* out,
                               int64_t out_stride, int64_t* idx, float* w, int32_t* pos,
                               int64_t* count, void* stream) {
  PerRange range("per_sample_sharded_p2p_rng");
  const PerRng rng{(unsigned long long)seed, reinterpret_cast<unsigned long long*>(counter)};
  return sample_sharded_p2p(store, rank, world, shard_base, mailboxes, nullptr, &rng, batch, beta,
                            out, out_stride, idx, w, pos, count, 0, stream);
}

int per_sample_sharded_p2p_local_rng(const per_store_t* store, int32_t rank, int32_t world,
                                     int64_t shard_base, void* const* mailboxes, uint64_t seed,
                                     uint64_t* counter, int64_t batch, float beta, float* out,
                                     int64_t out_stride, int64_t* idx, float* w, int32_t* pos,
                                     int64_t* count, void* stream) {
  PerRange range("per_sample_sharded_p2p_local_rng");
  const PerRng rng{(unsigned long long)seed, reinterpret_cast<unsigned long long*>(counter)};
  return sample_sharded_p2p(store, rank, world, shard_base, mailboxes, nullptr, &rng, batch, beta,
                            out, out_stride, idx, w, pos, count, 1, stream);
}

int per_sample_sharded_p2p_max_batch(const per_store_t* store, int64_t* max_batch) {
  int rc = check_store(store);
  if (rc) return rc;
  if (!max_batch) return PER_ERR_NULL_POINTER;
  return per_launch_sample_p2p_max_batch(tree_of(store), max_batch);
}

int per_normalize(float* w, const int64_t* count, const float* gmax, int64_t cap, void* stream) {
  PerRange range("per_normalize");
  if (!w || !count || !gmax) return PER_ERR_NULL_POINTER;
  if (cap < 0) return PER_ERR_INVALID_ARGUMENT;
  if (cap == 0) return PER_OK;
  return per_launch_normalize(w, count, gmax, cap, (cudaStream_t)stream);
}

int per_update_priorities_shard(const per_store_t* store, int64_t base, const int64_t* idx,
                                const float* td, int64_t n, void* stream) {
  PerRange range("per_update_priorities_shard");
  int rc = check_store(store);
  if (rc) return rc;
  if (!idx || !td) return PER_ERR_NULL_POINTER;
  if (base < 0) return PER_ERR_INVALID_ARGUMENT;
  if (n < 1) return PER_ERR_EMPTY;
  if (n >= (int64_t)0xffffffffLL) return PER_ERR_TOO_LARGE;
  return per_launch_update_shard(tree_of(store), base, 0, idx, td, n, nullptr, (cudaStream_t)stream);
}

int per_update_priorities_shard_count(const per_store_t* store, int64_t base, const int64_t* idx,
                                      const float* td, int64_t n, const int64_t* count,
                                      void* stream) {
  PerRange range("per_update_priorities_shard_count");
  int rc = check_store(store);
  if (rc) return rc;
  if (!idx || !td || !count) return PER_ERR_NULL_POINTER;
  if (base < 0) return PER_ERR_INVALID_ARGUMENT;
  if (n < 1) return PER_ERR_EMPTY;
  if (n >= (int64_t)0xffffffffLL) return PER_ERR_TOO_LARGE;
  if (((uintptr_t)count) % 8) return PER_ERR_MISALIGNED;
  return per_launch_update_shard(tree_of(store), base, 0, idx, td, n, count, (cudaStream_t)stream);
}

int per_rebuild_sums(const per_store_t* store, void* stream) {
  PerRange range("per_rebuild_sums");
  int rc = check_store(store);
  if (rc) return rc;
  return per_launch_rebuild(tree_of(store), (cudaStream_t)stream);
}

}  // extern "C"
