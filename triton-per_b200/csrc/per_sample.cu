// Fused prioritized sample: tree search, row gather and normalised IS
// weights in one launch.
//
// Reference behaviour (triton-per):
//   buffer.py:85          rand = torch.rand(B)             (input here)
//   buffer.py:112         block_cumsum = cumsum(block_sums) (per CTA, below)
//   sampling.py:27-55     level-1 bsearch, in-block scan, clamp to size-1,
//                         p reloaded at the clamped index
//   fused.py:35-43        total on device, u = rand * total, w = (size*p/total)^-beta
//   fused.py:45-52        row copy storage[idx] -> out[j]
//   buffer.py:92          w / w.max()
//
// Design (one draw per lane, 32 draws in flight per warp):
//   * Prologue: each CTA stages the float64 exclusive prefix of the top tree
//     level (<= PER_TOP_MAX float32 nodes) in shared memory, padded one slot
//     in 33 so that the power-of-two strides of a binary search spread over
//     the banks; every lane then searches it for its own draw.
//   * Each lower level: the warp copies the 32 children (one 128-byte line)
//     of each of its 32 draws into a shared-memory tile with cp.async (4
//     lines per instruction), then every lane searches the 32 children of its
//     own draw: quad sums, prefix over the 8 quads, then inside the quad.
//   * Arrive: the CTA publishes the max of its unnormalised weights and
//     arrives at a grid barrier, then gathers its rows while the other CTAs
//     finish, then waits, reads the global max and normalises its weights.
//   * Gather: every lane issues one Tensor Memory Accelerator bulk copy of
//     its row (16-byte aligned storage rows) into the warp's tile, completing
//     on the warp's mbarrier; the warp then writes the contiguous output rows
//     with coalesced vector stores. The bulk engine keeps far more row reads
//     in flight per SM than per-thread loads can. Rows that are not 16-byte
//     aligned use cp.async; rows wider than the tile are copied directly.
//   * Small batches use one-warp CTAs so that their rows are fetched by many
//     SMs at once; large batches use 8-warp CTAs.
// Sampling semantics: idx is the first slot whose inclusive prefix exceeds
// u = rand * total (fp32 product, as torch computes it), with prefixes in
// float64 so the result equals a search over exact prefixes; rounding
// fallbacks and empty-slot walk-backs are counted in the status words.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "per_internal.h"

namespace {

constexpr int kMaxWarps = 8;
constexpr int kStageMin = PER_NODE_TILE;
constexpr int kStageMax = 10240;  // per-warp staging bytes for row gathers

struct SampleArgs {
  PerTree t;
  const float* rand;
  int64_t batch;
  float beta;
  float* out;
  int64_t out_stride;
  int64_t* idx;
  float* w;
  int32_t nvec;            // vectors per row
  int32_t rows_per_stage;  // rows per staged batch (0: wide rows, direct copy)
  int32_t stage_bytes;     // per-warp staging bytes
  int32_t row_bytes;       // staged bytes per row (bulk: row_dim*4 rounded up to 16)
  int32_t use_bulk;        // rows are 16-byte aligned: gather with bulk copies
  int32_t gather4;         // bulk gathers take four rows per tensor-map gather
  int32_t group_bytes;     // staging bytes per group of four rows (gather4: 128-byte multiple)
  int32_t cp_bytes;        // cp.async piece size when not using bulk copies (4, 8, 16)
  int32_t pre_bytes;       // shared-memory bytes of the staged top level (128-byte multiple)
  int32_t draws_per_warp;  // draws per warp and tile (32 sharded; fewer for small batches and wide rows)
  int32_t wide;            // rows copied in this kernel piecewise by bulk copies (wide rows)
  int32_t wide_piece;      // wide mode: bytes per piece and per lane of the warp's tile
  int64_t num_tiles;
  // sharded mode: this store is shard `rank` of `world` shards
  const double* stats;           // [world][2] of every shard: total priority, live size
  int32_t rank;
  int32_t world;
  int64_t shard_base;            // global index of this shard's slot 0
  int32_t* pos;                  // global draw position of each compacted draw
  unsigned long long* count;     // draws owned by this shard (compacted output length)
  float* local_max;              // max unnormalised weight over this shard's draws
  PerMailbox* const* mailboxes;  // exchange over peer memory: every rank's mailbox
  int32_t p2p;                   // 1: exchange stats and max in-kernel through the mailboxes
  int32_t local_norm;            // p2p: weights normalised by this rank's max (no max exchange)
  // sharded, in-kernel exchange: each CTA routes its slice of `slice` global
  // draws first and searches only the draws this shard owns
  int32_t owned_only;
  int32_t slice;
  // uniforms from the in-kernel Philox stream instead of `rand`
  int32_t use_rng;
  unsigned long long rng_seed;
  unsigned long long* rng_counter;  // device: draws consumed so far (advanced by the kernel)
};

__device__ __forceinline__ float draw_uniform(const SampleArgs& a, unsigned long long cbase,
                                              int64_t j) {
  return a.use_rng ? per_philox_uniform(a.rng_seed, cbase + (unsigned long long)j)
                   : __ldg(a.rand + j);
}

// Padded position of prefix entry i: one spare double every 32.
__device__ __forceinline__ int ppos(int i) { return i + (i >> 5); }

// Number of k in [1, n] with pre[k] < t: the first node whose inclusive prefix
// reaches t (n if none).
__device__ __forceinline__ int lower_bound_pre(const double* pre, int n, double t) {
  int pos = 0;
  for (int step = 1 << (31 - __clz(n)); step > 0; step >>= 1) {
    const int np = pos + step;
    pos = (np <= n && pre[ppos(np)] < t) ? np : pos;
  }
  return pos;
}

// Number of k in [1, n] with pre[k] <= t, t given as its float64 bits: the
// top-level node holding t (n if t is at or past the total). Integer
// compares: non-negative float64 values order like their bit patterns, and a
// negative t (a draw owned by another shard) compares below every prefix, as
// in float64. Two forms:
//  - n <= 1024 (at most 32 groups of 32 nodes): lane l holds the prefix at
//    the end of group l (`grp`, bits; INT64_MAX past the last group); five
//    shuffle steps find the group, five shared-memory steps the node in it;
//  - larger n: a branch-free binary search over all n + 1 entries.
__device__ __forceinline__ int upper_bound_top(const double* pre, int n, long long tb,
                                               long long grp) {
  if (n <= 32 * 32) {
    const int G = n >> 5;
    int m = 0;
#pragma unroll
    for (int step = 16; step > 0; step >>= 1) {
      const int nm = m + step;
      const long long v = __shfl_sync(PER_FULL_MASK, grp, nm - 1);
      m = (nm <= G && v <= tb) ? nm : m;
    }
    if (m >= G) return n;
    int pos = m << 5;
#pragma unroll
    for (int step = 16; step > 0; step >>= 1) {
      const int np = pos + step;
      pos = __double_as_longlong(pre[ppos(np)]) <= tb ? np : pos;
    }
    return pos;
  }
  int pos = 0;
#pragma unroll
  for (int step = PER_TOP_MAX; step > 0; step >>= 1) {
    const int np = pos + step;
    const bool in = np <= n;
    const long long v = __double_as_longlong(pre[ppos(in ? np : 0)]);
    pos = (in && v <= tb) ? np : pos;
  }
  return pos;
}

// Search the 32 children c[] of a node for the first whose inclusive prefix
// exceeds r. Returns the child f, its exclusive prefix *ex and value *val;
// *fb is set when rounding left r at or past the node's sum (then the last
// positive child is taken).
__device__ __forceinline__ int search32(const float* c, double r, double* ex, float* val,
                                       bool* fb) {
  double q[8];
#pragma unroll
  for (int k = 0; k < 8; ++k)
    q[k] = ((double)c[4 * k] + (double)c[4 * k + 1]) + ((double)c[4 * k + 2] + (double)c[4 * k + 3]);
  double pre = 0.0, base = 0.0, lbase = 0.0;
  int kq = -1, lq = -1;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const double np = pre + q[k];
    if (kq < 0 && np > r) {
      kq = k;
      base = pre;
    }
    if (q[k] > 0.0) {
      lq = k;
      lbase = pre;
    }
    pre = np;
  }
  bool last = false;
  if (kq < 0) {  // past the node's sum: the last quad with mass
    *fb = true;
    last = true;
    kq = lq < 0 ? 0 : lq;
    base = lq < 0 ? 0.0 : lbase;
  }
  float e0 = c[0], e1 = c[1], e2 = c[2], e3 = c[3];
#pragma unroll
  for (int k = 1; k < 8; ++k)
    if (k == kq) {
      e0 = c[4 * k];
      e1 = c[4 * k + 1];
      e2 = c[4 * k + 2];
      e3 = c[4 * k + 3];
    }
  const double s1 = base + (double)e0, s2 = s1 + (double)e1, s3 = s2 + (double)e2;
  const double s4 = s3 + (double)e3;
  int j;
  if (!last && s1 > r) {
    j = 0;
  } else if (!last && s2 > r) {
    j = 1;
  } else if (!last && s3 > r) {
    j = 2;
  } else if (!last && s4 > r) {
    j = 3;
  } else {  // last positive element of the quad
    if (!last) *fb = true;
    j = e3 > 0.f ? 3 : e2 > 0.f ? 2 : e1 > 0.f ? 1 : 0;
  }
  *ex = j == 0 ? base : j == 1 ? s1 : j == 2 ? s2 : s3;
  *val = j == 0 ? e0 : j == 1 ? e1 : j == 2 ? e2 : e3;
  return 4 * kq + j;
}

template <int VEC>
struct VecT;
template <>
struct VecT<4> {
  using T = float4;
};
template <>
struct VecT<2> {
  using T = float2;
};
template <>
struct VecT<1> {
  using T = float;
};

__device__ __forceinline__ void cp_async(uint32_t saddr, const void* g, int bytes) {
  if (bytes == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
  else if (bytes == 8)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(saddr), "l"(g) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(saddr), "l"(g) : "memory");
}

// Store staged rows (row r at r * spitch vectors) to out rows j0 + r.
// Rows of >= 32 vectors: one flat lane-strided walk (coalesced stores);
// shorter rows: each lane stores its own row.
// Staged row r sits at group r / 4 (gpitch vectors apart), row r % 4 of the
// group (spitch vectors apart).
template <int VEC>
__device__ __forceinline__ void store_rows(const SampleArgs& a, const void* stage, int spitch,
                                           int gpitch, int64_t j0, int rn, int lane) {
  using V = typename VecT<VEC>::T;
  const int nvec = a.nvec;
  // the tile and the output never overlap: the loads of later pieces may go
  // out before the stores of earlier ones
  const V* __restrict__ sv = reinterpret_cast<const V*>(stage);
  V* __restrict__ dst = reinterpret_cast<V*>(a.out) + j0 * (a.out_stride / VEC);
  const int dstride = (int)(a.out_stride / VEC);
  if (nvec >= 32) {  // at most one row wrap per step of 32
    const int pieces = rn * nvec;
    int r = 0, c = lane;
#pragma unroll 4
    for (int p = lane; p < pieces; p += 32) {
      dst[r * dstride + c] = sv[(r >> 2) * gpitch + (r & 3) * spitch + c];
      c += 32;
      if (c >= nvec) {
        c -= nvec;
        ++r;
      }
    }
  } else if (lane < rn) {
    const V* src = sv + (lane >> 2) * gpitch + (lane & 3) * spitch;
    for (int c = 0; c < nvec; ++c) dst[lane * dstride + c] = src[c];
  }
}

// Issue the copies of rows s_idx[r0 .. r0+rn) into the warp's tile (row r
// at group r / 4, row r % 4 of the group): one Tensor Memory Accelerator
// gather of four rows per lane (`g4`: 16-byte aligned rows of at most 256
// words, a 128-byte aligned tile; the issue cost per copy instruction, not
// the bytes, bounds an SM's gather rate, so four rows per instruction), one
// bulk copy per lane (16-byte aligned rows), or one cp.async chain per lane
// (any 4-byte alignment; lower latency when an SM has only a few rows).
__device__ __forceinline__ void gather_issue(const SampleArgs& a, unsigned char* stage,
                                             const int32_t* s_idx, int r0, int rn, int lane,
                                             uint64_t* mbar, bool g4, const void* tmap,
                                             bool fence = true) {
  if (g4) {
    const int ng = (rn + 3) >> 2;
    if (fence) per_fence_proxy_async_smem();  // earlier generic accesses of the tile before the copies
    __syncwarp();
    if (lane == 0) per_mbar_arrive_expect_tx(mbar, (uint32_t)(ng * 4 * a.row_bytes));
    __syncwarp();
    if (lane < ng) {  // a short last group repeats its last row
      const int b = r0 + 4 * lane, last = r0 + rn - 1;
      per_tma_gather4(stage + lane * a.group_bytes, tmap, 0, s_idx[b], s_idx[min(b + 1, last)],
                      s_idx[min(b + 2, last)], s_idx[min(b + 3, last)], mbar);
    }
  } else if (a.use_bulk) {
    const float* row = a.t.storage + (int64_t)s_idx[r0 + min(lane, rn - 1)] * a.t.row_stride;
    per_fence_proxy_async_smem();  // earlier generic accesses of the tile before the bulk writes
    __syncwarp();
    if (lane == 0) per_mbar_arrive_expect_tx(mbar, (uint32_t)(rn * a.row_bytes));
    __syncwarp();
    if (lane < rn)
      per_bulk_load(stage + (lane >> 2) * a.group_bytes + (lane & 3) * a.row_bytes, row,
                    (uint32_t)a.row_bytes, mbar);
  } else if (lane < rn) {
    const float* row = a.t.storage + (int64_t)s_idx[r0 + lane] * a.t.row_stride;
    const uint32_t dst =
        per_smem_addr(stage + (lane >> 2) * a.group_bytes + (lane & 3) * a.row_bytes);
    const int cpb = a.cp_bytes;
    const int pieces = a.row_bytes / cpb;
    const char* src = reinterpret_cast<const char*>(row);
    for (int k = 0; k < pieces; ++k) cp_async(dst + (uint32_t)(k * cpb), src + k * cpb, cpb);
  }
}

// Wait for the copies issued by gather_issue and store the rows out.
template <int VEC>
__device__ __forceinline__ void gather_finish(const SampleArgs& a, unsigned char* stage,
                                              int64_t j0, int rn, int lane, uint64_t* mbar,
                                              uint32_t& phase) {
  if (a.use_bulk) {
    per_mbar_wait(mbar, phase, a.t.status);
    phase ^= 1u;
  } else {
    per_cp_async_wait_all();
  }
  __syncwarp();
  store_rows<VEC>(a, stage, a.row_bytes / (VEC * 4), a.group_bytes / (VEC * 4), j0, rn, lane);
  __syncwarp();
}

__device__ __forceinline__ void named_bar_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Mailbox `g` of the in-kernel exchange (the pointer array is read-only
// during the launch).
__device__ __forceinline__ PerMailbox* mailbox_of(PerMailbox* const* mailboxes, int g) {
  return reinterpret_cast<PerMailbox*>(
      __ldg(reinterpret_cast<const unsigned long long*>(mailboxes) + g));
}

// Named barriers between the compute warps and the CTA's helper warp.
constexpr int kBarMaxReady = 1;   // compute warps arrive: the CTA max is in s_cta_max
constexpr int kBarGmaxReady = 2;  // helper arrives: the global max is in s_gmax
constexpr int kMaxGrid = PER_MAX_GRID / 4;  // CTAs of one launch: one two-word slot each
constexpr int kBarRouted = 3;  // all warps: the CTA's owned draws are queued
constexpr int kBarBase = 4;    // helper arrives: the CTA's first output slot is in s_cbase
constexpr int kSliceMax = 1024;  // owned-only routing: global draws per CTA
constexpr int kAllToAllCtas = 64;  // max exchange: every CTA reads every slot up to this grid

// Poll the tagged slots of CTAs [0, n) of this launch until every one carries
// `tag` (bounded): lane l takes slots l, l + 32, ... and each poll issues all
// of a lane's pending loads before it looks at any of them, so one poll costs
// one L2 round trip however many slots are pending. Returns the max of the
// first words' data and the sum of the second words' data (sharded: the
// owned-draw counts), reduced over the warp; false on timeout.
template <bool SHARDED>
__device__ __forceinline__ bool gather_slots(const unsigned long long* slots, int n, uint32_t tag,
                                             int lane, uint32_t* mb_out,
                                             unsigned long long* owned_out) {
  constexpr int kChunk = 16;
  static_assert(kMaxGrid / 32 <= 32, "one pending bit per slot of a lane");
  uint32_t mb = 0u;
  unsigned long long owned = 0ull;
  const int nper = (n - lane + 31) / 32;  // slots of this lane
  uint32_t pending = nper >= 32 ? 0xffffffffu : ((1u << nper) - 1u);
  bool ok = true;
  for (uint32_t it = 0; __any_sync(PER_FULL_MASK, pending != 0u); ++it) {
    if (it > PER_SPIN_LIMIT) {
      ok = false;
      break;
    }
#pragma unroll
    for (int c0 = 0; c0 < 32; c0 += kChunk) {
      if (!__any_sync(PER_FULL_MASK, ((pending >> c0) & ((1u << kChunk) - 1u)) != 0u)) continue;
      unsigned long long v[kChunk], m[kChunk];
#pragma unroll
      for (int i = 0; i < kChunk; ++i) {
        const int c = lane + 32 * (c0 + i);
        const bool p = (pending >> (c0 + i)) & 1u;
        v[i] = p ? per_ld_relaxed_u64(slots + 2 * c) : 0ull;
        m[i] = (SHARDED && p) ? per_ld_relaxed_u64(slots + 2 * c + 1) : 0ull;
      }
#pragma unroll
      for (int i = 0; i < kChunk; ++i) {
        const bool p = (pending >> (c0 + i)) & 1u;
        if (p && (uint32_t)(v[i] >> 32) == tag && (!SHARDED || (uint32_t)(m[i] >> 32) == tag)) {
          mb = max(mb, (uint32_t)v[i]);
          owned += (uint32_t)m[i];
          pending &= ~(1u << (c0 + i));
        }
      }
    }
    if (pending) __nanosleep(PER_SPIN_SLEEP_NS);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mb = max(mb, __shfl_xor_sync(PER_FULL_MASK, mb, o));
    owned += __shfl_xor_sync(PER_FULL_MASK, owned, o);
  }
  *mb_out = mb;
  *owned_out = owned;
  return ok;
}

__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(per_smem_addr(ssrc)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// this thread's bulk stores have finished reading shared memory
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// this thread's bulk stores are complete
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Rows wider than a warp's staging tile (wide mode: 16-byte aligned rows and
// output rows): lane l < nact copies storage row `slot` to output row `orow`
// in pieces of a.wide_piece bytes through its own slot of the warp's tile, a
// bulk load (completing on the warp's mbarrier) then a bulk store per piece.
// The stores of the last piece may still be writing to the output when this
// returns (the kernel waits for them before it exits).
__device__ __forceinline__ void wide_copy(const SampleArgs& a, unsigned char* stage, int64_t slot,
                                          int64_t orow, int lane, int nact, uint64_t* mbar,
                                          uint32_t& phase) {
  const int64_t rb = a.t.row_dim * 4;
  const int64_t piece = a.wide_piece;
  const bool act = lane < nact;
  unsigned char* mine = stage + (int64_t)lane * piece;
  const char* src = reinterpret_cast<const char*>(a.t.storage + slot * a.t.row_stride);
  char* dst = reinterpret_cast<char*>(a.out + orow * a.out_stride);
  for (int64_t off = 0; off < rb; off += piece) {
    const uint32_t nb = (uint32_t)(rb - off < piece ? rb - off : piece);
    if (act) bulk_wait_read();  // the slot's previous stores have read it
    per_fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) per_mbar_arrive_expect_tx(mbar, nb * (uint32_t)nact);
    __syncwarp();
    if (act) per_bulk_load(mine, src + off, nb, mbar);
    per_mbar_wait(mbar, phase, a.t.status);
    phase ^= 1u;
    if (act) {
      bulk_store(dst + off, mine, nb);
      bulk_commit();
    }
  }
  // the tile is reused by the next tile's level lines: its stores must have
  // read it (their writes to the output may still be in flight)
  if (act) bulk_wait_read();
  __syncwarp();
}

// The sample kernel's body; two kernels below run it with different register
// budgets. WIDE: rows wider than a warp's staging tile, copied by bulk copies
// (a build of its own, so that the other builds carry none of that code).
template <int VEC, bool SHARDED, bool WIDE = false>
__device__ __forceinline__ void sample_body(const SampleArgs& a, const CUtensorMap& rows_map) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ double s_wsum[kMaxWarps + 1];
  __shared__ int32_t s_rows[kMaxWarps][32];
  __shared__ uint64_t s_mbar[kMaxWarps];
  __shared__ uint32_t s_cta_max;
  __shared__ uint32_t s_cta_own;  // sharded: draws this CTA owns (compacted)
  __shared__ unsigned long long s_cbase;  // owned-only routing: the CTA's first output slot
  __shared__ float s_gmax;
  __shared__ double s_stats[SHARDED ? PER_MAX_SHARDS : 1][2];
  __shared__ unsigned long long s_seq;
  __shared__ PerMailbox* s_mine;
  __shared__ unsigned long long s_owned;  // sharded: draws owned by this rank, all CTAs
  // owned-only routing: this CTA's owned draws (offsets in its slice), and the
  // output ranges its warps wrote (for the in-kernel normalisation)
  __shared__ int32_t s_q[SHARDED ? kSliceMax : 1];
  __shared__ float s_qu[SHARDED ? kSliceMax : 1];  // their uniforms (drawn once, while routing)
  __shared__ int32_t s_qn;
  __shared__ unsigned long long s_tbase[SHARDED ? kSliceMax / 32 : 1];
  __shared__ int32_t s_tcnt[SHARDED ? kSliceMax / 32 : 1];

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nthreads = blockDim.x;
  const int nwarps = (nthreads >> 5) - 1;  // compute warps; the last warp is the helper
  const bool helper = warp == nwarps;
  // draws per warp and tile: fewer than 32 for small batches (shorter row
  // stores and gathers per warp) and wide rows; 32 when sharded
  const int D = SHARDED ? 32 : a.draws_per_warp;
  const int64_t tile_draws = (int64_t)nwarps * D;
  const PerTree& t = a.t;
  PerScratch* sc = t.scratch;
  const int top = t.top_level;
  const int n_top = (int)t.level_len[top];
  double* s_pre = reinterpret_cast<double*>(smem);  // padded [n_top + 1]
  unsigned char* stage = smem + a.pre_bytes + (helper ? 0 : warp) * a.stage_bytes;
  // four-row tensor gathers need 128-byte aligned tiles (pre_bytes and
  // stage_bytes are multiples of 128); otherwise one bulk copy per row
  const bool g4 = a.gather4 && (per_smem_addr(smem) & 127u) == 0u;
  uint32_t phase = 0u;
  if (!helper && (a.use_bulk || WIDE) && lane == 0) {
    per_mbar_init(&s_mbar[warp], 1);
    per_fence_mbar_init();
  }
  per_wait_previous_grid();

  const uint32_t gen = SHARDED || helper ? per_ld_relaxed_u32(&sc->mx_gen) : 0u;
  const int64_t size = __ldg(t.size_cursor);
  // every CTA reads the stream position before it arrives at the max exchange;
  // CTA 0 advances it after the exchange has completed
  const unsigned long long cbase = a.use_rng ? per_ld_relaxed_u64(a.rng_counter) : 0ull;
  int64_t tile = blockIdx.x;
  float rnd0 = 0.f;  // this lane's first uniform
  // sharded, in-kernel exchange: this rank's mailbox and the sequence number
  // of its last call (thread 0), and the peers' mailboxes (warp 0 of CTA 0,
  // which publishes the statistics), loaded during the prologue
  PerMailbox* mine = nullptr;
  unsigned long long seq_prev = 0ull;
  PerMailbox* peer_lo = nullptr;  // mailbox of rank `lane`
  PerMailbox* peer_hi = nullptr;  // mailbox of rank `lane + 32`

  // ---- prologue (all warps): float64 exclusive prefix of the top level
  {
    const float4* topv4 = reinterpret_cast<const float4*>(t.levels[top]);
    const int nv4 = n_top >> 2;  // n_top is a multiple of 32
    const int per = (nv4 + nthreads - 1) / nthreads;
    const int beg = min(threadIdx.x * per, nv4);
    const int end = min(beg + per, nv4);
    constexpr int kReg = 8;  // float4 per thread kept in registers
    float4 q[kReg];
#pragma unroll
    for (int i = 0; i < kReg; ++i)
      q[i] = beg + i < end ? __ldg(topv4 + beg + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    // the mailbox loads go out behind the top level's (the sequence number
    // depends on the mailbox pointer; it is needed only after the scan)
    if (SHARDED && a.p2p) {
      if (threadIdx.x == 0) {
        mine = mailbox_of(a.mailboxes, a.rank);
        seq_prev = *(volatile unsigned long long*)&mine->seq;
      }
      if (blockIdx.x == 0 && warp == 0) {
        if (lane < a.world) peer_lo = mailbox_of(a.mailboxes, lane);
        if (lane + 32 < a.world) peer_hi = mailbox_of(a.mailboxes, lane + 32);
      }
    }
    // float64 sum of each float4 and their exclusive prefix within the thread,
    // in short dependency chains (pairs, then a 3-step scan)
    double f[kReg], pf[kReg];
#pragma unroll
    for (int i = 0; i < kReg; ++i)
      f[i] = ((double)q[i].x + (double)q[i].y) + ((double)q[i].z + (double)q[i].w);
#pragma unroll
    for (int i = 0; i < kReg; ++i) pf[i] = i ? f[i - 1] : 0.0;
#pragma unroll
    for (int d = 1; d < kReg; d <<= 1) {
      double nx[kReg];
#pragma unroll
      for (int i = 0; i < kReg; ++i) nx[i] = i >= d ? pf[i] + pf[i - d] : pf[i];
#pragma unroll
      for (int i = 0; i < kReg; ++i) pf[i] = nx[i];
    }
    double loc = pf[kReg - 1] + f[kReg - 1];
    for (int i0 = beg + kReg; i0 < end; ++i0) {  // long segments (few threads, big top level)
      const float4 v = __ldg(topv4 + i0);
      loc += ((double)v.x + (double)v.y) + ((double)v.z + (double)v.w);
    }
    // this lane's first uniform, while the scan below waits on shuffles
    // (owned-only routing: the first draw this lane routes)
    if (!helper && !(SHARDED && a.owned_only) && lane < D) {
      const int64_t j = tile * tile_draws + warp * D + lane;
      if (tile < a.num_tiles && j < a.batch) rnd0 = draw_uniform(a, cbase, j);
    } else if (!helper && SHARDED && a.owned_only) {
      const int64_t j = (int64_t)blockIdx.x * a.slice + warp * 32 + lane;
      if (j < min((int64_t)blockIdx.x * a.slice + a.slice, a.batch)) rnd0 = draw_uniform(a, cbase, j);
    }
    const double incl = per_warp_scan_incl(loc, lane);
    if (lane == 31) s_wsum[warp] = incl;
    if (threadIdx.x == 0) {
      s_cta_max = 0u;
      s_cta_own = 0u;
      if (SHARDED) s_qn = 0;
    }
    __syncthreads();
    double run = incl - loc;
    for (int k = 0; k < warp; ++k) run += s_wsum[k];
#pragma unroll
    for (int i = 0; i < kReg; ++i) {
      if (beg + i < end) {
        const int e = (beg + i) * 4;
        const double b = run + pf[i];
        const double bx = b + (double)q[i].x;
        const double bxy = bx + (double)q[i].y;
        s_pre[ppos(e)] = b;
        s_pre[ppos(e + 1)] = bx;
        s_pre[ppos(e + 2)] = bxy;
        s_pre[ppos(e + 3)] = bxy + (double)q[i].z;
      }
    }
    double run2 = run + (pf[kReg - 1] + f[kReg - 1]);
    for (int i0 = beg + kReg; i0 < end; ++i0) {
      const float4 v = __ldg(topv4 + i0);
      const int e = i0 * 4;
      s_pre[ppos(e)] = run2;
      run2 += (double)v.x;
      s_pre[ppos(e + 1)] = run2;
      run2 += (double)v.y;
      s_pre[ppos(e + 2)] = run2;
      run2 += (double)v.z;
      s_pre[ppos(e + 3)] = run2;
      run2 += (double)v.w;
    }
    run = run + loc;
    if (end == nv4 && end > beg) s_pre[ppos(n_top)] = run;
    if (SHARDED && a.p2p && threadIdx.x == 0) {
      s_mine = mine;
      s_seq = seq_prev + 1ull;
    }
    __syncthreads();
  }
  const double* stats = a.stats;
  if (SHARDED && a.p2p) {
    // ---- exchange the shard statistics over peer memory: CTA 0 publishes
    // this shard's (total, size) into slot `rank` of every rank's mailbox;
    // every CTA waits for all slots of its own mailbox to reach this call
    mine = s_mine;
    const uint32_t tag = per_mail_tag(s_seq);
    if (warp == 0) {
      const double tot = s_pre[ppos(n_top)];
      const double szd = (double)size;
      if (blockIdx.x == 0) {
        const unsigned long long tb = (unsigned long long)__double_as_longlong(tot);
        const unsigned long long sb = (unsigned long long)__double_as_longlong(szd);
        for (int g = lane; g < a.world; g += 32) {
          if (g == a.rank) continue;  // every CTA of this rank has its own values
          unsigned long long* slot = (g < 32 ? peer_lo : peer_hi)->stats[s_seq & 1ull][a.rank];
          per_mail_put(slot + 0, (uint32_t)tb, tag);
          per_mail_put(slot + 1, (uint32_t)(tb >> 32), tag);
          per_mail_put(slot + 2, (uint32_t)sb, tag);
          per_mail_put(slot + 3, (uint32_t)(sb >> 32), tag);
        }
      }
      for (int g = lane; g < a.world; g += 32) {
        if (g == a.rank) {
          s_stats[g][0] = tot;
          s_stats[g][1] = szd;
          continue;
        }
        uint32_t d[4] = {0u, 0u, 0u, 0u};
        per_mail_get(mine->stats[s_seq & 1ull][g], 4, tag, d, t.status);
        s_stats[g][0] = __longlong_as_double((long long)(((unsigned long long)d[1] << 32) | d[0]));
        s_stats[g][1] = __longlong_as_double((long long)(((unsigned long long)d[3] << 32) | d[2]));
      }
    }
    __syncthreads();
    stats = &s_stats[0][0];
  }
  if (!SHARDED && size <= 0) {  // host checks first; keep the device consistent anyway
    if (blockIdx.x == 0 && threadIdx.x == 0) per_flag(t.status, PER_EVT_EMPTY_BUFFER);
    return;
  }

  if (helper) {
    if (SHARDED && a.owned_only) {
      // owned-only routing: once the CTA's owned draws are queued, reserve
      // their output slots with one atomic (the compute warps read the base
      // after their searches, by which time it has long returned)
      named_bar_sync(kBarRouted, nthreads);
      if (lane == 0) {
        const uint32_t q = (uint32_t)s_qn;
        s_cbase = q ? atomicAdd(&sc->draws[gen & 1u], (unsigned long long)q) : 0ull;
        s_cta_own = q;
      }
      __syncwarp();
      named_bar_arrive(kBarBase, nthreads);
    }
    // ---- helper warp: exchange the batch max with the other CTAs while the
    // compute warps gather their rows
    if (SHARDED && a.p2p && blockIdx.x == 0) {  // peers' mailboxes, for the max put
      if (lane < a.world) peer_lo = mailbox_of(a.mailboxes, lane);
      if (lane + 32 < a.world) peer_hi = mailbox_of(a.mailboxes, lane + 32);
    }
    named_bar_sync(kBarMaxReady, nthreads);
    uint32_t mb = 0u;
    unsigned long long owned = 0ull;  // sharded: draws owned by this rank over all CTAs
    bool timed_out = false;
    // every CTA publishes its max weight and (sharded) its owned-draw count in
    // two words of its own slot, each tagged with this launch's generation;
    // the data travel in the tagged words themselves, so the accesses are
    // relaxed (no release store waiting on the SM's outstanding row traffic)
    const uint32_t tag = gen + 1u;
    unsigned long long* slots = sc->mx_slot;
    if (lane == 0) {
      per_st_relaxed_u64(&slots[2 * blockIdx.x], ((unsigned long long)tag << 32) | s_cta_max);
      if (SHARDED) per_st_relaxed_u64(&slots[2 * blockIdx.x + 1], ((unsigned long long)tag << 32) | s_cta_own);
    }
    if (gridDim.x <= kAllToAllCtas || blockIdx.x == 0) {
      // small grids: every helper reads all slots (at most two per lane, a
      // short poll loop); large grids: CTA 0 does, every lane issuing all its
      // loads of a poll together (gather_slots), and publishes two tagged totals
      if (gridDim.x > kAllToAllCtas) {
        timed_out = !gather_slots<SHARDED>(slots, (int)gridDim.x, tag, lane, &mb, &owned);
      } else {
        constexpr int kPer = kMaxGrid / 32;
        static_assert(kPer <= 64, "one pending bit per slot of a lane");
        unsigned long long pending = 0ull;  // bit i: slot lane + 32 i not seen yet
        for (int i = 0; i < kPer && lane + 32 * i < (int)gridDim.x; ++i) pending |= 1ull << i;
        for (uint32_t it = 0; __any_sync(PER_FULL_MASK, pending != 0ull); ++it) {
          if (it > PER_SPIN_LIMIT) {
            timed_out = true;
            break;
          }
          unsigned long long left = pending;
          while (left) {
            const int i = __ffsll((long long)left) - 1;
            left &= left - 1;
            const int c = lane + 32 * i;
            const unsigned long long v = per_ld_relaxed_u64(&slots[2 * c]);
            const unsigned long long n = SHARDED ? per_ld_relaxed_u64(&slots[2 * c + 1])
                                                 : ((unsigned long long)tag << 32);
            if ((uint32_t)(v >> 32) == tag && (uint32_t)(n >> 32) == tag) {
              mb = max(mb, (uint32_t)v);
              owned += (uint32_t)n;
              pending &= ~(1ull << i);
            }
          }
          if (pending) __nanosleep(PER_SPIN_SLEEP_NS);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          mb = max(mb, __shfl_xor_sync(PER_FULL_MASK, mb, o));
          owned += __shfl_xor_sync(PER_FULL_MASK, owned, o);
        }
      }
      if (lane == 0 && blockIdx.x == 0) {  // all CTAs have read gen: next generation
        if (SHARDED) sc->draws[(gen + 1u) & 1u] = 0ull;
        sc->mx_gen = gen + 1u;
        if (gridDim.x > kAllToAllCtas) {
          if (SHARDED)
            per_st_relaxed_u64(&sc->mx_result_cnt, ((unsigned long long)tag << 32) | (uint32_t)owned);
          per_st_relaxed_u64(&sc->mx_result, ((unsigned long long)tag << 32) | mb);
        }
      }
    } else if (lane == 0) {
      // large grids, CTAs other than 0: the totals CTA 0 published
      for (uint32_t it = 0;; ++it) {
        const unsigned long long v = per_ld_relaxed_u64(&sc->mx_result);
        const unsigned long long n = SHARDED ? per_ld_relaxed_u64(&sc->mx_result_cnt)
                                             : ((unsigned long long)tag << 32);
        if ((uint32_t)(v >> 32) == tag && (uint32_t)(n >> 32) == tag) {
          mb = (uint32_t)v;
          owned = (uint32_t)n;
          break;
        }
        if (it > PER_SPIN_LIMIT) {
          timed_out = true;
          break;
        }
        __nanosleep(PER_SPIN_SLEEP_NS);
      }
    }
    if (__any_sync(PER_FULL_MASK, timed_out) && lane == 0) {
      per_flag(t.status, PER_EVT_BARRIER_TIMEOUT);
      per_count(t.status, PER_STATUS_TIMEOUTS);
    }
    if (lane == 0) {
      s_gmax = __uint_as_float(mb);
      if (a.use_rng && blockIdx.x == 0) *a.rng_counter = cbase + (unsigned long long)a.batch;
      if (SHARDED) {  // every CTA has compacted its draws: the count is final
        s_owned = owned;
        if (blockIdx.x == 0) {
          *a.count = s_owned;
          if (!a.p2p) *a.local_max = s_gmax;
        }
      }
    }
    __syncwarp();
    if (SHARDED && a.p2p && a.local_norm) {
      // weights normalised by this rank's max (no exchange): record the call
      if (lane == 0 && blockIdx.x == 0) *(volatile unsigned long long*)&s_mine->seq = s_seq;
      __syncwarp();
    } else if (SHARDED && a.p2p) {
      // ---- max weight over all ranks: CTA 0 publishes this rank's max into
      // every mailbox, every CTA reduces the slots of its own mailbox
      const float lmax = s_gmax;
      const unsigned long long seq = s_seq;
      const uint32_t mtag = per_mail_tag(seq);
      mine = s_mine;
      if (blockIdx.x == 0) {
        for (int g = lane; g < a.world; g += 32)
          if (g != a.rank)
            per_mail_put(&(g < 32 ? peer_lo : peer_hi)->max_w[a.rank], __float_as_uint(lmax), mtag);
      }
      uint32_t gb = __float_as_uint(lmax);
      for (int g = lane; g < a.world; g += 32) {
        if (g == a.rank) continue;
        uint32_t d = 0u;
        per_mail_get(&mine->max_w[g], 1, mtag, &d, t.status);
        gb = max(gb, d);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) gb = max(gb, __shfl_xor_sync(PER_FULL_MASK, gb, o));
      if (lane == 0) {
        s_gmax = __uint_as_float(gb);
        // every CTA has read `seq` (all arrived at the grid exchange above)
        if (blockIdx.x == 0) *(volatile unsigned long long*)&mine->seq = seq;
      }
      __syncwarp();
    }
    named_bar_arrive(kBarGmaxReady, nthreads);
    return;
  }

  // ---- compute warps
  // local total (this store); global total, size and this store's offset in
  // the global prefix (sharded: summed over the shards in rank order)
  const double ltotal64 = s_pre[ppos(n_top)];
  double total64 = ltotal64, base64 = 0.0;
  float sizef = (float)size;
  if (SHARDED) {
    double S = 0.0, N = 0.0;
    for (int g = 0; g < a.world; ++g) {
      if (g == a.rank) base64 = S;
      S += stats[2 * g];
      N += stats[2 * g + 1];
    }
    total64 = S;
    sizef = __double2float_rn(N);
    if (!(N > 0.0) && blockIdx.x == 0 && threadIdx.x == 0) per_flag(t.status, PER_EVT_EMPTY_BUFFER);
  }
  const float total = __double2float_rn(total64);
  const float* leaves = t.levels[0];
  // end of top-level group `lane` (32 nodes per group), for upper_bound_top
  const long long grp = 32 * (lane + 1) <= n_top
                            ? __double_as_longlong(s_pre[ppos(32 * (lane + 1))])
                            : 0x7fffffffffffffffll;
  uint32_t n_fallback = 0, n_clamp = 0, n_zero = 0;
  uint32_t wmax_bits = 0u;
  float w_last = 0.f;  // this lane's unnormalised weight in its last tile
  long long slot_last = -1;  // sharded: output slot of this lane's draw in its last tile

  // owned-only routing (sharded, in-kernel exchange): the CTA routes its
  // slice of the global batch, queues the draws this shard owns, and its
  // warps then take the queue 32 draws at a time; tiles are local
  const bool owned_mode = SHARDED && a.owned_only;
  int64_t s0 = 0;
  int64_t ntiles = a.num_tiles, tstep = gridDim.x;
  if (owned_mode) {
    s0 = (int64_t)blockIdx.x * a.slice;
    const int64_t s1 = min(s0 + (int64_t)a.slice, a.batch);
    const int tc = warp * 32 + lane;
    for (int64_t j0 = s0; j0 < s1; j0 += (int64_t)nwarps * 32) {
      const int64_t j = j0 + tc;
      bool mine = false;
      float uj = 0.f;
      if (j < s1) {
        uj = j0 == s0 ? rnd0 : draw_uniform(a, cbase, j);
        const double r = (double)__fmul_rn(uj, total);
        double S = 0.0;
        int owner = -1, lastpos = 0;
        for (int g = 0; g < a.world; ++g) {
          const double tg = stats[2 * g];
          if (tg > 0.0) lastpos = g;
          S += tg;
          if (owner < 0 && S > r) owner = g;
        }
        if (owner < 0) owner = lastpos;
        mine = owner == a.rank && size > 0;
      }
      const uint32_t m = __ballot_sync(PER_FULL_MASK, mine);
      int qb = 0;
      if (lane == 0 && m) qb = atomicAdd(&s_qn, __popc(m));
      qb = __shfl_sync(PER_FULL_MASK, qb, 0);
      if (mine) {
        const int qp = qb + __popc(m & ((1u << lane) - 1u));
        s_q[qp] = (int32_t)(j - s0);
        s_qu[qp] = uj;
      }
    }
    named_bar_sync(kBarRouted, nthreads);  // with the helper, which reserves the slots
    ntiles = (s_qn + 31) / 32;
    tstep = nwarps;
    tile = warp;
    if (tile >= ntiles) {  // no draws for this warp: nothing to add to the CTA max
      __syncwarp();
      named_bar_sync(kBarBase, nthreads);  // every compute warp passes it once
      named_bar_arrive(kBarMaxReady, nthreads);
    }
  }

  // the warp's tile was written only by the level-line copies (generic
  // proxy, completed, read back) before its first gather: no proxy fence then
  bool first_tile = true;
  for (; tile < ntiles; tile += tstep) {
    const bool last_tile = tile + tstep >= ntiles;
    const int64_t wj0 = tile * tile_draws + warp * D;  // first draw of this warp
    int64_t j = wj0 + lane;
    bool ok = lane < D && j < a.batch;
    float rnd;
    if (owned_mode) {  // a queued draw: its position and the uniform routing drew
      const int64_t k = tile * 32 + lane;
      ok = k < s_qn;
      j = ok ? s0 + s_q[k] : 0;
      rnd = ok ? s_qu[k] : 0.f;
    } else {
      rnd = tile == blockIdx.x ? rnd0 : (ok ? draw_uniform(a, cbase, j) : 0.f);
    }

    const float u = __fmul_rn(rnd, total);
    double r = (double)u;
    bool own = ok;
    unsigned long long obase = 0ull;  // sharded: first output slot of this warp's draws
    uint32_t om = 0u;
    if (owned_mode) {  // the tile's slots follow the CTA's base (reserved by the helper)
      r -= base64;
      om = __ballot_sync(PER_FULL_MASK, own);
    } else if (SHARDED) {
      // the shard whose range of the global prefix holds u (the last shard
      // with mass if u is at or past the total)
      double S = 0.0;
      int owner = -1, lastpos = 0;
      for (int g = 0; g < a.world; ++g) {
        const double tg = stats[2 * g];
        if (tg > 0.0) lastpos = g;
        S += tg;
        if (owner < 0 && S > r) owner = g;
      }
      if (owner < 0) owner = lastpos;
      own = ok && owner == a.rank && size > 0;
      r -= base64;
      om = __ballot_sync(PER_FULL_MASK, own);
      // lane 0 reserves the warp's output slots; the result is broadcast only
      // after the search, so the atomic's round trip overlaps it
      if (lane == 0 && om) {
        obase = atomicAdd(&sc->draws[gen & 1u], (unsigned long long)__popc(om));
        atomicAdd(&s_cta_own, (uint32_t)__popc(om));
      }
    }

    // top level: binary search of the staged prefix
    bool fb = false;
    int k = upper_bound_top(s_pre, n_top, __double_as_longlong(r), grp);
    if (k >= n_top) {  // at or past the store's total: last node with mass
      k = lower_bound_pre(s_pre, n_top, ltotal64);
      if (k >= n_top) k = n_top - 1;
      fb = true;
    }
    int64_t node = k;
    r -= s_pre[ppos(k)];
    float p = 0.f;

    // lower levels: stage each draw's 32 children, search them per lane. Only
    // lanes with a draw (lanes 0 .. nact-1) fetch lines: idle lanes would all
    // walk toward slot 0 and pile onto one L2 line; their search reads stale
    // lines and is discarded.
    const int nact = __popc(__ballot_sync(PER_FULL_MASK, ok));
    for (int L = top - 1; L >= 0; --L) {
      __syncwarp();
      per_stage_lines(t.levels[L], stage, nact, lane,
                      [&](int d) { return __shfl_sync(PER_FULL_MASK, node, d); });
      const float4* my = reinterpret_cast<const float4*>(stage + lane * PER_LINE_STRIDE);
      float c[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 v = my[i];
        c[4 * i] = v.x;
        c[4 * i + 1] = v.y;
        c[4 * i + 2] = v.z;
        c[4 * i + 3] = v.w;
      }
      double ex;
      const int f = search32(c, r, &ex, &p, &fb);
      r -= ex;
      node = node * PER_FANOUT + f;
    }

    int64_t i = node;
    if (own) {
      if (i > size - 1 || ltotal64 <= 0.0) {  // sampling.py:49-51 clamp; p reloaded there
        i = size - 1;
        p = __ldg(leaves + i);
        ++n_clamp;
      }
      if (!(p > 0.f)) {  // never hand out an empty slot: walk back to the last positive one
        int64_t cb = i >> PER_LOG_FANOUT;
        for (int it = 0; it < 2048 && cb >= 0; ++it, --cb) {
          int found = -1;
          for (int q = 31; q >= 0; --q) {
            const int64_t s = cb * PER_FANOUT + q;
            if (s <= i && __ldg(leaves + s) > 0.f) {
              found = q;
              break;
            }
          }
          if (found >= 0) {
            i = cb * PER_FANOUT + found;
            p = __ldg(leaves + i);
            break;
          }
        }
        ++n_zero;
      }
      n_fallback += fb ? 1u : 0u;
    }

    // rows of this warp's draws: the first copies go out now and land while
    // the weights are computed
    int64_t row0;  // first output row of this warp's gathered rows
    int nrows;
    int orank = 0;
    if (SHARDED) {  // compact the owned draws into [obase, obase + popc(om))
      if (owned_mode) {
        if (first_tile) named_bar_sync(kBarBase, nthreads);  // once per compute warp
        obase = s_cbase + (unsigned long long)tile * 32ull;
      } else {
        obase = __shfl_sync(PER_FULL_MASK, obase, 0);
      }
      if (owned_mode && lane == 0) {
        s_tbase[tile] = obase;
        s_tcnt[tile] = __popc(om);
      }
      orank = __popc(om & ((1u << lane) - 1u));
      if (own) s_rows[warp][orank] = (int32_t)i;
      row0 = (int64_t)obase;
      nrows = __popc(om);
    } else {
      s_rows[warp][lane] = (int32_t)i;
      row0 = wj0;
      nrows = (int)min((int64_t)D, a.batch - wj0);
    }
    __syncwarp();
    const int rps = a.rows_per_stage;
    if (rps > 0 && nrows > 0)
      gather_issue(a, stage, s_rows[warp], 0, min(rps, nrows), lane, &s_mbar[warp], g4, &rows_map,
                   !first_tile);
    first_tile = false;

    float wv = 0.f;
    if (own) {
      const float prob = __fdiv_rn(p, total);
      wv = powf(__fmul_rn(sizef, prob), -a.beta);
      wmax_bits = max(wmax_bits, __float_as_uint(wv));
    }
    if (last_tile) {  // hand this warp's max to the helper warp and move on
      if (!SHARDED) w_last = wv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        wmax_bits = max(wmax_bits, __shfl_xor_sync(PER_FULL_MASK, wmax_bits, o));
      if (lane == 0) atomicMax(&s_cta_max, wmax_bits);
      __syncwarp();
      named_bar_arrive(kBarMaxReady, nthreads);
    }
    if (SHARDED) {
      if (own) {
        const unsigned long long slot = obase + orank;
        a.idx[slot] = a.shard_base + i;
        a.w[slot] = wv;
        a.pos[slot] = (int32_t)j;
        if (last_tile) {
          slot_last = (long long)slot;
          w_last = wv;
        }
      }
    } else if (ok) {
      a.idx[j] = i;
      if (!last_tile) a.w[j] = wv;
    }

    // ---- finish the gather of this warp's rows
    if (rps > 0) {
      for (int r0 = 0; r0 < nrows; r0 += rps) {
        const int rn = min(rps, nrows - r0);
        if (r0 > 0) gather_issue(a, stage, s_rows[warp], r0, rn, lane, &s_mbar[warp], g4, &rows_map);
        gather_finish<VEC>(a, stage, row0 + r0, rn, lane, &s_mbar[warp], phase);
      }
    } else if constexpr (WIDE) {
      if (nrows > 0) wide_copy(a, stage, i, j, lane, nrows, &s_mbar[warp], phase);
    }  // other rows wider than a stage: per_gather_rows_kernel after this kernel
  }

  if (lane == 0) {
    if (n_fallback) per_count(t.status, PER_STATUS_FALLBACKS, n_fallback);
    if (n_clamp) per_count(t.status, PER_STATUS_CLAMPS, n_clamp);
    if (n_zero) per_count(t.status, PER_STATUS_ZERO_WALKS, n_zero);
  }
  // ---- normalise this warp's weights by the global max from the helper warp
  // (sharded: the caller normalises after reducing the max over the shards)
  named_bar_sync(kBarGmaxReady, nthreads);
  if (SHARDED) {
    if (owned_mode) {  // normalise every weight this CTA wrote (its tiles' ranges)
      const float gmax = s_gmax;
      for (int64_t tl = warp; tl < ntiles; tl += nwarps) {
        const int64_t o = (int64_t)s_tbase[tl];
        if (lane < s_tcnt[tl]) a.w[o + lane] = __fdiv_rn(a.w[o + lane], gmax);
      }
    } else if (a.p2p && slot_last >= 0) {
      // in-kernel exchange (one tile per warp): normalise this lane's slot
      a.w[slot_last] = __fdiv_rn(w_last, s_gmax);
    }
    // entries past the owned draws read as padding (-1) for a following update
    for (int64_t j = (int64_t)s_owned + (int64_t)blockIdx.x * tile_draws + warp * 32 + lane;
         j < a.batch; j += (int64_t)gridDim.x * tile_draws)
      a.idx[j] = -1;
    return;
  }
  const float gmax = s_gmax;
  // earlier tiles' weights were stored unnormalised; the last tile's are in
  // registers (no load on the common one-tile path)
  int64_t tl = blockIdx.x;
  for (; tl + gridDim.x < a.num_tiles; tl += gridDim.x) {
    const int64_t j = tl * tile_draws + warp * D + lane;
    if (lane < D && j < a.batch) a.w[j] = __fdiv_rn(a.w[j], gmax);
  }
  if (tl < a.num_tiles) {
    const int64_t j = tl * tile_draws + warp * D + lane;
    if (lane < D && j < a.batch) a.w[j] = __fdiv_rn(w_last, gmax);
  }
  if constexpr (WIDE) bulk_wait_all();  // the last row stores are complete before the CTA exits
}

// CTAs of up to kMaxWarps + 1 warps, two per SM: the register allocator
// counts such a CTA as 10 warps, so two fit in 64 K registers at 96 per thread.
template <int VEC, bool SHARDED>
__global__ void __launch_bounds__((kMaxWarps + 1) * 32, 2)
    per_sample_kernel(SampleArgs a, const __grid_constant__ CUtensorMap rows_map) {
  sample_body<VEC, SHARDED>(a, rows_map);
}

// Rows wider than a warp's staging tile (wide mode), 112 registers.
template <int VEC>
__global__ void __maxnreg__(112)
    per_sample_kernel_wide(SampleArgs a, const __grid_constant__ CUtensorMap rows_map) {
  sample_body<VEC, false, true>(a, rows_map);
}

// CTAs of up to kR112Warps warps (helper included), two per SM at 112
// registers per thread (16 warps x 32 x 112 = 57,344): the same body without
// the 96-register build's spills.
constexpr int kR112Warps = 8;
template <int VEC, bool SHARDED>
__global__ void __maxnreg__(112)
    per_sample_kernel_r112(SampleArgs a, const __grid_constant__ CUtensorMap rows_map) {
  sample_body<VEC, SHARDED>(a, rows_map);
}

// Launch shapes already chosen, per device, kernel, batch and store geometry
// (small; a miss recomputes and overwrites round-robin).
struct ShapeKey {
  int dev;
  const void* fn;
  int64_t batch;
  int32_t world;  // owned-only routing: the number of shards; 0 otherwise
  int32_t pre_bytes;
  int32_t stage_bytes;
  bool operator==(const ShapeKey& o) const {
    return dev == o.dev && fn == o.fn && batch == o.batch && world == o.world &&
           pre_bytes == o.pre_bytes && stage_bytes == o.stage_bytes;
  }
};
struct Shape {
  int nw;
  int max_ctas;
  int sms;
  int slice;  // owned-only routing: global draws per CTA
  int d;      // draws per warp
};
constexpr int kShapeSlots = 64;
ShapeKey g_shape_key[kShapeSlots];
Shape g_shape[kShapeSlots];
int g_shape_used = 0, g_shape_next = 0;
std::mutex g_shape_mu;

bool shape_lookup(const ShapeKey& k, Shape* out) {
  std::lock_guard<std::mutex> lk(g_shape_mu);
  for (int i = 0; i < g_shape_used; ++i)
    if (g_shape_key[i] == k) {
      *out = g_shape[i];
      return true;
    }
  return false;
}

void shape_store(const ShapeKey& k, const Shape& v) {
  std::lock_guard<std::mutex> lk(g_shape_mu);
  const int i = g_shape_next;
  g_shape_next = (g_shape_next + 1) % kShapeSlots;
  if (g_shape_used < kShapeSlots) ++g_shape_used;
  g_shape_key[i] = k;
  g_shape[i] = v;
}

// Owned-only routing: the largest slice (global draws per CTA, a multiple of
// 32, at most kSliceMax) whose owned count stays within the CTA's c x 32
// lanes with margin — mean + 4 standard deviations of a binomial with the
// shard's expected share p (1.25 / world, for uneven masses) — so that every
// warp has at most one tile (a warp with two would double the kernel's
// latency chain).
int owned_slice(int c, int world) {
  const double p = world > 1 ? (1.25 / world < 1.0 ? 1.25 / world : 1.0) : 1.0;
  int best = 32 * c;
  for (int sl = 32 * c; sl <= kSliceMax; sl += 32) {
    const double mean = sl * p, sd = sqrt(sl * p * (1.0 - p));
    if (mean + 4.0 * sd > 32.0 * c) break;
    best = sl;
  }
  return best;
}

// Four-row tensor gathers of the rows (for every batch size: measured faster
// than cp.async chains at a few rows per SM and than one bulk copy per row
// at many); PER_GATHER4=0 turns them off.
bool gather4_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("PER_GATHER4");
    v = (s && s[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Tensor maps of row storages (2-D: row_stride words wide, capacity rows,
// a box of one row of `box` words), built once per storage geometry.
struct MapKey {
  const float* storage;
  int64_t row_stride;
  int64_t capacity;
  int box;
  bool operator==(const MapKey& o) const {
    return storage == o.storage && row_stride == o.row_stride && capacity == o.capacity &&
           box == o.box;
  }
};
constexpr int kMapSlots = 16;
MapKey g_map_key[kMapSlots];
CUtensorMap g_map[kMapSlots];
int g_map_used = 0, g_map_next = 0;
std::mutex g_map_mu;

bool rows_map(const PerTree& t, int box, CUtensorMap* out) {
  const MapKey k{t.storage, t.row_stride, t.capacity, box};
  std::lock_guard<std::mutex> lk(g_map_mu);
  for (int i = 0; i < g_map_used; ++i)
    if (g_map_key[i] == k) {
      *out = g_map[i];
      return true;
    }
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    looked_up = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    else
      cudaGetLastError();  // leave no sticky error behind
  }
  if (!encode || t.capacity < 1 || t.capacity > ((int64_t)1 << 31) || box < 4 || box > 256 ||
      box > t.row_stride || (t.row_stride * 4) % 16 || ((uintptr_t)t.storage) % 16)
    return false;
  const cuuint64_t dims[2] = {(cuuint64_t)t.row_stride, (cuuint64_t)t.capacity};
  const cuuint64_t strides[1] = {(cuuint64_t)t.row_stride * 4};
  const cuuint32_t boxdim[2] = {(cuuint32_t)box, 1};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  if (encode(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)t.storage, dims, strides, boxdim, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  const int i = g_map_next;
  g_map_next = (g_map_next + 1) % kMapSlots;
  if (g_map_used < kMapSlots) ++g_map_used;
  g_map_key[i] = k;
  g_map[i] = m;
  *out = m;
  return true;
}

// Shared-memory bytes of the padded float64 prefix of the top level
// (n_top + 1 entries, one spare every 32), rounded up to 128 (the row tiles
// behind it stay 128-byte aligned).
int32_t top_bytes(const PerTree& t) {
  const int n_top = (int)t.level_len[t.top_level];
  return (int32_t)(((n_top + 1 + (n_top >> 5) + 1) * 8 + 127) & ~127);
}

// Wide mode (rows wider than a warp's staging tile): one CTA per SM, each
// taking an equal share of the batch as nw compute warps (at most
// kR112Warps - 1) of D draws; every lane stages its row in pieces that fill
// the CTA's shared memory, right after its search (copies that start while
// other CTAs still walk the tree measured faster than copies held back until
// every walk is done).
constexpr size_t kWideSmem = 200 * 1024;

template <int VEC>
int launch_wide(SampleArgs a, cudaStream_t stream) {
  const void* fn = (const void*)per_sample_kernel_wide<VEC>;
  int dev = 0, sms = 148;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return per_record_cuda(e);
  const int64_t ctas = a.batch < sms ? a.batch : sms;
  const int64_t per_cta = (a.batch + ctas - 1) / ctas;
  const int nw = (int)(per_cta < kR112Warps - 1 ? per_cta : kR112Warps - 1);
  int64_t D = (per_cta + nw - 1) / nw;
  if (D > 32) D = 32;
  const int64_t rb = a.t.row_dim * 4;
  int64_t piece = ((int64_t)kWideSmem - a.pre_bytes) / (nw * D) / 16 * 16;
  if (piece > rb) piece = rb;
  if (piece < 16) return PER_ERR_TOO_LARGE;
  a.draws_per_warp = (int32_t)D;
  a.wide_piece = (int32_t)piece;
  a.stage_bytes = (int32_t)((D * piece + 127) & ~127ll);
  if (a.stage_bytes < kStageMin) a.stage_bytes = (kStageMin + 127) & ~127;
  const size_t smem = (size_t)a.pre_bytes + (size_t)nw * a.stage_bytes;
  int rc = per_set_smem(fn, smem);
  if (rc) return rc;
  const int threads = (nw + 1) * 32;
  int max_ctas = 0;
  rc = per_coresident_ctas(fn, threads, smem, &max_ctas);
  if (rc) return rc;
  a.num_tiles = (a.batch + nw * D - 1) / (nw * D);
  int64_t grid = a.num_tiles < max_ctas ? a.num_tiles : max_ctas;
  if (grid > kMaxGrid) grid = kMaxGrid;
  if (grid < 1) grid = 1;
  CUtensorMap tmap;  // unused in wide mode
  memset(&tmap, 0, sizeof(tmap));
  void* args[] = {&a, &tmap};
  e = per_launch(fn, (unsigned)grid, threads, smem, stream, args, grid > 1);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}

template <int VEC, bool SHARDED>
int launch_vec(SampleArgs a, cudaStream_t stream) {
  const void* fn = (const void*)per_sample_kernel<VEC, SHARDED>;
  const void* fn112 = (const void*)per_sample_kernel_r112<VEC, SHARDED>;
  // c compute warps + the helper: the 112-register build where it fits
  auto fn_for = [&](int64_t c) { return c + 1 <= kR112Warps ? fn112 : fn; };
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return per_record_cuda(e);
  if (a.world <= 1) a.owned_only = 0;  // one shard owns every draw: no routing pass
  // the shape chosen for this kernel, batch, world and store geometry is cached
  ShapeKey key{dev, fn, a.batch, a.owned_only ? a.world : 0, a.pre_bytes, a.stage_bytes};
  Shape sh;
  if (!shape_lookup(key, &sh)) {
    int sms = 148;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return per_record_cuda(e);
    // draws per warp: a batch that leaves SMs without a full warp of draws
    // is spread thinner (a multiple of 8, at least 8), which shortens every
    // warp's row gather and row stores; 32 otherwise (and when sharded)
    int d = 32;
    if (!SHARDED) {
      const int64_t per_sm = (a.batch + sms - 1) / sms;
      d = (int)((per_sm + 7) / 8 * 8);
      d = d < 8 ? 8 : d > 32 ? 32 : d;
    }
    const int64_t warp_tiles = (a.batch + d - 1) / d;
    int rc = per_set_smem(fn, (size_t)a.pre_bytes + (size_t)kMaxWarps * a.stage_bytes);
    if (rc) return rc;
    rc = per_set_smem(fn112, (size_t)a.pre_bytes + (size_t)(kR112Warps - 1) * a.stage_bytes);
    if (rc) return rc;
    int64_t nw = kMaxWarps, best_cost = -1, best_grid = 0;
    int max_ctas = 0, best_slice = 0;
    for (int c = kMaxWarps; c >= 1; --c) {
      int cap = 0;
      rc = per_coresident_ctas(fn_for(c), (c + 1) * 32,
                               (size_t)a.pre_bytes + (size_t)c * a.stage_bytes, &cap);
      if (rc) return rc;
      if (a.owned_only) {
        // owned-only: slices sized so that no warp gets two tiles; among the
        // shapes that fit one wave, the fewest busy warps on the busiest SM,
        // then the fewest CTAs
        const int sl = owned_slice(c, a.world);
        const int64_t grid = (a.batch + sl - 1) / sl;
        if (grid > cap || grid > kMaxGrid) continue;
        const double p = 1.25 / a.world < 1.0 ? 1.25 / a.world : 1.0;
        const int64_t busy = (int64_t)((sl * p + 31.0) / 32.0) < c ? (int64_t)((sl * p + 31.0) / 32.0) : c;
        const int64_t cost = busy * ((grid + sms - 1) / sms);
        if (best_cost < 0 || cost < best_cost || (cost == best_cost && grid < best_grid)) {
          best_cost = cost;
          best_grid = grid;
          nw = c;
          max_ctas = cap;
          best_slice = sl;
        }
        continue;
      }
      // compute warps per CTA: among the shapes that cover the batch in one
      // wave of co-resident CTAs (one tile per warp), the one whose busiest
      // SM holds the fewest warps (CTAs are spread round-robin over the SMs);
      // ties go to fewer, larger CTAs (fewer prologues). Beyond one wave: 8.
      const int64_t tiles = (warp_tiles + c - 1) / c;
      if (tiles > cap || tiles > kMaxGrid) continue;
      const int64_t cost = (int64_t)c * ((tiles + sms - 1) / sms);
      if (best_cost < 0 || cost < best_cost) {
        best_cost = cost;
        nw = c;
        max_ctas = cap;
      }
    }
    if (a.owned_only && best_cost < 0) return PER_ERR_TOO_LARGE;  // no one-wave shape
    if (best_cost < 0) {
      rc = per_coresident_ctas(fn_for(nw), (int)(nw + 1) * 32,
                               (size_t)a.pre_bytes + (size_t)nw * a.stage_bytes, &max_ctas);
      if (rc) return rc;
    }
    sh.nw = (int)nw;
    sh.max_ctas = max_ctas;
    sh.sms = sms;
    sh.slice = best_slice;
    sh.d = d;
    shape_store(key, sh);
  }
  const int64_t nw = sh.nw;
  const int D = sh.d;
  a.draws_per_warp = D;
  const int64_t warp_tiles = (a.batch + D - 1) / D;
  // without four-row gathers: a few rows per SM take cp.async chains (lower
  // latency), many take bulk copies (more rows in flight)
  const int64_t busy_tiles = a.owned_only ? (warp_tiles + a.world - 1) / a.world : warp_tiles;
  CUtensorMap tmap;  // the rows' tensor map when four-row gathers are on
  memset(&tmap, 0, sizeof(tmap));
  if (a.gather4 && !rows_map(a.t, a.row_bytes / 4, &tmap)) a.gather4 = 0;
  if (!a.gather4) {
    a.group_bytes = 4 * a.row_bytes;  // rows back to back in the tile
    if (a.use_bulk && busy_tiles <= sh.sms) a.use_bulk = 0;
  }
  const int threads = (int)(nw + 1) * 32;
  const size_t smem = (size_t)a.pre_bytes + (size_t)nw * a.stage_bytes;
  a.num_tiles = (a.batch + nw * D - 1) / (nw * D);
  int64_t grid;
  if (a.owned_only) {
    a.slice = sh.slice;
    grid = (a.batch + a.slice - 1) / a.slice;
  } else {
    grid = a.num_tiles < sh.max_ctas ? a.num_tiles : sh.max_ctas;
    if (grid > kMaxGrid) grid = kMaxGrid;
    if (grid < 1) grid = 1;
    if (a.p2p && a.num_tiles > grid) return PER_ERR_TOO_LARGE;  // one tile per warp
  }
  void* args[] = {&a, &tmap};
  e = per_launch(fn_for(nw), (unsigned)grid, threads, smem, stream, args, grid > 1);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}

// Largest batch that one wave of co-resident CTAs covers with one tile per
// warp (the in-kernel exchange needs every CTA resident at once).
template <int VEC>
int max_wave_vec(SampleArgs a, int64_t* out) {
  const void* fn = (const void*)per_sample_kernel<VEC, true>;
  const size_t smem = (size_t)a.pre_bytes + (size_t)kMaxWarps * a.stage_bytes;
  int rc = per_set_smem(fn, smem);
  if (rc) return rc;
  int max_ctas = 0;
  rc = per_coresident_ctas(fn, (kMaxWarps + 1) * 32, smem, &max_ctas);
  if (rc) return rc;
  if (max_ctas > kMaxGrid) max_ctas = kMaxGrid;
  *out = (int64_t)max_ctas * kMaxWarps * 32;
  return PER_OK;
}

}  // namespace

namespace {

void fill_common(SampleArgs& a, const PerTree& t, const float* rand, int64_t batch, float beta,
                 float* out, int64_t out_stride, int64_t* idx, float* w) {
  a.t = t;
  a.rand = rand;
  a.batch = batch;
  a.beta = beta;
  a.out = out;
  a.out_stride = out_stride;
  a.idx = idx;
  a.w = w;
  a.num_tiles = 0;
  a.pre_bytes = top_bytes(t);
  a.draws_per_warp = 32;
  a.wide = 0;
  a.wide_piece = 0;
  a.stats = nullptr;
  a.rank = 0;
  a.world = 1;
  a.shard_base = 0;
  a.pos = nullptr;
  a.count = nullptr;
  a.local_max = nullptr;
  a.mailboxes = nullptr;
  a.p2p = 0;
  a.local_norm = 0;
  a.owned_only = 0;
  a.slice = 0;
  a.use_rng = 0;
  a.rng_seed = 0ull;
  a.rng_counter = nullptr;
  // staged copies move whole pieces: 16 bytes when row starts and strides are
  // 16-byte aligned (rounding row_dim*4 up to 16 must stay inside the row
  // stride), else 8, else 4; bulk copies need the 16-byte case
  const int64_t rb = t.row_dim * 4;
  const uintptr_t sal = (uintptr_t)t.storage | (uintptr_t)(t.row_stride * 4);
  int cpb = 4;
  if (sal % 16 == 0 && (rb + 15) / 16 * 16 <= t.row_stride * 4)
    cpb = 16;
  else if (sal % 8 == 0 && (rb + 7) / 8 * 8 <= t.row_stride * 4)
    cpb = 8;
  const int64_t row_bytes = (rb + cpb - 1) / cpb * cpb;
  a.cp_bytes = cpb;
  a.use_bulk = (cpb == 16) ? 1 : 0;
  a.row_bytes = (int32_t)row_bytes;
  // four-row gathers: rows of at most 256 words, groups padded to 128 bytes
  a.gather4 = (a.use_bulk && row_bytes <= 1024 && gather4_enabled()) ? 1 : 0;
  a.group_bytes = (int32_t)(4 * row_bytes);
  if (a.gather4) {
    a.group_bytes = (int32_t)((4 * row_bytes + 127) & ~127ll);
    const int groups = kStageMax / a.group_bytes < 8 ? kStageMax / a.group_bytes : 8;
    a.stage_bytes = groups * a.group_bytes;
    a.rows_per_stage = 4 * groups;
  } else if (row_bytes <= kStageMax) {
    const int64_t want = 32 * row_bytes;
    a.stage_bytes = (int32_t)(want < kStageMax ? want : (kStageMax / row_bytes) * row_bytes);
    a.rows_per_stage = (int32_t)(a.stage_bytes / row_bytes);
  } else {
    a.stage_bytes = 0;
    a.rows_per_stage = 0;
    a.use_bulk = 0;
  }
  if (a.stage_bytes < kStageMin) a.stage_bytes = kStageMin;  // the level tiles share it
  a.stage_bytes = (a.stage_bytes + 127) & ~127;  // tiles stay 128-byte aligned
}

// widest vector that every row start and both bases allow
int vec_width(const PerTree& t, const float* out, int64_t out_stride) {
  const uintptr_t al = (uintptr_t)t.storage | (uintptr_t)out | (uintptr_t)(t.row_stride * 4) |
                       (uintptr_t)(out_stride * 4);
  return (al % 16 == 0 && t.row_dim % 4 == 0) ? 4 : (al % 8 == 0 && t.row_dim % 2 == 0) ? 2 : 1;
}

// ---- rows wider than a warp's staging tile (row_dim > 2560): the sample
// kernel writes the indices only, then this kernel copies the rows with the
// whole GPU: one row per CTA per step, every thread keeping 4 vectors in
// flight, streaming loads and stores (the rows are read once).
struct GatherArgs {
  const float* storage;
  int64_t row_stride;
  int64_t row_dim;
  float* out;
  int64_t out_stride;
  const int64_t* idx;
  int64_t base;                    // idx are global slot numbers (sharded): slot = idx - base
  const unsigned long long* count; // rows to copy on the device (sharded), or null
  int64_t batch;
};
constexpr int kGatherThreads = 256;
constexpr int kGatherUnroll = 4;

template <int VEC>
__global__ void __launch_bounds__(kGatherThreads) per_gather_rows_kernel(GatherArgs g) {
  per_wait_previous_grid();
  using V = typename VecT<VEC>::T;
  int64_t n = g.batch;
  if (g.count) n = min(n, (int64_t)*g.count);
  const int nvec = (int)(g.row_dim / VEC);
  for (int64_t j = blockIdx.x; j < n; j += gridDim.x) {
    const int64_t slot = g.idx[j] - g.base;
    const V* src = reinterpret_cast<const V*>(g.storage + slot * g.row_stride);
    V* dst = reinterpret_cast<V*>(g.out + j * g.out_stride);
    for (int c0 = 0; c0 < nvec; c0 += kGatherThreads * kGatherUnroll) {
      V buf[kGatherUnroll];
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        const int c = c0 + u * kGatherThreads + threadIdx.x;
        if (c < nvec) buf[u] = __ldcs(src + c);
      }
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        const int c = c0 + u * kGatherThreads + threadIdx.x;
        if (c < nvec) __stcs(dst + c, buf[u]);
      }
    }
  }
}

int launch_gather_rows(const SampleArgs& a, int vec, int64_t base, cudaStream_t stream) {
  GatherArgs g;
  g.storage = a.t.storage;
  g.row_stride = a.t.row_stride;
  g.row_dim = a.t.row_dim;
  g.out = a.out;
  g.out_stride = a.out_stride;
  g.idx = a.idx;
  g.base = base;
  g.count = a.count;
  g.batch = a.batch;
  const void* fn = vec == 4   ? (const void*)per_gather_rows_kernel<4>
                   : vec == 2 ? (const void*)per_gather_rows_kernel<2>
                              : (const void*)per_gather_rows_kernel<1>;
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  int64_t grid = (int64_t)sms * 8;  // 8 CTAs (2048 threads) per SM
  if (grid > a.batch) grid = a.batch;
  if (grid < 1) grid = 1;
  void* args[] = {&g};
  cudaError_t e = per_launch(fn, (unsigned)grid, kGatherThreads, 0, stream, args, false);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}

template <bool SHARDED>
int launch_any(SampleArgs& a, int vec, cudaStream_t stream) {
  a.nvec = (int32_t)(a.t.row_dim / vec);
  // rows wider than a stage: copied inside the sample kernel when rows and
  // output rows are 16-byte aligned (bulk copies), else by
  // per_gather_rows_kernel after it
  if (!SHARDED && a.rows_per_stage == 0 && a.cp_bytes == 16 && (a.t.row_dim * 4) % 16 == 0 &&
      ((uintptr_t)a.out) % 16 == 0 && (a.out_stride * 4) % 16 == 0) {
    a.wide = 1;
    return vec == 4   ? launch_wide<4>(a, stream)
           : vec == 2 ? launch_wide<2>(a, stream)
                      : launch_wide<1>(a, stream);
  }
  int rc = vec == 4   ? launch_vec<4, SHARDED>(a, stream)
           : vec == 2 ? launch_vec<2, SHARDED>(a, stream)
                      : launch_vec<1, SHARDED>(a, stream);
  if (rc || a.rows_per_stage > 0) return rc;
  return launch_gather_rows(a, vec, SHARDED ? a.shard_base : 0, stream);
}

}  // namespace

void set_rng(SampleArgs& a, const PerRng* rng) {
  if (!rng) return;
  a.use_rng = 1;
  a.rng_seed = rng->seed;
  a.rng_counter = rng->counter;
}

int per_launch_sample(const PerTree& t, const float* rand, const PerRng* rng, int64_t batch,
                      float beta, float* out, int64_t out_stride, int64_t* idx, float* w,
                      cudaStream_t stream) {
  SampleArgs a;
  fill_common(a, t, rand, batch, beta, out, out_stride, idx, w);
  set_rng(a, rng);
  return launch_any<false>(a, vec_width(t, out, out_stride), stream);
}

int per_launch_sample_sharded(const PerTree& t, int32_t rank, int32_t world, int64_t shard_base,
                              const double* stats, const float* rand, const PerRng* rng,
                              int64_t batch, float beta,
                              float* out, int64_t out_stride, int64_t* idx, float* w,
                              int32_t* pos, int64_t* count, float* local_max,
                              cudaStream_t stream) {
  SampleArgs a;
  fill_common(a, t, rand, batch, beta, out, out_stride, idx, w);
  a.stats = stats;
  a.rank = rank;
  a.world = world;
  a.shard_base = shard_base;
  a.pos = pos;
  a.count = reinterpret_cast<unsigned long long*>(count);
  a.local_max = local_max;
  set_rng(a, rng);
  // the kernel writes count, local_max and the -1 padding past the owned draws
  return launch_any<true>(a, vec_width(t, out, out_stride), stream);
}

int per_launch_sample_sharded_p2p(const PerTree& t, int32_t rank, int32_t world,
                                  int64_t shard_base, PerMailbox* const* mailboxes,
                                  const float* rand, const PerRng* rng, int64_t batch, float beta,
                                  float* out, int64_t out_stride, int64_t* idx, float* w,
                                  int32_t* pos, int64_t* count, int32_t local_norm,
                                  cudaStream_t stream) {
  SampleArgs a;
  fill_common(a, t, rand, batch, beta, out, out_stride, idx, w);
  a.rank = rank;
  a.world = world;
  a.shard_base = shard_base;
  a.pos = pos;
  a.count = reinterpret_cast<unsigned long long*>(count);
  a.mailboxes = mailboxes;
  a.p2p = 1;
  a.local_norm = local_norm ? 1 : 0;
  a.owned_only = 1;
  set_rng(a, rng);
  return launch_any<true>(a, vec_width(t, out, out_stride), stream);
}

int per_launch_sample_p2p_max_batch(const PerTree& t, int64_t* max_batch) {
  SampleArgs a;
  fill_common(a, t, nullptr, 1, 0.f, nullptr, t.row_dim, nullptr, nullptr);
  int64_t best = INT64_MAX, m = 0;
  int rc = max_wave_vec<4>(a, &m);
  if (!rc) best = m < best ? m : best;
  if (!rc) rc = max_wave_vec<2>(a, &m);
  if (!rc) best = m < best ? m : best;
  if (!rc) rc = max_wave_vec<1>(a, &m);
  if (!rc) best = m < best ? m : best;
  if (rc) return rc;
  *max_batch = best;
  return PER_OK;
}
