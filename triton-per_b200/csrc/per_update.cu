// Priority update, ring insert and exact rebuild of the sum tree.
//
// Reference behaviour (triton-per):
//   buffer.py:133-137  td = |td|; max_priority = max(max_priority, (max td + eps)^alpha)
//   update.py:32-35    new = (|td| + eps)^alpha; atomic_xchg(leaf); atomic_add(block_sum, new-old)
//   buffer.py:139-145  torch backend: leaf assign + exact recompute of touched blocks
//   buffer.py:156-162  exact refresh of all block sums every 512 updates
//   buffer.py:66-79    add: ring write, new leaves = max priority, touched blocks recomputed
//
// Design: instead of fp32 delta atomics (which drift and need the periodic
// refresh), every touched node is recomputed exactly from its 32 children
// (one coalesced 128-byte warp load, float64 butterfly sum), level by level.
// Exactly one writer per slot and per node is elected, which makes the result
// deterministic: for duplicate indices the last occurrence wins, and the sums
// never drift.
//   * batches of up to 2048 indices: CTAs that each own the entries under a
//     disjoint share of the top-level nodes (no coordination between CTAs),
//     warp elections by match, every level summed by one warp;
//   * larger batches: a co-resident grid, election with atomicMax on global
//     claim words, levels separated by grid barriers; claims are reset by
//     their owner in the phase that reads them, so the claim arrays are
//     all-zero between launches.
#include <cuda_runtime.h>
#include <stdint.h>

#include "per_internal.h"

namespace {

constexpr int kThreads = 256;
constexpr int kMaxPerThread = 32;  // entries per thread (bit mask width)

__device__ __forceinline__ int64_t live_nodes(int64_t capacity, int level) {
  const int64_t span = (int64_t)1 << (PER_LOG_FANOUT * level);
  return (capacity + span - 1) / span;
}

struct UpdateArgs {
  PerTree t;
  const int64_t* idx;
  const float* td;
  int64_t n;
  int64_t base;    // global index of slot 0 (sharded stores); 0 otherwise
  int32_t strict;  // 1: indices outside the store are errors; 0: another shard's (skipped)
  const unsigned long long* count;  // device: entries to apply (a prefix of idx), or null = n
};

// Entries to apply: all n, or the device count when one is given (read after
// the previous kernel's results are visible).
__device__ __forceinline__ int64_t entries_of(const UpdateArgs& a) {
  return a.count ? min(a.n, (int64_t)*a.count) : a.n;
}

// Slot of entry e in this store, or -1 (counted) if it is outside.
__device__ __forceinline__ int64_t slot_of(const UpdateArgs& a, int64_t e) {
  return a.idx[e] - a.base;
}

__device__ __forceinline__ float new_priority(const PerTree& t, float td) {
  return powf(fabsf(td) + t.eps, t.alpha);  // update.py:32, buffer.py:139
}

// ---------------------------------------------------------------- grid update
__global__ void __launch_bounds__(kThreads) per_update_kernel(UpdateArgs a) {
  per_wait_previous_grid();
  const PerTree& t = a.t;
  PerGridBarrier bar;
  bar.init(t.scratch);
  __shared__ uint32_t s_max;
  __shared__ __align__(16) unsigned char s_tiles[kThreads / 32][PER_NODE_TILE];
  if (threadIdx.x == 0) s_max = 0u;
  __syncthreads();

  const int lane = threadIdx.x & 31;
  unsigned char* tile = s_tiles[threadIdx.x >> 5];
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  uint32_t* tags = t.claims[0];
  float* leaves = t.levels[0];
  const int64_t n = entries_of(a);

  // P0: new priorities, winner election (largest position wins), max priority
  uint32_t active = 0u, tmax = 0u, nbad = 0u, nforeign = 0u;
  for (int q = 0; q < kMaxPerThread; ++q) {
    const int64_t e = tid + (int64_t)q * nth;
    if (e >= n) break;
    const int64_t i = slot_of(a, e);
    if (i < 0 || i >= t.capacity) {
      if (a.strict) ++nbad; else ++nforeign;
      continue;
    }
    tmax = max(tmax, __float_as_uint(new_priority(t, a.td[e])));
    atomicMax(tags + i, (uint32_t)(e + 1));
    active |= 1u << q;
  }
  if (nbad) {
    per_count(t.status, PER_STATUS_BAD_INDICES, nbad);
    per_flag(t.status, PER_EVT_BAD_INDEX);
  }
  if (nforeign) per_count(t.status, PER_STATUS_FOREIGN, nforeign);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tmax = max(tmax, __shfl_xor_sync(PER_FULL_MASK, tmax, o));
  if (lane == 0 && tmax) atomicMax(&s_max, tmax);
  __syncthreads();
  if (threadIdx.x == 0 && s_max) atomicMax(reinterpret_cast<unsigned int*>(t.max_priority), s_max);

  bar.sync(t.status);

  // P1: winners write their leaf and claim the chunk
  uint32_t next = 0u;
  for (uint32_t m = active; m; m &= m - 1) {
    const int q = __ffs(m) - 1;
    const int64_t e = tid + (int64_t)q * nth;
    const int64_t i = slot_of(a, e);
    if (__ldcg(tags + i) == (uint32_t)(e + 1)) {
      tags[i] = 0u;
      leaves[i] = new_priority(t, a.td[e]);
      atomicMax(t.claims[1] + (i >> PER_LOG_FANOUT), (uint32_t)(e + 1));
      next |= 1u << q;
    }
  }
  active = next;

  // P2..: the owner of each touched node recomputes it (with its warp), then
  // claims the parent
  for (int L = 1; L < t.num_levels; ++L) {
    bar.sync(t.status);
    next = 0u;
    uint32_t* cl = t.claims[L];
    const bool more = L + 1 < t.num_levels;
    const uint32_t wmask = __reduce_or_sync(PER_FULL_MASK, active);
    for (uint32_t m = wmask; m; m &= m - 1) {
      const int q = __ffs(m) - 1;
      const int64_t e = tid + (int64_t)q * nth;
      bool own = false;
      int64_t node = 0;
      if ((active >> q) & 1u) {
        node = slot_of(a, e) >> (PER_LOG_FANOUT * L);
        own = __ldcg(cl + node) == (uint32_t)(e + 1);
        if (own) cl[node] = 0u;
      }
      per_warp_recompute(t.levels[L - 1], t.levels[L], node, own, lane, tile);
      if (own) {
        if (more) atomicMax(t.claims[L + 1] + (node >> PER_LOG_FANOUT), (uint32_t)(e + 1));
        next |= 1u << q;
      }
    }
    active = next;
  }
}

// ---------------------------------------------------------------- partitioned update
// Batches of up to kWMaxN indices: K CTAs (a power of two), CTA k taking the
// entries whose top-level ancestor (the node of level T above the leaf, T the
// highest maintained level) hashes to k. Entries under different top-level
// nodes touch disjoint nodes at every level, so the CTAs never coordinate:
// each loads every entry, keeps its own in position order, and its warp 0
// applies them in rounds of 32 (one per lane) while the other warps compute
// the new priorities. A round fetches every lane's line of every level at
// once (duplicates included), elects the winner of each slot (the highest
// lane among equal slots: the last occurrence) and the owner of each touched
// node (the lowest lane among equal nodes) with warp matches while the lines
// are in flight, then patches the winning leaves into their owner's line and
// sums level by level, each owner patching its node into the line of its
// parent's owner. Later rounds see earlier rounds' writes (same warp, program
// order), so the last occurrence wins across rounds too. Node values are
// per_sum32_tree of the same children as in the grid path.
constexpr int kWMaxN = 2048;             // entries of a batch
constexpr int kWEntriesPerCta = 16;      // expected entries per CTA
constexpr int kWMaxT = 4;                // tree levels above the leaves (capacity <= 2^30)
constexpr int kWPer = kWMaxN / kThreads; // entries per thread
constexpr int kWarps = kThreads / 32;
static_assert(kWPer * kWarps <= 64, "warp counts scanned by one warp, two per lane");

// Named barrier 1 between the priority warps (arrive) and warp 0 (sync).
__device__ __forceinline__ void named_bar_arrive_upd(int count) {
  asm volatile("bar.arrive 1, %0;" ::"r"(count) : "memory");
}
__device__ __forceinline__ void named_bar_sync_upd(int count) {
  asm volatile("bar.sync 1, %0;" ::"r"(count) : "memory");
}

// CTA of a top-level node among a power-of-two number of CTAs (mask kmask)
__device__ __forceinline__ uint32_t top_cta(uint32_t top_node, uint32_t kmask) {
  return ((top_node * 2654435761u) >> 16) & kmask;
}

// Issue (no wait) the copies of lane d's line of level L (the children of
// its node of level L + 1) for lanes d < ra into lines d of `tile`, 4 lines
// per instruction. Called by a whole warp.
__device__ __forceinline__ void warp_issue_lines(const float* level, unsigned char* tile,
                                                 uint32_t leaf, int ra, int L, int lane) {
  const uint32_t base = per_smem_addr_generic(tile);
  uint32_t nd[8];
#pragma unroll
  for (int k = 0; k < 8; ++k)
    nd[k] = __shfl_sync(PER_FULL_MASK, leaf, (k * 32 + lane) >> 3) >> (PER_LOG_FANOUT * (L + 1));
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int q = k * 32 + lane;
    const int d = q >> 3, part = q & 7;
    if (d < ra)
      per_cp_async16(base + (uint32_t)(d * PER_LINE_STRIDE + part * 16),
                     level + (int64_t)nd[k] * PER_FANOUT + part * 4);
  }
}

__global__ void __launch_bounds__(kThreads) per_update_part_kernel(UpdateArgs a) {
  const PerTree& t = a.t;
  const int T = t.num_levels - 1;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  __shared__ uint32_t s_leaf[kWMaxN];  // this CTA's entries in position order (slots < 2^30)
  __shared__ float s_td[kWMaxN];
  __shared__ float s_np[kWMaxN];       // their new priorities
  __shared__ int s_wcnt[kWPer * kWarps];  // entries of (step q, warp w) at q * kWarps + w
  __shared__ int s_woff[kWPer * kWarps + 1];  // their offsets in position order, then the total
  __shared__ __align__(16) unsigned char s_lines[kWMaxT][32 * PER_LINE_STRIDE];
  per_wait_previous_grid();
  // entries threadIdx.x + q * kThreads for the steps q the batch reaches
  const int steps = (int)((a.n + kThreads - 1) / kThreads);
  int64_t li[kWPer];
  float tv[kWPer];
#pragma unroll
  for (int q = 0; q < kWPer; ++q) {
    li[q] = -1;
    tv[q] = 0.f;
    if (q >= steps) continue;  // the same for the whole block
    const int64_t e = threadIdx.x + q * kThreads;
    if (e < a.n) {
      li[q] = slot_of(a, e);
      tv[q] = a.td[e];
    }
  }
  const int64_t n = entries_of(a);
  // this CTA's entries (those whose top-level ancestor hashes to it), in
  // position order: warp counts, then offsets
  const int tshift = PER_LOG_FANOUT * T;
  const uint32_t kmask = gridDim.x - 1u;  // the launch uses a power-of-two grid
  uint32_t nbad = 0u, nforeign = 0u;
  bool mine[kWPer];
  uint32_t mm[kWPer];
#pragma unroll
  for (int q = 0; q < kWPer; ++q) {
    mine[q] = false;
    mm[q] = 0u;
    if (q >= steps) continue;
    const int64_t e = threadIdx.x + q * kThreads;
    const bool in = e < n;
    const bool valid = in && li[q] >= 0 && li[q] < t.capacity;
    if (in && !valid && blockIdx.x == 0) {
      if (a.strict) ++nbad; else ++nforeign;
    }
    mine[q] = valid && top_cta((uint32_t)li[q] >> tshift, kmask) == blockIdx.x;
    mm[q] = __ballot_sync(PER_FULL_MASK, mine[q]);
    if (lane == 0) s_wcnt[q * kWarps + warp] = __popc(mm[q]);
  }
  if (nbad) {
    per_count(t.status, PER_STATUS_BAD_INDICES, nbad);
    per_flag(t.status, PER_EVT_BAD_INDEX);
  }
  if (nforeign) per_count(t.status, PER_STATUS_FOREIGN, nforeign);
  __syncthreads();
  if (warp == 0) {  // offsets of the (step, warp) groups: one warp scan, two per lane
    const int nseg = steps * kWarps;
    const int c0 = lane < nseg ? s_wcnt[lane] : 0;
    const int c1 = lane + 32 < nseg ? s_wcnt[lane + 32] : 0;
    int x0 = c0, x1 = c1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y0 = __shfl_up_sync(PER_FULL_MASK, x0, o);
      const int y1 = __shfl_up_sync(PER_FULL_MASK, x1, o);
      if (lane >= o) {
        x0 += y0;
        x1 += y1;
      }
    }
    const int tot0 = __shfl_sync(PER_FULL_MASK, x0, 31);
    s_woff[lane] = x0 - c0;
    s_woff[lane + 32] = tot0 + x1 - c1;
    if (lane == 31) s_woff[kWPer * kWarps] = tot0 + x1;
  }
  __syncthreads();
  const int cnt = s_woff[kWPer * kWarps];
#pragma unroll
  for (int q = 0; q < kWPer; ++q) {
    if (q >= steps) continue;
    if (mine[q]) {
      const int r = s_woff[q * kWarps + warp] + __popc(mm[q] & ((1u << lane) - 1u));
      s_leaf[r] = (uint32_t)li[q];
      s_td[r] = tv[q];
    }
  }
  __syncthreads();
  if (warp > 0) {
    // the other warps: the new priorities of every entry of this CTA, while
    // warp 0 fetches lines and elects
    uint32_t tmax = 0u;
    for (int j = threadIdx.x - 32; j < cnt; j += kThreads - 32) {
      const float np = new_priority(t, s_td[j]);
      s_np[j] = np;
      tmax = max(tmax, __float_as_uint(np));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tmax = max(tmax, __shfl_xor_sync(PER_FULL_MASK, tmax, o));
    if (lane == 0 && tmax) atomicMax(reinterpret_cast<unsigned int*>(t.max_priority), tmax);
    named_bar_arrive_upd(kThreads);
    return;
  }

  // warp 0: rounds of 32 entries (one per lane)
  for (int r0 = 0; r0 < cnt; r0 += 32) {
    const int ra = min(32, cnt - r0);
    const bool act = lane < ra;
    const uint32_t leaf = act ? s_leaf[r0 + lane] : 0u;
#pragma unroll
    for (int L = 0; L < kWMaxT; ++L) {
      if (L >= T) break;
      warp_issue_lines(t.levels[L], s_lines[L], leaf, ra, L, lane);
    }
    // elections while the lines are in flight (inactive lanes get keys no
    // slot or node can have): the winner of a slot is the highest lane
    // holding it (last occurrence), a node's owner the lowest
    const uint32_t none = 0x80000000u | (uint32_t)lane;
    const uint32_t msl = __match_any_sync(PER_FULL_MASK, act ? leaf : none);
    const bool win = act && (31 - __clz(msl)) == lane;
    int owner[kWMaxT];
#pragma unroll
    for (int L = 0; L < kWMaxT; ++L) {
      owner[L] = lane;
      if (L >= T) break;
      const uint32_t key = act ? (leaf >> (PER_LOG_FANOUT * (L + 1))) : none;
      owner[L] = __ffs(__match_any_sync(PER_FULL_MASK, key)) - 1;
    }
    if (r0 == 0) named_bar_sync_upd(kThreads);  // the new priorities are in s_np
    const float np = act ? s_np[r0 + lane] : 0.f;
    per_cp_async_wait_all();
    __syncwarp();
    // winners: leaf to the store and into the line of their chunk's owner
    if (win) {
      t.levels[0][leaf] = np;
      reinterpret_cast<float*>(s_lines[0] + owner[0] * PER_LINE_STRIDE)[leaf & (PER_FANOUT - 1)] = np;
    }
    __syncwarp();
    // level by level: owners sum, store, patch into the parent owner's line
#pragma unroll
    for (int L = 0; L < kWMaxT; ++L) {
      if (L >= T) break;
      if (act && owner[L] == lane) {
        const float4* row = reinterpret_cast<const float4*>(s_lines[L] + lane * PER_LINE_STRIDE);
        float c[32];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 v = row[k];
          c[4 * k] = v.x;
          c[4 * k + 1] = v.y;
          c[4 * k + 2] = v.z;
          c[4 * k + 3] = v.w;
        }
        const float v = per_sum32_tree(c);
        const uint32_t node = leaf >> (PER_LOG_FANOUT * (L + 1));
        t.levels[L + 1][node] = v;
        if (L + 1 < T)
          reinterpret_cast<float*>(s_lines[L + 1] + owner[L + 1] * PER_LINE_STRIDE)
              [node & (PER_FANOUT - 1)] = v;
      }
      __syncwarp();
    }
  }
  if (cnt == 0) named_bar_sync_upd(kThreads);  // the other warps' barrier completes
}

// ---------------------------------------------------------------- add
struct AddArgs {
  PerTree t;
  per_field_t fields[PER_MAX_FIELDS];
  int32_t n_fields;
  int64_t n;
};

__global__ void __launch_bounds__(kThreads) per_add_kernel(AddArgs a) {
  per_wait_previous_grid();
  const PerTree& t = a.t;
  __shared__ __align__(16) unsigned char s_tiles[kThreads / 32][PER_NODE_TILE];
  PerGridBarrier bar;
  bar.init(t.scratch);
  const int lane = threadIdx.x & 31;
  unsigned char* tile = s_tiles[threadIdx.x >> 5];
  const int64_t C = t.capacity;
  const int64_t size = t.size_cursor[0];
  const int64_t cursor = t.size_cursor[1];
  const float maxp = *t.max_priority;
  const int64_t n0 = a.n > C ? a.n - C : 0;  // earlier rows would be overwritten in this call
  const int64_t m = a.n - n0;
  const int64_t start = (cursor + n0) % C;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;

  // P0: rows and leaves (one warp per row)
  for (int64_t k = gw; k < m; k += nw) {
    const int64_t src_row = n0 + k;
    int64_t pos = start + k;
    if (pos >= C) pos -= C;
    float* dst = t.storage + pos * t.row_stride;
    for (int f = 0; f < a.n_fields; ++f) {
      const per_field_t& fd = a.fields[f];
      const float* src = fd.data + src_row * fd.stride;
      for (int64_t c = lane; c < fd.dim; c += 32) dst[fd.col_offset + c] = src[c];
    }
    if (lane == 0) t.levels[0][pos] = maxp;
  }

  // touched leaf ranges: [start, start+m) on the ring, split at C
  const int64_t a0 = start, a1 = min(start + m, C);
  const int64_t b1 = start + m > C ? start + m - C : 0;
  for (int L = 1; L < t.num_levels; ++L) {
    bar.sync(t.status);
    const int sh = PER_LOG_FANOUT * L;
    const int64_t lo0 = a0 >> sh, hi0 = (a1 - 1) >> sh;
    const int64_t cnt0 = a1 > a0 ? hi0 - lo0 + 1 : 0;
    const int64_t hi1 = b1 > 0 ? (b1 - 1) >> sh : -1;
    const int64_t cnt1 = b1 > 0 ? hi1 + 1 : 0;
    const int64_t total = cnt0 + cnt1;
    for (int64_t base = gw * 32; base < total; base += nw * 32) {
      const int64_t k = base + lane;
      const bool own = k < total;
      const int64_t node = !own ? 0 : (k < cnt0 ? lo0 + k : k - cnt0);
      per_warp_recompute(t.levels[L - 1], t.levels[L], node, own, lane, tile);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    t.size_cursor[1] = (cursor + a.n) % C;
    t.size_cursor[0] = min(size + a.n, C);
  }
}

// ---------------------------------------------------------------- rebuild
__global__ void __launch_bounds__(kThreads) per_rebuild_kernel(PerTree t) {
  per_wait_previous_grid();
  __shared__ __align__(16) unsigned char s_tiles[kThreads / 32][PER_NODE_TILE];
  PerGridBarrier bar;
  bar.init(t.scratch);
  const int lane = threadIdx.x & 31;
  unsigned char* tile = s_tiles[threadIdx.x >> 5];
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const int64_t gw = tid >> 5;
  const int64_t nw = nth >> 5;
  for (int L = 0; L < t.num_levels; ++L)
    for (int64_t k = tid; k < t.level_len[L]; k += nth) t.claims[L][k] = 0u;
  for (int L = 1; L < t.num_levels; ++L) {
    bar.sync(t.status);
    const int64_t nodes = live_nodes(t.capacity, L);
    for (int64_t base = gw * 32; base < nodes; base += nw * 32) {
      const int64_t node = base + lane;
      per_warp_recompute(t.levels[L - 1], t.levels[L], node < nodes ? node : 0, node < nodes, lane,
                         tile);
    }
  }
}

int grid_for(const void* fn, int64_t work, int* grid) {
  int max_ctas = 0;
  int rc = per_coresident_ctas(fn, kThreads, 0, &max_ctas);
  if (rc) return rc;
  if (max_ctas > PER_MAX_GRID) max_ctas = PER_MAX_GRID;
  int64_t g = (work + kThreads - 1) / kThreads;
  if (g > max_ctas) g = max_ctas;
  if (g < 1) g = 1;
  *grid = (int)g;
  return PER_OK;
}

}  // namespace

int per_launch_update(const PerTree& t, const int64_t* idx, const float* td, int64_t n,
                      cudaStream_t stream) {
  return per_launch_update_shard(t, 0, 1, idx, td, n, nullptr, stream);
}

bool per_update_uses_grid(const PerTree& t, int64_t n) {
  return !(n <= kWMaxN && t.num_levels - 1 <= kWMaxT);
}

int per_launch_update_shard(const PerTree& t, int64_t base, int32_t strict, const int64_t* idx,
                            const float* td, int64_t n, const int64_t* count, cudaStream_t stream) {
  UpdateArgs a;
  a.t = t;
  a.idx = idx;
  a.td = td;
  a.n = n;
  a.base = base;
  a.strict = strict;
  a.count = reinterpret_cast<const unsigned long long*>(count);
  const int T = t.num_levels - 1;
  // up to kWMaxN entries: CTAs owning disjoint shares of the top-level nodes
  if (!per_update_uses_grid(t, n)) {
    const void* fw = (const void*)per_update_part_kernel;
    // a power of two near n / kWEntriesPerCta, at most the top level's nodes
    int64_t k = 1;
    while (k * kWEntriesPerCta < n && 2 * k <= t.level_len[T]) k *= 2;
    void* args[] = {&a};
    cudaError_t e = per_launch(fw, (unsigned)k, kThreads, 0, stream, args, false);
    return e == cudaSuccess ? PER_OK : per_record_cuda(e);
  }
  // larger batches: the co-resident grid
  const void* fn = (const void*)per_update_kernel;
  int grid = 0;
  int rc = grid_for(fn, n, &grid);
  if (rc) return rc;
  if ((int64_t)grid * kThreads * kMaxPerThread < n) return PER_ERR_TOO_LARGE;
  void* args[] = {&a};
  cudaError_t e = per_launch(fn, (unsigned)grid, kThreads, 0, stream, args, grid > 1);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}

int per_launch_add(const PerTree& t, const per_field_t* fields, int32_t n_fields, int64_t n,
                   cudaStream_t stream) {
  AddArgs a;
  a.t = t;
  for (int f = 0; f < n_fields; ++f) a.fields[f] = fields[f];
  a.n_fields = n_fields;
  a.n = n;
  const void* fn = (const void*)per_add_kernel;
  const int64_t rows = n < t.capacity ? n : t.capacity;
  int grid = 0;
  int rc = grid_for(fn, rows * 32, &grid);
  if (rc) return rc;
  void* args[] = {&a};
  cudaError_t e = per_launch(fn, (unsigned)grid, kThreads, 0, stream, args, grid > 1);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}

int per_launch_rebuild(const PerTree& t, cudaStream_t stream) {
  PerTree a = t;
  const void* fn = (const void*)per_rebuild_kernel;
  int grid = 0;
  int rc = grid_for(fn, t.level_len[0], &grid);
  if (rc) return rc;
  void* args[] = {&a};
  cudaError_t e = per_launch(fn, (unsigned)grid, kThreads, 0, stream, args, grid > 1);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}
