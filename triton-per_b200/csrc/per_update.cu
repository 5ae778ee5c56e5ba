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
//   * small batches (<= 1024 indices): one CTA, election in shared-memory
//     hash tables; per level the touched nodes are listed (warp counts, then
//     offsets) and recomputed 32 per warp; levels separated by __syncthreads;
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

constexpr uint32_t kEmpty = 0xffffffffu;

// ---------------------------------------------------------------- prefetched update
// Batches of up to kLMaxN indices whose lines fit in shared memory. The nodes
// that an update touches are known from the leaf indices alone (node of level
// L = leaf >> 5L), so every 32-child line the recompute needs (children of
// every touched node of every level) is fetched at once, right after the
// election: one L2 round trip for the whole update instead of one per level.
// The new values are then patched into the staged lines (winning leaves
// first, then each recomputed node into its parent's line) and every level
// is summed from shared memory. Node values are the same per_sum32_tree of
// the same children as in the other update paths, so the tree bits do not
// depend on the path.
constexpr int kLPer = 2;                   // entries per thread
constexpr int kLMaxN = kThreads * kLPer;   // 512
constexpr int kLHashBits = 10;
constexpr int kLHash = 1 << kLHashBits;    // load factor <= 1/2
constexpr int kLMaxT = 4;                  // tree levels above the leaves
constexpr size_t kLinesSmemMax = 200 * 1024;  // shared memory the kernel may ask for
constexpr int kLinesMaxPasses = 8;            // beyond this many passes: the grid path

__device__ __forceinline__ uint32_t lslot(uint32_t key) {
  return (key * 2654435761u) >> (32 - kLHashBits);
}

__device__ __forceinline__ int lset_insert(uint32_t* keys, uint32_t key) {
  uint32_t s = lslot(key);
  for (int probe = 0; probe < kLHash; ++probe) {
    const uint32_t prev = atomicCAS(&keys[s], kEmpty, key);
    if (prev == kEmpty || prev == key) return (int)s;
    s = (s + 1) & (kLHash - 1);
  }
  return -1;
}

// Shared-memory bytes of the prefetched update for T levels above the leaves
// and up to ncap nodes per level.
__host__ __device__ __forceinline__ size_t lines_smem(int T, int ncap) {
  return (size_t)T * ncap * PER_LINE_STRIDE          // staged lines
         + (size_t)(2 + 2 * T) * kLHash * 4          // election table, node sets + positions
         + (size_t)2 * T * ncap * 4;                 // node lists + parents' set slots
}

__global__ void __launch_bounds__(kThreads, 1) per_update_lines_kernel(UpdateArgs a, int ncap) {
  const PerTree& t = a.t;
  const int T = t.num_levels - 1;
  extern __shared__ __align__(16) unsigned char s_dyn[];
  unsigned char* lines = s_dyn;            // [T][ncap] staged lines
  uint32_t* wkey = reinterpret_cast<uint32_t*>(lines + (size_t)T * ncap * PER_LINE_STRIDE);
  uint32_t* wval = wkey + kLHash;
  uint32_t* skey = wval + kLHash;          // [T][kLHash] node sets
  uint32_t* spos = skey + T * kLHash;      // [T][kLHash] list position of each set slot
  uint32_t* list = spos + T * kLHash;      // [T][ncap] touched nodes per level
  uint32_t* pslot = list + T * ncap;       // [T][ncap] set slot of the node's parent
  __shared__ int s_cnt[kLMaxT];
  __shared__ uint32_t s_max;
  __shared__ uint32_t s_fresh[kThreads / 32][32];  // nodes a warp entered first, in list order
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t lbase = per_smem_addr_generic(lines);

  // the first pass's tables are cleared while the previous kernel may still run
  for (int k = threadIdx.x; k < kLHash; k += kThreads) {
    wkey[k] = kEmpty;
    wval[k] = 0u;
    for (int L = 0; L < T; ++L) skey[L * kLHash + k] = kEmpty;
  }
  if (threadIdx.x < kLMaxT) s_cnt[threadIdx.x] = 0;
  if (threadIdx.x == 0) s_max = 0u;
  per_wait_previous_grid();
  // the first pass's entries are loaded together with the device count (a
  // sharded update reads how many entries its sample owns): entries past the
  // count are loaded (inside the caller's n) but not used
  int64_t li[kLPer];
  float tdv[kLPer];
#pragma unroll
  for (int q = 0; q < kLPer; ++q) {
    const int64_t e = threadIdx.x + q * kThreads;
    const bool in = e < a.n && e < ncap;
    li[q] = in ? slot_of(a, e) : -1;
    tdv[q] = in ? a.td[e] : 0.f;
  }
  const int64_t n = entries_of(a);

  // passes of `ncap` entries in order; a later pass overwrites an earlier
  // one's leaves, so the last occurrence of a slot wins across passes too
  for (int64_t c0 = 0; c0 < n; c0 += ncap) {
    if (c0 > 0) {
      __syncthreads();
      for (int k = threadIdx.x; k < kLHash; k += kThreads) {
        wkey[k] = kEmpty;
        wval[k] = 0u;
        for (int L = 0; L < T; ++L) skey[L * kLHash + k] = kEmpty;
      }
      if (threadIdx.x < kLMaxT) s_cnt[threadIdx.x] = 0;
      if (threadIdx.x == 0) s_max = 0u;
    }
    const int64_t c1 = min(c0 + ncap, n);
#pragma unroll
    for (int q = 0; q < kLPer; ++q) {
      const int64_t e = c0 + threadIdx.x + q * kThreads;
      if (c0 > 0) {
        li[q] = e < c1 ? slot_of(a, e) : -1;
        tdv[q] = e < c1 ? a.td[e] : 0.f;
      } else if (e >= c1) {  // loaded past the device count: not an entry
        li[q] = -1;
        tdv[q] = 0.f;
      }
    }
    __syncthreads();

    // election (the last occurrence of a slot wins: largest position). Every
    // valid entry also enters the node of each level above its leaf; the
    // entry that adds a node first gives it a list position, and the warp
    // fetches its new nodes' lines right away (the winner of a slot touches
    // the same nodes)
    int slot[kLPer], lslot0[kLPer];
    float np[kLPer];
    uint32_t tmax = 0u, nbad = 0u, nforeign = 0u;
#pragma unroll
    for (int q = 0; q < kLPer; ++q) {
      const int64_t e = c0 + threadIdx.x + q * kThreads;
      slot[q] = -1;
      lslot0[q] = -1;
      np[q] = 0.f;
      // the same for every thread of the block: a pass past the last entry
      // has nothing to elect (a batch of at most kThreads takes one)
      if (c0 + (int64_t)q * kThreads >= c1) continue;
      bool valid = false;
      if (e < c1) {
        if (li[q] < 0 || li[q] >= t.capacity) {
          if (a.strict) ++nbad; else ++nforeign;
        } else {
          valid = true;
          // the slot's table entry first: the atomics' round trips overlap powf
          slot[q] = lset_insert(wkey, (uint32_t)li[q]);
          np[q] = new_priority(t, tdv[q]);
          tmax = max(tmax, __float_as_uint(np[q]));
          if (slot[q] >= 0) atomicMax(&wval[slot[q]], (uint32_t)(e + 1));
        }
      }
      uint32_t nd = valid ? (uint32_t)li[q] >> PER_LOG_FANOUT : 0u;
      int below_p = -1;  // list position of the node entered at the level below, if new
      for (int L = 0; L < T; ++L) {
        int sl = -1;
        bool fresh = false;
        if (valid) {
          uint32_t h = lslot(nd);
          uint32_t* keys = skey + L * kLHash;
          for (int probe = 0; probe < kLHash; ++probe) {
            const uint32_t prev = atomicCAS(&keys[h], kEmpty, nd);
            if (prev == kEmpty || prev == nd) {
              sl = (int)h;
              fresh = prev == kEmpty;
              break;
            }
            h = (h + 1) & (kLHash - 1);
          }
        }
        // list positions for the warp's new nodes: one shared counter add
        const uint32_t m = __ballot_sync(PER_FULL_MASK, fresh);
        int pbase = 0;
        if (lane == 0 && m) pbase = atomicAdd(&s_cnt[L], __popc(m));
        pbase = __shfl_sync(PER_FULL_MASK, pbase, 0);
        const int newp = fresh ? pbase + __popc(m & ((1u << lane) - 1u)) : -1;
        if (L == 0) lslot0[q] = sl;
        if (below_p >= 0) pslot[(L - 1) * ncap + below_p] = (uint32_t)sl;  // parent of that node
        const int nf = __popc(m);
        if (fresh) {
          list[L * ncap + newp] = nd;
          spos[L * kLHash + sl] = (uint32_t)newp;
          s_fresh[warp][newp - pbase] = nd;  // the node of the warp's (newp - pbase)-th new entry
        }
        __syncwarp();
        // the warp fetches its new nodes' lines together, 4 lines (8 x 16 B
        // each) per instruction: every node index is read first, then all
        // the copies go out back to back
        const float* clevel = t.levels[L];
        const int part = lane & 7;
        uint32_t gn[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int g = (lane >> 3) + 4 * i;
          gn[i] = g < nf ? s_fresh[warp][g] : 0u;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int g = (lane >> 3) + 4 * i;
          if (g < nf)
            per_cp_async16(lbase + (uint32_t)((L * ncap + pbase + g) * PER_LINE_STRIDE + part * 16),
                           clevel + (int64_t)gn[i] * PER_FANOUT + part * 4);
        }
        __syncwarp();
        below_p = newp;
        nd >>= PER_LOG_FANOUT;
      }
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

    // winners write their leaf; every thread waits for the lines it fetched
    bool win[kLPer];
#pragma unroll
    for (int q = 0; q < kLPer; ++q) {
      const int64_t e = c0 + threadIdx.x + q * kThreads;
      win[q] = slot[q] >= 0 && wval[slot[q]] == (uint32_t)(e + 1);
      if (win[q]) t.levels[0][li[q]] = np[q];
    }
    per_cp_async_wait_all();
    __syncthreads();

    // the winning leaves go into their chunk lines
#pragma unroll
    for (int q = 0; q < kLPer; ++q) {
      if (win[q]) {
        float* line = reinterpret_cast<float*>(lines + (size_t)spos[lslot0[q]] * PER_LINE_STRIDE);
        line[li[q] & (PER_FANOUT - 1)] = np[q];
      }
    }
    __syncthreads();

    // level by level: sum each touched node's line, store it, patch it into
    // its parent's line
    for (int L = 0; L < T; ++L) {
      for (int p = threadIdx.x; p < s_cnt[L]; p += kThreads) {
        const uint32_t node = list[L * ncap + p];
        const float4* row =
            reinterpret_cast<const float4*>(lines + (size_t)(L * ncap + p) * PER_LINE_STRIDE);
        float c[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 v = row[i];
          c[4 * i] = v.x;
          c[4 * i + 1] = v.y;
          c[4 * i + 2] = v.z;
          c[4 * i + 3] = v.w;
        }
        const float v = per_sum32_tree(c);
        t.levels[L + 1][node] = v;
        if (L + 1 < T) {
          const uint32_t pp = spos[(L + 1) * kLHash + pslot[L * ncap + p]];
          float* pline = reinterpret_cast<float*>(
              lines + (size_t)((L + 1) * ncap + pp) * PER_LINE_STRIDE);
          pline[node & (PER_FANOUT - 1)] = v;
        }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------- partitioned update
// Batches of up to kWMaxN indices: K one-warp CTAs, CTA k taking the entries
// whose top-level ancestor (the node of level T above the leaf, T the highest
// maintained level) hashes to k. Entries under different top-level nodes
// touch disjoint nodes at every level, so the CTAs never coordinate: each
// loads every entry, keeps its own in position order, and applies them in
// rounds of 32 (one per lane). A round fetches every lane's line of every
// level at once (duplicates included), elects the winner of each slot (the
// highest lane among equal slots: the last occurrence) and the owner of each
// touched node (the lowest lane among equal nodes) with warp matches while
// the lines are in flight, then patches the winning leaves into their
// owner's line and sums level by level, each owner patching its node into
// the line of its parent's owner. Later rounds see earlier rounds' writes
// (same warp, program order), so the last occurrence wins across rounds too.
// Node values are per_sum32_tree of the same children as in the other update
// paths.
constexpr int kWMaxN = 512;              // entries of a batch
constexpr int kWEntriesPerCta = 16;      // expected entries per CTA
constexpr int kWMaxT = 4;                // tree levels above the leaves

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

constexpr int kWPer = kWMaxN / kThreads;  // entries per thread

__global__ void __launch_bounds__(kThreads) per_update_warp_kernel(UpdateArgs a) {
  const PerTree& t = a.t;
  const int T = t.num_levels - 1;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  __shared__ uint32_t s_leaf[kWMaxN];  // this CTA's entries in position order (slots < 2^30)
  __shared__ float s_td[kWMaxN];
  __shared__ float s_np[kWMaxN];       // their new priorities
  __shared__ int s_wcnt[kWPer][kThreads / 32];
  __shared__ __align__(16) unsigned char s_lines[kWMaxT][32 * PER_LINE_STRIDE];
  per_wait_previous_grid();
  int64_t li[kWPer];
  float tv[kWPer];
#pragma unroll
  for (int q = 0; q < kWPer; ++q) {
    const int64_t e = threadIdx.x + q * kThreads;
    li[q] = e < a.n ? slot_of(a, e) : -1;
    tv[q] = e < a.n ? a.td[e] : 0.f;
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
    const int64_t e = threadIdx.x + q * kThreads;
    const bool in = e < n;
    const bool valid = in && li[q] >= 0 && li[q] < t.capacity;
    if (in && !valid && blockIdx.x == 0) {
      if (a.strict) ++nbad; else ++nforeign;
    }
    mine[q] = valid && top_cta((uint32_t)li[q] >> tshift, kmask) == blockIdx.x;
    mm[q] = __ballot_sync(PER_FULL_MASK, mine[q]);
    if (lane == 0) s_wcnt[q][warp] = __popc(mm[q]);
  }
  if (nbad) {
    per_count(t.status, PER_STATUS_BAD_INDICES, nbad);
    per_flag(t.status, PER_EVT_BAD_INDEX);
  }
  if (nforeign) per_count(t.status, PER_STATUS_FOREIGN, nforeign);
  __syncthreads();
  int cnt = 0;
#pragma unroll
  for (int q = 0; q < kWPer; ++q) {
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) {
      if (w == warp && mine[q]) {
        const int r = cnt + __popc(mm[q] & ((1u << lane) - 1u));
        s_leaf[r] = (uint32_t)li[q];
        s_td[r] = tv[q];
      }
      cnt += s_wcnt[q][w];
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

namespace {

// Entries per pass of the single-CTA prefetched update for this tree and
// batch (0 when it cannot serve the tree).
int lines_ncap(const PerTree& t, int64_t n) {
  const int T = t.num_levels - 1;
  if (T > kLMaxT) return 0;
  const int64_t want = n < kLMaxN ? n : kLMaxN;
  for (int c = (int)((want + 31) / 32 * 32); c >= 32; c -= 32)
    if (lines_smem(T, c) <= kLinesSmemMax) return c;
  return 0;
}

}  // namespace

bool per_update_uses_grid(const PerTree& t, int64_t n) {
  const int ncap = lines_ncap(t, n);
  return !(ncap > 0 && n <= (int64_t)kLinesMaxPasses * ncap);
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
  // up to kWMaxN entries: one-warp CTAs, each owning the entries under its
  // share of the top-level nodes
  if (n <= kWMaxN && T <= kWMaxT) {
    const void* fw = (const void*)per_update_warp_kernel;
    // a power of two near n / kWEntriesPerCta, at most the top level's nodes
    int64_t k = 1;
    while (k * kWEntriesPerCta < n && 2 * k <= t.level_len[T]) k *= 2;
    void* args[] = {&a};
    cudaError_t e = per_launch(fw, (unsigned)k, kThreads, 0, stream, args, false);
    return e == cudaSuccess ? PER_OK : per_record_cuda(e);
  }
  // one CTA, passes of `ncap` entries with every line prefetched, while the
  // passes stay few; larger batches take the grid path
  int ncap = lines_ncap(t, n);
  if (!per_update_uses_grid(t, n)) {
    const void* fl = (const void*)per_update_lines_kernel;
    const size_t smem = lines_smem(T, ncap);
    int rc = per_set_smem(fl, kLinesSmemMax);
    if (rc) return rc;
    void* args[] = {&a, &ncap};
    cudaError_t e = per_launch(fl, 1, kThreads, smem, stream, args, false);
    return e == cudaSuccess ? PER_OK : per_record_cuda(e);
  }
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
