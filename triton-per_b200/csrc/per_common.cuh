// Shared device helpers of the replay engine: store view, warp scans,
// bounded grid barrier, status counters.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "per_b200.h"

#define PER_FULL_MASK 0xffffffffu

// Spin limit of every wait: 2^22 polls (each an L2 round trip plus a short
// back-off), i.e. on the order of a second before the wait gives up and
// reports PER_EVT_BARRIER_TIMEOUT instead of hanging the GPU.
#define PER_SPIN_LIMIT (1u << 22)
#define PER_SPIN_SLEEP_NS 32
// Waits on another GPU (a peer rank's kernel, launched by another process)
// are bounded by time: 1 s on the global timer, and at most 2^26 polls.
#define PER_PEER_WAIT_NS 1000000000ull
#define PER_PEER_SPIN_LIMIT (1u << 26)

// Layout of store->scratch (PER_SCRATCH_BYTES).
struct PerScratch {
  uint32_t bar_count;    // arrivals at the current grid barrier
  uint32_t bar_gen;      // generation, bumped by the last arriver
  uint32_t mx_gen;       // sample: launch generation, bumped once every CTA has published
  uint32_t pad0[3];
  unsigned long long draws[2];  // sharded sample: owned-draw counter, by generation parity
  unsigned long long mx_result;      // sample, large grids: (generation + 1) << 32 | max bits
  unsigned long long mx_result_cnt;  // sample, large grids: (generation + 1) << 32 | owned draws
  uint32_t pad[50];      // keep mx_slot[] 256-byte aligned
  // sample: per CTA two words, (generation + 1) << 32 | CTA max weight bits
  // and (generation + 1) << 32 | draws the CTA owns (sharded)
  unsigned long long mx_slot[PER_MAX_GRID / 2];
};
static_assert(sizeof(PerScratch) == PER_SCRATCH_BYTES, "scratch layout");

// Sharded mode, exchange over peer memory: every rank owns one mailbox,
// mapped into every peer's process. Rank g writes its shard statistics and
// its max weight into slot g of every mailbox; each rank reads only its own
// mailbox. Every 64-bit word carries 32 bits of data and the 32-bit tag of
// the call it belongs to (one single-copy-atomic store: no fence on either
// side), and a reader waits until every word of a slot carries this call's
// tag.
struct PerMailbox {
  unsigned long long seq;  // sample calls completed by the owning rank (local)
  unsigned long long pad0[15];
  // slot g of call parity p: total (2 halves), size (2 halves); two parities,
  // because without the max exchange a peer may publish call k+1 while this
  // rank still reads call k
  unsigned long long stats[2][PER_MAX_SHARDS][4];
  unsigned long long max_w[PER_MAX_SHARDS];     // slot g: max weight bits
};
static_assert(sizeof(PerMailbox) <= PER_MAILBOX_BYTES, "mailbox layout");

// tag of call `seq` (never 0, the value of a fresh mailbox)
__device__ __forceinline__ uint32_t per_mail_tag(unsigned long long seq) {
  return (uint32_t)(seq & 0x7fffffffull) | 0x80000000u;
}

__device__ __forceinline__ void per_st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long per_ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void per_mail_put(unsigned long long* p, uint32_t data, uint32_t tag) {
  per_st_relaxed_sys_u64(p, ((unsigned long long)tag << 32) | data);
}

__device__ __forceinline__ void per_st_release_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long per_ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t per_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void per_st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float per_ld_relaxed_f32(const float* p) {
  float v;
  asm volatile("ld.relaxed.gpu.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t per_ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// atomic add with acquire-release semantics at GPU scope; returns the old value
__device__ __forceinline__ uint32_t per_atom_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void per_count(uint32_t* status, int word, uint32_t n = 1) {
  if (status) atomicAdd(status + word, n);
}

__device__ __forceinline__ void per_flag(uint32_t* status, uint32_t bit) {
  if (status) atomicOr(status + PER_STATUS_ERRORS, bit);
}

// Programmatic dependent launch: kernels are launched so that they may start
// while the previous kernel on the stream is still running. Each kernel waits
// here, before it reads anything an earlier kernel wrote (no-op when the
// launch had no programmatic dependency), then lets the next kernel launch.
__device__ __forceinline__ void per_wait_previous_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ unsigned long long per_globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void per_st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long per_ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until the mailbox words p[0..n) all carry `tag`; returns their
// data halves in out[]. False and a flagged peer timeout if the peer does not
// publish within PER_PEER_WAIT_NS (a rank that left the collective, or one
// far behind).
__device__ __forceinline__ bool per_mail_get(const unsigned long long* p, int n, uint32_t tag,
                                             uint32_t* out, uint32_t* status) {
  unsigned long long t0 = 0ull;
  for (uint32_t it = 0;; ++it) {
    bool ready = true;
    for (int k = 0; k < n; ++k) {
      const unsigned long long v = per_ld_relaxed_sys_u64(p + k);
      out[k] = (uint32_t)v;
      ready &= (uint32_t)(v >> 32) == tag;
    }
    if (ready) return true;
    if (it == 0) t0 = per_globaltimer();
    if (it > PER_PEER_SPIN_LIMIT ||
        ((it & 255u) == 255u && per_globaltimer() - t0 > PER_PEER_WAIT_NS)) {
      per_flag(status, PER_EVT_PEER_TIMEOUT);
      per_count(status, PER_STATUS_TIMEOUTS);
      return false;
    }
    __nanosleep(PER_SPIN_SLEEP_NS);
  }
}

// Positive floats order like their bit patterns, so max over non-negative
// values (and +inf / positive NaN, which sort above) is an integer max.
__device__ __forceinline__ void per_atomic_max_pos(float* addr, float v) {
  atomicMax(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

__device__ __forceinline__ uint32_t per_smem_addr_generic(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// Butterfly sum of one float64 per lane; every lane gets the same bits.
__device__ __forceinline__ double per_warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Inclusive warp scan in float64.
__device__ __forceinline__ double per_warp_scan_incl(double v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    double y = __shfl_up_sync(PER_FULL_MASK, v, o);
    if (lane >= o) v += y;
  }
  return v;
}

// Grid barrier across the CTAs of one launch, split into arrive and wait so
// that independent work can run between the two. All CTAs of the grid must
// be co-resident (grid <= occupancy x SMs; the launcher guarantees it).
// Every wait is bounded: on timeout it flags PER_EVT_BARRIER_TIMEOUT and
// returns, so a broken launch ends with an error status instead of a hang.
struct PerGridBarrier {
  PerScratch* s;
  uint32_t gen;  // generation this CTA waits to see bumped (thread 0 only)

  __device__ __forceinline__ void init(PerScratch* scratch) {
    s = scratch;
    if (threadIdx.x == 0) gen = per_ld_acquire(&s->bar_gen);
  }

  // Thread 0 only, after a __syncthreads that completed this CTA's writes.
  // Returns true for the last CTA to arrive.
  __device__ __forceinline__ bool arrive_thread0() {
    __threadfence();
    uint32_t ticket = atomicAdd(&s->bar_count, 1u);
    return ticket == gridDim.x - 1;
  }

  // Thread 0 of the last arriver: reset and release everyone.
  __device__ __forceinline__ void release_thread0() {
    s->bar_count = 0;
    __threadfence();
    per_st_release(&s->bar_gen, gen + 1);
  }

  // Thread 0 only. Returns false on timeout.
  __device__ __forceinline__ bool wait_thread0(uint32_t* status) {
    uint32_t it = 0;
    while (per_ld_acquire(&s->bar_gen) == gen) {
      if (++it > PER_SPIN_LIMIT) {
        per_flag(status, PER_EVT_BARRIER_TIMEOUT);
        per_count(status, PER_STATUS_TIMEOUTS);
        gen = gen + 1;
        return false;
      }
      __nanosleep(PER_SPIN_SLEEP_NS);
    }
    gen = gen + 1;
    __threadfence();
    return true;
  }

  // Full barrier for the whole CTA (all threads call it).
  __device__ __forceinline__ void sync(uint32_t* status) {
    __syncthreads();
    if (gridDim.x > 1) {
      if (threadIdx.x == 0) {
        if (arrive_thread0()) release_thread0();
        wait_thread0(status);
      }
      __syncthreads();
    }
  }
};

// Device view of the parts of a store that the kernels need.
struct PerTree {
  float* levels[PER_MAX_LEVELS];
  uint32_t* claims[PER_MAX_LEVELS];
  int64_t level_len[PER_MAX_LEVELS];
  int32_t num_levels;
  int32_t top_level;
  int64_t capacity;
  float* storage;
  int64_t row_dim;
  int64_t row_stride;
  int64_t* size_cursor;
  float* max_priority;
  uint32_t* status;
  PerScratch* scratch;
  float alpha;
  float eps;
};

// ---- node recomputation (the single definition of a node value)
//
// A node's value is the float32 rounding of the float64 sum of its 32
// children taken as a balanced tree in "butterfly" order: children i and
// i+16 first, then pairs 8 apart, 4, 2, 1. Every writer of the tree (update,
// add, rebuild) uses per_sum32_tree below, so a node always has the same bits
// whichever kernel wrote it.
__device__ __forceinline__ float per_sum32_tree(const float* c) {
  double p[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) p[i] = (double)c[i] + (double)c[i + 16];
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] += p[i + 8];
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] += p[i + 4];
  p[0] += p[2];
  p[1] += p[3];
  return __double2float_rn(p[0] + p[1]);
}


constexpr int PER_LINE_STRIDE = 144;                       // staged 128-byte line + 16 (no bank conflicts)
constexpr int PER_NODE_LINES = 32 * PER_LINE_STRIDE;       // 32 staged lines
constexpr int PER_NODE_TILE = PER_NODE_LINES + 32 * 8;     // + the warp's node list

__device__ __forceinline__ void per_cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}

__device__ __forceinline__ void per_cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Stage the 32-child lines of up to 32 nodes into `tile` (one per warp,
// PER_NODE_TILE bytes): line d holds the children of node nd(d). `node_of(d)`
// must be callable by every lane for d in [0, 32) (warp-uniform use of
// shuffles inside is allowed). 4 lines per cp.async instruction, coalesced.
// Loads bypass L1 (cp.async.cg): children may come from other CTAs of the launch.
template <typename NodeOf>
__device__ __forceinline__ void per_stage_lines(const float* child, unsigned char* tile, int cnt,
                                                int lane, NodeOf node_of) {
  const uint32_t base = per_smem_addr_generic(tile);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int q = i * 32 + lane;
    const int d = q >> 3, part = q & 7;
    const int64_t nd = node_of(d);
    if (d < cnt)
      per_cp_async16(base + (uint32_t)(d * PER_LINE_STRIDE + part * 16),
                     child + nd * PER_FANOUT + part * 4);
  }
  per_cp_async_wait_all();
  __syncwarp();
}

// Recompute node[l] of level `lvl` from level `child` for every lane whose
// `own` is set: the owners' lines are staged together (one L2 round trip for
// up to 32 nodes), then each owner sums its own line.
__device__ __forceinline__ void per_warp_recompute(const float* child, float* lvl, int64_t node,
                                                   bool own, int lane, unsigned char* tile) {
  const uint32_t m = __ballot_sync(PER_FULL_MASK, own);
  if (!m) return;
  const int cnt = __popc(m);
  const int rank = __popc(m & ((1u << lane) - 1u));
  int64_t* list = reinterpret_cast<int64_t*>(tile + PER_NODE_LINES);
  if (own) list[rank] = node;
  __syncwarp();
  per_stage_lines(child, tile, cnt, lane, [&](int d) { return d < cnt ? list[d] : (int64_t)0; });
  if (own) {
    const float4* row = reinterpret_cast<const float4*>(tile + rank * PER_LINE_STRIDE);
    float c[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = row[i];
      c[4 * i] = v.x;
      c[4 * i + 1] = v.y;
      c[4 * i + 2] = v.z;
      c[4 * i + 3] = v.w;
    }
    lvl[node] = per_sum32_tree(c);
  }
  __syncwarp();
}

// ---- Tensor Memory Accelerator bulk copies (no multicast) and mbarriers
__device__ __forceinline__ uint32_t per_smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void per_mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(per_smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void per_fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void per_mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(per_smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool per_mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(per_smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of an mbarrier; false (and a flagged
// timeout) if it did not complete within the spin limit.
__device__ __forceinline__ bool per_mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
  uint32_t it = 0;
  while (!per_mbar_try_wait(bar, parity)) {
    if (++it > PER_SPIN_LIMIT) {
      per_flag(status, PER_EVT_BARRIER_TIMEOUT);
      per_count(status, PER_STATUS_TIMEOUTS);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

// Order earlier generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) writes to the same shared memory.
__device__ __forceinline__ void per_fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Tensor Memory Accelerator gather of four rows (y0..y3, from column x) of
// the 2-D tensor described by `tmap` (a tensor map in parameter or global
// memory whose box is one row high) into four consecutive box rows of this
// CTA's shared memory at `sdst` (128-byte aligned), completing on `bar`.
// x times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void per_tma_gather4(void* sdst, const void* tmap, int x, int y0, int y1,
                                                int y2, int y3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(per_smem_addr(sdst)),
      "l"(tmap), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(per_smem_addr(bar))
      : "memory");
}

// Bring a tensor map (a kernel parameter or global memory) into the
// descriptor cache ahead of its first copy.
__device__ __forceinline__ void per_prefetch_tensormap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void per_bulk_load(void* sdst, const void* gsrc, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          per_smem_addr(sdst)),
      "l"(gsrc), "r"(bytes), "r"(per_smem_addr(bar))
      : "memory");
}

// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC 2011): 10 rounds of two
// 32x32->64 multiplies with the round keys bumped by the Weyl constants.
// Draw j of a stream uses counter (lo(j), hi(j), 0, 0) and key (lo(seed),
// hi(seed)); its uniform is the top 24 bits of the first output word times
// 2^-24, in [0, 1).
#define PER_PHILOX_M0 0xD2511F53u
#define PER_PHILOX_M1 0xCD9E8D57u
#define PER_PHILOX_W0 0x9E3779B9u
#define PER_PHILOX_W1 0xBB67AE85u

__host__ __device__ __forceinline__ void per_philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)PER_PHILOX_M0 * c[0];
    const uint64_t p1 = (uint64_t)PER_PHILOX_M1 * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n1 = (uint32_t)p1;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    const uint32_t n3 = (uint32_t)p0;
    c[0] = n0;
    c[1] = n1;
    c[2] = n2;
    c[3] = n3;
    k0 += PER_PHILOX_W0;
    k1 += PER_PHILOX_W1;
  }
}

__host__ __device__ __forceinline__ float per_philox_uniform(unsigned long long seed,
                                                             unsigned long long j) {
  uint32_t c[4] = {(uint32_t)j, (uint32_t)(j >> 32), 0u, 0u};
  per_philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  return (float)(c[0] >> 8) * 5.9604644775390625e-08f;  // 2^-24
}
