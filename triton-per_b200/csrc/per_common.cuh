// Shared device helpers of the replay engine: store view, warp scans,
// bounded grid barrier, status counters.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "per_b200.h"

#define PER_FULL_MASK 0xffffffffu

// Spin limit of every wait: about 2^22 polls with a 256 ns back-off, i.e.
// on the order of one second before the wait gives up and reports
// PER_EVT_BARRIER_TIMEOUT instead of hanging the GPU.
#define PER_SPIN_LIMIT (1u << 22)
#define PER_SPIN_SLEEP_NS 256

// Layout of store->scratch (PER_SCRATCH_BYTES).
struct PerScratch {
  uint32_t bar_count;  // arrivals at the current grid barrier
  uint32_t bar_gen;    // generation, bumped by the last arriver
  float gmax;          // value published by the last arriver
  uint32_t pad[61];    // keep partial[] 256-byte aligned
  float partial[PER_MAX_GRID];
};
static_assert(sizeof(PerScratch) == PER_SCRATCH_BYTES, "scratch layout");

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

__device__ __forceinline__ void per_count(uint32_t* status, int word, uint32_t n = 1) {
  if (status) atomicAdd(status + word, n);
}

__device__ __forceinline__ void per_flag(uint32_t* status, uint32_t bit) {
  if (status) atomicOr(status + PER_STATUS_ERRORS, bit);
}

// Positive floats order like their bit patterns, so max over non-negative
// values (and +inf / positive NaN, which sort above) is an integer max.
__device__ __forceinline__ void per_atomic_max_pos(float* addr, float v) {
  atomicMax(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
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

// Sum of the 32 children [32*node, 32*node+32) of level `lvl`, in float64,
// in a fixed order (deterministic). Loads bypass L1 because the children may
// have been written by other CTAs earlier in the same launch.
__device__ __forceinline__ double per_sum32(const float* lvl, int64_t node) {
  const float4* p = reinterpret_cast<const float4*>(lvl + node * PER_FANOUT);
  float4 q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = __ldcg(p + i);
  double s = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s += (double)q[i].x;
    s += (double)q[i].y;
    s += (double)q[i].z;
    s += (double)q[i].w;
  }
  return s;
}
