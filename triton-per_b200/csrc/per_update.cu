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
// refresh), every touched node is recomputed exactly from its 32 children in
// float64, level by level, separated by grid barriers. Exactly one writer per
// slot and per node is elected with atomicMax on a claim word, which makes the
// result deterministic: for duplicate indices the last occurrence wins, and
// the sums never drift. Claims are reset by their owner in the phase that
// reads them, so the claim arrays are all-zero between launches.
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
};

__global__ void __launch_bounds__(kThreads) per_update_kernel(UpdateArgs a) {
  const PerTree& t = a.t;
  PerGridBarrier bar;
  bar.init(t.scratch);
  __shared__ uint32_t s_max;
  if (threadIdx.x == 0) s_max = 0u;
  __syncthreads();

  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  uint32_t* tags = t.claims[0];
  float* leaves = t.levels[0];

  // P0: new priorities, winner election (largest position wins), max priority
  uint32_t active = 0u, tmax = 0u, nbad = 0u;
  for (int q = 0; q < kMaxPerThread; ++q) {
    const int64_t e = tid + (int64_t)q * nth;
    if (e >= a.n) break;
    const int64_t i = a.idx[e];
    if (i < 0 || i >= t.capacity) {
      ++nbad;
      continue;
    }
    const float np = powf(fabsf(a.td[e]) + t.eps, t.alpha);
    tmax = max(tmax, __float_as_uint(np));
    atomicMax(tags + i, (uint32_t)(e + 1));
    active |= 1u << q;
  }
  if (nbad) {
    per_count(t.status, PER_STATUS_BAD_INDICES, nbad);
    per_flag(t.status, PER_EVT_BAD_INDEX);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tmax = max(tmax, __shfl_xor_sync(PER_FULL_MASK, tmax, o));
  if ((threadIdx.x & 31) == 0 && tmax) atomicMax(&s_max, tmax);
  __syncthreads();
  if (threadIdx.x == 0 && s_max) atomicMax(reinterpret_cast<unsigned int*>(t.max_priority), s_max);

  bar.sync(t.status);

  // P1: winners write their leaf and claim the chunk
  uint32_t next = 0u;
  for (uint32_t m = active; m; m &= m - 1) {
    const int q = __ffs(m) - 1;
    const int64_t e = tid + (int64_t)q * nth;
    const int64_t i = a.idx[e];
    if (__ldcg(tags + i) == (uint32_t)(e + 1)) {
      tags[i] = 0u;
      leaves[i] = powf(fabsf(a.td[e]) + t.eps, t.alpha);
      atomicMax(t.claims[1] + (i >> PER_LOG_FANOUT), (uint32_t)(e + 1));
      next |= 1u << q;
    }
  }
  active = next;

  // P2..: owners recompute their node from its 32 children, then claim the parent
  for (int L = 1; L < t.num_levels; ++L) {
    bar.sync(t.status);
    next = 0u;
    uint32_t* cl = t.claims[L];
    for (uint32_t m = active; m; m &= m - 1) {
      const int q = __ffs(m) - 1;
      const int64_t e = tid + (int64_t)q * nth;
      const int64_t node = a.idx[e] >> (PER_LOG_FANOUT * L);
      if (__ldcg(cl + node) == (uint32_t)(e + 1)) {
        cl[node] = 0u;
        t.levels[L][node] = __double2float_rn(per_sum32(t.levels[L - 1], node));
        if (L + 1 < t.num_levels)
          atomicMax(t.claims[L + 1] + (node >> PER_LOG_FANOUT), (uint32_t)(e + 1));
        next |= 1u << q;
      }
    }
    active = next;
  }
}

struct AddArgs {
  PerTree t;
  per_field_t fields[PER_MAX_FIELDS];
  int32_t n_fields;
  int64_t n;
};

__global__ void __launch_bounds__(kThreads) per_add_kernel(AddArgs a) {
  const PerTree& t = a.t;
  PerGridBarrier bar;
  bar.init(t.scratch);
  const int64_t C = t.capacity;
  const int64_t size = t.size_cursor[0];
  const int64_t cursor = t.size_cursor[1];
  const float maxp = *t.max_priority;
  const int64_t n0 = a.n > C ? a.n - C : 0;  // earlier rows would be overwritten in this call
  const int64_t m = a.n - n0;
  const int64_t start = (cursor + n0) % C;

  // P0: rows and leaves (one warp per row)
  {
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
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
  }

  // touched leaf ranges: [start, start+m) on the ring, split at C
  const int64_t a0 = start, a1 = min(start + m, C);
  const int64_t b0 = 0, b1 = start + m > C ? start + m - C : 0;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int L = 1; L < t.num_levels; ++L) {
    bar.sync(t.status);
    const int sh = PER_LOG_FANOUT * L;
    const int64_t lo0 = a0 >> sh, hi0 = (a1 - 1) >> sh;
    const int64_t cnt0 = a1 > a0 ? hi0 - lo0 + 1 : 0;
    const int64_t lo1 = b0 >> sh, hi1 = b1 > b0 ? (b1 - 1) >> sh : -1;
    const int64_t cnt1 = b1 > b0 ? hi1 - lo1 + 1 : 0;
    for (int64_t k = tid; k < cnt0 + cnt1; k += nth) {
      const int64_t node = k < cnt0 ? lo0 + k : lo1 + (k - cnt0);
      t.levels[L][node] = __double2float_rn(per_sum32(t.levels[L - 1], node));
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    t.size_cursor[1] = (cursor + a.n) % C;
    t.size_cursor[0] = min(size + a.n, C);
  }
}

__global__ void __launch_bounds__(kThreads) per_rebuild_kernel(PerTree t) {
  PerGridBarrier bar;
  bar.init(t.scratch);
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int L = 0; L < t.num_levels; ++L)
    for (int64_t k = tid; k < t.level_len[L]; k += nth) t.claims[L][k] = 0u;
  for (int L = 1; L < t.num_levels; ++L) {
    bar.sync(t.status);
    const int64_t nodes = live_nodes(t.capacity, L);
    for (int64_t k = tid; k < nodes; k += nth)
      t.levels[L][k] = __double2float_rn(per_sum32(t.levels[L - 1], k));
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
  UpdateArgs a;
  a.t = t;
  a.idx = idx;
  a.td = td;
  a.n = n;
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
