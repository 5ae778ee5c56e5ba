// Small kernels of the sharded mode: shard statistics for the totals
// exchange, and the normalisation of a shard's weights by the max over all
// shards.
//
// Sharded sampling (no counterpart in the reference, which has no
// multi-GPU code): shard g owns global slots [g*C, (g+1)*C). Every shard
// draws the same global uniforms; u = rand * total over all shards, and a
// draw belongs to the shard whose range of the global prefix holds u, so the
// union of the shards' draws is exactly the draw of one buffer holding all
// slots. Each shard needs every shard's total and size (the stats exchanged
// between calls) and, to normalise, the max weight over all shards.
#include <cuda_runtime.h>
#include <stdint.h>

#include "per_internal.h"

namespace {

constexpr int kThreads = 256;

// out[0] = total priority of the store (float64 sum of its top-level nodes),
// out[1] = live size.
__global__ void __launch_bounds__(kThreads) per_shard_stats_kernel(PerTree t, double* out) {
  per_wait_previous_grid();
  __shared__ double s_part[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* topv = t.levels[t.top_level];
  const int n = (int)t.level_len[t.top_level];
  const int per = (n + kThreads - 1) / kThreads;
  const int beg = min((int)threadIdx.x * per, n), end = min(beg + per, n);
  double s = 0.0;
  for (int i = beg; i < end; ++i) s += (double)__ldg(topv + i);
  s = per_warp_sum(s);
  if (lane == 0) s_part[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) tot += s_part[w];
    out[0] = tot;
    out[1] = (double)__ldg(t.size_cursor);
  }
}

__global__ void per_normalize_kernel(float* w, const int64_t* count, const float* gmax,
                                     int64_t cap) {
  per_wait_previous_grid();
  const int64_t n = min(*count, cap);
  const float m = *gmax;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x)
    w[j] = __fdiv_rn(w[j], m);
}

}  // namespace

int per_launch_shard_stats(const PerTree& t, double* out, cudaStream_t stream) {
  PerTree a = t;
  void* args[] = {&a, &out};
  cudaError_t e = per_launch((const void*)per_shard_stats_kernel, 1, kThreads, 0, stream, args,
                             false);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}

int per_launch_normalize(float* w, const int64_t* count, const float* gmax, int64_t cap,
                         cudaStream_t stream) {
  int64_t grid = (cap + kThreads - 1) / kThreads;
  if (grid > 1184) grid = 1184;
  if (grid < 1) grid = 1;
  void* args[] = {&w, &count, &gmax, &cap};
  cudaError_t e = per_launch((const void*)per_normalize_kernel, (unsigned)grid, kThreads, 0,
                             stream, args, false);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}
