// Host-side helpers shared by the launchers and the C entry points.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "per_common.cuh"

// Record a CUDA error for per_last_cuda_error() and return PER_ERR_CUDA.
int per_record_cuda(cudaError_t e);

// The kernels' view of a store descriptor (16-bit rows as 4-byte words).
PerTree per_tree_of(const per_store_t* s);

// PER_OK if the descriptor is self-consistent with per_layout(); with
// with_scratch false, claims[] and scratch are not required (the caller
// supplies its own).
int per_check_store(const per_store_t* s, bool with_scratch);

// Largest grid of `fn` (threads per CTA, dynamic shared bytes) whose CTAs are
// all co-resident on the current device; cached per (device, fn, smem).
int per_coresident_ctas(const void* fn, int threads, size_t smem, int* out);

// Allow `fn` to use up to `smem` bytes of dynamic shared memory on the
// current device (needed whenever static + dynamic exceeds 48 KB); cached per
// (device, fn).
int per_set_smem(const void* fn, size_t smem);

// Launch `fn`. With grid_sync the CTAs wait on one another through
// PerGridBarrier, so the grid must not exceed per_coresident_ctas(); the
// launch then asks for co-scheduling (cooperative attribute) unless the
// stream is being captured into a graph.
cudaError_t per_launch(const void* fn, unsigned grid, unsigned threads, size_t smem,
                       cudaStream_t stream, void** args, bool grid_sync);

// In-kernel uniforms: Philox4x32-10 stream `seed`, position in *counter
// (device), advanced by the kernel by the batch size.
struct PerRng {
  unsigned long long seed;
  unsigned long long* counter;
};

// rng == nullptr: uniforms from `rand`
int per_launch_sample(const PerTree& t, const float* rand, const PerRng* rng, int64_t batch,
                      float beta, float* out, int64_t out_stride, int64_t* idx, float* w,
                      cudaStream_t stream);
int per_launch_update(const PerTree& t, const int64_t* idx, const float* td, int64_t n,
                      cudaStream_t stream);
// True when per_launch_update() of n entries takes the grid path (claim words
// and grid-barrier scratch); false for the partitioned path, which uses neither.
bool per_update_uses_grid(const PerTree& t, int64_t n);
// Update with global indices: slot = idx - base; indices outside the store
// are errors when strict, else skipped and counted as another shard's.
int per_launch_update_shard(const PerTree& t, int64_t base, int32_t strict, const int64_t* idx,
                            const float* td, int64_t n, const int64_t* count, cudaStream_t stream);
int per_launch_sample_sharded(const PerTree& t, int32_t rank, int32_t world, int64_t shard_base,
                              const double* stats, const float* rand, const PerRng* rng,
                              int64_t batch, float beta, float* out, int64_t out_stride,
                              int64_t* idx, float* w, int32_t* pos, int64_t* count,
                              float* local_max, cudaStream_t stream);
int per_launch_add(const PerTree& t, const per_field_t* fields, int32_t n_fields, int64_t n,
                   cudaStream_t stream);
int per_launch_rebuild(const PerTree& t, cudaStream_t stream);
int per_launch_shard_stats(const PerTree& t, double* out, cudaStream_t stream);
int per_launch_sample_p2p_max_batch(const PerTree& t, int64_t* max_batch);
int per_launch_sample_sharded_p2p(const PerTree& t, int32_t rank, int32_t world,
                                  int64_t shard_base, PerMailbox* const* mailboxes,
                                  const float* rand, const PerRng* rng, int64_t batch, float beta,
                                  float* out, int64_t out_stride, int64_t* idx, float* w,
                                  int32_t* pos, int64_t* count, int32_t local_norm,
                                  cudaStream_t stream);
int per_launch_normalize(float* w, const int64_t* count, const float* gmax, int64_t cap,
                         cudaStream_t stream);
