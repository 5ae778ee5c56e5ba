/*
 * per_oracle.c - TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of triton-per's `torch` backend, the reference semantics of
 * the replay hot path. The tests compare the CUDA engine against it and the
 * benchmark times it as the CPU baseline; nothing in the engine links or
 * calls it.
 *
 * Followed line by line (reference paths within its project):
 *   src/triton_per/buffer.py:96-105   _sample_torch: full-length cumsum,
 *                                     searchsorted(right=True), clamp to size-1,
 *                                     prob = p/total, w = (size*prob)^-beta
 *   src/triton_per/buffer.py:92       w / w.max()
 *   src/triton_per/buffer.py:133-145  update_priorities (torch backend):
 *                                     |td|, max-priority, leaf assign, touched
 *                                     block sums recomputed
 *   src/triton_per/buffer.py:66-79    add: ring write, leaves = max priority,
 *                                     touched block sums recomputed
 *
 * Arithmetic matches torch on CPU:
 *   - torch.cumsum on float32 accumulates sequentially in double and stores
 *     float32 (verified bit-for-bit against torch 2.11 on 1e6 elements);
 *   - products and quotients are float32 with round-to-nearest;
 *   - powf stands in for torch's float pow (results agree to 1 ulp);
 *   - duplicate indices in an assignment keep the last occurrence;
 *   - block sums are the float32 rounding of the double sum of the block
 *     (torch's own float32 reduction agrees within a few ulp).
 * Compiled without fast-math and without FP contraction.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_BLOCK_P 1024

/* buffer.py:98 csum = torch.cumsum(p) over p[0:capacity]. nthreads > 1
 * splits the scan into double-precision blocks (same values except on
 * double-rounding ties, for the timed baseline). */
void oracle_cumsum(const float* p, int64_t n, float* csum, int nthreads) {
  if (nthreads <= 1 || n < 65536) {
    double acc = 0.0;
    for (int64_t i = 0; i < n; ++i) {
      acc += (double)p[i];
      csum[i] = (float)acc;
    }
    return;
  }
#ifdef _OPENMP
  double* part = (double*)calloc((size_t)nthreads + 1, sizeof(double));
#pragma omp parallel num_threads(nthreads)
  {
    const int t = omp_get_thread_num();
    const int nt = omp_get_num_threads();
    const int64_t lo = n * t / nt, hi = n * (t + 1) / nt;
    double acc = 0.0;
    for (int64_t i = lo; i < hi; ++i) acc += (double)p[i];
    part[t + 1] = acc;
#pragma omp barrier
#pragma omp single
    for (int k = 1; k <= nt; ++k) part[k] += part[k - 1];
    acc = part[t];
    for (int64_t i = lo; i < hi; ++i) {
      acc += (double)p[i];
      csum[i] = (float)acc;
    }
  }
  free(part);
#else
  oracle_cumsum(p, n, csum, 1);
#endif
}

/* First i with csum[i] > u (torch.searchsorted(..., right=True)). */
static int64_t upper_bound_f32(const float* csum, int64_t n, float u) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = lo + (hi - lo) / 2;
    if (csum[mid] <= u)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

/* buffer.py:96-105 + :92 on a given cumsum. w_unnorm may be NULL. */
void oracle_sample_from_csum(const float* priorities, const float* csum, int64_t capacity,
                             int64_t size, const float* rand, int64_t batch, float beta,
                             int64_t* idx, float* w, float* w_unnorm, int nthreads) {
  const float total = csum[capacity - 1];
  const float sizef = (float)size;
  float wmax = -INFINITY;
  int any_nan = 0;
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) reduction(max : wmax) reduction(| : any_nan) schedule(static)
  for (int64_t j = 0; j < batch; ++j) {
    const float u = rand[j] * total;
    int64_t i = upper_bound_f32(csum, capacity, u);
    if (i > size - 1) i = size - 1;
    idx[j] = i;
    const float prob = priorities[i] / total;
    const float x = sizef * prob;
    const float wj = powf(x, -beta);
    w[j] = wj;
    if (wj != wj)
      any_nan = 1;
    else if (wj > wmax)
      wmax = wj;
  }
  if (any_nan) wmax = NAN; /* torch max propagates NaN */
  for (int64_t j = 0; j < batch; ++j) {
    if (w_unnorm) w_unnorm[j] = w[j];
    w[j] = w[j] / wmax;
  }
}

/* Full sample path. csum_out (length capacity) may be NULL. */
void oracle_sample(const float* priorities, int64_t capacity, int64_t size, const float* rand,
                   int64_t batch, float beta, int64_t* idx, float* w, float* csum_out,
                   int nthreads) {
  float* csum = csum_out ? csum_out : (float*)malloc((size_t)capacity * sizeof(float));
  oracle_cumsum(priorities, capacity, csum, nthreads);
  oracle_sample_from_csum(priorities, csum, capacity, size, rand, batch, beta, idx, w, NULL,
                          nthreads);
  if (!csum_out) free(csum);
}

/* IS weights of buffer.py:102-103 + :92 for GIVEN indices (used to check the
 * weights of a sample whose indices differ from the oracle's at ties). */
void oracle_weights_for(const float* priorities, float total, int64_t size, const int64_t* idx,
                        int64_t batch, float beta, float* w) {
  const float sizef = (float)size;
  float wmax = -INFINITY;
  for (int64_t j = 0; j < batch; ++j) {
    const float prob = priorities[idx[j]] / total;
    w[j] = powf(sizef * prob, -beta);
    if (w[j] > wmax) wmax = w[j];
  }
  for (int64_t j = 0; j < batch; ++j) w[j] = w[j] / wmax;
}

/* Block sums of the whole leaf array: float32 rounding of double sums. */
void oracle_block_sums(const float* priorities, int64_t num_blocks, float* block_sums) {
  for (int64_t b = 0; b < num_blocks; ++b) {
    double s = 0.0;
    for (int64_t k = 0; k < ORACLE_BLOCK_P; ++k) s += (double)priorities[b * ORACLE_BLOCK_P + k];
    block_sums[b] = (float)s;
  }
}

static void recompute_block(const float* priorities, float* block_sums, int64_t b) {
  double s = 0.0;
  for (int64_t k = 0; k < ORACLE_BLOCK_P; ++k) s += (double)priorities[b * ORACLE_BLOCK_P + k];
  block_sums[b] = (float)s;
}

/* buffer.py:133-145 (torch backend). Indices must be in [0, capacity). */
void oracle_update(float* priorities, float* block_sums, int64_t num_blocks, const int64_t* idx,
                   const float* td, int64_t n, float alpha, float eps, float* max_priority) {
  float tmax = -INFINITY;
  int any_nan = 0;
  for (int64_t e = 0; e < n; ++e) {
    const float a = fabsf(td[e]);
    if (a != a)
      any_nan = 1;
    else if (a > tmax)
      tmax = a;
  }
  if (any_nan) tmax = NAN; /* td.max() propagates NaN */
  const float cand = powf(tmax + eps, alpha);
  if (cand != cand || *max_priority != *max_priority)
    *max_priority = NAN;
  else if (cand > *max_priority)
    *max_priority = cand;
  unsigned char* touched = (unsigned char*)calloc((size_t)num_blocks, 1);
  for (int64_t e = 0; e < n; ++e) { /* sequential: the last occurrence wins */
    const int64_t i = idx[e];
    priorities[i] = powf(fabsf(td[e]) + eps, alpha);
    touched[i / ORACLE_BLOCK_P] = 1;
  }
  for (int64_t b = 0; b < num_blocks; ++b)
    if (touched[b]) recompute_block(priorities, block_sums, b);
  free(touched);
}

/* buffer.py:66-79. rows: float32[n, row_dim] packed; storage float32[capacity, row_dim].
 * cursor_size: int64[2] = {cursor, size}, updated in place. */
void oracle_add(float* storage, int64_t row_dim, float* priorities, float* block_sums,
                int64_t capacity, int64_t num_blocks, const float* rows, int64_t n,
                float max_priority, int64_t* cursor_size) {
  const int64_t cursor = cursor_size[0];
  unsigned char* touched = (unsigned char*)calloc((size_t)num_blocks, 1);
  for (int64_t k = 0; k < n; ++k) {
    const int64_t i = (k + cursor) % capacity;
    memcpy(storage + i * row_dim, rows + k * row_dim, (size_t)row_dim * sizeof(float));
    priorities[i] = max_priority;
    touched[i / ORACLE_BLOCK_P] = 1;
  }
  for (int64_t b = 0; b < num_blocks; ++b)
    if (touched[b]) recompute_block(priorities, block_sums, b);
  free(touched);
  cursor_size[0] = (cursor + n) % capacity;
  cursor_size[1] = cursor_size[1] + n < capacity ? cursor_size[1] + n : capacity;
}
