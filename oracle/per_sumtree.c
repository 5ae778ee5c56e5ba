/*
 * per_sumtree.c - TEST INFRASTRUCTURE ONLY (CPU baseline).
 *
 * C restatement of triton-per's classic CPU sum tree, the baseline the
 * reference benchmarks its kernels against
 * (src/triton_per/baselines/cpu_sumtree.py; bench/bench_sampling.py:23-36
 * "cpu-sumtree", bench/profile_utd.py's default backend). The benchmark times
 * it on the host cores beside the engine; the tests pin it to vectors that the
 * reference's own Python SumTree produced. Nothing in the engine links it.
 *
 * Followed step by step (reference paths within its project):
 *   cpu_sumtree.py:11-14   float64 array tree[2 * capacity], leaf i at
 *                          tree[capacity + i], node k = tree[2k] + tree[2k+1]
 *                          (an implicit binary heap; capacity need not be a
 *                          power of two)
 *   cpu_sumtree.py:19-24   update: delta = p - leaf, added to the leaf and
 *                          every ancestor (so the sums drift like the
 *                          reference's)
 *   cpu_sumtree.py:26-35   find: from the root, go left while u <= left sum,
 *                          else subtract it and go right
 *   cpu_sumtree.py:64-73   add: each new slot's leaf set to the running max
 *                          priority by update(), rows written at the cursor
 *   cpu_sumtree.py:75-89   sample: u = random * total (float64), idx =
 *                          min(find(u), size - 1), prob = leaf / total,
 *                          w = (size * prob)^-beta, w / max(w) as float32
 *   cpu_sumtree.py:91-97   update_priorities: p = (|td| + eps)^alpha per
 *                          index in order (duplicates: last one wins), max
 *                          priority tracked
 * One draw and one index at a time, as the reference's host loops do; all
 * arithmetic in double like numpy / Python floats. Compiled without
 * fast-math and without FP contraction.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* cpu_sumtree.py:19-24 */
void sumtree_update(double* tree, int64_t capacity, int64_t idx, double p) {
  int64_t i = idx + capacity;
  const double delta = p - tree[i];
  while (i >= 1) {
    tree[i] += delta;
    i /= 2;
  }
}

/* cpu_sumtree.py:26-35 */
int64_t sumtree_find(const double* tree, int64_t capacity, double u) {
  int64_t i = 1;
  while (i < capacity) {
    const int64_t left = 2 * i;
    if (u <= tree[left]) {
      i = left;
    } else {
      u -= tree[left];
      i = left + 1;
    }
  }
  return i - capacity;
}

/* Set-up only (not in the reference, which fills by repeated update()):
 * tree[capacity + i] = leaves[i], every inner node the sum of its children. */
void sumtree_build(double* tree, int64_t capacity, const double* leaves) {
  tree[0] = 0.0;
  memcpy(tree + capacity, leaves, (size_t)capacity * sizeof(double));
  for (int64_t k = capacity - 1; k >= 1; --k) tree[k] = tree[2 * k] + tree[2 * k + 1];
}

/* cpu_sumtree.py:75-89 with the uniforms given (np.random.random(n) there):
 * idx[j], w[j] (float32, normalised by the batch max). */
void sumtree_sample(const double* tree, int64_t capacity, int64_t size, const double* rand,
                    int64_t n, double beta, int64_t* idx, float* w, double* work) {
  const double total = tree[1];
  double wmax = 0.0;
  for (int64_t j = 0; j < n; ++j) {
    const double u = rand[j] * total;
    int64_t i = sumtree_find(tree, capacity, u);
    if (i > size - 1) i = size - 1;
    idx[j] = i;
    const double prob = tree[i + capacity] / total;
    const double wj = pow((double)size * prob, -beta);
    work[j] = wj;
    if (j == 0 || wj > wmax) wmax = wj;
  }
  for (int64_t j = 0; j < n; ++j) w[j] = (float)(work[j] / wmax);
}

/* cpu_sumtree.py:91-97: td are the float32 TD errors (|td| taken here). */
void sumtree_update_priorities(double* tree, int64_t capacity, const int64_t* idx,
                               const float* td, int64_t n, double alpha, double eps,
                               double* max_priority) {
  double mp = *max_priority;
  for (int64_t k = 0; k < n; ++k) {
    const double p = pow(fabs((double)td[k]) + eps, alpha);
    sumtree_update(tree, capacity, idx[k], p);
    if (p > mp) mp = p;
  }
  *max_priority = mp;
}

/* cpu_sumtree.py:64-73: n rows of row_dim floats at the ring cursor;
 * cursor_size = {cursor, size}, advanced here. */
void sumtree_add(double* tree, int64_t capacity, float* storage, int64_t row_dim,
                 const float* rows, int64_t n, double max_priority, int64_t* cursor_size) {
  const int64_t cursor = cursor_size[0];
  for (int64_t k = 0; k < n; ++k) sumtree_update(tree, capacity, (cursor + k) % capacity, max_priority);
  for (int64_t k = 0; k < n; ++k) {
    const int64_t i = (cursor + k) % capacity;
    memcpy(storage + i * row_dim, rows + k * row_dim, (size_t)row_dim * sizeof(float));
  }
  cursor_size[0] = (cursor + n) % capacity;
  cursor_size[1] = cursor_size[1] + n < capacity ? cursor_size[1] + n : capacity;
}

/* The rows of a sample (the reference gathers self.storage[idx]). */
void sumtree_gather(const float* storage, int64_t row_dim, const int64_t* idx, int64_t n,
                    float* out) {
  for (int64_t j = 0; j < n; ++j)
    memcpy(out + j * row_dim, storage + idx[j] * row_dim, (size_t)row_dim * sizeof(float));
}
