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
// Design:
//   * Prologue: each CTA stages the float64 exclusive prefix of the top tree
//     level (<= PER_TOP_MAX float32 nodes) in shared memory.
//   * Search: a warp owns DPW draws at a time. The top level is searched
//     32-ary with ballots over shared memory; every lower level is one
//     coalesced 128-byte warp load of the 32 children, a float64 warp scan
//     and a ballot. The loads of the DPW draws are issued back to back so
//     their L2 latencies overlap.
//   * Arrive: the CTA publishes the max of its unnormalised weights and
//     arrives at a grid barrier, then gathers its rows (the HBM-bound part)
//     while the other CTAs finish, then waits, reads the global max and
//     normalises its weights.
// Sampling semantics: idx is the first slot whose inclusive prefix exceeds
// u = rand * total (fp32 product, as torch computes it), with prefixes in
// float64 so the result equals a search over exact prefixes; rounding
// fallbacks and empty-slot walk-backs are counted in the status words.
#include <cuda_runtime.h>
#include <stdint.h>

#include "per_internal.h"

namespace {

constexpr int kSampleThreads = 256;
constexpr int kDPW = 4;           // draws per warp in flight
constexpr int kSegVec = 64;       // vectors per gather segment (2 per lane)
constexpr int kGatherUnroll = 4;  // segments per warp in flight

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

struct SampleArgs {
  PerTree t;
  const float* rand;
  int64_t batch;
  float beta;
  float* out;
  int64_t out_stride;
  int64_t* idx;
  float* w;
  int64_t draws_per_cta;
  int32_t nvec;  // vectors per row
  int32_t nseg;  // gather segments per row
};

// First k in [0, n) with pre[k + 1] > t (upper bound over the inclusive
// prefixes), or n if none. Warp-cooperative, 32-ary; pre is in shared memory.
__device__ __forceinline__ int top_upper_bound(const double* pre, int n, double t, int lane) {
  int lo = 0, len = n;
  while (len > 32) {
    const int step = (len + 31) >> 5;
    const int q = lo + min((lane + 1) * step, len) - 1;
    const uint32_t m = __ballot_sync(PER_FULL_MASK, pre[q + 1] > t);
    if (!m) return lo + len;
    const int f = __ffs(m) - 1;
    lo += f * step;
    len = min(step, len - f * step);
  }
  const uint32_t m = __ballot_sync(PER_FULL_MASK, lane < len && pre[lo + lane + 1] > t);
  return m ? lo + __ffs(m) - 1 : lo + len;
}

// First k in [0, n) with pre[k + 1] >= t, or n if none.
__device__ __forceinline__ int top_lower_bound(const double* pre, int n, double t, int lane) {
  int lo = 0, len = n;
  while (len > 32) {
    const int step = (len + 31) >> 5;
    const int q = lo + min((lane + 1) * step, len) - 1;
    const uint32_t m = __ballot_sync(PER_FULL_MASK, pre[q + 1] >= t);
    if (!m) return lo + len;
    const int f = __ffs(m) - 1;
    lo += f * step;
    len = min(step, len - f * step);
  }
  const uint32_t m = __ballot_sync(PER_FULL_MASK, lane < len && pre[lo + lane + 1] >= t);
  return m ? lo + __ffs(m) - 1 : lo + len;
}

template <int VEC>
__global__ void __launch_bounds__(kSampleThreads) per_sample_kernel(SampleArgs a) {
  extern __shared__ double s_pre[];  // [n_top + 1]
  __shared__ double s_wsum[32];
  __shared__ uint32_t s_max_bits;
  __shared__ int s_last;
  __shared__ float s_gmax;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const PerTree& t = a.t;

  PerGridBarrier bar;
  bar.init(t.scratch);

  const int64_t size = t.size_cursor[0];
  if (size <= 0) {  // host checks first; keep the device consistent anyway
    if (blockIdx.x == 0 && threadIdx.x == 0) per_flag(t.status, PER_EVT_EMPTY_BUFFER);
    return;
  }

  // ---- prologue: float64 exclusive prefix of the top level in shared memory
  const int top = t.top_level;
  const float* topv = t.levels[top];
  const int n_top = (int)t.level_len[top];
  {
    const int per = (n_top + blockDim.x - 1) / blockDim.x;
    const int beg = threadIdx.x * per;
    double loc = 0.0;
    for (int i = 0; i < per; ++i) {
      const int q = beg + i;
      if (q < n_top) loc += (double)__ldg(topv + q);
    }
    const double incl = per_warp_scan_incl(loc, lane);
    if (lane == 31) s_wsum[warp] = incl;
    if (threadIdx.x == 0) s_max_bits = 0u;
    __syncthreads();
    if (warp == 0) {
      const double x = lane < nwarps ? s_wsum[lane] : 0.0;
      const double xi = per_warp_scan_incl(x, lane);
      __syncwarp();
      s_wsum[lane] = xi - x;  // exclusive prefix of warp totals
    }
    __syncthreads();
    double run = s_wsum[warp] + (incl - loc);
    for (int i = 0; i < per; ++i) {
      const int q = beg + i;
      if (q < n_top) {
        s_pre[q] = run;
        run += (double)__ldg(topv + q);
        if (q == n_top - 1) s_pre[n_top] = run;
      }
    }
    __syncthreads();
  }
  const double total64 = s_pre[n_top];
  const float total = __double2float_rn(total64);
  const float sizef = (float)size;

  // ---- search: DPW draws per warp at a time
  const int64_t s0 = (int64_t)blockIdx.x * a.draws_per_cta;
  const int64_t e0 = min(s0 + a.draws_per_cta, a.batch);
  uint32_t local_max = 0u;
  uint32_t n_fallback = 0, n_clamp = 0, n_zero = 0;
  const float* leaves = t.levels[0];

  for (int64_t g = s0 + (int64_t)warp * kDPW; g < e0; g += (int64_t)nwarps * kDPW) {
    int64_t node[kDPW];
    double r[kDPW];
    bool ok[kDPW], fb[kDPW];
    float pv[kDPW];
#pragma unroll
    for (int d = 0; d < kDPW; ++d) {
      const int64_t j = g + d;
      ok[d] = j < e0;
      fb[d] = false;
      pv[d] = 0.f;
      const float u = __fmul_rn(ok[d] ? __ldg(a.rand + j) : 0.f, total);
      const double tu = (double)u;
      int k = top_upper_bound(s_pre, n_top, tu, lane);
      if (k >= n_top) {  // u >= total: fall back to the last node with mass
        k = top_lower_bound(s_pre, n_top, total64, lane);
        if (k >= n_top) k = n_top - 1;
        fb[d] = true;
      }
      node[d] = k;
      r[d] = tu - s_pre[k];
    }
    for (int L = top - 1; L >= 0; --L) {
      const float* lv = t.levels[L];
      float v[kDPW];
#pragma unroll
      for (int d = 0; d < kDPW; ++d) v[d] = ok[d] ? __ldg(lv + node[d] * PER_FANOUT + lane) : 0.f;
#pragma unroll
      for (int d = 0; d < kDPW; ++d) {
        const double sc = per_warp_scan_incl((double)v[d], lane);
        const uint32_t m = __ballot_sync(PER_FULL_MASK, sc > r[d]);
        int f;
        if (m) {
          f = __ffs(m) - 1;
        } else {  // rounding: residual at or past this node's sum
          const uint32_t mp = __ballot_sync(PER_FULL_MASK, v[d] > 0.f);
          f = mp ? 31 - __clz(mp) : 0;
          fb[d] = true;
        }
        double ex = __shfl_sync(PER_FULL_MASK, sc, f > 0 ? f - 1 : 0);
        if (f == 0) ex = 0.0;
        r[d] -= ex;
        node[d] = node[d] * PER_FANOUT + f;
        if (L == 0) pv[d] = __shfl_sync(PER_FULL_MASK, v[d], f);
      }
    }
#pragma unroll
    for (int d = 0; d < kDPW; ++d) {
      if (!ok[d]) continue;  // warp-uniform
      int64_t i = node[d];
      float p = pv[d];
      if (i > size - 1 || total64 <= 0.0) {  // sampling.py:49-51 clamp; p reloaded there
        i = size - 1;
        p = __ldg(leaves + i);
        ++n_clamp;
      }
      if (!(p > 0.f)) {  // never hand out an empty slot: walk back to the last positive one
        int64_t c = i >> PER_LOG_FANOUT;
        for (int it = 0; it < 64 && c >= 0; ++it, --c) {
          const int64_t q = c * PER_FANOUT + lane;
          const float vq = q <= i ? __ldg(leaves + q) : 0.f;
          const uint32_t mp = __ballot_sync(PER_FULL_MASK, vq > 0.f);
          if (mp) {
            const int f = 31 - __clz(mp);
            i = c * PER_FANOUT + f;
            p = __shfl_sync(PER_FULL_MASK, vq, f);
            break;
          }
        }
        ++n_zero;
      }
      n_fallback += fb[d] ? 1u : 0u;
      const float prob = __fdiv_rn(p, total);
      const float wv = powf(__fmul_rn(sizef, prob), -a.beta);
      local_max = max(local_max, __float_as_uint(wv));
      if (lane == d) {
        a.idx[g + d] = i;
        a.w[g + d] = wv;
      }
    }
  }
  if (lane == 0) {
    atomicMax(&s_max_bits, local_max);
    if (n_fallback) per_count(t.status, PER_STATUS_FALLBACKS, n_fallback);
    if (n_clamp) per_count(t.status, PER_STATUS_CLAMPS, n_clamp);
    if (n_zero) per_count(t.status, PER_STATUS_ZERO_WALKS, n_zero);
  }
  __syncthreads();

  // ---- arrive: publish this CTA's max weight
  const bool multi = gridDim.x > 1;
  if (multi) {
    if (threadIdx.x == 0) {
      t.scratch->partial[blockIdx.x] = __uint_as_float(s_max_bits);
      s_last = bar.arrive_thread0() ? 1 : 0;
    }
    __syncthreads();
    if (s_last) {  // last CTA: reduce the partial maxima and release the grid
      __threadfence();
      uint32_t m = 0u;
      for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x)
        m = max(m, __float_as_uint(__ldcg(&t.scratch->partial[i])));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(PER_FULL_MASK, m, o));
      if (lane == 0) atomicMax(&s_max_bits, m);
      __syncthreads();
      if (threadIdx.x == 0) {
        t.scratch->gmax = __uint_as_float(s_max_bits);
        bar.release_thread0();
      }
    }
  }

  // ---- gather rows storage[idx[j]] -> out[j] (idx written above by this CTA)
  {
    using V = typename VecT<VEC>::T;
    const int64_t nrows = e0 - s0;
    const int64_t nitems = nrows * a.nseg;
    const V* src_base = reinterpret_cast<const V*>(t.storage);
    V* dst_base = reinterpret_cast<V*>(a.out);
    const int64_t src_stride = t.row_stride / VEC;
    const int64_t dst_stride = a.out_stride / VEC;
    for (int64_t base = (int64_t)warp * kGatherUnroll; base < nitems;
         base += (int64_t)nwarps * kGatherUnroll) {
      V buf[kGatherUnroll][2];
      const V* src[kGatherUnroll];
      V* dst[kGatherUnroll];
      int nv[kGatherUnroll];
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        const int64_t it = base + u;
        nv[u] = 0;
        if (it < nitems) {
          const int64_t row = it / a.nseg;
          const int sg = (int)(it - row * a.nseg);
          const int64_t j = s0 + row;
          const int64_t sidx = a.idx[j];
          src[u] = src_base + sidx * src_stride + (int64_t)sg * kSegVec;
          dst[u] = dst_base + j * dst_stride + (int64_t)sg * kSegVec;
          nv[u] = min(kSegVec, a.nvec - sg * kSegVec);
        }
      }
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        if (lane < nv[u]) buf[u][0] = __ldcs(src[u] + lane);
        if (lane + 32 < nv[u]) buf[u][1] = __ldcs(src[u] + lane + 32);
      }
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        if (lane < nv[u]) dst[u][lane] = buf[u][0];
        if (lane + 32 < nv[u]) dst[u][lane + 32] = buf[u][1];
      }
    }
  }

  // ---- wait for the global max, then normalise this CTA's weights
  if (threadIdx.x == 0) {
    if (multi) {
      bar.wait_thread0(t.status);
      s_gmax = per_ld_relaxed_f32(&t.scratch->gmax);
    } else {
      s_gmax = __uint_as_float(s_max_bits);
    }
  }
  __syncthreads();
  const float gmax = s_gmax;
  for (int64_t j = s0 + threadIdx.x; j < e0; j += blockDim.x) a.w[j] = __fdiv_rn(a.w[j], gmax);
}

template <int VEC>
int launch_vec(const SampleArgs& a0, cudaStream_t stream) {
  SampleArgs a = a0;
  const void* fn = (const void*)per_sample_kernel<VEC>;
  const size_t smem = (size_t)(a.t.level_len[a.t.top_level] + 1) * sizeof(double);
  int max_ctas = 0;
  int rc = per_coresident_ctas(fn, kSampleThreads, smem, &max_ctas);
  if (rc) return rc;
  if (max_ctas > PER_MAX_GRID) max_ctas = PER_MAX_GRID;
  const int64_t per_cta_min = (int64_t)(kSampleThreads / 32) * kDPW;
  int64_t grid = (a.batch + per_cta_min - 1) / per_cta_min;
  if (grid > max_ctas) grid = max_ctas;
  if (grid < 1) grid = 1;
  a.draws_per_cta = (a.batch + grid - 1) / grid;
  grid = (a.batch + a.draws_per_cta - 1) / a.draws_per_cta;
  void* args[] = {&a};
  cudaError_t e = per_launch(fn, (unsigned)grid, kSampleThreads, smem, stream, args, grid > 1);
  return e == cudaSuccess ? PER_OK : per_record_cuda(e);
}

}  // namespace

int per_launch_sample(const PerTree& t, const float* rand, int64_t batch, float beta, float* out,
                      int64_t out_stride, int64_t* idx, float* w, cudaStream_t stream) {
  SampleArgs a;
  a.t = t;
  a.rand = rand;
  a.batch = batch;
  a.beta = beta;
  a.out = out;
  a.out_stride = out_stride;
  a.idx = idx;
  a.w = w;
  a.draws_per_cta = 0;
  // widest vector that every row start and both bases allow
  const uintptr_t al = (uintptr_t)t.storage | (uintptr_t)out |
                       (uintptr_t)(t.row_stride * 4) | (uintptr_t)(out_stride * 4);
  const int vec = (al % 16 == 0 && t.row_dim % 4 == 0) ? 4 : (al % 8 == 0 && t.row_dim % 2 == 0) ? 2 : 1;
  a.nvec = (int32_t)(t.row_dim / vec);
  a.nseg = (a.nvec + kSegVec - 1) / kSegVec;
  if (vec == 4) return launch_vec<4>(a, stream);
  if (vec == 2) return launch_vec<2>(a, stream);
  return launch_vec<1>(a, stream);
}
