// Per-member metric reductions and greedy ensemble selection.
//
// Metrics follow src/tabpackage/metrics.py: element terms are computed in fp32 exactly
// as the reference's elementwise ops do, and summed in fp64 (one block per member,
// warp shuffles + shared memory), so a member's value is its exact mean up to the
// final fp32 rounding.
//
// Greedy selection follows src/tabpackage/ensemble.py:95-263 on the device: each
// iteration scores every candidate's would-be ensemble lerp(pred_c, ens, w/(w+1))
// without materialising it, picks the best (ties: higher individual score, then lower
// index), stops when no candidate improves, and updates the ensemble in place.
#pragma once

#include "elementwise.cuh"

namespace tp {

enum : int {
  MET_MSE = 0,
  MET_MAE = 1,
  MET_ACCURACY = 2,         // integer predicted labels vs integer labels
  MET_BCE = 3,              // probabilities vs {0, 1} labels
  MET_CE = 4,               // (rows, classes) probabilities vs class labels
  MET_ACCURACY_ARGMAX = 5,  // (rows, classes) scores: argmax vs class labels
  MET_R2 = 6,
};

struct MetricSrc {
  int metric;
  int64_t N;       // rows
  int C;           // classes per row (1 unless CE / argmax accuracy)
  const float* yf;        // fp32 labels (regression)
  const int64_t* yi;      // integer labels
};

// torch's log clamped at -100 (binary_cross_entropy); the hardware logarithm (__logf,
// absolute error below 2^-21 on [0.5, 2]) keeps the metric kernels memory-bound, and its
// error is far below the metrics' fp32 tolerance.  Inputs below the normal range give -inf
// and clamp to -100 like the exact log (which is below -87 there).
__device__ __forceinline__ float log_clamped(float x) { return fmaxf(__logf(x), -100.0f); }

// Block-wide fp64 sum (blockDim.x multiple of 32, <= 1024).
__device__ __forceinline__ double block_sum(double v, double* sh) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x < 32) {
    t = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : 0.0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, off);
  }
  return t;  // valid in thread 0
}

// Per-row term of the single-output metrics for prediction value p of row i.
template <int MET>
__device__ __forceinline__ float metric_term(const MetricSrc& s, float p, int64_t i) {
  if (MET == MET_MSE || MET == MET_R2) {
    const float d = p - s.yf[i];
    return d * d;
  } else if (MET == MET_MAE) {
    return fabsf(p - s.yf[i]);
  } else {  // MET_BCE: torch's (t - 1) max(log(1 - p), -100) - t max(log(p), -100)
    const int64_t y = s.yi[i];
    if (y == 0 || y == 1) return -log_clamped(y ? p : 1.0f - p);  // the other term is exactly 0
    const float yf = (float)y;
    return -(yf * log_clamped(p) + (1.0f - yf) * log_clamped(1.0f - p));
  }
}

// Sum over rows [r0, r1) of the metric's per-row term for one prediction `val(i, c)`
// (this thread's share; the caller reduces over the block).  The single-output metrics read
// four rows per thread before any arithmetic (loads in flight) and keep two fp64
// accumulators.
template <int MET, typename RowVal>
__device__ __forceinline__ double metric_row_sum(const MetricSrc& s, RowVal val, int64_t r0, int64_t r1) {
  double acc0 = 0.0, acc1 = 0.0;
  const int64_t st = blockDim.x;
  int64_t i = r0 + threadIdx.x;
  if constexpr (MET == MET_MSE || MET == MET_R2 || MET == MET_MAE || MET == MET_BCE) {
    constexpr int U = 4;
    for (; i + (U - 1) * st < r1; i += U * st) {
      float p[U];
#pragma unroll
      for (int u = 0; u < U; ++u) p[u] = val(i + u * st, 0);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const double t = (double)metric_term<MET>(s, p[u], i + u * st);
        if (u & 1)
          acc1 += t;
        else
          acc0 += t;
      }
    }
    for (; i < r1; i += st) acc0 += (double)metric_term<MET>(s, val(i, 0), i);
  } else {
    for (; i < r1; i += st) {
      float t = 0.0f;
      if (MET == MET_CE) {
        const int64_t y = s.yi[i];  // a label outside [0, C) poisons the metric (the reference raises)
        t = (y >= 0 && y < s.C) ? -log_clamped(val(i, (int)y)) : __int_as_float(0x7fc00000);
      } else {  // MET_ACCURACY_ARGMAX
        int best = 0;
        float bv = val(i, 0);
        for (int c = 1; c < s.C; ++c) {
          const float v = val(i, c);
          if (v > bv || (v != v && bv == bv)) {  // first maximum; NaN wins like torch.argmax
            bv = v;
            best = c;
          }
        }
        t = (best == (int)s.yi[i]) ? 1.0f : 0.0f;
      }
      acc0 += (double)t;
    }
  }
  return acc0 + acc1;
}

// One block per prediction: out[p] = metric of y_pred[p].
template <int MET>
__global__ void __launch_bounds__(1024) metric_pack_kernel(MetricSrc s, const float* yp, const int64_t* yp_int,
                                                           float* out) {
  __shared__ double sh[32];
  const int p = blockIdx.x;
  double total;
  if (MET == MET_ACCURACY) {
    double acc = 0.0;
    const int64_t* q = yp_int + (size_t)p * s.N;
    for (int64_t i = threadIdx.x; i < s.N; i += blockDim.x) acc += (q[i] == s.yi[i]) ? 1.0 : 0.0;
    total = block_sum(acc, sh);
  } else {
    const float* q = yp + (size_t)p * s.N * s.C;
    total = block_sum(metric_row_sum<MET>(s, [&](int64_t i, int c) { return q[i * s.C + c]; }, 0, s.N), sh);
  }
  if (MET == MET_R2) {
    // denominator: sum (y - mean(y))^2 over the shared labels (two passes, fp64)
    double sy = 0.0;
    for (int64_t i = threadIdx.x; i < s.N; i += blockDim.x) sy += (double)s.yf[i];
    __shared__ double mean_sh;
    const double tot_y = block_sum(sy, sh);
    if (threadIdx.x == 0) mean_sh = tot_y / (double)s.N;
    __syncthreads();
    const double mean = mean_sh;
    double sd = 0.0;
    for (int64_t i = threadIdx.x; i < s.N; i += blockDim.x) {
      const double d = (double)s.yf[i] - mean;
      sd += d * d;
    }
    const double den = block_sum(sd, sh);
    if (threadIdx.x == 0) {
      double ratio = total / den;
      if (total == 0.0) ratio = 0.0;         // force_finite: perfect prediction
      else if (den == 0.0) ratio = 1.0;      // force_finite: constant target
      out[p] = s.N < 2 ? __int_as_float(0x7fc00000) : (float)(1.0 - ratio);
    }
    return;
  }
  if (threadIdx.x == 0) out[p] = (float)(total / (double)s.N);
}

// ---------------------------------------------------------------------------- greedy
struct GreedyState {
  double ens_score;   // score of the current ensemble (higher is better)
  int stop;           // 1: finished (no improvement, or size limit)
  int error;          // 1: a candidate score was NaN
  int wsum;           // number of selections so far
  int size;           // number of distinct members
  int best;           // candidate chosen in the last selection
  int iters;
};

struct GreedyArgs {
  MetricSrc s;
  int Cand;                // number of predictions
  const float* pred;       // (Cand, N, C)
  int sign;                // +1: maximise the metric, -1: minimise
  int with_replacement;
  int limit;               // stop once wsum reaches it
  int* counts;             // (Cand,)
  float* ens;              // (N, C)
  int S;                   // row segments per candidate in the scoring launch
  int64_t seg;             // rows per segment
  double* partials;        // (Cand, S) fp64 metric sums of the segments
  double* scores;          // (Cand,)
  double* ind_scores;      // (Cand,)
  GreedyState* st;
};

__device__ __forceinline__ float greedy_weight(int wsum) { return (float)((double)wsum / (double)(wsum + 1)); }

// partials[c][s] = sum over the rows of segment s of the metric terms of lerp(pred_c, ens, w)
// for every candidate c (grid: candidates x segments; greedy_select_kernel adds the
// segments of a candidate in order).
template <int MET>
__global__ void __launch_bounds__(256) greedy_score_kernel(GreedyArgs g) {
  __shared__ double sh[32];
  if (g.st->stop) return;
  const int c = blockIdx.x;
  const int64_t r0 = (int64_t)blockIdx.y * g.seg, r1 = min(g.s.N, r0 + g.seg);
  if (!g.with_replacement && g.counts[c] > 0) return;
  const float w = greedy_weight(g.st->wsum);
  const float* q = g.pred + (size_t)c * g.s.N * g.s.C;
  const float* e = g.ens;
  const int C = g.s.C;
  const double tot = block_sum(metric_row_sum<MET>(g.s, [&](int64_t i, int k) {
                                 return lerp_t(q[i * C + k], e[i * C + k], w);
                               }, r0, r1),
                               sh);
  if (threadIdx.x == 0) g.partials[(size_t)c * g.S + blockIdx.y] = tot;
}

// Pick the best candidate (single block), stop if it does not improve the ensemble.
__global__ void __launch_bounds__(1024) greedy_select_kernel(GreedyArgs g) {
  __shared__ double sb[32];
  __shared__ double si[32];
  __shared__ int sx[32];
  __shared__ int nan_seen;
  if (g.st->stop) return;
  if (threadIdx.x == 0) nan_seen = 0;
  __syncthreads();
  double bs = -INFINITY, bi = -INFINITY;
  int bx = 0x7FFFFFFF;
  for (int c = threadIdx.x; c < g.Cand; c += blockDim.x) {
    if (!g.with_replacement && g.counts[c] > 0) continue;
    double tot = 0.0;
    for (int k = 0; k < g.S; ++k) tot += g.partials[(size_t)c * g.S + k];
    const double s = (double)g.sign * (double)(float)(tot / (double)g.s.N), is = g.ind_scores[c];
    if (s != s) {
      nan_seen = 1;
      continue;
    }
    if (s > bs || (s == bs && (is > bi || (is == bi && c < bx)))) {
      bs = s;
      bi = is;
      bx = c;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const double os = __shfl_xor_sync(0xFFFFFFFFu, bs, off);
    const double oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
    const int ox = __shfl_xor_sync(0xFFFFFFFFu, bx, off);
    if (os > bs || (os == bs && (oi > bi || (oi == bi && ox < bx)))) {
      bs = os;
      bi = oi;
      bx = ox;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sb[w] = bs;
    si[w] = bi;
    sx[w] = bx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) {
      if (sb[k] > bs || (sb[k] == bs && (si[k] > bi || (si[k] == bi && sx[k] < bx)))) {
        bs = sb[k];
        bi = si[k];
        bx = sx[k];
      }
    }
    GreedyState* st = g.st;
    st->iters += 1;
    if (nan_seen) {  // torch's max propagates NaN; the reference then raises
      st->error = 1;
      st->stop = 1;
    } else if (bx == 0x7FFFFFFF || !(bs > st->ens_score)) {
      st->stop = 1;
    } else {
      st->best = bx;
      st->ens_score = bs;
      g.counts[bx] += 1;
      if (g.counts[bx] == 1) st->size += 1;
    }
  }
}

// ens = lerp(pred_best, ens, w) -- the chosen candidate's would-be ensemble.
__global__ void greedy_update_kernel(GreedyArgs g) {
  GreedyState* st = g.st;
  if (st->stop) return;
  const float w = greedy_weight(st->wsum);
  const float* q = g.pred + (size_t)st->best * g.s.N * g.s.C;
  const int64_t n = g.s.N * g.s.C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    g.ens[i] = lerp_t(q[i], g.ens[i], w);
}

// After the update: one more selection; the limit ends the loop.
__global__ void greedy_advance_kernel(GreedyArgs g) {
  GreedyState* st = g.st;
  if (st->stop) return;
  st->wsum += 1;
  if (st->wsum >= g.limit) st->stop = 1;
}

// Initial ensemble: top-k individual scores (stable descending), mean of their predictions.
__global__ void greedy_init_select_kernel(GreedyArgs g, int k, int* init_idx) {
  if (threadIdx.x != 0) return;
  for (int j = 0; j < k; ++j) {
    int bx = -1;
    double bv = 0.0;
    for (int c = 0; c < g.Cand; ++c) {
      bool taken = false;
      for (int q = 0; q < j; ++q) taken |= (init_idx[q] == c);
      if (taken) continue;
      const double v = g.ind_scores[c];
      if (bx < 0 || v > bv || (v != v && bv == bv)) {
        bv = v;
        bx = c;
      }
    }
    init_idx[j] = bx;
    g.counts[bx] = 1;
  }
  GreedyState* st = g.st;
  st->wsum = k;
  st->size = k;
  st->stop = (k >= g.limit) ? 1 : 0;
  st->error = 0;
  st->iters = 0;
  st->best = -1;
}

__global__ void greedy_init_mean_kernel(GreedyArgs g, int k, const int* init_idx) {
  const int64_t n = g.s.N * g.s.C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int j = 0; j < k; ++j) s += g.pred[(size_t)init_idx[j] * n + i];
    g.ens[i] = s / (float)k;
  }
}

template <int MET>
__global__ void __launch_bounds__(1024) greedy_init_score_kernel(GreedyArgs g) {
  __shared__ double sh[32];
  const float* e = g.ens;
  const int C = g.s.C;
  const double tot = block_sum(metric_row_sum<MET>(g.s, [&](int64_t i, int k) { return e[i * C + k]; }, 0, g.s.N), sh);
  if (threadIdx.x == 0) g.st->ens_score = (double)g.sign * (double)(float)(tot / (double)g.s.N);
}

// ind_scores = sign * metric(pred_c) as doubles of the fp32 metric values.
__global__ void greedy_sign_kernel(const float* metric, double* ind, int n, int sign) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) ind[i] = (double)sign * (double)metric[i];
}

// out[j] = sum_k w_k pred[idx_k][j] / sum_k w_k (w = 1 when weights is null), fp32 in
// member order -- compute_unsanitized_ensemble_predictions (ensemble.py:25-61).
__global__ void ensemble_mean_kernel(const float* pred, const int32_t* idx, const float* weights, int K, int64_t n,
                                     float* out) {
  float wsum = 0.0f;
  for (int k = 0; k < K; ++k) wsum += weights ? weights[k] : 1.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.0f;
    if (weights) {
      for (int k = 0; k < K; ++k) s += (weights[k] / wsum) * pred[(size_t)idx[k] * n + i];
    } else {
      for (int k = 0; k < K; ++k) s += pred[(size_t)idx[k] * n + i];
      s /= (float)K;
    }
    out[i] = s;
  }
}

// Row-wise softmax over the last dimension (C classes), fp32: the prediction transform
// `functools.partial(torch.softmax, dim=-1)` of classification runs.  One warp per row.
__global__ void softmax_rows_kernel(const float* x, int64_t rows, int C, float* out) {
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* r = x + row * C;
  float mx = -INFINITY;
  for (int c = lane; c < C; c += 32) mx = fmaxf(mx, r[c]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
  float s = 0.0f;
  for (int c = lane; c < C; c += 32) s += expf(r[c] - mx);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, off);
  for (int c = lane; c < C; c += 32) out[row * C + c] = expf(r[c] - mx) / s;
}

// keys[m][i] = (word 0 >> 1) of Philox4x32-10 with key = seed and counter
// (i, member_base + m, epoch, 0x9E3779B9): sorting each member's row keys gives a
// batch order that depends only on (seed, epoch, global member id).
__global__ void permutation_keys_kernel(uint32_t k0, uint32_t k1, uint32_t epoch, uint32_t member_base, int P,
                                        int64_t N, int32_t* keys) {
  const int64_t total = (int64_t)P * N;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(t / N);
    const uint32_t i = (uint32_t)(t - (int64_t)m * N);
    keys[t] = (int32_t)(philox4x32_10(make_uint4(i, member_base + (uint32_t)m, epoch, 0x9E3779B9u), k0, k1).x >> 1);
  }
}

}  // namespace tp
