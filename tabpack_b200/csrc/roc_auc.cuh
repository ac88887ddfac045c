// Per-member binary ROC AUC (binary_roc_auc_pack, src/tabpackage/metrics.py:117-150):
// the Mann-Whitney U statistic with midranks over each member's scores.
//
// One CTA of 1024 threads per member:
//   1. scores -> order-preserving unsigned keys (-0.0 folded into +0.0, every NaN to the
//      positive quiet-NaN pattern so NaNs sort last, as torch.argsort places them), labels
//      -> bytes;
//   2. stable LSD radix sort of (key, label), 8-bit digits.  Warp w owns the contiguous
//      index range [w * N / 32, (w + 1) * N / 32); per pass each warp counts its digits,
//      the block turns the counts into per-warp bucket cursors (bucket base + counts of the
//      warps before it), and each warp scatters its range 32 items at a time, ranking equal
//      digits inside a chunk with __match_any_sync.  Range order, chunk order and lane order
//      are the index order, so every pass is stable;
//   3. tie groups of equal keys (a NaN is never equal to anything, so each NaN is its own
//      group, as `x[:, 1:] != x[:, :-1]` treats it): a group spanning sorted positions
//      [first, last] has midrank (first + last) / 2 + 1, so 2 * sum over positives of the
//      midrank is sum over groups of positives_in_group * (first + last + 2), an exact
//      integer; 2U = that - n_pos (n_pos + 1) and AUC = 2U / (2 n_pos n_neg), NaN when
//      n_pos * n_neg == 0.  The reference accumulates the same sum in the scores' float
//      type; here it is exact.
#pragma once

#include "common.cuh"

namespace tp {

constexpr int AUC_THREADS = 1024;
constexpr int AUC_WARPS = AUC_THREADS / 32;

template <typename K>
struct AucKey;

template <>
struct AucKey<uint32_t> {
  using F = float;
  static constexpr uint32_t NAN_KEY = 0x7FC00000u ^ 0x80000000u;
  __device__ static uint32_t make(float x) {
    uint32_t b = __float_as_uint(x);
    if (x != x) b = 0x7FC00000u;  // one NaN pattern, positive
    if (x == 0.0f) b = 0u;        // -0.0 == +0.0
    return (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
  }
};

template <>
struct AucKey<uint64_t> {
  using F = double;
  static constexpr uint64_t NAN_KEY = 0x7FF8000000000000ull ^ 0x8000000000000000ull;
  __device__ static uint64_t make(double x) {
    uint64_t b = (uint64_t)__double_as_longlong(x);
    if (x != x) b = 0x7FF8000000000000ull;
    if (x == 0.0) b = 0ull;
    return (b & 0x8000000000000000ull) ? ~b : (b ^ 0x8000000000000000ull);
  }
};

struct AucArgs {
  int P;
  long long N;
  const void* scores;    // (P, N) fp32 or fp64
  const int64_t* labels; // (N,), nonzero = positive
  void* out;             // (P,) in the scores' type
  void* ws;              // per member: keys[2][N], labels[2][N]
};

template <typename K>
__device__ __forceinline__ int auc_digit(K key, int shift) {
  return (int)((key >> shift) & 0xFFu);
}

template <typename K>
__global__ void __launch_bounds__(AUC_THREADS) roc_auc_kernel(const AucArgs a) {
  using F = typename AucKey<K>::F;
  __shared__ uint32_t cur[AUC_WARPS][256];  // per-warp digit counts, then scatter cursors
  __shared__ unsigned long long red[AUC_WARPS];
  __shared__ unsigned long long red_pos[AUC_WARPS];
  const int m = blockIdx.x;
  const long long N = a.N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t lt_mask = (1u << lane) - 1u;

  // workspace of this member
  const size_t per_member = (size_t)N * (2 * sizeof(K) + 2);
  uint8_t* base = reinterpret_cast<uint8_t*>(a.ws) + (size_t)m * ((per_member + 255) & ~(size_t)255);
  K* keys[2] = {reinterpret_cast<K*>(base), reinterpret_cast<K*>(base) + N};
  uint8_t* labs[2] = {base + 2 * (size_t)N * sizeof(K), base + 2 * (size_t)N * sizeof(K) + N};

  const F* sc = reinterpret_cast<const F*>(a.scores) + (size_t)m * N;
  for (long long i = threadIdx.x; i < N; i += AUC_THREADS) {
    keys[0][i] = AucKey<K>::make(sc[i]);
    labs[0][i] = a.labels[i] != 0 ? 1 : 0;
  }
  __syncthreads();

  // warp ranges
  const long long r0 = (N * warp) / AUC_WARPS, r1 = (N * (warp + 1)) / AUC_WARPS;
  int src = 0;
  for (int shift = 0; shift < (int)(8 * sizeof(K)); shift += 8) {
    for (int d = lane; d < 256; d += 32) cur[warp][d] = 0;
    __syncwarp();
    // 1. per-warp digit counts
    for (long long i0 = r0; i0 < r1; i0 += 32) {
      const long long i = i0 + lane;
      const bool ok = i < r1;
      const int d = ok ? auc_digit(keys[src][i], shift) : 256 + lane;  // out-of-range lanes never match
      const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
      if (ok && (peers & lt_mask) == 0) cur[warp][d] += __popc(peers);
      __syncwarp();
    }
    __syncthreads();
    // 2. cursors: bucket base (exclusive scan of the totals) + counts of the earlier warps
    if (threadIdx.x < 256) {
      const int d = threadIdx.x;
      uint32_t run = 0;
      for (int w = 0; w < AUC_WARPS; ++w) {
        const uint32_t c = cur[w][d];
        cur[w][d] = run;
        run += c;
      }
      // run = total count of digit d; exclusive scan across the 256 digits (warps 0..7)
      uint32_t incl = run;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, off);
        if (lane >= off) incl += v;
      }
      __shared__ uint32_t wsum[8];
      if (lane == 31) wsum[warp] = incl;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      uint32_t before = 0;
      for (int w = 0; w < warp; ++w) before += wsum[w];
      const uint32_t excl = before + incl - run;
      for (int w = 0; w < AUC_WARPS; ++w) cur[w][d] += excl;
    }
    __syncthreads();
    // 3. stable scatter
    const int dst = src ^ 1;
    for (long long i0 = r0; i0 < r1; i0 += 32) {
      const long long i = i0 + lane;
      const bool ok = i < r1;
      K key = 0;
      uint8_t lab = 0;
      if (ok) {
        key = keys[src][i];
        lab = labs[src][i];
      }
      const int d = ok ? auc_digit(key, shift) : 256 + lane;
      const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
      if (ok) {
        const uint32_t pos = cur[warp][d] + __popc(peers & lt_mask);
        keys[dst][pos] = key;
        labs[dst][pos] = lab;
      }
      __syncwarp();
      if (ok && (peers & lt_mask) == 0) cur[warp][d] += __popc(peers);
      __syncwarp();
    }
    __syncthreads();
    src = dst;
  }

  // tie groups: thread t owns the groups that start in its contiguous chunk
  const K* ks = keys[src];
  const uint8_t* ls = labs[src];
  const long long c0 = (N * threadIdx.x) / AUC_THREADS, c1 = (N * (threadIdx.x + 1)) / AUC_THREADS;
  unsigned long long sum2 = 0, npos = 0;
  for (long long i = c0; i < c1; ++i) npos += ls[i];
  long long i = c0;
  while (i < c1) {
    const K k = ks[i];
    const bool starts = (i == 0) || k == AucKey<K>::NAN_KEY || ks[i - 1] != k;
    if (!starts) {
      ++i;
      continue;
    }
    long long j = i;
    unsigned long long pg = ls[i];
    if (k != AucKey<K>::NAN_KEY)
      while (j + 1 < N && ks[j + 1] == k) {
        ++j;
        pg += ls[j];
      }
    sum2 += pg * (unsigned long long)(i + j + 2);
    i = j + 1;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    sum2 += __shfl_xor_sync(0xFFFFFFFFu, sum2, off);
    npos += __shfl_xor_sync(0xFFFFFFFFu, npos, off);
  }
  if (lane == 0) {
    red[warp] = sum2;
    red_pos[warp] = npos;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long s2 = 0, np = 0;
    for (int w = 0; w < AUC_WARPS; ++w) {
      s2 += red[w];
      np += red_pos[w];
    }
    const long long nneg = N - (long long)np;
    F res;
    if (np == 0 || nneg == 0) {
      res = F(NAN);
    } else {
      const long long u2 = (long long)s2 - (long long)(np * (np + 1));
      res = F((double)u2 / (2.0 * (double)np * (double)nneg));
    }
    reinterpret_cast<F*>(a.out)[m] = res;
  }
}

// Bytes of workspace for P members of N scores (fp32 when key_bytes == 4, fp64 when 8).
inline size_t roc_auc_workspace_bytes(long long P, long long N, int key_bytes) {
  const size_t per_member = (size_t)N * (2 * (size_t)key_bytes + 2);
  return (size_t)P * ((per_member + 255) & ~(size_t)255);
}

}  // namespace tp
