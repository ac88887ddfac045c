// First layer of a TabPack over one-hot categorical features as a gather-sum
// (_OneHotEncoding, src/tabpackage/nn.py:1836-1871, feeding the first LinearPack,
// nn.py:792-816 via the concat of nn.py:2071-2107).
//
// With one-hot columns j = off_f + c_f(r) (c_f(r) the category of feature f in batch row r;
// the value `card_f` and anything outside [0, card_f) encode as zeros), the first layer is
//   y[m, r, n] = sum_{k < n_dense} x[m, r, k] W[m, n, k] + sum_f W[m, n, n_dense + off_f + c_f(r)] + b[m, n]
// and its weight gradient over the one-hot columns is a segmented sum of the pre-activation
// gradient G over the rows of each category:
//   dW[m, n, n_dense + off_f + v] = sum_{r : c_f(r) = v} G[m, r, n].
// The dense part runs on the tensor cores (K = n_dense instead of n_dense + n_onehot); the
// kernels here build the gathered addend E[m, r, n] = sum_f W[m, n, n_dense + off_f + c_f(r)]
// (from a transposed bf16 copy Wt[m, j, n] of the one-hot block, so every gathered row is
// contiguous), sort each member's batch rows by category (keys category << 32 | row, so rows
// ascend within a category), and form the segmented sums in ascending row order
// (deterministic).
#pragma once

#include "common.cuh"

namespace tp {

struct OneHotArgs {
  int P, B, n_cat, n_onehot;
  const int32_t* offsets;    // (n_cat + 1,) one-hot column offsets, total last
  const int64_t* x_cat;      // categories: row (row_index ? row_index[m, r] : r) + m * x_cat_ms
  long long x_cat_ms;        // member stride of x_cat in rows (0: shared by the members)
  const int64_t* row_index;  // (P or 1, B) or nullptr
  long long row_index_ms;    // member stride of row_index (0: shared)
  uint64_t* sorted_keys;     // (P, n_cat, B): (category << 32 | row) of each feature, ascending
  // forward addend
  const __nv_bfloat16* wt;   // (P, n_onehot, wt_ld): Wt[m, j, n] = W[m, n, n_dense + j]
  int wt_ld;
  const int32_t* out_f;      // (P,) or nullptr
  int max_out;
  float* addend;             // (P, B, add_ld)
  int add_ld;
  // weight gradient
  const void* g;             // (P, B, g_ld) pre-activation gradient, bf16 or fp32
  int g_ld, g_bf16;
  float* dw;                 // (P, dw_rows, dw_ld); columns dw_col0 .. dw_col0 + n_onehot written
  int dw_rows, dw_ld, dw_col0;
};

__device__ __forceinline__ long long onehot_xrow(const OneHotArgs& a, int m, int r) {
  const long long src = a.row_index != nullptr ? __ldg(a.row_index + m * a.row_index_ms + r) : (long long)r;
  return src + (long long)m * a.x_cat_ms;
}

// Category of feature f (card = its cardinality) in x_cat row xr: card for the unknown value
// and anything outside [0, card).
__device__ __forceinline__ uint32_t onehot_category(const OneHotArgs& a, long long xr, int f, int card) {
  const long long v = __ldg(a.x_cat + xr * a.n_cat + f);
  return (v < 0 || v >= card) ? (uint32_t)card : (uint32_t)v;
}

// Grid: (n_cat, P); `pow2` = B rounded up to a power of two, keys in dynamic shared memory.
// Bitonic sort of (category << 32 | row); the unknown category `card` sorts last.
__global__ void __launch_bounds__(1024) onehot_sort_kernel(const OneHotArgs a, int pow2) {
  extern __shared__ unsigned long long okeys[];
  const int f = blockIdx.x, m = blockIdx.y;
  const int off = __ldg(a.offsets + f), card = __ldg(a.offsets + f + 1) - off;
  for (int i = threadIdx.x; i < pow2; i += blockDim.x) {
    unsigned long long k = ~0ull;
    if (i < a.B) k = ((unsigned long long)onehot_category(a, onehot_xrow(a, m, i), f, card) << 32) | (uint32_t)i;
    okeys[i] = k;
  }
  __syncthreads();
  for (int size = 2; size <= pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < pow2 / 2; t += blockDim.x) {
        const int lo = 2 * t - (t & (stride - 1)), hi = lo + stride;
        const unsigned long long x = okeys[lo], y = okeys[hi];
        if ((x > y) == ((lo & size) == 0)) {
          okeys[lo] = y;
          okeys[hi] = x;
        }
      }
      __syncthreads();
    }
  }
  uint64_t* out = a.sorted_keys + ((size_t)m * a.n_cat + f) * a.B;
  for (int i = threadIdx.x; i < a.B; i += blockDim.x) out[i] = okeys[i];
}

// Grid: (ceil(B / 8), P), 256 threads: a warp builds the addend row of one batch row,
// 8 output features per lane and step (one 16-byte load of Wt per feature), features
// summed in order in fp32.
__global__ void __launch_bounds__(256) onehot_gather_kernel(const OneHotArgs a) {
  const int m = blockIdx.y;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= a.B) return;
  const int nv = a.out_f != nullptr ? min(__ldg(a.out_f + m), a.max_out) : a.max_out;
  const long long xr = onehot_xrow(a, m, r);
  const __nv_bfloat16* wt = a.wt + (size_t)m * a.n_onehot * a.wt_ld;
  float* e = a.addend + ((size_t)m * a.B + r) * a.add_ld;
  // the loops are warp-uniform (the feature rows travel by shuffles); lanes past the member's
  // width take part without loading or storing
  for (int base = 0; base < nv; base += 256) {
    const int c0 = base + lane * 8;
    const bool on = c0 < nv;
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.0f;
    for (int f0 = 0; f0 < a.n_cat; f0 += 32) {
      // lane i holds the Wt row of feature f0 + i (-1: no contribution)
      int j = -1;
      if (f0 + lane < a.n_cat) {
        const int f = f0 + lane;
        const int off = __ldg(a.offsets + f), card = __ldg(a.offsets + f + 1) - off;
        const uint32_t c = onehot_category(a, xr, f, card);
        j = c < (uint32_t)card ? off + (int)c : -1;
      }
      const int nf = min(32, a.n_cat - f0);
#pragma unroll 4
      for (int i = 0; i < nf; ++i) {
        const int ji = __shfl_sync(0xFFFFFFFFu, j, i);
        if (ji >= 0 && on) {
          const uint4 w = *reinterpret_cast<const uint4*>(wt + (size_t)ji * a.wt_ld + c0);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 v = __bfloat1622float2(h[k]);
            acc[2 * k] += v.x;
            acc[2 * k + 1] += v.y;
          }
        }
      }
    }
    if (on) {
      *reinterpret_cast<float4*>(e + c0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(e + c0 + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

// One-hot column j's sums of a warp's 64 output features (two per lane) into its staged
// 32-column chunk; the chunk is written when its last column arrives: 64 dW rows x 128 bytes.
template <int LD>
__device__ __forceinline__ void onehot_wgrad_emit(float (*T)[LD], float* dw, int dw_ld, int n_onehot, int n0,
                                                  int rows_here, int lane, int j, float v0, float v1) {
  T[j & 31][2 * lane] = v0;
  T[j & 31][2 * lane + 1] = v1;
  if ((j & 31) == 31 || j == n_onehot - 1) {
    __syncwarp();
    const int base = j & ~31, ncol = j - base + 1;
    if (lane < ncol)
      for (int r = 0; r < rows_here; ++r) dw[(size_t)(n0 + r) * dw_ld + base + lane] = T[lane][r];
    __syncwarp();
  }
}

constexpr int ONEHOT_WG_WARPS = 4;  // warps per CTA, each an independent task (33 KB of staging)
constexpr int ONEHOT_WG_N = 64;     // output features per warp task (two per lane)

// Grid: (ceil(P * ceil(dw_rows / 64) / 4), 1), 128 threads.  Warp task (m, nb) sums the one-hot
// columns for output features n0 = 64 nb .. n0 + 63 (lane: n0 + 2 lane and the next): it walks
// the member's sorted keys feature by feature (categories ascending, rows ascending within a
// category), reading 32 keys with one load and the 32 rows' G pairs (128-byte pieces)
// together, and closes a category's sums when the category changes.  Every 32 columns are
// staged in the warp's shared tile and written as 64 dW rows x 128 contiguous bytes.  Output
// features at or beyond the member's width and categories without rows get zeros.  G is bf16
// with an even g_ld.
__global__ void __launch_bounds__(32 * ONEHOT_WG_WARPS) onehot_wgrad_kernel(const OneHotArgs a, int nb_count) {
  __shared__ float tile[ONEHOT_WG_WARPS][32][ONEHOT_WG_N + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long task = (long long)blockIdx.x * ONEHOT_WG_WARPS + warp;
  if (task >= (long long)a.P * nb_count) return;
  const int m = (int)(task / nb_count), nb = (int)(task - (long long)m * nb_count);
  const int n0 = ONEHOT_WG_N * nb;
  const int nv = a.out_f != nullptr ? min(__ldg(a.out_f + m), a.max_out) : a.max_out;
  const int n = n0 + 2 * lane;
  const bool live0 = n < nv, live1 = n + 1 < nv;
  float(*T)[ONEHOT_WG_N + 1] = tile[warp];
  float* dw = a.dw + (size_t)m * a.dw_rows * a.dw_ld + a.dw_col0;
  const int rows_here = min(ONEHOT_WG_N, a.dw_rows - n0);
  // column j's sums go to the staged chunk; the chunk is written when its last column arrives
#define ONEHOT_EMIT(j_, v0_, v1_) onehot_wgrad_emit(T, dw, a.dw_ld, a.n_onehot, n0, rows_here, lane, (j_), (v0_), (v1_))
  if (n0 >= nv) {
    for (int j = 0; j < a.n_onehot; ++j) ONEHOT_EMIT(j, 0.0f, 0.0f);
    return;
  }
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(a.g) + (size_t)m * a.B * a.g_ld + n;
  const uint64_t* keys_m = a.sorted_keys + (size_t)m * a.n_cat * a.B;
  for (int f = 0; f < a.n_cat; ++f) {
    const int off = __ldg(a.offsets + f), card = __ldg(a.offsets + f + 1) - off;
    const uint64_t* keys = keys_m + (size_t)f * a.B;
    int v = 0;  // the category whose sums are open
    float acc0 = 0.0f, acc1 = 0.0f;
    bool done = card == 0;
    // keys of the next 32 positions are loaded while the current ones are consumed
    uint64_t kn = (!done && lane < a.B) ? __ldg(keys + lane) : ~0ull;
    for (int i0 = 0; i0 < a.B && !done; i0 += 32) {
      const uint64_t kl = kn;
      kn = (i0 + 32 + lane < a.B) ? __ldg(keys + i0 + 32 + lane) : ~0ull;
      const uint32_t rl = (uint32_t)kl, cl = (uint32_t)(kl >> 32);
      // the 32 rows' G pairs as raw words, all loads issued before any is used
      uint32_t gw[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const uint32_t r = __shfl_sync(0xFFFFFFFFu, rl, k), c = __shfl_sync(0xFFFFFFFFu, cl, k);
        gw[k] = (c < (uint32_t)card && live0) ? __ldg(reinterpret_cast<const uint32_t*>(g + (size_t)r * a.g_ld)) : 0u;
      }
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const uint32_t c = __shfl_sync(0xFFFFFFFFu, cl, k);
        if (c >= (uint32_t)card) {  // the unknown category (and the batch end): nothing follows
          done = true;
          break;
        }
        while ((uint32_t)v < c) {  // close category v (and the empty ones before c)
          ONEHOT_EMIT(off + v, acc0, acc1);
          acc0 = acc1 = 0.0f;
          ++v;
        }
        const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[k]));
        acc0 += x.x;
        acc1 += live1 ? x.y : 0.0f;
      }
    }
    for (; v < card; ++v) {  // the last category with rows, then the empty ones after it
      ONEHOT_EMIT(off + v, acc0, acc1);
      acc0 = acc1 = 0.0f;
    }
  }
#undef ONEHOT_EMIT
}

}  // namespace tp
