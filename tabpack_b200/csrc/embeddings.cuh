// Cosine numerical-feature embeddings (CosineEmbeddingsPack, src/tabpackage/nn.py:1627-1833,
// concat_input = True), forward and parameter gradients.
//
// Member m, feature f, embedding slot k < D (D = max_d_embedding):
//   cat_0 = x,  cat_k = cos(z_k),  z_k = 2pi*b[k-1] + 2pi*w[k-1] * x   (2pi*w, 2pi*b in fp32)
//   out_k = ab'_k + aw'_k * cat_k,  aw' / ab' = aw / ab where k < d_embedding[m], else 0
// written at column f * D + k of the member's output row, so the flattened embedding lands
// directly in the first layer's input (the one-hot block can follow in the same buffer).
//
// Backward, per (m, f, k), sums over the batch rows (fp32 runs of 16 rows added in fp64):
//   dab_k = [k < d] sum g,  daw_k = [k < d] sum g cat_k,
//   dz_k = g aw'_k (-sin z_k),  dw[k-1] = 2pi sum dz_k x,  db[k-1] = 2pi sum dz_k.
// Threads own one column (f, k) each and walk the rows, so parameter loads happen once per
// thread and the loads / stores of a warp are contiguous along the columns.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace tp {

constexpr float COS_EMB_TWO_PI = 6.28318530717958647692f;
constexpr int COS_EMB_THREADS = 128;

// z reduced to about [-pi, pi] by z - k 2pi, k = rint(z / 2pi), with 2pi split into a head of
// 12 significant bits (3217 / 512, so that k * head is exact for |k| < 4096) and an fp32 tail
// (Cody and Waite's argument reduction); the hardware cosine and sine are accurate to about
// 4e-7 absolute on that range.  k = rint(z / 2pi) is formed by adding and subtracting 1.5 * 2^23, which rounds to the nearest
// integer (ties to even) exactly like rintf for |z / 2pi| < 2^22, on the FMA pipe instead of
// the conversion unit that the cosine and sine already keep busy; the _rn intrinsics keep the
// product and the sums separately rounded.
__device__ __forceinline__ float cos_emb_reduce(float z) {
  const float t = __fmul_rn(z, 0.159154936671f);
  const float k = __fsub_rn(__fadd_rn(t, 12582912.0f), 12582912.0f);
  return fmaf(-k, -1.781781975e-05f, fmaf(-k, 6.283203125f, z));
}

struct CosEmbArgs {
  int P, B, F, D;
  int x_shared;            // x is (B, F) for every member, else (P, B, F)
  const float* x;
  const float* w;          // (P, F, D - 1)
  const float* b;          // (P, F, D - 1)
  const float* aw;         // (P, F, D)
  const float* ab;         // (P, F, D)
  const int32_t* d_emb;    // (P,) or nullptr (every slot active)
  void* out;               // (P, B, out_ld), fp32 or bf16
  int out_ld, out_bf16;
  const void* g;           // (P, B, g_ld) upstream gradient, fp32 or bf16
  int g_ld, g_bf16;
  int rows_per_block;      // rows of one block (the grid's z dimension covers B)
  double* partial;         // (4, gridDim.z, P, F * D) or nullptr when gridDim.z == 1
  float* dw;               // (P, F, D - 1)
  float* db;
  float* daw;              // (P, F, D)
  float* dab;
};

struct CosEmbCol {
  int f, k;
  bool valid;
  float aw, ab, w2, b2;
};

__device__ __forceinline__ CosEmbCol cos_emb_col(const CosEmbArgs& a, int m, int j) {
  CosEmbCol c;
  c.valid = j < a.F * a.D;
  c.f = c.valid ? j / a.D : 0;
  c.k = c.valid ? j - c.f * a.D : 0;
  const bool on = c.valid && (a.d_emb == nullptr || c.k < a.d_emb[m]);
  const size_t pa = ((size_t)m * a.F + c.f) * a.D + c.k;
  c.aw = on ? a.aw[pa] : 0.0f;
  c.ab = on ? a.ab[pa] : 0.0f;
  c.w2 = c.b2 = 0.0f;
  if (c.valid && c.k > 0) {
    const size_t pw = ((size_t)m * a.F + c.f) * (a.D - 1) + (c.k - 1);
    c.w2 = a.w[pw] * COS_EMB_TWO_PI;
    c.b2 = a.b[pw] * COS_EMB_TWO_PI;
  }
  return c;
}

__device__ __forceinline__ float cos_emb_value(const CosEmbCol& c, float x) {
  return c.ab + c.aw * (c.k == 0 ? x : __cosf(cos_emb_reduce(c.b2 + c.w2 * x)));
}

// Grid: (ceil(F * D / (2 COS_EMB_THREADS)), P, ceil(B / rows_per_block)).  A thread owns two
// adjacent columns (j0 = 2 t, j0 + 1), stored as one 4- or 8-byte pair when the row stride is
// even.  The output type is
// a template parameter and the row pointers advance by increments, so the loop body is the
// embedding arithmetic and the stores; four rows' x values are loaded (read-only path) before
// their stores, which the compiler could not move them past otherwise (x and out may alias).
template <bool BF16>
__global__ void __launch_bounds__(COS_EMB_THREADS) cos_emb_forward_kernel(const CosEmbArgs a) {
  using T = typename std::conditional<BF16, __nv_bfloat16, float>::type;
  const int m = blockIdx.y;
  const int j0 = 2 * (blockIdx.x * COS_EMB_THREADS + threadIdx.x);
  const CosEmbCol c0 = cos_emb_col(a, m, j0), c1 = cos_emb_col(a, m, j0 + 1);
  if (!c0.valid) return;
  const int r0 = blockIdx.z * a.rows_per_block, r1 = min(a.B, r0 + a.rows_per_block);
  const bool pair = c1.valid && (a.out_ld & 1) == 0;  // one 4- or 8-byte store for both columns
  const int F = a.F;
  const size_t ld = (size_t)a.out_ld;
  const float* xp = a.x + (a.x_shared ? (size_t)r0 : (size_t)m * a.B + r0) * F;
  const int f0 = c0.f, f1 = c1.f;  // f1 = 0 for an invalid second column: in bounds
  T* o = reinterpret_cast<T*>(a.out) + ((size_t)m * a.B + r0) * ld + j0;
  auto store = [&](T* q, float y0, float y1) {
    if constexpr (BF16) {
      if (pair) {
        *reinterpret_cast<uint32_t*>(q) = pack_bf16x2(y0, y1);
      } else {
        q[0] = __float2bfloat16_rn(y0);
        if (c1.valid) q[1] = __float2bfloat16_rn(y1);
      }
    } else {
      if (pair) {
        *reinterpret_cast<float2*>(q) = make_float2(y0, y1);
      } else {
        q[0] = y0;
        if (c1.valid) q[1] = y1;
      }
    }
  };
  int r = r0;
  for (; r + 4 <= r1; r += 4, xp += 4 * F, o += 4 * ld) {
    float xa[4], xb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xa[i] = __ldg(xp + i * F + f0);
      xb[i] = __ldg(xp + i * F + f1);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) store(o + i * ld, cos_emb_value(c0, xa[i]), c1.valid ? cos_emb_value(c1, xb[i]) : 0.0f);
  }
  for (; r < r1; ++r, xp += F, o += ld) {
    const float x0 = __ldg(xp + f0), x1 = __ldg(xp + f1);
    store(o, cos_emb_value(c0, x0), c1.valid ? cos_emb_value(c1, x1) : 0.0f);
  }
}

// Sums of one column over rows: sa = sum g, sw = sum g cat, s1 = sum dz x, s2 = sum dz.
struct CosEmbSums {
  double ab, aw, w, b;
};

// The same four sums over a run of at most COS_EMB_RUN rows in fp32, added to the fp64 sums
// at the end of the run: one conversion per sum and run instead of one per product (the
// conversions share the conversion unit with the sine and cosine).
struct CosEmbRun {
  float ab, aw, w, b;
};
constexpr int COS_EMB_RUN = 16;

__device__ __forceinline__ void cos_emb_accumulate(const CosEmbCol& c, float g, float x, CosEmbRun& s) {
  s.ab += g;
  if (c.k == 0) {
    s.aw = fmaf(g, x, s.aw);
  } else {
    float sn, cs;
    __sincosf(cos_emb_reduce(c.b2 + c.w2 * x), &sn, &cs);
    s.aw = fmaf(g, cs, s.aw);
    const float dz = -(g * c.aw) * sn;
    s.w = fmaf(dz, x, s.w);
    s.b += dz;
  }
}

__device__ __forceinline__ void cos_emb_flush(CosEmbRun& run, CosEmbSums& s) {
  s.ab += (double)run.ab;
  s.aw += (double)run.aw;
  s.w += (double)run.w;
  s.b += (double)run.b;
  run = CosEmbRun{0.0f, 0.0f, 0.0f, 0.0f};
}

__device__ __forceinline__ void cos_emb_write_sums(const CosEmbArgs& a, int m, int j, const CosEmbCol& c,
                                                   const CosEmbSums& s) {
  const size_t FD = (size_t)a.F * a.D;
  if (gridDim.z > 1) {
    const size_t slot = ((size_t)blockIdx.z * a.P + m) * FD + j;
    const size_t plane = (size_t)gridDim.z * a.P * FD;
    a.partial[slot] = s.ab;
    a.partial[plane + slot] = s.aw;
    a.partial[2 * plane + slot] = s.w;
    a.partial[3 * plane + slot] = s.b;
    return;
  }
  const bool on = a.d_emb == nullptr || c.k < a.d_emb[m];
  const size_t pa = ((size_t)m * a.F + c.f) * a.D + c.k;
  a.dab[pa] = on ? (float)s.ab : 0.0f;
  a.daw[pa] = on ? (float)s.aw : 0.0f;
  if (c.k > 0) {
    const size_t pw = ((size_t)m * a.F + c.f) * (a.D - 1) + (c.k - 1);
    a.dw[pw] = (float)s.w * COS_EMB_TWO_PI;
    a.db[pw] = (float)s.b * COS_EMB_TWO_PI;
  }
}

// Grid: (ceil(F * D / COS_EMB_THREADS), P, segments), one column a thread (two columns a thread
// measured slower: twice the accumulation chains per thread).  One block row segment per
// z; with gridDim.z == 1 the sums are final, otherwise they go to `partial` and
// cos_emb_finish_kernel adds the segments in order.
// The gradient's type is a template parameter and the row pointers advance by increments;
// rows are accumulated in order, eight loaded at a time, in fp32 runs of COS_EMB_RUN rows whose
// sums are added in fp64.
template <bool G_BF16>
__global__ void __launch_bounds__(COS_EMB_THREADS) cos_emb_backward_kernel(const CosEmbArgs a) {
  using T = typename std::conditional<G_BF16, __nv_bfloat16, float>::type;
  const int m = blockIdx.y;
  const int j = blockIdx.x * COS_EMB_THREADS + threadIdx.x;
  const CosEmbCol c = cos_emb_col(a, m, j);
  if (!c.valid) return;
  const int r0 = blockIdx.z * a.rows_per_block, r1 = min(a.B, r0 + a.rows_per_block);
  const int F = a.F;
  const size_t ld = (size_t)a.g_ld;
  const float* xp = a.x + (a.x_shared ? (size_t)r0 : (size_t)m * a.B + r0) * F + c.f;
  const T* gp = reinterpret_cast<const T*>(a.g) + ((size_t)m * a.B + r0) * ld + j;
  auto gval = [](T v) -> float {
    if constexpr (G_BF16)
      return __bfloat162float(v);
    else
      return v;
  };
  CosEmbSums sums{0.0, 0.0, 0.0, 0.0};
  CosEmbRun run{0.0f, 0.0f, 0.0f, 0.0f};
  int r = r0;
  constexpr int NR = 8;  // rows loaded ahead
  static_assert(COS_EMB_RUN % NR == 0, "runs hold whole row groups");
  for (; r + NR <= r1; r += NR, xp += NR * F, gp += NR * ld) {
    float gv[NR], xv[NR];
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      gv[i] = gval(gp[i * ld]);
      xv[i] = xp[i * F];
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) cos_emb_accumulate(c, gv[i], xv[i], run);
    if (((r + NR - r0) % COS_EMB_RUN) == 0) cos_emb_flush(run, sums);
  }
  for (; r < r1; ++r, xp += F, gp += ld) cos_emb_accumulate(c, gval(*gp), *xp, run);
  cos_emb_flush(run, sums);
  cos_emb_write_sums(a, m, j, c, sums);
}

// Adds the row segments' partial sums in segment order (deterministic).  Grid:
// (ceil(F * D / COS_EMB_THREADS), P).
__global__ void __launch_bounds__(COS_EMB_THREADS) cos_emb_finish_kernel(const CosEmbArgs a, int segments) {
  const int m = blockIdx.y;
  const int j = blockIdx.x * COS_EMB_THREADS + threadIdx.x;
  const size_t FD = (size_t)a.F * a.D;
  if (j >= (int)FD) return;
  const size_t plane = (size_t)segments * a.P * FD;
  double s[4] = {0.0, 0.0, 0.0, 0.0};
  for (int z = 0; z < segments; ++z) {
    const size_t slot = ((size_t)z * a.P + m) * FD + j;
#pragma unroll
    for (int q = 0; q < 4; ++q) s[q] += a.partial[q * plane + slot];
  }
  const int f = j / a.D, k = j - f * a.D;
  const bool on = a.d_emb == nullptr || k < a.d_emb[m];
  const size_t pa = ((size_t)m * a.F + f) * a.D + k;
  a.dab[pa] = on ? (float)s[0] : 0.0f;
  a.daw[pa] = on ? (float)s[1] : 0.0f;
  if (k > 0) {
    const size_t pw = ((size_t)m * a.F + f) * (a.D - 1) + (k - 1);
    a.dw[pw] = (float)s[2] * COS_EMB_TWO_PI;
    a.db[pw] = (float)s[3] * COS_EMB_TWO_PI;
  }
}

}  // namespace tp

namespace tp {

// ---------------------------------------------------------------------------
// First-layer input of a TabPack without numerical embeddings: the numerical columns
// followed by the one-hot encoding of each categorical feature (_OneHotEncoding,
// src/tabpackage/nn.py:1836-1871: value `card` is the unknown category and encodes as
// zeros), converted to the first layer's dtype and zero-padded to out_ld, in one pass.
// A warp writes one row: the numerical values and zeros as 16-byte stores (8 bf16 or 4 fp32
// values per lane and store), then one store per categorical feature for its 1.
// ---------------------------------------------------------------------------
struct InputArgs {
  long long rows;
  int n_num, n_cat;
  const float* x_num;       // (rows, n_num) or nullptr
  const int64_t* x_cat;     // (rows, n_cat) or nullptr
  const int64_t* row_index; // (rows,) source row of each output row, or nullptr
  const int32_t* offsets;   // (n_cat + 1,): first one-hot column of each feature (relative to n_num), total last
  void* out;                // (rows, out_ld)
  int out_ld, out_bf16;
  int out_col0;             // first column written
};

template <bool BF16>
__global__ void __launch_bounds__(256) tabpack_input_kernel(const InputArgs a) {
  constexpr int V = BF16 ? 8 : 4;  // values per 16-byte piece
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.rows) return;
  const long long src = a.row_index ? a.row_index[row] : row;  // the batch gather
  // pass 1: numerical columns and zeros, 16-byte stores
  const float* xr = a.x_num ? a.x_num + src * a.n_num : nullptr;
  for (int c0 = a.out_col0 + lane * V; c0 < a.out_ld; c0 += 32 * V) {
    const int k0 = c0 - a.out_col0;  // numerical feature of column c0
    float val[V];
#pragma unroll
    for (int e = 0; e < V; ++e) val[e] = (xr != nullptr && k0 + e < a.n_num) ? xr[k0 + e] : 0.0f;
    if (BF16) {
      uint4 u;
      u.x = pack_bf16x2(val[0], val[1]);
      u.y = pack_bf16x2(val[2], val[3]);
      u.z = pack_bf16x2(val[4], val[5]);
      u.w = pack_bf16x2(val[6], val[7]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.out_ld + c0) = u;
    } else {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + row * a.out_ld + c0) =
          make_float4(val[0], val[1], val[2], val[3]);
    }
  }
  // pass 2: one 1 per categorical feature (the warp's stores above precede it)
  __syncwarp();
  if (a.x_cat == nullptr) return;
  for (int f = lane; f < a.n_cat; f += 32) {
    const int64_t v = a.x_cat[src * a.n_cat + f];
    const int start = a.offsets[f], card = a.offsets[f + 1] - start;
    if (v < 0 || v >= card) continue;  // the unknown category `card` stays all zeros
    const size_t o = row * a.out_ld + a.out_col0 + a.n_num + start + (int)v;
    if (BF16)
      reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(1.0f);
    else
      reinterpret_cast<float*>(a.out)[o] = 1.0f;
  }
}

}  // namespace tp
