// Muon optimizer pack: momentum / Nesterov / weight decay, packing of each member's
// update into an oriented bf16 Newton-Schulz operand, Frobenius normalisation, and
// the final scaled update.  The Newton-Schulz GEMMs themselves run on the tcgen05
// kernel (MODE_NS / MODE_NS_BMN).
//
// Orientation: member m with out_m x in_m weights iterates on X = U (r = out_m,
// c = in_m) when out_m <= in_m and on X = U^T otherwise, so its Gram matrix X X^T
// is min(out_m, in_m) square.  In exact arithmetic this is the same function as
// the reference's pack-wide orientation (optim.py:477-489):
// a X + b (X X^T) X + c (X X^T)^2 X  ==  (a X^T + b (X^T X) X^T + c (X^T X)^2 X^T)^T.
#pragma once

#include "elementwise.cuh"

namespace tp {

struct MuonArgs {
  int P, max_out, max_in;
  float* p;
  float* g;
  float* m;
  const int32_t* out_f;  // (P,) or nullptr
  const int32_t* in_f;   // (P,) or nullptr
  const float* lr_pm;
  float lr_s;
  const float* mu_pm;
  float mu_s;
  const float* wd_pm;
  float wd_s;
  int wd_on;
  float wd_mult_s;       // 1 - lr * wd when both are scalars
  float one_m_mu_s;      // 1 - mu (scalar momentum)
  const float* scale_pm; // (P,) update scale, or nullptr -> scale_s
  float scale_s;
  int nesterov, mutate_grad;
  __nv_bfloat16* x;      // (P, R_s, C_s) oriented operand
  int R_s, C_s;
  float* norm2;          // (P,)
  float* partial;        // (P, tiles) per-32x32-tile sums of squares (fixed-order reduction)
  int tiles;             // ceil(max_out / 32) * ceil(max_in / 32)
  int32_t* rows;         // (P,) r_m
  int32_t* cols;         // (P,) c_m
  int32_t* trans;        // (P,) 1: X = U^T
  int32_t* active;       // (P,) norm2 > 0
};

__global__ void muon_geometry_kernel(MuonArgs a) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= a.P) return;
  const int o = a.out_f ? a.out_f[m] : a.max_out;
  const int n = a.in_f ? a.in_f[m] : a.max_in;
  a.rows[m] = min(o, n);
  a.cols[m] = max(o, n);
  a.trans[m] = o > n ? 1 : 0;
}

// 32x32 source tiles (o, n) of member blockIdx.z; 256 threads = 32 columns x 8 row lanes.
__global__ void __launch_bounds__(256) muon_prologue_kernel(MuonArgs a) {
  __shared__ float tile[32][33];
  __shared__ float red[8];
  const int mem = blockIdx.z;
  const int o0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  const int out_m = a.out_f ? a.out_f[mem] : a.max_out;
  const int in_m = a.in_f ? a.in_f[mem] : a.max_in;
  if (o0 >= out_m || n0 >= in_m) return;  // padding: never read, never written
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const float lr = a.lr_pm ? a.lr_pm[mem] : a.lr_s;
  const float mu = a.mu_pm ? a.mu_pm[mem] : a.mu_s;
  const float mult = (a.lr_pm || a.wd_pm) ? 1.0f - lr * (a.wd_pm ? a.wd_pm[mem] : a.wd_s) : a.wd_mult_s;
  const float one_m_mu = a.mu_pm ? 1.0f - mu : a.one_m_mu_s;
  float ss = 0.0f;
  // rows ty, ty + 8, ty + 16, ty + 24: all loads issued before any use
  float pv[4], gv[4], mv[4];
  bool ok[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int o = o0 + ty + 8 * k, n = n0 + tx;
    ok[k] = o < out_m && n < in_m;
    const size_t idx = ((size_t)mem * a.max_out + o) * a.max_in + n;
    pv[k] = ok[k] ? a.p[idx] : 0.0f;
    gv[k] = ok[k] ? a.g[idx] : 0.0f;
    mv[k] = ok[k] ? a.m[idx] : 0.0f;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = ty + 8 * k;
    float u = 0.0f;
    if (ok[k]) {
      const size_t idx = ((size_t)mem * a.max_out + (o0 + i)) * a.max_in + (n0 + tx);
      float p = pv[k];
      if (a.wd_on) p *= mult;
      const float m = lerp_t(mv[k], gv[k], one_m_mu);
      u = a.nesterov ? lerp_t(gv[k], m, mu) : m;
      a.p[idx] = p;
      a.m[idx] = m;
      if (a.nesterov && a.mutate_grad) a.g[idx] = u;
      u = __bfloat162float(__float2bfloat16_rn(u));
      ss += u * u;
    }
    tile[i][tx] = u;
  }
  // Frobenius norm of the bf16 update, per member
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
  if (tx == 0) red[ty] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < 8; ++i) t += red[i];
    a.partial[(size_t)mem * a.tiles + blockIdx.y * gridDim.x + blockIdx.x] = t;
  }
  // oriented bf16 operand
  const bool tr = out_m > in_m;
  __nv_bfloat16* x = a.x + (size_t)mem * a.R_s * a.C_s;
  for (int i = ty; i < 32; i += 8) {
    if (!tr) {
      const int o = o0 + i, n = n0 + tx;
      if (o < out_m && n < in_m) x[(size_t)o * a.C_s + n] = __float2bfloat16_rn(tile[i][tx]);
    } else {
      const int n = n0 + i, o = o0 + tx;  // X[n][o] = U[o][n]
      if (o < out_m && n < in_m) x[(size_t)n * a.C_s + o] = __float2bfloat16_rn(tile[tx][i]);
    }
  }
}

// norm2[m] = sum of the member's tile partials in a fixed order (deterministic),
// active[m] = norm2[m] > 0.  One block per member.
__global__ void __launch_bounds__(256) muon_norm_kernel(MuonArgs a, int tiles_x) {
  __shared__ float red[256];
  const int mem = blockIdx.x;
  const int out_m = a.out_f ? a.out_f[mem] : a.max_out;
  const int in_m = a.in_f ? a.in_f[mem] : a.max_in;
  const int ty_n = (out_m + 31) / 32, tx_n = (in_m + 31) / 32;  // tiles the prologue wrote
  float s = 0.0f;
  for (int t = threadIdx.x; t < ty_n * tx_n; t += blockDim.x) {
    const int ty = t / tx_n, tx = t - ty * tx_n;
    s += a.partial[(size_t)mem * a.tiles + ty * tiles_x + tx];
  }
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    a.norm2[mem] = red[0];
    a.active[mem] = red[0] > 0.0f ? 1 : 0;
  }
}

// X <- bf16(X / bf16(bf16(||X||_F) + 1e-7)) on the member's r x c block and exact zeros
// on [0, R_s-tile) x [0, C_s-tile) around it (the Newton-Schulz GEMMs read those pads
// along K).  Grid: (ceil(C_s / 256), R_s / 8, P), 256 threads, 8 rows x 32 x 8 columns.
__global__ void __launch_bounds__(256) muon_normalize_kernel(MuonArgs a, int row_pad, int col_pad) {
  const int mem = blockIdx.z;
  const int r = a.rows[mem], c = a.cols[mem];
  const int rr = min(a.R_s, (r + row_pad - 1) / row_pad * row_pad);
  const int cc = min(a.C_s, (c + col_pad - 1) / col_pad * col_pad);
  const float nrm2 = a.norm2[mem];
  if (nrm2 == 0.0f) return;  // all-zero update: Newton-Schulz is skipped for this member
  const float nrm = __bfloat162float(__float2bfloat16_rn(sqrtf(nrm2)));
  const float den = __bfloat162float(__float2bfloat16_rn(nrm + 1e-7f));
  const int row = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int col = blockIdx.x * 256 + (threadIdx.x & 31) * 8;
  if (row >= rr || col >= cc) return;
  __nv_bfloat16* x = a.x + (size_t)mem * a.R_s * a.C_s + (size_t)row * a.C_s + col;
  uint4 u = make_uint4(0, 0, 0, 0);
  if (row < r && col < c) {
    u = *reinterpret_cast<const uint4*>(x);
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      h[e] = (col + e < c) ? __float2bfloat16_rn(__bfloat162float(h[e]) / den) : __float2bfloat16_rn(0.0f);
  }
  *reinterpret_cast<uint4*>(x) = u;
}

// p[o][n] -= lr * scale * U[o][n] for the member's out x in block (U read back through
// the orientation).  Same tiling as the prologue.
__global__ void __launch_bounds__(256) muon_apply_kernel(MuonArgs a) {
  __shared__ float tile[32][33];
  const int mem = blockIdx.z;
  const int o0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  const int out_m = a.out_f ? a.out_f[mem] : a.max_out;
  const int in_m = a.in_f ? a.in_f[mem] : a.max_in;
  if (o0 >= out_m || n0 >= in_m || a.active[mem] == 0) return;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const bool tr = out_m > in_m;
  const __nv_bfloat16* x = a.x + (size_t)mem * a.R_s * a.C_s;
  // the four rows' weights are loaded together with the update tile
  float pv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int o = o0 + ty + 8 * k, n = n0 + tx;
    pv[k] = (o < out_m && n < in_m) ? a.p[((size_t)mem * a.max_out + o) * a.max_in + n] : 0.0f;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = ty + 8 * k;
    if (!tr) {
      const int o = o0 + i, n = n0 + tx;
      tile[i][tx] = (o < out_m && n < in_m) ? __bfloat162float(x[(size_t)o * a.C_s + n]) : 0.0f;
    } else {
      const int n = n0 + i, o = o0 + tx;
      tile[tx][i] = (o < out_m && n < in_m) ? __bfloat162float(x[(size_t)n * a.C_s + o]) : 0.0f;
    }
  }
  __syncthreads();
  const float lr = a.lr_pm ? a.lr_pm[mem] : a.lr_s;
  const float sc = a.scale_pm ? a.scale_pm[mem] : a.scale_s;
  const float slr = lr * sc;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = ty + 8 * k;
    const int o = o0 + i, n = n0 + tx;
    if (o < out_m && n < in_m) a.p[((size_t)mem * a.max_out + o) * a.max_in + n] = pv[k] - tile[i][tx] * slr;
  }
}

}  // namespace tp
