// Memory-bound kernels of the packed linear layer and the AdamW optimizer pack.
#pragma once

#include "gemm_simt.cuh"

namespace tp {

// ---------------------------------------------------------------------------
// Activation backward + bias gradient.
//   g[m, r, c]  = dy * (relu ? [y > 0] : 1) * (dropout ? keep(m,r,c) / p_keep : 1)
//                 for active members and c < out_m; 0 elsewhere (only the 64-column
//                 strips that the dgrad kernel reads are written)
//   dbias[m, c] = sum_r g[m, r, c]
// With relu on, [y > 0] already implies the element was kept, so the mask is
// only regenerated from Philox when dropout follows a plain linear layer.
// Grid: (ceil(W / 64), P); 256 threads = 8 column groups of 8 x 32 row lanes.
// ---------------------------------------------------------------------------
struct ActBwdArgs {
  int P, B, W;                // W = storage width of dy / y / g
  const int32_t* out_f;
  const int32_t* n_blocks;
  int block_index;
  int relu;
  const float* dropout_p;
  uint32_t k0, k1, offset, member_base;
  const void* dy;
  const void* y;
  void* g;                    // nullptr: do not write g (it equals dy)
  float* dbias;
  int db_cols;
};

template <typename T, bool VEC>
__global__ void __launch_bounds__(256) act_backward_kernel(const ActBwdArgs a) {
  __shared__ float red[32][65];
  const int m = blockIdx.y;
  const int strip = blockIdx.x * 64;
  const int cg = threadIdx.x & 7;
  const int rl = threadIdx.x >> 3;
  const int c0 = strip + cg * 8;
  const int out_m = a.out_f ? a.out_f[m] : a.W;
  const bool active = a.n_blocks == nullptr || a.n_blocks[m] > a.block_index;
  const bool live = active && strip < out_m;
  float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int a_rows_done = rl;  // first row of this thread's generic loop
  if (live) {
    float scale = 1.0f;
    uint32_t thr = 65536u;
    if (a.dropout_p) {
      scale = keep_scale(a.dropout_p[m]);
      thr = keep_threshold(a.dropout_p[m]);
    }
    const bool regen = (!a.relu) && a.dropout_p != nullptr && thr < 65536u;
    const T* dy = reinterpret_cast<const T*>(a.dy) + (size_t)m * a.B * a.W;
    const T* y = reinterpret_cast<const T*>(a.y) + (size_t)m * a.B * a.W;
    T* g = a.g ? reinterpret_cast<T*>(a.g) + (size_t)m * a.B * a.W : nullptr;
    if constexpr (VEC && sizeof(T) == 2) {
      if (a.relu && c0 + 8 <= a.W) {
        // bf16 + ReLU (the mask is implied by y > 0): four rows of 16-byte loads in flight
        // per thread before any use, streaming dy / y past L1
        constexpr int U = 4;
        int r0 = rl;
        for (; r0 + 32 * (U - 1) < a.B; r0 += 32 * U) {
          uint4 ud[U], uy[U];
#pragma unroll
          for (int i = 0; i < U; ++i) {
            const size_t off = (size_t)(r0 + 32 * i) * a.W + c0;
            ud[i] = __ldcs(reinterpret_cast<const uint4*>(dy + off));
            uy[i] = __ldcs(reinterpret_cast<const uint4*>(y + off));
          }
#pragma unroll
          for (int i = 0; i < U; ++i) {
            const __nv_bfloat16* hd = reinterpret_cast<const __nv_bfloat16*>(&ud[i]);
            const __nv_bfloat16* hy = reinterpret_cast<const __nv_bfloat16*>(&uy[i]);
            float gv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float v = __bfloat162float(hy[j]) > 0.f ? __bfloat162float(hd[j]) * scale : 0.f;
              if (c0 + j >= out_m) v = 0.f;
              gv[j] = v;
              sum[j] += v;
            }
            if (g) {
              uint4 u;
              u.x = pack_bf16x2(gv[0], gv[1]);
              u.y = pack_bf16x2(gv[2], gv[3]);
              u.z = pack_bf16x2(gv[4], gv[5]);
              u.w = pack_bf16x2(gv[6], gv[7]);
              *reinterpret_cast<uint4*>(g + (size_t)(r0 + 32 * i) * a.W + c0) = u;
            }
          }
        }
        // remaining rows fall through to the generic loop below
        a_rows_done = r0;
      }
    }
    for (int r = a_rows_done; r < a.B; r += 32) {
      float d[8], yy[8];
      const size_t off = (size_t)r * a.W + c0;
      if (VEC && c0 + 8 <= a.W) {
        if (sizeof(T) == 2) {
          const uint4 u = *reinterpret_cast<const uint4*>(dy + off);
          const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
          for (int j = 0; j < 8; ++j) d[j] = __bfloat162float(h[j]);
          if (a.relu) {
            const uint4 v = *reinterpret_cast<const uint4*>(y + off);
            const __nv_bfloat16* hy = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
            for (int j = 0; j < 8; ++j) yy[j] = __bfloat162float(hy[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; j += 4) {
            const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(dy) + off + j);
            d[j] = f.x; d[j + 1] = f.y; d[j + 2] = f.z; d[j + 3] = f.w;
            if (a.relu) {
              const float4 fy = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(y) + off + j);
              yy[j] = fy.x; yy[j + 1] = fy.y; yy[j + 2] = fy.z; yy[j + 3] = fy.w;
            }
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          d[j] = (c0 + j < a.W) ? to_f32<T>(dy[off + j]) : 0.f;
          yy[j] = (a.relu && c0 + j < a.W) ? to_f32<T>(y[off + j]) : 0.f;
        }
      }
      uint32_t bits = 0xFFu;
      if (regen) bits = dropout_bits8(a.k0, a.k1, (uint32_t)(c0 >> 3), (uint32_t)r, a.member_base + (uint32_t)m, a.offset, thr);
      float gv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float v = d[j] * scale;
        if (a.relu) v = yy[j] > 0.f ? v : 0.f;
        if (!((bits >> j) & 1u)) v = 0.f;
        if (c0 + j >= out_m) v = 0.f;
        gv[j] = v;
        sum[j] += v;
      }
      if (g) {
        if (VEC && c0 + 8 <= a.W) {
          if (sizeof(T) == 2) {
            uint4 u;
            u.x = pack_bf16x2(gv[0], gv[1]);
            u.y = pack_bf16x2(gv[2], gv[3]);
            u.z = pack_bf16x2(gv[4], gv[5]);
            u.w = pack_bf16x2(gv[6], gv[7]);
            *reinterpret_cast<uint4*>(g + off) = u;
          } else {
            float* gf = reinterpret_cast<float*>(g) + off;
            *reinterpret_cast<float4*>(gf) = make_float4(gv[0], gv[1], gv[2], gv[3]);
            *reinterpret_cast<float4*>(gf + 4) = make_float4(gv[4], gv[5], gv[6], gv[7]);
          }
        } else {
          for (int j = 0; j < 8; ++j)
            if (c0 + j < a.W) g[off + j] = from_f32<T>(gv[j]);
        }
      }
    }
  }
  if (a.dbias == nullptr) return;
#pragma unroll
  for (int j = 0; j < 8; ++j) red[rl][cg * 8 + j] = sum[j];
  __syncthreads();
  if (threadIdx.x < 64) {
    float s = 0.f;
    for (int i = 0; i < 32; ++i) s += red[i][threadIdx.x];
    const int c = strip + threadIdx.x;
    if (c < a.db_cols) a.dbias[(size_t)m * a.db_cols + c] = s;
  }
}

// ---------------------------------------------------------------------------
// Dropout keep mask (test hook)
// ---------------------------------------------------------------------------
__global__ void dropout_mask_kernel(uint32_t k0, uint32_t k1, uint32_t offset, uint32_t member_base,
                                    const float* p, int P, int B, int C, uint8_t* mask) {
  const long long total_groups = (long long)P * B * ((C + 7) / 8);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total_groups;
       i += (long long)gridDim.x * blockDim.x) {
    const int ng = (C + 7) / 8;
    const int grp = (int)(i % ng);
    const long long mr = i / ng;
    const int r = (int)(mr % B);
    const int m = (int)(mr / B);
    const uint32_t bits =
        dropout_bits8(k0, k1, (uint32_t)grp, (uint32_t)r, member_base + (uint32_t)m, offset, keep_threshold(p[m]));
    for (int j = 0; j < 8; ++j) {
      const int c = grp * 8 + j;
      if (c < C) mask[((size_t)m * B + r) * C + c] = (uint8_t)((bits >> j) & 1u);
    }
  }
}

// ---------------------------------------------------------------------------
// AdamW (decoupled weight decay), per-member hyperparameters.
// ---------------------------------------------------------------------------
struct AdamWScalars {
  // per-member arrays (nullptr -> scalar below)
  const float* lr;
  const float* beta1;
  const float* beta2;
  const float* eps;
  const float* wd;
  float lr_s, beta1_s, beta2_s, eps_s, wd_s;
  // host-precomputed values for the all-scalar case (the reference computes
  // them in Python double precision)
  int wd_on;               // 0: `_make_weight_decay_multiplier` returned None
  float wd_mult_s;         // 1 - lr*wd (all scalar)
  float one_m_b1_s, one_m_b2_s;
  int scalar_bias_corr;    // betas scalar and step scalar
  float bc1_s;             // 1 - beta1^step
  float step_size_s;       // lr / (1 - beta1^step), used iff lr also scalar
  float sqrt_bc2_s;        // sqrt(1 - beta2^step)
  int64_t step;
};

__device__ __forceinline__ float lerp_t(float a, float b, float w) {
  // torch's lerp: a + w (b - a) for |w| < 0.5, else b - (b - a)(1 - w)
  const float d = b - a;
  return fabsf(w) < 0.5f ? a + w * d : b - d * (1.0f - w);
}

struct AdamWTensors {
  tp_opt_tensor t[TP_MAX_OPT_TENSORS];
};

__global__ void __launch_bounds__(256) adamw_kernel(const AdamWTensors ts, const AdamWScalars s) {
  const tp_opt_tensor& T = ts.t[blockIdx.y];
  const int64_t n = T.numel;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / T.inner);
    const float lr = s.lr ? s.lr[m] : s.lr_s;
    const float b1 = s.beta1 ? s.beta1[m] : s.beta1_s;
    const float b2 = s.beta2 ? s.beta2[m] : s.beta2_s;
    const float eps = s.eps ? s.eps[m] : s.eps_s;
    float p = T.p[i];
    const float g = T.grad[i];
    float mm = T.exp_avg[i];
    float v = T.exp_avg_sq[i];
    if (s.wd_on) {
      const float mult = (s.lr || s.wd) ? 1.0f - lr * (s.wd ? s.wd[m] : s.wd_s) : s.wd_mult_s;
      p = p * mult;
    }
    mm = lerp_t(mm, g, s.beta1 ? 1.0f - b1 : s.one_m_b1_s);
    if (s.beta2) {
      v = lerp_t(v, g * g, 1.0f - b2);
    } else {
      v = v * b2;
      v = v + (s.one_m_b2_s * g) * g;
    }
    float step_size, sqrt_bc2;
    if (s.scalar_bias_corr && T.step == nullptr) {
      step_size = s.lr ? lr / s.bc1_s : s.step_size_s;
      sqrt_bc2 = s.sqrt_bc2_s;
    } else {
      const float st = (float)(T.step ? T.step[m] : s.step);
      const float bc1 = 1.0f - powf(b1, st);
      const float bc2 = 1.0f - powf(b2, st);
      step_size = lr / bc1;
      sqrt_bc2 = sqrtf(bc2);
    }
    const float denom = sqrtf(v) / sqrt_bc2 + eps;
    p = p - step_size * (mm / denom);
    T.p[i] = p;
    T.exp_avg[i] = mm;
    T.exp_avg_sq[i] = v;
  }
}


// ---------------------------------------------------------------------------
// bf16 compute copy of an fp32 weight pack: the cast autocast applies to the weight of
// LinearPack.forward (src/tabpackage/nn.py:806-808 under _training.py:161-167), restricted to
// what the grouped GEMMs read.  Member m's rows r < out_m get bf16(w) in the columns c < in_m
// and zeros in [in_m, dst_cols); rows at or beyond out_m and depth-inactive members are not
// written (the GEMMs read them only against exact zeros, so any finite contents do).  A warp
// converts one row: 8 columns per lane, one 16-byte store.
// ---------------------------------------------------------------------------
struct WeightCastArgs {
  int src_rows, src_cols, src_ld, dst_rows, dst_cols;
  const int32_t* out_f;
  const int32_t* in_f;
  const int32_t* n_blocks;
  int block_index;
  const float* src;
  __nv_bfloat16* dst;
};

// Grid: (ceil(src_rows / 8), P), 256 threads.
__global__ void __launch_bounds__(256) weight_cast_kernel(const WeightCastArgs a) {
  const int m = blockIdx.y;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (a.n_blocks != nullptr && __ldg(a.n_blocks + m) <= a.block_index) return;
  const int rows = a.out_f != nullptr ? min(__ldg(a.out_f + m), a.src_rows) : a.src_rows;
  if (r >= rows) return;
  const int cols = a.in_f != nullptr ? min(__ldg(a.in_f + m), a.src_cols) : a.src_cols;
  const float* s = a.src + ((size_t)m * a.src_rows + r) * a.src_ld;
  __nv_bfloat16* d = a.dst + ((size_t)m * a.dst_rows + r) * a.dst_cols;
  for (int c0 = lane * 8; c0 < a.dst_cols; c0 += 256) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = c0 + e < cols ? __ldg(s + c0 + e) : 0.0f;
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(d + c0) = u;
  }
}


// Transposed bf16 copy of a column block of an fp32 weight pack (the one-hot columns of a
// TabPack's first layer, gathered row-wise by onehot_gather_kernel):
// dst[m, j, n] = bf16(src[m, n, col0 + j]) for n < out_m, 0 for out_m <= n < round8(out_m);
// the rest of each dst row is not written (never read).  Tiles of 64 n x 128 j go through
// shared memory so that both the fp32 reads (128-byte pieces along j, 32 loads in flight per
// thread) and the bf16 writes (128-byte pieces along n) are contiguous.
struct WeightCastTArgs {
  int src_rows, src_ld, col0, ncols, dst_ld;
  const int32_t* out_f;
  const float* src;
  __nv_bfloat16* dst;
};

constexpr int CAST_T_N = 64, CAST_T_J = 128;

// Grid: (ceil(ncols / 128), ceil(src_rows / 64), P), 256 threads, 33 KB of dynamic shared memory.
__global__ void __launch_bounds__(256) weight_cast_t_kernel(const WeightCastTArgs a) {
  extern __shared__ float ct_tile[];  // [CAST_T_N][CAST_T_J + 1]
  const int m = blockIdx.z;
  const int j0 = blockIdx.x * CAST_T_J, n0 = blockIdx.y * CAST_T_N;
  const int rows = a.out_f != nullptr ? min(__ldg(a.out_f + m), a.src_rows) : a.src_rows;
  const int rows8 = (rows + 7) & ~7;
  if (n0 >= rows8) return;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const float* s = a.src + (size_t)m * a.src_rows * a.src_ld + a.col0;
  float v[CAST_T_N / 8][CAST_T_J / 32];
#pragma unroll
  for (int ii = 0; ii < CAST_T_N / 8; ++ii) {
    const int n = n0 + w + 8 * ii;
#pragma unroll
    for (int jj = 0; jj < CAST_T_J / 32; ++jj) {
      const int j = j0 + lane + 32 * jj;
      v[ii][jj] = (n < rows && j < a.ncols) ? __ldg(s + (size_t)n * a.src_ld + j) : 0.0f;
    }
  }
#pragma unroll
  for (int ii = 0; ii < CAST_T_N / 8; ++ii)
#pragma unroll
    for (int jj = 0; jj < CAST_T_J / 32; ++jj) ct_tile[(w + 8 * ii) * (CAST_T_J + 1) + lane + 32 * jj] = v[ii][jj];
  __syncthreads();
  __nv_bfloat16* d = a.dst + (size_t)m * a.ncols * a.dst_ld;
  const int n = n0 + 2 * lane;
  for (int jr = w; jr < CAST_T_J; jr += 8) {
    const int j = j0 + jr;
    if (j < a.ncols && n < rows8)
      *reinterpret_cast<uint32_t*>(d + (size_t)j * a.dst_ld + n) =
          pack_bf16x2(ct_tile[2 * lane * (CAST_T_J + 1) + jr], ct_tile[(2 * lane + 1) * (CAST_T_J + 1) + jr]);
  }
}

}  // namespace tp
