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
  // host-precomputed values (the reference computes them in Python double precision)
  int wd_on;               // 0: `_make_weight_decay_multiplier` returned None
  float wd_mult_s;         // 1 - lr*wd (all scalar)
  float one_m_b1_s, one_m_b2_s;
  int bc1_scalar;          // beta1 and step scalar: bc1_s holds 1 - beta1^step
  int bc2_scalar;          // beta2 and step scalar: sqrt_bc2_s holds sqrt(1 - beta2^step)
  float bc1_s;             // 1 - beta1^step
  float step_size_s;       // lr / (1 - beta1^step), used iff lr also scalar
  float sqrt_bc2_s;        // sqrt(1 - beta2^step)
  int64_t step;
};

__device__ __forceinline__ float lerp_t(float a, float b, float w) {
  // torch's lerp: a + w (b - a) for |w| < 0.5, else b - (b - a)(1 - w), each as one fused
  // multiply-add (fma(w, d, a) or fma(w - 1, d, b)) as torch's CPU kernel forms it; explicit
  // intrinsics so that the compiler fuses nothing else
  const float d = __fsub_rn(b, a);
  return fabsf(w) < 0.5f ? __fmaf_rn(w, d, a) : __fmaf_rn(__fsub_rn(w, 1.0f), d, b);
}

struct AdamWTensors {
  tp_opt_tensor t[TP_MAX_OPT_TENSORS];
};

// One element's AdamW update with its member's coefficients, rounded step by step as the
// reference's torch ops round (src/tabpackage/optim.py:400-427 on the CPU): each op's result
// is rounded to fp32; torch's lerp is one fused multiply-add, fma(w or w - 1, end - self,
// self or end); addcmul is fma(value * t1, t2, self); addcdiv is self + (value * t1) / t2.
// The intrinsics keep the compiler from fusing anything else.
struct AdamWMember {
  float mult, one_m_b1, b2, one_m_b2, step_size, sqrt_bc2, eps;
  bool wd_on, b2_pm, step_float;
};

__device__ __forceinline__ void adamw_elem(const AdamWMember& c, float& p, float g, float& mm, float& v) {
  if (c.wd_on) p = __fmul_rn(p, c.mult);                                   // p.mul_(1 - lr * wd)
  mm = lerp_t(mm, g, c.one_m_b1);                                       // exp_avg.lerp_(grad, 1 - beta1)
  if (c.b2_pm)
    v = lerp_t(v, __fmul_rn(g, g), c.one_m_b2);                         // exp_avg_sq.lerp_(grad^2, 1 - beta2)
  else
    v = __fmaf_rn(__fmul_rn(c.one_m_b2, g), g, __fmul_rn(v, c.b2));         // .mul_(beta2).addcmul_(g, g, 1 - beta2)
  const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), c.sqrt_bc2), c.eps);
  if (c.step_float)
    p = __fadd_rn(p, __fdiv_rn(__fmul_rn(-c.step_size, mm), denom));       // p.addcdiv_(m, denom, -step)
  else
    p = __fsub_rn(p, __fmul_rn(__fdiv_rn(mm, denom), c.step_size));         // p.add_((m / denom) * step, alpha=-1)
}

// Grid: (chunks of a member's elements, members, tensors), 256 threads.  Member m =
// member0 + blockIdx.y of tensor blockIdx.z owns elements [m * inner, (m + 1) * inner); its
// coefficients are formed once per thread, and 16-byte loads (four elements) keep enough
// bytes in flight when inner is a multiple of 4.
__global__ void __launch_bounds__(256) adamw_kernel(const AdamWTensors ts, const AdamWScalars s, int member0) {
  const tp_opt_tensor& T = ts.t[blockIdx.z];
  const int64_t inner = T.inner;
  const int m = member0 + (int)blockIdx.y;
  const int64_t base = (int64_t)m * inner;
  if (base >= T.numel) return;
  const float lr = s.lr ? s.lr[m] : s.lr_s;
  const float b1 = s.beta1 ? s.beta1[m] : s.beta1_s;
  const float b2 = s.beta2 ? s.beta2[m] : s.beta2_s;
  AdamWMember c;
  c.eps = s.eps ? s.eps[m] : s.eps_s;
  c.wd_on = s.wd_on != 0;
  // 1 - lr * wd as torch forms it from per-member tensors (two roundings), or the host's
  c.mult = (s.lr || s.wd) ? __fsub_rn(1.0f, __fmul_rn(lr, s.wd ? s.wd[m] : s.wd_s)) : s.wd_mult_s;
  c.one_m_b1 = s.beta1 ? __fsub_rn(1.0f, b1) : s.one_m_b1_s;
  c.b2_pm = s.beta2 != nullptr;
  c.b2 = b2;
  c.one_m_b2 = s.beta2 ? __fsub_rn(1.0f, b2) : s.one_m_b2_s;
  const bool step_scalar = T.step == nullptr;
  const float st = (float)(step_scalar ? s.step : T.step[m]);
  // step_size is a Python float in the reference iff lr, beta1 and the step are scalars
  c.step_float = !s.lr && s.bc1_scalar && step_scalar;
  if (c.step_float)
    c.step_size = s.step_size_s;
  else if (s.bc1_scalar && step_scalar)
    c.step_size = __fdiv_rn(lr, s.bc1_s);
  else
    c.step_size = __fdiv_rn(lr, __fsub_rn(1.0f, powf(b1, st)));
  c.sqrt_bc2 = (s.bc2_scalar && step_scalar) ? s.sqrt_bc2_s : __fsqrt_rn(__fsub_rn(1.0f, powf(b2, st)));
  float* P = T.p + base;
  const float* G = T.grad + base;
  float* M = T.exp_avg + base;
  float* V = T.exp_avg_sq + base;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t len = min(inner, T.numel - base);  // the last member of a ragged tensor may be short
  const bool vec = ((inner | len) & 3) == 0 && ((reinterpret_cast<uintptr_t>(T.p) | reinterpret_cast<uintptr_t>(T.grad) |
                                         reinterpret_cast<uintptr_t>(T.exp_avg) |
                                         reinterpret_cast<uintptr_t>(T.exp_avg_sq)) & 15u) == 0;
  if (vec) {
    const int64_t n4 = len >> 2;
    for (int64_t i = t0; i < n4; i += stride) {
      float4 p = reinterpret_cast<const float4*>(P)[i];
      const float4 g = __ldg(reinterpret_cast<const float4*>(G) + i);
      float4 mm = reinterpret_cast<const float4*>(M)[i];
      float4 v = reinterpret_cast<const float4*>(V)[i];
      adamw_elem(c, p.x, g.x, mm.x, v.x);
      adamw_elem(c, p.y, g.y, mm.y, v.y);
      adamw_elem(c, p.z, g.z, mm.z, v.z);
      adamw_elem(c, p.w, g.w, mm.w, v.w);
      reinterpret_cast<float4*>(P)[i] = p;
      reinterpret_cast<float4*>(M)[i] = mm;
      reinterpret_cast<float4*>(V)[i] = v;
    }
  } else {
    for (int64_t i = t0; i < len; i += stride) {
      float p = P[i], mm = M[i], v = V[i];
      adamw_elem(c, p, G[i], mm, v);
      P[i] = p;
      M[i] = mm;
      V[i] = v;
    }
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
