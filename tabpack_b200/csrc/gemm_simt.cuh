// CUDA-core path of the packed linear layer: the fp32 mode of the reference
// (no autocast) and shapes the tensor-core path does not take (widths that are
// not multiples of 8).  Same tile kinds and epilogue as the tcgen05 path; one
// CTA per 64x64 tile slot, 4x4 outputs per thread, fp32 accumulation.
#pragma once

#include <type_traits>

#include "linear_problem.cuh"

namespace tp {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// A(r, k) and B(n, k) of C[r, n] = sum_k A(r, k) B(n, k) for member m.
template <typename T, int MODE>
__device__ __forceinline__ float simt_a(const LinearProblem& p, int m, int r, int k, int k_len, int a_rows) {
  if (r >= a_rows || k >= k_len) return 0.0f;
  const T* a = reinterpret_cast<const T*>(p.a_ptr);
  if (MODE == MODE_FWD) {
    const size_t base = p.x_shared ? 0 : (size_t)m * p.B * p.max_in;
    return to_f32<T>(a[base + (size_t)r * p.max_in + k]);
  } else if (MODE == MODE_DGRAD) {
    return to_f32<T>(a[(size_t)m * p.B * p.max_out + (size_t)r * p.max_out + k]);
  } else {
    return to_f32<T>(a[(size_t)m * p.B * p.max_out + (size_t)k * p.max_out + r]);
  }
}

template <typename T, int MODE>
__device__ __forceinline__ float simt_b(const LinearProblem& p, int m, int n, int k, int k_len, int b_rows) {
  if (n >= b_rows || k >= k_len) return 0.0f;
  const T* b = reinterpret_cast<const T*>(p.b_ptr);
  if (MODE == MODE_FWD) {
    return to_f32<T>(b[(size_t)m * p.max_out * p.max_in + (size_t)n * p.max_in + k]);
  } else if (MODE == MODE_DGRAD) {
    return to_f32<T>(b[(size_t)m * p.max_out * p.max_in + (size_t)k * p.max_in + n]);
  } else {
    const size_t base = p.x_shared ? 0 : (size_t)m * p.B * p.max_in;
    return to_f32<T>(b[base + (size_t)k * p.max_in + n]);
  }
}

template <typename T, int MODE>
__global__ void __launch_bounds__(256) linear_gemm_simt(const LinearProblem p) {
  constexpr int TB = 64, TK = 16;
  __shared__ float As[TK][TB + 1];
  __shared__ float Bs[TK][TB + 1];
  const TileInfo ti = decode_tile(p, blockIdx.x, TK);
  const int m = ti.member;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int r0 = ti.mt * TB, c0 = ti.nt * TB;
  using OutT = typename std::conditional<MODE == MODE_WGRAD, float, T>::type;
  OutT* out = reinterpret_cast<OutT*>(p.out) + (size_t)m * p.out_ms;

  if (ti.kind != KIND_MMA) {
    const OutT* src = reinterpret_cast<const OutT*>(p.copy_src) + (size_t)m * p.out_ms;
    for (int i = threadIdx.x; i < TB * TB; i += 256) {
      const int r = r0 + i / TB, c = c0 + i % TB;
      if (r < p.out_rows && c < p.out_cols)
        out[(size_t)r * p.out_ld + c] = (ti.kind == KIND_COPY) ? src[(size_t)r * p.out_ld + c] : from_f32<OutT>(0.f);
    }
    return;
  }
  const int k_len = (p.mode == MODE_FWD) ? (p.in_f ? p.in_f[m] : p.max_in)
                    : (p.mode == MODE_DGRAD) ? (p.out_f ? p.out_f[m] : p.max_out)
                                             : p.B;
  const int a_rows = (MODE == MODE_WGRAD) ? p.max_out : p.B;
  const int b_rows = (MODE == MODE_FWD) ? p.max_out : p.max_in;

  float acc[4][4] = {};
  for (int k0 = 0; k0 < k_len; k0 += TK) {
    for (int i = threadIdx.x; i < TB * TK; i += 256) {
      int rr, kk;
      if (MODE == MODE_WGRAD) {  // contiguous along rows of A / columns of B
        rr = i % TB;
        kk = i / TB;
      } else {
        rr = i / TK;
        kk = i % TK;
      }
      As[kk][rr] = simt_a<T, MODE>(p, m, r0 + rr, k0 + kk, k_len, a_rows);
    }
    for (int i = threadIdx.x; i < TB * TK; i += 256) {
      int nn, kk;
      if (MODE == MODE_FWD) {
        nn = i / TK;
        kk = i % TK;
      } else {
        nn = i % TB;
        kk = i / TB;
      }
      Bs[kk][nn] = simt_b<T, MODE>(p, m, c0 + nn, k0 + kk, k_len, b_rows);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[kk][ty * 4 + i];
        b[i] = Bs[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

  const bool dropout_on = (MODE == MODE_FWD) && p.dropout_p != nullptr;
  uint32_t thr = 65536u;
  float scale = 1.0f;
  if (dropout_on) {
    thr = keep_threshold(p.dropout_p[m]);
    scale = keep_scale(p.dropout_p[m]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty * 4 + i;
    if (r >= p.out_rows) continue;
    const int cb = c0 + tx * 4;
    uint32_t bits = 0xFFu;
    if (dropout_on && thr < 65536u)
      bits = dropout_bits8(p.k0, p.k1, (uint32_t)(cb >> 3), (uint32_t)r, p.member_base + (uint32_t)m, p.offset, thr) >>
             (cb & 7);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = cb + j;
      if (c >= p.out_cols) continue;
      float bias = 0.f;
      if (MODE == MODE_FWD && p.bias != nullptr && c < ti.n_valid) bias = p.bias[(size_t)m * p.bias_ld + c];
      const float v = epilogue_value<MODE>(p, ti, r, c, acc[i][j], bias, (bits >> j) & 1u, scale);
      out[(size_t)r * p.out_ld + c] = from_f32<OutT>(v);
    }
  }
}

}  // namespace tp
