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
  float* partial;        // (P, tiles) per-tile sums of squares (fixed-order reduction)
  int tiles;             // ceil(max_out / 32) * ceil(max_in / 128)
  int32_t* rows;         // (P,) r_m
  int32_t* cols;         // (P,) c_m
  int32_t* trans;        // (P,) 1: X = U^T
  int32_t* active;       // (P,) norm2 > 0
  __nv_bfloat16* p_bf16; // optional bf16 copy of p written with the update, or nullptr
  int bf16_rows, bf16_cols;
  const int32_t* n_blocks;  // (P,) depths, or nullptr: members with n_blocks <= block_index have
  int block_index;          //   an exactly zero gradient (depth-gated)
  int gated_zero;           // 1: depth-gated members' momentum is zero as well (their update is zero)
};

__device__ __forceinline__ bool muon_gated(const MuonArgs& a, int mem) {
  return a.n_blocks != nullptr && __ldg(a.n_blocks + mem) <= a.block_index;
}

__global__ void muon_geometry_kernel(MuonArgs a) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= a.P) return;
  const int o = a.out_f ? a.out_f[m] : a.max_out;
  const int n = a.in_f ? a.in_f[m] : a.max_in;
  a.rows[m] = min(o, n);
  a.cols[m] = max(o, n);
  a.trans[m] = o > n ? 1 : 0;
}

// Dense lists of the Newton-Schulz launches' MMA tiles (BN = 256 columns by TM = 128 rows on
// single CTAs, 256 rows on CTA pairs): rr for the r x r product B = b A + c A^2, rc for the
// r x c update X <- a X + B X, and sym for the symmetric r x r product A = X X^T: only the tiles
// not entirely below the diagonal (n-tile nt, m-tile mt with TM mt < 256 nt + 256); the epilogue
// writes the others as transposes.  Entry = member << 16 | n-tile << 8 | m-tile (in TM rows); a
// member's tiles go column block by column block, down the rows within one.  Members whose
// update is zero (active == 0) have none.  One block of 1024 threads scans the members in
// chunks; list j (j = 0..5: rr, rc, sym with TM = 128, then with TM = 256) gets counts[j].
constexpr int NS_TILE_M = 128, NS_TILE_N = 256;
constexpr int NS_LISTS = 6;

struct NsTileLists {
  uint32_t* list[NS_LISTS];
  int* counts;
  int build[2];  // write the lists of 128-row (build[0]) / 256-row (build[1]) tiles (lengths always)
};

__device__ __forceinline__ int ns_sym_mtiles(int nt, int mt_all, int tm) {
  return min(mt_all, (nt + 1) * (NS_TILE_N / tm));
}

__global__ void __launch_bounds__(1024) ns_tile_list_kernel(MuonArgs a, NsTileLists L) {
  __shared__ int wsum[NS_LISTS][32];
  __shared__ int base[NS_LISTS];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid < NS_LISTS) base[tid] = 0;
  __syncthreads();
  for (int m0 = 0; m0 < a.P; m0 += 1024) {
    const int m = m0 + tid;
    int v[NS_LISTS] = {0, 0, 0, 0, 0, 0};
    int mt[2] = {0, 0}, nrr = 0;
    if (m < a.P && a.active[m] != 0) {
      const int r = a.rows[m], c = a.cols[m];
      nrr = (r + NS_TILE_N - 1) / NS_TILE_N;
      const int nrc = (c + NS_TILE_N - 1) / NS_TILE_N;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const int tm = NS_TILE_M << g;
        mt[g] = (r + tm - 1) / tm;
        v[3 * g] = mt[g] * nrr;
        v[3 * g + 1] = mt[g] * nrc;
        for (int nt = 0; nt < nrr; ++nt) v[3 * g + 2] += ns_sym_mtiles(nt, mt[g], tm);
      }
    }
    int incl[NS_LISTS];
#pragma unroll
    for (int j = 0; j < NS_LISTS; ++j) incl[j] = v[j];
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
#pragma unroll
      for (int j = 0; j < NS_LISTS; ++j) {
        const int o = __shfl_up_sync(0xFFFFFFFFu, incl[j], d);
        if (lane >= d) incl[j] += o;
      }
    }
    if (lane == 31) {
#pragma unroll
      for (int j = 0; j < NS_LISTS; ++j) wsum[j][wid] = incl[j];
    }
    __syncthreads();
    if (wid == 0) {
#pragma unroll
      for (int j = 0; j < NS_LISTS; ++j) {
        int x = wsum[j][lane];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int o = __shfl_up_sync(0xFFFFFFFFu, x, d);
          if (lane >= d) x += o;
        }
        wsum[j][lane] = x;  // inclusive over warps
      }
    }
    __syncthreads();
    int off[NS_LISTS];
#pragma unroll
    for (int j = 0; j < NS_LISTS; ++j) off[j] = base[j] + (wid > 0 ? wsum[j][wid - 1] : 0) + incl[j] - v[j];
    const uint32_t mk = (uint32_t)m << 16;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      if (!L.build[g]) continue;
      const int tm = NS_TILE_M << g, mtg = max(mt[g], 1);
      uint32_t* rr = L.list[3 * g];
      uint32_t* rc = L.list[3 * g + 1];
      uint32_t* sym = L.list[3 * g + 2];
      for (int i = 0; i < v[3 * g]; ++i) rr[off[3 * g] + i] = mk | ((uint32_t)(i / mtg) << 8) | (uint32_t)(i % mtg);
      for (int i = 0; i < v[3 * g + 1]; ++i)
        rc[off[3 * g + 1] + i] = mk | ((uint32_t)(i / mtg) << 8) | (uint32_t)(i % mtg);
      for (int nt = 0, o = off[3 * g + 2]; nt < nrr && v[3 * g + 2] > 0; ++nt)
        for (int t = 0; t < ns_sym_mtiles(nt, mt[g], tm); ++t) sym[o++] = mk | ((uint32_t)nt << 8) | (uint32_t)t;
    }
    __syncthreads();
    if (tid < NS_LISTS) base[tid] += wsum[tid][31];
    __syncthreads();
  }
  if (tid < NS_LISTS) L.counts[tid] = base[tid];
}

// Tiles of the Muon elementwise kernels: 32 weight rows (o) x 128 weight columns (n), 256
// threads; warp w takes rows w, w + 8, w + 16, w + 24 and lane l columns l, l + 32, l + 64,
// l + 96, so each load instruction covers 128 contiguous bytes and a thread has 16 elements
// (32 loads in the prologue) in flight.
constexpr int MUON_TM = 32, MUON_TN = 128;
constexpr int MUON_NORM_ROWS = 64;  // rows of a normalisation block
constexpr int MUON_UB_LD = MUON_TN + 8;  // bf16 staging row (16-byte aligned rows)

// The oriented operand X of the tile (o0, n0) from / to the staged bf16 update ub[o][n]:
// X[o][n] = U when the member is not transposed (rows of 8-byte pieces), X[n][o] = U otherwise
// (rows of 64 bytes, two 32-byte halves per thread).
__device__ __forceinline__ void muon_store_x(__nv_bfloat16* x, int C_s, bool tr, int o0, int n0,
                                             const __nv_bfloat16 (*ub)[MUON_UB_LD]) {
  const int t = threadIdx.x;
  if (!tr) {
    const int c4 = 4 * (t & 31);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (t >> 5) + 8 * i;
      *reinterpret_cast<uint2*>(x + (size_t)(o0 + r) * C_s + n0 + c4) = *reinterpret_cast<const uint2*>(&ub[r][c4]);
    }
  } else {
    const int nl = t >> 1, h = 16 * (t & 1);
    __align__(16) __nv_bfloat16 v[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = ub[h + e][nl];
    uint4* dst = reinterpret_cast<uint4*>(x + (size_t)(n0 + nl) * C_s + o0 + h);
    dst[0] = reinterpret_cast<const uint4*>(v)[0];
    dst[1] = reinterpret_cast<const uint4*>(v)[1];
  }
}

__device__ __forceinline__ void muon_load_x(const __nv_bfloat16* x, int C_s, bool tr, int o0, int n0,
                                            __nv_bfloat16 (*ub)[MUON_UB_LD]) {
  const int t = threadIdx.x;
  if (!tr) {
    const int c4 = 4 * (t & 31);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (t >> 5) + 8 * i;
      *reinterpret_cast<uint2*>(&ub[r][c4]) = *reinterpret_cast<const uint2*>(x + (size_t)(o0 + r) * C_s + n0 + c4);
    }
  } else {
    const int nl = t >> 1, h = 16 * (t & 1);
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(n0 + nl) * C_s + o0 + h);
    __align__(16) __nv_bfloat16 v[16];
    reinterpret_cast<uint4*>(v)[0] = src[0];
    reinterpret_cast<uint4*>(v)[1] = src[1];
#pragma unroll
    for (int e = 0; e < 16; ++e) ub[h + e][nl] = v[e];
  }
}

// Grid: (ceil(max_in / 128), ceil(max_out / 32), P).  Momentum (lerp toward the gradient),
// Nesterov, the bf16 update into the oriented operand (tiles wholly outside the member's
// out x in block are never read nor written; the rest of a partly covered tile gets zeros,
// which the normalisation keeps), and the tile's sum of squares of the bf16 update.  Weight
// decay is applied with the update in muon_apply_kernel.
__global__ void __launch_bounds__(256) muon_prologue_kernel(MuonArgs a) {
  __shared__ __align__(16) __nv_bfloat16 ub[MUON_TM][MUON_UB_LD];
  __shared__ float red[8];
  const int mem = blockIdx.z;
  const int o0 = blockIdx.y * MUON_TM, n0 = blockIdx.x * MUON_TN;
  const int out_m = a.out_f ? a.out_f[mem] : a.max_out;
  const int in_m = a.in_f ? a.in_f[mem] : a.max_in;
  if (o0 >= out_m || n0 >= in_m) return;  // padding: never read, never written
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const float mu = a.mu_pm ? a.mu_pm[mem] : a.mu_s;
  const float one_m_mu = a.mu_pm ? 1.0f - mu : a.one_m_mu_s;
  // a depth-gated member's gradient is exactly zero: it is not read, and its momentum is
  // written back only where it changes (nowhere once it is zero)
  const bool gated = muon_gated(a, mem);
  if (gated && a.gated_zero) {
    // its momentum is zero too, so its update is: nothing to read or write but this tile's
    // (zero) norm partial; the member stays inactive and its operand is never read
    if (threadIdx.x == 0) a.partial[(size_t)mem * a.tiles + blockIdx.y * gridDim.x + blockIdx.x] = 0.0f;
    return;
  }
  float gv[4][4], mv[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int o = o0 + w + 8 * i, n = n0 + lane + 32 * c;
      const bool ok = o < out_m && n < in_m;
      const size_t idx = ((size_t)mem * a.max_out + o) * a.max_in + n;
      gv[i][c] = (ok && !gated) ? a.g[idx] : 0.0f;
      mv[i][c] = ok ? a.m[idx] : 0.0f;
    }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int o = o0 + w + 8 * i, n = n0 + lane + 32 * c;
      __nv_bfloat16 ubv = __float2bfloat16_rn(0.0f);
      if (o < out_m && n < in_m) {
        const size_t idx = ((size_t)mem * a.max_out + o) * a.max_in + n;
        const float m = lerp_t(mv[i][c], gv[i][c], one_m_mu);
        const float u = a.nesterov ? lerp_t(gv[i][c], m, mu) : m;
        if (!gated || __float_as_uint(m) != __float_as_uint(mv[i][c])) a.m[idx] = m;
        if (a.nesterov && a.mutate_grad && (!gated || __float_as_uint(u) != 0u)) a.g[idx] = u;
        ubv = __float2bfloat16_rn(u);
        const float ub_f = __bfloat162float(ubv);
        ss += ub_f * ub_f;
      }
      ub[w + 8 * i][lane + 32 * c] = ubv;
    }
  // Frobenius norm of the bf16 update: this tile's partial, reduced in a fixed order
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
  if (lane == 0) red[w] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < 8; ++i) t += red[i];
    a.partial[(size_t)mem * a.tiles + blockIdx.y * gridDim.x + blockIdx.x] = t;
  }
  muon_store_x(a.x + (size_t)mem * a.R_s * a.C_s, a.C_s, out_m > in_m, o0, n0, ub);
}

// norm2[m] = sum of the member's tile partials in a fixed order (deterministic),
// active[m] = norm2[m] > 0.  One block per member.
__global__ void __launch_bounds__(256) muon_norm_kernel(MuonArgs a, int tiles_x) {
  __shared__ float red[256];
  const int mem = blockIdx.x;
  const int out_m = a.out_f ? a.out_f[mem] : a.max_out;
  const int in_m = a.in_f ? a.in_f[mem] : a.max_in;
  const int ty_n = (out_m + MUON_TM - 1) / MUON_TM, tx_n = (in_m + MUON_TN - 1) / MUON_TN;  // tiles the prologue wrote
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
// along K).  Grid: (ceil(C_s / 256), ceil(R_s / MUON_NORM_ROWS), P), 256 threads; warp w covers
// rows w, w + 8, ... of the block's MUON_NORM_ROWS, a lane 8 columns (16 bytes) of each.
// x / den from rcp = 1 / den (correctly rounded) with one fused correction step: q = x * rcp,
// then q + (x - q den) * rcp.  Markstein's method (P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): the
// residual x - q den is exact in one FMA, and the corrected fp32 quotient is within one ulp of
// x / den (it differs from the correctly rounded one for about 0.24 % of bf16 operand pairs).
// The normalisation stores the quotient in bf16, and there the results equal bf16(x / den) bit
// for bit: `tp_quotient_check` compares them with CUDA's correctly rounded division for every
// bf16 operand pair the normalisation can see.
__device__ __forceinline__ float quotient_from_reciprocal(float x, float den, float rcp) {
  const float q = x * rcp;
  // a zero dividend keeps its sign, as in x / den (the correction would add +0 to -0)
  return x == 0.0f ? x : fmaf(fmaf(-q, den, x), rcp, q);
}

// Exhaustive check of quotient_from_reciprocal against __fdiv_rn: block (bx, by) takes the
// positive bf16 divisor with bit pattern den_first + by and a stride of the 65536 bf16
// dividend patterns; pairs with a non-finite dividend or |x| > 2 den (outside what the
// normalisation divides: an element by its matrix's norm) are skipped.  counts[0] += fp32
// results that differ in any bit, counts[1] += results that differ after rounding to bf16,
// counts[2] += pairs checked, counts[3] += fp32 differences where the exact quotient or the
// reciprocal is subnormal.
__global__ void __launch_bounds__(256) quotient_check_kernel(int den_first, unsigned long long* counts) {
  const unsigned short dbits = (unsigned short)(den_first + blockIdx.y);
  const float den = __uint_as_float((unsigned)dbits << 16);
  const float rcp = 1.0f / den;
  unsigned long long m32 = 0, m16 = 0, n = 0, sub = 0;
  for (unsigned xb = blockIdx.x * blockDim.x + threadIdx.x; xb < 65536u; xb += gridDim.x * blockDim.x) {
    const float x = __uint_as_float(xb << 16);
    if (!isfinite(x) || fabsf(x) > 2.0f * den) continue;
    const float a = quotient_from_reciprocal(x, den, rcp);
    const float b = __fdiv_rn(x, den);
    m32 += __float_as_uint(a) != __float_as_uint(b);
    sub += (__float_as_uint(a) != __float_as_uint(b)) && (fabsf(b) < 1.17549435e-38f || fabsf(rcp) < 1.17549435e-38f);
    m16 += __bfloat16_as_ushort(__float2bfloat16_rn(a)) != __bfloat16_as_ushort(__float2bfloat16_rn(b));
    ++n;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m32 += __shfl_xor_sync(0xffffffffu, m32, o);
    m16 += __shfl_xor_sync(0xffffffffu, m16, o);
    n += __shfl_xor_sync(0xffffffffu, n, o);
    sub += __shfl_xor_sync(0xffffffffu, sub, o);
  }
  if ((threadIdx.x & 31) == 0) {
    if (m32) atomicAdd(counts + 0, m32);
    if (m16) atomicAdd(counts + 1, m16);
    atomicAdd(counts + 2, n);
    if (sub) atomicAdd(counts + 3, sub);
  }
}

__global__ void __launch_bounds__(256) muon_normalize_kernel(MuonArgs a, int row_pad, int col_pad) {
  const int mem = blockIdx.z;
  const int r = a.rows[mem], c = a.cols[mem];
  const int rr = min(a.R_s, (r + row_pad - 1) / row_pad * row_pad);
  const int cc = min(a.C_s, (c + col_pad - 1) / col_pad * col_pad);
  const int row0 = blockIdx.y * MUON_NORM_ROWS;
  const int col = blockIdx.x * 256 + (threadIdx.x & 31) * 8;
  if (row0 >= rr || col >= cc) return;
  const float nrm2 = a.norm2[mem];
  if (nrm2 == 0.0f) return;  // all-zero update: Newton-Schulz is skipped for this member
  const float nrm = __bfloat162float(__float2bfloat16_rn(sqrtf(nrm2)));
  const float den = __bfloat162float(__float2bfloat16_rn(nrm + 1e-7f));
  // x / den per element from one division per thread (quotient_from_reciprocal)
  const float rcp = 1.0f / den;
  constexpr int RPT = MUON_NORM_ROWS / 8;  // rows per thread, all loaded before any is written
  uint4 u[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int row = row0 + (threadIdx.x >> 5) + 8 * i;
    u[i] = make_uint4(0, 0, 0, 0);
    if (row < r && col < c) u[i] = *reinterpret_cast<const uint4*>(a.x + (size_t)mem * a.R_s * a.C_s + (size_t)row * a.C_s + col);
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int row = row0 + (threadIdx.x >> 5) + 8 * i;
    if (row >= rr) continue;
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&u[i]);
    if (row < r) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (col + e < c) {
          h[e] = __float2bfloat16_rn(quotient_from_reciprocal(__bfloat162float(h[e]), den, rcp));
        } else {
          h[e] = __float2bfloat16_rn(0.0f);
        }
    }
    *reinterpret_cast<uint4*>(a.x + (size_t)mem * a.R_s * a.C_s + (size_t)row * a.C_s + col) = u[i];
  }
}

// p <- p * (1 - lr wd) - lr * scale * U over the member's out x in block (weight decay first,
// rounded, as the reference's separate in-place steps; U read back through the orientation;
// members whose update was all zero take the weight decay alone).  Same tiling as the
// prologue.
__global__ void __launch_bounds__(256) muon_apply_kernel(MuonArgs a) {
  __shared__ __align__(16) __nv_bfloat16 ub[MUON_TM][MUON_UB_LD];
  const int mem = blockIdx.z;
  const int o0 = blockIdx.y * MUON_TM, n0 = blockIdx.x * MUON_TN;
  const int out_m = a.out_f ? a.out_f[mem] : a.max_out;
  const int in_m = a.in_f ? a.in_f[mem] : a.max_in;
  if (o0 >= out_m || n0 >= in_m) return;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const bool active = a.active[mem] != 0;
  const bool gated = muon_gated(a, mem);  // its rows of the bf16 copy are not read (depth-gated)
  float pv[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int o = o0 + w + 8 * i, n = n0 + lane + 32 * c;
      pv[i][c] = (o < out_m && n < in_m) ? a.p[((size_t)mem * a.max_out + o) * a.max_in + n] : 0.0f;
    }
  if (active) muon_load_x(a.x + (size_t)mem * a.R_s * a.C_s, a.C_s, out_m > in_m, o0, n0, ub);
  __syncthreads();
  const float lr = a.lr_pm ? a.lr_pm[mem] : a.lr_s;
  // 1 - lr * wd and lr * scale as the reference's per-member tensor ops round them (one rounding
  // each; intrinsics keep the compiler from fusing them), the update as addcmul's
  // fma(-update, lr * scale, p)
  const float mult =
      (a.lr_pm || a.wd_pm) ? __fsub_rn(1.0f, __fmul_rn(lr, a.wd_pm ? a.wd_pm[mem] : a.wd_s)) : a.wd_mult_s;
  const float sc = a.scale_pm ? a.scale_pm[mem] : a.scale_s;
  const float slr = __fmul_rn(lr, sc);
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int o = o0 + w + 8 * i, n = n0 + lane + 32 * c;
      if (o < out_m && n < in_m) {
        const float pw = a.wd_on ? __fmul_rn(pv[i][c], mult) : pv[i][c];
        const float u = active ? __bfloat162float(ub[w + 8 * i][lane + 32 * c]) : 0.0f;
        const float pn = __fmaf_rn(-u, slr, pw);
        a.p[((size_t)mem * a.max_out + o) * a.max_in + n] = pn;
        if (a.p_bf16 != nullptr && !gated)
          a.p_bf16[((size_t)mem * a.bf16_rows + o) * a.bf16_cols + n] = __float2bfloat16_rn(pn);
      }
    }
}

}  // namespace tp
