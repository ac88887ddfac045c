// Persistent, warp-specialised ragged grouped GEMM for the packed linear layer on
// sm_100a: TMA (no multicast) fills a ring of shared-memory stages, one thread
// issues tcgen05.mma into a double-buffered TMEM accumulator, and four epilogue
// warps drain TMEM with tcgen05.ld, apply the fused epilogue and store.
//
//   MODE_FWD  : C[B x out_m]  = X[B x in_m]  * W^T          A K-major, B K-major
//   MODE_DGRAD: C[B x in_m]   = G[B x out_m] * W            A K-major, B MN-major
//   MODE_WGRAD: C[out_m x in_m] = G^T * X  (K = batch rows)  A MN-major, B MN-major
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer, warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4) .. +31).
#pragma once

#include "linear_problem.cuh"

namespace tp {

template <int BN_, int MODE>
struct Sm100Cfg {
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int BK = 64;  // one 128-byte swizzle atom of bf16 along K
  static constexpr bool A_MN = (MODE == MODE_WGRAD);
  static constexpr bool B_MN = (MODE != MODE_FWD);
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int NUM_THREADS = 192;
  // stages + barriers (full, empty per stage; tfull, tempty x2; done) + tmem addr + abort
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
};

template <int BN, int MODE>
__global__ void __launch_bounds__(192, 1)
    linear_gemm_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const LinearProblem pr) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using Cfg = Sm100Cfg<BN, MODE>;
  extern __shared__ uint8_t dyn_smem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + Cfg::STAGES * Cfg::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + Cfg::STAGES;
  uint64_t* tfull = bars + 2 * Cfg::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done_bar = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int total_tiles = pr.P * pr.m_tiles * pr.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
        const TileInfo ti = decode_tile(pr, t, Cfg::BK);
        if (ti.kind != KIND_MMA) continue;
        const int zA = (MODE == MODE_FWD && pr.x_shared) ? 0 : ti.member;
        const int zB = (MODE == MODE_WGRAD && pr.x_shared) ? 0 : ti.member;
        for (int kb = 0; kb < ti.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) goto producer_done;
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          uint8_t* a = smA + stage * Cfg::A_BYTES;
          uint8_t* b = smB + stage * Cfg::B_BYTES;
          const int k0 = kb * Cfg::BK;
          if (!Cfg::A_MN) {
            tma_load_3d(a, &tmA, &full[stage], k0, ti.mt * Cfg::BM, zA);
          } else {
#pragma unroll
            for (int c = 0; c < Cfg::BM / 64; ++c)
              tma_load_3d(a + c * 64 * 128, &tmA, &full[stage], ti.mt * Cfg::BM + c * 64, k0, zA);
          }
          if (!Cfg::B_MN) {
            tma_load_3d(b, &tmB, &full[stage], k0, ti.nt * BN, zB);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(b + c * 64 * 128, &tmB, &full[stage], ti.nt * BN + c * 64, k0, zB);
          }
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      const uint32_t idesc = idesc_bf16_f32(BN, Cfg::A_MN, Cfg::B_MN);
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
        const TileInfo ti = decode_tile(pr, t, Cfg::BK);
        if (ti.kind != KIND_MMA) continue;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool aborted = false;
        for (int kb = 0; kb < ti.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smA + stage * Cfg::A_BYTES);
          const uint32_t b_base = smem_u32(smB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {
            const uint64_t adesc = Cfg::A_MN ? smem_desc_sw128(a_base + k * 2048, 64 * 128, 1024)
                                             : smem_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bdesc = Cfg::B_MN ? smem_desc_sw128(b_base + k * 2048, 64 * 128, 1024)
                                             : smem_desc_sw128(b_base + k * 32, 16, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (aborted) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Every MMA issued by this thread has completed once done_bar flips.
      umma_commit(done_bar);
      volatile int no_abort = 0;
      mbar_wait(done_bar, 0, &no_abort);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool dropout_on = (MODE == MODE_FWD) && pr.dropout_p != nullptr;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const TileInfo ti = decode_tile(pr, t, Cfg::BK);
      const int m = ti.member;
      const int row = ti.mt * Cfg::BM + row_in_tile;
      const bool row_ok = row < pr.out_rows;
      const int col_tile = ti.nt * BN;
      if (ti.kind == KIND_MMA) {
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) break;
        tc_fence_after();
        uint32_t thr = 65536u;
        float scale = 1.0f;
        if (dropout_on) {
          const float p = pr.dropout_p[m];
          thr = keep_threshold(p);
          scale = keep_scale(p);
        }
        const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          const int col0 = col_tile + c;
          if (col0 >= pr.out_cols) break;  // warp-uniform
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + (uint32_t)c, r);
          tmem_wait_ld();
          if (!row_ok) continue;
          const int nv = ti.n_valid - col0;  // valid columns in this chunk (may be <= 0)
          float v[32];
          if (MODE == MODE_FWD) {
            uint32_t keep_bits = 0xFFFFFFFFu;
            if (dropout_on && thr < 65536u && nv > 0) {
              keep_bits = 0;
#pragma unroll
              for (int g = 0; g < 4; ++g)
                keep_bits |= dropout_bits8(pr.k0, pr.k1, (uint32_t)(col0 >> 3) + g, (uint32_t)row,
                                           pr.member_base + (uint32_t)m, pr.offset, thr)
                             << (8 * g);
            }
            float bv[32];
            const float* bp = pr.bias ? pr.bias + (size_t)m * pr.bias_ld + col0 : nullptr;
            if (bp != nullptr && nv >= 32 && col0 + 32 <= pr.bias_ld) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 f = __ldg(reinterpret_cast<const float4*>(bp + j));
                bv[j] = f.x; bv[j + 1] = f.y; bv[j + 2] = f.z; bv[j + 3] = f.w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) bv[j] = (bp != nullptr && j < nv) ? __ldg(bp + j) : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float x = __uint_as_float(r[j]) + bv[j];
              if (pr.relu) x = fmaxf(x, 0.0f);
              x = ((keep_bits >> j) & 1u) ? x * scale : 0.0f;
              v[j] = j < nv ? x : 0.0f;
            }
          } else if (MODE == MODE_DGRAD) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = j < nv ? __uint_as_float(r[j]) : 0.0f;
          } else {
            const bool rv = row < ti.m_valid;
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = (rv && j < nv) ? __uint_as_float(r[j]) : 0.0f;
          }
          const int ncols = pr.out_cols - col0;  // storable columns in this chunk (> 0)
          if (MODE == MODE_WGRAD) {
            float* dst = reinterpret_cast<float*>(pr.out) + (size_t)m * pr.out_ms + (size_t)row * pr.out_ld + col0;
            if (ncols >= 32 && (pr.out_ld & 3) == 0) {
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < ncols) dst[j] = v[j];
            }
          } else {
            __nv_bfloat16* dst =
                reinterpret_cast<__nv_bfloat16*>(pr.out) + (size_t)m * pr.out_ms + (size_t)row * pr.out_ld + col0;
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              if (j < ncols) {  // out_cols is a multiple of 8 on this path
                uint4 u;
                u.x = pack_bf16x2(v[j], v[j + 1]);
                u.y = pack_bf16x2(v[j + 2], v[j + 3]);
                u.z = pack_bf16x2(v[j + 4], v[j + 5]);
                u.w = pack_bf16x2(v[j + 6], v[j + 7]);
                *reinterpret_cast<uint4*>(dst + j) = u;
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      } else if (row_ok) {
        // ZERO or COPY block: this thread's row, columns [col_tile, col_tile + BN)
        const int c_end = min(col_tile + BN, pr.out_cols);
        if (MODE == MODE_WGRAD) {
          float* dst = reinterpret_cast<float*>(pr.out) + (size_t)m * pr.out_ms + (size_t)row * pr.out_ld;
          if ((pr.out_ld & 3) == 0) {
            int c = col_tile;
            for (; c + 4 <= c_end; c += 4) *reinterpret_cast<float4*>(dst + c) = make_float4(0.f, 0.f, 0.f, 0.f);
            for (; c < c_end; ++c) dst[c] = 0.0f;
          } else {
            for (int c = col_tile; c < c_end; ++c) dst[c] = 0.0f;
          }
        } else {
          __nv_bfloat16* dst =
              reinterpret_cast<__nv_bfloat16*>(pr.out) + (size_t)m * pr.out_ms + (size_t)row * pr.out_ld;
          if (ti.kind == KIND_ZERO) {
            for (int c = col_tile; c < c_end; c += 8) *reinterpret_cast<uint4*>(dst + c) = make_uint4(0, 0, 0, 0);
          } else {
            const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(pr.copy_src) +
                                       (size_t)m * pr.out_ms + (size_t)row * pr.out_ld;
            for (int c = col_tile; c < c_end; c += 8)
              *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
#endif
}

}  // namespace tp
