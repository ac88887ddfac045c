// Persistent, warp-specialised ragged grouped GEMM for the packed linear layer and the
// Newton-Schulz iterations of Muon on sm_100a: TMA (one destination CTA per load) fills a ring
// of shared-memory stages, one thread issues tcgen05.mma into a double-buffered TMEM
// accumulator, and the epilogue warps drain TMEM with tcgen05.ld, apply the fused epilogue
// and store.
//
//   MODE_FWD    : C[B x out_m] = X[B x in_m] * W^T, + bias, ReLU, Philox dropout; A, B K-major
//   MODE_FWD_ADD: the forward with an fp32 addend E[B x out_m] summed before the bias
//   MODE_FWD_PAIR: the forward on CTA pairs (without dropout, or with a long K loop)
//   MODE_DGRAD  : C[B x in_m] = G[B x out_m] * W; A K-major, B MN-major; CTA pairs
//   MODE_WGRAD_TG: MODE_WGRAD_T on single CTAs with X gathered from a table by row index
//   MODE_WGRAD_T: C^T[in_m x out_m] = X^T * G stored into C (K = batch rows), A and B MN-major;
//                 a warp's 32 lanes hold 32 consecutive input features, so each output
//                 feature's column is one coalesced 128-byte fp32 store; CTA pairs
//   MODE_NS / MODE_NS_BMN: C = alpha * A B^T + beta * D over each member's r x (r|c) block
//                 (B K-major / MN-major); tiles claimed dynamically
//
// Warp roles: warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer, warp 2 = tile
// scheduler (claims and decodes the CTA's tiles ahead of use and publishes them in a
// shared-memory ring that the producer, the MMA thread and the epilogue warps read in order,
// so no per-tile global load or division sits on their critical paths), warps 3.. = epilogue
// (warp w reads TMEM lanes 32*(w%4) .. +31 and column slice (w-3)/4).  The forward runs 16 epilogue warps (four per SM sub-partition: its
// bias + ReLU + Philox epilogue is latency-bound, so four warps per scheduler hide each
// other's dependency stalls) over a 3-stage ring; the other modes run 8 epilogue warps.
#pragma once

#include "linear_problem.cuh"

namespace tp {

template <int BN_, int MODE>
struct Sm100Cfg {
  static constexpr int BM = 128;  // accumulator rows per CTA (TMEM lanes)
  static constexpr int BN = BN_;
  static constexpr int BK = 64;  // one 128-byte swizzle atom of bf16 along K
  // CTA pairs (cta_group::2) for the gradient GEMMs: the pair computes a 256 x BN tile,
  // each CTA stages its own 128 rows of A and half of B's columns, so the operand bytes
  // a CTA loads and its tensor core reads per MMA drop by a third.  The forward, whose
  // time goes to its bias / ReLU / dropout epilogue rather than to operand traffic, runs
  // on single CTAs (measured a few percent faster than on pairs).
  static constexpr bool PAIR = (MODE == MODE_DGRAD || MODE == MODE_WGRAD_T || MODE == MODE_FWD_PAIR ||
                                MODE == MODE_NS_P || MODE == MODE_NS_BMN_P) && BN_ == 256;
  static constexpr bool FWDK = (MODE == MODE_FWD || MODE == MODE_FWD_ADD || MODE == MODE_FWD_PAIR);  // forward epilogue
  static constexpr int TILE_M = PAIR ? 2 * BM : BM;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // B columns staged per CTA
  static constexpr bool A_MN = is_wgrad_t(MODE);
  static constexpr bool B_MN = (MODE == MODE_DGRAD || is_wgrad_t(MODE) || MODE == MODE_NS_BMN || MODE == MODE_NS_BMN_P);
  static constexpr int STAGES = PAIR ? (FWDK ? 5 : 6) : (BN == 256) ? (FWDK ? 3 : 4) : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int EPI_WARPS = FWDK ? 16 : 8;
  static constexpr int EPI_WARP0 = 3;  // first epilogue warp
  static constexpr int NUM_THREADS = 32 * EPI_WARP0 + 32 * EPI_WARPS;
  static constexpr int TRING = 4;      // slots of the decoded-tile ring
  // control block: barriers (full, empty per stage; tfull, tempty x2; done; tile ring full,
  // empty per slot), tmem address, abort flag (first 256 bytes), then the tile ring (8 ints
  // per slot)
  static constexpr int CTRL_BYTES = 512;
  // stages + control block + per-warp bias slice (BN / (EPI_WARPS / 4) floats per epilogue warp)
  static constexpr int BIAS_FLOATS_PER_WARP = BN / (EPI_WARPS / 4);
  // + per-warp staging tile for coalesced bf16 stores (32 rows x 32 columns, rows padded to 80 B)
  static constexpr int STAGE_ROW_BYTES = 80;
  static constexpr int STORE_STAGE_BYTES = 32 * STAGE_ROW_BYTES;
  static constexpr int SMEM_BYTES =
      1024 + STAGES * STAGE_BYTES + CTRL_BYTES + EPI_WARPS * BIAS_FLOATS_PER_WARP * 4 + EPI_WARPS * STORE_STAGE_BYTES;
};

// Forward epilogue of one 16-column chunk (columns col0.., col0 a multiple of 16) of one
// output row: (acc + b) * scale as one fma with the staged b * scale, ReLU (which commutes
// with the positive scale), Philox keep mask, bf16 pack into 32 bytes of the row's staging
// slot.  The chunk's two Philox chains are independent and interleave.
// The chunk's two Philox draws (independent of the accumulator: computed while its TMEM load
// is in flight).
__device__ __forceinline__ void fwd16_draws(const LinearProblem& pr, int m, int row, int col0, bool drop,
                                            uint4 (&q2)[2]) {
  if (drop) {
#pragma unroll
    for (int g = 0; g < 2; ++g)
      q2[g] = philox4x32_10_ks(
          make_uint4((uint32_t)(col0 >> 3) + g, (uint32_t)row, pr.member_base + (uint32_t)m, pr.offset), pr.ks);
  }
}

__device__ __forceinline__ void epi_fwd16(const LinearProblem& pr, const uint32_t (&r)[16], const uint4 (&q2)[2],
                                          int nv, bool drop, uint32_t thr, float scale, const float* sbias,
                                          uint8_t* stage) {
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int gv = nv - 8 * g;  // valid columns in this group of 8
    const float4 b0 = *reinterpret_cast<const float4*>(sbias + 8 * g);
    const float4 b1 = *reinterpret_cast<const float4*>(sbias + 8 * g + 4);
    const float b8[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    const uint32_t w[4] = {q2[g].x, q2[g].y, q2[g].z, q2[g].w};
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float t = fmaf(__uint_as_float(r[8 * g + j]), scale, b8[j]);
      if (pr.relu) t = fmaxf(t, 0.0f);
      if (drop) {
        const uint32_t r16 = (j & 1) ? (w[j >> 1] >> 16) : (w[j >> 1] & 0xFFFFu);
        t = r16 < thr ? t : 0.0f;
      }
      x[j] = t;
    }
    if (gv < 8) {  // ragged last group (warp-uniform): zeros beyond the member's columns
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j >= gv) x[j] = 0.0f;
    }
    uint4 u;
    u.x = pack_bf16x2(x[0], x[1]);
    u.y = pack_bf16x2(x[2], x[3]);
    u.z = pack_bf16x2(x[4], x[5]);
    u.w = pack_bf16x2(x[6], x[7]);
    *reinterpret_cast<uint4*>(stage + 16 * g) = u;
  }
}

// Newton-Schulz addend D (bf16) of one 32-column chunk of one row, zeros outside the
// member's valid columns (`drow` null outside its valid rows or without D).
__device__ __forceinline__ void ns_load_d(const __nv_bfloat16* drow, int col0, int nv, uint4 (&d)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    d[j] = (drow != nullptr && 8 * j < nv) ? *reinterpret_cast<const uint4*>(drow + col0 + 8 * j) : make_uint4(0, 0, 0, 0);
}

// alpha * acc + beta * D of one 32-column chunk (D preloaded), exact zeros outside the
// member's r x (r|c) block, bf16 into the row's staging slot.
__device__ __forceinline__ void ns_chunk(const LinearProblem& pr, bool rv, int nv, const uint32_t (&r)[32],
                                         const uint4 (&d)[4], uint8_t* stage) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&d[j]);
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      v[e] = (rv && 8 * j + e < nv) ? pr.alpha * __uint_as_float(r[8 * j + e]) + pr.beta * __bfloat162float(h[e]) : 0.0f;
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(stage + 16 * j) = u;
  }
}

// dgrad epilogue of one 32-column chunk of one output row held in registers `r` (raw fp32
// accumulator bits from tcgen05.ld): bf16 into the row's staging slot, zeros beyond the
// member's columns.
__device__ __forceinline__ void dgrad_chunk(const TileInfo& ti, int col0, const uint32_t (&r)[32], uint8_t* stage) {
  const int nv = ti.n_valid - col0;  // valid columns in this chunk (may be <= 0)
#pragma unroll
  for (int j = 0; j < 32; j += 8) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = j + e < nv ? __uint_as_float(r[j + e]) : 0.0f;
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(stage + j * 2) = u;
  }
}

// The transpose of a warp's staged 32 x 32 bf16 chunk (rows row_base.., columns col0..): row
// col0 + j of member m's output receives the chunk's column j in its columns row_base..+31 (a
// symmetric product's tile below the diagonal, which is not computed).  Four lanes per output
// row, 16 bytes each: lane l writes rows (l / 4) + 8k, k = 0..3, columns row_base + 8 (l % 4)..+7.
__device__ __forceinline__ void mirror_flush(const LinearProblem& pr, int m, int row_base, int col0,
                                             const uint8_t* stage_warp, int lane, int row_bytes) {
  const int c = lane & 3;
  if (row_base + 8 * c >= pr.out_cols) return;
  __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(pr.out) + (size_t)m * pr.out_ms + row_base + 8 * c;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int jj = (lane >> 2) + 8 * k;
    if (col0 + jj >= pr.out_rows) continue;
    uint32_t v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t lo = *reinterpret_cast<const unsigned short*>(stage_warp + (8 * c + 2 * e) * row_bytes + 2 * jj);
      const uint32_t hi = *reinterpret_cast<const unsigned short*>(stage_warp + (8 * c + 2 * e + 1) * row_bytes + 2 * jj);
      v[e] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(base + (size_t)(col0 + jj) * pr.out_ld) = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

// Writes a warp's staged 32 x 32 bf16 chunk (rows row_base.., columns col0..) to global
// memory with 4 lanes per row (64 contiguous bytes), so one store instruction covers
// 8 rows instead of 32 scattered 16-byte pieces.
__device__ __forceinline__ void stage_flush(const LinearProblem& pr, int m, int row_base, int col0,
                                            const uint8_t* stage_warp, int lane, int row_bytes) {
  const int c = lane & 3;
  if (col0 + 8 * c >= pr.out_cols) return;  // out_cols is a multiple of 8 on this path
  __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(pr.out) + (size_t)m * pr.out_ms + col0 + 8 * c;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = (lane >> 2) + 8 * k;
    const int grow = row_base + r;
    if (grow < pr.out_rows)
      *reinterpret_cast<uint4*>(base + (size_t)grow * pr.out_ld) =
          *reinterpret_cast<const uint4*>(stage_warp + r * row_bytes + c * 16);
  }
}

// Columns a CTA pair multiplies in tile `ti`: the member's remaining columns rounded up
// to 32 (each CTA's half a multiple of 16), at most BN.
template <int BN>
__device__ __forceinline__ int pair_n_mma(const TileInfo& ti) {
  return min(BN, (ti.n_valid - ti.nt * BN + 31) & ~31);
}

// Zeros in columns [c_begin, c_end) of the warp's 32 output rows (bf16, c_begin and c_end
// multiples of 8), lanes along 16-byte pieces so that a store instruction covers whole rows.
__device__ __forceinline__ void zero_fill_bf16(const LinearProblem& pr, int m, int row_base, int c_begin, int c_end,
                                               int lane) {
  __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(pr.out) + (size_t)m * pr.out_ms;
  const int nq = (c_end - c_begin) / 8;
  for (int i = lane; i < 32 * nq; i += 32) {
    const int r = i / nq, cc = c_begin + 8 * (i - r * nq);
    if (row_base + r < pr.out_rows)
      *reinterpret_cast<uint4*>(base + (size_t)(row_base + r) * pr.out_ld + cc) = make_uint4(0, 0, 0, 0);
  }
}

template <int BN, int MODE>
__global__ void __launch_bounds__(Sm100Cfg<BN, MODE>::NUM_THREADS, 1)
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
  constexpr int TRING = Cfg::TRING;
  uint64_t* tr_full = done_bar + 1;        // decoded-tile ring: published by the scheduler warp,
  uint64_t* tr_empty = tr_full + TRING;    //   read by the producer, the MMA thread and every epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tr_empty + TRING);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* tile_ring = reinterpret_cast<volatile int*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES + 256);
  // a pair's claimed tile-list indices, handed from the leader's scheduler to the peer's: CRING
  // slots after the tile ring, with a full barrier (arrived by the leader) and an empty barrier
  // (arrived by the peer) per slot
  constexpr int CRING = 4;
  volatile int* claim_val = tile_ring + 8 * TRING;
  uint64_t* claim_full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES + 256 + 32 * TRING + 16);
  uint64_t* claim_empty = claim_full + CRING;
  static_assert(256 + 32 * TRING + 16 + 16 * CRING <= Cfg::CTRL_BYTES, "control block holds the claim ring");

  const int warp = warp_id();
  const int lane = lane_id();
  const int total_tiles = pr.P * pr.m_tiles * pr.n_tiles;
  constexpr bool PAIR = Cfg::PAIR;
  // persistent tile loop over clusters: a CTA pair takes the same tiles
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tile_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  // With a tile list (single CTAs), tiles are claimed dynamically: ragged members' tiles
  // differ a lot in cost, so claiming them as CTAs free up balances the launch.
  // k-th tile of this CTA for a consumer warp (all its active lanes read; `arrive` frees the
  // slot, once per consumer warp); KIND_END ends the sequence
  auto ring_read = [&](int k, bool arrive) -> TileInfo {
    TileInfo ti;
    const int s = k & (TRING - 1);
    if (!mbar_wait(&tr_full[s], (uint32_t)(k / TRING) & 1u, abort_flag)) {
      ti.kind = KIND_END;
      return ti;
    }
    const volatile int* e = tile_ring + 8 * s;
    ti.member = e[0];
    ti.mt = e[1];
    ti.nt = e[2];
    ti.kind = e[3];
    ti.kblocks = e[4];
    ti.m_valid = e[5];
    ti.n_valid = e[6];
    __syncwarp(__activemask());
    if (arrive) mbar_arrive(&tr_empty[s]);
    return ti;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], PAIR ? 2 * Cfg::EPI_WARPS : Cfg::EPI_WARPS);  // the leader's counts both CTAs
    }
    mbar_init(done_bar, 1);
    if constexpr (PAIR) {
      for (int i = 0; i < CRING; ++i) {
        mbar_init(&claim_full[i], 1);
        mbar_init(&claim_empty[i], 1);
      }
    }
    for (int i = 0; i < TRING; ++i) {
      mbar_init(&tr_full[i], 1);
      // consumers: the producer, the epilogue warps and the MMA thread (a pair's leader only)
      mbar_init(&tr_empty[i], 1 + Cfg::EPI_WARPS + ((!PAIR || rank == 0) ? 1 : 0));
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    else
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && !PAIR && pr.row_index != nullptr) {
    // ------------------------------------------------------------------ producer, gathered A
    // A's rows come from a shared table by row index: each lane gathers four rows per k-block
    // (32 TMA gather4 loads fill the 128 x 64 stage), lane 0 loads B as usual.  Forward (A
    // K-major): lane l takes the tile's rows 4l..4l+3, the same for every k-block.  Transposed
    // weight gradient (A = X^T, MN-major, two 64-feature boxes of 64 batch rows): lane l takes
    // box l / 16 and batch rows 4 (l % 16)..+3 of the k-block.  Rows past the batch gather
    // table row 0: forward outputs of those rows are not stored, and in the weight gradient G
    // is zero there (its rows past the batch load as zeros).
    int stage = 0;
    uint32_t phase = 0;
    auto rows4 = [&](int m, int b0) -> int4 {
      const int32_t* ri = pr.row_index + (size_t)m * pr.B;
      int4 r;
      r.x = b0 < pr.B ? __ldg(ri + b0) : 0;
      r.y = b0 + 1 < pr.B ? __ldg(ri + b0 + 1) : 0;
      r.z = b0 + 2 < pr.B ? __ldg(ri + b0 + 2) : 0;
      r.w = b0 + 3 < pr.B ? __ldg(ri + b0 + 3) : 0;
      return r;
    };
    for (int k = 0;; ++k) {
      const TileInfo ti = ring_read(k, lane == 0);
      if (ti.kind == KIND_END) break;
      if (ti.kind != KIND_MMA) continue;
      int4 fr = make_int4(0, 0, 0, 0);
      if constexpr (!Cfg::A_MN) fr = rows4(ti.member, ti.mt * Cfg::BM + 4 * lane);
      const int a_col = ti.mt * Cfg::BM;  // transposed: the tile's first input feature
      const int b_col = ti.nt * BN;
      for (int kb = 0; kb < ti.kblocks; ++kb) {
        const int k0 = kb * Cfg::BK;
        int4 wr = make_int4(0, 0, 0, 0);
        if constexpr (Cfg::A_MN) wr = rows4(ti.member, k0 + 4 * (lane & 15));
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) goto gather_done;
        if (lane == 0) mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
        __syncwarp();
        uint8_t* a = smA + stage * Cfg::A_BYTES;
        uint8_t* b = smB + stage * Cfg::B_BYTES;
        if constexpr (!Cfg::A_MN)
          tma_gather4(a + lane * 512, &tmA, &full[stage], k0, fr);
        else
          tma_gather4(a + (lane >> 4) * 64 * 128 + (lane & 15) * 512, &tmA, &full[stage], a_col + (lane >> 4) * 64, wr);
        if (lane == 0) {
          if (!Cfg::B_MN) {
            tma_load_3d(b, &tmB, &full[stage], k0, b_col, ti.member);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_3d(b + c * 64 * 128, &tmB, &full[stage], b_col + c * 64, k0, ti.member);
          }
        }
        if (++stage == Cfg::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  gather_done:;
  } else if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int k = 0;; ++k) {
        const TileInfo ti = ring_read(k, true);
        if (ti.kind == KIND_END) break;
        if (ti.kind != KIND_MMA) continue;
        const int zA = ((Cfg::FWDK || is_wgrad_t(MODE)) && pr.x_shared) ? 0 : ti.member;  // NS operands are per member
        const int zB = ti.member;
        // this CTA's A rows and B columns: in a pair the leader takes rows 0..127 and the
        // first half of the (trimmed) columns, the peer rows 128..255 and the second half
        const int a_row = ti.mt * Cfg::TILE_M + (int)rank * Cfg::BM;
        const int b_col = ti.nt * BN + (PAIR ? (int)rank * (pair_n_mma<BN>(ti) / 2) : 0);
        for (int kb = 0; kb < ti.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) goto producer_done;
          uint8_t* a = smA + stage * Cfg::A_BYTES;
          uint8_t* b = smB + stage * Cfg::B_BYTES;
          const int k0 = kb * Cfg::BK;
          if constexpr (PAIR) {
            // both CTAs' bytes complete on the leader's full barrier
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            if (!Cfg::A_MN) {
              tma_load_3d_pair(a, &tmA, fb, k0, a_row, zA);
            } else {
#pragma unroll
              for (int c = 0; c < Cfg::BM / 64; ++c) tma_load_3d_pair(a + c * 64 * 128, &tmA, fb, a_row + c * 64, k0, zA);
            }
            if (!Cfg::B_MN) {
              tma_load_3d_pair(b, &tmB, fb, k0, b_col, zB);
            } else {
#pragma unroll
              for (int c = 0; c < Cfg::B_ROWS / 64; ++c) tma_load_3d_pair(b + c * 64 * 128, &tmB, fb, b_col + c * 64, k0, zB);
            }
          } else {
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          if (!Cfg::A_MN) {
            tma_load_3d(a, &tmA, &full[stage], k0, a_row, zA);
          } else {
#pragma unroll
            for (int c = 0; c < Cfg::BM / 64; ++c)
              tma_load_3d(a + c * 64 * 128, &tmA, &full[stage], a_row + c * 64, k0, zA);
          }
          if (!Cfg::B_MN) {
            tma_load_3d(b, &tmB, &full[stage], k0, b_col, zB);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(b + c * 64 * 128, &tmB, &full[stage], b_col + c * 64, k0, zB);
          }
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
    // (in a pair only the leader CTA issues; its MMAs fill both CTAs' TMEM)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int k = 0;; ++k) {
        const TileInfo ti = ring_read(k, true);
        if (ti.kind == KIND_END) break;
        if (ti.kind != KIND_MMA) continue;
        // the last column block of a member only multiplies its own columns (N multiple of
        // 16, of 32 for a pair so that each CTA's half is a multiple of 16)
        const int n_mma = PAIR ? pair_n_mma<BN>(ti) : min(BN, (ti.n_valid - ti.nt * BN + 15) & ~15);
        const uint32_t idesc = idesc_bf16_f32(n_mma, Cfg::A_MN, Cfg::B_MN, Cfg::TILE_M);
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
            if constexpr (PAIR)
              umma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
            else
              umma_f16(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          if constexpr (PAIR) {  // frees the stage in both CTAs
            umma_commit_pair(smem_u32(&empty[stage]));
            umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
          } else {
            umma_commit(&empty[stage]);
          }
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (aborted) break;
        if constexpr (PAIR) {
          umma_commit_pair(smem_u32(&tfull[acc]));
          umma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));
        } else {
          umma_commit(&tfull[acc]);
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Every MMA issued by this thread has completed once done_bar flips.
      if constexpr (PAIR)
        umma_commit_pair(smem_u32(done_bar));
      else
        umma_commit(done_bar);
      volatile int no_abort = 0;
      mbar_wait(done_bar, 0, &no_abort);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ tile scheduler
    // Claims (tile list) or enumerates (slots c, c + grid, ...) this CTA's tiles, decodes
    // them and publishes every tile that needs work, then KIND_END.
    if (lane == 0) {
      const int n_list = pr.tile_list != nullptr ? __ldg(pr.tile_count) : 0;
      int pub = 0;
      for (int k = 0;; ++k) {
        TileInfo ti;
        if (PAIR && pr.tile_list != nullptr) {
          // a pair claims each tile once: the leader's scheduler claims it and hands the index
          // to the peer's through the peer's shared memory; both decode and publish it
          const int cs = k & (CRING - 1);
          const uint32_t cph = (uint32_t)(k / CRING) & 1u;
          int i;
          if (rank == 0) {
            i = (k == 0) ? (int)tile0 : tile_step + atomicAdd(pr.tile_counter, 1);
            if (!mbar_wait<true>(&claim_empty[cs], cph ^ 1u, abort_flag)) break;
            st_shared_cluster_u32(mapa_shared(smem_u32((const void*)(claim_val + cs)), 1), (uint32_t)i);
            mbar_arrive_release_cluster(mapa_shared(smem_u32(&claim_full[cs]), 1));
          } else {
            if (!mbar_wait<true>(&claim_full[cs], cph, abort_flag)) break;
            i = claim_val[cs];
            mbar_arrive_release_cluster(mapa_shared(smem_u32(&claim_empty[cs]), 0));
          }
          if (i < n_list)
            ti = decode_list_entry(pr, __ldg(pr.tile_list + i), Cfg::BK);
          else
            ti.kind = KIND_END;
        } else if (pr.tile_list != nullptr) {
          const int i = (k == 0) ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(pr.tile_counter, 1);
          if (i < n_list)
            ti = decode_list_entry(pr, __ldg(pr.tile_list + i), Cfg::BK);
          else
            ti.kind = KIND_END;
        } else {
          const int t = tile0 + k * tile_step;
          if (t < total_tiles)
            ti = decode_tile(pr, t, Cfg::BK);
          else
            ti.kind = KIND_END;
          if (ti.kind == KIND_SKIP || (ti.kind == KIND_ZERO && pr.skip_zero)) continue;
        }
        const int s = pub & (TRING - 1);
        if (!mbar_wait(&tr_empty[s], ((uint32_t)(pub / TRING) & 1u) ^ 1u, abort_flag)) break;
        volatile int* e = tile_ring + 8 * s;
        e[0] = ti.member;
        e[1] = ti.mt;
        e[2] = ti.nt;
        e[3] = ti.kind;
        e[4] = ti.kblocks;
        e[5] = ti.m_valid;
        e[6] = ti.n_valid;
        mbar_arrive(&tr_full[s]);
        ++pub;
        if (ti.kind == KIND_END) break;
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    // Epilogue warp w drains TMEM lane quarter (w % 4) and column slice (w - 3) / 4
    // (EPI_WARPS / 4 slices of WCOLS columns).
    const int ew = warp - Cfg::EPI_WARP0;
    const int q = warp & 3;
    const int half = ew >> 2;
    constexpr int WCOLS = BN / (Cfg::EPI_WARPS / 4);
    constexpr int NCH = WCOLS / 32;
    float* sbias = reinterpret_cast<float*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES + Cfg::CTRL_BYTES) + ew * WCOLS;
    uint8_t* stage_warp = smem + Cfg::STAGES * Cfg::STAGE_BYTES + Cfg::CTRL_BYTES +
                          Cfg::EPI_WARPS * Cfg::BIAS_FLOATS_PER_WARP * 4 + ew * Cfg::STORE_STAGE_BYTES;
    uint8_t* stage_row = stage_warp + lane * Cfg::STAGE_ROW_BYTES;
    const int row_in_tile = (int)rank * Cfg::BM + q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool dropout_on = Cfg::FWDK && pr.dropout_p != nullptr;
    // tile metadata is decoded one tile ahead so its global loads overlap the current tile
    TileInfo nti;
    float np = 0.0f;
    // the bias slice of the next MMA tile is loaded into registers one tile ahead
    float bnext[NCH];
    auto load_bias = [&](const TileInfo& x) {
      const int cb = x.nt * BN + half * WCOLS;
#pragma unroll
      for (int i = 0; i < NCH; ++i) {
        const int col = cb + 32 * i + lane;
        bnext[i] = (Cfg::FWDK && x.kind == KIND_MMA && pr.bias != nullptr && col < x.n_valid)
                       ? __ldg(pr.bias + (size_t)x.member * pr.bias_ld + col)
                       : 0.0f;
      }
    };
    nti = ring_read(0, lane == 0);
    if (nti.kind != KIND_END) {
      if (dropout_on) np = __ldg(pr.dropout_p + nti.member);
      if (Cfg::FWDK) load_bias(nti);
    }
    for (int k = 0; nti.kind != KIND_END; ++k) {
      const TileInfo ti = nti;
      const float p_cur = np;
      nti = ring_read(k + 1, lane == 0);
      const bool has_next = nti.kind != KIND_END;
      if (has_next && dropout_on) np = __ldg(pr.dropout_p + nti.member);
      const int m = ti.member;
      const int row = ti.mt * Cfg::TILE_M + row_in_tile;
      const int cbase = ti.nt * BN + half * WCOLS;
      // a ZERO / COPY / SKIP tile stages no bias: prefetch the next tile's slice here, so the
      // MMA tile after it does not stage this tile's (zero) slice
      if (Cfg::FWDK && ti.kind != KIND_MMA && has_next) load_bias(nti);
      if (ti.kind == KIND_MMA) {
        uint32_t thr = 65536u;
        float scale = 1.0f;  // 1 / (1 - p): kept elements are (acc + b) * scale
        if (dropout_on) {
          thr = keep_threshold(p_cur);
          scale = keep_scale(p_cur);
        }
        if (Cfg::FWDK) {
          // this tile's bias slice times the keep scale (zero beyond n_valid) to smem, then
          // prefetch the next one; the epilogue forms (acc + b) * scale as fma(acc, scale, b * scale)
          __syncwarp();
#pragma unroll
          for (int i = 0; i < NCH; ++i) sbias[32 * i + lane] = bnext[i] * scale;
          __syncwarp();
          if (has_next) load_bias(nti);
        }
        // Newton-Schulz: the addend of the first chunk is loaded before the accumulator wait
        [[maybe_unused]] uint4 d_a[4], d_b[4];
        [[maybe_unused]] const __nv_bfloat16* d_row = nullptr;
        if constexpr (is_ns(MODE)) {
          if (pr.D != nullptr && row < ti.m_valid)
            d_row = reinterpret_cast<const __nv_bfloat16*>(pr.D) + (size_t)m * pr.out_ms + (size_t)row * pr.out_ld;
          ns_load_d(d_row, cbase, ti.n_valid - cbase, d_a);
        }
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) break;
        tc_fence_after();
        const uint32_t t_row =
            tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN) + (uint32_t)(half * WCOLS);
        // chunks of 32 columns that hold storable output (warp-uniform)
        const int nch = min(NCH, max(0, (pr.out_cols - cbase + 31) / 32));
        const int row_base = ti.mt * Cfg::TILE_M + (int)rank * Cfg::BM + q * 32;
        auto emit_chunk = [&](int col0, const uint32_t(&rr)[32]) {
          dgrad_chunk(ti, col0, rr, stage_row);
          __syncwarp();
          stage_flush(pr, m, row_base, col0, stage_warp, lane, Cfg::STAGE_ROW_BYTES);
          __syncwarp();
        };
        if constexpr (is_ns(MODE)) {
          // Chunks past the member's columns rounded up to a k-block (64) are never read: no
          // later GEMM's K loop reaches them, and as M / N rows they only feed outputs that are
          // written as zeros.  Two chunks' accumulators are loaded per TMEM wait; the addend of
          // the next pair is loaded while this pair is computed.
          const bool rv = row < ti.m_valid;
          const int nch_k = min(nch, max(0, (((ti.n_valid + 63) & ~63) - cbase + 31) / 32));
          // symmetric product: this warp's half is also written transposed into a tile below
          // the diagonal (one that the tile list leaves out) when that tile lies entirely there
          // (a pair's 256 x 256 tile: every tile above the diagonal; the diagonal tiles compute
          // both of their triangles)
          const bool mirror = pr.ns_sym && (PAIR ? ti.mt < ti.nt : ((ti.mt >> 1) * 2 + 2 <= 2 * ti.nt + half));
          uint32_t na[32], nb[32];
#pragma unroll 1
          for (int c = 0; c < nch_k; c += 2) {
            const int col0 = cbase + 32 * c;
            const bool two = c + 1 < nch_k;
            tmem_ld_32x32b_x32(t_row + (uint32_t)(32 * c), na);
            if (two) {
              tmem_ld_32x32b_x32(t_row + (uint32_t)(32 * (c + 1)), nb);
              ns_load_d(d_row, col0 + 32, ti.n_valid - col0 - 32, d_b);
            }
            tmem_wait_ld();
            ns_chunk(pr, rv, ti.n_valid - col0, na, d_a, stage_row);
            __syncwarp();
            stage_flush(pr, m, row_base, col0, stage_warp, lane, Cfg::STAGE_ROW_BYTES);
            if (mirror) mirror_flush(pr, m, row_base, col0, stage_warp, lane, Cfg::STAGE_ROW_BYTES);
            __syncwarp();
            if (two) {
              if (c + 2 < nch_k) ns_load_d(d_row, col0 + 64, ti.n_valid - col0 - 64, d_a);
              ns_chunk(pr, rv, ti.n_valid - col0 - 32, nb, d_b, stage_row);
              __syncwarp();
              stage_flush(pr, m, row_base, col0 + 32, stage_warp, lane, Cfg::STAGE_ROW_BYTES);
              if (mirror) mirror_flush(pr, m, row_base, col0 + 32, stage_warp, lane, Cfg::STAGE_ROW_BYTES);
              __syncwarp();
            }
          }
        } else if constexpr (is_wgrad_t(MODE)) {
          // lane = input feature `row`, register j = output feature col0 + j:
          // dW[o][row] for fixed o is 32 consecutive floats across the warp
          float* base = reinterpret_cast<float*>(pr.out) + (size_t)m * pr.out_ms;
          const bool in_store = row < pr.out_cols;
          const bool in_valid = row < ti.m_valid;
          // with the padding known zero, only the chunks that hold the member's output features
          const int nco = min(NCH, max(0, ((pr.skip_zero ? min(pr.out_rows, ti.n_valid) : pr.out_rows) - cbase + 31) / 32));
          uint32_t wa[32];
#pragma unroll 1
          for (int c = 0; c < nco; ++c) {
            const int o0 = cbase + 32 * c;
            tmem_ld_32x32b_x32(t_row + (uint32_t)(32 * c), wa);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int o = o0 + j;
              if (in_store && o < pr.out_rows)
                base[(size_t)o * pr.out_ld + row] = (in_valid && o < ti.n_valid) ? __uint_as_float(wa[j]) : 0.0f;
            }
          }
        } else if constexpr (Cfg::FWDK) {
          // 16-column TMEM loads (four warps per scheduler cover their latency); the staged
          // 32-column slot is flushed after every second chunk.  Only the 32-column chunks
          // that hold some of the member's columns run the epilogue; the padding after them
          // is written as plain zeros.
          const int ncomp = min(nch, max(0, (ti.n_valid - cbase + 31) / 32));
          const int n16 = 2 * ncomp;
          const bool drop = dropout_on && thr < 65536u;
          uint32_t fa[16];
#pragma unroll 1
          for (int c = 0; c < n16; ++c) {
            const int col0 = cbase + 16 * c;
            tmem_ld_32x32b_x16(t_row + (uint32_t)(16 * c), fa);
            const int nv = ti.n_valid - col0;
            uint4 q2[2];
            fwd16_draws(pr, m, row, col0, drop && nv > 0, q2);
            [[maybe_unused]] float4 ea[4];
            if constexpr (MODE == MODE_FWD_ADD) {
              // the gathered addend of this row's 16 columns (the ragged tail is zeroed below)
              const bool ev = nv > 0 && row < pr.B;
              const float4* ep = reinterpret_cast<const float4*>(pr.addend + ((size_t)m * pr.B + row) * pr.add_ld + col0);
#pragma unroll
              for (int i = 0; i < 4; ++i) ea[i] = ev ? __ldg(ep + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            tmem_wait_ld();
            if constexpr (MODE == MODE_FWD_ADD) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                fa[4 * i] = __float_as_uint(__uint_as_float(fa[4 * i]) + ea[i].x);
                fa[4 * i + 1] = __float_as_uint(__uint_as_float(fa[4 * i + 1]) + ea[i].y);
                fa[4 * i + 2] = __float_as_uint(__uint_as_float(fa[4 * i + 2]) + ea[i].z);
                fa[4 * i + 3] = __float_as_uint(__uint_as_float(fa[4 * i + 3]) + ea[i].w);
              }
            }
            epi_fwd16(pr, fa, q2, nv, drop && nv > 0, thr, scale, sbias + 16 * c, stage_row + 32 * (c & 1));
            if (c & 1) {
              __syncwarp();
              stage_flush(pr, m, row_base, col0 - 16, stage_warp, lane, Cfg::STAGE_ROW_BYTES);
              __syncwarp();
            }
          }
          const int z0 = cbase + 32 * ncomp, z1 = min(cbase + WCOLS, pr.out_cols);
          if (z0 < z1 && !pr.skip_zero) zero_fill_bf16(pr, m, row_base, z0, z1, lane);
        } else {
        uint32_t ra[32], rb[32];
        if (nch > 0) tmem_ld_32x32b_x32(t_row, ra);
#pragma unroll 1
        for (int c = 0; c < nch; c += 2) {
          tmem_wait_ld();
          if (c + 1 < nch) tmem_ld_32x32b_x32(t_row + (uint32_t)(32 * (c + 1)), rb);
          emit_chunk(cbase + 32 * c, ra);
          if (c + 1 < nch) {
            tmem_wait_ld();
            if (c + 2 < nch) tmem_ld_32x32b_x32(t_row + (uint32_t)(32 * (c + 2)), ra);
            emit_chunk(cbase + 32 * (c + 1), rb);
          }
        }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR)
            mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));  // the leader's MMA waits on it
          else
            mbar_arrive(&tempty[acc]);
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      } else if (ti.kind != KIND_SKIP) {
        // ZERO or COPY block: this warp's 32 rows x column slice, lanes along the columns
        const int row_base = ti.mt * Cfg::TILE_M + (int)rank * Cfg::BM + q * 32;
        const int c_end = min(cbase + WCOLS, pr.out_cols);
        if (is_wgrad_t(MODE)) {
          // zero block, transposed: output features cbase.. x input features row_base + lane
          float* base = reinterpret_cast<float*>(pr.out) + (size_t)m * pr.out_ms;
          const int i = row_base + lane;
          const int o_end = min(cbase + WCOLS, pr.out_rows);
          if (i < pr.out_cols)
            for (int o = cbase; o < o_end; ++o) base[(size_t)o * pr.out_ld + i] = 0.0f;
        } else {
          __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(pr.out) + (size_t)m * pr.out_ms;
          const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(pr.copy_src) + (size_t)m * pr.out_ms;
          const int nq = (c_end - cbase) / 8;  // 16-byte pieces per row (out_cols multiple of 8)
          const int npieces = 32 * nq;
          const bool copy = ti.kind == KIND_COPY;
          // batches of 8 pieces per lane: every load of a batch is in flight before its stores
          constexpr int UNR = 8;
          for (int i0 = 0; i0 < npieces; i0 += 32 * UNR) {
            uint4 v[UNR];
            int off[UNR];  // element offsets within the member's block (-1: outside), below 2^31
#pragma unroll
            for (int u = 0; u < UNR; ++u) {
              const int i = i0 + 32 * u + lane;
              const int r = (nq == WCOLS / 8) ? i / (WCOLS / 8) : i / max(nq, 1);
              const int cc = cbase + 8 * (i - r * nq);
              off[u] = (i < npieces && row_base + r < pr.out_rows) ? (row_base + r) * pr.out_ld + cc : -1;
              v[u] = (copy && off[u] >= 0) ? __ldg(reinterpret_cast<const uint4*>(src + off[u])) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < UNR; ++u)
              if (off[u] >= 0) *reinterpret_cast<uint4*>(base + off[u]) = v[u];
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // neither CTA leaves while the other may still signal it
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
#endif
}

}  // namespace tp
