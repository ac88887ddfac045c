// Tile scheduling shared by the tensor-core (tcgen05) and CUDA-core paths of the
// packed linear layer.
//
// One launch covers all P members of a pack.  Each member owns the same number
// of tile slots (m_tiles x n_tiles over the padded output), so tile t maps to
// member t / (m_tiles * n_tiles) without any prefix sums.  A slot is:
//   MMA  - a real BMxBN block of C = A * B^T, K = the member's own reduction length
//   ZERO - an output block that lies entirely in the member's padding (written 0)
//   COPY - a block of a depth-inactive member: y = x (forward) / dx = dy (dgrad)
#pragma once

#include "common.cuh"

namespace tp {

// MODE_NS / MODE_NS_BMN: one Newton-Schulz GEMM, C = alpha * A B^T + beta * D, with
// per-member shapes taken from (ns_rows, ns_cols) and B read K-major / MN-major.
enum : int { MODE_FWD = 0, MODE_DGRAD = 1, MODE_WGRAD = 2, MODE_NS = 3, MODE_NS_BMN = 4, MODE_WGRAD_T = 5 };
// Kernel instantiation of the forward whose epilogue also adds a per-element fp32 addend
// (the gathered one-hot columns of a TabPack's first layer); its problems carry
// mode = MODE_FWD, so tiles decode as the forward's.
enum : int { MODE_FWD_ADD = 6 };
// Kernel instantiation of the forward on CTA pairs (mode = MODE_FWD as well): used without
// dropout (no Philox draws, so the epilogue keeps up with the pair's faster k-blocks) and for
// long K loops, where operand delivery rather than the epilogue bounds a tile.
enum : int { MODE_FWD_PAIR = 7 };
// Kernel instantiation of the transposed weight gradient (problems carry MODE_WGRAD_T) on single
// CTAs whose A operand (X^T) is gathered from a table by row index.
enum : int { MODE_WGRAD_TG = 9 };
__host__ __device__ constexpr bool is_wgrad_t(int mode) { return mode == MODE_WGRAD_T || mode == MODE_WGRAD_TG; }
// Kernel instantiations of the Newton-Schulz GEMMs on CTA pairs (256-row tiles claimed from
// 256-row tile lists; problems carry MODE_NS / MODE_NS_BMN).
enum : int { MODE_NS_P = 10, MODE_NS_BMN_P = 11 };
__host__ __device__ constexpr bool is_ns(int mode) {
  return mode == MODE_NS || mode == MODE_NS_BMN || mode == MODE_NS_P || mode == MODE_NS_BMN_P;
}
// KIND_END marks the end of a CTA's tile sequence in the kernel's shared-memory tile ring.
enum : int { KIND_MMA = 0, KIND_ZERO = 1, KIND_COPY = 2, KIND_SKIP = 3, KIND_END = 4 };

struct LinearProblem {
  int mode;
  int P, B;
  int max_in, max_out;        // storage widths of x/w/y (multiples of 8 on the bf16 path)
  const int32_t* in_f;        // (P,) or nullptr
  const int32_t* out_f;       // (P,) or nullptr
  const int32_t* n_blocks;    // (P,) or nullptr
  int block_index;
  int x_shared;
  // forward epilogue
  int relu;
  const float* dropout_p;     // (P,) or nullptr
  uint32_t k0, k1, offset, member_base;
  uint32_t ks[20];            // Philox key schedule of (k0, k1)
  const float* bias;          // (P, bias_ld) or nullptr
  int bias_ld;
  // output: rows x cols per member, leading dim out_ld, member stride out_ms
  void* out;
  int out_rows, out_cols, out_ld;
  long long out_ms;
  // COPY source (depth-inactive members), same geometry as the output
  const void* copy_src;
  // operand pointers for the CUDA-core path (the tensor-core path uses TMA maps)
  const void* a_ptr;
  const void* b_ptr;
  int m_tiles, n_tiles;
  int BM, BN;
  int skip_zero;       // the output's padding already holds zeros: ZERO tiles are not written
  // gathered input (x is a shared table): member m's row b is x row row_index[m * B + b]; the
  // producer warp loads the A operand with TMA gather4 (4 table rows per load)
  const int32_t* row_index;
  FastDiv div_member;  // by m_tiles * n_tiles (tiles per member)
  FastDiv div_mt;      // by m_tiles
  // Dynamic scheduling (single-CTA launches): a dense list of the launch's MMA tiles, entry
  // member << 16 | n-tile << 8 | m-tile, its length (on the device) and a zeroed counter; CTA
  // c takes entry c first and claims the next ones with the counter.  Without a list CTA c
  // takes slots c, c + grid, ...
  const uint32_t* tile_list;
  const int* tile_count;
  int* tile_counter;
  // Newton-Schulz GEMMs: member m multiplies r = ns_rows[m], c = ns_cols[m] matrices;
  // ns_shape 1: (M, N, K) = (r, r, c), 2: (r, r, r), 3: (r, c, r); members with
  // active[m] == 0 are skipped.
  const int32_t* ns_rows;
  const int32_t* ns_cols;
  const int32_t* active;
  int ns_shape;
  int ns_sym;  // symmetric output (A = X X^T): tiles below the diagonal come as transposes
  float alpha, beta;
  const void* D;  // (optional) addend with the output's geometry
  // MODE_FWD_ADD: fp32 addend (P, B, add_ld) added to the accumulator before the bias
  const float* addend;
  int add_ld;
};

struct TileInfo {
  int member, mt, nt, kind, kblocks, m_valid, n_valid;
};

__device__ __forceinline__ bool member_active(const LinearProblem& p, int m) {
  return p.n_blocks == nullptr || __ldg(p.n_blocks + m) > p.block_index;
}

__device__ __forceinline__ TileInfo decode_tile(const LinearProblem& p, int t, int BK) {
  TileInfo ti;
  // Slot order (member, n-tile, m-tile): consecutive slots of one member walk down the
  // rows of one column block, so a persistent CTA that strides through the slots sees
  // every n-tile (a row-major order would pin a CTA to n-tile (cta % n_tiles) whenever
  // the grid is a multiple of n_tiles, and padding-only n-tiles would idle those CTAs).
  const int per_member = p.m_tiles * p.n_tiles;
  ti.member = (int)fastdiv((uint32_t)t, p.div_member);
  const int r = t - ti.member * per_member;
  ti.nt = (int)fastdiv((uint32_t)r, p.div_mt);
  ti.mt = r - ti.nt * p.m_tiles;
  const int m = ti.member;
  if (p.mode == MODE_NS || p.mode == MODE_NS_BMN) {
    const int r = __ldg(p.ns_rows + m), c = __ldg(p.ns_cols + m);
    ti.m_valid = r;
    ti.n_valid = (p.ns_shape == 3) ? c : r;
    const int k_len = (p.ns_shape == 1) ? c : r;
    ti.kblocks = (k_len + BK - 1) / BK;
    const bool act = p.active == nullptr || __ldg(p.active + m) != 0;
    ti.kind = (!act || ti.mt * p.BM >= ti.m_valid || ti.nt * p.BN >= ti.n_valid || ti.kblocks == 0) ? KIND_SKIP
                                                                                                     : KIND_MMA;
    return ti;
  }
  const int in_m = p.in_f ? __ldg(p.in_f + m) : p.max_in;
  const int out_m = p.out_f ? __ldg(p.out_f + m) : p.max_out;
  const bool active = member_active(p, m);
  int k_len;
  if (p.mode == MODE_FWD) {
    ti.m_valid = p.B;
    ti.n_valid = out_m;
    k_len = in_m;
  } else if (p.mode == MODE_DGRAD) {
    ti.m_valid = p.B;
    ti.n_valid = in_m;
    k_len = out_m;
  } else if (p.mode == MODE_WGRAD_T) {  // dW^T = X^T G: rows are input features
    ti.m_valid = in_m;
    ti.n_valid = out_m;
    k_len = p.B;
  } else {
    ti.m_valid = out_m;
    ti.n_valid = in_m;
    k_len = p.B;
  }
  ti.kblocks = (k_len + BK - 1) / BK;
  if (!active) {
    // a depth-gated member passes its input through (y = x, dx = dy) over its valid columns;
    // the source's padding columns beyond them are zeros, so those tiles are ZERO tiles
    // (nothing to read)
    ti.kind = (p.mode == MODE_WGRAD || p.mode == MODE_WGRAD_T || ti.nt * p.BN >= ti.n_valid) ? KIND_ZERO
                                                                                               : KIND_COPY;
  } else if (ti.mt * p.BM >= ti.m_valid || ti.nt * p.BN >= ti.n_valid || ti.kblocks == 0) {
    ti.kind = KIND_ZERO;
  } else {
    ti.kind = KIND_MMA;
  }
  return ti;
}

// A Newton-Schulz tile-list entry (see LinearProblem::tile_list).
__device__ __forceinline__ TileInfo decode_list_entry(const LinearProblem& p, uint32_t e, int BK) {
  TileInfo ti;
  ti.member = (int)(e >> 16);
  ti.nt = (int)((e >> 8) & 0xFFu);
  ti.mt = (int)(e & 0xFFu);
  const int r = __ldg(p.ns_rows + ti.member), c = __ldg(p.ns_cols + ti.member);
  ti.m_valid = r;
  ti.n_valid = (p.ns_shape == 3) ? c : r;
  ti.kblocks = ((p.ns_shape == 1 ? c : r) + BK - 1) / BK;
  ti.kind = KIND_MMA;
  return ti;
}

// Value written to output element (row, col) of member m given the fp32 dot product.
// `bits` carries the dropout keep bit of this column (bit 0), `keep_scale` its scale.
template <int MODE>
__device__ __forceinline__ float epilogue_value(const LinearProblem& p, const TileInfo& ti, int row, int col,
                                                float acc, float bias, bool keep, float scale) {
  if (MODE == MODE_FWD) {
    if (col >= ti.n_valid) return 0.0f;
    float v = acc + bias;
    if (p.relu) v = fmaxf(v, 0.0f);
    return keep ? v * scale : 0.0f;
  } else if (MODE == MODE_DGRAD) {
    return col < ti.n_valid ? acc : 0.0f;
  } else {
    return (row < ti.m_valid && col < ti.n_valid) ? acc : 0.0f;
  }
}

}  // namespace tp
