// Shared device helpers: error flag, Philox4x32-10, bounded mbarrier waits,
// and thin inline-PTX wrappers for TMA (cp.async.bulk.tensor) and tcgen05.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tabpack_b200.h"

namespace tp {

// Set (never cleared by kernels) when a bounded device-side wait gives up.
__device__ int g_device_error = 0;

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon et al., SC'11).  Dropout key/counter layout:
//   key = (seed lo, seed hi), counter = (col >> 3, row, member, offset);
//   element col uses the 16-bit slice (col & 7) of the 128-bit output.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    // one 32x32->64-bit multiply per product
    const uint64_t p0 = (uint64_t)0xD2511F53u * c.x;
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c.z;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// Philox4x32-10 with a precomputed key schedule ks[2*i], ks[2*i+1] = key words of round i
// (held in kernel parameters, i.e. constant-bank operands of the XORs).
__device__ __forceinline__ uint4 philox4x32_10_ks(uint4 c, const uint32_t* ks) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c.x;
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c.z;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    c = make_uint4(hi1 ^ c.y ^ ks[2 * i], lo1, hi0 ^ c.w ^ ks[2 * i + 1], lo0);
  }
  return c;
}

__host__ __device__ inline void philox_key_schedule(uint32_t k0, uint32_t k1, uint32_t* ks) {
  for (int i = 0; i < 10; ++i) {
    ks[2 * i] = k0;
    ks[2 * i + 1] = k1;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// floor(float32(1 - p) * 2^16): an element is kept iff its 16-bit draw is below it.
__device__ __forceinline__ uint32_t keep_threshold(float p) {
  const float keep = 1.0f - p;
  return (uint32_t)floorf(keep * 65536.0f);
}

// float32(1 / (1 - p)), correctly rounded.
__device__ __forceinline__ float keep_scale(float p) { return __frcp_rn(1.0f - p); }

// 8 keep bits (bit j = column 8*group + j) for one (row, member) and column group.
__device__ __forceinline__ uint32_t dropout_bits8(uint32_t k0, uint32_t k1, uint32_t group,
                                                   uint32_t row, uint32_t member,
                                                   uint32_t offset, uint32_t thr) {
  const uint4 r = philox4x32_10(make_uint4(group, row, member, offset), k0, k1);
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
  uint32_t bits = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t r16 = (w[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu;
    bits |= (r16 < thr ? 1u : 0u) << j;
  }
  return bits;
}

// ---------------------------------------------------------------------------
// Bounded waits.  A wait gives up after ~2 s of GPU time, records TP_ETIMEOUT in
// g_device_error and reports failure to its caller, which then unwinds.
// ---------------------------------------------------------------------------
#ifndef TP_WAIT_CYCLES
#define TP_WAIT_CYCLES 4000000000ull
#endif

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// CLUSTER: acquire at cluster scope (arrivals released by the peer CTA of a pair).
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  if (CLUSTER)
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
  else
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps (without issuing) until the phase
// completes or the hint expires, instead of spinning.
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  if (CLUSTER)
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(0x989680u)  // 10 ms
        : "memory");
  else
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(0x989680u)  // 10 ms
        : "memory");
  return ok != 0;
}

// Returns false on timeout or when *abort is already set.
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint32_t b = smem_u32(bar);
  if (mbar_try_wait<CLUSTER>(b, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait_sleep<CLUSTER>(b, parity)) return true;
    if (*abort) return false;
    if ((unsigned long long)(clock64() - t0) > TP_WAIT_CYCLES) {
      *abort = 1;
      atomicExch(&g_device_error, TP_ETIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA: tiled 3-D load into this CTA's shared memory, completion on an mbarrier.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Four rows of a 2-D table (tensor map box: 64 columns x 1 row) at column x into 512 consecutive
// bytes of shared memory, completing on `bar`: TMA gather4.  The shared-memory destination keeps
// the map's 128-byte swizzle, so four gathers at 512-byte steps fill a tile as one tiled load of
// those rows would.
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int4 rows) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(rows.x), "r"(rows.y), "r"(rows.z),
      "r"(rows.w)
      : "memory");
}

// CTA-pair form (cta_group::2): the data lands in this CTA's shared memory and the
// transaction bytes are counted on `bar_cluster`, a shared::cluster address that may
// name the mbarrier of the pair's leader CTA; the data goes to this CTA only.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---------------------------------------------------------------------------
// Division by a kernel-invariant divisor (Granlund & Montgomery, "Division by invariant
// integers using multiplication", PLDI 1994): for 0 <= n < 2^31 and d >= 1,
// n / d == (umulhi(n, m) + n) >> l with l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1.
// ---------------------------------------------------------------------------
struct FastDiv {
  uint32_t d, m, l;
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  f.d = d;
  f.l = 0;
  while ((1ull << f.l) < d) ++f.l;
  f.m = (uint32_t)((((1ull << f.l) - d) << 32) / d + 1);
  return f;
}

__device__ __forceinline__ uint32_t fastdiv(uint32_t n, const FastDiv& f) { return (__umulhi(n, f.m) + n) >> f.l; }

// ---------------------------------------------------------------------------
// Thread-block clusters (CTA pairs)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the variable at shared::cta address `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Every thread of both CTAs; orders shared-memory writes (barrier init) before the peer's use.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (own or peer CTA).  CTA-scope
// release: it only has to follow this thread's completed TMEM reads (ordered by the
// tcgen05 fences around it), not make its global stores visible cluster-wide, which
// would make it wait for every outstanding store.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// Arrive with release semantics at cluster scope: this thread's earlier shared-memory writes
// into the peer CTA (st_shared_cluster_u32) are visible to a thread that observes the phase
// with an acquire.cluster wait.
__device__ __forceinline__ void mbar_arrive_release_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// 32-bit store into shared memory given by its shared::cluster address (own or peer CTA).
__device__ __forceinline__ void st_shared_cluster_u32(uint32_t addr_cluster, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr_cluster), "r"(v) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core, accumulators in tensor memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// CTA-pair TMEM allocation: one warp with the same warp index in each CTA of the pair
// issues it, with the same shared-memory slot; both CTAs receive the same column base.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulation).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// CTA-pair MMA, issued by the leader CTA: M = 256 rows, A rows 0..127 from the
// leader's and 128..255 from the peer's shared memory (same offsets), B columns split
// in halves the same way, D rows 0..127 into the leader's TMEM and 128..255 into the peer's.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Pair form of umma_commit: the mbarrier may be in either CTA (shared::cluster address).
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: thread i of the warp gets lane (base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version bits.
//   K-major : rows of 128 B (64 bf16 along K), 8-row groups 1024 B apart (SBO).
//   MN-major: rows of 128 B (64 bf16 along M/N) per K index, 8-K-row groups
//             1024 B apart (SBO), 64-element M/N chunks `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, A = B = bf16, D = f32, M = 128.
__host__ __device__ __forceinline__ uint32_t idesc_bf16_f32(int n, bool a_mn_major, bool b_mn_major, int m = 128) {
  return (1u << 4)                     // D format f32
         | (1u << 7)                   // A format bf16
         | (1u << 10)                  // B format bf16
         | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17)    // N / 8
         | ((uint32_t)(m >> 4) << 24);    // M / 16
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

}  // namespace tp
