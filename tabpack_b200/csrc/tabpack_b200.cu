// C ABI of the B200 packed-ensemble hot path (declared in include/tabpack_b200.h).
// One translation unit: host-side validation, TMA descriptor encoding and kernel
// dispatch for every entry point.
#include <cudaTypedefs.h>

#include <algorithm>
#include <type_traits>

#include <cmath>
#include <cstdlib>
#include <cstdarg>
#include <cstdio>
#include <atomic>
#include <mutex>
#include <vector>
#include <string>

#include "elementwise.cuh"
#include "gemm_sm100.cuh"
#include "gemm_simt.cuh"
#include "muon.cuh"
#include "metrics.cuh"
#include "roc_auc.cuh"
#include "embeddings.cuh"
#include "onehot.cuh"

namespace tp {
namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(TP_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define TP_CUDA_TRY(expr)                           \
  do {                                              \
    cudaError_t e_ = (expr);                        \
    if (e_ != cudaSuccess) return cuda_fail(e_, #expr); \
  } while (0)

// ---- optional per-launch timing (tp_profile_start / tp_profile_stop) -----------------
// Off by default (one relaxed atomic load per launch).  When on, each kernel launch (or, for
// entry points without a GEMM inside, each call) is bracketed by two CUDA events taken from a
// pool that tp_profile_start creates on the current device; tp_profile_stop waits for them and
// adds up the elapsed time per kernel family.
std::atomic<int> g_prof_on{0};
std::mutex g_prof_mu;
std::vector<cudaEvent_t> g_prof_events;  // two per slot
std::vector<int> g_prof_kind;            // family of each slot
int g_prof_used = 0;
int g_prof_dropped = 0;

struct ProfScope {
  cudaStream_t st;
  int slot = -1;
  ProfScope(int kind, cudaStream_t s) : st(s) {
    if (!g_prof_on.load(std::memory_order_relaxed)) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (g_prof_used >= (int)g_prof_kind.size()) {
      ++g_prof_dropped;
      return;
    }
    slot = g_prof_used++;
    g_prof_kind[slot] = kind;
    cudaEventRecord(g_prof_events[2 * slot], st);
  }
  ~ProfScope() {
    if (slot >= 0) cudaEventRecord(g_prof_events[2 * slot + 1], st);
  }
  ProfScope(const ProfScope&) = delete;
  ProfScope& operator=(const ProfScope&) = delete;
};

#define TP_PROF_CAT2(a, b) a##b
#define TP_PROF_CAT(a, b) TP_PROF_CAT2(a, b)
#define TP_PROF(kind, stream) ProfScope TP_PROF_CAT(prof_scope_, __LINE__)((kind), (stream))

struct DeviceInfo {
  int sms = 0;
  int major = 0, minor = 0;
};

DeviceInfo device_info() {
  static std::mutex mu;
  static DeviceInfo cache[64];
  static bool have[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && !have[dev]) {
    cudaDeviceGetAttribute(&cache[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&cache[dev].major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&cache[dev].minor, cudaDevAttrComputeCapabilityMinor, dev);
    have[dev] = true;
  }
  return (dev >= 0 && dev < 64) ? cache[dev] : DeviceInfo{};
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 tensor (planes, rows, inner) with 128-byte swizzled boxes (box_inner x box_rows x 1).
int make_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t rows, uint64_t planes, uint32_t box_inner,
             uint32_t box_rows) {
  auto enc = encode_fn();
  if (!enc) return fail(TP_EUNSUPPORTED, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {inner, rows, planes};
  cuuint64_t strides[2] = {inner * 2, inner * rows * 2};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TP_EINVAL, "cuTensorMapEncodeTiled failed (%d) for dims %llu x %llu x %llu", (int)r,
                (unsigned long long)planes, (unsigned long long)rows, (unsigned long long)inner);
  return TP_OK;
}

// 2-D map over a (rows, inner) bf16 table for TMA gather4: a box of 64 columns x 1 row (gather4
// loads take one-row boxes), 128-byte swizzle like the tiled operand maps.
int make_gather_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t rows) {
  auto enc = encode_fn();
  if (!enc) return fail(TP_EUNSUPPORTED, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {64, 1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TP_EINVAL, "cuTensorMapEncodeTiled failed (%d) for a %llu x %llu gather table", (int)r,
                (unsigned long long)rows, (unsigned long long)inner);
  return TP_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Workspace of tp_linear_backward_noalloc (device memory reserved at module load).
// Host code must not pass this symbol to a kernel: on the host it is only a
// stand-in, and the device address is looked up per device below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[TP_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
// (context, device address) pairs: a module's symbol has one address per CUDA context, so a
// caller that drives a device through a non-primary context gets that context's copy.
struct NoallocEntry {
  CUcontext ctx;
  void* addr;
};
NoallocEntry g_noalloc_addr[64] = {};
int g_noalloc_n = 0;

PFN_cuCtxGetCurrent_v4000 ctx_current_fn() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  });
  return fn;
}

// Device address of g_noalloc_scratch in the current context (looked up once per context).
int noalloc_scratch(void** out) {
  auto cur = ctx_current_fn();
  if (!cur) return fail(TP_EUNSUPPORTED, "cuCtxGetCurrent is unavailable");
  CUcontext ctx = nullptr;
  if (cur(&ctx) != CUDA_SUCCESS) return fail(TP_EUNSUPPORTED, "cuCtxGetCurrent failed");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  for (int i = 0; ctx != nullptr && i < g_noalloc_n; ++i)
    if (g_noalloc_addr[i].ctx == ctx) {
      *out = g_noalloc_addr[i].addr;
      return TP_OK;
    }
  // the first lookup in a context; with no context current, the runtime makes the current
  // device's primary context current here
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
  if (ctx == nullptr && (cur(&ctx) != CUDA_SUCCESS || ctx == nullptr))
    return fail(TP_EUNSUPPORTED, "no current CUDA context after the symbol lookup");
  for (int i = 0; i < g_noalloc_n; ++i)
    if (g_noalloc_addr[i].ctx == ctx) {
      *out = g_noalloc_addr[i].addr;
      return TP_OK;
    }
  if (g_noalloc_n == 64) return fail(TP_EUNSUPPORTED, "more than 64 CUDA contexts used the no-alloc entry point");
  g_noalloc_addr[g_noalloc_n++] = NoallocEntry{ctx, p};
  *out = p;
  return TP_OK;
}

template <int BN, int MODE>
int launch_sm100(const LinearProblem& pr_in, const CUtensorMap& a, const CUtensorMap& b, cudaStream_t st) {
  LinearProblem pr = pr_in;
  pr.div_member = make_fastdiv((uint32_t)std::max(1, pr.m_tiles * pr.n_tiles));
  pr.div_mt = make_fastdiv((uint32_t)std::max(1, pr.m_tiles));
  using Cfg = Sm100Cfg<BN, MODE>;
  auto kern = linear_gemm_sm100<BN, MODE>;
  TP_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
  const long long total = (long long)pr.P * pr.m_tiles * pr.n_tiles;
  if (total > 0x7FFFFFFFLL) return fail(TP_EINVAL, "too many tiles");
  if (total == 0) return TP_OK;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(Cfg::NUM_THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = st;
  // persistent workers: CTAs, or CTA pairs (clusters of 2) for the pair modes
  int workers = device_info().sms;
  if constexpr (Cfg::PAIR) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static int max_clusters[64] = {};
    int dev = 0;
    TP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(TP_EUNSUPPORTED, "device index %d out of range", dev);
    if (max_clusters[dev] == 0) {
      cfg.gridDim = dim3(2 * (device_info().sms / 2));
      int n = 0;
      TP_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
      if (n <= 0) return fail(TP_EUNSUPPORTED, "no CTA pair of this kernel fits on the device");
      max_clusters[dev] = n;
    }
    workers = max_clusters[dev];
  }
  int grid = (int)std::min<long long>(total, workers);
  // A persistent CTA takes slots c, c + grid, ...  With the (member, n-tile, m-tile) slot
  // order its n-tile advances by (grid mod slots_per_member) / m_tiles per step; avoid
  // grids for which that step leaves a CTA on a subset of the column blocks.
  const int spm = pr.m_tiles * pr.n_tiles;
  auto gcd = [](int x, int y) { while (y) { const int r = x % y; x = y; y = r; } return x; };
  for (int g = grid; g > grid / 2 && pr.tile_list == nullptr && pr.n_tiles > 1 && total > grid; --g) {
    const int step = g % spm;
    const bool pinned = step == 0 || (step % pr.m_tiles == 0 && gcd(step / pr.m_tiles, pr.n_tiles) > 1);
    if (!pinned) {
      grid = g;
      break;
    }
  }
  cfg.gridDim = dim3(Cfg::PAIR ? 2 * grid : grid);
  constexpr int kind = (MODE == MODE_DGRAD) ? TP_PROF_DGRAD
                       : (MODE == MODE_WGRAD || is_wgrad_t(MODE)) ? TP_PROF_WGRAD
                       : (MODE == MODE_NS || MODE == MODE_NS_P) ? TP_PROF_NS
                       : (MODE == MODE_NS_BMN || MODE == MODE_NS_BMN_P) ? TP_PROF_NS_BMN
                                               : TP_PROF_FWD;
  TP_PROF(kind, st);
  TP_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, b, pr));
  return TP_OK;
}

template <typename T, int MODE>
int launch_simt(LinearProblem pr, cudaStream_t st) {
  pr.BM = pr.BN = 64;
  pr.m_tiles = (pr.out_rows + 63) / 64;
  pr.n_tiles = (pr.out_cols + 63) / 64;
  pr.div_member = make_fastdiv((uint32_t)std::max(1, pr.m_tiles * pr.n_tiles));
  pr.div_mt = make_fastdiv((uint32_t)std::max(1, pr.m_tiles));
  const long long total = (long long)pr.P * pr.m_tiles * pr.n_tiles;
  if (total > 0x7FFFFFFFLL) return fail(TP_EINVAL, "too many tiles");
  if (total == 0) return TP_OK;
  TP_PROF(TP_PROF_GEMM_F32, st);
  linear_gemm_simt<T, MODE><<<(unsigned)total, 256, 0, st>>>(pr);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int check_linear(const tp_linear_args* a) {
  if (!a) return fail(TP_EINVAL, "null arguments");
  if (a->P <= 0 || a->B <= 0 || a->max_in <= 0 || a->max_out <= 0)
    return fail(TP_EINVAL, "P, B, max_in and max_out must be positive (got %d, %d, %d, %d)", a->P, a->B, a->max_in,
                a->max_out);
  if (a->dtype != TP_DTYPE_F32 && a->dtype != TP_DTYPE_BF16) return fail(TP_EINVAL, "unknown dtype %d", a->dtype);
  if (a->n_blocks && a->max_in != a->max_out)
    return fail(TP_EINVAL, "depth gating needs max_in == max_out (inactive members pass their input through)");
  if (!a->w) return fail(TP_EINVAL, "w is null");
  if (a->row_index) {
    if (a->x_rows <= 0) return fail(TP_EINVAL, "a gathered input needs the table's row count (x_rows > 0)");
    if (a->x_shared || a->n_blocks)
      return fail(TP_EINVAL, "a gathered input is a shared table: no x_shared flag and no depth gating");
    if (a->dtype != TP_DTYPE_BF16 || device_info().major != 10 || (a->max_in % 8) != 0 || (a->max_out % 8) != 0)
      return fail(TP_EUNSUPPORTED, "a gathered input runs on the sm_100 bf16 tensor-core path only");
  }
  return TP_OK;
}

bool use_tensor_cores(const tp_linear_args* a) {
  const DeviceInfo d = device_info();
  return a->dtype == TP_DTYPE_BF16 && d.major == 10 && (a->max_in % 8) == 0 && (a->max_out % 8) == 0;
}

LinearProblem base_problem(const tp_linear_args* a) {
  LinearProblem p{};
  p.P = a->P;
  p.B = a->B;
  p.max_in = a->max_in;
  p.max_out = a->max_out;
  p.in_f = a->in_features;
  p.out_f = a->out_features;
  p.n_blocks = a->n_blocks;
  p.block_index = a->block_index;
  p.x_shared = a->x_shared;
  p.relu = a->relu;
  p.dropout_p = a->dropout_p;
  p.k0 = (uint32_t)(a->seed & 0xFFFFFFFFu);
  p.k1 = (uint32_t)(a->seed >> 32);
  philox_key_schedule(p.k0, p.k1, p.ks);
  p.offset = a->offset;
  p.member_base = a->member_base;
  p.bias = a->bias;
  p.bias_ld = a->max_out;
  return p;
}

struct MuonLayout {
  int R_s, C_s, tiles;
  size_t off_x0, off_x1, off_a, off_b, off_norm, off_rows, off_cols, off_trans, off_active, off_partial, off_counter,
      off_list[NS_LISTS], off_list_n, total;
};

constexpr int MUON_COUNTERS = 64;

// Workspace of Newton-Schulz operands for P members with (R_s, C_s) strides and
// `partials` per-tile norm partials.
MuonLayout muon_layout_rc(int P, int R_s, int C_s, size_t partials) {
  auto up = [](size_t v, size_t a) { return (v + a - 1) / a * a; };
  MuonLayout L{};
  L.R_s = R_s;
  L.C_s = C_s;
  size_t o = 0;
  auto take = [&](size_t bytes) { const size_t at = o; o = up(o + bytes, 256); return at; };
  L.off_x0 = take((size_t)P * L.R_s * L.C_s * 2);
  L.off_x1 = take((size_t)P * L.R_s * L.C_s * 2);
  L.off_a = take((size_t)P * L.R_s * L.R_s * 2);
  L.off_b = take((size_t)P * L.R_s * L.R_s * 2);
  L.off_norm = take((size_t)P * 4);
  L.off_rows = take((size_t)P * 4);
  L.off_cols = take((size_t)P * 4);
  L.off_trans = take((size_t)P * 4);
  L.off_active = take((size_t)P * 4);
  L.off_partial = take(partials * 4);
  L.off_counter = take(MUON_COUNTERS * 4);  // tile counters of the Newton-Schulz launches
  // dense tile lists of the Newton-Schulz launches (r x r and r x c outputs) and their lengths
  // (rr, rc, sym with 128-row tiles, then with 256-row tiles for CTA pairs)
  for (int g = 0; g < 2; ++g) {
    const size_t tm = (size_t)NS_TILE_M << g;
    const size_t mtl = ((size_t)L.R_s + tm - 1) / tm;
    L.off_list[3 * g] = take((size_t)P * mtl * ((L.R_s + NS_TILE_N - 1) / NS_TILE_N) * 4);
    L.off_list[3 * g + 1] = take((size_t)P * mtl * ((L.C_s + NS_TILE_N - 1) / NS_TILE_N) * 4);
    L.off_list[3 * g + 2] = take((size_t)P * mtl * ((L.R_s + NS_TILE_N - 1) / NS_TILE_N) * 4);
  }
  L.off_list_n = take(NS_LISTS * 4);
  L.total = o;
  return L;
}

// Operand strides of one group: r rounded to the 128-row tiles, c to the 256-column tiles.
int muon_rows_stride(int max_out, int max_in) { return (std::min(max_out, max_in) + 127) / 128 * 128; }
int muon_cols_stride(int max_out, int max_in) { return (std::max(max_out, max_in) + 255) / 256 * 256; }
int muon_prologue_tiles(int max_out, int max_in) {
  return ((max_out + MUON_TM - 1) / MUON_TM) * ((max_in + MUON_TN - 1) / MUON_TN);
}

MuonLayout muon_layout(int P, int max_out, int max_in) {
  const int tiles = muon_prologue_tiles(max_out, max_in);
  MuonLayout L = muon_layout_rc(P, muon_rows_stride(max_out, max_in), muon_cols_stride(max_out, max_in),
                                (size_t)P * tiles);
  L.tiles = tiles;
  return L;
}

// One Newton-Schulz GEMM over the pack: out = alpha * A_op B_op^T + beta * D.
template <int MODE>
int ns_gemm(const MuonArgs& ma, int shape, const void* a_op, int a_cols, const void* b_op, int b_cols,
            void* out, int out_cols, const void* d, float alpha, float beta, const uint32_t* list,
            const int* list_n, int* counter, cudaStream_t st, int sym = 0) {
  constexpr int BN = 256;
  static_assert(BN == NS_TILE_N && (Sm100Cfg<BN, MODE>::TILE_M == NS_TILE_M || Sm100Cfg<BN, MODE>::TILE_M == 2 * NS_TILE_M),
                "tile lists match the kernel's tiles");
  LinearProblem pr{};
  pr.tile_list = list;  // the launch's MMA tiles, claimed dynamically (ragged members)
  pr.tile_count = list_n;
  pr.ns_sym = sym;
  pr.tile_counter = counter;  // zeroed
  pr.mode = (MODE == MODE_NS_P) ? MODE_NS : (MODE == MODE_NS_BMN_P) ? MODE_NS_BMN : MODE;
  pr.P = ma.P;
  pr.ns_rows = ma.rows;
  pr.ns_cols = ma.cols;
  pr.active = ma.active;
  pr.ns_shape = shape;
  pr.alpha = alpha;
  pr.beta = beta;
  pr.D = d;
  pr.out = out;
  pr.out_rows = ma.R_s;
  pr.out_cols = out_cols;
  pr.out_ld = out_cols;
  pr.out_ms = (long long)ma.R_s * out_cols;
  using Cfg = Sm100Cfg<BN, MODE>;
  pr.BM = Cfg::TILE_M;
  pr.BN = BN;
  pr.m_tiles = (ma.R_s + Cfg::TILE_M - 1) / Cfg::TILE_M;
  pr.n_tiles = (out_cols + BN - 1) / BN;
  CUtensorMap mapA, mapB;
  int rc;
  if ((rc = make_map(&mapA, a_op, a_cols, ma.R_s, ma.P, 64, Cfg::BM))) return rc;
  if (!Cfg::B_MN) {
    if ((rc = make_map(&mapB, b_op, b_cols, ma.R_s, ma.P, 64, Cfg::B_ROWS))) return rc;
  } else {
    if ((rc = make_map(&mapB, b_op, b_cols, ma.R_s, ma.P, 64, 64))) return rc;
  }
  return launch_sm100<BN, MODE>(pr, mapA, mapB, st);
}

}  // namespace
}  // namespace tp

using namespace tp;

// Calls f(std::integral_constant<int, metric>) for a runtime metric code (kernels are
// specialised per metric).
template <typename F>
static void metric_dispatch(int metric, F f) {
  switch (metric) {
    case MET_MSE: f(std::integral_constant<int, MET_MSE>{}); break;
    case MET_MAE: f(std::integral_constant<int, MET_MAE>{}); break;
    case MET_ACCURACY: f(std::integral_constant<int, MET_ACCURACY>{}); break;
    case MET_BCE: f(std::integral_constant<int, MET_BCE>{}); break;
    case MET_CE: f(std::integral_constant<int, MET_CE>{}); break;
    case MET_ACCURACY_ARGMAX: f(std::integral_constant<int, MET_ACCURACY_ARGMAX>{}); break;
    default: f(std::integral_constant<int, MET_R2>{}); break;
  }
}

namespace tp {
namespace {
int linear_forward_impl(const tp_linear_args* a, const float* addend, int add_ld, void* stream);
int linear_backward_impl(const tp_linear_grad_args* ga, int dw_ld, void* stream);
}  // namespace
}  // namespace tp

extern "C" {

const char* tp_version(void) { return "tabpack_b200 0.1.0 (sm_100a)"; }

const char* tp_last_error_string(void) { return g_last_error.c_str(); }

int tp_device_error(void) {
  int v = 0;
  TP_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  const int zero = 0;
  TP_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  return v;
}

int tp_linear_forward(const tp_linear_args* a, void* stream) {
  return linear_forward_impl(a, nullptr, 0, stream);
}

int tp_profile_start(int32_t capacity) {
  if (capacity <= 0 || capacity > (1 << 20)) return fail(TP_EINVAL, "capacity must be in 1 .. 2^20 launches");
  if (g_prof_on.load()) return fail(TP_EINVAL, "profiling is already on");
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof_events.assign(2 * (size_t)capacity, nullptr);
  for (auto& e : g_prof_events) {
    const cudaError_t err = cudaEventCreate(&e);
    if (err != cudaSuccess) {
      for (auto& f : g_prof_events)
        if (f) cudaEventDestroy(f);
      g_prof_events.clear();
      return cuda_fail(err, "cudaEventCreate");
    }
  }
  g_prof_kind.assign((size_t)capacity, 0);
  g_prof_used = 0;
  g_prof_dropped = 0;
  g_prof_on.store(1);
  return TP_OK;
}

int tp_profile_stop(double* ms, int64_t* launches, int32_t n_kinds, int32_t* dropped) {
  if (!g_prof_on.load()) return fail(TP_EINVAL, "profiling is not on");
  g_prof_on.store(0);
  std::lock_guard<std::mutex> lk(g_prof_mu);
  int rc = TP_OK;
  for (int k = 0; k < n_kinds; ++k) {
    if (ms) ms[k] = 0.0;
    if (launches) launches[k] = 0;
  }
  for (int i = 0; i < g_prof_used && rc == TP_OK; ++i) {
    float t = 0.0f;
    cudaError_t err = cudaEventSynchronize(g_prof_events[2 * i + 1]);
    if (err == cudaSuccess) err = cudaEventElapsedTime(&t, g_prof_events[2 * i], g_prof_events[2 * i + 1]);
    if (err != cudaSuccess) {
      rc = cuda_fail(err, "reading a profiling event");
      break;
    }
    const int k = g_prof_kind[i];
    if (k >= 0 && k < n_kinds) {
      if (ms) ms[k] += t;
      if (launches) ++launches[k];
    }
  }
  if (dropped) *dropped = g_prof_dropped;
  for (auto& e : g_prof_events) cudaEventDestroy(e);
  g_prof_events.clear();
  g_prof_kind.clear();
  g_prof_used = 0;
  return rc;
}

}  // extern "C"

namespace tp {
namespace {

// The forward of tp_linear_forward; with `addend` (fp32 (P, B, add_ld)) the tensor-core
// forward adds it to the accumulator before the bias.
int linear_forward_impl(const tp_linear_args* a, const float* addend, int add_ld, void* stream) {
  int rc = check_linear(a);
  if (rc) return rc;
  if (!a->x || !a->y) return fail(TP_EINVAL, "x and y must be non-null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LinearProblem pr = base_problem(a);
  pr.addend = addend;
  pr.add_ld = add_ld;
  pr.mode = MODE_FWD;
  pr.skip_zero = a->y_pad_zero != 0;
  pr.out = a->y;
  pr.out_rows = a->B;
  pr.out_cols = a->max_out;
  pr.out_ld = a->max_out;
  pr.out_ms = (long long)a->B * a->max_out;
  pr.copy_src = a->x;
  pr.a_ptr = a->x;
  pr.b_ptr = a->w;
  if (a->n_blocks && a->x_shared) return fail(TP_EINVAL, "depth gating needs a per-member input");
  if (use_tensor_cores(a)) {
    if (!aligned16(a->x) || !aligned16(a->w) || !aligned16(a->y)) return fail(TP_EALIGN, "x, w, y must be 16-byte aligned");
    constexpr int BN = 256;
    using Cfg = Sm100Cfg<BN, MODE_FWD>;
    pr.BM = Cfg::TILE_M;
    pr.BN = BN;
    pr.m_tiles = (a->B + Cfg::TILE_M - 1) / Cfg::TILE_M;
    pr.n_tiles = (a->max_out + BN - 1) / BN;
    CUtensorMap ma, mb;
    if ((rc = make_map(&ma, a->x, a->max_in, a->B, a->x_shared ? 1 : a->P, 64, Cfg::BM))) return rc;
    if ((rc = make_map(&mb, a->w, a->max_in, a->max_out, a->P, 64, Cfg::B_ROWS))) return rc;
    static_assert(Sm100Cfg<BN, MODE_FWD_ADD>::TILE_M == Cfg::TILE_M && Sm100Cfg<BN, MODE_FWD_ADD>::B_ROWS == Cfg::B_ROWS,
                  "the forward with an addend shares the forward's tiling");
    if (addend != nullptr) return launch_sm100<BN, MODE_FWD_ADD>(pr, ma, mb, st);
    if (a->row_index) {  // A gathered from the table by row index, on single CTAs
      if ((rc = make_gather_map(&ma, a->x, a->max_in, a->x_rows))) return rc;
      pr.row_index = a->row_index;
      return launch_sm100<BN, MODE_FWD>(pr, ma, mb, st);
    }
    // CTA pairs (256-row tiles: a third less operand traffic per SM, more k-blocks in flight)
    // when there are no Philox draws, or when the K loop is long enough that operand delivery
    // rather than the dropout epilogue bounds the tile (a TabPack's first layer over its one-hot
    // columns); the keep mask depends only on (member, row, column), so it is the same either way
    if (a->dropout_p == nullptr || a->max_in >= 2048) {
      using CfgP = Sm100Cfg<BN, MODE_FWD_PAIR>;
      pr.BM = CfgP::TILE_M;
      pr.m_tiles = (a->B + CfgP::TILE_M - 1) / CfgP::TILE_M;
      CUtensorMap mbp;
      if ((rc = make_map(&mbp, a->w, a->max_in, a->max_out, a->P, 64, CfgP::B_ROWS))) return rc;
      return launch_sm100<BN, MODE_FWD_PAIR>(pr, ma, mbp, st);
    }
    return launch_sm100<BN, MODE_FWD>(pr, ma, mb, st);
  }
  if (addend != nullptr) return fail(TP_EUNSUPPORTED, "the gathered first layer runs on the sm_100 tensor-core path only");
  return a->dtype == TP_DTYPE_BF16 ? launch_simt<__nv_bfloat16, MODE_FWD>(pr, st) : launch_simt<float, MODE_FWD>(pr, st);
}

}  // namespace
}  // namespace tp

extern "C" {

int tp_linear_backward(const tp_linear_grad_args* ga, void* stream) { return linear_backward_impl(ga, 0, stream); }

}  // extern "C"

namespace tp {
namespace {

// tp_linear_backward with the row stride of dw given separately (dw_ld > dw_cols writes the
// first dw_cols columns of wider rows, e.g. the dense columns of a one-hot first layer).
int linear_backward_impl(const tp_linear_grad_args* ga, int dw_ld_in, void* stream) {
  if (!ga) return fail(TP_EINVAL, "null arguments");
  const tp_linear_args* a = &ga->fwd;
  int rc = check_linear(a);
  if (rc) return rc;
  if (!ga->dy) return fail(TP_EINVAL, "dy must be non-null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = a->dtype == TP_DTYPE_BF16;
  const bool need_g = a->relu || a->dropout_p || a->out_features || a->n_blocks;
  if (need_g && !ga->g) return fail(TP_EINVAL, "g workspace is required with relu, dropout, out_features or n_blocks");
  if ((a->relu) && !ga->y) return fail(TP_EINVAL, "y is required with relu");
  const void* G = need_g ? ga->g : ga->dy;

  // 1. g = dy * activation'(.) and dbias = sum_rows g
  if (!ga->g_ready && (need_g || ga->dbias)) {
    ActBwdArgs aa{};
    aa.P = a->P;
    aa.B = a->B;
    aa.W = a->max_out;
    aa.out_f = a->out_features;
    aa.n_blocks = a->n_blocks;
    aa.block_index = a->block_index;
    aa.relu = a->relu;
    aa.dropout_p = a->dropout_p;
    aa.k0 = (uint32_t)(a->seed & 0xFFFFFFFFu);
    aa.k1 = (uint32_t)(a->seed >> 32);
    aa.offset = a->offset;
    aa.member_base = a->member_base;
    aa.dy = ga->dy;
    aa.y = ga->y ? ga->y : ga->dy;
    aa.g = need_g ? ga->g : nullptr;
    aa.dbias = ga->dbias;
    aa.db_cols = ga->db_cols > 0 ? ga->db_cols : a->max_out;
    dim3 grid((a->max_out + 63) / 64, a->P);
    const bool vec = (a->max_out % 8) == 0 && aligned16(ga->dy) && aligned16(aa.y) && (!aa.g || aligned16(aa.g));
    TP_PROF(TP_PROF_ACT_BACKWARD, st);
    if (bf16) {
      if (vec) act_backward_kernel<__nv_bfloat16, true><<<grid, 256, 0, st>>>(aa);
      else act_backward_kernel<__nv_bfloat16, false><<<grid, 256, 0, st>>>(aa);
    } else {
      if (vec) act_backward_kernel<float, true><<<grid, 256, 0, st>>>(aa);
      else act_backward_kernel<float, false><<<grid, 256, 0, st>>>(aa);
    }
    TP_CUDA_TRY(cudaGetLastError());
  }

  const bool tc = use_tensor_cores(a);
  // 2. dx = g w   (dx = dy for depth-inactive members); with dx_cols, the input columns from
  // dx_cols on are written as zeros without their GEMM tiles
  if (ga->dx && a->row_index) return fail(TP_EINVAL, "a gathered input (a table) takes no input gradient");
  if (ga->dx) {
    if (ga->dx_cols < 0 || (ga->dx_cols > 0 && (a->in_features || a->n_blocks)))
      return fail(TP_EINVAL, "dx_cols needs a layer without per-member input widths or depth gating");
    LinearProblem pr = base_problem(a);
    const bool dx_part = ga->dx_cols > 0 && ga->dx_cols < a->max_in;
    // tensor cores: the members' input width (tiles past it are zero tiles)
    if (dx_part && tc) pr.max_in = ga->dx_cols;
    pr.mode = MODE_DGRAD;
    pr.skip_zero = ga->dx_pad_zero != 0;
    pr.out = ga->dx;
    pr.out_rows = a->B;
    pr.out_cols = a->max_in;
    pr.out_ld = a->max_in;
    pr.out_ms = (long long)a->B * a->max_in;
    pr.copy_src = ga->dy;
    pr.a_ptr = G;
    pr.b_ptr = a->w;
    pr.dropout_p = nullptr;
    if (tc) {
      if (!aligned16(G) || !aligned16(a->w) || !aligned16(ga->dx)) return fail(TP_EALIGN, "g, w, dx must be 16-byte aligned");
      constexpr int BN = 256;
      using Cfg = Sm100Cfg<BN, MODE_DGRAD>;
      pr.BM = Cfg::TILE_M;
      pr.BN = BN;
      pr.m_tiles = (a->B + Cfg::TILE_M - 1) / Cfg::TILE_M;
      pr.n_tiles = (a->max_in + BN - 1) / BN;
      CUtensorMap ma, mb;
      if ((rc = make_map(&ma, G, a->max_out, a->B, a->P, 64, Cfg::BM))) return rc;
      if ((rc = make_map(&mb, a->w, a->max_in, a->max_out, a->P, 64, 64))) return rc;
      if ((rc = launch_sm100<BN, MODE_DGRAD>(pr, ma, mb, st))) return rc;
    } else {
      rc = bf16 ? launch_simt<__nv_bfloat16, MODE_DGRAD>(pr, st) : launch_simt<float, MODE_DGRAD>(pr, st);
      if (rc) return rc;
      if (dx_part) {  // the CUDA-core path computes every column: clear the tail
        const size_t es = bf16 ? 2 : 4;
        TP_CUDA_TRY(cudaMemset2DAsync(static_cast<char*>(ga->dx) + ga->dx_cols * es, a->max_in * es, 0,
                                      (a->max_in - ga->dx_cols) * es, (size_t)a->P * a->B, st));
      }
    }
  }
  // 3. dw = g^T x
  if (ga->dw) {
    if (!a->x) return fail(TP_EINVAL, "x is required for the weight gradient");
    const int dw_rows = ga->dw_rows > 0 ? ga->dw_rows : a->max_out;
    const int dw_cols = ga->dw_cols > 0 ? ga->dw_cols : a->max_in;
    const int dw_ld = dw_ld_in > 0 ? dw_ld_in : dw_cols;
    if (dw_rows > a->max_out || dw_cols > a->max_in) return fail(TP_EINVAL, "dw is larger than the weight storage");
    if (dw_ld < dw_cols) return fail(TP_EINVAL, "dw row stride below its columns");
    LinearProblem pr = base_problem(a);
    pr.mode = MODE_WGRAD;
    pr.skip_zero = ga->dw_pad_zero != 0;
    pr.out = ga->dw;
    pr.out_rows = dw_rows;
    pr.out_cols = dw_cols;
    pr.out_ld = dw_ld;
    pr.out_ms = (long long)dw_rows * dw_ld;
    pr.copy_src = nullptr;
    pr.a_ptr = G;
    pr.b_ptr = a->x;
    pr.dropout_p = nullptr;
    if (tc) {
      if (!aligned16(G) || !aligned16(a->x)) return fail(TP_EALIGN, "g and x must be 16-byte aligned");
      // transposed on CTA pairs: rows of the tile are input features (the full input width
      // in 256-row pair tiles), columns the member's output features (trimmed to 32)
      constexpr int BN = 256;
      using Cfg = Sm100Cfg<BN, MODE_WGRAD_T>;
      pr.mode = MODE_WGRAD_T;
      pr.BM = Cfg::TILE_M;
      pr.BN = BN;
      pr.m_tiles = (dw_cols + Cfg::TILE_M - 1) / Cfg::TILE_M;
      pr.n_tiles = (dw_rows + BN - 1) / BN;
      CUtensorMap ma, mb;
      if ((rc = make_map(&mb, G, a->max_out, a->B, a->P, 64, 64))) return rc;
      if (a->row_index) {  // X gathered from the table by row index, on single CTAs
        using CfgG = Sm100Cfg<BN, MODE_WGRAD_TG>;
        pr.BM = CfgG::TILE_M;
        pr.m_tiles = (dw_cols + CfgG::TILE_M - 1) / CfgG::TILE_M;
        pr.row_index = a->row_index;
        if ((rc = make_gather_map(&ma, a->x, a->max_in, a->x_rows))) return rc;
        if ((rc = launch_sm100<BN, MODE_WGRAD_TG>(pr, ma, mb, st))) return rc;
      } else {
        if ((rc = make_map(&ma, a->x, a->max_in, a->B, a->x_shared ? 1 : a->P, 64, 64))) return rc;
        if ((rc = launch_sm100<BN, MODE_WGRAD_T>(pr, ma, mb, st))) return rc;
      }
    } else {
      rc = bf16 ? launch_simt<__nv_bfloat16, MODE_WGRAD>(pr, st) : launch_simt<float, MODE_WGRAD>(pr, st);
      if (rc) return rc;
    }
  }
  return TP_OK;
}

}  // namespace
}  // namespace tp

extern "C" {

int tp_linear_backward_noalloc(const tp_linear_grad_args* ga, void* stream) {
  if (!ga) return fail(TP_EINVAL, "null arguments");
  if (ga->g) return fail(TP_EINVAL, "tp_linear_backward_noalloc uses its own workspace: pass g = NULL");
  const tp_linear_args* a = &ga->fwd;
  int rc = check_linear(a);
  if (rc) return rc;
  tp_linear_grad_args b = *ga;
  b.g_ready = 0;
  const bool need_g = a->relu || a->dropout_p || a->out_features || a->n_blocks;
  if (need_g) {
    const unsigned long long elem = a->dtype == TP_DTYPE_BF16 ? 2ull : 4ull;
    const unsigned long long bytes = (unsigned long long)a->P * (unsigned long long)a->B *
                                     (unsigned long long)a->max_out * elem;
    if (bytes > (unsigned long long)TP_NOALLOC_SCRATCH_BYTES)
      return fail(TP_EINVAL,
                  "tp_linear_backward_noalloc: P*B*max_out = %d*%d*%d elements need %llu bytes of workspace, "
                  "more than the %u-byte built-in scratch; use tp_linear_backward with a caller-provided g",
                  a->P, a->B, a->max_out, bytes, (unsigned)TP_NOALLOC_SCRATCH_BYTES);
    void* scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch))) return rc;
    b.g = scratch;
  }
  return tp_linear_backward(&b, stream);
}

size_t tp_muon_workspace_size(int32_t P, int32_t max_out, int32_t max_in) {
  if (P <= 0 || max_out <= 0 || max_in <= 0) return 0;
  return muon_layout(P, max_out, max_in).total;
}

}  // extern "C"

namespace tp {
namespace {

// Checks one group's arguments and fills the per-group fields of m (hyperparameters, tensors,
// the bf16 copy, depth gating); the workspace fields are set by the caller.
int muon_group_args(const tp_muon_args* a, MuonArgs* out) {
  if (!a || a->P <= 0 || a->max_out <= 0 || a->max_in <= 0) return fail(TP_EINVAL, "bad Muon shapes");
  if (!a->p || !a->grad || !a->momentum_buffer) return fail(TP_EINVAL, "null Muon tensor");
  if (a->ns_steps < 0) return fail(TP_EINVAL, "negative Newton-Schulz step count");
  if (a->P > 65535) return fail(TP_EINVAL, "at most 65535 members per Muon call");
  if (a->p_bf16 != nullptr && (a->p_bf16_rows < a->max_out || a->p_bf16_cols < a->max_in))
    return fail(TP_EINVAL, "the bf16 copy (%d x %d per member) is smaller than p (%d x %d)", a->p_bf16_rows,
                a->p_bf16_cols, a->max_out, a->max_in);
  MuonArgs m{};
  m.P = a->P;
  m.max_out = a->max_out;
  m.max_in = a->max_in;
  m.p = a->p;
  m.g = a->grad;
  m.m = a->momentum_buffer;
  m.out_f = a->out_features;
  m.in_f = a->in_features;
  m.lr_pm = a->lr.per_member;
  m.lr_s = (float)a->lr.scalar;
  m.mu_pm = a->momentum.per_member;
  m.mu_s = (float)a->momentum.scalar;
  m.wd_pm = a->weight_decay.per_member;
  m.wd_s = (float)a->weight_decay.scalar;
  const bool lr_zero = !a->lr.per_member && a->lr.scalar == 0.0;
  const bool wd_zero = !a->weight_decay.per_member && a->weight_decay.scalar == 0.0;
  m.wd_on = !(lr_zero || wd_zero);
  m.wd_mult_s = (float)(1.0 - a->lr.scalar * a->weight_decay.scalar);
  m.one_m_mu_s = (float)(1.0 - a->momentum.scalar);
  m.scale_pm = a->update_scale;
  m.scale_s = (float)std::sqrt(std::max(1.0, (double)a->max_out / (double)a->max_in));
  m.nesterov = a->nesterov;
  m.mutate_grad = a->mutate_grad;
  m.p_bf16 = static_cast<__nv_bfloat16*>(a->p_bf16);
  m.n_blocks = a->n_blocks;
  m.block_index = a->block_index;
  m.gated_zero = a->n_blocks != nullptr && a->gated_momentum_zero != 0;
  m.bf16_rows = a->p_bf16_rows;
  m.bf16_cols = a->p_bf16_cols;
  *out = m;
  return TP_OK;
}

// Points a group's MuonArgs at members [first, first + P) of a workspace laid out by L, whose
// per-tile norm partials start at partial element `partial_first`.
void muon_bind(MuonArgs& m, const MuonLayout& L, uint8_t* ws, int first, size_t partial_first, int tiles) {
  m.R_s = L.R_s;
  m.C_s = L.C_s;
  m.x = reinterpret_cast<__nv_bfloat16*>(ws + L.off_x0) + (size_t)first * L.R_s * L.C_s;
  m.norm2 = reinterpret_cast<float*>(ws + L.off_norm) + first;
  m.rows = reinterpret_cast<int32_t*>(ws + L.off_rows) + first;
  m.cols = reinterpret_cast<int32_t*>(ws + L.off_cols) + first;
  m.trans = reinterpret_cast<int32_t*>(ws + L.off_trans) + first;
  m.active = reinterpret_cast<int32_t*>(ws + L.off_active) + first;
  m.partial = reinterpret_cast<float*>(ws + L.off_partial) + partial_first;
  m.tiles = tiles;
}

// Momentum, the oriented bf16 operand and its Frobenius normalisation for one bound group;
// (rows_ext, cols_ext) bound the normalisation grid (the group's own operand extent).
void muon_prepare(const MuonArgs& m, int rows_ext, int cols_ext, cudaStream_t st) {
  dim3 tiles((m.max_in + MUON_TN - 1) / MUON_TN, (m.max_out + MUON_TM - 1) / MUON_TM, m.P);
  dim3 ngrid((cols_ext + 255) / 256, (rows_ext + MUON_NORM_ROWS - 1) / MUON_NORM_ROWS, m.P);
  TP_PROF(TP_PROF_MUON_ELEMENTWISE, st);
  muon_geometry_kernel<<<(m.P + 255) / 256, 256, 0, st>>>(m);
  muon_prologue_kernel<<<tiles, 256, 0, st>>>(m);
  muon_norm_kernel<<<m.P, 256, 0, st>>>(m, (int)tiles.x);
  muon_normalize_kernel<<<ngrid, 256, 0, st>>>(m, 128, 256);
}

// The scaled update (and bf16 copy) of one bound group from the Newton-Schulz result x.
void muon_finish(MuonArgs m, __nv_bfloat16* x, cudaStream_t st) {
  m.x = x;
  dim3 tiles((m.max_in + MUON_TN - 1) / MUON_TN, (m.max_out + MUON_TM - 1) / MUON_TM, m.P);
  TP_PROF(TP_PROF_MUON_ELEMENTWISE, st);
  muon_apply_kernel<<<tiles, 256, 0, st>>>(m);
}

// ns_steps quintic Newton-Schulz iterations over every member of the workspace (mu: the
// workspace-wide view: P, rows, cols, active, R_s); *result receives the final operand.
// Bit mask of the Newton-Schulz products that run on CTA pairs (bit 0: A = X X^T, bit 1:
// B = b A + c A^2, bit 2: X <- a X + B X); the environment variable TP_NS_PAIRS (read once)
// overrides the default.  Both kernels compute every tile the same way, so the choice does not
// change the results.
int ns_pair_products() {
  static const int mask = [] {
    const char* e = std::getenv("TP_NS_PAIRS");
    if (e == nullptr || *e == 0) return 7;
    return (int)(std::strtol(e, nullptr, 0) & 7);
  }();
  return mask;
}

int muon_newton_schulz(const MuonArgs& mu, const MuonLayout& L, uint8_t* ws, int ns_steps, cudaStream_t st,
                       void** result) {
  if (L.R_s / NS_TILE_M > 255 || (L.C_s + NS_TILE_N - 1) / NS_TILE_N > 255)
    return fail(TP_EINVAL, "Muon matrices of at most 32640 x 65280 elements (operand strides %d x %d)", L.R_s,
                L.C_s);
  NsTileLists lists{};
  for (int j = 0; j < NS_LISTS; ++j) lists.list[j] = reinterpret_cast<uint32_t*>(ws + L.off_list[j]);
  lists.counts = reinterpret_cast<int*>(ws + L.off_list_n);
  const int* list_n = lists.counts;
  // which of the three products run on CTA pairs (256-row tiles)
  const int pairs = ns_pair_products();
  lists.build[0] = (pairs & 7) != 7;
  lists.build[1] = (pairs & 7) != 0;
  {
    TP_PROF(TP_PROF_MUON_ELEMENTWISE, st);
    ns_tile_list_kernel<<<1, 1024, 0, st>>>(mu, lists);
  }
  TP_CUDA_TRY(cudaGetLastError());
  // quintic Newton-Schulz, coefficients of optim.py:477
  const float ca = 3.4445f, cb = -4.7750f, cc = 2.0315f;
  void* X = ws + L.off_x0;
  void* Xn = ws + L.off_x1;
  void* A = ws + L.off_a;
  void* Bm = ws + L.off_b;
  int rc;
  // one zeroed tile counter per Newton-Schulz launch (the block is re-zeroed when it wraps;
  // stream order keeps the earlier launches' use of a counter before its memset)
  int* counters = reinterpret_cast<int*>(ws + L.off_counter);
  int launch = 0;
  auto counter = [&]() -> int* {
    if (launch % MUON_COUNTERS == 0 && cudaMemsetAsync(counters, 0, MUON_COUNTERS * 4, st) != cudaSuccess)
      return nullptr;
    return counters + (launch++ % MUON_COUNTERS);
  };
  const int sym_l = (pairs & 1) ? 5 : 2, b_l = (pairs & 2) ? 5 : 2, x_l = (pairs & 4) ? 4 : 1;
  for (int it = 0; it < ns_steps; ++it) {
    int* c1 = counter();
    int* c2 = counter();
    int* c3 = counter();
    if (!c1 || !c2 || !c3) return fail(TP_ECUDA, "cudaMemsetAsync of the tile counters failed");
    // A = X X^T is symmetric: only the tiles not below the diagonal, the rest written as transposes
    rc = (pairs & 1) ? ns_gemm<MODE_NS_P>(mu, 1, X, L.C_s, X, L.C_s, A, L.R_s, nullptr, 1.0f, 0.0f, lists.list[sym_l],
                                          list_n + sym_l, c1, st, 1)
                     : ns_gemm<MODE_NS>(mu, 1, X, L.C_s, X, L.C_s, A, L.R_s, nullptr, 1.0f, 0.0f, lists.list[sym_l],
                                        list_n + sym_l, c1, st, 1);
    if (rc) return rc;
    // B = b A + c A^2 is symmetric as well
    rc = (pairs & 2) ? ns_gemm<MODE_NS_P>(mu, 2, A, L.R_s, A, L.R_s, Bm, L.R_s, A, cc, cb, lists.list[b_l],
                                          list_n + b_l, c2, st, 1)
                     : ns_gemm<MODE_NS>(mu, 2, A, L.R_s, A, L.R_s, Bm, L.R_s, A, cc, cb, lists.list[b_l], list_n + b_l,
                                        c2, st, 1);
    if (rc) return rc;
    rc = (pairs & 4) ? ns_gemm<MODE_NS_BMN_P>(mu, 3, Bm, L.R_s, X, L.C_s, Xn, L.C_s, X, 1.0f, ca, lists.list[x_l],
                                              list_n + x_l, c3, st)
                     : ns_gemm<MODE_NS_BMN>(mu, 3, Bm, L.R_s, X, L.C_s, Xn, L.C_s, X, 1.0f, ca, lists.list[x_l],
                                            list_n + x_l, c3, st);
    if (rc) return rc;
    std::swap(X, Xn);
  }
  *result = X;
  return TP_OK;
}

int muon_check_device_and_workspace(const void* workspace, size_t have, size_t need) {
  if (device_info().major != 10) return fail(TP_EUNSUPPORTED, "Newton-Schulz GEMMs need an sm_100 device");
  if (!workspace) return fail(TP_EINVAL, "null Muon workspace");
  if (have < need) return fail(TP_EINVAL, "Muon workspace holds %zu bytes, needs %zu", have, need);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return fail(TP_EALIGN, "workspace must be 256-byte aligned");
  return TP_OK;
}

// Layout of a grouped call: every group's members one after another, common operand strides
// (the largest group's), each group's norm partials after the previous group's.
MuonLayout muon_grouped_layout(const tp_muon_args* g, int n) {
  int P = 0, R = 0, C = 0;
  size_t partials = 0;
  for (int i = 0; i < n; ++i) {
    P += g[i].P;
    R = std::max(R, muon_rows_stride(g[i].max_out, g[i].max_in));
    C = std::max(C, muon_cols_stride(g[i].max_out, g[i].max_in));
    partials += (size_t)g[i].P * muon_prologue_tiles(g[i].max_out, g[i].max_in);
  }
  return muon_layout_rc(P, R, C, partials);
}

}  // namespace
}  // namespace tp

extern "C" {

int tp_muon_step(const tp_muon_args* a, void* stream) {
  MuonArgs m{};
  int rc;
  if ((rc = muon_group_args(a, &m))) return rc;
  const MuonLayout L = muon_layout(a->P, a->max_out, a->max_in);
  if ((rc = muon_check_device_and_workspace(a->workspace, a->workspace_bytes, L.total))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  muon_bind(m, L, ws, 0, 0, L.tiles);
  muon_prepare(m, L.R_s, L.C_s, st);
  TP_CUDA_TRY(cudaGetLastError());
  void* X = nullptr;
  if ((rc = muon_newton_schulz(m, L, ws, a->ns_steps, st, &X))) return rc;
  muon_finish(m, static_cast<__nv_bfloat16*>(X), st);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

size_t tp_muon_grouped_workspace_size(const tp_muon_args* groups, int32_t n_groups) {
  if (!groups || n_groups <= 0) return 0;
  for (int i = 0; i < n_groups; ++i)
    if (groups[i].P <= 0 || groups[i].max_out <= 0 || groups[i].max_in <= 0) return 0;
  return muon_grouped_layout(groups, n_groups).total;
}

int tp_muon_step_grouped(const tp_muon_args* groups, int32_t n_groups, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (!groups || n_groups <= 0) return fail(TP_EINVAL, "no Muon groups");
  std::vector<MuonArgs> ms((size_t)n_groups);
  int rc;
  long long P = 0;
  for (int i = 0; i < n_groups; ++i) {
    if ((rc = muon_group_args(&groups[i], &ms[(size_t)i]))) return rc;
    if (groups[i].ns_steps != groups[0].ns_steps)
      return fail(TP_EINVAL, "grouped Muon steps share one Newton-Schulz step count (group %d: %d, group 0: %d)", i,
                  groups[i].ns_steps, groups[0].ns_steps);
    P += groups[i].P;
  }
  if (P > 65535) return fail(TP_EINVAL, "at most 65535 members over the groups of one grouped Muon call");
  const MuonLayout L = muon_grouped_layout(groups, n_groups);
  if ((rc = muon_check_device_and_workspace(workspace, workspace_bytes, L.total))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int first = 0;
  size_t partial_first = 0;
  for (int i = 0; i < n_groups; ++i) {
    const tp_muon_args& g = groups[i];
    const int tiles = muon_prologue_tiles(g.max_out, g.max_in);
    muon_bind(ms[(size_t)i], L, ws, first, partial_first, tiles);
    muon_prepare(ms[(size_t)i], muon_rows_stride(g.max_out, g.max_in), muon_cols_stride(g.max_out, g.max_in), st);
    first += g.P;
    partial_first += (size_t)g.P * tiles;
  }
  TP_CUDA_TRY(cudaGetLastError());
  // the Newton-Schulz launches run over the members of every group at once
  MuonArgs mu{};
  muon_bind(mu, L, ws, 0, 0, 0);
  mu.P = (int)P;
  void* X = nullptr;
  if ((rc = muon_newton_schulz(mu, L, ws, groups[0].ns_steps, st, &X))) return rc;
  first = 0;
  for (int i = 0; i < n_groups; ++i) {
    muon_finish(ms[(size_t)i], static_cast<__nv_bfloat16*>(X) + (size_t)first * L.R_s * L.C_s, st);
    first += groups[i].P;
  }
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int tp_metric_pack(const tp_metric_args* a, void* stream) {
  TP_PROF(TP_PROF_METRIC, static_cast<cudaStream_t>(stream));
  if (!a || a->P <= 0 || a->N <= 0 || !a->y_pred || !a->y_true || !a->out) return fail(TP_EINVAL, "bad metric arguments");
  if (a->metric < TP_METRIC_MSE || a->metric > TP_METRIC_R2) return fail(TP_EINVAL, "unknown metric %d", a->metric);
  MetricSrc s{};
  s.metric = a->metric;
  s.N = a->N;
  s.C = (a->metric == TP_METRIC_CE || a->metric == TP_METRIC_ACCURACY_ARGMAX) ? std::max(1, a->C) : 1;
  const bool float_labels = a->metric == TP_METRIC_MSE || a->metric == TP_METRIC_MAE || a->metric == TP_METRIC_R2;
  s.yf = float_labels ? static_cast<const float*>(a->y_true) : nullptr;
  s.yi = float_labels ? nullptr : static_cast<const int64_t*>(a->y_true);
  const bool int_pred = a->metric == TP_METRIC_ACCURACY;
  metric_dispatch(a->metric, [&](auto tag) {
    metric_pack_kernel<decltype(tag)::value><<<a->P, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
        s, int_pred ? nullptr : static_cast<const float*>(a->y_pred),
        int_pred ? static_cast<const int64_t*>(a->y_pred) : nullptr, a->out);
  });
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

constexpr int64_t GREEDY_SEG_ROWS = 16384;  // rows per block of the candidate scoring launch

static int greedy_segments(int64_t N) { return (int)((N + GREEDY_SEG_ROWS - 1) / GREEDY_SEG_ROWS); }

static size_t greedy_layout(int32_t n_pred, int64_t N, int32_t C, size_t* off_ens, size_t* off_sc, size_t* off_ind,
                            size_t* off_st, size_t* off_init, size_t* off_metric, size_t* off_part) {
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  size_t o = 0;
  *off_ens = o;
  o = up(o + (size_t)N * C * 4);
  *off_sc = o;
  o = up(o + (size_t)n_pred * 8);
  *off_ind = o;
  o = up(o + (size_t)n_pred * 8);
  *off_st = o;
  o = up(o + sizeof(GreedyState));
  *off_init = o;
  o = up(o + (size_t)n_pred * 4);
  *off_metric = o;
  o = up(o + (size_t)n_pred * 4);
  *off_part = o;
  o = up(o + (size_t)n_pred * greedy_segments(N) * 8);
  return o;
}

size_t tp_greedy_workspace_size(int32_t n_pred, int64_t N, int32_t C) {
  if (n_pred <= 0 || N <= 0 || C <= 0) return 0;
  size_t a, b, c, d, e, f, h;
  return greedy_layout(n_pred, N, C, &a, &b, &c, &d, &e, &f, &h);
}

int tp_greedy_ensemble(const tp_greedy_args* a, void* stream) {
  TP_PROF(TP_PROF_GREEDY, static_cast<cudaStream_t>(stream));
  if (!a || a->n_pred <= 0 || a->N <= 0 || !a->predictions || !a->y_true || !a->counts || !a->workspace || !a->status)
    return fail(TP_EINVAL, "bad greedy arguments");
  if (a->metric == TP_METRIC_ACCURACY || a->metric == TP_METRIC_R2 || a->metric < 0 || a->metric > TP_METRIC_R2)
    return fail(TP_EINVAL, "metric %d is not supported by the fused greedy selection", a->metric);
  if (a->init_top_k <= 0) return fail(TP_EINVAL, "`init_top_k` must be positive to initialize the ensemble with at least one member");
  if (a->with_replacement && a->max_ensemble_size <= 0)
    return fail(TP_EINVAL, "Set `max_ensemble_size` to limit the number of ensemble members when `with_replacement=True`");
  if (a->max_ensemble_size > 0 && a->init_top_k > a->max_ensemble_size)
    return fail(TP_EINVAL, "`init_top_k` must not exceed `max_ensemble_size`");
  const int C = std::max(1, a->C);
  size_t o_ens, o_sc, o_ind, o_st, o_init, o_met, o_part;
  const size_t need = greedy_layout(a->n_pred, a->N, C, &o_ens, &o_sc, &o_ind, &o_st, &o_init, &o_met, &o_part);
  if (a->workspace_bytes < need) return fail(TP_EINVAL, "greedy workspace holds %zu bytes, needs %zu", a->workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  GreedyArgs g{};
  g.s.metric = a->metric;
  g.s.N = a->N;
  g.s.C = (a->metric == TP_METRIC_CE || a->metric == TP_METRIC_ACCURACY_ARGMAX) ? C : 1;
  const bool float_labels = a->metric == TP_METRIC_MSE || a->metric == TP_METRIC_MAE;
  g.s.yf = float_labels ? static_cast<const float*>(a->y_true) : nullptr;
  g.s.yi = float_labels ? nullptr : static_cast<const int64_t*>(a->y_true);
  g.Cand = a->n_pred;
  g.pred = a->predictions;
  g.sign = a->maximize ? 1 : -1;
  g.with_replacement = a->with_replacement;
  g.limit = a->max_ensemble_size <= 0 ? a->n_pred
            : a->with_replacement   ? a->max_ensemble_size
                                    : std::min(a->n_pred, a->max_ensemble_size);
  g.counts = a->counts;
  g.ens = reinterpret_cast<float*>(ws + o_ens);
  g.scores = reinterpret_cast<double*>(ws + o_sc);
  g.S = greedy_segments(a->N);
  g.seg = GREEDY_SEG_ROWS;
  g.partials = reinterpret_cast<double*>(ws + o_part);
  g.ind_scores = reinterpret_cast<double*>(ws + o_ind);
  g.st = reinterpret_cast<GreedyState*>(ws + o_st);
  int* init_idx = reinterpret_cast<int*>(ws + o_init);
  float* metric = reinterpret_cast<float*>(ws + o_met);
  const int k = std::min(a->init_top_k, a->n_pred);
  TP_CUDA_TRY(cudaMemsetAsync(a->counts, 0, (size_t)a->n_pred * 4, st));
  // individual scores
  metric_dispatch(g.s.metric, [&](auto tag) {
    metric_pack_kernel<decltype(tag)::value><<<a->n_pred, 1024, 0, st>>>(g.s, a->predictions, nullptr, metric);
  });
  greedy_sign_kernel<<<(a->n_pred + 255) / 256, 256, 0, st>>>(metric, g.ind_scores, a->n_pred, g.sign);
  greedy_init_select_kernel<<<1, 32, 0, st>>>(g, k, init_idx);
  const int64_t n = a->N * (int64_t)g.s.C;
  const int eb = (int)std::min<int64_t>((n + 255) / 256, 1184);
  greedy_init_mean_kernel<<<eb, 256, 0, st>>>(g, k, init_idx);
  metric_dispatch(g.s.metric, [&](auto tag) { greedy_init_score_kernel<decltype(tag)::value><<<1, 1024, 0, st>>>(g); });
  TP_CUDA_TRY(cudaGetLastError());
  for (int it = k; it < g.limit; ++it) {
    metric_dispatch(g.s.metric, [&](auto tag) {
      greedy_score_kernel<decltype(tag)::value><<<dim3(a->n_pred, g.S), 256, 0, st>>>(g);
    });
    greedy_select_kernel<<<1, 1024, 0, st>>>(g);
    greedy_update_kernel<<<eb, 256, 0, st>>>(g);
    greedy_advance_kernel<<<1, 1, 0, st>>>(g);
  }
  TP_CUDA_TRY(cudaGetLastError());
  // status: iterations, distinct members, error
  TP_CUDA_TRY(cudaMemcpyAsync(a->status, &g.st->iters, 4, cudaMemcpyDeviceToDevice, st));
  TP_CUDA_TRY(cudaMemcpyAsync(a->status + 1, &g.st->size, 4, cudaMemcpyDeviceToDevice, st));
  TP_CUDA_TRY(cudaMemcpyAsync(a->status + 2, &g.st->error, 4, cudaMemcpyDeviceToDevice, st));
  return TP_OK;
}

int tp_ensemble_mean(const float* pred, const int32_t* idx, const float* weights, int32_t K, int64_t n, float* out,
                     void* stream) {
  TP_PROF(TP_PROF_OTHER, static_cast<cudaStream_t>(stream));
  if (!pred || !idx || !out || K <= 0 || n <= 0) return fail(TP_EINVAL, "bad ensemble-mean arguments");
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
  ensemble_mean_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(pred, idx, weights, K, n, out);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int tp_softmax_rows(const float* x, int64_t rows, int32_t C, float* out, void* stream) {
  TP_PROF(TP_PROF_OTHER, static_cast<cudaStream_t>(stream));
  if (!x || !out || rows <= 0 || C <= 0) return fail(TP_EINVAL, "bad softmax arguments");
  const int64_t threads = rows * 32;
  const int blocks = (int)std::min<int64_t>((threads + 255) / 256, 1 << 20);
  if ((int64_t)blocks * 256 < threads) return fail(TP_EINVAL, "too many rows for one softmax call");
  softmax_rows_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, rows, C, out);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

// Row segments of the embedding backward: enough blocks to fill 148 SMs (16 blocks of 128
// threads each), at least 64 rows per segment.
static int cos_emb_segments(int P, int B, int F, int D) {
  const long long cols = ((long long)F * D + COS_EMB_THREADS - 1) / COS_EMB_THREADS;
  const long long base = cols * P;
  // about four waves of 128-thread blocks (16 per SM): a single wave left a third of it as tail
  long long s = (148 * 16 * 4 + base - 1) / base;
  s = std::min<long long>(s, (B + 63) / 64);
  return (int)std::max<long long>(1, s);
}

static int check_cos_emb(const tp_cos_emb_args* a) {
  if (!a) return fail(TP_EINVAL, "null embedding arguments");
  if (a->P <= 0 || a->B <= 0 || a->F <= 0 || a->D <= 0)
    return fail(TP_EINVAL, "embedding needs P, B, F, D > 0 (got %d, %d, %d, %d)", a->P, a->B, a->F, a->D);
  if (!a->x || !a->affine_weight || !a->affine_bias || (a->D > 1 && (!a->weight || !a->bias)))
    return fail(TP_EINVAL, "null embedding parameter");
  return TP_OK;
}

static CosEmbArgs cos_emb_args(const tp_cos_emb_args* a) {
  CosEmbArgs k{};
  k.P = a->P;
  k.B = a->B;
  k.F = a->F;
  k.D = a->D;
  k.x_shared = a->x_shared;
  k.x = a->x;
  k.w = a->weight;
  k.b = a->bias;
  k.aw = a->affine_weight;
  k.ab = a->affine_bias;
  k.d_emb = a->d_embedding;
  k.out = a->out;
  k.out_ld = a->out_ld;
  k.out_bf16 = a->out_dtype == TP_DTYPE_BF16;
  k.g = a->grad_out;
  k.g_ld = a->grad_ld;
  k.g_bf16 = a->grad_dtype == TP_DTYPE_BF16;
  k.dw = a->dweight;
  k.db = a->dbias;
  k.daw = a->daffine_weight;
  k.dab = a->daffine_bias;
  return k;
}

size_t tp_cos_emb_workspace_size(int32_t P, int32_t B, int32_t F, int32_t D) {
  if (P <= 0 || B <= 0 || F <= 0 || D <= 0) return 0;
  const int s = cos_emb_segments(P, B, F, D);
  return s > 1 ? (size_t)4 * s * P * (size_t)F * D * sizeof(double) : 0;
}

int tp_tabpack_input(const tp_input_args* a, void* stream) {
  TP_PROF(TP_PROF_INPUT, static_cast<cudaStream_t>(stream));
  if (!a || a->rows <= 0 || a->n_num < 0 || a->n_cat < 0 || !a->out) return fail(TP_EINVAL, "bad input arguments");
  if (a->n_num > 0 && !a->x_num) return fail(TP_EINVAL, "x_num is null");
  if (a->n_cat > 0 && (!a->x_cat || !a->cat_offsets)) return fail(TP_EINVAL, "x_cat or cat_offsets is null");
  const bool bf16 = a->out_dtype == TP_DTYPE_BF16;
  if (!bf16 && a->out_dtype != TP_DTYPE_F32) return fail(TP_EINVAL, "bad output dtype");
  if (a->out_ld % (bf16 ? 8 : 4) != 0 || a->out_col0 < 0 || a->out_col0 % (bf16 ? 8 : 4) != 0 ||
      a->out_ld < a->out_col0 + a->n_num)
    return fail(TP_EINVAL, "out_ld and out_col0 must be multiples of %d with the columns inside a row", bf16 ? 8 : 4);
  if (!aligned16(a->out)) return fail(TP_EALIGN, "out must be 16-byte aligned");
  InputArgs k{a->rows,     a->n_num,   a->n_cat, a->n_num > 0 ? a->x_num : nullptr, a->n_cat > 0 ? a->x_cat : nullptr,
              a->row_index, a->cat_offsets, a->out, a->out_ld, bf16 ? 1 : 0, a->out_col0};
  const long long blocks = (a->rows + 7) / 8;
  if (blocks > 0x7FFFFFFFLL) return fail(TP_EINVAL, "too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bf16)
    tabpack_input_kernel<true><<<(unsigned)blocks, 256, 0, st>>>(k);
  else
    tabpack_input_kernel<false><<<(unsigned)blocks, 256, 0, st>>>(k);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int tp_cos_emb_forward(const tp_cos_emb_args* a, void* stream) {
  TP_PROF(TP_PROF_EMBEDDING, static_cast<cudaStream_t>(stream));
  int rc = check_cos_emb(a);
  if (rc) return rc;
  if (!a->out || a->out_ld < a->F * a->D) return fail(TP_EINVAL, "embedding output needs out_ld >= F * D");
  if (a->out_dtype != TP_DTYPE_F32 && a->out_dtype != TP_DTYPE_BF16) return fail(TP_EINVAL, "bad output dtype");
  CosEmbArgs k = cos_emb_args(a);
  k.rows_per_block = 64;
  const dim3 grid((a->F * a->D + 2 * COS_EMB_THREADS - 1) / (2 * COS_EMB_THREADS), a->P, (a->B + 63) / 64);
  if (grid.z > 65535) return fail(TP_EINVAL, "batch too large for one embedding call");
  if (k.out_bf16)
    cos_emb_forward_kernel<true><<<grid, COS_EMB_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(k);
  else
    cos_emb_forward_kernel<false><<<grid, COS_EMB_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(k);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int tp_cos_emb_backward(const tp_cos_emb_args* a, void* stream) {
  TP_PROF(TP_PROF_EMBEDDING, static_cast<cudaStream_t>(stream));
  int rc = check_cos_emb(a);
  if (rc) return rc;
  if (!a->grad_out || a->grad_ld < a->F * a->D) return fail(TP_EINVAL, "embedding gradient needs grad_ld >= F * D");
  if (a->grad_dtype != TP_DTYPE_F32 && a->grad_dtype != TP_DTYPE_BF16) return fail(TP_EINVAL, "bad gradient dtype");
  if (!a->dweight || !a->dbias || !a->daffine_weight || !a->daffine_bias)
    return fail(TP_EINVAL, "null embedding gradient output");
  CosEmbArgs k = cos_emb_args(a);
  const int s = cos_emb_segments(a->P, a->B, a->F, a->D);
  k.rows_per_block = (a->B + s - 1) / s;
  const size_t need = tp_cos_emb_workspace_size(a->P, a->B, a->F, a->D);
  if (need > 0) {
    if (!a->workspace || a->workspace_bytes < need)
      return fail(TP_EINVAL, "embedding backward workspace of %zu bytes is smaller than the %zu needed",
                  a->workspace_bytes, need);
    k.partial = static_cast<double*>(a->workspace);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned cols = (a->F * a->D + COS_EMB_THREADS - 1) / COS_EMB_THREADS;
  if (k.g_bf16)
    cos_emb_backward_kernel<true><<<dim3(cols, a->P, s), COS_EMB_THREADS, 0, st>>>(k);
  else
    cos_emb_backward_kernel<false><<<dim3(cols, a->P, s), COS_EMB_THREADS, 0, st>>>(k);
  if (s > 1) cos_emb_finish_kernel<<<dim3(cols, a->P), COS_EMB_THREADS, 0, st>>>(k, s);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

size_t tp_roc_auc_workspace_size(int32_t P, int64_t N, int32_t dtype) {
  if (P <= 0 || N <= 0 || (dtype != TP_DTYPE_F32 && dtype != TP_DTYPE_F64)) return 0;
  return roc_auc_workspace_bytes(P, N, dtype == TP_DTYPE_F64 ? 8 : 4);
}

int tp_binary_roc_auc(const void* scores, const int64_t* labels, int32_t P, int64_t N, int32_t dtype, void* out,
                      void* workspace, size_t workspace_bytes, void* stream) {
  TP_PROF(TP_PROF_ROC_AUC, static_cast<cudaStream_t>(stream));
  if (!scores || !labels || !out || !workspace) return fail(TP_EINVAL, "null ROC AUC argument");
  if (P <= 0 || N <= 0) return fail(TP_EINVAL, "ROC AUC needs P > 0 and N > 0 (got %d, %lld)", P, (long long)N);
  if (N >= (int64_t)1 << 31) return fail(TP_EINVAL, "ROC AUC supports N < 2^31");
  if (dtype != TP_DTYPE_F32 && dtype != TP_DTYPE_F64) return fail(TP_EINVAL, "ROC AUC scores must be fp32 or fp64");
  const size_t need = tp_roc_auc_workspace_size(P, N, dtype);
  if (workspace_bytes < need)
    return fail(TP_EINVAL, "ROC AUC workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
  AucArgs a{P, (long long)N, scores, labels, out, workspace};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TP_DTYPE_F64)
    roc_auc_kernel<uint64_t><<<P, AUC_THREADS, 0, st>>>(a);
  else
    roc_auc_kernel<uint32_t><<<P, AUC_THREADS, 0, st>>>(a);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int tp_permutation_keys(uint64_t seed, uint32_t epoch, uint32_t member_base, int32_t P, int64_t N, int32_t* keys,
                        void* stream) {
  TP_PROF(TP_PROF_OTHER, static_cast<cudaStream_t>(stream));
  if (!keys || P <= 0 || N <= 0) return fail(TP_EINVAL, "bad permutation-key arguments");
  const int blocks = (int)std::min<int64_t>(((int64_t)P * N + 255) / 256, 8192);
  permutation_keys_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      (uint32_t)(seed & 0xFFFFFFFFu), (uint32_t)(seed >> 32), epoch, member_base, P, N, keys);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int tp_dropout_mask(uint64_t seed, uint32_t offset, uint32_t member_base, const float* dropout_p, int32_t P, int32_t B,
                    int32_t cols, uint8_t* mask, void* stream) {
  if (!dropout_p || !mask || P <= 0 || B <= 0 || cols <= 0) return fail(TP_EINVAL, "bad dropout mask arguments");
  const long long groups = (long long)P * B * ((cols + 7) / 8);
  const int blocks = (int)std::min<long long>((groups + 255) / 256, 4096);
  dropout_mask_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      (uint32_t)(seed & 0xFFFFFFFFu), (uint32_t)(seed >> 32), offset, member_base, dropout_p, P, B, cols, mask);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int tp_quotient_check(int32_t den_first, int32_t den_count, unsigned long long* counts, void* stream) {
  if (!counts || den_count <= 0 || den_first <= 0 || den_first + den_count > 0x7F80)
    return fail(TP_EINVAL, "divisor patterns must be positive finite bf16 values (0x0001 .. 0x7F7F)");
  if (den_count > 65535) return fail(TP_EINVAL, "at most 65535 divisors a call");
  quotient_check_kernel<<<dim3(16, den_count), 256, 0, static_cast<cudaStream_t>(stream)>>>(den_first, counts);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int tp_weight_cast(const tp_weight_cast_args* a, void* stream) {
  TP_PROF(TP_PROF_WEIGHT_CAST, static_cast<cudaStream_t>(stream));
  if (!a || a->P <= 0 || a->src_rows <= 0 || a->src_cols <= 0 || !a->src || !a->dst)
    return fail(TP_EINVAL, "bad weight cast arguments");
  if (a->dst_rows < a->src_rows || a->dst_cols < a->src_cols || a->dst_cols % 8 != 0)
    return fail(TP_EINVAL, "destination (%d, %d) must cover the source (%d, %d) with a multiple of 8 columns",
                a->dst_rows, a->dst_cols, a->src_rows, a->src_cols);
  if (!aligned16(a->dst)) return fail(TP_EALIGN, "dst must be 16-byte aligned");
  if (a->P > 65535) return fail(TP_EINVAL, "too many members for one call");
  const int src_ld = a->src_ld > 0 ? a->src_ld : a->src_cols;
  if (src_ld < a->src_cols) return fail(TP_EINVAL, "src_ld %d is below src_cols %d", src_ld, a->src_cols);
  WeightCastArgs k{a->src_rows, a->src_cols, src_ld, a->dst_rows, a->dst_cols, a->out_features, a->in_features,
                   a->n_blocks, a->block_index, a->src, static_cast<__nv_bfloat16*>(a->dst)};
  const dim3 grid((a->src_rows + 7) / 8, a->P);
  weight_cast_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(k);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int tp_weight_cast_transposed(const tp_weight_cast_t_args* a, void* stream) {
  TP_PROF(TP_PROF_WEIGHT_CAST, static_cast<cudaStream_t>(stream));
  if (!a || a->P <= 0 || a->src_rows <= 0 || a->ncols <= 0 || a->col0 < 0 || !a->src || !a->dst)
    return fail(TP_EINVAL, "bad transposed weight cast arguments");
  if (a->src_ld < a->col0 + a->ncols) return fail(TP_EINVAL, "column block beyond the source rows");
  if (a->dst_ld % 2 != 0 || a->dst_ld < (a->src_rows + 7) / 8 * 8)
    return fail(TP_EINVAL, "dst_ld must be even and cover the source rows rounded up to 8");
  if (!aligned16(a->dst)) return fail(TP_EALIGN, "dst must be 16-byte aligned");
  if (a->P > 65535) return fail(TP_EINVAL, "too many members for one call");
  WeightCastTArgs k{a->src_rows, a->src_ld, a->col0, a->ncols, a->dst_ld, a->out_features, a->src,
                    static_cast<__nv_bfloat16*>(a->dst)};
  const dim3 grid((a->ncols + CAST_T_J - 1) / CAST_T_J, (a->src_rows + CAST_T_N - 1) / CAST_T_N, a->P);
  if (grid.y > 65535) return fail(TP_EINVAL, "too many rows for one call");
  constexpr int smem = CAST_T_N * (CAST_T_J + 1) * 4;
  TP_CUDA_TRY(cudaFuncSetAttribute(weight_cast_t_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  weight_cast_t_kernel<<<grid, 256, smem, static_cast<cudaStream_t>(stream)>>>(k);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

}  // extern "C"

namespace tp {
namespace {

constexpr int ONEHOT_MAX_ROWS = 16384;  // batch rows one sort CTA holds (128 KB of keys)

int check_onehot(const tp_linear_args* a, const tp_onehot_args* oh) {
  if (!oh) return fail(TP_EINVAL, "null one-hot arguments");
  if (oh->n_cat <= 0 || oh->n_onehot <= 0 || !oh->cat_offsets || !oh->x_cat)
    return fail(TP_EINVAL, "one-hot features, offsets and categories are required");
  if (oh->n_dense < 0 || oh->n_dense > a->max_in) return fail(TP_EINVAL, "n_dense must lie in [0, max_in]");
  if (a->B > ONEHOT_MAX_ROWS) return fail(TP_EUNSUPPORTED, "at most %d batch rows per gathered first layer", ONEHOT_MAX_ROWS);

  if (a->P > 65535 || oh->n_cat > 65535) return fail(TP_EINVAL, "too many members or features for one call");
  if (a->n_blocks) return fail(TP_EINVAL, "the first layer has no depth gating");
  return TP_OK;
}

OneHotArgs onehot_args(const tp_linear_args* a, const tp_onehot_args* oh) {
  OneHotArgs k{};
  k.P = a->P;
  k.B = a->B;
  k.n_cat = oh->n_cat;
  k.n_onehot = oh->n_onehot;
  k.offsets = oh->cat_offsets;
  k.x_cat = oh->x_cat;
  k.x_cat_ms = oh->x_cat_member_stride;
  k.row_index = oh->row_index;
  k.row_index_ms = oh->row_index_member_stride;
  k.sorted_keys = static_cast<uint64_t*>(oh->sorted_keys);
  k.wt = static_cast<const __nv_bfloat16*>(oh->w_onehot_t);
  k.wt_ld = oh->wt_ld;
  k.out_f = a->out_features;
  k.max_out = a->max_out;
  k.addend = oh->addend;
  k.add_ld = oh->addend_ld;
  return k;
}

}  // namespace
}  // namespace tp

extern "C" {

int tp_onehot_linear_forward(const tp_linear_args* a, const tp_onehot_args* oh, void* stream) {
  int rc = check_linear(a);
  if (rc) return rc;
  if ((rc = check_onehot(a, oh))) return rc;
  if (!use_tensor_cores(a)) return fail(TP_EUNSUPPORTED, "the gathered first layer runs on the sm_100 bf16 path only");
  if (!oh->w_onehot_t || oh->wt_ld < (a->max_out + 7) / 8 * 8 || oh->wt_ld % 8 != 0 || !aligned16(oh->w_onehot_t))
    return fail(TP_EINVAL, "w_onehot_t must be 16-byte aligned with wt_ld a multiple of 8 covering max_out");
  if (!oh->addend || oh->addend_ld % 16 != 0 || oh->addend_ld < a->max_out || !aligned16(oh->addend))
    return fail(TP_EINVAL, "addend must be 16-byte aligned with addend_ld a multiple of 16 covering max_out");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const OneHotArgs k = onehot_args(a, oh);
  {
  TP_PROF(TP_PROF_ONEHOT, st);
  if (oh->sorted_keys) {  // the category sort the backward reads
    int pow2 = 1;
    while (pow2 < a->B) pow2 <<= 1;
    const int smem = pow2 * 8;
    TP_CUDA_TRY(cudaFuncSetAttribute(onehot_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    onehot_sort_kernel<<<dim3(oh->n_cat, a->P), std::min(1024, std::max(32, pow2 / 2)), smem, st>>>(k, pow2);
    TP_CUDA_TRY(cudaGetLastError());
  }
  onehot_gather_kernel<<<dim3((a->B + 7) / 8, a->P), 256, 0, st>>>(k);
  TP_CUDA_TRY(cudaGetLastError());
  }
  return linear_forward_impl(a, oh->addend, oh->addend_ld, stream);
}

int tp_onehot_linear_backward(const tp_linear_grad_args* ga, const tp_onehot_args* oh, void* stream) {
  if (!ga) return fail(TP_EINVAL, "null arguments");
  const tp_linear_args* a = &ga->fwd;
  int rc = check_linear(a);
  if (rc) return rc;
  if ((rc = check_onehot(a, oh))) return rc;
  if (!use_tensor_cores(a)) return fail(TP_EUNSUPPORTED, "the gathered first layer runs on the sm_100 bf16 path only");
  const int dw_rows = ga->dw_rows > 0 ? ga->dw_rows : a->max_out;
  if (ga->dw && !oh->sorted_keys) return fail(TP_EINVAL, "the weight gradient needs the forward's sorted_keys");
  if (ga->dw && (ga->dw_cols != oh->n_dense + oh->n_onehot || dw_rows > a->max_out))
    return fail(TP_EINVAL, "dw must be (P, <= max_out, n_dense + n_onehot)");
  // activation gradient, dx and the dense columns of dw
  tp_linear_grad_args d = *ga;
  d.dw_cols = oh->n_dense;
  if (d.dw && oh->n_dense == 0) d.dw = nullptr;
  if ((rc = linear_backward_impl(&d, ga->dw_cols, stream))) return rc;
  if (!ga->dw) return TP_OK;
  // the one-hot columns: segmented sums of g over each category's rows
  const bool need_g = a->relu || a->dropout_p || a->out_features || a->n_blocks;
  OneHotArgs k = onehot_args(a, oh);
  k.g = need_g ? ga->g : ga->dy;
  k.g_ld = a->max_out;
  k.g_bf16 = 1;
  k.dw = ga->dw;
  k.dw_rows = dw_rows;
  k.dw_ld = ga->dw_cols;
  k.dw_col0 = oh->n_dense;
  const int nb_count = (dw_rows + ONEHOT_WG_N - 1) / ONEHOT_WG_N;
  const long long blocks = ((long long)a->P * nb_count + ONEHOT_WG_WARPS - 1) / ONEHOT_WG_WARPS;
  if (blocks > 0x7FFFFFFFLL) return fail(TP_EINVAL, "too many one-hot gradient tasks");
  TP_PROF(TP_PROF_ONEHOT, static_cast<cudaStream_t>(stream));
  onehot_wgrad_kernel<<<(unsigned)blocks, 32 * ONEHOT_WG_WARPS, 0, static_cast<cudaStream_t>(stream)>>>(k, nb_count);
  TP_CUDA_TRY(cudaGetLastError());
  return TP_OK;
}

int tp_adamw_step(const tp_adamw_args* a, void* stream) {
  TP_PROF(TP_PROF_ADAMW, static_cast<cudaStream_t>(stream));
  if (!a || a->n_tensors <= 0 || a->n_tensors > TP_MAX_OPT_TENSORS) return fail(TP_EINVAL, "bad tensor count");
  AdamWTensors ts{};
  int64_t max_inner = 0, max_members = 0;
  for (int i = 0; i < a->n_tensors; ++i) {
    const tp_opt_tensor& t = a->t[i];
    if (!t.p || !t.grad || !t.exp_avg || !t.exp_avg_sq || t.numel <= 0 || t.inner <= 0)
      return fail(TP_EINVAL, "tensor %d: null pointer or empty", i);
    ts.t[i] = t;
    max_inner = std::max(max_inner, t.inner);
    max_members = std::max(max_members, (t.numel + t.inner - 1) / t.inner);
  }
  AdamWScalars s{};
  s.lr = a->lr.per_member;
  s.beta1 = a->beta1.per_member;
  s.beta2 = a->beta2.per_member;
  s.eps = a->eps.per_member;
  s.wd = a->weight_decay.per_member;
  s.lr_s = (float)a->lr.scalar;
  s.beta1_s = (float)a->beta1.scalar;
  s.beta2_s = (float)a->beta2.scalar;
  s.eps_s = (float)a->eps.scalar;
  s.wd_s = (float)a->weight_decay.scalar;
  const bool lr_zero = !a->lr.per_member && a->lr.scalar == 0.0;
  const bool wd_zero = !a->weight_decay.per_member && a->weight_decay.scalar == 0.0;
  s.wd_on = !(lr_zero || wd_zero);
  s.wd_mult_s = (float)(1.0 - a->lr.scalar * a->weight_decay.scalar);
  s.one_m_b1_s = (float)(1.0 - a->beta1.scalar);
  s.one_m_b2_s = (float)(1.0 - a->beta2.scalar);
  s.bc1_scalar = !a->beta1.per_member;
  s.bc2_scalar = !a->beta2.per_member;
  s.step = a->step;
  if (s.bc1_scalar) {
    const double bc1 = 1.0 - std::pow(a->beta1.scalar, (double)a->step);
    s.bc1_s = (float)bc1;
    s.step_size_s = (float)(a->lr.scalar / bc1);
  }
  if (s.bc2_scalar) s.sqrt_bc2_s = (float)std::sqrt(1.0 - std::pow(a->beta2.scalar, (double)a->step));
  // blocks per member: up to 4 elements per thread per block pass, at most 64 blocks
  const int bx = (int)std::min<int64_t>((max_inner + 1023) / 1024, 64);
  for (int64_t m0 = 0; m0 < max_members; m0 += 65535) {
    dim3 grid(bx, (unsigned)std::min<int64_t>(65535, max_members - m0), a->n_tensors);
    adamw_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(ts, s, (int)m0);
    TP_CUDA_TRY(cudaGetLastError());
  }
  return TP_OK;
}

}  // extern "C"
