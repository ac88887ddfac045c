/*
 * tabpack_b200 — C ABI of the B200 (sm_100a) packed-ensemble hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as `void*`, i.e. a `cudaStream_t`), enqueues its kernels on that
 * stream and returns immediately.  All buffers are allocated and owned by the
 * caller.  Return value: TP_OK (0) or a negative TP_E* code; the message for the
 * last failure on the calling thread is available from tp_last_error_string().
 * Errors are reported, never thrown; no kernel traps.  Kernels that wait on an
 * mbarrier give up after a bounded time and record TP_ETIMEOUT in a device-side
 * flag that tp_device_error() reads (and clears).
 *
 * Layout conventions follow the reference's pack convention (PACK_DIM = 0,
 * BATCH_DIM = 1, src/tabpackage/nn.py:29-30): activations are padded
 * (P, B, width), weights (P, max_out, max_in), biases (P, max_out); columns at
 * or beyond a member's own width are exactly zero in every output.
 */
#ifndef TABPACK_B200_H_
#define TABPACK_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TP_OK 0
#define TP_EINVAL (-1)       /* bad shape, null pointer, unsupported combination */
#define TP_EALIGN (-2)       /* pointer or leading dimension not 16-byte aligned */
#define TP_EUNSUPPORTED (-3) /* not supported on this device / build */
#define TP_ECUDA (-4)        /* a CUDA runtime or driver call failed */
#define TP_ETIMEOUT (-5)     /* a device-side wait gave up (reported by tp_device_error) */

#define TP_DTYPE_F32 0  /* fp32 activations and weights, fp32 CUDA-core arithmetic */
#define TP_DTYPE_BF16 1 /* bf16 activations and weights, tcgen05 tensor cores, fp32 accumulation */
#define TP_DTYPE_F64 2  /* fp64 scores (tp_binary_roc_auc only) */

/* Arguments of one packed-linear call (one LinearPack, or one MLP block =
 * LinearPack -> ReLU -> DropoutPack).  Widths `max_in`/`max_out` are the
 * leading dimensions of x / y / w; in BF16 mode both must be multiples of 8. */
typedef struct tp_linear_args {
  int32_t P;              /* members in this call */
  int32_t B;              /* rows (batch) per member */
  int32_t max_in;         /* padded input width  = last dim of x and w */
  int32_t max_out;        /* padded output width = last dim of y, middle dim of w */
  int32_t dtype;          /* TP_DTYPE_* of x, w, y, g, dx */
  int32_t x_shared;       /* 1: x is (B, max_in), shared by every member */
  const int32_t* in_features;  /* device (P,) real input widths, or NULL (= max_in) */
  const int32_t* out_features; /* device (P,) real output widths, or NULL (= max_out) */
  const int32_t* n_blocks;     /* device (P,) depths, or NULL: member m is active
                                  iff n_blocks == NULL || n_blocks[m] > block_index; an
                                  inactive member's y is its x over its out_features columns
                                  (dx = dy over in_features in the backward) and zero beyond,
                                  where its x (dy) holds zeros as a pack's activations do */
  int32_t block_index;
  int32_t relu;                /* 1: ReLU after the bias */
  const float* dropout_p;      /* device (P,) dropout probabilities, or NULL (eval) */
  uint64_t seed;               /* Philox key */
  uint32_t offset;             /* Philox counter word 3 (call id) */
  uint32_t member_base;        /* global id of member 0 (counter word 2 = base + m) */
  const void* x;               /* (P or 1, B, max_in) */
  const void* w;               /* (P, max_out, max_in) */
  const float* bias;           /* (P, max_out) fp32, or NULL */
  void* y;                     /* (P, B, max_out) */
  int32_t y_pad_zero;          /* 1: y's padding already holds zeros (the columns at or beyond
                                  each member's out_features, in every row), e.g. a buffer that
                                  an earlier call with the same widths wrote: the forward writes
                                  each member's columns rounded up to a multiple of 32 and skips
                                  the rest.  0: it writes every column. */
  const int32_t* row_index;    /* device (P, B) dataset rows, or NULL.  With it, x is a
                                  (x_rows, max_in) table shared by every member and member m's
                                  row b is x[row_index[m * B + b]]: the training loop's per-step
                                  batch gather (src/tabpackage/_training.py:2667-2669) done by
                                  the GEMMs' operand loads (TMA gather4) instead of a gathered
                                  copy.  BF16 tensor-core path only; no depth gating and no
                                  input gradient (the table takes none). */
  int32_t x_rows;              /* rows of the table x when row_index is set */
} tp_linear_args;

/* Backward of tp_linear_forward with the same `fwd` arguments. */
typedef struct tp_linear_grad_args {
  tp_linear_args fwd;
  const void* dy;     /* (P, B, max_out) gradient w.r.t. y */
  const void* y;      /* forward output (read when relu or dropout is on) */
  void* g;            /* (P, B, max_out) workspace: gradient w.r.t. the pre-activation */
  float* dbias;       /* (P, max_out) fp32, or NULL */
  void* dx;           /* (P, B, max_in), or NULL (no input gradient) */
  float* dw;          /* (P, dw_rows, dw_cols) fp32, or NULL */
  int32_t dw_rows;    /* leading dims of dw (the parameter's real padded shape) */
  int32_t dw_cols;
  int32_t db_cols;    /* row length of dbias (the parameter's real max_out) */
  int32_t g_ready;    /* 1: g (and dbias) already hold this call's activation gradient;
                         only the requested dx / dw GEMMs run */
  int32_t dx_cols;    /* > 0: dx only for input columns < dx_cols (zeros beyond), e.g. the
                         embedding columns of a first layer whose one-hot columns take no
                         gradient; 0: every column */
  int32_t dw_pad_zero; /* 1: dw already holds zeros outside each active member's
                          out_features x in_features block and for every depth-inactive member
                          (a buffer that an earlier call with the same widths and depths wrote):
                          the weight gradient writes the active members' blocks only (output
                          features rounded up to a multiple of 32).  0: it writes every element. */
  int32_t dx_pad_zero; /* 1: dx already holds zeros beyond each member's input columns rounded
                          up to the GEMM's 256-column tiles (a buffer that an earlier call with
                          the same widths and depths wrote): the input gradient writes only the
                          column tiles that hold a member's columns.  0: every element. */
} tp_linear_grad_args;

/* LinearPack.forward (src/tabpackage/nn.py:792-816) fused with the ReLU and
 * DropoutPack.forward (nn.py:886-903) of MLPBackbonePack.Block.forward
 * (nn.py:1071-1079) and the depth gating of MLPBackbonePack._forward_dense
 * (nn.py:1272-1288): y = dropout(relu(x w^T + b)) for active members, y = x for
 * inactive ones (requires max_in == max_out). */
int tp_linear_forward(const tp_linear_args* a, void* stream);

/* Autograd of the same composition (replaces the BaddbmmBackward / MulBackward /
 * ReluBackward chain the reference records at nn.py:805-816, 897-901): writes g,
 * dbias, dx (columns >= in_features are zero) and dw (entries outside
 * out_features x in_features are zero). */
int tp_linear_backward(const tp_linear_grad_args* a, void* stream);

/* Size of the built-in workspace of tp_linear_backward_noalloc: 16 MiB. */
#define TP_NOALLOC_SCRATCH_BYTES (16u << 20)

/* No counterpart in the reference: an addition of this library.
 *
 * tp_linear_backward for callers that must not allocate device memory, for
 * example a host framework that owns all GPU memory through its own pool, or
 * code that runs where an allocation is not allowed.  The caller passes the
 * same arguments as for tp_linear_backward with `g` left NULL (inputs and
 * outputs stay caller-owned); the activation-gradient workspace comes from a
 * fixed device array inside this library, so the call allocates nothing.
 *
 * Limits and behaviour:
 *  - the workspace needs P * B * max_out elements (2 bytes in BF16 mode,
 *    4 bytes in F32 mode); larger calls are rejected with TP_EINVAL before any
 *    kernel runs;
 *  - the TP_NOALLOC_SCRATCH_BYTES array is reserved on a device the first time
 *    the library's module is used there (its first kernel launch or its first
 *    no-alloc call; at library load when CUDA_MODULE_LOADING=EAGER) and stays
 *    reserved until the process exits;
 *  - the first call in each CUDA context (the primary context of each device,
 *    or a context the caller created) looks up the array's device address in
 *    that context (set-up) and should come before any CUDA stream capture;
 *  - all calls share the one array and it keeps the last call's contents; calls
 *    whose kernels overlap on the GPU (different streams, no ordering) race;
 *  - `g_ready` is ignored: the activation gradient is always recomputed. */
int tp_linear_backward_noalloc(const tp_linear_grad_args* a, void* stream);

/* No counterpart in the reference: per-launch timing of this library's kernels.
 *
 * tp_profile_start(capacity) creates 2 * capacity CUDA events on the current device and
 * brackets each following kernel launch (for the GEMMs and the Muon kernels) or call (for
 * the other entry points) with two of them, until `capacity` launches are recorded (later
 * ones are counted in `dropped`).  tp_profile_stop waits for the recorded events, writes the
 * summed milliseconds and launch counts per family into ms / launches (n_kinds entries,
 * indexed by TP_PROF_*), destroys the events and turns the recording off.  Off by default,
 * where it costs one atomic load per launch; start / stop must not overlap other calls into
 * the library. */
#define TP_PROF_FWD 0              /* tensor-core forward GEMMs (all forward variants) */
#define TP_PROF_DGRAD 1            /* tensor-core dX GEMMs */
#define TP_PROF_WGRAD 2            /* tensor-core dW GEMMs */
#define TP_PROF_NS 3               /* Newton-Schulz A = X X^T and B = b A + c A^2 */
#define TP_PROF_NS_BMN 4           /* Newton-Schulz X <- a X + B X */
#define TP_PROF_GEMM_F32 5         /* fp32 CUDA-core GEMMs */
#define TP_PROF_ACT_BACKWARD 6     /* activation / bias gradient */
#define TP_PROF_MUON_ELEMENTWISE 7 /* Muon momentum, packing, norm, normalisation, update */
#define TP_PROF_ADAMW 8
#define TP_PROF_WEIGHT_CAST 9
#define TP_PROF_INPUT 10           /* first-layer input build (tp_tabpack_input) */
#define TP_PROF_EMBEDDING 11       /* cosine embeddings */
#define TP_PROF_ONEHOT 12          /* one-hot sort, gather and weight gradient */
#define TP_PROF_METRIC 13
#define TP_PROF_GREEDY 14
#define TP_PROF_ROC_AUC 15
#define TP_PROF_OTHER 16
#define TP_PROF_KINDS 17
int tp_profile_start(int32_t capacity);
int tp_profile_stop(double* ms, int64_t* launches, int32_t n_kinds, int32_t* dropped);

/* Test hook: the Philox keep mask of the dropout above, (P, B, cols) uint8. */
int tp_dropout_mask(uint64_t seed, uint32_t offset, uint32_t member_base,
                    const float* dropout_p, int32_t P, int32_t B, int32_t cols,
                    uint8_t* mask, void* stream);

/* Test hook: the Muon normalisation's quotient (x * (1/den) with one fused correction,
 * Markstein's method) against CUDA's correctly rounded division, exhaustively over bf16
 * operands: divisors with bit patterns den_first .. den_first + den_count - 1 (positive finite),
 * every finite bf16 dividend with |x| <= 2 den.  Adds to counts (device, 4 x uint64): fp32
 * quotients differing in any bit, quotients differing after rounding to bf16 (what the
 * normalisation stores), pairs checked, and the fp32 differences where the exact quotient or
 * the reciprocal is subnormal. */
int tp_quotient_check(int32_t den_first, int32_t den_count, unsigned long long* counts, void* stream);

/* One tensor of a grouped optimizer step.  Element e of the tensor belongs to
 * member e / inner. */
typedef struct tp_opt_tensor {
  float* p;
  float* grad;
  float* exp_avg;     /* AdamW m, or the Muon momentum buffer */
  float* exp_avg_sq;  /* AdamW v (unused by Muon) */
  const int64_t* step;/* per-member step counts (already incremented), or NULL */
  int64_t numel;
  int64_t inner;
} tp_opt_tensor;

/* Per-member hyperparameters: a device (P,) fp32 array, or NULL to use the
 * scalar.  Mirrors the group values of OptimizerPack (src/tabpackage/optim.py:92-117). */
typedef struct tp_hparam {
  const float* per_member;
  double scalar;
} tp_hparam;

#define TP_MAX_OPT_TENSORS 32

typedef struct tp_adamw_args {
  int32_t n_tensors;
  tp_opt_tensor t[TP_MAX_OPT_TENSORS];
  tp_hparam lr, beta1, beta2, eps, weight_decay;
  int64_t step;       /* scalar step (already incremented) when t[i].step == NULL */
} tp_adamw_args;

/* AdamWPack.step / MuonAdamWPack._step_adamw for up to TP_MAX_OPT_TENSORS
 * parameter packs of one group (src/tabpackage/optim.py:347-427, 776-846). */
int tp_adamw_step(const tp_adamw_args* a, void* stream);

/* One Muon parameter group: a packed weight (P, max_out, max_in) fp32 with its
 * gradient and momentum buffer.  Follows MuonAdamWPack._step_muon
 * (src/tabpackage/optim.py:682-774) with _zeropower_via_newtonschulz5
 * (optim.py:464-490): decoupled weight decay, momentum lerp, Nesterov, ns_steps
 * quintic Newton-Schulz iterations in bf16 (fp32 accumulation) on tensor cores,
 * p -= lr * scale * update.  Each member iterates on its own out x in block,
 * oriented so its Gram matrix is min(out, in) square; members whose update is all
 * zero skip the iterations (decided on the device, no host synchronisation).  The
 * padding of p / grad / momentum outside out_features x in_features is not touched. */
typedef struct tp_muon_args {
  int32_t P, max_out, max_in;
  float* p;
  float* grad;
  float* momentum_buffer;
  const int32_t* out_features;  /* (P,) or NULL (= max_out) */
  const int32_t* in_features;   /* (P,) or NULL (= max_in) */
  tp_hparam lr, momentum, weight_decay;
  const float* update_scale;    /* (P,) or NULL: sqrt(max(1, max_out / max_in)) */
  int32_t nesterov;
  int32_t mutate_grad;          /* 1: grad receives the Nesterov update (as the reference
                                   does with allow_inplace_grad_mutation=True) */
  int32_t ns_steps;
  void* workspace;              /* >= tp_muon_workspace_size(P, max_out, max_in) bytes */
  size_t workspace_bytes;
  /* Optional bf16 compute copy of p (the copy autocast's forward multiplies with): when
   * non-NULL, element (o, n) of member m with o < out_m, n < in_m receives bf16(p_new) at
   * p_bf16[(m * p_bf16_rows + o) * p_bf16_cols + n] in the same pass that writes p; other
   * elements of the copy are left as they are.  NULL: no copy is written. */
  void* p_bf16;
  int32_t p_bf16_rows, p_bf16_cols;
  /* Optional depth gating of the block this weight belongs to: members with
   * n_blocks[m] <= block_index pass their input through the block, so their gradient is
   * exactly zero; the step reads it as zero (their momentum still decays and, where it is
   * nonzero, they take the full update) and leaves their rows of the bf16 copy alone.
   * NULL: every member is stepped from its gradient. */
  const int32_t* n_blocks;
  int32_t block_index;
  /* 1: the momentum of every depth-gated member is zero (a caller that zeroes a member's state
   * whenever its depth changes): such a member's update is zero, so its gradient, momentum and
   * Newton-Schulz operand are neither read nor written, and only its weight decay is applied.
   * 0: a gated member's momentum is read (it decays and, where nonzero, updates the weights). */
  int32_t gated_momentum_zero;
} tp_muon_args;

size_t tp_muon_workspace_size(int32_t P, int32_t max_out, int32_t max_in);
int tp_muon_step(const tp_muon_args* a, void* stream);

/* Several Muon parameter groups in one call (MuonAdamWPack.step's loop over its Muon groups,
 * src/tabpackage/optim.py:682-774 per group): each group's momentum, normalisation and
 * update as tp_muon_step computes them, bit for bit, with the Newton-Schulz GEMMs of all
 * groups in shared launches (their tiles in one dynamically claimed list; fewer, fuller
 * launches than one set per group).  The groups' own workspace fields are ignored; the
 * call's workspace (256-byte aligned) holds every group's operands at common strides.  All
 * groups take the same ns_steps; at most 65535 members over all groups. */
size_t tp_muon_grouped_workspace_size(const tp_muon_args* groups, int32_t n_groups);
int tp_muon_step_grouped(const tp_muon_args* groups, int32_t n_groups, void* workspace, size_t workspace_bytes,
                         void* stream);

#define TP_METRIC_MSE 0
#define TP_METRIC_MAE 1
#define TP_METRIC_ACCURACY 2        /* int64 predicted labels (P, N) vs int64 labels */
#define TP_METRIC_BCE 3             /* probabilities (P, N) vs int64 {0, 1} labels */
#define TP_METRIC_CE 4              /* probabilities (P, N, C) vs int64 class labels */
#define TP_METRIC_ACCURACY_ARGMAX 5 /* scores (P, N, C): accuracy of the argmax class */
#define TP_METRIC_R2 6

/* Per-member metrics with labels shared by every member: mse_pack, mae_pack,
 * accuracy_pack, binary_cross_entropy_pack, multiclass_cross_entropy_pack and
 * r2_pack of src/tabpackage/metrics.py:76-253.  Terms in fp32, sums in fp64. */
typedef struct tp_metric_args {
  int32_t metric;
  int32_t P;              /* number of predictions */
  int64_t N;              /* rows */
  int32_t C;              /* classes (CE, argmax accuracy), else 1 */
  const void* y_pred;     /* fp32 (P, N[, C]), or int64 (P, N) for TP_METRIC_ACCURACY */
  const void* y_true;     /* fp32 (N,) for MSE / MAE / R2, int64 (N,) otherwise */
  float* out;             /* (P,) */
} tp_metric_args;
int tp_metric_pack(const tp_metric_args* a, void* stream);

/* Greedy ensemble selection, greedy_ensemble (src/tabpackage/ensemble.py:95-263),
 * for the metrics above: candidates (C_pred, N, C) fp32, scores = metric
 * (maximize = 1) or -metric, top-k initialisation, forward selection with or
 * without replacement, stop at no improvement or the size limit.  The whole loop
 * runs on the device; `counts[c]` receives how often prediction c was selected, and
 * `status` (device memory) {iterations, distinct members, error} once the stream
 * reaches the end of the call.  error = 1 means a NaN score (the reference raises). */
typedef struct tp_greedy_args {
  int32_t metric;
  int32_t maximize;
  int32_t n_pred;                /* candidate predictions */
  int64_t N;                     /* rows */
  int32_t C;                     /* classes per row */
  const float* predictions;      /* (n_pred, N, C) */
  const void* y_true;
  int32_t init_top_k;
  int32_t max_ensemble_size;     /* <= 0: no limit (only without replacement) */
  int32_t with_replacement;
  int32_t* counts;               /* (n_pred,) device */
  void* workspace;
  size_t workspace_bytes;
  int32_t* status;               /* (3,) device: iterations, distinct members, error */
} tp_greedy_args;
size_t tp_greedy_workspace_size(int32_t n_pred, int64_t N, int32_t C);
int tp_greedy_ensemble(const tp_greedy_args* a, void* stream);

/* (Weighted) mean of selected member predictions: compute_unsanitized_ensemble_predictions
 * (src/tabpackage/ensemble.py:25-61) and TabPackPredictor.EnsembleHead.forward
 * (src/tabpackage/_training.py:1955-1958).  pred (P, n), idx (K,) device, weights (K,)
 * device or NULL, out (n,). */
int tp_ensemble_mean(const float* pred, const int32_t* idx, const float* weights, int32_t K, int64_t n,
                     float* out, void* stream);

/* Row-wise softmax over the last dimension: the classification prediction transform
 * (torch.softmax(x, -1)) applied to packed outputs before metrics and ensembling
 * (_training.py:170-181).  x, out: (rows, C) fp32. */
int tp_softmax_rows(const float* x, int64_t rows, int32_t C, float* out, void* stream);

/* Per-member batch-order keys for make_shuffled_batch_indices_pack
 * (src/tabpackage/_training.py:323-338), whose `rand(P, N).argsort` draws from a global
 * RNG: here keys[m][i] is 31 bits of a Philox word of (seed, epoch, member_base + m, i), so sorting a
 * member's keys (stable) yields the same permutation on any number of GPUs.  keys: (P, N)
 * int32 in [0, 2^31). */
int tp_permutation_keys(uint64_t seed, uint32_t epoch, uint32_t member_base, int32_t P, int64_t N, int32_t* keys,
                        void* stream);

/* Per-member binary ROC AUC: binary_roc_auc_pack (src/tabpackage/metrics.py:117-150), the
 * Mann-Whitney U statistic with midranks for ties (_midranks_pack, metrics.py:85-114).
 * scores (P, N) fp32 (dtype TP_DTYPE_F32) or fp64 (TP_DTYPE_F64); labels (N,) int64, shared by
 * every member, nonzero = positive; out (P,) in the scores' type, NaN when one class is absent.
 * Ties and NaNs follow the reference: equal scores (-0.0 == +0.0) share their average rank,
 * NaNs rank last and are never tied.  The rank sum is exact (integer), where the reference
 * accumulates it in the scores' type.  One CTA per member sorts its scores (stable radix sort
 * in the workspace); N < 2^31. */
size_t tp_roc_auc_workspace_size(int32_t P, int64_t N, int32_t dtype);
int tp_binary_roc_auc(const void* scores, const int64_t* labels, int32_t P, int64_t N, int32_t dtype, void* out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Cosine numerical-feature embeddings: CosineEmbeddingsPack (src/tabpackage/nn.py:1627-1833,
 * forward nn.py:1783-1833) with concat_input.  Member m, feature f, slot k < D (D =
 * max_d_embedding): slot 0 is the raw value, slot k >= 1 is cos(2pi b[k-1] + 2pi w[k-1] x), then the
 * elementwise affine ab_k + aw_k * slot_k with aw, ab zero at k >= d_embedding[m].  The output
 * is written at column f * D + k of each row of `out` (leading dimension out_ld >= F * D), i.e.
 * the flattened embedding the first linear layer consumes.  Backward gives the parameter
 * gradients from the upstream gradient of that output (sums over the batch in fp64, fixed order;
 * the input x takes no gradient).  x: (P, B, F) fp32, or (B, F) when x_shared. */
typedef struct tp_cos_emb_args {
  int32_t P, B, F, D;
  int32_t x_shared;
  const float* x;
  const float* weight;           /* (P, F, D - 1) */
  const float* bias;             /* (P, F, D - 1) */
  const float* affine_weight;    /* (P, F, D) */
  const float* affine_bias;      /* (P, F, D) */
  const int32_t* d_embedding;    /* (P,) or NULL: every slot active */
  void* out;                     /* forward: (P, B, out_ld) */
  int32_t out_ld;
  int32_t out_dtype;             /* TP_DTYPE_F32 or TP_DTYPE_BF16 */
  const void* grad_out;          /* backward: (P, B, grad_ld) */
  int32_t grad_ld;
  int32_t grad_dtype;            /* TP_DTYPE_F32 or TP_DTYPE_BF16 */
  float* dweight;                /* (P, F, D - 1) */
  float* dbias;                  /* (P, F, D - 1) */
  float* daffine_weight;         /* (P, F, D) */
  float* daffine_bias;           /* (P, F, D) */
  void* workspace;               /* backward: >= tp_cos_emb_workspace_size(P, B, F, D) bytes */
  size_t workspace_bytes;
} tp_cos_emb_args;
size_t tp_cos_emb_workspace_size(int32_t P, int32_t B, int32_t F, int32_t D);

/* First-layer input of a TabPack without numerical embeddings, in one pass: row r gets its
 * n_num numerical values, then the one-hot encoding of each categorical feature
 * (_OneHotEncoding, src/tabpackage/nn.py:1836-1871; the value `cardinality` is the unknown
 * category and encodes as zeros; torch.cat of both parts, nn.py:2071-2107), converted to
 * out_dtype, then zeros up to out_ld.  cat_offsets: (n_cat + 1,) device int32 prefix sums of
 * the cardinalities.  out_ld must be a multiple of 8 (bf16) or 4 (fp32) and at least
 * n_num + cat_offsets[n_cat].  With row_index, output row r is built from dataset row
 * row_index[r]: the per-step batch gather of the training loop (`v[batch_idx]`,
 * src/tabpackage/_training.py:2667-2669) without materialising the gathered batch. */
typedef struct tp_input_args {
  int64_t rows;
  int32_t n_num;
  int32_t n_cat;
  const float* x_num;            /* (rows, n_num), or (dataset rows, n_num) with row_index; or NULL */
  const int64_t* x_cat;          /* (rows, n_cat), or (dataset rows, n_cat) with row_index; or NULL */
  const int64_t* row_index;      /* (rows,) dataset row of each output row, or NULL */
  const int32_t* cat_offsets;    /* (n_cat + 1,) */
  void* out;                     /* (rows, out_ld) */
  int32_t out_ld;
  int32_t out_dtype;             /* TP_DTYPE_F32 or TP_DTYPE_BF16 */
  int32_t out_col0;              /* columns [out_col0, out_ld) of each row are written (the
                                    numerical values start there); columns before it are left
                                    as they are, e.g. an embedding written by
                                    tp_cos_emb_forward.  out_col0 * element size must be a
                                    multiple of 16 */
} tp_input_args;
int tp_tabpack_input(const tp_input_args* a, void* stream);
int tp_cos_emb_forward(const tp_cos_emb_args* a, void* stream);
int tp_cos_emb_backward(const tp_cos_emb_args* a, void* stream);

/* bf16 compute copy of an fp32 weight pack for the tensor-core GEMMs: the weight cast of
 * torch.autocast at LinearPack.forward (src/tabpackage/nn.py:806-808, autocast region
 * src/tabpackage/_training.py:161-167), done once per weight update and only over what the
 * GEMMs read.  For every member m with n_blocks[m] > block_index (all members when n_blocks is
 * NULL) and every row r < min(out_features[m], src_rows): dst[m, r, c] = bf16(src[m, r, c])
 * (round to nearest even) for c < min(in_features[m], src_cols) and 0 for the other c <
 * dst_cols.  Other rows of dst are left as they are: a caller that starts from a zeroed dst
 * (or one written by an earlier call) hands the GEMMs finite values everywhere.  NULL widths
 * mean the full source extent. */
typedef struct tp_weight_cast_args {
  int32_t P;
  int32_t src_rows, src_cols;   /* fp32 source (P, src_rows, src_cols) */
  int32_t src_ld;               /* row stride of src in elements (0: src_cols), e.g. a column block */
  int32_t dst_rows, dst_cols;   /* bf16 destination (P, dst_rows, dst_cols); dst_cols % 8 == 0,
                                   dst_rows >= src_rows, dst_cols >= src_cols */
  const int32_t* out_features;  /* device (P,) or NULL */
  const int32_t* in_features;   /* device (P,) or NULL */
  const int32_t* n_blocks;      /* device (P,) or NULL */
  int32_t block_index;
  const float* src;
  void* dst;                    /* 16-byte aligned */
} tp_weight_cast_args;
int tp_weight_cast(const tp_weight_cast_args* a, void* stream);

/* Transposed bf16 copy of the column block [col0, col0 + ncols) of an fp32 weight pack:
 * dst[m, j, n] = bf16(src[m, n, col0 + j]) for n < min(out_features[m], src_rows) and 0 for
 * the n up to the next multiple of 8; the rest of each dst row is left as it is.  This is the
 * operand of tp_onehot_linear_forward (the one-hot block of a TabPack's first-layer weight,
 * whose rows the forward gathers).  dst_ld must be even and at least src_rows rounded up to 8. */
typedef struct tp_weight_cast_t_args {
  int32_t P;
  int32_t src_rows, src_ld;     /* fp32 source (P, src_rows, src_ld) */
  int32_t col0, ncols;          /* the column block */
  int32_t dst_ld;               /* bf16 destination (P, ncols, dst_ld) */
  const int32_t* out_features;  /* device (P,) or NULL */
  const float* src;
  void* dst;                    /* 16-byte aligned */
} tp_weight_cast_t_args;
int tp_weight_cast_transposed(const tp_weight_cast_t_args* a, void* stream);

/* First layer of a TabPack over one-hot categorical features as a gather-sum (bf16, tensor
 * cores).  The reference one-hot encodes each categorical feature (_OneHotEncoding,
 * src/tabpackage/nn.py:1836-1871), concatenates the blocks after the dense columns
 * (nn.py:2071-2107) and multiplies the whole width in its first LinearPack (nn.py:792-816).
 * Here the layer's weight W (P, max_out, n_dense + n_onehot) is split: the dense columns
 * (bf16 copy, tp_weight_cast with src_ld) multiply the dense input on the tensor cores with
 * K = n_dense, and the one-hot columns are gathered: one W column per feature and row, added
 * to the accumulator before the bias, ReLU and dropout.  Category values outside
 * [0, cardinality) (the unknown category `cardinality` included) contribute nothing, as
 * their one-hot rows are zero.
 *
 * tp_onehot_linear_forward: `a` is the forward of the dense part (x: (P or 1, B, max_in) dense
 * input, w: the bf16 dense weight copy (P, max_out, max_in), bias/relu/dropout as in
 * tp_linear_forward, dtype TP_DTYPE_BF16).  Writes y, and sorted_keys when it is non-NULL
 * (kept for the backward; a forward without a backward passes NULL and skips the sort), and
 * uses addend as scratch.
 * tp_onehot_linear_backward: as tp_linear_backward for the same `a` and `oh` (after the
 * forward wrote sorted_keys); dw is the full weight gradient (P, dw_rows, dw_cols)
 * with dw_cols = n_dense + n_onehot: the dense columns come from the tensor-core wgrad and
 * the one-hot columns from segmented sums of the pre-activation gradient over the rows of
 * each category, in ascending row order.  dx, when requested, is the dense input's gradient
 * (P, B, max_in). */
/* At most 16384 batch rows per call (TP_EUNSUPPORTED beyond). */
typedef struct tp_onehot_args {
  int32_t n_dense;               /* weight columns before the one-hot block (<= max_in of `a`) */
  int32_t n_cat;                 /* categorical features */
  int32_t n_onehot;              /* one-hot columns (= cat_offsets[n_cat]) */
  const int32_t* cat_offsets;    /* device (n_cat + 1,): first one-hot column of each feature */
  const int64_t* x_cat;          /* categories; batch row r of member m reads x_cat row
                                    (row_index ? row_index[m * row_index_member_stride + r] : r)
                                    + m * x_cat_member_stride */
  int64_t x_cat_member_stride;
  const int64_t* row_index;      /* device or NULL */
  int64_t row_index_member_stride;
  const void* w_onehot_t;        /* bf16 (P, n_onehot, wt_ld) from tp_weight_cast_transposed */
  int32_t wt_ld;                 /* >= max_out rounded up to 8 */
  void* sorted_keys;             /* (P, n_cat, B) uint64: (category << 32 | batch row), ascending per
                                    feature; the unknown category sorts last */
  float* addend;                 /* forward scratch (P, B, addend_ld), 16-byte aligned */
  int32_t addend_ld;             /* multiple of 16, >= max_out */
} tp_onehot_args;
int tp_onehot_linear_forward(const tp_linear_args* a, const tp_onehot_args* oh, void* stream);
int tp_onehot_linear_backward(const tp_linear_grad_args* ga, const tp_onehot_args* oh, void* stream);

/* Clears and returns the device-side error flag (TP_OK or TP_ETIMEOUT). */
int tp_device_error(void);

/* Message of the last failing call on this thread ("" if none). */
const char* tp_last_error_string(void);

/* Library version string. */
const char* tp_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TABPACK_B200_H_ */
