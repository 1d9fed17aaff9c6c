/*
 * wamffn.h -- C ABI of the B200 (sm_100a) FFN hot path of WAMInfer's video DiT.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), returns an int status (WAMFFN_OK == 0) and never throws.
 * On failure wamffn_last_error() returns a thread-local message.  No entry
 * point allocates device memory or synchronises the stream except the
 * *_create / *_destroy / wamffn_*_status / wamffn_trace_enable calls, so every
 * run call can be captured into a CUDA graph (the reference forbids tuning
 * during capture, _cublaslt_inference.cpp:167-168; *_create refuses the same way).
 *
 * Tensors are bf16 (uint16 storage), row-major, last dimension contiguous.
 * Weights use torch.nn.Linear's native [out_features, in_features] layout.
 *
 * Reference interfaces replaced (paths inside the WAMInfer project):
 *   wamffn_linear_plan_create   <- Plan::Plan(x, weight, bias, exhaustive, gelu)
 *                                  WAMInfer/_cublaslt_inference.cpp:161-174
 *   wamffn_linear_run           <- Plan::run(x, weight, bias)
 *                                  WAMInfer/_cublaslt_inference.cpp:177-188
 *                                  (op wam_infer::prepared_ffn_linear_v1,
 *                                   WAMInfer/ffn.py:38-45)
 *   wamffn_linear_configuration <- Plan::selected_configuration()
 *                                  WAMInfer/_cublaslt_inference.cpp:189
 *   wamffn_ffn_run              <- PreparedFFN.forward(layer_id, inputs)
 *                                  WAMInfer/ffn.py:96-107
 *   wamffn_modulated_norm       <- op wam_infer::modulated_norm
 *                                  WAMInfer/_triton_inference.py:130-221
 *   wamffn_block_run            <- VideoAdapter post-attention norm + FFN phase:
 *                                  WAMInfer/blocks.py:241-244 (CROSS_RESIDUAL norm),
 *                                  WAMInfer/blocks.py:246-272 (gather, FFN,
 *                                  cache scatter/concat, deferred gate) and the
 *                                  FFN_RESIDUAL fold of
 *                                  WAMInfer/_triton_inference.py:158-161
 *   wamffn_select_tokens        <- select_tokens(state, features)
 *                                  WAMInfer/approximation.py:55-67
 *   wamffn_rgb_mandatory        <- the RGB change test of TokenReuse.begin
 *                                  WAMInfer/approximation.py:31-36
 *   wamffn_masked_attention     <- op wam_infer::masked_attention_mask_tiles_v4
 *                                  WAMInfer/_triton_attention.py:238-263
 *   wamffn_joint_first_frame_attention <- op wam_infer::joint_first_frame_attention_v2
 *                                  WAMInfer/_triton_attention.py:327-334
 *   wamffn_current_frame_attention <- op wam_infer::current_frame_attention_v1
 *                                  WAMInfer/_triton_attention.py:429-484
 */
#ifndef WAMFFN_H
#define WAMFFN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WAMFFN_ABI_VERSION 2

/* Status codes returned by every entry point. */
#define WAMFFN_OK 0
#define WAMFFN_ERR_INVALID 1     /* bad argument: shape, stride, alignment, null pointer */
#define WAMFFN_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define WAMFFN_ERR_UNSUPPORTED 3 /* device is not sm_100 or geometry exceeds kernel limits */
#define WAMFFN_ERR_CAPTURE 4     /* plan creation/tuning attempted during stream capture */
#define WAMFFN_ERR_DEVICE 5      /* a kernel reported an error through the device status word */

/* Flags of wamffn_linear_plan_create. */
#define WAMFFN_LINEAR_GELU 1     /* tanh-GELU epilogue (the up projection) */
#define WAMFFN_WEIGHTS_PACKED 2  /* weights are in the tile-packed layout of wamffn_pack_weight */

/* Bits of the device status word (wamffn_*_status). */
#define WAMFFN_DEV_TIMEOUT 1u    /* a pipeline wait exceeded its time limit; the kernel bailed out */
#define WAMFFN_DEV_BAD_INDEX 2u  /* a gather/scatter index was outside [-1, seq) or >= cache rows */

/* Modes of wamffn_modulated_norm: the reference's MODE constants
 * (WAMInfer/_triton_inference.py:117-120). */
#define WAMFFN_SELF_INPUT 0
#define WAMFFN_SELF_RESIDUAL 1
#define WAMFFN_CROSS_RESIDUAL 2
#define WAMFFN_FFN_RESIDUAL 3

typedef struct wamffn_linear_plan wamffn_linear_plan;
typedef struct wamffn_block_plan wamffn_block_plan;

/* ABI version and the last error message of the calling thread. */
int wamffn_abi_version(void);
const char* wamffn_last_error(void);

/* Number of kernels this library has launched in the process (all devices). */
unsigned long long wamffn_launch_count(void);

/* Phase trace of the GEMM and layer-boundary kernels (profiling aid; no
 * reference counterpart: the reference relies on external Nsight traces).
 * With a device buffer of `records` x 8 uint64 (word 0 of record 0 is the
 * record counter, zeroed by the caller), every GEMM CTA appends {tag, start,
 * operands ready, MMAs issued, accumulator ready, epilogue done, SM id,
 * K blocks} and every layer-boundary CTA {tag, start, wait done, reduction
 * done, reduction done, end, SM id, 0} in globaltimer ns; tag = CTA x |
 * CTA y << 16 | kind << 32 (kind: the GEMM epilogue 0 GELU, 1 bias, 2 split-K
 * partials; 7 layer boundary).  The persistent pass kernel writes record
 * 1 + cta * 3 (layers + 1) + 3 layer + phase instead.  waminfer_b200/trace.py
 * decodes the buffer.  buffer == NULL switches tracing off.  Synchronous; not
 * for use in capture. */
int wamffn_trace_enable(int device, void* buffer, int records);

/* ------------------------------------------------------------------------
 * Linear plan: y[rows, n_out] = act(x[rows, k_in] . weight[n_out, k_in]^T + bias)
 * act = tanh-GELU with WAMFFN_LINEAR_GELU (no bf16 rounding between bias and
 * GELU, as in the reference's GELU_BIAS epilogue), identity otherwise.
 * With WAMFFN_WEIGHTS_PACKED the weight passed to run is the tile-packed copy
 * made by wamffn_pack_weight (the reference likewise runs on a repacked copy
 * made at prepare time, ffn.py:82-88); otherwise it is row-major [n_out, k_in].
 * fp32 accumulation, bf16 output.  Replaces Plan(...) (cpp:161-174).
 * `tune` != 0 times the candidate layouts (split-K factor x token groups)
 * on the device, each over weight copies larger than L2 so that the weights
 * stream from HBM as a model's per-layer weights do (like the reference's
 * exhaustive candidate timing, cpp:121-158), and keeps the fastest;
 * otherwise a static heuristic picks the configuration.
 * ---------------------------------------------------------------------- */
int wamffn_linear_plan_create(int device, int rows, int n_out, int k_in, int flags, int tune,
                              wamffn_linear_plan** plan);
int wamffn_linear_plan_destroy(wamffn_linear_plan* plan);

/* Replaces Plan::run (cpp:177-188). out must hold rows*n_out bf16. */
int wamffn_linear_run(wamffn_linear_plan* plan, void* stream, const void* x, const void* weight,
                      const void* bias, void* out);

/* Replaces Plan::selected_configuration (cpp:189).  Writes up to n values:
 * {feature_tile, token_pad, mma_count, stages, split_k, tmem_columns, tuned,
 *  streamk_groups, token_groups}.  streamk_groups > 0: a GELU plan whose
 * feature tiles leave SMs idle runs as stream-K, its tiles' K blocks cut into
 * that many equal ranges, one per CTA pair on every SM, with a fixed-order
 * fix-up of the split tiles (deterministic).  token_groups > 1: the rows are
 * cut into that many equal groups, each with its own CTAs (token_pad is then
 * per group). */
int wamffn_linear_configuration(const wamffn_linear_plan* plan, uint32_t* values, int n);

/* Sets a plan's layout explicitly: K split into `splits` (1..16; 1 for a GELU
 * plan) slices whose fp32 partials a second kernel sums in split order, and
 * the rows cut into `groups` (1..4) token groups.  No counterpart in the
 * reference (cuBLASLt's algorithm choice is internal to Plan::tune,
 * cpp:121-174); the tuner of wamffn_linear_plan_create picks among the same
 * layouts.  Reallocates the split-K workspace when `splits` changes;
 * synchronises the device; refused during CUDA Graph capture. */
int wamffn_linear_plan_set_layout(wamffn_linear_plan* plan, int splits, int groups);

/* Reads (and with clear != 0 resets) the device status word of a plan.
 * Synchronises the device. */
int wamffn_linear_status(wamffn_linear_plan* plan, uint32_t* status, int clear);

/* ------------------------------------------------------------------------
 * Allocation-free split-K linear.  No counterpart in the reference: it exists
 * for callers that must not allocate device memory at all -- code that runs
 * inside an allocator or memory-pool callback (a cudaMalloc there would
 * re-enter the allocator), plugin hosts that own every byte of device memory
 * and forbid allocations by plugins, and serving processes that reserved all
 * of HBM for their caches at start-up.  Such a caller cannot create a plan
 * (plan creation allocates its workspace and status word).
 *
 * out[rows, n_out] = x[rows, k_in] . weight^T + bias, bf16 in and out, fp32
 * accumulation, K split into `splits` (2..16) slices whose fp32 partials live
 * in one static device array of WAMFFN_STATIC_SCRATCH_BYTES per device (the
 * first 256 bytes hold a status word, the partials follow).  A call needs
 * 256 + splits * rows * n_out * 4 bytes of it; a call that needs more is
 * rejected with WAMFFN_ERR_INVALID before anything is launched.  flags accepts
 * WAMFFN_WEIGHTS_PACKED only (there is no GELU variant: the split-K reduction
 * applies the bias only).  Same shape limits as wamffn_linear_plan_create.
 *
 * The call allocates nothing: no cudaMalloc / cudaFree, no library routine
 * that allocates.  The first call on a device looks up the array's address
 * (cudaGetSymbolAddress with that device current, which may load the module
 * on it) and sets the kernels' shared-memory limit: make that first call
 * before any stream capture.  Later calls only encode tensor maps on the host
 * and launch.
 *
 * Every call on a device shares the one array, so calls that overlap in time
 * (two streams, or two host threads) race on it: serialise them.  Nothing in
 * the array needs to start at zero except the status word, which each call
 * clears on `stream` when `status` is null.  `status` may instead point at a
 * caller-owned device word (4-byte aligned, cleared by the caller) that the
 * kernels OR WAMFFN_DEV_* bits into; with null the bits land in the shared
 * word and are not reported, so a null `status` gives up error detection: a
 * call whose GEMM gave up on a timed-out pipeline wait writes no partials,
 * and its reduction then returns the previous call's result without any error.
 *
 * The array's address is looked up once per device and kept: calls after
 * cudaDeviceReset (or any teardown of the device's primary context) are not
 * supported.
 * ---------------------------------------------------------------------- */
#define WAMFFN_STATIC_SCRATCH_BYTES (16u << 20) /* 16 MiB per device */
int wamffn_linear_run_static(int device, void* stream, int rows, int n_out, int k_in, int splits,
                             int flags, const void* x, const void* weight, const void* bias, void* out,
                             uint32_t* status);

/* PreparedFFN.forward (ffn.py:96-107): out = down(gelu(up(x))).  `up` and
 * `down` are plans of matching rows; hidden is scratch owned by the up plan. */
int wamffn_ffn_run(wamffn_linear_plan* up, wamffn_linear_plan* down, void* stream, const void* x,
                   const void* w_up, const void* b_up, const void* w_down, const void* b_down,
                   void* out);

/* Weight repack for HBM streaming (replaces the repack of PreparedFFN.prepare,
 * ffn.py:82-88): dst[n_out/128][k_in/64][128][64] <- src[n_out][k_in], so that
 * every 128 x 64 tile a GEMM CTA loads is one contiguous 16 KB block.
 * n_out % 128 == 0, k_in % 64 == 0; src and dst hold n_out*k_in bf16. */
int wamffn_pack_weight(void* stream, const void* src, void* dst, int n_out, int k_in);

/* ------------------------------------------------------------------------
 * Modulated norm (op wam_infer::modulated_norm, _triton_inference.py:130-221)
 * x, update: [rows, dim] with row strides x_stride / update_stride (elements)
 * mod, previous: [6, dim]; time: per-row [rows, 6, dim] with time_stride
 * elements between rows, or time_stride == 0 for one shared [6, dim] row.
 * weight, bias: [dim] (SELF_RESIDUAL only).  Outputs y, norm: [rows, dim]
 * contiguous.  Batch 1, as the reference (grid = rows, _triton_inference.py:201).
 * ---------------------------------------------------------------------- */
typedef struct wamffn_norm_args {
  const void* x;
  int64_t x_stride;
  const void* update;
  int64_t update_stride;
  const void* mod;
  const void* previous;
  const void* time;
  int64_t time_stride;
  const void* weight;
  const void* bias;
  void* y;
  void* norm;
  int rows;
  int dim;
  int mode;
  float eps;
} wamffn_norm_args;

int wamffn_modulated_norm(void* stream, const wamffn_norm_args* args);

/* ------------------------------------------------------------------------
 * Fused FFN block (one DiT layer's FFN phase):
 *   y      = bf16(x + update)                            (CROSS_RESIDUAL, update may be NULL)
 *   n      = adaLN_{slots 3,4}(LayerNorm(y))             (_triton_inference.py:162-174)
 *   a[j]   = n[indices[j]]                               (gather, blocks.py:249-251)
 *   h      = bf16(gelu_tanh(a . W_up^T + b_up))          (up GEMM, tcgen05)
 *   o[j]   = bf16(h . W_down^T + b_down)                 (down GEMM, tcgen05, split-K)
 *   output[r] = o[j] where indices[j] == r; rows r < cache_rows that are not
 *               gathered take cache_in[r]                (index_copy + cat, blocks.py:259-264)
 *   cache_out[r] = output[r] for r < cache_rows          (token_outputs, blocks.py:264)
 *   x_out  = bf16(y + bf16(gate . output)),
 *            gate = bf16(mod[5] + time[r, 5])            (FFN_RESIDUAL fold / last layer,
 *                                                         _triton_inference.py:158-161,
 *                                                         blocks.py:265-268)
 * With `normalized` set, the first two lines are skipped (y = x, n = normalized),
 * matching VideoAdapter.ffn_at_layer_for_compile(layer_id, state, normalized, x)
 * (blocks.py:246).
 * indices: `rows` entries (int32 if index_bytes == 4, int64 if 8), -1 marks
 * a pad row that is computed on zeros and never scattered; NULL means the
 * identity (rows == seq).  Outputs that are NULL are not written.
 * cache_in may equal cache_out (in-place history update).
 * ---------------------------------------------------------------------- */
typedef struct wamffn_block_args {
  const void* x;          /* [seq, d] residual stream before the update */
  const void* update;     /* [seq, d] cross-attention output or NULL */
  const void* normalized; /* [seq, d] FFN input already normalised by the caller, or NULL.
                             When set, the norm step is skipped: x is the residual y
                             as-is (update must be NULL) and rows are gathered from here. */
  const void* mod;        /* [6, d] block.modulation */
  const void* time;       /* [seq, 6, d] per-token time modulation, or [6, d] */
  int64_t time_stride;    /* elements between time rows; 0 = shared row */
  const void* w_up;       /* [h, d] */
  const void* b_up;       /* [h] */
  const void* w_down;     /* [d, h] */
  const void* b_down;     /* [d] */
  int weights_packed;     /* 1: w_up / w_down are wamffn_pack_weight copies */
  const void* indices;    /* [rows] gather list or NULL */
  int index_bytes;        /* 4 or 8 */
  int rows;               /* gathered rows M */
  int seq;                /* sequence rows S */
  int cache_rows;         /* n: rows [0, n) are cacheable; 0 = no cache */
  const void* cache_in;   /* [n, d] previous FFN outputs or NULL */
  void* cache_out;        /* [n, d] or NULL */
  void* y;                /* [seq, d] residual after the update, or NULL */
  void* output;           /* [seq, d] FFN output in sequence order, or NULL */
  void* x_out;            /* [seq, d] gated residual, or NULL */
  float eps;              /* LayerNorm eps (norm2.eps) */
} wamffn_block_args;

/* Block plan: owns the gathered-activation, hidden and split-K scratch for up
 * to max_rows gathered rows and max_seq sequence rows. */
int wamffn_block_plan_create(int device, int max_rows, int max_seq, int d_model, int d_hidden,
                             int tune, wamffn_block_plan** plan);
int wamffn_block_plan_destroy(wamffn_block_plan* plan);
int wamffn_block_run(wamffn_block_plan* plan, void* stream, const wamffn_block_args* args);
int wamffn_block_status(wamffn_block_plan* plan, uint32_t* status, int clear);
/* Split-K factor of the down projection for `rows` gathered rows (rows = 0:
 * every row count up to max_rows); splits = 0 restores the heuristic, which
 * fills the SMs with feature tiles x splits CTAs.  No counterpart in the
 * reference (cuBLASLt picks its own split inside Plan::tune,
 * _cublaslt_inference.cpp:121-174).  A caller that runs several plans
 * concurrently on one device (independent requests on separate streams)
 * lowers it: the other lanes fill the SMs, and fewer splits move fewer fp32
 * partials through L2.  Applies to launches enqueued after the call. */
int wamffn_block_plan_set_splits(wamffn_block_plan* plan, int rows, int splits);
/* {up: feature_tile, token_pad, mma_count, stages, split_k, tmem_columns, tuned,
 *  down: same 7 values, up streamk_groups, down streamk_groups} for a given
 * row count (n = 14 omits the last two). */
int wamffn_block_configuration(const wamffn_block_plan* plan, int rows, uint32_t* values, int n);
/* Stream-K up projection on or off (default off; WAMFFN_STREAMK=1 changes
 * the default of new plans) for launches enqueued after the call.  No
 * counterpart in the reference (cuBLASLt picks its own schedule inside
 * Plan::tune).  With it the up projection's 56 feature-tile pairs
 * (h = 14336) are spread over every SM pair instead of leaving 36 SMs idle;
 * on B200 that measured slower (48 vs 36 us at 392 rows: the operand streams
 * of 148 SMs arrive more slowly per K block, and the split tiles' fp32
 * partials cross L2 twice).  Results differ from the data-parallel grid in
 * the last bits (a different fp32 summation order), so a caller that compares
 * lanes bit for bit sets the same schedule on every plan. */
int wamffn_block_plan_set_streamk(wamffn_block_plan* plan, int enabled);

/* ------------------------------------------------------------------------
 * FFN stack: the FFN phases of `layers` consecutive DiT layers in one call,
 * the way the reference's 30-layer loop runs them (joint.py:93-156 with
 * blocks.py:246-272): layers below first_gathered_layer recompute every row
 * (the reference's layer 0, blocks.py:248); later layers gather `indices`
 * (the same list for every layer, select_tokens, approximation.py:55-67) and
 * read / write the history slice [layer - first_gathered_layer] of
 * cache_in / cache_out ([layers - first_gathered_layer, cache_rows, d], the
 * packed cache of runtime.py:263).  Between layers the split-K reduction,
 * history scatter, gated residual and the next layer's norm + gather run as
 * one kernel.  No attention runs between the FFNs: every layer's norm input
 * is the previous layer's residual (update = NULL).
 * With the environment variable WAMFFN_PASS=1 a pass is one persistent
 * launch instead, whose CTAs (one per SM) synchronise through grid-wide
 * counters: it needs the whole device, so such passes must not run
 * concurrently with other work (several block plans on several streams);
 * a pass whose CTAs cannot all become resident ends with WAMFFN_DEV_TIMEOUT
 * in the status word.
 * ---------------------------------------------------------------------- */
typedef struct wamffn_layer_weights {
  const void* w_up;     /* [h, d] or packed */
  const void* b_up;     /* [h] */
  const void* w_down;   /* [d, h] or packed */
  const void* b_down;   /* [d] */
  const void* mod;      /* [6, d] block.modulation */
} wamffn_layer_weights;

typedef struct wamffn_stack_args {
  int layers;
  const wamffn_layer_weights* weights;  /* host array of `layers` entries */
  int weights_packed;
  const void* x;          /* [seq, d] residual entering the first layer */
  const void* time;       /* [seq, 6, d] per-token time modulation, or [6, d] */
  int64_t time_stride;
  int seq;
  const void* indices;    /* gather list of the gathered layers, or NULL (all rows) */
  int index_bytes;
  int rows;               /* entries of indices */
  int first_gathered_layer;
  int cache_rows;
  const void* cache_in;   /* [layers - first_gathered_layer, cache_rows, d] or NULL */
  void* cache_out;        /* same shape, or NULL */
  void* x_out;            /* [seq, d] residual after the last layer */
  float eps;
} wamffn_stack_args;

int wamffn_stack_run(wamffn_block_plan* plan, void* stream, const wamffn_stack_args* args);

/* ------------------------------------------------------------------------
 * Self-test of the failure path.  No counterpart in the reference.  Launches
 * one CTA on `stream` whose pipeline wait can never complete (a barrier no
 * one arrives on), with a wait limit of `limit_cycles` SM cycles
 * (1e3..1e9); the wait gives up, raises the CTA's abort flag and ORs
 * WAMFFN_DEV_TIMEOUT into *status (a 4-byte aligned device word the caller
 * cleared), a second role waiting on the same barrier leaves through the
 * abort flag, and the kernel returns.  Every pipeline wait of the library's
 * kernels ends this way after 4e9 cycles (2-4 s) instead of hanging; this lets
 * a test observe the mechanism in milliseconds without faulting the GPU.
 * ---------------------------------------------------------------------- */
int wamffn_selftest_wait_timeout(void* stream, uint32_t* status, int64_t limit_cycles);

/* ------------------------------------------------------------------------
 * Tensor-parallel FFN stack (the hidden dimension split across ranks).  The
 * reference runs each FFN on one GPU (blocks.py:252-258 over ffn.py:96-107);
 * this mode splits h column-wise for W_up / b_up and row-wise (over K) for
 * W_down, so `plan` is created with d_hidden = h / world and args->weights
 * hold this rank's slices (w_up [h/world, d], b_up [h/world], w_down
 * [d, h/world], full b_down and mod).  Per layer the rank's split-K partials
 * of the down projection are summed (split order) into reduce_buffer
 * ([rows, d] fp32, caller-owned, rows = that layer's GEMM rows), then
 * allreduce(user, reduce_buffer, rows * d, stream) is called on the host
 * while the layer is enqueued: it must enqueue a sum over all ranks into the
 * same buffer, ordered after the work already on `stream` and before the work
 * enqueued on it afterwards (an NCCL all-reduce on that stream, or a
 * torch.distributed one).  The bias, gated residual, history scatter and the
 * next layer's norm then run once on the reduced sum, identically on every
 * rank.  A non-zero return from allreduce aborts the call with that status.
 * ---------------------------------------------------------------------- */
typedef int (*wamffn_allreduce_fn)(void* user, float* buffer, int64_t count, void* stream);
int wamffn_stack_run_tp(wamffn_block_plan* plan, void* stream, const wamffn_stack_args* args, float* reduce_buffer,
                        wamffn_allreduce_fn allreduce, void* user);

/* ------------------------------------------------------------------------
 * Token selection (select_tokens, approximation.py:55-67):
 *   score[r] = 2 sum|now - before| / max(sum(|now| + |before|), 1e-6)  (fp32)
 *   mandatory rows score +inf; the `count` best rows (stable descending, ties
 *   to the smaller index) are written ascending to indices[0, count), then
 *   indices[count + k] = n + k for k < seq - n.  features_out (optional)
 *   receives a copy of the n current rows (the next request's history).
 * now: [n, dim] rows `now_stride` elements apart; before: [n, dim];
 * mandatory: n bytes (0/1) or NULL; indices: int64.  n <= 1024, count < n.
 * ---------------------------------------------------------------------- */
typedef struct wamffn_select_args {
  const void* now;
  int64_t now_stride;
  const void* before;
  const void* mandatory;
  int n;
  int dim;
  int count;
  int seq;
  void* indices;
  void* features_out;
} wamffn_select_args;

int wamffn_select_tokens(void* stream, const wamffn_select_args* args);

/* ------------------------------------------------------------------------
 * Mandatory rows of TokenReuse.begin (approximation.py:31-36) for uint8 HWC
 * observations now / before [height, width, 3]: mandatory[i] = 1 when the
 * mean |now - before| over patch i (row-major grid_h x grid_w patches of
 * height/grid_h x width/grid_w pixels, 3 channels) exceeds 5.0, else 0.
 * Integer sums, one float32 division: the reference's float32 mask exactly.
 * height and width must divide by the grid (the reference's reshape).
 * ---------------------------------------------------------------------- */
int wamffn_rgb_mandatory(void* stream, const void* now, const void* before, int height, int width, int grid_h,
                         int grid_w, void* mandatory);

/* ------------------------------------------------------------------------
 * Masked multi-head attention (op wam_infer::masked_attention_mask_tiles_v4,
 * WAMInfer/_triton_attention.py:18-145, 238-263):
 *   out[b, q, h*128:(h+1)*128] = softmax over k of (q . k / sqrt(128), keys where
 *   mask[b, h, q, k] is false at -inf) . v
 * with the reference's arithmetic (exp2 of scores scaled by 128^-0.5 log2 e,
 * probabilities rounded to bf16 before the value product, fp32 normaliser,
 * all-masked rows output 0).  q: [batch, nq, heads*128] rows q_row_stride
 * elements apart (batch stride == nq * row stride); k, v: [batch, nk, ...]
 * likewise; mask: bool bytes addressed b*mask_strides[0] + h*[1] + q*[2] +
 * k*[3] (0 = broadcast), or NULL; out: [batch, nq, heads*128] contiguous.
 * `status` (optional, 4-byte aligned device word) receives WAMFFN_DEV_* bits.
 * Head dim 128 only.  No scratch: K and V rows are read as they lie.
 * key_split: 0 picks the split of the keys across a cluster of CTAs per query
 * tile (1, 2 or 4: the largest that keeps the grid within one wave of SMs);
 * 1, 2 or 4 forces it (halved while it exceeds the 128-key blocks).  The split
 * moves the probabilities' bf16 rounding point, not the function.
 * ---------------------------------------------------------------------- */
typedef struct wamffn_attention_args {
  const void* q;
  int64_t q_row_stride;
  int64_t q_batch_stride;
  const void* k;
  int64_t k_row_stride;
  int64_t k_batch_stride;
  const void* v;
  int64_t v_row_stride;
  int64_t v_batch_stride;
  const void* mask;
  int64_t mask_strides[4];
  void* out;
  uint32_t* status;
  int batch;
  int nq;
  int nk;
  int heads;
  int head_dim;
  int key_split;
} wamffn_attention_args;

int wamffn_masked_attention(void* stream, const wamffn_attention_args* args);

/* One [batch, rows, heads*128] bf16 operand: rows row_stride elements apart,
 * batch_stride == rows * row_stride (a multiple of 8 elements, 16-byte aligned). */
typedef struct wamffn_rows_view {
  const void* data;
  int64_t row_stride;
  int64_t batch_stride;
} wamffn_rows_view;

/* ------------------------------------------------------------------------
 * Joint first-frame-causal attention (op wam_infer::joint_first_frame_attention_v2,
 * WAMInfer/_triton_attention.py:267-334): q, k, v [batch, count, heads*128]
 * (video rows then action rows); query rows [0, first) attend keys [0, first)
 * (the clean first frame sees neither the future video nor the action rows),
 * rows [first, count) attend all count keys.  out [batch, count, heads*128]
 * contiguous.  `video` (the video row count) is carried for the reference's
 * signature and changes nothing.  Arithmetic and key_split as
 * wamffn_masked_attention.
 * ---------------------------------------------------------------------- */
typedef struct wamffn_joint_attention_args {
  wamffn_rows_view q, k, v;
  void* out;
  uint32_t* status;
  int batch;
  int count;
  int video;
  int first;
  int heads;
  int head_dim;
  int key_split;
} wamffn_joint_attention_args;

int wamffn_joint_first_frame_attention(void* stream, const wamffn_joint_attention_args* args);

/* ------------------------------------------------------------------------
 * Current-frame attention over a cached prefix (op wam_infer::current_frame_attention_v1,
 * WAMInfer/_triton_attention.py:337-484): queries qv [batch, nv, .] then
 * qa [batch, na, .] attend the keys ck [nc] ++ kv [nv] ++ ka [na] with values
 * cv ++ vv ++ va, unmasked, without concatenating anything; outputs
 * ov [batch, nv, heads*128] and oa [batch, na, heads*128], contiguous.
 * Arithmetic and key_split as wamffn_masked_attention.
 * ---------------------------------------------------------------------- */
typedef struct wamffn_current_frame_args {
  wamffn_rows_view qv, qa, ck, kv, ka, cv, vv, va;
  void* ov;
  void* oa;
  uint32_t* status;
  int batch;
  int nc;
  int nv;
  int na;
  int heads;
  int head_dim;
  int key_split;
} wamffn_current_frame_args;

int wamffn_current_frame_attention(void* stream, const wamffn_current_frame_args* args);

#ifdef __cplusplus
}
#endif

#endif /* WAMFFN_H */
