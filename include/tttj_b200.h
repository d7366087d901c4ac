/*
 * tttj_b200.h -- C ABI of the B200 (sm_100a) forward path for the pre-LayerNorm
 * transformer stack of Scallion3008/tttj-2026:
 *
 *     for each block: x = x + out_proj(attn(LN1 x)); x = x + ffn_out(gelu(ffn_in(LN2 x)));
 *                     x = x.masked_fill(~valid_token_mask, 0)
 *     out = LN_final(x).masked_fill(~valid_token_mask, 0)
 *
 * (benchmarks/torch_transformer_benchmark.py:59-172 in the reference).
 *
 * The reference exposes this path to Python through a pybind11 module whose entry
 * point is forward(input, valid_mask, packed_weights, capture_debug)
 * (kernels/csrc/sequence_resident.cpp:23-32, host side
 * kernels/csrc/sequence_resident.cu:468-533), JIT-built and loaded by
 * kernels/sequence_resident.py:51-65.  This header is the C replacement for that
 * binding: plain pointers, sizes and a CUDA stream handle, no torch types.  All
 * device pointers are CUDA device addresses on the plan's device; `stream` is a
 * cudaStream_t (NULL = legacy default stream).
 *
 * Every function returns TTTJ_OK (0) or an error code; tttj_last_error() returns a
 * message for the calling thread's last failure.  Shape errors are reported the way
 * the reference's TORCH_CHECKs report them (kernels/csrc/sequence_resident.cu:473-496):
 * nothing is launched.
 */
#ifndef TTTJ_B200_H
#define TTTJ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTTJ_OK 0
#define TTTJ_ERR_INVALID 1        /* unsupported shape / bad argument (Python: ValueError) */
#define TTTJ_ERR_CUDA 2           /* CUDA runtime or driver error (Python: RuntimeError) */
#define TTTJ_ERR_DEVICE_TIMEOUT 3 /* a device-side wait hit its limit (Python: RuntimeError) */

#define TTTJ_DTYPE_F16 0
#define TTTJ_DTYPE_F32 1

/* Mirrors TransformerConfig (benchmarks/torch_transformer_benchmark.py:29-56). */
typedef struct tttj_config {
  int32_t batch_size;
  int32_t seq_len;
  int32_t d_model;
  int32_t num_heads;
  int32_t ffn_dim;
  int32_t num_layers;
  int32_t causal;
} tttj_config;

/* Fields of the packed weight buffer.  Matrices are fp16 in nn.Linear's [out, in]
 * layout; vectors are fp32.  Replaces pack_model_weights
 * (kernels/sequence_resident.py:74-109), which packs the same parameters into one
 * flat fp16 buffer in the order LN1, q, k, v, out, LN2, ffn_in, ffn_out, final LN. */
#define TTTJ_W_QKV 0     /* fp16 [3D, D]: rows q_proj | k_proj | v_proj */
#define TTTJ_W_OUT 1     /* fp16 [D, D]  out_proj.weight */
#define TTTJ_W_FFN_IN 2  /* fp16 [F, D]  ffn_in.weight */
#define TTTJ_W_FFN_OUT 3 /* fp16 [D, F]  ffn_out.weight */
#define TTTJ_B_QKV 4     /* fp32 [3D]    q|k|v biases */
#define TTTJ_B_OUT 5     /* fp32 [D] */
#define TTTJ_B_FFN_IN 6  /* fp32 [F] */
#define TTTJ_B_FFN_OUT 7 /* fp32 [D] */
#define TTTJ_LN1_W 8     /* fp32 [D]  norm1.weight */
#define TTTJ_LN1_B 9     /* fp32 [D]  norm1.bias */
#define TTTJ_LN2_W 10    /* fp32 [D]  norm2.weight */
#define TTTJ_LN2_B 11    /* fp32 [D]  norm2.bias */
#define TTTJ_LNF_W 12    /* fp32 [D]  final_norm.weight (layer index = num_layers) */
#define TTTJ_LNF_B 13    /* fp32 [D]  final_norm.bias   (layer index = num_layers) */

/* Last error message of the calling thread ("" if none). */
const char* tttj_last_error(void);

/* Library version string. */
const char* tttj_version(void);

/* Check a configuration against what the kernels support (head_dim a multiple of 8 up
 * to 256 -- heads narrower than 32 run padded to 32 columns inside the workspace --,
 * d_model and ffn_dim multiples of 32, ...).  Mirrors case_number_for_model's
 * ValueError contract (optimized_transformer.py:45-66): TTTJ_ERR_INVALID + message. */
int tttj_validate_config(const tttj_config* cfg);

/* Size of the packed weight buffer, and the byte offset/size of one field.
 * layer in [0, num_layers) for per-block fields, layer == num_layers for LNF. */
size_t tttj_weights_bytes(const tttj_config* cfg);
int tttj_weight_offset(const tttj_config* cfg, int layer, int field, size_t* offset,
                       size_t* bytes);

/* LayerNorm-folded weights.  Each block's LN1 affine is folded into a copy of its QKV
 * weights and LN2's into ffn_in (W' = W diag(gamma) in fp16, b' = b + W beta, column
 * sums of W'), so the GEMMs consume the raw residual and apply the row statistics in
 * their epilogue; padded-head layouts (head_dim < 32 or between kernel sizes) also get
 * a zero-column copy of out_proj here.  The folded weights depend on the layer shapes
 * only (not on batch_size / seq_len): one buffer serves every plan of a model.
 * tttj_fold_weights enqueues the one-time fold kernels on `stream`; the packed weights
 * must be complete in stream order, and plans may be created at once (they launch
 * nothing).  Buffers are device memory, 256-byte aligned.  Replaces the reference's
 * one-time packing step SequenceResidentTransformer.prepare
 * (kernels/sequence_resident.py:143-150). */
size_t tttj_folded_bytes(const tttj_config* cfg);
int tttj_fold_weights(const tttj_config* cfg, const void* weights, void* folded,
                      size_t folded_bytes, void* stream);

/* Device workspace of a plan (activations of the packed valid tokens, LayerNorm
 * statistics with their per-row pivots, token plan, device status word).  It must be
 * zero-filled once before the first forward (the plan never reads a byte the same
 * call did not write, except rows of earlier calls, which no result depends on). */
size_t tttj_workspace_bytes(const tttj_config* cfg);

/* A plan binds a configuration (batch_size, seq_len included) to one device, one packed
 * weight buffer, one folded weight buffer and one workspace (all owned by the caller),
 * and pre-builds every TMA descriptor.  Creating it launches nothing and does not
 * synchronise.  It owns a pinned host word mirroring its device status (see
 * tttj_forward) and an event ordering its forwards across streams; destroying it
 * waits for its last forward, so the caller may then free or reuse the workspace.
 * Replaces SequenceResidentTransformer's per-shape state
 * (kernels/sequence_resident.py:125-233). */
typedef struct tttj_plan tttj_plan;
int tttj_plan_create(const tttj_config* cfg, int device, const void* weights, const void* folded,
                     void* workspace, size_t workspace_bytes, tttj_plan** out_plan);
int tttj_plan_destroy(tttj_plan* plan);

/* One forward pass, enqueued on `stream` (no host synchronisation).
 *   x          [B, S, D] in x_dtype (TTTJ_DTYPE_F16 or TTTJ_DTYPE_F32)
 *   valid_mask [B, S] bytes (0 = padded token), or NULL = every token valid
 *   out        [B, S, D] in x_dtype; padded rows are written as exact zeros.
 * A forward on another stream than the plan's previous forward first waits for that
 * one (the workspace is the plan's): forwards of one plan never overlap.
 * Device errors surface without a synchronisation: the last kernel of each forward
 * copies a non-zero device status word (a bounded device wait gave up) into the plan's
 * pinned host mirror, and the next tttj_forward of the plan that finds it set returns
 * TTTJ_ERR_DEVICE_TIMEOUT (launching nothing) and clears it.
 * A forward enqueued while `stream` is capturing becomes part of the CUDA graph: it
 * builds its token plan from valid_mask at every replay, does not wait for the plan's
 * previous forward (the capturing caller orders the capture and its replays), and
 * from then on no forward of the plan reuses a token plan left in the workspace.
 * Per-kernel timing must be off while capturing; a replay's device errors are read
 * with tttj_plan_status.
 * Replaces the pybind forward(input, valid_mask, packed_weights, capture_debug)
 * (kernels/csrc/sequence_resident.cpp:23-32), its per-launch error check
 * (C10_CUDA_KERNEL_LAUNCH_CHECK, kernels/csrc/sequence_resident.cu:531) and the Python
 * forward SequenceResidentTransformer.forward (kernels/sequence_resident.py:227-233). */
int tttj_forward(tttj_plan* plan, const void* x, int x_dtype, const uint8_t* valid_mask,
                 void* out, void* stream);

/* ---- context parallelism: one sequence split across ranks ----
 *
 * For batches smaller than the number of GPUs (the north star's C4, 4 sequences of
 * 8192 tokens, on 8 GPUs): the valid tokens [0, seq_len_valid) of ONE sequence are
 * shared out between ranks in contiguous slices; rank r runs every GEMM of the stack on
 * its own rows only, and after each layer's QKV GEMM one exchange -- an all-gather of
 * the ranks' q|k|v rows, enqueued by the caller -- gives every rank the whole
 * sequence's keys and values, so its attention (its own queries against all earlier
 * keys) is exact.  No counterpart in the reference (single-GPU only).
 *
 * A split plan: cfg->batch_size = 1 and cfg->seq_len = this rank's row count; its rows
 * are [row_lo, row_lo + seq_len) of the sequence (row_lo a multiple of the attention
 * work item: 256 rows, 128 at head_dim 256; a share that ends before the sequence does
 * ends on such a multiple too).  The plan's q|k|v buffer holds full_rows (>= the valid
 * length) rows of the whole sequence, this rank's at their positions: with shares of
 * at most m rows, rank r's rows at r * m and full_rows = ranks * m, an in-place
 * all-gather of m-row slices fills it (the first rank takes the largest share, so the
 * slices are contiguous).  tttj_plan_cp_qkv reports where that buffer lives in the
 * workspace.  tttj_forward_cp calls exchange(user, layer, stream) once per layer,
 * after the rank's q|k|v rows are enqueued on `stream`; the callback enqueues the
 * all-gather on the same stream (returning non-zero aborts the forward).  x and out are
 * the rank's own rows [seq_len, d_model].  Under stream capture (as tttj_forward) the
 * callback runs once, while capturing, and its enqueued all-gathers become part of the
 * graph; every rank of the group must capture and replay the same forwards. */
typedef int (*tttj_exchange_fn)(void* user, int layer, void* stream);
size_t tttj_workspace_bytes_cp(const tttj_config* cfg, int full_rows);
int tttj_plan_create_cp(const tttj_config* cfg, int device, const void* weights, const void* folded,
                        int seq_len_valid, int row_lo, int full_rows, void* workspace,
                        size_t workspace_bytes, tttj_plan** out_plan);
int tttj_plan_cp_qkv(tttj_plan* plan, size_t* offset, size_t* row_bytes, int* full_rows);
int tttj_forward_cp(tttj_plan* plan, const void* x, int x_dtype, void* out,
                    tttj_exchange_fn exchange, void* user, void* stream);

/* Forward path of a plan.  The resident-stack kernel runs the whole forward of
 * sequences of at most 128 tokens in one launch (one CTA per sequence); it fits
 * d_model <= 128 or 256 with layout head_dim 32/64/128 and enough TMEM / shared memory.
 * TTTJ_PATH_AUTO (the default) takes it for the shapes where it measured faster than
 * the layer-by-layer kernels (small layers: few heads, little weight per layer), else
 * the layer-by-layer kernels; TTTJ_PATH_LAYERWISE always takes the layer-by-layer
 * kernels; TTTJ_PATH_RESIDENT takes the resident kernel whenever it fits (set_path
 * returns TTTJ_ERR_INVALID when it does not).  tttj_plan_path reports the choice.
 * The resident kernel replaces the reference's sequence-resident and fused Triton
 * megakernels (kernels/sequence_resident.py:125-233, kernels/fused_megakernel.py:1860). */
#define TTTJ_PATH_AUTO 0
#define TTTJ_PATH_LAYERWISE 1
#define TTTJ_PATH_RESIDENT 2
int tttj_plan_set_path(tttj_plan* plan, int path);
/* 1 if tttj_forward of this plan runs the resident-stack kernel, 0 if layer by layer. */
int tttj_plan_path(tttj_plan* plan);
/* Host-only view of the same decision for a configuration: *fits = 1 if the resident
 * kernel can run it (TTTJ_PATH_RESIDENT accepted), *preferred = 1 if TTTJ_PATH_AUTO
 * takes it, *heads_per_step = heads per attention step inside the resident kernel. */
int tttj_path_choice(const tttj_config* cfg, int* fits, int* preferred, int* heads_per_step);

/* Per-stage capture for numerics bisection: the same forward as tttj_forward (always
 * layer by layer), which also writes, for batch index `sequence` at block `layer`, the
 * stages of the reference's capture_debug dump (kernels/sequence_resident.py:28-46,
 * kernels/csrc/sequence_resident.cu:355-450, there fixed to sequence 0, layer 0) into
 * `debug` (device, fp32, tttj_debug_floats(cfg) values), in this order:
 *   layernorm [S, D]           LN1 output
 *   qkv.q, qkv.k, qkv.v [S, D] projections (LayerNorm-folded GEMM, fp16 values)
 *   scores [H, S, S]           q k^T hd^-0.5, -inf at masked keys
 *   softmax [H, S, S]          probabilities (recomputed in fp32 from q, k)
 *   pv [S, D]                  attention output before out_proj
 *   output_projection [S, D]   attention branch added to the residual
 *   ffn [S, D]                 FFN branch added to the residual
 * then 2 [S, D] scratch blocks.  Positions are the sequence's token positions; padded
 * positions are zeros (rows of padded queries too). */
size_t tttj_debug_floats(const tttj_config* cfg);
int tttj_forward_debug(tttj_plan* plan, const void* x, int x_dtype, const uint8_t* valid_mask,
                       void* out, int layer, int sequence, float* debug, void* stream);

/* Synchronise the plan's device and read (then clear) the device status word that
 * bounded device waits write on timeout, and its host mirror.  *device_status = 0
 * when healthy. */
int tttj_plan_status(tttj_plan* plan, int* device_status);

/* ---- instrumentation ---- */

/* Number of kernel launches the next tttj_forward of this plan enqueues if it is given
 * the same kind of mask as the last one: on the layer-by-layer path a forward without a
 * mask reuses the all-valid token plan the previous mask-free forward built, one launch
 * fewer. */
int tttj_plan_launch_count(tttj_plan* plan);

/* Kernel classes of the forward, for per-class timing. */
#define TTTJ_KCLASS_PLAN 0
#define TTTJ_KCLASS_LAYERNORM 1
#define TTTJ_KCLASS_GEMM_QKV 2
#define TTTJ_KCLASS_ATTENTION 3
#define TTTJ_KCLASS_GEMM_OUT 4
#define TTTJ_KCLASS_GEMM_FFN_IN 5
#define TTTJ_KCLASS_GEMM_FFN_OUT 6
#define TTTJ_KCLASS_FINAL_LN 7
#define TTTJ_KCLASS_RESIDENT 8 /* the whole stack in one launch (resident path) */
#define TTTJ_KCLASS_COUNT 9

/* With timing enabled, every later tttj_forward records a CUDA event pair around
 * each launch on the forward's stream; tttj_plan_kernel_times returns, per class,
 * the summed device milliseconds and launch count since timing was enabled (it
 * waits for the last timed forward).  Enabling resets the totals.  Replaces the
 * reference's per-step timing scripts (benchmarks/benchmark_step_6.py:40-54). */
int tttj_plan_enable_timing(tttj_plan* plan, int enable);
int tttj_plan_kernel_times(tttj_plan* plan, double* total_ms /* [TTTJ_KCLASS_COUNT] */,
                           long* launches /* [TTTJ_KCLASS_COUNT] */);
const char* tttj_kernel_class_name(int cls);

/* ---- per-kernel entry points (same kernels the forward launches) ---- */

/* Linear layer with fused epilogue: out = epi(a @ w^T + bias).
 * Replaces F.linear / nn.Linear on the hot path (torch_transformer_benchmark.py:93-95,
 * 118, 141) and the reference's Triton epilogue kernels linear_gelu /
 * linear_residual_layer_norm (kernels/case13_linear.py:262-376).
 *   a [rows, k] fp16 (row stride lda), w [n, k] fp16 (row stride ldw), bias [n] fp32,
 *   out [rows, n] fp16 (ldo); residual [rows, n] fp16 (ldr) for TTTJ_EPI_BIAS_RESIDUAL
 *   (out may equal residual).  rows_dev (nullable) holds a device row count <= rows.
 *   n % 32 == 0, k % 8 == 0, strides multiples of 8 elements. */
#define TTTJ_EPI_BIAS 0
#define TTTJ_EPI_BIAS_GELU 1
#define TTTJ_EPI_BIAS_RESIDUAL 2
#define TTTJ_EPI_BIAS_RESIDUAL_F32 3 /* out and residual fp32 (the forward's residual stream) */
int tttj_linear(const void* a, int lda, const void* w, int ldw, const float* bias, void* out,
                int ldo, const void* residual, int ldr, int rows, const int* rows_dev, int n, int k,
                int epilogue, int* status_dev, void* stream);

/* nn.LayerNorm over rows of an fp16 [rows, d] matrix (d % 8 == 0, d <= 2048),
 * fp32 statistics, biased variance.  Replaces standalone_layer_norm /
 * residual_layer_norm (kernels/case13_fusions.py:137-215, kernels/case8_fusions.py:223). */
int tttj_layernorm(const void* in, void* out, int rows, int d, const float* gamma,
                   const float* beta, float eps, void* stream);

/* Fused multi-head attention over the packed valid-token layout.
 *   qkv  [qkv_rows, 3*d_model] fp16: valid tokens of sequence 0, then 1, ... in token
 *        order; columns q | k | v with head h at h*head_dim; head_dim = d_model /
 *        num_heads must be 32, 64, 128 or 256.  qkv_rows (>= the number
 *        of valid tokens Tv) is the number of rows allocated in qkv and ctx.
 *   ctx  [qkv_rows, d_model] fp16 output (rows of valid tokens are written).
 *   valid_mask [batch, seq_len] bytes or NULL (all valid) -- defines the packing.
 * Replaces packed_causal_attention / two_pass_causal_attention
 * (kernels/case8_attention.py:168, kernels/case14_attention.py:181) and the
 * score/softmax/PV sequence of BaselineSelfAttention.forward
 * (torch_transformer_benchmark.py:97-117).  `workspace` (device, at least
 * tttj_attention_workspace_bytes) holds the token plan and work list. */
size_t tttj_attention_workspace_bytes(int batch, int seq_len, int num_heads);
int tttj_attention(const void* qkv, void* ctx, int qkv_rows, const uint8_t* valid_mask, int batch,
                   int seq_len, int d_model, int num_heads, int causal, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Allocation-free variant of tttj_attention (no counterpart in the reference).
 * For callers that cannot allocate device memory at call time -- code running inside
 * an allocator or memory-pool callback, hosts that forbid cudaMalloc after start-up,
 * runtimes that only pass pre-placed input/output buffers.  Same arguments and
 * results as tttj_attention, minus the workspace: the token plan and work list live
 * in a fixed device array of TTTJ_ATTENTION_NOALLOC_SCRATCH_BYTES inside the library
 * (held on every GPU that loads the library until the process exits).  Shapes whose
 * plan does not fit return TTTJ_ERR_INVALID without launching anything.  It calls no
 * allocation routine itself.  The first call in each CUDA context (the first call on a
 * device, and again after cudaDeviceReset) looks up the array's device address with
 * that device current, and under lazy module loading may make the CUDA runtime load
 * the library's device code, which allocates: make that first call -- a warm-up call
 * at start-up will do -- before any stream capture and outside any allocator or
 * memory-pool callback.  All calls on a device share the array, so calls that overlap
 * on the GPU race; nothing in it needs clearing between calls. */
#define TTTJ_ATTENTION_NOALLOC_SCRATCH_BYTES (4u << 20)
int tttj_attention_noalloc(const void* qkv, void* ctx, int qkv_rows, const uint8_t* valid_mask,
                           int batch, int seq_len, int d_model, int num_heads, int causal,
                           void* stream);

/* Failure-detection self test: launches a kernel whose bounded wait on an mbarrier
 * that is never signalled gives up after limit_ns and writes 0x1ff into *status_dev.
 * No counterpart in the reference (its device waits are unbounded). */
int tttj_selftest_wait_timeout(int* status_dev, uint64_t limit_ns, void* stream);
/* The same wait, reported through a plan (its device status word and host mirror, as a
 * forward's kernel would report it): the plan's next tttj_forward returns
 * TTTJ_ERR_DEVICE_TIMEOUT.  limit_ns <= 1 s. */
int tttj_plan_selftest_timeout(tttj_plan* plan, uint64_t limit_ns, void* stream);

/* Number of SMs of `device` (grid sizing of the persistent kernels). */
int tttj_device_sm_count(int device);

/* Tile shape of a GEMM of rows x n x k with `epilogue` on num_sms SMs, as tttj_linear
 * and the forward choose it: *bn = output columns per tile (64, 128 or 256), *pair = 1
 * for 256-row tiles computed by a CTA pair.  Host-only (no device is touched).
 * `epilogue` is a TTTJ_EPI_* code or one of the forward's fused epilogues below. */
#define TTTJ_EPI_RESIDUAL_F32_STATS 4 /* out_proj / ffn_out: fp32 residual + LN statistics */
#define TTTJ_EPI_LN_FOLD 5            /* QKV: LayerNorm folded into the weights */
#define TTTJ_EPI_LN_FOLD_GELU 6       /* ffn_in: LayerNorm fold + erf-GELU */
int tttj_gemm_tile(int rows, int n, int k, int epilogue, int num_sms, int* bn, int* pair);

#ifdef __cplusplus
}
#endif

#endif /* TTTJ_B200_H */
