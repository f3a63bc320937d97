/*
 * gdc.h — C ABI of the B200 GLiNER2.5-Decide classification backend.
 *
 * Drop-in for the GLiNERDecideCore hot path of shantanugoel/gliner-decide-metal:
 * model load from one fp16 safetensors file, bucketed batch classify returning
 * logits [B, maxHeads, maxOptions], and per-task probabilities. Each entry point
 * below names the reference interface it replaces (paths relative to that project).
 *
 * Conventions
 *  - Every function returns a gdc_status; nothing aborts. On failure a message is
 *    available from gdc_last_error() (thread-local, valid until the next call on
 *    the same thread).
 *  - Host pointers are caller-owned. Device pointers (the *_device entry points)
 *    are caller-owned device memory on the model's device.
 *  - A gdc_model lives on one CUDA device. Calls on one handle are serialised by
 *    an internal mutex; distinct handles may be used concurrently from different
 *    host threads.
 */
#ifndef GDC_H_
#define GDC_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDC_ABI_VERSION 1

/* Status codes. The first five mirror the reference's thrown errors:
 * WeightStoreError.{missingWeight, invalidShape, invalidInput} (Weights.swift:4-19)
 * and NativeTokenizerError.{inputDoesNotFit, noTaskLabels} (NativeTokenizer.swift:5-23).
 * The reference's precondition()/fatalError() traps (FusedKernels.swift:176-182,
 * 229-232, 269-272) become GDC_ERR_INVALID_INPUT here. */
typedef enum gdc_status {
  GDC_OK = 0,
  GDC_ERR_MISSING_WEIGHT = 1,
  GDC_ERR_INVALID_SHAPE = 2,
  GDC_ERR_INVALID_INPUT = 3,
  GDC_ERR_INPUT_DOES_NOT_FIT = 4,
  GDC_ERR_NO_TASK_LABELS = 5,
  GDC_ERR_IO = 6,            /* file missing, truncated or not safetensors */
  GDC_ERR_CUDA = 7,          /* CUDA runtime / driver error */
  GDC_ERR_OUT_OF_MEMORY = 8, /* device allocation failed */
  GDC_ERR_TIMEOUT = 9,       /* a bounded device-side wait gave up */
  GDC_ERR_UNSUPPORTED = 10,  /* configuration outside what the kernels implement */
  GDC_ERR_NULL_POINTER = 11,
  GDC_ERR_PARTIAL = 12       /* sharded call: some devices failed (see per-device codes) */
} gdc_status;

typedef enum gdc_dtype {
  GDC_INT32 = 0,
  GDC_INT64 = 1,
  GDC_FLOAT16 = 2,
  GDC_FLOAT32 = 3,
  GDC_UINT8 = 4
} gdc_dtype;

/* DeBERTaV2Configuration (Configuration.swift:3-49) plus the init flags of
 * GLiNERDecideClassifier.init (DeBERTa.swift:188-196). The flags choose between
 * MLX implementations in the reference; this backend has one native path and
 * accepts and ignores them. vocab_size is the word-embedding row count the loader
 * requires (the reference hard-checks 128011, DeBERTa.swift:199-202). */
typedef struct gdc_config {
  int32_t hidden_size;             /* 1024 */
  int32_t intermediate_size;       /* 4096 */
  int32_t num_hidden_layers;       /* 24 */
  int32_t num_attention_heads;     /* 16 */
  float layer_norm_eps;            /* 1e-7 */
  int32_t position_buckets;        /* 256 */
  int32_t max_relative_positions;  /* -1 (the forward uses 512, DeBERTa.swift:505) */
  int32_t pad_token_id;            /* 0 */
  int32_t vocab_size;              /* 128011 */
  int32_t use_fused_kernels;          /* accepted, ignored */
  int32_t use_compiled_graph;         /* accepted, ignored */
  int32_t use_fast_attention;         /* accepted, ignored */
  int32_t use_custom_relative_kernel; /* accepted, ignored */
  int32_t use_fused_attention_kernel; /* accepted, ignored */
} gdc_config;

/* DeBERTaV2Configuration.default (Configuration.swift:38-48). */
void gdc_config_default(gdc_config* cfg);

/* DecisionInput (DeBERTa.swift:22-58): host arrays, row-major.
 *  input_ids      [batch, seq_len]                 int32 or int64
 *  attention_mask [batch, seq_len]                 float16, float32, uint8, int32 or int64
 *                                                  (a position is valid when > 0)
 *  marker_indices [batch, max_heads, max_options]  int32 or int64, each in [0, seq_len)
 *  marker_mask    [batch, max_heads, max_options]  float32, float16 or uint8 */
typedef struct gdc_input {
  int32_t batch;
  int32_t seq_len;
  int32_t max_heads;
  int32_t max_options;
  const void* input_ids;
  gdc_dtype ids_dtype;
  const void* attention_mask;
  gdc_dtype mask_dtype;
  const void* marker_indices;
  gdc_dtype marker_dtype;
  const void* marker_mask;
  gdc_dtype marker_mask_dtype;
} gdc_input;

/* ProfileEvent (DeBERTa.swift:7-12). */
typedef struct gdc_profile_event {
  char name[48];
  uint64_t nanoseconds;
} gdc_profile_event;

/* InferenceResult (DeBERTa.swift:14-20). Caller-owned buffers:
 *  logits      float32 [batch, max_heads, max_options] (required)
 *  logits_f16  uint16 (IEEE half bits) same shape, optional (NULL to skip); these are
 *              the values the reference returns (its logits array is fp16).
 *  events      optional array of events_capacity entries, filled when profiling. */
typedef struct gdc_output {
  float* logits;
  uint16_t* logits_f16;
  uint64_t wall_ns;
  gdc_profile_event* events;
  int32_t events_capacity;
  int32_t events_count;
} gdc_output;

typedef struct gdc_model gdc_model;

/* GLiNERDecideClassifier.init(weightsURL:configuration:...) (DeBERTa.swift:188-242)
 * with WeightStore(url:) (Weights.swift:26-28). Loads every tensor from one
 * safetensors file (F16, or F32/BF16 converted to fp16), checks keys and shapes
 * (missing key -> GDC_ERR_MISSING_WEIGHT, wrong shape -> GDC_ERR_INVALID_SHAPE),
 * uploads them to `device`, and precomputes LN(rel_embeddings) and the per-layer
 * relative query/key projections on the device. cfg may be NULL (defaults). */
gdc_status gdc_model_load(const char* safetensors_path, const gdc_config* cfg, int device,
                          gdc_model** out);

/* Releases all device memory of the model. NULL is ignored. */
void gdc_model_free(gdc_model* model);

/* Device ordinal, and the classifier hidden width read from the file. */
int gdc_model_device(const gdc_model* model);
int gdc_model_classifier_hidden(const gdc_model* model);

/* GLiNERDecideClassifier.classify(_:collectProfile:) (DeBERTa.swift:244-272).
 * Copies the host input to the device, runs the forward, copies logits back and
 * synchronises. collect_profile != 0 records per-stage device times with the
 * reference's stage names (embedding, layer_i_attention_projection,
 * layer_i_attention, layer_i_attention_output, layer_i_feed_forward, classifier). */
gdc_status gdc_classify(gdc_model* model, const gdc_input* input, int collect_profile,
                        gdc_output* output);

/* Device-resident variant of gdc_classify for callers that keep inputs in HBM.
 * Same shapes as gdc_input; dtypes fixed: ids int32, attention_mask float16,
 * marker_indices int32, marker_mask float32; logits float32 device buffer (and
 * optional fp16). Enqueues on `stream` (a cudaStream_t, NULL = the model's stream)
 * and returns without synchronising. Inputs are checked on the device: an
 * out-of-range id or marker index sets a flag reported by gdc_check_errors().
 * All calls on one model share its device workspace: calls enqueued on different
 * streams must be ordered by the caller (the internal mutex only orders the host side). */
gdc_status gdc_classify_device(gdc_model* model, int32_t batch, int32_t seq_len,
                               int32_t max_heads, int32_t max_options,
                               const int32_t* d_input_ids, const uint16_t* d_attention_mask,
                               const int32_t* d_marker_indices, const float* d_marker_mask,
                               float* d_logits, uint16_t* d_logits_f16, void* stream);

/* Reads and clears the model's device error flags (bounded-wait timeouts,
 * out-of-range ids/markers seen by gdc_classify_device). Waits first for every forward
 * already enqueued by gdc_classify_device, on the model's stream or on a caller's stream
 * (each such call ends by making the model's stream wait on the caller's), so the flags of
 * those calls are complete when they are read. */
gdc_status gdc_check_errors(gdc_model* model);

/* The model's CUDA stream (cudaStream_t) — for event timing by callers. */
void* gdc_model_stream(gdc_model* model);

/* Encoder row layout. enabled != 0 (the default; environment GDC_PACK_ROWS=0 makes dense
 * the default): each batch row's positions [0, ext) are packed back to back and only those
 * rows go through the encoder, ext = 1 + the last position with attention_mask > 0 or an
 * active marker index, whichever is larger (ext = seq_len for a row with no valid
 * position). enabled == 0: the dense [batch, seq_len] grid, as the reference computes it.
 * The logits are bit-identical either way: positions at or past ext reach a logit neither
 * as a gathered marker row nor as a key (their softmax weight is exactly zero). No
 * counterpart in the reference (DeBERTa.swift:274-447 always runs the dense grid).
 * gdc_classify runs a batch whose every row ends in a valid position on the dense grid
 * (there is nothing to remove; the packing pass would only add work).
 * Synchronises the model's stream and drops captured forwards when the setting changes. */
gdc_status gdc_model_set_row_packing(gdc_model* model, int enabled);
int gdc_model_row_packing(const gdc_model* model);

/* Stage-time recording for gdc_classify_device: when enabled, CUDA events bracket
 * every kernel group; gdc_profile_read sums their device time per event name over
 * all calls since the last reset (ns) and returns the count of entries written. */
gdc_status gdc_profile_enable(gdc_model* model, int enabled);
gdc_status gdc_profile_reset(gdc_model* model);
int gdc_profile_read(gdc_model* model, gdc_profile_event* events, int capacity,
                     int32_t* launches);

/* Row-sharded classify over several models (one per device, same weights): rows
 * are split into contiguous blocks, one host thread per device, logits gathered
 * into output->logits. There is no reference counterpart (the reference is
 * single-device); the result equals gdc_classify on one device row for row.
 * per_device_status (optional, n_models entries) receives each device's status;
 * if some fail the call returns GDC_ERR_PARTIAL. */
gdc_status gdc_classify_sharded(gdc_model* const* models, int n_models, const gdc_input* input,
                                gdc_output* output, gdc_status* per_device_status);

/* Per-task decode, RawCLI.swift:182-223 (float64 on the host).
 * logits [batch, max_heads, max_options] float32; n_labels [batch, max_heads] (labels of
 * task h of row b; 0 = no task); multi_label [batch, max_heads] (0/1).
 * probabilities [batch, max_heads, max_options] float64 (unused slots = 0);
 * selected [batch, max_heads, max_options] uint8 (1 = label chosen).
 * Multi-label: sigmoid(x), select p >= 0.5, else the first argmax. Single-label:
 * max-subtracted softmax over the task's labels, first argmax. */
gdc_status gdc_decode(const float* logits, int32_t batch, int32_t max_heads, int32_t max_options,
                      const int32_t* n_labels, const uint8_t* multi_label,
                      double* probabilities, uint8_t* selected);

/* Same decode on the device (for callers keeping logits in HBM), RawCLI.swift:182-223:
 * float64 arithmetic as the reference's Double, probabilities stored as float32,
 * selections identical to gdc_decode's. All pointers are device pointers; enqueued on
 * `stream` (NULL = the model's stream). */
gdc_status gdc_decode_device(gdc_model* model, const float* d_logits, int32_t batch,
                             int32_t max_heads, int32_t max_options, const int32_t* d_n_labels,
                             const uint8_t* d_multi_label, float* d_probabilities,
                             uint8_t* d_selected, void* stream);

/* Length-bucket selection, NativeTokenizer.swift:85-88,134-137: the smallest bucket
 * >= unpadded_length over the sorted unique set of `buckets`.
 * GDC_ERR_INPUT_DOES_NOT_FIT if none fits or the set is empty. */
gdc_status gdc_select_bucket(int32_t unpadded_length, const int32_t* buckets, int32_t n_buckets,
                             int32_t* selected);

/* Padded row layout of NativeDecisionTokenizer.makeInput after tokenisation
 * (NativeTokenizer.swift:81-82,134-157). token_ids [n_tokens]; task t's label-marker
 * start positions are marker_positions[marker_offsets[t] .. marker_offsets[t+1]).
 * Writes the chosen bucket L, max_heads = max(n_tasks, 1), max_options =
 * max(labels per task, 1); then, if the caller's buffers are large enough
 * (capacities in elements), ids [L] (pad_id-filled), mask [L] (1/0 as float32),
 * marker_indices [max_heads*max_options] (unused slots 0) and marker_mask (0/1).
 * GDC_ERR_NO_TASK_LABELS when n_tasks == 0 or a task has no labels;
 * GDC_ERR_INPUT_DOES_NOT_FIT when no bucket fits. Buffers too small ->
 * GDC_ERR_INVALID_INPUT after writing the three sizes. */
gdc_status gdc_layout_row(const int32_t* token_ids, int32_t n_tokens,
                          const int32_t* marker_positions, const int32_t* marker_offsets,
                          int32_t n_tasks, const int32_t* buckets, int32_t n_buckets,
                          int32_t pad_id, int32_t* bucket_len, int32_t* max_heads,
                          int32_t* max_options, int32_t* ids_out, int32_t ids_capacity,
                          float* mask_out, int32_t* marker_out, float* marker_mask_out,
                          int32_t marker_capacity);

/* Relative-position gather index used by the attention kernels,
 * DeBERTa.swift:498-551: table[r + 511] = clip(bucket(r) + 256, 0, 511) for
 * r = q - k in [-511, 511] (1023 entries). c2p for (q, k) reads position
 * table[q - k + 511]; p2c reads the same index (the reference's p2c table is
 * clip(-bucket(k - q) + 256)). */
gdc_status gdc_relative_index_table(int32_t position_buckets, int32_t max_relative_positions,
                                    int32_t* table_out /* 1023 */);

/* ---- Kernel-level entry points (device pointers; enqueued on `stream`). ----
 * These mirror the reference's FusedKernels (FusedKernels.swift) and are what the
 * forward uses internally; they are exposed for microbenchmarks and tests. */

/* FusedKernels.residualLayerNorm (FusedKernels.swift:261-286):
 * out = LN(x + residual) * weight + bias over the last axis, fp32 statistics.
 * x, residual (may be NULL), out: [rows, cols] fp16; weight, bias: [cols] fp16.
 * cols must be a multiple of 256 and <= 4096. */
gdc_status gdc_residual_layer_norm(const uint16_t* x, const uint16_t* residual,
                                   const uint16_t* weight, const uint16_t* bias, uint16_t* out,
                                   int64_t rows, int32_t cols, float eps, void* stream);

/* FusedKernels.fusedAttention (FusedKernels.swift:160-210) with the position tables
 * of DeBERTa.swift:322-395: per (b, h) computes
 *   s[q,k] = (q.k)/sqrt(3d) + (q.PK[idx(q-k)] + k.PQ[idx(q-k)]) / sqrt(3d) + mask[k]
 * (mask[k] = -65504 where key_mask[b,k] <= 0), softmax over k, ctx = P V.
 * qkv: [batch*seq_len, 3*heads*64] fp16 (q | k | v column blocks, the QKV projection
 * output); pos_qk: [512, 2*heads*64] fp16 (PQ | PK column blocks);
 * key_mask: [batch, seq_len] fp16; ctx: [batch*seq_len, heads*64] fp16.
 * heads*64 must equal 1024 and seq_len must be in [1, 512]. */
gdc_status gdc_disentangled_attention(const uint16_t* qkv, const uint16_t* pos_qk,
                                      const uint16_t* key_mask, uint16_t* ctx, int32_t batch,
                                      int32_t seq_len, int32_t heads, void* stream);

/* Same contract as gdc_disentangled_attention, computed by a CUDA-core kernel with one
 * warp per query row (the structure of FusedKernels.swift:13-81). Used to cross-check
 * the tensor-core kernel on the device at sizes the CPU oracle cannot reach; the forward
 * does not use it. */
gdc_status gdc_disentangled_attention_scalar(const uint16_t* qkv, const uint16_t* pos_qk,
                                             const uint16_t* key_mask, uint16_t* ctx, int32_t batch,
                                             int32_t seq_len, int32_t heads, void* stream);

/* Allocation-free variant of gdc_disentangled_attention; it has no counterpart in the
 * reference. Same arguments, layout and results. It is for callers that cannot let a
 * library call cudaMalloc: hosts that reserve all device memory for their own pool up
 * front, or that must not take the implicit device synchronisation and address-space
 * change of an allocation in the middle of their run. The scratch that
 * gdc_disentangled_attention allocates (the expanded position table of the call, rebuilt
 * from pos_qk by every call, the relative index table and a status word; 4,194,560 bytes in
 * all) is a file-scope __device__ array that every device loading this library holds until
 * the process exits; nothing here calls cudaMalloc, cudaFree or an allocating library
 * routine.
 *  - Limit: heads must be 16 (the array holds one 1023 x 2048 table) and seq_len <= 512
 *    (the table covers |q - k| <= 511); other values return GDC_ERR_UNSUPPORTED.
 *  - The first call on a device sets the array up (resolves its device address and
 *    copies the relative index table in, synchronously); make that first call before any
 *    stream capture.
 *  - Each call clears the status word on `stream`, expands pos_qk into the array, launches,
 *    reads the status word back and synchronises `stream`, so it returns once the kernel has
 *    finished; a bounded-wait timeout is returned as GDC_ERR_TIMEOUT.
 *  - All calls on a device share the array and it keeps the last call's contents. Calls
 *    that overlap on the GPU (different streams or host threads) race on the expanded
 *    table and the status word. */
gdc_status gdc_disentangled_attention_noalloc(const uint16_t* qkv, const uint16_t* pos_qk,
                                              const uint16_t* key_mask, uint16_t* ctx, int32_t batch,
                                              int32_t seq_len, int32_t heads, void* stream);

/* addMM(bias, x, W^T) (DeBERTa.swift:69-71, 89-91) on tcgen05 tensor cores:
 * out[M,N] = act(a[M,K] . w[N,K]^T + bias[N]) in fp16 with fp32 accumulation;
 * act: 0 = none, 1 = exact-erf GELU, 2 = ReLU. N must be a multiple of 256 and K a
 * multiple of 64; a, w row-major; out row-major with leading dimension ldo. */
gdc_status gdc_linear(const uint16_t* a, const uint16_t* w, const uint16_t* bias, uint16_t* out,
                      int64_t M, int32_t N, int32_t K, int64_t ldo, int32_t act, void* stream);

/* Reads and clears the current device's error word used by the kernel-level entry
 * points above (bounded-wait timeouts). Synchronises the device. */
gdc_status gdc_kernels_check_errors(void);

/* Failure-detection self-test (no counterpart in the reference): launches a kernel whose
 * bounded wait on a barrier that nothing completes runs out after limit_us microseconds
 * (1 .. 1e6), exactly like a stuck wait in the forward's kernels. The kernel sets the
 * timeout bit of the current device's error word and returns, so the next
 * gdc_kernels_check_errors() reports GDC_ERR_TIMEOUT and clears it; the device stays usable. */
gdc_status gdc_selftest_wait_timeout(int32_t limit_us, void* stream);

/* Last error message of this thread. */
const char* gdc_last_error(void);

/* ABI version (GDC_ABI_VERSION) and a build string. */
int gdc_abi_version(void);
const char* gdc_build_info(void);

#ifdef __cplusplus
}
#endif

#endif /* GDC_H_ */
