/*
 * needle_b200.h — B200 extensions of the needle C ABI.
 *
 * The reference exposes only text-level calls (needle.h); its engine API
 * also has NeedleEngine::run_batch (crates/needle-infer/src/engine.rs:142-144)
 * and its tests drive NeedleModel::encode / decode_step directly
 * (crates/needle-core/tests/parity_tests.rs:345-594).  These entry points
 * expose the same paths on token IDs, batched and sharded for the GPU, plus
 * the INT4 kernels of crates/needle-core/src/quant.rs on device pointers.
 *
 * Return convention: int results are 0 (or a count) on success and -1 on
 * failure with needle_last_error() set.  All pointers are host pointers
 * unless NEEDLE_DEVICE_POINTERS is passed (batched calls) or the function
 * says "device".
 */
#ifndef NEEDLE_B200_H
#define NEEDLE_B200_H

#include "needle.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ── devices ─────────────────────────────────────────────────────────────── */

/* Number of visible CUDA devices (0 when none; never fails). */
int needle_device_count(void);

/* needle_load / needle_load_bytes onto an explicit device. */
NeedleHandle *needle_load_on_device(const char *weights_path, const char *vocab_path, int device);
NeedleHandle *needle_load_bytes_on_device(const uint8_t *weights_data, size_t weights_len,
                                          const uint8_t *vocab_data, size_t vocab_len, int device);

/* cfg[0..11] = d_model, num_heads, num_kv_heads, num_encoder_layers,
 * num_decoder_layers, vocab_size, max_enc_len, max_dec_len, ffn_dim,
 * no_feedforward, activation (0 drelu, 1 swiglu, 2 geglu), head_dim
 * (crates/needle-core/src/config.rs:22-69). */
int needle_model_config(NeedleHandle *handle, int64_t *cfg);
int needle_handle_device(NeedleHandle *handle);

/* ── batched generation on token IDs ─────────────────────────────────────── */

#define NEEDLE_STOP_ON_EOS 1u     /* end a request at EOS, as run_impl does (engine.rs:306-308) */
#define NEEDLE_DEVICE_POINTERS 2u /* prompt_ids / mask_bits / outputs are device pointers */
#define NEEDLE_NO_GRAPH 4u        /* launch decode steps one kernel at a time (no CUDA graph) */
#define NEEDLE_NO_PDL 8u          /* decode kernels wait for their predecessor to finish before they launch
                                     (no programmatic dependent launch); results are the same either way */

/* Greedy generation for n_req independent requests (run_batch,
 * engine.rs:142-144, with the decode loop of engine.rs:286-322 on IDs):
 *   prompt_ids      concatenated encoder inputs (each 1..max_enc_len ids < vocab)
 *   prompt_offsets  host array [n_req + 1]: request r = ids[off[r] .. off[r+1])
 *   max_new         decode steps, <= max_dec_len; decoding starts from EOS (1)
 *   mask_bits       NULL (unconstrained) or [n_req][max_new][ceil(V/64)] u64:
 *                   bit v of a step's row set = token v allowed (additive 0),
 *                   clear = additive -1e9 (constrained.rs:369-387)
 *   out_ids         [n_req][max_new] generated ids (EOS excluded when stopping)
 *   out_lens        [n_req] tokens generated per request
 * Ties pick the last maximal index (Iterator::max_by(total_cmp)). */
int needle_run_batch_ids(NeedleHandle *handle, const uint32_t *prompt_ids, const uint64_t *prompt_offsets,
                         size_t n_req, uint32_t max_new, const uint64_t *mask_bits, uint32_t flags,
                         uint32_t *out_ids, uint32_t *out_lens);

/* Prepared batch: needle_batch_prepare uploads the inputs and allocates the
 * per-call device state once; needle_batch_run enqueues prefill + decode on
 * the batch's own stream without host copies (re-running restarts from the
 * prompts); needle_batch_sync waits; needle_batch_results copies out. */
typedef struct NeedleBatch NeedleBatch;
NeedleBatch *needle_batch_prepare(NeedleHandle *handle, const uint32_t *prompt_ids, const uint64_t *prompt_offsets,
                                  size_t n_req, uint32_t max_new, const uint64_t *mask_bits, uint32_t flags);
int needle_batch_run(NeedleBatch *batch);
int needle_batch_sync(NeedleBatch *batch);
int needle_batch_results(NeedleBatch *batch, uint32_t *out_ids, uint32_t *out_lens);
/* Step-wise decoding for callers that build each step's vocabulary mask from
 * the tokens so far (the loop of engine.rs:286-322 with their own grammar):
 * needle_batch_begin runs the prefill; needle_batch_set_step_mask replaces
 * the mask rows [n_req][ceil(V/64)] of one step (the batch must have been
 * prepared with mask_bits); needle_batch_step runs the next decode step and
 * returns its token per request with lens / done (any may be NULL; the token
 * of a request that is done, at EOS or earlier, is unspecified). */
int needle_batch_begin(NeedleBatch *batch);
int needle_batch_set_step_mask(NeedleBatch *batch, uint32_t step, const uint64_t *rows);
int needle_batch_step(NeedleBatch *batch, uint32_t *tokens, uint32_t *lens, uint8_t *done);
/* The cudaStream_t the batch runs on (as void *), for the caller's events. */
void *needle_batch_stream(NeedleBatch *batch);
/* Kernels the last needle_batch_run launched. */
int64_t needle_batch_kernel_launches(NeedleBatch *batch);
/* Time one kernel class in later runs: CUDA events around each of its
 * launches on the batch's stream (decode steps then launch eagerly, without
 * a CUDA graph).  Classes: 0 none, 1 decoder cross-attention, 2 prefill
 * INT4 matmuls, 3 decode INT4 matmuls, 4 output head, 5 encoder attention,
 * 6 decoder self-attention, 7 elementwise kernels (norms, embedding, q/k
 * post-processing, step bookkeeping).
 * needle_batch_kernel_timing reports, for the last run, the summed device
 * time, the launch count and the algorithmic flops and bytes of those
 * launches (bytes: every operand read once and every result written once). */
int needle_batch_time_kernel(NeedleBatch *batch, int kernel_class);
int needle_batch_kernel_timing(NeedleBatch *batch, double *ms_total, int64_t *launches, double *flops,
                               double *bytes);
void needle_batch_free(NeedleBatch *batch);

/* Splits requests into `shards` groups of near-equal cost, longest first
 * (one group per GPU; no collective is needed).  assignment: [n_req]. */
int needle_shard_requests(const uint64_t *prompt_offsets, size_t n_req, int shards, int32_t *assignment);

/* ── parity entry points ─────────────────────────────────────────────────── */

/* encode (model.rs:153-192) then one decode_step (model.rs:235-265) per
 * dec_ids[i], teacher-forced.  enc_out: NULL or [n_enc][d_model] final
 * encoder hidden; logits: NULL or [n_dec][V]. */
int needle_debug_forward(NeedleHandle *handle, const uint32_t *enc_ids, size_t n_enc, const uint32_t *dec_ids,
                         size_t n_dec, float *enc_out, float *logits);

/* Batched greedy generation that also returns the masked logits of every
 * step: logits [n_req][max_new][V].  Otherwise as needle_run_batch_ids. */
int needle_run_batch_ids_logits(NeedleHandle *handle, const uint32_t *prompt_ids, const uint64_t *prompt_offsets,
                                size_t n_req, uint32_t max_new, const uint64_t *mask_bits, uint32_t flags,
                                uint32_t *out_ids, uint32_t *out_lens, float *logits);

/* ── text front end (needle_run's tokenizer, tool JSON, constrained decoding) ─ */

/* NeedleEngine::run_batch (crates/needle-infer/src/engine.rs:142-144): run n
 * (query, tools_json) requests, each as needle_run would, decoded together
 * on the GPU with one constrained-decoding state per request.  out_texts[i]
 * receives a string to free with needle_free_str.  0 on success, -1 on
 * failure (no strings left allocated). */
int needle_run_batch(NeedleHandle *handle, const char *const *queries, const char *const *tools_json, size_t n,
                     char **out_texts);

/* The SentencePiece vocabulary of crates/needle-infer/src/tokenizer.rs:31-246
 * (one "piece\tscore" per line, line index = id; BPE by score, greedy
 * longest match for a file without scores). */
typedef struct NeedleVocab NeedleVocab;
/* Parse vocabulary text; NULL (error set) if it is not UTF-8.  Free with
 * needle_vocab_free. */
NeedleVocab *needle_vocab_parse(const char *text, size_t len);
/* The vocabulary a handle loaded (owned by the handle). */
const NeedleVocab *needle_handle_vocab(NeedleHandle *handle);
size_t needle_vocab_size(const NeedleVocab *vocab);
/* Vocabulary::encode: token ids of text (trimmed, SentencePiece-normalised);
 * writes min(count, cap) ids and returns the count; (size_t)-1 if text is not
 * UTF-8. */
size_t needle_vocab_encode(const NeedleVocab *vocab, const char *text, uint32_t *out, size_t cap);
/* Vocabulary::decode_ids (free the result with needle_free_str). */
char *needle_vocab_decode(const NeedleVocab *vocab, const uint32_t *ids, size_t n);
void needle_vocab_free(NeedleVocab *vocab);
/* to_snake_case of tokenizer.rs:248-292 (free with needle_free_str). */
char *needle_snake_case(const char *name);
/* The tools JSON as the encoder sees it: tool names in snake_case, whitespace
 * outside strings removed (engine.rs:233-239, 354-471). */
char *needle_tools_encoder_text(const char *tools_json);
/* Output with the tools' snake_case names replaced by the original names
 * (restore_tool_names, engine.rs:473-546). */
char *needle_tools_restore_names(const char *tools_json, const char *output);

/* ConstrainedDecoder (crates/needle-infer/src/constrained.rs:300-375): JSON
 * state machine + name / argument-key tries over a tools JSON. */
typedef struct NeedleConstraint NeedleConstraint;
NeedleConstraint *needle_constraint_new(const char *tools_json, const NeedleVocab *vocab);
/* Advance past an emitted token / raw output bytes. */
int needle_constraint_update(NeedleConstraint *c, uint32_t token);
int needle_constraint_feed(NeedleConstraint *c, const char *bytes, size_t len);
/* Allowed-token bitmap for the next step into bits[ceil(vocab_size/64)]
 * (bit set = allowed, the mask_bits format of needle_run_batch_ids): returns
 * 1 when the step is constrained, 0 when every token is allowed (bits all
 * set), -1 on bad arguments. */
int needle_constraint_mask(NeedleConstraint *c, size_t vocab_size, uint64_t *bits);
/* 0 free, 1 inside a tool name, 2 inside an argument key. */
int needle_constraint_state(const NeedleConstraint *c);
void needle_constraint_free(NeedleConstraint *c);

/* ── INT4 kernels on device pointers (reference layout, quant.rs:45-58) ──── */
/* w_data: [(G*gs/2)][N] bytes, low nibble = row 2p, high = row 2p+1;
 * w_scales: [G][N] f32, gs = min(32, K).  stream: cudaStream_t or NULL. */

/* y[M][N] = x[M][K] @ W  (QuantizedWeight::matmul, quant.rs:400-410).  Up to
 * 8 rows run on the CUDA cores, 9 rows or more on the tensor-core GEMM. */
int needle_int4_matmul(const float *x, size_t M, size_t K, const uint8_t *w_data, const float *w_scales, size_t N,
                       size_t num_groups, float *y, void *stream);
/* needle_int4_matmul with launch flags.  NEEDLE_INT4_OVERLAP lets the launch
 * begin while the previous kernel in the stream is still running: its weight
 * and scale loads are issued at once, x is read only after that kernel has
 * finished (programmatic dependent launch).  The caller promises that no work
 * still in flight in the stream writes w_data or w_scales.  Used up to 8
 * rows; ignored by the tensor-core path. */
#define NEEDLE_INT4_OVERLAP 1u
int needle_int4_matmul_ex(const float *x, size_t M, size_t K, const uint8_t *w_data, const float *w_scales, size_t N,
                          size_t num_groups, float *y, uint32_t flags, void *stream);

/* A prepared INT4 weight for repeated matmuls (the engine's own form of a
 * projection: QuantizedWeight kept in the reference layout plus, for the
 * tensor-core path, its bf16 hi/lo staging and a workspace for up to max_m
 * rows of x).  needle_int4_plan_matmul is asynchronous in `stream` and
 * allocates nothing; calls on one plan must be ordered (one stream), since
 * they share the workspace.  needle_int4_plan_status synchronises the device
 * and returns -1 if a bounded wait inside a tensor-core launch expired since
 * the last check. */
typedef struct NeedleInt4Plan NeedleInt4Plan;
NeedleInt4Plan *needle_int4_plan_create(const uint8_t *w_data, const float *w_scales, size_t K, size_t N,
                                        size_t num_groups, size_t max_m, void *stream);
int needle_int4_plan_matmul(NeedleInt4Plan *plan, const float *x, size_t M, float *y, uint32_t flags, void *stream);
int needle_int4_plan_status(NeedleInt4Plan *plan);
void needle_int4_plan_free(NeedleInt4Plan *plan);

/* Pack w[K][N] f32 (QuantizedWeight::quantize, quant.rs:63-128), bit-exact:
 * data [(Kp/2)][N], scales [Kp/gs][N] with Kp = K padded to gs. */
int needle_int4_quantize(const float *w, size_t K, size_t N, uint8_t *data, float *scales, void *stream);
/* Unpack to out[K][N] f32 (quant.rs:131-155), bit-exact. */
int needle_int4_dequantize(const uint8_t *data, const float *scales, size_t K, size_t N, size_t num_groups,
                           float *out, void *stream);
/* Gated MLP over T tokens (ffn_forward, crates/needle-core/src/ffn.rs:19-56):
 * out[T][d] = down(act(x @ gate) * (x @ up)); act 0 drelu, 1 swiglu,
 * 2 geglu.  Gate and up are fused into one pass whose epilogue applies the
 * activation; the [T][d_ff] hidden lives in a device buffer allocated per
 * call. */
int needle_ffn_forward(const float *x, size_t T, size_t d_model, size_t d_ff, const uint8_t *gate_data,
                       const float *gate_scales, const uint8_t *up_data, const float *up_scales,
                       const uint8_t *down_data, const float *down_scales, int activation, float *out,
                       void *stream);

/* The MLP block of needle_ffn_forward for callers that cannot allocate device
 * memory during a call (a fixed device-memory budget handed over at start-up,
 * latency-critical steps that cannot take an allocator call or an
 * out-of-memory failure, embedders with their own memory manager).  No
 * counterpart in the reference, which has no device memory.  Arguments and
 * results are those of needle_ffn_forward; the difference:
 *   - the [T][d_ff] hidden activation lives in a fixed device array compiled
 *     into the library (1,048,576 floats = 4 MiB, held on every GPU that
 *     loads the library until the process exits); T * d_ff above that is
 *     rejected with an error; nothing is allocated and the matmuls run on the
 *     CUDA cores;
 *   - every call looks up that array's device address on the current
 *     device (cudaGetSymbolAddress); the first call on each device also sets
 *     kernel attributes, so make that first call before any stream capture,
 *     and none after a cudaDeviceReset of that device;
 *   - up to 8 tokens a block holds every token's input row in shared
 *     memory (2 floats per input element of the down projection), which
 *     must fit in 200 KB with the block's buffers, else the call fails and
 *     says so: d_ff up to 2,560 at 5-8 tokens and 5,248 at 3-4, d_model up
 *     to 5,376 at 8 tokens;
 *   - every call shares the one array, which keeps the last call's contents:
 *     calls whose work overlaps on the GPU (different streams, or threads
 *     without ordering) race on it and must be serialised by the caller. */
int needle_ffn_forward_noalloc(const float *x, size_t T, size_t d_model, size_t d_ff, const uint8_t *gate_data,
                               const float *gate_scales, const uint8_t *up_data, const float *up_scales,
                               const uint8_t *down_data, const float *down_scales, int activation, float *out,
                               void *stream);

/* A prepared MLP block for repeated calls (the engine's own form of
 * ffn_forward, crates/needle-core/src/ffn.rs:19-56): gate and up interleaved
 * into one INT4 weight, the tensor-core bf16 hi/lo staging of it and of
 * down, and a workspace for up to max_tokens rows, all allocated here.
 * needle_ffn_plan_forward is asynchronous in `stream` and allocates nothing;
 * from 9 tokens it runs x -> planes, one gate|up GEMM whose epilogue writes
 * act(gate) * up straight as the down GEMM's operand planes, and the down
 * GEMM.  Calls on one plan share its workspace and must be ordered (one
 * stream).  needle_ffn_plan_status synchronises the device and returns -1
 * if a bounded wait inside a tensor-core launch expired since the last
 * check.  Activations as needle_ffn_forward. */
typedef struct NeedleFfnPlan NeedleFfnPlan;
NeedleFfnPlan *needle_ffn_plan_create(size_t d_model, size_t d_ff, const uint8_t *gate_data, const float *gate_scales,
                                      const uint8_t *up_data, const float *up_scales, const uint8_t *down_data,
                                      const float *down_scales, size_t max_tokens, void *stream);
int needle_ffn_plan_forward(NeedleFfnPlan *plan, const float *x, size_t T, int activation, float *out, void *stream);
int needle_ffn_plan_status(NeedleFfnPlan *plan);
void needle_ffn_plan_free(NeedleFfnPlan *plan);

/* ── SafeTensors reader (crates/needle-infer/src/safetensors.rs:43-128) ── */
/* The weight-file reader needle_load uses, on a host buffer: header JSON with
 * a string-valued __metadata__ object, dtypes F32 / BF16 / F16 / I8 and the
 * packed I4.  needle_safetensors_parse returns NULL (error set) for a
 * malformed buffer (SafeTensors::from_bytes); _metadata returns a borrowed
 * string valid until _free, or NULL when the key is absent (get_metadata);
 * _get_f32 converts a tensor to f32 (get_f32), writes min(count, cap) values
 * and returns the count, or (size_t)-1 when the tensor is absent or is an I4
 * tensor whose byte count does not match its shape. */
typedef struct NeedleSafeTensors NeedleSafeTensors;
NeedleSafeTensors *needle_safetensors_parse(const uint8_t *data, size_t len);
const char *needle_safetensors_metadata(const NeedleSafeTensors *st, const char *key);
size_t needle_safetensors_get_f32(const NeedleSafeTensors *st, const char *name, float *out, size_t cap);
void needle_safetensors_free(NeedleSafeTensors *st);

/* Measurement helper (no reference counterpart): the device's streaming-read
 * bandwidth in GB/s, from `iters` timed grid-stride float4 read passes over a
 * fresh `bytes` buffer (allocated and freed here) on the current device's
 * default stream.  Returns 0, or -1 on a CUDA error. */
int needle_hbm_read_gbs(size_t bytes, int iters, double *gbs);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* NEEDLE_B200_H */
