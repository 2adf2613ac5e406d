/*
 * needle_oracle.h — CPU restatement of the needle-rs reference path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA product (libneedle_c.so) and the timed CPU baseline in bench.py.
 * Nothing in the product links, loads or calls it.
 *
 * Every function restates the arithmetic of the reference crate
 * `needle-core` (and the greedy loop of `needle-infer`) in C++, in the
 * same evaluation order, so that on the same inputs it produces the same
 * f32 results as the reference's AVX2 path on x86-64.  Transcendentals come
 * from glibc (the reference uses the `libm` crate 0.2.16, a port of musl);
 * sqrtf/roundf agree bit for bit, expf/powf/sinf/cosf may differ by <= 1 ulp.
 */
#ifndef NEEDLE_ORACLE_H
#define NEEDLE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ── INT4 group quantization (crates/needle-core/src/quant.rs) ───────────── */

/* Sizes of the packed form of a [in_feat, out_feat] f32 matrix. */
void orc_quant_sizes(size_t in_feat, size_t out_feat, size_t *data_bytes,
                     size_t *num_groups);
/* quant.rs:63-128.  data: [(in_pad/2) * out_feat], scales: [num_groups*out_feat]. */
void orc_quantize(const float *w, size_t in_feat, size_t out_feat,
                  uint8_t *data, float *scales);
/* quant.rs:131-155. */
void orc_dequantize(const uint8_t *data, const float *scales, size_t in_feat,
                    size_t out_feat, size_t num_groups, float *out);
/* quant.rs:160-297.  path: 0 = matvec_scalar (:184-206), 1 = matvec_avx2
 * (:209-297).  y is zeroed first, as in matvec (:164-166). */
void orc_matvec(const uint8_t *data, const float *scales, size_t in_feat,
                size_t out_feat, size_t num_groups, const float *x, float *y,
                int path);
/* quant.rs:400-410 — batch independent matvecs. */
void orc_matmul(const uint8_t *data, const float *scales, size_t in_feat,
                size_t out_feat, size_t num_groups, const float *x,
                size_t batch, float *y, int path);
/* quant.rs:413-419. */
int orc_sign_extend4(uint8_t nibble);

/* ── norm / rope / ops ───────────────────────────────────────────────────── */
void orc_zc_rms_norm(float *x, const float *scale, size_t n);   /* norm.rs:23-30 */
void orc_rope_table(size_t max_len, size_t head_dim, float base, float *cos_t,
                    float *sin_t);                                /* rope.rs:20-41 */
void orc_rope_apply(const float *cos_t, const float *sin_t, size_t half_dim,
                    float *x, size_t seq_len, size_t num_heads,
                    size_t head_dim, size_t offset);              /* rope.rs:44-77 */
void orc_softmax(float *x, size_t n);                             /* ops.rs:5-36 */
float orc_sigmoid(float x);                                       /* ops.rs:40-42 */
float orc_gelu(float x);                                          /* ops.rs:47-52 */
/* ffn.rs:19-56 for one token; act: 0 drelu, 1 swiglu, 2 geglu. */
void orc_ffn_forward(const uint8_t *g_data, const float *g_scales,
                     const uint8_t *u_data, const float *u_scales,
                     const uint8_t *d_data, const float *d_scales,
                     size_t d_model, size_t d_ff, const float *x, float *out,
                     int act);

/* ── model (crates/needle-core/src/model.rs) ─────────────────────────────── */

/* Load a SafeTensors weight file (crates/needle-infer/src/safetensors.rs +
 * engine.rs:578-792).  Returns NULL and fills err on failure. */
void *orc_model_load_file(const char *path, char *err, size_t errlen);
void *orc_model_load_bytes(const uint8_t *bytes, size_t len, char *err,
                           size_t errlen);
void orc_model_free(void *model);
/* cfg[0..11] = d_model, num_heads, num_kv_heads, num_layers, num_dec_layers,
 * vocab_size, max_enc_len, max_dec_len, ffn_dim, no_feedforward, activation,
 * head_dim. */
void orc_model_config(const void *model, int64_t *cfg);

/* encode (model.rs:153-192) then teacher-forced decode_step (model.rs:235-265)
 * for each dec_ids[i].  enc_out: [n_enc*d] or NULL; logits: [n_dec*V] or NULL. */
int orc_forward(const void *model, const uint32_t *enc_ids, size_t n_enc,
                const uint32_t *dec_ids, size_t n_dec, float *enc_out,
                float *logits);

/* Greedy generation, the loop of engine.rs:286-322 on token IDs.
 * Start token EOS_ID=1.  mask_bits: NULL or [max_new][ceil(V/64)] u64 words,
 * bit v set = token v allowed (additive 0), clear = additive -1e9.
 * stop_on_eos: 1 = break on EOS as the engine does; 0 = fixed max_new steps.
 * out_ids: [max_new]; margins: NULL or [max_new] (top1-top2 of the masked
 * logits); logits: NULL or [max_new*V] (masked logits).  Returns #tokens. */
size_t orc_generate(const void *model, const uint32_t *enc_ids, size_t n_enc,
                    size_t max_new, const uint64_t *mask_bits, int stop_on_eos,
                    uint32_t *out_ids, float *margins, float *logits);

/* Batch of independent requests (engine.rs:142-144 is a sequential loop;
 * this runs requests on n_threads host threads, one request per thread).
 * ids/offsets: CSR prompts (offsets[n_req+1]).  mask_bits: NULL or
 * [n_req][max_new][ceil(V/64)].  out_ids: [n_req*max_new]; out_lens [n_req];
 * margins: NULL or [n_req*max_new]. */
int orc_run_batch(const void *model, const uint32_t *ids,
                  const uint64_t *offsets, size_t n_req, size_t max_new,
                  const uint64_t *mask_bits, int stop_on_eos, uint32_t *out_ids,
                  uint32_t *out_lens, float *margins, int n_threads, float *tops);

/* KV-cache saturation semantics (attn.rs:53-67): pushes n_push rows into a
 * cache of max_len rows; returns the final len. */
size_t orc_kv_cache_push_count(size_t max_len, size_t n_push);
/* encode_contrastive (engine.rs:153-181): embedding length written to out
 * (0: the model has no contrastive head); no ids -> zero vector. */
size_t orc_encode_contrastive(const void *model, const uint32_t *ids, size_t n, float *out);
size_t orc_contrastive_dim(const void *model);

#ifdef __cplusplus
}
#endif
#endif
