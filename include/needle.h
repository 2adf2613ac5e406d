/*
 * needle.h — C ABI of the needle inference engine, B200 build.
 *
 * Declares the same ten entry points, with the same signatures, ownership and
 * error conventions, as the reference's C ABI (crates/needle-c/include/
 * needle.h:31-181, implemented in crates/needle-c/src/lib.rs:46-356), so a
 * program built against the reference header links against
 * libneedle_c.so unchanged.  The B200 additions live in needle_b200.h.
 *
 * Conventions kept from the reference:
 *   - failures return NULL / false / 0; needle_last_error() then holds a
 *     message (thread-local, borrowed, valid until the next needle_* call on
 *     the same thread — never free it);
 *   - a NULL handle passed to a run / query function returns NULL / 0
 *     without setting an error (lib.rs:81-83);
 *   - strings returned by needle_run / needle_run_stream are owned by the
 *     caller and freed with needle_free_str; handles with needle_free; both
 *     frees accept NULL.
 */
#ifndef NEEDLE_H
#define NEEDLE_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque engine handle (needle.h:32 of the reference). */
typedef struct NeedleHandle NeedleHandle;

/* Per-token streaming callback (needle.h:41-43): raw token id, the token's
 * UTF-8 text, and the caller's pointer passed through unchanged. */
typedef void (*NeedleStreamCallback)(uint32_t token_id, const char *piece, void *user_data);

/* Load weights (.safetensors) and vocabulary (one piece per line, optional
 * "\t<score>") from disk onto the default CUDA device (needle.h:56,
 * lib.rs:46-67).  The device is 0 unless the NEEDLE_DEVICE environment
 * variable names another. */
NeedleHandle *needle_load(const char *weights_path, const char *vocab_path);

/* Same, from in-memory buffers (needle.h:71-72, lib.rs:141-168). */
NeedleHandle *needle_load_bytes(const uint8_t *weights_data, size_t weights_len, const uint8_t *vocab_data,
                                size_t vocab_len);

/* Single-example tool-call generation (needle.h:88, lib.rs:76-105): query
 * text + tools JSON in, JSON tool calls out. */
char *needle_run(NeedleHandle *handle, const char *query, const char *tools_json);

/* As needle_run, calling `callback` for every generated token in order
 * before returning (needle.h:100-104, lib.rs:190-229).  callback may be NULL. */
char *needle_run_stream(NeedleHandle *handle, const char *query, const char *tools_json,
                        NeedleStreamCallback callback, void *user_data);

/* Contrastive retrieval head (needle.h:114-157, lib.rs:243-343).  Models
 * without the contrastive tensors report dimension 0 and return false / 0. */
size_t needle_contrastive_dim(NeedleHandle *handle);
bool needle_encode_contrastive(NeedleHandle *handle, const char *text, float *out, size_t dim);
size_t needle_retrieve_tools(NeedleHandle *handle, const char *query, const char **tool_descs, size_t n_tools,
                             size_t top_k, size_t *out_indices, float *out_scores);

/* Frees (needle.h:165,171; lib.rs:112-127).  NULL is a no-op. */
void needle_free_str(char *s);
void needle_free(NeedleHandle *handle);

/* Last error of the calling thread, or NULL (needle.h:181, lib.rs:349-356). */
const char *needle_last_error(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* NEEDLE_H */
