// kernels.h — host-side launchers of the needle sm_100a kernels.
//
// All pointers are device pointers.  Every launcher enqueues on `stream` and
// returns the launch status (cudaSuccess or the error cudaGetLastError saw).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ndl {

constexpr uint32_t kEosId = 1;  // tokenizer.rs:23 EOS_ID, also the decoder start token

struct AttnDims {
  int H = 8, KVH = 4, HD = 64;
  float scale = 0.125f;  // powf(hd, -0.5) computed on the host (attn.rs:142)
};

// Packed INT4 weight in the reference layout (quant.rs:45-58):
//   w[pair * N + n]: low nibble = row 2*pair, high nibble = row 2*pair+1
//   s[g * N + n]:    f32 scale of group g = row / gs, gs = min(32, K)
struct Int4Weight {
  const uint8_t *w = nullptr;
  const float *s = nullptr;
  int K = 0;   // in_feat (unpadded)
  int N = 0;   // out_feat (of the logical matrix; 2x each part in paired mode)
  int G = 0;   // num_groups
  int gs = 0;  // group size = min(32, K)
  // Paired mode (w2 != NULL): the logical weight interleaves the columns of
  // two same-shape weights, column 2i = w column i, 2i+1 = w2 column i
  // (gate / up of ffn.rs:19-56, each [K][N/2] in the reference layout).
  const uint8_t *w2 = nullptr;
  const float *s2 = nullptr;
};

enum Epilogue : int {
  EPI_STORE = 0,  // y = acc
  EPI_RESID = 1,  // y += gate * acc           (layers.rs:70-74 gated residual)
  EPI_ACT = 2,    // columns interleaved (gate_i, up_i) -> y[i] = act(gate_i, up_i); on the
                  // tensor-core path with planes[0] set, written instead as the
                  // bf16 hi/lo planes planes[0] / planes[1] (row stride ldy)
  EPI_KNORM = 3,  // y = acc, then per-64-column ZCRMSNorm with `vec` on blocks
                  // whose column-block index is even (the K half of K|V pairs)
  EPI_ARGMAX = 4, // output head: acc = logit of (row m, vocab n); add the mask,
                  // reduce to atomicMax(keys[m], (total-order key, n)); logits
                  // optionally stored (engine.rs:294-304)
  EPI_QKV = 5,    // fused Q|K|V projection of the encoder: per 64-column head,
                  // ZCRMSNorm + RoPE (Q, K) then bf16 hi/lo into the attention
                  // planes (tensor-core path only)
  EPI_QKV_DEC = 6,  // fused Q|K|V projection of one decoder step: per 64-column
                    // head, ZCRMSNorm + RoPE at position pos[m] (Q, K); Q f32 to
                    // y, K and V appended to the self-attention caches at row
                    // pos[m] when pos[m] < cache_cap (attn.rs:100-140, push_kv
                    // saturating as attn.rs:53-61; tensor-core path only)
};

enum Activation : int { ACT_DRELU = 0, ACT_SWIGLU = 1, ACT_GELU = 2 };

struct MatmulOut {
  float *y = nullptr;
  int64_t ldy = 0;           // row stride of y (floats)
  int col_block = 0;         // 0: plain; else columns are split into blocks of
  int64_t block_stride = 0;  //   col_block, block b written at y + b*block_stride
  int epi = EPI_STORE;
  // EPI_KNORM: width of each K or V block of the K|V pairs (0: col_block);
  // column n belongs to pair (n / kv_block) / 2, normed when that quotient is
  // even.  Lets col_block be narrower (one head) than a K or V block.
  int kv_block = 0;
  float gate = 0.0f;
  int act = ACT_DRELU;
  const float *vec = nullptr;  // EPI_KNORM: k_norm scale [64]
  // EPI_ARGMAX: request m is at step pos[m]; mask row (or NULL) at
  // mask + (m*max_new + pos[m]) * mask_words; logits (or NULL) at
  // logits + (m*max_new + pos[m]) * N.
  const uint64_t *mask = nullptr;
  int mask_words = 0, max_new = 0;
  const int32_t *pos = nullptr;
  unsigned long long *keys = nullptr;
  float *logits = nullptr;
  // EPI_QKV: row m has position pos[m] (rope tables [pos][32]); planes as in
  // AttnPlanes: Q [H][slab][64], K and V [KVH][slab][64], hi/lo each.
  const float *q_norm = nullptr, *k_norm = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
  void *planes[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  int slab = 0, heads_q = 0, heads_kv = 0;
  // EPI_QKV_DEC: caches [M][cache_cap][heads_kv*64] f32
  float *kcache = nullptr, *vcache = nullptr;
  int cache_cap = 0;
  // Tensor-core path: workspace of tc_splitk_ws_bytes() for the split-K
  // kernel's partial tiles, or NULL (no split).  Launches that share one
  // workspace must be ordered (one stream).
  float *splitk_ws = nullptr;
  // CUDA-core matvec only (int4_matmul_norms_input): each row of x is first
  // ZCRMSNorm'ed with this scale vector over its K columns (norm.rs:23-30:
  // ((1 + s) * x) / sqrt(mean(x^2) + 1e-6)), as the kernel loads it.
  const float *in_norm = nullptr;
};

// Y[M, N] (epilogue) X[M, K] @ W.  x row stride ldx (floats).
cudaError_t int4_matmul(const float *x, int64_t ldx, int M, const Int4Weight &W, const MatmulOut &o,
                        cudaStream_t stream, bool pdl = false);
// Whether int4_matmul takes MatmulOut::in_norm for these arguments (the
// CUDA-core matvec, up to 8 rows); elsewhere it refuses it.
bool int4_matmul_norms_input(int M, const Int4Weight &W, const MatmulOut &o);
// Dynamic shared memory (bytes) int4_matmul requests for these arguments;
// above kMaxDynSmem it refuses the call (cudaErrorInvalidValue).  Up to 8
// rows it holds x: M * (K rounded up to the group) floats and more.
size_t int4_matmul_smem(int M, const Int4Weight &W, const MatmulOut &o);

// ── tensor-core path (tc_gemm.cu) ──
// A pair of bf16 planes (hi, lo) of a [rows][Kp] K-contiguous operand, with
// the TMA descriptors the tcgen05 GEMM loads it through (boxes of 64 x
// box_rows, 128-byte swizzle).  Kp is a multiple of 64.
struct TcPlanes {
  alignas(64) unsigned char hi[128];  // CUtensorMap
  alignas(64) unsigned char lo[128];
  // the same planes in boxes of 64 x 64 (B operands of 64-column tiles)
  alignas(64) unsigned char hi64[128];
  alignas(64) unsigned char lo64[128];
  int rows = 0, Kp = 0, box_rows = 0;
  const void *hi_ptr = nullptr, *lo_ptr = nullptr;
};
constexpr int kTcMinRows = 128;  // batched GEMMs at least this tall use the tensor cores
int tc_padded_k(int K);
cudaError_t tc_make_planes(const void *hi, const void *lo, int rows, int Kp, int box_rows, TcPlanes &out);
// TMA descriptor (128-byte CUtensorMap written to `map`) of a row-major f32
// matrix [rows][cols] loaded in boxes of box_rows x box_cols, no swizzle,
// rows past the end read as zeros.
cudaError_t tma_map_f32(const void *base, int64_t rows, int cols, int box_rows, int box_cols, void *map);
// W (reference INT4 layout, paired mode allowed) -> bf16 planes [N][Kp].
cudaError_t tc_prep_weight(const Int4Weight &W, int Kp, void *hi, void *lo, cudaStream_t st);
// f32 rows [M][K] -> bf16 planes [M][Kp] (zero padded past K).
cudaError_t tc_split_rows(const float *x, int64_t ldx, int M, int K, int Kp, void *hi, void *lo, cudaStream_t st);
// Y[M, N] (epilogue) A @ B^T with A planes [M][Kp] and B planes [N][Kp]
// (tcgen05, 3-term bf16 split, f32 accumulation).  *err is set if a bounded
// wait inside the kernel expired.
// b_lo_zero: B's lo plane is all zero (a bf16-exact operand such as the
// embedding): the hi*lo product is skipped and the lo plane is not loaded.
cudaError_t tc_matmul(const TcPlanes &A, int M, const TcPlanes &B, int N, const MatmulOut &o, int *err,
                      cudaStream_t st, bool b_lo_zero = false);
cudaError_t init_tc_kernels();
// Bytes of the split-K workspace for the current device (one 128 x 128 f32
// partial tile per SM).
size_t tc_splitk_ws_bytes();

// ContrastiveHead::encode (engine.rs:37-69) after the mean pool of
// encode_contrastive (engine.rs:163-179), one CTA per request: out[r][c] from
// the encoder rows [off[r], off[r+1]) of enc [.][d], in the reference's
// sequential f32 order (no fused multiply-add).
cudaError_t contrastive_embed(const float *enc, const int64_t *off, int n_req, int d, const float *hk,
                              const float *hb, int h, const float *pk, int c, float *out, cudaStream_t st);

// ── tensor-core encoder attention (tc_attn.cu) ──
// Per-head bf16 hi/lo planes of the normed + RoPE'd Q, K and the V of one
// prefill chunk: Q [H][slab][64], K and V [KVH][slab][64] (buf: qh ql kh kl
// vh vl), with their TMA maps.
struct AttnPlanes {
  void *buf[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  int slab = 0;
  TcPlanes q, k, v;
};
cudaError_t attn_planes_make(void *const bufs[6], int H, int KVH, int slab, AttnPlanes &p);
// ZCRMSNorm + RoPE (positions pos[row]) of the Q and K heads of fused QKV
// rows, then the bf16 hi/lo split of Q, K and V into the planes.  HD = 64.
cudaError_t qkv_post(const float *qkv, int rows, const int32_t *pos, const float *q_norm, const float *k_norm,
                     const float *rope_cos, const float *rope_sin, AttnDims a, const AttnPlanes &p, cudaStream_t st);
// Bidirectional attention over the planes: items = int4 (request, 128-row
// query tile, Q head, 0) against chunk-relative seq_off.  The result goes to
// bf16 hi/lo planes [rows][ldp] (the O projection's input) when out_hi is
// set (out_rows rows; warps whose 32 rows lie inside one request write
// through TMA boxes), else to f32 out [rows][H*64].
cudaError_t encoder_attention_tc(const AttnPlanes &p, const int64_t *seq_off, const void *items, int n_items,
                                 float *out, void *out_hi, void *out_lo, int ldp, int out_rows, AttnDims a, int *err,
                                 cudaStream_t st);
// NEEDLE_NO_TMA_STORE=1 in the environment: every epilogue stores per thread.
bool tma_store_disabled();
cudaError_t init_tc_attn_kernels();

// Device packing / unpacking (quant.rs:63-155), bit-exact with the reference.
cudaError_t int4_quantize(const float *w, int K, int N, uint8_t *data, float *scales, cudaStream_t st);
cudaError_t int4_dequantize(const uint8_t *data, const float *scales, int K, int N, int G, float *out,
                            cudaStream_t st);

// out[r, :] = ZCRMSNorm(x[r, :], scale)   (norm.rs:23-30), d = row length.
cudaError_t rms_norm_rows(const float *x, int64_t ldx, float *out, int64_t ldo, const float *scale, int rows,
                          int d, cudaStream_t st);

// The same norm for d = 512 written as bf16 hi/lo planes (row stride ldp) for
// the tensor-core GEMM, and also as f32 to `out` when it is not NULL.
cudaError_t rms_norm_planes(const float *x, int64_t ldx, void *hi, void *lo, int64_t ldp, float *out, int64_t ldo,
                            const float *scale, int rows, int d, cudaStream_t st);

// x[t, :] = E[ids[t], :] * embed_scale  (model.rs:78-85, 158-164)
cudaError_t embed_rows(const uint32_t *ids, const float *emb, float *x, int rows, int d, float embed_scale,
                       cudaStream_t st);



// Largest dynamic shared memory any kernel here is allowed to request.
constexpr int kMaxDynSmem = 200 * 1024;

// Launches of the decode-step kernels (norm, tensor-core matmul, decoder
// attention, finish_step) made by this host thread use programmatic dependent
// launch while on: each such kernel lets its successor's CTAs start during its
// own tail and waits for its predecessor before touching global memory.
void set_pdl(bool on);
// Whether launches from this host thread use programmatic dependent launch.
bool pdl_on();

// Set per-device kernel attributes.  Call once per device, with it current.
cudaError_t init_kernels();
cudaError_t init_matmul_kernels();
cudaError_t init_attention_kernels();
cudaError_t init_head_kernels();

// Encoder prefill: in-place per-head ZCRMSNorm + RoPE (offset 0) on the
// Q|K|V rows produced by the fused projection: row t has Q [H*HD], K [KVH*HD],
// V [KVH*HD].  pos[t] = position of token t inside its request.
cudaError_t qk_norm_rope_rows(float *qkv, int rows, const int32_t *pos, const float *q_norm, const float *k_norm,
                              const float *rope_cos, const float *rope_sin, AttnDims a, cudaStream_t st);

// Bidirectional encoder attention over ragged requests (attn.rs:189-273).
// qkv rows as above; seq_off[r]..seq_off[r+1] = tokens of request r.
// out[t, H*HD].  max_len = the longest request.
cudaError_t encoder_attention(const float *qkv, const int64_t *seq_off, int n_req, int max_len, float *out,
                              AttnDims a, cudaStream_t st);

// Decoder self-attention for one new token per request (attn.rs:100-183):
// q|k|v from qkv rows [B, (H+2*KVH)*HD]; ZCRMSNorm + RoPE at position
// step[b], append k, v to the caches (saturating at cap), attend over the
// cache.  kc/vc: [B, cap, KVH*HD].  out: [B, H*HD] f32, or, when hi is set
// (head dim 64, two query heads per KV head), the bf16 hi/lo operand planes
// of the next tensor-core matmul, row stride ldp elements.  `prepared`
// (same head layout): the QKV projection ran with EPI_QKV_DEC, so q in qkv is
// already normed and rotated and k, v are already in the caches.
// max_rows > 0: no request attends over more rows than that (step[b] + 1 <=
// max_rows); it sizes the kernel's pass.
cudaError_t decoder_self_attention(const float *qkv, const int32_t *step, const float *q_norm,
                                   const float *k_norm, const float *rope_cos, const float *rope_sin, float *kc,
                                   float *vc, int cap, int B, float *out, AttnDims a, cudaStream_t st,
                                   void *hi = nullptr, void *lo = nullptr, int64_t ldp = 0, bool prepared = false,
                                   int max_rows = 0);

// Decoder cross-attention (attn.rs:281-337): q [B, H*HD] (q_norm applied
// here), K/V of request b at rows seq_off[b].. of kplane / vplane
// [*, KVH*HD].  out: [B, H*HD] f32, or the bf16 hi/lo planes as for
// decoder_self_attention.  The head-dim-64 kernel (two query heads per KV
// head) needs err (device flag set when a bounded wait gives up) and kv_map:
// a tma_map_f32 descriptor of head-major K/V planes ([*][64], 64 x 64
// boxes), in which request b's K rows of KV head g start at row k_row0 +
// g * head_rows + seq_off[b] and its V rows at v_row0 + g * head_rows +
// seq_off[b] (kplane / vplane are then not read).
cudaError_t decoder_cross_attention(const float *q, const float *q_norm, const float *kplane,
                                    const float *vplane, const int64_t *seq_off, int B, float *out, AttnDims a,
                                    cudaStream_t st, int max_len, void *hi = nullptr, void *lo = nullptr,
                                    int64_t ldp = 0, int *err = nullptr, const void *kv_map = nullptr,
                                    int64_t k_row0 = 0, int64_t v_row0 = 0, int64_t head_rows = 0);

// Output head (model.rs:89-149) + additive mask (engine.rs:294-297) + argmax
// (engine.rs:299-304), fused.  h: [B, d]; emb: [V, d].  Request b is at step
// pos[b]; its mask bitmap (bit v set = allowed) is mask[(b*max_new +
// pos[b]) * mask_words ...] (NULL = unconstrained) and its masked logits, when
// `logits` is set, go to logits[(b*max_new + pos[b]) * V ...].  keys[b] must
// be zero on entry and receives the packed (logit key, index) maximum.
cudaError_t head_argmax(const float *h, int B, const float *emb, int V, int d, const uint64_t *mask, int mask_words,
                        float *logits, int max_new, const int32_t *pos, unsigned long long *keys, cudaStream_t st,
                        const void *emb_bf16 = nullptr, int64_t ld_bf16 = 0);
// emb_bf16 (optional): the embedding as bf16 rows of stride ld_bf16, equal
// to emb value for value (a bf16-exact embedding); small batches then read
// it instead of the f32 copy.

// After head_argmax, for request b at step s = pos[b]: next = index of
// keys[b]; unless the request is done, append next to out_ids[b*max_new +
// lens[b]] (or, with stop_on_eos and next == EOS, mark it done and count it
// in n_done); clear keys[b]; pos[b] = s + 1; and embed the decoder input of
// step s+1 into x: next, or teacher[b*max_new + s + 1] when teacher is set
// (teacher forcing for parity checks).
cudaError_t finish_step(unsigned long long *keys, int B, int max_new, int stop_on_eos, uint32_t *out_ids,
                        uint32_t *lens, uint8_t *done, int32_t *pos, unsigned int *n_done, const uint32_t *teacher,
                        const float *emb, float *x, int d, float embed_scale, cudaStream_t st);

// Per-head ZCRMSNorm (no RoPE) of `heads` consecutive HD-wide heads in each of
// `rows` rows of stride ld (the cross-attention k_norm of fill_cross_kv,
// model.rs:211-219, for head dims the fused matmul epilogue does not cover).
cudaError_t head_norm_rows(float *x, int rows, int64_t ld, int heads, int HD, const float *scale, cudaStream_t st);

}  // namespace ndl
