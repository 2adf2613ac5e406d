// engine.h — device-resident Needle model and the batched greedy engine.
//
// Replaces the model + kernel layers of the reference (crates/needle-core:
// NeedleModel::{new, encode, decode_step}, model.rs:44-265) and the token-ID
// part of NeedleEngine::run_impl / run_batch (crates/needle-infer/src/
// engine.rs:142-144, 226-322).  One DevModel lives on one GPU; a Batch holds
// the per-call device state (prompt IDs, encoder K/V, decoder caches) so
// concurrent calls on one model never share mutable memory.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "kernels.h"
#include "safetensors.h"

namespace ndl {

// crates/needle-core/src/config.rs:22-69 (defaults) and :83-103 (validate)
struct Config {
  int d_model = 512, num_heads = 8, num_kv_heads = 4, num_layers = 12, num_dec_layers = 8;
  int vocab_size = 8192, max_enc_len = 1024, max_dec_len = 512, ffn_dim = 2048;
  bool no_feedforward = true;
  int activation = ACT_DRELU;
  float rope_theta = 10000.0f;
  int head_dim() const { return d_model / num_heads; }
  const char *validate() const;
};

struct Lin {  // packed INT4 weight on the device
  uint8_t *w = nullptr;
  float *s = nullptr;
  int K = 0, N = 0, G = 0, gs = 0;
  // tensor-core staging copy: bf16 hi/lo planes [N][Kp] of q * scale
  void *tc_hi = nullptr, *tc_lo = nullptr;
  bool tc_ready = false;
  TcPlanes tc;
  Int4Weight view() const { return Int4Weight{w, s, K, N, G, gs}; }
};

struct EncLayerDev {
  Lin qkv, o;                     // qkv: wq|wk|wv fused along N
  float *q_norm = nullptr, *k_norm = nullptr, *norm = nullptr;
  float gate = 0.0f;              // sigmoid(self_attn_gate), host-computed
  bool ffn = false;
  Lin gate_up, down;              // gate_up: (gate_i, up_i) interleaved along N
  float *ffn_norm = nullptr;
  float ffn_gate = 0.0f;
};

struct DecLayerDev {
  Lin sa_qkv, sa_o, ca_q, ca_o;
  float *sa_qn = nullptr, *sa_kn = nullptr, *sa_norm = nullptr;
  float *ca_qn = nullptr, *ca_norm = nullptr;
  float sa_gate = 0.0f, ca_gate = 0.0f;
  bool ffn = false;
  Lin gate_up, down;
  float *ffn_norm = nullptr;
  float ffn_gate = 0.0f;
};

struct DevModel {
  int device = 0;
  Config cfg;
  AttnDims ad;
  float embed_scale = 0.0f;
  float *emb = nullptr;        // [V][d] f32
  bool emb_bf16_exact = false;
  // tensor-core staging of the embedding for the batched head: bf16 hi/lo
  // planes [V][Kp] (lo all zero when the embedding is bf16-exact)
  void *emb_hi = nullptr, *emb_lo = nullptr;
  bool emb_tc_ready = false;
  TcPlanes emb_tc;
  std::vector<EncLayerDev> enc;
  std::vector<DecLayerDev> dec;
  Lin cross_kv;                // all decoder layers' cross wk|wv: [d, L*2*KVH*HD]
  float *cross_knorm = nullptr;  // [L][HD]
  float *enc_final_norm = nullptr, *dec_final_norm = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;  // [rope_len][HD/2]
  int rope_len = 0;
  cudaStream_t stream = nullptr;
  std::vector<void *> allocs;
  size_t weight_bytes = 0;
  int *kerr = nullptr;  // device flag: a bounded in-kernel wait expired
  // contrastive head (engine.rs:28-34, 548-573), when the file has it
  int c_hidden = 0, c_dim = 0;
  float *c_hk = nullptr, *c_hb = nullptr, *c_pk = nullptr;  // [d][h], [h], [h][c]

  ~DevModel();
};

// Loads a SafeTensors buffer onto `device` (engine.rs:578-792 semantics:
// config from __metadata__, missing tensors become zeros, F32 projection
// weights are quantized on load by the device packer).
std::unique_ptr<DevModel> load_model(std::vector<uint8_t> raw, int device, std::string &err);

// Kernel classes that can be timed (needle_batch_time_kernel).
enum TimedClass : int {
  TIME_NONE = 0,
  TIME_CROSS_ATTENTION = 1,  // decoder cross-attention (HBM-bound on encoder K/V)
  TIME_PREFILL_MATMUL = 2,   // encoder INT4 projections + cross K/V fill
  TIME_DECODE_MATMUL = 3,    // decoder INT4 projections
  TIME_HEAD = 4,             // output head + mask + argmax
  TIME_ENCODER_ATTENTION = 5,
  TIME_SELF_ATTENTION = 6,   // decoder self-attention with its cache append
  TIME_ELEMENTWISE = 7,      // norms, embedding, q/k post-processing, step bookkeeping
};

enum BatchFlags : uint32_t {
  BATCH_STOP_ON_EOS = 1u,     // engine.rs:306-308: stop a request at EOS
  BATCH_DEVICE_INPUTS = 2u,   // prompt ids / masks are device pointers
  BATCH_NO_GRAPH = 4u,        // launch each decode step eagerly
  BATCH_NO_PDL = 8u,          // no programmatic dependent launch in the decode step
};

struct BatchSpec {
  const uint32_t *ids = nullptr;       // concatenated prompts
  const uint64_t *offsets = nullptr;   // host, [n_req + 1]
  int n_req = 0;
  int max_new = 0;
  const uint64_t *mask = nullptr;      // [n_req][max_new][ceil(V/64)] or NULL
  const uint32_t *teacher = nullptr;   // host [n_req][max_new] teacher-forced decoder inputs, or NULL
  uint32_t flags = 0;
  bool want_logits = false;            // keep masked logits [n_req][max_new][V]
  bool want_enc_out = false;           // keep the final encoder hidden [sum T][d]
};

// Per-call device state; prepare() uploads inputs and allocates, run()
// executes prefill + max_new decode steps, download() copies results out.
class Batch {
 public:
  explicit Batch(DevModel *m);
  ~Batch();
  bool prepare(const BatchSpec &spec, std::string &err);
  // run() = begin() + every decode step (with an early exit once all
  // requests hit EOS under BATCH_STOP_ON_EOS).  Work is left enqueued on
  // stream(); download() synchronises.  A batch may run again: each run
  // starts from the uploaded prompts with a fresh decoder state.
  bool run(std::string &err);
  // Stepwise use (streaming): begin() runs the prefill, step() enqueues one
  // decode step, peek() synchronises and copies lens/done/tokens to the host.
  bool begin(std::string &err);
  bool step(std::string &err);
  bool peek(uint32_t *lens, uint8_t *done, uint32_t *ids, std::string &err);
  // Overwrite the vocabulary bitmap a request uses at one decode step
  // (ceil(V/64) words, host memory), ordered before later steps on the
  // batch's stream.  The batch must have been prepared with a mask.
  bool set_mask_row(int req, int step, const uint64_t *bits, std::string &err);
  // The same for every request at once: rows [n_req][ceil(V/64)] (one
  // strided copy).
  bool set_mask_step(int step, const uint64_t *rows, std::string &err);
  // Synchronise and read one step's tokens [n_req] plus lens / done.
  bool peek_step(int step, uint32_t *tokens, uint32_t *lens, uint8_t *done, std::string &err);
  bool download(uint32_t *out_ids, uint32_t *out_lens, float *logits, float *enc_out, std::string &err);
  cudaStream_t stream() const { return st_; }
  // Encoder output rows [ttot][d] (prepared with want_enc_out) and the
  // requests' row offsets [n_req + 1], on the device.
  const float *enc_out_dev() const { return enc_out_; }
  const int64_t *seq_off_dev() const { return seq_off_; }
  // Number of kernels one run() launches (reported by the benchmark).
  int64_t kernels_launched() const { return launches_; }
  // Optional timing of one kernel class: CUDA events around each of its
  // launches on the batch's stream (eager launches while enabled), plus the
  // algorithmic flops and bytes of every timed launch.
  void set_timed_class(int cls) { timed_cls_ = cls; }
  bool collect_timing(std::string &err);
  double timed_ms() const { return timed_ms_; }
  int64_t timed_launches() const { return timed_n_; }
  double timed_flops() const { return timed_flops_; }
  double timed_bytes() const { return timed_bytes_; }

 private:
  bool prefill(std::string &err);
  bool reset_decoder(std::string &err);
  // One decode step.  att_rows: no request attends over more self-attention
  // rows in this step (sizes the self-attention kernel's pass).
  bool decode_step(std::string &err, bool capture, int att_rows);
  // Self-attention row bound of decode step `step` and its graph slot: every
  // request is at most at position `step`, so it attends over at most
  // min(step + 1, cap) rows; the bound is rounded up to 16, 32 or cap.
  int att_rows(int step) const {
    const int r = step + 1 < cap_ ? step + 1 : cap_;
    return r <= 16 ? 16 : r <= 32 ? 32 : cap_;
  }
  static int att_slot(int rows) { return rows <= 16 ? 0 : rows <= 32 ? 1 : 2; }
  bool mm(int cls, bool capture, const float *x, int64_t ldx, int M, const Lin &w, const MatmulOut &o,
          std::string &err);
  bool mm_in(int cls, bool capture, const TcPlanes *planes, const float *x, int64_t ldx, int M, const Lin &w,
             const MatmulOut &o, std::string &err);
  const TcPlanes *tc_map(int Kp, int rows) const;
  template <class T>
  T *alloc(size_t n, std::string &err);

  DevModel *m_;
  cudaStream_t st_ = nullptr;  // each call has its own stream: calls on one model run concurrently
  BatchSpec spec_{};
  std::vector<uint64_t> off_h_;
  int64_t ttot_ = 0;
  int tmax_ = 0, cap_ = 0, W_ = 0;
  std::vector<void *> bufs_;
  // inputs
  uint32_t *ids_ = nullptr;
  int64_t *seq_off_ = nullptr;     // [n_req+1] absolute token offsets
  int32_t *tok_pos_ = nullptr;     // [ttot] position inside its request
  uint64_t *mask_ = nullptr;
  uint32_t *teacher_ = nullptr;
  // prefill chunks
  struct Chunk {
    int r0, r1;
    int64_t tok0, ntok;
    int tmax;
    int64_t *rel_off;  // device [r1-r0+1], chunk-relative offsets
    void *items;       // device int4 work items of the tensor-core encoder attention
    int n_items;
  };
  std::vector<Chunk> chunks_;
  int64_t chunk_tok_max_ = 0;
  float *px_ = nullptr, *pxn_ = nullptr, *pqkv_ = nullptr, *patt_ = nullptr, *pffn_ = nullptr;
  // encoder outputs
  // encoder K/V of the decoder layers (K0 V0 K1 V1 ...): head-major
  // [2L][KVH][ttot][64] when kv_map_ok_ (head dim 64, two query heads per KV
  // head: each head's rows are one contiguous stream for the cross-attention
  // kernel's tile loads), else [2L][ttot][KVH*HD]
  float *kv_planes_ = nullptr;
  alignas(64) unsigned char kv_map_[128] = {};  // TMA descriptor of the head-major planes (64 x 64 boxes)
  bool kv_map_ok_ = false;
  float *enc_out_ = nullptr;       // [ttot][d] when requested
  // decoder state
  float *self_k_ = nullptr, *self_v_ = nullptr;  // [L][B][cap][KVH*HD]
  float *x_ = nullptr, *xn_ = nullptr, *qkv_ = nullptr, *att_ = nullptr, *q_ = nullptr, *h_ = nullptr, *ffn_ = nullptr;
  // tensor-core encoder attention planes (per prefill chunk)
  bool tc_attn_ = false;
  AttnPlanes attn_planes_;
  // tensor-core activation staging (bf16 hi/lo planes) and its TMA maps
  void *tc_hi_ = nullptr, *tc_lo_ = nullptr;
  float *splitk_ws_ = nullptr;  // partial tiles of the split-K GEMMs (ordered on st_)
  std::vector<TcPlanes> tc_maps_;  // one per distinct padded K
  unsigned long long *keys_ = nullptr;
  int32_t *pos_ = nullptr;
  uint32_t *out_ids_ = nullptr, *lens_ = nullptr;
  uint8_t *done_ = nullptr;
  unsigned int *n_done_ = nullptr;
  float *logits_ = nullptr;
  cudaGraphExec_t graphs_[3] = {nullptr, nullptr, nullptr};  // decode step, by att_slot
  // host mask bitmaps are uploaded on cst_ (they are first read by the first
  // decode step, so the copy overlaps the prefill); mask_ev_ marks its end
  cudaStream_t cst_ = nullptr;
  cudaEvent_t mask_ev_ = nullptr;
  bool mask_async_ = false;
  bool use_graph_ = false;
  uint32_t *first_ids_ = nullptr;
  int steps_done_ = 0;
  int64_t launches_ = 0, step_launches_ = 0;
  int timed_cls_ = 0;
  double timed_ms_ = 0.0, timed_flops_ = 0.0, timed_bytes_ = 0.0;
  int64_t timed_n_ = 0;
  struct TimedLaunch {
    cudaEvent_t a, b;
    double flops, bytes;
  };
  std::vector<TimedLaunch> timed_;
  bool tbegin(int cls, bool capture, cudaEvent_t &a, std::string &err);
  bool tend(cudaEvent_t a, double flops, double bytes, std::string &err);
};

// Splits n requests with lengths len[] into `shards` groups of near-equal
// cost (cost ~ T^2 attention + T projections + decode), longest-first
// greedy (LPT).  assignment[i] = shard of request i.
void shard_requests(const uint64_t *offsets, int n_req, int shards, int32_t *assignment);

}  // namespace ndl
