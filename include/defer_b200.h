/*
 * defer_b200 — C ABI of the B200 backend for convo-lang/defer's token loop.
 *
 * Every entry point replaces one item of the reference crate's public Rust
 * API (paths below are relative to the reference project root) and keeps
 * its meaning and error behaviour. Plain pointers and sizes only; no
 * framework types. Handles belong to one CUDA device; calls on one handle
 * must be serialised by the caller; different devices may be driven from
 * different host threads.
 *
 * Status codes mirror DeferError (src/error.rs:5-14):
 *   0 ok, 1 Io, 2 Parse, 3 Model, 4 Checkpoint, 5 Wal, 6 Tokenizer,
 *   7 Divergence, plus 8 Cuda, 9 DeviceTimeout, 10 InvalidArgument.
 * On a non-zero status defer_last_error() returns the message (per thread).
 */
#ifndef DEFER_B200_H
#define DEFER_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DEFER_API __attribute__((visibility("default")))
#else
#define DEFER_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct defer_model defer_model;
typedef struct defer_cache defer_cache;
typedef struct defer_session defer_session;
typedef struct defer_wal_writer defer_wal_writer;

/* Model::Config (src/model.rs:24-39) plus device facts. */
typedef struct {
  uint32_t vocab_size, hidden_size, intermediate_size, num_layers;
  uint32_t num_heads, num_kv_heads, head_dim, max_seq_len;
  float rms_norm_eps, rope_theta;
  int32_t tie_word_embeddings, gelu, has_bias, weights_bf16;
  int64_t bos_token_id; /* -1 when absent */
  uint64_t weight_bytes; /* bytes one token step streams from HBM */
  int32_t device, sm_count;
} defer_config;

/* Message of the last failed call on this thread (src/error.rs:16-27). */
DEFER_API const char* defer_last_error(void);

/* ------------------------------------------------------------- model ---- */
/* Model::load (src/model.rs:286-299): parses the safetensors file, hashes
 * every byte (the signature), uploads the weights to `device`. */
DEFER_API int defer_model_load(const char* path, int device, defer_model** out);
DEFER_API void defer_model_free(defer_model* m);
DEFER_API int defer_model_config(const defer_model* m, defer_config* out);
/* Model::signature (src/model.rs:273-274). */
DEFER_API int defer_model_signature(const defer_model* m, uint8_t out[32]);
/* Config::eos_token_ids (src/model.rs:85-89). */
DEFER_API int defer_model_eos_tokens(const defer_model* m, uint32_t* out, size_t cap, size_t* n);
/* Model::forward / forward_ext (src/model.rs:376-520): one token at
 * position defer_cache_len(c); `masked` positions (< len) are hidden from the
 * query; logits (vocab_size floats) are copied to `logits_out` unless NULL.
 * Tracing (forward_traced) is not offered by this backend. */
DEFER_API int defer_forward(defer_model* m, defer_cache* c, uint32_t token, const size_t* masked, size_t n_masked,
                            float* logits_out);

/* Allocation-free forward step. No counterpart in the reference: it exists
 * for callers that cannot allocate device memory while they run — e.g. a
 * server whose memory pool already holds all free HBM, or a latency-bound
 * loop that must not enter the driver's allocator — and therefore cannot
 * use defer_forward, whose first call on a model allocates its scratch.
 * Same arithmetic and result as defer_forward on a cache of `cap`
 * positions, with the caller's buffers: k_cache and v_cache each hold
 * num_layers * num_kv_heads * cap * head_dim floats laid out
 * [layer][kv_head][position][dim], positions < pos filled by earlier calls;
 * position `pos` is written; logits_out receives vocab_size floats. All
 * three are device pointers. `stream` is a cudaStream_t (NULL = legacy
 * default stream); the call returns after the step has finished.
 * Limits: the step's scratch lives in one 4 MiB array inside this library
 * (held by every GPU that loads it until the process exits); a model/cap
 * whose scratch would exceed it is rejected with InvalidArgument. The first
 * call on a device is its set-up: it looks up that array's device address
 * and loads this step's device code (CUDA loads code lazily, and loading it
 * takes device memory), so make that first call before a memory pool
 * reserves the free HBM and before any stream capture; later calls
 * allocate nothing. The address is kept for the life of the process: after
 * a cudaDeviceReset of that device do not call this entry point again.
 * All calls share the array and each call reinitialises it, so calls must
 * not overlap on the GPU (different streams or threads racing each other
 * corrupt each other's scratch). */
DEFER_API int defer_forward_noalloc(defer_model* m, float* k_cache, float* v_cache, uint32_t cap, uint32_t pos,
                                    uint32_t token, float* logits_out, void* stream);

/* ------------------------------------------------------------- cache ---- */
/* Model::new_cache / KvCache (src/model.rs:184-243, 370-372). `cap` = 0
 * means max_position_embeddings positions. */
DEFER_API int defer_cache_new(defer_model* m, uint32_t cap, defer_cache** out);
DEFER_API void defer_cache_free(defer_cache* c);
DEFER_API size_t defer_cache_len(const defer_cache* c);
/* KvCache::truncate (src/model.rs:211-220). */
DEFER_API int defer_cache_truncate(defer_cache* c, size_t n);
/* KvCache::clone (derive, src/model.rs:184). */
DEFER_API int defer_cache_clone(const defer_cache* c, defer_cache** out);
/* KvCache::keys[layer] / values[layer] (src/model.rs:186-188) in the
 * reference layout [len, kv_dim]; each buffer holds len * kv_dim floats. */
DEFER_API int defer_cache_download(const defer_cache* c, uint32_t layer, float* keys, float* values);
/* KvCache::fingerprint (src/model.rs:233-242). */
DEFER_API int defer_cache_fingerprint(const defer_cache* c, uint8_t out[32]);
/* KvCache::bit_eq (src/model.rs:223-230). */
DEFER_API int defer_cache_bit_eq(const defer_cache* a, const defer_cache* b, int* equal);

/* --------------------------------------------------------- sampler/PRNG -- */
/* engine::seed_from_u64 (src/engine.rs:19-21). */
DEFER_API void defer_seed_from_u64(uint64_t seed, uint8_t out[32]);
/* ChaCha8Rng words [start, start + n) of the stream keyed by `seed`
 * (the words sampler.rs:92 draws, one per sampled token). */
DEFER_API int defer_chacha8_words(const uint8_t seed[32], uint64_t start, size_t n, uint32_t* out);
/* sampler::words_per_sample (src/sampler.rs:15-21). */
DEFER_API uint64_t defer_words_per_sample(float temperature);
/* sampler::sample_token (src/sampler.rs:78-109) run by the device sampler
 * on host logits, with the PRNG word already drawn (ignored when T == 0).
 * `margin` (nullable) receives the distance of r to the nearest CDF edge. */
DEFER_API int defer_sample_logits(int device, const float* logits, size_t n, float temperature, uint32_t word,
                                  uint32_t* token, float* margin);

/* ----------------------------------------------------------- session ---- */
/* Session::new (src/engine.rs:44-60). */
DEFER_API int defer_session_new(defer_model* m, const uint8_t seed[32], float temperature, defer_session** out);
DEFER_API void defer_session_free(defer_session* s);
/* Session::prompt (src/engine.rs:62-71). */
DEFER_API int defer_session_prompt(defer_session* s, const uint32_t* tokens, size_t n);
/* Session::step (src/engine.rs:113-117). */
DEFER_API int defer_session_step(defer_session* s, uint32_t* token);
/* Called after each generated token with the PRNG word position after it;
 * a non-zero return stops generation and is returned as the status. */
typedef int (*defer_token_cb)(void* user, uint32_t token, uint64_t rng_word_pos);
/* Session::generate (src/engine.rs:121-137). out_tokens holds max_tokens. */
DEFER_API int defer_session_generate(defer_session* s, size_t max_tokens, const uint32_t* stop, size_t n_stop,
                                     defer_token_cb cb, void* user, uint32_t* out_tokens, size_t* n_out);
/* Session::checkout (src/engine.rs:241-274) from checkpoint bytes. */
DEFER_API int defer_session_checkout(defer_model* m, const uint8_t* ckpt, size_t len, defer_session** out);
/* Session::checkpoint (src/engine.rs:223-232) as checkpoint bytes; with
 * buf == NULL only *len is set. */
DEFER_API int defer_session_checkpoint(const defer_session* s, uint8_t* buf, size_t cap, size_t* len);
/* Session::history / prompt_len / rng_word_pos / last_logits / cache
 * (src/engine.rs:194-221). The cache handle is borrowed. */
DEFER_API int defer_session_history(const defer_session* s, uint32_t* out, size_t cap, size_t* n);
DEFER_API size_t defer_session_prompt_len(const defer_session* s);
DEFER_API uint64_t defer_session_rng_word_pos(const defer_session* s);
DEFER_API int defer_session_last_logits(const defer_session* s, float* out);
DEFER_API defer_cache* defer_session_cache(defer_session* s);
/* Sampler margins of the last generate / checkout (diagnostics). */
DEFER_API int defer_session_margins(const defer_session* s, float* out, size_t cap, size_t* n);

/* ---------------------------------------------- checkpoint / WAL formats -- */
/* DeferCheckpoint (src/checkpoint.rs:26-108) as fields <-> bytes. */
typedef struct {
  uint8_t model_signature[32];
  uint8_t base_seed[32];
  float temperature;
  uint32_t prompt_len;
  uint64_t rng_word_pos_lo, rng_word_pos_hi;
  const uint32_t* history_tokens;
  size_t n_tokens;
} defer_checkpoint_fields;
DEFER_API int defer_checkpoint_encode(const defer_checkpoint_fields* f, uint8_t* buf, size_t cap, size_t* len);
/* Decodes and verifies (magic, version, CRC, lengths); the token pointer
 * refers into `tokens_out` (capacity `tokens_cap`). */
DEFER_API int defer_checkpoint_decode(const uint8_t* b, size_t len, defer_checkpoint_fields* f, uint32_t* tokens_out,
                                      size_t tokens_cap);
/* DeferCheckpoint::save / load (src/checkpoint.rs:92-108). */
DEFER_API int defer_checkpoint_save(const uint8_t* bytes, size_t len, const char* path);
DEFER_API int defer_checkpoint_load(const char* path, uint8_t* buf, size_t cap, size_t* len);

/* WalHeader (src/wal.rs:45-84). */
typedef struct {
  uint8_t model_signature[32];
  uint8_t base_seed[32];
  float temperature;
  uint32_t prompt_len;
  uint64_t start_rng_word_pos_lo, start_rng_word_pos_hi;
  const uint32_t* prefix_tokens;
  size_t n_prefix;
} defer_wal_header;
/* WalWriter::create / resume / append (src/wal.rs:221-250). */
DEFER_API int defer_wal_create(const char* path, const defer_wal_header* h, int durable, defer_wal_writer** out);
DEFER_API int defer_wal_resume(const char* path, int durable, defer_wal_writer** out);
DEFER_API int defer_wal_append(defer_wal_writer* w, uint32_t token, uint64_t rng_lo, uint64_t rng_hi);
DEFER_API void defer_wal_close(defer_wal_writer* w);
/* WalLog::parse + to_checkpoint (src/wal.rs:123-209): WAL bytes to
 * checkpoint bytes; reports the record count and a discarded torn tail. */
DEFER_API int defer_wal_to_checkpoint(const uint8_t* wal, size_t len, uint8_t* ckpt, size_t cap, size_t* ckpt_len,
                                      size_t* n_records, int* torn_tail, uint64_t* valid_len);

/* `defer verify` (src/main.rs:620-666): `runs` identical sessions (seed,
 * temperature, prompt, then Session::generate of max_tokens with the stop
 * tokens) must give run 0's tokens and KV fingerprint, and Session::checkout
 * of run 0's checkpoint must reproduce that fingerprint; otherwise
 * Divergence (7) with "run N diverged from run 0" or "checkout KV cache
 * differs from live cache". out_tokens (max_tokens entries) and
 * fingerprint receive run 0's results. */
DEFER_API int defer_verify(defer_model* m, const uint8_t seed[32], float temperature, const uint32_t* prompt,
                           size_t n_prompt, uint32_t runs, size_t max_tokens, const uint32_t* stop, size_t n_stop,
                           uint32_t* out_tokens, size_t* n_out, uint8_t fingerprint[32]);

/* ----------------------------------------------------- batched drivers --- */
/* Session::checkout for n checkpoints at once, `batch` sessions advancing
 * one position per step on the device. Per session: status (0 or the
 * DeferError code), first diverging step / the token replay sampled there
 * (-1 / 0 when none), optional KV fingerprint (n * 32 bytes). device_ms:
 * device time of the replay steps. */
DEFER_API int defer_replay_batch(defer_model* m, const uint8_t* const* ckpts, const size_t* lens, size_t n, int batch,
                                 int32_t* status, int32_t* div_step, uint32_t* div_token, uint8_t* fingerprints,
                                 double* device_ms);
/* Session::new + prompt + generate for n sessions at once. out_tokens[i]
 * holds max_tokens[i] entries; n_out[i] receives the count. */
DEFER_API int defer_generate_batch(defer_model* m, const uint32_t* const* prompts, const size_t* prompt_lens,
                                   const uint8_t* seeds, const float* temperatures, const size_t* max_tokens, size_t n,
                                   int batch, uint32_t* const* out_tokens, size_t* n_out, double* device_ms);
/* attribution::ablation_attribution (src/attribution.rs:224-264): base
 * log p(target | context) and the ablated log-probability of each position,
 * variants batched `batch` at a time. */
DEFER_API int defer_ablation(defer_model* m, const uint32_t* context, size_t n, uint32_t target,
                             const size_t* positions, size_t n_pos, int batch, double* base_logprob,
                             double* ablated_logprobs);
/* Instrumentation (no counterpart in the reference, which only prints tok/s
 * at src/main.rs:303-313): totals over every token-loop run of this model
 * since the last reset — device milliseconds between CUDA events recorded
 * on the model's stream around each launch, runs, kernel launches, tokens
 * fed, and algorithmic HBM bytes (weights once per step plus KV read and
 * written). Any pointer may be NULL; reset != 0 zeroes the totals after
 * reading them. */
DEFER_API int defer_model_timing(defer_model* m, double* device_ms, uint64_t* runs, uint64_t* launches,
                                 uint64_t* tokens, double* hbm_bytes, int reset);
/* Instrumentation (no counterpart in the reference): arms a per-stage time
 * trace of step `step` (< 0 disarms) of the next dataflow token-loop run on
 * this model. For every CTA and stage of that step the kernel records
 * globaltimer nanoseconds in 24 slots: 0 stage entry, 1 inputs received
 * (after the poll), 2 + w phase warp w finished its share; warp 0 also
 * marks sub-stages in slots 10-21 (RMS statistic ready, first weight piece
 * in shared memory; attention rows staged, scores, softmax, weighted sum,
 * units, combines; in select the sampler's records published, polled,
 * decoded and walked for the sum and for the CDF). Stages: 0 select, then
 * per layer l: 1 + 5l QKV, 2 + 5l attention, 3 + 5l O, 4 + 5l gate/up,
 * 5 + 5l down; then head and two unused slots. */
DEFER_API int defer_debug_trace_arm(defer_model* m, int32_t step);
/* The last trace: n = ctas * stages * 24 stamps (0 = not reached). */
DEFER_API int defer_debug_trace_read(const defer_model* m, uint64_t* out, size_t cap, size_t* n, int32_t* ctas,
                                     int32_t* stages);
/* Fault drill (no counterpart in the reference; the test of the device
 * failure detection): the next token-loop run on this model has CTA 0
 * withhold its first hand-off of step 0 (the dataflow kernel's step header,
 * the grid-barrier kernel's first arrival) and limits every bounded wait to
 * wait_us microseconds, so the run ends with DeviceTimeout (9) and no GPU
 * fault; later runs are unaffected. */
DEFER_API int defer_debug_stall(defer_model* m, uint32_t wait_us);
/* The tensor-core contraction of the batched attribution step on its own
 * (no counterpart in the reference; its check): y [m][n] = x [m][k] .
 * w [n][k]^T with fp32 host buffers, m <= 128, computed as split-bf16
 * products accumulated in fp32 by tcgen05 MMAs on `device`; with w_bf16
 * the weights are bf16-exact values stored as bf16. */
DEFER_API int defer_debug_tc_gemm(int device, const float* x, uint32_t m, const float* w, uint32_t n, uint32_t k,
                                  int32_t w_bf16, float* y);
/* attribution::log_softmax_at (src/attribution.rs:71-85). */
DEFER_API double defer_log_softmax_at(const float* logits, size_t n, size_t idx);

#ifdef __cplusplus
}
#endif
#endif
