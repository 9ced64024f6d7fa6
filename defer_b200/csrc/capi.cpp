// extern "C" boundary (include/defer_b200.h): handle management, error
// mapping to status codes, and thin wrappers over the engine.
#include "../../include/defer_b200.h"

#include <cmath>
#include <cstring>
#include <functional>
#include <memory>

#include "common.h"
#include "engine.h"
#include "tc.h"
#include "formats.h"
#include "hostutil.h"
#include "kernels.h"
#include "model.h"

struct defer_model {
  std::unique_ptr<defer::Model> m;
};
struct defer_cache {
  defer::KvCache* c = nullptr;
  bool owned = true;
  ~defer_cache() {
    if (owned) delete c;
  }
};
struct defer_session {
  std::unique_ptr<defer::Session> s;
  defer_cache cache_view;
};
struct defer_wal_writer {
  std::unique_ptr<defer::WalWriter> w;
};

namespace {

template <class F>
int guard(F&& f) {
  try {
    f();
    return defer::kOk;
  } catch (const defer::Error& e) {
    defer::set_last_error(e.what());
    return e.status;
  } catch (const std::bad_alloc&) {
    defer::set_last_error("host out of memory");
    return defer::kIo;
  } catch (const std::exception& e) {
    defer::set_last_error(e.what());
    return defer::kInvalidArgument;
  }
}

void need(const void* p, const char* what) {
  if (!p) defer::fail(defer::kInvalidArgument, std::string(what) + " is NULL");
}

defer::Checkpoint ck_from_bytes(const uint8_t* b, size_t n) {
  need(b, "checkpoint bytes");
  return defer::Checkpoint::from_bytes(b, n);
}

void put_bytes(const std::vector<uint8_t>& v, uint8_t* buf, size_t cap, size_t* len) {
  if (len) *len = v.size();
  if (!buf) return;
  if (cap < v.size()) defer::fail(defer::kInvalidArgument, "buffer too small");
  memcpy(buf, v.data(), v.size());
}

}  // namespace

extern "C" {

const char* defer_last_error(void) { return defer::last_error(); }

int defer_model_load(const char* path, int device, defer_model** out) {
  return guard([&] {
    need(path, "path");
    need(out, "out");
    std::unique_ptr<defer_model> h(new defer_model());
    h->m.reset(defer::load_model(path, device));
    *out = h.release();
  });
}

void defer_model_free(defer_model* m) { delete m; }

int defer_model_config(const defer_model* m, defer_config* out) {
  return guard([&] {
    need(m, "model");
    need(out, "out");
    const defer::Config& c = m->m->cfg;
    out->vocab_size = c.vocab_size;
    out->hidden_size = c.hidden_size;
    out->intermediate_size = c.intermediate_size;
    out->num_layers = c.num_layers;
    out->num_heads = c.num_heads;
    out->num_kv_heads = c.num_kv_heads;
    out->head_dim = c.head_dim;
    out->max_seq_len = c.max_seq_len;
    out->rms_norm_eps = c.rms_norm_eps;
    out->rope_theta = c.rope_theta;
    out->tie_word_embeddings = c.tie_word_embeddings;
    out->gelu = c.gelu;
    out->has_bias = m->m->has_bias;
    out->weights_bf16 = m->m->bf16;
    out->bos_token_id = c.bos_token_id;
    out->weight_bytes = m->m->weight_bytes;
    out->device = m->m->device;
    out->sm_count = m->m->sms;
  });
}

int defer_model_signature(const defer_model* m, uint8_t out[32]) {
  return guard([&] {
    need(m, "model");
    need(out, "out");
    memcpy(out, m->m->signature, 32);
  });
}

int defer_model_eos_tokens(const defer_model* m, uint32_t* out, size_t cap, size_t* n) {
  return guard([&] {
    need(m, "model");
    const auto& e = m->m->cfg.eos_token_ids;
    if (n) *n = e.size();
    if (out) {
      if (cap < e.size()) defer::fail(defer::kInvalidArgument, "buffer too small");
      std::copy(e.begin(), e.end(), out);
    }
  });
}

int defer_forward(defer_model* m, defer_cache* c, uint32_t token, const size_t* masked, size_t n_masked,
                  float* logits_out) {
  return guard([&] {
    need(m, "model");
    need(c, "cache");
    if (n_masked) need(masked, "masked");
    defer::model_forward(m->m.get(), c->c, token, masked, n_masked, logits_out);
  });
}

int defer_forward_noalloc(defer_model* m, float* k_cache, float* v_cache, uint32_t cap, uint32_t pos,
                          uint32_t token, float* logits_out, void* stream) {
  return guard([&] {
    need(m, "model");
    defer::forward_noalloc(m->m.get(), k_cache, v_cache, cap, pos, token, logits_out,
                           static_cast<cudaStream_t>(stream));
  });
}

int defer_cache_new(defer_model* m, uint32_t cap, defer_cache** out) {
  return guard([&] {
    need(m, "model");
    need(out, "out");
    std::unique_ptr<defer_cache> h(new defer_cache());
    h->c = defer::cache_new(m->m.get(), (int)cap);
    *out = h.release();
  });
}

void defer_cache_free(defer_cache* c) {
  if (c && c->owned) delete c;
}

size_t defer_cache_len(const defer_cache* c) { return c ? c->c->len : 0; }

int defer_cache_truncate(defer_cache* c, size_t n) {
  return guard([&] {
    need(c, "cache");
    if (n < c->c->len) c->c->len = n;
  });
}

int defer_cache_clone(const defer_cache* c, defer_cache** out) {
  return guard([&] {
    need(c, "cache");
    need(out, "out");
    std::unique_ptr<defer_cache> h(new defer_cache());
    h->c = defer::cache_clone(c->c);
    *out = h.release();
  });
}

int defer_cache_download(const defer_cache* c, uint32_t layer, float* keys, float* values) {
  return guard([&] {
    need(c, "cache");
    if (layer >= c->c->model->cfg.num_layers) defer::fail(defer::kInvalidArgument, "layer out of range");
    if (c->c->len) {
      need(keys, "keys");
      need(values, "values");
    }
    defer::cache_download(c->c, (int)layer, keys, values);
  });
}

int defer_cache_fingerprint(const defer_cache* c, uint8_t out[32]) {
  return guard([&] {
    need(c, "cache");
    need(out, "out");
    defer::cache_fingerprint(c->c, out);
  });
}

int defer_cache_bit_eq(const defer_cache* a, const defer_cache* b, int* equal) {
  return guard([&] {
    need(a, "a");
    need(b, "b");
    need(equal, "equal");
    const auto& ca = a->c->model->cfg;
    const auto& cb = b->c->model->cfg;
    *equal = 0;
    if (a->c->len != b->c->len || ca.kv_dim() != cb.kv_dim() || ca.num_layers != cb.num_layers) return;
    const size_t n = a->c->len * ca.kv_dim();
    std::vector<float> ka(n), va(n), kb(n), vb(n);
    for (uint32_t l = 0; l < ca.num_layers; l++) {
      defer::cache_download(a->c, (int)l, ka.data(), va.data());
      defer::cache_download(b->c, (int)l, kb.data(), vb.data());
      if (memcmp(ka.data(), kb.data(), n * 4) || memcmp(va.data(), vb.data(), n * 4)) return;
    }
    *equal = 1;
  });
}

void defer_seed_from_u64(uint64_t seed, uint8_t out[32]) { defer::seed_from_u64(seed, out); }

int defer_chacha8_words(const uint8_t seed[32], uint64_t start, size_t n, uint32_t* out) {
  return guard([&] {
    need(seed, "seed");
    if (n) need(out, "out");
    defer::ChaCha8 c(seed);
    c.words(start, n, out);
  });
}

uint64_t defer_words_per_sample(float temperature) { return temperature == 0.0f ? 0 : 1; }

int defer_sample_logits(int device, const float* logits, size_t n, float temperature, uint32_t word,
                        uint32_t* token, float* margin) {
  return guard([&] {
    // sampler.rs:79-83 asserts (panics) on these; the ABI reports them.
    if (n == 0) defer::fail(defer::kInvalidArgument, "cannot sample from empty logits");
    if (!(temperature >= 0.0f && std::isfinite(temperature)))
      defer::fail(defer::kInvalidArgument, "temperature must be finite and >= 0");
    need(logits, "logits");
    need(token, "token");
    DEFER_CUDA(cudaSetDevice(device));
    struct Buf {
      void* p = nullptr;
      ~Buf() {
        if (p) cudaFree(p);
      }
    } dl, dout;
    DEFER_CUDA(cudaMalloc(&dl.p, n * 4));
    DEFER_CUDA(cudaMalloc(&dout.p, 8));
    DEFER_CUDA(cudaMemcpy(dl.p, logits, n * 4, cudaMemcpyHostToDevice));
    uint32_t* o = static_cast<uint32_t*>(dout.p);
    defer::launch_sample_one(static_cast<float*>(dl.p), (int)n, temperature, word, o, reinterpret_cast<float*>(o + 1),
                             0);
    uint32_t r[2];
    DEFER_CUDA(cudaMemcpy(r, dout.p, 8, cudaMemcpyDeviceToHost));
    *token = r[0];
    if (margin) memcpy(margin, &r[1], 4);
  });
}

int defer_session_new(defer_model* m, const uint8_t seed[32], float temperature, defer_session** out) {
  return guard([&] {
    need(m, "model");
    need(seed, "seed");
    need(out, "out");
    std::unique_ptr<defer_session> h(new defer_session());
    h->s.reset(new defer::Session(m->m.get(), seed, temperature, 0));
    h->cache_view.c = h->s->cache;
    h->cache_view.owned = false;
    *out = h.release();
  });
}

void defer_session_free(defer_session* s) { delete s; }

int defer_session_prompt(defer_session* s, const uint32_t* tokens, size_t n) {
  return guard([&] {
    need(s, "session");
    if (n) need(tokens, "tokens");
    s->s->prompt(tokens, n);
  });
}

int defer_session_step(defer_session* s, uint32_t* token) {
  return guard([&] {
    need(s, "session");
    uint32_t t = s->s->step();
    if (token) *token = t;
  });
}

int defer_session_generate(defer_session* s, size_t max_tokens, const uint32_t* stop, size_t n_stop,
                           defer_token_cb cb, void* user, uint32_t* out_tokens, size_t* n_out) {
  size_t produced = 0;
  int rc = guard([&] {
    need(s, "session");
    if (n_stop) need(stop, "stop");
    std::vector<uint32_t> st(stop, stop + (stop ? n_stop : 0));
    std::function<int(uint32_t, uint64_t)> f = [&](uint32_t t, uint64_t pos) {
      if (out_tokens) out_tokens[produced] = t;
      produced++;
      return cb ? cb(user, t, pos) : 0;
    };
    s->s->generate(max_tokens, st, f);
  });
  if (n_out) *n_out = produced;
  return rc;
}

int defer_session_checkout(defer_model* m, const uint8_t* ckpt, size_t len, defer_session** out) {
  return guard([&] {
    need(m, "model");
    need(out, "out");
    defer::Checkpoint ck = ck_from_bytes(ckpt, len);
    std::unique_ptr<defer_session> h(new defer_session());
    h->s.reset(defer::Session::checkout(m->m.get(), ck, 0));
    h->cache_view.c = h->s->cache;
    h->cache_view.owned = false;
    *out = h.release();
  });
}

int defer_session_checkpoint(const defer_session* s, uint8_t* buf, size_t cap, size_t* len) {
  return guard([&] {
    need(s, "session");
    put_bytes(s->s->checkpoint().to_bytes(), buf, cap, len);
  });
}

int defer_session_history(const defer_session* s, uint32_t* out, size_t cap, size_t* n) {
  return guard([&] {
    need(s, "session");
    const auto& h = s->s->history;
    if (n) *n = h.size();
    if (out) {
      if (cap < h.size()) defer::fail(defer::kInvalidArgument, "buffer too small");
      std::copy(h.begin(), h.end(), out);
    }
  });
}

size_t defer_session_prompt_len(const defer_session* s) { return s ? s->s->prompt_len : 0; }
uint64_t defer_session_rng_word_pos(const defer_session* s) { return s ? s->s->rng_word_pos() : 0; }

int defer_session_last_logits(const defer_session* s, float* out) {
  return guard([&] {
    need(s, "session");
    need(out, "out");
    s->s->last_logits(out);
  });
}

defer_cache* defer_session_cache(defer_session* s) { return s ? &s->cache_view : nullptr; }

int defer_session_margins(const defer_session* s, float* out, size_t cap, size_t* n) {
  return guard([&] {
    need(s, "session");
    const auto& v = s->s->last_margins;
    if (n) *n = v.size();
    if (out) {
      if (cap < v.size()) defer::fail(defer::kInvalidArgument, "buffer too small");
      std::copy(v.begin(), v.end(), out);
    }
  });
}

int defer_checkpoint_encode(const defer_checkpoint_fields* f, uint8_t* buf, size_t cap, size_t* len) {
  return guard([&] {
    need(f, "fields");
    defer::Checkpoint c;
    memcpy(c.model_signature, f->model_signature, 32);
    memcpy(c.base_seed, f->base_seed, 32);
    c.temperature = f->temperature;
    c.prompt_len = f->prompt_len;
    c.rng_word_pos = defer::U128{f->rng_word_pos_lo, f->rng_word_pos_hi};
    if (f->n_tokens) need(f->history_tokens, "history_tokens");
    c.history_tokens.assign(f->history_tokens, f->history_tokens + f->n_tokens);
    put_bytes(c.to_bytes(), buf, cap, len);
  });
}

int defer_checkpoint_decode(const uint8_t* b, size_t len, defer_checkpoint_fields* f, uint32_t* tokens_out,
                            size_t tokens_cap) {
  return guard([&] {
    need(f, "fields");
    defer::Checkpoint c = ck_from_bytes(b, len);
    memcpy(f->model_signature, c.model_signature, 32);
    memcpy(f->base_seed, c.base_seed, 32);
    f->temperature = c.temperature;
    f->prompt_len = c.prompt_len;
    f->rng_word_pos_lo = c.rng_word_pos.lo;
    f->rng_word_pos_hi = c.rng_word_pos.hi;
    f->n_tokens = c.history_tokens.size();
    f->history_tokens = tokens_out;
    if (tokens_out) {
      if (tokens_cap < c.history_tokens.size()) defer::fail(defer::kInvalidArgument, "buffer too small");
      std::copy(c.history_tokens.begin(), c.history_tokens.end(), tokens_out);
    }
  });
}

int defer_checkpoint_save(const uint8_t* bytes, size_t len, const char* path) {
  return guard([&] {
    need(path, "path");
    ck_from_bytes(bytes, len).save(path);
  });
}

int defer_checkpoint_load(const char* path, uint8_t* buf, size_t cap, size_t* len) {
  return guard([&] {
    need(path, "path");
    put_bytes(defer::Checkpoint::load(path).to_bytes(), buf, cap, len);
  });
}

static defer::WalHeader wal_header(const defer_wal_header* h) {
  need(h, "header");
  defer::WalHeader w;
  memcpy(w.model_signature, h->model_signature, 32);
  memcpy(w.base_seed, h->base_seed, 32);
  w.temperature = h->temperature;
  w.prompt_len = h->prompt_len;
  w.start_rng_word_pos = defer::U128{h->start_rng_word_pos_lo, h->start_rng_word_pos_hi};
  if (h->n_prefix) need(h->prefix_tokens, "prefix_tokens");
  w.prefix_tokens.assign(h->prefix_tokens, h->prefix_tokens + h->n_prefix);
  return w;
}

int defer_wal_create(const char* path, const defer_wal_header* h, int durable, defer_wal_writer** out) {
  return guard([&] {
    need(path, "path");
    need(out, "out");
    std::unique_ptr<defer_wal_writer> w(new defer_wal_writer());
    w->w.reset(defer::WalWriter::create(path, wal_header(h), durable != 0));
    *out = w.release();
  });
}

int defer_wal_resume(const char* path, int durable, defer_wal_writer** out) {
  return guard([&] {
    need(path, "path");
    need(out, "out");
    std::unique_ptr<defer_wal_writer> w(new defer_wal_writer());
    w->w.reset(defer::WalWriter::resume(path, durable != 0, nullptr));
    *out = w.release();
  });
}

int defer_wal_append(defer_wal_writer* w, uint32_t token, uint64_t rng_lo, uint64_t rng_hi) {
  return guard([&] {
    need(w, "writer");
    w->w->append(token, defer::U128{rng_lo, rng_hi});
  });
}

void defer_wal_close(defer_wal_writer* w) { delete w; }

int defer_wal_to_checkpoint(const uint8_t* wal, size_t len, uint8_t* ckpt, size_t cap, size_t* ckpt_len,
                            size_t* n_records, int* torn_tail, uint64_t* valid_len) {
  return guard([&] {
    need(wal, "wal");
    defer::WalLog log = defer::WalLog::parse(wal, len);
    if (n_records) *n_records = log.records.size();
    if (torn_tail) *torn_tail = log.torn_tail ? 1 : 0;
    if (valid_len) *valid_len = log.valid_len;
    put_bytes(log.to_checkpoint().to_bytes(), ckpt, cap, ckpt_len);
  });
}

int defer_replay_batch(defer_model* m, const uint8_t* const* ckpts, const size_t* lens, size_t n, int batch,
                       int32_t* status, int32_t* div_step, uint32_t* div_token, uint8_t* fingerprints,
                       double* device_ms) {
  return guard([&] {
    need(m, "model");
    if (n) {
      need(ckpts, "ckpts");
      need(lens, "lens");
    }
    std::vector<defer::Checkpoint> good;
    std::vector<size_t> idx;
    std::vector<int> parse_err(n, 0);
    for (size_t i = 0; i < n; i++) {
      try {
        good.push_back(ck_from_bytes(ckpts[i], lens[i]));
        idx.push_back(i);
      } catch (const defer::Error& e) {
        parse_err[i] = e.status;
      }
    }
    std::vector<defer::ReplayOutcome> out;
    defer::replay_batch(m->m.get(), good, batch, fingerprints != nullptr, out, device_ms);
    for (size_t i = 0; i < n; i++) {
      if (status) status[i] = parse_err[i];
      if (div_step) div_step[i] = -1;
      if (div_token) div_token[i] = 0;
      if (fingerprints) memset(fingerprints + 32 * i, 0, 32);
    }
    for (size_t j = 0; j < idx.size(); j++) {
      const size_t i = idx[j];
      if (status) status[i] = out[j].status;
      if (div_step) div_step[i] = out[j].div_step;
      if (div_token) div_token[i] = out[j].div_token;
      if (fingerprints) memcpy(fingerprints + 32 * i, out[j].fingerprint, 32);
    }
  });
}

int defer_generate_batch(defer_model* m, const uint32_t* const* prompts, const size_t* prompt_lens,
                         const uint8_t* seeds, const float* temperatures, const size_t* max_tokens, size_t n,
                         int batch, uint32_t* const* out_tokens, size_t* n_out, double* device_ms) {
  return guard([&] {
    need(m, "model");
    if (n) {
      need(prompts, "prompts");
      need(prompt_lens, "prompt_lens");
      need(seeds, "seeds");
      need(temperatures, "temperatures");
      need(max_tokens, "max_tokens");
    }
    std::vector<defer::GenRequest> reqs(n);
    for (size_t i = 0; i < n; i++) {
      reqs[i].prompt.assign(prompts[i], prompts[i] + prompt_lens[i]);
      memcpy(reqs[i].seed, seeds + 32 * i, 32);
      reqs[i].temperature = temperatures[i];
      reqs[i].max_tokens = max_tokens[i];
    }
    std::vector<std::vector<uint32_t>> out;
    defer::generate_batch(m->m.get(), reqs, batch, out, device_ms);
    for (size_t i = 0; i < n; i++) {
      if (n_out) n_out[i] = out[i].size();
      if (out_tokens && out_tokens[i]) std::copy(out[i].begin(), out[i].end(), out_tokens[i]);
    }
  });
}

int defer_ablation(defer_model* m, const uint32_t* context, size_t n, uint32_t target, const size_t* positions,
                   size_t n_pos, int batch, double* base_logprob, double* ablated_logprobs) {
  return guard([&] {
    need(m, "model");
    if (n) need(context, "context");
    if (n_pos) {
      need(positions, "positions");
      need(ablated_logprobs, "ablated_logprobs");
    }
    double base = 0.0;
    defer::ablation_batch(m->m.get(), context, n, target, positions, n_pos, batch, &base, ablated_logprobs);
    if (base_logprob) *base_logprob = base;
  });
}

int defer_model_timing(defer_model* m, double* device_ms, uint64_t* runs, uint64_t* launches, uint64_t* tokens,
                       double* hbm_bytes, int reset) {
  return guard([&] {
    need(m, "model");
    const defer::Model& M = *m->m;
    if (device_ms) *device_ms = M.t_device_ms;
    if (runs) *runs = M.t_runs;
    if (launches) *launches = M.t_launches;
    if (tokens) *tokens = M.t_tokens;
    if (hbm_bytes) *hbm_bytes = M.t_bytes;
    if (reset) {
      M.t_device_ms = 0.0;
      M.t_runs = M.t_launches = M.t_tokens = 0;
      M.t_bytes = 0.0;
    }
  });
}

int defer_debug_trace_arm(defer_model* m, int32_t step) {
  return guard([&] {
    need(m, "model");
    m->m->dbg_trace_step = step < 0 ? -1 : step;
    m->m->dbg_trace.clear();
  });
}

int defer_debug_trace_read(const defer_model* m, uint64_t* out, size_t cap, size_t* n, int32_t* ctas,
                           int32_t* stages) {
  return guard([&] {
    need(m, "model");
    const defer::Model& M = *m->m;
    if (n) *n = M.dbg_trace.size();
    if (ctas) *ctas = M.dbg_trace_ctas;
    if (stages) *stages = M.dbg_trace_stages;
    if (out) {
      if (cap < M.dbg_trace.size()) defer::fail(defer::kInvalidArgument, "trace buffer too small");
      std::copy(M.dbg_trace.begin(), M.dbg_trace.end(), out);
    }
  });
}

int defer_verify(defer_model* m, const uint8_t seed[32], float temperature, const uint32_t* prompt, size_t n_prompt,
                 uint32_t runs, size_t max_tokens, const uint32_t* stop, size_t n_stop, uint32_t* out_tokens,
                 size_t* n_out, uint8_t fingerprint[32]) {
  return guard([&] {
    need(m, "model");
    if (!seed || !fingerprint || (n_prompt && !prompt) || (n_stop && !stop) || (max_tokens && !out_tokens))
      defer::fail(defer::kInvalidArgument, "null buffer");
    std::vector<uint32_t> p(prompt, prompt + n_prompt), st(stop, stop + n_stop);
    std::vector<uint32_t> out =
        defer::verify_runs(m->m.get(), seed, temperature, p, (int)runs, max_tokens, st, fingerprint);
    std::copy(out.begin(), out.end(), out_tokens);
    if (n_out) *n_out = out.size();
  });
}

int defer_debug_tc_gemm(int device, const float* x, uint32_t m, const float* w, uint32_t n, uint32_t k,
                        int32_t w_bf16, float* y) {
  return guard([&] {
    if (!x || !w || !y) defer::fail(defer::kInvalidArgument, "null buffer");
    defer::tc_gemm_check(device, x, (int)m, w, (int)n, (int)k, w_bf16 != 0, y);
  });
}

int defer_debug_stall(defer_model* m, uint32_t wait_us) {
  return guard([&] {
    need(m, "model");
    if (wait_us == 0 || wait_us > 10000000u) defer::fail(defer::kInvalidArgument, "wait_us must be in 1..10^7");
    m->m->dbg_stall = 1;
    m->m->dbg_wait_ns = (unsigned long long)wait_us * 1000ull;
  });
}

double defer_log_softmax_at(const float* logits, size_t n, size_t idx) {
  return defer::log_softmax_at(logits, n, idx);
}

}  // extern "C"
