// Token-loop engine: runners (device buffers for B concurrent sessions),
// sessions (reference src/engine.rs:23-274) and the batched replay / ablation
// drivers built on them.
#pragma once
#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "formats.h"
#include "hostutil.h"
#include "model.h"

namespace defer {

// One slot's program for a run (see DSession in device.cuh).
struct SlotProgram {
  KvCache* cache = nullptr;
  std::vector<uint32_t> tokens;  // n_total entries; generate-mode entries are filled by the run
  int n_prompt = 0;
  std::vector<uint32_t> words;   // PRNG words of the sampled steps (T > 0)
  float temperature = 0.0f;
  bool verify = false;
  std::vector<uint32_t> stop;
  bool want_margins = false;
  bool masked = false;  // the cache's mask bitmap applies to this run
  // Position-parallel replay (verify mode): programs lane = 0..lanes-1 of one
  // replay are consecutive in the run, share the cache, the tokens and the
  // words (given in the lane-0 program only) and one margins array.
  int lanes = 1, lane = 0;
};

struct SlotResult {
  int steps = 0;           // steps completed (tokens fed)
  int div_step = -1;       // first divergence (verify mode)
  uint32_t div_token = 0;  // token the replay sampled there
  std::vector<uint32_t> tokens;  // program tokens after the run
  std::vector<float> margins;
};

class Runner {
 public:
  Runner(const Model* m, int B, int max_cap);
  ~Runner();
  Runner(const Runner&) = delete;
  Runner& operator=(const Runner&) = delete;
  int capacity() const { return B_; }
  // Runs every program to completion (slot b = progs[b]).
  void run(std::vector<SlotProgram>& progs, std::vector<SlotResult>& results);
  const float* logits(int b) const;  // device pointer of slot b's logits
  void download_logits(int b, float* out) const;
  // Slot b's logits into slot db of `dst` (same model), on the model's stream.
  void copy_logits_to(int b, Runner& dst, int db) const;
  int last_steps() const { return last_steps_; }
  // Runs whose programs never sample and fit one 128-slot MMA tile take the
  // tensor-core step (DEFER_B200_TC=0 keeps them on the CUDA cores).
  bool use_tc = false;

 private:
  const Model* m_;
  int B_, max_cap_, max_chunks_, nblk_;
  float *x_ = nullptr, *q_ = nullptr, *att_ = nullptr, *g_ = nullptr, *logits_ = nullptr, *part_ = nullptr;
  int* tickets_ = nullptr;
  float* stats_ = nullptr;  // sampler block statistics, 5 arrays of [B][nblk]
  DSession* d_sess_ = nullptr;
  DSlotState* d_state_ = nullptr;
  int* d_ctrl_ = nullptr;  // status, any_active[2], barrier counter
  uint32_t* d_scratch_ = nullptr;
  size_t scratch_words_ = 0;
  uint64_t* flow_words_ = nullptr;  // tagged buffers of the dataflow kernel (B <= 8)
  size_t flow_n_ = 0;
  uint64_t flow_epoch_ = 1;         // first tag of the next run
  int last_steps_ = 0;
  cudaEvent_t ev_start_ = nullptr, ev_stop_ = nullptr;
};

// Whether runs use a persistent kernel (default) or one launch per phase
// (DEFER_B200_PHASED=1).
bool use_persistent();
// Lanes of a position-parallel checkout of n tokens (1 = one position per
// step); DEFER_B200_REPLAY_LANES overrides the default.
int replay_lanes(size_t n);
// Among the persistent kernels: 1 = the dataflow kernel where it applies,
// else the grid-barrier kernel (default); 0 = always the grid-barrier
// kernel (DEFER_B200_LOOP=barrier); 2 = the dataflow kernel or an error
// (DEFER_B200_LOOP=flow).
int loop_mode();

class Session {
 public:
  Session(const Model* m, const uint8_t seed[32], float temperature, int cache_cap);
  ~Session();
  void prompt(const uint32_t* tokens, size_t n);  // engine.rs:62-71
  uint32_t step();                                // engine.rs:113-117
  // engine.rs:121-137. on_token(token, rng_word_pos) -> status (0 = continue)
  std::vector<uint32_t> generate(size_t max_tokens, const std::vector<uint32_t>& stop,
                                 const std::function<int(uint32_t, uint64_t)>& on_token);
  // engine.rs:241-274. Long histories are replayed position-parallel: up to
  // replay_lanes() lanes feed interleaved positions of the one cache, each
  // verifying the token after the position it fed (same arithmetic per
  // position, so the same tokens, logits and KV bits as one at a time).
  static Session* checkout(const Model* m, const Checkpoint& ck, int cache_cap);
  Checkpoint checkpoint() const;                                                   // engine.rs:223-232
  bool has_logits() const { return has_logits_; }
  void last_logits(float* out) const;
  uint64_t rng_word_pos() const { return rng_.word_pos(); }

  const Model* model;
  KvCache* cache = nullptr;
  std::vector<uint32_t> history;
  size_t prompt_len = 0;
  uint8_t base_seed[32];
  float temperature;
  std::vector<float> last_margins;  // sampler margins of the last generate / checkout

 private:
  void feed_tokens(const uint32_t* t, size_t n);
  void refeed_last();
  std::unique_ptr<Runner> runner_;
  ChaCha8 rng_;
  bool has_logits_ = false;
};

// Model::forward_ext (model.rs:394-520) on a standalone cache with a
// model-owned single-slot runner; logits copied to `logits_out` if non-null.
void model_forward(Model* m, KvCache* c, uint32_t token, const size_t* masked, size_t n_masked, float* logits_out);

// Batched verified replay of many checkpoints (Session::checkout for each,
// all advanced one position per step).
struct ReplayOutcome {
  int status = 0;
  int div_step = -1;
  uint32_t div_token = 0;
  uint8_t fingerprint[32] = {0};
  std::string message;
};
void replay_batch(Model* m, const std::vector<Checkpoint>& cks, int batch, bool fingerprints,
                  std::vector<ReplayOutcome>& out, double* device_ms);

// Batched generation: n sessions (prompt, seed, temperature, max_tokens)
// run together; returns the generated tokens per session.
struct GenRequest {
  std::vector<uint32_t> prompt;
  uint8_t seed[32];
  float temperature = 0.0f;
  size_t max_tokens = 0;
};
void generate_batch(Model* m, const std::vector<GenRequest>& reqs, int batch,
                    std::vector<std::vector<uint32_t>>& out, double* device_ms);

// Leave-one-out ablation (attribution.rs:224-264), variants batched.
void ablation_batch(Model* m, const uint32_t* context, size_t n, uint32_t target, const size_t* positions,
                    size_t n_pos, int batch, double* base_logprob, double* ablated);

double log_softmax_at(const float* logits, size_t n, size_t idx);  // attribution.rs:71-85

// `defer verify` (main.rs:620-666): `runs` identical sessions must give the
// same tokens and KV fingerprint as run 0, and Session::checkout of run 0's
// checkpoint the same fingerprint; raises Divergence otherwise. Returns run
// 0's generated tokens and fingerprint.
std::vector<uint32_t> verify_runs(const Model* m, const uint8_t seed[32], float temperature,
                                  const std::vector<uint32_t>& prompt, int runs, size_t max_tokens,
                                  const std::vector<uint32_t>& stop, uint8_t fingerprint[32]);

// One forward step whose scratch lives in a fixed device array instead of
// allocated buffers (csrc/noalloc.cu); the caller owns the KV cache and the
// logits buffer.
void forward_noalloc(Model* m, float* k_cache, float* v_cache, uint32_t cap, uint32_t pos, uint32_t token,
                     float* logits_out, cudaStream_t st);

}  // namespace defer
