// Model loading (safetensors -> one HBM arena) and the device KV cache.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "device.cuh"
#include "tc.h"

namespace defer {

// Model::Config (reference src/model.rs:24-39).
struct Config {
  uint32_t vocab_size = 0, hidden_size = 0, intermediate_size = 0, num_layers = 0;
  uint32_t num_heads = 0, num_kv_heads = 0, head_dim = 0, max_seq_len = 0;
  float rms_norm_eps = 1e-6f, rope_theta = 10000.0f;
  bool tie_word_embeddings = false, gelu = false;
  int64_t bos_token_id = -1;
  std::vector<uint32_t> eos_token_ids;
  uint32_t kv_dim() const { return num_kv_heads * head_dim; }
  uint32_t q_dim() const { return num_heads * head_dim; }
};

struct Model {
  Config cfg;
  uint8_t signature[32];
  int device = 0;
  int sms = 0;
  bool bf16 = false;  // big matrices kept as bf16 in HBM
  // Every token loop of this model runs on the tensor-core step (its
  // arithmetic family): bf16-stored weights with hidden >= 2048, unless
  // DEFER_B200_TC=0 at load.
  bool tc_all = false;
  bool has_bias = false;
  void* arena = nullptr;
  size_t arena_bytes = 0;
  size_t weight_bytes = 0;  // bytes of all weights streamed by one token step
  DModel dm{};
  std::vector<DLayer> host_layers;
  DLayer* d_layers = nullptr;
  std::vector<float> inv_freq;
  cudaStream_t stream = nullptr;
  // Single-slot runner of the Model::forward entry point (owned).
  void* fwd_runner = nullptr;
  void (*fwd_runner_free)(void*) = nullptr;
  int fwd_runner_cap = 0;
  // Wide runner of position-parallel checkouts (owned, created on demand).
  mutable void* replay_runner = nullptr;
  mutable void (*replay_runner_free)(void*) = nullptr;
  mutable int replay_runner_B = 0, replay_runner_cap = 0;
  // Projections packed for the tensor-core step (built on first use).
  mutable TcModel* tc = nullptr;
  // Accumulated by every token-loop run on this model (see defer_model_timing):
  // device time between events recorded on `stream` around the launch, runs,
  // kernel launches, tokens fed, and algorithmic HBM bytes (weights once per
  // step + KV entries read and written).
  mutable double t_device_ms = 0.0;
  mutable uint64_t t_runs = 0, t_launches = 0, t_tokens = 0;
  mutable double t_bytes = 0.0;
  // Instrumentation and fault drills armed through the C ABI, each consumed
  // by the next token-loop run on this model.
  mutable int dbg_trace_step = -1;              // trace this step of the next dataflow run
  mutable std::vector<uint64_t> dbg_trace;      // last trace: [ctas][stages][kTraceSlots]
  mutable int dbg_trace_ctas = 0, dbg_trace_stages = 0;
  mutable int dbg_stall = 0;                    // withhold CTA 0's first hand-off
  mutable unsigned long long dbg_wait_ns = 0;   // bounded-wait limit of that run
  ~Model();
};

// Model::load (model.rs:286-299): parse + hash + convert + upload.
Model* load_model(const std::string& path, int device);

// Append-only KV cache of one session in HBM: K and V are
// [layers][kv_heads][cap][head_dim] fp32.
struct KvCache {
  const Model* model = nullptr;
  int cap = 0;
  size_t len = 0;
  float* k = nullptr;
  float* v = nullptr;
  uint32_t* mask = nullptr;  // [cap/32 + 1] masked-position bitmap
  ~KvCache();
  size_t layer_stride() const;  // floats per layer in k / v
};

KvCache* cache_new(const Model* m, int cap);
KvCache* cache_clone(const KvCache* c);
// Copies the first `len` positions of `src` into `dst` (same model, dst.cap >= len).
void cache_copy_prefix(KvCache* dst, const KvCache* src, size_t len, cudaStream_t st);
// Keys and values of one layer in the reference layout [len, kv_dim].
void cache_download(const KvCache* c, int layer, float* keys, float* values);
void cache_fingerprint(const KvCache* c, uint8_t out[32]);  // model.rs:233-242

}  // namespace defer
