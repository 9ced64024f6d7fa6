// Model::load for the B200 engine: a single sequential pass over the
// safetensors file (SHA-256 of every byte = model signature, reference
// src/safetensors.rs:142-237), the config (src/model.rs:44-118, 286-299),
// shape checks by HuggingFace tensor name (src/model.rs:301-347), and the
// upload into one HBM arena:
//
//   [embed][layer 0 .. L-1: attn_norm, wqkv, bqkv, wo, ffn_norm, wgu, wdown]
//   [final norm][lm_head if untied][rope cos][rope sin]
//
// wqkv rows are pair-interleaved so one warp owns both halves of every
// RoPE pair; wgu interleaves gate and up rows so one warp owns both inputs
// of each SiLU*up product. Big matrices stay bf16 when the file stores all
// of them as bf16 (exact), otherwise everything is fp32.
#include "model.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>

#include "common.h"
#include "hostutil.h"

namespace defer {

namespace {

enum class DType { F32, F16, BF16, F64 };

size_t dtype_size(DType d) { return d == DType::F64 ? 8 : (d == DType::F32 ? 4 : 2); }

struct TensorRef {
  std::string name;
  DType dtype;
  std::vector<uint64_t> shape;
  uint64_t start = 0, end = 0;
  const uint8_t* data = nullptr;
  uint64_t numel() const {
    uint64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
};

// IEEE binary16 -> binary32, exact (safetensors.rs:47-71).
float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1F;
  uint32_t mant = h & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else {
      int e = 0;
      uint32_t m = mant;
      while (!(m & 0x400)) {
        m <<= 1;
        e--;
      }
      m &= 0x3FF;
      bits = sign | ((uint32_t)(127 - 14 + e) << 23) | (m << 13);
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (mant << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

void to_f32(const TensorRef& t, uint64_t first, uint64_t n, float* out) {
  const uint8_t* p = t.data + first * dtype_size(t.dtype);
  switch (t.dtype) {
    case DType::F32: memcpy(out, p, n * 4); break;
    case DType::F16:
      for (uint64_t i = 0; i < n; i++) {
        uint16_t h;
        memcpy(&h, p + 2 * i, 2);
        out[i] = f16_to_f32(h);
      }
      break;
    case DType::BF16:
      for (uint64_t i = 0; i < n; i++) {
        uint16_t h;
        memcpy(&h, p + 2 * i, 2);
        uint32_t b = (uint32_t)h << 16;
        memcpy(out + i, &b, 4);
      }
      break;
    case DType::F64:
      for (uint64_t i = 0; i < n; i++) {
        double d;
        memcpy(&d, p + 8 * i, 8);
        out[i] = (float)d;
      }
      break;
  }
}

// Streams the arena image to the device through two pinned staging
// buffers; destinations are written in increasing offset order.
class Uploader {
 public:
  Uploader(char* dev, cudaStream_t st) : dev_(dev), st_(st) {
    DEFER_CUDA(cudaMallocHost(&buf_[0], kCap));
    DEFER_CUDA(cudaMallocHost(&buf_[1], kCap));
    DEFER_CUDA(cudaEventCreateWithFlags(&ev_[0], cudaEventDisableTiming));
    DEFER_CUDA(cudaEventCreateWithFlags(&ev_[1], cudaEventDisableTiming));
  }
  ~Uploader() {
    cudaStreamSynchronize(st_);
    cudaFreeHost(buf_[0]);
    cudaFreeHost(buf_[1]);
    cudaEventDestroy(ev_[0]);
    cudaEventDestroy(ev_[1]);
  }
  void seek(size_t off) {
    if (off < base_ + fill_) fail(kModel, "internal: arena written out of order");
    if (off != base_ + fill_) {
      flush();
      base_ = off;
    }
  }
  // Reserves n bytes of the staging buffer at the current position.
  char* reserve(size_t n) {
    if (n > kCap) fail(kModel, "internal: staging request too large");
    if (fill_ + n > kCap) flush();
    char* p = buf_[cur_] + fill_;
    fill_ += n;
    return p;
  }
  void flush() {
    if (fill_) {
      DEFER_CUDA(cudaMemcpyAsync(dev_ + base_, buf_[cur_], fill_, cudaMemcpyHostToDevice, st_));
      DEFER_CUDA(cudaEventRecord(ev_[cur_], st_));
      base_ += fill_;
      fill_ = 0;
      cur_ ^= 1;
      DEFER_CUDA(cudaEventSynchronize(ev_[cur_]));  // the other buffer is free again
    }
  }
  void finish() {
    flush();
    DEFER_CUDA(cudaStreamSynchronize(st_));
  }

 private:
  static constexpr size_t kCap = 32u << 20;
  char* dev_;
  cudaStream_t st_;
  char* buf_[2] = {nullptr, nullptr};
  cudaEvent_t ev_[2];
  int cur_ = 0;
  size_t base_ = 0, fill_ = 0;
};

struct MappedFile {
  int fd = -1;
  void* p = MAP_FAILED;
  size_t n = 0;
  ~MappedFile() {
    if (p != MAP_FAILED) munmap(p, n);
    if (fd >= 0) close(fd);
  }
};

std::string shape_str(const std::vector<uint64_t>& s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); i++) o += (i ? ", " : "") + std::to_string(s[i]);
  return o + "]";
}

size_t align_up(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

Model::~Model() {
  if (fwd_runner && fwd_runner_free) fwd_runner_free(fwd_runner);
  if (replay_runner && replay_runner_free) replay_runner_free(replay_runner);
  delete tc;
  if (arena) cudaFree(arena);
  if (d_layers) cudaFree(d_layers);
  if (stream) cudaStreamDestroy(stream);
}

static Config config_from_json(const Json& v, const std::map<std::string, TensorRef>& st) {
  auto num = [&](const char* k, uint64_t* out) {
    const Json* x = v.get(k);
    return x && x->as_u64(out);
  };
  auto flt = [&](const char* k, double* out) {
    const Json* x = v.get(k);
    return x && x->as_f64(out);
  };
  auto missing = [](const char* k) { fail(kModel, std::string("config is missing `") + k + "`"); };
  const TensorRef* embed = nullptr;
  for (const char* n : {"model.embed_tokens.weight", "embed_tokens.weight"}) {
    auto it = st.find(n);
    if (it != st.end()) {
      embed = &it->second;
      break;
    }
  }
  bool guess = embed && embed->shape.size() == 2;
  Config c;
  uint64_t u;
  double d;
  if (num("hidden_size", &u)) c.hidden_size = (uint32_t)u;
  else if (guess) c.hidden_size = (uint32_t)embed->shape[1];
  else missing("hidden_size");
  if (num("vocab_size", &u)) c.vocab_size = (uint32_t)u;
  else if (guess) c.vocab_size = (uint32_t)embed->shape[0];
  else missing("vocab_size");
  if (num("num_hidden_layers", &u)) {
    c.num_layers = (uint32_t)u;
  } else {
    uint32_t n = 0;
    while (st.count("model.layers." + std::to_string(n) + ".input_layernorm.weight")) n++;
    if (n == 0) missing("num_hidden_layers");
    c.num_layers = n;
  }
  if (num("intermediate_size", &u)) {
    c.intermediate_size = (uint32_t)u;
  } else {
    auto it = st.find("model.layers.0.mlp.gate_proj.weight");
    if (it == st.end() || it->second.shape.empty()) missing("intermediate_size");
    c.intermediate_size = (uint32_t)it->second.shape[0];
  }
  if (!num("num_attention_heads", &u)) missing("num_attention_heads");
  c.num_heads = (uint32_t)u;
  c.num_kv_heads = num("num_key_value_heads", &u) ? (uint32_t)u : c.num_heads;
  c.head_dim = num("head_dim", &u) ? (uint32_t)u : (c.num_heads ? c.hidden_size / c.num_heads : 0);
  const Json* act = v.get("hidden_act");
  std::string a = act && act->as_str() ? *act->as_str() : "silu";
  if (a == "silu" || a == "swish") c.gelu = false;
  else if (a.rfind("gelu", 0) == 0) c.gelu = true;
  else fail(kModel, "unsupported activation " + a);
  const Json* eos = v.get("eos_token_id");
  if (eos && eos->kind == Json::Array) {
    for (auto& x : eos->arr)
      if (x.as_u64(&u)) c.eos_token_ids.push_back((uint32_t)u);
  } else if (eos && eos->as_u64(&u)) {
    c.eos_token_ids.push_back((uint32_t)u);
  }
  bool has_lm_head = st.count("lm_head.weight") > 0;
  c.rms_norm_eps = flt("rms_norm_eps", &d) ? (float)d : 1e-6f;
  c.rope_theta = flt("rope_theta", &d) ? (float)d : 10000.0f;
  c.max_seq_len = num("max_position_embeddings", &u) ? (uint32_t)u : 4096;
  const Json* tie = v.get("tie_word_embeddings");
  bool t = (tie && tie->kind == Json::Bool) ? tie->b : !has_lm_head;
  c.tie_word_embeddings = t || !has_lm_head;
  if (num("bos_token_id", &u)) c.bos_token_id = (int64_t)u;
  if (c.num_kv_heads == 0 || c.num_heads % c.num_kv_heads != 0)
    fail(kModel, "num_attention_heads must be a multiple of num_key_value_heads");
  if (c.head_dim % 2 != 0) fail(kModel, "head_dim must be even for RoPE");
  return c;
}

Model* load_model(const std::string& path, int device) {
  DEFER_CUDA(cudaSetDevice(device));
  MappedFile mf;
  mf.fd = open(path.c_str(), O_RDONLY);
  if (mf.fd < 0) fail(kModel, "cannot open " + path + ": " + strerror(errno));
  struct stat sb;
  if (fstat(mf.fd, &sb) != 0) fail(kIo, "cannot stat " + path);
  mf.n = (size_t)sb.st_size;
  if (mf.n < 8) fail(kIo, "failed to fill whole buffer");
  mf.p = mmap(nullptr, mf.n, PROT_READ, MAP_PRIVATE, mf.fd, 0);
  if (mf.p == MAP_FAILED) fail(kIo, "cannot map " + path);
  madvise(mf.p, mf.n, MADV_SEQUENTIAL);
  const uint8_t* file = (const uint8_t*)mf.p;

  std::unique_ptr<Model> M(new Model());
  M->device = device;
  {
    Sha256 h;
    const size_t step = 64u << 20;
    for (size_t off = 0; off < mf.n; off += step) h.update(file + off, std::min(step, mf.n - off));
    h.finalize(M->signature);
  }
  uint64_t header_len;
  memcpy(&header_len, file, 8);
  if (header_len > 100ull * 1024 * 1024 || 8 + header_len > mf.n) fail(kModel, "invalid safetensors header length");
  std::string hs((const char*)file + 8, header_len);
  Json hdr = parse_json(hs);
  if (hdr.kind != Json::Object) fail(kModel, "safetensors header is not an object");
  std::vector<std::pair<std::string, std::string>> meta;
  std::vector<TensorRef> entries;
  for (auto& kv : hdr.obj) {
    const std::string& name = kv.first;
    const Json& v = kv.second;
    if (name == "__metadata__") {
      if (v.kind == Json::Object)
        for (auto& m : v.obj)
          if (m.second.as_str()) meta.emplace_back(m.first, *m.second.as_str());
      continue;
    }
    auto bad = [&]() { fail(kModel, "malformed header entry for " + name); };
    const Json* dt = v.get("dtype");
    if (!dt || !dt->as_str()) bad();
    TensorRef t;
    t.name = name;
    const std::string& ds = *dt->as_str();
    if (ds == "F32") t.dtype = DType::F32;
    else if (ds == "F16") t.dtype = DType::F16;
    else if (ds == "BF16") t.dtype = DType::BF16;
    else if (ds == "F64") t.dtype = DType::F64;
    else fail(kModel, "unsupported safetensors dtype " + ds);
    const Json* sh = v.get("shape");
    if (!sh || sh->kind != Json::Array) bad();
    for (auto& x : sh->arr) {
      uint64_t u;
      if (!x.as_u64(&u)) bad();
      t.shape.push_back(u);
    }
    const Json* offs = v.get("data_offsets");
    if (!offs || offs->kind != Json::Array || offs->arr.size() != 2) bad();
    if (!offs->arr[0].as_u64(&t.start) || !offs->arr[1].as_u64(&t.end)) bad();
    if (t.end < t.start || t.end - t.start != t.numel() * dtype_size(t.dtype))
      fail(kModel, "size mismatch for tensor " + name);
    entries.push_back(t);
  }
  std::sort(entries.begin(), entries.end(), [](const TensorRef& a, const TensorRef& b) {
    return a.start != b.start ? a.start < b.start : a.name < b.name;
  });
  const uint64_t data_len = mf.n - 8 - header_len;
  uint64_t pos = 0;
  std::map<std::string, TensorRef> st;
  for (auto& e : entries) {
    if (e.start < pos || e.end > data_len) fail(kModel, "overlapping/out of range tensor " + e.name);
    e.data = file + 8 + header_len + e.start;
    pos = e.end;
    st[e.name] = e;
  }

  // Config: `defer.config` metadata, else config.json beside the weights.
  Json cfgv;
  cfgv.kind = Json::Object;
  bool from_meta = false;
  for (auto& m : meta)
    if (m.first == "defer.config") {
      cfgv = parse_json(m.second);
      from_meta = true;
      break;
    }
  if (!from_meta) {
    size_t slash = path.find_last_of('/');
    std::string dir = slash == std::string::npos ? "" : path.substr(0, slash + 1);
    FILE* f = fopen((dir + "config.json").c_str(), "rb");
    if (f) {
      std::string s;
      char buf[4096];
      size_t n;
      while ((n = fread(buf, 1, sizeof(buf), f)) > 0) s.append(buf, n);
      fclose(f);
      cfgv = parse_json(s);
    }
  }
  Config c = config_from_json(cfgv, st);
  M->cfg = c;

  // from_safetensors: names and shapes.
  const char* embed_name = st.count("model.embed_tokens.weight") ? "model.embed_tokens.weight" : "embed_tokens.weight";
  M->has_bias = st.count("model.layers.0.self_attn.q_proj.bias") > 0;
  auto take = [&](const std::string& name, std::vector<uint64_t> shape) -> const TensorRef& {
    auto it = st.find(name);
    if (it == st.end()) fail(kModel, "missing tensor " + name);
    uint64_t n = 1;
    for (auto d : shape) n *= d;
    if (it->second.numel() != n)
      fail(kModel, "tensor " + name + " has shape " + shape_str(it->second.shape) + ", expected " + shape_str(shape));
    return it->second;
  };
  const uint64_t H = c.hidden_size, Q = c.q_dim(), KV = c.kv_dim(), FF = c.intermediate_size, V = c.vocab_size;
  const TensorRef& embed = take(embed_name, {V, H});
  struct LRefs {
    const TensorRef *an, *wq, *bq, *wk, *bk, *wv, *bv, *wo, *fn, *wg, *wu, *wd;
  };
  std::vector<LRefs> lr(c.num_layers);
  for (uint32_t i = 0; i < c.num_layers; i++) {
    std::string p = "model.layers." + std::to_string(i);
    LRefs& r = lr[i];
    r.an = &take(p + ".input_layernorm.weight", {H});
    r.wq = &take(p + ".self_attn.q_proj.weight", {Q, H});
    r.bq = M->has_bias ? &take(p + ".self_attn.q_proj.bias", {Q}) : nullptr;
    r.wk = &take(p + ".self_attn.k_proj.weight", {KV, H});
    r.bk = M->has_bias ? &take(p + ".self_attn.k_proj.bias", {KV}) : nullptr;
    r.wv = &take(p + ".self_attn.v_proj.weight", {KV, H});
    r.bv = M->has_bias ? &take(p + ".self_attn.v_proj.bias", {KV}) : nullptr;
    r.wo = &take(p + ".self_attn.o_proj.weight", {H, Q});
    r.fn = &take(p + ".post_attention_layernorm.weight", {H});
    r.wg = &take(p + ".mlp.gate_proj.weight", {FF, H});
    r.wu = &take(p + ".mlp.up_proj.weight", {FF, H});
    r.wd = &take(p + ".mlp.down_proj.weight", {H, FF});
  }
  const TensorRef& norm = take("model.norm.weight", {H});
  const TensorRef* head = c.tie_word_embeddings ? nullptr : &take("lm_head.weight", {V, H});

  // Device constraints of the canonical 16-byte chunking.
  bool all_bf16 = embed.dtype == DType::BF16 && (!head || head->dtype == DType::BF16);
  for (auto& r : lr)
    for (const TensorRef* t : {r.wq, r.wk, r.wv, r.wo, r.wg, r.wu, r.wd}) all_bf16 = all_bf16 && t->dtype == DType::BF16;
  M->bf16 = all_bf16;
  {
    const char* e = getenv("DEFER_B200_TC");
    M->tc_all = all_bf16 && c.hidden_size >= 2048 && !(e && e[0] == '0');
  }
  const uint64_t E = M->bf16 ? 8 : 4;
  if (H % E || Q % E || FF % E)
    fail(kModel, "hidden, q and intermediate sizes must be multiples of " + std::to_string(E) + " on the B200 path");
  if (c.head_dim % 4) fail(kModel, "head_dim must be a multiple of 4 on the B200 path");
  if (c.max_seq_len == 0) fail(kModel, "max_position_embeddings must be positive");

  // Arena layout.
  const size_t ws = M->bf16 ? 2 : 4;
  const uint64_t QKVR = Q + 2 * KV;
  const uint64_t half = c.head_dim / 2;
  size_t off = 0;
  auto place = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes);
    return o;
  };
  size_t o_embed = place(V * H * ws);
  struct LOff {
    size_t an, wqkv, bqkv, wo, fn, wgu, wd;
  };
  std::vector<LOff> lo(c.num_layers);
  for (auto& L : lo) {
    L.an = place(H * 4);
    L.wqkv = place(QKVR * H * ws);
    L.bqkv = M->has_bias ? place(QKVR * 4) : 0;
    L.wo = place(H * Q * ws);
    L.fn = place(H * 4);
    L.wgu = place(2 * FF * H * ws);
    L.wd = place(H * FF * ws);
  }
  size_t o_norm = place(H * 4);
  size_t o_head = head ? place(V * H * ws) : o_embed;
  size_t o_cos = place((size_t)c.max_seq_len * half * 4);
  size_t o_sin = place((size_t)c.max_seq_len * half * 4);
  M->arena_bytes = off;
  // Bytes one token step must stream: the embedding row, every layer's
  // matrices and norms, the final norm and the head.
  M->weight_bytes = H * ws + V * H * ws +
                    (size_t)c.num_layers * (2 * H * 4 + (QKVR * H + H * Q + 3 * FF * H) * ws +
                                            (M->has_bias ? QKVR * 4 : 0)) +
                    H * 4;

  int sms = 0;
  DEFER_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  M->sms = sms;
  DEFER_CUDA(cudaStreamCreateWithFlags(&M->stream, cudaStreamNonBlocking));
  DEFER_CUDA(cudaMalloc(&M->arena, M->arena_bytes));
  char* dev = (char*)M->arena;

  {
    Uploader up(dev, M->stream);
    // rows [r0, r0 + n) of t in the device dtype
    auto put_rows = [&](const TensorRef& t, uint64_t r0, uint64_t nrows, uint64_t cols) {
      const uint64_t n = nrows * cols;
      char* dst = up.reserve(n * ws);
      if (M->bf16) memcpy(dst, t.data + r0 * cols * 2, n * 2);
      else to_f32(t, r0 * cols, n, (float*)dst);
    };
    auto put_matrix = [&](const TensorRef& t, uint64_t rows, uint64_t cols) {
      const uint64_t chunk = std::max<uint64_t>(1, (8u << 20) / (cols * ws));
      for (uint64_t r = 0; r < rows; r += chunk) put_rows(t, r, std::min(chunk, rows - r), cols);
    };
    auto put_f32 = [&](const TensorRef& t) {
      char* dst = up.reserve(t.numel() * 4);
      to_f32(t, 0, t.numel(), (float*)dst);
    };
    up.seek(o_embed);
    put_matrix(embed, V, H);
    for (uint32_t l = 0; l < c.num_layers; l++) {
      const LRefs& r = lr[l];
      up.seek(lo[l].an);
      put_f32(*r.an);
      up.seek(lo[l].wqkv);
      // unit u -> rows (i, i + half) of one head of q, then k, then v
      const TensorRef* srcs[3] = {r.wq, r.wk, r.wv};
      const uint64_t heads[3] = {c.num_heads, c.num_kv_heads, c.num_kv_heads};
      for (int s = 0; s < 3; s++)
        for (uint64_t h = 0; h < heads[s]; h++)
          for (uint64_t i = 0; i < half; i++) {
            put_rows(*srcs[s], h * c.head_dim + i, 1, H);
            put_rows(*srcs[s], h * c.head_dim + i + half, 1, H);
          }
      if (M->has_bias) {
        up.seek(lo[l].bqkv);
        const TensorRef* bs[3] = {r.bq, r.bk, r.bv};
        for (int s = 0; s < 3; s++)
          for (uint64_t h = 0; h < heads[s]; h++)
            for (uint64_t i = 0; i < half; i++) {
              to_f32(*bs[s], h * c.head_dim + i, 1, (float*)up.reserve(4));
              to_f32(*bs[s], h * c.head_dim + i + half, 1, (float*)up.reserve(4));
            }
      }
      up.seek(lo[l].wo);
      put_matrix(*r.wo, H, Q);
      up.seek(lo[l].fn);
      put_f32(*r.fn);
      up.seek(lo[l].wgu);
      for (uint64_t j = 0; j < FF; j++) {
        put_rows(*r.wg, j, 1, H);
        put_rows(*r.wu, j, 1, H);
      }
      up.seek(lo[l].wd);
      put_matrix(*r.wd, H, FF);
    }
    up.seek(o_norm);
    put_f32(norm);
    if (head) {
      up.seek(o_head);
      put_matrix(*head, V, H);
    }
    // RoPE: inv_freq in f64 rounded to f32 (model.rs:348-353); the angle is
    // the f32 product pos * inv_freq, cos/sin from the host libm
    // (model.rs:438-445), so the tables are bit-identical to the CPU path.
    M->inv_freq.resize(half);
    for (uint64_t i = 0; i < half; i++) {
      double ex = (double)(2 * i) / (double)c.head_dim;
      M->inv_freq[i] = (float)(1.0 / pow((double)c.rope_theta, ex));
    }
    const size_t rows_per = std::max<size_t>(1, (4u << 20) / (half * 4));
    for (int which = 0; which < 2; which++) {
      up.seek(which ? o_sin : o_cos);
      for (size_t p0 = 0; p0 < c.max_seq_len; p0 += rows_per) {
        size_t n = std::min<size_t>(rows_per, c.max_seq_len - p0);
        float* dst = (float*)up.reserve(n * half * 4);
        for (size_t p = 0; p < n; p++)
          for (uint64_t i = 0; i < half; i++) {
            float angle = (float)(p0 + p) * M->inv_freq[i];
            dst[p * half + i] = which ? sinf(angle) : cosf(angle);
          }
      }
    }
    up.finish();
  }

  M->host_layers.resize(c.num_layers);
  for (uint32_t l = 0; l < c.num_layers; l++) {
    DLayer& L = M->host_layers[l];
    L.attn_norm = (const float*)(dev + lo[l].an);
    L.wqkv = dev + lo[l].wqkv;
    L.bqkv = M->has_bias ? (const float*)(dev + lo[l].bqkv) : nullptr;
    L.wo = dev + lo[l].wo;
    L.ffn_norm = (const float*)(dev + lo[l].fn);
    L.wgu = dev + lo[l].wgu;
    L.wdown = dev + lo[l].wd;
  }
  DEFER_CUDA(cudaMalloc(&M->d_layers, sizeof(DLayer) * std::max<uint32_t>(1, c.num_layers)));
  DEFER_CUDA(cudaMemcpy(M->d_layers, M->host_layers.data(), sizeof(DLayer) * c.num_layers, cudaMemcpyHostToDevice));

  DModel& d = M->dm;
  d.V = (int)V;
  d.H = (int)H;
  d.FF = (int)FF;
  d.L = (int)c.num_layers;
  d.NH = (int)c.num_heads;
  d.NKV = (int)c.num_kv_heads;
  d.HD = (int)c.head_dim;
  d.HALF = (int)half;
  d.QD = (int)Q;
  d.KVD = (int)KV;
  d.QKVR = (int)QKVR;
  d.max_seq = (int)c.max_seq_len;
  d.eps = c.rms_norm_eps;
  d.scale = 1.0f / sqrtf((float)c.head_dim);
  d.gelu = c.gelu ? 1 : 0;
  d.bf16 = M->bf16 ? 1 : 0;
  d.bias = M->has_bias ? 1 : 0;
  d.embed = dev + o_embed;
  d.head = dev + o_head;
  d.norm = (const float*)(dev + o_norm);
  d.rope_cos = (const float*)(dev + o_cos);
  d.rope_sin = (const float*)(dev + o_sin);
  d.layers = M->d_layers;
  return M.release();
}

// ----------------------------------------------------------------- KvCache
KvCache::~KvCache() {
  if (k) cudaFree(k);
  if (v) cudaFree(v);
  if (mask) cudaFree(mask);
}

size_t KvCache::layer_stride() const { return (size_t)model->cfg.num_kv_heads * cap * model->cfg.head_dim; }

KvCache* cache_new(const Model* m, int cap) {
  if (cap <= 0) cap = (int)m->cfg.max_seq_len;
  DEFER_CUDA(cudaSetDevice(m->device));
  std::unique_ptr<KvCache> c(new KvCache());
  c->model = m;
  c->cap = cap;
  size_t n = (size_t)m->cfg.num_layers * m->cfg.num_kv_heads * cap * m->cfg.head_dim;
  DEFER_CUDA(cudaMalloc(&c->k, std::max<size_t>(n, 1) * 4));
  DEFER_CUDA(cudaMalloc(&c->v, std::max<size_t>(n, 1) * 4));
  DEFER_CUDA(cudaMalloc(&c->mask, ((size_t)cap / 32 + 1) * 4));
  DEFER_CUDA(cudaMemset(c->mask, 0, ((size_t)cap / 32 + 1) * 4));
  return c.release();
}

void cache_copy_prefix(KvCache* dst, const KvCache* src, size_t len, cudaStream_t st) {
  const Config& c = src->model->cfg;
  if (len > (size_t)dst->cap) fail(kModel, "cache capacity exceeded");
  if (len == 0) return;
  const size_t row = (size_t)c.head_dim * 4;
  for (int kv = 0; kv < 2; kv++)
    DEFER_CUDA(cudaMemcpy2DAsync(kv ? dst->v : dst->k, (size_t)dst->cap * row, kv ? src->v : src->k,
                                 (size_t)src->cap * row, len * row, (size_t)c.num_layers * c.num_kv_heads,
                                 cudaMemcpyDeviceToDevice, st));
}

KvCache* cache_clone(const KvCache* src) {
  KvCache* c = cache_new(src->model, src->cap);
  cache_copy_prefix(c, src, src->len, src->model->stream);
  DEFER_CUDA(cudaStreamSynchronize(src->model->stream));
  c->len = src->len;
  return c;
}

void cache_download(const KvCache* c, int layer, float* keys, float* values) {
  const Config& cf = c->model->cfg;
  const size_t hd = cf.head_dim, nkv = cf.num_kv_heads, len = c->len;
  if (len == 0) return;
  DEFER_CUDA(cudaSetDevice(c->model->device));
  DEFER_CUDA(cudaStreamSynchronize(c->model->stream));
  std::vector<float> tmp(nkv * len * hd);
  for (int kv = 0; kv < 2; kv++) {
    const float* base = (kv ? c->v : c->k) + (size_t)layer * c->layer_stride();
    DEFER_CUDA(cudaMemcpy2D(tmp.data(), len * hd * 4, base, (size_t)c->cap * hd * 4, len * hd * 4, nkv,
                            cudaMemcpyDeviceToHost));
    float* out = kv ? values : keys;
    for (size_t t = 0; t < len; t++)
      for (size_t g = 0; g < nkv; g++) memcpy(out + (t * nkv + g) * hd, tmp.data() + (g * len + t) * hd, hd * 4);
  }
}

void cache_fingerprint(const KvCache* c, uint8_t out[32]) {
  const Config& cf = c->model->cfg;
  Sha256 h;
  uint64_t len = c->len;
  uint8_t lb[8];
  for (int i = 0; i < 8; i++) lb[i] = (uint8_t)(len >> (8 * i));
  h.update(lb, 8);
  std::vector<float> k(len * cf.kv_dim()), v(len * cf.kv_dim());
  for (uint32_t l = 0; l < cf.num_layers; l++) {
    cache_download(c, (int)l, k.data(), v.data());
    h.update(k.data(), k.size() * 4);  // little-endian host: the f32 bits in LE order
    h.update(v.data(), v.size() * 4);
  }
  h.finalize(out);
}

}  // namespace defer
