// Host-side byte/integer utilities of the engine: SHA-256 (model signature,
// KV fingerprint), CRC-32 (WAL / checkpoint integrity), ChaCha8 keystream
// (the sampler's PRNG), and a small order-preserving JSON reader for
// safetensors headers and model configs.
#pragma once
#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace defer {

// FIPS 180-4 SHA-256, streaming (reference: src/sha256.rs:16-120).
class Sha256 {
 public:
  Sha256();
  void update(const void* data, size_t n);
  void finalize(uint8_t out[32]);

 private:
  void compress(const uint8_t* block);
  uint32_t h_[8];
  uint8_t buf_[64];
  size_t buf_len_ = 0;
  uint64_t total_ = 0;
};

// IEEE reflected CRC-32, polynomial 0xEDB88320 (reference: src/crc32.rs:22-28).
uint32_t crc32(const uint8_t* data, size_t n);

// ChaCha with 8 rounds as a word stream: 32-byte key, 64-bit block counter
// from 0, stream id 0, keystream consumed as little-endian u32 words
// (rand_chacha 0.3.1 ChaCha8Rng as used at engine.rs:51 / sampler.rs:92).
// word_pos() is the number of words consumed (ChaCha8Rng::get_word_pos).
class ChaCha8 {
 public:
  explicit ChaCha8(const uint8_t seed[32]);
  uint32_t next_u32();
  uint64_t word_pos() const { return pos_; }
  void set_word_pos(uint64_t p) { pos_ = p; }
  // Words [start, start + n) of the stream without moving the position.
  void words(uint64_t start, size_t n, uint32_t* out);

 private:
  void block(uint64_t counter, uint32_t out[16]) const;
  uint32_t key_[8];
  uint64_t pos_ = 0;
  uint64_t cached_block_ = ~0ull;
  uint32_t cache_[16];
};

// rand_core 0.6.4 SeedableRng::seed_from_u64 (engine.rs:19-21).
void seed_from_u64(uint64_t seed, uint8_t out[32]);

// Minimal JSON value (objects keep insertion order).
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  const Json* get(const std::string& k) const;
  bool as_u64(uint64_t* out) const;
  bool as_f64(double* out) const;
  const std::string* as_str() const { return kind == String ? &str : nullptr; }
};

Json parse_json(const std::string& src);  // throws Error(kParse)

std::string to_hex(const uint8_t* b, size_t n);

}  // namespace defer
