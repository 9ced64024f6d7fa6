// Semantic checkpoint and write-ahead-log formats, byte-identical to the
// reference (src/checkpoint.rs:4-16, src/wal.rs:8-27). All integers are
// little-endian; the 128-bit PRNG word position is carried as (lo, hi).
#pragma once
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

namespace defer {

struct U128 {
  uint64_t lo = 0, hi = 0;
  bool operator==(const U128& o) const { return lo == o.lo && hi == o.hi; }
  bool operator!=(const U128& o) const { return !(*this == o); }
};

struct Checkpoint {
  uint8_t model_signature[32] = {0};
  uint8_t base_seed[32] = {0};
  float temperature = 0.0f;
  std::vector<uint32_t> history_tokens;
  uint32_t prompt_len = 0;
  U128 rng_word_pos;

  std::vector<uint8_t> to_bytes() const;                        // checkpoint.rs:44-60
  static Checkpoint from_bytes(const uint8_t* b, size_t n);     // checkpoint.rs:62-90
  void save(const std::string& path) const;                     // checkpoint.rs:92-103
  static Checkpoint load(const std::string& path);
};

struct WalHeader {
  uint8_t model_signature[32] = {0};
  uint8_t base_seed[32] = {0};
  float temperature = 0.0f;
  uint32_t prompt_len = 0;
  U128 start_rng_word_pos;
  std::vector<uint32_t> prefix_tokens;

  std::vector<uint8_t> to_bytes() const;  // wal.rs:55-71
  static WalHeader from_checkpoint(const Checkpoint& c);
};

struct WalRecord {
  uint32_t step = 0, token = 0;
  U128 rng_word_pos;
};

constexpr size_t kWalRecordSize = 29;
void wal_record_bytes(const WalRecord& r, uint8_t out[kWalRecordSize]);  // wal.rs:94-103

struct WalLog {
  WalHeader header;
  std::vector<WalRecord> records;
  uint64_t valid_len = 0;
  bool torn_tail = false;

  static WalLog parse(const uint8_t* b, size_t n);  // wal.rs:123-194
  static WalLog read(const std::string& path);
  Checkpoint to_checkpoint() const;                 // wal.rs:197-209
};

class WalWriter {
 public:
  static WalWriter* create(const std::string& path, const WalHeader& h, bool durable);  // wal.rs:221-228
  static WalWriter* resume(const std::string& path, bool durable, WalLog* log_out);     // wal.rs:231-239
  void append(uint32_t token, U128 rng_word_pos);                                       // wal.rs:241-250
  uint32_t next_step() const { return next_step_; }
  ~WalWriter();

 private:
  WalWriter() = default;
  FILE* f_ = nullptr;
  uint32_t next_step_ = 0;
  bool durable_ = false;
};

std::vector<uint8_t> read_file(const std::string& path);

}  // namespace defer
