#include "formats.h"

#include <unistd.h>

#include <cerrno>
#include <cstring>

#include "common.h"
#include "hostutil.h"

namespace defer {

static void put32(std::vector<uint8_t>& b, uint32_t v) {
  for (int i = 0; i < 4; i++) b.push_back((uint8_t)(v >> (8 * i)));
}
static void put64(std::vector<uint8_t>& b, uint64_t v) {
  for (int i = 0; i < 8; i++) b.push_back((uint8_t)(v >> (8 * i)));
}
static void put128(std::vector<uint8_t>& b, U128 v) {
  put64(b, v.lo);
  put64(b, v.hi);
}
static uint32_t get32(const uint8_t* p) {
  return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}
static uint64_t get64(const uint8_t* p) { return (uint64_t)get32(p) | (uint64_t)get32(p + 4) << 32; }
static U128 get128(const uint8_t* p) { return U128{get64(p), get64(p + 8)}; }
static uint32_t fbits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static float bitsf(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

std::vector<uint8_t> read_file(const std::string& path) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) fail(kIo, "cannot open " + path + ": " + strerror(errno));
  std::vector<uint8_t> out;
  uint8_t buf[1 << 16];
  size_t n;
  while ((n = fread(buf, 1, sizeof(buf), f)) > 0) out.insert(out.end(), buf, buf + n);
  bool bad = ferror(f);
  fclose(f);
  if (bad) fail(kIo, "read error on " + path);
  return out;
}

// -------------------------------------------------------------- checkpoint
static const uint8_t kCkptMagic[8] = {'D', 'E', 'F', 'E', 'R', 'C', 'K', 'P'};
static const uint8_t kWalMagic[8] = {'D', 'E', 'F', 'E', 'R', 'W', 'A', 'L'};

std::vector<uint8_t> Checkpoint::to_bytes() const {
  std::vector<uint8_t> b(kCkptMagic, kCkptMagic + 8);
  b.reserve(112 + 4 * history_tokens.size());
  put32(b, 1);
  b.insert(b.end(), model_signature, model_signature + 32);
  b.insert(b.end(), base_seed, base_seed + 32);
  put32(b, fbits(temperature));
  put32(b, prompt_len);
  put128(b, rng_word_pos);
  put64(b, history_tokens.size());
  for (uint32_t t : history_tokens) put32(b, t);
  put32(b, crc32(b.data(), b.size()));
  return b;
}

Checkpoint Checkpoint::from_bytes(const uint8_t* b, size_t n) {
  const size_t fixed = 8 + 4 + 32 + 32 + 4 + 4 + 16 + 8;
  if (n < fixed + 4 || memcmp(b, kCkptMagic, 8) != 0) fail(kCheckpoint, "not a defer checkpoint");
  size_t body = n - 4;
  if (crc32(b, body) != get32(b + body)) fail(kCheckpoint, "checksum mismatch (file corrupt)");
  if (get32(b + 8) != 1) fail(kCheckpoint, "unsupported checkpoint version");
  Checkpoint c;
  memcpy(c.model_signature, b + 12, 32);
  memcpy(c.base_seed, b + 44, 32);
  c.temperature = bitsf(get32(b + 76));
  c.prompt_len = get32(b + 80);
  c.rng_word_pos = get128(b + 84);
  uint64_t cnt = get64(b + 100);
  if (cnt > (body - fixed) / 4 || body != fixed + 4 * cnt) fail(kCheckpoint, "length mismatch");
  c.history_tokens.resize(cnt);
  for (uint64_t i = 0; i < cnt; i++) c.history_tokens[i] = get32(b + fixed + 4 * i);
  if (c.prompt_len > cnt) fail(kCheckpoint, "prompt_len exceeds history length");
  return c;
}

void Checkpoint::save(const std::string& path) const {
  // Write-then-rename so a crash never leaves a half-written file
  // (Path::with_extension("ckpt.tmp") semantics).
  std::string tmp = path;
  size_t slash = tmp.find_last_of('/');
  size_t dot = tmp.find_last_of('.');
  // a leading dot starts the name, not an extension (".hidden" -> ".hidden.ckpt.tmp")
  const size_t name0 = slash == std::string::npos ? 0 : slash + 1;
  if (dot != std::string::npos && dot > name0) tmp = tmp.substr(0, dot);
  tmp += ".ckpt.tmp";
  std::vector<uint8_t> b = to_bytes();
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) fail(kIo, "cannot create " + tmp + ": " + strerror(errno));
  size_t w = fwrite(b.data(), 1, b.size(), f);
  bool ok = w == b.size() && fflush(f) == 0 && fsync(fileno(f)) == 0;
  fclose(f);
  if (!ok) fail(kIo, "write error on " + tmp);
  if (rename(tmp.c_str(), path.c_str()) != 0) fail(kIo, "rename to " + path + " failed: " + strerror(errno));
}

Checkpoint Checkpoint::load(const std::string& path) {
  std::vector<uint8_t> b = read_file(path);
  return from_bytes(b.data(), b.size());
}

// --------------------------------------------------------------------- WAL
std::vector<uint8_t> WalHeader::to_bytes() const {
  std::vector<uint8_t> b(kWalMagic, kWalMagic + 8);
  put32(b, 1);
  b.insert(b.end(), model_signature, model_signature + 32);
  b.insert(b.end(), base_seed, base_seed + 32);
  put32(b, fbits(temperature));
  put32(b, prompt_len);
  put128(b, start_rng_word_pos);
  put32(b, (uint32_t)prefix_tokens.size());
  for (uint32_t t : prefix_tokens) put32(b, t);
  put32(b, crc32(b.data(), b.size()));
  return b;
}

WalHeader WalHeader::from_checkpoint(const Checkpoint& c) {
  WalHeader h;
  memcpy(h.model_signature, c.model_signature, 32);
  memcpy(h.base_seed, c.base_seed, 32);
  h.temperature = c.temperature;
  h.prompt_len = c.prompt_len;
  h.start_rng_word_pos = c.rng_word_pos;
  h.prefix_tokens = c.history_tokens;
  return h;
}

void wal_record_bytes(const WalRecord& r, uint8_t out[kWalRecordSize]) {
  out[0] = 0x01;
  for (int i = 0; i < 4; i++) out[1 + i] = (uint8_t)(r.step >> (8 * i));
  for (int i = 0; i < 4; i++) out[5 + i] = (uint8_t)(r.token >> (8 * i));
  for (int i = 0; i < 8; i++) out[9 + i] = (uint8_t)(r.rng_word_pos.lo >> (8 * i));
  for (int i = 0; i < 8; i++) out[17 + i] = (uint8_t)(r.rng_word_pos.hi >> (8 * i));
  uint32_t c = crc32(out, 25);
  for (int i = 0; i < 4; i++) out[25 + i] = (uint8_t)(c >> (8 * i));
}

static U128 add_u128(U128 a, uint64_t b) {
  U128 r{a.lo + b, a.hi};
  if (r.lo < a.lo) r.hi++;
  return r;
}

static std::string u128_str(U128 v) {
  if (v.hi == 0) return std::to_string(v.lo);
  unsigned __int128 x = ((unsigned __int128)v.hi << 64) | v.lo;
  std::string s;
  while (x) {
    s.insert(s.begin(), (char)('0' + (int)(x % 10)));
    x /= 10;
  }
  return s;
}

WalLog WalLog::parse(const uint8_t* b, size_t n) {
  const size_t fixed = 8 + 4 + 32 + 32 + 4 + 4 + 16 + 4;
  if (n < fixed + 4 || memcmp(b, kWalMagic, 8) != 0) fail(kWal, "not a defer WAL");
  if (get32(b + 8) != 1) fail(kWal, "unsupported WAL version");
  WalLog log;
  WalHeader& h = log.header;
  memcpy(h.model_signature, b + 12, 32);
  memcpy(h.base_seed, b + 44, 32);
  h.temperature = bitsf(get32(b + 76));
  h.prompt_len = get32(b + 80);
  h.start_rng_word_pos = get128(b + 84);
  uint32_t cnt = get32(b + 100);
  size_t header_end = fixed + 4 * (size_t)cnt;
  if (n < header_end + 4) fail(kWal, "truncated WAL header");
  h.prefix_tokens.resize(cnt);
  for (uint32_t i = 0; i < cnt; i++) h.prefix_tokens[i] = get32(b + fixed + 4 * (size_t)i);
  if (crc32(b, header_end) != get32(b + header_end)) fail(kWal, "WAL header checksum mismatch");
  if (h.prompt_len > cnt) fail(kWal, "prompt_len exceeds prefix length");

  size_t off = header_end + 4;
  uint32_t expect_step = cnt;
  U128 expect_rng = h.start_rng_word_pos;
  uint64_t wps = h.temperature == 0.0f ? 0 : 1;
  while (off < n) {
    if (n - off < kWalRecordSize) {
      log.torn_tail = true;
      break;
    }
    const uint8_t* r = b + off;
    if (r[0] != 0x01 || crc32(r, 25) != get32(r + 25)) {
      log.torn_tail = true;
      break;
    }
    WalRecord rec{get32(r + 1), get32(r + 5), get128(r + 9)};
    expect_rng = add_u128(expect_rng, wps);
    if (rec.step != expect_step || rec.rng_word_pos != expect_rng)
      fail(kWal, "record " + std::to_string(log.records.size()) + " is inconsistent (step " +
                     std::to_string(rec.step) + " / rng " + u128_str(rec.rng_word_pos) + ", expected " +
                     std::to_string(expect_step) + " / " + u128_str(expect_rng) + ")");
    expect_step++;
    log.records.push_back(rec);
    off += kWalRecordSize;
  }
  log.valid_len = off;
  return log;
}

WalLog WalLog::read(const std::string& path) {
  std::vector<uint8_t> b = read_file(path);
  return parse(b.data(), b.size());
}

Checkpoint WalLog::to_checkpoint() const {
  Checkpoint c;
  memcpy(c.model_signature, header.model_signature, 32);
  memcpy(c.base_seed, header.base_seed, 32);
  c.temperature = header.temperature;
  c.history_tokens = header.prefix_tokens;
  for (auto& r : records) c.history_tokens.push_back(r.token);
  c.prompt_len = header.prompt_len;
  c.rng_word_pos = records.empty() ? header.start_rng_word_pos : records.back().rng_word_pos;
  return c;
}

WalWriter* WalWriter::create(const std::string& path, const WalHeader& h, bool durable) {
  FILE* f = fopen(path.c_str(), "wb");
  if (!f) fail(kIo, "cannot create " + path + ": " + strerror(errno));
  std::vector<uint8_t> b = h.to_bytes();
  bool ok = fwrite(b.data(), 1, b.size(), f) == b.size() && fflush(f) == 0 && fsync(fileno(f)) == 0;
  if (!ok) {
    fclose(f);
    fail(kIo, "write error on " + path);
  }
  WalWriter* w = new WalWriter();
  w->f_ = f;
  w->next_step_ = (uint32_t)h.prefix_tokens.size();
  w->durable_ = durable;
  return w;
}

WalWriter* WalWriter::resume(const std::string& path, bool durable, WalLog* log_out) {
  WalLog log = WalLog::read(path);
  if (truncate(path.c_str(), (off_t)log.valid_len) != 0) fail(kIo, "cannot truncate " + path + ": " + strerror(errno));
  FILE* f = fopen(path.c_str(), "ab");
  if (!f) fail(kIo, "cannot open " + path + ": " + strerror(errno));
  fsync(fileno(f));
  WalWriter* w = new WalWriter();
  w->f_ = f;
  w->next_step_ = (uint32_t)(log.header.prefix_tokens.size() + log.records.size());
  w->durable_ = durable;
  if (log_out) *log_out = std::move(log);
  return w;
}

void WalWriter::append(uint32_t token, U128 rng_word_pos) {
  uint8_t rec[kWalRecordSize];
  wal_record_bytes(WalRecord{next_step_, token, rng_word_pos}, rec);
  if (fwrite(rec, 1, sizeof(rec), f_) != sizeof(rec) || fflush(f_) != 0) fail(kIo, "WAL append failed");
  if (durable_ && fdatasync(fileno(f_)) != 0) fail(kIo, "WAL fdatasync failed");
  next_step_++;
}

WalWriter::~WalWriter() {
  if (f_) fclose(f_);
}

}  // namespace defer
