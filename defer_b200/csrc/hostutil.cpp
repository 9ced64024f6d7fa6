#include "hostutil.h"

#include <cctype>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "common.h"

namespace defer {

// ----------------------------------------------------------------- errors
static thread_local std::string g_last_error;
void set_last_error(const std::string& m) { g_last_error = m; }
const char* last_error() { return g_last_error.c_str(); }

// ---------------------------------------------------------------- SHA-256
// Round constants: the first 32 bits of the fractional parts of the cube
// roots of the first 64 primes (FIPS 180-4 §4.2.2).
static const uint32_t kSha256K[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

static inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

Sha256::Sha256() {
  static const uint32_t init[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                                   0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  memcpy(h_, init, sizeof(h_));
}

void Sha256::compress(const uint8_t* p) {
  uint32_t w[64];
  for (int i = 0; i < 16; i++)
    w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
  for (int i = 16; i < 64; i++) {
    uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
    uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
  for (int i = 0; i < 64; i++) {
    uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + kSha256K[i] + w[i];
    uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
    h = g;
    g = f;
    f = e;
    e = d + t1;
    d = c;
    c = b;
    b = a;
    a = t1 + t2;
  }
  h_[0] += a;
  h_[1] += b;
  h_[2] += c;
  h_[3] += d;
  h_[4] += e;
  h_[5] += f;
  h_[6] += g;
  h_[7] += h;
}

void Sha256::update(const void* data, size_t n) {
  const uint8_t* p = (const uint8_t*)data;
  total_ += n;
  if (buf_len_) {
    size_t take = 64 - buf_len_ < n ? 64 - buf_len_ : n;
    memcpy(buf_ + buf_len_, p, take);
    buf_len_ += take;
    p += take;
    n -= take;
    if (buf_len_ == 64) {
      compress(buf_);
      buf_len_ = 0;
    }
  }
  while (n >= 64) {
    compress(p);
    p += 64;
    n -= 64;
  }
  if (n) {
    memcpy(buf_, p, n);
    buf_len_ = n;
  }
}

void Sha256::finalize(uint8_t out[32]) {
  uint64_t bits = total_ * 8;
  uint8_t pad[72] = {0x80};
  size_t padlen = (buf_len_ < 56) ? 56 - buf_len_ : 120 - buf_len_;
  uint8_t len[8];
  for (int i = 0; i < 8; i++) len[i] = (uint8_t)(bits >> (56 - 8 * i));
  update(pad, padlen);
  update(len, 8);
  for (int i = 0; i < 8; i++) {
    out[4 * i] = (uint8_t)(h_[i] >> 24);
    out[4 * i + 1] = (uint8_t)(h_[i] >> 16);
    out[4 * i + 2] = (uint8_t)(h_[i] >> 8);
    out[4 * i + 3] = (uint8_t)h_[i];
  }
}

// ------------------------------------------------------------------ CRC-32
uint32_t crc32(const uint8_t* data, size_t n) {
  static uint32_t table[256];
  static bool init = false;
  if (!init) {
    for (uint32_t i = 0; i < 256; i++) {
      uint32_t c = i;
      for (int k = 0; k < 8; k++) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
      table[i] = c;
    }
    init = true;
  }
  uint32_t c = 0xFFFFFFFFu;
  for (size_t i = 0; i < n; i++) c = table[(c ^ data[i]) & 0xFF] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

// ----------------------------------------------------------------- ChaCha8
ChaCha8::ChaCha8(const uint8_t seed[32]) {
  for (int i = 0; i < 8; i++)
    key_[i] = (uint32_t)seed[4 * i] | (uint32_t)seed[4 * i + 1] << 8 | (uint32_t)seed[4 * i + 2] << 16 |
              (uint32_t)seed[4 * i + 3] << 24;
}

static inline uint32_t rotl(uint32_t x, int n) { return (x << n) | (x >> (32 - n)); }

void ChaCha8::block(uint64_t counter, uint32_t out[16]) const {
  // State: the "expand 32-byte k" constants, the key, a 64-bit block counter
  // and a 64-bit stream id (0).
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
  for (int i = 0; i < 8; i++) s[4 + i] = key_[i];
  s[12] = (uint32_t)counter;
  s[13] = (uint32_t)(counter >> 32);
  s[14] = 0;
  s[15] = 0;
  uint32_t x[16];
  memcpy(x, s, sizeof(x));
  auto qr = [&](int a, int b, int c, int d) {
    x[a] += x[b]; x[d] = rotl(x[d] ^ x[a], 16);
    x[c] += x[d]; x[b] = rotl(x[b] ^ x[c], 12);
    x[a] += x[b]; x[d] = rotl(x[d] ^ x[a], 8);
    x[c] += x[d]; x[b] = rotl(x[b] ^ x[c], 7);
  };
  for (int r = 0; r < 8; r += 2) {  // 4 double rounds = 8 rounds
    qr(0, 4, 8, 12);
    qr(1, 5, 9, 13);
    qr(2, 6, 10, 14);
    qr(3, 7, 11, 15);
    qr(0, 5, 10, 15);
    qr(1, 6, 11, 12);
    qr(2, 7, 8, 13);
    qr(3, 4, 9, 14);
  }
  for (int i = 0; i < 16; i++) out[i] = x[i] + s[i];
}

uint32_t ChaCha8::next_u32() {
  uint64_t blk = pos_ / 16;
  if (blk != cached_block_) {
    block(blk, cache_);
    cached_block_ = blk;
  }
  return cache_[pos_++ % 16];
}

void ChaCha8::words(uint64_t start, size_t n, uint32_t* out) {
  uint64_t saved = pos_;
  pos_ = start;
  for (size_t i = 0; i < n; i++) out[i] = next_u32();
  pos_ = saved;
}

void seed_from_u64(uint64_t state, uint8_t out[32]) {
  // PCG32 (XSH-RR output) advanced once per 4 seed bytes.
  const uint64_t mul = 6364136223846793005ull, inc = 11634580027462260723ull;
  for (int i = 0; i < 8; i++) {
    state = state * mul + inc;
    uint32_t xs = (uint32_t)(((state >> 18) ^ state) >> 27);
    uint32_t rot = (uint32_t)(state >> 59);
    uint32_t v = (xs >> rot) | (xs << ((32 - rot) & 31));
    for (int k = 0; k < 4; k++) out[4 * i + k] = (uint8_t)(v >> (8 * k));
  }
}

std::string to_hex(const uint8_t* b, size_t n) {
  static const char* d = "0123456789abcdef";
  std::string s(2 * n, '0');
  for (size_t i = 0; i < n; i++) {
    s[2 * i] = d[b[i] >> 4];
    s[2 * i + 1] = d[b[i] & 15];
  }
  return s;
}

// -------------------------------------------------------------------- JSON
const Json* Json::get(const std::string& k) const {
  if (kind != Object) return nullptr;
  for (auto& kv : obj)
    if (kv.first == k) return &kv.second;
  return nullptr;
}

bool Json::as_u64(uint64_t* out) const {
  if (kind != Number || num < 0 || std::floor(num) != num || num > 1.8446744073709552e19) return false;
  *out = (uint64_t)num;
  return true;
}

bool Json::as_f64(double* out) const {
  if (kind != Number) return false;
  *out = num;
  return true;
}

namespace {
struct Parser {
  const std::string& s;
  size_t i = 0;
  [[noreturn]] void err(const char* m) { fail(kParse, std::string("JSON: ") + m + " at byte " + std::to_string(i)); }
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) i++;
  }
  void put_utf8(std::string& o, uint32_t cp) {
    if (cp < 0x80) {
      o += (char)cp;
    } else if (cp < 0x800) {
      o += (char)(0xC0 | (cp >> 6));
      o += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += (char)(0xE0 | (cp >> 12));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    } else {
      o += (char)(0xF0 | (cp >> 18));
      o += (char)(0x80 | ((cp >> 12) & 0x3F));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (i + 4 > s.size()) err("bad unicode escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; k++) {
      char c = s[i++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else err("bad unicode escape");
    }
    return v;
  }
  std::string string() {
    if (i >= s.size() || s[i] != '"') err("expected string");
    i++;
    std::string o;
    for (;;) {
      if (i >= s.size()) err("unterminated string");
      char c = s[i++];
      if (c == '"') break;
      if (c != '\\') {
        o += c;
        continue;
      }
      if (i >= s.size()) err("unterminated escape");
      char e = s[i++];
      switch (e) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00 && i + 6 <= s.size() && s[i] == '\\' && s[i + 1] == 'u') {
            i += 2;
            uint32_t lo = hex4();
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(o, cp);
          break;
        }
        default: err("bad escape");
      }
    }
    return o;
  }
  Json value(int depth) {
    if (depth > 256) err("nesting too deep");
    ws();
    if (i >= s.size()) err("unexpected end");
    Json v;
    char c = s[i];
    if (c == '{') {
      v.kind = Json::Object;
      i++;
      ws();
      if (i < s.size() && s[i] == '}') {
        i++;
        return v;
      }
      for (;;) {
        ws();
        std::string k = string();
        ws();
        if (i >= s.size() || s[i] != ':') err("expected ':'");
        i++;
        Json x = value(depth + 1);
        v.obj.emplace_back(std::move(k), std::move(x));
        ws();
        if (i < s.size() && s[i] == ',') {
          i++;
          continue;
        }
        if (i < s.size() && s[i] == '}') {
          i++;
          break;
        }
        err("expected ',' or '}'");
      }
    } else if (c == '[') {
      v.kind = Json::Array;
      i++;
      ws();
      if (i < s.size() && s[i] == ']') {
        i++;
        return v;
      }
      for (;;) {
        v.arr.push_back(value(depth + 1));
        ws();
        if (i < s.size() && s[i] == ',') {
          i++;
          continue;
        }
        if (i < s.size() && s[i] == ']') {
          i++;
          break;
        }
        err("expected ',' or ']'");
      }
    } else if (c == '"') {
      v.kind = Json::String;
      v.str = string();
    } else if (s.compare(i, 4, "true") == 0) {
      v.kind = Json::Bool;
      v.b = true;
      i += 4;
    } else if (s.compare(i, 5, "false") == 0) {
      v.kind = Json::Bool;
      i += 5;
    } else if (s.compare(i, 4, "null") == 0) {
      i += 4;
    } else {
      size_t st = i;
      if (s[i] == '-') i++;
      while (i < s.size() && (isdigit((unsigned char)s[i]) || s[i] == '.' || s[i] == 'e' || s[i] == 'E' ||
                              s[i] == '+' || s[i] == '-'))
        i++;
      if (st == i) err("unexpected character");
      v.kind = Json::Number;
      char* end = nullptr;
      std::string t = s.substr(st, i - st);
      v.num = strtod(t.c_str(), &end);
      if (!end || *end) err("bad number");
    }
    return v;
  }
};
}  // namespace

Json parse_json(const std::string& src) {
  Parser p{src};
  Json v = p.value(0);
  p.ws();
  if (p.i != src.size()) p.err("trailing characters");
  return v;
}

}  // namespace defer
