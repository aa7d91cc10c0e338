// overlay.cpp — the INT8 overlay loader: QuantizedWeights::{load,get}
// (src/cpu/quantized.rs:239-370) over the safetensors reader it stands on
// (Checkpoint::open / sha256 / tensor, src/checkpoint.rs:101-217).
//
// Every check of the reference runs on the host, in the reference's order, and
// fails with the same OcrError variant; only a fully validated overlay is
// uploaded.  The upload is one device allocation holding every matrix (each
// weight and scale array 256-byte aligned, as the tensor-core kernels' TMA
// maps need), filled through two pinned staging buffers so that reading the
// mapped file overlaps the copies; get() returns non-owning uocr_q8 views
// into it.
//
// Pieces written here from their public definitions:
//   - SHA-256 (FIPS 180-4), with the round constants derived at start-up from
//     their definition (the first 32 fractional bits of the cube roots of the
//     first 64 primes, and of the square roots of the first 8 for the initial
//     state), by exact integer root extraction;
//   - a JSON reader with the acceptance rules of the reference's typed
//     decoding (serde_json into u32/usize/String/[usize; 2]/maps): integers
//     for the numeric fields, strings for the metadata values, unknown object
//     keys ignored, the later of two equal keys kept.
#include <cpuid.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <immintrin.h>
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
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "../../include/uocr_q8.h"
#include "handles.h"

namespace uocr {
int record_error(int status, const char* message);  // capi.cu
}

namespace {

using uocr::record_error;

int err(int status, const std::string& m) { return record_error(status, m.c_str()); }
int format_err(const std::string& m) { return err(UOCR_ERR_FORMAT, "invalid checkpoint: " + m); }
int json_err(const std::string& m) { return err(UOCR_ERR_JSON, "JSON: " + m); }
int io_err(const std::string& what, int e) {
  return err(UOCR_ERR_IO, "I/O: " + what + ": " + std::strerror(e));
}

// ---- SHA-256 (FIPS 180-4) -----------------------------------------------------

using u128 = unsigned __int128;

// Largest x with x^k <= v (k = 2 or 3), by bisection on exact integers.
uint64_t iroot(u128 v, int k, uint64_t hi) {
  uint64_t lo = 0;
  while (lo < hi) {
    uint64_t mid = lo + (hi - lo + 1) / 2;
    u128 p = static_cast<u128>(mid) * mid;
    if (k == 3) p *= mid;
    if (p <= v) lo = mid; else hi = mid - 1;
  }
  return lo;
}

struct ShaConstants {
  uint32_t k[64];
  uint32_t h0[8];
  ShaConstants() {
    int primes[64], n = 0;
    for (int c = 2; n < 64; ++c) {
      bool prime = true;
      for (int d = 2; d * d <= c; ++d) if (c % d == 0) { prime = false; break; }
      if (prime) primes[n++] = c;
    }
    // frac(p^(1/3)) * 2^32 = floor(cbrt(p * 2^96)) mod 2^32 (p < 2^9, root < 2^35)
    for (int i = 0; i < 64; ++i)
      k[i] = static_cast<uint32_t>(iroot(static_cast<u128>(primes[i]) << 96, 3, 1ull << 36));
    // frac(p^(1/2)) * 2^32 = floor(sqrt(p * 2^64)) mod 2^32
    for (int i = 0; i < 8; ++i)
      h0[i] = static_cast<uint32_t>(iroot(static_cast<u128>(primes[i]) << 64, 2, 1ull << 40));
  }
};

const ShaConstants& sha_constants() {
  static const ShaConstants c;
  return c;
}

inline uint32_t rotr(uint32_t x, int r) { return (x >> r) | (x << (32 - r)); }

// The x86 SHA extensions: SHA256RNDS2 takes the state as {A,B,E,F} and
// {C,D,G,H} (lane 3 first) and two rounds' W+K in the low lanes of its third
// operand; SHA256MSG1/MSG2 compute four schedule words from the previous 16.
bool have_sha_ni() {
  unsigned a, b, c, d;
  if (!__get_cpuid(1, &a, &b, &c, &d)) return false;
  bool ssse3 = c & (1u << 9), sse41 = c & (1u << 19);
  if (!__get_cpuid_count(7, 0, &a, &b, &c, &d)) return false;
  return ssse3 && sse41 && (b & (1u << 29));
}

__attribute__((target("sha,sse4.1,ssse3")))
void blocks_sha_ni(uint32_t h[8], const uint32_t k[64], const uint8_t* p, size_t nblocks) {
  const __m128i bswap = _mm_set_epi64x(0x0c0d0e0f08090a0bll, 0x0405060700010203ll);
  // h[0..3] = a b c d, h[4..7] = e f g h  ->  ABEF, CDGH
  __m128i t = _mm_shuffle_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(h)), 0xB1);
  __m128i s1 = _mm_shuffle_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(h + 4)), 0x1B);
  __m128i s0 = _mm_alignr_epi8(t, s1, 8);
  s1 = _mm_blend_epi16(s1, t, 0xF0);
  for (; nblocks; --nblocks, p += 64) {
    const __m128i abef = s0, cdgh = s1;
    __m128i m[4];
    for (int g = 0; g < 16; ++g) {
      __m128i& cur = m[g & 3];
      if (g < 4) {
        cur = _mm_shuffle_epi8(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p + 16 * g)), bswap);
      } else {
        // W[t] = s1(W[t-2]) + W[t-7] + s0(W[t-15]) + W[t-16], four at a time
        __m128i x = _mm_sha256msg1_epu32(cur, m[(g + 1) & 3]);
        x = _mm_add_epi32(x, _mm_alignr_epi8(m[(g + 3) & 3], m[(g + 2) & 3], 4));
        cur = _mm_sha256msg2_epu32(x, m[(g + 3) & 3]);
      }
      __m128i wk = _mm_add_epi32(cur, _mm_loadu_si128(reinterpret_cast<const __m128i*>(k + 4 * g)));
      s1 = _mm_sha256rnds2_epu32(s1, s0, wk);
      s0 = _mm_sha256rnds2_epu32(s0, s1, _mm_shuffle_epi32(wk, 0x0E));
    }
    s0 = _mm_add_epi32(s0, abef);
    s1 = _mm_add_epi32(s1, cdgh);
  }
  t = _mm_shuffle_epi32(s0, 0x1B);   // a b e f
  s1 = _mm_shuffle_epi32(s1, 0xB1);  // g h c d
  _mm_storeu_si128(reinterpret_cast<__m128i*>(h), _mm_blend_epi16(t, s1, 0xF0));
  _mm_storeu_si128(reinterpret_cast<__m128i*>(h + 4), _mm_alignr_epi8(s1, t, 8));
}

void blocks_portable(uint32_t h_[8], const uint32_t k[64], const uint8_t* p, size_t nblocks) {
  for (; nblocks; --nblocks, p += 64) {
    uint32_t w[64];
    for (int t = 0; t < 16; ++t)
      w[t] = (uint32_t(p[4 * t]) << 24) | (uint32_t(p[4 * t + 1]) << 16) |
             (uint32_t(p[4 * t + 2]) << 8) | uint32_t(p[4 * t + 3]);
    for (int t = 16; t < 64; ++t) {
      uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
      uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
      w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
    for (int t = 0; t < 64; ++t) {
      uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[t] + w[t];
      uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h_[0] += a; h_[1] += b; h_[2] += c; h_[3] += d;
    h_[4] += e; h_[5] += f; h_[6] += g; h_[7] += h;
  }
}

// UOCR_SHA_PORTABLE=1 forces the portable rounds (for testing both forms).
bool use_sha_ni() {
  static const bool v = [] {
    const char* e = std::getenv("UOCR_SHA_PORTABLE");
    return !(e && *e == '1') && have_sha_ni();
  }();
  return v;
}

class Sha256 {
 public:
  Sha256() : c_(sha_constants()) { std::memcpy(h_, c_.h0, sizeof h_); }

  void update(const uint8_t* p, size_t n) {
    total_ += n;
    if (fill_) {
      size_t take = std::min(n, sizeof buf_ - fill_);
      std::memcpy(buf_ + fill_, p, take);
      fill_ += take; p += take; n -= take;
      if (fill_ < sizeof buf_) return;
      blocks(buf_, 1);
      fill_ = 0;
    }
    blocks(p, n / 64);
    p += n / 64 * 64;
    n %= 64;
    std::memcpy(buf_, p, n);
    fill_ = n;
  }

  std::string hex() {
    uint64_t bits = total_ * 8;
    uint8_t pad[72] = {0x80};
    size_t padn = (fill_ < 56 ? 56 : 120) - fill_;
    for (int i = 0; i < 8; ++i) pad[padn + i] = static_cast<uint8_t>(bits >> (56 - 8 * i));
    update(pad, padn + 8);
    static const char* digits = "0123456789abcdef";
    std::string out(64, '0');
    for (int i = 0; i < 8; ++i)
      for (int j = 0; j < 8; ++j) out[8 * i + j] = digits[(h_[i] >> (28 - 4 * j)) & 15];
    return out;
  }

 private:
  void blocks(const uint8_t* p, size_t n) {
    if (!n) return;
    if (use_sha_ni()) blocks_sha_ni(h_, c_.k, p, n);
    else blocks_portable(h_, c_.k, p, n);
  }

  const ShaConstants& c_;
  uint32_t h_[8];
  uint8_t buf_[64];
  size_t fill_ = 0;
  uint64_t total_ = 0;
};

// ---- JSON ----------------------------------------------------------------------

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool boolean = false;
  bool is_uint = false;  // a non-negative integer literal that fits 64 bits
  bool dup_keys = false;  // an object in which a key appeared twice
  uint64_t uint = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;  // keys unique, later value kept

  const Json* find(const std::string& key) const {
    for (auto& kv : obj) if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class JsonReader {
 public:
  JsonReader(const char* p, size_t n) : p_(p), end_(p + n) {}

  // The whole input as one value (surrounding white space allowed); the
  // input must be UTF-8.
  bool document(Json* out, std::string* why) {
    if (!valid_utf8()) { *why = "invalid unicode code point"; return false; }
    skip();
    if (!value(out, 0)) { *why = why_; return false; }
    skip();
    if (p_ != end_) { *why = "trailing characters"; return false; }
    return true;
  }

 private:
  bool valid_utf8() const {
    const auto* q = reinterpret_cast<const unsigned char*>(p_);
    const auto* e = reinterpret_cast<const unsigned char*>(end_);
    while (q < e) {
      unsigned c = *q;
      int n = c < 0x80 ? 0 : (c >> 5) == 6 ? 1 : (c >> 4) == 14 ? 2 : (c >> 3) == 30 ? 3 : -1;
      if (n < 0 || e - q <= n) return false;
      uint32_t cp = n == 0 ? c : n == 1 ? (c & 31) : n == 2 ? (c & 15) : (c & 7);
      for (int i = 1; i <= n; ++i) {
        if ((q[i] & 0xC0) != 0x80) return false;
        cp = (cp << 6) | (q[i] & 63);
      }
      static const uint32_t min_cp[4] = {0, 0x80, 0x800, 0x10000};
      if (cp < min_cp[n] || cp > 0x10FFFF || (cp >= 0xD800 && cp < 0xE000)) return false;
      q += n + 1;
    }
    return true;
  }

  void skip() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool fail(const char* m) { why_ = m; return false; }
  bool literal(const char* word) {
    size_t n = std::strlen(word);
    if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, word, n)) return fail("expected value");
    p_ += n;
    return true;
  }

  bool value(Json* v, int depth) {
    if (depth > 128) return fail("recursion limit exceeded");
    if (p_ >= end_) return fail("EOF while parsing a value");
    switch (*p_) {
      case '{': return object(v, depth);
      case '[': return array(v, depth);
      case '"': v->kind = Json::String; return string(&v->str);
      case 't': v->kind = Json::Bool; v->boolean = true; return literal("true");
      case 'f': v->kind = Json::Bool; v->boolean = false; return literal("false");
      case 'n': v->kind = Json::Null; return literal("null");
      default: return number(v);
    }
  }

  bool object(Json* v, int depth) {
    v->kind = Json::Object;
    ++p_;
    skip();
    if (p_ < end_ && *p_ == '}') { ++p_; return true; }
    for (;;) {
      skip();
      if (p_ >= end_ || *p_ != '"') return fail("key must be a string");
      std::string key;
      if (!string(&key)) return false;
      skip();
      if (p_ >= end_ || *p_ != ':') return fail("expected `:`");
      ++p_;
      skip();
      Json item;
      if (!value(&item, depth + 1)) return false;
      bool replaced = false;
      for (auto& kv : v->obj)
        if (kv.first == key) { kv.second = std::move(item); replaced = v->dup_keys = true; break; }
      if (!replaced) v->obj.emplace_back(std::move(key), std::move(item));
      skip();
      if (p_ < end_ && *p_ == ',') { ++p_; continue; }
      if (p_ < end_ && *p_ == '}') { ++p_; return true; }
      return fail("expected `,` or `}`");
    }
  }

  bool array(Json* v, int depth) {
    v->kind = Json::Array;
    ++p_;
    skip();
    if (p_ < end_ && *p_ == ']') { ++p_; return true; }
    for (;;) {
      skip();
      Json item;
      if (!value(&item, depth + 1)) return false;
      v->arr.push_back(std::move(item));
      skip();
      if (p_ < end_ && *p_ == ',') { ++p_; continue; }
      if (p_ < end_ && *p_ == ']') { ++p_; return true; }
      return fail("expected `,` or `]`");
    }
  }

  static void utf8(uint32_t c, std::string* s) {
    if (c < 0x80) {
      s->push_back(static_cast<char>(c));
    } else if (c < 0x800) {
      s->push_back(static_cast<char>(0xC0 | (c >> 6)));
      s->push_back(static_cast<char>(0x80 | (c & 63)));
    } else if (c < 0x10000) {
      s->push_back(static_cast<char>(0xE0 | (c >> 12)));
      s->push_back(static_cast<char>(0x80 | ((c >> 6) & 63)));
      s->push_back(static_cast<char>(0x80 | (c & 63)));
    } else {
      s->push_back(static_cast<char>(0xF0 | (c >> 18)));
      s->push_back(static_cast<char>(0x80 | ((c >> 12) & 63)));
      s->push_back(static_cast<char>(0x80 | ((c >> 6) & 63)));
      s->push_back(static_cast<char>(0x80 | (c & 63)));
    }
  }

  bool hex4(uint32_t* out) {
    if (end_ - p_ < 4) return fail("EOF while parsing a string");
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else return fail("invalid escape");
    }
    *out = v;
    return true;
  }

  bool string(std::string* s) {
    ++p_;  // opening quote
    for (;;) {
      if (p_ >= end_) return fail("EOF while parsing a string");
      unsigned char c = static_cast<unsigned char>(*p_++);
      if (c == '"') return true;
      if (c < 0x20) return fail("control character while parsing a string");
      if (c != '\\') { s->push_back(static_cast<char>(c)); continue; }
      if (p_ >= end_) return fail("EOF while parsing a string");
      char e = *p_++;
      switch (e) {
        case '"': s->push_back('"'); break;
        case '\\': s->push_back('\\'); break;
        case '/': s->push_back('/'); break;
        case 'b': s->push_back('\b'); break;
        case 'f': s->push_back('\f'); break;
        case 'n': s->push_back('\n'); break;
        case 'r': s->push_back('\r'); break;
        case 't': s->push_back('\t'); break;
        case 'u': {
          uint32_t u;
          if (!hex4(&u)) return false;
          if (u >= 0xD800 && u < 0xDC00) {  // high surrogate: a low one must follow
            uint32_t lo;
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return fail("lone leading surrogate");
            p_ += 2;
            if (!hex4(&lo)) return false;
            if (lo < 0xDC00 || lo >= 0xE000) return fail("lone leading surrogate");
            u = 0x10000 + ((u - 0xD800) << 10) + (lo - 0xDC00);
          } else if (u >= 0xDC00 && u < 0xE000) {
            return fail("lone trailing surrogate");
          }
          utf8(u, s);
          break;
        }
        default: return fail("invalid escape");
      }
    }
  }

  // RFC 8259 number grammar; non-negative integers that fit 64 bits are kept.
  bool number(Json* v) {
    v->kind = Json::Number;
    const char* start = p_;
    bool neg = false, integral = true;
    if (*p_ == '-') { neg = true; ++p_; }
    if (p_ >= end_ || *p_ < '0' || *p_ > '9') return fail("expected value");
    if (*p_ == '0') {
      ++p_;
    } else {
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    const char* int_end = p_;
    if (p_ < end_ && *p_ == '.') {
      integral = false;
      ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return fail("invalid number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      integral = false;
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return fail("invalid number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (integral && !neg) {
      uint64_t u = 0;
      bool fits = true;
      for (const char* q = start; q < int_end; ++q) {
        uint64_t d = static_cast<uint64_t>(*q - '0');
        if (u > (UINT64_MAX - d) / 10) { fits = false; break; }
        u = u * 10 + d;
      }
      v->is_uint = fits;
      v->uint = u;
    }
    return true;
  }

  const char* p_;
  const char* end_;
  std::string why_;
};

// Typed reads with the reference's decoding rules.
bool as_uint(const Json* v, uint64_t max, uint64_t* out) {
  if (!v || v->kind != Json::Number || !v->is_uint || v->uint > max) return false;
  *out = v->uint;
  return true;
}

// ---- mapped files ------------------------------------------------------------------

struct MappedFile {
  int fd = -1;
  const uint8_t* data = nullptr;
  size_t size = 0;
  ~MappedFile() {
    if (data && size) munmap(const_cast<uint8_t*>(data), size);
    if (fd >= 0) close(fd);
  }
  int open(const std::string& path) {
    fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return io_err(path, errno);
    struct stat st;
    if (fstat(fd, &st) != 0) return io_err(path, errno);
    size = static_cast<size_t>(st.st_size);
    if (size) {
      void* p = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
      if (p == MAP_FAILED) return io_err(path, errno);
      data = static_cast<const uint8_t*>(p);
    }
    return UOCR_OK;
  }
};

int read_file(const std::string& path, std::string* out) {
  MappedFile f;
  if (int st = f.open(path)) return st;
  out->assign(reinterpret_cast<const char*>(f.data), f.size);
  return UOCR_OK;
}

// Path::with_extension: the file name's last extension replaced, or added.
std::string with_extension(const std::string& path, const char* ext) {
  size_t slash = path.find_last_of('/');
  size_t name = slash == std::string::npos ? 0 : slash + 1;
  size_t dot = path.find_last_of('.');
  std::string stem = path;
  if (dot != std::string::npos && dot > name && path.compare(name, std::string::npos, "..") != 0)
    stem = path.substr(0, dot);
  return stem + "." + ext;
}

// ---- safetensors checkpoint (src/checkpoint.rs:13-31, 101-166) -------------------------

enum class DType { BF16, F16, F32, I64, I8 };

bool parse_dtype(const Json* v, DType* d) {
  if (!v || v->kind != Json::String) return false;
  static const std::pair<const char*, DType> names[] = {
      {"BF16", DType::BF16}, {"F16", DType::F16}, {"F32", DType::F32},
      {"I64", DType::I64},   {"I8", DType::I8}};
  for (auto& n : names) if (v->str == n.first) { *d = n.second; return true; }
  return false;
}

size_t dtype_bytes(DType d) {
  switch (d) {
    case DType::BF16: case DType::F16: return 2;
    case DType::F32: return 4;
    case DType::I64: return 8;
    case DType::I8: return 1;
  }
  return 0;
}

struct Descriptor {
  DType dtype;
  std::vector<uint64_t> shape;
  uint64_t start = 0, end = 0;
};

// A descriptor as the reference's derived decoding accepts it: an object with
// dtype/shape/data_offsets (other keys ignored) or the three in a sequence.
bool parse_descriptor(const Json& v, Descriptor* d, std::string* why) {
  const Json *dt, *sh, *off;
  if (v.kind == Json::Object) {
    if (v.dup_keys) { *why = "duplicate field in Descriptor"; return false; }
    dt = v.find("dtype");
    sh = v.find("shape");
    off = v.find("data_offsets");
    if (!dt) { *why = "missing field `dtype`"; return false; }
    if (!sh) { *why = "missing field `shape`"; return false; }
    if (!off) { *why = "missing field `data_offsets`"; return false; }
  } else if (v.kind == Json::Array && v.arr.size() == 3) {
    dt = &v.arr[0]; sh = &v.arr[1]; off = &v.arr[2];
  } else {
    *why = "invalid type, expected struct Descriptor";
    return false;
  }
  if (!parse_dtype(dt, &d->dtype)) { *why = "unknown or invalid dtype"; return false; }
  if (sh->kind != Json::Array) { *why = "invalid type for shape, expected a sequence"; return false; }
  d->shape.clear();
  for (auto& e : sh->arr) {
    uint64_t u;
    if (!as_uint(&e, SIZE_MAX, &u)) { *why = "invalid value in shape, expected usize"; return false; }
    d->shape.push_back(u);
  }
  if (off->kind != Json::Array || off->arr.size() != 2 || !as_uint(&off->arr[0], SIZE_MAX, &d->start) ||
      !as_uint(&off->arr[1], SIZE_MAX, &d->end)) {
    *why = "invalid data_offsets, expected an array of 2 usize";
    return false;
  }
  return true;
}

struct Checkpoint {
  MappedFile file;
  size_t data_start = 0;
  std::map<std::string, Descriptor> tensors;  // byte order of names, like a BTreeMap
  std::map<std::string, std::string> metadata;

  size_t payload() const { return file.size - data_start; }
  const uint8_t* bytes(const Descriptor& d) const { return file.data + data_start + d.start; }

  int open(const std::string& path) {
    if (int st = file.open(path)) return st;
    if (file.size < 8) return format_err("missing header length");
    uint64_t header_len = 0;
    for (int i = 7; i >= 0; --i) header_len = (header_len << 8) | file.data[i];
    if (header_len > 100000000ull) return format_err("header exceeds 100 MB");
    if (header_len + 8 > file.size) return format_err("truncated header");
    data_start = static_cast<size_t>(header_len) + 8;
    Json header;
    std::string why;
    JsonReader reader(reinterpret_cast<const char*>(file.data + 8), static_cast<size_t>(header_len));
    if (!reader.document(&header, &why)) return json_err(why);
    if (header.kind != Json::Object) return json_err("invalid type, expected a map");
    // sorted like the reference's BTreeMap<String, Value>
    std::map<std::string, const Json*> entries;
    for (auto& kv : header.obj) entries[kv.first] = &kv.second;
    auto meta = entries.find("__metadata__");
    if (meta != entries.end()) {
      const Json& m = *meta->second;
      if (m.kind != Json::Object) return json_err("invalid type for __metadata__, expected a map");
      for (auto& kv : m.obj) {
        if (kv.second.kind != Json::String)
          return json_err("invalid type in __metadata__, expected a string");
        metadata[kv.first] = kv.second.str;
      }
      entries.erase(meta);
    }
    for (auto& kv : entries) {
      Descriptor d;
      if (!parse_descriptor(*kv.second, &d, &why)) return json_err(why);
      // checked product of the shape, then times the element size
      size_t count = 1;
      bool ok = true;
      for (uint64_t dim : d.shape) {
        if (dim > SIZE_MAX || (dim != 0 && count > SIZE_MAX / dim)) { ok = false; break; }
        count *= static_cast<size_t>(dim);
      }
      if (ok && count > SIZE_MAX / dtype_bytes(d.dtype)) ok = false;
      if (ok) count *= dtype_bytes(d.dtype);
      if (!ok) return format_err("tensor size overflow: " + kv.first);
      if (d.end < d.start || d.end - d.start != count || d.end > payload())
        return format_err("invalid tensor offsets: " + kv.first);
      tensors.emplace(kv.first, std::move(d));
    }
    std::vector<std::pair<uint64_t, uint64_t>> spans;
    for (auto& kv : tensors) spans.emplace_back(kv.second.start, kv.second.end);
    std::sort(spans.begin(), spans.end());
    uint64_t cursor = 0;
    for (auto& s : spans) {
      if (s.first != cursor) return format_err("payload gaps or overlapping tensors");
      cursor = s.second;
    }
    if (cursor != payload()) return format_err("unclaimed trailing payload");
    return UOCR_OK;
  }

  std::string sha256() const {
    Sha256 h;
    const size_t chunk = 1 << 22;
    for (size_t off = 0; off < file.size; off += chunk)
      h.update(file.data + off, std::min(chunk, file.size - off));
    return h.hex();
  }
};

// ---- QuantizedWeights::load (src/cpu/quantized.rs:239-370) ---------------------------

constexpr const char* kFormat = "uocr-q8-block32-v1";
constexpr const char* kScaleSuffix = ".q8_scales";

bool is_decimal(const std::string& s) {
  // usize::parse: optional '+', then one or more digits, value < 2^64
  size_t i = (!s.empty() && s[0] == '+') ? 1 : 0;
  if (i >= s.size()) return false;
  uint64_t v = 0;
  for (; i < s.size(); ++i) {
    if (s[i] < '0' || s[i] > '9') return false;
    uint64_t d = static_cast<uint64_t>(s[i] - '0');
    if (v > (UINT64_MAX - d) / 10) return false;
    v = v * 10 + d;
  }
  return true;
}

bool strip(std::string* s, const char* prefix) {
  size_t n = std::strlen(prefix);
  if (s->compare(0, n, prefix) != 0) return false;
  s->erase(0, n);
  return true;
}

bool one_of(const std::string& s, std::initializer_list<const char*> names) {
  for (const char* n : names) if (s == n) return true;
  return false;
}

// eligible(): the projection matrices the overlay holds (quantized.rs:262-301).
bool eligible(const std::string& name) {
  if (name == "lm_head.weight") return true;
  std::string rest = name;
  if (!strip(&rest, "model.layers.")) return false;
  size_t dot = rest.find('.');
  if (dot == std::string::npos || !is_decimal(rest.substr(0, dot))) return false;
  rest.erase(0, dot + 1);
  if (strip(&rest, "self_attn."))
    return one_of(rest, {"q_proj.weight", "k_proj.weight", "v_proj.weight", "o_proj.weight"});
  if (!strip(&rest, "mlp.")) return false;
  if (!strip(&rest, "shared_experts.") && strip(&rest, "experts.")) {
    size_t d2 = rest.find('.');
    if (d2 == std::string::npos || !is_decimal(rest.substr(0, d2))) return false;
    rest.erase(0, d2 + 1);
  }
  return one_of(rest, {"gate_proj.weight", "up_proj.weight", "down_proj.weight"});
}

struct Manifest {
  uint64_t schema_version = 0, block_size = 0, matrix_count = 0, bytes = 0;
  std::string format, source_sha256, output_sha256;
};

int parse_manifest(const std::string& text, Manifest* m) {
  Json j;
  std::string why;
  JsonReader reader(text.data(), text.size());
  if (!reader.document(&j, &why)) return json_err(why);
  if (j.kind != Json::Object) return json_err("invalid type, expected struct Manifest");
  if (j.dup_keys) return json_err("duplicate field in Manifest");
  struct UField { const char* name; uint64_t max; uint64_t* out; };
  struct SField { const char* name; std::string* out; };
  // declaration order of the reference's Manifest: a missing or mistyped
  // field is reported in that order
  const char* order[] = {"schema_version", "format", "block_size", "source_sha256",
                         "output_sha256", "matrix_count", "bytes"};
  UField uf[] = {{"schema_version", 0xFFFFFFFFull, &m->schema_version},
                 {"block_size", SIZE_MAX, &m->block_size},
                 {"matrix_count", SIZE_MAX, &m->matrix_count},
                 {"bytes", SIZE_MAX, &m->bytes}};
  SField sf[] = {{"format", &m->format},
                 {"source_sha256", &m->source_sha256},
                 {"output_sha256", &m->output_sha256}};
  // a value of the wrong type fails when it is read (object order) ...
  for (auto& kv : j.obj) {
    for (auto& f : uf)
      if (kv.first == f.name && !as_uint(&kv.second, f.max, f.out))
        return json_err(std::string("invalid value for `") + f.name + "`, expected an integer");
    for (auto& f : sf)
      if (kv.first == f.name) {
        if (kv.second.kind != Json::String)
          return json_err(std::string("invalid type for `") + f.name + "`, expected a string");
        *f.out = kv.second.str;
      }
  }
  // ... a missing one after the whole object
  for (const char* name : order)
    if (!j.find(name)) return json_err(std::string("missing field `") + name + "`");
  return UOCR_OK;
}

// One validated matrix: where its arrays are in the overlay file and in the
// device allocation.
struct Planned {
  std::string name;
  size_t rows, cols;
  const uint8_t* w;
  const uint8_t* s;
  size_t w_off, s_off;  // device offsets
};

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

struct Loaded {
  Checkpoint overlay;
  Checkpoint source;
  std::vector<Planned> plan;
  size_t device_bytes = 0;
};

// Everything QuantizedWeights::load checks, in its order, on the host.
int validate(const char* overlay_path, const char* source_path, Loaded* L) {
  if (!overlay_path || !source_path) return err(UOCR_ERR_INVALID, "null path");
  // the source checkpoint is opened by the caller in the reference
  if (int st = L->source.open(source_path)) return st;
  std::string text;
  if (int st = read_file(with_extension(overlay_path, "json"), &text)) return st;
  Manifest man;
  if (int st = parse_manifest(text, &man)) return st;
  Checkpoint& ov = L->overlay;
  if (int st = ov.open(overlay_path)) return st;
  auto meta = [&](const char* key) -> const std::string* {
    auto it = ov.metadata.find(key);
    return it == ov.metadata.end() ? nullptr : &it->second;
  };
  const std::string* mf = meta("format");
  const std::string* mb = meta("block_size");
  const std::string* ms = meta("source_sha256");
  if (man.schema_version != 1 || man.format != kFormat || man.block_size != UOCR_Q8_BLOCK ||
      !mf || *mf != kFormat || !mb || *mb != "32" || !ms || *ms != man.source_sha256 ||
      ov.file.size != man.bytes)
    return format_err("INT8 overlay version or metadata mismatch");
  // both digests (the source's on a second thread); either mismatch is the
  // reference's one error
  std::string source_digest;
  std::thread hasher([&] { source_digest = L->source.sha256(); });
  std::string overlay_digest = ov.sha256();
  hasher.join();
  if (source_digest != man.source_sha256 || overlay_digest != man.output_sha256)
    return format_err("INT8 checksum or source model mismatch");
  std::vector<std::string> expected;
  for (auto& kv : L->source.tensors) if (eligible(kv.first)) expected.push_back(kv.first);
  if (expected.empty() || expected.size() != man.matrix_count ||
      ov.tensors.size() != expected.size() * 2)
    return format_err("INT8 matrix set mismatch");
  size_t off = 0;
  for (auto& name : expected) {
    const Descriptor& original = L->source.tensors.at(name);
    auto wi = ov.tensors.find(name);
    if (wi == ov.tensors.end()) return format_err("missing tensor: " + name);
    auto si = ov.tensors.find(name + kScaleSuffix);
    if (si == ov.tensors.end()) return format_err("missing tensor: " + name + kScaleSuffix);
    const Descriptor& w = wi->second;
    const Descriptor& s = si->second;
    bool bad = w.dtype != DType::I8 || w.shape.size() != 2 || w.shape != original.shape ||
               !(original.dtype == DType::BF16 || original.dtype == DType::F16 ||
                 original.dtype == DType::F32) ||
               s.dtype != DType::F32 ||
               s.shape != std::vector<uint64_t>{w.shape[0], w.shape[1] / UOCR_Q8_BLOCK +
                                                             (w.shape[1] % UOCR_Q8_BLOCK != 0)};
    const uint8_t* wb = ov.bytes(w);
    size_t wn = static_cast<size_t>(w.end - w.start);
    if (!bad && wn && std::memchr(wb, 128, wn)) bad = true;
    if (bad) return format_err("invalid INT8 matrix " + name);
    // Int8Matrix::from_parts (quantized.rs:23-41)
    size_t rows = static_cast<size_t>(w.shape[0]), cols = static_cast<size_t>(w.shape[1]);
    if (rows == 0 || cols == 0)
      return err(UOCR_ERR_SHAPE, "invalid tensor shape: INT8 matrix storage");
    const uint8_t* sb = ov.bytes(s);
    size_t ns = static_cast<size_t>(s.end - s.start) / 4;
    for (size_t i = 0; i < ns; ++i) {
      float v;
      std::memcpy(&v, sb + 4 * i, 4);  // little-endian F32, as the file stores it
      if (!std::isfinite(v) || v < 0.0f)
        return err(UOCR_ERR_NUMERICAL,
                   "nonfinite numerical input: INT8 scales must be finite and nonnegative");
    }
    if (rows > 0x7FFFFFFF || cols > 0x7FFFFFFF)
      return err(UOCR_ERR_UNSUPPORTED, "unsupported configuration: matrix extent above 2^31");
    Planned p{name, rows, cols, wb, sb, 0, 0};
    p.w_off = off;
    off = align_up(off + wn);
    p.s_off = off;
    off = align_up(off + ns * 4);
    L->plan.push_back(std::move(p));
  }
  L->device_bytes = off;
  return UOCR_OK;
}

}  // namespace

struct uocr_overlay {
  int device = 0;
  void* base = nullptr;  // one device allocation for every matrix
  size_t bytes = 0;
  std::map<std::string, uocr_q8*> matrices;
  std::vector<std::string> names;
  ~uocr_overlay() {
    for (auto& kv : matrices) delete kv.second;
    if (base) {
      int prev = -1;
      cudaGetDevice(&prev);
      if (prev != device) cudaSetDevice(device);
      cudaFree(base);
      if (prev >= 0 && prev != device) cudaSetDevice(prev);
    }
  }
};

namespace {

// Host -> device through two pinned staging buffers: the next chunk is read
// from the mapped file while the previous one is copied.
int upload(const Loaded& L, uocr_ctx* ctx, uint8_t* dev) {
  const size_t stage = size_t(32) << 20;
  uint8_t* pinned[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  cudaError_t e = cudaSuccess;
  for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
    e = cudaMallocHost(&pinned[b], stage);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming);
  }
  int which = 0;
  auto copy = [&](const uint8_t* src, size_t n, uint8_t* dst) {
    for (size_t o = 0; o < n && e == cudaSuccess; o += stage) {
      size_t c = std::min(stage, n - o);
      e = cudaEventSynchronize(done[which]);
      if (e != cudaSuccess) break;
      std::memcpy(pinned[which], src + o, c);
      e = cudaMemcpyAsync(dst + o, pinned[which], c, cudaMemcpyHostToDevice, ctx->stream);
      if (e == cudaSuccess) e = cudaEventRecord(done[which], ctx->stream);
      which ^= 1;
    }
  };
  for (auto& p : L.plan) {
    if (e != cudaSuccess) break;
    copy(p.w, p.rows * p.cols, dev + p.w_off);
    copy(p.s, p.rows * ((p.cols + UOCR_Q8_BLOCK - 1) / UOCR_Q8_BLOCK) * 4, dev + p.s_off);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  for (int b = 0; b < 2; ++b) {
    if (done[b]) cudaEventDestroy(done[b]);
    if (pinned[b]) cudaFreeHost(pinned[b]);
  }
  if (e != cudaSuccess) return err(UOCR_ERR_CUDA, std::string("overlay upload: ") + cudaGetErrorString(e));
  return UOCR_OK;
}

}  // namespace

extern "C" {

int uocr_overlay_check(const char* overlay_path, const char* source_path, size_t* matrix_count,
                       size_t* device_bytes) {
  Loaded L;
  if (int st = validate(overlay_path, source_path, &L)) return st;
  if (matrix_count) *matrix_count = L.plan.size();
  if (device_bytes) *device_bytes = L.device_bytes;
  return UOCR_OK;
}

int uocr_overlay_load(uocr_ctx* ctx, const char* overlay_path, const char* source_path,
                      uocr_overlay** out) {
  if (!ctx || !out) return err(UOCR_ERR_INVALID, "null argument");
  *out = nullptr;
  Loaded L;
  if (int st = validate(overlay_path, source_path, &L)) return st;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != ctx->device) cudaSetDevice(ctx->device);
  std::unique_ptr<uocr_overlay> ov(new uocr_overlay());
  ov->device = ctx->device;
  ov->bytes = L.device_bytes;
  int st = UOCR_OK;
  cudaError_t e = cudaMalloc(&ov->base, std::max<size_t>(L.device_bytes, kAlign));
  if (e != cudaSuccess) {
    ov->base = nullptr;
    st = err(UOCR_ERR_CUDA, std::string("overlay allocation: ") + cudaGetErrorString(e));
  }
  if (!st) st = upload(L, ctx, static_cast<uint8_t*>(ov->base));
  if (!st) {
    auto* base = static_cast<uint8_t*>(ov->base);
    for (auto& p : L.plan) {
      auto* m = new uocr_q8();
      m->device = ctx->device;
      m->rows = p.rows;
      m->cols = p.cols;
      m->w = reinterpret_cast<int8_t*>(base + p.w_off);
      m->s = reinterpret_cast<float*>(base + p.s_off);
      m->owns = false;
      ov->matrices[p.name] = m;
      ov->names.push_back(p.name);
    }
  }
  if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
  if (st) return st;
  *out = ov.release();
  return UOCR_OK;
}

int uocr_overlay_get(const uocr_overlay* ov, const char* name, const uocr_q8** out) {
  if (!ov || !name || !out) return err(UOCR_ERR_INVALID, "null argument");
  auto it = ov->matrices.find(name);
  *out = it == ov->matrices.end() ? nullptr : it->second;
  return UOCR_OK;
}

size_t uocr_overlay_count(const uocr_overlay* ov) { return ov ? ov->names.size() : 0; }

const char* uocr_overlay_name(const uocr_overlay* ov, size_t index) {
  if (!ov || index >= ov->names.size()) return nullptr;
  return ov->names[index].c_str();
}

size_t uocr_overlay_device_bytes(const uocr_overlay* ov) { return ov ? ov->bytes : 0; }

int uocr_overlay_free(uocr_overlay* ov) {
  delete ov;
  return UOCR_OK;
}

int uocr_sha256_file(const char* path, char* hex_out) {
  if (!path || !hex_out) return err(UOCR_ERR_INVALID, "null argument");
  MappedFile f;
  if (int st = f.open(path)) return st;
  Sha256 h;
  if (f.size) h.update(f.data, f.size);
  std::string hex = h.hex();
  std::memcpy(hex_out, hex.c_str(), 65);
  return UOCR_OK;
}

}  // extern "C"
