// Native reader of the reference's on-disk weight unit: a packed blob
// (blob.bin) plus its manifest (blob_manifest.json), as tools/pack_block.py
// writes them (name-sorted entries at 64-byte aligned offsets, zero fill,
// per-entry and whole-blob SHA-256). ltxb_blob_open does what
// ltx/loader.zig's Blob.open and the ring's first-touch check do
// (ltx/loader.zig:50-82, :270-276): parse the manifest, compare blob.bin's
// size with total_bytes (BlobSizeMismatch), map it read-only, check the
// layout (Misaligned / LayoutGap / TrailingBytes) and, on request, the
// digests (BlobDigestMismatch). Host code only; the mapped bytes and entry
// table feed ltxb_weights_upload / ltxb_core_upload.
//
// The manifest parser is a small recursive-descent JSON reader (RFC 8259)
// that keeps integers exact; the digest is SHA-256 as FIPS 180-4 defines it,
// with the round constants derived from their definition (the fractional
// parts of the square and cube roots of the first primes) and the x86 SHA
// extensions used when the host CPU has them.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#if defined(__x86_64__)
#include <cpuid.h>
#include <immintrin.h>
#endif

#include "kernels.h"

using ltxb::set_error;

namespace {

// ---------------------------------------------------------------------------
// SHA-256 (FIPS 180-4)
// ---------------------------------------------------------------------------

struct ShaConstants {
  uint32_t h0[8];
  uint32_t k[64];
};

// floor(x) for x = cbrt(v) or sqrt(v) of a 128-bit v, by bisection
static uint64_t iroot(unsigned __int128 v, int power) {
  uint64_t lo = 0, hi = uint64_t(1) << 40;  // every root taken here is < 2^36
  while (lo < hi) {
    const uint64_t mid = lo + (hi - lo + 1) / 2;
    unsigned __int128 p = mid;
    for (int i = 1; i < power; ++i) p *= mid;
    if (p <= v) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// H(0) = the first 32 bits of the fractional parts of the square roots of the
// first 8 primes; K = those of the cube roots of the first 64 primes. With
// r = floor(root(p) * 2^32) = floor(root(p * 2^(32*power))), the low 32 bits
// of r are exactly those fraction bits.
static const ShaConstants& sha_constants() {
  static const ShaConstants c = [] {
    ShaConstants s{};
    int primes[64], n = 0;
    for (int v = 2; n < 64; ++v) {
      bool prime = true;
      for (int i = 0; i < n && primes[i] * primes[i] <= v; ++i)
        if (v % primes[i] == 0) prime = false;
      if (prime) primes[n++] = v;
    }
    for (int i = 0; i < 8; ++i) s.h0[i] = (uint32_t)iroot((unsigned __int128)primes[i] << 64, 2);
    for (int i = 0; i < 64; ++i) s.k[i] = (uint32_t)iroot((unsigned __int128)primes[i] << 96, 3);
    return s;
  }();
  return c;
}

static inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
static inline uint32_t load_be32(const uint8_t* p) {
  return (uint32_t)p[0] << 24 | (uint32_t)p[1] << 16 | (uint32_t)p[2] << 8 | (uint32_t)p[3];
}

// FIPS 180-4 section 6.2.2 on `nblocks` 64-byte blocks
static void sha_blocks_portable(uint32_t st[8], const uint8_t* p, size_t nblocks) {
  const uint32_t* K = sha_constants().k;
  uint32_t w[64];
  for (; nblocks; --nblocks, p += 64) {
    for (int t = 0; t < 16; ++t) w[t] = load_be32(p + 4 * t);
    for (int t = 16; t < 64; ++t) {
      const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
      const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
      w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
    for (int t = 0; t < 64; ++t) {
      const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + K[t] + w[t];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      h = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    st[0] += a;
    st[1] += b;
    st[2] += c;
    st[3] += d;
    st[4] += e;
    st[5] += f;
    st[6] += g;
    st[7] += h;
  }
}

#if defined(__x86_64__)
// The same compression with the SHA extensions (SHA256RNDS2 / SHA256MSG1 /
// SHA256MSG2). RNDS2 runs two rounds on the state held as (A,B,E,F) and
// (C,D,G,H) words, taking W[t]+K[t] for its two rounds in the low 64 bits of
// its third operand; MSG1/MSG2 compute the message schedule's sigma0 and
// sigma1 terms four words at a time.
__attribute__((target("sha,sse4.1"))) static void sha_blocks_x86(uint32_t st[8], const uint8_t* p,
                                                                 size_t nblocks) {
  const uint32_t* K = sha_constants().k;
  const __m128i bswap = _mm_set_epi8(12, 13, 14, 15, 8, 9, 10, 11, 4, 5, 6, 7, 0, 1, 2, 3);
  // st = {a,b,c,d,e,f,g,h} -> abef = {f,e,b,a} (lanes 0..3), cdgh = {h,g,d,c}
  __m128i abcd = _mm_loadu_si128(reinterpret_cast<const __m128i*>(st));      // a b c d
  __m128i efgh = _mm_loadu_si128(reinterpret_cast<const __m128i*>(st + 4));  // e f g h
  __m128i badc = _mm_shuffle_epi32(abcd, 0xB1);                              // b a d c
  __m128i fehg = _mm_shuffle_epi32(efgh, 0xB1);                              // f e h g
  __m128i abef = _mm_unpacklo_epi64(fehg, badc);                             // f e b a
  __m128i cdgh = _mm_unpackhi_epi64(fehg, badc);                             // h g d c
  for (; nblocks; --nblocks, p += 64) {
    const __m128i abef0 = abef, cdgh0 = cdgh;
    __m128i m[4];
    for (int i = 0; i < 4; ++i)
      m[i] = _mm_shuffle_epi8(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p + 16 * i)), bswap);
    for (int q = 0; q < 16; ++q) {  // four rounds per step, words W[4q .. 4q+3] in m[q & 3]
      __m128i& cur = m[q & 3];
      if (q >= 4) {
        // W[t] = s1(W[t-2]) + W[t-7] + s0(W[t-15]) + W[t-16] for t = 4q .. 4q+3
        __m128i t = _mm_sha256msg1_epu32(cur, m[(q + 1) & 3]);            // W[t-16] + s0(W[t-15])
        t = _mm_add_epi32(t, _mm_alignr_epi8(m[(q + 3) & 3], m[(q + 2) & 3], 4));  // + W[t-7]
        cur = _mm_sha256msg2_epu32(t, m[(q + 3) & 3]);                       // + s1(W[t-2])
      }
      const __m128i wk = _mm_add_epi32(cur, _mm_loadu_si128(reinterpret_cast<const __m128i*>(K + 4 * q)));
      // rounds 4q, 4q+1 leave (A,B,E,F) in the register that held (C,D,G,H);
      // rounds 4q+2, 4q+3 then take the old (A,B,E,F) as their (C,D,G,H), so
      // after the pair each register holds its original role again
      cdgh = _mm_sha256rnds2_epu32(cdgh, abef, wk);
      abef = _mm_sha256rnds2_epu32(abef, cdgh, _mm_shuffle_epi32(wk, 0x0E));
    }
    abef = _mm_add_epi32(abef, abef0);
    cdgh = _mm_add_epi32(cdgh, cdgh0);
  }
  // back to a b c d | e f g h
  const __m128i feba = abef, hgdc = cdgh;
  abcd = _mm_shuffle_epi32(_mm_unpackhi_epi64(hgdc, feba), 0x1B);  // (d c b a) reversed -> a b c d
  efgh = _mm_shuffle_epi32(_mm_unpacklo_epi64(hgdc, feba), 0x1B);  // (h g f e) reversed -> e f g h
  _mm_storeu_si128(reinterpret_cast<__m128i*>(st), abcd);
  _mm_storeu_si128(reinterpret_cast<__m128i*>(st + 4), efgh);
}

// CPUID leaf 7 EBX bit 29: SHA extensions; leaf 1 ECX bit 19: SSE4.1
static bool cpu_has_sha() {
  static const bool has = [] {
    unsigned a, b, c, d;
    if (!__get_cpuid(1, &a, &b, &c, &d) || !(c & (1u << 19))) return false;
    if (!__get_cpuid_count(7, 0, &a, &b, &c, &d)) return false;
    return (b & (1u << 29)) != 0;
  }();
  return has;
}
#endif

// 0: the SHA extensions when the CPU has them; 1: the portable code only.
// ltxb_sha256_impl sets it so tests can compare the two implementations.
static std::atomic<int> g_sha_impl{0};

static void sha_blocks(uint32_t st[8], const uint8_t* p, size_t nblocks) {
#if defined(__x86_64__)
  if (g_sha_impl == 0 && cpu_has_sha()) return sha_blocks_x86(st, p, nblocks);
#endif
  sha_blocks_portable(st, p, nblocks);
}

static void sha256(const void* data, uint64_t bytes, uint8_t out[32]) {
  uint32_t st[8];
  memcpy(st, sha_constants().h0, sizeof st);
  const uint8_t* p = static_cast<const uint8_t*>(data);
  const uint64_t full = bytes / 64;
  sha_blocks(st, p, (size_t)full);
  // padding: 0x80, zeros to 56 mod 64, then the bit length big-endian
  uint8_t tail[128] = {};
  const size_t rem = (size_t)(bytes - full * 64);
  if (rem) memcpy(tail, p + full * 64, rem);
  tail[rem] = 0x80;
  const size_t tail_blocks = rem < 56 ? 1 : 2;
  const uint64_t bits = bytes * 8;
  for (int i = 0; i < 8; ++i) tail[tail_blocks * 64 - 1 - i] = (uint8_t)(bits >> (8 * i));
  sha_blocks(st, tail, tail_blocks);
  for (int i = 0; i < 8; ++i) {
    out[4 * i] = (uint8_t)(st[i] >> 24);
    out[4 * i + 1] = (uint8_t)(st[i] >> 16);
    out[4 * i + 2] = (uint8_t)(st[i] >> 8);
    out[4 * i + 3] = (uint8_t)st[i];
  }
}

static void sha256_hex(const void* data, uint64_t bytes, char hex[65]) {
  uint8_t d[32];
  sha256(data, bytes, d);
  static const char digits[] = "0123456789abcdef";
  for (int i = 0; i < 32; ++i) {
    hex[2 * i] = digits[d[i] >> 4];
    hex[2 * i + 1] = digits[d[i] & 15];
  }
  hex[64] = '\0';
}

// ---------------------------------------------------------------------------
// JSON (RFC 8259), enough for the manifest: a DOM with exact integers
// ---------------------------------------------------------------------------

struct JVal {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  bool is_int = false;  // an integer literal that fits in int64
  int64_t i = 0;
  double d = 0;
  std::string s;
  std::vector<JVal> a;
  std::vector<std::pair<std::string, JVal>> o;

  const JVal* get(const char* key) const {
    if (kind != OBJ) return nullptr;
    for (const auto& kv : o)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class JParser {
 public:
  JParser(const char* p, size_t n) : p_(p), end_(p + n) {}

  bool parse(JVal& out, std::string& err) {
    if (!value(out, 0)) {
      err = err_;
      return false;
    }
    ws();
    if (p_ != end_) {
      err = "trailing characters after the JSON value";
      return false;
    }
    return true;
  }

 private:
  const char* p_;
  const char* end_;
  std::string err_;

  bool fail(const char* msg) {
    if (err_.empty()) err_ = msg;
    return false;
  }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* w) {
    const size_t n = strlen(w);
    if ((size_t)(end_ - p_) < n || memcmp(p_, w, n) != 0) return fail("invalid literal");
    p_ += n;
    return true;
  }

  bool value(JVal& v, int depth) {
    if (depth > 64) return fail("nesting deeper than 64");
    ws();
    if (p_ >= end_) return fail("unexpected end of input");
    switch (*p_) {
      case '{': return object(v, depth);
      case '[': return array(v, depth);
      case '"': v.kind = JVal::STR; return string(v.s);
      case 't': v.kind = JVal::BOOL; v.b = true; return lit("true");
      case 'f': v.kind = JVal::BOOL; v.b = false; return lit("false");
      case 'n': v.kind = JVal::NUL; return lit("null");
      default: return number(v);
    }
  }

  bool object(JVal& v, int depth) {
    v.kind = JVal::OBJ;
    ++p_;
    ws();
    if (p_ < end_ && *p_ == '}') {
      ++p_;
      return true;
    }
    for (;;) {
      ws();
      if (p_ >= end_ || *p_ != '"') return fail("expected a member name");
      std::string key;
      if (!string(key)) return false;
      ws();
      if (p_ >= end_ || *p_ != ':') return fail("expected ':'");
      ++p_;
      v.o.emplace_back(std::move(key), JVal());
      if (!value(v.o.back().second, depth + 1)) return false;
      ws();
      if (p_ < end_ && *p_ == ',') {
        ++p_;
        continue;
      }
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      return fail("expected ',' or '}'");
    }
  }

  bool array(JVal& v, int depth) {
    v.kind = JVal::ARR;
    ++p_;
    ws();
    if (p_ < end_ && *p_ == ']') {
      ++p_;
      return true;
    }
    for (;;) {
      v.a.emplace_back();
      if (!value(v.a.back(), depth + 1)) return false;
      ws();
      if (p_ < end_ && *p_ == ',') {
        ++p_;
        continue;
      }
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      return fail("expected ',' or ']'");
    }
  }

  static int hexval(char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
  }
  bool hex4(uint32_t& u) {
    if (end_ - p_ < 4) return fail("short \\u escape");
    u = 0;
    for (int i = 0; i < 4; ++i) {
      const int h = hexval(p_[i]);
      if (h < 0) return fail("bad \\u escape");
      u = u * 16 + (uint32_t)h;
    }
    p_ += 4;
    return true;
  }
  static void utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) {
      s += (char)cp;
    } else if (cp < 0x800) {
      s += (char)(0xC0 | (cp >> 6));
      s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      s += (char)(0xE0 | (cp >> 12));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    } else {
      s += (char)(0xF0 | (cp >> 18));
      s += (char)(0x80 | ((cp >> 12) & 0x3F));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    }
  }

  bool string(std::string& s) {
    ++p_;  // opening quote
    while (p_ < end_ && *p_ != '"') {
      const unsigned char c = (unsigned char)*p_;
      if (c < 0x20) return fail("control character in a string");
      if (c != '\\') {
        s += (char)c;
        ++p_;
        continue;
      }
      if (++p_ >= end_) return fail("unterminated escape");
      const char e = *p_++;
      switch (e) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'n': s += '\n'; break;
        case 'r': s += '\r'; break;
        case 't': s += '\t'; break;
        case 'u': {
          uint32_t u;
          if (!hex4(u)) return false;
          if (u >= 0xD800 && u < 0xDC00) {  // a surrogate pair
            uint32_t lo;
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return fail("lone high surrogate");
            p_ += 2;
            if (!hex4(lo)) return false;
            if (lo < 0xDC00 || lo >= 0xE000) return fail("bad low surrogate");
            u = 0x10000 + ((u - 0xD800) << 10) + (lo - 0xDC00);
          } else if (u >= 0xDC00 && u < 0xE000) {
            return fail("lone low surrogate");
          }
          utf8(s, u);
          break;
        }
        default: return fail("unknown escape");
      }
    }
    if (p_ >= end_) return fail("unterminated string");
    ++p_;  // closing quote
    return true;
  }

  bool number(JVal& v) {
    const char* s = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return fail("invalid value");
    if (*p_ == '0') ++p_;
    else
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    bool integral = true;
    if (p_ < end_ && *p_ == '.') {
      integral = false;
      ++p_;
      if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return fail("invalid number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      integral = false;
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return fail("invalid number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    const std::string text(s, p_);
    v.kind = JVal::NUM;
    v.d = strtod(text.c_str(), nullptr);
    if (integral) {
      // exact int64, or not an integer this reader can hold
      const bool neg = text[0] == '-';
      unsigned __int128 mag = 0;
      bool fits = true;
      for (size_t k = neg ? 1 : 0; k < text.size() && fits; ++k) {
        mag = mag * 10 + (unsigned)(text[k] - '0');
        if (mag > ((unsigned __int128)1 << 63)) fits = false;
      }
      if (fits && (neg || mag < ((unsigned __int128)1 << 63))) {
        v.is_int = true;
        v.i = neg ? (int64_t)(0 - (uint64_t)mag) : (int64_t)mag;
      }
    }
    return true;
  }
};

// ---------------------------------------------------------------------------
// the blob
// ---------------------------------------------------------------------------

int dtype_code(const std::string& s) {
  if (s == "BF16") return LTXB_DT_BF16;
  if (s == "F32") return LTXB_DT_F32;
  if (s == "I8") return LTXB_DT_I8;
  return -1;
}

bool read_file(const std::string& path, std::string& out) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  char buf[1 << 16];
  size_t n;
  while ((n = fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
  const bool ok = !ferror(f);
  fclose(f);
  return ok;
}

}  // namespace

struct ltxb_blob {
  const uint8_t* data = nullptr;
  uint64_t bytes = 0;
  bool mapped = false;
  uint32_t align = 0;
  int64_t block = 0;
  std::string blob_sha256;
  std::vector<std::string> names;
  std::vector<std::string> entry_sha256;
  std::vector<ltxb_entry> entries;

  ~ltxb_blob() {
    if (mapped) munmap(const_cast<uint8_t*>(data), (size_t)bytes);
  }
};

namespace {

// the manifest's fields (ltx/loader.zig:20-43); unknown fields are ignored,
// as the reference's parser does
int parse_manifest(const std::string& text, ltxb_blob& b, uint64_t& total_bytes) {
  JVal root;
  std::string err;
  if (!JParser(text.data(), text.size()).parse(root, err))
    return set_error(LTXB_ELAYOUT, "blob manifest: %s", err.c_str());
  if (root.kind != JVal::OBJ) return set_error(LTXB_ELAYOUT, "blob manifest: not a JSON object");
  auto uint_field = [&](const JVal& obj, const char* key, uint64_t& out, const char* where) {
    const JVal* v = obj.get(key);
    if (!v || v->kind != JVal::NUM || !v->is_int || v->i < 0)
      return set_error(LTXB_ELAYOUT, "blob manifest: %s needs a non-negative integer '%s'", where, key);
    out = (uint64_t)v->i;
    return LTXB_OK;
  };
  uint64_t align = 0, total = 0;
  int rc = uint_field(root, "align", align, "the header");
  if (!rc) rc = uint_field(root, "total_bytes", total, "the header");
  if (rc) return rc;
  if (align == 0 || align > (1u << 20)) return set_error(LTXB_ELAYOUT, "blob manifest: align %llu", (unsigned long long)align);
  b.align = (uint32_t)align;
  total_bytes = total;
  const JVal* blk = root.get("block");
  if (blk && blk->kind == JVal::NUM && blk->is_int) b.block = blk->i;
  const JVal* sha = root.get("blob_sha256");
  if (sha && sha->kind == JVal::STR) b.blob_sha256 = sha->s;
  const JVal* ents = root.get("entries");
  if (!ents || ents->kind != JVal::ARR) return set_error(LTXB_ELAYOUT, "blob manifest: no 'entries' array");
  const size_t n = ents->a.size();
  if (n > (1u << 24)) return set_error(LTXB_ELAYOUT, "blob manifest: %zu entries", n);
  b.names.resize(n);
  b.entry_sha256.resize(n);
  b.entries.assign(n, ltxb_entry{});
  for (size_t i = 0; i < n; ++i) {
    const JVal& e = ents->a[i];
    if (e.kind != JVal::OBJ) return set_error(LTXB_ELAYOUT, "blob manifest: entry %zu is not an object", i);
    const JVal* name = e.get("name");
    const JVal* dt = e.get("dtype");
    const JVal* shape = e.get("shape");
    if (!name || name->kind != JVal::STR || !dt || dt->kind != JVal::STR || !shape || shape->kind != JVal::ARR)
      return set_error(LTXB_ELAYOUT, "blob manifest: entry %zu needs name, dtype and shape", i);
    ltxb_entry& x = b.entries[i];
    b.names[i] = name->s;
    char where[64];
    snprintf(where, sizeof where, "entry %zu", i);
    if ((rc = uint_field(e, "offset", x.offset, where))) return rc;
    if ((rc = uint_field(e, "nbytes", x.nbytes, where))) return rc;
    x.dtype = dtype_code(dt->s);
    x.ndim = (int32_t)shape->a.size();
    for (size_t d = 0; d < shape->a.size(); ++d) {
      const JVal& s = shape->a[d];
      if (s.kind != JVal::NUM || !s.is_int || s.i < 0)
        return set_error(LTXB_ELAYOUT, "blob manifest: entry %s has a bad shape", name->s.c_str());
      if (d < 2) x.shape[d] = s.i;
    }
    const JVal* es = e.get("sha256");
    if (es && es->kind == JVal::STR) b.entry_sha256[i] = es->s;
  }
  for (size_t i = 0; i < n; ++i) b.entries[i].name = b.names[i].c_str();
  return LTXB_OK;
}

int verify_digests(const ltxb_blob& b, int what) {
  if (what & LTXB_VERIFY_BLOB) {
    if (b.blob_sha256.empty()) return set_error(LTXB_ELAYOUT, "BlobDigestMismatch: the manifest has no blob_sha256");
    char hex[65];
    sha256_hex(b.data, b.bytes, hex);
    if (b.blob_sha256 != hex)
      return set_error(LTXB_ELAYOUT, "BlobDigestMismatch: blob.bin hashes to %s, the manifest says %s", hex,
                       b.blob_sha256.c_str());
  }
  if (what & LTXB_VERIFY_ENTRIES) {
    // entries are independent: hash them on all host cores
    const size_t n = b.entries.size();
    std::atomic<size_t> next{0};
    std::atomic<long long> bad{-1};
    auto work = [&] {
      for (size_t i; (i = next.fetch_add(1)) < n;) {
        char hex[65];
        sha256_hex(b.data + b.entries[i].offset, b.entries[i].nbytes, hex);
        if (b.entry_sha256[i] != hex) {
          long long expect = -1;
          bad.compare_exchange_strong(expect, (long long)i);
        }
      }
    };
    const unsigned hw = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    const size_t nt = std::min<size_t>(hw, n);
    std::vector<std::thread> pool;
    for (size_t t = 1; t < nt; ++t) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    if (bad.load() >= 0) {
      const size_t i = (size_t)bad.load();
      return set_error(LTXB_ELAYOUT, "BlobDigestMismatch: entry %s does not hash to its manifest digest",
                       b.names[i].c_str());
    }
  }
  return LTXB_OK;
}

std::string normalize(const char* name) {
  std::string s;
  for (const char* p = name; *p; ++p) {
    if (p[0] == ':' && p[1] == ':') {
      s += '_';
      ++p;
    } else {
      s += *p == '.' ? '_' : *p;
    }
  }
  return s;
}

}  // namespace

extern "C" {

// checkLayout (ltx/loader.zig:73-82): aligned offsets, increasing, gaps only
// alignment fill, the last entry ending at the blob's end. Every entry is
// also checked to lie inside the blob, so no sum below wraps around.
int ltxb_blob_check_layout(const ltxb_entry* entries, int n_entries, uint64_t blob_bytes, uint32_t align) {
  if (n_entries < 0 || (n_entries > 0 && !entries) || align == 0) return set_error(LTXB_EINVAL, "bad arguments");
  uint64_t end = 0;
  for (int i = 0; i < n_entries; ++i) {
    const ltxb_entry& e = entries[i];
    const char* name = e.name ? e.name : "(unnamed)";
    if (e.offset % align) return set_error(LTXB_ELAYOUT, "Misaligned: %s at %llu", name, (unsigned long long)e.offset);
    if (e.offset < end || e.offset - end >= align)
      return set_error(LTXB_ELAYOUT, "LayoutGap: %s at %llu after %llu", name, (unsigned long long)e.offset,
                       (unsigned long long)end);
    if (e.nbytes > blob_bytes || e.offset > blob_bytes - e.nbytes)
      return set_error(LTXB_ELAYOUT, "TrailingBytes: %s (%llu bytes at %llu) ends past the blob's %llu bytes", name,
                       (unsigned long long)e.nbytes, (unsigned long long)e.offset, (unsigned long long)blob_bytes);
    end = e.offset + e.nbytes;
  }
  if (end != blob_bytes)
    return set_error(LTXB_ELAYOUT, "TrailingBytes: entries end at %llu, blob is %llu", (unsigned long long)end,
                     (unsigned long long)blob_bytes);
  return LTXB_OK;
}

int ltxb_blob_open(const char* dir, int verify, ltxb_blob** out) {
  if (!out) return set_error(LTXB_EINVAL, "blob open: out is null");
  *out = nullptr;
  if (!dir) return set_error(LTXB_EINVAL, "blob open: dir is null");
  if (verify & ~(LTXB_VERIFY_BLOB | LTXB_VERIFY_ENTRIES)) return set_error(LTXB_EINVAL, "blob open: verify flags %d", verify);
  const std::string d(dir);
  std::string text;
  if (!read_file(d + "/blob_manifest.json", text))
    return set_error(LTXB_EMISSING, "blob open: cannot read %s/blob_manifest.json", dir);
  auto* b = new ltxb_blob();
  uint64_t total = 0;
  int rc = parse_manifest(text, *b, total);
  if (rc) {
    delete b;
    return rc;
  }
  const std::string path = d + "/blob.bin";
  const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) {
    delete b;
    return set_error(LTXB_EMISSING, "blob open: cannot open %s", path.c_str());
  }
  struct stat st {};
  if (fstat(fd, &st) != 0) {
    close(fd);
    delete b;
    return set_error(LTXB_EMISSING, "blob open: cannot stat %s", path.c_str());
  }
  if ((uint64_t)st.st_size != total) {
    close(fd);
    delete b;
    return set_error(LTXB_ELAYOUT, "BlobSizeMismatch: blob.bin has %llu bytes, the manifest says %llu",
                     (unsigned long long)st.st_size, (unsigned long long)total);
  }
  b->bytes = total;
  if (total > 0) {
    void* p = mmap(nullptr, (size_t)total, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) {
      close(fd);
      delete b;
      return set_error(LTXB_ENOMEM, "blob open: mmap of %llu bytes failed", (unsigned long long)total);
    }
    b->data = static_cast<const uint8_t*>(p);
    b->mapped = true;
  }
  close(fd);
  rc = ltxb_blob_check_layout(b->entries.data(), (int)b->entries.size(), b->bytes, b->align);
  if (!rc) rc = verify_digests(*b, verify);
  if (rc) {
    delete b;
    return rc;
  }
  *out = b;
  return LTXB_OK;
}

void ltxb_blob_close(ltxb_blob* blob) { delete blob; }

int ltxb_blob_view(const ltxb_blob* blob, const void** data, uint64_t* bytes, const ltxb_entry** entries,
                   int* n_entries, uint32_t* align, int64_t* block) {
  if (!blob) return set_error(LTXB_EINVAL, "blob view: null blob");
  if (data) *data = blob->data;
  if (bytes) *bytes = blob->bytes;
  if (entries) *entries = blob->entries.empty() ? nullptr : blob->entries.data();
  if (n_entries) *n_entries = (int)blob->entries.size();
  if (align) *align = blob->align;
  if (block) *block = blob->block;
  return LTXB_OK;
}

int ltxb_blob_find(const ltxb_blob* blob, const char* name, const ltxb_entry** out) {
  if (!blob || !name || !out) return set_error(LTXB_EINVAL, "blob find: null argument");
  *out = nullptr;
  for (const ltxb_entry& e : blob->entries)
    if (normalize(e.name) == name) {
      *out = &e;
      return LTXB_OK;
    }
  return set_error(LTXB_EMISSING, "blob %lld: no entry named %s", (long long)blob->block, name);
}

int ltxb_blob_verify(const ltxb_blob* blob, int verify) {
  if (!blob) return set_error(LTXB_EINVAL, "blob verify: null blob");
  if (verify & ~(LTXB_VERIFY_BLOB | LTXB_VERIFY_ENTRIES)) return set_error(LTXB_EINVAL, "blob verify: flags %d", verify);
  return verify_digests(*blob, verify);
}

void ltxb_sha256_hex(const void* data, uint64_t bytes, char hex[65]) { sha256_hex(data, bytes, hex); }

int ltxb_sha256_impl(int portable_only) {
  g_sha_impl = portable_only ? 1 : 0;
#if defined(__x86_64__)
  return portable_only ? 0 : (cpu_has_sha() ? 1 : 0);
#else
  return 0;
#endif
}

}  // extern "C"
