// Canonical JSON text and SHA-256 layer hashes (see canonical.hpp).
#include "canonical.hpp"

#include <algorithm>
#include <cerrno>
#include <charconv>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <vector>

namespace b2canon {

// ---------------------------------------------------------------- SHA-256
// FIPS 180-4 section 6.2: 64-byte blocks, eight 32-bit working variables, the
// first 32 bits of the fractional parts of the cube roots of the first 64
// primes as round constants and of the square roots of the first 8 primes as
// the initial hash value.
namespace {
constexpr uint32_t kRound[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
}  // namespace

Sha256::Sha256()
    : h_{0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19} {}

void Sha256::block(const uint8_t* p) {
  uint32_t w[64];
  for (int i = 0; i < 16; ++i)
    w[i] = uint32_t(p[4 * i]) << 24 | uint32_t(p[4 * i + 1]) << 16 | uint32_t(p[4 * i + 2]) << 8 | p[4 * i + 3];
  for (int i = 16; i < 64; ++i) {
    const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
    const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
  for (int i = 0; i < 64; ++i) {
    const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + kRound[i] + w[i];
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
  h_[0] += a; h_[1] += b; h_[2] += c; h_[3] += d; h_[4] += e; h_[5] += f; h_[6] += g; h_[7] += h;
}

void Sha256::update(const void* data, size_t n) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  bytes_ += n;
  while (n > 0) {
    if (fill_ == 0 && n >= 64) {
      block(p);
      p += 64;
      n -= 64;
      continue;
    }
    const size_t take = std::min(n, 64 - fill_);
    std::memcpy(buf_ + fill_, p, take);
    fill_ += take;
    p += take;
    n -= take;
    if (fill_ == 64) {
      block(buf_);
      fill_ = 0;
    }
  }
}

std::array<uint8_t, 32> Sha256::digest() {
  const uint64_t bits = bytes_ * 8;
  const uint8_t one = 0x80, zero = 0;
  update(&one, 1);
  while (fill_ != 56) update(&zero, 1);
  uint8_t len[8];
  for (int i = 0; i < 8; ++i) len[i] = uint8_t(bits >> (56 - 8 * i));
  update(len, 8);
  std::array<uint8_t, 32> out{};
  for (int i = 0; i < 8; ++i)
    for (int k = 0; k < 4; ++k) out[size_t(4 * i + k)] = uint8_t(h_[i] >> (24 - 8 * k));
  return out;
}

std::string Sha256::hex() {
  static const char* digits = "0123456789abcdef";
  std::string s;
  for (uint8_t b : digest()) {
    s.push_back(digits[b >> 4]);
    s.push_back(digits[b & 15]);
  }
  return s;
}

// ---------------------------------------------------------------- canonical text
std::string python_float(double v) {
  if (v == 0.0) return std::signbit(v) ? "-0.0" : "0.0";
  // shortest round-trip digits in scientific form: d.ddd...e[+-]X
  char buf[64];
  auto res = std::to_chars(buf, buf + sizeof(buf), v, std::chars_format::scientific);
  std::string sci(buf, res.ptr);
  std::string sign;
  if (sci[0] == '-') {
    sign = "-";
    sci.erase(0, 1);
  }
  const size_t epos = sci.find('e');
  const int exponent = std::atoi(sci.c_str() + epos + 1);
  std::string digits;
  for (size_t i = 0; i < epos; ++i)
    if (sci[i] != '.') digits.push_back(sci[i]);
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  if (exponent < -4 || exponent >= 16) {
    std::string out = sign + digits.substr(0, 1);
    if (digits.size() > 1) out += "." + digits.substr(1);
    char e[16];
    std::snprintf(e, sizeof(e), "e%c%02d", exponent < 0 ? '-' : '+', exponent < 0 ? -exponent : exponent);
    return out + e;
  }
  const int point = exponent + 1;  // digits before the decimal point
  if (point <= 0) return sign + "0." + std::string(size_t(-point), '0') + digits;
  if (size_t(point) >= digits.size()) return sign + digits + std::string(size_t(point) - digits.size(), '0') + ".0";
  return sign + digits.substr(0, size_t(point)) + "." + digits.substr(size_t(point));
}

namespace {

template <class Out>
struct Writer {
  Out& out;
  std::string buf;
  void flush() {
    put(out, buf);
    buf.clear();
  }
  static void put(Sha256& h, const std::string& s) { h.update(s); }
  static void put(std::string& t, const std::string& s) { t += s; }

  void string(const std::string& s) {
    static const char* hex = "0123456789abcdef";
    buf.push_back('"');
    for (unsigned char c : s) {
      switch (c) {
        case '"': buf += "\\\""; break;
        case '\\': buf += "\\\\"; break;
        case '\b': buf += "\\b"; break;
        case '\f': buf += "\\f"; break;
        case '\n': buf += "\\n"; break;
        case '\r': buf += "\\r"; break;
        case '\t': buf += "\\t"; break;
        default:
          if (c < 0x20) {
            buf += "\\u00";
            buf.push_back(hex[c >> 4]);
            buf.push_back(hex[c & 15]);
          } else {
            buf.push_back(char(c));
          }
      }
    }
    buf.push_back('"');
  }

  void number(const std::string& t) {
    bool integer = !t.empty();
    for (size_t i = (t[0] == '-'); i < t.size(); ++i) integer &= t[i] >= '0' && t[i] <= '9';
    if (integer) {
      // integers within 64 bits print in decimal; larger ones are reals
      errno = 0;
      if (t[0] == '-') {
        long long v = std::strtoll(t.c_str(), nullptr, 10);
        if (!errno) {
          buf += std::to_string(v);
          return;
        }
      } else {
        unsigned long long v = std::strtoull(t.c_str(), nullptr, 10);
        if (!errno) {
          buf += std::to_string(v);
          return;
        }
      }
    }
    buf += python_float(std::strtod(t.c_str(), nullptr));
  }

  void value(const b2json::Value& v) {
    using T = b2json::Value::Type;
    switch (v.type()) {
      case T::Null: buf += "null"; break;
      case T::Bool: buf += v.boolean() ? "true" : "false"; break;
      case T::Number: number(v.number_text()); break;
      case T::String: string(v.str()); break;
      case T::Array: {
        buf.push_back('[');
        bool first = true;
        for (const auto& x : v.arr()) {
          if (!first) buf.push_back(',');
          first = false;
          value(x);
          if (buf.size() > (1 << 16)) flush();
        }
        buf.push_back(']');
        break;
      }
      case T::Object: {
        // code-point order of UTF-8 keys == byte order; a repeated key keeps
        // its last value, as a JSON object map does
        std::vector<const std::pair<std::string, b2json::Value>*> members;
        for (const auto& kv : v.obj()) members.push_back(&kv);
        std::stable_sort(members.begin(), members.end(), [](auto* a, auto* b) { return a->first < b->first; });
        buf.push_back('{');
        bool first = true;
        for (size_t i = 0; i < members.size(); ++i) {
          if (i + 1 < members.size() && members[i + 1]->first == members[i]->first) continue;
          if (!first) buf.push_back(',');
          first = false;
          string(members[i]->first);
          buf.push_back(':');
          value(members[i]->second);
        }
        buf.push_back('}');
        break;
      }
    }
  }
};

}  // namespace

void write(const b2json::Value& v, Sha256& out) {
  Writer<Sha256> w{out, {}};
  w.value(v);
  w.flush();
}

std::string text(const b2json::Value& v) {
  std::string out;
  Writer<std::string> w{out, {}};
  w.value(v);
  w.flush();
  return out;
}

// ---------------------------------------------------------------- protocol
Layers layer_hashes(const b2json::Value& root) {
  auto hash = [&](const char* layer) {
    Sha256 h;
    write(root.at(layer), h);
    return h.hex();
  };
  return {hash("definition"), hash("instance"), hash("run")};
}

std::string expected_protocol(const b2json::Value& root, const Layers& layers) {
  // protocol_identifiers (model.rs:16-24)
  const std::string& schema = root.at("schema").str();
  std::string name, encoding;
  if (schema == "atlasir-v1") {
    name = "atlasir";
    encoding = "atlasir-canonical-json-v1";
  } else if (schema == "b2ir-v1" || schema.rfind("b2ir-gate0-probe-v3", 0) == 0) {
    name = "b2ir";
    encoding = "b2ir-canonical-json-v1";
  } else {
    throw b2json::Error("unsupported AtlasIR schema");
  }
  // keys in canonical order
  return "{\"canonical_encoding\":\"" + encoding + "\",\"hash_algorithm\":\"sha256\",\"layers\":{\"definition\":\"" +
         layers.definition + "\",\"instance\":\"" + layers.instance + "\",\"run\":\"" + layers.run +
         "\"},\"name\":\"" + name + "\",\"version\":{\"major\":1,\"minor\":0}}";
}

void verify_protocol(const b2json::Value& root) {
  const b2json::Value* actual = root.find("protocol");
  if (!actual || text(*actual) != expected_protocol(root, layer_hashes(root)))
    throw b2json::Error("AtlasIR canonical layer hash mismatch");
}

bool migrate_probe(b2json::Value& root) {
  // prepare_protocol's predecessor branch (brian2-rust/src/model.rs:4733-4777)
  const std::string schema = root.at("schema").str();
  if (schema != "b2ir-gate0-probe-v34" && schema != "b2ir-gate0-probe-v35" && schema != "b2ir-gate0-probe-v36" &&
      schema != "b2ir-gate0-probe-v37")
    return false;
  if (schema == "b2ir-gate0-probe-v34") {
    if (root.find("protocol")) throw b2json::Error("legacy AtlasIR has a protocol envelope");
  } else {
    verify_protocol(root);
  }
  b2json::Value* definition = root.find_mut("definition");
  b2json::Value* populations = definition ? definition->find_mut("populations") : nullptr;
  if (!populations || !populations->is_array()) throw b2json::Error("legacy AtlasIR has no population table");
  for (auto& population : populations->arr_mut()) {
    if (!population.is_object()) throw b2json::Error("invalid legacy population definition");
    if (!population.find("linked_variables")) population.set("linked_variables", b2json::Value::array());
  }
  b2json::Value* functions = definition->find_mut("functions");
  if (!functions || !functions->is_array()) throw b2json::Error("legacy AtlasIR has no Function table");
  for (auto& function : functions->arr_mut()) {
    if (!function.is_object()) throw b2json::Error("invalid legacy Function definition");
    function.set("abi", b2json::Value::string("b2ir-function-v1"));
    if (!function.find("backend_implementations")) function.set("backend_implementations", b2json::Value::object());
  }
  root.set("schema", b2json::Value::string("atlasir-v1"));
  const std::string protocol = expected_protocol(root, layer_hashes(root));
  root.set("protocol", b2json::parse(protocol.data(), protocol.size()));
  return true;
}

}  // namespace b2canon
