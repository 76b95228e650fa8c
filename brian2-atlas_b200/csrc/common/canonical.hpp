// Canonical JSON and SHA-256 layer hashes of AtlasIR documents.
//
// The reference identifies the three layers of a document (definition,
// instance, run) by the SHA-256 of their canonical JSON text and refuses to
// run a document whose `protocol.layers` disagree ("AtlasIR canonical layer
// hash mismatch", brian2-rust/src/model.rs:4656-4661, 4677-4795).  The
// canonical text (brian2-rust/src/canonical.rs) is what Python's
// json.dumps(sort_keys=True, separators=(",", ":"), ensure_ascii=False)
// writes: object keys in code-point order, no whitespace, integers in
// decimal, reals in Python's repr format, strings with JSON's minimal
// escapes and raw UTF-8.
#pragma once

#include <array>
#include <cstdint>
#include <string>

#include "json.hpp"

namespace b2canon {

// SHA-256 (FIPS 180-4), streaming.
class Sha256 {
 public:
  Sha256();
  void update(const void* data, size_t n);
  void update(const std::string& s) { update(s.data(), s.size()); }
  std::array<uint8_t, 32> digest();
  std::string hex();

 private:
  void block(const uint8_t* p);
  uint32_t h_[8];
  uint8_t buf_[64];
  size_t fill_ = 0;
  uint64_t bytes_ = 0;
};

// Canonical text of a JSON value, streamed into `out` (a Sha256 or a string).
void write(const b2json::Value& v, Sha256& out);
std::string text(const b2json::Value& v);

// Python repr() of a double (shortest round-trip digits; fixed notation for
// decimal exponents -4..15, else d.ddde+XX).
std::string python_float(double v);

struct Layers {
  std::string definition, instance, run;
};
Layers layer_hashes(const b2json::Value& root);

// The reference's expected `protocol` envelope for a document with this
// schema, as canonical text; throws for an unknown schema.
std::string expected_protocol(const b2json::Value& root, const Layers& layers);

// Throws "AtlasIR canonical layer hash mismatch" unless root.protocol equals
// the expected envelope.
void verify_protocol(const b2json::Value& root);

// Migrates a b2ir-gate0-probe-v34..v37 document in place to atlasir-v1 as
// the reference does before hashing (v34: no envelope allowed; v35..v37:
// envelope verified first; populations gain `linked_variables: []`, functions
// the `b2ir-function-v1` ABI and empty `backend_implementations`; the
// envelope is recomputed).  Returns false for any other schema.
bool migrate_probe(b2json::Value& root);

}  // namespace b2canon
