// B2DMP001 / B2EVT001 / summary.json writers; layout per
// brian2-rust/src/executor.rs:3142-3405 and 4749-4824.
#include "dump.hpp"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>

namespace b2dump {

namespace {

class Writer {
 public:
  explicit Writer(const std::string& path) : out_(path, std::ios::binary) {
    b2ir::check(bool(out_), "cannot create '" + path + "'");
  }
  void bytes(const void* data, size_t n) {
    if (n) out_.write(static_cast<const char*>(data), std::streamsize(n));
    written_ += n;
  }
  void u64(uint64_t v) { bytes(&v, 8); }  // host is little-endian (x86_64 / aarch64)
  void f64(double v) { bytes(&v, 8); }
  void pairs(const std::vector<TickIndex>& v) {
    for (const auto& p : v) {
      int64_t t = int64_t(p.first), i = int64_t(p.second);
      bytes(&t, 8);
      bytes(&i, 8);
    }
  }
  void indices(const std::vector<uint64_t>& v) {
    for (uint64_t x : v) {
      int64_t y = int64_t(x);
      bytes(&y, 8);
    }
  }
  void column(const Column& c) { bytes(c.bytes.data(), c.bytes.size()); }
  uint64_t finish() {
    out_.flush();
    b2ir::check(bool(out_), "result write failed");
    return written_;
  }

 private:
  std::ofstream out_;
  uint64_t written_ = 0;
};

uint64_t column_bytes(const std::vector<Column>& cs) {
  uint64_t s = 0;
  for (const auto& c : cs) s += c.bytes.size();
  return s;
}

}  // namespace

uint64_t dump_size(const ResultSet& r) {
  uint64_t size = 40;
  for (const auto& p : r.populations) {
    size += 64 + column_bytes(p.samples) + p.spikes.size() * 16 + p.counts.size() * 8 +
            p.last_fired.size() * 8 + column_bytes(p.states);
    if (p.has_refractory) size += p.lastspike.size() * 8 + p.not_refractory.size();
  }
  size += 24;
  for (const auto& s : r.synapses) size += 24 + column_bytes(s.states) + column_bytes(s.monitor_samples);
  return size;
}

uint64_t event_dump_size(const ResultSet& r) {
  if (!r.has_events) return 0;
  uint64_t size = 32;
  for (const auto& p : r.populations)
    for (const auto& h : p.event_history) size += 8 + h.size() * 16;
  for (const auto& p : r.populations)
    for (const auto& m : p.event_monitors) size += 16 + m.events.size() * 16 + column_bytes(m.samples);
  return size;
}

std::pair<uint64_t, uint64_t> write_dumps(const ResultSet& r, const std::string& directory) {
  const uint64_t size = dump_size(r);
  Writer w(directory + "/results.bin");
  w.bytes("B2DMP001", 8);
  uint32_t version = 3, marker = 0x01020304u;
  w.bytes(&version, 4);
  w.bytes(&marker, 4);
  w.u64(r.populations.size());
  w.u64(r.neuron_count);
  w.u64(size);
  for (const auto& p : r.populations) {
    w.u64(p.count);
    w.u64(p.steps);
    w.u64(p.record_count);
    w.u64(p.variable_count);
    w.u64(p.states.size());
    w.u64(p.spikes.size());
    w.u64(p.last_fired.size());
    w.u64(p.has_refractory ? 1 : 0);
    for (const auto& c : p.samples) w.column(c);
    w.pairs(p.spikes);
    w.indices(p.counts);
    w.indices(p.last_fired);
    for (const auto& c : p.states) w.column(c);
    if (p.has_refractory) {
      for (double x : p.lastspike) w.f64(x);
      w.bytes(p.not_refractory.data(), p.not_refractory.size());
    }
  }
  w.u64(r.synapses.size());
  for (const auto& s : r.synapses) {
    w.u64(s.states.size());
    w.u64(s.edge_count);
    for (const auto& c : s.states) w.column(c);
    for (const auto& c : s.monitor_samples) w.column(c);
    w.u64(s.delivered);
  }
  w.f64(r.final_time);
  w.bytes("B2END001", 8);
  uint64_t written = w.finish();
  b2ir::check(written == size, "result dump size mismatch");

  uint64_t event_bytes = 0;
  if (r.has_events) {
    const uint64_t esize = event_dump_size(r);
    Writer e(directory + "/events.bin");
    e.bytes("B2EVT001", 8);
    uint64_t streams = 0, monitors = 0;
    for (const auto& p : r.populations) {
      streams += p.event_history.size();
      monitors += p.event_monitors.size();
    }
    e.u64(streams);
    for (const auto& p : r.populations)
      for (const auto& h : p.event_history) {
        e.u64(h.size());
        e.pairs(h);
      }
    e.u64(monitors);
    for (const auto& p : r.populations)
      for (const auto& m : p.event_monitors) {
        e.u64(m.events.size());
        e.u64(m.samples.size());
        e.pairs(m.events);
        for (const auto& c : m.samples) e.column(c);
      }
    e.bytes("B2EEND01", 8);
    event_bytes = e.finish();
    b2ir::check(event_bytes == esize, "event monitor dump size mismatch");
  }
  return {written, event_bytes};
}

std::string format_double(double v) {
  if (!std::isfinite(v)) return "null";
  if (v == std::floor(v) && std::fabs(v) < 1e16) {
    char buf[64];
    std::snprintf(buf, sizeof buf, "%.1f", v);
    return buf;
  }
  char buf[64];
  for (int prec = 1; prec <= 17; ++prec) {
    std::snprintf(buf, sizeof buf, "%.*g", prec, v);
    if (std::strtod(buf, nullptr) == v) break;
  }
  std::string s = buf;
  // serde_json (ryu) prints exponents as e-7 / e16 without zero padding or '+'.
  auto e = s.find('e');
  if (e != std::string::npos) {
    std::string mant = s.substr(0, e), ex = s.substr(e + 1);
    bool neg = !ex.empty() && ex[0] == '-';
    size_t i = (ex[0] == '-' || ex[0] == '+') ? 1 : 0;
    while (i + 1 < ex.size() && ex[i] == '0') ++i;
    s = mant + "e" + (neg ? "-" : "") + ex.substr(i);
  }
  return s;
}

std::string summary_json(const ResultSet& r, uint64_t dump_bytes, uint64_t event_dump_bytes,
                         double simulation_seconds, double dump_seconds,
                         const std::vector<std::pair<std::string, std::string>>& extra) {
  uint64_t spikes = 0, events = 0;
  for (const auto& p : r.populations) spikes += p.spikes.size();
  for (const auto& s : r.synapses) events += s.delivered;
  std::ostringstream o;
  o << "{\n";
  o << "  \"dump_bytes\": " << dump_bytes << ",\n";
  o << "  \"event_dump_bytes\": " << event_dump_bytes << ",\n";
  for (const auto& kv : extra)
    if (kv.first < "final_time_seconds") o << "  \"" << kv.first << "\": " << kv.second << ",\n";
  o << "  \"final_time_seconds\": " << format_double(r.final_time) << ",\n";
  o << "  \"neuron_count\": " << r.neuron_count << ",\n";
  o << "  \"population_count\": " << r.populations.size() << ",\n";
  o << "  \"schema\": \"b2-result-dump-v3\",\n";
  o << "  \"spike_count\": " << spikes << ",\n";
  o << "  \"synaptic_events\": " << events << ",\n";
  o << "  \"timings\": {\n";
  o << "    \"dump_write_seconds\": " << format_double(dump_seconds) << ",\n";
  o << "    \"simulation_and_recording_seconds\": " << format_double(simulation_seconds) << "\n";
  o << "  }";
  for (const auto& kv : extra)
    if (!(kv.first < "final_time_seconds")) o << ",\n  \"" << kv.first << "\": " << kv.second;
  o << "\n}\n";
  return o.str();
}

}  // namespace b2dump
