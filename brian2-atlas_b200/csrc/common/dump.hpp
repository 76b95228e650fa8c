// Result writers for the b2-runner output contract:
//   results.bin  `B2DMP001` version 3 (brian2-rust/src/executor.rs:3142-3339)
//   events.bin   `B2EVT001`          (executor.rs:3341-3405)
//   summary.json                     (executor.rs:4749-4824)
// Both the CPU oracle and the GPU engine fill a ResultSet and hand it here, so
// the byte layout lives in exactly one place.
#pragma once

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "ir.hpp"

namespace b2dump {

// A typed little-endian array exactly as the reference `StateArray::dump`
// writes it: bool as u8, f32/i32/u32 as 4 bytes, f64/i64/u64 as 8 bytes.
struct Column {
  b2ir::DType dtype = b2ir::DType::F64;
  std::vector<uint8_t> bytes;
  size_t size() const { return bytes.size() / b2ir::dtype_bytes(dtype); }
};

using TickIndex = std::pair<uint64_t, uint64_t>;  // (tick, neuron)

struct EventMonitorResult {
  std::vector<TickIndex> events;
  std::vector<Column> samples;
};

struct PopulationResult {
  uint64_t count = 0, steps = 0;
  uint64_t record_count = 0, variable_count = 0;
  std::vector<Column> samples;            // one per monitor variable
  std::vector<TickIndex> spikes;          // SpikeMonitor list
  std::vector<uint64_t> counts;           // SpikeMonitor per-neuron counts
  std::vector<uint64_t> last_fired;       // spikes of the final tick
  std::vector<Column> states;             // final state, definition order
  bool has_refractory = false;
  std::vector<double> lastspike;
  std::vector<uint8_t> not_refractory;
  std::vector<std::vector<TickIndex>> event_history;  // one per event stream
  std::vector<EventMonitorResult> event_monitors;
};

struct SynapseResult {
  uint64_t edge_count = 0;
  std::vector<Column> states;
  std::vector<Column> monitor_samples;
  uint64_t delivered = 0;
};

struct ResultSet {
  uint64_t neuron_count = 0;
  double final_time = 0.0;
  bool has_events = false;  // any population with event streams or event monitors
  std::vector<PopulationResult> populations;
  std::vector<SynapseResult> synapses;
};

// Size of results.bin as the reference precomputes it (dump_size, :3252).
uint64_t dump_size(const ResultSet& r);
uint64_t event_dump_size(const ResultSet& r);

// Write results.bin / events.bin into `directory` (which must exist) and
// return the byte counts.  Throws b2ir::Error on I/O failure or a size
// mismatch against the precomputed size.
std::pair<uint64_t, uint64_t> write_dumps(const ResultSet& r, const std::string& directory);

// summary.json with the reference's keys (serde_json pretty, sorted keys).
std::string summary_json(const ResultSet& r, uint64_t dump_bytes, uint64_t event_dump_bytes,
                         double simulation_seconds, double dump_seconds,
                         const std::vector<std::pair<std::string, std::string>>& extra = {});

// Shortest round-trip decimal text of a finite double, serde_json style.
std::string format_double(double v);

}  // namespace b2dump
