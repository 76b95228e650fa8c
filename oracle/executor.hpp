// ORACLE (test infrastructure only): a single-threaded CPU restatement of the
// reference executor `b2-runner` (brian2-rust/src/executor.rs) for the
// per-tick simulation path.  It is the parity checker for the GPU engine and the
// timed CPU baseline in bench.py; the product never links or calls it.
//
// Parity pin: tests/test_oracle_golden.py checks it byte for byte against the
// reference's own golden b2-runner output
// (brian2-rust/tests/fixtures/reference-v1/reference/{results,events}.bin).
#pragma once

#include <string>

#include "../brian2-atlas_b200/csrc/common/dump.hpp"
#include "../brian2-atlas_b200/csrc/common/ir.hpp"

namespace oracle {

struct RunStats {
  double simulation_seconds = 0.0;
  uint64_t ticks = 0;
};

// Execute the whole run (executor.rs:4774 `execute`, minus file output).
b2dump::ResultSet execute(const b2ir::Model& model, RunStats* stats = nullptr,
                          uint64_t max_ticks = UINT64_MAX);

// Timing harness for the CPU baseline: build once, run `warmup` ticks, then
// time `timed` ticks; returns the synaptic events and spikes of the timed part.
struct TimedSample {
  uint64_t ticks = 0, synaptic_events = 0, spikes = 0;
  double build_seconds = 0.0, seconds = 0.0;
};
TimedSample timed_sample(const b2ir::Model& model, uint64_t warmup, uint64_t timed);

}  // namespace oracle
