// B200 engine for the AtlasIR per-tick hot path.
//
// One Engine owns one GPU (one process per GPU; ranks exchange spikes over
// NCCL).  Construction turns a validated b2ir::Model into:
//   * SoA device state (native storage dtypes), refractory arrays, parameters;
//   * per pathway a source-major (pre) or target-major (post) CSR whose row
//     order is the reference's edge creation order (edge_csr,
//     brian2-rust/src/executor.rs:6168-6183);
//   * per event stream a device spike ring: the ascending fired list of every
//     tick is appended once and read in place by pathways of any delay, which
//     replaces the reference's PathwayQueue ring (executor.rs:6160-6212);
//   * one NVRTC-compiled sm_100a module with fused kernels per schedule step.
// step() replays CUDA graphs of `chunk_ticks` ticks; the tick cursor lives in
// device memory (RunCtl), so one instantiated graph serves every chunk.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../common/dump.hpp"
#include "../common/ir.hpp"
#include "program.hpp"

namespace b2gpu {

struct Options {
  int device = -1;              // -1: current device
  uint32_t chunk_ticks = 128;   // ticks per CUDA-graph replay
  uint64_t ring_capacity = 0;   // spike ring entries per event stream (0: automatic)
  // Multi-GPU: this engine is rank `rank` of `world_size` processes, one per
  // GPU, each owning a contiguous block of every population (the reference's
  // owner rule, brian2_rust/distributed.py:80-81).  Spikes travel between
  // GPUs inside the tick kernels; exchange waits give up after
  // exchange_timeout_ms and poison the engine.
  int rank = 0, world_size = 1;
  uint32_t exchange_timeout_ms = 10000;
  bool use_graphs = true;
  bool verbose = false;
  unsigned neurons_per_thread = 0;  // 1, 2 or 4 (0: default 4)
  // Build the plan and compile the generated kernels for sm_100a without
  // touching a GPU (device pointers are placeholders).  step() is disabled.
  bool dry_run = false;
};

struct Stats {
  uint64_t ticks = 0;
  uint64_t synaptic_events = 0;
  uint64_t spikes = 0;
  uint64_t kernel_launches = 0;      // launches of this engine's kernels
  uint64_t launches_per_tick = 0;
  double simulation_seconds = 0.0;   // wall time of step() calls
  double device_seconds = 0.0;       // CUDA-event time of the tick kernels
  double build_seconds = 0.0;        // topology + compile
  double compile_seconds = 0.0;
  uint64_t h2d_bytes = 0;            // host->device bytes moved by step()
  uint64_t d2h_bytes = 0;            // device->host bytes moved by step() (spike drain)
};

struct KernelTime {
  std::string name;
  uint64_t launches = 0;
  double total_ms = 0.0;
};

struct DeviceBuffer {
  void* ptr = nullptr;
  size_t bytes = 0;
  DeviceBuffer() = default;
  explicit DeviceBuffer(size_t n);
  ~DeviceBuffer();
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  DeviceBuffer(DeviceBuffer&& o) noexcept;
  DeviceBuffer& operator=(DeviceBuffer&& o) noexcept;
  template <class T> T* as() const { return static_cast<T*>(ptr); }
};

class Engine {
 public:
  Engine(const b2ir::Model& model, const Options& options);
  ~Engine();
  Engine(const Engine&) = delete;
  Engine& operator=(const Engine&) = delete;

  // Advance at most max_ticks ticks; returns true when the run is complete.
  bool step(uint64_t max_ticks);
  bool finished() const;
  b2dump::ResultSet results();
  Stats stats() const;
  const std::string& generated_source() const;
  // Copy a population state array (native storage bytes) to host memory.
  void read_state(size_t population, const std::string& name, std::vector<uint8_t>& out);
  // Spike ids of one tick of a population's `spike` stream (host copy).
  std::vector<uint32_t> spikes_at(size_t population, uint64_t tick) const;
  // Advance `ticks` ticks launching each kernel directly with CUDA events
  // around it on the engine stream; returns per-kernel launch counts and time.
  std::vector<KernelTime> profile(uint64_t ticks);

  // ---- multi-GPU (world_size > 1)
  // CUDA IPC handle (opaque bytes) of this rank's shared allocation: the
  // spike-exchange buffers every peer writes into and the staging area rank 0
  // reads results from.
  std::vector<uint8_t> ipc_handle() const;
  // Map every other rank's shared allocation; `handles` holds every rank's
  // ipc_handle() in rank order.  Must precede the first step().
  void connect(const std::vector<std::vector<uint8_t>>& handles);
  // Copy this rank's final local results (state, monitors, event counters)
  // into its staging area.  Every rank publishes, the ranks synchronise on
  // the host, and then rank 0's results() merges all ranks' staging areas.
  void publish();
  // Global index range [lo, hi) of `population` owned by this rank.
  std::pair<uint64_t, uint64_t> owned_range(size_t population) const;

  struct Impl;

 private:
  std::unique_ptr<Impl> impl_;
};

}  // namespace b2gpu
