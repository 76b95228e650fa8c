// extern "C" boundary of libb2gpu.so (declarations and reference mapping in
// include/b2gpu.h).
#include "../../include/b2gpu.h"

#include <sys/stat.h>

#include <algorithm>
#include <chrono>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <functional>
#include <fstream>
#include <memory>
#include <string>

#include "common/dump.hpp"
#include "common/canonical.hpp"
#include "common/ir.hpp"
#include "engine/engine.hpp"
#include "engine/spikes.hpp"

struct b2g_engine {
  std::unique_ptr<b2gpu::Engine> engine;
  bool failed = false;
};

namespace {

void set_error(char* error, size_t cap, const std::string& msg) {
  if (!error || cap == 0) return;
  size_t n = std::min(cap - 1, msg.size());
  std::memcpy(error, msg.data(), n);
  error[n] = '\0';
}

template <class F>
int guarded(b2g_engine* e, char* error, size_t cap, F f) {
  if (!e) {
    set_error(error, cap, "null engine");
    return 1;
  }
  if (e->failed) {
    set_error(error, cap, "execution failed; create a new executor");
    return 1;
  }
  try {
    f();
    set_error(error, cap, "");
    return 0;
  } catch (const std::exception& ex) {
    e->failed = true;
    set_error(error, cap, ex.what());
    return 1;
  }
}

// Fields past struct_size keep their defaults (older callers).
constexpr size_t kOptionsV1 = offsetof(b2g_options, rank);

b2gpu::Options to_options(const b2g_options* o) {
  b2gpu::Options opt;
  if (!o) return opt;
  if (o->struct_size < kOptionsV1) throw b2ir::Error("b2g_options.struct_size too small");
  opt.device = o->device;
  if (o->chunk_ticks) opt.chunk_ticks = o->chunk_ticks;
  opt.use_graphs = o->use_graphs != 0;
  opt.ring_capacity = o->ring_capacity;
  if (o->struct_size >= offsetof(b2g_options, reserved0)) {
    opt.rank = o->rank;
    opt.world_size = o->world_size;
    if (o->exchange_timeout_ms) opt.exchange_timeout_ms = o->exchange_timeout_ms;
  }
  return opt;
}

}  // namespace

extern "C" {

void b2g_default_options(b2g_options* o) {
  if (!o) return;
  std::memset(o, 0, sizeof(*o));
  o->struct_size = sizeof(b2g_options);
  o->device = -1;
  o->chunk_ticks = 128;
  o->use_graphs = 1;
}

b2g_engine* b2g_create(const char* json, size_t len, const b2g_options* options, char* error, size_t cap) {
  try {
    if (!json) throw b2ir::Error("null model document");
    b2gpu::Options opt = to_options(options);
    b2ir::Model m = b2ir::load_model(json, len);
    auto e = std::make_unique<b2g_engine>();
    e->engine = std::make_unique<b2gpu::Engine>(m, opt);
    set_error(error, cap, "");
    return e.release();
  } catch (const std::exception& ex) {
    set_error(error, cap, ex.what());
    return nullptr;
  }
}

int b2g_step(b2g_engine* e, uint64_t max_ticks, int* finished, char* error, size_t cap) {
  return guarded(e, error, cap, [&] {
    bool done = e->engine->step(max_ticks);
    if (finished) *finished = done ? 1 : 0;
  });
}

int b2g_write_results(b2g_engine* e, const char* outdir, char* error, size_t cap) {
  return guarded(e, error, cap, [&] {
    if (!outdir) throw b2ir::Error("null output directory");
    auto t0 = std::chrono::steady_clock::now();
    b2dump::ResultSet r = e->engine->results();
    auto sizes = b2dump::write_dumps(r, outdir);
    double dump_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    b2gpu::Stats s = e->engine->stats();
    std::string summary = b2dump::summary_json(r, sizes.first, sizes.second, s.simulation_seconds, dump_seconds);
    std::ofstream f(std::string(outdir) + "/summary.json");
    f << summary;
    if (!f) throw b2ir::Error("cannot write summary.json");
  });
}

int b2g_summary_json(b2g_engine* e, char* buffer, size_t capacity, size_t* length, char* error, size_t cap) {
  return guarded(e, error, cap, [&] {
    if (!length) throw b2ir::Error("null length");
    b2dump::ResultSet r = e->engine->results();
    b2gpu::Stats s = e->engine->stats();
    // the sizes write_results would produce; nothing is written, so no dump time
    const std::string text =
        b2dump::summary_json(r, b2dump::dump_size(r), b2dump::event_dump_size(r), s.simulation_seconds, 0.0);
    *length = text.size();
    if (buffer && capacity) {
      const size_t n = std::min(text.size(), capacity - 1);
      std::memcpy(buffer, text.data(), n);
      buffer[n] = '\0';
    }
  });
}

int b2g_get_stats(const b2g_engine* e, b2g_stats* out, char* error, size_t cap) {
  return guarded(const_cast<b2g_engine*>(e), error, cap, [&] {
    if (!out) throw b2ir::Error("null stats");
    b2gpu::Stats s = e->engine->stats();
    out->ticks = s.ticks;
    out->synaptic_events = s.synaptic_events;
    out->spikes = s.spikes;
    out->kernel_launches = s.kernel_launches;
    out->launches_per_tick = s.launches_per_tick;
    out->simulation_seconds = s.simulation_seconds;
    out->build_seconds = s.build_seconds;
    out->compile_seconds = s.compile_seconds;
    out->device_seconds = s.device_seconds;
    out->h2d_bytes = s.h2d_bytes;
    out->d2h_bytes = s.d2h_bytes;
  });
}

int b2g_profile(b2g_engine* e, uint64_t ticks, b2g_kernel_time* out, size_t capacity, size_t* count, char* error,
                size_t cap) {
  return guarded(e, error, cap, [&] {
    auto times = e->engine->profile(ticks);
    if (count) *count = times.size();
    for (size_t i = 0; i < times.size() && out && i < capacity; ++i) {
      std::memset(out[i].name, 0, sizeof(out[i].name));
      std::strncpy(out[i].name, times[i].name.c_str(), sizeof(out[i].name) - 1);
      out[i].launches = times[i].launches;
      out[i].total_ms = times[i].total_ms;
    }
  });
}

int b2g_read_state(b2g_engine* e, uint32_t population, const char* name, void* dst, size_t capacity, size_t* needed,
                   char* error, size_t cap) {
  return guarded(e, error, cap, [&] {
    std::vector<uint8_t> bytes;
    e->engine->read_state(population, name ? name : "", bytes);
    if (needed) *needed = bytes.size();
    if (dst) {
      if (capacity < bytes.size()) throw b2ir::Error("destination buffer too small");
      std::memcpy(dst, bytes.data(), bytes.size());
    }
  });
}

int b2g_spikes(b2g_engine* e, uint32_t population, uint64_t tick, uint32_t* dst, size_t capacity, size_t* count,
               char* error, size_t cap) {
  return guarded(e, error, cap, [&] {
    std::vector<uint32_t> ids = e->engine->spikes_at(population, tick);
    if (count) *count = ids.size();
    if (dst) {
      if (capacity < ids.size()) throw b2ir::Error("destination buffer too small");
      std::memcpy(dst, ids.data(), ids.size() * 4);
    }
  });
}

int b2g_generated_source(const b2g_engine* e, char* dst, size_t capacity, size_t* needed) {
  if (!e || !e->engine) return 1;
  const std::string& s = e->engine->generated_source();
  if (needed) *needed = s.size() + 1;
  if (dst) {
    if (capacity < s.size() + 1) return 1;
    std::memcpy(dst, s.c_str(), s.size() + 1);
  }
  return 0;
}

int b2g_codegen(const char* json, size_t len, const b2g_options* options, char* dst, size_t capacity, size_t* needed,
                char* error, size_t cap) {
  try {
    if (!json) throw b2ir::Error("null model document");
    b2gpu::Options opt = to_options(options);
    b2ir::Model m = b2ir::load_model(json, len);
    opt.dry_run = true;
    b2gpu::Engine engine(m, opt);
    const std::string& s = engine.generated_source();
    if (needed) *needed = s.size() + 1;
    if (dst) {
      if (capacity < s.size() + 1) throw b2ir::Error("destination buffer too small");
      std::memcpy(dst, s.c_str(), s.size() + 1);
    }
    set_error(error, cap, "");
    return 0;
  } catch (const std::exception& ex) {
    set_error(error, cap, ex.what());
    return 1;
  }
}

void b2g_partition(uint64_t count, int32_t rank, int32_t world_size, uint64_t* lo, uint64_t* hi) {
  uint64_t l = 0, h = 0;
  if (world_size > 0 && rank >= 0 && rank < world_size) {
    // floor(count * r / G) without overflow for any u64 count
    auto at = [&](uint64_t r) {
      const unsigned __int128 x = static_cast<unsigned __int128>(count) * r;
      return static_cast<uint64_t>(x / static_cast<uint64_t>(world_size));
    };
    l = at(uint64_t(rank));
    h = at(uint64_t(rank) + 1);
  }
  if (lo) *lo = l;
  if (hi) *hi = h;
}

int b2g_ipc_handle(b2g_engine* e, void* handle, size_t capacity, size_t* length, char* error, size_t cap) {
  return guarded(e, error, cap, [&] {
    std::vector<uint8_t> h = e->engine->ipc_handle();
    if (length) *length = h.size();
    if (handle) {
      if (capacity < h.size()) throw b2ir::Error("handle buffer too small");
      std::memcpy(handle, h.data(), h.size());
    }
  });
}

int b2g_connect(b2g_engine* e, const void* handles, size_t handle_length, size_t count, char* error, size_t cap) {
  return guarded(e, error, cap, [&] {
    if (!handles) throw b2ir::Error("null handles");
    std::vector<std::vector<uint8_t>> hs(count);
    const uint8_t* b = static_cast<const uint8_t*>(handles);
    for (size_t q = 0; q < count; ++q) hs[q].assign(b + q * handle_length, b + (q + 1) * handle_length);
    e->engine->connect(hs);
  });
}

int b2g_publish_results(b2g_engine* e, char* error, size_t cap) {
  return guarded(e, error, cap, [&] { e->engine->publish(); });
}

size_t b2g_spikes_scratch_bytes(uint64_t nbits) { return std::max<size_t>(16, b2gpu::bitmap_tiles(nbits) * 4); }

int b2g_spikes_from_bitmap(const uint32_t* d_words, uint64_t nbits, uint32_t* d_ids, uint32_t* d_count,
                           void* d_scratch, size_t scratch_bytes, void* stream, char* error, size_t cap) {
  try {
    if (!d_count || (nbits && (!d_words || !d_ids || !d_scratch))) throw b2ir::Error("null device pointer");
    if (scratch_bytes < b2g_spikes_scratch_bytes(nbits)) throw b2ir::Error("scratch buffer too small");
    b2gpu::bitmap_to_spikes(d_words, nbits, d_ids, d_count, static_cast<uint32_t*>(d_scratch),
                            static_cast<cudaStream_t>(stream));
    set_error(error, cap, "");
    return 0;
  } catch (const std::exception& ex) {
    set_error(error, cap, ex.what());
    return 1;
  }
}

int b2g_spikes_from_bitmap_noalloc(const uint32_t* d_words, uint64_t nbits, uint32_t* d_ids, uint32_t* d_count,
                                   void* stream, char* error, size_t cap) {
  static_assert(B2G_SPIKES_NOALLOC_MAX_BITS == b2gpu::kNoAllocMaxBits, "no-alloc limit mismatch");
  try {
    if (!d_count || (nbits && (!d_words || !d_ids))) throw b2ir::Error("null device pointer");
    b2gpu::bitmap_to_spikes_noalloc(d_words, nbits, d_ids, d_count, static_cast<cudaStream_t>(stream));
    set_error(error, cap, "");
    return 0;
  } catch (const std::exception& ex) {
    set_error(error, cap, ex.what());
    return 1;
  }
}

void b2g_destroy(b2g_engine* e) { delete e; }

const char* b2g_version(void) { return "brian2-atlas-b200 0.1 (abi 1, sm_100a)"; }

namespace {

// The runner's opt-in process budgets (brian2-rust/src/resource_limits.rs):
// an environment variable of decimal digits in 1..maximum, else the default.
uint64_t runner_budget(const char* name, uint64_t fallback, uint64_t maximum) {
  const char* text = std::getenv(name);
  if (!text) return fallback;
  const std::string t = text;
  bool digits = !t.empty() && t.size() <= 20;
  for (char c : t) digits &= c >= '0' && c <= '9';
  const uint64_t v = digits ? std::strtoull(t.c_str(), nullptr, 10) : 0;
  b2ir::check(digits && v >= 1 && v <= maximum,
              std::string(name) + " requires decimal digits in 1.." + std::to_string(maximum));
  return v;
}

// Budgets run_cli applies (model.rs:4605-4608 and the model checks they
// feed): IR bytes, neuron count, population steps and neuron-steps, states
// and parameters per population, statements per code object, TimedArray
// values, explicit edges per projection, instance values.
b2ir::Model load_for_runner(const char* path) {
  const uint64_t max_ir = runner_budget("B2_MAX_IR_BYTES", 2048ull * 1048576ull, 64ull * 1073741824ull);
  const uint64_t max_values = runner_budget("B2_MAX_INITIAL_VALUES", 100000000ull, 8000000000ull);
  const uint64_t max_neurons = runner_budget("B2_MAX_NEURONS", 1000000ull, 16000000ull);
  const uint64_t max_steps = runner_budget("B2_MAX_POPULATION_STEPS", 10000000ull, 10000000ull);
  struct stat st;
  b2ir::check(stat(path, &st) == 0, std::string("cannot open ") + path);
  b2ir::check(uint64_t(st.st_size) <= max_ir, "IR exceeds the configured byte budget");
  b2ir::Model m = b2ir::load_model_file(path);
  b2ir::check(m.neuron_count >= 1 && m.neuron_count <= max_neurons, "invalid neuron count");
  const uint64_t max_states = runner_budget("B2_MAX_POPULATION_STATES", 32, 1024);
  const uint64_t max_parameters = runner_budget("B2_MAX_POPULATION_PARAMETERS", 128, 1024);
  const uint64_t max_statements = runner_budget("B2_MAX_STATEMENTS", 128, 1024);
  const uint64_t max_edges = runner_budget("B2_MAX_EXPLICIT_SYNAPSES", 50000000ull, 1000000000ull);
  const uint64_t max_table = runner_budget("B2_MAX_TIMED_ARRAY_VALUES", 10000000ull, 1000000000ull);
  std::function<void(const b2ir::ExprPtr&)> tables = [&](const b2ir::ExprPtr& e) {
    if (!e) return;
    if (e->op == b2ir::Op::TimedArray) b2ir::check(e->ta_values.size() <= max_table, "invalid TimedArray layout");
    for (const auto& a : e->args) tables(a);
  };
  auto statements = [&](const std::vector<b2ir::CodeObject>& codes) {
    for (const auto& c : codes) {
      b2ir::check(c.scalar.size() + c.vector.size() <= max_statements, "too many statements");
      for (const auto* list : {&c.scalar, &c.vector})
        for (const auto& st : *list) tables(st.value);
    }
  };
  for (const auto& f : m.functions) tables(f.body);
  for (const auto& p : m.populations) {
    b2ir::check(p.steps <= max_steps, "positive population dt and valid Clock interval required");
    b2ir::check((unsigned __int128)p.count * p.steps <= 250000000000ull, "probe population duration budget exceeded");
    b2ir::check(p.states.size() <= max_states, "population state arrays do not match definition");
    b2ir::check(p.parameters.size() <= max_parameters, "population parameter arrays do not match definition");
    statements(p.code_objects);
  }
  for (size_t s = 0; s < m.synapses.size(); ++s) {
    const auto& inst = m.synapse_instances[s];
    if (inst.topology.kind == b2ir::Topology::Kind::Explicit)
      b2ir::check(inst.source.size() <= max_edges, "invalid synaptic topology");
    statements(m.synapses[s].code_objects);
  }
  // Instance values counted as the reference's validation counts them:
  // state and parameter arrays, refractory arrays (2 per neuron), generator
  // schedules (2 per spike), explicit edge lists (2 per edge), delay arrays.
  uint64_t values = 0;
  for (size_t p = 0; p < m.populations.size(); ++p) {
    const auto& inst = m.population_instances[p];
    for (const auto* table : {&inst.initial_state, &inst.parameters})
      for (const auto& kv : *table) values += kv.second.size();
    if (inst.refractory) values += 2 * m.populations[p].count;
    if (inst.spike_generator) values += 2 * inst.spike_generator->spike_ticks.size();
  }
  for (const auto& inst : m.synapse_instances) {
    for (const auto* table : {&inst.initial_state, &inst.parameters})
      for (const auto& kv : *table) values += kv.second.size();
    if (inst.topology.kind == b2ir::Topology::Kind::Explicit) values += 2 * inst.source.size();
    for (const auto& pw : inst.pathways) values += pw.delay.size() + pw.delay_ticks.size();
  }
  b2ir::check(values <= max_values, "probe array budget exceeded");
  return m;
}

}  // namespace

int b2g_run_cli(int argc, const char* const* argv) {
  try {
    b2ir::check(argc == 3,
                "usage: b2-runner MODEL.json OUTPUT_DIRECTORY | b2-runner --validate MODEL.json | "
                "b2-runner --canonical-hashes MODEL.json");
    std::string first = argv[1];
    if (first == "--validate") {
      b2ir::Model m = load_for_runner(argv[2]);
      (void)m;
      std::printf("validated AtlasIR\n");
      return 0;
    }
    if (first == "--canonical-hashes") {
      // validated (hashes included) first, then the layers object as
      // run_cli prints it (model.rs:4668-4670): keys in order, compact
      b2ir::Model m = load_for_runner(argv[2]);
      (void)m;
      std::ifstream f(argv[2], std::ios::binary);
      std::string data((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
      b2json::Value doc = b2json::parse(data.data(), data.size());
      b2canon::migrate_probe(doc);  // hashes of the migrated layers, as the reference prints them
      const b2canon::Layers h = b2canon::layer_hashes(doc);
      std::printf("{\"definition\":\"%s\",\"instance\":\"%s\",\"run\":\"%s\"}\n", h.definition.c_str(),
                  h.instance.c_str(), h.run.c_str());
      return 0;
    }
    b2ir::check(first.rfind("--", 0) != 0, "unknown b2-runner option");
    struct stat st;
    b2ir::check(stat(argv[2], &st) != 0, "output directory already exists; choose a new directory");
    b2ir::Model m = load_for_runner(argv[1]);
    b2gpu::Options opt;
    b2gpu::Engine engine(m, opt);
    engine.step(UINT64_MAX);
    b2ir::check(mkdir(argv[2], 0777) == 0, "cannot create output directory");
    auto t0 = std::chrono::steady_clock::now();
    b2dump::ResultSet r = engine.results();
    auto sizes = b2dump::write_dumps(r, argv[2]);
    double dump_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    b2gpu::Stats s = engine.stats();
    std::ofstream(std::string(argv[2]) + "/summary.json")
        << b2dump::summary_json(r, sizes.first, sizes.second, s.simulation_seconds, dump_seconds);
    std::printf("completed %zu populations for %llu neurons\n", r.populations.size(),
                (unsigned long long)r.neuron_count);
    return 0;
  } catch (const std::exception& ex) {
    std::fprintf(stderr, "b2-runner: %s\n", ex.what());
    return 1;
  }
}

}  // extern "C"
