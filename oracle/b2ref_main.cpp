// ORACLE (test infrastructure only): command-line front end of the CPU
// restatement, with the b2-runner argv/exit/output contract
// (brian2-rust/src/model.rs:4596-4677, main.rs:2-7):
//
//   b2ref MODEL.json OUTDIR            full run, writes results.bin/events.bin/summary.json
//   b2ref --sample K MODEL.json        run at most K ticks, print one JSON line of
//                                      {"ticks","synaptic_events","simulation_seconds"}
//                                      (bench.py's bounded CPU baseline)
#include <sys/stat.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>

#include "executor.hpp"

int main(int argc, char** argv) {
  try {
    if (argc == 5 && std::strcmp(argv[1], "--timed") == 0) {
      // b2ref --timed WARMUP_TICKS TIMED_TICKS MODEL.json
      b2ir::Model m = b2ir::load_model_file(argv[4]);
      oracle::TimedSample s = oracle::timed_sample(m, std::stoull(argv[2]), std::stoull(argv[3]));
      std::printf("{\"ticks\": %llu, \"synaptic_events\": %llu, \"spikes\": %llu, \"seconds\": %.9f, "
                  "\"build_seconds\": %.6f}\n",
                  (unsigned long long)s.ticks, (unsigned long long)s.synaptic_events,
                  (unsigned long long)s.spikes, s.seconds, s.build_seconds);
      return 0;
    }
    if (argc == 4 && std::strcmp(argv[1], "--sample") == 0) {
      uint64_t k = std::stoull(argv[2]);
      b2ir::Model m = b2ir::load_model_file(argv[3]);
      oracle::RunStats stats;
      b2dump::ResultSet r = oracle::execute(m, &stats, k);
      uint64_t events = 0, spikes = 0;
      for (const auto& s : r.synapses) events += s.delivered;
      for (const auto& p : r.populations) spikes += p.spikes.size();
      std::printf("{\"ticks\": %llu, \"synaptic_events\": %llu, \"spikes\": %llu, \"simulation_seconds\": %.9f}\n",
                  (unsigned long long)stats.ticks, (unsigned long long)events, (unsigned long long)spikes,
                  stats.simulation_seconds);
      return 0;
    }
    b2ir::check(argc == 3, "usage: b2ref MODEL.json OUTPUT_DIRECTORY | b2ref --sample TICKS MODEL.json");
    b2ir::check(argv[1][0] != '-' || argv[1][1] != '-', "unknown option");
    struct stat st;
    b2ir::check(stat(argv[2], &st) != 0, "output directory already exists; choose a new directory");
    b2ir::Model m = b2ir::load_model_file(argv[1]);
    oracle::RunStats stats;
    b2dump::ResultSet r = oracle::execute(m, &stats);
    b2ir::check(mkdir(argv[2], 0777) == 0, "cannot create output directory");
    auto t0 = std::chrono::steady_clock::now();
    auto sizes = b2dump::write_dumps(r, argv[2]);
    double dump_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::string summary = b2dump::summary_json(r, sizes.first, sizes.second, stats.simulation_seconds, dump_seconds);
    std::ofstream(std::string(argv[2]) + "/summary.json") << summary;
    std::printf("completed %zu populations for %llu neurons\n", r.populations.size(),
                (unsigned long long)r.neuron_count);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "b2ref: %s\n", e.what());
    return 1;
  }
}
