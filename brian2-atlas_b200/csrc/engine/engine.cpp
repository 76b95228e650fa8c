// B200 engine: plan construction, kernel generation, device state, tick loop.
// Reference semantics: brian2-rust/src/executor.rs `Runtime::new` (:3473-3901)
// and `Runtime::advance` (:3927-4360).
//
// Engine::Impl, in file order:
//   checks        capability errors before any device work
//   populations   SoA state, parameters, event streams, monitors, partition
//                 (target-owned blocks, replicated populations)
//   synapses      CSRs (explicit, binary, procedural on the device), per-edge
//                 state and parameters, delays, pending events, summed rows
//   streams       spike rings, exchange buffers, result staging layout
//   codegen       per-model CUDA source: step kernels (update, threshold,
//                 compaction, reset), pathway kernels (constant-addend
//                 atomics, edge-parallel, target-ordered buckets and scan,
//                 serial fold), summed variables, synapse programs,
//                 monitors, the multi-GPU exchange
//   plan          schedule analysis: fusion, deferral, merging, one launch
//                 per tick node
//   compile/run   NVRTC for sm_100a, CUDA graphs of chunk ticks with
//                 programmatic dependent launch, drains, error words
//   results       the reference's dump layout, multi-GPU merge on rank 0
#include "engine.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <optional>
#include <cstdio>
#include <cstring>
#include <functional>
#include <set>
#include <sstream>
#include <unordered_map>
#include <unordered_set>

#include "cuda_util.hpp"
#include "topology.hpp"

namespace b2gpu {

extern const char* const kDeviceLibSource;  // device_lib.cuh, embedded at build time

using b2ir::check;
using b2ir::Error;

// ------------------------------------------------------- host initializers
namespace {

// Topology counter draws (brian2-rust/src/large_topology.rs; the device
// generators in topology.cu use the same constants and steps).
uint64_t host_topo_draw(uint64_t seed, uint64_t stream, uint64_t edge, uint64_t attempt) {
  uint64_t v = seed ^ (stream * 0xd2b74407b1ce6e93ull) ^ (edge * 0x9e3779b97f4a7c15ull) ^
               (attempt * 0xca5a826395121157ull);
  v += 0x9e3779b97f4a7c15ull;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

double host_topo_unit(uint64_t seed, uint64_t stream, uint64_t edge, uint64_t attempt) {
  return (double(host_topo_draw(seed, stream, edge, attempt) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

// Clipped-normal per-edge values (materialize_initializer and
// materialize_delay_initializer, brian2-rust/src/executor.rs:120-188): per
// edge the first of up to 1000 Box-Muller draws (u1 on `stream`, u2 on
// `stream + 1`; sqrt, log and cos are the host's, as the reference's f64
// calls) that lies in [minimum, maximum].  Delays clip the bounds to
// [max(minimum, 0), maximum or dt * 1e6].  Host arithmetic keeps the values
// bit-identical to the reference's; the edge count is that of one projection.
std::vector<double> clipped_normal_host(uint64_t n, uint64_t seed, const b2ir::Initializer& in,
                                        std::optional<double> delay_dt) {
  std::optional<double> lo = in.minimum, hi = in.maximum;
  if (delay_dt) {
    lo = std::fmax(lo.value_or(0.0), 0.0);
    hi = hi.value_or(*delay_dt * 1000000.0);
  }
  std::vector<double> out(n);
  for (uint64_t e = 0; e < n; ++e) {
    bool found = false;
    for (uint64_t attempt = 0; attempt < 1000 && !found; ++attempt) {
      const double u1 = host_topo_unit(seed, in.stream, e, attempt * 2);
      const double u2 = host_topo_unit(seed, in.stream + 1, e, attempt * 2 + 1);
      const double v = in.mean + in.std * (std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
      if ((!lo || v >= *lo) && (!hi || v <= *hi)) {
        out[e] = v;
        found = true;
      }
    }
    check(found, "clipped-normal rejection limit exceeded");
  }
  return out;
}

}  // namespace

// ------------------------------------------------------------------ buffers
DeviceBuffer::DeviceBuffer(size_t n) : bytes(n) {
  if (n) B2_CUDA(cudaMalloc(&ptr, n));
}
DeviceBuffer::~DeviceBuffer() {
  if (ptr) cudaFree(ptr);
}
DeviceBuffer::DeviceBuffer(DeviceBuffer&& o) noexcept : ptr(o.ptr), bytes(o.bytes) {
  o.ptr = nullptr;
  o.bytes = 0;
}
DeviceBuffer& DeviceBuffer::operator=(DeviceBuffer&& o) noexcept {
  if (this != &o) {
    if (ptr) cudaFree(ptr);
    ptr = o.ptr;
    bytes = o.bytes;
    o.ptr = nullptr;
    o.bytes = 0;
  }
  return *this;
}

namespace {

constexpr unsigned kThreads = 256;
constexpr unsigned kMaxNpt = 4;                 // neurons per thread in neuron kernels (1, 2 or 4)

constexpr unsigned kScatterUnroll = 1;          // default row entries per thread per scatter work item
static_assert(kMaxNpt * (kThreads / 32) <= 32, "one warp scans the per-(kk, warp) spike counts");

// Smallest double d >= 0 with (d + 1e-3*dt) / dt >= target, evaluated in
// IEEE f64 exactly as Brian2 timestep() does (model.rs:981-992).  The map is
// monotone in d, so a bisection over the ordered bit patterns of
// non-negative doubles finds the threshold.
double timestep_threshold(double dt, double target) {
  auto steps = [dt](double d) {
    volatile double x = d + 1e-3 * dt;
    return x / dt;
  };
  auto bits = [](double v) {
    uint64_t r;
    std::memcpy(&r, &v, 8);
    return r;
  };
  auto value = [](uint64_t r) {
    double v;
    std::memcpy(&v, &r, 8);
    return v;
  };
  if (steps(0.0) >= target) return 0.0;
  uint64_t lo = bits(0.0), hi = bits(1.7976931348623157e308);
  if (!(steps(value(hi)) >= target)) return INFINITY;
  while (hi - lo > 1) {
    uint64_t mid = lo + (hi - lo) / 2;
    if (steps(value(mid)) >= target) hi = mid;
    else lo = mid;
  }
  return value(hi);
}


constexpr uint32_t kErrNonfinite = 0x1, kErrTimestep = 0x2, kErrBinomial = 0x4, kErrPoisson = 0x8,
                   kErrRing = 0x10, kErrIntDiv = 0x40, kErrTimedArray = 0x80,
                   kErrCast = 0x100, kErrExchange = 0x200, kErrBarrier = 0x400;

std::string error_message(uint32_t e) {
  if (e & kErrNonfinite) return "non-finite numeric value";
  if (e & kErrTimestep) return "timestep outside Brian2 int64 range";
  if (e & kErrBinomial) return "invalid binomial probability";
  if (e & kErrPoisson) return "invalid poisson lambda";
  if (e & kErrIntDiv) return "integer division by zero";
  if (e & kErrTimedArray) return "TimedArray index/value outside supported range";
  if (e & kErrCast) return "unsupported cast source";
  if (e & kErrRing) return "spike ring overflow (raise the ring capacity)";
  if (e & kErrExchange) return "spike exchange with a peer GPU timed out (a rank stopped or fell behind)";
  if (e & kErrBarrier) return "grid barrier of the tick kernel timed out";
  return "device error";
}

std::string sanitize(const std::string& s) {
  std::string o;
  for (char c : s) o.push_back(std::isalnum((unsigned char)c) ? c : '_');
  return o.substr(0, 40);
}

uint64_t next_pow2(uint64_t v) {
  uint64_t p = 1;
  while (p < v) p <<= 1;
  return p;
}

std::string u64lit(uint64_t v) { return std::to_string(v) + "ull"; }

struct NodeEffects {
  std::set<std::string> reads, writes;
};

bool conflicts(const NodeEffects& a, const NodeEffects& b) {
  for (const auto& w : a.writes)
    if (b.reads.count(w) || b.writes.count(w)) return true;
  for (const auto& w : b.writes)
    if (a.reads.count(w)) return true;
  return false;
}

}  // namespace

// ------------------------------------------------------------------ impl
// Blocks of a stand-alone list-layout kernel (gen_consumer): each reads every
// tile count of the tick and copies its share of the list into the ring.
constexpr unsigned kLayoutBlocks = 16;
// One GPU: populations of at least this many step tiles get a layout kernel.
constexpr size_t kLayoutMinTiles = 1024;
// Blocks of a presynaptic replicate kernel (each writes one flag per rank).
constexpr unsigned kReplicaBlocks = 8;

struct Engine::Impl {
  b2ir::Model m;
  Options opt;
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaLibrary_t module = nullptr;
  std::vector<DeviceBuffer> owned;
  std::vector<uint64_t> ptrs;  // device pointer table (__constant__ g_ptr)
  DeviceBuffer ctl;
  std::string source;
  Stats st;

  // ---- populations
  struct Slot {  // one state variable of a population
    DType dtype;
    int ptr;
  };
  struct EventStreamDev {
    size_t pop = 0, event = 0;
    uint64_t cap = 0, mask = 0;
    int ring = -1, tick_start = -1, tile_count = -1, stage = -1, done = -1;
    bool produced = false, ascending = true;
    size_t max_delay = 0;  // deepest consumer delay
    // multi-GPU: every rank's ascending list of its block's spikes arrives
    // in the inbox (offset x_off of each rank's shared allocation; g_ptr slot
    // xptr[q] is rank q's inbox), two halves of x_half words used on
    // alternate ticks; a receive kernel (alone or fused with the delay-0
    // scatter) lays them out as the tick's ascending global list.
    bool exchanged = false;
    // multi-GPU: a partitioned population's list that only its own rank
    // consumes (on_post rows over the rank's targets, resets, results) stays
    // local: no exchange wait; rank 0 merges every rank's drained list for
    // the results (global ids, rank order = ascending order)
    bool local = false;
    size_t x_off = 0;
    std::vector<int> xptr;
    // Inbox layout (words per parity half, x_half in all): rank q's region
    // starts at word x_base[q] with the count words of its x_tiles[q] tiles
    // (adjacent, so a reader loads them coalesced), followed by room for
    // x_tile_n[q] ids per tile.  A producing block publishes its tile's count
    // and ids as soon as it has compacted them.
    uint64_t x_half = 0;
    std::vector<uint64_t> x_tiles, x_tile_n, x_base;
    // The producing step leaves the tick's list as per-tile counts and ids
    // (tile_count and stage, or the inboxes) and the first kernel that reads
    // the list lays it out in the ring (gen_consumer): single GPU when a
    // delay-0 constant-addend scatter directly follows the step, and every
    // exchanged list.
    bool consumer_layout = false;
    // fired bitmap ring for target-ordered pathways: slot rel % bm_slots holds
    // the tick's ballot words (bit i = neuron i fired), written by the step
    // kernel that produces the stream
    bool needs_bitmap = false;
    int bitmap = -1;
    uint64_t bm_words = 0, bm_slots = 0;
    // host copy of drained spikes
    std::vector<uint32_t> ids;
    std::vector<uint64_t> starts;  // host positions per tick: starts[rel] .. starts[rel+1]
    uint64_t drained_pos = 0;
  };
  struct PopDev {
    size_t count = 0, start_tick = 0, end_tick = 0, steps = 0;  // count: neurons owned by this rank
    uint64_t lo = 0, global_count = 0;                            // owned block [lo, lo + count)
    // multi-GPU: every rank evaluates the whole population (no synapse
    // targets it, so its evolution depends on its own state and counter-based
    // draws only); its event lists are complete on every rank without an
    // exchange, and rank 0 stages its results
    bool replicated = false;
    double dt = 0.0;
    std::vector<Slot> states;
    int lastspike = -1, not_refractory = -1;
    uint64_t period_ticks = 0;
    bool fixed_refractory = false;
    std::map<std::string, int> param_ptr;      // per-neuron parameter arrays
    std::map<std::string, double> param_const; // scalar or uniform parameters
    std::vector<int> stream_of_event;          // event index -> event stream id
    bool has_spike_monitor = false;
    // per EventMonitor: its event stream, and 1 when its schedule node runs
    // before the node that produces the event in a tick (it then records the
    // previous tick's list, as the reference's `fired` still holds it)
    std::vector<int> evmon_stream, evmon_lag;
    // per EventMonitor with recorded variables: one sample ring per variable,
    // indexed like the event stream's ring (record j of the stream's list at
    // ring position j), drained to host bytes alongside the spikes
    struct EvMonVars {
      std::vector<int> ring;
      std::vector<size_t> width;
      std::vector<std::vector<uint8_t>> host;
      uint64_t drained = 0;
    };
    std::vector<EvMonVars> evmon_vars;
    // state monitor
    int mon_records = -1;
    size_t mon_nrec = 0;            // records owned by this rank
    std::vector<int> mon_samples;  // per monitor variable
    std::vector<DType> mon_dtypes;
    uint64_t mon_ticks = 0, mon_first_tick = 0;
    // spike generator
    int gen_offsets = -1, gen_ids = -1;
  };
  std::vector<PopDev> pops;
  std::vector<EventStreamDev> streams;

  // ---- synapses
  struct AtomicAdd {
    size_t state = 0;           // post state index
    double addend = 0.0;
    bool gated = false;         // only where the target's not_refractory is set
  };
  struct PathwayDev {
    size_t synapse = 0, index = 0;
    bool is_pre = true;
    size_t endpoint_pop = 0, other_pop = 0;
    size_t endpoint_start = 0, endpoint_count = 0;
    int stream = -1;
    int offsets = -1, row_other = -1, row_edge = -1, row_delay = -1;  // CSR
    bool uniform = true;
    size_t delay = 0, max_delay = 0;
    uint64_t max_row = 0;  // longest CSR row (sizes the scatter work split)
    int delivered_slot = 0;
    enum class Mode { Atomic, EdgeParallel, Targets, Serial } mode = Mode::Serial;
    std::vector<AtomicAdd> atomic_adds;
    // Targets mode: target-major view (per target: entries by delay
    // descending, then source ascending, then creation order)
    int tm_off = -1, tm_src = -1, tm_edge = -1, tm_delay = -1;
    uint64_t tm_targets = 0, tm_lo = 0;  // local targets [tm_lo, tm_lo + tm_targets) (synapse-level)
    uint64_t tm_max_deg = 0;             // longest in-edge list
    unsigned tm_warps = 1;               // warps per target (targets_group)
    // event-driven variant (one delay): a scatter kernel appends each event
    // (source << 32 | row position) to its target's bucket (capacity = the
    // target's in-degree, at tm_off) and lists the targets it touched; a
    // delivery kernel sorts each listed bucket and runs the bodies in order
    bool tm_events = false;
    int tm_cnt = -1, tm_bucket = -1, tm_active = -1, tm_nactive = -1;
    int pend_offsets = -1, pend_items = -1, pend_src = -1, pend_tgt = -1;
    bool has_pending = false;
    // counted delivery (constant-addend pathways into f32 state): the
    // scatter adds 1 to the target's event counter (count_ptr, u32 per
    // target) and the next dense kernel of the target population applies
    // the pathway's map that many times (StepSpec::applies)
    bool counted = false;
    int count_ptr = -1;
    // Two counted pathways of one launch may share a u32 counter per target
    // (16 bits each, this pathway's at count_shift) when each delivers fewer
    // than 2^16 events to one target in a tick: max_indeg bounds that (the
    // pathway's largest in-degree; a single delay gives each edge at most
    // one event per tick).
    bool count_packed = false;
    int count_shift = 0;
    uint64_t max_indeg = UINT64_MAX;
  };
  struct SynDev {
    uint64_t edges = 0;        // global edge count (the `N` of synaptic code)
    uint64_t local_edges = 0;  // edges whose target this rank owns (== edges on one GPU)
    bool procedural = false;
    std::vector<Slot> states;
    std::map<std::string, int> param_ptr;
    std::map<std::string, double> param_const;
    std::vector<PathwayDev> pathways;
    bool identity_edges = true;  // row position == edge id for pre CSR
    // `(summed)` variables in code-object order: the destination endpoint's
    // CSR (rows = destination neurons, entries in edge creation order)
    struct Summed {
      size_t code = 0;            // code-object index
      bool to_pre = false;
      size_t dest_pop = 0, dest_state = 0, dest_start = 0, dest_count = 0;
      int offsets = -1, row_other = -1, row_edge = -1;
    };
    std::vector<Summed> summed;
    // per-edge endpoints (synapse-level source and target of each local
    // edge) for programs that run over every edge
    int edge_src = -1, edge_tgt = -1;
  };
  std::vector<SynDev> syns;
  struct SummedSpec {
    size_t synapse = 0, k = 0;
    const Program* program = nullptr;
    size_t result = 0;  // register of `_synaptic_var`
    std::map<size_t, int> pre_replica;  // presynaptic state -> replica read (multi-GPU)
  };
  int delivered_ptr = -1;
  size_t delivered_count = 0;
  // per event stream: oldest ring position the host or a delayed consumer
  // still needs (ring positions count per stream), read by the appending
  // kernels' overflow checks
  int floors_ptr = -1;
  std::vector<uint64_t> floors_host_;
  std::string floor_of(size_t sid) const { return P(floors_ptr, "const u64") + "[" + std::to_string(sid) + "]"; }

  // ---- kernels
  struct Op {
    std::string name;
    cudaKernel_t fn = nullptr;
    unsigned grid = 1, block = kThreads;
  };
  std::vector<Op> ops;
  std::vector<std::string> kernel_sources;
  cudaGraphExec_t graph_exec = nullptr;
  uint32_t graph_ticks = 0;
  cudaEvent_t ev_start = nullptr, ev_stop = nullptr;

  // ---- run state
  size_t start_tick = 0, steps = 0, cur_rel = 0;
  double dt = 0.0;
  bool failed = false;

  // ---- multi-GPU partition
  int world = 1, rank = 0;
  DeviceBuffer arena;                 // exchange buffers + result staging (CUDA IPC exported)
  size_t arena_stage_off = 0;
  std::vector<void*> peer_base;       // other ranks' arenas, mapped by connect()
  bool connected = false, published = false;
  std::vector<DeviceBuffer> published_lists;  // local event lists exported by publish()
  bool lists_merged = false;
  void* gptr_table = nullptr;         // device address of the module's g_ptr table
  uint64_t part_lo(uint64_t n, int r) const { return n * uint64_t(r) / uint64_t(world); }
  // Block of population p whose results rank q stages (replicated
  // populations: all of it on rank 0, nothing elsewhere).
  uint64_t stage_lo(size_t p, int q) const {
    const uint64_t n = m.populations[p].count;
    return pops[p].replicated ? (q == 0 ? 0 : n) : part_lo(n, q);
  }
  uint64_t stage_count(size_t p, int q) const {
    const uint64_t n = m.populations[p].count;
    return pops[p].replicated ? (q == 0 ? n : 0) : part_lo(n, q + 1) - part_lo(n, q);
  }
  bool replicate_ = true;  // multi-GPU: replicate populations that no synapse targets
  bool local_streams_ = true;  // multi-GPU: keep lists that only their own rank reads local
  // A population that no synapse targets, and that is no spike generator
  // (which already emits its global list on every rank).
  bool replicable(size_t p) const {
    if (world == 1 || !replicate_ || m.population_instances[p].spike_generator) return false;
    for (const auto& s : m.synapses)
      if (s.target_population == p) return false;
    return true;
  }

  Impl(const b2ir::Model& model, const Options& o) : m(model), opt(o), world(o.world_size), rank(o.rank) {
    if (const char* e = std::getenv("B2GPU_NPT")) npt_ = unsigned(std::atoi(e));
    if (o.neurons_per_thread) npt_ = o.neurons_per_thread;
    check(npt_ == 1 || npt_ == 2 || npt_ == 4, "neurons per thread must be 1, 2 or 4");
    if (const char* e = std::getenv("B2GPU_MINBLOCKS")) min_blocks_ = unsigned(std::atoi(e));
    // Diagnostic: plan every schedule node as its own kernel (same work,
    // same results) to attribute time per node.
    if (const char* e = std::getenv("B2GPU_NO_FUSE")) no_fuse_ = std::atoi(e) != 0;
    // Diagnostic: plain stream-ordered launches instead of programmatic
    // dependent launches (same results) for A/B timing.
    if (const char* e = std::getenv("B2GPU_PDL")) use_pdl_ = std::atoi(e) != 0;
    if (const char* e = std::getenv("B2GPU_PDL_TRIGGER")) pdl_trigger_end_ = std::string(e) != "start";
    if (const char* e = std::getenv("B2GPU_CONSUMER_BLOCKS")) consumer_blocks_ = unsigned(std::atoi(e));
    // Tuning knobs (same results): wave-balanced neuron tiles, and row
    // entries per thread in constant-addend scatters (1..8).
    if (const char* e = std::getenv("B2GPU_BALANCE")) balance_tiles_ = std::atoi(e) != 0;
    // Diagnostic: deliver constant-addend pathways into f32 state with a
    // compare-and-swap per event instead of counted delivery (same results).
    if (const char* e = std::getenv("B2GPU_COUNTED")) counted_ = std::atoi(e) != 0;
    // Counted delivery also into f64 state (the map x <- x + w is applied by
    // the next dense kernel instead of a red.add.f64 per event; same results).
    if (const char* e = std::getenv("B2GPU_COUNTED_F64")) counted_f64_ = std::atoi(e) != 0;
    // One cooperative launch per chunk runs every tick's kernels as phases
    // separated by grid barriers (same results).
    if (const char* e = std::getenv("B2GPU_MEGA")) mega_ = std::atoi(e) != 0;
    // __launch_bounds__ blocks-per-SM hint of constant-addend scatter kernels
    // (0: none).
    if (const char* e = std::getenv("B2GPU_SCATTER_MINBLOCKS")) scatter_min_blocks_ = unsigned(std::atoi(e));
    if (const char* e = std::getenv("B2GPU_PACK_COUNTS")) pack_counts_ = std::atoi(e) != 0;
    if (const char* e = std::getenv("B2GPU_FUSE_LAYOUT")) fuse_layout_ = std::atoi(e) != 0;
    if (const char* e = std::getenv("B2GPU_L2_HINTS")) l2_hints_ = std::atoi(e) != 0;
    if (const char* e = std::getenv("B2GPU_SCATTER_BLOCKS")) scatter_blocks_ = unsigned(std::atoi(e));
    // Diagnostic: constant-addend scatter items per block, one row entry per
    // thread, instead of per warp (same results).
    if (const char* e = std::getenv("B2GPU_SCATTER_WARP")) scatter_warp_ = std::atoi(e) != 0;
    if (const char* e = std::getenv("B2GPU_TILE")) tile_override_ = size_t(std::atoll(e));
    check(tile_override_ % 32 == 0 && tile_override_ <= size_t(kThreads) * 32, "B2GPU_TILE must be a multiple of 32 up to 8192");
    if (const char* e = std::getenv("B2GPU_SCATTER_UNROLL")) scatter_unroll_ = unsigned(std::atoi(e));
    if (const char* e = std::getenv("B2GPU_FUSE_EXCHANGE")) fuse_exchange_ = std::atoi(e) != 0;
    // Diagnostic: deliver ordered pathways with one serial thread instead of
    // the target-ordered kernel (same results) for A/B timing.
    if (const char* e = std::getenv("B2GPU_TARGETS")) use_targets_ = std::atoi(e) != 0;
    // Diagnostic: one launch per population step (same results).
    if (const char* e = std::getenv("B2GPU_FUSE_STEPS")) fuse_steps_ = std::atoi(e) != 0;
    if (const char* e = std::getenv("B2GPU_TARGETS_UNROLL")) targets_unroll_ = unsigned(std::atoi(e));
    check(targets_unroll_ >= 1 && targets_unroll_ <= 16, "target-ordered unroll must be 1 to 16");
    if (const char* e = std::getenv("B2GPU_TARGETS_WARPS")) targets_warps_ = unsigned(std::atoi(e));
    if (const char* e = std::getenv("B2GPU_TARGETS_SMEM")) targets_smem_bitmap_ = std::atoi(e) != 0;
    // Diagnostic: deliver single-delay target-ordered pathways with the
    // bitmap scan instead of the event buckets (same results).
    if (const char* e = std::getenv("B2GPU_TARGETS_SCAN")) targets_scan_ = std::atoi(e) != 0;
    check(targets_warps_ == 0 || targets_warps_ == 1 || targets_warps_ == 2 || targets_warps_ == 4 ||
              targets_warps_ == 8,
          "warps per target must be 1, 2, 4 or 8");
    // Diagnostic: partition and exchange every population on N > 1 GPUs
    // (same results) instead of replicating the ones no synapse targets.
    if (const char* e = std::getenv("B2GPU_REPLICATE")) replicate_ = std::atoi(e) != 0;
    // Diagnostic: exchange every partitioned population's list (same results).
    if (const char* e = std::getenv("B2GPU_LOCAL_STREAMS")) local_streams_ = std::atoi(e) != 0;
    check(scatter_unroll_ >= 1 && scatter_unroll_ <= 8, "scatter unroll must be 1 to 8");
  }
  bool no_fuse_ = false;
  bool counted_ = true;  // counted delivery of constant-addend pathways into f32 state
  bool counted_f64_ = false;  // ... and into f64 state
  // Chunk kernel: the tick's kernels as device functions, called by a
  // co-resident grid for their virtual blocks, with a grid barrier after each
  // (B2GPU_MEGA); mega_grid is the launch's block count (0: not available).
  bool mega_ = false;
  unsigned scatter_min_blocks_ = 0;
  bool pack_counts_ = true;  // B2GPU_PACK_COUNTS: two counted pathways share 16-bit halves of one counter
  bool fuse_layout_ = true;  // B2GPU_FUSE_LAYOUT: a layout / receive kernel joins the scatter launch before it
  unsigned scatter_blocks_ = 0;  // B2GPU_SCATTER_BLOCKS: grid of delayed / unfused scatters (0: 1184)
  bool l2_hints_ = true;     // B2GPU_L2_HINTS: counted scatters stream rows evict-first, counters evict-last
  unsigned mega_grid = 0;
  cudaKernel_t mega_fn = nullptr;
  DeviceBuffer mega_bar;
  bool scatter_warp_ = true;  // constant-addend scatter items per warp (else per block)
  unsigned consumer_blocks_ = 0;  // B2GPU_CONSUMER_BLOCKS: scatter blocks of a fused list consumer (0: one per tile)
  bool use_targets_ = true;  // target-ordered delivery for ordered pathways (else one serial thread)
  bool fuse_steps_ = true;   // one launch for consecutive step kernels of different populations
  unsigned targets_unroll_ = 4;  // 32-entry groups each warp of a target-ordered kernel keeps in flight
  unsigned targets_warps_ = 0;   // warps per target (0: targets_group chooses)
  bool targets_smem_bitmap_ = true;  // stage the fired bitmap slot in shared memory
  bool targets_scan_ = false;        // scan variant also for single-delay pathways
  bool use_pdl_ = true;
  bool pdl_trigger_end_ = true;  // trigger dependents after a block's work (B2GPU_PDL_TRIGGER=start: before)
  bool balance_tiles_ = true;                // tile_n_for: spread small populations over a whole wave
  size_t tile_override_ = 0;                 // B2GPU_TILE: neurons per tile (multiple of 32)
  // Multi-GPU: the receiving kernel of an exchanged stream also delivers the
  // delay-0 constant-addend scatter that follows it (0: a separate receive
  // launch, then the scatter reads the ring; same results).
  bool fuse_exchange_ = true;
  unsigned scatter_unroll_ = kScatterUnroll;  // row entries per thread per scatter work item
  uint64_t row_chunk() const { return uint64_t(kThreads) * scatter_unroll_; }

  unsigned npt_ = 2;         // neurons per thread in neuron kernels (config 2: 18.2 ms per 1000 ticks at 2, 19.9 at 4)
  // __launch_bounds__ occupancy hint for neuron kernels (0: none).  Four
  // resident 256-thread blocks per SM (<= 64 registers) measured fastest for
  // the fused CUBA step: 25.3 us vs 28.6 us per 1M-neuron tick without it.
  unsigned min_blocks_ = 4;
  unsigned sm_count_ = 148;   // multiprocessors of the device (dry runs: a B200's 148)
  // Neurons per block tile of a neuron kernel.  A population that fills at
  // least one wave of resident blocks (SMs x occupancy hint) at kThreads *
  // npt_ neurons per block keeps that tile: config 2 (1M neurons) runs as
  // 1954 tiles of 512.  Measured there (ms per 1000 ticks, 4 neurons per
  // thread): 977 tiles of 1024 over 592 resident blocks ran in 19.98, one
  // wave of 590 tiles of 1696 that each walk 1.66 chunks in 21.12.  A
  // smaller population (one GPU's share of a partitioned network) is spread
  // over all resident slots in whole 32-neuron words, at least one block of
  // threads per tile: 125k neurons run as 489 blocks of 256 instead of 245
  // blocks of 512.  The step kernel walks a tile in chunks of kThreads *
  // npt_, so larger tiles (B2GPU_TILE) are valid too.
  size_t tile_n_for(size_t count) const {
    const size_t max_tile = size_t(kThreads) * npt_;
    if (tile_override_) return tile_override_;
    const size_t slots = size_t(sm_count_) * std::max(1u, min_blocks_);
    if (!balance_tiles_ || count >= max_tile * slots) return max_tile;
    size_t t = (count + slots - 1) / slots;
    t = (t + 31) / 32 * 32;
    return std::min(max_tile, std::max<size_t>(t, std::min<size_t>(kThreads, max_tile)));
  }
  size_t tiles_for(size_t count) const {
    const size_t tile = tile_n_for(count);
    return std::max<size_t>(1, (count + tile - 1) / tile);
  }

  ~Impl() {
    for (void* pb : peer_base)
      if (pb) cudaIpcCloseMemHandle(pb);
    if (ev_start) cudaEventDestroy(ev_start);
    if (ev_stop) cudaEventDestroy(ev_stop);
    if (graph_exec) cudaGraphExecDestroy(graph_exec);
    if (module) cudaLibraryUnload(module);
    owned.clear();
    ctl = DeviceBuffer();
    if (stream) cudaStreamDestroy(stream);
  }

  int add_ptr(void* p) {
    ptrs.push_back(reinterpret_cast<uint64_t>(p));
    return int(ptrs.size() - 1);
  }
  int alloc(size_t bytes) {
    if (opt.dry_run) return add_ptr(reinterpret_cast<void*>(uintptr_t(0x100000) * (ptrs.size() + 1)));
    owned.emplace_back(std::max<size_t>(bytes, 16));
    return add_ptr(owned.back().ptr);
  }
  // Device copy of host bytes.  Callers pad empty arrays to one element so
  // every pointer is valid; the data of an empty std::vector may be null, in
  // which case the padding is zero-filled instead of copied.  The copy is
  // complete when this returns, so callers may pass temporaries.
  int upload(const void* host, size_t bytes) {
    int k = alloc(bytes);
    if (bytes && !opt.dry_run) {
      if (host) {
        B2_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(ptrs[size_t(k)]), host, bytes, cudaMemcpyHostToDevice, stream));
        B2_CUDA(cudaStreamSynchronize(stream));
      } else {
        B2_CUDA(cudaMemsetAsync(reinterpret_cast<void*>(ptrs[size_t(k)]), 0, bytes, stream));
      }
    }
    return k;
  }
  void memset_dev(int k, size_t bytes) {
    if (!opt.dry_run) B2_CUDA(cudaMemsetAsync(dptr(k), 0, bytes, stream));
  }
  int adopt(DeviceBuffer&& b) {
    owned.push_back(std::move(b));
    return add_ptr(owned.back().ptr);
  }
  void* dptr(int k) const { return reinterpret_cast<void*>(ptrs[size_t(k)]); }

  // ================================================================ checks
  void check_capabilities() {
    check(m.clocks.size() == 1, "the GPU engine supports models with a single clock");
    dt = m.clocks[0].dt;
    start_tick = m.run_clocks[0].start_tick;
    steps = m.run_clocks[0].steps;
    for (const auto& p : m.populations) {
      check(p.linked_variable_count == 0, "linked variables are not supported by the GPU engine");
      check(!p.spatial, "spatial neurons are not supported by the GPU engine");
      check(p.rate_monitor_count == 0, "rate monitors are not supported by the GPU engine");
      for (const auto& em : p.event_monitors)
        for (const auto& v : em.variables) {
          check(world == 1, "multi-GPU runs do not support EventMonitor variables");
          bool known = false;
          for (const auto& st : p.states) known |= st.name == v;
          for (const auto& pa : p.parameters) known |= pa.name == v && pa.dtype == DType::F64;
          check(known, "EventMonitor variable '" + v + "' must be a state or an f64 parameter of its population");
        }
      check(p.steps == steps, "population steps must match the run clock");
      for (const auto& c : p.code_objects) check(!c.adaptive, "adaptive integrators are not supported by the GPU engine");
    }
    for (const auto& s : m.synapses) {
      check(!s.source_synapse && !s.target_synapse, "synapse-to-synapse projections are not supported by the GPU engine");
      check(s.linked_variable_count == 0, "synaptic linked variables are not supported by the GPU engine");
      check(s.state_monitor_count == 0, "synapse state monitors are not supported by the GPU engine");
      for (const auto& c : s.code_objects)
        check(c.kind == "synapses" || c.kind == "synapses_post" || c.kind == "summed_variable" ||
                  c.kind == "synapse_state_update" || c.kind == "synapse_subexpression_update" ||
                  c.kind == "synapse_run_regularly",
              "synapse code object kind '" + c.kind + "' is not supported by the GPU engine");
    }
    // one warp lane per destination rank stores a fired word: at most 32 ranks
    check(world >= 1 && world <= 32 && rank >= 0 && rank < world, "invalid rank / world size (1 to 32 GPUs)");
    if (world > 1) {
      // Target-owned partition (brian2_rust/distributed.py: rank-local neuron
      // and synapse state, incoming CSR per rank).  What a rank cannot
      // evaluate from its own block is rejected before any device work.
      // Per-edge programs (synaptic state updates, subexpressions,
      // run_regularly) run over the rank's own edges, and a summed variable
      // into the target population sums the rank's own targets' in-edges;
      // a sum into the source population would need every rank's edges.
      for (const auto& s : m.synapses) {
        for (const auto& c : s.code_objects)
          check(c.kind != "summed_variable" || !(c.summed_target && *c.summed_target == "pre"),
                "multi-GPU runs do not support summed variables into the presynaptic population");
      }
      for (size_t k = 0; k < m.synapses.size(); ++k) {
        const auto& inst = m.synapse_instances[k];
        if (inst.topology.kind != b2ir::Topology::Kind::Explicit) {
          check(m.synapses[k].states.empty(), "multi-GPU runs need explicit topologies for plastic synapses");
          check(inst.topology.initializers.empty(), "multi-GPU runs do not support procedural per-edge initializers");
        }
      }
    }
  }

  // ================================================================ populations
  void build_populations() {
    for (size_t p = 0; p < m.populations.size(); ++p) {
      const auto& def = m.populations[p];
      const auto& inst = m.population_instances[p];
      PopDev pd;
      pd.global_count = def.count;
      pd.replicated = replicable(p);
      pd.lo = pd.replicated ? 0 : part_lo(def.count, rank);
      check(def.count < UINT32_MAX, "populations must hold fewer than 2^32 - 1 neurons");
      pd.count = pd.replicated ? def.count : part_lo(def.count, rank + 1) - pd.lo;
      const size_t lo = pd.lo, n = pd.count;
      pd.start_tick = start_tick;
      pd.steps = def.steps;
      pd.end_tick = start_tick + def.steps;
      pd.dt = def.dt;
      for (const auto& s : def.states) {
        const auto& arr = inst.initial_state.at(s.name);
        check(arr.size() == def.count, "initial state '" + s.name + "' has the wrong length");
        const size_t w = b2ir::dtype_bytes(s.dtype);
        std::vector<uint8_t> bytes(n * w);
        for (size_t i = 0; i < n; ++i) std::memcpy(&bytes[i * w], &arr.raw[lo + i], w);
        pd.states.push_back({s.dtype, upload(bytes.data(), bytes.size())});
      }
      if (inst.refractory) {
        pd.lastspike = upload(inst.refractory->initial_lastspike.data() + lo, n * 8);
        pd.not_refractory = upload(inst.refractory->initial_not_refractory.data() + lo, n);
        pd.period_ticks = inst.refractory->period_ticks;
        pd.fixed_refractory = def.refractory && def.refractory->mode == "fixed";
      }
      for (const auto& s : def.parameters) {
        const auto& arr = inst.parameters.at(s.name);
        bool uniform = true;
        for (size_t i = 1; i < arr.size(); ++i) uniform &= arr.raw[i] == arr.raw[0];
        if (s.index_domain == b2ir::IndexDomain::Scalar || uniform) {
          pd.param_const[s.name] = arr.as_f64(0);
        } else {
          check(arr.size() == def.count, "parameter '" + s.name + "' has the wrong length");
          std::vector<double> v(n);
          for (size_t i = 0; i < n; ++i) v[i] = arr.as_f64(lo + i);
          pd.param_ptr[s.name] = upload(v.data(), std::max<size_t>(n, 1) * 8);
        }
      }
      pd.stream_of_event.assign(def.events.size(), -1);
      for (size_t e = 0; e < def.events.size(); ++e) {
        EventStreamDev es;
        es.pop = p;
        es.event = e;
        pd.stream_of_event[e] = int(streams.size());
        streams.push_back(std::move(es));
      }
      for (const auto& node : m.schedule)
        if (node.owner_kind == b2ir::OwnerKind::Population && node.owner_index == p &&
            node.operation == b2ir::ScheduleOp::SpikeMonitor)
          pd.has_spike_monitor = true;
      // state monitor buffers
      if (!def.state_monitors.empty() && !def.monitor.record.empty() && !def.monitor.variables.empty()) {
        // Records this rank owns, as local indices, in record order.
        std::vector<uint32_t> rec;
        for (auto r : def.monitor.record) {
          check(r < def.count, "state monitor record index out of range");
          if (r >= lo && r < lo + n) rec.push_back(uint32_t(r - lo));
        }
        pd.mon_nrec = rec.size();
        if (!rec.empty()) pd.mon_records = upload(rec.data(), rec.size() * 4);
        uint64_t window = std::min<uint64_t>(def.monitor.window_steps, def.steps);
        pd.mon_ticks = window;
        pd.mon_first_tick = pd.end_tick - window;
        for (const auto& name : def.monitor.variables) {
          DType d = DType::F64;
          bool found = false;
          for (const auto& s : def.states) if (s.name == name) { d = s.dtype; found = true; }
          for (const auto& s : def.parameters) if (s.name == name) { d = s.dtype; found = true; }
          check(found, "monitor symbol missing from population");
          pd.mon_dtypes.push_back(d);
          pd.mon_samples.push_back(alloc(window * pd.mon_nrec * b2ir::dtype_bytes(d)));
        }
      }
      if (inst.spike_generator) {
        // Precompute each tick's fired list with the reference cursor rule
        // (emit_spike_generator, executor.rs:3008-3036).
        const auto& g = *inst.spike_generator;
        std::vector<uint64_t> offs(def.steps + 1, 0);
        std::vector<uint32_t> ids;
        size_t cursor = 0;
        for (size_t k = 0; k < def.steps; ++k) {
          size_t tick = start_tick + k;
          while (cursor < g.spike_ticks.size() && g.spike_ticks[cursor] < tick) ++cursor;
          while (cursor < g.spike_ticks.size() && g.spike_ticks[cursor] == tick) {
            check(g.spike_indices[cursor] < def.count, "spike generator index out of range");
            ids.push_back(uint32_t(g.spike_indices[cursor++]));
          }
          offs[k + 1] = ids.size();
        }
        pd.gen_offsets = upload(offs.data(), offs.size() * 8);
        pd.gen_ids = upload(ids.data(), std::max<size_t>(ids.size(), 1) * 4);
      }
      pops.push_back(std::move(pd));
    }
  }

  // ================================================================ synapses
  void build_synapses() {
    std::vector<uint64_t> delivered_init;
    for (size_t s = 0; s < m.synapses.size(); ++s) {
      const auto& def = m.synapses[s];
      const auto& inst = m.synapse_instances[s];
      SynDev sd;
      const auto& topo = inst.topology;
      std::vector<uint32_t> src_h, tgt_h;  // explicit only
      std::map<std::string, std::vector<double>> generated_params;
      std::vector<std::vector<size_t>> delays;
      // a binary_csr graph is an explicit edge list stored in a file
      const bool binary = topo.kind == b2ir::Topology::Kind::BinaryCsr;
      bool procedural = topo.kind != b2ir::Topology::Kind::Explicit && !binary;
      sd.procedural = procedural;
      b2ir::BinaryCsr csr;
      if (binary)
        csr = b2ir::read_binary_csr(topo.path, def.source_count, def.target_count, topo.edge_count, topo.column_count,
                                    topo.sha256, true);
      // Edges this rank stores: every edge on one GPU; otherwise the edges
      // whose target it owns, in creation order (local edge k is global edge
      // edge_ids[k]).  Per-edge arrays are indexed by local edge.
      std::vector<uint32_t> edge_ids;
      const PopDev& tpop = pops[def.target_population];
      // Procedural topologies: the source-major device CSR (rows hold the
      // global synapse-level target j; the edge id is the row position, the
      // reference's creation order), built once per synapse and shared by its
      // pathways, per-edge programs and summed variables.
      int proc_off = -1, proc_rows = -1;
      uint64_t proc_max_row = 0;
      auto procedural_csr = [&]() {
        if (proc_off >= 0) return;
        if (opt.dry_run) {
          proc_off = alloc(0);
          proc_rows = alloc(0);
          return;
        }
        DeviceBuffer offs, rows;
        uint64_t local_edges = 0;
        // synapse-level targets j whose population index target_start + j
        // this rank owns
        auto clampj = [&](uint64_t x) {
          return x <= def.target_start ? uint64_t(0) : std::min<uint64_t>(x - def.target_start, def.target_count);
        };
        const uint64_t j0 = clampj(tpop.lo), j1 = clampj(tpop.lo + tpop.count);
        if (topo.kind == b2ir::Topology::Kind::FixedIndegree)
          build_fixed_indegree_csr(def.source_count, def.target_count, topo.indegree, topo.seed, j0, j1, offs, rows,
                                   local_edges, stream);
        else
          build_fixed_total_csr(def.source_count, def.target_count, topo.edge_count, topo.seed, j0, j1, offs, rows,
                                local_edges, stream);
        check(world > 1 || local_edges == sd.edges, "procedural edge count mismatch");
        if (world > 1) sd.local_edges = local_edges;
        std::vector<uint64_t> host_offs(def.source_count + 1);
        B2_CUDA(cudaMemcpy(host_offs.data(), offs.ptr, host_offs.size() * 8, cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < def.source_count; ++i)
          proc_max_row = std::max<uint64_t>(proc_max_row, host_offs[i + 1] - host_offs[i]);
        proc_off = adopt(std::move(offs));
        proc_rows = adopt(std::move(rows));
      };
      if (!procedural) {
        src_h = binary ? std::move(csr.source) : inst.source;
        tgt_h = binary ? std::move(csr.target) : inst.target;
        sd.edges = src_h.size();
        check(tgt_h.size() == sd.edges, "explicit source and target arrays differ in length");
        for (const auto& pw : inst.pathways) delays.push_back(pw.delay_ticks);
        if (world > 1) {
          for (size_t e = 0; e < tgt_h.size(); ++e) {
            const uint64_t tp = def.target_start + uint64_t(tgt_h[e]);
            if (tp >= tpop.lo && tp < tpop.lo + tpop.count) edge_ids.push_back(uint32_t(e));
          }
        }
      } else {
        sd.edges = topo.edge_count;
        for (const auto& pw : inst.pathways) {
          if (pw.delay_initializer) {
            // drawn per edge on the device below (edge id = source-major position)
            check(pw.kind == "pre" && world == 1,
                  "procedural delay initializers are supported on on_pre pathways of one GPU");
          }
          delays.push_back(pw.delay_ticks);
        }
      }
      const bool all_edges = world == 1 || procedural;
      sd.local_edges = all_edges ? sd.edges : edge_ids.size();
      auto gid = [&](size_t k) -> size_t { return all_edges ? k : edge_ids[k]; };
      // synapse states
      for (const auto& sym : def.states) {
        auto it = inst.initial_state.find(sym.name);
        check(it != inst.initial_state.end() && it->second.size() == sd.edges,
              "synapse state '" + sym.name + "' has the wrong length");
        size_t w = b2ir::dtype_bytes(sym.dtype);
        std::vector<uint8_t> bytes(sd.local_edges * w);
        for (size_t k = 0; k < sd.local_edges; ++k) std::memcpy(&bytes[k * w], &it->second.raw[gid(k)], w);
        sd.states.push_back({sym.dtype, upload(bytes.data(), std::max<size_t>(bytes.size(), 1))});
      }
      // parameters (per-edge arrays indexed by edge id)
      for (const auto& sym : def.parameters) {
        auto init = topo.initializers.find(sym.name);
        if (procedural && init != topo.initializers.end()) {
          const auto& in = init->second;
          if (in.kind == b2ir::Initializer::Kind::ClippedNormal) {
            // rejection sampling with transcendentals: drawn on the host
            const std::vector<double> v = clipped_normal_host(opt.dry_run ? 0 : sd.edges, topo.seed, in, std::nullopt);
            sd.param_ptr[sym.name] = upload(v.data(), std::max<size_t>(sd.edges, 1) * 8);
            continue;
          }
          int k = alloc(sd.edges * 8);
          if (!opt.dry_run)
            uniform_initializer_device(static_cast<double*>(dptr(k)), sd.edges, topo.seed, in.stream, *in.minimum,
                                       *in.maximum, 0, stream);
          sd.param_ptr[sym.name] = k;
          continue;
        }
        auto col = binary ? topo.columns.find(sym.name) : topo.columns.end();
        if (col != topo.columns.end()) {
          const std::vector<double>& values = csr.columns[size_t(col->second)];
          std::vector<double> v(sd.local_edges);
          for (size_t k = 0; k < sd.local_edges; ++k) v[k] = values[gid(k)];
          sd.param_ptr[sym.name] = upload(v.data(), std::max<size_t>(v.size(), 1) * 8);
          continue;
        }
        const auto& arr = inst.parameters.at(sym.name);
        bool uniform = true;
        for (size_t i = 1; i < arr.size(); ++i) uniform &= arr.raw[i] == arr.raw[0];
        if (sym.index_domain == b2ir::IndexDomain::Scalar || uniform) {
          check(arr.size() > 0, "empty parameter '" + sym.name + "'");
          sd.param_const[sym.name] = arr.as_f64(0);
        } else {
          check(arr.size() == sd.edges, "synapse parameter '" + sym.name + "' has the wrong length");
          check(world == 1 || !procedural, "multi-GPU runs need explicit topologies for per-edge parameters");
          std::vector<double> v(sd.local_edges);
          for (size_t k = 0; k < sd.local_edges; ++k) v[k] = arr.as_f64(gid(k));
          sd.param_ptr[sym.name] = upload(v.data(), std::max<size_t>(v.size(), 1) * 8);
        }
      }
      // pathways
      for (size_t k = 0; k < inst.pathways.size(); ++k) {
        const auto& pw = inst.pathways[k];
        PathwayDev pd;
        pd.synapse = s;
        pd.index = k;
        pd.is_pre = pw.kind == "pre";
        pd.endpoint_pop = pd.is_pre ? def.source_population : def.target_population;
        pd.other_pop = pd.is_pre ? def.target_population : def.source_population;
        pd.endpoint_start = pd.is_pre ? def.source_start : def.target_start;
        pd.endpoint_count = pd.is_pre ? def.source_count : def.target_count;
        const auto& endpoint = m.populations[pd.endpoint_pop];
        auto ev = std::find(endpoint.events.begin(), endpoint.events.end(), pw.event);
        check(ev != endpoint.events.end(), "pathway event missing from endpoint");
        pd.stream = pops[pd.endpoint_pop].stream_of_event[size_t(ev - endpoint.events.begin())];
        const auto& d = delays[k];
        int init_delay = -1;  // device per-edge delays of a procedural delay initializer
        if (procedural && pw.delay_initializer && pw.delay_initializer->kind == b2ir::Initializer::Kind::ClippedNormal) {
          // drawn on the host (rejection sampling with transcendentals)
          const double ddt = m.populations[def.source_population].dt;
          const std::vector<double> v = clipped_normal_host(opt.dry_run ? 0 : sd.edges, topo.seed, *pw.delay_initializer, ddt);
          std::vector<uint16_t> ticks(v.size());
          uint64_t dmin = UINT64_MAX, dmax = 0;
          for (size_t e = 0; e < v.size(); ++e) {
            const double t = std::floor(v[e] / ddt + 0.5);
            check(t >= 0.0 && t < 65535.0, "procedural delay outside 0 to 65534 ticks");
            ticks[e] = uint16_t(t);
            dmin = std::min<uint64_t>(dmin, ticks[e]);
            dmax = std::max<uint64_t>(dmax, ticks[e]);
          }
          if (opt.dry_run) dmin = 0, dmax = 1;  // plan as per-edge delays
          init_delay = upload(ticks.data(), std::max<size_t>(ticks.size(), 1) * 2);
          pd.uniform = dmin == dmax;
          pd.delay = dmin;
          pd.max_delay = dmax;
        } else if (procedural && pw.delay_initializer) {
          const auto& in = *pw.delay_initializer;
          const double ddt = m.populations[def.source_population].dt;
          // materialize_uniform_ticks' own check
          check(std::isfinite(*in.minimum) && std::isfinite(*in.maximum) && *in.minimum >= 0.0 &&
                    *in.minimum <= *in.maximum && std::isfinite(ddt) && ddt > 0.0 && *in.maximum / ddt < 1000001.0,
                "invalid uniform delay initializer");
          uint64_t dmin = 0, dmax = 0;
          if (opt.dry_run) {
            init_delay = alloc(0);
            dmax = 1;  // plan as per-edge delays
          } else {
            DeviceBuffer ticks;
            delay_ticks_uniform_device(sd.edges, topo.seed, in.stream, *in.minimum, *in.maximum, ddt, ticks, dmin, dmax,
                                       stream);
            init_delay = adopt(std::move(ticks));
          }
          pd.uniform = dmin == dmax;
          pd.delay = dmin;
          pd.max_delay = dmax;
        } else {
          check(!d.empty(), "pathway has no delay");
          pd.uniform = std::all_of(d.begin(), d.end(), [&](size_t x) { return x == d[0]; });
          pd.delay = d[0];
          pd.max_delay = *std::max_element(d.begin(), d.end());
          if (!pd.uniform) check(d.size() == sd.edges, "per-edge delay array has the wrong length");
        }
        // CSR over the endpoint (source for pre, target for post), rows in
        // edge creation order (stable counting sort).
        if (!procedural) {
          const auto& idx = pd.is_pre ? src_h : tgt_h;
          const auto& other = pd.is_pre ? tgt_h : src_h;
          const size_t L = sd.local_edges;
          std::vector<uint64_t> offs(pd.endpoint_count + 1, 0);
          for (size_t k = 0; k < L; ++k) offs[idx[gid(k)] + 1]++;
          for (size_t i = 0; i < pd.endpoint_count; ++i) offs[i + 1] += offs[i];
          std::vector<uint64_t> next(offs.begin(), offs.end() - 1);
          std::vector<uint32_t> row_other(L), row_edge(L);
          std::vector<uint16_t> row_delay;
          if (!pd.uniform) row_delay.resize(L);
          bool identity = true;
          for (size_t k = 0; k < L; ++k) {
            const size_t e = gid(k);
            uint64_t pos = next[idx[e]]++;
            row_other[pos] = other[e];
            row_edge[pos] = uint32_t(k);
            identity &= pos == k;
            if (!pd.uniform) {
              check(d[e] < 65535, "per-edge delay exceeds 65534 ticks");
              row_delay[pos] = uint16_t(d[e]);
            }
          }
          check(idx.size() <= UINT32_MAX, "explicit edge count must fit u32");
          for (size_t i = 0; i < pd.endpoint_count; ++i) pd.max_row = std::max<uint64_t>(pd.max_row, offs[i + 1] - offs[i]);
          if (pd.is_pre) {
            std::vector<uint32_t> indeg(def.target_count, 0);
            uint64_t most = 0;
            for (size_t k = 0; k < L; ++k) most = std::max<uint64_t>(most, ++indeg[tgt_h[gid(k)]]);
            pd.max_indeg = most;
          }
          pd.offsets = upload(offs.data(), offs.size() * 8);
          pd.row_other = upload(row_other.data(), std::max<size_t>(row_other.size(), 1) * 4);
          if (!identity) pd.row_edge = upload(row_edge.data(), std::max<size_t>(row_edge.size(), 1) * 4);
          if (!pd.uniform) pd.row_delay = upload(row_delay.data(), std::max<size_t>(row_delay.size(), 1) * 2);
        } else {
          check(pd.uniform || init_delay >= 0,
                "procedural topologies with per-edge delays are not supported by the GPU engine yet");
          check(pd.is_pre || world == 1, "multi-GPU runs support on_pre pathways on procedural topologies only");
          procedural_csr();
          if (pd.is_pre) {
            pd.offsets = proc_off;
            pd.row_other = proc_rows;
            pd.max_row = proc_max_row;
            pd.max_indeg = topo.kind == b2ir::Topology::Kind::FixedIndegree ? uint64_t(topo.indegree)
                                                                             : uint64_t(topo.edge_count);
            if (!pd.uniform) pd.row_delay = init_delay;  // row position == edge id
          } else if (opt.dry_run) {
            pd.offsets = alloc(0);
            pd.row_other = alloc(0);
            pd.row_edge = alloc(0);
          } else {
            // rows over targets: the target-major view (sources, edge ids)
            DeviceBuffer off, src, edge, unused;
            build_target_major(static_cast<const uint64_t*>(dptr(proc_off)),
                               static_cast<const uint32_t*>(dptr(proc_rows)), nullptr, nullptr, 0, def.source_count,
                               sd.local_edges, 0, def.target_count, off, src, edge, unused, stream);
            std::vector<uint64_t> host_offs(def.target_count + 1);
            B2_CUDA(cudaMemcpy(host_offs.data(), off.ptr, host_offs.size() * 8, cudaMemcpyDeviceToHost));
            for (size_t i = 0; i < def.target_count; ++i)
              pd.max_row = std::max<uint64_t>(pd.max_row, host_offs[i + 1] - host_offs[i]);
            pd.offsets = adopt(std::move(off));
            pd.row_other = adopt(std::move(src));
            pd.row_edge = adopt(std::move(edge));
          }
        }
        // Pending (continuation) events, validated like model.rs:4315-4337,
        // then laid out as a CSR by the tick that consumes them: the reference
        // queues an event in ring slot delivery_tick % slots before the run and
        // drains that slot at the first tick with that residue
        // (PathwayQueue::new, executor.rs:6185-6212).  With a uniform delay an
        // item is an endpoint index (its whole row is delivered); otherwise it
        // is one edge, delivered with its source and target.
        if (!pw.pending.empty()) {
          check(pd.uniform || !procedural, "pending events on per-edge-delay procedural pathways are not supported");
          const size_t end_tick = start_tick + endpoint.steps;
          bool valid = pw.pending.size() <= 10'000'000;
          for (size_t x = 0; valid && x < pw.pending.size(); ++x) {
            const auto& ev2 = pw.pending[x];
            valid = ev2.delivery_tick >= start_tick && ev2.delivery_tick < end_tick &&
                    ev2.item < (pd.uniform ? pd.endpoint_count : sd.edges) &&
                    (x == 0 || pw.pending[x - 1].delivery_tick <= ev2.delivery_tick);
          }
          check(valid, "invalid pending synaptic pathway event");
          // multi-GPU: an edge item belongs to the rank that stores the edge
          std::unordered_map<uint32_t, uint32_t> local_of;
          if (!pd.uniform && !all_edges)
            for (size_t k = 0; k < edge_ids.size(); ++k) local_of.emplace(edge_ids[k], uint32_t(k));
          size_t slots = std::min(pd.max_delay + 1, endpoint.steps);
          struct Item { uint32_t item, src, tgt; };
          std::vector<std::vector<Item>> per(steps);
          for (const auto& ev2 : pw.pending) {
            size_t slot = ev2.delivery_tick % slots;
            size_t first = start_tick + ((slot + slots - start_tick % slots) % slots);
            if (first >= start_tick + steps) continue;
            if (pd.uniform) {
              per[first - start_tick].push_back({uint32_t(ev2.item), 0, 0});
            } else {
              const uint32_t e = uint32_t(ev2.item);
              uint32_t local = e;
              if (!all_edges) {
                auto it = local_of.find(e);
                if (it == local_of.end()) continue;
                local = it->second;
              }
              per[first - start_tick].push_back({local, src_h[e], tgt_h[e]});
            }
          }
          std::vector<uint64_t> offs(steps + 1, 0);
          std::vector<uint32_t> items, srcs, tgts;
          for (size_t t = 0; t < steps; ++t) {
            for (const Item& it : per[t]) {
              items.push_back(it.item);
              srcs.push_back(it.src);
              tgts.push_back(it.tgt);
            }
            offs[t + 1] = items.size();
          }
          pd.pend_offsets = upload(offs.data(), offs.size() * 8);
          pd.pend_items = upload(items.data(), std::max<size_t>(items.size(), 1) * 4);
          if (!pd.uniform) {
            pd.pend_src = upload(srcs.data(), std::max<size_t>(srcs.size(), 1) * 4);
            pd.pend_tgt = upload(tgts.data(), std::max<size_t>(tgts.size(), 1) * 4);
          }
          pd.has_pending = !items.empty();
        }
        pd.delivered_slot = int(delivered_count++);
        StreamUse(pd.stream, pd.max_delay);
        sd.pathways.push_back(std::move(pd));
      }
      // per-edge programs (synapse_state_update / _subexpression_update /
      // _run_regularly) visit every edge with its endpoints
      bool edge_programs = false;
      for (const auto& code : def.code_objects)
        edge_programs |= code.kind == "synapse_state_update" || code.kind == "synapse_subexpression_update" ||
                         code.kind == "synapse_run_regularly";
      if (edge_programs && procedural) {
        // edge id = source-major position: its target is the row entry, its
        // source the row that holds it
        procedural_csr();
        sd.edge_tgt = proc_rows;
        if (opt.dry_run) {
          sd.edge_src = alloc(0);
        } else {
          DeviceBuffer src;
          csr_row_sources(static_cast<const uint64_t*>(dptr(proc_off)), def.source_count, sd.local_edges, src, stream);
          sd.edge_src = adopt(std::move(src));
        }
      } else if (edge_programs) {
        std::vector<uint32_t> es(sd.local_edges), et(sd.local_edges);
        for (size_t k = 0; k < sd.local_edges; ++k) {
          es[k] = src_h[gid(k)];
          et[k] = tgt_h[gid(k)];
        }
        sd.edge_src = upload(es.data(), std::max<size_t>(es.size(), 1) * 4);
        sd.edge_tgt = upload(et.data(), std::max<size_t>(et.size(), 1) * 4);
      }
      // summed variables (executor.rs:3657-3731): each destination neuron
      // adds its edges' values in edge creation order, so the device walks a
      // CSR by destination with ascending edge ids per row
      for (size_t c = 0; c < def.code_objects.size(); ++c) {
        const auto& code = def.code_objects[c];
        if (code.kind != "summed_variable") continue;
        SynDev::Summed sv;
        sv.code = c;
        sv.to_pre = code.summed_target && *code.summed_target == "pre";
        check(world == 1 || !sv.to_pre, "multi-GPU runs cannot sum into presynaptic neurons");
        sv.dest_pop = sv.to_pre ? def.source_population : def.target_population;
        sv.dest_start = sv.to_pre ? def.source_start : def.target_start;
        sv.dest_count = sv.to_pre ? def.source_count : def.target_count;
        const auto& dpop = m.populations[sv.dest_pop];
        check(bool(code.summed_state), "missing summed target state");
        sv.dest_state = dpop.states.size();
        for (size_t k = 0; k < dpop.states.size(); ++k)
          if (dpop.states[k].name == *code.summed_state) sv.dest_state = k;
        check(sv.dest_state < dpop.states.size(), "missing summed target state");
        const DType dt = dpop.states[sv.dest_state].dtype;
        check(dt == DType::F64 || dt == DType::F32, "summed variables require floating-point state");
        if (procedural) {
          // to_pre: the source-major CSR itself (edge id = position); to_post:
          // its target-major view (positions ascending per target)
          procedural_csr();
          if (sv.to_pre) {
            sv.offsets = proc_off;
            sv.row_other = proc_rows;
          } else if (opt.dry_run) {
            sv.offsets = alloc(0);
            sv.row_other = alloc(0);
            sv.row_edge = alloc(0);
          } else {
            DeviceBuffer off, src, edge, unused;
            build_target_major(static_cast<const uint64_t*>(dptr(proc_off)),
                               static_cast<const uint32_t*>(dptr(proc_rows)), nullptr, nullptr, 0, def.source_count,
                               sd.local_edges, 0, def.target_count, off, src, edge, unused, stream);
            sv.offsets = adopt(std::move(off));
            sv.row_other = adopt(std::move(src));
            sv.row_edge = adopt(std::move(edge));
          }
          sd.summed.push_back(sv);
          continue;
        }
        const auto& idx = sv.to_pre ? src_h : tgt_h;
        const auto& other = sv.to_pre ? tgt_h : src_h;
        const size_t L = sd.local_edges;
        std::vector<uint64_t> offs(sv.dest_count + 1, 0);
        for (size_t k = 0; k < L; ++k) offs[idx[gid(k)] + 1]++;
        for (size_t i = 0; i < sv.dest_count; ++i) offs[i + 1] += offs[i];
        std::vector<uint64_t> next(offs.begin(), offs.end() - 1);
        std::vector<uint32_t> row_other(L), row_edge(L);
        for (size_t k = 0; k < L; ++k) {  // ascending local edge == creation order
          const size_t e = gid(k);
          const uint64_t pos = next[idx[e]]++;
          row_other[pos] = other[e];
          row_edge[pos] = uint32_t(k);
        }
        sv.offsets = upload(offs.data(), offs.size() * 8);
        sv.row_other = upload(row_other.data(), std::max<size_t>(L, 1) * 4);
        sv.row_edge = upload(row_edge.data(), std::max<size_t>(L, 1) * 4);
        sd.summed.push_back(sv);
      }
      syns.push_back(std::move(sd));
    }
    delivered_init.assign(std::max<size_t>(delivered_count, 1), 0);
    delivered_ptr = upload(delivered_init.data(), delivered_init.size() * 8);
  }

  void StreamUse(int s, size_t delay) { streams[size_t(s)].max_delay = std::max(streams[size_t(s)].max_delay, delay); }

  // Header at the start of every rank's shared allocation, checked by each
  // peer in connect(): the GPU's UUID (ranks must sit on distinct GPUs: the
  // exchange waits of one GPU are satisfied by kernels of the others only),
  // and the rank, world size and allocation size (equal models and layouts).
  struct ArenaHeader {
    unsigned char uuid[16];
    int32_t rank, world;
    uint64_t bytes;
    uint64_t magic;
  };
  static constexpr uint64_t kArenaMagic = 0x42324750555845ull;  // "B2GPUXE"
  static constexpr size_t kArenaHeaderBytes = 256;
  size_t arena_bytes_of(int q) const { return arena_stage_off + stage_layout(q).bytes; }

  void build_streams() {
    floors_host_.assign(std::max<size_t>(streams.size(), 1), 0);
    floors_ptr = upload(floors_host_.data(), floors_host_.size() * 8);
    size_t x_bytes = kArenaHeaderBytes;
    for (auto& es : streams) {
      const PopDev& pd = pops[es.pop];
      // the ring holds the population's global spike list (every rank's)
      uint64_t want = opt.ring_capacity ? opt.ring_capacity
                                        : uint64_t(std::max<size_t>(pd.global_count, 1)) * (opt.chunk_ticks + es.max_delay + 2);
      es.cap = next_pow2(std::max<uint64_t>(want, 1024));
      es.mask = es.cap - 1;
      es.ring = alloc(es.cap * 4);
      es.tick_start = alloc((steps + 1) * 8);
      memset_dev(es.tick_start, 8);
      size_t tiles = tiles_for(pd.count), tile_n = tile_n_for(pd.count);
      if (world > 1 && pd.gen_offsets < 0 && !pd.replicated && local_streams_) {
        // local unless an on_pre pathway reads it (it needs every rank's spikes)
        es.local = true;
        for (const auto& sd : syns)
          for (const auto& pw : sd.pathways)
            if (pw.stream == int(&es - streams.data()) && pw.is_pre) es.local = false;
      }
      if (world > 1 && pd.gen_offsets < 0 && !pd.replicated && !es.local) {
        // spike generators emit their (global, precomputed) list on every
        // rank, and replicated populations compute it on every rank
        es.exchanged = true;
        es.consumer_layout = true;
        for (int q = 0; q < world; ++q) {
          const uint64_t cq = part_lo(pd.global_count, q + 1) - part_lo(pd.global_count, q);
          es.x_base.push_back(es.x_half);
          es.x_tiles.push_back(tiles_for(cq));
          es.x_tile_n.push_back(tile_n_for(cq));
          es.x_half += es.x_tiles.back() * (1 + es.x_tile_n.back());
        }
        check(es.x_tiles[size_t(rank)] == tiles && es.x_tile_n[size_t(rank)] == tile_n, "inbox layout mismatch");
        es.x_off = x_bytes;
        x_bytes += (2 * es.x_half * 8 + 255) / 256 * 256;
      }
      es.tile_count = alloc(tiles * 4);
      es.stage = alloc(tiles * tile_n * 4);
      es.done = alloc(8);
      memset_dev(es.done, 8);
      es.starts.assign(1, 0);
    }
    if (world > 1) {
      arena_x_end = x_bytes;
      for (auto& es : streams) {
        if (!es.exchanged) continue;
        for (int q = 0; q < world; ++q) es.xptr.push_back(add_ptr(nullptr));  // own: build_arena; peers: connect()
      }
    }
  }

  // Allocate this rank's shared allocation once the plan has reserved every
  // region in it (inboxes, presynaptic replicas), and point this rank's own
  // slots at it; the peers' slots are filled by connect().
  void build_arena() {
    if (world == 1) return;
    arena_stage_off = (arena_x_end + 255) / 256 * 256;
    const size_t total = arena_bytes_of(rank);
    if (!opt.dry_run) {
      arena = DeviceBuffer(total);
      B2_CUDA(cudaMemsetAsync(arena.ptr, 0, total, stream));  // tag 0 never matches a tick
      cudaDeviceProp prop;
      B2_CUDA(cudaGetDeviceProperties(&prop, device));
      ArenaHeader h{};
      std::memcpy(h.uuid, prop.uuid.bytes, 16);
      h.rank = rank;
      h.world = world;
      h.bytes = total;
      h.magic = kArenaMagic;
      B2_CUDA(cudaMemcpyAsync(arena.ptr, &h, sizeof(h), cudaMemcpyHostToDevice, stream));
      B2_CUDA(cudaStreamSynchronize(stream));
    }
    auto own = [&](size_t off) {
      return opt.dry_run ? uint64_t(0x100000) * (off / 256 + 1)
                         : reinterpret_cast<uint64_t>(static_cast<char*>(arena.ptr) + off);
    };
    for (auto& es : streams)
      if (es.exchanged) ptrs[size_t(es.xptr[size_t(rank)])] = own(es.x_off);
    for (auto& r : replicas) {
      ptrs[size_t(r.rptr[size_t(rank)])] = own(r.off);
      ptrs[size_t(r.fptr[size_t(rank)])] = own(r.flags_off);
    }
  }

  // Read-only replica of one presynaptic state for one reading kernel
  // (multi-GPU; the reference's MPI path keeps the same, distributed.py:255,
  // mpi_codegen.py:300): every rank's block of the variable, copied into
  // every rank's region by a replicate kernel right before the reader, two
  // halves used on alternate ticks, and per (rank, replicate block) a
  // tagged flag.
  struct Replica {
    size_t pop = 0, state = 0, width = 8;
    size_t off = 0, flags_off = 0;  // arena offsets of the data halves and the flag halves
    std::vector<int> rptr, fptr;    // g_ptr slots of every rank's data and flags
  };
  std::vector<Replica> replicas;
  size_t arena_x_end = 0;
  int new_replica(size_t pop, size_t state) {
    Replica r;
    r.pop = pop;
    r.state = state;
    r.width = b2ir::dtype_bytes(m.populations[pop].states[state].dtype);
    r.off = (arena_x_end + 255) / 256 * 256;
    r.flags_off = r.off + (2 * pops[pop].global_count * r.width + 255) / 256 * 256;
    arena_x_end = r.flags_off + 2 * size_t(world) * kReplicaBlocks * 8;
    for (int q = 0; q < world; ++q) r.rptr.push_back(add_ptr(nullptr));
    for (int q = 0; q < world; ++q) r.fptr.push_back(add_ptr(nullptr));
    replicas.push_back(r);
    return int(replicas.size() - 1);
  }

  // Result staging of rank q inside its shared allocation, relative to the
  // staging base: per population the owned state columns, refractory arrays
  // and owned monitor records' samples; per synapse the local edges' states;
  // then the per-pathway event counters.  A pure function of (model, q,
  // world), so rank 0 can read any rank's staging area.
  struct StageLayout {
    size_t bytes = 0, delivered = 0;
    std::vector<uint64_t> lo, count;
    std::vector<std::vector<size_t>> state, monitor, syn_state;
    std::vector<size_t> lastspike, not_refractory;
    std::vector<std::vector<size_t>> mon_positions;  // owned record positions, in record order
    std::vector<std::vector<uint32_t>> syn_edges;    // global ids of the local edges
    std::vector<size_t> local_starts, local_handle;  // per event stream (local streams only)
  };
  StageLayout stage_layout(int q) const {
    StageLayout L;
    auto take = [&L](size_t b) {
      size_t o = L.bytes;
      L.bytes += (b + 255) / 256 * 256;
      return o;
    };
    for (size_t p = 0; p < m.populations.size(); ++p) {
      const auto& def = m.populations[p];
      const PopDev& pd = pops[p];
      const uint64_t lo = stage_lo(p, q), n = stage_count(p, q);
      L.lo.push_back(lo);
      L.count.push_back(n);
      L.state.emplace_back();
      for (const auto& st : def.states) L.state.back().push_back(take(n * b2ir::dtype_bytes(st.dtype)));
      L.lastspike.push_back(pd.lastspike >= 0 ? take(n * 8) : 0);
      L.not_refractory.push_back(pd.lastspike >= 0 ? take(n) : 0);
      L.mon_positions.emplace_back();
      L.monitor.emplace_back();
      if (!pd.mon_dtypes.empty()) {
        for (size_t k = 0; k < def.monitor.record.size(); ++k)
          if (def.monitor.record[k] >= lo && def.monitor.record[k] < lo + n) L.mon_positions.back().push_back(k);
        for (DType d : pd.mon_dtypes)
          L.monitor.back().push_back(take(pd.mon_ticks * L.mon_positions.back().size() * b2ir::dtype_bytes(d)));
      }
    }
    for (size_t s = 0; s < m.synapses.size(); ++s) {
      const auto& def = m.synapses[s];
      const auto& inst = m.synapse_instances[s];
      L.syn_edges.emplace_back();
      L.syn_state.emplace_back();
      if (def.states.empty()) continue;
      const uint64_t lo = part_lo(m.populations[def.target_population].count, q);
      const uint64_t hi = part_lo(m.populations[def.target_population].count, q + 1);
      for (size_t e = 0; e < inst.target.size(); ++e) {
        const uint64_t tp = def.target_start + uint64_t(inst.target[e]);
        if (tp >= lo && tp < hi) L.syn_edges.back().push_back(uint32_t(e));
      }
      for (const auto& st : def.states)
        L.syn_state.back().push_back(take(L.syn_edges.back().size() * b2ir::dtype_bytes(st.dtype)));
    }
    L.delivered = take(std::max<size_t>(delivered_count, 1) * 8);
    // local event lists: per tick the rank's list start (steps + 1 positions),
    // the list length and the CUDA IPC handle of a device copy of the list
    for (const auto& es : streams) {
      L.local_starts.push_back(es.local ? take((steps + 1) * 8) : 0);
      L.local_handle.push_back(es.local ? take(64 + 8) : 0);
    }
    return L;
  }

  // ================================================================ inputs
  std::map<std::string, Input> population_inputs(size_t p, std::map<std::string, WriteTarget>& writable) {
    const auto& def = m.populations[p];
    const PopDev& pd = pops[p];
    std::map<std::string, Input> in;
    in["dt"] = Input::constant(def.dt, DType::F64);
    in["t"] = Input::make(Input::Kind::Time);
    in["N"] = Input::constant(double(def.count), DType::Index);
    in["i"] = Input::make(Input::Kind::Index, Domain::Neuron);
    for (size_t s = 0; s < def.states.size(); ++s) {
      in[def.states[s].name] = Input::make(Input::Kind::State, Domain::Neuron, s, def.states[s].dtype);
      writable[def.states[s].name] = WriteTarget{WriteTarget::Kind::Neuron, s};
    }
    if (pd.lastspike >= 0) {
      in["lastspike"] = Input::make(Input::Kind::LastSpike);
      in["not_refractory"] = Input::make(Input::Kind::Available, Domain::Neuron);
      writable["not_refractory"] = WriteTarget{WriteTarget::Kind::Available, 0};
    }
    for (size_t k = 0; k < def.parameters.size(); ++k) {
      const auto& sym = def.parameters[k];
      auto c = pd.param_const.find(sym.name);
      if (c != pd.param_const.end()) in[sym.name] = Input::constant(c->second, sym.dtype);
      else in[sym.name] = Input::make(Input::Kind::Parameter, Domain::Neuron, k, sym.dtype);
    }
    return in;
  }

  std::map<std::string, Input> synapse_inputs(size_t s, bool is_pre, std::map<std::string, WriteTarget>& writable) {
    const auto& def = m.synapses[s];
    const SynDev& sd = syns[s];
    const auto& src = m.populations[def.source_population];
    const auto& tgt = m.populations[def.target_population];
    std::map<std::string, Input> in;
    in["dt"] = Input::constant((is_pre ? src : tgt).dt, DType::F64);
    in["t"] = Input::make(Input::Kind::Time);
    in["N"] = Input::constant(double(sd.edges), DType::Index);
    in["N_pre"] = Input::constant(double(def.source_count), DType::Index);
    in["N_post"] = Input::constant(double(def.target_count), DType::Index);
    in["i"] = Input::make(Input::Kind::Index, Domain::Pre);
    in["j"] = Input::make(Input::Kind::Index, Domain::Post);
    for (size_t k = 0; k < def.states.size(); ++k) {
      in[def.states[k].name] = Input::make(Input::Kind::SynapseState, Domain::Edge, k, def.states[k].dtype);
    }
    auto index_of = [](const std::vector<b2ir::Symbol>& syms, const std::string& name) {
      for (size_t k = 0; k < syms.size(); ++k)
        if (syms[k].name == name) return k;
      throw Error("alias to unknown state '" + name + "'");
    };
    if (is_pre) {
      for (const auto& [alias, state] : def.pre_state_aliases) {
        size_t k = index_of(src.states, state);
        in[alias] = Input::make(Input::Kind::PreState, Domain::Pre, k, src.states[k].dtype);
        writable[alias] = WriteTarget{WriteTarget::Kind::PreNeuron, k};
      }
    } else {
      for (const auto& [alias, state] : def.pre_state_aliases) {
        size_t k = index_of(src.states, state);
        in[alias] = Input::make(Input::Kind::PreState, Domain::Pre, k, src.states[k].dtype);
      }
    }
    for (const auto& [alias, state] : def.post_state_aliases) {
      size_t k = index_of(tgt.states, state);
      in[alias] = Input::make(Input::Kind::PostState, Domain::Post, k, tgt.states[k].dtype);
      writable[alias] = WriteTarget{WriteTarget::Kind::Neuron, k};
    }
    for (size_t k = 0; k < def.states.size(); ++k)
      writable[def.states[k].name] = WriteTarget{WriteTarget::Kind::Synapse, k};
    if (pops[def.target_population].lastspike >= 0)
      in["not_refractory_post"] = Input::make(Input::Kind::Available, Domain::Post);
    for (size_t k = 0; k < def.parameters.size(); ++k) {
      const auto& sym = def.parameters[k];
      auto c = sd.param_const.find(sym.name);
      if (c != sd.param_const.end()) in[sym.name] = Input::constant(c->second, sym.dtype);
      else in[sym.name] = Input::make(Input::Kind::Parameter, Domain::Edge, k, sym.dtype);
    }
    return in;
  }

  // ================================================================ codegen helpers
  std::string P(int k, const char* type) const { return "((" + std::string(type) + "*)g_ptr[" + std::to_string(k) + "])"; }

  // Neuron-domain context: state slots sv<k>, refractory slots ls/nr.
  // Global neuron index of local lane index `i` (the neuron's identity for
  // the `i` variable and the RNG counter, unchanged by the partition).
  std::string global_index(size_t p) const {
    return pops[p].lo ? "((u64)i + " + u64lit(pops[p].lo) + ")" : "(u64)i";
  }

  EmitContext neuron_ctx(size_t p) {
    EmitContext c;
    const PopDev& pd = pops[p];
    const auto& def = m.populations[p];
    const std::string gi = global_index(p);
    c.load = [this, p, &def, gi](const Input& in) -> std::string {
      const PopDev& pd2 = pops[p];
      switch (in.kind) {
        case Input::Kind::State: return widen(def.states[in.index].dtype, "sv" + std::to_string(in.index));
        case Input::Kind::Parameter: return P(pd2.param_ptr.at(def.parameters[in.index].name), "const double") + "[i]";
        case Input::Kind::Index: return pd2.lo ? "((double)" + gi + ")" : "((double)i)";
        case Input::Kind::LastSpike: return "ls";
        case Input::Kind::Available: return "(nr ? 1.0 : 0.0)";
        default: throw Error("input kind not available in a neuron program");
      }
    };
    (void)pd;
    c.seed = u64lit(m.rng_seed);
    c.tick = "tick";
    c.time = "t";
    c.tables = &const_tables;
    c.device_array = [this](const std::vector<double>& v) { return device_table(v); };
    for (auto& ix : c.index_for_domain) ix = gi;
    return c;
  }

  // Slots a set of neuron programs touch (state indices).
  std::set<size_t> slots_used(const std::vector<const Program*>& progs) {
    std::set<size_t> out;
    for (const Program* pr : progs) {
      for (const auto& b : pr->bindings)
        if (b.second.kind == Input::Kind::State) out.insert(b.second.index);
      for (const auto& w : pr->writes)
        if (w.first.kind == WriteTarget::Kind::Neuron) out.insert(w.first.index);
    }
    return out;
  }
  std::set<size_t> slots_written(const std::vector<const Program*>& progs) {
    std::set<size_t> out;
    for (const Program* pr : progs)
      for (const auto& w : pr->writes)
        if (w.first.kind == WriteTarget::Kind::Neuron) out.insert(w.first.index);
    return out;
  }
  bool writes_available(const std::vector<const Program*>& progs) {
    for (const Program* pr : progs)
      for (const auto& w : pr->writes)
        if (w.first.kind == WriteTarget::Kind::Available) return true;
    return false;
  }

  std::string commits(const Program& pr, size_t p, const std::string& prefix) {
    std::ostringstream o;
    const auto& def = m.populations[p];
    for (const auto& [w, r] : pr.writes) {
      if (w.kind == WriteTarget::Kind::Neuron)
        o << "  sv" << w.index << " = " << narrow(def.states[w.index].dtype, reg_expr(pr, r, prefix)) << ";\n";
      else if (w.kind == WriteTarget::Kind::Available)
        o << "  nr = (u8)(" << reg_expr(pr, r, prefix) << " != 0.0);\n";
    }
    return o.str();
  }

  // Every tick kernel is launched as a programmatic dependent of the previous
  // one: it reads the host-written tick cursor, then waits for its
  // predecessor grid to complete and flush (griddepcontrol.wait) before
  // touching any other memory, and each of its blocks lets the next kernel
  // launch once it has done its work (launch_dependents in kernel_tail).
  // Launch latency and block rasterisation overlap the predecessor's tail;
  // without the launch attribute the wait returns at once.  Triggering at
  // the start instead (B2GPU_PDL_TRIGGER=start) let the next kernel's waiting
  // blocks hold SM slots through long kernels: config 3 ran 430 ms per 1000
  // ticks that way, 248 with the trigger at the end and 251 without PDL;
  // config 2 18.20 / 18.23 / 19.20.
  std::string kernel_head(const std::string& name, unsigned min_blocks = 0) {
    std::string bounds = std::to_string(kThreads) + (min_blocks ? ", " + std::to_string(min_blocks) : "");
    return "extern \"C\" __global__ void __launch_bounds__(" + bounds + ") " + name +
           "(RunCtl* __restrict__ ctl, u32 k) {\n  u32 err = 0;\n" +
           std::string(pdl_trigger_end_ ? "" : "  asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");\n") +
           "  const u64 tick = ctl->tick_base + k;\n"
           "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n"
           "  const u64 rel = tick - " + u64lit(start_tick) + ";\n  const double t = (double)tick * " +
           double_literal(dt) + ";\n  (void)rel; (void)t;\n";
  }
  // With pdl_trigger_end_ a block lets the dependent grid launch only when it
  // has done its work (a block that returns early counts as triggered when it
  // exits), so waiting blocks of the next kernel do not hold SM slots for the
  // whole of a long kernel.
  std::string kernel_tail() const {
    return std::string(pdl_trigger_end_ ? "  asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");\n" : "") +
           "  if (err) atomicOr(&ctl->error, err);\n}\n";
  }

  // ================================================================ step kernels
  // Population step: optional update U, optional threshold X (with ascending
  // compaction into the event ring), optional reset R on fired lanes.
  std::string gen_pop_step(const std::string& name, size_t p, const Program* U, const Program* X, size_t x_event,
                           bool x_is_spike, const Program* R, const std::vector<const Program*>& deferred = {},
                           bool flush = false, bool as_fn = false, const std::vector<PathwayDev*>& applies = {},
                           const Program* post_R = nullptr, const std::vector<PathwayDev*>& deferred_applies = {},
                           const Program* deferred_post_R = nullptr) {
    // One block owns a tile of tile_n consecutive neurons (whole 32-neuron
    // words) and walks it in chunks of kThreads * npt neurons; in a chunk,
    // thread t handles neurons chunk_base + kk*kThreads + t for kk < npt: all
    // loads of the npt neurons are issued before any arithmetic
    // (memory-level parallelism), every access is coalesced, and the fired
    // lanes are counted per (chunk, kk, warp) with ballots.  Tiles are sized
    // so that one wave of resident blocks covers the population with equal
    // shares (tile_n_for), instead of a last partial wave of full tiles.
    //
    // `deferred` programs are trailing neuron maps of the previous tick (e.g.
    // PoissonInput) that the schedule analysis moved to the start of this
    // kernel; they run with the previous tick's t and RNG counter.  A flush
    // kernel applies the last tick's copy at the end of a run or before a
    // state read, and marks it done so the next prologue skips it.
    const auto& def = m.populations[p];
    const PopDev& pd = pops[p];
    const unsigned tile_n = unsigned(tile_n_for(pd.count));
    const unsigned chunk_n = std::min<unsigned>(tile_n, kThreads * npt_);
    const unsigned chunks = (tile_n + chunk_n - 1) / chunk_n;
    const unsigned npt = (chunk_n + kThreads - 1) / kThreads;  // neuron slots per thread and chunk
    constexpr unsigned W = kThreads / 32;
    const unsigned words = tile_n / 32;  // ballot words per tile
    check(tile_n % 32 == 0 && chunks * npt <= 32 && words <= kThreads, "neuron tile layout out of range");
    // offset of slot kk of this thread inside the tile, and whether it lies
    // inside the tile (only needed when the tile is not a whole number of
    // chunks of kThreads)
    const std::string slot_off = "ch * " + std::to_string(chunk_n) + "u + kk * " + std::to_string(kThreads) + "u";
    const bool ragged = tile_n % kThreads != 0 || tile_n % chunk_n != 0;
    const std::string in_tile = ragged ? slot_off + " + threadIdx.x < " + std::to_string(tile_n) + "u && " : "";
    std::vector<const Program*> progs(deferred.begin(), deferred.end());
    for (const Program* pr : {U, X, R, post_R, deferred_post_R})
      if (pr) progs.push_back(pr);
    std::set<size_t> used = slots_used(progs), written = slots_written(progs);
    std::vector<PathwayDev*> all_applies(deferred_applies.begin(), deferred_applies.end());
    all_applies.insert(all_applies.end(), applies.begin(), applies.end());
    for (const PathwayDev* pw : all_applies)
      for (const auto& ad : pw->atomic_adds) {
        used.insert(ad.state);
        written.insert(ad.state);
      }
    bool refr = pd.lastspike >= 0;
    bool touch_refr = refr && (X || (U && pd.fixed_refractory && !flush) || writes_available(progs));
    bool read_refr = refr;
    std::ostringstream o;
    // as_fn: the same code as a device function over one tile, for a launch
    // that steps several populations (block ranges dispatch to the functions)
    if (as_fn)
      o << "__device__ __forceinline__ void " << name
        << "(RunCtl* __restrict__ ctl, u64 tick, u64 rel, double t, u32 tile, u32& err) {\n"
        << "  (void)ctl; (void)tick; (void)rel; (void)t;\n";
    else
      o << kernel_head(name, min_blocks_);
    const EventStreamDev* es = X ? &streams[size_t(pd.stream_of_event[x_event])] : nullptr;
    const bool exchange = es && es->exchanged;
    size_t tiles = tiles_for(pd.count);
    if (!as_fn) o << "  const u32 tile = blockIdx.x;\n";
    if (X) {
      o << "  __shared__ u32 s_ballot[" << words << "];\n  __shared__ u32 s_off[" << words << "];\n";
      if (!es->consumer_layout) o << "  __shared__ u32 s_last;\n";
      o << "  u32 fired_bits = 0;  // bit ch * " << npt << " + kk: this thread's slot fired\n";
    }
    o << "  const u32 lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;\n  (void)lane; (void)warp;\n";
    const bool any_deferred = !deferred.empty() || !deferred_applies.empty() || deferred_post_R;
    if (any_deferred) {
      o << "  const bool run_deferred = rel > 0 && " << P(deferred_flags, "const u64") << "[" << p << "] != tick - 1;\n";
      o << "  const u64 tick_prev = tick - 1;\n  const double t_prev = (double)tick_prev * " << double_literal(dt) << ";\n";
      o << "  (void)t_prev;\n";
    }
    o << "#pragma unroll 1\n  for (u32 ch = 0; ch < " << chunks << "u; ++ch) {\n";
    // ---- load phase
    // Loads of state and of anything an earlier kernel of the tick wrote go
    // through L2 (ld.global.cg), never the read-only path: with programmatic
    // dependent launch the kernel is resident before its predecessor ends,
    // and a read-only (ld.global.nc) load may legally be scheduled ahead of
    // griddepcontrol.wait, reading the value from before that predecessor.
    auto ld = [&](int ptr, const char* ct) { return "__ldcg(" + P(ptr, ct) + " + i)"; };
    for (size_t s : used) {
      const char* ct = storage_ctype(def.states[s].dtype);
      o << "  " << ct << " sva" << s << "[" << npt << "];\n";
    }
    if (read_refr) o << "  double lsa[" << npt << "];\n  u8 nra[" << npt << "];\n";
    // event counters of the counted applies: the previous tick's (deferred)
    // first, then this tick's
    for (size_t a = 0; a < all_applies.size(); ++a) o << "  u32 cna" << a << "[" << npt << "];\n";
    o << "#pragma unroll\n  for (u32 kk = 0; kk < " << npt << "u; ++kk) {\n";
    o << "    const u32 i = tile * " << tile_n << "u + " << slot_off << " + threadIdx.x;\n";
    o << "    if (" << in_tile << "i < " << pd.count << "u) {\n";
    for (size_t a = 0; a < all_applies.size(); ++a) {
      size_t same = a;  // a packed pathway shares the counter word of an earlier one
      for (size_t b = 0; b < a; ++b)
        if (all_applies[b]->count_ptr == all_applies[a]->count_ptr) same = std::min(same, b);
      if (same < a)
        o << "      cna" << a << "[kk] = cna" << same << "[kk];\n";
      else
        o << "      cna" << a << "[kk] = __ldcg(" << P(all_applies[a]->count_ptr, "const u32") << " + i);\n";
    }
    for (size_t s : used) {
      const char* ct = storage_ctype(def.states[s].dtype);
      o << "      sva" << s << "[kk] = " << ld(pops[p].states[s].ptr, ct) << ";\n";
    }
    if (read_refr)
      o << "      lsa[kk] = " << ld(pd.lastspike, "const double") << ";\n      nra[kk] = " << ld(pd.not_refractory, "const u8") << ";\n";
    o << "    }\n  }\n";
    // ---- compute / store phase
    EmitContext ctx = neuron_ctx(p);
    EmitContext prev_ctx = ctx;
    prev_ctx.tick = "tick_prev";
    prev_ctx.time = "t_prev";
    o << "#pragma unroll\n  for (u32 kk = 0; kk < " << npt << "u; ++kk) {\n";
    o << "  const u32 i = tile * " << tile_n << "u + " << slot_off << " + threadIdx.x;\n";
    o << "  const bool active = " << in_tile << "i < " << pd.count << "u;\n";
    o << "  bool fired = false;\n  (void)fired;\n";
    o << "  if (active) {\n";
    for (size_t s : used) o << "  " << storage_ctype(def.states[s].dtype) << " sv" << s << " = sva" << s << "[kk];\n";
    if (read_refr) o << "  double ls = lsa[kk];\n  u8 nr = nra[kk];\n  (void)ls;\n";
    // counted deliveries (in schedule order): the pathway's map applied as
    // often as events reached this neuron, each result rounded to the
    // storage type and checked finite like one delivery of the reference's
    // (executor.rs:2166-2251 per event); the gate is the target's
    // not_refractory as stored by the delivering tick's threshold
    // A finite value plus a constant stays non-finite once it is (inf + w =
    // inf, NaN + w = NaN), so one finite check after the n applications
    // flags exactly the runs in which some application was non-finite.
    auto emit_apply = [&](size_t a, const std::string& cond) {
      const PathwayDev* pw = all_applies[a];
      const std::string c = "cna" + std::to_string(a) + "[kk]";
      o << "  if (" << cond << c << ") {\n    const u32 n_ev = "
        << (pw->count_packed ? "(" + c + " >> " + std::to_string(pw->count_shift) + ") & 65535u" : c) << ";\n";
      o << "    " << P(pw->count_ptr, "u32") << "[i] = 0u;\n";
      o << "    for (u32 r = 0; r < n_ev; ++r) {\n";
      for (const auto& ad : pw->atomic_adds) {
        const std::string v = "sv" + std::to_string(ad.state);
        o << "      " << (ad.gated ? "if (nr) { " : "{ ");
        if (def.states[ad.state].dtype == DType::F64)
          o << v << " = " << v << " + " << double_literal(ad.addend) << ";";
        else
          o << v << " = (float)((double)" << v << " + " << double_literal(ad.addend) << ");";
        o << " }\n";
      }
      o << "    }\n";
      for (const auto& ad : pw->atomic_adds) {
        const std::string v = "sv" + std::to_string(ad.state);
        o << "    if (!b2_finite((double)" << v << ")) err |= " << kErrNonfinite << "u;\n";
      }
      o << "  }\n";
    };
    // the previous tick's trailing dense kernel, in its order: its applies,
    // its program, its reset of the lanes that tick fired
    for (size_t a = 0; a < deferred_applies.size(); ++a) emit_apply(a, "run_deferred && ");
    for (size_t d = 0; d < deferred.size(); ++d) {
      std::string pre = "d" + std::to_string(d) + "_";
      o << "  if (run_deferred) {\n" << emit_program(*deferred[d], prev_ctx, pre) << commits(*deferred[d], p, pre) << "  }\n";
    }
    if (deferred_post_R) {
      check(read_refr, "deferred reset without lastspike");
      o << "  if (run_deferred && ls == t_prev) {\n" << emit_program(*deferred_post_R, prev_ctx, "dr_")
        << commits(*deferred_post_R, p, "dr_") << "  }\n";
    }
    for (size_t a = deferred_applies.size(); a < all_applies.size(); ++a) emit_apply(a, "");
    if (U) {
      if (refr && pd.fixed_refractory && !flush) {
        // timestep(t - lastspike, dt) >= period (model.rs:981-992) is monotone
        // in the f64 difference, so it equals d >= d_star for the host-computed
        // smallest such double; the reference's range errors become d outside
        // [0, d_max).  Same decision for every d, no per-neuron division.
        const double d_star = timestep_threshold(pd.dt, double(pd.period_ticks));
        const double d_max = timestep_threshold(pd.dt, 9223372036854775808.0);
        o << "  { const double d_ls = t - ls;\n";
        o << "    if (!(d_ls >= 0.0 && d_ls < " << double_literal(d_max) << ")) err |= " << kErrTimestep << "u;\n";
        o << "    nr = (u8)(d_ls >= " << double_literal(d_star) << "); }\n";
      }
      o << "  {\n" << emit_program(*U, ctx, "u_") << commits(*U, p, "u_") << "  }\n";
    }
    if (X) {
      o << "  {\n" << emit_program(*X, ctx, "h_");
      o << "  fired = " << reg_expr(*X, size_t(X->condition), "h_") << " != 0.0";
      if (x_is_spike && refr) o << " && nr";
      o << ";\n";
      o << commits(*X, p, "h_") << "  }\n";
      if (x_is_spike && refr) o << "  if (fired) { ls = t; nr = 0; }\n";
    }
    if (R) o << "  if (fired) {\n" << emit_program(*R, ctx, "r_") << commits(*R, p, "r_") << "  }\n";
    if (post_R) {
      check(read_refr, "trailing reset without lastspike");
      o << "  if (ls == t) {\n" << emit_program(*post_R, ctx, "pr_") << commits(*post_R, p, "pr_") << "  }\n";
    }
    for (size_t s : written) {
      const char* ct = storage_ctype(def.states[s].dtype);
      o << "  " << P(pops[p].states[s].ptr, ct) << "[i] = sv" << s << ";\n";
    }
    if (touch_refr) {
      if (X && x_is_spike) o << "  if (fired) " << P(pd.lastspike, "double") << "[i] = ls;\n";
      o << "  " << P(pd.not_refractory, "u8") << "[i] = nr;\n";
    }
    o << "  }\n";  // active
    if (X) {
      // ballot word ch * npt * W + kk * W + warp of the tile covers its
      // neurons 32 * (that word) .. + 31 (chunks are whole words)
      const std::string word = "ch * " + std::to_string(npt * W) + "u + kk * " + std::to_string(W) + "u + warp";
      const std::string warp_in_tile =
          ragged ? slot_off + " + warp * 32u < " + std::to_string(tile_n) + "u" : std::string("true");
      o << "  const u32 b = __ballot_sync(0xffffffffu, fired);\n";
      o << "  if (lane == 0 && " << warp_in_tile << ") s_ballot[" << word << "] = b;\n";
      if (es->bitmap >= 0) {
        // fired bitmap for target-ordered pathways: word w covers neurons
        // 32w .. 32w + 31 (tile_n is a multiple of 32)
        o << "  { const u32 bw = tile * " << words << "u + " << word << ";\n";
        o << "    if (lane == 0 && " << warp_in_tile << " && bw < " << es->bm_words << "u) " << P(es->bitmap, "u32")
          << "[(rel % " << es->bm_slots << "ull) * " << es->bm_words << "ull + bw] = b; }\n";
      }
      o << "  fired_bits |= (fired ? 1u : 0u) << (ch * " << npt << "u + kk);\n";
    }
    o << "  }\n";  // kk loop
    o << "  }\n";  // chunk loop
    if (flush) o << "  if (blockIdx.x == 0 && threadIdx.x == 0) " << P(deferred_flags, "u64") << "[" << p << "] = tick;\n";
    if (X) {
      // Tile-local ascending compaction (warp 0 scans the tile's ballot
      // words, per lane a contiguous run of them).  Then one of:
      //  * exchanged list: the tile's count and ids go straight to every
      //    rank's inbox (tagged 8-byte peer stores), no wait on other blocks;
      //  * list laid out by its consumer: the tile's count and ids stay in
      //    tile_count / stage for the next kernel;
      //  * otherwise the last block to finish lays all tiles out in the ring
      //    (b2_finalize_spikes).
      const unsigned per = (words + 31) / 32;
      const std::string gid =
          ((es->local || exchange) && pd.lo ? std::to_string(pd.lo) + "u + " : std::string()) + "tile * " +
          std::to_string(tile_n) + "u + " + slot_off + " + threadIdx.x";
      // rank q's inbox words of this tile: its count, and its first id
      auto peer = [&](const std::string& q, bool ids) {
        return "(((u64*)g_ptr[" + std::to_string(es->xptr[0]) + " + " + q + "]) + (rel & 1ull) * " +
               std::to_string(es->x_half) + "ull + " + std::to_string(exchange ? es->x_base[size_t(rank)] : 0) +
               (ids ? "ull + " + std::to_string(tiles) + "ull + (u64)tile * " + std::to_string(tile_n) + "ull)"
                    : "ull + (u64)tile)");
      };
      o << "  __syncthreads();\n";
      o << "  if (warp == 0) {\n";
      o << "    u32 c = 0;\n";
      o << "#pragma unroll\n    for (u32 j = 0; j < " << per << "u; ++j) { const u32 w = lane * " << per
        << "u + j; if (w < " << words << "u) c += __popc(s_ballot[w]); }\n";
      o << "    u32 x = c;\n";
      o << "#pragma unroll\n    for (int d = 1; d < 32; d <<= 1) { u32 y = __shfl_up_sync(0xffffffffu, x, d); if (lane >= (u32)d) x += y; }\n";
      o << "    u32 acc = x - c;\n";
      o << "#pragma unroll\n    for (u32 j = 0; j < " << per << "u; ++j) { const u32 w = lane * " << per
        << "u + j; if (w < " << words << "u) { s_off[w] = acc; acc += __popc(s_ballot[w]); } }\n";
      if (exchange)
        o << "    if (lane == 31) for (u32 q = 0; q < " << world << "u; ++q) b2_ll_store(" << peer("q", false)
          << ", x, (u32)(rel + 1ull));\n";
      else
        o << "    if (lane == 31) " << P(es->tile_count, "u32") << "[tile] = x;\n";
      o << "  }\n";
      o << "  __syncthreads();\n";
      o << "  if (fired_bits) {\n";
      if (!exchange) o << "    u32* stage = " << P(es->stage, "u32") << " + (u64)tile * " << tile_n << "u;\n";
      o << "    for (u32 f = fired_bits; f; f &= f - 1u) {\n";
      o << "      const u32 bit = (u32)(__ffs(f) - 1), ch = bit / " << npt << "u, kk = bit % " << npt << "u;\n";
      o << "      const u32 slot = ch * " << npt * W << "u + kk * " << W << "u + warp;\n";
      o << "      const u32 pos = s_off[slot] + __popc(s_ballot[slot] & ((1u << lane) - 1u));\n";
      // global ids (a multi-GPU list covers the block [lo, lo + count))
      if (exchange)
        o << "      for (u32 q = 0; q < " << world << "u; ++q) b2_ll_store(" << peer("q", true) << " + pos, " << gid
          << ", (u32)(rel + 1ull));\n";
      else
        o << "      stage[pos] = " << gid << ";\n";
      o << "    }\n  }\n";
      if (!es->consumer_layout) {
        // Only the threads that staged ids, and the one that wrote the
        // tile's count, need their writes visible to the last block: they
        // fence, the barrier orders the fences before the ticket.
        o << "  if (fired_bits || (warp == 0 && lane == 31)) __threadfence();\n  __syncthreads();\n";
        o << "  if (threadIdx.x == 0) s_last = (atomicAdd((unsigned long long*)" << P(es->done, "u64") << ", 1ull) % "
          << tiles << "ull) == " << tiles - 1 << "ull;\n";
        o << "  __syncthreads();\n";
        o << "  if (s_last) {\n    __threadfence();\n";
        o << "    b2_finalize_spikes<" << kThreads << ">(" << tiles << "u, " << tile_n << "u, " << P(es->tile_count, "const u32")
          << ", " << P(es->stage, "const u32") << ", " << P(es->ring, "u32") << ", " << u64lit(es->mask) << ", "
          << P(es->tick_start, "u64") << ", rel, " << u64lit(es->cap) << ", " << floor_of(size_t(pd.stream_of_event[x_event]))
          << ", err);\n  }\n";
      }
    }
    o << (as_fn ? std::string("}\n") : kernel_tail());
    return o.str();
  }

  // The layout part of a list consumer: the definitions that read the
  // tick's per-tile counts and ids (this rank's inbox when the list is
  // exchanged, else the step's tile_count / stage) and the layout blocks
  // (the first `lb` blocks of the launch) that lay the list out in the ring
  // and write tick_start[rel + 1].  Used by gen_consumer and by a scatter
  // kernel that lays out another tick's list alongside its delivery.
  std::string emit_list_layout(int stream_id, unsigned lb) {
    const EventStreamDev& es = streams[size_t(stream_id)];
    const PopDev& pd = pops[es.pop];
    const bool remote = es.exchanged;
    const uint64_t timeout_ns = uint64_t(opt.exchange_timeout_ms) * 1000000ull;
    uint64_t pairs = 0;
    std::vector<uint64_t> pair_start;  // remote: first pair of each rank
    if (remote) {
      for (int q = 0; q < world; ++q) {
        pair_start.push_back(pairs);
        pairs += es.x_tiles[size_t(q)];
      }
    } else {
      pairs = tiles_for(pd.count);
    }
    check(pairs <= 8192, "spike list layout: too many tiles");
    const unsigned per = unsigned((pairs + kThreads - 1) / kThreads);
    std::ostringstream o;
    if (remote) {
      // once the run has failed (e.g. an earlier wait expired) later ticks
      // must not wait again: their results are discarded anyway
      o << "  const bool poisoned = *(volatile const u32*)&ctl->error != 0u;\n";
      o << "  const u64* inbox = ((const u64*)g_ptr[" << es.xptr[size_t(rank)] << "]) + (rel & 1ull) * " << es.x_half
        << "ull;\n";
      o << "  const u32 tag = (u32)(rel + 1ull);\n";
      // words of pair p's count and of its first id in this rank's inbox
      o << "  auto slot = [](u32 p) -> u64 {\n";
      for (int q = world - 1; q >= 0; --q)
        o << "    " << (q ? "if (p >= " + std::to_string(pair_start[size_t(q)]) + "u) " : std::string()) << "return "
          << es.x_base[size_t(q)] << "ull + (u64)(p - " << pair_start[size_t(q)] << "u);\n";
      o << "  };\n";
      o << "  auto id_slot = [](u32 p) -> u64 {\n";
      for (int q = world - 1; q >= 0; --q)
        o << "    " << (q ? "if (p >= " + std::to_string(pair_start[size_t(q)]) + "u) " : std::string()) << "return "
          << es.x_base[size_t(q)] + es.x_tiles[size_t(q)] << "ull + (u64)(p - " << pair_start[size_t(q)] << "u) * "
          << es.x_tile_n[size_t(q)] << "ull;\n";
      o << "  };\n";
      // a thread whose wait has expired waits no more (the run is failed)
      o << "  auto count_of = [&](u32 p) -> u32 { return poisoned || (err & " << kErrExchange
        << "u) ? 0u : b2_ll_wait(inbox + slot(p), tag, " << timeout_ns << "ull, err); };\n";
      o << "  auto id_of = [&](u32 p, u32 k) -> u32 { return poisoned || (err & " << kErrExchange
        << "u) ? 0u : b2_ll_wait(inbox + id_slot(p) + k, tag, " << timeout_ns << "ull, err); };\n";
    } else {
      o << "  auto count_of = [&](u32 p) -> u32 { return __ldcg(" << P(es.tile_count, "const u32") << " + p); };\n";
      o << "  auto id_of = [&](u32 p, u32 k) -> u32 { return __ldcg(" << P(es.stage, "const u32") << " + (u64)p * "
        << tile_n_for(pd.count) << "u + k); };\n";
    }
    // ---- layout blocks
    o << "  if (blockIdx.x < " << lb << "u) {\n";
    o << "    __shared__ u32 s_pre[" << pairs + 1 << "];\n";
    // every pair's count into s_pre, coalesced (thread x reads pairs x,
    // x + threads, ...), all loads in flight together; an exchanged word
    // whose tag is not yet this tick's is waited for (bounded)
    o << "    {\n";
    if (remote) {
      o << "      u64 raw[" << per << "];\n";
      o << "#pragma unroll\n      for (u32 j = 0; j < " << per << "u; ++j) { const u32 p = j * " << kThreads
        << "u + threadIdx.x; raw[j] = p < " << pairs << "u && !poisoned ? b2_ll_load(inbox + slot(p)) : 0ull; }\n";
      o << "#pragma unroll\n      for (u32 j = 0; j < " << per << "u; ++j) { const u32 p = j * " << kThreads
        << "u + threadIdx.x; if (p < " << pairs << "u) s_pre[p] = (u32)(raw[j] >> 32) == tag ? (u32)raw[j] : count_of(p); }\n";
    } else {
      o << "      u32 cv[" << per << "];\n";
      o << "#pragma unroll\n      for (u32 j = 0; j < " << per << "u; ++j) { const u32 p = j * " << kThreads
        << "u + threadIdx.x; cv[j] = p < " << pairs << "u ? count_of(p) : 0u; }\n";
      o << "#pragma unroll\n      for (u32 j = 0; j < " << per << "u; ++j) { const u32 p = j * " << kThreads
        << "u + threadIdx.x; if (p < " << pairs << "u) s_pre[p] = cv[j]; }\n";
    }
    o << "    }\n    __syncthreads();\n";
    // then each thread scans a contiguous run of pairs
    o << "    u32 cnt[" << per << "];\n";
    o << "#pragma unroll\n    for (u32 j = 0; j < " << per << "u; ++j) { const u32 p = threadIdx.x * " << per
      << "u + j; cnt[j] = p < " << pairs << "u ? s_pre[p] : 0u; }\n";
    o << "    u32 c = 0;\n#pragma unroll\n    for (u32 j = 0; j < " << per << "u; ++j) c += cnt[j];\n";
    o << "    u32 total;\n    u32 off = b2_block_exclusive_scan<" << kThreads << ">(c, &total);\n";
    o << "#pragma unroll\n    for (u32 j = 0; j < " << per << "u; ++j) { const u32 p = threadIdx.x * " << per
      << "u + j; if (p < " << pairs << "u) { s_pre[p] = off; off += cnt[j]; } }\n";
    o << "    if (threadIdx.x == 0) s_pre[" << pairs << "] = total;\n";
    o << "    __syncthreads();\n";
    o << "    const u64 base = " << P(es.tick_start, "const u64") << "[rel];\n";
    o << "    u32* ring = " << P(es.ring, "u32") << ";\n";
    // last pair whose offset is <= g (pairs with no ids share the next
    // pair's offset, so the last one is the pair that holds position g)
    o << "    for (u32 g = blockIdx.x * " << kThreads << "u + threadIdx.x; g < total; g += " << lb * kThreads << "u) {\n";
    o << "      u32 lo = 0, hi = " << pairs - 1 << "u;\n";
    o << "      while (lo < hi) { const u32 mid = (lo + hi + 1u) >> 1; if (s_pre[mid] <= g) lo = mid; else hi = mid - 1u; }\n";
    o << "      ring[(base + g) & " << u64lit(es.mask) << "] = id_of(lo, g - s_pre[lo]);\n    }\n";
    o << "    if (blockIdx.x == 0 && threadIdx.x == 0) {\n";
    o << "      const u64 end = base + total;\n      " << P(es.tick_start, "u64") << "[rel + 1] = end;\n";
    o << "      if (end - " << floor_of(size_t(stream_id)) << " > " << u64lit(es.cap) << ") err |= " << kErrRing
      << "u;\n    }\n";
    o << "  }\n";
    return o.str();
  }

  // Consumer layout of a tick's list (gen_pop_step leaves it as per-tile
  // counts and ids): pair p = (rank, tile) in rank-then-tile order, which is
  // ascending neuron order.  No block waits for another:
  //  * layout blocks (the first `lb` of the grid) each read every pair's
  //    count (waiting, bounded, for a peer's tagged word where the list is
  //    exchanged), scan them into the pairs' offsets, so that position g of
  //    the list lies in the last pair whose offset is <= g, and copy the list
  //    into the ring (position g -> thread g of the layout blocks); block 0
  //    writes tick_start[rel + 1].  Rank order is global order, so an
  //    exchanged list is ascending without a sort (the reference's MPI path
  //    sorts the gathered ids, mpi_codegen.py:79-82);
  //  * `fused`: the delay-0 constant-addend pathways of the stream, whose
  //    result does not depend on the order of events, are delivered by the
  //    other blocks straight from the tile lists: block b takes pairs b,
  //    b + blocks, ... (one count read per pair, all of a block's at once),
  //    and its warps share the block's work items (id, 256-entry row chunk),
  //    so the scatter needs no ring read, no prefix over all tiles and no
  //    kernel boundary of its own.
  std::string gen_consumer(const std::string& name, int stream_id, const std::vector<PathwayDev*>& fused,
                           unsigned grid, unsigned lb) {
    const EventStreamDev& es = streams[size_t(stream_id)];
    const PopDev& pd = pops[es.pop];
    const bool remote = es.exchanged;
    const uint64_t timeout_ns = uint64_t(opt.exchange_timeout_ms) * 1000000ull;
    uint64_t pairs = 0;
    std::vector<uint64_t> pair_start;  // remote: first pair of each rank
    if (remote) {
      for (int q = 0; q < world; ++q) {
        pair_start.push_back(pairs);
        pairs += es.x_tiles[size_t(q)];
      }
    } else {
      pairs = tiles_for(pd.count);
    }
    check(pairs <= 8192, "spike list layout: too many tiles");
    check(lb >= 1 && lb <= grid && (fused.empty() ? lb == grid : grid > lb), "spike list layout: bad grid split");
    const unsigned per = unsigned((pairs + kThreads - 1) / kThreads);
    constexpr unsigned W = kThreads / 32;
    std::ostringstream o;
    o << kernel_head(name);
    o << "  const u32 lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;\n  (void)lane; (void)warp;\n";
    o << emit_list_layout(stream_id, lb);
    if (!fused.empty()) {
      // ---- scatter blocks
      const unsigned blocks = grid - lb;
      const unsigned mine = unsigned((pairs + blocks - 1) / blocks);  // pairs per block, at most
      check(mine <= kThreads, "spike list layout: too many tiles per scatter block");
      const PathwayDev& p0 = *fused.front();
      const size_t endpoint_count = m.populations[p0.endpoint_pop].count;
      uint64_t chunks = 1;
      for (const PathwayDev* pw : fused) chunks = std::max<uint64_t>(chunks, (pw->max_row + 255) / 256);
      o << "  else {\n";
      // per pair its count and, fetched in the same round trip, its first id
      // (most tiles hold at most one spike): the first id's word is read
      // before the count is known and used once the count says it is part of
      // this tick's list (exchanged: once its tag is this tick's)
      o << "    __shared__ u32 s_cnt[" << mine << "], s_id0[" << mine << "];\n";
      o << "    const u32 b = blockIdx.x - " << lb << "u;\n";
      o << "    if (threadIdx.x < " << mine << "u) {\n      const u32 p = b + threadIdx.x * " << blocks
        << "u;\n      u32 c = 0, i0 = 0;\n";
      o << "      if (p < " << pairs << "u) {\n";
      if (remote)
        o << "        const u64 v0 = poisoned ? 0ull : b2_ll_load(inbox + id_slot(p));\n"
          << "        c = count_of(p);\n"
          << "        if (c) i0 = (u32)(v0 >> 32) == tag ? (u32)v0 : id_of(p, 0u);\n";
      else
        o << "        i0 = id_of(p, 0u);\n        c = count_of(p);\n";
      o << "      }\n      s_cnt[threadIdx.x] = c;\n      s_id0[threadIdx.x] = i0;\n    }\n";
      o << "    __syncthreads();\n";
      for (size_t k = 0; k < fused.size(); ++k) o << "    u64 events" << k << " = 0;\n";
      // the block's items in (pair, id, chunk) order; warp w takes items
      // w, w + W, ...
      o << "    u32 item = 0;\n";
      o << "    for (u32 j = 0; j < " << mine << "u; ++j) {\n";
      o << "      const u32 n = s_cnt[j], p = b + j * " << blocks << "u;\n";
      o << "      for (u32 kk = 0; kk < n; ++kk)\n";
      o << "        for (u32 c = 0; c < " << chunks << "u; ++c, ++item) {\n";
      o << "          if (item % " << W << "u != warp) continue;\n";
      o << "          const u32 s = kk == 0u ? s_id0[j] : id_of(p, kk);\n";
      for (size_t k = 0; k < fused.size(); ++k) {
        const PathwayDev& pw = *fused[k];
        const size_t lo = pw.endpoint_start, hi = pw.endpoint_start + pw.endpoint_count;
        const bool full = lo == 0 && hi == endpoint_count;
        o << "          " << (full ? "{" : "if (s >= " + std::to_string(lo) + "u && s < " + std::to_string(hi) + "u) {")
          << "\n";
        o << "            const u64* off = " << P(pw.offsets, "const u64") << ";\n";
        o << "            const u32* other = " << P(pw.row_other, "const u32") << ";\n";
        o << "            const u32 ep = s - " << lo << "u;\n";
        o << "            const u64 r0 = __ldg(off + ep), r1 = __ldg(off + ep + 1);\n";
        o << "            if (c == 0 && lane == 0) events" << k << " += r1 - r0;\n";
        o << "            const u64 q0 = r0 + c * 256ull;\n";
        o << "            const u64 q1 = q0 + 256ull < r1 ? q0 + 256ull : r1;\n";
        o << emit_warp_chunk(pw, "            ");
        o << "          }\n";
      }
      o << "        }\n    }\n";
      for (size_t k = 0; k < fused.size(); ++k)
        o << "    if (lane == 0 && events" << k << ") atomicAdd((unsigned long long*)" << P(delivered_ptr, "u64") << " + "
          << fused[k]->delivered_slot << ", events" << k << ");\n";
      o << "  }\n";
    }
    o << kernel_tail();
    return o.str();
  }

  // `(summed)` variable (run_summed_program, executor.rs:2548-2597): one
  // thread per destination neuron this rank owns clears it and adds its
  // edges' values in creation order, rounding each addition to the storage
  // type (StateArray::add_f64, executor.rs:517-523).  Destinations are
  // independent (a summed expression never reads its own summed variable),
  // so the per-neuron order is the reference's whole order.
  std::string gen_summed_body(const std::string& fname, const SummedSpec& ss) {
    const auto& def = m.synapses[ss.synapse];
    std::ostringstream o;
    o << "__device__ __forceinline__ double " << fname << "(u32 src, u32 tgt, u64 edge, u64 tick, double t, u32& err) {\n";
    o << "  const u64 src_state = (u64)src + " << def.source_start << "ull;\n";
    o << "  const u64 tgt_state = (u64)tgt + " << target_bias(def) << "ull;\n";
    o << "  (void)src_state; (void)tgt_state; (void)t; (void)tick; (void)edge;\n";
    PathwayDev none;
    o << emit_program(*ss.program, event_ctx(ss.synapse, none, &ss.pre_replica), "e_");
    o << "  return " << reg_expr(*ss.program, ss.result, "e_") << ";\n}\n";
    return o.str();
  }

  std::string gen_summed(const std::string& name, const std::string& body, const SummedSpec& ss) {
    const SynDev::Summed& sv = syns[ss.synapse].summed[ss.k];
    const PopDev& dp = pops[sv.dest_pop];
    const DType dt = m.populations[sv.dest_pop].states[sv.dest_state].dtype;
    const char* ct = storage_ctype(dt);
    // destinations (synapse-level indices) whose neuron this rank owns
    auto clampd = [&](uint64_t x) {
      return x <= sv.dest_start ? uint64_t(0) : std::min<uint64_t>(x - sv.dest_start, sv.dest_count);
    };
    const uint64_t d0 = clampd(dp.lo), d1 = clampd(dp.lo + dp.count);
    std::ostringstream o;
    o << kernel_head(name);
    o << "  const u64 d = " << d0 << "ull + blockIdx.x * (u64)blockDim.x + threadIdx.x;\n";
    o << "  if (d < " << d1 << "ull) {\n";
    o << "    const u64* off = " << P(sv.offsets, "const u64") << ";\n";
    o << "    const u32* other = " << P(sv.row_other, "const u32") << ";\n";
    if (sv.row_edge >= 0) o << "    const u32* ed = " << P(sv.row_edge, "const u32") << ";\n";
    const std::string edge = sv.row_edge >= 0 ? "(u64)ed[q]" : "q";
    o << "    " << ct << " acc = " << narrow(dt, "0.0") << ";\n";
    o << "    for (u64 q = off[d]; q < off[d + 1]; ++q) {\n";
    if (sv.to_pre)
      o << "      const double v = " << body << "((u32)d, other[q], " << edge << ", tick, t, err);\n";
    else
      o << "      const double v = " << body << "(other[q], (u32)d, " << edge << ", tick, t, err);\n";
    o << "      acc = " << narrow(dt, widen(dt, "acc") + " + v") << ";\n    }\n";
    o << "    " << P(dp.states[sv.dest_state].ptr, ct) << "[d + " << uint64_t(sv.dest_start) - dp.lo << "ull] = acc;\n";
    o << "  }\n";
    o << kernel_tail();
    return o.str();
  }

  // Reset over the tick's fired list (one thread per spike).
  // No initial lastspike of population p is at or after the run's first
  // tick, so during the run lastspike == t holds exactly for the neurons the
  // tick's threshold fired.
  bool lastspike_before_start(size_t p) const {
    const auto& inst = m.population_instances[p];
    if (!inst.refractory) return false;
    const double t0 = double(start_tick) * dt;
    for (double v : inst.refractory->initial_lastspike)
      if (v >= t0) return false;
    return true;
  }

  std::string gen_reset(const std::string& name, size_t p, const Program& R, int stream_id) {
    const auto& def = m.populations[p];
    const EventStreamDev& es = streams[size_t(stream_id)];
    std::vector<const Program*> progs{&R};
    std::set<size_t> used = slots_used(progs), written = slots_written(progs);
    bool refr = pops[p].lastspike >= 0;
    std::ostringstream o;
    o << kernel_head(name);
    o << "  const u64* ts = " << P(es.tick_start, "u64") << ";\n  const u64 a = ts[rel], b = ts[rel + 1];\n";
    o << "  for (u64 j = a + blockIdx.x * (u64)blockDim.x + threadIdx.x; j < b; j += (u64)gridDim.x * blockDim.x) {\n";
    if (world > 1) {
      o << "    const u32 sid = " << P(es.ring, "const u32") << "[j & " << u64lit(es.mask) << "];\n";
      o << "    if (sid < " << pops[p].lo << "u || sid >= " << pops[p].lo + pops[p].count << "u) continue;\n";
      o << "    const u32 i = sid - " << pops[p].lo << "u;\n";
    } else {
      o << "    const u32 i = " << P(es.ring, "const u32") << "[j & " << u64lit(es.mask) << "];\n";
    }
    for (size_t s : used) {
      const char* ct = storage_ctype(def.states[s].dtype);
      o << "    " << ct << " sv" << s << " = " << P(pops[p].states[s].ptr, ct) << "[i];\n";
    }
    if (refr) o << "    double ls = " << P(pops[p].lastspike, "double") << "[i];\n    u8 nr = " << P(pops[p].not_refractory, "u8") << "[i];\n    (void)ls; (void)nr;\n";
    EmitContext ctx = neuron_ctx(p);
    o << "  {\n" << emit_program(R, ctx, "r_") << commits(R, p, "r_") << "  }\n";
    for (size_t s : written) {
      const char* ct = storage_ctype(def.states[s].dtype);
      o << "    " << P(pops[p].states[s].ptr, ct) << "[i] = sv" << s << ";\n";
    }
    if (refr && writes_available(progs)) o << "    " << P(pops[p].not_refractory, "u8") << "[i] = nr;\n";
    o << "  }\n" << kernel_tail();
    return o.str();
  }

  std::string gen_state_monitor(const std::string& name, size_t p) {
    const auto& def = m.populations[p];
    const PopDev& pd = pops[p];
    size_t nrec = pd.mon_nrec, nvar = def.monitor.variables.size();
    std::ostringstream o;
    o << kernel_head(name);
    o << "  if (tick < " << u64lit(pd.mon_first_tick) << ") return;\n";
    o << "  const u64 row = tick - " << u64lit(pd.mon_first_tick) << ";\n";
    o << "  const u32 x = blockIdx.x * blockDim.x + threadIdx.x;\n  if (x >= " << nrec * nvar << "u) return;\n";
    o << "  const u32 var = x / " << nrec << "u, r = x % " << nrec << "u;\n";
    o << "  const u32 i = " << P(pd.mon_records, "const u32") << "[r];\n  (void)i;\n";
    for (size_t v = 0; v < nvar; ++v) {
      const std::string& vname = def.monitor.variables[v];
      DType d = pd.mon_dtypes[v];
      const char* ct = storage_ctype(d);
      std::string value;
      bool is_state = false;
      for (size_t s = 0; s < def.states.size(); ++s)
        if (def.states[s].name == vname) {
          value = P(pd.states[s].ptr, ct) + "[i]";
          is_state = true;
        }
      if (!is_state) {
        auto c = pd.param_const.find(vname);
        std::string reg = c != pd.param_const.end() ? double_literal(c->second)
                                                    : P(pd.param_ptr.at(vname), "const double") + "[i]";
        value = narrow(d, reg);
      }
      o << "  if (var == " << v << "u) " << P(pd.mon_samples[v], ct) << "[row * " << nrec << "ull + r] = " << value << ";\n";
    }
    o << kernel_tail();
    return o.str();
  }

  std::string gen_event_source(const std::string& name, size_t p, int stream_id) {
    const PopDev& pd = pops[p];
    const EventStreamDev& es = streams[size_t(stream_id)];
    std::ostringstream o;
    o << kernel_head(name);
    o << "  const u64* go = " << P(pd.gen_offsets, "const u64") << ";\n  const u64 a = go[rel], b = go[rel + 1];\n";
    o << "  const u64 base = " << P(es.tick_start, "u64") << "[rel];\n";
    o << "  for (u64 j = a + threadIdx.x; j < b; j += blockDim.x) " << P(es.ring, "u32") << "[(base + j - a) & "
      << u64lit(es.mask) << "] = " << P(pd.gen_ids, "const u32") << "[j];\n";
    o << "  if (threadIdx.x == 0) {\n    " << P(es.tick_start, "u64") << "[rel + 1] = base + (b - a);\n";
    o << "    if (base + (b - a) - " << floor_of(size_t(stream_id)) << " > " << u64lit(es.cap) << ") err |= " << kErrRing << "u;\n  }\n";
    o << kernel_tail();
    return o.str();
  }

  // EventMonitor variables (record_events, executor.rs:3053-3080): for every
  // event of the monitored list (this tick's, or the previous tick's when the
  // monitor runs before the event's producer), the variables' current values,
  // stored at the event's ring position.
  std::string gen_evmon(const std::string& name, size_t p, size_t k) {
    const auto& def = m.populations[p];
    const PopDev& pd = pops[p];
    const auto& em = def.event_monitors[k];
    const EventStreamDev& es = streams[size_t(pd.evmon_stream[k])];
    const size_t lag = size_t(pd.evmon_lag[k]);
    std::ostringstream o;
    o << kernel_head(name);
    o << "  if (rel < " << lag << "ull) return;\n  const u64 te = rel - " << lag << "ull;\n";
    o << "  const u64* ts = " << P(es.tick_start, "const u64") << ";\n";
    o << "  for (u64 j = ts[te] + blockIdx.x * (u64)blockDim.x + threadIdx.x; j < ts[te + 1]; j += (u64)gridDim.x * blockDim.x) {\n";
    o << "    const u64 r = j & " << u64lit(es.mask) << ";\n";
    o << "    const u32 n = " << P(es.ring, "const u32") << "[r];\n";
    for (size_t v = 0; v < em.variables.size(); ++v) {
      const std::string& name_v = em.variables[v];
      const int out = pd.evmon_vars[k].ring[v];
      bool done_v = false;
      for (size_t s = 0; s < def.states.size() && !done_v; ++s)
        if (def.states[s].name == name_v) {
          const char* ct = storage_ctype(def.states[s].dtype);
          o << "    ((" << ct << "*)g_ptr[" << out << "])[r] = " << P(pd.states[s].ptr, ct) << "[n];\n";
          done_v = true;
        }
      if (done_v) continue;
      auto ptr = pd.param_ptr.find(name_v);
      if (ptr != pd.param_ptr.end())
        o << "    ((double*)g_ptr[" << out << "])[r] = " << P(ptr->second, "const double") << "[n];\n";
      else
        o << "    ((double*)g_ptr[" << out << "])[r] = " << double_literal(pd.param_const.at(name_v)) << ";\n";
    }
    o << "  }\n";
    o << kernel_tail();
    return o.str();
  }

  std::string gen_empty_stream(const std::string& name, int stream_id) {
    const EventStreamDev& es = streams[size_t(stream_id)];
    std::ostringstream o;
    o << kernel_head(name);
    o << "  if (threadIdx.x == 0) " << P(es.tick_start, "u64") << "[rel + 1] = " << P(es.tick_start, "u64") << "[rel];\n";
    o << kernel_tail();
    return o.str();
  }

  // ---------------------------------------------------------------- pathways
  // Offset from a synapse-level target index j to the target's local state
  // index: target_start + j - (first neuron this rank owns), modulo 2^64 (the
  // true value is never negative for a stored edge).
  uint64_t target_bias(const b2ir::SynapseDef& def) const {
    return uint64_t(def.target_start) - pops[def.target_population].lo;
  }

  EmitContext event_ctx(size_t s, const PathwayDev& pw, const std::map<size_t, int>* pre_replica = nullptr) {
    EmitContext c;
    const auto& def = m.synapses[s];
    c.load = [this, s, &def, pre_replica](const Input& in) -> std::string {
      const SynDev& sd = syns[s];
      const auto& src = m.populations[def.source_population];
      const auto& tgt = m.populations[def.target_population];
      switch (in.kind) {
        case Input::Kind::PreState: {
          DType d = src.states[in.index].dtype;
          if (pre_replica && pre_replica->count(in.index)) {
            // every rank's block, copied this tick (half (tick - start) & 1)
            const Replica& r = replicas[size_t(pre_replica->at(in.index))];
            return widen(d, "__ldcg(" + P(r.rptr[size_t(rank)], (std::string("const ") + storage_ctype(d)).c_str()) +
                                " + ((tick - " + u64lit(start_tick) + ") & 1ull) * " +
                                std::to_string(pops[def.source_population].global_count) + "ull + src_state)");
          }
          return widen(d, P(pops[def.source_population].states[in.index].ptr, storage_ctype(d)) + "[src_state]");
        }
        case Input::Kind::PostState: {
          DType d = tgt.states[in.index].dtype;
          return widen(d, P(pops[def.target_population].states[in.index].ptr, storage_ctype(d)) + "[tgt_state]");
        }
        case Input::Kind::SynapseState: {
          DType d = def.states[in.index].dtype;
          return widen(d, P(sd.states[in.index].ptr, storage_ctype(d)) + "[edge]");
        }
        case Input::Kind::Parameter:
          return P(sd.param_ptr.at(def.parameters[in.index].name), "const double") + "[edge]";
        case Input::Kind::Index: return in.domain == Domain::Pre ? "((double)src)" : "((double)tgt)";
        case Input::Kind::Available: {
          int nrp = in.domain == Domain::Post ? pops[def.target_population].not_refractory
                                              : pops[def.source_population].not_refractory;
          check(nrp >= 0, "not_refractory read without refractory state");
          return "(" + P(nrp, "const u8") + "[" + (in.domain == Domain::Post ? "tgt_state" : "src_state") + "] ? 1.0 : 0.0)";
        }
        default: throw Error("input kind not available in a pathway program");
      }
    };
    (void)pw;
    c.seed = u64lit(m.rng_seed);
    c.tick = "tick";
    c.time = "t";
    c.index_for_domain[int(Domain::Neuron)] = "edge";
    c.index_for_domain[int(Domain::Pre)] = "(u64)src";
    c.index_for_domain[int(Domain::Post)] = "(u64)tgt";
    c.index_for_domain[int(Domain::Edge)] = "edge";
    return c;
  }

  // synapse_only: commit only synapse-state writes (commit_synapses,
  // executor.rs:5615-5623), as per-edge update programs do
  std::string gen_pathway_body(const std::string& fname, size_t s, const PathwayDev& pw, const Program& pr,
                               bool synapse_only = false, const std::map<size_t, int>* pre_replica = nullptr) {
    const auto& def = m.synapses[s];
    const SynDev& sd = syns[s];
    std::ostringstream o;
    o << "__device__ __forceinline__ void " << fname
      << "(u32 src, u32 tgt, u64 edge, u64 tick, double t, u32& err) {\n";
    o << "  const u64 src_state = (u64)src + " << def.source_start << "ull;\n";
    o << "  const u64 tgt_state = (u64)tgt + " << target_bias(def) << "ull;\n";
    o << "  (void)src_state; (void)tgt_state; (void)t; (void)tick;\n";
    o << emit_program(pr, event_ctx(s, pw, pre_replica), "e_");
    const auto& src = m.populations[def.source_population];
    const auto& tgt = m.populations[def.target_population];
    for (const auto& [w, r] : pr.writes) {
      std::string v = reg_expr(pr, r, "e_");
      if (synapse_only && w.kind != WriteTarget::Kind::Synapse) continue;
      switch (w.kind) {
        case WriteTarget::Kind::Neuron: {
          DType d = tgt.states[w.index].dtype;
          o << "  " << P(pops[def.target_population].states[w.index].ptr, storage_ctype(d)) << "[tgt_state] = " << narrow(d, v) << ";\n";
          break;
        }
        case WriteTarget::Kind::PreNeuron: {
          DType d = src.states[w.index].dtype;
          o << "  " << P(pops[def.source_population].states[w.index].ptr, storage_ctype(d)) << "[src_state] = " << narrow(d, v) << ";\n";
          break;
        }
        case WriteTarget::Kind::Synapse: {
          DType d = def.states[w.index].dtype;
          o << "  " << P(sd.states[w.index].ptr, storage_ctype(d)) << "[edge] = " << narrow(d, v) << ";\n";
          break;
        }
        case WriteTarget::Kind::Available: break;
      }
    }
    o << "}\n";
    return o.str();
  }

  // Classify the delivery of one pathway (see PathwayDev::Mode).
  void classify_pathway(PathwayDev& pw, const Program& pr) {
    const auto& def = m.synapses[pw.synapse];
    bool only_post = true, only_syn = true;
    for (const auto& [w, r] : pr.writes) {
      only_post &= w.kind == WriteTarget::Kind::Neuron;
      only_syn &= w.kind == WriteTarget::Kind::Synapse;
    }
    if (pw.has_pending || !pw.uniform) {
      pw.mode = targets_ok(pw, pr) ? PathwayDev::Mode::Targets : PathwayDev::Mode::Serial;
      return;
    }
    if (only_post && !pr.writes.empty() && pw.is_pre) {
      // x_post = x_post + c with a plan-time constant c, optionally rounded to
      // f32 and optionally gated by the target's not_refractory flag (which
      // this pathway does not write).  Every event reaching one target then
      // applies the same map, so the result does not depend on the order in
      // which hardware atomics land and equals the sequential reference fold.
      bool ok = true;
      std::set<size_t> seen;
      std::vector<AtomicAdd> adds;
      size_t consumed = 0;
      auto producer_of = [&](size_t r) -> const Instr* {
        for (const auto& in : pr.vector)
          if (in.output == r) return &in;
        return nullptr;
      };
      for (const auto& [w, r0] : pr.writes) {
        DType d = m.populations[def.target_population].states[w.index].dtype;
        auto post_reg = pr.post_state_register(w.index);
        const Instr* in = producer_of(r0);
        if (!in || !post_reg || seen.count(w.index) || !(d == DType::F64 || d == DType::F32)) {
          ok = false;
          break;
        }
        seen.insert(w.index);
        long cond = -1;
        if (in->op == IOp::Select) {
          const Input* g = in->guard >= 0 ? pr.binding_of(size_t(in->guard)) : nullptr;
          if (!g || g->kind != Input::Kind::Available || g->domain != Domain::Post || in->right != *post_reg) {
            ok = false;
            break;
          }
          cond = in->guard;
          ++consumed;
          in = producer_of(in->left);
        }
        if (in && in->op == IOp::RoundF32 && in->guard == cond && d == DType::F32) {
          ++consumed;
          in = producer_of(in->left);
        }
        if (!in || in->guard != cond) {
          ok = false;
          break;
        }
        const RegInfo& L = pr.regs[in->left];
        const RegInfo& R = pr.regs[in->right];
        double c;
        if (in->op == IOp::Add && in->left == *post_reg && R.kind == RegKind::Const && R.finite) c = R.value;
        else if (in->op == IOp::Add && in->right == *post_reg && L.kind == RegKind::Const && L.finite) c = L.value;
        else if (in->op == IOp::Sub && in->left == *post_reg && R.kind == RegKind::Const && R.finite) c = -R.value;
        else {
          ok = false;
          break;
        }
        ++consumed;
        adds.push_back({w.index, c, cond >= 0});
      }
      // Any other lane work (reads of other state, draws) disqualifies.
      size_t lane_instrs = 0;
      for (const auto& in : pr.vector)
        if (pr.regs[in.output].kind != RegKind::Const) ++lane_instrs;
      if (ok && lane_instrs == consumed) {
        pw.mode = PathwayDev::Mode::Atomic;
        pw.atomic_adds = adds;
        return;
      }
    }
    if (only_syn && !pr.writes.empty()) {
      pw.mode = PathwayDev::Mode::EdgeParallel;
      return;
    }
    pw.mode = targets_ok(pw, pr) ? PathwayDev::Mode::Targets : PathwayDev::Mode::Serial;
  }

  // Target-ordered delivery (Mode::Targets) reproduces the sequential event
  // order per target: events reaching one target keep their canonical order
  // (emission tick, source, creation order), and events of different targets
  // touch disjoint state when the body writes only its target's neuron state
  // and its own edge's synapse state, reads presynaptic state that no event
  // writes, and draws from counter-based streams keyed by index.  The source
  // stream must come from a step kernel (which writes the fired bitmap).
  bool targets_ok(const PathwayDev& pw, const Program& pr) const {
    if (!pw.is_pre || pw.has_pending || !use_targets_) return false;
    const auto& def = m.synapses[pw.synapse];
    for (const auto& [w, r] : pr.writes)
      if (w.kind == WriteTarget::Kind::PreNeuron) return false;
    if (def.source_population == def.target_population)
      for (const auto& b : pr.bindings)
        if (b.second.kind == Input::Kind::PreState)
          for (const auto& [w, r] : pr.writes)
            if (w.kind == WriteTarget::Kind::Neuron && w.index == b.second.index) return false;
    if (syns[pw.synapse].local_edges > UINT32_MAX || def.target_count >= UINT32_MAX) return false;
    if (pw.uniform && !targets_scan_) return true;  // event buckets: any source stream
    const EventStreamDev& es = streams[size_t(pw.stream)];
    const uint64_t words = (m.populations[es.pop].count + 31) / 32;
    if (words * (es.max_delay + 1) * 4 > (uint64_t(1) << 30)) return false;
    return stream_from_threshold(size_t(pw.stream));
  }

  // True when a threshold code object (compiled into a step kernel) produces
  // the event stream and no spike generator does.
  bool stream_from_threshold(size_t sid) const {
    const EventStreamDev& es = streams[sid];
    const auto& def = m.populations[es.pop];
    size_t producers = 0;
    for (const auto& n : m.schedule) {
      if (n.owner_kind != b2ir::OwnerKind::Population || n.owner_index != es.pop) continue;
      if (n.operation == b2ir::ScheduleOp::EventSource) return false;
      if (n.operation != b2ir::ScheduleOp::CodeObject) continue;
      const auto& c = def.code_objects[n.item_index];
      if (c.kind == "threshold" && c.event_name && *c.event_name == def.events[es.event]) ++producers;
    }
    return producers == 1 && !es.exchanged;
  }

  // Device target-major view of a Targets-mode pathway's CSR.
  void build_targets_view(PathwayDev& pw) {
    const auto& def = m.synapses[pw.synapse];
    const SynDev& sd = syns[pw.synapse];
    // synapse-level targets j whose population index target_start + j this rank owns
    const PopDev& tp = pops[def.target_population];
    auto clampj = [&](uint64_t x) {
      return x <= def.target_start ? uint64_t(0) : std::min<uint64_t>(x - def.target_start, def.target_count);
    };
    pw.tm_lo = clampj(tp.lo);
    pw.tm_targets = clampj(tp.lo + tp.count) - pw.tm_lo;
    EventStreamDev& es = streams[size_t(pw.stream)];
    pw.tm_events = pw.uniform && !targets_scan_;
    es.needs_bitmap |= !pw.tm_events;
    if (pw.tm_events) {
      pw.tm_cnt = alloc(std::max<uint64_t>(pw.tm_targets, 1) * 4);
      memset_dev(pw.tm_cnt, std::max<uint64_t>(pw.tm_targets, 1) * 4);
      pw.tm_bucket = alloc(std::max<uint64_t>(sd.local_edges, 1) * 8);
      pw.tm_active = alloc(std::max<uint64_t>(pw.tm_targets, 1) * 4);
      pw.tm_nactive = alloc(16);
      memset_dev(pw.tm_nactive, 16);
    }
    pw.tm_max_deg = sd.local_edges;  // dry runs: upper bound
    if (opt.dry_run) {
      pw.tm_off = alloc(0);
      pw.tm_src = alloc(0);
      pw.tm_edge = alloc(0);
      if (!pw.uniform) pw.tm_delay = alloc(0);
      return;
    }
    DeviceBuffer off, src, edge, delay;
    build_target_major(static_cast<const uint64_t*>(dptr(pw.offsets)), static_cast<const uint32_t*>(dptr(pw.row_other)),
                       pw.row_edge >= 0 ? static_cast<const uint32_t*>(dptr(pw.row_edge)) : nullptr,
                       pw.uniform ? nullptr : static_cast<const uint16_t*>(dptr(pw.row_delay)), pw.max_delay,
                       pw.endpoint_count, sd.local_edges, pw.tm_lo, pw.tm_targets, off, src, edge, delay, stream);
    std::vector<uint64_t> toff(pw.tm_targets + 1);
    B2_CUDA(cudaMemcpy(toff.data(), off.ptr, toff.size() * 8, cudaMemcpyDeviceToHost));
    pw.tm_max_deg = 0;
    for (uint64_t j = 0; j < pw.tm_targets; ++j) pw.tm_max_deg = std::max(pw.tm_max_deg, toff[j + 1] - toff[j]);
    pw.tm_off = adopt(std::move(off));
    if (pw.tm_events) return;  // the buckets carry sources and positions
    pw.tm_src = adopt(std::move(src));
    pw.tm_edge = adopt(std::move(edge));
    if (!pw.uniform) pw.tm_delay = adopt(std::move(delay));
  }

  // Warps per target of a target-ordered kernel: 1, or (when targets are too
  // few to fill the GPU with one warp each) up to 8 warps that test disjoint
  // 32*U-entry tiles of the target's list into shared-memory hit masks, after
  // which the group's first warp delivers in order.  The masks of a block
  // (8/G targets) must fit 48 KB.
  unsigned targets_group(const PathwayDev& pw) const {
    const uint64_t tile = 32ull * targets_unroll_;
    const uint64_t tiles = (pw.tm_max_deg + tile - 1) / tile;
    unsigned g = 1;
    if (targets_warps_) g = targets_warps_;
    else
      while (g < 8 && 2ull * g <= tiles && pw.tm_targets * 2ull * g <= uint64_t(sm_count_) * 64) g *= 2;
    const uint64_t nw = targets_mask_words(pw);
    return nw * (kThreads / 32 / g) * 4 <= 48 * 1024 ? g : 1u;
  }
  uint64_t targets_mask_words(const PathwayDev& pw) const {
    const uint64_t u = targets_unroll_;
    return ((pw.tm_max_deg + 31) / 32 + u - 1) / u * u;
  }

  // Spike-list traversal shared by pathway kernels: warp per fired endpoint,
  // lanes over its CSR row.
  // Constant-addend delivery for one or more pathways that read the same spike
  // stream at the same delay and write disjoint target variables.  Work item
  // = (fired source, row chunk of row_chunk() entries); blocks stride over the
  // items, threads over the chunk, so a tick's events spread over the whole
  // GPU.  f64 updates are fire-and-forget reductions (red.global.add.f64); a
  // non-finite result is caught by the next program that reads the variable
  // (every operation of every neuron program is checked).
  // Constant-addend delivery of one row chunk [q0, q1): every thread first
  // loads its kScatterUnroll row entries (and, for gated adds, the targets'
  // not_refractory flags), then issues the reductions, so each thread keeps
  // several independent loads in flight instead of one dependent chain per
  // entry.
  std::string emit_atomic_chunk(const PathwayDev& pw, const std::string& ind) {
    const auto& def = m.synapses[pw.synapse];
    const auto& tgt = m.populations[def.target_population];
    const PopDev& tp = pops[def.target_population];
    bool gated = false;
    for (const auto& ad : pw.atomic_adds) gated |= ad.gated;
    const unsigned U = scatter_unroll_;
    std::ostringstream o;
    // target state indices in 32 bits (populations hold fewer than 2^32
    // neurons; the bias wraps like the 64-bit one)
    o << ind << "u32 tq[" << U << "];\n" << ind << "bool tv[" << U << "];\n";
    o << ind << "#pragma unroll\n" << ind << "for (u32 u = 0; u < " << U << "u; ++u) {\n";
    o << ind << "  const u64 q = q0 + threadIdx.x + u * " << kThreads << "ull;\n";
    o << ind << "  tv[u] = q < q1;\n";
    o << ind << "  tq[u] = tv[u] ? __ldg(other + q) + " << uint32_t(target_bias(def)) << "u : 0u;\n" << ind << "}\n";
    if (pw.counted) {
      // counted delivery: one event more for the target (the gate and the
      // map are applied by the target's next dense kernel)
      o << ind << "#pragma unroll\n" << ind << "for (u32 u = 0; u < " << U << "u; ++u) if (tv[u]) atomicAdd("
        << P(pw.count_ptr, "u32") << " + tq[u], " << (1u << pw.count_shift) << "u);\n";
      return o.str();
    }
    if (gated) {
      o << ind << "u8 tg[" << U << "];\n";
      o << ind << "#pragma unroll\n" << ind << "for (u32 u = 0; u < " << U << "u; ++u) tg[u] = tv[u] ? __ldcg("
        << P(tp.not_refractory, "const u8") << " + tq[u]) : (u8)0;\n";
    }
    o << ind << "#pragma unroll\n" << ind << "for (u32 u = 0; u < " << U << "u; ++u) {\n";
    o << ind << "  if (!tv[u]) continue;\n";
    for (const auto& ad : pw.atomic_adds) {
      DType d = tgt.states[ad.state].dtype;
      int ptr = tp.states[ad.state].ptr;
      std::string gate = ad.gated ? "if (tg[u]) " : "";
      if (d == DType::F64)
        o << ind << "  " << gate << "atomicAdd(" << P(ptr, "double") << " + tq[u], " << double_literal(ad.addend) << ");\n";
      else
        o << ind << "  " << gate << "{ if (!b2_atomic_add_f32_via_f64(" << P(ptr, "float") << " + tq[u], "
          << double_literal(ad.addend) << ")) err |= " << kErrNonfinite << "u; }\n";
    }
    o << ind << "}\n";
    return o.str();
  }

  // One warp delivers row entries [q0, q1) (at most 256) of a constant-addend
  // pathway: every lane loads its eight entries first, then applies them.
  std::string emit_warp_chunk(const PathwayDev& pw, const std::string& ind) {
    const auto& def = m.synapses[pw.synapse];
    const auto& tgt = m.populations[def.target_population];
    const PopDev& tp = pops[def.target_population];
    bool gated = false;
    for (const auto& ad : pw.atomic_adds) gated |= ad.gated;
    std::ostringstream o;
    const bool hints = l2_hints_ && pw.counted;
    o << ind << "u32 tq[8];\n" << ind << "bool tv[8];\n";
    if (hints) o << ind << "const u64 pol_rows = b2_policy_evict_first(), pol_cnt = b2_policy_evict_last();\n";
    o << ind << "#pragma unroll\n" << ind << "for (u32 u = 0; u < 8u; ++u) {\n";
    o << ind << "  const u64 q = q0 + lane + u * 32ull;\n";
    o << ind << "  tv[u] = q < q1;\n";
    o << ind << "  tq[u] = tv[u] ? " << (hints ? "b2_ld_rows(other + q, pol_rows)" : "__ldg(other + q)") << " + "
      << uint32_t(target_bias(def)) << "u : 0u;\n" << ind << "}\n";
    if (pw.counted) {
      if (hints)
        o << ind << "#pragma unroll\n" << ind << "for (u32 u = 0; u < 8u; ++u) if (tv[u]) b2_red_add_hint("
          << P(pw.count_ptr, "u32") << " + tq[u], " << (1u << pw.count_shift) << "u, pol_cnt);\n";
      else
        o << ind << "#pragma unroll\n" << ind << "for (u32 u = 0; u < 8u; ++u) if (tv[u]) atomicAdd("
          << P(pw.count_ptr, "u32") << " + tq[u], " << (1u << pw.count_shift) << "u);\n";
      return o.str();
    }
    if (gated) {
      o << ind << "u8 tg[8];\n";
      o << ind << "#pragma unroll\n" << ind << "for (u32 u = 0; u < 8u; ++u) tg[u] = tv[u] ? __ldcg("
        << P(tp.not_refractory, "const u8") << " + tq[u]) : (u8)0;\n";
    }
    o << ind << "#pragma unroll\n" << ind << "for (u32 u = 0; u < 8u; ++u) {\n";
    o << ind << "  if (!tv[u]) continue;\n";
    for (const auto& ad : pw.atomic_adds) {
      DType d = tgt.states[ad.state].dtype;
      int ptr = tp.states[ad.state].ptr;
      std::string gate = ad.gated ? "if (tg[u]) " : "";
      if (d == DType::F64)
        o << ind << "  " << gate << "atomicAdd(" << P(ptr, "double") << " + tq[u], " << double_literal(ad.addend) << ");\n";
      else
        o << ind << "  " << gate << "{ if (!b2_atomic_add_f32_via_f64(" << P(ptr, "float") << " + tq[u], "
          << double_literal(ad.addend) << ")) err |= " << kErrNonfinite << "u; }\n";
    }
    o << ind << "}\n";
    return o.str();
  }

  // Constant-addend scatter of one or more pathways on one spike stream:
  // work item = (fired source, 256-entry row chunk).  Items go to warps (a
  // block holds eight independent ring -> row bounds -> row -> update chains,
  // each lane loading its eight entries before applying them); with
  // B2GPU_SCATTER_WARP=0 to whole blocks, one entry per thread.
  // With layout_sid >= 0 the launch's first lb blocks lay that stream's list
  // of this tick out in the ring (emit_list_layout; for a list no kernel of
  // the tick reads, e.g. config 3's, whose deliveries come 15 ticks later)
  // while the other blocks deliver: one launch instead of two.
  std::string gen_atomic_kernel(const std::string& name, const std::vector<PathwayDev*>& pws, int layout_sid = -1,
                                unsigned lb = 0) {
    const PathwayDev& p0 = *pws.front();
    const EventStreamDev& es = streams[size_t(p0.stream)];
    const size_t endpoint_count = m.populations[p0.endpoint_pop].count;
    const bool per_warp = scatter_warp_;
    const uint64_t span = per_warp ? 256 : row_chunk();
    uint64_t chunks = 1;
    for (const PathwayDev* pw : pws) chunks = std::max<uint64_t>(chunks, (pw->max_row + span - 1) / span);
    std::ostringstream o;
    o << kernel_head(name, scatter_min_blocks_);
    if (layout_sid >= 0) {
      o << emit_list_layout(layout_sid, lb);
      o << "  else {\n";
    }
    // delivery blocks: b2_bid of b2_nblk (the blocks after the layout blocks)
    o << "  const u32 b2_bid = blockIdx.x - " << lb << "u, b2_nblk = gridDim.x - " << lb << "u;\n";
    o << "  if ((i64)rel - " << p0.delay << "ll < 0) return;\n  const u64 te = rel - " << p0.delay << "ull;\n";
    o << "  const u64* ts = " << P(es.tick_start, "const u64") << ";\n  const u64 a = ts[te], b = ts[te + 1];\n";
    o << "  const u32* ring = " << P(es.ring, "const u32") << ";\n";
    o << "  const u32 lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;\n  (void)lane; (void)warp;\n";
    for (size_t k = 0; k < pws.size(); ++k) o << "  u64 events" << k << " = 0;\n";
    o << "  const u64 items = (b - a) * " << chunks << "ull;\n";
    if (per_warp)
      o << "  for (u64 w = (u64)b2_bid * " << kThreads / 32 << "u + warp; w < items; w += (u64)b2_nblk * "
        << kThreads / 32 << "u) {\n";
    else
      o << "  for (u64 w = b2_bid; w < items; w += b2_nblk) {\n";
    o << "    const u64 j = a + w / " << chunks << "ull;\n    const u64 c = w % " << chunks << "ull;\n";
    o << "    const u32 s = __ldcg(ring + (j & " << u64lit(es.mask) << "));\n";
    for (size_t k = 0; k < pws.size(); ++k) {
      const PathwayDev& pw = *pws[k];
      const size_t lo = pw.endpoint_start, hi = pw.endpoint_start + pw.endpoint_count;
      const bool full = lo == 0 && hi == endpoint_count;
      o << "    " << (full ? "{" : "if (s >= " + std::to_string(lo) + "u && s < " + std::to_string(hi) + "u) {") << "\n";
      o << "      const u64* off = " << P(pw.offsets, "const u64") << ";\n";
      o << "      const u32* other = " << P(pw.row_other, "const u32") << ";\n";
      o << "      const u32 ep = s - " << lo << "u;\n";
      o << "      const u64 r0 = __ldg(off + ep), r1 = __ldg(off + ep + 1);\n";
      o << "      if (c == 0 && " << (per_warp ? "lane" : "threadIdx.x") << " == 0) events" << k << " += r1 - r0;\n";
      o << "      const u64 q0 = r0 + c * " << span << "ull;\n";
      o << "      const u64 q1 = q0 + " << span << "ull < r1 ? q0 + " << span << "ull : r1;\n";
      o << (per_warp ? emit_warp_chunk(pw, "      ") : emit_atomic_chunk(pw, "      "));
      o << "    }\n";
    }
    o << "  }\n";
    for (size_t k = 0; k < pws.size(); ++k)
      o << "  if (" << (per_warp ? "lane" : "threadIdx.x") << " == 0 && events" << k << ") atomicAdd((unsigned long long*)"
        << P(delivered_ptr, "u64") << " + " << pws[k]->delivered_slot << ", events" << k << ");\n";
    if (layout_sid >= 0) o << "  }\n";
    o << kernel_tail();
    return o.str();
  }

  std::string gen_pathway_kernel(const std::string& name, const std::string& body_fn, const PathwayDev& pw) {
    const EventStreamDev& es = streams[size_t(pw.stream)];
    const size_t lo = pw.endpoint_start, hi = pw.endpoint_start + pw.endpoint_count;
    const bool full = lo == 0 && hi == m.populations[pw.endpoint_pop].count;
    std::ostringstream o;
    o << kernel_head(name);
    std::string edge_of_q = pw.row_edge >= 0 ? "(u64)" + P(pw.row_edge, "const u32") + "[q]" : "q";
    if (pw.mode == PathwayDev::Mode::Serial) {
      // Canonical order: pending items first, then emission ticks oldest
      // first, sources ascending, row (creation) order (executor.rs:2326-2378).
      o << "  if (blockIdx.x != 0 || threadIdx.x != 0) return;\n";
      o << "  const u64* off = " << P(pw.offsets, "const u64") << ";\n";
      o << "  const u32* other = " << P(pw.row_other, "const u32") << ";\n";
      o << "  u64 events = 0;\n";
      std::string call_pre = pw.is_pre ? body_fn + "(ep, other[q], e, tick, t, err);" : body_fn + "(other[q], ep, e, tick, t, err);";
      auto deliver_row = [&](const std::string& filter) {
        std::ostringstream r;
        r << "      for (u64 q = off[ep]; q < off[ep + 1]; ++q) {\n";
        if (!filter.empty()) r << "        if (!(" << filter << ")) continue;\n";
        r << "        const u64 e = " << edge_of_q << ";\n        " << call_pre << "\n        ++events;\n      }\n";
        return r.str();
      };
      if (pw.has_pending) {
        // Pending items were queued before any runtime push, so they come first
        // in their slot; with a uniform delay an item is an endpoint index,
        // otherwise one edge (local index, with its source and target).
        o << "  { const u64* po = " << P(pw.pend_offsets, "const u64") << "; const u32* pi = " << P(pw.pend_items, "const u32") << ";\n";
        o << "    for (u64 x = po[rel]; x < po[rel + 1]; ++x) {\n";
        if (pw.uniform) {
          o << "      const u32 ep = pi[x];\n" << deliver_row("");
        } else {
          o << "      " << body_fn << "(" << P(pw.pend_src, "const u32") << "[x], " << P(pw.pend_tgt, "const u32")
            << "[x], (u64)pi[x], tick, t, err);\n      ++events;\n";
        }
        o << "    }\n  }\n";
      }
      o << "  const u64* ts = " << P(es.tick_start, "const u64") << ";\n";
      o << "  const u32* ring = " << P(es.ring, "const u32") << ";\n";
      if (pw.uniform) {
        o << "  if ((i64)rel - " << pw.delay << "ll >= 0) {\n    const u64 te = rel - " << pw.delay << "ull;\n";
        o << "    for (u64 j = ts[te]; j < ts[te + 1]; ++j) {\n      const u32 s = ring[j & " << u64lit(es.mask) << "];\n";
        if (!full) o << "      if (s < " << lo << "u || s >= " << hi << "u) continue;\n";
        o << "      const u32 ep = s - " << lo << "u;\n" << deliver_row("") << "    }\n  }\n";
      } else {
        o << "  const u16* dl = " << P(pw.row_delay, "const u16") << ";\n";
        o << "  for (i64 te = (i64)rel - " << pw.max_delay << "ll; te <= (i64)rel; ++te) {\n    if (te < 0) continue;\n";
        o << "    const u64 lag = rel - (u64)te;\n";
        o << "    for (u64 j = ts[te]; j < ts[te + 1]; ++j) {\n      const u32 s = ring[j & " << u64lit(es.mask) << "];\n";
        if (!full) o << "      if (s < " << lo << "u || s >= " << hi << "u) continue;\n";
        o << "      const u32 ep = s - " << lo << "u;\n" << deliver_row("dl[q] == lag") << "    }\n  }\n";
      }
      o << "  if (events) atomicAdd((unsigned long long*)" << P(delivered_ptr, "u64") << " + " << pw.delivered_slot << ", events);\n";
      o << kernel_tail();
      return o.str();
    }
    if (pw.mode == PathwayDev::Mode::Targets && pw.tm_events) {
      // Bucket scatter: work items (fired source, row chunk) as in the
      // edge-parallel kernel; each event takes the next slot of its target's
      // bucket, and the first event of a target lists the target.  The
      // delivery kernel of the same tick consumes list rel & 1; this kernel
      // clears the other list's count, which the previous tick consumed.
      const uint64_t chunks = std::max<uint64_t>(1, (pw.max_row + row_chunk() - 1) / row_chunk());
      o << "  if ((i64)rel - " << pw.delay << "ll < 0) return;\n  const u64 te = rel - " << pw.delay << "ull;\n";
      o << "  u32* nact = " << P(pw.tm_nactive, "u32") << ";\n";
      o << "  if (blockIdx.x == 0 && threadIdx.x == 0) nact[(rel + 1ull) & 1ull] = 0u;\n";
      o << "  u32* cnt = " << P(pw.tm_cnt, "u32") << ";\n  u64* bucket = " << P(pw.tm_bucket, "u64") << ";\n";
      o << "  u32* active = " << P(pw.tm_active, "u32") << ";\n  const u64* toff = " << P(pw.tm_off, "const u64") << ";\n";
      o << "  const u64* ts = " << P(es.tick_start, "const u64") << ";\n  const u64 a = ts[te], b = ts[te + 1];\n";
      o << "  const u32* ring = " << P(es.ring, "const u32") << ";\n";
      o << "  const u64* off = " << P(pw.offsets, "const u64") << ";\n  const u32* other = " << P(pw.row_other, "const u32") << ";\n";
      o << "  u64 events = 0;\n";
      o << "  const u64 items = (b - a) * " << chunks << "ull;\n";
      o << "  for (u64 w = blockIdx.x; w < items; w += gridDim.x) {\n";
      o << "    const u64 j = a + w / " << chunks << "ull;\n    const u64 c = w % " << chunks << "ull;\n";
      o << "    const u32 s = __ldcg(ring + (j & " << u64lit(es.mask) << "));\n";
      if (!full) o << "    if (s < " << lo << "u || s >= " << hi << "u) continue;\n";
      o << "    const u32 ep = s - " << lo << "u;\n    const u64 r0 = __ldg(off + ep), r1 = __ldg(off + ep + 1);\n";
      o << "    if (c == 0 && threadIdx.x == 0) events += r1 - r0;\n";
      o << "    const u64 q0 = r0 + c * " << row_chunk() << "ull;\n    if (q0 >= r1) continue;\n";
      o << "    const u64 q1 = q0 + " << row_chunk() << "ull < r1 ? q0 + " << row_chunk() << "ull : r1;\n";
      o << "    for (u64 q = q0 + threadIdx.x; q < q1; q += " << kThreads << "ull) {\n";
      o << "      const u32 tj = __ldg(other + q) - " << pw.tm_lo << "u;\n";
      o << "      const u32 slot = atomicAdd(cnt + tj, 1u);\n";
      o << "      bucket[__ldg(toff + tj) + slot] = ((u64)ep << 32) | q;\n";
      o << "      if (slot == 0u) active[atomicAdd(nact + (rel & 1ull), 1u)] = tj;\n";
      o << "    }\n  }\n";
      o << "  if (threadIdx.x == 0 && events) atomicAdd((unsigned long long*)" << P(delivered_ptr, "u64") << " + "
        << pw.delivered_slot << ", events);\n";
      o << kernel_tail();
      return o.str();
    }
    if (pw.mode == PathwayDev::Mode::Targets) {
      // Warp per target over its in-edges (delay descending, source
      // ascending, creation order, i.e. the canonical delivery order): lanes
      // test 32 entries at a time against the emission tick's fired bitmap,
      // and the hits run one lane at a time in lane order, separated by
      // __syncwarp (which orders the lanes' memory accesses).
      const unsigned U = targets_unroll_;  // independent 32-entry groups in flight per warp
      const std::string bm = P(es.bitmap, "const u32");
      o << "  const u32 lane = threadIdx.x & 31u;\n";
      o << "  const u64 warps = (u64)gridDim.x * (blockDim.x >> 5);\n";
      o << "  const u64* toff = " << P(pw.tm_off, "const u64") << ";\n";
      o << "  const u32* tsrc = " << P(pw.tm_src, "const u32") << ";\n";
      o << "  const u32* tedge = " << P(pw.tm_edge, "const u32") << ";\n";
      // With one delay the emission tick's bitmap slot is staged in shared
      // memory once per block, so each entry's test is one global load (its
      // source id) and one shared-memory lookup.
      const uint64_t mask_bytes = pw.tm_warps > 1 ? targets_mask_words(pw) * (kThreads / 32 / pw.tm_warps) * 4 : 0;
      const bool smem_bm = pw.uniform && es.bm_words * 4 + mask_bytes <= 48 * 1024 && targets_smem_bitmap_;
      if (pw.uniform) {
        o << "  if ((i64)rel - " << pw.delay << "ll < 0) return;\n";
        o << "  const u32* bmw = " << bm << " + ((rel - " << pw.delay << "ull) % " << es.bm_slots << "ull) * "
          << es.bm_words << "ull;\n";
        if (smem_bm) {
          o << "  __shared__ u32 s_bm[" << es.bm_words << "];\n";
          o << "  for (u32 w = threadIdx.x; w < " << es.bm_words << "u; w += blockDim.x) s_bm[w] = __ldcg(bmw + w);\n";
          o << "  __syncthreads();\n";
        }
      } else {
        o << "  const u16* tdel = " << P(pw.tm_delay, "const u16") << ";\n";
      }
      o << "  u64 events = 0;\n";
      // hit test of the U 32-entry groups at `tb` (u64, local names q/s/h)
      auto hit_test = [&](const std::string& tb, const std::string& end) {
        std::ostringstream h;
        h << "      u32 sv[" << U << "], mk[" << U << "];\n      bool in[" << U << "];\n";
        h << "#pragma unroll\n      for (u32 u = 0; u < " << U << "u; ++u) {\n";
        h << "        const u64 q = " << tb << " + u * 32u + lane;\n        in[u] = q < " << end << ";\n";
        h << "        sv[u] = in[u] ? __ldg(tsrc + q) : 0u;\n      }\n";
        h << "#pragma unroll\n      for (u32 u = 0; u < " << U << "u; ++u) {\n";
        h << "        bool h = false;\n";
        h << "        if (in[u]) {\n          const u32 s = sv[u] + " << pw.endpoint_start << "u;\n";
        if (pw.uniform) {
          h << "          h = (" << (smem_bm ? "s_bm[s >> 5]" : "__ldcg(bmw + (s >> 5))") << " >> (s & 31u)) & 1u;\n";
        } else {
          h << "          const u64 lag = __ldg(tdel + " << tb << " + u * 32u + lane);\n";
          h << "          if (lag <= rel) h = (__ldcg(" << bm << " + ((rel - lag) % " << es.bm_slots << "ull) * "
            << es.bm_words << "ull + (s >> 5)) >> (s & 31u)) & 1u;\n";
        }
        h << "        }\n        mk[u] = __ballot_sync(0xffffffffu, h);\n      }\n";
        return h.str();
      };
      if (pw.tm_warps > 1) {
        // G warps per target: warp g of the group tests tiles g, g+G, ... of
        // 32*U entries into the target's shared hit masks; after the block
        // barrier the group's first warp walks the masks in entry order.
        const unsigned G = pw.tm_warps, TPB = kThreads / 32 / G;
        const uint64_t NW = targets_mask_words(pw);
        o << "  __shared__ u32 s_mask[" << TPB * NW << "];\n";
        o << "  const u32 warp = threadIdx.x >> 5, slot = warp / " << G << "u, gw = warp % " << G << "u;\n";
        o << "  u32* msk = s_mask + slot * " << NW << "u;\n";
        o << "  for (u64 t0 = (u64)blockIdx.x * " << TPB << "u; t0 < " << pw.tm_targets << "ull; t0 += (u64)gridDim.x * "
          << TPB << "u) {\n";
        o << "    const u64 j = t0 + slot;\n    const bool live = j < " << pw.tm_targets << "ull;\n";
        o << "    const u64 o0 = live ? __ldg(toff + j) : 0ull, o1 = live ? __ldg(toff + j + 1) : 0ull;\n";
        o << "    for (u64 tb = o0 + (u64)gw * " << 32 * U << "u; tb < o1; tb += " << uint64_t(G) * 32 * U << "ull) {\n";
        o << hit_test("tb", "o1");
        o << "      const u32 w0 = (u32)((tb - o0) >> 5);\n";
        o << "#pragma unroll\n      for (u32 u = 0; u < " << U << "u; ++u) if (lane == u) msk[w0 + u] = mk[u];\n";
        o << "    }\n    __syncthreads();\n";
        o << "    if (gw == 0 && live) {\n";
        o << "      const u32 nw = (u32)((o1 - o0 + 31u) >> 5);\n";
        o << "      for (u32 w0 = 0; w0 < nw; w0 += 32u) {\n";
        o << "        const u32 m = w0 + lane < nw ? msk[w0 + lane] : 0u;\n";
        o << "        events += __popc(m);\n";
        o << "        u32 any = __ballot_sync(0xffffffffu, m != 0u);\n";
        o << "        while (any) {\n          const u32 L = __ffs(any) - 1u;\n          any &= any - 1u;\n";
        o << "          u32 mm = __shfl_sync(0xffffffffu, m, L);\n";
        o << "          while (mm) {\n            const u32 b = __ffs(mm) - 1u;\n            mm &= mm - 1u;\n";
        o << "            if (lane == b) {\n              const u64 q = o0 + (u64)(w0 + L) * 32u + b;\n";
        o << "              " << body_fn << "(__ldg(tsrc + q), (u32)(j + " << pw.tm_lo
          << "ull), (u64)__ldg(tedge + q), tick, t, err);\n            }\n";
        o << "            __syncwarp();\n          }\n        }\n      }\n    }\n";
        o << "    __syncthreads();\n  }\n";
        o << "  if (events) atomicAdd((unsigned long long*)" << P(delivered_ptr, "u64") << " + " << pw.delivered_slot
          << ", events);\n";
        o << kernel_tail();
        return o.str();
      }
      o << "  for (u64 j = (blockIdx.x * (u64)blockDim.x + threadIdx.x) >> 5; j < " << pw.tm_targets << "ull; j += warps) {\n";
      o << "    const u64 o0 = __ldg(toff + j), o1 = __ldg(toff + j + 1);\n";
      o << "    for (u64 base = o0; base < o1; base += " << 32 * U << "ull) {\n";
      o << hit_test("base", "o1");
      o << "#pragma unroll\n      for (u32 u = 0; u < " << U << "u; ++u) {\n";
      o << "        u32 mm = mk[u];\n        events += lane == 0 ? __popc(mm) : 0u;\n";
      o << "        while (mm) {\n          const u32 b = __ffs(mm) - 1u;\n          mm &= mm - 1u;\n";
      o << "          if (lane == b) " << body_fn << "(sv[u], (u32)(j + " << pw.tm_lo
        << "ull), (u64)__ldg(tedge + base + u * 32u + lane), tick, t, err);\n";
      o << "          __syncwarp();\n        }\n      }\n    }\n  }\n";
      o << "  if (lane == 0 && events) atomicAdd((unsigned long long*)" << P(delivered_ptr, "u64") << " + "
        << pw.delivered_slot << ", events);\n";
      o << kernel_tail();
      return o.str();
    }
    // Edge-parallel traversal (bodies that write only synapse state, so
    // events commute).  Work item = (fired endpoint, row chunk of row_chunk()
    // entries); blocks stride over items, threads over the chunk, so a tick's
    // events spread across the whole GPU instead of one warp per spike.
    // (Constant-addend pathways use gen_atomic_kernel.)
    check(pw.mode == PathwayDev::Mode::EdgeParallel, "pathway kernel mode mismatch");
    const uint64_t chunks = std::max<uint64_t>(1, (pw.max_row + row_chunk() - 1) / row_chunk());
    o << "  if ((i64)rel - " << pw.delay << "ll < 0) return;\n  const u64 te = rel - " << pw.delay << "ull;\n";
    o << "  const u64* ts = " << P(es.tick_start, "const u64") << ";\n  const u64 a = ts[te], b = ts[te + 1];\n";
    o << "  const u32* ring = " << P(es.ring, "const u32") << ";\n";
    o << "  const u64* off = " << P(pw.offsets, "const u64") << ";\n  const u32* other = " << P(pw.row_other, "const u32") << ";\n";
    o << "  u64 events = 0;\n";
    o << "  const u64 items = (b - a) * " << chunks << "ull;\n";
    o << "  for (u64 w = blockIdx.x; w < items; w += gridDim.x) {\n";
    o << "    const u64 j = a + w / " << chunks << "ull;\n    const u64 c = w % " << chunks << "ull;\n";
    o << "    const u32 s = ring[j & " << u64lit(es.mask) << "];\n";
    if (!full) o << "    if (s < " << lo << "u || s >= " << hi << "u) continue;\n";
    o << "    const u32 ep = s - " << lo << "u;\n    const u64 r0 = off[ep], r1 = off[ep + 1];\n";
    o << "    if (c == 0 && threadIdx.x == 0) events += r1 - r0;\n";
    o << "    const u64 q0 = r0 + c * " << row_chunk() << "ull;\n    if (q0 >= r1) continue;\n";
    o << "    const u64 q1 = q0 + " << row_chunk() << "ull < r1 ? q0 + " << row_chunk() << "ull : r1;\n";
    o << "#pragma unroll 4\n    for (u64 q = q0 + threadIdx.x; q < q1; q += " << kThreads << "ull) {\n";
    o << "      const u64 e = " << edge_of_q << ";\n";
    if (pw.is_pre) o << "      " << body_fn << "(ep, other[q], e, tick, t, err);\n";
    else o << "      " << body_fn << "(other[q], ep, e, tick, t, err);\n";
    o << "    }\n  }\n";
    o << "  if (threadIdx.x == 0 && events) atomicAdd((unsigned long long*)" << P(delivered_ptr, "u64") << " + "
      << pw.delivered_slot << ", events);\n";
    o << kernel_tail();
    return o.str();
  }

  // Bucket delivery of a single-delay target-ordered pathway: one thread per
  // listed target sorts its bucket (keys source << 32 | row position, i.e.
  // the canonical order: source ascending, then creation order) and runs the
  // bodies in that order, then clears the target's count.
  //
  // One warp per listed target (interleaved across blocks so a tick's few
  // thousand targets spread over every SM).  Up to 32 events: lane k holds
  // key k, its rank among the keys comes from 32 shuffles, every lane
  // prefetches its event's state into L1 at once, and the bodies then run one
  // lane at a time in rank order (separated by __syncwarp), so the chain of
  // dependent accesses per target is paid once rather than per event.  More
  // events: lane 0 sorts the bucket in place and runs them in order.
  std::string gen_targets_deliver(const std::string& name, const std::string& body_fn, const std::string& prefetch_fn,
                                  const PathwayDev& pw) {
    std::ostringstream o;
    o << kernel_head(name);
    o << "  if ((i64)rel - " << pw.delay << "ll < 0) return;\n";
    o << "  const u32 n = " << P(pw.tm_nactive, "const u32") << "[rel & 1ull];\n";
    o << "  u32* cnt = " << P(pw.tm_cnt, "u32") << ";\n  u64* bucket = " << P(pw.tm_bucket, "u64") << ";\n";
    o << "  const u32* active = " << P(pw.tm_active, "const u32") << ";\n  const u64* toff = " << P(pw.tm_off, "const u64")
      << ";\n";
    if (pw.row_edge >= 0) o << "  const u32* red = " << P(pw.row_edge, "const u32") << ";\n";
    const std::string edge = pw.row_edge >= 0 ? "(u64)red[(u32)key]" : "(u64)(u32)key";
    o << "  const u32 lane = threadIdx.x & 31u;\n";
    o << "  for (u32 x = (threadIdx.x >> 5) * gridDim.x + blockIdx.x; x < n; x += gridDim.x * (blockDim.x >> 5)) {\n";
    o << "    const u32 tj = active[x];\n    const u32 c = cnt[tj];\n    u64* bk = bucket + toff[tj];\n";
    o << "    const u32 tgt = tj + " << pw.tm_lo << "u;\n";
    o << "    if (c <= 32u) {\n";
    o << "      const u64 key = lane < c ? bk[lane] : ~0ull;\n";
    o << "      u32 rank = 0;\n";
    o << "      for (u32 L = 0; L < c; ++L) rank += __shfl_sync(0xffffffffu, key, L) < key ? 1u : 0u;\n";
    o << "      u64 e = 0;\n";
    o << "      if (lane < c) {\n        e = " << edge << ";\n        " << prefetch_fn << "((u32)(key >> 32), tgt, e);\n      }\n";
    o << "      for (u32 r = 0; r < c; ++r) {\n";
    o << "        if (lane < c && rank == r) " << body_fn << "((u32)(key >> 32), tgt, e, tick, t, err);\n";
    o << "        __syncwarp();\n      }\n";
    o << "    } else if (lane == 0u) {\n";
    o << "      b2_sort_u64(bk, c);\n";
    o << "      for (u32 k = 0; k < c; ++k) {\n        const u64 key = bk[k];\n";
    o << "        " << body_fn << "((u32)(key >> 32), tgt, " << edge << ", tick, t, err);\n      }\n";
    o << "    }\n";
    o << "    __syncwarp();\n    if (lane == 0u) cnt[tj] = 0u;\n  }\n";
    o << kernel_tail();
    return o.str();
  }

  // L1 prefetch of every state and per-edge parameter element a pathway body
  // reads (same addresses as the body's loads).
  std::string gen_pathway_prefetch(const std::string& fname, size_t s, const Program& pr,
                                   const std::map<size_t, int>* pre_replica = nullptr) {
    const auto& def = m.synapses[s];
    const SynDev& sd = syns[s];
    const auto& src = m.populations[def.source_population];
    const auto& tgt = m.populations[def.target_population];
    std::ostringstream o;
    o << "__device__ __forceinline__ void " << fname << "(u32 src, u32 tgt, u64 edge) {\n";
    o << "  const u64 src_state = (u64)src + " << def.source_start << "ull;\n";
    o << "  const u64 tgt_state = (u64)tgt + " << target_bias(def) << "ull;\n";
    o << "  (void)src_state; (void)tgt_state; (void)edge;\n";
    std::set<std::string> seen;
    for (const auto& [slot, in] : pr.bindings) {
      std::string addr;
      if (in.kind == Input::Kind::PreState && pre_replica && pre_replica->count(in.index))
        continue;  // read from this tick's replica, not the rank's own block
      if (in.kind == Input::Kind::PreState)
        addr = P(pops[def.source_population].states[in.index].ptr, storage_ctype(src.states[in.index].dtype)) + " + src_state";
      else if (in.kind == Input::Kind::PostState)
        addr = P(pops[def.target_population].states[in.index].ptr, storage_ctype(tgt.states[in.index].dtype)) + " + tgt_state";
      else if (in.kind == Input::Kind::SynapseState)
        addr = P(sd.states[in.index].ptr, storage_ctype(def.states[in.index].dtype)) + " + edge";
      else if (in.kind == Input::Kind::Parameter && sd.param_ptr.count(def.parameters[in.index].name))
        addr = P(sd.param_ptr.at(def.parameters[in.index].name), "const double") + " + edge";
      else
        continue;
      if (seen.insert(addr).second) o << "  b2_prefetch(" << addr << ");\n";
    }
    o << "}\n";
    return o.str();
  }

  // ================================================================ plan
  NodeEffects effects_of(const b2ir::ScheduleNode& node) {
    NodeEffects e;
    e.reads.insert(node.effects.reads.begin(), node.effects.reads.end());
    e.writes.insert(node.effects.writes.begin(), node.effects.writes.end());
    if (node.operation == b2ir::ScheduleOp::CodeObject && node.owner_kind == b2ir::OwnerKind::Population) {
      const auto& def = m.populations[node.owner_index];
      const auto& code = def.code_objects[node.item_index];
      if (def.refractory) {
        std::string ls = "population/" + std::to_string(node.owner_index) + "/refractory/lastspike";
        std::string nr = "population/" + std::to_string(node.owner_index) + "/refractory/not_refractory";
        if (code.kind == "threshold" && code.event_name && *code.event_name == "spike") {
          e.reads.insert(nr);
          e.writes.insert(ls);
          e.writes.insert(nr);
        } else if (code.kind == "state_update" && def.refractory->mode == "fixed") {
          e.reads.insert(ls);
          e.writes.insert(nr);
        }
      }
    }
    return e;
  }

  std::vector<Program> programs;  // owned programs (stable addresses via reserve)
  std::map<std::string, std::string> const_tables;  // file-scope tables referenced by emitted code
  std::map<const double*, int> device_tables;       // uploaded TimedArray tables by source array
  std::string device_table(const std::vector<double>& v) {
    auto it = device_tables.find(v.data());
    if (it == device_tables.end())
      it = device_tables.emplace(v.data(), upload(v.data(), std::max<size_t>(v.size(), 1) * 8)).first;
    return P(it->second, "const double");
  }

  // A kernel in the tick, generated once the whole schedule is analysed.
  struct StepSpec {
    size_t pop = 0;
    const Program* U = nullptr;
    const Program* X = nullptr;
    size_t x_event = 0;
    bool x_spike = false;
    const Program* R = nullptr;
    std::vector<const Program*> deferred;  // previous tick's trailing neuron maps
    std::vector<PathwayDev*> applies;      // counted pathways of this tick, applied first, in order
    const Program* post_R = nullptr;       // spike reset of this tick, on lanes whose lastspike is t
    // the previous tick's trailing dense kernel, run in this kernel's
    // prologue: its counted applies, then its program (in `deferred`), then
    // its reset on lanes whose lastspike is the previous tick's t
    std::vector<PathwayDev*> deferred_applies;
    const Program* deferred_post_R = nullptr;
    size_t node_pos = 0;
  };
  struct PathSpec {
    std::vector<PathwayDev*> pathways;
    std::vector<const Program*> programs;
    std::vector<std::string> codes;
    std::string body;  // device function of a single non-atomic pathway
    std::map<size_t, int> pre_replica;  // presynaptic state -> replica read (multi-GPU)
  };
  struct OpSpec {
    enum class Kind { Text, Step, Path } kind = Kind::Text;
    std::string base, text;
    size_t index = 0;
    unsigned grid = 1, block = kThreads;
    int fuse_path = -1;  // exchange: PathSpec delivered inside the same kernel
    std::vector<size_t> fused_steps;  // Step: further StepSpecs stepped by the same launch
    size_t item = 0;                  // evmon: EventMonitor index within its population
    int reads = -1;                   // Text ops: the event stream whose lists they read
    unsigned lb = 1;                  // list consumers: blocks that lay the list out in the ring
    int layout_sid = -1;              // Path: a stream whose tick list its first lb blocks lay out
  };
  // Deferred work of a population's last tick that a flush kernel applies at
  // the end of a run or before a state read.
  struct Flush {
    size_t pop = 0;
    const Program* program = nullptr;
    std::vector<PathwayDev*> applies;
    const Program* post_R = nullptr;
  };
  std::vector<Flush> flushes;
  std::vector<SummedSpec> summed_specs;
  struct SynProgSpec {
    size_t synapse = 0;
    const Program* program = nullptr;
    std::map<size_t, int> pre_replica;  // presynaptic state -> replica read (multi-GPU)
  };
  std::vector<SynProgSpec> synprog_specs;
  std::vector<Op> flush_ops;
  int deferred_flags = -1;                                  // per-population u64 tick of the last flush
  // Multi-GPU: the presynaptic states a synaptic program reads from a
  // partitioned source population get a replica each, refreshed by a
  // replicate kernel and a wait kernel placed right before the reader (the
  // value is the current one: every earlier writer of the tick is already in
  // `specs`).  Presynaptic refractoriness is not replicated.
  std::map<size_t, int> replicate_pre_state(const Program& pr, size_t s, std::vector<OpSpec>& specs_out,
                                            const std::string& code_name) {
    std::map<size_t, int> out;
    if (world == 1) return out;
    const size_t sp = m.synapses[s].source_population;
    for (const auto& b : pr.bindings) {
      check(pops[sp].replicated || !(b.second.kind == Input::Kind::Available && b.second.domain == Domain::Pre),
            "multi-GPU runs cannot read presynaptic refractoriness across GPUs ('" + code_name + "')");
      if (b.second.kind != Input::Kind::PreState || pops[sp].replicated || out.count(b.second.index)) continue;
      const int r = new_replica(sp, b.second.index);
      out[b.second.index] = r;
      const std::string var = sanitize(m.populations[sp].name + "_" + m.populations[sp].states[b.second.index].name);
      OpSpec rep;
      rep.base = var + "_replicate";
      rep.text = "replicate";
      rep.index = size_t(r);
      rep.grid = kReplicaBlocks;
      specs_out.push_back(rep);
      OpSpec w;
      w.base = var + "_replica_wait";
      w.text = "replica_wait";
      w.index = size_t(r);
      w.grid = 1;
      specs_out.push_back(w);
    }
    return out;
  }

  // Copy this rank's block of the replicated state into every rank's replica
  // half of this tick (plain peer stores over NVLink), then, per block, a
  // system-scope fence and one tagged flag per rank.
  std::string gen_replicate(const std::string& name, const Replica& r) {
    const PopDev& pd = pops[r.pop];
    const char* ct = storage_ctype(m.populations[r.pop].states[r.state].dtype);
    std::ostringstream o;
    o << kernel_head(name);
    o << "  const u64 half = (rel & 1ull) * " << pd.global_count << "ull;\n";
    o << "  const " << ct << "* mine = " << P(pd.states[r.state].ptr, (std::string("const ") + ct).c_str()) << ";\n";
    o << "  for (u64 i = blockIdx.x * (u64)blockDim.x + threadIdx.x; i < " << pd.count
      << "ull; i += (u64)gridDim.x * blockDim.x) {\n";
    o << "    const " << ct << " v = mine[i];\n";
    o << "    for (u32 q = 0; q < " << world << "u; ++q) ((" << ct << "*)g_ptr[" << r.rptr[0] << " + q])[half + "
      << pd.lo << "ull + i] = v;\n  }\n";
    o << "  __threadfence_system();\n  __syncthreads();\n";
    o << "  if (threadIdx.x < " << world << "u) b2_ll_store(((u64*)g_ptr[" << r.fptr[0] << " + threadIdx.x]) + (rel & 1ull) * "
      << world * kReplicaBlocks << "ull + " << rank * int(kReplicaBlocks) << "ull + blockIdx.x, 1u, (u32)(rel + 1ull));\n";
    o << kernel_tail();
    return o.str();
  }

  // Wait (bounded) for every rank's replicate flags of this tick; the fence
  // after them orders the peers' stores before the readers that follow.
  std::string gen_replica_wait(const std::string& name, const Replica& r) {
    const uint64_t timeout_ns = uint64_t(opt.exchange_timeout_ms) * 1000000ull;
    std::ostringstream o;
    o << kernel_head(name);
    o << "  const bool poisoned = *(volatile const u32*)&ctl->error != 0u;\n";
    o << "  if (threadIdx.x < " << world * kReplicaBlocks << "u && !poisoned) b2_ll_wait(((const u64*)g_ptr["
      << r.fptr[size_t(rank)] << "]) + (rel & 1ull) * " << world * kReplicaBlocks << "ull + threadIdx.x, (u32)(rel + 1ull), "
      << timeout_ns << "ull, err);\n";
    o << "  __syncthreads();\n  __threadfence_system();\n";
    o << kernel_tail();
    return o.str();
  }

  // The chunk kernel (B2GPU_MEGA): every op of the tick becomes a device
  // function of a virtual block index, its kernel text with the block index
  // and grid size replaced, no programmatic-launch instructions, and loads
  // through L2 (ld.global.cg) instead of the read-only path, since data that
  // other blocks wrote earlier in the same launch is not read-only.  The
  // kernel runs ticks k0 .. k0+n-1; per tick and op its blocks take the op's
  // virtual blocks in turn, then meet at a grid barrier, which orders the ops
  // as the launch boundaries of the per-op kernels do.  Ops that are not a
  // single 256-thread kernel (fused multi-population steps) disable it.
  static void replace_all(std::string& t, const std::string& a, const std::string& b) {
    for (size_t at = t.find(a); at != std::string::npos; at = t.find(a, at + b.size())) t.replace(at, a.size(), b);
  }
  // A kernel's `return` ends the thread; in a device function it only ends
  // the op for that virtual block, and the thread goes on to the next one.
  // That is the same unless some threads of a block return while others go
  // on to a block or warp barrier (bar.sync, a *_sync intrinsic) of the same
  // op, which in the chunk kernel they would meet at a different place.  An
  // op qualifies if its only returns are the block-uniform tick guards, or it
  // has no barrier at all.
  static bool divergent_return_before_barrier(const std::string& t) {
    bool divergent = false;
    std::istringstream in(t);
    for (std::string line; std::getline(in, line);) {
      if (line.find("return;") == std::string::npos) continue;
      const bool uniform = line.rfind("  if ((i64)rel - ", 0) == 0 || line.rfind("  if (rel < ", 0) == 0 ||
                           line.rfind("  if (tick < ", 0) == 0;
      divergent |= !uniform;
    }
    if (!divergent) return false;
    for (const char* b : {"__syncthreads", "_sync(", "b2_block_exclusive_scan", "b2_finalize_spikes", "b2_tile_offsets"})
      if (t.find(b) != std::string::npos) return true;
    return false;
  }
  std::string gen_chunk_kernel(const std::vector<std::string>& texts) {
    for (size_t i = 0; i < ops.size(); ++i) {
      size_t globals = 0;
      for (size_t at = texts[i].find("__global__"); at != std::string::npos; at = texts[i].find("__global__", at + 1))
        ++globals;
      if (globals != 1 || ops[i].block != kThreads || texts[i].find("__device__") != std::string::npos ||
          divergent_return_before_barrier(texts[i])) {
        mega_ = false;
        return "";
      }
    }
    std::ostringstream o;
    for (size_t i = 0; i < ops.size(); ++i) {
      std::string t = texts[i];
      const size_t h = t.find("extern \"C\" __global__ void");
      const size_t brace = t.find('{', h);
      t.replace(h, brace - h,
                "__device__ __forceinline__ void " + ops[i].name + "_m(RunCtl* __restrict__ ctl, u32 k, u32 b2_vb, u32 b2_vgrid) ");
      replace_all(t, "asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");", "");
      replace_all(t, "asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");", "");
      replace_all(t, "blockIdx.x", "b2_vb");
      replace_all(t, "gridDim.x", "b2_vgrid");
      replace_all(t, "__ldg(", "__ldcg(");
      o << t;
    }
    const uint64_t timeout_ns = uint64_t(opt.exchange_timeout_ms) * 1000000ull;
    o << "extern \"C\" __global__ void __launch_bounds__(" << kThreads << ", " << std::max(1u, min_blocks_)
      << ") b2_chunk(RunCtl* __restrict__ ctl, u32 k0, u32 n, u32* __restrict__ bar) {\n";
    o << "  u32 target = 0;\n";
    o << "  for (u32 k = k0; k < k0 + n; ++k) {\n";
    for (size_t i = 0; i < ops.size(); ++i) {
      // a block barrier between virtual blocks: an op's shared arrays are
      // reused by the block's next virtual block
      o << "    for (u32 vb = blockIdx.x; vb < " << ops[i].grid << "u; vb += gridDim.x) { " << ops[i].name
        << "_m(ctl, k, vb, " << ops[i].grid << "u); __syncthreads(); }\n";
      o << "    target += gridDim.x;\n    b2_grid_barrier(bar, target, ctl, " << timeout_ns << "ull);\n";
    }
    o << "  }\n}\n";
    return o.str();
  }

  bool deferred_pending = false;

  void build_plan() {
    const auto& nodes = m.schedule;
    check(!nodes.empty(), "model has no schedule");
    std::vector<NodeEffects> eff;
    for (const auto& n : nodes) eff.push_back(effects_of(n));
    programs.reserve(nodes.size() * 2 + 8);
    std::vector<bool> done(nodes.size(), false);
    std::vector<OpSpec> specs;
    std::vector<StepSpec> steps_;
    std::vector<PathSpec> paths;
    std::map<size_t, size_t> step_of_pop;  // population -> StepSpec index (state-update step)
    auto code_of = [&](const b2ir::ScheduleNode& n) -> const b2ir::CodeObject& {
      return n.owner_kind == b2ir::OwnerKind::Population ? m.populations[n.owner_index].code_objects[n.item_index]
                                                         : m.synapses[n.owner_index].code_objects[n.item_index];
    };
    auto compile_pop = [&](size_t p, const b2ir::CodeObject& c) -> const Program* {
      std::map<std::string, WriteTarget> writable;
      auto inputs = population_inputs(p, writable);
      programs.push_back(Program::compile(c, inputs, writable, m.functions));
      return &programs.back();
    };
    // Can the node at `from` move up to just after `to`, past every node in
    // between that is not already folded into an earlier kernel?
    auto can_hoist = [&](size_t to, size_t from) {
      for (size_t y = to + 1; y < from; ++y)
        if (!done[y] && conflicts(eff[from], eff[y])) return false;
      return true;
    };
    std::vector<bool> stream_produced(streams.size(), false);
    for (size_t idx = 0; idx < nodes.size(); ++idx) {
      if (done[idx]) continue;
      const auto& node = nodes[idx];
      done[idx] = true;
      if (node.owner_kind == b2ir::OwnerKind::Population) {
        size_t p = node.owner_index;
        const auto& def = m.populations[p];
        switch (node.operation) {
          case b2ir::ScheduleOp::StateMonitor: {
            if (pops[p].mon_records < 0) break;
            OpSpec o;
            o.base = def.name + "_statemon";
            size_t n = pops[p].mon_nrec * def.monitor.variables.size();
            o.grid = unsigned((n + kThreads - 1) / kThreads);
            o.index = p;
            o.text = "statemon";
            specs.push_back(o);
            for (size_t y = idx + 1; y < nodes.size(); ++y)
              if (nodes[y].operation == b2ir::ScheduleOp::StateMonitor && nodes[y].owner_kind == b2ir::OwnerKind::Population &&
                  nodes[y].owner_index == p && can_hoist(idx, y))
                done[y] = true;
            break;
          }
          case b2ir::ScheduleOp::SpikeMonitor: break;  // read from the drained spike ring
          case b2ir::ScheduleOp::EventMonitor: {
            // read from the drained ring at results time; no kernel
            check(node.item_index < def.event_monitors.size(), "scheduled EventMonitor has no definition");
            const auto& em = def.event_monitors[node.item_index];
            auto ev = std::find(def.events.begin(), def.events.end(), em.event);
            check(ev != def.events.end(), "EventMonitor event missing from population");
            const size_t e = size_t(ev - def.events.begin());
            size_t producer = nodes.size();
            for (size_t y = 0; y < nodes.size(); ++y) {
              const auto& n2 = nodes[y];
              if (n2.owner_kind != b2ir::OwnerKind::Population || n2.owner_index != p) continue;
              if (n2.operation == b2ir::ScheduleOp::EventSource && e == 0) producer = y;
              if (n2.operation == b2ir::ScheduleOp::CodeObject) {
                const auto& c2 = def.code_objects[n2.item_index];
                if (c2.kind == "threshold" && c2.event_name && *c2.event_name == em.event) producer = y;
              }
            }
            PopDev& pdv = pops[p];
            pdv.evmon_stream.resize(def.event_monitors.size(), -1);
            pdv.evmon_lag.resize(def.event_monitors.size(), 0);
            pdv.evmon_stream[node.item_index] = pdv.stream_of_event[e];
            pdv.evmon_lag[node.item_index] = producer < idx ? 0 : 1;
            if (!em.variables.empty()) {
              // sample kernel at the monitor's place in the tick; with lag 1
              // the previous tick's list must still be in the ring
              EventStreamDev& es = streams[size_t(pdv.stream_of_event[e])];
              es.max_delay = std::max<size_t>(es.max_delay, size_t(pdv.evmon_lag[node.item_index]));
              pdv.evmon_vars.resize(def.event_monitors.size());
              auto& ev = pdv.evmon_vars[node.item_index];
              for (const auto& v : em.variables) {
                size_t w = 8;
                for (const auto& st : def.states)
                  if (st.name == v) w = b2ir::dtype_bytes(st.dtype);
                ev.width.push_back(w);
                ev.ring.push_back(alloc(es.cap * w));
                ev.host.emplace_back();
              }
              OpSpec o;
              o.base = def.name + "_" + em.name;
              o.text = "evmon";
              o.index = p;
              o.grid = 148;
              o.item = node.item_index;
              o.reads = pops[p].evmon_stream[node.item_index];
              specs.push_back(o);
            }
            break;
          }
          case b2ir::ScheduleOp::EventSource: {
            check(pops[p].gen_offsets >= 0, "event source without spike generator");
            OpSpec o;
            o.base = def.name + "_generator";
            o.text = "generator";
            o.index = p;
            stream_produced[size_t(pops[p].stream_of_event[0])] = true;
            specs.push_back(o);
            break;
          }
          case b2ir::ScheduleOp::CodeObject: {
            const auto& code = def.code_objects[node.item_index];
            if (code.kind == "state_update" || code.kind == "threshold") {
              StepSpec st;
              st.pop = p;
              st.node_pos = idx;
              size_t x_pos = idx;
              if (code.kind == "state_update") {
                st.U = compile_pop(p, code);
                for (size_t y = idx + 1; y < nodes.size(); ++y) {
                  const auto& n2 = nodes[y];
                  if (done[y] || n2.owner_kind != b2ir::OwnerKind::Population || n2.owner_index != p ||
                      n2.operation != b2ir::ScheduleOp::CodeObject)
                    continue;
                  const auto& c2 = code_of(n2);
                  if (c2.kind == "threshold" && !no_fuse_ && can_hoist(idx, y)) {
                    st.X = compile_pop(p, c2);
                    done[y] = true;
                    x_pos = y;
                    st.x_event = size_t(std::find(def.events.begin(), def.events.end(), *c2.event_name) - def.events.begin());
                    st.x_spike = *c2.event_name == "spike";
                  }
                  break;
                }
              } else {
                st.X = compile_pop(p, code);
                st.x_event = size_t(std::find(def.events.begin(), def.events.end(), *code.event_name) - def.events.begin());
                st.x_spike = *code.event_name == "spike";
              }
              if (st.X) {
                check(st.x_event < def.events.size(), "threshold event is unknown");
                stream_produced[size_t(pops[p].stream_of_event[st.x_event])] = true;
                for (size_t y = x_pos + 1; y < nodes.size(); ++y) {
                  const auto& n2 = nodes[y];
                  if (done[y] || n2.owner_kind != b2ir::OwnerKind::Population || n2.owner_index != p ||
                      n2.operation != b2ir::ScheduleOp::CodeObject)
                    continue;
                  const auto& c2 = code_of(n2);
                  if (c2.kind == "reset" && c2.event_name && *c2.event_name == def.events[st.x_event]) {
                    bool movable = true;
                    for (size_t z = idx + 1; z < y; ++z)
                      if (!done[z] && conflicts(eff[y], eff[z])) movable = false;
                    if (movable && !no_fuse_) {
                      st.R = compile_pop(p, c2);
                      done[y] = true;
                    }
                    break;
                  }
                }
              }
              OpSpec o;
              o.kind = OpSpec::Kind::Step;
              o.base = def.name + (st.X ? "_step" : "_update");
              o.index = steps_.size();
              o.grid = unsigned(tiles_for(pops[p].count));
              if (st.U) step_of_pop[p] = steps_.size();
              steps_.push_back(st);
              specs.push_back(o);
              if (st.X && streams[size_t(pops[p].stream_of_event[st.x_event])].exchanged) {
                OpSpec x;
                x.base = def.name + "_receive";
                x.text = "exchange";
                x.index = size_t(pops[p].stream_of_event[st.x_event]);
                x.grid = x.lb = kLayoutBlocks;
                specs.push_back(x);
              }
            } else if (code.kind == "reset") {
              OpSpec o;
              o.base = def.name + "_reset";
              size_t e = size_t(std::find(def.events.begin(), def.events.end(), *code.event_name) - def.events.begin());
              check(e < def.events.size(), "reset event is unknown");
              const Program* R = compile_pop(p, code);
              // The spike reset of a population whose threshold sets
              // lastspike, scheduled right after a dense kernel of the same
              // population in this tick (Brunel: after the PoissonInput
              // kernel, which follows the synaptic deliveries): that kernel
              // applies it to the lanes whose lastspike is this tick's t --
              // exactly the tick's fired neurons, since the threshold writes
              // lastspike = t on firing and no initial lastspike is at or
              // after the run's start -- instead of a kernel walking the list.
              if (!no_fuse_ && *code.event_name == "spike" && pops[p].lastspike >= 0 && lastspike_before_start(p) &&
                  stream_produced[size_t(pops[p].stream_of_event[e])] && !specs.empty() &&
                  specs.back().kind == OpSpec::Kind::Step && specs.back().fused_steps.empty()) {
                StepSpec& prev = steps_[specs.back().index];
                std::vector<const Program*> rp{R};
                if (prev.pop == p && !prev.R && !prev.post_R && !writes_available(rp)) {
                  prev.post_R = R;
                  break;
                }
              }
              o.text = gen_reset("@NAME@", p, *R, pops[p].stream_of_event[e]);
              o.reads = pops[p].stream_of_event[e];
              o.grid = 148 * 4;
              specs.push_back(o);
            } else if (code.kind == "poisson_input" || code.kind == "run_regularly" || code.kind == "subexpression_update") {
              const Program* pr = compile_pop(p, code);
              // Defer to the prologue of the population's next state-update
              // step when this node commutes with everything between here and
              // that step in the next tick (the schedule is cyclic).
              auto it = step_of_pop.find(p);
              bool defer = it != step_of_pop.end() && !no_fuse_;
              if (defer) {
                for (size_t y = idx + 1; y < nodes.size() && defer; ++y)
                  if (!done[y] && conflicts(eff[idx], eff[y])) defer = false;
                for (size_t y = 0; y < steps_[it->second].node_pos && defer; ++y)
                  if (conflicts(eff[idx], eff[y])) defer = false;
              }
              if (defer) {
                steps_[it->second].deferred.push_back(pr);
                flushes.push_back({p, pr, {}, nullptr});
              } else {
                StepSpec st;
                st.pop = p;
                st.U = pr;
                st.node_pos = idx;
                OpSpec o;
                o.kind = OpSpec::Kind::Step;
                o.base = def.name + "_" + code.kind;
                o.index = steps_.size();
                o.grid = unsigned(tiles_for(pops[p].count));
                steps_.push_back(st);
                specs.push_back(o);
              }
            } else {
              throw Error("population code object kind '" + code.kind + "' is not supported by the GPU engine");
            }
            break;
          }
        }
      } else {
        check(node.operation == b2ir::ScheduleOp::CodeObject, "synapse monitors are not supported by the GPU engine");
        size_t s = node.owner_index;
        const auto& code = code_of(node);
        if (code.kind == "synapse_state_update" || code.kind == "synapse_subexpression_update" ||
            code.kind == "synapse_run_regularly") {
          // run_synapse_program (executor.rs:2513-2546): every edge, only
          // synapse-state writes committed; edges are independent (a program
          // reads neuron state, which it cannot write, and its own edge's
          // synapse state), so one thread per edge reproduces the edge loop
          const auto& def = m.synapses[s];
          std::map<std::string, WriteTarget> writable;
          auto inputs = synapse_inputs(s, true, writable);
          if (code.kind == "synapse_state_update") {
            std::map<std::string, WriteTarget> clock_driven;
            for (const auto& name : def.clock_driven_states)
              for (size_t k = 0; k < def.states.size(); ++k)
                if (def.states[k].name == name) clock_driven[name] = WriteTarget{WriteTarget::Kind::Synapse, k};
            writable = clock_driven;
          }
          programs.push_back(Program::compile(code, inputs, writable, m.functions));
          const Program& pr = programs.back();
          if (world > 1)
            check(!pr.uses_rng(), "multi-GPU runs do not support random draws in synaptic code ('" + code.name + "')");
          auto rep = replicate_pre_state(pr, s, specs, code.name);
          OpSpec o;
          o.base = code.name;
          o.text = "synprog";
          o.index = synprog_specs.size();
          o.grid = unsigned(std::max<uint64_t>(1, (syns[s].local_edges + kThreads - 1) / kThreads));
          synprog_specs.push_back({s, &pr, rep});
          specs.push_back(o);
          continue;
        }
        if (code.kind == "summed_variable") {
          size_t k = 0;
          while (k < syns[s].summed.size() && syns[s].summed[k].code != node.item_index) ++k;
          check(k < syns[s].summed.size(), "missing summed-variable runtime program");
          const SynDev::Summed& sv = syns[s].summed[k];
          std::map<std::string, WriteTarget> writable;
          auto inputs = synapse_inputs(s, true, writable);
          inputs["dt"] = Input::constant(m.populations[sv.dest_pop].dt, DType::F64);
          programs.push_back(Program::compile(code, inputs, {}, m.functions));
          const Program& pr = programs.back();
          auto res = pr.symbols.find("_synaptic_var");
          check(res != pr.symbols.end(), "missing summed expression result");
          for (const auto& b : pr.bindings) {
            const bool own = b.second.index == sv.dest_state &&
                             (sv.to_pre ? b.second.kind == Input::Kind::PreState : b.second.kind == Input::Kind::PostState);
            check(!own, "a summed expression that reads its own summed variable is not supported by the GPU engine");
          }
          check(world == 1 || !pr.uses_rng(), "multi-GPU runs do not support random draws in synaptic code ('" + code.name + "')");
          auto rep = replicate_pre_state(pr, s, specs, code.name);
          OpSpec o;
          o.base = code.name;
          o.text = "summed";
          o.index = summed_specs.size();
          const PopDev& dp = pops[sv.dest_pop];
          o.grid = unsigned(std::max<size_t>(1, (dp.count + kThreads - 1) / kThreads));
          summed_specs.push_back({s, k, &pr, res->second, rep});
          specs.push_back(o);
          continue;
        }
        check(bool(code.pathway_name), "scheduled pathway has no name");
        const auto& pws = m.synapse_instances[s].pathways;
        size_t pos = pws.size();
        for (size_t k = 0; k < pws.size(); ++k)
          if (pws[k].name == *code.pathway_name) pos = k;
        check(pos < pws.size(), "scheduled pathway has no runtime instance");
        PathwayDev& pw = syns[s].pathways[pos];
        std::map<std::string, WriteTarget> writable;
        auto inputs = synapse_inputs(s, pw.is_pre, writable);
        programs.push_back(Program::compile(code, inputs, writable, m.functions));
        const Program& pr = programs.back();
        std::map<size_t, int> pre_rep;
        if (world > 1) {
          // presynaptic state is complete on every rank for a replicated
          // source; a partitioned one's is copied to every rank first
          pre_rep = replicate_pre_state(pr, s, specs, code.name);
          for (const auto& w : pr.writes)
            check(w.first.kind != WriteTarget::Kind::PreNeuron,
                  "multi-GPU runs cannot write presynaptic state across GPUs ('" + code.name + "')");
          check(!pr.uses_rng(), "multi-GPU runs do not support random draws in synaptic code ('" + code.name + "')");
        }
        classify_pathway(pw, pr);
        if (pw.mode == PathwayDev::Mode::Targets) build_targets_view(pw);
        // Constant-addend pathways reading one spike stream at one delay and
        // writing disjoint target variables share a scatter launch.
        bool merged = false;
        if (pw.mode == PathwayDev::Mode::Atomic && !no_fuse_ && !specs.empty() && specs.back().kind == OpSpec::Kind::Path) {
          PathSpec& ps = paths[specs.back().index];
          PathwayDev* first = ps.pathways.front();
          bool ok = first->mode == PathwayDev::Mode::Atomic && first->stream == pw.stream && first->delay == pw.delay &&
                    m.synapses[first->synapse].target_population == m.synapses[s].target_population;
          for (PathwayDev* other : ps.pathways)
            for (const auto& a : other->atomic_adds)
              for (const auto& b : pw.atomic_adds) ok &= a.state != b.state;
          if (ok) {
            ps.pathways.push_back(&pw);
            ps.programs.push_back(&pr);
            ps.codes.push_back(code.name);
            specs.back().base += "_" + code.name;
            merged = true;
          }
        }
        if (!merged) {
          PathSpec ps;
          ps.pathways.push_back(&pw);
          ps.programs.push_back(&pr);
          ps.codes.push_back(code.name);
          ps.pre_replica = pre_rep;
          OpSpec o;
          o.kind = OpSpec::Kind::Path;
          o.index = paths.size();
          o.base = code.name;
          bool serial = pw.mode == PathwayDev::Mode::Serial;
          o.grid = serial ? 1u : (scatter_blocks_ ? scatter_blocks_ : 148u * 8u);
          o.block = serial ? 32u : kThreads;
          if (pw.mode == PathwayDev::Mode::Targets && !pw.tm_events) {  // tm_warps warps per target
            pw.tm_warps = targets_group(pw);
            const uint64_t per_block = kThreads / 32 / pw.tm_warps;
            o.grid = unsigned(std::max<uint64_t>(1, std::min<uint64_t>((pw.tm_targets + per_block - 1) / per_block,
                                                                        148u * 16u)));
          }
          paths.push_back(ps);
          specs.push_back(o);
          if (pw.mode == PathwayDev::Mode::Targets && pw.tm_events) {
            OpSpec d;  // bucket delivery after the scatter
            d.base = code.name + "_deliver";
            d.text = "tdeliver";
            d.index = paths.size() - 1;
            d.grid = 148u * 8u;
            specs.push_back(d);
          }
        }
      }
    }
    for (size_t sidx = 0; sidx < streams.size(); ++sidx) {
      streams[sidx].produced = stream_produced[sidx];
      EventStreamDev& es = streams[sidx];
      if (es.needs_bitmap) {
        check(stream_produced[sidx], "target-ordered pathway without a threshold producer");
        es.bm_words = (m.populations[es.pop].count + 31) / 32;
        es.bm_slots = es.max_delay + 1;
        const size_t bytes = size_t(es.bm_words * es.bm_slots * 4);
        es.bitmap = alloc(bytes);
        memset_dev(es.bitmap, bytes);
      }
      if (!stream_produced[sidx]) {
        OpSpec o;
        o.base = "empty_stream";
        o.text = gen_empty_stream("@NAME@", int(sidx));
        o.block = 32;
        specs.push_back(o);
      }
    }
    if (!flushes.empty()) {
      std::vector<uint64_t> init(m.populations.size(), UINT64_MAX);
      deferred_flags = upload(init.data(), init.size() * 8);
    }
    // Counted delivery: a run of constant-addend scatters into f32 state of
    // one population, directly followed in the tick by a dense kernel of that
    // population, only counts each target's events (an integer reduction
    // instead of a compare-and-swap loop per event, and no gate load); the
    // dense kernel applies each pathway's map as often, pathways in schedule
    // order, before its own programs.  Every event of a pathway applies the
    // same map, so the result is the reference's sequential one, and nothing
    // between the scatters and that kernel touches the target population.
    // The counts commute, so the scatters of one stream and delay then share
    // a launch.
    if (!no_fuse_ && counted_) {
      auto target_of = [&](const OpSpec& o, size_t& T) -> bool {
        if (o.kind != OpSpec::Kind::Path) return false;
        const auto& pws = paths[o.index].pathways;
        if (pws.empty()) return false;
        for (const PathwayDev* pw : pws) {
          if (pw->mode != PathwayDev::Mode::Atomic || pw->has_pending || !pw->uniform) return false;
          const size_t tpop = m.synapses[pw->synapse].target_population;
          if (pw != pws.front() && tpop != T) return false;
          T = tpop;
          for (const auto& ad : pw->atomic_adds) {
            const DType d = m.populations[T].states[ad.state].dtype;
            if (d != DType::F32 && !(d == DType::F64 && counted_f64_)) return false;
          }
        }
        return true;
      };
      for (size_t i = 0; i < specs.size(); ++i) {
        size_t T = 0, T2 = 0;
        if (!target_of(specs[i], T)) continue;
        size_t j = i + 1;
        while (j < specs.size() && target_of(specs[j], T2) && T2 == T) ++j;
        // The scatters may also end the tick: then the tick's first kernel,
        // T's state-update step, applies the counts in its prologue ahead of
        // the programs deferred into it (they follow the scatters in the
        // schedule, or commute with them), and so does T's flush kernel
        // after the last tick.
        const bool wrap = j >= specs.size() && i > 0 && specs[0].kind == OpSpec::Kind::Step &&
                          steps_[specs[0].index].pop == T && !steps_[specs[0].index].deferred.empty() &&
                          std::any_of(flushes.begin(), flushes.end(), [&](const Flush& f) { return f.pop == T; });
        if (!wrap && (j >= specs.size() || specs[j].kind != OpSpec::Kind::Step || steps_[specs[j].index].pop != T))
          continue;
        Flush* fl = nullptr;
        if (wrap)
          for (Flush& f : flushes)
            if (f.pop == T && !fl) fl = &f;
        std::vector<PathwayDev*> group;
        for (size_t k = i; k < j; ++k)
          for (PathwayDev* pw : paths[specs[k].index].pathways) group.push_back(pw);
        const bool packed = pack_counts_ && group.size() == 2 && group[0]->max_indeg < 65536 &&
                            group[1]->max_indeg < 65536;
        int shared_count = -1;
        if (packed) {
          shared_count = alloc(std::max<size_t>(pops[T].count, 1) * 4);
          memset_dev(shared_count, std::max<size_t>(pops[T].count, 1) * 4);
        }
        for (size_t k = i; k < j; ++k)
          for (PathwayDev* pw : paths[specs[k].index].pathways) {
            pw->counted = true;
            if (packed) {
              pw->count_ptr = shared_count;
              pw->count_packed = true;
              pw->count_shift = pw == group[0] ? 0 : 16;
            } else {
              pw->count_ptr = alloc(std::max<size_t>(pops[T].count, 1) * 4);
              memset_dev(pw->count_ptr, std::max<size_t>(pops[T].count, 1) * 4);
            }
            if (wrap) {
              steps_[specs[0].index].deferred_applies.push_back(pw);
              fl->applies.push_back(pw);
            } else {
              steps_[specs[j].index].applies.push_back(pw);
            }
          }
        for (size_t k = i + 1; k < j;) {
          PathSpec& a = paths[specs[i].index];
          const PathSpec& b = paths[specs[k].index];
          if (a.pathways.front()->stream == b.pathways.front()->stream &&
              a.pathways.front()->delay == b.pathways.front()->delay) {
            a.pathways.insert(a.pathways.end(), b.pathways.begin(), b.pathways.end());
            a.programs.insert(a.programs.end(), b.programs.begin(), b.programs.end());
            a.codes.insert(a.codes.end(), b.codes.begin(), b.codes.end());
            specs[i].base += "_" + specs[k].base;
            specs.erase(specs.begin() + long(k));
            --j;
          } else {
            ++k;
          }
        }
        specs[i].base += "_count";
        i = j;  // the dense kernel
      }
    }
    // One GPU: a step directly followed by the delay-0 constant-addend
    // scatter of the list it produces leaves the list as tile counts and
    // ids, and the scatter lays it out in the ring while delivering it
    // (gen_consumer): the step kernel then has no last-block pass.
    auto fusable = [&](const OpSpec& o, int sid) {
      if (o.kind != OpSpec::Kind::Path) return false;
      for (const PathwayDev* pw : paths[o.index].pathways)
        if (!(pw->mode == PathwayDev::Mode::Atomic && pw->stream == sid && pw->delay == 0 && pw->uniform &&
              !pw->has_pending))
          return false;
      return true;
    };
    if (world == 1 && !no_fuse_ && fuse_exchange_) {
      for (size_t i = 0; i + 1 < specs.size(); ++i) {
        if (specs[i].kind != OpSpec::Kind::Step) continue;
        const StepSpec& st = steps_[specs[i].index];
        if (!st.X) continue;
        const int sid = pops[st.pop].stream_of_event[st.x_event];
        if (!fusable(specs[i + 1], sid) || streams[size_t(sid)].bitmap >= 0) continue;
        streams[size_t(sid)].consumer_layout = true;
        OpSpec& c = specs[i + 1];
        c.fuse_path = int(c.index);
        c.kind = OpSpec::Kind::Text;
        c.text = "exchange";
        c.index = size_t(sid);
        c.base += "_atomic";
        c.lb = 2;  // ~ a few hundred ids per tick at config 2
        // one tile list per scatter block (config 2, ms per 1000 ticks:
        // 17.36 with 1954 blocks for 1954 tiles, against 18.19 with 1184,
        // 17.44 with 888 and 17.47 with 3908)
        c.grid = consumer_blocks_ ? consumer_blocks_
                                  : unsigned(std::max<size_t>(tiles_for(pops[st.pop].count), 148));
        c.grid += c.lb;
      }
    }
    // One GPU, large populations whose list no fused scatter lays out: a
    // layout kernel of kLayoutBlocks blocks after the step (moved below to
    // just before the list's first reader) instead of the step's last block,
    // which would copy a big tick's ids alone (config 3: ~17k ids per tick,
    // 88 us of a 4M-neuron step).
    if (world == 1 && !no_fuse_ && fuse_exchange_) {
      for (size_t i = 0; i < specs.size(); ++i) {
        if (specs[i].kind != OpSpec::Kind::Step) continue;
        const StepSpec& st = steps_[specs[i].index];
        if (!st.X) continue;
        const int sid = pops[st.pop].stream_of_event[st.x_event];
        EventStreamDev& es = streams[size_t(sid)];
        if (es.consumer_layout || tiles_for(pops[st.pop].count) < kLayoutMinTiles) continue;
        es.consumer_layout = true;
        OpSpec x;
        x.base = m.populations[st.pop].name + "_layout";
        x.text = "exchange";
        x.index = size_t(sid);
        x.grid = x.lb = kLayoutBlocks;
        specs.insert(specs.begin() + long(i) + 1, x);
      }
    }
    // Multi-GPU: a receive directly followed by the delay-0 constant-addend
    // scatter of the same stream delivers the spikes itself (gen_consumer),
    // saving a kernel boundary and the ring read per tick.
    if (world > 1 && !no_fuse_ && fuse_exchange_) {
      for (size_t i = 0; i + 1 < specs.size(); ++i) {
        if (specs[i].text != "exchange" || specs[i].fuse_path >= 0 || !fusable(specs[i + 1], int(specs[i].index)))
          continue;
        specs[i].fuse_path = int(specs[i + 1].index);
        specs[i].base += "_" + specs[i + 1].base + "_atomic";
        specs[i].lb = 4;
        // the scatter's own grid (config 2 on two GPUs, ms per 1000 ticks:
        // 15.59 with 1184 scatter blocks, 15.91 with one per (rank, tile)
        // list, which is the better choice on one GPU)
        specs[i].grid = (consumer_blocks_ ? consumer_blocks_ : specs[i + 1].grid) + specs[i].lb;
        specs.erase(specs.begin() + long(i) + 1);
      }
    }
    // A receive or layout kernel whose list nothing reads later in the same
    // tick (every consumer delivers it after a delay) moves to just before
    // the first op that does, or to the end of the tick: on several GPUs the
    // peers' lists then arrive while this rank delivers older ticks' spikes.
    if (!no_fuse_ && fuse_exchange_) {
      auto reads_now = [&](const OpSpec& o, int sid) {
        if (o.kind == OpSpec::Kind::Path) {
          for (const PathwayDev* pw : paths[o.index].pathways)
            if (pw->stream == sid && (pw->delay == 0 || !pw->uniform || pw->has_pending)) return true;
          return false;
        }
        if (o.kind == OpSpec::Kind::Step) return false;  // steps publish lists, they read none
        if (o.text == "tdeliver") return paths[o.index].pathways.front()->stream == sid;
        return o.reads == sid || o.text == "exchange";
      };
      std::set<int> placed;
      for (size_t i = 0; i < specs.size();) {
        if (specs[i].text != "exchange" || specs[i].fuse_path >= 0 || placed.count(int(specs[i].index))) {
          ++i;
          continue;
        }
        const int sid = int(specs[i].index);
        placed.insert(sid);
        size_t j = i + 1;
        while (j < specs.size() && !reads_now(specs[j], sid)) ++j;
        OpSpec moved = specs[i];
        specs.erase(specs.begin() + long(i));
        specs.insert(specs.begin() + long(j - 1), moved);  // i now holds the next unvisited op
      }
    }
    // The tick's last dense kernel of a population (after it only list
    // layout or receive kernels, which touch no population state), when the
    // tick's first kernel is that population's state-update step: nothing
    // runs between the two, so the dense kernel's work -- its counted
    // applies, its program, its reset of the lanes the tick fired -- moves
    // into the step's prologue, with the previous tick's t and RNG counter
    // (config 3: the PoissonInput kernel).  A flush kernel applies the last
    // tick's copy at the end of a run or before a state read.
    if (!no_fuse_ && specs.size() >= 2) {
      size_t last = specs.size();
      while (last > 0 && specs[last - 1].text == "exchange" && specs[last - 1].fuse_path < 0) --last;
      if (last >= 2 && specs[last - 1].kind == OpSpec::Kind::Step && specs[0].kind == OpSpec::Kind::Step) {
        const StepSpec T = steps_[specs[last - 1].index];
        StepSpec& S = steps_[specs[0].index];
        if (T.pop == S.pop && T.U && !T.X && !T.R && T.deferred.empty() && T.deferred_applies.empty() &&
            !T.deferred_post_R && S.U && S.deferred.empty() && S.deferred_applies.empty() && !S.deferred_post_R &&
            specs[last - 1].fused_steps.empty() && specs[0].fused_steps.empty()) {
          S.deferred.push_back(T.U);
          S.deferred_applies = T.applies;
          S.deferred_post_R = T.post_R;
          flushes.push_back({T.pop, T.U, T.applies, T.post_R});
          if (deferred_flags < 0) {
            std::vector<uint64_t> init(m.populations.size(), UINT64_MAX);
            deferred_flags = upload(init.data(), init.size() * 8);
          }
          specs.erase(specs.begin() + long(last - 1));
        }
      }
    }
    // A layout or receive kernel right after a constant-addend scatter that
    // reads older ticks of the lists only: the scatter launch lays the list
    // out in its first blocks (gen_atomic_kernel) instead.  Neither reads
    // what the other writes (the layout writes ring positions of this tick
    // and tick_start[rel + 1]; the scatter reads the lists of ticks at least
    // one back), and on several GPUs the layout blocks wait for the peers'
    // lists while the other blocks deliver.
    if (!no_fuse_ && fuse_layout_) {
      for (size_t i = 1; i < specs.size();) {
        OpSpec& prev = specs[i - 1];
        bool ok = specs[i].text == "exchange" && specs[i].fuse_path < 0 && prev.kind == OpSpec::Kind::Path &&
                  prev.layout_sid < 0;
        if (ok) {
          const auto& pws = paths[prev.index].pathways;
          ok = !(pws.size() == 1 && pws[0]->mode != PathwayDev::Mode::Atomic);
          for (const PathwayDev* pw : pws)
            ok = ok && pw->mode == PathwayDev::Mode::Atomic && pw->uniform && !pw->has_pending && pw->delay > 0;
        }
        if (!ok) {
          ++i;
          continue;
        }
        prev.layout_sid = int(specs[i].index);
        prev.lb = specs[i].lb;
        prev.grid += specs[i].lb;
        prev.base += "_" + specs[i].base;
        specs.erase(specs.begin() + long(i));
      }
    }
    // Consecutive step kernels of different populations touch disjoint state
    // (population code reads and writes only its own population), so one
    // launch steps them all: block ranges dispatch to per-population tiles,
    // saving a dependent launch per tick.
    if (!no_fuse_ && fuse_steps_) {
      for (size_t i = 0; i + 1 < specs.size();) {
        OpSpec& a = specs[i];
        const OpSpec& b = specs[i + 1];
        bool ok = a.kind == OpSpec::Kind::Step && b.kind == OpSpec::Kind::Step;
        if (ok) {
          std::set<size_t> seen{steps_[a.index].pop};
          for (size_t f : a.fused_steps) seen.insert(steps_[f].pop);
          ok = !seen.count(steps_[b.index].pop);
        }
        if (!ok) {
          ++i;
          continue;
        }
        a.fused_steps.push_back(b.index);
        a.base += "_" + b.base;
        a.grid += b.grid;
        specs.erase(specs.begin() + long(i) + 1);
      }
    }
    // ---- emit
    std::ostringstream src, bodies, kernels;
    src << "// generated by brian2-atlas_b200 for one AtlasIR model\n";
    src << kDeviceLibSource << "\n";
    src << "__constant__ u64 g_ptr[PTR_COUNT_PLACEHOLDER];\n\n";
    int kid = 0;
    std::vector<std::string> op_text;  // each op's kernel source (for the chunk kernel)
    for (auto& o : specs) {
      const size_t text_from = kernels.str().size();
      std::string nm = "b2_" + std::to_string(kid++) + "_" + sanitize(o.base);
      switch (o.kind) {
        case OpSpec::Kind::Text:
          if (o.text == "statemon") kernels << gen_state_monitor(nm, o.index);
          else if (o.text == "generator") kernels << gen_event_source(nm, o.index, pops[o.index].stream_of_event[0]);
          else if (o.text == "evmon") kernels << gen_evmon(nm, o.index, o.item);
          else if (o.text == "tdeliver") {
            PathSpec& ps = paths[o.index];
            const std::string pf = ps.body + "_prefetch";
            bodies << gen_pathway_prefetch(pf, ps.pathways[0]->synapse, *ps.programs[0], &ps.pre_replica);
            kernels << gen_targets_deliver(nm, ps.body, pf, *ps.pathways[0]);
          }
          else if (o.text == "synprog") {
            const SynProgSpec& sp = synprog_specs[o.index];
            std::string body = "b2_synprog_" + std::to_string(kid);
            PathwayDev none;
            bodies << gen_pathway_body(body, sp.synapse, none, *sp.program, true, &sp.pre_replica);
            const SynDev& sd = syns[sp.synapse];
            std::ostringstream k;
            k << kernel_head(nm);
            k << "  const u64 e = blockIdx.x * (u64)blockDim.x + threadIdx.x;\n";
            k << "  if (e < " << sd.local_edges << "ull) " << body << "(" << P(sd.edge_src, "const u32") << "[e], "
              << P(sd.edge_tgt, "const u32") << "[e], e, tick, t, err);\n";
            k << kernel_tail();
            kernels << k.str();
          } else if (o.text == "summed") {
            const SummedSpec& ss = summed_specs[o.index];
            std::string body = "b2_summed_" + std::to_string(kid);
            bodies << gen_summed_body(body, ss);
            kernels << gen_summed(nm, body, ss);
          } else if (o.text == "replicate")
            kernels << gen_replicate(nm, replicas[o.index]);
          else if (o.text == "replica_wait")
            kernels << gen_replica_wait(nm, replicas[o.index]);
          else if (o.text == "exchange")
            kernels << gen_consumer(nm, int(o.index),
                                    o.fuse_path >= 0 ? paths[size_t(o.fuse_path)].pathways : std::vector<PathwayDev*>{},
                                    o.grid, o.lb);
          else {
            std::string t = o.text;
            t.replace(t.find("@NAME@"), 6, nm);
            kernels << t;
          }
          break;
        case OpSpec::Kind::Step: {
          if (o.fused_steps.empty()) {
            const StepSpec& st = steps_[o.index];
            kernels << gen_pop_step(nm, st.pop, st.U, st.X, st.x_event, st.x_spike, st.R, st.deferred, false, false,
                                    st.applies, st.post_R, st.deferred_applies, st.deferred_post_R);
            break;
          }
          std::vector<size_t> group{o.index};
          group.insert(group.end(), o.fused_steps.begin(), o.fused_steps.end());
          std::ostringstream disp;
          uint64_t first = 0;
          for (size_t g = 0; g < group.size(); ++g) {
            const StepSpec& st = steps_[group[g]];
            const std::string fn = nm + "_part" + std::to_string(g);
            kernels << gen_pop_step(fn, st.pop, st.U, st.X, st.x_event, st.x_spike, st.R, st.deferred, false, true,
                                    st.applies, st.post_R, st.deferred_applies, st.deferred_post_R);
            const uint64_t tiles = tiles_for(pops[st.pop].count);
            disp << "  " << (g ? "else if" : "if") << " (blockIdx.x < " << first + tiles << "u) " << fn
                 << "(ctl, tick, rel, t, blockIdx.x - " << first << "u, err);\n";
            first += tiles;
          }
          check(first == o.grid, "fused step grid mismatch");
          kernels << kernel_head(nm, min_blocks_) << disp.str() << kernel_tail();
          break;
        }
        case OpSpec::Kind::Path: {
          PathSpec& ps = paths[o.index];
          if (ps.pathways.size() == 1 && ps.pathways[0]->mode != PathwayDev::Mode::Atomic) {
            std::string body = "b2_body_" + std::to_string(kid) + "_" + sanitize(ps.codes[0]);
            bodies << gen_pathway_body(body, ps.pathways[0]->synapse, *ps.pathways[0], *ps.programs[0], false,
                                       &ps.pre_replica);
            ps.body = body;
            const auto md = ps.pathways[0]->mode;
            const char* mode = md == PathwayDev::Mode::EdgeParallel ? "_edges"
                               : md == PathwayDev::Mode::Targets    ? "_targets"
                                                                    : "_serial";
            nm += mode;
            kernels << gen_pathway_kernel(nm, body, *ps.pathways[0]);
          } else {
            nm += "_atomic";
            kernels << gen_atomic_kernel(nm, ps.pathways, o.layout_sid, o.layout_sid >= 0 ? o.lb : 0);
          }
          break;
        }
      }
      ops.push_back({nm, nullptr, o.grid, o.block});
      op_text.push_back(kernels.str().substr(text_from));
    }
    if (mega_) kernels << gen_chunk_kernel(op_text);
    for (size_t f = 0; f < flushes.size(); ++f) {
      size_t p = flushes[f].pop;
      std::string nm = "b2_flush_" + std::to_string(f) + "_" + sanitize(m.populations[p].name);
      kernels << gen_pop_step(nm, p, flushes[f].program, nullptr, 0, false, nullptr, {}, true, false, flushes[f].applies,
                              flushes[f].post_R);
      flush_ops.push_back({nm, nullptr, unsigned(tiles_for(pops[p].count)), kThreads});
    }
    for (const auto& [name, def] : const_tables) src << def << "\n";
    src << bodies.str() << "\n" << kernels.str();
    source = src.str();
    std::string placeholder = "PTR_COUNT_PLACEHOLDER";
    source.replace(source.find(placeholder), placeholder.size(), std::to_string(std::max<size_t>(ptrs.size(), 1)));
  }

  // ================================================================ compile
  void compile_module() {
    auto t0 = std::chrono::steady_clock::now();
    nvrtcProgram prog;
    B2_NVRTC(nvrtcCreateProgram(&prog, source.c_str(), "b2_model.cu", 0, nullptr, nullptr));
    int major = 10, minor = 0;  // dry runs compile for sm_100a
    if (!opt.dry_run) {
      B2_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
      B2_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
    }
    std::string arch = "--gpu-architecture=sm_" + std::to_string(major) + std::to_string(minor) + (major >= 9 ? "a" : "");
    const char* opts[] = {arch.c_str(), "--std=c++17", "--fmad=false", "--prec-div=true", "--prec-sqrt=true",
                          "--ftz=false", "-default-device", "-lineinfo"};
    nvrtcResult res = nvrtcCompileProgram(prog, int(sizeof(opts) / sizeof(opts[0])), opts);
    size_t log_size = 0;
    nvrtcGetProgramLogSize(prog, &log_size);
    std::string log(log_size, '\0');
    if (log_size) nvrtcGetProgramLog(prog, log.data());
    if (res != NVRTC_SUCCESS) {
      nvrtcDestroyProgram(&prog);
      throw Error("kernel compilation failed: " + log.substr(0, 4000));
    }
    size_t cubin_size = 0;
    B2_NVRTC(nvrtcGetCUBINSize(prog, &cubin_size));
    std::vector<char> cubin(cubin_size);
    B2_NVRTC(nvrtcGetCUBIN(prog, cubin.data()));
    nvrtcDestroyProgram(&prog);
    st.compile_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    cubin_bytes = cubin.size();
    if (opt.dry_run) return;
    B2_CUDA(cudaLibraryLoadData(&module, cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0));
    void* table = nullptr;
    size_t table_bytes = 0;
    B2_CUDA(cudaLibraryGetGlobal(&table, &table_bytes, module, "g_ptr"));
    check(table_bytes >= ptrs.size() * 8, "pointer table size mismatch");
    gptr_table = table;
    B2_CUDA(cudaStreamSynchronize(stream));
    if (!ptrs.empty()) B2_CUDA(cudaMemcpy(table, ptrs.data(), ptrs.size() * 8, cudaMemcpyHostToDevice));
    for (auto& op : ops) B2_CUDA(cudaLibraryGetKernel(&op.fn, module, op.name.c_str()));
    for (auto& op : flush_ops) B2_CUDA(cudaLibraryGetKernel(&op.fn, module, op.name.c_str()));
    if (mega_) {
      B2_CUDA(cudaLibraryGetKernel(&mega_fn, module, "b2_chunk"));
      int per_sm = 0;
      B2_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reinterpret_cast<const void*>(mega_fn), int(kThreads), 0));
      int sms = 0;
      B2_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
      mega_grid = unsigned(std::max(0, per_sm) * sms);
      check(mega_grid > 0, "the chunk kernel cannot be resident on this device");
      mega_bar = DeviceBuffer(256);
    }
  }
  size_t cubin_bytes = 0;

  // ================================================================ run loop
  void launch_tick(uint32_t k) {
    void* ctl_ptr = ctl.ptr;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    for (auto& op : ops) {
      void* args[] = {&ctl_ptr, &k};
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(op.grid);
      cfg.blockDim = dim3(op.block);
      cfg.stream = stream;
      cfg.attrs = attr;
      cfg.numAttrs = use_pdl_ ? 1 : 0;
      B2_CUDA(cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(op.fn), args));
    }
  }

  // One cooperative launch of the chunk kernel for ticks 0 .. n-1 of the
  // chunk (the driver refuses the launch if the grid cannot be co-resident,
  // so the grid barriers cannot wait on a block that never runs).
  void launch_chunk(uint32_t n) {
    B2_CUDA(cudaMemsetAsync(mega_bar.ptr, 0, 4, stream));
    void* ctl_ptr = ctl.ptr;
    void* bar_ptr = mega_bar.ptr;
    uint32_t k0 = 0;
    void* args[] = {&ctl_ptr, &k0, &n, &bar_ptr};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(mega_grid);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    B2_CUDA(cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(mega_fn), args));
  }

  void ensure_graph(uint32_t ticks) {
    if (graph_exec && graph_ticks == ticks) return;
    if (graph_exec) {
      cudaGraphExecDestroy(graph_exec);
      graph_exec = nullptr;
    }
    cudaGraph_t graph;
    B2_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    for (uint32_t k = 0; k < ticks; ++k) launch_tick(k);
    B2_CUDA(cudaStreamEndCapture(stream, &graph));
    B2_CUDA(cudaGraphInstantiate(&graph_exec, graph, 0));
    cudaGraphDestroy(graph);
    graph_ticks = ticks;
  }

  uint64_t tick_host_ = 0;  // pageable staging: the copy is complete when the call returns

  void drain(size_t rel0, size_t rel1) {
    for (auto& es : streams) {
      std::vector<uint64_t> ts(rel1 - rel0 + 1);
      B2_CUDA(cudaMemcpy(ts.data(), static_cast<uint64_t*>(dptr(es.tick_start)) + rel0, ts.size() * 8, cudaMemcpyDeviceToHost));
      st.d2h_bytes += ts.size() * 8 + (ts.back() - ts.front()) * 4;
      check(ts[0] == es.drained_pos, "spike ring bookkeeping mismatch");
      uint64_t a = ts.front(), b = ts.back();
      size_t old = es.ids.size();
      es.ids.resize(old + (b - a));
      uint64_t pos = a;
      while (pos < b) {
        uint64_t idx = pos & es.mask;
        uint64_t n = std::min<uint64_t>(b - pos, es.cap - idx);
        B2_CUDA(cudaMemcpy(es.ids.data() + old + (pos - a), static_cast<uint32_t*>(dptr(es.ring)) + idx, n * 4,
                           cudaMemcpyDeviceToHost));
        pos += n;
      }
      for (size_t k = 1; k < ts.size(); ++k) es.starts.push_back(ts[k]);
      es.drained_pos = b;
    }
    // EventMonitor samples of the ticks whose sample kernel has run: all of
    // [rel0, rel1) for lag 0, one tick less for a monitor that samples the
    // previous tick's list
    for (auto& pd : pops)
      for (size_t k = 0; k < pd.evmon_vars.size(); ++k) {
        auto& ev = pd.evmon_vars[k];
        if (ev.ring.empty()) continue;
        const EventStreamDev& es = streams[size_t(pd.evmon_stream[k])];
        const size_t lag = size_t(pd.evmon_lag[k]);
        if (rel1 < lag) continue;
        const uint64_t b = es.starts[rel1 - lag];
        for (size_t v = 0; v < ev.ring.size(); ++v) {
          const size_t w = ev.width[v];
          auto& host = ev.host[v];
          const size_t old = host.size();
          host.resize(old + (b - ev.drained) * w);
          uint64_t pos = ev.drained;
          while (pos < b) {
            uint64_t idx = pos & es.mask;
            uint64_t n = std::min<uint64_t>(b - pos, es.cap - idx);
            B2_CUDA(cudaMemcpy(host.data() + old + (pos - ev.drained) * w, static_cast<uint8_t*>(dptr(ev.ring[v])) + idx * w,
                               n * w, cudaMemcpyDeviceToHost));
            pos += n;
          }
          st.d2h_bytes += (b - ev.drained) * w;
        }
        ev.drained = b;
      }
  }

  void update_floor(size_t rel_now) {
    // Per stream, the oldest ring position a consumer may still read in the
    // next chunk (everything older has been drained to the host).
    for (size_t k = 0; k < streams.size(); ++k) {
      const auto& es = streams[k];
      size_t back = rel_now > es.max_delay ? rel_now - es.max_delay : 0;
      floors_host_[k] = es.starts.size() > back ? es.starts[back] : 0;
    }
    B2_CUDA(cudaMemcpy(dptr(floors_ptr), floors_host_.data(), floors_host_.size() * 8, cudaMemcpyHostToDevice));
    st.h2d_bytes += floors_host_.size() * 8;
  }

  // Per-kernel timing: direct launches bracketed by events (no graph).
  // Per-kernel timing: the chunk is captured as a CUDA graph like step()'s,
  // with an event record node after every kernel (so kernels run back to
  // back without host launch gaps, in plain stream order: the event nodes
  // replace the programmatic overlap); each event interval is one kernel.
  std::vector<KernelTime> profile(uint64_t ticks) {
    check(!opt.dry_run && !failed, "profiling needs a live engine");
    check(world == 1 || connected, "a multi-GPU engine must connect() to its peers before stepping");
    std::vector<KernelTime> out(ops.size());
    for (size_t i = 0; i < ops.size(); ++i) out[i].name = ops[i].name;
    const size_t per_tick = ops.size();
    std::vector<cudaEvent_t> evs(size_t(opt.chunk_ticks) * per_tick + 1);
    for (auto& e : evs) B2_CUDA(cudaEventCreate(&e));
    cudaGraphExec_t exec = nullptr;
    uint32_t exec_ticks = 0;
    auto release = [&] {
      if (exec) cudaGraphExecDestroy(exec);
      for (auto& e : evs) cudaEventDestroy(e);
    };
    uint64_t remaining = std::min<uint64_t>(ticks, steps - cur_rel);
    try {
      while (remaining > 0) {
        uint32_t n = uint32_t(std::min<uint64_t>(remaining, opt.chunk_ticks));
        if (!exec || exec_ticks != n) {
          if (exec) cudaGraphExecDestroy(exec);
          exec = nullptr;
          cudaGraph_t graph;
          B2_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
          // external record nodes: the events are timed after the replay
          B2_CUDA(cudaEventRecordWithFlags(evs[0], stream, cudaEventRecordExternal));
          void* ctl_ptr = ctl.ptr;
          for (uint32_t k = 0; k < n; ++k)
            for (size_t i = 0; i < per_tick; ++i) {
              uint32_t kk = k;
              void* args[] = {&ctl_ptr, &kk};
              B2_CUDA(cudaLaunchKernel(reinterpret_cast<const void*>(ops[i].fn), dim3(ops[i].grid),
                                       dim3(ops[i].block), args, 0, stream));
              B2_CUDA(cudaEventRecordWithFlags(evs[size_t(k) * per_tick + i + 1], stream, cudaEventRecordExternal));
            }
          B2_CUDA(cudaStreamEndCapture(stream, &graph));
          B2_CUDA(cudaGraphInstantiate(&exec, graph, 0));
          cudaGraphDestroy(graph);
          exec_ticks = n;
        }
        tick_host_ = start_tick + cur_rel;
        B2_CUDA(cudaMemcpyAsync(ctl.ptr, &tick_host_, 8, cudaMemcpyHostToDevice, stream));
        B2_CUDA(cudaGraphLaunch(exec, stream));
        B2_CUDA(cudaStreamSynchronize(stream));
        for (uint32_t k = 0; k < n; ++k)
          for (size_t i = 0; i < per_tick; ++i) {
            float ms = 0.f;
            const size_t at = size_t(k) * per_tick + i;
            B2_CUDA(cudaEventElapsedTime(&ms, evs[at], evs[at + 1]));
            out[i].total_ms += ms;
            out[i].launches += 1;
          }
        st.kernel_launches += uint64_t(n) * per_tick;
        check_error();
        drain(cur_rel, cur_rel + n);
        cur_rel += n;
        remaining -= n;
        update_floor(cur_rel);
        deferred_pending = !flushes.empty();
      }
    } catch (...) {
      release();
      throw;
    }
    release();
    if (cur_rel >= steps) flush_deferred();
    st.ticks = cur_rel;
    return out;
  }



  void check_error() {
    uint32_t err = 0;
    B2_CUDA(cudaMemcpy(&err, static_cast<char*>(ctl.ptr) + 8, 4, cudaMemcpyDeviceToHost));
    if (err) {
      failed = true;
      throw Error(error_message(err));
    }
  }

  bool step(uint64_t max_ticks) {
    check(!opt.dry_run, "a dry-run engine cannot step");
    check(!failed, "execution failed; create a new executor");
    check(max_ticks > 0, "step requires a positive tick budget");
    check(world == 1 || connected, "a multi-GPU engine must connect() to its peers before stepping");
    auto t0 = std::chrono::steady_clock::now();
    try {
      uint64_t remaining = std::min<uint64_t>(max_ticks, steps - cur_rel);
      while (remaining > 0) {
        uint32_t n = uint32_t(std::min<uint64_t>(remaining, opt.chunk_ticks));
        tick_host_ = start_tick + cur_rel;
        B2_CUDA(cudaMemcpyAsync(ctl.ptr, &tick_host_, 8, cudaMemcpyHostToDevice, stream));
        st.h2d_bytes += 8;
        if (!mega_ && opt.use_graphs && n == opt.chunk_ticks) ensure_graph(n);
        B2_CUDA(cudaEventRecord(ev_start, stream));
        if (mega_) {
          launch_chunk(n);
        } else if (opt.use_graphs && n == opt.chunk_ticks) {
          B2_CUDA(cudaGraphLaunch(graph_exec, stream));
        } else {
          for (uint32_t k = 0; k < n; ++k) launch_tick(k);
        }
        B2_CUDA(cudaEventRecord(ev_stop, stream));
        st.kernel_launches += mega_ ? 1 : uint64_t(n) * ops.size();
        B2_CUDA(cudaStreamSynchronize(stream));
        float ms = 0.f;
        B2_CUDA(cudaEventElapsedTime(&ms, ev_start, ev_stop));
        st.device_seconds += double(ms) * 1e-3;
        check_error();
        drain(cur_rel, cur_rel + n);
        cur_rel += n;
        remaining -= n;
        update_floor(cur_rel);
        deferred_pending = !flushes.empty();
      }
      if (cur_rel >= steps) flush_deferred();
    } catch (...) {
      failed = true;
      st.simulation_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      throw;
    }
    st.simulation_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    st.ticks = cur_rel;
    return cur_rel >= steps;
  }

  // Apply the deferred trailing neuron maps of the last simulated tick (they
  // normally run in the next tick's step prologue) so that state reads and
  // results see exactly the reference's state after that tick.
  void flush_deferred() {
    if (!deferred_pending || cur_rel == 0) return;
    tick_host_ = start_tick + cur_rel - 1;
    B2_CUDA(cudaMemcpy(ctl.ptr, &tick_host_, 8, cudaMemcpyHostToDevice));
    void* ctl_ptr = ctl.ptr;
    uint32_t k = 0;
    for (auto& op : flush_ops) {
      void* args[] = {&ctl_ptr, &k};
      B2_CUDA(cudaLaunchKernel(reinterpret_cast<const void*>(op.fn), dim3(op.grid), dim3(op.block), args, 0, stream));
      st.kernel_launches += 1;
    }
    B2_CUDA(cudaStreamSynchronize(stream));
    check_error();
    deferred_pending = false;
  }

  // ================================================================ results
  std::vector<uint8_t> read_bytes(int k, size_t bytes) {
    std::vector<uint8_t> out(bytes);
    if (bytes) B2_CUDA(cudaMemcpy(out.data(), dptr(k), bytes, cudaMemcpyDeviceToHost));
    return out;
  }

  // ---------------------------------------------------------------- multi-GPU
  std::vector<uint8_t> ipc_handle() const {
    check(world > 1 && !opt.dry_run, "IPC handles exist for live multi-GPU engines only");
    cudaIpcMemHandle_t h;
    B2_CUDA(cudaIpcGetMemHandle(&h, arena.ptr));
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&h);
    return std::vector<uint8_t>(b, b + sizeof(h));
  }

  void connect(const std::vector<std::vector<uint8_t>>& handles) {
    check(world > 1, "connect() is for multi-GPU engines");
    check(!opt.dry_run && !failed, "connect() needs a live engine");
    check(!connected, "engine is already connected");
    check(handles.size() == size_t(world), "connect() needs one handle per rank");
    peer_base.assign(size_t(world), nullptr);
    for (int q = 0; q < world; ++q) {
      if (q == rank) continue;
      check(handles[size_t(q)].size() == sizeof(cudaIpcMemHandle_t), "malformed IPC handle");
      cudaIpcMemHandle_t h;
      std::memcpy(&h, handles[size_t(q)].data(), sizeof(h));
      B2_CUDA(cudaIpcOpenMemHandle(&peer_base[size_t(q)], h, cudaIpcMemLazyEnablePeerAccess));
    }
    std::vector<ArenaHeader> heads(static_cast<size_t>(world));
    for (int q = 0; q < world; ++q) {
      const void* src = q == rank ? arena.ptr : peer_base[size_t(q)];
      B2_CUDA(cudaMemcpy(&heads[size_t(q)], src, sizeof(ArenaHeader), cudaMemcpyDeviceToHost));
      const ArenaHeader& h = heads[size_t(q)];
      check(h.magic == kArenaMagic && h.rank == q && h.world == world,
            "IPC handle " + std::to_string(q) + " is not rank " + std::to_string(q) + " of this run");
      check(h.bytes == arena_bytes_of(q), "rank " + std::to_string(q) + " built a different model or partition");
      for (int r = 0; r < q; ++r)
        check(std::memcmp(heads[size_t(r)].uuid, h.uuid, 16) != 0,
              "ranks " + std::to_string(r) + " and " + std::to_string(q) + " share one GPU; use one GPU per rank");
    }
    for (auto& es : streams) {
      if (!es.exchanged) continue;
      for (int q = 0; q < world; ++q)
        if (q != rank)
          ptrs[size_t(es.xptr[size_t(q)])] = reinterpret_cast<uint64_t>(static_cast<char*>(peer_base[size_t(q)]) + es.x_off);
    }
    for (auto& r : replicas)
      for (int q = 0; q < world; ++q)
        if (q != rank) {
          ptrs[size_t(r.rptr[size_t(q)])] = reinterpret_cast<uint64_t>(static_cast<char*>(peer_base[size_t(q)]) + r.off);
          ptrs[size_t(r.fptr[size_t(q)])] =
              reinterpret_cast<uint64_t>(static_cast<char*>(peer_base[size_t(q)]) + r.flags_off);
        }
    B2_CUDA(cudaMemcpy(gptr_table, ptrs.data(), ptrs.size() * 8, cudaMemcpyHostToDevice));
    connected = true;
  }

  void publish() {
    check(world > 1, "publish() is for multi-GPU engines");
    check(!failed && cur_rel >= steps, "publish requires a completed execution");
    flush_deferred();
    const StageLayout L = stage_layout(rank);
    char* base = static_cast<char*>(arena.ptr) + arena_stage_off;
    auto put = [&](size_t off, int k, size_t bytes) {
      if (bytes) B2_CUDA(cudaMemcpyAsync(base + off, dptr(k), bytes, cudaMemcpyDeviceToDevice, stream));
    };
    for (size_t p = 0; p < m.populations.size(); ++p) {
      const auto& def = m.populations[p];
      const PopDev& pd = pops[p];
      // a replicated population is staged by rank 0 only (count 0 elsewhere)
      const uint64_t n = L.count[p];
      for (size_t s = 0; s < def.states.size(); ++s)
        put(L.state[p][s], pd.states[s].ptr, n * b2ir::dtype_bytes(def.states[s].dtype));
      if (pd.lastspike >= 0) {
        put(L.lastspike[p], pd.lastspike, n * 8);
        put(L.not_refractory[p], pd.not_refractory, n);
      }
      if (pd.mon_records >= 0 && !L.mon_positions[p].empty())
        for (size_t v = 0; v < pd.mon_samples.size(); ++v)
          put(L.monitor[p][v], pd.mon_samples[v], pd.mon_ticks * pd.mon_nrec * b2ir::dtype_bytes(pd.mon_dtypes[v]));
    }
    for (size_t s = 0; s < m.synapses.size(); ++s)
      for (size_t k = 0; k < syns[s].states.size(); ++k)
        put(L.syn_state[s][k], syns[s].states[k].ptr, syns[s].local_edges * b2ir::dtype_bytes(m.synapses[s].states[k].dtype));
    put(L.delivered, delivered_ptr, delivered_count * 8);
    // local event lists: a device copy of the drained list, exported by IPC
    // handle, and the per-tick starts (kept until the engine is destroyed, so
    // rank 0 can read them after the host barrier)
    for (size_t k = 0; k < streams.size(); ++k) {
      const EventStreamDev& es = streams[k];
      if (!es.local) continue;
      check(es.starts.size() == steps + 1, "local event list bookkeeping mismatch");
      published_lists.emplace_back(std::max<size_t>(es.ids.size(), 4) * 4);
      DeviceBuffer& buf = published_lists.back();
      if (!es.ids.empty())
        B2_CUDA(cudaMemcpyAsync(buf.ptr, es.ids.data(), es.ids.size() * 4, cudaMemcpyHostToDevice, stream));
      cudaIpcMemHandle_t h;
      B2_CUDA(cudaIpcGetMemHandle(&h, buf.ptr));
      const uint64_t n = es.ids.size();
      B2_CUDA(cudaMemcpyAsync(base + L.local_starts[k], es.starts.data(), (steps + 1) * 8, cudaMemcpyHostToDevice, stream));
      B2_CUDA(cudaMemcpyAsync(base + L.local_handle[k], &h, 64, cudaMemcpyHostToDevice, stream));
      B2_CUDA(cudaMemcpyAsync(base + L.local_handle[k] + 64, &n, 8, cudaMemcpyHostToDevice, stream));
      B2_CUDA(cudaStreamSynchronize(stream));  // h and n are stack values
    }
    B2_CUDA(cudaStreamSynchronize(stream));
    published = true;
  }

  // Every rank's staging area as host bytes (rank 0, after all ranks published).
  std::vector<std::vector<uint8_t>> gather_stages(std::vector<StageLayout>& layouts) {
    check(rank == 0, "rank 0 assembles the results of a multi-GPU run");
    check(published, "every rank must publish() before rank 0 reads results");
    std::vector<std::vector<uint8_t>> out(static_cast<size_t>(world));
    for (int q = 0; q < world; ++q) {
      layouts.push_back(stage_layout(q));
      const char* src = static_cast<const char*>(q == rank ? arena.ptr : peer_base[size_t(q)]) + arena_stage_off;
      out[size_t(q)].resize(layouts.back().bytes);
      if (layouts.back().bytes)
        B2_CUDA(cudaMemcpy(out[size_t(q)].data(), src, layouts.back().bytes, cudaMemcpyDeviceToHost));
    }
    return out;
  }

  b2dump::ResultSet results() {
    check(!failed && cur_rel >= steps, "results require a completed execution");
    flush_deferred();
    B2_CUDA(cudaStreamSynchronize(stream));
    std::vector<StageLayout> lay;
    std::vector<std::vector<uint8_t>> stg;
    if (world > 1) stg = gather_stages(lay);
    if (world > 1 && !lists_merged) {
      // local lists: every rank's list per tick, in rank order (= ascending)
      for (size_t k = 0; k < streams.size(); ++k) {
        EventStreamDev& es = streams[k];
        if (!es.local) continue;
        std::vector<std::vector<uint32_t>> ids(static_cast<size_t>(world));
        std::vector<std::vector<uint64_t>> starts(static_cast<size_t>(world), std::vector<uint64_t>(steps + 1));
        for (int q = 0; q < world; ++q) {
          const uint8_t* b = stg[size_t(q)].data();
          std::memcpy(starts[size_t(q)].data(), b + lay[size_t(q)].local_starts[k], (steps + 1) * 8);
          uint64_t n = 0;
          std::memcpy(&n, b + lay[size_t(q)].local_handle[k] + 64, 8);
          if (q == rank) {
            ids[size_t(q)] = es.ids;
          } else if (n) {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, b + lay[size_t(q)].local_handle[k], 64);
            void* peer = nullptr;
            B2_CUDA(cudaIpcOpenMemHandle(&peer, h, cudaIpcMemLazyEnablePeerAccess));
            ids[size_t(q)].resize(n);
            cudaError_t e = cudaMemcpy(ids[size_t(q)].data(), peer, n * 4, cudaMemcpyDeviceToHost);
            cudaIpcCloseMemHandle(peer);
            B2_CUDA(e);
          }
          check(ids[size_t(q)].size() == n && starts[size_t(q)][steps] == n, "local event list size mismatch");
        }
        std::vector<uint32_t> merged;
        std::vector<uint64_t> mstarts(1, 0);
        for (size_t rel = 0; rel < steps; ++rel) {
          for (int q = 0; q < world; ++q)
            merged.insert(merged.end(), ids[size_t(q)].begin() + long(starts[size_t(q)][rel]),
                          ids[size_t(q)].begin() + long(starts[size_t(q)][rel + 1]));
          mstarts.push_back(merged.size());
        }
        es.ids = std::move(merged);
        es.starts = std::move(mstarts);
      }
      lists_merged = true;
    }
    // population column: local device array on one GPU, else every rank's
    // block in rank order
    auto pop_column = [&](size_t p, int k, size_t elem, const std::function<size_t(const StageLayout&)>& off) {
      if (world == 1) return read_bytes(k, m.populations[p].count * elem);
      std::vector<uint8_t> out;
      for (int q = 0; q < world; ++q) {
        const StageLayout& L = lay[size_t(q)];
        const uint8_t* b = stg[size_t(q)].data() + off(L);
        out.insert(out.end(), b, b + L.count[p] * elem);
      }
      return out;
    };
    b2dump::ResultSet r;
    r.neuron_count = m.neuron_count;
    r.final_time = m.run_start + m.run_duration;
    for (size_t p = 0; p < m.populations.size(); ++p) {
      const auto& def = m.populations[p];
      const PopDev& pd = pops[p];
      r.has_events |= !def.events.empty() || !def.event_monitors.empty();
      b2dump::PopulationResult pr;
      pr.count = def.count;
      pr.steps = def.steps;
      pr.record_count = def.monitor.record.size();
      pr.variable_count = def.monitor.variables.size();
      for (size_t v = 0; v < def.monitor.variables.size(); ++v) {
        b2dump::Column c;
        c.dtype = pd.mon_dtypes.empty() ? DType::F64 : pd.mon_dtypes[v];
        const size_t w = b2ir::dtype_bytes(c.dtype), nrec = def.monitor.record.size();
        if (world == 1) {
          if (pd.mon_records >= 0) c.bytes = read_bytes(pd.mon_samples[v], pd.mon_ticks * nrec * w);
        } else if (!pd.mon_dtypes.empty()) {
          // samples are [tick][record]; each rank holds its owned records
          c.bytes.assign(pd.mon_ticks * nrec * w, 0);
          for (int q = 0; q < world; ++q) {
            const StageLayout& L = lay[size_t(q)];
            const auto& pos = L.mon_positions[p];
            const uint8_t* b = stg[size_t(q)].data() + L.monitor[p][v];
            for (uint64_t row = 0; row < pd.mon_ticks; ++row)
              for (size_t j = 0; j < pos.size(); ++j)
                std::memcpy(&c.bytes[(row * nrec + pos[j]) * w], b + (row * pos.size() + j) * w, w);
          }
        }
        pr.samples.push_back(std::move(c));
      }
      uint64_t window_first = pd.end_tick - std::min<uint64_t>(def.monitor.window_steps, pd.end_tick);
      pr.event_history.resize(def.events.size());
      for (size_t e = 0; e < def.events.size(); ++e) {
        const EventStreamDev& es = streams[size_t(pd.stream_of_event[e])];
        for (size_t rel = 0; rel < steps; ++rel) {
          uint64_t tick = start_tick + rel;
          if (tick < window_first) continue;
          for (uint64_t x = es.starts[rel]; x < es.starts[rel + 1]; ++x)
            pr.event_history[e].push_back({tick, es.ids[x]});
        }
      }
      // EventMonitors: every tick's list of their event (no window), or the
      // previous tick's for a monitor scheduled before the event's producer
      for (size_t k = 0; k < def.event_monitors.size(); ++k) {
        b2dump::EventMonitorResult er;
        const int sid = k < pd.evmon_stream.size() ? pd.evmon_stream[k] : -1;
        if (sid >= 0) {
          const EventStreamDev& es = streams[size_t(sid)];
          const size_t lag = size_t(pd.evmon_lag[k]);
          for (size_t rel = lag; rel < steps; ++rel)
            for (uint64_t x = es.starts[rel - lag]; x < es.starts[rel - lag + 1]; ++x)
              er.events.push_back({start_tick + rel, es.ids[x]});
          check(er.events.size() <= 10'000'000, "EventMonitor recording budget exceeded");
          if (k < pd.evmon_vars.size())
            for (size_t v = 0; v < pd.evmon_vars[k].ring.size(); ++v) {
              b2dump::Column c;
              const std::string& vn = def.event_monitors[k].variables[v];
              c.dtype = DType::F64;
              for (const auto& st2 : def.states)
                if (st2.name == vn) c.dtype = st2.dtype;
              c.bytes = pd.evmon_vars[k].host[v];
              check(c.bytes.size() == er.events.size() * b2ir::dtype_bytes(c.dtype), "EventMonitor sample count mismatch");
              er.samples.push_back(std::move(c));
            }
        }
        pr.event_monitors.push_back(std::move(er));
      }
      pr.counts.assign(def.count, 0);
      auto spike_it = std::find(def.events.begin(), def.events.end(), "spike");
      if (spike_it != def.events.end()) {
        size_t e = size_t(spike_it - def.events.begin());
        const EventStreamDev& es = streams[size_t(pd.stream_of_event[e])];
        if (pd.has_spike_monitor) {
          pr.spikes = pr.event_history[e];
          for (const auto& sp : pr.spikes) pr.counts[sp.second]++;
        }
        if (steps > 0)
          for (uint64_t x = es.starts[steps - 1]; x < es.starts[steps]; ++x) pr.last_fired.push_back(es.ids[x]);
      }
      for (size_t s = 0; s < def.states.size(); ++s) {
        b2dump::Column c;
        c.dtype = def.states[s].dtype;
        c.bytes = pop_column(p, pd.states[s].ptr, b2ir::dtype_bytes(c.dtype), [p, s](const StageLayout& L) { return L.state[p][s]; });
        pr.states.push_back(std::move(c));
      }
      if (pd.lastspike >= 0) {
        pr.has_refractory = true;
        auto ls = pop_column(p, pd.lastspike, 8, [p](const StageLayout& L) { return L.lastspike[p]; });
        pr.lastspike.resize(def.count);
        std::memcpy(pr.lastspike.data(), ls.data(), ls.size());
        pr.not_refractory = pop_column(p, pd.not_refractory, 1, [p](const StageLayout& L) { return L.not_refractory[p]; });
      }
      r.populations.push_back(std::move(pr));
    }
    std::vector<uint64_t> delivered(std::max<size_t>(delivered_count, 1), 0);
    if (world == 1) {
      B2_CUDA(cudaMemcpy(delivered.data(), dptr(delivered_ptr), delivered.size() * 8, cudaMemcpyDeviceToHost));
    } else {
      for (int q = 0; q < world; ++q)
        for (size_t k = 0; k < delivered_count; ++k) {
          uint64_t x;
          std::memcpy(&x, stg[size_t(q)].data() + lay[size_t(q)].delivered + k * 8, 8);
          delivered[k] += x;
        }
    }
    for (size_t s = 0; s < m.synapses.size(); ++s) {
      const auto& def = m.synapses[s];
      const SynDev& sd = syns[s];
      b2dump::SynapseResult sr;
      sr.edge_count = sd.edges;
      for (size_t k = 0; k < def.states.size(); ++k) {
        b2dump::Column c;
        c.dtype = def.states[k].dtype;
        const size_t w = b2ir::dtype_bytes(c.dtype);
        if (world == 1) {
          c.bytes = read_bytes(sd.states[k].ptr, sd.edges * w);
        } else {
          // local edges back to global edge order
          c.bytes.assign(sd.edges * w, 0);
          for (int q = 0; q < world; ++q) {
            const StageLayout& L = lay[size_t(q)];
            const uint8_t* b = stg[size_t(q)].data() + L.syn_state[s][k];
            for (size_t j = 0; j < L.syn_edges[s].size(); ++j) std::memcpy(&c.bytes[size_t(L.syn_edges[s][j]) * w], b + j * w, w);
          }
        }
        sr.states.push_back(std::move(c));
      }
      for (const auto& pw : sd.pathways) sr.delivered += delivered[size_t(pw.delivered_slot)];
      r.synapses.push_back(std::move(sr));
    }
    return r;
  }

  void build() {
    auto t0 = std::chrono::steady_clock::now();
    check_capabilities();
    if (!opt.dry_run) {
      if (opt.device >= 0) B2_CUDA(cudaSetDevice(opt.device));
      B2_CUDA(cudaGetDevice(&device));
      B2_CUDA(cudaFree(nullptr));  // establish the primary context
      int sms = 0;
      B2_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
      if (sms > 0) sm_count_ = unsigned(sms);
      B2_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
      B2_CUDA(cudaEventCreate(&ev_start));
      B2_CUDA(cudaEventCreate(&ev_stop));
      ctl = DeviceBuffer(64);
      B2_CUDA(cudaMemsetAsync(ctl.ptr, 0, 64, stream));
    }
    build_populations();
    build_synapses();
    build_streams();
    build_plan();
    build_arena();
    compile_module();
    if (!opt.dry_run) B2_CUDA(cudaStreamSynchronize(stream));
    st.launches_per_tick = ops.size();
    st.build_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  }
};

// ------------------------------------------------------------------ facade
Engine::Engine(const b2ir::Model& model, const Options& options) : impl_(std::make_unique<Impl>(model, options)) {
  impl_->build();
}
Engine::~Engine() = default;
bool Engine::step(uint64_t max_ticks) { return impl_->step(max_ticks); }
bool Engine::finished() const { return impl_->cur_rel >= impl_->steps; }
b2dump::ResultSet Engine::results() { return impl_->results(); }
Stats Engine::stats() const {
  Stats s = impl_->st;
  uint64_t spikes = 0;
  for (const auto& es : impl_->streams) spikes += es.ids.size();
  s.spikes = spikes;
  if (!impl_->opt.dry_run && impl_->delivered_ptr >= 0 && impl_->delivered_count) {
    std::vector<uint64_t> d(impl_->delivered_count);
    if (cudaMemcpy(d.data(), impl_->dptr(impl_->delivered_ptr), d.size() * 8, cudaMemcpyDeviceToHost) == cudaSuccess)
      for (auto x : d) s.synaptic_events += x;
  }
  return s;
}
const std::string& Engine::generated_source() const { return impl_->source; }

void Engine::read_state(size_t population, const std::string& name, std::vector<uint8_t>& out) {
  check(population < impl_->m.populations.size(), "population index out of range");
  if (!impl_->opt.dry_run && !impl_->failed) impl_->flush_deferred();
  const auto& def = impl_->m.populations[population];
  for (size_t s = 0; s < def.states.size(); ++s)
    if (def.states[s].name == name) {
      out = impl_->read_bytes(impl_->pops[population].states[s].ptr,
                              impl_->pops[population].count * b2ir::dtype_bytes(def.states[s].dtype));
      return;
    }
  throw Error("unknown state '" + name + "'");
}

std::vector<KernelTime> Engine::profile(uint64_t ticks) { return impl_->profile(ticks); }
std::vector<uint8_t> Engine::ipc_handle() const { return impl_->ipc_handle(); }
void Engine::connect(const std::vector<std::vector<uint8_t>>& handles) { impl_->connect(handles); }
void Engine::publish() { impl_->publish(); }
std::pair<uint64_t, uint64_t> Engine::owned_range(size_t population) const {
  check(population < impl_->m.populations.size(), "population index out of range");
  const auto& pd = impl_->pops[population];
  return {pd.lo, pd.lo + pd.count};
}

std::vector<uint32_t> Engine::spikes_at(size_t population, uint64_t tick) const {
  check(population < impl_->m.populations.size(), "population index out of range");
  const auto& def = impl_->m.populations[population];
  auto it = std::find(def.events.begin(), def.events.end(), "spike");
  check(it != def.events.end(), "population has no spike event");
  const auto& es = impl_->streams[size_t(impl_->pops[population].stream_of_event[size_t(it - def.events.begin())])];
  check(tick >= impl_->start_tick && tick - impl_->start_tick + 1 < es.starts.size(), "tick not simulated yet");
  size_t rel = tick - impl_->start_tick;
  return std::vector<uint32_t>(es.ids.begin() + long(es.starts[rel]), es.ids.begin() + long(es.starts[rel + 1]));
}

}  // namespace b2gpu
