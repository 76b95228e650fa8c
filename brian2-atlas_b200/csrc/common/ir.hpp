// AtlasIR `atlasir-v1` document model: the subset of the wire contract that the
// per-tick simulation path consumes.
//
// Field names and meanings follow the Rust reader in
// brian2-rust/src/model.rs:29-650 (Model, Definition, PopulationDefinition,
// SynapseDefinition, CodeObjectSpec, Statement, Expr, Instance, Run).  Model
// floats arrive as IEEE-754 bit strings (model.rs:860-937) and are decoded to
// exact binary values here; nothing is parsed through decimal text.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

namespace b2ir {

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

inline void check(bool ok, const std::string& message) {
  if (!ok) throw Error(message);
}

// Storage and logical expression dtypes (model.rs:296-309).
enum class DType : uint8_t { F32, F64, I32, I64, U32, U64, Bool, Index, Tick };

DType parse_dtype(const std::string& s);
const char* dtype_name(DType d);
inline bool is_integer(DType d) {
  return d == DType::I32 || d == DType::I64 || d == DType::U32 || d == DType::U64;
}
size_t dtype_bytes(DType d);  // storage width of a public dtype

enum class IndexDomain : uint8_t { Scalar, Neuron, Synapse };

// Expression operators, one per `op` tag of the Expr enum (model.rs:643-848).
enum class Op : uint8_t {
  Literal, Boolean, Integer, Cast, Rand, Randn, Binomial, Poisson, TimedArray,
  BoolToF64, IndexToF64, TickToF64, F32ToF64, F64ToF32, Timestep, TickOffset, Load, Call,
  Neg, Not, Abs, Arccos, Arcsin, Arctan, Ceil, Cos, Cosh, Exp, Expm1, Exprel, Floor, Trunc,
  Log, Log10, Log1p, Sign, Sin, Sinh, Sqrt, Tan, Tanh,
  Add, Sub, Mul, Div, Pow, Mod, FloorDiv, Eq, Ne, Gt, Ge, Lt, Le, And, Or, Clip,
};
const char* op_name(Op op);
bool is_unary_math(Op op);   // Neg .. Tanh
bool is_binary(Op op);       // Add .. Or

struct Expr;
using ExprPtr = std::shared_ptr<const Expr>;

struct Expr {
  Op op = Op::Literal;
  // Children in wire order: {arg} | {left,right} | {value,min,max} | {p} |
  // {lambda} | {time[,index]} | {tick} | call arguments.
  std::vector<ExprPtr> args;
  double literal = 0.0;        // Literal (decoded f64)
  uint64_t raw = 0;            // Integer: two's-complement bits widened as the
                               // reference register holds them (i32 -> u32 -> u64)
  DType dtype = DType::F64;    // Integer / Cast target dtype
  bool boolean = false;        // Boolean
  uint64_t stream = 0;         // Rand / Randn / Binomial / Poisson
  uint64_t n = 0;              // Binomial trials
  bool approximate = false;    // Binomial normal approximation switch
  int64_t offset = 0;          // TickOffset
  std::string name;            // Load symbol / Call function
  // TimedArray
  std::vector<double> ta_values;
  size_t ta_rows = 0;
  int64_t ta_columns = -1;     // -1: one-dimensional
  double ta_epsilon = 0.0;
  size_t ta_upsampling = 1;
};

struct Statement {
  std::string target;
  DType dtype = DType::F64;
  ExprPtr value;
  std::optional<std::string> condition;
};

struct Symbol {
  std::string name;
  DType dtype = DType::F64;
  IndexDomain index_domain = IndexDomain::Neuron;
};

struct Effects {
  std::vector<std::string> reads, writes;
};

struct CodeObject {
  std::string name, kind, when;
  int32_t order = 0;
  size_t clock = 0;
  std::string iteration_domain;
  std::vector<Statement> scalar, vector;
  Effects effects;
  std::optional<std::string> summed_target, summed_state, pathway_name, event_name;
  bool adaptive = false;  // adaptive integrators are not on this path
};

struct Refractory {
  std::vector<std::string> frozen_states;
  std::string mode;
};

struct StateMonitor {
  std::string name;
  std::vector<std::string> variables;
  std::vector<size_t> record;
  size_t clock = 0;
};

struct EventMonitor {
  std::string name, event;
  std::vector<std::string> variables;
  size_t clock = 0;
};

struct MonitorSpec {
  std::vector<std::string> variables;
  std::vector<size_t> record;
  size_t window_steps = 0;
};

struct PopulationDef {
  std::string name;
  size_t offset = 0, count = 0;
  std::vector<Symbol> states, parameters;
  size_t linked_variable_count = 0;
  bool spatial = false;
  std::optional<Refractory> refractory;
  std::vector<std::string> events;
  std::vector<CodeObject> code_objects;
  std::vector<StateMonitor> state_monitors;
  std::vector<EventMonitor> event_monitors;
  std::optional<std::string> spike_monitor;
  size_t rate_monitor_count = 0;
  MonitorSpec monitor;
  size_t clock = 0;
  double dt = 0.0;
  size_t steps = 0;
};

struct SynapseDef {
  std::string name;
  std::vector<Symbol> states;
  std::vector<std::string> clock_driven_states;
  std::vector<Symbol> parameters;
  size_t linked_variable_count = 0;
  std::map<std::string, std::string> pre_state_aliases, post_state_aliases;
  size_t source_population = 0, target_population = 0;
  std::optional<size_t> source_synapse, target_synapse;
  size_t source_start = 0, target_start = 0, source_count = 0, target_count = 0;
  std::vector<CodeObject> code_objects;
  size_t state_monitor_count = 0;
};

struct FunctionArg {
  std::string name;
  DType dtype = DType::F64;
};

struct Function {
  std::string name;
  std::vector<FunctionArg> arguments;
  DType return_dtype = DType::F64;
  ExprPtr body;  // portable body; null for native-only functions
};

enum class ScheduleOp : uint8_t { CodeObject, StateMonitor, SpikeMonitor, EventMonitor, EventSource };
enum class OwnerKind : uint8_t { Population, Synapse };

struct ScheduleNode {
  std::string id;
  ScheduleOp operation = ScheduleOp::CodeObject;
  OwnerKind owner_kind = OwnerKind::Population;
  size_t owner_index = 0, item_index = 0, clock = 0;
  std::string when;
  int32_t order = 0;
  std::string name;
  Effects effects;
};

struct Clock {
  std::string name;
  double dt = 0.0;
};

// Typed array as it arrives on the wire: raw bit patterns, one per element.
// f64 -> bits, f32 -> u32 bits, ints -> two's complement, bool -> 0/1.
struct EncodedArray {
  DType dtype = DType::F64;
  std::vector<uint64_t> raw;
  double as_f64(size_t i) const;  // decode_typed_float semantics (model.rs:883)
  size_t size() const { return raw.size(); }
};

struct RefractoryInstance {
  double period = 0.0;
  uint64_t period_ticks = 0;
  std::vector<double> initial_lastspike;
  std::vector<uint8_t> initial_not_refractory;
};

struct SpikeGenerator {
  std::vector<size_t> spike_ticks, spike_indices;
};

struct PopulationInstance {
  std::map<std::string, EncodedArray> initial_state, parameters;
  std::optional<RefractoryInstance> refractory;
  std::optional<SpikeGenerator> spike_generator;
};

struct Initializer {
  enum class Kind : uint8_t { ClippedNormal, Uniform } kind = Kind::Uniform;
  double mean = 0.0, std = 0.0;
  std::optional<double> minimum, maximum;
  uint64_t stream = 0;
};

struct Topology {
  enum class Kind : uint8_t { Explicit, FixedTotal, FixedIndegree, BinaryCsr } kind = Kind::Explicit;
  uint64_t edge_count = 0, indegree = 0, seed = 0;
  std::map<std::string, Initializer> initializers;
  // binary_csr: external B2CSR001 file, its SHA-256 and the per-edge
  // parameter -> value column mapping
  std::string path, sha256;
  uint64_t column_count = 0;
  std::map<std::string, uint64_t> columns;
};

// A B2CSR001 source-major graph (brian2-rust/src/binary_topology.rs): the
// header (magic, sources, targets, edges, columns as u64 LE), sources + 1 u64
// row offsets, edges u32 targets in creation order, then `columns` f64
// columns of per-edge values.  Shape, length, checksum and contents are
// validated with the reference's messages; arrays are filled only when
// `materialize` is set.
struct BinaryCsr {
  std::vector<uint32_t> source, target;
  std::vector<std::vector<double>> columns;
};
BinaryCsr read_binary_csr(const std::string& path, uint64_t sources, uint64_t targets, uint64_t edges,
                          uint64_t columns, const std::string& sha256, bool materialize);

struct PendingEvent {
  size_t delivery_tick = 0, item = 0;
};

struct PathwayInstance {
  std::string name, kind, event;
  std::vector<double> delay;
  std::vector<size_t> delay_ticks;
  std::optional<Initializer> delay_initializer;
  std::vector<PendingEvent> pending;
};

struct SynapseInstance {
  std::vector<uint32_t> source, target;  // explicit topology, creation order
  Topology topology;
  std::map<std::string, EncodedArray> initial_state, parameters;
  std::vector<PathwayInstance> pathways;
  size_t edge_count() const {
    return topology.kind == Topology::Kind::Explicit ? source.size() : size_t(topology.edge_count);
  }
};

struct RunClock {
  size_t start_tick = 0, steps = 0;
};

struct Model {
  std::string schema;
  std::vector<PopulationDef> populations;
  std::vector<SynapseDef> synapses;
  std::vector<Clock> clocks;
  std::vector<Function> functions;
  std::vector<ScheduleNode> schedule;
  size_t neuron_count = 0;
  uint64_t rng_seed = 0;
  std::vector<PopulationInstance> population_instances;
  std::vector<SynapseInstance> synapse_instances;
  double run_start = 0.0, run_duration = 0.0;
  std::vector<RunClock> run_clocks;
};

// Parse an atlasir-v1 (or the legacy b2ir-v1 envelope, whose layers are
// identical) document.  Throws b2ir::Error with a one-line message.
Model load_model(const char* json, size_t size);
Model load_model_file(const std::string& path);

// Hex-bit decoders (model.rs:860-937).
double decode_f64_bits(const std::string& bits);
float decode_f32_bits(const std::string& bits);
uint64_t decode_raw(const std::string& bits, DType dtype);  // register raw bits
double decode_typed_float(const std::string& bits, DType dtype);

// Brian2 timestep(): floor((t + 1e-3 dt) / dt) (model.rs:981-992).
uint64_t timestep(double time, double dt);

}  // namespace b2ir
