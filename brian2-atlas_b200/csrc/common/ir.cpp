// AtlasIR loader: JSON DOM -> b2ir::Model.
//
// Follows the serde layout of brian2-rust/src/model.rs:29-650.  Unknown keys are
// tolerated (the reference rejects them; this loader is a consumer of documents
// the reference producer wrote).  The legacy `b2ir-v1` envelope is accepted
// as-is because its layers are byte-identical to atlasir-v1
// (model.rs:4719-4730 `prepare_protocol`).
#include "ir.hpp"

#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstring>
#include <fstream>
#include <set>
#include <sstream>

#include "canonical.hpp"
#include "json.hpp"

namespace b2ir {

using b2json::Value;

DType parse_dtype(const std::string& s) {
  if (s == "f32") return DType::F32;
  if (s == "f64") return DType::F64;
  if (s == "i32") return DType::I32;
  if (s == "i64") return DType::I64;
  if (s == "u32") return DType::U32;
  if (s == "u64") return DType::U64;
  if (s == "bool") return DType::Bool;
  if (s == "index") return DType::Index;
  if (s == "tick") return DType::Tick;
  throw Error("unknown dtype '" + s + "'");
}

const char* dtype_name(DType d) {
  switch (d) {
    case DType::F32: return "f32";
    case DType::F64: return "f64";
    case DType::I32: return "i32";
    case DType::I64: return "i64";
    case DType::U32: return "u32";
    case DType::U64: return "u64";
    case DType::Bool: return "bool";
    case DType::Index: return "index";
    case DType::Tick: return "tick";
  }
  return "?";
}

size_t dtype_bytes(DType d) {
  switch (d) {
    case DType::Bool: return 1;
    case DType::F32: case DType::I32: case DType::U32: return 4;
    case DType::F64: case DType::I64: case DType::U64: return 8;
    default: throw Error("logical dtype has no storage width");
  }
}

namespace {

struct OpName {
  const char* name;
  Op op;
};

const OpName kOps[] = {
    {"literal", Op::Literal}, {"boolean", Op::Boolean}, {"integer", Op::Integer},
    {"cast", Op::Cast}, {"rand", Op::Rand}, {"randn", Op::Randn}, {"binomial", Op::Binomial},
    {"poisson", Op::Poisson}, {"timed_array", Op::TimedArray}, {"bool_to_f64", Op::BoolToF64},
    {"index_to_f64", Op::IndexToF64}, {"tick_to_f64", Op::TickToF64},
    {"f32_to_f64", Op::F32ToF64}, {"f64_to_f32", Op::F64ToF32}, {"timestep", Op::Timestep},
    {"tick_offset", Op::TickOffset}, {"load", Op::Load}, {"call", Op::Call}, {"neg", Op::Neg},
    {"not", Op::Not}, {"abs", Op::Abs}, {"arccos", Op::Arccos}, {"arcsin", Op::Arcsin},
    {"arctan", Op::Arctan}, {"ceil", Op::Ceil}, {"cos", Op::Cos}, {"cosh", Op::Cosh},
    {"exp", Op::Exp}, {"expm1", Op::Expm1}, {"exprel", Op::Exprel}, {"floor", Op::Floor},
    {"trunc", Op::Trunc}, {"log", Op::Log}, {"log10", Op::Log10}, {"log1p", Op::Log1p},
    {"sign", Op::Sign}, {"sin", Op::Sin}, {"sinh", Op::Sinh}, {"sqrt", Op::Sqrt},
    {"tan", Op::Tan}, {"tanh", Op::Tanh}, {"add", Op::Add}, {"sub", Op::Sub}, {"mul", Op::Mul},
    {"div", Op::Div}, {"pow", Op::Pow}, {"mod", Op::Mod}, {"floor_div", Op::FloorDiv},
    {"eq", Op::Eq}, {"ne", Op::Ne}, {"gt", Op::Gt}, {"ge", Op::Ge}, {"lt", Op::Lt},
    {"le", Op::Le}, {"and", Op::And}, {"or", Op::Or}, {"clip", Op::Clip},
};

Op parse_op(const std::string& s) {
  for (const auto& e : kOps)
    if (s == e.name) return e.op;
  throw Error("unknown expression op '" + s + "'");
}

bool is_hex_lower(const std::string& s, size_t len) {
  if (s.size() != len) return false;
  for (char c : s)
    if (!((c >= '0' && c <= '9') || (c >= 'a' && c <= 'f'))) return false;
  return true;
}

uint64_t parse_hex(const std::string& s) {
  uint64_t v = 0;
  for (char c : s) v = (v << 4) | uint64_t(c <= '9' ? c - '0' : c - 'a' + 10);
  return v;
}

std::string str(const Value& v, const char* key) { return v.at(key).str(); }
size_t usz(const Value& v, const char* key) { return size_t(v.at(key).u64()); }

std::optional<std::string> opt_str(const Value& v, const char* key) {
  if (v.absent(key)) return std::nullopt;
  return v.at(key).str();
}

std::vector<std::string> str_list(const Value& v) {
  std::vector<std::string> out;
  for (const auto& x : v.arr()) out.push_back(x.str());
  return out;
}

std::vector<size_t> size_list(const Value& v) {
  std::vector<size_t> out;
  out.reserve(v.arr().size());
  for (const auto& x : v.arr()) out.push_back(size_t(x.u64()));
  return out;
}

ExprPtr parse_expr(const Value& v, int depth = 0);

ExprPtr child(const Value& v, const char* key, int depth) { return parse_expr(v.at(key), depth + 1); }

ExprPtr parse_expr(const Value& v, int depth) {
  check(depth < 4096, "expression nesting too deep");
  auto e = std::make_shared<Expr>();
  e->op = parse_op(str(v, "op"));
  switch (e->op) {
    case Op::Literal: e->literal = decode_f64_bits(str(v, "bits")); break;
    case Op::Boolean: e->boolean = v.at("value").boolean(); break;
    case Op::Integer: {
      e->dtype = parse_dtype(str(v, "dtype"));
      const std::string& text = str(v, "value");
      check(is_integer(e->dtype) && !text.empty(), "invalid integer literal dtype");
      errno = 0;
      switch (e->dtype) {
        case DType::I32: {
          long long x = std::stoll(text);
          check(x >= INT32_MIN && x <= INT32_MAX, "i32 literal out of range");
          e->raw = uint64_t(uint32_t(int32_t(x)));
          break;
        }
        case DType::I64: e->raw = uint64_t(int64_t(std::stoll(text))); break;
        case DType::U32: {
          unsigned long long x = std::stoull(text);
          check(text[0] != '-' && x <= UINT32_MAX, "u32 literal out of range");
          e->raw = x;
          break;
        }
        case DType::U64:
          check(text[0] != '-', "u64 literal out of range");
          e->raw = std::stoull(text);
          break;
        default: break;
      }
      break;
    }
    case Op::Cast:
      e->dtype = parse_dtype(str(v, "dtype"));
      e->args.push_back(child(v, "arg", depth));
      break;
    case Op::Rand:
    case Op::Randn: e->stream = v.at("stream").u64(); break;
    case Op::Binomial:
      e->stream = v.at("stream").u64();
      e->n = v.at("n").u64();
      e->approximate = v.at("approximate").boolean();
      e->args.push_back(child(v, "p", depth));
      break;
    case Op::Poisson:
      e->stream = v.at("stream").u64();
      e->args.push_back(child(v, "lambda", depth));
      break;
    case Op::TimedArray:
      for (const auto& x : v.at("values").arr()) e->ta_values.push_back(decode_f64_bits(x.str()));
      e->ta_rows = usz(v, "rows");
      e->ta_columns = v.absent("columns") ? -1 : int64_t(v.at("columns").u64());
      e->ta_epsilon = decode_f64_bits(str(v, "epsilon"));
      e->ta_upsampling = usz(v, "upsampling");
      e->args.push_back(child(v, "time", depth));
      if (!v.absent("index")) e->args.push_back(child(v, "index", depth));
      break;
    case Op::Timestep:
      e->args.push_back(child(v, "time", depth));
      e->args.push_back(child(v, "dt", depth));
      break;
    case Op::TickOffset:
      e->offset = v.at("offset").i64();
      e->args.push_back(child(v, "tick", depth));
      break;
    case Op::Load: e->name = str(v, "name"); break;
    case Op::Call:
      e->name = str(v, "function");
      for (const auto& a : v.at("arguments").arr()) e->args.push_back(parse_expr(a, depth + 1));
      break;
    case Op::Clip:
      e->args.push_back(child(v, "value", depth));
      e->args.push_back(child(v, "min", depth));
      e->args.push_back(child(v, "max", depth));
      break;
    default:
      if (is_binary(e->op)) {
        e->args.push_back(child(v, "left", depth));
        e->args.push_back(child(v, "right", depth));
      } else {
        e->args.push_back(child(v, "arg", depth));
      }
  }
  return e;
}

std::vector<Statement> parse_statements(const Value& v) {
  std::vector<Statement> out;
  for (const auto& s : v.arr()) {
    Statement st;
    st.target = str(s, "target");
    st.dtype = parse_dtype(str(s, "dtype"));
    st.value = parse_expr(s.at("value"));
    st.condition = opt_str(s, "condition");
    out.push_back(std::move(st));
  }
  return out;
}

Effects parse_effects(const Value& v) {
  Effects e;
  e.reads = str_list(v.at("reads"));
  e.writes = str_list(v.at("writes"));
  return e;
}

CodeObject parse_code(const Value& v) {
  CodeObject c;
  c.name = str(v, "name");
  c.kind = str(v, "kind");
  c.when = str(v, "when");
  c.order = int32_t(v.at("order").i64());
  c.clock = usz(v, "clock");
  c.iteration_domain = str(v, "iteration_domain");
  c.scalar = parse_statements(v.at("scalar"));
  c.vector = parse_statements(v.at("vector"));
  c.effects = parse_effects(v.at("effects"));
  c.summed_target = opt_str(v, "summed_target");
  c.summed_state = opt_str(v, "summed_state");
  c.pathway_name = opt_str(v, "pathway_name");
  c.event_name = opt_str(v, "event_name");
  c.adaptive = !v.absent("adaptive");
  return c;
}

std::vector<Symbol> parse_symbols(const Value& v) {
  std::vector<Symbol> out;
  for (const auto& s : v.arr()) {
    Symbol sym;
    sym.name = str(s, "name");
    sym.dtype = parse_dtype(str(s, "dtype"));
    const std::string& d = str(s, "index_domain");
    sym.index_domain = d == "scalar" ? IndexDomain::Scalar
                       : d == "neuron" ? IndexDomain::Neuron
                       : d == "synapse" ? IndexDomain::Synapse
                                        : throw Error("unknown index domain '" + d + "'");
    out.push_back(sym);
  }
  return out;
}

EncodedArray decode_array(const Value& v, DType dtype) {
  EncodedArray a;
  a.dtype = dtype;
  const auto& items = v.arr();
  a.raw.resize(items.size());
  for (size_t i = 0; i < items.size(); ++i) {
    const std::string& s = items[i].str();
    if (i > 0 && s == items[i - 1].str()) {
      a.raw[i] = a.raw[i - 1];
      continue;
    }
    a.raw[i] = decode_raw(s, dtype);
  }
  return a;
}

const Symbol* find_symbol(const std::vector<Symbol>& a, const std::vector<Symbol>& b,
                          const std::string& name) {
  for (const auto& s : a)
    if (s.name == name) return &s;
  for (const auto& s : b)
    if (s.name == name) return &s;
  return nullptr;
}

std::map<std::string, EncodedArray> decode_table(const Value& v, const std::vector<Symbol>& a,
                                                 const std::vector<Symbol>& b) {
  std::map<std::string, EncodedArray> out;
  for (const auto& kv : v.obj()) {
    const Symbol* sym = find_symbol(a, b, kv.first);
    check(sym != nullptr, "instance array '" + kv.first + "' has no symbol");
    out.emplace(kv.first, decode_array(kv.second, sym->dtype));
  }
  return out;
}

Initializer parse_initializer(const Value& v) {
  Initializer init;
  const std::string& kind = str(v, "kind");
  init.stream = v.at("stream").u64();
  if (kind == "clipped_normal") {
    init.kind = Initializer::Kind::ClippedNormal;
    init.mean = decode_f64_bits(str(v, "mean"));
    init.std = decode_f64_bits(str(v, "std"));
    if (!v.absent("minimum")) init.minimum = decode_f64_bits(str(v, "minimum"));
    if (!v.absent("maximum")) init.maximum = decode_f64_bits(str(v, "maximum"));
    check(init.std >= 0.0 && (!init.minimum || !init.maximum || *init.minimum <= *init.maximum),
          "invalid clipped-normal initializer");
  } else if (kind == "uniform") {
    init.kind = Initializer::Kind::Uniform;
    init.minimum = decode_f64_bits(str(v, "minimum"));
    init.maximum = decode_f64_bits(str(v, "maximum"));
    check(*init.minimum <= *init.maximum, "invalid uniform initializer");
  } else {
    throw Error("unknown initializer kind '" + kind + "'");
  }
  return init;
}

Topology parse_topology(const Value& v) {
  Topology t;
  const std::string& kind = str(v, "kind");
  if (kind == "explicit") {
    t.kind = Topology::Kind::Explicit;
    return t;
  }
  if (kind == "binary_csr") {
    t.kind = Topology::Kind::BinaryCsr;
    t.edge_count = v.at("edge_count").u64();
    t.path = str(v, "path");
    t.sha256 = str(v, "sha256");
    t.column_count = v.at("column_count").u64();
    for (const auto& kv : v.at("initializers").obj()) t.columns[kv.first] = kv.second.u64();
    return t;
  }
  t.kind = kind == "fixed_total" ? Topology::Kind::FixedTotal
           : kind == "fixed_indegree" ? Topology::Kind::FixedIndegree
                                      : throw Error("unknown topology kind '" + kind + "'");
  t.edge_count = v.at("edge_count").u64();
  t.seed = v.at("seed").u64();
  if (t.kind == Topology::Kind::FixedIndegree) t.indegree = v.at("indegree").u64();
  for (const auto& kv : v.at("initializers").obj())
    t.initializers.emplace(kv.first, parse_initializer(kv.second));
  return t;
}

ScheduleOp parse_schedule_op(const std::string& s) {
  if (s == "code_object") return ScheduleOp::CodeObject;
  if (s == "state_monitor") return ScheduleOp::StateMonitor;
  if (s == "spike_monitor") return ScheduleOp::SpikeMonitor;
  if (s == "event_monitor") return ScheduleOp::EventMonitor;
  if (s == "event_source") return ScheduleOp::EventSource;
  throw Error("unknown schedule operation '" + s + "'");
}

}  // namespace

const char* op_name(Op op) {
  for (const auto& e : kOps)
    if (e.op == op) return e.name;
  return "?";
}

bool is_unary_math(Op op) { return op >= Op::Neg && op <= Op::Tanh; }
bool is_binary(Op op) { return op >= Op::Add && op <= Op::Or; }

double decode_f64_bits(const std::string& bits) {
  check(is_hex_lower(bits, 16), "f64 must be 16 lowercase hex digits (IEEE-754 bits)");
  uint64_t raw = parse_hex(bits);
  double v;
  std::memcpy(&v, &raw, 8);
  check(std::isfinite(v), "non-finite numeric value");
  return v;
}

float decode_f32_bits(const std::string& bits) {
  check(is_hex_lower(bits, 8), "f32 must be 8 lowercase hex digits (IEEE-754 bits)");
  uint32_t raw = uint32_t(parse_hex(bits));
  float v;
  std::memcpy(&v, &raw, 4);
  check(std::isfinite(v), "non-finite numeric value");
  return v;
}

uint64_t decode_raw(const std::string& bits, DType dtype) {
  switch (dtype) {
    case DType::F64: {
      double v = decode_f64_bits(bits);
      uint64_t raw;
      std::memcpy(&raw, &v, 8);
      return raw;
    }
    case DType::F32: {
      float v = decode_f32_bits(bits);
      uint32_t raw;
      std::memcpy(&raw, &v, 4);
      return raw;
    }
    case DType::Bool:
      check(bits == "00" || bits == "01", "bool must be encoded as 00 or 01");
      return bits == "01" ? 1 : 0;
    case DType::I32:
    case DType::U32:
      check(is_hex_lower(bits, 8), "32-bit integer must be 8 lowercase hex digits");
      return parse_hex(bits);
    case DType::I64:
    case DType::U64:
      check(is_hex_lower(bits, 16), "64-bit integer must be 16 lowercase hex digits");
      return parse_hex(bits);
    default: throw Error("numeric array requires a public storage dtype");
  }
}

double decode_typed_float(const std::string& bits, DType dtype) {
  EncodedArray a;
  a.dtype = dtype;
  a.raw.push_back(decode_raw(bits, dtype));
  return a.as_f64(0);
}

double EncodedArray::as_f64(size_t i) const {
  uint64_t r = raw[i];
  double v;
  switch (dtype) {
    case DType::F64: std::memcpy(&v, &r, 8); return v;
    case DType::F32: {
      uint32_t r32 = uint32_t(r);
      float f;
      std::memcpy(&f, &r32, 4);
      return double(f);
    }
    case DType::Bool: return r ? 1.0 : 0.0;
    default:
      // Integer parameters become registers holding their raw bit pattern
      // (decode_typed_float, model.rs:904-927).
      std::memcpy(&v, &r, 8);
      return v;
  }
}

uint64_t timestep(double time, double dt) {
  double steps = (time + 1e-3 * dt) / dt;
  check(time >= 0.0 && std::isfinite(dt) && dt > 0.0 && std::isfinite(steps) &&
            steps < 9223372036854775808.0,
        "timestep outside Brian2 int64 range");
  return uint64_t(steps);
}

Model load_model(const char* json, size_t size) {
  Value doc;
  try {
    doc = b2json::parse(json, size);
  } catch (const b2json::Error& e) {
    throw Error(e.what());
  }
  try {
    Model m;
    // the probe predecessors are migrated (and their envelopes checked) on
    // entry, like the legacy b2ir-v1 envelope below
    b2canon::migrate_probe(doc);
    m.schema = str(doc, "schema");
    check(m.schema == "atlasir-v1" || m.schema == "b2ir-v1",
          "unsupported AtlasIR schema '" + m.schema + "'");
    // prepare_protocol (model.rs:4719-4730) verifies a legacy envelope's
    // hashes before migrating it
    if (m.schema == "b2ir-v1") b2canon::verify_protocol(doc);
    const Value& d = doc.at("definition");
    check(str(d, "numeric_profile") == "reference-f64", "unsupported numeric profile");
    check(str(d, "rng_algorithm") == "splitmix64-counter-v1", "unsupported RNG algorithm");
    for (const auto& c : d.at("clocks").arr()) m.clocks.push_back({str(c, "name"), decode_f64_bits(str(c, "dt"))});
    for (const auto& f : d.at("functions").arr()) {
      Function fn;
      fn.name = str(f, "name");
      for (const auto& a : f.at("arguments").arr())
        fn.arguments.push_back({str(a, "name"), parse_dtype(str(a, "dtype"))});
      fn.return_dtype = parse_dtype(str(f, "return_dtype"));
      if (!f.absent("body")) fn.body = parse_expr(f.at("body"));
      m.functions.push_back(std::move(fn));
    }
    for (const auto& p : d.at("populations").arr()) {
      PopulationDef pd;
      pd.name = str(p, "name");
      pd.offset = usz(p, "offset");
      pd.count = usz(p, "count");
      pd.states = parse_symbols(p.at("states"));
      pd.parameters = parse_symbols(p.at("parameters"));
      if (const Value* lv = p.find("linked_variables")) pd.linked_variable_count = lv->arr().size();
      pd.spatial = !p.absent("spatial");
      if (!p.absent("refractory")) {
        const Value& r = p.at("refractory");
        pd.refractory = Refractory{str_list(r.at("frozen_states")), str(r, "mode")};
      }
      pd.events = str_list(p.at("events"));
      for (const auto& c : p.at("code_objects").arr()) pd.code_objects.push_back(parse_code(c));
      for (const auto& s : p.at("state_monitors").arr()) {
        StateMonitor sm;
        sm.name = str(s, "name");
        sm.variables = str_list(s.at("variables"));
        sm.record = size_list(s.at("record"));
        sm.clock = usz(s, "clock");
        pd.state_monitors.push_back(std::move(sm));
      }
      for (const auto& s : p.at("event_monitors").arr()) {
        EventMonitor em;
        em.name = str(s, "name");
        em.event = str(s, "event");
        em.variables = str_list(s.at("variables"));
        em.clock = usz(s, "clock");
        pd.event_monitors.push_back(std::move(em));
      }
      pd.spike_monitor = opt_str(p, "spike_monitor");
      if (const Value* rm = p.find("rate_monitors")) pd.rate_monitor_count = rm->arr().size();
      const Value& mon = p.at("monitor");
      pd.monitor.variables = str_list(mon.at("variables"));
      pd.monitor.record = size_list(mon.at("record"));
      pd.monitor.window_steps = usz(mon, "window_steps");
      pd.clock = usz(p, "clock");
      pd.dt = decode_f64_bits(str(p, "dt"));
      pd.steps = usz(p, "steps");
      m.populations.push_back(std::move(pd));
    }
    for (const auto& s : d.at("synapses").arr()) {
      SynapseDef sd;
      sd.name = str(s, "name");
      sd.states = parse_symbols(s.at("states"));
      sd.clock_driven_states = str_list(s.at("clock_driven_states"));
      sd.parameters = parse_symbols(s.at("parameters"));
      if (const Value* lv = s.find("linked_variables")) sd.linked_variable_count = lv->arr().size();
      for (const auto& kv : s.at("pre_state_aliases").obj()) sd.pre_state_aliases[kv.first] = kv.second.str();
      for (const auto& kv : s.at("post_state_aliases").obj()) sd.post_state_aliases[kv.first] = kv.second.str();
      sd.source_population = usz(s, "source_population");
      sd.target_population = usz(s, "target_population");
      if (!s.absent("source_synapse")) sd.source_synapse = usz(s, "source_synapse");
      if (!s.absent("target_synapse")) sd.target_synapse = usz(s, "target_synapse");
      sd.source_start = usz(s, "source_start");
      sd.target_start = usz(s, "target_start");
      sd.source_count = usz(s, "source_count");
      sd.target_count = usz(s, "target_count");
      for (const auto& c : s.at("code_objects").arr()) sd.code_objects.push_back(parse_code(c));
      if (const Value* sm = s.find("state_monitors")) sd.state_monitor_count = sm->arr().size();
      m.synapses.push_back(std::move(sd));
    }
    for (const auto& n : d.at("schedule").at("nodes").arr()) {
      ScheduleNode node;
      node.id = str(n, "id");
      node.operation = parse_schedule_op(str(n, "operation"));
      const std::string& owner = str(n, "owner_kind");
      node.owner_kind = owner == "population" ? OwnerKind::Population
                        : owner == "synapse" ? OwnerKind::Synapse
                                             : throw Error("unknown schedule owner '" + owner + "'");
      node.owner_index = usz(n, "owner_index");
      node.item_index = usz(n, "item_index");
      node.clock = usz(n, "clock");
      node.when = str(n, "when");
      node.order = int32_t(n.at("order").i64());
      node.name = str(n, "name");
      node.effects = parse_effects(n.at("effects"));
      m.schedule.push_back(std::move(node));
    }

    const Value& inst = doc.at("instance");
    m.neuron_count = usz(inst, "neuron_count");
    m.rng_seed = inst.at("rng_seed").u64();
    const auto& pops = inst.at("populations").arr();
    check(pops.size() == m.populations.size(), "population instance count mismatch");
    for (size_t pi = 0; pi < pops.size(); ++pi) {
      const Value& p = pops[pi];
      const PopulationDef& pd = m.populations[pi];
      PopulationInstance pin;
      pin.initial_state = decode_table(p.at("initial_state"), pd.states, {});
      pin.parameters = decode_table(p.at("parameters"), pd.parameters, {});
      if (!p.absent("refractory")) {
        const Value& r = p.at("refractory");
        RefractoryInstance ri;
        ri.period = decode_f64_bits(str(r, "period"));
        ri.period_ticks = r.at("period_ticks").u64();
        for (const auto& x : r.at("initial_lastspike").arr()) ri.initial_lastspike.push_back(decode_f64_bits(x.str()));
        for (const auto& x : r.at("initial_not_refractory").arr()) ri.initial_not_refractory.push_back(x.boolean() ? 1 : 0);
        check(ri.initial_lastspike.size() == pd.count && ri.initial_not_refractory.size() == pd.count,
              "invalid refractory array shape");
        check(ri.period_ticks <= 1000000 && timestep(ri.period, pd.dt) == ri.period_ticks,
              "invalid refractory period/ticks");
        pin.refractory = std::move(ri);
      }
      if (!p.absent("spike_generator")) {
        const Value& g = p.at("spike_generator");
        SpikeGenerator sg;
        sg.spike_ticks = size_list(g.at("spike_ticks"));
        sg.spike_indices = size_list(g.at("spike_indices"));
        check(sg.spike_ticks.size() == sg.spike_indices.size(), "invalid spike generator");
        pin.spike_generator = std::move(sg);
      }
      for (const auto& s : pd.states) {
        auto it = pin.initial_state.find(s.name);
        check(it != pin.initial_state.end() && it->second.size() == pd.count,
              "population '" + pd.name + "' state '" + s.name + "' has the wrong length");
      }
      for (const auto& s : pd.parameters) {
        auto it = pin.parameters.find(s.name);
        check(it != pin.parameters.end(), "population parameter '" + s.name + "' missing");
        size_t want = s.index_domain == IndexDomain::Scalar ? 1 : pd.count;
        check(it->second.size() == want, "population parameter '" + s.name + "' has the wrong length");
      }
      m.population_instances.push_back(std::move(pin));
    }
    const auto& syns = inst.at("synapses").arr();
    check(syns.size() == m.synapses.size(), "synapse instance count mismatch");
    for (size_t si = 0; si < syns.size(); ++si) {
      const Value& s = syns[si];
      const SynapseDef& sd = m.synapses[si];
      SynapseInstance sin;
      for (const auto& x : s.at("source").arr()) sin.source.push_back(uint32_t(x.u64()));
      for (const auto& x : s.at("target").arr()) sin.target.push_back(uint32_t(x.u64()));
      check(sin.source.size() == sin.target.size(), "synapse endpoint arrays differ in length");
      sin.topology = parse_topology(s.at("topology"));
      sin.initial_state = decode_table(s.at("initial_state"), sd.states, {});
      sin.parameters = decode_table(s.at("parameters"), sd.parameters, {});
      for (const auto& pw : s.at("pathways").arr()) {
        PathwayInstance pi;
        pi.name = str(pw, "name");
        pi.kind = str(pw, "kind");
        pi.event = str(pw, "event");
        check(pi.kind == "pre" || pi.kind == "post", "pathway kind must be pre or post");
        for (const auto& x : pw.at("delay").arr()) pi.delay.push_back(decode_f64_bits(x.str()));
        pi.delay_ticks = size_list(pw.at("delay_ticks"));
        if (!pw.absent("delay_initializer")) pi.delay_initializer = parse_initializer(pw.at("delay_initializer"));
        for (const auto& e : pw.at("pending").arr())
          pi.pending.push_back({size_t(e.at("delivery_tick").u64()), size_t(e.at("item").u64())});
        sin.pathways.push_back(std::move(pi));
      }
      if (sin.topology.kind == Topology::Kind::Explicit) {
        for (size_t e = 0; e < sin.source.size(); ++e)
          check(sin.source[e] < sd.source_count && sin.target[e] < sd.target_count,
                "synapse endpoint index out of range");
      }
      m.synapse_instances.push_back(std::move(sin));
    }
    const Value& run = doc.at("run");
    m.run_start = decode_f64_bits(str(run, "start"));
    m.run_duration = decode_f64_bits(str(run, "duration"));
    for (const auto& c : run.at("clocks").arr()) m.run_clocks.push_back({usz(c, "start_tick"), usz(c, "steps")});
    check(m.run_clocks.size() == m.clocks.size(), "run clock count mismatch");
    for (const auto& p : m.populations) check(p.clock < m.clocks.size(), "population clock out of range");
    // binary_csr mapping rules and file contents (model.rs:2163-2205)
    for (size_t s = 0; s < m.synapses.size() && s < m.synapse_instances.size(); ++s) {
      const SynapseDef& def = m.synapses[s];
      const SynapseInstance& inst = m.synapse_instances[s];
      const Topology& t = inst.topology;
      if (t.kind != Topology::Kind::BinaryCsr) continue;
      std::set<std::string> names, mapped;
      bool ok = inst.source.empty() && inst.target.empty() && def.states.empty();
      for (const auto& p : def.parameters)
        if (p.index_domain == IndexDomain::Synapse) {
          names.insert(p.name);
          ok &= p.dtype == DType::F64;
        }
      std::set<uint64_t> cols;
      for (const auto& [name, col] : t.columns) {
        mapped.insert(name);
        cols.insert(col);
        ok &= col < t.column_count;
      }
      ok &= names == mapped && cols.size() == t.column_count;
      ok &= t.sha256.size() == 64 && std::all_of(t.sha256.begin(), t.sha256.end(), [](char c) { return std::isxdigit(uint8_t(c)); });
      for (const auto& p : inst.pathways) ok &= p.kind == "pre" && !p.delay_initializer && p.delay.size() == 1;
      check(ok, "invalid binary CSR mapping/pathway");
      read_binary_csr(t.path, def.source_count, def.target_count, t.edge_count, t.column_count, t.sha256, false);
    }
    // A current-schema document is checked after its content, as run_cli
    // does (model.rs:4651-4661); a legacy envelope was checked on entry.
    if (m.schema == "atlasir-v1") b2canon::verify_protocol(doc);
    return m;
  } catch (const b2json::Error& e) {
    throw Error(e.what());
  } catch (const std::invalid_argument&) {
    throw Error("invalid integer literal");
  } catch (const std::out_of_range&) {
    throw Error("integer literal out of range");
  }
}

BinaryCsr read_binary_csr(const std::string& path, uint64_t sources, uint64_t targets, uint64_t edges,
                          uint64_t columns, const std::string& sha256, bool materialize) {
  check(sources > 0 && targets > 0 && sources <= 1'000'000 && targets <= 1'000'000 && edges > 0 &&
            edges <= 100'000'000 && columns <= 128,
        "invalid binary CSR shape");
  std::ifstream f(path, std::ios::binary);
  check(bool(f), "cannot open binary CSR file '" + path + "'");
  const uint64_t expected = 40 + (sources + 1) * 8 + edges * (4 + 8 * columns);
  f.seekg(0, std::ios::end);
  check(uint64_t(f.tellg()) == expected, "binary CSR file length mismatch");
  f.seekg(0);
  {
    b2canon::Sha256 digest;
    std::vector<char> chunk(1 << 16);
    while (f) {
      f.read(chunk.data(), std::streamsize(chunk.size()));
      digest.update(chunk.data(), size_t(f.gcount()));
    }
    std::string want = sha256;
    for (char& c : want) c = char(std::tolower(uint8_t(c)));
    check(digest.hex() == want, "binary CSR checksum mismatch");
  }
  f.clear();
  f.seekg(0);
  std::vector<char> bytes(expected);
  f.read(bytes.data(), std::streamsize(expected));
  check(uint64_t(f.gcount()) == expected, "binary CSR file length mismatch");
  const char* p = bytes.data();
  auto u64 = [&p]() {
    uint64_t v;
    std::memcpy(&v, p, 8);  // little-endian host
    p += 8;
    return v;
  };
  check(std::memcmp(p, "B2CSR001", 8) == 0, "binary CSR header mismatch");
  p += 8;
  const uint64_t hs = u64(), ht = u64(), he = u64(), hc = u64();
  check(hs == sources && ht == targets && he == edges && hc == columns, "binary CSR header mismatch");
  BinaryCsr out;
  if (materialize) {
    out.source.reserve(edges);
    out.target.reserve(edges);
  }
  uint64_t previous = u64();
  check(previous == 0, "binary CSR offsets must start at zero");
  for (uint64_t neuron = 0; neuron < sources; ++neuron) {
    const uint64_t next = u64();
    check(next >= previous && next <= edges, "invalid binary CSR offsets");
    if (materialize) out.source.resize(next, uint32_t(neuron));
    previous = next;
  }
  check(previous == edges, "binary CSR final offset mismatch");
  for (uint64_t e = 0; e < edges; ++e) {
    uint32_t v;
    std::memcpy(&v, p, 4);
    p += 4;
    check(v < targets, "binary CSR target outside population");
    if (materialize) out.target.push_back(v);
  }
  for (uint64_t c = 0; c < columns; ++c) {
    std::vector<double> column;
    if (materialize) column.reserve(edges);
    for (uint64_t e = 0; e < edges; ++e) {
      double v;
      std::memcpy(&v, p, 8);
      p += 8;
      check(std::isfinite(v), "nonfinite binary CSR parameter");
      if (materialize) column.push_back(v);
    }
    if (materialize) out.columns.push_back(std::move(column));
  }
  return out;
}

Model load_model_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  check(bool(f), "cannot open model file '" + path + "'");
  std::stringstream ss;
  ss << f.rdbuf();
  std::string data = ss.str();
  return load_model(data.data(), data.size());
}

}  // namespace b2ir
