// ORACLE (test infrastructure only): CPU restatement of the reference executor.
//
// Structure mirrors brian2-rust/src/executor.rs so every rule can be checked
// line against line:
//   StateArray register semantics ........ executor.rs:346-573
//   Program::compile / statements ......... executor.rs:5046-5486
//   Program::prepare / run / commit ....... executor.rs:5488-5670
//   evaluate (per-op semantics) ........... executor.rs:5725-6158
//   population build ...................... executor.rs:1757-2112
//   run_population_update ................. executor.rs:2139-2164
//   deliver_event / run_pathway ........... executor.rs:2166-2382
//   emit_threshold / monitors ............. executor.rs:2949-3097
//   Runtime::new / advance ................ executor.rs:3473-4360
//   PathwayQueue / edge_csr ............... executor.rs:6160-6212
//   materialize_projection ................ executor.rs:19-188, large_topology.rs:115-260
#include "executor.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <optional>
#include <set>
#include <thread>
#include <unordered_set>

#include "rng.hpp"

namespace oracle {

using namespace b2ir;
using b2dump::TickIndex;

namespace {

constexpr size_t LANES = 256;

inline uint64_t bits_of(double v) {
  uint64_t r;
  std::memcpy(&r, &v, 8);
  return r;
}
inline double from_bits(uint64_t r) {
  double v;
  std::memcpy(&v, &r, 8);
  return v;
}

enum class Domain { Neuron, Pre, Post, Edge };

// ---------------------------------------------------------------- StateArray
struct StateArray {
  DType dtype = DType::F64;
  std::vector<uint8_t> bytes;
  size_t n = 0;

  static StateArray empty(DType d) {
    dtype_bytes(d);
    StateArray s;
    s.dtype = d;
    return s;
  }
  static StateArray from_encoded(const EncodedArray& a) {
    StateArray s = empty(a.dtype);
    s.n = a.size();
    s.bytes.resize(s.n * dtype_bytes(a.dtype));
    for (size_t i = 0; i < s.n; ++i) s.store_raw(i, a.raw[i]);
    return s;
  }
  size_t width() const { return dtype_bytes(dtype); }
  void store_raw(size_t i, uint64_t raw) { std::memcpy(&bytes[i * width()], &raw, width()); }
  uint64_t load_raw(size_t i) const {
    uint64_t r = 0;
    std::memcpy(&r, &bytes[i * width()], width());
    return r;
  }
  // get_register (executor.rs:422-432)
  double get(size_t i) const {
    switch (dtype) {
      case DType::Bool: return bytes[i] ? 1.0 : 0.0;
      case DType::F32: {
        float f;
        std::memcpy(&f, &bytes[i * 4], 4);
        return double(f);
      }
      case DType::F64: return from_bits(load_raw(i));
      default: return from_bits(load_raw(i));  // ints: zero-extended raw bits
    }
  }
  // set_register (executor.rs:457-467)
  void set(size_t i, double v) {
    switch (dtype) {
      case DType::Bool: bytes[i] = v != 0.0 ? 1 : 0; break;
      case DType::F32: {
        float f = float(v);
        std::memcpy(&bytes[i * 4], &f, 4);
        break;
      }
      case DType::F64: store_raw(i, bits_of(v)); break;
      default: store_raw(i, bits_of(v)); break;  // ints keep the low bytes of the bits
    }
  }
  void push(double v) {
    bytes.resize((n + 1) * width());
    ++n;
    set(n - 1, v);
  }
  b2dump::Column column() const { return b2dump::Column{dtype, bytes}; }
};

// ---------------------------------------------------------------- Batch
struct Batch {
  size_t start = 0, len = 0, source = 0, target = 0, source_state = 0, target_state = 0, edge = 0;
  static Batch neurons(size_t start, size_t len) {
    Batch b;
    b.start = start;
    b.len = len;
    return b;
  }
  size_t index(Domain d, size_t lane) const {
    switch (d) {
      case Domain::Neuron: return start + lane;
      case Domain::Pre: return source;
      case Domain::Post: return target;
      case Domain::Edge: return edge;
    }
    return 0;
  }
};

struct RefractoryRuntime {
  std::vector<double> lastspike;
  std::vector<uint8_t> not_refractory;
};

// ---------------------------------------------------------------- Input
struct Input {
  enum class Kind { Constant, Time, Index, State, PreState, PostState, SynapseState, Parameter,
                    LastSpike, Available, Random, Normal } kind = Kind::Constant;
  double value = 0.0;
  DType dtype = DType::F64;
  Domain domain = Domain::Neuron;
  size_t index = 0;
  uint64_t stream = 0;
  std::shared_ptr<const std::vector<double>> values;

  bool scalar() const { return kind == Kind::Constant || kind == Kind::Time; }
  DType type() const {
    switch (kind) {
      case Kind::Constant: case Kind::State: case Kind::PreState: case Kind::PostState:
      case Kind::SynapseState: case Kind::Parameter: return dtype;
      case Kind::Time: case Kind::LastSpike: case Kind::Random: case Kind::Normal: return DType::F64;
      case Kind::Index: return DType::Index;
      case Kind::Available: return DType::Bool;
    }
    return DType::F64;
  }
  static Input constant(double v, DType d) { Input i; i.kind = Kind::Constant; i.value = v; i.dtype = d; return i; }
  static Input make(Kind k) { Input i; i.kind = k; return i; }
};

struct WriteTarget {
  enum class Kind { Neuron, PreNeuron, Synapse, Available } kind = Kind::Neuron;
  size_t index = 0;
};

// ---------------------------------------------------------------- instructions
enum class IOp {
  Neg, Not, Abs, Arccos, Arcsin, Arctan, Ceil, Cos, Cosh, Exp, Expm1, Exprel, Floor, Trunc,
  RoundF32, Cast, IntNeg, IntAbs, IntBinary, Timestep, TickOffset, Log, Log10, Log1p, Sign,
  Sin, Sinh, Sqrt, Tan, Tanh, Add, Sub, Mul, Div, Pow, Mod, FloorDiv, Eq, Ne, Gt, Ge, Lt, Le,
  And, Or, Clip, Select, Binomial, Poisson, TimedArray,
};
enum class IntOp { Add, Sub, Mul, Mod, FloorDiv, Gt, Ge, Lt, Le };

struct Instruction {
  IOp op = IOp::Add;
  size_t left = 0, right = 0, output = 0;
  long third = -1, guard = -1;
  DType src = DType::F64, dst = DType::F64;  // Cast; dst also the integer op dtype
  IntOp intop = IntOp::Add;
  uint64_t stream = 0, n = 0;
  bool approximate = false;
  Domain domain = Domain::Neuron;
  int64_t offset = 0;
  const Expr* ta = nullptr;
};

// cast_register (executor.rs:5780-5829)
double cast_register(double value, DType source, DType target) {
  uint64_t b = bits_of(value);
  if (target == DType::F64) {
    switch (source) {
      case DType::Bool: return value != 0.0 ? 1.0 : 0.0;
      case DType::F32: case DType::F64: return value;
      case DType::I32: return double(int32_t(uint32_t(b)));
      case DType::I64: return double(int64_t(b));
      case DType::U32: return double(uint32_t(b));
      case DType::U64: return double(b);
      default: throw Error("unsupported cast source");
    }
  }
  auto encode_signed = [&](__int128 v) -> uint64_t {
    switch (target) {
      case DType::I32: return uint64_t(uint32_t(int32_t(v)));
      case DType::I64: return uint64_t(int64_t(v));
      case DType::U32: return uint64_t(uint32_t(v));
      case DType::U64: return uint64_t(v);
      default: throw Error("unsupported cast target");
    }
  };
  switch (source) {
    case DType::I32: return from_bits(encode_signed(__int128(int32_t(uint32_t(b)))));
    case DType::I64: return from_bits(encode_signed(__int128(int64_t(b))));
    case DType::U32: return from_bits(encode_signed(__int128(uint32_t(b))));
    case DType::U64: return from_bits(encode_signed(__int128(b)));
    default: break;
  }
  double numeric;
  if (source == DType::Bool) numeric = value != 0.0 ? 1.0 : 0.0;
  else if (source == DType::F32 || source == DType::F64) numeric = value;
  else throw Error("unsupported cast source");
  // Rust float->int `as` casts saturate and map NaN to 0.
  auto sat_i64 = [](double x) -> int64_t {
    if (std::isnan(x)) return 0;
    if (x <= -9223372036854775808.0) return INT64_MIN;
    if (x >= 9223372036854775808.0) return INT64_MAX;
    return int64_t(x);
  };
  auto sat_u64 = [](double x) -> uint64_t {
    if (std::isnan(x) || x <= 0.0) return 0;
    if (x >= 18446744073709551616.0) return UINT64_MAX;
    return uint64_t(x);
  };
  switch (target) {
    case DType::I32: {
      int64_t v = sat_i64(numeric);
      int32_t w = v < INT32_MIN ? INT32_MIN : v > INT32_MAX ? INT32_MAX : int32_t(v);
      return from_bits(uint64_t(uint32_t(w)));
    }
    case DType::I64: return from_bits(uint64_t(sat_i64(numeric)));
    case DType::U32: {
      uint64_t v = sat_u64(numeric);
      return from_bits(v > UINT32_MAX ? UINT32_MAX : v);
    }
    case DType::U64: return from_bits(sat_u64(numeric));
    default: throw Error("unsupported cast target");
  }
}

template <class T>
T floor_mod(T a, T b) {
  T q = T(a / b), r = T(a % b);
  T fq = (r != 0 && ((r < 0) != (b < 0))) ? T(q - 1) : q;
  return T(a - fq * b);
}
template <class T>
T floor_div(T a, T b) {
  T q = T(a / b), r = T(a % b);
  return (r != 0 && ((r < 0) != (b < 0))) ? T(q - 1) : q;
}

// integer_binary_value (executor.rs:5847-5930); wrapping arithmetic via unsigned.
double integer_binary(DType dtype, IntOp op, double left, double right) {
  uint64_t lb = bits_of(left), rb = bits_of(right);
  auto rel = [&](auto a, auto b) -> std::optional<double> {
    switch (op) {
      case IntOp::Gt: return a > b ? 1.0 : 0.0;
      case IntOp::Ge: return a >= b ? 1.0 : 0.0;
      case IntOp::Lt: return a < b ? 1.0 : 0.0;
      case IntOp::Le: return a <= b ? 1.0 : 0.0;
      default: return std::nullopt;
    }
  };
  switch (dtype) {
    case DType::I32: {
      int32_t a = int32_t(uint32_t(lb)), b = int32_t(uint32_t(rb));
      if (auto r = rel(a, b)) return *r;
      uint32_t ua = uint32_t(a), ub = uint32_t(b), v = 0;
      switch (op) {
        case IntOp::Add: v = ua + ub; break;
        case IntOp::Sub: v = ua - ub; break;
        case IntOp::Mul: v = ua * ub; break;
        case IntOp::Mod:
          check(b != 0, "integer modulo by zero");
          v = (a == INT32_MIN && b == -1) ? 0u : uint32_t(floor_mod<int32_t>(a, b));
          break;
        case IntOp::FloorDiv:
          check(b != 0, "integer division by zero");
          v = (a == INT32_MIN && b == -1) ? uint32_t(INT32_MIN) : uint32_t(floor_div<int32_t>(a, b));
          break;
        default: break;
      }
      return from_bits(uint64_t(v));
    }
    case DType::I64: {
      int64_t a = int64_t(lb), b = int64_t(rb);
      if (auto r = rel(a, b)) return *r;
      uint64_t v = 0;
      switch (op) {
        case IntOp::Add: v = lb + rb; break;
        case IntOp::Sub: v = lb - rb; break;
        case IntOp::Mul: v = lb * rb; break;
        case IntOp::Mod:
          check(b != 0, "integer modulo by zero");
          v = (a == INT64_MIN && b == -1) ? 0 : uint64_t(floor_mod<int64_t>(a, b));
          break;
        case IntOp::FloorDiv:
          check(b != 0, "integer division by zero");
          v = (a == INT64_MIN && b == -1) ? uint64_t(INT64_MIN) : uint64_t(floor_div<int64_t>(a, b));
          break;
        default: break;
      }
      return from_bits(v);
    }
    case DType::U32: {
      uint32_t a = uint32_t(lb), b = uint32_t(rb);
      if (auto r = rel(a, b)) return *r;
      uint32_t v = 0;
      switch (op) {
        case IntOp::Add: v = a + b; break;
        case IntOp::Sub: v = a - b; break;
        case IntOp::Mul: v = a * b; break;
        case IntOp::Mod: check(b != 0, "integer modulo by zero"); v = a % b; break;
        case IntOp::FloorDiv: check(b != 0, "integer division by zero"); v = a / b; break;
        default: break;
      }
      return from_bits(uint64_t(v));
    }
    case DType::U64: {
      uint64_t a = lb, b = rb;
      if (auto r = rel(a, b)) return *r;
      uint64_t v = 0;
      switch (op) {
        case IntOp::Add: v = a + b; break;
        case IntOp::Sub: v = a - b; break;
        case IntOp::Mul: v = a * b; break;
        case IntOp::Mod: check(b != 0, "integer modulo by zero"); v = a % b; break;
        case IntOp::FloorDiv: check(b != 0, "integer division by zero"); v = a / b; break;
        default: break;
      }
      return from_bits(v);
    }
    default: throw Error("invalid integer operation dtype");
  }
}

// ---------------------------------------------------------------- Program
struct Program {
  std::vector<std::vector<double>> registers;
  std::map<std::string, size_t> symbols;
  std::map<std::string, DType> symbol_dtypes;
  std::map<std::string, Input> inputs;
  std::vector<std::pair<size_t, Input>> bindings;
  std::set<size_t> scalar_random_bindings;
  std::vector<size_t> broadcast;
  std::vector<Instruction> scalar, vector;
  std::vector<std::pair<WriteTarget, size_t>> writes;
  long condition = -1;
  uint64_t rng_seed = 0, tick = 0;
  Domain rng_domain = Domain::Neuron;
  std::map<std::string, const Function*> functions;

  static Program compile(const CodeObject& code, std::map<std::string, Input> inputs,
                         const std::map<std::string, WriteTarget>& writable, uint64_t rng_seed,
                         const std::vector<Function>& functions) {
    check(!code.adaptive, "adaptive integrators are outside the simulated path");
    Program p;
    for (const auto& kv : inputs) p.symbol_dtypes[kv.first] = kv.second.type();
    p.inputs = std::move(inputs);
    p.rng_seed = rng_seed;
    p.rng_domain = (code.iteration_domain == "all_synapses" || code.iteration_domain == "active_synapses")
                       ? Domain::Edge : Domain::Neuron;
    for (const auto& f : functions) p.functions[f.name] = &f;
    p.scalar = p.statements(code.scalar);
    for (const auto& b : p.bindings)
      if (b.second.kind == Input::Kind::Random || b.second.kind == Input::Kind::Normal)
        p.scalar_random_bindings.insert(b.first);
    for (size_t i = 0; i < p.registers.size(); ++i) p.broadcast.push_back(i);
    p.vector = p.statements(code.vector);
    for (const auto& b : p.bindings)
      if (b.second.scalar()) p.broadcast.push_back(b.first);
    std::sort(p.broadcast.begin(), p.broadcast.end());
    p.broadcast.erase(std::unique(p.broadcast.begin(), p.broadcast.end()), p.broadcast.end());
    for (const auto& name : code.effects.writes) {
      auto w = writable.find(name);
      check(w != writable.end(), "write to non-writable symbol '" + name + "'");
      auto s = p.symbols.find(name);
      check(s != p.symbols.end(), "written symbol '" + name + "' was never assigned");
      p.writes.push_back({w->second, s->second});
    }
    if (code.kind == "threshold") {
      auto c = p.symbols.find("_cond");
      check(c != p.symbols.end(), "missing threshold condition");
      p.condition = long(c->second);
    }
    return p;
  }

  size_t reg() {
    registers.emplace_back(LANES, 0.0);
    return registers.size() - 1;
  }
  size_t input(const Input& v) {
    size_t slot = reg();
    bindings.push_back({slot, v});
    return slot;
  }
  size_t resolve(const std::string& name) {
    auto it = symbols.find(name);
    if (it != symbols.end()) return it->second;
    auto in = inputs.find(name);
    check(in != inputs.end(), "missing plan input '" + name + "'");
    size_t slot = input(in->second);
    symbols[name] = slot;
    return slot;
  }

  // Expr::infer, dtype part only (model.rs:1251-1546).
  DType infer(const Expr& e) {
    switch (e.op) {
      case Op::Literal: return DType::F64;
      case Op::Boolean: return DType::Bool;
      case Op::Integer: return e.dtype;
      case Op::Cast: return e.dtype;
      case Op::Rand: case Op::Randn: case Op::Binomial: case Op::Poisson: case Op::TimedArray:
      case Op::BoolToF64: case Op::IndexToF64: case Op::TickToF64: case Op::F32ToF64:
        return DType::F64;
      case Op::F64ToF32: return DType::F32;
      case Op::Timestep: case Op::TickOffset: return DType::Tick;
      case Op::Load: {
        auto it = symbol_dtypes.find(e.name);
        check(it != symbol_dtypes.end(), "undefined symbol: " + e.name);
        return it->second;
      }
      case Op::Call: {
        auto it = functions.find(e.name);
        check(it != functions.end(), "undefined function: " + e.name);
        return it->second->return_dtype;
      }
      case Op::Neg: case Op::Abs: return infer(*e.args[0]);
      case Op::Not: case Op::Eq: case Op::Ne: case Op::And: case Op::Or:
      case Op::Gt: case Op::Ge: case Op::Lt: case Op::Le: return DType::Bool;
      case Op::Add: case Op::Sub: case Op::Mul: case Op::Pow: case Op::Mod: case Op::FloorDiv: {
        DType l = infer(*e.args[0]), r = infer(*e.args[1]);
        return (l == r && is_integer(l)) ? l : DType::F64;
      }
      default: return DType::F64;
    }
  }

  size_t expression(const Expr& e, long guard, std::vector<Instruction>& ops) {
    Instruction ins;
    ins.guard = guard;
    switch (e.op) {
      case Op::Literal: return input(Input::constant(e.literal, DType::F64));
      case Op::Boolean: return input(Input::constant(e.boolean ? 1.0 : 0.0, DType::Bool));
      case Op::Integer: return input(Input::constant(from_bits(e.raw), e.dtype));
      case Op::Rand: {
        Input i = Input::make(Input::Kind::Random);
        i.stream = e.stream;
        i.domain = rng_domain;
        return input(i);
      }
      case Op::Randn: {
        Input i = Input::make(Input::Kind::Normal);
        i.stream = e.stream;
        i.domain = rng_domain;
        return input(i);
      }
      case Op::Load: return resolve(e.name);
      case Op::BoolToF64: case Op::IndexToF64: case Op::TickToF64: case Op::F32ToF64:
        return expression(*e.args[0], guard, ops);
      case Op::Call: {
        auto it = functions.find(e.name);
        check(it != functions.end(), "missing Function contract in execution plan");
        const Function& fn = *it->second;
        check(fn.arguments.size() == e.args.size(), "function argument count does not match contract");
        std::vector<size_t> slots;
        for (const auto& a : e.args) slots.push_back(expression(*a, guard, ops));
        std::vector<std::pair<std::string, std::optional<size_t>>> prev;
        std::vector<std::pair<std::string, std::optional<DType>>> prev_types;
        for (size_t k = 0; k < fn.arguments.size(); ++k) {
          const auto& name = fn.arguments[k].name;
          auto s = symbols.find(name);
          prev.push_back({name, s == symbols.end() ? std::nullopt : std::optional<size_t>(s->second)});
          symbols[name] = slots[k];
          auto t = symbol_dtypes.find(name);
          prev_types.push_back({name, t == symbol_dtypes.end() ? std::nullopt : std::optional<DType>(t->second)});
          symbol_dtypes[name] = fn.arguments[k].dtype;
        }
        check(bool(fn.body), "reference executor cannot execute a native-only Function");
        size_t result = expression(*fn.body, guard, ops);
        for (auto& kv : prev) {
          if (kv.second) symbols[kv.first] = *kv.second;
          else symbols.erase(kv.first);
        }
        for (auto& kv : prev_types) {
          if (kv.second) symbol_dtypes[kv.first] = *kv.second;
          else symbol_dtypes.erase(kv.first);
        }
        return result;
      }
      case Op::Cast:
        ins.op = IOp::Cast;
        ins.src = infer(*e.args[0]);
        ins.dst = e.dtype;
        ins.left = ins.right = expression(*e.args[0], guard, ops);
        break;
      case Op::Binomial:
        ins.op = IOp::Binomial;
        ins.stream = e.stream;
        ins.n = e.n;
        ins.approximate = e.approximate;
        ins.domain = rng_domain;
        ins.left = ins.right = expression(*e.args[0], guard, ops);
        break;
      case Op::Poisson:
        ins.op = IOp::Poisson;
        ins.stream = e.stream;
        ins.domain = rng_domain;
        ins.left = ins.right = expression(*e.args[0], guard, ops);
        break;
      case Op::TimedArray: {
        ins.op = IOp::TimedArray;
        ins.ta = &e;
        size_t t = expression(*e.args[0], guard, ops);
        ins.left = t;
        ins.right = e.args.size() > 1 ? expression(*e.args[1], guard, ops) : t;
        break;
      }
      case Op::F64ToF32:
        ins.op = IOp::RoundF32;
        ins.left = ins.right = expression(*e.args[0], guard, ops);
        break;
      case Op::Timestep:
        ins.op = IOp::Timestep;
        ins.left = expression(*e.args[0], guard, ops);
        ins.right = expression(*e.args[1], guard, ops);
        break;
      case Op::TickOffset:
        ins.op = IOp::TickOffset;
        ins.offset = e.offset;
        ins.left = ins.right = expression(*e.args[0], guard, ops);
        break;
      case Op::Clip:
        ins.op = IOp::Clip;
        ins.left = expression(*e.args[0], guard, ops);
        ins.right = expression(*e.args[1], guard, ops);
        ins.third = long(expression(*e.args[2], guard, ops));
        break;
      default:
        if (is_unary_math(e.op)) {
          size_t slot = expression(*e.args[0], guard, ops);
          DType dt = infer(*e.args[0]);
          ins.left = ins.right = slot;
          switch (e.op) {
            case Op::Neg: if (is_integer(dt)) { ins.op = IOp::IntNeg; ins.dst = dt; } else ins.op = IOp::Neg; break;
            case Op::Not: ins.op = IOp::Not; break;
            case Op::Abs: if (is_integer(dt)) { ins.op = IOp::IntAbs; ins.dst = dt; } else ins.op = IOp::Abs; break;
            case Op::Arccos: ins.op = IOp::Arccos; break;
            case Op::Arcsin: ins.op = IOp::Arcsin; break;
            case Op::Arctan: ins.op = IOp::Arctan; break;
            case Op::Ceil: ins.op = IOp::Ceil; break;
            case Op::Cos: ins.op = IOp::Cos; break;
            case Op::Cosh: ins.op = IOp::Cosh; break;
            case Op::Exp: ins.op = IOp::Exp; break;
            case Op::Expm1: ins.op = IOp::Expm1; break;
            case Op::Exprel: ins.op = IOp::Exprel; break;
            case Op::Floor: ins.op = IOp::Floor; break;
            case Op::Trunc: ins.op = IOp::Trunc; break;
            case Op::Log: ins.op = IOp::Log; break;
            case Op::Log10: ins.op = IOp::Log10; break;
            case Op::Log1p: ins.op = IOp::Log1p; break;
            case Op::Sign: ins.op = IOp::Sign; break;
            case Op::Sin: ins.op = IOp::Sin; break;
            case Op::Sinh: ins.op = IOp::Sinh; break;
            case Op::Sqrt: ins.op = IOp::Sqrt; break;
            case Op::Tan: ins.op = IOp::Tan; break;
            case Op::Tanh: ins.op = IOp::Tanh; break;
            default: throw Error("unsupported unary op");
          }
        } else if (is_binary(e.op)) {
          DType dt = infer(*e.args[0]);
          bool integer = is_integer(dt);
          auto intop = [&](IntOp k) { ins.op = IOp::IntBinary; ins.intop = k; ins.dst = dt; };
          switch (e.op) {
            case Op::Add: if (integer) intop(IntOp::Add); else ins.op = IOp::Add; break;
            case Op::Sub: if (integer) intop(IntOp::Sub); else ins.op = IOp::Sub; break;
            case Op::Mul: if (integer) intop(IntOp::Mul); else ins.op = IOp::Mul; break;
            case Op::Mod: if (integer) intop(IntOp::Mod); else ins.op = IOp::Mod; break;
            case Op::FloorDiv: if (integer) intop(IntOp::FloorDiv); else ins.op = IOp::FloorDiv; break;
            case Op::Gt: if (integer) intop(IntOp::Gt); else ins.op = IOp::Gt; break;
            case Op::Ge: if (integer) intop(IntOp::Ge); else ins.op = IOp::Ge; break;
            case Op::Lt: if (integer) intop(IntOp::Lt); else ins.op = IOp::Lt; break;
            case Op::Le: if (integer) intop(IntOp::Le); else ins.op = IOp::Le; break;
            case Op::Div: ins.op = IOp::Div; break;
            case Op::Pow: ins.op = IOp::Pow; break;
            case Op::Eq: ins.op = IOp::Eq; break;
            case Op::Ne: ins.op = IOp::Ne; break;
            case Op::And: ins.op = IOp::And; break;
            case Op::Or: ins.op = IOp::Or; break;
            default: throw Error("unsupported binary op");
          }
          ins.left = expression(*e.args[0], guard, ops);
          ins.right = expression(*e.args[1], guard, ops);
        } else {
          throw Error(std::string("unsupported expression op ") + op_name(e.op));
        }
    }
    ins.output = reg();
    ops.push_back(ins);
    return ins.output;
  }

  std::vector<Instruction> statements(const std::vector<Statement>& sts) {
    std::vector<Instruction> ops;
    for (const auto& st : sts) {
      long guard = st.condition ? long(resolve(*st.condition)) : -1;
      std::optional<size_t> old;
      if (guard >= 0) {
        auto s = symbols.find(st.target);
        if (s != symbols.end()) old = s->second;
        else if (inputs.count(st.target)) old = resolve(st.target);
      }
      size_t value = expression(*st.value, guard, ops);
      size_t output = value;
      if (old) {
        Instruction sel;
        sel.op = IOp::Select;
        sel.left = value;
        sel.right = *old;
        sel.guard = guard;
        sel.output = reg();
        ops.push_back(sel);
        output = sel.output;
      }
      symbols[st.target] = output;
      symbol_dtypes[st.target] = st.dtype;
    }
    return ops;
  }

  void prepare(double time, uint64_t t) {
    tick = t;
    for (const auto& [slot, in] : bindings) {
      if (in.kind == Input::Kind::Constant) registers[slot][0] = in.value;
      else if (in.kind == Input::Kind::Time) registers[slot][0] = time;
      else if (in.kind == Input::Kind::Random && scalar_random_bindings.count(slot))
        registers[slot][0] = counter_uniform(rng_seed, in.stream, tick, 0);
      else if (in.kind == Input::Kind::Normal && scalar_random_bindings.count(slot))
        registers[slot][0] = counter_normal(rng_seed, in.stream, tick, 0);
    }
    evaluate(scalar, 1, Batch::neurons(0, 1));
    for (size_t slot : broadcast) {
      double v = registers[slot][0];
      std::fill(registers[slot].begin(), registers[slot].end(), v);
    }
  }

  static void copy_state(std::vector<double>& out, const StateArray& s, Domain d, const Batch& b) {
    if (d == Domain::Neuron) {
      for (size_t l = 0; l < b.len; ++l) out[l] = s.get(b.start + l);
    } else {
      double v = s.get(b.index(d, 0));
      std::fill(out.begin(), out.begin() + long(b.len), v);
    }
  }

  void run(const std::vector<StateArray>& states, const std::vector<StateArray>& pre,
           const std::vector<StateArray>& post, const std::vector<StateArray>& syn,
           const RefractoryRuntime* refr, const Batch& b) {
    for (const auto& [slot, in] : bindings) {
      if (scalar_random_bindings.count(slot)) continue;
      auto& out = registers[slot];
      switch (in.kind) {
        case Input::Kind::State: copy_state(out, states[in.index], in.domain, b); break;
        case Input::Kind::PreState: std::fill(out.begin(), out.begin() + long(b.len), pre[in.index].get(b.source_state)); break;
        case Input::Kind::PostState: std::fill(out.begin(), out.begin() + long(b.len), post[in.index].get(b.target_state)); break;
        case Input::Kind::SynapseState: copy_state(out, syn[in.index], Domain::Edge, b); break;
        case Input::Kind::Parameter:
          if (in.domain == Domain::Neuron) {
            for (size_t l = 0; l < b.len; ++l) out[l] = (*in.values)[b.start + l];
          } else {
            std::fill(out.begin(), out.begin() + long(b.len), (*in.values)[b.index(in.domain, 0)]);
          }
          break;
        case Input::Kind::Index:
          for (size_t l = 0; l < b.len; ++l) out[l] = double(b.index(in.domain, l));
          break;
        case Input::Kind::LastSpike:
          check(refr != nullptr, "missing refractory");
          for (size_t l = 0; l < b.len; ++l) out[l] = refr->lastspike[b.start + l];
          break;
        case Input::Kind::Available: {
          check(refr != nullptr, "missing refractory");
          for (size_t l = 0; l < b.len; ++l) {
            size_t idx = in.domain == Domain::Post ? b.target_state
                         : in.domain == Domain::Pre ? b.source_state : b.index(in.domain, l);
            out[l] = refr->not_refractory[idx] ? 1.0 : 0.0;
          }
          break;
        }
        case Input::Kind::Random:
          for (size_t l = 0; l < b.len; ++l) out[l] = counter_uniform(rng_seed, in.stream, tick, b.index(in.domain, l));
          break;
        case Input::Kind::Normal:
          for (size_t l = 0; l < b.len; ++l) out[l] = counter_normal(rng_seed, in.stream, tick, b.index(in.domain, l));
          break;
        case Input::Kind::Constant: case Input::Kind::Time: break;
      }
    }
    evaluate(vector, b.len, b);
  }

  void evaluate(const std::vector<Instruction>& ins, size_t len, const Batch& b) {
    for (const auto& I : ins) {
      const double* L = registers[I.left].data();
      const double* R = registers[I.right].data();
      const double* T = I.third >= 0 ? registers[size_t(I.third)].data() : nullptr;
      const double* G = I.guard >= 0 ? registers[size_t(I.guard)].data() : nullptr;
      double* O = registers[I.output].data();
      bool valid = true;
      auto each = [&](auto fn) {
        for (size_t l = 0; l < len; ++l) {
          if (G && G[l] == 0.0) continue;
          O[l] = fn(L[l], R[l], l);
          valid &= std::isfinite(O[l]);
        }
        check(valid, "non-finite numeric value");
      };
      auto each_raw = [&](auto fn) {
        for (size_t l = 0; l < len; ++l) {
          if (G && G[l] == 0.0) continue;
          O[l] = fn(L[l], R[l], l);
        }
      };
      switch (I.op) {
        case IOp::Neg: each([](double a, double, size_t) { return -a; }); break;
        case IOp::Not: each([](double a, double, size_t) { return a == 0.0 ? 1.0 : 0.0; }); break;
        case IOp::Abs: each([](double a, double, size_t) { return std::fabs(a); }); break;
        case IOp::Arccos: each([](double a, double, size_t) { return std::acos(a); }); break;
        case IOp::Arcsin: each([](double a, double, size_t) { return std::asin(a); }); break;
        case IOp::Arctan: each([](double a, double, size_t) { return std::atan(a); }); break;
        case IOp::Ceil: each([](double a, double, size_t) { return std::ceil(a); }); break;
        case IOp::Cos: each([](double a, double, size_t) { return std::cos(a); }); break;
        case IOp::Cosh: each([](double a, double, size_t) { return std::cosh(a); }); break;
        case IOp::Exp: each([](double a, double, size_t) { return std::exp(a); }); break;
        case IOp::Expm1: each([](double a, double, size_t) { return std::expm1(a); }); break;
        case IOp::Exprel:
          each([](double a, double, size_t) {
            if (std::fabs(a) < 1e-16) return 1.0;
            if (a > 717.0) return double(INFINITY);
            return std::expm1(a) / a;
          });
          break;
        case IOp::Floor: each([](double a, double, size_t) { return std::floor(a); }); break;
        case IOp::Trunc:
          each([](double a, double, size_t) { return std::fabs(a) <= 9007199254740992.0 ? std::trunc(a) : NAN; });
          break;
        case IOp::RoundF32:
          each([](double a, double, size_t) {
            float f = float(a);
            return std::isfinite(f) ? double(f) : NAN;
          });
          break;
        case IOp::Cast: each_raw([&](double a, double, size_t) { return cast_register(a, I.src, I.dst); }); break;
        case IOp::IntNeg:
          each_raw([&](double a, double, size_t) {
            uint64_t r = bits_of(a);
            if (I.dst == DType::I32) return from_bits(uint64_t(uint32_t(0u - uint32_t(r))));
            return from_bits(0ull - r);
          });
          break;
        case IOp::IntAbs:
          each_raw([&](double a, double, size_t) {
            uint64_t r = bits_of(a);
            if (I.dst == DType::I32) {
              int32_t v = int32_t(uint32_t(r));
              return from_bits(uint64_t(v < 0 ? uint32_t(0u - uint32_t(v)) : uint32_t(v)));
            }
            int64_t v = int64_t(r);
            return from_bits(v < 0 ? 0ull - uint64_t(v) : uint64_t(v));
          });
          break;
        case IOp::IntBinary: each_raw([&](double a, double c, size_t) { return integer_binary(I.dst, I.intop, a, c); }); break;
        case IOp::Timestep:
          each_raw([&](double a, double c, size_t) {
            uint64_t v = timestep(a, c);
            check(v <= 9007199254740992ull, "timestep outside exact f64 execution range");
            return double(v);
          });
          break;
        case IOp::TickOffset:
          each([&](double a, double, size_t) {
            double r = a + double(I.offset);
            return std::fabs(r) <= 9007199254740992.0 ? r : NAN;
          });
          break;
        case IOp::Log: each([](double a, double, size_t) { return std::log(a); }); break;
        case IOp::Log10: each([](double a, double, size_t) { return std::log10(a); }); break;
        case IOp::Log1p: each([](double a, double, size_t) { return std::log1p(a); }); break;
        case IOp::Sign: each([](double a, double, size_t) { return a > 0.0 ? 1.0 : a < 0.0 ? -1.0 : 0.0; }); break;
        case IOp::Sin: each([](double a, double, size_t) { return std::sin(a); }); break;
        case IOp::Sinh: each([](double a, double, size_t) { return std::sinh(a); }); break;
        case IOp::Sqrt: each([](double a, double, size_t) { return std::sqrt(a); }); break;
        case IOp::Tan: each([](double a, double, size_t) { return std::tan(a); }); break;
        case IOp::Tanh: each([](double a, double, size_t) { return std::tanh(a); }); break;
        case IOp::Add: each([](double a, double c, size_t) { return a + c; }); break;
        case IOp::Sub: each([](double a, double c, size_t) { return a - c; }); break;
        case IOp::Mul: each([](double a, double c, size_t) { return a * c; }); break;
        case IOp::Div: each([](double a, double c, size_t) { return a / c; }); break;
        case IOp::Pow: each([](double a, double c, size_t) { return std::pow(a, c); }); break;
        case IOp::Mod: each([](double a, double c, size_t) { return a - c * std::floor(a / c); }); break;
        case IOp::FloorDiv: each([](double a, double c, size_t) { return std::floor(a / c); }); break;
        case IOp::Eq: each([](double a, double c, size_t) { return a == c ? 1.0 : 0.0; }); break;
        case IOp::Ne: each([](double a, double c, size_t) { return a != c ? 1.0 : 0.0; }); break;
        case IOp::Gt: each([](double a, double c, size_t) { return a > c ? 1.0 : 0.0; }); break;
        case IOp::Ge: each([](double a, double c, size_t) { return a >= c ? 1.0 : 0.0; }); break;
        case IOp::Lt: each([](double a, double c, size_t) { return a < c ? 1.0 : 0.0; }); break;
        case IOp::Le: each([](double a, double c, size_t) { return a <= c ? 1.0 : 0.0; }); break;
        case IOp::And: each([](double a, double c, size_t) { return (a != 0.0 && c != 0.0) ? 1.0 : 0.0; }); break;
        case IOp::Or: each([](double a, double c, size_t) { return (a != 0.0 || c != 0.0) ? 1.0 : 0.0; }); break;
        case IOp::Clip:
          each([&](double a, double c, size_t l) { return std::fmin(std::fmax(a, c), T[l]); });
          break;
        case IOp::Select:
          check(G != nullptr, "missing mask");
          for (size_t l = 0; l < len; ++l) O[l] = G[l] != 0.0 ? L[l] : R[l];
          break;
        case IOp::Binomial: {
          bool ok = true;
          for (size_t l = 0; l < len; ++l) {
            if (G && G[l] == 0.0) continue;
            double p = L[l];
            bool lane_ok = std::isfinite(p) && p >= 0.0 && p <= 1.0;
            ok &= lane_ok;
            if (lane_ok)
              O[l] = counter_binomial(rng_seed, I.stream, tick, b.index(I.domain, l), I.n, p, I.approximate);
          }
          check(ok, "invalid binomial probability");
          break;
        }
        case IOp::Poisson: {
          bool ok = true;
          for (size_t l = 0; l < len; ++l) {
            if (G && G[l] == 0.0) continue;
            O[l] = counter_poisson(rng_seed, I.stream, tick, b.index(I.domain, l), L[l]);
            ok &= std::isfinite(O[l]);
          }
          check(ok, "invalid poisson lambda");
          break;
        }
        case IOp::TimedArray: {
          const Expr& ta = *I.ta;
          size_t width = ta.ta_columns >= 0 ? size_t(ta.ta_columns) : 1;
          bool ok = true;
          for (size_t l = 0; l < len; ++l) {
            if (G && G[l] == 0.0) continue;
            double raw_row = std::trunc((L[l] / ta.ta_epsilon + 0.5) / double(ta.ta_upsampling));
            size_t row = raw_row <= 0.0 ? 0 : std::min(size_t(raw_row), ta.ta_rows - 1);
            size_t column = 0;
            if (ta.ta_columns >= 0) {
              double raw = R[l];
              if (!std::isfinite(raw) || raw < 0.0 || raw >= double(width)) {
                ok = false;
                continue;
              }
              column = size_t(raw);
            }
            O[l] = ta.ta_values[row * width + column];
            ok &= std::isfinite(O[l]);
          }
          check(ok, "TimedArray index/value outside supported range");
          break;
        }
      }
    }
  }

  void commit_neurons(std::vector<StateArray>& states, size_t start, size_t len) const {
    for (const auto& [t, r] : writes)
      if (t.kind == WriteTarget::Kind::Neuron)
        for (size_t l = 0; l < len; ++l) states[t.index].set(start + l, registers[r][l]);
  }
  void commit_available(RefractoryRuntime& refr, size_t start, size_t len) const {
    for (const auto& [t, r] : writes)
      if (t.kind == WriteTarget::Kind::Available)
        for (size_t l = 0; l < len; ++l) refr.not_refractory[start + l] = registers[r][l] != 0.0;
  }
  // commit_synapses (executor.rs:5615-5623): only synapse-state writes
  void commit_synapses(std::vector<StateArray>& syn, size_t edge) const {
    for (const auto& [t, r] : writes)
      if (t.kind == WriteTarget::Kind::Synapse) syn[t.index].set(edge, registers[r][0]);
  }
  void commit_event(std::vector<StateArray>* pre, std::vector<StateArray>& post,
                    std::vector<StateArray>& syn, size_t source_neuron, size_t target_neuron,
                    size_t edge) const {
    for (const auto& [t, r] : writes) {
      switch (t.kind) {
        case WriteTarget::Kind::Neuron: post[t.index].set(target_neuron, registers[r][0]); break;
        case WriteTarget::Kind::PreNeuron: (*pre)[t.index].set(source_neuron, registers[r][0]); break;
        case WriteTarget::Kind::Synapse: syn[t.index].set(edge, registers[r][0]); break;
        case WriteTarget::Kind::Available: break;
      }
    }
  }
};

// ---------------------------------------------------------------- runtime
enum class MonitorKind { State, Scalar, Parameter };
struct MonitorValue {
  MonitorKind kind = MonitorKind::State;
  size_t state = 0;
  double scalar = 0.0;
  std::shared_ptr<const std::vector<double>> values;
};

struct EventMonitorRuntime {
  size_t event_index = 0;
  std::vector<MonitorValue> values;
  std::vector<TickIndex> events;
  std::vector<StateArray> samples;
};

struct PopulationRuntime {
  std::vector<StateArray> states;
  std::optional<Program> subexpression_update, update;
  std::vector<Program> thresholds, poisson_inputs, regular, resets;
  std::vector<std::pair<size_t, size_t>> spike_schedule;
  size_t spike_cursor = 0;
  std::optional<RefractoryRuntime> refractory;
  size_t tick = 0, end_tick = 0;
  std::vector<std::vector<size_t>> fired;
  std::vector<std::vector<TickIndex>> event_history;
  std::vector<uint64_t> counts;
  std::vector<uint64_t> last_fired;
  std::vector<StateArray> samples;
  std::vector<TickIndex> spikes;
  std::vector<MonitorValue> monitor_values;
  std::vector<EventMonitorRuntime> event_monitors;
};

struct PathwayQueue {
  std::vector<size_t> offsets;
  std::vector<uint32_t> edges;  // edge ids (edge counts are checked to fit 32 bits)
  std::vector<std::vector<size_t>> queue;
  std::optional<size_t> uniform_delay;
  uint64_t delivered = 0;
};

struct PathwayRuntime {
  Program program;
  PathwayQueue topology;
  std::vector<size_t> delay_ticks;
  bool is_pre = true;
  size_t event_index = 0;
  std::vector<size_t> active_sources;
};

// SummedRuntime (executor.rs:1417-1426): the program of one `(summed)`
// variable, the register of its `_synaptic_var` result and the endpoint
// state it accumulates into.
struct SummedRuntime {
  Program program;
  size_t result = 0, target_population = 0, target_start = 0, target_count = 0, target_state = 0;
  bool target_is_pre = false;
};

struct SynapseRuntime {
  std::vector<uint32_t> source, target;  // endpoint indices per edge (counts checked to fit 32 bits)
  std::vector<StateArray> states;
  std::vector<PathwayRuntime> pathways;
  std::vector<SummedRuntime> summed;  // in code-object order
  // per-edge programs run over every edge (executor.rs:3612-3653):
  // synapse_state_update (clock-driven states writable),
  // synapse_subexpression_update and synapse_run_regularly (all writable,
  // but only synapse states are committed)
  std::optional<Program> update, subexpression;
  std::vector<Program> regular;  // in code-object order
};

std::shared_ptr<const std::vector<double>> decode_values(const EncodedArray& a) {
  auto v = std::make_shared<std::vector<double>>(a.size());
  for (size_t i = 0; i < a.size(); ++i) (*v)[i] = a.as_f64(i);
  return v;
}

// add_parameters (executor.rs:6214-6242)
void add_parameters(std::map<std::string, Input>& inputs, const std::vector<Symbol>& symbols,
                    const std::map<std::string, EncodedArray>& values, Domain domain,
                    const std::map<std::string, std::vector<double>>& generated) {
  for (const auto& s : symbols) {
    std::shared_ptr<const std::vector<double>> arr;
    auto g = generated.find(s.name);
    if (g != generated.end()) {
      arr = std::make_shared<std::vector<double>>(g->second);
    } else {
      auto it = values.find(s.name);
      check(it != values.end(), "missing parameter values for '" + s.name + "'");
      arr = decode_values(it->second);
    }
    if (s.index_domain == IndexDomain::Scalar) {
      check(!arr->empty(), "empty scalar parameter '" + s.name + "'");
      inputs[s.name] = Input::constant((*arr)[0], s.dtype);
    } else {
      Input in = Input::make(Input::Kind::Parameter);
      in.values = arr;
      in.domain = domain;
      in.dtype = s.dtype;
      inputs[s.name] = in;
    }
  }
}

PopulationRuntime population_runtime(const Model& m, size_t index) {
  const PopulationDef& def = m.populations[index];
  const PopulationInstance& inst = m.population_instances[index];
  check(def.linked_variable_count == 0, "linked variables are outside the oracle's subset");
  check(!def.spatial, "spatial neurons are outside the simulated path");
  PopulationRuntime rt;
  std::map<std::string, size_t> state_indices;
  for (size_t i = 0; i < def.states.size(); ++i) {
    state_indices[def.states[i].name] = i;
    rt.states.push_back(StateArray::from_encoded(inst.initial_state.at(def.states[i].name)));
  }
  if (inst.refractory)
    rt.refractory = RefractoryRuntime{inst.refractory->initial_lastspike, inst.refractory->initial_not_refractory};
  std::map<std::string, Input> inputs;
  inputs["dt"] = Input::constant(def.dt, DType::F64);
  inputs["t"] = Input::make(Input::Kind::Time);
  inputs["N"] = Input::constant(double(def.count), DType::Index);
  Input iidx = Input::make(Input::Kind::Index);
  iidx.domain = Domain::Neuron;
  inputs["i"] = iidx;
  for (const auto& [name, idx] : state_indices) {
    Input s = Input::make(Input::Kind::State);
    s.index = idx;
    s.domain = Domain::Neuron;
    s.dtype = def.states[idx].dtype;
    inputs[name] = s;
  }
  if (rt.refractory) {
    inputs["lastspike"] = Input::make(Input::Kind::LastSpike);
    Input a = Input::make(Input::Kind::Available);
    a.domain = Domain::Neuron;
    inputs["not_refractory"] = a;
  }
  add_parameters(inputs, def.parameters, inst.parameters, Domain::Neuron, {});
  std::map<std::string, WriteTarget> writable;
  for (const auto& [name, idx] : state_indices) writable[name] = WriteTarget{WriteTarget::Kind::Neuron, idx};
  if (rt.refractory) writable["not_refractory"] = WriteTarget{WriteTarget::Kind::Available, 0};
  auto compile = [&](const CodeObject& c) { return Program::compile(c, inputs, writable, m.rng_seed, m.functions); };
  for (const auto& c : def.code_objects) {
    if (c.kind == "state_update") { if (!rt.update) rt.update = compile(c); }
    else if (c.kind == "subexpression_update") { if (!rt.subexpression_update) rt.subexpression_update = compile(c); }
    else if (c.kind == "threshold") rt.thresholds.push_back(compile(c));
    else if (c.kind == "poisson_input") rt.poisson_inputs.push_back(compile(c));
    else if (c.kind == "run_regularly") rt.regular.push_back(compile(c));
    else if (c.kind == "reset") rt.resets.push_back(compile(c));
    else throw Error("population code object kind '" + c.kind + "' is outside the oracle's subset");
  }
  if (inst.spike_generator)
    for (size_t k = 0; k < inst.spike_generator->spike_ticks.size(); ++k)
      rt.spike_schedule.push_back({inst.spike_generator->spike_ticks[k], inst.spike_generator->spike_indices[k]});
  std::map<std::string, size_t> parameter_indices;
  for (size_t i = 0; i < def.parameters.size(); ++i) parameter_indices[def.parameters[i].name] = i;
  auto monitor_value = [&](const std::string& name) {
    MonitorValue mv;
    auto s = state_indices.find(name);
    if (s != state_indices.end()) {
      mv.kind = MonitorKind::State;
      mv.state = s->second;
      return mv;
    }
    auto p = parameter_indices.find(name);
    check(p != parameter_indices.end(), "monitor symbol missing from population");
    const Symbol& sym = def.parameters[p->second];
    auto vals = decode_values(inst.parameters.at(name));
    if (sym.index_domain == IndexDomain::Scalar) {
      mv.kind = MonitorKind::Scalar;
      mv.scalar = (*vals)[0];
    } else {
      mv.kind = MonitorKind::Parameter;
      mv.values = vals;
    }
    return mv;
  };
  auto symbol_dtype = [&](const std::string& name) {
    for (const auto& s : def.states) if (s.name == name) return s.dtype;
    for (const auto& s : def.parameters) if (s.name == name) return s.dtype;
    throw Error("monitor symbol missing from population");
  };
  for (const auto& name : def.monitor.variables) {
    rt.monitor_values.push_back(monitor_value(name));
    rt.samples.push_back(StateArray::empty(symbol_dtype(name)));
  }
  for (const auto& em : def.event_monitors) {
    EventMonitorRuntime er;
    auto it = std::find(def.events.begin(), def.events.end(), em.event);
    check(it != def.events.end(), "EventMonitor event missing from population");
    er.event_index = size_t(it - def.events.begin());
    for (const auto& name : em.variables) {
      er.values.push_back(monitor_value(name));
      er.samples.push_back(StateArray::empty(symbol_dtype(name)));
    }
    rt.event_monitors.push_back(std::move(er));
  }
  rt.tick = m.run_clocks[def.clock].start_tick;
  rt.end_tick = rt.tick + def.steps;
  rt.fired.resize(def.events.size());
  rt.event_history.resize(def.events.size());
  rt.counts.assign(def.count, 0);
  return rt;
}

// edge_csr (executor.rs:6168-6183): stable counting sort of edge ids by endpoint.
void edge_csr(const std::vector<uint32_t>& indices, size_t count, std::vector<size_t>& offsets,
              std::vector<uint32_t>& edges) {
  offsets.assign(count + 1, 0);
  for (uint32_t i : indices) offsets[i + 1] += 1;
  for (size_t i = 0; i < count; ++i) offsets[i + 1] += offsets[i];
  std::vector<size_t> next(offsets.begin(), offsets.end() - 1);
  edges.assign(indices.size(), 0);
  for (size_t e = 0; e < indices.size(); ++e) edges[next[indices[e]]++] = uint32_t(e);
}

// Worker threads for the one-time topology build (not the timed tick loop,
// which stays single-threaded like b2-runner): at most the host's hardware
// threads, one per 4096 targets.
unsigned build_threads(uint64_t targets) {
  unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  return unsigned(std::max<uint64_t>(1, std::min<uint64_t>({uint64_t(hw), 64, targets / 4096 + 1})));
}

template <class F>
void parallel_chunks(unsigned n, F f) {
  if (n == 1) {
    f(0u);
    return;
  }
  std::vector<std::thread> pool;
  for (unsigned c = 0; c < n; ++c) pool.emplace_back(f, c);
  for (auto& t : pool) t.join();
}

std::vector<double> materialize_initializer(uint64_t edge_count, uint64_t seed, const Initializer& init,
                                            std::optional<double> delay_dt = std::nullopt) {
  std::vector<double> out(edge_count);
  if (init.kind == Initializer::Kind::Uniform) {
    double lo = *init.minimum, hi = *init.maximum;
    for (uint64_t e = 0; e < edge_count; ++e) out[e] = lo + (hi - lo) * topo_uniform_open(seed, init.stream, e, 0);
    return out;
  }
  std::optional<double> lo = init.minimum, hi = init.maximum;
  if (delay_dt) {  // materialize_delay_initializer (executor.rs:160-188)
    lo = std::fmax(lo.value_or(0.0), 0.0);
    hi = hi.value_or(*delay_dt * 1000000.0);
  }
  for (uint64_t e = 0; e < edge_count; ++e) {
    bool found = false;
    for (uint64_t attempt = 0; attempt < 1000; ++attempt) {
      double v = init.mean + init.std * topo_normal(seed, init.stream, e, attempt);
      if ((!lo || v >= *lo) && (!hi || v <= *hi)) {
        out[e] = v;
        found = true;
        break;
      }
    }
    check(found, "clipped-normal rejection limit exceeded");
  }
  return out;
}

// materialize_projection (executor.rs:19-137)
void materialize_projection(const Model& m, const SynapseDef& def, const SynapseInstance& inst,
                            std::vector<uint32_t>& source, std::vector<uint32_t>& target,
                            std::map<std::string, std::vector<double>>& params,
                            std::vector<std::vector<size_t>>& delays) {
  const Topology& t = inst.topology;
  // 32-bit edge and endpoint storage (the reference keeps usize; the
  // values are the same while they fit)
  check(def.source_count <= UINT32_MAX && def.target_count <= UINT32_MAX && t.edge_count <= UINT32_MAX &&
            inst.source.size() <= UINT32_MAX,
        "projections beyond 2^32 edges or neurons are outside the oracle's subset");
  switch (t.kind) {
    case Topology::Kind::Explicit:
      source.assign(inst.source.begin(), inst.source.end());
      target.assign(inst.target.begin(), inst.target.end());
      for (const auto& p : inst.pathways) delays.push_back(p.delay_ticks);
      return;
    case Topology::Kind::BinaryCsr: {
      // executor.rs:35-57: source-major edges in file order, mapped columns
      // as per-edge parameters, the pathways' scalar delays
      BinaryCsr csr = read_binary_csr(t.path, def.source_count, def.target_count, t.edge_count, t.column_count,
                                      t.sha256, true);
      source.assign(csr.source.begin(), csr.source.end());
      target.assign(csr.target.begin(), csr.target.end());
      for (const auto& [name, col] : t.columns) params[name] = csr.columns[size_t(col)];
      for (const auto& p : inst.pathways) delays.push_back(p.delay_ticks);
      return;
    }
    case Topology::Kind::FixedTotal: {
      uint64_t S = def.source_count, T = def.target_count, E = t.edge_count;
      check(S && T && E && E <= UINT32_MAX, "invalid fixed-total topology specification");
      std::vector<uint32_t> counts(S, 0);
      for (uint64_t e = 0; e < E; ++e) counts[topo_bounded(t.seed, 0, e, S)]++;
      std::vector<uint64_t> cursor(S, 0);
      for (uint64_t s = 1; s < S; ++s) cursor[s] = cursor[s - 1] + counts[s - 1];
      source.assign(E, 0);
      target.assign(E, 0);
      for (uint64_t e = 0; e < E; ++e) {
        uint64_t s = topo_bounded(t.seed, 0, e, S);
        uint64_t pos = cursor[s]++;
        source[pos] = s;
        target[pos] = topo_bounded(t.seed, 1, e, T);
      }
      break;
    }
    case Topology::Kind::FixedIndegree: {
      uint64_t S = def.source_count, T = def.target_count, K = t.indegree;
      check(S && T && K && K <= S && T * K <= UINT32_MAX, "invalid fixed-indegree topology specification");
      check(T * K == t.edge_count, "fixed-indegree edge count mismatch");
      // Stable counting sort of the target-major draws by source, as the
      // serial two passes would do it, split over target ranges: chunk c's
      // edges of source s start after the earlier chunks' edges of s.
      const unsigned nth = build_threads(T);
      std::vector<std::vector<uint32_t>> cursor(nth, std::vector<uint32_t>(S, 0));
      auto targets_of = [&](unsigned c) { return std::make_pair(T * c / nth, T * (c + 1) / nth); };
      parallel_chunks(nth, [&](unsigned c) {
        FloydSet selected(K);
        auto [a, b] = targets_of(c);
        for (uint64_t tg = a; tg < b; ++tg)
          fixed_indegree_sources(S, K, tg, t.seed, selected, [&](uint64_t s) { cursor[c][s]++; });
      });
      uint64_t acc = 0;
      for (uint64_t s = 0; s < S; ++s)
        for (unsigned c = 0; c < nth; ++c) {
          const uint32_t n = cursor[c][s];
          cursor[c][s] = uint32_t(acc);
          acc += n;
        }
      source.assign(T * K, 0);
      target.assign(T * K, 0);
      parallel_chunks(nth, [&](unsigned c) {
        FloydSet selected(K);
        auto [a, b] = targets_of(c);
        for (uint64_t tg = a; tg < b; ++tg)
          fixed_indegree_sources(S, K, tg, t.seed, selected, [&](uint64_t s) {
            uint64_t pos = cursor[c][s]++;
            source[pos] = uint32_t(s);
            target[pos] = uint32_t(tg);
          });
      });
      break;
    }
  }
  for (const auto& [name, init] : t.initializers) params[name] = materialize_initializer(t.edge_count, t.seed, init);
  for (const auto& p : inst.pathways) {
    if (p.delay_initializer) {
      double dt = p.kind == "pre" ? m.populations[def.source_population].dt : m.populations[def.target_population].dt;
      const Initializer& di = *p.delay_initializer;
      // materialize_uniform_ticks validates before drawing
      if (di.kind == Initializer::Kind::Uniform)
        check(std::isfinite(*di.minimum) && std::isfinite(*di.maximum) && *di.minimum >= 0.0 &&
                  *di.minimum <= *di.maximum && std::isfinite(dt) && dt > 0.0 && *di.maximum / dt < 1000001.0,
              "invalid uniform delay initializer");
      auto d = materialize_initializer(t.edge_count, t.seed, *p.delay_initializer, dt);
      std::vector<size_t> ticks(d.size());
      for (size_t e = 0; e < d.size(); ++e) ticks[e] = size_t(std::floor(d[e] / dt + 0.5));
      delays.push_back(std::move(ticks));
    } else {
      delays.push_back(p.delay_ticks);
    }
  }
}

struct Runtime {
  const Model& m;
  std::vector<PopulationRuntime> populations;
  std::vector<SynapseRuntime> synapses;
  std::vector<size_t> clock_ticks, clock_end_ticks;
  double clock_epsilon = 0.0;

  explicit Runtime(const Model& model) : m(model) {
    for (size_t p = 0; p < m.populations.size(); ++p) populations.push_back(population_runtime(m, p));
    for (size_t s = 0; s < m.synapses.size(); ++s) synapses.push_back(build_synapse(s));
    for (const auto& c : m.run_clocks) {
      clock_ticks.push_back(c.start_tick);
      clock_end_ticks.push_back(c.start_tick + c.steps);
    }
    double min_dt = INFINITY;
    for (const auto& c : m.clocks) min_dt = std::fmin(min_dt, c.dt);
    clock_epsilon = min_dt * 1e-12;
  }

  SynapseRuntime build_synapse(size_t index) {
    const SynapseDef& def = m.synapses[index];
    const SynapseInstance& inst = m.synapse_instances[index];
    check(!def.source_synapse && !def.target_synapse, "synapse-to-synapse projections are outside the oracle's subset");
    check(def.linked_variable_count == 0, "synaptic linked variables are outside the oracle's subset");
    SynapseRuntime rt;
    std::map<std::string, std::vector<double>> generated;
    std::vector<std::vector<size_t>> delays;
    materialize_projection(m, def, inst, rt.source, rt.target, generated, delays);
    const PopulationDef& src = m.populations[def.source_population];
    const PopulationDef& tgt = m.populations[def.target_population];
    std::map<std::string, size_t> src_idx, tgt_idx, syn_idx;
    for (size_t i = 0; i < src.states.size(); ++i) src_idx[src.states[i].name] = i;
    for (size_t i = 0; i < tgt.states.size(); ++i) tgt_idx[tgt.states[i].name] = i;
    for (size_t i = 0; i < def.states.size(); ++i) {
      syn_idx[def.states[i].name] = i;
      auto it = inst.initial_state.find(def.states[i].name);
      check(it != inst.initial_state.end() && it->second.size() == rt.source.size(),
            "synapse state '" + def.states[i].name + "' has the wrong length");
      rt.states.push_back(StateArray::from_encoded(it->second));
    }
    std::map<std::string, Input> inputs;
    inputs["dt"] = Input::constant(src.dt, DType::F64);
    inputs["t"] = Input::make(Input::Kind::Time);
    inputs["N"] = Input::constant(double(rt.source.size()), DType::Index);
    inputs["N_pre"] = Input::constant(double(def.source_count), DType::Index);
    inputs["N_post"] = Input::constant(double(def.target_count), DType::Index);
    Input ii = Input::make(Input::Kind::Index);
    ii.domain = Domain::Pre;
    inputs["i"] = ii;
    Input jj = Input::make(Input::Kind::Index);
    jj.domain = Domain::Post;
    inputs["j"] = jj;
    for (const auto& [name, pos] : syn_idx) {
      Input s = Input::make(Input::Kind::SynapseState);
      s.index = pos;
      s.dtype = def.states[pos].dtype;
      inputs[name] = s;
    }
    std::map<std::string, WriteTarget> writable;
    for (const auto& [alias, state] : def.pre_state_aliases) {
      size_t pos = src_idx.at(state);
      Input s = Input::make(Input::Kind::PreState);
      s.index = pos;
      s.dtype = src.states[pos].dtype;
      inputs[alias] = s;
      writable[alias] = WriteTarget{WriteTarget::Kind::PreNeuron, pos};
    }
    for (const auto& [alias, state] : def.post_state_aliases) {
      size_t pos = tgt_idx.at(state);
      Input s = Input::make(Input::Kind::PostState);
      s.index = pos;
      s.dtype = tgt.states[pos].dtype;
      inputs[alias] = s;
      writable[alias] = WriteTarget{WriteTarget::Kind::Neuron, pos};
    }
    for (const auto& [name, pos] : syn_idx) writable[name] = WriteTarget{WriteTarget::Kind::Synapse, pos};
    if (tgt.refractory) {
      Input a = Input::make(Input::Kind::Available);
      a.domain = Domain::Post;
      inputs["not_refractory_post"] = a;
    }
    add_parameters(inputs, def.parameters, inst.parameters, Domain::Edge, generated);
    std::map<std::string, WriteTarget> post_writable;
    for (const auto& [name, pos] : syn_idx) post_writable[name] = WriteTarget{WriteTarget::Kind::Synapse, pos};
    for (const auto& [alias, state] : def.post_state_aliases)
      post_writable[alias] = WriteTarget{WriteTarget::Kind::Neuron, tgt_idx.at(state)};
    for (const auto& c : def.code_objects)
      check(c.kind == "synapses" || c.kind == "synapses_post" || c.kind == "summed_variable" ||
                c.kind == "synapse_state_update" || c.kind == "synapse_subexpression_update" ||
                c.kind == "synapse_run_regularly",
            "synapse code object kind '" + c.kind + "' is outside the oracle's subset");
    {
      std::map<std::string, WriteTarget> clock_driven;
      for (const auto& name : def.clock_driven_states) {
        check(syn_idx.count(name) > 0, "clock-driven state is not a synapse state");
        clock_driven[name] = WriteTarget{WriteTarget::Kind::Synapse, syn_idx.at(name)};
      }
      for (const auto& c : def.code_objects) {
        if (c.kind == "synapse_state_update" && !rt.update)
          rt.update = Program::compile(c, inputs, clock_driven, m.rng_seed, m.functions);
        else if (c.kind == "synapse_subexpression_update" && !rt.subexpression)
          rt.subexpression = Program::compile(c, inputs, writable, m.rng_seed, m.functions);
        else if (c.kind == "synapse_run_regularly")
          rt.regular.push_back(Program::compile(c, inputs, writable, m.rng_seed, m.functions));
      }
    }
    // summed variables (executor.rs:3657-3731): compiled with no writable
    // symbol; `_synaptic_var` is the per-edge value
    for (const auto& c : def.code_objects) {
      if (c.kind != "summed_variable") continue;
      const bool to_pre = c.summed_target && *c.summed_target == "pre";
      const size_t tp = to_pre ? def.source_population : def.target_population;
      const PopulationDef& tdef = m.populations[tp];
      check(bool(c.summed_state), "missing summed target state");
      size_t ts = tdef.states.size();
      for (size_t i = 0; i < tdef.states.size(); ++i)
        if (tdef.states[i].name == *c.summed_state) ts = i;
      check(ts < tdef.states.size(), "missing summed target state");
      check(tdef.states[ts].dtype == DType::F64 || tdef.states[ts].dtype == DType::F32,
            "summed variables require floating-point state");
      auto sin = inputs;
      sin["dt"] = Input::constant(tdef.dt, DType::F64);
      SummedRuntime sr{Program::compile(c, sin, {}, m.rng_seed, m.functions), 0, tp,
                       to_pre ? def.source_start : def.target_start, to_pre ? def.source_count : def.target_count, ts,
                       to_pre};
      auto r = sr.program.symbols.find("_synaptic_var");
      check(r != sr.program.symbols.end(), "missing summed expression result");
      sr.result = r->second;
      rt.summed.push_back(std::move(sr));
    }
    for (size_t k = 0; k < inst.pathways.size(); ++k) {
      const PathwayInstance& pw = inst.pathways[k];
      bool is_pre = pw.kind == "pre";
      const CodeObject* code = nullptr;
      for (const auto& c : def.code_objects)
        if (c.pathway_name && *c.pathway_name == pw.name) code = &c;
      check(code != nullptr, "missing pathway code object");
      const PopulationDef& endpoint = m.populations[is_pre ? def.source_population : def.target_population];
      auto pin = inputs;
      pin["dt"] = Input::constant(endpoint.dt, DType::F64);
      PathwayRuntime pr{Program::compile(*code, pin, is_pre ? writable : post_writable, m.rng_seed, m.functions),
                        {}, delays[k], is_pre, 0, {}};
      // PathwayQueue::new (executor.rs:6186-6211)
      const auto& idx = is_pre ? rt.source : rt.target;
      edge_csr(idx, is_pre ? def.source_count : def.target_count, pr.topology.offsets, pr.topology.edges);
      const auto& d = pr.delay_ticks;
      if (!d.empty() && std::all_of(d.begin(), d.end(), [&](size_t x) { return x == d[0]; }))
        pr.topology.uniform_delay = d[0];
      size_t max_delay = d.empty() ? 0 : *std::max_element(d.begin(), d.end());
      size_t slots = std::min(max_delay + 1, endpoint.steps);
      check(slots > 0, "pathway queue has no slots");
      pr.topology.queue.resize(slots);
      for (const auto& ev : pw.pending) pr.topology.queue[ev.delivery_tick % slots].push_back(ev.item);
      if (!pr.topology.uniform_delay) check(d.size() == rt.source.size(), "per-edge delay array has the wrong length");
      auto it = std::find(endpoint.events.begin(), endpoint.events.end(), pw.event);
      check(it != endpoint.events.end(), "pathway event missing from endpoint");
      pr.event_index = size_t(it - endpoint.events.begin());
      rt.pathways.push_back(std::move(pr));
    }
    return rt;
  }

  // deliver_event (executor.rs:2166-2251)
  void deliver_event(Program& prog, const SynapseDef& def, SynapseRuntime& syn, size_t source, size_t target, size_t edge) {
    Batch b;
    b.len = 1;
    b.source = source;
    b.target = target;
    b.source_state = source + def.source_start;
    b.target_state = target + def.target_start;
    b.edge = edge;
    PopulationRuntime& sp = populations[def.source_population];
    PopulationRuntime& tp = populations[def.target_population];
    const RefractoryRuntime* refr = tp.refractory ? &*tp.refractory : nullptr;
    prog.run(tp.states, sp.states, tp.states, syn.states, refr, b);
    // Same-population pathways write pre and post aliases into one table.
    prog.commit_event(&sp.states, tp.states, syn.states, b.source_state, b.target_state, edge);
  }

  // run_synapse_program (executor.rs:2513-2546): every edge in creation
  // order, committing only synapse-state writes
  void run_synapse_program(Program& prog, const SynapseDef& def, SynapseRuntime& syn, double time, size_t tick) {
    prog.prepare(time, tick);
    PopulationRuntime& sp = populations[def.source_population];
    PopulationRuntime& tp = populations[def.target_population];
    const RefractoryRuntime* refr = tp.refractory ? &*tp.refractory : nullptr;
    for (size_t edge = 0; edge < syn.source.size(); ++edge) {
      Batch b;
      b.len = 1;
      b.source = syn.source[edge];
      b.target = syn.target[edge];
      b.source_state = b.source + def.source_start;
      b.target_state = b.target + def.target_start;
      b.edge = edge;
      prog.run(tp.states, sp.states, tp.states, syn.states, refr, b);
      prog.commit_synapses(syn.states, edge);
    }
  }

  // run_summed_program (executor.rs:2548-2597): clear the endpoint range,
  // then add each edge's value in creation order (f32 targets round each
  // addition, StateArray::add_f64 executor.rs:517-523)
  void run_summed(SummedRuntime& s, const SynapseDef& def, SynapseRuntime& syn, double time) {
    PopulationRuntime& dest_pop = populations[s.target_population];
    StateArray& dest = dest_pop.states[s.target_state];
    for (size_t i = s.target_start; i < s.target_start + s.target_count; ++i) dest.set(i, 0.0);
    s.program.prepare(time, dest_pop.tick);
    PopulationRuntime& sp = populations[def.source_population];
    PopulationRuntime& tp = populations[def.target_population];
    const RefractoryRuntime* refr = tp.refractory ? &*tp.refractory : nullptr;
    for (size_t edge = 0; edge < syn.source.size(); ++edge) {
      Batch b;
      b.len = 1;
      b.source = syn.source[edge];
      b.target = syn.target[edge];
      b.source_state = b.source + def.source_start;
      b.target_state = b.target + def.target_start;
      b.edge = edge;
      s.program.run(tp.states, sp.states, tp.states, syn.states, refr, b);
      const size_t at = s.target_is_pre ? b.source_state : b.target_state;
      dest.set(at, dest.get(at) + s.program.registers[s.result][0]);
    }
  }

  // run_pathway (executor.rs:2292-2382)
  void run_pathway(PathwayRuntime& pw, const SynapseDef& def, SynapseRuntime& syn, double time) {
    size_t endpoint_pop = pw.is_pre ? def.source_population : def.target_population;
    size_t endpoint_start = pw.is_pre ? def.source_start : def.target_start;
    size_t endpoint_count = pw.is_pre ? def.source_count : def.target_count;
    size_t tick = populations[endpoint_pop].tick;
    size_t end_tick = populations[endpoint_pop].end_tick;
    pw.active_sources.clear();
    for (size_t neuron : populations[endpoint_pop].fired[pw.event_index])
      if (neuron >= endpoint_start && neuron < endpoint_start + endpoint_count)
        pw.active_sources.push_back(neuron - endpoint_start);
    auto& q = pw.topology;
    size_t qsize = q.queue.size();
    if (q.uniform_delay) {
      size_t delivery = tick + *q.uniform_delay;
      if (delivery < end_tick) {
        auto& slot = q.queue[delivery % qsize];
        slot.insert(slot.end(), pw.active_sources.begin(), pw.active_sources.end());
      }
    } else {
      for (size_t ep : pw.active_sources)
        for (size_t k = q.offsets[ep]; k < q.offsets[ep + 1]; ++k) {
          size_t edge = q.edges[k];
          size_t delivery = tick + pw.delay_ticks[edge];
          if (delivery < end_tick) q.queue[delivery % qsize].push_back(edge);
        }
    }
    std::vector<size_t> pending;
    pending.swap(q.queue[tick % qsize]);
    pw.program.prepare(time, tick);
    if (q.uniform_delay) {
      for (size_t ep : pending)
        for (size_t k = q.offsets[ep]; k < q.offsets[ep + 1]; ++k) {
          size_t edge = q.edges[k];
          deliver_event(pw.program, def, syn, syn.source[edge], syn.target[edge], edge);
          q.delivered += 1;
        }
    } else {
      for (size_t edge : pending) {
        deliver_event(pw.program, def, syn, syn.source[edge], syn.target[edge], edge);
        q.delivered += 1;
      }
    }
    pending.clear();
    q.queue[tick % qsize].swap(pending);
  }

  // emit_threshold (executor.rs:2949-3006)
  void emit_threshold(PopulationRuntime& rt, const PopulationDef& def, size_t position, size_t event_index,
                      bool is_spike, double time) {
    rt.fired[event_index].clear();
    check(position < rt.thresholds.size(), "scheduled threshold has no runtime program");
    Program& th = rt.thresholds[position];
    th.prepare(time, rt.tick);
    check(th.condition >= 0, "missing threshold condition");
    for (size_t start = 0; start < def.count; start += LANES) {
      size_t len = std::min(LANES, def.count - start);
      th.run(rt.states, rt.states, rt.states, {}, rt.refractory ? &*rt.refractory : nullptr, Batch::neurons(start, len));
      for (size_t l = 0; l < len; ++l) {
        size_t neuron = start + l;
        if (th.registers[size_t(th.condition)][l] != 0.0 &&
            (!is_spike || !rt.refractory || rt.refractory->not_refractory[neuron])) {
          rt.fired[event_index].push_back(neuron);
          if (is_spike && rt.refractory) {
            rt.refractory->lastspike[neuron] = time;
            rt.refractory->not_refractory[neuron] = 0;
          }
        }
      }
    }
    if (rt.tick >= rt.end_tick - def.monitor.window_steps) {
      check(rt.event_history[event_index].size() + rt.fired[event_index].size() <= 10000000,
            "event stream recording budget exceeded");
      for (size_t n : rt.fired[event_index]) rt.event_history[event_index].push_back({rt.tick, n});
    }
  }

  double monitor_sample(const PopulationRuntime& rt, const MonitorValue& v, size_t neuron) {
    switch (v.kind) {
      case MonitorKind::State: return rt.states[v.state].get(neuron);
      case MonitorKind::Scalar: return v.scalar;
      case MonitorKind::Parameter: return (*v.values)[neuron];
    }
    return 0.0;
  }

  void run_program_neurons(Program& p, PopulationRuntime& rt, size_t count, double time, size_t tick) {
    p.prepare(time, tick);
    for (size_t start = 0; start < count; start += LANES) {
      size_t len = std::min(LANES, count - start);
      p.run(rt.states, rt.states, rt.states, {}, rt.refractory ? &*rt.refractory : nullptr, Batch::neurons(start, len));
      p.commit_neurons(rt.states, start, len);
    }
  }

  static size_t kind_position(const std::vector<CodeObject>& codes, size_t item, const char* kind) {
    size_t n = 0;
    for (size_t k = 0; k < item; ++k) n += codes[k].kind == kind;
    return n;
  }

  uint64_t advance(uint64_t max_ticks) {
    uint64_t ticks = 0;
    for (; ticks < max_ticks; ++ticks) {
      std::optional<double> next;
      for (size_t c = 0; c < m.clocks.size(); ++c)
        if (clock_ticks[c] < clock_end_ticks[c]) {
          double t = double(clock_ticks[c]) * m.clocks[c].dt;
          next = next ? std::fmin(*next, t) : t;
        }
      if (!next) break;
      std::vector<bool> active(m.clocks.size(), false);
      for (size_t c = 0; c < m.clocks.size(); ++c)
        if (clock_ticks[c] < clock_end_ticks[c])
          active[c] = std::fabs(double(clock_ticks[c]) * m.clocks[c].dt - *next) <= clock_epsilon;
      check(!m.schedule.empty(), "model has no schedule");
      std::vector<bool> recorded(populations.size(), false);
      for (const auto& node : m.schedule) {
        if (!active[node.clock]) continue;
        size_t owner_clock = node.owner_kind == OwnerKind::Population ? m.populations[node.owner_index].clock : node.clock;
        double time = double(clock_ticks[owner_clock]) * m.clocks[owner_clock].dt;
        if (node.owner_kind == OwnerKind::Population) {
          PopulationRuntime& rt = populations[node.owner_index];
          const PopulationDef& def = m.populations[node.owner_index];
          switch (node.operation) {
            case ScheduleOp::StateMonitor:
              if (!recorded[node.owner_index]) {
                if (rt.tick >= rt.end_tick - def.monitor.window_steps)
                  for (size_t neuron : def.monitor.record)
                    for (size_t k = 0; k < rt.samples.size(); ++k)
                      rt.samples[k].push(monitor_sample(rt, rt.monitor_values[k], neuron));
                recorded[node.owner_index] = true;
              }
              break;
            case ScheduleOp::SpikeMonitor: {
              if (rt.tick < rt.end_tick - def.monitor.window_steps) break;
              auto it = std::find(def.events.begin(), def.events.end(), "spike");
              check(it != def.events.end(), "SpikeMonitor without spike event");
              for (size_t n : rt.fired[size_t(it - def.events.begin())]) {
                rt.counts[n] += 1;
                rt.spikes.push_back({rt.tick, n});
              }
              break;
            }
            case ScheduleOp::EventMonitor: {
              check(node.item_index < rt.event_monitors.size(), "scheduled EventMonitor has no runtime state");
              auto& mon = rt.event_monitors[node.item_index];
              auto fired = rt.fired[mon.event_index];
              for (size_t n : fired) {
                mon.events.push_back({rt.tick, n});
                for (size_t k = 0; k < mon.samples.size(); ++k) mon.samples[k].push(monitor_sample(rt, mon.values[k], n));
              }
              break;
            }
            case ScheduleOp::EventSource: {
              rt.fired[0].clear();
              while (rt.spike_cursor < rt.spike_schedule.size() && rt.spike_schedule[rt.spike_cursor].first < rt.tick)
                rt.spike_cursor++;
              while (rt.spike_cursor < rt.spike_schedule.size() && rt.spike_schedule[rt.spike_cursor].first == rt.tick)
                rt.fired[0].push_back(rt.spike_schedule[rt.spike_cursor++].second);
              if (rt.tick >= rt.end_tick - def.monitor.window_steps)
                for (size_t n : rt.fired[0]) rt.event_history[0].push_back({rt.tick, n});
              break;
            }
            case ScheduleOp::CodeObject: {
              const CodeObject& code = def.code_objects[node.item_index];
              size_t tick = clock_ticks[node.clock];
              if (code.kind == "subexpression_update") {
                check(bool(rt.subexpression_update), "missing population subexpression program");
                run_program_neurons(*rt.subexpression_update, rt, def.count, time, tick);
              } else if (code.kind == "state_update") {
                if (def.refractory && def.refractory->mode == "fixed" && rt.refractory) {
                  uint64_t period = m.population_instances[node.owner_index].refractory->period_ticks;
                  for (size_t n = 0; n < def.count; ++n)
                    rt.refractory->not_refractory[n] = timestep(time - rt.refractory->lastspike[n], def.dt) >= period;
                }
                check(bool(rt.update), "missing population state program");
                Program& p = *rt.update;
                p.prepare(time, tick);
                for (size_t start = 0; start < def.count; start += LANES) {
                  size_t len = std::min(LANES, def.count - start);
                  p.run(rt.states, rt.states, rt.states, {}, rt.refractory ? &*rt.refractory : nullptr, Batch::neurons(start, len));
                  p.commit_neurons(rt.states, start, len);
                  if (rt.refractory) p.commit_available(*rt.refractory, start, len);
                }
              } else if (code.kind == "threshold") {
                check(bool(code.event_name), "scheduled threshold has no event");
                auto it = std::find(def.events.begin(), def.events.end(), *code.event_name);
                check(it != def.events.end(), "scheduled threshold event is unknown");
                emit_threshold(rt, def, kind_position(def.code_objects, node.item_index, "threshold"),
                               size_t(it - def.events.begin()), *code.event_name == "spike", time);
              } else if (code.kind == "poisson_input") {
                run_program_neurons(rt.poisson_inputs.at(kind_position(def.code_objects, node.item_index, "poisson_input")),
                                    rt, def.count, time, tick);
              } else if (code.kind == "run_regularly") {
                run_program_neurons(rt.regular.at(kind_position(def.code_objects, node.item_index, "run_regularly")),
                                    rt, def.count, time, tick);
              } else if (code.kind == "reset") {
                Program& reset = rt.resets.at(kind_position(def.code_objects, node.item_index, "reset"));
                check(bool(code.event_name), "scheduled reset has no event");
                auto it = std::find(def.events.begin(), def.events.end(), *code.event_name);
                check(it != def.events.end(), "scheduled reset event is unknown");
                reset.prepare(time, tick);
                for (size_t n : rt.fired[size_t(it - def.events.begin())]) {
                  reset.run(rt.states, rt.states, rt.states, {}, rt.refractory ? &*rt.refractory : nullptr, Batch::neurons(n, 1));
                  reset.commit_neurons(rt.states, n, 1);
                }
              } else {
                throw Error("unsupported scheduled population operation");
              }
              break;
            }
          }
        } else {
          check(node.operation == ScheduleOp::CodeObject, "synapse monitors are outside the oracle's subset");
          const SynapseDef& def = m.synapses[node.owner_index];
          const CodeObject& code = def.code_objects[node.item_index];
          if (code.kind == "synapse_state_update" || code.kind == "synapse_subexpression_update" ||
              code.kind == "synapse_run_regularly") {
            SynapseRuntime& syn = synapses[node.owner_index];
            Program* prog = nullptr;
            if (code.kind == "synapse_state_update") prog = syn.update ? &*syn.update : nullptr;
            else if (code.kind == "synapse_subexpression_update") prog = syn.subexpression ? &*syn.subexpression : nullptr;
            else {
              size_t position = 0;
              for (size_t k = 0; k < node.item_index; ++k) position += def.code_objects[k].kind == "synapse_run_regularly";
              if (position < syn.regular.size()) prog = &syn.regular[position];
            }
            check(prog != nullptr, "missing synapse program");
            run_synapse_program(*prog, def, syn, time, clock_ticks[node.clock]);
            continue;
          }
          if (code.kind == "summed_variable") {
            size_t position = 0;
            for (size_t k = 0; k < node.item_index; ++k) position += def.code_objects[k].kind == "summed_variable";
            SynapseRuntime& syn = synapses[node.owner_index];
            check(position < syn.summed.size(), "missing summed-variable runtime program");
            run_summed(syn.summed[position], def, syn, time);
            continue;
          }
          check(code.kind == "synapses" || code.kind == "synapses_post", "unsupported scheduled synapse operation");
          check(bool(code.pathway_name), "scheduled pathway has no name");
          const auto& pws = m.synapse_instances[node.owner_index].pathways;
          size_t pos = pws.size();
          for (size_t k = 0; k < pws.size(); ++k)
            if (pws[k].name == *code.pathway_name) pos = k;
          check(pos < pws.size(), "scheduled pathway has no runtime instance");
          SynapseRuntime& syn = synapses[node.owner_index];
          run_pathway(syn.pathways[pos], def, syn, time);
        }
      }
      for (size_t p = 0; p < populations.size(); ++p) {
        const PopulationDef& def = m.populations[p];
        if (!active[def.clock]) continue;
        auto it = std::find(def.events.begin(), def.events.end(), "spike");
        auto& rt = populations[p];
        rt.last_fired.clear();
        if (it != def.events.end())
          for (size_t n : rt.fired[size_t(it - def.events.begin())]) rt.last_fired.push_back(n);
        rt.tick = clock_ticks[def.clock] + 1;
      }
      for (size_t c = 0; c < clock_ticks.size(); ++c) clock_ticks[c] += active[c] ? 1 : 0;
    }
    return ticks;
  }

  bool finished() const {
    for (size_t c = 0; c < clock_ticks.size(); ++c)
      if (clock_ticks[c] < clock_end_ticks[c]) return false;
    return true;
  }

  b2dump::ResultSet results() const {
    b2dump::ResultSet r;
    r.neuron_count = m.neuron_count;
    r.final_time = m.run_start + m.run_duration;
    for (size_t p = 0; p < populations.size(); ++p) {
      const auto& def = m.populations[p];
      const auto& rt = populations[p];
      r.has_events |= !def.events.empty() || !def.event_monitors.empty();
      b2dump::PopulationResult pr;
      pr.count = def.count;
      pr.steps = def.steps;
      pr.record_count = def.monitor.record.size();
      pr.variable_count = def.monitor.variables.size();
      for (const auto& s : rt.samples) pr.samples.push_back(s.column());
      pr.spikes = rt.spikes;
      pr.counts = rt.counts;
      pr.last_fired = rt.last_fired;
      for (const auto& s : rt.states) pr.states.push_back(s.column());
      if (rt.refractory) {
        pr.has_refractory = true;
        pr.lastspike = rt.refractory->lastspike;
        pr.not_refractory = rt.refractory->not_refractory;
      }
      pr.event_history = rt.event_history;
      for (const auto& em : rt.event_monitors) {
        b2dump::EventMonitorResult er;
        er.events = em.events;
        for (const auto& s : em.samples) er.samples.push_back(s.column());
        pr.event_monitors.push_back(std::move(er));
      }
      r.populations.push_back(std::move(pr));
    }
    for (const auto& s : synapses) {
      b2dump::SynapseResult sr;
      sr.edge_count = s.source.size();
      for (const auto& st : s.states) sr.states.push_back(st.column());
      for (const auto& pw : s.pathways) sr.delivered += pw.topology.delivered;
      r.synapses.push_back(std::move(sr));
    }
    return r;
  }
};

}  // namespace

TimedSample timed_sample(const Model& model, uint64_t warmup, uint64_t timed) {
  TimedSample s;
  auto t0 = std::chrono::steady_clock::now();
  Runtime rt(model);
  auto t1 = std::chrono::steady_clock::now();
  s.build_seconds = std::chrono::duration<double>(t1 - t0).count();
  rt.advance(warmup);
  auto count = [&](uint64_t& events, uint64_t& spikes) {
    events = spikes = 0;
    for (const auto& syn : rt.synapses)
      for (const auto& pw : syn.pathways) events += pw.topology.delivered;
    for (const auto& p : rt.populations)
      for (const auto& h : p.event_history) spikes += h.size();
  };
  uint64_t e0, s0, e1, s1;
  count(e0, s0);
  auto t2 = std::chrono::steady_clock::now();
  s.ticks = rt.advance(timed);
  auto t3 = std::chrono::steady_clock::now();
  count(e1, s1);
  s.seconds = std::chrono::duration<double>(t3 - t2).count();
  s.synaptic_events = e1 - e0;
  s.spikes = s1 - s0;
  return s;
}

b2dump::ResultSet execute(const Model& model, RunStats* stats, uint64_t max_ticks) {
  for (const auto& p : model.populations)
    check(p.rate_monitor_count == 0, "rate monitors are outside the oracle's subset");
  Runtime rt(model);
  auto t0 = std::chrono::steady_clock::now();
  uint64_t ticks = rt.advance(max_ticks);
  auto t1 = std::chrono::steady_clock::now();
  if (stats) {
    stats->simulation_seconds = std::chrono::duration<double>(t1 - t0).count();
    stats->ticks = ticks;
  }
  if (max_ticks == UINT64_MAX) check(rt.finished(), "results require a completed execution");
  return rt.results();
}

}  // namespace oracle
