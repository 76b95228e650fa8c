// SSA construction, constant folding and CUDA emission for one CodeObject.
// Construction rules: brian2-rust/src/executor.rs:5046-5486 (compile,
// expression, statements).  Per-op semantics: executor.rs:5725-6158.
#include "program.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <sstream>

namespace b2gpu {

using b2ir::check;
using b2ir::Error;
using b2ir::Expr;
using b2ir::Op;

namespace {
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
// Error bits; keep in sync with device_lib.cuh.
constexpr uint32_t ERR_NONFINITE = 0x1, ERR_TIMESTEP = 0x2, ERR_BINOMIAL = 0x4, ERR_POISSON = 0x8,
                   ERR_INTDIV = 0x40, ERR_TIMEDARRAY = 0x80, ERR_CAST = 0x100;
}  // namespace

DType Input::type() const {
  switch (kind) {
    case Kind::Constant: case Kind::State: case Kind::PreState: case Kind::PostState:
    case Kind::SynapseState: case Kind::Parameter: return dtype;
    case Kind::Time: case Kind::LastSpike: case Kind::Random: case Kind::Normal: return DType::F64;
    case Kind::Index: return DType::Index;
    case Kind::Available: return DType::Bool;
  }
  return DType::F64;
}

Input Input::constant(double v, DType d) {
  Input i;
  i.kind = Kind::Constant;
  i.value = v;
  i.dtype = d;
  return i;
}

Input Input::make(Kind k, Domain d, size_t index, DType dtype) {
  Input i;
  i.kind = k;
  i.domain = d;
  i.index = index;
  i.dtype = dtype;
  return i;
}

// ------------------------------------------------------------------ compile
Program Program::compile(const b2ir::CodeObject& code, std::map<std::string, Input> inputs,
                         const std::map<std::string, WriteTarget>& writable,
                         const std::vector<b2ir::Function>& functions) {
  check(!code.adaptive, "adaptive integrators are not supported by the GPU engine");
  Program p;
  for (const auto& kv : inputs) p.symbol_dtypes[kv.first] = kv.second.type();
  p.inputs_ = std::move(inputs);
  for (const auto& f : functions) p.functions_[f.name] = &f;
  p.rng_domain = (code.iteration_domain == "all_synapses" || code.iteration_domain == "active_synapses")
                     ? Domain::Edge : Domain::Neuron;
  p.scalar = p.statements(code.scalar);
  for (const auto& b : p.bindings)
    if (b.second.kind == Input::Kind::Random || b.second.kind == Input::Kind::Normal)
      p.scalar_random.insert(b.first);
  p.vector = p.statements(code.vector);
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
  p.classify();
  return p;
}

size_t Program::reg() { return register_count++; }

size_t Program::input(const Input& v) {
  size_t slot = reg();
  bindings.push_back({slot, v});
  return slot;
}

size_t Program::resolve(const std::string& name) {
  auto it = symbols.find(name);
  if (it != symbols.end()) return it->second;
  auto in = inputs_.find(name);
  check(in != inputs_.end(), "missing plan input '" + name + "'");
  size_t slot = input(in->second);
  symbols[name] = slot;
  return slot;
}

DType Program::infer(const Expr& e) {
  switch (e.op) {
    case Op::Literal: return DType::F64;
    case Op::Boolean: return DType::Bool;
    case Op::Integer: case Op::Cast: return e.dtype;
    case Op::Rand: case Op::Randn: case Op::Binomial: case Op::Poisson: case Op::TimedArray:
    case Op::BoolToF64: case Op::IndexToF64: case Op::TickToF64: case Op::F32ToF64: return DType::F64;
    case Op::F64ToF32: return DType::F32;
    case Op::Timestep: case Op::TickOffset: return DType::Tick;
    case Op::Load: {
      auto it = symbol_dtypes.find(e.name);
      check(it != symbol_dtypes.end(), "undefined symbol: " + e.name);
      return it->second;
    }
    case Op::Call: {
      auto it = functions_.find(e.name);
      check(it != functions_.end(), "undefined function: " + e.name);
      return it->second->return_dtype;
    }
    case Op::Neg: case Op::Abs: return infer(*e.args[0]);
    case Op::Not: case Op::Eq: case Op::Ne: case Op::And: case Op::Or:
    case Op::Gt: case Op::Ge: case Op::Lt: case Op::Le: return DType::Bool;
    case Op::Add: case Op::Sub: case Op::Mul: case Op::Pow: case Op::Mod: case Op::FloorDiv: {
      DType l = infer(*e.args[0]), r = infer(*e.args[1]);
      return (l == r && b2ir::is_integer(l)) ? l : DType::F64;
    }
    default: return DType::F64;
  }
}

size_t Program::expression(const Expr& e, long guard, std::vector<Instr>& ops) {
  Instr ins;
  ins.guard = guard;
  switch (e.op) {
    case Op::Literal: return input(Input::constant(e.literal, DType::F64));
    case Op::Boolean: return input(Input::constant(e.boolean ? 1.0 : 0.0, DType::Bool));
    case Op::Integer: return input(Input::constant(from_bits(e.raw), e.dtype));
    case Op::Rand: {
      Input i = Input::make(Input::Kind::Random, rng_domain);
      i.stream = e.stream;
      return input(i);
    }
    case Op::Randn: {
      Input i = Input::make(Input::Kind::Normal, rng_domain);
      i.stream = e.stream;
      return input(i);
    }
    case Op::Load: return resolve(e.name);
    case Op::BoolToF64: case Op::IndexToF64: case Op::TickToF64: case Op::F32ToF64:
      return expression(*e.args[0], guard, ops);
    case Op::Call: {
      auto it = functions_.find(e.name);
      check(it != functions_.end(), "missing Function contract in execution plan");
      const b2ir::Function& fn = *it->second;
      check(fn.arguments.size() == e.args.size(), "function argument count does not match contract");
      check(bool(fn.body), "native-only Functions are not supported by the GPU engine");
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
      check(ins.src != DType::Index && ins.src != DType::Tick, "unsupported cast source");
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
      const size_t t = expression(*e.args[0], guard, ops);
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
      if (b2ir::is_unary_math(e.op)) {
        size_t slot = expression(*e.args[0], guard, ops);
        DType dt = infer(*e.args[0]);
        ins.left = ins.right = slot;
        static const std::pair<Op, IOp> map[] = {
            {Op::Not, IOp::Not}, {Op::Arccos, IOp::Arccos}, {Op::Arcsin, IOp::Arcsin},
            {Op::Arctan, IOp::Arctan}, {Op::Ceil, IOp::Ceil}, {Op::Cos, IOp::Cos}, {Op::Cosh, IOp::Cosh},
            {Op::Exp, IOp::Exp}, {Op::Expm1, IOp::Expm1}, {Op::Exprel, IOp::Exprel}, {Op::Floor, IOp::Floor},
            {Op::Trunc, IOp::Trunc}, {Op::Log, IOp::Log}, {Op::Log10, IOp::Log10}, {Op::Log1p, IOp::Log1p},
            {Op::Sign, IOp::Sign}, {Op::Sin, IOp::Sin}, {Op::Sinh, IOp::Sinh}, {Op::Sqrt, IOp::Sqrt},
            {Op::Tan, IOp::Tan}, {Op::Tanh, IOp::Tanh}};
        if (e.op == Op::Neg) {
          if (b2ir::is_integer(dt)) { ins.op = IOp::IntNeg; ins.dst = dt; } else ins.op = IOp::Neg;
        } else if (e.op == Op::Abs) {
          if (b2ir::is_integer(dt)) { ins.op = IOp::IntAbs; ins.dst = dt; } else ins.op = IOp::Abs;
        } else {
          bool found = false;
          for (const auto& m : map)
            if (m.first == e.op) { ins.op = m.second; found = true; }
          check(found, "unsupported unary op");
        }
      } else if (b2ir::is_binary(e.op)) {
        DType dt = infer(*e.args[0]);
        bool integer = b2ir::is_integer(dt);
        auto iop = [&](IntOp k, IOp f) {
          if (integer) { ins.op = IOp::IntBinary; ins.intop = k; ins.dst = dt; } else ins.op = f;
        };
        switch (e.op) {
          case Op::Add: iop(IntOp::Add, IOp::Add); break;
          case Op::Sub: iop(IntOp::Sub, IOp::Sub); break;
          case Op::Mul: iop(IntOp::Mul, IOp::Mul); break;
          case Op::Mod: iop(IntOp::Mod, IOp::Mod); break;
          case Op::FloorDiv: iop(IntOp::FloorDiv, IOp::FloorDiv); break;
          case Op::Gt: iop(IntOp::Gt, IOp::Gt); break;
          case Op::Ge: iop(IntOp::Ge, IOp::Ge); break;
          case Op::Lt: iop(IntOp::Lt, IOp::Lt); break;
          case Op::Le: iop(IntOp::Le, IOp::Le); break;
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
        throw Error(std::string("unsupported expression op ") + b2ir::op_name(e.op));
      }
  }
  ins.output = reg();
  ops.push_back(ins);
  return ins.output;
}

std::vector<Instr> Program::statements(const std::vector<b2ir::Statement>& sts) {
  std::vector<Instr> ops;
  for (const auto& st : sts) {
    long guard = st.condition ? long(resolve(*st.condition)) : -1;
    std::optional<size_t> old;
    if (guard >= 0) {
      auto s = symbols.find(st.target);
      if (s != symbols.end()) old = s->second;
      else if (inputs_.count(st.target)) old = resolve(st.target);
    }
    size_t value = expression(*st.value, guard, ops);
    size_t output = value;
    if (old) {
      Instr sel;
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

const Input* Program::binding_of(size_t r) const {
  for (const auto& b : bindings)
    if (b.first == r) return &b.second;
  return nullptr;
}

std::optional<size_t> Program::post_state_register(size_t index) const {
  for (const auto& b : bindings)
    if (b.second.kind == Input::Kind::PostState && b.second.index == index) return b.first;
  return std::nullopt;
}

bool Program::uses_rng() const {
  for (const auto& b : bindings)
    if (b.second.kind == Input::Kind::Random || b.second.kind == Input::Kind::Normal) return true;
  for (const auto* list : {&scalar, &vector})
    for (const auto& i : *list)
      if (i.op == IOp::Binomial || i.op == IOp::Poisson) return true;
  return false;
}

// ------------------------------------------------------------------ host eval
namespace {
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
uint64_t to64(DType src, uint64_t raw) {  // two's complement widening of an integer register
  switch (src) {
    case DType::I32: return uint64_t(int64_t(int32_t(uint32_t(raw))));
    case DType::U32: return uint64_t(uint32_t(raw));
    default: return raw;
  }
}
uint64_t narrow_int(DType dst, uint64_t v) {
  return (dst == DType::I32 || dst == DType::U32) ? uint64_t(uint32_t(v)) : v;
}
int64_t sat_i64(double x) {
  if (std::isnan(x)) return 0;
  if (x <= -9223372036854775808.0) return INT64_MIN;
  if (x >= 9223372036854775808.0) return INT64_MAX;
  return int64_t(x);
}
uint64_t sat_u64(double x) {
  if (std::isnan(x) || x <= 0.0) return 0;
  if (x >= 18446744073709551616.0) return UINT64_MAX;
  return uint64_t(x);
}
}  // namespace

bool eval_host(const Instr& in, double a, double b, double c, double& out, uint32_t& err) {
  auto fin = [&](double v) {
    out = v;
    if (!std::isfinite(v)) { err |= ERR_NONFINITE; return false; }
    return true;
  };
  switch (in.op) {
    case IOp::Neg: return fin(-a);
    case IOp::Not: return fin(a == 0.0 ? 1.0 : 0.0);
    case IOp::Abs: return fin(std::fabs(a));
    case IOp::Arccos: return fin(std::acos(a));
    case IOp::Arcsin: return fin(std::asin(a));
    case IOp::Arctan: return fin(std::atan(a));
    case IOp::Ceil: return fin(std::ceil(a));
    case IOp::Cos: return fin(std::cos(a));
    case IOp::Cosh: return fin(std::cosh(a));
    case IOp::Exp: return fin(std::exp(a));
    case IOp::Expm1: return fin(std::expm1(a));
    case IOp::Exprel: return fin(std::fabs(a) < 1e-16 ? 1.0 : a > 717.0 ? INFINITY : std::expm1(a) / a);
    case IOp::Floor: return fin(std::floor(a));
    case IOp::Trunc: return fin(std::fabs(a) <= 9007199254740992.0 ? std::trunc(a) : NAN);
    case IOp::RoundF32: {
      float f = float(a);
      return fin(std::isfinite(f) ? double(f) : NAN);
    }
    case IOp::Log: return fin(std::log(a));
    case IOp::Log10: return fin(std::log10(a));
    case IOp::Log1p: return fin(std::log1p(a));
    case IOp::Sign: return fin(a > 0.0 ? 1.0 : a < 0.0 ? -1.0 : 0.0);
    case IOp::Sin: return fin(std::sin(a));
    case IOp::Sinh: return fin(std::sinh(a));
    case IOp::Sqrt: return fin(std::sqrt(a));
    case IOp::Tan: return fin(std::tan(a));
    case IOp::Tanh: return fin(std::tanh(a));
    case IOp::Add: return fin(a + b);
    case IOp::Sub: return fin(a - b);
    case IOp::Mul: return fin(a * b);
    case IOp::Div: return fin(a / b);
    case IOp::Pow: return fin(std::pow(a, b));
    case IOp::Mod: return fin(a - b * std::floor(a / b));
    case IOp::FloorDiv: return fin(std::floor(a / b));
    case IOp::Eq: return fin(a == b ? 1.0 : 0.0);
    case IOp::Ne: return fin(a != b ? 1.0 : 0.0);
    case IOp::Gt: return fin(a > b ? 1.0 : 0.0);
    case IOp::Ge: return fin(a >= b ? 1.0 : 0.0);
    case IOp::Lt: return fin(a < b ? 1.0 : 0.0);
    case IOp::Le: return fin(a <= b ? 1.0 : 0.0);
    case IOp::And: return fin((a != 0.0 && b != 0.0) ? 1.0 : 0.0);
    case IOp::Or: return fin((a != 0.0 || b != 0.0) ? 1.0 : 0.0);
    case IOp::Clip: return fin(std::fmin(std::fmax(a, b), c));
    case IOp::TickOffset: {
      double r = a + double(in.offset);
      return fin(std::fabs(r) <= 9007199254740992.0 ? r : NAN);
    }
    case IOp::Timestep: {
      double steps = (a + 1e-3 * b) / b;
      if (!(a >= 0.0 && std::isfinite(b) && b > 0.0 && std::isfinite(steps) && steps < 9223372036854775808.0)) {
        err |= ERR_TIMESTEP;
        out = 0.0;
        return false;
      }
      uint64_t v = uint64_t(steps);
      if (v > 9007199254740992ull) {
        err |= ERR_TIMESTEP;
        out = 0.0;
        return false;
      }
      out = double(v);
      return true;
    }
    case IOp::Cast: {
      uint64_t raw = bits_of(a);
      if (in.dst == DType::F64) {
        switch (in.src) {
          case DType::Bool: out = a != 0.0 ? 1.0 : 0.0; return true;
          case DType::F32: case DType::F64: out = a; return true;
          case DType::I32: out = double(int32_t(uint32_t(raw))); return true;
          case DType::I64: out = double(int64_t(raw)); return true;
          case DType::U32: out = double(uint32_t(raw)); return true;
          case DType::U64: out = double(raw); return true;
          default: err |= ERR_CAST; return false;
        }
      }
      if (b2ir::is_integer(in.src)) {
        out = from_bits(narrow_int(in.dst, to64(in.src, raw)));
        return true;
      }
      double numeric;
      if (in.src == DType::Bool) numeric = a != 0.0 ? 1.0 : 0.0;
      else if (in.src == DType::F32 || in.src == DType::F64) numeric = a;
      else { err |= ERR_CAST; return false; }
      switch (in.dst) {
        case DType::I32: {
          int64_t v = sat_i64(numeric);
          int32_t w = v < INT32_MIN ? INT32_MIN : v > INT32_MAX ? INT32_MAX : int32_t(v);
          out = from_bits(uint64_t(uint32_t(w)));
          return true;
        }
        case DType::I64: out = from_bits(uint64_t(sat_i64(numeric))); return true;
        case DType::U32: {
          uint64_t v = sat_u64(numeric);
          out = from_bits(v > UINT32_MAX ? UINT32_MAX : v);
          return true;
        }
        case DType::U64: out = from_bits(sat_u64(numeric)); return true;
        default: err |= ERR_CAST; return false;
      }
    }
    case IOp::IntNeg: {
      uint64_t r = bits_of(a);
      out = in.dst == DType::I32 ? from_bits(uint64_t(uint32_t(0u - uint32_t(r)))) : from_bits(0ull - r);
      return true;
    }
    case IOp::IntAbs: {
      uint64_t r = bits_of(a);
      if (in.dst == DType::I32) {
        int32_t v = int32_t(uint32_t(r));
        out = from_bits(uint64_t(v < 0 ? uint32_t(0u - uint32_t(v)) : uint32_t(v)));
      } else {
        int64_t v = int64_t(r);
        out = from_bits(v < 0 ? 0ull - uint64_t(v) : uint64_t(v));
      }
      return true;
    }
    case IOp::IntBinary: {
      uint64_t lb = bits_of(a), rb = bits_of(b);
      auto rel = [&](auto x, auto y) -> int {
        switch (in.intop) {
          case IntOp::Gt: return x > y;
          case IntOp::Ge: return x >= y;
          case IntOp::Lt: return x < y;
          case IntOp::Le: return x <= y;
          default: return -1;
        }
      };
      auto finish = [&](auto x, auto y, auto wrap) -> bool {
        int r = rel(x, y);
        if (r >= 0) { out = r ? 1.0 : 0.0; return true; }
        using T = decltype(x);
        T v{};
        switch (in.intop) {
          case IntOp::Add: v = wrap(x, y, 0); break;
          case IntOp::Sub: v = wrap(x, y, 1); break;
          case IntOp::Mul: v = wrap(x, y, 2); break;
          case IntOp::Mod:
            if (y == 0) { err |= ERR_INTDIV; return false; }
            v = wrap(x, y, 3);
            break;
          case IntOp::FloorDiv:
            if (y == 0) { err |= ERR_INTDIV; return false; }
            v = wrap(x, y, 4);
            break;
          default: break;
        }
        out = from_bits(narrow_int(in.dst, uint64_t(v)));
        return true;
      };
      switch (in.dst) {
        case DType::I32: {
          int32_t x = int32_t(uint32_t(lb)), y = int32_t(uint32_t(rb));
          return finish(x, y, [](int32_t p, int32_t q, int k) -> int32_t {
            uint32_t up = uint32_t(p), uq = uint32_t(q);
            switch (k) {
              case 0: return int32_t(up + uq);
              case 1: return int32_t(up - uq);
              case 2: return int32_t(up * uq);
              case 3: return (p == INT32_MIN && q == -1) ? 0 : floor_mod<int32_t>(p, q);
              default: return (p == INT32_MIN && q == -1) ? INT32_MIN : floor_div<int32_t>(p, q);
            }
          });
        }
        case DType::I64: {
          int64_t x = int64_t(lb), y = int64_t(rb);
          return finish(x, y, [](int64_t p, int64_t q, int k) -> int64_t {
            uint64_t up = uint64_t(p), uq = uint64_t(q);
            switch (k) {
              case 0: return int64_t(up + uq);
              case 1: return int64_t(up - uq);
              case 2: return int64_t(up * uq);
              case 3: return (p == INT64_MIN && q == -1) ? 0 : floor_mod<int64_t>(p, q);
              default: return (p == INT64_MIN && q == -1) ? INT64_MIN : floor_div<int64_t>(p, q);
            }
          });
        }
        case DType::U32: {
          uint32_t x = uint32_t(lb), y = uint32_t(rb);
          return finish(x, y, [](uint32_t p, uint32_t q, int k) -> uint32_t {
            switch (k) {
              case 0: return p + q;
              case 1: return p - q;
              case 2: return p * q;
              case 3: return p % q;
              default: return p / q;
            }
          });
        }
        default: {
          uint64_t x = lb, y = rb;
          return finish(x, y, [](uint64_t p, uint64_t q, int k) -> uint64_t {
            switch (k) {
              case 0: return p + q;
              case 1: return p - q;
              case 2: return p * q;
              case 3: return p % q;
              default: return p / q;
            }
          });
        }
      }
    }
    case IOp::Select: out = c != 0.0 ? a : b; return true;  // c carries the guard
    default: throw Error("instruction cannot be folded on the host");
  }
}

// ------------------------------------------------------------------ classify
void Program::classify() {
  regs.assign(register_count, RegInfo{});
  std::vector<bool> assigned(register_count, false);
  for (const auto& [slot, in] : bindings) {
    RegInfo& r = regs[slot];
    assigned[slot] = true;
    if (in.kind == Input::Kind::Constant) {
      r.kind = RegKind::Const;
      r.value = in.value;
    } else if (in.kind == Input::Kind::Time) {
      r.kind = RegKind::Tick;
    } else if ((in.kind == Input::Kind::Random || in.kind == Input::Kind::Normal) && scalar_random.count(slot)) {
      r.kind = RegKind::Tick;
    } else {
      r.kind = RegKind::Lane;
    }
  }
  auto guard_is_bool_binding = [&](long g) {
    if (g < 0) return false;
    const Input* b = binding_of(size_t(g));
    return b && b->type() == DType::Bool;
  };
  auto process = [&](const std::vector<Instr>& list, bool scalar_block) {
    for (const auto& in : list) {
      // Operand info under this instruction's guard.
      auto operand = [&](size_t r) -> RegInfo {
        if (in.guard >= 0 && size_t(in.guard) == r && guard_is_bool_binding(in.guard) && in.op != IOp::Select) {
          RegInfo one;
          one.kind = RegKind::Const;
          one.value = 1.0;
          return one;
        }
        return regs[r];
      };
      RegInfo L = operand(in.left), R = operand(in.right);
      RegInfo T = in.third >= 0 ? operand(size_t(in.third)) : RegInfo{RegKind::Const, 0.0, true, 0};
      RegInfo G = in.guard >= 0 ? regs[size_t(in.guard)] : RegInfo{RegKind::Const, 1.0, true, 0};
      // A guard only decides whether an instruction runs; the value it would
      // produce from constant operands is itself a constant (lanes where it
      // does not run hold a stale register in the reference and are never
      // read unguarded by a well-formed model).  Select is the exception: its
      // result depends on the guard.
      RegKind k = std::max({L.kind, R.kind, T.kind});
      if (in.op == IOp::Select) k = std::max(k, G.kind);
      if (in.op == IOp::Binomial || in.op == IOp::Poisson || in.op == IOp::TimedArray) k = RegKind::Lane;
      RegInfo& out = regs[in.output];
      assigned[in.output] = true;
      if (k == RegKind::Const) {
        out.kind = RegKind::Const;
        if (G.kind == RegKind::Const && G.value == 0.0 && in.op != IOp::Select) {
          out.value = 0.0;  // never evaluated: register keeps its initial 0.0
          continue;
        }
        uint32_t err = 0;
        double v = 0.0;
        bool ok = true;
        if (in.op == IOp::Select) ok = eval_host(in, L.value, R.value, G.value, v, err);
        else ok = eval_host(in, L.value, R.value, T.value, v, err);
        out.value = v;
        out.finite = ok && L.finite && R.finite && T.finite;
        out.error = err | (L.finite ? 0 : L.error) | (R.finite ? 0 : R.error);
        if (scalar_block && !ok)
          throw Error(err & ERR_TIMESTEP ? "timestep outside Brian2 int64 range" : "non-finite numeric value");
      } else {
        out.kind = k;
      }
    }
  };
  process(scalar, true);
  process(vector, false);
  for (size_t r = 0; r < register_count; ++r)
    if (!assigned[r]) regs[r].kind = RegKind::Const;  // never written: stays 0.0
}

// ------------------------------------------------------------------ emission
std::string double_literal(double v) {
  if (!std::isfinite(v)) {
    char buf[64];
    std::snprintf(buf, sizeof buf, "b2_bits(0x%016llxull)", (unsigned long long)bits_of(v));
    return buf;
  }
  if (v == 0.0) return std::signbit(v) ? "(-0.0)" : "0.0";
  char buf[64];
  std::snprintf(buf, sizeof buf, "(%a)", v);
  return buf;
}

const char* storage_ctype(DType d) {
  switch (d) {
    case DType::Bool: return "u8";
    case DType::F32: return "float";
    case DType::F64: return "double";
    case DType::I32: return "i32";
    case DType::I64: return "i64";
    case DType::U32: return "u32";
    case DType::U64: return "u64";
    default: throw Error("logical dtype has no storage type");
  }
}

std::string widen(DType storage, const std::string& e) {
  switch (storage) {
    case DType::Bool: return "((" + e + ") ? 1.0 : 0.0)";
    case DType::F32: return "((double)(" + e + "))";
    case DType::F64: return "(" + e + ")";
    case DType::I32: return "b2_bits((u64)(u32)(" + e + "))";
    case DType::U32: return "b2_bits((u64)(" + e + "))";
    case DType::I64: return "b2_bits((u64)(" + e + "))";
    case DType::U64: return "b2_bits(" + e + ")";
    default: throw Error("logical dtype has no storage type");
  }
}

std::string narrow(DType storage, const std::string& r) {
  switch (storage) {
    case DType::Bool: return "(u8)((" + r + ") != 0.0)";
    case DType::F32: return "(float)(" + r + ")";
    case DType::F64: return "(" + r + ")";
    case DType::I32: return "(i32)(u32)b2_raw(" + r + ")";
    case DType::U32: return "(u32)b2_raw(" + r + ")";
    case DType::I64: return "(i64)b2_raw(" + r + ")";
    case DType::U64: return "b2_raw(" + r + ")";
    default: throw Error("logical dtype has no storage type");
  }
}

std::string reg_expr(const Program& p, size_t r, const std::string& prefix) {
  if (p.regs[r].kind == RegKind::Const) return double_literal(p.regs[r].value);
  return prefix + "r" + std::to_string(r);
}

namespace {
const char* dtype_code(DType d) {
  switch (d) {
    case DType::I32: return "0";
    case DType::I64: return "1";
    case DType::U32: return "2";
    default: return "3";
  }
}
const char* intop_code(IntOp o) {
  static const char* names[] = {"0", "1", "2", "3", "4", "5", "6", "7", "8"};
  return names[int(o)];
}

// Thresholds of the binomial inversion over the probabilities tab[x] =
// P(X = x), x < K (executor.rs:224-268 walks them with u -= P(X = x)): for
// each x the largest m in [0, 2^53) whose draw u = m * 2^-53 passes the
// loop's test at x, u - tab[0] - ... - tab[x-1] <= tab[x] (subtractions
// rounded in that order, as the loop does them), then the running maximum
// over x.  Passing draws form a prefix because rounded subtraction is
// non-decreasing in u; m = 0 always passes (its remainders are <= 0).
std::vector<uint64_t> binomial_thresholds(const std::vector<double>& tab) {
  std::vector<uint64_t> thr(tab.size());
  uint64_t run = 0;
  for (size_t x = 0; x < tab.size(); ++x) {
    auto passes = [&](uint64_t m) {
      double u = double(m) * 0x1p-53;
      for (size_t j = 0; j < x; ++j) u -= tab[j];
      return u <= tab[x];
    };
    uint64_t lo = 0, hi = (uint64_t(1) << 53) - 1;
    if (passes(hi)) {
      lo = hi;
    } else {
      while (hi - lo > 1) {  // passes(lo) and !passes(hi)
        const uint64_t mid = lo + (hi - lo) / 2;
        (passes(mid) ? lo : hi) = mid;
      }
    }
    run = std::max(run, lo);
    thr[x] = run;
  }
  return thr;
}
}  // namespace

namespace {

// Ops whose result the reference checks with is_finite (binary/ternary,
// executor.rs:5725-5778) and that can produce a non-finite value.
// Comparisons, logic and sign yield 0/1/-1 and need no check.
bool finite_checked(IOp op) {
  switch (op) {
    case IOp::Not: case IOp::Sign: case IOp::Eq: case IOp::Ne: case IOp::Gt: case IOp::Ge: case IOp::Lt:
    case IOp::Le: case IOp::And: case IOp::Or: case IOp::Cast: case IOp::IntNeg: case IOp::IntAbs:
    case IOp::IntBinary: case IOp::Timestep: case IOp::Select: case IOp::Binomial: case IOp::TimedArray:
      return false;
    default:
      return true;
  }
}

// Does operand `pos` of `in` carry a non-finite input into the output?
// (inf/NaN through +,-,*, the dividend, sign changes, roundings and sqrt stays
// non-finite; a divisor, comparisons, exp(-inf), clip and pow can mask it.)
bool propagates(const Instr& in, int pos) {
  switch (in.op) {
    case IOp::Add: case IOp::Sub: case IOp::Mul: return pos <= 1;
    case IOp::Div: case IOp::Neg: case IOp::Abs: case IOp::Floor: case IOp::Ceil: case IOp::Trunc:
    case IOp::Sqrt: case IOp::RoundF32: return pos == 0;
    case IOp::Select: return pos == 0;  // the value taken where the guard holds
    default: return false;
  }
}

}  // namespace

std::string emit_program(const Program& p, const EmitContext& ctx, const std::string& prefix) {
  std::ostringstream o;
  auto name = [&](size_t r) { return prefix + "r" + std::to_string(r); };
  // ---- finiteness coverage.  The reference rejects a non-finite result at
  // the op that produces it.  A value whose every use carries the non-finite
  // value on (under the same guard) into a value that is itself checked
  // raises the same error in the same tick without its own check; values that
  // are committed are checked once at the end.  Dropping the redundant checks
  // roughly halves the instruction count of an exact-linear update.
  const size_t R = p.register_count;
  std::vector<const Instr*> producer(R, nullptr);
  std::vector<std::vector<std::pair<const Instr*, int>>> uses(R);
  for (const auto* list : {&p.scalar, &p.vector})
    for (const auto& in : *list) {
      producer[in.output] = &in;
      uses[in.left].push_back({&in, 0});
      if (in.right != in.left) uses[in.right].push_back({&in, 1});
      if (in.third >= 0) uses[size_t(in.third)].push_back({&in, 2});
      if (in.guard >= 0) uses[size_t(in.guard)].push_back({&in, 3});
    }
  std::vector<bool> committed(R, false), floating(R, false), checked_here(R, false), safe(R, false);
  for (const auto& w : p.writes) committed[w.second] = true;
  for (const auto* list : {&p.scalar, &p.vector})
    for (const auto& in : *list)
      floating[in.output] = finite_checked(in.op) || (in.op == IOp::Select && floating[in.left]);
  std::vector<const Instr*> order;
  for (const auto* list : {&p.scalar, &p.vector})
    for (const auto& in : *list) order.push_back(&in);
  for (auto it = order.rbegin(); it != order.rend(); ++it) {
    const Instr& in = **it;
    size_t r = in.output;
    if (p.regs[r].kind == RegKind::Const) continue;
    bool covered = !uses[r].empty();
    for (const auto& [user, pos] : uses[r]) {
      if (!propagates(*user, pos) || user->guard != in.guard || !safe[user->output]) {
        covered = false;
        break;
      }
    }
    checked_here[r] = finite_checked(in.op) && !covered && !committed[r];
    safe[r] = covered || checked_here[r] || committed[r];
  }
  // Bindings: loaded at program start, like Program::run copies its inputs.
  for (const auto& [slot, in] : p.bindings) {
    const RegInfo& ri = p.regs[slot];
    if (ri.kind == RegKind::Const) continue;
    std::string value;
    if (in.kind == Input::Kind::Time) value = ctx.time;
    else if (in.kind == Input::Kind::Random && p.scalar_random.count(slot))
      value = "b2_uniform(" + ctx.seed + ", " + std::to_string(in.stream) + "ull, " + ctx.tick + ", 0ull)";
    else if (in.kind == Input::Kind::Normal && p.scalar_random.count(slot))
      value = "b2_normal(" + ctx.seed + ", " + std::to_string(in.stream) + "ull, " + ctx.tick + ", 0ull)";
    else if (in.kind == Input::Kind::Random)
      value = "b2_uniform(" + ctx.seed + ", " + std::to_string(in.stream) + "ull, " + ctx.tick + ", " +
              ctx.index_for_domain[int(in.domain)] + ")";
    else if (in.kind == Input::Kind::Normal)
      value = "b2_normal(" + ctx.seed + ", " + std::to_string(in.stream) + "ull, " + ctx.tick + ", " +
              ctx.index_for_domain[int(in.domain)] + ")";
    else value = ctx.load(in);
    o << "  double " << name(slot) << " = " << value << ";\n";
  }
  auto emit_list = [&](const std::vector<Instr>& list) {
    for (const auto& in : list) {
      const RegInfo& out = p.regs[in.output];
      // Operand r is exactly the constant v (bit for bit) where `in` runs.
      auto is_const = [&](size_t r, double v) {
        if (in.guard >= 0 && size_t(in.guard) == r && in.op != IOp::Select) {
          const Input* b = p.binding_of(r);
          if (b && b->type() == DType::Bool) return bits_of(v) == bits_of(1.0);
        }
        return p.regs[r].kind == RegKind::Const && bits_of(p.regs[r].value) == bits_of(v);
      };
      auto opnd = [&](size_t r) -> std::string {
        if (in.guard >= 0 && size_t(in.guard) == r && in.op != IOp::Select) {
          const Input* b = p.binding_of(r);
          if (b && b->type() == DType::Bool) return "1.0";
        }
        return reg_expr(p, r, prefix);
      };
      std::string guard = in.guard >= 0 ? reg_expr(p, size_t(in.guard), prefix) : "";
      bool guard_const = in.guard < 0 || p.regs[size_t(in.guard)].kind == RegKind::Const;
      if (out.kind == RegKind::Const) {
        // Folded on the host; a folded error still fires where the op would run.
        if (!out.finite && in.op != IOp::Select) {
          std::string bits = std::to_string(out.error ? out.error : ERR_NONFINITE) + "u";
          if (guard_const) o << "  err |= " << bits << ";\n";
          else o << "  if (" << guard << " != 0.0) err |= " << bits << ";\n";
        }
        continue;
      }
      std::string a = opnd(in.left), b = opnd(in.right);
      std::string c = in.third >= 0 ? opnd(size_t(in.third)) : "0.0";
      std::string expr;
      uint32_t check_bit = ERR_NONFINITE;
      bool check_finite = true;
      bool statement = false;  // expr is a full statement assigning the output
      std::string out_name = name(in.output);
      switch (in.op) {
        case IOp::Neg: expr = "-" + a; break;
        case IOp::Not: expr = "(" + a + " == 0.0 ? 1.0 : 0.0)"; break;
        case IOp::Abs: expr = "fabs(" + a + ")"; break;
        case IOp::Arccos: expr = "acos(" + a + ")"; break;
        case IOp::Arcsin: expr = "asin(" + a + ")"; break;
        case IOp::Arctan: expr = "atan(" + a + ")"; break;
        case IOp::Ceil: expr = "ceil(" + a + ")"; break;
        case IOp::Cos: expr = "cos(" + a + ")"; break;
        case IOp::Cosh: expr = "cosh(" + a + ")"; break;
        case IOp::Exp: expr = "exp(" + a + ")"; break;
        case IOp::Expm1: expr = "expm1(" + a + ")"; break;
        case IOp::Exprel: expr = "b2_exprel(" + a + ")"; break;
        case IOp::Floor: expr = "floor(" + a + ")"; break;
        case IOp::Trunc: expr = "b2_trunc(" + a + ")"; break;
        case IOp::RoundF32: expr = "b2_round_f32(" + a + ")"; break;
        case IOp::Log: expr = "log(" + a + ")"; break;
        case IOp::Log10: expr = "log10(" + a + ")"; break;
        case IOp::Log1p: expr = "log1p(" + a + ")"; break;
        case IOp::Sign: expr = "(" + a + " > 0.0 ? 1.0 : " + a + " < 0.0 ? -1.0 : 0.0)"; break;
        case IOp::Sin: expr = "sin(" + a + ")"; break;
        case IOp::Sinh: expr = "sinh(" + a + ")"; break;
        case IOp::Sqrt: expr = "sqrt(" + a + ")"; break;
        case IOp::Tan: expr = "tan(" + a + ")"; break;
        case IOp::Tanh: expr = "tanh(" + a + ")"; break;
        case IOp::Add: expr = "(" + a + " + " + b + ")"; break;
        // IEEE identities that hold for every x including -0, inf and NaN:
        // x - (+0) == x, x * 1 == 1 * x == x, x / 1 == x.
        case IOp::Sub: expr = is_const(in.right, 0.0) ? a : "(" + a + " - " + b + ")"; break;
        case IOp::Mul:
          expr = is_const(in.right, 1.0) ? a : is_const(in.left, 1.0) ? b : "(" + a + " * " + b + ")";
          break;
        case IOp::Div: expr = is_const(in.right, 1.0) ? a : "(" + a + " / " + b + ")"; break;
        case IOp::Pow: expr = "pow(" + a + ", " + b + ")"; break;
        case IOp::Mod: expr = "b2_fmod_floor(" + a + ", " + b + ")"; break;
        case IOp::FloorDiv: expr = "floor(" + a + " / " + b + ")"; break;
        case IOp::Eq: expr = "(" + a + " == " + b + " ? 1.0 : 0.0)"; break;
        case IOp::Ne: expr = "(" + a + " != " + b + " ? 1.0 : 0.0)"; break;
        case IOp::Gt: expr = "(" + a + " > " + b + " ? 1.0 : 0.0)"; break;
        case IOp::Ge: expr = "(" + a + " >= " + b + " ? 1.0 : 0.0)"; break;
        case IOp::Lt: expr = "(" + a + " < " + b + " ? 1.0 : 0.0)"; break;
        case IOp::Le: expr = "(" + a + " <= " + b + " ? 1.0 : 0.0)"; break;
        case IOp::And: expr = "((" + a + " != 0.0 && " + b + " != 0.0) ? 1.0 : 0.0)"; break;
        case IOp::Or: expr = "((" + a + " != 0.0 || " + b + " != 0.0) ? 1.0 : 0.0)"; break;
        case IOp::Clip: expr = "fmin(fmax(" + a + ", " + b + "), " + c + ")"; break;
        case IOp::TickOffset:
          expr = "b2_tick_offset(" + a + ", " + std::to_string(in.offset) + "ll)";
          break;
        case IOp::Select:
          expr = "(" + guard + " != 0.0 ? " + a + " : " + b + ")";
          check_finite = false;
          break;
        case IOp::Cast: {
          check_finite = false;
          std::string raw = "b2_raw(" + a + ")";
          if (in.dst == DType::F64) {
            switch (in.src) {
              case DType::Bool: expr = "(" + a + " != 0.0 ? 1.0 : 0.0)"; break;
              case DType::F32: case DType::F64: expr = a; break;
              case DType::I32: expr = "(double)(i32)(u32)" + raw; break;
              case DType::I64: expr = "(double)(i64)" + raw; break;
              case DType::U32: expr = "(double)(u32)" + raw; break;
              case DType::U64: expr = "(double)" + raw; break;
              default: throw Error("unsupported cast source");
            }
          } else if (b2ir::is_integer(in.src)) {
            std::string wide = in.src == DType::I32 ? "(u64)(i64)(i32)(u32)" + raw
                               : in.src == DType::U32 ? "(u64)(u32)" + raw : raw;
            expr = (in.dst == DType::I32 || in.dst == DType::U32) ? "b2_bits((u64)(u32)(" + wide + "))"
                                                                  : "b2_bits(" + wide + ")";
          } else {
            std::string num = in.src == DType::Bool ? "(" + a + " != 0.0 ? 1.0 : 0.0)" : a;
            switch (in.dst) {
              case DType::I32: expr = "b2_bits((u64)(u32)b2_f2i32(" + num + "))"; break;
              case DType::I64: expr = "b2_bits((u64)b2_f2i64(" + num + "))"; break;
              case DType::U32: expr = "b2_bits((u64)b2_f2u32(" + num + "))"; break;
              case DType::U64: expr = "b2_bits(b2_f2u64(" + num + "))"; break;
              default: throw Error("unsupported cast target");
            }
          }
          break;
        }
        case IOp::IntNeg:
          check_finite = false;
          expr = std::string("b2_int_neg(") + dtype_code(in.dst) + ", " + a + ")";
          break;
        case IOp::IntAbs:
          check_finite = false;
          expr = std::string("b2_int_abs(") + dtype_code(in.dst) + ", " + a + ")";
          break;
        case IOp::IntBinary:
          check_finite = false;
          expr = std::string("b2_int_binary(") + dtype_code(in.dst) + ", " + intop_code(in.intop) + ", " + a +
                 ", " + b + ", err)";
          break;
        case IOp::Timestep:
          check_finite = false;
          expr = "b2_timestep_reg(" + a + ", " + b + ", err)";
          break;
        case IOp::Binomial: {
          check_bit = ERR_BINOMIAL;
          check_finite = false;
          std::string idx = ctx.index_for_domain[int(in.domain)];
          std::string head = ctx.seed + ", " + std::to_string(in.stream) + "ull, " + ctx.tick + ", " + idx;
          const RegInfo& pr = p.regs[in.left];
          if (pr.kind == RegKind::Const && !(in.guard >= 0 && size_t(in.guard) == in.left)) {
            double pv = pr.value;
            if (!(std::isfinite(pv) && pv >= 0.0 && pv <= 1.0)) {
              statement = true;
              expr = "err |= " + std::to_string(ERR_BINOMIAL) + "u;";
            } else if (pv <= 0.0) {
              expr = "0.0";
            } else if (pv >= 1.0) {
              expr = double_literal(double(in.n));
            } else {
              double nf = double(in.n), loc = nf * pv, complement = nf * (1.0 - pv);
              if (in.approximate && loc > 5.0 && complement > 5.0) {
                expr = "(b2_normal(" + head + ") * " + double_literal(std::sqrt(loc * (1.0 - pv))) + " + " +
                       double_literal(loc) + ")";
              } else {
                bool reverse = pv > 0.5;
                double prob = reverse ? 1.0 - pv : pv;
                double q = 1.0 - prob;
                double qn = std::exp(nf * std::log(q));
                double bound = std::fmin(nf, nf * prob + 10.0 * std::sqrt(nf * prob * q + 1.0));
                const double kf = std::floor(bound) + 1.0;  // probabilities P(X = x) the loop can reach
                if (ctx.tables && kf <= 64.0) {
                  // The inversion's probabilities depend only on (n, p): build
                  // them here with the loop's own products and division, in
                  // the same order (-ffp-contract=off), so the device only
                  // compares and subtracts.
                  const size_t K = size_t(kf);
                  std::vector<double> tab(K);
                  tab[0] = qn;
                  for (size_t x = 1; x < K; ++x) {
                    const uint64_t xu = x;
                    tab[x] = ((double)(in.n - xu + 1) * prob * tab[x - 1]) / ((double)xu * q);
                  }
                  // The loop returns the first x whose remainder u - tab[0]
                  // - ... - tab[x-1] (each subtraction rounded) is <= tab[x].
                  // IEEE subtraction is non-decreasing in u, so for each x
                  // the draws passing that test form a prefix of [0, 2^53):
                  // its last element, found by bisection on the loop's own
                  // arithmetic, made non-decreasing over x (a draw stopped
                  // by an earlier x is counted there), is the threshold
                  // b2_binomial_thr compares the draw's bits against.
                  const std::vector<uint64_t> thr = binomial_thresholds(tab);
                  std::string body;
                  for (size_t x = 0; x < K; ++x) body += (x ? ", " : "") + std::to_string(thr[x]) + "ull";
                  std::string name = "b2_bthr_" + std::to_string(ctx.tables->size());
                  for (const auto& [nm, def] : *ctx.tables)
                    if (def.find("{" + body + "}") != std::string::npos) name = nm;
                  (*ctx.tables)[name] = "// inversion thresholds of binomial(n = " + std::to_string(in.n) + ", p = " +
                                        double_literal(pv) + ")\n__constant__ u64 " + name + "[" + std::to_string(K) +
                                        "] = {" + body + "};";
                  expr = "b2_binomial_thr<" + std::to_string(K) + "u>(" + head + ", " + std::to_string(in.n) + "ull, " +
                         name + ", " + (reverse ? "true" : "false") + ")";
                } else {
                  expr = "b2_binomial_inv(" + head + ", " + std::to_string(in.n) + "ull, " + double_literal(prob) +
                         ", " + double_literal(q) + ", " + double_literal(qn) + ", " + double_literal(bound) + ", " +
                         (reverse ? "true" : "false") + ")";
                }
              }
            }
          } else {
            expr = "b2_binomial_checked(" + head + ", " + std::to_string(in.n) + "ull, " + a + ", " +
                   (in.approximate ? "true" : "false") + ", err)";
          }
          break;
        }
        case IOp::Poisson: {
          check_bit = ERR_POISSON;
          std::string idx = ctx.index_for_domain[int(in.domain)];
          expr = "b2_poisson(" + ctx.seed + ", " + std::to_string(in.stream) + "ull, " + ctx.tick + ", " + idx +
                 ", " + a + ")";
          break;
        }
        case IOp::TimedArray: {
          // Op::TimedArray (executor.rs:6121-6154): row from the time, column
          // from the index, both range-checked; a non-finite value is an error
          check(bool(ctx.device_array), "TimedArray needs device tables");
          const b2ir::Expr& ta = *in.ta;
          const uint64_t width = ta.ta_columns >= 0 ? uint64_t(ta.ta_columns) : 1;
          check(ta.ta_rows > 0 && ta.ta_values.size() == ta.ta_rows * width, "TimedArray table has the wrong size");
          check_bit = ERR_TIMEDARRAY;
          check_finite = true;
          expr = "b2_timed_array(" + ctx.device_array(ta.ta_values) + ", " + std::to_string(ta.ta_rows) + "ull, " +
                 std::to_string(width) + "ull, " + (ta.ta_columns >= 0 ? "true" : "false") + ", " +
                 double_literal(ta.ta_epsilon) + ", " + double_literal(double(ta.ta_upsampling)) + ", " + a + ", " +
                 b + ", err)";
          break;
        }
      }
      o << "  double " << out_name << " = 0.0;\n";
      std::string body;
      if (statement) {
        body = expr;
      } else {
        body = out_name + " = " + expr + ";";
        bool need = check_finite && (checked_here[in.output] || check_bit != ERR_NONFINITE);
        if (need) body += " if (!b2_finite(" + out_name + ")) err |= " + std::to_string(check_bit) + "u;";
      }
      if (in.op == IOp::Select || guard_const) {
        if (!guard_const && in.op != IOp::Select) o << "  if (" << guard << " != 0.0) { " << body << " }\n";
        else if (guard_const && in.guard >= 0 && p.regs[size_t(in.guard)].value == 0.0 && in.op != IOp::Select)
          o << "  /* never evaluated */\n";
        else o << "  " << body << "\n";
      } else {
        o << "  if (" << guard << " != 0.0) { " << body << " }\n";
      }
    }
  };
  emit_list(p.scalar);
  emit_list(p.vector);
  // Committed floating values: one check each, where the commit happens.
  std::set<size_t> done;
  for (const auto& w : p.writes) {
    size_t r = w.second;
    if (p.regs[r].kind == RegKind::Const || !floating[r] || done.count(r)) continue;
    done.insert(r);
    o << "  if (!b2_finite(" << name(r) << ")) err |= " << ERR_NONFINITE << "u;\n";
  }
  return o.str();
}

}  // namespace b2gpu
