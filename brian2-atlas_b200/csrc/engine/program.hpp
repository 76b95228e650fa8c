// Compile one AtlasIR CodeObject into straight-line CUDA C++.
//
// The SSA construction (registers, input bindings, guarded statements turned
// into Select, scalar block then vector block) follows the reference's
// Program::compile (brian2-rust/src/executor.rs:5046-5486) so that every
// arithmetic step, rounding and error check happens in the same order.  On top
// of that the compiler classifies each register:
//   Const - known at plan time: literals, scalar parameters, the scalar block,
//           and vector instructions whose operands are all Const.  These are
//           evaluated here on the host in f64 with glibc libm (the libm the
//           reference's Rust f64 methods call), and emitted as exact literals.
//   Tick  - uniform over lanes but dependent on t or a per-tick scalar draw;
//           evaluated on the device once per thread.
//   Lane  - per-neuron / per-event work.
// Inside a statement guarded by a bool condition c, a read of c is known to be
// 1.0 (the instruction only runs where c != 0), which lets the exact-linear
// integrators' exp(dt/tau * not_refractory) fold to a host constant.
#pragma once

#include <functional>
#include <map>
#include <optional>
#include <set>
#include <string>
#include <vector>

#include "../common/ir.hpp"

namespace b2gpu {

using b2ir::DType;

enum class Domain : uint8_t { Neuron, Pre, Post, Edge };

struct Input {
  enum class Kind : uint8_t { Constant, Time, Index, State, PreState, PostState, SynapseState,
                              Parameter, LastSpike, Available, Random, Normal } kind = Kind::Constant;
  double value = 0.0;          // Constant
  DType dtype = DType::F64;
  Domain domain = Domain::Neuron;
  size_t index = 0;            // state / parameter table index
  uint64_t stream = 0;         // Random / Normal
  bool scalar() const { return kind == Kind::Constant || kind == Kind::Time; }
  DType type() const;
  static Input constant(double v, DType d);
  static Input make(Kind k, Domain d = Domain::Neuron, size_t index = 0, DType dtype = DType::F64);
};

struct WriteTarget {
  enum class Kind : uint8_t { Neuron, PreNeuron, Synapse, Available } kind = Kind::Neuron;
  size_t index = 0;
};

enum class IOp : uint8_t {
  Neg, Not, Abs, Arccos, Arcsin, Arctan, Ceil, Cos, Cosh, Exp, Expm1, Exprel, Floor, Trunc,
  RoundF32, Cast, IntNeg, IntAbs, IntBinary, Timestep, TickOffset, Log, Log10, Log1p, Sign,
  Sin, Sinh, Sqrt, Tan, Tanh, Add, Sub, Mul, Div, Pow, Mod, FloorDiv, Eq, Ne, Gt, Ge, Lt, Le,
  And, Or, Clip, Select, Binomial, Poisson, TimedArray,
};
enum class IntOp : uint8_t { Add, Sub, Mul, Mod, FloorDiv, Gt, Ge, Lt, Le };

struct Instr {
  IOp op = IOp::Add;
  size_t left = 0, right = 0, output = 0;
  long third = -1, guard = -1;
  DType src = DType::F64, dst = DType::F64;
  IntOp intop = IntOp::Add;
  uint64_t stream = 0, n = 0;
  bool approximate = false;
  Domain domain = Domain::Neuron;
  int64_t offset = 0;
  const b2ir::Expr* ta = nullptr;
};

enum class RegKind : uint8_t { Const, Tick, Lane };

struct RegInfo {
  RegKind kind = RegKind::Lane;
  double value = 0.0;     // Const
  bool finite = true;     // Const: evaluation produced a finite value / no error
  uint32_t error = 0;     // Const: B2_ERR bit the evaluation would raise
};

// The SSA program of one CodeObject.
class Program {
 public:
  static Program compile(const b2ir::CodeObject& code, std::map<std::string, Input> inputs,
                         const std::map<std::string, WriteTarget>& writable,
                         const std::vector<b2ir::Function>& functions);

  size_t register_count = 0;
  std::vector<std::pair<size_t, Input>> bindings;
  std::set<size_t> scalar_random;
  std::vector<Instr> scalar, vector;
  std::vector<std::pair<WriteTarget, size_t>> writes;
  long condition = -1;
  Domain rng_domain = Domain::Neuron;
  std::map<std::string, size_t> symbols;
  std::map<std::string, DType> symbol_dtypes;

  // Filled by classify().
  std::vector<RegInfo> regs;
  // Classify registers and fold constants.  `rng_seed` is needed to fold
  // plan-time-constant draws (none in practice: draws depend on the tick).
  void classify();
  // Input binding of a register, or nullptr.
  const Input* binding_of(size_t reg) const;
  // Register that holds the post-state value `index` as loaded at program
  // start, if any.
  std::optional<size_t> post_state_register(size_t index) const;
  // True if any instruction draws random numbers or any binding is random.
  bool uses_rng() const;

 private:
  std::map<std::string, Input> inputs_;
  std::map<std::string, const b2ir::Function*> functions_;
  size_t reg();
  size_t input(const Input& v);
  size_t resolve(const std::string& name);
  DType infer(const b2ir::Expr& e);
  size_t expression(const b2ir::Expr& e, long guard, std::vector<Instr>& ops);
  std::vector<Instr> statements(const std::vector<b2ir::Statement>& sts);
};

// Host evaluation of one instruction on scalars with the reference's
// semantics; returns false (and the error bit) where the reference would raise.
bool eval_host(const Instr& in, double a, double b, double c, double& out, uint32_t& err);

// Emission context: how a kernel reads each kind of input for the current
// lane, and how it writes commits.  Strings are C++ expressions.
struct EmitContext {
  std::function<std::string(const Input&)> load;
  std::string seed;     // expression for the RNG seed
  std::string tick;     // expression for the current tick (u64)
  std::string index_for_domain[4];  // RNG counter index per Domain (u64)
  std::string time;     // expression for t (double)
  // Optional sink for file-scope constant tables (name -> definition) that
  // emitted code may reference; null disables table-based emission.
  std::map<std::string, std::string>* tables = nullptr;
  // Expression for a device pointer to a copy of `values` (TimedArray
  // tables); empty disables TimedArray emission.
  std::function<std::string(const std::vector<double>& values)> device_array;
};

// Emit the body of a program: declarations of every non-Const register used,
// input loads, instructions with guards and finite checks (errors OR-ed into
// a local `err`).  Register r is named "<prefix>r<r>".  Const registers are
// emitted as exact literals.
std::string emit_program(const Program& p, const EmitContext& ctx, const std::string& prefix);

// C++ expression for a register after emit_program (literal or name).
std::string reg_expr(const Program& p, size_t r, const std::string& prefix);

// Exact C++ literal of a double (hex float; NaN/Inf via bit casts).
std::string double_literal(double v);

// Storage conversions mirroring StateArray::get_register / set_register
// (executor.rs:422-467): widen a storage-typed C++ expression to a register
// double, and narrow a register double to the storage type.
std::string widen(DType storage, const std::string& expr);
std::string narrow(DType storage, const std::string& reg);
const char* storage_ctype(DType d);

}  // namespace b2gpu
