// ir.h — the plugin's in-memory form of a StableHLO module (after parsing, with calls inlined).
//
// The reference holds the module as MLIR (src/jam/parse.cc:53-63) and lowers it op by op into
// MPSGraph nodes (src/jam/lower.mm:208-314).  MLIR is not available here, so the parser
// (parse.cc) builds this small SSA graph instead: one `Op` per StableHLO operation, `Value`s with
// static tensor types, and the few attributes the lowering needs.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace b200 {

enum class DT : uint8_t { kPred, kS8, kS16, kS32, kS64, kU8, kU16, kU32, kU64, kF16, kBF16, kF32, kF64, kInvalid };

int DTBytes(DT t);
const char* DTName(DT t);            // MLIR spelling: i1 i8 ... bf16 f32
bool DTIsFloat(DT t);
bool DTIsSigned(DT t);
bool DTIsUnsigned(DT t);
DT DTFromMlir(const std::string& s);

// PJRT_Buffer_Type code of an element type as the kernel entry points take it (B200_DT_*), or -1.
inline int KernelTypeCode(DT t) {
  switch (t) {
    case DT::kF32: return 11;
    case DT::kBF16: return 13;
    case DT::kF16: return 10;
    case DT::kS32: return 4;
    case DT::kS64: return 5;
    default: return -1;
  }
}

struct TensorType {
  DT dt = DT::kInvalid;
  std::vector<int64_t> dims;
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : dims) n *= d;
    return n;
  }
  int64_t bytes() const { return numel() * DTBytes(dt); }
  int rank() const { return (int)dims.size(); }
  std::string str() const;
  bool operator==(const TensorType& o) const { return dt == o.dt && dims == o.dims; }
};

struct Op;

struct Value {
  int id = -1;
  TensorType type;
  Op* def = nullptr;       // null for function arguments
  int arg_index = -1;      // >= 0 for @main arguments
  std::vector<Op*> users;
};

enum class ReduceKind { kAdd, kMax, kMin, kMul, kAnd, kOr, kNone };

struct Op {
  std::string name;                          // without the "stablehlo." prefix, e.g. "add"
  std::vector<Value*> operands;
  std::vector<Value*> results;
  std::map<std::string, std::vector<int64_t>> ints;   // dims, permutation, dimension numbers, ...
  std::map<std::string, std::string> strs;            // comparison_direction, compare_type, target
  ReduceKind reduce = ReduceKind::kNone;              // reduce / all_reduce / scatter region kind
  // constants: raw little-endian bytes of one element (splat) or of all elements
  std::vector<uint8_t> data;
  bool splat = false;
  int index = 0;                             // position in the graph's op list
  Value* result() const { return results.empty() ? nullptr : results[0]; }
};

struct Graph {
  std::string name;
  int num_partitions = 1;
  int num_replicas = 1;
  std::vector<std::unique_ptr<Value>> values;
  std::vector<std::unique_ptr<Op>> ops;      // program order
  std::vector<Value*> args;
  std::vector<Value*> outputs;
  // per @main argument: the result its buffer may become (`tf.aliasing_output`, -1: none), and
  // whether the caller may give up its buffer at all (an alias, or `jax.buffer_donor`)
  std::vector<int> arg_alias_output;
  std::vector<bool> arg_donor;

  Value* NewValue(const TensorType& t) {
    values.emplace_back(new Value());
    values.back()->id = (int)values.size() - 1;
    values.back()->type = t;
    return values.back().get();
  }
  Op* NewOp(const std::string& name) {
    ops.emplace_back(new Op());
    ops.back()->name = name;
    return ops.back().get();
  }
  void Renumber();                           // recompute Op::index and Value::users
};

// Parses StableHLO MLIR text (pretty + generic forms for the supported op subset) into `g`.
// Returns an empty string on success, else an error message (the op or token that failed).
std::string ParseModule(const char* text, size_t size, Graph* g);

// Checks operand counts, shapes and attribute ranges of the supported ops (verify.cc); "" if the
// graph is well formed, else the first violation.  ParseModule runs it.
std::string VerifyGraph(const Graph& g);

// One line per op of a parsed graph: name, operand / result value ids and types, integer
// attributes, the attributes the lowering reads as strings, reduce kind and the constant data
// (splat flag + FNV-1a hash of the bytes).  Two spellings of one program (pretty or generic text,
// MLIR bytecode) parse to the same dump.
std::string DumpGraph(const Graph& g);

// Reads the value of a float/int scalar constant as double.
double ConstScalar(const Op* op);

}  // namespace b200
