// verify.cc — shape and arity checks of a parsed program, before lowering.
//
// The reference's programs pass MLIR's op verifiers when they are deserialized
// (src/jam/parse.cc:53-63).  This compiler reads text and bytecode itself, so it checks what its
// kernels rely on: every op of the supported subset has its operand count, operand / result shapes
// and attribute ranges as StableHLO defines them.  A malformed program is rejected at compile time
// (INVALID_ARGUMENT through PJRT_Client_Compile) instead of becoming a kernel that reads or writes
// outside its buffers.  Ops outside the subset are left to the lowering, which names them.
#include <algorithm>
#include <string>
#include <unordered_set>

#include "ir.h"

namespace b200 {
namespace {

struct Bad {
  std::string msg;
};

const std::unordered_set<std::string> kUnaryOps = {
    "negate", "exponential", "exponential_minus_one", "log", "log_plus_one", "tanh", "sqrt", "rsqrt",
    "cbrt", "abs", "sine", "cosine", "tan", "floor", "ceil", "sign", "round_nearest_even",
    "round_nearest_afz", "logistic", "not", "is_finite", "popcnt", "count_leading_zeros", "erf",
    "reduce_precision", "convert", "bitcast_convert"};
const std::unordered_set<std::string> kBinaryOps = {
    "add", "subtract", "multiply", "divide", "maximum", "minimum", "power", "remainder", "atan2",
    "and", "or", "xor", "shift_left", "shift_right_logical", "shift_right_arithmetic", "compare"};

std::string Dims(const std::vector<int64_t>& d) {
  std::string s = "[";
  for (size_t k = 0; k < d.size(); ++k) s += (k ? "," : "") + std::to_string(d[k]);
  return s + "]";
}

class Verifier {
 public:
  explicit Verifier(const Op* op) : op_(op), n_(op->name) {}

  void Run() {
    const auto& in = op_->operands;
    if (n_ == "custom_call" || n_ == "all_reduce" || n_ == "all_gather" || n_ == "reduce_scatter" || n_ == "all_to_all" ||
        n_ == "collective_broadcast" || n_ == "collective_permute") {
      if (in.empty()) Fail("needs an operand");
      return;   // shapes follow the sharding / rank count, checked where they are lowered
    }
    if (kUnaryOps.count(n_)) {
      Arity(1);
      // a bitcast between element types of different widths changes the shape (the lowering
      // names it as unsupported)
      if (!(n_ == "bitcast_convert" && DTBytes(Dt(0)) != DTBytes(RDt()))) SameDims(0);
      if (n_ != "convert" && n_ != "bitcast_convert" && n_ != "is_finite" && Dt(0) != RDt()) Fail("operand and result types differ");
      return;
    }
    if (kBinaryOps.count(n_)) {
      Arity(2);
      SameDims(0);
      SameDims(1);
      if (Dt(0) != Dt(1)) Fail("operand types differ");
      if (n_ != "compare" && Dt(0) != RDt()) Fail("operand and result types differ");
      return;
    }
    if (n_ == "select" || n_ == "clamp") {
      // select(pred, on_true, on_false); clamp(min, x, max): the scalar operand may be rank 0
      Arity(3);
      SameDims(1);
      const size_t scalar_ok[2] = {0, n_ == "select" ? (size_t)0 : (size_t)2};
      for (size_t k : {(size_t)0, (size_t)2}) {
        const bool may_be_scalar = k == scalar_ok[0] || k == scalar_ok[1];
        if (!(may_be_scalar && In(k).rank() == 0)) SameDims(k);
      }
      if (n_ == "select") {
        if (Dt(0) != DT::kPred) Fail("predicate is not i1");
        if (Dt(1) != RDt() || Dt(2) != RDt()) Fail("branch types differ from the result");
      } else if (Dt(0) != RDt() || Dt(1) != RDt() || Dt(2) != RDt()) {
        Fail("operand types differ");
      }
      return;
    }
    if (n_ == "constant" || n_ == "iota" || n_ == "partition_id" || n_ == "replica_id") {
      Arity(0);
      if (n_ == "iota") {
        int64_t d = Int("dim", 0);
        if (d < 0 || d >= R().rank()) Fail("iota dimension out of range");
      }
      if ((n_ == "partition_id" || n_ == "replica_id") && R().rank() != 0) Fail("result is not a scalar");
      return;
    }
    if (n_ == "reshape") {
      Arity(1);
      if (In(0).numel() != R().numel()) Fail("element count changes from " + Dims(In(0).dims) + " to " + Dims(R().dims));
      if (Dt(0) != RDt()) Fail("operand and result types differ");
      return;
    }
    if (n_ == "broadcast_in_dim") {
      Arity(1);
      const auto& d = Ints("dims");
      if ((int)d.size() != In(0).rank()) Fail("broadcast_dimensions does not match the operand rank");
      for (size_t k = 0; k < d.size(); ++k) {
        if (d[k] < 0 || d[k] >= R().rank()) Fail("broadcast dimension out of range");
        if (k && d[k] <= d[k - 1]) Fail("broadcast dimensions not increasing");
        if (In(0).dims[k] != 1 && In(0).dims[k] != R().dims[d[k]]) Fail("operand dimension does not broadcast");
      }
      return;
    }
    if (n_ == "broadcast") {
      Arity(1);
      const auto& sz = Ints("sizes");
      std::vector<int64_t> want = sz;
      want.insert(want.end(), In(0).dims.begin(), In(0).dims.end());
      if (R().dims != want) Fail("result shape is not broadcast_sizes followed by the operand shape");
      if (Dt(0) != RDt()) Fail("operand and result types differ");
      return;
    }
    if (n_ == "transpose") {
      Arity(1);
      const auto& p = Ints("dims");
      if ((int)p.size() != In(0).rank() || R().rank() != In(0).rank()) Fail("permutation does not match the rank");
      std::vector<int64_t> s = p;
      std::sort(s.begin(), s.end());
      for (size_t k = 0; k < s.size(); ++k)
        if (s[k] != (int64_t)k) Fail("not a permutation");
      for (size_t k = 0; k < p.size(); ++k)
        if (R().dims[k] != In(0).dims[p[k]]) Fail("result shape is not the permuted operand shape");
      return;
    }
    if (n_ == "reverse") {
      Arity(1);
      SameDims(0);
      const auto& d = op_->ints.count("dims") ? op_->ints.at("dims") : Ints("dimensions");
      for (int64_t x : d)
        if (x < 0 || x >= R().rank()) Fail("reverse dimension out of range");
      return;
    }
    if (n_ == "slice") {
      Arity(1);
      const auto &st = Ints("start_indices"), &li = Ints("limit_indices"), &sd = Ints("strides");
      const int r = In(0).rank();
      if ((int)st.size() != r || (int)li.size() != r || (int)sd.size() != r || R().rank() != r) Fail("index lists do not match the rank");
      for (int k = 0; k < r; ++k) {
        if (st[k] < 0 || st[k] > li[k] || li[k] > In(0).dims[k] || sd[k] < 1) Fail("slice bounds out of range");
        if (R().dims[k] != (li[k] - st[k] + sd[k] - 1) / sd[k]) Fail("result shape does not match the slice");
      }
      return;
    }
    if (n_ == "pad") {
      Arity(2);
      if (In(1).rank() != 0) Fail("padding value is not a scalar");
      const auto& lo = op_->ints.count("low") ? op_->ints.at("low") : Ints("edge_padding_low");
      const auto& hi = op_->ints.count("high") ? op_->ints.at("high") : Ints("edge_padding_high");
      const auto& it = op_->ints.count("interior") ? op_->ints.at("interior") : Ints("interior_padding");
      const int r = In(0).rank();
      if ((int)lo.size() != r || (int)hi.size() != r || (int)it.size() != r || R().rank() != r) Fail("padding lists do not match the rank");
      for (int k = 0; k < r; ++k) {
        const int64_t d = In(0).dims[k];
        if (it[k] < 0 || R().dims[k] != lo[k] + hi[k] + d + std::max<int64_t>(d - 1, 0) * it[k] || R().dims[k] < 0)
          Fail("result shape does not match the padding");
      }
      return;
    }
    if (n_ == "concatenate") {
      if (op_->operands.empty()) Fail("needs an operand");
      const int64_t d = Int("dim", 0);
      const int r = R().rank();
      if (d < 0 || d >= r) Fail("concatenate dimension out of range");
      int64_t sum = 0;
      for (size_t k = 0; k < op_->operands.size(); ++k) {
        if (In(k).rank() != r) Fail("operand ranks differ");
        for (int j = 0; j < r; ++j)
          if (j != d && In(k).dims[j] != R().dims[j]) Fail("operand shapes differ off the concatenated dimension");
        sum += In(k).dims[d];
      }
      if (sum != R().dims[d]) Fail("result size along the concatenated dimension is wrong");
      return;
    }
    if (n_ == "dot_general") {
      Arity(2);
      auto get = [&](const char* k) { auto it = op_->ints.find(k); return it == op_->ints.end() ? std::vector<int64_t>{} : it->second; };
      const auto lb = get("batching_dims.lhs"), rb = get("batching_dims.rhs");
      const auto lc = get("contracting_dims.lhs"), rc = get("contracting_dims.rhs");
      if (lb.size() != rb.size() || lc.size() != rc.size()) Fail("dimension lists of lhs and rhs differ in length");
      std::vector<int64_t> out;
      std::vector<bool> used_l(In(0).rank(), false), used_r(In(1).rank(), false);
      auto mark = [&](const std::vector<int64_t>& d, std::vector<bool>& used, int side) {
        for (int64_t x : d) {
          if (x < 0 || x >= (int64_t)used.size() || used[x]) Fail("dimension number out of range or repeated");
          used[x] = true;
        }
        (void)side;
      };
      mark(lb, used_l, 0); mark(lc, used_l, 0); mark(rb, used_r, 1); mark(rc, used_r, 1);
      for (size_t k = 0; k < lb.size(); ++k) {
        if (In(0).dims[lb[k]] != In(1).dims[rb[k]]) Fail("batch dimensions differ");
        out.push_back(In(0).dims[lb[k]]);
      }
      for (size_t k = 0; k < lc.size(); ++k)
        if (In(0).dims[lc[k]] != In(1).dims[rc[k]]) Fail("contracting dimensions differ");
      for (int k = 0; k < In(0).rank(); ++k) if (!used_l[k]) out.push_back(In(0).dims[k]);
      for (int k = 0; k < In(1).rank(); ++k) if (!used_r[k]) out.push_back(In(1).dims[k]);
      if (out != R().dims) Fail("result shape " + Dims(R().dims) + " is not " + Dims(out));
      if (Dt(0) != Dt(1) && !(DTIsFloat(Dt(0)) && DTIsFloat(Dt(1)))) Fail("operand types differ");
      return;
    }
    if (n_ == "reduce") {
      const size_t m = op_->operands.size();
      if (m < 2 || m % 2 || op_->results.size() != m / 2) Fail("needs inputs and as many init values");
      const auto& d = Ints("dimensions");
      std::vector<bool> red(In(0).rank(), false);
      for (int64_t x : d) {
        if (x < 0 || x >= In(0).rank() || red[x]) Fail("reduced dimension out of range or repeated");
        red[x] = true;
      }
      std::vector<int64_t> out;
      for (int k = 0; k < In(0).rank(); ++k) if (!red[k]) out.push_back(In(0).dims[k]);
      for (size_t k = 0; k < m / 2; ++k) {
        if (In(k).dims != In(0).dims) Fail("input shapes differ");
        if (In(m / 2 + k).rank() != 0) Fail("init value is not a scalar");
        if (op_->results[k]->type.dims != out) Fail("result shape is not the reduced input shape");
      }
      return;
    }
    if (n_ == "dynamic_slice" || n_ == "dynamic_update_slice") {
      const bool upd = n_ == "dynamic_update_slice";
      const int r = In(0).rank();
      const size_t first = upd ? 2 : 1;
      if (op_->operands.size() != first + r) Fail("needs one start index per dimension");
      for (size_t k = first; k < op_->operands.size(); ++k)
        if (In(k).rank() != 0 || DTIsFloat(Dt(k)) || Dt(k) == DT::kPred) Fail("start indices must be integer scalars");
      if (upd) {
        SameDims(0);
        if (In(1).rank() != r) Fail("update rank differs");
        for (int k = 0; k < r; ++k)
          if (In(1).dims[k] > In(0).dims[k]) Fail("update larger than the operand");
        if (Dt(1) != Dt(0)) Fail("update type differs");
      } else {
        const auto& s = Ints("sizes");
        if ((int)s.size() != r || R().dims != s) Fail("slice sizes do not match the result");
        for (int k = 0; k < r; ++k)
          if (s[k] < 0 || s[k] > In(0).dims[k]) Fail("slice size out of range");
      }
      if (RDt() != Dt(0)) Fail("result type differs from the operand");
      return;
    }
    if (n_ == "gather") {
      Arity(2);
      if (DTIsFloat(Dt(1)) || Dt(1) == DT::kPred) Fail("indices are not integers");
      return;   // the supported form is checked where it is lowered
    }
    if (n_ == "scatter") {
      Arity(3);
      if (DTIsFloat(Dt(1)) || Dt(1) == DT::kPred) Fail("indices are not integers");
      SameDims(0);
      return;
    }
    if (n_ == "optimization_barrier") {
      if (op_->operands.size() != op_->results.size()) Fail("operand and result counts differ");
      for (size_t k = 0; k < op_->operands.size(); ++k)
        if (!(op_->operands[k]->type == op_->results[k]->type)) Fail("operand and result types differ");
      return;
    }
  }

 private:
  const Op* op_;
  const std::string& n_;

  [[noreturn]] void Fail(const std::string& m) const { throw Bad{"op '" + n_ + "': " + m}; }
  void Arity(size_t k) const {
    if (op_->operands.size() != k)
      Fail("expects " + std::to_string(k) + " operand(s), has " + std::to_string(op_->operands.size()));
    if (op_->results.empty()) Fail("has no result");
  }
  const TensorType& In(size_t k) const { return op_->operands[k]->type; }
  const TensorType& R() const {
    if (op_->results.empty()) Fail("has no result");
    return op_->results[0]->type;
  }
  DT Dt(size_t k) const { return In(k).dt; }
  DT RDt() const { return R().dt; }
  void SameDims(size_t k) const {
    if (In(k).dims != R().dims) Fail("operand " + std::to_string(k) + " shape " + Dims(In(k).dims) + " differs from the result " + Dims(R().dims));
  }
  const std::vector<int64_t>& Ints(const char* key) const {
    auto it = op_->ints.find(key);
    if (it == op_->ints.end()) Fail(std::string("lacks attribute ") + key);
    return it->second;
  }
  int64_t Int(const char* key, size_t k) const {
    const auto& v = Ints(key);
    if (v.size() <= k) Fail(std::string("bad attribute ") + key);
    return v[k];
  }
};

}  // namespace

std::string VerifyGraph(const Graph& g) {
  try {
    for (const auto& op : g.ops) Verifier(op.get()).Run();
  } catch (const Bad& b) {
    return b.msg;
  }
  return "";
}

}  // namespace b200
