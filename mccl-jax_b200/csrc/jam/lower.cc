// lower.cc — StableHLO graph -> B200 plan: pattern matching, fusion decisions and CUDA C codegen.
//
// Follows the reference's lowering walk (src/jam/lower.mm:208-314, :460-566) in what it accepts and
// how it treats shard_map and collectives, but emits different work:
//   * `dot_general` -> a GemmStep (tcgen05 GEMM; operands brought to K-major [batch, rows, K] first,
//     the canonicalisation of src/jam/ops/linalg.mm:68-104);
//   * the dot_general -> (scale) -> (causal select) -> softmax -> dot_general chain -> one fused
//     AttentionStep (the reference only matches the softmax, src/jam/ops/elementwise.mm:71-89);
//   * chains of elementwise / broadcast / convert / index-map ops -> generated loop kernels, and
//     `reduce` -> generated row / column reduction kernels with the producer chain inlined;
//   * all_reduce / all_gather / reduce_scatter -> CollectiveSteps (NCCL); with one rank they are
//     identities (lower.mm:346-352); all_gather / reduce_scatter only along dim 0 (lower.mm:391-410).
// An op outside the supported set fails compilation with its name (lower.mm:309).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <set>
#include <sstream>
#include <unordered_map>
#include <unordered_set>

#include "plan.h"
#include "../kernels/kernels.h"


namespace b200 {
namespace {

struct LowerError {
  std::string msg;
};

// ------------------------------------------------------------------------------------ op classes
const std::unordered_set<std::string> kBinary = {
    "add", "subtract", "multiply", "divide", "maximum", "minimum", "power", "remainder",
    "atan2", "and", "or", "xor", "shift_left", "shift_right_logical", "shift_right_arithmetic"};
const std::unordered_set<std::string> kUnary = {
    "negate", "exponential", "exponential_minus_one", "log", "log_plus_one", "tanh", "sqrt",
    "rsqrt", "cbrt", "abs", "sine", "cosine", "tan", "floor", "ceil", "sign", "round_nearest_even",
    "round_nearest_afz", "logistic", "not", "is_finite", "popcnt", "count_leading_zeros", "erf",
    "reduce_precision"};
const std::unordered_set<std::string> kIndexMap = {
    "broadcast_in_dim", "reshape", "transpose", "slice", "concatenate", "pad", "iota",
    "constant", "convert", "bitcast_convert", "gather", "reverse", "dynamic_slice", "dynamic_update_slice",
    "broadcast"};
// index maps whose operand index depends on runtime data (an index tensor or scalar offsets)
bool DataDependentIndex(const Op* op) {
  return op->name == "gather" || op->name == "dynamic_slice" || op->name == "dynamic_update_slice";
}
const std::unordered_set<std::string> kAliasCustom = {"Sharding", "SPMDFullToShardShape", "SPMDShardToFullShape"};

bool IsElementwise(const Op* op) {
  return kBinary.count(op->name) || kUnary.count(op->name) || kIndexMap.count(op->name) ||
         op->name == "compare" || op->name == "select" || op->name == "clamp";
}
bool IsAlias(const Op* op) {
  if (op->name == "custom_call") {
    auto it = op->strs.find("call_target_name");
    return it != op->strs.end() && kAliasCustom.count(it->second);
  }
  return op->name == "optimization_barrier";
}

// ------------------------------------------------------------------------------------ C helpers
std::string CType(DT t) {   // register ("compute") type
  switch (t) {
    case DT::kPred: return "bool";
    case DT::kS8: case DT::kS16: case DT::kS32: return "int";
    case DT::kS64: return "long long";
    case DT::kU8: case DT::kU16: case DT::kU32: return "unsigned";
    case DT::kU64: return "unsigned long long";
    case DT::kF16: case DT::kBF16: case DT::kF32: return "float";
    case DT::kF64: return "double";
    default: return "void";
  }
}
int DTBits(DT t) { return 8 * DTBytes(t); }
// all-ones mask of an integer type's width, as an unsigned long long literal
std::string WidthMask(DT t) {
  int w = DTBits(t);
  return w >= 64 ? std::string("0xffffffffffffffffULL") : std::to_string((1ULL << w) - 1) + "ULL";
}
// unsigned / signed C types of an integer type's width
std::string UType(DT t) { return DTBytes(t) == 8 ? "unsigned long long" : "unsigned"; }
std::string SType(DT t) {
  switch (DTBytes(t)) {
    case 1: return "signed char";
    case 2: return "short";
    case 4: return "int";
    default: return "long long";
  }
}

std::string MemType(DT t) {  // storage type
  switch (t) {
    case DT::kPred: return "unsigned char";
    case DT::kS8: return "signed char";
    case DT::kS16: return "short";
    case DT::kS32: return "int";
    case DT::kS64: return "long long";
    case DT::kU8: return "unsigned char";
    case DT::kU16: return "unsigned short";
    case DT::kU32: return "unsigned";
    case DT::kU64: return "unsigned long long";
    case DT::kF16: case DT::kBF16: return "unsigned short";
    case DT::kF32: return "float";
    case DT::kF64: return "double";
    default: return "void";
  }
}
std::string LoadExpr(DT t, const std::string& ptr, const std::string& idx) {
  std::string raw = ptr + "[" + idx + "]";
  if (t == DT::kBF16) return "bf2f(" + raw + ")";
  if (t == DT::kF16) return "h2f(" + raw + ")";
  if (t == DT::kPred) return "(" + raw + " != 0)";
  return "(" + CType(t) + ")" + raw;
}
// A bf16-typed register always holds a value that bf16 represents exactly (loads are exact and
// every op that makes a bf16 value rounds it), so storing it is a shift, not a conversion.
std::string StoreExpr(DT t, const std::string& v) {
  if (t == DT::kBF16) return "bf_bits(" + v + ")";
  if (t == DT::kF16) return "f2h(" + v + ")";
  if (t == DT::kPred) return "(unsigned char)(" + v + ")";
  return "(" + MemType(t) + ")(" + v + ")";
}

// two 16-bit float values packed into one 32-bit word, the first in the low half
std::string Pack16(DT t, const std::string& a, const std::string& b) {
  if (t == DT::kBF16) return "((__float_as_uint(" + a + ") >> 16) | (__float_as_uint(" + b + ") & 0xffff0000u))";
  return "((unsigned)f2h(" + a + ") | ((unsigned)f2h(" + b + ") << 16))";
}

std::string FloatLit(double d) {
  float f = (float)d;
  uint32_t u;
  std::memcpy(&u, &f, 4);
  char buf[48];
  std::snprintf(buf, sizeof(buf), "__int_as_float(0x%08x)", u);
  return buf;
}
std::string DoubleLit(double d) {
  uint64_t u;
  std::memcpy(&u, &d, 8);
  char buf[64];
  std::snprintf(buf, sizeof(buf), "__longlong_as_double(0x%016llxLL)", (unsigned long long)u);
  return buf;
}
// round-to-nearest-even of a float to bf16 precision (host side, for literals)
float RoundBf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return f;   // NaN stays NaN
  u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  std::memcpy(&f, &u, 4);
  return f;
}

std::string Literal(DT t, double v) {
  if (t == DT::kBF16) return FloatLit(RoundBf16((float)v));
  if (t == DT::kF32 || t == DT::kF16) return FloatLit(v);
  if (t == DT::kF64) return DoubleLit(v);
  if (t == DT::kPred) return v != 0 ? "true" : "false";
  if (DTIsUnsigned(t)) return std::to_string((unsigned long long)v) + "ULL";
  return "(" + CType(t) + ")(" + std::to_string((long long)v) + "LL)";
}

const char* kPrelude = R"(
// ---- generated by the B200 PJRT plugin (sm_100a) ----
__device__ __forceinline__ float bf2f(unsigned short h) { return __uint_as_float(((unsigned)h) << 16); }
__device__ __forceinline__ unsigned short f2bf(float f) {
  unsigned short r; asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f)); return r; }
__device__ __forceinline__ float h2f(unsigned short h) {
  float f; asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h)); return f; }
__device__ __forceinline__ unsigned short f2h(float f) {
  unsigned short r; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(r) : "f"(f)); return r; }
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }
__device__ __forceinline__ float fmax_nan(float a, float b) { float r; asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b)); return r; }
__device__ __forceinline__ float ex2a(float x) { float r; asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x)); return r; }
__device__ __forceinline__ unsigned short bf_bits(float f) { return (unsigned short)(__float_as_uint(f) >> 16); }
__device__ __forceinline__ float rhf(float f) { return h2f(f2h(f)); }
__device__ __forceinline__ float fmax_n(float a, float b) { return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b); }
__device__ __forceinline__ float fmin_n(float a, float b) { return (a != a || b != b) ? __int_as_float(0x7fc00000) : fminf(a, b); }
__device__ __forceinline__ double dmax_n(double a, double b) { return (a != a || b != b) ? __longlong_as_double(0x7ff8000000000000LL) : fmax(a, b); }
__device__ __forceinline__ double dmin_n(double a, double b) { return (a != a || b != b) ? __longlong_as_double(0x7ff8000000000000LL) : fmin(a, b); }
template <typename T> __device__ __forceinline__ T imax(T a, T b) { return a > b ? a : b; }
template <typename T> __device__ __forceinline__ T imin(T a, T b) { return a < b ? a : b; }
__device__ __forceinline__ float fsign(float x) { return x > 0.f ? 1.f : (x < 0.f ? -1.f : x); }
__device__ __forceinline__ float frne(float x) { return rintf(x); }
__device__ __forceinline__ float fafz(float x) { return roundf(x); }
__device__ __forceinline__ float flogistic(float x) { return 1.f / (1.f + expf(-x)); }
// tanh(u) = 1 - 2 / (e^(2u) + 1) to an absolute error of a few 1e-7 (relative accuracy is lost for
// |u| << 1), exponential and reciprocal on the SFU; for readers that only form 1 +- tanh(u)
__device__ __forceinline__ float ftanh_abs(float u) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + ex2a(u * 2.88539008177792681f)));  // 2 log2(e)
  return fmaf(-2.f, r, 1.f);
}
// 1 / (1 + e^(-2u)) = (1 + tanh(u)) / 2, with the exponential and the reciprocal on the SFU
__device__ __forceinline__ float fsig2(float u) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + ex2a(u * -2.88539008177792681f)));  // -2 log2(e)
  return r;
}
__device__ __forceinline__ float warp_sum(float v) { for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o); return v; }
__device__ __forceinline__ double warp_sum(double v) { for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o); return v; }
)";

// ------------------------------------------------------------------------------------ codegen
// Emits the per-element expression of a fusion: values that are not materialized are computed
// inline from their operands; materialized values are loaded from their slot.
struct Gen {
  const std::vector<int>* slot_of;        // value id -> slot (-1 if not materialized)
  std::vector<int> in_slots;              // kernel input params (slots)
  std::unordered_map<int, int> param_of;  // slot -> param index
  std::unordered_map<std::string, std::string> cse;
  std::unordered_map<int, std::string> group_regs;  // slot of a group member -> its register
  std::vector<std::string> identity;      // loop index names of the current group shape
  std::vector<int64_t> group_dims;
  bool conflict = false;
  std::set<int> nonident;                 // slots some load reads away from the element being computed
  std::ostringstream body;
  int tmp = 0;
  std::string indent = "    ";

  std::string Var(DT t, const std::string& expr) {
    std::string n = "t" + std::to_string(tmp++);
    body << indent << CType(t) << " " << n << " = " << expr << ";\n";
    return n;
  }

  std::string Param(int slot) {
    auto it = param_of.find(slot);
    if (it != param_of.end()) return "in" + std::to_string(it->second);
    int k = (int)in_slots.size();
    in_slots.push_back(slot);
    param_of[slot] = k;
    return "in" + std::to_string(k);
  }

  static std::string Linear(const std::vector<std::string>& idx, const std::vector<int64_t>& dims) {
    if (dims.empty()) return "0";
    std::string s;
    for (size_t k = 0; k < dims.size(); ++k) {
      if (k == 0) s = "(long long)(" + idx[0] + ")";
      else if (dims[k] == 1) s = "(" + s + ")";
      else s = "(" + s + ")*" + std::to_string(dims[k]) + "LL+(" + idx[k] + ")";
    }
    return s;
  }

  std::string Round(DT t, const std::string& v) {
    if (t == DT::kBF16) return Var(t, "rbf(" + v + ")");
    if (t == DT::kF16) return Var(t, "rhf(" + v + ")");
    return v;
  }

  std::string Emit(const Value* v, const std::vector<std::string>& idx) {
    std::string key = std::to_string(v->id);
    for (auto& s : idx) key += "|" + s;
    auto hit = cse.find(key);
    if (hit != cse.end()) return hit->second;
    std::string r = EmitUncached(v, idx);
    cse[key] = r;
    return r;
  }

  // Vector mode (loop kernels whose innermost extent is a multiple of 4): the element function
  // handles 4 consecutive elements; lane v's innermost loop index is named `vinner_v`.  A leaf read
  // whose innermost index is exactly that name (and whose other indices do not depend on it) is
  // contiguous and 4-aligned across the lanes, so lane 0 issues one vector load for all four.
  bool vec = false;
  std::string vinner;
  int branch_depth = 0;                                   // inside concatenate / pad branches
  std::unordered_map<std::string, std::string> vloads;    // leaf base -> vector register
  std::unordered_map<std::string, std::vector<std::string>> reindex_cse;   // vector-mode reshapes
  std::vector<std::vector<std::string>> lane_identity;   // identity index per lane (vector mode)
  std::unordered_map<int, std::vector<std::string>> lane_group_regs;
  // Ragged-row walks (non-empty shift_dims): the lanes' four elements are 16-byte aligned only in
  // tensors of exactly these dims read at the current row (index prefix shift_prefix); other reads
  // are scalar.
  std::vector<int64_t> shift_dims;
  std::vector<std::string> shift_prefix;

  // Lane-affine index strings: the innermost index of lane l equals lane 0's (`base`) plus l.  The
  // group's own lane names (vinner_l) are; reshapes, slices and pads that keep four consecutive
  // elements consecutive produce more (canonical names, see Canon), each recorded here with whether
  // its lane-0 value is a multiple of 4 (then lane 0 may issue one vector access for all four).
  struct LaneIx {
    std::string base;
    int lane = 0;
    bool al4 = false;
    bool exact = true;       // the string's value is base + lane (false: clamped at the row's end)
  };
  std::unordered_map<std::string, LaneIx> lane_ix;
  bool lanes_clamped = false;   // padded ragged rows: lanes past the end hold the last index
  bool LaneInfo(const std::string& s, LaneIx* out) const {
    if (!vec) return false;
    if (s.size() == vinner.size() + 2 && s.compare(0, vinner.size() + 1, vinner + "_") == 0 && s.back() >= '0' &&
        s.back() <= '3') {
      *out = LaneIx{vinner + "_0", s.back() - '0', shift_dims.empty(), !lanes_clamped};
      return true;
    }
    auto it = lane_ix.find(s);
    if (it == lane_ix.end()) return false;
    *out = it->second;
    return true;
  }
  std::string Canon(const std::string& base, int l) const {
    if (l == 0) return base;
    if (base == vinner + "_0") return vinner + "_" + std::to_string(l);
    return "(" + base + "+" + std::to_string(l) + ")";
  }
  // records the lane strings of a derived lane-0 index `b0` and returns lane l's
  std::string DeriveLane(const std::string& b0, int l, bool al4) {
    lane_ix[b0] = LaneIx{b0, 0, al4};
    const std::string c = Canon(b0, l);
    lane_ix[c] = LaneIx{b0, l, al4};
    return c;
  }

  int LaneOf(const std::vector<std::string>& idx) const {
    if (!vec || idx.empty()) return -1;
    LaneIx li;
    if (!LaneInfo(idx.back(), &li)) return -1;
    for (size_t k = 0; k + 1 < idx.size(); ++k)
      if (idx[k].find(vinner + "_") != std::string::npos || lane_ix.count(idx[k])) return -1;
    return li.lane;
  }

  std::string VecLoad(DT dt, int slot, const std::vector<std::string>& idx, int lane) {
    std::vector<std::string> base = idx;
    LaneIx li;
    LaneInfo(idx.back(), &li);
    base.back() = li.base;
    std::string key = std::to_string(slot);
    for (auto& s : base) key += "|" + s;
    auto it = vloads.find(key);
    std::string name;
    if (it == vloads.end()) {
      name = "v" + std::to_string(tmp++);
      if (dt == DT::kF32) body << indent << "const float4 " << name << " = *(const float4*)(" << Param(slot) << " + (" << LinearDims(base) << "));\n";
      else body << indent << "const uint2 " << name << " = *(const uint2*)(" << Param(slot) << " + (" << LinearDims(base) << "));\n";
      vloads[key] = name;
    } else {
      name = it->second;
    }
    if (dt == DT::kF32) {
      static const char* c[] = {".x", ".y", ".z", ".w"};
      return name + c[lane];
    }
    // 4 x 16-bit: .x = lanes 0,1 (low half first), .y = lanes 2,3
    std::string word = name + (lane < 2 ? ".x" : ".y");
    std::string half = (lane & 1) ? "(unsigned short)(" + word + " >> 16)" : "(unsigned short)(" + word + " & 0xffffu)";
    return Var(dt, dt == DT::kBF16 ? "bf2f(" + half + ")" : "h2f(" + half + ")");
  }
  std::vector<int64_t> cur_dims;   // dims of the leaf being vector-loaded (set by the caller)
  int64_t cur_pitch = 0;           // and its padded row pitch (0: dense)
  std::string LinearDims(const std::vector<std::string>& idx) const {
    return cur_pitch ? PitchedLinear(idx, cur_dims, cur_pitch) : Linear(idx, cur_dims);
  }
  // slots stored with a padded innermost row pitch (a dot's output whose rows break the 16-byte
  // rule, or a dot operand stored for in-place use)
  const std::unordered_map<int, int64_t>* slot_pitch = nullptr;
  const std::unordered_set<int>* slot_f32 = nullptr;   // slots holding 16-bit values as f32
  int64_t SlotPitch(int slot) const {
    if (!slot_pitch) return 0;
    auto it = slot_pitch->find(slot);
    return it == slot_pitch->end() ? 0 : it->second;
  }
  static std::string PitchedLinear(const std::vector<std::string>& idx, const std::vector<int64_t>& dims, int64_t pitch) {
    std::vector<std::string> outer(idx.begin(), idx.end() - 1);
    std::vector<int64_t> od(dims.begin(), dims.end() - 1);
    return "(" + Linear(outer, od) + ")*" + std::to_string(pitch) + "LL+(" + idx.back() + ")";
  }

  // Row-group mode: values already reduced or computed for the current row live in registers and
  // may only be read at the row's own index (`row_ident`; unit dims may read index 0).
  std::unordered_map<int, std::string> fixed;   // value id -> register
  std::vector<std::string> row_ident;
  std::vector<int64_t> row_dims;
  // idx (over dims) names the current row: its non-unit entries are the row's non-unit indices
  // (an index into a unit dim can only be 0)
  bool SameRow(const std::vector<std::string>& idx, const std::vector<int64_t>& dims) const {
    std::vector<std::string> a, b;
    for (size_t k = 0; k < dims.size(); ++k) if (dims[k] != 1) a.push_back(idx[k]);
    for (size_t k = 0; k < row_dims.size(); ++k) if (row_dims[k] != 1) b.push_back(row_ident[k]);
    return a == b;
  }
  // the index of the current row in a row-shaped value of shape dims
  std::vector<std::string> RowIndex(const std::vector<int64_t>& dims) const {
    std::vector<std::string> b, out;
    for (size_t k = 0; k < row_dims.size(); ++k) if (row_dims[k] != 1) b.push_back(row_ident[k]);
    size_t q = 0;
    for (int64_t d : dims) out.push_back(d != 1 && q < b.size() ? b[q++] : "0");
    return out;
  }

  static bool IsSplat(const Value* v) {
    while (v->def && v->def->name == "broadcast_in_dim") v = v->def->operands[0];
    return v->def && v->def->name == "constant" && v->def->splat;
  }
  // t = tanh(u) read only through sums / differences with constants (1 + t, 1 - t) and its square
  // t * t, itself read only through such sums: the readers need t to an absolute, not a relative,
  // accuracy (the tanh-GELU derivative 0.5 (1 + t) + ... (1 - t^2) ...)
  static bool TanhOnlyNearOne(const Value* t) {
    if (t->users.empty()) return false;
    auto const_sum = [](const Op* u, const Value* x) {
      return (u->name == "add" || u->name == "subtract") && u->operands.size() == 2 &&
             ((u->operands[0] == x && IsSplat(u->operands[1])) || (u->operands[1] == x && IsSplat(u->operands[0])));
    };
    for (const Op* u : t->users) {
      if (const_sum(u, t)) continue;
      if (u->name == "multiply" && u->operands.size() == 2 && u->operands[0] == t && u->operands[1] == t) {
        const Value* sq = u->result();
        if (sq->users.empty()) return false;
        for (const Op* w : sq->users)
          if (!const_sum(w, sq)) return false;
        continue;
      }
      return false;
    }
    return true;
  }
  static bool SplatIs(const Value* v, double want) {
    while (v->def && v->def->name == "broadcast_in_dim") v = v->def->operands[0];
    return v->def && v->def->name == "constant" && v->def->splat && ConstScalar(v->def) == want;
  }
  // v = (0.5 * h) * (1 + tanh(u)), operands of each product and sum in either order, all f32
  static bool GeluTanhForm(const Value* v, const Value** h, const Value** u) {
    const Op* m = v->def;
    if (!m || m->name != "multiply" || m->operands.size() != 2) return false;
    for (int s = 0; s < 2; ++s) {
      const Op* half = m->operands[s]->def;
      const Op* sum = m->operands[1 - s]->def;
      if (!half || !sum || half->name != "multiply" || sum->name != "add") continue;
      const Value* hv = SplatIs(half->operands[0], 0.5) ? half->operands[1] : SplatIs(half->operands[1], 0.5) ? half->operands[0] : nullptr;
      const Value* tv = SplatIs(sum->operands[0], 1.0) ? sum->operands[1] : SplatIs(sum->operands[1], 1.0) ? sum->operands[0] : nullptr;
      if (!hv || !tv || !tv->def || tv->def->name != "tanh" || hv->type.dt != DT::kF32 || tv->type.dt != DT::kF32) continue;
      *h = hv;
      *u = tv->def->operands[0];
      return true;
    }
    return false;
  }

  std::string EmitUncached(const Value* v, const std::vector<std::string>& idx) {
    const TensorType& ty = v->type;
    auto fx = fixed.find(v->id);
    if (fx != fixed.end()) {
      if (!SameRow(idx, ty.dims)) conflict = true;
      return fx->second;
    }
    int slot = (*slot_of)[v->id];
    if (slot >= 0) {
      auto g = group_regs.find(slot);
      if (g != group_regs.end()) {
        if (idx == identity && ty.dims == group_dims) return g->second;
        if (vec && ty.dims == group_dims) {
          auto lg = lane_group_regs.find(slot);
          for (size_t l = 0; lg != lane_group_regs.end() && l < lane_identity.size(); ++l)
            if (idx == lane_identity[l] && l < lg->second.size()) return lg->second[l];
        }
        conflict = true;
      }
      const int lane = branch_depth == 0 ? LaneOf(idx) : -1;
      LaneIx li;
      const bool lane_ok = lane >= 0 && LaneInfo(idx.back(), &li);
      // a padded row pitch (a multiple of 4 elements) keeps every row 16-byte aligned
      const int64_t pitch = SlotPitch(slot);
      const bool aligned4 = lane_ok && (shift_dims.empty()
                                ? li.al4 && !ty.dims.empty() && (pitch ? pitch % 4 == 0 : ty.dims.back() % 4 == 0)
                                : !pitch && ty.dims == shift_dims && idx.size() == shift_prefix.size() + 1 && li.base == vinner + "_0" &&
                                      std::equal(shift_prefix.begin(), shift_prefix.end(), idx.begin()));
      const bool wide16 = slot_f32 && slot_f32->count(slot) && (ty.dt == DT::kBF16 || ty.dt == DT::kF16);
      if (ty.dims != group_dims || (idx != identity && std::find(lane_identity.begin(), lane_identity.end(), idx) == lane_identity.end()))
        nonident.insert(slot);
      if (lane >= 0 && (ty.dt == DT::kF32 || ty.dt == DT::kBF16 || ty.dt == DT::kF16) && aligned4) {
        cur_dims = ty.dims;
        cur_pitch = pitch;
        if (wide16) return Round(ty.dt, Var(DT::kF32, VecLoad(DT::kF32, slot, idx, lane)));
        std::string r = VecLoad(ty.dt, slot, idx, lane);
        return ty.dt == DT::kF32 ? Var(ty.dt, r) : r;
      }
      const std::string lin = pitch ? PitchedLinear(idx, ty.dims, pitch) : Linear(idx, ty.dims);
      if (wide16) return Round(ty.dt, Var(DT::kF32, LoadExpr(DT::kF32, Param(slot), lin)));
      return Var(ty.dt, LoadExpr(ty.dt, Param(slot), lin));
    }
    const Op* op = v->def;
    if (!op) throw LowerError{"internal: unmaterialized argument"};
    const std::string& n = op->name;
    auto opnd = [&](int k, const std::vector<std::string>& i) { return Emit(op->operands[k], i); };
    if (IsAlias(op)) return opnd(0, idx);
    if (n == "constant") {
      if (!op->splat) throw LowerError{"internal: non-splat constant not materialized"};
      return Literal(ty.dt, ConstScalar(op));
    }
    if (n == "iota") {
      int d = (int)op->ints.at("dim")[0];
      return Round(ty.dt, Var(ty.dt, "(" + CType(ty.dt) + ")(" + idx[d] + ")"));
    }
    if (n == "broadcast_in_dim") {
      const auto& dims = op->ints.at("dims");
      const auto& in = op->operands[0]->type.dims;
      std::vector<std::string> j(in.size());
      for (size_t k = 0; k < in.size(); ++k) j[k] = (in[k] == 1 && ty.dims[dims[k]] != 1) ? "0" : idx[dims[k]];
      return opnd(0, j);
    }
    if (n == "reshape" || (n == "bitcast_convert" && DTBytes(ty.dt) == DTBytes(op->operands[0]->type.dt) && false)) {
      const auto& in = op->operands[0]->type.dims;
      LaneIx li;
      if (vec && !idx.empty() && !in.empty() && ty.dims.back() % 4 == 0 && in.back() % 4 == 0 && LaneInfo(idx.back(), &li) &&
          li.al4 && li.exact) {
        // four consecutive, 4-aligned elements of the result are four consecutive elements of the
        // operand's innermost dim: lane l reads lane 0's operand index with the innermost + l
        std::vector<std::string> idx0 = idx;
        idx0.back() = li.base;
        std::string key;
        for (auto& q : idx0) key += q + "|";
        for (int64_t d : in) key += std::to_string(d) + ",";
        auto hit = reindex_cse.find(key);
        std::vector<std::string> j0 = hit != reindex_cse.end() ? hit->second : Reindex(idx0, ty.dims, in);
        reindex_cse[key] = j0;
        std::vector<std::string> j = j0;
        j.back() = DeriveLane(j0.back(), li.lane, true);
        return opnd(0, j);
      }
      return opnd(0, Reindex(idx, ty.dims, in));
    }
    if (n == "transpose") {
      const auto& perm = op->ints.at("dims");
      std::vector<std::string> j(perm.size());
      for (size_t k = 0; k < perm.size(); ++k) j[perm[k]] = idx[k];
      return opnd(0, j);
    }
    if (n == "broadcast") {
      // the legacy broadcast prepends dimensions: the operand is indexed by the trailing ones
      const size_t lead = ty.dims.size() - op->operands[0]->type.dims.size();
      return opnd(0, std::vector<std::string>(idx.begin() + lead, idx.end()));
    }
    if (n == "reverse") {
      const auto& dims = op->ints.count("dims") ? op->ints.at("dims") : op->ints.at("dimensions");
      std::vector<std::string> j = idx;
      for (int64_t d : dims) j[d] = "(" + std::to_string(ty.dims[d] - 1) + "-(" + idx[d] + "))";
      return opnd(0, j);
    }
    if (n == "slice") {
      const auto& st = op->ints.at("start_indices");
      const auto& sd = op->ints.at("strides");
      std::vector<std::string> j(idx.size());
      for (size_t k = 0; k < idx.size(); ++k)
        j[k] = "(" + std::to_string(st[k]) + "+(" + idx[k] + ")*" + std::to_string(sd[k]) + ")";
      LaneIx li;
      if (!idx.empty() && sd.back() == 1 && LaneInfo(idx.back(), &li) && li.exact)
        j.back() = DeriveLane("(" + std::to_string(st.back()) + "+(" + li.base + ")*1)", li.lane, li.al4 && st.back() % 4 == 0);
      return opnd(0, j);
    }
    if (n == "bitcast_convert") {
      // same-width reinterpretation of the bits (a 16-bit float register holds an exactly
      // representable value, so its bits are a shift / exact conversion away)
      DT from = op->operands[0]->type.dt, to = ty.dt;
      if (DTBytes(from) != DTBytes(to) || from == DT::kPred || to == DT::kPred || op->operands[0]->type.dims != ty.dims)
        throw LowerError{std::string("bitcast_convert from ") + DTName(from) + " to " + DTName(to) +
                         " is not supported (only between element types of the same width)"};
      std::string x = opnd(0, idx), b;
      if (from == DT::kF32) b = "(unsigned long long)__float_as_uint(" + x + ")";
      else if (from == DT::kBF16) b = "(unsigned long long)(__float_as_uint(" + x + ") >> 16)";
      else if (from == DT::kF16) b = "(unsigned long long)f2h(" + x + ")";
      else if (from == DT::kF64) b = "(unsigned long long)__double_as_longlong(" + x + ")";
      else b = "((unsigned long long)(" + x + ") & " + WidthMask(from) + ")";
      b = Var(DT::kU64, b);
      std::string e;
      if (to == DT::kF32) e = "__uint_as_float((unsigned)" + b + ")";
      else if (to == DT::kBF16) e = "__uint_as_float((unsigned)" + b + " << 16)";
      else if (to == DT::kF16) e = "h2f((unsigned short)" + b + ")";
      else if (to == DT::kF64) e = "__longlong_as_double((long long)" + b + ")";
      else if (DTIsSigned(to)) e = "(" + CType(to) + ")(" + SType(to) + ")" + b;
      else e = "(" + CType(to) + ")(" + MemType(to) + ")" + b;
      return Var(to, e);
    }
    if (n == "dynamic_slice" || n == "dynamic_update_slice") {
      // start offsets are runtime scalars, clamped so the window stays inside the operand (the
      // StableHLO rule): start_k = clamp(start_k, 0, dim_k - window_k)
      const bool upd = n == "dynamic_update_slice";
      const auto& in = op->operands[0]->type.dims;
      const size_t first = upd ? 2 : 1;
      if (op->operands.size() != first + in.size()) throw LowerError{n + ": expected one scalar start index per dimension"};
      std::vector<int64_t> win(in.size());
      for (size_t k = 0; k < in.size(); ++k) {
        if (upd) win[k] = op->operands[1]->type.dims[k];
        else win[k] = op->ints.count("sizes") ? op->ints.at("sizes")[k] : ty.dims[k];
      }
      std::vector<std::string> st(in.size());
      for (size_t k = 0; k < in.size(); ++k) {
        if (!op->operands[first + k]->type.dims.empty()) throw LowerError{n + ": start indices must be scalars"};
        std::string sv = Emit(op->operands[first + k], {});
        const DT it = op->operands[first + k]->type.dt;
        const std::string hi = std::to_string(in[k] - win[k]);
        if (it == DT::kU64 || it == DT::kU32 || it == DT::kU16 || it == DT::kU8)
          // unsigned starts are never below 0; clamp in unsigned arithmetic so a u64 start of 2^63 or
          // more stays a large value (clamped to dim - window), not a negative one
          st[k] = Var(DT::kS64, "(long long)((unsigned long long)(" + sv + ") < " + hi + "ULL ? (unsigned long long)(" + sv +
                                ") : " + hi + "ULL)");
        else
          st[k] = Var(DT::kS64, "imin(imax((long long)(" + sv + "), 0LL), " + hi + "LL)");
      }
      if (!upd) {
        std::vector<std::string> j(idx.size());
        for (size_t k = 0; k < idx.size(); ++k) j[k] = "(" + st[k] + "+(" + idx[k] + "))";
        return opnd(0, j);
      }
      std::string r = "t" + std::to_string(tmp++);
      body << indent << CType(ty.dt) << " " << r << ";\n";
      std::string cond = "true";
      std::vector<std::string> j(idx.size());
      for (size_t k = 0; k < idx.size(); ++k) {
        j[k] = "((" + idx[k] + ")-" + st[k] + ")";
        cond += " && " + j[k] + " >= 0 && " + j[k] + " < " + std::to_string(win[k]) + "LL";
      }
      std::string save = indent;
      for (int side = 0; side < 2; ++side) {
        body << save << (side == 0 ? "if (" + cond + ") {\n" : std::string("} else {\n"));
        indent = save + "  ";
        auto saved = cse;
        auto saved_r = reindex_cse;
        ++branch_depth;
        std::string x = side == 0 ? Emit(op->operands[1], j) : opnd(0, idx);
        --branch_depth;
        cse = saved;
        reindex_cse = saved_r;
        body << indent << r << " = " << x << ";\n";
      }
      indent = save;
      body << indent << "}\n";
      return r;
    }
    if (n == "convert") {
      DT from = op->operands[0]->type.dt, to = ty.dt;
      std::string x = opnd(0, idx);
      if (to == DT::kPred) return Var(to, "(" + x + " != 0)");
      if (DTIsFloat(from) && !DTIsFloat(to)) {
        // float -> int: truncate toward zero, NaN -> 0, saturate (cvt.rzi semantics)
        if (from == DT::kF64) return Var(to, "(" + CType(to) + ")(" + x + ")");
        return Var(to, "(" + CType(to) + ")(" + x + ")");
      }
      std::string c = "(" + CType(to) + ")(" + x + ")";
      if (from == DT::kF64 && (to == DT::kBF16 || to == DT::kF16)) c = "(float)(" + x + ")";  // double rounding accepted
      return Round(to, Var(to, c));
    }
    if (n == "compare") {
      DT t = op->operands[0]->type.dt;
      std::string a = opnd(0, idx), b = opnd(1, idx);
      std::string d = op->strs.at("comparison_direction");
      auto ct = op->strs.find("compare_type");
      if (ct != op->strs.end() && ct->second == "UNSIGNED" && DTIsSigned(t)) {
        std::string u = t == DT::kS64 ? "(unsigned long long)" : "(unsigned)";
        a = u + a;
        b = u + b;
      }
      static const std::map<std::string, std::string> sym = {
          {"EQ", "=="}, {"NE", "!="}, {"LT", "<"}, {"LE", "<="}, {"GT", ">"}, {"GE", ">="}};
      return Var(DT::kPred, "(" + a + " " + sym.at(d) + " " + b + ")");
    }
    if (n == "select") {
      const auto& pd = op->operands[0]->type.dims;
      std::string p = Emit(op->operands[0], pd.empty() ? std::vector<std::string>{} : idx);
      std::string a = opnd(1, idx), b = opnd(2, idx);
      return Var(ty.dt, "(" + p + " ? " + a + " : " + b + ")");
    }
    if (n == "clamp") {
      auto sc = [&](int k) { return op->operands[k]->type.dims.empty() ? std::vector<std::string>{} : idx; };
      std::string lo = Emit(op->operands[0], sc(0)), x = opnd(1, idx), hi = Emit(op->operands[2], sc(2));
      if (DTIsFloat(ty.dt)) return Var(ty.dt, "fmin_n(fmax_n(" + x + ", " + lo + "), " + hi + ")");
      return Var(ty.dt, "imin(imax(" + x + ", " + lo + "), " + hi + ")");
    }
    if (n == "concatenate") {
      int d = (int)op->ints.at("dim")[0];
      std::string r = "t" + std::to_string(tmp++);
      body << indent << CType(ty.dt) << " " << r << ";\n";
      int64_t off = 0;
      std::string save = indent;
      for (size_t k = 0; k < op->operands.size(); ++k) {
        int64_t len = op->operands[k]->type.dims[d];
        std::vector<std::string> j = idx;
        j[d] = "((" + idx[d] + ")-" + std::to_string(off) + ")";
        body << indent << (k ? "else " : "") << "if ((" << idx[d] << ") < " << off + len << ") {\n";
        indent += "  ";
        auto saved = cse;          // values computed inside a branch are not visible outside
        auto saved_r = reindex_cse;
        ++branch_depth;
        std::string x = Emit(op->operands[k], j);
        --branch_depth;
        cse = saved;
        reindex_cse = saved_r;
        body << indent << r << " = " << x << ";\n";
        indent = save;
        body << indent << "}\n";
        off += len;
      }
      return r;
    }
    if (n == "pad") {
      // pretty form: low / high / interior; generic form: edge_padding_low / interior_padding
      const auto& lo = op->ints.count("low") ? op->ints.at("low") : op->ints.at("edge_padding_low");
      const auto& it = op->ints.count("interior") ? op->ints.at("interior") : op->ints.at("interior_padding");
      const auto& ind = op->operands[0]->type.dims;
      LaneIx li;
      if (vec && branch_depth == 0 && !idx.empty() && LaneInfo(idx.back(), &li) && li.al4 && li.exact && li.lane == 0 &&
          lo.back() % 4 == 0 && it.back() == 0 && ind.back() % 4 == 0 && ty.dims.back() % 4 == 0) {
        // the four lanes lie on the same side of every edge: one branch computes all four (their
        // reads inside may then be one vector access) and lanes 1-3 are left in the value cache
        std::string pv = Emit(op->operands[1], {});
        std::vector<std::string> r(4), cond_parts;
        for (int l = 0; l < 4; ++l) {
          r[l] = "t" + std::to_string(tmp++);
          body << indent << CType(ty.dt) << " " << r[l] << " = " << pv << ";\n";
        }
        std::string cond = "true";
        std::vector<std::string> j(idx.size());
        for (size_t k = 0; k < idx.size(); ++k) {
          std::string q = "((" + idx[k] + ")-(" + std::to_string(lo[k]) + "))";
          int64_t s = it[k] + 1;
          cond += " && " + q + " >= 0 && " + q + " < " + std::to_string((ind[k] - 1) * s + 1);
          if (s > 1) cond += " && " + q + " % " + std::to_string(s) + " == 0";
          j[k] = s > 1 ? "(" + q + "/" + std::to_string(s) + ")" : q;
        }
        const std::string q0 = j.back();
        body << indent << "if (" << cond << ") {\n";
        std::string save = indent;
        indent += "  ";
        auto saved = cse;
        auto saved_v = vloads;
        auto saved_r = reindex_cse;
        for (int l = 0; l < 4; ++l) {
          std::vector<std::string> jl = j;
          jl.back() = DeriveLane(q0, l, true);
          const std::string x = Emit(op->operands[0], jl);
          body << indent << r[l] << " = " << x << ";\n";
        }
        cse = saved;
        vloads = saved_v;
        reindex_cse = saved_r;
        indent = save;
        body << indent << "}\n";
        for (int l = 1; l < 4; ++l) {
          std::string key = std::to_string(v->id);
          for (size_t k = 0; k + 1 < idx.size(); ++k) key += "|" + idx[k];
          key += "|" + Canon(li.base, l);
          cse[key] = r[l];
        }
        return r[0];
      }
      std::string pv = Emit(op->operands[1], {});
      std::string r = "t" + std::to_string(tmp++);
      body << indent << CType(ty.dt) << " " << r << " = " << pv << ";\n";
      const auto& in = op->operands[0]->type.dims;
      std::string cond = "true";
      std::vector<std::string> j(idx.size());
      for (size_t k = 0; k < idx.size(); ++k) {
        std::string q = "((" + idx[k] + ")-(" + std::to_string(lo[k]) + "))";
        int64_t s = it[k] + 1;
        cond += " && " + q + " >= 0 && " + q + " < " + std::to_string((in[k] - 1) * s + 1);
        if (s > 1) cond += " && " + q + " % " + std::to_string(s) + " == 0";
        j[k] = s > 1 ? "(" + q + "/" + std::to_string(s) + ")" : q;
      }
      body << indent << "if (" << cond << ") {\n";
      std::string save = indent;
      indent += "  ";
      auto saved = cse;
      auto saved_r = reindex_cse;
      ++branch_depth;
      std::string x = Emit(op->operands[0], j);
      --branch_depth;
      cse = saved;
      reindex_cse = saved_r;
      body << indent << r << " = " << x << ";\n";
      indent = save;
      body << indent << "}\n";
      return r;
    }
    if (n == "gather") {
      // row take: table[V, D...] indexed by ids at the batch positions (see CheckGather)
      const Value* table = op->operands[0];
      const Value* ids = op->operands[1];
      const auto& offset_dims = op->ints.at("offset_dims");
      std::vector<std::string> bidx;
      for (size_t k = 0; k < idx.size(); ++k)
        if (std::find(offset_dims.begin(), offset_dims.end(), (int64_t)k) == offset_dims.end()) bidx.push_back(idx[k]);
      bidx.push_back("0");   // index_vector_dim (size 1)
      std::string id = Emit(ids, bidx);
      int64_t V = table->type.dims[0];
      std::string row = Var(DT::kS64, "(long long)(" + id + ") < 0 ? 0LL : ((long long)(" + id + ") > " +
                                          std::to_string(V - 1) + "LL ? " + std::to_string(V - 1) + "LL : (long long)(" + id + "))");
      std::vector<std::string> t{row};
      for (size_t k = 0; k < offset_dims.size(); ++k) t.push_back(idx[offset_dims[k]]);
      return Emit(table, t);
    }
    if (n == "tanh" && ty.dt == DT::kF32 && TanhOnlyNearOne(v)) {
      // every reader forms 1 + t, 1 - t, c - t or t * t: an absolute error of a few 1e-7 is all
      // the result can carry, which tanh(u) = 1 - 2 / (e^(2u) + 1) on the SFU delivers
      return Var(DT::kF32, "ftanh_abs(" + opnd(0, idx) + ")");
    }
    if (kUnary.count(n)) {
      std::string x = opnd(0, idx);
      DT t = ty.dt;
      bool f = DTIsFloat(t), d = t == DT::kF64;
      std::string e;
      if (n == "negate") e = "-" + x;
      else if (n == "abs") e = f ? (d ? "fabs(" + x + ")" : "fabsf(" + x + ")") : "(" + x + " < 0 ? -" + x + " : " + x + ")";
      else if (n == "not") e = t == DT::kPred ? "!" + x : "~" + x;
      else if (n == "is_finite") e = "isfinite(" + opnd(0, idx) + ")";
      else if (n == "sign") e = d ? "(double)((" + x + " > 0) - (" + x + " < 0))" : f ? "fsign(" + x + ")" : "((" + x + " > 0) - (" + x + " < 0))";
      else if (n == "popcnt" || n == "count_leading_zeros") {
        if (f || t == DT::kPred) throw LowerError{"unsupported op '" + n + "' for " + DTName(t)};
        // counted over the type's own width (8- / 16-bit values sit sign-extended in registers)
        const int w = DTBits(t);
        std::string u = "((unsigned long long)(" + x + ") & " + WidthMask(t) + ")";
        if (n == "popcnt") e = w == 64 ? "__popcll(" + u + ")" : "__popc((unsigned)" + u + ")";
        else e = w == 64 ? "__clzll((long long)" + u + ")" : "(__clz((int)(unsigned)" + u + ") - " + std::to_string(32 - w) + ")";
        e = "(" + CType(t) + ")(" + e + ")";
      } else if (n == "erf") {
        if (!f) throw LowerError{std::string("erf of ") + DTName(t) + " is not supported"};
        e = (d ? "erf(" : "erff(") + x + ")";
      } else if (n == "reduce_precision") {
        // the formats of the 16-bit float types (as the reference lowers them, a cast to bf16 / f16
        // and back) and formats at least as wide as the operand's own (no change)
        const int eb = (int)op->ints.at("exponent_bits")[0], mb = (int)op->ints.at("mantissa_bits")[0];
        const int own_e = t == DT::kF64 ? 11 : t == DT::kF32 || t == DT::kBF16 ? 8 : 5;
        const int own_m = t == DT::kF64 ? 52 : t == DT::kF32 ? 23 : t == DT::kBF16 ? 7 : 10;
        if (!f) throw LowerError{std::string("reduce_precision of ") + DTName(t)};
        if (eb >= own_e && mb >= own_m) e = x;
        else if (eb == 8 && mb == 7 && t != DT::kF64) e = t == DT::kF16 ? "rhf(rbf(" + x + "))" : "rbf(" + x + ")";
        else if (eb == 5 && mb == 10 && t != DT::kF64) e = t == DT::kBF16 ? "rbf(rhf(" + x + "))" : "rhf(" + x + ")";
        else
          throw LowerError{"reduce_precision to e" + std::to_string(eb) + "m" + std::to_string(mb) + " of " + DTName(t) +
                           " is not supported (e8m7, e5m10 and formats at least as wide as the operand are)"};
      }
      else {
        static const std::map<std::string, std::pair<std::string, std::string>> fn = {
            {"exponential", {"expf", "exp"}}, {"exponential_minus_one", {"expm1f", "expm1"}},
            {"log", {"logf", "log"}}, {"log_plus_one", {"log1pf", "log1p"}}, {"tanh", {"tanhf", "tanh"}},
            {"sqrt", {"sqrtf", "sqrt"}}, {"rsqrt", {"rsqrtf", "rsqrt"}}, {"cbrt", {"cbrtf", "cbrt"}},
            {"sine", {"sinf", "sin"}}, {"cosine", {"cosf", "cos"}}, {"tan", {"tanf", "tan"}},
            {"floor", {"floorf", "floor"}}, {"ceil", {"ceilf", "ceil"}},
            {"round_nearest_even", {"frne", "rint"}}, {"round_nearest_afz", {"fafz", "round"}},
            {"logistic", {"flogistic", "flogistic"}}};
        auto it = fn.find(n);
        if (it == fn.end() || !f) throw LowerError{"unsupported elementwise op '" + n + "' for " + DTName(t)};
        e = (d ? it->second.second : it->second.first) + "(" + x + ")";
      }
      if (n == "is_finite") return Var(DT::kPred, e);
      return Round(t, Var(t, e));
    }
    if (n == "multiply" && ty.dt == DT::kF32) {
      // (0.5 h) (1 + tanh u), the tanh form of GELU, as h / (1 + e^(-2u)): the same function
      // without the cancellation in 1 + tanh(u) for u < 0, in five instructions instead of ~20
      const Value *h = nullptr, *u = nullptr;
      if (GeluTanhForm(v, &h, &u)) {
        std::string hs = Emit(h, idx), us = Emit(u, idx);
        return Var(DT::kF32, hs + " * fsig2(" + us + ")");
      }
    }
    if (kBinary.count(n)) {
      std::string a = opnd(0, idx), b = opnd(1, idx);
      DT t = ty.dt;
      bool f = DTIsFloat(t), d = t == DT::kF64;
      std::string e;
      if (n == "add") e = a + " + " + b;
      else if (n == "subtract") e = a + " - " + b;
      else if (n == "multiply") e = t == DT::kPred ? a + " && " + b : a + " * " + b;
      else if (n == "divide") e = f ? a + " / " + b : "(" + b + " == 0 ? (" + CType(t) + ")-1 : " + a + " / " + b + ")";
      else if (n == "remainder") e = f ? (d ? "fmod(" : "fmodf(") + a + ", " + b + ")" : "(" + b + " == 0 ? " + a + " : " + a + " % " + b + ")";
      else if (n == "maximum") e = f ? (d ? "dmax_n(" : "fmax_n(") + a + ", " + b + ")" : "imax(" + a + ", " + b + ")";
      else if (n == "minimum") e = f ? (d ? "dmin_n(" : "fmin_n(") + a + ", " + b + ")" : "imin(" + a + ", " + b + ")";
      else if (n == "power") e = f ? (d ? "pow(" : "powf(") + a + ", " + b + ")" : "";
      else if (n == "atan2") e = (d ? "atan2(" : "atan2f(") + a + ", " + b + ")";
      else if (n == "and") e = t == DT::kPred ? a + " && " + b : a + " & " + b;
      else if (n == "or") e = t == DT::kPred ? a + " || " + b : a + " | " + b;
      else if (n == "xor") e = t == DT::kPred ? a + " != " + b : a + " ^ " + b;
      else if (n == "shift_left" || n == "shift_right_logical" || n == "shift_right_arithmetic") {
        // a shift by at least the type's width (the amount read as unsigned) gives 0, or the sign
        // fill for the arithmetic right shift; 8- / 16-bit values sit sign-extended in registers
        if (f || t == DT::kPred) throw LowerError{"unsupported op '" + n + "' for " + DTName(t)};
        const std::string W = std::to_string(DTBits(t));
        const std::string amt = "((unsigned long long)(" + b + ") & " + WidthMask(t) + ")";
        const std::string ua = "(((unsigned long long)(" + a + ")) & " + WidthMask(t) + ")";
        if (n == "shift_left")
          e = "(" + amt + " >= " + W + " ? (" + CType(t) + ")0 : (" + CType(t) + ")(" + SType(t) + ")(" + UType(t) + ")(" + ua + " << " + amt + "))";
        else if (n == "shift_right_logical")
          e = "(" + amt + " >= " + W + " ? (" + CType(t) + ")0 : (" + CType(t) + ")(" + SType(t) + ")(" + UType(t) + ")(" + ua + " >> " + amt + "))";
        else
          e = "(" + CType(t) + ")(" + (DTIsSigned(t) ? SType(t) : MemType(t)) + ")((long long)(" + SType(t) + ")(" + UType(t) + ")" + ua +
              " >> (" + amt + " >= " + W + " ? " + std::to_string(DTBits(t) - 1) + "ULL : " + amt + "))";
        if (DTIsUnsigned(t)) e = "(" + CType(t) + ")((unsigned long long)(" + e + ") & " + WidthMask(t) + ")";
      }
      if (e.empty()) throw LowerError{"unsupported op '" + n + "' for " + DTName(t)};
      return Round(t, Var(t, e));
    }
    throw LowerError{"unsupported op '" + n + "' inside a fusion"};
  }

  // Index of a reshape operand from the index of its result (row-major linearisation).
  std::vector<std::string> Reindex(const std::vector<std::string>& idx, const std::vector<int64_t>& out,
                                   const std::vector<int64_t>& in) {
    // fast path: only unit dims inserted/removed
    std::vector<int> on, inn;
    for (size_t k = 0; k < out.size(); ++k) if (out[k] != 1) on.push_back((int)k);
    for (size_t k = 0; k < in.size(); ++k) if (in[k] != 1) inn.push_back((int)k);
    bool same = on.size() == inn.size();
    for (size_t k = 0; same && k < on.size(); ++k) same = out[on[k]] == in[inn[k]];
    std::vector<std::string> j(in.size(), "0");
    if (same) {
      for (size_t k = 0; k < inn.size(); ++k) j[inn[k]] = idx[on[k]];
      return j;
    }
    // general reshape: through the row-major linear index (32-bit arithmetic when it fits: division
    // by a constant is a multiply-high, far cheaper than the 64-bit sequence)
    int64_t total = 1;
    for (int64_t d : in) total *= d;
    const bool narrow = total < (1LL << 31);
    std::string lin = narrow ? Var(DT::kU32, "(unsigned)(" + Linear(idx, out) + ")") : Var(DT::kS64, Linear(idx, out));
    const std::string suf = narrow ? "u" : "LL";
    int64_t stride = 1;
    for (int k = (int)in.size() - 1; k >= 0; --k) {
      std::string e = "(int)((" + lin + " / " + std::to_string(stride) + suf + ") % " + std::to_string(in[k]) + suf + ")";
      if (k == 0) e = "(int)(" + lin + " / " + std::to_string(stride) + suf + ")";
      if (stride == 1 && k != 0) e = "(int)(" + lin + " % " + std::to_string(in[k]) + suf + ")";
      j[k] = Var(DT::kS32, e);
      stride *= in[k];
    }
    return j;
  }
};

// `shared_in` / `shared_out`: parameters that may point at the same memory (an output written in
// place of a donated input) and so are declared without __restrict__.
std::string KernelParams(const std::vector<int>& ins, int n_out, bool scratch, const std::set<int>& shared_in = {},
                         const std::set<int>& shared_out = {}) {
  std::string s;
  for (size_t k = 0; k < ins.size(); ++k)
    s += (k ? ", " : "") + std::string(shared_in.count((int)k) ? "const void* p" : "const void* __restrict__ p") + std::to_string(k);
  for (int k = 0; k < n_out; ++k)
    s += (s.empty() ? "" : ", ") + std::string(shared_out.count(k) ? "void* q" : "void* __restrict__ q") + std::to_string(k);
  if (scratch) s += (s.empty() ? "" : ", ") + std::string("void* __restrict__ scratch");
  return s;
}

std::string ParamCasts(const std::vector<int>& ins, const std::vector<DT>& in_dts, const std::vector<DT>& out_dts,
                       const std::set<int>& shared_in = {}, const std::set<int>& shared_out = {}) {
  std::ostringstream o;
  for (size_t k = 0; k < ins.size(); ++k)
    o << "  const " << MemType(in_dts[k]) << (shared_in.count((int)k) ? "* in" : "* __restrict__ in") << k << " = (const "
      << MemType(in_dts[k]) << "*)p" << k << ";\n";
  for (size_t k = 0; k < out_dts.size(); ++k)
    o << "  " << MemType(out_dts[k]) << (shared_out.count((int)k) ? "* out" : "* __restrict__ out") << k << " = ("
      << MemType(out_dts[k]) << "*)q" << k << ";\n";
  return o.str();
}

// Delinearises loop variable `lin` over `dims` into named indices; returns the names.
std::vector<std::string> Delinearize(std::ostringstream& o, const std::string& lin, const std::vector<int64_t>& dims,
                                     const std::string& prefix, const std::string& ind, bool wide) {
  std::vector<std::string> names(dims.size());
  std::string it = wide ? "long long" : "unsigned";
  std::string cur = prefix + "r";
  o << ind << it << " " << cur << " = (" << it << ")(" << lin << ");\n";
  for (int k = (int)dims.size() - 1; k >= 0; --k) {
    names[k] = prefix + std::to_string(k);
    if (k == 0) {
      o << ind << "int " << names[k] << " = (int)" << cur << ";\n";
    } else if (dims[k] == 1) {
      o << ind << "const int " << names[k] << " = 0;\n";
    } else {
      o << ind << "int " << names[k] << " = (int)(" << cur << " % " << dims[k] << (wide ? "LL" : "u") << "); "
        << cur << " /= " << dims[k] << (wide ? "LL" : "u") << ";\n";
    }
  }
  return names;
}

// ------------------------------------------------------------------------------------ lowering
class Lowerer {
 public:
  Lowerer(Graph& g, const CompileOptions& opt, Plan* p) : g_(g), opt_(opt), p_(p) {}

  // partition_id / replica_id become constants: one process drives one device, so the id is this
  // process's rank in the dimension the program is partitioned / replicated over, else 0 (the
  // reference binds both to its rank, src/jam/ops/collectives.mm:16-29)
  void RankConstants() {
    for (auto& up : g_.ops) {
      Op* op = up.get();
      if (op->name == "all_to_all" || op->name == "collective_broadcast" || op->name == "collective_permute") {
        // one process: every rank's data is its own (the reference binds these to their operand,
        // src/jam/ops/collectives.mm:16-29); across processes they are not lowered
        if (opt_.num_processes > 1) throw LowerError{op->name + " across processes is not supported"};
        if (op->operands.size() != 1 || op->results.size() != 1 || !(op->operands[0]->type == op->result()->type))
          throw LowerError{op->name + ": expected one operand of the result's type"};
        if (op->name == "collective_permute") {
          const auto it = op->ints.find("source_target_pairs");
          bool self = false;
          if (it != op->ints.end())
            for (size_t k = 0; k + 1 < it->second.size(); k += 2) self = self || (it->second[k] == 0 && it->second[k + 1] == 0);
          if (!self) throw LowerError{"collective_permute without a (0, 0) pair at one process (a zero result) is not supported"};
        }
        op->name = "optimization_barrier";   // an alias of its operand
        continue;
      }
      if (op->name != "partition_id" && op->name != "replica_id") continue;
      const bool split = op->name == "partition_id" ? g_.num_partitions > 1 : g_.num_replicas > 1;
      const uint64_t id = split ? (uint64_t)opt_.rank : 0;
      const Value* r = op->result();
      if (!r->type.dims.empty() || !DTIsUnsigned(r->type.dt) && !DTIsSigned(r->type.dt))
        throw LowerError{op->name + " must give an integer scalar"};
      op->name = "constant";
      op->splat = true;
      op->data.assign((const uint8_t*)&id, (const uint8_t*)&id + DTBytes(r->type.dt));
    }
  }

  void Run() {
    slot_of_.assign(g_.values.size(), -1);
    dead_.assign(g_.ops.size(), false);
    Retype();
    RankConstants();
    if (opt_.fuse_attention) MatchAttention();
    // Two passes: the first decides with recomputation walking down to arguments and heavy results;
    // the second lets a value be recomputed from what the first pass stored (a LayerNorm's x - mean
    // and (x - mean) * rstd are then rebuilt by the backward from the stored residual and row
    // statistics instead of being written and read back as f32 tensors).
    DecideMaterialization();
    if (!std::getenv("B200_NO_RECOMPUTE")) {
      const std::vector<bool> first = need_;
      recompute_stop_ = &first;
      DecideMaterialization();
      recompute_stop_ = nullptr;
    }
    DecideStoredTypes();
    BindLeaves();
    FindAliases();
    EmitSteps();
    BindOutputs();
    MergeTinyLoops();
    GroupSmallCollectives();
    PackAllReduces();
    MarkAsyncCollectives();
    ComputeLastUse();
    DecideInPlace();
    EndKernel();
    p_->cuda_prelude = kPrelude;
    p_->cuda_source = kPrelude;
    for (const auto& k : p_->kernel_sources) p_->cuda_source += k;
    p_->num_partitions = g_.num_partitions;
  }

 private:
  Graph& g_;
  const CompileOptions& opt_;
  Plan* p_;
  std::vector<int> slot_of_;
  std::vector<bool> dead_;
  std::vector<bool> need_;                 // value must be materialized
  std::vector<bool> ext_use_;              // read by a program output, a library step or attention
  std::vector<std::set<int>> cons_;        // materialized consumers of each value
  std::unordered_map<int, DT> demote_;     // value id -> narrower type its buffer holds

  // An f32 value read only by dots whose other operand is 16-bit and whose result is 16-bit is
  // rounded to that type when the dot runs (such a dot rounds its f32 operand once, an error of the
  // size of its own result's rounding); its producing kernel stores it rounded instead (half the
  // bytes, no conversion pass).  A dot with an f32 result keeps its f32 operand exact.
  void DecideStoredTypes() {
    if (std::getenv("B200_DOT_MIXED_F32")) return;
    std::unordered_set<int> outs;
    for (Value* o : g_.outputs) outs.insert(o->id);
    for (auto& opp : g_.ops) {
      const Op* op = opp.get();
      if (dead_[op->index] || op->results.size() != 1 || !IsElementwise(op) || IsAlias(op) || op->name == "constant") continue;
      const Value* r = op->result();
      if (!need_[r->id] || r->type.dt != DT::kF32 || outs.count(r->id) || attn_.count(r->id)) continue;
      bool any_attn = false;
      for (auto& kv : attn_in_) for (const Value* v : kv.second) any_attn = any_attn || v == r;
      if (any_attn) continue;
      DT narrow = DT::kF32;
      bool ok = !r->users.empty();
      // a padded row pitch lets every dot read it in place when its innermost extent is not a
      // multiple of 8 (TMA row strides are multiples of 16 bytes): allowed when each dot uses the
      // innermost dim alone as its contracting or free dim, with the operand otherwise in order
      const int rank = r->type.rank();
      bool pitch_ok = rank >= 2 && r->type.dims.back() % 8 != 0;
      for (const Op* u : r->users) {
        if (dead_[u->index]) continue;
        if (u->name != "dot_general" && u->name != "dot") { ok = false; break; }
        const Value* other = u->operands[0] == r ? u->operands[1] : u->operands[0];
        if (u->operands[0] == r && u->operands[1] == r) { ok = false; break; }
        DT t = other->type.dt;
        if (t != DT::kBF16 && t != DT::kF16) { ok = false; break; }
        if (u->results.size() != 1 || u->result()->type.dt != t) { ok = false; break; }
        if (narrow != DT::kF32 && narrow != t) { ok = false; break; }
        narrow = t;
        std::vector<int64_t> bat, fr, ct;
        DotDims(u, u->operands[0] == r ? 0 : 1, &bat, &fr, &ct);
        auto in_order = [&](std::vector<int64_t> o, const std::vector<int64_t>& y, const std::vector<int64_t>& z) {
          o.insert(o.end(), y.begin(), y.end());
          o.insert(o.end(), z.begin(), z.end());
          for (size_t k = 0; k < o.size(); ++k) if (o[k] != (int64_t)k) return false;
          return true;
        };
        const std::vector<int64_t> last{rank - 1};
        pitch_ok = pitch_ok && ((ct == last && in_order(bat, fr, ct)) || (fr == last && in_order(bat, ct, fr)));
      }
      if (ok && narrow != DT::kF32) {
        demote_[r->id] = narrow;
        if (pitch_ok) pitch_[r->id] = (r->type.dims.back() + 7) / 8 * 8;
      }
    }
    // A tensor-core dot whose result rows break the 16-byte rule (the LM head's f32 logits, 50257
    // wide) writes them with a padded pitch -- the TMA-store epilogue then applies, and the
    // generated kernels that read the result get 16-byte aligned rows -- when every reader is such a
    // kernel (elementwise / index maps other than reshape / reductions).
    for (auto& opp : g_.ops) {
      const Op* op = opp.get();
      if (dead_[op->index] || (op->name != "dot_general" && op->name != "dot") || op->results.size() != 1) continue;
      const Value* r = op->result();
      const DT dt = r->type.dt;
      if (r->type.rank() < 2 || (dt != DT::kF32 && dt != DT::kBF16 && dt != DT::kF16) || outs.count(r->id) ||
          attn_.count(r->id) || bwd_of_.count(r->id) || pitch_.count(r->id))
        continue;
      const int64_t n = r->type.dims.back(), esz = DTBytes(dt);
      if ((n * esz) % 16 == 0) continue;
      std::vector<int64_t> bat, fr, ct;
      DotDims(op, 1, &bat, &fr, &ct);
      if (fr.size() != 1 || op->operands[1]->type.dims[fr[0]] != n) continue;
      const DT at = op->operands[0]->type.dt, bt = op->operands[1]->type.dt;
      if ((at == DT::kF32 || at == DT::kF64) && (bt == DT::kF32 || bt == DT::kF64)) continue;   // SIMT path
      bool ok = !r->users.empty();
      for (const Op* u : r->users) {
        if (dead_[u->index]) continue;
        const bool gen = (IsElementwise(u) && u->name != "reshape" && u->name != "bitcast_convert" && !DataDependentIndex(u)) ||
                         (u->name == "reduce" && u->operands[0] == r && u->results.size() == 1);
        if (!gen) { ok = false; break; }
      }
      bool in_attn = false;
      for (auto& kv : attn_in_) for (const Value* v : kv.second) in_attn = in_attn || v == r;
      if (ok && !in_attn) pitch_[r->id] = (n * esz + 15) / 16 * 16 / esz;
    }
  }
  // batch / free / contracting dims of operand `side` (0 lhs, 1 rhs) of a dot
  static void DotDims(const Op* op, int side, std::vector<int64_t>* bat, std::vector<int64_t>* fr, std::vector<int64_t>* ct) {
    auto get = [&](const char* k) { auto it = op->ints.find(k); return it == op->ints.end() ? std::vector<int64_t>{} : it->second; };
    const Value* v = op->operands[side];
    *bat = get(side ? "batching_dims.rhs" : "batching_dims.lhs");
    *ct = get(side ? "contracting_dims.rhs" : "contracting_dims.lhs");
    if (op->name == "dot") *ct = {side ? 0 : v->type.rank() - 1};
    fr->clear();
    for (int k = 0; k < v->type.rank(); ++k)
      if (std::find(bat->begin(), bat->end(), k) == bat->end() && std::find(ct->begin(), ct->end(), k) == ct->end()) fr->push_back(k);
  }
  std::unordered_map<int, int64_t> pitch_;   // value id -> padded innermost row pitch (elements)
  int64_t StoredPitch(const Value* v) const {
    auto it = pitch_.find(v->id);
    return it == pitch_.end() ? 0 : it->second;
  }
  int64_t StoredBytes(const Value* v) const {
    const int64_t p = StoredPitch(v), n = v->type.numel();
    if (!p) return n * DTBytes(StoredDt(v));
    return n / v->type.dims.back() * p * DTBytes(StoredDt(v));
  }
  // element offset of linear index `i` (whose per-dim indices are `names`) in the buffer of v: with
  // a padded pitch, the outer dims' linear index times the pitch plus the innermost index
  std::string StoredIndex(const Value* v, const std::string& i, const std::vector<std::string>& names) const {
    const int64_t p = StoredPitch(v);
    if (!p) return i;
    const auto& d = v->type.dims;
    std::vector<std::string> outer(names.begin(), names.end() - 1);
    std::vector<int64_t> od(d.begin(), d.end() - 1);
    return "(" + Gen::Linear(outer, od) + " * " + std::to_string(p) + "LL + (" + names.back() + "))";
  }
  DT StoredDt(const Value* v) const {
    auto it = demote_.find(v->id);
    if (it != demote_.end()) return it->second;
    return promote_.count(v->id) ? DT::kF32 : v->type.dt;
  }
  // 16-bit values kept in f32 storage and rounded where they are read: a split-K dot's f32
  // accumulator or the attention backward's dQ accumulator needs no separate rounding pass when
  // every reader is a generated kernel
  std::unordered_set<int> promote_;
  std::unordered_set<int> slot_f32_;             // slots holding such values
  bool PromotableToF32(const Value* v) const {
    if ((v->type.dt != DT::kBF16 && v->type.dt != DT::kF16) || pitch_.count(v->id) || std::getenv("B200_NO_PROMOTE"))
      return false;
    for (const Value* o : g_.outputs) if (o == v) return false;
    if (v->users.empty()) return false;
    for (const Op* u : v->users) {
      if (dead_[u->index]) continue;
      const bool gen = (IsElementwise(u) && u->name != "reshape" && u->name != "bitcast_convert" && !DataDependentIndex(u)) ||
                       (u->name == "reduce" && u->operands[0] == v && u->results.size() == 1);
      if (!gen) return false;
    }
    for (auto& kv : attn_in_) for (const Value* x : kv.second) if (x == v) return false;
    for (const BwdMatch& m : bwd_) for (const Value* x : {m.Q, m.K, m.V, m.O, m.G}) if (x == v) return false;
    return true;
  }
  // the value to store for root v into a buffer of type `dt` (rounded when the buffer is narrower)
  static std::string StoreVal(const Value* v, DT dt, const std::string& x) {
    if (dt == v->type.dt) return x;
    return dt == DT::kBF16 ? "rbf(" + x + ")" : "rhf(" + x + ")";
  }
  std::unordered_map<int, AttentionStep> attn_;  // result value id of the 2nd dot -> matched attention
  std::unordered_map<int, std::array<const Value*, 3>> attn_in_;
  std::ostringstream src_;
  // Each finished kernel's source becomes its own unit so NVRTC can compile them in parallel.
  // Every generated kernel starts with griddepcontrol.wait: launched as a programmatic dependent of
  // the previous kernel it may be scheduled while that one drains, and waits here (before its first
  // read) until the previous grid has completed and its writes are visible.  It then lets its own
  // dependent be scheduled (launch_dependents), which waits the same way.
  void EndKernel() {
    std::string k = src_.str();
    if (!k.empty()) {
      const std::string tag = "extern \"C\" __global__";
      for (size_t at = k.find(tag); at != std::string::npos; at = k.find(tag, at + 1)) {
        const size_t open = k.find(") {\n", at);
        if (open == std::string::npos) break;
        k.insert(open + 4, "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n"
                           "  asm volatile(\"griddepcontrol.launch_dependents;\");\n");
      }
      p_->kernel_sources.push_back(k);
    }
    src_.str("");
    src_.clear();
  }
  int kcount_ = 0;

  int NewSlot(int64_t bytes) {
    p_->slots.push_back(Slot());
    p_->slots.back().bytes = std::max<int64_t>(bytes, 0);
    return (int)p_->slots.size() - 1;
  }

  const Value* Resolve(const Value* v) const {
    while (v->def && IsAlias(v->def)) {
      const Op* op = v->def;
      size_t k = 0;
      for (; k < op->results.size(); ++k) if (op->results[k] == v) break;
      v = op->operands[std::min(k, op->operands.size() - 1)];
    }
    return v;
  }

  // shard_map: an argument that reaches SPMDFullToShardShape is passed per device at shard shape
  // (the reference retypes the placeholder, src/jam/lower.mm:273-289).
  void Retype() {
    p_->arg_types.clear();
    for (Value* a : g_.args) p_->arg_types.push_back(a->type);
    for (auto& op : g_.ops) {
      if (op->name != "custom_call" || op->strs["call_target_name"] != "SPMDFullToShardShape") continue;
      const Value* src = Resolve(op->operands[0]);
      if (src->arg_index >= 0) p_->arg_types[src->arg_index] = op->result()->type;
    }
  }

  // ---------------------------------------------------------------- attention pattern
  // dot(Q,K^T) [* scale] [select(causal, ., -inf)] -> max -> exp(x - max) -> sum -> div -> [convert] -> dot(., V)
  static const Value* Through(const Value* v) {   // skip reshapes / broadcasts that only add unit dims
    while (v->def && (v->def->name == "reshape" || v->def->name == "broadcast_in_dim") &&
           v->def->operands[0]->type.numel() == v->type.numel())
      v = v->def->operands[0];
    return v;
  }
  static const Value* RowBroadcastOf(const Value* v) {  // broadcast_in_dim(x, dims=[0..r-2]) of a row vector
    if (!v->def || v->def->name != "broadcast_in_dim") return nullptr;
    const Value* x = Through(v->def->operands[0]);
    return x;
  }
  static bool IsScalarConst(const Value* v, double* out) {
    while (v->def && v->def->name == "broadcast_in_dim") v = v->def->operands[0];
    if (!v->def || v->def->name != "constant" || !v->def->splat) return false;
    *out = ConstScalar(v->def);
    return true;
  }
  bool SingleUse(const Value* v) const { return v->users.size() == 1; }

  // The forward chain ending at d2 = dot(P', V).  strict: every intermediate has the single use the
  // inference form gives it (the chain can simply disappear); otherwise intermediates may also feed
  // a backward pass, which MatchAttentionTraining accounts for.
  struct FwdChain {
    const Value *Q = nullptr, *K = nullptr, *V = nullptr, *S = nullptr, *x = nullptr, *P = nullptr, *P16 = nullptr;
    std::vector<const Op*> ops;   // the chain's ops other than d2
    bool causal = false;
    double scale = 1.0;
  };
  bool MatchFwdChain(const Op* d2, bool strict, FwdChain* fc) const {
    auto ints = [&](const Op* o, const char* k) {
      auto it = o->ints.find(k);
      return it == o->ints.end() ? std::vector<int64_t>{} : it->second;
    };
    auto single = [&](const Value* v) { return !strict || SingleUse(v); };
    if (d2->name != "dot_general" || d2->operands.size() != 2) return false;
    const std::vector<int64_t> b01 = {0, 1};
    if (ints(d2, "batching_dims.lhs") != b01 || ints(d2, "batching_dims.rhs") != b01) return false;
    if (ints(d2, "contracting_dims.lhs") != std::vector<int64_t>{3} || ints(d2, "contracting_dims.rhs") != std::vector<int64_t>{2})
      return false;
    std::vector<const Op*> chain;
    const Value* p = d2->operands[0];
    const Value* V = d2->operands[1];
    fc->P16 = p;
    if (p->def && p->def->name == "convert") {
      chain.push_back(p->def);
      if (!single(p)) return false;
      p = p->def->operands[0];
    }
    fc->P = p;
    if (!p->def || p->def->name != "divide" || !single(p)) return false;
    const Op* div = p->def;
    chain.push_back(div);
    const Value* e = div->operands[0];
    const Value* sumb = div->operands[1];
    if (!e->def || e->def->name != "exponential") return false;
    // sum = reduce_add(e, dims=[3]) seen through reshapes/broadcasts
    const Value* sum = RowBroadcastOf(sumb);
    if (!sum || !sum->def || sum->def->name != "reduce" || sum->def->reduce != ReduceKind::kAdd) return false;
    if (sum->def->operands[0] != e || ints(sum->def, "dimensions") != std::vector<int64_t>{3}) return false;
    if (strict && e->users.size() != 2) return false;
    chain.push_back(e->def);
    chain.push_back(sum->def);
    for (const Value* y = sumb; y != sum; y = y->def->operands[0]) {
      if (strict && y->users.size() != 1) return false;
      chain.push_back(y->def);
    }
    const Value* sub = e->def->operands[0];
    if (!sub->def || sub->def->name != "subtract" || !single(sub)) return false;
    chain.push_back(sub->def);
    const Value* x = sub->def->operands[0];
    const Value* maxb = sub->def->operands[1];
    const Value* mx = RowBroadcastOf(maxb);
    if (!mx || !mx->def || mx->def->name != "reduce" || mx->def->reduce != ReduceKind::kMax) return false;
    if (mx->def->operands[0] != x || ints(mx->def, "dimensions") != std::vector<int64_t>{3}) return false;
    if (strict && x->users.size() != 2) return false;
    chain.push_back(mx->def);
    for (const Value* y = maxb; y != mx; y = y->def->operands[0]) {
      if (strict && y->users.size() != 1) return false;
      chain.push_back(y->def);
    }
    fc->x = x;
    const Value* s = x;
    if (s->def && s->def->name == "select") {
      // select(broadcast(compare(iota0 GE iota1)), s, -inf)
      const Op* sel = s->def;
      double ninf;
      if (!IsScalarConst(sel->operands[2], &ninf) || !(std::isinf(ninf) && ninf < 0)) return false;
      const Value* m = Through(sel->operands[0]);
      if (m->def && m->def->name == "broadcast_in_dim") m = m->def->operands[0];
      if (!m->def || m->def->name != "compare") return false;
      const Op* cmp = m->def;
      auto iota_dim = [](const Value* v) -> int {
        while (v->def && v->def->name == "broadcast_in_dim") v = v->def->operands[0];
        return (v->def && v->def->name == "iota") ? (int)v->def->ints.at("dim")[0] : -1;
      };
      std::string dir = cmp->strs.at("comparison_direction");
      int li = iota_dim(cmp->operands[0]), ri = iota_dim(cmp->operands[1]);
      if (!((dir == "GE" && li == 0 && ri == 1) || (dir == "LE" && li == 1 && ri == 0))) return false;
      if (m->type.rank() != 2) return false;
      fc->causal = true;
      chain.push_back(sel);
      s = sel->operands[1];
      if (!single(s)) return false;
    }
    if (s->def && s->def->name == "multiply") {
      double c;
      const Op* mul = s->def;
      const Value* other = nullptr;
      if (IsScalarConst(mul->operands[1], &c)) other = mul->operands[0];
      else if (IsScalarConst(mul->operands[0], &c)) other = mul->operands[1];
      if (!other || (s != x && !single(s))) return false;
      fc->scale = c;
      chain.push_back(mul);
      s = other;
    }
    if (!s->def || s->def->name != "dot_general" || (s != x && !single(s))) return false;
    const Op* d1 = s->def;
    if (ints(d1, "batching_dims.lhs") != b01 || ints(d1, "batching_dims.rhs") != b01 ||
        ints(d1, "contracting_dims.lhs") != std::vector<int64_t>{3} || ints(d1, "contracting_dims.rhs") != std::vector<int64_t>{3})
      return false;
    const Value* Q = d1->operands[0];
    const Value* K = d1->operands[1];
    if (Q->type.dt != DT::kBF16 || K->type.dt != DT::kBF16 || V->type.dt != DT::kBF16) return false;
    if (d2->result()->type.dt != DT::kBF16) return false;
    if (!(Q->type.dims == K->type.dims && Q->type.dims == V->type.dims)) return false;
    if (s->type.dt != DT::kF32) return false;
    const int Dh = (int)Q->type.dims[3];
    if (Dh != 64 || Q->type.dims[2] % 256 != 0 || fc->scale <= 0) return false;
    chain.push_back(d1);
    fc->Q = Q;
    fc->K = K;
    fc->V = V;
    fc->S = s;
    fc->ops = chain;
    return true;
  }

  void RegisterAttention(const Op* d2, const FwdChain& fc) {
    AttentionStep a;
    a.B = (int)fc.Q->type.dims[0];
    a.H = (int)fc.Q->type.dims[1];
    a.S = (int)fc.Q->type.dims[2];
    a.D = (int)fc.Q->type.dims[3];
    a.causal = fc.causal;
    a.scale = (float)fc.scale;
    attn_[d2->result()->id] = a;
    attn_in_[d2->result()->id] = {fc.Q, fc.K, fc.V};
    for (const Op* o : fc.ops) dead_[o->index] = true;
  }

  void MatchAttention() {
    for (auto& opp : g_.ops) {
      const Op* d2 = opp.get();
      FwdChain fc;
      if (MatchFwdChain(d2, true, &fc)) RegisterAttention(d2, fc);
      else if (MatchFwdChain(d2, false, &fc) && !std::getenv("B200_NO_FLASH_BWD")) MatchAttentionTraining(d2, fc);
    }
  }

  // ---------------------------------------------------------------- attention in training
  // The forward chain's intermediates also feed its VJP.  Recognised by anchors: dV = dot(P', G)
  // contracting the query dim, dP = dot(G, V) contracting the head dim, and one value T read by
  // dQ = dot(T, K) and dK = dot(Q, T) (or dot(T, Q)).  T is accepted when it evaluates, on sample
  // rows of random scores and cotangents, to scale * mask * P * (dP - rowsum(P * dP)) -- whatever
  // elementwise / row-reduction ops compute it.  Then the forward runs as the flash forward (also
  // writing lse2) and the three dots as one flash-backward step; the S x S intermediates vanish.
  struct BwdMatch {
    int d2 = -1;                                     // forward result value id (O)
    const Value *Q = nullptr, *K = nullptr, *V = nullptr, *O = nullptr, *G = nullptr;
    const Value *dq = nullptr, *dk = nullptr, *dv = nullptr;
    bool dk_t = false;                               // dK delivered as [B, H, D, S]
    bool emitted = false;
  };
  std::vector<BwdMatch> bwd_;
  std::unordered_map<int, int> bwd_of_;              // dq / dk / dv dot result id -> bwd_ index
  std::unordered_set<int> bwd_in_;                   // values the backward step reads (G)

  // Row evaluator: the value of `v` at a full index, in double precision, for the ops a softmax VJP
  // is made of; `leaf` supplies the scores S and the cotangent dP.  Returns false for other ops.
  struct RowEval {
    std::function<bool(const Value*, const std::vector<int64_t>&, double*)> leaf;
    std::map<std::pair<int, std::vector<int64_t>>, double> memo;
    int budget = 4000000;
    bool At(const Value* v, const std::vector<int64_t>& idx, double* out) {
      if (--budget < 0) return false;
      if (leaf(v, idx, out)) return true;
      auto key = std::make_pair(v->id, idx);
      auto it = memo.find(key);
      if (it != memo.end()) { *out = it->second; return true; }
      const Op* op = v->def;
      if (!op) return false;
      const std::string& n = op->name;
      double r = 0;
      auto at = [&](int k, const std::vector<int64_t>& j, double* o) { return At(op->operands[k], j, o); };
      if (n == "constant") {
        if (!op->splat) return false;
        r = ConstScalar(op);
      } else if (n == "iota") {
        r = (double)idx[op->ints.at("dim")[0]];
      } else if (n == "broadcast_in_dim") {
        const auto& dims = op->ints.at("dims");
        const auto& in = op->operands[0]->type.dims;
        std::vector<int64_t> j(in.size());
        for (size_t k = 0; k < in.size(); ++k) j[k] = in[k] == 1 ? 0 : idx[dims[k]];
        if (!at(0, j, &r)) return false;
      } else if (n == "reshape" || IsAlias(op)) {
        const auto& od = v->type.dims;
        const auto& in = op->operands[0]->type.dims;
        int64_t lin = 0;
        for (size_t k = 0; k < od.size(); ++k) lin = lin * od[k] + idx[k];
        std::vector<int64_t> j(in.size());
        for (int k = (int)in.size() - 1; k >= 0; --k) { j[k] = in[k] ? lin % in[k] : 0; lin = in[k] ? lin / in[k] : 0; }
        if (!at(0, j, &r)) return false;
      } else if (n == "transpose") {
        const auto& perm = op->ints.at("dims");
        std::vector<int64_t> j(perm.size());
        for (size_t k = 0; k < perm.size(); ++k) j[perm[k]] = idx[k];
        if (!at(0, j, &r)) return false;
      } else if (n == "convert") {
        if (!at(0, idx, &r)) return false;
        if (v->type.dt == DT::kBF16) r = RoundBf16((float)r);
        else if (v->type.dt == DT::kF32) r = (float)r;
        else if (v->type.dt == DT::kPred) r = r != 0;
        else if (!DTIsFloat(v->type.dt)) r = std::trunc(r);
      } else if (n == "compare") {
        double a, b;
        if (!at(0, idx, &a) || !at(1, idx, &b)) return false;
        const std::string& d = op->strs.at("comparison_direction");
        r = d == "EQ" ? a == b : d == "NE" ? a != b : d == "LT" ? a < b : d == "LE" ? a <= b : d == "GT" ? a > b : a >= b;
      } else if (n == "select") {
        double c;
        const auto& pd = op->operands[0]->type.dims;
        if (!At(op->operands[0], pd.empty() ? std::vector<int64_t>{} : idx, &c)) return false;
        if (!at(c != 0 ? 1 : 2, idx, &r)) return false;
      } else if (n == "negate" || n == "exponential" || n == "log" || n == "sqrt" || n == "rsqrt" || n == "tanh") {
        double a;
        if (!at(0, idx, &a)) return false;
        r = n == "negate" ? -a : n == "exponential" ? std::exp(a) : n == "log" ? std::log(a) : n == "sqrt" ? std::sqrt(a)
            : n == "rsqrt" ? 1.0 / std::sqrt(a) : std::tanh(a);
      } else if (n == "add" || n == "subtract" || n == "multiply" || n == "divide" || n == "maximum" || n == "minimum") {
        double a, b;
        if (!at(0, idx, &a) || !at(1, idx, &b)) return false;
        r = n == "add" ? a + b : n == "subtract" ? a - b : n == "multiply" ? a * b : n == "divide" ? a / b
            : n == "maximum" ? std::max(a, b) : std::min(a, b);
      } else if (n == "reduce" && (op->reduce == ReduceKind::kAdd || op->reduce == ReduceKind::kMax) && op->results.size() == 1) {
        std::vector<int64_t> rd = op->ints.at("dimensions");
        std::sort(rd.begin(), rd.end());
        const auto& xd = op->operands[0]->type.dims;
        double init;
        if (!At(op->operands[1], {}, &init)) return false;
        std::vector<int64_t> j(xd.size());
        size_t q = 0;
        for (size_t k = 0; k < xd.size(); ++k) if (!std::binary_search(rd.begin(), rd.end(), (int64_t)k)) j[k] = idx[q++];
        int64_t total = 1;
        for (int64_t d : rd) total *= xd[d];
        r = init;
        for (int64_t t = 0; t < total; ++t) {
          int64_t rem = t;
          for (int k = (int)rd.size() - 1; k >= 0; --k) { j[rd[k]] = rem % xd[rd[k]]; rem /= xd[rd[k]]; }
          double x;
          if (!at(0, j, &x)) return false;
          r = op->reduce == ReduceKind::kAdd ? r + x : std::max(r, x);
        }
      } else {
        return false;
      }
      memo[key] = r;
      *out = r;
      return true;
    }
  };

  // deterministic pseudo-random value in [-1, 1) for an index
  static double Hash01(uint64_t a, uint64_t b, uint64_t salt) {
    uint64_t h = a * 0x9E3779B97F4A7C15ULL ^ (b + salt) * 0xC2B2AE3D27D4EB4FULL;
    h ^= h >> 29;
    h *= 0xBF58476D1CE4E5B9ULL;
    h ^= h >> 32;
    return (double)(h >> 11) / (double)(1ULL << 52) - 1.0;
  }

  // T == scale * mask * P * (dP - rowsum(P * dP)) on sample rows of random S and dP?
  bool VerifySoftmaxVjp(const Value* T, const Value* S, const Value* dP, const FwdChain& fc) const {
    const auto& d = T->type.dims;
    if (d.size() != 4 || S->type.dims != d || dP->type.dims != d) return false;
    const int64_t n = d[3];
    for (int64_t q : {n / 2 + 3, n - 1, (int64_t)1}) {
      if (q >= d[2]) continue;
      RowEval ev;
      ev.leaf = [&](const Value* v, const std::vector<int64_t>& idx, double* out) {
        if (v == S) { *out = 3.0 * Hash01(idx[2], idx[3], 1); return true; }
        if (v == dP) { *out = RoundBf16((float)Hash01(idx[2], idx[3], 2)); return true; }
        return false;
      };
      // reference row in double
      std::vector<double> x(n), pr(n), dp(n);
      double mx = -INFINITY;
      for (int64_t k = 0; k < n; ++k) {
        const bool keep = !fc.causal || k <= q;
        x[k] = keep ? fc.scale * 3.0 * Hash01(q, k, 1) : -INFINITY;
        mx = std::max(mx, x[k]);
        dp[k] = RoundBf16((float)Hash01(q, k, 2));
      }
      double sum = 0, dot = 0;
      for (int64_t k = 0; k < n; ++k) { pr[k] = std::exp(x[k] - mx); sum += pr[k]; }
      for (int64_t k = 0; k < n; ++k) { pr[k] /= sum; dot += pr[k] * dp[k]; }
      double worst = 0, big = 1e-30;
      for (int64_t k = 0; k < n; ++k) {
        const double ref = fc.scale * pr[k] * (dp[k] - dot);
        double got;
        if (!ev.At(T, {1 % d[0], 1 % d[1], q, k}, &got)) return false;
        worst = std::max(worst, std::fabs(got - ref));
        big = std::max(big, std::fabs(ref));
      }
      if (!(worst <= 2e-2 * big)) return false;
    }
    return true;
  }

  void MatchAttentionTraining(const Op* d2, const FwdChain& fc) {
    auto ints = [&](const Op* o, const char* k) {
      auto it = o->ints.find(k);
      return it == o->ints.end() ? std::vector<int64_t>{} : it->second;
    };
    auto is_dot = [&](const Op* o, const Value* l, const Value* r, int64_t lc, int64_t rc) {
      return o->name == "dot_general" && o->operands.size() == 2 && o->operands[0] == l && (!r || o->operands[1] == r) &&
             ints(o, "batching_dims.lhs") == std::vector<int64_t>{0, 1} && ints(o, "batching_dims.rhs") == std::vector<int64_t>{0, 1} &&
             ints(o, "contracting_dims.lhs") == std::vector<int64_t>{lc} && ints(o, "contracting_dims.rhs") == std::vector<int64_t>{rc} &&
             o->result()->type.dt == DT::kBF16;
    };
    // dV = dot(P', G) contracting the query dim
    const Op* dv_op = nullptr;
    for (const Op* u : fc.P16->users)
      if (u != d2 && is_dot(u, fc.P16, nullptr, 2, 2)) dv_op = u;
    if (!dv_op) return;
    const Value* G = dv_op->operands[1];
    if (G->type.dims != fc.Q->type.dims || G->type.dt != DT::kBF16) return;
    // dP = dot(G, V) contracting the head dim
    const Op* dp_op = nullptr;
    for (const Op* u : G->users)
      if (is_dot(u, G, fc.V, 3, 3)) dp_op = u;
    if (!dp_op) return;
    // dQ = dot(T, K) [3 x 2]; dK = dot(Q, T) [2 x 2] or dot(T, Q) [2 x 2]
    const Op* dq_op = nullptr;
    for (const Op* u : fc.K->users)
      if (u->name == "dot_general" && u->operands.size() == 2 && u->operands[1] == fc.K && is_dot(u, u->operands[0], fc.K, 3, 2) &&
          u->operands[0]->type.dims == fc.S->type.dims)
        dq_op = u;
    if (!dq_op) return;
    const Value* T = dq_op->operands[0];
    const Op* dk_op = nullptr;
    bool dk_t = false;
    for (const Op* u : T->users) {
      if (is_dot(u, fc.Q, T, 2, 2)) { dk_op = u; dk_t = true; }
      else if (is_dot(u, T, fc.Q, 2, 2)) { dk_op = u; dk_t = false; }
    }
    if (!dk_op || T->users.size() != 2) return;
    if (!VerifySoftmaxVjp(T, fc.S, dp_op->result(), fc)) return;
    // the ops that compute T from S, dP and the forward intermediates
    std::unordered_set<const Op*> kill(fc.ops.begin(), fc.ops.end());
    kill.insert(dp_op);
    std::vector<const Value*> stack{T};
    while (!stack.empty()) {
      const Value* v = stack.back();
      stack.pop_back();
      if (!v->def || v == fc.S || IndexOnly(v) || kill.count(v->def)) continue;
      if (v == dp_op->result()) continue;
      const std::string& n = v->def->name;
      if (!(IsElementwise(v->def) || n == "reduce") || n == "dot_general") return;
      kill.insert(v->def);
      for (const Value* o : v->def->operands) stack.push_back(o);
    }
    // nothing outside may read what is about to disappear
    std::unordered_set<const Op*> ok_users(kill.begin(), kill.end());
    for (const Op* o : {d2, dv_op, dq_op, dk_op}) ok_users.insert(o);
    for (const Op* o : kill)
      for (const Value* r : o->results)
        for (const Op* u : r->users)
          if (!dead_[u->index] && !ok_users.count(u)) return;
    // dK = dot(Q, T) comes out [B, H, D, S]; when its one reader transposes it back to [B, H, S, D]
    // the backward writes that transpose's value in its own layout and the dot disappears
    const Value* dk_val = dk_op->result();
    const Op* dk_dead = nullptr;
    if (dk_t && dk_val->users.size() == 1 && std::find(g_.outputs.begin(), g_.outputs.end(), dk_val) == g_.outputs.end()) {
      const Op* tr = dk_val->users[0];
      auto pm = tr->ints.find("dims");
      if (tr->name == "transpose" && pm != tr->ints.end() && pm->second == std::vector<int64_t>{0, 1, 3, 2}) {
        dk_val = tr->result();
        dk_t = false;
        dk_dead = dk_op;
      }
    }
    FwdChain keep = fc;
    keep.ops.clear();
    RegisterAttention(d2, keep);
    for (const Op* o : kill) dead_[o->index] = true;
    if (dk_dead) dead_[dk_dead->index] = true;
    BwdMatch m;
    m.d2 = d2->result()->id;
    m.Q = fc.Q;
    m.K = fc.K;
    m.V = fc.V;
    m.O = d2->result();
    m.G = G;
    m.dq = dq_op->result();
    m.dk = dk_val;
    m.dv = dv_op->result();
    m.dk_t = dk_t;
    const int idx = (int)bwd_.size();
    bwd_.push_back(m);
    for (const Value* r : {m.dq, m.dk, m.dv}) bwd_of_[r->id] = idx;
    bwd_in_.insert(G->id);
    lse_for_[m.d2] = -1;
  }
  std::unordered_map<int, int> lse_for_;   // forward result id -> lse2 slot (training forward)

  // ---------------------------------------------------------------- materialization
  bool IsHeavy(const Op* op) const {
    const std::string& n = op->name;
    return n == "dot_general" || n == "dot" || n == "scatter" || n == "all_reduce" || n == "all_gather" ||
           n == "reduce_scatter" || n == "reduce";
  }
  bool Cheap(const Value* v) const {
    const Op* op = v->def;
    if (!op) return true;
    if (IsAlias(op)) return Cheap(op->operands[0]);
    const std::string& n = op->name;
    if (n == "constant" || n == "iota") return true;
    if (n == "broadcast_in_dim" || n == "reshape" || n == "transpose" || n == "slice" || n == "convert" || n == "reverse")
      return true;
    if (n == "compare" || n == "select" || n == "and" || n == "or" || n == "not") {
      for (const Value* o : op->operands) if (!IndexOnly(o)) return false;
      return true;
    }
    return false;
  }
  bool IndexOnly(const Value* v) const {   // a pure function of the element index (masks)
    const Op* op = v->def;
    if (!op) return false;
    const std::string& n = op->name;
    if (n == "constant") return op->splat;
    if (n == "iota") return true;
    if (n == "broadcast_in_dim" || n == "reshape" || n == "transpose" || n == "convert" || n == "compare" ||
        n == "and" || n == "or" || n == "not" || n == "select") {
      for (const Value* o : op->operands) if (!IndexOnly(o)) return false;
      return true;
    }
    return false;
  }

  // A value read by several fusion kernels is stored once unless recomputing it in each reader is
  // cheaper: its expression (down to arguments, reductions and other non-elementwise results) has a
  // few ops and reads at most one tensor of its own size, the rest being small broadcast operands
  // (row statistics, labels, biases).  Each reader then reads that one tensor instead of the stored
  // copy: the same bytes, minus the store.  (exp(z - max) and one-hot(labels) of a cross entropy,
  // x - mean of a LayerNorm, x + bias before an activation.)
  const std::vector<bool>* recompute_stop_ = nullptr;   // need_ of the first materialisation pass
  bool Recomputable(const Value* v) const {
    if (std::getenv("B200_NO_RECOMPUTE")) return false;
    const int64_t n = v->type.numel();
    int ops = 0;
    std::unordered_set<int> big, seen;
    std::vector<const Value*> stack{v};
    while (!stack.empty()) {
      const Value* x = stack.back();
      stack.pop_back();
      if (!seen.insert(x->id).second) continue;
      const Op* op = x->def;
      // with a first materialisation pass done, values it stored are read, not recomputed
      const bool stored = x != v && recompute_stop_ && (*recompute_stop_)[x->id];
      const bool leaf = stored || !op || !IsElementwise(op) || DataDependentIndex(op) || (op->name == "constant" && !op->splat);
      if (leaf || (op->name == "constant") || op->name == "iota") {
        if (!stored && op && (op->name == "constant" || op->name == "iota")) continue;
        if (x->type.numel() * 16 > n) big.insert(x->id);
        if (big.size() > 1) return false;
        continue;
      }
      if (IsAlias(op) || op->name == "broadcast_in_dim" || op->name == "reshape" || op->name == "convert") {
        // free in the generated code
      } else if (++ops > 12) {
        return false;
      }
      for (const Value* o : op->operands) stack.push_back(o);
    }
    return true;
  }

  void DecideMaterialization() {
    size_t nv = g_.values.size();
    need_.assign(nv, false);
    ext_use_.assign(nv, false);
    // materialized consumers of each value (reached through unmaterialized chains)
    cons_.assign(nv, {});
    auto& cons = cons_;
    for (Value* o : g_.outputs) need_[o->id] = ext_use_[o->id] = true;
    for (auto& kv : attn_in_) for (const Value* v : kv.second) need_[v->id] = ext_use_[v->id] = true;
    for (const BwdMatch& m : bwd_)
      for (const Value* v : {m.Q, m.K, m.V, m.O, m.G}) need_[v->id] = ext_use_[v->id] = true;
    for (int i = (int)g_.ops.size() - 1; i >= 0; --i) {
      Op* op = g_.ops[i].get();
      if (dead_[i]) continue;
      for (Value* r : op->results) {
        std::set<int> c;
        for (Op* u : r->users) {
          if (dead_[u->index]) continue;
          if (u->results.size() == 1 && bwd_of_.count(u->result()->id)) continue;   // run by the attention backward
          if (IsHeavy(u) && u->name != "reduce") { need_[r->id] = ext_use_[r->id] = true; continue; }
          if (u->name == "reduce") {
            if (u->operands[0] == r) c.insert(u->result()->id);
            continue;                       // the init value is folded into the reduction kernel

          }
          if (IsAlias(u)) {
            // an alias of r: consumers of the alias are consumers of r
            for (Value* ur : u->results) {
              if (need_[ur->id]) c.insert(ur->id);
              else c.insert(cons[ur->id].begin(), cons[ur->id].end());
            }
            continue;
          }
          Value* ur = u->result();
          if (need_[ur->id]) c.insert(ur->id);
          else c.insert(cons[ur->id].begin(), cons[ur->id].end());
        }
        if (attn_.count(r->id) || bwd_of_.count(r->id)) need_[r->id] = true;
        cons[r->id] = c;
        if (IsHeavy(op)) need_[r->id] = true;
        if (!op->results.empty() && op->name == "constant" && !op->splat) need_[r->id] = true;
        if (!need_[r->id] && IsElementwise(op) && c.size() >= 2 && !Cheap(r) && !Recomputable(r)) need_[r->id] = true;
        if (IsAlias(op) && need_[r->id]) {
          // the alias source carries the buffer
          need_[op->operands[0]->id] = true;
        }
      }
    }
    for (Value* a : g_.args) need_[a->id] = true;
  }

  // ---------------------------------------------------------------- slots for args / constants
  void BindLeaves() {
    p_->arg_slots.clear();
    for (size_t k = 0; k < g_.args.size(); ++k) {
      int s = NewSlot(p_->arg_types[k].bytes());
      p_->slots[s].arg_index = (int)k;
      slot_of_[g_.args[k]->id] = s;
      p_->arg_slots.push_back(s);
    }
  }

  // ---------------------------------------------------------------- buffer donation
  // `tf.aliasing_output = k` on argument i (jax.jit's donate_argnums) lets result k live in argument
  // i's buffer.  alias_arg_slot_ maps the value result k is computed as to argument i's slot, so the
  // loop kernel that writes it can be generated for running in place.
  std::unordered_map<int, int> alias_arg_slot_;
  void FindAliases() {
    const size_t n = g_.args.size();
    if (g_.arg_alias_output.size() != n) return;
    std::set<int> seen;
    for (size_t i = 0; i < n; ++i) {
      const int k = g_.arg_alias_output[i];
      if (k < 0) continue;
      if (k >= (int)g_.outputs.size())
        throw LowerError{"argument " + std::to_string(i) + ": tf.aliasing_output = " + std::to_string(k) + ", but @main has " +
                         std::to_string(g_.outputs.size()) + " results"};
      if (!seen.insert(k).second) throw LowerError{"result " + std::to_string(k) + " is the tf.aliasing_output of two arguments"};
      const TensorType& at = p_->arg_types[i];
      const TensorType& rt = g_.outputs[k]->type;
      if (at.dt != rt.dt || at.dims != rt.dims)
        throw LowerError{"argument " + std::to_string(i) + " (" + at.str() + ") cannot alias result " + std::to_string(k) +
                         " (" + rt.str() + ")"};
      const Value* v = Resolve(g_.outputs[k]);
      if (v->arg_index < 0) alias_arg_slot_[v->id] = p_->arg_slots[i];
    }
  }
  // Which aliased results can be written in place: the one step that writes the result's slot is the
  // output copy of the argument itself, or a loop kernel that reads the argument only at the element
  // it writes, and no later step reads the argument.  Other aliased results get fresh buffers (the
  // donated argument's buffer is then released after the execution).
  void DecideInPlace() {
    const size_t n = p_->arg_slots.size();
    p_->arg_alias.assign(n, -1);
    p_->arg_donor.assign(n, false);
    p_->out_inplace_arg.assign(p_->out_slots.size(), -1);
    if (g_.arg_alias_output.size() != n) return;
    for (size_t i = 0; i < n; ++i) {
      p_->arg_alias[i] = g_.arg_alias_output[i];
      p_->arg_donor[i] = g_.arg_donor[i];
      const int k = g_.arg_alias_output[i];
      if (k < 0) continue;
      const int sa = p_->arg_slots[i], so = p_->out_slots[k];
      int writer = -1, writers = 0;
      for (int j = 0; j < (int)p_->steps.size(); ++j) {
        std::set<int> r, w;
        StepRW(p_->steps[j], &r, &w);
        if (w.count(so)) writer = j, ++writers;
      }
      if (writers != 1) continue;
      const Step& st = p_->steps[writer];
      bool ok = false;
      if (st.kind == StepKind::kCopy) {
        ok = st.copy.src == sa;                // the result is the argument itself
      } else if (st.kind == StepKind::kFusion && st.launches.size() == 1 && p_->slots[sa].last_use <= writer) {
        const Launch& L = st.launches[0];
        const bool pair = std::find(L.inplace.begin(), L.inplace.end(), std::make_pair(sa, so)) != L.inplace.end();
        // in a merged launch the argument must be read by the writing kernel alone
        ok = pair && std::count(L.in_slots.begin(), L.in_slots.end(), sa) <= 1;
      }
      if (ok) p_->out_inplace_arg[k] = (int)i;
    }
  }

  std::unordered_map<int, int64_t> slot_pitch_;   // slot -> padded row pitch (elements)
  int SlotFor(const Value* v) {
    v = Resolve(v);
    if (slot_of_[v->id] < 0) {
      slot_of_[v->id] = NewSlot(StoredBytes(v));
      if (const int64_t p = StoredPitch(v)) slot_pitch_[slot_of_[v->id]] = p;
      if (promote_.count(v->id)) slot_f32_.insert(slot_of_[v->id]);
    }
    return slot_of_[v->id];
  }

  // ---------------------------------------------------------------- step emission
  struct LoopGroup {
    std::vector<const Value*> roots;
    std::vector<int64_t> dims;
    DT dummy = DT::kF32;
  };

  void EmitSteps() {
    std::vector<const Value*> pending;   // loop roots of the open group
    std::vector<const Value*> row;       // members of the open row group
    std::vector<int64_t> row_x;          // its row space X = [rows..., L]
    std::vector<Op*> colred;             // sibling column reductions emitted as one kernel
    // Reductions of the open row group's per-row results (a loss summed over the rows) and the loop
    // roots computed from them are held back behind the group, so that later full-row members (the
    // loss gradient over the same rows) can still join it: one walk of the rows instead of two.
    // `tainted` holds the values computed from held-back results; an op that needs one closes the
    // group first.  Collectives of held-back values wait with them.
    std::vector<Op*> deferred;
    std::unordered_set<int> tainted;
    std::vector<Op*> held_colls;
    std::unordered_set<const Op*> hoisted;
    auto emit_deferred = [&]() {
      std::vector<const Value*> roots;
      auto flush_roots = [&]() {
        if (!roots.empty()) EmitLoopGroup(roots);
        roots.clear();
      };
      for (Op* d : deferred) {
        if (d->name == "reduce") {
          flush_roots();
          if (d->results.size() == 2) EmitArgReduce(d);
          else EmitReduce(d);
        } else {
          const Value* r = d->result();
          if (!roots.empty() && roots[0]->type.dims != r->type.dims) flush_roots();
          roots.push_back(r);
        }
      }
      flush_roots();
      deferred.clear();
      tainted.clear();
      for (Op* c : held_colls) EmitCollective(c);
      held_colls.clear();
    };
    auto flush = [&]() {
      // queued column reductions precede every open row / loop group in program order
      if (!colred.empty()) EmitColumnReduceGroup(colred);
      colred.clear();
      if (!row.empty()) TryRow(row, row_x, false);
      row.clear();
      if (!pending.empty()) EmitLoopGroup(pending);
      pending.clear();
      emit_deferred();
    };
    auto reads_tainted = [&](const Op* op) {
      if (tainted.empty()) return false;
      for (const Value* o : op->operands)
        if (tainted.count(o->id) || tainted.count(Resolve(o)->id)) return true;
      return false;
    };
    const bool defer_ok = !std::getenv("B200_NO_DEFER");
    // true if r joined the open row group
    auto join_row = [&](const Value* r) {
      if (row.empty()) return false;
      if (r->type.dims != row_x && !RowShaped(r->type.dims, row_x)) return false;
      std::vector<const Value*> cand = row;
      cand.push_back(r);
      if (!TryRow(cand, row_x, true)) return false;
      row = cand;
      return true;
    };
    // Collectives are issued as soon as their operand exists (the reference hoists them too,
    // src/jam/lower.mm:438-458): a gradient's all_reduce then overlaps the rest of the backward pass.
    std::vector<std::pair<int, Op*>> hoist;   // (index of the operand's producer, collective)
    if (opt_.num_processes > 1 && !std::getenv("B200_NO_HOIST")) {
      for (auto& opp : g_.ops) {
        Op* op = opp.get();
        if (dead_[op->index] || !(op->name == "all_reduce" || op->name == "all_gather" || op->name == "reduce_scatter")) continue;
        if (op->operands.size() != 1) continue;
        const Value* x = Resolve(op->operands[0]);
        hoist.push_back({x->def ? x->def->index : -1, op});
      }
    }
    size_t next_hoist = 0;
    std::sort(hoist.begin(), hoist.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
    for (auto& opp : g_.ops) {
      Op* op = opp.get();
      while (next_hoist < hoist.size() && hoist[next_hoist].first < op->index) {
        Op* c = hoist[next_hoist++].second;
        if (c->index <= op->index || hoisted.count(c)) continue;
        hoisted.insert(c);
        if (reads_tainted(c)) { held_colls.push_back(c); continue; }
        flush();
        EmitCollective(c);
      }
      if (dead_[op->index] || hoisted.count(op)) continue;
      const std::string& n = op->name;
      if (reads_tainted(op)) {
        // values computed inline carry the taint; a held-back loop root joins the held-back ops;
        // anything else waits until the held-back ops are emitted
        if (IsElementwise(op) && !IsAlias(op) && op->results.size() == 1 && n != "gather") {
          Value* r = op->result();
          if (!need_[r->id]) { tainted.insert(r->id); continue; }
          if (!row.empty() && !deferred.empty()) { deferred.push_back(op); tainted.insert(r->id); continue; }
        }
        flush();
      }
      if (IsAlias(op)) {
        for (size_t k = 0; k < op->results.size(); ++k) {
          const Value* src = Resolve(op->results[k]);
          if (slot_of_[src->id] >= 0) slot_of_[op->results[k]->id] = slot_of_[src->id];
        }
        continue;
      }
      Value* r = op->result();
      if (attn_.count(r->id)) { flush(); EmitAttention(op); continue; }
      if (n == "constant") {
        if (!op->splat || need_[r->id]) {
          int s = NewSlot(r->type.bytes());
          p_->consts.push_back(ConstBlob());
          auto& blob = p_->consts.back().bytes;
          if (op->splat) {
            for (int64_t e = 0; e < r->type.numel(); ++e) blob.insert(blob.end(), op->data.begin(), op->data.end());
          } else {
            blob = op->data;
          }
          p_->slots[s].const_index = (int)p_->consts.size() - 1;
          slot_of_[r->id] = s;
        }
        continue;
      }
      if (bwd_of_.count(r->id)) {
        BwdMatch& m = bwd_[bwd_of_.at(r->id)];
        if (!m.emitted) { flush(); EmitAttentionBwd(m); m.emitted = true; }
        continue;
      }
      if (n == "dot_general" || n == "dot") { flush(); EmitDot(op); continue; }
      if (n == "reduce") {
        if (RowReducible(op)) {
          const auto& X = op->operands[0]->type.dims;
          if (!row.empty() && row_x == X && join_row(r)) continue;
          // the loop roots just before it (e.g. masked scores) join when they have its shape
          if (row.empty() && !pending.empty() && pending[0]->type.dims == X) {
            std::vector<const Value*> cand = pending;
            cand.push_back(r);
            if (TryRow(cand, X, true)) {
              pending.clear();
              row = cand;
              row_x = X;
              continue;
            }
          }
          flush();
          row = {r};
          row_x = X;
          continue;
        }
        // a reduction of the open group's per-row results waits behind the group (see `deferred`)
        if (defer_ok && !row.empty() && op->results.size() == 1 && RowShaped(op->operands[0]->type.dims, row_x) &&
            op->operands[0]->type.dims != row_x) {
          deferred.push_back(op);
          tainted.insert(r->id);
          continue;
        }
        if (op->results.size() == 1 && VecColumnReduce(op)) {
          // reductions of one shape over the same dims, none reading another's result, share a
          // kernel (and the reads of their common operands: dbeta and dgamma both read dy)
          if (!colred.empty() && SameColumnReduce(colred[0], op) && !ReadsAny(op->operands[0], colred) && row.empty() &&
              pending.empty()) {
            colred.push_back(op);
            continue;
          }
          flush();
          colred.push_back(op);
          continue;
        }
        flush();
        if (op->results.size() == 2) EmitArgReduce(op);
        else EmitReduce(op);
        continue;
      }
      if (n == "scatter") { flush(); EmitScatter(op); continue; }
      if (n == "all_reduce" || n == "all_gather" || n == "reduce_scatter") { flush(); EmitCollective(op); continue; }
      if (n == "custom_call") throw LowerError{"unsupported custom_call @" + op->strs["call_target_name"]};
      if (!IsElementwise(op)) throw LowerError{"unsupported op '" + n + "'"};
      if (n == "gather") CheckGather(op);
      if (!need_[r->id]) continue;
      if (n == "reshape" && slot_of_[Resolve(op->operands[0])->id] >= 0 && need_[op->operands[0]->id]) {
        slot_of_[r->id] = slot_of_[Resolve(op->operands[0])->id];   // contiguous reshape: same buffer
        continue;
      }
      if (!row.empty()) {
        if (join_row(r)) continue;
        flush();
      }
      // a value computed from the open column reductions' results alone (a gradient rounded to bf16
      // for its all_reduce) waits behind them, so a later sibling reduction still joins their kernel
      if (defer_ok && !colred.empty() && pending.empty() && FromColumnReductions(op, colred, tainted)) {
        deferred.push_back(op);
        tainted.insert(r->id);
        continue;
      }
      if (!pending.empty() && (pending[0]->type.dims != r->type.dims)) flush();
      pending.push_back(r);
    }
    flush();
  }

  // True if every operand of `op` is the result of one of `group`'s reductions or a value already
  // held back behind them.
  bool FromColumnReductions(const Op* op, const std::vector<Op*>& group, const std::unordered_set<int>& held) const {
    if (op->operands.empty()) return false;
    for (const Value* o : op->operands) {
      if (held.count(o->id) || held.count(Resolve(o)->id)) continue;
      const Op* d = Resolve(o)->def;
      if (!d || std::find(group.begin(), group.end(), d) == group.end()) return false;
    }
    return true;
  }

  void CheckGather(const Op* op) {
    // supported: row take — operand rank >= 1, collapsed_slice_dims=[0], start_index_map=[0],
    // index_vector_dim = last index dim of size 1, slice_sizes = [1, full rest]
    auto get = [&](const char* k) { auto it = op->ints.find(k); return it == op->ints.end() ? std::vector<int64_t>{} : it->second; };
    const Value* t = op->operands[0];
    const Value* ids = op->operands[1];
    bool ok = get("collapsed_slice_dims") == std::vector<int64_t>{0} && get("start_index_map") == std::vector<int64_t>{0};
    auto ivd = get("index_vector_dim");
    ok = ok && ivd.size() == 1 && ivd[0] == ids->type.rank() - 1 && ids->type.dims.back() == 1;
    auto ss = get("slice_sizes");
    ok = ok && (int)ss.size() == t->type.rank() && ss[0] == 1;
    for (int k = 1; ok && k < t->type.rank(); ++k) ok = ss[k] == t->type.dims[k];
    auto od = get("offset_dims");
    ok = ok && (int)od.size() == t->type.rank() - 1;
    for (size_t k = 0; ok && k < od.size(); ++k) ok = od[k] == (int64_t)(ids->type.rank() - 1 + k);
    if (!ok) throw LowerError{"unsupported gather form (only row take along dim 0 is supported)"};
  }

  std::string KName() { return "k" + std::to_string(kcount_++); }

  static std::vector<DT> SlotDts(const std::vector<int>& slots, const std::unordered_map<int, DT>& dt_of) {
    std::vector<DT> out;
    for (int s : slots) out.push_back(dt_of.at(s));
    return out;
  }

  // A group of loop roots with one shape -> one kernel with several outputs.  Wide rows (inner extent
  // >= 512, enough rows to fill the GPU) run as a row kernel: the row's index math and its row-shaped
  // operands (statistics, labels) are computed once per row instead of once per element.
  void EmitLoopGroup(const std::vector<const Value*>& roots) {
    const auto& X = roots[0]->type.dims;
    if (X.size() >= 2 && X.back() >= 512 && !std::getenv("B200_NO_ROWLOOP")) {
      int64_t rows = 1;
      for (size_t k = 0; k + 1 < X.size(); ++k) rows *= X[k];
      const bool enough = X.back() > 8192 ? rows >= 148 * 4 : rows >= 148 * 32;
      if (enough && TryRow(roots, X, true)) {
        TryRow(roots, X, false);
        return;
      }
    }
    // greedily split where a later root reads an earlier one at a non-identity index
    size_t start = 0;
    while (start < roots.size()) {
      size_t end = start + 1;
      while (end < roots.size() && TryLoop(std::vector<const Value*>(roots.begin() + start, roots.begin() + end + 1), true)) ++end;
      TryLoop(std::vector<const Value*>(roots.begin() + start, roots.begin() + end), false);
      start = end;
    }
  }

  bool TryLoop(const std::vector<const Value*>& roots, bool dry) {
    const auto& dims = roots[0]->type.dims;
    int64_t n = roots[0]->type.numel();
    bool wide = n >= (1LL << 31);
    std::vector<int> out_slots;
    std::vector<DT> out_dts;
    std::vector<int> saved(slot_of_);
    size_t saved_slots = p_->slots.size();
    for (const Value* r : roots) {
      out_slots.push_back(SlotFor(r));
      out_dts.push_back(StoredDt(r));
    }
    Gen gen;
    gen.slot_of = &slot_of_;
    gen.slot_pitch = &slot_pitch_;
    gen.slot_f32 = &slot_f32_;
    gen.group_dims = dims;
    std::ostringstream pre;
    std::string ind = "    ";
    // vector mode: four consecutive elements per call (innermost extent a multiple of 4)
    const bool vec = !dims.empty() && dims.back() % 4 == 0 && n % 4 == 0 && !std::getenv("B200_NO_VEC");
    std::vector<std::string> regs;                     // scalar mode: one register per root
    std::vector<std::vector<std::string>> lregs;       // vector mode: four registers per root
    if (!vec) {
      gen.identity = Delinearize(pre, "i", dims, "i", ind, wide);
      gen.body << pre.str();
      for (size_t k = 0; k < roots.size(); ++k) {
        // a root is computed from its defining op (not loaded from its own slot)
        int s = slot_of_[roots[k]->id];
        slot_of_[roots[k]->id] = -1;
        std::string v = gen.Emit(roots[k], gen.identity);
        slot_of_[roots[k]->id] = s;
        gen.group_regs[s] = v;
        regs.push_back(v);
      }
    } else {
      std::vector<std::string> names = Delinearize(pre, "i", dims, "i", ind, wide);
      const std::string inner = names.back();
      pre << ind << "const int " << inner << "_0 = " << inner << ", " << inner << "_1 = " << inner << " + 1, " << inner
          << "_2 = " << inner << " + 2, " << inner << "_3 = " << inner << " + 3;\n";
      gen.body << pre.str();
      gen.vec = true;
      gen.vinner = inner;
      for (int l = 0; l < 4; ++l) {
        std::vector<std::string> id = names;
        id.back() = inner + "_" + std::to_string(l);
        gen.lane_identity.push_back(id);
      }
      gen.identity = gen.lane_identity[0];
      for (size_t k = 0; k < roots.size(); ++k) {
        int s = slot_of_[roots[k]->id];
        slot_of_[roots[k]->id] = -1;
        std::vector<std::string> rl;
        for (int l = 0; l < 4; ++l) rl.push_back(gen.Emit(roots[k], gen.lane_identity[l]));
        slot_of_[roots[k]->id] = s;
        gen.group_regs[s] = rl[0];
        gen.lane_group_regs[s] = rl;
        lregs.push_back(rl);
      }
    }
    if (dry) {
      bool ok = !gen.conflict;
      slot_of_ = saved;
      p_->slots.resize(saved_slots);
      return ok;
    }
    if (gen.conflict) throw LowerError{"internal: fusion conflict"};
    std::vector<DT> in_dts;
    for (int s : gen.in_slots) in_dts.push_back(SlotDt(s));
    // results that a donated argument's buffer may hold (tf.aliasing_output): written in place when
    // this kernel reads the argument only at the element it writes
    std::vector<std::pair<int, int>> inplace;
    std::set<int> shared_in, shared_out;
    for (size_t k = 0; k < roots.size(); ++k) {
      auto al = alias_arg_slot_.find(roots[k]->id);
      if (al == alias_arg_slot_.end()) continue;
      const int sa = al->second;
      if (p_->slots[sa].bytes != p_->slots[out_slots[k]].bytes || slot_pitch_.count(out_slots[k])) continue;
      auto pi = gen.param_of.find(sa);
      if (pi != gen.param_of.end()) {
        if (gen.nonident.count(sa)) continue;
        shared_in.insert(pi->second);
      }
      shared_out.insert((int)k);
      inplace.push_back({sa, out_slots[k]});
    }
    std::string fn = KName();
    // The per-element body is an inlined device function; the grid-stride loop calls it for four
    // independent elements per iteration so each thread keeps four loads in flight (one 4-byte load
    // per thread cannot cover HBM latency: Little's law caps that near 1.5 TB/s on 148 SMs).
    std::string args_decl, args_use;
    for (size_t k = 0; k < gen.in_slots.size(); ++k) {
      args_decl += ", const " + MemType(in_dts[k]) + (shared_in.count((int)k) ? "* in" : "* __restrict__ in") + std::to_string(k);
      args_use += ", in" + std::to_string(k);
    }
    for (size_t k = 0; k < out_dts.size(); ++k) {
      args_decl += ", " + MemType(out_dts[k]) + (shared_out.count((int)k) ? "* out" : "* __restrict__ out") + std::to_string(k);
      args_use += ", out" + std::to_string(k);
    }
    // In vector mode the element function's argument is the vector index t (elements 4t .. 4t+3).
    const int64_t trip = vec ? n / 4 : n;
    src_ << "static __device__ __forceinline__ void " << fn << "_elem(long long " << (vec ? "t" : "i") << args_decl << ") {\n";
    if (vec) src_ << "    const long long i = t * 4;\n";
    src_ << gen.body.str();
    for (size_t k = 0; k < roots.size(); ++k) {
      if (!vec) {
        src_ << "    out" << k << "[" << StoredIndex(roots[k], "i", vec ? gen.lane_identity[0] : gen.identity) << "] = " << StoreExpr(out_dts[k], StoreVal(roots[k], out_dts[k], regs[k])) << ";\n";
        continue;
      }
      std::vector<std::string> r4 = lregs[k];
      for (auto& x : r4) x = StoreVal(roots[k], out_dts[k], x);
      if (out_dts[k] == DT::kF32) {
        src_ << "    *(float4*)(out" << k << " + " << StoredIndex(roots[k], "i", vec ? gen.lane_identity[0] : gen.identity) << ") = make_float4(" << r4[0] << ", " << r4[1] << ", " << r4[2] << ", " << r4[3] << ");\n";
      } else if (out_dts[k] == DT::kBF16 || out_dts[k] == DT::kF16) {
        src_ << "    *(uint2*)(out" << k << " + " << StoredIndex(roots[k], "i", vec ? gen.lane_identity[0] : gen.identity) << ") = make_uint2(" << Pack16(out_dts[k], r4[0], r4[1]) << ", "
             << Pack16(out_dts[k], r4[2], r4[3]) << ");\n";
      } else {
        for (int l = 0; l < 4; ++l) src_ << "    out" << k << "[" << StoredIndex(roots[k], "i", vec ? gen.lane_identity[0] : gen.identity) << " + " << l << "] = " << StoreExpr(out_dts[k], r4[l]) << ";\n";
      }
    }
    src_ << "}\n";
    src_ << "extern \"C\" __global__ void __launch_bounds__(256, 4) " << fn << "("
         << KernelParams(gen.in_slots, (int)out_slots.size(), false, shared_in, shared_out) << ") {\n"
         << ParamCasts(gen.in_slots, in_dts, out_dts, shared_in, shared_out)
         << "  const long long st = (long long)gridDim.x * 256;\n"
         << "  long long i = (long long)blockIdx.x * 256 + threadIdx.x;\n"
         << "  for (; i + 3 * st < " << trip << "LL; i += 4 * st) {\n"
         << "    " << fn << "_elem(i" << args_use << ");\n"
         << "    " << fn << "_elem(i + st" << args_use << ");\n"
         << "    " << fn << "_elem(i + 2 * st" << args_use << ");\n"
         << "    " << fn << "_elem(i + 3 * st" << args_use << ");\n"
         << "  }\n"
         << "  for (; i < " << trip << "LL; i += st) " << fn << "_elem(i" << args_use << ");\n"
         << "}\n";
    EndKernel();
    Launch L;
    L.fn = fn;
    L.in_slots = gen.in_slots;
    L.out_slots = out_slots;
    L.block = 256;
    L.grid_x = std::max<int64_t>(1, (trip + 255) / 256);
    L.grid_stride = true;
    L.inplace = inplace;
    Step st;
    st.kind = StepKind::kFusion;
    st.launches.push_back(L);
    st.label = "loop" + std::string(" ") + roots[0]->type.str() + " x" + std::to_string(roots.size());
    p_->steps.push_back(st);
    for (size_t k = 0; k < roots.size(); ++k) RecordDt(out_slots[k], out_dts[k]);
    return true;
  }

  std::unordered_map<int, DT> slot_dt_;
  void RecordDt(int s, DT t) { slot_dt_[s] = t; }
  DT SlotDt(int s) {
    auto it = slot_dt_.find(s);
    if (it != slot_dt_.end()) return it->second;
    // find a value bound to this slot
    for (auto& v : g_.values)
      if (slot_of_[v->id] == s) return v->type.dt;
    throw LowerError{"internal: slot without dtype"};
  }

  // ---------------------------------------------------------------- row groups
  // A reduction over the trailing axis of X = [rows..., L] opens a row group.  Later materialized
  // values of shape X ("full" members) or of the row shape ("row scalars"), and further trailing
  // reductions over the same X, join it while every read of a member stays inside its own row.  The
  // group is one kernel: a warp (a block, for long rows) owns a row and walks it once per member in
  // program order.  Reduction results and row scalars live in registers; full members are
  // recomputed by the members that read them and stored only when something outside the group reads
  // them.  Re-walks of a row hit L1/L2, so DRAM sees each input once (LayerNorm, softmax and
  // logsumexp each become one kernel).
  bool RowReducible(const Op* op) const {
    if (op->results.size() != 1 || op->reduce == ReduceKind::kNone || std::getenv("B200_NO_ROWFUSE")) return false;
    const auto& xd = op->operands[0]->type.dims;
    const auto& rd = op->ints.at("dimensions");
    if (xd.size() < 2 || rd.size() != 1 || rd[0] != (int64_t)xd.size() - 1) return false;
    DT odt = op->result()->type.dt;
    if (!(DTIsFloat(odt) || odt == DT::kS32 || odt == DT::kS64)) return false;
    int64_t L = xd.back(), rows = op->result()->type.numel();
    return L >= 32 && L < (1LL << 30) && (rows >= 148 * 4 || L < 8192);
  }
  // dims has the row shape of X = [rows..., L] up to unit dims
  static bool RowShaped(const std::vector<int64_t>& dims, const std::vector<int64_t>& X) {
    std::vector<int64_t> a, b;
    for (int64_t d : dims) if (d != 1) a.push_back(d);
    for (size_t k = 0; k + 1 < X.size(); ++k) if (X[k] != 1) b.push_back(X[k]);
    return a == b;
  }
  static std::string Combine(ReduceKind kind, DT acc_dt, const std::string& a, const std::string& b) {
    bool f = DTIsFloat(acc_dt), d = acc_dt == DT::kF64;
    switch (kind) {
      case ReduceKind::kAdd: return a + " + " + b;
      case ReduceKind::kMul: return a + " * " + b;
      case ReduceKind::kMax: return f ? (d ? "dmax_n(" : "fmax_n(") + a + ", " + b + ")" : "imax(" + a + ", " + b + ")";
      case ReduceKind::kMin: return f ? (d ? "dmin_n(" : "fmin_n(") + a + ", " + b + ")" : "imin(" + a + ", " + b + ")";
      case ReduceKind::kAnd: return acc_dt == DT::kPred ? a + " && " + b : a + " & " + b;
      case ReduceKind::kOr: return acc_dt == DT::kPred ? a + " || " + b : a + " | " + b;
      default: return a;
    }
  }
  static DT AccDt(DT odt) { return odt == DT::kF64 ? DT::kF64 : DTIsFloat(odt) ? DT::kF32 : odt; }
  // register value of a reduction result held in the accumulator type (rounded like a stored value)
  static std::string FromAcc(DT odt, const std::string& e) {
    if (odt == DT::kBF16) return "rbf(" + e + ")";
    if (odt == DT::kF16) return "rhf(" + e + ")";
    return "(" + CType(odt) + ")(" + e + ")";
  }
  std::string InitExpr(const Value* init, DT acc_dt) {
    Gen ig;
    ig.slot_of = &slot_of_;
    ig.tmp = 1000000;
    std::string iv = ig.Emit(init, {});
    if (!ig.in_slots.empty()) throw LowerError{"reduce init must be a constant"};
    if (!ig.body.str().empty()) throw LowerError{"reduce init must be a splat constant"};
    return "(" + CType(acc_dt) + ")(" + iv + ")";
  }

  // rmax = max(A) over the row (identity init) and rsum = sum(exp(A - rmax)) (identity init), both
  // f32, where the subtracted value reads rmax at the current row: one online walk computes both.
  bool OnlinePair(const Value* rmax, const Value* rsum, const Gen& g) const {
    const Op* a = rmax->def;
    const Op* b = rsum->def;
    if (!a || !b || a->name != "reduce" || b->name != "reduce" || a->reduce != ReduceKind::kMax || b->reduce != ReduceKind::kAdd)
      return false;
    if (rmax->type.dt != DT::kF32 || rsum->type.dt != DT::kF32 || a->operands[0]->type.dt != DT::kF32) return false;
    double ia = 0, ib = 1;
    if (!IsScalarConst(a->operands[1], &ia) || !IsScalarConst(b->operands[1], &ib) || !(std::isinf(ia) && ia < 0) || ib != 0)
      return false;
    const Value* e = b->operands[0];
    if (!e->def || e->def->name != "exponential") return false;
    const Value* d = e->def->operands[0];
    if (!d->def || d->def->name != "subtract" || d->def->operands[0] != a->operands[0]) return false;
    // the subtrahend must be rmax of this row: emit it with rmax as a marked register
    Gen probe;
    probe.slot_of = &slot_of_;
    probe.row_ident = g.row_ident;
    probe.row_dims = g.row_dims;
    probe.fixed[rmax->id] = "RMAX";
    std::vector<std::string> id = g.row_ident;
    id.push_back("j");
    std::string r = probe.Emit(d->def->operands[1], id);
    return !probe.conflict && r == "RMAX" && probe.in_slots.empty();
  }

  // reduce-add over the row of select(iota_j == label, x, 0) (either operand order of the compare,
  // label a row-shaped integer): the cross-entropy's picked logit
  bool OneHotPick(const Op* op, const std::vector<int64_t>& X, const Value** x, const Value** label) const {
    if (op->reduce != ReduceKind::kAdd || op->operands.size() != 2 || std::getenv("B200_NO_PICK")) return false;
    double init = 1;
    if (!IsScalarConst(op->operands[1], &init) || init != 0) return false;
    const Value* sel = op->operands[0];
    if (!sel->def || sel->def->name != "select" || sel->type.dims != X) return false;
    double z = 1;
    if (!IsScalarConst(sel->def->operands[2], &z) || z != 0) return false;
    const Value* c = sel->def->operands[0];
    if (!c->def || c->def->name != "compare") return false;
    auto dir = c->def->strs.find("comparison_direction");
    if (dir == c->def->strs.end() || dir->second != "EQ") return false;
    const int last = (int)X.size() - 1;
    auto is_iota_last = [&](const Value* v) {
      return v->def && v->def->name == "iota" && v->type.dims == X && v->def->ints.at("dim")[0] == last;
    };
    auto row_label = [&](const Value* v) -> const Value* {
      if (!v->def || v->def->name != "broadcast_in_dim" || v->type.dims != X) return nullptr;
      const Value* s = v->def->operands[0];
      const auto& bd = v->def->ints.at("dims");
      for (int64_t d : bd) if (d == last) return nullptr;                  // constant along the row
      if (!DTIsSigned(s->type.dt) && !DTIsUnsigned(s->type.dt)) return nullptr;
      return s;
    };
    const Value* a = c->def->operands[0];
    const Value* b = c->def->operands[1];
    const Value* lab = is_iota_last(a) ? row_label(b) : is_iota_last(b) ? row_label(a) : nullptr;
    if (!lab) return false;
    *x = sel->def->operands[1];
    *label = lab;
    return true;
  }

  bool TryRow(const std::vector<const Value*>& members, const std::vector<int64_t>& X, bool dry) {
    const std::vector<int64_t> kept(X.begin(), X.end() - 1);
    const int64_t L = X.back();
    int64_t rows = 1;
    for (int64_t d : kept) rows *= d;
    const bool wide = rows * L >= (1LL << 31);
    const bool block_mode = L > 8192;
    const int T = block_mode ? 512 : 32;          // threads that share a row
    // Each thread takes four elements per step: consecutive ones with vector loads when L % 4 == 0,
    // else four T-strided ones (coalesced scalar loads) whose indices are clamped into the row and
    // whose lanes past the end (ok_l false) contribute nothing.
    const bool vec = L % 4 == 0 && !std::getenv("B200_NO_VEC");
    std::vector<int> saved(slot_of_);
    size_t saved_slots = p_->slots.size();
    std::set<int> ids;
    for (const Value* m : members) ids.insert(m->id);
    std::vector<int> out_slots, out_of(members.size(), -1);
    std::vector<DT> out_dts;
    for (size_t k = 0; k < members.size(); ++k) {
      const Value* m = members[k];
      bool ext = ext_use_[m->id];
      for (int c : cons_[m->id]) if (!ids.count(c)) ext = true;
      if (!ext) continue;
      out_of[k] = (int)out_slots.size();
      out_slots.push_back(SlotFor(m));
      out_dts.push_back(StoredDt(m));
    }
    std::vector<int> member_slot;
    for (const Value* m : members) {
      member_slot.push_back(slot_of_[m->id]);
      slot_of_[m->id] = -1;                     // members are recomputed or held in registers
    }
    Gen gen;
    gen.slot_of = &slot_of_;
    gen.slot_pitch = &slot_pitch_;
    gen.slot_f32 = &slot_f32_;
    gen.group_dims = X;
    std::ostringstream ob, body;
    gen.row_ident = Delinearize(ob, "row", kept, "a", "    ", wide);
    gen.row_dims = kept;
    std::vector<std::string> ident = gen.row_ident;
    ident.push_back("j");
    std::vector<std::vector<std::string>> lanes;
    for (int l = 0; l < 4; ++l) {
      lanes.push_back(gen.row_ident);
      lanes.back().push_back("j_" + std::to_string(l));
    }
    const std::string Ls = std::to_string(L), Ts = std::to_string(T), last = std::to_string(L - 1);
    // A short row that splits evenly over the threads is walked by a fully unrolled loop: every
    // phase then reads the same addresses, so the row's loads are issued together once and the
    // later phases reuse the registers instead of re-reading L1.
    const int64_t n_it = vec && L % (4 * T) == 0 ? L / (4 * T) : 0;
    const bool unrolled = vec && n_it > 0 && n_it <= 8;
    // A row loop without reductions over too few rows to give every warp several: the rows are cut
    // into segments (multiples of 128 elements) and the warps take (row, segment) items, which fill
    // the GPU's rounds evenly.
    bool any_reduce = false;
    for (const Value* m : members) any_reduce = any_reduce || (m->def && m->def->name == "reduce");
    int64_t nseg = 1, seg = L;
    if (!any_reduce && !block_mode && vec && !unrolled) {
      const int64_t warps = 148 * 32;
      while (nseg < 8 && rows * nseg < warps * 4 && (L + nseg) / (nseg + 1) >= 256) ++nseg;
      seg = ((L + nseg - 1) / nseg + 127) / 128 * 128;
      nseg = (L + seg - 1) / seg;
    }
    if (nseg > 1)
      ob << "    const int j_lo = sg * " << seg << ", j_hi = j_lo + " << seg << " < " << Ls << " ? j_lo + " << seg << " : " << Ls << ";\n";
    const std::string loop_head =
        unrolled
            ? "#pragma unroll\n    for (int jj = 0; jj < " + std::to_string(n_it) + "; ++jj) {\n      const int j = lt * 4 + jj * " +
                  std::to_string(4 * T) + ";\n      const int j_0 = j, j_1 = j + 1, j_2 = j + 2, j_3 = j + 3;\n"
        : vec && nseg > 1
            ? "#pragma unroll 8\n    for (int j = j_lo + lt * 4; j < j_hi; j += " + std::to_string(4 * T) + ") {\n" +
                  "      const int j_0 = j, j_1 = j + 1, j_2 = j + 2, j_3 = j + 3;\n"
        : vec ? "#pragma unroll 8\n    for (int j = lt * 4; j < " + Ls + "; j += " + std::to_string(4 * T) + ") {\n" +
                  "      const int j_0 = j, j_1 = j + 1, j_2 = j + 2, j_3 = j + 3;\n"
            : "#pragma unroll 2\n    for (int j = lt; j < " + Ls + "; j += " + std::to_string(4 * T) + ") {\n" +
                  "      const bool ok_1 = j + " + Ts + " < " + Ls + ", ok_2 = j + " + std::to_string(2 * T) + " < " + Ls +
                  ", ok_3 = j + " + std::to_string(3 * T) + " < " + Ls + ";\n" +
                  "      const int j_0 = j, j_1 = ok_1 ? j + " + Ts + " : " + last + ", j_2 = ok_2 ? j + " + std::to_string(2 * T) +
                  " : " + last + ", j_3 = ok_3 ? j + " + std::to_string(3 * T) + " : " + last + ";\n";
    // Rows of a ragged length (L % 4 != 0) start at varying alignments.  Each row is then walked in
    // two loops: four-element groups from the row's first 16-byte aligned element (hd), where the
    // reads and writes of [rows..., L] tensors are vector accesses, and a scalar loop over the at
    // most six elements left at the two ends.
    // Ragged rows whose full-shape reads all come from buffers with a padded, 16-byte aligned row
    // pitch (a dot's output): four-element groups from element 0, the padding read but the lanes
    // past the end masked (clamped indices, ok flags); stores to padded outputs stay vector stores.
    bool padded = false;
    if (!vec && L >= 4 * T && !std::getenv("B200_NO_VEC")) {
      std::set<int> memb;
      for (const Value* m : members) memb.insert(m->id);
      int pitched = 0, plain = 0;
      std::set<int> seen;
      std::vector<const Value*> st(members.begin(), members.end());
      while (!st.empty()) {
        const Value* v = st.back();
        st.pop_back();
        if (!seen.insert(v->id).second) continue;
        if (!memb.count(v->id) && slot_of_[Resolve(v)->id] >= 0) {          // a leaf the kernel reads
          if (v->type.dims == X) {
            const int64_t pt = StoredPitch(Resolve(v));
            if (pt && pt % 4 == 0) ++pitched;
            else ++plain;
          }
          continue;
        }
        if (v->def)
          for (const Value* o : v->def->operands) st.push_back(o);
      }
      padded = pitched > 0 && plain == 0;
    }
    const bool shift = !vec && !padded && L >= 4 * T && !std::getenv("B200_NO_VEC");
    if (shift)
      ob << "    const int hd = (int)((4 - (int)((row * " << Ls << "LL) & 3)) & 3), nv = (" << Ls << " - hd) >> 2, nrem = " << Ls
         << " - 4 * nv;\n";
    const std::string shift_head = "#pragma unroll 8\n    for (int jv = lt; jv < nv; jv += " + Ts +
                                   ") {\n      const int j = hd + 4 * jv;\n      const int j_0 = j, j_1 = j + 1, j_2 = j + 2, j_3 = j + 3;\n";
    const std::string rem_head = "    for (int j = lt; j < nrem; j += " + Ts +
                                 ") {\n      const bool ok_1 = false, ok_2 = false, ok_3 = false;\n"
                                 "      const int j_0 = j < hd ? j : j + 4 * nv, j_1 = j_0, j_2 = j_0, j_3 = j_0;\n";
    const std::string padded_head = "#pragma unroll 8\n    for (int j = lt * 4; j < " + Ls + "; j += " + std::to_string(4 * T) +
                                    ") {\n      const bool ok_1 = j + 1 < " + Ls + ", ok_2 = j + 2 < " + Ls + ", ok_3 = j + 3 < " + Ls +
                                    ";\n      const int j_0 = j, j_1 = ok_1 ? j + 1 : " + last + ", j_2 = ok_2 ? j + 2 : " + last +
                                    ", j_3 = ok_3 ? j + 3 : " + last + ";\n";
    bool cur_vec = vec || padded;   // the walk being emitted has four consecutive elements per thread
    std::string cur_head = padded ? padded_head : loop_head;
    gen.lanes_clamped = padded;
    auto ok = [&](int l) { return (cur_vec && !padded) || l == 0 ? std::string() : "ok_" + std::to_string(l); };
    auto elem_index = [&](const Value* m, int l) {
      const int64_t p = StoredPitch(m);
      return "(long long)row * " + (p ? std::to_string(p) : Ls) + "LL + j_" + std::to_string(l);
    };
    // a phase over the row: element values of `v` (one per lane in vector mode)
    auto phase_begin = [&]() {
      gen.cse.clear();
      gen.vloads.clear();
      gen.reindex_cse.clear();
      gen.body.str("");
      gen.body.clear();
      gen.indent = "      ";
      gen.vec = cur_vec;
      gen.shift_dims = shift && cur_vec ? X : std::vector<int64_t>{};
      gen.shift_prefix = gen.row_ident;
      gen.vinner = "j";
      gen.lane_identity = lanes;
      gen.identity = lanes[0];
    };
    // the loops of one walk over the row; `lane_code` emits the phase's values and returns the code
    // that consumes them
    auto walk = [&](const std::function<std::string()>& lane_code) {
      std::string out;
      for (int pass = 0; pass < (shift ? 2 : 1); ++pass) {
        cur_vec = shift ? pass == 0 : vec || padded;
        cur_head = shift ? (pass == 0 ? shift_head : rem_head) : padded ? padded_head : loop_head;
        const std::string tail = lane_code();
        out += cur_head + gen.body.str() + tail + "    }\n";
      }
      cur_vec = vec || padded;
      return out;
    };
    auto phase_vals = [&](const Value* v) {
      std::vector<std::string> vals;
      for (int l = 0; l < 4; ++l) vals.push_back(gen.Emit(v, lanes[l]));
      return vals;
    };
    auto row_phase = [&](const Value* v) {
      phase_begin();
      return phase_vals(v);
    };
    std::vector<std::pair<std::string, std::string>> shared;   // block mode: (type, name)
    std::vector<bool> done(members.size(), false);
    for (size_t k = 0; k < members.size(); ++k) {
      if (done[k]) continue;
      const Value* m = members[k];
      const Op* op = m->def;
      const std::string rk = "r" + std::to_string(k);
      const std::string o = out_of[k] >= 0 ? "out" + std::to_string(out_of[k]) : "";
      // the next reduction, past full members only (they read at most this row's earlier results)
      size_t k2 = k + 1;
      while (k2 < members.size() && members[k2]->type.dims == X && !(members[k2]->def && members[k2]->def->name == "reduce")) ++k2;
      if (op && op->name == "reduce" && k2 < members.size() && OnlinePair(m, members[k2], gen)) {
        // max(x) then sum(exp(x - max)) in one walk of the row: (mx, s) with s = sum exp(x_i - mx)
        // over the elements seen so far, rescaled when mx grows.  Edge cases match the two-pass
        // form: a NaN makes both NaN; an all -inf row or a +inf element makes the sum NaN.
        const std::string k1 = std::to_string(k), kk = std::to_string(k2);
        const std::string mx = "mx" + k1, s = "sx" + k1, bad = "bad" + k1, NINF = "(-__int_as_float(0x7f800000))";
        const std::string nmx = "nmx" + k1;
        body << "    float " << mx << " = " << NINF << ", " << s << " = 0.f, " << nmx << " = " << NINF << ";\n    int " << bad << " = 0;\n";
        body << walk([&]() {
          std::vector<std::string> vals = row_phase(op->operands[0]);
          std::ostringstream t;
          t << "      {\n";
          for (int l = 0; l < 4; ++l)
            t << "        const float c" << l << " = " << (ok(l).empty() ? vals[l] : ok(l) + " ? " + vals[l] + " : " + NINF) << ";\n";
          // exp(d) as 2^(d log2 e) on the SFU: d = c_l - mx is formed first so the scaling only
          // rounds the (small) exponent; NaN inputs are seen by a NaN-propagating max kept beside mx
          t << "        " << nmx << " = fmax_nan(" << nmx << ", fmax_nan(fmax_nan(c0, c1), fmax_nan(c2, c3)));\n"
            << "        const float c = fmaxf(fmaxf(c0, c1), fmaxf(c2, c3));\n"
            << "        if (c > " << mx << ") { " << s << " *= ex2a((" << mx << " - c) * 1.4426950408889634f); " << mx << " = c; }\n"
            << "        if (" << mx << " > " << NINF << ") " << s << " += (ex2a((c0 - " << mx << ") * 1.4426950408889634f) + ex2a((c1 - " << mx
            << ") * 1.4426950408889634f)) + (ex2a((c2 - " << mx << ") * 1.4426950408889634f) + ex2a((c3 - " << mx
            << ") * 1.4426950408889634f));\n      }\n";
          return t.str();
        });
        body << "    " << bad << " = " << nmx << " != " << nmx << ";\n";
        auto merge = [&](const std::string& om, const std::string& os) {
          return "{ const float nm = fmaxf(" + mx + ", " + om + "); " + s + " = (" + mx + " == " + NINF + " ? 0.f : " + s +
                 " * expf(" + mx + " - nm)) + (" + om + " == " + NINF + " ? 0.f : " + os + " * expf(" + om + " - nm)); " + mx +
                 " = nm; }";
        };
        body << "    for (int o = 16; o; o >>= 1) { const float om = __shfl_xor_sync(0xffffffffu, " << mx
             << ", o), os = __shfl_xor_sync(0xffffffffu, " << s << ", o); " << bad << " |= __shfl_xor_sync(0xffffffffu, " << bad
             << ", o); " << merge("om", "os") << " }\n";
        if (block_mode) {
          std::string rm = "redm" + k1, rs = "reds" + k1, rb = "redb" + k1;
          shared.push_back({"float", rm});
          shared.push_back({"float", rs});
          shared.push_back({"int", rb});
          body << "    if ((threadIdx.x & 31) == 0) { " << rm << "[threadIdx.x >> 5] = " << mx << "; " << rs << "[threadIdx.x >> 5] = "
               << s << "; " << rb << "[threadIdx.x >> 5] = " << bad << "; }\n    __syncthreads();\n"
               << "    " << mx << " = " << rm << "[0]; " << s << " = " << rs << "[0]; " << bad << " = " << rb << "[0];\n"
               << "    for (int w = 1; w < " << T / 32 << "; ++w) { " << bad << " |= " << rb << "[w]; " << merge(rm + "[w]", rs + "[w]")
               << " }\n    __syncthreads();\n";
        }
        body << "    if (" << bad << ") { " << mx << " = __int_as_float(0x7fc00000); " << s << " = " << mx << "; } else if (isinf(" << mx
             << ")) " << s << " = __int_as_float(0x7fc00000);\n"
             << "    const float r" << k1 << " = " << mx << ", r" << kk << " = " << s << ";\n";
        for (size_t q : {k, k2}) {
          if (out_of[q] >= 0)
            body << "    if (lt == 0) out" << out_of[q] << "[row] = r" << q << ";\n";
          gen.fixed[members[q]->id] = "r" + std::to_string(q);
        }
        done[k2] = true;
        continue;
      }
      const Value* pick_x = nullptr;
      const Value* pick_label = nullptr;
      if (op && op->name == "reduce" && OneHotPick(op, X, &pick_x, &pick_label)) {
        // sum_j (label == j ? x[j] : 0) is x[label] (+ 0, so -0 comes out +0 as the sum gives it),
        // or 0 for a label outside the row: one load instead of a walk of the row
        DT odt = m->type.dt, acc_dt = AccDt(odt);
        std::string acc_t = CType(acc_dt);
        std::string init = InitExpr(op->operands[1], acc_dt);
        gen.cse.clear();
        gen.body.str("");
        gen.body.clear();
        gen.indent = "    ";
        gen.vec = false;
        gen.identity = gen.row_ident;
        const std::string lab = gen.Emit(pick_label, gen.RowIndex(pick_label->type.dims));
        const std::string li = "pk" + std::to_string(k);
        body << gen.body.str() << "    const long long " << li << " = (long long)(" << lab << ");\n";
        gen.body.str("");
        gen.body.clear();
        std::vector<std::string> at = gen.row_ident;
        at.push_back("(int)(" + li + " < 0 || " + li + " >= " + Ls + "LL ? 0 : " + li + ")");
        const std::string xv = gen.Emit(pick_x, at);
        body << gen.body.str() << "    const " << CType(odt) << " " << rk << " = "
             << FromAcc(odt, Combine(op->reduce, acc_dt, init, "((" + li + " < 0 || " + li + " >= " + Ls + "LL) ? (" + acc_t +
                                                                ")0 : (" + acc_t + ")(" + xv + ") + (" + acc_t + ")0)"))
             << ";\n";
        if (!o.empty()) body << "    if (lt == 0) " << o << "[row] = " << StoreExpr(odt, rk) << ";\n";
        gen.fixed[m->id] = rk;
        continue;
      }
      if (op && op->name == "reduce") {
        DT odt = m->type.dt, acc_dt = AccDt(odt);
        std::string acc_t = CType(acc_dt), acc = "acc" + std::to_string(k);
        std::string init = InitExpr(op->operands[1], acc_dt);
        body << "    " << acc_t << " " << acc << " = (" << acc_t << ")(" << IdentityOf(op->reduce, acc_dt) << ");\n";
        body << walk([&]() {
          std::vector<std::string> vals = row_phase(op->operands[0]);
          std::string t;
          for (int l = 0; l < 4; ++l) {
            std::string x = "(" + acc_t + ")(" + vals[l] + ")";
            if (!ok(l).empty()) x = "(" + ok(l) + " ? " + x + " : (" + acc_t + ")(" + IdentityOf(op->reduce, acc_dt) + "))";
            t += "      " + acc + " = " + Combine(op->reduce, acc_dt, acc, x) + ";\n";
          }
          return t;
        });
        body << "    for (int o = 16; o; o >>= 1) { " << acc_t << " oth = __shfl_xor_sync(0xffffffffu, " << acc << ", o); "
             << acc << " = " << Combine(op->reduce, acc_dt, acc, "oth") << "; }\n";
        if (block_mode) {
          std::string red = "red" + std::to_string(k);
          shared.push_back({acc_t, red});
          body << "    if ((threadIdx.x & 31) == 0) " << red << "[threadIdx.x >> 5] = " << acc << ";\n    __syncthreads();\n"
               << "    " << acc << " = " << red << "[0];\n"
               << "    for (int w = 1; w < " << T / 32 << "; ++w) " << acc << " = " << Combine(op->reduce, acc_dt, acc, red + "[w]") << ";\n"
               << "    __syncthreads();\n";
        }
        body << "    const " << CType(odt) << " " << rk << " = " << FromAcc(odt, Combine(op->reduce, acc_dt, init, acc)) << ";\n";
        if (!o.empty()) body << "    if (lt == 0) " << o << "[row] = " << StoreExpr(odt, rk) << ";\n";
        gen.fixed[m->id] = rk;
      } else if (m->type.dims == X) {
        // a run of consecutive full members shares one walk of the row; internal ones are not
        // stored (the members that read them recompute them)
        size_t k_end = k;
        while (k_end < members.size() && !done[k_end] && members[k_end]->type.dims == X &&
               !(members[k_end]->def && members[k_end]->def->name == "reduce"))
          ++k_end;
        std::vector<size_t> stored;
        for (size_t q = k; q < k_end; ++q) {
          done[q] = true;
          if (out_of[q] >= 0) stored.push_back(q);
        }
        k = k_end - 1;
        if (stored.empty()) continue;
        body << walk([&]() {
          phase_begin();
          std::vector<std::vector<std::string>> vals_of;
          for (size_t q : stored) vals_of.push_back(phase_vals(members[q]));
          std::ostringstream t;
          for (size_t i = 0; i < stored.size(); ++i) {
            const Value* mq = members[stored[i]];
            const std::string oq = "out" + std::to_string(out_of[stored[i]]);
            std::vector<std::string>& vals = vals_of[i];
            DT dt = StoredDt(mq);
            for (auto& x : vals) x = StoreVal(mq, dt, x);
            // vector stores need the row's alignment: with a ragged row only an unpadded output has it
            const bool vstore = padded ? StoredPitch(mq) % 4 == 0 && StoredPitch(mq) > 0 : cur_vec && (!shift || StoredPitch(mq) == 0);
            if (!vstore || (dt != DT::kF32 && dt != DT::kBF16 && dt != DT::kF16)) {
              for (int l = 0; l < 4; ++l)
                t << "      " << (ok(l).empty() ? "" : "if (" + ok(l) + ") ") << oq << "[" << elem_index(mq, l) << "] = " << StoreExpr(dt, vals[l]) << ";\n";
            } else if (dt == DT::kF32) {
              t << "      *(float4*)(" << oq << " + " << elem_index(mq, 0) << ") = make_float4(" << vals[0] << ", " << vals[1] << ", " << vals[2] << ", " << vals[3] << ");\n";
            } else {
              t << "      *(uint2*)(" << oq << " + " << elem_index(mq, 0) << ") = make_uint2(" << Pack16(dt, vals[0], vals[1]) << ", " << Pack16(dt, vals[2], vals[3]) << ");\n";
            }
          }
          return t.str();
        });
      } else {
        // row scalar: every thread of the row computes it
        gen.cse.clear();
        gen.reindex_cse.clear();
        gen.body.str("");
        gen.body.clear();
        gen.indent = "    ";
        gen.vec = false;
        gen.identity = gen.row_ident;
        std::string v = gen.Emit(m, gen.RowIndex(m->type.dims));
        body << gen.body.str() << "    const " << CType(m->type.dt) << " " << rk << " = " << v << ";\n";
        if (!o.empty()) body << "    if (lt == 0) " << o << "[row] = " << StoreExpr(StoredDt(m), StoreVal(m, StoredDt(m), rk)) << ";\n";
        gen.fixed[m->id] = rk;
      }
    }
    if (dry || gen.conflict) {
      bool ok = !gen.conflict;
      slot_of_ = saved;
      p_->slots.resize(saved_slots);
      if (!dry) throw LowerError{"internal: row fusion conflict"};
      return ok;
    }
    for (size_t k = 0; k < members.size(); ++k) slot_of_[members[k]->id] = member_slot[k];
    std::vector<DT> in_dts;
    for (int s : gen.in_slots) in_dts.push_back(SlotDt(s));
    // a row loop of elementwise members only is one walk over each row: a result aliased to a
    // donated argument that the walk reads only at the element it writes can be written in place
    std::vector<std::pair<int, int>> inplace;
    std::set<int> shared_in, shared_out;
    bool one_walk = !any_reduce;
    for (const Value* m : members) one_walk = one_walk && m->type.dims == X;
    for (size_t k = 0; one_walk && k < members.size(); ++k) {
      auto al = alias_arg_slot_.find(members[k]->id);
      if (al == alias_arg_slot_.end() || out_of[k] < 0) continue;
      const int sa = al->second, so = out_slots[out_of[k]];
      if (p_->slots[sa].bytes != p_->slots[so].bytes || slot_pitch_.count(so)) continue;
      auto pi = gen.param_of.find(sa);
      if (pi != gen.param_of.end()) {
        if (gen.nonident.count(sa)) continue;
        shared_in.insert(pi->second);
      }
      shared_out.insert(out_of[k]);
      inplace.push_back({sa, so});
    }
    std::string fn = KName();
    const int threads = block_mode ? 512 : 256;
    src_ << "extern \"C\" __global__ void __launch_bounds__(" << threads << ", " << (block_mode ? 2 : 4) << ") " << fn << "("
         << KernelParams(gen.in_slots, (int)out_slots.size(), false, shared_in, shared_out) << ") {\n"
         << ParamCasts(gen.in_slots, in_dts, out_dts, shared_in, shared_out);
    for (const auto& s : shared) src_ << "  __shared__ " << s.first << " " << s.second << "[32];\n";
    if (block_mode)
      src_ << "  const int lt = threadIdx.x;\n"
           << "  for (long long row = blockIdx.x; row < " << rows << "LL; row += gridDim.x) {\n";
    else if (nseg > 1)
      src_ << "  const int lt = threadIdx.x & 31;\n"
           << "  for (long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); w < " << rows * nseg
           << "LL; w += (long long)gridDim.x * 8) {\n"
           << "    const long long row = w / " << nseg << ";\n    const int sg = (int)(w % " << nseg << ");\n";
    else
      src_ << "  const int lt = threadIdx.x & 31;\n"
           << "  for (long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); row < " << rows
           << "LL; row += (long long)gridDim.x * 8) {\n";
    src_ << ob.str() << body.str() << "  }\n}\n";
    EndKernel();
    Launch Lc;
    Lc.fn = fn;
    Lc.in_slots = gen.in_slots;
    Lc.out_slots = out_slots;
    Lc.block = threads;
    Lc.grid_x = block_mode ? std::max<int64_t>(1, rows) : std::max<int64_t>(1, (rows * nseg + 7) / 8);
    Lc.grid_stride = true;
    Lc.inplace = inplace;
    Step st;
    st.kind = StepKind::kFusion;
    st.launches.push_back(Lc);
    st.label = "rowloop " + members[0]->type.str() + " x" + std::to_string(members.size());
    for (const Value* m : members)
      if (m->def && m->def->name == "reduce") {
        st.label = "row " + m->def->operands[0]->type.str() + " x" + std::to_string(members.size());
        break;
      }
    p_->steps.push_back(st);
    for (size_t k = 0; k < out_slots.size(); ++k) RecordDt(out_slots[k], out_dts[k]);
    return true;
  }

  // ---------------------------------------------------------------- argmax / argmin
  // The two-operand reduce jnp.argmax / argmin emit: (x, iota along the axis) with inits
  // (-inf | +inf | int extreme, 0) and a reducer whose first comparison is GT (argmax) or LT (argmin),
  // recognised as the reference's DetectArgReduce does (src/jam/ops/reduce.mm:29-43).  Result: the
  // extreme value and the smallest index holding it; a NaN counts as the extreme (the first NaN
  // wins), which is what the jnp reducer body computes when folded in index order.
  void EmitArgReduce(Op* op) {
    auto fail = [&]() { throw LowerError{"variadic reduce other than argmax / argmin is not supported"}; };
    if (op->operands.size() != 4 || op->results.size() != 2) fail();
    auto rc = op->strs.find("region_compare");
    if (rc == op->strs.end() || (rc->second != "GT" && rc->second != "LT")) fail();
    const bool is_max = rc->second == "GT";
    const std::vector<int64_t> rd = op->ints.at("dimensions");
    if (rd.size() != 1) fail();
    const Value* x = op->operands[0];
    const Value* io = op->operands[1];
    const int ax = (int)rd[0];
    if (!io->def || io->def->name != "iota" || io->def->ints.at("dim")[0] != ax || io->type.dims != x->type.dims) fail();
    double i0 = 0;
    if (!IsScalarConst(op->operands[3], &i0) || i0 != 0) fail();
    const DT vdt = x->type.dt, idt = op->results[1]->type.dt;
    if (!(DTIsFloat(vdt) || DTIsSigned(vdt)) || !(idt == DT::kS32 || idt == DT::kS64)) fail();
    const bool fl = DTIsFloat(vdt);
    const DT acc_dt = AccDt(vdt);
    const std::string at = CType(acc_dt), it = CType(idt);
    const auto& xd = x->type.dims;
    std::vector<int64_t> kept;
    for (int k = 0; k < (int)xd.size(); ++k) if (k != ax) kept.push_back(xd[k]);
    const int64_t L = xd[ax];
    int64_t n_out = 1;
    for (int64_t d : kept) n_out *= d;
    const bool wide = x->type.numel() >= (1LL << 31);
    const bool inner = ax == (int)xd.size() - 1;
    const int out_v = SlotFor(op->results[0]), out_i = SlotFor(op->results[1]);
    std::string init = InitExpr(op->operands[2], acc_dt);
    // better(a, b): a NaN beats any number (the smaller index among NaNs), else the larger (smaller)
    // value, else the smaller index
    const std::string cmp = is_max ? ">" : "<";
    std::string better = "static __device__ __forceinline__ bool " + std::string("%FN%_better(") + at + " av, " + it + " ai, " + at +
                         " bv, " + it + " bi) {\n";
    if (fl) better += "  if (av != av) return bv == bv || ai < bi;\n  if (bv != bv) return false;\n";
    better += "  if (av != bv) return av " + cmp + " bv;\n  return ai < bi;\n}\n";
    Gen gen;
    gen.slot_of = &slot_of_;
    gen.slot_pitch = &slot_pitch_;
    gen.slot_f32 = &slot_f32_;
    gen.indent = "      ";
    std::ostringstream ob, jb;
    auto names_k = Delinearize(ob, inner ? "row" : "o", kept, "a", "    ", wide);
    std::vector<std::string> idx(xd.size());
    for (int k = 0, q = 0; k < (int)xd.size(); ++k) idx[k] = k == ax ? "j" : names_k[q++];
    std::string v = gen.Emit(x, idx);
    std::vector<DT> in_dts;
    for (int sl : gen.in_slots) in_dts.push_back(SlotDt(sl));
    std::string fn = KName();
    size_t pos;
    while ((pos = better.find("%FN%")) != std::string::npos) better.replace(pos, 4, fn);
    std::ostringstream k;
    k << better << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(" << KernelParams(gen.in_slots, 2, false)
      << ") {\n" << ParamCasts(gen.in_slots, in_dts, {vdt, idt});
    const std::string scan = "      { const " + at + " cv = (" + at + ")(" + v + "); if (" + fn + "_better(cv, (" + it +
                             ")j, bv, bi)) { bv = cv; bi = (" + it + ")j; } }\n";
    Launch Lc;
    Lc.fn = fn;
    Lc.in_slots = gen.in_slots;
    Lc.out_slots = {out_v, out_i};
    Lc.block = 256;
    Lc.grid_stride = true;
    if (inner) {
      k << "  const int lane = threadIdx.x & 31;\n"
        << "  for (long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); row < " << n_out << "LL; row += (long long)gridDim.x * 8) {\n"
        << ob.str() << "    " << at << " bv = " << init << "; " << it << " bi = 0;\n"
        << "    for (long long j = lane; j < " << L << "LL; j += 32) {\n" << gen.body.str() << scan << "    }\n"
        << "    for (int o = 16; o; o >>= 1) {\n"
        << "      const " << at << " ov = __shfl_xor_sync(0xffffffffu, bv, o); const " << it << " oi = __shfl_xor_sync(0xffffffffu, bi, o);\n"
        << "      if (" << fn << "_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }\n    }\n"
        << "    if (lane == 0) { out0[row] = " << StoreExpr(vdt, FromAcc(vdt, "bv")) << "; out1[row] = bi; }\n  }\n}\n";
      Lc.grid_x = std::max<int64_t>(1, (n_out + 7) / 8);
    } else {
      k << "  for (long long o = (long long)blockIdx.x * 256 + threadIdx.x; o < " << n_out << "LL; o += (long long)gridDim.x * 256) {\n"
        << ob.str() << "    " << at << " bv = " << init << "; " << it << " bi = 0;\n"
        << "    for (long long j = 0; j < " << L << "LL; ++j) {\n" << gen.body.str() << scan << "    }\n"
        << "    out0[o] = " << StoreExpr(vdt, FromAcc(vdt, "bv")) << "; out1[o] = bi;\n  }\n}\n";
      Lc.grid_x = std::max<int64_t>(1, (n_out + 255) / 256);
    }
    src_ << k.str();
    EndKernel();
    Step st;
    st.kind = StepKind::kFusion;
    st.launches.push_back(Lc);
    st.label = std::string(is_max ? "argmax " : "argmin ") + x->type.str();
    p_->steps.push_back(st);
    RecordDt(out_v, vdt);
    RecordDt(out_i, idt);
  }

  // ---------------------------------------------------------------- reductions
  // a reduction over leading dims whose kept contiguous dim is a multiple of 4 (the vectorised
  // column path), accumulating in f32
  bool VecColumnReduce(const Op* op) const {
    if (op->results.size() != 1 || op->reduce == ReduceKind::kNone || std::getenv("B200_NO_VEC")) return false;
    const auto& xd = op->operands[0]->type.dims;
    std::vector<int64_t> rd = op->ints.at("dimensions");
    if (xd.empty() || rd.empty() || std::find(rd.begin(), rd.end(), (int64_t)xd.size() - 1) != rd.end()) return false;
    const DT odt = op->result()->type.dt;
    if (odt != DT::kF32 && odt != DT::kBF16 && odt != DT::kF16) return false;
    return xd.back() % 4 == 0 && op->result()->type.numel() % 4 == 0;
  }
  static bool SameColumnReduce(const Op* a, const Op* b) {
    std::vector<int64_t> ra = a->ints.at("dimensions"), rb = b->ints.at("dimensions");
    std::sort(ra.begin(), ra.end());
    std::sort(rb.begin(), rb.end());
    return ra == rb && a->operands[0]->type.dims == b->operands[0]->type.dims;
  }
  // whether the value v (through the values computed inline) reads the result of any of `ops`
  bool ReadsAny(const Value* v, const std::vector<Op*>& ops) const {
    std::set<int> res;
    for (const Op* o : ops) res.insert(o->result()->id);
    std::set<int> seen;
    std::vector<const Value*> st{v};
    while (!st.empty()) {
      const Value* x = st.back();
      st.pop_back();
      if (!seen.insert(x->id).second) continue;
      if (res.count(x->id)) return true;
      if (slot_of_[Resolve(x)->id] >= 0 && !x->def) continue;
      if (x->def && !IsHeavy(x->def))
        for (const Value* o : x->def->operands) st.push_back(o);
    }
    return false;
  }

  // Column reductions (the contiguous dim kept; siblings of one operand shape over the same dims
  // together) as one kernel: a block is TX column quads x TY row lanes; each thread owns four
  // adjacent outputs of every reduction and reads them with one vector load per reduced index, the
  // TY lanes of a block combine in shared memory, and each block writes one partial row per
  // reduction; a second kernel combines the blocks' partials with coalesced reads (a warp covers
  // 32 consecutive outputs).
  void EmitColumnReduceGroup(const std::vector<Op*>& ops) {
    const int K = (int)ops.size();
    const Value* x0 = ops[0]->operands[0];
    std::vector<int64_t> rd = ops[0]->ints.at("dimensions");
    std::sort(rd.begin(), rd.end());
    const auto& xd = x0->type.dims;
    std::vector<int64_t> kept, red;
    std::vector<int> kept_ax, red_ax;
    for (int k = 0; k < (int)xd.size(); ++k) {
      if (std::binary_search(rd.begin(), rd.end(), (int64_t)k)) { red.push_back(xd[k]); red_ax.push_back(k); }
      else { kept.push_back(xd[k]); kept_ax.push_back(k); }
    }
    const int64_t n_out = ops[0]->result()->type.numel();
    int64_t L = 1;
    for (int64_t d : red) L *= d;
    const bool wide = x0->type.numel() >= (1LL << 31);
    auto combine = [&](ReduceKind kind, const std::string& a, const std::string& b) { return Combine(kind, DT::kF32, a, b); };
    std::vector<std::string> init_expr(K), ident(K);
    std::vector<int> out_slot(K);
    std::vector<DT> odt(K);
    for (int q = 0; q < K; ++q) {
      init_expr[q] = InitExpr(ops[q]->operands[1], DT::kF32);
      ident[q] = "(float)(" + IdentityOf(ops[q]->reduce, DT::kF32) + ")";
      out_slot[q] = SlotFor(ops[q]->result());
      odt[q] = ops[q]->result()->type.dt;
    }
    const int64_t n4 = n_out / 4;
    const int TX = (int)std::min<int64_t>(32, n4), TY = 256 / TX;
    const int64_t gx = (n4 + TX - 1) / TX;
    // row chunks: about four blocks per SM, each row lane taking >= 8 reduced indices
    int64_t chunks = std::max<int64_t>(1, std::min<int64_t>((148 * 4 + gx - 1) / gx, L / (8 * TY)));
    chunks = std::min<int64_t>(chunks, 1024);
    const int64_t per = (L + chunks - 1) / chunks;       // reduced indices per block
    chunks = (L + per - 1) / per;
    Gen gen;
    gen.slot_of = &slot_of_;
    gen.slot_pitch = &slot_pitch_;
    gen.slot_f32 = &slot_f32_;
    gen.indent = "      ";
    std::ostringstream ob, inner_pre, k;
    auto names_k = Delinearize(ob, "o4", kept, "a", "  ", wide);
    auto names_r = Delinearize(inner_pre, "j", red, "b", "      ", wide);
    const std::string vin = names_k.back();
    std::vector<std::vector<std::string>> lanes(4, std::vector<std::string>(xd.size()));
    for (int l = 0; l < 4; ++l) {
      for (size_t q = 0; q < kept_ax.size(); ++q) lanes[l][kept_ax[q]] = names_k[q];
      lanes[l][kept_ax.back()] = vin + "_" + std::to_string(l);
      for (size_t q = 0; q < red_ax.size(); ++q) lanes[l][red_ax[q]] = names_r[q];
    }
    gen.vec = true;
    gen.vinner = vin;
    gen.lane_identity = lanes;
    gen.identity = lanes[0];
    gen.body << inner_pre.str();
    std::vector<std::vector<std::string>> vals(K);
    for (int q = 0; q < K; ++q)
      for (int l = 0; l < 4; ++l) vals[q].push_back(gen.Emit(ops[q]->operands[0], lanes[l]));
    std::vector<DT> in_dts;
    for (int s : gen.in_slots) in_dts.push_back(SlotDt(s));
    const int scratch = chunks > 1 ? NewSlot((int64_t)K * chunks * n_out * 4) : -1;
    const std::string fn = KName();
    std::vector<DT> out_dts = chunks > 1 ? std::vector<DT>{DT::kF32} : odt;
    k << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "("
      << KernelParams(gen.in_slots, (int)out_dts.size(), false) << ") {\n" << ParamCasts(gen.in_slots, in_dts, out_dts)
      << "  __shared__ float4 red_s[" << K << "][" << TY << "][" << TX << "];\n"
      << "  const int tx = threadIdx.x % " << TX << ", ty = threadIdx.x / " << TX << ";\n"
      << "  const long long o = (long long)blockIdx.x * " << TX << " + tx;\n"
      << "  const bool live = o < " << n4 << "LL;\n"
      << "  const long long o4 = (live ? o : 0) * 4;\n" << ob.str()
      << "  const int " << vin << "_0 = " << vin << ", " << vin << "_1 = " << vin << " + 1, " << vin << "_2 = " << vin << " + 2, "
      << vin << "_3 = " << vin << " + 3;\n";
    for (int q = 0; q < K; ++q)
      for (int l = 0; l < 4; ++l) k << "  float acc" << q << "_" << l << " = " << ident[q] << ";\n";
    k << "  const long long jb = (long long)blockIdx.y * " << per << "LL;\n"
      << "  const long long je = jb + " << per << "LL < " << L << "LL ? jb + " << per << "LL : " << L << "LL;\n"
      << "#pragma unroll 4\n  for (long long j = jb + ty; j < je; j += " << TY << ") {\n" << gen.body.str();
    for (int q = 0; q < K; ++q)
      for (int l = 0; l < 4; ++l) {
        const std::string a = "acc" + std::to_string(q) + "_" + std::to_string(l);
        k << "      " << a << " = " << combine(ops[q]->reduce, a, "(float)(" + vals[q][l] + ")") << ";\n";
      }
    k << "  }\n";
    for (int q = 0; q < K; ++q)
      k << "  red_s[" << q << "][ty][tx] = make_float4(acc" << q << "_0, acc" << q << "_1, acc" << q << "_2, acc" << q << "_3);\n";
    k << "  __syncthreads();\n  if (ty == 0 && live) {\n";
    for (int q = 0; q < K; ++q) {
      const std::string a = "acc" + std::to_string(q) + "_";
      k << "    for (int y = 1; y < " << TY << "; ++y) {\n      const float4 t = red_s[" << q << "][y][tx];\n";
      static const char* c[] = {"x", "y", "z", "w"};
      for (int l = 0; l < 4; ++l) k << "      " << a << l << " = " << combine(ops[q]->reduce, a + std::to_string(l), std::string("t.") + c[l]) << ";\n";
      k << "    }\n";
      if (chunks > 1)
        k << "    *(float4*)(out0 + ((long long)" << q << " * " << chunks << "LL + blockIdx.y) * " << n_out << "LL + o4) = make_float4("
          << a << "0, " << a << "1, " << a << "2, " << a << "3);\n";
      else
        for (int l = 0; l < 4; ++l)
          k << "    out" << q << "[o4 + " << l << "] = "
            << StoreExpr(odt[q], FromAcc(odt[q], combine(ops[q]->reduce, init_expr[q], a + std::to_string(l)))) << ";\n";
    }
    k << "  }\n}\n";
    Launch L1;
    L1.fn = fn;
    L1.in_slots = gen.in_slots;
    L1.out_slots = chunks > 1 ? std::vector<int>{scratch} : out_slot;
    L1.block = TX * TY;
    L1.grid_x = gx;
    L1.grid_y = chunks;
    Step st;
    st.kind = StepKind::kFusion;
    st.label = (K > 1 ? "reduce x" + std::to_string(K) + " " : std::string("reduce ")) + x0->type.str() + " -> " +
               ops[0]->result()->type.str();
    st.launches.push_back(L1);
    if (chunks > 1) {
      // finish: a block per 32 consecutive (reduction, output) pairs; its 8 warps take every 8th
      // partial row (coalesced 128-byte reads), then combine in shared memory in a fixed order
      const std::string fn2 = KName();
      k << "extern \"C\" __global__ void __launch_bounds__(256) " << fn2 << "(const void* __restrict__ p0";
      for (int q = 0; q < K; ++q) k << ", void* __restrict__ q" << q;
      k << ") {\n  const float* part = (const float*)p0;\n  __shared__ float fin_s[8][32];\n"
        << "  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;\n"
        << "  const long long w = (long long)blockIdx.x * 32 + tx;\n"
        << "  const bool live = w < " << K * n_out << "LL;\n"
        << "  const int q = live ? (int)(w / " << n_out << "LL) : 0;\n"
        << "  const long long o = live ? w - (long long)q * " << n_out << "LL : 0;\n"
        << "  const float* pq = part + (long long)q * " << chunks * n_out << "LL + o;\n"
        << "  float acc = 0.f;\n";
      for (int q = 0; q < K; ++q)
        k << "  " << (q ? "else " : "") << "if (q == " << q << ") {\n    acc = " << ident[q] << ";\n"
          << "#pragma unroll 4\n    for (int c = ty; c < " << chunks << "; c += 8) acc = "
          << combine(ops[q]->reduce, "acc", "pq[(long long)c * " + std::to_string(n_out) + "LL]") << ";\n  }\n";
      k << "  fin_s[ty][tx] = acc;\n  __syncthreads();\n  if (ty == 0 && live) {\n";
      for (int q = 0; q < K; ++q)
        k << "    " << (q ? "else " : "") << "if (q == " << q << ") {\n      for (int y = 1; y < 8; ++y) acc = "
          << combine(ops[q]->reduce, "acc", "fin_s[y][tx]") << ";\n      ((" << MemType(odt[q]) << "*)q" << q << ")[o] = "
          << StoreExpr(odt[q], FromAcc(odt[q], combine(ops[q]->reduce, init_expr[q], "acc"))) << ";\n    }\n";
      k << "  }\n}\n";
      Launch L2;
      L2.fn = fn2;
      L2.in_slots = {scratch};
      L2.out_slots = out_slot;
      L2.block = 256;
      L2.grid_x = std::max<int64_t>(1, (K * n_out + 31) / 32);
      st.launches.push_back(L2);
      RecordDt(scratch, DT::kF32);
    }
    src_ << k.str();
    EndKernel();
    for (int q = 0; q < K; ++q) RecordDt(out_slot[q], odt[q]);
    p_->steps.push_back(st);
  }

  void EmitReduce(Op* op) {
    if (op->results.size() != 1) throw LowerError{"variadic reduce (argmax/argmin) is not supported yet"};
    const Value* x = op->operands[0];
    const Value* init = op->operands[1];
    Value* r = op->result();
    std::vector<int64_t> rd = op->ints.at("dimensions");
    std::sort(rd.begin(), rd.end());
    const auto& xd = x->type.dims;
    std::vector<int64_t> kept, red;
    std::vector<int> kept_ax, red_ax;
    for (int k = 0; k < (int)xd.size(); ++k) {
      if (std::binary_search(rd.begin(), rd.end(), (int64_t)k)) { red.push_back(xd[k]); red_ax.push_back(k); }
      else { kept.push_back(xd[k]); kept_ax.push_back(k); }
    }
    int64_t n_out = r->type.numel(), L = 1;
    for (int64_t d : red) L *= d;
    ReduceKind kind = op->reduce;
    if (kind == ReduceKind::kNone) throw LowerError{"reduce with an unrecognised reducer body"};
    DT odt = r->type.dt;
    DT acc_dt = odt == DT::kF64 ? DT::kF64 : DTIsFloat(odt) ? DT::kF32 : odt;
    std::string acc_t = CType(acc_dt);
    auto combine = [&](const std::string& a, const std::string& b) -> std::string {
      bool f = DTIsFloat(acc_dt), d = acc_dt == DT::kF64;
      switch (kind) {
        case ReduceKind::kAdd: return a + " + " + b;
        case ReduceKind::kMul: return a + " * " + b;
        case ReduceKind::kMax: return f ? (d ? "dmax_n(" : "fmax_n(") + a + ", " + b + ")" : "imax(" + a + ", " + b + ")";
        case ReduceKind::kMin: return f ? (d ? "dmin_n(" : "fmin_n(") + a + ", " + b + ")" : "imin(" + a + ", " + b + ")";
        case ReduceKind::kAnd: return acc_dt == DT::kPred ? a + " && " + b : a + " & " + b;
        case ReduceKind::kOr: return acc_dt == DT::kPred ? a + " || " + b : a + " | " + b;
        default: return a;
      }
    };
    bool inner = !red_ax.empty() && red_ax.back() == (int)xd.size() - 1;  // reduces the contiguous dim
    int out_slot = SlotFor(r);
    Gen gen;
    gen.slot_of = &slot_of_;
    gen.slot_pitch = &slot_pitch_;
    gen.slot_f32 = &slot_f32_;
    std::ostringstream pre;
    // init value (scalar expression)
    std::string init_expr;
    {
      Gen ig;
      ig.slot_of = &slot_of_;
      ig.tmp = 1000000;
      std::string iv = ig.Emit(init, {});
      if (!ig.in_slots.empty()) throw LowerError{"reduce init must be a constant"};
      init_expr = "(" + acc_t + ")(" + iv + ")";
      if (!ig.body.str().empty()) throw LowerError{"reduce init must be a splat constant"};
    }
    std::string fn = KName();
    std::ostringstream k;
    Step st;
    st.kind = StepKind::kFusion;
    st.label = "reduce " + x->type.str() + " -> " + r->type.str();
    bool wide = x->type.numel() >= (1LL << 31);
    const std::string shfl_red = R"(    for (int o = 16; o; o >>= 1) { )" + acc_t + " oth = __shfl_xor_sync(0xffffffffu, acc, o); acc = " +
                                 combine("acc", "oth") + "; }\n";
    if (inner && L >= 16 && (n_out >= 148 * 4 || L < 8192)) {
      // warp or block per output row; reduced index split into (kept, reduced) dims
      bool block_per_row = L >= 4096;
      int threads = block_per_row ? 512 : 256;
      gen.indent = "      ";
      std::ostringstream ob;
      // element index: kept part from `row`, reduced part from `j`
      auto names_k = Delinearize(ob, "row", kept, "a", "    ", wide);
      std::ostringstream inner_pre;
      auto names_r = Delinearize(inner_pre, "j", red, "b", "      ", wide);
      std::vector<std::string> idx(xd.size());
      for (size_t q = 0; q < kept_ax.size(); ++q) idx[kept_ax[q]] = names_k[q];
      for (size_t q = 0; q < red_ax.size(); ++q) idx[red_ax[q]] = names_r[q];
      gen.body << inner_pre.str();
      // cse entries made inside the loop must not leak outside: emit everything inside the loop
      std::string v = gen.Emit(x, idx);
      std::vector<DT> in_dts;
      for (int s : gen.in_slots) in_dts.push_back(SlotDt(s));
      k << "extern \"C\" __global__ void __launch_bounds__(" << threads << ") " << fn << "("
        << KernelParams(gen.in_slots, 1, false) << ") {\n" << ParamCasts(gen.in_slots, in_dts, {odt});
      if (block_per_row) {
        k << "  __shared__ " << acc_t << " red[32];\n"
          << "  for (long long row = blockIdx.x; row < " << n_out << "LL; row += gridDim.x) {\n"
          << ob.str() << "    " << acc_t << " acc = " << "(" + acc_t + ")(" + IdentityOf(kind, acc_dt) + ")" << ";\n"
          << "#pragma unroll 4\n    for (long long j = threadIdx.x; j < " << L << "LL; j += " << threads << ") {\n"
          << gen.body.str() << "      acc = " << combine("acc", "(" + acc_t + ")(" + v + ")") << ";\n    }\n"
          << shfl_red
          << "    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;\n    __syncthreads();\n"
          << "    if (threadIdx.x < 32) {\n      acc = threadIdx.x < " << threads / 32 << " ? red[threadIdx.x] : (" << acc_t << ")(" << IdentityOf(kind, acc_dt) << ");\n"
          << "  " << shfl_red
          << "      if (threadIdx.x == 0) out0[row] = " << StoreExpr(odt, FromAcc(odt, combine(init_expr, "acc"))) << ";\n    }\n    __syncthreads();\n  }\n}\n";
        Launch Lc;
        Lc.fn = fn;
        Lc.in_slots = gen.in_slots;
        Lc.out_slots = {out_slot};
        Lc.block = threads;
        Lc.grid_x = std::max<int64_t>(1, n_out);
        Lc.grid_stride = true;
        st.launches.push_back(Lc);
      } else {
        k << "  const int lane = threadIdx.x & 31;\n"
          << "  for (long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); row < " << n_out << "LL; row += (long long)gridDim.x * 8) {\n"
          << ob.str() << "    " << acc_t << " acc = " << "(" + acc_t + ")(" + IdentityOf(kind, acc_dt) + ")" << ";\n"
          << "#pragma unroll 4\n    for (long long j = lane; j < " << L << "LL; j += 32) {\n"
          << gen.body.str() << "      acc = " << combine("acc", "(" + acc_t + ")(" + v + ")") << ";\n    }\n"
          << shfl_red << "    if (lane == 0) out0[row] = " << StoreExpr(odt, FromAcc(odt, combine(init_expr, "acc"))) << ";\n  }\n}\n";
        Launch Lc;
        Lc.fn = fn;
        Lc.in_slots = gen.in_slots;
        Lc.out_slots = {out_slot};
        Lc.block = 256;
        Lc.grid_x = std::max<int64_t>(1, (n_out + 7) / 8);
        Lc.grid_stride = true;
        st.launches.push_back(Lc);
      }
    } else if (!inner && !kept_ax.empty() && kept_ax.back() == (int)xd.size() - 1 && kept.back() % 4 == 0 &&
               acc_dt == DT::kF32 && !std::getenv("B200_NO_VEC")) {
      // Column reduction (the contiguous dim is kept): a thread owns four adjacent outputs and reads
      // them with one vector load per reduced index; the reduced range is split over `chunks` blocks
      // in y whose partials a second kernel combines.
      const int64_t n4 = n_out / 4;
      int64_t chunks = 1;
      const int64_t want_threads = 148LL * 2048;
      if (L > 16) chunks = std::min<int64_t>((want_threads + n4 - 1) / n4, std::max<int64_t>(1, L / 16));
      chunks = std::max<int64_t>(1, std::min<int64_t>(chunks, 1024));
      const int64_t per = (L + chunks - 1) / chunks;
      chunks = (L + per - 1) / per;
      const int bt = (int)std::min<int64_t>(256, (n4 + 31) / 32 * 32);
      gen.indent = "      ";
      std::ostringstream ob;
      auto names_k = Delinearize(ob, "o4", kept, "a", "  ", wide);
      std::ostringstream inner_pre;
      auto names_r = Delinearize(inner_pre, "j", red, "b", "      ", wide);
      const std::string vin = names_k.back();
      std::vector<std::vector<std::string>> lanes(4, std::vector<std::string>(xd.size()));
      for (int l = 0; l < 4; ++l) {
        for (size_t q = 0; q < kept_ax.size(); ++q) lanes[l][kept_ax[q]] = names_k[q];
        lanes[l][kept_ax.back()] = vin + "_" + std::to_string(l);
        for (size_t q = 0; q < red_ax.size(); ++q) lanes[l][red_ax[q]] = names_r[q];
      }
      gen.vec = true;
      gen.vinner = vin;
      gen.lane_identity = lanes;
      gen.identity = lanes[0];
      gen.body << inner_pre.str();
      std::vector<std::string> vals;
      for (int l = 0; l < 4; ++l) vals.push_back(gen.Emit(x, lanes[l]));
      std::vector<DT> in_dts;
      for (int s : gen.in_slots) in_dts.push_back(SlotDt(s));
      int scratch = -1;
      if (chunks > 1) scratch = NewSlot(chunks * n_out * 4);
      const std::string ident = "(" + acc_t + ")(" + IdentityOf(kind, acc_dt) + ")";
      k << "extern \"C\" __global__ void __launch_bounds__(" << bt << ") " << fn << "("
        << KernelParams(gen.in_slots, 1, false) << ") {\n" << ParamCasts(gen.in_slots, in_dts, {chunks > 1 ? DT::kF32 : odt})
        << "  const long long o = (long long)blockIdx.x * " << bt << " + threadIdx.x;\n  if (o >= " << n4 << "LL) return;\n"
        << "  const long long o4 = o * 4;\n" << ob.str()
        << "  const int " << vin << "_0 = " << vin << ", " << vin << "_1 = " << vin << " + 1, " << vin << "_2 = " << vin << " + 2, "
        << vin << "_3 = " << vin << " + 3;\n";
      for (int l = 0; l < 4; ++l) k << "  " << acc_t << " acc" << l << " = " << (chunks > 1 ? ident : init_expr) << ";\n";
      k << "  const long long j0 = (long long)blockIdx.y * " << per << "LL;\n"
        << "  const long long j1 = j0 + " << per << "LL < " << L << "LL ? j0 + " << per << "LL : " << L << "LL;\n"
        << "#pragma unroll 8\n  for (long long j = j0; j < j1; ++j) {\n" << gen.body.str();
      for (int l = 0; l < 4; ++l)
        k << "      acc" << l << " = " << combine("acc" + std::to_string(l), "(" + acc_t + ")(" + vals[l] + ")") << ";\n";
      k << "  }\n";
      if (chunks > 1)
        k << "  *(float4*)(out0 + (long long)blockIdx.y * " << n_out << "LL + o4) = make_float4(acc0, acc1, acc2, acc3);\n}\n";
      else
        for (int l = 0; l < 4; ++l) k << "  out0[o4 + " << l << "] = " << StoreExpr(odt, FromAcc(odt, "acc" + std::to_string(l))) << ";\n";
      if (chunks == 1) k << "}\n";
      Launch L1;
      L1.fn = fn;
      L1.in_slots = gen.in_slots;
      L1.out_slots = {chunks > 1 ? scratch : out_slot};
      L1.block = bt;
      L1.grid_x = (n4 + bt - 1) / bt;
      L1.grid_y = chunks;
      st.launches.push_back(L1);
      if (chunks > 1) {
        std::string fn2 = KName();
        k << "extern \"C\" __global__ void __launch_bounds__(256) " << fn2 << "(const void* __restrict__ p0, void* __restrict__ q0) {\n"
          << "  const float* part = (const float*)p0;\n  " << MemType(odt) << "* out0 = (" << MemType(odt) << "*)q0;\n"
          << "  const int lane = threadIdx.x & 31;\n"
          << "  for (long long o = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); o < " << n_out << "LL; o += (long long)gridDim.x * 8) {\n"
          << "    " << acc_t << " acc = " << ident << ";\n"
          << "#pragma unroll 4\n"
          << "    for (int c = lane; c < " << chunks << "; c += 32) acc = " << combine("acc", "part[(long long)c * " + std::to_string(n_out) + "LL + o]") << ";\n"
          << "  " << shfl_red
          << "    if (lane == 0) out0[o] = " << StoreExpr(odt, FromAcc(odt, combine(init_expr, "acc"))) << ";\n  }\n}\n";
        Launch L2;
        L2.fn = fn2;
        L2.in_slots = {scratch};
        L2.out_slots = {out_slot};
        L2.block = 256;
        L2.grid_x = std::max<int64_t>(1, (n_out + 7) / 8);
        L2.grid_stride = true;
        st.launches.push_back(L2);
        RecordDt(scratch, DT::kF32);
      }
    } else {
      // thread per output, reduced range split over `chunks` blocks in y; partials to scratch, then
      // a second kernel combines the chunks.  The output index space is the kept dims in order.
      int64_t chunks = 1;
      int64_t want_threads = 148LL * 2048;
      if (n_out < want_threads && L > 64) chunks = std::min<int64_t>((want_threads + n_out - 1) / n_out, std::max<int64_t>(1, L / 32));
      chunks = std::max<int64_t>(1, std::min<int64_t>(chunks, 1024));
      int64_t per = (L + chunks - 1) / chunks;
      gen.indent = "      ";
      std::ostringstream ob;
      auto names_k = Delinearize(ob, "o", kept, "a", "    ", wide);
      std::ostringstream inner_pre;
      auto names_r = Delinearize(inner_pre, "j", red, "b", "      ", wide);
      std::vector<std::string> idx(xd.size());
      for (size_t q = 0; q < kept_ax.size(); ++q) idx[kept_ax[q]] = names_k[q];
      for (size_t q = 0; q < red_ax.size(); ++q) idx[red_ax[q]] = names_r[q];
      gen.body << inner_pre.str();
      std::string v = gen.Emit(x, idx);
      std::vector<DT> in_dts;
      for (int s : gen.in_slots) in_dts.push_back(SlotDt(s));
      int scratch = -1;
      if (chunks > 1) scratch = NewSlot(chunks * n_out * DTBytes(acc_dt));
      k << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "("
        << KernelParams(gen.in_slots, 1, chunks > 1) << ") {\n" << ParamCasts(gen.in_slots, in_dts, {odt})
        << "  long long o = (long long)blockIdx.x * 256 + threadIdx.x;\n  if (o >= " << n_out << "LL) return;\n"
        << ob.str() << "  " << acc_t << " acc = " << (chunks > 1 ? "(" + acc_t + ")(" + IdentityOf(kind, acc_dt) + ")" : init_expr) << ";\n"
        << "    long long j0 = (long long)blockIdx.y * " << per << "LL;\n"
        << "    long long j1 = j0 + " << per << "LL < " << L << "LL ? j0 + " << per << "LL : " << L << "LL;\n"
        << "#pragma unroll 4\n    for (long long j = j0; j < j1; ++j) {\n"
        << gen.body.str() << "      acc = " << combine("acc", "(" + acc_t + ")(" + v + ")") << ";\n    }\n";
      if (chunks > 1) k << "  ((" << acc_t << "*)scratch)[(long long)blockIdx.y * " << n_out << "LL + o] = acc;\n}\n";
      else k << "  out0[o] = " << StoreExpr(odt, FromAcc(odt, "acc")) << ";\n}\n";
      Launch L1;
      L1.fn = fn;
      L1.in_slots = gen.in_slots;
      L1.out_slots = chunks > 1 ? std::vector<int>{} : std::vector<int>{out_slot};
      L1.scratch = scratch;
      L1.block = 256;
      L1.grid_x = (n_out + 255) / 256;
      L1.grid_y = chunks;
      if (chunks > 1) {
        // stage 1 writes no output; patch signature: it declares one output param q0, pass scratch as q0 too
        L1.out_slots = {scratch};
      }
      st.launches.push_back(L1);
      if (chunks > 1) {
        std::string fn2 = KName();
        // second pass: a warp per output, its lanes striding over the chunk partials (independent
        // loads in flight), then a shuffle tree; one thread per output would wait out one L2
        // round trip per chunk
        k << "extern \"C\" __global__ void __launch_bounds__(256) " << fn2 << "(const void* __restrict__ p0, void* __restrict__ q0) {\n"
          << "  const " << acc_t << "* part = (const " << acc_t << "*)p0;\n  " << MemType(odt) << "* out0 = (" << MemType(odt) << "*)q0;\n"
          << "  const int lane = threadIdx.x & 31;\n"
          << "  for (long long o = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); o < " << n_out << "LL; o += (long long)gridDim.x * 8) {\n"
          << "    " << acc_t << " acc = (" << acc_t << ")(" << IdentityOf(kind, acc_dt) << ");\n"
          << "#pragma unroll 4\n"
          << "    for (int c = lane; c < " << chunks << "; c += 32) acc = " << combine("acc", "part[(long long)c * " + std::to_string(n_out) + "LL + o]") << ";\n"
          << "  " << shfl_red
          << "    if (lane == 0) out0[o] = " << StoreExpr(odt, FromAcc(odt, combine(init_expr, "acc"))) << ";\n  }\n}\n";
        Launch L2;
        L2.fn = fn2;
        L2.in_slots = {scratch};
        L2.out_slots = {out_slot};
        L2.block = 256;
        L2.grid_x = std::max<int64_t>(1, (n_out + 7) / 8);
        L2.grid_stride = true;
        st.launches.push_back(L2);
        RecordDt(scratch, acc_dt);
      }
    }
    src_ << k.str();
    EndKernel();
    RecordDt(out_slot, odt);
    p_->steps.push_back(st);
  }

  static std::string IdentityOf(ReduceKind k, DT t) {
    bool f = DTIsFloat(t);
    switch (k) {
      case ReduceKind::kAdd: return "0";
      case ReduceKind::kMul: return "1";
      case ReduceKind::kMax: return f ? "-__int_as_float(0x7f800000)" : (t == DT::kS64 ? "(-9223372036854775807LL-1)" : DTIsUnsigned(t) ? "0" : "(-2147483647-1)");
      case ReduceKind::kMin: return f ? "__int_as_float(0x7f800000)" : (t == DT::kS64 ? "9223372036854775807LL" : DTIsUnsigned(t) ? "0xffffffffu" : "2147483647");
      case ReduceKind::kAnd: return t == DT::kPred ? "true" : "-1";
      case ReduceKind::kOr: return t == DT::kPred ? "false" : "0";
      default: return "0";
    }
  }

  // ---------------------------------------------------------------- dot_general
  // Materialises `v` permuted by `perm` (and optionally converted) into a new slot.
  // A permutation that moves the innermost dim: 32 x 32 tiles through shared memory so both the
  // reads (along the source's innermost dim) and the writes (along the output's) are coalesced.
  // Output dim q holds the source's innermost dim; the output's innermost dim is source dim perm[r-1].
  void EmitTiledTranspose(const Value* v, const std::vector<int>& perm, const std::vector<int64_t>& od, DT out_dt,
                          int64_t pitch, int src, int dst) {
    const int r = (int)perm.size();
    const auto& sd = v->type.dims;
    std::vector<int64_t> sstr(r, 1), ostr(r, 1);
    for (int k = r - 2; k >= 0; --k) sstr[k] = sstr[k + 1] * sd[k + 1];
    ostr[r - 1] = 1;
    if (r >= 2) ostr[r - 2] = pitch;
    for (int k = r - 3; k >= 0; --k) ostr[k] = ostr[k + 1] * od[k + 1];
    int q = 0;
    for (int k = 0; k < r; ++k) if (perm[k] == r - 1) q = k;
    const int64_t A = od[q], Bn = od[r - 1];
    const int64_t S_in = sstr[perm[r - 1]];      // source stride of the output's innermost dim
    const int64_t O_q = ostr[q];                 // output stride of dim q
    std::vector<int> rest_dims;
    int64_t R = 1;
    for (int k = 0; k < r; ++k)
      if (k != q && k != r - 1) { rest_dims.push_back(k); R *= od[k]; }
    DT in_dt = StoredDt(v);
    std::string fn = KName();
    std::ostringstream o;
    o << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(const void* __restrict__ p0, void* __restrict__ q0) {\n"
      << "  const " << MemType(in_dt) << "* __restrict__ in0 = (const " << MemType(in_dt) << "*)p0;\n"
      << "  " << MemType(out_dt) << "* __restrict__ out0 = (" << MemType(out_dt) << "*)q0;\n"
      << "  __shared__ " << CType(in_dt) << " tile[32][33];\n"
      << "  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;\n"
      << "  const long long a0 = (long long)blockIdx.y * 32, b0 = (long long)blockIdx.x * 32;\n"
      << "  for (long long rr = blockIdx.z; rr < " << R << "LL; rr += gridDim.z) {\n"
      << "    long long rem = rr, soff = 0, ooff = 0;\n";
    for (int k = (int)rest_dims.size() - 1; k >= 0; --k) {
      int d = rest_dims[k];
      o << "    { long long ix = rem % " << od[d] << "LL; rem /= " << od[d] << "LL; soff += ix * " << sstr[perm[d]]
        << "LL; ooff += ix * " << ostr[d] << "LL; }\n";
    }
    o << "#pragma unroll\n    for (int j = 0; j < 4; ++j) {\n"
      << "      const long long a = a0 + tx, bb = b0 + ty + 8 * j;\n"
      << "      if (a < " << A << "LL && bb < " << Bn << "LL) tile[ty + 8 * j][tx] = " << LoadExpr(in_dt, "in0", "soff + a + bb * " + std::to_string(S_in) + "LL") << ";\n"
      << "    }\n    __syncthreads();\n"
      << "#pragma unroll\n    for (int j = 0; j < 4; ++j) {\n"
      << "      const long long bb = b0 + tx, a = a0 + ty + 8 * j;\n"
      << "      if (a < " << A << "LL && bb < " << Bn << "LL) out0[ooff + a * " << O_q << "LL + bb] = " << StoreExpr(out_dt, "tile[tx][ty + 8 * j]") << ";\n"
      << "    }\n    __syncthreads();\n  }\n}\n";
    src_ << o.str();
    EndKernel();
    Launch L;
    L.fn = fn;
    L.in_slots = {src};
    L.out_slots = {dst};
    L.block = 256;
    L.grid_x = (Bn + 31) / 32;
    L.grid_y = (A + 31) / 32;
    L.grid_z = std::max<int64_t>(1, std::min<int64_t>(R, 65535));
    Step st;
    st.kind = StepKind::kFusion;
    st.launches.push_back(L);
    st.label = "transpose " + v->type.str();
    p_->steps.push_back(st);
    RecordDt(dst, out_dt);
  }

  // Materialises `v` permuted by `perm` (and converted to out_dt) into a new slot.  With
  // `inner_pitch` > 0 the innermost dim is stored with that row pitch (elements), leaving the pad
  // columns unwritten: used to give TMA a 16-byte-aligned row stride.
  int EmitPermute(const Value* v, const std::vector<int>& perm, const std::vector<int64_t>& out_dims, DT out_dt,
                  int64_t inner_pitch = 0) {
    int src = SlotFor(v);
    int64_t n = 1;
    for (int64_t d : out_dims) n *= d;
    const int64_t inner = out_dims.empty() ? 1 : out_dims.back();
    const int64_t pitch = inner_pitch > 0 ? inner_pitch : inner;
    int dst = NewSlot(n / std::max<int64_t>(inner, 1) * pitch * DTBytes(out_dt));
    const int rank = (int)perm.size();
    if (rank >= 2 && perm.back() != rank - 1 && n > 0) {
      EmitTiledTranspose(v, perm, out_dims, out_dt, pitch, src, dst);
      return dst;
    }
    std::ostringstream body;
    auto names = Delinearize(body, "i", out_dims, "i", "    ", n >= (1LL << 31));
    // out index k corresponds to source dim perm[k]
    std::vector<std::string> sidx(v->type.rank());
    for (size_t k = 0; k < perm.size(); ++k) sidx[perm[k]] = names[k];
    std::string fn = KName();
    DT in_dt = StoredDt(v);
    std::string oidx = pitch == inner ? "i" : "(i / " + std::to_string(inner) + "LL) * " + std::to_string(pitch) +
                                                 "LL + i % " + std::to_string(inner) + "LL";
    src_ << "extern \"C\" __global__ void __launch_bounds__(256) " << fn << "(const void* __restrict__ p0, void* __restrict__ q0) {\n"
         << "  const " << MemType(in_dt) << "* in0 = (const " << MemType(in_dt) << "*)p0;\n"
         << "  " << MemType(out_dt) << "* out0 = (" << MemType(out_dt) << "*)q0;\n"
         << "  for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < " << n << "LL; i += (long long)gridDim.x * 256) {\n"
         << body.str() << "    out0[" << oidx << "] = " << StoreExpr(out_dt, LoadExpr(in_dt, "in0", Gen::Linear(sidx, v->type.dims))) << ";\n  }\n}\n";
    EndKernel();
    Launch L;
    L.fn = fn;
    L.in_slots = {src};
    L.out_slots = {dst};
    L.grid_x = std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16));
    Step st;
    st.kind = StepKind::kFusion;
    st.launches.push_back(L);
    st.label = "transpose " + v->type.str();
    p_->steps.push_back(st);
    RecordDt(dst, out_dt);
    return dst;
  }

  void EmitDot(Op* op) {
    const Value* a = op->operands[0];
    const Value* b = op->operands[1];
    Value* r = op->result();
    auto get = [&](const char* k) { auto it = op->ints.find(k); return it == op->ints.end() ? std::vector<int64_t>{} : it->second; };
    std::vector<int64_t> lb = get("batching_dims.lhs"), rb = get("batching_dims.rhs");
    std::vector<int64_t> lc = get("contracting_dims.lhs"), rc = get("contracting_dims.rhs");
    if (op->name == "dot") { lc = {a->type.rank() - 1}; rc = {0}; }
    std::vector<int64_t> lf, rf;
    for (int k = 0; k < a->type.rank(); ++k)
      if (std::find(lb.begin(), lb.end(), k) == lb.end() && std::find(lc.begin(), lc.end(), k) == lc.end()) lf.push_back(k);
    for (int k = 0; k < b->type.rank(); ++k)
      if (std::find(rb.begin(), rb.end(), k) == rb.end() && std::find(rc.begin(), rc.end(), k) == rc.end()) rf.push_back(k);
    auto prod = [](const Value* v, const std::vector<int64_t>& ax) { int64_t p = 1; for (int64_t k : ax) p *= v->type.dims[k]; return p; };
    GemmStep g;
    g.batch = prod(a, lb);
    g.M = prod(a, lf);
    g.N = prod(b, rf);
    g.K = prod(a, lc);
    DT at = StoredDt(a), bt = StoredDt(b);
    if (!DTIsFloat(at) || !DTIsFloat(bt)) throw LowerError{"dot_general on non-float operands is not supported"};
    if (at == DT::kF64 || bt == DT::kF64) throw LowerError{"dot_general on f64 operands is not supported"};
    g.out = r->type.dt;
    if (g.out != DT::kF32 && g.out != DT::kBF16 && g.out != DT::kF16) throw LowerError{"dot_general result type not supported"};
    // Arithmetic of the GEMM:
    //  * two 16-bit operands: the tensor cores in that type (bf16 for a bf16 x f16 pair);
    //  * an f32 operand with an f32 result: f32-accurate, each f32 operand split into three bf16
    //    pieces on the tensor cores (b200k::GemmSplit) -- f32 x f32 when it is large enough to
    //    gain from that, else the SIMT f32 kernel;
    //  * an f32 operand with a 16-bit result and a 16-bit other operand (the cotangent of an f32 dot
    //    result meeting bf16 weights in a backward pass): the f32 operand is rounded to the 16-bit
    //    type once, an error of the size of the result's own rounding; B200_DOT_MIXED_F32=1 makes
    //    these f32-accurate too.
    auto wide = [](DT t) { return t == DT::kF32; };
    DT ab;
    bool split = false;
    if (!wide(at) && !wide(bt)) {
      ab = at == bt ? at : DT::kBF16;
    } else if (wide(at) && wide(bt)) {
      ab = DT::kF32;
      split = (double)prod(a, lb) * prod(a, lf) * prod(b, rf) * prod(a, lc) >= (double)(1LL << 26) &&
              !std::getenv("B200_GEMM_F32_SIMT");
    } else if (g.out == DT::kF32 || std::getenv("B200_DOT_MIXED_F32")) {
      ab = DT::kF32;
      split = true;
    } else {
      ab = wide(at) ? bt : at;
    }
    g.ab = ab;
    g.split = split;
    // Each operand is used where it lies when its dims are [batch, rows, K] (K-major) or [batch, K,
    // rows] (MN-major) in order; otherwise it is copied K-major.  The tensor cores read either form
    // through TMA, which needs 16-byte row strides: rows % 8 == 0 for MN-major, and a 16-bit K-major
    // copy with K % 8 != 0 gets a padded pitch.
    const bool tc = ab != DT::kF32;
    struct Opnd { int slot; bool mn; int64_t ld; DT dt; };
    auto identity = [](const std::vector<int64_t>& o) {
      for (size_t k = 0; k < o.size(); ++k) if (o[k] != (int64_t)k) return false;
      return true;
    };
    auto cat = [](std::vector<int64_t> x, const std::vector<int64_t>& y, const std::vector<int64_t>& z) {
      x.insert(x.end(), y.begin(), y.end());
      x.insert(x.end(), z.begin(), z.end());
      return x;
    };
    auto operand = [&](const Value* v, const std::vector<int64_t>& bat, const std::vector<int64_t>& fr,
                       const std::vector<int64_t>& ct, int64_t rows) -> Opnd {
      const std::vector<int64_t> kord = cat(bat, fr, ct), mord = cat(bat, ct, fr);
      const DT held = StoredDt(v);
      if (const int64_t p = StoredPitch(v)) {      // stored with a padded pitch for exactly this use
        const std::vector<int64_t> last{v->type.rank() - 1};
        if (identity(kord) && ct == last) return {SlotFor(v), false, p, held};
        if (identity(mord) && fr == last) return {SlotFor(v), true, p, held};
        throw LowerError{"internal: padded operand used out of place"};
      }
      if (split) {
        // the split kernel reads either form in its stored type (f32 / bf16 / f16)
        if (identity(kord)) return {SlotFor(v), false, g.K, held};
        if (identity(mord)) return {SlotFor(v), true, rows, held};
        std::vector<int> perm(kord.begin(), kord.end());
        std::vector<int64_t> od;
        for (int q : perm) od.push_back(v->type.dims[q]);
        return {EmitPermute(v, perm, od, held), false, g.K, held};
      }
      if (identity(kord) && held == ab && !(tc && g.K % 8)) return {SlotFor(v), false, g.K, held};
      if (identity(mord) && (!tc || rows % 8 == 0) && !std::getenv("B200_GEMM_NO_MN")) {
        if (held == ab) return {SlotFor(v), true, rows, held};
        std::vector<int> same(v->type.rank());
        for (int k = 0; k < v->type.rank(); ++k) same[k] = k;
        return {EmitPermute(v, same, v->type.dims, ab), true, rows, ab};   // convert only
      }
      const int64_t pitch = (tc && g.K % 8 != 0) ? (g.K + 7) / 8 * 8 : 0;
      std::vector<int> perm(kord.begin(), kord.end());
      std::vector<int64_t> od;
      for (int q : perm) od.push_back(v->type.dims[q]);
      return {EmitPermute(v, perm, od, ab, pitch), false, pitch ? pitch : g.K, ab};
    };
    Opnd oa = operand(a, lb, lf, lc, g.M), ob = operand(b, rb, rf, rc, g.N);
    g.a = oa.slot;
    g.a_mn = oa.mn;
    g.lda = oa.ld;
    g.b = ob.slot;
    g.b_mn = ob.mn;
    g.ldb = ob.ld;
    g.a_dt = oa.dt;
    g.b_dt = ob.dt;
    const bool split_k = tc && g.out != DT::kF32 && !StoredPitch(r) && b200k::GemmSplitK(g.batch, g.M, g.N, g.K, 148) > 1;
    if (split_k && PromotableToF32(r)) {         // readers round the f32 partial sums themselves
      promote_.insert(r->id);
      g.out = DT::kF32;
    }
    g.c = SlotFor(r);
    g.ldc = StoredPitch(r);                      // 0: dense rows of N
    if (split_k && g.out != DT::kF32) {
      g.ws = NewSlot(g.batch * g.M * g.N * 4);   // split-K partial sums
      RecordDt(g.ws, DT::kF32);
    }
    if (split) {                                 // bf16 pieces of the f32 operands
      const size_t bytes = b200k::GemmSplitScratchBytes(g.batch, g.M, g.N, g.K, KernelTypeCode(g.a_dt), KernelTypeCode(g.b_dt),
                                                        g.a_mn, g.b_mn, g.lda, g.ldb);
      if (bytes) {
        g.split_ws = NewSlot((int64_t)bytes);
        g.split_ws_bytes = (int64_t)bytes;
        RecordDt(g.split_ws, DT::kBF16);
      }
    }
    Step st;
    st.kind = StepKind::kGemm;
    st.gemm = g;
    st.label = "gemm b" + std::to_string(g.batch) + " " + std::to_string(g.M) + "x" + std::to_string(g.N) + "x" + std::to_string(g.K) +
               (g.a_mn || g.b_mn ? std::string(" ") + (g.a_mn ? "m" : "k") + (g.b_mn ? "n" : "k") : "") +
               (g.split ? " f32-split" : g.ab == DT::kF32 ? " f32-simt" : "");
    p_->steps.push_back(st);
    RecordDt(g.c, StoredDt(r));
  }

  void EmitAttention(Op* d2) {
    AttentionStep a = attn_.at(d2->result()->id);
    auto ins = attn_in_.at(d2->result()->id);
    a.q = SlotFor(ins[0]);
    a.k = SlotFor(ins[1]);
    a.v = SlotFor(ins[2]);
    a.o = SlotFor(d2->result());
    a.dt = DT::kBF16;
    auto lf = lse_for_.find(d2->result()->id);
    if (lf != lse_for_.end()) {                  // training: the backward needs lse2
      a.lse = NewSlot((int64_t)a.B * a.H * a.S * 4);
      lf->second = a.lse;
      RecordDt(a.lse, DT::kF32);
    }
    Step st;
    st.kind = StepKind::kAttention;
    st.attn = a;
    st.label = std::string("attention ") + (a.causal ? "causal " : "") + (a.lse >= 0 ? "+lse " : "") + ins[0]->type.str();
    p_->steps.push_back(st);
    RecordDt(a.o, DT::kBF16);
  }

  void EmitAttentionBwd(const BwdMatch& m) {
    const AttentionStep& a = attn_.at(m.d2);
    AttentionBwdStep b;
    b.B = a.B;
    b.H = a.H;
    b.S = a.S;
    b.D = a.D;
    b.causal = a.causal;
    b.scale = a.scale;
    b.q = SlotFor(m.Q);
    b.k = SlotFor(m.K);
    b.v = SlotFor(m.V);
    b.o = SlotFor(m.O);
    b.dout = SlotFor(m.G);
    b.lse = lse_for_.at(m.d2);
    if (b.lse < 0) throw LowerError{"internal: attention backward before its forward"};
    const bool dq_f32 = PromotableToF32(m.dq);   // readers round dQ from its f32 accumulator
    if (dq_f32) promote_.insert(m.dq->id);
    b.dq = dq_f32 ? -1 : SlotFor(m.dq);
    b.dk = SlotFor(m.dk);
    b.dv = SlotFor(m.dv);
    const int64_t rows = (int64_t)a.B * a.H * a.S;
    b.dq_acc = dq_f32 ? SlotFor(m.dq) : NewSlot(rows * a.D * 4);
    b.delta = NewSlot(rows * 4);
    b.dk_t = m.dk_t;                             // the kernel writes dK in the dot's [B, H, D, S] layout
    for (int s : {b.dq, b.dk, b.dv}) if (s >= 0) RecordDt(s, DT::kBF16);
    for (int s : {b.dq_acc, b.delta}) RecordDt(s, DT::kF32);
    Step st;
    st.kind = StepKind::kAttentionBwd;
    st.bwd = b;
    st.label = std::string("attention_bwd ") + (a.causal ? "causal " : "") + m.Q->type.str();
    p_->steps.push_back(st);
  }

  // ---------------------------------------------------------------- scatter (embedding VJP)
  void EmitScatter(Op* op) {
    if (op->operands.size() != 3 || op->reduce != ReduceKind::kAdd)
      throw LowerError{"unsupported scatter (only scatter-add of rows is supported)"};
    const Value* base = op->operands[0];
    const Value* idx = op->operands[1];
    const Value* upd = op->operands[2];
    auto get = [&](const char* k) { auto it = op->ints.find(k); return it == op->ints.end() ? std::vector<int64_t>{} : it->second; };
    if (base->type.rank() != 2 || get("inserted_window_dims") != std::vector<int64_t>{0} ||
        get("scatter_dims_to_operand_dims") != std::vector<int64_t>{0} || idx->type.dims.back() != 1 ||
        get("update_window_dims") != std::vector<int64_t>{upd->type.rank() - 1})
      throw LowerError{"unsupported scatter form (only row scatter-add along dim 0)"};
    ScatterStep s;
    s.rows = base->type.dims[0];
    s.row_len = base->type.dims[1];
    s.n_upd = upd->type.numel() / s.row_len;
    s.dt = base->type.dt;
    s.idx_dt = idx->type.dt;
    if (s.dt != DT::kF32 && s.dt != DT::kBF16) throw LowerError{"scatter-add supports f32 / bf16 rows"};
    if (s.idx_dt != DT::kS32 && s.idx_dt != DT::kS64) throw LowerError{"scatter indices must be s32/s64"};
    s.base = SlotFor(base);
    s.idx = SlotFor(idx);
    s.upd = SlotFor(upd);
    s.out = SlotFor(op->result());
    Step st;
    st.kind = StepKind::kScatterAdd;
    st.scatter = s;
    st.label = "scatter_add " + base->type.str();
    p_->steps.push_back(st);
    RecordDt(s.out, s.dt);
  }

  // ---------------------------------------------------------------- collectives
  void EmitCollective(Op* op) {
    const Value* x = op->operands[0];
    Value* r = op->result();
    if (op->operands.size() != 1 || op->results.size() != 1) throw LowerError{"variadic collectives not yet supported"};
    const std::string& n = op->name;
    if (n != "all_reduce") {
      const char* key = n == "all_gather" ? "all_gather_dim" : "scatter_dimension";
      auto it = op->ints.find(key);
      if (it != op->ints.end() && !it->second.empty() && it->second[0] != 0)
        throw LowerError{n + " only supported along dim 0"};
    }
    // Across processes the communicator spans every rank in rank order, so the program's replica
    // groups must be that one group (a jax shard_map over all devices writes it so); other groupings
    // would need sub-communicators and are a compile error rather than a silently world-wide
    // collective.  At one process every collective is the identity, as in the reference.
    if (opt_.num_processes > 1) {
      auto g = op->ints.find("replica_groups");
      auto gc = op->ints.find("replica_groups.count");
      if (g != op->ints.end() && !g->second.empty()) {
        const int64_t count = gc == op->ints.end() || gc->second.empty() ? -1 : gc->second[0];
        bool ok = (int64_t)g->second.size() == opt_.num_processes && (count == 1 || count == -1);
        for (size_t k = 0; ok && k < g->second.size(); ++k) ok = g->second[k] == (int64_t)k;
        if (!ok) throw LowerError{n + ": replica_groups other than one group of all " + std::to_string(opt_.num_processes) +
                                  " ranks in rank order are not supported"};
      }
    }
    if (opt_.num_processes <= 1 && x->type.dims == r->type.dims) {
      // one rank: identity (the reference does the same, src/jam/lower.mm:346-352)
      slot_of_[r->id] = SlotFor(x);
      return;
    }
    CollectiveStep c;
    c.op = n == "all_reduce" ? CollKind::kAllReduce : n == "all_gather" ? CollKind::kAllGather : CollKind::kReduceScatter;
    c.reduce = op->reduce == ReduceKind::kNone ? ReduceKind::kAdd : op->reduce;
    if (c.op != CollKind::kAllGather && op->reduce == ReduceKind::kNone)
      throw LowerError{n + " reducer is not a recognized add/max/min/multiply"};
    c.in = SlotFor(x);
    c.out = SlotFor(r);
    c.send_count = x->type.numel();
    c.recv_count = r->type.numel();
    c.dt = x->type.dt;
    Step st;
    st.kind = StepKind::kCollective;
    st.coll = c;
    st.label = n + " " + x->type.str();
    p_->steps.push_back(st);
    RecordDt(c.out, c.dt);
  }

  // ---------------------------------------------------------------- horizontal fusion
  static void StepRW(const Step& S, std::set<int>* r, std::set<int>* w) {
    auto R = [&](std::initializer_list<int> l) { for (int x : l) if (x >= 0) r->insert(x); };
    auto W = [&](std::initializer_list<int> l) { for (int x : l) if (x >= 0) w->insert(x); };
    switch (S.kind) {
      case StepKind::kFusion:
        for (const Launch& L : S.launches) {
          for (int x : L.in_slots) R({x});
          for (int x : L.out_slots) W({x});
          W({L.scratch});
        }
        break;
      case StepKind::kGemm: R({S.gemm.a, S.gemm.b}); W({S.gemm.c, S.gemm.ws, S.gemm.split_ws}); break;
      case StepKind::kAttention: R({S.attn.q, S.attn.k, S.attn.v}); W({S.attn.o, S.attn.lse}); break;
      case StepKind::kAttentionBwd:
        R({S.bwd.q, S.bwd.k, S.bwd.v, S.bwd.o, S.bwd.dout, S.bwd.lse});
        W({S.bwd.dq, S.bwd.dk, S.bwd.dv, S.bwd.dq_acc, S.bwd.delta});
        break;
      case StepKind::kScatterAdd: R({S.scatter.base, S.scatter.idx, S.scatter.upd}); W({S.scatter.out}); break;
      case StepKind::kCollective:
        R({S.coll.in});
        W({S.coll.out});
        for (int x : S.coll.packed_in) R({x});
        for (int x : S.coll.packed_out) W({x});
        break;
      case StepKind::kCopy: R({S.copy.src}); W({S.copy.dst}); break;
    }
  }
  bool TinyLoop(const Step& S) const {
    if (S.kind != StepKind::kFusion || S.launches.size() != 1 || S.label.compare(0, 5, "loop ") != 0) return false;
    const Launch& L = S.launches[0];
    return L.block == 256 && L.grid_y == 1 && L.grid_z == 1 && L.scratch < 0 && L.smem == 0 && L.grid_x <= 4;
  }
  // Loop kernels of at most four CTAs (the optimizer updates of biases and LayerNorm parameters)
  // that do not depend on each other, nor on the steps they are moved across, run as one launch:
  // each becomes a device function taking its CTA index and count, and one kernel dispatches its
  // CTAs to them by range.
  void MergeTinyLoops() {
    if (std::getenv("B200_NO_HMERGE")) return;
    std::vector<Step>& steps = p_->steps;
    std::vector<Step> out;
    std::vector<bool> taken(steps.size(), false);
    for (size_t i = 0; i < steps.size(); ++i) {
      if (taken[i]) continue;
      if (!TinyLoop(steps[i])) { out.push_back(steps[i]); continue; }
      std::vector<size_t> group{i};
      std::set<int> gr, gw, br, bw;           // group reads / writes, steps passed over
      StepRW(steps[i], &gr, &gw);
      size_t params = steps[i].launches[0].in_slots.size() + steps[i].launches[0].out_slots.size();
      for (size_t j = i + 1; j < steps.size() && j < i + 96 && group.size() < 24; ++j) {
        if (taken[j]) continue;
        std::set<int> r, w;
        StepRW(steps[j], &r, &w);
        auto meets = [](const std::set<int>& a, const std::set<int>& b) {
          for (int x : a) if (b.count(x)) return true;
          return false;
        };
        const size_t np = TinyLoop(steps[j]) ? steps[j].launches[0].in_slots.size() + steps[j].launches[0].out_slots.size() : 0;
        if (TinyLoop(steps[j]) && params + np <= 480 && !meets(r, bw) && !meets(w, br) && !meets(w, bw) && !meets(r, gw) &&
            !meets(w, gr) && !meets(w, gw)) {
          group.push_back(j);
          gr.insert(r.begin(), r.end());
          gw.insert(w.begin(), w.end());
          params += np;
          continue;
        }
        br.insert(r.begin(), r.end());
        bw.insert(w.begin(), w.end());
      }
      if (group.size() == 1) { out.push_back(steps[i]); continue; }
      for (size_t g : group) taken[g] = true;
      out.push_back(MergeLoopSteps(group));
    }
    steps = std::move(out);
  }
  Step MergeLoopSteps(const std::vector<size_t>& group) {
    std::vector<Step>& steps = p_->steps;
    const std::string fn = KName();
    std::ostringstream unit, wrap_params, body;
    Launch M;
    M.fn = fn;
    M.block = 256;
    M.grid_stride = false;
    int64_t base = 0;
    std::vector<std::string> in_args, out_args;
    for (size_t q = 0; q < group.size(); ++q) {
      const Launch& L = steps[group[q]].launches[0];
      // move the kernel's source unit, turned into a device function of (CTA index, CTA count)
      auto& ks = p_->kernel_sources;
      const std::string head = "extern \"C\" __global__ void __launch_bounds__(256, 4) " + L.fn + "(";
      size_t u = 0;
      while (u < ks.size() && ks[u].find(head) == std::string::npos) ++u;
      if (u == ks.size()) throw LowerError{"internal: kernel " + L.fn + " not found for merging"};
      std::string src = ks[u];
      ks.erase(ks.begin() + (long)u);
      const size_t at = src.find(head);
      const size_t open = src.find(") {\n", at);
      std::string kern = src.substr(at, open - at) + ", const unsigned hbx, const unsigned hgx" + src.substr(open);
      kern.replace(0, head.size() - L.fn.size() - 1, "static __device__ __forceinline__ void ");
      for (const char* from : {"blockIdx.x", "gridDim.x"}) {
        const std::string to = std::string(from) == "blockIdx.x" ? "hbx" : "hgx";
        for (size_t p = kern.find(from); p != std::string::npos; p = kern.find(from, p + to.size())) kern.replace(p, std::strlen(from), to);
      }
      unit << src.substr(0, at) << kern;
      std::vector<std::string> args;
      auto shared = [&](int slot, bool in) {
        for (auto& pr : L.inplace)
          if ((in ? pr.first : pr.second) == slot) return true;
        return false;
      };
      for (size_t k = 0; k < L.in_slots.size(); ++k) {
        const std::string a = "h" + std::to_string(q) + "p" + std::to_string(k);
        in_args.push_back((shared(L.in_slots[k], true) ? "const void* " : "const void* __restrict__ ") + a);
        args.push_back(a);
        M.in_slots.push_back(L.in_slots[k]);
      }
      for (size_t k = 0; k < L.out_slots.size(); ++k) {
        const std::string a = "h" + std::to_string(q) + "q" + std::to_string(k);
        out_args.push_back((shared(L.out_slots[k], false) ? "void* " : "void* __restrict__ ") + a);
        args.push_back(a);
        M.out_slots.push_back(L.out_slots[k]);
      }
      M.inplace.insert(M.inplace.end(), L.inplace.begin(), L.inplace.end());
      body << "  " << (q ? "else " : "") << "if (b < " << base + L.grid_x << "u) " << L.fn << "(";
      for (auto& a : args) body << a << ", ";
      body << "b - " << base << "u, " << L.grid_x << "u);\n";
      base += L.grid_x;
    }
    std::string plist;
    for (auto& a : in_args) plist += (plist.empty() ? "" : ", ") + a;
    for (auto& a : out_args) plist += (plist.empty() ? "" : ", ") + a;
    unit << "extern \"C\" __global__ void __launch_bounds__(256, 4) " << fn << "(" << plist << ") {\n"
         << "  const unsigned b = blockIdx.x;\n" << body.str() << "}\n";
    p_->kernel_sources.push_back(unit.str());
    M.grid_x = base;
    Step st;
    st.kind = StepKind::kFusion;
    st.launches.push_back(M);
    st.label = "loops x" + std::to_string(group.size()) + " (merged small kernels)";
    return st;
  }

  // ---------------------------------------------------------------- outputs
  void BindOutputs() {
    p_->out_slots.clear();
    p_->out_types.clear();
    std::set<int> used;
    for (Value* o : g_.outputs) {
      const Value* v = Resolve(o);
      int s = slot_of_[v->id];
      if (s < 0) s = slot_of_[o->id];
      if (s < 0) throw LowerError{"internal: output not materialized"};
      TensorType t = o->type;
      // shard_map outputs stay per-device shards (src/jam/lower.mm:290-298)
      if (o->def && IsAlias(o->def)) t.dims = v->type.dims, t = v->type;
      const Slot sl = p_->slots[s];   // by value: NewSlot below may reallocate the slot vector
      if (sl.arg_index >= 0 || sl.const_index >= 0 || used.count(s)) {
        int d = NewSlot(sl.bytes);
        Step st;
        st.kind = StepKind::kCopy;
        st.copy.src = s;
        st.copy.dst = d;
        st.copy.bytes = sl.bytes;
        st.label = "copy output";
        p_->steps.push_back(st);
        s = d;
      }
      used.insert(s);
      p_->slots[s].output = true;
      p_->out_slots.push_back(s);
      p_->out_types.push_back(t);
    }
  }

  // slots a step reads
  static std::vector<int> StepReads(const Step& st) {
    std::vector<int> r;
    switch (st.kind) {
      case StepKind::kFusion:
        for (auto& L : st.launches) r.insert(r.end(), L.in_slots.begin(), L.in_slots.end());
        break;
      case StepKind::kGemm: r = {st.gemm.a, st.gemm.b}; break;
      case StepKind::kAttention: r = {st.attn.q, st.attn.k, st.attn.v}; break;
      case StepKind::kAttentionBwd: r = {st.bwd.q, st.bwd.k, st.bwd.v, st.bwd.o, st.bwd.dout, st.bwd.lse}; break;
      case StepKind::kScatterAdd: r = {st.scatter.base, st.scatter.idx, st.scatter.upd}; break;
      case StepKind::kCollective:
        r = {st.coll.in};
        r.insert(r.end(), st.coll.packed_in.begin(), st.coll.packed_in.end());
        break;
      case StepKind::kCopy: r = {st.copy.src}; break;
    }
    return r;
  }
  // Small all-reduces (at most 256 KiB each: bias, LayerNorm-parameter and loss gradients) are held
  // back from where hoisting put them and issued together, as one NCCL group, with the next large
  // collective, or just before the first step that needs one of their results or writes one of
  // their operands -- or when the held ones reach 4 MiB.  The reference buckets the same in-place
  // all-reduces of <= 256 KiB into one call through a packed buffer (src/jam/jam_run.mm:186-248);
  // an NCCL group does it without the packing copies.
  // B200_COLL_BUCKET=all holds every all-reduce, whatever its size, until a step needs one of their
  // results: the gradients of a train step then go to NCCL as one group after the backward pass,
  // instead of overlapping it (NCCL kernels then share no SMs with the backward's kernels).
  void GroupSmallCollectives() {
    if (opt_.num_processes <= 1 || std::getenv("B200_NO_COLL_GROUPS")) return;
    const char* bucket = std::getenv("B200_COLL_BUCKET");
    const bool all = bucket && std::strcmp(bucket, "all") == 0;
    const int64_t kSmall = all ? INT64_MAX : 256 << 10, kFlushBytes = all ? INT64_MAX : 4 << 20;
    std::vector<Step> out, held;
    std::set<int> held_out, held_in;
    int64_t held_bytes = 0;
    int next_group = 0;
    auto flush = [&]() {
      if (held.empty()) return;
      const int g = held.size() > 1 ? next_group++ : -1;
      for (Step& h : held) {
        h.coll.group = g;
        if (g >= 0) h.label += " [group " + std::to_string(g) + "]";
        out.push_back(std::move(h));
      }
      held.clear();
      held_out.clear();
      held_in.clear();
      held_bytes = 0;
    };
    for (Step& st : p_->steps) {
      const bool coll = st.kind == StepKind::kCollective;
      const int64_t bytes = coll ? st.coll.send_count * DTBytes(st.coll.dt) : 0;
      if (coll && st.coll.op == CollKind::kAllReduce && bytes <= kSmall) {
        held_out.insert(st.coll.out);
        held_in.insert(st.coll.in);
        held_bytes += bytes;
        held.push_back(std::move(st));
        if (held_bytes >= kFlushBytes) flush();
        continue;
      }
      if (coll) {
        // a large collective takes the held ones along in its group (their operands are older)
        held.push_back(std::move(st));
        flush();
        continue;
      }
      std::set<int> r, w;
      StepRW(st, &r, &w);
      bool conflict = false;
      for (int x : r) conflict = conflict || held_out.count(x);
      for (int x : w) conflict = conflict || held_in.count(x) || held_out.count(x);
      if (conflict) flush();
      out.push_back(std::move(st));
    }
    flush();
    p_->steps = std::move(out);
  }

  // A run of grouped all-reduces of one type and reduction becomes one all-reduce over a bucket:
  // each member's input and output slots live at the same offset inside the bucket (the producers
  // write straight into it, the reduction is in place, the readers read from it), so NCCL runs one
  // large operation instead of one per gradient (~20 us of latency each on NVLink).  A member
  // qualifies when nothing but its all-reduce reads its input, its output is not a program output,
  // and neither slot is an argument, a constant or row-padded.  B200_NO_PACK=1 turns this off.
  void PackAllReduces() {
    if (opt_.num_processes <= 1 || std::getenv("B200_NO_PACK")) return;
    std::vector<Step>& steps = p_->steps;
    std::vector<int> readers(p_->slots.size(), 0), writers(p_->slots.size(), 0);
    for (const Step& st : steps) {
      std::set<int> r, w;
      StepRW(st, &r, &w);
      for (int x : r) ++readers[x];
      for (int x : w) ++writers[x];
    }
    auto plain = [&](int s) {
      const Slot& sl = p_->slots[s];
      return sl.arg_index < 0 && sl.const_index < 0 && !sl.output && sl.alias_of < 0 && !slot_pitch_.count(s);
    };
    std::vector<Step> out;
    for (size_t i = 0; i < steps.size();) {
      if (steps[i].kind != StepKind::kCollective || steps[i].coll.group < 0) { out.push_back(std::move(steps[i++])); continue; }
      size_t j = i;
      while (j < steps.size() && steps[j].kind == StepKind::kCollective && steps[j].coll.group == steps[i].coll.group) ++j;
      // members by (type, reduction)
      std::map<std::pair<int, int>, std::vector<size_t>> by_kind;
      for (size_t k = i; k < j; ++k) {
        const CollectiveStep& c = steps[k].coll;
        if (c.op != CollKind::kAllReduce || c.in == c.out || !plain(c.in) || !plain(c.out)) continue;
        if (readers[c.in] != 1 || writers[c.out] != 1 || p_->slots[c.in].bytes != p_->slots[c.out].bytes) continue;
        by_kind[{(int)c.dt, (int)c.reduce}].push_back(k);
      }
      std::vector<bool> packed(j - i, false);
      std::vector<Step> buckets;
      for (auto& kv : by_kind) {
        if (kv.second.size() < 2) continue;
        int64_t total = 0;
        for (size_t k : kv.second) total += (p_->slots[steps[k].coll.in].bytes + 255) / 256 * 256;
        const int bucket = NewSlot(total);
        Step b;
        b.kind = StepKind::kCollective;
        b.coll = steps[kv.second[0]].coll;
        b.coll.in = b.coll.out = bucket;
        b.coll.packed_in.clear();
        b.coll.packed_out.clear();
        int64_t off = 0;
        for (size_t k : kv.second) {
          const CollectiveStep& c = steps[k].coll;
          for (int x : {c.in, c.out}) {
            p_->slots[x].alias_of = bucket;
            p_->slots[x].alias_off = off;
          }
          b.coll.packed_in.push_back(c.in);
          b.coll.packed_out.push_back(c.out);
          off += (p_->slots[c.in].bytes + 255) / 256 * 256;
          packed[k - i] = true;
        }
        const int64_t esz = DTBytes(b.coll.dt);
        b.coll.send_count = b.coll.recv_count = total / esz;
        b.label = "all_reduce packed x" + std::to_string(kv.second.size()) + " (" + std::to_string(total) + " bytes)" +
                  (b.coll.group >= 0 ? " [group " + std::to_string(b.coll.group) + "]" : "");
        buckets.push_back(std::move(b));
      }
      for (size_t k = i; k < j; ++k)
        if (!packed[k - i]) out.push_back(std::move(steps[k]));
      for (Step& b : buckets) out.push_back(std::move(b));
      i = j;
    }
    steps = std::move(out);
  }

  // Collectives of a multi-process program run on the communication stream; the first step that
  // reads a collective's result waits for it (later readers are ordered behind that step).
  std::vector<int> coll_until_;   // step index -> step that waits for it (async collectives)
  void MarkAsyncCollectives() {
    coll_until_.assign(p_->steps.size(), -1);
    if (opt_.num_processes <= 1 || std::getenv("B200_SYNC_COLLECTIVES")) return;
    for (int k = 0; k < (int)p_->steps.size(); ++k) {
      Step& c = p_->steps[k];
      if (c.kind != StepKind::kCollective) continue;
      c.async = true;
      for (int j = k + 1; j < (int)p_->steps.size(); ++j) {
        const std::vector<int> rd = StepReads(p_->steps[j]);
        bool reads = std::find(rd.begin(), rd.end(), c.coll.out) != rd.end();
        for (int x : c.coll.packed_out) reads = reads || std::find(rd.begin(), rd.end(), x) != rd.end();
        if (reads) {
          p_->steps[j].wait_coll.push_back(k);
          coll_until_[k] = j;
          break;
        }
      }
      if (coll_until_[k] < 0) coll_until_[k] = (int)p_->steps.size() - 1;   // waited for at the end
    }
  }

  void ComputeLastUse() {
    auto touch = [&](int s, int i) { if (s >= 0) p_->slots[s].last_use = std::max(p_->slots[s].last_use, i); };
    for (int i = 0; i < (int)p_->steps.size(); ++i) {
      const Step& st = p_->steps[i];
      switch (st.kind) {
        case StepKind::kFusion:
          for (auto& L : st.launches) {
            for (int s : L.in_slots) touch(s, i);
            for (int s : L.out_slots) touch(s, i);
            touch(L.scratch, i);
          }
          break;
        case StepKind::kGemm:
          touch(st.gemm.a, i); touch(st.gemm.b, i); touch(st.gemm.c, i); touch(st.gemm.ws, i); touch(st.gemm.split_ws, i);
          break;
        case StepKind::kAttention:
          touch(st.attn.q, i); touch(st.attn.k, i); touch(st.attn.v, i); touch(st.attn.o, i); touch(st.attn.lse, i);
          break;
        case StepKind::kAttentionBwd:
          for (int s : {st.bwd.q, st.bwd.k, st.bwd.v, st.bwd.o, st.bwd.dout, st.bwd.lse, st.bwd.dq, st.bwd.dk, st.bwd.dv,
                        st.bwd.dq_acc, st.bwd.delta})
            touch(s, i);
          break;
        case StepKind::kScatterAdd: touch(st.scatter.base, i); touch(st.scatter.idx, i); touch(st.scatter.upd, i); touch(st.scatter.out, i); break;
        case StepKind::kCollective: {
          // an overlapped collective keeps its buffers until the step that waits for it
          const int until = st.async && i < (int)coll_until_.size() ? std::max(i, coll_until_[i]) : i;
          touch(st.coll.in, until);
          touch(st.coll.out, until);
          for (int x : st.coll.packed_in) touch(x, until);
          for (int x : st.coll.packed_out) touch(x, until);
          break;
        }
        case StepKind::kCopy: touch(st.copy.src, i); touch(st.copy.dst, i); break;
      }
    }
  }
};

}  // namespace

std::string Plan::dump() const {
  std::ostringstream o;
  o << "plan: " << slots.size() << " slots, " << steps.size() << " steps, " << consts.size() << " constants\n";
  for (size_t i = 0; i < steps.size(); ++i) {
    o << "  [" << i << "] " << steps[i].label;
    for (size_t k = 0; k < steps[i].launches.size(); ++k) o << (k ? ", " : "  {") << steps[i].launches[k].fn;
    o << (steps[i].launches.empty() ? "" : "}") << "\n";
  }
  for (size_t i = 0; i < arg_alias.size(); ++i) {
    if (arg_alias[i] < 0 && !arg_donor[i]) continue;
    o << "  donated argument " << i;
    if (arg_alias[i] >= 0)
      o << " -> result " << arg_alias[i]
        << (out_inplace_arg[arg_alias[i]] == (int)i ? " (written in place)" : " (fresh buffer; argument released)");
    o << "\n";
  }
  return o.str();
}

std::string Lower(Graph& g, const CompileOptions& opt, Plan* plan) {
  try {
    Lowerer l(g, opt, plan);
    l.Run();
  } catch (const LowerError& e) {
    return e.msg;
  } catch (const std::exception& e) {
    return std::string("lowering failed: ") + e.what();
  }
  return "";
}

}  // namespace b200
