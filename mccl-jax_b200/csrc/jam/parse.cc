// parse.cc — StableHLO MLIR-text front end of the plugin compiler.
//
// Replaces the reference's MLIR deserialization + normalization (src/jam/parse.cc:17-63): the
// plugin reads the module *text* jax prints (`jit(f).lower(...).as_text()`), in the pretty forms of
// elementwise / shape / reduce / dot ops and the generic `"stablehlo.x"(...) <{...}> ({...})` form
// (which gather / scatter / collectives always use, and which every op takes in MLIR bytecode:
// bytecode input is first decoded to text by bytecode.cc).  `func.call`s are inlined while building the graph, which is what
// the reference's lowering walk does (src/jam/lower.mm:245-268); `optimization_barrier`, tuples'
// absence and the shard_map custom calls are handled by the planner.
#include "ir.h"

#include "bytecode.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <sstream>
#include <unordered_map>

namespace b200 {

int DTBytes(DT t) {
  switch (t) {
    case DT::kPred: case DT::kS8: case DT::kU8: return 1;
    case DT::kS16: case DT::kU16: case DT::kF16: case DT::kBF16: return 2;
    case DT::kS32: case DT::kU32: case DT::kF32: return 4;
    case DT::kS64: case DT::kU64: case DT::kF64: return 8;
    default: return 0;
  }
}
const char* DTName(DT t) {
  static const char* n[] = {"i1", "i8", "i16", "i32", "i64", "ui8", "ui16", "ui32", "ui64",
                            "f16", "bf16", "f32", "f64", "invalid"};
  return n[(int)t];
}
bool DTIsFloat(DT t) { return t == DT::kF16 || t == DT::kBF16 || t == DT::kF32 || t == DT::kF64; }
bool DTIsSigned(DT t) { return t == DT::kS8 || t == DT::kS16 || t == DT::kS32 || t == DT::kS64; }
bool DTIsUnsigned(DT t) { return t == DT::kU8 || t == DT::kU16 || t == DT::kU32 || t == DT::kU64; }
DT DTFromMlir(const std::string& s) {
  static const std::unordered_map<std::string, DT> m = {
      {"i1", DT::kPred}, {"i8", DT::kS8}, {"i16", DT::kS16}, {"i32", DT::kS32}, {"i64", DT::kS64},
      {"ui8", DT::kU8}, {"ui16", DT::kU16}, {"ui32", DT::kU32}, {"ui64", DT::kU64},
      {"f16", DT::kF16}, {"bf16", DT::kBF16}, {"f32", DT::kF32}, {"f64", DT::kF64}};
  auto it = m.find(s);
  return it == m.end() ? DT::kInvalid : it->second;
}

std::string TensorType::str() const {
  std::string s = "tensor<";
  for (int64_t d : dims) s += std::to_string(d) + "x";
  return s + DTName(dt) + ">";
}

void Graph::Renumber() {
  for (auto& v : values) v->users.clear();
  for (size_t i = 0; i < ops.size(); ++i) {
    ops[i]->index = (int)i;
    for (Value* v : ops[i]->operands) v->users.push_back(ops[i].get());
  }
}

double ConstScalar(const Op* op) {
  DT t = op->result()->type.dt;
  const uint8_t* p = op->data.data();
  switch (t) {
    case DT::kPred: return p[0] ? 1.0 : 0.0;
    case DT::kS8: return (double)*(const int8_t*)p;
    case DT::kU8: return (double)*(const uint8_t*)p;
    case DT::kS16: return (double)*(const int16_t*)p;
    case DT::kU16: return (double)*(const uint16_t*)p;
    case DT::kS32: return (double)*(const int32_t*)p;
    case DT::kU32: return (double)*(const uint32_t*)p;
    case DT::kS64: return (double)*(const int64_t*)p;
    case DT::kU64: return (double)*(const uint64_t*)p;
    case DT::kF32: return (double)*(const float*)p;
    case DT::kF64: return *(const double*)p;
    case DT::kBF16: {
      uint32_t u = (uint32_t)(*(const uint16_t*)p) << 16;
      float f;
      std::memcpy(&f, &u, 4);
      return f;
    }
    case DT::kF16: {
      uint16_t h = *(const uint16_t*)p;
      uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 31, man = h & 1023;
      double v;
      if (exp == 0) v = std::ldexp((double)man, -24);
      else if (exp == 31) v = man ? NAN : INFINITY;
      else v = std::ldexp((double)(man | 1024), (int)exp - 25);
      return sign ? -v : v;
    }
    default: return 0;
  }
}

namespace {

// ------------------------------------------------------------------------------------ tokens
struct Lexer {
  std::vector<std::string> toks;
  std::string err;

  static bool IdStart(char c) { return std::isalpha((unsigned char)c) || c == '_'; }
  static bool IdChar(char c) { return std::isalnum((unsigned char)c) || c == '_' || c == '.' || c == '$'; }

  bool Run(const char* s, size_t n) {
    size_t i = 0;
    while (i < n) {
      char c = s[i];
      if (std::isspace((unsigned char)c)) { ++i; continue; }
      if (c == '/' && i + 1 < n && s[i + 1] == '/') {
        while (i < n && s[i] != '\n') ++i;
        continue;
      }
      size_t j = i;
      if (c == '"') {
        ++j;
        while (j < n && s[j] != '"') { if (s[j] == '\\') ++j; ++j; }
        toks.emplace_back(s + i, j + 1 - i);
        i = j + 1;
        continue;
      }
      if (c == '%' || c == '@' || c == '^') {
        ++j;
        while (j < n && (IdChar(s[j]) || s[j] == '#')) ++j;
        toks.emplace_back(s + i, j - i);
        i = j;
        continue;
      }
      if (c == '-' && i + 1 < n && s[i + 1] == '>') { toks.push_back("->"); i += 2; continue; }
      if (IdStart(c) || c == '#' || c == '!') {
        ++j;
        while (j < n && IdChar(s[j])) ++j;
        std::string word(s + i, j - i);
        if (j < n && s[j] == '<' &&
            (word == "tensor" || word == "dense" || word == "array" || word[0] == '#' || word[0] == '!')) {
          // whole balanced <...> group as one token
          int depth = 1;
          ++j;
          while (j < n && depth) {
            if (s[j] == '<') ++depth;
            else if (s[j] == '>' && s[j - 1] != '-') --depth;
            else if (s[j] == '"') { ++j; while (j < n && s[j] != '"') ++j; }
            ++j;
          }
          toks.emplace_back(s + i, j - i);
          i = j;
          continue;
        }
        toks.push_back(word);
        i = j;
        continue;
      }
      if (std::isdigit((unsigned char)c) || ((c == '-' || c == '+') && i + 1 < n && std::isdigit((unsigned char)s[i + 1]))) {
        ++j;
        while (j < n && (std::isalnum((unsigned char)s[j]) || s[j] == '.' ||
                         ((s[j] == '-' || s[j] == '+') && (s[j - 1] == 'e' || s[j - 1] == 'E'))))
          ++j;
        toks.emplace_back(s + i, j - i);
        i = j;
        continue;
      }
      if (std::strchr("()[]{},:=<>*", c)) { toks.emplace_back(1, c); ++i; continue; }
      err = std::string("unexpected character '") + c + "'";
      return false;
    }
    return true;
  }
};

// ------------------------------------------------------------------------------------ AST
struct OpAst {
  std::string name;                 // full name, e.g. stablehlo.add / func.call / func.return
  std::vector<std::string> results;
  std::vector<std::string> operands;
  std::map<std::string, std::vector<int64_t>> ints;
  std::map<std::string, std::string> strs;
  std::vector<TensorType> in_types, out_types;
  std::vector<std::string> region_ops;   // op names in the (first) region body
  std::string dense;                     // constant literal token
};

struct FuncAst {
  std::string name;
  std::vector<std::pair<std::string, TensorType>> args;
  std::vector<std::map<std::string, std::string>> arg_attrs;   // per argument (empty if none)
  std::vector<TensorType> results;
  std::vector<OpAst> ops;
};

struct ParseError {
  std::string msg;
};

std::vector<int64_t> ParseIntsAttr(const std::string& s);
int64_t ReplicaGroupCount(const std::string& s);
void ParseDimNumbers(const std::string& s, const std::string& prefix, Op* op);

class Parser {
 public:
  explicit Parser(std::vector<std::string> t) : t_(std::move(t)) {}

  std::map<std::string, FuncAst> funcs;
  int num_partitions = 1, num_replicas = 1;
  std::string module_name;

  void Module() {
    if (Accept("module")) {
      if (!Peek().empty() && Peek()[0] == '@') module_name = Next().substr(1);
      if (Accept("attributes")) {
        auto d = AttrDict();
        if (d.count("mhlo.num_partitions")) num_partitions = std::stoi(d["mhlo.num_partitions"]);
        if (d.count("mhlo.num_replicas")) num_replicas = std::stoi(d["mhlo.num_replicas"]);
      }
      Expect("{");
    }
    while (!AtEnd() && Peek() != "}") {
      FuncAst f = Func();
      funcs[f.name] = std::move(f);
    }
  }

 private:
  std::vector<std::string> t_;
  size_t i_ = 0;

  bool AtEnd() const { return i_ >= t_.size(); }
  const std::string& Peek(size_t k = 0) const {
    static const std::string empty;
    return i_ + k < t_.size() ? t_[i_ + k] : empty;
  }
  std::string Next() {
    if (AtEnd()) throw ParseError{"unexpected end of input"};
    return t_[i_++];
  }
  void Expect(const std::string& s) {
    std::string got = Next();
    if (got != s) {
      std::string ctx;
      for (size_t k = (i_ > 6 ? i_ - 6 : 0); k < std::min(t_.size(), i_ + 4); ++k) ctx += t_[k] + " ";
      throw ParseError{"expected '" + s + "' but got '" + got + "' near: " + ctx};
    }
  }
  bool Accept(const std::string& s) {
    if (Peek() == s) { ++i_; return true; }
    return false;
  }

  static TensorType Type(const std::string& tok) {
    if (tok.rfind("tensor<", 0) != 0) throw ParseError{"expected a tensor type, got '" + tok + "'"};
    std::string body = tok.substr(7, tok.size() - 8);
    size_t comma = body.find(',');
    if (comma != std::string::npos) body = body.substr(0, comma);
    TensorType t;
    size_t start = 0;
    while (true) {
      size_t x = body.find('x', start);
      // a dim is all digits; the element type is the remainder
      if (x == std::string::npos || x == start) break;
      std::string d = body.substr(start, x - start);
      bool digits = !d.empty() && std::all_of(d.begin(), d.end(), [](char c) { return std::isdigit((unsigned char)c); });
      if (!digits) break;
      t.dims.push_back(std::stoll(d));
      start = x + 1;
    }
    t.dt = DTFromMlir(body.substr(start));
    if (t.dt == DT::kInvalid) throw ParseError{"unsupported element type in '" + tok + "'"};
    return t;
  }

  std::vector<int64_t> IntList() {
    std::vector<int64_t> out;
    Expect("[");
    while (!Accept("]")) {
      std::string tok = Next();
      if (tok == ",") continue;
      if (tok == "[") {  // nested: flatten
        --i_;
        auto inner = IntList();
        out.insert(out.end(), inner.begin(), inner.end());
        continue;
      }
      // non-integer list entries (e.g. precision = [DEFAULT, DEFAULT]) carry no shape information
      if (!tok.empty() && (std::isdigit((unsigned char)tok[0]) || (tok[0] == '-' && tok.size() > 1)))
        out.push_back(std::stoll(tok));
    }
    return out;
  }

  std::string SkipBalanced() {
    std::string open = Peek();
    std::string close = open == "(" ? ")" : open == "[" ? "]" : open == "{" ? "}" : "";
    if (close.empty()) return Next();
    std::string raw;
    int depth = 0;
    while (true) {
      std::string tok = Next();
      raw += tok + " ";
      if (tok == "(" || tok == "[" || tok == "{") ++depth;
      else if (tok == ")" || tok == "]" || tok == "}") {
        if (--depth == 0) return raw;
      }
    }
  }

  std::string AttrValue(bool typed, std::string* type_out = nullptr) {
    if (Peek() == "[") {
      auto v = IntList();
      std::string s;
      for (size_t k = 0; k < v.size(); ++k) s += (k ? "," : "") + std::to_string(v[k]);
      return "[" + s + "]";
    }
    if (Peek() == "{" || Peek() == "(") return SkipBalanced();
    std::string v = Next();
    if (typed && Peek() == ":") {
      const std::string& ty = Peek(1);
      bool is_type = ty.rfind("tensor<", 0) == 0 || ty == "index" ||
                     (ty.size() >= 2 && (ty[0] == 'i' || ty[0] == 'f' || ty[0] == 'u') && std::isdigit((unsigned char)ty.back()));
      if (is_type) {
        Next();
        const std::string t = Next();
        if (type_out) *type_out = t;
      }
    }
    return v;
  }

  std::map<std::string, std::string> AttrDict() {
    std::map<std::string, std::string> d;
    Expect("{");
    while (!Accept("}")) {
      std::string key = Next();
      if (key == ",") continue;
      std::string val = "true", ty;
      if (Accept("=")) val = AttrValue(true, &ty);
      d[key] = val;
      // the group structure of replica_groups is in its type (tensor<GROUPSxSIZExi64>), which a
      // hex literal does not show
      if (key == "replica_groups" && !ty.empty()) d["replica_groups.type"] = ty;
    }
    return d;
  }

  std::vector<std::pair<std::string, TensorType>> BlockArgs() {
    std::vector<std::pair<std::string, TensorType>> args;
    Expect("(");
    while (!Accept(")")) {
      if (Peek() == ",") { Next(); continue; }
      std::string a = Next();
      Expect(":");
      args.push_back({a, Type(Next())});
    }
    return args;
  }

  FuncAst Func() {
    Expect("func.func");
    if (Peek() == "public" || Peek() == "private") Next();
    FuncAst f;
    f.name = Next().substr(1);
    Expect("(");
    while (!Accept(")")) {
      if (Peek() == ",") { Next(); continue; }
      std::string a = Next();
      Expect(":");
      TensorType ty = Type(Next());
      f.arg_attrs.push_back(Peek() == "{" ? AttrDict() : std::map<std::string, std::string>());
      f.args.push_back({a, ty});
    }
    if (Accept("->")) {
      if (Accept("(")) {
        while (!Accept(")")) {
          if (Peek() == ",") { Next(); continue; }
          f.results.push_back(Type(Next()));
          if (Peek() == "{") AttrDict();
        }
      } else {
        f.results.push_back(Type(Next()));
      }
    }
    if (Accept("attributes")) AttrDict();
    f.ops = BlockBody();
    return f;
  }

  // `{ [^bb0(args):] ops }` — returns the op list (block args are only named, never used by us).
  std::vector<OpAst> BlockBody() {
    Expect("{");
    std::vector<OpAst> ops;
    if (!Peek().empty() && Peek()[0] == '^') {
      Next();
      BlockArgs();
      Expect(":");
    }
    while (!Accept("}")) ops.push_back(Operation());
    return ops;
  }

  std::vector<std::string> ParenOperands() {
    std::vector<std::string> v;
    Expect("(");
    while (!Accept(")")) {
      std::string tok = Next();
      if (tok != ",") v.push_back(tok);
    }
    return v;
  }

  void FnType(OpAst& op, size_t n_operands) {
    if (Accept("(")) {
      while (!Accept(")")) {
        if (Peek() == ",") { Next(); continue; }
        op.in_types.push_back(Type(Next()));
      }
      Expect("->");
      if (Accept("(")) {
        while (!Accept(")")) {
          if (Peek() == ",") { Next(); continue; }
          op.out_types.push_back(Type(Next()));
        }
      } else {
        op.out_types.push_back(Type(Next()));
      }
      return;
    }
    TensorType t = Type(Next());
    if (Accept("->")) {        // `: T -> U`, as chlo's unary ops print
      op.in_types.assign(n_operands, t);
      op.out_types.push_back(Type(Next()));
      return;
    }
    op.out_types.push_back(t);
    op.in_types.assign(n_operands, t);
  }

  static void RegionSummary(OpAst& op, const std::vector<OpAst>& body) {
    for (const OpAst& b : body) {
      op.region_ops.push_back(b.name);
      // the first comparison of a reducer body tells argmax (GT) from argmin (LT), as the
      // reference's DetectArgReduce reads it (src/jam/ops/reduce.mm:29-43)
      if (b.name == "stablehlo.compare" && !op.strs.count("region_compare")) {
        auto it = b.strs.find("comparison_direction");
        if (it != b.strs.end()) op.strs["region_compare"] = it->second;
      }
    }
  }

  OpAst Operation() {
    OpAst op;
    const std::string& p0 = Peek();
    if (!p0.empty() && p0[0] == '%' &&
        (Peek(1) == "=" || Peek(1) == "," || (Peek(1) == ":" && Peek(3) == "="))) {
      while (true) {
        std::string r = Next();
        if (Accept(":")) {
          int cnt = std::stoi(Next());
          for (int k = 0; k < cnt; ++k) op.results.push_back(r + "#" + std::to_string(k));
        } else {
          op.results.push_back(r);
        }
        if (!Accept(",")) break;
      }
      Expect("=");
    }
    std::string name = Next();
    if (name[0] == '"') return Generic(name.substr(1, name.size() - 2), std::move(op));
    if (name == "return" || name == "func.return" || name == "stablehlo.return") {
      op.name = name == "stablehlo.return" ? name : "func.return";
      while (!Peek().empty() && Peek()[0] == '%') {
        op.operands.push_back(Next());
        Accept(",");
      }
      if (Accept(":")) {
        for (size_t k = 0; k < op.operands.size(); ++k) {
          if (k) Expect(",");
          op.in_types.push_back(Type(Next()));
        }
      }
      return op;
    }
    op.name = name;
    if (name == "call" || name == "func.call") {
      op.name = "func.call";
      op.strs["callee"] = Next().substr(1);
      op.operands = ParenOperands();
      Expect(":");
      FnType(op, op.operands.size());
      return op;
    }
    if (name == "stablehlo.reduce") return Reduce(std::move(op));
    if (name == "stablehlo.custom_call") {
      op.strs["call_target_name"] = Next().substr(1);
      op.operands = ParenOperands();
      if (Peek() == "{") {
        for (auto& kv : AttrDict()) op.strs[kv.first] = kv.second;
      }
      Expect(":");
      FnType(op, op.operands.size());
      return op;
    }
    return Pretty(std::move(op));
  }

  OpAst Pretty(OpAst op) {
    std::vector<std::string> bare;
    while (Peek() != ":") {
      if (AtEnd()) throw ParseError{"unterminated op " + op.name};
      const std::string& tok = Peek();
      if (tok[0] == '%') {
        op.operands.push_back(Next());
      } else if (tok == ",") {
        Next();
      } else if (tok == "[" && op.name == "stablehlo.slice") {
        Next();
        std::vector<int64_t> st, li, sd;
        while (!Accept("]")) {
          if (Peek() == ",") { Next(); continue; }
          std::vector<int64_t> parts{std::stoll(Next())};
          while (Accept(":")) parts.push_back(std::stoll(Next()));
          st.push_back(parts[0]);
          li.push_back(parts.size() > 1 ? parts[1] : parts[0] + 1);
          sd.push_back(parts.size() > 2 ? parts[2] : 1);
        }
        op.ints["start_indices"] = st;
        op.ints["limit_indices"] = li;
        op.ints["strides"] = sd;
      } else if (tok == "{") {
        for (auto& kv : AttrDict()) op.strs[kv.first] = kv.second;
      } else if (Peek(1) == "=") {
        std::string key = Next();
        Next();
        if (Peek() == "[") {
          auto lhs = IntList();
          if (Accept("x")) {
            op.ints[key + ".lhs"] = lhs;
            op.ints[key + ".rhs"] = IntList();
          } else if (key != "precision") {   // precision = [DEFAULT, DEFAULT]: no shape information
            op.ints[key] = lhs;
          }
        } else {
          std::string v = AttrValue(false);
          bool num = !v.empty() && (std::isdigit((unsigned char)v[0]) || v[0] == '-');
          if (num) op.ints[key] = {std::stoll(v)};
          else op.strs[key] = v;
        }
      } else if (tok.rfind("dense<", 0) == 0) {
        op.dense = Next();
      } else {
        bare.push_back(Next());
      }
    }
    Expect(":");
    if (op.name == "stablehlo.compare") {
      if (!bare.empty()) op.strs["comparison_direction"] = bare[0];
      if (bare.size() > 1) op.strs["compare_type"] = bare[1];
    }
    if (op.name == "stablehlo.select" && Peek() != "(") {
      TensorType pt = Type(Next());
      Expect(",");
      TensorType rt = Type(Next());
      op.in_types = {pt, rt, rt};
      op.out_types = {rt};
      return op;
    }
    if (op.name == "stablehlo.optimization_barrier" && Peek() != "(") {
      for (size_t k = 0; k < op.operands.size(); ++k) {
        if (k) Expect(",");
        op.out_types.push_back(Type(Next()));
      }
      op.in_types = op.out_types;
      return op;
    }
    FnType(op, op.operands.size());
    return op;
  }

  OpAst Reduce(OpAst op) {
    std::vector<std::string> xs, inits;
    while (true) {
      Expect("(");
      xs.push_back(Next());
      Expect("init");
      Expect(":");
      inits.push_back(Next());
      Expect(")");
      if (!Accept(",")) break;
    }
    op.operands = xs;
    op.operands.insert(op.operands.end(), inits.begin(), inits.end());
    std::string applies;
    if (Accept("applies")) applies = Next();
    Expect("across");
    Expect("dimensions");
    Expect("=");
    op.ints["dimensions"] = IntList();
    Expect(":");
    FnType(op, op.operands.size());
    if (!applies.empty()) {
      op.region_ops.push_back(applies);
    } else {
      Expect("reducer");
      while (Peek() == "(") BlockArgs();
      RegionSummary(op, BlockBody());
    }
    return op;
  }

  OpAst Generic(const std::string& name, OpAst op) {
    op.name = name;
    op.operands = ParenOperands();
    if (Peek() == "<") {
      Next();
      for (auto& kv : AttrDict()) op.strs[kv.first] = kv.second;
      Expect(">");
    }
    if (Accept("(")) {
      bool first = true;
      while (!Accept(")")) {
        if (Peek() == ",") { Next(); continue; }
        auto body = BlockBody();
        if (first) RegionSummary(op, body);
        first = false;
      }
    }
    if (Peek() == "{") {
      for (auto& kv : AttrDict()) op.strs[kv.first] = kv.second;
    }
    Expect(":");
    FnType(op, op.operands.size());
    NormalizeGeneric(op);
    return op;
  }

  // The generic form spells attributes as StableHLO's op definitions name them
  // (broadcast_dimensions, permutation, #stablehlo.dot<...>, ...); the lowering reads the keys the
  // pretty form gives (Pretty / Reduce above).  Both forms must give one IR.
  static void NormalizeGeneric(OpAst& op) {
    auto take = [&](const char* key, std::string* out) {
      auto it = op.strs.find(key);
      if (it == op.strs.end()) return false;
      *out = it->second;
      op.strs.erase(it);
      return true;
    };
    auto ints_of = [&](const char* key, const char* as) {
      std::string v;
      if (take(key, &v)) op.ints[as] = ParseIntsAttr(v);
    };
    // "#stablehlo<comparison_direction GE>" -> "GE"
    auto enum_word = [](const std::string& v) {
      std::string s = v;
      size_t gt = s.rfind('>');
      if (gt != std::string::npos) s = s.substr(0, gt);
      size_t sp = s.find_last_of(" <");
      return sp == std::string::npos ? s : s.substr(sp + 1);
    };
    const std::string& n = op.name;
    std::string v;
    if (n == "func.call") {
      if (take("callee", &v)) op.strs["callee"] = v.empty() || v[0] != '@' ? v : v.substr(1);
    } else if (n == "stablehlo.broadcast_in_dim") {
      ints_of("broadcast_dimensions", "dims");
    } else if (n == "stablehlo.transpose") {
      ints_of("permutation", "dims");
    } else if (n == "stablehlo.broadcast") {
      ints_of("broadcast_sizes", "sizes");
    } else if (n == "stablehlo.reverse") {
      ints_of("dimensions", "dims");
    } else if (n == "stablehlo.dynamic_slice") {
      ints_of("slice_sizes", "sizes");
    } else if (n == "stablehlo.reduce_precision") {
      ints_of("exponent_bits", "exponent_bits");
      ints_of("mantissa_bits", "mantissa_bits");
    } else if (n == "stablehlo.iota") {
      ints_of("iota_dimension", "dim");
    } else if (n == "stablehlo.concatenate") {
      ints_of("dimension", "dim");
    } else if (n == "stablehlo.reduce") {
      ints_of("dimensions", "dimensions");
    } else if (n == "stablehlo.slice") {
      ints_of("start_indices", "start_indices");
      ints_of("limit_indices", "limit_indices");
      ints_of("strides", "strides");
    } else if (n == "stablehlo.pad") {
      ints_of("edge_padding_low", "low");
      ints_of("edge_padding_high", "high");
      ints_of("interior_padding", "interior");
    } else if (n == "stablehlo.compare") {
      if (take("comparison_direction", &v)) op.strs["comparison_direction"] = enum_word(v);
      if (take("compare_type", &v)) op.strs["compare_type"] = enum_word(v);
    } else if (n == "stablehlo.constant") {
      if (take("value", &v)) op.dense = v;
    } else if (n == "stablehlo.custom_call") {
      if (take("call_target_name", &v)) {
        if (v.size() >= 2 && v.front() == '"') v = v.substr(1, v.size() - 2);
        op.strs["call_target_name"] = v;
      }
    } else if (n == "stablehlo.dot_general") {
      if (take("dot_dimension_numbers", &v)) {
        Op scratch;
        ParseDimNumbers(v, "", &scratch);
        static const char* kMap[][2] = {{"lhs_batching_dimensions", "batching_dims.lhs"},
                                        {"rhs_batching_dimensions", "batching_dims.rhs"},
                                        {"lhs_contracting_dimensions", "contracting_dims.lhs"},
                                        {"rhs_contracting_dimensions", "contracting_dims.rhs"}};
        for (auto& m : kMap) {
          auto it = scratch.ints.find(m[0]);
          if (it != scratch.ints.end()) op.ints[m[1]] = it->second;
        }
      }
    }
  }
};

// ------------------------------------------------------------------------------------ constants
bool HexBytes(const std::string& hex, std::vector<uint8_t>* out) {
  if (hex.size() % 2) return false;
  out->clear();
  for (size_t k = 0; k < hex.size(); k += 2) out->push_back((uint8_t)std::stoul(hex.substr(k, 2), nullptr, 16));
  return true;
}

uint16_t FloatToBF16RNE(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

uint16_t FloatToHalf(double d) {
  // round-to-nearest-even double -> binary16
  float f = (float)d;
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  int32_t exp = (int32_t)((x >> 23) & 0xff) - 127 + 15;
  uint32_t man = x & 0x7fffffu;
  if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0));
  if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    man |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - exp);
    uint32_t half = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1))) ++half;
    return (uint16_t)(sign | half);
  }
  uint32_t h = sign | ((uint32_t)exp << 10) | (man >> 13);
  uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;
  return (uint16_t)h;
}

void AppendScalar(DT dt, const std::string& tok, std::vector<uint8_t>* out) {
  auto put = [&](const void* p, int n) { out->insert(out->end(), (const uint8_t*)p, (const uint8_t*)p + n); };
  int width = DTBytes(dt);
  if (tok.rfind("0x", 0) == 0) {
    uint64_t bits = std::stoull(tok.substr(2), nullptr, 16);
    put(&bits, width);
    return;
  }
  if (tok == "true" || tok == "false") {
    uint8_t b = tok == "true";
    put(&b, 1);
    return;
  }
  if (DTIsFloat(dt)) {
    double d = tok == "inf" ? INFINITY : tok == "-inf" ? -INFINITY : tok == "nan" ? NAN : std::stod(tok);
    if (dt == DT::kF32) { float f = (float)d; put(&f, 4); }
    else if (dt == DT::kF64) put(&d, 8);
    else if (dt == DT::kBF16) { uint16_t h = FloatToBF16RNE((float)d); put(&h, 2); }
    else { uint16_t h = FloatToHalf(d); put(&h, 2); }
    return;
  }
  if (dt == DT::kPred) { uint8_t b = std::stod(tok) != 0; put(&b, 1); return; }
  if (DTIsUnsigned(dt)) { uint64_t u = std::stoull(tok); put(&u, width); return; }
  int64_t v = std::stoll(tok);
  put(&v, width);
}

void ParseDense(const std::string& tok, const TensorType& ty, Op* op) {
  std::string body = tok.substr(6, tok.size() - 7);
  while (!body.empty() && std::isspace((unsigned char)body[0])) body.erase(0, 1);
  if (body.rfind("\"0x", 0) == 0) {
    std::vector<uint8_t> raw;
    HexBytes(body.substr(3, body.size() - 4), &raw);
    op->splat = (int64_t)raw.size() == DTBytes(ty.dt) && ty.numel() != 1;
    op->data = raw;
    if ((int64_t)raw.size() != DTBytes(ty.dt) && (int64_t)raw.size() != ty.bytes())
      throw ParseError{"dense hex literal has the wrong size"};
    if (ty.numel() == 1) op->splat = true;
    return;
  }
  if (body[0] != '[') {
    op->splat = true;
    AppendScalar(ty.dt, body, &op->data);
    return;
  }
  // nested list: collect scalar tokens
  std::string cur;
  for (char c : body) {
    if (c == '[' || c == ']' || c == ',' || std::isspace((unsigned char)c)) {
      if (!cur.empty()) { AppendScalar(ty.dt, cur, &op->data); cur.clear(); }
    } else {
      cur.push_back(c);
    }
  }
  if (!cur.empty()) AppendScalar(ty.dt, cur, &op->data);
  op->splat = false;
  if ((int64_t)op->data.size() != ty.bytes()) throw ParseError{"dense literal has the wrong element count"};
  if (ty.numel() == 1) op->splat = true;
}

ReduceKind KindOfRegion(const std::vector<std::string>& ops) {
  for (const auto& n : ops) {
    if (n == "stablehlo.add") return ReduceKind::kAdd;
    if (n == "stablehlo.maximum") return ReduceKind::kMax;
    if (n == "stablehlo.minimum") return ReduceKind::kMin;
    if (n == "stablehlo.multiply") return ReduceKind::kMul;
    if (n == "stablehlo.and") return ReduceKind::kAnd;
    if (n == "stablehlo.or") return ReduceKind::kOr;
  }
  return ReduceKind::kNone;
}

std::vector<int64_t> ParseIntsAttr(const std::string& s) {
  // "array<i64: 1, 768>" or "[1,2]" or "dense<[[0, 1]]> " -> integers
  std::vector<int64_t> out;
  if (s.rfind("dense<\"0x", 0) == 0) {
    // hex form (how MLIR prints, and the bytecode reader writes, dense integer data): the integer
    // attributes read here (replica_groups) are i64, little-endian
    size_t end = s.find('"', 9);
    std::string hex = s.substr(9, end == std::string::npos ? std::string::npos : end - 9);
    if (hex.size() % 16) throw ParseError{"dense integer attribute is not i64: " + s};
    for (size_t k = 0; k < hex.size(); k += 16) {
      uint64_t v = 0;
      for (int b = 7; b >= 0; --b) v = (v << 8) | std::stoul(hex.substr(k + 2 * b, 2), nullptr, 16);
      out.push_back((int64_t)v);
    }
    return out;
  }
  size_t start = s.find(':');
  if (s.rfind("array<", 0) != 0) start = 0;
  else if (start == std::string::npos) return out;   // "array<i64>": empty
  std::string cur;
  for (size_t k = (start == std::string::npos ? 0 : start + (s.rfind("array<", 0) == 0 ? 1 : 0)); k < s.size(); ++k) {
    char c = s[k];
    if (std::isdigit((unsigned char)c) || (c == '-' && cur.empty())) cur.push_back(c);
    else if (!cur.empty()) {
      if (cur != "-") out.push_back(std::stoll(cur));
      cur.clear();
    }
  }
  if (!cur.empty() && cur != "-") out.push_back(std::stoll(cur));
  return out;
}

// Number of groups in a replica_groups attribute: the leading extent of its tensor type when the
// text carries one ("dense<...> : tensor<2x4xi64>"), else the bracket nesting of the literal
// ("[[0, 1], [2, 3]]" has 2 groups, a flat "[0, 1]" one); -1 when neither tells.
int64_t ReplicaGroupCount(const std::string& s) {
  const size_t t = s.find("tensor<");
  if (t != std::string::npos) {
    size_t k = t + 7;
    int64_t g = 0;
    bool any = false;
    while (k < s.size() && std::isdigit((unsigned char)s[k])) { g = g * 10 + (s[k++] - '0'); any = true; }
    if (any && k < s.size() && s[k] == 'x') return g;
  }
  if (s.find("0x") != std::string::npos) return -1;
  const size_t a = s.find('[');
  if (a == std::string::npos) return -1;
  if (a + 1 < s.size() && s.find_first_not_of(" ", a + 1) != std::string::npos && s[s.find_first_not_of(" ", a + 1)] != '[')
    return 1;
  int64_t inner = 0;
  for (size_t k = a + 1; k < s.size(); ++k) if (s[k] == '[') ++inner;
  return inner;
}

// "#stablehlo.gather<offset_dims = [1], collapsed_slice_dims = [0], index_vector_dim = 1>"
void ParseDimNumbers(const std::string& s, const std::string& prefix, Op* op) {
  size_t lt = s.find('<');
  if (lt == std::string::npos) return;
  std::string body = s.substr(lt + 1, s.size() - lt - 2);
  size_t k = 0;
  while (k < body.size()) {
    size_t eq = body.find('=', k);
    if (eq == std::string::npos) break;
    std::string key = body.substr(k, eq - k);
    key.erase(0, key.find_first_not_of(" ,"));
    key.erase(key.find_last_not_of(' ') + 1);
    size_t v0 = body.find_first_not_of(' ', eq + 1);
    if (v0 == std::string::npos) throw ParseError{"malformed dimension numbers: " + s};
    size_t v1;
    if (body[v0] == '[') {
      v1 = body.find(']', v0);
      if (v1 == std::string::npos) throw ParseError{"malformed dimension numbers: " + s};
      ++v1;
    } else {
      v1 = body.find(',', v0);
    }
    if (v1 == std::string::npos) v1 = body.size();
    op->ints[prefix + key] = ParseIntsAttr(body.substr(v0, v1 - v0));
    k = v1;
  }
}

// ------------------------------------------------------------------------------------ graph build
class Builder {
 public:
  Builder(const std::map<std::string, FuncAst>& funcs, Graph* g) : funcs_(funcs), g_(g) {}

  void BuildMain() {
    auto it = funcs_.find("main");
    if (it == funcs_.end()) throw ParseError{"module has no @main"};
    std::unordered_map<std::string, Value*> env;
    for (size_t k = 0; k < it->second.args.size(); ++k) {
      Value* v = g_->NewValue(it->second.args[k].second);
      v->arg_index = (int)k;
      g_->args.push_back(v);
      env[it->second.args[k].first] = v;
      // buffer donation as jax marks it (jit's donate_argnums): `tf.aliasing_output = k` when the
      // argument's buffer may become result k, `jax.buffer_donor` when it may be reused freely
      const auto& at = it->second.arg_attrs[k];
      int alias = -1;
      auto al = at.find("tf.aliasing_output");
      if (al != at.end()) {
        char* end = nullptr;
        const long x = std::strtol(al->second.c_str(), &end, 10);
        if (end == al->second.c_str() || *end || x < 0 || x > INT32_MAX)
          throw ParseError{"argument " + std::to_string(k) + ": bad tf.aliasing_output " + al->second};
        alias = (int)x;
      }
      auto dn = at.find("jax.buffer_donor");
      g_->arg_alias_output.push_back(alias);
      g_->arg_donor.push_back(alias >= 0 || (dn != at.end() && dn->second == "true"));
    }
    g_->outputs = Walk(it->second, env, 0);
  }

 private:
  const std::map<std::string, FuncAst>& funcs_;
  Graph* g_;

  std::vector<Value*> Walk(const FuncAst& f, std::unordered_map<std::string, Value*>& env, int depth) {
    if (depth > 64) throw ParseError{"func.call nesting too deep"};
    for (const OpAst& a : f.ops) {
      auto lookup = [&](const std::string& n) -> Value* {
        auto e = env.find(n);
        if (e == env.end()) throw ParseError{"use of undefined value " + n + " in " + a.name};
        return e->second;
      };
      if (a.name == "func.return") {
        std::vector<Value*> r;
        for (auto& n : a.operands) r.push_back(lookup(n));
        return r;
      }
      if (a.name == "func.call") {
        auto cf = funcs_.find(a.strs.at("callee"));
        if (cf == funcs_.end()) throw ParseError{"func.call to unknown callee @" + a.strs.at("callee")};
        std::unordered_map<std::string, Value*> inner;
        if (cf->second.args.size() != a.operands.size()) throw ParseError{"func.call arity mismatch"};
        for (size_t k = 0; k < a.operands.size(); ++k) inner[cf->second.args[k].first] = lookup(a.operands[k]);
        auto rets = Walk(cf->second, inner, depth + 1);
        if (rets.size() != a.results.size()) throw ParseError{"func.call result count mismatch"};
        for (size_t k = 0; k < rets.size(); ++k) env[a.results[k]] = rets[k];
        continue;
      }
      std::string opname;
      if (a.name == "chlo.erf") opname = "erf";
      else if (a.name.rfind("stablehlo.", 0) == 0) opname = a.name.substr(10);
      else throw ParseError{"unsupported op '" + a.name + "'"};
      {
        // custom_call @mhlo.erf carries chlo.erf through a pipeline without the chlo dialect
        auto t = a.strs.find("call_target_name");
        if (opname == "custom_call" && t != a.strs.end() && t->second == "mhlo.erf") opname = "erf";
      }
      Op* op = g_->NewOp(opname);
      for (auto& n : a.operands) op->operands.push_back(lookup(n));
      // the operand types the text states must be the types of the values it names
      if (a.in_types.size() == a.operands.size()) {
        for (size_t k = 0; k < a.operands.size(); ++k)
          if (!(op->operands[k]->type == a.in_types[k]))
            throw ParseError{"malformed program: operand " + std::to_string(k) + " of " + a.name + " is " +
                             op->operands[k]->type.str() + " but the op states " + a.in_types[k].str()};
      }
      op->ints = a.ints;
      op->strs = a.strs;
      if (a.out_types.size() != a.results.size())
        throw ParseError{"op " + a.name + ": result/type count mismatch"};
      for (size_t k = 0; k < a.results.size(); ++k) {
        Value* v = g_->NewValue(a.out_types[k]);
        v->def = op;
        op->results.push_back(v);
        env[a.results[k]] = v;
      }
      if (!a.region_ops.empty()) op->reduce = KindOfRegion(a.region_ops);
      if (op->name == "reduce_precision" && op->strs.count("format")) {
        // pretty form: format = e5m10
        const std::string& f = op->strs["format"];
        size_t m = f.find('m');
        if (f.size() < 4 || f[0] != 'e' || m == std::string::npos) throw ParseError{"bad reduce_precision format " + f};
        op->ints["exponent_bits"] = {std::stoll(f.substr(1, m - 1))};
        op->ints["mantissa_bits"] = {std::stoll(f.substr(m + 1))};
      }
      if (op->name == "constant") ParseDense(a.dense, op->result()->type, op);
      if (op->name == "gather") {
        ParseDimNumbers(op->strs["dimension_numbers"], "", op);
        op->ints["slice_sizes"] = ParseIntsAttr(op->strs["slice_sizes"]);
      }
      if (op->name == "scatter") ParseDimNumbers(op->strs["scatter_dimension_numbers"], "", op);
      for (const char* key : {"all_gather_dim", "scatter_dimension", "split_dimension", "concat_dimension"}) {
        auto s = op->strs.find(key);
        if (s != op->strs.end()) op->ints[key] = ParseIntsAttr(s->second);
      }
      if (op->strs.count("replica_groups")) {
        const std::string& rg = op->strs["replica_groups"];
        op->ints["replica_groups"] = ParseIntsAttr(rg);
        auto ty = op->strs.find("replica_groups.type");
        op->ints["replica_groups.count"] = {ReplicaGroupCount(ty == op->strs.end() ? rg : rg + " : " + ty->second)};
        if (ty != op->strs.end()) op->strs.erase(ty);
      }
      if (op->strs.count("source_target_pairs")) op->ints["source_target_pairs"] = ParseIntsAttr(op->strs["source_target_pairs"]);
    }
    throw ParseError{"function @" + f.name + " has no return"};
  }
};

}  // namespace

std::string DumpGraph(const Graph& g) {
  std::ostringstream o;
  o << "graph partitions=" << g.num_partitions << " replicas=" << g.num_replicas << " args:";
  for (const Value* v : g.args) o << " %" << v->id << ":" << v->type.str();
  o << "\n";
  static const char* kStrKeys[] = {"comparison_direction", "compare_type", "call_target_name", "mhlo.sharding", "region_compare"};
  for (const auto& op : g.ops) {
    for (size_t k = 0; k < op->results.size(); ++k) o << (k ? ", " : "") << "%" << op->results[k]->id;
    o << " = " << op->name << "(";
    for (size_t k = 0; k < op->operands.size(); ++k) o << (k ? ", " : "") << "%" << op->operands[k]->id;
    o << ") ->";
    for (const Value* v : op->results) o << " " << v->type.str();
    for (const auto& kv : op->ints) {
      o << " " << kv.first << "=[";
      for (size_t k = 0; k < kv.second.size(); ++k) o << (k ? "," : "") << kv.second[k];
      o << "]";
    }
    for (const char* key : kStrKeys) {
      auto it = op->strs.find(key);
      if (it != op->strs.end()) o << " " << key << "=" << it->second;
    }
    if (op->reduce != ReduceKind::kNone) o << " reduce=" << (int)op->reduce;
    if (op->name == "constant") {
      uint64_t h = 1469598103934665603ull;
      for (uint8_t b : op->data) h = (h ^ b) * 1099511628211ull;
      o << " splat=" << op->splat << " bytes=" << op->data.size() << " fnv=" << std::hex << h << std::dec;
    }
    o << "\n";
  }
  o << "outputs:";
  for (const Value* v : g.outputs) o << " %" << v->id;
  o << "\n";
  return o.str();
}

std::string ParseModule(const char* text, size_t size, Graph* g) {
  std::string decoded;
  if (IsMlirBytecode(text, size)) {
    std::string err = MlirBytecodeToText(text, size, &decoded);
    if (!err.empty()) return err;
    if (const char* dump = std::getenv("B200_DUMP_BYTECODE_TEXT")) {
      if (FILE* f = std::fopen(dump, "w")) {
        std::fwrite(decoded.data(), 1, decoded.size(), f);
        std::fclose(f);
      }
    }
    text = decoded.data();
    size = decoded.size();
  }
  try {
    Lexer lx;
    if (!lx.Run(text, size)) return "lex error: " + lx.err;
    Parser p(std::move(lx.toks));
    p.Module();
    g->name = p.module_name;
    g->num_partitions = p.num_partitions;
    g->num_replicas = p.num_replicas;
    Builder b(p.funcs, g);
    b.BuildMain();
    g->Renumber();
    std::string bad = VerifyGraph(*g);
    if (!bad.empty()) return "malformed program: " + bad;
  } catch (const ParseError& e) {
    return e.msg;
  } catch (const std::exception& e) {
    return std::string("parse error: ") + e.what();
  }
  return "";
}

}  // namespace b200
