// bytecode.cc — MLIR bytecode reader of the plugin compiler.
//
// PJRT_Program format "mlir" is MLIR text or MLIR bytecode (pjrt_c_api.h:539-552).  The reference
// hands either to MLIR's own reader (src/jam/parse.cc:53-63, `stablehlo::deserializePortableArtifact`).
// MLIR is not available here, so this file decodes the bytecode container itself, following the
// published format (mlir/docs/BytecodeFormat.md: magic "ML\xefR", version, producer, then sections
// of strings, dialects / op names, attribute and type offsets and data, IR, resources, properties)
// and the builtin dialect's attribute / type encodings, and writes the module out as MLIR text —
// `module` and `func.func` in their pretty forms, every other op in the generic form — for the
// text parser (parse.cc), which accepts both op forms.  Versions 0 through 6 of the format are read.
//
// What it reads: builtin attributes and types (strings, symbol refs, integers, floats, arrays,
// dictionaries, dense arrays, dense int / float elements, types; locations are skipped), the
// textual fallback that the writer uses for attributes and types of dialects without a bytecode
// interface (e.g. `#stablehlo<comparison_direction GE>` when the writer's context did not know
// stablehlo), properties of unregistered ops (one dictionary) and of builtin.module / func.func /
// func.call / func.return.  What it rejects with an error naming the construct: dialect-specific
// binary encodings (e.g. the VHLO dialect's), properties of other registered ops, successors,
// use-list orders, dense_resource blobs.
//
// Every read is bounds-checked: a truncated or corrupt input gives an error, never a crash.
#include "bytecode.h"

#include <cinttypes>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace b200 {
namespace {

struct Fail {
  std::string msg;
};

[[noreturn]] void Bad(const std::string& m) { throw Fail{m}; }

// ------------------------------------------------------------------------------ byte reader
struct Cursor {
  const uint8_t* p = nullptr;
  size_t n = 0, i = 0;
  Cursor() = default;
  Cursor(const uint8_t* d, size_t size) : p(d), n(size) {}
  bool empty() const { return i >= n; }
  uint8_t Byte() {
    if (i >= n) Bad("truncated bytecode");
    return p[i++];
  }
  const uint8_t* Take(uint64_t k) {
    if (k > n - i) Bad("truncated bytecode");
    const uint8_t* r = p + i;
    i += (size_t)k;
    return r;
  }
  // prefix varint: the count of trailing zero bits of the first byte + 1 is the length in bytes;
  // a first byte of 0 means eight more bytes hold the value
  uint64_t VarInt() {
    uint8_t b0 = Byte();
    if (b0 == 0) {
      const uint8_t* q = Take(8);
      uint64_t v = 0;
      for (int k = 7; k >= 0; --k) v = (v << 8) | q[k];
      return v;
    }
    int len = __builtin_ctz(b0) + 1;
    uint64_t v = b0;
    const uint8_t* q = Take(len - 1);
    for (int k = 0; k < len - 1; ++k) v |= (uint64_t)q[k] << (8 * (k + 1));
    return v >> len;
  }
  int64_t SVarInt() {   // zigzag
    uint64_t v = VarInt();
    return (int64_t)(v >> 1) ^ -(int64_t)(v & 1);
  }
  std::string CStr() {
    size_t j = i;
    while (j < n && p[j] != 0) ++j;
    if (j >= n) Bad("unterminated string in bytecode");
    std::string s((const char*)p + i, j - i);
    i = j + 1;
    return s;
  }
};

enum Section : uint8_t {
  kString = 0, kDialect = 1, kAttrType = 2, kAttrTypeOffset = 3, kIR = 4, kResource = 5,
  kResourceOffset = 6, kDialectVersions = 7, kProperties = 8, kNumSections = 9,
};

// op encoding mask bits
constexpr uint8_t kHasAttrs = 0x01, kHasResults = 0x02, kHasOperands = 0x04, kHasSuccessors = 0x08,
                  kHasInlineRegions = 0x10, kHasUseListOrders = 0x20, kHasProperties = 0x40;

// format versions that change the layout
constexpr uint64_t kDialectVersioning = 1, kLazyLoading = 2, kUseListOrdering = 3,
                   kElideUnknownBlockArgLocation = 4, kOpNameCount = 4, kNativePropertiesEncoding = 5,
                   kMaxVersion = 6;

// reads a section header (id, length, optional alignment + padding) and returns its body;
// alignment is counted from `base`, the start of the bytecode buffer
Cursor SectionAt(Cursor& c, uint8_t* id, const uint8_t* base) {
  uint8_t b = c.Byte();
  *id = b & 0x7f;
  uint64_t len = c.VarInt();
  if (b & 0x80) {
    uint64_t align = c.VarInt();
    if (align == 0 || (align & (align - 1)) || align > 4096) Bad("bad section alignment");
    // padding bytes up to the alignment, counted from the start of the buffer
    while ((size_t)(c.p + c.i - base) % align) {
      if (c.Byte() != 0xCB) Bad("bad section padding");
    }
  }
  const uint8_t* d = c.Take(len);
  return Cursor(d, len);
}

std::string Quote(const std::string& s) {
  std::string o = "\"";
  for (unsigned char ch : s) {
    if (ch == '"' || ch == '\\') { o += '\\'; o += (char)ch; }
    else if (ch < 0x20 || ch >= 0x7f) {
      char b[4];
      std::snprintf(b, sizeof b, "\\%02X", ch);
      o += b;
    } else {
      o += (char)ch;
    }
  }
  return o + "\"";
}

std::string Hex(const uint8_t* p, size_t n) {
  static const char* d = "0123456789ABCDEF";
  std::string s;
  s.reserve(2 * n);
  for (size_t k = 0; k < n; ++k) { s += d[p[k] >> 4]; s += d[p[k] & 15]; }
  return s;
}

// ------------------------------------------------------------------------------ the decoder
class Decoder {
 public:
  Decoder(const uint8_t* d, size_t n) : file_(d, n) {}

  std::string Run() {
    if (file_.n < 4 || std::memcmp(file_.p, "ML\xefR", 4) != 0) Bad("not MLIR bytecode");
    file_.i = 4;
    version_ = file_.VarInt();
    if (version_ > kMaxVersion) Bad("MLIR bytecode version " + std::to_string(version_) + " is newer than this reader (<= 6)");
    producer_ = file_.CStr();
    bool seen[kNumSections] = {};
    while (!file_.empty()) {
      uint8_t id;
      Cursor s = SectionAt(file_, &id, file_.p);
      if (id >= kNumSections) Bad("unknown bytecode section " + std::to_string(id));
      if (seen[id]) Bad("duplicate bytecode section " + std::to_string(id));
      seen[id] = true;
      sec_[id] = s;
    }
    for (uint8_t id : {kString, kDialect, kAttrType, kAttrTypeOffset, kIR})
      if (!seen[id]) Bad("bytecode lacks section " + std::to_string(id));
    ReadStrings();
    ReadDialects();
    ReadAttrTypeOffsets();
    if (seen[kProperties]) ReadProperties();
    return ReadIR();
  }

 private:
  // nesting limit for regions and for attributes / types that refer to one another
  int depth_ = 0, attr_depth_ = 0;
  struct DepthGuard {
    int& d;
    explicit DepthGuard(int& x) : d(x) {
      if (++d > 64) Bad("nesting too deep");
    }
    ~DepthGuard() { --d; }
  };

  Cursor file_;
  Cursor sec_[kNumSections];
  uint64_t version_ = 0;
  std::string producer_;

  std::vector<std::string> strings_;
  std::vector<std::string> dialects_;
  struct OpName {
    std::string dialect, name;
    bool registered = true;
    std::string full() const { return dialect + "." + name; }
  };
  std::vector<OpName> op_names_;

  struct Entry {
    size_t dialect = 0;
    const uint8_t* data = nullptr;
    size_t size = 0;
    bool custom = false;
  };
  std::vector<Entry> attr_entries_, type_entries_;
  std::vector<Cursor> props_;

  // decoded attributes / types (text form plus the structure the printer needs)
  struct AttrV {
    enum Kind { kText, kString, kDict, kArray, kType, kUnit, kInt, kFloat, kSymRef, kLoc, kDenseArray, kDense } kind = kText;
    std::string text;                       // MLIR text of the attribute
    std::string str;                        // kString: the value
    std::vector<std::pair<size_t, size_t>> dict;   // kDict: (name attr, value attr)
    std::vector<size_t> elems;              // kArray
    size_t type = SIZE_MAX;                 // kType / kInt / kFloat / kDense
  };
  struct TypeV {
    enum Kind { kText, kOther, kFunc } kind = kOther;
    std::string text;
    std::vector<size_t> inputs, results;    // kFunc
    int bits = 0;                           // integer / float width (0 if not scalar)
    bool is_int = false, is_index = false;
  };
  std::vector<std::unique_ptr<AttrV>> attrs_;
  std::vector<std::unique_ptr<TypeV>> types_;
  std::vector<uint8_t> attr_busy_, type_busy_;

  // ---------------------------------------------------------------- sections
  void ReadStrings() {
    Cursor c = sec_[kString];
    uint64_t n = c.VarInt();
    if (n > c.n) Bad("bad string count");
    std::vector<uint64_t> len(n);
    for (uint64_t k = 0; k < n; ++k) len[n - 1 - k] = c.VarInt();   // stored in reverse order
    strings_.reserve(n);
    for (uint64_t k = 0; k < n; ++k) {
      if (len[k] == 0) Bad("bad string length");
      const uint8_t* d = c.Take(len[k]);
      if (d[len[k] - 1] != 0) Bad("string not NUL-terminated");
      strings_.emplace_back((const char*)d, len[k] - 1);
    }
  }
  const std::string& Str(uint64_t k) {
    if (k >= strings_.size()) Bad("string index out of range");
    return strings_[k];
  }

  void ReadDialects() {
    Cursor c = sec_[kDialect];
    uint64_t n = c.VarInt();
    if (n > c.n) Bad("bad dialect count");
    for (uint64_t k = 0; k < n; ++k) {
      if (version_ < kDialectVersioning) {
        dialects_.push_back(Str(c.VarInt()));
        continue;
      }
      uint64_t v = c.VarInt();
      dialects_.push_back(Str(v >> 1));
      if (v & 1) {   // a dialect version follows as a nested section; this reader does not need it
        uint8_t id;
        SectionAt(c, &id, file_.p);
      }
    }
    if (version_ >= kOpNameCount) c.VarInt();   // total number of op names
    while (!c.empty()) {
      uint64_t d = c.VarInt();
      if (d >= dialects_.size()) Bad("dialect index out of range");
      uint64_t cnt = c.VarInt();
      if (cnt > c.n) Bad("bad op name count");
      for (uint64_t k = 0; k < cnt; ++k) {
        OpName on;
        on.dialect = dialects_[d];
        uint64_t v = c.VarInt();
        if (version_ >= kNativePropertiesEncoding) {
          on.registered = v & 1;
          v >>= 1;
        }
        on.name = Str(v);
        op_names_.push_back(on);
      }
    }
  }

  void ReadAttrTypeOffsets() {
    Cursor c = sec_[kAttrTypeOffset];
    uint64_t na = c.VarInt(), nt = c.VarInt();
    if (na > sec_[kAttrType].n + 1 || nt > sec_[kAttrType].n + 1) Bad("bad attribute / type count");
    size_t off = 0;
    auto group = [&](std::vector<Entry>& out, uint64_t total) {
      while (out.size() < total) {
        uint64_t d = c.VarInt();
        if (d >= dialects_.size()) Bad("dialect index out of range");
        uint64_t cnt = c.VarInt();
        if (cnt > total - out.size()) Bad("bad attribute / type group");
        for (uint64_t k = 0; k < cnt; ++k) {
          uint64_t v = c.VarInt();
          Entry e;
          e.dialect = d;
          e.custom = v & 1;
          e.size = v >> 1;
          if (e.size > sec_[kAttrType].n - off) Bad("attribute / type entry out of range");
          e.data = sec_[kAttrType].p + off;
          off += e.size;
          out.push_back(e);
        }
      }
    };
    group(attr_entries_, na);
    group(type_entries_, nt);
    attrs_.resize(na);
    types_.resize(nt);
    attr_busy_.assign(na, 0);
    type_busy_.assign(nt, 0);
  }

  void ReadProperties() {
    Cursor c = sec_[kProperties];
    uint64_t n = c.VarInt();
    if (n > c.n) Bad("bad properties count");
    for (uint64_t k = 0; k < n; ++k) {
      uint64_t len = c.VarInt();
      props_.emplace_back(c.Take(len), len);
    }
  }

  // ---------------------------------------------------------------- types
  const TypeV& Type(uint64_t k) {
    if (k >= types_.size()) Bad("type index out of range");
    if (types_[k]) return *types_[k];
    DepthGuard guard(attr_depth_);
    if (type_busy_[k]) Bad("cyclic type reference");
    type_busy_[k] = 1;
    auto t = std::make_unique<TypeV>();
    const Entry& e = type_entries_[k];
    Cursor c(e.data, e.size);
    if (!e.custom) {
      t->kind = TypeV::kText;
      t->text = c.CStr();
    } else {
      if (dialects_[e.dialect] != "builtin") Bad("type of dialect '" + dialects_[e.dialect] + "' uses its own bytecode encoding, which this reader does not know");
      DecodeBuiltinType(c, t.get());
    }
    type_busy_[k] = 0;
    types_[k] = std::move(t);
    return *types_[k];
  }

  std::string TypeList(Cursor& c, std::vector<size_t>* ids) {
    uint64_t n = c.VarInt();
    if (n > c.n) Bad("bad type list");
    std::string s;
    for (uint64_t k = 0; k < n; ++k) {
      uint64_t id = c.VarInt();
      if (ids) ids->push_back(id);
      s += (k ? ", " : "") + Type(id).text;
    }
    return s;
  }

  std::string Shape(Cursor& c) {
    uint64_t n = c.VarInt();
    if (n > c.n) Bad("bad shape");
    std::string s;
    for (uint64_t k = 0; k < n; ++k) {
      int64_t d = c.SVarInt();
      s += (d < 0 ? std::string("?") : std::to_string(d)) + "x";
    }
    return s;
  }

  void DecodeBuiltinType(Cursor& c, TypeV* t) {
    uint64_t code = c.VarInt();
    switch (code) {
      case 0: {   // IntegerType: width << 2 | signedness (0 signless, 1 signed, 2 unsigned)
        uint64_t v = c.VarInt();
        uint64_t w = v >> 2, sg = v & 3;
        t->text = std::string(sg == 1 ? "si" : sg == 2 ? "ui" : "i") + std::to_string(w);
        t->bits = (int)w;
        t->is_int = true;
        return;
      }
      case 1: t->text = "index"; t->bits = 64; t->is_int = t->is_index = true; return;
      case 2: {   // FunctionType
        t->kind = TypeV::kFunc;
        std::string in = TypeList(c, &t->inputs), out = TypeList(c, &t->results);
        t->text = "(" + in + ") -> (" + out + ")";
        return;
      }
      case 3: t->text = "bf16"; t->bits = 16; return;
      case 4: t->text = "f16"; t->bits = 16; return;
      case 5: t->text = "f32"; t->bits = 32; return;
      case 6: t->text = "f64"; t->bits = 64; return;
      case 7: t->text = "f80"; t->bits = 80; return;
      case 8: t->text = "f128"; t->bits = 128; return;
      case 9: t->text = "complex<" + Type(c.VarInt()).text + ">"; return;
      case 12: t->text = "none"; return;
      case 13: {  // RankedTensorType: shape, element type
        std::string sh = Shape(c);
        t->text = "tensor<" + sh + Type(c.VarInt()).text + ">";
        return;
      }
      case 14: {  // RankedTensorType with encoding: encoding, shape, element type
        std::string enc = Attr(c.VarInt()).text;
        std::string sh = Shape(c);
        t->text = "tensor<" + sh + Type(c.VarInt()).text + ", " + enc + ">";
        return;
      }
      case 15: {  // TupleType
        std::string l = TypeList(c, nullptr);
        t->text = "tuple<" + l + ">";
        return;
      }
      case 18: t->text = "tensor<*x" + Type(c.VarInt()).text + ">"; return;   // UnrankedTensorType
      default:
        Bad("builtin type code " + std::to_string(code) + " is not supported by this reader");
    }
  }

  // ---------------------------------------------------------------- attributes
  const AttrV& Attr(uint64_t k) {
    if (k >= attrs_.size()) Bad("attribute index out of range");
    if (attrs_[k]) return *attrs_[k];
    DepthGuard guard(attr_depth_);
    if (attr_busy_[k]) Bad("cyclic attribute reference");
    attr_busy_[k] = 1;
    auto a = std::make_unique<AttrV>();
    const Entry& e = attr_entries_[k];
    Cursor c(e.data, e.size);
    if (!e.custom) {
      a->kind = AttrV::kText;
      a->text = c.CStr();
    } else {
      if (dialects_[e.dialect] != "builtin")
        Bad("attribute of dialect '" + dialects_[e.dialect] + "' uses its own bytecode encoding, which this reader does not know");
      DecodeBuiltinAttr(c, a.get());
    }
    attr_busy_[k] = 0;
    attrs_[k] = std::move(a);
    return *attrs_[k];
  }

  // APInt of a known bit width: <= 8 bits one byte, <= 64 a signed varint, else a word count and
  // signed-varint words (least significant first)
  std::vector<uint64_t> APInt(Cursor& c, int bits) {
    if (bits <= 8) return {(uint64_t)c.Byte()};
    if (bits <= 64) return {(uint64_t)c.SVarInt()};
    uint64_t nw = c.VarInt();
    if (nw > c.n) Bad("bad APInt");
    std::vector<uint64_t> w;
    for (uint64_t k = 0; k < nw; ++k) w.push_back((uint64_t)c.SVarInt());
    return w;
  }

  static std::string IntText(uint64_t raw, int bits, bool is_unsigned) {
    if (bits == 1) return (raw & 1) ? "true" : "false";
    if (bits < 64) {
      uint64_t mask = (1ull << bits) - 1;
      raw &= mask;
      if (!is_unsigned && (raw >> (bits - 1))) return std::to_string((int64_t)(raw | ~mask));
      return std::to_string(raw);
    }
    return is_unsigned ? std::to_string(raw) : std::to_string((int64_t)raw);
  }

  std::string ElemsText(const std::string& elem_type, const uint8_t* d, size_t n) {
    // dense arrays: element type i1 (one byte each), i8..i64, f32, f64
    int w = elem_type == "i1" ? 1 : elem_type == "i8" ? 1 : elem_type == "i16" ? 2 : elem_type == "i32" ? 4 :
            elem_type == "i64" ? 8 : elem_type == "f32" ? 4 : elem_type == "f64" ? 8 : 0;
    if (!w || n % w) Bad("dense array of " + elem_type + " is not supported by this reader");
    std::string s;
    for (size_t k = 0; k < n / w; ++k) {
      uint64_t raw = 0;
      std::memcpy(&raw, d + k * w, w);
      s += k ? ", " : ": ";
      if (elem_type == "f32") {
        char b[32];
        float f;
        std::memcpy(&f, &raw, 4);
        std::snprintf(b, sizeof b, "%.9g", f);
        s += b;
      } else if (elem_type == "f64") {
        char b[40];
        double f;
        std::memcpy(&f, &raw, 8);
        std::snprintf(b, sizeof b, "%.17g", f);
        s += b;
      } else if (elem_type == "i1") {
        s += raw ? "true" : "false";
      } else {
        s += IntText(raw, 8 * w, false);
      }
    }
    return s;
  }

  void DecodeBuiltinAttr(Cursor& c, AttrV* a) {
    uint64_t code = c.VarInt();
    switch (code) {
      case 0: {   // ArrayAttr
        a->kind = AttrV::kArray;
        uint64_t n = c.VarInt();
        if (n > c.n) Bad("bad array attribute");
        a->text = "[";
        for (uint64_t k = 0; k < n; ++k) {
          size_t id = c.VarInt();
          a->elems.push_back(id);
          a->text += (k ? ", " : "") + Attr(id).text;
        }
        a->text += "]";
        return;
      }
      case 1: {   // DictionaryAttr: (name, value) pairs
        a->kind = AttrV::kDict;
        uint64_t n = c.VarInt();
        if (n > c.n) Bad("bad dictionary attribute");
        for (uint64_t k = 0; k < n; ++k) {
          size_t name = c.VarInt(), value = c.VarInt();
          a->dict.push_back({name, value});
        }
        a->text = DictText(a->dict);
        return;
      }
      case 2:     // StringAttr
        a->kind = AttrV::kString;
        a->str = Str(c.VarInt());
        a->text = Quote(a->str);
        return;
      case 3: {   // StringAttr with type
        a->kind = AttrV::kString;
        a->str = Str(c.VarInt());
        a->text = Quote(a->str) + " : " + Type(c.VarInt()).text;
        return;
      }
      case 4: {   // FlatSymbolRefAttr: root reference (a StringAttr)
        a->kind = AttrV::kSymRef;
        a->text = "@" + SymName(StringOf(c.VarInt()));
        return;
      }
      case 5: {   // SymbolRefAttr: root, nested flat references
        a->kind = AttrV::kSymRef;
        a->text = "@" + SymName(StringOf(c.VarInt()));
        uint64_t n = c.VarInt();
        if (n > c.n) Bad("bad symbol reference");
        for (uint64_t k = 0; k < n; ++k) a->text += "::" + Attr(c.VarInt()).text;
        return;
      }
      case 6:     // TypeAttr
        a->kind = AttrV::kType;
        a->type = c.VarInt();
        a->text = Type(a->type).text;
        return;
      case 7: a->kind = AttrV::kUnit; a->text = "unit"; return;
      case 8: {   // IntegerAttr: type, value
        a->kind = AttrV::kInt;
        a->type = c.VarInt();
        const TypeV& t = Type(a->type);
        if (!t.is_int || t.bits == 0) Bad("integer attribute of non-integer type " + t.text);
        auto w = APInt(c, t.bits);
        if (w.size() != 1) Bad("integer attributes wider than 64 bits are not supported by this reader");
        a->text = IntText(w[0], t.bits, t.text.rfind("ui", 0) == 0) + " : " + t.text;
        if (t.bits == 1) a->text = (w[0] & 1) ? "true" : "false";
        return;
      }
      case 9: {   // FloatAttr: type, value bits
        a->kind = AttrV::kFloat;
        a->type = c.VarInt();
        const TypeV& t = Type(a->type);
        if (t.bits != 16 && t.bits != 32 && t.bits != 64) Bad("float attribute of type " + t.text + " is not supported by this reader");
        auto w = APInt(c, t.bits);
        if (w.size() != 1) Bad("bad float attribute");
        char b[40];
        std::snprintf(b, sizeof b, "0x%0*" PRIX64, t.bits / 4, t.bits == 64 ? w[0] : (w[0] & ((1ull << t.bits) - 1)));
        a->text = std::string(b) + " : " + t.text;
        return;
      }
      case 10: case 11: case 12: case 13: case 14: case 15: case 22:   // locations
        a->kind = AttrV::kLoc;
        a->text = "loc(unknown)";
        return;
      case 16: Bad("dense_resource attributes are not supported by this reader");
      case 17: {  // DenseArrayAttr: element type, element count, raw data blob
        a->kind = AttrV::kDenseArray;
        std::string et = Type(c.VarInt()).text;
        c.VarInt();   // element count (implied by the blob size)
        uint64_t sz = c.VarInt();
        const uint8_t* d = c.Take(sz);
        a->text = "array<" + et + ElemsText(et, d, sz) + ">";
        return;
      }
      case 18: {  // DenseIntOrFPElementsAttr: shaped type, raw data blob
        a->kind = AttrV::kDense;
        a->type = c.VarInt();
        const std::string& ty = Type(a->type).text;
        uint64_t sz = c.VarInt();
        const uint8_t* d = c.Take(sz);
        std::vector<uint8_t> bytes(d, d + sz);
        // i1 elements are stored one bit each, least significant bit first, and a splat as one
        // byte of all ones or all zeros (a constant whose elements are all equal is always a
        // splat); the text form wants one byte per element
        if ((ty.size() > 4 && ty.compare(ty.size() - 4, 4, "xi1>") == 0) || ty == "tensor<i1>") {
          int64_t n = NumElements(ty);
          if (sz == 1 && (d[0] == 0x00 || d[0] == 0xFF)) bytes = {(uint8_t)(d[0] ? 1 : 0)};
          else if ((int64_t)sz == (n + 7) / 8) {
            bytes.assign(n, 0);
            for (int64_t k = 0; k < n; ++k) bytes[k] = (d[k / 8] >> (k % 8)) & 1;
          } else {
            for (auto& b : bytes) b = b ? 1 : 0;
          }
        }
        a->text = "dense<\"0x" + Hex(bytes.data(), bytes.size()) + "\"> : " + ty;
        return;
      }
      default:
        Bad("builtin attribute code " + std::to_string(code) + " is not supported by this reader");
    }
  }

  static int64_t NumElements(const std::string& tensor_type) {
    // "tensor<4x8xi1>" -> 32
    int64_t n = 1;
    size_t k = 7;
    while (k < tensor_type.size()) {
      size_t x = tensor_type.find('x', k);
      if (x == std::string::npos) break;
      std::string d = tensor_type.substr(k, x - k);
      if (d.empty() || d.find_first_not_of("0123456789") != std::string::npos) break;
      n *= std::stoll(d);
      k = x + 1;
    }
    return n;
  }

  const std::string& StringOf(uint64_t attr) {
    const AttrV& a = Attr(attr);
    if (a.kind != AttrV::kString) Bad("expected a string attribute");
    return a.str;
  }

  static std::string SymName(const std::string& s) {
    bool plain = !s.empty() && (std::isalpha((unsigned char)s[0]) || s[0] == '_');
    for (char ch : s) plain = plain && (std::isalnum((unsigned char)ch) || ch == '_' || ch == '.' || ch == '$');
    return plain ? s : Quote(s);
  }

  static std::string KeyText(const std::string& k) {
    bool plain = !k.empty() && (std::isalpha((unsigned char)k[0]) || k[0] == '_');
    for (char ch : k) plain = plain && (std::isalnum((unsigned char)ch) || ch == '_' || ch == '.' || ch == '$');
    return plain ? k : Quote(k);
  }

  std::string DictText(const std::vector<std::pair<size_t, size_t>>& d) {
    std::string s = "{";
    for (size_t k = 0; k < d.size(); ++k) {
      const std::string& key = StringOf(d[k].first);
      const AttrV& v = Attr(d[k].second);
      s += (k ? ", " : "") + KeyText(key);
      if (v.kind != AttrV::kUnit) s += " = " + v.text;
    }
    return s + "}";
  }

  // ---------------------------------------------------------------- properties
  // property reader: plain attribute index, or (index << 1 | present) for an optional one
  struct PropReader {
    Decoder* d;
    Cursor c;
    size_t Required() { return c.VarInt(); }
    int64_t Optional() {
      uint64_t v = c.VarInt();
      return (v & 1) ? (int64_t)(v >> 1) : -1;
    }
  };

  // named property values of one op
  using Props = std::vector<std::pair<std::string, size_t>>;

  Props ReadOpProps(const OpName& on, uint64_t index) {
    if (index >= props_.size()) Bad("properties index out of range");
    PropReader r{this, props_[index]};
    Props out;
    auto opt = [&](const char* name) {
      int64_t v = r.Optional();
      if (v >= 0) out.push_back({name, (size_t)v});
    };
    auto req = [&](const char* name) { out.push_back({name, r.Required()}); };
    if (!on.registered) {
      // an unregistered op keeps its properties as one attribute (a dictionary)
      const AttrV& a = Attr(r.Required());
      if (a.kind != AttrV::kDict) Bad("properties of unregistered op " + on.full() + " are not a dictionary");
      for (auto& kv : a.dict) out.push_back({StringOf(kv.first), kv.second});
      return out;
    }
    std::string n = on.full();
    // the ODS-generated writer stores the properties in name order, required ones as an attribute
    // index and optional ones as (index << 1 | present); which properties an op has depends on the
    // MLIR release that wrote the file, so the layout is picked by the number of entries
    size_t count = 0;
    for (Cursor t = r.c; !t.empty(); ++count) t.VarInt();
    if (n == "builtin.module" && count == 2) {
      opt("sym_name");
      opt("sym_visibility");
    } else if (n == "func.func" && (count == 5 || count == 6)) {
      opt("arg_attrs");
      req("function_type");
      if (count == 6) opt("no_inline");
      opt("res_attrs");
      req("sym_name");
      opt("sym_visibility");
    } else if (n == "func.call" && count <= 4) {
      if (count == 4) opt("arg_attrs");
      req("callee");
      if (count >= 2) opt("no_inline");
      if (count == 4) opt("res_attrs");
    } else {
      Bad("cannot read the properties of registered op " + n + " (" + std::to_string(count) +
          " entries; dialect-specific encoding)");
    }
    if (!r.c.empty()) Bad("unexpected trailing properties data for " + n);
    return out;
  }

  // ---------------------------------------------------------------- IR
  struct Scope {
    std::vector<std::string> values;       // value names by bytecode value number
    std::vector<size_t> next;              // next free slot of each open region
  };
  std::vector<Scope> scopes_;
  size_t value_counter_ = 0;
  std::string out_;

  std::string NewValue() { return "%v" + std::to_string(value_counter_++); }

  void PushRegion(uint64_t num_values, size_t bytes_left) {
    Scope& s = scopes_.back();
    s.next.push_back(s.values.size());
    // every value is defined by a block argument or an op result, each at least one byte
    if (num_values > bytes_left) Bad("bad value count");
    s.values.resize(s.values.size() + num_values);
  }
  void PopRegion(uint64_t num_values) {
    Scope& s = scopes_.back();
    s.values.resize(s.values.size() - num_values);
    s.next.pop_back();
  }
  std::string Define() {
    Scope& s = scopes_.back();
    size_t& k = s.next.back();
    if (k >= s.values.size()) Bad("more values defined than the region declares");
    s.values[k] = NewValue();
    return s.values[k++];
  }
  const std::string& Use(uint64_t k) {
    Scope& s = scopes_.back();
    if (k >= s.values.size() || s.values[k].empty()) Bad("use of an undefined value (forward references are not supported)");
    return s.values[k];
  }

  std::string ReadIR() {
    Cursor c = sec_[kIR];
    scopes_.emplace_back();
    // the IR section holds one block of top-level ops (the module)
    uint64_t hdr = c.VarInt();
    if (hdr & 1) Bad("top-level block with arguments");
    PushRegion(0, 0);
    for (uint64_t k = 0; k < (hdr >> 1); ++k) ReadOp(c, "");
    return out_;
  }

  struct OpData {
    const OpName* name = nullptr;
    uint8_t mask = 0;
    Props attrs;                       // discardable attribute dictionary
    Props props;                       // properties
    std::vector<size_t> result_types;
    std::vector<std::string> operands;
    std::vector<std::string> operand_types;
    std::vector<std::string> results;
    uint64_t num_regions = 0;
    bool isolated = false;
  };

  void ReadOp(Cursor& c, const std::string& ind) {
    DepthGuard guard(depth_);
    OpData op;
    uint64_t ni = c.VarInt();
    if (ni >= op_names_.size()) Bad("op name index out of range");
    op.name = &op_names_[ni];
    op.mask = c.Byte();
    c.VarInt();   // location
    if (op.mask & kHasAttrs) {
      const AttrV& a = Attr(c.VarInt());
      if (a.kind != AttrV::kDict) Bad("op attributes are not a dictionary");
      for (auto& kv : a.dict) op.attrs.push_back({StringOf(kv.first), kv.second});
    }
    if (op.mask & kHasProperties) {
      if (version_ < kNativePropertiesEncoding) Bad("properties in bytecode older than version 5");
      op.props = ReadOpProps(*op.name, c.VarInt());
    }
    if (op.mask & kHasResults) {
      uint64_t n = c.VarInt();
      if (n > c.n) Bad("bad result count");
      for (uint64_t k = 0; k < n; ++k) op.result_types.push_back(c.VarInt());
    }
    if (op.mask & kHasOperands) {
      uint64_t n = c.VarInt();
      if (n > c.n) Bad("bad operand count");
      for (uint64_t k = 0; k < n; ++k) op.operands.push_back(Use(c.VarInt()));
    }
    if (op.mask & kHasSuccessors) Bad("ops with successor blocks are not supported (" + op.name->full() + ")");
    if (op.mask & kHasUseListOrders) Bad("use-list orders are not supported by this reader");
    for (size_t k = 0; k < op.result_types.size(); ++k) op.results.push_back(Define());
    if (op.mask & kHasInlineRegions) {
      uint64_t v = c.VarInt();
      op.num_regions = v >> 1;
      op.isolated = v & 1;
      if (op.num_regions > c.n) Bad("bad region count");
    }
    Emit(c, op, ind);
  }

  // operand types are not stored with the op: they are the types of the values, which this
  // printer tracks by name
  std::map<std::string, std::string> value_types_;

  void ReadRegions(Cursor& c, const OpData& op, const std::string& ind, bool func_body) {
    Cursor sub;
    Cursor* rc = &c;
    if (op.isolated) {
      if (version_ >= kLazyLoading) {
        uint8_t id;
        sub = SectionAt(c, &id, file_.p);
        if (id != kIR) Bad("isolated region not in an IR section");
        rc = &sub;
      }
      scopes_.emplace_back();
    }
    for (uint64_t r = 0; r < op.num_regions; ++r) {
      if (r) out_ += ", ";
      ReadRegion(*rc, ind, func_body && r == 0);
    }
    if (op.isolated) scopes_.pop_back();
  }

  // a region: block count, value count, blocks; `func_body` prints the entry block's arguments in
  // the func.func signature (already written by the caller) instead of as a block label
  void ReadRegion(Cursor& c, const std::string& ind, bool func_body) {
    uint64_t nb = c.VarInt();
    if (nb == 0) {
      out_ += "{\n" + ind + "}";
      return;
    }
    if (nb != 1) Bad("regions with more than one block are not supported");
    uint64_t nv = c.VarInt();
    PushRegion(nv, c.n - c.i);
    uint64_t hdr = c.VarInt();
    uint64_t nops = hdr >> 1;
    std::vector<std::string> args;
    std::vector<std::string> arg_types;
    if (hdr & 1) {
      uint64_t na = c.VarInt();
      if (na > c.n) Bad("bad block argument count");
      for (uint64_t k = 0; k < na; ++k) {
        uint64_t ty;
        if (version_ >= kElideUnknownBlockArgLocation) {
          uint64_t v = c.VarInt();
          ty = v >> 1;
          if (v & 1) c.VarInt();
        } else {
          ty = c.VarInt();
          c.VarInt();
        }
        std::string name = Define();
        value_types_[name] = Type(ty).text;
        args.push_back(name);
        arg_types.push_back(Type(ty).text);
      }
      if (version_ >= kUseListOrdering) {
        if (c.Byte() != 0) Bad("use-list orders are not supported by this reader");
      }
    }
    if (func_body) {
      // the caller left "func.func @f(" open: finish the signature
      std::string sig;
      for (size_t k = 0; k < args.size(); ++k) {
        sig += (k ? ", " : "") + args[k] + ": " + arg_types[k];
        if (k < func_arg_attrs_.size() && !func_arg_attrs_[k].empty()) sig += " " + func_arg_attrs_[k];
      }
      func_arg_attrs_.clear();
      out_ += sig + func_sig_tail_ + " {\n";
    } else {
      out_ += "{\n";
      if (!args.empty()) {
        out_ += ind + "^bb0(";
        for (size_t k = 0; k < args.size(); ++k) out_ += (k ? ", " : "") + args[k] + ": " + arg_types[k];
        out_ += "):\n";
      }
    }
    for (uint64_t k = 0; k < nops; ++k) ReadOp(c, ind + "  ");
    out_ += ind + "}";
    PopRegion(nv);
  }
  std::string func_sig_tail_;
  std::vector<std::string> func_arg_attrs_;   // per argument of the func.func being written: "{...}" or ""

  const AttrV* Find(const Props& p, const char* name) {
    for (auto& kv : p)
      if (kv.first == name) return &Attr(kv.second);
    return nullptr;
  }

  std::string PropsText(const Props& p, std::initializer_list<const char*> skip = {}) {
    std::string s;
    for (auto& kv : p) {
      bool sk = false;
      for (const char* x : skip) sk = sk || kv.first == x;
      if (sk) continue;
      const AttrV& v = Attr(kv.second);
      s += (s.empty() ? "" : ", ") + KeyText(kv.first);
      if (v.kind != AttrV::kUnit) s += " = " + v.text;
    }
    return s;
  }

  void Emit(Cursor& c, const OpData& op, const std::string& ind) {
    std::string full = op.name->full();
    std::vector<std::string> rtypes;
    for (size_t k = 0; k < op.result_types.size(); ++k) {
      rtypes.push_back(Type(op.result_types[k]).text);
      value_types_[op.results[k]] = rtypes.back();
    }
    if (full == "builtin.module") {
      Props all = op.props;
      all.insert(all.end(), op.attrs.begin(), op.attrs.end());
      out_ += ind + "module";
      if (const AttrV* n = Find(all, "sym_name")) out_ += " @" + SymName(n->str);
      std::string at = PropsText(all, {"sym_name", "sym_visibility"});
      if (!at.empty()) out_ += " attributes {" + at + "}";
      out_ += " ";
      if (op.num_regions != 1) Bad("module without exactly one region");
      ReadRegions(c, op, ind, false);
      out_ += "\n";
      return;
    }
    if (full == "func.func") {
      Props all = op.props;
      all.insert(all.end(), op.attrs.begin(), op.attrs.end());
      const AttrV* name = Find(all, "sym_name");
      const AttrV* fty = Find(all, "function_type");
      if (!name || !fty || fty->kind != AttrV::kType) Bad("func.func without sym_name / function_type");
      const TypeV& ft = Type(fty->type);
      if (ft.kind != TypeV::kFunc) Bad("func.func type is not a function type");
      out_ += ind + "func.func ";
      if (const AttrV* vis = Find(all, "sym_visibility")) out_ += vis->str + " ";
      out_ += "@" + SymName(name->str) + "(";
      func_sig_tail_ = ") -> (";
      for (size_t k = 0; k < ft.results.size(); ++k) func_sig_tail_ += (k ? ", " : "") + Type(ft.results[k]).text;
      func_sig_tail_ += ")";
      func_arg_attrs_.clear();
      if (const AttrV* aa = Find(all, "arg_attrs")) {
        if (aa->kind != AttrV::kArray) Bad("func.func arg_attrs is not an array");
        for (size_t e : aa->elems) {
          const AttrV& d = Attr(e);
          if (d.kind != AttrV::kDict) Bad("func.func arg_attrs entry is not a dictionary");
          func_arg_attrs_.push_back(d.dict.empty() ? std::string() : d.text);
        }
      }
      if (op.num_regions != 1) Bad("external func.func declarations are not supported");
      ReadRegions(c, op, ind, true);
      out_ += "\n";
      return;
    }
    // generic form
    out_ += ind;
    for (size_t k = 0; k < op.results.size(); ++k) out_ += (k ? ", " : "") + op.results[k];
    if (!op.results.empty()) out_ += " = ";
    out_ += Quote(full) + "(";
    std::string in_types;
    for (size_t k = 0; k < op.operands.size(); ++k) {
      out_ += (k ? ", " : "") + op.operands[k];
      auto it = value_types_.find(op.operands[k]);
      if (it == value_types_.end()) Bad("operand of unknown type");
      in_types += (k ? ", " : "") + it->second;
    }
    out_ += ")";
    std::string pt = PropsText(op.props);
    if (!op.props.empty()) out_ += " <{" + pt + "}>";
    if (op.num_regions) {
      out_ += " (";
      ReadRegions(c, op, ind + "  ", false);
      out_ += ")";
    }
    std::string at = PropsText(op.attrs);
    if (!at.empty()) out_ += " {" + at + "}";
    out_ += " : (" + in_types + ") -> (";
    for (size_t k = 0; k < rtypes.size(); ++k) out_ += (k ? ", " : "") + rtypes[k];
    out_ += ")\n";
  }
};

}  // namespace

bool IsMlirBytecode(const void* data, size_t size) {
  return size >= 4 && std::memcmp(data, "ML\xefR", 4) == 0;
}

std::string MlirBytecodeToText(const void* data, size_t size, std::string* text) {
  try {
    Decoder d((const uint8_t*)data, size);
    *text = d.Run();
  } catch (const Fail& f) {
    return "MLIR bytecode: " + f.msg;
  } catch (const std::exception& e) {
    return std::string("MLIR bytecode: ") + e.what();
  }
  return "";
}

}  // namespace b200
