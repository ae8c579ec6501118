// compile_options.cc — see compile_options.h.  A protobuf wire-format reader restated from the
// published encoding: each field is a varint key (field number << 3 | wire type) followed by a varint
// (type 0), 8 bytes (type 1), a varint length and that many bytes (type 2), or 4 bytes (type 5).
#include "compile_options.h"

namespace b200 {
namespace {

class Reader {
 public:
  Reader(const uint8_t* p, size_t n) : p_(p), end_(p + n) {}
  bool done() const { return p_ >= end_; }

  std::string Varint(uint64_t* v) {
    uint64_t r = 0;
    for (int shift = 0; shift < 64; shift += 7) {
      if (p_ >= end_) return "truncated varint";
      const uint8_t b = *p_++;
      r |= (uint64_t)(b & 0x7f) << shift;
      if (!(b & 0x80)) {
        *v = r;
        return "";
      }
    }
    return "varint longer than 10 bytes";
  }
  // The next field: number, wire type and, for length-delimited fields, its payload.
  std::string Field(uint32_t* number, uint32_t* type, const uint8_t** payload, size_t* len, uint64_t* value) {
    uint64_t key = 0;
    std::string e = Varint(&key);
    if (!e.empty()) return e;
    *number = (uint32_t)(key >> 3);
    *type = (uint32_t)(key & 7);
    if (*number == 0) return "field number 0";
    switch (*type) {
      case 0:
        return Varint(value);
      case 1:
        if (end_ - p_ < 8) return "truncated fixed64";
        p_ += 8;
        return "";
      case 2: {
        uint64_t n = 0;
        e = Varint(&n);
        if (!e.empty()) return e;
        if (n > (uint64_t)(end_ - p_)) return "length-delimited field runs past the end";
        *payload = p_;
        *len = (size_t)n;
        p_ += n;
        return "";
      }
      case 5:
        if (end_ - p_ < 4) return "truncated fixed32";
        p_ += 4;
        return "";
      default:
        return "unsupported wire type " + std::to_string(*type);
    }
  }

 private:
  const uint8_t* p_;
  const uint8_t* end_;
};

// Calls fn(number, type, payload, len, value) for every field of a message.
template <typename Fn>
std::string ForEachField(const uint8_t* p, size_t n, Fn fn) {
  Reader r(p, n);
  while (!r.done()) {
    uint32_t num = 0, type = 0;
    const uint8_t* payload = nullptr;
    size_t len = 0;
    uint64_t value = 0;
    std::string e = r.Field(&num, &type, &payload, &len, &value);
    if (!e.empty()) return e;
    e = fn(num, type, payload, len, value);
    if (!e.empty()) return e;
  }
  return "";
}

std::string ParseComputationDevice(const uint8_t* p, size_t n, std::vector<int64_t>* ids) {
  return ForEachField(p, n, [&](uint32_t num, uint32_t type, const uint8_t* payload, size_t len, uint64_t value) {
    if (num != 1) return std::string();
    if (type == 0) {                                   // unpacked repeated int64
      ids->push_back((int64_t)value);
      return std::string();
    }
    if (type == 2) {                                   // packed
      Reader r(payload, len);
      while (!r.done()) {
        uint64_t v = 0;
        std::string e = r.Varint(&v);
        if (!e.empty()) return e;
        ids->push_back((int64_t)v);
      }
      return std::string();
    }
    return std::string("replica_device_ids: unexpected wire type");
  });
}

std::string ParseDeviceAssignment(const uint8_t* p, size_t n, CompileOptionsInfo* out) {
  return ForEachField(p, n, [&](uint32_t num, uint32_t type, const uint8_t* payload, size_t len, uint64_t value) {
    if (num == 1 && type == 0) out->da_replicas = (int64_t)value;
    else if (num == 2 && type == 0) out->da_computations = (int64_t)value;
    else if (num == 3 && type == 2) {
      out->da_devices.emplace_back();
      return ParseComputationDevice(payload, len, &out->da_devices.back());
    }
    return std::string();
  });
}

std::string ParseBuildOptions(const uint8_t* p, size_t n, CompileOptionsInfo* out) {
  return ForEachField(p, n, [&](uint32_t num, uint32_t type, const uint8_t* payload, size_t len, uint64_t value) {
    if (num == 4 && type == 0) out->num_replicas = (int64_t)value;
    else if (num == 5 && type == 0) out->num_partitions = (int64_t)value;
    else if (num == 9 && type == 2) return ParseDeviceAssignment(payload, len, out);
    return std::string();
  });
}

}  // namespace

std::string ParseCompileOptions(const uint8_t* data, size_t size, CompileOptionsInfo* out) {
  *out = CompileOptionsInfo();
  if (!data || size == 0) return "";
  return ForEachField(data, size, [&](uint32_t num, uint32_t type, const uint8_t* payload, size_t len, uint64_t) {
    if (num == 3 && type == 2) return ParseBuildOptions(payload, len, out);
    return std::string();
  });
}

}  // namespace b200
