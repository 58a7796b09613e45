// model_artifact.cpp - compiled-model loading for the CUDA runtime: the
// CIM22ModelV1 descriptor of a model shared library (include/CIM22/Runtime/
// ModelABI.h), its Protobuf artifact (schema/cim22_model.proto, decoded here
// from the wire format without generated code), the artifact checks of
// runtime/src/ModelArtifact.cpp:101-186 with the same error texts, and a
// model session whose transactions run on the CUDA session of runner.cu
// (the role of cim22_session_load_shared / cim22_session_invoke,
// runtime/Runtime.cpp:73-114,292-339).
#include "cim_internal.h"

#include <dlfcn.h>

#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

namespace cim {
namespace {

// --------------------------------------------------------------------------
// Protobuf wire format: varint (0), 64-bit (1), length-delimited (2), 32-bit
// (5). Unknown fields are skipped; packed and unpacked repeated scalars are
// both accepted, as protobuf parsers do.

struct Wire {
  const uint8_t *p, *end;
  bool ok = true;

  bool more() const { return ok && p < end; }
  // Field number and wire type of the next field; field 0 is malformed.
  bool tag(int &field, int &type) {
    const uint64_t v = varint();
    field = static_cast<int>(v >> 3);
    type = static_cast<int>(v & 7);
    if (!ok || field == 0 || (v >> 3) > 0x1fffffff)
      ok = false;
    return ok;
  }
  uint64_t varint() {
    uint64_t v = 0;
    for (int shift = 0; shift < 64; shift += 7) {
      if (p >= end) {
        ok = false;
        return 0;
      }
      const uint8_t b = *p++;
      v |= static_cast<uint64_t>(b & 0x7f) << shift;
      if (!(b & 0x80))
        return v;
    }
    ok = false;
    return 0;
  }
  uint32_t fixed32() {
    if (end - p < 4) {
      ok = false;
      return 0;
    }
    uint32_t v;
    std::memcpy(&v, p, 4);
    p += 4;
    return v;
  }
  uint64_t fixed64() {
    if (end - p < 8) {
      ok = false;
      return 0;
    }
    uint64_t v;
    std::memcpy(&v, p, 8);
    p += 8;
    return v;
  }
  Wire sub() {
    const uint64_t n = varint();
    if (!ok || n > static_cast<uint64_t>(end - p)) {
      ok = false;
      return Wire{p, p, false};
    }
    Wire w{p, p + n};
    p += n;
    return w;
  }
  void skip(int type) {
    switch (type) {
    case 0:
      varint();
      break;
    case 1:
      fixed64();
      break;
    case 2:
      sub();
      break;
    case 5:
      fixed32();
      break;
    default:
      ok = false;
    }
  }
};

struct Opt64 {
  bool has = false;
  int64_t value = 0;
  void set(uint64_t v) {
    has = true;
    value = static_cast<int64_t>(v);
  }
};

// Repeated sfixed32 (packed or not).
bool read_sfixed32(Wire &w, int type, std::vector<int32_t> &out) {
  if (type == 2) {
    Wire s = w.sub();
    while (s.more())
      out.push_back(static_cast<int32_t>(s.fixed32()));
    return s.ok && w.ok;
  }
  if (type == 5)
    out.push_back(static_cast<int32_t>(w.fixed32()));
  else
    w.skip(type); // a wire type the field cannot have is an unknown field
  return w.ok;
}

std::string read_bytes(Wire &w) {
  Wire s = w.sub();
  return std::string(reinterpret_cast<const char *>(s.p), s.end - s.p);
}

struct PbWork {
  Opt64 work_id, core_slot, macro_slot;
  std::vector<int32_t> route;
};
struct PbGroup {
  Opt64 group_id;
  std::vector<PbWork> works;
};
struct PbWeight {
  Opt64 group_id, work_id, core_slot, macro_slot;
  std::string resource, values, exponents;
  std::vector<int32_t> route, words;
  int64_t data_type = 0;
};
struct PbPacket {
  int64_t kind = 0;
  std::vector<int32_t> route, test_core;
  Opt64 group_id, work_id, macro_slot, cache_address;
  int64_t data_type = 0;
};
struct PbInput {
  Opt64 group_id, work_id, macro_slot, input_slot, input_cache_address;
  int64_t data_type = 0;
};
struct PbReadback {
  Opt64 group_id, work_id, macro_slot, output_cache_address;
  std::vector<int32_t> route, test_core;
  int64_t data_type = 0;
};
struct PbTransaction {
  std::string target_profile;
  std::vector<PbGroup> groups;
  std::vector<PbWeight> weights;
  std::vector<PbPacket> packets;
  std::vector<PbInput> inputs;
  std::vector<PbReadback> readbacks;
  int64_t flits = 0;
};
struct PbTensor {
  std::vector<int64_t> dims;
  int64_t data_type = 0;
};
struct PbKernel {
  std::string name;
  bool has_transaction = false;
  PbTransaction transaction;
};
struct PbModel {
  uint64_t schema_version = 0;
  std::vector<PbTensor> inputs, outputs;
  std::vector<PbKernel> kernels;
  int64_t backend = 0;
};

// Proto DataType / PacketKind / RuntimeBackend values.
constexpr int64_t kPbInt8 = 1, kPbBF16 = 2, kPbFP32 = 3, kPbInt32 = 4;
constexpr int64_t kPbControl = 1, kPbWeight = 2, kPbWeightExponent = 3, kPbWork = 4,
                  kPbInputCacheWrite = 5, kPbReturnRoute = 6, kPbOutputCacheRead = 7;

bool parse(Wire w, PbWork &m) {
  while (w.more()) {
    int f, t;
    if (!w.tag(f, t))
      return false;
    if (f == 1 && t == 0) m.work_id.set(w.varint());
    else if (f == 2 && t == 0) m.core_slot.set(w.varint());
    else if (f == 3 && t == 0) m.macro_slot.set(w.varint());
    else if (f == 4) { if (!read_sfixed32(w, t, m.route)) return false; }
    else w.skip(t);
  }
  return w.ok;
}

bool parse(Wire w, PbGroup &m) {
  while (w.more()) {
    int f, t;
    if (!w.tag(f, t))
      return false;
    if (f == 1 && t == 0) m.group_id.set(w.varint());
    else if (f == 2 && t == 2) { m.works.emplace_back(); if (!parse(w.sub(), m.works.back())) return false; }
    else w.skip(t);
  }
  return w.ok;
}

bool parse(Wire w, PbWeight &m) {
  while (w.more()) {
    int f, t;
    if (!w.tag(f, t))
      return false;
    if (f == 1 && t == 0) m.group_id.set(w.varint());
    else if (f == 2 && t == 0) m.work_id.set(w.varint());
    else if (f == 3 && t == 0) m.core_slot.set(w.varint());
    else if (f == 4 && t == 0) m.macro_slot.set(w.varint());
    else if (f == 5 && t == 2) m.resource = read_bytes(w);
    else if (f == 6) { if (!read_sfixed32(w, t, m.route)) return false; }
    else if (f == 7) { if (!read_sfixed32(w, t, m.words)) return false; }
    else if (f == 8 && t == 2) m.values = read_bytes(w);
    else if (f == 9 && t == 2) m.exponents = read_bytes(w);
    else if (f == 10 && t == 0) m.data_type = static_cast<int32_t>(w.varint());
    else w.skip(t);
  }
  return w.ok;
}

bool parse(Wire w, PbPacket &m) {
  while (w.more()) {
    int f, t;
    if (!w.tag(f, t))
      return false;
    if (f == 1 && t == 0) m.kind = static_cast<int32_t>(w.varint());
    else if (f == 2) { if (!read_sfixed32(w, t, m.route)) return false; }
    else if (f == 3 && t == 0) m.group_id.set(w.varint());
    else if (f == 4 && t == 0) m.work_id.set(w.varint());
    else if (f == 5 && t == 0) m.macro_slot.set(w.varint());
    else if (f == 6 && t == 0) m.cache_address.set(w.varint());
    else if (f == 7) { if (!read_sfixed32(w, t, m.test_core)) return false; }
    else if (f == 8 && t == 0) m.data_type = static_cast<int32_t>(w.varint());
    else w.skip(t);
  }
  return w.ok;
}

bool parse(Wire w, PbInput &m) {
  while (w.more()) {
    int f, t;
    if (!w.tag(f, t))
      return false;
    if (f == 1 && t == 0) m.group_id.set(w.varint());
    else if (f == 2 && t == 0) m.work_id.set(w.varint());
    else if (f == 3 && t == 0) m.macro_slot.set(w.varint());
    else if (f == 4 && t == 0) m.input_slot.set(w.varint());
    else if (f == 5 && t == 0) m.data_type = static_cast<int32_t>(w.varint());
    else if (f == 6 && t == 0) m.input_cache_address.set(w.varint());
    else w.skip(t);
  }
  return w.ok;
}

bool parse(Wire w, PbReadback &m) {
  while (w.more()) {
    int f, t;
    if (!w.tag(f, t))
      return false;
    if (f == 1 && t == 0) m.group_id.set(w.varint());
    else if (f == 2 && t == 0) m.work_id.set(w.varint());
    else if (f == 3 && t == 0) m.macro_slot.set(w.varint());
    else if (f == 4 && t == 0) m.output_cache_address.set(w.varint());
    else if (f == 5) { if (!read_sfixed32(w, t, m.route)) return false; }
    else if (f == 6) { if (!read_sfixed32(w, t, m.test_core)) return false; }
    else if (f == 7 && t == 0) m.data_type = static_cast<int32_t>(w.varint());
    else w.skip(t);
  }
  return w.ok;
}

bool parse(Wire w, PbTransaction &m) {
  while (w.more()) {
    int f, t;
    if (!w.tag(f, t))
      return false;
    if (f == 1 && t == 2) m.target_profile = read_bytes(w);
    else if (f == 2 && t == 2) { m.groups.emplace_back(); if (!parse(w.sub(), m.groups.back())) return false; }
    else if (f == 3 && t == 2) { m.weights.emplace_back(); if (!parse(w.sub(), m.weights.back())) return false; }
    else if (f == 4 && t == 2) { m.packets.emplace_back(); if (!parse(w.sub(), m.packets.back())) return false; }
    else if (f == 5 && t == 2) { m.inputs.emplace_back(); if (!parse(w.sub(), m.inputs.back())) return false; }
    else if (f == 6 && t == 2) { m.readbacks.emplace_back(); if (!parse(w.sub(), m.readbacks.back())) return false; }
    else if (f == 7 && t == 2) { Wire s = w.sub(); while (s.more()) { s.fixed64(); ++m.flits; } if (!s.ok) return false; }
    else if (f == 7 && t == 1) { w.fixed64(); ++m.flits; }
    else w.skip(t);
  }
  return w.ok;
}

bool parse(Wire w, PbTensor &m) {
  while (w.more()) {
    int f, t;
    if (!w.tag(f, t))
      return false;
    if (f == 1 && t == 2) { Wire s = w.sub(); while (s.more()) m.dims.push_back(static_cast<int64_t>(s.varint())); if (!s.ok) return false; }
    else if (f == 1 && t == 0) m.dims.push_back(static_cast<int64_t>(w.varint()));
    else if (f == 2 && t == 0) m.data_type = static_cast<int32_t>(w.varint());
    else w.skip(t);
  }
  return w.ok;
}

bool parse(Wire w, PbKernel &m) {
  while (w.more()) {
    int f, t;
    if (!w.tag(f, t))
      return false;
    if (f == 1 && t == 2) m.name = read_bytes(w);
    else if (f == 2 && t == 2) { m.has_transaction = true; if (!parse(w.sub(), m.transaction)) return false; }
    else w.skip(t);
  }
  return w.ok;
}

bool parse(Wire w, PbModel &m) {
  while (w.more()) {
    int f, t;
    if (!w.tag(f, t))
      return false;
    if (f == 1 && t == 0) m.schema_version = w.varint();
    else if (f == 2 && t == 2) { m.inputs.emplace_back(); if (!parse(w.sub(), m.inputs.back())) return false; }
    else if (f == 3 && t == 2) { m.outputs.emplace_back(); if (!parse(w.sub(), m.outputs.back())) return false; }
    else if (f == 4 && t == 2) { m.kernels.emplace_back(); if (!parse(w.sub(), m.kernels.back())) return false; }
    else if (f == 5 && t == 0) m.backend = static_cast<int32_t>(w.varint());
    else w.skip(t);
  }
  return w.ok;
}

// --------------------------------------------------------------------------
// Artifact checks (runtime/src/ModelArtifact.cpp:91-186), same error texts.

std::string invalid(const std::string &reason) {
  return "invalid CIM22 Protobuf model: " + reason + "; recompile the model";
}

bool valid_type(int64_t t) { return t == kPbInt8 || t == kPbBF16; }

template <typename B> bool has_binding(const B &b) {
  return b.group_id.has && b.work_id.has && b.macro_slot.has;
}

std::string validate_transaction(const PbTransaction &t, bool require_usb) {
  if (t.target_profile != "cim22-4x5-v1")
    return invalid("unsupported transaction profile");
  using Key = std::pair<int64_t, int64_t>;
  std::set<int64_t> groups;
  std::map<Key, const PbWork *> works;
  for (const auto &g : t.groups) {
    if (!g.group_id.has || g.group_id.value < 0 || !groups.insert(g.group_id.value).second ||
        g.works.empty())
      return invalid("missing/duplicate group or empty works");
    std::set<Key> placements;
    for (const auto &w : g.works)
      if (!w.work_id.has || !w.core_slot.has || !w.macro_slot.has || w.work_id.value < 0 ||
          w.core_slot.value < 0 || w.core_slot.value >= 20 || w.macro_slot.value < 0 ||
          w.macro_slot.value >= 2 || w.route.size() != 6 ||
          !works.emplace(Key{g.group_id.value, w.work_id.value}, &w).second ||
          !placements.emplace(w.core_slot.value, w.macro_slot.value).second)
        return invalid("missing/duplicate work, placement or route length");
  }
  if (works.empty() || t.flits == 0)
    return invalid("empty transaction works/flits");
  std::map<Key, const PbWeight *> weights;
  std::map<Key, const PbInput *> inputs;
  std::map<Key, const PbReadback *> readbacks;
  auto placement = [&](const auto &b) {
    if (!has_binding(b))
      return false;
    auto found = works.find({b.group_id.value, b.work_id.value});
    return found != works.end() && b.macro_slot.value == found->second->macro_slot.value &&
           valid_type(b.data_type);
  };
  for (const auto &w : t.weights) {
    if (!placement(w) || !w.core_slot.has)
      return invalid("weight binding, array length or datatype");
    const PbWork *work = works.at({w.group_id.value, w.work_id.value});
    if (w.core_slot.value != work->core_slot.value || w.resource.empty() ||
        w.route.size() != 6 || w.words.size() != 256 || w.values.size() != 1024 ||
        w.exponents.size() != 16 || w.route != work->route ||
        !weights.emplace(Key{w.group_id.value, w.work_id.value}, &w).second)
      return invalid("weight binding, array length or datatype");
  }
  for (const auto &b : t.inputs)
    if (!placement(b) || !b.input_slot.has || b.input_slot.value < 0 ||
        (require_usb && !b.input_cache_address.has) || b.input_cache_address.value < 0 ||
        b.input_cache_address.value >= 8 ||
        !inputs.emplace(Key{b.group_id.value, b.work_id.value}, &b).second)
      return invalid("input binding or datatype");
  for (const auto &b : t.readbacks) {
    if (!placement(b) || !b.output_cache_address.has || b.output_cache_address.value < 0 ||
        b.output_cache_address.value >= 8 || b.route.size() != 6 || b.test_core.size() != 3 ||
        b.route != works.at({b.group_id.value, b.work_id.value})->route ||
        !readbacks.emplace(Key{b.group_id.value, b.work_id.value}, &b).second)
      return invalid("readback binding, array length or datatype");
  }
  if (weights.size() != works.size() || inputs.size() != works.size() ||
      readbacks.size() != works.size())
    return invalid("incomplete work bindings");
  for (const auto &[key, weight] : weights)
    if (weight->data_type != inputs.at(key)->data_type ||
        weight->data_type != readbacks.at(key)->data_type)
      return invalid("inconsistent work datatypes");
  std::map<Key, std::set<int64_t>> kinds;
  for (size_t index = 0; index < t.packets.size(); ++index) {
    const PbPacket &p = t.packets[index];
    if (p.kind < kPbControl || p.kind > kPbOutputCacheRead || !valid_type(p.data_type) ||
        !has_binding(p) || !p.cache_address.has || p.route.size() != 6 ||
        p.test_core.size() != 3 || p.group_id.value < -1 || p.work_id.value < -1 ||
        p.macro_slot.value < -1 || p.macro_slot.value >= 2 || p.cache_address.value < -1 ||
        p.cache_address.value >= 8)
      return invalid("packet enum, missing field or array/address");
    if (p.group_id.value >= 0 && !groups.count(p.group_id.value))
      return invalid("packet references unknown group");
    if (p.work_id.value >= 0 && !placement(p))
      return invalid("packet references unknown work/placement");
    if (p.kind == kPbWork) {
      if (p.group_id.value < 0)
        return invalid("work packet missing group");
    } else if (p.kind != kPbControl && p.work_id.value < 0) {
      return invalid("packet missing work binding");
    }
    const Key key{p.group_id.value, p.work_id.value};
    if (p.work_id.value >= 0 && p.data_type != weights.at(key)->data_type)
      return invalid("packet datatype differs from work");
    kinds[key].insert(p.kind);
    if (p.work_id.value >= 0) {
      const auto &route = p.kind == kPbReturnRoute || p.kind == kPbOutputCacheRead
                              ? readbacks.at(key)->route
                              : weights.at(key)->route;
      if (p.kind != kPbControl && p.kind != kPbWork && p.route != route)
        return invalid("packet route differs from binding");
      if (p.kind == kPbReturnRoute) {
        if (p.test_core != readbacks.at(key)->test_core)
          return invalid("packet test core differs from readback");
        if (index + 2 >= t.packets.size())
          return invalid("incomplete readback packet sequence");
        for (size_t offset = 1; offset <= 2; ++offset) {
          const PbPacket &next = t.packets[index + offset];
          if (next.kind != (offset == 1 ? kPbControl : kPbOutputCacheRead) ||
              next.group_id.value != p.group_id.value ||
              next.work_id.value != p.work_id.value ||
              next.macro_slot.value != p.macro_slot.value || next.data_type != p.data_type ||
              next.route.size() != 6 || next.route != route)
            return invalid("inconsistent readback packet sequence");
        }
      }
    }
    if (p.kind == kPbOutputCacheRead &&
        p.cache_address.value != readbacks.at(key)->output_cache_address.value)
      return invalid("packet readback address differs from binding");
  }
  for (const auto &[key, weight] : weights) {
    const auto &k = kinds[key];
    for (int64_t kind : {kPbWeight, kPbInputCacheWrite, kPbReturnRoute, kPbControl,
                         kPbOutputCacheRead})
      if (!k.count(kind))
        return invalid("work binding has no matching packet");
    if (weight->data_type == kPbBF16 && !k.count(kPbWeightExponent))
      return invalid("BF16 weight binding has no exponent packet");
  }
  return "";
}

std::string validate(const PbModel &m) {
  if (m.backend != 0 && m.backend != 1)
    return invalid("unsupported runtime backend");
  for (const auto *tensors : {&m.inputs, &m.outputs})
    for (const auto &tensor : *tensors) {
      if (tensor.data_type != kPbInt8 && tensor.data_type != kPbFP32 &&
          tensor.data_type != kPbInt32)
        return invalid("boundary requires contiguous CPU INT8, FP32 or INT32 tensors");
      int64_t elements = 1;
      for (int64_t dim : tensor.dims)
        if (dim <= 0 || __builtin_mul_overflow(elements, dim, &elements))
          return invalid("static tensor shape/element count");
    }
  std::set<std::string> names;
  for (const auto &k : m.kernels) {
    if (k.name.empty() || !names.insert(k.name).second || !k.has_transaction)
      return invalid("missing/duplicate kernel name or transaction");
    const std::string e = validate_transaction(k.transaction, m.backend == 1);
    if (!e.empty())
      return e;
  }
  return "";
}

std::string decode(const uint8_t *data, uint64_t size, PbModel &model) {
  if (!data || size == 0 || size > 0x7fffffffu || !parse(Wire{data, data + size}, model))
    return invalid("malformed data (old custom binary is unsupported)");
  return validate(model);
}

// Owned native copy of one transaction in the C ABI layout.
struct NativeTransaction {
  std::vector<std::vector<cim22_work>> works;
  std::vector<cim22_group> groups;
  std::vector<std::vector<int32_t>> words;
  std::vector<cim22_static_weight> weights;
  std::vector<cim22_frame_packet> packets;
  std::vector<cim22_input_binding> inputs;
  std::vector<cim22_readback_binding> readbacks;
  std::string profile;
  cim22_transaction c{};
};

int32_t native_type(int64_t t) { return t == kPbBF16 ? CIM22_DATA_BF16 : CIM22_DATA_INT8; }
int32_t native_kind(int64_t k) { return static_cast<int32_t>(k - 1); } // CONTROL=1 -> 0 ...

template <size_t N> void copy_array(const std::vector<int32_t> &from, int32_t (&to)[N]) {
  for (size_t i = 0; i < N; ++i)
    to[i] = i < from.size() ? from[i] : 0;
}

void to_native(const PbTransaction &t, NativeTransaction &n) {
  n.profile = t.target_profile;
  n.works.reserve(t.groups.size());
  for (const auto &g : t.groups) {
    std::vector<cim22_work> ws;
    for (const auto &w : g.works) {
      cim22_work cw{};
      cw.work_id = w.work_id.value;
      cw.core_slot = w.core_slot.value;
      cw.macro_slot = w.macro_slot.value;
      copy_array(w.route, cw.route);
      ws.push_back(cw);
    }
    n.works.push_back(std::move(ws));
  }
  for (size_t i = 0; i < t.groups.size(); ++i)
    n.groups.push_back(cim22_group{t.groups[i].group_id.value, n.works[i].data(),
                                   static_cast<int64_t>(n.works[i].size())});
  n.words.reserve(t.weights.size());
  for (const auto &w : t.weights) {
    n.words.push_back(w.words);
    cim22_static_weight cw{};
    cw.group_id = w.group_id.value;
    cw.work_id = w.work_id.value;
    cw.core_slot = w.core_slot.value;
    cw.macro_slot = w.macro_slot.value;
    copy_array(w.route, cw.route);
    cw.words = n.words.back().data();
    cw.num_words = static_cast<int64_t>(n.words.back().size());
    std::memcpy(cw.values, w.values.data(), 1024);
    std::memcpy(cw.exponents, w.exponents.data(), 16);
    cw.data_type = native_type(w.data_type);
    n.weights.push_back(cw);
  }
  for (const auto &p : t.packets) {
    cim22_frame_packet cp{};
    cp.kind = native_kind(p.kind);
    copy_array(p.route, cp.route);
    cp.group_id = p.group_id.value;
    cp.work_id = p.work_id.value;
    cp.macro_slot = p.macro_slot.value;
    cp.cache_address = p.cache_address.value;
    copy_array(p.test_core, cp.test_core);
    cp.data_type = native_type(p.data_type);
    n.packets.push_back(cp);
  }
  for (const auto &b : t.inputs)
    n.inputs.push_back(cim22_input_binding{b.group_id.value, b.work_id.value,
                                           b.macro_slot.value, b.input_slot.value,
                                           native_type(b.data_type),
                                           b.input_cache_address.value});
  for (const auto &b : t.readbacks) {
    cim22_readback_binding cb{};
    cb.group_id = b.group_id.value;
    cb.work_id = b.work_id.value;
    cb.macro_slot = b.macro_slot.value;
    cb.output_cache_address = b.output_cache_address.value;
    copy_array(b.route, cb.route);
    copy_array(b.test_core, cb.test_core);
    cb.data_type = native_type(b.data_type);
    n.readbacks.push_back(cb);
  }
  n.c.target_profile = n.profile.c_str();
  n.c.target_profile_version = 1;
  n.c.execution_plan_version = 1;
  n.c.groups = n.groups.data();
  n.c.num_groups = static_cast<int64_t>(n.groups.size());
  n.c.weights = n.weights.data();
  n.c.num_weights = static_cast<int64_t>(n.weights.size());
  n.c.packets = n.packets.data();
  n.c.num_packets = static_cast<int64_t>(n.packets.size());
  n.c.inputs = n.inputs.data();
  n.c.num_inputs = static_cast<int64_t>(n.inputs.size());
  n.c.readbacks = n.readbacks.data();
  n.c.num_readbacks = static_cast<int64_t>(n.readbacks.size());
}

// The model library's descriptor (include/CIM22/Runtime/ModelABI.h).
struct ModelV1 {
  uint64_t abi_version;
  const uint8_t *data;
  uint64_t data_size;
  void (*invoke)(void **);
};

// Make this library's dispatch symbols visible to model libraries loaded
// with RTLD_LOCAL: promote it to the global scope (it may have been opened
// with RTLD_LOCAL, as ctypes does).
void promote_self() {
  static std::once_flag once;
  std::call_once(once, [] {
    Dl_info info{};
    if (dladdr(reinterpret_cast<void *>(&promote_self), &info) && info.dli_fname)
      dlopen(info.dli_fname, RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);
  });
}

} // namespace
} // namespace cim

using namespace cim;

struct cim22_cuda_model {
  void *library = nullptr;
  void (*invoke)(void **) = nullptr;
  cim22_cuda_session *session = nullptr;
  std::vector<std::vector<int64_t>> shapes;
  std::vector<int64_t> types;
  int64_t num_inputs = 0;
  int64_t backend = 0;
  bool counted = false; // the session's dispatch counter belongs to the last invoke
  std::string error;
  std::mutex mutex;
};

extern "C" {

int cim22_cuda_model_validate(const uint8_t *data, uint64_t size, char *error,
                              size_t error_capacity) {
  PbModel model;
  const std::string e = decode(data, size, model);
  if (!e.empty()) {
    copy_error(e, error, error_capacity);
    return 1;
  }
  return 0;
}

cim22_cuda_model *cim22_cuda_model_load_shared(const char *path, int device, char *error,
                                               size_t error_capacity) {
  promote_self();
  void *library = path ? dlopen(path, RTLD_NOW | RTLD_LOCAL) : nullptr;
  if (!library) {
    const char *why = path ? dlerror() : "missing model library path";
    copy_error(why ? why : "cannot open model library", error, error_capacity);
    return nullptr;
  }
  auto get = reinterpret_cast<const ModelV1 *(*)()>(dlsym(library, "cim22_model_v1"));
  const ModelV1 *descriptor = get ? get() : nullptr;
  if (!descriptor || descriptor->abi_version != 1 || !descriptor->data || !descriptor->invoke) {
    copy_error("incompatible CIM22 model ABI", error, error_capacity);
    dlclose(library);
    return nullptr;
  }
  PbModel pb;
  const std::string e = decode(descriptor->data, descriptor->data_size, pb);
  if (!e.empty()) {
    copy_error(e, error, error_capacity);
    dlclose(library);
    return nullptr;
  }
  auto *model = new cim22_cuda_model();
  model->library = library;
  model->invoke = descriptor->invoke;
  model->backend = pb.backend;
  model->num_inputs = static_cast<int64_t>(pb.inputs.size());
  for (const auto *tensors : {&pb.inputs, &pb.outputs})
    for (const auto &t : *tensors) {
      model->shapes.push_back(t.dims);
      model->types.push_back(t.data_type);
    }
  model->session = cim22_cuda_session_create(device, error, error_capacity);
  if (!model->session) {
    cim22_cuda_model_destroy(model);
    return nullptr;
  }
  // The CUDA session replaces the software backend only; a USB-backend model
  // fails each dispatch as the reference does before configure_usb.
  if (pb.backend == 1)
    session_refuse_dispatch(model->session,
                            "USB runtime is not configured; call configure_usb first");
  for (const auto &k : pb.kernels) {
    NativeTransaction native;
    to_native(k.transaction, native);
    if (cim22_cuda_session_add_transaction(model->session, &native.c, k.name.c_str(), error,
                                           error_capacity) < 0) {
      cim22_cuda_model_destroy(model);
      return nullptr;
    }
  }
  return model;
}

void cim22_cuda_model_destroy(cim22_cuda_model *model) {
  if (!model)
    return;
  if (model->session)
    cim22_cuda_session_destroy(model->session);
  if (model->library)
    dlclose(model->library);
  delete model;
}

int64_t cim22_cuda_model_num_inputs(const cim22_cuda_model *model) {
  return model ? model->num_inputs : -1;
}

int64_t cim22_cuda_model_num_outputs(const cim22_cuda_model *model) {
  return model ? static_cast<int64_t>(model->shapes.size()) - model->num_inputs : -1;
}

int64_t cim22_cuda_model_rank(const cim22_cuda_model *model, int64_t tensor) {
  if (!model || tensor < 0 || tensor >= static_cast<int64_t>(model->shapes.size()))
    return -1;
  return static_cast<int64_t>(model->shapes[tensor].size());
}

int64_t cim22_cuda_model_dim(const cim22_cuda_model *model, int64_t tensor, int64_t axis) {
  if (!model || tensor < 0 || tensor >= static_cast<int64_t>(model->shapes.size()) ||
      axis < 0 || axis >= static_cast<int64_t>(model->shapes[tensor].size()))
    return -1;
  return model->shapes[tensor][axis];
}

int64_t cim22_cuda_model_dtype(const cim22_cuda_model *model, int64_t tensor) {
  if (!model || tensor < 0 || tensor >= static_cast<int64_t>(model->types.size()))
    return -1;
  return model->types[tensor];
}

int64_t cim22_cuda_model_num_transactions(const cim22_cuda_model *model) {
  return model ? cim22_cuda_session_num_transactions(model->session) : -1;
}

uint64_t cim22_cuda_model_dispatch_count(const cim22_cuda_model *model) {
  return model && model->counted ? cim22_cuda_session_dispatch_count(model->session) : 0;
}

const char *cim22_cuda_model_error(const cim22_cuda_model *model) {
  return model ? model->error.c_str() : "null session";
}

int cim22_cuda_model_invoke(cim22_cuda_model *model, void **buffers, const int64_t *counts,
                            int64_t num_buffers) {
  if (!model)
    return 1;
  std::lock_guard<std::mutex> lock(model->mutex);
  model->error.clear();
  model->counted = false;
  if (!buffers || !counts || num_buffers != static_cast<int64_t>(model->shapes.size())) {
    model->error = "runtime buffer count mismatch";
    return 1;
  }
  // MLIR ranked descriptors: allocated and aligned pointers, offset 0, sizes,
  // row-major strides (runtime/Runtime.cpp:303-331).
  std::vector<std::vector<int64_t>> descriptors(num_buffers);
  std::vector<void *> pointers(num_buffers), packed(num_buffers);
  for (int64_t i = 0; i < num_buffers; ++i) {
    const auto &shape = model->shapes[i];
    auto &desc = descriptors[i];
    desc.assign(3 + 2 * shape.size(), 0);
    std::memcpy(desc.data(), &buffers[i], sizeof(void *));
    std::memcpy(desc.data() + 1, &buffers[i], sizeof(void *));
    int64_t elements = 1;
    for (int64_t dim = static_cast<int64_t>(shape.size()) - 1; dim >= 0; --dim) {
      desc[3 + dim] = shape[dim];
      desc[3 + shape.size() + dim] = elements;
      if (__builtin_mul_overflow(elements, shape[dim], &elements)) {
        model->error = "runtime shape element count overflows";
        return 1;
      }
    }
    if (!buffers[i] || counts[i] != elements) {
      model->error = "runtime buffer element count mismatch";
      return 1;
    }
    pointers[i] = desc.data();
    packed[i] = &pointers[i];
  }
  cim22_cuda_session_begin_invoke(model->session);
  model->counted = true;
  model->invoke(packed.data());
  if (cim22_cuda_session_end_invoke(model->session)) {
    model->error = cim22_cuda_session_error(model->session);
    return 1;
  }
  return 0;
}

} // extern "C"
