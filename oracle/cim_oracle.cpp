// ORACLE - test infrastructure only.
//
// CPU restatement of mlir-cim22's software-simulated CIM execution path, used
// as the parity checker for the CUDA backend. Only tests/, the smoke check in
// __graft_entry__.py and bench.py's CPU baseline legs load this library; the
// product never links, imports or executes it.
//
// What it restates (paths relative to the mlir-cim22 source tree):
//   * BF16 numeric support: prealignBF16Vector, prealignBF16WeightTile and
//     int21ToBF16 (lib/Support/BF16Support.cpp:18-96).
//   * BF16 peripherals: scaleBF16Input, effectiveBF16Exponent,
//     compensateBF16Output, validateBF16Group, prepareBF16Input,
//     hasBF16Support and restoreBF16Output
//     (lib/Execution/BF16Compensation.cpp:15-164).
//   * The software runner: Plan construction with wave batching and readback
//     partitioning (lib/Execution/CIMSoftwareRunner.cpp:39-287), runImpl with
//     weight residency, Macro output Caches, trace events and readback
//     publication (:289-482), and the weight catalog/residency table
//     (include/CIM22/Execution/WeightResidency.h:28-92).
//   * The Host code the compiler emits around the tiles: K/N tiling with zero
//     padding and the f32/i32 cross-K accumulation
//     (lib/Conversion/LinalgToCIM/Passes.cpp:760-857,1054-1059), the sign-split
//     decomposition and merge (:2304-2420), the FP32->BF16 preparation
//     (:2422-2476) and the INT8 range proof (:592-627).
//
// BF16 arithmetic follows the reference's APFloat usage by computing the exact
// value in binary64 and rounding it once to BF16 with round-to-nearest-even,
// written here from the IEEE 754 definitions.

#include "../include/cim22_cuda.h"

#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <thread>
#include <vector>

namespace oracle {

constexpr int kIn = 64;
constexpr int kOut = 16;
constexpr int kCores = 20;
constexpr int kMacros = 2;
constexpr int kCacheRows = 8;
constexpr int32_t kI21Min = -(1 << 20);
constexpr int32_t kI21MaxExclusive = 1 << 20;

enum Mode { kNone = 0, kLegacy = 1, kSignSplit = 2 };

// ---------------------------------------------------------------------------
// BF16 <-> binary64.

double bf16ToDouble(uint16_t bits) {
  const int exponent = (bits >> 7) & 0xff;
  const int fraction = bits & 0x7f;
  double magnitude;
  if (exponent == 0xff)
    magnitude = fraction ? NAN : INFINITY;
  else if (exponent == 0)
    magnitude = std::ldexp(static_cast<double>(fraction), -133);
  else
    magnitude = std::ldexp(static_cast<double>(128 + fraction), exponent - 134);
  return (bits & 0x8000) ? -magnitude : magnitude;
}

// Round a binary64 value to BF16, ties to even; overflow gives infinity.
uint16_t doubleToBF16(double value) {
  if (std::isnan(value))
    return 0x7fc0;
  const uint16_t sign = std::signbit(value) ? 0x8000 : 0;
  const double magnitude = std::fabs(value);
  if (std::isinf(magnitude))
    return sign | 0x7f80;
  if (magnitude == 0)
    return sign;
  int e2 = 0;
  std::frexp(magnitude, &e2); // magnitude = f * 2^e2, f in [0.5, 1)
  const int unbiased = e2 - 1;
  // Spacing of BF16 values around the magnitude: 2^(unbiased-7) when normal,
  // 2^-133 in the subnormal range.
  const int quantum = unbiased >= -126 ? unbiased - 7 : -133;
  const double units = std::nearbyint(std::ldexp(magnitude, -quantum));
  const double rounded = std::ldexp(units, quantum);
  if (rounded < std::ldexp(1.0, -126))
    return sign | static_cast<uint16_t>(units); // subnormal or zero
  std::frexp(rounded, &e2);
  const int biased = e2 - 1 + 127;
  if (biased >= 255)
    return sign | 0x7f80;
  const double significand = std::ldexp(rounded, -(e2 - 1)); // [1, 2)
  const int fraction = static_cast<int>((significand - 1.0) * 128.0);
  return sign | static_cast<uint16_t>(biased << 7) |
         static_cast<uint16_t>(fraction);
}

// FP32 -> BF16 with round-to-nearest-even (arith.truncf / APFloat convert).
uint16_t floatToBF16(float value) {
  return doubleToBF16(static_cast<double>(value));
}

float bf16ToFloat(uint16_t bits) {
  uint32_t word = static_cast<uint32_t>(bits) << 16;
  float value;
  std::memcpy(&value, &word, sizeof value);
  return value;
}

bool bf16Finite(uint16_t bits) { return ((bits >> 7) & 0xff) != 0xff; }

// ---------------------------------------------------------------------------
// lib/Support/BF16Support.cpp

struct Prealigned {
  uint8_t exponent = 0;
  std::array<int8_t, kIn> mantissas{};
};

// BF16Support.cpp:18-54: supplier ExpPrealign.
Prealigned prealign(const std::array<uint16_t, kIn> &values) {
  Prealigned out;
  for (uint16_t v : values)
    out.exponent = std::max<uint8_t>(out.exponent, (v >> 7) & 0xff);
  for (int i = 0; i < kIn; ++i) {
    const uint16_t v = values[i];
    const bool negative = v >> 15;
    const int e = (v >> 7) & 0xff;
    int mantissa = v & 0x7f;
    int gap;
    if (e == 0) {
      gap = out.exponent - 1; // subnormals use exp_max - 1 (may be -1)
    } else {
      gap = out.exponent - e;
      mantissa |= 0x80;
    }
    const int complemented = negative ? ((~mantissa + 1) & 0xff) : mantissa;
    int aligned = 0;
    if (gap < 7) {
      const int shifted = (complemented >> (gap + 1)) & 0xff;
      aligned = (shifted + (negative ? 0x80 : 0)) & 0xff;
    }
    out.mantissas[i] = static_cast<int8_t>(static_cast<uint8_t>(aligned));
  }
  return out;
}

// BF16Support.cpp:56-70.
void prealignTile(const uint16_t *bits /*[16][64]*/, int8_t *values,
                  uint8_t *exponents) {
  for (int lane = 0; lane < kOut; ++lane) {
    std::array<uint16_t, kIn> row;
    std::copy_n(bits + lane * kIn, kIn, row.begin());
    Prealigned p = prealign(row);
    exponents[lane] = p.exponent;
    std::copy(p.mantissas.begin(), p.mantissas.end(), values + lane * kIn);
  }
}

// BF16Support.cpp:72-96: keep the top eight magnitude bits (truncating),
// exponent Ew + Ei + 1 + shift clamped to [0, 255].
uint16_t int21ToBF16(int32_t value, uint8_t we, uint8_t ie) {
  const bool negative = value < 0;
  const int64_t magnitude = negative ? -static_cast<int64_t>(value) : value;
  int shift = 0;
  uint64_t kept = 0;
  if (magnitude != 0) {
    int high = 0;
    for (int64_t r = magnitude; r > 1; r >>= 1)
      ++high;
    shift = high - 7;
    kept = shift >= 0 ? static_cast<uint64_t>(magnitude) >> shift
                      : static_cast<uint64_t>(magnitude) << -shift;
  }
  const int exponent = std::clamp(static_cast<int>(we) + ie + 1 + shift, 0, 255);
  return static_cast<uint16_t>((negative ? 0x8000 : 0) | (exponent << 7) |
                               (kept & 0x7f));
}

// ---------------------------------------------------------------------------
// lib/Execution/BF16Compensation.cpp

// :15-19 scalbn in BF16 with round-to-nearest-even.
uint16_t scaleBF16(uint16_t bits, int exponent) {
  return doubleToBF16(std::ldexp(bf16ToDouble(bits), exponent));
}

// :23-31
int effectiveExponent(uint16_t maximum) {
  const int e = (maximum >> 7) & 0xff;
  if (e)
    return e;
  int high = 0;
  for (int f = maximum & 0x7f; f > 1; f >>= 1)
    ++high;
  return high - 6;
}

// :33-51
bool compensate(uint16_t bits, int exponent, uint16_t &out,
                std::string &error) {
  if (!bf16Finite(bits)) {
    error = "CIM BF16 chip output is not finite";
    return false;
  }
  const double scaled = std::ldexp(bf16ToDouble(bits), exponent);
  if (!std::isfinite(scaled)) {
    error = "CIM BF16 compensation is not finite";
    return false;
  }
  out = doubleToBF16(scaled);
  if (!bf16Finite(out)) {
    error = "CIM BF16 compensated tile exceeds BF16";
    return false;
  }
  return true;
}

struct Prepared {
  std::array<uint16_t, kIn> chip{};
  Prealigned aligned;
  uint64_t support = 0;
  int effective = 0;
  int scaleDelta = 0;
};

// :84-137
bool prepareInput(const uint16_t *input, int mode, Prepared &out,
                  std::string &error) {
  out = Prepared{};
  std::copy_n(input, kIn, out.chip.begin());
  for (int i = 0; i < kIn; ++i)
    if (((input[i] >> 7) & 0xff) == 0xff) {
      error = "CIM BF16 input does not support NaN or infinity";
      return false;
    }
  if (mode == kSignSplit) {
    uint16_t maximum = 0;
    for (uint16_t &v : out.chip) {
      if ((v & 0x8000) && (v & 0x7fff)) {
        error = "CIM nonnegative BF16 mode rejects negative inputs";
        return false;
      }
      v &= 0x7fff;
      maximum = std::max(maximum, v);
    }
    if (!maximum)
      return true;
    out.effective = effectiveExponent(maximum);
    const int shift = 127 - out.effective;
    if (shift)
      for (uint16_t &v : out.chip)
        v = scaleBF16(v, shift);
    out.aligned = prealign(out.chip);
    if (out.aligned.exponent != 127) {
      error = "CIM nonnegative BF16 normalization did not produce input "
              "exponent 127";
      return false;
    }
    for (int k = 0; k < kIn; ++k) {
      if (out.aligned.mantissas[k] < 0) {
        error = "CIM nonnegative BF16 normalization changed sign";
        return false;
      }
      if (out.aligned.mantissas[k])
        out.support |= uint64_t{1} << k;
    }
    return true;
  }
  out.aligned = prealign(out.chip);
  if (mode == kLegacy) {
    out.scaleDelta = std::max(0, static_cast<int>(out.aligned.exponent) - 240);
    if (out.scaleDelta) {
      const auto original = out.aligned.mantissas;
      for (uint16_t &v : out.chip)
        v = scaleBF16(v, -out.scaleDelta);
      out.aligned = prealign(out.chip);
      if (out.aligned.exponent > 240 || out.aligned.mantissas != original) {
        error = "CIM legacy BF16 group scaling changed prealigned input "
                "mantissas";
        return false;
      }
    }
  }
  return true;
}

// :55-81
bool validateGroup(const int8_t *values /*[16][64]*/,
                   const uint8_t *exponents, const Prepared &input, int mode,
                   std::string &error) {
  if (mode == kLegacy &&
      std::all_of(input.aligned.mantissas.begin(),
                  input.aligned.mantissas.end(),
                  [](int8_t v) { return v == -128; })) {
    for (int lane = 0; lane < kOut; ++lane)
      if (std::all_of(values + lane * kIn, values + (lane + 1) * kIn,
                      [](int8_t v) { return v == -128; })) {
        error = "CIM BF16 result exceeds signed i21 range";
        return false;
      }
  }
  if (mode != kSignSplit)
    return true;
  for (int lane = 0; lane < kOut; ++lane)
    if (exponents[lane] == 255) {
      error = "CIM nonnegative BF16 weight exponent is not finite";
      return false;
    }
  uint8_t bits = 0;
  for (int i = 0; i < kOut * kIn; ++i)
    bits |= static_cast<uint8_t>(values[i]);
  if (bits & 0x80) {
    error = "CIM nonnegative BF16 mode rejects negative prepared weights";
    return false;
  }
  return true;
}

// :141-146
bool hasSupport(const int8_t *lane, uint64_t support) {
  for (; support; support &= support - 1)
    if (lane[__builtin_ctzll(support)])
      return true;
  return false;
}

// :149-164
bool restoreOutput(uint16_t bits, uint8_t we, bool support,
                   const Prepared &input, int mode, uint16_t &out,
                   std::string &error) {
  if (mode == kNone) {
    out = bits;
    return true;
  }
  if (mode == kSignSplit && !support) {
    out = 0;
    return true;
  }
  const int exponent = mode == kSignSplit
                           ? static_cast<int>(we) + input.effective - 260
                           : static_cast<int>(we) + input.scaleDelta - 133;
  return compensate(bits, exponent, out, error);
}

// ---------------------------------------------------------------------------
// Transaction model (include/CIM22/Execution/CIMExecutable.h).

struct Weight {
  int64_t group = -1, work = -1, core = -1, macro = -1;
  std::array<int32_t, 6> route{};
  std::vector<int32_t> words;
  std::array<int8_t, kOut * kIn> values{};
  std::array<uint8_t, kOut> exponents{};
  int type = 0;
};

struct Txn {
  std::string profile;
  int64_t profileVersion = 0, planVersion = 0;
  std::vector<cim22_group> groupsRaw;
  std::vector<std::vector<cim22_work>> works; // per group
  std::vector<Weight> weights;
  std::vector<cim22_frame_packet> packets;
  std::vector<cim22_input_binding> inputs;
  std::vector<cim22_readback_binding> readbacks;
};

Txn copyTransaction(const cim22_transaction &t) {
  Txn out;
  out.profile = t.target_profile ? t.target_profile : "";
  out.profileVersion = t.target_profile_version;
  out.planVersion = t.execution_plan_version;
  for (int64_t g = 0; g < t.num_groups; ++g) {
    out.groupsRaw.push_back(t.groups[g]);
    out.works.emplace_back(t.groups[g].works,
                           t.groups[g].works + t.groups[g].num_works);
  }
  for (int64_t i = 0; i < t.num_weights; ++i) {
    const cim22_static_weight &s = t.weights[i];
    Weight w;
    w.group = s.group_id;
    w.work = s.work_id;
    w.core = s.core_slot;
    w.macro = s.macro_slot;
    std::copy_n(s.route, 6, w.route.begin());
    if (s.words && s.num_words > 0)
      w.words.assign(s.words, s.words + s.num_words);
    std::copy_n(s.values, kOut * kIn, w.values.begin());
    std::copy_n(s.exponents, kOut, w.exponents.begin());
    w.type = s.data_type;
    out.weights.push_back(std::move(w));
  }
  out.packets.assign(t.packets, t.packets + t.num_packets);
  out.inputs.assign(t.inputs, t.inputs + t.num_inputs);
  out.readbacks.assign(t.readbacks, t.readbacks + t.num_readbacks);
  return out;
}

bool sameRoute(const int32_t *a, const int32_t *b, int n) {
  return std::equal(a, a + n, b);
}

// CIMSoftwareRunner.cpp:39-129 binding lookups (first match wins).
const cim22_work *findWork(const Txn &t, int64_t group, int64_t work) {
  for (size_t g = 0; g < t.groupsRaw.size(); ++g) {
    if (t.groupsRaw[g].group_id != group)
      continue;
    for (const cim22_work &w : t.works[g])
      if (w.work_id == work)
        return &w;
  }
  return nullptr;
}
int findWeight(const Txn &t, int64_t group, int64_t work) {
  for (size_t i = 0; i < t.weights.size(); ++i)
    if (t.weights[i].group == group && t.weights[i].work == work)
      return static_cast<int>(i);
  return -1;
}
int findInput(const Txn &t, int64_t group, int64_t work) {
  for (size_t i = 0; i < t.inputs.size(); ++i)
    if (t.inputs[i].group_id == group && t.inputs[i].work_id == work)
      return static_cast<int>(i);
  return -1;
}
int findReadback(const Txn &t, int64_t group, int64_t work, int64_t macro) {
  for (size_t i = 0; i < t.readbacks.size(); ++i)
    if (t.readbacks[i].group_id == group && t.readbacks[i].work_id == work &&
        t.readbacks[i].macro_slot == macro)
      return static_cast<int>(i);
  return -1;
}
bool readbackSequence(const Txn &t, const cim22_readback_binding &b,
                      size_t &index) {
  const auto &p = t.packets;
  for (size_t i = 0; i + 2 < p.size(); ++i) {
    const auto &route = p[i], &control = p[i + 1], &read = p[i + 2];
    if (route.kind != CIM22_PACKET_RETURN_ROUTE ||
        control.kind != CIM22_PACKET_CONTROL ||
        read.kind != CIM22_PACKET_OUTPUT_CACHE_READ)
      continue;
    if (route.group_id != b.group_id || route.work_id != b.work_id ||
        route.macro_slot != b.macro_slot || !sameRoute(route.route, b.route, 6) ||
        !sameRoute(route.test_core, b.test_core, 3) ||
        route.data_type != b.data_type || control.group_id != b.group_id ||
        control.work_id != b.work_id || control.macro_slot != b.macro_slot ||
        !sameRoute(control.route, b.route, 6) ||
        control.data_type != b.data_type || read.group_id != b.group_id ||
        read.work_id != b.work_id || read.macro_slot != b.macro_slot ||
        !sameRoute(read.route, b.route, 6) || read.data_type != b.data_type ||
        read.cache_address != b.output_cache_address)
      continue;
    index = i;
    return true;
  }
  return false;
}
bool hasInputPacket(const Txn &t, const cim22_input_binding &b) {
  for (const auto &p : t.packets)
    if (p.kind == CIM22_PACKET_INPUT_CACHE_WRITE && p.group_id == b.group_id &&
        p.work_id == b.work_id && p.macro_slot == b.macro_slot &&
        p.data_type == b.data_type)
      return true;
  return false;
}
bool hasWeightPacket(const Txn &t, const Weight &w, int kind) {
  for (const auto &p : t.packets)
    if (p.kind == kind && p.group_id == w.group && p.work_id == w.work &&
        p.macro_slot == w.macro && p.data_type == w.type)
      return true;
  return false;
}

// :131-155
const char *validateWork(const Txn &t, const cim22_work &work, int input,
                         int weight, int readback) {
  if (input < 0 || weight < 0)
    return "CIM work has incomplete input or weight binding";
  const auto &in = t.inputs[input];
  const auto &w = t.weights[weight];
  if (work.core_slot < 0 || work.core_slot >= kCores || work.macro_slot < 0 ||
      work.macro_slot >= kMacros || in.macro_slot != work.macro_slot ||
      w.core != work.core_slot || w.macro != work.macro_slot)
    return "CIM work has inconsistent Core or Macro placement";
  if (!hasInputPacket(t, in))
    return "CIM input binding has no input Cache packet";
  if (!hasWeightPacket(t, w, CIM22_PACKET_WEIGHT))
    return "CIM weight section has no weight packet";
  if (w.type == CIM22_DATA_BF16 &&
      !hasWeightPacket(t, w, CIM22_PACKET_WEIGHT_EXPONENT))
    return "CIM BF16 weight section has no Weight_EXP packet";
  if (readback < 0)
    return "CIM work has no readback binding";
  if (in.data_type != w.type || t.readbacks[readback].data_type != in.data_type)
    return "CIM work has inconsistent data mode";
  return nullptr;
}

bool readbackPlacement(const cim22_readback_binding &b, const cim22_work *w) {
  return w && w->core_slot >= 0 && w->core_slot < kCores &&
         w->macro_slot == b.macro_slot;
}

struct Plan {
  struct PWork {
    const cim22_work *work;
    int input, weight, readback;
    const char *error;
  };
  struct PGroup {
    size_t index; // into Txn::groupsRaw
    std::vector<PWork> works;
  };
  struct PReadback {
    size_t binding;
    const cim22_work *work;
    std::optional<size_t> packet;
  };
  struct Wave {
    size_t groupEnd;
    std::vector<PReadback> readbacks;
  };
  std::vector<PGroup> groups;
  std::vector<Wave> waves;
};

// :211-287
Plan makePlan(const Txn &t, bool batch) {
  Plan plan;
  for (size_t g = 0; g < t.groupsRaw.size(); ++g)
    plan.groups.push_back({g, {}});
  std::stable_sort(plan.groups.begin(), plan.groups.end(),
                   [&](const Plan::PGroup &a, const Plan::PGroup &b) {
                     return t.groupsRaw[a.index].group_id <
                            t.groupsRaw[b.index].group_id;
                   });
  uint32_t waveCores = 0;
  bool waveBatchable = false;
  auto finishWave = [&] {
    if (!waveBatchable)
      return;
    auto &rb = plan.waves.back().readbacks;
    std::stable_partition(rb.begin(), rb.end(), [&](const Plan::PReadback &r) {
      return t.readbacks[r.binding].macro_slot == 0;
    });
  };
  for (size_t gi = 0; gi < plan.groups.size(); ++gi) {
    auto &entry = plan.groups[gi];
    const int64_t gid = t.groupsRaw[entry.index].group_id;
    uint32_t groupCores = 0;
    bool groupBatchable = true;
    for (const cim22_work &work : t.works[entry.index]) {
      int in = findInput(t, gid, work.work_id);
      int w = findWeight(t, gid, work.work_id);
      int rb = findReadback(t, gid, work.work_id, work.macro_slot);
      const char *err = validateWork(t, work, in, w, rb);
      entry.works.push_back({&work, in, w, rb, err});
      if (err)
        groupBatchable = false;
      else
        groupCores |= uint32_t{1} << work.core_slot;
    }
    std::vector<Plan::PReadback> groupReadbacks;
    for (size_t i = 0; i < t.readbacks.size(); ++i) {
      const auto &b = t.readbacks[i];
      if (b.group_id != gid)
        continue;
      size_t index = 0;
      const bool found = readbackSequence(t, b, index);
      const cim22_work *work = findWork(t, b.group_id, b.work_id);
      groupReadbacks.push_back(
          {i, work, found ? std::optional<size_t>(index) : std::nullopt});
      if (!found || !readbackPlacement(b, work))
        groupBatchable = false;
      else
        groupCores |= uint32_t{1} << work->core_slot;
    }
    if (plan.waves.empty() || !waveBatchable || !groupBatchable ||
        (waveCores & groupCores) != 0) {
      finishWave();
      plan.waves.push_back({gi + 1, {}});
      waveCores = 0;
      waveBatchable = batch && groupBatchable;
    }
    auto &wave = plan.waves.back();
    wave.groupEnd = gi + 1;
    wave.readbacks.insert(wave.readbacks.end(), groupReadbacks.begin(),
                          groupReadbacks.end());
    waveCores |= groupCores;
  }
  finishWave();
  return plan;
}

// WeightResidency.h:28-92
struct Image {
  std::vector<int32_t> words;
  std::array<int8_t, kOut * kIn> values;
  std::array<uint8_t, kOut> exponents;
  std::array<int32_t, 6> route;
  int type;
};

struct State {
  std::vector<Image> catalog;
  struct Slot {
    int image = -1;
    int mode = kNone;
  };
  std::array<Slot, kCores * kMacros> slots{};
  uint64_t writes = 0, hits = 0;

  int intern(const Weight &w) {
    for (size_t i = 0; i < catalog.size(); ++i) {
      const Image &im = catalog[i];
      if (im.words == w.words && im.values == w.values &&
          im.exponents == w.exponents && im.route == w.route &&
          im.type == w.type)
        return static_cast<int>(i);
    }
    catalog.push_back({w.words, w.values, w.exponents, w.route, w.type});
    return static_cast<int>(catalog.size() - 1);
  }
  void clear() { slots.fill({}); }
};

struct Trace {
  cim22_trace_callback cb = nullptr;
  void *ctx = nullptr;
  uint64_t sequence = 0;
  void emit(int kind, int64_t g = -1, int64_t w = -1, int64_t m = -1,
            int64_t p = -1, int64_t c = -1) {
    if (!cb)
      return;
    cim22_trace_event e{sequence++, kind, g, w, m, p, c};
    cb(ctx, &e);
  }
};

// :172-208
bool validateBindings(const Txn &t, const void *const *inputs, int64_t ni,
                      void *const *outputs, int64_t no, std::string &error) {
  if (t.profile != "cim22-4x5-v1" || t.profileVersion != 1 ||
      t.planVersion != 1) {
    error = "unsupported CIM executable profile or version";
    return false;
  }
  if (static_cast<size_t>(ni) != t.inputs.size()) {
    error = "CIM input count does not match executable bindings";
    return false;
  }
  if (static_cast<size_t>(no) != t.readbacks.size()) {
    error = "CIM output count does not match executable bindings";
    return false;
  }
  for (int64_t i = 0; i < ni; ++i)
    if (!inputs[i]) {
      error = t.inputs[i].data_type == CIM22_DATA_INT8
                  ? "CIM input view must contain exactly 64 INT8 values"
                  : "CIM input view must contain exactly 64 BF16 values";
      return false;
    }
  for (int64_t i = 0; i < no; ++i)
    if (!outputs[i]) {
      error = t.readbacks[i].data_type == CIM22_DATA_INT8
                  ? "CIM output view must contain exactly 16 INT32 values"
                  : "CIM output view must contain exactly 16 BF16 values";
      return false;
    }
  for (const auto &b : t.readbacks)
    if (b.macro_slot < 0 || b.macro_slot >= kMacros ||
        b.output_cache_address < 0 || b.output_cache_address >= kCacheRows) {
      error = "CIM readback binding is outside the target profile";
      return false;
    }
  return true;
}

struct MacroState {
  std::array<int8_t, kIn> input{};
  Prepared bf16;
  std::array<std::array<int32_t, kOut>, kCacheRows> cache{};
};

// :315-482 (with the residency overload :302-313).
bool run(State &state, const Txn &t, const Plan &plan, int mode,
         const void *const *inputs, int64_t ni, void *const *outputs,
         int64_t no, bool residency, Trace &trace, std::string &error) {
  auto fail = [&](const std::string &message) {
    trace.emit(CIM22_TRACE_ERROR);
    error = message;
    return false;
  };
  if (!validateBindings(t, inputs, ni, outputs, no, error)) {
    trace.emit(CIM22_TRACE_ERROR);
    return false;
  }
  std::vector<int> identities;
  if (residency)
    for (const Weight &w : t.weights)
      identities.push_back(state.intern(w));

  std::array<int, kCores * kMacros> macroIndex;
  macroIndex.fill(-1);
  std::vector<MacroState> macros;
  trace.emit(CIM22_TRACE_BEGIN_RUN);

  auto executeGroup = [&](const Plan::PGroup &entry) -> bool {
    const int64_t gid = t.groupsRaw[entry.index].group_id;
    for (const Plan::PWork &pw : entry.works) {
      if (pw.error)
        return fail(pw.error);
      const cim22_work &work = *pw.work;
      const auto &in = t.inputs[pw.input];
      const Weight &weight = t.weights[pw.weight];
      const size_t slot = work.core_slot * kMacros + work.macro_slot;
      int &index = macroIndex[slot];
      if (index < 0) {
        index = static_cast<int>(macros.size());
        macros.emplace_back();
      }
      MacroState &macro = macros[index];
      if (in.data_type == CIM22_DATA_BF16) {
        Prepared prepared;
        std::string message;
        if (!prepareInput(static_cast<const uint16_t *>(inputs[pw.input]),
                          mode, prepared, message))
          return fail(message);
        if (!validateGroup(weight.values.data(), weight.exponents.data(),
                           prepared, mode, message))
          return fail(message);
        macro.bf16 = prepared;
        macro.input = prepared.aligned.mantissas;
      } else {
        std::memcpy(macro.input.data(), inputs[pw.input], kIn);
      }
      const Image *resident = nullptr;
      bool wrote = true;
      if (residency) {
        const int identity = identities[pw.weight];
        auto &s = state.slots[slot];
        if (s.image == identity && s.mode == mode) {
          resident = &state.catalog[identity];
          wrote = false;
          ++state.hits;
        } else {
          s = {identity, mode};
          resident = &state.catalog[identity];
          ++state.writes;
        }
      }
      const int8_t *values =
          residency ? resident->values.data() : weight.values.data();
      const uint8_t *exps =
          residency ? resident->exponents.data() : weight.exponents.data();
      trace.emit(CIM22_TRACE_CONFIGURE_INPUT, gid, work.work_id,
                 work.macro_slot);
      if (wrote)
        trace.emit(CIM22_TRACE_CONFIGURE_WEIGHT, gid, work.work_id,
                   work.macro_slot);
      trace.emit(CIM22_TRACE_SELECT_MACRO, gid, work.work_id, work.macro_slot);
      trace.emit(CIM22_TRACE_START_WORK, gid, work.work_id, work.macro_slot);
      std::array<int32_t, kOut> result{};
      for (int row = 0; row < kOut; ++row) {
        const int8_t *lane = values + row * kIn;
        const bool support = in.data_type != CIM22_DATA_BF16 ||
                             mode != kSignSplit ||
                             hasSupport(lane, macro.bf16.support);
        if (!support)
          continue;
        int32_t sum = 0;
        for (int k = 0; k < kIn; ++k)
          sum += static_cast<int32_t>(lane[k]) *
                 static_cast<int32_t>(macro.input[k]);
        if (sum < kI21Min || sum >= kI21MaxExclusive)
          return fail("CIM software result exceeds signed i21 range");
        if (in.data_type == CIM22_DATA_BF16) {
          const uint8_t chipExponent = mode == kNone ? exps[row] : 0;
          const uint16_t chip =
              int21ToBF16(sum, chipExponent, macro.bf16.aligned.exponent);
          uint16_t restored = 0;
          std::string message;
          if (!restoreOutput(chip, exps[row], support, macro.bf16, mode,
                             restored, message))
            return fail(message);
          result[row] = restored;
        } else {
          result[row] = sum;
        }
      }
      macro.cache[t.readbacks[pw.readback].output_cache_address] = result;
    }
    return true;
  };

  size_t gi = 0;
  for (const Plan::Wave &wave : plan.waves) {
    for (; gi < wave.groupEnd; ++gi)
      if (!executeGroup(plan.groups[gi]))
        return false;
    for (const Plan::PReadback &r : wave.readbacks) {
      const auto &b = t.readbacks[r.binding];
      if (!r.packet)
        return fail("CIM readback is missing 1010/control/0101 sequence");
      if (!readbackPlacement(b, r.work))
        return fail("CIM readback references unknown placement");
      const int index =
          macroIndex[r.work->core_slot * kMacros + r.work->macro_slot];
      if (index < 0)
        return fail("CIM readback references an unconfigured Macro");
      const MacroState &macro = macros[index];
      trace.emit(CIM22_TRACE_CONFIGURE_RETURN_ROUTE, b.group_id, b.work_id,
                 b.macro_slot, static_cast<int64_t>(*r.packet));
      trace.emit(CIM22_TRACE_READ_OUTPUT, b.group_id, b.work_id, b.macro_slot,
                 static_cast<int64_t>(*r.packet + 2), b.output_cache_address);
      const auto &row = macro.cache[b.output_cache_address];
      if (b.data_type == CIM22_DATA_BF16) {
        uint16_t *out = static_cast<uint16_t *>(outputs[r.binding]);
        for (int i = 0; i < kOut; ++i)
          out[i] = static_cast<uint16_t>(row[i]);
      } else {
        std::memcpy(outputs[r.binding], row.data(), sizeof(int32_t) * kOut);
      }
    }
  }
  trace.emit(CIM22_TRACE_COMPLETE);
  return true;
}

void copyError(const std::string &message, char *buffer, size_t capacity) {
  if (buffer && capacity) {
    const size_t n = std::min(capacity - 1, message.size());
    std::memcpy(buffer, message.data(), n);
    buffer[n] = '\0';
  }
}

// ---------------------------------------------------------------------------
// Host code the compiler emits around the tiles.

// Passes.cpp:2304-2420: activation split. xp = (x < 0 ? 0 : x), then
// (x == 0 ? +0 : xp); xn = (x < 0 ? -x : 0). With a nonnegativity proof only
// the (x == 0 ? +0 : x) select remains. Both then truncf to BF16 (:2449-2451).
void splitActivation(float x, bool nonnegative, uint16_t &xp, uint16_t &xn) {
  const float zero = 0.0f;
  float p = x;
  float n = zero;
  if (!nonnegative) {
    const bool negative = x < zero;
    p = negative ? zero : x;
    n = negative ? -x : zero;
  }
  p = (x == zero) ? zero : p;
  xp = floatToBF16(p);
  xn = floatToBF16(n);
}

// Weight split (Passes.cpp:2360-2373) followed by RNE to BF16 (:2440-2447).
void splitWeight(float w, uint16_t &wp, uint16_t &wn) {
  const bool negative = std::signbit(w);
  const bool zero = w == 0.0f;
  wp = (negative || zero) ? 0 : floatToBF16(w);
  wn = (!negative || zero) ? 0 : floatToBF16(-w);
}

struct TileWeights {
  // [branch][ntile][ktile] -> 16x64 prealigned mantissas and 16 exponents.
  int64_t nTiles = 0, kTiles = 0;
  std::vector<int8_t> values;
  std::vector<uint8_t> exponents;
  const int8_t *tile(int branch, int64_t j, int64_t t) const {
    return values.data() + ((branch * nTiles + j) * kTiles + t) * kOut * kIn;
  }
  const uint8_t *exps(int branch, int64_t j, int64_t t) const {
    return exponents.data() + ((branch * nTiles + j) * kTiles + t) * kOut;
  }
};

bool prepareWeights(const float *w, int64_t n, int64_t k, TileWeights &out,
                    std::string &error) {
  for (int64_t i = 0; i < n * k; ++i)
    if (!std::isfinite(w[i])) {
      error = "BF16 correction requires finite fixed weights";
      return false;
    }
  out.nTiles = (n + kOut - 1) / kOut;
  out.kTiles = (k + kIn - 1) / kIn;
  out.values.assign(2 * out.nTiles * out.kTiles * kOut * kIn, 0);
  out.exponents.assign(2 * out.nTiles * out.kTiles * kOut, 0);
  std::vector<uint16_t> bits(kOut * kIn);
  for (int branch = 0; branch < 2; ++branch)
    for (int64_t j = 0; j < out.nTiles; ++j)
      for (int64_t t = 0; t < out.kTiles; ++t) {
        std::fill(bits.begin(), bits.end(), 0);
        for (int lane = 0; lane < kOut; ++lane)
          for (int i = 0; i < kIn; ++i) {
            const int64_t row = j * kOut + lane, col = t * kIn + i;
            if (row >= n || col >= k)
              continue;
            uint16_t wp, wn;
            splitWeight(w[row * k + col], wp, wn);
            bits[lane * kIn + i] = branch == 0 ? wp : wn;
          }
        prealignTile(bits.data(),
                     const_cast<int8_t *>(out.tile(branch, j, t)),
                     const_cast<uint8_t *>(out.exps(branch, j, t)));
      }
  return true;
}

// One SignSplit Work: the arithmetic of runImpl for a BF16 input row and a
// prepared weight tile (CIMSoftwareRunner.cpp:357-365,406-430).
bool signSplitWork(const uint16_t *row, const int8_t *values,
                   const uint8_t *exps, uint16_t *out, std::string &error) {
  Prepared p;
  if (!prepareInput(row, kSignSplit, p, error))
    return false;
  if (!validateGroup(values, exps, p, kSignSplit, error))
    return false;
  for (int lane = 0; lane < kOut; ++lane) {
    const int8_t *lw = values + lane * kIn;
    out[lane] = 0;
    if (!hasSupport(lw, p.support))
      continue;
    int32_t sum = 0;
    for (int k = 0; k < kIn; ++k)
      sum += static_cast<int32_t>(lw[k]) * p.aligned.mantissas[k];
    if (sum < kI21Min || sum >= kI21MaxExclusive) {
      error = "CIM software result exceeds signed i21 range";
      return false;
    }
    const uint16_t chip = int21ToBF16(sum, 0, p.aligned.exponent);
    if (!restoreOutput(chip, exps[lane], true, p, kSignSplit, out[lane], error))
      return false;
  }
  return true;
}

// Cross-K f32 accumulation of one branch for one column and N tile
// (Passes.cpp:828-857): sum in tile order, truncf to BF16 when T > 1, extf.
void accumulate(const std::vector<std::array<uint16_t, kOut>> &tiles,
                float *out) {
  const size_t T = tiles.size();
  for (int lane = 0; lane < kOut; ++lane) {
    if (T == 1) {
      out[lane] = bf16ToFloat(tiles[0][lane]);
      continue;
    }
    float acc = bf16ToFloat(tiles[0][lane]);
    for (size_t t = 1; t < T; ++t)
      acc = acc + bf16ToFloat(tiles[t][lane]);
    out[lane] = bf16ToFloat(floatToBF16(acc));
  }
}

} // namespace oracle

using namespace oracle;

// ---------------------------------------------------------------------------
// C API for the tests (ctypes).

extern "C" {

uint16_t oracle_int21_to_bf16(int32_t value, uint8_t we, uint8_t ie) {
  return int21ToBF16(value, we, ie);
}

void oracle_prealign(const uint16_t *values, uint8_t *exponent,
                     int8_t *mantissas) {
  std::array<uint16_t, kIn> row;
  std::copy_n(values, kIn, row.begin());
  Prealigned p = prealign(row);
  *exponent = p.exponent;
  std::copy(p.mantissas.begin(), p.mantissas.end(), mantissas);
}

void oracle_prealign_tile(const uint16_t *bits, int8_t *values,
                          uint8_t *exponents) {
  prealignTile(bits, values, exponents);
}

uint16_t oracle_scale_bf16(uint16_t bits, int exponent) {
  return scaleBF16(bits, exponent);
}

uint16_t oracle_float_to_bf16(float value) { return floatToBF16(value); }

// Prepare one 64-element BF16 row; returns 0 and fills the outputs, or 1 with
// the error message.
int oracle_prepare_input(const uint16_t *input, int mode, int8_t *mantissas,
                         uint8_t *exponent, int32_t *effective,
                         int32_t *scale_delta, uint64_t *support, char *error,
                         size_t capacity) {
  Prepared p;
  std::string message;
  if (!prepareInput(input, mode, p, message)) {
    copyError(message, error, capacity);
    return 1;
  }
  std::copy(p.aligned.mantissas.begin(), p.aligned.mantissas.end(), mantissas);
  *exponent = p.aligned.exponent;
  *effective = p.effective;
  *scale_delta = p.scaleDelta;
  *support = p.support;
  return 0;
}

// Restore one chip output (BF16Compensation.cpp:149-164).
int oracle_restore(uint16_t bits, uint8_t we, int support, int32_t effective,
                   int32_t scale_delta, int mode, uint16_t *out, char *error,
                   size_t capacity) {
  Prepared p;
  p.effective = effective;
  p.scaleDelta = scale_delta;
  std::string message;
  if (!restoreOutput(bits, we, support != 0, p, mode, *out, message)) {
    copyError(message, error, capacity);
    return 1;
  }
  return 0;
}

struct OracleRunner {
  State state;
};

void *oracle_runner_create() { return new OracleRunner(); }
void oracle_runner_destroy(void *r) { delete static_cast<OracleRunner *>(r); }
void oracle_runner_stats(void *r, uint64_t *writes, uint64_t *hits) {
  auto *o = static_cast<OracleRunner *>(r);
  *writes = o->state.writes;
  *hits = o->state.hits;
}
void oracle_runner_clear(void *r) {
  static_cast<OracleRunner *>(r)->state.clear();
}

// CIMSoftwareRunner::run with a freshly built Plan. With use_residency the
// runner's catalog and slots are used and cleared on failure.
int oracle_runner_run(void *r, const cim22_transaction *transaction,
                      int batch_readbacks, int mode, const void *const *inputs,
                      int64_t num_inputs, void *const *outputs,
                      int64_t num_outputs, int use_residency,
                      cim22_trace_callback trace, void *trace_context,
                      char *error, size_t capacity) {
  auto *o = static_cast<OracleRunner *>(r);
  Txn t = copyTransaction(*transaction);
  Plan plan = makePlan(t, batch_readbacks != 0);
  Trace tr{trace, trace_context, 0};
  std::string message;
  if (!run(o->state, t, plan, mode, inputs, num_inputs, outputs, num_outputs,
           use_residency != 0, tr, message)) {
    if (use_residency)
      o->state.clear();
    copyError(message, error, capacity);
    return 1;
  }
  return 0;
}

// INT8 range proof of a [n, k] int8 weight matrix over every int8 input
// (Passes.cpp:592-627). Returns 1 when every (lane, K tile) partial fits i21.
int oracle_int8_range_safe(const int8_t *w, int64_t n, int64_t k) {
  for (int64_t o = 0; o < n; ++o)
    for (int64_t r = 0; r < k; r += kIn) {
      int64_t lower = 0, upper = 0;
      const int64_t size = std::min<int64_t>(kIn, k - r);
      for (int64_t i = 0; i < size; ++i) {
        const int64_t v = w[o * k + r + i];
        upper += v >= 0 ? 127 * v : -128 * v;
        lower += v >= 0 ? -128 * v : 127 * v;
      }
      auto fits = [](int64_t x) { return x >= -(1 << 20) && x < (1 << 20); };
      if (!fits(lower) || !fits(upper))
        return 0;
    }
  return 1;
}

// INT8 CIM layer: y[m, n] = wrapping-i32 sum over K tiles of the signed-i21
// 64x16 tile results (Passes.cpp:1054-1059, CIMSoftwareRunner.cpp:415-420).
int oracle_linear_int8(const int8_t *x, int64_t m, int64_t k, const int8_t *w,
                       int64_t n, int32_t *y, char *error, size_t capacity) {
  const int64_t T = (k + kIn - 1) / kIn;
  for (int64_t col = 0; col < m; ++col)
    for (int64_t o = 0; o < n; ++o) {
      uint32_t acc = 0;
      for (int64_t t = 0; t < T; ++t) {
        int32_t partial = 0;
        for (int64_t i = t * kIn; i < std::min(k, (t + 1) * kIn); ++i)
          partial += static_cast<int32_t>(w[o * k + i]) * x[col * k + i];
        if (partial < kI21Min || partial >= kI21MaxExclusive) {
          copyError("CIM software result exceeds signed i21 range", error,
                    capacity);
          return 1;
        }
        acc += static_cast<uint32_t>(partial);
      }
      y[col * n + o] = static_cast<int32_t>(acc);
    }
  return 0;
}

// BF16 sign-split CIM layer on columns x[m, k] with weights w[n, k]:
// y[m, n] = ((pp - pn) - np) + nn (+ bias). branches = 2 drops the xn terms,
// which the compiler does when the input is provably nonnegative. Each column
// block [c0, c1) is computed independently; threads > 1 splits the columns
// over host threads.
int oracle_linear_bf16(const float *x, int64_t m, int64_t k, const float *w,
                       int64_t n, const float *bias, int branches, float *y,
                       int threads, char *error, size_t capacity) {
  TileWeights tw;
  std::string message;
  if (!prepareWeights(w, n, k, tw, message)) {
    copyError(message, error, capacity);
    return 1;
  }
  const int64_t T = tw.kTiles, J = tw.nTiles;
  const bool nonnegative = branches == 2;
  std::atomic<int> failed{0};
  std::string firstError;
  std::mutex errorLock;
  int64_t firstColumn = INT64_MAX;
  auto work = [&](int64_t c0, int64_t c1) {
    std::vector<uint16_t> xp(T * kIn), xn(T * kIn);
    std::vector<std::array<uint16_t, kOut>> tiles(T);
    std::array<std::array<float, kOut>, 4> branch;
    for (int64_t col = c0; col < c1; ++col) {
      std::fill(xp.begin(), xp.end(), 0);
      std::fill(xn.begin(), xn.end(), 0);
      for (int64_t i = 0; i < k; ++i)
        splitActivation(x[col * k + i], nonnegative, xp[i], xn[i]);
      for (int64_t j = 0; j < J; ++j) {
        for (int b = 0; b < branches; ++b) {
          const int wb = b & 1;                     // Wp, Wn, Wp, Wn
          const std::vector<uint16_t> &xv = b < 2 ? xp : xn; // xp, xp, xn, xn
          for (int64_t t = 0; t < T; ++t) {
            std::string e;
            if (!signSplitWork(xv.data() + t * kIn, tw.tile(wb, j, t),
                               tw.exps(wb, j, t), tiles[t].data(), e)) {
              std::lock_guard<std::mutex> lock(errorLock);
              if (col < firstColumn) {
                firstColumn = col;
                firstError = e;
              }
              failed.store(1);
              return;
            }
          }
          accumulate(tiles, branch[b].data());
        }
        for (int lane = 0; lane < kOut; ++lane) {
          const int64_t o = j * kOut + lane;
          if (o >= n)
            continue;
          float r = branch[0][lane] - branch[1][lane];
          if (branches == 4) {
            r = r - branch[2][lane];
            r = r + branch[3][lane];
          }
          if (bias)
            r = r + bias[o];
          y[col * n + o] = r;
        }
      }
    }
  };
  if (threads <= 1) {
    work(0, m);
  } else {
    std::vector<std::thread> pool;
    const int64_t per = (m + threads - 1) / threads;
    for (int i = 0; i < threads; ++i) {
      const int64_t c0 = i * per, c1 = std::min(m, c0 + per);
      if (c0 < c1)
        pool.emplace_back(work, c0, c1);
    }
    for (auto &th : pool)
      th.join();
  }
  if (failed.load()) {
    copyError(firstError, error, capacity);
    return 1;
  }
  return 0;
}

// BF16 CIM layer in the Legacy or None compensation mode (mode = 1 or 0):
// no sign split (the SplitCIMBF16Signs pass returns early for these modes,
// Passes.cpp:2343-2344), so the BF16-rounded signed weights and activations
// go through one contraction. Per (column, 16-lane N tile, K tile) Work the
// runner's arithmetic applies (CIMSoftwareRunner.cpp:357-365,406-430):
// prepareBF16Input in the mode, the Legacy all -128 validation, the signed
// dot with its i21 gate, int21ToBF16 with the weight exponent only in None
// mode, and the mode's restore; then the Host f32 sum in tile order with a
// final truncf when T > 1 (Passes.cpp:828-857), then + bias.
int oracle_linear_bf16_mode(const float *x, int64_t m, int64_t k, const float *w, int64_t n,
                            const float *bias, int mode, float *y, char *error,
                            size_t capacity) {
  if (mode != kNone && mode != kLegacy) {
    copyError("oracle_linear_bf16_mode handles the legacy and none modes", error, capacity);
    return 1;
  }
  for (int64_t i = 0; i < n * k; ++i)
    if (!std::isfinite(w[i])) {
      copyError("BF16 correction requires finite fixed weights", error, capacity);
      return 1;
    }
  const int64_t T = (k + kIn - 1) / kIn, J = (n + kOut - 1) / kOut;
  std::vector<int8_t> values(J * T * kOut * kIn);
  std::vector<uint8_t> exps(J * T * kOut);
  std::vector<uint16_t> bits(kOut * kIn);
  for (int64_t j = 0; j < J; ++j)
    for (int64_t t = 0; t < T; ++t) {
      std::fill(bits.begin(), bits.end(), 0);
      for (int lane = 0; lane < kOut; ++lane)
        for (int i = 0; i < kIn; ++i) {
          const int64_t row = j * kOut + lane, col = t * kIn + i;
          if (row < n && col < k)
            bits[lane * kIn + i] = floatToBF16(w[row * k + col]);
        }
      prealignTile(bits.data(), values.data() + (j * T + t) * kOut * kIn,
                   exps.data() + (j * T + t) * kOut);
    }
  std::vector<uint16_t> row(T * kIn);
  std::vector<std::array<uint16_t, kOut>> tiles(T);
  std::array<float, kOut> sums;
  for (int64_t col = 0; col < m; ++col) {
    std::fill(row.begin(), row.end(), 0);
    for (int64_t i = 0; i < k; ++i)
      row[i] = floatToBF16(x[col * k + i]);
    for (int64_t j = 0; j < J; ++j) {
      for (int64_t t = 0; t < T; ++t) {
        Prepared p;
        std::string message;
        const int8_t *vals = values.data() + (j * T + t) * kOut * kIn;
        const uint8_t *ew = exps.data() + (j * T + t) * kOut;
        if (!prepareInput(row.data() + t * kIn, mode, p, message) ||
            !validateGroup(vals, ew, p, mode, message)) {
          copyError(message, error, capacity);
          return 1;
        }
        for (int lane = 0; lane < kOut; ++lane) {
          int32_t sum = 0;
          for (int i = 0; i < kIn; ++i)
            sum += static_cast<int32_t>(vals[lane * kIn + i]) * p.aligned.mantissas[i];
          if (sum < kI21Min || sum >= kI21MaxExclusive) {
            copyError("CIM software result exceeds signed i21 range", error, capacity);
            return 1;
          }
          const uint16_t chip =
              int21ToBF16(sum, mode == kNone ? ew[lane] : 0, p.aligned.exponent);
          if (!restoreOutput(chip, ew[lane], true, p, mode, tiles[t][lane], message)) {
            copyError(message, error, capacity);
            return 1;
          }
        }
      }
      accumulate(tiles, sums.data());
      for (int lane = 0; lane < kOut; ++lane) {
        const int64_t o = j * kOut + lane;
        if (o < n)
          y[col * n + o] = bias ? sums[lane] + bias[o] : sums[lane];
      }
    }
  }
  return 0;
}

// The same layer driven through the restated runner exactly as compiled
// models drive the software runner: per column, every (branch, N tile,
// K tile) Work is packed into transactions of at most 40 Works (20 Cores x 2
// Macros, Passes.cpp:437-438), each with a Plan built once and reused, weight
// residency on, and the Host reductions applied to the [R,16] readbacks.
// This is the CPU baseline's execution structure.
int oracle_linear_bf16_runner(const float *x, int64_t m, int64_t k,
                              const float *w, int64_t n, const float *bias,
                              int branches, float *y, int threads, char *error,
                              size_t capacity) {
  TileWeights tw;
  std::string message;
  if (!prepareWeights(w, n, k, tw, message)) {
    copyError(message, error, capacity);
    return 1;
  }
  const int64_t T = tw.kTiles, J = tw.nTiles;
  const bool nonnegative = branches == 2;
  // Work list per column: (branch, j, t).
  struct Item {
    int b;
    int64_t j, t;
  };
  std::vector<Item> items;
  for (int b = 0; b < branches; ++b)
    for (int64_t j = 0; j < J; ++j)
      for (int64_t t = 0; t < T; ++t)
        items.push_back({b, j, t});
  // Build one transaction per chunk of <= 40 Works.
  struct Chunk {
    Txn txn;
    Plan plan;
    std::vector<Item> items;
  };
  std::vector<std::unique_ptr<Chunk>> chunks;
  for (size_t s = 0; s < items.size(); s += 40) {
    auto c = std::make_unique<Chunk>();
    Txn &t = c->txn;
    t.profile = "cim22-4x5-v1";
    t.profileVersion = t.planVersion = 1;
    cim22_group g{};
    g.group_id = 0;
    t.groupsRaw.push_back(g);
    t.works.emplace_back();
    const size_t e = std::min(items.size(), s + 40);
    for (size_t i = s; i < e; ++i) {
      const Item &it = items[i];
      const int64_t slot = static_cast<int64_t>(i - s);
      const int64_t work = slot;
      cim22_work wk{};
      wk.work_id = work;
      wk.core_slot = slot / 2;
      wk.macro_slot = slot % 2;
      t.works[0].push_back(wk);
      Weight wt;
      wt.group = 0;
      wt.work = work;
      wt.core = slot / 2;
      wt.macro = slot % 2;
      wt.type = CIM22_DATA_BF16;
      const int wb = it.b & 1;
      std::copy_n(tw.tile(wb, it.j, it.t), kOut * kIn, wt.values.begin());
      std::copy_n(tw.exps(wb, it.j, it.t), kOut, wt.exponents.begin());
      t.weights.push_back(wt);
      cim22_input_binding in{0, work, slot % 2, work, CIM22_DATA_BF16, 0};
      t.inputs.push_back(in);
      cim22_readback_binding rb{};
      rb.group_id = 0;
      rb.work_id = work;
      rb.macro_slot = slot % 2;
      rb.output_cache_address = 0;
      rb.data_type = CIM22_DATA_BF16;
      t.readbacks.push_back(rb);
      auto packet = [&](int kind, int64_t address) {
        cim22_frame_packet p{};
        p.kind = kind;
        p.group_id = 0;
        p.work_id = work;
        p.macro_slot = slot % 2;
        p.cache_address = address;
        p.data_type = CIM22_DATA_BF16;
        t.packets.push_back(p);
      };
      packet(CIM22_PACKET_INPUT_CACHE_WRITE, -1);
      packet(CIM22_PACKET_WEIGHT_EXPONENT, -1);
      packet(CIM22_PACKET_WEIGHT, -1);
      packet(CIM22_PACKET_RETURN_ROUTE, -1);
      packet(CIM22_PACKET_CONTROL, -1);
      packet(CIM22_PACKET_OUTPUT_CACHE_READ, 0);
      c->items.push_back(it);
    }
    c->plan = makePlan(c->txn, true);
    chunks.push_back(std::move(c));
  }
  std::atomic<int> failed{0};
  std::string firstError;
  auto body = [&](int64_t c0, int64_t c1) {
    State state; // one session per thread
    std::vector<uint16_t> xp(T * kIn), xn(T * kIn);
    std::vector<std::array<uint16_t, kIn>> rows(40);
    std::vector<std::array<uint16_t, kOut>> outs(40);
    std::vector<const void *> inPtr(40);
    std::vector<void *> outPtr(40);
    // results[b][j][t]
    std::vector<std::array<uint16_t, kOut>> tiles(branches * J * T);
    std::vector<std::array<uint16_t, kOut>> perT(T);
    std::array<std::array<float, kOut>, 4> branch;
    for (int64_t col = c0; col < c1; ++col) {
      std::fill(xp.begin(), xp.end(), 0);
      std::fill(xn.begin(), xn.end(), 0);
      for (int64_t i = 0; i < k; ++i)
        splitActivation(x[col * k + i], nonnegative, xp[i], xn[i]);
      for (auto &c : chunks) {
        const size_t R = c->items.size();
        for (size_t r = 0; r < R; ++r) {
          const Item &it = c->items[r];
          const std::vector<uint16_t> &xv = it.b < 2 ? xp : xn;
          std::copy_n(xv.data() + it.t * kIn, kIn, rows[r].begin());
          inPtr[r] = rows[r].data();
          outs[r].fill(0); // dispatch zero-fills outputs (Runtime.cpp:154-155)
          outPtr[r] = outs[r].data();
        }
        Trace tr;
        std::string e;
        if (!run(state, c->txn, c->plan, kSignSplit, inPtr.data(),
                 static_cast<int64_t>(R), outPtr.data(),
                 static_cast<int64_t>(R), true, tr, e)) {
          if (failed.fetch_add(1) == 0)
            firstError = e;
          return;
        }
        for (size_t r = 0; r < R; ++r) {
          const Item &it = c->items[r];
          tiles[(it.b * J + it.j) * T + it.t] = outs[r];
        }
      }
      for (int64_t j = 0; j < J; ++j) {
        for (int b = 0; b < branches; ++b) {
          for (int64_t t = 0; t < T; ++t)
            perT[t] = tiles[(b * J + j) * T + t];
          accumulate(perT, branch[b].data());
        }
        for (int lane = 0; lane < kOut; ++lane) {
          const int64_t o = j * kOut + lane;
          if (o >= n)
            continue;
          float r = branch[0][lane] - branch[1][lane];
          if (branches == 4) {
            r = r - branch[2][lane];
            r = r + branch[3][lane];
          }
          if (bias)
            r = r + bias[o];
          y[col * n + o] = r;
        }
      }
    }
  };
  if (threads <= 1) {
    body(0, m);
  } else {
    std::vector<std::thread> pool;
    const int64_t per = (m + threads - 1) / threads;
    for (int i = 0; i < threads; ++i) {
      const int64_t c0 = i * per, c1 = std::min(m, c0 + per);
      if (c0 < c1)
        pool.emplace_back(body, c0, c1);
    }
    for (auto &th : pool)
      th.join();
  }
  if (failed.load()) {
    copyError(firstError, error, capacity);
    return 1;
  }
  return 0;
}

} // extern "C"
