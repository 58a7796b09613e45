// runner.cu - CUDA executor for CIM transactions, behind the reference's
// CIMRunner contract (include/CIM22/Execution/CIMRunner.h:75-154), plus the
// session and the _mlir_ciface_cim22_dispatch* tile ABI (runtime/Runtime.cpp:
// 120-247).
//
// The host resolves the plan once (bindings, waves, readback packets and the
// errors the reference raises from static data, CIMSoftwareRunner.cpp:39-287)
// and interns weight tiles into a device-resident catalog. A run copies the
// caller's rows into one device arena that preserves their relative byte
// layout (so rows that alias each other alias on the device too), executes
// every wave in order in a single CTA - all Works of a wave in parallel, one
// warp per Work, then the Macro output-Cache commit and the readback
// publication in binding order - and copies the output rows back. The first
// failing Work or readback stops the run exactly where the CPU runner stops;
// the trace and the residency counters are then replayed on the host up to
// that point.
#include "cim_internal.h"
#include "cim_numeric.cuh"

#include <algorithm>
#include <cstring>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <vector>

namespace cim {
namespace {

constexpr int kCores = 20, kMacros = 2, kCacheRows = 8;
constexpr unsigned kFull = 0xffffffffu;

// Error codes; messages follow the reference's runner verbatim.
enum Code : int32_t {
  kOk = 0,
  // Static plan errors (CIMSoftwareRunner.cpp:131-155).
  kIncompleteBinding,
  kPlacement,
  kNoInputPacket,
  kNoWeightPacket,
  kNoExpPacket,
  kNoReadback,
  kDataMode,
  // Prepare/validate stage (BF16Compensation.cpp:55-137).
  kInputNotFinite,
  kNegativeInput,
  kNormExponent,
  kNormSign,
  kLegacyScaling,
  kLegacyI21,
  kWeightExp255,
  kNegativeWeight,
  // Lane stage (CIMSoftwareRunner.cpp:419-430, BF16Compensation.cpp:33-51).
  kI21Range,
  kChipNotFinite,
  kTileExceeds,
  // Readback (CIMSoftwareRunner.cpp:446-458).
  kMissingSequence,
  kUnknownPlacement,
  kUnconfiguredMacro,
};

const char *code_message(int32_t code) {
  switch (code) {
  case kIncompleteBinding: return "CIM work has incomplete input or weight binding";
  case kPlacement: return "CIM work has inconsistent Core or Macro placement";
  case kNoInputPacket: return "CIM input binding has no input Cache packet";
  case kNoWeightPacket: return "CIM weight section has no weight packet";
  case kNoExpPacket: return "CIM BF16 weight section has no Weight_EXP packet";
  case kNoReadback: return "CIM work has no readback binding";
  case kDataMode: return "CIM work has inconsistent data mode";
  case kInputNotFinite: return "CIM BF16 input does not support NaN or infinity";
  case kNegativeInput: return "CIM nonnegative BF16 mode rejects negative inputs";
  case kNormExponent:
    return "CIM nonnegative BF16 normalization did not produce input exponent 127";
  case kNormSign: return "CIM nonnegative BF16 normalization changed sign";
  case kLegacyScaling:
    return "CIM legacy BF16 group scaling changed prealigned input mantissas";
  case kLegacyI21: return "CIM BF16 result exceeds signed i21 range";
  case kWeightExp255: return "CIM nonnegative BF16 weight exponent is not finite";
  case kNegativeWeight: return "CIM nonnegative BF16 mode rejects negative prepared weights";
  case kI21Range: return "CIM software result exceeds signed i21 range";
  case kChipNotFinite: return "CIM BF16 chip output is not finite";
  case kTileExceeds: return "CIM BF16 compensated tile exceeds BF16";
  case kMissingSequence: return "CIM readback is missing 1010/control/0101 sequence";
  case kUnknownPlacement: return "CIM readback references unknown placement";
  case kUnconfiguredMacro: return "CIM readback references an unconfigured Macro";
  default: return "CIM runner failure";
  }
}

bool lane_stage(int32_t code) { return code >= kI21Range && code <= kTileExceeds; }

// Device-resident weight image with validation flags precomputed on the host.
struct alignas(16) DevImage {
  int8_t values[16 * 64];
  uint8_t exponents[16];
  int32_t flags; // bit0 exponent 255, bit1 negative value, bits 16-31 lanes all -128
  int32_t pad[3];
};
static_assert(sizeof(DevImage) == 1056, "image layout");

struct DevWork {
  int32_t input;        // dynamic input binding index
  int32_t image;        // catalog image
  int32_t slot;         // core * 2 + macro
  int32_t cache_row;    // readback output Cache address
  int32_t static_error; // plan error or 0
  int32_t bf16;         // input data type
};

struct DevReadback {
  int32_t binding;
  int32_t slot;
  int32_t cache_row;
  int32_t bf16;
  int32_t static_error;
};

struct DevWave {
  int32_t work_begin, work_end, rb_begin, rb_end;
};

__device__ __forceinline__ uint16_t load_u16(const uint8_t *p) {
  return static_cast<uint16_t>(p[0] | (p[1] << 8));
}

// One warp executes one Work: input preparation (BF16 modes), the 16-lane x
// 64 MAC dot, the signed-i21 gate and the BF16 convert/restore, producing 16
// Cache payloads and the first error in the reference's check order.
__device__ void execute_work(const DevWork &w, const DevImage &img,
                             const uint8_t *src, int mode, int8_t *s_in,
                             int32_t *result, int32_t *code_out) {
  const int lane = threadIdx.x & 31;
  int32_t code = kOk;
  int ie = 0, effective = 0, delta = 0;
  if (!w.bf16) {
    s_in[lane] = static_cast<int8_t>(src[lane]);
    s_in[lane + 32] = static_cast<int8_t>(src[lane + 32]);
  } else {
    uint16_t v[2] = {load_u16(src + 2 * lane), load_u16(src + 2 * (lane + 32))};
    int8_t a[2] = {0, 0};
    const bool nonfinite = ((v[0] >> 7) & 0xff) == 0xff || ((v[1] >> 7) & 0xff) == 0xff;
    if (__any_sync(kFull, nonfinite)) {
      code = kInputNotFinite;
    } else if (mode == CIM22_BF16_SIGN_SPLIT) {
      const bool negative = ((v[0] & 0x8000) && (v[0] & 0x7fff)) ||
                            ((v[1] & 0x8000) && (v[1] & 0x7fff));
      if (__any_sync(kFull, negative)) {
        code = kNegativeInput;
      } else {
        v[0] &= 0x7fff;
        v[1] &= 0x7fff;
        const uint32_t mx = __reduce_max_sync(kFull, max(v[0], v[1]));
        if (mx != 0) {
          effective = effective_exponent(static_cast<uint16_t>(mx));
          const int shift = 127 - effective;
          if (shift) {
            v[0] = bf16_scalbn(v[0], shift);
            v[1] = bf16_scalbn(v[1], shift);
          }
          ie = static_cast<int>(__reduce_max_sync(
              kFull, max((v[0] >> 7) & 0xff, (v[1] >> 7) & 0xff)));
          a[0] = prealign_element(v[0], ie);
          a[1] = prealign_element(v[1], ie);
          if (ie != 127)
            code = kNormExponent;
          else if (__any_sync(kFull, a[0] < 0 || a[1] < 0))
            code = kNormSign;
        }
      }
    } else {
      ie = static_cast<int>(__reduce_max_sync(
          kFull, max((v[0] >> 7) & 0xff, (v[1] >> 7) & 0xff)));
      a[0] = prealign_element(v[0], ie);
      a[1] = prealign_element(v[1], ie);
      if (mode == CIM22_BF16_LEGACY) {
        delta = ie > 240 ? ie - 240 : 0;
        if (delta) {
          const uint16_t s0 = bf16_scalbn(v[0], -delta), s1 = bf16_scalbn(v[1], -delta);
          const int ie2 = static_cast<int>(__reduce_max_sync(
              kFull, max((s0 >> 7) & 0xff, (s1 >> 7) & 0xff)));
          const int8_t b0 = prealign_element(s0, ie2), b1 = prealign_element(s1, ie2);
          if (ie2 > 240 || __any_sync(kFull, b0 != a[0] || b1 != a[1]))
            code = kLegacyScaling;
          ie = ie2;
        }
      }
    }
    if (code == kOk) {
      // validateBF16Group (BF16Compensation.cpp:55-81).
      if (mode == CIM22_BF16_LEGACY && __all_sync(kFull, a[0] == -128 && a[1] == -128) &&
          (img.flags >> 16) != 0)
        code = kLegacyI21;
      else if (mode == CIM22_BF16_SIGN_SPLIT && (img.flags & 1))
        code = kWeightExp255;
      else if (mode == CIM22_BF16_SIGN_SPLIT && (img.flags & 2))
        code = kNegativeWeight;
    }
    s_in[lane] = a[0];
    s_in[lane + 32] = a[1];
  }
  __syncwarp();
  if (code != kOk) {
    if (lane == 0)
      *code_out = code;
    return;
  }
  // Lane l = lane & 15 sums half h = lane >> 4 of its 64 products.
  const int l = lane & 15, h = lane >> 4;
  int sum = 0;
  bool support = false;
  const int8_t *wrow = img.values + l * 64 + h * 32;
  const int8_t *arow = s_in + h * 32;
#pragma unroll 8
  for (int k = 0; k < 32; ++k) {
    const int wv = wrow[k], av = arow[k];
    sum += wv * av;
    support |= (wv != 0) && (av != 0);
  }
  sum += __shfl_down_sync(kFull, sum, 16);
  support = (__shfl_down_sync(kFull, static_cast<int>(support), 16) != 0) || support;
  int32_t lane_code = kOk;
  int32_t value = 0;
  if (lane < 16) {
    const bool has = !w.bf16 || mode != CIM22_BF16_SIGN_SPLIT || support;
    if (has) {
      if (sum < -(1 << 20) || sum >= (1 << 20)) {
        lane_code = kI21Range;
      } else if (w.bf16) {
        const int ew = img.exponents[l];
        const uint16_t chip = int21_to_bf16(sum, mode == CIM22_BF16_NONE ? ew : 0, ie);
        if (mode == CIM22_BF16_NONE) {
          value = chip;
        } else {
          const int exponent = mode == CIM22_BF16_SIGN_SPLIT ? ew + effective - 260
                                                             : ew + delta - 133;
          uint16_t restored = 0;
          int err = 0;
          if (compensate(chip, exponent, restored, err))
            value = restored;
          else
            lane_code = err == 1 ? kChipNotFinite : kTileExceeds;
        }
      } else {
        value = sum;
      }
    }
    result[l] = value;
  }
  const unsigned failing = __ballot_sync(kFull, lane_code != kOk) & 0xffffu;
  const int first = failing ? __ffs(failing) - 1 : 0;
  const int32_t first_code = __shfl_sync(kFull, lane_code, first);
  if (lane == 0)
    *code_out = failing ? first_code : kOk;
}

// outcome[0] = 0 success, 1 failing Work, 2 failing readback; [1] index;
// [2] code.
__global__ void __launch_bounds__(1024)
    runner_kernel(const DevWork *__restrict__ works,
                  const DevReadback *__restrict__ rbs,
                  const DevWave *__restrict__ waves, int num_waves,
                  const DevImage *__restrict__ images,
                  const int64_t *__restrict__ in_off,
                  const int64_t *__restrict__ out_off, uint8_t *arena, int mode,
                  int32_t *results, int32_t *codes, int32_t *outcome) {
  __shared__ int32_t cache[kCores * kMacros][kCacheRows][16];
  __shared__ int8_t s_in[32][64];
  __shared__ int s_fail;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < kCores * kMacros * kCacheRows * 16; i += blockDim.x)
    (&cache[0][0][0])[i] = 0;
  if (tid == 0) {
    s_fail = 0;
    outcome[0] = outcome[1] = outcome[2] = 0;
  }
  __syncthreads();
  const int nwarps = blockDim.x >> 5;
  for (int wv = 0; wv < num_waves; ++wv) {
    const DevWave wave = waves[wv];
    for (int i = wave.work_begin + warp; i < wave.work_end; i += nwarps) {
      const DevWork w = works[i];
      if (w.static_error) {
        if (lane == 0)
          codes[i] = kOk;
        continue;
      }
      execute_work(w, images[w.image], arena + in_off[w.input], mode, s_in[warp],
                   results + static_cast<int64_t>(i) * 16, codes + i);
    }
    __syncthreads();
    if (tid == 0) {
      for (int i = wave.work_begin; i < wave.work_end; ++i) {
        const DevWork w = works[i];
        const int32_t code = w.static_error ? w.static_error : codes[i];
        if (code != kOk) {
          outcome[0] = 1;
          outcome[1] = i;
          outcome[2] = code;
          s_fail = 1;
          break;
        }
        for (int j = 0; j < 16; ++j)
          cache[w.slot][w.cache_row][j] = results[static_cast<int64_t>(i) * 16 + j];
      }
    }
    __syncthreads();
    if (s_fail)
      return;
    if (warp == 0) {
      for (int r = wave.rb_begin; r < wave.rb_end; ++r) {
        const DevReadback rb = rbs[r];
        if (rb.static_error) {
          if (lane == 0) {
            outcome[0] = 2;
            outcome[1] = r;
            outcome[2] = rb.static_error;
            s_fail = 1;
          }
          break;
        }
        uint8_t *dst = arena + out_off[rb.binding];
        if (lane < 16) {
          const int32_t v = cache[rb.slot][rb.cache_row][lane];
          if (rb.bf16) {
            dst[2 * lane] = static_cast<uint8_t>(v & 0xff);
            dst[2 * lane + 1] = static_cast<uint8_t>((v >> 8) & 0xff);
          } else {
            for (int b = 0; b < 4; ++b)
              dst[4 * lane + b] = static_cast<uint8_t>((static_cast<uint32_t>(v) >> (8 * b)) & 0xff);
          }
        }
        __syncwarp();
      }
    }
    __syncthreads();
    if (s_fail)
      return;
  }
}

// ---------------------------------------------------------------------------
// Host side.

struct Image {
  std::vector<int32_t> words;
  std::vector<int8_t> values;
  std::vector<uint8_t> exponents;
  std::vector<int32_t> route;
  int type;
};

bool same6(const int32_t *a, const int32_t *b, int n) { return std::equal(a, a + n, b); }

struct HostWork {
  int64_t group_id, work_id;
  int32_t macro_slot;
  int32_t slot;
  int32_t static_error;
};

struct HostReadback {
  int64_t group_id, work_id, macro_slot, address;
  int64_t packet;
  int32_t static_error;
};

struct HostWave {
  int32_t work_begin, work_end, rb_begin, rb_end;
};

} // namespace
} // namespace cim

using namespace cim;

struct cim22_cuda_runner {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::vector<Image> catalog;          // exact payloads
  DevImage *d_images = nullptr;        // device copies
  size_t image_capacity = 0;
  struct Slot {
    int image = -1;
    int mode = 0;
  };
  Slot slots[kCores * kMacros];
  uint64_t writes = 0, hits = 0;
  // Reused per-run buffers.
  uint8_t *d_arena = nullptr;
  size_t arena_capacity = 0;
  uint8_t *h_stage = nullptr;
  size_t stage_capacity = 0;
  int32_t *d_scratch = nullptr; // results + codes
  size_t scratch_capacity = 0;

  int intern(const cim22_static_weight &w) {
    for (size_t i = 0; i < catalog.size(); ++i) {
      const Image &im = catalog[i];
      if (im.type == w.data_type &&
          std::equal(im.values.begin(), im.values.end(), w.values) &&
          std::equal(im.exponents.begin(), im.exponents.end(), w.exponents) &&
          std::equal(im.route.begin(), im.route.end(), w.route) &&
          im.words.size() == static_cast<size_t>(std::max<int64_t>(0, w.num_words)) &&
          (im.words.empty() || std::equal(im.words.begin(), im.words.end(), w.words)))
        return static_cast<int>(i);
    }
    Image im;
    if (w.words && w.num_words > 0)
      im.words.assign(w.words, w.words + w.num_words);
    im.values.assign(w.values, w.values + 1024);
    im.exponents.assign(w.exponents, w.exponents + 16);
    im.route.assign(w.route, w.route + 6);
    im.type = w.data_type;
    catalog.push_back(std::move(im));
    return static_cast<int>(catalog.size() - 1);
  }

  bool sync_images() {
    if (catalog.size() > image_capacity) {
      size_t cap = std::max<size_t>(64, image_capacity * 2);
      while (cap < catalog.size())
        cap *= 2;
      DevImage *fresh = nullptr;
      if (!cuda_ok(cudaMalloc(&fresh, cap * sizeof(DevImage)), "cudaMalloc"))
        return false;
      if (d_images) {
        cudaMemcpy(fresh, d_images, image_capacity * sizeof(DevImage),
                   cudaMemcpyDeviceToDevice);
        cudaFree(d_images);
      }
      d_images = fresh;
      image_capacity = cap;
    }
    return true;
  }

  bool upload_image(int index) {
    const Image &im = catalog[index];
    DevImage d{};
    std::memcpy(d.values, im.values.data(), 1024);
    std::memcpy(d.exponents, im.exponents.data(), 16);
    int32_t flags = 0;
    for (int l = 0; l < 16; ++l)
      if (im.exponents[l] == 255)
        flags |= 1;
    for (int i = 0; i < 1024; ++i)
      if (im.values[i] < 0)
        flags |= 2;
    for (int l = 0; l < 16; ++l) {
      bool all = true;
      for (int k = 0; k < 64; ++k)
        all &= im.values[l * 64 + k] == -128;
      if (all)
        flags |= 1 << (16 + l);
    }
    d.flags = flags;
    return cuda_ok(cudaMemcpy(d_images + index, &d, sizeof d, cudaMemcpyHostToDevice),
                   "cudaMemcpy");
  }
};

struct cim22_cuda_plan {
  cim22_cuda_runner *runner = nullptr;
  std::string profile;
  int64_t profile_version = 0, plan_version = 0;
  std::vector<cim22_input_binding> inputs;
  std::vector<cim22_readback_binding> readbacks;
  std::vector<HostWork> works;       // execution order
  std::vector<int32_t> work_images;  // per work (catalog image)
  std::vector<HostReadback> rbs;     // publication order
  std::vector<int32_t> rb_binding;   // binding index per rb
  std::vector<HostWave> waves;
  DevWork *d_works = nullptr;
  DevReadback *d_rbs = nullptr;
  DevWave *d_waves = nullptr;
};

namespace cim {
namespace {

// Plan construction (CIMSoftwareRunner.cpp:39-287).
bool build_plan(cim22_cuda_plan &plan, const cim22_transaction &t, bool batch,
                std::string &error) {
  cim22_cuda_runner &runner = *plan.runner;
  plan.profile = t.target_profile ? t.target_profile : "";
  plan.profile_version = t.target_profile_version;
  plan.plan_version = t.execution_plan_version;
  plan.inputs.assign(t.inputs, t.inputs + t.num_inputs);
  plan.readbacks.assign(t.readbacks, t.readbacks + t.num_readbacks);
  const cim22_frame_packet *P = t.packets;
  const int64_t NP = t.num_packets;

  auto find_input = [&](int64_t g, int64_t w) -> int64_t {
    for (int64_t i = 0; i < t.num_inputs; ++i)
      if (t.inputs[i].group_id == g && t.inputs[i].work_id == w)
        return i;
    return -1;
  };
  auto find_weight = [&](int64_t g, int64_t w) -> int64_t {
    for (int64_t i = 0; i < t.num_weights; ++i)
      if (t.weights[i].group_id == g && t.weights[i].work_id == w)
        return i;
    return -1;
  };
  auto find_readback = [&](int64_t g, int64_t w, int64_t m) -> int64_t {
    for (int64_t i = 0; i < t.num_readbacks; ++i)
      if (t.readbacks[i].group_id == g && t.readbacks[i].work_id == w &&
          t.readbacks[i].macro_slot == m)
        return i;
    return -1;
  };
  auto find_work = [&](int64_t g, int64_t w) -> const cim22_work * {
    for (int64_t gi = 0; gi < t.num_groups; ++gi) {
      if (t.groups[gi].group_id != g)
        continue;
      for (int64_t wi = 0; wi < t.groups[gi].num_works; ++wi)
        if (t.groups[gi].works[wi].work_id == w)
          return &t.groups[gi].works[wi];
    }
    return nullptr;
  };
  auto has_packet = [&](int kind, int64_t g, int64_t w, int64_t m, int type) {
    for (int64_t i = 0; i < NP; ++i)
      if (P[i].kind == kind && P[i].group_id == g && P[i].work_id == w &&
          P[i].macro_slot == m && P[i].data_type == type)
        return true;
    return false;
  };
  auto readback_sequence = [&](const cim22_readback_binding &b) -> int64_t {
    for (int64_t i = 0; i + 2 < NP; ++i) {
      const auto &r = P[i], &c = P[i + 1], &o = P[i + 2];
      if (r.kind != CIM22_PACKET_RETURN_ROUTE || c.kind != CIM22_PACKET_CONTROL ||
          o.kind != CIM22_PACKET_OUTPUT_CACHE_READ)
        continue;
      const bool match =
          r.group_id == b.group_id && r.work_id == b.work_id &&
          r.macro_slot == b.macro_slot && same6(r.route, b.route, 6) &&
          same6(r.test_core, b.test_core, 3) && r.data_type == b.data_type &&
          c.group_id == b.group_id && c.work_id == b.work_id &&
          c.macro_slot == b.macro_slot && same6(c.route, b.route, 6) &&
          c.data_type == b.data_type && o.group_id == b.group_id &&
          o.work_id == b.work_id && o.macro_slot == b.macro_slot &&
          same6(o.route, b.route, 6) && o.data_type == b.data_type &&
          o.cache_address == b.output_cache_address;
      if (match)
        return i;
    }
    return -1;
  };
  auto placement_ok = [&](const cim22_readback_binding &b, const cim22_work *w) {
    return w && w->core_slot >= 0 && w->core_slot < kCores &&
           w->macro_slot == b.macro_slot;
  };

  // Groups in ascending id (stable for equal ids).
  std::vector<int64_t> order(t.num_groups);
  for (int64_t i = 0; i < t.num_groups; ++i)
    order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int64_t a, int64_t b) {
    return t.groups[a].group_id < t.groups[b].group_id;
  });

  struct PendingRb {
    int64_t binding;
    const cim22_work *work;
    int64_t packet;
  };
  std::vector<std::vector<PendingRb>> wave_rbs;
  std::vector<std::pair<int32_t, int32_t>> wave_works; // [begin, end)
  std::vector<bool> wave_batchable;
  uint32_t wave_cores = 0;
  bool current_batchable = false;
  auto finish_wave = [&] {
    if (wave_rbs.empty() || !current_batchable)
      return;
    auto &rb = wave_rbs.back();
    std::stable_partition(rb.begin(), rb.end(), [&](const PendingRb &r) {
      return t.readbacks[r.binding].macro_slot == 0;
    });
  };
  for (int64_t gi : order) {
    const cim22_group &group = t.groups[gi];
    uint32_t group_cores = 0;
    bool group_batchable = true;
    const int32_t begin = static_cast<int32_t>(plan.works.size());
    for (int64_t wi = 0; wi < group.num_works; ++wi) {
      const cim22_work &work = group.works[wi];
      const int64_t in = find_input(group.group_id, work.work_id);
      const int64_t wt = find_weight(group.group_id, work.work_id);
      const int64_t rb = find_readback(group.group_id, work.work_id, work.macro_slot);
      int32_t err = kOk;
      if (in < 0 || wt < 0) {
        err = kIncompleteBinding;
      } else {
        const auto &ib = t.inputs[in];
        const auto &ws = t.weights[wt];
        if (work.core_slot < 0 || work.core_slot >= kCores || work.macro_slot < 0 ||
            work.macro_slot >= kMacros || ib.macro_slot != work.macro_slot ||
            ws.core_slot != work.core_slot || ws.macro_slot != work.macro_slot)
          err = kPlacement;
        else if (!has_packet(CIM22_PACKET_INPUT_CACHE_WRITE, ib.group_id, ib.work_id,
                             ib.macro_slot, ib.data_type))
          err = kNoInputPacket;
        else if (!has_packet(CIM22_PACKET_WEIGHT, ws.group_id, ws.work_id, ws.macro_slot,
                             ws.data_type))
          err = kNoWeightPacket;
        else if (ws.data_type == CIM22_DATA_BF16 &&
                 !has_packet(CIM22_PACKET_WEIGHT_EXPONENT, ws.group_id, ws.work_id,
                             ws.macro_slot, ws.data_type))
          err = kNoExpPacket;
        else if (rb < 0)
          err = kNoReadback;
        else if (ib.data_type != ws.data_type ||
                 t.readbacks[rb].data_type != ib.data_type)
          err = kDataMode;
      }
      HostWork hw{group.group_id, work.work_id, static_cast<int32_t>(work.macro_slot),
                  err ? 0 : static_cast<int32_t>(work.core_slot * kMacros + work.macro_slot),
                  err};
      plan.works.push_back(hw);
      int32_t image = 0;
      int32_t row = 0;
      if (!err) {
        image = runner.intern(t.weights[wt]);
        row = static_cast<int32_t>(t.readbacks[rb].output_cache_address);
        if (row < 0 || row >= kCacheRows)
          row = 0; // rejected by validateBindings before any Work runs
      }
      plan.work_images.push_back(image);
      (void)row;
      if (err)
        group_batchable = false;
      else
        group_cores |= 1u << work.core_slot;
    }
    const int32_t end = static_cast<int32_t>(plan.works.size());
    std::vector<PendingRb> group_rbs;
    for (int64_t i = 0; i < t.num_readbacks; ++i) {
      const auto &b = t.readbacks[i];
      if (b.group_id != group.group_id)
        continue;
      const int64_t seq = readback_sequence(b);
      const cim22_work *w = find_work(b.group_id, b.work_id);
      group_rbs.push_back({i, w, seq});
      if (seq < 0 || !placement_ok(b, w))
        group_batchable = false;
      else
        group_cores |= 1u << w->core_slot;
    }
    if (wave_rbs.empty() || !current_batchable || !group_batchable ||
        (wave_cores & group_cores) != 0) {
      finish_wave();
      wave_rbs.emplace_back();
      wave_works.push_back({begin, begin});
      wave_cores = 0;
      current_batchable = batch && group_batchable;
    }
    wave_works.back().second = end;
    wave_rbs.back().insert(wave_rbs.back().end(), group_rbs.begin(), group_rbs.end());
    wave_cores |= group_cores;
  }
  finish_wave();

  // Flatten readbacks and resolve their static errors and slots.
  std::vector<bool> configured(kCores * kMacros, false);
  std::vector<DevWork> dworks;
  std::vector<DevReadback> drbs;
  std::vector<DevWave> dwaves;
  for (size_t wv = 0; wv < wave_rbs.size(); ++wv) {
    DevWave dw{};
    dw.work_begin = wave_works[wv].first;
    dw.work_end = wave_works[wv].second;
    for (int32_t i = dw.work_begin; i < dw.work_end; ++i)
      if (!plan.works[i].static_error)
        configured[plan.works[i].slot] = true;
    dw.rb_begin = static_cast<int32_t>(plan.rbs.size());
    for (const PendingRb &p : wave_rbs[wv]) {
      const auto &b = t.readbacks[p.binding];
      HostReadback hr{b.group_id, b.work_id, b.macro_slot, b.output_cache_address,
                      p.packet, kOk};
      int32_t slot = 0;
      if (p.packet < 0)
        hr.static_error = kMissingSequence;
      else if (!placement_ok(b, p.work))
        hr.static_error = kUnknownPlacement;
      else {
        slot = static_cast<int32_t>(p.work->core_slot * kMacros + p.work->macro_slot);
        if (!configured[slot])
          hr.static_error = kUnconfiguredMacro;
      }
      plan.rbs.push_back(hr);
      plan.rb_binding.push_back(static_cast<int32_t>(p.binding));
      DevReadback d{};
      d.binding = static_cast<int32_t>(p.binding);
      d.slot = slot;
      d.cache_row = static_cast<int32_t>(
          std::clamp<int64_t>(b.output_cache_address, 0, kCacheRows - 1));
      d.bf16 = b.data_type == CIM22_DATA_BF16;
      d.static_error = hr.static_error;
      drbs.push_back(d);
    }
    dw.rb_end = static_cast<int32_t>(plan.rbs.size());
    dwaves.push_back(dw);
    plan.waves.push_back({dw.work_begin, dw.work_end, dw.rb_begin, dw.rb_end});
  }
  for (size_t i = 0; i < plan.works.size(); ++i) {
    const HostWork &hw = plan.works[i];
    DevWork d{};
    d.static_error = hw.static_error;
    if (!hw.static_error) {
      const int64_t in = find_input(hw.group_id, hw.work_id);
      const int64_t rb = find_readback(hw.group_id, hw.work_id, hw.macro_slot);
      d.input = static_cast<int32_t>(in);
      d.image = plan.work_images[i];
      d.slot = hw.slot;
      d.cache_row = static_cast<int32_t>(
          std::clamp<int64_t>(t.readbacks[rb].output_cache_address, 0, kCacheRows - 1));
      d.bf16 = t.inputs[in].data_type == CIM22_DATA_BF16;
    }
    dworks.push_back(d);
  }
  if (!runner.sync_images()) {
    error = last_error();
    return false;
  }
  for (size_t i = 0; i < runner.catalog.size(); ++i)
    if (!runner.upload_image(static_cast<int>(i))) {
      error = last_error();
      return false;
    }
  auto upload = [&](auto &dst, const auto &src) {
    using T = typename std::decay_t<decltype(src)>::value_type;
    const size_t bytes = std::max<size_t>(1, src.size()) * sizeof(T);
    if (!cuda_ok(cudaMalloc(&dst, bytes), "cudaMalloc"))
      return false;
    return src.empty() || cuda_ok(cudaMemcpy(dst, src.data(), src.size() * sizeof(T),
                                             cudaMemcpyHostToDevice),
                                  "cudaMemcpy");
  };
  if (!upload(plan.d_works, dworks) || !upload(plan.d_rbs, drbs) ||
      !upload(plan.d_waves, dwaves)) {
    error = last_error();
    return false;
  }
  return true;
}

struct Trace {
  cim22_trace_callback cb;
  void *ctx;
  uint64_t seq = 0;
  void emit(int kind, int64_t g = -1, int64_t w = -1, int64_t m = -1, int64_t p = -1,
            int64_t c = -1) {
    if (!cb)
      return;
    cim22_trace_event e{seq++, kind, g, w, m, p, c};
    cb(ctx, &e);
  }
};

} // namespace
} // namespace cim

extern "C" {

cim22_cuda_runner *cim22_cuda_runner_create(int device, char *error,
                                            size_t error_capacity) {
  auto runner = std::make_unique<cim22_cuda_runner>();
  runner->device = device;
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice") ||
      !cuda_ok(cudaStreamCreateWithFlags(&runner->stream, cudaStreamNonBlocking),
               "cudaStreamCreate")) {
    copy_error(last_error(), error, error_capacity);
    return nullptr;
  }
  return runner.release();
}

void cim22_cuda_runner_destroy(cim22_cuda_runner *runner) {
  if (!runner)
    return;
  cudaSetDevice(runner->device);
  if (runner->stream)
    cudaStreamDestroy(runner->stream);
  cudaFree(runner->d_images);
  cudaFree(runner->d_arena);
  cudaFree(runner->d_scratch);
  cudaFreeHost(runner->h_stage);
  delete runner;
}

cim22_cuda_plan *cim22_cuda_plan_create(cim22_cuda_runner *runner,
                                        const cim22_transaction *transaction,
                                        int batch_readbacks, char *error,
                                        size_t error_capacity) {
  if (!runner || !transaction) {
    copy_error("invalid CIM plan arguments", error, error_capacity);
    return nullptr;
  }
  cudaSetDevice(runner->device);
  auto plan = std::make_unique<cim22_cuda_plan>();
  plan->runner = runner;
  std::string message;
  if (!build_plan(*plan, *transaction, batch_readbacks != 0, message)) {
    copy_error(message, error, error_capacity);
    cim22_cuda_plan_destroy(plan.release());
    return nullptr;
  }
  return plan.release();
}

void cim22_cuda_plan_destroy(cim22_cuda_plan *plan) {
  if (!plan)
    return;
  cudaSetDevice(plan->runner->device);
  cudaFree(plan->d_works);
  cudaFree(plan->d_rbs);
  cudaFree(plan->d_waves);
  delete plan;
}

void cim22_cuda_runner_weight_stats(const cim22_cuda_runner *runner,
                                    uint64_t *writes, uint64_t *hits) {
  if (writes)
    *writes = runner ? runner->writes : 0;
  if (hits)
    *hits = runner ? runner->hits : 0;
}

void cim22_cuda_runner_clear_residency(cim22_cuda_runner *runner) {
  if (runner)
    for (auto &s : runner->slots)
      s = {};
}

int cim22_cuda_runner_run(cim22_cuda_runner *runner,
                          const cim22_cuda_plan *plan,
                          int32_t bf16_compensation, const void *const *inputs,
                          int64_t num_inputs, void *const *outputs,
                          int64_t num_outputs, int use_residency,
                          cim22_trace_callback trace_cb, void *trace_context,
                          char *error, size_t error_capacity) {
  Trace trace{trace_cb, trace_context};
  auto fail = [&](const std::string &message) {
    trace.emit(CIM22_TRACE_ERROR);
    if (use_residency && runner)
      cim22_cuda_runner_clear_residency(runner);
    copy_error(message, error, error_capacity);
    return 1;
  };
  if (!runner || !plan || plan->runner != runner || bf16_compensation < 0 ||
      bf16_compensation > 2)
    return fail("invalid CIM runner arguments");
  // validateBindings (CIMSoftwareRunner.cpp:172-208).
  if (plan->profile != "cim22-4x5-v1" || plan->profile_version != 1 ||
      plan->plan_version != 1)
    return fail("unsupported CIM executable profile or version");
  if (static_cast<size_t>(num_inputs) != plan->inputs.size())
    return fail("CIM input count does not match executable bindings");
  if (static_cast<size_t>(num_outputs) != plan->readbacks.size())
    return fail("CIM output count does not match executable bindings");
  for (int64_t i = 0; i < num_inputs; ++i)
    if (!inputs[i])
      return fail(plan->inputs[i].data_type == CIM22_DATA_INT8
                      ? "CIM input view must contain exactly 64 INT8 values"
                      : "CIM input view must contain exactly 64 BF16 values");
  for (int64_t i = 0; i < num_outputs; ++i)
    if (!outputs[i])
      return fail(plan->readbacks[i].data_type == CIM22_DATA_INT8
                      ? "CIM output view must contain exactly 16 INT32 values"
                      : "CIM output view must contain exactly 16 BF16 values");
  for (const auto &b : plan->readbacks)
    if (b.macro_slot < 0 || b.macro_slot >= kMacros || b.output_cache_address < 0 ||
        b.output_cache_address >= kCacheRows)
      return fail("CIM readback binding is outside the target profile");

  cudaSetDevice(runner->device);
  // Arena: merge the byte ranges of every row.
  struct Range {
    uintptr_t lo, hi;
  };
  std::vector<Range> ranges;
  ranges.reserve(num_inputs + num_outputs);
  for (int64_t i = 0; i < num_inputs; ++i) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(inputs[i]);
    ranges.push_back({a, a + (plan->inputs[i].data_type == CIM22_DATA_BF16 ? 128u : 64u)});
  }
  for (int64_t i = 0; i < num_outputs; ++i) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(outputs[i]);
    ranges.push_back({a, a + (plan->readbacks[i].data_type == CIM22_DATA_BF16 ? 32u : 64u)});
  }
  std::vector<Range> merged = ranges;
  std::sort(merged.begin(), merged.end(),
            [](const Range &a, const Range &b) { return a.lo < b.lo; });
  std::vector<Range> spans;
  for (const Range &r : merged) {
    if (!spans.empty() && r.lo < spans.back().hi)
      spans.back().hi = std::max(spans.back().hi, r.hi);
    else
      spans.push_back(r);
  }
  std::vector<size_t> span_offset(spans.size());
  size_t arena = 0;
  for (size_t i = 0; i < spans.size(); ++i) {
    // Keep each span's alignment modulo 16 so rows keep their natural
    // alignment relative to one another.
    arena = round_up(arena, 16) + (spans[i].lo & 15);
    span_offset[i] = arena;
    arena += spans[i].hi - spans[i].lo;
  }
  auto offset_of = [&](uintptr_t a) -> int64_t {
    auto it = std::upper_bound(spans.begin(), spans.end(), a,
                               [](uintptr_t v, const Range &r) { return v < r.lo; });
    const size_t idx = static_cast<size_t>(it - spans.begin()) - 1;
    return static_cast<int64_t>(span_offset[idx] + (a - spans[idx].lo));
  };
  const size_t arena_bytes = round_up(std::max<size_t>(arena, 16), 16);
  const size_t offsets_bytes = sizeof(int64_t) * (num_inputs + num_outputs);
  const size_t outcome_off = round_up(arena_bytes + offsets_bytes, 16);
  const size_t total = outcome_off + 16;
  if (total > runner->arena_capacity) {
    cudaFree(runner->d_arena);
    runner->d_arena = nullptr;
    if (!cuda_ok(cudaMalloc(&runner->d_arena, total * 2), "cudaMalloc"))
      return fail(last_error());
    runner->arena_capacity = total * 2;
  }
  if (total > runner->stage_capacity) {
    cudaFreeHost(runner->h_stage);
    runner->h_stage = nullptr;
    if (!cuda_ok(cudaMallocHost(&runner->h_stage, total * 2), "cudaMallocHost"))
      return fail(last_error());
    runner->stage_capacity = total * 2;
  }
  const size_t works = plan->works.size();
  const size_t scratch = std::max<size_t>(1, works) * 17;
  if (scratch > runner->scratch_capacity) {
    cudaFree(runner->d_scratch);
    runner->d_scratch = nullptr;
    if (!cuda_ok(cudaMalloc(&runner->d_scratch, scratch * 2 * sizeof(int32_t)), "cudaMalloc"))
      return fail(last_error());
    runner->scratch_capacity = scratch * 2;
  }
  uint8_t *stage = runner->h_stage;
  for (size_t i = 0; i < spans.size(); ++i)
    std::memcpy(stage + span_offset[i], reinterpret_cast<const void *>(spans[i].lo),
                spans[i].hi - spans[i].lo);
  int64_t *offs = reinterpret_cast<int64_t *>(stage + arena_bytes);
  for (int64_t i = 0; i < num_inputs; ++i)
    offs[i] = offset_of(reinterpret_cast<uintptr_t>(inputs[i]));
  for (int64_t i = 0; i < num_outputs; ++i)
    offs[num_inputs + i] = offset_of(reinterpret_cast<uintptr_t>(outputs[i]));
  cudaStream_t s = runner->stream;
  int32_t *results = runner->d_scratch;
  int32_t *codes = runner->d_scratch + std::max<size_t>(1, works) * 16;
  int32_t *d_outcome = reinterpret_cast<int32_t *>(runner->d_arena + outcome_off);
  bool ok = cuda_ok(cudaMemcpyAsync(runner->d_arena, stage, outcome_off,
                                    cudaMemcpyHostToDevice, s),
                    "cudaMemcpyAsync");
  if (ok) {
    runner_kernel<<<1, 1024, 0, s>>>(
        plan->d_works, plan->d_rbs, plan->d_waves, static_cast<int>(plan->waves.size()),
        runner->d_images, reinterpret_cast<const int64_t *>(runner->d_arena + arena_bytes),
        reinterpret_cast<const int64_t *>(runner->d_arena + arena_bytes) + num_inputs,
        runner->d_arena, bf16_compensation, results, codes, d_outcome);
    ok = cuda_ok(cudaGetLastError(), "runner launch") &&
         cuda_ok(cudaMemcpyAsync(stage, runner->d_arena, total, cudaMemcpyDeviceToHost, s),
                 "cudaMemcpyAsync") &&
         cuda_ok(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  }
  if (!ok)
    return fail(last_error());
  const int32_t *outcome = reinterpret_cast<const int32_t *>(stage + outcome_off);
  // Publish output rows back to the caller.
  for (int64_t i = 0; i < num_outputs; ++i) {
    const size_t bytes = plan->readbacks[i].data_type == CIM22_DATA_BF16 ? 32 : 64;
    std::memcpy(outputs[i], stage + offs[num_inputs + i], bytes);
  }
  // Replay residency and trace in execution order up to the failure.
  const int fail_kind = outcome[0];
  const int fail_index = outcome[1];
  const int32_t fail_code = outcome[2];
  trace.emit(CIM22_TRACE_BEGIN_RUN);
  for (const HostWave &wave : plan->waves) {
    for (int32_t i = wave.work_begin; i < wave.work_end; ++i) {
      const HostWork &hw = plan->works[i];
      const bool failing = fail_kind == 1 && fail_index == i;
      if (failing && !lane_stage(fail_code))
        return fail(code_message(fail_code));
      bool wrote = true;
      if (use_residency) {
        auto &slot = runner->slots[hw.slot];
        const int image = plan->work_images[i];
        if (slot.image == image && slot.mode == bf16_compensation) {
          wrote = false;
          ++runner->hits;
        } else {
          slot = {image, bf16_compensation};
          ++runner->writes;
        }
      }
      trace.emit(CIM22_TRACE_CONFIGURE_INPUT, hw.group_id, hw.work_id, hw.macro_slot);
      if (wrote)
        trace.emit(CIM22_TRACE_CONFIGURE_WEIGHT, hw.group_id, hw.work_id, hw.macro_slot);
      trace.emit(CIM22_TRACE_SELECT_MACRO, hw.group_id, hw.work_id, hw.macro_slot);
      trace.emit(CIM22_TRACE_START_WORK, hw.group_id, hw.work_id, hw.macro_slot);
      if (failing)
        return fail(code_message(fail_code));
    }
    for (int32_t r = wave.rb_begin; r < wave.rb_end; ++r) {
      const HostReadback &rb = plan->rbs[r];
      if (fail_kind == 2 && fail_index == r)
        return fail(code_message(fail_code));
      trace.emit(CIM22_TRACE_CONFIGURE_RETURN_ROUTE, rb.group_id, rb.work_id,
                 rb.macro_slot, rb.packet);
      trace.emit(CIM22_TRACE_READ_OUTPUT, rb.group_id, rb.work_id, rb.macro_slot,
                 rb.packet + 2, rb.address);
    }
  }
  if (fail_kind != 0)
    return fail(code_message(fail_code));
  trace.emit(CIM22_TRACE_COMPLETE);
  return 0;
}

} // extern "C"

// ---------------------------------------------------------------------------
// Session and the tile dispatch ABI (runtime/Runtime.cpp:120-247,249-340).

struct cim22_cuda_session {
  cim22_cuda_runner *runner = nullptr;
  struct Entry {
    cim22_cuda_plan *plan = nullptr;
    std::string kernel;
    int64_t inputs = 0, readbacks = 0;
    bool all_int8 = true, all_bf16 = true;
  };
  std::vector<Entry> transactions;
  std::string error;
  std::string refusal;
  uint64_t dispatches = 0;
  cim22_cuda_session *previous = nullptr;
};

namespace cim {
void session_refuse_dispatch(cim22_cuda_session *session, const std::string &message) {
  if (session)
    session->refusal = message;
}
} // namespace cim

namespace {
thread_local cim22_cuda_session *active_session = nullptr;

template <typename Input, typename Output>
void dispatch(int64_t id, cim22_memref2d *input, cim22_memref2d *output,
              int32_t mode) {
  if (!active_session)
    return;
  cim22_cuda_session &s = *active_session;
  constexpr bool int8 = std::is_same_v<Input, int8_t>;
  if (id < 0 || static_cast<size_t>(id) >= s.transactions.size() || !input ||
      !output || !input->aligned || !output->aligned || input->offset < 0 ||
      output->offset < 0 || input->sizes[0] < 0 || output->sizes[0] < 0 ||
      input->sizes[1] != 64 || input->strides[1] != 1 || input->strides[0] != 64 ||
      output->sizes[1] != 16 || output->strides[1] != 1 || output->strides[0] != 16) {
    s.error = "invalid native CIM dispatch descriptor";
    return;
  }
  const auto &entry = s.transactions[id];
  if (input->sizes[0] != entry.inputs || output->sizes[0] != entry.readbacks ||
      (int8 ? !entry.all_int8 : !entry.all_bf16)) {
    s.error = "native CIM dispatch transaction type or count mismatch";
    return;
  }
  Input *in = static_cast<Input *>(input->aligned) + input->offset;
  Output *out = static_cast<Output *>(output->aligned) + output->offset;
  std::fill_n(out, output->sizes[0] * 16, Output{0});
  if (!s.error.empty())
    return;
  if (!s.refusal.empty()) {
    s.error = s.refusal;
    return;
  }
  std::vector<const void *> rows(input->sizes[0]);
  std::vector<void *> outs(output->sizes[0]);
  for (int64_t i = 0; i < input->sizes[0]; ++i)
    rows[i] = in + i * 64;
  for (int64_t i = 0; i < output->sizes[0]; ++i)
    outs[i] = out + i * 16;
  ++s.dispatches;
  char message[512];
  if (cim22_cuda_runner_run(s.runner, entry.plan, mode, rows.data(),
                            static_cast<int64_t>(rows.size()), outs.data(),
                            static_cast<int64_t>(outs.size()), 1, nullptr, nullptr,
                            message, sizeof message))
    s.error = entry.kernel + ": " + message;
}
} // namespace

extern "C" {

cim22_cuda_session *cim22_cuda_session_create(int device, char *error,
                                              size_t error_capacity) {
  cim22_cuda_runner *runner = cim22_cuda_runner_create(device, error, error_capacity);
  if (!runner)
    return nullptr;
  auto *s = new cim22_cuda_session();
  s->runner = runner;
  return s;
}

void cim22_cuda_session_destroy(cim22_cuda_session *session) {
  if (!session)
    return;
  if (active_session == session)
    active_session = session->previous;
  for (auto &e : session->transactions)
    cim22_cuda_plan_destroy(e.plan);
  cim22_cuda_runner_destroy(session->runner);
  delete session;
}

int64_t cim22_cuda_session_add_transaction(cim22_cuda_session *session,
                                           const cim22_transaction *transaction,
                                           const char *kernel_name, char *error,
                                           size_t error_capacity) {
  if (!session || !transaction) {
    copy_error("invalid CIM session arguments", error, error_capacity);
    return -1;
  }
  cim22_cuda_plan *plan =
      cim22_cuda_plan_create(session->runner, transaction, 1, error, error_capacity);
  if (!plan)
    return -1;
  cim22_cuda_session::Entry e;
  e.plan = plan;
  e.kernel = kernel_name ? kernel_name : "";
  e.inputs = transaction->num_inputs;
  e.readbacks = transaction->num_readbacks;
  for (int64_t i = 0; i < transaction->num_inputs; ++i) {
    e.all_int8 &= transaction->inputs[i].data_type == CIM22_DATA_INT8;
    e.all_bf16 &= transaction->inputs[i].data_type == CIM22_DATA_BF16;
  }
  for (int64_t i = 0; i < transaction->num_readbacks; ++i) {
    e.all_int8 &= transaction->readbacks[i].data_type == CIM22_DATA_INT8;
    e.all_bf16 &= transaction->readbacks[i].data_type == CIM22_DATA_BF16;
  }
  session->transactions.push_back(std::move(e));
  return static_cast<int64_t>(session->transactions.size() - 1);
}

int64_t cim22_cuda_session_num_transactions(const cim22_cuda_session *session) {
  return session ? static_cast<int64_t>(session->transactions.size()) : -1;
}

void cim22_cuda_session_begin_invoke(cim22_cuda_session *session) {
  if (!session)
    return;
  session->error.clear();
  session->dispatches = 0;
  session->previous = active_session;
  active_session = session;
}

int cim22_cuda_session_end_invoke(cim22_cuda_session *session) {
  if (!session)
    return 1;
  if (active_session == session)
    active_session = session->previous;
  session->previous = nullptr;
  if (!session->error.empty())
    cim22_cuda_runner_clear_residency(session->runner);
  return session->error.empty() ? 0 : 1;
}

uint64_t cim22_cuda_session_dispatch_count(const cim22_cuda_session *session) {
  return session ? session->dispatches : 0;
}

const char *cim22_cuda_session_error(const cim22_cuda_session *session) {
  return session ? session->error.c_str() : "null session";
}

void _mlir_ciface_cim22_dispatch(int64_t id, cim22_memref2d *input,
                                 cim22_memref2d *output) {
  dispatch<uint16_t, uint16_t>(id, input, output, CIM22_BF16_NONE);
}

void _mlir_ciface_cim22_dispatch_sign_split(int64_t id, cim22_memref2d *input,
                                            cim22_memref2d *output) {
  dispatch<uint16_t, uint16_t>(id, input, output, CIM22_BF16_SIGN_SPLIT);
}

void _mlir_ciface_cim22_dispatch_legacy(int64_t id, cim22_memref2d *input,
                                        cim22_memref2d *output) {
  dispatch<uint16_t, uint16_t>(id, input, output, CIM22_BF16_LEGACY);
}

void _mlir_ciface_cim22_dispatch_int8(int64_t id, cim22_memref2d *input,
                                      cim22_memref2d *output) {
  dispatch<int8_t, int32_t>(id, input, output, CIM22_BF16_NONE);
}

} // extern "C"
