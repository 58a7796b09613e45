// ORACLE - test infrastructure only.
//
// C entry points over the reference's own software CIM runner: the
// mlir-cim22 sources lib/Execution/CIMSoftwareRunner.cpp,
// lib/Execution/BF16Compensation.cpp and lib/Support/BF16Support.cpp,
// compiled unmodified (oracle/Makefile) against the clean-room LLVM support
// subset in oracle/llvm_shim. Used by the tests to check the restated oracle
// against the reference on random transactions, and by the benchmark's CPU
// legs as the reference's CPU simulation.
//
// ref_linear_bf16_runner drives the runner the way a compiled model does: the
// Host glue of the reference's lowering (lib/Conversion/LinalgToCIM/Passes.cpp)
// is restated here - weights split into Wp/Wn and rounded to BF16
// (:2360-2373,2440-2447) and prealigned per 16x64 tile at compile time with
// the reference's prealignBF16WeightTile (lib/Dialect/CIMFrame/Transforms/
// Passes.cpp:129-137); activations split into xp/xn and rounded to BF16
// (:2379-2399,2422-2476); K/N tiled with zero padding (:760-826); each column's
// crossbar tiles dispatched in transactions of at most 40 Works
// (:437-438) with a reused Plan and weight residency (runtime/Runtime.cpp:
// 187-204); BF16 tiles summed in f32 in tile order and rounded to BF16 when
// there is more than one K tile (:828-857); branches merged as
// ((pp - pn) - np) + nn (:2395-2416); then the bias.
#include "CIM22/Execution/CIMRunner.h"
#include "CIM22/Support/BF16Support.h"

#include "../include/cim22_cuda.h"

#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

using namespace cim22::execution;

namespace {

constexpr int kIn = 64, kOut = 16, kMaxWorks = 40;

void copyError(const std::string &message, char *error, size_t capacity) {
  if (!error || capacity == 0)
    return;
  const size_t n = std::min(message.size(), capacity - 1);
  std::memcpy(error, message.data(), n);
  error[n] = '\0';
}

CIMDataType dataType(int32_t t) {
  return t == CIM22_DATA_BF16 ? CIMDataType::BF16 : CIMDataType::Int8;
}

std::array<int32_t, 6> route6(const int32_t *r) {
  std::array<int32_t, 6> out{};
  std::copy_n(r, 6, out.begin());
  return out;
}

std::array<int32_t, 3> route3(const int32_t *r) {
  std::array<int32_t, 3> out{};
  std::copy_n(r, 3, out.begin());
  return out;
}

// The C transaction (include/cim22_cuda.h mirrors CIMExecutable.h) as the
// reference's CIMTransaction.
std::unique_ptr<CIMTransaction> toTransaction(const cim22_transaction &t) {
  std::vector<CIMGroup> groups;
  for (int64_t g = 0; g < t.num_groups; ++g) {
    CIMGroup group;
    group.groupId = t.groups[g].group_id;
    for (int64_t w = 0; w < t.groups[g].num_works; ++w) {
      const cim22_work &src = t.groups[g].works[w];
      group.works.push_back({src.work_id, src.core_slot, src.macro_slot, route6(src.route)});
    }
    groups.push_back(std::move(group));
  }
  std::vector<StaticWeightSection> weights;
  for (int64_t i = 0; i < t.num_weights; ++i) {
    const cim22_static_weight &src = t.weights[i];
    StaticWeightSection w;
    w.groupId = src.group_id;
    w.workId = src.work_id;
    w.coreSlot = src.core_slot;
    w.macroSlot = src.macro_slot;
    w.route = route6(src.route);
    if (src.words && src.num_words > 0)
      w.words.assign(src.words, src.words + src.num_words);
    std::copy_n(src.values, kOut * kIn, w.values.begin());
    std::copy_n(src.exponents, kOut, w.exponents.begin());
    w.dataType = dataType(src.data_type);
    weights.push_back(std::move(w));
  }
  std::vector<CIMFramePacket> packets;
  for (int64_t i = 0; i < t.num_packets; ++i) {
    const cim22_frame_packet &src = t.packets[i];
    CIMFramePacket p{static_cast<CIMPacketKind>(src.kind)};
    p.route = route6(src.route);
    p.groupId = src.group_id;
    p.workId = src.work_id;
    p.macroSlot = src.macro_slot;
    p.cacheAddress = src.cache_address;
    p.testCore = route3(src.test_core);
    p.dataType = dataType(src.data_type);
    packets.push_back(p);
  }
  std::vector<DynamicInputBinding> inputs;
  for (int64_t i = 0; i < t.num_inputs; ++i) {
    const cim22_input_binding &src = t.inputs[i];
    inputs.push_back({src.group_id, src.work_id, src.macro_slot, src.input_slot,
                      dataType(src.data_type), src.input_cache_address});
  }
  std::vector<ReadbackBinding> readbacks;
  for (int64_t i = 0; i < t.num_readbacks; ++i) {
    const cim22_readback_binding &src = t.readbacks[i];
    ReadbackBinding r;
    r.groupId = src.group_id;
    r.workId = src.work_id;
    r.macroSlot = src.macro_slot;
    r.outputCacheAddress = src.output_cache_address;
    r.route = route6(src.route);
    r.testCore = route3(src.test_core);
    r.dataType = dataType(src.data_type);
    readbacks.push_back(r);
  }
  return std::make_unique<CIMTransaction>(
      t.target_profile ? t.target_profile : "", t.target_profile_version,
      t.execution_plan_version, std::move(groups), std::move(weights), std::move(packets),
      std::move(inputs), std::move(readbacks), std::vector<uint64_t>{});
}

// A session: one runner, its weight catalog and Macro weight residency.
struct Session {
  explicit Session(BF16Compensation mode) : runner(mode) {}
  CIMSoftwareRunner runner;
  CIMWeightCatalog catalog;
  CIMWeightResidency residency;
};

// A prepared transaction: the reference's Plan and weight identities.
struct Prepared {
  std::unique_ptr<CIMTransaction> transaction;
  std::unique_ptr<CIMSoftwareRunner::Plan> plan;
  std::vector<CIMWeightIdentity> identities;
};

Prepared prepare(std::unique_ptr<CIMTransaction> txn, bool batch, CIMWeightCatalog &catalog) {
  Prepared p;
  p.transaction = std::move(txn);
  p.plan = std::make_unique<CIMSoftwareRunner::Plan>(*p.transaction, batch);
  for (const StaticWeightSection &w : p.transaction->getStaticWeights())
    p.identities.push_back(catalog.intern(w));
  return p;
}

// arith.truncf: FP32 -> BF16 bits, round to nearest even; NaN stays NaN.
uint16_t f32ToBF16(float v) {
  uint32_t bits;
  std::memcpy(&bits, &v, sizeof bits);
  if (std::isnan(v))
    return static_cast<uint16_t>((bits >> 16) | 0x40u);
  bits += 0x7fffu + ((bits >> 16) & 1u);
  return static_cast<uint16_t>(bits >> 16);
}

float bf16ToF32(uint16_t b) {
  const uint32_t bits = static_cast<uint32_t>(b) << 16;
  float v;
  std::memcpy(&v, &bits, sizeof v);
  return v;
}

} // namespace

extern "C" {

void *ref_runner_create(int mode) {
  return new Session(static_cast<BF16Compensation>(mode));
}

void ref_runner_destroy(void *session) { delete static_cast<Session *>(session); }

void ref_runner_stats(void *session, uint64_t *writes, uint64_t *hits) {
  const auto *s = static_cast<Session *>(session);
  *writes = s->residency.stats.writes;
  *hits = s->residency.stats.hits;
}

// CIMSoftwareRunner::run on one transaction with a freshly built Plan; rows
// are 64 int8 or BF16 inputs in dynamic-input binding order and 16 int32 or
// BF16 outputs in readback order, by each binding's data type. With
// use_residency the session's catalog and residency are used. Returns 0, or
// 1 with the runner's error text.
int ref_runner_run(void *session, const cim22_transaction *transaction, int batch_readbacks,
                   const void *const *inputs, int64_t num_inputs, void *const *outputs,
                   int64_t num_outputs, int use_residency, char *error, size_t capacity) {
  auto *s = static_cast<Session *>(session);
  Prepared p = prepare(toTransaction(*transaction), batch_readbacks != 0, s->catalog);
  const auto in_bindings = p.transaction->getDynamicInputs();
  const auto rb = p.transaction->getReadbacks();
  std::vector<CIMInputView> in(static_cast<size_t>(num_inputs));
  for (int64_t i = 0; i < num_inputs; ++i) {
    if (!inputs[i])
      continue;
    const bool bf16 = static_cast<size_t>(i) < in_bindings.size() &&
                      in_bindings[i].dataType == CIMDataType::BF16;
    if (bf16)
      in[i].bf16Values = llvm::ArrayRef<uint16_t>(static_cast<const uint16_t *>(inputs[i]), kIn);
    else
      in[i].values = llvm::ArrayRef<int8_t>(static_cast<const int8_t *>(inputs[i]), kIn);
  }
  std::vector<CIMOutputView> out(static_cast<size_t>(num_outputs));
  for (int64_t i = 0; i < num_outputs; ++i) {
    if (!outputs[i])
      continue;
    const bool bf16 = static_cast<size_t>(i) < rb.size() && rb[i].dataType == CIMDataType::BF16;
    if (bf16)
      out[i].bf16Values = llvm::MutableArrayRef<uint16_t>(static_cast<uint16_t *>(outputs[i]), kOut);
    else
      out[i].values = llvm::MutableArrayRef<int32_t>(static_cast<int32_t *>(outputs[i]), kOut);
  }
  CIMRunInputs run_in{llvm::ArrayRef<CIMInputView>(in)};
  CIMRunOutputs run_out{llvm::MutableArrayRef<CIMOutputView>(out)};
  llvm::Error e = use_residency
                      ? s->runner.run(*p.plan, run_in, run_out, s->residency, p.identities)
                      : s->runner.run(*p.plan, run_in, run_out);
  if (e) {
    copyError(llvm::toString(std::move(e)), error, capacity);
    return 1;
  }
  return 0;
}

// A sign-split BF16 layer y[m, n] = x[m, k] W[n, k]^T (+ bias) computed by the
// reference's runner, one column at a time, on `threads` host threads (one
// session each). branches: 4, or 2 when every x >= 0.
int ref_linear_bf16_runner(const float *x, int64_t m, int64_t k, const float *w, int64_t n,
                           const float *bias, int branches, float *y, int threads, char *error,
                           size_t capacity) {
  for (int64_t i = 0; i < n * k; ++i)
    if (!std::isfinite(w[i])) {
      copyError("BF16 correction requires finite fixed weights", error, capacity);
      return 1;
    }
  const int64_t T = (k + kIn - 1) / kIn, J = (n + kOut - 1) / kOut;
  // Compile time: split, round and prealign the weight tiles [sign][j][t].
  std::vector<mlir::cim22::BF16PrealignedWeightTile> tiles(2 * J * T);
  for (int sign = 0; sign < 2; ++sign)
    for (int64_t j = 0; j < J; ++j)
      for (int64_t t = 0; t < T; ++t) {
        std::array<uint16_t, kOut * kIn> bits{};
        for (int lane = 0; lane < kOut; ++lane)
          for (int i = 0; i < kIn; ++i) {
            const int64_t row = j * kOut + lane, col = t * kIn + i;
            if (row >= n || col >= k)
              continue;
            const float v = w[row * k + col];
            const bool negative = std::signbit(v), zero = v == 0.0f;
            if (sign == 0)
              bits[lane * kIn + i] = (negative || zero) ? 0 : f32ToBF16(v);
            else
              bits[lane * kIn + i] = (!negative || zero) ? 0 : f32ToBF16(-v);
          }
        tiles[(sign * J + j) * T + t] = mlir::cim22::prealignBF16WeightTile(bits);
      }
  struct Item {
    int b;
    int64_t j, t;
  };
  std::vector<Item> items;
  for (int b = 0; b < branches; ++b)
    for (int64_t j = 0; j < J; ++j)
      for (int64_t t = 0; t < T; ++t)
        items.push_back({b, j, t});
  // Transactions of at most 40 Works: one group, Work s on Core s/2, Macro
  // s%2, each with its input write, weight exponent, weight, return route,
  // control and output Cache read packets.
  struct Chunk {
    std::vector<Item> items;
    cim22_transaction c{};
    std::vector<cim22_work> works;
    cim22_group group{};
    std::vector<cim22_static_weight> weights;
    std::vector<cim22_frame_packet> packets;
    std::vector<cim22_input_binding> inputs;
    std::vector<cim22_readback_binding> readbacks;
  };
  std::vector<std::unique_ptr<Chunk>> chunks;
  for (size_t s0 = 0; s0 < items.size(); s0 += kMaxWorks) {
    auto c = std::make_unique<Chunk>();
    const size_t e = std::min(items.size(), s0 + kMaxWorks);
    for (size_t i = s0; i < e; ++i) {
      const Item &it = items[i];
      const int64_t slot = static_cast<int64_t>(i - s0);
      cim22_work wk{};
      wk.work_id = slot;
      wk.core_slot = slot / 2;
      wk.macro_slot = slot % 2;
      c->works.push_back(wk);
      cim22_static_weight sw{};
      sw.group_id = 0;
      sw.work_id = slot;
      sw.core_slot = slot / 2;
      sw.macro_slot = slot % 2;
      sw.data_type = CIM22_DATA_BF16;
      const auto &tile = tiles[((it.b & 1) * J + it.j) * T + it.t];
      std::copy(tile.mantissas.begin(), tile.mantissas.end(), sw.values);
      std::copy(tile.exponents.begin(), tile.exponents.end(), sw.exponents);
      c->weights.push_back(sw);
      c->inputs.push_back({0, slot, slot % 2, slot, CIM22_DATA_BF16, 0});
      cim22_readback_binding rbk{};
      rbk.group_id = 0;
      rbk.work_id = slot;
      rbk.macro_slot = slot % 2;
      rbk.output_cache_address = 0;
      rbk.data_type = CIM22_DATA_BF16;
      c->readbacks.push_back(rbk);
      for (int kind : {CIM22_PACKET_INPUT_CACHE_WRITE, CIM22_PACKET_WEIGHT_EXPONENT,
                       CIM22_PACKET_WEIGHT, CIM22_PACKET_RETURN_ROUTE, CIM22_PACKET_CONTROL,
                       CIM22_PACKET_OUTPUT_CACHE_READ}) {
        cim22_frame_packet p{};
        p.kind = kind;
        p.group_id = 0;
        p.work_id = slot;
        p.macro_slot = slot % 2;
        p.cache_address = kind == CIM22_PACKET_OUTPUT_CACHE_READ ? 0 : -1;
        p.data_type = CIM22_DATA_BF16;
        c->packets.push_back(p);
      }
      c->items.push_back(it);
    }
    c->group.group_id = 0;
    c->group.works = c->works.data();
    c->group.num_works = static_cast<int64_t>(c->works.size());
    c->c.target_profile = "cim22-4x5-v1";
    c->c.target_profile_version = 1;
    c->c.execution_plan_version = 1;
    c->c.groups = &c->group;
    c->c.num_groups = 1;
    c->c.weights = c->weights.data();
    c->c.num_weights = static_cast<int64_t>(c->weights.size());
    c->c.packets = c->packets.data();
    c->c.num_packets = static_cast<int64_t>(c->packets.size());
    c->c.inputs = c->inputs.data();
    c->c.num_inputs = static_cast<int64_t>(c->inputs.size());
    c->c.readbacks = c->readbacks.data();
    c->c.num_readbacks = static_cast<int64_t>(c->readbacks.size());
    chunks.push_back(std::move(c));
  }
  std::atomic<int> failed{0};
  std::mutex lock;
  std::string firstError;
  int64_t firstColumn = INT64_MAX;
  auto body = [&](int64_t c0, int64_t c1) {
    Session session(BF16Compensation::SignSplit);
    std::vector<Prepared> plans;
    for (const auto &c : chunks)
      plans.push_back(prepare(toTransaction(c->c), true, session.catalog));
    std::vector<uint16_t> xp(T * kIn), xn(T * kIn);
    std::vector<std::array<uint16_t, kIn>> rows(kMaxWorks);
    std::vector<std::array<uint16_t, kOut>> outs(kMaxWorks);
    std::vector<CIMInputView> in(kMaxWorks);
    std::vector<CIMOutputView> out(kMaxWorks);
    std::vector<std::array<uint16_t, kOut>> results(branches * J * T);
    for (int64_t col = c0; col < c1; ++col) {
      std::fill(xp.begin(), xp.end(), 0);
      std::fill(xn.begin(), xn.end(), 0);
      for (int64_t i = 0; i < k; ++i) {
        const float v = x[col * k + i];
        float pos = v, neg = 0.0f;
        if (branches == 4) {
          pos = v < 0.0f ? 0.0f : v;
          neg = v < 0.0f ? -v : 0.0f;
        }
        if (v == 0.0f)
          pos = 0.0f; // -0 -> +0
        xp[i] = f32ToBF16(pos);
        xn[i] = f32ToBF16(neg);
      }
      for (size_t ci = 0; ci < chunks.size(); ++ci) {
        const Chunk &c = *chunks[ci];
        const size_t R = c.items.size();
        for (size_t r = 0; r < R; ++r) {
          const Item &it = c.items[r];
          const std::vector<uint16_t> &src = it.b < 2 ? xp : xn;
          std::copy_n(src.data() + it.t * kIn, kIn, rows[r].begin());
          outs[r].fill(0); // the dispatch zero-fills outputs (Runtime.cpp:154-155)
          in[r].bf16Values = llvm::ArrayRef<uint16_t>(rows[r]);
          out[r].bf16Values = llvm::MutableArrayRef<uint16_t>(outs[r]);
        }
        CIMRunInputs run_in{llvm::ArrayRef<CIMInputView>(in.data(), R)};
        CIMRunOutputs run_out{llvm::MutableArrayRef<CIMOutputView>(out.data(), R)};
        llvm::Error e = session.runner.run(*plans[ci].plan, run_in, run_out, session.residency,
                                           plans[ci].identities);
        if (e) {
          std::lock_guard<std::mutex> g(lock);
          if (col < firstColumn) {
            firstColumn = col;
            firstError = llvm::toString(std::move(e));
          }
          failed.store(1);
          return;
        }
        for (size_t r = 0; r < R; ++r) {
          const Item &it = c.items[r];
          results[(it.b * J + it.j) * T + it.t] = outs[r];
        }
      }
      for (int64_t j = 0; j < J; ++j) {
        float branch[4][kOut];
        for (int b = 0; b < branches; ++b)
          for (int lane = 0; lane < kOut; ++lane) {
            float acc = bf16ToF32(results[(b * J + j) * T][lane]);
            for (int64_t t = 1; t < T; ++t)
              acc = acc + bf16ToF32(results[(b * J + j) * T + t][lane]);
            branch[b][lane] = T > 1 ? bf16ToF32(f32ToBF16(acc)) : acc;
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
