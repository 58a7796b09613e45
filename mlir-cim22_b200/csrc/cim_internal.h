// cim_internal.h - shared host-side definitions of the CUDA backend.
#pragma once

#include "../../include/cim22_cuda.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

namespace cim {

// Thread-local diagnostic of the last failing C-ABI call.
void set_last_error(const std::string &message);
const std::string &last_error();

// Copy a message into a caller buffer (truncating, NUL-terminated), the
// convention of runtime/Runtime.cpp:64-71.
void copy_error(const std::string &message, char *buffer, size_t capacity);

// Makes every later dispatch on the session fail with `message` after the
// descriptor checks and the output zero fill, as a USB-backend model without
// a configured board does (runtime/Runtime.cpp:175-179).
void session_refuse_dispatch(cim22_cuda_session *session, const std::string &message);

inline bool cuda_ok(cudaError_t e, const char *what) {
  if (e == cudaSuccess)
    return true;
  set_last_error(std::string(what) + ": " + cudaGetErrorString(e));
  return false;
}

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// Lane padding of resident weights: a multiple of every N tile width the
// layer kernels use.
constexpr int64_t kLanePad = 128;
// Column padding of prepared activations: a multiple of the M tile.
constexpr int64_t kColumnPad = 128;

// Division by an invariant divisor as a multiply-high and shift (Granlund and
// Montgomery, "Division by invariant integers using multiplication", 1994):
// q = (umulhi(n, mul) + n) >> shift for 0 <= n < 2^31, with
// shift = ceil(log2 d) and mul = floor(2^32 (2^shift - d) / d) + 1.
struct FastDiv {
  uint32_t d, mul, shift;
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f{d, 0, 0};
  uint32_t l = 0;
  while ((uint64_t{1} << l) < d)
    ++l;
  f.shift = l;
  f.mul = static_cast<uint32_t>(((uint64_t{1} << 32) * ((uint64_t{1} << l) - d)) / d + 1);
  return f;
}

#if defined(__CUDACC__)
__device__ __forceinline__ int fdiv(int n, const FastDiv &f) {
  return static_cast<int>((__umulhi(static_cast<uint32_t>(n), f.mul) + static_cast<uint32_t>(n)) >> f.shift);
}
#endif

// Programmatic dependent launch. Layer and glue kernels are launched with
// launch_pdl, so the next kernel in the stream (or CUDA graph) is scheduled
// while the current one drains; each kernel calls pdl_launch_dependents()
// once its CTAs run and pdl_wait() before its first access to memory that
// another kernel reads or writes (only barrier setup, TMEM allocation and
// reads of resident weights come earlier). griddepcontrol.wait returns once
// every earlier grid has completed and its writes are visible; without the
// launch attribute both instructions are no-ops.
#if defined(__CUDACC__)
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
#endif

} // namespace cim

// Prepared CIM layer weights resident in device memory.
struct cim22_cuda_layer {
  int device = 0;
  bool bf16 = false;
  int mode = CIM22_BF16_SIGN_SPLIT; // BF16 compensation (Legacy / None: signed, unsplit)
  int64_t n = 0, k = 0;         // logical output lanes and reduction length
  int64_t n_pad = 0, k_pad = 0; // padded to kLanePad and 64
  int64_t tiles = 0;            // K tiles (k_pad / 64)
  bool range_safe = true;       // INT8 range proof result
  // BF16: int8 mantissas [2][n_pad][k_pad] (Wp then Wn) and int32 lane
  // exponents [2][tiles][n_pad], the per-tile, per-32-lane-block
  // weight-exponent ranges [tiles][n_pad / 32][4] and the f32 weight scales
  // 2^(Ew - 133) [2][tiles][n_pad]. BF16 Legacy / None: int8 [n_pad][k_pad]
  // signed, int32 exponents [tiles][n_pad] then per (tile, 16-lane tile) a
  // flag for a lane of all -128 mantissas. INT8: int8 [n_pad][k_pad].
  int8_t *weights = nullptr;
  int32_t *exponents = nullptr;
  // BF16 sign-split layers of at least kOperandMinLanes lanes whose nonzero
  // weight lanes all have exponents in [kOperandEwMin, kOperandEwMax]: the
  // scaled BF16 operands b * 2^(Ew - 133)
  // [2][n_pad][k_pad] of the tensor-core contraction with BF16 operands, and
  // the window [ex_lo, ex_hi] of activation group exponents whose prepared
  // values a * 2^(Ex - 133) it multiplies exactly (null / empty otherwise).
  uint16_t *operands = nullptr;
  int32_t ex_lo = 1, ex_hi = 0;
};

namespace cim {
// Layers of at least this many output lanes take BF16 operands. Measured on
// B200: the contraction with BF16 operands is faster wherever it runs, and
// with the TMA-stored prepare its two bytes per element cost less than that
// gain from 64 lanes on (every ResNet-18 and event-CNN convolution after the
// first, the Linear stacks); narrower layers stay on int8 mantissas.
constexpr int64_t kOperandMinLanes = 64;
// The weight exponents that BF16 operands admit: every nonzero scaled weight
// b * 2^(Ew - 133) (1 <= b <= 127) is a normal BF16 value, and a dot p < 2^20
// of unscaled activation mantissas times them stays a finite normal f32.
constexpr int kOperandEwMin = 8, kOperandEwMax = 241;
// Activation group exponents with scaled operands: a * 2^(Ex - 133) normal
// (Ex >= 8), the preparation's offset 2^(Ex - 110) finite (Ex <= 237), and
// for every weight exponent of the layer 140 <= Ex + Ew <= 374, so that a
// dot's f32 value p * 2^(Ex + Ew - 266) is normal and finite.
constexpr int kOperandExMin = 8, kOperandExMax = 237;
} // namespace cim
