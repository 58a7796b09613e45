// signsplit_prep.cuh - device routines shared by the sign-split layer
// kernels (layers.cu), the contraction that prepares its own operand tiles
// (gemm_tc.cu) and the fused layer-chain kernel (chain.cu): the 8-thread group
// preparation of activations (split, RNE to BF16, group maximum,
// ExpPrealign), the thread-per-group finish of a prepared group and its
// stores, the exact slow restore of one tile and the epilogue activations.
#pragma once

#include "cim_internal.h"
#include "cim_numeric.cuh"
#include "tma_util.cuh"

#include <cuda_bf16.h>

namespace cim {
namespace {

constexpr unsigned kFull = 0xffffffffu;

// Exact path for groups whose maximum is tiny (exponent < 8): RNE scaling of
// the element, then ExpPrealign at exponent 127. Out of line so the fast path
// is not predicated through it.
__device__ __noinline__ uint32_t slow_align(uint32_t p, int shift) {
  return static_cast<uint8_t>(prealign_element(bf16_scalbn(static_cast<uint16_t>(p), shift), 127));
}

// Low bytes of four words, in order, as one word.
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c,
                                                   uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

constexpr int kGroupThreads = 8;

// Split, round and prealign the thread's eight values of a group shared by
// the eight lanes of `mask` (sub = lane within them): out[a] holds the eight
// aligned bytes of activation branch a, emax[a] the group exponent
// (kZeroGroup for an all-zero group).
//
// Split and round: xp = max(x, 0), xn = max(-x, 0) equal the reference's
// selects for every non-NaN x up to the sign of zero, which the preparation
// clears anyway (BF16Compensation.cpp:97). cvt.rn.bf16x2.f32 rounds to
// nearest even, as arith.truncf does. NaN, infinity and finite values that
// round to BF16 infinity (|x| >= 0x1.fep127) mark the group non-finite:
// through the BF16 exponent 0xff of the maximum for a 2-branch layer, through
// |x| of the raw inputs otherwise (the max with 0 drops NaN).
// Split and round eight values: packed[a] holds the BF16 magnitudes of
// activation branch a in pairs (element 2e in the low half), mx[a] their
// maximum. flags accumulates what marks a group: for 4-branch layers the
// largest |x| bit pattern (non-finite when >= 0x7f7f8000: NaN, infinity or a
// value that rounds to BF16 infinity), for 2-branch layers the largest BF16
// bit pattern of either half (above 0x8000 exactly when some input rounds to
// a negative nonzero BF16 value, which the reference's sign split rejects;
// -0 is cleared to +0).
template <int kActBranches>
__device__ __forceinline__ void split8(const float (&v)[8], uint32_t (&packed)[2][4],
                                       uint32_t (&mx)[2], uint32_t &flags) {
  if (kActBranches == 2) {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      flags = max(flags, __float_as_uint(v[e]) & 0x7fffffffu);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const __nv_bfloat162 hp = __floats2bfloat162_rn(fmaxf(v[e], 0.0f), fmaxf(v[e + 1], 0.0f));
      const __nv_bfloat162 hn =
          __floats2bfloat162_rn(fmaxf(-v[e], 0.0f), fmaxf(-v[e + 1], 0.0f));
      packed[0][e / 2] = *reinterpret_cast<const uint32_t *>(&hp) & 0x7fff7fffu;
      packed[kActBranches - 1][e / 2] = *reinterpret_cast<const uint32_t *>(&hn) & 0x7fff7fffu;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const __nv_bfloat162 hp = __floats2bfloat162_rn(v[e], v[e + 1]);
      const uint32_t bits = *reinterpret_cast<const uint32_t *>(&hp);
      flags = __vmaxu2(flags, bits);
      packed[0][e / 2] = bits & 0x7fff7fffu;
    }
  }
#pragma unroll
  for (int a = 0; a < kActBranches; ++a) {
    const uint32_t m2 = __vmaxu2(__vmaxu2(packed[a][0], packed[a][1]),
                                 __vmaxu2(packed[a][2], packed[a][3]));
    mx[a] = max(mx[a], max(m2 & 0xffffu, m2 >> 16));
  }
}

// The group verdict from its maxima and flags: non-finite (status, and every
// branch a zero group), negative input to a 2-branch layer (status), and the
// group exponent of each branch (kZeroGroup for an all-zero branch).
template <int kActBranches>
__device__ __forceinline__ void group_exponents(uint32_t (&mx)[2], uint32_t flags, bool report,
                                                int32_t *status, int (&emax)[2]) {
  if (kActBranches == 2 && flags >= 0x7f7f8000u)
    mx[0] = 0xffffu;
  const bool nonfinite = mx[0] >= 0x7f80u;
  if (report && nonfinite)
    atomicOr(status, CIM22_STATUS_INPUT_NOT_FINITE);
  if (kActBranches == 1 && max(flags & 0xffffu, flags >> 16) > 0x8000u && !nonfinite)
    atomicOr(status, CIM22_STATUS_NEGATIVE_INPUT);
#pragma unroll
  for (int a = 0; a < kActBranches; ++a) {
    const bool zero = mx[a] == 0 || nonfinite;
    emax[a] = zero ? kZeroGroup : effective_exponent(static_cast<uint16_t>(mx[a]));
  }
}

// ExpPrealign of eight BF16 magnitudes (packed in pairs) against a group of
// maximum mx and exponent emax; zeros for a zero group (emax == kZeroGroup),
// which never enters the exact path (a caller's select on the zero case may
// be if-converted into evaluating this function for it).
__device__ __forceinline__ uint2 align8(const uint32_t (&packed)[4], uint32_t mx, int emax) {
  uint32_t lo = 0, hi = 0;
  const bool zero = emax == kZeroGroup;
  if (zero || (mx >> 7) >= 8) {
    const float scale = __uint_as_float(static_cast<uint32_t>(260 - emax) << 23);
    uint32_t q[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      q[2 * e] =
          __float_as_uint(__fmaf_rz(__uint_as_float(packed[e] << 16), scale, 8388608.0f));
      q[2 * e + 1] = __float_as_uint(
          __fmaf_rz(__uint_as_float(packed[e] & 0xffff0000u), scale, 8388608.0f));
    }
    lo = zero ? 0u : pack_low_bytes(q[0], q[1], q[2], q[3]);
    hi = zero ? 0u : pack_low_bytes(q[4], q[5], q[6], q[7]);
  } else {
    const int shift = 127 - emax;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      lo |= slow_align((packed[e / 2] >> (16 * (e & 1))) & 0xffffu, shift) << (8 * e);
      hi |= slow_align((packed[2 + e / 2] >> (16 * (e & 1))) & 0xffffu, shift) << (8 * e);
    }
  }
  return make_uint2(lo, hi);
}

// Scaled BF16 operand values of four aligned elements for the contraction
// with BF16 operands: r holds 2^23 + a for each aligned mantissa a (the bit
// patterns of the alignment fma); one packed fma per pair computes
// a * s = r * s + off (off = -2^23 * s, exact), rounded to BF16 exactly (a has
// at most 7 significant bits). s = 2^(Ex - 133) inside the layer's window,
// else 1: the unscaled mantissa, restored exactly by the epilogue.
__device__ __forceinline__ uint2 scale_pairs(const uint32_t (&r)[4], uint64_t s2,
                                             uint64_t off2) {
  uint32_t y[4];
#pragma unroll
  for (int h = 0; h < 2; ++h)
    asm("{\n\t.reg .b64 a, d;\n\tmov.b64 a, {%2, %3};\n\t"
        "fma.rn.f32x2 d, a, %4, %5;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=r"(y[2 * h]), "=r"(y[2 * h + 1])
        : "r"(r[2 * h]), "r"(r[2 * h + 1]), "l"(s2), "l"(off2));
  const __nv_bfloat162 lo = __floats2bfloat162_rn(__uint_as_float(y[0]), __uint_as_float(y[1]));
  const __nv_bfloat162 hi = __floats2bfloat162_rn(__uint_as_float(y[2]), __uint_as_float(y[3]));
  return make_uint2(*reinterpret_cast<const uint32_t *>(&lo),
                    *reinterpret_cast<const uint32_t *>(&hi));
}

// The pair {s, s} and {off, off} of scale_pairs for a group of exponent emax
// (the fast alignment path: emax >= 8).
__device__ __forceinline__ void operand_scale(int emax, int win_lo, int win_hi, uint64_t &s2,
                                              uint64_t &off2) {
  const bool in = emax >= win_lo && emax <= win_hi;
  const uint32_t s = in ? static_cast<uint32_t>(emax - 6) << 23 : 0x3f800000u;
  const uint32_t off = in ? 0x80000000u | (static_cast<uint32_t>(emax + 17) << 23) : 0xcb000000u;
  s2 = (static_cast<uint64_t>(s) << 32) | s;
  off2 = (static_cast<uint64_t>(off) << 32) | off;
}

// align8 for the contraction with BF16 operands: the eight elements as
// scaled BF16 operand values (scale_pairs; unscaled for a group outside
// [win_lo, win_hi] and for tiny maxima, whose exponent lies below every
// window), zeros for a zero group.
__device__ __forceinline__ uint4 align8_b16(const uint32_t (&packed)[4], uint32_t mx, int emax,
                                            int win_lo, int win_hi) {
  if (emax == kZeroGroup)
    return make_uint4(0, 0, 0, 0);
  if ((mx >> 7) >= 8) {
    const float scale = __uint_as_float(static_cast<uint32_t>(260 - emax) << 23);
    uint32_t r[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      r[2 * e] =
          __float_as_uint(__fmaf_rz(__uint_as_float(packed[e] << 16), scale, 8388608.0f));
      r[2 * e + 1] = __float_as_uint(
          __fmaf_rz(__uint_as_float(packed[e] & 0xffff0000u), scale, 8388608.0f));
    }
    uint64_t s2, off2;
    operand_scale(emax, win_lo, win_hi, s2, off2);
    const uint32_t r0[4] = {r[0], r[1], r[2], r[3]}, r1[4] = {r[4], r[5], r[6], r[7]};
    const uint2 lo = scale_pairs(r0, s2, off2), hi = scale_pairs(r1, s2, off2);
    return make_uint4(lo.x, lo.y, hi.x, hi.y);
  }
  const int shift = 127 - emax;
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t b0 = slow_align(packed[e] & 0xffffu, shift);
    const uint32_t b1 = slow_align(packed[e] >> 16, shift);
    w[e] = static_cast<uint32_t>(f32_to_bf16(static_cast<float>(b0))) |
           (static_cast<uint32_t>(f32_to_bf16(static_cast<float>(b1))) << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// ExpPrealign of four BF16 magnitudes (packed in pairs) against a group of
// maximum mx and exponent emax, as bytes of one word; 0 for a zero group
// (emax == kZeroGroup), which never enters the exact path.
__device__ __forceinline__ uint32_t align4(uint32_t p0, uint32_t p1, uint32_t mx, int emax) {
  const bool zero = emax == kZeroGroup;
  if (zero || (mx >> 7) >= 8) {
    const float scale = __uint_as_float(static_cast<uint32_t>(260 - emax) << 23);
    const uint32_t q0 = __float_as_uint(__fmaf_rz(__uint_as_float(p0 << 16), scale, 8388608.0f));
    const uint32_t q1 =
        __float_as_uint(__fmaf_rz(__uint_as_float(p0 & 0xffff0000u), scale, 8388608.0f));
    const uint32_t q2 = __float_as_uint(__fmaf_rz(__uint_as_float(p1 << 16), scale, 8388608.0f));
    const uint32_t q3 =
        __float_as_uint(__fmaf_rz(__uint_as_float(p1 & 0xffff0000u), scale, 8388608.0f));
    return zero ? 0u : pack_low_bytes(q0, q1, q2, q3);
  }
  const int shift = 127 - emax;
  return slow_align(p0 & 0xffffu, shift) | (slow_align(p0 >> 16, shift) << 8) |
         (slow_align(p1 & 0xffffu, shift) << 16) | (slow_align(p1 >> 16, shift) << 24);
}

template <int kActBranches>
__device__ __forceinline__ void convert8(const float (&v)[8], unsigned mask, int sub,
                                         int32_t *status, uint2 (&out)[2], int (&emax)[2]) {
  uint32_t packed[2][4];
  uint32_t mx[2] = {0, 0};
  uint32_t flags = 0;
  split8<kActBranches>(v, packed, mx, flags);
  // A non-finite element of any thread marks the whole group: fold it into
  // the maximum before the reduction. The negative-input check of a 2-branch
  // layer is per thread.
  if (kActBranches == 2 && flags >= 0x7f7f8000u)
    mx[0] = 0xffffu;
#pragma unroll
  for (int a = 0; a < kActBranches; ++a)
#pragma unroll
    for (int o = 4; o; o >>= 1)
      mx[a] = max(mx[a], __shfl_xor_sync(mask, mx[a], o, kGroupThreads));
  group_exponents<kActBranches>(mx, kActBranches == 2 ? 0u : flags, sub == 0, status, emax);
#pragma unroll
  for (int a = 0; a < kActBranches; ++a)
    out[a] = emax[a] == kZeroGroup ? make_uint2(0, 0) : align8(packed[a], mx[a], emax[a]);
}

// convert8 with the eight elements of each branch as scaled BF16 operand
// values (align8_b16).
template <int kActBranches>
__device__ __forceinline__ void convert8_b16(const float (&v)[8], unsigned mask, int sub,
                                             int32_t *status, int win_lo, int win_hi,
                                             uint4 (&out)[2], int (&emax)[2]) {
  uint32_t packed[2][4];
  uint32_t mx[2] = {0, 0};
  uint32_t flags = 0;
  split8<kActBranches>(v, packed, mx, flags);
  if (kActBranches == 2 && flags >= 0x7f7f8000u)
    mx[0] = 0xffffu;
#pragma unroll
  for (int a = 0; a < kActBranches; ++a)
#pragma unroll
    for (int o = 4; o; o >>= 1)
      mx[a] = max(mx[a], __shfl_xor_sync(mask, mx[a], o, kGroupThreads));
  group_exponents<kActBranches>(mx, kActBranches == 2 ? 0u : flags, sub == 0, status, emax);
#pragma unroll
  for (int a = 0; a < kActBranches; ++a)
    out[a] = align8_b16(packed[a], mx[a], emax[a], win_lo, win_hi);
}

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == CIM22_ACT_RELU)
    return (v > 0.0f || v != v) ? v : 0.0f; // NaN propagates, as torch.relu
  if (act == CIM22_ACT_GELU)
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  return v;
}

// Exact restore of one tile value outside the fast exponent window (subnormal
// or overflowing results), out of line so the fast path is not predicated
// through it. Returns the updated f32 branch sum.
__device__ __noinline__ float slow_tile_add(float acc, int p, int ew, int ex, int32_t *status) {
  if (ex == kZeroGroup)
    return acc;
  const uint16_t tile = signsplit_tile(static_cast<uint32_t>(p), ew, ex);
  if (tile == kBF16Inf)
    atomicOr(status, CIM22_STATUS_TILE_OVERFLOW);
  return __fadd_rn(acc, bf16_to_f32(tile));
}

// Branch a of two signed BF16 halves, sign cleared: for a 2-branch layer the
// value itself (its sign is flagged separately); for a 4-branch layer xp =
// max(v, 0) (a = 0) or xn = max(-v, 0) (a = 1).
template <int kActBranches>
__device__ __forceinline__ uint32_t branch_pair(uint32_t pair, int a) {
  if (kActBranches == 1)
    return pair & 0x7fff7fffu;
  const uint32_t neg = ((pair >> 15) & 0x00010001u) * 0xffffu; // halves with the sign set
  return (a == 0 ? pair & ~neg : pair & neg) & 0x7fff7fffu;
}

// The rest of one (column m, K tile t) group once its 64 signed BF16 pairs
// and raw maximum are known: branch maxima, the non-finite and
// negative-input flags, ExpPrealign, the group exponent and the prepared
// group of each branch - 64 aligned int8 mantissas (four 16-byte stores), or
// with kB16 the 64 scaled BF16 operand values (eight 16-byte stores; scaled
// for groups whose exponent lies in [win_lo, win_hi], unscaled otherwise).
// kStore: where the prepared group goes.
//   kStoreGlobal  16-byte stores into A (the workspace), the exponent into ex
//   kStoreStaged  the warp's 32 columns (consecutive, all in the call) are
//                 written into the warp's shared-memory tile `stage` (per
//                 branch 32 rows of 64 or 128 bytes, 16-byte chunks swizzled
//                 as `omap` describes) and leave with one TMA store per
//                 branch, so that whole lines reach global memory
//   kStoreOperand the same swizzled rows, left in shared memory as the warp's
//                 32 rows of a contraction's 128-row operand tile (1-branch
//                 BF16 operands, 128-byte swizzle); the exponent goes to
//                 ex[m] (a shared-memory ring slot). The caller fences the
//                 writes for the tensor cores (async proxy) and signals them.
constexpr int kStoreGlobal = 0, kStoreStaged = 1, kStoreOperand = 2;

template <int kActBranches, bool kB16 = false, int kStore = kStoreGlobal>
__device__ __forceinline__ void finish_group(const uint32_t (&signed_pairs)[32],
                                             uint32_t raw_max, int32_t *status,
                                             int8_t *__restrict__ A, int32_t *__restrict__ ex,
                                             int m_pad, int k_pad, int T, int t, int m,
                                             int kbeg, int win_lo = 1, int win_hi = 0,
                                             uint8_t *stage = nullptr,
                                             const CUtensorMap *omap = nullptr) {
  constexpr bool kStaged = kStore == kStoreStaged;
  constexpr bool kShared = kStore != kStoreGlobal;
  static_assert(kStore != kStoreOperand || (kActBranches == 1 && kB16),
                "operand tiles hold one branch of BF16 operand values");
  constexpr int kRowBytes = kB16 ? 128 : 64;
  const int lane = static_cast<int>(threadIdx.x & 31);
  if constexpr (kStaged) {
    // The tile's previous stores must have read it before it is rewritten.
    if (lane == 0)
      bulk_wait_read();
    __syncwarp();
  }
  uint32_t mx[2] = {0, 0};
  // A 2-branch layer whose BF16 inputs carry no sign bit (the usual case:
  // the layer reads a ReLU output) has the raw maximum as its maximum; a -0
  // or a negative input takes the loop over the cleared magnitudes.
  const uint32_t raw_half = max(raw_max & 0xffffu, raw_max >> 16);
  if (kActBranches == 1 && raw_half < 0x8000u) {
    mx[0] = raw_half;
  } else {
#pragma unroll
    for (int a = 0; a < kActBranches; ++a) {
      uint32_t m2 = 0;
#pragma unroll
      for (int e = 0; e < 32; ++e)
        m2 = __vmaxu2(m2, branch_pair<kActBranches>(signed_pairs[e], a));
      mx[a] = max(m2 & 0xffffu, m2 >> 16);
    }
  }
  // Non-finite groups: BF16 exponent 0xff in a branch maximum (the two
  // branches of a 4-branch layer hold every magnitude between them, NaNs
  // included). A 2-branch layer flags a negative nonzero BF16 input, the
  // reference's sign-split rejection (-0 is cleared to +0).
  const bool nonfinite = max(mx[0], mx[1]) >= 0x7f80u;
  if (nonfinite)
    atomicOr(status, CIM22_STATUS_INPUT_NOT_FINITE);
  else if (kActBranches == 1 && raw_half > 0x8000u)
    atomicOr(status, CIM22_STATUS_NEGATIVE_INPUT);
  // Pass 2: align and store.
  constexpr int kWords = kB16 ? 32 : 16;
#pragma unroll
  for (int a = 0; a < kActBranches; ++a) {
    const bool zero = mx[a] == 0 || nonfinite;
    const int emax = zero ? kZeroGroup : effective_exponent(static_cast<uint16_t>(mx[a]));
    uint32_t out[kWords];
    if (zero) {
#pragma unroll
      for (int q = 0; q < kWords; ++q)
        out[q] = 0;
    } else if ((mx[a] >> 7) >= 8) {
      const float scale = __uint_as_float(static_cast<uint32_t>(260 - emax) << 23);
      const uint64_t scale2 = (static_cast<uint64_t>(__float_as_uint(scale)) << 32) |
                              __float_as_uint(scale);
      const uint64_t magic2 = 0x4b0000004b000000ull; // 2^23 in both halves
      uint64_t s2 = 0, off2 = 0;
      if (kB16)
        operand_scale(emax, win_lo, win_hi, s2, off2);
      // A 2-branch layer aligns the raw halves: -0 aligns to 0 as +0 does,
      // and a negative nonzero input has failed the call already.
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        uint32_t r[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t pk = kActBranches == 1
                                  ? signed_pairs[2 * q + h]
                                  : branch_pair<kActBranches>(signed_pairs[2 * q + h], a);
          // Both halves in one packed f32x2 fma (each half rounds toward zero
          // as __fmaf_rz).
          asm("{\n\t.reg .b64 a, d;\n\tmov.b64 a, {%2, %3};\n\t"
              "fma.rz.f32x2 d, a, %4, %5;\n\tmov.b64 {%0, %1}, d;\n\t}"
              : "=r"(r[2 * h]), "=r"(r[2 * h + 1])
              : "r"(pk << 16), "r"(pk & 0xffff0000u), "l"(scale2), "l"(magic2));
        }
        if constexpr (kB16) {
          const uint2 w = scale_pairs(r, s2, off2);
          out[2 * q] = w.x;
          out[2 * q + 1] = w.y;
        } else {
          out[q] = pack_low_bytes(r[0], r[1], r[2], r[3]);
        }
      }
    } else {
      // Tiny maxima (exponent < 8): exact alignment; with kB16 the unscaled
      // mantissas (such a group is outside every window).
      const int shift = 127 - emax;
      for (int q = 0; q < 16; ++q) {
        uint32_t bytes[4];
        for (int h = 0; h < 4; ++h)
          bytes[h] = slow_align((branch_pair<kActBranches>(signed_pairs[2 * q + h / 2], a) >>
                                 (16 * (h & 1))) & 0xffffu,
                                shift);
        if constexpr (kB16) {
          out[2 * q] = static_cast<uint32_t>(f32_to_bf16(static_cast<float>(bytes[0]))) |
                       (static_cast<uint32_t>(f32_to_bf16(static_cast<float>(bytes[1]))) << 16);
          out[2 * q + 1] =
              static_cast<uint32_t>(f32_to_bf16(static_cast<float>(bytes[2]))) |
              (static_cast<uint32_t>(f32_to_bf16(static_cast<float>(bytes[3]))) << 16);
        } else {
          out[q] = bytes[0] | (bytes[1] << 8) | (bytes[2] << 16) | (bytes[3] << 24);
        }
      }
    }
    if constexpr (kShared) {
      // Row `lane` of the branch's tile; chunk q at q ^ (the swizzle's row
      // bits): lane & 7 for 128-byte rows, (lane >> 1) & 3 for 64-byte rows.
      uint8_t *row = stage + (a * 32 + lane) * kRowBytes;
      const int swz = kB16 ? (lane & 7) : ((lane >> 1) & 3);
#pragma unroll
      for (int q = 0; q < kWords / 4; ++q)
        *reinterpret_cast<uint4 *>(row + ((q ^ swz) << 4)) =
            make_uint4(out[4 * q], out[4 * q + 1], out[4 * q + 2], out[4 * q + 3]);
    } else {
      constexpr int kElemBytes = kB16 ? 2 : 1;
      uint4 *dst = reinterpret_cast<uint4 *>(
          A + ((static_cast<int64_t>(a) * m_pad + m) * k_pad + kbeg) * kElemBytes);
#pragma unroll
      for (int q = 0; q < kWords / 4; ++q)
        dst[q] = make_uint4(out[4 * q], out[4 * q + 1], out[4 * q + 2], out[4 * q + 3]);
    }
    if constexpr (kStore == kStoreOperand)
      ex[m] = emax;
    else
      ex[(static_cast<int64_t>(a) * T + t) * m_pad + m] = emax;
  }
  if constexpr (kStaged) {
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
#pragma unroll
      for (int a = 0; a < kActBranches; ++a)
        tma_store_2d(omap, stage + a * 32 * kRowBytes, kbeg, a * m_pad + (m - lane));
      bulk_commit();
    }
  }
}

} // namespace
} // namespace cim
