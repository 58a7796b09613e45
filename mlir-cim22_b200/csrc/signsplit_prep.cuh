// signsplit_prep.cuh - device routines shared by the sign-split layer
// kernels (layers.cu) and the fused layer-chain kernel (chain.cu): the
// 8-thread group preparation of activations (split, RNE to BF16, group
// maximum, ExpPrealign), the exact slow restore of one tile and the
// epilogue activations.
#pragma once

#include "cim_internal.h"
#include "cim_numeric.cuh"

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

} // namespace
} // namespace cim
