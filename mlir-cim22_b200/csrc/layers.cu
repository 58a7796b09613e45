// layers.cu - CIM layers over device memory: weight preparation, the
// activation prepare/im2col kernel and the CUDA-core contraction kernels.
//
// A CIM layer computes, for every column m and output lane n,
//   BF16 sign-split: y = ((pp - pn) - np) + nn (+ bias, activation), where
//     each branch is the f32 sum over 64-element K tiles, in tile order, of
//     the restored tile values RNE_bf16(Q(p) * 2^(Ew + Ex - 266)), rounded to
//     BF16 once more when there is more than one tile
//     (lib/Conversion/LinalgToCIM/Passes.cpp:828-857,2304-2420 with
//     lib/Execution/BF16Compensation.cpp:84-164);
//   INT8: y = wrapping int32 sum of the signed-i21 tile partials
//     (Passes.cpp:1054-1059, lib/Execution/CIMSoftwareRunner.cpp:406-420).
//
// Data layout in HBM (row-major, K innermost):
//   prepared activations  int8 A[branch][m_pad][k_pad], int32 Ex[branch][T][m_pad]
//   resident weights      int8 B[branch][n_pad][k_pad], int32 Ew[branch][T][n_pad]
//   outputs               f32 / int32 y[m][n]
#include "cim_internal.h"
#include "cim_numeric.cuh"

#include <cuda_bf16.h>
#include "gemm_tc.h"

#include <algorithm>
#include <climits>
#include <cmath>
#include <vector>

namespace cim {
namespace {

constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------------------
// Gather of the K x columns operand (linear rows or conv im2col), with 32-bit
// index arithmetic (checked on the host) and the K decomposition hoisted out
// of the column loop.

// Division by an invariant divisor as a multiply-high and shift (Granlund and
// Montgomery, "Division by invariant integers using multiplication", 1994):
// q = (umulhi(n, mul) + n) >> shift for 0 <= n < 2^31, with
// shift = ceil(log2 d) and mul = floor(2^32 (2^shift - d) / d) + 1.
struct FastDiv {
  uint32_t d, mul, shift;
};

FastDiv make_fastdiv(uint32_t d) {
  FastDiv f{d, 0, 0};
  uint32_t l = 0;
  while ((uint64_t{1} << l) < d)
    ++l;
  f.shift = l;
  f.mul = static_cast<uint32_t>(((uint64_t{1} << 32) * ((uint64_t{1} << l) - d)) / d + 1);
  return f;
}

__device__ __forceinline__ int fdiv(int n, const FastDiv &f) {
  return static_cast<int>((__umulhi(static_cast<uint32_t>(n), f.mul) + static_cast<uint32_t>(n)) >> f.shift);
}

struct Gather32 {
  FastDiv div_ohw, div_ow, div_khw, div_kw;
  int kind, C, H, W, KH, KW, SH, SW, PH, PW, OH, OW;
  int PK, PS, SRC_H, SRC_W; // fused max pool (NHWC), PK == 0 when absent
  int M, K;
  int pair_rows; // rows layout: 2 when K % 4 == 0 and x is 16-byte aligned (float4 loads)
};

// One element of image n at (ih, iw, c); `img` already points at image n.
// With a fused max pool it reads the max over the pool window of the
// pre-pool image (NaN propagates like torch.max_pool2d).
__device__ __forceinline__ float image_load(const float *__restrict__ img,
                                            const Gather32 &g, int ih, int iw,
                                            int c) {
  if (g.kind == CIM22_GATHER_CONV_NCHW)
    return img[(c * g.H + ih) * g.W + iw];
  if (g.PK == 0)
    return img[(ih * g.W + iw) * g.C + c];
  float m = 0.0f;
  bool any = false;
  for (int dy = 0; dy < g.PK; ++dy)
    for (int dx = 0; dx < g.PK; ++dx) {
      const float v = img[((ih * g.PS + dy) * g.SRC_W + iw * g.PS + dx) * g.C + c];
      if (!any || v > m || v != v) {
        m = v;
        any = true;
      }
    }
  return m;
}

// Sign-split preparation of a 64-element group (prepareBF16Input,
// BF16Compensation.cpp:92-118). Fast path: when the group maximum is a normal
// BF16 with biased exponent Ex >= 8, scaling by 2^(127-Ex) is exact for every
// element that stays normal, and ExpPrealign then yields (0x80 | m) >>
// (Ex - e + 1) for a gap Ex - e < 7; elements that would turn subnormal (or
// are subnormal) have gaps >= 7 and align to 0. Other groups take the exact
// RNE scaling of bf16_scalbn. The scaled maximum lies in [1, 2), so the
// prealign exponent is always 127.
__device__ __forceinline__ int8_t fast_align(uint32_t p, int emax) {
  const int e = static_cast<int>(p >> 7);
  const int gap = emax - e;
  return (e >= 1 && gap < 7)
             ? static_cast<int8_t>((0x80u | (p & 0x7fu)) >> (gap + 1))
             : int8_t{0};
}

// Exact path for groups whose maximum is tiny (exponent < 8): RNE scaling of
// the element, then ExpPrealign at exponent 127. Out of line so the fast path
// is not predicated through it.
__device__ __noinline__ uint32_t slow_align(uint32_t p, int shift) {
  return static_cast<uint8_t>(prealign_element(bf16_scalbn(static_cast<uint16_t>(p), shift), 127));
}

// Activation split (Passes.cpp:2379-2399): xp = (x < 0 ? 0 : x) then
// (x == 0 ? +0 : xp), xn = (x < 0 ? -x : 0), each rounded to BF16 (RNE); a
// 2-branch layer applies only the (x == 0 ? +0 : x) select.
template <int kActBranches>
__device__ __forceinline__ void split_bits(float v, uint32_t &bp, uint32_t &bn) {
  const float zero = 0.0f;
  float p = v, q = zero;
  if (kActBranches == 2) {
    const bool negative = v < zero;
    p = negative ? zero : v;
    q = negative ? -v : zero;
  }
  p = (v == zero) ? zero : p; // -0 becomes +0
  bp = f32_to_bf16(p);
  bn = f32_to_bf16(q);
}

// Element source of one group: consecutive K indices of one column, with the
// conv (c, i, j) decomposition stepped incrementally.
struct GroupCursor {
  const float *base; // rows: the column's row; conv: image n
  int ih0, iw0;      // conv window origin (oh * SH - PH, ow * SW - PW)
  int c, i, j;       // conv position of the current k
  int k;
  bool column_valid;
};

__device__ __forceinline__ GroupCursor open_group(const float *__restrict__ x, const Gather32 &g,
                                                  int m, int kbeg) {
  GroupCursor cur{};
  cur.k = kbeg;
  cur.column_valid = m < g.M;
  if (g.kind == CIM22_GATHER_ROWS) {
    cur.base = x + static_cast<int64_t>(m) * g.K;
  } else if (cur.column_valid) {
    const int n = fdiv(m, g.div_ohw);
    const int r = m - n * g.OH * g.OW;
    const int oh = fdiv(r, g.div_ow);
    const int ow = r - oh * g.OW;
    const int64_t image = g.kind == CIM22_GATHER_CONV_NCHW || g.PK == 0
                              ? static_cast<int64_t>(g.C) * g.H * g.W
                              : static_cast<int64_t>(g.C) * g.SRC_H * g.SRC_W;
    cur.base = x + n * image;
    cur.ih0 = oh * g.SH - g.PH;
    cur.iw0 = ow * g.SW - g.PW;
    cur.c = fdiv(kbeg, g.div_khw);
    const int rk = kbeg - cur.c * g.KH * g.KW;
    cur.i = fdiv(rk, g.div_kw);
    cur.j = rk - cur.i * g.KW;
  }
  return cur;
}

__device__ __forceinline__ float next_value(const float *__restrict__ x, const Gather32 &g,
                                            GroupCursor &cur) {
  float v = 0.0f;
  if (cur.column_valid && cur.k < g.K) {
    if (g.kind == CIM22_GATHER_ROWS) {
      v = cur.base[cur.k];
    } else {
      const int ih = cur.ih0 + cur.i;
      const int iw = cur.iw0 + cur.j;
      if (static_cast<unsigned>(ih) < static_cast<unsigned>(g.H) &&
          static_cast<unsigned>(iw) < static_cast<unsigned>(g.W))
        v = image_load(cur.base, g, ih, iw, cur.c);
      if (++cur.j == g.KW) {
        cur.j = 0;
        if (++cur.i == g.KH) {
          cur.i = 0;
          ++cur.c;
        }
      }
    }
  }
  ++cur.k;
  return v;
}

// Prepare: eight threads per (column m, K tile t) group, eight consecutive
// elements each; groups are ordered t-fastest so a warp's four groups read
// one contiguous stretch of a row. The group maximum of each branch is an
// xor-shuffle reduction within the 8-lane subgroup; each thread then writes
// its 8 aligned bytes per branch. Padding columns (m >= M) and padding K are
// zero; an all-zero group records the exponent kZeroGroup.
constexpr int kGroupThreads = 8;

template <int kActBranches>
__global__ void __launch_bounds__(256)
    prepare_kernel(const float *__restrict__ x, Gather32 g, FastDiv div_t, int m_pad,
                   int k_pad, int8_t *__restrict__ A, int32_t *__restrict__ ex,
                   int32_t *status) {
  const int T = static_cast<int>(div_t.d);
  const int group = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) / kGroupThreads);
  const int sub = static_cast<int>(threadIdx.x % kGroupThreads);
  if (group >= m_pad * T)
    return; // uniform per 8-lane subgroup (blockDim is a multiple of 8)
  const unsigned mask = 0xffu << (threadIdx.x & 24);
  const int m = fdiv(group, div_t);
  const int t = group - m * T;
  const int kbeg = t * kTileK + sub * 8;
  float v[8];
  if (kbeg >= g.K || m >= g.M) {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      v[e] = 0.0f; // K or column padding
  } else if (g.kind == CIM22_GATHER_ROWS && g.pair_rows == 2 && kbeg + 8 <= g.K) {
    const float4 *src = reinterpret_cast<const float4 *>(x + static_cast<int64_t>(m) * g.K + kbeg);
    const float4 lo = src[0], hi = src[1];
    v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
    v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
  } else {
    GroupCursor cur = open_group(x, g, m, kbeg);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      v[e] = next_value(x, g, cur);
  }
  // Split and round: xp = max(x, 0), xn = max(-x, 0) equal the reference's
  // selects for every non-NaN x up to the sign of zero, which the preparation
  // clears anyway (BF16Compensation.cpp:97); NaN, infinity and finite values
  // that round to BF16 infinity (|x| >= 0x1.fep127) are caught on x itself.
  // cvt.rn.bf16x2.f32 rounds to nearest even, as arith.truncf does.
  uint32_t bits[2][8];
  uint32_t mx[2] = {0, 0};
  bool nonfinite = false, negative = false;
  uint32_t packed[2][4];
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    float p0 = v[e], p1 = v[e + 1], q0 = 0.0f, q1 = 0.0f;
    nonfinite |= !(fabsf(p0) < 3.3961548e38f) || !(fabsf(p1) < 3.3961548e38f);
    if (kActBranches == 2) {
      q0 = fmaxf(-p0, 0.0f);
      q1 = fmaxf(-p1, 0.0f);
      p0 = fmaxf(p0, 0.0f);
      p1 = fmaxf(p1, 0.0f);
    } else {
      negative |= p0 < 0.0f || p1 < 0.0f;
    }
    const __nv_bfloat162 hp = __floats2bfloat162_rn(p0, p1);
    packed[0][e / 2] = *reinterpret_cast<const uint32_t *>(&hp) & 0x7fff7fffu;
    if (kActBranches == 2) {
      const __nv_bfloat162 hn = __floats2bfloat162_rn(q0, q1);
      packed[1][e / 2] = *reinterpret_cast<const uint32_t *>(&hn) & 0x7fff7fffu;
    }
  }
#pragma unroll
  for (int a = 0; a < kActBranches; ++a) {
    const uint32_t m2 = __vmaxu2(__vmaxu2(packed[a][0], packed[a][1]),
                                 __vmaxu2(packed[a][2], packed[a][3]));
    mx[a] = max(m2 & 0xffffu, m2 >> 16);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      bits[a][e] = (packed[a][e / 2] >> (16 * (e & 1))) & 0xffffu;
  }
#pragma unroll
  for (int a = 0; a < kActBranches; ++a)
#pragma unroll
    for (int o = 4; o; o >>= 1)
      mx[a] = max(mx[a], __shfl_xor_sync(mask, mx[a], o, kGroupThreads));
  nonfinite = __any_sync(mask, nonfinite);
  if (sub == 0 && nonfinite)
    atomicOr(status, CIM22_STATUS_INPUT_NOT_FINITE);
  if (negative && !nonfinite)
    atomicOr(status, CIM22_STATUS_NEGATIVE_INPUT);
#pragma unroll
  for (int a = 0; a < kActBranches; ++a) {
    const bool zero = mx[a] == 0 || nonfinite;
    const int emax = zero ? kZeroGroup : effective_exponent(static_cast<uint16_t>(mx[a]));
    const bool fast = static_cast<int>(mx[a] >> 7) >= 8;
    const int shift = 127 - emax;
    uint32_t lo = 0, hi = 0;
    if (!zero) {
      if (fast) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          lo |= static_cast<uint32_t>(static_cast<uint8_t>(fast_align(bits[a][e], emax))) << (8 * e);
          hi |= static_cast<uint32_t>(static_cast<uint8_t>(fast_align(bits[a][e + 4], emax)))
                << (8 * e);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          lo |= slow_align(bits[a][e], shift) << (8 * e);
          hi |= slow_align(bits[a][e + 4], shift) << (8 * e);
        }
      }
    }
    *reinterpret_cast<uint2 *>(A + (static_cast<int64_t>(a) * m_pad + m) * k_pad + kbeg) =
        make_uint2(lo, hi);
    if (sub == 0)
      ex[(static_cast<int64_t>(a) * T + t) * m_pad + m] = emax;
  }
}


__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == CIM22_ACT_RELU)
    return v > 0.0f ? v : 0.0f;
  if (act == CIM22_ACT_GELU)
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  return v;
}

// ---------------------------------------------------------------------------
// Sign-split contraction on CUDA cores (dp4a). CTA tile kBM columns x kBN
// lanes, all branches; thread (tr, tc) owns columns tr + i * kTR (i < kRM)
// and lanes 4tc .. 4tc + 3.
constexpr int kRowStride = 80;

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

template <int kActBranches, int kTC, int kRM>
__global__ void __launch_bounds__(256)
    signsplit_simt_kernel(const int8_t *__restrict__ A,
                          const int32_t *__restrict__ exA, int64_t m_pad,
                          const int8_t *__restrict__ B,
                          const int32_t *__restrict__ exB, int64_t n_pad,
                          int64_t k_pad, int T, int64_t M, int64_t N,
                          const float *__restrict__ bias, int act,
                          float *__restrict__ y, int32_t *status) {
  constexpr int kBN = 4 * kTC, kTR = 256 / kTC, kBM = kTR * kRM;
  __shared__ __align__(16) int8_t As[kActBranches][kBM][kRowStride];
  __shared__ __align__(16) int8_t Bs[2][kBN][kRowStride];
  __shared__ int sExA[kActBranches][kBM];
  __shared__ int sExB[2][kBN];
  __shared__ float sSw[2][kBN];
  __shared__ int sFast;
  __shared__ int sLive[kActBranches];
  const int tid = threadIdx.x;
  const int tr = tid / kTC, tc = tid % kTC;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kBM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * kBN;
  float acc[kActBranches][2][kRM][4];
#pragma unroll
  for (int a = 0; a < kActBranches; ++a)
#pragma unroll
    for (int w = 0; w < 2; ++w)
#pragma unroll
      for (int r = 0; r < kRM; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          acc[a][w][r][c] = 0.0f;

  for (int t = 0; t < T; ++t) {
    for (int i = tid; i < 2 * kBN * 4; i += 256) {
      const int w = i / (kBN * 4), r = (i >> 2) % kBN, c = i & 3;
      *reinterpret_cast<int4 *>(&Bs[w][r][c * 16]) = *reinterpret_cast<const int4 *>(
          B + (static_cast<int64_t>(w) * n_pad + n0 + r) * k_pad +
          static_cast<int64_t>(t) * kTileK + c * 16);
    }
    for (int i = tid; i < kActBranches * kBM; i += 256)
      sExA[i / kBM][i % kBM] =
          exA[(static_cast<int64_t>(i / kBM) * T + t) * m_pad + m0 + i % kBM];
    for (int i = tid; i < 2 * kBN; i += 256) {
      const int e = exB[(static_cast<int64_t>(i / kBN) * T + t) * n_pad + n0 + i % kBN];
      sExB[i / kBN][i % kBN] = e;
      sSw[i / kBN][i % kBN] = exp2i(e - 133);
    }
    __syncthreads();
    if (tid < 32) {
      int mnA = INT_MAX, mxA = INT_MIN, mnB = INT_MAX, mxB = INT_MIN;
      int live[kActBranches];
#pragma unroll
      for (int a = 0; a < kActBranches; ++a)
        live[a] = 0;
      for (int i = tid; i < kActBranches * kBM; i += 32) {
        const int v = sExA[i / kBM][i % kBM];
        if (v == kZeroGroup)
          continue;
        live[i / kBM] = 1;
        mnA = min(mnA, v);
        mxA = max(mxA, v);
      }
#pragma unroll
      for (int a = 0; a < kActBranches; ++a) {
        live[a] = __any_sync(kFull, live[a]);
        if (tid == 0)
          sLive[a] = live[a];
      }
      for (int i = tid; i < 2 * kBN; i += 32) {
        const int v = sExB[i / kBN][i % kBN];
        mnB = min(mnB, v);
        mxB = max(mxB, v);
      }
      mnA = __reduce_min_sync(kFull, mnA);
      mxA = __reduce_max_sync(kFull, mxA);
      mnB = __reduce_min_sync(kFull, mnB);
      mxB = __reduce_max_sync(kFull, mxB);
      if (tid == 0)
        sFast = mxA == INT_MIN || ((mnA + mnB >= 140) && (mxA + mxB <= 374) && (mxA <= 240));
    }
    __syncthreads();
    const bool fast = sFast != 0;
    bool live[kActBranches];
#pragma unroll
    for (int a = 0; a < kActBranches; ++a)
      live[a] = sLive[a] != 0;
    // Activation tiles of live branches only (an all-zero branch is skipped).
    for (int i = tid; i < kActBranches * kBM * 4; i += 256) {
      const int a = i / (kBM * 4), r = (i >> 2) % kBM, c = i & 3;
      if (live[a])
        *reinterpret_cast<int4 *>(&As[a][r][c * 16]) = *reinterpret_cast<const int4 *>(
            A + (static_cast<int64_t>(a) * m_pad + m0 + r) * k_pad +
            static_cast<int64_t>(t) * kTileK + c * 16);
    }
    __syncthreads();
    int p[kActBranches][2][kRM][4];
#pragma unroll
    for (int a = 0; a < kActBranches; ++a)
#pragma unroll
      for (int w = 0; w < 2; ++w)
#pragma unroll
        for (int r = 0; r < kRM; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            p[a][w][r][c] = 0;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      int4 av[kActBranches][kRM], bv[2][4];
#pragma unroll
      for (int a = 0; a < kActBranches; ++a)
#pragma unroll
        for (int r = 0; r < kRM; ++r)
          av[a][r] = *reinterpret_cast<const int4 *>(&As[a][tr + kTR * r][kk * 16]);
#pragma unroll
      for (int w = 0; w < 2; ++w)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          bv[w][c] = *reinterpret_cast<const int4 *>(&Bs[w][tc * 4 + c][kk * 16]);
#pragma unroll
      for (int a = 0; a < kActBranches; ++a)
        if (live[a])
#pragma unroll
        for (int w = 0; w < 2; ++w)
#pragma unroll
          for (int r = 0; r < kRM; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              int s = p[a][w][r][c];
              s = __dp4a(av[a][r].x, bv[w][c].x, s);
              s = __dp4a(av[a][r].y, bv[w][c].y, s);
              s = __dp4a(av[a][r].z, bv[w][c].z, s);
              s = __dp4a(av[a][r].w, bv[w][c].w, s);
              p[a][w][r][c] = s;
            }
    }
#pragma unroll
    for (int a = 0; a < kActBranches; ++a) {
      if (!live[a])
        continue; // every group of this branch is zero: its tiles add +0
      if (fast) {
#pragma unroll
        for (int r = 0; r < kRM; ++r) {
          const int exr = sExA[a][tr + kTR * r];
          const float sx = exr == kZeroGroup ? 1.0f : exp2i(exr - 133);
#pragma unroll
          for (int w = 0; w < 2; ++w)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const float q = __fmul_rn(trunc8f(p[a][w][r][c]), sx);
              acc[a][w][r][c] = fmaf(q, sSw[w][tc * 4 + c], acc[a][w][r][c]);
            }
        }
      } else {
#pragma unroll
        for (int r = 0; r < kRM; ++r) {
          const int exr = sExA[a][tr + kTR * r];
#pragma unroll
          for (int w = 0; w < 2; ++w)
#pragma unroll
            for (int c = 0; c < 4; ++c)
              acc[a][w][r][c] = slow_tile_add(acc[a][w][r][c], p[a][w][r][c],
                                              sExB[w][tc * 4 + c], exr, status);
        }
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int r = 0; r < kRM; ++r) {
    const int64_t row = m0 + tr + kTR * r;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int64_t lane = n0 + tc * 4 + c;
      float br[kActBranches][2];
#pragma unroll
      for (int a = 0; a < kActBranches; ++a)
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const float v = acc[a][w][r][c];
          br[a][w] = T > 1 ? bf16_to_f32(f32_to_bf16(v)) : v;
        }
      float out = __fsub_rn(br[0][0], br[0][1]);
      if (kActBranches == 2) {
        out = __fsub_rn(out, br[1][0]);
        out = __fadd_rn(out, br[1][1]);
      }
      if (bias != nullptr && lane < N)
        out = __fadd_rn(out, bias[lane]);
      out = apply_act(out, act);
      if (row < M && lane < N)
        y[row * N + lane] = out;
    }
  }
}

// Tile shape per layer: 8 or 16-lane tiles for layers of at most 8 or 16
// lanes, 32 otherwise; 2 column rows per thread when that still gives every
// SM two CTAs.
template <int kAB>
void launch_signsplit_simt(const int8_t *A, const int32_t *exA, int64_t m_pad,
                           const int8_t *B, const int32_t *exB, int64_t n_pad,
                           int64_t k_pad, int T, int64_t M, int64_t N,
                           const float *bias, int act, float *y, int32_t *status,
                           cudaStream_t s) {
  const int64_t target = 2 * 148;
  if (N <= 8) {
    signsplit_simt_kernel<kAB, 2, 1><<<dim3(static_cast<unsigned>(m_pad / 128), 1), 256, 0, s>>>(
        A, exA, m_pad, B, exB, n_pad, k_pad, T, M, N, bias, act, y, status);
  } else if (N <= 16) {
    const unsigned ny = static_cast<unsigned>((N + 15) / 16);
    if ((m_pad / 128) * ny >= target)
      signsplit_simt_kernel<kAB, 4, 2><<<dim3(static_cast<unsigned>(m_pad / 128), ny), 256, 0, s>>>(
          A, exA, m_pad, B, exB, n_pad, k_pad, T, M, N, bias, act, y, status);
    else
      signsplit_simt_kernel<kAB, 4, 1><<<dim3(static_cast<unsigned>(m_pad / 64), ny), 256, 0, s>>>(
          A, exA, m_pad, B, exB, n_pad, k_pad, T, M, N, bias, act, y, status);
  } else {
    const unsigned ny = static_cast<unsigned>((N + 31) / 32);
    if ((m_pad / 64) * ny >= target)
      signsplit_simt_kernel<kAB, 8, 2><<<dim3(static_cast<unsigned>(m_pad / 64), ny), 256, 0, s>>>(
          A, exA, m_pad, B, exB, n_pad, k_pad, T, M, N, bias, act, y, status);
    else
      signsplit_simt_kernel<kAB, 8, 1><<<dim3(static_cast<unsigned>(m_pad / 32), ny), 256, 0, s>>>(
          A, exA, m_pad, B, exB, n_pad, k_pad, T, M, N, bias, act, y, status);
  }
}

// ---------------------------------------------------------------------------
// INT8 on CUDA cores: CTA tile 64 x 64, thread owns 4 columns x 4 lanes.
__global__ void pad_int8_kernel(const int8_t *__restrict__ x, int64_t M,
                                int64_t K, int64_t m_pad, int64_t k_pad,
                                int8_t *__restrict__ out) {
  const int64_t total = m_pad * k_pad;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < total; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / k_pad, k = i - m * k_pad;
    out[i] = (m < M && k < K) ? x[m * K + k] : int8_t{0};
  }
}

__global__ void __launch_bounds__(256)
    int8_simt_kernel(const int8_t *__restrict__ A, const int8_t *__restrict__ B,
                     int64_t k_pad, int T, int64_t M, int64_t N,
                     int checked, int32_t *__restrict__ y, int32_t *status) {
  __shared__ __align__(16) int8_t As[64][kRowStride];
  __shared__ __align__(16) int8_t Bs[64][kRowStride];
  const int tid = threadIdx.x;
  const int tr = tid >> 4, tc = tid & 15;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * 64;
  uint32_t acc[4][4] = {};
  bool overflow = false;
  for (int t = 0; t < T; ++t) {
    {
      const int r = tid >> 2, c = tid & 3;
      *reinterpret_cast<int4 *>(&As[r][c * 16]) = *reinterpret_cast<const int4 *>(
          A + (m0 + r) * k_pad + static_cast<int64_t>(t) * kTileK + c * 16);
      *reinterpret_cast<int4 *>(&Bs[r][c * 16]) = *reinterpret_cast<const int4 *>(
          B + (n0 + r) * k_pad + static_cast<int64_t>(t) * kTileK + c * 16);
    }
    __syncthreads();
    int p[4][4] = {};
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      int4 av[4], bv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
        av[r] = *reinterpret_cast<const int4 *>(&As[tr + 16 * r][kk * 16]);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        bv[c] = *reinterpret_cast<const int4 *>(&Bs[tc * 4 + c][kk * 16]);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          int s = p[r][c];
          s = __dp4a(av[r].x, bv[c].x, s);
          s = __dp4a(av[r].y, bv[c].y, s);
          s = __dp4a(av[r].z, bv[c].z, s);
          s = __dp4a(av[r].w, bv[c].w, s);
          p[r][c] = s;
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (checked && (p[r][c] < -(1 << 20) || p[r][c] >= (1 << 20)))
          overflow = true;
        acc[r][c] += static_cast<uint32_t>(p[r][c]);
      }
    __syncthreads();
  }
  if (overflow)
    atomicOr(status, CIM22_STATUS_I21_RANGE);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t row = m0 + tr + 16 * r;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int64_t lane = n0 + tc * 4 + c;
      if (row < M && lane < N)
        y[row * N + lane] = static_cast<int32_t>(acc[r][c]);
    }
  }
}

bool check_gather(const cim22_gather &g, int64_t m, int64_t k) {
  if (m >= (int64_t{1} << 31) - kColumnPad || k >= (int64_t{1} << 30))
    return false;
  if (g.kind == CIM22_GATHER_ROWS)
    return m * k < (int64_t{1} << 40);
  if (g.pool_kernel < 0 || (g.pool_kernel > 0 &&
      (g.kind != CIM22_GATHER_CONV_NHWC || g.pool_stride <= 0 ||
       (g.pool_src_h - g.pool_kernel) / g.pool_stride + 1 != g.height ||
       (g.pool_src_w - g.pool_kernel) / g.pool_stride + 1 != g.width ||
       g.pool_src_h < g.pool_kernel || g.pool_src_w < g.pool_kernel)))
    return false;
  if (g.kind != CIM22_GATHER_CONV_NCHW && g.kind != CIM22_GATHER_CONV_NHWC)
    return false;
  if (g.batch <= 0 || g.channels <= 0 || g.height <= 0 || g.width <= 0 ||
      g.kernel_h <= 0 || g.kernel_w <= 0 || g.stride_h <= 0 || g.stride_w <= 0 ||
      g.pad_h < 0 || g.pad_w < 0)
    return false;
  const int64_t image = static_cast<int64_t>(g.channels) *
                        (g.pool_kernel > 0 ? static_cast<int64_t>(g.pool_src_h) * g.pool_src_w
                                           : static_cast<int64_t>(g.height) * g.width);
  if (image >= (int64_t{1} << 31))
    return false;
  const int oh = (g.height + 2 * g.pad_h - g.kernel_h) / g.stride_h + 1;
  const int ow = (g.width + 2 * g.pad_w - g.kernel_w) / g.stride_w + 1;
  return oh == g.out_h && ow == g.out_w &&
         static_cast<int64_t>(g.batch) * oh * ow == m &&
         static_cast<int64_t>(g.channels) * g.kernel_h * g.kernel_w == k;
}

Gather32 to_device_gather(const cim22_gather &g, int64_t m, int64_t k, const float *x) {
  Gather32 d{};
  d.kind = g.kind;
  d.pair_rows = (g.kind == CIM22_GATHER_ROWS && (k & 3) == 0 &&
                 (reinterpret_cast<uintptr_t>(x) & 15) == 0) ? 2 : 0;
  d.M = static_cast<int>(m);
  d.K = static_cast<int>(k);
  if (g.kind != CIM22_GATHER_ROWS) {
    d.C = g.channels;
    d.H = g.height;
    d.W = g.width;
    d.KH = g.kernel_h;
    d.KW = g.kernel_w;
    d.SH = g.stride_h;
    d.SW = g.stride_w;
    d.PH = g.pad_h;
    d.PW = g.pad_w;
    d.OH = g.out_h;
    d.OW = g.out_w;
    d.PK = g.pool_kernel;
    d.PS = g.pool_stride;
    d.SRC_H = g.pool_src_h;
    d.SRC_W = g.pool_src_w;
    d.div_ohw = make_fastdiv(static_cast<uint32_t>(g.out_h * g.out_w));
    d.div_ow = make_fastdiv(static_cast<uint32_t>(g.out_w));
    d.div_khw = make_fastdiv(static_cast<uint32_t>(g.kernel_h * g.kernel_w));
    d.div_kw = make_fastdiv(static_cast<uint32_t>(g.kernel_w));
  }
  return d;
}

} // namespace

// Host-side BF16 weight preparation: split, RNE, prealign per lane and K tile.
static void prepare_bf16_weights(const float *w, int64_t n, int64_t k,
                                 int64_t n_pad, int64_t k_pad, int64_t T,
                                 std::vector<int8_t> &mant,
                                 std::vector<int32_t> &exps) {
  mant.assign(2 * n_pad * k_pad, 0);
  exps.assign(2 * T * n_pad, 127);
  uint16_t group[kTileK];
  for (int b = 0; b < 2; ++b)
    for (int64_t lane = 0; lane < n; ++lane)
      for (int64_t t = 0; t < T; ++t) {
        int exp_max = 0;
        for (int i = 0; i < kTileK; ++i) {
          const int64_t col = t * kTileK + i;
          uint16_t bits = 0;
          if (col < k) {
            const float v = w[lane * k + col];
            const bool negative = std::signbit(v), zero = v == 0.0f;
            if (b == 0)
              bits = (negative || zero) ? 0 : f32_to_bf16(v);
            else
              bits = (!negative || zero) ? 0 : f32_to_bf16(-v);
          }
          group[i] = bits;
          exp_max = std::max(exp_max, (bits >> 7) & 0xff);
        }
        bool any = false;
        int8_t *dst = mant.data() + (b * n_pad + lane) * k_pad + t * kTileK;
        for (int i = 0; i < kTileK; ++i) {
          dst[i] = prealign_element(group[i], exp_max);
          any |= dst[i] != 0;
        }
        // A lane whose prealigned tile is all zero contributes +0 for every
        // input; keep its exponent at 127 so it never forces the exact
        // (slow) restore path.
        exps[(b * T + t) * n_pad + lane] = any ? exp_max : 127;
      }
}

static bool int8_range_proof(const int8_t *w, int64_t n, int64_t k) {
  for (int64_t o = 0; o < n; ++o)
    for (int64_t r = 0; r < k; r += kTileK) {
      int64_t lower = 0, upper = 0;
      for (int64_t i = r; i < std::min<int64_t>(k, r + kTileK); ++i) {
        const int64_t v = w[o * k + i];
        upper += v >= 0 ? 127 * v : -128 * v;
        lower += v >= 0 ? -128 * v : 127 * v;
      }
      if (lower < -(1 << 20) || lower >= (1 << 20) || upper < -(1 << 20) ||
          upper >= (1 << 20))
        return false;
    }
  return true;
}

} // namespace cim

using namespace cim;

extern "C" {

cim22_cuda_layer *cim22_cuda_layer_create_bf16(int device, const float *weight,
                                               int64_t n, int64_t k,
                                               char *error,
                                               size_t error_capacity) {
  if (!weight || n <= 0 || k <= 0) {
    copy_error("invalid CIM layer shape", error, error_capacity);
    return nullptr;
  }
  for (int64_t i = 0; i < n * k; ++i)
    if (!std::isfinite(weight[i])) {
      copy_error("BF16 correction requires finite fixed weights", error,
                 error_capacity);
      return nullptr;
    }
  auto *layer = new cim22_cuda_layer();
  layer->device = device;
  layer->bf16 = true;
  layer->n = n;
  layer->k = k;
  layer->n_pad = round_up(n, kLanePad);
  layer->k_pad = round_up(k, kTileK);
  layer->tiles = layer->k_pad / kTileK;
  std::vector<int8_t> mant;
  std::vector<int32_t> exps;
  prepare_bf16_weights(weight, n, k, layer->n_pad, layer->k_pad, layer->tiles,
                       mant, exps);
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice") ||
      !cuda_ok(cudaMalloc(&layer->weights, mant.size()), "cudaMalloc") ||
      !cuda_ok(cudaMalloc(&layer->exponents, exps.size() * sizeof(int32_t)),
               "cudaMalloc") ||
      !cuda_ok(cudaMemcpy(layer->weights, mant.data(), mant.size(),
                          cudaMemcpyHostToDevice),
               "cudaMemcpy") ||
      !cuda_ok(cudaMemcpy(layer->exponents, exps.data(),
                          exps.size() * sizeof(int32_t), cudaMemcpyHostToDevice),
               "cudaMemcpy")) {
    copy_error(last_error(), error, error_capacity);
    cim22_cuda_layer_destroy(layer);
    return nullptr;
  }
  return layer;
}

cim22_cuda_layer *cim22_cuda_layer_create_int8(int device, const int8_t *weight,
                                               int64_t n, int64_t k,
                                               char *error,
                                               size_t error_capacity) {
  if (!weight || n <= 0 || k <= 0) {
    copy_error("invalid CIM layer shape", error, error_capacity);
    return nullptr;
  }
  auto *layer = new cim22_cuda_layer();
  layer->device = device;
  layer->bf16 = false;
  layer->n = n;
  layer->k = k;
  layer->n_pad = round_up(n, kLanePad);
  layer->k_pad = round_up(k, kTileK);
  layer->tiles = layer->k_pad / kTileK;
  layer->range_safe = int8_range_proof(weight, n, k);
  std::vector<int8_t> padded(layer->n_pad * layer->k_pad, 0);
  for (int64_t o = 0; o < n; ++o)
    std::copy_n(weight + o * k, k, padded.data() + o * layer->k_pad);
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice") ||
      !cuda_ok(cudaMalloc(&layer->weights, padded.size()), "cudaMalloc") ||
      !cuda_ok(cudaMemcpy(layer->weights, padded.data(), padded.size(),
                          cudaMemcpyHostToDevice),
               "cudaMemcpy")) {
    copy_error(last_error(), error, error_capacity);
    cim22_cuda_layer_destroy(layer);
    return nullptr;
  }
  return layer;
}

void cim22_cuda_layer_destroy(cim22_cuda_layer *layer) {
  if (!layer)
    return;
  cudaSetDevice(layer->device);
  if (layer->weights)
    cudaFree(layer->weights);
  if (layer->exponents)
    cudaFree(layer->exponents);
  delete layer;
}

int cim22_cuda_layer_range_safe(const cim22_cuda_layer *layer) {
  return layer && layer->range_safe ? 1 : 0;
}
int64_t cim22_cuda_layer_n(const cim22_cuda_layer *layer) { return layer ? layer->n : -1; }
int64_t cim22_cuda_layer_k(const cim22_cuda_layer *layer) { return layer ? layer->k : -1; }

size_t cim22_cuda_layer_workspace_bf16(const cim22_cuda_layer *layer,
                                       int64_t m, int32_t branches) {
  if (!layer || m <= 0)
    return 0;
  const int64_t m_pad = round_up(m, kColumnPad);
  const int64_t ab = branches == 2 ? 1 : 2;
  const int64_t a_bytes = round_up(ab * m_pad * layer->k_pad, 256);
  return static_cast<size_t>(a_bytes + ab * layer->tiles * m_pad * 4);
}

size_t cim22_cuda_layer_workspace_int8(const cim22_cuda_layer *layer, int64_t m) {
  if (!layer || m <= 0)
    return 0;
  return static_cast<size_t>(round_up(m, kColumnPad) * layer->k_pad);
}

int cim22_cuda_layer_prepare_bf16(const cim22_cuda_layer *layer,
                                  const float *x, const cim22_gather *gather,
                                  int64_t m, int32_t branches, void *workspace,
                                  size_t workspace_bytes, int32_t *status,
                                  void *stream) {
  cim22_gather rows{};
  rows.kind = CIM22_GATHER_ROWS;
  const cim22_gather &g = gather ? *gather : rows;
  if (!layer || !layer->bf16 || !x || !status || m <= 0 ||
      (branches != 2 && branches != 4) || !check_gather(g, m, layer->k) ||
      !workspace ||
      workspace_bytes < cim22_cuda_layer_workspace_bf16(layer, m, branches)) {
    set_last_error("invalid arguments to cim22_cuda_layer_prepare_bf16");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t m_pad = round_up(m, kColumnPad);
  const int ab = branches == 2 ? 1 : 2;
  const int T = static_cast<int>(layer->tiles);
  if (m_pad * T * kGroupThreads >= (int64_t{1} << 31)) {
    set_last_error("cim22_cuda_layer_prepare_bf16: columns x K tiles too large for one launch");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  int8_t *A = static_cast<int8_t *>(workspace);
  int32_t *ex = reinterpret_cast<int32_t *>(
      static_cast<char *>(workspace) + round_up(ab * m_pad * layer->k_pad, 256));
  const Gather32 dg = to_device_gather(g, m, layer->k, x);
  const unsigned blocks = static_cast<unsigned>((m_pad * T * kGroupThreads + 255) / 256);
  const FastDiv div_t = make_fastdiv(static_cast<uint32_t>(T));
  if (ab == 1)
    prepare_kernel<1><<<blocks, 256, 0, s>>>(x, dg, div_t, static_cast<int>(m_pad),
                                             static_cast<int>(layer->k_pad), A, ex, status);
  else
    prepare_kernel<2><<<blocks, 256, 0, s>>>(x, dg, div_t, static_cast<int>(m_pad),
                                             static_cast<int>(layer->k_pad), A, ex, status);
  return cuda_ok(cudaGetLastError(), "prepare launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

int cim22_cuda_layer_contract_bf16(const cim22_cuda_layer *layer, int64_t m,
                                   const float *bias, int32_t activation,
                                   int32_t branches, float *y,
                                   const void *workspace,
                                   size_t workspace_bytes, int32_t *status,
                                   void *stream) {
  if (!layer || !layer->bf16 || !y || !status || m <= 0 ||
      (branches != 2 && branches != 4) || activation < 0 || activation > 2 ||
      !workspace ||
      workspace_bytes < cim22_cuda_layer_workspace_bf16(layer, m, branches)) {
    set_last_error("invalid arguments to cim22_cuda_layer_contract_bf16");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t m_pad = round_up(m, kColumnPad);
  const int ab = branches == 2 ? 1 : 2;
  const int T = static_cast<int>(layer->tiles);
  const int8_t *A = static_cast<const int8_t *>(workspace);
  const int32_t *ex = reinterpret_cast<const int32_t *>(
      static_cast<const char *>(workspace) + round_up(ab * m_pad * layer->k_pad, 256));
  if (tc::signsplit_available() &&
      tc::launch_signsplit(A, ex, m_pad, layer->weights, layer->exponents,
                           layer->n_pad, layer->k_pad, T, m, layer->n, bias,
                           activation, ab, y, status, s))
    return cuda_ok(cudaGetLastError(), "signsplit launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
  if (ab == 1)
    launch_signsplit_simt<1>(A, ex, m_pad, layer->weights, layer->exponents, layer->n_pad,
                             layer->k_pad, T, m, layer->n, bias, activation, y, status, s);
  else
    launch_signsplit_simt<2>(A, ex, m_pad, layer->weights, layer->exponents, layer->n_pad,
                             layer->k_pad, T, m, layer->n, bias, activation, y, status, s);
  return cuda_ok(cudaGetLastError(), "signsplit launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

int cim22_cuda_layer_forward_bf16(const cim22_cuda_layer *layer, const float *x,
                                  const cim22_gather *gather, int64_t m,
                                  const float *bias, int32_t activation,
                                  int32_t branches, float *y, void *workspace,
                                  size_t workspace_bytes, int32_t *status,
                                  void *stream) {
  if (!y || activation < 0 || activation > 2) {
    set_last_error("invalid arguments to cim22_cuda_layer_forward_bf16");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  const int rc = cim22_cuda_layer_prepare_bf16(layer, x, gather, m, branches, workspace,
                                               workspace_bytes, status, stream);
  if (rc)
    return rc;
  return cim22_cuda_layer_contract_bf16(layer, m, bias, activation, branches, y, workspace,
                                        workspace_bytes, status, stream);
}

int cim22_cuda_layer_forward_int8(const cim22_cuda_layer *layer,
                                  const int8_t *x, int64_t m, int32_t *y,
                                  void *workspace, size_t workspace_bytes,
                                  int32_t *status, void *stream) {
  if (!layer || layer->bf16 || !x || !y || !status || m <= 0 || !workspace ||
      workspace_bytes < cim22_cuda_layer_workspace_int8(layer, m)) {
    set_last_error("invalid arguments to cim22_cuda_layer_forward_int8");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t m_pad = round_up(m, kColumnPad);
  if (layer->range_safe && tc::int8_available() && layer->k % 16 == 0 &&
      tc::launch_int8(x, m, layer->k, layer->weights, layer->n_pad, layer->k_pad, m, layer->n,
                      y, status, s))
    return cuda_ok(cudaGetLastError(), "int8 launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
  int8_t *A = static_cast<int8_t *>(workspace);
  const int64_t total = m_pad * layer->k_pad;
  const unsigned blocks =
      static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 32));
  pad_int8_kernel<<<blocks, 256, 0, s>>>(x, m, layer->k, m_pad, layer->k_pad, A);
  if (!cuda_ok(cudaGetLastError(), "pad launch"))
    return CIM22_STATUS_BAD_ARGUMENT;
  const int T = static_cast<int>(layer->tiles);
  if (layer->range_safe && tc::int8_available() &&
      tc::launch_int8(A, m_pad, layer->k_pad, layer->weights, layer->n_pad, layer->k_pad, m,
                      layer->n, y, status, s))
    return cuda_ok(cudaGetLastError(), "int8 launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
  const dim3 grid(static_cast<unsigned>(m_pad / 64),
                  static_cast<unsigned>((layer->n + 63) / 64));
  int8_simt_kernel<<<grid, 256, 0, s>>>(A, layer->weights, layer->k_pad, T, m,
                                        layer->n, layer->range_safe ? 0 : 1, y,
                                        status);
  return cuda_ok(cudaGetLastError(), "int8 launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

} // extern "C"
