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
#include "signsplit_prep.cuh"
#include "tma_util.cuh"

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstring>
#include <type_traits>
#include <vector>

namespace cim {
namespace {


// ---------------------------------------------------------------------------
// Gather of the K x columns operand (linear rows or conv im2col), with 32-bit
// index arithmetic (checked on the host) and the K decomposition hoisted out
// of the column loop.

struct Gather32 {
  FastDiv div_ohw, div_ow, div_khw, div_kw;
  int kind, C, H, W, KH, KW, SH, SW, PH, PW, OH, OW;
  int PK;         // fused max pool window (NHWC), 0 when absent
  int sC, sH, sW; // element strides of a channel, row and column of the gathered image
  int pdy, pdx;   // strides of the pool window rows and columns in the pre-pool image
  int image;      // elements per image
  int M, K;
  int pair_rows; // rows layout: 2 when K % 4 == 0 and x is 16-byte aligned (float4 loads)
};

// Prepare kernels by gather: linear rows, convolution windows, convolution
// windows over a fused max pool.
enum PrepareMode { kPrepRows = 0, kPrepConv = 1, kPrepConvPool = 2 };

// One element at offset `off` of image `img`; with a fused max pool the max
// over the pool window of the pre-pool image (NaN propagates like
// torch.max_pool2d).
template <int kMode, bool kPool2 = false>
__device__ __forceinline__ float window_load(const float *__restrict__ img, const Gather32 &g,
                                             int off) {
  if (kMode != kPrepConvPool)
    return __ldg(img + off);
  if (kPool2 || g.PK == 2) {
    // The common 2x2 window: four independent loads, then the ordered max.
    const float v0 = __ldg(img + off), v1 = __ldg(img + off + g.pdx);
    const float v2 = __ldg(img + off + g.pdy), v3 = __ldg(img + off + g.pdy + g.pdx);
    float m = v0;
    m = (v1 > m || v1 != v1) ? v1 : m;
    m = (v2 > m || v2 != v2) ? v2 : m;
    return (v3 > m || v3 != v3) ? v3 : m;
  }
  float m = 0.0f;
  bool any = false;
  for (int dy = 0; dy < g.PK; ++dy)
    for (int dx = 0; dx < g.PK; ++dx) {
      const float v = __ldg(img + off + dy * g.pdy + dx * g.pdx);
      if (!any || v > m || v != v) {
        m = v;
        any = true;
      }
    }
  return m;
}


// Sign-split preparation of 64-element groups (prepareBF16Input,
// BF16Compensation.cpp:92-118, on the gathered operand of the reference's
// im2col / row layout). Eight threads share a (column m, K tile t) group,
// eight consecutive K elements each; the group maximum of each branch is an
// xor-shuffle reduction within the 8-lane subgroup, then each thread writes
// its 8 aligned bytes per branch. A block serves one K tile and 32 * cols
// columns, so every thread decomposes its eight K indices into
// (channel, kernel row, kernel column) offsets once and reuses them for
// `cols` columns. Padding columns (m >= M) and padding K are zero; an
// all-zero group records the exponent kZeroGroup.
//
// Alignment fast path: when the group maximum is a normal BF16 with biased
// exponent Ex >= 8, scaling by 2^(127-Ex) is exact for every element that
// stays normal and ExpPrealign yields (0x80 | m) >> (Ex - e + 1), i.e.
// floor(v * 2^(133 - Ex)) for the BF16 value v, which is 0 for gaps >= 7 and
// subnormal elements; fma(v, 2^(133 - Ex), 2^23) rounded toward zero holds
// that floor in its low mantissa bits. Other groups take the exact RNE
// scaling of bf16_scalbn. The scaled maximum lies in [1, 2), so the prealign
// exponent is always 127.

// The eight K indices kbeg .. kbeg+7 of one thread: image offsets (channel,
// kernel row, kernel column) relative to a window origin, and which are < K.
struct Taps8 {
  int rel[8], di[8], dj[8];
  unsigned kvalid;
};

template <int kMode>
__device__ __forceinline__ Taps8 make_taps8(const Gather32 &g, int kbeg) {
  Taps8 tp;
  tp.kvalid = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    tp.kvalid |= (kbeg + e < g.K ? 1u : 0u) << e;
  if (kMode != kPrepRows) {
    int c = fdiv(kbeg, g.div_khw);
    const int rk = kbeg - c * g.KH * g.KW;
    int i = fdiv(rk, g.div_kw);
    int j = rk - i * g.KW;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      tp.rel[e] = c * g.sC + i * g.sH + j * g.sW;
      tp.di[e] = i;
      tp.dj[e] = j;
      if (++j == g.KW) {
        j = 0;
        if (++i == g.KH) {
          i = 0;
          ++c;
        }
      }
    }
  }
  return tp;
}

// The eight gathered values of column m at the thread's taps (zero for
// padding columns, padding K and conv padding).
template <int kMode>
__device__ __forceinline__ void gather8(const float *__restrict__ x, const Gather32 &g,
                                        const Taps8 &tp, int m, int kbeg, float (&v)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e)
    v[e] = 0.0f;
  if (m >= g.M || !tp.kvalid)
    return;
  if (kMode == kPrepRows) {
    const float *row = x + static_cast<int64_t>(m) * g.K;
    if (g.pair_rows == 2 && tp.kvalid == 0xffu) {
      const float4 *src = reinterpret_cast<const float4 *>(row + kbeg);
      const float4 lo = __ldg(src), hi = __ldg(src + 1);
      v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
      v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if ((tp.kvalid >> e) & 1u)
          v[e] = __ldg(row + kbeg + e);
    }
    return;
  }
  const int n = fdiv(m, g.div_ohw);
  const int rm = m - n * g.OH * g.OW;
  const int oh = fdiv(rm, g.div_ow);
  const int ow = rm - oh * g.OW;
  const int ih0 = oh * g.SH - g.PH, iw0 = ow * g.SW - g.PW;
  const float *img = x + static_cast<int64_t>(n) * g.image;
  const int org = ih0 * g.sH + iw0 * g.sW;
  if (tp.kvalid == 0xffu && ih0 >= 0 && iw0 >= 0 && ih0 + g.KH <= g.H && iw0 + g.KW <= g.W) {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      v[e] = window_load<kMode>(img, g, org + tp.rel[e]);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (((tp.kvalid >> e) & 1u) &&
          static_cast<unsigned>(ih0 + tp.di[e]) < static_cast<unsigned>(g.H) &&
          static_cast<unsigned>(iw0 + tp.dj[e]) < static_cast<unsigned>(g.W))
        v[e] = window_load<kMode>(img, g, org + tp.rel[e]);
  }
}


template <int kActBranches, int kMode, bool kB16>
__global__ void __launch_bounds__(256)
    prepare_kernel(const float *__restrict__ x, Gather32 g, FastDiv div_chunks, int T, int cols,
                   int m_pad, int k_pad, int8_t *__restrict__ A, int32_t *__restrict__ ex,
                   int32_t *status, int win_lo, int win_hi) {
  pdl_launch_dependents();
  pdl_wait();
  const int blk = static_cast<int>(blockIdx.x);
  const int t = fdiv(blk, div_chunks);
  const int chunk = blk - t * static_cast<int>(div_chunks.d);
  const int grp = static_cast<int>(threadIdx.x / kGroupThreads);
  const int sub = static_cast<int>(threadIdx.x % kGroupThreads);
  const unsigned mask = 0xffu << (threadIdx.x & 24);
  const int kbeg = t * kTileK + sub * 8;
  const Taps8 tp = make_taps8<kMode>(g, kbeg);
  for (int r = 0; r < cols; ++r) {
    const int m = (chunk * cols + r) * 32 + grp;
    if (m >= m_pad)
      break; // uniform per 8-lane subgroup
    float v[8];
    gather8<kMode>(x, g, tp, m, kbeg, v);
    int emax[2];
    if constexpr (kB16) {
      uint4 out[2];
      convert8_b16<kActBranches>(v, mask, sub, status, win_lo, win_hi, out, emax);
#pragma unroll
      for (int a = 0; a < kActBranches; ++a)
        *reinterpret_cast<uint4 *>(A + ((static_cast<int64_t>(a) * m_pad + m) * k_pad + kbeg) *
                                           2) = out[a];
    } else {
      uint2 out[2];
      convert8<kActBranches>(v, mask, sub, status, out, emax);
#pragma unroll
      for (int a = 0; a < kActBranches; ++a)
        *reinterpret_cast<uint2 *>(A + (static_cast<int64_t>(a) * m_pad + m) * k_pad + kbeg) =
            out[a];
    }
#pragma unroll
    for (int a = 0; a < kActBranches; ++a)
      if (sub == 0)
        ex[(static_cast<int64_t>(a) * T + t) * m_pad + m] = emax[a];
  }
}

// NCHW convolution gathers: one thread per (column m, K tile t) group. A
// block serves one K tile and 256 consecutive columns, so a warp's 32 threads
// read the same kernel tap of 32 neighbouring output pixels - contiguous (or
// pool-stride spaced) floats of one channel row - and every thread owns its
// whole 64-element group: the maximum needs no shuffles and the 64 aligned
// bytes leave as four 16-byte stores. The K decomposition depends on the tile
// only: the block tabulates its 64 image offsets in shared memory once (read
// four at a time), with the bit sets of its elements by kernel row and column,
// from which each column forms the bit set of its in-bounds elements with
// four lookups; a load is one bit test. A 4-branch layer keeps the signed
// BF16 pairs and splits them into the xp/xn branches when aligning: RNE
// commutes with max(., 0) and negation. The fused-pool form handles 2x2
// windows. Kernels of at most kTapMasks rows and columns.
constexpr int kTapMasks = 16;

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
// kStaged: the warp's 32 columns (consecutive, all in the call) are written
// into the warp's shared-memory tile `stage` (per branch 32 rows of 64 or
// 128 bytes, 16-byte chunks swizzled as `omap` describes) and leave with one
// TMA store per branch, so that whole lines reach global memory.
template <int kActBranches, bool kB16 = false, bool kStaged = false>
__device__ __forceinline__ void finish_group(const uint32_t (&signed_pairs)[32],
                                             uint32_t raw_max, int32_t *status,
                                             int8_t *__restrict__ A, int32_t *__restrict__ ex,
                                             int m_pad, int k_pad, int T, int t, int m,
                                             int kbeg, int win_lo = 1, int win_hi = 0,
                                             uint8_t *stage = nullptr,
                                             const CUtensorMap *omap = nullptr) {
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
    if constexpr (kStaged) {
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

template <int kActBranches, bool kPool, bool kB16>
__global__ void __launch_bounds__(256, kActBranches == 2 ? 2 : 4)
    prepare_nchw_kernel(const float *__restrict__ x, Gather32 g, FastDiv div_chunks, int T,
                        int cols, int m_pad, int k_pad, int8_t *__restrict__ A,
                        int32_t *__restrict__ ex, int32_t *status, int win_lo, int win_hi) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int kMode = kPool ? kPrepConvPool : kPrepConv;
  __shared__ __align__(16) int sRel[kTileK];
  // sRows[r] (sCols[r]): the tile's elements (< K) of kernel rows (columns) < r.
  __shared__ unsigned long long sRows[kTapMasks + 1], sCols[kTapMasks + 1];
  const int blk = static_cast<int>(blockIdx.x);
  const int t = fdiv(blk, div_chunks);
  const int chunk0 = (blk - t * static_cast<int>(div_chunks.d)) * cols;
  const int kbeg = t * kTileK;
  if (threadIdx.x < kTileK) {
    const int k = kbeg + static_cast<int>(threadIdx.x);
    const int c = fdiv(k, g.div_khw);
    const int rk = k - c * g.KH * g.KW;
    const int i = fdiv(rk, g.div_kw);
    const int j = rk - i * g.KW;
    const bool valid = k < g.K;
    sRel[threadIdx.x] = valid ? c * g.sC + i * g.sH + j * g.sW : 0;
    const int half = static_cast<int>(threadIdx.x) >> 5; // low or high word of the masks
    for (int r = 0; r <= g.KH; ++r) {
      const unsigned b = __ballot_sync(kFull, valid && i < r);
      if ((threadIdx.x & 31) == 0)
        reinterpret_cast<unsigned *>(&sRows[r])[half] = b;
    }
    for (int q = 0; q <= g.KW; ++q) {
      const unsigned b = __ballot_sync(kFull, valid && j < q);
      if ((threadIdx.x & 31) == 0)
        reinterpret_cast<unsigned *>(&sCols[q])[half] = b;
    }
  }
  __syncthreads();
  // The block's `cols` chunks of 256 consecutive columns, one column per
  // thread and chunk.
  for (int r = 0; r < cols; ++r) {
  const int m = (chunk0 + r) * 256 + static_cast<int>(threadIdx.x);
  if (m >= m_pad)
    break; // whole warps: m_pad is a multiple of 128
  const float *base = x; // the column's window origin (may lie before the image)
  unsigned long long inb = 0; // in-bounds elements of this column
  if (m < g.M) {
    const int n = fdiv(m, g.div_ohw);
    const int rm = m - n * g.OH * g.OW;
    const int oh = fdiv(rm, g.div_ow);
    const int ow = rm - oh * g.OW;
    const int ih0 = oh * g.SH - g.PH, iw0 = ow * g.SW - g.PW;
    base = x + static_cast<int64_t>(n) * g.image + (ih0 * g.sH + iw0 * g.sW);
    const int rlo = min(max(-ih0, 0), g.KH), rhi = max(min(g.H - ih0, g.KH), rlo);
    const int clo = min(max(-iw0, 0), g.KW), chi = max(min(g.W - iw0, g.KW), clo);
    inb = (sRows[rhi] & ~sRows[rlo]) & (sCols[chi] & ~sCols[clo]);
  }
  // Pass 1: gather and round to signed BF16 pairs (for a 2-branch layer,
  // also their largest bit pattern as unsigned halves: above 0x8000 exactly
  // when some BF16 input is negative and nonzero). The loads of the next 16
  // elements are issued before the current 16 are converted, so that two
  // chunks of loads are in flight.
  uint32_t signed_pairs[32];
  uint32_t raw_max = 0;
  auto load_chunk = [&](int chunk, float (&v)[16]) {
    if (kbeg + chunk >= g.K) {
      // K padding: zeros, no loads.
#pragma unroll
      for (int e = 0; e < 16; ++e)
        v[e] = 0.0f;
      return;
    }
#pragma unroll
    for (int e4 = 0; e4 < 16; e4 += 4) {
      const int4 rel = *reinterpret_cast<const int4 *>(&sRel[chunk + e4]);
      const int r4[4] = {rel.x, rel.y, rel.z, rel.w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        v[e4 + e] = (inb >> (chunk + e4 + e)) & 1ull
                        ? window_load<kMode, kPool>(base, g, r4[e])
                        : 0.0f;
    }
  };
  float vbuf[2][16];
  load_chunk(0, vbuf[0]);
#pragma unroll
  for (int c = 0; c < kTileK / 16; ++c) {
    if (c + 1 < kTileK / 16)
      load_chunk((c + 1) * 16, vbuf[(c + 1) & 1]);
    const float(&v)[16] = vbuf[c & 1];
    const int chunk = c * 16;
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      const int q = (chunk + e) / 2;
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[e], v[e + 1]);
      signed_pairs[q] = *reinterpret_cast<const uint32_t *>(&h);
      if (kActBranches == 1)
        raw_max = __vmaxu2(raw_max, signed_pairs[q]);
    }
  }
  finish_group<kActBranches, kB16>(signed_pairs, raw_max, status, A, ex, m_pad, k_pad, T, t,
                                   m, kbeg, win_lo, win_hi);
  }
}



// NCHW convolution gathers staged by TMA: a work item is 256 consecutive
// columns (whole output rows of one image, or whole images) and one K tile.
// One bulk-tensor copy brings the input window those columns read - the
// tile's channels, the rows and columns of its kernel windows, with the
// padding - into shared memory; the copy reads the zero padding itself
// (elements outside the image read as +0), so the gather has no bounds
// tests and every element is one shared-memory load at a column base plus a
// per-tile offset (the last K tile of a layer whose K is not a multiple of 64
// takes zeros for the elements past K). Then the same split, rounding,
// prealign and stores as prepare_nchw_kernel.
//
// Block b takes a run of consecutive items [b * run, (b + 1) * run) in
// column-chunk-major order (the K tiles of a chunk, then the next chunk), so
// the blocks resident at one time read neighbouring windows, which share
// channels and halo rows in L2. A ring of three window stages: the copies
// of the block's next two items are in flight while it converts the
// current one; a stage's full barrier completes with its copy, its empty
// barrier when all eight warps have read it. The window offsets of the 64
// elements of a tile depend only on the tile's first element modulo KH * KW,
// so one table per phase is built when the block starts. Runs of up to
// eight items keep several waves of blocks, so the
// hardware scheduler fills SMs as the neighbouring kernels' blocks leave
// (programmatic dependent launch overlaps the tails).
struct BoxGather {
  int wb, hb, cb, nb; // box extents: columns, rows, channels, images
  int x0;             // first box column (a multiple of 4, <= -PW)
  int words;          // wb * hb * cb * nb
  int stage_floats;   // one stage of the window ring: words rounded up to 128 bytes
  int stages;         // window stages in the ring (at most kBoxStages)
};

constexpr int kBoxStages = 3;
constexpr int kBoxWarps = 8; // 256 threads

template <int kActBranches, bool kB16>
__global__ void __launch_bounds__(256, kActBranches == 2 ? 2 : 3)
    prepare_nchw_box_kernel(const __grid_constant__ CUtensorMap map,
                            const __grid_constant__ CUtensorMap omap, Gather32 g, BoxGather b,
                            FastDiv div_T, int T, int items, int run, int m_pad, int k_pad,
                            int8_t *__restrict__ A, int32_t *__restrict__ ex, int32_t *status,
                            int win_lo, int win_hi) {
  extern __shared__ __align__(1024) unsigned char box_raw[];
  // Each warp's output tiles first (1024-byte aligned for the swizzle; the
  // launch adds the alignment slack), then the window ring, then the offset
  // table.
  constexpr int kOutTile = kActBranches * 32 * (kB16 ? 128 : 64);
  uint8_t *out_tiles = box_raw + ((1024u - (shared_addr(box_raw) & 1023u)) & 1023u);
  uint8_t *my_tile = out_tiles + (threadIdx.x >> 5) * kOutTile;
  float *ring = reinterpret_cast<float *>(out_tiles + kBoxWarps * kOutTile);
  int *rel_table = reinterpret_cast<int *>(ring + b.stages * b.stage_floats);
  __shared__ __align__(8) uint64_t full[kBoxStages], empty[kBoxStages];
  pdl_launch_dependents();
  const int khw = g.KH * g.KW;
  const int hw = g.OH * g.OW;
  const int tid = static_cast<int>(threadIdx.x);
  const int item0 = static_cast<int>(blockIdx.x) * run;
  const int n_items = min(run, items - item0);
  if (tid == 0)
    for (int s = 0; s < b.stages; ++s) {
      barrier_init(&full[s], 1);
      barrier_init(&empty[s], kBoxWarps);
    }
  // Window byte offsets of the 64 K elements of a tile for every phase
  // ph = kbeg mod (KH * KW): element e is k = c0 * KH * KW + ph + e.
  for (int idx = tid; idx < khw * kTileK; idx += 256) {
    const int r = idx / kTileK + idx % kTileK; // ph + e
    const int c = r / khw, rk = r - c * khw;
    const int i = rk / g.KW, j = rk - i * g.KW;
    rel_table[idx] = 4 * ((c * b.hb + i) * b.wb + j);
  }
  __syncthreads();
  pdl_wait();
  // First input row of an item's box: its first output row's window, or the
  // image's top padding when the 256 columns hold whole images.
  auto issue = [&](int i) {
    const int item = item0 + i, s = i % b.stages;
    const int chunk = fdiv(item, div_T);
    const int t = item - chunk * T;
    const int m0 = chunk * 256;
    const int n0 = fdiv(m0, g.div_ohw);
    const int ih0 = hw >= 256 ? fdiv(m0 - n0 * hw, g.div_ow) * g.SH - g.PH : -g.PH;
    barrier_expect_tx(&full[s], static_cast<uint32_t>(b.words) * 4u);
    tma_load_4d(ring + s * b.stage_floats, &map, &full[s], b.x0, ih0, (t * kTileK) / khw, n0);
  };
  int issued = 0;
  if (tid == 0)
    for (; issued < min(b.stages - 1, n_items); ++issued)
      issue(issued);
  int i = 0; // items this thread has seen arrive
  for (; i < n_items; ++i) {
    const int s = i % b.stages;
    if (tid == 0 && issued < n_items) {
      // The stage of item i + stages - 1 last held item i - 1: every warp
      // has left it when its empty barrier completes.
      if (i >= 1 && !barrier_wait(&empty[issued % b.stages], ((i - 1) / b.stages) & 1))
        break;
      issue(issued++);
    }
    if (!barrier_wait(&full[s], (i / b.stages) & 1))
      break;
    const int item = item0 + i;
    const int chunk = fdiv(item, div_T);
    const int t = item - chunk * T;
    const int kbeg = t * kTileK;
    const int m0 = chunk * 256;
    const int m = m0 + tid;
    if (m < m_pad) { // whole warps: m_pad is a multiple of 128
      uint32_t signed_pairs[32];
      uint32_t raw_max = 0;
      if (m < g.M) {
        const int n0 = fdiv(m0, g.div_ohw);
        const int ih0 = hw >= 256 ? fdiv(m0 - n0 * hw, g.div_ow) * g.SH - g.PH : -g.PH;
        const int n = fdiv(m, g.div_ohw);
        const int rm = m - n * hw;
        const int oh = fdiv(rm, g.div_ow);
        const int ow = rm - oh * g.OW;
        // 32-bit shared-memory byte addresses: the column's window origin
        // plus the element's byte offset.
        const uint32_t base =
            shared_addr(ring) +
            4u * static_cast<uint32_t>(s * b.stage_floats +
                                       ((n - n0) * b.cb * b.hb + (oh * g.SH - g.PH - ih0)) * b.wb +
                                       (ow * g.SW - g.PW - b.x0));
        const int *rel = rel_table + (kbeg - (kbeg / khw) * khw) * kTileK;
        auto convert4 = [&](int e4, float v0, float v1, float v2, float v3) {
          const __nv_bfloat162 h0 = __floats2bfloat162_rn(v0, v1);
          const __nv_bfloat162 h1 = __floats2bfloat162_rn(v2, v3);
          signed_pairs[e4 / 2] = *reinterpret_cast<const uint32_t *>(&h0);
          signed_pairs[e4 / 2 + 1] = *reinterpret_cast<const uint32_t *>(&h1);
          if (kActBranches == 1)
            raw_max =
                __vmaxu2(raw_max, __vmaxu2(signed_pairs[e4 / 2], signed_pairs[e4 / 2 + 1]));
        };
        if (kbeg + kTileK <= g.K) {
#pragma unroll
          for (int e4 = 0; e4 < kTileK; e4 += 4) {
            const int4 r4 = *reinterpret_cast<const int4 *>(&rel[e4]);
            convert4(e4, lds_f32(base + r4.x), lds_f32(base + r4.y), lds_f32(base + r4.z),
                     lds_f32(base + r4.w));
          }
        } else {
          // The layer's last K tile: zeros for the elements past K.
          const int kv = g.K - kbeg;
#pragma unroll
          for (int e4 = 0; e4 < kTileK; e4 += 4) {
            const int4 r4 = *reinterpret_cast<const int4 *>(&rel[e4]);
            convert4(e4, e4 < kv ? lds_f32(base + r4.x) : 0.0f,
                     e4 + 1 < kv ? lds_f32(base + r4.y) : 0.0f,
                     e4 + 2 < kv ? lds_f32(base + r4.z) : 0.0f,
                     e4 + 3 < kv ? lds_f32(base + r4.w) : 0.0f);
          }
        }
      } else {
#pragma unroll
        for (int q = 0; q < 32; ++q)
          signed_pairs[q] = 0; // a padding column: an all-zero group
      }
      finish_group<kActBranches, kB16, true>(signed_pairs, raw_max, status, A, ex, m_pad,
                                             k_pad, T, t, m, kbeg, win_lo, win_hi, my_tile,
                                             &omap);
    }
    // This warp is done with the stage.
    __syncwarp();
    if ((tid & 31) == 0)
      barrier_arrive(&empty[s]);
  }
  if (i < n_items) {
    // A wait ran out: report it; the issuing thread waits (bounded) for the
    // copies it issued that it has not seen complete (at most one per stage,
    // so each is its stage's current phase).
    atomicOr(status, CIM22_STATUS_TIMEOUT);
    if (tid == 0)
      for (int j = i; j < issued; ++j)
        barrier_wait(&full[j % b.stages], (j / b.stages) & 1, 100000000ull);
  }
  // The warp's output stores complete before the block leaves.
  if ((tid & 31) == 0)
    bulk_wait();
}

// The box of the TMA-staged gather for a layer, or false when its columns do
// not tile into whole output rows or whole images per 256-column block, the
// image rows are not 16-byte multiples, or the box exceeds kBoxSmemLimit.
constexpr int kBoxSmemLimit = 47 * 1024;

static int device_sms() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      return 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Dynamic shared memory of prepare_nchw_box_kernel: the window ring (one
// stage rounded up to 128 bytes, plus 128 bytes for the ring's alignment) and
// the offset table of every kernel-window phase.
static size_t box_smem(const BoxGather &b, int khw, int act_branches, bool b16) {
  const size_t out_tiles = static_cast<size_t>(kBoxWarps) * act_branches * 32 * (b16 ? 128 : 64);
  return out_tiles +
         (static_cast<size_t>(b.stages) * b.stage_floats + static_cast<size_t>(khw) * kTileK) *
             sizeof(float) +
         1024;
}

static bool plan_box_gather(const Gather32 &g, const float *x, int T, BoxGather &b) {
  if (g.kind != CIM22_GATHER_CONV_NCHW || g.PK != 0 || (g.W & 3) != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 15) != 0 || g.sW != 1 || g.sH != g.W ||
      g.sC != g.H * g.W)
    return false;
  const int hw = g.OH * g.OW;
  if (hw >= 256) {
    if (256 % g.OW != 0 || hw % 256 != 0)
      return false;
    b.nb = 1;
    b.hb = (256 / g.OW - 1) * g.SH + g.KH;
  } else {
    if (256 % hw != 0)
      return false;
    b.nb = 256 / hw;
    b.hb = (g.OH - 1) * g.SH + g.KH;
  }
  b.x0 = -((g.PW + 3) / 4) * 4;
  b.wb = (((g.OW - 1) * g.SW - g.PW + g.KW - b.x0) + 3) / 4 * 4;
  const int khw = g.KH * g.KW;
  b.cb = 0;
  for (int t = 0; t < T; ++t) {
    const int lo = t * kTileK / khw, hi = std::min(g.C - 1, (t * kTileK + kTileK - 1) / khw);
    b.cb = std::max(b.cb, hi - lo + 1);
  }
  if (b.wb > 256 || b.hb > 256 || b.cb > 256 || b.nb > 256)
    return false;
  const int64_t words = int64_t{b.wb} * b.hb * b.cb * b.nb;
  if (words * 4 + 128 > kBoxSmemLimit)
    return false;
  b.words = static_cast<int>(words);
  b.stage_floats = (b.words + 31) / 32 * 32;
  const int64_t items = (int64_t{g.M} + 255) / 256 * T;
  // Three stages (the copies of the next two items in flight): measured
  // faster on ResNet-18's convolutions than two, also where the third stage
  // costs a resident block (a stride-2 convolution's larger window).
  b.stages = kBoxStages;
  // The largest output tiles (4-branch, BF16 operands) must fit beside them.
  return items < (int64_t{1} << 31) && box_smem(b, khw, 2, true) <= 200 * 1024;
}

// ---------------------------------------------------------------------------
// Sign-split contraction on CUDA cores (dp4a). CTA tile kBM columns x kBN
// lanes, all branches; thread (tr, tc) owns columns tr + i * kTR (i < kRM)
// and lanes 4tc .. 4tc + 3.
constexpr int kRowStride = 80;


// kFuse < 0: A and Ex come from the prepare kernel's workspace. kFuse =
// kPrepRows / kPrepConv / kPrepConvPool: the CTA gathers and prealigns its own
// activation tiles from x (eight threads per 64-element group, as
// prepare_kernel does) into shared memory, so a narrow layer is one launch
// and its prepared columns never travel through HBM.
template <int kActBranches, int kTC, int kRM, int kFuse>
__global__ void __launch_bounds__(256)
    signsplit_simt_kernel(const int8_t *__restrict__ A,
                          const int32_t *__restrict__ exA, int64_t m_pad,
                          const int8_t *__restrict__ B,
                          const int32_t *__restrict__ exB, int64_t n_pad,
                          int64_t k_pad, int T, int64_t M, int64_t N,
                          const float *__restrict__ bias,
                          const float *__restrict__ post_scale,
                          const float *__restrict__ post_shift,
                          const float *__restrict__ residual, int act, int64_t out_pixels,
                          float *__restrict__ y, int32_t *status,
                          const float *__restrict__ x, Gather32 g, int k_logical) {
  pdl_launch_dependents();
  pdl_wait();
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
    if (kFuse < 0) {
      for (int i = tid; i < kActBranches * kBM; i += 256)
        sExA[i / kBM][i % kBM] =
            exA[(static_cast<int64_t>(i / kBM) * T + t) * m_pad + m0 + i % kBM];
    } else {
      // 32 groups per pass: eight threads each own eight K elements.
      constexpr int kPrepMode = kFuse < 0 ? kPrepRows : kFuse;
      const int grp = tid / kGroupThreads, sub = tid % kGroupThreads;
      const unsigned mask = 0xffu << (tid & 24);
      const int kbeg = t * kTileK + sub * 8;
      const Taps8 tp = make_taps8<kPrepMode>(g, kbeg);
#pragma unroll
      for (int r0 = 0; r0 < kBM; r0 += 32) {
        const int row = r0 + grp;
        float v[8];
        gather8<kPrepMode>(x, g, tp, static_cast<int>(m0) + row, kbeg, v);
        uint2 out[2];
        int emax[2];
        convert8<kActBranches>(v, mask, sub, status, out, emax);
#pragma unroll
        for (int a = 0; a < kActBranches; ++a) {
          *reinterpret_cast<uint2 *>(&As[a][row][sub * 8]) = out[a];
          if (sub == 0)
            sExA[a][row] = emax[a];
        }
      }
    }
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
    if (kFuse < 0) {
      for (int i = tid; i < kActBranches * kBM * 4; i += 256) {
        const int a = i / (kBM * 4), r = (i >> 2) % kBM, c = i & 3;
        if (live[a])
          *reinterpret_cast<int4 *>(&As[a][r][c * 16]) = *reinterpret_cast<const int4 *>(
              A + (static_cast<int64_t>(a) * m_pad + m0 + r) * k_pad +
              static_cast<int64_t>(t) * kTileK + c * 16);
      }
      __syncthreads();
    }
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
    // 16-element chunks past K hold zeros in both operands: skip them.
    const int kk_end = min(4, (k_logical - t * kTileK + 15) / 16);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      if (kk >= kk_end)
        break;
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
    // Rows layout y[row][lane], or NCHW images y[image][lane][pixel].
    int64_t base = row * N, lane_stride = 1;
    if (out_pixels > 0) {
      const int64_t image = row / out_pixels;
      base = image * N * out_pixels + (row - image * out_pixels);
      lane_stride = out_pixels;
    }
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
      if (post_scale != nullptr && lane < N)
        out = __fmaf_rn(out, post_scale[lane], post_shift[lane]);
      if (residual != nullptr && row < M && lane < N)
        out = __fadd_rn(out, residual[base + lane * lane_stride]);
      out = apply_act(out, act);
      if (row < M && lane < N)
        y[base + lane * lane_stride] = out;
    }
  }
}

// Tile shape per layer: 8 or 16-lane tiles for layers of at most 8 or 16
// lanes, 32 otherwise; 2 column rows per thread when that still gives every
// SM two CTAs.
template <int kAB, int kFuse = -1>
void launch_signsplit_simt(const int8_t *A, const int32_t *exA, int64_t m_pad,
                           const int8_t *B, const int32_t *exB, int64_t n_pad,
                           int64_t k_pad, int T, int64_t M, int64_t N,
                           const float *bias, const float *post_scale,
                           const float *post_shift, const float *residual, int act,
                           int64_t out_pixels, float *y, int32_t *status, cudaStream_t s,
                           int k_logical, const float *x = nullptr, Gather32 g = Gather32{}) {
  const int64_t target = 2 * 148;
  auto go = [&](auto kernel, int64_t rows_per_cta, unsigned ny) {
    launch_pdl(kernel, dim3(static_cast<unsigned>(m_pad / rows_per_cta), ny), 256, 0, s, A, exA, m_pad, B, exB, n_pad, k_pad, T, M, N, bias, post_scale, post_shift,
        residual, act, out_pixels, y, status, x, g, k_logical);
  };
  if (N <= 8) {
    go(signsplit_simt_kernel<kAB, 2, 1, kFuse>, 128, 1);
  } else if (N <= 16) {
    const unsigned ny = static_cast<unsigned>((N + 15) / 16);
    if ((m_pad / 128) * ny >= target)
      go(signsplit_simt_kernel<kAB, 4, 2, kFuse>, 128, ny);
    else
      go(signsplit_simt_kernel<kAB, 4, 1, kFuse>, 64, ny);
  } else {
    const unsigned ny = static_cast<unsigned>((N + 31) / 32);
    if ((m_pad / 64) * ny >= target)
      go(signsplit_simt_kernel<kAB, 8, 2, kFuse>, 64, ny);
    else
      go(signsplit_simt_kernel<kAB, 8, 1, kFuse>, 32, ny);
  }
}

// ---------------------------------------------------------------------------
// One-tile sign-split layers (K <= 64) of at most kDirectLanes lanes, such as
// the first convolution of an image network. Each thread owns kCols columns
// 256 apart: per column it gathers the group through the block's tap table
// (a warp reads one tap of 32 neighbouring output pixels), splits, rounds and
// prealigns it in registers (the thread owns the whole group: no shuffles);
// then, lane by lane, every weight word read from shared memory (a broadcast)
// is dotted with all of the thread's columns. The prepared operand never
// leaves the registers, and a warp's outputs of one lane and column slot are
// 32 consecutive columns (128-byte stores into NCHW planes). kWords (even) is
// the number of 4-byte K words holding the layer's K elements. With one K tile
// there is no K sum: each branch value is its restored tile added to +0, as
// in the multi-tile kernels.
constexpr int kDirectLanes = 64;

// Columns per thread (at most 4): the aligned operand of all of them stays
// within 48 registers.
template <int kActBranches, int kWords>
constexpr int direct_columns() {
  return 48 / (kActBranches * kWords) >= 4   ? 4
         : 48 / (kActBranches * kWords) >= 1 ? 48 / (kActBranches * kWords)
                                             : 1;
}

// The K elements of a one-tile layer as seen from a column's window origin,
// passed in kernel parameter space so that the unrolled gather reads each
// offset as an instruction operand. rows[t] (cols[t]) is the bit set of the K
// elements whose kernel row (column) is below t; a column's valid elements are
// those of its in-bounds kernel rows and columns. A rows gather has one
// "kernel row" of K elements at offsets 0 .. K-1.
struct DirectTaps {
  int rel[kTileK];
  unsigned long long rows[kTileK + 1], cols[kTileK + 1];
};

DirectTaps make_direct_taps(const Gather32 &g) {
  DirectTaps t{};
  const bool conv = g.kind != CIM22_GATHER_ROWS;
  const int KH = conv ? g.KH : 1, KW = conv ? g.KW : 1;
  unsigned long long rowbits[kTileK] = {}, colbits[kTileK] = {};
  for (int k = 0; k < g.K; ++k) {
    int i = 0, j = 0;
    if (conv) {
      const int c = k / (KH * KW), r = k % (KH * KW);
      i = r / KW;
      j = r % KW;
      t.rel[k] = c * g.sC + i * g.sH + j * g.sW;
    } else {
      t.rel[k] = k;
    }
    rowbits[i] |= 1ull << k;
    colbits[j] |= 1ull << k;
  }
  for (int r = 0; r < KH; ++r)
    t.rows[r + 1] = t.rows[r] | rowbits[r];
  for (int c = 0; c < KW; ++c)
    t.cols[c + 1] = t.cols[c] | colbits[c];
  return t;
}

// Gather, split, round and prealign the group of column m: aw[a] holds the
// aligned bytes of activation branch a, ex[a] its group exponent (kZeroGroup
// for an all-zero branch). Returns whether the column can take the fast
// restore for weight exponents in [win_lo, win_hi]: every branch is a zero
// group or has 7 <= ex <= 230 and 140 <= ex + ew <= 374 (then p * 2^(ex-133)
// is a normal f32 that one FMA against -2^23 * 2^(ex-133) yields exactly, and
// the tile Q(p) * 2^(ex+ew-266) is a normal BF16).
template <int kActBranches, int kMode, int kWords>
__device__ __forceinline__ bool direct_prepare(const float *__restrict__ x, const Gather32 &g,
                                               const DirectTaps &tp, int m, bool col_valid,
                                               int win_lo, int win_hi, int32_t *status,
                                               uint32_t (&aw)[kActBranches][kWords],
                                               int (&ex)[kActBranches]) {
  static_assert(kMode != kPrepConvPool, "direct layers gather without a fused pool");
  constexpr int kE = 4 * kWords; // gathered elements (a multiple of 8)
  uint32_t signed_pairs[kE / 2];
  uint32_t raw_max = 0;
  const float *src = x;
  unsigned long long valid = 0;
  if (col_valid) {
    if (kMode == kPrepRows) {
      src = x + static_cast<int64_t>(m) * g.K;
      valid = tp.rows[1];
    } else {
      const int n = fdiv(m, g.div_ohw);
      const int rm = m - n * g.OH * g.OW;
      const int oh = fdiv(rm, g.div_ow);
      const int ow = rm - oh * g.OW;
      const int ih0 = oh * g.SH - g.PH, iw0 = ow * g.SW - g.PW;
      src = x + static_cast<int64_t>(n) * g.image + (ih0 * g.sH + iw0 * g.sW);
      // In-bounds kernel rows [rlo, rhi) and columns [clo, chi).
      const int rlo = min(max(-ih0, 0), g.KH), rhi = max(min(g.H - ih0, g.KH), rlo);
      const int clo = min(max(-iw0, 0), g.KW), chi = max(min(g.W - iw0, g.KW), clo);
      valid = (tp.rows[rhi] & ~tp.rows[rlo]) & (tp.cols[chi] & ~tp.cols[clo]);
    }
  }
#pragma unroll
  for (int chunk = 0; chunk < kE; chunk += 8) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      v[e] = (valid >> (chunk + e)) & 1ull ? __ldg(src + tp.rel[chunk + e]) : 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[e], v[e + 1]);
      signed_pairs[(chunk + e) / 2] = *reinterpret_cast<const uint32_t *>(&h);
      if (kActBranches == 1)
        raw_max = __vmaxu2(raw_max, signed_pairs[(chunk + e) / 2]);
    }
  }
  uint32_t mx[2] = {0, 0};
  // Inputs without a sign bit: the raw maximum is the maximum.
  const uint32_t raw_half = max(raw_max & 0xffffu, raw_max >> 16);
  if (kActBranches == 1 && raw_half < 0x8000u) {
    mx[0] = raw_half;
  } else {
#pragma unroll
    for (int a = 0; a < kActBranches; ++a) {
      uint32_t m2 = 0;
#pragma unroll
      for (int e = 0; e < kE / 2; ++e)
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
  bool fast = true;
#pragma unroll
  for (int a = 0; a < kActBranches; ++a) {
    const bool zero = mx[a] == 0 || nonfinite;
    ex[a] = zero ? kZeroGroup : effective_exponent(static_cast<uint16_t>(mx[a]));
    fast &= zero || (ex[a] >= 7 && ex[a] <= 230 && ex[a] + win_lo >= 140 &&
                     ex[a] + win_hi <= 374);
#pragma unroll
    for (int q = 0; q < kWords; ++q)
      aw[a][q] = zero ? 0u
                      : align4(branch_pair<kActBranches>(signed_pairs[2 * q], a),
                               branch_pair<kActBranches>(signed_pairs[2 * q + 1], a), mx[a],
                               ex[a]);
  }
  return fast;
}

// Dots of one weight row (kWords words, pairs in shared memory) with the
// first kBr activation branches of every column.
template <int kBr, int kCols, int kAB, int kWords>
__device__ __forceinline__ void direct_dots(const uint2 *row,
                                            const uint32_t (&aw)[kCols][kAB][kWords],
                                            int (&p)[kCols][kAB]) {
#pragma unroll
  for (int c = 0; c < kCols; ++c)
#pragma unroll
    for (int a = 0; a < kBr; ++a)
      p[c][a] = 0;
#pragma unroll
  for (int h = 0; h < kWords / 2; ++h) {
    const uint2 b = row[h];
#pragma unroll
    for (int c = 0; c < kCols; ++c)
#pragma unroll
      for (int a = 0; a < kBr; ++a) {
        p[c][a] = __dp4a(static_cast<int>(aw[c][a][2 * h]), static_cast<int>(b.x), p[c][a]);
        p[c][a] = __dp4a(static_cast<int>(aw[c][a][2 * h + 1]), static_cast<int>(b.y), p[c][a]);
      }
  }
}

// The lane loop of the direct kernel when every column of the warp lies in
// the fast-restore window, over the first kBr activation branches.
template <int kBr, int kCols, int kAB, int kWords>
__device__ __forceinline__ void direct_fast_lanes(
    int N, const uint2 (*Bs)[kDirectLanes][kWords / 2], const float (*sSw)[kDirectLanes],
    const float *sBias, const float *sScale, const float *sShift,
    const uint32_t (&aw)[kCols][kAB][kWords], const float (&sx)[kCols][kAB],
    const float (&nsx)[kCols][kAB], float floor_v, float *const (&yp)[kCols],
    const bool (&valid)[kCols], int64_t lane_stride) {
  for (int n = 0; n < N; ++n) {
    float br[kCols][kAB][2];
    int p[2][kCols][kAB];
    direct_dots<kBr>(Bs[0][n], aw, p[0]);
    direct_dots<kBr>(Bs[1][n], aw, p[1]);
    const float sw0 = sSw[0][n], sw1 = sSw[1][n];
#pragma unroll
    for (int c = 0; c < kCols; ++c)
#pragma unroll
      for (int a = 0; a < kBr; ++a) {
        // The two weight signs of one column and branch as one f32x2 pair.
        float v0, v1;
        fma2(__uint_as_float(static_cast<uint32_t>(p[0][c][a]) + 0x4b000000u),
             __uint_as_float(static_cast<uint32_t>(p[1][c][a]) + 0x4b000000u), sx[c][a],
             sx[c][a], nsx[c][a], nsx[c][a], v0, v1);
        fma2(__uint_as_float(__float_as_uint(v0) & 0xffff0000u),
             __uint_as_float(__float_as_uint(v1) & 0xffff0000u), sw0, sw1, 0.0f, 0.0f,
             br[c][a][0], br[c][a][1]);
      }
    const float bn = sBias[n], sn = sScale[n], hn = sShift[n];
    const int64_t off = static_cast<int64_t>(n) * lane_stride;
#pragma unroll
    for (int c = 0; c < kCols; ++c) {
      float out = __fsub_rn(br[c][0][0], br[c][0][1]);
      if (kBr == 2) {
        out = __fsub_rn(out, br[c][1][0]);
        out = __fadd_rn(out, br[c][1][1]);
      }
      out = fmaxf(__fmaf_rn(__fadd_rn(out, bn), sn, hn), floor_v);
      if (valid[c])
        yp[c][off] = out;
    }
  }
}

template <int kActBranches, int kMode, int kWords>
__global__ void __launch_bounds__(256, 2)
    signsplit_direct_kernel(const float *__restrict__ x, Gather32 g,
                            const __grid_constant__ DirectTaps tp,
                            const int8_t *__restrict__ B, const int32_t *__restrict__ exB,
                            int n_pad, int k_pad, int N, const float *__restrict__ bias,
                            const float *__restrict__ post_scale,
                            const float *__restrict__ post_shift, int act, int out_pixels,
                            float *__restrict__ y, int32_t *status) {
  constexpr int kCols = direct_columns<kActBranches, kWords>();
  __shared__ __align__(16) uint2 Bs[2][kDirectLanes][kWords / 2];
  __shared__ float sSw[2][kDirectLanes];
  __shared__ int sExB[2][kDirectLanes];
  __shared__ float sBias[kDirectLanes], sScale[kDirectLanes], sShift[kDirectLanes];
  __shared__ int sWin[2];
  const int tid = static_cast<int>(threadIdx.x);
  // Resident weights first: no earlier kernel writes them.
  for (int i = tid; i < 2 * N * (kWords / 2); i += 256) {
    const int c = i % (kWords / 2), r = (i / (kWords / 2)) % N, w = i / ((kWords / 2) * N);
    Bs[w][r][c] = __ldg(reinterpret_cast<const uint2 *>(
        B + (static_cast<int64_t>(w) * n_pad + r) * k_pad + c * 8));
  }
  if (tid < 2 * N) {
    const int w = tid / N, r = tid - w * N;
    const int e = __ldg(exB + w * n_pad + r); // Ew[w][tile 0][lane]
    sExB[w][r] = e;
    sSw[w][r] = exp2i(e - 133);
  }
  if (tid >= 128 && tid < 160) {
    // Range of the weight exponents: the fast-restore window of the block.
    int lo = INT_MAX, hi = INT_MIN;
    for (int i = tid - 128; i < 2 * N; i += 32) {
      const int e = __ldg(exB + (i / N) * n_pad + i % N);
      lo = min(lo, e);
      hi = max(hi, e);
    }
    lo = __reduce_min_sync(kFull, lo);
    hi = __reduce_max_sync(kFull, hi);
    if (tid == 128) {
      sWin[0] = lo;
      sWin[1] = hi;
    }
  }
  pdl_launch_dependents();
  pdl_wait();
  if (tid < N) {
    // Neutral values where the epilogue has no bias or scale: the merged
    // branch sum is never -0, so adding +0 and fma(v, 1, +0) leave it as it is.
    sBias[tid] = bias != nullptr ? bias[tid] : 0.0f;
    sScale[tid] = post_scale != nullptr ? post_scale[tid] : 1.0f;
    sShift[tid] = post_scale != nullptr ? post_shift[tid] : 0.0f;
  }
  __syncthreads();
  const int win_lo = sWin[0], win_hi = sWin[1];
  uint32_t aw[kCols][kActBranches][kWords];
  int ex[kCols][kActBranches];
  int m[kCols];
  bool valid[kCols];
  bool fast = true;
#pragma unroll
  for (int c = 0; c < kCols; ++c) {
    m[c] = (static_cast<int>(blockIdx.x) * kCols + c) * 256 + tid;
    valid[c] = m[c] < g.M;
    fast &= direct_prepare<kActBranches, kMode, kWords>(x, g, tp, m[c], valid[c], win_lo,
                                                        win_hi, status, aw[c], ex[c]) ||
            !valid[c];
  }
  // Output of lane n: y[m][n] (rows) or y[image][n][pixel] (NCHW planes).
  float *yp[kCols];
  const int64_t lane_stride = out_pixels > 0 ? out_pixels : 1;
#pragma unroll
  for (int c = 0; c < kCols; ++c) {
    int64_t base = static_cast<int64_t>(m[c]) * N;
    if (out_pixels > 0) {
      const int image = m[c] / out_pixels;
      base = static_cast<int64_t>(image) * N * out_pixels + (m[c] - image * out_pixels);
    }
    yp[c] = y + base;
  }
  if (__all_sync(kFull, fast) && act != CIM22_ACT_GELU) {
    // Every column of the warp in the fast window: the tile of dot p is
    // (fma(2^23 + p, sx, -2^23 sx) with the low 16 bits cleared) * sw, exact.
    float sx[kCols][kActBranches], nsx[kCols][kActBranches];
    bool neg_live = false; // some column's xn branch is not a zero group
#pragma unroll
    for (int c = 0; c < kCols; ++c)
#pragma unroll
      for (int a = 0; a < kActBranches; ++a) {
        const bool zero = ex[c][a] == kZeroGroup;
        sx[c][a] = zero ? 0.0f : exp2i(ex[c][a] - 133);
        nsx[c][a] = -8388608.0f * sx[c][a];
        neg_live |= a == 1 && !zero;
      }
    // ReLU as max(v, 0): v is finite and never -0 here; -inf leaves v as is.
    const float floor_v = act == CIM22_ACT_RELU ? 0.0f : -INFINITY;
    // Where the warp's xn branches are all zero groups their tiles are +0 and
    // ((pp - pn) - 0) + 0 == pp - pn (never -0): the 2-branch merge.
    if (kActBranches == 2 && !__any_sync(kFull, neg_live))
      direct_fast_lanes<1>(N, Bs, sSw, sBias, sScale, sShift, aw, sx, nsx, floor_v, yp, valid,
                           lane_stride);
    else
      direct_fast_lanes<kActBranches>(N, Bs, sSw, sBias, sScale, sShift, aw, sx, nsx, floor_v,
                                      yp, valid, lane_stride);
    return;
  }
  for (int n = 0; n < N; ++n) {
    float br[kCols][kActBranches][2];
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      int p[kCols][kActBranches];
      direct_dots<kActBranches>(Bs[w][n], aw, p);
      const int ew = sExB[w][n];
      const float sw = sSw[w][n];
#pragma unroll
      for (int c = 0; c < kCols; ++c)
#pragma unroll
        for (int a = 0; a < kActBranches; ++a) {
          const int e = ex[c][a], s = e + ew;
          if (e == kZeroGroup)
            br[c][a][w] = 0.0f;
          else if (e <= 240 && s >= 140 && s <= 374)
            br[c][a][w] = fmaf(__fmul_rn(trunc8f(p[c][a]), exp2i(e - 133)), sw, 0.0f);
          else
            br[c][a][w] = slow_tile_add(0.0f, p[c][a], ew, e, status);
        }
    }
#pragma unroll
    for (int c = 0; c < kCols; ++c) {
      float out = __fsub_rn(br[c][0][0], br[c][0][1]);
      if (kActBranches == 2) {
        out = __fsub_rn(out, br[c][1][0]);
        out = __fadd_rn(out, br[c][1][1]);
      }
      if (bias != nullptr)
        out = __fadd_rn(out, sBias[n]);
      if (post_scale != nullptr)
        out = __fmaf_rn(out, sScale[n], sShift[n]);
      out = apply_act(out, act);
      if (valid[c])
        yp[c][static_cast<int64_t>(n) * lane_stride] = out;
    }
  }
}

// Whether cim22_cuda_layer_forward_bf16 may run a layer through
// signsplit_direct_kernel (one K tile, at most kDirectLanes lanes).
bool direct_layer(const cim22_cuda_layer *layer) {
  return layer->tiles == 1 && layer->n <= kDirectLanes;
}

// Whether the direct kernel beats the prepare and tensor-core contract
// kernels for this layer (crossovers measured on B200 over one-tile 3x3
// convolutions and linear layers of 2^20 columns). Its cost grows with lanes
// x K words x activation branches; NCHW planes take coalesced stores, rows
// outputs (one column's lanes contiguous) do not.
bool direct_preferred(const cim22_cuda_layer *layer, int branches, int64_t out_pixels) {
  const int64_t words = (layer->k + 7) / 8 * 2, n = layer->n;
  if (out_pixels <= 0)
    return n <= 16 && words <= 8;
  return words <= 8 || n <= 16 || (branches == 2 && n <= 32);
}

// The fused CUDA-core kernel of narrow layers (at most 16 lanes, two K
// tiles) saves a launch, which pays up to about 2^17 columns; above that the
// prepare and tensor-core contract kernels were measured faster.
constexpr int64_t kFusedSimtColumns = int64_t{1} << 17;

template <int kAB, int kMode>
void launch_signsplit_direct(const cim22_cuda_layer *layer, const float *x, const Gather32 &g,
                             int64_t m, const float *bias, const float *post_scale,
                             const float *post_shift, int act, int64_t out_pixels, float *y,
                             int32_t *status, cudaStream_t s) {
  const int words = static_cast<int>((layer->k + 7) / 8) * 2; // even, K <= 4 * words
  const DirectTaps taps = make_direct_taps(g);
  auto go = [&](auto words_tag) {
    constexpr int kWords = decltype(words_tag)::value;
    constexpr int kCols = direct_columns<kAB, kWords>();
    const unsigned grid = static_cast<unsigned>((m + 256 * kCols - 1) / (256 * kCols));
    launch_pdl(signsplit_direct_kernel<kAB, kMode, kWords>, dim3(grid), 256, 0, s, x, g, taps,
               static_cast<const int8_t *>(layer->weights),
               static_cast<const int32_t *>(layer->exponents), static_cast<int>(layer->n_pad),
               static_cast<int>(layer->k_pad), static_cast<int>(layer->n), bias, post_scale,
               post_shift, act, static_cast<int>(out_pixels), y, status);
  };
  switch (words) {
  case 2: go(std::integral_constant<int, 2>{}); break;
  case 4: go(std::integral_constant<int, 4>{}); break;
  case 6: go(std::integral_constant<int, 6>{}); break;
  case 8: go(std::integral_constant<int, 8>{}); break;
  case 10: go(std::integral_constant<int, 10>{}); break;
  case 12: go(std::integral_constant<int, 12>{}); break;
  case 14: go(std::integral_constant<int, 14>{}); break;
  default: go(std::integral_constant<int, 16>{}); break;
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

// Columns of an INT8 convolution (the im2col of normalizeCIMInt8Conv,
// Passes.cpp:1511-1552): A[m][k] for column m = (image, oh, ow) and
// k = (c * KH + i) * KW + j is the input at row oh * SH - PH + i, column
// ow * SW - PW + j of channel c, zero outside the image (padding), for
// k >= K and for m >= M. One thread writes 16 consecutive bytes of a row.
__global__ void __launch_bounds__(256)
    im2col_int8_kernel(const int8_t *__restrict__ x, Gather32 g, int64_t m_pad, int64_t k_pad,
                       int8_t *__restrict__ A) {
  pdl_wait();
  const int chunks = static_cast<int>(k_pad / 16);
  const int64_t total = m_pad * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / chunks);
    const int kb = static_cast<int>(i - static_cast<int64_t>(m) * chunks) * 16;
    uint32_t word[4] = {0, 0, 0, 0};
    if (m < g.M && kb < g.K) {
      const int n = fdiv(m, g.div_ohw);
      const int rm = m - n * g.OH * g.OW;
      const int oh = fdiv(rm, g.div_ow);
      const int ow = rm - oh * g.OW;
      const int ih0 = oh * g.SH - g.PH, iw0 = ow * g.SW - g.PW;
      const int8_t *img = x + static_cast<int64_t>(n) * g.image;
      int c = fdiv(kb, g.div_khw);
      const int rk = kb - c * g.KH * g.KW;
      int ki = fdiv(rk, g.div_kw);
      int kj = rk - ki * g.KW;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int ih = ih0 + ki, iw = iw0 + kj;
        if (kb + e < g.K && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W) {
          const uint32_t b = static_cast<uint8_t>(__ldg(img + c * g.sC + ih * g.sH + iw * g.sW));
          word[e >> 2] |= b << (8 * (e & 3));
        }
        if (++kj == g.KW) {
          kj = 0;
          if (++ki == g.KH) {
            ki = 0;
            ++c;
          }
        }
      }
    }
    *reinterpret_cast<uint4 *>(A + static_cast<int64_t>(m) * k_pad + kb) =
        make_uint4(word[0], word[1], word[2], word[3]);
  }
  pdl_launch_dependents();
}

__global__ void __launch_bounds__(256)
    int8_simt_kernel(const int8_t *__restrict__ A, const int8_t *__restrict__ B,
                     int64_t k_pad, int T, int64_t M, int64_t N,
                     int checked, const int32_t *__restrict__ bias, int64_t out_pixels,
                     FastDiv div_pix, int32_t *__restrict__ y, int32_t *status) {
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
    if (row >= M)
      continue;
    // Rows [M][N], or NCHW images [M / out_pixels][N][out_pixels].
    int64_t base = row * N, step = 1;
    if (out_pixels > 0) {
      const int64_t img = fdiv(static_cast<int>(row), div_pix);
      base = img * N * out_pixels + (row - img * out_pixels);
      step = out_pixels;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int64_t lane = n0 + tc * 4 + c;
      if (lane < N)
        y[base + lane * step] =
            static_cast<int32_t>(acc[r][c] + (bias ? static_cast<uint32_t>(bias[lane]) : 0u));
    }
  }
}

bool check_gather(const cim22_gather &g, int64_t m, int64_t k) {
  if (m >= (int64_t{1} << 31) - kColumnPad || k >= (int64_t{1} << 30))
    return false;
  if (g.kind == CIM22_GATHER_ROWS)
    return m * k < (int64_t{1} << 40);
  if (g.pool_kernel < 0 || (g.pool_kernel > 0 &&
      (g.kind == CIM22_GATHER_ROWS || g.pool_stride <= 0 ||
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
  // The prepare kernel forms element offsets within an image, window
  // origins included, in 32-bit arithmetic: bound every term.
  const int64_t ps = g.pool_kernel > 0 ? g.pool_stride : 1;
  const int64_t src_h = g.pool_kernel > 0 ? g.pool_src_h : g.height;
  const int64_t src_w = g.pool_kernel > 0 ? g.pool_src_w : g.width;
  const int64_t reach =
      (static_cast<int64_t>(g.height) + g.pad_h + g.kernel_h) * ps * src_w * g.channels +
      (static_cast<int64_t>(g.width) + g.pad_w + g.kernel_w) * ps * g.channels +
      static_cast<int64_t>(g.channels + 1) * src_h * src_w +
      static_cast<int64_t>(g.pool_kernel) * (src_w + 1) * g.channels;
  if (image >= (int64_t{1} << 30) || reach >= (int64_t{1} << 30))
    return false;
  const int oh = (g.height + 2 * g.pad_h - g.kernel_h) / g.stride_h + 1;
  const int ow = (g.width + 2 * g.pad_w - g.kernel_w) / g.stride_w + 1;
  return oh == g.out_h && ow == g.out_w &&
         static_cast<int64_t>(g.batch) * oh * ow == m &&
         static_cast<int64_t>(g.channels) * g.kernel_h * g.kernel_w == k;
}

// Gathers of INT8 layers: rows, or a convolution without a fused pool whose
// bottom/right padding may differ from the top/left padding (pad_h, pad_w),
// as ONNX ConvInteger pads allow; a negative pad_bottom/pad_right means the
// same as the top/left one.
bool check_gather_int8(const cim22_gather &g, int64_t m, int64_t k, int32_t pad_bottom,
                       int32_t pad_right) {
  if (m >= (int64_t{1} << 31) - kColumnPad || k >= (int64_t{1} << 30))
    return false;
  if (g.kind == CIM22_GATHER_ROWS)
    return m * k < (int64_t{1} << 40);
  if ((g.kind != CIM22_GATHER_CONV_NCHW && g.kind != CIM22_GATHER_CONV_NHWC) ||
      g.pool_kernel != 0 || g.batch <= 0 || g.channels <= 0 || g.height <= 0 ||
      g.width <= 0 || g.kernel_h <= 0 || g.kernel_w <= 0 || g.stride_h <= 0 ||
      g.stride_w <= 0 || g.pad_h < 0 || g.pad_w < 0)
    return false;
  const int64_t pb = pad_bottom < 0 ? g.pad_h : pad_bottom;
  const int64_t pr = pad_right < 0 ? g.pad_w : pad_right;
  const int64_t span_h = g.height + g.pad_h + pb, span_w = g.width + g.pad_w + pr;
  const int64_t image = static_cast<int64_t>(g.channels) * g.height * g.width;
  const int64_t reach = (span_h + g.kernel_h) * g.width * g.channels +
                        (span_w + g.kernel_w) * g.channels +
                        static_cast<int64_t>(g.channels + 1) * g.height * g.width;
  if (image >= (int64_t{1} << 30) || reach >= (int64_t{1} << 30) || span_h < g.kernel_h ||
      span_w < g.kernel_w)
    return false;
  const int64_t oh = (span_h - g.kernel_h) / g.stride_h + 1;
  const int64_t ow = (span_w - g.kernel_w) / g.stride_w + 1;
  return oh == g.out_h && ow == g.out_w && static_cast<int64_t>(g.batch) * oh * ow == m &&
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
    if (g.kind == CIM22_GATHER_CONV_NCHW && g.pool_kernel == 0) {
      d.sC = g.height * g.width;
      d.sH = g.width;
      d.sW = 1;
      d.image = g.channels * g.height * g.width;
    } else if (g.kind == CIM22_GATHER_CONV_NCHW) {
      // Pooled (ih, iw) starts at pre-pool (ih * PS, iw * PS) of its plane.
      d.sC = g.pool_src_h * g.pool_src_w;
      d.sH = g.pool_stride * g.pool_src_w;
      d.sW = g.pool_stride;
      d.pdy = g.pool_src_w;
      d.pdx = 1;
      d.image = g.channels * g.pool_src_h * g.pool_src_w;
    } else if (g.pool_kernel == 0) {
      d.sC = 1;
      d.sH = g.width * g.channels;
      d.sW = g.channels;
      d.image = g.channels * g.height * g.width;
    } else {
      // Pooled (ih, iw) starts at pre-pool (ih * PS, iw * PS).
      d.sC = 1;
      d.sH = g.pool_stride * g.pool_src_w * g.channels;
      d.sW = g.pool_stride * g.channels;
      d.pdy = g.pool_src_w * g.channels;
      d.pdx = g.channels;
      d.image = g.channels * g.pool_src_h * g.pool_src_w;
    }
    d.div_ohw = make_fastdiv(static_cast<uint32_t>(g.out_h * g.out_w));
    d.div_ow = make_fastdiv(static_cast<uint32_t>(g.out_w));
    d.div_khw = make_fastdiv(static_cast<uint32_t>(g.kernel_h * g.kernel_w));
    d.div_kw = make_fastdiv(static_cast<uint32_t>(g.kernel_w));
  }
  return d;
}


// ---------------------------------------------------------------------------
// Legacy and None BF16 compensation (diagnostic modes, no sign split): the
// BF16-rounded signed activations and weights go through one contraction.
// Per 64-element group: prepareBF16Input (BF16Compensation.cpp:84-137) -
// non-finite inputs rejected, prealignment at the raw maximum exponent, and
// for Legacy the group scaling by 2^-scaleDelta with scaleDelta =
// max(0, Eprealigned - 240) that must leave the mantissas unchanged. Per
// (column, lane, tile): the signed dot with its i21 gate, int21ToBF16 with
// the weight exponent only in None mode, the mode's restore
// (BF16Compensation.cpp:149-164), then the Host f32 sum in tile order with a
// final BF16 rounding when T > 1 (Passes.cpp:828-857), + bias.
//
// Workspace: int8 A[m_pad][k_pad], int32 ie[T][m_pad] (the prealign
// exponent), int32 sd[T][m_pad] (Legacy scaleDelta in bits 0-7, bit 8 set
// when every prealigned mantissa of the group is -128).

constexpr int kAllMinus128 = 0x100;

template <int kMode>
__global__ void __launch_bounds__(256)
    prepare_mode_kernel(const float *__restrict__ x, Gather32 g, int T, int m_pad, int k_pad,
                        int compensation, int8_t *__restrict__ A, int32_t *__restrict__ ie,
                        int32_t *__restrict__ sd, int32_t *status) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t group = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (group >= static_cast<int64_t>(m_pad) * T)
    return;
  const int m = static_cast<int>(group / T), t = static_cast<int>(group % T);
  uint16_t bits[kTileK];
  int exp_max = 0;
  bool nonfinite = false;
#pragma unroll 1
  for (int s8 = 0; s8 < 8; ++s8) {
    const int kbeg = t * kTileK + s8 * 8;
    const Taps8 tp = make_taps8<kMode>(g, kbeg);
    float v[8];
    gather8<kMode>(x, g, tp, m, kbeg, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint16_t b = f32_to_bf16(v[e]);
      bits[s8 * 8 + e] = b;
      const int ex = (b >> 7) & 0xff;
      nonfinite |= ex == 0xff;
      exp_max = max(exp_max, ex);
    }
  }
  int8_t *dst = A + static_cast<int64_t>(m) * k_pad + t * kTileK;
  int delta = 0;
  bool all_min = true;
  if (nonfinite) {
    atomicOr(status, CIM22_STATUS_INPUT_NOT_FINITE);
    exp_max = 0;
    for (int i = 0; i < kTileK; ++i)
      dst[i] = 0;
    all_min = false;
  } else {
    for (int i = 0; i < kTileK; ++i) {
      dst[i] = prealign_element(bits[i], exp_max);
      all_min &= dst[i] == -128;
    }
    if (compensation == CIM22_BF16_LEGACY) {
      delta = max(0, exp_max - 240);
      if (delta) {
        int scaled_max = 0;
        uint16_t scaled[kTileK];
        for (int i = 0; i < kTileK; ++i) {
          scaled[i] = bf16_scalbn(bits[i], -delta);
          scaled_max = max(scaled_max, (scaled[i] >> 7) & 0xff);
        }
        bool same = scaled_max <= 240;
        for (int i = 0; i < kTileK && same; ++i)
          same = prealign_element(scaled[i], scaled_max) == dst[i];
        if (!same)
          atomicOr(status, CIM22_STATUS_LEGACY_SCALING);
        exp_max = scaled_max;
      }
    }
  }
  ie[static_cast<int64_t>(t) * m_pad + m] = exp_max;
  sd[static_cast<int64_t>(t) * m_pad + m] = delta | (all_min ? kAllMinus128 : 0);
}

// CTA tile 64 columns x 32 lanes; thread (tr, tc) owns columns tr, tr + 32
// and lanes 4 tc .. 4 tc + 3.
__global__ void __launch_bounds__(256)
    mode_simt_kernel(const int8_t *__restrict__ A, const int32_t *__restrict__ ie,
                     const int32_t *__restrict__ sd, int m_pad, const int8_t *__restrict__ B,
                     const int32_t *__restrict__ exB, const int32_t *__restrict__ wmin,
                     int n_pad, int k_pad, int T, int M, int N, int compensation,
                     const float *__restrict__ bias, const float *__restrict__ post_scale,
                     const float *__restrict__ post_shift, int act, int out_pixels,
                     float *__restrict__ y, int32_t *status) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ __align__(16) int8_t As[64][kRowStride];
  __shared__ __align__(16) int8_t Bs[32][kRowStride];
  __shared__ int sIe[64], sSd[64], sEw[32], sMin[2];
  const int tid = static_cast<int>(threadIdx.x);
  const int tr = tid / 8, tc = tid % 8;
  const int m0 = static_cast<int>(blockIdx.x) * 64, n0 = static_cast<int>(blockIdx.y) * 32;
  float acc[2][4];
  for (int t = 0; t < T; ++t) {
    for (int i = tid; i < 64 * 4; i += 256) {
      const int r = i / 4, c = i % 4;
      *reinterpret_cast<int4 *>(&As[r][c * 16]) = *reinterpret_cast<const int4 *>(
          A + static_cast<int64_t>(m0 + r) * k_pad + t * kTileK + c * 16);
    }
    for (int i = tid; i < 32 * 4; i += 256) {
      const int r = i / 4, c = i % 4;
      *reinterpret_cast<int4 *>(&Bs[r][c * 16]) = *reinterpret_cast<const int4 *>(
          B + static_cast<int64_t>(n0 + r) * k_pad + t * kTileK + c * 16);
    }
    if (tid < 64) {
      sIe[tid] = ie[static_cast<int64_t>(t) * m_pad + m0 + tid];
      sSd[tid] = sd[static_cast<int64_t>(t) * m_pad + m0 + tid];
    } else if (tid < 96) {
      sEw[tid - 64] = exB[static_cast<int64_t>(t) * n_pad + n0 + tid - 64];
    } else if (tid < 98) {
      // Some lane of this 16-lane weight tile is all -128 (Legacy validation).
      sMin[tid - 96] = wmin[static_cast<int64_t>(t) * (n_pad / 16) + n0 / 16 + tid - 96];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = tr + 32 * r;
      const int ie_r = sIe[row], sd_r = sSd[row];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int lane = 4 * tc + c;
        int p = 0;
#pragma unroll
        for (int q = 0; q < 16; ++q)
          p = __dp4a(*reinterpret_cast<const int *>(&As[row][q * 4]),
                     *reinterpret_cast<const int *>(&Bs[lane][q * 4]), p);
        const bool live = m0 + row < M && n0 + lane < N;
        if (compensation == CIM22_BF16_LEGACY && (sd_r & kAllMinus128) && sMin[lane / 16]) {
          // validateBF16Group rejects the Work before its dots are formed.
          if (live)
            atomicOr(status, CIM22_STATUS_LEGACY_I21);
          p = 0;
        } else if (p < -(1 << 20) || p >= (1 << 20)) {
          if (live)
            atomicOr(status, CIM22_STATUS_I21_RANGE);
          p = 0;
        }
        const int ew = sEw[lane];
        const uint16_t chip =
            int21_to_bf16(p, compensation == CIM22_BF16_NONE ? ew : 0, ie_r);
        uint16_t tile = chip;
        if (compensation == CIM22_BF16_LEGACY) {
          int error = 0;
          if (!compensate(chip, ew + (sd_r & 0xff) - 133, tile, error)) {
            if (live)
              atomicOr(status, error == 1 ? CIM22_STATUS_CHIP_NOT_FINITE
                                          : CIM22_STATUS_TILE_OVERFLOW);
            tile = 0;
          }
        }
        const float v = bf16_to_f32(tile);
        acc[r][c] = t == 0 ? v : __fadd_rn(acc[r][c], v);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = m0 + tr + 32 * r;
    if (row >= M)
      continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int lane = n0 + 4 * tc + c;
      if (lane >= N)
        continue;
      float out = T > 1 ? bf16_to_f32(f32_to_bf16(acc[r][c])) : acc[r][c];
      if (bias != nullptr)
        out = __fadd_rn(out, bias[lane]);
      if (post_scale != nullptr)
        out = __fmaf_rn(out, post_scale[lane], post_shift[lane]);
      out = apply_act(out, act);
      if (out_pixels > 0) {
        const int image = row / out_pixels;
        y[(static_cast<int64_t>(image) * N + lane) * out_pixels + (row - image * out_pixels)] =
            out;
      } else {
        y[static_cast<int64_t>(row) * N + lane] = out;
      }
    }
  }
}
} // namespace

// Host-side BF16 weight preparation: split, RNE, prealign per lane and K tile.
static void prepare_bf16_weights(const float *w, int64_t n, int64_t k,
                                 int64_t n_pad, int64_t k_pad, int64_t T,
                                 std::vector<int8_t> &mant,
                                 std::vector<int32_t> &exps,
                                 std::vector<uint16_t> &operands, int32_t &ex_lo,
                                 int32_t &ex_hi) {
  mant.assign(2 * n_pad * k_pad, 0);
  exps.assign(2 * T * n_pad + (n_pad / 32) * T * 4 + 4 * T * n_pad +
                  T * (n_pad / 32) * tc::kScaleBlockWords,
              127);
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
  // Per tile and 32-lane block: the range of the weight exponents of both
  // signs, which decides the tensor-core epilogue's exact-FMA window.
  int32_t *ranges = exps.data() + 2 * T * n_pad;
  for (int64_t t = 0; t < T; ++t)
    for (int64_t nb = 0; nb < n_pad / 32; ++nb) {
      int lo = 1 << 30, hi = -(1 << 30);
      for (int b = 0; b < 2; ++b)
        for (int64_t lane = nb * 32; lane < nb * 32 + 32; ++lane) {
          const int e = exps[(b * T + t) * n_pad + lane];
          lo = std::min(lo, e);
          hi = std::max(hi, e);
        }
      // With them, the block's window of activation group exponents Ex for
      // the epilogue's exact fast restore (Ex + 16 - kScaleShift and
      // Ew - 133 + kScaleShift normal, Ex + Ew in [140, 374]; empty when an
      // exponent exceeds 260 - kScaleShift).
      constexpr int X = tc::kScaleShift;
      int32_t *r = ranges + (t * (n_pad / 32) + nb) * 4;
      r[0] = lo;
      r[1] = hi;
      r[2] = std::max(X + 7, 140 - lo);
      r[3] = hi <= 260 - X ? std::min(X + 111, 374 - hi) : -1;
    }
  // The weight scales 2^(Ew - 133) as f32 bit patterns (exact: Ew - 133 lies
  // in [-133, 121], inside f32's normal and subnormal range), then the
  // tensor-core epilogue's 2^(Ew - 133 + kScaleShift) (normal for
  // Ew <= 260 - kScaleShift; tiles with a larger exponent take the exact
  // integer restore, so the clamp is never used).
  int32_t *scales = ranges + (n_pad / 32) * T * 4;
  int32_t *tc_scales = scales + 2 * T * n_pad;
  for (int64_t i = 0; i < 2 * T * n_pad; ++i) {
    const float f = std::ldexp(1.0f, exps[i] - 133);
    std::memcpy(&scales[i], &f, 4);
    const float g = std::ldexp(1.0f, std::min(exps[i] - 133 + tc::kScaleShift, 127));
    std::memcpy(&tc_scales[i], &g, 4);
  }
  // The same epilogue scales and windows per (K tile, 32-lane block) in one
  // record {Wp scales [32], Wn scales [32], range [4]}, so that the
  // tensor-core kernel fetches a tile's weight data with one bulk copy.
  int32_t *blocks = tc_scales + 2 * T * n_pad;
  for (int64_t t = 0; t < T; ++t)
    for (int64_t nb = 0; nb < n_pad / 32; ++nb) {
      int32_t *rec = blocks + (t * (n_pad / 32) + nb) * tc::kScaleBlockWords;
      for (int b = 0; b < 2; ++b)
        std::memcpy(rec + 32 * b, tc_scales + (b * T + t) * n_pad + nb * 32, 32 * 4);
      std::memcpy(rec + 64, ranges + (t * (n_pad / 32) + nb) * 4, 4 * 4);
    }
  // Scaled BF16 operands b * 2^(Ew - 133) (exact: b has at most 7 significant
  // bits and the value is normal for Ew >= kOperandEwMin), for layers of at
  // least kOperandMinLanes lanes whose lanes with a nonzero mantissa all have
  // an admitted exponent; the activation window then follows from the
  // extreme exponents of those lanes.
  operands.clear();
  ex_lo = 1;
  ex_hi = 0;
  int ew_min = 1 << 30, ew_max = -(1 << 30);
  for (int b = 0; b < 2; ++b)
    for (int64_t t = 0; t < T; ++t)
      for (int64_t lane = 0; lane < n; ++lane) {
        const int8_t *src = mant.data() + (b * n_pad + lane) * k_pad + t * kTileK;
        if (std::any_of(src, src + kTileK, [](int8_t v) { return v != 0; })) {
          const int e = exps[(b * T + t) * n_pad + lane];
          ew_min = std::min(ew_min, e);
          ew_max = std::max(ew_max, e);
        }
      }
  if (ew_min > ew_max) { // no nonzero weight: every dot is 0
    ew_min = kOperandEwMin;
    ew_max = kOperandEwMin;
  }
  const int lo = std::max(kOperandExMin, 140 - ew_min);
  const int hi = std::min(kOperandExMax, 374 - ew_max);
  if (n < kOperandMinLanes || ew_min < kOperandEwMin || ew_max > kOperandEwMax || lo > hi)
    return;
  operands.assign(2 * n_pad * k_pad, 0);
  for (int b = 0; b < 2; ++b)
    for (int64_t lane = 0; lane < n; ++lane)
      for (int64_t t = 0; t < T; ++t) {
        const int e = exps[(b * T + t) * n_pad + lane];
        const int64_t off = (b * n_pad + lane) * k_pad + t * kTileK;
        for (int i = 0; i < kTileK; ++i)
          if (mant[off + i] != 0)
            operands[off + i] = f32_to_bf16(std::ldexp(static_cast<float>(mant[off + i]), e - 133));
      }
  ex_lo = lo;
  ex_hi = hi;
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
  std::vector<uint16_t> operands;
  prepare_bf16_weights(weight, n, k, layer->n_pad, layer->k_pad, layer->tiles,
                       mant, exps, operands, layer->ex_lo, layer->ex_hi);
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice") ||
      !cuda_ok(cudaMalloc(&layer->weights, mant.size()), "cudaMalloc") ||
      !cuda_ok(cudaMalloc(&layer->exponents, exps.size() * sizeof(int32_t)),
               "cudaMalloc") ||
      !cuda_ok(cudaMemcpy(layer->weights, mant.data(), mant.size(),
                          cudaMemcpyHostToDevice),
               "cudaMemcpy") ||
      !cuda_ok(cudaMemcpy(layer->exponents, exps.data(),
                          exps.size() * sizeof(int32_t), cudaMemcpyHostToDevice),
               "cudaMemcpy") ||
      (!operands.empty() &&
       (!cuda_ok(cudaMalloc(&layer->operands, operands.size() * sizeof(uint16_t)),
                 "cudaMalloc") ||
        !cuda_ok(cudaMemcpy(layer->operands, operands.data(),
                            operands.size() * sizeof(uint16_t), cudaMemcpyHostToDevice),
                 "cudaMemcpy")))) {
    copy_error(last_error(), error, error_capacity);
    cim22_cuda_layer_destroy(layer);
    return nullptr;
  }
  return layer;
}

cim22_cuda_layer *cim22_cuda_layer_create_bf16_mode(int device, const float *weight,
                                                    int64_t n, int64_t k, int32_t compensation,
                                                    char *error, size_t error_capacity) {
  if (compensation == CIM22_BF16_SIGN_SPLIT)
    return cim22_cuda_layer_create_bf16(device, weight, n, k, error, error_capacity);
  if (compensation != CIM22_BF16_LEGACY && compensation != CIM22_BF16_NONE) {
    copy_error("BF16 compensation must be sign-split, legacy or none", error, error_capacity);
    return nullptr;
  }
  if (!weight || n <= 0 || k <= 0) {
    copy_error("invalid CIM layer shape", error, error_capacity);
    return nullptr;
  }
  for (int64_t i = 0; i < n * k; ++i)
    if (!std::isfinite(weight[i])) {
      copy_error("BF16 correction requires finite fixed weights", error, error_capacity);
      return nullptr;
    }
  auto *layer = new cim22_cuda_layer();
  layer->device = device;
  layer->bf16 = true;
  layer->mode = compensation;
  layer->n = n;
  layer->k = k;
  layer->n_pad = round_up(n, kLanePad);
  layer->k_pad = round_up(k, kTileK);
  layer->tiles = layer->k_pad / kTileK;
  const int64_t T = layer->tiles, n_pad = layer->n_pad, k_pad = layer->k_pad;
  // Signed BF16 weights prealigned per (lane, K tile) at the lane's raw
  // maximum exponent (prealignBF16WeightTile, BF16Support.cpp:56-70), then
  // per (K tile, 16-lane tile) whether some lane is all -128.
  std::vector<int8_t> mant(n_pad * k_pad, 0);
  std::vector<int32_t> exps(T * n_pad + T * (n_pad / 16), 0);
  uint16_t group[kTileK];
  for (int64_t lane = 0; lane < n; ++lane)
    for (int64_t t = 0; t < T; ++t) {
      int exp_max = 0;
      for (int i = 0; i < kTileK; ++i) {
        const int64_t col = t * kTileK + i;
        group[i] = col < k ? f32_to_bf16(weight[lane * k + col]) : 0;
        exp_max = std::max(exp_max, (group[i] >> 7) & 0xff);
      }
      bool all_min = true;
      for (int i = 0; i < kTileK; ++i) {
        const int8_t v = prealign_element(group[i], exp_max);
        mant[lane * k_pad + t * kTileK + i] = v;
        all_min &= v == -128;
      }
      exps[t * n_pad + lane] = exp_max;
      if (all_min)
        exps[T * n_pad + t * (n_pad / 16) + lane / 16] = 1;
    }
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice") ||
      !cuda_ok(cudaMalloc(&layer->weights, mant.size()), "cudaMalloc") ||
      !cuda_ok(cudaMalloc(&layer->exponents, exps.size() * sizeof(int32_t)), "cudaMalloc") ||
      !cuda_ok(cudaMemcpy(layer->weights, mant.data(), mant.size(), cudaMemcpyHostToDevice),
               "cudaMemcpy") ||
      !cuda_ok(cudaMemcpy(layer->exponents, exps.data(), exps.size() * sizeof(int32_t),
                          cudaMemcpyHostToDevice),
               "cudaMemcpy")) {
    copy_error(last_error(), error, error_capacity);
    cim22_cuda_layer_destroy(layer);
    return nullptr;
  }
  return layer;
}

int32_t cim22_cuda_layer_compensation(const cim22_cuda_layer *layer) {
  return layer ? layer->mode : -1;
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
  if (layer->operands)
    cudaFree(layer->operands);
  delete layer;
}

int cim22_cuda_layer_range_safe(const cim22_cuda_layer *layer) {
  return layer && layer->range_safe ? 1 : 0;
}
int cim22_cuda_layer_bf16_operands(const cim22_cuda_layer *layer) {
  return layer && layer->operands ? 1 : 0;
}
int64_t cim22_cuda_layer_n(const cim22_cuda_layer *layer) { return layer ? layer->n : -1; }
int64_t cim22_cuda_layer_k(const cim22_cuda_layer *layer) { return layer ? layer->k : -1; }

size_t cim22_cuda_layer_workspace_bf16(const cim22_cuda_layer *layer,
                                       int64_t m, int32_t branches) {
  if (!layer || m <= 0)
    return 0;
  const int64_t m_pad = round_up(m, kColumnPad);
  if (layer->mode != CIM22_BF16_SIGN_SPLIT)
    return static_cast<size_t>(round_up(m_pad * layer->k_pad, 256) +
                               2 * layer->tiles * m_pad * 4);
  const int64_t ab = branches == 2 ? 1 : 2;
  // Room for the BF16 operand values wherever the layer admits them.
  const int64_t elem = layer->operands ? 2 : 1;
  const int64_t a_bytes = round_up(ab * m_pad * layer->k_pad * elem, 256);
  return static_cast<size_t>(a_bytes + ab * layer->tiles * m_pad * 4);
}

size_t cim22_cuda_layer_workspace_int8(const cim22_cuda_layer *layer, int64_t m) {
  if (!layer || m <= 0)
    return 0;
  return static_cast<size_t>(round_up(m, kColumnPad) * layer->k_pad);
}

// The prepared-column format of a sign-split call, decided the same way by
// the prepare and the contraction: scaled BF16 operand values for the
// tensor-core contraction with BF16 operands where the layer holds BF16
// operands (at least kOperandMinLanes lanes, weight exponents in the operand
// range) and that kernel runs (sm_100, a 16-byte aligned workspace); int8
// mantissas otherwise.
static bool bf16_operands(const cim22_cuda_layer *layer, const void *workspace) {
  return layer->operands != nullptr && layer->mode == CIM22_BF16_SIGN_SPLIT && layer->n > 8 &&
         (reinterpret_cast<uintptr_t>(workspace) & 15) == 0 && tc::signsplit_available();
}

// Byte offset of the group exponents in a sign-split workspace.
static int64_t exponent_offset(const cim22_cuda_layer *layer, int64_t m_pad, int ab, bool b16) {
  return round_up(ab * m_pad * layer->k_pad * (b16 ? 2 : 1), 256);
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
  const bool b16 = bf16_operands(layer, workspace);
  int32_t *ex = reinterpret_cast<int32_t *>(static_cast<char *>(workspace) +
                                            exponent_offset(layer, m_pad, ab, b16));
  const int win_lo = layer->ex_lo, win_hi = layer->ex_hi;
  const Gather32 dg = to_device_gather(g, m, layer->k, x);
  if (layer->mode != CIM22_BF16_SIGN_SPLIT) {
    // Legacy / None: one thread per (column, K tile) group.
    int32_t *ie = reinterpret_cast<int32_t *>(static_cast<char *>(workspace) +
                                              round_up(m_pad * layer->k_pad, 256));
    int32_t *sd = ie + T * m_pad;
    const unsigned blocks = static_cast<unsigned>((m_pad * T + 255) / 256);
    const int mode = g.kind == CIM22_GATHER_ROWS ? kPrepRows
                     : g.pool_kernel > 0         ? kPrepConvPool
                                                 : kPrepConv;
    auto go = [&](auto kernel) {
      launch_pdl(kernel, blocks, 256, 0, s, x, dg, T, static_cast<int>(m_pad),
                 static_cast<int>(layer->k_pad), layer->mode, A, ie, sd, status);
    };
    if (mode == kPrepRows)
      go(prepare_mode_kernel<kPrepRows>);
    else if (mode == kPrepConv)
      go(prepare_mode_kernel<kPrepConv>);
    else
      go(prepare_mode_kernel<kPrepConvPool>);
    return cuda_ok(cudaGetLastError(), "prepare launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
  }
  // Convolutions whose 256-column blocks cover whole output rows or whole
  // images gather from a TMA-staged window in shared memory.
  BoxGather box{};
  if (tc::signsplit_available() && plan_box_gather(dg, x, T, box)) {
    CUtensorMap map, omap;
    const int n_images = static_cast<int>(g.batch);
    if (tc::encode_nchw_box(&map, x, dg.W, dg.H, dg.C, n_images, box.wb, box.hb, box.cb,
                            box.nb) &&
        tc::encode_prepared_store(&omap, A, static_cast<uint64_t>(ab) * m_pad, layer->k_pad,
                                  b16)) {
      const int items = static_cast<int>((m_pad + 255) / 256 * T);
      const size_t smem = box_smem(box, dg.KH * dg.KW, ab, b16);
      // Runs of items per block: up to eight, keeping at least four waves.
      auto launch = [&](auto kernel) {
        int per_sm = 0;
        if (!cuda_ok(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)),
                     "prepare shared memory") ||
            !cuda_ok(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, smem),
                     "prepare occupancy") ||
            per_sm < 1)
          return false;
        const int64_t resident = int64_t{device_sms()} * per_sm;
        const int run = static_cast<int>(std::clamp<int64_t>(items / (4 * resident), 1, 8));
        const int grid = (items + run - 1) / run;
        launch_pdl(kernel, dim3(static_cast<unsigned>(grid)), 256, smem, s, map, omap, dg, box,
                   make_fastdiv(static_cast<uint32_t>(T)), T, items, run, static_cast<int>(m_pad),
                   static_cast<int>(layer->k_pad), A, ex, status, win_lo, win_hi);
        return true;
      };
      const bool launched =
          ab == 1 ? (b16 ? launch(prepare_nchw_box_kernel<1, true>)
                         : launch(prepare_nchw_box_kernel<1, false>))
                  : (b16 ? launch(prepare_nchw_box_kernel<2, true>)
                         : launch(prepare_nchw_box_kernel<2, false>));
      return launched && cuda_ok(cudaGetLastError(), "prepare launch") ? 0
                                                                      : CIM22_STATUS_BAD_ARGUMENT;
    }
  }
  // The thread-per-group NCHW kernel serves convolutions over enough columns
  // to fill the GPU (measured 1.3-1.6x faster than the kernel below on
  // ResNet-18 and the event-frame CNN, whose loads it coalesces); short column
  // counts (a flatten -> Linear over a small batch) go to the
  // eight-threads-per-group kernel.
  if (g.kind == CIM22_GATHER_CONV_NCHW && (g.pool_kernel == 0 || g.pool_kernel == 2) &&
      g.kernel_h <= kTapMasks && g.kernel_w <= kTapMasks &&
      ((m_pad + 255) / 256) * T >= 148 * 2) {
    // Chunks of 256 columns per block: as many as (up to four) still give
    // four waves of blocks on 148 SMs, to spread the block's tap table.
    const int64_t chunks = (m_pad + 255) / 256;
    int per_block = 4;
    while (per_block > 1 && ((chunks + per_block - 1) / per_block) * T < 148 * 4 * 4)
      per_block /= 2;
    const int64_t groups = (chunks + per_block - 1) / per_block;
    const FastDiv div_chunks = make_fastdiv(static_cast<uint32_t>(groups));
    const unsigned blocks = static_cast<unsigned>(groups * T);
    auto launch = [&](auto kernel) {
      launch_pdl(kernel, blocks, 256, 0, s, x, dg, div_chunks, T, per_block,
                 static_cast<int>(m_pad), static_cast<int>(layer->k_pad), A, ex, status, win_lo,
                 win_hi);
    };
    const bool pool = g.pool_kernel > 0;
    if (ab == 1) {
      if (b16)
        launch(pool ? prepare_nchw_kernel<1, true, true> : prepare_nchw_kernel<1, false, true>);
      else
        launch(pool ? prepare_nchw_kernel<1, true, false> : prepare_nchw_kernel<1, false, false>);
    } else {
      if (b16)
        launch(pool ? prepare_nchw_kernel<2, true, true> : prepare_nchw_kernel<2, false, true>);
      else
        launch(pool ? prepare_nchw_kernel<2, true, false> : prepare_nchw_kernel<2, false, false>);
    }
    return cuda_ok(cudaGetLastError(), "prepare launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
  }
  // Columns per group thread: as many as still give four waves of 256-thread
  // blocks on a B200 (148 SMs, four resident blocks each).
  int cols = 4;
  while (cols > 1 && ((m_pad + 32 * cols - 1) / (32 * cols)) * T < 148 * 4 * 4)
    cols /= 2;
  const int64_t chunks = (m_pad + 32 * cols - 1) / (32 * cols);
  const unsigned blocks = static_cast<unsigned>(chunks * T);
  const FastDiv div_chunks = make_fastdiv(static_cast<uint32_t>(chunks));
  const int mode = g.kind == CIM22_GATHER_ROWS ? kPrepRows
                   : g.pool_kernel > 0         ? kPrepConvPool
                                               : kPrepConv;
  auto launch = [&](auto kernel) {
    launch_pdl(kernel, blocks, 256, 0, s, x, dg, div_chunks, T, cols, static_cast<int>(m_pad),
               static_cast<int>(layer->k_pad), A, ex, status, win_lo, win_hi);
  };
  auto pick = [&](auto ab_tag, auto b16_tag) {
    constexpr int kAB = decltype(ab_tag)::value;
    constexpr bool kB = decltype(b16_tag)::value;
    launch(mode == kPrepRows   ? prepare_kernel<kAB, kPrepRows, kB>
           : mode == kPrepConv ? prepare_kernel<kAB, kPrepConv, kB>
                               : prepare_kernel<kAB, kPrepConvPool, kB>);
  };
  if (ab == 1)
    b16 ? pick(std::integral_constant<int, 1>{}, std::true_type{})
        : pick(std::integral_constant<int, 1>{}, std::false_type{});
  else
    b16 ? pick(std::integral_constant<int, 2>{}, std::true_type{})
        : pick(std::integral_constant<int, 2>{}, std::false_type{});
  return cuda_ok(cudaGetLastError(), "prepare launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

// Legacy / None layers: the CUDA-core contraction over the mode's workspace.
static int contract_mode(const cim22_cuda_layer *layer, int64_t m, int64_t out_pixels,
                         const float *bias, const float *post_scale, const float *post_shift,
                         int32_t activation, float *y, const void *workspace, int32_t *status,
                         cudaStream_t s) {
  const int64_t m_pad = round_up(m, kColumnPad);
  const int T = static_cast<int>(layer->tiles);
  const int8_t *A = static_cast<const int8_t *>(workspace);
  const int32_t *ie = reinterpret_cast<const int32_t *>(
      static_cast<const char *>(workspace) + round_up(m_pad * layer->k_pad, 256));
  const int32_t *sd = ie + T * m_pad;
  const int32_t *wmin = layer->exponents + T * layer->n_pad;
  const dim3 grid(static_cast<unsigned>(m_pad / 64), static_cast<unsigned>((layer->n + 31) / 32));
  launch_pdl(mode_simt_kernel, grid, 256, 0, s, A, ie, sd, static_cast<int>(m_pad),
             layer->weights, layer->exponents, wmin, static_cast<int>(layer->n_pad),
             static_cast<int>(layer->k_pad), T, static_cast<int>(m), static_cast<int>(layer->n),
             layer->mode, bias, post_scale, post_shift, activation,
             static_cast<int>(out_pixels), y, status);
  return cuda_ok(cudaGetLastError(), "mode contraction launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

int cim22_cuda_layer_contract_bf16_res(const cim22_cuda_layer *layer, int64_t m,
                                       int64_t out_pixels, const float *bias,
                                       const float *post_scale, const float *post_shift,
                                       const float *residual, int32_t activation,
                                       int32_t branches, float *y, const void *workspace,
                                       size_t workspace_bytes, int32_t *status, void *stream) {
  if (!layer || !layer->bf16 || !y || !status || m <= 0 ||
      (branches != 2 && branches != 4) || activation < 0 || activation > 2 ||
      !workspace || out_pixels < 0 || (out_pixels > 0 && m % out_pixels != 0) ||
      (post_scale == nullptr) != (post_shift == nullptr) ||
      (residual != nullptr && layer->mode != CIM22_BF16_SIGN_SPLIT) ||
      workspace_bytes < cim22_cuda_layer_workspace_bf16(layer, m, branches)) {
    set_last_error("invalid arguments to cim22_cuda_layer_contract_bf16");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  auto s = static_cast<cudaStream_t>(stream);
  if (layer->mode != CIM22_BF16_SIGN_SPLIT)
    return contract_mode(layer, m, out_pixels, bias, post_scale, post_shift, activation, y,
                         workspace, status, s);
  const int64_t m_pad = round_up(m, kColumnPad);
  const int ab = branches == 2 ? 1 : 2;
  const int T = static_cast<int>(layer->tiles);
  const int8_t *A = static_cast<const int8_t *>(workspace);
  const bool b16 = bf16_operands(layer, workspace);
  const int32_t *ex = reinterpret_cast<const int32_t *>(static_cast<const char *>(workspace) +
                                                        exponent_offset(layer, m_pad, ab, b16));
  if (b16) {
    // The prepare wrote BF16 operand values: only the contraction with BF16
    // operands reads them.
    if (!tc::launch_signsplit_b16(reinterpret_cast<const uint16_t *>(A), ex, m_pad,
                                  layer->operands, layer->exponents, layer->n_pad, layer->k_pad, T,
                                  m, layer->n, layer->ex_lo, layer->ex_hi, bias, post_scale,
                                  post_shift, residual, activation, ab, out_pixels, y, status,
                                  s)) {
      set_last_error("cim22_cuda_layer_contract_bf16: the contraction with BF16 operands "
                     "did not launch");
      return CIM22_STATUS_BAD_ARGUMENT;
    }
    return cuda_ok(cudaGetLastError(), "signsplit launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
  }
  if (tc::signsplit_available() &&
      tc::launch_signsplit(A, ex, m_pad, layer->weights, layer->exponents,
                           layer->n_pad, layer->k_pad, T, m, layer->n, bias, post_scale,
                           post_shift, residual, activation, ab, out_pixels, y, status, s))
    return cuda_ok(cudaGetLastError(), "signsplit launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
  if (ab == 1)
    launch_signsplit_simt<1>(A, ex, m_pad, layer->weights, layer->exponents, layer->n_pad,
                             layer->k_pad, T, m, layer->n, bias, post_scale, post_shift,
                             residual, activation, out_pixels, y, status, s,
                             static_cast<int>(layer->k));
  else
    launch_signsplit_simt<2>(A, ex, m_pad, layer->weights, layer->exponents, layer->n_pad,
                             layer->k_pad, T, m, layer->n, bias, post_scale, post_shift,
                             residual, activation, out_pixels, y, status, s,
                             static_cast<int>(layer->k));
  return cuda_ok(cudaGetLastError(), "signsplit launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

int cim22_cuda_layer_contract_bf16_peers(const cim22_cuda_layer *layer, int64_t m,
                                         const float *bias, int32_t activation,
                                         int32_t branches, const cim22_peer_outputs *peers,
                                         const void *workspace, size_t workspace_bytes,
                                         int32_t *status, void *stream) {
  if (!layer || !layer->bf16 || !peers || !status || m <= 0 ||
      (branches != 2 && branches != 4) || activation < 0 || activation > 2 || !workspace ||
      workspace_bytes < cim22_cuda_layer_workspace_bf16(layer, m, branches)) {
    set_last_error("invalid arguments to cim22_cuda_layer_contract_bf16_peers");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  if (!bf16_operands(layer, workspace)) {
    set_last_error("cim22_cuda_layer_contract_bf16_peers: the layer does not take BF16 "
                   "operands (see cim22_cuda_layer_bf16_operands)");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  const int64_t m_pad = round_up(m, kColumnPad);
  const int ab = branches == 2 ? 1 : 2;
  const uint16_t *A = static_cast<const uint16_t *>(workspace);
  const int32_t *ex = reinterpret_cast<const int32_t *>(static_cast<const char *>(workspace) +
                                                        exponent_offset(layer, m_pad, ab, true));
  if (!tc::launch_signsplit_b16(A, ex, m_pad, layer->operands, layer->exponents, layer->n_pad,
                                layer->k_pad, static_cast<int>(layer->tiles), m, layer->n,
                                layer->ex_lo, layer->ex_hi, bias, nullptr, nullptr, nullptr,
                                activation, ab, 0, nullptr, status,
                                static_cast<cudaStream_t>(stream), peers)) {
    set_last_error("cim22_cuda_layer_contract_bf16_peers: invalid peer outputs (1 to 8 "
                   "ranks, lanes within the layer, columns within row_stride)");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  return cuda_ok(cudaGetLastError(), "signsplit launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

int cim22_cuda_layer_contract_bf16_ex(const cim22_cuda_layer *layer, int64_t m,
                                      int64_t out_pixels, const float *bias,
                                      const float *post_scale, const float *post_shift,
                                      int32_t activation, int32_t branches, float *y,
                                      const void *workspace, size_t workspace_bytes,
                                      int32_t *status, void *stream) {
  return cim22_cuda_layer_contract_bf16_res(layer, m, out_pixels, bias, post_scale, post_shift,
                                            nullptr, activation, branches, y, workspace,
                                            workspace_bytes, status, stream);
}

int cim22_cuda_layer_contract_bf16(const cim22_cuda_layer *layer, int64_t m,
                                   const float *bias, int32_t activation,
                                   int32_t branches, float *y,
                                   const void *workspace,
                                   size_t workspace_bytes, int32_t *status,
                                   void *stream) {
  return cim22_cuda_layer_contract_bf16_ex(layer, m, 0, bias, nullptr, nullptr, activation,
                                           branches, y, workspace, workspace_bytes, status,
                                           stream);
}

int cim22_cuda_layer_forward_bf16_ex(const cim22_cuda_layer *layer, const float *x,
                                     const cim22_gather *gather, int64_t m, int64_t out_pixels,
                                     const float *bias, const float *post_scale,
                                     const float *post_shift, int32_t activation,
                                     int32_t branches, float *y, void *workspace,
                                     size_t workspace_bytes, int32_t *status, void *stream) {
  if (!y || activation < 0 || activation > 2 || out_pixels < 0 ||
      (out_pixels > 0 && m % out_pixels != 0) ||
      (post_scale == nullptr) != (post_shift == nullptr)) {
    set_last_error("invalid arguments to cim22_cuda_layer_forward_bf16");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  if (cim22_cuda_layer_fused_forward(layer)) {
    // Narrow layer: one CUDA-core kernel gathers, prealigns and contracts.
    cim22_gather rows{};
    rows.kind = CIM22_GATHER_ROWS;
    const cim22_gather &g = gather ? *gather : rows;
    const int64_t m_pad = round_up(m, kColumnPad);
    const int T = static_cast<int>(layer->tiles);
    if (!x || !status || m <= 0 || (branches != 2 && branches != 4) ||
        !check_gather(g, m, layer->k) || !workspace ||
        workspace_bytes < cim22_cuda_layer_workspace_bf16(layer, m, branches) ||
        m_pad * T * kGroupThreads >= (int64_t{1} << 31)) {
      set_last_error("invalid arguments to cim22_cuda_layer_forward_bf16");
      return CIM22_STATUS_BAD_ARGUMENT;
    }
    auto s = static_cast<cudaStream_t>(stream);
    const Gather32 dg = to_device_gather(g, m, layer->k, x);
    const int mode = g.kind == CIM22_GATHER_ROWS ? kPrepRows
                     : g.pool_kernel > 0         ? kPrepConvPool
                                                 : kPrepConv;
    if (direct_layer(layer) && mode != kPrepConvPool &&
        direct_preferred(layer, branches, out_pixels)) {
      auto direct = [&](auto ab_tag, auto mode_tag) {
        launch_signsplit_direct<decltype(ab_tag)::value, decltype(mode_tag)::value>(
            layer, x, dg, m, bias, post_scale, post_shift, activation, out_pixels, y, status,
            s);
      };
      using R = std::integral_constant<int, kPrepRows>;
      using C = std::integral_constant<int, kPrepConv>;
      using B1 = std::integral_constant<int, 1>;
      using B2 = std::integral_constant<int, 2>;
      if (branches == 2) {
        if (mode == kPrepRows) direct(B1{}, R{});
        else direct(B1{}, C{});
      } else {
        if (mode == kPrepRows) direct(B2{}, R{});
        else direct(B2{}, C{});
      }
      return cuda_ok(cudaGetLastError(), "fused layer launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
    }
    if (layer->n <= 16 && layer->tiles <= 2 && m < kFusedSimtColumns) {
    // The CUDA-core contraction builds its own activation tiles.
    auto launch = [&](auto ab_tag, auto mode_tag) {
      constexpr int kAB = decltype(ab_tag)::value, kMode = decltype(mode_tag)::value;
      launch_signsplit_simt<kAB, kMode>(nullptr, nullptr, m_pad, layer->weights,
                                        layer->exponents, layer->n_pad, layer->k_pad, T, m,
                                        layer->n, bias, post_scale, post_shift, nullptr,
                                        activation, out_pixels, y, status, s,
                                        static_cast<int>(layer->k), x, dg);
    };
    using R = std::integral_constant<int, kPrepRows>;
    using C = std::integral_constant<int, kPrepConv>;
    using P = std::integral_constant<int, kPrepConvPool>;
    using B1 = std::integral_constant<int, 1>;
    using B2 = std::integral_constant<int, 2>;
    if (branches == 2) {
      if (mode == kPrepRows) launch(B1{}, R{});
      else if (mode == kPrepConv) launch(B1{}, C{});
      else launch(B1{}, P{});
    } else {
      if (mode == kPrepRows) launch(B2{}, R{});
      else if (mode == kPrepConv) launch(B2{}, C{});
      else launch(B2{}, P{});
    }
    return cuda_ok(cudaGetLastError(), "fused layer launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
    }
    // Other one-tile layers: the prepare and contract kernels below.
  }
  const int rc = cim22_cuda_layer_prepare_bf16(layer, x, gather, m, branches, workspace,
                                               workspace_bytes, status, stream);
  if (rc)
    return rc;
  return cim22_cuda_layer_contract_bf16_ex(layer, m, out_pixels, bias, post_scale, post_shift,
                                           activation, branches, y, workspace, workspace_bytes,
                                           status, stream);
}

int cim22_cuda_layer_fused_forward(const cim22_cuda_layer *layer) {
  return layer && layer->bf16 && layer->mode == CIM22_BF16_SIGN_SPLIT &&
                 (direct_layer(layer) || (layer->n <= 16 && layer->tiles <= 2))
             ? 1
             : 0;
}

int cim22_cuda_layer_forward_bf16(const cim22_cuda_layer *layer, const float *x,
                                  const cim22_gather *gather, int64_t m,
                                  const float *bias, int32_t activation,
                                  int32_t branches, float *y, void *workspace,
                                  size_t workspace_bytes, int32_t *status,
                                  void *stream) {
  return cim22_cuda_layer_forward_bf16_ex(layer, x, gather, m, 0, bias, nullptr, nullptr,
                                          activation, branches, y, workspace, workspace_bytes,
                                          status, stream);
}

int cim22_cuda_layer_forward_int8_ex(const cim22_cuda_layer *layer, const int8_t *x,
                                     const cim22_gather *gather, int64_t m, int32_t pad_bottom,
                                     int32_t pad_right, const int32_t *bias, int64_t out_pixels,
                                     int32_t exact_unproven, int32_t *y, void *workspace,
                                     size_t workspace_bytes, int32_t *status, void *stream) {
  cim22_gather rows{};
  rows.kind = CIM22_GATHER_ROWS;
  const cim22_gather &g = gather ? *gather : rows;
  if (!layer || layer->bf16 || !x || !y || !status || m <= 0 || !workspace ||
      workspace_bytes < cim22_cuda_layer_workspace_int8(layer, m) ||
      !check_gather_int8(g, m, layer->k, pad_bottom, pad_right) || out_pixels < 0 ||
      (out_pixels > 0 && (m % out_pixels || out_pixels >= (int64_t{1} << 31)))) {
    set_last_error("invalid arguments to cim22_cuda_layer_forward_int8");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t m_pad = round_up(m, kColumnPad);
  // Proven layers cannot leave i21 on any tile, so whole-K accumulation is
  // exact; unproven ones either run the checked per-tile kernel or, with
  // exact_unproven, are computed as the Host computes them.
  const bool exact = layer->range_safe || exact_unproven;
  const bool conv = g.kind != CIM22_GATHER_ROWS;
  if (!conv && exact && tc::int8_available() && layer->k % 16 == 0 &&
      tc::launch_int8(x, m, layer->k, layer->weights, layer->n_pad, layer->k_pad, m, layer->n,
                      bias, out_pixels, y, status, s))
    return cuda_ok(cudaGetLastError(), "int8 launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
  int8_t *A = static_cast<int8_t *>(workspace);
  if (conv) {
    const Gather32 dg = to_device_gather(g, m, layer->k, nullptr);
    const int64_t total = m_pad * (layer->k_pad / 16);
    const unsigned blocks =
        static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 16));
    im2col_int8_kernel<<<blocks, 256, 0, s>>>(x, dg, m_pad, layer->k_pad, A);
  } else {
    const int64_t total = m_pad * layer->k_pad;
    const unsigned blocks =
        static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 32));
    pad_int8_kernel<<<blocks, 256, 0, s>>>(x, m, layer->k, m_pad, layer->k_pad, A);
  }
  if (!cuda_ok(cudaGetLastError(), "int8 gather launch"))
    return CIM22_STATUS_BAD_ARGUMENT;
  const int T = static_cast<int>(layer->tiles);
  if (exact && tc::int8_available() &&
      tc::launch_int8(A, m_pad, layer->k_pad, layer->weights, layer->n_pad, layer->k_pad, m,
                      layer->n, bias, out_pixels, y, status, s))
    return cuda_ok(cudaGetLastError(), "int8 launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
  const dim3 grid(static_cast<unsigned>(m_pad / 64),
                  static_cast<unsigned>((layer->n + 63) / 64));
  const FastDiv div_pix = make_fastdiv(static_cast<uint32_t>(out_pixels > 0 ? out_pixels : 1));
  int8_simt_kernel<<<grid, 256, 0, s>>>(A, layer->weights, layer->k_pad, T, m, layer->n,
                                        exact ? 0 : 1, bias, out_pixels, div_pix, y, status);
  return cuda_ok(cudaGetLastError(), "int8 launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

int cim22_cuda_layer_forward_int8(const cim22_cuda_layer *layer,
                                  const int8_t *x, int64_t m, int32_t *y,
                                  void *workspace, size_t workspace_bytes,
                                  int32_t *status, void *stream) {
  return cim22_cuda_layer_forward_int8_ex(layer, x, nullptr, m, -1, -1, nullptr, 0, 0, y,
                                          workspace, workspace_bytes, status, stream);
}

} // extern "C"
