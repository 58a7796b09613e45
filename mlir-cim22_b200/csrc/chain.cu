// chain.cu - a chain of small sign-split CIM layers in one persistent kernel.
//
// For networks whose per-image activations fit in shared memory (LeNet-5,
// the MNIST MLP) the per-layer kernels are dominated by launch latency and by
// HBM round trips of tiny activations. Here every CTA carries whole images
// through all layers with the activations in shared memory:
//
//   for each image of the CTA (persistent over images):
//     load the image into shared memory
//     for each layer:
//       for each chunk of output columns (pixels):
//         prepare   8 threads per (column, K tile) group gather the im2col
//                   group from the shared-memory input, split x into xp/xn,
//                   round to BF16, take the group maximum and prealign
//                   (convert8, the same routine as the prepare kernels)
//         contract  one thread per (column, lane): per K tile the dp4a dots
//                   of every branch pair, the exact restore
//                   RNE_bf16(Q(p) * 2^(Ew + Ex - 266)), the f32 branch sums
//                   in tile order, BF16 rounding when T > 1, the merge
//                   ((pp - pn) - np) + nn, bias and activation
//       optional 2x2 stride-2 max pool of the layer output
//     store the last layer's output
//
// A Linear layer is the convolution whose kernel covers its whole input
// (K in flatten order c * H * W + h * W + w, one output column), so one code
// path serves both. The numerics are those of the per-layer kernels
// (layers.cu), so the outputs are bit-identical to them and to the oracle.
#include "cim_internal.h"
#include "cim_numeric.cuh"
#include "signsplit_prep.cuh"

#include <algorithm>
#include <cstring>

namespace cim {
namespace {

constexpr int kChainThreads = 256;
constexpr int kMaxChainLayers = 8;
constexpr int kMaxLaneBlock = 8;

struct ChainLayerDev {
  const int8_t *B;    // resident mantissas [2][n_pad][k_pad] (Wp, Wn)
  const int32_t *exB; // lane exponents [2][T][n_pad]
  const float *sw;    // weight scales 2^(Ew - 133) [2][T][n_pad]
  const float *bias;  // [N] or null
  int C, H, W;        // input image; a Linear layer reads [K][1][1]
  int N;              // output lanes
  int KH, KW, S, P;   // kernel, stride, zero padding
  int OH, OW;         // output pixels (columns) before the pool
  int K, k_pad, T, n_pad;
  int act_br;         // activation branches: 2 for a 4-branch layer, else 1
  int act;            // CIM22_ACT_*
  int pool;           // 0, or 2: 2x2 stride-2 max pool after the activation
  int chunk;          // columns prepared per pass
  int row_stride;     // bytes per prepared column in shared memory
  int lanes_per_item; // lanes one contraction thread carries (1 .. kMaxLaneBlock)
  int many_groups;    // prepare one thread per group through the tap table
  int direct;         // one thread per column (chain_direct)
  int split;          // one column, items per (lane, weight sign, tile): chain_contract_split
};

struct ChainParams {
  ChainLayerDev layer[kMaxChainLayers];
  int n_layers;
  int in_elems, out_elems; // per image
  int buf_floats;          // each of the two activation buffers
  int as_bytes;            // prepared-column area
  int ex_ints;             // group exponents area
  int tap_ints;            // im2col tap table (two ints per K element)
};

// The eight K elements kbeg .. kbeg + 7 of column `col` of layer L, read from
// the shared-memory input (zero past K and in the conv padding).
__device__ __forceinline__ void chain_gather8(const float *in, const ChainLayerDev &L, int col,
                                              int kbeg, float (&v)[8]) {
  const int oh = col / L.OW, ow = col - oh * L.OW;
  const int ih0 = oh * L.S - L.P, iw0 = ow * L.S - L.P;
  const int khw = L.KH * L.KW;
  int c = kbeg / khw;
  const int rk = kbeg - c * khw;
  int i = rk / L.KW, j = rk - i * L.KW;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int ih = ih0 + i, iw = iw0 + j;
    v[e] = (kbeg + e < L.K && ih >= 0 && ih < L.H && iw >= 0 && iw < L.W)
               ? in[(c * L.H + ih) * L.W + iw]
               : 0.0f;
    if (++j == L.KW) {
      j = 0;
      if (++i == L.KH) {
        i = 0;
        ++c;
      }
    }
  }
}

// Preparation with eight threads per (column, K tile) group (convert8, as the
// prepare kernels): for layers with few groups, such as a Linear layer's one
// column.
template <int kActBranches>
__device__ void chain_prepare8(const float *in, const ChainLayerDev &L, int col0, int ch,
                               int8_t *As, int *sEx, int32_t *status) {
  const int tid = static_cast<int>(threadIdx.x);
  const int sub = tid % kGroupThreads;
  const unsigned mask = 0xffu << (tid & 24);
  // The eight threads of a group share g, so the group's shuffles are uniform.
  for (int g = tid / kGroupThreads; g < ch * L.T; g += kChainThreads / kGroupThreads) {
    const int col = g % ch, t = g / ch;
    const int kbeg = t * kTileK + sub * 8;
    float v[8];
    chain_gather8(in, L, col0 + col, kbeg, v);
    uint2 out[2];
    int emax[2];
    convert8<kActBranches>(v, mask, sub, status, out, emax);
#pragma unroll
    for (int a = 0; a < kActBranches; ++a) {
      *reinterpret_cast<uint2 *>(As + (a * L.chunk + col) * L.row_stride + kbeg) = out[a];
      if (sub == 0)
        sEx[(a * L.T + t) * L.chunk + col] = emax[a];
    }
  }
}

// Preparation with one thread per (column, K tile) group, for layers with
// many groups: the group's elements come from the layer's tap table (element
// offset from the window origin; kernel row and column for the padding test),
// a first pass takes the maxima, a second one aligns and stores. The split,
// maxima, verdicts and alignment are convert8's routines, so the bytes and
// exponents are the same.
template <int kActBranches>
__device__ void chain_prepare_groups(const float *in, const ChainLayerDev &L, const int *taps,
                                     int col0, int ch, int8_t *As, int *sEx, int32_t *status) {
  for (int g = static_cast<int>(threadIdx.x); g < ch * L.T; g += kChainThreads) {
    const int col = g % ch, t = g / ch;
    const int m = col0 + col;
    const int oh = m / L.OW, ow = m - oh * L.OW;
    const int ih0 = oh * L.S - L.P, iw0 = ow * L.S - L.P;
    const int org = ih0 * L.W + iw0;
    const bool interior = ih0 >= 0 && iw0 >= 0 && ih0 + L.KH <= L.H && iw0 + L.KW <= L.W;
    const int k0 = t * kTileK;
    const int valid = min(kTileK, L.K - k0);
    auto load8 = [&](int e0, float (&v)[8]) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float x = 0.0f;
        if (e0 + e < valid) {
          const int2 tp = reinterpret_cast<const int2 *>(taps)[k0 + e0 + e];
          if (interior) {
            x = in[org + tp.x];
          } else {
            const int ih = ih0 + (tp.y >> 16), iw = iw0 + (tp.y & 0xffff);
            if (ih >= 0 && ih < L.H && iw >= 0 && iw < L.W)
              x = in[org + tp.x];
          }
        }
        v[e] = x;
      }
    };
    uint32_t mx[2] = {0, 0}, flags = 0;
    uint32_t packed[2][4];
    for (int e0 = 0; e0 < valid; e0 += 8) {
      float v[8];
      load8(e0, v);
      split8<kActBranches>(v, packed, mx, flags);
    }
    int emax[2];
    group_exponents<kActBranches>(mx, flags, true, status, emax);
    for (int e0 = 0; e0 < kTileK; e0 += 8) {
      uint2 out[2] = {make_uint2(0, 0), make_uint2(0, 0)};
      if (e0 < valid) {
        float v[8];
        load8(e0, v);
        uint32_t unused[2] = {0, 0}, f = 0;
        split8<kActBranches>(v, packed, unused, f);
#pragma unroll
        for (int a = 0; a < kActBranches; ++a)
          if (emax[a] != kZeroGroup)
            out[a] = align8(packed[a], mx[a], emax[a]);
      }
#pragma unroll
      for (int a = 0; a < kActBranches; ++a)
        *reinterpret_cast<uint2 *>(As + (a * L.chunk + col) * L.row_stride + k0 + e0) = out[a];
    }
#pragma unroll
    for (int a = 0; a < kActBranches; ++a)
      sEx[(a * L.T + t) * L.chunk + col] = emax[a];
  }
}

// Dot of one prepared 64-byte activation row with one weight row: four
// independent partial sums (integer, exact in any order).
__device__ __forceinline__ int dot64(const int4 (&a)[4], const int4 (&b)[4]) {
  int p[4] = {0, 0, 0, 0};
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    p[kk] = __dp4a(a[kk].x, b[kk].x, p[kk]);
    p[kk] = __dp4a(a[kk].y, b[kk].y, p[kk]);
    p[kk] = __dp4a(a[kk].z, b[kk].z, p[kk]);
    p[kk] = __dp4a(a[kk].w, b[kk].w, p[kk]);
  }
  return (p[0] + p[1]) + (p[2] + p[3]);
}

// The restored tile value RNE_bf16(Q(p) * 2^(ex + ew - 266)) added to a
// branch sum: inside the window (ex <= 240, 140 <= ex + ew <= 374) Q(p) *
// 2^(ex - 133) is exact and its product with 2^(ew - 133) the representable
// tile value; outside it the integer path.
__device__ __forceinline__ float tile_add(float acc, int p, int ex, float sx, int ew, float sw,
                                          int32_t *status) {
  const int s = ex + ew;
  if (ex <= 240 && s >= 140 && s <= 374)
    return fmaf(__fmul_rn(trunc8f(p), sx), sw, acc);
  return slow_tile_add(acc, p, ew, ex, status);
}

// Merge of the branch sums, bias and activation.
template <int kActBranches>
__device__ __forceinline__ float finish(const float (&acc)[kActBranches][2], int T,
                                        const float *bias, int lane, int act) {
  float br[kActBranches][2];
#pragma unroll
  for (int a = 0; a < kActBranches; ++a)
#pragma unroll
    for (int w = 0; w < 2; ++w)
      br[a][w] = T > 1 ? bf16_to_f32(f32_to_bf16(acc[a][w])) : acc[a][w];
  float v = __fsub_rn(br[0][0], br[0][1]);
  if (kActBranches == 2) {
    v = __fsub_rn(v, br[1][0]);
    v = __fadd_rn(v, br[1][1]);
  }
  if (bias != nullptr)
    v = __fadd_rn(v, __ldg(bias + lane));
  return apply_act(v, act);
}

__device__ __forceinline__ void load_weights(const ChainLayerDev &L, int w, int lane, int t,
                                             int4 (&b)[4]) {
  const int4 *src = reinterpret_cast<const int4 *>(
      L.B + (static_cast<int64_t>(w) * L.n_pad + lane) * L.k_pad + t * kTileK);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    b[kk] = __ldg(src + kk);
}

// One thread per (column, lane), software-pipelined over the (tile, sign)
// steps: the weight row, exponent and scale of step s + 1 are loaded while
// step s is dotted and restored, so a Linear layer's lane runs at the load
// rate rather than paying a full load latency per tile.
template <int kActBranches>
__device__ void chain_contract_lane(const ChainLayerDev &L, int col0, int ch, const int8_t *As,
                                    const int *sEx, float *out, int32_t *status) {
  const int pixels = L.OH * L.OW;
  const int steps = 2 * L.T;
  for (int item = static_cast<int>(threadIdx.x); item < ch * L.N; item += kChainThreads) {
    const int col = item % ch, lane = item / ch;
    float acc[kActBranches][2];
#pragma unroll
    for (int a = 0; a < kActBranches; ++a)
      acc[a][0] = acc[a][1] = 0.0f;
    int4 bw[2][4];
    int ew[2];
    float sw[2];
    auto fetch = [&](int step, int slot) {
      const int t = step >> 1, w = step & 1;
      load_weights(L, w, lane, t, bw[slot]);
      ew[slot] = __ldg(L.exB + (w * L.T + t) * L.n_pad + lane);
      sw[slot] = __ldg(L.sw + (w * L.T + t) * L.n_pad + lane);
    };
    fetch(0, 0);
    int4 av[kActBranches][4];
    int ex[kActBranches];
    float sx[kActBranches];
    for (int step = 0; step < steps; step += 2) {
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        const int st = step + w, t = step >> 1;
        if (st + 1 < steps)
          fetch(st + 1, w ^ 1);
        if (w == 0) {
#pragma unroll
          for (int a = 0; a < kActBranches; ++a) {
            ex[a] = sEx[(a * L.T + t) * L.chunk + col];
            sx[a] = ex[a] == kZeroGroup ? 0.0f : exp2i(ex[a] - 133);
            const int4 *row = reinterpret_cast<const int4 *>(
                As + (a * L.chunk + col) * L.row_stride + t * kTileK);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              av[a][kk] = row[kk];
          }
        }
#pragma unroll
        for (int a = 0; a < kActBranches; ++a)
          if (ex[a] != kZeroGroup) // a zero group's tiles add +0
            acc[a][w] = tile_add(acc[a][w], dot64(av[a], bw[w]), ex[a], sx[a], ew[w], sw[w],
                                 status);
      }
    }
    out[lane * pixels + col0 + col] = finish<kActBranches>(acc, L.T, L.bias, lane, L.act);
  }
}

// Layers of one column (Linear) with fewer lanes than threads and several K
// tiles: one item per (lane, weight sign, K tile) restores that tile's value
// into shared memory (vals, after the layer's outputs in the output buffer),
// then one thread per lane adds its tiles in tile order and finishes. Inside
// the fast window tile_add's fma adds an exactly representable product, so
// acc + (that product) rounds as the fma does; a zero group's tile is +0,
// which leaves the (never -0) sum as it is; the slow path adds the same BF16
// tile value. The result is the sequential chain_contract_lane's.
template <int kActBranches>
__device__ void chain_contract_split(const ChainLayerDev &L, const int8_t *As, const int *sEx,
                                     float *out, int32_t *status) {
  float *vals = out + ((L.N + 3) & ~3); // [branch][sign][lane][tile]
  const int items = 2 * L.N * L.T;
  for (int it = static_cast<int>(threadIdx.x); it < items; it += kChainThreads) {
    const int t = it % L.T, lane = (it / L.T) % L.N, w = it / (L.T * L.N);
    int4 bw[4];
    load_weights(L, w, lane, t, bw);
    const int ew = __ldg(L.exB + (w * L.T + t) * L.n_pad + lane);
    const float sw = __ldg(L.sw + (w * L.T + t) * L.n_pad + lane);
#pragma unroll
    for (int a = 0; a < kActBranches; ++a) {
      const int ex = sEx[(a * L.T + t) * L.chunk];
      float v = 0.0f; // a zero group's tile adds +0
      if (ex != kZeroGroup) {
        int4 av[4];
        const int4 *row = reinterpret_cast<const int4 *>(As + a * L.chunk * L.row_stride +
                                                         t * kTileK);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          av[kk] = row[kk];
        v = tile_add(0.0f, dot64(av, bw), ex, exp2i(ex - 133), ew, sw, status);
      }
      vals[((a * 2 + w) * L.N + lane) * L.T + t] = v;
    }
  }
  __syncthreads();
  for (int lane = static_cast<int>(threadIdx.x); lane < L.N; lane += kChainThreads) {
    float acc[kActBranches][2];
#pragma unroll
    for (int a = 0; a < kActBranches; ++a)
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        const float *v = vals + ((a * 2 + w) * L.N + lane) * L.T;
        float sum = 0.0f;
        for (int t = 0; t < L.T; ++t)
          sum = __fadd_rn(sum, v[t]);
        acc[a][w] = sum;
      }
    out[lane] = finish<kActBranches>(acc, L.T, L.bias, lane, L.act);
  }
}

// One thread per (column, block of up to kMaxLaneBlock lanes): per K tile the
// column's prepared rows are read once, each lane's weight rows (the same for
// the whole warp: a broadcast) are dotted with them, and each restored tile is
// added to its branch sum in tile order.
template <int kActBranches>
__device__ void chain_contract(const ChainLayerDev &L, int col0, int ch, const int8_t *As,
                               const int *sEx, float *out, int32_t *status) {
  // Lanes per item: up to 8 for 2-branch layers, 4 for 4-branch layers
  // (the same register budget for the branch sums).
  constexpr int kLB = kActBranches == 2 ? kMaxLaneBlock / 2 : kMaxLaneBlock;
  const int pixels = L.OH * L.OW;
  const int lb = L.lanes_per_item;
  const int blocks = (L.N + lb - 1) / lb;
  for (int item = static_cast<int>(threadIdx.x); item < ch * blocks; item += kChainThreads) {
    const int col = item % ch, lane0 = (item / ch) * lb;
    const int nl = min(lb, L.N - lane0);
    float acc[kLB][kActBranches][2];
#pragma unroll
    for (int l = 0; l < kLB; ++l)
#pragma unroll
      for (int a = 0; a < kActBranches; ++a)
        acc[l][a][0] = acc[l][a][1] = 0.0f;
    for (int t = 0; t < L.T; ++t) {
      int4 av[kActBranches][4];
      int ex[kActBranches];
      float sx[kActBranches];
#pragma unroll
      for (int a = 0; a < kActBranches; ++a) {
        ex[a] = sEx[(a * L.T + t) * L.chunk + col];
        sx[a] = ex[a] == kZeroGroup ? 0.0f : exp2i(ex[a] - 133);
        const int4 *row = reinterpret_cast<const int4 *>(
            As + (a * L.chunk + col) * L.row_stride + t * kTileK);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          av[a][kk] = row[kk];
      }
#pragma unroll
      for (int l = 0; l < kLB; ++l) {
        if (l >= nl)
          break;
        const int lane = lane0 + l;
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          int4 bw[4];
          load_weights(L, w, lane, t, bw);
          const int ew = __ldg(L.exB + (w * L.T + t) * L.n_pad + lane);
          const float sw = __ldg(L.sw + (w * L.T + t) * L.n_pad + lane);
#pragma unroll
          for (int a = 0; a < kActBranches; ++a)
            if (ex[a] != kZeroGroup) // a zero group's tiles add +0
              acc[l][a][w] = tile_add(acc[l][a][w], dot64(av[a], bw), ex[a], sx[a], ew, sw,
                                      status);
        }
      }
    }
#pragma unroll
    for (int l = 0; l < kLB; ++l) {
      if (l >= nl)
        break;
      const int lane = lane0 + l;
      out[lane * pixels + col0 + col] = finish<kActBranches>(acc[l], L.T, L.bias, lane, L.act);
    }
  }
}

// One-tile layers of few lanes (K <= kDirectMaxK, at most kDirectMaxLanes
// lanes: the first convolution of LeNet). One thread per column gathers its
// group from the shared-memory input, splits, rounds and prealigns it in
// registers with the routines of the prepare passes (split8,
// group_exponents, align8), and dots it with every lane's weight rows; the
// restore and the merge are tile_add and finish. The result is the one the
// staged passes give (elements past kDirectMaxK are K padding, zero in both
// operands), without the prepared columns in shared memory and the barriers
// between the passes.
constexpr int kDirectMaxK = 32;
constexpr int kDirectMaxLanes = 16;

template <int kActBranches>
__device__ void chain_direct(const float *in, const ChainLayerDev &L, float *out,
                             int32_t *status) {
  constexpr int kChunks = kDirectMaxK / 8;
  const int cols = L.OH * L.OW;
  for (int col = static_cast<int>(threadIdx.x); col < cols; col += kChainThreads) {
    uint32_t packed[kChunks][2][4];
    uint32_t mx[2] = {0, 0};
    uint32_t flags = 0;
#pragma unroll
    for (int c8 = 0; c8 < kChunks; ++c8) {
      float v[8];
      chain_gather8(in, L, col, c8 * 8, v);
      split8<kActBranches>(v, packed[c8], mx, flags);
    }
    int emax[2];
    group_exponents<kActBranches>(mx, flags, true, status, emax);
    uint32_t aw[kActBranches][2 * kChunks];
    float sx[kActBranches];
#pragma unroll
    for (int a = 0; a < kActBranches; ++a) {
#pragma unroll
      for (int c8 = 0; c8 < kChunks; ++c8) {
        const uint2 w2 = align8(packed[c8][a], mx[a], emax[a]);
        aw[a][2 * c8] = w2.x;
        aw[a][2 * c8 + 1] = w2.y;
      }
      sx[a] = emax[a] == kZeroGroup ? 0.0f : exp2i(emax[a] - 133);
    }
    for (int lane = 0; lane < L.N; ++lane) {
      float acc[kActBranches][2];
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        const int4 *row = reinterpret_cast<const int4 *>(
            L.B + (static_cast<int64_t>(w) * L.n_pad + lane) * L.k_pad);
        const int4 b0 = __ldg(row), b1 = __ldg(row + 1);
        const int bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        const int ew = __ldg(L.exB + w * L.n_pad + lane); // Ew[w][tile 0][lane]
        const float sw = __ldg(L.sw + w * L.n_pad + lane);
#pragma unroll
        for (int a = 0; a < kActBranches; ++a) {
          int p = 0;
#pragma unroll
          for (int q = 0; q < 2 * kChunks; ++q)
            p = __dp4a(static_cast<int>(aw[a][q]), bw[q], p);
          acc[a][w] = emax[a] != kZeroGroup // a zero group's tile adds +0
                          ? tile_add(0.0f, p, emax[a], sx[a], ew, sw, status)
                          : 0.0f;
        }
      }
      out[lane * cols + col] = finish<kActBranches>(acc, L.T, L.bias, lane, L.act);
    }
  }
}

// 2x2 stride-2 max pool of [N][OH][OW] into [N][OH/2][OW/2], NaN propagating
// in window order as torch.max_pool2d.
__device__ void chain_pool(const float *src, const ChainLayerDev &L, float *dst) {
  const int ph = L.OH / 2, pw = L.OW / 2;
  for (int i = static_cast<int>(threadIdx.x); i < L.N * ph * pw; i += kChainThreads) {
    const int c = i / (ph * pw), r = i - c * ph * pw;
    const int y = r / pw, x = r - y * pw;
    const float *s = src + (c * L.OH + 2 * y) * L.OW + 2 * x;
    const float v[4] = {s[0], s[1], s[L.OW], s[L.OW + 1]};
    float m = v[0];
#pragma unroll
    for (int e = 1; e < 4; ++e)
      m = (v[e] > m || v[e] != v[e]) ? v[e] : m;
    dst[i] = m;
  }
}

// Two CTAs per SM: 128 registers per thread at most.
__global__ void __launch_bounds__(kChainThreads, 2)
    chain_kernel(const __grid_constant__ ChainParams prm, const float *__restrict__ x,
                 float *__restrict__ y, int batch, int32_t *status) {
  extern __shared__ __align__(16) uint8_t smem[];
  float *buf[2] = {reinterpret_cast<float *>(smem),
                   reinterpret_cast<float *>(smem) + prm.buf_floats};
  int8_t *As = reinterpret_cast<int8_t *>(smem + 8 * static_cast<size_t>(prm.buf_floats));
  int *sEx = reinterpret_cast<int *>(As + prm.as_bytes);
  int *taps = sEx + prm.ex_ints;
  pdl_launch_dependents();
  pdl_wait();
  for (int img = static_cast<int>(blockIdx.x); img < batch; img += static_cast<int>(gridDim.x)) {
    const float *xi = x + static_cast<int64_t>(img) * prm.in_elems;
    for (int i = static_cast<int>(threadIdx.x); i < prm.in_elems; i += kChainThreads)
      buf[0][i] = xi[i];
    __syncthreads();
    int cur = 0;
    for (int l = 0; l < prm.n_layers; ++l) {
      const ChainLayerDev &L = prm.layer[l];
      const float *in = buf[cur];
      float *out = buf[cur ^ 1];
      const int cols = L.OH * L.OW;
      if (L.direct) {
        if (L.act_br == 2)
          chain_direct<2>(in, L, out, status);
        else
          chain_direct<1>(in, L, out, status);
        __syncthreads();
      } else if (L.many_groups) {
        // Tap table: offset of K element k from the window origin, and its
        // kernel row and column.
        for (int k = static_cast<int>(threadIdx.x); k < L.K; k += kChainThreads) {
          const int khw = L.KH * L.KW;
          const int c = k / khw, r = k - c * khw;
          const int i = r / L.KW, j = r - i * L.KW;
          taps[2 * k] = (c * L.H + i) * L.W + j;
          taps[2 * k + 1] = (i << 16) | j;
        }
        __syncthreads();
      }
      for (int col0 = 0; col0 < cols && !L.direct; col0 += L.chunk) {
        const int ch = min(L.chunk, cols - col0);
        if (L.many_groups) {
          if (L.act_br == 2)
            chain_prepare_groups<2>(in, L, taps, col0, ch, As, sEx, status);
          else
            chain_prepare_groups<1>(in, L, taps, col0, ch, As, sEx, status);
        } else if (L.act_br == 2) {
          chain_prepare8<2>(in, L, col0, ch, As, sEx, status);
        } else {
          chain_prepare8<1>(in, L, col0, ch, As, sEx, status);
        }
        __syncthreads();
        if (L.split) {
          if (L.act_br == 2)
            chain_contract_split<2>(L, As, sEx, out, status);
          else
            chain_contract_split<1>(L, As, sEx, out, status);
        } else if (L.lanes_per_item == 1) {
          if (L.act_br == 2)
            chain_contract_lane<2>(L, col0, ch, As, sEx, out, status);
          else
            chain_contract_lane<1>(L, col0, ch, As, sEx, out, status);
        } else if (L.act_br == 2) {
          chain_contract<2>(L, col0, ch, As, sEx, out, status);
        } else {
          chain_contract<1>(L, col0, ch, As, sEx, out, status);
        }
        __syncthreads();
      }
      if (L.pool) {
        // The input is dead: the pooled map replaces it.
        chain_pool(out, L, buf[cur]);
        __syncthreads();
      } else {
        cur ^= 1;
      }
    }
    float *yi = y + static_cast<int64_t>(img) * prm.out_elems;
    for (int i = static_cast<int>(threadIdx.x); i < prm.out_elems; i += kChainThreads)
      yi[i] = buf[cur][i];
    __syncthreads();
  }
}

} // namespace
} // namespace cim

using namespace cim;

extern "C" {

int cim22_cuda_chain_forward(const cim22_chain_layer *layers, int32_t n_layers, const float *x,
                             int64_t batch, float *y, int32_t *status, void *stream) {
  if (!layers || n_layers <= 0 || n_layers > kMaxChainLayers || !x || !y || !status ||
      batch <= 0 || batch >= (int64_t{1} << 31)) {
    set_last_error("invalid arguments to cim22_cuda_chain_forward");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  ChainParams prm{};
  prm.n_layers = n_layers;
  int64_t buf = 0, as_bytes = 0, ex_ints = 0, tap_ints = 0;
  int c = layers[0].channels, h = layers[0].height, w = layers[0].width;
  prm.in_elems = c * h * w;
  for (int l = 0; l < n_layers; ++l) {
    const cim22_chain_layer &s = layers[l];
    const cim22_cuda_layer *lay = s.layer;
    ChainLayerDev &d = prm.layer[l];
    const bool conv = s.kind == CIM22_CHAIN_CONV;
    // A Linear layer flattens its input: [C][H][W] -> [K][1][1].
    if (!conv) {
      c = c * h * w;
      h = w = 1;
    }
    if (!lay || !lay->bf16 || lay->mode != CIM22_BF16_SIGN_SPLIT ||
        (s.kind != CIM22_CHAIN_CONV && s.kind != CIM22_CHAIN_LINEAR) ||
        (s.branches != 2 && s.branches != 4) || s.activation < 0 || s.activation > 2 ||
        (s.pool != 0 && s.pool != 2) || c <= 0 || h <= 0 || w <= 0) {
      set_last_error("invalid chain layer");
      return CIM22_STATUS_BAD_ARGUMENT;
    }
    const int kh = conv ? s.kernel_h : 1, kw = conv ? s.kernel_w : 1;
    const int st = conv ? s.stride : 1, pd = conv ? s.pad : 0;
    if (kh <= 0 || kw <= 0 || st <= 0 || pd < 0 || h + 2 * pd < kh || w + 2 * pd < kw ||
        static_cast<int64_t>(c) * kh * kw != lay->k) {
      set_last_error("chain layer geometry does not match its weights");
      return CIM22_STATUS_BAD_ARGUMENT;
    }
    d.B = lay->weights;
    d.exB = lay->exponents;
    d.sw = reinterpret_cast<const float *>(lay->exponents + 2 * lay->tiles * lay->n_pad +
                                           (lay->n_pad / 32) * lay->tiles * 4);
    d.bias = s.bias;
    d.C = c;
    d.H = h;
    d.W = w;
    d.N = static_cast<int>(lay->n);
    d.KH = kh;
    d.KW = kw;
    d.S = st;
    d.P = pd;
    d.OH = (h + 2 * pd - kh) / st + 1;
    d.OW = (w + 2 * pd - kw) / st + 1;
    d.K = static_cast<int>(lay->k);
    d.k_pad = static_cast<int>(lay->k_pad);
    d.T = static_cast<int>(lay->tiles);
    d.n_pad = static_cast<int>(lay->n_pad);
    d.act_br = s.branches == 4 ? 2 : 1;
    d.act = s.activation;
    d.pool = s.pool;
    d.row_stride = d.k_pad + 16;
    const int cols = d.OH * d.OW;
    // Columns per pass: up to 256 within a 48 KB prepared area.
    const int per_col = d.act_br * d.row_stride;
    d.chunk = std::max(1, std::min({cols, 256, (48 << 10) / per_col}));
    // Contraction items: the fewest lanes per thread that still fit the
    // block in one pass (up to kMaxLaneBlock).
    const int max_lb = d.act_br == 2 ? kMaxLaneBlock / 2 : kMaxLaneBlock;
    d.lanes_per_item = max_lb;
    for (int lb = 1; lb <= max_lb; ++lb)
      if (static_cast<int64_t>(d.chunk) * ((d.N + lb - 1) / lb) <= kChainThreads) {
        d.lanes_per_item = lb;
        break;
      }
    // One thread per prepare group once there are enough groups for the block.
    d.many_groups = static_cast<int64_t>(d.chunk) * d.T >= kChainThreads / 2 ? 1 : 0;
    d.direct = d.T == 1 && d.K <= kDirectMaxK && d.N <= kDirectMaxLanes ? 1 : 0;
    if (d.direct)
      d.many_groups = 0;
    // One column over fewer lanes than threads and several tiles: per-tile
    // items, their values after the outputs in the output buffer.
    d.split = cols == 1 && d.T >= 2 && d.N < kChainThreads && !d.direct ? 1 : 0;
    if (d.split)
      buf = std::max<int64_t>(buf, (d.N + 3) / 4 * 4 +
                                       2 * static_cast<int64_t>(d.N) * d.T * d.act_br);
    if (s.pool && (d.OH < 2 || d.OW < 2)) {
      set_last_error("chain pool needs an output of at least 2x2");
      return CIM22_STATUS_BAD_ARGUMENT;
    }
    buf = std::max<int64_t>({buf, static_cast<int64_t>(c) * h * w,
                             static_cast<int64_t>(d.N) * cols});
    as_bytes = std::max<int64_t>(as_bytes, static_cast<int64_t>(d.chunk) * per_col);
    ex_ints = std::max<int64_t>(ex_ints, static_cast<int64_t>(d.act_br) * d.T * d.chunk);
    if (d.many_groups)
      tap_ints = std::max<int64_t>(tap_ints, 2 * static_cast<int64_t>(d.K));

    c = d.N;
    h = s.pool ? d.OH / 2 : d.OH;
    w = s.pool ? d.OW / 2 : d.OW;
  }
  prm.out_elems = c * h * w;
  prm.buf_floats = static_cast<int>((buf + 3) / 4 * 4);
  prm.as_bytes = static_cast<int>((as_bytes + 15) / 16 * 16);
  // Areas in 16-byte units: the tap table is read as int2.
  prm.ex_ints = static_cast<int>((ex_ints + 3) / 4 * 4);
  prm.tap_ints = static_cast<int>((tap_ints + 3) / 4 * 4);
  const size_t smem = 8 * static_cast<size_t>(prm.buf_floats) + prm.as_bytes +
                      4 * (static_cast<size_t>(prm.ex_ints) + prm.tap_ints);
  if (smem > 200 * 1024) {
    set_last_error("chain activations do not fit in shared memory");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  if (!cuda_ok(cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)),
               "chain smem attribute"))
    return CIM22_STATUS_BAD_ARGUMENT;
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, chain_kernel, kChainThreads, smem);
  int device = 0, sms = 148;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int64_t grid = std::min<int64_t>(batch, static_cast<int64_t>(std::max(1, per_sm)) * sms);
  launch_pdl(chain_kernel, dim3(static_cast<unsigned>(grid)), kChainThreads, smem,
             static_cast<cudaStream_t>(stream), prm, x, y, static_cast<int>(batch), status);
  return cuda_ok(cudaGetLastError(), "chain launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

} // extern "C"
