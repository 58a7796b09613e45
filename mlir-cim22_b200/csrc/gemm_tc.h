// gemm_tc.h - tensor-core (tcgen05) CIM contraction kernels for sm_100a.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/cim22_cuda.h"

namespace cim::tc {

// The weight scales of the sign-split contraction are stored as
// 2^(Ew - 133 + kScaleShift): the epilogue reads each crossbar dot p as the
// f32 subnormal p * 2^-149 and multiplies it by 2^(Ex + 16 - kScaleShift),
// which is exact and normal for 67 <= Ex <= 171, so the product with the
// shifted weight scale is Q(p) * 2^(Ex + Ew - 266) as before.
constexpr int kScaleShift = 60;

// Words of one per-(K tile, 32-lane block) weight record of the sign-split
// contraction: the Wp and Wn epilogue scales of the block's 32 lanes, then
// its exponent range {min, max, ex_lo, ex_hi}.
constexpr int kScaleBlockWords = 32 + 32 + 4;

// True when the tcgen05 kernels are compiled in and the current device is an
// sm_100 part.
bool signsplit_available();
bool int8_available();

// Launch the sign-split contraction over prepared operands (layout of
// layers.cu): A int8 [act_branches * m_pad][k_pad], exA int32
// [act_branches][T][m_pad], B int8 [2 * n_pad][k_pad] (Wp rows, then Wn),
// exB int32 [2][T][n_pad] followed by the weight-exponent ranges
// [T][n_pad / 32][4] = {min, max, ex_lo, ex_hi} over both signs of each tile
// and 32-lane block (ex_lo..ex_hi: the activation exponents the epilogue
// restores on its fast path), by the f32 weight scales 2^(Ew - 133) [2][T][n_pad] and by
// the epilogue's f32 scales 2^(Ew - 133 + kScaleShift) [2][T][n_pad] and by
// the same scales and ranges as records [T][n_pad / 32][kScaleBlockWords].
// Returns false when the shape is not handled by the tensor-core
// kernel, in which case nothing was launched. out_pixels = 0 writes y as
// rows [M][N]; out_pixels > 0 writes NCHW images [M / out_pixels][N][out_pixels].
// A non-null post_scale applies fma(out, post_scale[n], post_shift[n]) after
// the bias and before the activation.
bool launch_signsplit(const int8_t *A, const int32_t *exA, int64_t m_pad,
                      const int8_t *B, const int32_t *exB, int64_t n_pad,
                      int64_t k_pad, int T, int64_t M, int64_t N,
                      const float *bias, const float *post_scale,
                      const float *post_shift, const float *residual, int act,
                      int act_branches, int64_t out_pixels, float *y, int32_t *status,
                      cudaStream_t stream);

// The sign-split contraction with BF16 operands: A holds the prepared
// activation groups as BF16 values [act_branches * m_pad][k_pad] - a * 2^(Ex -
// 133) for groups whose exponent Ex lies in [ex_lo, ex_hi], the unscaled
// mantissas a otherwise - and exA their exponents [act_branches][T][m_pad];
// B holds the weights b * 2^(Ew - 133) [2 * n_pad][k_pad] (Wp rows, then Wn)
// and exB the lane exponents [2][T][n_pad] of launch_signsplit's layout. The
// tcgen05 MMAs (kind::f16, f32 accumulation) then give each crossbar dot as
// the exact f32 value p * 2^(Ex + Ew - 266) (p * 2^(Ew - 133) for unscaled
// groups). Same outputs, options and return convention as launch_signsplit.
// With peers (rows output, no residual) every output row is stored into all
// ranks' full outputs instead of y (see cim22_cuda_layer_contract_bf16_peers).
bool launch_signsplit_b16(const uint16_t *A, const int32_t *exA, int64_t m_pad,
                          const uint16_t *B, const int32_t *exB, int64_t n_pad, int64_t k_pad,
                          int T, int64_t M, int64_t N, int ex_lo, int ex_hi, const float *bias,
                          const float *post_scale, const float *post_shift,
                          const float *residual, int act, int act_branches, int64_t out_pixels,
                          float *y, int32_t *status, cudaStream_t stream,
                          const cim22_peer_outputs *peers = nullptr);

// INT8 contraction with whole-K int32 accumulation (exact: range-proven
// layers, or unproven ones computed as the Host computes them).
// A is int8 [a_rows][a_cols] (a_cols <= k_pad, a multiple of 16; rows >= M),
// B is the resident [n_pad][k_pad] weight matrix. bias (optional) is a
// wrapping int32 add per lane; out_pixels > 0 writes NCHW images
// [M / out_pixels][N][out_pixels] instead of rows [M][N].
bool launch_int8(const int8_t *A, int64_t a_rows, int64_t a_cols, const int8_t *B,
                 int64_t n_pad, int64_t k_pad, int64_t M, int64_t N, const int32_t *bias,
                 int64_t out_pixels, int32_t *y, int32_t *status, cudaStream_t stream);

// Tensor map of an f32 NCHW tensor [N][C][H][W] (W contiguous, W % 4 == 0,
// 16-byte aligned) for per-CTA loads of [nb][cb][hb][wb] boxes; elements
// outside the tensor read as +0. False when the driver rejects it.
bool encode_nchw_box(CUtensorMap *map, const float *x, uint64_t W, uint64_t H, uint64_t C,
                     uint64_t N, uint32_t wb, uint32_t hb, uint32_t cb, uint32_t nb);

// Tensor map of prepared activation columns [rows][k_pad] (int8, or BF16
// with b16) for TMA stores of 32-row x 64-element boxes from a swizzled
// shared-memory tile: 64-byte swizzle for int8 rows, 128-byte for BF16 rows.
// False when the driver rejects it.
bool encode_prepared_store(CUtensorMap *map, void *base, uint64_t rows, uint64_t k_pad,
                           bool b16);

} // namespace cim::tc
