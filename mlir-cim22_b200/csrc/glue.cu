// glue.cu - the f32 Host glue the compiler emits around CIM layers
// (ReLU, residual add, GELU, pooling, batch-norm affine, softmax, layout),
// lowered by the reference through upstream Linalg to loops
// (lib/Compiler/Pipelines.cpp:61-72). Memory-bound: grid-stride loops with
// 128-bit accesses where the shape allows, images in NHWC or NCHW as named.
#include "cim_internal.h"

#include <algorithm>
#include <cfloat>

namespace cim {
namespace {

unsigned grid_for(int64_t work, int threads = 256) {
  const int64_t blocks = (work + threads - 1) / threads;
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(blocks, 148 * 16)));
}

__device__ __forceinline__ float act_fn(float v, int act) {
  if (act == CIM22_ACT_RELU)
    return (v > 0.0f || v != v) ? v : 0.0f; // NaN propagates, as torch.relu
  if (act == CIM22_ACT_GELU)
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  return v;
}

template <int kAct>
__global__ void unary_kernel(const float *__restrict__ x, float *__restrict__ y,
                             int64_t count) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t vec = count / 4;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (aligned) {
    for (int64_t i = i0; i < vec; i += stride) {
      float4 v = reinterpret_cast<const float4 *>(x)[i];
      v.x = act_fn(v.x, kAct);
      v.y = act_fn(v.y, kAct);
      v.z = act_fn(v.z, kAct);
      v.w = act_fn(v.w, kAct);
      reinterpret_cast<float4 *>(y)[i] = v;
    }
    for (int64_t i = vec * 4 + i0; i < count; i += stride)
      y[i] = act_fn(x[i], kAct);
  } else {
    for (int64_t i = i0; i < count; i += stride)
      y[i] = act_fn(x[i], kAct);
  }
}

__global__ void add_kernel(const float *__restrict__ a, const float *__restrict__ b,
                           float *__restrict__ y, int64_t count, int act) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < count; i += stride)
    y[i] = act_fn(__fadd_rn(a[i], b[i]), act);
}

// Elementwise arithmetic and comparisons of the Host glue (stateful LIF
// updates and other f32 elementwise code the compiler leaves on the Host).
// Each operation rounds once, as PyTorch's CPU kernels do; comparisons give
// 1.0f / 0.0f (false for NaN operands, as in IEEE). Operands may alias y.
__device__ __forceinline__ float binary_op(float x, float z, int op) {
  switch (op) {
  case CIM22_BINARY_ADD: return __fadd_rn(x, z);
  case CIM22_BINARY_SUB: return __fsub_rn(x, z);
  case CIM22_BINARY_MUL: return __fmul_rn(x, z);
  case CIM22_BINARY_DIV: return __fdiv_rn(x, z);
  case CIM22_BINARY_GE: return x >= z ? 1.0f : 0.0f;
  case CIM22_BINARY_GT: return x > z ? 1.0f : 0.0f;
  case CIM22_BINARY_LE: return x <= z ? 1.0f : 0.0f;
  case CIM22_BINARY_LT: return x < z ? 1.0f : 0.0f;
  case CIM22_BINARY_EQ: return x == z ? 1.0f : 0.0f;
  case CIM22_BINARY_NE: return x != z ? 1.0f : 0.0f;
  case CIM22_BINARY_MAX: return (x != x || z != z) ? __int_as_float(0x7fc00000) : fmaxf(x, z);
  default: return (x != x || z != z) ? __int_as_float(0x7fc00000) : fminf(x, z);
  }
}

__global__ void binary_kernel(const float *a, const float *b, float *y, int64_t count, int op,
                              float a_scalar, float b_scalar) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride)
    y[i] = binary_op(a ? a[i] : a_scalar, b ? b[i] : b_scalar, op);
}

__global__ void fill_kernel(float *__restrict__ y, int64_t count, float value) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride)
    y[i] = value;
}

// 32-bit word copy (f32, int32, or float-coded bool data).
__global__ void copy_kernel(const uint32_t *__restrict__ src, uint32_t *__restrict__ dst,
                            int64_t count) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride)
    dst[i] = src[i];
}

// Strided block copy: `blocks` runs of `inner` 32-bit words, run b read at
// src + b * src_stride and written at dst + b * dst_stride (a select along an
// inner axis, or the slice insert of select_scatter).
__global__ void slice_copy_kernel(const uint32_t *__restrict__ src, uint32_t *__restrict__ dst,
                                  int64_t blocks, int64_t inner, int64_t src_stride,
                                  int64_t dst_stride) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t count = blocks * inner;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride) {
    const int64_t b = i / inner, j = i - b * inner;
    dst[b * dst_stride + j] = src[b * src_stride + j];
  }
}

__global__ void maxpool_kernel(const float *__restrict__ x, float *__restrict__ y,
                               int n, int h, int w, int c, int k, int s, int pad,
                               int oh, int ow) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = static_cast<int64_t>(n) * oh * ow * c;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < total; i += stride) {
    const int ch = static_cast<int>(i % c);
    int64_t r = i / c;
    const int ox = static_cast<int>(r % ow);
    r /= ow;
    const int oy = static_cast<int>(r % oh);
    const int b = static_cast<int>(r / oh);
    float m = -FLT_MAX;
    bool any = false;
    for (int dy = 0; dy < k; ++dy)
      for (int dx = 0; dx < k; ++dx) {
        const int iy = oy * s - pad + dy, ix = ox * s - pad + dx;
        if (iy < 0 || iy >= h || ix < 0 || ix >= w)
          continue;
        const float v = x[((static_cast<int64_t>(b) * h + iy) * w + ix) * c + ch];
        // NaN propagates like torch.max_pool2d.
        if (!any || v > m || v != v) {
          m = v;
          any = true;
        }
      }
    y[i] = m;
  }
}

__global__ void avgpool_kernel(const float *__restrict__ x, float *__restrict__ y,
                               int n, int h, int w, int c, int k, int s, int oh,
                               int ow) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = static_cast<int64_t>(n) * oh * ow * c;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const float inv = 1.0f / static_cast<float>(k * k);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < total; i += stride) {
    const int ch = static_cast<int>(i % c);
    int64_t r = i / c;
    const int ox = static_cast<int>(r % ow);
    r /= ow;
    const int oy = static_cast<int>(r % oh);
    const int b = static_cast<int>(r / oh);
    float sum = 0.0f;
    for (int dy = 0; dy < k; ++dy)
      for (int dx = 0; dx < k; ++dx)
        sum += x[((static_cast<int64_t>(b) * h + oy * s + dy) * w + ox * s + dx) * c + ch];
    y[i] = sum * inv;
  }
}

// Mean over the spatial plane: one block per (image, 32-channel group),
// warps stride the plane, shared-memory reduction.
__global__ void gap_kernel(const float *__restrict__ x, float *__restrict__ y,
                           int h, int w, int c) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  const int c0 = blockIdx.y * 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const int ch = c0 + lane;
  const int plane = h * w;
  float sum = 0.0f;
  if (ch < c)
    for (int p = warp; p < plane; p += warps)
      sum += x[(static_cast<int64_t>(b) * plane + p) * c + ch];
  __shared__ float part[32][33];
  part[warp][lane] = sum;
  __syncthreads();
  if (warp == 0) {
    float total = 0.0f;
    for (int i = 0; i < warps; ++i)
      total += part[i][lane];
    if (ch < c)
      y[static_cast<int64_t>(b) * c + ch] = total / static_cast<float>(plane);
  }
}

__global__ void affine_kernel(const float *__restrict__ x, const float *__restrict__ scale,
                              const float *__restrict__ shift, float *__restrict__ y,
                              int64_t rows, int c, int act) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = rows * c;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < total; i += stride) {
    const int ch = static_cast<int>(i % c);
    y[i] = act_fn(fmaf(x[i], scale[ch], shift[ch]), act);
  }
}

// One warp per row.
__global__ void softmax_kernel(const float *__restrict__ x, float *__restrict__ y,
                               int64_t rows, int cols) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows)
    return;
  const float *in = x + row * cols;
  float *out = y + row * cols;
  float m = -INFINITY;
  for (int i = lane; i < cols; i += 32)
    m = fmaxf(m, in[i]);
  for (int o = 16; o; o >>= 1)
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.0f;
  for (int i = lane; i < cols; i += 32)
    s += expf(in[i] - m);
  for (int o = 16; o; o >>= 1)
    s += __shfl_xor_sync(0xffffffffu, s, o);
  for (int i = lane; i < cols; i += 32)
    out[i] = expf(in[i] - m) / s;
}

__global__ void nhwc_to_nchw_kernel(const float *__restrict__ x, float *__restrict__ y,
                                    int n, int h, int w, int c) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = static_cast<int64_t>(n) * h * w * c;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < total; i += stride) {
    // i indexes the NCHW output.
    const int xw = static_cast<int>(i % w);
    int64_t r = i / w;
    const int xh = static_cast<int>(r % h);
    r /= h;
    const int ch = static_cast<int>(r % c);
    const int b = static_cast<int>(r / c);
    y[i] = x[((static_cast<int64_t>(b) * h + xh) * w + xw) * c + ch];
  }
}

__global__ void nchw_to_nhwc_kernel(const float *__restrict__ x, float *__restrict__ y,
                                    int n, int c, int h, int w) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = static_cast<int64_t>(n) * h * w * c;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < total; i += stride) {
    // i indexes the NHWC output.
    const int ch = static_cast<int>(i % c);
    int64_t r = i / c;
    const int xw = static_cast<int>(r % w);
    r /= w;
    const int xh = static_cast<int>(r % h);
    const int b = static_cast<int>(r / h);
    y[i] = x[((static_cast<int64_t>(b) * c + ch) * h + xh) * w + xw];
  }
}

// NCHW pooling: output index i = ((b * c + ch) * oh + oy) * ow + ox, so a
// warp's threads read neighbouring pixels of one plane.
__global__ void maxpool_nchw_kernel(const float *__restrict__ x, float *__restrict__ y,
                                    int64_t planes, int h, int w, int k, int s, int pad,
                                    int oh, int ow) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = planes * oh * ow;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < total; i += stride) {
    const int ox = static_cast<int>(i % ow);
    const int64_t r = i / ow;
    const int oy = static_cast<int>(r % oh);
    const float *plane = x + (r / oh) * h * w;
    float m = -FLT_MAX;
    bool any = false;
    for (int dy = 0; dy < k; ++dy)
      for (int dx = 0; dx < k; ++dx) {
        const int iy = oy * s - pad + dy, ix = ox * s - pad + dx;
        if (iy < 0 || iy >= h || ix < 0 || ix >= w)
          continue;
        const float v = plane[iy * w + ix];
        // NaN propagates like torch.max_pool2d.
        if (!any || v > m || v != v) {
          m = v;
          any = true;
        }
      }
    y[i] = m;
  }
}

__global__ void avgpool_nchw_kernel(const float *__restrict__ x, float *__restrict__ y,
                                    int64_t planes, int h, int w, int k, int s, int oh,
                                    int ow) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = planes * oh * ow;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const float inv = 1.0f / static_cast<float>(k * k);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < total; i += stride) {
    const int ox = static_cast<int>(i % ow);
    const int64_t r = i / ow;
    const int oy = static_cast<int>(r % oh);
    const float *plane = x + (r / oh) * h * w;
    float sum = 0.0f;
    for (int dy = 0; dy < k; ++dy)
      for (int dx = 0; dx < k; ++dx)
        sum += plane[(oy * s + dy) * w + ox * s + dx];
    y[i] = sum * inv;
  }
}

// Mean of each plane: one warp per (image, channel) plane.
__global__ void gap_nchw_kernel(const float *__restrict__ x, float *__restrict__ y,
                                int64_t planes, int64_t hw) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t plane = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (plane >= planes)
    return;
  const float *p = x + plane * hw;
  float sum = 0.0f;
  for (int64_t i = lane; i < hw; i += 32)
    sum += p[i];
  for (int o = 16; o; o >>= 1)
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0)
    y[plane] = sum / static_cast<float>(hw);
}

// Mean of each small plane (at most 64 elements, a multiple of 4, 16-byte
// aligned): one thread per plane, 128-bit loads, the elements summed in
// order; a warp's 32 planes are contiguous.
__global__ void gap_nchw_small_kernel(const float4 *__restrict__ x, float *__restrict__ y,
                                      int64_t planes, int quads) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t plane = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (plane >= planes)
    return;
  const float4 *p = x + plane * quads;
  float sum = 0.0f;
  for (int i = 0; i < quads; ++i) {
    const float4 v = __ldg(p + i);
    sum += v.x;
    sum += v.y;
    sum += v.z;
    sum += v.w;
  }
  y[plane] = sum / static_cast<float>(4 * quads);
}

// Per-channel affine over NCHW planes, 128-bit accesses: planes of a
// multiple of 4 elements, flat index below 2^31 quads.
__global__ void affine_nchw_vec_kernel(const float4 *__restrict__ x,
                                       const float *__restrict__ scale,
                                       const float *__restrict__ shift, float4 *__restrict__ y,
                                       int quads, FastDiv div_plane, FastDiv div_c, int act) {
  pdl_launch_dependents();
  pdl_wait();
  const int stride = static_cast<int>(gridDim.x * blockDim.x);
  for (int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x); i < quads; i += stride) {
    const int plane = fdiv(i, div_plane);
    const int ch = plane - fdiv(plane, div_c) * static_cast<int>(div_c.d);
    const float sc = __ldg(scale + ch), sh = __ldg(shift + ch);
    float4 v = x[i];
    v.x = act_fn(fmaf(v.x, sc, sh), act);
    v.y = act_fn(fmaf(v.y, sc, sh), act);
    v.z = act_fn(fmaf(v.z, sc, sh), act);
    v.w = act_fn(fmaf(v.w, sc, sh), act);
    y[i] = v;
  }
}

// Per-channel affine over NCHW planes: block (x, plane) strides one plane.
__global__ void affine_nchw_kernel(const float *__restrict__ x, const float *__restrict__ scale,
                                   const float *__restrict__ shift, float *__restrict__ y,
                                   int64_t planes, int c, int64_t hw, int act) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t plane = blockIdx.y + static_cast<int64_t>(blockIdx.z) * gridDim.y;
  if (plane >= planes)
    return;
  const int ch = static_cast<int>(plane % c);
  const float sc = scale[ch], sh = shift[ch];
  const float *src = x + plane * hw;
  float *dst = y + plane * hw;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < hw;
       i += stride)
    dst[i] = act_fn(fmaf(src[i], sc, sh), act);
}

// Column-shard reassembly: src holds `ranks` blocks [rank][rows][cols] as an
// all-gather stacks them; dst is [rows][total] with block r in columns
// [r * cols, r * cols + cols) (columns at or past `total` are the last
// block's padding and are dropped).
__global__ void unshard_columns_kernel(const float *__restrict__ src, float *__restrict__ dst,
                                       int ranks, int64_t rows, int64_t cols, int64_t total) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t count = rows * total;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride) {
    const int64_t row = i / total, col = i - row * total;
    const int64_t r = col / cols, j = col - r * cols;
    dst[i] = src[(r * rows + row) * cols + j];
  }
}

int launched(const char *what) {
  return cuda_ok(cudaGetLastError(), what) ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

int bad(const char *what) {
  set_last_error(std::string("invalid arguments to ") + what);
  return CIM22_STATUS_BAD_ARGUMENT;
}

} // namespace
} // namespace cim

using namespace cim;

extern "C" {

int cim22_cuda_relu(const float *x, float *y, int64_t count, void *stream) {
  if (!x || !y || count < 0)
    return bad("cim22_cuda_relu");
  if (count == 0)
    return 0;
  launch_pdl(unary_kernel<CIM22_ACT_RELU>, grid_for((count + 3) / 4), 256, 0, static_cast<cudaStream_t>(stream), x, y, count);
  return launched("relu");
}

int cim22_cuda_gelu(const float *x, float *y, int64_t count, void *stream) {
  if (!x || !y || count < 0)
    return bad("cim22_cuda_gelu");
  if (count == 0)
    return 0;
  launch_pdl(unary_kernel<CIM22_ACT_GELU>, grid_for((count + 3) / 4), 256, 0, static_cast<cudaStream_t>(stream), x, y, count);
  return launched("gelu");
}

int cim22_cuda_add(const float *a, const float *b, float *y, int64_t count,
                   int32_t activation, void *stream) {
  if (!a || !b || !y || count < 0 || activation < 0 || activation > 2)
    return bad("cim22_cuda_add");
  if (count == 0)
    return 0;
  launch_pdl(add_kernel, grid_for(count), 256, 0, static_cast<cudaStream_t>(stream), a, b, y, count, activation);
  return launched("add");
}

int cim22_cuda_binary(const float *a, const float *b, float *y, int64_t count, int32_t op,
                      float a_scalar, float b_scalar, void *stream) {
  if (!y || count < 0 || op < CIM22_BINARY_ADD || op > CIM22_BINARY_MIN)
    return bad("cim22_cuda_binary");
  if (count == 0)
    return 0;
  launch_pdl(binary_kernel, grid_for(count), 256, 0, static_cast<cudaStream_t>(stream), a, b, y,
             count, static_cast<int>(op), a_scalar, b_scalar);
  return launched("binary");
}

int cim22_cuda_fill(float *y, int64_t count, float value, void *stream) {
  if (!y || count < 0)
    return bad("cim22_cuda_fill");
  if (count == 0)
    return 0;
  launch_pdl(fill_kernel, grid_for(count), 256, 0, static_cast<cudaStream_t>(stream), y, count,
             value);
  return launched("fill");
}

int cim22_cuda_copy(const void *src, void *dst, int64_t words, void *stream) {
  if (!src || !dst || words < 0)
    return bad("cim22_cuda_copy");
  if (words == 0 || src == dst)
    return 0;
  launch_pdl(copy_kernel, grid_for(words), 256, 0, static_cast<cudaStream_t>(stream),
             static_cast<const uint32_t *>(src), static_cast<uint32_t *>(dst), words);
  return launched("copy");
}

int cim22_cuda_slice_copy(const void *src, void *dst, int64_t blocks, int64_t inner,
                          int64_t src_stride, int64_t dst_stride, void *stream) {
  if (!src || !dst || blocks < 0 || inner < 0 || src_stride < 0 || dst_stride < 0)
    return bad("cim22_cuda_slice_copy");
  if (blocks == 0 || inner == 0)
    return 0;
  launch_pdl(slice_copy_kernel, grid_for(blocks * inner), 256, 0,
             static_cast<cudaStream_t>(stream), static_cast<const uint32_t *>(src),
             static_cast<uint32_t *>(dst), blocks, inner, src_stride, dst_stride);
  return launched("slice_copy");
}

int cim22_cuda_maxpool2d_nhwc(const float *x, float *y, int32_t n, int32_t h,
                              int32_t w, int32_t c, int32_t kernel,
                              int32_t stride, int32_t pad, void *stream) {
  if (!x || !y || n <= 0 || h <= 0 || w <= 0 || c <= 0 || kernel <= 0 ||
      stride <= 0 || pad < 0 || 2 * pad > kernel)
    return bad("cim22_cuda_maxpool2d_nhwc");
  const int oh = (h + 2 * pad - kernel) / stride + 1;
  const int ow = (w + 2 * pad - kernel) / stride + 1;
  if (oh <= 0 || ow <= 0)
    return bad("cim22_cuda_maxpool2d_nhwc");
  launch_pdl(maxpool_kernel, grid_for(static_cast<int64_t>(n) * oh * ow * c), 256, 0, static_cast<cudaStream_t>(stream), x, y, n, h, w, c, kernel,
                                                        stride, pad, oh, ow);
  return launched("maxpool2d");
}

int cim22_cuda_avgpool2d_nhwc(const float *x, float *y, int32_t n, int32_t h,
                              int32_t w, int32_t c, int32_t kernel,
                              int32_t stride, void *stream) {
  if (!x || !y || n <= 0 || h <= 0 || w <= 0 || c <= 0 || kernel <= 0 ||
      stride <= 0 || kernel > h || kernel > w)
    return bad("cim22_cuda_avgpool2d_nhwc");
  const int oh = (h - kernel) / stride + 1, ow = (w - kernel) / stride + 1;
  launch_pdl(avgpool_kernel, grid_for(static_cast<int64_t>(n) * oh * ow * c), 256, 0, static_cast<cudaStream_t>(stream), x, y, n, h, w, c, kernel,
                                                        stride, oh, ow);
  return launched("avgpool2d");
}

int cim22_cuda_global_avgpool_nhwc(const float *x, float *y, int32_t n,
                                   int32_t h, int32_t w, int32_t c,
                                   void *stream) {
  if (!x || !y || n <= 0 || h <= 0 || w <= 0 || c <= 0 || n > 65535 * 64)
    return bad("cim22_cuda_global_avgpool_nhwc");
  const dim3 grid(static_cast<unsigned>(n), static_cast<unsigned>((c + 31) / 32));
  launch_pdl(gap_kernel, grid, 256, 0, static_cast<cudaStream_t>(stream), x, y, h, w, c);
  return launched("global_avgpool");
}

int cim22_cuda_channel_affine_nhwc(const float *x, const float *scale,
                                   const float *shift, float *y, int64_t rows,
                                   int32_t c, int32_t activation, void *stream) {
  if (!x || !scale || !shift || !y || rows < 0 || c <= 0 || activation < 0 ||
      activation > 2)
    return bad("cim22_cuda_channel_affine_nhwc");
  if (rows == 0)
    return 0;
  launch_pdl(affine_kernel, grid_for(rows * c), 256, 0, static_cast<cudaStream_t>(stream), x, scale, shift, y, rows, c, activation);
  return launched("channel_affine");
}

int cim22_cuda_softmax(const float *x, float *y, int64_t rows, int32_t cols,
                       void *stream) {
  if (!x || !y || rows < 0 || cols <= 0)
    return bad("cim22_cuda_softmax");
  if (rows == 0)
    return 0;
  const unsigned blocks = static_cast<unsigned>((rows * 32 + 255) / 256);
  launch_pdl(softmax_kernel, blocks, 256, 0, static_cast<cudaStream_t>(stream), x, y, rows, cols);
  return launched("softmax");
}

int cim22_cuda_nhwc_to_nchw(const float *x, float *y, int32_t n, int32_t h,
                            int32_t w, int32_t c, void *stream) {
  if (!x || !y || n <= 0 || h <= 0 || w <= 0 || c <= 0)
    return bad("cim22_cuda_nhwc_to_nchw");
  launch_pdl(nhwc_to_nchw_kernel, grid_for(static_cast<int64_t>(n) * h * w * c), 256, 0, static_cast<cudaStream_t>(stream), x, y, n, h, w, c);
  return launched("nhwc_to_nchw");
}

int cim22_cuda_nchw_to_nhwc(const float *x, float *y, int32_t n, int32_t c,
                            int32_t h, int32_t w, void *stream) {
  if (!x || !y || n <= 0 || h <= 0 || w <= 0 || c <= 0)
    return bad("cim22_cuda_nchw_to_nhwc");
  launch_pdl(nchw_to_nhwc_kernel, grid_for(static_cast<int64_t>(n) * h * w * c), 256, 0, static_cast<cudaStream_t>(stream), x, y, n, c, h, w);
  return launched("nchw_to_nhwc");
}

int cim22_cuda_unshard_columns(const float *src, float *dst, int32_t ranks, int64_t rows,
                               int64_t cols, int64_t total, void *stream) {
  if (!src || !dst || ranks <= 0 || rows < 0 || cols <= 0 || total <= 0 ||
      total > static_cast<int64_t>(ranks) * cols)
    return bad("cim22_cuda_unshard_columns");
  if (rows == 0)
    return 0;
  launch_pdl(unshard_columns_kernel, grid_for(rows * total), 256, 0, static_cast<cudaStream_t>(stream), src, dst, ranks, rows, cols, total);
  return launched("unshard_columns");
}

int cim22_cuda_maxpool2d_nchw(const float *x, float *y, int32_t n, int32_t c,
                              int32_t h, int32_t w, int32_t kernel,
                              int32_t stride, int32_t pad, void *stream) {
  if (!x || !y || n <= 0 || h <= 0 || w <= 0 || c <= 0 || kernel <= 0 ||
      stride <= 0 || pad < 0 || 2 * pad > kernel)
    return bad("cim22_cuda_maxpool2d_nchw");
  const int oh = (h + 2 * pad - kernel) / stride + 1;
  const int ow = (w + 2 * pad - kernel) / stride + 1;
  if (oh <= 0 || ow <= 0)
    return bad("cim22_cuda_maxpool2d_nchw");
  const int64_t planes = static_cast<int64_t>(n) * c;
  launch_pdl(maxpool_nchw_kernel, grid_for(planes * oh * ow), 256, 0, static_cast<cudaStream_t>(stream), x, y, planes, h, w, kernel, stride, pad, oh, ow);
  return launched("maxpool2d");
}

int cim22_cuda_avgpool2d_nchw(const float *x, float *y, int32_t n, int32_t c,
                              int32_t h, int32_t w, int32_t kernel,
                              int32_t stride, void *stream) {
  if (!x || !y || n <= 0 || h <= 0 || w <= 0 || c <= 0 || kernel <= 0 ||
      stride <= 0 || kernel > h || kernel > w)
    return bad("cim22_cuda_avgpool2d_nchw");
  const int oh = (h - kernel) / stride + 1, ow = (w - kernel) / stride + 1;
  const int64_t planes = static_cast<int64_t>(n) * c;
  launch_pdl(avgpool_nchw_kernel, grid_for(planes * oh * ow), 256, 0, static_cast<cudaStream_t>(stream), x, y, planes, h, w, kernel, stride, oh, ow);
  return launched("avgpool2d");
}

int cim22_cuda_global_avgpool_nchw(const float *x, float *y, int32_t n,
                                   int32_t c, int32_t h, int32_t w,
                                   void *stream) {
  if (!x || !y || n <= 0 || h <= 0 || w <= 0 || c <= 0)
    return bad("cim22_cuda_global_avgpool_nchw");
  const int64_t planes = static_cast<int64_t>(n) * c;
  const int64_t hw = static_cast<int64_t>(h) * w;
  if (hw <= 64 && hw % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    launch_pdl(gap_nchw_small_kernel, static_cast<unsigned>((planes + 255) / 256), 256, 0,
               static_cast<cudaStream_t>(stream), reinterpret_cast<const float4 *>(x), y,
               planes, static_cast<int>(hw / 4));
    return launched("global_avgpool");
  }
  const unsigned blocks = static_cast<unsigned>((planes * 32 + 255) / 256);
  launch_pdl(gap_nchw_kernel, blocks, 256, 0, static_cast<cudaStream_t>(stream), x, y, planes, hw);
  return launched("global_avgpool");
}

int cim22_cuda_channel_affine_nchw(const float *x, const float *scale,
                                   const float *shift, float *y, int32_t n,
                                   int32_t c, int64_t hw, int32_t activation,
                                   void *stream) {
  if (!x || !scale || !shift || !y || n < 0 || c <= 0 || hw < 0 || activation < 0 ||
      activation > 2)
    return bad("cim22_cuda_channel_affine_nchw");
  const int64_t planes = static_cast<int64_t>(n) * c;
  if (planes == 0 || hw == 0)
    return 0;
  const int64_t quads = planes * hw / 4;
  if (hw % 4 == 0 && quads < (int64_t{1} << 31) && planes < (int64_t{1} << 31) &&
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0) {
    launch_pdl(affine_nchw_vec_kernel, grid_for(quads), 256, 0, static_cast<cudaStream_t>(stream), reinterpret_cast<const float4 *>(x), scale, shift, reinterpret_cast<float4 *>(y),
        static_cast<int>(quads), make_fastdiv(static_cast<uint32_t>(hw / 4)),
        make_fastdiv(static_cast<uint32_t>(c)), activation);
    return launched("channel_affine");
  }
  // Planes over grid.y and grid.z (blocks past the last plane return), the
  // plane itself over grid.x.
  const int64_t gy = std::min<int64_t>(planes, 65535);
  const int64_t gz = (planes + gy - 1) / gy;
  if (gz > 65535)
    return bad("cim22_cuda_channel_affine_nchw");
  const unsigned gx = static_cast<unsigned>(std::min<int64_t>((hw + 255) / 256, 64));
  launch_pdl(affine_nchw_kernel, dim3(gx, static_cast<unsigned>(gy), static_cast<unsigned>(gz)), 256, 0, static_cast<cudaStream_t>(stream), x, scale, shift, y, planes, c, hw,
                                                            activation);
  return launched("channel_affine");
}

} // extern "C"
