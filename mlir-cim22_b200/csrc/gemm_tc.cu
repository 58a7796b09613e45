// gemm_tc.cu - tcgen05 (5th-generation tensor core) CIM contractions, sm_100a.
//
// INT8 layers whose weights pass the signed-i21 range proof
// (lib/Conversion/LinalgToCIM/Passes.cpp:592-627) accumulate every 64-K
// crossbar partial exactly in int32, so the whole K range of a 128x128 output
// tile accumulates in one TMEM accumulator:
//
//   warp 0 (one thread)   TMA producer: A and B K-blocks of 128 bytes into a
//                          4-stage ring of 128B-swizzled shared-memory tiles
//   warp 1 (one thread)   tcgen05.mma.cta_group::1.kind::i8, M=128 N=128 K=32,
//                          4 MMAs per K-block, tcgen05.commit frees a stage
//   warps 2-5             epilogue: tcgen05.ld 32x32b from TMEM, int32 stores
//
// Every mbarrier wait is bounded in time (kWaitLimitNs of the global timer);
// a wait that runs out sets CIM22_STATUS_TIMEOUT, the CTA stops issuing work,
// waits (bounded) for the copies it has in flight, frees its TMEM and
// returns. Every load is a plain per-CTA copy into this CTA's shared memory.
#include "gemm_tc.h"

#include "cim_internal.h"
#include "cim_numeric.cuh"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>

namespace cim::tc {
namespace {

constexpr int kBM = 128, kBN = 128, kBK = 128, kStages = 4;
constexpr int kThreads = 192;
// Longest any single mbarrier wait may take before the kernel gives up.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint32_t kTileBytes = kBM * kBK; // A and B tiles are the same size

struct alignas(1024) SmemInt8 {
  int8_t a[kStages][kBM * kBK];
  int8_t b[kStages][kBN * kBK];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t done;
  uint32_t tmem;
  int failed;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity to complete, for at most
// limit_ns of the global timer (read once every 32 polls). Returns false
// when the limit was reached.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitLimitNs) {
  const uint32_t addr = smem_u32(bar);
  uint64_t start = 0;
  for (uint32_t i = 1;; ++i) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done)
                 : "r"(addr), "r"(parity)
                 : "memory");
    if (done)
      return true;
    if ((i & 31) == 0) {
      const uint64_t now = global_ns();
      if (start == 0)
        start = now;
      else if (now - start > limit_ns)
        return false;
    }
  }
}

// Dynamic shared memory rounded up to a 1024-byte boundary (the 128-byte
// swizzle atoms), derived from the extern array so that the compiler keeps
// addressing it as shared memory.
template <typename T> __device__ __forceinline__ T &smem_aligned(uint8_t *raw) {
  return *reinterpret_cast<T *>(raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u));
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128
// bytes in 8-row (1024-byte) atoms. Bits [0,14) address >> 4, [32,46) stride
// byte offset >> 4, [46,48) = 1, [61,64) layout (2 = SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(const void *tile) {
  const uint64_t addr = smem_u32(tile);
  return ((addr & 0x3ffffull) >> 4) | (uint64_t{1024 >> 4} << 32) | (uint64_t{1} << 46) |
         (uint64_t{2} << 61);
}

// Instruction descriptor of tcgen05.mma .kind::i8: D s32 (bits [4,6) = 2),
// A and B signed 8-bit (bits [7,10), [10,13) = 1), both K-major, N >> 3 at
// bit 17, M >> 4 at bit 24.
constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
               " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
               "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, "
               "%9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, "
               "%24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                 "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
                 "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                 "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                 "=r"(r[30]), "=r"(r[31])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    int8_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB, int num_kb, int64_t M, int64_t N,
                   const int32_t *__restrict__ bias, int64_t out_pixels, FastDiv div_pix,
                   int32_t *__restrict__ y, int32_t *status) {
  extern __shared__ uint8_t smem_raw[];
  SmemInt8 &s = smem_aligned<SmemInt8>(smem_raw);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m0 = static_cast<int>(blockIdx.x) * kBM;
  const int n0 = static_cast<int>(blockIdx.y) * kBN;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    mbar_init(&s.done, 1);
    s.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem)),
                 "r"(kBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s.tmem;

  if (warp == 0 && lane == 0) {
    // TMA producer.
    int issued = 0;
    for (int kb = 0; kb < num_kb; ++kb) {
      const int stage = kb % kStages;
      const uint32_t parity = ((kb / kStages) & 1) ^ 1;
      if (!mbar_wait(&s.empty[stage], parity)) {
        s.failed = 1;
        break;
      }
      if (*reinterpret_cast<volatile int *>(&s.failed))
        break;
      mbar_expect_tx(&s.full[stage], 2 * kTileBytes);
      tma_load_2d(s.a[stage], &tmA, &s.full[stage], kb * kBK, m0);
      tma_load_2d(s.b[stage], &tmB, &s.full[stage], kb * kBK, n0);
      issued = kb + 1;
    }
    // Never leave with copies in flight: wait (bounded) for the stages this
    // thread filled but the MMA thread may not have consumed.
    for (int kb = issued > kStages ? issued - kStages : 0; kb < issued; ++kb)
      mbar_wait(&s.full[kb % kStages], (kb / kStages) & 1);
  } else if (warp == 1 && lane == 0) {
    // MMA issuer.
    constexpr uint32_t idesc = idesc_i8(kBM, kBN);
    bool ok = true;
    for (int kb = 0; kb < num_kb && ok; ++kb) {
      const int stage = kb % kStages;
      if (!mbar_wait(&s.full[stage], (kb / kStages) & 1) ||
          *reinterpret_cast<volatile int *>(&s.failed)) {
        s.failed = 1;
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint64_t adesc = sw128_desc(s.a[stage]);
      const uint64_t bdesc = sw128_desc(s.b[stage]);
#pragma unroll
      for (int kk = 0; kk < kBK / 32; ++kk)
        mma_i8(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
      mma_commit(&s.empty[stage]);
    }
    mma_commit(&s.done);
  } else if (warp >= 2) {
    // Epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31 (= tile rows).
    const int quad = warp % 4;
    const bool ok = mbar_wait(&s.done, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ok || *reinterpret_cast<volatile int *>(&s.failed)) {
      if (lane == 0)
        atomicOr(status, CIM22_STATUS_TIMEOUT);
    } else {
      // Row r of the tile is column m0 + r; with out_pixels the output is
      // NCHW: column = image * out_pixels + pixel, lane = channel. The bias is
      // an exact wrapping int32 add, as the Host adds it.
      const int64_t row = m0 + quad * 32 + lane;
      int64_t base = row * N, step = 1;
      if (out_pixels > 0 && row < M) {
        const int64_t img = fdiv(static_cast<int>(row), div_pix);
        base = img * N * out_pixels + (row - img * out_pixels);
        step = out_pixels;
      }
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + c * 32, r);
        if (row < M) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int64_t n = n0 + c * 32 + j;
            if (n < N)
              y[base + n * step] =
                  static_cast<int32_t>(r[j] + (bias ? static_cast<uint32_t>(bias[n]) : 0u));
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBN));
  }
}

// ---------------------------------------------------------------------------
// BF16 sign-split contraction. Per 64-K crossbar tile t the two MMAs of each
// activation branch (xp, xn) produce 128 columns x 2L lanes of int32 dots in
// TMEM: one N=2L MMA covers both weight branches (L Wp rows, then L Wn rows).
// L = 32 lanes for 4-branch layers and 64 for 2-branch layers, so a TMEM
// buffer is 128 columns wide and every epilogue thread restores 32 dots per
// crossbar tile in both cases. The kernel is persistent: each CTA walks the
// output tiles (128 columns x L lanes) blockIdx.x, blockIdx.x + gridDim.x, ...
// and every crossbar tile of every output tile flows through three rings:
//
//   warp 0 (one thread)   TMA producer: per K-block of 128 bytes (two
//                          crossbar tiles) the activation tile of each branch
//                          and the stacked Wp/Wn tile into a 4-stage ring;
//                          per crossbar tile the activation exponents of the
//                          128 columns, the 2 x L weight scales and the tile's
//                          weight-exponent range into a 16-slot ring
//                          (cp.async.bulk, per CTA)
//   warp 1 (one thread)   tcgen05.mma kind::i8 into one of 4 TMEM buffers
//   warps 2-17            epilogue: warp w reads TMEM lanes 32 * (w % 4) and
//                          L / 4 of the L lanes; it restores each dot as
//                          RNE_bf16(Q(p) * 2^(Ew + Ex - 266)) and adds it to
//                          its f32 branch sum in tile order, then rounds,
//                          merges ((pp - pn) - np) + nn, adds the bias and
//                          applies the activation
//
// Inside the fast window (kScaleShift + 7 <= Ex <= kScaleShift + 111,
// 140 <= Ex + Ew <= 374 and Ew <= 260 - kScaleShift for every weight exponent
// of the tile) the restore is exact in three f32 operations on the dot p as
// read from TMEM: its bit pattern is the f32 subnormal p * 2^-149, so
// p * 2^(Ex + 16 - kScaleShift) = p * 2^(Ex - 133 - kScaleShift) is an exact
// normal f32; clearing its low 16 bits keeps Q(p) (the truncating INT21->BF16
// converter); and the product with the stored weight scale
// 2^(Ew - 133 + kScaleShift) is the exactly representable tile value
// Q(p) * 2^(Ex + Ew - 266), so one FMA adds it with the single rounding of the
// reference's f32 add. Outside the window the integer path (signsplit_tile)
// restores the tile.
constexpr int kSBM = 128, kSBK = 128, kSStages = 4;
constexpr int kEpiWarps = 16;
constexpr int kSThreads = 64 + 32 * kEpiWarps;
constexpr int kExpSlots = 16, kTmemBufs = 4;
constexpr uint32_t kBufCols = 128;
constexpr int kParamLanes = 512;

template <int kAB> struct SSShape {
  static constexpr int L = kAB == 1 ? 64 : 32; // lanes per output tile
  static constexpr int LT = L / 4;             // lanes per epilogue thread
  static constexpr int N = 2 * L;              // MMA N: Wp and Wn rows
};

// One kScaleBlockWords weight record: the epilogue scales
// 2^(Ew - 133 + kScaleShift) of a 32-lane block's Wp and Wn lanes and the
// block's weight-exponent range {min, max, ex_lo, ex_hi}.
struct alignas(16) ExpBlock {
  float w[2][32];
  int32_t range[4];
};
static_assert(sizeof(ExpBlock) == kScaleBlockWords * 4, "weight record layout");

struct alignas(16) ExpSlot {
  int32_t a[2][kSBM]; // activation group exponents per branch
  ExpBlock blk[2];    // the tile's weight records of the output tile's 32-lane blocks
};

template <int kAB> struct alignas(1024) SmemSS {
  int8_t a[kSStages][kAB][kSBM * kSBK];
  int8_t b[kSStages][SSShape<kAB>::N * kSBK];
  ExpSlot ex[kExpSlots];
  uint64_t full[kSStages];
  uint64_t empty[kSStages];
  uint64_t exfull[kExpSlots];
  uint64_t exempty[kExpSlots];
  uint64_t dfull[kTmemBufs];
  uint64_t dempty[kTmemBufs];
  uint32_t tmem;
  int failed;
  // Bias, batch-norm scale and shift of every lane (layers of at most
  // kParamLanes lanes), copied once per CTA for the output stores.
  alignas(16) float lane_params[3][kParamLanes];
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], "
               "%2, [%3];" ::"r"(smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Issue a 32x32b TMEM load of 8 columns; the values are valid after
// tmem_wait.
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// Wait for the outstanding TMEM loads. The registers are in/out operands so
// no use of them is scheduled before the wait.
__device__ __forceinline__ void tmem_wait(uint32_t (&r)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7])::"memory");
}

// tcgen05.ld of 16 columns and the wait for it in one statement, so the
// registers are written once.
__device__ __forceinline__ void tmem_ld_wait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, "
               "%9, %10, %11, %12, %13, %14, %15}, [%16];\n"
               "tcgen05.wait::ld.sync.aligned;"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                 "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(taddr)
               : "memory");
}

// Exact restore of one tile value outside the fast window (out of line).
__device__ __noinline__ float tc_slow_tile_add(float acc, int p, int ew, int ex,
                                               int32_t *status) {
  const uint16_t tile = signsplit_tile(static_cast<uint32_t>(p), ew, ex);
  if (tile == kBF16Inf)
    atomicOr(status, CIM22_STATUS_TILE_OVERFLOW);
  return __fadd_rn(acc, bf16_to_f32(tile));
}

__device__ __forceinline__ float act_tc(float v, int act) {
  if (act == CIM22_ACT_RELU)
    return (v > 0.0f || v != v) ? v : 0.0f; // NaN propagates, as torch.relu
  if (act == CIM22_ACT_GELU)
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  return v;
}

// Add the restored dots of one (activation branch, weight branch) pair of a
// crossbar tile to the branch sums, three f32 operations per dot:
//   v = p_bits * sx      (p_bits: the dot's bit pattern, the subnormal
//                         p * 2^-149; sx = 2^(Ex + 16 - kScaleShift)), exact
//   q = v with its low 16 bits cleared = Q(p) * 2^(Ex - 133 - kScaleShift)
//   acc = fma(q, sw, acc) (sw = 2^(Ew - 133 + kScaleShift)), one rounding
// Rows outside the fast window carry sx = 0, so their sums gain exactly +0
// here and restore_slow_rows then adds their tile values; all sums are >= +0.
// sw points at the tile's weight scales in shared memory (16-byte aligned).
// The sums start at +0 for each output tile: fma(q, sw, +0) of the first
// crossbar tile is the exact q * sw (one code path for every tile, measured
// faster than a first-tile multiply).
template <int kLT>
__device__ __forceinline__ void restore_fast(float (&acc)[kLT], const uint32_t (&p)[kLT],
                                             float sx, const float *__restrict__ sw) {
#pragma unroll
  for (int j4 = 0; j4 < kLT; j4 += 4) {
    const float4 s4 = *reinterpret_cast<const float4 *>(sw + j4);
    const float s[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float v = __fmul_rn(__uint_as_float(p[j4 + j]), sx);
      const float q = __uint_as_float(__float_as_uint(v) & 0xffff0000u);
      acc[j4 + j] = __fmaf_rn(q, s[j], acc[j4 + j]);
    }
  }
}

// The exact integer restore of the tile values of rows outside the fast
// window (subnormal or overflowing tiles), added to sums that the fast pass
// left unchanged for them.
template <int kLT>
__device__ __forceinline__ void restore_slow_rows(float (&acc)[kLT], const uint32_t (&p)[kLT],
                                                  const int32_t *__restrict__ exB,
                                                  int64_t ew_index, int ex, int32_t *status) {
#pragma unroll
  for (int j = 0; j < kLT; ++j)
    acc[j] = tc_slow_tile_add(acc[j], static_cast<int>(p[j]), exB[ew_index + j], ex, status);
}

// Address of the residual addend of one output row's first lane (laid out
// like y: rows, or NCHW planes) and the stride between lanes.
__device__ __forceinline__ const float *residual_row(const float *residual, int row, int lane0,
                                                     int N, int out_pixels, FastDiv div_pix,
                                                     int64_t &lane_stride) {
  int64_t base = static_cast<int64_t>(row) * N + lane0;
  lane_stride = 1;
  if (out_pixels > 0) {
    const int image = fdiv(row, div_pix);
    base = (static_cast<int64_t>(image) * N + lane0) * out_pixels + (row - image * out_pixels);
    lane_stride = out_pixels;
  }
  return residual + base;
}

// Pull one output row's residual addends into L2 when its output tile
// starts, so that the epilogue's loads of them do not wait on HBM.
template <int LT>
__device__ __forceinline__ void prefetch_residual(const float *residual, int row, int lane0,
                                                  int M, int N, int out_pixels,
                                                  FastDiv div_pix) {
  if (residual == nullptr || row >= M)
    return;
  int64_t stride;
  const float *p = residual_row(residual, row, lane0, N, out_pixels, div_pix, stride);
#pragma unroll
  for (int j = 0; j < LT; ++j)
    if (lane0 + j < N)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p + j * stride));
}

// Final merge of one output row's LT lanes: BF16 rounding of each branch sum
// when there is more than one K tile, ((pp - pn) - np) + nn, bias, the
// optional per-lane fma, the optional residual add, the activation, then the
// store - rows, or NCHW
// planes where a warp's 32 consecutive rows store 32 consecutive floats of a
// lane. The branch sums are finite or infinite, never NaN, so the hardware
// RNE conversion rounds them as the reference's truncf does. cache, when not
// null, holds the bias, scale and shift of every lane in shared memory.
template <int kAB, int LT>
__device__ __forceinline__ void tile_values(float (&acc)[kAB][2][LT], int row, int lane0, int N,
                                            int T, const float (*cache)[kParamLanes],
                                            const float *__restrict__ bias,
                                            const float *__restrict__ post_scale,
                                            const float *__restrict__ post_shift,
                                            const float *__restrict__ residual, int act, int vec,
                                            int out_pixels, FastDiv div_pix, float (&o)[LT],
                                            const float *res_tile = nullptr,
                                            int res_stride = 0) {
  if (T > 1) {
#pragma unroll
    for (int a = 0; a < kAB; ++a)
#pragma unroll
      for (int w = 0; w < 2; ++w)
#pragma unroll
        for (int j = 0; j < LT; j += 2) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(acc[a][w][j], acc[a][w][j + 1]);
          acc[a][w][j] = __low2float(h);
          acc[a][w][j + 1] = __high2float(h);
        }
  }
#pragma unroll
  for (int j = 0; j < LT; ++j) {
    o[j] = __fsub_rn(acc[0][0][j], acc[0][1][j]);
    if (kAB == 2)
      o[j] = __fadd_rn(__fsub_rn(o[j], acc[kAB - 1][0][j]), acc[kAB - 1][1][j]);
  }
  const bool full = lane0 + LT <= N;
  if (bias != nullptr) {
    if (cache != nullptr && full) {
#pragma unroll
      for (int j4 = 0; j4 < LT; j4 += 4) {
        const float4 b = *reinterpret_cast<const float4 *>(&cache[0][lane0 + j4]);
        o[j4] = __fadd_rn(o[j4], b.x);
        o[j4 + 1] = __fadd_rn(o[j4 + 1], b.y);
        o[j4 + 2] = __fadd_rn(o[j4 + 2], b.z);
        o[j4 + 3] = __fadd_rn(o[j4 + 3], b.w);
      }
    } else if (full && (vec & 1)) {
#pragma unroll
      for (int j4 = 0; j4 < LT; j4 += 4) {
        const float4 b = __ldg(reinterpret_cast<const float4 *>(bias + lane0 + j4));
        o[j4] = __fadd_rn(o[j4], b.x);
        o[j4 + 1] = __fadd_rn(o[j4 + 1], b.y);
        o[j4 + 2] = __fadd_rn(o[j4 + 2], b.z);
        o[j4 + 3] = __fadd_rn(o[j4 + 3], b.w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < LT; ++j)
        if (lane0 + j < N)
          o[j] = __fadd_rn(o[j], __ldg(bias + lane0 + j));
    }
  }
  if (post_scale != nullptr) {
    if (cache != nullptr && full) {
#pragma unroll
      for (int j4 = 0; j4 < LT; j4 += 4) {
        const float4 sc = *reinterpret_cast<const float4 *>(&cache[1][lane0 + j4]);
        const float4 sh = *reinterpret_cast<const float4 *>(&cache[2][lane0 + j4]);
        o[j4] = __fmaf_rn(o[j4], sc.x, sh.x);
        o[j4 + 1] = __fmaf_rn(o[j4 + 1], sc.y, sh.y);
        o[j4 + 2] = __fmaf_rn(o[j4 + 2], sc.z, sh.z);
        o[j4 + 3] = __fmaf_rn(o[j4 + 3], sc.w, sh.w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < LT; ++j)
        if (lane0 + j < N)
          o[j] = __fmaf_rn(o[j], __ldg(post_scale + lane0 + j), __ldg(post_shift + lane0 + j));
    }
  }
  if (res_tile != nullptr) {
    // The residual addends of the row's lanes, staged in shared memory by
    // TMA while the output tile was computed: one f32 add as the glue.
#pragma unroll
    for (int j = 0; j < LT; ++j)
      if (lane0 + j < N)
        o[j] = __fadd_rn(o[j], res_tile[j * res_stride]);
  } else if (residual != nullptr) {
    // A residual add fused after the batch norm (prefetched into L2 when the
    // output tile started): one f32 add as the glue computes it.
    int64_t stride;
    const float *p = residual_row(residual, row, lane0, N, out_pixels, div_pix, stride);
#pragma unroll
    for (int j = 0; j < LT; ++j)
      if (lane0 + j < N)
        o[j] = __fadd_rn(o[j], __ldg(p + j * stride));
  }
  if (act == CIM22_ACT_RELU) {
#pragma unroll
    for (int j = 0; j < LT; ++j)
      o[j] = (o[j] > 0.0f || o[j] != o[j]) ? o[j] : 0.0f; // NaN propagates
  } else if (act == CIM22_ACT_GELU) {
#pragma unroll
    for (int j = 0; j < LT; ++j)
      o[j] = act_tc(o[j], CIM22_ACT_GELU);
  }
}

template <int kAB, int LT>
__device__ __forceinline__ void store_tile(float (&acc)[kAB][2][LT], int row, int lane0, int M,
                                           int N, int T, const float (*cache)[kParamLanes],
                                           const float *__restrict__ bias,
                                           const float *__restrict__ post_scale,
                                           const float *__restrict__ post_shift,
                                           const float *__restrict__ residual, int act,
                                           int vec, int out_pixels, FastDiv div_pix,
                                           float *__restrict__ y,
                                           const float *res_tile = nullptr,
                                           int res_stride = 0) {
  if (row >= M)
    return;
  float o[LT];
  tile_values<kAB, LT>(acc, row, lane0, N, T, cache, bias, post_scale, post_shift, residual, act,
                       vec, out_pixels, div_pix, o, res_tile, res_stride);
  const bool full = lane0 + LT <= N;
  if (out_pixels > 0) {
    const int image = fdiv(row, div_pix);
    float *dst = y + (static_cast<int64_t>(image) * N + lane0) * out_pixels +
                 (row - image * out_pixels);
#pragma unroll
    for (int j = 0; j < LT; ++j)
      if (lane0 + j < N)
        dst[static_cast<int64_t>(j) * out_pixels] = o[j];
  } else {
    float *dst = y + static_cast<int64_t>(row) * N + lane0;
    if (full && (vec & 2)) {
#pragma unroll
      for (int j4 = 0; j4 < LT; j4 += 4)
        *reinterpret_cast<float4 *>(dst + j4) = make_float4(o[j4], o[j4 + 1], o[j4 + 2], o[j4 + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < LT; ++j)
        if (lane0 + j < N)
          dst[j] = o[j];
    }
  }
}

// store_tile for a column-sharded layer: the row's LT lanes go into every
// rank's full output (peer memory mapped on this device) at the rank's lane
// offset; lanes at or past peers.lanes are padding and are not stored.
// vec4: row_stride, lane_offset and every output base allow float4 stores.
template <int kAB, int LT>
__device__ __forceinline__ void store_tile_peers(float (&acc)[kAB][2][LT], int row, int lane0,
                                                 int M, int N, int T,
                                                 const float (*cache)[kParamLanes],
                                                 const float *__restrict__ bias,
                                                 const float *__restrict__ post_scale,
                                                 const float *__restrict__ post_shift, int act,
                                                 int vec, const cim22_peer_outputs &peers,
                                                 bool vec4) {
  if (row >= M)
    return;
  float o[LT];
  tile_values<kAB, LT>(acc, row, lane0, N, T, cache, bias, post_scale, post_shift, nullptr, act,
                       vec, 0, FastDiv{1, 0, 0}, o);
  const int64_t off = static_cast<int64_t>(row) * peers.row_stride + peers.lane_offset + lane0;
  const bool full = lane0 + LT <= peers.lanes;
  for (int p = 0; p < peers.ranks; ++p) {
    float *dst = peers.out[p] + off;
    if (full && vec4) {
#pragma unroll
      for (int j4 = 0; j4 < LT; j4 += 4)
        *reinterpret_cast<float4 *>(dst + j4) = make_float4(o[j4], o[j4 + 1], o[j4 + 2], o[j4 + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < LT; ++j)
        if (lane0 + j < peers.lanes)
          dst[j] = o[j];
    }
  }
}

// kRes: the layer has a residual addend (a separate instance, so that layers
// without one keep the registers the residual path would take).
template <int kAB, bool kRes>
__global__ void __launch_bounds__(kSThreads, 1)
    signsplit_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const int32_t *__restrict__ exA,
                        int m_pad, const int32_t *__restrict__ exB, int n_pad, int T, int M,
                        int N, FastDiv div_nb, const float *__restrict__ bias,
                        const float *__restrict__ post_scale,
                        const float *__restrict__ post_shift,
                        const float *__restrict__ residual_arg, int act, int vec,
                        int out_pixels, FastDiv div_pix, float *__restrict__ y,
                        int32_t *status) {
  const float *residual = kRes ? residual_arg : nullptr;
  using S = SSShape<kAB>;
  constexpr int L = S::L, LT = S::LT, SN = S::N;
  extern __shared__ uint8_t smem_raw[];
  SmemSS<kAB> &s = smem_aligned<SmemSS<kAB>>(smem_raw);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int num_kb = (T + 1) / 2;
  const int num_nb = (N + L - 1) / L;
  const int num_tiles = ((M + kSBM - 1) / kSBM) * num_nb;
  const int32_t *ranges = exB + int64_t{2} * T * n_pad; // [T][n_pad / 32][4]
  // The epilogue's weight scales 2^(Ew - 133 + kScaleShift) follow the plain
  // scales 2^(Ew - 133) [2][T][n_pad] that the CUDA-core kernels read.
  const float *scales =
      reinterpret_cast<const float *>(ranges + int64_t{n_pad / 32} * T * 4) + 2 * T * n_pad;
  // Then the per-(tile, 32-lane block) weight records.
  const int32_t *wrecs = reinterpret_cast<const int32_t *>(scales) + 2 * T * n_pad;
  constexpr uint32_t kTmemCols = kTmemBufs * kBufCols;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < kExpSlots; ++i) {
      mbar_init(&s.exfull[i], 1);
      mbar_init(&s.exempty[i], kEpiWarps);
    }
    for (int i = 0; i < kTmemBufs; ++i) {
      mbar_init(&s.dfull[i], 1);
      mbar_init(&s.dempty[i], kEpiWarps);
    }
    s.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  // The per-lane epilogue parameters are resident constants of the layer
  // (no earlier kernel writes them), so they are copied before the PDL wait.
  const bool cached = N <= kParamLanes;
  if (cached)
    for (int i = threadIdx.x; i < N; i += kSThreads) {
      s.lane_params[0][i] = bias ? bias[i] : 0.0f;
      s.lane_params[1][i] = post_scale ? post_scale[i] : 0.0f;
      s.lane_params[2][i] = post_shift ? post_shift[i] : 0.0f;
    }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s.tmem;
  volatile int *failed = &s.failed;
  // Barriers and TMEM are set up; everything below touches memory that
  // earlier kernels write.
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0 && lane == 0) {
    // Ring positions and phase parities advance incrementally (this
    // thread's per-tile instruction chain is on the kernel's critical path);
    // a failure elsewhere shows up as a bounded wait that runs out.
    uint32_t kbi = 0, gi = 0, stage = 0, sphase = 0, slot = 0, xphase = 0;
    bool ok = true;
    for (int ot = blockIdx.x; ot < num_tiles && ok; ot += gridDim.x) {
      const int mb = fdiv(ot, div_nb);
      const int m0 = mb * kSBM, nb = ot - mb * num_nb, n0 = nb * L;
      const int32_t *wrec = wrecs + static_cast<int64_t>(n0 / 32) * kScaleBlockWords;
      for (int kb = 0; kb < num_kb; ++kb, ++kbi) {
        if (!mbar_wait(&s.empty[stage], sphase ^ 1)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&s.full[stage], kAB * kSBM * kSBK + SN * kSBK);
#pragma unroll
        for (int a = 0; a < kAB; ++a)
          tma_load_2d(s.a[stage][a], &tmA, &s.full[stage], kb * kSBK, a * m_pad + m0);
        tma_load_2d(s.b[stage], &tmB, &s.full[stage], kb * kSBK, n0);
        tma_load_2d(s.b[stage] + L * kSBK, &tmB, &s.full[stage], kb * kSBK, n_pad + n0);
        if (++stage == kSStages) {
          stage = 0;
          sphase ^= 1;
        }
        for (int t = 2 * kb; t < 2 * kb + 2 && t < T; ++t, ++gi) {
          if (!mbar_wait(&s.exempty[slot], xphase ^ 1)) {
            ok = false;
            break;
          }
          ExpSlot &e = s.ex[slot];
          mbar_expect_tx(&s.exfull[slot], kAB * kSBM * 4 + (L / 32) * kScaleBlockWords * 4);
#pragma unroll
          for (int a = 0; a < kAB; ++a)
            bulk_load(e.a[a], exA + (static_cast<int64_t>(a) * T + t) * m_pad + m0, kSBM * 4,
                      &s.exfull[slot]);
          bulk_load(e.blk, wrec + static_cast<int64_t>(t) * (n_pad / 32) * kScaleBlockWords,
                    (L / 32) * kScaleBlockWords * 4, &s.exfull[slot]);
          if (++slot == kExpSlots) {
            slot = 0;
            xphase ^= 1;
          }
        }
        if (!ok) {
          ++kbi;
          break;
        }
      }
    }
    if (!ok)
      *failed = 1;
    // Never leave with copies in flight: wait (bounded) for the stages and
    // exponent slots this thread filled but the consumers may not have used.
    for (uint32_t i = kbi > kSStages ? kbi - kSStages : 0; i < kbi; ++i)
      mbar_wait(&s.full[i % kSStages], (i / kSStages) & 1);
    for (uint32_t i = gi > kExpSlots ? gi - kExpSlots : 0; i < gi; ++i)
      mbar_wait(&s.exfull[i % kExpSlots], (i / kExpSlots) & 1);
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: two K=32 MMAs per branch per crossbar tile.
    // The kernel's critical path: ring positions advance incrementally and
    // the descriptors step by constant strides.
    constexpr uint32_t idesc = idesc_i8(kSBM, SN);
    constexpr uint64_t kAStep = sizeof(s.a[0]) >> 4, kBStep = sizeof(s.b[0]) >> 4;
    const uint64_t adesc0 = sw128_desc(s.a[0][0]), bdesc0 = sw128_desc(s.b[0]);
    uint32_t kbi = 0, gi = 0, stage = 0, sphase = 0, buf = 0, dphase = 0;
    bool ok = true;
    for (int ot = blockIdx.x; ot < num_tiles && ok; ot += gridDim.x) {
      for (int t = 0; t < T; ++t, ++gi) {
        const int half = t & 1;
        if ((half == 0 && !mbar_wait(&s.full[stage], sphase)) ||
            !mbar_wait(&s.dempty[buf], dphase ^ 1)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t bdesc = bdesc0 + stage * kBStep + half * 4;
#pragma unroll
        for (int a = 0; a < kAB; ++a) {
          const uint64_t adesc = adesc0 + stage * kAStep + a * (kSBM * kSBK >> 4) + half * 4;
          const uint32_t d = tmem + buf * kBufCols + a * SN;
          mma_i8(d, adesc, bdesc, idesc, 0u);
          mma_i8(d, adesc + 2, bdesc + 2, idesc, 1u);
        }
        mma_commit(&s.dfull[buf]);
        if (half == 1 || t == T - 1) {
          mma_commit(&s.empty[stage]);
          ++kbi;
          if (++stage == kSStages) {
            stage = 0;
            sphase ^= 1;
          }
        }
        if (++buf == kTmemBufs) {
          buf = 0;
          dphase ^= 1;
        }
      }
    }
    if (!ok)
      *failed = 1;
    // Let the last MMAs land before TMEM is freed.
    if (gi > 0)
      mbar_wait(&s.dfull[(gi - 1) % kTmemBufs], ((gi - 1) / kTmemBufs) & 1);
  } else if (warp >= 2) {
    // Epilogue.
    const int quad = warp % 4, sub = (warp - 2) / 4;
    const int row_local = quad * 32 + lane;
    const uint32_t tlane = static_cast<uint32_t>(quad * 32) << 16;
    // The thread's lanes within the output tile: record (sub * LT) / 32 of
    // a tile's weight records, from lane (sub * LT) % 32 on.
    const int rec = (sub * LT) >> 5, rec_lane = (sub * LT) & 31;
    uint32_t gi = 0, buf = 0, dphase = 0, slot = 0, xphase = 0;
    bool ok = true;
    for (int ot = blockIdx.x; ot < num_tiles && ok; ot += gridDim.x) {
      const int mb = fdiv(ot, div_nb);
      const int m0 = mb * kSBM, n0 = (ot - mb * num_nb) * L;
      const int lane0 = n0 + sub * LT;
      prefetch_residual<LT>(residual, m0 + row_local, lane0, M, N, out_pixels, div_pix);
      float acc[kAB][2][LT];
#pragma unroll
      for (int a = 0; a < kAB; ++a)
#pragma unroll
        for (int w = 0; w < 2; ++w)
#pragma unroll
          for (int j = 0; j < LT; ++j)
            acc[a][w][j] = 0.0f;
      // Two crossbar tiles per iteration for 4-branch layers (measured 2%
      // faster there; 2-branch layers run slower unrolled).
#pragma unroll(kAB == 2 ? 2 : 1)
      for (int t = 0; t < T; ++t, ++gi) {
        // A failure elsewhere in the CTA shows up here as a wait that runs
        // out, so the per-tile waits do not poll the failure flag.
        if (!mbar_wait(&s.exfull[slot], xphase)) {
          ok = false;
          break;
        }
        const ExpSlot &e = s.ex[slot];
        // Fast window for this tile's weights, ex_lo <= Ex <= ex_hi: the
        // intersection of its 32-lane blocks' windows (tabulated at load).
        int ex_lo = e.blk[0].range[2], ex_hi = e.blk[0].range[3];
        if (L == 64) {
          ex_lo = max(ex_lo, e.blk[1].range[2]);
          ex_hi = min(ex_hi, e.blk[1].range[3]);
        }
        float sx[kAB];
        bool fast[kAB];
        int ex[kAB];
#pragma unroll
        for (int a = 0; a < kAB; ++a) {
          ex[a] = e.a[a][row_local];
          const bool zero = ex[a] == kZeroGroup;
          const bool window = ex[a] >= ex_lo && ex[a] <= ex_hi;
          fast[a] = zero || window;
          // 2^(Ex - 133), a normal f32 inside the window (Ex >= 7).
          // 2^(Ex + 16 - kScaleShift), a normal f32 inside the window.
          sx[a] = window && !zero
                      ? __uint_as_float(static_cast<uint32_t>(ex[a] + 143 - kScaleShift) << 23)
                      : 0.0f;
        }
        if (!mbar_wait(&s.dfull[buf], dphase)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t col0 = tmem + tlane + buf * kBufCols + sub * LT;
        if constexpr (kAB == 1) {
          // 2-branch layers (LT = 16): one weight sign at a time, 16 dots in
          // registers (measured faster than both signs at once: fewer live
          // registers under the 96-register budget of 576 threads).
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            uint32_t p[LT];
            tmem_ld_wait(col0 + w * L, p);
            restore_fast<LT>(acc[0][w], p, sx[0], &e.blk[rec].w[w][rec_lane]);
            // One warp-uniform test: rows outside the window (rare) add their
            // exact tile values to the sums the fast pass kept.
            if (__any_sync(0xffffffffu, !fast[0])) {
              if (!fast[0])
                restore_slow_rows<LT>(acc[0][w], p, exB,
                                      (static_cast<int64_t>(w) * T + t) * n_pad + lane0, ex[0],
                                      status);
            }
          }
        } else {
          // 4-branch layers (LT = 8): both weight signs of one activation
          // branch at a time, 2 x 8 dots in registers.
#pragma unroll
          for (int a = 0; a < kAB; ++a) {
            uint32_t p0[LT], p1[LT];
            tmem_ld(col0 + a * SN, p0);
            tmem_ld(col0 + a * SN + L, p1);
            tmem_wait(p0);
            tmem_wait(p1);
            restore_fast<LT>(acc[a][0], p0, sx[a], &e.blk[rec].w[0][rec_lane]);
            restore_fast<LT>(acc[a][1], p1, sx[a], &e.blk[rec].w[1][rec_lane]);
            if (__any_sync(0xffffffffu, !fast[a])) {
              if (!fast[a]) {
                const int64_t ew0 = static_cast<int64_t>(t) * n_pad + lane0;
                restore_slow_rows<LT>(acc[a][0], p0, exB, ew0, ex[a], status);
                restore_slow_rows<LT>(acc[a][1], p1, exB, ew0 + static_cast<int64_t>(T) * n_pad,
                                      ex[a], status);
              }
            }
          }
        }
        // Hand the TMEM buffer and the exponent slot back once every lane
        // has read them.
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s.dempty[buf]);
          mbar_arrive(&s.exempty[slot]);
        }
        if (++buf == kTmemBufs) {
          buf = 0;
          dphase ^= 1;
        }
        if (++slot == kExpSlots) {
          slot = 0;
          xphase ^= 1;
        }
      }
      if (!ok)
        break;
      store_tile<kAB, LT>(acc, m0 + row_local, lane0, M, N, T,
                          cached ? s.lane_params : nullptr, bias, post_scale, post_shift,
                          residual, act, vec, out_pixels, div_pix, y);
    }
    if (!ok) {
      *failed = 1;
      if (lane == 0)
        atomicOr(status, CIM22_STATUS_TIMEOUT);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// BF16 sign-split contraction with BF16 operands. The prepare stores each
// activation group as BF16 values a * 2^(Ex - 133) (a: the ExpPrealign
// mantissas, 0..127) and the layer stores its weights as b * 2^(Ew - 133);
// every product a * b * 2^(Ex + Ew - 266) and every partial sum is then an
// integer multiple of 2^(Ex + Ew - 266) below 2^20 of them, which the
// tensor core's f32 accumulation holds exactly. So a tcgen05.mma kind::f16
// leaves each crossbar dot in TMEM as the exact f32 value
// v = p * 2^(Ex + Ew - 266), normal and finite inside the layer's window
// (ex_lo <= Ex <= ex_hi, which the layer derives from its weight exponents
// so that 140 <= Ex + Ew <= 374 for every lane). The restore of the
// reference - RNE_bf16(Q(p) * 2^(Ew + Ex - 266)), Q keeping the top 8 bits of
// p - is then v with its low 16 bits cleared (exactly representable), and
// the tile-order f32 sum adds it with one rounding: two operations per dot,
// no per-tile scales.
//
// Groups outside the window are stored unscaled (a itself), so their dots
// arrive as p * 2^(Ew - 133) (exact: the layer's weight exponents lie in
// [kOperandEwMin, kOperandEwMax]); a row of such a group takes the exact
// integer restore for that tile. The epilogue tells them apart by the group
// exponents, which the producer copies per tile into a 16-slot ring that the
// epilogue releases (a load per tile from global memory would put its
// latency on every tile).
//
// Same warp roles, TMEM buffers and output stores as signsplit_tc_kernel; the
// ring holds one crossbar tile per stage (128 bytes of K per row) and the MMA
// warp issues four K=16 MMAs per activation branch and tile.
// kRes: the layer has a residual addend, which one epilogue thread loads per
// output tile into shared memory by TMA (NCHW outputs whose 128-row tiles
// cover whole images or runs of one image); the ring gives up a stage for it
// where shared memory is short.
template <int kAB, bool kRes> struct SBShape {
  static constexpr int kStages = kAB == 1 ? (kRes ? 5 : 6) : 4;
  static constexpr int kExSlots = 16;                       // activation exponent ring
  static constexpr int kATile = kSBM * 64;                  // BF16 elements per branch
  static constexpr int kBTile = SSShape<kAB>::N * 64;       // BF16 elements
  static constexpr int kResTile = kRes ? kSBM * SSShape<kAB>::L : 4; // f32 addends
};

template <int kAB, bool kRes> struct alignas(1024) SmemSB {
  using Shape = SBShape<kAB, kRes>;
  uint16_t a[Shape::kStages][kAB][Shape::kATile];
  uint16_t b[Shape::kStages][Shape::kBTile];
  int32_t exa[Shape::kExSlots][kAB][kSBM];
  alignas(128) float res[Shape::kResTile]; // [images][lanes][pixels] of the tile
  uint64_t full[Shape::kStages];
  uint64_t empty[Shape::kStages];
  uint64_t exfull[Shape::kExSlots];
  uint64_t exempty[Shape::kExSlots];
  uint64_t dfull[kTmemBufs];
  uint64_t dempty[kTmemBufs];
  uint64_t rfull, rempty;
  uint32_t tmem;
  int failed;
  alignas(16) float lane_params[3][kParamLanes];
};

// A 3-D tiled bulk-tensor load into this CTA's shared memory (no cluster
// forms); x must be 16-byte aligned in bytes.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Instruction descriptor of tcgen05.mma .kind::f16 with BF16 A and B and an
// f32 accumulator: D format (bits [4,6)) 1 = F32, A and B formats (bits
// [7,10), [10,13)) 1 = BF16, both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
               " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
               "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Add one (activation branch, weight sign) slice of a crossbar tile to the
// branch sums: q = v with its low 16 bits cleared, acc += q (the sums start
// at +0 for each output tile). kPacked: two lanes per packed f32x2 add, each
// half rounding as the scalar f32 add.
template <int kLT, bool kPacked>
__device__ __forceinline__ void restore_b16(float (&acc)[kLT], const uint32_t (&v)[kLT]) {
  static_assert(kLT % 2 == 0, "lanes come in pairs");
  if constexpr (kPacked) {
#pragma unroll
    for (int j = 0; j < kLT; j += 2)
      add2(acc[j], acc[j + 1], __uint_as_float(v[j] & 0xffff0000u),
           __uint_as_float(v[j + 1] & 0xffff0000u), acc[j], acc[j + 1]);
  } else {
#pragma unroll
    for (int j = 0; j < kLT; ++j)
      acc[j] = __fadd_rn(acc[j], __uint_as_float(v[j] & 0xffff0000u));
  }
}

// The same slice when some row of the warp holds an unscaled group: this
// thread's row restores p = v * 2^(133 - Ew) exactly through the integer path
// when `raw`, else as restore_b16.
template <int kLT>
__device__ __forceinline__ void restore_b16_raw(float (&acc)[kLT], const uint32_t (&v)[kLT],
                                             bool raw, const int32_t *__restrict__ exB,
                                             int64_t ew_index, int ex, int32_t *status) {
  if (!raw) {
    restore_b16<kLT, false>(acc, v);
    return;
  }
#pragma unroll
  for (int j = 0; j < kLT; ++j) {
    const int ew = exB[ew_index + j];
    const float unscale = __uint_as_float(static_cast<uint32_t>(260 - ew) << 23);
    const int p = __float2int_rn(__fmul_rn(__uint_as_float(v[j]), unscale));
    acc[j] = tc_slow_tile_add(acc[j], p, ew, ex, status);
  }
}

// kPeer: a column-sharded layer whose rows go to every rank's full output
// (store_tile_peers), made visible system-wide before the CTA ends.
template <int kAB, bool kRes, bool kPeer>
__global__ void __launch_bounds__(kSThreads, 1)
    signsplit_b16_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB,
                         const int32_t *__restrict__ exA, int m_pad,
                         const int32_t *__restrict__ exB, int n_pad, int T, int M, int N,
                         int ex_lo, int ex_hi, FastDiv div_nb, const float *__restrict__ bias,
                         const float *__restrict__ post_scale,
                         const float *__restrict__ post_shift,
                         const float *__restrict__ residual_arg, int act, int vec,
                         int out_pixels, FastDiv div_pix, float *__restrict__ y,
                         int32_t *status, const __grid_constant__ cim22_peer_outputs peers,
                         int peer_vec4, const __grid_constant__ CUtensorMap tmR, int res_bp) {
  const float *residual = kRes ? residual_arg : nullptr;
  using S = SSShape<kAB>;
  constexpr int L = S::L, LT = S::LT, SN = S::N;
  using Shape = SBShape<kAB, kRes>;
  constexpr int kStages = Shape::kStages, kExSlots = Shape::kExSlots;
  extern __shared__ uint8_t smem_raw[];
  SmemSB<kAB, kRes> &s = smem_aligned<SmemSB<kAB, kRes>>(smem_raw);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int num_nb = (N + L - 1) / L;
  const int num_tiles = ((M + kSBM - 1) / kSBM) * num_nb;
  constexpr uint32_t kTmemCols = kTmemBufs * kBufCols;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < kExSlots; ++i) {
      mbar_init(&s.exfull[i], 1);
      mbar_init(&s.exempty[i], kEpiWarps);
    }
    for (int i = 0; i < kTmemBufs; ++i) {
      mbar_init(&s.dfull[i], 1);
      mbar_init(&s.dempty[i], kEpiWarps);
    }
    mbar_init(&s.rfull, 1);
    mbar_init(&s.rempty, kEpiWarps);
    s.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  // Resident per-lane epilogue parameters, copied before the PDL wait.
  const bool cached = N <= kParamLanes;
  if (cached)
    for (int i = threadIdx.x; i < N; i += kSThreads) {
      s.lane_params[0][i] = bias ? bias[i] : 0.0f;
      s.lane_params[1][i] = post_scale ? post_scale[i] : 0.0f;
      s.lane_params[2][i] = post_shift ? post_shift[i] : 0.0f;
    }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s.tmem;
  volatile int *failed = &s.failed;
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0 && lane == 0) {
    // TMA producer: per crossbar tile the activation tile of each branch
    // and the stacked Wp / Wn tile into the stage ring, the tile's activation
    // exponents of the 128 rows into the exponent ring.
    // Ring positions and phase parities advance incrementally: this thread
    // is the ring's only producer, and its per-tile instruction chain (not
    // the copies) is on the kernel's critical path. A failure elsewhere
    // shows up as a bounded wait that runs out.
    uint32_t it = 0, stage = 0, sphase = 0, slot = 0, xphase = 0;
    bool ok = true;
    for (int ot = blockIdx.x; ot < num_tiles && ok; ot += gridDim.x) {
      const int mb = fdiv(ot, div_nb);
      const int m0 = mb * kSBM, nb = ot - mb * num_nb, n0 = nb * L;
      for (int t = 0; t < T; ++t, ++it) {
        if (!mbar_wait(&s.empty[stage], sphase ^ 1) ||
            !mbar_wait(&s.exempty[slot], xphase ^ 1)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&s.full[stage], (kAB * Shape::kATile + Shape::kBTile) * 2);
#pragma unroll
        for (int a = 0; a < kAB; ++a)
          tma_load_2d(s.a[stage][a], &tmA, &s.full[stage], t * 64, a * m_pad + m0);
        tma_load_2d(s.b[stage], &tmB, &s.full[stage], t * 64, n0);
        tma_load_2d(s.b[stage] + L * 64, &tmB, &s.full[stage], t * 64, n_pad + n0);
        mbar_expect_tx(&s.exfull[slot], kAB * kSBM * 4);
#pragma unroll
        for (int a = 0; a < kAB; ++a)
          bulk_load(s.exa[slot][a], exA + (static_cast<int64_t>(a) * T + t) * m_pad + m0,
                    kSBM * 4, &s.exfull[slot]);
        if (++stage == kStages) {
          stage = 0;
          sphase ^= 1;
        }
        if (++slot == kExSlots) {
          slot = 0;
          xphase ^= 1;
        }
      }
    }
    if (!ok)
      *failed = 1;
    // Never leave with copies in flight: wait (bounded) for the last use of
    // every stage and exponent slot this thread filled (`it` counts the
    // filled tiles; a wait that failed filled none).
    for (uint32_t i = it > static_cast<uint32_t>(kStages) ? it - kStages : 0; i < it; ++i)
      mbar_wait(&s.full[i % kStages], (i / kStages) & 1);
    for (uint32_t i = it > static_cast<uint32_t>(kExSlots) ? it - kExSlots : 0; i < it; ++i)
      mbar_wait(&s.exfull[i % kExSlots], (i / kExSlots) & 1);
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: four K=16 MMAs per activation branch and crossbar tile.
    // The critical path of the kernel: ring positions advance incrementally
    // and the descriptors step by constant strides.
    constexpr uint32_t idesc = idesc_bf16(kSBM, SN);
    constexpr uint64_t kAStep = sizeof(s.a[0]) >> 4, kBStep = sizeof(s.b[0]) >> 4;
    const uint64_t adesc0 = sw128_desc(s.a[0][0]), bdesc0 = sw128_desc(s.b[0]);
    uint32_t gi = 0, stage = 0, sphase = 0, buf = 0, dphase = 0;
    bool ok = true;
    for (int ot = blockIdx.x; ot < num_tiles && ok; ot += gridDim.x) {
      for (int t = 0; t < T; ++t, ++gi) {
        if (!mbar_wait(&s.full[stage], sphase) || !mbar_wait(&s.dempty[buf], dphase ^ 1)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t bdesc = bdesc0 + stage * kBStep;
#pragma unroll
        for (int a = 0; a < kAB; ++a) {
          const uint64_t adesc = adesc0 + stage * kAStep + a * (kSBM * 64 * 2 >> 4);
          const uint32_t d = tmem + buf * kBufCols + a * SN;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_bf16(d, adesc + 2 * k, bdesc + 2 * k, idesc, k > 0 ? 1u : 0u);
        }
        mma_commit(&s.dfull[buf]);
        mma_commit(&s.empty[stage]);
        if (++stage == kStages) {
          stage = 0;
          sphase ^= 1;
        }
        if (++buf == kTmemBufs) {
          buf = 0;
          dphase ^= 1;
        }
      }
    }
    if (!ok)
      *failed = 1;
    // Let the last MMAs land before TMEM is freed.
    if (gi > 0)
      mbar_wait(&s.dfull[(gi - 1) % kTmemBufs], ((gi - 1) / kTmemBufs) & 1);
  } else if (warp >= 2) {
    // Epilogue.
    const int quad = warp % 4, sub = (warp - 2) / 4;
    const int row_local = quad * 32 + lane;
    const uint32_t tlane = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t span = static_cast<uint32_t>(ex_hi - ex_lo);
    uint32_t gi = 0, buf = 0, dphase = 0, slot = 0, xphase = 0;
    // Residual tiles by TMA: output tiles this CTA has started (the loads
    // warp 2's lane 0 issued) and finished (whose addends every warp read).
    const bool res_tma = kRes && res_bp > 0;
    const bool res_issuer = res_tma && warp == 2 && lane == 0;
    uint32_t res_started = 0, res_done = 0;
    bool ok = true;
    for (int ot = blockIdx.x; ot < num_tiles && ok; ot += gridDim.x) {
      const int mb = fdiv(ot, div_nb);
      const int m0 = mb * kSBM, n0 = (ot - mb * num_nb) * L;
      const int lane0 = n0 + sub * LT;
      const int row = m0 + row_local; // < m_pad
      if (res_tma) {
        if (res_issuer) {
          // The previous tile's addends have been read by every warp; this
          // tile's arrive while its crossbar tiles are computed. The box is
          // res_bp pixels x L lanes x (128 / res_bp) images from pixel
          // m0 mod HW of image m0 / HW.
          if (res_started > 0 && !mbar_wait(&s.rempty, (res_started - 1) & 1)) {
            ok = false;
            break;
          }
          const int img0 = fdiv(m0, div_pix);
          mbar_expect_tx(&s.rfull, Shape::kResTile * 4);
          tma_load_3d(s.res, &tmR, &s.rfull, m0 - img0 * out_pixels, n0, img0);
        }
        ++res_started;
      } else {
        prefetch_residual<LT>(residual, row, lane0, M, N, out_pixels, div_pix);
      }
      float acc[kAB][2][LT];
#pragma unroll
      for (int a = 0; a < kAB; ++a)
#pragma unroll
        for (int w = 0; w < 2; ++w)
#pragma unroll
          for (int j = 0; j < LT; ++j)
            acc[a][w][j] = 0.0f;
      for (int t = 0; t < T; ++t, ++gi) {
        // A failure elsewhere in the CTA shows up here as a wait that runs out.
        if (!mbar_wait(&s.exfull[slot], xphase)) {
          ok = false;
          break;
        }
        int ex[kAB];
        bool raw[kAB];
#pragma unroll
        for (int a = 0; a < kAB; ++a) {
          ex[a] = s.exa[slot][a][row_local];
          raw[a] = ex[a] != kZeroGroup && static_cast<uint32_t>(ex[a] - ex_lo) > span;
        }
        if (!mbar_wait(&s.dfull[buf], dphase)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t col0 = tmem + tlane + buf * kBufCols + sub * LT;
        if constexpr (kAB == 1) {
          const bool any_raw = __any_sync(0xffffffffu, raw[0]);
          if (any_raw) {
#pragma unroll
            for (int w = 0; w < 2; ++w) {
              uint32_t v[LT];
              tmem_ld_wait(col0 + w * L, v);
              restore_b16_raw<LT>(acc[0][w], v, raw[0], exB,
                                  (static_cast<int64_t>(w) * T + t) * n_pad + lane0, ex[0],
                                  status);
            }
          } else {
            // Both weight signs' columns in flight before one wait, then
            // packed adds (with one load and wait per sign the packed form
            // measured slower than scalar adds).
            static_assert(LT == 16, "two 8-column halves per weight sign");
            uint32_t v[2][2][8];
#pragma unroll
            for (int w = 0; w < 2; ++w) {
              tmem_ld(col0 + w * L, v[w][0]);
              tmem_ld(col0 + w * L + 8, v[w][1]);
            }
#pragma unroll
            for (int w = 0; w < 2; ++w) {
              tmem_wait(v[w][0]);
              tmem_wait(v[w][1]);
            }
#pragma unroll
            for (int w = 0; w < 2; ++w)
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                float(&a8)[8] = *reinterpret_cast<float(*)[8]>(&acc[0][w][8 * h]);
                restore_b16<8, true>(a8, v[w][h]);
              }
          }
        } else {
#pragma unroll
          for (int a = 0; a < kAB; ++a) {
            uint32_t v0[LT], v1[LT];
            tmem_ld(col0 + a * SN, v0);
            tmem_ld(col0 + a * SN + L, v1);
            tmem_wait(v0);
            tmem_wait(v1);
            if (__any_sync(0xffffffffu, raw[a])) {
              const int64_t ew0 = static_cast<int64_t>(t) * n_pad + lane0;
              restore_b16_raw<LT>(acc[a][0], v0, raw[a], exB, ew0, ex[a], status);
              restore_b16_raw<LT>(acc[a][1], v1, raw[a], exB,
                                  ew0 + static_cast<int64_t>(T) * n_pad, ex[a], status);
            } else {
              restore_b16<LT, true>(acc[a][0], v0);
              restore_b16<LT, true>(acc[a][1], v1);
            }
          }
        }
        // Hand the TMEM buffer and the exponent slot back once every lane
        // has read them.
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s.dempty[buf]);
          mbar_arrive(&s.exempty[slot]);
        }
        if (++buf == kTmemBufs) {
          buf = 0;
          dphase ^= 1;
        }
        if (++slot == kExSlots) {
          slot = 0;
          xphase ^= 1;
        }
      }
      if (!ok)
        break;
      if constexpr (kPeer) {
        store_tile_peers<kAB, LT>(acc, row, lane0, M, N, T, cached ? s.lane_params : nullptr,
                                  bias, post_scale, post_shift, act, vec, peers, peer_vec4 != 0);
      } else if (res_tma) {
        if (!mbar_wait(&s.rfull, res_done & 1)) {
          ok = false;
          break;
        }
        // Row r of the tile is pixel r mod res_bp of the tile's image
        // r / res_bp; lane j of the thread sits res_bp floats further on.
        const float *res_row =
            s.res + ((row_local / res_bp) * L + sub * LT) * res_bp + row_local % res_bp;
        store_tile<kAB, LT>(acc, row, lane0, M, N, T, cached ? s.lane_params : nullptr, bias,
                            post_scale, post_shift, residual, act, vec, out_pixels, div_pix, y,
                            res_row, res_bp);
        __syncwarp();
        if (lane == 0)
          mbar_arrive(&s.rempty);
        ++res_done;
      } else {
        store_tile<kAB, LT>(acc, row, lane0, M, N, T, cached ? s.lane_params : nullptr, bias,
                            post_scale, post_shift, residual, act, vec, out_pixels, div_pix, y);
      }
    }
    // Never leave with the residual copy in flight (bounded).
    if (res_issuer && res_started > res_done)
      mbar_wait(&s.rfull, (res_started - 1) & 1);
    if (!ok) {
      *failed = 1;
      if (lane == 0)
        atomicOr(status, CIM22_STATUS_TIMEOUT);
    }
    if constexpr (kPeer)
      __threadfence_system();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// INT8 contraction, persistent: 128 x 256 output tiles (one tcgen05.mma
// kind::i8 of M=128, N=256, K=32 per 32 bytes of K), a 4-stage TMA ring of
// 128-byte K blocks (16 KB of A and 32 KB of B per stage), and two 256-column
// TMEM accumulators so the epilogue of one tile overlaps the MMAs of the next.
//
//   warp 0 (one thread)  TMA producer over every tile of the CTA
//   warp 1 (one thread)  MMA issuer; commits each stage back to the producer
//                        and each finished accumulator to the epilogue
//   warps 2-9            epilogue: warp w reads TMEM lanes 32 * (w % 4) (tile
//                        rows) and one 128-column half of the accumulator,
//                        adds the bias and stores rows or NCHW planes
//
// Tiles are walked column-major (consecutive CTAs take consecutive row
// blocks of the same weight block), so a weight block is read from HBM once
// per wave and the activations stay in L2. Every wait is bounded; a wait
// that runs out stops the CTA, which waits (bounded) for its copies in flight
// and frees its TMEM.
constexpr int kIBM = 128, kIBN = 256, kIBK = 128, kIStages = 4;
constexpr int kIEpiWarps = 8;
constexpr int kIThreads = 64 + 32 * kIEpiWarps;
constexpr uint32_t kIBufCols = kIBN;
constexpr uint32_t kIStageBytes = (kIBM + kIBN) * kIBK;

struct alignas(1024) SmemI8P {
  int8_t a[kIStages][kIBM * kIBK];
  int8_t b[kIStages][kIBN * kIBK];
  uint64_t full[kIStages];
  uint64_t empty[kIStages];
  uint64_t dfull[2];
  uint64_t dempty[2];
  uint32_t tmem;
  int failed;
};

__global__ void __launch_bounds__(kIThreads, 1)
    int8_persistent_kernel(const __grid_constant__ CUtensorMap tmA,
                           const __grid_constant__ CUtensorMap tmB, int num_kb, int M, int N,
                           int num_mb, FastDiv div_mb, const int32_t *__restrict__ bias,
                           int out_pixels, FastDiv div_pix, int vec, int32_t *__restrict__ y,
                           int32_t *status) {
  extern __shared__ uint8_t smem_raw[];
  SmemI8P &s = smem_aligned<SmemI8P>(smem_raw);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int num_tiles = num_mb * ((N + kIBN - 1) / kIBN);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kIStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.dfull[i], 1);
      mbar_init(&s.dempty[i], kIEpiWarps);
    }
    s.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem)),
                 "r"(2 * kIBufCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s.tmem;
  volatile int *failed = &s.failed;
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0 && lane == 0) {
    uint32_t kbi = 0;
    bool ok = true;
    for (int ot = blockIdx.x; ot < num_tiles && ok; ot += gridDim.x) {
      const int nb = fdiv(ot, div_mb);
      const int m0 = (ot - nb * num_mb) * kIBM, n0 = nb * kIBN;
      for (int kb = 0; kb < num_kb; ++kb, ++kbi) {
        const int stage = kbi % kIStages;
        if (!mbar_wait(&s.empty[stage], ((kbi / kIStages) & 1) ^ 1) || *failed) {
          ok = false;
          break;
        }
        mbar_expect_tx(&s.full[stage], kIStageBytes);
        tma_load_2d(s.a[stage], &tmA, &s.full[stage], kb * kIBK, m0);
        tma_load_2d(s.b[stage], &tmB, &s.full[stage], kb * kIBK, n0);
      }
    }
    if (!ok)
      *failed = 1;
    // Never leave with copies in flight.
    for (uint32_t i = kbi > kIStages ? kbi - kIStages : 0; i < kbi; ++i)
      mbar_wait(&s.full[i % kIStages], (i / kIStages) & 1);
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_i8(kIBM, kIBN);
    uint32_t kbi = 0, ti = 0;
    bool ok = true;
    for (int ot = blockIdx.x; ot < num_tiles && ok; ot += gridDim.x) {
      const int buf = ti & 1;
      if (!mbar_wait(&s.dempty[buf], ((ti >> 1) & 1) ^ 1) || *failed) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t d = tmem + buf * kIBufCols;
      for (int kb = 0; kb < num_kb; ++kb, ++kbi) {
        const int stage = kbi % kIStages;
        if (!mbar_wait(&s.full[stage], (kbi / kIStages) & 1) || *failed) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t adesc = sw128_desc(s.a[stage]);
        const uint64_t bdesc = sw128_desc(s.b[stage]);
#pragma unroll
        for (int kk = 0; kk < kIBK / 32; ++kk)
          mma_i8(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&s.empty[stage]);
      }
      // Commit the accumulator (also after a failed wait, so every MMA
      // issued is tracked before TMEM is freed).
      mma_commit(&s.dfull[buf]);
      ++ti;
    }
    if (!ok)
      *failed = 1;
    // Let the last MMAs land before TMEM is freed.
    if (ti > 0)
      mbar_wait(&s.dfull[(ti - 1) & 1], ((ti - 1) >> 1) & 1);
  } else if (warp >= 2) {
    const int quad = warp % 4, half = (warp - 2) / 4;
    const uint32_t tlane = static_cast<uint32_t>(quad * 32) << 16;
    uint32_t ti = 0;
    bool ok = true;
    for (int ot = blockIdx.x; ot < num_tiles; ot += gridDim.x, ++ti) {
      const int buf = ti & 1;
      const int nb = fdiv(ot, div_mb);
      const int row = (ot - nb * num_mb) * kIBM + quad * 32 + lane;
      const int n_half = nb * kIBN + half * (kIBN / 2);
      if (!mbar_wait(&s.dfull[buf], (ti >> 1) & 1) || *failed) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      int64_t base = static_cast<int64_t>(row) * N, step = 1;
      if (out_pixels > 0 && row < M) {
        const int64_t img = fdiv(row, div_pix);
        base = img * N * out_pixels + (row - img * out_pixels);
        step = out_pixels;
      }
#pragma unroll 1
      for (int c = 0; c < kIBN / 2 / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + tlane + buf * kIBufCols + half * (kIBN / 2) + c * 32, r);
        const int n0 = n_half + c * 32;
        if (row >= M)
          continue;
        if (bias != nullptr)
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j < N)
              r[j] += static_cast<uint32_t>(bias[n0 + j]);
        if (step == 1 && vec && n0 + 32 <= N) {
          int4 *dst = reinterpret_cast<int4 *>(y + base + n0);
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            dst[j / 4] = make_int4(static_cast<int>(r[j]), static_cast<int>(r[j + 1]),
                                   static_cast<int>(r[j + 2]), static_cast<int>(r[j + 3]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j < N)
              y[base + static_cast<int64_t>(n0 + j) * step] = static_cast<int32_t>(r[j]);
        }
      }
      // The accumulator is free once every epilogue warp has read it.
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0)
        mbar_arrive(&s.dempty[buf]);
    }
    if (!ok) {
      *failed = 1;
      if (lane == 0)
        atomicOr(status, CIM22_STATUS_TIMEOUT);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(2 * kIBufCols));
  }
}

// ---------------------------------------------------------------------------
// Host side.

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D int8 tensor [rows][cols] (cols contiguous), box 128 x 128, 128B swizzle.
bool encode_int8_2d(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                    uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn)
    return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols};
  const cuuint32_t box[2] = {kBK, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D BF16 tensor [rows][cols] (cols contiguous), box 64 x box_rows (128
// bytes of a row: one crossbar tile), 128B swizzle.
bool encode_bf16_2d(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                    uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn)
    return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
            box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

} // namespace

// 4-D f32 tensor [N][C][H][W] (W contiguous, W % 4 == 0), box
// [nb][cb][hb][wb], no swizzle; out-of-range elements of a box read as +0.
bool encode_nchw_box(CUtensorMap *map, const float *x, uint64_t W, uint64_t H, uint64_t C,
                     uint64_t N, uint32_t wb, uint32_t hb, uint32_t cb, uint32_t nb) {
  auto fn = encode_fn();
  if (!fn)
    return false;
  const cuuint64_t dims[4] = {W, H, C, N};
  const cuuint64_t strides[3] = {W * 4, H * W * 4, C * H * W * 4};
  const cuuint32_t box[4] = {wb, hb, cb, nb};
  const cuuint32_t elem[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(x), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_prepared_store(CUtensorMap *map, void *base, uint64_t rows, uint64_t k_pad,
                           bool b16) {
  auto fn = encode_fn();
  if (!fn)
    return false;
  const cuuint64_t dims[2] = {k_pad, rows};
  const cuuint64_t strides[1] = {k_pad * (b16 ? 2 : 1)};
  const cuuint32_t box[2] = {64, 32};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, b16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base,
            dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
            b16 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

bool sm100(cudaStream_t) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess)
    return false;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

constexpr size_t kSmemInt8 = sizeof(SmemInt8) + 1024;

int sm_count() {
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

} // namespace

std::atomic<int64_t> g_tc_launches{0};

template <int kAB> constexpr size_t smem_ss() { return sizeof(SmemSS<kAB>) + 1024; }

bool signsplit_available() { return sm100(nullptr) && encode_fn() != nullptr; }

bool int8_available() { return sm100(nullptr) && encode_fn() != nullptr; }

bool launch_signsplit(const int8_t *A, const int32_t *exA, int64_t m_pad, const int8_t *B,
                      const int32_t *exB, int64_t n_pad, int64_t k_pad, int T, int64_t M,
                      int64_t N, const float *bias, const float *post_scale,
                      const float *post_shift, const float *residual, int act,
                      int act_branches, int64_t out_pixels, float *y, int32_t *status,
                      cudaStream_t stream) {
  // Layers of at most 8 lanes leave most of a 32- or 64-lane tile idle; the
  // CUDA-core kernel serves them. The exponent copies need 16-byte aligned
  // rows: m_pad and n_pad are multiples of 128 and both exponent arrays
  // start 16-byte aligned.
  const int L = act_branches == 2 ? SSShape<2>::L : SSShape<1>::L;
  if (M < 1 || N <= 8 || m_pad % kSBM || n_pad % 128 || k_pad % 64 ||
      static_cast<int64_t>(act_branches) * m_pad >= (int64_t{1} << 31) ||
      (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15) ||
      (reinterpret_cast<uintptr_t>(exA) & 15) || (reinterpret_cast<uintptr_t>(exB) & 15))
    return false;
  CUtensorMap ta, tb;
  if (!encode_int8_2d(&ta, A, act_branches * m_pad, k_pad, kSBM) ||
      !encode_int8_2d(&tb, B, 2 * n_pad, k_pad, static_cast<uint32_t>(L)))
    return false;
  // Vector bias loads (bit 0) and row stores (bit 1) where the bias and the
  // output rows start 16-byte aligned.
  const int vec = (N % 4 == 0 && (reinterpret_cast<uintptr_t>(bias) & 15) == 0 ? 1 : 0) |
                  (N % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 ? 2 : 0);
  const int64_t tiles = ((M + kSBM - 1) / kSBM) * ((N + L - 1) / L);
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>(tiles, sm_count())));
  auto launch = [&](auto kernel, size_t smem) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return false;
    launch_pdl(kernel, grid, kSThreads, smem, stream, ta, tb, exA, static_cast<int>(m_pad), exB, static_cast<int>(n_pad), T,
        static_cast<int>(M), static_cast<int>(N),
        make_fastdiv(static_cast<uint32_t>((N + L - 1) / L)), bias, post_scale, post_shift,
        residual, act, vec, static_cast<int>(out_pixels),
        make_fastdiv(static_cast<uint32_t>(out_pixels > 0 ? out_pixels : 1)), y, status);
    return true;
  };
  const bool res = residual != nullptr;
  if (!(act_branches == 2
            ? (res ? launch(signsplit_tc_kernel<2, true>, smem_ss<2>())
                   : launch(signsplit_tc_kernel<2, false>, smem_ss<2>()))
            : (res ? launch(signsplit_tc_kernel<1, true>, smem_ss<1>())
                   : launch(signsplit_tc_kernel<1, false>, smem_ss<1>()))))
    return false;
  g_tc_launches.fetch_add(1, std::memory_order_relaxed);
  return true;
}

template <int kAB, bool kRes> constexpr size_t smem_sb() {
  return sizeof(SmemSB<kAB, kRes>) + 1024;
}
static_assert(smem_sb<1, false>() <= 232448 && smem_sb<2, false>() <= 232448 &&
                  smem_sb<1, true>() <= 232448 && smem_sb<2, true>() <= 232448,
              "the BF16 operand ring must fit the 227 KB of dynamic shared memory per CTA");

bool launch_signsplit_b16(const uint16_t *A, const int32_t *exA, int64_t m_pad,
                          const uint16_t *B, const int32_t *exB, int64_t n_pad, int64_t k_pad,
                          int T, int64_t M, int64_t N, int ex_lo, int ex_hi, const float *bias,
                          const float *post_scale, const float *post_shift,
                          const float *residual, int act, int act_branches, int64_t out_pixels,
                          float *y, int32_t *status, cudaStream_t stream,
                          const cim22_peer_outputs *peers) {
  const int L = act_branches == 2 ? SSShape<2>::L : SSShape<1>::L;
  cim22_peer_outputs none{};
  const bool peer = peers != nullptr;
  if (peer && (out_pixels != 0 || residual != nullptr || peers->ranks < 1 ||
               peers->ranks > CIM22_MAX_PEERS || peers->lanes < 1 || peers->lanes > N ||
               peers->lane_offset < 0 || peers->lane_offset + peers->lanes > peers->row_stride))
    return false;
  int peer_vec4 = 0;
  if (peer) {
    peer_vec4 = peers->row_stride % 4 == 0 && peers->lane_offset % 4 == 0;
    for (int p = 0; p < peers->ranks; ++p) {
      if (!peers->out[p])
        return false;
      if (reinterpret_cast<uintptr_t>(peers->out[p]) & 15)
        peer_vec4 = 0;
    }
  }
  if (M < 1 || N <= 8 || m_pad % kSBM || n_pad % 128 || k_pad % 64 || ex_lo > ex_hi ||
      static_cast<int64_t>(act_branches) * m_pad >= (int64_t{1} << 31) ||
      (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15) ||
      (reinterpret_cast<uintptr_t>(exA) & 15) || (reinterpret_cast<uintptr_t>(exB) & 15))
    return false;
  CUtensorMap ta, tb;
  if (!encode_bf16_2d(&ta, A, act_branches * m_pad, k_pad, kSBM) ||
      !encode_bf16_2d(&tb, B, 2 * n_pad, k_pad, static_cast<uint32_t>(L)))
    return false;
  const int vec = (N % 4 == 0 && (reinterpret_cast<uintptr_t>(bias) & 15) == 0 ? 1 : 0) |
                  (N % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 ? 2 : 0);
  // NCHW residual addends whose 128-row tiles cover whole images or runs of
  // one image come as one TMA box per output tile: res_bp pixels x L lanes x
  // 128 / res_bp images (lanes and images past the tensor read as +0).
  CUtensorMap tr{};
  int res_bp = 0;
  if (residual != nullptr && out_pixels > 0 && out_pixels % 4 == 0 && M % out_pixels == 0 &&
      (out_pixels % kSBM == 0 || kSBM % out_pixels == 0) &&
      (reinterpret_cast<uintptr_t>(residual) & 15) == 0) {
    auto fn = encode_fn();
    const uint32_t bp = static_cast<uint32_t>(std::min<int64_t>(out_pixels, kSBM));
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(out_pixels), static_cast<cuuint64_t>(N),
                                static_cast<cuuint64_t>(M / out_pixels)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(out_pixels) * 4,
                                   static_cast<cuuint64_t>(N * out_pixels) * 4};
    const cuuint32_t box[3] = {bp, static_cast<cuuint32_t>(L), kSBM / bp};
    const cuuint32_t elem[3] = {1, 1, 1};
    if (fn && fn(&tr, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(residual), dims,
                 strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      res_bp = static_cast<int>(bp);
  }
  const int64_t tiles = ((M + kSBM - 1) / kSBM) * ((N + L - 1) / L);
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>(tiles, sm_count())));
  auto launch = [&](auto kernel, size_t smem) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return false;
    launch_pdl(kernel, grid, kSThreads, smem, stream, ta, tb, exA, static_cast<int>(m_pad), exB,
               static_cast<int>(n_pad), T, static_cast<int>(M), static_cast<int>(N), ex_lo,
               ex_hi, make_fastdiv(static_cast<uint32_t>((N + L - 1) / L)), bias, post_scale,
               post_shift, residual, act, vec, static_cast<int>(out_pixels),
               make_fastdiv(static_cast<uint32_t>(out_pixels > 0 ? out_pixels : 1)), y, status,
               peer ? *peers : none, peer_vec4, tr, res_bp);
    return true;
  };
  const bool res = residual != nullptr;
  bool launched;
  if (peer)
    launched = act_branches == 2
                   ? launch(signsplit_b16_kernel<2, false, true>, smem_sb<2, false>())
                   : launch(signsplit_b16_kernel<1, false, true>, smem_sb<1, false>());
  else
    launched = act_branches == 2
                   ? (res ? launch(signsplit_b16_kernel<2, true, false>, smem_sb<2, true>())
                          : launch(signsplit_b16_kernel<2, false, false>, smem_sb<2, false>()))
                   : (res ? launch(signsplit_b16_kernel<1, true, false>, smem_sb<1, true>())
                          : launch(signsplit_b16_kernel<1, false, false>, smem_sb<1, false>()));
  if (!launched)
    return false;
  g_tc_launches.fetch_add(1, std::memory_order_relaxed);
  return true;
}

bool launch_int8(const int8_t *A, int64_t a_rows, int64_t a_cols, const int8_t *B,
                 int64_t n_pad, int64_t k_pad, int64_t M, int64_t N, const int32_t *bias,
                 int64_t out_pixels, int32_t *y, int32_t *status, cudaStream_t stream) {
  if (n_pad % kBN || k_pad % 64 || a_cols % 16 || a_cols > k_pad || a_rows < M ||
      M >= (int64_t{1} << 31) - kBM || (reinterpret_cast<uintptr_t>(A) & 15) ||
      (reinterpret_cast<uintptr_t>(B) & 15) || out_pixels < 0 ||
      (out_pixels > 0 && M % out_pixels))
    return false;
  const FastDiv div_pix = make_fastdiv(static_cast<uint32_t>(out_pixels > 0 ? out_pixels : 1));
  // Enough 128 x 256 tiles for every SM: the persistent kernel.
  const int64_t num_mb = (M + kIBM - 1) / kIBM;
  const int64_t p_tiles = num_mb * ((N + kIBN - 1) / kIBN);
  if (p_tiles >= sm_count() && p_tiles < (int64_t{1} << 31)) {
    CUtensorMap ta, tb;
    if (!encode_int8_2d(&ta, A, a_rows, a_cols, kIBM) ||
        !encode_int8_2d(&tb, B, n_pad, k_pad, kIBN))
      return false;
    constexpr size_t smem = sizeof(SmemI8P) + 1024;
    if (cudaFuncSetAttribute(int8_persistent_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return false;
    const int vec = (N % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) ? 1 : 0;
    const int grid = static_cast<int>(std::min<int64_t>(p_tiles, sm_count()));
    if (launch_pdl(int8_persistent_kernel, dim3(grid), kIThreads, smem, stream, ta, tb,
                   static_cast<int>((k_pad + kIBK - 1) / kIBK), static_cast<int>(M),
                   static_cast<int>(N), static_cast<int>(num_mb),
                   make_fastdiv(static_cast<uint32_t>(num_mb)), bias,
                   static_cast<int>(out_pixels), div_pix, vec, y, status) != cudaSuccess)
      return false;
    g_tc_launches.fetch_add(1, std::memory_order_relaxed);
    return true;
  }
  // Columns beyond a_cols (to k_pad) and rows beyond a_rows read TMA's zero fill.
  CUtensorMap ta, tb;
  if (!encode_int8_2d(&ta, A, a_rows, a_cols, kBM) || !encode_int8_2d(&tb, B, n_pad, k_pad, kBN))
    return false;
  const int64_t m_pad = (M + kBM - 1) / kBM * kBM;
  if (cudaFuncSetAttribute(int8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kSmemInt8)) != cudaSuccess)
    return false;
  const int num_kb = static_cast<int>((k_pad + kBK - 1) / kBK);
  const dim3 grid(static_cast<unsigned>(m_pad / kBM), static_cast<unsigned>((N + kBN - 1) / kBN));
  int8_tc_kernel<<<grid, kThreads, kSmemInt8, stream>>>(ta, tb, num_kb, M, N, bias,
                                                        out_pixels, div_pix, y, status);
  g_tc_launches.fetch_add(1, std::memory_order_relaxed);
  return true;
}

// One CTA waits, with the pipelines' bounded wait, on an mbarrier that
// nothing completes: the wait gives up after limit_ns and the kernel reports
// CIM22_STATUS_TIMEOUT. It holds no TMEM and issues no copies, so its
// return leaves nothing in flight.
__global__ void wait_timeout_kernel(uint64_t limit_ns, int32_t *status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const bool done = mbar_wait(&bar, 0, limit_ns);
  if (!done && threadIdx.x == 0)
    atomicOr(status, CIM22_STATUS_TIMEOUT);
  __syncthreads();
}

} // namespace cim::tc

extern "C" int cim22_cuda_check_wait_timeout(uint64_t limit_ns, int32_t *status, void *stream) {
  if (!status || limit_ns == 0 || limit_ns > 10000000000ull) {
    cim::set_last_error("cim22_cuda_check_wait_timeout: status must be a device int32 and "
                        "0 < limit_ns <= 10 s");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  cim::tc::wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns,
                                                                               status);
  return cim::cuda_ok(cudaGetLastError(), "wait check launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

extern "C" int64_t cim22_cuda_tensor_core_launches(void) {
  return cim::tc::g_tc_launches.load(std::memory_order_relaxed);
}
