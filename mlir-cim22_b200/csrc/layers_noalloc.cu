// layers_noalloc.cu - BF16 sign-split CIM layer without caller scratch.
//
// cim22_cuda_layer_forward_bf16 needs a workspace for the prepared activation
// columns (int8 mantissas, or BF16 operand values for layers of 64 lanes and
// more, and per-group exponents). Some callers cannot
// provide one: generated model code that, like the reference's compiled Host
// code, only owns stack buffers and has no device allocator of its own, and
// embedders whose device memory is owned and budgeted by another component.
// This entry point keeps that scratch in a fixed-size array in device global
// memory that belongs to the library, so the call allocates nothing.
//
// Facts a caller must know:
//  * Every GPU that loads the library holds kScratchBytes of device memory
//    for this array until the process exits.
//  * All calls on one device share the array and it keeps the contents of the
//    last call. Two calls whose kernels overlap on the GPU (different streams
//    without ordering between them) race on it and give wrong results; order
//    them on one stream or with events.
//  * Nothing in the array has to start at zero: the prepare kernel writes
//    every byte the contraction kernel later reads for the same call.
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current, and caches it. That
//    first call may load the module, so make it before any stream capture
//    starts on that device.
#include "cim_internal.h"

#include <mutex>

namespace cim {
namespace {

constexpr size_t kScratchBytes = size_t{16} << 20; // 16 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_layer_scratch[kScratchBytes];

std::mutex g_scratch_lock;
void *g_scratch_address[kMaxDevices] = {};

// Device address of g_layer_scratch for the current device, looked up once.
void *scratch_for_current_device(int device) {
  std::lock_guard<std::mutex> lock(g_scratch_lock);
  if (!g_scratch_address[device]) {
    void *address = nullptr;
    if (!cuda_ok(cudaGetSymbolAddress(&address, g_layer_scratch),
                 "cudaGetSymbolAddress"))
      return nullptr;
    g_scratch_address[device] = address;
  }
  return g_scratch_address[device];
}

} // namespace
} // namespace cim

using namespace cim;

extern "C" {

size_t cim22_cuda_layer_noalloc_scratch_bytes(void) { return kScratchBytes; }

int cim22_cuda_layer_forward_bf16_noalloc(const cim22_cuda_layer *layer,
                                          const float *x,
                                          const cim22_gather *gather, int64_t m,
                                          const float *bias,
                                          int32_t activation, int32_t branches,
                                          float *y, int32_t *status,
                                          void *stream) {
  if (!layer || !layer->bf16 || m <= 0 || (branches != 2 && branches != 4)) {
    set_last_error("invalid arguments to cim22_cuda_layer_forward_bf16_noalloc");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  const size_t need = cim22_cuda_layer_workspace_bf16(layer, m, branches);
  if (need > kScratchBytes) {
    set_last_error("cim22_cuda_layer_forward_bf16_noalloc: " + std::to_string(m) +
                   " columns need " + std::to_string(need) +
                   " bytes of scratch, more than the " + std::to_string(kScratchBytes) +
                   "-byte static scratch; use cim22_cuda_layer_forward_bf16 with a "
                   "workspace");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  int device = -1;
  if (!cuda_ok(cudaGetDevice(&device), "cudaGetDevice"))
    return CIM22_STATUS_BAD_ARGUMENT;
  if (device != layer->device || device < 0 || device >= kMaxDevices) {
    set_last_error("cim22_cuda_layer_forward_bf16_noalloc: make the layer's device "
                   "current before the call");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  void *scratch = scratch_for_current_device(device);
  if (!scratch)
    return CIM22_STATUS_BAD_ARGUMENT;
  return cim22_cuda_layer_forward_bf16(layer, x, gather, m, bias, activation, branches,
                                       y, scratch, kScratchBytes, status, stream);
}

} // extern "C"
