// capi.cpp - diagnostics and ABI self-description of the C interface.
#include "cim_internal.h"

#include <algorithm>
#include <cstring>

namespace cim {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string &message) { g_last_error = message; }
const std::string &last_error() { return g_last_error; }

void copy_error(const std::string &message, char *buffer, size_t capacity) {
  if (buffer && capacity) {
    const size_t n = std::min(capacity - 1, message.size());
    std::memcpy(buffer, message.data(), n);
    buffer[n] = '\0';
  }
}

} // namespace cim

extern "C" {

const char *cim22_cuda_status_message(int32_t status) {
  if (status & CIM22_STATUS_INPUT_NOT_FINITE)
    return "CIM BF16 input does not support NaN or infinity";
  if (status & CIM22_STATUS_TILE_OVERFLOW)
    return "CIM BF16 compensated tile exceeds BF16";
  if (status & CIM22_STATUS_I21_RANGE)
    return "CIM software result exceeds signed i21 range";
  if (status & CIM22_STATUS_NORMALIZATION)
    return "CIM nonnegative BF16 normalization did not produce input exponent 127";
  if (status & CIM22_STATUS_BAD_ARGUMENT)
    return "invalid CIM layer launch arguments";
  if (status & CIM22_STATUS_NEGATIVE_INPUT)
    return "CIM nonnegative BF16 mode rejects negative inputs";
  if (status & CIM22_STATUS_TIMEOUT)
    return "CIM tensor-core pipeline wait timed out";
  if (status & CIM22_STATUS_LEGACY_SCALING)
    return "CIM legacy BF16 group scaling changed prealigned input mantissas";
  if (status & CIM22_STATUS_LEGACY_I21)
    return "CIM BF16 result exceeds signed i21 range";
  if (status & CIM22_STATUS_CHIP_NOT_FINITE)
    return "CIM BF16 chip output is not finite";
  return "";
}

const char *cim22_cuda_last_error(void) { return cim::last_error().c_str(); }

int cim22_cuda_abi_sizes(int64_t *sizes, int capacity) {
  const int64_t all[] = {
      sizeof(cim22_frame_packet), sizeof(cim22_static_weight),
      sizeof(cim22_input_binding), sizeof(cim22_readback_binding),
      sizeof(cim22_work),          sizeof(cim22_group),
      sizeof(cim22_transaction),   sizeof(cim22_trace_event),
      sizeof(cim22_memref2d),      sizeof(cim22_gather),
      sizeof(cim22_chain_layer),   sizeof(cim22_peer_outputs),
      sizeof(cim22_peer_flags)};
  const int n = static_cast<int>(sizeof(all) / sizeof(all[0]));
  if (sizes)
    for (int i = 0; i < std::min(n, capacity); ++i)
      sizes[i] = all[i];
  return n;
}

} // extern "C"
