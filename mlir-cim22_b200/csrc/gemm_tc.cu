// gemm_tc.cu - tcgen05 contraction kernels (sm_100a).
#include "gemm_tc.h"

namespace cim::tc {

bool signsplit_available() { return false; }
bool int8_available() { return false; }

bool launch_signsplit(const int8_t *, const int32_t *, int64_t, const int8_t *,
                      const int32_t *, int64_t, int64_t, int, int64_t, int64_t,
                      const float *, int, int, float *, int32_t *, cudaStream_t) {
  return false;
}

bool launch_int8(const int8_t *, int64_t, const int8_t *, int64_t, int64_t, int,
                 int64_t, int64_t, int32_t *, int32_t *, cudaStream_t) {
  return false;
}

} // namespace cim::tc
