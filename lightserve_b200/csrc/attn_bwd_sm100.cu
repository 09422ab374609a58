// tcgen05 FlashAttention backward (placeholder: not yet eligible for any input).
#include "common.cuh"

namespace lsb {
struct Strides4;
bool attn_bwd_tc_eligible(const void*, const void*, const void*, const void*, const void*,
                          const void*, const void*, const void*, int64_t, int64_t, int64_t,
                          int64_t, const int64_t*, const int64_t*, const int64_t*, const int64_t*,
                          const int64_t*, const int64_t*, const int64_t*, const int64_t*, int) {
  return false;
}
int attn_bwd_tc(const void*, const void*, const void*, const void*, const void*, const float*,
                void*, void*, void*, int64_t, int64_t, int64_t, int64_t, const int64_t*,
                const int64_t*, const int64_t*, const int64_t*, const int64_t*, const int64_t*,
                const int64_t*, const int64_t*, float, int, int, float*, float*, cudaStream_t) {
  set_error("attn_bwd: tcgen05 kernel not built");
  return LSB_ERR_UNSUPPORTED;
}
int attn_bwd_tc_device_error() { return 0; }
}  // namespace lsb
