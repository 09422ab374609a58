// tcgen05 FlashAttention forward (placeholder: not yet eligible for any input).
#include "common.cuh"

namespace lsb {
bool attn_fwd_tc_eligible(const void*, const void*, const void*, const void*, int64_t, int64_t,
                          int64_t, int64_t, const int64_t*, const int64_t*, const int64_t*,
                          const int64_t*, int) {
  return false;
}
int attn_fwd_tc(const void*, const void*, const void*, void*, float*, int64_t, int64_t, int64_t,
                int64_t, const int64_t*, const int64_t*, const int64_t*, const int64_t*, float,
                int, int, cudaStream_t) {
  set_error("attn_fwd: tcgen05 kernel not built");
  return LSB_ERR_UNSUPPORTED;
}
}  // namespace lsb
