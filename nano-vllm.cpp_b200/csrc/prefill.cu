// prefill.cu -- causal paged prefill (placeholder until the tcgen05 kernel lands).
#include "internal.h"

namespace nvattn {

nvattn_status launch_paged_prefill(nvattn_handle*, int, int, int, const uint16_t*,
                                   const int32_t*, const int32_t*, const int32_t*,
                                   const int32_t*, int, int, const uint16_t*, const uint16_t*,
                                   float*, cudaStream_t) {
  return NVATTN_ERR_UNSUPPORTED;
}

}  // namespace nvattn
