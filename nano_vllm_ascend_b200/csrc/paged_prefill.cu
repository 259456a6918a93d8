// Causal prefill attention (paged and dense). The tcgen05 kernel lands here;
// until then both entry points report NVK_ERR_UNSUPPORTED.
#include "host_common.h"

extern "C" int nvk_paged_prefill(void*, const void*, const void*, const void*, int, int, const int32_t*, int,
                                 const int32_t*, const int32_t*, int, int, int, int, int, int, float, int*,
                                 nvk_stream_t) {
  return nvk::fail(NVK_ERR_UNSUPPORTED, "paged_prefill: not built yet");
}

extern "C" int nvk_dense_prefill(void*, const void*, const void*, const void*, const int32_t*, const int32_t*, int,
                                 int, int, int, int, int, int, float, int*, nvk_stream_t) {
  return nvk::fail(NVK_ERR_UNSUPPORTED, "dense_prefill: not built yet");
}
