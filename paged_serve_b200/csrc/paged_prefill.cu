// Causal paged prefill (tcgen05/TMEM) — entry point; kernel under construction.
#include "capi_internal.h"

using namespace ps;

extern "C" int ps_paged_prefill(void*, int64_t, const void*, int64_t, const void*, const void*,
                                int64_t, const int32_t*, int64_t, const int32_t*, const int32_t*,
                                const int32_t*, int, int, int, int, int, int, int, float, int,
                                int32_t*, void*) {
  return fail(PS_ERR_UNSUPPORTED, "ps_paged_prefill: not available in this build");
}
