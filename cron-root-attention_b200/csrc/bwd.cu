// placeholder, replaced by the backward kernels
#include "../../include/cra.h"
extern "C" {
size_t cra_bwd_workspace_bytes(int, int, int, int, int, int, int) { return 0; }
int cra_bwd(const void*, const void*, const void*, const void*, const void*, const float*, const void*, const void*,
            const int32_t*, const int64_t*, const int64_t*, const int64_t*, const int64_t*, const int64_t*, int, int,
            int, int, int, int, int, int, float, const float*, void*, void*, void*, const int64_t*, const int64_t*,
            const int64_t*, float*, void*, size_t, int*, void*) {
  return CRA_ERR_UNSUPPORTED;
}
}
