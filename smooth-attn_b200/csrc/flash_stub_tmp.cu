#include "sa_common.cuh"
extern "C" int64_t sa_flash_bwd_workspace_size(int64_t, int64_t, int64_t, int64_t, int64_t) { return 0; }
extern "C" int sa_flash_bwd(const void*, const void*, const void*, const void*, const void*, const float*, void*, void*, void*, void*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, const int64_t*, const int64_t*, const int64_t*, const int64_t*, const int64_t*, const int64_t*, const int64_t*, const int64_t*, float, int64_t, int, int, void*) { return SA_ERR_UNSUPPORTED; }
