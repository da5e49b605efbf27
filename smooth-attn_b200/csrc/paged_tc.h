// Launch plan of the tensor-core paged-decode kernel (paged_tc.cu), shared
// with the entry point in paged.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sa {

struct PtcPlan {
  int GT;                // query heads per unit (the MMA's N columns in use)
  int64_t grid;          // CTAs (one per SM at most)
  int slots;             // partial-record slots per unit
  int64_t ticket_bytes;  // tickets [units], padded to 256 bytes
  int64_t part_bytes;    // partial records [units][slots][GT*128 + 16] fp32
};

bool paged_tc_plan(int64_t B, int64_t Hq, int64_t Hkv, int64_t max_blocks, int64_t bs, int64_t D, int dtype,
                   int sms, PtcPlan* p);
int paged_tc_launch(const void* q, const void* k_cache, const void* v_cache, void* out, const int32_t* bt,
                    const int32_t* cl, void* workspace, int64_t B, int64_t Hq, int64_t Hkv, int64_t num_blocks,
                    int64_t bs, int64_t max_blocks, float scale, const PtcPlan& p, cudaStream_t st);

}  // namespace sa
