// Stage 3 (fused): expert FFN with the hidden tile kept on chip.
#include "common.cuh"

extern "C" int cti_moe_expert_ffn_fused(const void*, const void*, const float*, const void*,
                                        const float*, const int32_t*, int, int, int64_t, int, int,
                                        int, void*, int32_t*, void*) {
  return CTI_ERR_UNSUPPORTED;
}
