// Fused single-token MoE decode layer (persistent kernel) -- placeholder
// until the fused path is enabled; the general path serves m == 1.
#include "moe.cuh"

namespace focr {

bool moe_fused_eligible(const focr_moe_layer *) { return false; }

int moe_decode_fused_m1(focr_moe_layer *, const float *, float *, int32_t *, float *,
                        cudaStream_t) {
    return fail(FOCR_E_UNSUPPORTED, "fused m=1 path not available");
}

}  // namespace focr
