// tcgen05 int8 GEMM for M >= 64 (placeholder: the GEMV family serves all M).
#include "common.cuh"

namespace focr {

bool tc_igemm_eligible(const void *, const int8_t *, size_t, size_t, size_t, const int32_t *) {
    return false;
}

int launch_tc_igemm(const void *, bool, const int8_t *, size_t, size_t, size_t, int32_t *,
                    cudaStream_t) {
    return fail(FOCR_E_UNSUPPORTED, "tcgen05 igemm not available");
}

}  // namespace focr
