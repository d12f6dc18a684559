// Prefill-side (M >= 64) dequant-GEMM on the tcgen05 tensor cores.
#include "oq_common.cuh"

namespace oq {

int gemm_tcgen05_supported(int64_t, int64_t, int64_t, int, const void *, const uint8_t *, const float *) {
    return 0;
}

int gemm_tcgen05_launch(const void *, int, const uint8_t *, const float *, float *, int64_t, int64_t, int64_t, int,
                        cudaStream_t) {
    set_error("tcgen05 GEMM not available");
    return OQ_ERR_UNSUPPORTED;
}

}  // namespace oq
