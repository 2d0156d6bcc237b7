// tcgen05 grouped GEMM for segment_mm / gather_mm (TF32 and BF16).
#include "grouped_mm.cuh"

namespace bgl {

bool gmm_tensor_core_supported(int64_t d1, int64_t d2, int dtype) {
    (void)d1;
    (void)d2;
    (void)dtype;
    return false;
}

int gmm_tensor_core(const void *, const void *, void *, const GmmLayout &, int64_t, int64_t,
                    int64_t, int64_t, int, cudaStream_t) {
    return fail(BGL_E_UNSUPPORTED, "tensor-core grouped mm not available");
}

}  // namespace bgl
