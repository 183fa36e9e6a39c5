// Instantiations of the K-specialised INT4 GEMV, residual epilogue (w4_gemv_spec.cuh).
#include "w4_gemv_spec.cuh"

namespace fb {

bool w4_spec_residual(const W4Args& a, int rows_per_lane, int num_sms, cudaStream_t s, bool pdl, cudaError_t* err) {
    return rows_per_lane == 4 ? w4::spec_dispatch<4, kW4Residual>(a, num_sms, s, pdl, err)
                              : w4::spec_dispatch<2, kW4Residual>(a, num_sms, s, pdl, err);
}

}  // namespace fb
