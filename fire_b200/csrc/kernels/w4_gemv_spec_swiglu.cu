// Instantiations of the K-specialised INT4 GEMV, SwiGLU epilogue (w4_gemv_spec.cuh).
// Gate/up are packed per 4-row tile, so only R = 4 with a full warp per row exists.
#include "w4_gemv_spec.cuh"

namespace fb {

bool w4_spec_swiglu(const W4Args& a, int num_sms, cudaStream_t s, bool pdl, cudaError_t* err) {
    switch (a.K) {
    case 1024: *err = w4::spec_launch<32, 1, 4, kW4Swiglu>(a, num_sms, s, pdl); return true;
    case 2048: *err = w4::spec_launch<32, 2, 4, kW4Swiglu>(a, num_sms, s, pdl); return true;
    case 4096: *err = w4::spec_launch<32, 4, 4, kW4Swiglu>(a, num_sms, s, pdl); return true;
    default: return false;
    }
}

}  // namespace fb
