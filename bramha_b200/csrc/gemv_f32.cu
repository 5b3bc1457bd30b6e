// gemv_f32.cu -- instantiates the decode GEMV (gemv_impl.cuh) for BRAMHA_FMT_F32.
#include "gemv_impl.cuh"

namespace bramha {
cudaError_t launch_gemv_f32(const GemvArgs& a, int num_sms, cudaStream_t stream) {
    return run_gemv<BRAMHA_FMT_F32>(a, num_sms, stream);
}
}  // namespace bramha
