// gemv_w8.cu -- instantiates the decode GEMV (gemv_impl.cuh) for BRAMHA_FMT_W8.
#include "gemv_impl.cuh"

namespace bramha {
cudaError_t launch_gemv_w8(const GemvArgs& a, int num_sms, cudaStream_t stream) {
    return run_gemv<BRAMHA_FMT_W8>(a, num_sms, stream);
}
}  // namespace bramha
