// gemv.cu -- format dispatch for the decode GEMV (kernels in gemv_impl.cuh).
#include "common.cuh"

namespace bramha {
cudaError_t launch_gemv_w4zp8(const GemvArgs& a, int num_sms, cudaStream_t stream);
cudaError_t launch_gemv_log4(const GemvArgs& a, int num_sms, cudaStream_t stream);
cudaError_t launch_gemv_w8(const GemvArgs& a, int num_sms, cudaStream_t stream);
cudaError_t launch_gemv_f32(const GemvArgs& a, int num_sms, cudaStream_t stream);

cudaError_t launch_gemv(int fmt, const GemvArgs& a, int num_sms, cudaStream_t stream) {
    switch (fmt) {
        case BRAMHA_FMT_W4ZP8: return launch_gemv_w4zp8(a, num_sms, stream);
        case BRAMHA_FMT_LOG4: return launch_gemv_log4(a, num_sms, stream);
        case BRAMHA_FMT_W8: return launch_gemv_w8(a, num_sms, stream);
        case BRAMHA_FMT_F32: return launch_gemv_f32(a, num_sms, stream);
        default: return cudaErrorInvalidValue;
    }
}
}  // namespace bramha
