// gemv.cu -- format dispatch for the decode GEMV (kernels in gemv_impl.cuh).
#include "common.cuh"

namespace bramha {
cudaError_t launch_gemv_w4zp8(const GemvArgs& a, int num_sms, cudaStream_t stream);
cudaError_t launch_gemv_log4(const GemvArgs& a, int num_sms, cudaStream_t stream);
cudaError_t launch_gemv_w8(const GemvArgs& a, int num_sms, cudaStream_t stream);
cudaError_t launch_gemv_f32(const GemvArgs& a, int num_sms, cudaStream_t stream);

// Batches of 1, 2, 4 and 8 rows have their own kernels; any other batch size
// is split into those (largest first), each part a separate launch.
cudaError_t launch_gemv(int fmt, const GemvArgs& a, int num_sms, cudaStream_t stream) {
    GemvArgs part = a;
    int done = 0;
    while (done < a.batch) {
        const int left = a.batch - done;
        const int bc = left >= 8 ? 8 : left >= 4 ? 4 : left >= 2 ? 2 : 1;
        part.batch = bc;
        part.x = a.x + (int64_t)done * a.ldx;
        for (int i = 0; i < a.nseg; ++i) part.seg[i].y = a.seg[i].y + (int64_t)done * a.seg[i].ldy;
        cudaError_t e;
        switch (fmt) {
            case BRAMHA_FMT_W4ZP8: e = launch_gemv_w4zp8(part, num_sms, stream); break;
            case BRAMHA_FMT_LOG4: e = launch_gemv_log4(part, num_sms, stream); break;
            case BRAMHA_FMT_W8: e = launch_gemv_w8(part, num_sms, stream); break;
            case BRAMHA_FMT_F32: e = launch_gemv_f32(part, num_sms, stream); break;
            default: return cudaErrorInvalidValue;
        }
        if (e != cudaSuccess) return e;
        done += bc;
    }
    return cudaSuccess;
}
}  // namespace bramha
