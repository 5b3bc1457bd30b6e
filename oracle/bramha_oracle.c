/*
 * bramha_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU arithmetic for the quantized
 * linear-layer path (akshaybhlrp/bramha).  The reference is Rust and cannot be
 * compiled in this environment, so this file restates it operation by
 * operation: same loop structure, same accumulator interleave, same fp32
 * rounding points.  It must be compiled WITHOUT -ffast-math and WITH
 * -ffp-contract=off: Rust/LLVM neither reassociates nor contracts a*b+c into
 * an FMA, and gcc does contract by default in GNU C mode.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load this library, and only as the checker or the timed CPU
 * baseline.  The CUDA product path never calls it.
 *
 * Parity pinning: the reference's own known-answer test for this path is
 * `test_quantization_correctness` (src/inference/cpu_engine.rs:3501-3682);
 * tests/test_oracle.py restates it against this file.  The log4 decoder
 * (spanda-engine/src/lib.rs:332-342) has no reference test: it is pinned only
 * by the reference code itself and by the independent numpy restatement that
 * generated tests/golden/.
 *
 * Threading mirrors Rayon's `par_iter_mut().with_min_len(256)` over output
 * rows with OpenMP dynamic chunks of 256 rows; each row's arithmetic is
 * independent of the thread that runs it, so results do not depend on the
 * thread count.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BRO_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* Rust `f32 as u8` / `f32 as i8` casts saturate and map NaN to 0.            */
static inline uint8_t rust_f32_as_u8(float v) {
    if (isnan(v)) return 0;
    if (v <= 0.0f) return 0;
    if (v >= 255.0f) return 255;
    return (uint8_t)v; /* truncation toward zero, as Rust */
}
static inline int8_t rust_f32_as_i8(float v) {
    if (isnan(v)) return 0;
    if (v <= -128.0f) return -128;
    if (v >= 127.0f) return 127;
    return (int8_t)v;
}
/* Rust `f32::clamp(lo, hi)`: NaN stays NaN. */
static inline float rust_clamp(float v, float lo, float hi) {
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}
/* Rust `f32::round`: half away from zero == C roundf. */
static inline float rust_round(float v) { return roundf(v); }

/* Row max |w| exactly as the reference loop: `if abs > max_abs` (NaN never wins). */
static inline float row_max_abs(const float* row, int64_t K) {
    float m = 0.0f;
    for (int64_t i = 0; i < K; ++i) {
        float a = fabsf(row[i]);
        if (a > m) m = a;
    }
    return m;
}

/* ------------------------------------------------------------------------- */
/* quantize_to_int8  -- src/models/quantization.rs:7-38                        */
BRO_API void bro_quantize_to_int8(const float* w, int64_t N, int64_t K, int8_t* q, float* scales) {
    for (int64_t j = 0; j < N; ++j) {
        const float* row = w + j * K;
        float max_abs = row_max_abs(row, K);
        float scale = (max_abs == 0.0f) ? 1.0f : max_abs / 127.0f;
        scales[j] = scale;
        for (int64_t i = 0; i < K; ++i) {
            float v = rust_clamp(rust_round(row[i] / scale), -127.0f, 127.0f);
            q[j * K + i] = rust_f32_as_i8(v);
        }
    }
}

/* quantize_to_int4  -- src/models/quantization.rs:41-83
 * Returns -1 when K is odd (the reference asserts, :46-49). */
BRO_API int bro_quantize_to_int4(const float* w, int64_t N, int64_t K, uint8_t* q, float* scales) {
    if (K % 2 != 0) return -1;
    const int64_t half = K / 2;
    for (int64_t j = 0; j < N; ++j) {
        const float* row = w + j * K;
        float max_abs = row_max_abs(row, K);
        float scale = (max_abs == 0.0f) ? 1.0f : max_abs / 7.0f;
        scales[j] = scale;
        for (int64_t i = 0; i < half; ++i) {
            float x1 = row[2 * i], x2 = row[2 * i + 1];
            uint8_t q1 = rust_f32_as_u8(rust_clamp(rust_round(x1 / scale), -7.0f, 7.0f) + 8.0f);
            uint8_t q2 = rust_f32_as_u8(rust_clamp(rust_round(x2 / scale), -7.0f, 7.0f) + 8.0f);
            /* `(q1 << 4) | (q2 & 0x0F)` on u8: q1 << 4 wraps modulo 256 in the
             * reference only in debug-panic terms; q1 <= 15 so it never does. */
            q[j * half + i] = (uint8_t)(((q1 << 4) & 0xFF) | (q2 & 0x0F));
        }
    }
    return 0;
}

/* dequantize_int8 -- src/models/quantization.rs:86-99 */
BRO_API void bro_dequantize_int8(const int8_t* q, const float* scales, int64_t N, int64_t K, float* out) {
    for (int64_t j = 0; j < N; ++j)
        for (int64_t i = 0; i < K; ++i) out[j * K + i] = (float)q[j * K + i] * scales[j];
}

/* dequantize_int4 -- src/models/quantization.rs:102-122 */
BRO_API void bro_dequantize_int4(const uint8_t* q, const float* scales, int64_t N, int64_t K, float* out) {
    const int64_t half = K / 2;
    for (int64_t j = 0; j < N; ++j) {
        float s = scales[j];
        for (int64_t i = 0; i < half; ++i) {
            uint8_t b = q[j * half + i];
            float q1 = (float)((b >> 4) & 0x0F) - 8.0f;
            float q2 = (float)(b & 0x0F) - 8.0f;
            out[j * K + 2 * i] = q1 * s;
            out[j * K + 2 * i + 1] = q2 * s;
        }
    }
}

/* dequantize_log4 -- spanda-engine/src/lib.rs:332-342
 * For code c (high nibble first): signum(c) * (2^|c| - 1) * scale.
 * c >= 0 and f32::signum(+0.0) == +1.0, so the value is ((2^c - 1) * 1) * scale,
 * evaluated left to right as the reference does: (signum * (pow - 1)) * scale. */
static inline float log4_decode(unsigned c, float scale) {
    float v = (float)c;
    float sg = 1.0f;                      /* signum of a non-negative float */
    float p = ldexpf(1.0f, (int)c);       /* 2.0f32.powf(c) is exact for c in 0..15 */
    (void)v;
    return (sg * (p - 1.0f)) * scale;
}

BRO_API void bro_dequantize_log4(const uint8_t* data, int64_t nbytes, float scale, float* out) {
    for (int64_t i = 0; i < nbytes; ++i) {
        uint8_t b = data[i];
        out[2 * i] = log4_decode((unsigned)(b >> 4), scale);
        out[2 * i + 1] = log4_decode((unsigned)(b & 0x0F), scale);
    }
}

/* Row-wise log4 dequantization with one scale per output row (the format this
 * project registers: scales.len() == N). */
BRO_API void bro_dequantize_log4_rows(const uint8_t* q, const float* scales, int64_t N, int64_t K, float* out) {
    const int64_t half = K / 2;
    for (int64_t j = 0; j < N; ++j) bro_dequantize_log4(q + j * half, half, scales[j], out + j * K);
}

/* quantize_to_log4 -- DEFINED BY THIS PROJECT (the reference has no encoder).
 * Per row: s = max|w| / 32767 (1.0 for an all-zero row), so the largest code
 * (15 -> 2^15 - 1 = 32767) reproduces max|w|.  Each |w| maps to the code whose
 * decoded value fl((2^c - 1) * s) is nearest, ties to the lower code.  The
 * sign is dropped because the reference decoder cannot represent it.  Byte i
 * of a row holds column 2i in the high nibble, column 2i+1 in the low nibble.
 * Returns -1 when K is odd. */
BRO_API int bro_quantize_to_log4(const float* w, int64_t N, int64_t K, uint8_t* q, float* scales) {
    if (K % 2 != 0) return -1;
    const int64_t half = K / 2;
    for (int64_t j = 0; j < N; ++j) {
        const float* row = w + j * K;
        float max_abs = row_max_abs(row, K);
        float s = (max_abs == 0.0f) ? 1.0f : max_abs / 32767.0f;
        scales[j] = s;
        float d[16];
        for (unsigned c = 0; c < 16; ++c) d[c] = log4_decode(c, s);
        for (int64_t i = 0; i < half; ++i) {
            unsigned code[2];
            for (int t = 0; t < 2; ++t) {
                float a = fabsf(row[2 * i + t]);
                unsigned best = 0;
                float best_err = fabsf(a - d[0]);
                for (unsigned c = 1; c < 16; ++c) {
                    float e = fabsf(a - d[c]);
                    if (e < best_err) { best = c; best_err = e; }
                }
                code[t] = best;
            }
            q[j * half + i] = (uint8_t)((code[0] << 4) | code[1]);
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------- */
/* LUT_Q1 / LUT_Q2 -- src/inference/cpu_engine.rs:108-126 */
static float LUT_Q1[256], LUT_Q2[256];
static float LUT_L1[256], LUT_L2[256]; /* log4 analogue: 2^c - 1 */
static void luts_init(void) {
    static int done = 0;
    if (done) return;
    for (int i = 0; i < 256; ++i) {
        LUT_Q1[i] = (float)((i >> 4) & 0x0F) - 8.0f;
        LUT_Q2[i] = (float)(i & 0x0F) - 8.0f;
        LUT_L1[i] = ldexpf(1.0f, (i >> 4) & 0x0F) - 1.0f;
        LUT_L2[i] = ldexpf(1.0f, i & 0x0F) - 1.0f;
    }
    done = 1;
}

static inline void set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

/* matvec_mul_into, Float branch -- cpu_engine.rs:1311-1335 */
static inline float row_dot_f32_into(const float* h, const float* w, int64_t K) {
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int64_t chunks = K / 4, rem = K % 4;
    for (int64_t i = 0; i < chunks; ++i) {
        int64_t b = i * 4;
        s0 += h[b] * w[b];
        s1 += h[b + 1] * w[b + 1];
        s2 += h[b + 2] * w[b + 2];
        s3 += h[b + 3] * w[b + 3];
    }
    for (int64_t i = chunks * 4; i < chunks * 4 + rem; ++i) s0 += h[i] * w[i];
    return s0 + s1 + s2 + s3;
}

/* matvec_mul_into, QuantizedI8 branch -- cpu_engine.rs:1337-1361 */
static inline float row_dot_i8_into(const float* h, const int8_t* w, int64_t K) {
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int64_t chunks = K / 4, rem = K % 4;
    for (int64_t i = 0; i < chunks; ++i) {
        int64_t b = i * 4;
        s0 += h[b] * (float)w[b];
        s1 += h[b + 1] * (float)w[b + 1];
        s2 += h[b + 2] * (float)w[b + 2];
        s3 += h[b + 3] * (float)w[b + 3];
    }
    for (int64_t i = chunks * 4; i < chunks * 4 + rem; ++i) s0 += h[i] * (float)w[i];
    return s0 + s1 + s2 + s3;
}

/* matvec_mul_into, QuantizedU4 branch -- cpu_engine.rs:1363-1411.
 * Also used with the log4 tables for the fused log4 CPU baseline. */
static inline float row_dot_nib_into(const float* h, const uint8_t* rb, int64_t half,
                                     const float* L1, const float* L2) {
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int64_t chunks = half / 8;
    for (int64_t c = 0; c < chunks; ++c) {
        int64_t bb = c * 8, bh = c * 16;
        uint8_t b0 = rb[bb], b1 = rb[bb + 1], b2 = rb[bb + 2], b3 = rb[bb + 3];
        uint8_t b4 = rb[bb + 4], b5 = rb[bb + 5], b6 = rb[bb + 6], b7 = rb[bb + 7];
        s0 += h[bh] * L1[b0] + h[bh + 1] * L2[b0];
        s1 += h[bh + 2] * L1[b1] + h[bh + 3] * L2[b1];
        s2 += h[bh + 4] * L1[b2] + h[bh + 5] * L2[b2];
        s3 += h[bh + 6] * L1[b3] + h[bh + 7] * L2[b3];
        s0 += h[bh + 8] * L1[b4] + h[bh + 9] * L2[b4];
        s1 += h[bh + 10] * L1[b5] + h[bh + 11] * L2[b5];
        s2 += h[bh + 12] * L1[b6] + h[bh + 13] * L2[b6];
        s3 += h[bh + 14] * L1[b7] + h[bh + 15] * L2[b7];
    }
    float sum = s0 + s1 + s2 + s3;
    for (int64_t i = chunks * 8; i < half; ++i) {
        uint8_t b = rb[i];
        sum += h[2 * i] * L1[b] + h[2 * i + 1] * L2[b];
    }
    return sum;
}

BRO_API void bro_matvec_into_f32(const float* h, int64_t K, const float* w, int64_t N, float* out, int threads) {
    set_threads(threads);
#pragma omp parallel for schedule(dynamic, 256) if (threads != 1)
    for (int64_t j = 0; j < N; ++j) out[j] = row_dot_f32_into(h, w + j * K, K);
}

BRO_API void bro_matvec_into_i8(const float* h, int64_t K, const int8_t* q, const float* scales, int64_t N,
                                float* out, int threads) {
    set_threads(threads);
#pragma omp parallel for schedule(dynamic, 256) if (threads != 1)
    for (int64_t j = 0; j < N; ++j) out[j] = row_dot_i8_into(h, q + j * K, K) * scales[j];
}

BRO_API void bro_matvec_into_u4(const float* h, int64_t K, const uint8_t* q, const float* scales, int64_t N,
                                float* out, int threads) {
    luts_init();
    const int64_t half = K / 2;
    set_threads(threads);
#pragma omp parallel for schedule(dynamic, 256) if (threads != 1)
    for (int64_t j = 0; j < N; ++j) out[j] = row_dot_nib_into(h, q + j * half, half, LUT_Q1, LUT_Q2) * scales[j];
}

/* log4 GEMV as the reference would run it: dequantize_log4 of each row with
 * that row's scale (spanda-engine/src/lib.rs:332-342), then the Float branch
 * of matvec_mul_into (cpu_engine.rs:1311-1335).  This is the parity oracle. */
BRO_API void bro_matvec_into_log4(const float* h, int64_t K, const uint8_t* q, const float* scales, int64_t N,
                                  float* out, int threads) {
    const int64_t half = K / 2;
    set_threads(threads);
#pragma omp parallel
    {
        float* row = (float*)malloc(sizeof(float) * (size_t)(K > 0 ? K : 1));
#pragma omp for schedule(dynamic, 256)
        for (int64_t j = 0; j < N; ++j) {
            bro_dequantize_log4(q + j * half, half, scales[j], row);
            if (K % 2) row[K - 1] = 0.0f; /* odd K: the packed row covers K-1 columns */
            out[j] = row_dot_f32_into(h, row, K);
        }
        free(row);
    }
}

/* Fused log4 GEMV in the reference's U4 loop style (same 8-byte chunking and
 * accumulator interleave, tables 2^c - 1 instead of q - 8, scale at the end).
 * It is the timed CPU baseline for log4: the reference has no fused log4
 * GEMV, and dequantizing each row first would only make the CPU slower. */
BRO_API void bro_matvec_fused_log4(const float* h, int64_t K, const uint8_t* q, const float* scales, int64_t N,
                                   float* out, int threads) {
    luts_init();
    const int64_t half = K / 2;
    set_threads(threads);
#pragma omp parallel for schedule(dynamic, 256) if (threads != 1)
    for (int64_t j = 0; j < N; ++j) out[j] = row_dot_nib_into(h, q + j * half, half, LUT_L1, LUT_L2) * scales[j];
}

/* ------------------------------------------------------------------------- */
/* matvec_mul (allocating variant, single accumulator) -- cpu_engine.rs:355-562 */
BRO_API void bro_matvec_f32(const float* h, int64_t K, const float* w, int64_t N, float* out) {
    for (int64_t j = 0; j < N; ++j) {
        float s = 0.0f;
        for (int64_t i = 0; i < K; ++i) s += h[i] * w[j * K + i];
        out[j] = s;
    }
}
BRO_API void bro_matvec_i8(const float* h, int64_t K, const int8_t* q, const float* scales, int64_t N, float* out) {
    for (int64_t j = 0; j < N; ++j) {
        float s = 0.0f;
        for (int64_t i = 0; i < K; ++i) s += h[i] * (float)q[j * K + i];
        out[j] = s * scales[j];
    }
}
BRO_API void bro_matvec_u4(const float* h, int64_t K, const uint8_t* q, const float* scales, int64_t N, float* out) {
    const int64_t half = K / 2;
    for (int64_t j = 0; j < N; ++j) {
        float s = 0.0f;
        for (int64_t i = 0; i < half; ++i) {
            uint8_t b = q[j * half + i];
            float q1 = (float)((b >> 4) & 0x0F) - 8.0f;
            float q2 = (float)(b & 0x0F) - 8.0f;
            s += h[2 * i] * q1 + h[2 * i + 1] * q2;
        }
        out[j] = s * scales[j];
    }
}

/* ------------------------------------------------------------------------- */
/* gemm_cpu, sequential branch -- cpu_engine.rs:565-706.  Loop j outer, b inner. */
BRO_API void bro_gemm_f32(const float* hb, int64_t M, int64_t K, const float* w, int64_t N, float* out) {
    for (int64_t j = 0; j < N; ++j) {
        const float* ws = w + j * K;
        for (int64_t b = 0; b < M; ++b) {
            const float* hr = hb + b * K;
            float s = 0.0f;
            for (int64_t i = 0; i < K; ++i) s += hr[i] * ws[i];
            out[b * N + j] = s;
        }
    }
}
BRO_API void bro_gemm_i8(const float* hb, int64_t M, int64_t K, const int8_t* q, const float* scales, int64_t N,
                         float* out) {
    for (int64_t j = 0; j < N; ++j) {
        const int8_t* ws = q + j * K;
        float sc = scales[j];
        for (int64_t b = 0; b < M; ++b) {
            const float* hr = hb + b * K;
            float s = 0.0f;
            for (int64_t i = 0; i < K; ++i) s += hr[i] * (float)ws[i];
            out[b * N + j] = s * sc;
        }
    }
}
BRO_API void bro_gemm_u4(const float* hb, int64_t M, int64_t K, const uint8_t* q, const float* scales, int64_t N,
                         float* out) {
    luts_init();
    const int64_t half = K / 2;
    for (int64_t j = 0; j < N; ++j) {
        const uint8_t* rb = q + j * half;
        float sc = scales[j];
        for (int64_t b = 0; b < M; ++b)
            out[b * N + j] = row_dot_nib_into(hb + b * K, rb, half, LUT_Q1, LUT_Q2) * sc;
    }
}
/* log4 prefill as the reference would run it: dequantize, then gemm_cpu Float. */
BRO_API void bro_gemm_log4(const float* hb, int64_t M, int64_t K, const uint8_t* q, const float* scales, int64_t N,
                           float* out) {
    float* w = (float*)malloc(sizeof(float) * (size_t)(N * K > 0 ? N * K : 1));
    bro_dequantize_log4_rows(q, scales, N, K, w);
    if (K % 2)
        for (int64_t j = 0; j < N; ++j) w[j * K + K - 1] = 0.0f;
    bro_gemm_f32(hb, M, K, w, N, out);
    free(w);
}

/* Multi-threaded row-parallel variant of the gemm used only for timing large
 * CPU samples (gemm_cpu itself is sequential in the reference). */
BRO_API void bro_gemm_u4_par(const float* hb, int64_t M, int64_t K, const uint8_t* q, const float* scales,
                             int64_t N, float* out, int threads) {
    luts_init();
    const int64_t half = K / 2;
    set_threads(threads);
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t j = 0; j < N; ++j) {
        const uint8_t* rb = q + j * half;
        float sc = scales[j];
        for (int64_t b = 0; b < M; ++b)
            out[b * N + j] = row_dot_nib_into(hb + b * K, rb, half, LUT_Q1, LUT_Q2) * sc;
    }
}

BRO_API int bro_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---- decode step -------------------------------------
 * The per-token operations around the quantized GEMVs, in the reference's own
 * loop order (sequential fp32 sums, no FMA contraction). */

/* rms_norm_into, src/inference/cpu_engine.rs:1292-1302 */
BRO_API void bro_rms_norm(const float* x, const float* w, int64_t n, float eps, float* out) {
    float variance = 0.0f;
    for (int64_t i = 0; i < n; ++i) variance += x[i] * x[i];
    variance /= (float)n;
    const float scale = 1.0f / sqrtf(variance + eps);
    for (int64_t i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

/* apply_rope_cpu, cpu_engine.rs:1682-1698, with get_rope_thetas
 * (theta_i = 1 / base^(2i / head_dim), cpu_engine.rs:1515-1530): the two
 * halves of each head rotate together ("half-split"). */
BRO_API void bro_rope(float* v, int64_t pos, int num_heads, int head_dim, float rope_theta) {
    const int half = head_dim / 2;
    for (int h = 0; h < num_heads; ++h) {
        float* hv = v + (int64_t)h * head_dim;
        for (int i = 0; i < half; ++i) {
            const float theta = 1.0f / powf(rope_theta, (float)(2 * i) / (float)head_dim);
            const float freq = (float)pos * theta;
            const float c = cosf(freq), s = sinf(freq);
            const float x1 = hv[i], x2 = hv[i + half];
            hv[i] = x1 * c - x2 * s;
            hv[i + half] = x2 * c + x1 * s;
        }
    }
}

/* flash_attention_single_into, cpu_engine.rs:1450-1509: per query head, one
 * pass over the cached tokens with a running max m, sum l and output o.
 * k_cache / v_cache are [kv_len][num_kv_heads * head_dim]. */
BRO_API void bro_attention(const float* q, const float* k_cache, const float* v_cache, int64_t kv_len,
                           int num_q_heads, int num_kv_heads, int head_dim, float* out) {
    const float scale = 1.0f / sqrtf((float)head_dim);
    const int heads_per_kv = num_q_heads / num_kv_heads;
    float o[256];
    for (int head = 0; head < num_q_heads; ++head) {
        const int kv_head = head / heads_per_kv;
        const float* qh = q + (int64_t)head * head_dim;
        for (int d = 0; d < head_dim; ++d) o[d] = 0.0f;
        float m = -INFINITY, l = 0.0f;
        for (int64_t t = 0; t < kv_len; ++t) {
            const int64_t off = t * num_kv_heads * head_dim + (int64_t)kv_head * head_dim;
            float dot = 0.0f;
            for (int d = 0; d < head_dim; ++d) dot += qh[d] * k_cache[off + d];
            const float score = dot * scale;
            if (score > m) {
                const float e = expf(m - score);
                l = l * e + 1.0f;
                for (int d = 0; d < head_dim; ++d) o[d] = o[d] * e + v_cache[off + d];
                m = score;
            } else {
                const float e = expf(score - m);
                l += e;
                for (int d = 0; d < head_dim; ++d) o[d] += e * v_cache[off + d];
            }
        }
        const float inv_l = 1.0f / l;
        for (int d = 0; d < head_dim; ++d) out[(int64_t)head * head_dim + d] = o[d] * inv_l;
    }
}

/* SwiGLU of run_mlp_into, cpu_engine.rs:2023-2026 (dense branch of :1775-2035): silu(g) * u with
 * silu(g) = g * (1 / (1 + exp(-g))). */
BRO_API void bro_silu_mul(const float* g, const float* u, int64_t n, float* out) {
    for (int64_t d = 0; d < n; ++d) {
        const float silu = g[d] * (1.0f / (1.0f + expf(-g[d])));
        out[d] = silu * u[d];
    }
}

/* Repetition penalty 1.15 over every entry of the generated list (an id that
 * appears twice is penalised twice), then greedy argmax (first maximum);
 * cpu_engine.rs:2985-3031.  Modifies logits in place. */
BRO_API int64_t bro_penalty_argmax(float* logits, int64_t vocab, const int32_t* generated, int64_t n_generated,
                                   float penalty) {
    for (int64_t i = 0; i < n_generated; ++i) {
        const int64_t idx = (int64_t)(uint32_t)generated[i];
        if (idx < vocab) {
            const float logit = logits[idx];
            logits[idx] = logit > 0.0f ? logit / penalty : logit * penalty;
        }
    }
    int64_t max_idx = 0;
    float max_val = -INFINITY;
    for (int64_t i = 0; i < vocab; ++i)
        if (logits[i] > max_val) {
            max_val = logits[i];
            max_idx = i;
        }
    return max_idx;
}

/* ---- 2:4 structured sparsity ------------------------------------------------
 * The two kept columns of a group of four.  The reference sorts the pairs
 * (index, |w|) with Rust's stable slice::sort_by under
 * `b.1.partial_cmp(&a.1).unwrap_or(Equal)` (spanda-engine/src/sparse.rs:35-47,
 * cpu_engine.rs:1542-1552, bin/convert.rs:65-74); for four elements the
 * standard library runs insertion sort (insertion_sort_shift_left), in which an
 * element moves left only past strictly smaller magnitudes.  Restated here
 * literally: descending magnitude, ties in column order, a NaN never moves. */
static void top2_of4(const float m[4], int* i1, int* i2) {
    int o[4] = {0, 1, 2, 3};
    for (int i = 1; i < 4; ++i) {
        const int t = o[i];
        int j = i;
        while (j > 0 && m[t] > m[o[j - 1]]) {
            o[j] = o[j - 1];
            --j;
        }
        o[j] = t;
    }
    *i1 = o[0];
    *i2 = o[1];
}

/* Unscaled code of column c of row `row` for fmt 0 = f32, 1 = i8, 2 = int4
 * (even column in the high nibble, value nibble - 8). */
static float sp_code(int fmt, const void* row, int64_t c) {
    if (fmt == 0) return ((const float*)row)[c];
    if (fmt == 1) return (float)((const int8_t*)row)[c];
    const uint8_t b = ((const uint8_t*)row)[c / 2];
    return (float)((c % 2 == 0) ? ((b >> 4) & 0x0F) : (b & 0x0F)) - 8.0f;
}

/* sparse_matvec_mul_2_4_tensor_into, cpu_engine.rs:1532-1640 (its f32 arm is
 * sparse_matvec_mul_2_4, sparse.rs:19-61): per row, the top two products of
 * every whole group of four (largest magnitude first), then the K % 4
 * trailing columns densely; times the row scale for i8 / int4.  Rows in
 * parallel when threads > 1 (the reference's par_iter_mut). */
BRO_API void bro_sparse_matvec_2_4(int fmt, const float* h, int64_t K, const void* q, const float* scales, int64_t N,
                                   float* out, int threads) {
    const int64_t rb = fmt == 0 ? K * 4 : fmt == 1 ? K : K / 2;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1) if (threads > 1)
    for (int64_t j = 0; j < N; ++j) {
        const void* row = (const uint8_t*)q + j * rb;
        float sum = 0.0f;
        int64_t c = 0;
        while (c + 4 <= K) {
            float v[4], m[4];
            for (int i = 0; i < 4; ++i) {
                v[i] = sp_code(fmt, row, c + i);
                m[i] = fabsf(v[i]);
            }
            int i1, i2;
            top2_of4(m, &i1, &i2);
            sum += v[i1] * h[c + i1];
            sum += v[i2] * h[c + i2];
            c += 4;
        }
        while (c < K) {
            sum += sp_code(fmt, row, c) * h[c];
            ++c;
        }
        out[j] = fmt == 0 ? sum : sum * scales[j];
    }
}

/* sparse_matvec_2_4_compressed, sparse.rs:100-138: masks [rows][cols/4] (low 4
 * bits), values consumed in column order from 2*r*(cols/4) while any remain;
 * columns past the last whole group are ignored. */
BRO_API void bro_sparse_matvec_2_4_compressed(const float* x, const uint16_t* masks, const float* values,
                                              int64_t n_values, int64_t rows, int64_t cols, float* out,
                                              int threads) {
    const int64_t cpr = cols / 4;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1) if (threads > 1)
    for (int64_t r = 0; r < rows; ++r) {
        int64_t vi = r * cpr * 2;
        float sum = 0.0f;
        for (int64_t c = 0; c < cpr; ++c) {
            const uint16_t m = masks[r * cpr + c];
            for (int bit = 0; bit < 4; ++bit)
                if ((m & (1u << bit)) && vi < n_values) {
                    sum += values[vi] * x[c * 4 + bit];
                    ++vi;
                }
        }
        out[r] = sum;
    }
}

/* bin/convert.rs:55-92: 2:4 compression of a flat f32 tensor whose length is a
 * multiple of 4: per group of four consecutive elements the mask of the top
 * two and their values in index order.  Returns the number of values (n/2). */
BRO_API int64_t bro_compress_2_4(const float* w, int64_t n, uint16_t* masks, float* values) {
    int64_t nv = 0;
    for (int64_t g = 0; g < n / 4; ++g) {
        float m[4];
        for (int i = 0; i < 4; ++i) m[i] = fabsf(w[4 * g + i]);
        int i1, i2;
        top2_of4(m, &i1, &i2);
        const uint16_t mask = (uint16_t)((1u << i1) | (1u << i2));
        masks[g] = mask;
        for (int bit = 0; bit < 4; ++bit)
            if (mask & (1u << bit)) values[nv++] = w[4 * g + bit];
    }
    return nv;
}

/* ---- MoE expert MLP (run_mlp_into's MoE branch, cpu_engine.rs:1799-1989) -----
 * One decode token per row of h [T][H]; router logits [T][E] given (the router
 * itself is a matvec_mul_into, :1801-1803, restated above).  Per token:
 *  - softmax: max by f32::max fold, exps = exp(l - max), sequential sum, probs
 *    = exps / sum when sum > 0 (:1805-1820);
 *  - stable sort by probability, descending (slice::sort_by with
 *    partial_cmp, :1822-1825): for finite values the order (-p, index);
 *  - the first top_k, skipping weights <= 0 (:1826-1834);
 *  - per expert: gate and up by matvec_mul_into, silu(g) = g / (1 + exp(-g))
 *    times up (:1924-1936), down by matvec_mul_into (:1938-1942), then
 *    out += down * weight in the sorted order (:1944-1946), from out = 0.
 * fmt: 0 f32, 1 int8, 2 int4, 3 log4; expert weights stacked [E][I][.] for
 * gate / up and [E][H][.] for down, scales [E][I] / [E][H].  Tokens in
 * parallel when threads > 1; each token's arithmetic is sequential. */
static void matvec_into_fmt(int fmt, const float* h, int64_t K, const void* q, const float* s, int64_t N, float* out) {
    switch (fmt) {
        case 0: bro_matvec_into_f32(h, K, (const float*)q, N, out, 1); break;
        case 1: bro_matvec_into_i8(h, K, (const int8_t*)q, s, N, out, 1); break;
        case 2: bro_matvec_into_u4(h, K, (const uint8_t*)q, s, N, out, 1); break;
        default: bro_matvec_into_log4(h, K, (const uint8_t*)q, s, N, out, 1); break;
    }
}

static int64_t fmt_row_bytes(int fmt, int64_t K) { return fmt == 0 ? 4 * K : fmt == 1 ? K : K / 2; }

BRO_API void bro_moe_mlp(int fmt, const float* h, int64_t T, int64_t H, int64_t I, int E, int top_k,
                         const float* logits, const void* gate_q, const float* gate_s, const void* up_q,
                         const float* up_s, const void* down_q, const float* down_s, float* out,
                         int32_t* sel_ids, float* sel_w, int threads) {
    luts_init();
    const int64_t gb = fmt_row_bytes(fmt, H) * I, db = fmt_row_bytes(fmt, I) * H;
    const int k = top_k < E ? top_k : E;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1) if (threads > 1)
    for (int64_t t = 0; t < T; ++t) {
        const float* lg = logits + t * E;
        float* probs = (float*)malloc(sizeof(float) * (size_t)E);
        int* order = (int*)malloc(sizeof(int) * (size_t)E);
        float* g = (float*)malloc(sizeof(float) * (size_t)(3 * I + H));
        float* u = g + I;
        float* m = u + I;
        float* dn = m + I;
        float mx = -INFINITY;
        for (int i = 0; i < E; ++i) mx = fmaxf(mx, lg[i]);
        float sum = 0.0f;
        for (int i = 0; i < E; ++i) {
            probs[i] = expf(lg[i] - mx);
            sum += probs[i];
        }
        for (int i = 0; i < E; ++i) probs[i] = sum > 0.0f ? probs[i] / sum : 0.0f;
        for (int i = 0; i < E; ++i) order[i] = i;
        for (int i = 1; i < E; ++i) {  /* stable insertion sort, descending */
            const int o = order[i];
            int j = i;
            while (j > 0 && probs[o] > probs[order[j - 1]]) {
                order[j] = order[j - 1];
                --j;
            }
            order[j] = o;
        }
        float* y = out + t * H;
        for (int64_t d = 0; d < H; ++d) y[d] = 0.0f;
        for (int r = 0; r < k; ++r) {
            const int e = order[r];
            const float w = probs[e];
            if (sel_ids) sel_ids[t * k + r] = e;
            if (sel_w) sel_w[t * k + r] = w;
            if (w <= 0.0f) continue;
            const float* hh = h + t * H;
            matvec_into_fmt(fmt, hh, H, (const uint8_t*)gate_q + e * gb, gate_s ? gate_s + (int64_t)e * I : NULL, I, g);
            matvec_into_fmt(fmt, hh, H, (const uint8_t*)up_q + e * gb, up_s ? up_s + (int64_t)e * I : NULL, I, u);
            for (int64_t d = 0; d < I; ++d) {
                const float gd = g[d];
                const float silu = gd / (1.0f + expf(-gd));
                m[d] = silu * u[d];
            }
            matvec_into_fmt(fmt, m, I, (const uint8_t*)down_q + e * db, down_s ? down_s + (int64_t)e * H : NULL, H, dn);
            for (int64_t d = 0; d < H; ++d) y[d] += dn[d] * w;
        }
        free(g);
        free(order);
        free(probs);
    }
}
