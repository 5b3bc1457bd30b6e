// decode.cu -- the per-token operations of a decoder-only model's single-token
// decode step around the quantized GEMVs, restating the
// reference's fast decode path, src/inference/cpu_engine.rs:2819-3064:
//   embedding lookup (:2821-2825), RMSNorm (:1292-1302), bias + RoPE
//   (:2895-2903, :1682-1698, thetas :1515-1530) + KV append (:2909),
//   single-token GQA attention (:1450-1509), SiLU * up (:2023-2026), and the
//   repetition penalty 1.15 + greedy argmax (:2985-3031).
// Every kernel reads the token id and position from device memory, so a whole
// decode step (these kernels and the GEMV launches) can be captured once in a
// CUDA graph and replayed token after token without host work.  All are
// programmatically dependent launches (see pdl_entry).
// Floating-point expressions keep the reference's operation order; products
// and sums that the reference writes separately are kept separate
// (__fmul_rn / __fadd_rn: no FMA contraction) where a kernel restates a
// formula term by term.  Reductions (RMSNorm, attention, argmax) use a fixed
// tree order, so results are bit-reproducible run to run.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "common.cuh"

namespace bramha {
namespace {

constexpr int kNormThreads = 1024;

// Programmatic dependent launch: every kernel here is launched with the PDL
// attribute.  At entry it lets the next kernel of the stream be scheduled, then
// waits for the previous one to complete (and its writes to be visible) before
// touching any data, so the launch latency of consecutive kernels overlaps.
__device__ __forceinline__ void pdl_entry() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Block-wide sum in a fixed order (warp trees, then warp 0 over the partials).
template <int THREADS>
__device__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = lane < THREADS / 32 ? red[lane] : 0.f;
    if (warp == 0) v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
    __syncthreads();
    v = red[0];
    __syncthreads();
    return v;
}

// x = table[(token mod vocab)]
__global__ void embed_kernel(const float* __restrict__ table, int64_t vocab, int64_t hidden,
                             const int32_t* __restrict__ token, float* __restrict__ x) {
    pdl_entry();
    const uint32_t t = (uint32_t)*token;
    const int64_t row = (int64_t)(t % (uint64_t)vocab);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hidden; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = table[row * hidden + i];
}

// x += delta (when given: the residual of the previous block), then
// out = x * (1 / sqrt(mean(x^2) + eps)) * w.  One CTA.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta,
                                                               const float* __restrict__ w, int n, float eps,
                                                               float* __restrict__ out) {
    __shared__ float red[32];
    pdl_entry();
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += kNormThreads) {
        float v = x[i];
        if (delta) {
            v = __fadd_rn(v, delta[i]);
            x[i] = v;
        }
        ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
    const float var = block_sum<kNormThreads>(ss, red) / (float)n;
    const float scale = 1.0f / sqrtf(__fadd_rn(var, eps));
    for (int i = threadIdx.x; i < n; i += kNormThreads) out[i] = __fmul_rn(__fmul_rn(x[i], scale), w[i]);
}

// Biases, RoPE of q and k at position *pos (half-split pairs (i, i + hd/2)),
// then k and v appended to the caches at row *pos (rows >= max_ctx are not
// written: the host keeps positions below the cache capacity).
__global__ void qkv_rope_kernel(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                                const float* __restrict__ bq, const float* __restrict__ bk,
                                const float* __restrict__ bv, int nq, int nkv, int hd, float rope_theta,
                                const int32_t* __restrict__ pos_ptr, int64_t max_ctx, float* __restrict__ k_cache,
                                float* __restrict__ v_cache) {
    pdl_entry();
    const int pos = *pos_ptr;
    const bool store_kv = pos >= 0 && pos < max_ctx;
    const int half = hd / 2;
    const int64_t row = (int64_t)pos * nkv * hd;
    const int npairs = (nq + nkv) * half;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < npairs; idx += gridDim.x * blockDim.x) {
        const int h = idx / half, i = idx - h * half;
        const float theta = 1.0f / powf(rope_theta, (float)(2 * i) / (float)hd);
        const float freq = __fmul_rn((float)pos, theta);
        const float c = cosf(freq), s = sinf(freq);
        if (h < nq) {
            const int a = h * hd + i, b = a + half;
            const float x1 = bq ? __fadd_rn(q[a], bq[a]) : q[a];
            const float x2 = bq ? __fadd_rn(q[b], bq[b]) : q[b];
            q[a] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
            q[b] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
        } else {
            const int hk = h - nq;
            const int a = hk * hd + i, b = a + half;
            const float x1 = bk ? __fadd_rn(k[a], bk[a]) : k[a];
            const float x2 = bk ? __fadd_rn(k[b], bk[b]) : k[b];
            if (store_kv) {
                k_cache[row + a] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
                k_cache[row + b] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
                v_cache[row + a] = bv ? __fadd_rn(v[a], bv[a]) : v[a];
                v_cache[row + b] = bv ? __fadd_rn(v[b], bv[b]) : v[b];
            }
        }
    }
}

// Single-token attention (grouped-query: query head h reads kv head
// h / (nq / nkv)), split over the cached tokens: a grid of nq x S CTAs, S =
// attn_splits(max_ctx), CTA (h, s) takes the s-th contiguous range of the
// *pos + 1 tokens.  It computes the scores of its range (a warp per token,
// lanes across the head dims), its own softmax statistics m_s = max score and
// l_s = sum exp(score - m_s), and o_s = sum exp(score - m_s) v; the last CTA of a
// head to finish (a ticket) combines the splits in split order:
// out = sum_s o_s exp(m_s - M) / sum_s l_s exp(m_s - M), M = max_s m_s.  The same
// softmax as the reference's single pass up to rounding, in a fixed order (bit-
// reproducible).
// A launch is a short chain of dependent memory round trips, so every step
// issues all its loads before it uses any: before the programmatic-launch wait
// the CTA prefetches its range's key and value rows into L2 (rows written by
// earlier steps; a prefetch does not change what a later load returns), the
// range is copied into shared memory kAttnChunk rows at a time with all loads of
// a chunk in flight, and the combining CTA copies the head's S partial results
// into shared memory in one pass.  The arithmetic and its order are those of a
// plain row-by-row loop (warp w takes rows w, w + 4, ... of the range).
// Split count measured on the Qwen2-0.5B step (14 heads, 512-640 tokens, loads
// not yet staged): one CTA per head 2.23 ms/token, 8 splits 1.67, 16 splits
// 1.38, 32 splits 1.33, 64 splits 1.49: a split takes about kAttnSplitTokens of
// the cache's capacity, at most kAttnMaxSplits splits.
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxHd = 128;
constexpr int kAttnSplitTokens = 20;
constexpr int kAttnMaxSplits = 64;
constexpr int kAttnChunk = 32;  // cache rows staged in shared memory at a time
// workspace floats per (head, split): m, l, two unused, o[hd] (16-byte aligned rows)
constexpr int kAttnPart = 4 + kAttnMaxHd;
// shared staging: a chunk of key and value rows, or the S partial results of a head
constexpr int kAttnStage = 2 * kAttnChunk * kAttnMaxHd > kAttnMaxSplits * kAttnPart ? 2 * kAttnChunk * kAttnMaxHd
                                                                                       : kAttnMaxSplits * kAttnPart;
static_assert(kAttnChunk % (kAttnThreads / 32) == 0, "a row keeps its warp from chunk to chunk");
inline int attn_splits(int64_t max_ctx) {
    const int64_t s = (max_ctx + kAttnSplitTokens - 1) / kAttnSplitTokens;
    return (int)(s < 1 ? 1 : s > kAttnMaxSplits ? kAttnMaxSplits : s);
}

// Rows [t0, t0 + n) of the kv_len cached tokens belong to split `split` of S.
__device__ __forceinline__ void attn_range(int kv_len, int S, int split, int& t0, int& n) {
    const int per = (kv_len + S - 1) / S;
    t0 = min(kv_len, split * per);
    n = min(kv_len, t0 + per) - t0;
}

// L2 prefetch of this CTA's key and value rows, for a position read before the
// programmatic-launch wait: a hint only (any value read gives rows inside the
// caches' max_ctx rows).
__device__ __forceinline__ void attn_prefetch(const int32_t* pos_ptr, int64_t max_ctx, const float* k_cache,
                                              const float* v_cache, int kvh, int ld, int hd) {
    const int kv_len = (int)min((int64_t)max(__ldcg(pos_ptr) + 1, 1), max_ctx);
    int t0, n;
    attn_range(kv_len, gridDim.y, blockIdx.y, t0, n);
    const int lines = (hd + 31) / 32;  // 128-byte lines of a row
    const int per_cache = n * lines;
    for (int e = threadIdx.x; e < 2 * per_cache; e += kAttnThreads) {
        const int which = e >= per_cache, rem = which ? e - per_cache : e;
        const int r = rem / lines, b = rem - r * lines;
        const float* p = (which ? v_cache : k_cache) + (int64_t)(t0 + r) * ld + kvh * hd + b * 32;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
    }
}

// Copies rows [c0, c0 + nc) of kv head kvh from cache a into as (row stride hd
// floats), and from cache b into bs when bs is not null; row `newrow` comes from
// an / bn instead when they are given.  vec4 (hd % 4 == 0, 16-byte aligned
// caches and rows): float4 loads, every load of the chunk in flight before the
// first store.
__device__ __forceinline__ void attn_stage(const float* __restrict__ a, const float* an, float* as,
                                           const float* __restrict__ b, const float* bn, float* bs, int newrow,
                                           int kvh, int ld, int hd, int c0, int nc, bool vec4) {
    if (vec4) {
        constexpr int kPer = kAttnChunk * kAttnMaxHd / 4 / kAttnThreads;
        const int hd4 = hd >> 2, tot = nc * hd4;
        float4 ra[kPer], rb[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int e = threadIdx.x + j * kAttnThreads;
            if (e < tot) {
                const int r = e / hd4, c = e - r * hd4, t = c0 + r;
                const bool fresh = an && t == newrow;
                const int64_t off = (int64_t)t * ld + kvh * hd;
                ra[j] = reinterpret_cast<const float4*>(fresh ? an : a + off)[c];
                if (bs) rb[j] = reinterpret_cast<const float4*>(fresh ? bn : b + off)[c];
            }
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int e = threadIdx.x + j * kAttnThreads;
            if (e < tot) {
                reinterpret_cast<float4*>(as)[e] = ra[j];
                if (bs) reinterpret_cast<float4*>(bs)[e] = rb[j];
            }
        }
    } else {
        for (int e = threadIdx.x; e < nc * hd; e += kAttnThreads) {
            const int r = e / hd, d = e - r * hd, t = c0 + r;
            const bool fresh = an && t == newrow;
            const int64_t off = (int64_t)t * ld + kvh * hd + d;
            as[e] = fresh ? an[d] : a[off];
            if (bs) bs[e] = fresh ? bn[d] : b[off];
        }
    }
}

// The attention core of one CTA (see above).  qs: the query head (shared
// memory); kn / vn: the newest token's key / value row (shared memory, 16-byte
// aligned) used for token kv_len - 1 instead of the cache, or null; sc: shared
// scores of the CTA's range; stage: kAttnStage floats of 16-byte aligned shared
// memory.
__device__ void attend_split(const float* qs, const float* kn, const float* vn, const float* __restrict__ k_cache,
                             const float* __restrict__ v_cache, int kvh, int ld, int hd, int kv_len, int head,
                             float* sc, float* red, float (*part)[kAttnMaxHd], float* stage, float* __restrict__ ws,
                             int* __restrict__ tickets, float* __restrict__ out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = gridDim.y, split = blockIdx.y;
    int t0, n;
    attn_range(kv_len, S, split, t0, n);
    const float scale = 1.0f / sqrtf((float)hd);
    const bool vec4 =
        (hd & 3) == 0 && ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) == 0;
    float* ks = stage;
    float* vs = stage + kAttnChunk * kAttnMaxHd;
    const bool one_chunk = n <= kAttnChunk;  // the value rows are staged with the key rows
    const int newrow = kv_len - 1;
    // scores: warp w takes rows w, w + 4, ...; lane sums dims lane, lane + 32, ...
    float mx = -INFINITY;
    for (int c0 = 0; c0 < n; c0 += kAttnChunk) {
        const int nc = min(kAttnChunk, n - c0);
        attn_stage(k_cache, kn, ks, v_cache, vn, one_chunk ? vs : nullptr, newrow, kvh, ld, hd, t0 + c0, nc, vec4);
        __syncthreads();
        for (int i = warp; i < nc; i += kAttnThreads / 32) {
            const float* kr = ks + i * hd;
            float dot = 0.f;
            for (int d = lane; d < hd; d += 32) dot = __fadd_rn(dot, __fmul_rn(qs[d], kr[d]));
            dot = warp_sum(dot);
            const float sv = __fmul_rn(dot, scale);
            if (lane == 0) sc[c0 + i] = sv;
            mx = fmaxf(mx, sv);
        }
        __syncthreads();
    }
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = lane < kAttnThreads / 32 ? red[lane] : -INFINITY;
    mx = warp_max(mx);
    __syncthreads();
    float sum = 0.f;
    for (int i = threadIdx.x; i < n; i += kAttnThreads) {
        const float p = expf(sc[i] - mx);
        sc[i] = p;
        sum = __fadd_rn(sum, p);
    }
    sum = block_sum<kAttnThreads>(sum, red);
    // weighted values: warp w takes rows w, w + 4, ...; lanes split the head dims
    float acc[kAttnMaxHd / 32];
#pragma unroll
    for (int j = 0; j < kAttnMaxHd / 32; ++j) acc[j] = 0.f;
    for (int c0 = 0; c0 < n; c0 += kAttnChunk) {
        const int nc = min(kAttnChunk, n - c0);
        if (!one_chunk) {
            attn_stage(v_cache, vn, vs, nullptr, nullptr, nullptr, newrow, kvh, ld, hd, t0 + c0, nc, vec4);
            __syncthreads();
        }
        for (int i = warp; i < nc; i += kAttnThreads / 32) {
            const float p = sc[c0 + i];
            const float* vr = vs + i * hd;
#pragma unroll
            for (int j = 0; j < kAttnMaxHd / 32; ++j) {
                const int d = lane + 32 * j;
                if (d < hd) acc[j] = __fadd_rn(acc[j], __fmul_rn(p, vr[d]));
            }
        }
        if (!one_chunk) __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < kAttnMaxHd / 32; ++j) {
        const int d = lane + 32 * j;
        if (d < hd) part[warp][d] = acc[j];
    }
    __syncthreads();
    // this split's statistics and weighted sum -> workspace, then the head's ticket
    float* wp = ws + ((int64_t)head * S + split) * kAttnPart;
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnThreads / 32; ++w) o = __fadd_rn(o, part[w][d]);
        wp[4 + d] = o;
    }
    if (threadIdx.x == 0) {
        wp[0] = mx;   // -inf for an empty range
        wp[1] = sum;  // 0 for an empty range
    }
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) last = atomicAdd(&tickets[head], 1) == S - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    // the head's last CTA: its S partial results -> shared memory (all loads in
    // flight), then combined in split order
    const int pw = (4 + hd + 3) / 4;  // float4 of a partial result
    const int P = 4 * pw;
    const float4* hp = reinterpret_cast<const float4*>(ws + (int64_t)head * S * kAttnPart);
    float4* st4 = reinterpret_cast<float4*>(stage);
    const int tot = S * pw;
    constexpr int kBatch = 8;
    for (int base = 0; base < tot; base += kBatch * kAttnThreads) {
        float4 r[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int e = base + threadIdx.x + j * kAttnThreads;
            if (e < tot) {
                const int q = e / pw;
                r[j] = __ldcg(hp + q * (kAttnPart / 4) + (e - q * pw));
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int e = base + threadIdx.x + j * kAttnThreads;
            if (e < tot) st4[e] = r[j];
        }
    }
    __shared__ float wq[kAttnMaxSplits];  // exp(m_s - M) of each split with l_s > 0
    __syncthreads();
    if (warp == 0) {
        float M = -INFINITY;
        for (int q = lane; q < S; q += 32)
            if (stage[q * P + 1] > 0.f) M = fmaxf(M, stage[q * P]);
        M = warp_max(M);
        for (int q = lane; q < S; q += 32) wq[q] = stage[q * P + 1] > 0.f ? expf(stage[q * P] - M) : 0.f;
    }
    __syncthreads();
    float L = 0.f;
    for (int q = 0; q < S; ++q) {
        const float l = stage[q * P + 1];
        if (l > 0.f) L = __fadd_rn(L, __fmul_rn(l, wq[q]));
    }
    const float inv = 1.0f / L;
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
        float o = 0.f;
        for (int q = 0; q < S; ++q)
            if (stage[q * P + 1] > 0.f) o = __fadd_rn(o, __fmul_rn(stage[q * P + 4 + d], wq[q]));
        out[head * hd + d] = __fmul_rn(o, inv);
    }
    if (threadIdx.x == 0) tickets[head] = 0;  // ready for the next launch
}

// Attention over the caches (the new row already appended by qkv_rope_kernel).
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const float* __restrict__ q,
                                                                 const float* __restrict__ k_cache,
                                                                 const float* __restrict__ v_cache,
                                                                 const int32_t* __restrict__ pos_ptr, int64_t max_ctx,
                                                                 int nq, int nkv, int hd, float* __restrict__ ws,
                                                                 int* __restrict__ tickets, float* __restrict__ out) {
    extern __shared__ float sc[];  // the CTA's scores, then probabilities
    __shared__ __align__(16) float stage[kAttnStage];
    __shared__ float qs[kAttnMaxHd];
    __shared__ float red[32];
    __shared__ float part[kAttnThreads / 32][kAttnMaxHd];
    const int head = blockIdx.x;
    const int kvh = head / (nq / nkv);
    attn_prefetch(pos_ptr, max_ctx, k_cache, v_cache, kvh, nkv * hd, hd);
    pdl_entry();
    const int kv_len = (int)min((int64_t)max(*pos_ptr + 1, 1), max_ctx);
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) qs[d] = q[head * hd + d];
    __syncthreads();
    attend_split(qs, nullptr, nullptr, k_cache, v_cache, kvh, nkv * hd, hd, kv_len, head, sc, red, part, stage, ws,
                 tickets, out);
}

// Fused form of qkv_rope_kernel + attention_kernel: every CTA of a query head
// adds the biases and rotates its query head and the current token's key (of
// its kv head) itself and attends over its range of cache rows 0 .. pos-1 plus
// that new row (held in shared memory); split 0 of the first query head of each
// kv group appends the new key / value row to the caches (a row no CTA reads
// from the cache in this launch).  Same arithmetic as the two kernels.
__global__ void __launch_bounds__(kAttnThreads) rope_attention_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ bq, const float* __restrict__ bk, const float* __restrict__ bv, float rope_theta,
    const int32_t* __restrict__ pos_ptr, int64_t max_ctx, float* __restrict__ k_cache, float* __restrict__ v_cache,
    int nq, int nkv, int hd, float* __restrict__ ws, int* __restrict__ tickets, float* __restrict__ out) {
    extern __shared__ float sc[];  // the CTA's scores, then probabilities
    __shared__ __align__(16) float stage[kAttnStage];
    __shared__ __align__(16) float kn[kAttnMaxHd];
    __shared__ __align__(16) float vn[kAttnMaxHd];
    __shared__ float qs[kAttnMaxHd];
    __shared__ float red[32];
    __shared__ float part[kAttnThreads / 32][kAttnMaxHd];
    const int head = blockIdx.x;
    const int group = nq / nkv;
    const int kvh = head / group;
    const int ld = nkv * hd;
    attn_prefetch(pos_ptr, max_ctx, k_cache, v_cache, kvh, ld, hd);
    pdl_entry();
    const int pos = *pos_ptr;
    const int kv_len = (int)min((int64_t)max(pos + 1, 1), max_ctx);  // rows 0 .. kv_len-2 cached, kv_len-1 new
    const int half = hd / 2;
    for (int i = threadIdx.x; i < half; i += kAttnThreads) {
        const float theta = 1.0f / powf(rope_theta, (float)(2 * i) / (float)hd);
        const float freq = __fmul_rn((float)pos, theta);
        const float c = cosf(freq), s = sinf(freq);
        const int a = head * hd + i, b = a + half;
        float x1 = bq ? __fadd_rn(q[a], bq[a]) : q[a];
        float x2 = bq ? __fadd_rn(q[b], bq[b]) : q[b];
        qs[i] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        qs[i + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
        const int ka = kvh * hd + i, kb = ka + half;
        x1 = bk ? __fadd_rn(k[ka], bk[ka]) : k[ka];
        x2 = bk ? __fadd_rn(k[kb], bk[kb]) : k[kb];
        kn[i] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        kn[i + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
        vn[i] = bv ? __fadd_rn(v[ka], bv[ka]) : v[ka];
        vn[i + half] = bv ? __fadd_rn(v[kb], bv[kb]) : v[kb];
    }
    __syncthreads();
    if (head % group == 0 && blockIdx.y == 0 && pos >= 0 && pos < max_ctx)
        for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
            k_cache[(int64_t)pos * ld + kvh * hd + d] = kn[d];
            v_cache[(int64_t)pos * ld + kvh * hd + d] = vn[d];
        }
    attend_split(qs, kn, vn, k_cache, v_cache, kvh, ld, hd, kv_len, head, sc, red, part, stage, ws, tickets, out);
}

// out = silu(g) * u, silu(g) = g * (1 / (1 + exp(-g)))
__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, int64_t n,
                                float* __restrict__ out) {
    pdl_entry();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float gi = g[i];
        const float silu = __fmul_rn(gi, 1.0f / __fadd_rn(1.0f, expf(-gi)));
        out[i] = __fmul_rn(silu, u[i]);
    }
}

// Token selection.  greedy != 0: the repetition penalty over every entry of
// generated[0 .. *count) in order (in place on the logits), then the first
// index of the maximum becomes the next token; it is appended to `generated`
// (while *count < max_gen) and written to *token.  In both modes *pos += 1.
constexpr int kSelThreads = 1024;
__global__ void __launch_bounds__(kSelThreads) select_kernel(float* __restrict__ logits, int64_t vocab,
                                                             int32_t* __restrict__ generated,
                                                             int32_t* __restrict__ count, int64_t max_gen,
                                                             float penalty, int greedy, int32_t* __restrict__ token,
                                                             int32_t* __restrict__ pos) {
    __shared__ float bv[kSelThreads / 32];
    __shared__ int64_t bi[kSelThreads / 32];
    pdl_entry();
    if (greedy) {
        if (threadIdx.x == 0) {
            const int n = *count;
            for (int i = 0; i < n; ++i) {
                const int64_t idx = (int64_t)(uint32_t)generated[i];
                if (idx < vocab) {
                    const float l = logits[idx];
                    logits[idx] = l > 0.f ? l / penalty : __fmul_rn(l, penalty);
                }
            }
        }
        __syncthreads();
        // per thread: its first strict maximum (NaN never wins; all -inf -> index 0)
        float best = -INFINITY;
        int64_t besti = 0;
        for (int64_t i = threadIdx.x; i < vocab; i += kSelThreads) {
            const float v = logits[i];
            if (v > best) {
                best = v;
                besti = i;
            }
        }
        // the maximum with the smallest index (the reference's first maximum)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, besti, o);
            if (ov > best || (ov == best && oi < besti)) {
                best = ov;
                besti = oi;
            }
        }
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        if (lane == 0) {
            bv[warp] = best;
            bi[warp] = besti;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float b = bv[0];
            int64_t id = bi[0];
            for (int w = 1; w < kSelThreads / 32; ++w)
                if (bv[w] > b || (bv[w] == b && bi[w] < id)) {
                    b = bv[w];
                    id = bi[w];
                }
            const int n = *count;
            if (n < max_gen) {
                generated[n] = (int32_t)id;
                *count = n + 1;
            }
            *token = (int32_t)id;
        }
    }
    if (threadIdx.x == 0) *pos += 1;
}

}  // namespace

cudaError_t launch_embed(const float* table, int64_t vocab, int64_t hidden, const int32_t* token, float* x,
                         cudaStream_t st) {
    const int threads = 256;
    const int blocks = (int)((hidden + threads - 1) / threads);
    return launch_pdl(embed_kernel, dim3(blocks), dim3(threads), 0, st, table, vocab, hidden, token, x);
}

cudaError_t launch_rmsnorm(float* x, const float* delta, const float* w, int64_t n, float eps, float* out,
                           cudaStream_t st) {
    if (n <= 0 || n > (1 << 24)) return cudaErrorInvalidValue;
    return launch_pdl(rmsnorm_kernel, dim3(1), dim3(kNormThreads), 0, st, x, delta, w, (int)n, eps, out);
}

cudaError_t launch_qkv_rope(float* q, const float* k, const float* v, const float* bq, const float* bk,
                            const float* bv, int nq, int nkv, int hd, float rope_theta, const int32_t* pos,
                            int64_t max_ctx, float* k_cache, float* v_cache, cudaStream_t st) {
    if (nq <= 0 || nkv <= 0 || hd <= 0 || (hd & 1) || nq % nkv || max_ctx <= 0) return cudaErrorInvalidValue;
    const int npairs = (nq + nkv) * (hd / 2);
    const int threads = 256;
    return launch_pdl(qkv_rope_kernel, dim3((npairs + threads - 1) / threads), dim3(threads), 0, st, q, k, v, bq, bk,
                      bv, nq, nkv, hd, rope_theta, pos, max_ctx, k_cache, v_cache);
}

// The attention kernels hold about 38 KB of static shared memory; dynamic
// shared memory (the scores of a split) beyond what is left of the default 48 KB
// is opted into per launch.
constexpr size_t kAttnDefaultDynSmem = 8 * 1024;
constexpr size_t kAttnMaxDynSmem = 160 * 1024;
// The split workspace holds nq x S partial results in 16-byte aligned rows.
inline bool attn_ws_ok(const float* ws, int64_t ws_floats, const int* tickets, int64_t n_tickets, int nq, int S) {
    return ws && tickets && (reinterpret_cast<uintptr_t>(ws) & 15) == 0 && (int64_t)nq * S * kAttnPart <= ws_floats &&
           nq <= n_tickets;
}

cudaError_t launch_attention(const float* q, const float* k_cache, const float* v_cache, const int32_t* pos, int nq,
                             int nkv, int hd, int64_t max_ctx, float* ws, int64_t ws_floats, int* tickets,
                             int64_t n_tickets, float* out, cudaStream_t st) {
    if (nq <= 0 || nkv <= 0 || nq % nkv || hd <= 0 || hd > kAttnMaxHd || max_ctx <= 0) return cudaErrorInvalidValue;
    const int S = attn_splits(max_ctx);
    if (!attn_ws_ok(ws, ws_floats, tickets, n_tickets, nq, S)) return cudaErrorInvalidValue;
    const size_t smem = (size_t)((max_ctx + S - 1) / S) * sizeof(float);
    if (smem > kAttnMaxDynSmem) return cudaErrorInvalidValue;
    if (smem > kAttnDefaultDynSmem) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(attention_kernel, dim3(nq, S), dim3(kAttnThreads), smem, st, q, k_cache, v_cache, pos,
                      max_ctx, nq, nkv, hd, ws, tickets, out);
}

cudaError_t launch_rope_attention(const float* q, const float* k, const float* v, const float* bq, const float* bk,
                                  const float* bv, float rope_theta, const int32_t* pos, int64_t max_ctx,
                                  float* k_cache, float* v_cache, int nq, int nkv, int hd, float* ws, int64_t ws_floats,
                                  int* tickets, int64_t n_tickets, float* out, cudaStream_t st) {
    if (nq <= 0 || nkv <= 0 || nq % nkv || hd <= 0 || (hd & 1) || hd > kAttnMaxHd || max_ctx <= 0)
        return cudaErrorInvalidValue;
    const int S = attn_splits(max_ctx);
    if (!attn_ws_ok(ws, ws_floats, tickets, n_tickets, nq, S)) return cudaErrorInvalidValue;
    const size_t smem = (size_t)((max_ctx + S - 1) / S) * sizeof(float);
    if (smem > kAttnMaxDynSmem) return cudaErrorInvalidValue;
    if (smem > kAttnDefaultDynSmem) {
        cudaError_t e =
            cudaFuncSetAttribute(rope_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(rope_attention_kernel, dim3(nq, S), dim3(kAttnThreads), smem, st, q, k, v, bq, bk, bv,
                      rope_theta, pos, max_ctx, k_cache, v_cache, nq, nkv, hd, ws, tickets, out);
}

cudaError_t launch_silu_mul(const float* g, const float* u, int64_t n, float* out, cudaStream_t st) {
    const int threads = 256;
    const int blocks = (int)((n + threads - 1) / threads < 4096 ? (n + threads - 1) / threads : 4096);
    if (n <= 0) return cudaSuccess;
    return launch_pdl(silu_mul_kernel, dim3(blocks), dim3(threads), 0, st, g, u, n, out);
}

cudaError_t launch_select(float* logits, int64_t vocab, int32_t* generated, int32_t* count, int64_t max_gen,
                          float penalty, int greedy, int32_t* token, int32_t* pos, cudaStream_t st) {
    if (vocab <= 0) return cudaErrorInvalidValue;
    return launch_pdl(select_kernel, dim3(1), dim3(kSelThreads), 0, st, logits, vocab, generated, count, max_gen,
                      penalty, greedy, token, pos);
}

}  // namespace bramha
