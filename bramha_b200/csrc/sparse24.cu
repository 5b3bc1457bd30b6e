// sparse24.cu -- 2:4 structured-sparse GEMV on the CUDA cores, and the
// registration-time pruning that produces its device layout.
//
// The reference has two 2:4 paths (spanda-engine/src/sparse.rs:19-138,
// src/inference/cpu_engine.rs:1532-1640):
//  * on-the-fly: every call sorts each group of 4 weights of a row by
//    magnitude (Rust's stable sort_by, descending) and sums the top two
//    products -- over f32, int8 and int4 weights;
//  * compressed: u16 masks (low 4 bits, one per group) plus the kept values
//    in index order (the .spanda BlockSparse2_4 tensor, bin/convert.rs:55-92).
// The selection depends on the weights only, so here it is made once, when
// the weight is registered (sp24_prune_kernel; the compressed form is
// canonicalised on the host), into one device layout for both paths:
//
//   vals [N][Cp] : the two kept codes of each group, in the weight's own code
//                  type -- f32 pair (8 B), int8 pair stored offset-binary
//                  (q + 128, 2 B), or int4 pair (slot 0 low nibble, slot 1
//                  high nibble, raw q, 1 B);
//   idx  [N][Cp/8] u32 : 4 bits per group (group j of the word at bits
//                  4j..4j+3): the id p of its column pair (a < b), p = 0..5
//                  for (0,1) (0,2) (0,3) (1,2) (1,3) (2,3); slot 0 holds the
//                  code of column a, slot 1 that of column b;
//   tail [N][4] f32 : codes of the K % 4 columns after the last full group
//                  (on-the-fly path only: the reference adds them densely);
//   scales [N].
// Cp = groups per row rounded up to 8 (padding groups hold zero codes).
// Bytes per group of 4 weights: 8.5 (f32), 2.5 (int8), 1.5 (int4).
//
// GEMV: y[r] = s[r] * (sum over groups of v0 * x[4g + a] + v1 * x[4g + b]
// + tail).  A block (16 warps) owns 64 rows and one K-slice.  It stages the
// slice of x in shared memory as all six column pairs of every group,
// (x[4g+a], x[4g+b]) as one float2, so a group's two activations are ONE
// 64-bit shared load picked by its pair id.  Lane l streams groups 8l..8l+7
// of each 256-group segment (one vector load of codes and one u32 of pair
// ids); the pair p of (segment t, group 8l+j) sits at float2 index
// ((t*8 + j)*6 + p)*32 + l, so the 16 lanes of each half-warp always hit 16
// distinct bank pairs.  Decoding and the two products of a group use
// Blackwell's packed f32x2 add and fma (two fp32 accumulators per row).
// K-slices are summed by the last block of each row tile (an atomic ticket,
// no waiting), in slice order, so results are deterministic.
#include "common.cuh"

namespace bramha {
namespace {

constexpr int kSpThreads = 512;
constexpr int kSpWarps = kSpThreads / 32;
constexpr int kSpTileRows = 64;
constexpr int kSpSegChunks = 256;               // groups covered by one warp pass
constexpr int kSpSegBytes = kSpSegChunks * 48;  // six float2 pairs per group
constexpr int kSpMaxSegs = 8;                   // x slice <= 8 segments = 96 KB of shared memory
constexpr int kSpMaxSplit = 16;

template <int FMT>
struct SpFmt;
template <>
struct SpFmt<BRAMHA_FMT_F32> {
    static constexpr int kVB = 8;  // bytes per group
    static constexpr int kU = 2;   // rows a warp streams at once
};
template <>
struct SpFmt<BRAMHA_FMT_W8> {
    static constexpr int kVB = 2;
    static constexpr int kU = 4;
};
template <>
struct SpFmt<BRAMHA_FMT_W4ZP8> {
    static constexpr int kVB = 1;
    static constexpr int kU = 4;
};

struct SpArgs {
    const uint8_t* vals;
    int64_t ldv;  // bytes per row
    const uint32_t* idx;
    int64_t ldi;  // words per row
    const float* tail;
    const float* scales;
    const float* x;
    float* y;
    float* ws;
    int* tickets;
    int N, K, C, Cp;  // C = real groups (K / 4), Cp = padded groups
    int tail_cols;    // K % 4 (tail != nullptr)
    int slice;        // groups per K-slice (multiple of 8)
    int ks;           // K-slices
    int row_tiles;
};

__device__ __forceinline__ uint4 ld_stream4(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ld_stream2(const void* p) {
    uint2 r;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ld_stream1(const void* p) {
    uint32_t r;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

// Codes of one group of 8 chunks, as 32-bit words, and their pair ids.
template <int FMT>
struct Group {
    static constexpr int kWords = SpFmt<FMT>::kVB * 8 / 4;
    uint32_t w[kWords];
    uint32_t idx;
};

template <int FMT>
__device__ __forceinline__ void load_at(const uint8_t* vp, const uint32_t* ip, Group<FMT>& G) {
    if constexpr (Group<FMT>::kWords >= 4) {
#pragma unroll
        for (int v = 0; v < Group<FMT>::kWords / 4; ++v) {
            const uint4 q = ld_stream4(vp + 16 * v);
            G.w[4 * v] = q.x;
            G.w[4 * v + 1] = q.y;
            G.w[4 * v + 2] = q.z;
            G.w[4 * v + 3] = q.w;
        }
    } else {
        const uint2 q = ld_stream2(vp);
        G.w[0] = q.x;
        G.w[1] = q.y;
    }
    G.idx = ld_stream1(ip);
}

// Byte offset of pair p's float2 row within a (segment, group) block: p * 256.
__device__ __forceinline__ uint32_t pair_off(uint32_t idx, int j) {
    const int s = 4 * j;  // field at bits s..s+2; wanted at bits 8..10
    return s >= 8 ? (idx >> (s - 8)) & 0x700u : (idx << (8 - s)) & 0x700u;
}

// Two fp32 lanes in one 64-bit register (packed f32x2 arithmetic, sm_100).
__device__ __forceinline__ uint64_t pack2(uint32_t lo, uint32_t hi) { return (uint64_t)lo | ((uint64_t)hi << 32); }
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Byte b of `word` under the exponent of 2^23: the float 2^23 + byte, exactly.
__device__ __forceinline__ uint32_t magic_byte(uint32_t word, int b) {
    return __byte_perm(word, 0x4B000000u, 0x7540u | (uint32_t)b);
}

// Adds the 16 kept products of one group of 8 chunks to acc (slot-0 products
// in the low lane, slot-1 products in the high lane).  lt: byte offset of
// (segment, chunk 0, pair 0, this lane) in the staged pairs; its bits 8..10
// are zero, so the pair offset is OR-ed in and j*1536 is a constant offset.
template <int FMT>
__device__ __forceinline__ uint64_t group_dot(const Group<FMT>& G, const char* xb, uint32_t lt, uint64_t acc) {
    uint32_t lo4 = 0, hi4 = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint64_t xp = *reinterpret_cast<const uint64_t*>(xb + (uint32_t)j * 1536u + (lt | pair_off(G.idx, j)));
        uint64_t v;
        if constexpr (FMT == BRAMHA_FMT_F32) {
            v = pack2(G.w[2 * j], G.w[2 * j + 1]);
        } else if constexpr (FMT == BRAMHA_FMT_W8) {  // (2^23 + q + 128) - (2^23 + 128)
            const uint32_t wd = G.w[j >> 1];
            v = add2(pack2(magic_byte(wd, 2 * (j & 1)), magic_byte(wd, 2 * (j & 1) + 1)),
                     pack2(0xCB000080u, 0xCB000080u));
        } else {  // int4 pair, slot 0 low nibble, slot 1 high nibble: (2^23 + q) - (2^23 + 8)
            if ((j & 3) == 0) {
                lo4 = G.w[j >> 2] & 0x0F0F0F0Fu;
                hi4 = (G.w[j >> 2] >> 4) & 0x0F0F0F0Fu;
            }
            v = add2(pack2(magic_byte(lo4, j & 3), magic_byte(hi4, j & 3)), pack2(0xCB000008u, 0xCB000008u));
        }
        acc = fma2(v, xp, acc);
    }
    return acc;
}

template <int FMT>
__global__ void __launch_bounds__(kSpThreads, 2) sp24_gemv_kernel(SpArgs a) {
    extern __shared__ float xs[];
    constexpr int U = SpFmt<FMT>::kU;
    constexpr int GB = SpFmt<FMT>::kVB * 8;  // code bytes of a group of 8 chunks
    const int tile = blockIdx.x % a.row_tiles;
    const int ksl = blockIdx.x / a.row_tiles;
    const int g0 = ksl * a.slice;           // first group of the slice
    const int S = min(a.slice, a.Cp - g0);  // groups in the slice (multiple of 8)
    const int segs = (S + kSpSegChunks - 1) / kSpSegChunks;
    const int full_segs = S / kSpSegChunks;

    // Stage the six column pairs of every group of the slice; columns of
    // padding groups (and of the tail, which has its own term) are zero.
    float2* xp = reinterpret_cast<float2*>(xs);
    for (int e = threadIdx.x; e < segs * kSpSegChunks; e += kSpThreads) {
        const int t = e >> 8, j = (e >> 5) & 7, l = e & 31;
        const int c = g0 + (t << 8) + (l << 3) + j;  // group index in the row
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (c < a.C) {
            const float4 q = __ldg(reinterpret_cast<const float4*>(a.x) + c);
            v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
        }
        float2* d = xp + (t * 8 + j) * 192 + l;
#pragma unroll
        for (int p = 0; p < 6; ++p) d[p * 32] = make_float2(v[sp24_pair_a(p)], v[sp24_pair_b(p)]);
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const char* xb = reinterpret_cast<const char*>(xs);
    const bool last_slice = ksl == a.ks - 1;
    const int row_end = min(a.N, (tile + 1) * kSpTileRows);
    for (int r0 = tile * kSpTileRows + warp * U; r0 < row_end; r0 += kSpWarps * U) {
        // rows past N repeat row N-1 (in bounds) and are not written
        const uint8_t* vp[U];
        const uint32_t* ip[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int row = min(r0 + u, a.N - 1);
            vp[u] = a.vals + (int64_t)row * a.ldv + (int64_t)(g0 / 8 + lane) * GB;
            ip[u] = a.idx + (int64_t)row * a.ldi + g0 / 8 + lane;
        }
        uint64_t acc[U];
#pragma unroll
        for (int u = 0; u < U; ++u) acc[u] = 0;
        int t = 0;
#pragma unroll 2
        for (; t < full_segs; ++t) {
            Group<FMT> G[U];
#pragma unroll
            for (int u = 0; u < U; ++u) load_at<FMT>(vp[u] + t * 32 * GB, ip[u] + t * 32, G[u]);
#pragma unroll
            for (int u = 0; u < U; ++u)
                acc[u] = group_dot<FMT>(G[u], xb, (uint32_t)t * (uint32_t)kSpSegBytes + (uint32_t)lane * 8u, acc[u]);
        }
        if (t < segs && 8 * (t * 32 + lane) < S) {  // the partial last segment
            Group<FMT> G[U];
#pragma unroll
            for (int u = 0; u < U; ++u) load_at<FMT>(vp[u] + t * 32 * GB, ip[u] + t * 32, G[u]);
#pragma unroll
            for (int u = 0; u < U; ++u)
                acc[u] = group_dot<FMT>(G[u], xb, (uint32_t)t * (uint32_t)kSpSegBytes + (uint32_t)lane * 8u, acc[u]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float s = __uint_as_float((uint32_t)acc[u]) + __uint_as_float((uint32_t)(acc[u] >> 32));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            const int row = r0 + u;
            if (lane == 0 && row < a.N) {
                if (last_slice && a.tail) {
                    const int c0 = 4 * a.C;
                    for (int i = 0; i < a.tail_cols; ++i) s = fmaf(a.tail[(int64_t)row * 4 + i], a.x[c0 + i], s);
                }
                if (a.ks == 1)
                    a.y[row] = s * a.scales[row];
                else
                    a.ws[(int64_t)ksl * a.N + row] = s;
            }
        }
    }
    if (a.ks == 1) return;

    // Last block of this row tile sums the slices in order.
    __shared__ int s_last;
    __threadfence();  // this thread's partials, before the ticket
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(a.tickets + tile, 1);
        s_last = prev == a.ks - 1;
        if (s_last) a.tickets[tile] = 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int row = tile * kSpTileRows + threadIdx.x; row < row_end; row += kSpThreads) {
        float s = 0.f;
        for (int k = 0; k < a.ks; ++k) s += __ldcg(a.ws + (int64_t)k * a.N + row);
        a.y[row] = s * a.scales[row];
    }
}

// ---------------------------------------------------------------- pruning

// Top two of four magnitudes the way the reference picks them: Rust's stable
// slice::sort_by with `b.partial_cmp(a).unwrap_or(Equal)` runs insertion sort
// on four elements; an element moves left only past strictly smaller
// magnitudes, so ties keep the lower column first (and a NaN moves nowhere).
__device__ __forceinline__ void top2_of4(const float m[4], int& i1, int& i2) {
    int o[4] = {0, 1, 2, 3};
#pragma unroll
    for (int i = 1; i < 4; ++i) {
        const int t = o[i];
        int j = i;
        while (j > 0 && m[t] > m[o[j - 1]]) {
            o[j] = o[j - 1];
            --j;
        }
        o[j] = t;
    }
    i1 = o[0];
    i2 = o[1];
}

// Code value (unscaled) of column c of a reference-layout row.
template <int FMT>
__device__ __forceinline__ float code_at(const uint8_t* row, int64_t c) {
    if constexpr (FMT == BRAMHA_FMT_F32) {
        float v;
        memcpy(&v, row + 4 * c, 4);
        return v;
    } else if constexpr (FMT == BRAMHA_FMT_W8) {
        return (float)(int8_t)row[c];
    } else {  // even column in the high nibble (quantize_to_int4)
        const uint8_t b = row[c >> 1];
        return (float)((c & 1) ? (b & 0xF) : (b >> 4)) - 8.0f;
    }
}

// One thread per (row, group of 8) -- one per row when K < 4 -- selects the
// kept pair of each group and writes codes, indices and (group 0's thread)
// the tail.
template <int FMT>
__global__ void sp24_prune_kernel(const uint8_t* src, int64_t row_bytes, int64_t N, int64_t K, int64_t C,
                                  int64_t Cp, uint8_t* vals, int64_t ldv, uint32_t* idx, int64_t ldi, float* tail) {
    const int64_t gpr = Cp > 0 ? Cp / 8 : 1;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= N * gpr) return;
    const int64_t row = tid / gpr, g = tid % gpr;
    const uint8_t* r = src + row * row_bytes;
    if (tail && g == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) tail[row * 4 + i] = 4 * C + i < K ? code_at<FMT>(r, 4 * C + i) : 0.f;
    }
    if (Cp == 0) return;
    uint32_t iw = 0;
    uint32_t w[SpFmt<FMT>::kVB * 2];
#pragma unroll
    for (int k = 0; k < SpFmt<FMT>::kVB * 2; ++k) w[k] = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int64_t c = g * 8 + j;
        int i1 = 0, i2 = 1;
        float v1 = 0.f, v2 = 0.f;
        if (c < C) {
            float v[4], m[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[i] = code_at<FMT>(r, 4 * c + i);
                m[i] = fabsf(v[i]);
            }
            top2_of4(m, i1, i2);
            if (i1 > i2) {  // slots in column order
                const int t = i1;
                i1 = i2;
                i2 = t;
            }
            v1 = v[i1];
            v2 = v[i2];
        }
        iw |= (uint32_t)sp24_pair_id(i1, i2) << (4 * j);
        if constexpr (FMT == BRAMHA_FMT_F32) {
            w[2 * j] = __float_as_uint(v1);
            w[2 * j + 1] = __float_as_uint(v2);
        } else if constexpr (FMT == BRAMHA_FMT_W8) {
            const uint32_t b = ((uint32_t)((int)v1 + 128)) | ((uint32_t)((int)v2 + 128) << 8);
            w[j >> 1] |= b << (16 * (j & 1));
        } else {
            const uint32_t b = ((uint32_t)((int)v1 + 8)) | ((uint32_t)((int)v2 + 8) << 4);
            w[j >> 2] |= b << (8 * (j & 3));
        }
    }
    idx[row * ldi + g] = iw;
    uint32_t* dst = reinterpret_cast<uint32_t*>(vals + row * ldv + g * (SpFmt<FMT>::kVB * 8));
#pragma unroll
    for (int k = 0; k < SpFmt<FMT>::kVB * 2; ++k) dst[k] = w[k];
}

template <int FMT>
cudaError_t set_smem_attr() {
    static int done[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && done[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(sp24_gemv_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSpMaxSegs * kSpSegBytes + 512);
    if (e == cudaSuccess && dev < 64) done[dev] = 1;
    return e;
}

template <int FMT>
cudaError_t launch_gemv_t(const Sp24Weight& w, const float* x, float* y, float* ws, int64_t ws_floats, int* tickets,
                          int n_tickets, int num_sms, cudaStream_t st) {
    cudaError_t e = set_smem_attr<FMT>();
    if (e != cudaSuccess) return e;
    SpArgs a{};
    a.vals = w.vals;
    a.ldv = w.ldv;
    a.idx = w.idx;
    a.ldi = w.ldi;
    a.tail = w.tail;
    a.scales = w.scales;
    a.x = x;
    a.y = y;
    a.ws = ws;
    a.tickets = tickets;
    a.N = (int)w.N;
    a.K = (int)w.K;
    a.C = (int)(w.K / 4);
    a.Cp = (int)w.Cp;
    a.tail_cols = (int)(w.K % 4);
    a.row_tiles = (int)((w.N + kSpTileRows - 1) / kSpTileRows);
    const int groups = a.Cp / 8;
    // K-split: enough blocks for two per SM, slices of at least one warp pass,
    // at most kSpMaxSegs segments of x per block.
    int ks = (2 * num_sms + a.row_tiles - 1) / a.row_tiles;
    ks = min(ks, max(1, groups / 32));
    ks = max(ks, (a.Cp + kSpMaxSegs * kSpSegChunks - 1) / (kSpMaxSegs * kSpSegChunks));
    ks = min(ks, kSpMaxSplit);
    if (ks > 1 && ((int64_t)ks * a.N > ws_floats || a.row_tiles > n_tickets)) ks = 1;
    if (a.Cp == 0) {  // fewer than 4 columns: the tail is the whole row
        a.slice = 8;
        a.ks = 1;
    } else {
        const int slice_groups8 = (groups + ks - 1) / ks;  // groups of 8 chunks per slice
        a.slice = slice_groups8 * 8;
        a.ks = (a.Cp + a.slice - 1) / a.slice;
    }
    if (a.slice > kSpMaxSegs * kSpSegChunks) return cudaErrorInvalidValue;  // N too large for the workspace
    const int segs = a.Cp == 0 ? 0 : (a.slice + kSpSegChunks - 1) / kSpSegChunks;
    // + 512 B: even a pair id of 6 or 7 (never written) stays inside the allocation
    const size_t smem = segs ? (size_t)segs * kSpSegBytes + 512 : 0;
    sp24_gemv_kernel<FMT><<<a.row_tiles * a.ks, kSpThreads, smem, st>>>(a);
    return cudaGetLastError();
}

template <int FMT>
cudaError_t launch_prune_t(const uint8_t* src, int64_t row_bytes, const Sp24Weight& w, cudaStream_t st) {
    const int64_t threads = w.N * (w.Cp > 0 ? w.Cp / 8 : 1);
    if (threads == 0) return cudaSuccess;
    const int bs = 256;
    sp24_prune_kernel<FMT><<<(unsigned)((threads + bs - 1) / bs), bs, 0, st>>>(
        src, row_bytes, w.N, w.K, w.K / 4, w.Cp, w.vals, w.ldv, w.idx, w.ldi, w.tail);
    return cudaGetLastError();
}

}  // namespace

int sp24_value_bytes(int base_fmt) {
    switch (base_fmt) {
        case BRAMHA_FMT_F32: return SpFmt<BRAMHA_FMT_F32>::kVB;
        case BRAMHA_FMT_W8: return SpFmt<BRAMHA_FMT_W8>::kVB;
        case BRAMHA_FMT_W4ZP8: return SpFmt<BRAMHA_FMT_W4ZP8>::kVB;
        default: return 0;
    }
}

cudaError_t launch_sp24_gemv(int base_fmt, const Sp24Weight& w, const float* x, float* y, float* ws,
                             int64_t ws_floats, int* tickets, int n_tickets, int num_sms, cudaStream_t st) {
    if (w.N == 0) return cudaSuccess;
    switch (base_fmt) {
        case BRAMHA_FMT_F32:
            return launch_gemv_t<BRAMHA_FMT_F32>(w, x, y, ws, ws_floats, tickets, n_tickets, num_sms, st);
        case BRAMHA_FMT_W8:
            return launch_gemv_t<BRAMHA_FMT_W8>(w, x, y, ws, ws_floats, tickets, n_tickets, num_sms, st);
        case BRAMHA_FMT_W4ZP8:
            return launch_gemv_t<BRAMHA_FMT_W4ZP8>(w, x, y, ws, ws_floats, tickets, n_tickets, num_sms, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_sp24_prune(int base_fmt, const uint8_t* src, int64_t row_bytes, const Sp24Weight& w,
                              cudaStream_t st) {
    switch (base_fmt) {
        case BRAMHA_FMT_F32: return launch_prune_t<BRAMHA_FMT_F32>(src, row_bytes, w, st);
        case BRAMHA_FMT_W8: return launch_prune_t<BRAMHA_FMT_W8>(src, row_bytes, w, st);
        case BRAMHA_FMT_W4ZP8: return launch_prune_t<BRAMHA_FMT_W4ZP8>(src, row_bytes, w, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace bramha
