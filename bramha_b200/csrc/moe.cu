// moe.cu -- the MoE expert MLP of a batch of decode tokens on one GPU.
//
// The reference runs, per token, the MoE branch of run_mlp_into
// (src/inference/cpu_engine.rs:1799-1989): softmax of the router logits, a
// stable descending sort, the first top_k experts (no renormalisation,
// weights <= 0 skipped), per expert gate/up GEMVs, silu(g) * up, the down
// GEMV, and out += down * weight in the sorted order.  Here the tokens of a
// batch are grouped by expert so each expert's weights are streamed once for
// all the tokens routed to it:
//
//   moe_route_kernel   one warp per token: probabilities, top-k, per-expert
//                      row counts;
//   moe_place_kernel   one CTA per expert: its row offset, its rows in token
//                      order, and its tiles of the two grouped GEMMs;
//   moe_gather_kernel  activations of the routed (token, expert) pairs, in
//                      expert order;
//   grouped GEMM       gate and up of every expert in one launch (weights
//                      stacked [E][2I][H]), tcgen05 (gemm_tcgen05.cu);
//   moe_silu_kernel    silu(g) * up;
//   grouped GEMM       down of every expert in one launch ([E][H][I]);
//   moe_combine_kernel out[t] = sum over the token's kept experts, in the
//                      sorted order, of down * weight.
// Scratch (routing state and the intermediate activations) comes from the
// stream-ordered pool and is released at the end of the call.
#include <cuda_runtime.h>

#include "common.cuh"

namespace bramha {
namespace {

struct Route {
    float* probs;   // [T][E]
    int* sel_e;     // [T][k] r-th expert of the sorted order
    float* sel_w;   // [T][k] its probability
    int* slot;      // [T][k] row of the grouped activations, -1 when skipped (weight <= 0)
    int* tok;       // [T*k] token of each grouped row
    int* cnt;       // [E]
    int* off;       // [E + 1] first grouped row of each expert; off[E] = rows in use
    int4* tiles_gu; // tile table of the gate+up GEMM
    int4* tiles_dn; // tile table of the down GEMM
    int* ntiles;    // [2] entries of the two tables
};

// One warp per token: softmax of the router logits (max by a shuffle fold --
// exact in any order -- and the sum of the exponentials added sequentially by
// lane 0, as the reference does), then the first k of the stable descending
// order, one warp argmax per rank (largest probability after the previous pick;
// equal probabilities keep the lower expert first).  Counts the rows of each
// expert (atomic increments: the totals do not depend on their order).
__global__ void moe_route_kernel(const float* __restrict__ logits, int T, int E, int k, Route r,
                                 int32_t* selected) {
    extern __shared__ float sp[];  // [warps][E] probabilities
    const int wpb = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * wpb + w;
    if (t >= T) return;
    float* p = sp + w * E;
    const float* lg = logits + (int64_t)t * E;
    float mx = -INFINITY;
    for (int i = lane; i < E; i += 32) mx = fmaxf(mx, lg[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int i = lane; i < E; i += 32) p[i] = expf(lg[i] - mx);
    __syncwarp();
    float sum = 0.f;
    if (lane == 0)
        for (int i = 0; i < E; ++i) sum = __fadd_rn(sum, p[i]);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int i = lane; i < E; i += 32) p[i] = sum > 0.f ? __fdiv_rn(p[i], sum) : 0.f;
    __syncwarp();
    float pp = INFINITY;
    int pi = -1;
    for (int j = 0; j < k; ++j) {
        float bp = -INFINITY;
        int best = 0x7fffffff;
        for (int i = lane; i < E; i += 32) {
            const float v = p[i];
            if ((v < pp || (v == pp && i > pi)) && (v > bp || (v == bp && i < best))) {
                bp = v;
                best = i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bp, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best, o);
            if (ov > bp || (ov == bp && oi < best)) {
                bp = ov;
                best = oi;
            }
        }
        pp = bp;
        pi = best;
        if (lane == 0) {
            r.sel_e[t * k + j] = bp > 0.f ? best : -1;
            r.sel_w[t * k + j] = bp;
            r.slot[t * k + j] = -1;
            if (selected) selected[t * k + j] = best;
            if (bp > 0.f) atomicAdd(r.cnt + best, 1);
        }
    }
}

// Routing given by the caller: row t goes to expert ids[t] (weight 1; an id
// outside [0, E) drops the row, whose output is then 0).
__global__ void moe_given_route_kernel(const int32_t* __restrict__ ids, int T, int E, Route r) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const int e = ids[t];
    const bool ok = e >= 0 && e < E;
    r.sel_e[t] = ok ? e : -1;
    r.sel_w[t] = ok ? 1.f : 0.f;
    r.slot[t] = -1;
    if (ok) atomicAdd(r.cnt + e, 1);
}

// One block per expert: its first row (the counts of the experts before it),
// its rows in token order (a block-wide ordered scan over the choices), and
// its tiles of the two grouped GEMMs.  Block 0 also writes the totals.
__global__ void moe_place_kernel(int T, int E, int k, int nblk_gu, int nblk_dn, Route r) {
    __shared__ int warp_sum[32];
    __shared__ int s_base;
    const int e = blockIdx.x, nk = T * k;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int o = 0, tiles_before = 0;
    for (int i = 0; i < e; ++i) {  // uniform over the block: counts are final
        const int c = __ldg(r.cnt + i);
        o += c;
        tiles_before += (c + kGemmGroupTok - 1) / kGemmGroupTok;
    }
    const int c = __ldg(r.cnt + e);
    if (threadIdx.x == 0) {
        r.off[e] = o;
        s_base = o;
        if (e == 0) {
            int tot = 0, mt = 0;
            for (int i = 0; i < E; ++i) {
                const int ci = __ldg(r.cnt + i);
                tot += ci;
                mt += (ci + kGemmGroupTok - 1) / kGemmGroupTok;
            }
            r.off[E] = tot;
            r.ntiles[0] = mt * nblk_gu;
            r.ntiles[1] = mt * nblk_dn;
        }
    }
    __syncthreads();
    // ordered placement, one chunk of blockDim.x choices at a time
    for (int i0 = 0; i0 < nk; i0 += blockDim.x) {
        const int i = i0 + threadIdx.x;
        const bool mine = i < nk && __ldg(r.sel_e + i) == e;
        const unsigned bal = __ballot_sync(0xffffffffu, mine);
        if (lane == 0) warp_sum[w] = __popc(bal);
        __syncthreads();
        int before = 0, total = 0;
        for (int q = 0; q < nw; ++q) {
            before += q < w ? warp_sum[q] : 0;
            total += warp_sum[q];
        }
        if (mine) {
            const int s = s_base + before + __popc(bal & ((1u << lane) - 1u));
            r.slot[i] = s;
            r.tok[s] = i / k;
        }
        __syncthreads();
        if (threadIdx.x == 0) s_base += total;
        __syncthreads();
    }
    const int mt = (c + kGemmGroupTok - 1) / kGemmGroupTok;
    for (int q = threadIdx.x; q < mt * (nblk_gu + nblk_dn); q += blockDim.x) {
        const int m = q / (nblk_gu + nblk_dn), nb = q % (nblk_gu + nblk_dn);
        const int tok0 = o + m * kGemmGroupTok, mc = min(kGemmGroupTok, c - m * kGemmGroupTok);
        if (nb < nblk_gu)
            r.tiles_gu[tiles_before * nblk_gu + m * nblk_gu + nb] = make_int4(e * nblk_gu + nb, tok0, mc, nb * 128);
        else
            r.tiles_dn[tiles_before * nblk_dn + m * nblk_dn + (nb - nblk_gu)] =
                make_int4(e * nblk_dn + nb - nblk_gu, tok0, mc, (nb - nblk_gu) * 128);
    }
}

// xg[s] = x[tok[s]] for the rows in use, zero for the rest.
__global__ void moe_gather_kernel(const float* __restrict__ x, int64_t H, const int* __restrict__ tok,
                                  const int* __restrict__ off_end, int64_t rows, float* __restrict__ xg) {
    const int64_t s = blockIdx.y;
    const int used = __ldg(off_end);
    for (int64_t d = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; d < H; d += (int64_t)gridDim.x * blockDim.x)
        xg[s * H + d] = s < used ? __ldg(x + (int64_t)__ldg(tok + s) * H + d) : 0.f;
}

// act[s][i] = silu(g) * up with silu(g) = g / (1 + exp(-g)) (cpu_engine.rs:1931-1935),
// g = y[s][i], up = y[s][I + i].
__global__ void moe_silu_kernel(const float* __restrict__ y, int64_t I, int64_t rows, float* __restrict__ act) {
    const int64_t n = rows * I;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t s = i / I, c = i % I;
        const float g = y[s * 2 * I + c], u = y[s * 2 * I + I + c];
        const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        act[i] = __fmul_rn(silu, u);
    }
}

// out[t][d] = sum over r < k (kept choices, sorted order) of down[slot][d] * w,
// starting from 0, one rounding per product and per sum (cpu_engine.rs:1944-1946).
__global__ void moe_combine_kernel(const float* __restrict__ down, int64_t H, int k, const int* __restrict__ slot,
                                   const float* __restrict__ w, float* __restrict__ out) {
    const int64_t t = blockIdx.y;
    for (int64_t d = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; d < H; d += (int64_t)gridDim.x * blockDim.x) {
        float acc = 0.f;
        for (int j = 0; j < k; ++j) {
            const int s = __ldg(slot + t * k + j);
            if (s >= 0) acc = __fadd_rn(acc, __fmul_rn(__ldg(down + (int64_t)s * H + d), __ldg(w + t * k + j)));
        }
        out[t * H + d] = acc;
    }
}

template <class T>
T* carve(uint8_t*& p, int64_t n) {
    T* r = reinterpret_cast<T*>(p);
    p += (n * (int64_t)sizeof(T) + 255) / 256 * 256;
    return r;
}

cudaError_t launch_moe(const MoeWeights& w, int top_k, const float* x, const float* logits, const int32_t* given,
                       int64_t T, float* out, int32_t* selected, int* err, cudaStream_t st);

}  // namespace

cudaError_t launch_moe_mlp(const MoeWeights& w, int top_k, const float* x, const float* logits, int64_t T, float* out,
                           int32_t* selected, int* err, cudaStream_t st) {
    return launch_moe(w, top_k, x, logits, nullptr, T, out, selected, err, st);
}

cudaError_t launch_moe_experts(const MoeWeights& w, const float* x, const int32_t* ids, int64_t R, float* y, int* err,
                               cudaStream_t st) {
    return launch_moe(w, 1, x, nullptr, ids, R, y, nullptr, err, st);
}

cudaError_t launch_moe_route(const float* logits, int64_t T, int64_t E, int top_k, int32_t* ids, float* weights,
                             cudaStream_t st) {
    const int k = (int)(top_k < E ? top_k : E);
    if (T <= 0) return cudaSuccess;
    if (E <= 0 || E > kMoeMaxExperts || k <= 0) return cudaErrorInvalidValue;
    uint8_t* base = nullptr;
    auto pad = [](int64_t b) { return (b + 255) / 256 * 256; };  // each carved piece is padded
    const int64_t bytes = 2 * pad(T * k * 4) + pad(E * 4);
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&base), (size_t)bytes, st);
    if (e != cudaSuccess) return e;
    uint8_t* p = base;
    Route r{};
    r.sel_e = carve<int>(p, T * k);
    r.slot = carve<int>(p, T * k);
    r.cnt = carve<int>(p, E);
    r.sel_w = weights;
    const int wpb = 8;
    const size_t smem = (size_t)wpb * E * sizeof(float);
    e = cudaMemsetAsync(r.cnt, 0, (size_t)E * sizeof(int), st);
    if (e == cudaSuccess && smem > 48 * 1024)
        e = cudaFuncSetAttribute(moe_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) {
        moe_route_kernel<<<(unsigned)((T + wpb - 1) / wpb), 32 * wpb, smem, st>>>(logits, (int)T, (int)E, k, r, ids);
        e = cudaGetLastError();
    }
    cudaError_t e2 = cudaFreeAsync(base, st);
    return e == cudaSuccess ? e2 : e;
}

namespace {
// The whole layer; with `given` (one expert id per row, k = 1) the routing is
// the caller's and out[t] is that expert's output.
cudaError_t launch_moe(const MoeWeights& w, int top_k, const float* x, const float* logits, const int32_t* given,
                       int64_t T, float* out, int32_t* selected, int* err, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const int64_t E = w.E, H = w.H, I = w.I;
    const int k = (int)(top_k < E ? top_k : E);
    if (E <= 0 || E > kMoeMaxExperts || k <= 0 || T * k > kMoeMaxAssignments || (2 * I) % 128 || H % 128)
        return cudaErrorInvalidValue;
    const int nblk_gu = (int)(2 * I / 128), nblk_dn = (int)(H / 128);
    const int64_t rows = T * k;                                   // grouped rows, at most
    const int64_t mtiles = rows / kGemmGroupTok + E;              // sum over experts of ceil(cnt / 64)
    const int64_t max_gu = mtiles * nblk_gu, max_dn = mtiles * nblk_dn;
    // scratch layout (256-byte aligned pieces)
    auto pad = [](int64_t b) { return (b + 255) / 256 * 256; };
    const int64_t bytes = pad(T * E * 4) + pad(rows * 4) * 4 + pad(E * 4) + pad((E + 1) * 4) +
                          pad(max_gu * 16) + pad(max_dn * 16) + pad(8) + pad(rows * H * 4) +
                          pad(rows * 2 * I * 4) + pad(rows * I * 4) + pad(rows * H * 4);
    uint8_t* base = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&base), (size_t)bytes, st);
    if (e != cudaSuccess) return e;
    uint8_t* p = base;
    Route r;
    r.probs = carve<float>(p, T * E);
    r.sel_e = carve<int>(p, rows);
    r.sel_w = carve<float>(p, rows);
    r.slot = carve<int>(p, rows);
    r.tok = carve<int>(p, rows);
    r.cnt = carve<int>(p, E);
    r.off = carve<int>(p, E + 1);
    r.tiles_gu = carve<int4>(p, max_gu);
    r.tiles_dn = carve<int4>(p, max_dn);
    r.ntiles = carve<int>(p, 2);
    float* xg = carve<float>(p, rows * H);
    float* y1 = carve<float>(p, rows * 2 * I);
    float* act = carve<float>(p, rows * I);
    float* y2 = carve<float>(p, rows * H);

    const int wpb = 8;  // tokens per routing block
    const size_t smem = (size_t)wpb * E * sizeof(float);
    e = cudaMemsetAsync(r.cnt, 0, (size_t)E * sizeof(int), st);
    if (e == cudaSuccess && smem > 48 * 1024)
        e = cudaFuncSetAttribute(moe_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) {
        if (given)
            moe_given_route_kernel<<<(unsigned)((T + 255) / 256), 256, 0, st>>>(given, (int)T, (int)E, r);
        else
            moe_route_kernel<<<(unsigned)((T + wpb - 1) / wpb), 32 * wpb, smem, st>>>(logits, (int)T, (int)E, k, r,
                                                                                     selected);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        moe_place_kernel<<<(unsigned)E, 256, 0, st>>>((int)T, (int)E, k, nblk_gu, nblk_dn, r);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        moe_gather_kernel<<<dim3((unsigned)((H + 255) / 256), (unsigned)rows), 256, 0, st>>>(x, H, r.tok, r.off + E,
                                                                                           rows, xg);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess)
        e = launch_gemm_tcgen05_grouped(w.fmt, w.gate_up, w.gate_up_scales, 2 * I, H, xg, H, rows, y1, 2 * I,
                                        r.tiles_gu, r.ntiles, max_gu, err, st);
    if (e == cudaSuccess) {
        const int64_t n = rows * I;
        moe_silu_kernel<<<(unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096), 256, 0, st>>>(y1, I, rows,
                                                                                                   act);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess)
        e = launch_gemm_tcgen05_grouped(w.fmt, w.down, w.down_scales, H, I, act, I, rows, y2, H, r.tiles_dn,
                                        r.ntiles + 1, max_dn, err, st);
    if (e == cudaSuccess) {
        moe_combine_kernel<<<dim3((unsigned)((H + 255) / 256), (unsigned)T), 256, 0, st>>>(y2, H, k, r.slot, r.sel_w,
                                                                                         out);
        e = cudaGetLastError();
    }
    cudaError_t e2 = cudaFreeAsync(base, st);
    return e == cudaSuccess ? e2 : e;
}

}  // namespace

}  // namespace bramha
