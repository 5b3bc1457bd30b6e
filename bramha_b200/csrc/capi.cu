// capi.cu -- the extern "C" boundary declared in include/bramha_cuda.h.
//
// Host-side equivalent of the reference's `WgpuComputePlane`
// (src/compute/wgpu_backend.rs:100-1728): a per-device context with a
// persistent weight registry keyed by "model:layer" (get_or_create_op,
// :603-722), least-recently-used eviction under a device-memory cap
// (ModelBuffers, :25-82), and synchronous host-buffer GEMV calls with the
// reference's error behaviour (size mismatch -> error string, :1096-1104;
// N == 0 or K == 0 -> zeros, :1092-1095).  Every entry point returns a status
// and records a message for bramha_cuda_last_error(); nothing throws across
// the boundary.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <list>
#include <utility>
#include <mutex>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

using namespace bramha;

struct bramha_weight {
    std::string key;
    int fmt = 0;
    int64_t N = 0, K = 0;
    int64_t row_bytes = 0, ldq = 0;
    uint8_t* q = nullptr;
    float* scales = nullptr;
    size_t bytes = 0;
    bool live = true;
    bool keyed = false;
    bramha_ctx* ctx = nullptr;
    std::list<std::string>::iterator lru_it;
    Sp24Weight sp{};  // 2:4 sparse layout inside q (is_sp24(fmt))
    bool shard = false;    // rows [row0, row0 + N) of an n_full-row weight (column-shard group)
    int64_t row0 = 0, n_full = 0;
};

struct bramha_ctx {
    int device = 0;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    std::mutex mu;  // registry + LRU
    std::unordered_map<std::string, bramha_weight*> reg;
    std::list<std::string> lru;          // front = least recently used
    std::vector<bramha_weight*> dead;    // evicted handles: stale pointers fail cleanly
    size_t cap = 0, used = 0;
    std::mutex io_mu;                    // device staging for host-buffer calls
    float* dev_x = nullptr;
    float* dev_y = nullptr;
    size_t dev_x_cap = 0, dev_y_cap = 0;
    // host-buffer chains: input and output copies on their own streams, ordered
    // against the GEMV launches block by block through events (created on first use)
    cudaStream_t copy_in = nullptr, copy_out = nullptr;
    std::vector<cudaEvent_t> events;
    DevStatus* d_status = nullptr;       // error word, wait bound, test fault switch (device)
    int* d_err = nullptr;                // &d_status->err: what kernels are handed
    int* h_err = nullptr;                // pinned host copy of the error word
    float* split_ws = nullptr;           // K-split partials of the tensor-core GEMV
    int* split_tickets = nullptr;        // per-tile arrival counters (kept zero between launches)
    int gemv_kernel = BRAMHA_GEMV_AUTO;  // kernel choice for the tiled formats
    // GEMV tuning (measured on the Qwen2-7B step: L2 lookahead slowed the large
    // launches, next-launch prefetch of 8 MB was neutral to slightly positive,
    // and a K-split whose tiles are short makes the epilogue the bottleneck)
    int64_t pf_lookahead = 0;            // GEMV L2 lookahead per CTA, bytes
    int64_t pf_next = 8 << 20;           // GEMV chain: bytes of the next launch requested into L2
    int evict_first = 0;                 // GEMV weight copies marked first to be evicted from L2
    int split_cost = 240;                // GEMV K-split plan: cost of splitting, eighths of a block
    int cc_depth = 4;                    // CUDA-core GEMV: CTAs per SM its K split aims for
    // GEMV programs: L2 lookahead per CTA, bytes (measured on the Qwen2-7B step:
    // 0 -> 1.48 ms, 128 KiB -> 1.52, 256 KiB -> 1.72; off by default)
    int64_t prog_lookahead = 0;
    // column-shard group (bramha_cuda_shard_*): this rank's symmetric arena
    // (control block, then allocations from the bottom and host-chain staging
    // from the top) and the peers' arenas opened through CUDA IPC
    int shard_world = 0, shard_rank = 0;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0, arena_used = 0, arena_top = 0;
    uint8_t* peer_arena[kMaxShardWorld] = {};
};

namespace {
// Control block at the start of every arena.
constexpr size_t kArenaArrive = 0;     // u32 arrive[world]: CTAs of rank r whose rows are here
constexpr size_t kArenaExpected = 64;  // u32 expected[world]: arrivals through the last launch
constexpr size_t kArenaDone = 128;     // u32: CTAs of the running launch that finished
constexpr size_t kArenaHeader = 4096;  // allocations start here
}  // namespace

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    cudaGetLastError();  // clear a sticky launch error so the next call can proceed
    return fail(e == cudaErrorMemoryAllocation ? BRAMHA_ERR_OOM : BRAMHA_ERR_CUDA, "CUDA error in %s: %s", what,
                cudaGetErrorString(e));
}

#define CK(call, what)                                   \
    do {                                                 \
        cudaError_t e_ = (call);                         \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

const char* fmt_name(int fmt) {
    switch (fmt) {
        case BRAMHA_FMT_F32: return "F32";
        case BRAMHA_FMT_W8: return "INT8";
        case BRAMHA_FMT_W4ZP8: return "INT4";
        case BRAMHA_FMT_LOG4: return "LOG4";
        case BRAMHA_FMT_SP24_F32: return "2:4 F32";
        case BRAMHA_FMT_SP24_W8: return "2:4 INT8";
        case BRAMHA_FMT_SP24_W4ZP8: return "2:4 INT4";
        default: return "?";
    }
}

bool valid_fmt(int fmt) { return fmt >= BRAMHA_FMT_F32 && fmt <= BRAMHA_FMT_LOG4; }

// Expected packed length, with the reference's wording for mismatches.
int check_sizes(int fmt, int64_t N, int64_t K, size_t q_bytes, size_t n_scales, bool scales_given) {
    if (!valid_fmt(fmt)) return fail(BRAMHA_ERR_INVALID, "unknown weight format %d", fmt);
    if (N < 0 || K < 0) return fail(BRAMHA_ERR_INVALID, "negative shape %lld x %lld", (long long)N, (long long)K);
    const int64_t rb = row_bytes_of(fmt, K);
    const int64_t unit = fmt == BRAMHA_FMT_F32 ? 4 : 1;
    const uint64_t expect = (uint64_t)N * (uint64_t)rb;
    if ((uint64_t)q_bytes != expect) {
        if (fmt == BRAMHA_FMT_W4ZP8 || fmt == BRAMHA_FMT_LOG4)
            return fail(BRAMHA_ERR_SIZE,
                        "Quantized %s weight size mismatch: weight length is %zu, expected %lld x (%lld / 2) = %llu",
                        fmt_name(fmt), q_bytes, (long long)N, (long long)K, (unsigned long long)expect);
        if (fmt == BRAMHA_FMT_W8)
            return fail(BRAMHA_ERR_SIZE,
                        "Quantized INT8 weight size mismatch: weight length is %zu, expected %lld x %lld = %llu",
                        q_bytes, (long long)N, (long long)K, (unsigned long long)expect);
        return fail(BRAMHA_ERR_SIZE, "Weight size mismatch: weight length is %zu, expected %lld x %lld = %llu",
                    q_bytes / unit, (long long)N, (long long)K, (unsigned long long)(expect / unit));
    }
    if (fmt != BRAMHA_FMT_F32) {
        if (!scales_given && N > 0) return fail(BRAMHA_ERR_INVALID, "scales pointer is NULL");
        if ((int64_t)n_scales != N)
            return fail(BRAMHA_ERR_SIZE, "Scale length mismatch: scales length is %zu, expected %lld", n_scales,
                        (long long)N);
    }
    return BRAMHA_OK;
}

void free_weight_memory(bramha_weight* w) {
    if (w->q) cudaFree(w->q);
    if (w->scales) cudaFree(w->scales);
    w->q = nullptr;
    w->scales = nullptr;
    w->live = false;
}

// Caller holds ctx->mu.
void evict_locked(bramha_ctx* ctx, const std::string& key) {
    auto it = ctx->reg.find(key);
    if (it == ctx->reg.end()) return;
    bramha_weight* w = it->second;
    cudaDeviceSynchronize();  // no launch, on any stream, may still read it
    ctx->used -= w->bytes;
    ctx->lru.erase(w->lru_it);
    ctx->reg.erase(it);
    free_weight_memory(w);
    ctx->dead.push_back(w);
}

void touch_locked(bramha_ctx* ctx, bramha_weight* w) { ctx->lru.splice(ctx->lru.end(), ctx->lru, w->lru_it); }

// Allocates and uploads (H2D when host, D2D otherwise) into the device
// layout: quantized formats are tiled by a kernel (from a temporary
// row-major copy when the source is in host memory); f32 rows are padded.
int upload(bramha_ctx* ctx, bramha_weight* w, const void* q, const float* scales, bool from_device,
           cudaStream_t st) {
    w->row_bytes = row_bytes_of(w->fmt, w->K);
    w->ldq = pitch_of(w->row_bytes);
    const bool tiled = is_tiled(w->fmt);
    const size_t qbytes = tiled ? (size_t)tiled_bytes(w->fmt, w->N, held_columns(w->fmt, w->K))
                                : (size_t)w->N * (size_t)w->ldq;
    const size_t sbytes = w->fmt == BRAMHA_FMT_F32 ? 0 : (size_t)w->N * sizeof(float);
    w->bytes = qbytes + sbytes;
    if (qbytes > 0) CK(cudaMalloc(&w->q, qbytes), "cudaMalloc(weight)");
    if (sbytes > 0) {
        cudaError_t e = cudaMalloc(&w->scales, sbytes);
        if (e != cudaSuccess) {
            free_weight_memory(w);
            return cuda_fail(e, "cudaMalloc(scales)");
        }
    }
    const cudaMemcpyKind kind = from_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    cudaError_t e = cudaSuccess;
    uint8_t* staging = nullptr;
    if (qbytes > 0 && tiled) {
        const uint8_t* src = static_cast<const uint8_t*>(q);
        const size_t raw = (size_t)w->N * (size_t)w->row_bytes;
        if (!from_device && raw > 0) {
            e = cudaMalloc(&staging, raw);
            if (e == cudaSuccess) e = cudaMemcpyAsync(staging, q, raw, cudaMemcpyHostToDevice, st);
            src = staging;
        }
        if (e == cudaSuccess) e = launch_tile_weights(w->fmt, src, w->row_bytes, w->N, w->K, w->q, st);
    } else if (qbytes > 0) {
        if (w->ldq != w->row_bytes) e = cudaMemsetAsync(w->q, 0, qbytes, st);
        if (e == cudaSuccess && w->row_bytes > 0)
            e = cudaMemcpy2DAsync(w->q, (size_t)w->ldq, q, (size_t)w->row_bytes, (size_t)w->row_bytes,
                                  (size_t)w->N, kind, st);
    }
    if (e == cudaSuccess && sbytes > 0) e = cudaMemcpyAsync(w->scales, scales, sbytes, kind, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (staging) cudaFree(staging);
    if (e != cudaSuccess) {
        free_weight_memory(w);
        return cuda_fail(e, "weight upload");
    }
    return BRAMHA_OK;
}

// Registry insert shared by every registration path: returns the cached
// weight for a known key (same shape and format required), otherwise evicts
// down to the cap, creates the weight and lets `fill` allocate and upload it
// (fill sets w->bytes and frees what it allocated on failure).
template <class Fill>
int register_with(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K, size_t need, Fill&& fill,
                  bramha_weight** out) {
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->mu);
    auto it = ctx->reg.find(key);
    if (it != ctx->reg.end()) {
        bramha_weight* w = it->second;
        if (w->fmt != fmt || w->N != N || w->K != K)
            return fail(BRAMHA_ERR_SIZE, "key '%s' is registered with a different shape or format", key);
        touch_locked(ctx, w);
        *out = w;
        return BRAMHA_OK;
    }
    // enforce_limits (wgpu_backend.rs:65-81): evict least recently used first.
    while (ctx->cap > 0 && ctx->used + need > ctx->cap && !ctx->lru.empty()) evict_locked(ctx, ctx->lru.front());
    bramha_weight* w = new (std::nothrow) bramha_weight();
    if (!w) return fail(BRAMHA_ERR_OOM, "host allocation failed");
    w->key = key;
    w->fmt = fmt;
    w->N = N;
    w->K = K;
    w->keyed = true;
    w->ctx = ctx;
    int rc = fill(w);
    if (rc) {
        delete w;
        return rc;
    }
    ctx->used += w->bytes;
    ctx->lru.push_back(w->key);
    w->lru_it = std::prev(ctx->lru.end());
    ctx->reg.emplace(w->key, w);
    *out = w;
    return BRAMHA_OK;
}

int register_impl(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K, const void* q,
                  size_t q_bytes, const float* scales, size_t n_scales, bool from_device, cudaStream_t st,
                  bramha_weight** out) {
    if (!ctx || !out) return fail(BRAMHA_ERR_INVALID, "null context or output pointer");
    if (!key) return fail(BRAMHA_ERR_INVALID, "null weight key");
    int rc = check_sizes(fmt, N, K, q_bytes, n_scales, scales != nullptr);
    if (rc) return rc;
    if (!q && q_bytes > 0) return fail(BRAMHA_ERR_INVALID, "weight pointer is NULL");
    const size_t need = (is_tiled(fmt) ? (size_t)tiled_bytes(fmt, N, held_columns(fmt, K))
                                       : (size_t)N * (size_t)pitch_of(row_bytes_of(fmt, K))) +
                        (fmt == BRAMHA_FMT_F32 ? 0 : (size_t)N * sizeof(float));
    return register_with(
        ctx, key, fmt, N, K, need,
        [&](bramha_weight* w) { return upload(ctx, w, q, scales, from_device, st ? st : ctx->stream); }, out);
}

// ---- 2:4 sparse weights ---------------------------------------------------

// Device bytes of a 2:4 weight: code pairs, column pairs, tail, scales.
size_t sp24_bytes(int base_fmt, int64_t N, int64_t K, size_t* idx_off, size_t* tail_off) {
    const int64_t cp = sp24_groups_padded(K);
    const size_t v = (size_t)N * (size_t)(cp * sp24_value_bytes(base_fmt));
    const size_t i = (size_t)N * (size_t)(cp / 8) * 4;
    const size_t t = (K % 4) ? (size_t)N * 4 * sizeof(float) : 0;
    if (idx_off) *idx_off = v;
    if (tail_off) *tail_off = v + i;
    return v + i + t + (size_t)N * sizeof(float);
}

// Allocates the 2:4 layout of w (w->fmt, N, K set) and fills in w->sp.
int sp24_alloc(bramha_weight* w, bool with_tail) {
    const int base = sp24_base(w->fmt);
    size_t idx_off = 0, tail_off = 0;
    const size_t total = sp24_bytes(base, w->N, w->K, &idx_off, &tail_off);
    const size_t qbytes = total - (size_t)w->N * sizeof(float);
    w->bytes = total;
    if (qbytes > 0) CK(cudaMalloc(&w->q, qbytes), "cudaMalloc(2:4 weight)");
    if (w->N > 0) {
        cudaError_t e = cudaMalloc(&w->scales, (size_t)w->N * sizeof(float));
        if (e != cudaSuccess) {
            free_weight_memory(w);
            return cuda_fail(e, "cudaMalloc(scales)");
        }
    }
    Sp24Weight& sp = w->sp;
    sp.N = w->N;
    sp.K = w->K;
    sp.Cp = sp24_groups_padded(w->K);
    sp.ldv = sp.Cp * sp24_value_bytes(base);
    sp.ldi = sp.Cp / 8;
    sp.vals = w->q;
    sp.idx = reinterpret_cast<uint32_t*>(w->q + idx_off);
    sp.tail = (with_tail && (w->K % 4)) ? reinterpret_cast<float*>(w->q + tail_off) : nullptr;
    sp.scales = w->scales;
    return BRAMHA_OK;
}

// The on-the-fly selection of sparse_matvec_mul_2_4_tensor_into
// (cpu_engine.rs:1532-1640), made once: uploads the reference-layout weight
// to a staging buffer and prunes it on the device.
int sp24_fill_pruned(bramha_weight* w, const void* q, const float* scales, bool from_device,
                     cudaStream_t st) {
    int rc = sp24_alloc(w, true);
    if (rc) return rc;
    const int base = sp24_base(w->fmt);
    const int64_t rb = row_bytes_of(base, w->K);
    const size_t raw = (size_t)w->N * (size_t)rb;
    const cudaMemcpyKind kind = from_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    cudaError_t e = cudaSuccess;
    uint8_t* staging = nullptr;
    const uint8_t* src = static_cast<const uint8_t*>(q);
    if (!from_device && raw > 0) {
        e = cudaMalloc(&staging, raw);
        if (e == cudaSuccess) e = cudaMemcpyAsync(staging, q, raw, cudaMemcpyHostToDevice, st);
        src = staging;
    }
    if (e == cudaSuccess && raw > 0) e = launch_sp24_prune(base, src, rb, w->sp, st);
    if (e == cudaSuccess && w->N > 0) {
        if (base == BRAMHA_FMT_F32) {  // the reference's f32 arm has no scale
            std::vector<float> ones((size_t)w->N, 1.0f);
            e = cudaMemcpyAsync(w->scales, ones.data(), ones.size() * sizeof(float), cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        } else {
            e = cudaMemcpyAsync(w->scales, scales, (size_t)w->N * sizeof(float), kind, st);
        }
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (staging) cudaFree(staging);
    if (e != cudaSuccess) {
        free_weight_memory(w);
        return cuda_fail(e, "2:4 weight upload");
    }
    return BRAMHA_OK;
}

int sp24_check_pruned(int fmt, int64_t N, int64_t K, size_t q_bytes, size_t n_scales, bool scales_given) {
    if (fmt != BRAMHA_FMT_F32 && fmt != BRAMHA_FMT_W8 && fmt != BRAMHA_FMT_W4ZP8)
        return fail(BRAMHA_ERR_INVALID, "2:4 selection takes F32, W8 or W4ZP8 weights, not format %d", fmt);
    int rc = check_sizes(fmt, N, K, q_bytes, n_scales, scales_given);
    if (rc) return rc;
    // The reference's int4 arm reads byte (c + 2) / 2 of a K/2-byte row and
    // panics for odd K (cpu_engine.rs:1604-1633).
    if (fmt == BRAMHA_FMT_W4ZP8 && (K % 2) != 0)
        return fail(BRAMHA_ERR_UNSUPPORTED, "2:4 INT4 selection needs an even in_features (got %lld)", (long long)K);
    if (K > (int64_t)1 << 30 || N > 0x7fffffffLL) return fail(BRAMHA_ERR_UNSUPPORTED, "2:4 weight too large");
    return BRAMHA_OK;
}

// sparse_matvec_2_4_compressed (spanda-engine/src/sparse.rs:100-138) reads,
// for row r, masks[r*C + c] (C = cols / 4, low 4 bits, ascending bit order)
// and consumes values from index 2*r*C onwards while any remain.  The walk is
// restated here once and each group's (column, value) pairs are stored in
// the 2:4 layout (in column order, which is the order the reference consumes
// them), with the id of their column pair.  A group that
// consumes more than two values is not 2:4 and is refused.
int sp24_canonicalise(int64_t rows, int64_t cols, const uint16_t* masks, const float* values, size_t n_values,
                      std::vector<uint8_t>& vals, std::vector<uint32_t>& idx) {
    const int64_t C = cols / 4, cp = sp24_groups_padded(cols);
    vals.assign((size_t)(rows * cp * 8), 0);
    idx.assign((size_t)(rows * (cp / 8)), 0);
    for (int64_t r = 0; r < rows; ++r) {
        size_t vi = (size_t)(r * C * 2);
        for (int64_t c = 0; c < C; ++c) {
            const unsigned m = masks[r * C + c] & 0xFu;
            int n = 0, col[2] = {0, 1};
            float val[2] = {0.f, 0.f};
            for (int bit = 0; bit < 4; ++bit) {
                if (!(m & (1u << bit)) || vi >= n_values) continue;
                if (n == 2)
                    return fail(BRAMHA_ERR_UNSUPPORTED,
                                "2:4 mask of row %lld group %lld keeps more than two of four columns (mask 0x%x)",
                                (long long)r, (long long)c, masks[r * C + c]);
                col[n] = bit;
                val[n] = values[vi++];
                ++n;
            }
            if (n == 1) {  // an empty slot: value 0 at another column, slots in column order
                col[1] = col[0] == 0 ? 1 : 0;
                if (col[1] < col[0]) {
                    std::swap(col[0], col[1]);
                    std::swap(val[0], val[1]);
                }
            }
            memcpy(&vals[(size_t)((r * cp + c) * 8)], val, 8);
            idx[(size_t)(r * (cp / 8) + c / 8)] |= (uint32_t)sp24_pair_id(col[0], col[1]) << (4 * (c % 8));
        }
        // padding groups: zero values at pair 0 (columns 0 and 1), id bits 0
    }
    return BRAMHA_OK;
}

int sp24_fill_compressed(bramha_weight* w, const std::vector<uint8_t>& vals, const std::vector<uint32_t>& idx,
                         cudaStream_t st) {
    int rc = sp24_alloc(w, false);
    if (rc) return rc;
    cudaError_t e = cudaSuccess;
    if (!vals.empty()) e = cudaMemcpyAsync(w->sp.vals, vals.data(), vals.size(), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && !idx.empty())
        e = cudaMemcpyAsync(w->sp.idx, idx.data(), idx.size() * 4, cudaMemcpyHostToDevice, st);
    std::vector<float> ones((size_t)w->N, 1.0f);
    if (e == cudaSuccess && w->N > 0)
        e = cudaMemcpyAsync(w->scales, ones.data(), ones.size() * sizeof(float), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        free_weight_memory(w);
        return cuda_fail(e, "2:4 weight upload");
    }
    return BRAMHA_OK;
}

int sp24_check_compressed(int64_t rows, int64_t cols, size_t n_masks, const uint16_t* masks, const float* values,
                          size_t n_values) {
    if (rows < 0 || cols < 0) return fail(BRAMHA_ERR_INVALID, "negative shape");
    if (cols > (int64_t)1 << 30 || rows > 0x7fffffffLL) return fail(BRAMHA_ERR_UNSUPPORTED, "2:4 weight too large");
    // masks[r * C + c] must exist for every row (the reference would panic).
    if ((uint64_t)n_masks < (uint64_t)rows * (uint64_t)(cols / 4))
        return fail(BRAMHA_ERR_SIZE, "2:4 masks length is %zu, expected %lld x (%lld / 4) = %lld", n_masks,
                    (long long)rows, (long long)cols, (long long)(rows * (cols / 4)));
    if ((!masks && n_masks > 0) || (!values && n_values > 0))
        return fail(BRAMHA_ERR_INVALID, "null masks or values pointer");
    return BRAMHA_OK;
}

int check_weight(const bramha_ctx* ctx, const bramha_weight* w) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (!w) return fail(BRAMHA_ERR_INVALID, "null weight");
    if (w->ctx != ctx) return fail(BRAMHA_ERR_INVALID, "weight belongs to another context");
    if (!w->live) return fail(BRAMHA_ERR_NOT_FOUND, "weight '%s' was evicted", w->key.c_str());
    return BRAMHA_OK;
}

// Core device GEMV over several weights sharing x.  x must be 16-byte aligned
// with row pitch ldx (a multiple of 4 floats when batch > 1).
// x_up (optional, tensor-core formats only): the activation is silu(x) * x_up.
// next_ws (optional): the weights of the next launch of a chain, whose first
// bytes the tensor-core GEMV requests into L2 at its tail.
int gemv_device_sharded(bramha_ctx* ctx, int n, const bramha_weight* const* ws, const float* x, int64_t ldx,
                        int64_t batch, float* const* ys, cudaStream_t st, const float* x_up, int next_n,
                        const bramha_weight* const* next_ws);

// RMSNorm folded into a batch-1 GEMV's activation staging (GemvArgs::norm_w).
struct NormIn {
    const float* w;      // norm weight [K]
    const float* delta;  // residual added to x first (may be null)
    float* x_out;        // receives x + delta (may be null)
    float eps;
};

int gemv_device(bramha_ctx* ctx, int n, const bramha_weight* const* ws, const float* x, int64_t ldx,
                int64_t batch, float* const* ys, cudaStream_t st, const float* x_up = nullptr, int next_n = 0,
                const bramha_weight* const* next_ws = nullptr, const NormIn* norm = nullptr) {
    const int fmt = ws[0]->fmt;
    const int64_t K = ws[0]->K;
    for (int i = 1; i < n; ++i)
        if (ws[i]->shard != ws[0]->shard)
            return fail(BRAMHA_ERR_INVALID, "one launch cannot mix sharded and unsharded weights");
    if (ws[0]->shard) return gemv_device_sharded(ctx, n, ws, x, ldx, batch, ys, st, x_up, next_n, next_ws);
    if (batch <= 0) return BRAMHA_OK;
    if (K == 0) {
        for (int i = 0; i < n; ++i)
            if (ws[i]->N > 0) CK(cudaMemsetAsync(ys[i], 0, sizeof(float) * ws[i]->N * batch, st), "memset(y)");
        return BRAMHA_OK;
    }
    if (K > 0x7fffffffLL) return fail(BRAMHA_ERR_UNSUPPORTED, "K too large");
    if (is_sp24(fmt)) {  // one launch per weight and activation row
        for (int i = 0; i < n; ++i)
            for (int64_t b = 0; b < batch; ++b)
                CK(launch_sp24_gemv(sp24_base(fmt), ws[i]->sp, x + b * ldx, ys[i] + b * ws[i]->N, ctx->split_ws,
                                    kSplitWsFloats, ctx->split_tickets, kSplitTickets, ctx->num_sms, st),
                   "2:4 gemv launch");
        return BRAMHA_OK;
    }
    if (is_tiled(fmt) && batch > kMaxGemvBatch) {
        // More activation rows than the GEMV kernels take: the tcgen05 GEMM with
        // the weights as the M operand and the rows as N (f32 rows split into
        // bf16 hi + lo halves of the MMA's N, so each weight block is read once;
        // K-split when the weight has fewer 128-row blocks than SMs), the
        // reference's batched form being gemm_cpu (cpu_engine.rs:565-912).
        const float* xin = x;
        float* act = nullptr;
        if (x_up) {  // SwiGLU: silu(x) * x_up first, rounded as bramha_cuda_op_silu_mul
            CK(cudaMallocAsync(reinterpret_cast<void**>(&act), sizeof(float) * (size_t)(batch * ldx), st),
               "cudaMallocAsync(swiglu activations)");
            cudaError_t e = launch_silu_mul(x, x_up, batch * ldx, act, st);
            if (e != cudaSuccess) {
                cudaFreeAsync(act, st);
                return cuda_fail(e, "silu_mul launch");
            }
            xin = act;
        }
        GemmOut outs[kMaxSegments];
        for (int i = 0; i < n; ++i) outs[i] = GemmOut{ws[i]->q, ws[i]->scales, ws[i]->N, ys[i], ws[i]->N};
        cudaError_t e = launch_gemm_tcgen05_multi(fmt, n, outs, held_columns(fmt, K), xin, 1, ldx, batch, ctx->d_err,
                                                  ctx->split_ws, kSplitWsFloats, ctx->split_tickets, kSplitTickets, st);
        if (act) {
            cudaError_t e2 = cudaFreeAsync(act, st);
            if (e == cudaSuccess) e = e2;
        }
        if (e != cudaSuccess) return cuda_fail(e, "tcgen05 gemm launch (batched gemv)");
        return BRAMHA_OK;
    }
    for (int64_t b0 = 0; b0 < batch; b0 += kMaxGemvBatch) {
        const int bc = (int)((batch - b0) < kMaxGemvBatch ? (batch - b0) : kMaxGemvBatch);
        GemvArgs a{};
        a.x = x + b0 * ldx;
        a.x_up = x_up ? x_up + b0 * ldx : nullptr;
        a.ldx = ldx;
        // Columns the packed rows actually hold: with odd K a nibble row has
        // K/2 bytes and the last activation is ignored (cpu_engine.rs:1364).
        a.K = (int)held_columns(fmt, K);
        a.batch = bc;
        a.nseg = 0;
        a.ldq_min = 0x7fffffff;
        for (int i = 0; i < n; ++i) {
            if (ws[i]->N == 0) continue;
            if (ws[i]->N > 0x7fffffffLL) return fail(BRAMHA_ERR_UNSUPPORTED, "N too large");
            GemvSeg& s = a.seg[a.nseg++];
            s.q = ws[i]->q;
            s.scales = ws[i]->scales;
            s.ldq = ws[i]->ldq;
            s.ldy = ws[i]->N;
            s.y = ys[i] + b0 * ws[i]->N;
            s.N = (int)ws[i]->N;
            if (ws[i]->ldq < a.ldq_min) a.ldq_min = (int)ws[i]->ldq;
        }
        if (a.nseg == 0) return BRAMHA_OK;
        a.err = ctx->d_err;
        a.split_ws = ctx->split_ws;
        a.split_ws_floats = kSplitWsFloats;
        a.split_tickets = ctx->split_tickets;
        a.split_tickets_n = kSplitTickets;
        a.pf_ahead = (int)(ctx->pf_lookahead / (2 * 8192));
        a.evict_first = ctx->evict_first;
        a.split_cost = ctx->split_cost;
        a.cc_depth = ctx->cc_depth;
        a.pf_next_n = 0;
        a.pf_next_total = 0;
        if (b0 + kMaxGemvBatch >= batch) {  // the last chunk of this op hands over to the next op
            for (int i = 0; i < next_n && i < kMaxSegments; ++i) {
                const bramha_weight* nw = next_ws[i];
                if (!nw || !is_tiled(nw->fmt) || nw->N == 0 || nw->K == 0) continue;
                a.pf_next_ptr[a.pf_next_n] = nw->q;
                a.pf_next_bytes[a.pf_next_n] = tiled_bytes(nw->fmt, nw->N, held_columns(nw->fmt, nw->K));
                ++a.pf_next_n;
            }
            a.pf_next_total = a.pf_next_n ? ctx->pf_next : 0;
        }
        const bool cc = !x_up && (ctx->gemv_kernel == BRAMHA_GEMV_CUDA_CORE
                                      ? is_tiled(fmt) && a.batch == 1
                                      : ctx->gemv_kernel == BRAMHA_GEMV_AUTO && gemv_cc_eligible(fmt, a));
        if (norm) {  // only the CUDA-core kernel forms the RMSNorm (the caller checked cc)
            if (!cc || a.batch != 1 || a.K != K) return fail(BRAMHA_ERR_INVALID, "internal: fused RMSNorm without the CUDA-core GEMV");
            a.norm_w = norm->w;
            a.delta = norm->delta;
            a.x_out = norm->x_out;
            a.eps = norm->eps;
        }
        if (cc)
            CK(launch_gemv_cc(fmt, a, ctx->num_sms, st), "cuda-core gemv launch");
        else if (is_tiled(fmt))
            CK(launch_gemv_tc(fmt, a, ctx->num_sms, st), "tensor-core gemv launch");
        else
            CK(launch_gemv_f32(a, ctx->num_sms, st), "gemv launch");
    }
    return BRAMHA_OK;
}

// Shard-group view of the context for the kernels.
ShardArgs shard_args(bramha_ctx* ctx) {
    ShardArgs sa{};
    sa.world = ctx->shard_world;
    sa.rank = ctx->shard_rank;
    sa.arrive = reinterpret_cast<unsigned*>(ctx->arena + kArenaArrive);
    sa.expected = reinterpret_cast<unsigned*>(ctx->arena + kArenaExpected);
    sa.done = reinterpret_cast<unsigned*>(ctx->arena + kArenaDone);
    for (int r = 0; r < ctx->shard_world; ++r) {
        sa.peer_arrive[r] = reinterpret_cast<unsigned*>(ctx->peer_arena[r] + kArenaArrive);
        sa.grid_of[r] = 1;
    }
    return sa;
}

bool in_arena(const bramha_ctx* ctx, const void* p, size_t bytes) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    return b >= ctx->arena + kArenaHeader && b + bytes <= ctx->arena + ctx->arena_bytes;
}

// GEMV of sharded weights: this rank's rows of every output, stored into every
// rank's copy of it by the tensor-core GEMV's epilogue (see ShardArgs).
int gemv_device_sharded(bramha_ctx* ctx, int n, const bramha_weight* const* ws, const float* x, int64_t ldx,
                        int64_t batch, float* const* ys, cudaStream_t st, const float* x_up, int next_n,
                        const bramha_weight* const* next_ws) {
    if (ctx->shard_world < 2) return fail(BRAMHA_ERR_INVALID, "sharded weights need a shard group (bramha_cuda_shard_init)");
    if (batch < 1 || batch > kMaxGemvBatch)
        return fail(BRAMHA_ERR_UNSUPPORTED, "a sharded GEMV takes batch 1..%d (got %lld)", kMaxGemvBatch, (long long)batch);
    const int fmt = ws[0]->fmt;
    const int64_t K = ws[0]->K;
    for (int i = 0; i < n; ++i)
        if (!ys[i] || !in_arena(ctx, ys[i], sizeof(float) * (size_t)(batch * ws[i]->n_full)))
            return fail(BRAMHA_ERR_INVALID,
                        "the output of a sharded GEMV must lie in the shard arena (bramha_cuda_shard_malloc), "
                        "[batch][N] for the full N");
    ShardArgs sa = shard_args(ctx);
    // every rank's grid for this launch (each rank's rows of each weight, the
    // same plan as the launch): what the ranks' arrivals must add up to
    if (held_columns(fmt, K) > 0 && K <= 0x7fffffffLL)
        for (int r = 0; r < ctx->shard_world; ++r) {
            int64_t nt = 0;
            for (int i = 0; i < n; ++i) {
                const int64_t n_full = ws[i]->n_full;
                nt += row_tiles(n_full * (r + 1) / ctx->shard_world - n_full * r / ctx->shard_world);
            }
            const int gr = nt == 0 ? 1
                                   : gemv_tc_grid(fmt, (int)batch, (int)nt, (int)held_columns(fmt, K), ctx->num_sms,
                                                  ctx->split_cost, kSplitWsFloats, kSplitTickets);
            if (gr <= 0) return fail(BRAMHA_ERR_UNSUPPORTED, "sharded GEMV: no launch plan for rank %d", r);
            sa.grid_of[r] = gr;
        }
    if (held_columns(fmt, K) == 0) {  // an empty input: every rank zeroes its own copies
        for (int i = 0; i < n; ++i)
            CK(cudaMemsetAsync(ys[i], 0, sizeof(float) * (size_t)(batch * ws[i]->n_full), st), "memset(y)");
        CK(launch_shard_signal(sa, ctx->d_err, 1, st), "shard signal launch");
        return BRAMHA_OK;
    }
    if (K > 0x7fffffffLL) return fail(BRAMHA_ERR_UNSUPPORTED, "K too large");
    GemvArgs a{};
    a.x = x;
    a.x_up = x_up;
    a.ldx = ldx;
    a.K = (int)held_columns(fmt, K);
    a.batch = (int)batch;
    a.ldq_min = 0x7fffffff;
    for (int i = 0; i < n; ++i) {
        if (ws[i]->N == 0) continue;
        const int si = a.nseg++;
        GemvSeg& g = a.seg[si];
        g.q = ws[i]->q;
        g.scales = ws[i]->scales;
        g.ldq = ws[i]->ldq;
        g.ldy = ws[i]->n_full;
        g.y = ys[i];
        g.N = (int)ws[i]->N;
        sa.row0[si] = ws[i]->row0;
        for (int r = 0; r < ctx->shard_world; ++r)
            sa.peer_y[si][r] = reinterpret_cast<float*>(ctx->peer_arena[r] +
                                                        (reinterpret_cast<uint8_t*>(ys[i]) - ctx->arena));
    }
    if (a.nseg == 0) {  // no rows here: take part in the launch order only
        CK(launch_shard_signal(sa, ctx->d_err, 1, st), "shard signal launch");
        return BRAMHA_OK;
    }
    a.err = ctx->d_err;
    a.split_ws = ctx->split_ws;
    a.split_ws_floats = kSplitWsFloats;
    a.split_tickets = ctx->split_tickets;
    a.split_tickets_n = kSplitTickets;
    a.pf_ahead = (int)(ctx->pf_lookahead / (2 * 8192));
    a.evict_first = ctx->evict_first;
    a.split_cost = ctx->split_cost;
    a.cc_depth = ctx->cc_depth;
    for (int i = 0; i < next_n && i < kMaxSegments; ++i) {
        const bramha_weight* nw = next_ws[i];
        if (!nw || !is_tiled(nw->fmt) || nw->N == 0 || nw->K == 0) continue;
        a.pf_next_ptr[a.pf_next_n] = nw->q;
        a.pf_next_bytes[a.pf_next_n] = tiled_bytes(nw->fmt, nw->N, held_columns(nw->fmt, nw->K));
        ++a.pf_next_n;
    }
    a.pf_next_total = a.pf_next_n ? ctx->pf_next : 0;
    a.shard = sa;
    CK(launch_gemv_tc(fmt, a, ctx->num_sms, st), "sharded tensor-core gemv launch");
    return BRAMHA_OK;
}

// Waits for the stream, then reports (and clears) a device-side failure: the
// error word is read back in the same stream, so one wait covers both.
int check_device_error(bramha_ctx* ctx, cudaStream_t st) {
    CK(cudaMemcpyAsync(ctx->h_err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, st), "read error word");
    CK(cudaStreamSynchronize(st), "stream sync");
    const int h = *ctx->h_err;
    if (h != 0) {
        cudaMemsetAsync(ctx->d_err, 0, sizeof(int), st);
        // an aborted launch may leave K-split tickets taken
        cudaMemsetAsync(ctx->split_tickets, 0, sizeof(int) * (size_t)kSplitTickets, st);
        cudaStreamSynchronize(st);
        return fail(h == BRAMHA_ERR_TIMEOUT ? BRAMHA_ERR_TIMEOUT : BRAMHA_ERR_CUDA,
                    "a kernel gave up a bounded wait (device error word %d)", h);
    }
    return BRAMHA_OK;
}

// Prefill GEMM on the tensor cores for the quantized formats; dense f32
// weights go through the GEMV kernels in batch chunks.
int gemm_device(bramha_ctx* ctx, const bramha_weight* w, const void* x, int x_is_f32, int64_t ldx, int64_t M,
                float* y, cudaStream_t st) {
    if (M <= 0 || w->N == 0) return BRAMHA_OK;
    if (w->K == 0) {
        CK(cudaMemsetAsync(y, 0, sizeof(float) * w->N * M, st), "memset(y)");
        return BRAMHA_OK;
    }
    if (w->fmt == BRAMHA_FMT_F32 || is_sp24(w->fmt)) {
        if (!x_is_f32) return fail(BRAMHA_ERR_UNSUPPORTED, "%s weights take f32 activations", fmt_name(w->fmt));
        const bramha_weight* ws[1] = {w};
        float* ys[1] = {y};
        return gemv_device(ctx, 1, ws, static_cast<const float*>(x), ldx, M, ys, st);
    }
    const int64_t keff = (w->fmt == BRAMHA_FMT_W4ZP8 || w->fmt == BRAMHA_FMT_LOG4) ? (w->K / 2) * 2 : w->K;
    if (keff == 0) {
        CK(cudaMemsetAsync(y, 0, sizeof(float) * w->N * M, st), "memset(y)");
        return BRAMHA_OK;
    }
    CK(launch_gemm_tcgen05(w->fmt, w->q, w->ldq, w->scales, w->N, keff, x, x_is_f32, ldx, M, y, w->N, ctx->d_err,
                           ctx->split_ws, kSplitWsFloats, ctx->split_tickets, kSplitTickets, st),
       "tcgen05 gemm launch");
    return BRAMHA_OK;
}

int ensure_staging(bramha_ctx* ctx, size_t x_elems, size_t y_elems) {
    if (x_elems > ctx->dev_x_cap) {
        if (ctx->dev_x) cudaFree(ctx->dev_x);
        ctx->dev_x = nullptr;
        ctx->dev_x_cap = 0;
        CK(cudaMalloc(&ctx->dev_x, x_elems * sizeof(float)), "cudaMalloc(x staging)");
        ctx->dev_x_cap = x_elems;
    }
    if (y_elems > ctx->dev_y_cap) {
        if (ctx->dev_y) cudaFree(ctx->dev_y);
        ctx->dev_y = nullptr;
        ctx->dev_y_cap = 0;
        CK(cudaMalloc(&ctx->dev_y, y_elems * sizeof(float)), "cudaMalloc(y staging)");
        ctx->dev_y_cap = y_elems;
    }
    return BRAMHA_OK;
}

// The host-buffer chain's copy streams and at least n events (caller holds io_mu).
int ensure_copy_streams(bramha_ctx* ctx, size_t n_events) {
    if (!ctx->copy_in) CK(cudaStreamCreateWithFlags(&ctx->copy_in, cudaStreamNonBlocking), "cudaStreamCreate(copy in)");
    if (!ctx->copy_out)
        CK(cudaStreamCreateWithFlags(&ctx->copy_out, cudaStreamNonBlocking), "cudaStreamCreate(copy out)");
    while (ctx->events.size() < n_events) {
        cudaEvent_t ev;
        CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "cudaEventCreate");
        ctx->events.push_back(ev);
    }
    return BRAMHA_OK;
}

// Host-buffer GEMV/GEMM: H2D x, launch, D2H y, wait.
int gemv_host(bramha_ctx* ctx, const bramha_weight* w, const float* x_host, int64_t batch, float* y_host) {
    if (batch < 0) return fail(BRAMHA_ERR_INVALID, "negative batch");
    if (w->shard) {  // every rank's rows, through the host-buffer chain (y_host is [batch][full N])
        const bramha_weight* ws[1] = {w};
        float* ys[1] = {y_host};
        const bramha_gemv_op op = {1, ws, x_host, nullptr, ys};
        return bramha_cuda_gemv_chain(ctx, 1, &op, batch);
    }
    if (batch > 0 && ((!x_host && w->K > 0) || (!y_host && w->N > 0)))
        return fail(BRAMHA_ERR_INVALID, "null host buffer");
    if (batch == 0 || w->N == 0) return BRAMHA_OK;
    if (w->K == 0) {
        memset(y_host, 0, sizeof(float) * (size_t)(w->N * batch));
        return BRAMHA_OK;
    }
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->io_mu);
    const int64_t ldx = (w->K + 3) / 4 * 4;
    int rc = ensure_staging(ctx, (size_t)(ldx * batch), (size_t)(w->N * batch));
    if (rc) return rc;
    cudaStream_t st = ctx->stream;
    CK(cudaMemcpy2DAsync(ctx->dev_x, ldx * sizeof(float), x_host, w->K * sizeof(float), w->K * sizeof(float),
                         (size_t)batch, cudaMemcpyHostToDevice, st),
       "H2D x");
    const bramha_weight* ws[1] = {w};
    float* ys[1] = {ctx->dev_y};
    rc = gemv_device(ctx, 1, ws, ctx->dev_x, ldx, batch, ys, st);
    if (rc) return rc;
    CK(cudaMemcpyAsync(y_host, ctx->dev_y, sizeof(float) * (size_t)(w->N * batch), cudaMemcpyDeviceToHost, st),
       "D2H y");
    return check_device_error(ctx, st);
}

}  // namespace

extern "C" {

const char* bramha_cuda_last_error(void) { return g_last_error.c_str(); }

int bramha_cuda_abi_version(void) { return BRAMHA_CUDA_ABI_VERSION; }

int bramha_cuda_init(int device, bramha_ctx** out) {
    if (!out) return fail(BRAMHA_ERR_INVALID, "null output pointer");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(BRAMHA_ERR_CUDA, "no CUDA device available (%s)", cudaGetErrorString(e));
    }
    if (device < 0 || device >= n) return fail(BRAMHA_ERR_INVALID, "device %d out of range (%d devices)", device, n);
    cudaDeviceProp p;
    CK(cudaGetDeviceProperties(&p, device), "cudaGetDeviceProperties");
    if (p.major != 10)
        return fail(BRAMHA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", device,
                    p.major, p.minor);
    bramha_ctx* ctx = new (std::nothrow) bramha_ctx();
    if (!ctx) return fail(BRAMHA_ERR_OOM, "host allocation failed");
    ctx->device = device;
    ctx->num_sms = p.multiProcessorCount;
    DeviceGuard g(device);
    e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete ctx;
        return cuda_fail(e, "cudaStreamCreate");
    }
    e = cudaMalloc(&ctx->d_status, sizeof(DevStatus));
    if (e == cudaSuccess) {
        const DevStatus init = {0, kFaultNone, kDefaultTimeoutNs};
        e = cudaMemcpy(ctx->d_status, &init, sizeof init, cudaMemcpyHostToDevice);
        ctx->d_err = &ctx->d_status->err;
    }
    if (e == cudaSuccess) e = cudaMallocHost(&ctx->h_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->split_ws, sizeof(float) * (size_t)kSplitWsFloats);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->split_tickets, sizeof(int) * (size_t)kSplitTickets);
    if (e == cudaSuccess) e = cudaMemset(ctx->split_tickets, 0, sizeof(int) * (size_t)kSplitTickets);
    if (e != cudaSuccess) {
        if (ctx->d_status) cudaFree(ctx->d_status);
        if (ctx->h_err) cudaFreeHost(ctx->h_err);
        if (ctx->split_ws) cudaFree(ctx->split_ws);
        if (ctx->split_tickets) cudaFree(ctx->split_tickets);
        cudaStreamDestroy(ctx->stream);
        delete ctx;
        return cuda_fail(e, "cudaMalloc(context scratch)");
    }
    *out = ctx;
    return BRAMHA_OK;
}

int bramha_cuda_destroy(bramha_ctx* ctx) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    DeviceGuard g(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        for (auto& kv : ctx->reg) {
            free_weight_memory(kv.second);
            delete kv.second;
        }
        for (bramha_weight* w : ctx->dead) delete w;
        ctx->reg.clear();
        ctx->dead.clear();
    }
    if (ctx->dev_x) cudaFree(ctx->dev_x);
    if (ctx->dev_y) cudaFree(ctx->dev_y);
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->h_err) cudaFreeHost(ctx->h_err);
    if (ctx->split_ws) cudaFree(ctx->split_ws);
    if (ctx->split_tickets) cudaFree(ctx->split_tickets);
    for (int r = 0; r < ctx->shard_world; ++r)
        if (r != ctx->shard_rank && ctx->peer_arena[r]) cudaIpcCloseMemHandle(ctx->peer_arena[r]);
    if (ctx->arena) cudaFree(ctx->arena);
    for (cudaEvent_t ev : ctx->events) cudaEventDestroy(ev);
    if (ctx->copy_in) cudaStreamDestroy(ctx->copy_in);
    if (ctx->copy_out) cudaStreamDestroy(ctx->copy_out);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return BRAMHA_OK;
}

int bramha_cuda_set_gemv_kernel(bramha_ctx* ctx, int kind) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (kind != BRAMHA_GEMV_AUTO && kind != BRAMHA_GEMV_TENSOR_CORE && kind != BRAMHA_GEMV_CUDA_CORE)
        return fail(BRAMHA_ERR_INVALID, "unknown GEMV kernel choice %d", kind);
    ctx->gemv_kernel = kind;
    return BRAMHA_OK;
}

int bramha_cuda_set_wait_timeout(bramha_ctx* ctx, uint64_t ns) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    const unsigned long long v = ns ? (unsigned long long)ns : kDefaultTimeoutNs;
    DeviceGuard g(ctx->device);
    CK(cudaMemcpy(&ctx->d_status->timeout_ns, &v, sizeof v, cudaMemcpyHostToDevice), "set wait timeout");
    return BRAMHA_OK;
}

int bramha_cuda_test_fault(bramha_ctx* ctx, int kind) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (kind != BRAMHA_TEST_FAULT_NONE && kind != BRAMHA_TEST_FAULT_GEMV && kind != BRAMHA_TEST_FAULT_GEMM)
        return fail(BRAMHA_ERR_INVALID, "unknown test fault %d", kind);
    static_assert(BRAMHA_TEST_FAULT_GEMV == kFaultGemvWithholdCopy && BRAMHA_TEST_FAULT_GEMM == kFaultGemmWithholdCopy,
                  "test fault codes");
    DeviceGuard g(ctx->device);
    CK(cudaMemcpy(&ctx->d_status->fault, &kind, sizeof kind, cudaMemcpyHostToDevice), "set test fault");
    return BRAMHA_OK;
}

int bramha_cuda_set_prefetch(bramha_ctx* ctx, int64_t lookahead_bytes, int64_t next_launch_bytes) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (lookahead_bytes < 0 || next_launch_bytes < 0) return fail(BRAMHA_ERR_INVALID, "negative prefetch size");
    ctx->pf_lookahead = lookahead_bytes;
    ctx->pf_next = next_launch_bytes;
    return BRAMHA_OK;
}

int bramha_cuda_set_gemv_tuning(bramha_ctx* ctx, int what, int64_t value) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (value < 0) return fail(BRAMHA_ERR_INVALID, "negative tuning value");
    switch (what) {
        case BRAMHA_TUNE_LOOKAHEAD_BYTES: ctx->pf_lookahead = value; break;
        case BRAMHA_TUNE_NEXT_LAUNCH_BYTES: ctx->pf_next = value; break;
        case BRAMHA_TUNE_EVICT_FIRST: ctx->evict_first = value ? 1 : 0; break;
        case BRAMHA_TUNE_PROGRAM_LOOKAHEAD_BYTES: ctx->prog_lookahead = value; break;
        case BRAMHA_TUNE_CC_SPLIT_DEPTH:
            if (value < 1 || value > 64) return fail(BRAMHA_ERR_INVALID, "CUDA-core split depth out of range (1..64)");
            ctx->cc_depth = (int)value;
            break;
        case BRAMHA_TUNE_SPLIT_COST:
            if (value > 1 << 20) return fail(BRAMHA_ERR_INVALID, "split cost out of range");
            ctx->split_cost = (int)value;
            break;
        default: return fail(BRAMHA_ERR_INVALID, "unknown tuning key %d", what);
    }
    return BRAMHA_OK;
}

int bramha_cuda_set_memory_cap(bramha_ctx* ctx, size_t bytes) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->mu);
    ctx->cap = bytes;
    while (ctx->cap > 0 && ctx->used > ctx->cap && !ctx->lru.empty()) evict_locked(ctx, ctx->lru.front());
    return BRAMHA_OK;
}

int bramha_cuda_memory_used(bramha_ctx* ctx, size_t* bytes) {
    if (!ctx || !bytes) return fail(BRAMHA_ERR_INVALID, "null argument");
    std::lock_guard<std::mutex> lk(ctx->mu);
    *bytes = ctx->used;
    return BRAMHA_OK;
}

int bramha_cuda_register_weight(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K, const void* q,
                                size_t q_bytes, const float* scales, size_t n_scales, bramha_weight** out) {
    return register_impl(ctx, key, fmt, N, K, q, q_bytes, scales, n_scales, false, nullptr, out);
}

int bramha_cuda_register_weight_dev(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K,
                                    const void* q_dev, size_t q_bytes, const float* scales_dev, size_t n_scales,
                                    void* stream, bramha_weight** out) {
    return register_impl(ctx, key, fmt, N, K, q_dev, q_bytes, scales_dev, n_scales, true,
                         static_cast<cudaStream_t>(stream), out);
}

int bramha_cuda_lookup_weight(bramha_ctx* ctx, const char* key, bramha_weight** out) {
    if (!ctx || !key || !out) return fail(BRAMHA_ERR_INVALID, "null argument");
    std::lock_guard<std::mutex> lk(ctx->mu);
    auto it = ctx->reg.find(key);
    if (it == ctx->reg.end()) return fail(BRAMHA_ERR_NOT_FOUND, "no weight registered under '%s'", key);
    touch_locked(ctx, it->second);
    *out = it->second;
    return BRAMHA_OK;
}

int bramha_cuda_evict_weight(bramha_ctx* ctx, const char* key) {
    if (!ctx || !key) return fail(BRAMHA_ERR_INVALID, "null argument");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (ctx->reg.find(key) == ctx->reg.end()) return fail(BRAMHA_ERR_NOT_FOUND, "no weight registered under '%s'", key);
    evict_locked(ctx, key);
    return BRAMHA_OK;
}

int bramha_cuda_clear(bramha_ctx* ctx) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->mu);
    while (!ctx->lru.empty()) evict_locked(ctx, ctx->lru.front());
    return BRAMHA_OK;
}

int bramha_cuda_weight_info(const bramha_weight* w, int* fmt, int64_t* N, int64_t* K, size_t* device_bytes) {
    if (!w) return fail(BRAMHA_ERR_INVALID, "null weight");
    if (!w->live) return fail(BRAMHA_ERR_NOT_FOUND, "weight '%s' was evicted", w->key.c_str());
    if (fmt) *fmt = w->fmt;
    if (N) *N = w->N;
    if (K) *K = w->K;
    if (device_bytes) *device_bytes = w->bytes;
    return BRAMHA_OK;
}

int bramha_cuda_gemv(bramha_ctx* ctx, const bramha_weight* w, const float* x_host, int64_t batch, float* y_host) {
    int rc = check_weight(ctx, w);
    if (rc) return rc;
    return gemv_host(ctx, w, x_host, batch, y_host);
}

int bramha_cuda_gemv_dev(bramha_ctx* ctx, const bramha_weight* w, const float* x_dev, int64_t batch, float* y_dev,
                         void* stream) {
    const bramha_weight* ws[1] = {w};
    float* ys[1] = {y_dev};
    return bramha_cuda_gemv_multi_dev(ctx, 1, ws, x_dev, batch, ys, stream);
}

int bramha_cuda_gemv_multi_dev(bramha_ctx* ctx, int n_weights, const bramha_weight* const* ws, const float* x_dev,
                               int64_t batch, float* const* y_devs, void* stream) {
    if (!ctx || !ws || !y_devs) return fail(BRAMHA_ERR_INVALID, "null argument");
    if (n_weights < 1 || n_weights > kMaxSegments)
        return fail(BRAMHA_ERR_INVALID, "n_weights must be in 1..%d", kMaxSegments);
    if (batch < 0) return fail(BRAMHA_ERR_INVALID, "negative batch");
    for (int i = 0; i < n_weights; ++i) {
        int rc = check_weight(ctx, ws[i]);
        if (rc) return rc;
        if (ws[i]->fmt != ws[0]->fmt || ws[i]->K != ws[0]->K)
            return fail(BRAMHA_ERR_SIZE, "fused weights must share format and K");
        if (!y_devs[i] && ws[i]->N > 0 && batch > 0) return fail(BRAMHA_ERR_INVALID, "null output pointer");
    }
    const int64_t K = ws[0]->K;
    if (batch > 0 && K > 0) {
        if (!x_dev) return fail(BRAMHA_ERR_INVALID, "null input pointer");
        if ((reinterpret_cast<uintptr_t>(x_dev) & 15) != 0 || (batch > 1 && (K & 3) != 0))
            return fail(BRAMHA_ERR_INVALID,
                        "x_dev must be 16-byte aligned (and K a multiple of 4 when batch > 1); "
                        "use bramha_cuda_gemv for unaligned input");
    }
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    return gemv_device(ctx, n_weights, ws, x_dev, K, batch, y_devs, st);
}

namespace {
// Checks one op of a GEMV chain (the rules of gemv_multi_dev / gemv_swiglu_dev);
// on the device path x and x_up must be 16-byte aligned.
int check_chain_op(bramha_ctx* ctx, const bramha_gemv_op& op, int64_t batch, bool device_ptrs) {
    if (op.n_weights < 1 || op.n_weights > kMaxSegments || !op.weights || !op.y)
        return fail(BRAMHA_ERR_INVALID, "gemv chain: an op needs 1..%d weights and outputs", kMaxSegments);
    for (int i = 0; i < op.n_weights; ++i) {
        int rc = check_weight(ctx, op.weights[i]);
        if (rc) return rc;
        if (op.weights[i]->fmt != op.weights[0]->fmt || op.weights[i]->K != op.weights[0]->K)
            return fail(BRAMHA_ERR_SIZE, "fused weights must share format and K");
        if (!op.y[i] && op.weights[i]->N > 0 && batch > 0) return fail(BRAMHA_ERR_INVALID, "null output pointer");
    }
    const int64_t K = op.weights[0]->K;
    if (op.x_up && !is_tiled(op.weights[0]->fmt))
        return fail(BRAMHA_ERR_UNSUPPORTED, "gemv chain: SwiGLU ops take LOG4, W4ZP8 or W8 weights");
    if (batch > 0 && K > 0) {
        if (!op.x) return fail(BRAMHA_ERR_INVALID, "null input pointer");
        if (device_ptrs && (((reinterpret_cast<uintptr_t>(op.x) | reinterpret_cast<uintptr_t>(op.x_up)) & 15) != 0 ||
                            (batch > 1 && (K & 3) != 0)))
            return fail(BRAMHA_ERR_INVALID,
                        "gemv chain: x must be 16-byte aligned (and K a multiple of 4 when batch > 1); "
                        "use bramha_cuda_gemv_chain for unaligned input");
    }
    return BRAMHA_OK;
}

// Launches ops [i0, i1) of an n_ops chain in order; each launch requests the
// next op's weights into L2 (also across i1 when i1 < n_ops).  xs / ups / ldxs /
// ys override the ops' pointers (device staging of the host chain).
int chain_range(bramha_ctx* ctx, int i0, int i1, int n_ops, const bramha_gemv_op* ops, int64_t batch,
                cudaStream_t st, const float* const* xs = nullptr, const float* const* ups = nullptr,
                const int64_t* ldxs = nullptr, float* const* const* ys = nullptr) {
    for (int i = i0; i < i1; ++i) {
        const bramha_gemv_op& op = ops[i];
        const int nn = i + 1 < n_ops ? ops[i + 1].n_weights : 0;
        const bramha_weight* const* nw = i + 1 < n_ops ? ops[i + 1].weights : nullptr;
        const float* x = xs ? xs[i] : op.x;
        const float* up = ups ? ups[i] : op.x_up;
        const int64_t ldx = ldxs ? ldxs[i] : op.weights[0]->K;
        int rc = gemv_device(ctx, op.n_weights, op.weights, x, ldx, batch, ys ? ys[i] : op.y, st, up, nn, nw);
        if (rc) return rc;
    }
    return BRAMHA_OK;
}

int chain_device(bramha_ctx* ctx, int n_ops, const bramha_gemv_op* ops, int64_t batch, cudaStream_t st,
                 const float* const* xs = nullptr, const float* const* ups = nullptr, const int64_t* ldxs = nullptr,
                 float* const* const* ys = nullptr) {
    return chain_range(ctx, 0, n_ops, n_ops, ops, batch, st, xs, ups, ldxs, ys);
}
}  // namespace

int bramha_cuda_gemv_chain_dev(bramha_ctx* ctx, int n_ops, const bramha_gemv_op* ops, int64_t batch, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (n_ops < 0 || (n_ops > 0 && !ops)) return fail(BRAMHA_ERR_INVALID, "gemv chain: bad op list");
    if (batch < 0) return fail(BRAMHA_ERR_INVALID, "negative batch");
    for (int i = 0; i < n_ops; ++i) {
        int rc = check_chain_op(ctx, ops[i], batch, true);
        if (rc) return rc;
    }
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    return chain_device(ctx, n_ops, ops, batch, st);
}

namespace {
// Device staging of a host-buffer chain: every op's x (and x_up) at a 16-byte
// aligned pitch, then every output, back to back (outputs of sharded ops --
// every rank's rows -- are staged at the top of the shard arena, where the
// other ranks' GEMVs can store theirs).
struct ChainLayout {
    std::vector<int64_t> ldx, xo, uo, yo;
    std::vector<char> in_arena_y;
    std::vector<size_t> y0;  // index of each op's first output in yo
    size_t xe = 0, ye = 0, ya = 0;
    bool any_shard = false;
};

ChainLayout chain_layout(int n_ops, const bramha_gemv_op* ops, int64_t batch) {
    ChainLayout L;
    L.ldx.resize((size_t)n_ops);
    L.xo.resize((size_t)n_ops);
    L.uo.resize((size_t)n_ops);
    L.y0.assign((size_t)n_ops + 1, 0);
    for (int i = 0; i < n_ops; ++i) {
        const int64_t K = ops[i].weights[0]->K;
        L.ldx[(size_t)i] = (K + 3) / 4 * 4;
        L.xo[(size_t)i] = (int64_t)L.xe;
        L.xe += (size_t)(L.ldx[(size_t)i] * batch);
        L.uo[(size_t)i] = ops[i].x_up ? (int64_t)L.xe : -1;
        if (ops[i].x_up) L.xe += (size_t)(L.ldx[(size_t)i] * batch);
        for (int j = 0; j < ops[i].n_weights; ++j) {
            const bramha_weight* w = ops[i].weights[j];
            if (w->shard) {
                L.any_shard = true;
                L.yo.push_back((int64_t)L.ya);
                L.ya += (size_t)(w->n_full * batch);
            } else {
                L.yo.push_back((int64_t)L.ye);
                L.ye += (size_t)(w->N * batch);
            }
            L.in_arena_y.push_back(w->shard ? 1 : 0);
        }
        L.y0[(size_t)i + 1] = L.y0[(size_t)i] + (size_t)ops[i].n_weights;
    }
    return L;
}

// Boundaries of the copy blocks of an n-op host chain: 1, 2, 4, 8, 16, ..., 16,
// 8, 4, 2, 1 ops (short blocks at both ends: the first launch waits only for
// its own inputs, the last outputs start back as soon as their launch is done).
std::vector<int> chain_blocks(int n_ops) {
    std::vector<int> head, tail;
    for (int lo = 0, hi = n_ops, size = 1; lo < hi; size = size < 16 ? size * 2 : 16) {
        int t = std::min(size, hi - lo);
        head.push_back(t);
        lo += t;
        if (lo >= hi) break;
        t = std::min(size, hi - lo);
        tail.push_back(t);
        hi -= t;
    }
    std::vector<int> bs{0};
    for (int t : head) bs.push_back(bs.back() + t);
    for (auto it = tail.rbegin(); it != tail.rend(); ++it) bs.push_back(bs.back() + *it);
    return bs;
}

// Enqueues a host-buffer chain staged in dev_x / dev_y (arena_y for sharded
// outputs): inputs in, the launches, outputs out, on the context's stream (and,
// unsharded, its two copy streams, joined back into the stream at the end).
// No wait; capturable into a CUDA graph when unsharded.
int host_chain_enqueue(bramha_ctx* ctx, int n_ops, const bramha_gemv_op* ops, int64_t batch, const ChainLayout& lay,
                       float* dev_x, float* dev_y, float* arena_y) {
    cudaStream_t st = ctx->stream;
    std::vector<const float*> xs((size_t)n_ops), ups((size_t)n_ops, nullptr);
    std::vector<std::vector<float*>> yv((size_t)n_ops);
    std::vector<float* const*> ys((size_t)n_ops);
    size_t yi = 0;
    for (int i = 0; i < n_ops; ++i) {
        xs[(size_t)i] = dev_x + lay.xo[(size_t)i];
        if (ops[i].x_up) ups[(size_t)i] = dev_x + lay.uo[(size_t)i];
        for (int j = 0; j < ops[i].n_weights; ++j, ++yi)
            yv[(size_t)i].push_back((lay.in_arena_y[yi] ? arena_y : dev_y) + lay.yo[yi]);
        ys[(size_t)i] = yv[(size_t)i].data();
    }
    auto h2d = [&](int i, cudaStream_t cs) -> int {  // op i's inputs
        const int64_t K = ops[i].weights[0]->K;
        if (K <= 0) return BRAMHA_OK;
        const size_t pitch = (size_t)lay.ldx[(size_t)i] * sizeof(float), row = (size_t)K * sizeof(float);
        CK(cudaMemcpy2DAsync(const_cast<float*>(xs[(size_t)i]), pitch, ops[i].x, row, row, (size_t)batch,
                             cudaMemcpyHostToDevice, cs),
           "H2D x");
        if (ops[i].x_up)
            CK(cudaMemcpy2DAsync(const_cast<float*>(ups[(size_t)i]), pitch, ops[i].x_up, row, row, (size_t)batch,
                                 cudaMemcpyHostToDevice, cs),
               "H2D x_up");
        return BRAMHA_OK;
    };
    auto d2h = [&](int i, cudaStream_t cs) -> int {  // op i's outputs
        for (int j = 0; j < ops[i].n_weights; ++j) {
            const size_t k = lay.y0[(size_t)i] + (size_t)j;
            const bramha_weight* w = ops[i].weights[j];
            const size_t n = (size_t)((w->shard ? w->n_full : w->N) * batch);
            if (n > 0)
                CK(cudaMemcpyAsync(ops[i].y[j], (lay.in_arena_y[k] ? arena_y : dev_y) + lay.yo[k], n * sizeof(float),
                                   cudaMemcpyDeviceToHost, cs),
                   "D2H y");
        }
        return BRAMHA_OK;
    };
    int rc = BRAMHA_OK;
    if (lay.any_shard) {  // every copy on the chain's stream; outputs after every rank's rows landed
        for (int i = 0; i < n_ops; ++i)
            if ((rc = h2d(i, st))) return rc;
        rc = chain_device(ctx, n_ops, ops, batch, st, xs.data(), ups.data(), lay.ldx.data(), ys.data());
        if (rc) return rc;
        CK(launch_shard_signal(shard_args(ctx), ctx->d_err, 0, st), "shard sync launch");
        for (int i = 0; i < n_ops; ++i)
            if ((rc = d2h(i, st))) return rc;
        return BRAMHA_OK;
    }
    // Copies overlap the launches: ops in blocks of 1, 2, 4, 8, 16, ..., 16, 8,
    // 4, 2, 1 (short blocks at both ends: the first launch waits only for its
    // own inputs, the last outputs start back as soon as their launch is done);
    // block k's inputs go in on copy_in (one block ahead of the launches), its
    // launches wait for them, and its outputs come back on copy_out while the
    // later blocks run.
    const std::vector<int> bs = chain_blocks(n_ops);
    const int nb = (int)bs.size() - 1;
    if ((rc = ensure_copy_streams(ctx, (size_t)(2 * nb + 2)))) return rc;
    cudaEvent_t* ev = ctx->events.data();  // [0] start, [1] outputs copied, [2 + k] block k in, [2 + nb + k] done
    auto overlapped = [&]() -> int {
        CK(cudaEventRecord(ev[0], st), "event record");
        CK(cudaStreamWaitEvent(ctx->copy_in, ev[0], 0), "stream wait");
        CK(cudaStreamWaitEvent(ctx->copy_out, ev[0], 0), "stream wait");
        auto in_block = [&](int k) -> int {
            for (int i = bs[(size_t)k]; i < bs[(size_t)k + 1]; ++i)
                if (int r = h2d(i, ctx->copy_in)) return r;
            CK(cudaEventRecord(ev[2 + k], ctx->copy_in), "event record");
            return BRAMHA_OK;
        };
        if (int r = in_block(0)) return r;
        for (int k = 0; k < nb; ++k) {
            if (k + 1 < nb)
                if (int r = in_block(k + 1)) return r;
            CK(cudaStreamWaitEvent(st, ev[2 + k], 0), "stream wait");
            if (int r = chain_range(ctx, bs[(size_t)k], bs[(size_t)k + 1], n_ops, ops, batch, st, xs.data(), ups.data(),
                                    lay.ldx.data(), ys.data()))
                return r;
            CK(cudaEventRecord(ev[2 + nb + k], st), "event record");
        }
        for (int k = 0; k < nb; ++k) {
            CK(cudaStreamWaitEvent(ctx->copy_out, ev[2 + nb + k], 0), "stream wait");
            for (int i = bs[(size_t)k]; i < bs[(size_t)k + 1]; ++i)
                if (int r = d2h(i, ctx->copy_out)) return r;
        }
        CK(cudaEventRecord(ev[1], ctx->copy_out), "event record");
        CK(cudaStreamWaitEvent(st, ev[1], 0), "stream wait");
        return BRAMHA_OK;
    };
    return overlapped();
}

// After a failed enqueue: nothing may still read or write the caller's buffers.
void host_chain_drain(bramha_ctx* ctx) {
    if (ctx->copy_in) cudaStreamSynchronize(ctx->copy_in);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->copy_out) cudaStreamSynchronize(ctx->copy_out);
}
}  // namespace

int bramha_cuda_gemv_chain(bramha_ctx* ctx, int n_ops, const bramha_gemv_op* ops, int64_t batch) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (n_ops < 0 || (n_ops > 0 && !ops)) return fail(BRAMHA_ERR_INVALID, "gemv chain: bad op list");
    if (batch < 0) return fail(BRAMHA_ERR_INVALID, "negative batch");
    for (int i = 0; i < n_ops; ++i) {
        int rc = check_chain_op(ctx, ops[i], batch, false);
        if (rc) return rc;
    }
    if (n_ops == 0 || batch == 0) return BRAMHA_OK;
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->io_mu);
    const ChainLayout lay = chain_layout(n_ops, ops, batch);
    int rc = ensure_staging(ctx, lay.xe, lay.ye > 0 ? lay.ye : 1);
    if (rc) return rc;
    float* arena_y = nullptr;
    if (lay.any_shard) {
        if (!ctx->arena || ctx->shard_world < 2) return fail(BRAMHA_ERR_INVALID, "sharded weights need a shard group");
        const size_t need = (lay.ya * sizeof(float) + 255) / 256 * 256;
        if (need > ctx->arena_bytes - ctx->arena_used)
            return fail(BRAMHA_ERR_OOM, "shard arena too small to stage this chain's outputs (%zu bytes)", need);
        if (ctx->arena_bytes - need < ctx->arena_top) ctx->arena_top = ctx->arena_bytes - need;
        arena_y = reinterpret_cast<float*>(ctx->arena + (ctx->arena_bytes - need));
    }
    rc = host_chain_enqueue(ctx, n_ops, ops, batch, lay, ctx->dev_x, ctx->dev_y, arena_y);
    if (rc) {
        host_chain_drain(ctx);
        return rc;
    }
    return check_device_error(ctx, ctx->stream);
}

struct bramha_host_chain {
    int n_ops = 0;
    int64_t batch = 0;
    std::vector<std::vector<const bramha_weight*>> w;
    std::vector<std::vector<float*>> y;
    std::vector<bramha_gemv_op> ops;  // views of w / y and the caller's x, x_up
    ChainLayout lay;
    float* dev_x = nullptr;           // the chain's own staging
    float* dev_y = nullptr;
    cudaGraphExec_t exec = nullptr;   // null: launched eagerly every run
};

namespace {
bool is_pinned(const void* p) {
    if (!p) return true;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

void host_chain_free(bramha_host_chain* c) {
    if (c->exec) cudaGraphExecDestroy(c->exec);
    if (c->dev_x) cudaFree(c->dev_x);
    if (c->dev_y) cudaFree(c->dev_y);
    delete c;
}
}  // namespace

int bramha_cuda_host_chain_create(bramha_ctx* ctx, int n_ops, const bramha_gemv_op* ops, int64_t batch,
                                  bramha_host_chain** out) {
    if (!ctx || !out) return fail(BRAMHA_ERR_INVALID, "null argument");
    *out = nullptr;
    if (n_ops < 1 || !ops) return fail(BRAMHA_ERR_INVALID, "host chain: needs at least one op");
    if (batch < 1) return fail(BRAMHA_ERR_INVALID, "host chain: batch must be at least 1");
    for (int i = 0; i < n_ops; ++i) {
        int rc = check_chain_op(ctx, ops[i], batch, false);
        if (rc) return rc;
    }
    bramha_host_chain* c = new (std::nothrow) bramha_host_chain();
    if (!c) return fail(BRAMHA_ERR_OOM, "host allocation failed");
    c->n_ops = n_ops;
    c->batch = batch;
    c->w.resize((size_t)n_ops);
    c->y.resize((size_t)n_ops);
    c->ops.resize((size_t)n_ops);
    bool pinned = true;
    for (int i = 0; i < n_ops; ++i) {
        const bramha_gemv_op& op = ops[i];
        c->w[(size_t)i].assign(op.weights, op.weights + op.n_weights);
        c->y[(size_t)i].assign(op.y, op.y + op.n_weights);
        c->ops[(size_t)i] = bramha_gemv_op{op.n_weights, c->w[(size_t)i].data(), op.x, op.x_up, c->y[(size_t)i].data()};
        pinned = pinned && is_pinned(op.x) && is_pinned(op.x_up);
        for (int j = 0; j < op.n_weights; ++j) pinned = pinned && is_pinned(op.y[j]);
    }
    c->lay = chain_layout(n_ops, c->ops.data(), batch);
    if (c->lay.any_shard) {  // staged in the shard arena by each run's bramha_cuda_gemv_chain
        *out = c;
        return BRAMHA_OK;
    }
    DeviceGuard g(ctx->device);
    cudaError_t e = cudaMalloc(&c->dev_x, sizeof(float) * std::max<size_t>(c->lay.xe, 1));
    if (e == cudaSuccess) e = cudaMalloc(&c->dev_y, sizeof(float) * std::max<size_t>(c->lay.ye, 1));
    if (e != cudaSuccess) {
        host_chain_free(c);
        return cuda_fail(e, "cudaMalloc(host chain staging)");
    }
    if (pinned) {  // one CUDA graph of the copies and launches; on any failure, eager runs
        std::lock_guard<std::mutex> lk(ctx->io_mu);
        const size_t nb = chain_blocks(n_ops).size() - 1;
        if (ensure_copy_streams(ctx, 2 * nb + 2) == BRAMHA_OK &&
            cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int rc = host_chain_enqueue(ctx, n_ops, c->ops.data(), batch, c->lay, c->dev_x, c->dev_y, nullptr);
            cudaGraph_t graph = nullptr;
            const cudaError_t ee = cudaStreamEndCapture(ctx->stream, &graph);
            if (rc == BRAMHA_OK && ee == cudaSuccess && graph &&
                cudaGraphInstantiate(&c->exec, graph, 0) != cudaSuccess)
                c->exec = nullptr;
            if (graph) cudaGraphDestroy(graph);
        }
        cudaGetLastError();
        g_last_error.clear();
    }
    *out = c;
    return BRAMHA_OK;
}

int bramha_cuda_host_chain_uses_graph(bramha_ctx* ctx, const bramha_host_chain* chain, int* out) {
    if (!ctx || !chain || !out) return fail(BRAMHA_ERR_INVALID, "null argument");
    *out = chain->exec ? 1 : 0;
    return BRAMHA_OK;
}

int bramha_cuda_host_chain_run(bramha_ctx* ctx, bramha_host_chain* c) {
    if (!ctx || !c) return fail(BRAMHA_ERR_INVALID, "null argument");
    if (c->lay.any_shard) return bramha_cuda_gemv_chain(ctx, c->n_ops, c->ops.data(), c->batch);
    for (int i = 0; i < c->n_ops; ++i) {  // every weight still registered
        int rc = check_chain_op(ctx, c->ops[(size_t)i], c->batch, false);
        if (rc) return rc;
    }
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->io_mu);
    if (c->exec) {
        CK(cudaGraphLaunch(c->exec, ctx->stream), "cudaGraphLaunch(host chain)");
    } else {
        const int rc = host_chain_enqueue(ctx, c->n_ops, c->ops.data(), c->batch, c->lay, c->dev_x, c->dev_y, nullptr);
        if (rc) {
            host_chain_drain(ctx);
            return rc;
        }
    }
    return check_device_error(ctx, ctx->stream);
}

int bramha_cuda_host_chain_destroy(bramha_ctx* ctx, bramha_host_chain* c) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (!c) return BRAMHA_OK;
    DeviceGuard g(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    host_chain_free(c);
    return BRAMHA_OK;
}

struct bramha_gemv_program {
    bramha_ctx* ctx = nullptr;
    ChainProgram* prog = nullptr;
};

int bramha_cuda_gemv_program_create(bramha_ctx* ctx, int n_ops, const bramha_gemv_op* ops, int64_t batch,
                                    bramha_gemv_program** out) {
    if (!ctx || !out) return fail(BRAMHA_ERR_INVALID, "null argument");
    *out = nullptr;
    if (n_ops < 1 || !ops) return fail(BRAMHA_ERR_INVALID, "gemv program: needs at least one op");
    if (batch < 1 || batch > kMaxGemvBatch)
        return fail(BRAMHA_ERR_UNSUPPORTED, "gemv program: batch must be in 1..%d", kMaxGemvBatch);
    const int fmt = ops[0].n_weights > 0 && ops[0].weights && ops[0].weights[0] ? ops[0].weights[0]->fmt : -1;
    std::vector<GemvArgs> args((size_t)n_ops);
    for (int i = 0; i < n_ops; ++i) {
        const bramha_gemv_op& op = ops[i];
        int rc = check_chain_op(ctx, op, batch, true);
        if (rc) return rc;
        const int64_t K = op.weights[0]->K;
        if (op.weights[0]->fmt != fmt || !is_tiled(fmt))
            return fail(BRAMHA_ERR_UNSUPPORTED, "gemv program: every op must use the same one of LOG4, W4ZP8, W8");
        if (held_columns(fmt, K) <= 0 || K > 0x7fffffffLL)
            return fail(BRAMHA_ERR_UNSUPPORTED, "gemv program: op %d has no input columns", i);
        GemvArgs& a = args[(size_t)i];
        a = GemvArgs{};
        a.x = op.x;
        a.x_up = op.x_up;
        a.ldx = K;
        a.K = (int)held_columns(fmt, K);
        a.batch = (int)batch;
        for (int j = 0; j < op.n_weights; ++j) {
            const bramha_weight* w = op.weights[j];
            if (w->shard) return fail(BRAMHA_ERR_UNSUPPORTED, "gemv program: sharded weights are not supported");
            if (w->N <= 0 || w->N > 0x7fffffffLL)
                return fail(BRAMHA_ERR_UNSUPPORTED, "gemv program: op %d weight %d has no rows", i, j);
            GemvSeg& g = a.seg[a.nseg++];
            g.q = w->q;
            g.scales = w->scales;
            g.y = op.y[j];
            g.ldy = w->N;
            g.N = (int)w->N;
        }
    }
    bramha_gemv_program* p = new (std::nothrow) bramha_gemv_program();
    if (!p) return fail(BRAMHA_ERR_OOM, "host allocation failed");
    DeviceGuard g(ctx->device);
    cudaError_t e = chain_program_create(fmt, (int)batch, n_ops, args.data(), ctx->num_sms, ctx->split_cost,
                                         ctx->split_ws, kSplitWsFloats, ctx->split_tickets, kSplitTickets, &p->prog);
    if (e != cudaSuccess) {
        delete p;
        return cuda_fail(e, "gemv program create");
    }
    p->ctx = ctx;
    *out = p;
    return BRAMHA_OK;
}

int bramha_cuda_gemv_program_run_dev(bramha_ctx* ctx, bramha_gemv_program* prog, void* stream) {
    if (!ctx || !prog || prog->ctx != ctx) return fail(BRAMHA_ERR_INVALID, "null program or another context's");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    CK(chain_program_run(prog->prog, ctx->d_err, ctx->prog_lookahead, st), "gemv program launch");
    return BRAMHA_OK;
}

int bramha_cuda_gemv_program_trace(bramha_ctx* ctx, bramha_gemv_program* prog, int on) {
    if (!ctx || !prog || prog->ctx != ctx) return fail(BRAMHA_ERR_INVALID, "null program or another context's");
    DeviceGuard g(ctx->device);
    CK(chain_program_trace(prog->prog, on), "gemv program trace");
    return BRAMHA_OK;
}

int bramha_cuda_gemv_program_read_trace(bramha_ctx* ctx, bramha_gemv_program* prog, uint64_t* out, size_t n,
                                        int* grid) {
    if (!ctx || !prog || prog->ctx != ctx || !out || !grid) return fail(BRAMHA_ERR_INVALID, "null argument");
    DeviceGuard g(ctx->device);
    CK(chain_program_read_trace(prog->prog, reinterpret_cast<unsigned long long*>(out), n, grid),
       "gemv program trace (is tracing on?)");
    return BRAMHA_OK;
}

int bramha_cuda_gemv_program_destroy(bramha_ctx* ctx, bramha_gemv_program* prog) {
    if (!ctx || !prog || prog->ctx != ctx) return fail(BRAMHA_ERR_INVALID, "null program or another context's");
    DeviceGuard g(ctx->device);
    cudaDeviceSynchronize();  // no run may still use its tables
    chain_program_destroy(prog->prog);
    delete prog;
    return BRAMHA_OK;
}

int bramha_cuda_gemv_swiglu_dev(bramha_ctx* ctx, const bramha_weight* w, const float* gate_dev, const float* up_dev,
                                int64_t batch, float* y_dev, void* stream) {
    int rc = check_weight(ctx, w);
    if (rc) return rc;
    if (!is_tiled(w->fmt))
        return fail(BRAMHA_ERR_UNSUPPORTED, "gemv_swiglu_dev: %s weights are not supported (LOG4, W4ZP8, W8 only)",
                    fmt_name(w->fmt));
    if (batch < 0) return fail(BRAMHA_ERR_INVALID, "negative batch");
    if (batch > 0 && w->K > 0) {
        if (!gate_dev || !up_dev) return fail(BRAMHA_ERR_INVALID, "null input pointer");
        if (((reinterpret_cast<uintptr_t>(gate_dev) | reinterpret_cast<uintptr_t>(up_dev)) & 15) != 0 ||
            (batch > 1 && (w->K & 3) != 0))
            return fail(BRAMHA_ERR_INVALID, "gate_dev / up_dev must be 16-byte aligned (and K a multiple of 4 when batch > 1)");
    }
    if (!y_dev && w->N > 0 && batch > 0) return fail(BRAMHA_ERR_INVALID, "null output pointer");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    const bramha_weight* ws[1] = {w};
    float* ys[1] = {y_dev};
    return gemv_device(ctx, 1, ws, gate_dev, w->K, batch, ys, st, up_dev);
}

namespace {
bool overlaps(const float* a, const float* b, int64_t n) {
    return a && b && a < b + n && b < a + n;
}
// The CUDA-core GEMV takes this launch (so it can form the RMSNorm itself).
bool norm_fusable(bramha_ctx* ctx, int n, const bramha_weight* const* ws) {
    const int fmt = ws[0]->fmt;
    const int64_t K = ws[0]->K;
    if (!is_tiled(fmt) || ctx->gemv_kernel == BRAMHA_GEMV_TENSOR_CORE || held_columns(fmt, K) != K || K > 1024)
        return false;  // (the fused kernel keeps the whole residual, <= 1024 columns, in shared memory)
    GemvArgs a{};
    a.batch = 1;
    a.K = (int)K;
    for (int i = 0; i < n; ++i)
        if (ws[i]->N > 0) {
            if (ws[i]->N > 0x7fffffffLL) return false;
            a.seg[a.nseg++].N = (int)ws[i]->N;
        }
    if (a.nseg == 0) return false;
    if (ctx->gemv_kernel == BRAMHA_GEMV_CUDA_CORE) return true;
    a.split_ws = ctx->split_ws;
    a.split_ws_floats = kSplitWsFloats;
    a.split_tickets = ctx->split_tickets;
    a.split_tickets_n = kSplitTickets;
    return gemv_cc_eligible(fmt, a);
}
}  // namespace

int bramha_cuda_gemv_rmsnorm_dev(bramha_ctx* ctx, int n_weights, const bramha_weight* const* ws, const float* x_dev,
                                 const float* delta_dev, const float* norm_w_dev, float eps, float* x_out_dev,
                                 float* const* y_devs, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (n_weights < 1 || n_weights > kMaxSegments)
        return fail(BRAMHA_ERR_INVALID, "gemv_rmsnorm_dev: 1..%d weights (got %d)", kMaxSegments, n_weights);
    if (!ws || !y_devs) return fail(BRAMHA_ERR_INVALID, "null argument");
    for (int i = 0; i < n_weights; ++i) {
        int rc = check_weight(ctx, ws[i]);
        if (rc) return rc;
        if (ws[i]->fmt != ws[0]->fmt || ws[i]->K != ws[0]->K)
            return fail(BRAMHA_ERR_INVALID, "gemv_rmsnorm_dev: every weight must have the same format and K");
        if (ws[i]->shard) return fail(BRAMHA_ERR_UNSUPPORTED, "gemv_rmsnorm_dev: sharded weights are not supported");
        if (ws[i]->N > 0 && !y_devs[i]) return fail(BRAMHA_ERR_INVALID, "null output pointer");
    }
    const int64_t K = ws[0]->K;
    if (K <= 0 || K > (1 << 24)) return fail(BRAMHA_ERR_INVALID, "gemv_rmsnorm_dev: K = %lld out of range", (long long)K);
    if (!x_dev || !norm_w_dev) return fail(BRAMHA_ERR_INVALID, "null device pointer");
    if (overlaps(x_out_dev, x_dev, K) || overlaps(x_out_dev, delta_dev, K))
        return fail(BRAMHA_ERR_INVALID, "gemv_rmsnorm_dev: x_out_dev must not overlap x_dev or delta_dev");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    if (norm_fusable(ctx, n_weights, ws)) {
        const NormIn nin = {norm_w_dev, delta_dev, x_out_dev, eps};
        return gemv_device(ctx, n_weights, ws, x_dev, K, 1, y_devs, st, nullptr, 0, nullptr, &nin);
    }
    // Otherwise the RMSNorm kernel, then the GEMV (the same values, two launches):
    // r and the normalised activations in stream-ordered scratch.
    const int64_t kp = (K + 3) & ~int64_t(3);
    float* tmp = nullptr;
    CK(cudaMallocAsync(reinterpret_cast<void**>(&tmp), sizeof(float) * (size_t)(2 * kp), st),
       "cudaMallocAsync(rmsnorm scratch)");
    float* h = tmp;
    float* r = x_out_dev ? x_out_dev : tmp + kp;
    cudaError_t e = cudaMemcpyAsync(r, x_dev, sizeof(float) * (size_t)K, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = launch_rmsnorm(r, delta_dev, norm_w_dev, K, eps, h, st);
    int rc = e == cudaSuccess ? gemv_device(ctx, n_weights, ws, h, K, 1, y_devs, st) : cuda_fail(e, "rmsnorm launch");
    cudaError_t e2 = cudaFreeAsync(tmp, st);
    if (rc == BRAMHA_OK && e2 != cudaSuccess) rc = cuda_fail(e2, "cudaFreeAsync(rmsnorm scratch)");
    return rc;
}

int bramha_cuda_matvec(bramha_ctx* ctx, int fmt, const float* h, int64_t K, const void* q_weight, size_t q_bytes,
                       const float* scales, size_t n_scales, int64_t N, const char* model_name,
                       const char* layer_name, float* out) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (!valid_fmt(fmt)) return fail(BRAMHA_ERR_INVALID, "unknown weight format %d", fmt);
    if (N < 0 || K < 0) return fail(BRAMHA_ERR_INVALID, "negative shape");
    if (N > 0 && !out) return fail(BRAMHA_ERR_INVALID, "null output pointer");
    // wgpu_backend.rs:1092-1095: an empty input or output gives zeros.
    if (K == 0 || N == 0) {
        if (N > 0) memset(out, 0, sizeof(float) * (size_t)N);
        return BRAMHA_OK;
    }
    int rc = check_sizes(fmt, N, K, q_bytes, n_scales, scales != nullptr);
    if (rc) return rc;
    if (model_name && layer_name) {
        std::string key = std::string(model_name) + ":" + layer_name;
        bramha_weight* w = nullptr;
        rc = register_impl(ctx, key.c_str(), fmt, N, K, q_weight, q_bytes, scales, n_scales, false, nullptr, &w);
        if (rc) return rc;
        return gemv_host(ctx, w, h, 1, out);
    }
    // Temporary buffers for this call only (wgpu_backend.rs:1118-1171).
    DeviceGuard g(ctx->device);
    bramha_weight tmp;
    tmp.fmt = fmt;
    tmp.N = N;
    tmp.K = K;
    tmp.ctx = ctx;
    tmp.key = "<temporary>";
    rc = upload(ctx, &tmp, q_weight, scales, false, ctx->stream);
    if (rc) return rc;
    rc = gemv_host(ctx, &tmp, h, 1, out);
    free_weight_memory(&tmp);
    return rc;
}

// ---- 2:4 structured-sparse GEMV --------------------------------------------
namespace {
int register_sparse24_impl(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K, const void* q,
                           size_t q_bytes, const float* scales, size_t n_scales, bool from_device, cudaStream_t st,
                           bramha_weight** out) {
    if (!ctx || !out) return fail(BRAMHA_ERR_INVALID, "null context or output pointer");
    if (!key) return fail(BRAMHA_ERR_INVALID, "null weight key");
    int rc = sp24_check_pruned(fmt, N, K, q_bytes, n_scales, scales != nullptr);
    if (rc) return rc;
    if (!q && q_bytes > 0) return fail(BRAMHA_ERR_INVALID, "weight pointer is NULL");
    const int sfmt = fmt - BRAMHA_FMT_F32 + BRAMHA_FMT_SP24_F32;
    return register_with(
        ctx, key, sfmt, N, K, sp24_bytes(fmt, N, K, nullptr, nullptr),
        [&](bramha_weight* w) { return sp24_fill_pruned(w, q, scales, from_device, st ? st : ctx->stream); }, out);
}

int register_sparse24_compressed_impl(bramha_ctx* ctx, const char* key, int64_t rows, int64_t cols,
                                      const uint16_t* masks, size_t n_masks, const float* values, size_t n_values,
                                      bramha_weight** out) {
    if (!ctx || !out) return fail(BRAMHA_ERR_INVALID, "null context or output pointer");
    if (!key) return fail(BRAMHA_ERR_INVALID, "null weight key");
    int rc = sp24_check_compressed(rows, cols, n_masks, masks, values, n_values);
    if (rc) return rc;
    {  // a cached key skips the host walk
        std::lock_guard<std::mutex> lk(ctx->mu);
        auto it = ctx->reg.find(key);
        if (it != ctx->reg.end()) {
            bramha_weight* w = it->second;
            if (w->fmt != BRAMHA_FMT_SP24_F32 || w->N != rows || w->K != cols)
                return fail(BRAMHA_ERR_SIZE, "key '%s' is registered with a different shape or format", key);
            touch_locked(ctx, w);
            *out = w;
            return BRAMHA_OK;
        }
    }
    std::vector<uint8_t> vals;
    std::vector<uint32_t> idx;
    rc = sp24_canonicalise(rows, cols, masks, values, n_values, vals, idx);
    if (rc) return rc;
    return register_with(
        ctx, key, BRAMHA_FMT_SP24_F32, rows, cols, sp24_bytes(BRAMHA_FMT_F32, rows, cols, nullptr, nullptr),
        [&](bramha_weight* w) { return sp24_fill_compressed(w, vals, idx, ctx->stream); }, out);
}
}  // namespace

int bramha_cuda_register_sparse24(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K, const void* q,
                                  size_t q_bytes, const float* scales, size_t n_scales, bramha_weight** out) {
    return register_sparse24_impl(ctx, key, fmt, N, K, q, q_bytes, scales, n_scales, false, nullptr, out);
}

int bramha_cuda_register_sparse24_dev(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K,
                                      const void* q_dev, size_t q_bytes, const float* scales_dev, size_t n_scales,
                                      void* stream, bramha_weight** out) {
    return register_sparse24_impl(ctx, key, fmt, N, K, q_dev, q_bytes, scales_dev, n_scales, true,
                                  static_cast<cudaStream_t>(stream), out);
}

int bramha_cuda_register_sparse24_compressed(bramha_ctx* ctx, const char* key, int64_t rows, int64_t cols,
                                             const uint16_t* masks, size_t n_masks, const float* values,
                                             size_t n_values, bramha_weight** out) {
    return register_sparse24_compressed_impl(ctx, key, rows, cols, masks, n_masks, values, n_values, out);
}

int bramha_cuda_sparse_matvec_2_4(bramha_ctx* ctx, int fmt, const float* h, int64_t K, const void* q_weight,
                                  size_t q_bytes, const float* scales, size_t n_scales, int64_t N,
                                  const char* model_name, const char* layer_name, float* out) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (N < 0 || K < 0) return fail(BRAMHA_ERR_INVALID, "negative shape");
    if (N > 0 && !out) return fail(BRAMHA_ERR_INVALID, "null output pointer");
    if (K == 0 || N == 0) {
        if (N > 0) memset(out, 0, sizeof(float) * (size_t)N);
        return BRAMHA_OK;
    }
    int rc = sp24_check_pruned(fmt, N, K, q_bytes, n_scales, scales != nullptr);
    if (rc) return rc;
    if (model_name && layer_name) {
        std::string key = std::string(model_name) + ":" + layer_name;
        bramha_weight* w = nullptr;
        rc = register_sparse24_impl(ctx, key.c_str(), fmt, N, K, q_weight, q_bytes, scales, n_scales, false, nullptr,
                                    &w);
        if (rc) return rc;
        return gemv_host(ctx, w, h, 1, out);
    }
    DeviceGuard g(ctx->device);
    bramha_weight tmp;
    tmp.fmt = fmt - BRAMHA_FMT_F32 + BRAMHA_FMT_SP24_F32;
    tmp.N = N;
    tmp.K = K;
    tmp.ctx = ctx;
    tmp.key = "<temporary>";
    rc = sp24_fill_pruned(&tmp, q_weight, scales, false, ctx->stream);
    if (rc) return rc;
    rc = gemv_host(ctx, &tmp, h, 1, out);
    free_weight_memory(&tmp);
    return rc;
}

int bramha_cuda_sparse_matvec_2_4_compressed(bramha_ctx* ctx, const float* x, int64_t cols, const uint16_t* masks,
                                             size_t n_masks, const float* values, size_t n_values, int64_t rows,
                                             const char* model_name, const char* layer_name, float* out) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (rows < 0 || cols < 0) return fail(BRAMHA_ERR_INVALID, "negative shape");
    if (rows > 0 && !out) return fail(BRAMHA_ERR_INVALID, "null output pointer");
    if (rows == 0 || cols < 4) {  // no whole group: every output is 0 (sparse.rs:107-135)
        if (rows > 0) memset(out, 0, sizeof(float) * (size_t)rows);
        return BRAMHA_OK;
    }
    int rc = sp24_check_compressed(rows, cols, n_masks, masks, values, n_values);
    if (rc) return rc;
    if (model_name && layer_name) {
        std::string key = std::string(model_name) + ":" + layer_name;
        bramha_weight* w = nullptr;
        rc = register_sparse24_compressed_impl(ctx, key.c_str(), rows, cols, masks, n_masks, values, n_values, &w);
        if (rc) return rc;
        return gemv_host(ctx, w, x, 1, out);
    }
    std::vector<uint8_t> vals;
    std::vector<uint32_t> idx;
    rc = sp24_canonicalise(rows, cols, masks, values, n_values, vals, idx);
    if (rc) return rc;
    DeviceGuard g(ctx->device);
    bramha_weight tmp;
    tmp.fmt = BRAMHA_FMT_SP24_F32;
    tmp.N = rows;
    tmp.K = cols;
    tmp.ctx = ctx;
    tmp.key = "<temporary>";
    rc = sp24_fill_compressed(&tmp, vals, idx, ctx->stream);
    if (rc) return rc;
    rc = gemv_host(ctx, &tmp, x, 1, out);
    free_weight_memory(&tmp);
    return rc;
}

// ---- MoE expert MLP ----------------------------------------------------------
namespace {
int moe_check(bramha_ctx* ctx, const bramha_weight* gu, const bramha_weight* dn, int E, int top_k, int64_t T,
              MoeWeights* mw) {
    int rc = check_weight(ctx, gu);
    if (rc) return rc;
    rc = check_weight(ctx, dn);
    if (rc) return rc;
    if (gu->fmt != dn->fmt || (gu->fmt != BRAMHA_FMT_LOG4 && gu->fmt != BRAMHA_FMT_W4ZP8 && gu->fmt != BRAMHA_FMT_W8))
        return fail(BRAMHA_ERR_UNSUPPORTED, "moe: gate_up and down must share one of LOG4, W4ZP8, W8");
    if (E <= 0 || E > kMoeMaxExperts) return fail(BRAMHA_ERR_INVALID, "moe: num_experts must be in 1..%lld",
                                                  (long long)kMoeMaxExperts);
    if (top_k <= 0 || T < 0) return fail(BRAMHA_ERR_INVALID, "moe: top_k must be positive and T non-negative");
    if (gu->N % E != 0 || dn->N % E != 0)
        return fail(BRAMHA_ERR_SIZE, "moe: stacked weights must hold num_experts equal blocks of rows");
    const int64_t two_i = gu->N / E, H = gu->K, I = two_i / 2;
    if (two_i % 128 != 0 || H % 128 != 0)
        return fail(BRAMHA_ERR_UNSUPPORTED, "moe: 2 * intermediate (%lld) and hidden (%lld) must be multiples of 128",
                    (long long)two_i, (long long)H);
    if (dn->N != E * H || dn->K != I)
        return fail(BRAMHA_ERR_SIZE, "moe: down is %lld x %lld, expected %lld x %lld", (long long)dn->N,
                    (long long)dn->K, (long long)(E * H), (long long)I);
    const int64_t k = top_k < E ? top_k : E;
    if (T * k > kMoeMaxAssignments)
        return fail(BRAMHA_ERR_UNSUPPORTED, "moe: T * top_k = %lld exceeds %lld per call; split the batch",
                    (long long)(T * k), (long long)kMoeMaxAssignments);
    *mw = MoeWeights{gu->fmt, gu->q, gu->scales, dn->q, dn->scales, E, H, I};
    return BRAMHA_OK;
}
}  // namespace

int bramha_cuda_moe_mlp_dev(bramha_ctx* ctx, const bramha_weight* gate_up, const bramha_weight* down,
                            int num_experts, int top_k, const float* x_dev, const float* logits_dev, int64_t T,
                            float* out_dev, int32_t* selected_dev, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    MoeWeights mw;
    int rc = moe_check(ctx, gate_up, down, num_experts, top_k, T, &mw);
    if (rc) return rc;
    if (T == 0) return BRAMHA_OK;
    if (!x_dev || !logits_dev || !out_dev) return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    CK(launch_moe_mlp(mw, top_k, x_dev, logits_dev, T, out_dev, selected_dev, ctx->d_err, st), "moe launch");
    return BRAMHA_OK;
}

int bramha_cuda_moe_route_dev(bramha_ctx* ctx, const float* logits_dev, int64_t T, int num_experts, int top_k,
                              int32_t* ids_dev, float* weights_dev, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (num_experts <= 0 || num_experts > kMoeMaxExperts || top_k <= 0 || T < 0)
        return fail(BRAMHA_ERR_INVALID, "moe_route: bad num_experts, top_k or T");
    if (T == 0) return BRAMHA_OK;
    if (!logits_dev || !ids_dev || !weights_dev) return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    CK(launch_moe_route(logits_dev, T, num_experts, top_k, ids_dev, weights_dev, st), "moe route launch");
    return BRAMHA_OK;
}

int bramha_cuda_moe_experts_dev(bramha_ctx* ctx, const bramha_weight* gate_up, const bramha_weight* down,
                                int num_experts, const float* x_dev, const int32_t* ids_dev, int64_t R, float* y_dev,
                                void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    MoeWeights mw;
    int rc = moe_check(ctx, gate_up, down, num_experts, 1, R, &mw);
    if (rc) return rc;
    if (R == 0) return BRAMHA_OK;
    if (!x_dev || !ids_dev || !y_dev) return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    CK(launch_moe_experts(mw, x_dev, ids_dev, R, y_dev, ctx->d_err, st), "moe experts launch");
    return BRAMHA_OK;
}

int bramha_cuda_moe_mlp(bramha_ctx* ctx, const bramha_weight* gate_up, const bramha_weight* down, int num_experts,
                        int top_k, const float* x_host, const float* logits_host, int64_t T, float* out_host,
                        int32_t* selected_host) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    MoeWeights mw;
    int rc = moe_check(ctx, gate_up, down, num_experts, top_k, T, &mw);
    if (rc) return rc;
    if (T == 0) return BRAMHA_OK;
    if (!x_host || !logits_host || !out_host) return fail(BRAMHA_ERR_INVALID, "null host buffer");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->io_mu);
    cudaStream_t st = ctx->stream;
    const int64_t k = top_k < num_experts ? top_k : num_experts;
    const size_t bx = (size_t)(T * mw.H) * 4, bl = (size_t)(T * num_experts) * 4, bs = (size_t)(T * k) * 4;
    uint8_t* buf = nullptr;
    CK(cudaMallocAsync(reinterpret_cast<void**>(&buf), 2 * bx + bl + bs, st), "moe staging");
    float* xd = reinterpret_cast<float*>(buf);
    float* od = reinterpret_cast<float*>(buf + bx);
    float* ld = reinterpret_cast<float*>(buf + 2 * bx);
    int32_t* sd = reinterpret_cast<int32_t*>(buf + 2 * bx + bl);
    cudaError_t e = cudaMemcpyAsync(xd, x_host, bx, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ld, logits_host, bl, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = launch_moe_mlp(mw, top_k, xd, ld, T, od, sd, ctx->d_err, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out_host, od, bx, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && selected_host) e = cudaMemcpyAsync(selected_host, sd, bs, cudaMemcpyDeviceToHost, st);
    cudaError_t e2 = cudaFreeAsync(buf, st);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) return cuda_fail(e, "moe (host buffers)");
    return check_device_error(ctx, st);
}

int bramha_cuda_gemm(bramha_ctx* ctx, const bramha_weight* w, const float* h_host, int64_t M, float* out_host) {
    int rc = check_weight(ctx, w);
    if (rc) return rc;
    if (M < 0) return fail(BRAMHA_ERR_INVALID, "negative block size");
    if (M == 0 || w->N == 0) return BRAMHA_OK;
    if (w->K == 0) {
        memset(out_host, 0, sizeof(float) * (size_t)(w->N * M));
        return BRAMHA_OK;
    }
    if (!h_host || !out_host) return fail(BRAMHA_ERR_INVALID, "null host buffer");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lk(ctx->io_mu);
    const int64_t ldx = (w->K + 3) / 4 * 4;
    rc = ensure_staging(ctx, (size_t)(ldx * M), (size_t)(w->N * M));
    if (rc) return rc;
    cudaStream_t st = ctx->stream;
    CK(cudaMemcpy2DAsync(ctx->dev_x, ldx * sizeof(float), h_host, w->K * sizeof(float), w->K * sizeof(float),
                         (size_t)M, cudaMemcpyHostToDevice, st),
       "H2D h_block");
    rc = gemm_device(ctx, w, ctx->dev_x, 1, ldx, M, ctx->dev_y, st);
    if (rc) return rc;
    CK(cudaMemcpyAsync(out_host, ctx->dev_y, sizeof(float) * (size_t)(w->N * M), cudaMemcpyDeviceToHost, st),
       "D2H out");
    return check_device_error(ctx, st);
}

int bramha_cuda_gemm_dev(bramha_ctx* ctx, const bramha_weight* w, const void* x_dev, int x_dtype, int64_t M,
                         float* y_dev, void* stream) {
    int rc = check_weight(ctx, w);
    if (rc) return rc;
    if (x_dtype != BRAMHA_DTYPE_F32 && x_dtype != BRAMHA_DTYPE_BF16)
        return fail(BRAMHA_ERR_INVALID, "gemm_dev: unknown activation dtype %d", x_dtype);
    if (M < 0) return fail(BRAMHA_ERR_INVALID, "negative block size");
    if (M > 0 && w->N > 0 && (!x_dev || !y_dev)) return fail(BRAMHA_ERR_INVALID, "null device pointer");
    if (x_dtype == BRAMHA_DTYPE_F32 && M > 0 && w->K > 0 &&
        ((reinterpret_cast<uintptr_t>(x_dev) & 15) != 0 || (M > 1 && (w->K & 3) != 0)))
        return fail(BRAMHA_ERR_INVALID, "f32 x_dev must be 16-byte aligned (and K a multiple of 4 when M > 1)");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    return gemm_device(ctx, w, x_dev, x_dtype == BRAMHA_DTYPE_F32 ? 1 : 0, w->K, M, y_dev, st);
}

int bramha_cuda_gemm_noalloc_dev(bramha_ctx* ctx, const bramha_weight* w, const void* x_dev, int64_t M,
                                 float* y_dev, void* stream) {
    int rc = check_weight(ctx, w);
    if (rc) return rc;
    if (M < 0) return fail(BRAMHA_ERR_INVALID, "negative block size");
    if (M > kNoAllocMaxTokens)
        return fail(BRAMHA_ERR_UNSUPPORTED,
                    "gemm_noalloc_dev: M = %lld tokens exceeds the fixed scratch of this entry point "
                    "(%lld tokens); split the block or use bramha_cuda_gemm_dev",
                    (long long)M, (long long)kNoAllocMaxTokens);
    if (w->fmt == BRAMHA_FMT_F32 || is_sp24(w->fmt))
        return fail(BRAMHA_ERR_UNSUPPORTED, "gemm_noalloc_dev: %s weights are not supported", fmt_name(w->fmt));
    if (M == 0 || w->N == 0) return BRAMHA_OK;
    if (!x_dev || !y_dev) return fail(BRAMHA_ERR_INVALID, "null device pointer");
    const int64_t keff = (w->fmt == BRAMHA_FMT_W4ZP8 || w->fmt == BRAMHA_FMT_LOG4) ? (w->K / 2) * 2 : w->K;
    if ((w->K % 8) != 0 || (reinterpret_cast<uintptr_t>(x_dev) & 15) != 0)
        return fail(BRAMHA_ERR_INVALID,
                    "gemm_noalloc_dev: x_dev must be 16-byte aligned bf16 [M][K] with K a multiple of 8");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    if (keff == 0) {  // an empty input gives zeros, as bramha_cuda_gemm_dev (a memset allocates nothing)
        CK(cudaMemsetAsync(y_dev, 0, sizeof(float) * (size_t)(w->N * M), st), "memset(y)");
        return BRAMHA_OK;
    }
    float* scratch = nullptr;
    if (w->fmt == BRAMHA_FMT_LOG4) CK(noalloc_rowsum_scratch(ctx->device, &scratch), "cudaGetSymbolAddress(scratch)");
    CK(launch_gemm_tcgen05_bf16_noalloc(w->fmt, w->q, w->ldq, w->scales, w->N, keff, x_dev, w->K, M, y_dev, w->N,
                                        ctx->d_err, scratch, st),
       "tcgen05 gemm (no-alloc) launch");
    return BRAMHA_OK;
}

// ---- column-shard group ----------------------------------------------------
int bramha_cuda_shard_handle(bramha_ctx* ctx, size_t arena_bytes, bramha_ipc_handle* out) {
    if (!ctx || !out) return fail(BRAMHA_ERR_INVALID, "null argument");
    if (ctx->arena) return fail(BRAMHA_ERR_INVALID, "this context already has a shard arena");
    if (arena_bytes < 2 * kArenaHeader) return fail(BRAMHA_ERR_INVALID, "shard arena of %zu bytes is too small", arena_bytes);
    static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(bramha_ipc_handle), "IPC handle size");
    DeviceGuard g(ctx->device);
    arena_bytes = (arena_bytes + 255) / 256 * 256;
    CK(cudaMalloc(&ctx->arena, arena_bytes), "cudaMalloc(shard arena)");
    cudaError_t e = cudaMemset(ctx->arena, 0, kArenaHeader);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ctx->arena);
    if (e != cudaSuccess) {
        cudaFree(ctx->arena);
        ctx->arena = nullptr;
        return cuda_fail(e, "shard arena IPC handle");
    }
    memcpy(out->bytes, &h, sizeof h);
    ctx->arena_bytes = arena_bytes;
    ctx->arena_used = kArenaHeader;
    ctx->arena_top = arena_bytes;
    return BRAMHA_OK;
}

int bramha_cuda_shard_init(bramha_ctx* ctx, int world, int rank, const bramha_ipc_handle* handles) {
    if (!ctx || !handles) return fail(BRAMHA_ERR_INVALID, "null argument");
    if (world < 2 || world > kMaxShardWorld || rank < 0 || rank >= world)
        return fail(BRAMHA_ERR_INVALID, "shard group of %d ranks (rank %d): 2..%d ranks", world, rank, kMaxShardWorld);
    if (!ctx->arena) return fail(BRAMHA_ERR_INVALID, "call bramha_cuda_shard_handle first");
    if (ctx->shard_world) return fail(BRAMHA_ERR_INVALID, "this context is already in a shard group");
    DeviceGuard g(ctx->device);
    for (int r = 0; r < world; ++r) {
        if (r == rank) {
            ctx->peer_arena[r] = ctx->arena;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, handles[r].bytes, sizeof h);
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != rank && ctx->peer_arena[q]) cudaIpcCloseMemHandle(ctx->peer_arena[q]);
            for (int q = 0; q < world; ++q) ctx->peer_arena[q] = nullptr;
            return cuda_fail(e, "open a peer's shard arena (cudaIpcOpenMemHandle)");
        }
        ctx->peer_arena[r] = static_cast<uint8_t*>(p);
    }
    ctx->shard_world = world;
    ctx->shard_rank = rank;
    return BRAMHA_OK;
}

int bramha_cuda_shard_malloc(bramha_ctx* ctx, size_t bytes, void** out) {
    if (!ctx || !out) return fail(BRAMHA_ERR_INVALID, "null argument");
    if (!ctx->arena) return fail(BRAMHA_ERR_INVALID, "no shard arena");
    const size_t b = (bytes + 255) / 256 * 256;
    if (ctx->arena_used + b > ctx->arena_top)
        return fail(BRAMHA_ERR_OOM, "shard arena exhausted (%zu of %zu bytes in use, %zu asked)", ctx->arena_used,
                    ctx->arena_bytes, bytes);
    *out = ctx->arena + ctx->arena_used;
    ctx->arena_used += b;
    return BRAMHA_OK;
}

int bramha_cuda_shard_rows(bramha_ctx* ctx, int64_t N, int64_t* row0, int64_t* rows) {
    if (!ctx || !row0 || !rows) return fail(BRAMHA_ERR_INVALID, "null argument");
    if (N < 0) return fail(BRAMHA_ERR_INVALID, "negative N");
    const int w = ctx->shard_world ? ctx->shard_world : 1, r = ctx->shard_rank;
    *row0 = N * r / w;
    *rows = N * (r + 1) / w - *row0;
    return BRAMHA_OK;
}

namespace {
int register_shard_impl(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K, const void* q,
                        size_t q_bytes, const float* scales, size_t n_scales, bool from_device, cudaStream_t st,
                        bramha_weight** out) {
    if (!ctx || !out || !key) return fail(BRAMHA_ERR_INVALID, "null argument");
    if (ctx->shard_world < 2) return fail(BRAMHA_ERR_INVALID, "no shard group (bramha_cuda_shard_init)");
    int rc = check_sizes(fmt, N, K, q_bytes, n_scales, scales != nullptr);
    if (rc) return rc;
    if (!is_tiled(fmt)) return fail(BRAMHA_ERR_UNSUPPORTED, "sharded weights take LOG4, W4ZP8 or W8");
    int64_t row0 = 0, rows = 0;
    bramha_cuda_shard_rows(ctx, N, &row0, &rows);
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        auto it = ctx->reg.find(key);
        if (it != ctx->reg.end() && (!it->second->shard || it->second->n_full != N || it->second->row0 != row0))
            return fail(BRAMHA_ERR_SIZE, "key '%s' is registered with a different shape or sharding", key);
    }
    const int64_t rb = row_bytes_of(fmt, K);
    const uint8_t* qs = static_cast<const uint8_t*>(q) + (q ? row0 * rb : 0);
    const float* ss = scales ? scales + row0 : nullptr;
    bramha_weight* w = nullptr;
    rc = register_impl(ctx, key, fmt, rows, K, rows ? qs : nullptr, (size_t)(rows * rb), ss, (size_t)rows, from_device,
                       st, &w);
    if (rc) return rc;
    w->shard = true;
    w->row0 = row0;
    w->n_full = N;
    *out = w;
    return BRAMHA_OK;
}
}  // namespace

int bramha_cuda_register_weight_shard(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K, const void* q,
                                      size_t q_bytes, const float* scales, size_t n_scales, bramha_weight** out) {
    return register_shard_impl(ctx, key, fmt, N, K, q, q_bytes, scales, n_scales, false, nullptr, out);
}

int bramha_cuda_register_weight_shard_dev(bramha_ctx* ctx, const char* key, int fmt, int64_t N, int64_t K,
                                          const void* q_dev, size_t q_bytes, const float* scales_dev, size_t n_scales,
                                          void* stream, bramha_weight** out) {
    return register_shard_impl(ctx, key, fmt, N, K, q_dev, q_bytes, scales_dev, n_scales, true,
                               static_cast<cudaStream_t>(stream), out);
}

int bramha_cuda_shard_sync_dev(bramha_ctx* ctx, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (ctx->shard_world < 2) return fail(BRAMHA_ERR_INVALID, "no shard group");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    CK(launch_shard_signal(shard_args(ctx), ctx->d_err, 0, st), "shard sync launch");
    return BRAMHA_OK;
}

int bramha_cuda_stream_sync(bramha_ctx* ctx, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    CK(cudaStreamSynchronize(st), "stream sync");
    return check_device_error(ctx, st);
}

int bramha_cuda_quantize_dev(bramha_ctx* ctx, int fmt, int64_t N, int64_t K, const float* w_dev, void* q_dev,
                             float* scales_dev, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (fmt != BRAMHA_FMT_W8 && fmt != BRAMHA_FMT_W4ZP8 && fmt != BRAMHA_FMT_LOG4)
        return fail(BRAMHA_ERR_INVALID, "quantize: format %d is not a quantized format", fmt);
    if (N < 0 || K < 0) return fail(BRAMHA_ERR_INVALID, "negative shape");
    if ((fmt == BRAMHA_FMT_W4ZP8 || fmt == BRAMHA_FMT_LOG4) && (K % 2) != 0)
        return fail(BRAMHA_ERR_INVALID, "in_features must be a multiple of 2 for %s packing", fmt_name(fmt));
    if (N == 0 || K == 0) return BRAMHA_OK;
    if (!w_dev || !q_dev || !scales_dev) return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    CK(launch_quantize(fmt, N, K, w_dev, static_cast<uint8_t*>(q_dev), scales_dev, st), "quantize launch");
    return BRAMHA_OK;
}

// ---- decode-step operations (decode.cu) -----------------------------------
namespace {
cudaStream_t op_stream(bramha_ctx* ctx, void* stream) {
    return stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
}
}  // namespace

int bramha_cuda_op_embed(bramha_ctx* ctx, const float* table_dev, int64_t vocab, int64_t hidden,
                         const int32_t* token_dev, float* x_dev, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (vocab <= 0 || hidden <= 0) return fail(BRAMHA_ERR_INVALID, "embed: empty table");
    if (!table_dev || !token_dev || !x_dev) return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    CK(launch_embed(table_dev, vocab, hidden, token_dev, x_dev, op_stream(ctx, stream)), "embed launch");
    return BRAMHA_OK;
}

int bramha_cuda_op_rmsnorm(bramha_ctx* ctx, float* x_dev, const float* delta_dev, const float* weight_dev, int64_t n,
                           float eps, float* out_dev, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (n <= 0 || n > (1 << 24)) return fail(BRAMHA_ERR_INVALID, "rmsnorm: size %lld out of range", (long long)n);
    if (!x_dev || !weight_dev || !out_dev) return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    CK(launch_rmsnorm(x_dev, delta_dev, weight_dev, n, eps, out_dev, op_stream(ctx, stream)), "rmsnorm launch");
    return BRAMHA_OK;
}

int bramha_cuda_op_qkv_rope(bramha_ctx* ctx, float* q_dev, const float* k_dev, const float* v_dev,
                            const float* bq_dev, const float* bk_dev, const float* bv_dev, int num_q_heads,
                            int num_kv_heads, int head_dim, float rope_theta, const int32_t* pos_dev, int64_t max_ctx,
                            float* k_cache_dev, float* v_cache_dev, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || head_dim <= 0 || (head_dim & 1) ||
        max_ctx <= 0)
        return fail(BRAMHA_ERR_INVALID, "qkv_rope: bad head layout");
    if (!q_dev || !k_dev || !v_dev || !pos_dev || !k_cache_dev || !v_cache_dev)
        return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    CK(launch_qkv_rope(q_dev, k_dev, v_dev, bq_dev, bk_dev, bv_dev, num_q_heads, num_kv_heads, head_dim, rope_theta,
                       pos_dev, max_ctx, k_cache_dev, v_cache_dev, op_stream(ctx, stream)),
       "qkv_rope launch");
    return BRAMHA_OK;
}

int bramha_cuda_op_attention(bramha_ctx* ctx, const float* q_dev, const float* k_cache_dev, const float* v_cache_dev,
                             const int32_t* pos_dev, int num_q_heads, int num_kv_heads, int head_dim, int64_t max_ctx,
                             float* out_dev, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || head_dim <= 0 || head_dim > 128 ||
        max_ctx <= 0 || max_ctx > 51200)
        return fail(BRAMHA_ERR_INVALID, "attention: heads, head_dim (<= 128) or max_ctx (<= 51200) out of range");
    if (!q_dev || !k_cache_dev || !v_cache_dev || !pos_dev || !out_dev)
        return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    CK(launch_attention(q_dev, k_cache_dev, v_cache_dev, pos_dev, num_q_heads, num_kv_heads, head_dim, max_ctx,
                        ctx->split_ws, kSplitWsFloats, ctx->split_tickets, kSplitTickets, out_dev,
                        op_stream(ctx, stream)),
       "attention launch");
    return BRAMHA_OK;
}

int bramha_cuda_op_rope_attention(bramha_ctx* ctx, const float* q_dev, const float* k_dev, const float* v_dev,
                                  const float* bq_dev, const float* bk_dev, const float* bv_dev, int num_q_heads,
                                  int num_kv_heads, int head_dim, float rope_theta, const int32_t* pos_dev,
                                  int64_t max_ctx, float* k_cache_dev, float* v_cache_dev, float* out_dev,
                                  void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || head_dim <= 0 || (head_dim & 1) ||
        head_dim > 128 || max_ctx <= 0 || max_ctx > 51200)
        return fail(BRAMHA_ERR_INVALID, "rope_attention: heads, head_dim (even, <= 128) or max_ctx (<= 51200) out of range");
    if (!q_dev || !k_dev || !v_dev || !pos_dev || !k_cache_dev || !v_cache_dev || !out_dev)
        return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    CK(launch_rope_attention(q_dev, k_dev, v_dev, bq_dev, bk_dev, bv_dev, rope_theta, pos_dev, max_ctx, k_cache_dev,
                             v_cache_dev, num_q_heads, num_kv_heads, head_dim, ctx->split_ws, kSplitWsFloats,
                             ctx->split_tickets, kSplitTickets, out_dev, op_stream(ctx, stream)),
       "rope_attention launch");
    return BRAMHA_OK;
}

int bramha_cuda_op_silu_mul(bramha_ctx* ctx, const float* g_dev, const float* u_dev, int64_t n, float* out_dev,
                            void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (n < 0) return fail(BRAMHA_ERR_INVALID, "negative size");
    if (n > 0 && (!g_dev || !u_dev || !out_dev)) return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    CK(launch_silu_mul(g_dev, u_dev, n, out_dev, op_stream(ctx, stream)), "silu_mul launch");
    return BRAMHA_OK;
}

int bramha_cuda_op_select(bramha_ctx* ctx, float* logits_dev, int64_t vocab, int32_t* generated_dev,
                          int32_t* count_dev, int64_t max_generated, float penalty, int greedy, int32_t* token_dev,
                          int32_t* pos_dev, void* stream) {
    if (!ctx) return fail(BRAMHA_ERR_INVALID, "null context");
    if (vocab <= 0 || max_generated < 0) return fail(BRAMHA_ERR_INVALID, "select: bad sizes");
    if (!pos_dev || (greedy && (!logits_dev || !generated_dev || !count_dev || !token_dev)))
        return fail(BRAMHA_ERR_INVALID, "null device pointer");
    DeviceGuard g(ctx->device);
    CK(launch_select(logits_dev, vocab, generated_dev, count_dev, max_generated, penalty, greedy, token_dev, pos_dev,
                     op_stream(ctx, stream)),
       "select launch");
    return BRAMHA_OK;
}

}  // extern "C"
