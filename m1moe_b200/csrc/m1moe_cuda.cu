// m1moe_cuda.cu — C ABI (include/m1moe_cuda.h) over the sm_100a kernels.
//
// The context owns all device memory (the HBM expert table, the bf16 router
// table and per-call scratch); callers own their buffers and lend them for the
// duration of a call, as in the reference where MetalContext owns the expert
// slots (MetalContext.swift:154-178) and WeightStore owns the mmap
// (WeightStore.swift:78-81).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "m1moe_cuda.h"
#include "common.cuh"
#include "matvec4.cuh"
#include "moe_decode.cuh"
#include "pipeline.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<long long> g_launches{0};

m1moe_status fail(m1moe_status st, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}

m1moe_status cuda_fail(cudaError_t e, const char *what) {
    m1moe_status st = (e == cudaErrorMemoryAllocation) ? M1MOE_ERR_OUT_OF_MEMORY : M1MOE_ERR_CUDA;
    return fail(st, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define M1_CK(call)                                              \
    do {                                                         \
        cudaError_t e_ = (call);                                 \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);      \
    } while (0)

#define M1_LAUNCHED()                                            \
    do {                                                         \
        cudaError_t e_ = cudaGetLastError();                     \
        if (e_ != cudaSuccess) return cuda_fail(e_, "kernel launch"); \
        g_launches.fetch_add(1, std::memory_order_relaxed);      \
    } while (0)

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

bool valid_dtype(int32_t d) { return d == M1MOE_DTYPE_F32 || d == M1MOE_DTYPE_BF16; }

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
    return n > 0 ? n : 148;
}

void expert_offsets(int h, int I, int gs, long long off[9]) {
    // InferenceEngine.swift:79-97
    const long long gw = (long long)I * (h / 8) * 4, gsb = (long long)I * (h / gs) * 2;
    const long long dw = (long long)h * (I / 8) * 4, dsb = (long long)h * (I / gs) * 2;
    off[0] = 0;
    off[1] = off[0] + gw;
    off[2] = off[1] + gsb;
    off[3] = off[2] + gsb;
    off[4] = off[3] + gw;
    off[5] = off[4] + gsb;
    off[6] = off[5] + gsb;
    off[7] = off[6] + dw;
    off[8] = off[7] + dsb;
}

template <int NT>
cudaError_t launch_matvec_nt(const m1::MatvecParams &p, long long groups, int grid_cap,
                             cudaStream_t st) {
    constexpr int R = 4;
    (void)groups;
    const long long warps_needed = (long long)p.num_mats * ((p.out_dim + R - 1) / R);
    long long grid = std::min<long long>((warps_needed + 7) / 8, grid_cap);
    if (grid < 1) grid = 1;
    m1::k_matvec4<NT, R><<<(unsigned)grid, 256, 0, st>>>(p);
    return cudaGetLastError();
}

}  // namespace

struct m1moe_cuda_ctx {
    m1moe_cuda_cfg cfg{};
    int e0 = 0, ne = 0;
    size_t expert_bytes = 0;
    long long off[9] = {};
    uint8_t *table = nullptr;     // [layers][ne][expert_bytes]
    uint16_t *router = nullptr;   // [layers][E][h]
    std::vector<uint8_t> layer_loaded, router_loaded;
    float *logits = nullptr;      // [max_batch][E]
    uint16_t *xT = nullptr;       // [max_batch][h] bf16, pair-permuted chunk-transposed
    float *xsum = nullptr;        // [max_batch][h/32]
    uint16_t *actT = nullptr;     // [max_batch*K][I] bf16, pair-permuted chunk-transposed
    int *err = nullptr;           // device error word (pipeline.cuh kErr*)
    m1::RouteInfo *route = nullptr;  // routing decision of the current call
    int *ticket = nullptr;        // router grid's last-CTA ticket
    unsigned long long *trace = nullptr;  // optional phase timestamps (caller-owned)
    // synchronous host-buffer path
    float *hx = nullptr, *hres = nullptr, *hout = nullptr;
    int *hidx = nullptr;
    float *hw = nullptr;
    cudaStream_t stream = nullptr;  // for the *_host calls and staging copies
    void *pinned[2] = {nullptr, nullptr};
    size_t pinned_bytes = 0;
    cudaEvent_t staged[2] = {nullptr, nullptr};
    int num_sms = 148;
};

namespace {

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

void free_ctx(m1moe_cuda_ctx *c) {
    if (!c) return;
    cudaFree(c->table);
    cudaFree(c->router);
    cudaFree(c->logits);
    cudaFree(c->xT);
    cudaFree(c->xsum);
    cudaFree(c->actT);
    cudaFree(c->err);
    cudaFree(c->route);
    cudaFree(c->ticket);
    cudaFree(c->hx);
    cudaFree(c->hres);
    cudaFree(c->hout);
    cudaFree(c->hidx);
    cudaFree(c->hw);
    for (int i = 0; i < 2; ++i) {
        if (c->pinned[i]) cudaFreeHost(c->pinned[i]);
        if (c->staged[i]) cudaEventDestroy(c->staged[i]);
    }
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

m1::MoeParams moe_params(m1moe_cuda_ctx *c, int layer, int B) {
    m1::MoeParams p{};
    const m1moe_cuda_cfg &g = c->cfg;
    p.table = c->table + (size_t)layer * c->ne * c->expert_bytes;
    p.expert_bytes = (long long)c->expert_bytes;
    for (int i = 0; i < 9; ++i) p.off[i] = c->off[i];
    p.router = c->router + (size_t)layer * g.num_experts * g.hidden_dim;
    p.E = g.num_experts;
    p.K = g.top_k;
    p.h = g.hidden_dim;
    p.I = g.intermediate_dim;
    p.gs = g.group_size;
    p.norm = g.norm_topk_prob;
    p.e0 = c->e0;
    p.ne = c->ne;
    p.ntok = B;
    p.logits = c->logits;
    p.xT = c->xT;
    p.xsum = c->xsum;
    p.actT = c->actT;
    p.err = c->err;
    p.route = c->route;
    p.ticket = c->ticket;
    p.trace = c->trace;
    return p;
}

// Shared-memory pipeline geometry.  A gate/up CTA and a down CTA are sized to
// be resident on one SM together (so the down grid can prefetch while gate/up
// runs): rings of ~100 KB and ~88 KB.
struct Geometry {
    int grid, router_grid;
    size_t gu_smem, dn_smem, router_smem;
};


int round_up(int v, int m) { return (v + m - 1) / m * m; }

constexpr size_t kMaxDynSmem = 227 * 1024;  // per-CTA opt-in limit on sm_100

// Pipeline geometry for a batch of NT (template) tokens; rt_gu / rt_dn are the
// kernels' rows per tile (TileRows<NT>).  Each ring gets the shared memory left
// after the kernel's fixed parts.
Geometry plan_geometry(m1::MoeParams &p, int num_sms, int nt, int rt_gu, int rt_dn) {
    Geometry g{};
    g.grid = num_sms;
    const int srb_h = (p.h / p.gs) * 2, srb_i = (p.I / p.gs) * 2;
    const int nch = p.h / m1::kChunkCols, nchI = p.I / m1::kChunkCols;
    const int maxU = std::min(p.ntok * p.K, p.ne);
    // ---- gate/up: tile = rt rows of gate and of up, each W + S span + B span
    // (a span rounded out to 16 bytes adds at most 32 bytes).
    const int pair_bytes = 2 * (p.h / 2) + 4 * srb_h;
    p.gu_stage_bytes = round_up(rt_gu * pair_bytes + 4 * 32, 128);
    p.gu_nslices = nt <= 2 ? (nch + 31) / 32 : 1;
    const long long gu_units = (long long)maxU * (p.I / rt_gu);
    p.gu_rows_max = (int)((gu_units + g.grid - 1) / g.grid) * rt_gu;
    p.x_smem = (size_t)nt * p.h * 2 <= 32 * 1024;
    size_t gu_fixed = sizeof(m1::Ctl) + 16;
    if (p.x_smem) gu_fixed += (size_t)nt * p.h * 2 + (size_t)nt * nch * 4;
    if (p.gu_nslices > 1) gu_fixed += (size_t)p.gu_rows_max * p.gu_nslices * 2 * nt * 4;
    p.gu_nstages = (int)std::min<size_t>(
        m1::kMaxStages, (kMaxDynSmem - gu_fixed) / (p.gu_stage_bytes + 2 * sizeof(uint64_t)));
    g.gu_smem = (size_t)p.gu_nstages * (p.gu_stage_bytes + 2 * sizeof(uint64_t)) + gu_fixed;
    // ---- down: tile = up to rt rows of down of one expert
    const int row_bytes = p.I / 2 + 2 * srb_i;
    p.dn_stage_bytes = round_up(rt_dn * row_bytes + 2 * 32, 128);
    p.dn_nslices = nt <= 2 ? (nchI + 31) / 32 : 1;
    p.dn_rows_max = (p.h + g.grid - 1) / g.grid;
    const size_t dn_fixed = sizeof(m1::Ctl) + 16 +
                            (size_t)p.ntok * p.K * p.dn_rows_max * p.dn_nslices * sizeof(float);
    p.dn_nstages = (int)std::min<size_t>(
        m1::kMaxStages, (kMaxDynSmem - dn_fixed) / (p.dn_stage_bytes + 2 * sizeof(uint64_t)));
    g.dn_smem = (size_t)p.dn_nstages * (p.dn_stage_bytes + 2 * sizeof(uint64_t)) + dn_fixed;
    // ---- router
    g.router_grid = std::min(num_sms, std::max(p.E, 1));
    const int per = (p.E + g.router_grid - 1) / g.router_grid;
    g.router_smem = (size_t)per * p.h * 2 + 16 + 8 * m1::kMaxTok * sizeof(float);
    return g;
}

template <typename Kern>
cudaError_t allow_smem(Kern kern, size_t bytes) {
    // Idempotent; called before every launch so each instantiation is covered.
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// Launch with Programmatic Dependent Launch enabled: the kernel may start while
// its stream predecessor is still running; griddepcontrol.wait inside the
// kernel orders it after the predecessor's completion.
template <typename Kern>
cudaError_t launch_pdl(Kern kern, int grid, int block, size_t smem, cudaStream_t st,
                       const m1::MoeParams &p) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

#define M1_TRY_LAUNCH(expr)                                      \
    do {                                                         \
        cudaError_t e_ = (expr);                                 \
        if (e_ != cudaSuccess) return cuda_fail(e_, #expr);      \
        g_launches.fetch_add(1, std::memory_order_relaxed);      \
    } while (0)

// route_only: router + routing (no expert work), for m1moe_cuda_router_topk.
template <int NT>
m1moe_status launch_moe(m1moe_cuda_ctx *c, m1::MoeParams p, cudaStream_t st, bool route_only) {
    Geometry g = plan_geometry(p, c->num_sms, NT, m1::TileRows<NT>::gu, m1::TileRows<NT>::dn);
    if (g.gu_smem > kMaxDynSmem || g.dn_smem > kMaxDynSmem || p.gu_nstages < 2 || p.dn_nstages < 2)
        return fail(M1MOE_ERR_UNSUPPORTED, "shape needs more shared memory than an SM has");
    M1_CK(allow_smem(m1::k_router<NT>, g.router_smem));
    M1_TRY_LAUNCH(launch_pdl(m1::k_router<NT>, g.router_grid, m1::kRouterThreads, g.router_smem,
                             st, p));
    if (route_only) return M1MOE_OK;  // the router grid's last CTA wrote the outputs
    M1_CK(allow_smem(m1::k_moe_gateup<NT>, g.gu_smem));
    M1_TRY_LAUNCH(launch_pdl(m1::k_moe_gateup<NT>, g.grid, m1::kPipeThreads, g.gu_smem, st, p));
    M1_CK(allow_smem(m1::k_moe_down<NT>, g.dn_smem));
    M1_TRY_LAUNCH(launch_pdl(m1::k_moe_down<NT>, g.grid, m1::kPipeThreads, g.dn_smem, st, p));
    return M1MOE_OK;
}

m1moe_status dispatch_moe(m1moe_cuda_ctx *c, const m1::MoeParams &p, cudaStream_t st,
                          bool route_only) {
    if (p.ntok == 1) return launch_moe<1>(c, p, st, route_only);
    if (p.ntok == 2) return launch_moe<2>(c, p, st, route_only);
    if (p.ntok <= 4) return launch_moe<4>(c, p, st, route_only);
    return launch_moe<8>(c, p, st, route_only);
}

m1moe_status check_layer(m1moe_cuda_ctx *c, int32_t layer) {
    if (!c) return fail(M1MOE_ERR_INVALID_ARG, "ctx is NULL");
    if (layer < 0 || layer >= c->cfg.num_layers)
        return fail(M1MOE_ERR_INVALID_ARG, "layer %d out of range [0,%d)", layer, c->cfg.num_layers);
    return M1MOE_OK;
}

}  // namespace

extern "C" {

int32_t m1moe_cuda_abi_version(void) { return M1MOE_CUDA_ABI_VERSION; }

const char *m1moe_cuda_last_error(void) { return g_last_error.c_str(); }

int64_t m1moe_cuda_launch_count(void) { return g_launches.load(); }

m1moe_status m1moe_cuda_set_trace(m1moe_cuda_ctx *c, uint64_t *d_trace) {
    if (!c) return fail(M1MOE_ERR_INVALID_ARG, "ctx is NULL");
    c->trace = reinterpret_cast<unsigned long long *>(d_trace);
    return M1MOE_OK;
}

size_t m1moe_cuda_expert_bytes(int32_t h, int32_t I, int32_t gs) {
    if (h <= 0 || I <= 0 || gs <= 0 || h % gs || I % gs || h % 8 || I % 8) return 0;
    long long off[9];
    expert_offsets(h, I, gs, off);
    return (size_t)(off[8] + (long long)h * (I / gs) * 2);
}

m1moe_status m1moe_cuda_create(const m1moe_cuda_cfg *cfg, m1moe_cuda_ctx **out_ctx) {
    if (!cfg || !out_ctx) return fail(M1MOE_ERR_INVALID_ARG, "cfg/out_ctx is NULL");
    *out_ctx = nullptr;
    const m1moe_cuda_cfg g = *cfg;
    if (g.hidden_dim <= 0 || g.intermediate_dim <= 0 || g.num_layers <= 0)
        return fail(M1MOE_ERR_INVALID_ARG, "dims must be positive");
    if (g.hidden_dim % 64 || g.intermediate_dim % 64)
        return fail(M1MOE_ERR_INVALID_ARG, "hidden_dim and intermediate_dim must be multiples of 64");
    if (g.group_size <= 0 || g.group_size % 32 || g.hidden_dim % g.group_size ||
        g.intermediate_dim % g.group_size)
        return fail(M1MOE_ERR_UNSUPPORTED,
                    "group_size %d: must be a multiple of 32 dividing hidden and intermediate dims",
                    g.group_size);
    if (g.num_experts <= 0 || g.num_experts > m1::kMaxExperts)
        return fail(M1MOE_ERR_UNSUPPORTED, "num_experts %d outside [1,%d]", g.num_experts,
                    m1::kMaxExperts);
    if (g.top_k <= 0 || g.top_k > g.num_experts || g.top_k > m1::kMaxTopK)
        return fail(M1MOE_ERR_INVALID_ARG, "top_k %d invalid", g.top_k);
    if (g.max_batch <= 0 || g.max_batch > m1::kMaxTok)
        return fail(M1MOE_ERR_INVALID_ARG, "max_batch %d outside [1,%d]", g.max_batch, m1::kMaxTok);
    const int e0 = g.expert_begin, ne = g.expert_count ? g.expert_count : g.num_experts;
    if (e0 < 0 || ne <= 0 || e0 + ne > g.num_experts)
        return fail(M1MOE_ERR_INVALID_ARG, "expert shard [%d,%d) outside [0,%d)", e0, e0 + ne,
                    g.num_experts);
    int ndev = 0;
    M1_CK(cudaGetDeviceCount(&ndev));
    if (g.device < 0 || g.device >= ndev)
        return fail(M1MOE_ERR_INVALID_ARG, "device %d outside [0,%d)", g.device, ndev);
    DeviceGuard dg(g.device);

    auto *c = new m1moe_cuda_ctx();
    c->cfg = g;
    c->e0 = e0;
    c->ne = ne;
    c->expert_bytes = m1moe_cuda_expert_bytes(g.hidden_dim, g.intermediate_dim, g.group_size);
    expert_offsets(g.hidden_dim, g.intermediate_dim, g.group_size, c->off);
    c->layer_loaded.assign(g.num_layers, 0);
    c->router_loaded.assign(g.num_layers, 0);
    c->num_sms = sm_count();
    const size_t B = g.max_batch, E = g.num_experts, K = g.top_k;
    cudaError_t e;
#define M1_ALLOC(ptr, bytes)                                        \
    e = cudaMalloc((void **)&(ptr), (bytes));                       \
    if (e != cudaSuccess) {                                         \
        m1moe_status st_ = cuda_fail(e, "cudaMalloc " #ptr);       \
        free_ctx(c);                                                \
        return st_;                                                 \
    }
    // +64: tile copies round scale/bias ranges out to 16-byte boundaries and
    // may read up to 15 bytes past the last array of the last expert.
    M1_ALLOC(c->table, (size_t)g.num_layers * ne * c->expert_bytes + 64);
    M1_ALLOC(c->router, (size_t)g.num_layers * E * g.hidden_dim * 2);
    M1_ALLOC(c->logits, B * E * 4);
    M1_ALLOC(c->xT, B * g.hidden_dim * 2);
    M1_ALLOC(c->xsum, B * (g.hidden_dim / 32) * 4);
    M1_ALLOC(c->actT, B * K * g.intermediate_dim * 2);
    M1_ALLOC(c->err, 4);
    M1_ALLOC(c->route, sizeof(m1::RouteInfo));
    M1_ALLOC(c->ticket, 4);
    M1_ALLOC(c->hx, B * g.hidden_dim * 4);
    M1_ALLOC(c->hres, B * g.hidden_dim * 4);
    M1_ALLOC(c->hout, B * g.hidden_dim * 4);
    M1_ALLOC(c->hidx, B * K * 4);
    M1_ALLOC(c->hw, B * K * 4);
#undef M1_ALLOC
    e = cudaMemset(c->err, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(c->ticket, 0, 4);
    if (e != cudaSuccess) {
        m1moe_status st = cuda_fail(e, "cudaMemset err");
        free_ctx(c);
        return st;
    }
    e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        m1moe_status st = cuda_fail(e, "cudaStreamCreate");
        free_ctx(c);
        return st;
    }
    *out_ctx = c;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_destroy(m1moe_cuda_ctx *ctx) {
    if (!ctx) return M1MOE_OK;
    DeviceGuard dg(ctx->cfg.device);
    cudaStreamSynchronize(ctx->stream);
    free_ctx(ctx);
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_load_expert_layer(m1moe_cuda_ctx *c, int32_t layer, const void *h_bytes,
                                          size_t nbytes) {
    if (m1moe_status st = check_layer(c, layer)) return st;
    if (!h_bytes) return fail(M1MOE_ERR_INVALID_ARG, "layer bytes pointer is NULL");
    const size_t want = (size_t)c->cfg.num_experts * c->expert_bytes;
    if (nbytes != want)
        return fail(M1MOE_ERR_INVALID_ARG, "layer %d: %zu bytes, expected %zu (= %d x %zu)", layer,
                    nbytes, want, c->cfg.num_experts, c->expert_bytes);
    DeviceGuard dg(c->cfg.device);
    // Double-buffered pinned staging: memcpy into one bounce buffer while the
    // other is in flight to HBM.
    const size_t chunk = 32u << 20;
    if (!c->pinned[0]) {
        for (int i = 0; i < 2; ++i) {
            M1_CK(cudaHostAlloc(&c->pinned[i], chunk, cudaHostAllocDefault));
            M1_CK(cudaEventCreateWithFlags(&c->staged[i], cudaEventDisableTiming));
        }
        c->pinned_bytes = chunk;
    }
    const uint8_t *src = static_cast<const uint8_t *>(h_bytes) + (size_t)c->e0 * c->expert_bytes;
    uint8_t *dst = c->table + (size_t)layer * c->ne * c->expert_bytes;
    const size_t total = (size_t)c->ne * c->expert_bytes;
    int buf = 0;
    bool used[2] = {false, false};
    for (size_t done = 0; done < total; done += chunk, buf ^= 1) {
        const size_t n = std::min(chunk, total - done);
        if (used[buf]) M1_CK(cudaEventSynchronize(c->staged[buf]));
        memcpy(c->pinned[buf], src + done, n);
        M1_CK(cudaMemcpyAsync(dst + done, c->pinned[buf], n, cudaMemcpyHostToDevice, c->stream));
        M1_CK(cudaEventRecord(c->staged[buf], c->stream));
        used[buf] = true;
    }
    M1_CK(cudaStreamSynchronize(c->stream));
    c->layer_loaded[layer] = 1;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_load_expert_layer_device(m1moe_cuda_ctx *c, int32_t layer,
                                                 const void *d_bytes, size_t nbytes, void *stream) {
    if (m1moe_status st = check_layer(c, layer)) return st;
    if (!d_bytes) return fail(M1MOE_ERR_INVALID_ARG, "layer bytes pointer is NULL");
    const size_t want = (size_t)c->cfg.num_experts * c->expert_bytes;
    if (nbytes != want)
        return fail(M1MOE_ERR_INVALID_ARG, "layer %d: %zu bytes, expected %zu", layer, nbytes, want);
    DeviceGuard dg(c->cfg.device);
    M1_CK(cudaMemcpyAsync(c->table + (size_t)layer * c->ne * c->expert_bytes,
                          static_cast<const uint8_t *>(d_bytes) + (size_t)c->e0 * c->expert_bytes,
                          (size_t)c->ne * c->expert_bytes, cudaMemcpyDeviceToDevice,
                          as_stream(stream)));
    c->layer_loaded[layer] = 1;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_load_router(m1moe_cuda_ctx *c, int32_t layer, const uint16_t *h_router,
                                    size_t count) {
    if (m1moe_status st = check_layer(c, layer)) return st;
    if (!h_router) return fail(M1MOE_ERR_INVALID_ARG, "router pointer is NULL");
    const size_t want = (size_t)c->cfg.num_experts * c->cfg.hidden_dim;
    if (count != want)
        return fail(M1MOE_ERR_INVALID_ARG, "router: %zu elements, expected %zu", count, want);
    DeviceGuard dg(c->cfg.device);
    M1_CK(cudaMemcpy(c->router + (size_t)layer * want, h_router, want * 2, cudaMemcpyHostToDevice));
    c->router_loaded[layer] = 1;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_matvec4_strided(const uint32_t *d_w, const uint16_t *d_s,
                                        const uint16_t *d_b, int64_t mat_stride, int32_t num_mats,
                                        const void *d_x, int32_t x_dtype, void *d_y,
                                        int32_t y_dtype, int32_t out_dim, int32_t in_dim,
                                        int32_t gs, int32_t batch, void *stream) {
    if (!d_w || !d_s || !d_b || !d_x || !d_y) return fail(M1MOE_ERR_INVALID_ARG, "NULL pointer");
    if (!valid_dtype(x_dtype) || !valid_dtype(y_dtype))
        return fail(M1MOE_ERR_INVALID_ARG, "dtype must be F32 (0) or BF16 (1)");
    if (out_dim <= 0 || in_dim <= 0 || in_dim % 64)
        return fail(M1MOE_ERR_INVALID_ARG, "in_dim %d must be a positive multiple of 64", in_dim);
    if (gs <= 0 || gs % 32 || in_dim % gs)
        return fail(M1MOE_ERR_UNSUPPORTED, "group_size %d must be a multiple of 32 dividing in_dim",
                    gs);
    if (batch < 1 || batch > m1::kMaxTok)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d outside [1,%d]", batch, m1::kMaxTok);
    if (num_mats < 1 || (num_mats > 1 && (mat_stride <= 0 || mat_stride % 16)))
        return fail(M1MOE_ERR_INVALID_ARG, "num_mats/mat_stride invalid");
    if ((reinterpret_cast<uintptr_t>(d_w) & 15) || (reinterpret_cast<uintptr_t>(d_x) & 15))
        return fail(M1MOE_ERR_INVALID_ARG, "weights and x must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(d_s) & 1) || (reinterpret_cast<uintptr_t>(d_b) & 1))
        return fail(M1MOE_ERR_INVALID_ARG, "scales/biases must be 2-byte aligned");
    m1::MatvecParams p{};
    p.w = reinterpret_cast<const uint8_t *>(d_w);
    p.s = reinterpret_cast<const uint8_t *>(d_s);
    p.b = reinterpret_cast<const uint8_t *>(d_b);
    p.mat_stride = num_mats > 1 ? mat_stride : 0;
    p.num_mats = num_mats;
    p.x = d_x;
    p.x_bf16 = x_dtype == M1MOE_DTYPE_BF16;
    p.y = d_y;
    p.y_bf16 = y_dtype == M1MOE_DTYPE_BF16;
    p.out_dim = out_dim;
    p.in_dim = in_dim;
    p.gs = gs;
    p.ntok = batch;
    const int cap = 4 * sm_count();
    cudaStream_t st = as_stream(stream);
    cudaError_t e;
    if (batch == 1) e = launch_matvec_nt<1>(p, 0, cap, st);
    else if (batch == 2) e = launch_matvec_nt<2>(p, 0, cap, st);
    else if (batch <= 4) e = launch_matvec_nt<4>(p, 0, cap, st);
    else e = launch_matvec_nt<8>(p, 0, cap, st);
    if (e != cudaSuccess) return cuda_fail(e, "k_matvec4 launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_matvec4(const uint32_t *d_w, const uint16_t *d_s, const uint16_t *d_b,
                                const void *d_x, int32_t x_dtype, void *d_y, int32_t y_dtype,
                                int32_t out_dim, int32_t in_dim, int32_t gs, int32_t batch,
                                void *stream) {
    return m1moe_cuda_matvec4_strided(d_w, d_s, d_b, 0, 1, d_x, x_dtype, d_y, y_dtype, out_dim,
                                      in_dim, gs, batch, stream);
}

m1moe_status m1moe_cuda_unpack4(const uint32_t *d_w, uint8_t *d_q, int32_t rows, int32_t cols,
                                void *stream) {
    if (!d_w || !d_q) return fail(M1MOE_ERR_INVALID_ARG, "NULL pointer");
    if (rows <= 0 || cols <= 0 || cols % 8)
        return fail(M1MOE_ERR_INVALID_ARG, "rows/cols invalid (cols %% 8 == 0 required)");
    if (reinterpret_cast<uintptr_t>(d_q) & 7)
        return fail(M1MOE_ERR_INVALID_ARG, "q must be 8-byte aligned");
    const long long nwords = (long long)rows * (cols / 8);
    const int grid = (int)std::min<long long>((nwords + 255) / 256, 8LL * sm_count());
    m1::k_unpack4<<<std::max(grid, 1), 256, 0, as_stream(stream)>>>(d_w, d_q, nwords);
    M1_LAUNCHED();
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_router_topk(m1moe_cuda_ctx *c, int32_t layer, const void *d_x,
                                    int32_t x_dtype, int32_t B, int32_t *d_idx, float *d_w,
                                    float *d_scores, void *stream) {
    if (m1moe_status st = check_layer(c, layer)) return st;
    if (!d_x || !valid_dtype(x_dtype)) return fail(M1MOE_ERR_INVALID_ARG, "x/x_dtype invalid");
    if (B < 1 || B > c->cfg.max_batch)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d outside [1,%d]", B, c->cfg.max_batch);
    if (!c->router_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "router of layer %d not loaded", layer);
    DeviceGuard dg(c->cfg.device);
    m1::MoeParams p = moe_params(c, layer, B);
    p.x = d_x;
    p.x_bf16 = x_dtype == M1MOE_DTYPE_BF16;
    p.user_idx = d_idx;
    p.user_w = d_w;
    p.user_scores = d_scores;
    return dispatch_moe(c, p, as_stream(stream), true);
}

m1moe_status m1moe_cuda_moe_layer(m1moe_cuda_ctx *c, int32_t layer, const void *d_x,
                                  int32_t x_dtype, const void *d_res, int32_t res_dtype, void *d_out,
                                  int32_t out_dtype, int32_t B, int32_t *d_idx, float *d_w,
                                  void *stream) {
    if (m1moe_status st = check_layer(c, layer)) return st;
    if (!d_x || !d_out) return fail(M1MOE_ERR_INVALID_ARG, "x/out is NULL");
    if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype) || (d_res && !valid_dtype(res_dtype)))
        return fail(M1MOE_ERR_INVALID_ARG, "dtype must be F32 (0) or BF16 (1)");
    if (B < 1 || B > c->cfg.max_batch)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d outside [1,%d]", B, c->cfg.max_batch);
    if ((reinterpret_cast<uintptr_t>(d_x) & 15))
        return fail(M1MOE_ERR_INVALID_ARG, "x must be 16-byte aligned");
    if (!c->router_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "router of layer %d not loaded", layer);
    if (!c->layer_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "experts of layer %d not loaded", layer);
    DeviceGuard dg(c->cfg.device);
    m1::MoeParams p = moe_params(c, layer, B);
    p.x = d_x;
    p.x_bf16 = x_dtype == M1MOE_DTYPE_BF16;
    p.res = d_res;
    p.res_bf16 = res_dtype == M1MOE_DTYPE_BF16;
    p.out = d_out;
    p.out_bf16 = out_dtype == M1MOE_DTYPE_BF16;
    p.user_idx = d_idx;
    p.user_w = d_w;
    return dispatch_moe(c, p, as_stream(stream), false);
}

m1moe_status m1moe_cuda_moe_layer_host(m1moe_cuda_ctx *c, int32_t layer, const float *h_x,
                                       const float *h_res, float *h_out, int32_t B,
                                       int32_t *h_idx, float *h_w) {
    if (m1moe_status st = check_layer(c, layer)) return st;
    if (!h_x || !h_out) return fail(M1MOE_ERR_INVALID_ARG, "x/out is NULL");
    if (B < 1 || B > c->cfg.max_batch)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d outside [1,%d]", B, c->cfg.max_batch);
    DeviceGuard dg(c->cfg.device);
    const size_t hb = (size_t)B * c->cfg.hidden_dim * 4, kb = (size_t)B * c->cfg.top_k * 4;
    M1_CK(cudaMemcpyAsync(c->hx, h_x, hb, cudaMemcpyHostToDevice, c->stream));
    if (h_res) M1_CK(cudaMemcpyAsync(c->hres, h_res, hb, cudaMemcpyHostToDevice, c->stream));
    m1moe_status st = m1moe_cuda_moe_layer(c, layer, c->hx, M1MOE_DTYPE_F32,
                                           h_res ? c->hres : nullptr, M1MOE_DTYPE_F32, c->hout,
                                           M1MOE_DTYPE_F32, B, c->hidx, c->hw, c->stream);
    if (st) return st;
    M1_CK(cudaMemcpyAsync(h_out, c->hout, hb, cudaMemcpyDeviceToHost, c->stream));
    if (h_idx) M1_CK(cudaMemcpyAsync(h_idx, c->hidx, kb, cudaMemcpyDeviceToHost, c->stream));
    if (h_w) M1_CK(cudaMemcpyAsync(h_w, c->hw, kb, cudaMemcpyDeviceToHost, c->stream));
    M1_CK(cudaStreamSynchronize(c->stream));
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_synchronize(m1moe_cuda_ctx *c) {
    if (!c) return fail(M1MOE_ERR_INVALID_ARG, "ctx is NULL");
    DeviceGuard dg(c->cfg.device);
    M1_CK(cudaDeviceSynchronize());
    int word = 0;
    M1_CK(cudaMemcpy(&word, c->err, 4, cudaMemcpyDeviceToHost));
    if (word) {
        M1_CK(cudaMemset(c->err, 0, 4));
        return fail(M1MOE_ERR_DEVICE, "device error word 0x%x (1: pipeline wait timed out)", word);
    }
    return M1MOE_OK;
}

}  // extern "C"
