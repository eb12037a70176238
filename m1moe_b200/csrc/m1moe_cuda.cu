// m1moe_cuda.cu — C ABI (include/m1moe_cuda.h) over the sm_100a kernels.
//
// The context owns all device memory (the HBM expert table, the bf16 router
// table and per-call scratch); callers own their buffers and lend them for the
// duration of a call, as in the reference where MetalContext owns the expert
// slots (MetalContext.swift:154-178) and WeightStore owns the mmap
// (WeightStore.swift:78-81).
#include <cuda.h>
#include <cuda_runtime.h>

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "m1moe_cuda.h"
#include "common.cuh"
#include "host_io.cuh"
#include "matvec4.cuh"
#include "moe_layer.cuh"
#include "pipeline.cuh"
#include "prefill.cuh"
#include "tiled_layout.cuh"

// Error reporting and the launch counter, shared with the dense step (dense.cu).
namespace m1abi {

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

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

m1moe_status moe_compatible(const m1moe_cuda_ctx *moe, int hidden, int layers, int batch, int device);

}  // namespace m1abi

namespace {

using m1abi::cuda_fail;
using m1abi::fail;
using m1abi::g_last_error;
using m1abi::g_launches;

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

constexpr size_t kMaxDynSmem = 227 * 1024;  // per-CTA opt-in shared memory on sm_100
constexpr size_t kStageTarget = 40 * 1024;  // bulk copies this large run at HBM speed
size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

template <int NT>
cudaError_t launch_matvec_ring(const m1::MatvecParams &p, const m1::MatvecRing &g, int num_sms,
                               size_t smem, cudaStream_t st) {
    cudaError_t e = cudaFuncSetAttribute(m1::k_matvec4_ring<NT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const long long tiles = (long long)p.num_mats * ((p.out_dim + g.tile_rows - 1) / g.tile_rows);
    const int grid = (int)std::min<long long>(tiles, num_sms);
    m1::k_matvec4_ring<NT><<<grid, m1::kRingThreads, smem, st>>>(p, g, nullptr);
    return cudaGetLastError();
}

// Ring plan for a matvec stream, or false if the shape does not suit it
// (rows not 16-byte aligned, or too few tiles to fill the SMs).
bool plan_matvec_ring(const m1::MatvecParams &p, int nt, int num_sms, m1::MatvecRing &g,
                      size_t &smem) {
    const size_t wrow = (size_t)p.in_dim / 2, srow = (size_t)(p.in_dim / p.gs) * 2;
    if (wrow % 16 || srow % 16 || (p.num_mats > 1 && p.mat_stride % 16)) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(p.w) | reinterpret_cast<uintptr_t>(p.s) |
                         reinterpret_cast<uintptr_t>(p.b);
    if (al & 15) return false;
    // tiles of ~kStageTarget bytes (measured on config 0: 24 KB tiles stream at
    // 74 % of the HBM copy peak, 32-40 KB at 87 %, 96 KB at 82 %; 32-row tiles,
    // exactly 32 KB of weights each, at 84 %: tile offsets that are not a power
    // of two spread the CTAs' concurrent copies better)
    const size_t row = wrow + 2 * srow;
    int tr = (int)std::max<size_t>(m1::kRingRows, kStageTarget / row);
    tr = std::max(m1::kRingRows, tr / m1::kRingRows * m1::kRingRows);
    const long long tiles = (long long)p.num_mats * ((p.out_dim + tr - 1) / tr);
    if (tiles < 2LL * num_sms) return false;
    g.tile_rows = tr;
    g.stage_bytes = (int)m1::round_up_ll((long long)tr * row, 128);
    size_t off = 0;
    const size_t xs = (size_t)nt * p.in_dim * 2, xsum = (size_t)nt * (p.in_dim / m1::kChunkCols) * 8;
    const size_t fixed = align16(sizeof(m1::RingCtl)) + align16(xs) + align16(xsum);
    const size_t per_stage = (size_t)g.stage_bytes + 16;
    if (fixed + 2 * per_stage + 16 > kMaxDynSmem) return false;
    g.nstages = (int)std::min<size_t>(m1::kRingMaxStages, (kMaxDynSmem - fixed - 16) / per_stage);
    off = (size_t)g.nstages * g.stage_bytes;
    g.off_bars = (int)off;
    off = align16(off + 16 * (size_t)g.nstages);
    g.off_ctl = (int)off;
    off = align16(off + sizeof(m1::RingCtl));
    g.off_xs = (int)off;
    off = align16(off + xs);
    g.off_xsum = (int)off;
    off = align16(off + xsum);
    smem = off;
    return true;
}

template <int NT>
cudaError_t launch_matvec_nt(const m1::MatvecParams &p, int num_sms, cudaStream_t st) {
    m1::MatvecRing g;
    size_t rsmem = 0;
    if (plan_matvec_ring(p, NT, num_sms, g, rsmem)) return launch_matvec_ring<NT>(p, g, num_sms, rsmem, st);
    constexpr int R = m1::MatvecRows<NT>::R;
    const long long units = (long long)p.num_mats * ((p.out_dim + R - 1) / R);
    const long long warps = m1::kMatvecThreads / 32;
    const long long grid = std::max<long long>(1, std::min<long long>((units + warps - 1) / warps,
                                                                      3LL * num_sms));
    const size_t smem = m1::matvec_smem(NT, p.in_dim);
    cudaError_t e = cudaFuncSetAttribute(m1::k_matvec4<NT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    m1::k_matvec4<NT><<<(unsigned)grid, m1::kMatvecThreads, smem, st>>>(p);
    return cudaGetLastError();
}

#ifndef M1_SLOT_TILE_BYTES
#define M1_SLOT_TILE_BYTES (40 * 1024)
#endif
// gate/up tiles of the slot path: smaller tiles keep more of them in flight
constexpr long long kSlotTileBytes = M1_SLOT_TILE_BYTES;
static_assert(m1::kLayerSlots <= m1::kMaxStages, "slot arrays are kMaxStages long");
constexpr size_t kStagingBytes = 256u << 20;  // device staging for cold-start repacking

}  // namespace

struct m1moe_cuda_ctx {
    m1moe_cuda_cfg cfg{};
    int e0 = 0, ne = 0;
    size_t expert_bytes = 0;      // reference block size (ModelSpec.expertBytes4Bit)
    long long off[9] = {};        // reference block offsets
    m1::TiledLayout tl{};         // HBM table block layout
    uint8_t *table = nullptr;     // [layers][ne] tiled blocks
    uint16_t *router = nullptr;   // [layers][E][h]
    std::vector<uint8_t> layer_loaded, router_loaded;
    unsigned long long *xlog = nullptr;  // [nbox][box_words] tagged partial logits
    int grid = 0;                        // the layer kernel's grid (one CTA per SM)
    int nbox = 0;                        // logit boxes (CTA c polls box c % nbox)
    int box_words = 0;                   // logit_box_words(grid, E, h)
    float *acc = nullptr;                // [max_batch][h] fp32 sums for bf16 output
    int *done = nullptr;                 // [2] CTAs finished / past the exchange (accumulator output)
    unsigned *epochs = nullptr;          // per-CTA call counters (moe_layer.cuh)
    int *err = nullptr;           // device error word (pipeline.cuh kErr*)
    unsigned long long *trace = nullptr;  // optional phase timestamps (caller-owned)
    uint8_t *staging = nullptr;   // device staging for repacking host layer images
    size_t staging_bytes = 0;
    // synchronous host-buffer path
    // m1moe_cuda_moe_layer_host: device inputs [x | residual] and outputs
    // [out | idx | w], each laid out per call so that one copy moves them,
    // and a pinned host mirror of both
    float *hin = nullptr, *hio = nullptr;
    void *hpin = nullptr;           // mapped pinned: [x | residual | out | idx | w | flag]
    void *hpin_dev = nullptr;       // hpin as the device sees it
    unsigned *hflag = nullptr;      // host word k_stage_out stores the sequence number to
    unsigned *hseq_dev = nullptr;   // device copy of the last sequence number
    unsigned host_seq = 0;          // the last sequence number the host saw
    cudaStream_t stream = nullptr;  // for the *_host calls and staging copies
    void *pinned[2] = {nullptr, nullptr};
    cudaEvent_t staged[2] = {nullptr, nullptr};
    int num_sms = 148;
    // prefill (prefill.cuh): scratch for up to pf_cap tokens, grown on demand,
    // and the tensor maps of the table (made on first use)
    int pf_cap = 0, pf_nsplit = 0, pf_max_tiles = 0;
    int *pf_idx = nullptr, *pf_tok_slot = nullptr, *pf_slot_tok = nullptr, *pf_ntiles = nullptr;
    float *pf_w = nullptr, *pf_ypart = nullptr;
    m1::PfTile *pf_tiles = nullptr;
    uint8_t *pf_xg = nullptr, *pf_act = nullptr;
    bool pf_maps = false;
    CUtensorMap pf_map_gu{}, pf_map_dn{};
    // native cold-start loader (m1moe_cuda_load_expert_files): two device
    // staging buffers, a ring of pinned chunk buffers and their copy events
    void *ld_stage[2] = {nullptr, nullptr};
    void *ld_pinned[8] = {};
    cudaEvent_t ld_ev[8] = {};
    // expert parallelism over peer memory (moe_layer.cuh EpLayout)
    int ep_world = 1, ep_rank = 0, ep_b = 0;
    uint8_t *ep_region = nullptr;              // this rank's exchange region
    uint8_t *ep_peer[m1::kMaxRanks] = {};      // every rank's region as mapped here
    bool ep_ipc[m1::kMaxRanks] = {};           // mapped by cudaIpcOpenMemHandle (closed at destroy)
    bool ep_ready = false;                     // every peer mapped
    int *ep_own_idx = nullptr;                 // this rank's tokens' top-K [b][K] (route-only call)
    float *ep_own_w = nullptr;
    uint32_t ep_wait_limit = m1::kWaitLimit;   // polls of an expert-parallel flag wait
    // dynamic shared memory last set per k_moe_layer variant (a driver call
    // per launch otherwise): index by NT (1, 2, 4, 8) and the slot flag
    int layer_smem_set[4][2] = {};
    // the synchronous host call as one CUDA graph per (layer, batch, residual
    // given): copy in, the layer, copy out (m1moe_cuda_moe_layer_host)
    std::vector<cudaGraphExec_t> host_graphs;
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

// Bytes of the host call's [out | idx | w] block, a whole number of float4s.
size_t host_out_bytes(size_t B, size_t h, size_t K) { return (B * h * 4 + 2 * B * K * 4 + 15) & ~size_t(15); }

void free_ctx(m1moe_cuda_ctx *c) {
    if (!c) return;
    cudaFree(c->table);
    cudaFree(c->router);
    cudaFree(c->xlog);
    cudaFree(c->acc);
    cudaFree(c->done);
    cudaFree(c->epochs);
    cudaFree(c->err);
    cudaFree(c->staging);
    cudaFree(c->hin);
    cudaFree(c->hio);
    cudaFree(c->hseq_dev);
    if (c->hpin) cudaFreeHost(c->hpin);
    for (void *q : {(void *)c->pf_idx, (void *)c->pf_tok_slot, (void *)c->pf_slot_tok,
                    (void *)c->pf_ntiles, (void *)c->pf_w, (void *)c->pf_ypart, (void *)c->pf_tiles,
                    (void *)c->pf_xg, (void *)c->pf_act})
        cudaFree(q);
    for (int r = 0; r < m1::kMaxRanks; ++r)
        if (c->ep_ipc[r]) cudaIpcCloseMemHandle(c->ep_peer[r]);
    cudaFree(c->ep_region);
    cudaFree(c->ep_own_idx);
    cudaFree(c->ep_own_w);
    for (int i = 0; i < 2; ++i) {
        if (c->pinned[i]) cudaFreeHost(c->pinned[i]);
        if (c->staged[i]) cudaEventDestroy(c->staged[i]);
    }
    for (int i = 0; i < 2; ++i) cudaFree(c->ld_stage[i]);
    for (int i = 0; i < 8; ++i) {
        if (c->ld_pinned[i]) cudaFreeHost(c->ld_pinned[i]);
        if (c->ld_ev[i]) cudaEventDestroy(c->ld_ev[i]);
    }
    for (cudaGraphExec_t g : c->host_graphs)
        if (g) cudaGraphExecDestroy(g);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    cudaGetLastError();  // a failed free above must not surface in a later call
}

#ifndef M1_BOX_SHARE
#define M1_BOX_SHARE 4
#endif
constexpr int kBoxShare = M1_BOX_SHARE;  // CTAs polling one logit box
constexpr size_t kEpochBytes = (size_t)m1::kMaxCtas * m1::kEpochStride * sizeof(unsigned);

// Partial sums per router logit: h is cut into `parts` column ranges, each
// summed by its own CTA, so that up to E*parts CTAs share the router product
// instead of E.  At least 256 (token, 8-column block) pairs per part, at most
// 16 parts, and the box (ntok*E*parts tagged words) within
// kMaxTok*kMaxExperts words.  (The row-group kernels use one part.)
int logit_parts(int grid, int E, int ntok, int h) {
    int P = std::min(std::max(1, grid / E), 16);
    P = std::min(P, std::max(1, ntok * h / 2048));
    while (P > 1 && ntok * E * P > m1::kMaxTok * m1::kMaxExperts) --P;
    return P;
}

// Words of one logit box: the largest ntok*E*parts of any batch.
int logit_box_words(int grid, int E, int h) {
    int w = 0;
    for (int b = 1; b <= m1::kMaxTok; ++b) w = std::max(w, b * E * logit_parts(grid, E, b, h));
    return w;
}

// Zero the epoch words and the tagged logits (tag 0 is never a call's tag,
// so no stale word can match after this).
cudaError_t clear_exchange(m1moe_cuda_ctx *c) {
    cudaError_t e = cudaMemset(c->epochs, 0, kEpochBytes);
    if (e == cudaSuccess) e = cudaMemset(c->done, 0, 8);
    if (e == cudaSuccess) e = cudaMemset(c->xlog, 0, (size_t)c->nbox * c->box_words * 8);
    return e;
}

m1::LayerParams layer_params(m1moe_cuda_ctx *c, int layer, int B) {
    m1::LayerParams p{};
    const m1moe_cuda_cfg &g = c->cfg;
    p.table = c->table + (size_t)layer * c->ne * c->tl.block;
    p.tl = c->tl;
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
    p.xlog = c->xlog;
    p.nbox = c->nbox;
    p.box_words = c->box_words;
    p.acc = c->acc;
    p.done = c->done;
    p.epochs = c->epochs;
    p.err = c->err;
    p.ep_wait_limit = c->ep_wait_limit;
    p.trace = c->trace;
    return p;
}


// Largest divisor of n that is a multiple of m and at most cap (>= m).
int divisor_tile(int n, int m, long long cap) {
    int best = m;
    for (int d = m; d <= n; d += m)
        if (n % d == 0 && d <= cap) best = d;
    return best;
}

// Shared-memory map of a routing-only call (route_only): the kernel stops
// after the top-K and weights, so it needs no x staging, tile ring or
// activation buffers -- only the control block, the ranking keys and logits,
// the slot arrays and, in the ring's place, room for the partial logits
// (at most kMaxTok * kMaxExperts floats).  Fits an SM for any hidden size.
size_t plan_route_only(m1::LayerParams &p, int grid, int nt, bool slot) {
    p.fd_G = m1::make_fastdiv(grid);
    p.bal_beta = 0;  // no row split to compute
    p.ring_bytes = m1::kMaxTok * m1::kMaxExperts * 4;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align16(off + bytes);
        return at;
    };
    const size_t ctl = take(sizeof(m1::Ctl));
    const size_t dummy = take(16);  // the unused regions all point here
    const size_t keys = take((size_t)nt * p.E * 8);
    const size_t rlog = take((size_t)nt * p.E * 4);
    const size_t lpart = take(8 * m1::kMaxTok * 4);
    const size_t slots = slot ? take(sizeof(m1::Slots)) : 0;
    const size_t bars = (size_t)p.ring_bytes;
    const size_t base = align16(bars + 2 * sizeof(uint64_t) * (size_t)m1::kLayerSlots);
    p.off_bars = (int)bars;
    p.off_ctl = (int)(base + ctl);
    p.off_xs = p.off_xsum = p.off_gup = p.off_actf = p.off_act = p.off_xseg = p.off_blk =
        (int)(base + dummy);
    p.off_keys = (int)(base + keys);
    p.off_rlog = (int)(base + rlog);
    p.off_lpart = (int)(base + lpart);
    p.off_slots = (int)(base + slots);
    return base + off;
}

// Plan tiles, stages and the shared-memory map of k_moe_layer<nt>.  Returns
// the dynamic shared memory size, or 0 if the shape does not fit an SM.
size_t plan_layer(m1::LayerParams &p, int grid, int nt, bool slot) {
    if (p.route_only) return plan_route_only(p, grid, nt, slot);
    const m1::TiledLayout &tl = p.tl;
    const int nch = p.h / m1::kChunkCols;
    const int maxU = std::min(p.ntok * p.K, p.ne);
    const int gcb = p.gs / 8;  // column blocks per group
    if (tl.rc / 32 > m1::kConsumerWarps) return 0;  // see down_row_chunk
    // down tile: a run of column blocks (a multiple of gcb) of one row chunk,
    // plus the scale/bias words of its groups; as large as kStageTarget allows
    const long long per_group = (long long)(gcb + 1) * tl.rc * 4;
    p.dn_max_cb = gcb * (int)std::max<long long>(1, (long long)kStageTarget / per_group);
    const long long dn_bytes = (long long)p.dn_max_cb * tl.rc * 4 + (long long)(p.dn_max_cb / gcb) * tl.rc * 4;
    // gate/up tile: GT pair-rows, GT | I and 8 | GT (row pairs R, R+4 stay in
    // one tile), filling the stage the down tiles need (at least kStageTarget/2)
    const long long stage_target = std::max<long long>(dn_bytes, kStageTarget / 2);
    // (the slot path has no row pairs: any multiple of 4 rows)
    const int gmul = slot ? 4 : 8;
    const long long gu_target = slot ? std::min<long long>(stage_target, kSlotTileBytes) : stage_target;
    p.gu_tile_rows = divisor_tile(p.I, gmul, std::max<long long>(gmul, gu_target / tl.pr));
    p.stage_bytes = (int)m1::round_up_ll(std::max<long long>(p.gu_tile_rows * tl.pr, dn_bytes), 128);
    p.gu_nslices = (!slot && nt <= 2) ? (nch + 31) / 32 : 1;
    p.nic = p.h / tl.rc;
    p.fd_G = m1::make_fastdiv(grid);
    p.fd_GT = m1::make_fastdiv(p.gu_tile_rows);
    p.fd_I = m1::make_fastdiv(p.I);
    p.fd_ncbE = m1::make_fastdiv(p.I / 8);
    p.fd_gcb = m1::make_fastdiv(gcb);
    p.fd_gs = m1::make_fastdiv(p.gs);
    p.fd_iptg = m1::make_fastdiv(m1::gu_items_per_tile(slot, nt, p.gu_tile_rows, p.gu_nslices));
    p.fd_nslg = m1::make_fastdiv(p.gu_nslices);
    if (tl.rc % (32 * m1::dn_lane_rows(slot, nt))) return 0;
    p.fd_iptd = m1::make_fastdiv(tl.rc / (32 * m1::dn_lane_rows(slot, nt)));
    // rows per CTA: an even split, or the cost-weighted one (route_geometry):
    // a CTA's cost share is at most ceil(total / grid) and a unit costs at
    // least beta + 1, so it gets at most share / (beta + 1) + 1 units
    const long long n8 = p.I / 8;
    p.bal_beta = p.ntok > 1 ? m1::kBalBeta : 0;
    if (p.bal_beta == 0) {
        const long long units = (long long)maxU * n8;
        p.gu_rows_max = (int)((units + grid - 1) / grid) * 8;
    } else {
        const long long pairs = (long long)p.ntok * std::min(p.K, p.ne);
        const long long total = n8 * (p.bal_beta * (long long)maxU + pairs);
        if (total * grid >= (1LL << 31)) return 0;  // route_geometry's int costs
        const long long share = (total + grid - 1) / grid;
        p.gu_rows_max = (int)std::min<long long>(share / (p.bal_beta + 1) + 2, maxU * n8) * 8;
    }
    p.act_cb = p.gu_rows_max / 8;
    p.xseg_max = p.gu_rows_max / p.gs + 2;
    // fixed part of the shared-memory map (after the ring and its barriers)
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align16(off + bytes);
        return at;
    };
    const size_t ctl = take(sizeof(m1::Ctl));
    const size_t xs = take((size_t)nt * p.h * 2);
    const size_t xsum = take((size_t)nt * nch * 8);
    const size_t gup = take(p.gu_nslices > 1 ? (size_t)p.gu_rows_max * p.gu_nslices * 2 * nt * 4 : 16);
    const size_t actf = take((size_t)nt * p.act_cb * 8 * 4);
    // the int16 activations and block statistics are written once gate/up is
    // done; the slot path places them over the staged x, which is dead then
    const size_t act_bytes = align16((size_t)nt * p.act_cb * 16), blk_bytes = (size_t)nt * p.act_cb * 8;
    const bool alias_x = slot && act_bytes + blk_bytes <= (size_t)nt * p.h * 2;
    const size_t act = alias_x ? xs : take(act_bytes);
    const size_t xseg = take((size_t)nt * p.xseg_max * 8);
    const size_t blk = alias_x ? xs + act_bytes : take(blk_bytes);
    const size_t keys = take((size_t)nt * p.E * 8);
    const size_t rlog = take((size_t)nt * p.E * 4);
    const size_t lpart = take(8 * m1::kMaxTok * 4);
    const size_t slots = slot ? take(sizeof(m1::Slots)) : 0;
    const size_t fixed = off;
    // the tile ring: everything else, tiles packed back to back, at most
    // kLayerSlots of them in flight (each slot has a full and an empty barrier)
    const size_t bar_bytes = 2 * sizeof(uint64_t) * (size_t)m1::kLayerSlots;
    if (fixed + bar_bytes + 32 > kMaxDynSmem) return 0;
    p.ring_bytes = (int)((kMaxDynSmem - fixed - bar_bytes - 16) / 128 * 128);
    if (p.ring_bytes < 2 * p.stage_bytes) return 0;
    const size_t bars = (size_t)p.ring_bytes;
    const size_t base = align16(bars + bar_bytes);
    p.off_bars = (int)bars;
    p.off_ctl = (int)(base + ctl);
    p.off_xs = (int)(base + xs);
    p.off_xsum = (int)(base + xsum);
    p.off_gup = (int)(base + gup);
    p.off_actf = (int)(base + actf);
    p.off_act = (int)(base + act);
    p.off_xseg = (int)(base + xseg);
    p.off_blk = (int)(base + blk);
    p.off_keys = (int)(base + keys);
    p.off_rlog = (int)(base + rlog);
    p.off_lpart = (int)(base + lpart);
    p.off_slots = (int)(base + slots);
    return base + fixed;
}

template <int NT, bool SL>
m1moe_status launch_layer(m1moe_cuda_ctx *c, m1::LayerParams p, cudaStream_t st) {
    const int grid = c->grid;  // one CTA per SM
    p.lparts = SL ? logit_parts(grid, p.E, NT, p.h) : 1;  // slot path: boxes padded to NT tokens
    const size_t smem = plan_layer(p, grid, NT, SL);
    if (smem == 0 || smem > kMaxDynSmem)
        return fail(M1MOE_ERR_UNSUPPORTED, "shape needs more shared memory than an SM has");
    {
        int &set = c->layer_smem_set[NT == 1 ? 0 : (NT == 2 ? 1 : (NT == 4 ? 2 : 3))][SL ? 1 : 0];
        if (set < (int)smem) {
            M1_CK(cudaFuncSetAttribute(m1::k_moe_layer<NT, SL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
            set = (int)smem;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(m1::kLayerThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    // Cooperative: every CTA is resident at once, which the waits on other
    // CTAs need.  Programmatic stream serialisation: the launch may be
    // scheduled while the previous kernel in the stream finishes (the kernel
    // waits for that grid before touching memory), hiding the launch gap.
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, m1::k_moe_layer<NT, SL>, p);
    if (e != cudaSuccess) return cuda_fail(e, "k_moe_layer launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return M1MOE_OK;
}

m1moe_status dispatch_layer(m1moe_cuda_ctx *c, const m1::LayerParams &p, cudaStream_t st) {
    if (p.ntok == 1) return launch_layer<1, false>(c, p, st);
    if (p.ntok == 2)
        return m1::slot_path(2, p.h) ? launch_layer<2, true>(c, p, st) : launch_layer<2, false>(c, p, st);
    if (p.ntok <= 4) return launch_layer<4, true>(c, p, st);
    return launch_layer<8, true>(c, p, st);
}

// ---- router top-K without allocation (m1moe_cuda_router_topk_noalloc) ----
// Scratch of the k_moe_layer routing pass in a file-scope device array instead
// of a context's cudaMalloc'd buffers: the tagged logits (8 tokens x 256
// experts x 8 bytes) and one 128-byte epoch line per CTA for up to 256 CTAs.
// 49,152 bytes on every GPU that loads the library.  (The device error word
// is the caller's d_status.)
constexpr int kNoAllocMaxCtas = 256;
constexpr size_t kNoAllocXlog = (size_t)m1::kMaxTok * m1::kMaxExperts * 8;
constexpr size_t kNoAllocEpochs = (size_t)kNoAllocMaxCtas * m1::kEpochStride * 4;
constexpr size_t kNoAllocBytes = kNoAllocXlog + kNoAllocEpochs;
static __device__ __align__(256) uint8_t g_route_scratch[kNoAllocBytes];

// Per-device address of g_route_scratch (host code cannot use the symbol as a
// device address) and SM count, looked up once with that device current.
constexpr int kNoAllocMaxDevices = 64;
struct NoAllocDevice {
    std::atomic<int> ready{0};
    uint8_t *scratch = nullptr;
    int num_sms = 0;
};
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

m1moe_status noalloc_setup(int dev, NoAllocDevice *&out) {
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(M1MOE_ERR_UNSUPPORTED, "device %d beyond %d", dev, kNoAllocMaxDevices);
    NoAllocDevice &d = g_noalloc_dev[dev];
    if (!d.ready.load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!d.ready.load(std::memory_order_relaxed)) {
            void *ptr = nullptr;
            M1_CK(cudaGetSymbolAddress(&ptr, g_route_scratch));
            // epoch words and logit tags must start equal (zero) on every CTA
            M1_CK(cudaMemset(ptr, 0, kNoAllocBytes));
            M1_CK(cudaDeviceSynchronize());
            int n = 0;
            M1_CK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
            d.scratch = static_cast<uint8_t *>(ptr);
            d.num_sms = n > 0 ? n : 148;
            d.ready.store(1, std::memory_order_release);
        }
    }
    out = &d;
    return M1MOE_OK;
}

template <int NT, bool SL>
m1moe_status launch_route_noalloc(m1::LayerParams p, int grid, cudaStream_t st) {
    p.lparts = SL ? logit_parts(grid, p.E, NT, p.h) : 1;
    const size_t smem = plan_layer(p, grid, NT, SL);
    if (smem == 0 || smem > kMaxDynSmem)
        return fail(M1MOE_ERR_UNSUPPORTED, "shape needs more shared memory than an SM has");
    M1_CK(cudaFuncSetAttribute(m1::k_moe_layer<NT, SL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(m1::kLayerThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, m1::k_moe_layer<NT, SL>, p);
    if (e != cudaSuccess) return cuda_fail(e, "k_moe_layer (routing) launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return M1MOE_OK;
}

m1moe_status check_layer(m1moe_cuda_ctx *c, int32_t layer) {
    if (!c) return fail(M1MOE_ERR_INVALID_ARG, "ctx is NULL");
    if (layer < 0 || layer >= c->cfg.num_layers)
        return fail(M1MOE_ERR_INVALID_ARG, "layer %d out of range [0,%d)", layer, c->cfg.num_layers);
    return M1MOE_OK;
}

// Repack `n` reference-layout expert blocks at d_src (device) into the table.
m1moe_status repack_experts(m1moe_cuda_ctx *c, const uint8_t *d_src, uint8_t *d_dst, int n,
                            cudaStream_t st) {
    m1::RefOffsets ro;
    for (int i = 0; i < 9; ++i) ro.off[i] = c->off[i];
    const long long rows = (long long)n * (c->cfg.intermediate_dim + c->cfg.hidden_dim);
    const int grid = (int)std::min<long long>(rows, 64LL * c->num_sms);
    m1::k_repack_tiled<<<grid, 128, 0, st>>>(d_src, (long long)c->expert_bytes, d_dst, c->tl, ro, n,
                                              c->cfg.hidden_dim, c->cfg.intermediate_dim,
                                              c->cfg.group_size);
    M1_LAUNCHED();
    return M1MOE_OK;
}

// ---------------------------------------------------------------- prefill ----
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The two tensor maps of the table: gate/up pair-rows as bytes [blocks][I][pr]
// (box 32 bytes x 128 rows: one 64-column step of 128 rows), and the down
// words [blocks][h/rc * I/8][rc] (box 128 rows x 8 column blocks).
m1moe_status pf_make_maps(m1moe_cuda_ctx *c) {
    if (c->pf_maps) return M1MOE_OK;
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    M1_CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (!fn || q != cudaDriverEntryPointSuccess)
        return fail(M1MOE_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    auto encode = reinterpret_cast<EncodeTiledFn>(fn);
    const m1::TiledLayout &tl = c->tl;
    const cuuint64_t nblk = (cuuint64_t)c->cfg.num_layers * c->ne;
    const cuuint32_t one[3] = {1, 1, 1};
    {
        const cuuint64_t dims[3] = {(cuuint64_t)tl.pr, (cuuint64_t)c->cfg.intermediate_dim, nblk};
        const cuuint64_t strides[2] = {(cuuint64_t)tl.pr, (cuuint64_t)tl.block};
        const cuuint32_t box[3] = {32, (cuuint32_t)m1::kPfRows, 1};
        const CUresult r = encode(&c->pf_map_gu, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, c->table, dims,
                                  strides, box, one, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(M1MOE_ERR_CUDA, "gate/up tensor map: error %d", (int)r);
    }
    {
        const cuuint64_t dims[3] = {(cuuint64_t)tl.rc,
                                    (cuuint64_t)(c->cfg.hidden_dim / tl.rc) * tl.ncbI, nblk};
        const cuuint64_t strides[2] = {(cuuint64_t)tl.rc * 4, (cuuint64_t)tl.block};
        const cuuint32_t box[3] = {(cuuint32_t)m1::kPfRows, 8, 1};
        const CUresult r = encode(&c->pf_map_dn, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3,
                                  c->table + tl.dn_w, dims, strides, box, one,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(M1MOE_ERR_CUDA, "down tensor map: error %d", (int)r);
    }
    c->pf_maps = true;
    return M1MOE_OK;
}

// Scratch for T tokens (grown, never shrunk; a synchronous reallocation).
m1moe_status pf_reserve(m1moe_cuda_ctx *c, int T) {
    if (T <= c->pf_cap) return M1MOE_OK;
    const m1moe_cuda_cfg &g = c->cfg;
    const long long pairs = (long long)T * g.top_k;
    const int max_tiles = (int)std::min<long long>(c->ne, pairs) + (int)(pairs / m1::kPfTileTok) + 1;
    const long long rows = pairs + 16LL * max_tiles;  // padded tile rows
    // K splits of the down product: about four units per SM for one tile per
    // used expert, each split at least 8 steps of 64 columns
    const long long dn_units = (long long)std::min<long long>(c->ne, pairs) * (g.hidden_dim / m1::kPfRows);
    int nsplit = (int)std::max<long long>(1, (4LL * c->num_sms + dn_units - 1) / dn_units);
    nsplit = std::min(nsplit, std::max(1, g.intermediate_dim / 64 / 8));
    M1_CK(cudaDeviceSynchronize());
    for (void *q : {(void *)c->pf_idx, (void *)c->pf_tok_slot, (void *)c->pf_slot_tok,
                    (void *)c->pf_ntiles, (void *)c->pf_w, (void *)c->pf_ypart, (void *)c->pf_tiles,
                    (void *)c->pf_xg, (void *)c->pf_act})
        cudaFree(q);
    c->pf_idx = c->pf_tok_slot = c->pf_slot_tok = c->pf_ntiles = nullptr;
    c->pf_w = c->pf_ypart = nullptr;
    c->pf_tiles = nullptr;
    c->pf_xg = c->pf_act = nullptr;
    c->pf_cap = 0;
    M1_CK(cudaMalloc((void **)&c->pf_idx, pairs * 4));
    M1_CK(cudaMalloc((void **)&c->pf_tok_slot, pairs * 4));
    M1_CK(cudaMalloc((void **)&c->pf_slot_tok, pairs * 4));
    M1_CK(cudaMalloc((void **)&c->pf_ntiles, 4));
    M1_CK(cudaMalloc((void **)&c->pf_w, pairs * 4));
    M1_CK(cudaMalloc((void **)&c->pf_ypart, (size_t)nsplit * pairs * g.hidden_dim * 4));
    M1_CK(cudaMalloc((void **)&c->pf_tiles, (size_t)max_tiles * sizeof(m1::PfTile)));
    M1_CK(cudaMalloc((void **)&c->pf_xg, (size_t)rows * g.hidden_dim * 2));
    M1_CK(cudaMalloc((void **)&c->pf_act, (size_t)rows * g.intermediate_dim * 2));
    c->pf_cap = T;
    c->pf_nsplit = nsplit;
    c->pf_max_tiles = max_tiles;
    return M1MOE_OK;
}

template <int KIND>
m1moe_status pf_gemm(m1moe_cuda_ctx *c, const m1::PrefillParams &p, const CUtensorMap &map,
                     cudaStream_t st) {
    const int smem = m1::PfStage<KIND>::smem;
    M1_CK(cudaFuncSetAttribute(m1::k_prefill_gemm<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem));
    m1::k_prefill_gemm<KIND><<<c->num_sms, m1::kPfThreads, smem, st>>>(p, map);
    M1_LAUNCHED();
    return M1MOE_OK;
}

}  // namespace

m1moe_status m1abi::moe_compatible(const m1moe_cuda_ctx *c, int hidden, int layers, int batch,
                                   int device) {
    if (!c) return fail(M1MOE_ERR_INVALID_ARG, "MoE ctx is NULL");
    if (c->cfg.hidden_dim != hidden || c->cfg.num_layers != layers || c->cfg.device != device)
        return fail(M1MOE_ERR_INVALID_ARG,
                    "MoE context (hidden %d, %d layers, device %d) does not match the dense one "
                    "(hidden %d, %d layers, device %d)",
                    c->cfg.hidden_dim, c->cfg.num_layers, c->cfg.device, hidden, layers, device);
    if (batch > c->cfg.max_batch)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d above the MoE context's max_batch %d", batch,
                    c->cfg.max_batch);
    return M1MOE_OK;
}

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
    if (g.hidden_dim % 128 || g.intermediate_dim % 64)
        return fail(M1MOE_ERR_INVALID_ARG,
                    "hidden_dim must be a multiple of 128 and intermediate_dim of 64");
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
    c->tl = m1::make_tiled_layout(g.hidden_dim, g.intermediate_dim, g.group_size);
    c->layer_loaded.assign(g.num_layers, 0);
    c->router_loaded.assign(g.num_layers, 0);
    c->num_sms = sm_count();
    c->grid = std::min(c->num_sms, m1::kMaxCtas);
    c->nbox = (c->grid + kBoxShare - 1) / kBoxShare;
    c->box_words = logit_box_words(c->grid, g.num_experts, g.hidden_dim);
    const size_t B = g.max_batch, E = g.num_experts, K = g.top_k;
    cudaError_t e;
#define M1_ALLOC(ptr, bytes)                                        \
    e = cudaMalloc((void **)&(ptr), (bytes));                       \
    if (e != cudaSuccess) {                                         \
        m1moe_status st_ = cuda_fail(e, "cudaMalloc " #ptr);       \
        free_ctx(c);                                                \
        return st_;                                                 \
    }
    M1_ALLOC(c->table, (size_t)g.num_layers * ne * c->tl.block);
    M1_ALLOC(c->router, (size_t)g.num_layers * E * g.hidden_dim * 2);
    M1_ALLOC(c->xlog, (size_t)c->nbox * c->box_words * 8);
    M1_ALLOC(c->acc, B * g.hidden_dim * 4);
    M1_ALLOC(c->done, 8);
    M1_ALLOC(c->epochs, kEpochBytes);
    M1_ALLOC(c->err, 4);
    M1_ALLOC(c->hin, 2 * B * g.hidden_dim * 4);
    M1_ALLOC(c->hio, host_out_bytes(B, g.hidden_dim, K));
    M1_ALLOC(c->hseq_dev, 4);
#undef M1_ALLOC
    {
        // [x | residual] (2·B·h floats), [out | idx | w] rounded up to 16
        // bytes, then the flag word on its own 64 bytes
        const size_t in_b = 2 * B * g.hidden_dim * 4, out_b = host_out_bytes(B, g.hidden_dim, K);
        e = cudaHostAlloc(&c->hpin, in_b + out_b + 64, cudaHostAllocMapped);
        if (e == cudaSuccess) e = cudaHostGetDevicePointer(&c->hpin_dev, c->hpin, 0);
        if (e != cudaSuccess) {
            m1moe_status st_ = cuda_fail(e, "cudaHostAlloc host-call staging");
            free_ctx(c);
            return st_;
        }
        c->hflag = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(c->hpin) + in_b + out_b);
        *reinterpret_cast<volatile unsigned *>(c->hflag) = 0;
    }
    e = cudaMemset(c->err, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(c->hseq_dev, 0, 4);
    if (e == cudaSuccess) e = clear_exchange(c);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        m1moe_status st = cuda_fail(e, "context setup");
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
    // Host image -> pinned bounce buffers (double-buffered) -> device staging
    // (whole experts) -> repack into the tiled table.
    const size_t chunk = 32u << 20;
    if (!c->pinned[0]) {
        for (int i = 0; i < 2; ++i) {
            M1_CK(cudaHostAlloc(&c->pinned[i], chunk, cudaHostAllocDefault));
            M1_CK(cudaEventCreateWithFlags(&c->staged[i], cudaEventDisableTiming));
        }
    }
    const int per = (int)std::max<size_t>(1, kStagingBytes / c->expert_bytes);
    if (!c->staging) {
        c->staging_bytes = (size_t)std::min(per, c->ne) * c->expert_bytes;
        M1_CK(cudaMalloc(&c->staging, c->staging_bytes));
    }
    const uint8_t *src = static_cast<const uint8_t *>(h_bytes) + (size_t)c->e0 * c->expert_bytes;
    uint8_t *dst = c->table + (size_t)layer * c->ne * c->tl.block;
    int buf = 0;
    bool used[2] = {false, false};
    for (int e = 0; e < c->ne; e += per) {
        const int n = std::min(per, c->ne - e);
        const size_t total = (size_t)n * c->expert_bytes;
        const uint8_t *s = src + (size_t)e * c->expert_bytes;
        for (size_t done = 0; done < total; done += chunk, buf ^= 1) {
            const size_t m = std::min(chunk, total - done);
            if (used[buf]) M1_CK(cudaEventSynchronize(c->staged[buf]));
            memcpy(c->pinned[buf], s + done, m);
            M1_CK(cudaMemcpyAsync(c->staging + done, c->pinned[buf], m, cudaMemcpyHostToDevice,
                                  c->stream));
            M1_CK(cudaEventRecord(c->staged[buf], c->stream));
            used[buf] = true;
        }
        if (m1moe_status st = repack_experts(c, c->staging, dst + (size_t)e * c->tl.block, n, c->stream))
            return st;
        M1_CK(cudaStreamSynchronize(c->stream));  // staging is reused by the next experts
    }
    c->layer_loaded[layer] = 1;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_load_expert_files(m1moe_cuda_ctx *c, const char *dir, int32_t io_threads) {
    if (!c || !dir) return fail(M1MOE_ERR_INVALID_ARG, "ctx/dir is NULL");
    const m1moe_cuda_cfg &g = c->cfg;
    const size_t eb = c->expert_bytes, want = (size_t)g.num_experts * eb;
    const int nthr = std::max(1, std::min<int>(io_threads, 64));
    // every file is checked before any copy: a missing or short file fails the
    // whole load (the converter's size check, extract_olmoe.py:340-344; the
    // reference engine would silently zero the expert, InferenceEngine.swift
    // :274-279)
    std::vector<int> fds(g.num_layers, -1);
    auto close_all = [&]() {
        for (int fd : fds)
            if (fd >= 0) close(fd);
    };
    for (int L = 0; L < g.num_layers; ++L) {
        char path[4096];
        snprintf(path, sizeof(path), "%s/layer_%02d.bin", dir, L);
        fds[L] = open(path, O_RDONLY);
        struct stat st;
        if (fds[L] < 0 || fstat(fds[L], &st) != 0) {
            close_all();
            return fail(M1MOE_ERR_INVALID_ARG, "%s: cannot open (%s)", path, strerror(errno));
        }
        if ((size_t)st.st_size != want) {
            close_all();
            return fail(M1MOE_ERR_INVALID_ARG, "%s: %lld bytes, expected %zu (= %d experts x %zu)", path,
                        (long long)st.st_size, want, g.num_experts, eb);
        }
#ifdef POSIX_FADV_SEQUENTIAL
        posix_fadvise(fds[L], 0, 0, POSIX_FADV_SEQUENTIAL);
#endif
    }
    DeviceGuard dg(g.device);
    // Work list: per layer, groups of `per` experts of this shard (one device
    // staging buffer each, two buffers alternating), each group cut into
    // chunks read by the io threads into a ring of pinned buffers.  Copies and
    // repacks go on one stream, so a staging buffer is reused only after the
    // repack that read it.
    const size_t chunk = 32u << 20;
    constexpr int R = 8;  // pinned ring slots
    const int per = (int)std::max<size_t>(1, (kStagingBytes / 2) / eb);
    struct Chunk {
        int layer, group, e;  // group's first expert (shard-relative) and experts in it
        int ng;
        size_t file_off, stage_off, bytes;
        bool last;
    };
    std::vector<Chunk> work;
    int ngroups = 0;
    for (int L = 0; L < g.num_layers; ++L)
        for (int e = 0; e < c->ne; e += per, ++ngroups) {
            const int n = std::min(per, c->ne - e);
            const size_t total = (size_t)n * eb, base = (size_t)(c->e0 + e) * eb;
            for (size_t off = 0; off < total; off += chunk)
                work.push_back({L, ngroups, e, n, base + off, off, std::min(chunk, total - off),
                                off + chunk >= total});
        }
    if (!c->ld_stage[0]) {
        const size_t sb = (size_t)std::min(per, c->ne) * eb;
        M1_CK(cudaMalloc(&c->ld_stage[0], sb));
        M1_CK(cudaMalloc(&c->ld_stage[1], sb));
    }
    if (!c->ld_pinned[0]) {
        for (int i = 0; i < R; ++i) {
            M1_CK(cudaHostAlloc(&c->ld_pinned[i], chunk, cudaHostAllocDefault));
            M1_CK(cudaEventCreateWithFlags(&c->ld_ev[i], cudaEventDisableTiming));
        }
    }
    const long long nwork = (long long)work.size();
    std::mutex mu;
    std::condition_variable cv;
    std::vector<uint8_t> ready(nwork, 0);
    long long consumed = 0;           // chunks whose copy the main thread has issued
    std::atomic<long long> next{0};   // next chunk for an io thread
    std::atomic<bool> stop{false};
    std::string io_err;
    auto worker = [&]() {
        for (;;) {
            const long long k = next.fetch_add(1);
            if (k >= nwork || stop.load()) return;
            const int slot = (int)(k % R);
            {
                // the slot's previous chunk (k - R) must have been handed to the GPU ...
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [&] { return consumed > k - R || stop.load(); });
            }
            if (stop.load()) return;
            // ... and copied out of the slot
            if (k >= R && cudaEventSynchronize(c->ld_ev[slot]) != cudaSuccess) {
                std::lock_guard<std::mutex> lk(mu);
                io_err = "waiting for a pinned buffer's copy failed";
                stop = true;
                cv.notify_all();
                return;
            }
            const Chunk &w = work[k];
            uint8_t *dst = static_cast<uint8_t *>(c->ld_pinned[slot]);
            size_t got = 0;
            while (got < w.bytes) {
                const ssize_t r = pread(fds[w.layer], dst + got, w.bytes - got, (off_t)(w.file_off + got));
                if (r <= 0) break;
                got += (size_t)r;
            }
            std::lock_guard<std::mutex> lk(mu);
            if (got != w.bytes) {
                char buf[256];
                snprintf(buf, sizeof(buf), "layer_%02d.bin: short read at byte %zu", w.layer,
                         w.file_off + got);
                io_err = buf;
                stop = true;
            }
            ready[k] = 1;
            cv.notify_all();
        }
    };
    std::vector<std::thread> pool;
    for (int i = 0; i < nthr; ++i) pool.emplace_back(worker);
    m1moe_status st = M1MOE_OK;
    for (long long k = 0; k < nwork && st == M1MOE_OK; ++k) {
        {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return ready[k] || stop.load(); });
            if (stop.load() && !io_err.empty()) {
                st = fail(M1MOE_ERR_INVALID_ARG, "%s", io_err.c_str());
                break;
            }
        }
        const Chunk &w = work[k];
        const int slot = (int)(k % R);
        uint8_t *stage = static_cast<uint8_t *>(c->ld_stage[w.group & 1]);
        cudaError_t e = cudaMemcpyAsync(stage + w.stage_off, c->ld_pinned[slot], w.bytes,
                                        cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess) e = cudaEventRecord(c->ld_ev[slot], c->stream);
        if (e != cudaSuccess) {
            st = cuda_fail(e, "expert file copy");
            break;
        }
        if (w.last) {
            uint8_t *dst = c->table + ((size_t)w.layer * c->ne + w.e) * c->tl.block;
            st = repack_experts(c, stage, dst, w.ng, c->stream);
        }
        {
            std::lock_guard<std::mutex> lk(mu);
            consumed = k + 1;
        }
        cv.notify_all();
    }
    {
        std::lock_guard<std::mutex> lk(mu);
        if (st != M1MOE_OK) stop = true;
        consumed = nwork + R;
    }
    cv.notify_all();
    for (auto &t : pool) t.join();
    close_all();
    const cudaError_t e = cudaStreamSynchronize(c->stream);
    if (st != M1MOE_OK) return st;
    if (e != cudaSuccess) return cuda_fail(e, "expert file load");
    for (int L = 0; L < g.num_layers; ++L) c->layer_loaded[L] = 1;
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
    if (m1moe_status st = repack_experts(
            c, static_cast<const uint8_t *>(d_bytes) + (size_t)c->e0 * c->expert_bytes,
            c->table + (size_t)layer * c->ne * c->tl.block, c->ne, as_stream(stream)))
        return st;
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
    p.y_ntok = batch;
    if (m1::matvec_smem(1, in_dim) > kMaxDynSmem)
        return fail(M1MOE_ERR_UNSUPPORTED, "in_dim %d does not fit shared memory", in_dim);
    const int nsm = sm_count();
    cudaStream_t st = as_stream(stream);
    // Tokens go in groups whose staged x fits one CTA's shared memory (each
    // group reads the weights once more).
    const size_t xtok = (size_t)in_dim * (x_dtype == M1MOE_DTYPE_BF16 ? 2 : 4);
    for (int t0 = 0; t0 < batch;) {
        int n = batch - t0;
        auto nt_of = [](int k) { return k <= 2 ? k : (k <= 4 ? 4 : 8); };
        while (m1::matvec_smem(nt_of(n), in_dim) > kMaxDynSmem) n = n > 4 ? 4 : (n > 2 ? 2 : 1);
        m1::MatvecParams q = p;
        q.x = static_cast<const uint8_t *>(d_x) + (size_t)t0 * xtok;
        q.ntok = n;
        q.y_t0 = t0;
        cudaError_t e;
        if (n == 1) e = launch_matvec_nt<1>(q, nsm, st);
        else if (n == 2) e = launch_matvec_nt<2>(q, nsm, st);
        else if (n <= 4) e = launch_matvec_nt<4>(q, nsm, st);
        else e = launch_matvec_nt<8>(q, nsm, st);
        if (e != cudaSuccess) return cuda_fail(e, "k_matvec4 launch");
        g_launches.fetch_add(1, std::memory_order_relaxed);
        t0 += n;
    }
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
    m1::LayerParams p = layer_params(c, layer, B);
    p.x = d_x;
    p.x_bf16 = x_dtype == M1MOE_DTYPE_BF16;
    p.user_idx = d_idx;
    p.user_w = d_w;
    p.user_scores = d_scores;
    p.route_only = 1;
    return dispatch_layer(c, p, as_stream(stream));
}

m1moe_status m1moe_cuda_router_topk_noalloc(const uint16_t *d_router, int32_t num_experts,
                                            int32_t hidden_dim, int32_t top_k,
                                            int32_t norm_topk_prob, const void *d_x,
                                            int32_t x_dtype, int32_t B, int32_t *d_idx, float *d_w,
                                            float *d_scores, int32_t *d_status, void *stream) {
    const int E = num_experts, h = hidden_dim, K = top_k;
    if (!d_router || !d_x || !valid_dtype(x_dtype))
        return fail(M1MOE_ERR_INVALID_ARG, "router/x/x_dtype invalid");
    if (E < 1 || E > m1::kMaxExperts)
        return fail(M1MOE_ERR_INVALID_ARG, "num_experts %d outside [1,%d] (fixed scratch size)", E,
                    m1::kMaxExperts);
    if (K < 1 || K > E || K > m1::kMaxTopK)
        return fail(M1MOE_ERR_INVALID_ARG, "top_k %d invalid", K);
    if (B < 1 || B > m1::kMaxTok)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d outside [1,%d] (fixed scratch size)", B,
                    m1::kMaxTok);
    if (h <= 0 || h % 64)
        return fail(M1MOE_ERR_INVALID_ARG, "hidden_dim %d must be a positive multiple of 64", h);
    if ((reinterpret_cast<uintptr_t>(d_router) | reinterpret_cast<uintptr_t>(d_x)) & 15)
        return fail(M1MOE_ERR_INVALID_ARG, "router and x must be 16-byte aligned");
    // The call is stream-ordered, so a device-side failure can only reach the
    // caller through a word the caller reads after the stream: without one
    // it would pass unseen.
    if (!d_status)
        return fail(M1MOE_ERR_INVALID_ARG,
                    "d_status is NULL: the device status word is required (a bounded wait that "
                    "gives up is reported only there)");
    int dev = 0;
    M1_CK(cudaGetDevice(&dev));
    NoAllocDevice *nd = nullptr;
    if (m1moe_status st = noalloc_setup(dev, nd)) return st;
    m1::LayerParams p{};
    // The routing pass of k_moe_layer reads only the router and x; the tiled
    // layout and intermediate size (64) only size its shared-memory plan.
    p.tl = m1::make_tiled_layout(h, 64, 64);
    p.router = d_router;
    p.E = E;
    p.K = K;
    p.h = h;
    p.I = 64;
    p.gs = 64;
    p.norm = norm_topk_prob ? 1 : 0;
    p.e0 = 0;
    p.ne = E;
    p.ntok = B;
    p.x = d_x;
    p.x_bf16 = x_dtype == M1MOE_DTYPE_BF16;
    p.user_idx = d_idx;
    p.user_w = d_w;
    p.user_scores = d_scores;
    p.xlog = reinterpret_cast<unsigned long long *>(nd->scratch);
    p.nbox = 1;  // one shared box: the fixed scratch has no room for a box per CTA
    p.box_words = 0;
    p.epochs = reinterpret_cast<unsigned *>(nd->scratch + kNoAllocXlog);
    p.err = d_status;
    p.route_only = 1;
    cudaStream_t st = as_stream(stream);
    M1_CK(cudaMemsetAsync(p.err, 0, sizeof(int), st));
    const int grid = std::min(nd->num_sms, kNoAllocMaxCtas);
    // the kernel variant per batch is the one m1moe_cuda_router_topk takes
    // (dispatch_layer), so both give bit-identical results
    if (B == 1) return launch_route_noalloc<1, false>(p, grid, st);
    if (B == 2)
        return m1::slot_path(2, h) ? launch_route_noalloc<2, true>(p, grid, st)
                                   : launch_route_noalloc<2, false>(p, grid, st);
    if (B <= 4) return launch_route_noalloc<4, true>(p, grid, st);
    return launch_route_noalloc<8, true>(p, grid, st);
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
    if (!c->router_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "router of layer %d not loaded", layer);
    if (!c->layer_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "experts of layer %d not loaded", layer);
    {
        // out is written (from the residual) while other CTAs still read x
        const uintptr_t xb = reinterpret_cast<uintptr_t>(d_x), ob = reinterpret_cast<uintptr_t>(d_out);
        const uintptr_t xe = xb + (uintptr_t)B * c->cfg.hidden_dim * (x_dtype == M1MOE_DTYPE_BF16 ? 2 : 4);
        const uintptr_t oe = ob + (uintptr_t)B * c->cfg.hidden_dim * (out_dtype == M1MOE_DTYPE_BF16 ? 2 : 4);
        if (xb < oe && ob < xe) return fail(M1MOE_ERR_INVALID_ARG, "out must not overlap x");
    }
    DeviceGuard dg(c->cfg.device);
    m1::LayerParams p = layer_params(c, layer, B);
    p.x = d_x;
    p.x_bf16 = x_dtype == M1MOE_DTYPE_BF16;
    p.res = d_res;
    p.res_bf16 = res_dtype == M1MOE_DTYPE_BF16;
    p.out = d_out;
    p.out_bf16 = out_dtype == M1MOE_DTYPE_BF16;
    // the down items add four adjacent fp32 rows with one 16-byte atomic
    p.out_acc = p.out_bf16 || (reinterpret_cast<uintptr_t>(d_out) & 15) != 0;
    p.user_idx = d_idx;
    p.user_w = d_w;
    return dispatch_layer(c, p, as_stream(stream));
}

m1moe_status m1moe_cuda_moe_prefill(m1moe_cuda_ctx *c, int32_t layer, const void *d_x,
                                    int32_t x_dtype, const void *d_res, int32_t res_dtype,
                                    void *d_out, int32_t out_dtype, int32_t T, int32_t *d_idx,
                                    float *d_w, void *stream) {
    if (m1moe_status st = check_layer(c, layer)) return st;
    if (!d_x || !d_out) return fail(M1MOE_ERR_INVALID_ARG, "x/out is NULL");
    if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype) || (d_res && !valid_dtype(res_dtype)))
        return fail(M1MOE_ERR_INVALID_ARG, "dtype must be F32 (0) or BF16 (1)");
    if (T < 1) return fail(M1MOE_ERR_INVALID_ARG, "tokens %d < 1", T);
    const m1moe_cuda_cfg &g = c->cfg;
    if (g.group_size != 64 || g.intermediate_dim % m1::kPfRows)
        return fail(M1MOE_ERR_UNSUPPORTED,
                    "prefill needs group_size 64 and intermediate_dim a multiple of 128");
    if ((long long)T * g.top_k > (1LL << 24))
        return fail(M1MOE_ERR_INVALID_ARG, "tokens %d: at most %d (token, expert) pairs", T, 1 << 24);
    if (!c->router_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "router of layer %d not loaded", layer);
    if (!c->layer_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "experts of layer %d not loaded", layer);
    DeviceGuard dg(g.device);
    if (m1moe_status st = pf_make_maps(c)) return st;
    if (m1moe_status st = pf_reserve(c, T)) return st;
    m1::PrefillParams p{};
    p.table = c->table + (size_t)layer * c->ne * c->tl.block;
    p.tl = c->tl;
    p.router = c->router + (size_t)layer * g.num_experts * g.hidden_dim;
    p.E = g.num_experts;
    p.K = g.top_k;
    p.h = g.hidden_dim;
    p.I = g.intermediate_dim;
    p.gs = g.group_size;
    p.norm = g.norm_topk_prob;
    p.e0 = c->e0;
    p.ne = c->ne;
    p.zblock = layer * c->ne;
    p.T = T;
    p.x = d_x;
    p.x_bf16 = x_dtype == M1MOE_DTYPE_BF16;
    p.res = d_res;
    p.res_bf16 = res_dtype == M1MOE_DTYPE_BF16;
    p.out = d_out;
    p.out_bf16 = out_dtype == M1MOE_DTYPE_BF16;
    p.user_idx = d_idx;
    p.user_w = d_w;
    p.idx = c->pf_idx;
    p.w = c->pf_w;
    p.tok_slot = c->pf_tok_slot;
    p.slot_tok = c->pf_slot_tok;
    p.tiles = c->pf_tiles;
    p.ntiles = c->pf_ntiles;
    p.max_tiles = c->pf_max_tiles;
    p.xg = c->pf_xg;
    p.act = c->pf_act;
    p.ypart = c->pf_ypart;
    p.nsplit = c->pf_nsplit;
    p.err = c->err;
    cudaStream_t st = as_stream(stream);
    const size_t rsmem = (size_t)g.hidden_dim * 4;
    if (rsmem > 48 * 1024)
        M1_CK(cudaFuncSetAttribute(m1::k_prefill_route, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)rsmem));
    m1::k_prefill_route<<<T, 256, rsmem, st>>>(p);
    M1_LAUNCHED();
    m1::k_prefill_plan<<<1, 1024, 0, st>>>(p);
    M1_LAUNCHED();
    m1::k_prefill_gather<<<dim3(p.max_tiles, m1::kPfTileTok / 8), 256, 0, st>>>(p);
    M1_LAUNCHED();
    if (m1moe_status s2 = pf_gemm<m1::kGateUp>(c, p, c->pf_map_gu, st)) return s2;
    if (m1moe_status s2 = pf_gemm<m1::kDown>(c, p, c->pf_map_dn, st)) return s2;
    m1::k_prefill_combine<<<dim3(T, (g.hidden_dim + 255) / 256), 256, 0, st>>>(p);
    M1_LAUNCHED();
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_ep_region(m1moe_cuda_ctx *c, int32_t world, int32_t tokens_per_rank,
                                 void *h_handle) {
    if (!c || !h_handle) return fail(M1MOE_ERR_INVALID_ARG, "ctx/handle is NULL");
    if (world < 2 || world > m1::kMaxRanks)
        return fail(M1MOE_ERR_INVALID_ARG, "world %d outside [2,%d]", world, m1::kMaxRanks);
    if (tokens_per_rank < 1 || (long long)world * tokens_per_rank > c->cfg.max_batch)
        return fail(M1MOE_ERR_INVALID_ARG, "world %d x tokens %d exceeds max_batch %d", world,
                    tokens_per_rank, c->cfg.max_batch);
    if (c->ep_region) return fail(M1MOE_ERR_INVALID_ARG, "exchange region already made");
    DeviceGuard dg(c->cfg.device);
    const m1::EpLayout el = m1::ep_layout(world, tokens_per_rank, c->cfg.hidden_dim);
    M1_CK(cudaMalloc((void **)&c->ep_region, (size_t)el.bytes));
    M1_CK(cudaMemset(c->ep_region, 0, (size_t)el.bytes));
    M1_CK(cudaMalloc((void **)&c->ep_own_idx, (size_t)tokens_per_rank * c->cfg.top_k * 4));
    M1_CK(cudaMalloc((void **)&c->ep_own_w, (size_t)tokens_per_rank * c->cfg.top_k * 4));
    cudaIpcMemHandle_t hnd;
    M1_CK(cudaIpcGetMemHandle(&hnd, c->ep_region));
    std::memcpy(h_handle, &hnd, sizeof(hnd));
    c->ep_world = world;
    c->ep_b = tokens_per_rank;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_ep_connect(m1moe_cuda_ctx *c, int32_t rank, const void *h_handles) {
    if (!c || !h_handles) return fail(M1MOE_ERR_INVALID_ARG, "ctx/handles is NULL");
    if (!c->ep_region) return fail(M1MOE_ERR_INVALID_ARG, "no exchange region (m1moe_cuda_ep_region)");
    if (rank < 0 || rank >= c->ep_world)
        return fail(M1MOE_ERR_INVALID_ARG, "rank %d outside [0,%d)", rank, c->ep_world);
    DeviceGuard dg(c->cfg.device);
    const uint8_t *hb = static_cast<const uint8_t *>(h_handles);
    for (int o = 0; o < c->ep_world; ++o) {
        if (o == rank) {
            c->ep_peer[o] = c->ep_region;
            continue;
        }
        cudaIpcMemHandle_t hnd;
        std::memcpy(&hnd, hb + (size_t)o * sizeof(hnd), sizeof(hnd));
        void *ptr = nullptr;
        M1_CK(cudaIpcOpenMemHandle(&ptr, hnd, cudaIpcMemLazyEnablePeerAccess));
        c->ep_peer[o] = static_cast<uint8_t *>(ptr);
        c->ep_ipc[o] = true;
    }
    c->ep_rank = rank;
    c->ep_ready = true;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_ep_connect_local(m1moe_cuda_ctx *c, int32_t rank, m1moe_cuda_ctx *const *ctxs) {
    if (!c || !ctxs) return fail(M1MOE_ERR_INVALID_ARG, "ctx/ctxs is NULL");
    if (!c->ep_region) return fail(M1MOE_ERR_INVALID_ARG, "no exchange region (m1moe_cuda_ep_region)");
    if (rank < 0 || rank >= c->ep_world)
        return fail(M1MOE_ERR_INVALID_ARG, "rank %d outside [0,%d)", rank, c->ep_world);
    if (ctxs[rank] != c) return fail(M1MOE_ERR_INVALID_ARG, "ctxs[rank] must be this context");
    DeviceGuard dg(c->cfg.device);
    for (int o = 0; o < c->ep_world; ++o) {
        const m1moe_cuda_ctx *q = ctxs[o];
        if (!q || !q->ep_region || q->ep_world != c->ep_world || q->ep_b != c->ep_b)
            return fail(M1MOE_ERR_INVALID_ARG, "rank %d's context has no matching exchange region", o);
        if (q->cfg.device != c->cfg.device) {
            int can = 0;
            M1_CK(cudaDeviceCanAccessPeer(&can, c->cfg.device, q->cfg.device));
            if (!can)
                return fail(M1MOE_ERR_UNSUPPORTED, "device %d cannot access device %d", c->cfg.device,
                            q->cfg.device);
            const cudaError_t e = cudaDeviceEnablePeerAccess(q->cfg.device, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceEnablePeerAccess");
        }
        c->ep_peer[o] = q->ep_region;
    }
    c->ep_rank = rank;
    c->ep_ready = true;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_set_wait_limit(m1moe_cuda_ctx *c, uint32_t polls) {
    if (!c) return fail(M1MOE_ERR_INVALID_ARG, "ctx is NULL");
    c->ep_wait_limit = polls ? polls : m1::kWaitLimit;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_moe_layer_ep(m1moe_cuda_ctx *c, int32_t layer, const void *d_x,
                                     int32_t x_dtype, const void *d_res, int32_t res_dtype,
                                     void *d_out, int32_t out_dtype, int32_t *d_idx, float *d_w,
                                     void *stream) {
    if (m1moe_status st = check_layer(c, layer)) return st;
    if (!d_x || !d_out) return fail(M1MOE_ERR_INVALID_ARG, "x/out is NULL");
    if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype) || (d_res && !valid_dtype(res_dtype)))
        return fail(M1MOE_ERR_INVALID_ARG, "dtype must be F32 (0) or BF16 (1)");
    if (!c->ep_ready) return fail(M1MOE_ERR_INVALID_ARG, "not connected (m1moe_cuda_ep_connect)");
    if (!c->router_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "router of layer %d not loaded", layer);
    if (!c->layer_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "experts of layer %d not loaded", layer);
    DeviceGuard dg(c->cfg.device);
    // 1. from 4 gathered tokens on, route this rank's own tokens once, here
    //    (a route-only call at the cheap batch of ep_b tokens) and let the
    //    routing travel with the tokens: the receivers then skip the batch-B
    //    logit exchange and ranking (~13 us at batch 8), at the cost of one
    //    more launch (which is more than batch 2's routing costs)
    const bool pre = c->ep_world * c->ep_b >= 4;
    if (pre) {
        m1::LayerParams r = layer_params(c, layer, c->ep_b);
        r.x = d_x;
        r.x_bf16 = x_dtype == M1MOE_DTYPE_BF16;
        r.user_idx = c->ep_own_idx;
        r.user_w = c->ep_own_w;
        r.route_only = 1;
        if (m1moe_status st = dispatch_layer(c, r, as_stream(stream))) return st;
    }
    // 2. gather every rank's tokens and routing, apply the local experts,
    //    return each rank its own tokens' sums
    const int B = c->ep_world * c->ep_b;
    m1::LayerParams p = layer_params(c, layer, B);
    p.ep_pre = pre;
    p.ep_own_idx = c->ep_own_idx;
    p.ep_own_w = c->ep_own_w;
    p.x = d_x;
    p.x_bf16 = x_dtype == M1MOE_DTYPE_BF16;
    p.res = d_res;
    p.res_bf16 = res_dtype == M1MOE_DTYPE_BF16;
    p.out = d_out;
    p.out_bf16 = out_dtype == M1MOE_DTYPE_BF16;
    p.out_acc = 1;  // sums in the accumulator; the last CTA exchanges and writes out
    p.user_idx = d_idx;
    p.user_w = d_w;
    p.ep_world = c->ep_world;
    p.ep_rank = c->ep_rank;
    p.ep_b = c->ep_b;
    for (int o = 0; o < c->ep_world; ++o) p.ep_base[o] = c->ep_peer[o];
    return dispatch_layer(c, p, as_stream(stream));
}

m1moe_status m1moe_cuda_moe_layer_host(m1moe_cuda_ctx *c, int32_t layer, const float *h_x,
                                       const float *h_res, float *h_out, int32_t B,
                                       int32_t *h_idx, float *h_w) {
    if (m1moe_status st = check_layer(c, layer)) return st;
    if (!h_x || !h_out) return fail(M1MOE_ERR_INVALID_ARG, "x/out is NULL");
    if (B < 1 || B > c->cfg.max_batch)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d outside [1,%d]", B, c->cfg.max_batch);
    DeviceGuard dg(c->cfg.device);
    const size_t n = (size_t)B * c->cfg.hidden_dim, hb = n * 4, kb = (size_t)B * c->cfg.top_k * 4;
    // inputs and outputs pass through mapped pinned memory: k_stage_in loads
    // [x | residual] into device memory, the layer runs, k_stage_out stores
    // [out | idx | w] back and then a sequence number that this thread polls
    float *pin_in = static_cast<float *>(c->hpin);
    float *pin_out = pin_in + 2 * c->cfg.max_batch * (size_t)c->cfg.hidden_dim;
    if (!c->router_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "router of layer %d not loaded", layer);
    if (!c->layer_loaded[layer]) return fail(M1MOE_ERR_NOT_LOADED, "experts of layer %d not loaded", layer);
    // the three kernels go out as one CUDA graph (captured on the first call
    // of this layer, batch and residual flag), chained by programmatic
    // dependent launch
    const size_t key = ((size_t)layer * m1::kMaxTok + (B - 1)) * 2 + (h_res ? 1 : 0);
    if (c->host_graphs.empty()) c->host_graphs.assign((size_t)c->cfg.num_layers * m1::kMaxTok * 2, nullptr);
    if (!c->host_graphs[key]) {
        float *d_out = c->hio;
        int32_t *d_idx = reinterpret_cast<int32_t *>(d_out + n);
        float *d_w = reinterpret_cast<float *>(d_idx) + (size_t)B * c->cfg.top_k;
        // the residual sits right after x (at n) in both the pinned and the
        // device block, so one stage-in moves both
        float *dev_in = static_cast<float *>(c->hpin_dev);
        float *dev_out = dev_in + (pin_out - pin_in);
        const int in4 = (int)((h_res ? 2 * hb : hb) / 16), out4 = (int)((hb + 2 * kb + 15) / 16);
        M1_CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        m1::k_stage_in<<<(in4 + 255) / 256, 256, 0, c->stream>>>(reinterpret_cast<const float4 *>(dev_in),
                                                                 reinterpret_cast<float4 *>(c->hin), in4);
        cudaError_t e = cudaGetLastError();
        m1moe_status st = M1MOE_OK;
        if (e == cudaSuccess)
            st = m1moe_cuda_moe_layer(c, layer, c->hin, M1MOE_DTYPE_F32, h_res ? c->hin + n : nullptr,
                                      M1MOE_DTYPE_F32, d_out, M1MOE_DTYPE_F32, B, d_idx, d_w, c->stream);
        if (e == cudaSuccess && st == M1MOE_OK) {
            cudaLaunchConfig_t lc = {};
            lc.gridDim = dim3(1);
            lc.blockDim = dim3(std::min(1024, std::max(32, (out4 + 31) / 32 * 32)));
            lc.stream = c->stream;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            at[0].val.programmaticStreamSerializationAllowed = 1;
            lc.attrs = at;
            lc.numAttrs = 1;
            e = cudaLaunchKernelEx(&lc, m1::k_stage_out, reinterpret_cast<const float4 *>(d_out),
                                   reinterpret_cast<float4 *>(dev_out), out4, c->hseq_dev,
                                   reinterpret_cast<unsigned *>(static_cast<uint8_t *>(c->hpin_dev) +
                                                                (reinterpret_cast<uint8_t *>(c->hflag) -
                                                                 static_cast<uint8_t *>(c->hpin))));
        }
        cudaGraph_t graph = nullptr;
        const cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
        if (st != M1MOE_OK) {
            if (graph) cudaGraphDestroy(graph);
            return st;
        }
        if (e == cudaSuccess) e = e2;
        cudaGraphExec_t exec = nullptr;
        if (e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        if (e != cudaSuccess) return cuda_fail(e, "host-call graph");
        c->host_graphs[key] = exec;
    }
    memcpy(pin_in, h_x, hb);
    if (h_res) memcpy(pin_in + n, h_res, hb);
    const unsigned want = c->host_seq + 1;
    M1_CK(cudaGraphLaunch(c->host_graphs[key], c->stream));
    g_launches.fetch_add(3, std::memory_order_relaxed);
    // poll the flag; every 256 polls ask the stream whether it failed or
    // finished without the flag (bounded: a minute)
    const volatile unsigned *flag = c->hflag;
    const auto t0 = std::chrono::steady_clock::now();
    for (uint32_t it = 1;; ++it) {
        if (*flag == want) break;
        if ((it & 255u) == 0) {
            const cudaError_t q = cudaStreamQuery(c->stream);
            if (q == cudaSuccess && *flag == want) break;
            if (q != cudaSuccess && q != cudaErrorNotReady) return cuda_fail(q, "host-call graph");
            if (q == cudaSuccess || std::chrono::steady_clock::now() - t0 > std::chrono::seconds(60)) {
                cudaStreamSynchronize(c->stream);
                c->host_seq = *flag;
                return fail(M1MOE_ERR_DEVICE, "host call: no completion flag (sequence %u, saw %u)", want,
                            c->host_seq);
            }
        }
    }
    c->host_seq = want;
    std::atomic_thread_fence(std::memory_order_acquire);
    memcpy(h_out, pin_out, hb);
    if (h_idx) memcpy(h_idx, pin_out + n, kb);
    if (h_w) memcpy(h_w, reinterpret_cast<const uint8_t *>(pin_out + n) + kb, kb);
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_synchronize(m1moe_cuda_ctx *c) {
    if (!c) return fail(M1MOE_ERR_INVALID_ARG, "ctx is NULL");
    DeviceGuard dg(c->cfg.device);
    M1_CK(cudaDeviceSynchronize());
    int word = 0;
    M1_CK(cudaMemcpy(&word, c->err, 4, cudaMemcpyDeviceToHost));
    if (word) {
        // A kernel gave up on a wait: clear the word and the exchange buffers
        // so that the next call starts from a clean state.
        M1_CK(cudaMemset(c->err, 0, 4));
        M1_CK(clear_exchange(c));
        return fail(M1MOE_ERR_DEVICE, "device error word 0x%x (1: a bounded wait timed out; 2: an index out of "
                                      "range; 4: a value beyond the fp16 range of the tensor-core operands)",
                    word);
    }
    return M1MOE_OK;
}

}  // extern "C"
