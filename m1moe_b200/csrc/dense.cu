// dense.cu — C ABI of the dense half of a decode step and of the whole token
// step (include/m1moe_cuda.h, m1moe_cuda_dense_* and m1moe_cuda_decode_step).
//
// The dense context owns the non-expert weights (embedding, norms, attention
// projections, QK-norm weights, LM head), the bf16 KV cache and the per-step
// buffers, as the reference's WeightStore (mmap'd model_weights.bin,
// WeightStore.swift:47-126) and MetalContext (f32 scratch and KV buffers,
// MetalContext.swift:134-152) do.  A decode step joins it with an MoE
// context (m1moe_cuda.cu) for the expert blocks.
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "m1moe_cuda.h"
#include "dense.cuh"

// The error helpers and launch counter of m1moe_cuda.cu (one library).
namespace m1abi {
m1moe_status fail(m1moe_status st, const char *fmt, ...);
m1moe_status cuda_fail(cudaError_t e, const char *what);
void count_launch();
m1moe_status moe_compatible(const m1moe_cuda_ctx *moe, int hidden, int layers, int batch, int device);
}  // namespace m1abi

using m1abi::cuda_fail;
using m1abi::fail;

#define D_CK(call)                                               \
    do {                                                         \
        cudaError_t e_ = (call);                                 \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);      \
    } while (0)

struct m1moe_dense_ctx {
    m1moe_dense_cfg cfg{};
    int qd = 0, kvd = 0, qkv_rows = 0, hd = 0;
    uint16_t *embed = nullptr, *lm_head = nullptr, *final_norm = nullptr;  // [V][h], [V][h], [h]
    uint16_t *in_norm = nullptr, *post_norm = nullptr;                     // [L][h]
    uint16_t *wqkv = nullptr;  // [L][qd + 2 kvd][h]: q rows, then k, then v
    uint16_t *wo = nullptr;    // [L][h][qd]
    uint16_t *qn = nullptr, *kn = nullptr;  // [L][hd]
    uint16_t *kc = nullptr, *vc = nullptr;  // [L][max_batch][nkv][max_seq][hd]
    float *residual = nullptr, *h_mid = nullptr, *qkv = nullptr, *attn_out = nullptr;
    float *part = nullptr;        // [max_batch][nh][nsplit][hd + 2]
    float *ss_acc = nullptr;      // [kDenseMaxTok]
    unsigned *done = nullptr;
    unsigned long long *keys = nullptr;  // [kDenseMaxTok]
    unsigned *attn_cnt = nullptr;        // [kDenseMaxTok][nkv]
    int *pos = nullptr;                  // device position
    int *err = nullptr;                  // device error word
    int nsplit = 1;
    int num_sms = 148;
    // token-parallel prefill (m1moe_cuda_prefill_step): buffers for pf_cap
    // tokens (grown on demand) and the cuBLAS handle of its projections
    int pf_cap = 0;
    float *pf_res = nullptr, *pf_qkv = nullptr, *pf_hmid = nullptr;
    __nv_bfloat16 *pf_xn = nullptr, *pf_attn = nullptr;
    cublasHandle_t blas = nullptr;
    // which tensors are loaded: [tensor][layer]
    std::vector<std::vector<uint8_t>> loaded;
};

namespace {

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DevGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

constexpr int kNumTensors = 11;
bool per_layer(int t) {
    return t == M1MOE_W_INPUT_NORM || t == M1MOE_W_POST_NORM || t == M1MOE_W_Q || t == M1MOE_W_K ||
           t == M1MOE_W_V || t == M1MOE_W_O || t == M1MOE_W_Q_NORM || t == M1MOE_W_K_NORM;
}

// Destination and element count of one tensor in the context.
m1moe_status tensor_slot(m1moe_dense_ctx *c, int tensor, int layer, size_t count, uint16_t *&dst,
                         size_t &want) {
    const m1moe_dense_cfg &g = c->cfg;
    const size_t h = g.hidden_dim, V = g.vocab_size, qd = c->qd, kvd = c->kvd, hd = c->hd;
    if (tensor < 0 || tensor >= kNumTensors) return fail(M1MOE_ERR_INVALID_ARG, "tensor %d unknown", tensor);
    if (per_layer(tensor) && (layer < 0 || layer >= g.num_layers))
        return fail(M1MOE_ERR_INVALID_ARG, "layer %d out of range [0,%d)", layer, g.num_layers);
    const size_t L = per_layer(tensor) ? (size_t)layer : 0;
    const size_t qkv_layer = (size_t)c->qkv_rows * h;
    switch (tensor) {
    case M1MOE_W_EMBED: dst = c->embed; want = V * h; break;
    case M1MOE_W_LM_HEAD: dst = c->lm_head; want = V * h; break;
    case M1MOE_W_FINAL_NORM: dst = c->final_norm; want = h; break;
    case M1MOE_W_INPUT_NORM: dst = c->in_norm + L * h; want = h; break;
    case M1MOE_W_POST_NORM: dst = c->post_norm + L * h; want = h; break;
    case M1MOE_W_Q: dst = c->wqkv + L * qkv_layer; want = qd * h; break;
    case M1MOE_W_K: dst = c->wqkv + L * qkv_layer + qd * h; want = kvd * h; break;
    case M1MOE_W_V: dst = c->wqkv + L * qkv_layer + (qd + kvd) * h; want = kvd * h; break;
    case M1MOE_W_O: dst = c->wo + L * h * qd; want = h * qd; break;
    case M1MOE_W_Q_NORM:
    case M1MOE_W_K_NORM: {
        if (!g.qk_norm) return fail(M1MOE_ERR_INVALID_ARG, "the model has no QK-norm (qk_norm 0)");
        dst = (tensor == M1MOE_W_Q_NORM ? c->qn : c->kn) + L * hd;
        // the model file holds [qd] / [kvd]; the reference applies the first hd
        // to every head (InferenceEngine.swift:538-548), so either size is taken
        const size_t full = tensor == M1MOE_W_Q_NORM ? qd : kvd;
        if (count != hd && count != full)
            return fail(M1MOE_ERR_INVALID_ARG, "QK-norm weight: %zu elements, expected %zu or %zu", count,
                        hd, full);
        want = count;
        return M1MOE_OK;
    }
    default: return fail(M1MOE_ERR_INVALID_ARG, "tensor %d unknown", tensor);
    }
    if (count != want)
        return fail(M1MOE_ERR_INVALID_ARG, "tensor %d: %zu elements, expected %zu", tensor, count, want);
    return M1MOE_OK;
}

size_t copy_count(m1moe_dense_ctx *c, int tensor, size_t count) {
    return (tensor == M1MOE_W_Q_NORM || tensor == M1MOE_W_K_NORM) ? (size_t)c->hd : count;
}

void free_dense(m1moe_dense_ctx *c) {
    if (!c) return;
    for (void *q : {(void *)c->embed, (void *)c->lm_head, (void *)c->final_norm, (void *)c->in_norm,
                    (void *)c->post_norm, (void *)c->wqkv, (void *)c->wo, (void *)c->qn, (void *)c->kn,
                    (void *)c->kc, (void *)c->vc, (void *)c->residual, (void *)c->h_mid, (void *)c->qkv,
                    (void *)c->attn_out, (void *)c->part, (void *)c->ss_acc, (void *)c->done,
                    (void *)c->keys, (void *)c->attn_cnt, (void *)c->pos, (void *)c->err,
                    (void *)c->pf_res, (void *)c->pf_qkv, (void *)c->pf_hmid, (void *)c->pf_xn,
                    (void *)c->pf_attn})
        cudaFree(q);
    if (c->blas) cublasDestroy(c->blas);
    delete c;
}

// Launch with programmatic stream serialisation (the kernel waits for its
// predecessor with griddepcontrol.wait before touching its outputs).
template <typename... KArgs, typename... Args>
m1moe_status launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                        const char *what, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    if (e != cudaSuccess) return cuda_fail(e, what);
    m1abi::count_launch();
    return M1MOE_OK;
}

constexpr size_t kGemvSmemCap = 227 * 1024 - 2048;  // dynamic shared memory (static use aside)

template <int NT, int EPI>
m1moe_status gemv_nt(m1::GemvParams p, int num_sms, cudaStream_t st) {
    const int nw = p.K / m1::kGemvColsPerWarp;
    // one CTA per SM (the ring takes most of its shared memory), at least a
    // stage of rows per CTA
    const int sr = p.K <= 2048 ? 16 : 8;
    const int grid = std::max(1, std::min(num_sms, (p.rows + sr - 1) / sr));
    const m1::GemvPlan g = m1::gemv_plan(p.K, NT, (p.rows + grid - 1) / grid, kGemvSmemCap);
    p.stage_rows = g.stage_rows;
    p.nstages = g.nstages;
    p.off_bars = g.off_bars;
    p.off_part = g.off_part;
    auto kern = m1::k_dense_gemv<NT, EPI>;
    D_CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, g.smem));
    return launch_pdl(kern, dim3(grid), dim3((nw + 1) * 32), (size_t)g.smem, st, "k_dense_gemv launch", p);
}

template <int EPI>
m1moe_status gemv(const m1::GemvParams &p, int num_sms, cudaStream_t st) {
    if (p.ntok == 1) return gemv_nt<1, EPI>(p, num_sms, st);
    if (p.ntok == 2) return gemv_nt<2, EPI>(p, num_sms, st);
    if (p.ntok <= 4) return gemv_nt<4, EPI>(p, num_sms, st);
    return gemv_nt<8, EPI>(p, num_sms, st);
}

m1moe_status check_gemv_shape(int rows, int K, int B) {
    if (rows <= 0 || K <= 0 || K % m1::kGemvColsPerWarp || K > m1::kGemvColsPerWarp * m1::kGemvMaxWarps)
        return fail(M1MOE_ERR_UNSUPPORTED, "in_dim %d: a positive multiple of %d up to %d", K,
                    m1::kGemvColsPerWarp, m1::kGemvColsPerWarp * m1::kGemvMaxWarps);
    if (B < 1 || B > m1::kDenseMaxTok)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d outside [1,%d]", B, m1::kDenseMaxTok);
    return M1MOE_OK;
}

// Position splits per (token, KV head): about one CTA per SM over the
// batch's (token, KV head) pairs (each CTA streams its rows through a
// two-stage ring; fewer splits keep the final merge short).
int attn_splits(int num_sms, int nkv, int B, int max_seq) {
    const int want = num_sms / (nkv * B);  // one wave: at most one CTA per SM
    return std::max(1, std::min(std::min(want, m1::kAttnMaxSplit), (max_seq + 31) / 32));
}

m1::AttnParams attn_params(m1moe_dense_ctx *c, int layer, const float *qkv, int B, float *out) {
    const m1moe_dense_cfg &g = c->cfg;
    m1::AttnParams p{};
    p.qkv = qkv;
    p.qkv_stride = c->qkv_rows;
    p.nh = g.num_heads;
    p.nkv = g.num_kv_heads;
    p.ntok = B;
    p.pos = c->pos;
    p.max_seq = g.max_seq;
    p.qn_w = g.qk_norm ? c->qn + (size_t)layer * c->hd : nullptr;
    p.kn_w = g.qk_norm ? c->kn + (size_t)layer * c->hd : nullptr;
    p.eps = g.rms_norm_eps;
    p.theta = g.rope_theta;
    p.scale = 1.0f / sqrtf((float)c->hd);  // InferenceEngine.swift encodeAttention: 1/sqrt(hd)
    const size_t cache_layer = (size_t)g.max_batch * g.num_kv_heads * g.max_seq * c->hd;
    p.kc = c->kc + (size_t)layer * cache_layer;
    p.vc = c->vc + (size_t)layer * cache_layer;
    p.nsplit = attn_splits(c->num_sms, g.num_kv_heads, B, g.max_seq);
    p.part = c->part;
    p.cnt = c->attn_cnt;
    p.out = out;
    p.err = c->err;
    return p;
}

template <int HP>
m1moe_status launch_attn_hp(dim3 grid, dim3 block, size_t smem, cudaStream_t st, const m1::AttnParams &p) {
    D_CK(cudaFuncSetAttribute(m1::k_attn_decode<HP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    return launch_pdl(m1::k_attn_decode<HP>, grid, block, smem, st, "k_attn_decode launch", p);
}

m1moe_status launch_attn(m1moe_dense_ctx *c, const m1::AttnParams &p, int B, cudaStream_t st) {
    const int hp = c->cfg.num_heads / c->cfg.num_kv_heads;
    const dim3 grid(p.nsplit, c->cfg.num_kv_heads, B), block(m1::kAttnThreads);
    const size_t smem = m1::attn_smem();
    switch (hp) {
    case 1: return launch_attn_hp<1>(grid, block, smem, st, p);
    case 2: return launch_attn_hp<2>(grid, block, smem, st, p);
    case 4: return launch_attn_hp<4>(grid, block, smem, st, p);
    case 8: return launch_attn_hp<8>(grid, block, smem, st, p);
    default: return fail(M1MOE_ERR_UNSUPPORTED, "heads per KV head %d: 1, 2, 4 or 8", hp);
    }
}

m1moe_status check_loaded(m1moe_dense_ctx *c) {
    for (int t = 0; t < kNumTensors; ++t) {
        if ((t == M1MOE_W_Q_NORM || t == M1MOE_W_K_NORM) && !c->cfg.qk_norm) continue;
        const int n = per_layer(t) ? c->cfg.num_layers : 1;
        for (int L = 0; L < n; ++L)
            if (!c->loaded[t][L]) return fail(M1MOE_ERR_NOT_LOADED, "dense tensor %d of layer %d not loaded", t, L);
    }
    return M1MOE_OK;
}

// Buffers for T prefill tokens (grown, never shrunk; a synchronous reallocation).
m1moe_status pf_dense_reserve(m1moe_dense_ctx *c, int T) {
    if (!c->blas) {
        if (cublasCreate(&c->blas) != CUBLAS_STATUS_SUCCESS)
            return fail(M1MOE_ERR_CUDA, "cublasCreate failed");
    }
    if (T <= c->pf_cap) return M1MOE_OK;
    D_CK(cudaDeviceSynchronize());
    for (void *q : {(void *)c->pf_res, (void *)c->pf_qkv, (void *)c->pf_hmid, (void *)c->pf_xn,
                    (void *)c->pf_attn})
        cudaFree(q);
    c->pf_res = c->pf_qkv = c->pf_hmid = nullptr;
    c->pf_xn = c->pf_attn = nullptr;
    c->pf_cap = 0;
    const size_t h = c->cfg.hidden_dim;
    D_CK(cudaMalloc((void **)&c->pf_res, (size_t)T * h * 4));
    D_CK(cudaMalloc((void **)&c->pf_hmid, (size_t)T * h * 4));
    D_CK(cudaMalloc((void **)&c->pf_qkv, (size_t)T * c->qkv_rows * 4));
    D_CK(cudaMalloc((void **)&c->pf_xn, (size_t)T * h * 2));
    D_CK(cudaMalloc((void **)&c->pf_attn, (size_t)T * c->qd * 2));
    c->pf_cap = T;
    return M1MOE_OK;
}

// Y[T][N] = X[T][K] . W[N][K]^T (+ Y if accumulate): a plain bf16 GEMM with
// fp32 accumulation and output (cuBLAS; column-major view: Y^T = W . X^T).
m1moe_status gemm_bf16(m1moe_dense_ctx *c, const uint16_t *W, const __nv_bfloat16 *X, float *Y, int N, int K,
                       int T, bool accumulate, cudaStream_t st) {
    if (cublasSetStream(c->blas, st) != CUBLAS_STATUS_SUCCESS) return fail(M1MOE_ERR_CUDA, "cublasSetStream");
    const float alpha = 1.f, beta = accumulate ? 1.f : 0.f;
    const cublasStatus_t r = cublasGemmEx(c->blas, CUBLAS_OP_T, CUBLAS_OP_N, N, T, K, &alpha, W, CUDA_R_16BF, K, X,
                                          CUDA_R_16BF, K, &beta, Y, CUDA_R_32F, N, CUBLAS_COMPUTE_32F,
                                          CUBLAS_GEMM_DEFAULT);
    if (r != CUBLAS_STATUS_SUCCESS) return fail(M1MOE_ERR_CUDA, "cublasGemmEx failed (%d)", (int)r);
    return M1MOE_OK;
}

}  // namespace

extern "C" {

m1moe_status m1moe_cuda_dense_create(const m1moe_dense_cfg *cfg, m1moe_dense_ctx **out) {
    if (!cfg || !out) return fail(M1MOE_ERR_INVALID_ARG, "cfg/out is NULL");
    *out = nullptr;
    const m1moe_dense_cfg g = *cfg;
    if (g.hidden_dim <= 0 || g.num_heads <= 0 || g.num_kv_heads <= 0 || g.num_layers <= 0 ||
        g.vocab_size <= 0 || g.max_seq <= 0)
        return fail(M1MOE_ERR_INVALID_ARG, "dims must be positive");
    if (g.head_dim != m1::kHeadDim)
        return fail(M1MOE_ERR_UNSUPPORTED, "head_dim %d: only %d", g.head_dim, m1::kHeadDim);
    if (g.num_heads % g.num_kv_heads)
        return fail(M1MOE_ERR_INVALID_ARG, "num_heads %d not a multiple of num_kv_heads %d", g.num_heads,
                    g.num_kv_heads);
    const int hp = g.num_heads / g.num_kv_heads;
    if (hp != 1 && hp != 2 && hp != 4 && hp != 8)
        return fail(M1MOE_ERR_UNSUPPORTED, "heads per KV head %d: 1, 2, 4 or 8", hp);
    const int qd = g.num_heads * g.head_dim;
    if (m1moe_status st = check_gemv_shape(qd, g.hidden_dim, 1)) return st;
    if (m1moe_status st = check_gemv_shape(g.hidden_dim, qd, 1)) return st;
    if (g.max_batch < 1 || g.max_batch > m1::kDenseMaxTok)
        return fail(M1MOE_ERR_INVALID_ARG, "max_batch %d outside [1,%d]", g.max_batch, m1::kDenseMaxTok);
    int ndev = 0;
    D_CK(cudaGetDeviceCount(&ndev));
    if (g.device < 0 || g.device >= ndev)
        return fail(M1MOE_ERR_INVALID_ARG, "device %d outside [0,%d)", g.device, ndev);
    DevGuard dg(g.device);
    auto *c = new m1moe_dense_ctx();
    c->cfg = g;
    c->hd = g.head_dim;
    c->qd = qd;
    c->kvd = g.num_kv_heads * g.head_dim;
    c->qkv_rows = c->qd + 2 * c->kvd;
    int nsm = 0;
    if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, g.device) == cudaSuccess && nsm > 0)
        c->num_sms = nsm;
    // position splits (chosen per call by attn_splits); the partials are
    // sized for the most, at batch 1
    c->nsplit = attn_splits(c->num_sms, g.num_kv_heads, 1, g.max_seq);
    c->loaded.assign(kNumTensors, std::vector<uint8_t>(g.num_layers, 0));
    const size_t h = g.hidden_dim, V = g.vocab_size, L = g.num_layers, B = g.max_batch;
    const size_t cache = L * B * g.num_kv_heads * (size_t)g.max_seq * c->hd;
    cudaError_t e = cudaSuccess;
    auto alloc = [&](auto *&ptr, size_t bytes) {
        if (e == cudaSuccess) e = cudaMalloc((void **)&ptr, bytes);
    };
    alloc(c->embed, V * h * 2);
    alloc(c->lm_head, V * h * 2);
    alloc(c->final_norm, h * 2);
    alloc(c->in_norm, L * h * 2);
    alloc(c->post_norm, L * h * 2);
    alloc(c->wqkv, L * c->qkv_rows * h * 2);
    alloc(c->wo, L * h * c->qd * 2);
    alloc(c->qn, L * c->hd * 2);
    alloc(c->kn, L * c->hd * 2);
    alloc(c->kc, cache * 2);
    alloc(c->vc, cache * 2);
    alloc(c->residual, B * h * 4);
    alloc(c->h_mid, B * h * 4);
    alloc(c->qkv, B * c->qkv_rows * 4);
    alloc(c->attn_out, B * c->qd * 4);
    alloc(c->part, B * g.num_heads * (size_t)c->nsplit * (c->hd + 2) * 4);
    alloc(c->ss_acc, m1::kDenseMaxTok * 4);
    alloc(c->done, 4);
    alloc(c->keys, m1::kDenseMaxTok * 8);
    alloc(c->attn_cnt, (size_t)m1::kDenseMaxTok * g.num_kv_heads * 4);
    alloc(c->pos, 4);
    alloc(c->err, 4);
    if (e == cudaSuccess) e = cudaMemset(c->ss_acc, 0, m1::kDenseMaxTok * 4);
    if (e == cudaSuccess) e = cudaMemset(c->done, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(c->keys, 0, m1::kDenseMaxTok * 8);
    if (e == cudaSuccess) e = cudaMemset(c->attn_cnt, 0, (size_t)m1::kDenseMaxTok * g.num_kv_heads * 4);
    if (e == cudaSuccess) e = cudaMemset(c->pos, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(c->err, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(c->kc, 0, cache * 2);
    if (e == cudaSuccess) e = cudaMemset(c->vc, 0, cache * 2);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        m1moe_status st = cuda_fail(e, "dense context set-up");
        free_dense(c);
        return st;
    }
    *out = c;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_dense_destroy(m1moe_dense_ctx *c) {
    if (!c) return M1MOE_OK;
    DevGuard dg(c->cfg.device);
    cudaDeviceSynchronize();
    free_dense(c);
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_dense_load(m1moe_dense_ctx *c, int32_t tensor, int32_t layer,
                                   const uint16_t *h_bf16, size_t count) {
    if (!c || !h_bf16) return fail(M1MOE_ERR_INVALID_ARG, "ctx/data is NULL");
    uint16_t *dst = nullptr;
    size_t want = 0;
    if (m1moe_status st = tensor_slot(c, tensor, layer, count, dst, want)) return st;
    DevGuard dg(c->cfg.device);
    D_CK(cudaMemcpy(dst, h_bf16, copy_count(c, tensor, count) * 2, cudaMemcpyHostToDevice));
    c->loaded[tensor][per_layer(tensor) ? layer : 0] = 1;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_dense_load_device(m1moe_dense_ctx *c, int32_t tensor, int32_t layer,
                                          const uint16_t *d_bf16, size_t count, void *stream) {
    if (!c || !d_bf16) return fail(M1MOE_ERR_INVALID_ARG, "ctx/data is NULL");
    uint16_t *dst = nullptr;
    size_t want = 0;
    if (m1moe_status st = tensor_slot(c, tensor, layer, count, dst, want)) return st;
    DevGuard dg(c->cfg.device);
    D_CK(cudaMemcpyAsync(dst, d_bf16, copy_count(c, tensor, count) * 2, cudaMemcpyDeviceToDevice,
                         as_stream(stream)));
    c->loaded[tensor][per_layer(tensor) ? layer : 0] = 1;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_dense_kv_cache(m1moe_dense_ctx *c, int32_t layer, void **d_k, void **d_v) {
    if (!c || !d_k || !d_v) return fail(M1MOE_ERR_INVALID_ARG, "NULL pointer");
    if (layer < 0 || layer >= c->cfg.num_layers)
        return fail(M1MOE_ERR_INVALID_ARG, "layer %d out of range [0,%d)", layer, c->cfg.num_layers);
    const size_t cache_layer = (size_t)c->cfg.max_batch * c->cfg.num_kv_heads * c->cfg.max_seq * c->hd;
    *d_k = c->kc + (size_t)layer * cache_layer;
    *d_v = c->vc + (size_t)layer * cache_layer;
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_dense_set_position(m1moe_dense_ctx *c, int32_t pos) {
    if (!c) return fail(M1MOE_ERR_INVALID_ARG, "ctx is NULL");
    if (pos < 0 || pos >= c->cfg.max_seq)
        return fail(M1MOE_ERR_INVALID_ARG, "position %d outside [0,%d)", pos, c->cfg.max_seq);
    DevGuard dg(c->cfg.device);
    D_CK(cudaDeviceSynchronize());
    D_CK(cudaMemcpy(c->pos, &pos, 4, cudaMemcpyHostToDevice));
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_dense_get_position(m1moe_dense_ctx *c, int32_t *pos) {
    if (!c || !pos) return fail(M1MOE_ERR_INVALID_ARG, "NULL pointer");
    DevGuard dg(c->cfg.device);
    D_CK(cudaDeviceSynchronize());
    D_CK(cudaMemcpy(pos, c->pos, 4, cudaMemcpyDeviceToHost));
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_dense_reset(m1moe_dense_ctx *c) {
    if (!c) return fail(M1MOE_ERR_INVALID_ARG, "ctx is NULL");
    DevGuard dg(c->cfg.device);
    const size_t cache = (size_t)c->cfg.num_layers * c->cfg.max_batch * c->cfg.num_kv_heads *
                         c->cfg.max_seq * c->hd;
    D_CK(cudaDeviceSynchronize());
    D_CK(cudaMemset(c->kc, 0, cache * 2));
    D_CK(cudaMemset(c->vc, 0, cache * 2));
    D_CK(cudaMemset(c->pos, 0, 4));
    D_CK(cudaDeviceSynchronize());
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_dense_synchronize(m1moe_dense_ctx *c) {
    if (!c) return fail(M1MOE_ERR_INVALID_ARG, "ctx is NULL");
    DevGuard dg(c->cfg.device);
    D_CK(cudaDeviceSynchronize());
    int word = 0;
    D_CK(cudaMemcpy(&word, c->err, 4, cudaMemcpyDeviceToHost));
    if (word) {
        D_CK(cudaMemset(c->err, 0, 4));
        return fail(M1MOE_ERR_DEVICE, "dense error word 0x%x (2: a token id or KV position was out of range)", word);
    }
    return M1MOE_OK;
}

m1moe_status m1moe_cuda_dense_gemv(const uint16_t *d_w, int32_t rows, int32_t in_dim, const void *d_x,
                                   int32_t x_dtype, const uint16_t *d_norm_w, float eps,
                                   const float *d_res, float *d_y, int32_t batch, void *stream) {
    if (!d_w || !d_x || !d_y) return fail(M1MOE_ERR_INVALID_ARG, "NULL pointer");
    if (x_dtype != M1MOE_DTYPE_F32 && x_dtype != M1MOE_DTYPE_BF16)
        return fail(M1MOE_ERR_INVALID_ARG, "dtype must be F32 (0) or BF16 (1)");
    if (m1moe_status st = check_gemv_shape(rows, in_dim, batch)) return st;
    if ((reinterpret_cast<uintptr_t>(d_w) | reinterpret_cast<uintptr_t>(d_x)) & 15)
        return fail(M1MOE_ERR_INVALID_ARG, "weights and x must be 16-byte aligned");
    m1::GemvParams p{};
    p.w = d_w;
    p.rows = rows;
    p.K = in_dim;
    p.x = d_x;
    p.x_bf16 = x_dtype == M1MOE_DTYPE_BF16;
    p.norm_w = d_norm_w;
    p.eps = eps;
    p.y = d_y;
    p.res = d_res;
    p.ntok = batch;
    p.err = nullptr;
    int dev = 0, nsm = 148;
    D_CK(cudaGetDevice(&dev));
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    return gemv<m1::kEpiStore>(p, nsm, as_stream(stream));
}

m1moe_status m1moe_cuda_dense_rmsnorm(const void *d_x, int32_t x_dtype, const uint16_t *d_w, float eps,
                                      float *d_y, int32_t dim, int32_t batch, void *stream) {
    if (!d_x || !d_w || !d_y) return fail(M1MOE_ERR_INVALID_ARG, "NULL pointer");
    if (x_dtype != M1MOE_DTYPE_F32 && x_dtype != M1MOE_DTYPE_BF16)
        return fail(M1MOE_ERR_INVALID_ARG, "dtype must be F32 (0) or BF16 (1)");
    if (dim <= 0 || batch < 1 || batch > 65535) return fail(M1MOE_ERR_INVALID_ARG, "dim/batch invalid");
    return launch_pdl(m1::k_rmsnorm, dim3(batch), dim3(256), 0, as_stream(stream), "k_rmsnorm launch",
                      d_x, (int)(x_dtype == M1MOE_DTYPE_BF16), d_w, eps, d_y, (int)dim);
}

m1moe_status m1moe_cuda_dense_attention(m1moe_dense_ctx *c, int32_t layer, const float *d_qkv,
                                        int32_t batch, float *d_out, void *stream) {
    if (!c || !d_qkv || !d_out) return fail(M1MOE_ERR_INVALID_ARG, "NULL pointer");
    if (layer < 0 || layer >= c->cfg.num_layers)
        return fail(M1MOE_ERR_INVALID_ARG, "layer %d out of range [0,%d)", layer, c->cfg.num_layers);
    if (batch < 1 || batch > c->cfg.max_batch)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d outside [1,%d]", batch, c->cfg.max_batch);
    if ((reinterpret_cast<uintptr_t>(d_qkv) | reinterpret_cast<uintptr_t>(d_out)) & 15)
        return fail(M1MOE_ERR_INVALID_ARG, "qkv and out must be 16-byte aligned");
    if (c->cfg.qk_norm && !(c->loaded[M1MOE_W_Q_NORM][layer] && c->loaded[M1MOE_W_K_NORM][layer]))
        return fail(M1MOE_ERR_NOT_LOADED, "QK-norm weights of layer %d not loaded", layer);
    DevGuard dg(c->cfg.device);
    return launch_attn(c, attn_params(c, layer, d_qkv, batch, d_out), batch, as_stream(stream));
}

m1moe_status m1moe_cuda_dense_lm_head(m1moe_dense_ctx *c, const float *d_x, int32_t batch,
                                      int32_t *d_tokens, float *d_logits, void *stream) {
    if (!c || !d_x || !d_tokens) return fail(M1MOE_ERR_INVALID_ARG, "NULL pointer");
    if (batch < 1 || batch > c->cfg.max_batch)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d outside [1,%d]", batch, c->cfg.max_batch);
    if (!c->loaded[M1MOE_W_LM_HEAD][0] || !c->loaded[M1MOE_W_FINAL_NORM][0])
        return fail(M1MOE_ERR_NOT_LOADED, "LM head or final norm not loaded");
    DevGuard dg(c->cfg.device);
    m1::GemvParams p{};
    p.w = c->lm_head;
    p.rows = c->cfg.vocab_size;
    p.K = c->cfg.hidden_dim;
    p.x = d_x;
    p.norm_w = c->final_norm;
    p.eps = c->cfg.rms_norm_eps;
    p.y = d_logits;
    p.ntok = batch;
    p.done = c->done;
    p.keys = c->keys;
    p.tokens = d_tokens;
    p.err = c->err;
    return gemv<m1::kEpiArgmax>(p, c->num_sms, as_stream(stream));
}

m1moe_status m1moe_cuda_decode_step(m1moe_dense_ctx *c, m1moe_cuda_ctx *moe, const int32_t *d_tokens,
                                    int32_t batch, int32_t *d_next_tokens, float *d_logits,
                                    void *stream) {
    if (!c || !moe || !d_tokens || !d_next_tokens) return fail(M1MOE_ERR_INVALID_ARG, "NULL pointer");
    const m1moe_dense_cfg &g = c->cfg;
    if (batch < 1 || batch > g.max_batch)
        return fail(M1MOE_ERR_INVALID_ARG, "batch %d outside [1,%d]", batch, g.max_batch);
    if (m1moe_status st = check_loaded(c)) return st;
    if (m1moe_status st = m1abi::moe_compatible(moe, g.hidden_dim, g.num_layers, batch, g.device))
        return st;
    DevGuard dg(g.device);
    cudaStream_t st = as_stream(stream);
    const int h = g.hidden_dim;
    // 1. embed (InferenceEngine.swift:127-129)
    if (m1moe_status s = launch_pdl(m1::k_embed, dim3(batch), dim3(256), 0, st, "k_embed launch",
                                    (const uint16_t *)c->embed, d_tokens, (int)g.vocab_size, h,
                                    c->residual, (int)batch, c->err))
        return s;
    for (int L = 0; L < g.num_layers; ++L) {
        // 2. CMD1: input RMSNorm + q/k/v projections (:176-192)
        m1::GemvParams q{};
        q.w = c->wqkv + (size_t)L * c->qkv_rows * h;
        q.rows = c->qkv_rows;
        q.K = h;
        q.x = c->residual;
        q.norm_w = c->in_norm + (size_t)L * h;
        q.eps = g.rms_norm_eps;
        q.y = c->qkv;
        q.ntok = batch;
        q.err = c->err;
        if (m1moe_status s = gemv<m1::kEpiStore>(q, c->num_sms, st)) return s;
        // 3. QK-norm, RoPE, KV store (:194-220) and attention (CMD2, :225)
        if (m1moe_status s = launch_attn(c, attn_params(c, L, c->qkv, batch, c->attn_out), batch, st))
            return s;
        // 4. o_proj + residual add + post-attention RMSNorm (:226-236)
        m1::GemvParams o{};
        o.w = c->wo + (size_t)L * h * c->qd;
        o.rows = h;
        o.K = c->qd;
        o.x = c->attn_out;
        o.eps = g.rms_norm_eps;
        o.y = c->residual;
        o.res = c->residual;
        o.ntok = batch;
        o.post_w = c->post_norm + (size_t)L * h;
        o.post_out = c->h_mid;
        o.ss_acc = c->ss_acc;
        o.done = c->done;
        o.err = c->err;
        if (m1moe_status s = gemv<m1::kEpiPostNorm>(o, c->num_sms, st)) return s;
        // 5. the MoE block: residual += sum_k w_k Expert_k(h_mid) (:240-266)
        if (m1moe_status s = m1moe_cuda_moe_layer(moe, L, c->h_mid, M1MOE_DTYPE_F32, c->residual,
                                                   M1MOE_DTYPE_F32, c->residual, M1MOE_DTYPE_F32, batch,
                                                   nullptr, nullptr, stream))
            return s;
    }
    // 6. final RMSNorm + LM head + greedy sample (:140-155); the position advances
    m1::GemvParams lm{};
    lm.w = c->lm_head;
    lm.rows = g.vocab_size;
    lm.K = h;
    lm.x = c->residual;
    lm.norm_w = c->final_norm;
    lm.eps = g.rms_norm_eps;
    lm.y = d_logits;
    lm.ntok = batch;
    lm.done = c->done;
    lm.keys = c->keys;
    lm.tokens = d_next_tokens;
    lm.pos = c->pos;
    lm.pos_add = 1;
    lm.err = c->err;
    return gemv<m1::kEpiArgmax>(lm, c->num_sms, st);
}

m1moe_status m1moe_cuda_prefill_step(m1moe_dense_ctx *c, m1moe_cuda_ctx *moe, const int32_t *d_tokens,
                                     int32_t T, int32_t *d_next_token, float *d_logits, void *stream) {
    if (!c || !moe || !d_tokens || !d_next_token) return fail(M1MOE_ERR_INVALID_ARG, "NULL pointer");
    const m1moe_dense_cfg &g = c->cfg;
    if (T < 1 || T > g.max_seq) return fail(M1MOE_ERR_INVALID_ARG, "tokens %d outside [1,%d]", T, g.max_seq);
    if (m1moe_status st = check_loaded(c)) return st;
    if (m1moe_status st = m1abi::moe_compatible(moe, g.hidden_dim, g.num_layers, 1, g.device)) return st;
    DevGuard dg(g.device);
    if (m1moe_status st = pf_dense_reserve(c, T)) return st;
    D_CK(cudaFuncSetAttribute(m1::k_attn_prefill_tiled, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)m1::attn_prefill_smem()));
    cudaStream_t st = as_stream(stream);
    const int h = g.hidden_dim, hd = c->hd;
    const size_t cache_layer = (size_t)g.max_batch * g.num_kv_heads * g.max_seq * hd;
    // 1. embed the prompt (InferenceEngine.swift:482-488, per token in the reference)
    if (m1moe_status s = launch_pdl(m1::k_embed, dim3(T), dim3(256), 0, st, "k_embed launch",
                                    (const uint16_t *)c->embed, d_tokens, (int)g.vocab_size, h, c->pf_res,
                                    (int)T, c->err))
        return s;
    for (int L = 0; L < g.num_layers; ++L) {
        // 2. input RMSNorm (bf16 operand) and the q|k|v projection of all tokens
        if (m1moe_status s = launch_pdl(m1::k_rmsnorm_bf16, dim3(T), dim3(256), 0, st, "k_rmsnorm_bf16 launch",
                                        (const float *)c->pf_res, (const uint16_t *)(c->in_norm + (size_t)L * h),
                                        (float)g.rms_norm_eps, c->pf_xn, h))
            return s;
        if (m1moe_status s = gemm_bf16(c, c->wqkv + (size_t)L * c->qkv_rows * h, c->pf_xn, c->pf_qkv,
                                       c->qkv_rows, h, T, false, st))
            return s;
        // 3. QK-norm, RoPE, KV store at positions pos .. pos+T-1, then causal attention
        uint16_t *kc = c->kc + (size_t)L * cache_layer, *vc = c->vc + (size_t)L * cache_layer;
        const uint16_t *qn = g.qk_norm ? c->qn + (size_t)L * hd : nullptr;
        const uint16_t *kn = g.qk_norm ? c->kn + (size_t)L * hd : nullptr;
        if (m1moe_status s = launch_pdl(m1::k_qk_rope_store, dim3(T, g.num_heads + g.num_kv_heads), dim3(32), 0, st,
                                        "k_qk_rope_store launch", c->pf_qkv, c->qkv_rows, (int)g.num_heads,
                                        (int)g.num_kv_heads, (const int *)c->pos, (int)g.max_seq, qn, kn,
                                        (float)g.rms_norm_eps, (float)g.rope_theta, kc, vc, c->err))
            return s;
        if (m1moe_status s = launch_pdl(m1::k_attn_prefill_tiled,
                                        dim3((T + m1::kPfQ - 1) / m1::kPfQ, g.num_heads), dim3(256),
                                        m1::attn_prefill_smem(), st, "k_attn_prefill_tiled launch",
                                        (const float *)c->pf_qkv, c->qkv_rows, (int)g.num_heads,
                                        (int)g.num_kv_heads, (int)T, (const int *)c->pos, (int)g.max_seq,
                                        1.0f / sqrtf((float)hd), (const uint16_t *)kc, (const uint16_t *)vc,
                                        c->pf_attn))
            return s;
        // 4. o projection added to the residual, then the post-attention RMSNorm
        if (m1moe_status s = gemm_bf16(c, c->wo + (size_t)L * h * c->qd, c->pf_attn, c->pf_res, h, c->qd, T,
                                       true, st))
            return s;
        if (m1moe_status s = launch_pdl(m1::k_rmsnorm, dim3(T), dim3(256), 0, st, "k_rmsnorm launch",
                                        (const void *)c->pf_res, 0, (const uint16_t *)(c->post_norm + (size_t)L * h),
                                        (float)g.rms_norm_eps, c->pf_hmid, h))
            return s;
        // 5. the MoE block of all tokens on the tensor cores
        if (m1moe_status s = m1moe_cuda_moe_prefill(moe, L, c->pf_hmid, M1MOE_DTYPE_F32, c->pf_res,
                                                    M1MOE_DTYPE_F32, c->pf_res, M1MOE_DTYPE_F32, T, nullptr,
                                                    nullptr, stream))
            return s;
    }
    // 6. the last token's final norm, LM head and greedy token; the position
    //    advances past the prompt
    m1::GemvParams lm{};
    lm.w = c->lm_head;
    lm.rows = g.vocab_size;
    lm.K = h;
    lm.x = c->pf_res + (size_t)(T - 1) * h;
    lm.norm_w = c->final_norm;
    lm.eps = g.rms_norm_eps;
    lm.y = d_logits;
    lm.ntok = 1;
    lm.done = c->done;
    lm.keys = c->keys;
    lm.tokens = d_next_token;
    lm.pos = c->pos;
    lm.pos_add = T;
    lm.err = c->err;
    return gemv<m1::kEpiArgmax>(lm, c->num_sms, st);
}

}  // extern "C"
