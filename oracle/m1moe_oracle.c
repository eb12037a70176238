/*
 * m1moe_oracle.c — CPU restatement of M1MoE's int4 expert-FFN arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
 * The product (m1moe_b200) never links or calls it.  Each function cites the
 * reference file:line it restates; see m1moe_oracle.h for the parity pin.
 *
 * Build: gcc -O3 -march=native -ffp-contract=off -fPIC -shared -pthread
 * (-ffp-contract=off keeps every FMA exactly where the reference writes one).
 */
#include "m1moe_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

float orc_bf16_to_f32(uint16_t b) {
    /* Shaders.metal:11-14: uint(b) << 16 reinterpreted as float. */
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t orc_f32_to_bf16(float f) {
    /* extract_olmoe.py:104-111: u32 + 0x7FFF + bit16, then >> 16. */
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t rounding_bias = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7FFFu + rounding_bias) >> 16);
}

size_t orc_expert_bytes(int hidden, int inter, int gs) {
    /* ModelSpec.swift:36-52. */
    size_t h = (size_t)hidden, i = (size_t)inter;
    size_t gw = i * (h / 8) * 4, gsb = i * (h / (size_t)gs) * 2;
    size_t dw = h * (i / 8) * 4, dsb = h * (i / (size_t)gs) * 2;
    return gw + gsb * 2 + gw + gsb * 2 + dw + dsb * 2;
}

void orc_expert_offsets(int hidden, int inter, int gs, size_t off[9]) {
    /* InferenceEngine.swift:79-97. */
    size_t h = (size_t)hidden, i = (size_t)inter;
    size_t gw = i * (h / 8) * 4, gsb = i * (h / (size_t)gs) * 2;
    size_t dw = h * (i / 8) * 4, dsb = h * (i / (size_t)gs) * 2;
    off[0] = 0;              /* gateW */
    off[1] = off[0] + gw;    /* gateS */
    off[2] = off[1] + gsb;   /* gateB */
    off[3] = off[2] + gsb;   /* upW   */
    off[4] = off[3] + gw;    /* upS   */
    off[5] = off[4] + gsb;   /* upB   */
    off[6] = off[5] + gsb;   /* downW */
    off[7] = off[6] + dw;    /* downS */
    off[8] = off[7] + dsb;   /* downB */
}

#define ORC_TG 64 /* threads per threadgroup, InferenceEngine.swift:463-464 */

void orc_matvec4bit_rows(const uint32_t *W, const uint16_t *S, const uint16_t *B,
                         const float *x, float *y, int out_dim, int in_dim, int gs,
                         int row0, int row1) {
    /* Shaders.metal:39-92. */
    const unsigned numWords = (unsigned)in_dim / 8;
    const unsigned numGroups = (unsigned)in_dim / (unsigned)gs;
    float shared[ORC_TG];
    for (int row = row0; row < row1 && row < out_dim; ++row) {
        const uint32_t *wRow = W + (size_t)row * numWords;
        const uint16_t *sRow = S + (size_t)row * numGroups;
        const uint16_t *bRow = B + (size_t)row * numGroups;
        for (unsigned lid = 0; lid < ORC_TG; ++lid) {
            float acc = 0.0f;
            for (unsigned w = lid; w < numWords; w += ORC_TG) {
                uint32_t packed = wRow[w];
                unsigned g = (w * 8) / (unsigned)gs;
                float scale = orc_bf16_to_f32(sRow[g]);
                float bias = orc_bf16_to_f32(bRow[g]);
                unsigned base = w * 8;
                for (unsigned b = 0; b < 8; ++b) {
                    float nibble = (float)((packed >> (b * 4)) & 0xFu);
                    float xv = x[base + b];
                    /* Shaders.metal:77 */
                    acc = fmaf(nibble, scale * xv, fmaf(bias, xv, acc));
                }
            }
            shared[lid] = acc;
        }
        /* Shaders.metal:86-90: tree reduction. */
        for (unsigned s = ORC_TG / 2; s > 0; s >>= 1)
            for (unsigned lid = 0; lid < s; ++lid) shared[lid] += shared[lid + s];
        y[row] = shared[0];
    }
}

/* The same arithmetic as orc_matvec4bit_rows, lane by lane in the same
 * order (for each lane: words lid, lid+64, ... ascending, nibbles 0..7), but
 * with the 64 lanes innermost so that the compiler vectorises across lanes:
 * per block of 64 words, x is read transposed (xT[b][lid] = x[8*(w0+lid)+b])
 * and the lanes' scales and biases are gathered once.  Bit-identical to the
 * plain restatement (tests/test_oracle_golden.py checks it); used for the
 * timed CPU baseline and for the large parity checks. */
void orc_matvec4bit_rows_lanes(const uint32_t *W, const uint16_t *S, const uint16_t *B,
                               const float *x, float *y, int out_dim, int in_dim, int gs,
                               int row0, int row1) {
    const unsigned numWords = (unsigned)in_dim / 8;
    const unsigned numGroups = (unsigned)in_dim / (unsigned)gs;
    const unsigned nblk = (numWords + ORC_TG - 1) / ORC_TG;
    float *xT = (float *)malloc(sizeof(float) * (size_t)nblk * 8 * ORC_TG);
    if (!xT) {
        orc_matvec4bit_rows(W, S, B, x, y, out_dim, in_dim, gs, row0, row1);
        return;
    }
    for (unsigned k = 0; k < nblk; ++k)
        for (unsigned b = 0; b < 8; ++b)
            for (unsigned lid = 0; lid < ORC_TG; ++lid) {
                const unsigned w = k * ORC_TG + lid;
                xT[((size_t)k * 8 + b) * ORC_TG + lid] = w < numWords ? x[w * 8 + b] : 0.0f;
            }
    float acc[ORC_TG], sc[ORC_TG], bi[ORC_TG], nib[ORC_TG];
    for (int row = row0; row < row1 && row < out_dim; ++row) {
        const uint32_t *wRow = W + (size_t)row * numWords;
        const uint16_t *sRow = S + (size_t)row * numGroups;
        const uint16_t *bRow = B + (size_t)row * numGroups;
        for (unsigned lid = 0; lid < ORC_TG; ++lid) acc[lid] = 0.0f;
        for (unsigned k = 0; k < nblk; ++k) {
            const unsigned w0 = k * ORC_TG;
            const unsigned nl = numWords - w0 < ORC_TG ? numWords - w0 : ORC_TG;
            for (unsigned lid = 0; lid < nl; ++lid) {
                const unsigned g = ((w0 + lid) * 8) / (unsigned)gs;
                sc[lid] = orc_bf16_to_f32(sRow[g]);
                bi[lid] = orc_bf16_to_f32(bRow[g]);
            }
            for (unsigned b = 0; b < 8; ++b) {
                const float *xb = xT + ((size_t)k * 8 + b) * ORC_TG;
                for (unsigned lid = 0; lid < nl; ++lid)
                    nib[lid] = (float)((wRow[w0 + lid] >> (b * 4)) & 0xFu);
                for (unsigned lid = 0; lid < nl; ++lid) {
                    const float xv = xb[lid];
                    /* Shaders.metal:77 */
                    acc[lid] = fmaf(nib[lid], sc[lid] * xv, fmaf(bi[lid], xv, acc[lid]));
                }
            }
        }
        /* Shaders.metal:86-90: tree reduction. */
        for (unsigned s2 = ORC_TG / 2; s2 > 0; s2 >>= 1)
            for (unsigned lid = 0; lid < s2; ++lid) acc[lid] += acc[lid + s2];
        y[row] = acc[0];
    }
    free(xT);
}

void orc_matvec4bit(const uint32_t *W, const uint16_t *S, const uint16_t *B,
                    const float *x, float *y, int out_dim, int in_dim, int gs) {
    orc_matvec4bit_rows_lanes(W, S, B, x, y, out_dim, in_dim, gs, 0, out_dim);
}

/* A persistent pool of host threads for row-partitioned work (threads are
 * created once, not per call): the caller publishes `njobs` row ranges of one
 * function, bumps the generation, runs job 0 itself and waits for the others. */
typedef void (*orc_rows_fn)(const void *arg, int row0, int row1);
typedef struct {
    orc_rows_fn fn;
    const void *arg;
    int row0, row1;
} orc_job;

#define ORC_MAX_THREADS 256
static struct {
    pthread_mutex_t mu;
    pthread_cond_t go, done;
    pthread_t th[ORC_MAX_THREADS];
    int nthreads;          /* workers started (jobs 1..nthreads) */
    unsigned gen;          /* bumped per batch of jobs */
    int pending;           /* jobs of this batch not finished yet */
    int njobs;
    orc_job jobs[ORC_MAX_THREADS];
} orc_pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER, PTHREAD_COND_INITIALIZER};
static pthread_mutex_t orc_pool_call = PTHREAD_MUTEX_INITIALIZER; /* one batch at a time */

static void *orc_pool_worker(void *arg) {
    const int id = (int)(intptr_t)arg;
    unsigned seen = 0;
    pthread_mutex_lock(&orc_pool.mu);
    for (;;) {
        while (orc_pool.gen == seen) pthread_cond_wait(&orc_pool.go, &orc_pool.mu);
        seen = orc_pool.gen;
        if (id < orc_pool.njobs) {
            orc_job j = orc_pool.jobs[id];
            pthread_mutex_unlock(&orc_pool.mu);
            j.fn(j.arg, j.row0, j.row1);
            pthread_mutex_lock(&orc_pool.mu);
            if (--orc_pool.pending == 0) pthread_cond_signal(&orc_pool.done);
        }
    }
    return NULL;
}

/* Run fn over rows [0, n) split into `nthreads` contiguous ranges. */
static void orc_parallel_rows(orc_rows_fn fn, const void *arg, int n, int nthreads) {
    if (nthreads <= 1 || n < 2 * nthreads) {
        fn(arg, 0, n);
        return;
    }
    if (nthreads > ORC_MAX_THREADS) nthreads = ORC_MAX_THREADS;
    pthread_mutex_lock(&orc_pool_call);
    pthread_mutex_lock(&orc_pool.mu);
    while (orc_pool.nthreads < nthreads - 1) { /* grow the pool on demand, once */
        const int id = orc_pool.nthreads + 1;
        if (pthread_create(&orc_pool.th[id - 1], NULL, orc_pool_worker, (void *)(intptr_t)id) != 0)
            break;
        ++orc_pool.nthreads;
    }
    const int workers = orc_pool.nthreads + 1 < nthreads ? orc_pool.nthreads + 1 : nthreads;
    const int per = (n + workers - 1) / workers;
    int njobs = 0;
    for (int t = 0; t < workers; ++t) {
        const int r0 = t * per, r1 = (t + 1) * per < n ? (t + 1) * per : n;
        if (r0 >= r1) break;
        orc_pool.jobs[t] = (orc_job){fn, arg, r0, r1};
        ++njobs;
    }
    orc_pool.njobs = njobs;
    orc_pool.pending = njobs - 1;
    ++orc_pool.gen;
    pthread_cond_broadcast(&orc_pool.go);
    orc_job j0 = orc_pool.jobs[0];
    pthread_mutex_unlock(&orc_pool.mu);
    j0.fn(j0.arg, j0.row0, j0.row1);
    pthread_mutex_lock(&orc_pool.mu);
    while (orc_pool.pending > 0) pthread_cond_wait(&orc_pool.done, &orc_pool.mu);
    pthread_mutex_unlock(&orc_pool.mu);
    pthread_mutex_unlock(&orc_pool_call);
}

typedef struct {
    const uint32_t *W;
    const uint16_t *S, *B;
    const float *x;
    float *y;
    int out_dim, in_dim, gs;
} orc_mv4_arg;

static void orc_mv4_rows(const void *a, int r0, int r1) {
    const orc_mv4_arg *j = (const orc_mv4_arg *)a;
    orc_matvec4bit_rows_lanes(j->W, j->S, j->B, j->x, j->y, j->out_dim, j->in_dim, j->gs, r0, r1);
}

void orc_matvec4bit_mt(const uint32_t *W, const uint16_t *S, const uint16_t *B,
                       const float *x, float *y, int out_dim, int in_dim, int gs,
                       int nthreads) {
    /* The reference dispatches one threadgroup per row (InferenceEngine.swift:463);
     * here rows are partitioned over host threads. */
    const orc_mv4_arg a = {W, S, B, x, y, out_dim, in_dim, gs};
    orc_parallel_rows(orc_mv4_rows, &a, out_dim, nthreads);
}

void orc_swiglu(const float *gate, const float *up, float *act, int n) {
    /* Shaders.metal:138-149 (the reference compiles with fastMath; this uses expf). */
    for (int i = 0; i < n; ++i) {
        float g = gate[i];
        act[i] = (g / (1.0f + expf(-g))) * up[i];
    }
}

void orc_moe_combine(const float *expert_outs, const float *w, const float *residual,
                     float *out, int K, int h) {
    /* Shaders.metal:360-376: residual first, then k ascending. */
    for (int i = 0; i < h; ++i) {
        float acc = residual[i];
        for (int k = 0; k < K; ++k) acc += w[k] * expert_outs[(size_t)k * h + i];
        out[i] = acc;
    }
}

void orc_router_scores(const uint16_t *router_bf16, const float *x, int E, int h,
                       float *scores) {
    /* InferenceEngine.swift:490-508. */
    for (int e = 0; e < E; ++e) {
        float dot = 0.0f;
        const uint16_t *row = router_bf16 + (size_t)e * h;
        for (int d = 0; d < h; ++d) dot += orc_bf16_to_f32(row[d]) * x[d];
        scores[e] = dot;
    }
    float mx = scores[0];
    for (int e = 1; e < E; ++e)
        if (scores[e] > mx) mx = scores[e];
    float sum = 0.0f;
    for (int e = 0; e < E; ++e) {
        scores[e] = expf(scores[e] - mx);
        sum += scores[e];
    }
    float inv = 1.0f / sum;
    for (int e = 0; e < E; ++e) scores[e] *= inv;
}

void orc_select_topk(const float *scores, int E, int K, int norm, int32_t *idx, float *w) {
    /* InferenceEngine.swift:510-519: selection of the K largest, descending,
     * ties to the lower index (a stable descending sort prefix). */
    unsigned char taken[4096];
    memset(taken, 0, sizeof(taken));
    for (int k = 0; k < K; ++k) {
        int best = -1;
        for (int e = 0; e < E; ++e) {
            if (taken[e]) continue;
            if (best < 0 || scores[e] > scores[best]) best = e;
        }
        taken[best] = 1;
        idx[k] = best;
        w[k] = scores[best];
    }
    if (norm) {
        /* reduce(0) { $0 + $1.1 }: sum in selection order, then divide. */
        float s = 0.0f;
        for (int k = 0; k < K; ++k) s += w[k];
        for (int k = 0; k < K; ++k) w[k] = w[k] / s;
    }
}

static void orc_expert_forward_mt(const uint8_t *block, const float *x, int hidden, int inter,
                                  int gs, float *y, float *scratch, int nthreads) {
    /* InferenceEngine.swift:401-444. */
    size_t off[9];
    orc_expert_offsets(hidden, inter, gs, off);
    float *gate = scratch, *up = scratch + inter, *act = scratch + 2 * (size_t)inter;
    orc_matvec4bit_mt((const uint32_t *)(block + off[0]), (const uint16_t *)(block + off[1]),
                      (const uint16_t *)(block + off[2]), x, gate, inter, hidden, gs, nthreads);
    orc_matvec4bit_mt((const uint32_t *)(block + off[3]), (const uint16_t *)(block + off[4]),
                      (const uint16_t *)(block + off[5]), x, up, inter, hidden, gs, nthreads);
    orc_swiglu(gate, up, act, inter);
    orc_matvec4bit_mt((const uint32_t *)(block + off[6]), (const uint16_t *)(block + off[7]),
                      (const uint16_t *)(block + off[8]), act, y, hidden, inter, gs, nthreads);
}

void orc_expert_forward(const uint8_t *block, const float *x, int hidden, int inter, int gs,
                        float *y, float *scratch) {
    orc_expert_forward_mt(block, x, hidden, inter, gs, y, scratch, 1);
}

int orc_moe_layer(const uint8_t *table, const uint16_t *router_bf16, const float *h_mid,
                  const float *residual, float *out, int B, int hidden, int inter, int E,
                  int K, int gs, int norm, int32_t *idx, float *w, int nthreads) {
    /* InferenceEngine.swift:240-266 (router, per-slot expert forward, combine). */
    if (E <= 0 || E > 4096 || K <= 0 || K > E) return -1;
    size_t eb = orc_expert_bytes(hidden, inter, gs);
    float *scores = (float *)malloc(sizeof(float) * (size_t)E);
    float *outs = (float *)malloc(sizeof(float) * (size_t)K * hidden);
    float *scratch = (float *)malloc(sizeof(float) * 3 * (size_t)inter);
    if (!scores || !outs || !scratch) {
        free(scores);
        free(outs);
        free(scratch);
        return -2;
    }
    for (int t = 0; t < B; ++t) {
        const float *x = h_mid + (size_t)t * hidden;
        orc_router_scores(router_bf16, x, E, hidden, scores);
        orc_select_topk(scores, E, K, norm, idx + (size_t)t * K, w + (size_t)t * K);
        for (int k = 0; k < K; ++k) {
            const uint8_t *block = table + (size_t)idx[(size_t)t * K + k] * eb;
            orc_expert_forward_mt(block, x, hidden, inter, gs, outs + (size_t)k * hidden,
                                  scratch, nthreads);
        }
        orc_moe_combine(outs, w + (size_t)t * K, residual + (size_t)t * hidden,
                        out + (size_t)t * hidden, K, hidden);
    }
    free(scores);
    free(outs);
    free(scratch);
    return 0;
}

/* ===================== the dense half of a decode step ===================== */

void orc_rmsnorm(const float *x, const uint16_t *w, float eps, float *y, int dim) {
    /* Shaders.metal:97-134: rmsNormSum with 256 threads (lane lid sums x[i]^2
     * for i = lid, lid+256, ...; tree reduction s = 128 .. 1), then
     * rmsNormApply: out = x * rsqrt(sumSq/dim + eps) * w. */
    float shared[256];
    for (int lid = 0; lid < 256; ++lid) {
        float acc = 0.0f;
        for (int i = lid; i < dim; i += 256) {
            const float v = x[i];
            acc += v * v;
        }
        shared[lid] = acc;
    }
    for (int s2 = 128; s2 > 0; s2 >>= 1)
        for (int lid = 0; lid < s2; ++lid) shared[lid] += shared[lid + s2];
    const float rms = 1.0f / sqrtf(shared[0] / (float)dim + eps);
    for (int i = 0; i < dim; ++i) y[i] = x[i] * rms * orc_bf16_to_f32(w[i]);
}

typedef struct {
    const uint16_t *W;
    const float *x;
    float *y;
    int out_dim, in_dim;
} orc_mv16_arg;

static void orc_mv16_rows(const void *a, int row0, int row1) {
    /* Shaders.metal:328-353 (matvecBF16): 64 threads per row, lane lid sums
     * bf16(w[i]) * x[i] for i = lid, lid+64, ...; tree reduction 32 .. 1.
     * Lanes innermost (vectorisable); each lane's order is the reference's. */
    const orc_mv16_arg *j = (const orc_mv16_arg *)a;
    float acc[64];
    for (int row = row0; row < row1 && row < j->out_dim; ++row) {
        const uint16_t *wr = j->W + (size_t)row * j->in_dim;
        for (int lid = 0; lid < 64; ++lid) acc[lid] = 0.0f;
        for (int i0 = 0; i0 < j->in_dim; i0 += 64) {
            const int nl = j->in_dim - i0 < 64 ? j->in_dim - i0 : 64;
            for (int lid = 0; lid < nl; ++lid)
                acc[lid] += orc_bf16_to_f32(wr[i0 + lid]) * j->x[i0 + lid];
        }
        for (int s2 = 32; s2 > 0; s2 >>= 1)
            for (int lid = 0; lid < s2; ++lid) acc[lid] += acc[lid + s2];
        j->y[row] = acc[0];
    }
}

void orc_matvec_bf16(const uint16_t *W, const float *x, float *y, int out_dim, int in_dim,
                     int nthreads) {
    const orc_mv16_arg a = {W, x, y, out_dim, in_dim};
    orc_parallel_rows(orc_mv16_rows, &a, out_dim, nthreads);
}

void orc_head_rmsnorm(float *buf, int num_heads, int head_dim, const uint16_t *w, float eps) {
    /* InferenceEngine.swift:538-548: every head uses the first head_dim weights. */
    for (int head = 0; head < num_heads; ++head) {
        float *b = buf + (size_t)head * head_dim;
        float ss = 0.0f;
        for (int d = 0; d < head_dim; ++d) ss += b[d] * b[d];
        const float rms = 1.0f / sqrtf(ss / (float)head_dim + eps);
        for (int d = 0; d < head_dim; ++d) b[d] *= rms * orc_bf16_to_f32(w[d]);
    }
}

void orc_rope(float *buf, int num_heads, int head_dim, float theta, int pos) {
    /* InferenceEngine.swift:521-536: half-split pairs (i, i + hd/2). */
    const int half = head_dim / 2;
    for (int head = 0; head < num_heads; ++head) {
        float *b = buf + (size_t)head * head_dim;
        for (int pair = 0; pair < half; ++pair) {
            const float freq = 1.0f / powf(theta, (float)(2 * pair) / (float)head_dim);
            const float angle = (float)pos * freq;
            const float c = cosf(angle), s = sinf(angle);
            const float x0 = b[pair], x1 = b[pair + half];
            b[pair] = x0 * c - x1 * s;
            b[pair + half] = x0 * s + x1 * c;
        }
    }
}

void orc_attention(const float *q, const uint16_t *kc, const uint16_t *vc, int num_heads,
                   int num_kv_heads, int head_dim, int max_seq, int seq_len, float *out) {
    /* Shaders.metal:209-313 (attnScores, attnSoftmax, attnValues) for one
     * sequence, with the cache in the B200 layout [kv_head][max_seq][head_dim]
     * (bf16; the reference keeps f32 rows [pos][kvDim]).  scale = 1/sqrt(hd)
     * (InferenceEngine.swift:358); heads per kv head = num_heads/num_kv_heads. */
    const int hpkv = num_heads / num_kv_heads;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float *scores = (float *)malloc(sizeof(float) * (size_t)seq_len);
    if (!scores) return;
    for (int head = 0; head < num_heads; ++head) {
        const int kvh = head / hpkv;
        const float *qh = q + (size_t)head * head_dim;
        const uint16_t *kb = kc + (size_t)kvh * max_seq * head_dim;
        const uint16_t *vb = vc + (size_t)kvh * max_seq * head_dim;
        /* scores: 64 threads per (head, pos), strided over head_dim, tree */
        for (int p = 0; p < seq_len; ++p) {
            float sh[64];
            for (int lid = 0; lid < 64; ++lid) {
                float acc = 0.0f;
                for (int i = lid; i < head_dim; i += 64)
                    acc += qh[i] * orc_bf16_to_f32(kb[(size_t)p * head_dim + i]);
                sh[lid] = acc;
            }
            for (int s2 = 32; s2 > 0; s2 >>= 1)
                for (int lid = 0; lid < s2; ++lid) sh[lid] += sh[lid + s2];
            scores[p] = sh[0] * scale;
        }
        /* softmax: 256 threads, max tree, exp-sum tree, multiply by 1/sum */
        float sh[256];
        for (int lid = 0; lid < 256; ++lid) {
            float mx = -INFINITY;
            for (int i = lid; i < seq_len; i += 256) mx = scores[i] > mx ? scores[i] : mx;
            sh[lid] = mx;
        }
        for (int s2 = 128; s2 > 0; s2 >>= 1)
            for (int lid = 0; lid < s2; ++lid) sh[lid] = sh[lid + s2] > sh[lid] ? sh[lid + s2] : sh[lid];
        const float maxv = sh[0];
        for (int lid = 0; lid < 256; ++lid) {
            float sum = 0.0f;
            for (int i = lid; i < seq_len; i += 256) {
                const float e = expf(scores[i] - maxv);
                scores[i] = e;
                sum += e;
            }
            sh[lid] = sum;
        }
        for (int s2 = 128; s2 > 0; s2 >>= 1)
            for (int lid = 0; lid < s2; ++lid) sh[lid] += sh[lid + s2];
        const float inv = 1.0f / sh[0];
        for (int i = 0; i < seq_len; ++i) scores[i] *= inv;
        /* values: one thread per (head, dim), positions in order */
        for (int d = 0; d < head_dim; ++d) {
            float acc = 0.0f;
            for (int p = 0; p < seq_len; ++p)
                acc += scores[p] * orc_bf16_to_f32(vb[(size_t)p * head_dim + d]);
            out[(size_t)head * head_dim + d] = acc;
        }
    }
    free(scores);
}

int orc_argmax(const float *logits, int n) {
    /* InferenceEngine.swift:552-555: the first maximum wins. */
    int best = 0;
    float bv = logits[0];
    for (int i = 1; i < n; ++i)
        if (logits[i] > bv) {
            bv = logits[i];
            best = i;
        }
    return best;
}
