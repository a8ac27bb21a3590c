/*
 * moe_oracle.c -- CPU restatement of jero-engine's MoE FFN path (test infrastructure only).
 *
 * Compiled with -ffp-contract=off so that every multiply and add below rounds
 * separately unless fmaf() is written out. Each function cites the reference
 * code it restates; paths are relative to the jero-engine source tree.
 */
#include "moe_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ formats */

/* IEEE binary16 -> binary32 (exact). The reference decodes block scales the same
 * way inside jero-core / jero-kernels-rvv; KAT: 0x3C00 -> 1.0, 0x3800 -> 0.5
 * (src/gemma.rs:1628-1662). */
float orc_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* GGUF block sizes: Q8_0 = 32 values in 34 B (f16 d + 32 x int8); Q4_K = 256
 * values in 144 B (f16 d, f16 dmin, 12 B of 6-bit scales/mins, 128 B nibbles);
 * the reference asserts 288 B for a 512-element Q4_K tensor (src/weights.rs:1204-1208). */
size_t orc_row_bytes(int type, int cols)
{
    if (cols <= 0) return 0;
    switch (type) {
    case ORC_F32: return (size_t)cols * 4;
    case ORC_F16: return (size_t)cols * 2;
    case ORC_Q8_0: return (cols % 32) ? 0 : (size_t)(cols / 32) * 34;
    case ORC_Q4_K: return (cols % 256) ? 0 : (size_t)(cols / 256) * 144;
    default: return 0;
    }
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* 6-bit scale and min of sub-block j (0..7) from the 12 packed bytes of a Q4_K
 * super-block (GGUF layout: j<4 low 6 bits of bytes j / j+4; j>=4 a nibble of
 * byte j+4 plus the top two bits of bytes j-4 / j). */
static inline void q4k_scale_min(const uint8_t *sc12, int j, int *sc, int *mn)
{
    if (j < 4) {
        *sc = sc12[j] & 63;
        *mn = sc12[j + 4] & 63;
    } else {
        *sc = (sc12[j + 4] & 0x0F) | ((sc12[j - 4] >> 6) << 4);
        *mn = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
    }
}

/* Dequantise one row (the reference's dequantize_token_row, src/gemma.rs:1628-1662;
 * Q4_K element = d*sc*q - dmin*m, nibble l of byte 32g+l is value 64g+l (low)
 * and 64g+32+l (high)). */
int orc_dequantize_row(int type, const uint8_t *row, int cols, float *dst)
{
    if (!orc_row_bytes(type, cols)) return ORC_ERR_ARG;
    if (type == ORC_F32) { memcpy(dst, row, (size_t)cols * 4); return ORC_OK; }
    if (type == ORC_F16) {
        for (int i = 0; i < cols; i++) dst[i] = orc_f16_to_f32(rd16(row + 2 * i));
        return ORC_OK;
    }
    if (type == ORC_Q8_0) {
        for (int b = 0; b < cols / 32; b++) {
            const uint8_t *blk = row + 34 * b;
            float d = orc_f16_to_f32(rd16(blk));
            for (int i = 0; i < 32; i++) dst[32 * b + i] = d * (float)(int8_t)blk[2 + i];
        }
        return ORC_OK;
    }
    /* Q4_K */
    for (int s = 0; s < cols / 256; s++) {
        const uint8_t *blk = row + 144 * s;
        float d = orc_f16_to_f32(rd16(blk));
        float dmin = orc_f16_to_f32(rd16(blk + 2));
        const uint8_t *sc12 = blk + 4, *qs = blk + 16;
        float *y = dst + 256 * s;
        for (int g = 0; g < 4; g++) {
            int sc0, m0, sc1, m1;
            q4k_scale_min(sc12, 2 * g, &sc0, &m0);
            q4k_scale_min(sc12, 2 * g + 1, &sc1, &m1);
            float d0 = d * (float)sc0, n0 = dmin * (float)m0;
            float d1 = d * (float)sc1, n1 = dmin * (float)m1;
            for (int l = 0; l < 32; l++) {
                y[64 * g + l] = d0 * (float)(qs[32 * g + l] & 0x0F) - n0;
                y[64 * g + 32 + l] = d1 * (float)(qs[32 * g + l] >> 4) - n1;
            }
        }
    }
    return ORC_OK;
}

/* ------------------------------------------------------ activation blocks */

/* The build's definition of the activation side of a quantised dot (the
 * reference's vec_dot_q8_0 / vec_dot_q4_k_m take f32 input and their inner
 * numerics are not visible): each run of 32 values becomes int8 q = round(x*127/amax)
 * (half away from zero, clamped to +-127, NaN -> -127) with scale d = amax/127. */
int orc_quantize_act(const float *x, int cols, int8_t *xq, float *dx)
{
    if (cols <= 0 || cols % 32) return ORC_ERR_ARG;
    for (int b = 0; b < cols / 32; b++) {
        const float *v = x + 32 * b;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(v[i]));
        float id = amax > 0.0f ? 127.0f / amax : 0.0f;
        for (int i = 0; i < 32; i++) {
            float r = roundf(v[i] * id);
            r = fminf(fmaxf(r, -127.0f), 127.0f);
            xq[32 * b + i] = (int8_t)r;
        }
        dx[b] = amax / 127.0f;
    }
    return ORC_OK;
}

int orc_block_dots(int type, const uint8_t *wrow, const int8_t *xq, int cols,
                   int32_t *isum, int32_t *xsum)
{
    if (!orc_row_bytes(type, cols) || (type != ORC_Q8_0 && type != ORC_Q4_K)) return ORC_ERR_ARG;
    if (type == ORC_Q8_0) {
        for (int b = 0; b < cols / 32; b++) {
            const int8_t *q = (const int8_t *)(wrow + 34 * b + 2);
            int32_t s = 0, t = 0;
            for (int i = 0; i < 32; i++) { s += (int32_t)q[i] * xq[32 * b + i]; t += xq[32 * b + i]; }
            isum[b] = s;
            if (xsum) xsum[b] = t;
        }
        return ORC_OK;
    }
    for (int sb = 0; sb < cols / 256; sb++) {
        const uint8_t *qs = wrow + 144 * sb + 16;
        const int8_t *a = xq + 256 * sb;
        for (int g = 0; g < 4; g++) {
            int32_t s0 = 0, s1 = 0, t0 = 0, t1 = 0;
            for (int l = 0; l < 32; l++) {
                s0 += (int32_t)(qs[32 * g + l] & 0x0F) * a[64 * g + l];
                s1 += (int32_t)(qs[32 * g + l] >> 4) * a[64 * g + 32 + l];
                t0 += a[64 * g + l];
                t1 += a[64 * g + 32 + l];
            }
            isum[8 * sb + 2 * g] = s0;
            isum[8 * sb + 2 * g + 1] = s1;
            if (xsum) { xsum[8 * sb + 2 * g] = t0; xsum[8 * sb + 2 * g + 1] = t1; }
        }
    }
    return ORC_OK;
}

/* Scaling of the integer block sums (build-defined, see orc_quantize_act):
 *   Q8_0 block b:       (d_w * d_x[b]) * isum[b]
 *   Q4_K sub-block j:   d_x[j] * ((d*sc_j) * isum[j] - (dmin*m_j) * xsum[j])
 * summed in block order in f32. */
float orc_row_dot_q(int type, const uint8_t *wrow, const int8_t *xq, const float *dx, int cols)
{
    int32_t isum[1024], xsum[1024];
    float acc = 0.0f;
    if (cols / 32 > 1024) return NAN;
    if (orc_block_dots(type, wrow, xq, cols, isum, xsum)) return NAN;
    if (type == ORC_Q8_0) {
        for (int b = 0; b < cols / 32; b++) {
            float dw = orc_f16_to_f32(rd16(wrow + 34 * b));
            acc += (dw * dx[b]) * (float)isum[b];
        }
        return acc;
    }
    for (int sb = 0; sb < cols / 256; sb++) {
        const uint8_t *blk = wrow + 144 * sb;
        float d = orc_f16_to_f32(rd16(blk)), dmin = orc_f16_to_f32(rd16(blk + 2));
        for (int j = 0; j < 8; j++) {
            int sc, mn;
            q4k_scale_min(blk + 4, j, &sc, &mn);
            int b = 8 * sb + j;
            acc += dx[b] * ((d * (float)sc) * (float)isum[b] - (dmin * (float)mn) * (float)xsum[b]);
        }
    }
    return acc;
}

/* f32 row dot for F32 weights: sequential multiply-then-add, the natural
 * reading of dot_product_f32_scalar (src/gemma.rs:186). */
static float row_dot_f32(const float *w, const float *x, int cols)
{
    float acc = 0.0f;
    for (int i = 0; i < cols; i++) acc += w[i] * x[i];
    return acc;
}

/* ------------------------------------------------------------------ router */

/* Router logits in the build's canonical f32 order (the reference's
 * dot_product_f32_scalar order is not visible, so one order is fixed here and
 * in the CUDA router): element h goes to partial (h/4) mod 32, each partial is
 * an fmaf chain in increasing h, and the 32 partials are combined by the xor
 * butterfly with offsets 16, 8, 4, 2, 1. Row e of the router is logit e
 * (view [H, E], src/qwen_deepseek.rs:2665-2673). */
void orc_router_logits(const float *w, const float *x, int E, int H, float *logits)
{
    for (int e = 0; e < E; e++) {
        const float *row = w + (size_t)e * H;
        float p[32], q[32];
        for (int l = 0; l < 32; l++) p[l] = 0.0f;
        for (int h = 0; h < H; h++) {
            int l = (h >> 2) & 31;
            p[l] = fmaf(row[h], x[h], p[l]);
        }
        for (int off = 16; off >= 1; off >>= 1) {
            for (int l = 0; l < 32; l++) q[l] = p[l] + p[l ^ off];
            memcpy(p, q, sizeof p);
        }
        logits[e] = p[0];
    }
}

/* RMSNorm of one row in the build's fixed f32 order (the reference's
 * rmsnorm_standard, src/qwen_deepseek.rs:521-528, calls a kernel of the
 * un-vendored jero-kernels-rvv crate whose order is not visible): element h
 * goes to partial (h/4) mod 32 as x*x fmaf chains in increasing h, the 32
 * partials are combined by the xor butterfly 16..1, then mean = sum / H,
 * inv = 1 / sqrt(mean + eps) and out = (x * inv) * w, each rounded once.
 * w NULL: ones. Same order as the library's rmsnorm_kernel. */
void orc_rmsnorm(const float *x, const float *w, int H, float eps, float *out)
{
    float p[32], q[32];
    for (int l = 0; l < 32; l++) p[l] = 0.0f;
    for (int h = 0; h < H; h++) {
        int l = (h >> 2) & 31;
        p[l] = fmaf(x[h], x[h], p[l]);
    }
    for (int off = 16; off >= 1; off >>= 1) {
        for (int l = 0; l < 32; l++) q[l] = p[l] + p[l ^ off];
        memcpy(p, q, sizeof p);
    }
    const float mean = p[0] / (float)H;
    const float inv = 1.0f / sqrtf(mean + eps);
    for (int h = 0; h < H; h++) {
        const float y = x[h] * inv;
        out[h] = w ? y * w[h] : y;
    }
}

/* Rust f32::total_cmp as a signed-integer key (src/gemma.rs:417). */
static inline int32_t total_key(float f)
{
    int32_t b;
    memcpy(&b, &f, 4);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

static inline int rank_before(int32_t ka, int ia, int32_t kb, int ib)
{
    return ka > kb || (ka == kb && ia < ib);
}

/* Softmax over all E logits exactly as select_top_k_experts computes it
 * (src/gemma.rs:368-400): max over finite logits, exp(l - max) for finite l
 * else 0, sequential f32 sum, divide; uniform 1/E when the sum is 0 or not finite. */
static void softmax_a2(const float *lg, int E, float *p)
{
    float mx = -INFINITY;
    for (int e = 0; e < E; e++) if (isfinite(lg[e])) mx = fmaxf(mx, lg[e]);
    float sum = 0.0f;
    for (int e = 0; e < E; e++) {
        p[e] = (isfinite(lg[e]) && isfinite(mx)) ? expf(lg[e] - mx) : 0.0f;
        sum += p[e];
    }
    if (sum > 0.0f && isfinite(sum)) {
        for (int e = 0; e < E; e++) p[e] /= sum;
    } else {
        float u = 1.0f / (float)E;
        for (int e = 0; e < E; e++) p[e] = u;
    }
}

/* Expert selection for one token. Restates:
 *   - select_top_k_experts (src/gemma.rs:362-442): rank by logit with
 *     total_cmp descending, non-finite -> -inf, ties to the lower index; take k;
 *     renormalise over the chosen (uniform 1/k if the sum is 0 or not finite).
 *   - select_experts_with_optional_bias (src/qwen_deepseek.rs:773-831): with
 *     exp_probs_b, rank on logit+bias, weigh with the unbiased softmax, renormalise.
 * Build-defined extensions (no reference counterpart): logit_bias added to the
 * logits first; group-limited selection (group score = best member key, keep
 * topk_groups groups, ties to the lower group); normalize==0 returns the raw
 * softmax probabilities times scale. */
int orc_select(const orc_layer *L, const float *logits_in, int32_t *idx, float *w)
{
    int E = L->n_experts, k = L->top_k < E ? L->top_k : E;
    if (E <= 0 || k <= 0) return 0;
    float *lg = (float *)malloc(sizeof(float) * E * 2);
    int32_t *key = (int32_t *)malloc(sizeof(int32_t) * E);
    unsigned char *cand = (unsigned char *)malloc(E);
    if (!lg || !key || !cand) { free(lg); free(key); free(cand); return -ORC_ERR_NOMEM; }
    float *p = lg + E;

    for (int e = 0; e < E; e++) lg[e] = L->logit_bias ? logits_in[e] + L->logit_bias[e] : logits_in[e];
    for (int e = 0; e < E; e++) {
        float s = L->sel_bias ? lg[e] + L->sel_bias[e] : lg[e];
        key[e] = total_key(isfinite(s) ? s : -INFINITY);
        cand[e] = 1;
    }
    if (L->n_groups > 0 && L->topk_groups > 0 && L->topk_groups < L->n_groups && E % L->n_groups == 0) {
        int G = L->n_groups, gs = E / G;
        int32_t gkey[256];
        unsigned char gsel[256];
        if (G > 256) { free(lg); free(key); free(cand); return -ORC_ERR_ARG; }
        for (int g = 0; g < G; g++) {
            int32_t best = key[g * gs];
            for (int j = 1; j < gs; j++) if (key[g * gs + j] > best) best = key[g * gs + j];
            gkey[g] = best;
            gsel[g] = 0;
        }
        for (int r = 0; r < L->topk_groups; r++) {
            int bi = -1;
            for (int g = 0; g < G; g++)
                if (!gsel[g] && (bi < 0 || rank_before(gkey[g], g, gkey[bi], bi))) bi = g;
            gsel[bi] = 1;
        }
        for (int e = 0; e < E; e++) cand[e] = gsel[e / gs];
        int nc = 0;
        for (int e = 0; e < E; e++) nc += cand[e];
        if (k > nc) k = nc;
    }
    for (int r = 0; r < k; r++) {
        int bi = -1;
        for (int e = 0; e < E; e++)
            if (cand[e] && (bi < 0 || rank_before(key[e], e, key[bi], bi))) bi = e;
        idx[r] = bi;
        cand[bi] = 0;
    }

    if (L->sel_bias) {
        /* select_experts_with_optional_bias: probs[idx] / sum_probs, 0 if the sum is bad */
        float mx = -INFINITY, sum = 0.0f;
        for (int e = 0; e < E; e++) if (isfinite(lg[e])) mx = fmaxf(mx, lg[e]);
        for (int e = 0; e < E; e++) {
            p[e] = (isfinite(lg[e]) && isfinite(mx)) ? expf(lg[e] - mx) : 0.0f;
            sum += p[e];
        }
        for (int r = 0; r < k; r++) w[r] = (sum > 0.0f && isfinite(sum)) ? p[idx[r]] / sum : 0.0f;
        float ss = 0.0f;
        for (int r = 0; r < k; r++) ss += w[r];
        if (ss > 0.0f && isfinite(ss)) {
            for (int r = 0; r < k; r++) w[r] /= ss;
        } else {
            for (int r = 0; r < k; r++) w[r] = 1.0f / (float)k;
        }
    } else {
        softmax_a2(lg, E, p);
        for (int r = 0; r < k; r++) w[r] = p[idx[r]];
        if (L->normalize) {
            float ss = 0.0f;
            for (int r = 0; r < k; r++) ss += w[r];
            if (ss > 0.0f && isfinite(ss)) {
                for (int r = 0; r < k; r++) w[r] /= ss;
            } else {
                for (int r = 0; r < k; r++) w[r] = 1.0f / (float)k;
            }
        } else if (L->scale != 1.0f) {
            for (int r = 0; r < k; r++) w[r] *= L->scale;
        }
    }
    free(lg); free(key); free(cand);
    return k;
}

/* --------------------------------------------------------------- matvecs */

/* Row split of matvec_any (src/gemma.rs:114-133): rows >= 64 and more than
 * one thread -> chunks of clamp(ceil(rows/threads), 16, 2048) rows. */
static int chunk_rows(int rows, int n_threads)
{
    if (rows < 64 || n_threads <= 1) return rows;
    int c = (rows + n_threads - 1) / n_threads;
    if (c < 16) c = 16;
    if (c > 2048) c = 2048;
    return c;
}

/* One row chunk of a matvec: the work unit that the reference hands to a
 * pool thread (try_par_chunks_mut, src/gemma.rs:126-131). */
typedef struct {
    const orc_matrix *m;      /* NULL: router rows */
    const float *router;
    int e, H, r0, r1;
    const float *x;
    const int8_t *xq;         /* NULL: quantised rows are dequantised and dotted with x in f32 */
    const float *dx;
    float *out;
} mv_chunk;

static void run_chunk(const mv_chunk *c)
{
    if (!c->m) {
        orc_router_logits(c->router + (size_t)c->r0 * c->H, c->x, c->r1 - c->r0, c->H, c->out + c->r0);
        return;
    }
    const orc_matrix *m = c->m;
    size_t rb = orc_row_bytes(m->type, m->cols);
    const uint8_t *base = m->data + (size_t)c->e * m->expert_stride;
    float wrow[16384];
    for (int r = c->r0; r < c->r1; r++) {
        const uint8_t *row = base + (size_t)r * rb;
        if (m->type == ORC_F32) {
            c->out[r] = row_dot_f32((const float *)row, c->x, m->cols);
        } else if (c->xq) {
            c->out[r] = orc_row_dot_q(m->type, row, c->xq, c->dx, m->cols);
        } else if (m->cols <= 16384 && orc_dequantize_row(m->type, row, m->cols, wrow) == ORC_OK) {
            c->out[r] = row_dot_f32(wrow, c->x, m->cols);   /* the other reading of vec_dot_* */
        } else {
            c->out[r] = NAN;
        }
    }
}

/* A persistent pool of worker threads, like the reference's WorkerPool
 * (src/affinity.rs:1991): the caller publishes the chunks of one matvec, the
 * workers and the caller take chunks until none is left, the caller waits. */
static struct {
    pthread_mutex_t mu;
    pthread_cond_t work, done;
    pthread_t th[255];
    int n_workers;
    mv_chunk *jobs;
    int n_jobs, next, pending;
    unsigned gen;
    int stop;
} g_pool = {.mu = PTHREAD_MUTEX_INITIALIZER, .work = PTHREAD_COND_INITIALIZER, .done = PTHREAD_COND_INITIALIZER};

static void pool_drain(void)
{
    for (;;) {
        pthread_mutex_lock(&g_pool.mu);
        if (g_pool.next >= g_pool.n_jobs) {
            pthread_mutex_unlock(&g_pool.mu);
            return;
        }
        mv_chunk *c = &g_pool.jobs[g_pool.next++];
        pthread_mutex_unlock(&g_pool.mu);
        run_chunk(c);
        pthread_mutex_lock(&g_pool.mu);
        if (--g_pool.pending == 0) pthread_cond_broadcast(&g_pool.done);
        pthread_mutex_unlock(&g_pool.mu);
    }
}

static void *pool_worker(void *arg)
{
    (void)arg;
    unsigned seen = 0;
    for (;;) {
        pthread_mutex_lock(&g_pool.mu);
        while (g_pool.gen == seen && !g_pool.stop) pthread_cond_wait(&g_pool.work, &g_pool.mu);
        if (g_pool.stop) {
            pthread_mutex_unlock(&g_pool.mu);
            return NULL;
        }
        seen = g_pool.gen;
        pthread_mutex_unlock(&g_pool.mu);
        pool_drain();
    }
}

static void pool_resize(int n_workers)
{
    if (n_workers > 255) n_workers = 255;
    if (n_workers == g_pool.n_workers) return;
    pthread_mutex_lock(&g_pool.mu);
    g_pool.stop = 1;
    pthread_cond_broadcast(&g_pool.work);
    pthread_mutex_unlock(&g_pool.mu);
    for (int i = 0; i < g_pool.n_workers; i++) pthread_join(g_pool.th[i], NULL);
    g_pool.stop = 0;
    g_pool.n_workers = 0;
    for (int i = 0; i < n_workers; i++) {
        if (pthread_create(&g_pool.th[i], NULL, pool_worker, NULL) != 0) break;
        g_pool.n_workers++;
    }
}

/* Runs the chunks of one matvec on the pool (chunk work also on the caller). */
static void run_chunks(mv_chunk *cs, int n)
{
    if (n <= 1 || g_pool.n_workers == 0) {
        for (int i = 0; i < n; i++) run_chunk(&cs[i]);
        return;
    }
    pthread_mutex_lock(&g_pool.mu);
    g_pool.jobs = cs;
    g_pool.n_jobs = n;
    g_pool.next = 0;
    g_pool.pending = n;
    g_pool.gen++;
    pthread_cond_broadcast(&g_pool.work);
    pthread_mutex_unlock(&g_pool.mu);
    pool_drain();
    pthread_mutex_lock(&g_pool.mu);
    while (g_pool.pending > 0) pthread_cond_wait(&g_pool.done, &g_pool.mu);
    g_pool.n_jobs = 0;
    pthread_mutex_unlock(&g_pool.mu);
}

static void split_rows(mv_chunk tmpl, int rows, int n_threads)
{
    int chunk = chunk_rows(rows, n_threads);
    int n = (rows + chunk - 1) / chunk;
    mv_chunk cs[256];
    if (n > 256) n = 256, chunk = (rows + 255) / 256;
    for (int i = 0; i < n; i++) {
        cs[i] = tmpl;
        cs[i].r0 = i * chunk;
        cs[i].r1 = (i + 1) * chunk < rows ? (i + 1) * chunk : rows;
    }
    run_chunks(cs, n);
}

/* out[r] = row r of matrix e . x, for a quantised matrix (xq/dx) or F32 (x). */
static void matvec(const orc_matrix *m, int e, const float *x, const int8_t *xq, const float *dx,
                   float *out, int n_threads)
{
    mv_chunk t = {m, NULL, e, 0, 0, 0, x, xq, dx, out};
    split_rows(t, m->rows, n_threads);
}

static void router_matvec(const float *w, const float *x, int E, int H, float *logits, int n_threads)
{
    mv_chunk t = {NULL, w, 0, H, 0, 0, x, NULL, NULL, logits};
    split_rows(t, E, n_threads);
}

typedef struct {
    float *g, *u, *a, *y, *adx;
    int8_t *aq;
} expert_scratch;

/* run_single_swiglu_expert (src/qwen_deepseek.rs:748-771): gate and up matvecs,
 * a = silu(g)*u with silu(g) = g / (1 + exp(-g)), then the down matvec. */
static void swiglu_expert(const orc_matrix *G, const orc_matrix *U, const orc_matrix *D, int e,
                          const float *x, const int8_t *xq, const float *dx,
                          expert_scratch *s, int n_threads)
{
    int I = G->rows;
    matvec(G, e, x, xq, dx, s->g, n_threads);
    matvec(U, e, x, xq, dx, s->u, n_threads);
    for (int i = 0; i < I; i++) s->a[i] = (s->g[i] / (1.0f + expf(-s->g[i]))) * s->u[i];
    /* xq == NULL: f32 activations throughout (no block quantisation of a) */
    int quant = D->type != ORC_F32 && xq != NULL;
    if (quant) orc_quantize_act(s->a, I, s->aq, s->adx);
    matvec(D, e, s->a, quant ? s->aq : NULL, s->adx, s->y, n_threads);
}

static int check_matrix(const orc_matrix *m, int rows, int cols)
{
    if (!m->data) return ORC_ERR_ARG;
    if (m->rows != rows || m->cols != cols) return ORC_ERR_ARG;
    if (!orc_row_bytes(m->type, cols)) return ORC_ERR_ARG;
    return ORC_OK;
}

/* dispatch_qwen3_moe_ffn (src/qwen_deepseek.rs:847-951) for T tokens, one
 * token at a time like the reference prefill loop (src/qwen_deepseek.rs:2298-2312):
 * out = 0; out += shared(x); logits; select; for each chosen (e, w) in rank
 * order out += w * expert_e(x) (multiply, then add). sel_idx/sel_w get T*k
 * entries in rank order. */
int orc_moe_forward(const orc_layer *L, int T, const float *x, float *out,
                    int32_t *sel_idx, float *sel_w, int n_threads)
{
    return orc_moe_forward_ex(L, T, x, out, sel_idx, sel_w, n_threads, 0);
}

/* act_f32 = 1: the same block with the other reading of the reference's
 * quantised dots (vec_dot_q8_0 / vec_dot_q4_k_m, src/gemma.rs:66-95): every
 * weight row dequantised to f32 (orc_dequantize_row) and dotted with the f32
 * activations (sequential multiply-then-add), no activation quantisation of x
 * or of the SwiGLU output. Routing is the same in both readings. */
int orc_moe_forward_ex(const orc_layer *L, int T, const float *x, float *out,
                       int32_t *sel_idx, float *sel_w, int n_threads, int act_f32)
{
    int H = L->hidden, E = L->n_experts, k = L->top_k;
    if (T < 0 || H <= 0 || E <= 0 || k <= 0 || k > E || !L->router) return ORC_ERR_ARG;
    int I = L->gate.rows;
    if (check_matrix(&L->gate, I, H) || check_matrix(&L->up, I, H) || check_matrix(&L->down, H, I))
        return ORC_ERR_ARG;
    int S = L->sh_gate.data ? L->sh_gate.rows : 0;
    if (S && (check_matrix(&L->sh_gate, S, H) || check_matrix(&L->sh_up, S, H) ||
              check_matrix(&L->sh_down, H, S)))
        return ORC_ERR_ARG;
    int need_q = !act_f32 && (L->gate.type != ORC_F32 || L->up.type != ORC_F32 ||
                              (S && (L->sh_gate.type != ORC_F32 || L->sh_up.type != ORC_F32)));
    if (need_q && H % 32) return ORC_ERR_ARG;
    if (n_threads < 1) n_threads = 1;
    pool_resize(n_threads - 1);

    int W = I > S ? I : S;
    size_t fl = (size_t)E + 4 * (size_t)W + 2 * (size_t)H + (size_t)W / 32 + (size_t)H / 32 + 8 + (size_t)k;
    float *buf = (float *)calloc(fl, sizeof(float));
    int8_t *qb = (int8_t *)calloc((size_t)H + (size_t)W + 64, 1);
    int32_t *idx = (int32_t *)calloc((size_t)k, sizeof(int32_t));
    if (!buf || !qb || !idx) { free(buf); free(qb); free(idx); return ORC_ERR_NOMEM; }
    float *logits = buf, *wsel = logits + E;
    expert_scratch s;
    s.g = wsel + k; s.u = s.g + W; s.a = s.u + W; s.y = s.a + W;
    float *xdx = s.y + H; s.adx = xdx + H / 32 + 1;
    int8_t *xq = qb; s.aq = qb + H;

    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * H;
        float *ot = out + (size_t)t * H;
        if (need_q) orc_quantize_act(xt, H, xq, xdx);
        for (int h = 0; h < H; h++) ot[h] = 0.0f;
        if (S) {
            swiglu_expert(&L->sh_gate, &L->sh_up, &L->sh_down, 0, xt, act_f32 ? NULL : xq, xdx, &s, n_threads);
            for (int h = 0; h < H; h++) ot[h] += s.y[h];
        }
        router_matvec(L->router, xt, E, H, logits, n_threads);
        int n = orc_select(L, logits, idx, wsel);
        for (int r = 0; r < n; r++) {
            swiglu_expert(&L->gate, &L->up, &L->down, idx[r], xt, act_f32 ? NULL : xq, xdx, &s, n_threads);
            for (int h = 0; h < H; h++) ot[h] += wsel[r] * s.y[h];
        }
        for (int r = 0; r < k; r++) {
            if (sel_idx) sel_idx[(size_t)t * k + r] = r < n ? idx[r] : -1;
            if (sel_w) sel_w[(size_t)t * k + r] = r < n ? wsel[r] : 0.0f;
        }
    }
    free(buf); free(qb); free(idx);
    return ORC_OK;
}

/* project_lm_head (src/qwen_deepseek.rs:584-632) for T rows. head: GGUF bytes
 * of the chosen tensor (output.weight, else token_embd.weight; NULL: none),
 * shaped = its shape is [hidden, head_rows] with head_rows > 0, else
 * head_rows = elements / hidden (0: not whole rows). Per row: the first
 * min(n_logits, head_rows) logits are the matvec (matvec_any: F32 rows
 * sequential multiply-then-add, quantised rows with int8 activation blocks as
 * the experts), the rest normed[i mod hidden] * 0.05; the unshaped head is used
 * only when head_rows == n_logits; otherwise base + normed[i mod hidden] * 0.1 +
 * (i mod 13) * 0.01 with base = tanh(sum(normed) / 16), the sum in element
 * order. */
int orc_lm_head(int type, const uint8_t *head, int shaped, int64_t head_rows, int hidden, int T,
                const float *normed, int n_logits, float *logits)
{
    if (n_logits <= 0 || T <= 0) return ORC_OK;
    if (hidden <= 0) return ORC_ERR_ARG;
    const int product = head && head_rows > 0 && (shaped || head_rows == n_logits);
    int8_t *xq = NULL;
    float *dx = NULL;
    if (product && type != ORC_F32) {
        xq = (int8_t *)malloc((size_t)hidden);
        dx = (float *)malloc((size_t)(hidden / 32 + 1) * sizeof(float));
        if (!xq || !dx) { free(xq); free(dx); return ORC_ERR_ARG; }
    }
    const size_t rb = product ? orc_row_bytes(type, hidden) : 0;
    if (product && !rb) { free(xq); free(dx); return ORC_ERR_ARG; }
    for (int t = 0; t < T; t++) {
        const float *x = normed + (size_t)t * hidden;
        float *out = logits + (size_t)t * n_logits;
        if (product) {
            const int target = n_logits < head_rows ? n_logits : (int)head_rows;
            if (type != ORC_F32 && orc_quantize_act(x, hidden, xq, dx) != ORC_OK) { free(xq); free(dx); return ORC_ERR_ARG; }
            for (int r = 0; r < target; r++) {
                const uint8_t *row = head + (size_t)r * rb;
                out[r] = type == ORC_F32 ? row_dot_f32((const float *)row, x, hidden)
                                         : orc_row_dot_q(type, row, xq, dx, hidden);
            }
            for (int i = target; i < n_logits; i++) out[i] = x[i % hidden] * 0.05f;
        } else {
            float sum = 0.0f;
            for (int i = 0; i < hidden; i++) sum += x[i];
            const float base = tanhf(sum / 16.0f);
            for (int i = 0; i < n_logits; i++) out[i] = base + x[i % hidden] * 0.1f + (float)(i % 13) * 0.01f;
        }
    }
    free(xq);
    free(dx);
    return ORC_OK;
}

/* Canonical dispatch order of the batched path: slots grouped by expert
 * ascending, tokens ascending inside each expert (a stable counting sort). */
int orc_permutation(const int32_t *sel_idx, int T, int k, int E, int32_t *offsets, int32_t *perm_token)
{
    for (int e = 0; e <= E; e++) offsets[e] = 0;
    for (size_t i = 0; i < (size_t)T * k; i++) {
        int e = sel_idx[i];
        if (e < 0 || e >= E) return ORC_ERR_ARG;
        offsets[e + 1]++;
    }
    for (int e = 0; e < E; e++) offsets[e + 1] += offsets[e];
    int32_t *fill = (int32_t *)malloc(sizeof(int32_t) * (E > 0 ? E : 1));
    if (!fill) return ORC_ERR_NOMEM;
    for (int e = 0; e < E; e++) fill[e] = offsets[e];
    for (int t = 0; t < T; t++)
        for (int r = 0; r < k; r++) perm_token[fill[sel_idx[(size_t)t * k + r]]++] = t;
    free(fill);
    return ORC_OK;
}

/* ------------------------------------------------------ synthetic inputs */

/* Seeded inputs of the benchmark configurations, restated independently of
 * the library's moe_gen_normal / moe_quantize_rows so that the reference arm
 * of the benchmark can build the same layers without loading the product
 * library (tests check the two byte for byte). */

static inline uint64_t orc_mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;   /* splitmix64 finaliser (Vigna) */
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

typedef struct {
    uint64_t key, lo, hi, n;
    float sigma;
    float *dst;
} gen_job;

static void *gen_run(void *arg)
{
    const gen_job *j = (const gen_job *)arg;
    const uint64_t G = 0x9E3779B97F4A7C15ull;
    for (uint64_t m = j->lo; m < j->hi; m++) {
        /* pair m: two uniforms from the counter stream, Box-Muller */
        uint64_t r1 = orc_mix64(j->key + (2 * m + 1) * G);
        uint64_t r2 = orc_mix64(j->key + (2 * m + 2) * G);
        double u1 = (double)((r1 >> 11) + 1) * 0x1.0p-53;
        double u2 = (double)(r2 >> 11) * 0x1.0p-53;
        double rad = sqrt(-2.0 * log(u1));
        double th = 6.283185307179586 * u2;
        j->dst[2 * m] = (float)(rad * cos(th) * (double)j->sigma);
        if (2 * m + 1 < j->n) j->dst[2 * m + 1] = (float)(rad * sin(th) * (double)j->sigma);
    }
    return NULL;
}

/* Element i of (seed, stream): normal pair i/2 of the counter stream keyed by
 * mix(seed ^ mix(stream + G)), G the splitmix64 increment. */
int orc_gen_normal(uint64_t seed, uint64_t stream, uint64_t n, float sigma, float *dst, int n_threads)
{
    const uint64_t G = 0x9E3779B97F4A7C15ull;
    uint64_t key = orc_mix64(seed ^ orc_mix64(stream + G));
    uint64_t pairs = (n + 1) / 2;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 64) n_threads = 64;
    if ((uint64_t)n_threads > pairs) n_threads = pairs ? (int)pairs : 1;
    pthread_t th[64];
    gen_job jobs[64];
    int ok[64] = {0};
    uint64_t chunk = (pairs + n_threads - 1) / n_threads;
    for (int t = 0; t < n_threads; t++) {
        jobs[t].key = key;
        jobs[t].lo = t * chunk < pairs ? t * chunk : pairs;
        jobs[t].hi = (t + 1) * chunk < pairs ? (t + 1) * chunk : pairs;
        jobs[t].n = n;
        jobs[t].sigma = sigma;
        jobs[t].dst = dst;
    }
    for (int t = 1; t < n_threads; t++) ok[t] = pthread_create(&th[t], NULL, gen_run, &jobs[t]) == 0;
    gen_run(&jobs[0]);
    for (int t = 1; t < n_threads; t++) {
        if (ok[t]) pthread_join(th[t], NULL);
        else gen_run(&jobs[t]);
    }
    return ORC_OK;
}

static inline uint16_t f32_to_f16_rne(float f)
{
    _Float16 h = (_Float16)f;   /* round to nearest even */
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

static inline float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Q8_0 block: d = f16(amax / 127); q = round(x / d) with the f16 d, clamped to
 * +-127 (GGUF layout: f16 d, 32 x int8). */
static void q8_0_row(const float *x, int cols, uint8_t *dst)
{
    for (int b = 0; b < cols / 32; b++) {
        const float *v = x + 32 * b;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(v[i]));
        uint16_t dh = f32_to_f16_rne(amax / 127.0f);
        float d = orc_f16_to_f32(dh);
        float id = d > 0.0f ? 1.0f / d : 0.0f;
        uint8_t *o = dst + 34 * b;
        o[0] = (uint8_t)(dh & 0xFF);
        o[1] = (uint8_t)(dh >> 8);
        for (int i = 0; i < 32; i++) o[2 + i] = (uint8_t)(int8_t)clampf(roundf(v[i] * id), -127.0f, 127.0f);
    }
}

/* Q4_K super-block of 256 values: per 32-value sub-block j, scale_j = (max -
 * min) / 15 and min_j = -min (min taken with 0); d = max scale_j / 63 and
 * dmin = max min_j / 63 as f16; sc_j = round(scale_j / d), m_j = round(min_j /
 * dmin) in 0..63; q = round((x + dmin m_j) / (d sc_j)) in 0..15. GGUF layout:
 * f16 d, f16 dmin, 12 bytes of 6-bit sc / m, 128 bytes of nibbles (value 64g+l
 * low nibble of byte 32g+l, value 64g+32+l its high nibble). */
static void q4_k_row(const float *x, int cols, uint8_t *dst)
{
    for (int sb = 0; sb < cols / 256; sb++) {
        const float *v = x + 256 * sb;
        float scale[8], mn[8];
        for (int j = 0; j < 8; j++) {
            float lo = 0.0f, hi = -INFINITY;
            for (int i = 0; i < 32; i++) {
                lo = fminf(lo, v[32 * j + i]);
                hi = fmaxf(hi, v[32 * j + i]);
            }
            scale[j] = (hi - lo) / 15.0f;
            mn[j] = -lo;
        }
        float ms = 0.0f, mm = 0.0f;
        for (int j = 0; j < 8; j++) {
            ms = fmaxf(ms, scale[j]);
            mm = fmaxf(mm, mn[j]);
        }
        uint16_t dh = f32_to_f16_rne(ms / 63.0f), mh = f32_to_f16_rne(mm / 63.0f);
        float d = orc_f16_to_f32(dh), dmin = orc_f16_to_f32(mh);
        int sc[8], m[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = d > 0.0f ? (int)clampf(roundf(scale[j] / d), 0.0f, 63.0f) : 0;
            m[j] = dmin > 0.0f ? (int)clampf(roundf(mn[j] / dmin), 0.0f, 63.0f) : 0;
        }
        uint8_t *o = dst + 144 * sb;
        o[0] = (uint8_t)(dh & 0xFF);
        o[1] = (uint8_t)(dh >> 8);
        o[2] = (uint8_t)(mh & 0xFF);
        o[3] = (uint8_t)(mh >> 8);
        uint8_t *k = o + 4;
        for (int j = 0; j < 4; j++) {   /* the inverse of q4k_scale_min */
            k[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            k[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
            k[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
        }
        uint8_t q[256];
        for (int j = 0; j < 8; j++) {
            float ds = d * (float)sc[j], dm = dmin * (float)m[j];
            for (int i = 0; i < 32; i++)
                q[32 * j + i] = (uint8_t)clampf(ds > 0.0f ? roundf((v[32 * j + i] + dm) / ds) : 0.0f, 0.0f, 15.0f);
        }
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++) o[16 + 32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
    }
}

typedef struct {
    int type, cols;
    const float *src;
    uint8_t *dst;
    int64_t lo, hi;
} quant_job;

static void *quant_run(void *arg)
{
    const quant_job *j = (const quant_job *)arg;
    size_t rb = orc_row_bytes(j->type, j->cols);
    for (int64_t r = j->lo; r < j->hi; r++) {
        const float *x = j->src + (size_t)r * j->cols;
        uint8_t *o = j->dst + (size_t)r * rb;
        if (j->type == ORC_F32) memcpy(o, x, rb);
        else if (j->type == ORC_Q8_0) q8_0_row(x, j->cols, o);
        else q4_k_row(x, j->cols, o);
    }
    return NULL;
}

/* rows x cols f32 -> GGUF rows of type (F32, Q8_0 or Q4_K). */
int orc_quantize_rows(int type, const float *src, int64_t rows, int cols, uint8_t *dst, int n_threads)
{
    if (!orc_row_bytes(type, cols) || (type != ORC_F32 && type != ORC_Q8_0 && type != ORC_Q4_K) || rows < 0)
        return ORC_ERR_ARG;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 64) n_threads = 64;
    if (rows < n_threads) n_threads = rows > 0 ? (int)rows : 1;
    pthread_t th[64];
    quant_job jobs[64];
    int64_t chunk = (rows + n_threads - 1) / n_threads;
    int ok[64] = {0};
    for (int t = 0; t < n_threads; t++) {
        jobs[t] = (quant_job){type, cols, src, dst, t * chunk < rows ? t * chunk : rows,
                              (t + 1) * chunk < rows ? (t + 1) * chunk : rows};
    }
    for (int t = 1; t < n_threads; t++) ok[t] = pthread_create(&th[t], NULL, quant_run, &jobs[t]) == 0;
    quant_run(&jobs[0]);
    for (int t = 1; t < n_threads; t++) {
        if (ok[t]) pthread_join(th[t], NULL);
        else quant_run(&jobs[t]);
    }
    return ORC_OK;
}

