/*
 * moe_oracle.c -- CPU restatement of the motorIa MoE FFN block.
 *
 * TEST INFRASTRUCTURE ONLY (see moe_oracle.h).  Compile with
 *   gcc -std=c99 -O2 -fPIC -shared   (ISO mode: -ffp-contract=off, so every
 *   float multiply and add rounds on its own, exactly like the reference's
 *   scalar build on x86).
 * Every function names the reference file:line whose arithmetic it restates;
 * the operation order inside each is the reference's, because the GPU
 * kernels are checked against it bit for bit where the reference is
 * deterministic (quantizer, Q8_0 dots, router logits, top-k, permutation).
 */
#define _POSIX_C_SOURCE 200809L
#include "moe_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static size_t round_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

/* src/storage/mia_file.c:275-278 and tools/internal/mia/format.go:160-163:
 * gate at 0, up at align64(mat), down after another align64(mat). */
size_t orc_off_up(const orc_shape *s) {
    size_t mat = (size_t)s->expert_hidden * (size_t)(s->dim / ORC_QK) *
                 sizeof(orc_block_q8);
    return round_up(mat, 64);
}

size_t orc_off_down(const orc_shape *s) { return 2 * orc_off_up(s); }

size_t orc_blob_bytes(const orc_shape *s) {
    size_t down = (size_t)s->dim * (size_t)(s->expert_hidden / ORC_QK) *
                  sizeof(orc_block_q8);
    return round_up(orc_off_down(s) + down, 16384); /* format.go ExpertAlign */
}

/* src/tensor/quant.c:11-27: d = amax/127, id = 1/d (0 for an all-zero
 * block), q = (int8)roundf(x*id) -- roundf rounds halves away from zero. */
void orc_quantize_row_q8(const float *x, orc_block_q8 *y, int n) {
    for (int b = 0; b < n / ORC_QK; b++) {
        const float *xb = x + (size_t)b * ORC_QK;
        float amax = 0.0f;
        for (int i = 0; i < ORC_QK; i++) {
            float a = fabsf(xb[i]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[b].d = d;
        for (int i = 0; i < ORC_QK; i++) y[b].q[i] = (int8_t)roundf(xb[i] * id);
    }
}

/* src/tensor/quant.c:29-38 (Q8_0 branch). */
void orc_dequantize_row_q8(const orc_block_q8 *y, float *x, int n) {
    for (int b = 0; b < n / ORC_QK; b++)
        for (int i = 0; i < ORC_QK; i++)
            x[(size_t)b * ORC_QK + i] = y[b].d * (float)y[b].q[i];
}

/* src/tensor/matmul.c:19-28: exact int32 block dot, then
 * s += ((float)acc * w.d) * x.d, blocks in order. */
float orc_dot_q8(const orc_block_q8 *w, const orc_block_q8 *x, int nb) {
    float s = 0.0f;
    for (int b = 0; b < nb; b++) {
        int32_t acc = 0;
        for (int i = 0; i < ORC_QK; i++) acc += (int32_t)w[b].q[i] * x[b].q[i];
        s += (float)acc * w[b].d * x[b].d;
    }
    return s;
}

/* src/tensor/matmul.c:13-17: sequential fp32 sum of rounded products. */
float orc_dot_f32(const float *a, const float *b, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

/* src/tensor/matmul.c:83-87 with rows_kernel :75-80 (Q8_0). */
void orc_matvec_q8(float *out, const void *w, const float *x, orc_block_q8 *xq,
                   int rows, int cols) {
    const int nb = cols / ORC_QK;
    const orc_block_q8 *wq = (const orc_block_q8 *)w;
    orc_quantize_row_q8(x, xq, cols);
    for (int r = 0; r < rows; r++) out[r] = orc_dot_q8(wq + (size_t)r * nb, xq, nb);
}

/* src/tensor/matmul.c:69-74 (F32 rows). */
void orc_matvec_f32(float *out, const float *w, const float *x, int rows,
                    int cols) {
    for (int r = 0; r < rows; r++) out[r] = orc_dot_f32(w + (size_t)r * cols, x, cols);
}

/* src/model/forward.c:75-81: double accumulator, float scale. */
void orc_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    double ss = 0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * x[i];
    float inv = (float)(1.0 / sqrt(ss / n + eps));
    for (int i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

/* src/model/forward.c:95-101. */
void orc_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) mx = x[i] > mx ? x[i] : mx;
    float sum = 0;
    for (int i = 0; i < n; i++) sum += x[i] = expf(x[i] - mx);
    for (int i = 0; i < n; i++) x[i] /= sum;
}

/* src/model/forward.c:104-114: k rounds of first-maximum selection among
 * the not-yet-taken entries (strict '>', so ties go to the lower index). */
void orc_top_k(const float *p, int n, int k, int *idx) {
    for (int j = 0; j < k; j++) {
        int best = -1;
        for (int i = 0; i < n; i++) {
            int taken = 0;
            for (int t = 0; t < j; t++) taken |= idx[t] == i;
            if (!taken && (best < 0 || p[i] > p[best])) best = i;
        }
        idx[j] = best;
    }
}

/* src/model/forward.c:174-181, plus an optional per-expert logit bias added
 * between the router matvec and the softmax (the skewed-load benchmark
 * configurations; the reference has no bias, bias == NULL reproduces it). */
static void route_one(const orc_shape *s, const float *ffn_norm,
                      const float *router, const float *bias, const float *x,
                      float *xn, float *logits, int32_t *idx, float *w) {
    int k_idx[64];
    const int E = s->n_experts, K = s->n_active;
    orc_rmsnorm(xn, x, ffn_norm, s->dim, s->norm_eps);
    orc_matvec_f32(logits, router, xn, E, s->dim);
    if (bias)
        for (int e = 0; e < E; e++) logits[e] += bias[e];
    orc_softmax(logits, E);
    orc_top_k(logits, E, K, k_idx);
    float sum = 0;
    for (int j = 0; j < K; j++) sum += w[j] = logits[k_idx[j]];
    if (s->norm_topk)
        for (int j = 0; j < K; j++) w[j] /= sum;
    for (int j = 0; j < K; j++) idx[j] = k_idx[j];
}

void orc_route(const orc_shape *s, const float *ffn_norm, const float *router,
               const float *bias, const float *x, float *xn, int32_t *idx,
               float *w) {
    float *logits = (float *)malloc(sizeof(float) * (size_t)s->n_experts);
    route_one(s, ffn_norm, router, bias, x, xn, logits, idx, w);
    free(logits);
}

/* src/model/forward.c:183-195 for one token, after routing. */
static void experts_one(const orc_shape *s, const uint8_t *blobs,
                        size_t blob_stride, const int32_t *idx, const float *w,
                        const float *xn, float *x, float *gate, float *up,
                        float *tmp, orc_block_q8 *xq) {
    const int d = s->dim, eh = s->expert_hidden;
    const size_t off_up = orc_off_up(s), off_down = orc_off_down(s);
    for (int j = 0; j < s->n_active; j++) {
        const uint8_t *blob = blobs + (size_t)idx[j] * blob_stride;
        orc_matvec_q8(gate, blob, xn, xq, eh, d);
        orc_matvec_q8(up, blob + off_up, xn, xq, eh, d);
        for (int i = 0; i < eh; i++) {
            float g = gate[i];
            gate[i] = g / (1.0f + expf(-g)) * up[i];
        }
        orc_matvec_q8(tmp, blob + off_down, gate, xq, d, eh);
        for (int i = 0; i < d; i++) x[i] += w[j] * tmp[i];
    }
}

typedef struct {
    const orc_shape *s;
    const float *ffn_norm, *router, *bias;
    const uint8_t *blobs;
    size_t blob_stride;
    float *x_rw;       /* moe: updated in place */
    const float *x_ro; /* route only */
    int32_t *idx;
    float *w;
    int t0, t1, route_only;
} job;

static void *run_job(void *arg) {
    job *J = (job *)arg;
    const orc_shape *s = J->s;
    const int d = s->dim, eh = s->expert_hidden, E = s->n_experts, K = s->n_active;
    int maxc = d > eh ? d : eh;
    float *xn = (float *)malloc(sizeof(float) * (size_t)d);
    float *logits = (float *)malloc(sizeof(float) * (size_t)E);
    float *gate = (float *)malloc(sizeof(float) * (size_t)eh);
    float *up = (float *)malloc(sizeof(float) * (size_t)eh);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)d);
    orc_block_q8 *xq = (orc_block_q8 *)malloc(sizeof(orc_block_q8) * (size_t)(maxc / ORC_QK));
    int32_t lidx[64];
    float lw[64];
    for (int t = J->t0; t < J->t1; t++) {
        const float *xt = J->route_only ? J->x_ro + (size_t)t * d : J->x_rw + (size_t)t * d;
        route_one(s, J->ffn_norm, J->router, J->bias, xt, xn, logits, lidx, lw);
        if (J->idx) memcpy(J->idx + (size_t)t * K, lidx, sizeof(int32_t) * (size_t)K);
        if (J->w) memcpy(J->w + (size_t)t * K, lw, sizeof(float) * (size_t)K);
        if (!J->route_only)
            experts_one(s, J->blobs, J->blob_stride, lidx, lw, xn,
                        J->x_rw + (size_t)t * d, gate, up, tmp, xq);
    }
    free(xn), free(logits), free(gate), free(up), free(tmp), free(xq);
    return NULL;
}

static int run_threads(job *proto, int T, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > T) n_threads = T > 0 ? T : 1;
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)n_threads);
    job *jobs = (job *)malloc(sizeof(job) * (size_t)n_threads);
    for (int i = 0; i < n_threads; i++) {
        jobs[i] = *proto;
        jobs[i].t0 = (int)((long)T * i / n_threads);
        jobs[i].t1 = (int)((long)T * (i + 1) / n_threads);
    }
    for (int i = 1; i < n_threads; i++) pthread_create(&th[i], NULL, run_job, &jobs[i]);
    run_job(&jobs[0]);
    for (int i = 1; i < n_threads; i++) pthread_join(th[i], NULL);
    free(th), free(jobs);
    return 0;
}

int orc_route_batch(const orc_shape *s, const float *ffn_norm,
                    const float *router, const float *bias, const float *x,
                    int T, int32_t *idx, float *w, int n_threads) {
    if (s->n_active > 64 || s->n_active > s->n_experts) return -1;
    job J;
    memset(&J, 0, sizeof J);
    J.s = s, J.ffn_norm = ffn_norm, J.router = router, J.bias = bias;
    J.x_ro = x, J.idx = idx, J.w = w, J.route_only = 1;
    return run_threads(&J, T, n_threads);
}

int orc_moe(const orc_shape *s, const float *ffn_norm, const float *router,
            const float *bias, const uint8_t *blobs, size_t blob_stride,
            float *x, int T, int32_t *idx, float *w, int n_threads) {
    if (s->n_active > 64 || s->n_active > s->n_experts) return -1; /* forward.c:172 */
    job J;
    memset(&J, 0, sizeof J);
    J.s = s, J.ffn_norm = ffn_norm, J.router = router, J.bias = bias;
    J.blobs = blobs, J.blob_stride = blob_stride, J.x_rw = x;
    J.idx = idx, J.w = w;
    return run_threads(&J, T, n_threads);
}

/* Canonical dispatch order (no reference counterpart: the reference runs one
 * token at a time).  A counting sort over experts visiting pairs in (t, j)
 * order is stable, which is exactly "by expert, then t, then j". */
void orc_permute(const int32_t *idx, int T, int K, int E, int32_t *counts,
                 int32_t *offsets, int32_t *perm, int32_t *inv) {
    const int P = T * K;
    for (int e = 0; e < E; e++) counts[e] = 0;
    for (int p = 0; p < P; p++) counts[idx[p]]++;
    offsets[0] = 0;
    for (int e = 0; e < E; e++) offsets[e + 1] = offsets[e] + counts[e];
    int32_t *next = (int32_t *)malloc(sizeof(int32_t) * (size_t)(E > 0 ? E : 1));
    for (int e = 0; e < E; e++) next[e] = offsets[e];
    for (int p = 0; p < P; p++) {
        int pos = next[idx[p]]++;
        perm[pos] = p;
        if (inv) inv[p] = pos;
    }
    free(next);
}
