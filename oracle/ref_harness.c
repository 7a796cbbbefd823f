/*
 * ref_harness.c -- drives the reference engine's own MoE code, compiled from
 * the reference's sources, so the oracle restatement (moe_oracle.c) and the
 * golden vectors are pinned to the real thing.
 *
 * TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into
 * oracle/_ref/libmia_ref.so from the reference tree (REF=<path>); nothing is
 * copied into this repository.  The reference's src/model/forward.c is
 * #included so its file-static moe(), rmsnorm(), softmax() and top_k() are
 * callable; src/tensor/{matmul,quant}.c, src/storage/expert_cache.c and
 * src/storage/mia_file.c are compiled unchanged beside it.
 *
 * Expert residency: every thread gets its own mia_model and its own
 * mia_expert_cache whose slab is the caller's read-only blob array with every
 * (layer, expert) key already resident, so mia_cache_get (expert_cache.c:59-85)
 * always takes its hit path and nothing is copied.  The LRU links the hit
 * path rewrites are per thread.
 */
#include "src/model/forward.c"

#include <pthread.h>
#include <stdio.h>

typedef struct {
    int32_t dim, n_experts, n_active, expert_hidden, norm_topk;
    float norm_eps;
} ref_shape;

static void fill_file(mia_file *f, mia_layer *layer, const ref_shape *s,
                      const float *ffn_norm, const float *router) {
    memset(f, 0, sizeof(*f));
    memset(layer, 0, sizeof(*layer));
    memcpy(f->h.magic, "MIA1", 4);
    f->h.version = 1;
    f->h.wtype = MIA_Q8_0;
    f->h.dim = (uint32_t)s->dim;
    f->h.n_layers = 1;
    /* Attention sizes are unused by moe(); keep them small and non-zero so
     * mia_model_init allocates nothing of size 0. */
    f->h.n_heads = 1, f->h.n_kv_heads = 1, f->h.head_dim = 32, f->h.vocab = 1;
    f->h.n_experts = (uint32_t)s->n_experts;
    f->h.n_active = (uint32_t)s->n_active;
    f->h.expert_hidden = (uint32_t)s->expert_hidden;
    f->h.norm_topk = (uint32_t)s->norm_topk;
    f->h.norm_eps = s->norm_eps;
    f->h.rope_theta = 1e6f;
    f->wt = MIA_Q8_0;
    f->fd = -1;
    layer->ffn_norm = ffn_norm;
    layer->router = router;
    f->layers = layer;
    /* mia_file.c:275-278 */
    size_t mat = (size_t)s->expert_hidden * mia_row_bytes(MIA_Q8_0, s->dim);
    f->off_up = (mat + 63) / 64 * 64;
    f->off_down = 2 * f->off_up;
}

static int never_load(void *ctx, int layer, int expert, void *dst) {
    (void)ctx, (void)layer, (void)expert, (void)dst;
    return -1;
}

/* A cache whose every key is resident in the caller's blob array. */
static int resident_cache(mia_expert_cache *c, int n_experts, size_t stride,
                          const unsigned char *blobs) {
    memset(c, 0, sizeof(*c));
    c->n_layers = 1, c->n_experts = n_experts, c->n_slots = n_experts;
    c->blob_size = stride;
    c->slab = (unsigned char *)blobs; /* read only: the hit path never writes */
    c->slot_of = malloc(sizeof(int) * (size_t)n_experts);
    c->key_of = malloc(sizeof(int) * (size_t)n_experts);
    c->prev = malloc(sizeof(int) * (size_t)n_experts);
    c->next = malloc(sizeof(int) * (size_t)n_experts);
    if (!c->slot_of || !c->key_of || !c->prev || !c->next) return -1;
    for (int k = 0; k < n_experts; k++) {
        c->slot_of[k] = k, c->key_of[k] = k;
        c->prev[k] = k - 1;
        c->next[k] = k + 1 < n_experts ? k + 1 : -1;
    }
    c->head = 0, c->tail = n_experts - 1;
    c->load = never_load;
    return 0;
}

static void free_cache(mia_expert_cache *c) {
    free(c->slot_of), free(c->key_of), free(c->prev), free(c->next);
    memset(c, 0, sizeof(*c));
}

/* Routing exactly as moe() does it (forward.c:174-181), with the optional
 * logit bias added between the router matvec and softmax. */
static void route_ref(mia_model *m, dims s, const float *bias, int32_t *idx,
                      float *w) {
    const mia_file *f = m->f;
    const mia_layer *L = &f->layers[0];
    int k_idx[64];
    rmsnorm(m->xn, m->x, L->ffn_norm, s.d, f->h.norm_eps);
    mia_matvec(m->router, L->router, MIA_F32, m->xn, NULL, s.E, s.d);
    if (bias)
        for (int e = 0; e < s.E; e++) m->router[e] += bias[e];
    softmax(m->router, s.E);
    top_k(m->router, s.E, s.K, k_idx);
    float sum = 0;
    for (int j = 0; j < s.K; j++) sum += w[j] = m->router[k_idx[j]];
    if (f->h.norm_topk)
        for (int j = 0; j < s.K; j++) w[j] /= sum;
    for (int j = 0; j < s.K; j++) idx[j] = k_idx[j];
}

/* The expert loop of moe() (forward.c:183-195) on routing already made. */
static int experts_ref(mia_model *m, dims s, const int32_t *idx, const float *w) {
    const mia_file *f = m->f;
    for (int j = 0; j < s.K; j++) {
        const unsigned char *blob = mia_cache_get(m->cache, 0, idx[j]);
        if (!blob) return -1;
        mia_matvec(m->gate, blob, f->wt, m->xn, m->xq, s.eh, s.d);
        mia_matvec(m->up, blob + f->off_up, f->wt, m->xn, m->xq, s.eh, s.d);
        for (int i = 0; i < s.eh; i++) {
            float g = m->gate[i];
            m->gate[i] = g / (1.0f + expf(-g)) * m->up[i];
        }
        mia_matvec(m->tmp, blob + f->off_down, f->wt, m->gate, m->xq, s.d, s.eh);
        for (int i = 0; i < s.d; i++) m->x[i] += w[j] * m->tmp[i];
    }
    return 0;
}

typedef struct {
    const ref_shape *s;
    const float *ffn_norm, *router, *bias;
    const unsigned char *blobs;
    size_t stride;
    float *x;
    int32_t *idx;
    float *w;
    int t0, t1, route_only, rc;
} ref_job;

static void *ref_run(void *arg) {
    ref_job *J = (ref_job *)arg;
    mia_file f;
    mia_layer layer;
    mia_expert_cache cache;
    mia_model m;
    fill_file(&f, &layer, J->s, J->ffn_norm, J->router);
    J->rc = -1;
    if (resident_cache(&cache, J->s->n_experts, J->stride, J->blobs) != 0) {
        free_cache(&cache);
        return NULL;
    }
    if (mia_model_init(&m, &f, &cache, 1) != 0) {
        free_cache(&cache);
        return NULL;
    }
    dims s = dims_of(&f.h);
    int32_t lidx[64];
    float lw[64];
    J->rc = 0;
    for (int t = J->t0; t < J->t1 && J->rc == 0; t++) {
        float *xt = J->x + (size_t)t * s.d;
        memcpy(m.x, xt, sizeof(float) * (size_t)s.d);
        if (J->idx || J->w || J->bias || J->route_only) {
            route_ref(&m, s, J->bias, lidx, lw);
            if (J->idx) memcpy(J->idx + (size_t)t * s.K, lidx, sizeof(int32_t) * (size_t)s.K);
            if (J->w) memcpy(J->w + (size_t)t * s.K, lw, sizeof(float) * (size_t)s.K);
        }
        if (J->route_only) continue;
        if (J->bias) {
            /* xn is already in m->xn from route_ref. */
            J->rc = experts_ref(&m, s, lidx, lw);
        } else {
            /* The unmodified static moe(): it recomputes the routing itself. */
            J->rc = moe(&m, s, 0);
        }
        memcpy(xt, m.x, sizeof(float) * (size_t)s.d);
    }
    mia_model_free(&m);
    free_cache(&cache);
    return NULL;
}

static int ref_dispatch(ref_job *proto, int T, int n_threads) {
    if (proto->s->n_active > 64) return -1;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > T) n_threads = T > 0 ? T : 1;
    pthread_t *th = malloc(sizeof(pthread_t) * (size_t)n_threads);
    ref_job *jobs = malloc(sizeof(ref_job) * (size_t)n_threads);
    for (int i = 0; i < n_threads; i++) {
        jobs[i] = *proto;
        jobs[i].t0 = (int)((long)T * i / n_threads);
        jobs[i].t1 = (int)((long)T * (i + 1) / n_threads);
    }
    for (int i = 1; i < n_threads; i++) pthread_create(&th[i], NULL, ref_run, &jobs[i]);
    ref_run(&jobs[0]);
    int rc = jobs[0].rc;
    for (int i = 1; i < n_threads; i++) {
        pthread_join(th[i], NULL);
        if (jobs[i].rc) rc = jobs[i].rc;
    }
    free(th), free(jobs);
    return rc;
}

/* MoE block over T tokens (x [T][dim] in/out).  idx/w (nullable) receive
 * the routing.  bias == NULL runs the reference's unmodified moe(). */
int ref_moe(const ref_shape *s, const float *ffn_norm, const float *router,
            const float *bias, const unsigned char *blobs, size_t stride,
            float *x, int T, int32_t *idx, float *w, int n_threads) {
    ref_job J;
    memset(&J, 0, sizeof J);
    J.s = s, J.ffn_norm = ffn_norm, J.router = router, J.bias = bias;
    J.blobs = blobs, J.stride = stride, J.x = x, J.idx = idx, J.w = w;
    return ref_dispatch(&J, T, n_threads);
}

/* Routing only (x is copied, not modified). */
int ref_route(const ref_shape *s, const float *ffn_norm, const float *router,
              const float *bias, const float *x, int T, int32_t *idx, float *w,
              int n_threads) {
    float *xc = malloc(sizeof(float) * (size_t)T * (size_t)s->dim);
    if (!xc) return -1;
    memcpy(xc, x, sizeof(float) * (size_t)T * (size_t)s->dim);
    ref_job J;
    memset(&J, 0, sizeof J);
    J.s = s, J.ffn_norm = ffn_norm, J.router = router, J.bias = bias;
    J.x = xc, J.idx = idx, J.w = w, J.route_only = 1;
    J.stride = 0, J.blobs = NULL;
    /* resident_cache needs a non-empty table even when nothing is fetched */
    int rc = ref_dispatch(&J, T, n_threads);
    free(xc);
    return rc;
}

/* Public reference entry points, re-exported under ref_ names. */
void ref_quantize_row_q8(const float *x, void *y, int n) {
    mia_quantize_row_q8(x, (mia_block_q8 *)y, n);
}
void ref_matvec(float *out, const void *w, int wtype, const float *x, void *xq,
                int rows, int cols) {
    mia_matvec(out, w, (mia_wtype)wtype, x, (mia_block_q8 *)xq, rows, cols);
}
void ref_matvec_scalar(float *out, const void *w, int wtype, const float *x,
                       void *xq, int rows, int cols) {
    mia_matvec_scalar(out, w, (mia_wtype)wtype, x, (mia_block_q8 *)xq, rows, cols);
}
void ref_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    rmsnorm(out, x, w, n, eps);
}
void ref_softmax(float *x, int n) { softmax(x, n); }
void ref_top_k(const float *p, int n, int k, int *idx) { top_k(p, n, k, idx); }
int ref_block_bytes(void) { return (int)sizeof(mia_block_q8); }

/* The reference's .mia reader (src/storage/mia_file.c:41-126) behind opaque
 * handles, for tests that check files written by libmiag's writer and load
 * them through the loader port.  ref_mia_read_expert has the loader port's
 * signature (it is mia_file_read_expert). */
void *ref_mia_open(const char *path, char *err, size_t errlen) {
    mia_file *f = calloc(1, sizeof(mia_file));
    if (!f) return NULL;
    if (mia_file_open(f, path, err, errlen) != 0) {
        free(f);
        return NULL;
    }
    return f;
}
void ref_mia_close(void *f) {
    if (!f) return;
    mia_file_close((mia_file *)f);
    free(f);
}
int ref_mia_read_expert(void *f, int layer, int expert, void *dst) {
    return mia_file_read_expert(f, layer, expert, dst);
}
/* header fields: dim, n_layers, n_heads, n_kv_heads, head_dim, vocab,
 * n_experts, n_active, expert_hidden, norm_topk */
void ref_mia_dims(void *fp, int32_t *out) {
    const mia_header *h = &((mia_file *)fp)->h;
    const uint32_t v[10] = {h->dim, h->n_layers, h->n_heads, h->n_kv_heads, h->head_dim,
                            h->vocab, h->n_experts, h->n_active, h->expert_hidden, h->norm_topk};
    for (int i = 0; i < 10; i++) out[i] = (int32_t)v[i];
}
float ref_mia_norm_eps(void *fp) { return ((mia_file *)fp)->h.norm_eps; }
uint64_t ref_mia_blob_bytes(void *fp) { return ((mia_file *)fp)->h.expert_blob_size; }
const float *ref_mia_ffn_norm(void *fp, int l) { return ((mia_file *)fp)->layers[l].ffn_norm; }
const float *ref_mia_router(void *fp, int l) { return ((mia_file *)fp)->layers[l].router; }
const void *ref_mia_tensor(void *fp, int l, int which) {
    const mia_file *f = (const mia_file *)fp;
    switch (which) {
    case 0: return f->token_embd;
    case 1: return f->output;
    case 2: return f->output_norm;
    case 3: return f->layers[l].wq;
    case 4: return f->layers[l].attn_norm;
    default: return NULL;
    }
}


/* The reference engine's whole model step (mia_model_step,
 * src/model/forward.c:199-217) over a .mia file, every expert resident in
 * its cache (src/storage/expert_cache.c), for the model-level parity tests. */
typedef struct {
    mia_file f;
    mia_expert_cache cache;
    mia_model m;
} ref_model;

void *ref_model_open(const char *path, int max_seq, char *err, size_t errlen) {
    ref_model *r = calloc(1, sizeof(ref_model));
    if (!r) return NULL;
    if (mia_file_open(&r->f, path, err, errlen) != 0) {
        free(r);
        return NULL;
    }
    const int slots = (int)(r->f.h.n_layers * r->f.h.n_experts);
    if (mia_cache_init(&r->cache, (int)r->f.h.n_layers, (int)r->f.h.n_experts,
                       r->f.h.expert_blob_size, slots, mia_file_read_expert, &r->f) != 0 ||
        mia_model_init(&r->m, &r->f, &r->cache, max_seq) != 0) {
        snprintf(err, errlen, "reference model: out of memory");
        mia_file_close(&r->f);
        free(r);
        return NULL;
    }
    return r;
}
const float *ref_model_step(void *h, int token, int pos) {
    return mia_model_step(&((ref_model *)h)->m, token, pos);
}
void ref_model_close(void *h) {
    ref_model *r = (ref_model *)h;
    if (!r) return;
    mia_model_free(&r->m);
    mia_cache_free(&r->cache);
    mia_file_close(&r->f);
    free(r);
}
