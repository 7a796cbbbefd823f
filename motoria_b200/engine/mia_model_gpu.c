/*
 * mia_model_gpu.c -- the motorIa engine's model layer on the GPU.
 *
 * Implements include/mia/model.h (mia_model_init / mia_model_free /
 * mia_model_step / mia_model_state_bytes), which src/model/forward.c
 * implements on the CPU, over libmiag's whole-model decode (miag_model_*,
 * include/miag/miag.h).  Linked in place of forward.c it leaves the rest of
 * the engine as it is: the applications mia, mia-serve and mia-dump
 * (src/app/main.c, serve.c, dump.c), the runtime and RAM planner
 * (src/model/runtime.c), the .mia reader (src/storage/mia_file.c), the
 * tokenizer and the sampler.  The build recipe is this directory's Makefile.
 *
 *   mia_model_init   opens a miag context for the file's MoE shape on
 *                    $MIAG_DEVICE (default 0), fills its HBM expert store
 *                    through the reference loader port (mia_file_read_expert,
 *                    include/mia/mia_file.h:44), and uploads the file's dense
 *                    section (mia_file.dense) into a miag_model with the KV
 *                    cache of max_seq positions in HBM;
 *   mia_model_step   one CUDA graph replay (miag_model_step); the logits,
 *                    equal to forward.c's bit for bit up to glibc's expf, in
 *                    host memory owned by the model (valid until the next
 *                    step), NULL for a token or position out of range
 *                    (forward.c:202-203) or a device error (on stderr);
 *   cache counters   every expert stays resident, so each step's
 *                    n_layers * n_active lookups count as hits and the
 *                    engine reports a 100% hit rate with no bytes read.
 *
 * C99; one mia_model per host thread, as the reference's.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "mia/model.h"
#include "miag/miag.h"

/* mia_model has no field for the GPU state; the engine holds one model per
 * sequence, so a short list keyed by the mia_model's address suffices. */
typedef struct gpu_model {
    const mia_model *owner;
    miag_ctx *ctx;
    miag_model *g;
    struct gpu_model *next;
} gpu_model;

static gpu_model *g_models;

static gpu_model *find_model(const mia_model *m) {
    for (gpu_model *p = g_models; p; p = p->next)
        if (p->owner == m) return p;
    return NULL;
}

/* The GPU model behind an engine model (NULL if none): for the loops that
 * call libmiag directly, e.g. a prompt through miag_model_prefill. */
miag_model *mia_model_gpu(const mia_model *m) {
    gpu_model *p = find_model(m);
    return p ? p->g : NULL;
}

size_t mia_model_state_bytes(const mia_file *f, int max_seq) {
    (void)max_seq; /* activations and the KV cache live in HBM */
    return (size_t)f->h.vocab * sizeof(float); /* the host copy of the logits */
}

int mia_model_init(mia_model *m, const mia_file *f, mia_expert_cache *cache, int max_seq) {
    memset(m, 0, sizeof(*m));
    m->f = f, m->cache = cache, m->max_seq = max_seq;
    if (f->wt != MIA_Q8_0) {
        fprintf(stderr, "mia_model_gpu: only Q8_0 models run on the GPU\n");
        return -1;
    }
    const mia_header *h = &f->h;
    const miag_shape shape = {(int32_t)h->dim,           (int32_t)h->n_layers,  (int32_t)h->n_experts,
                              (int32_t)h->n_active,      (int32_t)h->expert_hidden,
                              (int32_t)h->norm_topk,     h->norm_eps};
    const miag_mia_config cfg = {h->dim,       h->n_layers,  h->n_heads,       h->n_kv_heads,
                                 h->head_dim,  h->vocab,     h->n_experts,     h->n_active,
                                 h->expert_hidden, h->norm_topk, h->rope_theta, h->norm_eps};
    const char *dev = getenv("MIAG_DEVICE");
    char err[512] = "";
    gpu_model *p = calloc(1, sizeof(*p));
    if (!p) return -1;
    if (miag_open(&p->ctx, &shape, dev ? atoi(dev) : 0, err, sizeof(err)) != 0 ||
        miag_load_experts(p->ctx, mia_file_read_expert, (void *)f, err, sizeof(err)) != 0 ||
        miag_model_open(&p->g, p->ctx, &cfg, f->dense, (size_t)h->dense_size, max_seq, err,
                        sizeof(err)) != 0) {
        fprintf(stderr, "mia_model_gpu: %s\n", err);
        if (p->ctx) miag_close(p->ctx);
        free(p);
        return -1;
    }
    p->owner = m;
    p->next = g_models;
    g_models = p;
    return 0;
}

void mia_model_free(mia_model *m) {
    gpu_model **pp = &g_models;
    while (*pp && (*pp)->owner != m) pp = &(*pp)->next;
    if (*pp) {
        gpu_model *p = *pp;
        *pp = p->next;
        miag_model_close(p->g);
        miag_close(p->ctx);
        free(p);
    }
    memset(m, 0, sizeof(*m));
}

const float *mia_model_step(mia_model *m, int token, int pos) {
    gpu_model *p = find_model(m);
    if (!p || pos < 0 || pos >= m->max_seq || token < 0 || token >= (int)m->f->h.vocab) return NULL;
    char err[512] = "";
    const float *logits = miag_model_step(p->g, token, pos, err, sizeof(err));
    if (!logits) {
        fprintf(stderr, "mia_model_gpu: %s\n", err);
        return NULL;
    }
    if (m->cache) m->cache->hits += (uint64_t)m->f->h.n_layers * m->f->h.n_active;
    m->logits = (float *)logits;
    return logits;
}
