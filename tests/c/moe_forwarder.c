/*
 * moe_forwarder.c -- a C99 consumer of libmiag, as the motorIa engine would
 * be one: it includes only include/miag/miag.h, fills the HBM store through
 * the reference's loader port (the signature of mia_file_read_expert,
 * include/mia/mia_file.h:44), and runs the block through the moe() forwarder
 * given in INTEGRATION.md, once per token, the way mia_model_step calls moe()
 * (src/model/forward.c:212).  The result is compared with the reference's own
 * moe() (src/model/forward.c:167-197, compiled from its sources into
 * oracle/_ref/libmia_ref.so by oracle/Makefile; test infrastructure only).
 *
 * Inputs are generated here (splitmix64 + Box-Muller), in the .mia expert
 * blob layout: gate | up | down, rows of 36-byte {f32 d; int8 q[32]} Q8_0
 * blocks (src/storage/mia_file.c:275-278).  Exit 0 when every token's MoE
 * update is within 1e-3 relative L2 of the reference's (most are bit-exact;
 * the rest differ through glibc's expf).
 *
 *   usage: moe_forwarder [n_tokens]
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "miag/miag.h"

/* the reference harness (oracle/ref_harness.c) */
typedef struct {
    int32_t dim, n_experts, n_active, expert_hidden, norm_topk;
    float norm_eps;
} ref_shape;
int ref_moe(const ref_shape *s, const float *ffn_norm, const float *router, const float *bias,
            const unsigned char *blobs, size_t stride, float *x, int T, int32_t *idx, float *w,
            int n_threads);

static uint64_t rng_state;
static uint64_t splitmix(void) {
    uint64_t z = (rng_state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static double uniform01(void) { return ((splitmix() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
static float gauss(float sd) {
    const double u = uniform01(), v = uniform01();
    return (float)(sd * sqrt(-2.0 * log(u)) * cos(6.283185307179586 * v));
}

/* One Q8_0 matrix of rows x cols at dst: int8 uniform in [-127, 127], each
 * block's scale |N(0, 0.02)| / 127. */
static void q8_matrix(unsigned char *dst, int rows, int cols) {
    const int nb = cols / 32;
    for (int r = 0; r < rows; r++)
        for (int b = 0; b < nb; b++) {
            unsigned char *blk = dst + ((size_t)r * nb + b) * 36;
            const float d = fabsf(gauss(0.02f)) / 127.0f;
            memcpy(blk, &d, 4);
            for (int i = 0; i < 32; i++) blk[4 + i] = (unsigned char)(int8_t)((int)(splitmix() % 255) - 127);
        }
}

typedef struct {
    const unsigned char *blobs;
    size_t stride;
} blob_source;

/* The reference loader port: fills dst with the blob of (layer, expert). */
static int load_blob(void *ctx, int layer, int expert, void *dst) {
    const blob_source *src = (const blob_source *)ctx;
    if (layer != 0) return -1;
    memcpy(dst, src->blobs + (size_t)expert * src->stride, src->stride);
    return 0;
}

/* moe() of src/model/forward.c becomes this forwarder. */
static int moe(miag_ctx *gpu, int l, float *x) {
    char err[256];
    if (miag_moe(gpu, l, x, 1, err, sizeof err) != 0) {
        fprintf(stderr, "miag_moe: %s\n", err);
        return -1;
    }
    return 0;
}

int main(int argc, char **argv) {
    const int T = argc > 1 ? atoi(argv[1]) : 6;
    const miag_shape sh = {2048, 1, 128, 8, 768, 1, 1e-6f};
    const ref_shape rs = {2048, 128, 8, 768, 1, 1e-6f};
    const int d = sh.dim, E = sh.n_experts, eh = sh.expert_hidden;
    const size_t stride = miag_blob_bytes(&sh);
    const size_t mat = (size_t)eh * (d / 32) * 36, off_up = (mat + 63) / 64 * 64;
    rng_state = 20240611u;
    float *ffn_norm = malloc(sizeof(float) * d), *router = malloc(sizeof(float) * (size_t)E * d);
    unsigned char *blobs = calloc((size_t)E, stride);
    float *x = malloc(sizeof(float) * (size_t)T * d), *xr = malloc(sizeof(float) * (size_t)T * d);
    float *x0 = malloc(sizeof(float) * (size_t)T * d);
    if (!ffn_norm || !router || !blobs || !x || !xr || !x0) {
        fprintf(stderr, "out of host memory\n");
        return 2;
    }
    for (int i = 0; i < d; i++) ffn_norm[i] = 1.0f;
    for (size_t i = 0; i < (size_t)E * d; i++) router[i] = gauss(0.02f);
    for (int e = 0; e < E; e++) {
        unsigned char *b = blobs + (size_t)e * stride;
        q8_matrix(b, eh, d);              /* gate */
        q8_matrix(b + off_up, eh, d);     /* up */
        q8_matrix(b + 2 * off_up, d, eh); /* down */
    }
    for (int t = 0; t < T; t++) {
        double ss = 0;
        for (int i = 0; i < d; i++) {
            const float v = gauss(1.0f);
            x0[(size_t)t * d + i] = v;
            ss += (double)v * v;
        }
        const float inv = (float)(1.0 / sqrt(ss / d));
        for (int i = 0; i < d; i++) x0[(size_t)t * d + i] *= inv;
    }
    memcpy(x, x0, sizeof(float) * (size_t)T * d);
    memcpy(xr, x0, sizeof(float) * (size_t)T * d);

    char err[256];
    miag_ctx *gpu = NULL;
    blob_source src = {blobs, stride};
    if (miag_open(&gpu, &sh, 0, err, sizeof err) != 0 ||
        miag_load_experts(gpu, load_blob, &src, err, sizeof err) != 0 ||
        miag_set_layer(gpu, 0, ffn_norm, router, NULL, err, sizeof err) != 0) {
        fprintf(stderr, "set-up: %s\n", err);
        return 2;
    }
    for (int t = 0; t < T; t++)  /* one token a call, as mia_model_step does */
        if (moe(gpu, 0, x + (size_t)t * d) != 0) return 2;
    miag_close(gpu);

    if (ref_moe(&rs, ffn_norm, router, NULL, blobs, stride, xr, T, NULL, NULL, 1) != 0) {
        fprintf(stderr, "reference moe() failed\n");
        return 2;
    }
    int exact = 0, bad = 0;
    double worst = 0;
    for (int t = 0; t < T; t++) {
        double num = 0, den = 0;
        int same = 1;
        for (int i = 0; i < d; i++) {
            const size_t k = (size_t)t * d + i;
            const double a = (double)x[k] - x0[k], b = (double)xr[k] - x0[k];
            num += (a - b) * (a - b), den += b * b;
            if (memcmp(&x[k], &xr[k], 4)) same = 0;
        }
        const double rel = sqrt(num / (den > 0 ? den : 1e-300));
        worst = rel > worst ? rel : worst;
        exact += same, bad += rel > 1e-3;
    }
    printf("moe() forwarder vs reference moe(): %d tokens, %d bit-exact, worst rel-L2 %.2e: %s\n",
           T, exact, worst, bad ? "FAIL" : "ok");
    free(ffn_norm), free(router), free(blobs), free(x), free(xr), free(x0);
    return bad ? 1 : 0;
}
