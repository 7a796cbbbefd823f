/*
 * moe_oracle.h -- CPU oracle for the motorIa Qwen3-MoE FFN block.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (motoria_b200/, the
 * libmiag C-ABI) links, loads or calls this code; only tests/, the smoke
 * check in __graft_entry__.py and the cpu_baseline leg of bench.py do, and
 * only as the checker.
 *
 * The oracle restates, in plain C99, the x86 scalar arithmetic of the
 * reference engine (nextocodeoficial/motorIa):
 *   quantizer   src/tensor/quant.c:11-27      (mia_quantize_row_q8)
 *   Q8_0 dot    src/tensor/matmul.c:19-28     (dot_q8_scalar)
 *   f32 dot     src/tensor/matmul.c:13-17     (dot_f32_scalar)
 *   matvec      src/tensor/matmul.c:66-87     (rows_kernel, mia_matvec_scalar)
 *   rmsnorm     src/model/forward.c:75-81
 *   softmax     src/model/forward.c:95-101
 *   top_k       src/model/forward.c:104-114
 *   moe()       src/model/forward.c:167-197
 * It is pinned against the reference compiled from its own sources
 * (oracle/_ref, built by oracle/Makefile) and against the golden vectors in
 * tests/golden/, which that build produced.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK 32

/* One Q8_0 block, byte-compatible with mia_block_q8 (include/mia/quant.h:12-15). */
typedef struct {
    float d;
    int8_t q[ORC_QK];
} orc_block_q8;

/* The header fields the MoE block reads (include/mia/mia_file.h:10-19). */
typedef struct {
    int32_t dim, n_experts, n_active, expert_hidden, norm_topk;
    float norm_eps;
} orc_shape;

/* Byte offsets of up / down inside an expert blob (src/storage/mia_file.c:275-278). */
size_t orc_off_up(const orc_shape *s);
size_t orc_off_down(const orc_shape *s);
size_t orc_blob_bytes(const orc_shape *s); /* down end, rounded to 16 KiB */

void orc_quantize_row_q8(const float *x, orc_block_q8 *y, int n);
void orc_dequantize_row_q8(const orc_block_q8 *y, float *x, int n);
float orc_dot_q8(const orc_block_q8 *w, const orc_block_q8 *x, int nb);
float orc_dot_f32(const float *a, const float *b, int n);
/* out[r] = W[r] . x with W in Q8_0 rows; quantizes x into xq first. */
void orc_matvec_q8(float *out, const void *w, const float *x, orc_block_q8 *xq,
                   int rows, int cols);
void orc_matvec_f32(float *out, const float *w, const float *x, int rows,
                    int cols);
void orc_rmsnorm(float *out, const float *x, const float *w, int n, float eps);
void orc_softmax(float *x, int n);
void orc_top_k(const float *p, int n, int k, int *idx);

/* Router of one token: rmsnorm -> logits (+bias) -> softmax -> top-k ->
 * renormalised weights.  xn receives the normalised input. */
void orc_route(const orc_shape *s, const float *ffn_norm, const float *router,
               const float *bias, const float *x, float *xn, int32_t *idx,
               float *w);

/* Routing only for T tokens (x is read, not modified). */
int orc_route_batch(const orc_shape *s, const float *ffn_norm,
                    const float *router, const float *bias, const float *x,
                    int T, int32_t *idx, float *w, int n_threads);

/* Full MoE block for T independent tokens; x [T][dim] updated in place
 * (residual += sum_j w_j down_j).  idx/w may be NULL.  Returns 0. */
int orc_moe(const orc_shape *s, const float *ffn_norm, const float *router,
            const float *bias, const uint8_t *blobs, size_t blob_stride,
            float *x, int T, int32_t *idx, float *w, int n_threads);

/* Canonical dispatch permutation: (token t, slot j) pairs stably sorted by
 * expert, then t, then j.  counts[E], offsets[E+1], perm[T*K] = pair id
 * t*K+j at each sorted position, inv[T*K] = sorted position of each pair. */
void orc_permute(const int32_t *idx, int T, int K, int E, int32_t *counts,
                 int32_t *offsets, int32_t *perm, int32_t *inv);

#ifdef __cplusplus
}
#endif
#endif
