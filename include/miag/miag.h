/*
 * miag.h -- C ABI of the B200 (sm_100a) MoE FFN block for the motorIa engine.
 *
 * libmiag.so replaces, for one layer's MoE feed-forward block, the body of
 * motorIa's static `moe()` (src/model/forward.c:167-197) and the Q8_0 /
 * f32 `mia_matvec` it calls (src/tensor/matmul.c:91-106).  The expert
 * weights live in HBM for the lifetime of the context, so the reference's
 * disk-streamed LRU cache (src/storage/expert_cache.c:59-85) is not needed;
 * its loader port (include/mia/expert_cache.h:8) is still how blobs arrive.
 *
 * Conventions follow the reference: functions return 0 on success and -1 on
 * failure, writing a message into err[errlen] (mia_file_open,
 * include/mia/mia_file.h:40).  Nothing here calls exit() or prints.  No CPU
 * fallback exists: without an sm_100a GPU every compute entry point fails.
 * A context is used by one host thread at a time (like mia_model).
 */
#ifndef MIAG_H
#define MIAG_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct miag_ctx miag_ctx;

/* The mia_header fields the MoE block reads (include/mia/mia_file.h:10-19).
 * dim and expert_hidden are multiples of 32; n_active <= 64 (forward.c:172). */
typedef struct {
    int32_t dim;           /* d, 2048 for Qwen3-30B-A3B */
    int32_t n_layers;      /* layers whose experts are kept resident */
    int32_t n_experts;     /* E <= 1024 */
    int32_t n_active;      /* K, top-k per token */
    int32_t expert_hidden; /* eh */
    int32_t norm_topk;     /* renormalise the top-k weights (forward.c:180) */
    float norm_eps;        /* rmsnorm epsilon */
} miag_shape;

/* The reference loader port, include/mia/expert_cache.h:8: fills dst with the
 * expert blob (layer, expert) in .mia layout (gate | up | down, Q8_0 rows,
 * offsets as src/storage/mia_file.c:275-278).  mia_file_read_expert
 * (include/mia/mia_file.h:44) has this signature. */
typedef int (*miag_expert_loader)(void *ctx, int layer, int expert, void *dst);

/* Byte size of one expert blob in .mia layout for this shape
 * (tools/internal/mia/format.go:160-163, 16 KiB aligned). */
size_t miag_blob_bytes(const miag_shape *shape);

/* Writes a .mia model file (the converter's output, tools/internal/mia/
 * format.go:200-263, as src/storage/mia_file.c:41-111 reads it) from a
 * model held elsewhere, one tensor or expert at a time: for a machine where
 * the reference's Go converter cannot run.  Dense tensors come as f32 by
 * their canonical names (token_embd; blk.<l>.attn_norm, wq, wk, wv, wo,
 * q_norm, k_norm, ffn_norm, router; output_norm, output) and matrices are
 * quantized to Q8_0 as the reference quantizes (src/tensor/quant.c:11-27);
 * experts come already in .mia blob layout through the loader port
 * signature.  Weight type Q8_0.  Host code only: no GPU needed. */
typedef struct {
    uint32_t dim, n_layers, n_heads, n_kv_heads, head_dim, vocab;
    uint32_t n_experts, n_active, expert_hidden, norm_topk;
    float rope_theta, norm_eps;
} miag_mia_config;
/* Fills dst with the n f32 values (row-major) of the dense tensor `name`. */
typedef int (*miag_mia_dense_source)(void *ctx, const char *name, float *dst, size_t n);
int miag_mia_write(const char *path, const miag_mia_config *config,
                   miag_mia_dense_source dense, miag_expert_loader expert, void *source_ctx,
                   const void *tokenizer, size_t tokenizer_bytes, char *err, size_t errlen);
/* The file's expert_blob_size for this config. */
size_t miag_mia_expert_blob_bytes(const miag_mia_config *config);

/* Creates a context on CUDA device `device`: validates the shape, allocates
 * HBM for every layer's experts and dense router tensors.  Replaces
 * mia_cache_init (include/mia/expert_cache.h:28-30) for the MoE path. */
int miag_open(miag_ctx **out, const miag_shape *shape, int device, char *err,
              size_t errlen);
void miag_close(miag_ctx *c);

/* Per-layer dense tensors of the block: ffn_norm [dim] and router
 * [n_experts][dim] f32 (src/storage/mia_file.c:265-266).  bias [n_experts]
 * is an optional logit offset added after the router matvec (NULL for the
 * reference's behaviour). */
int miag_set_layer(miag_ctx *c, int layer, const float *ffn_norm,
                   const float *router, const float *bias, char *err,
                   size_t errlen);

/* Uploads n expert blobs of one layer from host memory (blob e at
 * blobs + (e - first) * stride) into the resident HBM store. */
int miag_upload_experts(miag_ctx *c, int layer, int first, int n,
                        const void *blobs, size_t stride, char *err,
                        size_t errlen);

/* Uploads every (layer, expert) through the reference loader port, the way
 * mia_cache_get fills a slot on a miss (src/storage/expert_cache.c:78).  A
 * loader failure aborts with -1 and leaves the store unchanged for that
 * expert. */
int miag_load_experts(miag_ctx *c, miag_expert_loader load, void *load_ctx,
                      char *err, size_t errlen);

/* miag_upload_experts from DEVICE memory (no reference counterpart: for
 * blobs that already sit in HBM, e.g. generated there).  Only enqueues on
 * `stream` (NULL = the context's stream); blobs_dev must stay valid until
 * the stream has passed this point. */
int miag_upload_experts_device(miag_ctx *c, int layer, int first, int n,
                               const void *blobs_dev, size_t stride, void *stream,
                               char *err, size_t errlen);

/* The MoE block, replacing forward.c:167-197 for n_tokens independent
 * tokens: x [n_tokens][dim] f32 is the residual stream, read and updated in
 * place (x += sum_j w_j * down_j(silu(gate_j xn) * up_j xn)).
 * miag_moe takes a HOST pointer and returns when x holds the result.
 * miag_moe_async takes a DEVICE pointer and only enqueues on `stream`
 * (a cudaStream_t; NULL = the context's own stream). */
int miag_moe(miag_ctx *c, int layer, float *x, int n_tokens, char *err,
             size_t errlen);
int miag_moe_async(miag_ctx *c, int layer, float *x_dev, int n_tokens,
                   void *stream, char *err, size_t errlen);
/* miag_moe with at least 2048 tokens moves them through in `chunks` pieces
 * (default 4; 1: one piece): a copy stream brings piece k + 1 in and takes
 * piece k - 1 out while the block runs on piece k, so most of the host
 * transfers hide behind the kernels.  With three or more pieces the first
 * and the last hold n / (2 chunks) tokens, which shortens the exposed
 * copies; the others split the rest.  Tokens are independent in the block,
 * so the results equal one pass over all of them bit for bit; the
 * inspection calls (miag_routing, miag_router_logits) then describe the
 * last piece.  No reference counterpart (the reference has no device). */
int miag_set_transfer_chunks(miag_ctx *c, int chunks);
/* miag_moe with a pageable host buffer of 1 MiB to 1 GiB (malloc'd, like
 * the reference's m->x) copies it through a pinned staging buffer of the
 * context with `threads` host threads (the calling one included), piece by
 * piece, so that the host copies overlap the transfers and the block.
 * Default min(8, cores - 1); 0 leaves pageable buffers to the CUDA driver's
 * own staged copies, and so does a call whose pinned staging buffer or
 * threads cannot be had.  Pinned (registered) buffers are always copied
 * directly.  Results are the same bits either way.  No reference
 * counterpart. */
int miag_set_host_copy_threads(miag_ctx *c, int threads);

/* The MoE block with nothing allocated during the call.  No counterpart in
 * the reference (motorIa sizes all scratch once, from its RAM budget).  For
 * callers that cannot let a call allocate device memory: an engine that
 * reserves every byte of HBM up front under a fixed budget, or a serving
 * loop that cannot take cudaMalloc's implicit device-wide synchronisation in
 * the middle of a step (miag_moe_async grows its workspace with cudaMalloc
 * when a batch is larger than any before it).  Same kernels and results as
 * miag_moe_async; x_dev and stream as there.  The scratch is one fixed
 * 11 MiB array inside the loaded library, held by every GPU that loads
 * libmiag until the process exits, which bounds a batch to 92 tokens at
 * Qwen3-30B-A3B shapes; larger batches return -1 with a message.  The
 * first call on a device looks the array's address up (make it before any
 * stream capture) and keeps it for the life of the process, so a device
 * reset while libmiag is loaded is not supported.  All calls share the
 * array, so calls whose work overlaps on the GPU race on it and must be
 * serialised by the caller.  When a call reports a device error
 * (miag_sync), the counters at the head of the array, which every call
 * expects at zero, are cleared again before miag_sync returns. */
int miag_moe_noalloc(miag_ctx *c, int layer, float *x_dev, int n_tokens,
                     void *stream, char *err, size_t errlen);

/* The same block in three device steps, for expert parallelism: each GPU
 * routes its own tokens, the caller moves (row, expert) pairs to the GPUs
 * that hold the experts, those run the expert products, and the results come
 * back to be combined where the tokens live.  moe() (forward.c:174-194) is
 * exactly route -> experts -> combine; the split changes no arithmetic, so
 * the results are those of miag_moe_async bit for bit.  All pointers are
 * device pointers; all calls only enqueue on `stream` (NULL = own stream).
 *
 * miag_route_async: forward.c:174-181 for n_tokens rows of x [n][dim]:
 *   idx, w [n][n_active] (the top-k and its weights), and the Q8_0 form of
 *   the normalised rows that the expert products read (quant.c:11-27):
 *   xq [n][dim] int8 values, dx [n][miag_dx_stride()] f32 block scales.
 * miag_experts_async: the expert products of n_pairs pairs; pair p is row
 *   pair_row[p] (< n_rows) of xq/dx against expert pair_expert[p]
 *   (forward.c:186-193, SwiGLU included): y [n_pairs][dim] f32, in pair order.
 * miag_combine_async: x[t] += sum_j w[t][j] * y[row(t*n_active + j)], j in
 *   order (forward.c:194), for t < n_tokens; row(p) = y_pos[p], or p when
 *   y_pos is NULL (y in pair order).  While the context's device error word
 *   is set (an earlier step failed and miag_sync has not reported it yet),
 *   the combine leaves x unchanged. */
int miag_route_async(miag_ctx *c, int layer, const float *x_dev, int n_tokens,
                     int32_t *idx, float *w, int8_t *xq, float *dx, void *stream,
                     char *err, size_t errlen);
int miag_experts_async(miag_ctx *c, int layer, const int8_t *xq, const float *dx,
                       int n_rows, const int32_t *pair_row,
                       const int32_t *pair_expert, int n_pairs, float *y,
                       void *stream, char *err, size_t errlen);
int miag_combine_async(miag_ctx *c, float *x_dev, int n_tokens, const float *w,
                       const float *y, const int32_t *y_pos, void *stream,
                       char *err, size_t errlen);
/* f32 scales per row of dx: dim/32 rounded up to a multiple of four. */
int miag_dx_stride(const miag_shape *s);

/* The exchange of expert parallelism (no reference counterpart: the
 * reference runs on one device).  Experts are split over n_ranks ranks
 * (1..8), experts_per_rank each: expert e lives on rank e / experts_per_rank,
 * or on e % n_ranks when strided is nonzero.  Order on every rank: rows
 * grouped by destination rank, tokens ascending; pairs grouped by
 * destination, pair id t*n_active + j ascending.
 * miag_ep_plan_async: from idx [n_tokens][n_active] (miag_route_async),
 *   counts [n_ranks][2] int64 (rows, pairs) to each rank; send_rows
 *   [n_tokens*n_ranks] the token of each row to send (the first
 *   sum(rows) are used); pair_meta [n_tokens*n_active][2] (row within the
 *   destination's block from this rank, expert) in pair order as above;
 *   y_pos [n_tokens*n_active] the place of pair t*n_active + j in that
 *   order, for miag_combine_async.
 * miag_ep_pack_async: the send buffers of rank `rank`.  rec [n_rows] records
 *   of dim int8 values then miag_dx_stride f32 scales, the rows of xq/dx
 *   named by send_rows; meta_out [n_pairs][2] the pair records with each row
 *   renumbered in the receiver's buffer, where lower ranks' rows come first.
 *   all_counts [n_ranks][n_ranks][2] holds every rank's counts, in rank
 *   order (an all-gather of counts). */
int miag_ep_plan_async(miag_ctx *c, const int32_t *idx, int n_tokens, int n_ranks,
                       int experts_per_rank, int strided, int64_t *counts,
                       int32_t *send_rows, int32_t *pair_meta, int32_t *y_pos,
                       void *stream, char *err, size_t errlen);
int miag_ep_pack_async(miag_ctx *c, const int8_t *xq, const float *dx,
                       const int32_t *send_rows, int n_rows, const int32_t *pair_meta,
                       int n_pairs, const int64_t *all_counts, int rank, int n_ranks,
                       uint8_t *rec, int32_t *meta_out, void *stream, char *err,
                       size_t errlen);

/* The return of the y rows over NVLink peer memory (no reference
 * counterpart).  Each rank's exchange buffer holds the y rows of its own
 * pairs, in its send order, and one completion flag per rank; the peers map
 * it through CUDA IPC, so the ranks must be processes on distinct GPUs of
 * one node.
 * miag_ep_buffer: allocates (or grows) this rank's buffer for y_rows rows of
 *   dim f32; returns the rows, the flags [8] (zeroed when allocated) and a
 *   64-byte cudaIpcMemHandle_t for the peers.  Growing frees the old buffer:
 *   every peer must have closed its mapping first (miag_ep_close_peers).
 * miag_ep_open_peer: maps a peer's buffer (its handle); returns its rows and
 *   flags.  miag_ep_close_peers unmaps every peer buffer opened.
 * miag_experts_to_ranks_async: miag_experts_async, except that the y row of
 *   pair p, received from rank s (pairs [src_end[s-1], src_end[s]), in rank
 *   order), is stored at dst[s] + (p - src_end[s-1]) rows on rank s; when
 *   all rows are stored, flags[r][rank] = seq on every rank r.  src_end,
 *   dst and flags are host arrays of n_ranks entries (dst, flags: device
 *   addresses as miag_ep_buffer / miag_ep_open_peer gave them).  With no
 *   pairs it only sets the flags.
 * miag_ep_wait_async: enqueues a wait until flags[r] >= seq for every rank
 *   r < n_ranks (this rank's own flags); then every row stored for this rank
 *   has landed.  The wait gives up after two seconds and reports it as a
 *   device error at the next miag_sync.  After such an error the combine
 *   leaves x as it was (every combine skips while the error word is set),
 *   and a late peer store may still land in the buffer: close the peers,
 *   re-create the buffers (zeroed flags) and re-open them on every rank
 *   before the exchange is used again. */
int miag_ep_buffer(miag_ctx *c, size_t y_rows, void **y_dev, unsigned **flags_dev,
                   void *ipc_handle, char *err, size_t errlen);
int miag_ep_open_peer(miag_ctx *c, const void *ipc_handle, void **y_dev,
                      unsigned **flags_dev, char *err, size_t errlen);
int miag_ep_close_peers(miag_ctx *c, char *err, size_t errlen);
int miag_experts_to_ranks_async(miag_ctx *c, int layer, const int8_t *xq, const float *dx,
                                int n_rows, const int32_t *pair_row,
                                const int32_t *pair_expert, int n_pairs, int n_ranks,
                                int rank, const int32_t *src_end, float *const *dst,
                                unsigned *const *flags, unsigned seq, void *stream,
                                char *err, size_t errlen);
int miag_ep_wait_async(miag_ctx *c, const unsigned *flags, int n_ranks, unsigned seq,
                       void *stream, char *err, size_t errlen);

/* The expert-parallel block in one call (no reference counterpart: the
 * reference runs moe(), src/model/forward.c:167-197, on one device).  The
 * ranks of an NCCL communicator, one GPU each on one node (2..8; 1 works
 * too), each hold E / N experts of every layer in their context's store:
 * rank r the experts r*E/N .. (r+1)*E/N - 1 (contiguous), or r, r+N,
 * r+2N, ... when strided is nonzero; the caller uploads them (miag_ep_rank
 * says which).  Each rank brings its own tokens.  miag_moe_ep_async is then
 * moe() for n_tokens rows of x on every rank at once: route here, the
 * (row, expert) pairs to the ranks that hold the experts (NCCL send/recv,
 * after one all-gather of the per-rank counts, the one host
 * synchronisation of a step), the expert products there, each result row
 * stored back into this rank's memory over NVLink, the combine here.  The
 * outputs equal miag_moe's bit for bit.  Every rank must make the same
 * sequence of calls (collectives inside), with any n_tokens >= 0.
 * NCCL is loaded at run time (libnccl.so.2).  The context's exchange buffer
 * (miag_ep_buffer) belongs to the block while it is open.
 *
 * miag_nccl_unique_id: 128 bytes for rank 0 to share with the others
 *   (ncclGetUniqueId); miag_nccl_comm_init: this rank's communicator on
 *   `device` (ncclCommInitRank); miag_nccl_comm_destroy frees it (after
 *   miag_ep_close).
 * miag_ep_open: binds a context to a communicator.  Refuses ranks that
 *   share a GPU (their flag waits could not both run).
 * miag_moe_ep_async: x_dev a DEVICE pointer, enqueued on `stream` (NULL =
 *   the context's stream); device errors (a peer that never stores its
 *   rows: the bounded wait gives up after two seconds) reach the next
 *   miag_sync.  miag_moe_ep: the same from a HOST pointer, returning when x
 *   holds the result.
 * miag_ep_rank: this rank, the number of ranks, and its experts: first,
 *   count, and the step between them.  miag_ep_last_received: the rows and
 *   pairs this rank's experts worked on in the last step. */
typedef struct miag_ep miag_ep;
int miag_nccl_unique_id(void *id, char *err, size_t errlen);
int miag_nccl_comm_init(void **comm, int n_ranks, const void *id, int rank, int device,
                        char *err, size_t errlen);
void miag_nccl_comm_destroy(void *comm);
int miag_ep_open(miag_ep **out, miag_ctx *c, void *nccl_comm, int strided, char *err,
                 size_t errlen);
void miag_ep_close(miag_ep *ep);
int miag_moe_ep_async(miag_ep *ep, int layer, float *x_dev, int n_tokens, void *stream,
                      char *err, size_t errlen);
int miag_moe_ep(miag_ep *ep, int layer, float *x, int n_tokens, char *err, size_t errlen);
int miag_ep_rank(const miag_ep *ep, int *rank, int *n_ranks, int *first_expert,
                 int *n_experts_here, int *stride);
int miag_ep_last_received(const miag_ep *ep, int *rows, int *pairs);

/* Waits for the context's work on `stream` (NULL = own stream) and reports
 * any device-side error (a bounded wait that gave up, a bad index). */
int miag_sync(miag_ctx *c, void *stream, char *err, size_t errlen);

/* Self-test of the failure path (no reference counterpart): runs one bounded
 * wait on a barrier that never completes, with a limit of timeout_us
 * (1..100000), and reports it as the block's kernels report a tile that
 * never lands.  Returns -1 with "device error 1: ... timed out ..." in err
 * when the wait gave up, as it always should; the context stays usable. */
int miag_selftest_wait_timeout(miag_ctx *c, int timeout_us, char *err, size_t errlen);

/* Routing of the most recent miag_moe / miag_moe_async call, copied to host
 * (any pointer may be NULL): idx, w [n_tokens][n_active]; counts [E];
 * offsets [E+1]; perm [n_tokens*n_active] (pair id t*K+j at each position of
 * the canonical expert-sorted order). */
int miag_routing(miag_ctx *c, int32_t *idx, float *w, int32_t *counts,
                 int32_t *offsets, int32_t *perm, char *err, size_t errlen);

/* Router logits (+ bias) [n_tokens][n_experts] of the most recent call: the
 * values forward.c:175 leaves in m->router before softmax. */
int miag_router_logits(miag_ctx *c, float *logits, char *err, size_t errlen);

/* Device kernels behind the reference's public math ABI, on device pointers
 * and a stream (NULL = legacy default stream):
 *   miag_quantize_row_q8  <- mia_quantize_row_q8 (include/mia/quant.h:18,
 *                            src/tensor/quant.c:11-27); y holds n/32 36-byte
 *                            mia_block_q8 records.
 *   miag_matvec           <- mia_matvec (include/mia/matmul.h:11-12); w is
 *                            row-major f32 (wtype 0) or Q8_0 blocks (wtype 1);
 *                            xq is scratch for cols/32 blocks (Q8_0 only). */
int miag_quantize_row_q8(const float *x, void *y, int n, void *stream);
int miag_matvec(float *out, const void *w, int wtype, const float *x,
                void *xq, int rows, int cols, void *stream);

/* Number of kernels the most recent miag_moe / miag_moe_async launched. */
int miag_last_launch_count(const miag_ctx *c);

/* Which kernels run the expert products of prefill-size batches (more than
 * 8 (token, expert) pairs per expert on average; no reference counterpart --
 * the reference has one scalar matvec, src/tensor/matmul.c:19-28).  Both
 * give the same bits.  MIAG_PREFILL_MMA (the default): the mma.sync kernels
 * of the decode regime.  MIAG_PREFILL_TCGEN05 (where the shape allows: dim
 * and expert_hidden multiples of 256): the block dots on the tcgen05 tensor
 * cores into tensor memory, the exact FP32 steps in separate epilogue
 * warps, weights read from HBM once per launch.  miag_set_prefill_kernel
 * waits for the context's stream. */
#define MIAG_PREFILL_MMA 0
#define MIAG_PREFILL_TCGEN05 1
int miag_set_prefill_kernel(miag_ctx *c, int kind, char *err, size_t errlen);
int miag_prefill_kernel(const miag_ctx *c);

/* ---- The whole decode step ---------------------------------------------
 * A model in HBM: the .mia dense section (embedding, attention, norms,
 * routers, LM head), an f32 KV cache of max_seq positions per layer, and the
 * MoE blocks of a miag_ctx.  Replaces the reference's model state and step
 * (mia_model_init / mia_model_step, include/mia/model.h:17-27,
 * src/model/forward.c:36-62 and 199-217); the logits equal mia_model_step's
 * bit for bit.  One step is one CUDA graph replay (captured on first use).
 *
 * miag_model_open: `moe` holds the experts (miag_load_experts) and must
 *   have the model's MoE shape; it is not owned.  `dense` is the file's
 *   dense section (mia_file.dense, mia_header.dense_size bytes) in host
 *   memory, uploaded here, or NULL to fill it with miag_model_synth.
 * miag_model_open_file: opens a Q8_0 .mia file (mia_file_open,
 *   src/storage/mia_file.c:41-111) on `device`, experts and all; the model
 *   owns its context.
 * miag_model_synth: seeded random weights on the device (no reference
 *   counterpart; benchmarks without a converted checkpoint): Q8_0 matrices
 *   with q uniform on [-127, 127] and d = |N(0, 0.02)| / 127, routers
 *   N(0, 0.02), norms 1.
 * miag_model_step: one token at one position; returns the logits [vocab]
 *   in host memory owned by the model (valid until the next call), or NULL
 *   with a message (token or position out of range, as forward.c:202-203).
 *   miag_model_step_async only enqueues; miag_model_logits_device holds the
 *   result once miag_model_sync returns 0.
 * miag_model_generate: the prompt one position at a time, then n_new
 *   greedy tokens (argmax, the lowest index on ties), entirely on the device;
 *   tokens_out receives the n_new tokens.  The _async form leaves them at
 *   miag_model_tokens_device()[n_prompt ...].
 * Not re-entrant; one host thread per model, as mia_model. */
typedef struct miag_model miag_model;
int miag_model_open(miag_model **out, miag_ctx *moe, const miag_mia_config *config,
                    const void *dense, size_t dense_bytes, int max_seq, char *err,
                    size_t errlen);
int miag_model_open_file(miag_model **out, const char *path, int device, int max_seq,
                         char *err, size_t errlen);
void miag_model_close(miag_model *m);
int miag_model_synth(miag_model *m, uint64_t seed, char *err, size_t errlen);
const float *miag_model_step(miag_model *m, int token, int pos, char *err, size_t errlen);
int miag_model_step_async(miag_model *m, int token, int pos, char *err, size_t errlen);
int miag_model_generate(miag_model *m, const int32_t *prompt, int n_prompt, int n_new,
                        int32_t *tokens_out, char *err, size_t errlen);
int miag_model_generate_async(miag_model *m, const int32_t *prompt, int n_prompt, int n_new,
                              char *err, size_t errlen);
/* n_steps more greedy steps from where the last step left the model's
 * device state (its next token and position); enqueues only.  A step whose
 * position reaches max_seq fails at miag_model_sync. */
int miag_model_continue_async(miag_model *m, int n_steps, char *err, size_t errlen);
int miag_model_sync(miag_model *m, char *err, size_t errlen);
const float *miag_model_logits_device(const miag_model *m);
const int32_t *miag_model_tokens_device(const miag_model *m);
void *miag_model_stream(const miag_model *m);  /* a cudaStream_t */
miag_ctx *miag_model_moe(const miag_model *m);
int miag_model_launches_per_step(const miag_model *m);
/* 1 when steps run as CUDA graph replays, 0 when they are launched directly
 * (the capture failed) or no step has run yet. */
int miag_model_uses_graph(const miag_model *m);

/* Batched prefill.  Replaces the reference's prompt loop, one
 * mia_model_step per prompt token (src/app/main.c:119-124,
 * src/app/serve.c:92-107), with one pass per layer over all n positions:
 * each dense weight tile is staged once for 32 positions, the MoE block runs
 * once per layer over the n tokens (the prefill-regime expert kernels), and
 * the LM head runs for the last position only.  Every position's arithmetic
 * is mia_model_step's, so the KV cache and the logits of position pos + n - 1
 * (miag_model_logits_device) equal those of n single steps bit for bit.
 * The head also picks the next token (greedy: argmax, lowest index on ties)
 * into miag_model_tokens_device()[pos + n] and leaves the step arguments at
 * (that token, pos + n), so miag_model_continue_async generates from there.
 * Enqueues only; errors of the launches surface at miag_model_sync.
 * miag_model_generate* run their prompt this way when it has more than one
 * token, unless miag_model_set_batched_prefill(m, 0) asks for one step per
 * position.  miag_model_prefill waits and returns the last position's
 * logits in host memory owned by the model, or NULL with a message, as
 * miag_model_step.  miag_model_prefill_launches: kernels the last prefill
 * launched. */
const float *miag_model_prefill(miag_model *m, const int32_t *tokens, int n, int pos, char *err,
                                size_t errlen);
int miag_model_prefill_async(miag_model *m, const int32_t *tokens, int n, int pos, char *err,
                             size_t errlen);
int miag_model_set_batched_prefill(miag_model *m, int on);

/* The next-token choice on the device.  Replaces mia_sampler_init /
 * mia_sample (include/mia/sampler.h, src/tokenizer/sampler.c:5-66) in the
 * generation loops of src/app/main.c:126-141 and serve.c:115-133: with
 * temperature > 0 every step (and a prefill) draws its next token as
 * mia_sample does -- e = expf((l - max) / temperature) with the serial sum,
 * the candidates p >= (1 - top_p) / (n - 1) in the order of glibc's stable
 * qsort (p descending, then index), the smallest prefix reaching top_p, and
 * the xorshift64* draw from `seed` (0: the reference's fixed default) -- so
 * a generation equals the reference loop's token for token.  Temperature
 * <= 0: the greedy argmax of the head (the default).  Waits for the model's
 * stream; the next step re-captures its graph. */
int miag_model_set_sampler(miag_model *m, float temperature, float top_p, uint64_t seed, char *err,
                           size_t errlen);
int miag_model_prefill_launches(const miag_model *m);

/* Per-kernel timing (no reference counterpart; the reference only has
 * wall-clock stats, src/app/main.c:146-158).  While enabled, every kernel of
 * the block is bracketed by CUDA events on the stream it is launched on.
 * miag_profile_read waits for them and returns, per kernel stage i <
 * miag_profile_stages(), the summed milliseconds and launch count since the
 * last read (which resets them).  miag_profile_stage_name(i) names stage i. */
int miag_profile(miag_ctx *c, int enable);
int miag_profile_stages(void);
const char *miag_profile_stage_name(int i);
int miag_profile_read(miag_ctx *c, double *ms, int32_t *launches, char *err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif
