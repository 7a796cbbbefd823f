// kernels.cuh -- launchers of the MoE block kernels (host-side declarations).
#pragma once

#include "common.cuh"

namespace miag {

// Device workspace of one MoE call over T tokens, P = T*K pairs.
constexpr int kEpMaxRanks = 8;  // one node

// Expert parallelism: where the down launch stores the y row of each pair
// it received.  Pairs arrive grouped by source rank: pairs [end[s-1], end[s])
// came from rank s (end[-1] = 0), and pair p's row goes to
// dst[s] + (p - end[s-1]) rows, in rank s's memory (a peer mapping).  When
// every CTA's rows are stored, the launch's last CTA sets flags[r][me] = seq
// on every rank r.  n == 0: y in pair order in Work::y, no flags.
struct YRoute {
    int n, me;
    unsigned seq;
    int end[kEpMaxRanks];
    float *dst[kEpMaxRanks];
    unsigned *flags[kEpMaxRanks];
    unsigned *done;  // CTAs of the launch done so far; zero between launches
};

struct Work {
    int T, P, nchunks;
    int8_t *xq;            // [T][d]        quantized normalised input (Q8_0 values)
    float *dx;             // [T][xs_pad]   its block scales
    float *logits;         // [T][E]        router logits (+ bias)
    int32_t *idx;          // [T][K]
    float *w;              // [T][K]
    int32_t *rank;         // [P]           stable rank of a pair inside its chunk
    int32_t *chunk_cnt;    // [nchunks][E]
    int32_t *chunk_base;   // [nchunks][E]
    int32_t *counts;       // [E]
    int32_t *offsets;      // [E+1]
    int32_t *active;       // [E]           experts with >= 1 pair, ascending
    int32_t *n_active;     // [1]
    int32_t *chunk_pre;    // [E+1]         exclusive prefix over active experts of ceil(n_e / chunk)
    int4 *chunk_info;      // [chunks]      per pair chunk: (expert, chunk of it, its first sorted
                           //               position, pairs); chunks <= P / kTokChunkNarrow + E
    int32_t *max_chunk;    // [1]           largest chunk (pairs)
    int32_t *chunk_done;   // [chunks]      decode regime: gate/up warp-tiles finished per chunk
                           //               (zeroed by the permutation)
    uint8_t *shares;       // [kShareKinds] ShareState: the expert launches' SM shares; zero at
                           //               creation, kept by the launches themselves
    int32_t *perm;         // [P]           pair id at each sorted position
    int32_t *inv;          // [P]           sorted position of each pair
    float *h;              // [P][2 eh]     gate/up products (gate even, up odd), sorted order
    int8_t *hq;            // [P][eh]       Q8_0 silu(gate) * up, sorted order
    float *hs;             // [P][xs_h]     its block scales (xs_h = scale_pad(eh / 32))
    float *y;              // [P][d]        down projections, pair order
    int32_t *tg_count;     // [T]           route: CTAs done per token group; zero between calls
    YRoute yr;                // down's stores to other ranks (n == 0: none)
    const int32_t *pair_row;  // [P]        expert products over given pairs: each pair's row of
    int n_rows;               //              xq/dx (null: pair p is row p / K, the moe() case)
    const int32_t *y_pos;     // [P]        combine: row of y holding pair p (null: row p)
};

struct LayerDev {
    const float *ffn_norm;  // [d]
    const float *router_t;  // [ceil(E/32)][d/4][32][4]  router, 32-expert groups contiguous
    const float *bias;      // [E] or nullptr
    const uint8_t *experts; // E * layout.expert_bytes
};

struct Dims {
    int d, eh, E, K, norm_topk;
    float eps;
};

constexpr int kPermChunk = 1024;

// How an expert launch (gate/up or down, narrow or wide regime) splits its
// items over the SMs: shares in proportion to each SM's measured item rate.
// A launch reads rate[launches & 1] and writes the other buffer; the last
// CTA to finish clears `taken`, `done` and counts the launch.
constexpr int kMaxSlots = 160;
constexpr int kShareKinds = 4;
struct ShareState {
    int launches;              // launches finished
    int done;                  // CTAs finished in the running launch
    int taken[kMaxSlots];      // slot claimed in the running launch
    float rate[2][kMaxSlots];  // items a microsecond, a running average (0: none yet)
};
// Pairs of one expert handled per expert-GEMV item: 32 once experts average
// more than 8 pairs (the wide regime), 16 below that, where the expert
// launches then need no four-n-tile path and keep every value in registers.
constexpr int kTokChunk = 32;
constexpr int kTokChunkNarrow = 16;
__host__ __device__ inline bool wide_batch(int P, int E) { return (long)P > 8L * E; }
__host__ __device__ inline int tok_chunk(int P, int E) {
    return wide_batch(P, E) ? kTokChunk : kTokChunkNarrow;
}

// Device-side view of one layer of a context (api.cu), for launch sequences
// that bring their own workspace.
struct CtxView {
    int device, num_sms;
    cudaStream_t stream;  // the context's own stream
    Dims dims;
    StoreLayout lay;
    LayerDev layer;
    int *d_err;
};

// route.cu
void launch_route(const Dims &m, const LayerDev &L, const float *x, const Work &w,
                  int *err, cudaStream_t s);
// permute.cu (includes softmax / top-k)
void launch_permute(const Dims &m, const Work &w, int *err, cudaStream_t s);
int permute_launches(int P, int E);
// gemv.cu
void launch_gateup(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w,
                   int num_sms, int *err, cudaStream_t s);
void launch_down(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w,
                 int num_sms, int *err, cudaStream_t s);
void launch_combine(const Dims &m, const Work &w, float *x, int *err, cudaStream_t s);
int down_launches(const Dims &m, int P);  // kernels launch_down issues
int gemv_setup_attributes(const Dims &m, const StoreLayout &lay);

// Expert parallelism (ep.cu): the dispatch plan, the send records, and the
// completion flags of the y rows that down stores at their origin ranks.
int ep_plan_tiles(int T);  // tiles of the plan: tiles[] holds 2 * kEpMaxRanks ints each
void launch_ep_plan(const int32_t *idx, int T, int K, int G, int per_rank, bool strided,
                    int *tiles, long long *counts, int32_t *send_rows, int32_t *pair_meta,
                    int32_t *y_pos, int *err, cudaStream_t s);
void launch_ep_signal(const YRoute &yr, cudaStream_t s);
void launch_ep_wait(const unsigned *flags, int n_ranks, unsigned seq, long long timeout_ns,
                    int *err, cudaStream_t s);
void launch_ep_pack(const int8_t *xq, const float *dx, int d, int xs, const int32_t *send_rows,
                    int n_rows, const int32_t *pair_meta, int n_pairs, const long long *all_counts,
                    int me, int G, uint8_t *rec, int32_t *meta_out, int num_sms, cudaStream_t s);
// noalloc.cu: zeroes the counters at the head of the no-allocation array on
// `device` (a no-op where it was never set up)
void noalloc_clear_counters(int device, cudaStream_t s);
// store.cu
void launch_repack(const Dims &m, const StoreLayout &lay, const uint8_t *aos, size_t aos_stride,
                   int n, uint8_t *dst, cudaStream_t s);
void launch_transpose_router(const float *router, float *router_t, int E, int d,
                             cudaStream_t s);

}  // namespace miag
