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


// Row of pair `pid` (pair order) of the down projections: y itself, or under
// expert parallelism the row at the pair's origin rank (YRoute).  The source
// rank is found by compares on compile-time indices, so the route stays in
// the parameter bank.
__device__ __forceinline__ float *y_route_row(const YRoute &yr, float *y, int d, int pid) {
    if (yr.n == 0) return y + (size_t)pid * d;
    float *base = yr.dst[0];
    int start = 0;
#pragma unroll
    for (int i = 0; i < kEpMaxRanks - 1; i++)
        if (i + 1 < yr.n && pid >= yr.end[i]) base = yr.dst[i + 1], start = yr.end[i];
    return base + (size_t)(pid - start) * d;
}

// Expert parallelism: after the CTA's y rows (stores to peer memory among
// them) the CTA is counted, and the launch's last CTA sets this rank's flag
// on every rank (st.release.sys), so a rank that sees its flags at seq may
// read every row stored for it.
__device__ __forceinline__ void ep_signal_done(const YRoute &yr) {
    __threadfence_system();  // this thread's y stores, before the CTA is counted
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(yr.done, 1u) == gridDim.x - 1) {
        __threadfence_system();
        *yr.done = 0;  // for the next launch
        for (int r = 0; r < yr.n; r++) st_release_sys(yr.flags[r] + yr.me, yr.seq);
    }
}

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
    int32_t *chunk_brow;   // [chunks]      first row of each chunk in the pair-tile buffers bx / bh:
                           //               the pairs of earlier chunks, each chunk rounded up to 16
    int chunk;             // pairs per chunk (0: tok_chunk(P, E))
    int tc;                // prefill regime on the tcgen05 kernels (tc.cu)
    uint8_t *bx;           // tcgen05 prefill: gate/up activations as swizzled pair tiles (tc.cu)
    uint8_t *bh;           // tcgen05 prefill: down activations (Q8_0 h) as pair tiles
    int32_t *tc_sched;     // [4] tcgen05 launches' item counters (gate/up, down): zero between
                           //               launches (kept by the launches; zero at creation)
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
    size_t x_stride;          // bytes between rows of xq (0: d)
    size_t dx_stride;         // floats between rows of dx (0: scale_pad(d / 32)); records that
                              //            carry a row's values and scales together set both
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
constexpr int kTcChunk = 128;  // pairs per chunk of the tcgen05 prefill kernels (one MMA's N)
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

// tc.cu: the prefill regime on the 5th-generation tensor cores
bool tc_supported(const Dims &m);              // shapes the tcgen05 kernels take
size_t tc_tile_bytes(const Dims &m, int P, bool gu);  // bytes of bx (gu) or bh
void launch_tc_gather(const Dims &m, const StoreLayout &lay, const Work &w, int num_sms, int *err,
                      cudaStream_t s);  // gate/up's pair tiles (bx)
void launch_tc_swiglu(const Dims &m, const StoreLayout &lay, const Work &w, int num_sms, int *err,
                      cudaStream_t s);  // h = silu(gate) * up as Q8_0 pair tiles (bh)
void launch_gateup_tc(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w,
                      int num_sms, int *err, cudaStream_t s);
void launch_down_tc(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w,
                    int num_sms, int *err, cudaStream_t s);
int tc_setup_attributes();
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
