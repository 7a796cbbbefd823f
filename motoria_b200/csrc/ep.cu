// Expert parallelism: the dispatch plan and the send records of one rank.
//
// Under expert parallelism each rank routes its own tokens and sends every
// token row once to each rank that holds one of its top-k experts, with one
// (row, expert) record per (token, expert) pair; the expert products come
// back one f32 row per pair and are combined in top-k order, so the results
// equal the one-device block (src/model/forward.c:167-197) bit for bit.
// The reference has no multi-device path; these kernels compute the plan
// of motoria_b200/ep.py:plan_dispatch and the records it sends, so
// that the host only reads the per-rank counts its collectives need.
//
// Order (the one every rank agrees on): rows grouped by destination rank,
// tokens ascending within a destination; pairs grouped by destination, pair
// id t*K + j ascending within a destination.
#include <algorithm>
#include <cstdint>

#include "kernels.cuh"

namespace miag {

namespace {

constexpr int kPlanThreads = 1024;  // tokens a plan CTA places (one tile)

__device__ __forceinline__ int dest_of(int e, int per_rank, int G, bool strided) {
    return strided ? e % G : e / per_rank;
}

// Inclusive scan over the CTA of four 64-bit words a thread, each word four
// 16-bit fields (no field carries into the next: every prefix fits 16 bits).
// Returns the inclusive prefix; `total` gets the CTA's sums.
__device__ __forceinline__ void block_scan4(uint64_t (&v)[4], uint64_t (&total)[4],
                                            uint64_t (*warp_sums)[4]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint64_t u = __shfl_up_sync(0xffffffffu, v[i], o);
            if (lane >= o) v[i] += u;
        }
    }
    if (lane == 31) {
#pragma unroll
        for (int i = 0; i < 4; i++) warp_sums[warp][i] = v[i];
    }
    __syncthreads();
    if (warp == 0) {
        uint64_t s[4];
#pragma unroll
        for (int i = 0; i < 4; i++) s[i] = warp_sums[lane][i];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint64_t u = __shfl_up_sync(0xffffffffu, s[i], o);
                if (lane >= o) s[i] += u;
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) warp_sums[lane][i] = s[i];  // inclusive over warps
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; i++) {
        if (warp > 0) v[i] += warp_sums[warp - 1][i];
        total[i] = warp_sums[31][i];
    }
    __syncthreads();  // warp_sums is reused by the next tile
}

// Field f of the packed words (f < 32): rows to rank g in field 2g, pairs
// to g in field 2g + 1.  Words picked by compare, not by index, so that the
// words stay in registers.
__device__ __forceinline__ int field(const uint64_t (&v)[4], int f) {
    uint64_t w = 0;
#pragma unroll
    for (int i = 0; i < 4; i++)
        if ((f >> 2) == i) w = v[i];
    return (int)((w >> (16 * (f & 3))) & 0xffffu);
}
__device__ __forceinline__ void add_field(uint64_t (&v)[4], int f) {
#pragma unroll
    for (int i = 0; i < 4; i++)
        if ((f >> 2) == i) v[i] += 1ull << (16 * (f & 3));
}

// The destinations of token t's pairs: per destination rank g, whether the
// token goes there (bit g of hit) and its pairs to g (field 2g + 1 of v);
// field 2g of v gets the hit.  A routing index outside [0, E) is placed
// as expert 0 (in bounds) and reported.
__device__ __forceinline__ unsigned token_dests(const int32_t *idx, int t, int K, int E,
                                                int per_rank, int G, bool strided, uint64_t (&v)[4],
                                                int *err) {
    unsigned hit = 0;
    for (int j = 0; j < K; j++) {
        int e = __ldg(idx + (size_t)t * K + j);
        if ((unsigned)e >= (unsigned)E) {
            if (err) set_error(err, kErrBadExpert);
            e = 0;
        }
        const int g = dest_of(e, per_rank, G, strided);
        hit |= 1u << g;
        add_field(v, 2 * g + 1);
    }
#pragma unroll
    for (int g = 0; g < kEpMaxRanks; g++)
        if ((hit >> g) & 1u) add_field(v, 2 * g);
    return hit;
}

// Pass 1, one CTA per tile of 1024 tokens: the tile's rows and pairs to each
// destination, into tiles[tile][2g] and [2g + 1].
__global__ void __launch_bounds__(kPlanThreads, 1)
    k_ep_count(const int32_t *idx, int T, int K, int G, int per_rank, int strided, int *tiles,
               int *err) {
    __shared__ uint64_t warp_sums[32][4];
    const int t = blockIdx.x * kPlanThreads + (int)threadIdx.x;
    uint64_t v[4] = {0, 0, 0, 0};
    if (t < T) token_dests(idx, t, K, per_rank * G, per_rank, G, strided != 0, v, err);
    uint64_t total[4];
    block_scan4(v, total, warp_sums);
    if (threadIdx.x < 2 * kEpMaxRanks)
        tiles[blockIdx.x * 2 * kEpMaxRanks + threadIdx.x] = field(total, (int)threadIdx.x);
}

// Pass 2, one CTA per tile: each token's rows and pairs at their places.
// Every CTA derives the blocks' starts (and its tile's place in them) from
// all tiles' counts; CTA 0 also writes the per-destination counts.
__global__ void __launch_bounds__(kPlanThreads, 1)
    k_ep_place(const int32_t *idx, int T, int K, int G, int per_rank, int strided,
               const int *tiles, int n_tiles, long long *counts, int32_t *send_rows,
               int2 *pair_meta, int32_t *y_pos) {
    __shared__ int row_off[kEpMaxRanks], pair_off[kEpMaxRanks];  // where each block starts
    __shared__ int row_pre[kEpMaxRanks], pair_pre[kEpMaxRanks];  // in earlier tiles
    __shared__ uint64_t warp_sums[32][4];
    if (threadIdx.x < kEpMaxRanks) {
        const int g = threadIdx.x;
        int rows = 0, pairs = 0, rb = 0, pb = 0;
        if (g < G) {
            for (int i = 0; i < n_tiles; i++) {
                const int r = tiles[i * 2 * kEpMaxRanks + 2 * g];
                const int q = tiles[i * 2 * kEpMaxRanks + 2 * g + 1];
                if (i < (int)blockIdx.x) rb += r, pb += q;
                rows += r, pairs += q;
            }
        }
        row_pre[g] = rb, pair_pre[g] = pb;
        row_off[g] = rows, pair_off[g] = pairs;  // totals; made exclusive below
        if (blockIdx.x == 0 && g < G) counts[2 * g] = rows, counts[2 * g + 1] = pairs;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int r = 0, q = 0;
        for (int g = 0; g < kEpMaxRanks; g++) {
            const int tr = row_off[g], tq = pair_off[g];
            row_off[g] = r, pair_off[g] = q;
            r += tr, q += tq;
        }
    }
    const int t = blockIdx.x * kPlanThreads + (int)threadIdx.x;
    const int E = per_rank * G;
    const bool str = strided != 0;
    uint64_t v[4] = {0, 0, 0, 0};
    unsigned hit = 0;
    if (t < T) hit = token_dests(idx, t, K, E, per_rank, G, str, v, nullptr);
    const uint64_t own[4] = {v[0], v[1], v[2], v[3]};
    uint64_t total[4];
    block_scan4(v, total, warp_sums);  // its barriers also publish row_off / pair_off
    if (t >= T) return;
    uint64_t ex[4];
#pragma unroll
    for (int i = 0; i < 4; i++) ex[i] = v[i] - own[i];
#pragma unroll
    for (int g = 0; g < kEpMaxRanks; g++)
        if (g < G && ((hit >> g) & 1u)) send_rows[row_off[g] + row_pre[g] + field(ex, 2 * g)] = t;
    uint64_t seen = 0;  // 8-bit fields: this token's pairs to each rank so far
    for (int j = 0; j < K; j++) {
        const int e = __ldg(idx + (size_t)t * K + j);
        const int g = dest_of((unsigned)e >= (unsigned)E ? 0 : e, per_rank, G, str);
        const int c = (int)((seen >> (8 * g)) & 0xffu);
        seen += 1ull << (8 * g);
        const int pos = pair_off[g] + pair_pre[g] + field(ex, 2 * g + 1) + c;
        y_pos[(size_t)t * K + j] = pos;
        pair_meta[pos] = make_int2(row_pre[g] + field(ex, 2 * g), e);
    }
}

// The send buffers of one rank: rec[i] = the Q8_0 row of token send_rows[i]
// (dim int8 values, then its f32 block scales), and each pair record with
// its row renumbered in the receiver's buffer, where the rows of lower
// ranks come first: row + sum over ranks s < me of counts[s][g].rows.
// all_counts [G][G][2] is every rank's counts (all-gathered).
__global__ void k_ep_pack(const int8_t *xq, const float *dx, int d, int xs,
                          const int32_t *send_rows, int n_rows, const int2 *pair_meta, int n_pairs,
                          const long long *all_counts, int me, int G, uint8_t *rec, int2 *meta_out,
                          int row_blocks) {
    if ((int)blockIdx.x < row_blocks) {
        const int vq = d / 16, vpr = vq + xs / 4;  // 16-byte vectors a record
        const long nv = (long)n_rows * vpr;
        for (long v = (long)blockIdx.x * blockDim.x + threadIdx.x; v < nv;
             v += (long)row_blocks * blockDim.x) {
            const int i = (int)(v / vpr), k = (int)(v % vpr);
            const int t = __ldg(send_rows + i);
            const uint4 *src = k < vq ? reinterpret_cast<const uint4 *>(xq + (size_t)t * d) + k
                                      : reinterpret_cast<const uint4 *>(dx + (size_t)t * xs) + (k - vq);
            reinterpret_cast<uint4 *>(rec + (size_t)i * (d + 4 * xs))[k] = __ldg(src);
        }
        return;
    }
    const int i = (int)(blockIdx.x - row_blocks) * blockDim.x + threadIdx.x;
    if (i >= n_pairs) return;
    int g = 0, q = 0;
    for (; g < G - 1; g++) {  // destination of record i: this rank's pair counts in order
        q += (int)all_counts[2 * (me * G + g) + 1];
        if (i < q) break;
    }
    int start = 0;
    for (int s = 0; s < me; s++) start += (int)all_counts[2 * (s * G + g)];
    const int2 m = pair_meta[i];
    meta_out[i] = make_int2(m.x + start, m.y);
}

// A rank that received no pairs runs no down launch: it still tells every
// rank that it has stored all it had for them (one thread).
__global__ void k_ep_signal(YRoute yr) {
    __threadfence_system();
    for (int r = 0; r < yr.n; r++) st_release_sys(yr.flags[r] + yr.me, yr.seq);
}

// Waits until every rank's flag here has reached seq: then every y row that
// the ranks' down launches stored for this rank has landed.  One lane per
// rank; gives up after timeout_ns (the error word says so) rather than spin
// on a rank that will never signal.
__global__ void k_ep_wait(const unsigned *flags, int n_ranks, unsigned seq, long long timeout_ns,
                          int *err) {
    const int r = threadIdx.x;
    if (r >= n_ranks) return;
    const unsigned long long t0 = global_ns();
    while ((int)(ld_acquire_sys(flags + r) - seq) < 0) {
        if ((long long)(global_ns() - t0) > timeout_ns) {
            set_error(err, kErrWaitPeer);
            return;
        }
        __nanosleep(200);
    }
}

}  // namespace

void launch_ep_signal(const YRoute &yr, cudaStream_t s) { k_ep_signal<<<1, 1, 0, s>>>(yr); }

void launch_ep_wait(const unsigned *flags, int n_ranks, unsigned seq, long long timeout_ns,
                    int *err, cudaStream_t s) {
    k_ep_wait<<<1, 32, 0, s>>>(flags, n_ranks, seq, timeout_ns, err);
}

int ep_plan_tiles(int T) { return (T + kPlanThreads - 1) / kPlanThreads; }

void launch_ep_plan(const int32_t *idx, int T, int K, int G, int per_rank, bool strided,
                    int *tiles, long long *counts, int32_t *send_rows, int32_t *pair_meta,
                    int32_t *y_pos, int *err, cudaStream_t s) {
    const int n = std::max(1, ep_plan_tiles(T));  // one CTA even for no tokens: it writes counts
    k_ep_count<<<n, kPlanThreads, 0, s>>>(idx, T, K, G, per_rank, strided ? 1 : 0, tiles, err);
    k_ep_place<<<n, kPlanThreads, 0, s>>>(idx, T, K, G, per_rank, strided ? 1 : 0, tiles, n,
                                          counts, send_rows, reinterpret_cast<int2 *>(pair_meta),
                                          y_pos);
}

void launch_ep_pack(const int8_t *xq, const float *dx, int d, int xs, const int32_t *send_rows,
                    int n_rows, const int32_t *pair_meta, int n_pairs, const long long *all_counts,
                    int me, int G, uint8_t *rec, int32_t *meta_out, int num_sms, cudaStream_t s) {
    const long nv = (long)n_rows * (d / 16 + xs / 4);
    const int row_blocks = n_rows > 0 ? (int)std::min<long>((nv + 255) / 256, 4L * num_sms) : 0;
    const int meta_blocks = (n_pairs + 255) / 256;
    if (row_blocks + meta_blocks == 0) return;
    k_ep_pack<<<row_blocks + meta_blocks, 256, 0, s>>>(
        xq, dx, d, xs, send_rows, n_rows, reinterpret_cast<const int2 *>(pair_meta), n_pairs,
        all_counts, me, G, rec, reinterpret_cast<int2 *>(meta_out), row_blocks);
}

}  // namespace miag
