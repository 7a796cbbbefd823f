// Expert parallelism: the dispatch plan and the send records of one rank.
//
// Under expert parallelism each rank routes its own tokens and sends every
// token row once to each rank that holds one of its top-k experts, with one
// (row, expert) record per (token, expert) pair; the expert products come
// back one f32 row per pair and are combined in top-k order, so the results
// equal the one-device block (src/model/forward.c:167-197) bit for bit.
// The reference has no multi-device path; these two kernels compute the
// plan of motoria_b200/ep.py:plan_dispatch and the records it sends, so
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

constexpr int kPlanThreads = 1024;  // one CTA: the plan is a few hundred KB of indices

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

__global__ void __launch_bounds__(kPlanThreads, 1)
    k_ep_plan(const int32_t *idx, int T, int K, int G, int per_rank, int strided,
              long long *counts, int32_t *send_rows, int2 *pair_meta, int32_t *y_pos, int *err) {
    __shared__ int tot_rows[kEpMaxRanks], tot_pairs[kEpMaxRanks];
    __shared__ int row_off[kEpMaxRanks], pair_off[kEpMaxRanks];  // where each block starts
    __shared__ int run_rows[kEpMaxRanks], run_pairs[kEpMaxRanks];  // in earlier tiles
    __shared__ uint64_t warp_sums[32][4];
    const int E = per_rank * G;
    const bool str = strided != 0;
    if (threadIdx.x < kEpMaxRanks) {
        tot_rows[threadIdx.x] = tot_pairs[threadIdx.x] = 0;
        run_rows[threadIdx.x] = run_pairs[threadIdx.x] = 0;
    }
    __syncthreads();

    // pass 1: rows and pairs to each destination
    {
        int rows[kEpMaxRanks], pairs[kEpMaxRanks];
#pragma unroll
        for (int g = 0; g < kEpMaxRanks; g++) rows[g] = pairs[g] = 0;
        for (int t = threadIdx.x; t < T; t += kPlanThreads) {
            unsigned hit = 0;
            for (int j = 0; j < K; j++) {
                int e = __ldg(idx + (size_t)t * K + j);
                if ((unsigned)e >= (unsigned)E) set_error(err, kErrBadExpert), e = 0;
                const int g = dest_of(e, per_rank, G, str);
                hit |= 1u << g;
#pragma unroll
                for (int gg = 0; gg < kEpMaxRanks; gg++) pairs[gg] += gg == g;
            }
#pragma unroll
            for (int gg = 0; gg < kEpMaxRanks; gg++) rows[gg] += (hit >> gg) & 1u;
        }
#pragma unroll
        for (int g = 0; g < kEpMaxRanks; g++) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                rows[g] += __shfl_xor_sync(0xffffffffu, rows[g], o);
                pairs[g] += __shfl_xor_sync(0xffffffffu, pairs[g], o);
            }
        }
        if ((threadIdx.x & 31) == 0) {
#pragma unroll
            for (int g = 0; g < kEpMaxRanks; g++)
                if (g < G) atomicAdd(&tot_rows[g], rows[g]), atomicAdd(&tot_pairs[g], pairs[g]);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int r = 0, q = 0;
        for (int g = 0; g < G; g++) {
            row_off[g] = r, pair_off[g] = q;
            counts[2 * g] = tot_rows[g], counts[2 * g + 1] = tot_pairs[g];
            r += tot_rows[g], q += tot_pairs[g];
        }
    }
    __syncthreads();

    // pass 2: each token's rows and pairs at their places, a tile at a time
    for (int base = 0; base < T; base += kPlanThreads) {
        const int t = base + (int)threadIdx.x;
        uint64_t v[4] = {0, 0, 0, 0};
        unsigned hit = 0;
        if (t < T) {
            for (int j = 0; j < K; j++) {
                int e = __ldg(idx + (size_t)t * K + j);
                if ((unsigned)e >= (unsigned)E) e = 0;
                const int g = dest_of(e, per_rank, G, str);
                hit |= 1u << g;
                add_field(v, 2 * g + 1);
            }
#pragma unroll
            for (int g = 0; g < kEpMaxRanks; g++)
                if ((hit >> g) & 1u) add_field(v, 2 * g);
        }
        const uint64_t own[4] = {v[0], v[1], v[2], v[3]};
        uint64_t total[4];
        block_scan4(v, total, warp_sums);
        if (t < T) {
            // exclusive prefixes: the token's row within each destination's
            // block, and the place of its first pair to each destination
            uint64_t ex[4];
#pragma unroll
            for (int i = 0; i < 4; i++) ex[i] = v[i] - own[i];
            int row_in[kEpMaxRanks], next[kEpMaxRanks];
#pragma unroll
            for (int g = 0; g < kEpMaxRanks; g++) {
                const bool live = g < G;
                row_in[g] = live ? run_rows[g] + field(ex, 2 * g) : 0;
                next[g] = live ? pair_off[g] + run_pairs[g] + field(ex, 2 * g + 1) : 0;
                if (live && ((hit >> g) & 1u)) send_rows[row_off[g] + row_in[g]] = t;
            }
            for (int j = 0; j < K; j++) {
                const int e = __ldg(idx + (size_t)t * K + j);
                const int g = dest_of((unsigned)e >= (unsigned)E ? 0 : e, per_rank, G, str);
                int pos = 0, row = 0;
#pragma unroll
                for (int gg = 0; gg < kEpMaxRanks; gg++)
                    if (gg == g) pos = next[gg]++, row = row_in[gg];
                y_pos[(size_t)t * K + j] = pos;
                pair_meta[pos] = make_int2(row, e);
            }
        }
        __syncthreads();  // every thread has read run_rows / run_pairs
        if (threadIdx.x < kEpMaxRanks && (int)threadIdx.x < G) {
            run_rows[threadIdx.x] += field(total, 2 * threadIdx.x);
            run_pairs[threadIdx.x] += field(total, 2 * threadIdx.x + 1);
        }
        __syncthreads();
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

void launch_ep_plan(const int32_t *idx, int T, int K, int G, int per_rank, bool strided,
                    long long *counts, int32_t *send_rows, int32_t *pair_meta, int32_t *y_pos,
                    int *err, cudaStream_t s) {
    k_ep_plan<<<1, kPlanThreads, 0, s>>>(idx, T, K, G, per_rank, strided ? 1 : 0, counts, send_rows,
                                         reinterpret_cast<int2 *>(pair_meta), y_pos, err);
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
