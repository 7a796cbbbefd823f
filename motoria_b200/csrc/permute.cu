// permute.cu -- canonical dispatch order of (token, slot) pairs.
//
// The reference runs one token at a time and has no permutation
// (src/model/forward.c:183-195 loops over the token's own top-k).  Batching
// tokens needs one: pairs p = t*K + j are stably sorted by expert, so within
// an expert they stay in (t, j) order.  Deterministic: no order-dependent
// atomics; ranks come from warp match masks and per-warp prefix counts.
//
// The top-k indices come from the router kernel (route.cu).
// Small batches (T*K <= 1024 pairs), one CTA of 1024 threads:
//   k_permute_small  ranks, counts, offsets, active list and scatter
// Larger batches:
//   k_perm_count   per chunk of 1024 pairs: stable rank of each pair among
//                  the chunk's pairs of the same expert, and chunk histograms
//   k_perm_scan    per expert: chunk bases, counts, offsets, active list
//   k_perm_scatter perm[pos] = p, inv[p] = pos
#include "kernels.cuh"

namespace miag {

constexpr int kPermThreads = 256;
constexpr int kPermWarps = kPermThreads / 32;

__global__ void __launch_bounds__(kPermThreads)
k_perm_count(const int32_t *idx, int P, int E, int32_t *rank, int32_t *chunk_cnt, int *err) {
    pdl_wait();
    pdl_launch_dependents();
    extern __shared__ int32_t sh[];  // cnt[E], wcnt[kPermWarps][E]
    int32_t *cnt = sh;
    int32_t *wcnt = sh + E;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int base = blockIdx.x * kPermChunk;
    for (int e = tid; e < E; e += kPermThreads) cnt[e] = 0;
    for (int sub = 0; sub < kPermChunk; sub += kPermThreads) {
        for (int i = tid; i < kPermWarps * E; i += kPermThreads) wcnt[i] = 0;
        __syncthreads();
        const int p = base + sub + tid;
        int e = -1;
        if (p < P) {
            e = idx[p];
            if (e < 0 || e >= E) {
                set_error(err, kErrBadExpert);
                e = -1;
            }
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int lr = __popc(peers & ((1u << lane) - 1u));
        if (e >= 0 && lr == 0) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        for (int x = tid; x < E; x += kPermThreads) {
            int run = cnt[x];
            for (int w = 0; w < kPermWarps; w++) {
                int c = wcnt[w * E + x];
                wcnt[w * E + x] = run;
                run += c;
            }
            cnt[x] = run;
        }
        __syncthreads();
        if (e >= 0) rank[p] = wcnt[warp * E + e] + lr;
        __syncthreads();
    }
    for (int e = tid; e < E; e += kPermThreads) chunk_cnt[(size_t)blockIdx.x * E + e] = cnt[e];
}

// Exclusive block scan of one value per thread (blockDim.x <= 1024).
__device__ int block_excl_scan(int v, int *total, int *sh /* >= 33 ints */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) sh[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int nw = (blockDim.x + 31) >> 5;
        int s = lane < nw ? sh[lane] : 0;
        int si = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int n = __shfl_up_sync(0xffffffffu, si, o);
            if (lane >= o) si += n;
        }
        sh[lane] = si - s;
        if (lane == 31) sh[32] = si;
    }
    __syncthreads();
    int r = sh[warp] + incl - v;
    *total = sh[32];
    __syncthreads();
    return r;
}

// The pair chunks of one active expert (n pairs from sorted position off),
// numbered from cpos in the list the expert launches walk: (e, chunk, first
// sorted position of the expert, pairs in the chunk); each chunk's
// completion counter (gate/up tiles done) starts at zero, and its first row
// in the pair-tile buffers is brow0 (the expert's, the sum of the earlier
// experts' pairs each rounded up to 16) plus the chunks before it (chunk is
// a multiple of 16, so only an expert's last chunk is ragged).  Workspaces
// without pair tiles pass no chunk_brow.
__device__ __forceinline__ void write_chunks(int4 *chunk_info, int32_t *chunk_done,
                                             int32_t *chunk_brow, int cpos, int e, int off, int n,
                                             int chunk, int brow0) {
    for (int tc = 0; tc * chunk < n; tc++) {
        chunk_info[cpos + tc] = make_int4(e, tc, off, min(chunk, n - tc * chunk));
        chunk_done[cpos + tc] = 0;
        if (chunk_brow) chunk_brow[cpos + tc] = brow0 + tc * chunk;
    }
}

__global__ void __launch_bounds__(1024)
k_perm_scan(int nchunks, int E, const int32_t *chunk_cnt, int32_t *chunk_base, int32_t *counts,
            int32_t *offsets, int32_t *active, int32_t *n_active, int32_t *chunk_pre,
            int4 *chunk_info, int32_t *chunk_done, int32_t *chunk_brow, int32_t *max_chunk,
            int chunk) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ int sh[33];
    __shared__ int smax;
    const int e = threadIdx.x;
    int run = 0;
    if (e < E) {
        for (int c = 0; c < nchunks; c++) {
            int v = chunk_cnt[(size_t)c * E + e];
            chunk_base[(size_t)c * E + e] = run;
            run += v;
        }
        counts[e] = run;
    }
    int total;
    const int off = block_excl_scan(e < E ? run : 0, &total, sh);
    int nact, nchk;
    const int apos = block_excl_scan((e < E && run > 0) ? 1 : 0, &nact, sh);
    const int cpos = block_excl_scan(e < E ? (run + chunk - 1) / chunk : 0, &nchk, sh);
    int nrow;
    const int brow = block_excl_scan(e < E ? (run + 15) & ~15 : 0, &nrow, sh);
    if (e == 0) smax = 0;
    __syncthreads();
    if (e < E) {
        offsets[e] = off;
        if (run > 0) {
            active[apos] = e;
            chunk_pre[apos] = cpos;
            write_chunks(chunk_info, chunk_done, chunk_brow, cpos, e, off, run, chunk, brow);
            atomicMax(&smax, min(chunk, run));
        }
        for (int c = 0; c < nchunks; c++) chunk_base[(size_t)c * E + e] += off;
    }
    __syncthreads();
    if (e == 0) {
        offsets[E] = total;
        *n_active = nact;
        chunk_pre[nact] = nchk;
        *max_chunk = smax;
    }
}

__global__ void k_perm_scatter(const int32_t *idx, int P, int E, const int32_t *rank,
                               const int32_t *chunk_base, int32_t *perm, int32_t *inv) {
    pdl_wait();
    pdl_launch_dependents();
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= P) return;
    const int e = idx[p];
    if (e < 0 || e >= E) return;
    const int pos = chunk_base[(size_t)(p / kPermChunk) * E + e] + rank[p];
    perm[pos] = p;
    inv[p] = pos;
}

// Exclusive block scan of one 64-bit value per thread (blockDim.x <= 1024).
__device__ long long block_excl_scan64(long long v, long long *total, long long *sh /* >= 33 */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    long long incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) sh[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int nw = (blockDim.x + 31) >> 5;
        const long long s = lane < nw ? sh[lane] : 0;
        long long si = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long n = __shfl_up_sync(0xffffffffu, si, o);
            if (lane >= o) si += n;
        }
        sh[lane] = si - s;
        if (lane == 31) sh[32] = si;
    }
    __syncthreads();
    const long long r = sh[warp] + incl - v;
    *total = sh[32];
    __syncthreads();
    return r;
}

// Everything between the top-k and the expert products, for at most 1024
// pairs, in one CTA of max(P, E) threads rounded to warps (one pair each;
// thread e < E also owns expert e).
__global__ void __launch_bounds__(1024)
k_permute_small(const int32_t *idx, int P, int E, int32_t *counts, int32_t *offsets,
                int32_t *active, int32_t *n_active, int32_t *chunk_pre, int4 *chunk_info,
                int32_t *chunk_done, int32_t *chunk_brow, int32_t *max_chunk, int chunk,
                int32_t *perm, int32_t *inv, int *err) {
    pdl_wait();
    pdl_launch_dependents();
    extern __shared__ int32_t sm_i[];  // wcnt [warps][E], base [E]
    __shared__ long long sh[33];
    __shared__ int smax;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    int32_t *wcnt = sm_i;
    int32_t *base = wcnt + nw * E;
    for (int i = tid; i < nw * E; i += blockDim.x) wcnt[i] = 0;
    if (tid == 0) smax = 0;
    __syncthreads();
    const int p = tid;
    int e = -1;
    if (p < P) {
        e = idx[p];
        if (e < 0 || e >= E) {
            set_error(err, kErrBadExpert);
            e = -1;
        }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int lr = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && lr == 0) wcnt[warp * E + e] = __popc(peers);
    __syncthreads();
    int run = 0;
    if (tid < E) {
        for (int ww = 0; ww < nw; ww++) {
            const int c = wcnt[ww * E + tid];
            wcnt[ww * E + tid] = run;
            run += c;
        }
        counts[tid] = run;
    }
    // the three scans at once, in 21-bit fields (each total is at most
    // P + E + P / chunk < 2^21): pairs, active experts, chunks
    constexpr long long kF = (1ll << 21) - 1;
    const long long v = tid < E ? (long long)run | ((long long)(run > 0) << 21) |
                                      ((long long)((run + chunk - 1) / chunk) << 42)
                                : 0ll;
    long long tot;
    const long long ex = block_excl_scan64(v, &tot, sh);
    const int off = (int)(ex & kF), apos = (int)((ex >> 21) & kF), cpos = (int)(ex >> 42);
    const int total = (int)(tot & kF), nact = (int)((tot >> 21) & kF), nchk = (int)(tot >> 42);
    long long nrow;
    const int brow = (int)block_excl_scan64(tid < E ? (long long)((run + 15) & ~15) : 0ll, &nrow, sh);
    if (tid < E) {
        offsets[tid] = off;
        base[tid] = off;
        if (run > 0) {
            active[apos] = tid;
            chunk_pre[apos] = cpos;
            write_chunks(chunk_info, chunk_done, chunk_brow, cpos, tid, off, run, chunk, brow);
            atomicMax(&smax, min(chunk, run));
        }
    }
    __syncthreads();
    if (tid == 0) {
        offsets[E] = total;
        *n_active = nact;
        chunk_pre[nact] = nchk;
        *max_chunk = smax;
    }
    if (e >= 0) {
        const int pos = base[e] + wcnt[warp * E + e] + lr;
        perm[pos] = p;
        inv[p] = pos;
    }
}

void launch_permute(const Dims &m, const Work &w, int *err, cudaStream_t s) {
    const int P = w.P, E = m.E;
    const int chunk = w.chunk > 0 ? w.chunk : tok_chunk(P, E);
    const int threads = ((P > E ? P : E) + 31) / 32 * 32;
    const size_t small_smem = (size_t)(threads / 32 * E) * 4 + (size_t)E * 4;
    if (P <= kPermChunk && E <= 1024 && small_smem <= 200 * 1024) {
        cudaFuncSetAttribute(k_permute_small, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)small_smem);
        launch_dependent(k_permute_small, dim3(1), dim3(threads), small_smem, s, w.idx, P, E, w.counts,
                         w.offsets, w.active, w.n_active, w.chunk_pre, w.chunk_info, w.chunk_done,
                         w.chunk_brow, w.max_chunk, chunk, w.perm, w.inv, err);
        return;
    }
    const size_t smem = sizeof(int32_t) * (size_t)E * (1 + kPermWarps);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(k_perm_count, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_dependent(k_perm_count, dim3(w.nchunks), dim3(kPermThreads), smem, s, w.idx, P, E, w.rank,
                     w.chunk_cnt, err);
    const int st = ((E + 31) / 32) * 32;
    launch_dependent(k_perm_scan, dim3(1), dim3(st < 64 ? 64 : st), 0, s, w.nchunks, E, w.chunk_cnt,
                     w.chunk_base, w.counts, w.offsets, w.active, w.n_active, w.chunk_pre,
                     w.chunk_info, w.chunk_done, w.chunk_brow, w.max_chunk, chunk);
    launch_dependent(k_perm_scatter, dim3((P + 255) / 256), dim3(256), 0, s, w.idx, P, E, w.rank,
                     w.chunk_base, w.perm, w.inv);
}

int permute_launches(int P, int E) {
    const int threads = ((P > E ? P : E) + 31) / 32 * 32;
    return (P <= kPermChunk && E <= 1024 && (size_t)(threads / 32 * E) * 4 + (size_t)E * 4 <= 200 * 1024)
               ? 1
               : 3;
}

}  // namespace miag
