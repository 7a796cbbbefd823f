// tc.cu -- the prefill-regime expert products on the 5th-generation tensor
// cores (tcgen05): gate+up and down for batches with more than 8 pairs per
// expert on average (configs 3 and 5, and every expert-parallel step).
//
// Reference: the three mia_matvec calls per active expert in moe()
// (src/model/forward.c:186-193) -> rows_kernel (src/tensor/matmul.c:75-80)
// -> dot_q8_scalar (:19-28), SwiGLU :188-191 and the re-quantization of h
// inside mia_matvec (:93, quant.c:11-27).
//
// The reference's Q8_0 dot is, per (row, pair),
//     s = 0;  for each 32-block b in order:  s = s + ((float)dot_b * w.d_b) * x.d_b
// with dot_b the exact int32 dot of the block's int8 values.  The tensor cores
// compute every dot_b exactly (tcgen05.mma kind::i8, K = 32 = one block, one
// MMA per block into its own tensor-memory columns); the FP32 steps, each
// rounded on its own and in block order, run on the CUDA cores.  Those steps
// are the bound (four FP32 operations per (row, pair, block) against 64 int8
// MACs of tensor work), so the kernel is organised around keeping the FP32
// pipes busy:
//
//   warp 0       copies: per stage, two k tiles of the expert's weight tile
//                (the store's 18 KiB units, swizzled int8 + scales, one bulk
//                copy) and the same two k tiles of the chunk's activations
//                (pair tiles laid out by k_tc_gather / k_tc_swiglu, one bulk
//                copy), into a ring of 3 stages;
//   warp 1       allocates 512 tensor-memory columns; one thread issues the
//                MMAs: M = 128 weight rows, N = the chunk's pairs rounded up
//                to 16 (at most 128), K = 32, block j of a k tile into
//                buffer j % 4 (128 columns each), each committed to its own
//                barrier;
//   warps 2-17   epilogue, four warpgroups, one weight row per thread (the
//                row's tensor-memory lane); warpgroup h owns the pair groups
//                g = h and h+4 (16 pairs each).  Per block it loads its dots
//                (tcgen05.ld), writes the magic constant back so the next
//                MMA into the buffer accumulates onto it, releases the
//                buffer, and applies the reference's step to 32 accumulators
//                held in registers, two pairs per packed FP32 instruction.
//                Four epilogue warps per scheduler keep the FP32 pipe fed
//                across the steps' fixed latencies.
//
// The MMA accumulates onto kMagicBits (the bits of 1.5 * 2^23): |dot| < 2^22,
// so the int32 result read as a float is exactly 12582912 + dot and one exact
// subtraction gives (float)dot on the FMA pipe (the same trick as the decode
// kernels' mma.sync).  The buffers are filled with it once at the start;
// afterwards every column an MMA wrote is reset by the warp that read it.
//
// Work items are (expert, 128-row tile, chunk of up to 128 pairs), ordered
// expert-major, then row tile, then chunk.  One CTA per SM takes them in
// order from a counter (items differ in cost: an expert's last chunk is
// ragged), so the items running at any moment are neighbours in the list:
// the CTAs that run the chunks of one (expert, row tile) stream the same
// weight tiles, which cross HBM once and come from L2 for the others;
// activations (a few MB) stay in L2.
#include "kernels.cuh"

namespace miag {

namespace {

constexpr int kTcEpiWG = 4;                        // epilogue warpgroups (two 16-pair groups each)
constexpr int kTcEpiWarps = 4 * kTcEpiWG;
constexpr int kTcThreads = 64 + 32 * kTcEpiWarps;  // warp 0 copies, warp 1 MMAs, warps 2-17 epilogue
constexpr int kTcQueue = 4;                        // items in flight between the roles
constexpr int kTcStages = 3;
constexpr int kTcPairRowBytes = 144;                     // per pair and k tile: 128 int8 + 4 f32
constexpr int kTcStageA = 2 * kUnitBytes;                // two k tiles of weights, scales included
constexpr int kTcStageB = 2 * kTcChunk * kTcPairRowBytes;  // two k tiles of up to 128 pairs
constexpr int kTcStageBytes = kTcStageA + kTcStageB;
constexpr int kTcTmemBufs = 4;     // one Q8_0 block's dots each
constexpr int kTcBufCols = 128;    // columns per buffer (up to 128 pairs)
constexpr int kTcTmemCols = kTcTmemBufs * kTcBufCols;
constexpr int kTcHeadBytes = 1024;
constexpr int kTcSmemBytes = kTcStages * kTcStageBytes + kTcHeadBytes;

struct TcHead {
    uint64_t full[kTcStages];     // stage landed (bulk copies, complete_tx)
    uint64_t empty[kTcStages];    // stage free: its MMAs done (commit) and 8 epilogue warps
    uint64_t tfull[kTcTmemBufs];  // buffer holds a block's dots (commit)
    uint64_t tempty[kTcTmemBufs]; // buffer read and reset by the 8 epilogue warps
    uint64_t qfull[kTcQueue];     // item queue: index written (producer)
    uint64_t qempty[kTcQueue];    // item queue: read by the MMA thread and the epilogue warps
    uint64_t mma_done;            // the last MMAs of the CTA have completed
    uint32_t tmem_base;
    int copies;                   // stages the producer filled
    int item_q[kTcQueue];
};
static_assert(sizeof(TcHead) <= kTcHeadBytes, "tc head");

struct TcParams {
    int d, eh, E, K;
    int RT, KT, rows;            // row tiles, k tiles, matrix rows
    size_t expert_bytes;
    const uint8_t *weights;      // this matrix (gate/up or down) of expert 0
    const int32_t *n_active, *chunk_pre, *chunk_brow, *perm;
    const int4 *chunk_info;      // (expert, chunk of it, expert's first sorted position, pairs)
    const uint8_t *tiles;        // the pair tiles (bx or bh)
    float *h;                    // gate/up: [P][2 eh] products, sorted order
    float *y;                    // down: [P][d], pair order
    YRoute yr;                   // down under expert parallelism: rows at their origin ranks
    float one;                   // 1.0f, opaque to the compiler (see q8_step_x2)
    int *sched;                  // [2] items taken, CTAs done: zero between launches
    int *err;
};

// ---- tcgen05 wrappers (cta_group::1; every address is this CTA's own)

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory descriptor of a K-major operand in the 128-byte swizzle:
// 8-row atoms of 8 x 128 B, 1024 B apart (stride byte offset); the leading
// byte offset is unused for this layout; version 1 (bits 46-47); layout
// type 2 = SWIZZLE_128B (bits 61-63).  A start inside the atom's row (the
// 32-byte block j of a k tile) is the tile's address + 32 j.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;               // leading byte offset (unused), 16 B
    d |= (uint64_t)(1024 >> 4) << 32;     // stride byte offset
    d |= (uint64_t)1 << 46;               // version
    d |= (uint64_t)2 << 61;               // SWIZZLE_128B
    return d;
}

// Instruction descriptor of kind::i8: D s32 (bits 4-5 = 2), A and B signed
// 8-bit (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at 24.
__device__ __forceinline__ uint32_t i8_idesc(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, one thread.
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 lanes x 16 columns of 32 bits: lane i of the warp gets its TMEM lane's
// 16 consecutive columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// The reference step s = s + ((float)dot * w.d) * x.d (matmul.c:25) for the
// 16 pairs of a group: dots d as returned by kind::i8 (int32 bits), the
// weight row's block scale w, the pairs' activation scales at shared address
// xs ([16] f32).  (float)dot is exact: the bits of dot + 0x4B400000 read as a
// float are 12582912 + dot (|dot| < 2^22), and subtracting 12582912 is exact.
// Every operation is rounded on its own, as in the reference.
__device__ __forceinline__ void q8_steps16(float (&acc)[16], const uint32_t (&d)[16], float w,
                                           uint32_t xs) {
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
        const float4 x4 = lds128(xs + (uint32_t)(4 * k));
        const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const float f = __fadd_rn(__uint_as_float(d[k + u] + (uint32_t)kMagicBits), -kMagic);
            acc[k + u] = __fadd_rn(acc[k + u], __fmul_rn(__fmul_rn(f, w), xv[u]));
        }
    }
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- items

struct TcItem {
    int e, rt, k;   // expert, row tile, chunk of the expert
    int pos0;       // sorted position of the chunk's first pair
    int n, Nc;      // pairs, and the MMA's N (pairs rounded up to 16)
    int brow;       // first row of the chunk in the pair tiles
};

// Item i: items are (expert, row tile, chunk), experts ascending (active
// ones), then row tiles, then chunks.  chunk_pre[a] counts the chunks of the
// active experts before a.
__device__ __forceinline__ TcItem tc_item(const TcParams &p, int n_act, int i) {
    const int ci = i / p.RT;
    int lo = 0, hi = n_act;  // chunk_pre[lo] <= ci < chunk_pre[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (__ldcg(p.chunk_pre + mid) <= ci) lo = mid;
        else hi = mid;
    }
    const int c0 = __ldcg(p.chunk_pre + lo), nch = __ldcg(p.chunk_pre + lo + 1) - c0;
    const int rem = i - c0 * p.RT;
    TcItem it;
    it.rt = rem / nch;
    it.k = rem - it.rt * nch;
    const int4 info = __ldcg(p.chunk_info + c0 + it.k);
    it.e = info.x;
    it.pos0 = info.z + info.y * kTcChunk;
    it.n = info.w;
    it.Nc = (info.w + 15) & ~15;
    it.brow = __ldcg(p.chunk_brow + c0 + it.k);
    return it;
}

// Pair-tile layout (written by k_tc_gather / k_tc_swiglu, read by one bulk
// copy per stage): a chunk of Nc rows (pairs) occupies KT * 144 * Nc bytes
// from byte brow * KT * 144.  Stage ks (k tiles 2ks, 2ks+1) is 288 * Nc
// bytes at ks * 288 * Nc: the two int8 tiles (Nc rows x 128 B each, the
// 128-byte swizzle of the weight tiles, rows 16 B chunk c at c ^ (r % 8)),
// then the two scale blocks, [4 Q8_0 blocks][Nc] f32 each.
__host__ __device__ __forceinline__ size_t tc_chunk_off(int brow, int KT) {
    return (size_t)brow * KT * kTcPairRowBytes;
}
__host__ __device__ __forceinline__ uint32_t tc_tile_off(int Nc, int kt) {
    return (uint32_t)((kt >> 1) * 2 * kTcPairRowBytes * Nc + (kt & 1) * kTileK * Nc);
}
__host__ __device__ __forceinline__ uint32_t tc_scale_off(int Nc, int kt, int j, int r) {
    return (uint32_t)((kt >> 1) * 2 * kTcPairRowBytes * Nc + 2 * kTileK * Nc + (kt & 1) * 16 * Nc +
                      (j * Nc + r) * 4);
}

template <bool kGU>
__global__ void __launch_bounds__(kTcThreads, 1) k_expert_tc(TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    TcHead *hd = reinterpret_cast<TcHead *>(smem + kTcStages * kTcStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // The hardware swizzle of the operands follows the shared-memory address
    // bits: the stages must start on a 1024-byte boundary.
    const bool aligned = (smem_addr(smem) & 1023u) == 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; s++) {
            mbar_init(&hd->full[s], 1);
            mbar_init(&hd->empty[s], 1 + kTcEpiWarps);
        }
        for (int b = 0; b < kTcTmemBufs; b++) {
            mbar_init(&hd->tfull[b], 1);
            mbar_init(&hd->tempty[b], kTcEpiWarps);
        }
        for (int q = 0; q < kTcQueue; q++) {
            mbar_init(&hd->qfull[q], 1);
            mbar_init(&hd->qempty[q], 1 + kTcEpiWarps);
        }
        mbar_init(&hd->mma_done, 1);
        fence_barrier_init();
        if (!aligned) set_error(p.err, kErrItemList);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&hd->tmem_base)),
                     "r"(kTcTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = hd->tmem_base;

    // Everything below reads the permutation and the pair tiles of the
    // launches before this one.
    pdl_wait();
    pdl_launch_dependents();
    const int n_act = __ldcg(p.n_active);
    const int n_items = aligned ? __ldcg(p.chunk_pre + n_act) * p.RT : 0;
    const int NS = p.KT / 2;  // stages per item
    const uint32_t stage0 = smem_addr(smem);
    bool failed = false;
    int copies = 0;  // stages whose copies this CTA issued (thread 0)

    if (warp == 0) {
        // ---------------- items and copies
        // Items are taken from the launch's counter one ahead of the one
        // being copied, so the atomic's round trip overlaps the copies; each
        // goes to the MMA and epilogue warps through the item queue.  The
        // first index past the list tells them to stop.
        if (lane == 0) {
            int s = 0, q = 0;
            uint32_t ph = 0, qph = 0;
            int cur = atomicAdd(p.sched, 1);
            while (true) {
                const int next = cur < n_items ? atomicAdd(p.sched, 1) : cur;
                if (!failed && !mbar_wait(&hd->qempty[q], qph ^ 1u)) {
                    set_error(p.err, kErrWaitEmpty);
                    failed = true;
                }
                hd->item_q[q] = cur;
                mbar_arrive(&hd->qfull[q]);
                if (++q == kTcQueue) q = 0, qph ^= 1u;
                if (cur >= n_items) break;
                const TcItem it = tc_item(p, n_act, cur);
                const bool ok = (unsigned)it.e < (unsigned)p.E && it.rt < p.RT && it.n > 0 &&
                                it.n <= kTcChunk;
                if (!ok) set_error(p.err, kErrItemList);
                const uint8_t *a_src = p.weights + (size_t)it.e * p.expert_bytes +
                                       (size_t)it.rt * p.KT * kUnitBytes;
                const uint8_t *b_src = p.tiles + tc_chunk_off(it.brow, p.KT);
                const uint32_t b_bytes = (uint32_t)(2 * kTcPairRowBytes * it.Nc);
                for (int ks = 0; ks < NS; ks++) {
                    if (!failed && !mbar_wait(&hd->empty[s], ph ^ 1u)) {
                        set_error(p.err, kErrWaitEmpty);
                        failed = true;
                    }
                    if (ok) {  // a bad entry is never copied: its consumers time out
                        uint8_t *dst = smem + (size_t)s * kTcStageBytes;
                        mbar_arrive_expect_tx(&hd->full[s], kTcStageA + b_bytes);
                        bulk_g2s(dst, a_src + (size_t)ks * kTcStageA, kTcStageA, &hd->full[s]);
                        bulk_g2s(dst + kTcStageA, b_src + (size_t)ks * b_bytes, b_bytes,
                                 &hd->full[s]);
                        copies++;
                    }
                    if (++s == kTcStages) s = 0, ph ^= 1u;
                }
                cur = next;
            }
            hd->copies = copies;
        }
    } else if (warp == 1) {
        // ---------------- MMA issue
        // One thread issues every MMA, so its instruction stream is the
        // critical path: the loop over a stage's 8 blocks is unrolled, the
        // descriptors are the stage's two base descriptors plus compile-time
        // offsets, and block (which, j) always goes to buffer j with barrier
        // parity `which` (8 blocks a stage, 4 buffers: every buffer is used
        // twice a stage).  Measured on B200: an MMA of M = 128, N = 128,
        // K = 32 then issues every 64 cycles (the tensor core's int8 rate);
        // descriptors and buffer indices computed per MMA at run time cost
        // ~500 cycles an MMA, whatever its size.
        if (lane == 0) {
            int s = 0, q = 0;
            uint32_t ph = 0, qph = 0;
            bool any = false;
            while (true) {
                if (!failed && !mbar_wait(&hd->qfull[q], qph)) {
                    set_error(p.err, kErrWaitFull);
                    failed = true;
                }
                const int i = failed ? n_items : hd->item_q[q];
                mbar_arrive(&hd->qempty[q]);
                if (++q == kTcQueue) q = 0, qph ^= 1u;
                if (i >= n_items) break;
                const TcItem it = tc_item(p, n_act, i);
                const int Nc = max(16, min(it.Nc, kTcChunk));
                const uint32_t idesc = i8_idesc(kTileRows, Nc);
                const uint64_t b_step = (uint64_t)((kTileK * Nc) >> 4);  // second k tile of the pairs
                for (int ks = 0; ks < NS; ks++) {
                    if (!failed && !mbar_wait(&hd->full[s], ph)) {
                        set_error(p.err, kErrWaitFull);
                        failed = true;
                    }
                    tc_fence_after();
                    const uint32_t sa = stage0 + (uint32_t)(s * kTcStageBytes);
                    const uint64_t a0 = sw128_desc(sa), b0 = sw128_desc(sa + kTcStageA);
#pragma unroll
                    for (int which = 0; which < 2; which++) {
#pragma unroll
                        for (int j = 0; j < kTcTmemBufs; j++) {
                            // the buffer was read and reset to the magic constant
                            if (!failed && !mbar_wait(&hd->tempty[j], (uint32_t)which)) {
                                set_error(p.err, kErrWaitEmpty);
                                failed = true;
                            }
                            tc_fence_after();
                            mma_i8(tbase + (uint32_t)(j * kTcBufCols),
                                   a0 + (uint64_t)((which * kUnitBytes + 32 * j) >> 4),
                                   b0 + (uint64_t)which * b_step + (uint64_t)(2 * j), idesc, 0u);
                            tc_commit(&hd->tfull[j]);
                            any = true;
                        }
                    }
                    tc_commit(&hd->empty[s]);  // the stage's operands are no longer read
                    if (++s == kTcStages) s = 0, ph ^= 1u;
                }
            }
            // Before the columns are freed, every MMA must have completed.
            if (any) {
                tc_commit(&hd->mma_done);
                if (!mbar_wait(&hd->mma_done, 0)) set_error(p.err, kErrWaitFull);
            }
        }
    } else {
        // ---------------- epilogue: one weight row per thread
        // Warpgroup wg owns the 16-pair groups g0 = wg and g1 = wg + 4 of
        // every item.  Block b of an item (stage b / 8, k tile (b / 4) % 2,
        // Q8_0 block b % 4) is in buffer b % 4 with phase parity (b / 4) % 2;
        // the buffer is released once both groups' dots are in registers.
        // (Loading one group ahead while the other's steps run measured
        // slower: the wait for the next block then comes before the steps
        // that would have given the MMA time to finish it.)
        const int wg = (warp - 2) >> 2;
        const int g0 = wg, g1 = wg + kTcEpiWG;
        const int quarter = warp & 3;           // the TMEM lanes this warp may access
        const int row = quarter * 32 + lane;    // row within the 128-row tile
        const uint32_t trow = tbase + ((uint32_t)(quarter * 32) << 16);
        __syncwarp();
        if (lane == 0)  // every buffer is free at the start
            for (int b = 0; b < kTcTmemBufs; b++) mbar_arrive(&hd->tempty[b]);

        int s = 0, q = 0;
        uint32_t ph = 0, qph = 0;
        while (true) {
            if (!failed && !mbar_wait(&hd->qfull[q], qph)) {
                set_error(p.err, kErrWaitFull);
                failed = true;
            }
            const int i = failed ? n_items : hd->item_q[q];
            __syncwarp();
            if (lane == 0) mbar_arrive(&hd->qempty[q]);
            if (++q == kTcQueue) q = 0, qph ^= 1u;
            if (i >= n_items) break;
            const TcItem it = tc_item(p, n_act, i);
            const int ng = it.Nc >> 4;  // groups of 16 pairs
            const int Nc = it.Nc;
            const bool live0 = g0 < ng, live1 = g1 < ng;
            const int nblk = NS * 8;
            float acc0[16], acc1[16];
#pragma unroll
            for (int k = 0; k < 16; k++) acc0[k] = acc1[k] = 0.0f;
            for (int blk = 0; blk < nblk; blk++) {
                const int j = blk & 3, which = (blk >> 2) & 1;
                if ((blk & 7) == 0 && !failed && !mbar_wait(&hd->full[s], ph)) {
                    set_error(p.err, kErrWaitFull);  // the stage's scales
                    failed = true;
                }
                if (!failed && !mbar_wait(&hd->tfull[j], (uint32_t)which)) {
                    set_error(p.err, kErrWaitFull);
                    failed = true;
                }
                tc_fence_after();
                const uint32_t sa = stage0 + (uint32_t)(s * kTcStageBytes);
                const float wj = lds32(sa + (uint32_t)(which * kUnitBytes + kTileBytes + row * 16 + 4 * j));
                const uint32_t xs = sa + kTcStageA + tc_scale_off(Nc, which, j, 0);
                const uint32_t tb = trow + (uint32_t)(j * kTcBufCols);
                uint32_t d[16];
                if (live0) tmem_ld16(tb + (uint32_t)(16 * g0), d);
                tmem_wait_ld();
                if (live0) q8_steps16(acc0, d, wj, xs + (uint32_t)(64 * g0));
                if (live1) tmem_ld16(tb + (uint32_t)(16 * g1), d);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&hd->tempty[j]);  // the buffer is read
                if (live1) q8_steps16(acc1, d, wj, xs + (uint32_t)(64 * g1));
                if ((blk & 7) == 7) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&hd->empty[s]);  // done with the stage's scales
                    if (++s == kTcStages) s = 0, ph ^= 1u;
                }
            }
            // outputs: row rt*128 + row of every pair of the chunk
            const int R = it.rt * kTileRows + row;
            if (R < p.rows) {
#pragma unroll
                for (int gi = 0; gi < 2; gi++) {
                    const int g = gi ? g1 : g0;
                    if (g < ng) {
#pragma unroll
                        for (int k = 0; k < 16; k++) {
                            const int qa = 16 * g + k;
                            const float v = gi ? acc1[k] : acc0[k];
                            if (qa < it.n) {
                                if (kGU) p.h[(size_t)(it.pos0 + qa) * p.rows + R] = v;
                                else y_route_row(p.yr, p.y, p.d, __ldg(p.perm + it.pos0 + qa))[R] = v;
                            }
                        }
                    }
                }
            }
        }
    }
    // After a wait that gave up, copies may still be in flight into the ring:
    // let the last ones land (bounded) before the CTA's shared memory goes.
    if (__syncthreads_or(failed) && threadIdx.x == 0) {
        const int total = hd->copies;
        for (int j = total - 1; j >= 0 && j >= total - kTcStages; j--)
            mbar_wait(&hd->full[j % kTcStages], (uint32_t)((j / kTcStages) & 1));
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase),
                     "r"(kTcTmemCols)
                     : "memory");
    }
    // The launch's item counter back to zero for the next launch: the last
    // CTA to finish resets it (every CTA has taken its last index by now).
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
            p.sched[0] = 0;
            p.sched[1] = 0;
            __threadfence();
        }
    }
    if (!kGU && p.yr.n > 0) ep_signal_done(p.yr);
}

// ---- the pair tiles

struct TcTileParams {
    int d, eh, K, KT, xs, n_rows;
    size_t x_row, dx_row;  // strides of the rows of xq (bytes) and dx (floats)
    const int32_t *n_active, *chunk_pre, *chunk_brow, *perm, *pair_row;
    const int4 *chunk_info;
    const int8_t *xq;      // gate/up: [rows][d]
    const float *dx;       // [rows][xs]
    const float *h;        // down: [P][2 eh] gate/up products, sorted order
    uint8_t *tiles;
    int *err;
};

// gate/up: each chunk's activation rows (the router's Q8_0 xn of the pair's
// token, or the row pair_row names) as pair tiles.  Rows Nc - n of a ragged
// chunk are zero.  One CTA per chunk at a time.
__global__ void __launch_bounds__(256) k_tc_gather(TcTileParams p) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ int tok[kTcChunk];
    const int nchk = __ldcg(p.chunk_pre + __ldcg(p.n_active));
    const int pieces = p.d / 16, nb = p.d / MIAG_QK;
    for (int c = blockIdx.x; c < nchk; c += gridDim.x) {
        const int4 info = __ldcg(p.chunk_info + c);
        const int n = info.w, Nc = (n + 15) & ~15, pos0 = info.z + info.y * kTcChunk;
        uint8_t *dst = p.tiles + tc_chunk_off(__ldcg(p.chunk_brow + c), p.KT);
        __syncthreads();  // the previous chunk's rows are no longer read
        if ((int)threadIdx.x < Nc) {
            int t = -1;
            if ((int)threadIdx.x < n) {
                const int pid = __ldcg(p.perm + pos0 + threadIdx.x);
                t = p.pair_row ? __ldg(p.pair_row + pid) : pid / p.K;
                if (t < 0 || t >= p.n_rows) {
                    set_error(p.err, kErrBadExpert);
                    t = -1;
                }
            }
            tok[threadIdx.x] = t;
        }
        __syncthreads();
        for (int v = threadIdx.x; v < Nc * pieces; v += blockDim.x) {
            const int r = v / pieces, pc = v - r * pieces;
            const int t = tok[r];
            uint4 val = make_uint4(0u, 0u, 0u, 0u);
            if (t >= 0) val = __ldg(reinterpret_cast<const uint4 *>(p.xq + (size_t)t * p.x_row) + pc);
            const int kt = pc >> 3;
            *reinterpret_cast<uint4 *>(dst + tc_tile_off(Nc, kt) + tile_chunk_offset(r, pc & 7)) = val;
        }
        for (int v = threadIdx.x; v < Nc * nb; v += blockDim.x) {
            const int r = v / nb, blk = v - r * nb;
            const int t = tok[r];
            const float sv = t >= 0 ? __ldg(p.dx + (size_t)t * p.dx_row + blk) : 0.0f;
            *reinterpret_cast<float *>(dst + tc_scale_off(Nc, blk >> 2, blk & 3, r)) = sv;
        }
    }
}

// down: h = silu(gate) * up (forward.c:188-191) of every pair, quantized to
// Q8_0 exactly as mia_matvec quantizes its input (matmul.c:93,
// quant.c:11-27), written as pair tiles; the same arithmetic as k_swiglu_q8.
// Four threads per (pair, 32-block), eight values each; the block maximum is
// combined over the four lanes (max is exact in any order).  Grid: (chunk
// slot, slice of the chunk's tasks).
__global__ void __launch_bounds__(256) k_tc_swiglu(TcTileParams p) {
    pdl_wait();
    pdl_launch_dependents();
    const int nchk = __ldcg(p.chunk_pre + __ldcg(p.n_active));
    const int nb = p.eh / MIAG_QK;
    for (int c = blockIdx.x; c < nchk; c += gridDim.x) {
        const int4 info = __ldcg(p.chunk_info + c);
        const int n = info.w, Nc = (n + 15) & ~15, pos0 = info.z + info.y * kTcChunk;
        uint8_t *dst = p.tiles + tc_chunk_off(__ldcg(p.chunk_brow + c), p.KT);
        const int tasks = Nc * nb * 4;
        for (int v0 = blockIdx.y * blockDim.x; v0 < tasks; v0 += gridDim.y * blockDim.x) {
            const int v = v0 + (int)threadIdx.x;
            const bool live = v < tasks;  // whole quads (tasks % 4 == 0)
            const int blkid = live ? v >> 2 : 0, q = v & 3;
            const int r = blkid / nb, blk = blkid - r * nb;
            const bool real = live && r < n;
            float val[8];
            if (real) {
                const float4 *src = reinterpret_cast<const float4 *>(
                                        p.h + (size_t)(pos0 + r) * 2 * p.eh + (size_t)blk * 2 * MIAG_QK) +
                                    4 * q;
                float4 g[4];
#pragma unroll
                for (int k = 0; k < 4; k++) g[k] = __ldg(src + k);
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    val[2 * k] = swiglu_ref(g[k].x, g[k].y);
                    val[2 * k + 1] = swiglu_ref(g[k].z, g[k].w);
                }
            } else {
#pragma unroll
                for (int k = 0; k < 8; k++) val[k] = 0.0f;
            }
            float a = 0.0f;
#pragma unroll
            for (int k = 0; k < 8; k++) a = fmaxf(a, fabsf(val[k]));
            a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
            a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
            if (!live) continue;
            const float dq = __fdiv_rn(a, 127.0f);
            const float id = dq != 0.0f ? __fdiv_rn(1.0f, dq) : 0.0f;
            uint32_t w[2];
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                uint32_t u = 0;
#pragma unroll
                for (int k = 0; k < 4; k++)
                    u |= (uint32_t)(uint8_t)(int8_t)roundf(__fmul_rn(val[4 * hh + k], id)) << (8 * k);
                w[hh] = u;
            }
            // values 8q .. 8q+7 of block blk: k tile blk / 4, 16-byte chunk
            // 2 (blk % 4) + q / 2, half q % 2
            const int kt = blk >> 2, j = blk & 3;
            *reinterpret_cast<uint2 *>(dst + tc_tile_off(Nc, kt) +
                                       tile_chunk_offset(r, 2 * j + (q >> 1)) + 8 * (q & 1)) =
                make_uint2(w[0], w[1]);
            if (q == 0) *reinterpret_cast<float *>(dst + tc_scale_off(Nc, kt, j, r)) = dq;
        }
    }
}

TcParams tc_params(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w, bool gu,
                   int *err) {
    TcParams p{};
    p.d = m.d, p.eh = m.eh, p.E = m.E, p.K = m.K;
    p.RT = gu ? lay.gu_rt : lay.dn_rt;
    p.KT = gu ? lay.gu_kt : lay.dn_kt;
    p.rows = gu ? 2 * m.eh : m.d;
    p.expert_bytes = lay.expert_bytes;
    p.weights = L.experts + (gu ? lay.gu_off : lay.dn_off);
    p.n_active = w.n_active, p.chunk_pre = w.chunk_pre, p.chunk_brow = w.chunk_brow;
    p.perm = w.perm, p.chunk_info = w.chunk_info;
    p.tiles = gu ? w.bx : w.bh;
    p.h = w.h, p.y = w.y, p.yr = w.yr;
    p.one = 1.0f;
    p.sched = w.tc_sched + (gu ? 0 : 2);
    p.err = err;
    return p;
}

TcTileParams tile_params(const Dims &m, const StoreLayout &lay, const Work &w, bool gu, int *err) {
    TcTileParams t{};
    t.d = m.d, t.eh = m.eh, t.K = m.K;
    t.KT = gu ? lay.gu_kt : lay.dn_kt;
    t.xs = scale_pad(m.d / MIAG_QK);
    t.x_row = w.x_stride ? w.x_stride : (size_t)m.d;
    t.dx_row = w.dx_stride ? w.dx_stride : (size_t)t.xs;
    t.n_rows = w.pair_row ? w.n_rows : w.T;
    t.n_active = w.n_active, t.chunk_pre = w.chunk_pre, t.chunk_brow = w.chunk_brow;
    t.perm = w.perm, t.pair_row = w.pair_row, t.chunk_info = w.chunk_info;
    t.xq = w.xq, t.dx = w.dx, t.h = w.h;
    t.tiles = gu ? w.bx : w.bh;
    t.err = err;
    return t;
}

int chunk_bound(const Dims &m, int P) { return P / kTcChunk + m.E; }

}  // namespace

bool tc_supported(const Dims &m) {
    // two k tiles per stage, whole 128-byte k tiles, row tiles addressable
    return m.d % 256 == 0 && m.eh % 256 == 0 && m.d >= 256 && m.eh >= 256 && m.K <= 64;
}

size_t tc_tile_bytes(const Dims &m, int P, bool gu) {
    const int KT = gu ? m.d / kTileK : m.eh / kTileK;
    // every expert's pairs rounded up to 16 rows
    return ((size_t)P + 15u * (size_t)m.E) * KT * kTcPairRowBytes;
}

int tc_setup_attributes() {
    const auto attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
    if (cudaFuncSetAttribute(k_expert_tc<true>, attr, kTcSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(k_expert_tc<false>, attr, kTcSmemBytes) != cudaSuccess)
        return -1;
    return 0;
}

void launch_tc_gather(const Dims &m, const StoreLayout &lay, const Work &w, int num_sms, int *err,
                      cudaStream_t s) {
    const TcTileParams t = tile_params(m, lay, w, true, err);
    launch_dependent(k_tc_gather, dim3((unsigned)min(chunk_bound(m, w.P), 4 * num_sms)), dim3(256),
                     0, s, t);
}

void launch_tc_swiglu(const Dims &m, const StoreLayout &lay, const Work &w, int num_sms, int *err,
                      cudaStream_t s) {
    const TcTileParams t = tile_params(m, lay, w, false, err);
    launch_dependent(k_tc_swiglu, dim3((unsigned)chunk_bound(m, w.P), 4), dim3(256), 0, s, t);
    (void)num_sms;
}

void launch_gateup_tc(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w,
                      int num_sms, int *err, cudaStream_t s) {
    const int cb = chunk_bound(m, w.P);
    const TcParams p = tc_params(m, lay, L, w, true, err);
    const int items = cb * p.RT;
    launch_dependent(k_expert_tc<true>, dim3((unsigned)min(items, num_sms)), dim3(kTcThreads),
                     kTcSmemBytes, s, p);
}

void launch_down_tc(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w,
                    int num_sms, int *err, cudaStream_t s) {
    const int cb = chunk_bound(m, w.P);
    const TcParams p = tc_params(m, lay, L, w, false, err);
    const int items = cb * p.RT;
    launch_dependent(k_expert_tc<false>, dim3((unsigned)min(items, num_sms)), dim3(kTcThreads),
                     kTcSmemBytes, s, p);
}

}  // namespace miag
