// gemv.cu -- grouped Q8_0 expert products for the decode regime.
//
// Reference: the three mia_matvec calls per active expert in moe()
// (src/model/forward.c:186-193) -> rows_kernel (src/tensor/matmul.c:75-80)
// -> dot_q8_scalar (:19-28); SwiGLU :188-191 and the re-quantization of h
// inside mia_matvec (:93, quant.c:11-27) in k_swiglu_q8 between the two
// expert launches; weighted combine :194.
//
// Work is grouped by expert: every weight tile is read from HBM once per
// group of up to 32 of that expert's (token, slot) pairs.  An item is
// (active expert, 128-row tile, chunk of 32 pairs); persistent CTAs (one per
// SM) own contiguous item ranges, so consecutive items share their
// activations, which are staged in shared memory once.  Each item's K range
// streams through a ring of stages in shared memory, one 1-D TMA bulk copy
// of two tile units (16 KiB swizzled int8 tile + its 2 KiB of scales, each)
// per stage; the warp that releases a stage last issues its refill.
//
// Eight consumer warps each own 16 rows of the tile.  Per Q8_0 block (K =
// 32) a warp issues one int8 tensor-core MMA, m16n8k32 (16 rows x 8 pairs),
// whose int32 results are the block's exact integer dots.  Every lane holds
// the same four (row, pair) positions for all blocks, so it carries their
// fp32 accumulators in registers and applies the reference's step
//     s = s + ((float)dot * w.d) * x.d        (matmul.c:25, blocks in order)
// with round-to-nearest intrinsics: the result equals mia_matvec_scalar bit
// for bit.  Operands come from shared memory through ldmatrix; the 128-byte
// XOR swizzle of the tiles (and the odd 16-byte stride of activation rows)
// keeps those reads free of bank conflicts.
#include <type_traits>

#include "kernels.cuh"

namespace miag {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumers;  // no producer warp: see run_item
constexpr int kItemTable = 256;           // decoded items cached per CTA
constexpr int kTableBytes = kItemTable * 16;
constexpr int kStageKT = 2;  // k tiles per stage
constexpr int kStageBytes = kStageKT * kUnitBytes;  // one bulk copy
constexpr int kMaxStages = 12;
constexpr int kBarBytes = 1024;
constexpr int kRingOff = kBarBytes + kTableBytes;  // head | item table | ring | activations
constexpr int kSmemBudget = 227 * 1024;
constexpr uint32_t kFull = 0xffffffffu;

struct GemvParams {
    Dims m;
    StoreLayout lay;
    const uint8_t *experts;
    const int32_t *offsets, *perm, *active, *n_active, *chunk_pre;
    const int4 *chunk_info;    // per pair chunk: (expert, chunk of it, segment start, pairs)
    const int32_t *max_chunk;  // largest chunk
    int32_t *chunk_done;       // decode regime: gate/up row tiles finished per chunk
    ShareState *share;         // this launch kind's SM shares
    int num_sms;
    const int8_t *xq;  // [rows][d]
    const float *dx;   // [rows][xs]
    const int32_t *pair_row;  // [P] activation row of each pair, or null: pair / K
    int n_rows;        // rows of xq / dx
    size_t x_row;      // bytes between rows of xq
    size_t dx_row;     // floats between rows of dx
    float *h;          // [P][2 eh] gate/up products (gate even, up odd), sorted order
    const int8_t *hq;  // [P][eh]   Q8_0 h = silu(gate) * up, sorted order (down's input)
    const float *hs;   // [P][xs]   its block scales
    float *y;          // [P][d], pair order
    YRoute yr;         // expert parallelism: y rows stored at their origin ranks instead
    int stages;
    int chunk;                 // pairs per chunk (tok_chunk)
    uint32_t x_stride;         // row stride of the staged activations
    float one;                 // 1.0f, opaque to the compiler (see q8_step_x2)
    int *err;
};

__device__ __forceinline__ void consumer_sync() { __syncthreads(); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t &r0, uint32_t &r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
                 : "=r"(r0), "=r"(r1)
                 : "r"(addr));
}

// D = A(16x32 s8, row) * B(32x8 s8, col) + kMagicBits, int32, exact.
__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%10, %10, %10, %10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(kMagicBits));
}

// An item: expert e, row tile rt, pair chunk tc, which covers pairs
// [seg0 + 32 tc, + nq) of the expert-sorted order.
struct ItemInfo {
    int e, rt, tc, seg0, nq;
};

// Item `item` of the launch: row tile item % RT of pair chunk item / RT in
// the permutation's chunk list (experts ascending, chunks in order).
__device__ __forceinline__ ItemInfo decode_item(const GemvParams &p, int RT, int item) {
    const int4 c = __ldcg(p.chunk_info + item / RT);
    ItemInfo it;
    it.e = c.x, it.tc = c.y, it.seg0 = c.z, it.nq = c.w;
    it.rt = item % RT;
    return it;
}

// Table form of an item: (e, rt | tc << 8, seg0, nq).
__device__ __forceinline__ int4 pack_item(const ItemInfo &ii) {
    return make_int4(ii.e, ii.rt | (ii.tc << 8), ii.seg0, ii.nq);
}
__device__ __forceinline__ ItemInfo unpack_item(int4 v) {
    ItemInfo ii;
    ii.e = v.x, ii.rt = v.y & 255, ii.tc = v.y >> 8, ii.seg0 = v.z, ii.nq = v.w;
    return ii;
}

// The head of the CTA's shared memory: the ring's barriers and release
// counters, and the activation rows of the chunk being staged.
struct RingHead {
    uint64_t full[kMaxStages];      // stage holds its k tiles (TMA complete_tx)
    uint32_t released[kMaxStages];  // warps done with the stage, summed over rounds
    int tok[kTokChunk];             // activation rows of the pairs being staged
    int slot, first, n_mine;        // this CTA's share of the items
    int parity;                     // rate buffer read (-1: shares not weighted)
    unsigned long long t_start;     // when the share's work began
};
static_assert(sizeof(RingHead) <= kBarBytes, "ring head");

// Item first + k of the launch (this CTA's k-th) as its table entry.
__device__ __forceinline__ int4 item_entry(const GemvParams &p, const int4 *table, int first,
                                           int RT, int k) {
    if (k < kItemTable) return table[k];
    return pack_item(decode_item(p, RT, first + k));
}

// The CTA's copy stream: iteration j brings k stage ks of its item k
// (counted from the CTA's first item) into ring stage j % S.
//
// Every warp walks its own Feed in step with its ring position, S
// iterations ahead, so the warp that frees a stage last issues the refill
// straight from registers.  (Working the source out at that moment -- three
// runtime divisions and a table read queued behind the tile loads of the
// other warps -- cost about as much as the copy's whole k-stage of compute,
// and it fell on the one warp that, being slowed by it, stayed the last.)
struct FeedCtx {
    const uint8_t *weights;  // this matrix (gate/up or down) of expert 0
    const int4 *table;
    size_t expert_bytes;
    int first, RT, KT, NS, E;
    int n_items;             // items in the CTA's list as far as this thread knows
};

struct Feed {
    const uint8_t *src;  // bytes of iteration j
    int j, ks, k;
    int4 next;           // table entry of item k + 1
};

// Source of an item's first k stage; null for an entry naming a tile outside
// the store, which is then never copied.
__device__ __forceinline__ const uint8_t *item_src(const FeedCtx &fc, int4 v) {
    if ((unsigned)v.x >= (unsigned)fc.E || (v.y & 255) >= fc.RT) return nullptr;
    return fc.weights + (size_t)v.x * fc.expert_bytes + (size_t)(v.y & 255) * fc.KT * kUnitBytes;
}

__device__ __forceinline__ Feed feed_at(const GemvParams &p, const FeedCtx &fc, int j0) {
    Feed f;
    f.j = j0, f.k = j0 / fc.NS, f.ks = j0 % fc.NS;
    const uint8_t *src = f.k < fc.n_items ? item_src(fc, item_entry(p, fc.table, fc.first, fc.RT, f.k))
                                          : nullptr;
    f.src = src ? src + (size_t)f.ks * kStageBytes : nullptr;
    f.next = f.k + 1 < fc.n_items ? item_entry(p, fc.table, fc.first, fc.RT, f.k + 1)
                                  : make_int4(0, 0, 0, 0);
    return f;
}

__device__ __forceinline__ void feed_next(const GemvParams &p, const FeedCtx &fc, Feed &f) {
    f.j++;
    if (++f.ks == fc.NS) {
        f.ks = 0, f.k++;
        f.src = item_src(fc, f.next);
        if (f.k + 1 < fc.n_items) f.next = item_entry(p, fc.table, fc.first, fc.RT, f.k + 1);
    } else {
        f.src = f.src ? f.src + kStageBytes : nullptr;
    }
}

// Issues iteration f.j into stage s, completing on its full barrier.  A null
// source (an entry outside the store) is never copied: the error word
// records it and the stage stays empty, so its consumers time out instead.
__device__ __forceinline__ void feed_issue(const GemvParams &p, const FeedCtx &fc, const Feed &f,
                                           uint8_t *smem, int s) {
    RingHead *h = reinterpret_cast<RingHead *>(smem);
    if (!f.src) {
        set_error(p.err, kErrItemList);
        return;
    }
    const uint32_t bytes = (uint32_t)min(kStageKT, fc.KT - f.ks * kStageKT) * kUnitBytes;
    mbar_arrive_expect_tx(&h->full[s], bytes);
    bulk_g2s(smem + kRingOff + (size_t)s * kStageBytes, f.src, bytes, &h->full[s]);
}

// N-tiles (of 8 pairs) the consumers run for a chunk of nq pairs.  Two
// regimes, chosen per launch from the batch (wide_batch): chunks of up to 16
// pairs (decode) run one or two n-tiles, chunks of up to 32 (prefill) one or
// four.  Two shapes a kernel keep every value in registers; three spilled.
__host__ __device__ inline int n_tiles(int nq, bool wide) {
    return nq <= 8 ? 1 : wide ? 4 : 2;
}

// Bytes of the activation region for chunks of up to nq pairs: nq int8 rows
// at x_stride, then the pair-interleaved scale rows that the lanes of
// n_tiles(nq) n-tiles address (four per n-tile, whether or not those pairs
// exist).
__host__ __device__ inline uint32_t region_size(int nq, bool wide, uint32_t x_stride, int xs) {
    const uint32_t b = (uint32_t)nq * x_stride +
                       4u * (uint32_t)n_tiles(nq, wide) * smem_stride((uint32_t)xs * 8);
    return (b + 127u) & ~127u;
}

// Consumers: stage the activations of pairs [t0, t0+n) of the expert segment
// starting at seg0 in the shared region: int8 rows at x_stride, then the
// scales of pairs 2q and 2q+1 interleaved in one row per q, [block][2] f32 at
// their own odd-16-byte stride, so a lane loads its two pair columns' scales
// of a block as one f32 pair.
//   gate/up: xq[token(pair)] and dx[token] (quantized by the router);
//   down:    hq[pair] and hs[pair] (quantized by k_swiglu_q8).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_all;" ::: "memory");
}

// Called by all consumer threads between two CTA barriers.  Every copy is an
// asynchronous global-to-shared copy issued before the first wait, so a fill
// costs one round trip for the data (plus one for the token rows of gate/up)
// however many vectors each thread moves.
template <bool kGU>
__device__ void fill_region(const GemvParams &p, uint8_t *region, int rows_cap, int seg0, int t0,
                            int n, int row_bytes, int nscale, int *tok) {
    const int srow = (int)smem_stride((uint32_t)nscale * 8);  // scale row of a pair of pairs
    uint8_t *rs = region + (size_t)rows_cap * p.x_stride;
    const int8_t *q_src = kGU ? p.xq : p.hq;
    const float *s_src = kGU ? p.dx : p.hs;
    if (kGU) {  // the chunk's activation rows
        if ((int)threadIdx.x < n) {
            const int pr = __ldg(p.perm + seg0 + t0 + threadIdx.x);
            int t = p.pair_row ? __ldg(p.pair_row + pr) : pr / p.m.K;
            if (t < 0 || t >= p.n_rows) {  // a caller's row index out of range
                set_error(p.err, kErrBadExpert);
                t = 0;
            }
            tok[threadIdx.x] = t;
        }
        consumer_sync();
    }
    const int qv = row_bytes / 16, sv = nscale / 4;  // 16-byte vectors per row / scale row
    const int per = qv + sv, total = n * per;
    for (int v = threadIdx.x; v < total; v += kConsumers) {
        const int j = v / per, k = v - j * per;
        const int t = kGU ? tok[j] : seg0 + t0 + j;
        const size_t q_row = kGU ? p.x_row : (size_t)row_bytes;
        const size_t s_row = kGU ? p.dx_row : (size_t)nscale;
        if (k < qv) {
            cp_async16(region + (size_t)j * p.x_stride + 16 * k, q_src + (size_t)t * q_row + 16 * k);
        } else {
            const float *src = s_src + (size_t)t * s_row + 4 * (k - qv);
            float *dst = reinterpret_cast<float *>(rs + (size_t)(j >> 1) * srow) + 8 * (k - qv) + (j & 1);
#pragma unroll
            for (int i = 0; i < 4; i++) cp_async4(dst + 2 * i, src + i);
        }
    }
    cp_async_wait_all();
}

// Decode regime, down: stage the activations of pairs [t0, t0+n) of the
// expert segment at seg0 straight from gate/up's products, forming
// h = silu(gate) * up (forward.c:188-191) and quantizing it to Q8_0 as
// mia_matvec quantizes its input (matmul.c:93, quant.c:11-27) -- the work of
// k_swiglu_q8 for these pairs, four threads per 32-block, eight values
// each; the block maximum is combined over the four lanes.  Layout as
// fill_region.  Whole warps run every round (the shuffles need them).
__device__ void fill_region_swiglu(const GemvParams &p, uint8_t *region, int rows_cap, int seg0,
                                   int t0, int n, int eh, int nscale) {
    const int srow = (int)smem_stride((uint32_t)nscale * 8);
    uint8_t *rs = region + (size_t)rows_cap * p.x_stride;
    const int nb = eh / MIAG_QK, total = n * nb * 4;
    for (int v0 = 0; v0 < total; v0 += kConsumers) {
        const int v = v0 + (int)threadIdx.x;
        const bool live = v < total;  // whole quads (total % 4 == 0)
        const int blk = live ? v >> 2 : 0, q = v & 3;
        const int j = blk / nb, b = blk - j * nb;
        const float4 *src = reinterpret_cast<const float4 *>(
            p.h + (size_t)(seg0 + t0 + j) * 2 * eh + (size_t)b * 2 * MIAG_QK) + 4 * q;
        float4 g[4];
#pragma unroll
        for (int k = 0; k < 4; k++) g[k] = live ? __ldcg(src + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        float h[8];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            h[2 * k] = swiglu_ref(g[k].x, g[k].y);
            h[2 * k + 1] = swiglu_ref(g[k].z, g[k].w);
        }
        float a = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) a = fmaxf(a, fabsf(h[k]));
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
                u |= (uint32_t)(uint8_t)(int8_t)roundf(__fmul_rn(h[4 * hh + k], id)) << (8 * k);
            w[hh] = u;
        }
        *reinterpret_cast<uint2 *>(region + (size_t)j * p.x_stride + (size_t)b * MIAG_QK + 8 * q) =
            make_uint2(w[0], w[1]);
        if (q == 0) reinterpret_cast<float *>(rs + (size_t)(j >> 1) * srow)[2 * b + (j & 1)] = dq;
    }
}

// Decode regime: chunk c's gate/up products are complete once all its row
// tiles are counted (gate/up adds a CTA's tiles of a chunk when it leaves
// the chunk, after a CTA barrier and a fence).  Thread 0 waits (bounded).
__device__ __forceinline__ int ld_acquire(const int32_t *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ void wait_chunk(const GemvParams &p, int c) {
    const int target = p.lay.gu_rt;
    const long long t0 = clock64();
    while (ld_acquire(p.chunk_done + c) < target) {
        if (clock64() - t0 > kWaitCycles) {
            set_error(p.err, kErrWaitFull);
            return;
        }
        __nanosleep(64);
    }
}

// h = silu(gate) * up (forward.c:188-191) for every pair, quantized to Q8_0
// exactly as mia_matvec quantizes its input (matmul.c:93, quant.c:11-27).
// A launch of its own because the SiLU's exp runs in double precision
// (expf_cr), whose latency only many threads hide: four threads per
// (pair, 32-block), eight values each, their loads issued together; the
// block maximum is combined over the four lanes (max is exact in any order).
__global__ void k_swiglu_q8(const float *gu, int P, int eh, int xs, int8_t *hq, float *hs) {
    // lets down start its prologue (see k_expert_mma) before the products
    // are complete
    pdl_launch_dependents();
    pdl_wait();
    const int nb = eh / MIAG_QK;
    const long task = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const long n_tasks = (long)P * nb * 4;
    const bool live = task < n_tasks;  // whole quads are live or not (n_tasks % 4 == 0)
    const long blk = live ? task >> 2 : 0;
    const int j = (int)(blk / nb), b = (int)(blk % nb), q = (int)(task & 3);
    // values 8q .. 8q+7 of the block: (gate, up) floats 16q .. 16q+15
    const float4 *src = reinterpret_cast<const float4 *>(gu + (size_t)j * 2 * eh + (size_t)b * 2 * MIAG_QK) + 4 * q;
    float4 g[4];
#pragma unroll
    for (int k = 0; k < 4; k++) g[k] = live ? __ldg(src + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    float v[8];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        v[2 * k] = swiglu_ref(g[k].x, g[k].y);
        v[2 * k + 1] = swiglu_ref(g[k].z, g[k].w);
    }
    float a = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) a = fmaxf(a, fabsf(v[k]));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    if (!live) return;
    const float dq = __fdiv_rn(a, 127.0f);
    const float id = dq != 0.0f ? __fdiv_rn(1.0f, dq) : 0.0f;
    uint32_t w[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        uint32_t u = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) u |= (uint32_t)(uint8_t)(int8_t)roundf(__fmul_rn(v[4 * h + k], id)) << (8 * k);
        w[h] = u;
    }
    *reinterpret_cast<uint2 *>(hq + (size_t)j * eh + (size_t)b * MIAG_QK + 8 * q) = make_uint2(w[0], w[1]);
    if (q == 0) hs[(size_t)j * xs + b] = dq;
}

// Per-lane roles in the warp's 16-row slice of a tile, as shared-memory
// byte offsets fixed for the whole kernel.
struct Lanes {
    int g, tq;              // mma groupID, thread-in-group
    int r0;                 // first of this lane's two rows (r0, r0 + 8) in the tile
    uint32_t w0, w1;        // offsets of rows r0, r0 + 8 in a scale tile
    uint32_t b_off;         // ldmatrix B role: pair row lane & 7, 16-byte half
    int b_pair;
    uint32_t b_blk;         // ldmatrix.x4 B role: lanes 16-31 load the next block
    uint32_t a_off[4];      // ldmatrix A role: swizzled offset of block j in a tile
};

__device__ __forceinline__ Lanes lane_roles(int warp, int lane) {
    Lanes l;
    l.g = lane >> 2, l.tq = lane & 3;
    l.r0 = 16 * warp + l.g;
    l.w0 = 16u * (uint32_t)l.r0, l.w1 = 16u * (uint32_t)(l.r0 + 8);
    // A (x4): lanes 0-7 rows 0-7, 8-15 rows 8-15, 16-31 the same rows' second
    // 16-byte half.  B (x2): lanes 0-7 pairs 0-7, 8-15 their second half.
    const int a_row = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8, a_half = lane >> 4;
#pragma unroll
    for (int j = 0; j < 4; j++) l.a_off[j] = tile_chunk_offset(a_row, 2 * j + a_half);
    l.b_pair = lane & 7;
    l.b_off = 16u * (uint32_t)((lane >> 3) & 1);
    l.b_blk = (uint32_t)(lane >> 4);
    return l;
}

__device__ __forceinline__ void lds_2x64(uint32_t addr, uint64_t &a, uint64_t &b) {
    asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}

// One k tile (4 Q8_0 blocks; kFull = all four inside K) for NT n-tiles of
// 8 pairs.  tile/sc: the k tile's int8 and scale tiles in the stage.
// acc[n][0]: row r0 x pairs (2tq, 2tq+1) of n-tile n; acc[n][1]: row r0 + 8.
template <int NT, bool kFull>
__device__ __forceinline__ void k_tile(uint64_t (&acc)[NT][2], uint32_t tile, uint32_t sc, int kt,
                                       int nbk, const Lanes &ln, const uint32_t (&b_row)[NT],
                                       const uint32_t (&xp)[NT], uint64_t neg_magic2,
                                       uint64_t one2) {
    uint32_t A[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++)
        if (kFull || j < nbk) ldsm_x4(tile + ln.a_off[j], A[j][0], A[j][1], A[j][2], A[j][3]);
    const float4 w0 = lds128(sc + ln.w0), w1 = lds128(sc + ln.w1);
    const uint64_t wa[4] = {pack2(w0.x, w0.x), pack2(w0.y, w0.y), pack2(w0.z, w0.z), pack2(w0.w, w0.w)};
    const uint64_t wb[4] = {pack2(w1.x, w1.x), pack2(w1.y, w1.y), pack2(w1.z, w1.z), pack2(w1.w, w1.w)};
    // Two n-tiles at a time: both tiles' dots first, then the steps block by
    // block across them (four independent accumulator chains per step).
#pragma unroll
    for (int n0 = 0; n0 < NT; n0 += 2) {
        constexpr int G = 2;
        int C[G][4][4];
        uint64_t x2[G][4];  // per n-tile and block: the scales of this lane's two pair columns
#pragma unroll
        for (int g = 0; g < G; g++) {
            const int n = n0 + g;
            if (n >= NT) break;
            const uint32_t brow = b_row[n] + (uint32_t)(kt * kTileK);
            uint32_t B[4][2];
            if (kFull) {
                // one ldmatrix.x4 per two blocks: lanes 16-31 address the second block
                const uint32_t b4 = brow + 32u * ln.b_blk;
                ldsm_x4(b4, B[0][0], B[0][1], B[1][0], B[1][1]);
                ldsm_x4(b4 + 64u, B[2][0], B[2][1], B[3][0], B[3][1]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (j < nbk) ldsm_x2(brow + 32 * j, B[j][0], B[j][1]);
            }
            lds_2x64(xp[n] + 32u * (uint32_t)kt, x2[g][0], x2[g][1]);
            lds_2x64(xp[n] + 32u * (uint32_t)kt + 16u, x2[g][2], x2[g][3]);
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (kFull || j < nbk) mma_s8(C[g][j], A[j][0], A[j][1], A[j][2], A[j][3], B[j][0], B[j][1]);
        }
        // block order, as the reference's loop over blocks
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (kFull || j < nbk) {
#pragma unroll
                for (int g = 0; g < G; g++) {
                    const int n = n0 + g;
                    if (n >= NT) break;
                    q8_step_x2(acc[n][0], pack2i(C[g][j][0], C[g][j][1]), wa[j], x2[g][j], neg_magic2, one2);
                    q8_step_x2(acc[n][1], pack2i(C[g][j][2], C[g][j][3]), wb[j], x2[g][j], neg_magic2, one2);
                }
            }
        }
    }
}

// The row of pair `pid` (pair order) in y (see y_route_row).
__device__ __forceinline__ float *y_row(const GemvParams &p, int pid) {
    return y_route_row(p.yr, p.y, p.m.d, pid);
}

// What one item needs besides the kernel parameters.
struct ItemCtx {
    uint32_t stages;         // shared address of stage 0
    uint32_t x_rows, x_scl;  // shared addresses of the activation rows / scale rows
    uint32_t xpp_bytes;      // stride of the scale rows (one per pair of pairs)
    int S, KT, NS, nb, rows;
    int rt, seg0, t0, nq;    // the item: row tile, expert segment, first pair, pairs
};

// Position in the ring: iteration it uses stage s = it % S in phase
// (it / S) & 1; advanced without divisions.
struct RingPos {
    int it, s;
    uint32_t phase;
    __device__ __forceinline__ void next(int S) {
        it++;
        if (++s == S) s = 0, phase ^= 1u;
    }
};

// One item: its k tiles through the ring, then its outputs.
//
// There is no producer warp.  Thread 0 issues the first S stages; after
// that, the warp that is the last of the eight to finish with a stage
// refills it with the iteration S ahead, which its Feed holds.  With eight warps per CTA the
// register file allows 255 registers a thread (a ninth warp capped it at
// 168, which the tile shapes exceed).
template <bool kGU, int NT>
__device__ __forceinline__ void run_item(const GemvParams &p, const ItemCtx &ic, const Lanes &ln,
                                         uint8_t *smem, RingPos &rp, const FeedCtx &fc, Feed &fd,
                                         bool &failed) {
    RingHead *head = reinterpret_cast<RingHead *>(smem);
    const int lane = threadIdx.x & 31;
    const int nq = ic.nq;
    // per n-tile: this lane's B row (pairs past nq repeat the last pair; their
    // columns are never written out) and the scale row of its two columns
    uint32_t b_row[NT], xp[NT];
#pragma unroll
    for (int n = 0; n < NT; n++) {
        b_row[n] = ic.x_rows + (uint32_t)min(8 * n + ln.b_pair, nq - 1) * p.x_stride + ln.b_off;
        xp[n] = ic.x_scl + (uint32_t)(4 * n + ln.tq) * ic.xpp_bytes;
    }
    const uint64_t neg_magic2 = pack2(-kMagic, -kMagic), one2 = pack2(p.one, p.one);
    uint64_t acc[NT][2];
#pragma unroll
    for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = 0ull;  // +0.0f in both lanes

    const bool full_tiles = (ic.KT % kStageKT) == 0 && 4 * ic.KT == ic.nb;
    for (int ks = 0; ks < ic.NS; ks++, rp.next(ic.S)) {
        const int s = rp.s;
        if (!failed) {
            bool got = true;
            if (lane == 0) got = mbar_wait(&head->full[s], rp.phase);
            if (!__shfl_sync(kFull, got, 0)) {
                // Keep walking (on stale data) so every consumer reaches the
                // same barriers: no warp may leave early.
                set_error(p.err, kErrWaitFull);
                failed = true;
            }
        }
        const uint32_t stg = ic.stages + (uint32_t)(s * kStageBytes);
        const uint32_t scl = stg + kTileBytes;  // unit kk: tile at kk units, its scales after it
        const int kt0 = ks * kStageKT;
        if (full_tiles) {
            // both k tiles in straight-line code while the registers allow
#pragma unroll (NT == 1 ? kStageKT : 1)
            for (int kk = 0; kk < kStageKT; kk++)
                k_tile<NT, true>(acc, stg + kk * kUnitBytes, scl + kk * kUnitBytes, kt0 + kk, 4,
                                 ln, b_row, xp, neg_magic2, one2);
        } else {
            const int nkt = min(kStageKT, ic.KT - kt0);
            for (int kk = 0; kk < nkt; kk++)
                k_tile<NT, false>(acc, stg + kk * kUnitBytes, scl + kk * kUnitBytes, kt0 + kk,
                                  min(4, ic.nb - 4 * (kt0 + kk)), ln, b_row, xp, neg_magic2, one2);
        }
        __syncwarp();
        if (lane == 0) {
            // release the stage; the eighth release of a round refills it
            __threadfence_block();
            const uint32_t done = atomicAdd(&head->released[s], 1u);
            if ((done % kConsumerWarps) == kConsumerWarps - 1 && fd.k < fc.n_items) {
                __threadfence_block();
                fence_proxy_async_smem();
                feed_issue(p, fc, fd, smem, s);
            }
        }
        feed_next(p, fc, fd);
    }

    // outputs: this lane holds rows r0, r0 + 8 x pairs 8n + 2tq, 8n + 2tq + 1
    const int R0 = ic.rt * kTileRows + ln.r0, R1 = R0 + 8;
    const int rows = ic.rows;
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const int qa = 8 * n + 2 * ln.tq, qb = qa + 1;
        const float2 u0 = unpack2(acc[n][0]), u1 = unpack2(acc[n][1]);
        const float o[4] = {u0.x, u0.y, u1.x, u1.y};  // (r0,qa) (r0,qb) (r1,qa) (r1,qb)
        if (kGU) {
            // the products as they are, gate (even rows) beside up (odd
            // rows); the down launch forms silu(gate) * up while staging them
            if (qa < nq) {
                float *hp = p.h + (size_t)(ic.seg0 + ic.t0 + qa) * rows;
                if (R0 < rows) hp[R0] = o[0];
                if (R1 < rows) hp[R1] = o[2];
            }
            if (qb < nq) {
                float *hp = p.h + (size_t)(ic.seg0 + ic.t0 + qb) * rows;
                if (R0 < rows) hp[R0] = o[1];
                if (R1 < rows) hp[R1] = o[3];
            }
        } else {
            // y goes out in pair order, so the combine (and a remote caller)
            // finds pair t*K + j's row without the permutation
            if (qa < nq) {
                float *yp = y_row(p, __ldg(p.perm + ic.seg0 + ic.t0 + qa));
                if (R0 < rows) yp[R0] = o[0];
                if (R1 < rows) yp[R1] = o[2];
            }
            if (qb < nq) {
                float *yp = y_row(p, __ldg(p.perm + ic.seg0 + ic.t0 + qb));
                if (R0 < rows) yp[R0] = o[1];
                if (R1 < rows) yp[R1] = o[3];
            }
        }
    }
}

// SM shares.  On B200 some SMs stream and compute the same items 15-35 %
// slower than others, and the same SMs every launch; with equal shares the
// launch ends with them.  So a launch with one CTA per SM gives slot s (the
// CTA on SM s, normally) a contiguous share in proportion to rate[s], the
// items a microsecond slot s achieved in earlier launches, and measures it
// again (in the narrow regime, where items cost alike).  Every slot is
// claimed exactly once whichever SMs the CTAs land on,
// and every CTA derives the shares the same way from the same rates, so the
// shares always partition the items; placement only decides how even the
// end is.

// Slot of this CTA: its SM's, else the next free one (thread 0).
__device__ int claim_slot(ShareState *sh, int G, int *err) {
    const int s0 = (int)(sm_id() % (unsigned)G);
    for (int i = 0; i < G; i++) {
        const int c = (s0 + i) % G;
        if (atomicExch(&sh->taken[c], 1) == 0) return c;
    }
    set_error(err, kErrItemList);  // no free slot: the state was not reset
    return -1;
}

// Sums of the rates of slots [0, ja), [0, jb) and [0, G): the same floats in
// every CTA and nondecreasing in j.  Lane l holds slots [5l, 5l + 5); the
// lane sums below a slot's lane are added one by one in lane order, then
// the slot's first j - 5l rates in order, so every prefix is a sequential
// sum of the one before it and a nonnegative term, and rounding is
// monotone.  One pass over the lanes serves all three.
struct RatePrefix {
    float a, b, total;
};
__device__ RatePrefix rate_prefixes(const float (&r)[kMaxSlots / 32], int ja, int jb) {
    constexpr int per = kMaxSlots / 32;
    float own = 0.0f;
#pragma unroll
    for (int i = 0; i < per; i++) own = __fadd_rn(own, r[i]);
    const int la = min(ja / per, 32), lb = min(jb / per, 32);
    float ea = 0.0f, eb = 0.0f, et = 0.0f;
    for (int q = 0; q < 32; q++) {
        const float o = __shfl_sync(0xffffffffu, own, q);
        if (q < la) ea = __fadd_rn(ea, o);
        if (q < lb) eb = __fadd_rn(eb, o);
        et = __fadd_rn(et, o);
    }
    float ba = 0.0f, bb = 0.0f;
#pragma unroll
    for (int i = 0; i < per; i++) {
        const float va = __shfl_sync(0xffffffffu, r[i], min(la, 31));
        const float vb = __shfl_sync(0xffffffffu, r[i], min(lb, 31));
        if (la < 32 && i < ja - per * la) ba = __fadd_rn(ba, va);
        if (lb < 32 && i < jb - per * lb) bb = __fadd_rn(bb, vb);
    }
    RatePrefix rp;
    rp.a = la < 32 && ja > per * la ? __fadd_rn(ea, ba) : ea;
    rp.b = lb < 32 && jb > per * lb ? __fadd_rn(eb, bb) : eb;
    rp.total = et;
    return rp;
}

// gate+up (kGU) or down: one launch over all items of all active experts.
// Items (row tile, pair chunk) are numbered chunk by chunk, experts
// ascending; each CTA runs a contiguous share (see SM shares above), so
// consecutive items share their activations.  (Handing the last 15-30 % of
// the items out one by one from an atomic counter evened out the end times
// too, but cost more in activation stagings than it saved.)
template <bool kGU, bool kWide>
__global__ void __launch_bounds__(kGemvThreads, 1) k_expert_mma(GemvParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int d = p.m.d, eh = p.m.eh;
    const int RT = kGU ? p.lay.gu_rt : p.lay.dn_rt;
    const int KT = kGU ? p.lay.gu_kt : p.lay.dn_kt;
    const int Kb = kGU ? d : eh;             // bytes of K (= values)
    const int rows = kGU ? 2 * eh : d;       // matrix rows
    const int nb = Kb / MIAG_QK, xs = scale_pad(nb);
    const int NS = (KT + kStageKT - 1) / kStageKT;  // stages per item
    // gate/up reads what the router and the permutation just wrote; down,
    // whose items and weights were settled before gate/up began (gate/up
    // lets it start only after its own wait), decodes them and fills its
    // ring while gate/up and the SwiGLU finish, and waits only before its
    // activations.  Reads of the permutation go through L2.
    if (kGU) pdl_wait();
    const int n_items = __ldcg(p.chunk_pre + __ldcg(p.n_active)) * RT;
    const int G = gridDim.x;

    // The activation region holds the largest chunk of the launch; the rest
    // of shared memory deepens the ring.
    const int nq_max = max(1, __ldcg(p.max_chunk));
    const uint32_t region_bytes = region_size(nq_max, kWide, p.x_stride, xs);
    const int S = min(kMaxStages, (int)((kSmemBudget - kRingOff - (int)region_bytes) / kStageBytes));

    RingHead *head = reinterpret_cast<RingHead *>(smem);
    uint8_t *stages = smem + kRingOff;
    int4 *table = reinterpret_cast<int4 *>(smem + kBarBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // this CTA's share
    ShareState *sh = p.share;
    // (the wide regime keeps equal shares: there an item's cost follows its
    // pair count, and rates measured on one launch's mix misled the next)
    const bool weighted = !kWide && sh && G == p.num_sms && G <= kMaxSlots && n_items >= 4 * G;
    const int parity = weighted ? (__ldcg(&sh->launches) & 1) : 0;
    if (warp == 0) {
        int slot = blockIdx.x;
        int first = (int)((long)n_items * blockIdx.x / G);
        int last = (int)((long)n_items * (blockIdx.x + 1) / G);
        if (weighted) {
            // the rates load while the slot is claimed (neither needs the other)
            constexpr int per = kMaxSlots / 32;
            float r[per];
#pragma unroll
            for (int i = 0; i < per; i++) {
                const int c = per * lane + i;
                r[i] = c < G ? __ldcg(&sh->rate[parity][c]) : 0.0f;
            }
            if (lane == 0) slot = claim_slot(sh, G, p.err);
            slot = __shfl_sync(0xffffffffu, slot, 0);
            bool ok = true;
#pragma unroll
            for (int i = 0; i < per; i++)
                if (per * lane + i < G && !(r[i] > 0.0f && r[i] < 1e30f)) ok = false;
            if (slot >= 0 && __all_sync(0xffffffffu, ok)) {
                const RatePrefix rp = rate_prefixes(r, slot, slot + 1);
                const float n = (float)n_items;
                first = (int)__fdiv_rn(__fmul_rn(n, rp.a), rp.total);
                last = slot + 1 == G ? n_items : (int)__fdiv_rn(__fmul_rn(n, rp.b), rp.total);
                first = min(first, n_items), last = min(last, n_items);
            } else if (slot >= 0) {  // no rates yet: equal shares
                first = (int)((long)n_items * slot / G);
                last = (int)((long)n_items * (slot + 1) / G);
            }
        }
        if (lane == 0) {
            head->slot = slot, head->first = first, head->n_mine = max(0, last - first);
            head->parity = weighted && slot >= 0 ? parity : -1;
        }
    }
    __syncthreads();
    const int first = head->first, n_mine = head->n_mine;
    // Decode down works its share from the first chunk that starts inside
    // it: the chunk it shares with the previous slot, whose gate/up rows
    // another SM may still be producing, goes last.  (The list is rotated by
    // k0 items; only when the whole list fits the table.)
    int k0 = 0;
    if (!kGU && !kWide && n_mine <= kItemTable) {
        const int lead = (RT - first % RT) % RT;
        if (lead < n_mine) k0 = lead;
    }
    for (int k = threadIdx.x; k < min(n_mine, kItemTable); k += kGemvThreads)
        table[k] = pack_item(decode_item(p, RT, first + (k + k0) % n_mine));
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&head->full[s], 1);
            head->released[s] = 0;
        }
        fence_barrier_init();
    }
    __syncthreads();
    FeedCtx fc;
    fc.weights = p.experts + (kGU ? p.lay.gu_off : p.lay.dn_off);
    fc.table = table, fc.expert_bytes = p.lay.expert_bytes;
    fc.first = first, fc.RT = RT, fc.KT = KT, fc.NS = NS, fc.E = p.m.E, fc.n_items = n_mine;
    if (threadIdx.x == 0) {
        Feed f = feed_at(p, fc, 0);
        for (int j = 0; j < min(S, n_mine * NS); j++, feed_next(p, fc, f)) feed_issue(p, fc, f, smem, j);
    }
    Feed fd = feed_at(p, fc, S);  // the refill of iteration 0
    // Decode regime: gate/up counts each chunk's finished row tiles and down
    // waits chunk by chunk, so down's CTAs (on the SMs gate/up has left, and
    // on the chunks those SMs just finished) start before gate/up ends; down
    // forms the SwiGLU itself while staging.  Prefill: the SwiGLU launch sits
    // between, and down waits for it as a whole.
    constexpr bool kSignal = kGU && !kWide, kChunkWait = !kGU && !kWide;
    if (!kGU && kWide) pdl_wait();
    pdl_launch_dependents();

    // ---- consumers
    uint8_t *region = smem + kRingOff + (size_t)S * kStageBytes;
    const Lanes ln = lane_roles(warp, lane);
    ItemCtx ic;
    ic.stages = smem_addr(stages);
    ic.x_rows = smem_addr(region);
    ic.x_scl = ic.x_rows + (uint32_t)nq_max * p.x_stride;
    ic.xpp_bytes = smem_stride((uint32_t)xs * 8);
    ic.S = S, ic.KT = KT, ic.NS = NS, ic.nb = nb, ic.rows = rows;

    int cur_e = -1, cur_tc = -1;
    int cur_c = -1, tiles_c = 0;  // chunk being worked on, its row tiles done here (kSignal)
    RingPos rp{0, 0, 0u};
    bool failed = false;
    if (threadIdx.x == 0) head->t_start = global_ns();
    for (int k = 0; k < n_mine; k++) {
        const ItemInfo ii = unpack_item(item_entry(p, table, first, RT, k));
        const int seg0 = ii.seg0, t0 = ii.tc * p.chunk, nq = ii.nq;
        if (ii.e != cur_e || ii.tc != cur_tc) {
            consumer_sync();  // nobody still reads the region (or writes the last chunk)
            const int c = (first + (k + k0) % n_mine) / RT;  // its chunk in the permutation's list
            if (kSignal && threadIdx.x == 0 && cur_c >= 0) {
                __threadfence();  // the CTA's products of chunk cur_c, before they are counted
                atomicAdd(p.chunk_done + cur_c, tiles_c);
            }
            if (kChunkWait) {
                if (threadIdx.x == 0) wait_chunk(p, c);
                consumer_sync();
                fill_region_swiglu(p, region, nq_max, seg0, t0, nq, eh, xs);
            } else {
                fill_region<kGU>(p, region, nq_max, seg0, t0, nq, Kb, xs, head->tok);
            }
            cur_e = ii.e, cur_tc = ii.tc, cur_c = c, tiles_c = 0;
            consumer_sync();
        }
        tiles_c++;
        ic.rt = ii.rt, ic.seg0 = seg0, ic.t0 = t0, ic.nq = nq;
        // Two tile shapes (n_tiles): one n-tile of 8 pairs, or the chunk's
        // full width (columns past nq run on repeated rows, not written).
        if (nq <= 8) run_item<kGU, 1>(p, ic, ln, smem, rp, fc, fd, failed);
        else run_item<kGU, kWide ? 4 : 2>(p, ic, ln, smem, rp, fc, fd, failed);
    }
    if (kSignal) {
        consumer_sync();
        if (threadIdx.x == 0 && cur_c >= 0) {
            __threadfence();
            atomicAdd(p.chunk_done + cur_c, tiles_c);
        }
    }
    // After a timed-out wait, let every issued copy land (bounded) before the
    // CTA's shared memory goes away.  All refills are issued by now.
    const int total = n_mine * NS;
    if (__syncthreads_or(failed) && threadIdx.x == 0) {
        for (int j = total - 1; j >= 0 && j >= total - S; j--)
            mbar_wait(&head->full[j % S], (j / S) & 1);
    }
    if (threadIdx.x == 0 && head->parity >= 0) {
        // this share's rate, into the buffer the next launch reads
        const int parity = head->parity, slot = head->slot;
        ShareState *sh = p.share;
        const float old = __ldcg(&sh->rate[parity][slot]);
        const float us = (float)(global_ns() - head->t_start) * 1e-3f;
        float rate = old;
        if (n_mine > 0 && us > 0.5f) {
            const float now = (float)n_mine / us;
            rate = old > 0.0f ? 0.75f * old + 0.25f * now : now;
        }
        sh->rate[parity ^ 1][slot] = rate;
        __threadfence();
        if (atomicAdd(&sh->done, 1) == G - 1) {  // the last CTA: clear for the next launch
            for (int c = 0; c < G; c++) sh->taken[c] = 0;
            sh->done = 0;
            __threadfence();
            atomicAdd(&sh->launches, 1);
        }
    }
    // decode down waited per chunk only; its end must still imply gate/up's
    if (kChunkWait) pdl_wait();
    if (!kGU && p.yr.n > 0) ep_signal_done(p.yr);
}

// x[t] += w_j * y_j for j = 0..K-1 in order (forward.c:194).
// Pair t*K + j is token t's j-th expert; its row of y is pos[t*K + j]
// (pos null: y is in pair order).  A thread owns four columns (d % 4 == 0)
// and loads all K of its y rows before the ordered adds.  When an earlier
// step of the call has set the error word (a wait that gave up, a bad index),
// y may be partly written: x is then left as it was, and the caller learns of
// the error at its next miag_sync.
constexpr int kCombineMaxK = 16;
__global__ void k_combine(float *x, int d, int K, const float *w, const float *y,
                          const int32_t *pos, const int *err) {
    pdl_wait();
    pdl_launch_dependents();
    if (err && __ldcg(err) != kErrNone) return;
    const int t = blockIdx.x;
    const int i = 4 * (blockIdx.y * blockDim.x + threadIdx.x);
    if (i >= d) return;
    float4 v = *reinterpret_cast<const float4 *>(x + (size_t)t * d + i);
    for (int j0 = 0; j0 < K; j0 += kCombineMaxK) {  // slots in order, 16 loads in flight
        float4 yv[kCombineMaxK];
        float wv[kCombineMaxK];
#pragma unroll
        for (int u = 0; u < kCombineMaxK; u++) {
            if (j0 + u < K) {
                const size_t p = (size_t)t * K + j0 + u;
                const size_t row = pos ? (size_t)__ldg(pos + p) : p;
                wv[u] = __ldg(w + p);
                yv[u] = __ldcs(reinterpret_cast<const float4 *>(y + row * d + i));
            }
        }
#pragma unroll
        for (int u = 0; u < kCombineMaxK; u++) {
            if (j0 + u < K) {
                v.x = __fadd_rn(v.x, __fmul_rn(wv[u], yv[u].x));
                v.y = __fadd_rn(v.y, __fmul_rn(wv[u], yv[u].y));
                v.z = __fadd_rn(v.z, __fmul_rn(wv[u], yv[u].z));
                v.w = __fadd_rn(v.w, __fmul_rn(wv[u], yv[u].w));
            }
        }
    }
    *reinterpret_cast<float4 *>(x + (size_t)t * d + i) = v;
}

// ---------------------------------------------------------------------------
// Host side.

static void fill_params(GemvParams &p, const Dims &m, const StoreLayout &lay, const LayerDev &L,
                        const Work &w, int *err) {
    p.m = m, p.lay = lay, p.experts = L.experts;
    p.offsets = w.offsets, p.perm = w.perm, p.active = w.active, p.n_active = w.n_active;
    p.chunk_pre = w.chunk_pre, p.chunk_info = w.chunk_info, p.max_chunk = w.max_chunk;
    p.chunk_done = w.chunk_done;
    p.xq = w.xq, p.dx = w.dx, p.h = w.h, p.hq = w.hq, p.hs = w.hs, p.y = w.y, p.err = err;
    p.yr = w.yr;
    p.pair_row = w.pair_row, p.n_rows = w.pair_row ? w.n_rows : w.T;
    p.x_row = w.x_stride ? w.x_stride : (size_t)m.d;
    p.dx_row = w.dx_stride ? w.dx_stride : (size_t)scale_pad(m.d / MIAG_QK);
    p.one = 1.0f;
    p.chunk = tok_chunk(w.P, m.E);
}

// Shared memory: head | item table | ring | activation region.  Every CTA
// gets the whole budget and splits it itself: the region for its largest
// chunk, the rest as ring stages.  Returns the stages a full 32-pair chunk
// leaves (the fewest any CTA gets).
static int geometry(GemvParams &p, bool gu) {
    const int Kb = gu ? p.m.d : p.m.eh;
    const int xs = scale_pad(Kb / MIAG_QK);
    p.x_stride = smem_stride((uint32_t)Kb);
    const long room =
        (long)kSmemBudget - kRingOff - (long)region_size(kTokChunk, true, p.x_stride, xs);
    return room > 0 ? (int)(room / kStageBytes) : 0;
}

// The dynamic shared-memory limit is an attribute of the kernel, shared by
// every context in the process, so it is raised to the whole budget rather
// than to one shape's need.
int gemv_setup_attributes(const Dims &m, const StoreLayout &lay) {
    GemvParams p{};
    p.m = m, p.lay = lay;
    if (lay.gu_rt > 255 || lay.dn_rt > 255) return -1;  // the item table packs rt in 8 bits
    if (geometry(p, true) < 2 || geometry(p, false) < 2) return -1;
    const auto attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
    if (cudaFuncSetAttribute(k_expert_mma<true, false>, attr, kSmemBudget) != cudaSuccess ||
        cudaFuncSetAttribute(k_expert_mma<true, true>, attr, kSmemBudget) != cudaSuccess ||
        cudaFuncSetAttribute(k_expert_mma<false, false>, attr, kSmemBudget) != cudaSuccess ||
        cudaFuncSetAttribute(k_expert_mma<false, true>, attr, kSmemBudget) != cudaSuccess)
        return -1;
    return 0;
}

// The prefill regime once an expert gets more than one n-tile of pairs on
// average.
static bool wide_regime(const Dims &m, const Work &w) { return wide_batch(w.P, m.E); }

static int grid_for(const Dims &m, int RT, int num_sms, int P) {
    // items <= RT * (chunks), chunks <= P / kTokChunkNarrow + (active experts)
    const long max_items = (long)RT * ((long)P / kTokChunkNarrow + m.E);
    return (int)(max_items < num_sms ? max_items : num_sms);
}

// The SM-share state of launch kind `kind` (gate/up, down x narrow, wide).
static void set_share(GemvParams &p, const Work &w, int num_sms, int kind) {
    p.share = w.shares ? reinterpret_cast<ShareState *>(w.shares) + kind : nullptr;
    p.num_sms = num_sms;
}

void launch_gateup(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w,
                   int num_sms, int *err, cudaStream_t s) {
    GemvParams p{};
    fill_params(p, m, lay, L, w, err);
    geometry(p, true);
    set_share(p, w, num_sms, 0 + (wide_regime(m, w) ? 1 : 0));
    const dim3 grid(grid_for(m, lay.gu_rt, num_sms, w.P));
    launch_dependent(wide_regime(m, w) ? k_expert_mma<true, true> : k_expert_mma<true, false>, grid,
                     dim3(kGemvThreads), kSmemBudget, s, p);
}

int down_launches(const Dims &m, int P) { return P > 0 && wide_batch(P, m.E) ? 2 : 1; }

void launch_down(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w,
                 int num_sms, int *err, cudaStream_t s) {
    if (w.P > 0 && wide_regime(m, w)) {  // decode: down forms the SwiGLU while staging
        const long tasks = (long)w.P * (m.eh / MIAG_QK) * 4;
        launch_dependent(k_swiglu_q8, dim3((unsigned)((tasks + 127) / 128)), dim3(128), 0, s, w.h,
                         w.P, m.eh, scale_pad(m.eh / MIAG_QK), w.hq, w.hs);
    }
    GemvParams p{};
    fill_params(p, m, lay, L, w, err);
    geometry(p, false);
    set_share(p, w, num_sms, 2 + (wide_regime(m, w) ? 1 : 0));
    const dim3 grid(grid_for(m, lay.dn_rt, num_sms, w.P));
    launch_dependent(wide_regime(m, w) ? k_expert_mma<false, true> : k_expert_mma<false, false>,
                     grid, dim3(kGemvThreads), kSmemBudget, s, p);
}

void launch_combine(const Dims &m, const Work &w, float *x, int *err, cudaStream_t s) {
    dim3 grid(w.T, (m.d / 4 + 127) / 128);
    launch_dependent(k_combine, grid, dim3(128), 0, s, x, m.d, m.K, w.w, w.y, w.y_pos,
                     (const int *)err);
}

}  // namespace miag
