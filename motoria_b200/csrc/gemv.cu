// gemv.cu -- grouped Q8_0 expert products for the decode regime.
//
// Reference: the three mia_matvec calls per active expert in moe()
// (src/model/forward.c:186-193) -> rows_kernel (src/tensor/matmul.c:75-80)
// -> dot_q8_scalar (:19-28); SwiGLU :188-191; re-quantization of h inside
// mia_matvec (:93, quant.c:11-27); weighted combine :194.
//
// Work is grouped by expert: every staged weight tile is read from HBM once
// and applied to all of that expert's (token, slot) pairs.  Persistent CTAs
// (one per SM) walk a list of items = (active expert, row chunk).  A producer
// warp streams each item's rows into a ring of shared-memory stages with
// 1-D TMA bulk copies (one copy per row, into bank-skewed row slots); eight
// consumer warps compute from shared memory.
//
// Lane <-> row: each lane owns one weight row and walks its Q8_0 blocks in
// order, so the fp32 sum is the reference's serial sum
//   s += ((float)int_dot * w.d) * x.d
// and the result equals mia_matvec_scalar bit for bit.
#include "kernels.cuh"

namespace miag {

constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kGuRowPairs = 8;             // gate/up rows per item: 8 gate + 8 up
constexpr int kGuRows = 2 * kGuRowPairs;
constexpr int kDnRows = 32;                // down rows per item
constexpr int kMaxStages = 8;
constexpr int kBarBytes = 256;
constexpr int kSmemBudget = 227 * 1024;

struct GemvParams {
    Dims m;
    StoreLayout lay;
    const uint8_t *experts;
    const int32_t *offsets, *perm, *active, *n_active;
    const int8_t *xq;  // [T][d]
    const float *dx;   // [T][xs]
    float *h;          // [P][eh]
    const int8_t *hq;  // [P][eh]
    const float *dh;   // [P][hs]
    float *y;          // [P][d]
    int stages;
    uint32_t q_stride, s_stride, stage_bytes;
    int *err;
};

struct GuTile {
    static constexpr int kRows = kGuRows;
    __device__ static int items_per_expert(const GemvParams &p) { return p.m.eh / kGuRowPairs; }
    __device__ static uint32_t q_bytes(const GemvParams &p) { return (uint32_t)p.m.d; }
    __device__ static uint32_t s_bytes(const GemvParams &p) { return p.lay.gu_s_row; }
    __device__ static size_t q_off(const GemvParams &p, int c) {
        return p.lay.gu_q_off + (size_t)c * kRows * p.m.d;
    }
    __device__ static size_t s_off(const GemvParams &p, int c) {
        return p.lay.gu_s_off + (size_t)c * kRows * p.lay.gu_s_row;
    }
};

struct DnTile {
    static constexpr int kRows = kDnRows;
    __device__ static int items_per_expert(const GemvParams &p) { return p.m.d / kDnRows; }
    __device__ static uint32_t q_bytes(const GemvParams &p) { return (uint32_t)p.m.eh; }
    __device__ static uint32_t s_bytes(const GemvParams &p) { return p.lay.dn_s_row; }
    __device__ static size_t q_off(const GemvParams &p, int c) {
        return p.lay.dn_q_off + (size_t)c * kRows * p.m.eh;
    }
    __device__ static size_t s_off(const GemvParams &p, int c) {
        return p.lay.dn_s_off + (size_t)c * kRows * p.lay.dn_s_row;
    }
};

// Serial reference dot of one staged weight row with one activation row.
__device__ __forceinline__ float row_dot(const uint8_t *qr, const float *sr, const int8_t *xr,
                                         const float *xs, int nb) {
    float acc = 0.0f;
    for (int b0 = 0; b0 < nb; b0 += 4) {
        const float4 ws = *reinterpret_cast<const float4 *>(sr + b0);
        const float4 xv = __ldg(reinterpret_cast<const float4 *>(xs + b0));
        const float wa[4] = {ws.x, ws.y, ws.z, ws.w};
        const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
        int dots[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (b0 + u < nb) {
                const int b = b0 + u;
                const int4 w0 = *reinterpret_cast<const int4 *>(qr + 32 * b);
                const int4 w1 = *reinterpret_cast<const int4 *>(qr + 32 * b + 16);
                const int4 x0 = ldg_nc_v4(xr + 32 * b);
                const int4 x1 = ldg_nc_v4(xr + 32 * b + 16);
                dots[u] = dot_block_i8(w0, w1, x0, x1);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (b0 + u < nb) acc = q8_step(acc, dots[u], wa[u], xa[u]);
    }
    return acc;
}

// Pipeline skeleton shared by the gate/up and down kernels.
template <class Tile, class Consume>
__device__ __forceinline__ void run_pipeline(const GemvParams &p, uint8_t *smem, Consume consume) {
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMaxStages;
    uint8_t *stages = smem + kBarBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.stages;
    const int ipe = Tile::items_per_expert(p);
    const int n_items = __ldg(p.n_active) * ipe;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    const uint32_t qb = Tile::q_bytes(p), sb = Tile::s_bytes(p);
    if (warp == kConsumerWarps) {
        // Producer warp.
        int it = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, it++) {
            const int s = it % S, round = it / S;
            if (round > 0) {
                bool got = true;
                if (lane == 0) got = mbar_wait(&empty[s], (round - 1) & 1);
                got = __shfl_sync(0xffffffffu, got, 0);
                if (!got) {
                    set_error(p.err, kErrWaitEmpty);
                    ok = false;
                    break;
                }
            }
            const int e = __ldg(p.active + item / ipe), c = item % ipe;
            const uint8_t *base = p.experts + (size_t)e * p.lay.expert_bytes;
            const uint8_t *src_q = base + Tile::q_off(p, c);
            const uint8_t *src_s = base + Tile::s_off(p, c);
            uint8_t *dst = stages + (size_t)s * p.stage_bytes;
            if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)Tile::kRows * (qb + sb));
            __syncwarp();
            for (int r = lane; r < Tile::kRows; r += 32) {
                bulk_g2s(dst + (size_t)r * p.q_stride, src_q + (size_t)r * qb, qb, &full[s]);
                bulk_g2s(dst + (size_t)Tile::kRows * p.q_stride + (size_t)r * p.s_stride,
                         src_s + (size_t)r * sb, sb, &full[s]);
            }
        }
        if (!ok && lane == 0) {
            // Let copies already issued land before the CTA's shared memory goes away.
            const int issued = it;
            for (int j = issued - 1; j >= 0 && j >= issued - S; j--)
                mbar_wait(&full[j % S], (j / S) & 1);
        }
        return;
    }

    // Consumer warps.
    int it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, it++) {
        const int s = it % S, round = it / S;
        bool got = true;
        if (lane == 0) got = mbar_wait(&full[s], round & 1);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
            set_error(p.err, kErrWaitFull);
            return;
        }
        const int e = __ldg(p.active + item / ipe), c = item % ipe;
        const uint8_t *stg = stages + (size_t)s * p.stage_bytes;
        consume(e, c, stg, stg + (size_t)Tile::kRows * p.q_stride, warp, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

__global__ void __launch_bounds__(kGemvThreads, 1) k_gateup(GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int d = p.m.d, eh = p.m.eh, K = p.m.K;
    const int nb = d / MIAG_QK, xs = scale_pad(nb);
    run_pipeline<GuTile>(p, smem, [&](int e, int c, const uint8_t *sq, const uint8_t *ss, int warp,
                                      int lane) {
        const int row = lane & 15, half = lane >> 4;
        const uint8_t *qr = sq + (size_t)row * p.q_stride;
        const float *sr = reinterpret_cast<const float *>(ss + (size_t)row * p.s_stride);
        const int seg0 = __ldg(p.offsets + e), n_e = __ldg(p.offsets + e + 1) - seg0;
        for (int k0 = 2 * warp; k0 < n_e; k0 += 2 * kConsumerWarps) {
            const int k = k0 + half;
            float acc = 0.0f;
            int pos = 0;
            if (k < n_e) {
                pos = seg0 + k;
                const int t = __ldg(p.perm + pos) / K;
                acc = row_dot(qr, sr, p.xq + (size_t)t * d, p.dx + (size_t)t * xs, nb);
            }
            const float up = __shfl_xor_sync(0xffffffffu, acc, 1);
            if (k < n_e && (row & 1) == 0)
                p.h[(size_t)pos * eh + c * kGuRowPairs + (row >> 1)] = swiglu_ref(acc, up);
        }
    });
}

__global__ void __launch_bounds__(kGemvThreads, 1) k_down(GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int d = p.m.d, eh = p.m.eh;
    const int nb = eh / MIAG_QK, hs = scale_pad(nb);
    run_pipeline<DnTile>(p, smem, [&](int e, int c, const uint8_t *sq, const uint8_t *ss, int warp,
                                      int lane) {
        const uint8_t *qr = sq + (size_t)lane * p.q_stride;
        const float *sr = reinterpret_cast<const float *>(ss + (size_t)lane * p.s_stride);
        const int seg0 = __ldg(p.offsets + e), n_e = __ldg(p.offsets + e + 1) - seg0;
        for (int k = warp; k < n_e; k += kConsumerWarps) {
            const int pos = seg0 + k;
            const float acc =
                row_dot(qr, sr, p.hq + (size_t)pos * eh, p.dh + (size_t)pos * hs, nb);
            p.y[(size_t)pos * d + c * kDnRows + lane] = acc;
        }
    });
}

// Q8_0 of each pair's h (quant.c:11-27), one warp per 32-block.
__global__ void k_quant_h(const float *h, int P, int eh, int8_t *hq, float *dh) {
    const int lane = threadIdx.x & 31;
    const int nb = eh / MIAG_QK, hs = scale_pad(nb);
    const long gw = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (gw >= (long)P * nb) return;
    const int pos = (int)(gw / nb), b = (int)(gw % nb);
    const float v = h[(size_t)pos * eh + b * MIAG_QK + lane];
    float a = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const float dq = __fdiv_rn(a, 127.0f);
    const float id = dq != 0.0f ? __fdiv_rn(1.0f, dq) : 0.0f;
    hq[(size_t)pos * eh + b * MIAG_QK + lane] = (int8_t)roundf(__fmul_rn(v, id));
    if (lane == 0) dh[(size_t)pos * hs + b] = dq;
}

// x[t] += w_j * y_j for j = 0..K-1 in order (forward.c:194).
__global__ void k_combine(float *x, int d, int K, const float *w, const int32_t *inv,
                          const float *y) {
    const int t = blockIdx.x;
    const int i = blockIdx.y * blockDim.x + threadIdx.x;
    if (i >= d) return;
    float v = x[(size_t)t * d + i];
    for (int j = 0; j < K; j++) {
        const int pos = __ldg(inv + (size_t)t * K + j);
        v = __fadd_rn(v, __fmul_rn(__ldg(w + (size_t)t * K + j), y[(size_t)pos * d + i]));
    }
    x[(size_t)t * d + i] = v;
}

static void fill_params(GemvParams &p, const Dims &m, const StoreLayout &lay, const LayerDev &L,
                        const Work &w, int *err) {
    p.m = m, p.lay = lay, p.experts = L.experts;
    p.offsets = w.offsets, p.perm = w.perm, p.active = w.active, p.n_active = w.n_active;
    p.xq = w.xq, p.dx = w.dx, p.h = w.h, p.hq = w.hq, p.dh = w.dh, p.y = w.y, p.err = err;
}

static void gu_geometry(GemvParams &p) {
    p.q_stride = smem_stride((uint32_t)p.m.d);
    p.s_stride = smem_stride(p.lay.gu_s_row);
    p.stage_bytes = (uint32_t)kGuRows * (p.q_stride + p.s_stride);
    int st = (kSmemBudget - kBarBytes) / (int)p.stage_bytes;
    p.stages = st > kMaxStages ? kMaxStages : st;
}

static void dn_geometry(GemvParams &p) {
    p.q_stride = smem_stride((uint32_t)p.m.eh);
    p.s_stride = smem_stride(p.lay.dn_s_row);
    p.stage_bytes = (uint32_t)kDnRows * (p.q_stride + p.s_stride);
    int st = (kSmemBudget - kBarBytes) / (int)p.stage_bytes;
    p.stages = st > kMaxStages ? kMaxStages : st;
}

int gemv_setup_attributes(const Dims &m, const StoreLayout &lay) {
    GemvParams p{};
    p.m = m, p.lay = lay;
    gu_geometry(p);
    if (p.stages < 2) return -1;
    size_t smem = kBarBytes + (size_t)p.stages * p.stage_bytes;
    if (cudaFuncSetAttribute(k_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return -1;
    dn_geometry(p);
    if (p.stages < 2) return -1;
    smem = kBarBytes + (size_t)p.stages * p.stage_bytes;
    if (cudaFuncSetAttribute(k_down, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return -1;
    return 0;
}

void launch_gateup(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w,
                   int num_sms, int *err, cudaStream_t s) {
    GemvParams p{};
    fill_params(p, m, lay, L, w, err);
    gu_geometry(p);
    const size_t smem = kBarBytes + (size_t)p.stages * p.stage_bytes;
    const int max_items = m.E * (m.eh / kGuRowPairs);
    const int grid = num_sms < max_items ? num_sms : max_items;
    k_gateup<<<grid, kGemvThreads, smem, s>>>(p);
}

void launch_down(const Dims &m, const StoreLayout &lay, const LayerDev &L, const Work &w,
                 int num_sms, int *err, cudaStream_t s) {
    GemvParams p{};
    fill_params(p, m, lay, L, w, err);
    dn_geometry(p);
    const size_t smem = kBarBytes + (size_t)p.stages * p.stage_bytes;
    const int max_items = m.E * (m.d / kDnRows);
    const int grid = num_sms < max_items ? num_sms : max_items;
    k_down<<<grid, kGemvThreads, smem, s>>>(p);
}

void launch_quant_h(const Dims &m, const Work &w, cudaStream_t s) {
    const long warps = (long)w.P * (m.eh / MIAG_QK);
    const long blocks = (warps * 32 + 255) / 256;
    k_quant_h<<<(unsigned)blocks, 256, 0, s>>>(w.h, w.P, m.eh, w.hq, w.dh);
}

void launch_combine(const Dims &m, const Work &w, float *x, cudaStream_t s) {
    dim3 grid(w.T, (m.d + 255) / 256);
    k_combine<<<grid, 256, 0, s>>>(x, m.d, m.K, w.w, w.inv, w.y);
}

}  // namespace miag
