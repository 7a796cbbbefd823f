// route.cu -- rmsnorm + activation quantization + router logits + top-k.
//
// Reference: src/model/forward.c:174-181 (rmsnorm :75-81, router matvec
// src/tensor/matmul.c:13-17, softmax :95-101, top_k :104-114) and the
// activation quantizer src/tensor/quant.c:11-27 that mia_matvec applies to
// xn before the expert gate/up products (matmul.c:93).
//
// Grid: (token groups, expert groups of 32).  A CTA has W consumer warps,
// each owning R tokens, and one producer warp:
//   1. each warp rmsnorms its tokens into shared memory, certified to equal
//      the reference's serial double sum (see rms_scale);
//   2. the expert groups' CTAs quantize xn to Q8_0 for the expert GEMVs,
//      each a share of the blocks, once the router logits (3.) are out: a
//      warp quantizes the rows of the warp half a CTA away;
//   3. lane e computes the router logit of expert 32*eg + e for the warp's
//      tokens as the reference's serial fp32 sum (rounded multiply, then
//      rounded add, i = 0..d-1 in order).  The group's router slice, stored
//      [group][i/4][32][4] so it is contiguous, streams through a ring of
//      shared-memory chunks that the producer fills with 1-D TMA bulk copies
//      and all consumer warps read;
//   4. the last CTA of a token group to finish (a counter per group) runs
//      softmax, top-k and renormalisation for the group's tokens (topk.cuh),
//      one warp per token.
#include "kernels.cuh"
#include "topk.cuh"

namespace miag {

struct RouteParams {
    Dims m;
    LayerDev L;
    const float *x;      // [T][d]
    int T;
    int8_t *xq;          // [T][d]
    float *dx;           // [T][xs_pad]
    float *logits;       // [T][E]
    int32_t *idx;        // [T][K]  top-k experts
    float *w;            // [T][K]  their weights
    int32_t *tg_count;   // [token groups]: zero between calls
    int *err;
};

constexpr int kRouteChunk = 256;  // router rows per bulk copy: 256 x 128 B = 32 KiB
constexpr int kRouteStages = 4;   // ring depth at most (a launch may use fewer)

// Shared memory: barriers | ring [stages][kRouteChunk][32] f32 |
// x, then xn in place [W*R][d] f32 | ffn_norm [d] f32.  After the router loop
// the ring is free and holds the top-k scratch, E floats per warp.
constexpr int kRouteBarBytes = 256;
__host__ __device__ inline size_t route_smem(int d, int R, int W, int stages) {
    return kRouteBarBytes + (size_t)stages * kRouteChunk * 128 + (size_t)W * R * d * 4 +
           (size_t)d * 4;
}

// Router rows of a chunk for R tokens, `groups` groups of four rows:
// acc[r] += w_i * xn[r][i] in order, each product and sum rounded
// (matmul.c:13-17), with scalar round-to-nearest intrinsics, which the
// compiler never fuses.  w4: this lane's weights of row group g at w4[32 g]
// (one 16-byte load).  The chain of adds is serial, so the products of the
// next group are formed between the adds of this one: on B200 the loop alone
// measured 5.8 cycles a row for one token, against 9 with the four rows'
// loads and products in line and 5.2 for the bare chain of adds.
template <int R, int kGroups = 0>  // kGroups > 0: a compile-time group count, fully unrolled
__device__ __forceinline__ void router_chunk(float (&acc)[R], const float4 *w4, const float *xc,
                                             int d, int groups_rt) {
    const int groups = kGroups > 0 ? kGroups : groups_rt;
    float p[R][4];
    {
        const float4 w = w4[0];
#pragma unroll
        for (int r = 0; r < R; r++) {
            const float4 xv = *reinterpret_cast<const float4 *>(xc + (size_t)r * d);
            p[r][0] = __fmul_rn(w.x, xv.x), p[r][1] = __fmul_rn(w.y, xv.y);
            p[r][2] = __fmul_rn(w.z, xv.z), p[r][3] = __fmul_rn(w.w, xv.w);
        }
    }
#pragma unroll (kGroups > 0 ? kGroups : 16)
    for (int g = 1; g < groups; g++) {
        const float4 w = w4[g * 32];
        float4 xv[R];
#pragma unroll
        for (int r = 0; r < R; r++) xv[r] = *reinterpret_cast<const float4 *>(xc + (size_t)r * d + 4 * g);
#pragma unroll
        for (int r = 0; r < R; r++) {
            acc[r] = __fadd_rn(acc[r], p[r][0]);
            const float q0 = __fmul_rn(w.x, xv[r].x);
            acc[r] = __fadd_rn(acc[r], p[r][1]);
            const float q1 = __fmul_rn(w.y, xv[r].y);
            acc[r] = __fadd_rn(acc[r], p[r][2]);
            const float q2 = __fmul_rn(w.z, xv[r].z);
            acc[r] = __fadd_rn(acc[r], p[r][3]);
            const float q3 = __fmul_rn(w.w, xv[r].w);
            p[r][0] = q0, p[r][1] = q1, p[r][2] = q2, p[r][3] = q3;
        }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
        acc[r] = __fadd_rn(acc[r], p[r][0]);
        acc[r] = __fadd_rn(acc[r], p[r][1]);
        acc[r] = __fadd_rn(acc[r], p[r][2]);
        acc[r] = __fadd_rn(acc[r], p[r][3]);
    }
}

// Grid: (token groups of W*R, expert groups of 32); W consumer warps own R
// tokens each and load them themselves; one producer warp streams the
// group's router slice.  The last of a token group's CTAs to finish its
// logits also runs softmax / top-k / renormalisation for the group's tokens.
template <int R>
__global__ void __launch_bounds__(9 * 32, 1) k_route(RouteParams p, int W, int stages) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int d = p.m.d, E = p.m.E;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kRouteStages;
    int *last_flag = reinterpret_cast<int *>(empty + kRouteStages);
    float *ring = reinterpret_cast<float *>(smem + kRouteBarBytes);
    float *xs_all = ring + (size_t)stages * kRouteChunk * 32;  // [W*R][d]
    float *norm = xs_all + (size_t)W * R * d;
    const int nchunks = (d + kRouteChunk - 1) / kRouteChunk;
    const float *slice = p.L.router_t + (size_t)blockIdx.y * d * 32;
    const int tg0 = blockIdx.x * W * R;                 // first token of the CTA

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == W) {
        // (the router is the layer's own: streamed before the previous
        // kernel of the stream has finished)
        // Producer: the router chunks, 32 KiB bulk copies (on B200 a bulk copy
        // occupies the copy engine ~0.26 us whatever its size up to ~8 KiB,
        // so small chunks cap the SM's ingest).
        if (lane == 0) {
            for (int ch = 0; ch < nchunks; ch++) {
                const int s = ch % stages, round = ch / stages;
                if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1)) {
                    set_error(p.err, kErrWaitEmpty);
                    for (int j = ch - 1; j >= 0 && j >= ch - stages; j--)
                        mbar_wait(&full[j % stages], (j / stages) & 1);
                    break;
                }
                const int rows = min(kRouteChunk, d - ch * kRouteChunk);
                const uint32_t bytes = (uint32_t)rows * 128u;
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(ring + (size_t)s * kRouteChunk * 32,
                         slice + (size_t)ch * kRouteChunk * 32, bytes, &full[s]);
            }
        }
        return;
    }

    // the layer's ffn_norm is constant: loaded before the wait (shared by the
    // consumer warps)
    {
        const float4 *src = reinterpret_cast<const float4 *>(p.L.ffn_norm);
        float4 *dst = reinterpret_cast<float4 *>(norm);
        const int stride = 32 * W;
        for (int i0 = warp * 32 + lane; i0 < d / 4; i0 += 4 * stride) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (i0 + stride * u < d / 4) v[u] = __ldg(src + i0 + stride * u);
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (i0 + stride * u < d / 4) dst[i0 + stride * u] = v[u];
        }
    }
    pdl_wait();  // x, and the counters and outputs the previous call used
    const int tw0 = tg0 + warp * R;  // this warp's first token
    const int nt = max(0, min(R, p.T - tw0));
    float *xw = xs_all + (size_t)warp * R * d;  // this warp's rows: x, then xn in place
    bool failed = false;
    // The warp's token rows and the shared ffn_norm come in through plain
    // coalesced loads: with these rows bulk-copied instead, the norm and the
    // router loop that follow measured 2-2.5x slower on B200.
    // Loads go out sixteen at a time before their stores, so a row of up to
    // 2048 costs one memory latency.
    for (int r = 0; r < nt; r++) {
        const float4 *src = reinterpret_cast<const float4 *>(p.x + (size_t)(tw0 + r) * d);
        float4 *dst = reinterpret_cast<float4 *>(xw + (size_t)r * d);
        for (int i0 = lane; i0 < d / 4; i0 += 16 * 32) {
            float4 v[16];
#pragma unroll
            for (int u = 0; u < 16; u++)
                if (i0 + 32 * u < d / 4) v[u] = __ldg(src + i0 + 32 * u);
#pragma unroll
            for (int u = 0; u < 16; u++)
                if (i0 + 32 * u < d / 4) dst[i0 + 32 * u] = v[u];
        }
    }
    named_barrier_sync(1, W * 32);  // consumer warps only
    // 1. rmsnorm (forward.c:75-81).  Lane l holds elements 4l + 128k
    // (k < d/128) of a token: eight lanes cover one 32-block, so the Q8_0
    // block maxima of phase 2 take three shuffles.
    const int nq4 = d / 128;  // float4 per lane (d is a multiple of 32; see tail)
    for (int r = 0; r < nt; r++) {
        float *xr = xw + (size_t)r * d;
        // four independent partial sums: the certified bracket covers any order
        double s4[4] = {0.0, 0.0, 0.0, 0.0};
        for (int k = 0; k < nq4; k++) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + 4 * lane + 128 * k);
            s4[0] = __dadd_rn(s4[0], __dmul_rn((double)v.x, (double)v.x));
            s4[1] = __dadd_rn(s4[1], __dmul_rn((double)v.y, (double)v.y));
            s4[2] = __dadd_rn(s4[2], __dmul_rn((double)v.z, (double)v.z));
            s4[3] = __dadd_rn(s4[3], __dmul_rn((double)v.w, (double)v.w));
        }
        for (int i = 128 * nq4 + lane; i < d; i += 32) {  // d % 128 tail
            const double v = (double)xr[i];
            s4[0] = __dadd_rn(s4[0], __dmul_rn(v, v));
        }
        const double ss = __dadd_rn(__dadd_rn(s4[0], s4[1]), __dadd_rn(s4[2], s4[3]));
        const float inv = rms_scale_certified(ss, xr, d, p.m.eps, lane);
        // xn in place (its Q8_0 comes after the router logits)
#pragma unroll 4
        for (int k = 0; k < nq4; k++) {
            const int i = 4 * lane + 128 * k;
            float4 v = *reinterpret_cast<const float4 *>(xr + i);
            const float4 w = *reinterpret_cast<const float4 *>(norm + i);
            v.x = __fmul_rn(__fmul_rn(v.x, inv), w.x);
            v.y = __fmul_rn(__fmul_rn(v.y, inv), w.y);
            v.z = __fmul_rn(__fmul_rn(v.z, inv), w.z);
            v.w = __fmul_rn(__fmul_rn(v.w, inv), w.w);
            *reinterpret_cast<float4 *>(xr + i) = v;
        }
        for (int i = 128 * nq4 + lane; i < d; i += 32) {  // tail (d % 128 == 32, 64, 96)
            xr[i] = __fmul_rn(__fmul_rn(xr[i], inv), norm[i]);
        }
    }
    __syncwarp();

    // 3. Router logits, serial over i like dot_f32_scalar (matmul.c:13-17).
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = 0.0f;
    for (int ch = 0; ch < nchunks; ch++) {
        const int s = ch % stages;
        if (!failed) {
            bool got = true;
            if (lane == 0) got = mbar_wait(&full[s], (ch / stages) & 1);
            if (!__shfl_sync(0xffffffffu, got, 0)) {
                set_error(p.err, kErrWaitFull);
                failed = true;
            }
        }
        const float4 *w4 = reinterpret_cast<const float4 *>(ring + (size_t)s * kRouteChunk * 32) + lane;
        const float *xc = xw + (size_t)ch * kRouteChunk;
        // a warp past the last token only keeps the ring turning; rows is a
        // multiple of four (d is a multiple of 32)
        const int rows = nt > 0 ? min(kRouteChunk, d - ch * kRouteChunk) : 0;
        // full chunks in straight-line code: with a remainder loop after an
        // unrolled body the loop ran at ~9.7 cycles a row on B200
        if (rows == kRouteChunk) router_chunk<R, kRouteChunk / 4>(acc, w4, xc, d, kRouteChunk / 4);
        else if (rows > 0) router_chunk<R>(acc, w4, xc, d, rows / 4);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    const int e = blockIdx.y * 32 + lane;
    if (e < E) {
        for (int r = 0; r < nt; r++) {
            float l = acc[r];
            if (p.L.bias) l = __fadd_rn(l, p.L.bias[e]);
            p.logits[(size_t)(tw0 + r) * E + e] = l;
        }
    }

    // 4. Softmax, top-k, renormalisation (forward.c:176-181), by the token
    // group's last CTA once all expert groups' logits are out.  Writers fence
    // before counting; the last one fences after, then reads through L2.
    __threadfence();
    named_barrier_sync(1, W * 32);
    if (threadIdx.x == 0) {
        const int before = atomicAdd(&p.tg_count[blockIdx.x], 1);
        const int last = before == (int)gridDim.y - 1;
        if (last) p.tg_count[blockIdx.x] = 0;  // back to zero for the next call
        *last_flag = last;
    }
    named_barrier_sync(1, W * 32);
    // 2. Q8_0 of xn (quant.c:11-27) for the expert products, which read it
    // only after this launch: each warp quantizes the rows of the warp half a
    // CTA away, so that with one token (the other warp idle) the quantization
    // runs beside the last CTA's top-k instead of before the router adds.
    // The expert-group CTAs of a token share it: group g takes every G-th run
    // of four float4 per lane (16 blocks); the d % 128 tail blocks go to
    // group 0, one warp-wide pass per 32-block.
    {
        const int qw = (warp + (W + 1) / 2) % W;
        const int tq0 = tg0 + qw * R;
        const int nqt = max(0, min(R, p.T - tq0));
        const int xs = scale_pad(d / MIAG_QK);
        for (int r = 0; r < nqt; r++) {
            const int t = tq0 + r;
            const float *xr = xs_all + ((size_t)qw * R + r) * d;
            for (int k0 = 4 * (int)blockIdx.y; k0 < nq4; k0 += 4 * (int)gridDim.y) {
                float4 v[4];
                float a[4], dq[4], id[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    v[u] = k0 + u < nq4 ? *reinterpret_cast<const float4 *>(xr + 4 * lane + 128 * (k0 + u))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
                    a[u] = fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w)));
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1)
#pragma unroll
                    for (int u = 0; u < 4; u++) a[u] = fmaxf(a[u], __shfl_xor_sync(0xffffffffu, a[u], o));
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    dq[u] = __fdiv_rn(a[u], 127.0f);
                    id[u] = dq[u] != 0.0f ? __fdiv_rn(1.0f, dq[u]) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    if (k0 + u >= nq4) break;
                    const int i = 4 * lane + 128 * (k0 + u);
                    const uint32_t q0 = (uint8_t)(int8_t)roundf(__fmul_rn(v[u].x, id[u]));
                    const uint32_t q1 = (uint8_t)(int8_t)roundf(__fmul_rn(v[u].y, id[u]));
                    const uint32_t q2 = (uint8_t)(int8_t)roundf(__fmul_rn(v[u].z, id[u]));
                    const uint32_t q3 = (uint8_t)(int8_t)roundf(__fmul_rn(v[u].w, id[u]));
                    *reinterpret_cast<uint32_t *>(p.xq + (size_t)t * d + i) =
                        q0 | (q1 << 8) | (q2 << 16) | (q3 << 24);
                    if ((lane & 7) == 0) p.dx[(size_t)t * xs + i / MIAG_QK] = dq[u];
                }
            }
            if (blockIdx.y == 0 && 128 * nq4 < d) {
                for (int b = 4 * nq4; b < d / MIAG_QK; b++) {
                    const float v = xr[b * MIAG_QK + lane];
                    float a = fabsf(v);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
                    const float dq = __fdiv_rn(a, 127.0f);
                    const float id = dq != 0.0f ? __fdiv_rn(1.0f, dq) : 0.0f;
                    p.xq[(size_t)t * d + b * MIAG_QK + lane] = (int8_t)roundf(__fmul_rn(v, id));
                    if (lane == 0) p.dx[(size_t)t * xs + b] = dq;
                }
            }
        }
    }
    if (!*last_flag) return;
    __threadfence();
    float *buf = ring + (size_t)warp * E;  // the ring is idle now: every chunk was consumed
    for (int r = 0; r < nt; r++) {
        const int t = tw0 + r;
        topk_warp_any(p.logits + (size_t)t * E, E, p.m.K, p.m.norm_topk,
                      p.idx + (size_t)t * p.m.K, p.w + (size_t)t * p.m.K, buf, lane);
    }
}

// Tokens per warp R, consumer warps W and ring depth by batch size.  The
// warps of a CTA all read each router row from shared memory, and four of
// them (with the ring's own fill) saturate it, so few-token batches use two
// warps of one token each and more CTAs.  Larger batches put more tokens on
// a warp, which reads a row once for all of them; their rows then take the
// shared memory a deeper ring would.
static void route_shape(int T, int &R, int &W, int &stages) {
    if (T <= 128) R = 1, W = 2, stages = 4;
    else R = 2, W = 8, stages = 2;  // B200 sweep at T = 300..2048: best of R 2-4, W 1-8
}

template <int R>
static void launch_r(const RouteParams &p, dim3 grid, int W, int stages, size_t smem,
                     cudaStream_t s) {
    cudaFuncSetAttribute(k_route<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_dependent(k_route<R>, grid, dim3((W + 1) * 32), smem, s, p, W, stages);
}

void launch_route(const Dims &m, const LayerDev &L, const float *x, const Work &w, int *err,
                  cudaStream_t s) {
    RouteParams p;
    p.m = m, p.L = L, p.x = x, p.T = w.T;
    p.xq = w.xq, p.dx = w.dx, p.logits = w.logits, p.idx = w.idx, p.w = w.w;
    p.tg_count = w.tg_count, p.err = err;
    int R, W, stages;
    route_shape(w.T, R, W, stages);
    const dim3 grid((w.T + R * W - 1) / (R * W), (m.E + 31) / 32);
    const size_t smem = route_smem(m.d, R, W, stages);
    if (R == 1) launch_r<1>(p, grid, W, stages, smem, s);
    else if (R == 2) launch_r<2>(p, grid, W, stages, smem, s);
    else launch_r<4>(p, grid, W, stages, smem, s);
}

}  // namespace miag
