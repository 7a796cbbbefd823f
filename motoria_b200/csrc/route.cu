// route.cu -- rmsnorm + activation quantization + router + softmax/top-k.
//
// Reference: src/model/forward.c:174-181 (rmsnorm :75-81, router matvec
// src/tensor/matmul.c:13-17, softmax :95-101, top_k :104-114) and the
// activation quantizer src/tensor/quant.c:11-27 that mia_matvec applies to
// xn before the expert gate/up products (matmul.c:93).
//
// Grid: (token groups of R, expert groups of 32).  Each CTA is one warp:
//   1. rmsnorm of its R tokens into shared memory, certified to equal the
//      reference's serial double sum (see rms_scale);
//   2. expert-group 0 quantizes xn to Q8_0 for the expert GEMVs;
//   3. lane e computes the router logit of expert 32*eg + e for the R tokens
//      as the reference's serial fp32 sum (rounded multiply, then rounded
//      add, i = 0..d-1 in order; f32x2 instructions round each half exactly
//      like the scalar ones);
//   4. the last CTA of a token group to finish (atomic ticket, no waiting)
//      runs softmax, top-k and renormalisation for the group.
#include "kernels.cuh"

namespace miag {

// (float)(1.0 / sqrt(ss / n + eps)) in IEEE double, as forward.c:79.
__device__ __forceinline__ float rms_scale_of(double ss, int n, float eps) {
    double q = __dadd_rn(__ddiv_rn(ss, (double)n), (double)eps);
    return __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(q)));
}

// The reference sums x_i^2 serially in double (forward.c:78).  Each square is
// exact in double and all terms are >= 0, so any summation order lands
// within (n-1)*2^-53 relative of the exact sum, and so does the reference's.
// The warp-parallel sum therefore brackets the reference's value; the scale
// is monotone in the sum, so when both ends of the bracket give the same
// float the reference's float is that one.  Otherwise (probability ~1e-5)
// lane 0 repeats the serial sum.
__device__ float rms_scale(const float *x, int n, float eps, int lane) {
    double ss = 0.0;
    for (int i = lane; i < n; i += 32) {
        double v = (double)x[i];
        ss = __dadd_rn(ss, __dmul_rn(v, v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    float r = 0.0f;
    if (lane == 0) {
        const double rel = (2.02 * (double)n + 8.0) * 1.1102230246251565e-16;  // 2^-53
        float a = rms_scale_of(ss * (1.0 - rel), n, eps);
        float b = rms_scale_of(ss * (1.0 + rel), n, eps);
        if (a == b) {
            r = a;
        } else {
            double s2 = 0.0;
            for (int i = 0; i < n; i++) {
                double v = (double)x[i];
                s2 = __dadd_rn(s2, __dmul_rn(v, v));
            }
            r = rms_scale_of(s2, n, eps);
        }
    }
    return __shfl_sync(0xffffffffu, r, 0);
}

struct RouteParams {
    Dims m;
    LayerDev L;
    const float *x;      // [T][d]
    int T;
    int8_t *xq;          // [T][d]
    float *dx;           // [T][xs_pad]
    float *logits;       // [T][E]
    int32_t *ticket;     // [ceil(T/R)]
    int32_t *idx;        // [T][K]
    float *w;            // [T][K]
    int *err;
};

// Softmax, top-k and renormalisation of one token's logits (one warp).
__device__ void topk_token(const RouteParams &p, int t, float *buf, int lane) {
    const int E = p.m.E, K = p.m.K;
    const float *lg = p.logits + (size_t)t * E;
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, __ldcg(lg + e));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int e = lane; e < E; e += 32) buf[e] = expf_cr(__fsub_rn(__ldcg(lg + e), mx));
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0)
        for (int e = 0; e < E; e++) sum = __fadd_rn(sum, buf[e]);  // forward.c:99 order
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int e = lane; e < E; e += 32) buf[e] = __fdiv_rn(buf[e], sum);
    __syncwarp();
    // K rounds of first-maximum selection (forward.c:104-114): ties go to the
    // lower index; `taken` bit k of a lane marks expert lane + 32k.
    uint32_t taken = 0;
    int sel[64];
    for (int j = 0; j < K; j++) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int e = lane, k = 0; e < E; e += 32, k++) {
            float v = buf[e];
            if (!((taken >> k) & 1u) && (bi == 0x7fffffff || v > bv)) bv = v, bi = e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            bool take = (oi != 0x7fffffff) &&
                        (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi));
            if (take) bv = ov, bi = oi;
        }
        sel[j] = bi;
        if (bi != 0x7fffffff && (bi & 31) == lane) taken |= 1u << (bi >> 5);
    }
    if (lane == 0) {
        float s = 0.0f, wv[64];
        for (int j = 0; j < K; j++) {
            wv[j] = buf[sel[j]];
            s = __fadd_rn(s, wv[j]);  // forward.c:179
        }
        for (int j = 0; j < K; j++) {
            p.idx[(size_t)t * K + j] = sel[j];
            p.w[(size_t)t * K + j] = p.m.norm_topk ? __fdiv_rn(wv[j], s) : wv[j];
        }
    }
    __syncwarp();
}

template <int R>
__global__ void __launch_bounds__(32) k_route(RouteParams p) {
    extern __shared__ __align__(16) float sm[];  // xn [d][R], then E floats of top-k scratch
    const int d = p.m.d, E = p.m.E, lane = threadIdx.x;
    const int t0 = blockIdx.x * R;
    const int nt = min(R, p.T - t0);
    float *xn = sm;

    // 1. rmsnorm of the group's tokens (forward.c:75-81 with w = ffn_norm).
    for (int r = 0; r < R; r++) {
        if (r < nt) {
            const float *x = p.x + (size_t)(t0 + r) * d;
            float inv = rms_scale(x, d, p.m.eps, lane);
            for (int i = lane; i < d; i += 32)
                xn[i * R + r] = __fmul_rn(__fmul_rn(x[i], inv), p.L.ffn_norm[i]);
        } else {
            for (int i = lane; i < d; i += 32) xn[i * R + r] = 0.0f;
        }
    }
    __syncwarp();

    // 2. Q8_0 of xn (quant.c:11-27), once per token.
    if (blockIdx.y == 0) {
        const int nb = d / MIAG_QK, xs = scale_pad(nb);
        for (int r = 0; r < nt; r++) {
            for (int b = 0; b < nb; b++) {
                float v = xn[(b * MIAG_QK + lane) * R + r];
                float a = fabsf(v);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
                float dq = __fdiv_rn(a, 127.0f);
                float id = dq != 0.0f ? __fdiv_rn(1.0f, dq) : 0.0f;
                p.xq[(size_t)(t0 + r) * d + b * MIAG_QK + lane] = (int8_t)roundf(__fmul_rn(v, id));
                if (lane == 0) p.dx[(size_t)(t0 + r) * xs + b] = dq;
            }
        }
    }

    // 3. Router logits, serial over i like dot_f32_scalar (matmul.c:13-17).
    const int e = blockIdx.y * 32 + lane;
    if (e < E) {
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = 0.0f;
        const float *wt = p.L.router_t + e;
        int i = 0;
        for (; i + 8 <= d; i += 8) {
            float wv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) wv[u] = __ldg(wt + (size_t)(i + u) * E);
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float *xv = xn + (i + u) * R;
#pragma unroll
                for (int r = 0; r + 1 < R; r += 2) {
                    float2 pr = __fmul2_rn(make_float2(wv[u], wv[u]), make_float2(xv[r], xv[r + 1]));
                    float2 a2 = __fadd2_rn(make_float2(acc[r], acc[r + 1]), pr);
                    acc[r] = a2.x, acc[r + 1] = a2.y;
                }
                if (R & 1) acc[R - 1] = __fadd_rn(acc[R - 1], __fmul_rn(wv[u], xv[R - 1]));
            }
        }
        for (; i < d; i++) {
            float wv = __ldg(wt + (size_t)i * E);
#pragma unroll
            for (int r = 0; r < R; r++) acc[r] = __fadd_rn(acc[r], __fmul_rn(wv, xn[i * R + r]));
        }
        for (int r = 0; r < nt; r++) {
            float l = acc[r];
            if (p.L.bias) l = __fadd_rn(l, p.L.bias[e]);
            p.logits[(size_t)(t0 + r) * E + e] = l;
        }
    }

    // 4. Last CTA of the token group runs softmax/top-k.
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(p.ticket + blockIdx.x, 1) == (int)gridDim.y - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    float *buf = sm + (size_t)d * R;
    for (int r = 0; r < nt; r++) topk_token(p, t0 + r, buf, lane);
    if (lane == 0) p.ticket[blockIdx.x] = 0;
}

int route_group(int T) { return T <= 256 ? 2 : (T <= 1024 ? 4 : 8); }

void launch_route(const Dims &m, const LayerDev &L, const float *x, const Work &w, int *err,
                  cudaStream_t s) {
    RouteParams p;
    p.m = m, p.L = L, p.x = x, p.T = w.T;
    p.xq = w.xq, p.dx = w.dx, p.logits = w.logits, p.ticket = w.ticket;
    p.idx = w.idx, p.w = w.w, p.err = err;
    const int R = route_group(w.T);
    dim3 grid((w.T + R - 1) / R, (m.E + 31) / 32);
    size_t smem = ((size_t)m.d * R + (size_t)m.E) * sizeof(float);
    switch (R) {
        case 2:
            cudaFuncSetAttribute(k_route<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            k_route<2><<<grid, 32, smem, s>>>(p);
            break;
        case 4:
            cudaFuncSetAttribute(k_route<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            k_route<4><<<grid, 32, smem, s>>>(p);
            break;
        default:
            cudaFuncSetAttribute(k_route<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            k_route<8><<<grid, 32, smem, s>>>(p);
            break;
    }
}

}  // namespace miag
