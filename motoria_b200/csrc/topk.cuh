// topk.cuh -- softmax, top-k and renormalisation of one token, one warp.
//
// Reference: src/model/forward.c:176-181 -- softmax (:95-101: max, then
// e_i = expf(l_i - max) summed in index order, then p_i = e_i / sum), top_k
// by K rounds of first-maximum selection (:104-114, ties to the lower
// index), weights w_j = p_idx[j] renormalised by their in-order sum.
//
// expf is evaluated as the float nearest CUDA's double exp (expf_cr), which
// is glibc's expf except where glibc itself misrounds.  Selection runs on the
// probabilities like the reference: all p_i >= 0, so their IEEE bit patterns
// order like unsigned integers and one redux.sync max finds the round's
// winning value, one redux.sync min the lowest index holding it.  Lane l
// keeps entries l + 32u (u < NPL) in registers throughout.
#pragma once

#include "common.cuh"

namespace miag {

// buf: E floats of shared scratch for this warp (16-byte aligned).
// E <= 32 * NPL, K <= 64.
template <int NPL>
__device__ __forceinline__ void topk_warp(const float *logits, int E, int K, int norm_topk,
                                          int32_t *idx_out, float *w_out, float *buf, int lane) {
    constexpr uint32_t full = 0xffffffffu;
    // 1. logits (all loads in flight at once, through L2), max
    float v[NPL];
#pragma unroll
    for (int u = 0; u < NPL; u++) v[u] = lane + 32 * u < E ? __ldcg(logits + lane + 32 * u) : -INFINITY;
    float mx = v[0];
#pragma unroll
    for (int u = 1; u < NPL; u++) mx = fmaxf(mx, v[u]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(full, mx, o));
    // 2. exponentials, parked in shared memory for the ordered sum
#pragma unroll
    for (int u = 0; u < NPL; u++) {
        const bool in = lane + 32 * u < E;
        v[u] = in ? expf_cr(__fsub_rn(v[u], mx)) : 0.0f;
        if (in) buf[lane + 32 * u] = v[u];
    }
    __syncwarp();
    // 3. the sum in index order (forward.c:99), by lane 0, 32 values loaded
    // ahead of each run of 32 dependent adds
    float sum = 0.0f;
    if (lane == 0) {
        int e = 0;
        if ((E & 3) == 0) {
            for (; e + 32 <= E; e += 32) {
                float4 t[8];
#pragma unroll
                for (int u = 0; u < 8; u++) t[u] = *reinterpret_cast<const float4 *>(buf + e + 4 * u);
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    sum = __fadd_rn(sum, t[u].x);
                    sum = __fadd_rn(sum, t[u].y);
                    sum = __fadd_rn(sum, t[u].z);
                    sum = __fadd_rn(sum, t[u].w);
                }
            }
        }
        for (; e < E; e++) sum = __fadd_rn(sum, buf[e]);
    }
    sum = __shfl_sync(full, sum, 0);
    // 4. probabilities
#pragma unroll
    for (int u = 0; u < NPL; u++) v[u] = __fdiv_rn(v[u], sum);
    // 5. K rounds of selection.  Every lane learns each round's winning
    // value (the redux max), so the renormalising sum (forward.c:179-181)
    // accumulates in selection order as the rounds go.
    uint32_t taken = 0;
    int sel_lo = 0, sel_hi = 0;       // selection j kept by lane j % 32
    float w_lo = 0.0f, w_hi = 0.0f;
    float s = 0.0f;
    for (int j = 0; j < K; j++) {
        uint32_t best = 0, bidx = 0xffffffffu;
        bool have = false;
#pragma unroll
        for (int u = 0; u < NPL; u++) {
            const bool ok = lane + 32 * u < E && !((taken >> u) & 1u);
            const uint32_t bits = __float_as_uint(v[u]);
            if (ok && (!have || bits > best)) best = bits, bidx = (uint32_t)(lane + 32 * u), have = true;
        }
        const uint32_t gmax = __reduce_max_sync(full, have ? best : 0u);
        const uint32_t cand = (have && best == gmax) ? bidx : 0xffffffffu;
        const uint32_t win = __reduce_min_sync(full, cand);
        if ((int)(win & 31u) == lane) taken |= 1u << (win >> 5);
        const float wj = __uint_as_float(gmax);
        s = __fadd_rn(s, wj);
        if (lane == (j & 31)) {
            if (j < 32) sel_lo = (int)win, w_lo = wj;
            else sel_hi = (int)win, w_hi = wj;
        }
    }
    if (lane < K) {
        idx_out[lane] = sel_lo;
        w_out[lane] = norm_topk ? __fdiv_rn(w_lo, s) : w_lo;
    }
    if (lane + 32 < K) {
        idx_out[lane + 32] = sel_hi;
        w_out[lane + 32] = norm_topk ? __fdiv_rn(w_hi, s) : w_hi;
    }
    __syncwarp();
}

// Picks the register footprint for E (E <= 1024).
__device__ __forceinline__ void topk_warp_any(const float *logits, int E, int K, int norm_topk,
                                              int32_t *idx_out, float *w_out, float *buf,
                                              int lane) {
    if (E <= 128) topk_warp<4>(logits, E, K, norm_topk, idx_out, w_out, buf, lane);
    else if (E <= 256) topk_warp<8>(logits, E, K, norm_topk, idx_out, w_out, buf, lane);
    else topk_warp<32>(logits, E, K, norm_topk, idx_out, w_out, buf, lane);  // E <= 1024
}

}  // namespace miag
