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
// winning value, one redux.sync min the lowest index holding it.
#pragma once

#include "common.cuh"

namespace miag {

// buf: E floats of shared scratch for this warp.  K <= 64, E <= 1024.
__device__ __forceinline__ void topk_warp(const float *logits, int E, int K, int norm_topk,
                                          int32_t *idx_out, float *w_out, float *buf, int lane) {
    constexpr uint32_t full = 0xffffffffu;
    // 1. max, then exponentials (four per lane in flight).
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) {
        const float l = __ldcg(logits + e);
        buf[e] = l;
        mx = fmaxf(mx, l);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(full, mx, o));
    for (int e0 = lane; e0 < E; e0 += 128) {
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int e = e0 + 32 * u;
            v[u] = e < E ? expf_cr(__fsub_rn(buf[e], mx)) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (e0 + 32 * u < E) buf[e0 + 32 * u] = v[u];
    }
    __syncwarp();
    // 2. the sum in index order (forward.c:99), by lane 0.
    float sum = 0.0f;
    if (lane == 0) {
        int e = 0;
        for (; e + 8 <= E; e += 8) {
            float t[8];
#pragma unroll
            for (int u = 0; u < 8; u++) t[u] = buf[e + u];
#pragma unroll
            for (int u = 0; u < 8; u++) sum = __fadd_rn(sum, t[u]);
        }
        for (; e < E; e++) sum = __fadd_rn(sum, buf[e]);
    }
    sum = __shfl_sync(full, sum, 0);
    // 3. probabilities; lane keeps bit patterns of its entries lane + 32k.
    for (int e = lane; e < E; e += 32) buf[e] = __fdiv_rn(buf[e], sum);
    __syncwarp();
    // 4. K rounds of selection.
    uint32_t taken = 0;
    int sel_lo = 0, sel_hi = 0;  // selection j kept by lane j % 32
    for (int j = 0; j < K; j++) {
        uint32_t best = 0, bidx = 0xffffffffu;
        bool have = false;
        for (int e = lane, k = 0; e < E; e += 32, k++) {
            if ((taken >> k) & 1u) continue;
            const uint32_t bits = __float_as_uint(buf[e]);
            if (!have || bits > best) best = bits, bidx = (uint32_t)e, have = true;
        }
        const uint32_t gmax = __reduce_max_sync(full, have ? best : 0u);
        const uint32_t cand = (have && best == gmax) ? bidx : 0xffffffffu;
        const uint32_t win = __reduce_min_sync(full, cand);
        if ((int)(win & 31u) == lane) taken |= 1u << (win >> 5);
        if (lane == (j & 31)) {
            if (j < 32) sel_lo = (int)win;
            else sel_hi = (int)win;
        }
    }
    // 5. weights, renormalised by their in-order sum (forward.c:179-181).
    const float w_lo = lane < K ? buf[sel_lo] : 0.0f;
    const float w_hi = lane + 32 < K ? buf[sel_hi] : 0.0f;
    float s = 0.0f;
    for (int j = 0; j < K; j++) {
        const float wj = __shfl_sync(full, j < 32 ? w_lo : w_hi, j & 31);
        s = __fadd_rn(s, wj);
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

}  // namespace miag
