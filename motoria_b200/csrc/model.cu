// model.cu -- the whole decode step on the GPU: the reference's model state
// and layer loop (mia_model_init / mia_model_step, src/model/forward.c:
// 36-62 and 199-217) with every weight, the KV cache and the MoE experts
// resident in HBM.
//
// One step = one token at one position, as mia_model_step:
//   embed      x = dequant(token_embd[token])                   (:205-208)
//   per layer  attention (:118-165), then the MoE block (:167-197) through
//              the context's own launch sequence (miag_moe_async, T = 1)
//   head       logits = output . rmsnorm(x, output_norm)         (:214-215)
// Launches per step: 1 + n_layers * (3 + the MoE block's) + 1, each with
// programmatic dependent launch, captured once into a CUDA graph and
// replayed; the step's token and position live in device memory, so the
// same graph serves every position.  The head's last CTA also picks the
// next token (the next prompt token, else the greedy argmax) and advances
// the position, so a whole prompt + generation runs as graph replays with
// no host round trip.
//
// Arithmetic is the reference's, operation for operation (x86 scalar build,
// no FMA contraction), so logits match mia_model_step bit for bit:
//   * Q8_0 matvecs: the input quantized as mia_quantize_row_q8
//     (src/tensor/quant.c:11-27), s = s + ((float)dot * w.d) * x.d over the
//     row's blocks in order (matmul.c:19-28); block dots are exact int32;
//   * rmsnorm (:75-81): the double sum of squares through the certified
//     scale (common.cuh), then x * inv * w;
//   * NeoX RoPE (:84-93): cos/sin of pos * pow(theta, -2i/hd) taken from a
//     table the host fills with the same libm calls, the rotation in double;
//   * attention (:142-161): serial float dot per position, softmax with the
//     serial float sum, serial accumulation over positions per dimension.
// The serial orders are kept where the reference's rounding depends on
// them; the parallelism is across heads, positions, dimensions and rows.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <cub/device/device_radix_sort.cuh>

#include "kernels.cuh"
#include "mia_layout.h"

struct miag_ctx;

namespace miag {
// api.cu
int ctx_device(const miag_ctx *c);
const miag_shape *ctx_shape(const miag_ctx *c);
int ctx_num_sms(const miag_ctx *c);
const void *ctx_reserve(miag_ctx *c, int T, char *err, size_t errlen);
const void *ctx_workspace(const miag_ctx *c);
int ctx_set_layer_device(miag_ctx *c, int layer, const float *ffn_norm, const float *router,
                         cudaStream_t s, char *err, size_t errlen);
struct CtxView;
}  // namespace miag

namespace miag {
namespace {

constexpr int kErrStepArgs = 16;  // a step's token or position out of range (device check)
constexpr int kErrModelWait = 17;  // a dense matvec gave up waiting for a staged tile

void put_err(char *err, size_t errlen, const char *fmt, ...) {
    if (!err || !errlen) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------
// Embedding row: mia_dequantize_row (src/tensor/quant.c:29-38), x = d * q.

__global__ void k_embed(float *x, const uint8_t *embd, const int32_t *args, int d, int vocab,
                        int max_seq, int *err) {
    pdl_launch_dependents();
    pdl_wait();  // the previous step's head wrote args
    const int token = args[0], pos = args[1];
    if (token < 0 || token >= vocab || pos < 0 || pos >= max_seq) {
        if (threadIdx.x == 0 && blockIdx.x == 0) set_error(err, kErrStepArgs);
        return;
    }
    const uint8_t *row = embd + (size_t)token * (size_t)(d / MIAG_QK) * 36;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x) {
        const uint8_t *blk = row + (size_t)(i / MIAG_QK) * 36;
        const float dq = *reinterpret_cast<const float *>(blk);
        x[i] = __fmul_rn(dq, (float)(int8_t)blk[4 + i % MIAG_QK]);
    }
}

// ---------------------------------------------------------------------------
// Dense Q8_0 matvec of one token (mia_matvec, matmul.c:91-106), rows kept
// in the file's layout: row r = nb consecutive 36-byte {f32 d; int8 q[32]}
// blocks.  A CTA walks tiles of R consecutive rows, each one contiguous
// bulk copy (kGemvStages in flight); the input is normalised and quantized
// once per CTA while its first tiles land.  Warp roles per tile:
//   8 term warps   the exact terms ((float)dot_b * w.d) * x.d of every
//                  (row, block) of the tile into shared memory (a thread a
//                  term: consecutive threads take consecutive blocks of a
//                  row, so the 36-byte blocks fall in distinct banks);
//   2 chain warps  a lane a row: s = s + term over the row's blocks in
//                  order (matmul.c:23-26), from shared memory; lane 0 of the
//                  first also refills each stage as soon as the term warps
//                  are done with it.
// The term buffer is double-buffered, so the chains of one tile overlap the
// terms of the next.  Tiles are sized on the host so that a small matrix
// spreads over every SM in one wave.  Up to three weight matrices that
// share the input (wq, wk, wv) run as segments of one launch.

constexpr int kGemvTermWarps = 8, kGemvChainWarps = 2;
constexpr int kGemvThreads = (kGemvTermWarps + kGemvChainWarps) * 32;
constexpr int kGemvStages = 2;
constexpr int kGemvMaxRows = 32 * kGemvChainWarps;  // rows per tile
constexpr size_t kGemvSmemBudget = 220 * 1024;

struct GemvSeg {
    const uint8_t *w;
    float *out;
    int rows, tile0;
};

struct GemvParams {
    GemvSeg seg[3];
    int nseg, ntiles, R, cols, nb, row_bytes, stage_bytes;
    const float *in;    // [cols]
    const float *norm;  // rmsnorm weight [cols], or null: the input is used as it is
    float eps;
    int resid;  // out[r] += s (the residual stream, forward.c:164) instead of out[r] = s
    // next token (the head only): argmax over the rows of segment 0, then the
    // step's arguments advance
    unsigned long long *amax;
    unsigned *ticket;
    int32_t *args;
    const int32_t *prompt;
    int n_prompt;
    int32_t *tokens;
    int max_seq;
    int32_t *best;  // sampling: the argmax goes here and the sampler advances the step
    int *err;
};

struct GemvSmem {
    size_t terms, xq, xin, nrm, red, bars, total;
};

__host__ __device__ inline GemvSmem gemv_smem(int stage_bytes, int R, int cols, int nb) {
    GemvSmem g;
    g.terms = (size_t)kGemvStages * stage_bytes;
    g.xq = g.terms + (((size_t)2 * R * (nb + 1) * 4 + 15) & ~(size_t)15);
    g.xin = g.xq + (((size_t)nb * 36 + 15) & ~(size_t)15);
    g.nrm = g.xin + (size_t)cols * 4;
    g.red = g.nrm + (size_t)cols * 4;
    g.bars = g.red + 32 * 8;
    g.total = g.bars + (kGemvStages + 4) * 8 + 16;
    return g;
}

// Argmax key: larger value first, then the lower row (ties go to the first
// row, as a strict > scan does).
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)row);
}

__global__ void __launch_bounds__(kGemvThreads, 1) k_gemv(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvSmem L = gemv_smem(p.stage_bytes, p.R, p.cols, p.nb);
    float *terms = reinterpret_cast<float *>(smem + L.terms);  // [2][R][nb + 1]
    uint8_t *xq = smem + L.xq;
    float *xin = reinterpret_cast<float *>(smem + L.xin);
    float *nrm = reinterpret_cast<float *>(smem + L.nrm);
    double *red = reinterpret_cast<double *>(smem + L.red);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);  // [kGemvStages]
    uint64_t *tfull = full + kGemvStages;                           // [2] terms written
    uint64_t *tempty = tfull + 2;                                   // [2] terms consumed
    __shared__ float s_inv;
    __shared__ int s_abort;
    __shared__ unsigned long long s_amax;
    __shared__ int s_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = p.nb, ts = nb + 1;  // term row stride (odd for even nb: no bank conflicts)
    const int my_tiles = (int)blockIdx.x < p.ntiles
                             ? (p.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                             : 0;
    auto tile_rows = [&](int j, int &seg, int &r0) {
        const int g = (int)blockIdx.x + j * (int)gridDim.x;
        seg = (p.nseg > 2 && g >= p.seg[2].tile0) ? 2 : (p.nseg > 1 && g >= p.seg[1].tile0) ? 1 : 0;
        r0 = (g - p.seg[seg].tile0) * p.R;
        const int n = p.seg[seg].rows - r0;
        return n < p.R ? n : p.R;
    };
    auto issue = [&](int j) {  // tile j of this CTA into stage j % kGemvStages
        int seg, r0;
        const int n = tile_rows(j, seg, r0);
        const uint32_t bytes = ((uint32_t)n * (uint32_t)p.row_bytes + 15u) & ~15u;
        uint64_t *bar = &full[j % kGemvStages];
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(smem + (size_t)(j % kGemvStages) * p.stage_bytes,
                 p.seg[seg].w + (size_t)r0 * (size_t)p.row_bytes, bytes, bar);
    };
    const bool producer = warp == kGemvTermWarps && lane == 0;

    if (tid == 0) {
        for (int s = 0; s < kGemvStages; s++) mbar_init(&full[s], 1);
        for (int b = 0; b < 2; b++) mbar_init(&tfull[b], kGemvTermWarps), mbar_init(&tempty[b], kGemvChainWarps);
        fence_barrier_init();
        s_abort = 0;
        s_amax = 0ull;
    }
    __syncthreads();
    int issued = 0;
    if (producer)
        for (; issued < kGemvStages && issued < my_tiles; issued++) issue(issued);  // weights: constant
    // the norm weight is constant too: on its way before the wait
    if (p.norm)
        for (int i = 4 * tid; i < p.cols; i += 4 * kGemvThreads) cp_async16(nrm + i, p.norm + i);
    cp_async_commit();
    pdl_launch_dependents();
    pdl_wait();  // the input vector
    // the input row in one round trip (every copy in flight before one wait)
    for (int i = 4 * tid; i < p.cols; i += 4 * kGemvThreads) cp_async16(xin + i, p.in + i);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();

    // Input: rmsnorm (forward.c:75-81) when a weight is given, then Q8_0.
    constexpr int kWarps = kGemvThreads / 32;
    double ss = 0.0;
    for (int i = tid; i < p.cols; i += kGemvThreads) {
        const float v = xin[i];
        ss = __dadd_rn(ss, __dmul_rn((double)v, (double)v));
    }
    if (p.norm) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
            const float inv = rms_scale_certified(lane < kWarps ? red[lane] : 0.0, xin, p.cols, p.eps, lane);
            if (lane == 0) s_inv = inv;
        }
        __syncthreads();
        const float inv = s_inv;
        for (int i = tid; i < p.cols; i += kGemvThreads)
            xin[i] = __fmul_rn(__fmul_rn(xin[i], inv), nrm[i]);
    }
    __syncthreads();
    for (int b = warp; b < nb; b += kWarps) {  // mia_quantize_row_q8, one warp a block
        const float v = xin[b * MIAG_QK + lane];
        float a = fabsf(v);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        const float dq = __fdiv_rn(a, 127.0f);
        const float id = dq != 0.0f ? __fdiv_rn(1.0f, dq) : 0.0f;
        xq[b * 36 + 4 + lane] = (uint8_t)(int8_t)roundf(__fmul_rn(v, id));
        if (lane == 0) *reinterpret_cast<float *>(xq + b * 36) = dq;
    }
    __syncthreads();

    if (warp < kGemvTermWarps) {
        // ---- term warps
        const uint32_t xq_a = smem_addr(xq);
        for (int j = 0; j < my_tiles; j++) {
            const int s = j % kGemvStages, tb = j & 1;
            if (*(volatile int *)&s_abort || !mbar_wait(&full[s], (uint32_t)(j / kGemvStages) & 1u) ||
                (j >= 2 && !mbar_wait(&tempty[tb], (uint32_t)((j >> 1) - 1) & 1u))) {
                set_error(p.err, kErrModelWait);
                *(volatile int *)&s_abort = 1;
                break;
            }
            int seg, r0;
            const int n = tile_rows(j, seg, r0);
            const uint32_t tile = smem_addr(smem) + (uint32_t)s * (uint32_t)p.stage_bytes;
            float *tt = terms + (size_t)tb * p.R * ts;
            for (int q = tid; q < n * nb; q += kGemvTermWarps * 32) {
                const int r = q / nb, b = q - r * nb;
                const uint32_t a = tile + (uint32_t)r * (uint32_t)p.row_bytes + (uint32_t)b * 36u;
                const uint32_t xa = xq_a + (uint32_t)b * 36u;
                int acc = 0;
#pragma unroll
                for (int k = 1; k < 9; k++) acc = __dp4a((int)lds_u32(a + 4u * k), (int)lds_u32(xa + 4u * k), acc);
                tt[r * ts + b] = __fmul_rn(__fmul_rn(__int2float_rn(acc), lds32(a)), lds32(xa));
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&tfull[tb]);
        }
    } else {
        // ---- chain warps (lane = row) and the producer
        const int cw = warp - kGemvTermWarps, r = cw * 32 + lane;
        unsigned long long best = 0ull;
        int j = 0;
        for (; j < my_tiles; j++) {
            const int tb = j & 1;
            if (*(volatile int *)&s_abort || !mbar_wait(&tfull[tb], (uint32_t)(j >> 1) & 1u)) {
                set_error(p.err, kErrModelWait);
                *(volatile int *)&s_abort = 1;
                break;
            }
            if (producer && issued < my_tiles) issue(issued++);  // the term warps left stage j's tile
            int seg, r0;
            const int n = tile_rows(j, seg, r0);
            if (r < n) {
                const float *tr = terms + (size_t)tb * p.R * ts + (size_t)r * ts;
                float sum = 0.0f;
#pragma unroll 8
                for (int b = 0; b < nb; b++) sum = __fadd_rn(sum, tr[b]);
                float *o = p.seg[seg].out + r0 + r;
                *o = p.resid ? __fadd_rn(*o, sum) : sum;
                if (p.amax && seg == 0) {
                    const unsigned long long k = argmax_key(sum, r0 + r);
                    best = k > best ? k : best;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[tb]);
        }
        if (producer) {
            // Nothing may still be landing in shared memory when the CTA
            // leaves: after a failed wait, wait (bounded) for each stage's
            // last copy.
            for (int t = issued - kGemvStages < 0 ? 0 : issued - kGemvStages; t < issued; t++)
                if (*(volatile int *)&s_abort) mbar_wait(&full[t % kGemvStages], (uint32_t)(t / kGemvStages) & 1u);
        }
        if (p.amax) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
                best = v > best ? v : best;
            }
            if (lane == 0) atomicMax(&s_amax, best);
        }
    }
    if (!p.amax) return;
    __syncthreads();
    if (tid == 0) {
        atomicMax(p.amax, s_amax);
        __threadfence();
        s_last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last || tid != 0) return;
    // The last CTA: every row is in, the step's next token is known.
    __threadfence();
    const unsigned long long k = atomicAdd(p.amax, 0ull);
    const int arg = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    const int pos = p.args[1];
    if (p.best) {
        *p.best = arg;
    } else if (pos >= 0 && pos + 1 < p.max_seq) {
        const int next = pos + 1;
        const int token = next < p.n_prompt ? p.prompt[next] : arg;
        p.tokens[next] = token;
        p.args[0] = token;
        p.args[1] = next;
    } else {
        p.args[1] = p.max_seq;  // the next step reports the position out of range
    }
    *p.amax = 0ull;
    *p.ticket = 0u;
}

// ---------------------------------------------------------------------------
// Attention of one layer at one position (forward.c:127-161), GQA.
// Grid (n_heads, kAttnSplit).  Every CTA normalises and rotates its head's
// q and its kv head's k (cheap, and bit-identical in each CTA); CTA y of
// head h scores the position slices y, y + kAttnSplit, ... (a thread a
// position: the reference's serial dot, then * scale) into a scratch row;
// k_attn_out then forms the softmax and the accumulation over positions.
// The new k and v rows are written to the cache by the first CTA of each
// kv group; at position pos every CTA uses its own copies.

constexpr int kAttnThreads = 256, kAttnSplit = 4, kAttnRows = 256;

struct AttnParams {
    const float *qkv;  // q [qd] | k [kvd] | v [kvd]
    const float *q_norm, *k_norm;
    const double2 *rope;  // [max_seq][hd / 2] (cos, sin)
    float *kc, *vc;       // this layer's cache, [max_seq][kvd]
    float *scores;        // [n_heads][max_seq]
    unsigned *ticket;     // [n_heads], zero between launches
    float *att;           // [qd]
    const int32_t *args;
    int nh, nkv, hd, max_seq;
    float eps, scale;
    int *err;
};

// Probabilities are padded to 4 floats so the vectors after them stay
// 16-byte aligned.
__host__ __device__ inline int attn_prob_len(int max_seq) { return (max_seq + 3) & ~3; }

__host__ __device__ inline size_t attn_smem_bytes(int hd, int max_seq) {
    return (size_t)kAttnRows * (hd + 4) * 4   // K slice (V tiles reuse it)
           + (size_t)attn_prob_len(max_seq) * 4  // probabilities
           + (size_t)7 * hd * 4;              // qn, kn, vv, 2 x norm scratch, q/k norm weights
}

// rmsnorm of one head (forward.c:129/134, in place there) then NeoX RoPE
// (:84-93), by one warp; tmp is scratch of hd floats.
__device__ void head_norm_rope(const float *src, const float *w, float *dst, float *tmp, int hd,
                               float eps, const double2 *cs, int lane) {
    double ss = 0.0;
    for (int i = lane; i < hd; i += 32) {
        const float v = src[i];
        ss = __dadd_rn(ss, __dmul_rn((double)v, (double)v));
    }
    const float inv = rms_scale_certified(ss, src, hd, eps, lane);
    for (int i = lane; i < hd; i += 32) tmp[i] = __fmul_rn(__fmul_rn(src[i], inv), w[i]);
    __syncwarp();
    const int half = hd / 2;
    for (int i = lane; i < half; i += 32) {
        const double x0 = (double)tmp[i], x1 = (double)tmp[i + half];
        const double c = cs[i].x, s = cs[i].y;
        dst[i] = __double2float_rn(__dsub_rn(__dmul_rn(x0, c), __dmul_rn(x1, s)));
        dst[i + half] = __double2float_rn(__dadd_rn(__dmul_rn(x0, s), __dmul_rn(x1, c)));
    }
}

__global__ void __launch_bounds__(kAttnThreads, 1) k_attn(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) float fsm[];
    const int hd = p.hd, kvd = p.nkv * hd, qd = p.nh * hd, group = p.nh / p.nkv;
    float *kt = fsm;                                  // [kAttnRows][hd + 4]
    float *prob = kt + (size_t)kAttnRows * (hd + 4);  // [max_seq]
    float *qn = prob + attn_prob_len(p.max_seq), *kn = qn + hd, *vv = kn + hd, *tmp = vv + hd;  // tmp: 2 x hd
    float *wqn = tmp + 2 * hd, *wkn = wqn + hd;  // the q and k norm weights
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x, kvh = h / group;
    // the layer's norm weights are constant: on their way before the wait
    for (int i = tid; i < hd; i += kAttnThreads) {
        wqn[i] = p.q_norm[i];
        wkn[i] = p.k_norm[i];
    }
    pdl_launch_dependents();
    pdl_wait();
    const int pos = p.args[1];
    if (pos < 0 || pos >= p.max_seq) {
        if (tid == 0 && h == 0 && blockIdx.y == 0) set_error(p.err, kErrStepArgs);
        return;
    }
    const float *qh = p.qkv + (size_t)h * hd;
    const float *kh = p.qkv + qd + (size_t)kvh * hd;
    const float *vh = p.qkv + qd + kvd + (size_t)kvh * hd;
    const double2 *cs = p.rope + (size_t)pos * (hd / 2);
    __syncthreads();  // the norm weights
    if (warp == 0) head_norm_rope(qh, wqn, qn, tmp, hd, p.eps, cs, lane);
    else if (warp == 1) head_norm_rope(kh, wkn, kn, tmp + hd, hd, p.eps, cs, lane);
    else if (warp == 2) for (int i = lane; i < hd; i += 32) vv[i] = vh[i];
    __syncthreads();
    if (h % group == 0 && blockIdx.y == 0)  // forward.c:139-140
        for (int i = tid; i < hd; i += kAttnThreads) {
            p.kc[(size_t)pos * kvd + (size_t)kvh * hd + i] = kn[i];
            p.vc[(size_t)pos * kvd + (size_t)kvh * hd + i] = vv[i];
        }

    // Scores (forward.c:148-153).
    const int c4 = hd / 4, n = pos + 1;
    for (int sl = blockIdx.y; sl * kAttnRows < n; sl += gridDim.y) {
        const int t0 = sl * kAttnRows, m = n - t0 < kAttnRows ? n - t0 : kAttnRows;
        for (int i = tid; i < m * c4; i += kAttnThreads) {
            const int r = i / c4, c = i % c4, t = t0 + r;
            float *o = kt + (size_t)r * (hd + 4) + 4 * c;
            if (t == pos)
                *reinterpret_cast<float4 *>(o) = *reinterpret_cast<const float4 *>(kn + 4 * c);
            else
                cp_async16(o, p.kc + (size_t)t * kvd + (size_t)kvh * hd + 4 * c);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        if (tid < m) {
            const float *kr = kt + (size_t)tid * (hd + 4);
            float d = 0.0f;
            for (int i = 0; i < hd; i += 4) {
                const float4 k4 = *reinterpret_cast<const float4 *>(kr + i);
                const float4 q4 = *reinterpret_cast<const float4 *>(qn + i);
                d = __fadd_rn(d, __fmul_rn(q4.x, k4.x));
                d = __fadd_rn(d, __fmul_rn(q4.y, k4.y));
                d = __fadd_rn(d, __fmul_rn(q4.z, k4.z));
                d = __fadd_rn(d, __fmul_rn(q4.w, k4.w));
            }
            p.scores[(size_t)h * p.max_seq + t0 + tid] = __fmul_rn(d, p.scale);
        }
        __syncthreads();
    }

}

// The rest of the attention (forward.c:154-161), a launch of its own so that
// the V rows of a head are read by several CTAs: grid (n_heads,
// kAttnOutSplit), CTA y the output dimensions [y hd / S, (y + 1) hd / S).
// Every CTA forms the head's softmax from the scores (max, exp, the serial
// sum, the division: the same operations on the same values, so the same
// probabilities), then accumulates its dimensions over the positions in
// order, V streamed through shared memory.
constexpr int kAttnOutSplit = 4, kAttnOutRows = 64, kAttnOutBufs = 4;

// Dimension slices a head's output is split into: four where a slice stays
// a whole number of 16-byte chunks, else one.
__host__ __device__ inline int attn_out_split(int hd) { return hd % 16 == 0 ? kAttnOutSplit : 1; }
__host__ __device__ inline size_t attn_out_smem_bytes(int hd, int max_seq) {
    return (size_t)attn_prob_len(max_seq) * 4 + (size_t)kAttnOutBufs * kAttnOutRows * (hd / attn_out_split(hd)) * 4;
}

__global__ void __launch_bounds__(kAttnThreads, 1) k_attn_out(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) float fsm[];
    const int hd = p.hd, kvd = p.nkv * hd, group = p.nh / p.nkv;
    const int dq = hd / (int)gridDim.y, d0 = blockIdx.y * dq, c4 = dq / 4;
    float *prob = fsm;                                   // [max_seq]
    float *vt = prob + attn_prob_len(p.max_seq);         // [bufs][rows][dq]
    __shared__ float red[kAttnThreads / 32];
    __shared__ float s_val;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x, kvh = h / group;
    pdl_launch_dependents();
    pdl_wait();  // the scores, and the cache rows of this position
    const int pos = p.args[1];
    if (pos < 0 || pos >= p.max_seq) return;  // reported by k_attn
    const int n = pos + 1;
    const int ntile = (n + kAttnOutRows - 1) / kAttnOutRows;
    auto load_v = [&](int k) {  // always commits a group (empty past the end)
        if (k < ntile) {
            float *dst = vt + (size_t)(k % kAttnOutBufs) * kAttnOutRows * dq;
            const int t0 = k * kAttnOutRows, m = n - t0 < kAttnOutRows ? n - t0 : kAttnOutRows;
            for (int i = tid; i < m * c4; i += kAttnThreads) {
                const int r = i / c4, c = i % c4;
                cp_async16(dst + (size_t)r * dq + 4 * c, p.vc + (size_t)(t0 + r) * kvd + (size_t)kvh * hd + d0 + 4 * c);
            }
        }
        cp_async_commit();
    };
    for (int k = 0; k < kAttnOutBufs - 1; k++) load_v(k);

    // softmax (forward.c:95-101)
    float mx = -INFINITY;
    for (int t = tid; t < n; t += kAttnThreads) {
        const float v = __ldcg(p.scores + (size_t)h * p.max_seq + t);
        prob[t] = v;
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        float m = red[0];
        for (int w = 1; w < kAttnThreads / 32; w++) m = fmaxf(m, red[w]);
        s_val = m;
    }
    __syncthreads();
    mx = s_val;
    for (int t = tid; t < n; t += kAttnThreads) prob[t] = expf_cr(__fsub_rn(prob[t], mx));
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
#pragma unroll 8
        for (int t = 0; t < n; t++) sum = __fadd_rn(sum, prob[t]);
        s_val = sum;
    }
    __syncthreads();
    const float sum = s_val;
    for (int t = tid; t < n; t += kAttnThreads) prob[t] = __fdiv_rn(prob[t], sum);

    // out[i] = sum over t of p_t * v_t[i], t in order (forward.c:155-160).
    float acc = 0.0f;
    for (int k = 0; k < ntile; k++) {
        load_v(k + kAttnOutBufs - 1);  // into the buffer read at k - 1
        cp_async_wait<kAttnOutBufs - 1>();  // tile k has landed
        __syncthreads();
        if (tid < dq) {
            const float *v = vt + (size_t)(k % kAttnOutBufs) * kAttnOutRows * dq;
            const int t0 = k * kAttnOutRows, m = n - t0 < kAttnOutRows ? n - t0 : kAttnOutRows;
#pragma unroll 8
            for (int r = 0; r < m; r++) acc = __fadd_rn(acc, __fmul_rn(prob[t0 + r], v[(size_t)r * dq + tid]));
        }
        __syncthreads();  // before the next load_v reuses a buffer
    }
    if (tid < dq) p.att[(size_t)h * hd + d0 + tid] = acc;
}

// ---------------------------------------------------------------------------
// Synthetic weights (benchmarks): the counter-based splitmix64 streams of
// motoria_b200/synth.py, generated on the device.  Q8_0 matrices get
// q uniform on [-127, 127] and d = |N(0, 1)| * sigma / 127; f32 tensors
// N(0, 1) * sigma, or ones.

constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;
constexpr int kTagRouter = 1, kTagQw = 2, kTagDw = 3, kTagDense = 5;

__host__ __device__ inline uint64_t sm_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ inline uint64_t sm_next(uint64_t z) { return sm_mix(z + kGamma); }
inline uint64_t sm_key(uint64_t seed, std::initializer_list<uint64_t> ids) {
    uint64_t k = sm_next(seed);
    for (uint64_t i : ids) k = sm_next(k ^ i);
    return k;
}
__device__ __forceinline__ uint64_t sm_stream(uint64_t k, uint64_t i) {
    return sm_mix(k + (i + 1) * kGamma);
}
__device__ __forceinline__ double sm_uniform(uint64_t k, uint64_t i) {
    return ((double)(sm_stream(k, i) >> 11) + 1.0) * 1.1102230246251565e-16;
}
__device__ __forceinline__ double sm_normal(uint64_t k, uint64_t i) {
    const double u0 = sm_uniform(k, 2 * i), u1 = sm_uniform(k, 2 * i + 1);
    return sqrt(-2.0 * log(u0)) * cos(6.283185307179586 * u1);
}

// nblocks Q8_0 blocks at dst (block b at dst + b * 36).
// Q8_0 block b of a matrix: d = |N(0, 1)| * sigma / 127 from stream kd,
// q uniform on [-127, 127] from 16-bit chunks of stream kq.
__device__ __forceinline__ void synth_q8_block(uint8_t *blk, size_t b, uint64_t kq, uint64_t kd,
                                               double sigma) {
    const float dq = (float)(fabs(sm_normal(kd, b)) * sigma / 127.0);
    memcpy(blk, &dq, 4);
    for (int w = 0; w < 8; w++) {  // 16-bit chunks of the q stream, 4 per word
        const uint64_t word = sm_stream(kq, b * 8 + w);
        for (int c = 0; c < 4; c++) {
            const uint32_t hbits = (uint32_t)(word >> (16 * c)) & 0xFFFFu;
            blk[4 + w * 4 + c] = (uint8_t)(int8_t)((int)((hbits * 255u) >> 16) - 127);
        }
    }
}

__global__ void k_synth_q8(uint8_t *dst, size_t nblocks, uint64_t kq, uint64_t kd, double sigma) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += stride)
        synth_q8_block(dst + b * 36, b, kq, kd, sigma);
}

// The experts of one staging batch in one launch: expert k's matrix mat
// (gate, up, down) at dst + k * blob + off[mat], nb[mat] blocks, keys
// key[k][mat] -- the values k_synth_q8 gives each matrix on its own.
constexpr int kSynthBatch = 16;
struct SynthExperts {
    uint8_t *dst;
    size_t blob, off[3], nb[3];
    int n;
    uint64_t kq[kSynthBatch][3], kd[kSynthBatch][3];
    double sigma;
};
__global__ void k_synth_experts(const __grid_constant__ SynthExperts p) {
    const size_t per = p.nb[0] + p.nb[1] + p.nb[2];
    const size_t total = per * (size_t)p.n, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += stride) {
        const int k = (int)(g / per);
        size_t b = g - (size_t)k * per;
        int mat = 0;
        while (mat < 2 && b >= p.nb[mat]) b -= p.nb[mat++];
        synth_q8_block(p.dst + (size_t)k * p.blob + p.off[mat] + b * 36, b, p.kq[k][mat], p.kd[k][mat],
                       p.sigma);
    }
}

__global__ void k_synth_f32(float *dst, size_t n, uint64_t k, double sigma, int ones) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = ones ? 1.0f : (float)(sm_normal(k, i) * sigma);
}

// ---------------------------------------------------------------------------
// Batched prefill: the positions pos0 .. pos0 + n - 1 of a prompt in one pass
// per layer.  The reference prefills one position per mia_model_step
// (src/app/main.c:119-124, serve.c:92-107); here every position's
// arithmetic is still that step's, operation for operation (the same
// kernels' arithmetic as the one-position path above), so the KV cache and
// the last position's logits equal those of n single steps bit for bit.
// What changes is the order of work: each dense weight tile is staged once
// for 32 positions, the MoE block runs once per layer over all n tokens (the
// grouped expert kernels of the prefill regime), and the head runs for the
// last position only.

constexpr int kPfTok = 32;       // positions per token tile
constexpr int kPfThreads = 128;  // 4 warps: 8 positions each
constexpr int kPfAttnThreads = 256;

// Bytes per position of the quantized inputs: the int8 values [cols], then
// the block scales [cols / 32] f32, padded to an odd number of 16-byte units
// so that the 16-byte loads of consecutive positions fall in distinct banks.
__host__ __device__ inline int pf_pitch(int cols) {
    int p = (cols + cols / MIAG_QK * 4 + 15) & ~15;
    if (((p >> 4) & 1) == 0) p += 16;
    return p;
}

// A weight tile is 16 rows (one int8 MMA's M), staged with a 16-byte pad per
// row where the row length allows (rows land in distinct banks).
constexpr int kPfRows = 16;
__host__ __device__ inline int pf_wstride(int cols) {
    const int rb = cols / MIAG_QK * 36;
    return rb % 16 == 0 ? rb + 16 : rb;
}
__host__ inline size_t pf_gemv_smem(int cols) {
    return (((size_t)kPfRows * pf_wstride(cols) + 15) & ~(size_t)15) + (size_t)kPfTok * pf_pitch(cols);
}

// x[t] = dequant(token_embd[tokens[t]]) (forward.c:205-208, quant.c:29-38).
__global__ void k_pf_embed(float *x, const uint8_t *embd, const int32_t *tokens, int d, int vocab,
                           int *err) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, token = tokens[t];
    if (token < 0 || token >= vocab) {
        if (threadIdx.x == 0) set_error(err, kErrStepArgs);
        return;
    }
    const uint8_t *row = embd + (size_t)token * (size_t)(d / MIAG_QK) * 36;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const uint8_t *blk = row + (size_t)(i / MIAG_QK) * 36;
        x[(size_t)t * d + i] = __fmul_rn(*reinterpret_cast<const float *>(blk), (float)(int8_t)blk[4 + i % MIAG_QK]);
    }
}

// One position's matvec input, as k_gemv prepares it: rmsnorm with `norm`
// (forward.c:75-81, the certified scale) when given, then mia_quantize_row_q8
// (quant.c:11-27) into xq[t]: int8 [cols], scales [cols / 32].  Grid: n.
__global__ void __launch_bounds__(kPfThreads) k_pf_quant(const float *in, int in_stride, const float *norm,
                                                         float eps, int cols, uint8_t *xq, int pitch) {
    extern __shared__ __align__(16) float xin[];  // [cols]
    __shared__ double red[kPfThreads / 32];
    __shared__ float s_inv;
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float *src = in + (size_t)t * in_stride;
    double ss = 0.0;
    for (int i = tid; i < cols; i += kPfThreads) {
        const float v = src[i];
        xin[i] = v;
        ss = __dadd_rn(ss, __dmul_rn((double)v, (double)v));
    }
    if (norm) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
            const float inv = rms_scale_certified(lane < kPfThreads / 32 ? red[lane] : 0.0, xin, cols, eps, lane);
            if (lane == 0) s_inv = inv;
        }
        __syncthreads();
        const float inv = s_inv;
        for (int i = tid; i < cols; i += kPfThreads) xin[i] = __fmul_rn(__fmul_rn(xin[i], inv), norm[i]);
    }
    __syncthreads();
    uint8_t *dst = xq + (size_t)t * pitch;
    const int nb = cols / MIAG_QK;
    for (int b = warp; b < nb; b += kPfThreads / 32) {
        const float v = xin[b * MIAG_QK + lane];
        float a = fabsf(v);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        const float dq = __fdiv_rn(a, 127.0f);
        const float id = dq != 0.0f ? __fdiv_rn(1.0f, dq) : 0.0f;
        dst[b * MIAG_QK + lane] = (uint8_t)(int8_t)roundf(__fmul_rn(v, id));
        if (lane == 0) reinterpret_cast<float *>(dst + cols)[b] = dq;
    }
}

struct PfGemvParams {
    const uint8_t *w;   // [rows][cols / 32] 36-byte Q8_0 blocks (the file's layout)
    int rows, cols;
    const uint8_t *xq;  // [n][pitch] (k_pf_quant)
    int pitch, n;
    float *out;         // out[t * out_stride + r]
    int out_stride, resid;
    int *err;
};

__device__ __forceinline__ void pf_mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    // D = A * B + kMagicBits: the int32 dot of each (row, position), exact,
    // read as a float it is 12582912 + dot (|dot| < 2^22)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%10, %10, %10, %10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(kMagicBits));
}

// out[t][r] (+)= the Q8_0 dot of weight row r with position t's input: per
// 32-block the exact int32 dot (one int8 tensor-core MMA, m16n8k32, for 16
// rows x 8 positions), then ((float)dot * w.d) * x.d added in block order
// (matmul.c:19-28), each operation rounded on its own.  Grid (row tiles of
// 16, position tiles of 32); a CTA stages its rows (cp.async, padded) and 32
// positions' inputs, then warp w takes positions 8w .. 8w + 7; each lane
// holds the sums of rows (g, g + 8) x positions (2tq, 2tq + 1).
__global__ void __launch_bounds__(kPfThreads) k_pf_gemv(const __grid_constant__ PfGemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int nb = p.cols / MIAG_QK, row_bytes = nb * 36, ws = pf_wstride(p.cols);
    uint8_t *wt = smem;
    uint8_t *xt = smem + (((size_t)kPfRows * ws + 15) & ~(size_t)15);
    const int r0 = blockIdx.x * kPfRows, t0 = blockIdx.y * kPfTok;
    const int nr = min(kPfRows, p.rows - r0), nt = min(kPfTok, p.n - t0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
    // weights are constant: their copies go out before the wait
    if (ws != row_bytes) {
        const int cpr = row_bytes / 16;  // 16-byte chunks a row
        for (int v = tid; v < nr * cpr; v += kPfThreads) {
            const int r = v / cpr, c = v - r * cpr;
            cp_async16(wt + (size_t)r * ws + 16 * c, p.w + (size_t)(r0 + r) * row_bytes + 16 * c);
        }
    } else {  // rows of a length that is no multiple of 16: the tile as it lies
        const int chunks = (nr * row_bytes + 15) / 16;  // may read 15 bytes past (the section has slack)
        for (int v = tid; v < chunks; v += kPfThreads)
            cp_async16(wt + 16 * v, p.w + (size_t)r0 * row_bytes + 16 * v);
    }
    pdl_launch_dependents();
    pdl_wait();  // the inputs (and, for a residual, the outputs) of earlier launches
    {
        const int cpt = p.pitch / 16;
        for (int v = tid; v < nt * cpt; v += kPfThreads)
            cp_async16(xt + 16 * v, p.xq + (size_t)t0 * p.pitch + 16 * v);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    const int tw = 8 * warp;  // this warp's first position in the tile
    if (tw >= nt) return;
    // rows g and g + 8 (clamped into the tile: a row past the matrix is read,
    // never stored), positions tw + g (B operand) and tw + 2tq, + 1 (sums)
    const int ra = min(g, nr - 1), rb = min(g + 8, nr - 1);
    const uint32_t wa = smem_addr(wt) + (uint32_t)(ra * ws), wb = smem_addr(wt) + (uint32_t)(rb * ws);
    const int tb = min(tw + g, nt - 1);
    const uint32_t xb = smem_addr(xt) + (uint32_t)(tb * p.pitch);
    const int t_lo = min(tw + 2 * tq, nt - 1), t_hi = min(tw + 2 * tq + 1, nt - 1);
    const uint32_t xs_lo = smem_addr(xt) + (uint32_t)(t_lo * p.pitch + p.cols);
    const uint32_t xs_hi = smem_addr(xt) + (uint32_t)(t_hi * p.pitch + p.cols);
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int b = 0; b < nb; b++) {
        const uint32_t ba = wa + (uint32_t)(b * 36), bb = wb + (uint32_t)(b * 36);
        const uint32_t a0 = lds_u32(ba + 4u + 4u * tq), a1 = lds_u32(bb + 4u + 4u * tq);
        const uint32_t a2 = lds_u32(ba + 20u + 4u * tq), a3 = lds_u32(bb + 20u + 4u * tq);
        const uint32_t xq0 = xb + (uint32_t)(b * 32);
        const uint32_t b0 = lds_u32(xq0 + 4u * tq), b1 = lds_u32(xq0 + 16u + 4u * tq);
        int c[4];
        pf_mma_s8(c, a0, a1, a2, a3, b0, b1);
        const float wd_a = lds32(ba), wd_b = lds32(bb);
        const float xd_lo = lds32(xs_lo + 4u * b), xd_hi = lds32(xs_hi + 4u * b);
        const float d0 = __fadd_rn(__int_as_float(c[0]), -kMagic), d1 = __fadd_rn(__int_as_float(c[1]), -kMagic);
        const float d2 = __fadd_rn(__int_as_float(c[2]), -kMagic), d3 = __fadd_rn(__int_as_float(c[3]), -kMagic);
        s[0] = __fadd_rn(s[0], __fmul_rn(__fmul_rn(d0, wd_a), xd_lo));
        s[1] = __fadd_rn(s[1], __fmul_rn(__fmul_rn(d1, wd_a), xd_hi));
        s[2] = __fadd_rn(s[2], __fmul_rn(__fmul_rn(d2, wd_b), xd_lo));
        s[3] = __fadd_rn(s[3], __fmul_rn(__fmul_rn(d3, wd_b), xd_hi));
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int r = (k < 2 ? g : g + 8), t = tw + 2 * tq + (k & 1);
        if (r < nr && t < nt) {
            float *o = p.out + (size_t)(t0 + t) * p.out_stride + r0 + r;
            *o = p.resid ? __fadd_rn(*o, s[k]) : s[k];
        }
    }
}

struct PfQkParams {
    const float *qkv;  // [n][qd + 2 kvd]
    const float *q_norm, *k_norm;
    const double2 *rope;
    float *q;          // [n][qd] normalised and rotated
    float *kc, *vc;    // this layer's cache, [max_seq][kvd]
    int nh, nkv, hd, pos0;
    float eps;
};

// Per position: q and k head rmsnorm + NeoX RoPE (forward.c:127-136, the
// arithmetic of head_norm_rope), k and v into the cache at pos0 + t
// (:139-140).  Grid (n, n_heads + n_kv_heads), one warp.
__global__ void k_pf_qk(const __grid_constant__ PfQkParams p) {
    extern __shared__ __align__(16) float tmp[];  // [hd]
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, h = blockIdx.y, lane = threadIdx.x;
    const int qd = p.nh * p.hd, kvd = p.nkv * p.hd, pos = p.pos0 + t;
    const float *row = p.qkv + (size_t)t * (qd + 2 * kvd);
    const double2 *cs = p.rope + (size_t)pos * (p.hd / 2);
    if (h < p.nh) {
        head_norm_rope(row + (size_t)h * p.hd, p.q_norm, p.q + (size_t)t * qd + (size_t)h * p.hd, tmp, p.hd,
                       p.eps, cs, lane);
    } else {
        const int j = h - p.nh;
        head_norm_rope(row + qd + (size_t)j * p.hd, p.k_norm, p.kc + (size_t)pos * kvd + (size_t)j * p.hd, tmp,
                       p.hd, p.eps, cs, lane);
        for (int i = lane; i < p.hd; i += 32)
            p.vc[(size_t)pos * kvd + (size_t)j * p.hd + i] = row[qd + kvd + (size_t)j * p.hd + i];
    }
}

struct PfAttnParams {
    const float *q;            // [n][qd]
    const float *kc, *vc;      // this layer's cache
    float *att;                // [n][qd]
    int nh, nkv, hd, pos0, max_seq, n;
    float scale;
};

// Attention of position pos0 + t, head h, over positions 0 .. pos0 + t
// (forward.c:142-161), the arithmetic of k_attn: serial float dot per
// position, then * scale; max; exp; the serial sum; the division; the
// accumulation over positions in order, a thread a dimension.  Grid
// (n_heads, n).
__global__ void __launch_bounds__(kPfAttnThreads) k_pf_attn(const __grid_constant__ PfAttnParams p) {
    extern __shared__ __align__(16) float fsh[];
    const int hd = p.hd, kvd = p.nkv * hd, qd = p.nh * hd, group = p.nh / p.nkv;
    float *qs = fsh;                  // [hd]
    float *prob = qs + hd;             // [max_seq]
    __shared__ float red[kPfAttnThreads / 32];
    __shared__ float s_val;
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, t = blockIdx.y, kvh = h / group, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int n = p.pos0 + t + 1;
    for (int i = tid; i < hd; i += kPfAttnThreads) qs[i] = p.q[(size_t)t * qd + (size_t)h * hd + i];
    __syncthreads();
    const float *kbase = p.kc + (size_t)kvh * hd;
    float mx = -INFINITY;
    for (int j = tid; j < n; j += kPfAttnThreads) {
        const float *kr = kbase + (size_t)j * kvd;
        float d = 0.0f;
        for (int i = 0; i < hd; i += 4) {
            const float4 k4 = *reinterpret_cast<const float4 *>(kr + i);
            d = __fadd_rn(d, __fmul_rn(qs[i], k4.x));
            d = __fadd_rn(d, __fmul_rn(qs[i + 1], k4.y));
            d = __fadd_rn(d, __fmul_rn(qs[i + 2], k4.z));
            d = __fadd_rn(d, __fmul_rn(qs[i + 3], k4.w));
        }
        const float v = __fmul_rn(d, p.scale);
        prob[j] = v;
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        float m = red[0];
        for (int w = 1; w < kPfAttnThreads / 32; w++) m = fmaxf(m, red[w]);
        s_val = m;
    }
    __syncthreads();
    mx = s_val;
    for (int j = tid; j < n; j += kPfAttnThreads) prob[j] = expf_cr(__fsub_rn(prob[j], mx));
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
#pragma unroll 8
        for (int j = 0; j < n; j++) sum = __fadd_rn(sum, prob[j]);
        s_val = sum;
    }
    __syncthreads();
    const float sum = s_val;
    for (int j = tid; j < n; j += kPfAttnThreads) prob[j] = __fdiv_rn(prob[j], sum);
    __syncthreads();
    for (int i = tid; i < hd; i += kPfAttnThreads) {
        const float *vb = p.vc + (size_t)kvh * hd + i;
        float acc = 0.0f;
        int j = 0;
        for (; j + 8 <= n; j += 8) {  // eight loads in flight, the adds in order
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = vb[(size_t)(j + u) * kvd];
#pragma unroll
            for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, __fmul_rn(prob[j + u], v[u]));
        }
        for (; j < n; j++) acc = __fadd_rn(acc, __fmul_rn(prob[j], vb[(size_t)j * kvd]));
        p.att[(size_t)t * qd + (size_t)h * hd + i] = acc;
    }
}

// The same attention for prompts that fit: a CTA takes one kv head and TQ
// positions, i.e. the QN = group * TQ queries that read the same K and V
// rows, and streams those rows through shared memory once for all of them.
// Arithmetic as k_pf_attn (and k_attn), query by query: each score a serial
// dot over the head dimensions, the softmax's serial sum over positions in
// order, each output dimension a serial sum over positions in order.
// Threads: four per query (a quarter of the positions for the scores and
// the exponentials, a quarter of the dimensions for the accumulation).
constexpr int kPfQ = 32, kPfTJ = 32;  // queries a CTA, positions a K/V tile
constexpr int kPfTiledMaxPos = 1280;  // scores of every query stay in shared memory
constexpr int kPfTiledMaxHd = 128;

__host__ __device__ inline int pf_tq(int group) { return group >= kPfQ ? 1 : kPfQ / group; }
__host__ __device__ inline size_t pf_attn_tiled_smem(int hd, int npos) {
    return ((size_t)(kPfQ + kPfTJ) * (hd + 4) + (size_t)kPfQ * ((npos + 3) & ~3)) * 4;
}

__global__ void __launch_bounds__(4 * kPfQ) k_pf_attn_tiled(const __grid_constant__ PfAttnParams p) {
    extern __shared__ __align__(16) float fsh[];
    const int hd = p.hd, kvd = p.nkv * hd, qd = p.nh * hd, group = p.nh / p.nkv;
    // the longest (last) positions first, so that the short ones fill the
    // last wave
    const int TQ = pf_tq(group), g = blockIdx.x, t0 = ((int)gridDim.y - 1 - (int)blockIdx.y) * TQ;
    const int tid = threadIdx.x, q = tid >> 2, part = tid & 3;
    const int rs = hd + 4;  // padded row stride: four rows' 16-byte loads in distinct banks
    const int n_cta = p.pos0 + min(t0 + TQ, p.n);  // positions any query of the CTA reads
    const int npad = (n_cta + 3) & ~3;
    float *qs = fsh, *kv = qs + (size_t)kPfQ * rs, *sc = kv + (size_t)kPfTJ * rs;
    const int hg = q / TQ, tt = q - hg * TQ;
    const int h = g * group + hg, t = t0 + tt;
    const bool live = hg < group && t < p.n;
    const int pq = p.pos0 + t;  // this query's position: it reads positions 0 .. pq
    pdl_launch_dependents();
    pdl_wait();
    for (int v = tid; v < kPfQ * (hd / 4); v += 4 * kPfQ) {
        const int r = v / (hd / 4), c = v - r * (hd / 4);
        const int rhg = r / TQ, rt = t0 + (r - rhg * TQ);
        if (rhg < group && rt < p.n)
            cp_async16(qs + (size_t)r * rs + 4 * c, p.q + (size_t)rt * qd + (size_t)(g * group + rhg) * hd + 4 * c);
    }
    const float *kb = p.kc + (size_t)g * hd, *vb = p.vc + (size_t)g * hd;
    auto load_tile = [&](const float *base, int j0) {
        const int m = min(kPfTJ, n_cta - j0);
        for (int v = tid; v < m * (hd / 4); v += 4 * kPfQ) {
            const int r = v / (hd / 4), c = v - r * (hd / 4);
            cp_async16(kv + (size_t)r * rs + 4 * c, base + (size_t)(j0 + r) * kvd + 4 * c);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
    };
    // scores: positions part, part + 4, ... of each tile
    for (int j0 = 0; j0 < n_cta; j0 += kPfTJ) {
        load_tile(kb, j0);
        if (live) {
            float acc[kPfTJ / 4];
#pragma unroll
            for (int m = 0; m < kPfTJ / 4; m++) acc[m] = 0.0f;
            const float *qr = qs + (size_t)q * rs;
            for (int i = 0; i < hd; i += 4) {
                const float4 q4 = *reinterpret_cast<const float4 *>(qr + i);
#pragma unroll
                for (int m = 0; m < kPfTJ / 4; m++) {
                    const float4 k4 = *reinterpret_cast<const float4 *>(kv + (size_t)(part + 4 * m) * rs + i);
                    acc[m] = __fadd_rn(acc[m], __fmul_rn(q4.x, k4.x));
                    acc[m] = __fadd_rn(acc[m], __fmul_rn(q4.y, k4.y));
                    acc[m] = __fadd_rn(acc[m], __fmul_rn(q4.z, k4.z));
                    acc[m] = __fadd_rn(acc[m], __fmul_rn(q4.w, k4.w));
                }
            }
#pragma unroll
            for (int m = 0; m < kPfTJ / 4; m++) {
                const int j = j0 + part + 4 * m;
                if (j <= pq) sc[(size_t)q * npad + j] = __fmul_rn(acc[m], p.scale);
            }
        }
        __syncthreads();  // before the next tile overwrites this one
    }
    // softmax of each query's row (forward.c:95-101)
    float *row = sc + (size_t)q * npad;
    float mx = -INFINITY;
    if (live)
        for (int j = part; j <= pq; j += 4) mx = fmaxf(mx, row[j]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (live)
        for (int j = part; j <= pq; j += 4) row[j] = expf_cr(__fsub_rn(row[j], mx));
    __syncwarp();
    float sum = 0.0f;
    if (live && part == 0) {
#pragma unroll 8
        for (int j = 0; j <= pq; j++) sum = __fadd_rn(sum, row[j]);
    }
    sum = __shfl_sync(0xffffffffu, sum, (tid & 31) & ~3);
    if (live)
        for (int j = part; j <= pq; j += 4) row[j] = __fdiv_rn(row[j], sum);
    __syncthreads();
    // out[i] = sum over positions of p_j * v_j[i], positions in order
    // (:155-160).  This thread's dimensions: the 16-byte chunks part,
    // part + 4, ... (the four threads of a query read distinct banks).
    const int nch = hd / 16;  // chunks a thread
    float acc[kPfTiledMaxHd / 4];
#pragma unroll
    for (int u = 0; u < kPfTiledMaxHd / 4; u++) acc[u] = 0.0f;
    for (int j0 = 0; j0 < n_cta; j0 += kPfTJ) {
        load_tile(vb, j0);
        if (live) {
            const int m = min(kPfTJ, pq + 1 - j0);
            for (int jj = 0; jj < m; jj++) {
                const float pj = row[j0 + jj];
                const float *vr = kv + (size_t)jj * rs + 4 * part;
#pragma unroll
                for (int k = 0; k < kPfTiledMaxHd / 16; k++) {
                    if (k < nch) {
                        const float4 v4 = *reinterpret_cast<const float4 *>(vr + 16 * k);
                        acc[4 * k] = __fadd_rn(acc[4 * k], __fmul_rn(pj, v4.x));
                        acc[4 * k + 1] = __fadd_rn(acc[4 * k + 1], __fmul_rn(pj, v4.y));
                        acc[4 * k + 2] = __fadd_rn(acc[4 * k + 2], __fmul_rn(pj, v4.z));
                        acc[4 * k + 3] = __fadd_rn(acc[4 * k + 3], __fmul_rn(pj, v4.w));
                    }
                }
            }
        }
        __syncthreads();
    }
    if (live) {
        float *out = p.att + (size_t)t * qd + (size_t)h * hd + 4 * part;
#pragma unroll
        for (int k = 0; k < kPfTiledMaxHd / 16; k++)
            if (k < nch) *reinterpret_cast<float4 *>(out + 16 * k) = make_float4(acc[4 * k], acc[4 * k + 1], acc[4 * k + 2], acc[4 * k + 3]);
    }
}

// ---------------------------------------------------------------------------
// Sampling on the device: mia_sample (src/tokenizer/sampler.c:33-66) with a
// temperature above zero, after the head has found the argmax (:34-37).
//   e_i = expf((l_i - l_best) / temperature), sum = e_0 + e_1 + ... serially
//   p_i = e_i / sum; the candidates p_i >= (1 - top_p) / (n - 1), sorted by
//   p descending -- glibc's qsort is a merge sort, stable, so equal p keep
//   the index order: the sort key (~bits(p), i) gives the same order;
//   the smallest prefix whose serial cumulative sum reaches top_p, then
//   r = rand01() * cum and the first candidate whose running sum exceeds r.
// The serial sums are the reference's, in its order; one thread adds while
// the CTA stages the next tile of values in shared memory.

constexpr int kSmpThreads = 256, kSmpTile = 4096, kSmpPickTile = 2048;

struct SmpState {
    unsigned long long rng;  // xorshift64* state (sampler.c:24-29)
    float sum, cum;
    int best, last, m;
};

// xorshift64*: the next state and its float in [0, 1) (sampler.c:24-29).
__device__ __forceinline__ float smp_rand01(unsigned long long &s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return __fdiv_rn((float)((s * 0x2545F4914F6CDD1DULL) >> 40), 16777216.0f);
}

// e_i and their serial sum.  One CTA: tile k + 1's exponentials are formed
// while thread 0 adds tile k's.
__global__ void __launch_bounds__(kSmpThreads) k_smp_sum(const float *logits, int n, float temp, float *e,
                                                         SmpState *st) {
    __shared__ float buf[2][kSmpTile];
    const int tid = threadIdx.x;
    const float mx = logits[st->best];
    const int ntile = (n + kSmpTile - 1) / kSmpTile;
    auto fill = [&](int k) {
        for (int j = tid; j < kSmpTile; j += kSmpThreads) {
            const int i = k * kSmpTile + j;
            if (i < n) {
                const float v = expf_cr(__fdiv_rn(__fsub_rn(logits[i], mx), temp));
                buf[k & 1][j] = v;
                e[i] = v;
            }
        }
    };
    fill(0);
    __syncthreads();
    float sum = 0.0f;
    for (int k = 0; k < ntile; k++) {
        if (k + 1 < ntile) fill(k + 1);
        if (tid == 0) {
            const int m = min(kSmpTile, n - k * kSmpTile);
            const float *b = buf[k & 1];
#pragma unroll 8
            for (int j = 0; j < m; j++) sum = __fadd_rn(sum, b[j]);
        }
        __syncthreads();
    }
    if (tid == 0) st->sum = sum;
}

// p_i and the sort keys: (~bits(p_i)) << 32 | i for the candidates (p >= 0,
// so its bits order like its value), all ones for the rest.
__global__ void k_smp_keys(const float *e, int n, float top_p, SmpState *st, float *p,
                           unsigned long long *keys) {
    const float sum = st->sum;
    const float cutoff = __fdiv_rn(__fsub_rn(1.0f, top_p), (float)(n > 1 ? n - 1 : 1));
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = __fdiv_rn(e[i], sum);
        p[i] = v;
        keys[i] = v >= cutoff ? ((unsigned long long)(~__float_as_uint(v)) << 32) | (unsigned)i : ~0ull;
    }
}

// The nucleus and the draw over the sorted candidates; then the step
// advances as the head's greedy path does (the prompt's own next token while
// the prompt lasts, without drawing).
__global__ void __launch_bounds__(kSmpThreads) k_smp_pick(const unsigned long long *keys, const float *p, int n,
                                                          float top_p, SmpState *st, int32_t *args,
                                                          const int32_t *prompt, int n_prompt, int32_t *tokens,
                                                          int max_seq) {
    __shared__ float buf[2][kSmpPickTile];
    __shared__ int ibuf[2][kSmpPickTile];
    __shared__ int s_stop, s_m;
    const int tid = threadIdx.x;
    const int pos = args[1];
    if (pos < 0 || pos + 1 >= max_seq) {
        if (tid == 0) args[1] = max_seq;  // the next step reports the position out of range
        return;
    }
    const int next = pos + 1;
    if (next < n_prompt) {
        if (tid == 0) {
            tokens[next] = prompt[next];
            args[0] = prompt[next];
            args[1] = next;
        }
        return;
    }
    // pass 0: the cumulative sum up to top_p; pass 1: the draw
    int token = st->best;
    float cum = 0.0f, r = 0.0f, acc = 0.0f;
    int last = -1, m = n;
    if (tid == 0) s_m = n;
    for (int pass = 0; pass < 2; pass++) {
        const int end = pass == 0 ? n : last + 1;
        const int ntile = (end + kSmpPickTile - 1) / kSmpPickTile;
        auto fill = [&](int k) {
            for (int j = tid; j < kSmpPickTile; j += kSmpThreads) {
                const int q = k * kSmpPickTile + j;
                const unsigned long long key = q < end ? keys[q] : ~0ull;
                const int i = key == ~0ull ? -1 : (int)(key & 0xFFFFFFFFull);
                ibuf[k & 1][j] = i;
                buf[k & 1][j] = i >= 0 ? p[i] : 0.0f;
            }
        };
        if (tid == 0) s_stop = 0;
        if (ntile > 0) fill(0);
        __syncthreads();
        for (int k = 0; k < ntile && !s_stop; k++) {
            if (k + 1 < ntile) fill(k + 1);
            if (tid == 0) {
                const int cnt = min(kSmpPickTile, end - k * kSmpPickTile);
                for (int j = 0; j < cnt; j++) {
                    const int i = ibuf[k & 1][j];
                    const int q = k * kSmpPickTile + j;
                    if (pass == 0) {
                        if (i < 0) {  // past the candidates
                            s_m = q;
                            s_stop = 1;
                            break;
                        }
                        cum = __fadd_rn(cum, buf[k & 1][j]);
                        if (cum >= top_p) {
                            last = q;
                            s_stop = 1;
                            break;
                        }
                    } else {
                        acc = __fadd_rn(acc, buf[k & 1][j]);
                        if (r < acc) {
                            token = i;
                            s_stop = 1;
                            break;
                        }
                        if (q == last) token = i;  // no candidate passed r: the last one
                    }
                }
            }
            __syncthreads();
        }
        if (pass == 0) {
            if (tid == 0) {
                m = s_m;
                if (last < 0) last = m - 1;
                if (last >= 0) {
                    unsigned long long s = st->rng;
                    r = __fmul_rn(smp_rand01(s), cum);
                    st->rng = s;
                }
                s_m = last;  // broadcast
            }
            __syncthreads();
            last = s_m;
            if (last < 0) break;  // no candidate: the argmax
        }
    }
    if (tid == 0) {
        st->cum = cum, st->last = last;
        tokens[next] = token;
        args[0] = token;
        args[1] = next;
    }
}

}  // namespace
}  // namespace miag

using namespace miag;

struct miag_model {
    miag_ctx *moe = nullptr;
    bool owns_moe = false;
    miag_mia_config cfg{};
    int device = 0, max_seq = 0, num_sms = 0;
    int d = 0, qd = 0, kvd = 0, hd = 0;
    cudaStream_t stream = nullptr;
    std::vector<MiaTensor> layout;
    size_t dense_bytes = 0;
    uint8_t *dense = nullptr;  // the dense section, as in the file
    double2 *rope = nullptr;
    float *kc = nullptr, *vc = nullptr;
    float *x = nullptr, *qkv = nullptr, *att = nullptr, *logits = nullptr, *scores = nullptr;
    int32_t *args = nullptr, *prompt = nullptr, *tokens = nullptr;
    int n_prompt = 0;
    unsigned *tickets = nullptr;  // [n_heads] attention, [1] head
    unsigned long long *amax = nullptr;
    int *d_err = nullptr;
    float *h_logits = nullptr;  // pinned
    int32_t *h_args = nullptr;  // pinned
    GemvParams qkv_p{}, wo_p{}, head_p{};
    size_t qkv_smem = 0, wo_smem = 0, head_smem = 0, attn_smem = 0;
    cudaGraphExec_t exec = nullptr;
    const void *graph_ws = nullptr;
    bool dense_set = false;
    bool eager = false;  // the step could not be captured: launched directly
    int last_launches = 0;
    // batched prefill (miag_model_prefill_async): buffers for pf_cap positions
    bool batched_prefill = true;
    int pf_cap = 0, pf_last_launches = 0;
    float *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_att = nullptr;
    uint8_t *pf_xq = nullptr;
    int32_t *pf_tok = nullptr;
    int32_t *h_pf_tok = nullptr;  // pinned, pf_cap entries
    // sampling (miag_model_set_sampler): temperature 0 = greedy in the head
    float smp_temp = 0.0f, smp_top_p = 1.0f;
    SmpState *smp = nullptr;
    float *smp_e = nullptr, *smp_p = nullptr;
    unsigned long long *smp_k0 = nullptr, *smp_k1 = nullptr;
    void *smp_tmp = nullptr;
    size_t smp_tmp_bytes = 0;
};

namespace {

const uint8_t *tensor(const miag_model *m, size_t i) { return m->dense + m->layout[i].offset; }
const float *tensor_f(const miag_model *m, size_t i) {
    return reinterpret_cast<const float *>(tensor(m, i));
}

cudaError_t gemv_launch(const GemvParams &p, int grid, size_t smem, cudaStream_t s) {
    if (!p.in || !p.err) return cudaErrorInvalidValue;
    for (int i = 0; i < p.nseg; i++)
        if (!p.seg[i].w || !p.seg[i].out) return cudaErrorInvalidValue;
    return launch_dependent(k_gemv, dim3(grid), dim3(kGemvThreads), smem, s, p);
}

// Tiling of a matvec over `cols` inputs (segments' rows filled in by the
// caller): the largest R (a multiple of 4, so every tile starts 16-byte
// aligned) whose stages fit in shared memory, lowered to spread a small
// matrix over the SMs in one wave.
void gemv_plan(GemvParams &p, int cols, int num_sms, size_t *smem) {
    p.cols = cols;
    p.nb = cols / MIAG_QK;
    p.row_bytes = p.nb * 36;
    int rmax = kGemvMaxRows;
    while (rmax > 4 && gemv_smem(rmax * p.row_bytes, rmax, cols, p.nb).total > kGemvSmemBudget) rmax -= 4;
    int rows = 0;
    for (int i = 0; i < p.nseg; i++) rows += p.seg[i].rows;
    const int rbal = ((rows + num_sms - 1) / num_sms + 3) & ~3;
    p.R = rbal < 4 ? 4 : rbal < rmax ? rbal : rmax;
    p.stage_bytes = p.R * p.row_bytes;
    int tiles = 0;
    for (int i = 0; i < p.nseg; i++) {
        p.seg[i].tile0 = tiles;
        tiles += (p.seg[i].rows + p.R - 1) / p.R;
    }
    p.ntiles = tiles;
    *smem = gemv_smem(p.stage_bytes, p.R, cols, p.nb).total;
}

int grid_of(const miag_model *m, const GemvParams &p) {
    return p.ntiles < m->num_sms ? p.ntiles : m->num_sms;
}

#define MCU(x)                                                                    \
    do {                                                                          \
        cudaError_t e_ = (x);                                                     \
        if (e_ != cudaSuccess) {                                                  \
            put_err(err, errlen, "%s: %s", #x, cudaGetErrorString(e_));           \
            return -1;                                                            \
        }                                                                         \
    } while (0)

// The draw after the head (temperature > 0): the exponentials and their
// serial sum, the candidates' keys, their sort, the nucleus and the draw.
int enqueue_sample(miag_model *m, cudaStream_t s, char *err, size_t errlen) {
    const int n = (int)m->cfg.vocab;
    k_smp_sum<<<1, kSmpThreads, 0, s>>>(m->logits, n, m->smp_temp, m->smp_e, m->smp);
    MCU(cudaGetLastError());
    k_smp_keys<<<(n + 255) / 256, 256, 0, s>>>(m->smp_e, n, m->smp_top_p, m->smp, m->smp_p, m->smp_k0);
    MCU(cudaGetLastError());
    size_t bytes = m->smp_tmp_bytes;
    MCU(cub::DeviceRadixSort::SortKeys(m->smp_tmp, bytes, m->smp_k0, m->smp_k1, n, 0, 64, s));
    k_smp_pick<<<1, kSmpThreads, 0, s>>>(m->smp_k1, m->smp_p, n, m->smp_top_p, m->smp, m->args, m->prompt,
                                          m->head_p.n_prompt, m->tokens, m->max_seq);
    MCU(cudaGetLastError());
    return 0;
}

// The launch sequence of one step on stream s (captured into the graph).
int enqueue_step(miag_model *m, cudaStream_t s, char *err, size_t errlen) {
    const miag_mia_config &c = m->cfg;
    int launches = 0;
    MCU(launch_dependent(k_embed, dim3((m->d + 255) / 256), dim3(256), 0, s, m->x, tensor(m, 0),
                         (const int32_t *)m->args, m->d, (int)c.vocab, m->max_seq, m->d_err));
    launches++;
    for (int l = 0; l < (int)c.n_layers; l++) {
        GemvParams q = m->qkv_p;
        q.seg[0].w = tensor(m, mia_layer_tensor(l, kWq));
        q.seg[1].w = tensor(m, mia_layer_tensor(l, kWk));
        q.seg[2].w = tensor(m, mia_layer_tensor(l, kWv));
        q.norm = tensor_f(m, mia_layer_tensor(l, kAttnNorm));
        MCU(gemv_launch(q, grid_of(m, q), m->qkv_smem, s));
        AttnParams a{};
        a.qkv = m->qkv;
        a.q_norm = tensor_f(m, mia_layer_tensor(l, kQNorm));
        a.k_norm = tensor_f(m, mia_layer_tensor(l, kKNorm));
        a.rope = m->rope;
        const size_t layer_off = (size_t)l * m->max_seq * m->kvd;
        a.kc = m->kc + layer_off, a.vc = m->vc + layer_off;
        a.scores = m->scores, a.ticket = m->tickets, a.att = m->att, a.args = m->args;
        a.nh = (int)c.n_heads, a.nkv = (int)c.n_kv_heads, a.hd = m->hd, a.max_seq = m->max_seq;
        a.eps = c.norm_eps;
        a.scale = 1.0f / sqrtf((float)m->hd);  // forward.c:143
        a.err = m->d_err;
        MCU(launch_dependent(k_attn, dim3(c.n_heads, kAttnSplit), dim3(kAttnThreads), m->attn_smem, s, a));
        MCU(launch_dependent(k_attn_out, dim3(c.n_heads, attn_out_split(m->hd)), dim3(kAttnThreads),
                             attn_out_smem_bytes(m->hd, m->max_seq), s, a));
        GemvParams o = m->wo_p;
        o.seg[0].w = tensor(m, mia_layer_tensor(l, kWo));
        MCU(gemv_launch(o, grid_of(m, o), m->wo_smem, s));
        launches += 4;
        if (miag_moe_async(m->moe, l, m->x, 1, s, err, errlen) != 0) return -1;
        launches += miag_last_launch_count(m->moe);
    }
    GemvParams hp = m->head_p;
    const size_t nt = m->layout.size();  // ..., output_norm, output
    hp.seg[0].w = tensor(m, nt - 1);
    hp.norm = tensor_f(m, nt - 2);
    hp.best = m->smp_temp > 0.0f ? &m->smp->best : nullptr;
    MCU(gemv_launch(hp, grid_of(m, hp), m->head_smem, s));
    launches++;
    if (m->smp_temp > 0.0f) {
        if (enqueue_sample(m, s, err, errlen)) return -1;
        launches += 3;
    }
    m->last_launches = launches;
    return 0;
}

int capture(miag_model *m, char *err, size_t errlen) {
    if (m->exec) {
        cudaGraphExecDestroy(m->exec);
        m->exec = nullptr;
    }
    const void *ws = ctx_reserve(m->moe, 1, err, errlen);
    if (!ws) return -1;
    cudaGraph_t g = nullptr;
    MCU(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue_step(m, m->stream, err, errlen);
    const cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (rc != 0) {
        if (g) cudaGraphDestroy(g);
        return -1;
    }
    MCU(e);
    const cudaError_t ie = cudaGraphInstantiate(&m->exec, g, 0);
    cudaGraphDestroy(g);
    MCU(ie);
    m->graph_ws = ws;
    return 0;
}

// Reads and clears the model's error word, then the MoE context's (after a
// synchronisation of the model's stream).
int check_errors(miag_model *m, char *err, size_t errlen) {
    MCU(cudaStreamSynchronize(m->stream));
    int code = 0;
    MCU(cudaMemcpy(&code, m->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (code != 0) {
        MCU(cudaMemset(m->d_err, 0, sizeof(int)));
        // a step cut short may leave the tickets and the argmax set
        MCU(cudaMemset(m->tickets, 0, ((size_t)m->cfg.n_heads + 1) * sizeof(unsigned)));
        MCU(cudaMemset(m->amax, 0, sizeof(unsigned long long)));
        put_err(err, errlen, "device error %d: %s", code,
                code == kErrStepArgs ? "a step's token or position was out of range"
                                     : "a dense matvec timed out waiting for a staged tile");
        return -1;
    }
    return miag_sync(m->moe, m->stream, err, errlen);
}

// Steps as graph replays; where the capture fails (a driver without
// programmatic edges in graphs, say) the same sequence is launched directly.
int launch_steps(miag_model *m, int n, char *err, size_t errlen) {
    if (!m->eager && (!m->exec || ctx_workspace(m->moe) != m->graph_ws)) {
        char why[256] = "";
        if (capture(m, why, sizeof why)) {
            cudaGetLastError();
            if (!ctx_reserve(m->moe, 1, err, errlen)) return -1;
            m->eager = true;
        }
    }
    for (int i = 0; i < n; i++) {
        if (m->eager) {
            if (enqueue_step(m, m->stream, err, errlen)) return -1;
        } else {
            MCU(cudaGraphLaunch(m->exec, m->stream));
        }
    }
    return 0;
}

bool shape_matches(const miag_shape &s, const miag_mia_config &c) {
    return s.dim == (int)c.dim && s.n_layers == (int)c.n_layers && s.n_experts == (int)c.n_experts &&
           s.n_active == (int)c.n_active && s.expert_hidden == (int)c.expert_hidden &&
           s.norm_topk == (int)c.norm_topk && s.norm_eps == c.norm_eps;
}

// Hands the dense section's routers and ffn norms to the MoE context.
int set_moe_layers(miag_model *m, char *err, size_t errlen) {
    for (int l = 0; l < (int)m->cfg.n_layers; l++)
        if (ctx_set_layer_device(m->moe, l, tensor_f(m, mia_layer_tensor(l, kFfnNorm)),
                                 tensor_f(m, mia_layer_tensor(l, kRouter)), m->stream, err, errlen))
            return -1;
    MCU(cudaStreamSynchronize(m->stream));
    m->dense_set = true;
    return 0;
}

}  // namespace

extern "C" void miag_model_close(miag_model *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    void *bufs[] = {m->dense, m->rope, m->kc, m->vc, m->x, m->qkv, m->att, m->logits, m->scores,
                    m->args, m->prompt, m->tokens, m->tickets, m->amax, m->d_err};
    for (void *b : bufs) cudaFree(b);
    for (void *b : {(void *)m->pf_x, (void *)m->pf_qkv, (void *)m->pf_q, (void *)m->pf_att,
                    (void *)m->pf_xq, (void *)m->pf_tok})
        if (b) cudaFree(b);
    if (m->h_pf_tok) cudaFreeHost(m->h_pf_tok);
    for (void *b : {(void *)m->smp, (void *)m->smp_e, (void *)m->smp_p, (void *)m->smp_k0, (void *)m->smp_k1,
                    m->smp_tmp})
        if (b) cudaFree(b);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    if (m->h_args) cudaFreeHost(m->h_args);
    if (m->stream) cudaStreamDestroy(m->stream);
    if (m->owns_moe) miag_close(m->moe);
    delete m;
}

extern "C" int miag_model_open(miag_model **out, miag_ctx *moe, const miag_mia_config *config,
                               const void *dense, size_t dense_bytes, int max_seq, char *err,
                               size_t errlen) {
    if (!out || !moe || !config) {
        put_err(err, errlen, "null argument");
        return -1;
    }
    *out = nullptr;
    const miag_mia_config &c = *config;
    if (!mia_config_ok(c) || c.head_dim % 4 || c.head_dim > 256) {
        put_err(err, errlen, "unsupported model shape (head_dim a multiple of 4, at most 256)");
        return -1;
    }
    if (!shape_matches(*ctx_shape(moe), c)) {
        put_err(err, errlen, "the MoE context's shape differs from the model's");
        return -1;
    }
    const int qd = (int)(c.n_heads * c.head_dim);
    if (c.dim > 8192 || qd > 8192) {
        put_err(err, errlen, "dim and n_heads * head_dim are limited to 8192");
        return -1;
    }
    if (max_seq <= 0) {
        put_err(err, errlen, "context length must be positive");
        return -1;
    }
    if (attn_smem_bytes((int)c.head_dim, max_seq) > 227 * 1024) {
        put_err(err, errlen, "context length %d too long for the attention kernel", max_seq);
        return -1;
    }
    miag_model *m = new miag_model;
    m->moe = moe;
    m->cfg = c;
    m->device = ctx_device(moe);
    m->num_sms = ctx_num_sms(moe);
    m->max_seq = max_seq;
    m->d = (int)c.dim, m->qd = qd, m->hd = (int)c.head_dim, m->kvd = (int)(c.n_kv_heads * c.head_dim);
    m->layout = mia_dense_layout(c, &m->dense_bytes);
    if (dense && dense_bytes != m->dense_bytes) {
        put_err(err, errlen, "dense section of %zu bytes, the layout needs %zu", dense_bytes,
                m->dense_bytes);
        delete m;
        return -1;
    }
    auto fail = [&](const char *what, cudaError_t e) {
        put_err(err, errlen, "%s: %s", what, cudaGetErrorString(e));
        miag_model_close(m);
        return -1;
    };
    cudaError_t e;
    if ((e = cudaSetDevice(m->device)) != cudaSuccess) return fail("cudaSetDevice", e);
    if ((e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking)) != cudaSuccess)
        return fail("cudaStreamCreate", e);
    const size_t L = c.n_layers, kv = L * (size_t)max_seq * m->kvd;
    struct {
        void **p;
        size_t bytes;
    } allocs[] = {
        {(void **)&m->dense, m->dense_bytes + 256},  // tiles read up to 15 bytes past a matrix
        {(void **)&m->rope, (size_t)max_seq * (m->hd / 2) * sizeof(double2)},
        {(void **)&m->kc, kv * 4},
        {(void **)&m->vc, kv * 4},
        {(void **)&m->x, (size_t)m->d * 4},
        {(void **)&m->qkv, (size_t)(qd + 2 * m->kvd) * 4},
        {(void **)&m->att, (size_t)qd * 4},
        {(void **)&m->logits, (size_t)c.vocab * 4},
        {(void **)&m->scores, (size_t)c.n_heads * max_seq * 4},
        {(void **)&m->args, 2 * sizeof(int32_t)},
        {(void **)&m->prompt, (size_t)max_seq * sizeof(int32_t)},
        {(void **)&m->tokens, (size_t)max_seq * sizeof(int32_t)},
        {(void **)&m->tickets, (c.n_heads + 1) * sizeof(unsigned)},
        {(void **)&m->amax, sizeof(unsigned long long)},
        {(void **)&m->d_err, sizeof(int)},
    };
    for (auto &a : allocs) {
        if ((e = cudaMalloc(a.p, a.bytes)) != cudaSuccess) return fail("cudaMalloc", e);
        if ((e = cudaMemsetAsync(*a.p, 0, a.bytes, m->stream)) != cudaSuccess)
            return fail("cudaMemset", e);
    }
    if ((e = cudaMallocHost(&m->h_logits, (size_t)c.vocab * 4)) != cudaSuccess)
        return fail("cudaMallocHost", e);
    if ((e = cudaMallocHost(&m->h_args, 2 * sizeof(int32_t))) != cudaSuccess)
        return fail("cudaMallocHost", e);

    // RoPE table: the reference's own libm calls (forward.c:87-88), here on
    // the host, so the device rotates with the same cos and sin.
    {
        const int half = m->hd / 2;
        std::vector<double2> tab((size_t)max_seq * half);
        for (int i = 0; i < half; i++) {
            const double freq = pow((double)c.rope_theta, -2.0 * i / m->hd);
            for (int pos = 0; pos < max_seq; pos++) {
                const double a = pos * freq;
                tab[(size_t)pos * half + i] = make_double2(cos(a), sin(a));
            }
        }
        if ((e = cudaMemcpyAsync(m->rope, tab.data(), tab.size() * sizeof(double2),
                                 cudaMemcpyHostToDevice, m->stream)) != cudaSuccess)
            return fail("rope upload", e);
        if ((e = cudaStreamSynchronize(m->stream)) != cudaSuccess) return fail("rope upload", e);
    }

    // Matvec plans (weights bound per layer at launch).
    GemvParams &q = m->qkv_p;
    q.nseg = 3;
    q.seg[0] = {nullptr, m->qkv, qd, 0};
    q.seg[1] = {nullptr, m->qkv + qd, m->kvd, 0};
    q.seg[2] = {nullptr, m->qkv + qd + m->kvd, m->kvd, 0};
    q.in = m->x, q.eps = c.norm_eps, q.err = m->d_err;
    gemv_plan(q, m->d, m->num_sms, &m->qkv_smem);
    GemvParams &o = m->wo_p;
    o.nseg = 1;
    o.seg[0] = {nullptr, m->x, m->d, 0};
    o.in = m->att, o.norm = nullptr, o.resid = 1, o.err = m->d_err;
    gemv_plan(o, qd, m->num_sms, &m->wo_smem);
    GemvParams &hp = m->head_p;
    hp.nseg = 1;
    hp.seg[0] = {nullptr, m->logits, (int)c.vocab, 0};
    hp.in = m->x, hp.eps = c.norm_eps, hp.err = m->d_err;
    hp.amax = m->amax, hp.ticket = m->tickets + c.n_heads, hp.args = m->args;
    hp.prompt = m->prompt, hp.tokens = m->tokens, hp.max_seq = max_seq;
    gemv_plan(hp, m->d, m->num_sms, &m->head_smem);
    m->attn_smem = attn_smem_bytes(m->hd, max_seq);
    {
        size_t need = m->qkv_smem;
        need = need > m->wo_smem ? need : m->wo_smem;
        need = need > m->head_smem ? need : m->head_smem;
        if ((e = cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need)) !=
                cudaSuccess ||
            (e = cudaFuncSetAttribute(k_attn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)m->attn_smem)) != cudaSuccess ||
            (e = cudaFuncSetAttribute(k_attn_out, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)attn_out_smem_bytes(m->hd, max_seq))) != cudaSuccess)
            return fail("kernel attributes", e);
    }
    *out = m;
    if (dense) {
        if ((e = cudaMemcpy(m->dense, dense, dense_bytes, cudaMemcpyHostToDevice)) != cudaSuccess) {
            *out = nullptr;
            return fail("dense upload", e);
        }
        if (set_moe_layers(m, err, errlen)) {
            *out = nullptr;
            miag_model_close(m);
            return -1;
        }
    }
    return 0;
}

// The loader port of the file: blob (layer, expert) by pread.
namespace {
struct FileSource {
    FILE *f;
    uint64_t off, blob, n_experts;
};
int file_expert(void *ctx, int layer, int expert, void *dst) {
    FileSource *s = (FileSource *)ctx;
    const uint64_t at = s->off + ((uint64_t)layer * s->n_experts + (uint64_t)expert) * s->blob;
    if (fseeko(s->f, (off_t)at, SEEK_SET) != 0) return -1;
    return fread(dst, 1, s->blob, s->f) == s->blob ? 0 : -1;
}
}  // namespace

extern "C" int miag_model_open_file(miag_model **out, const char *path, int device, int max_seq,
                                    char *err, size_t errlen) {
    if (!out || !path) {
        put_err(err, errlen, "null argument");
        return -1;
    }
    *out = nullptr;
    FILE *f = fopen(path, "rb");
    if (!f) {
        put_err(err, errlen, "open %s failed", path);
        return -1;
    }
    MiaHeader h;
    if (fread(&h, 1, sizeof h, f) != sizeof h || memcmp(h.magic, "MIA1", 4) != 0 || h.version != 1) {
        fclose(f);
        put_err(err, errlen, "%s: not a .mia v1 file", path);
        return -1;
    }
    if (h.wtype != 1) {
        fclose(f);
        put_err(err, errlen, "%s: only Q8_0 models run on the GPU", path);
        return -1;
    }
    miag_mia_config c{};
    c.dim = h.dim, c.n_layers = h.n_layers, c.n_heads = h.n_heads, c.n_kv_heads = h.n_kv_heads;
    c.head_dim = h.head_dim, c.vocab = h.vocab, c.n_experts = h.n_experts, c.n_active = h.n_active;
    c.expert_hidden = h.expert_hidden, c.norm_topk = h.norm_topk, c.rope_theta = h.rope_theta;
    c.norm_eps = h.norm_eps;
    size_t dense_bytes = 0;
    if (mia_config_ok(c)) mia_dense_layout(c, &dense_bytes);
    if (!mia_config_ok(c) || h.dense_size != dense_bytes || h.expert_blob_size != miag_mia_expert_blob_bytes(&c)) {
        fclose(f);
        put_err(err, errlen, "%s: layout does not match its header", path);
        return -1;
    }
    std::vector<uint8_t> dense(dense_bytes);
    if (fseeko(f, (off_t)h.dense_offset, SEEK_SET) != 0 || fread(dense.data(), 1, dense_bytes, f) != dense_bytes) {
        fclose(f);
        put_err(err, errlen, "%s: short dense section", path);
        return -1;
    }
    miag_shape s{(int32_t)c.dim, (int32_t)c.n_layers, (int32_t)c.n_experts, (int32_t)c.n_active,
                 (int32_t)c.expert_hidden, (int32_t)c.norm_topk, c.norm_eps};
    miag_ctx *ctx = nullptr;
    if (miag_open(&ctx, &s, device, err, errlen)) {
        fclose(f);
        return -1;
    }
    FileSource src{f, h.experts_offset, h.expert_blob_size, h.n_experts};
    miag_model *m = nullptr;
    if (miag_load_experts(ctx, file_expert, &src, err, errlen) ||
        miag_model_open(&m, ctx, &c, dense.data(), dense_bytes, max_seq, err, errlen)) {
        fclose(f);
        miag_close(ctx);
        return -1;
    }
    fclose(f);
    m->owns_moe = true;
    *out = m;
    return 0;
}

extern "C" int miag_model_synth(miag_model *m, uint64_t seed, char *err, size_t errlen) {
    if (!m) {
        put_err(err, errlen, "null model");
        return -1;
    }
    MCU(cudaSetDevice(m->device));
    const miag_mia_config &c = m->cfg;
    const int grid = 4 * m->num_sms;
    for (size_t i = 0; i < m->layout.size(); i++) {
        const MiaTensor &t = m->layout[i];
        uint8_t *p = m->dense + t.offset;
        const bool is_router = t.name.size() > 6 && t.name.compare(t.name.size() - 6, 6, "router") == 0;
        if (t.quantized) {
            k_synth_q8<<<grid, 256, 0, m->stream>>>(p, t.rows * (t.cols / MIAG_QK),
                                                     sm_key(seed, {kTagDense, i, 0}),
                                                     sm_key(seed, {kTagDense, i, 1}), 0.02);
        } else if (is_router) {
            const int layer = (int)((i - 1) / kMiaLayerTensors);
            k_synth_f32<<<grid, 256, 0, m->stream>>>((float *)p, t.rows * t.cols,
                                                      sm_key(seed, {kTagRouter, (uint64_t)layer}),
                                                      0.02, 0);
        } else {
            k_synth_f32<<<grid, 256, 0, m->stream>>>((float *)p, t.rows * t.cols, 0, 0.0, 1);
        }
        MCU(cudaGetLastError());
    }
    // Experts: .mia blobs generated in device staging, then stored.
    const miag_shape &s = *ctx_shape(m->moe);
    const size_t blob = miag_blob_bytes(&s);
    const size_t nbg = (size_t)c.expert_hidden * (c.dim / MIAG_QK);   // gate / up blocks
    const size_t nbd = (size_t)c.dim * (c.expert_hidden / MIAG_QK);   // down blocks
    const size_t off_up = mia_align_up(nbg * 36, kMiaTensorAlign), off_down = 2 * off_up;
    const int batch = kSynthBatch;
    uint8_t *stage = nullptr;
    MCU(cudaMalloc(&stage, batch * blob));
    int rc = 0;
    for (int l = 0; l < (int)c.n_layers && rc == 0; l++)
        for (int e0 = 0; e0 < (int)c.n_experts && rc == 0; e0 += batch) {
            const int n = (int)c.n_experts - e0 < batch ? (int)c.n_experts - e0 : batch;
            SynthExperts se{};
            se.dst = stage, se.blob = blob, se.n = n, se.sigma = 0.02;
            se.off[0] = 0, se.off[1] = off_up, se.off[2] = off_down;
            se.nb[0] = nbg, se.nb[1] = nbg, se.nb[2] = nbd;
            for (int k = 0; k < n; k++)
                for (int mat = 0; mat < 3; mat++) {
                    const uint64_t e = (uint64_t)(e0 + k);
                    se.kq[k][mat] = sm_key(seed, {kTagQw, (uint64_t)l, e, (uint64_t)mat});
                    se.kd[k][mat] = sm_key(seed, {kTagDw, (uint64_t)l, e, (uint64_t)mat});
                }
            k_synth_experts<<<grid, 256, 0, m->stream>>>(se);
            if (cudaGetLastError() != cudaSuccess ||
                miag_upload_experts_device(m->moe, l, e0, n, stage, blob, m->stream, err, errlen))
                rc = -1;
        }
    cudaStreamSynchronize(m->stream);
    cudaFree(stage);
    if (rc) return -1;
    MCU(cudaStreamSynchronize(m->stream));
    return set_moe_layers(m, err, errlen);
}

// ---- batched prefill

namespace {

// Buffers for n positions (grown, never shrunk), and the MoE workspace for n
// tokens, reserved here while the model's stream is idle: a workspace grown
// by the MoE call itself would be freed under launches still queued on it.
int ensure_prefill(miag_model *m, int n, char *err, size_t errlen) {
    if (!ctx_reserve(m->moe, n, err, errlen)) return -1;
    if (n <= m->pf_cap) return 0;
    int cap = m->pf_cap ? m->pf_cap : 64;
    while (cap < n) cap *= 2;
    if (cap > m->max_seq) cap = m->max_seq;
    for (void *b : {(void *)m->pf_x, (void *)m->pf_qkv, (void *)m->pf_q, (void *)m->pf_att,
                    (void *)m->pf_xq, (void *)m->pf_tok})
        if (b) cudaFree(b);
    if (m->h_pf_tok) cudaFreeHost(m->h_pf_tok);
    m->pf_x = m->pf_qkv = m->pf_q = m->pf_att = nullptr;
    m->pf_xq = nullptr, m->pf_tok = nullptr, m->h_pf_tok = nullptr;
    m->pf_cap = 0;
    const size_t pitch = (size_t)(pf_pitch(m->d) > pf_pitch(m->qd) ? pf_pitch(m->d) : pf_pitch(m->qd));
    struct {
        void **p;
        size_t bytes;
    } allocs[] = {
        {(void **)&m->pf_x, (size_t)cap * m->d * 4},
        {(void **)&m->pf_qkv, (size_t)cap * (m->qd + 2 * m->kvd) * 4},
        {(void **)&m->pf_q, (size_t)cap * m->qd * 4},
        {(void **)&m->pf_att, (size_t)cap * m->qd * 4},
        {(void **)&m->pf_xq, (size_t)cap * pitch},
        {(void **)&m->pf_tok, (size_t)cap * 4},
    };
    for (auto &a : allocs) MCU(cudaMalloc(a.p, a.bytes));
    MCU(cudaMallocHost(&m->h_pf_tok, (size_t)cap * 4));
    const size_t gsm = std::max(pf_gemv_smem(m->d), pf_gemv_smem(m->qd));
    MCU(cudaFuncSetAttribute(k_pf_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm));
    MCU(cudaFuncSetAttribute(k_pf_attn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)((m->hd + m->max_seq) * 4)));
    if (m->hd <= kPfTiledMaxHd)
        MCU(cudaFuncSetAttribute(k_pf_attn_tiled, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)pf_attn_tiled_smem(m->hd, kPfTiledMaxPos)));
    MCU(cudaFuncSetAttribute(k_pf_quant, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)((m->d > m->qd ? m->d : m->qd) * 4)));
    m->pf_cap = cap;
    return 0;
}

int pf_gemv(miag_model *m, const uint8_t *w, int rows, int cols, float *out, int out_stride, int resid,
            int n, cudaStream_t s, char *err, size_t errlen) {
    PfGemvParams g{};
    g.w = w, g.rows = rows, g.cols = cols;
    g.xq = m->pf_xq, g.pitch = pf_pitch(cols), g.n = n;
    g.out = out, g.out_stride = out_stride, g.resid = resid, g.err = m->d_err;
    const dim3 grid((unsigned)((rows + kPfRows - 1) / kPfRows), (unsigned)((n + kPfTok - 1) / kPfTok));
    MCU(launch_dependent(k_pf_gemv, grid, dim3(kPfThreads), pf_gemv_smem(cols), s, g));
    return 0;
}

// The launch sequence of a prefill of n positions from pos0 (tokens in
// pf_tok): per layer 8 launches and the MoE block's, then the head.
int enqueue_prefill(miag_model *m, int n, int pos0, cudaStream_t s, char *err, size_t errlen) {
    const miag_mia_config &c = m->cfg;
    const int d = m->d, qd = m->qd, kvd = m->kvd, hd = m->hd, qkv_w = qd + 2 * kvd;
    int launches = 0;
    MCU(launch_dependent(k_pf_embed, dim3((unsigned)n), dim3(256), 0, s, m->pf_x, tensor(m, 0),
                         (const int32_t *)m->pf_tok, d, (int)c.vocab, m->d_err));
    launches++;
    for (int l = 0; l < (int)c.n_layers; l++) {
        MCU(launch_dependent(k_pf_quant, dim3((unsigned)n), dim3(kPfThreads), (size_t)d * 4, s,
                             (const float *)m->pf_x, d, tensor_f(m, mia_layer_tensor(l, kAttnNorm)),
                             c.norm_eps, d, m->pf_xq, pf_pitch(d)));
        if (pf_gemv(m, tensor(m, mia_layer_tensor(l, kWq)), qd, d, m->pf_qkv, qkv_w, 0, n, s, err, errlen) ||
            pf_gemv(m, tensor(m, mia_layer_tensor(l, kWk)), kvd, d, m->pf_qkv + qd, qkv_w, 0, n, s, err,
                    errlen) ||
            pf_gemv(m, tensor(m, mia_layer_tensor(l, kWv)), kvd, d, m->pf_qkv + qd + kvd, qkv_w, 0, n, s, err,
                    errlen))
            return -1;
        const size_t layer_off = (size_t)l * m->max_seq * kvd;
        PfQkParams qk{};
        qk.qkv = m->pf_qkv;
        qk.q_norm = tensor_f(m, mia_layer_tensor(l, kQNorm));
        qk.k_norm = tensor_f(m, mia_layer_tensor(l, kKNorm));
        qk.rope = m->rope, qk.q = m->pf_q;
        qk.kc = m->kc + layer_off, qk.vc = m->vc + layer_off;
        qk.nh = (int)c.n_heads, qk.nkv = (int)c.n_kv_heads, qk.hd = hd, qk.pos0 = pos0;
        qk.eps = c.norm_eps;
        MCU(launch_dependent(k_pf_qk, dim3((unsigned)n, c.n_heads + c.n_kv_heads), dim3(32), (size_t)hd * 4, s,
                             qk));
        PfAttnParams at{};
        at.q = m->pf_q, at.kc = m->kc + layer_off, at.vc = m->vc + layer_off, at.att = m->pf_att;
        at.nh = (int)c.n_heads, at.nkv = (int)c.n_kv_heads, at.hd = hd, at.pos0 = pos0, at.max_seq = m->max_seq;
        at.scale = 1.0f / sqrtf((float)hd);  // forward.c:143
        at.n = n;
        const int group = (int)(c.n_heads / c.n_kv_heads);
        if (pos0 + n <= kPfTiledMaxPos && hd <= kPfTiledMaxHd && hd % 16 == 0 && group <= kPfQ) {
            const int TQ = pf_tq(group);
            MCU(launch_dependent(k_pf_attn_tiled, dim3(c.n_kv_heads, (unsigned)((n + TQ - 1) / TQ)),
                                 dim3(4 * kPfQ), pf_attn_tiled_smem(hd, pos0 + n), s, at));
        } else {
            MCU(launch_dependent(k_pf_attn, dim3(c.n_heads, (unsigned)n), dim3(kPfAttnThreads),
                                 (size_t)(hd + pos0 + n) * 4, s, at));
        }
        MCU(launch_dependent(k_pf_quant, dim3((unsigned)n), dim3(kPfThreads), (size_t)qd * 4, s,
                             (const float *)m->pf_att, qd, (const float *)nullptr, c.norm_eps, qd, m->pf_xq,
                             pf_pitch(qd)));
        if (pf_gemv(m, tensor(m, mia_layer_tensor(l, kWo)), d, qd, m->pf_x, d, 1, n, s, err, errlen)) return -1;
        launches += 8;
        if (miag_moe_async(m->moe, l, m->pf_x, n, s, err, errlen) != 0) return -1;
        launches += miag_last_launch_count(m->moe);
    }
    GemvParams hp = m->head_p;
    const size_t nt = m->layout.size();
    hp.seg[0].w = tensor(m, nt - 1);
    hp.norm = tensor_f(m, nt - 2);
    hp.in = m->pf_x + (size_t)(n - 1) * d;
    hp.best = m->smp_temp > 0.0f ? &m->smp->best : nullptr;
    MCU(gemv_launch(hp, grid_of(m, hp), m->head_smem, s));
    launches++;
    if (m->smp_temp > 0.0f) {
        if (enqueue_sample(m, s, err, errlen)) return -1;
        launches += 3;
    }
    m->pf_last_launches = launches;
    return 0;
}

// Checks and stages a prefill of tokens[0 .. n) at positions pos0 .. :
// the tokens into pf_tok and the sequence record, the step arguments as the
// one-position path leaves them before the last position's head.
int stage_prefill(miag_model *m, const int32_t *tokens, int n, int pos0, char *err, size_t errlen) {
    if (!m || !m->dense_set) {
        put_err(err, errlen, m ? "the model has no weights (miag_model_synth)" : "null model");
        return -1;
    }
    if (!tokens || n < 1 || pos0 < 0 || (size_t)pos0 + (size_t)n > (size_t)m->max_seq) {
        put_err(err, errlen, "bad prefill: %d tokens from position %d (context %d)", n, pos0, m->max_seq);
        return -1;
    }
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= (int)m->cfg.vocab) {
            put_err(err, errlen, "prompt token %d out of range", i);
            return -1;
        }
    MCU(cudaSetDevice(m->device));
    MCU(cudaStreamSynchronize(m->stream));  // pinned staging free; no launch uses the workspace
    if (ensure_prefill(m, n, err, errlen)) return -1;
    memcpy(m->h_pf_tok, tokens, (size_t)n * 4);
    MCU(cudaMemcpyAsync(m->pf_tok, m->h_pf_tok, (size_t)n * 4, cudaMemcpyHostToDevice, m->stream));
    MCU(cudaMemcpyAsync(m->tokens + pos0, m->pf_tok, (size_t)n * 4, cudaMemcpyDeviceToDevice, m->stream));
    m->h_args[0] = tokens[n - 1], m->h_args[1] = pos0 + n - 1;
    MCU(cudaMemcpyAsync(m->args, m->h_args, 8, cudaMemcpyHostToDevice, m->stream));
    return 0;
}

}  // namespace

extern "C" int miag_model_prefill_async(miag_model *m, const int32_t *tokens, int n, int pos, char *err,
                                        size_t errlen) {
    if (stage_prefill(m, tokens, n, pos, err, errlen)) return -1;
    return enqueue_prefill(m, n, pos, m->stream, err, errlen);
}

extern "C" const float *miag_model_prefill(miag_model *m, const int32_t *tokens, int n, int pos, char *err,
                                           size_t errlen) {
    if (miag_model_prefill_async(m, tokens, n, pos, err, errlen)) return nullptr;
    if (cudaMemcpyAsync(m->h_logits, m->logits, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost,
                        m->stream) != cudaSuccess) {
        put_err(err, errlen, "logits copy failed");
        return nullptr;
    }
    if (check_errors(m, err, errlen)) return nullptr;
    return m->h_logits;
}

extern "C" int miag_model_set_sampler(miag_model *m, float temperature, float top_p, uint64_t seed, char *err,
                                      size_t errlen) {
    if (!m) {
        put_err(err, errlen, "null model");
        return -1;
    }
    MCU(cudaSetDevice(m->device));
    MCU(cudaStreamSynchronize(m->stream));
    const int n = (int)m->cfg.vocab;
    if (!m->smp) {
        MCU(cudaMalloc(&m->smp, sizeof(SmpState)));
        MCU(cudaMemset(m->smp, 0, sizeof(SmpState)));
        MCU(cudaMalloc(&m->smp_e, (size_t)n * 4));
        MCU(cudaMalloc(&m->smp_p, (size_t)n * 4));
        MCU(cudaMalloc(&m->smp_k0, (size_t)n * 8));
        MCU(cudaMalloc(&m->smp_k1, (size_t)n * 8));
        size_t bytes = 0;
        MCU(cub::DeviceRadixSort::SortKeys(nullptr, bytes, m->smp_k0, m->smp_k1, n, 0, 64, m->stream));
        MCU(cudaMalloc(&m->smp_tmp, bytes));
        m->smp_tmp_bytes = bytes;
    }
    // sampler.c:7-10: top_p outside (0, 1] means 1; a zero seed a fixed one
    SmpState st{};
    st.rng = seed ? seed : 0x2545F4914F6CDD1DULL;
    MCU(cudaMemcpy(m->smp, &st, sizeof st, cudaMemcpyHostToDevice));
    m->smp_temp = temperature > 0.0f ? temperature : 0.0f;
    m->smp_top_p = top_p > 0.0f && top_p <= 1.0f ? top_p : 1.0f;
    if (m->exec) cudaGraphExecDestroy(m->exec);  // the step's launches change
    m->exec = nullptr;
    return 0;
}

extern "C" int miag_model_set_batched_prefill(miag_model *m, int on) {
    if (!m) return -1;
    m->batched_prefill = on != 0;
    return 0;
}

extern "C" int miag_model_prefill_launches(const miag_model *m) { return m ? m->pf_last_launches : -1; }

extern "C" int miag_model_step_async(miag_model *m, int token, int pos, char *err, size_t errlen) {
    if (!m || !m->dense_set) {
        put_err(err, errlen, m ? "the model has no weights (miag_model_synth)" : "null model");
        return -1;
    }
    if (pos < 0 || pos >= m->max_seq || token < 0 || token >= (int)m->cfg.vocab) {  // forward.c:202-203
        put_err(err, errlen, "token %d at position %d out of range", token, pos);
        return -1;
    }
    MCU(cudaSetDevice(m->device));
    const int32_t a[2] = {token, pos};
    MCU(cudaStreamSynchronize(m->stream));  // the pinned arguments are free again
    memcpy(m->h_args, a, sizeof a);
    MCU(cudaMemcpyAsync(m->args, m->h_args, sizeof a, cudaMemcpyHostToDevice, m->stream));
    return launch_steps(m, 1, err, errlen);
}

extern "C" const float *miag_model_step(miag_model *m, int token, int pos, char *err, size_t errlen) {
    if (miag_model_step_async(m, token, pos, err, errlen)) return nullptr;
    if (cudaMemcpyAsync(m->h_logits, m->logits, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost,
                        m->stream) != cudaSuccess) {
        put_err(err, errlen, "logits copy failed");
        return nullptr;
    }
    if (check_errors(m, err, errlen)) return nullptr;
    return m->h_logits;
}

extern "C" int miag_model_generate_async(miag_model *m, const int32_t *prompt, int n_prompt,
                                         int n_new, char *err, size_t errlen) {
    if (!m || !m->dense_set || !prompt || n_prompt < 1 || n_new < 0 ||
        (size_t)n_prompt + (size_t)n_new > (size_t)m->max_seq) {
        put_err(err, errlen, "bad arguments (a prompt of >= 1 token; prompt + new <= context)");
        return -1;
    }
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= (int)m->cfg.vocab) {
            put_err(err, errlen, "prompt token %d out of range", i);
            return -1;
        }
    MCU(cudaSetDevice(m->device));
    MCU(cudaStreamSynchronize(m->stream));
    MCU(cudaMemcpyAsync(m->prompt, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, m->stream));
    MCU(cudaMemcpyAsync(m->tokens, prompt, 4, cudaMemcpyHostToDevice, m->stream));
    m->h_args[0] = prompt[0], m->h_args[1] = 0;
    MCU(cudaMemcpyAsync(m->args, m->h_args, 8, cudaMemcpyHostToDevice, m->stream));
    // the head reads n_prompt from its parameters: set it and re-capture
    if (m->head_p.n_prompt != n_prompt) {
        m->head_p.n_prompt = n_prompt;
        if (m->exec) cudaGraphExecDestroy(m->exec);
        m->exec = nullptr;
    }
    if (m->batched_prefill && n_prompt > 1) {
        // the prompt in one batched pass: its head leaves the first new
        // token and the position n_prompt in the step arguments
        if (stage_prefill(m, prompt, n_prompt, 0, err, errlen) ||
            enqueue_prefill(m, n_prompt, 0, m->stream, err, errlen))
            return -1;
        return launch_steps(m, n_new > 0 ? n_new - 1 : 0, err, errlen);
    }
    const int steps = n_prompt + n_new - 1;
    return launch_steps(m, steps, err, errlen);
}

extern "C" int miag_model_continue_async(miag_model *m, int n_steps, char *err, size_t errlen) {
    if (!m || !m->dense_set || n_steps < 0) {
        put_err(err, errlen, "bad arguments");
        return -1;
    }
    MCU(cudaSetDevice(m->device));
    return launch_steps(m, n_steps, err, errlen);
}

extern "C" int miag_model_generate(miag_model *m, const int32_t *prompt, int n_prompt, int n_new,
                                   int32_t *tokens_out, char *err, size_t errlen) {
    if (!tokens_out && n_new > 0) {
        put_err(err, errlen, "null output");
        return -1;
    }
    if (miag_model_generate_async(m, prompt, n_prompt, n_new, err, errlen)) return -1;
    if (n_new > 0 && cudaMemcpyAsync(tokens_out, m->tokens + n_prompt, (size_t)n_new * 4,
                                     cudaMemcpyDeviceToHost, m->stream) != cudaSuccess) {
        put_err(err, errlen, "token copy failed");
        return -1;
    }
    return check_errors(m, err, errlen);
}

extern "C" int miag_model_sync(miag_model *m, char *err, size_t errlen) {
    if (!m) {
        put_err(err, errlen, "null model");
        return -1;
    }
    MCU(cudaSetDevice(m->device));
    return check_errors(m, err, errlen);
}

extern "C" const float *miag_model_logits_device(const miag_model *m) { return m ? m->logits : nullptr; }
extern "C" const int32_t *miag_model_tokens_device(const miag_model *m) { return m ? m->tokens : nullptr; }
extern "C" void *miag_model_stream(const miag_model *m) { return m ? (void *)m->stream : nullptr; }
extern "C" miag_ctx *miag_model_moe(const miag_model *m) { return m ? m->moe : nullptr; }
extern "C" int miag_model_launches_per_step(const miag_model *m) { return m ? m->last_launches : -1; }
extern "C" int miag_model_uses_graph(const miag_model *m) { return m && m->exec && !m->eager ? 1 : 0; }
