// mathapi.cu -- device versions of the reference's public math ABI.
//
//   miag_quantize_row_q8 <- mia_quantize_row_q8 (src/tensor/quant.c:11-27)
//   miag_matvec          <- mia_matvec          (src/tensor/matmul.c:91-106)
//
// Both keep the reference's data layouts (36-byte Q8_0 blocks, row-major
// f32) and its exact arithmetic; they serve engine callers outside the MoE
// block (attention and LM-head matvecs) and are the unit-level parity probes
// of the quantizer and the Q8_0 dot.
#include "../../include/miag/miag.h"
#include "kernels.cuh"

namespace miag {

// One warp per 32-value block; y is an array of 36-byte mia_block_q8.
__global__ void k_quantize_aos(const float *x, uint8_t *y, int nblocks) {
    const int lane = threadIdx.x & 31;
    const long b = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (b >= nblocks) return;
    const float v = x[b * MIAG_QK + lane];
    float a = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const float dq = __fdiv_rn(a, 127.0f);
    const float id = dq != 0.0f ? __fdiv_rn(1.0f, dq) : 0.0f;
    uint8_t *blk = y + b * 36;
    blk[4 + lane] = (uint8_t)(int8_t)roundf(__fmul_rn(v, id));
    if (lane == 0) *reinterpret_cast<float *>(blk) = dq;
}

// One thread per output row, blocks in order: dot_q8_scalar (matmul.c:19-28).
__global__ void k_matvec_q8_aos(float *out, const uint8_t *w, const uint8_t *xq, int rows,
                                int nb) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const uint8_t *wr = w + (size_t)r * nb * 36;
    float s = 0.0f;
    for (int b = 0; b < nb; b++) {
        const uint32_t *wb = reinterpret_cast<const uint32_t *>(wr + (size_t)b * 36);
        const uint32_t *xb = reinterpret_cast<const uint32_t *>(xq + (size_t)b * 36);
        int acc = 0;
#pragma unroll
        for (int k = 1; k < 9; k++) acc = __dp4a((int)__ldg(wb + k), (int)__ldg(xb + k), acc);
        s = q8_step(s, acc, __uint_as_float(__ldg(wb)), __uint_as_float(__ldg(xb)));
    }
    out[r] = s;
}

// One thread per output row, serial: dot_f32_scalar (matmul.c:13-17).
__global__ void k_matvec_f32(float *out, const float *w, const float *x, int rows, int cols) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const float *wr = w + (size_t)r * cols;
    float s = 0.0f;
    for (int i = 0; i < cols; i++) s = __fadd_rn(s, __fmul_rn(__ldg(wr + i), __ldg(x + i)));
    out[r] = s;
}

}  // namespace miag

extern "C" int miag_quantize_row_q8(const float *x, void *y, int n, void *stream) {
    if (!x || !y || n < 0 || n % MIAG_QK) return -1;
    const int nb = n / MIAG_QK;
    if (nb == 0) return 0;
    const long threads = (long)nb * 32;
    miag::k_quantize_aos<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        x, (uint8_t *)y, nb);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

extern "C" int miag_matvec(float *out, const void *w, int wtype, const float *x, void *xq,
                           int rows, int cols, void *stream) {
    if (!out || !w || !x || rows < 0 || cols < 0) return -1;
    if (rows == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    const unsigned grid = (unsigned)((rows + 127) / 128);
    if (wtype == 0) {
        miag::k_matvec_f32<<<grid, 128, 0, s>>>(out, (const float *)w, x, rows, cols);
    } else if (wtype == 1) {
        if (!xq || cols % MIAG_QK) return -1;
        if (miag_quantize_row_q8(x, xq, cols, stream) != 0) return -1;
        miag::k_matvec_q8_aos<<<grid, 128, 0, s>>>(out, (const uint8_t *)w, (const uint8_t *)xq,
                                                    rows, cols / MIAG_QK);
    } else {
        return -1;
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
