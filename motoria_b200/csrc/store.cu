// store.cu -- HBM-resident expert store, filled once at load time.
//
// Replaces the reference's disk-streamed LRU slot cache
// (src/storage/expert_cache.c:59-85): blobs arrive in .mia layout (gate | up
// | down, each a row-major matrix of 36-byte {f32 d; int8 q[32]} blocks,
// src/storage/mia_file.c:275-278) and are repacked on the device into the
// row-aligned planes of StoreLayout (common.cuh).  Values are copied, never
// re-quantized, so the stored weights are the reference's bit for bit.
#include "kernels.cuh"

namespace miag {

// One thread per Q8_0 block of one output row.
__global__ void k_repack(const uint8_t *aos, size_t aos_stride, size_t off_up, size_t off_down,
                         int d, int eh, StoreLayout lay, uint8_t *dst) {
    const int row = blockIdx.x;  // 0 .. 2*eh + d - 1
    const int ex = blockIdx.y;
    const uint8_t *blob = aos + (size_t)ex * aos_stride;
    uint8_t *out = dst + (size_t)ex * lay.expert_bytes;
    const uint8_t *src;
    uint8_t *q_out;
    float *s_out;
    int nb;
    uint32_t s_row;
    if (row < 2 * eh) {
        const int i = row >> 1;
        nb = d / MIAG_QK;
        src = blob + ((row & 1) ? off_up : 0) + (size_t)i * nb * 36;
        q_out = out + lay.gu_q_off + (size_t)row * d;
        s_out = reinterpret_cast<float *>(out + lay.gu_s_off + (size_t)row * lay.gu_s_row);
        s_row = lay.gu_s_row;
    } else {
        const int r = row - 2 * eh;
        nb = eh / MIAG_QK;
        src = blob + off_down + (size_t)r * nb * 36;
        q_out = out + lay.dn_q_off + (size_t)r * eh;
        s_out = reinterpret_cast<float *>(out + lay.dn_s_off + (size_t)r * lay.dn_s_row);
        s_row = lay.dn_s_row;
    }
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
        const uint32_t *blk = reinterpret_cast<const uint32_t *>(src + (size_t)b * 36);
        s_out[b] = __uint_as_float(blk[0]);
        uint32_t *qo = reinterpret_cast<uint32_t *>(q_out + (size_t)b * MIAG_QK);
#pragma unroll
        for (int k = 0; k < 8; k++) qo[k] = blk[1 + k];
    }
    // zero the 16-byte padding of the scale row
    for (int b = nb + threadIdx.x; b < (int)(s_row / 4); b += blockDim.x) s_out[b] = 0.0f;
}

__global__ void k_transpose(const float *in, float *out, int rows, int cols) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int r = r0 + k, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[k][threadIdx.x] = in[(size_t)r * cols + c];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int c = c0 + k, r = r0 + threadIdx.x;
        if (r < rows && c < cols) out[(size_t)c * rows + r] = tile[threadIdx.x][k];
    }
}

void launch_repack(const Dims &m, const StoreLayout &lay, const uint8_t *aos, size_t aos_stride,
                   int n, uint8_t *dst, cudaStream_t s) {
    const size_t mat = (size_t)m.eh * (m.d / MIAG_QK) * 36;
    const size_t off_up = round_up_sz(mat, 64);
    const size_t off_down = 2 * off_up;
    dim3 grid(2 * m.eh + m.d, n);
    k_repack<<<grid, 64, 0, s>>>(aos, aos_stride, off_up, off_down, m.d, m.eh, lay, dst);
}

void launch_transpose_router(const float *router, float *router_t, int E, int d,
                             cudaStream_t s) {
    dim3 grid((d + 31) / 32, (E + 31) / 32);
    k_transpose<<<grid, dim3(32, 8), 0, s>>>(router, router_t, E, d);
}

}  // namespace miag
