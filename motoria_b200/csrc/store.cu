// store.cu -- HBM-resident expert store, filled once at load time.
//
// Replaces the reference's disk-streamed LRU slot cache
// (src/storage/expert_cache.c:59-85): blobs arrive in .mia layout (gate | up
// | down, each a row-major matrix of 36-byte {f32 d; int8 q[32]} blocks,
// src/storage/mia_file.c:275-278) and are repacked on the device into the
// swizzled 128 x 128 B tile units of StoreLayout (common.cuh).  Values are
// copied, never re-quantized, so the stored weights are the reference's bit
// for bit.
#include "kernels.cuh"

namespace miag {

// One thread per Q8_0 block of one matrix row: the 32 int8 values become two
// 16-byte chunks of a swizzled tile, the scale one f32 of the scale tile.
__global__ void k_repack(const uint8_t *aos, size_t aos_stride, size_t off_up, size_t off_down,
                         int d, int eh, StoreLayout lay, uint8_t *dst) {
    const int row = blockIdx.x;  // 0 .. 2*eh + d - 1
    const int ex = blockIdx.y;
    const uint8_t *blob = aos + (size_t)ex * aos_stride;
    uint8_t *out = dst + (size_t)ex * lay.expert_bytes;
    const uint8_t *src;
    uint8_t *units;
    int nb, r, kt_count;
    if (row < 2 * eh) {
        const int i = row >> 1;
        nb = d / MIAG_QK;
        src = blob + ((row & 1) ? off_up : 0) + (size_t)i * nb * 36;
        units = out + lay.gu_off;
        r = row, kt_count = lay.gu_kt;
    } else {
        r = row - 2 * eh;
        nb = eh / MIAG_QK;
        src = blob + off_down + (size_t)r * nb * 36;
        units = out + lay.dn_off;
        kt_count = lay.dn_kt;
    }
    const int rt = r / kTileRows, rr = r % kTileRows;
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
        const uint32_t *blk = reinterpret_cast<const uint32_t *>(src + (size_t)b * 36);
        const int kt = b / 4, jb = b % 4;
        uint8_t *tq = units + ((size_t)rt * kt_count + kt) * kUnitBytes;
        reinterpret_cast<float *>(tq + kTileBytes)[rr * 4 + jb] = __uint_as_float(blk[0]);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            uint4 v = make_uint4(blk[1 + 4 * h], blk[2 + 4 * h], blk[3 + 4 * h], blk[4 + 4 * h]);
            *reinterpret_cast<uint4 *>(tq + tile_chunk_offset(rr, 2 * jb + h)) = v;
        }
    }
}

// router [E][d] -> grouped [ceil(E/32)][d/4][32][4]: a group of 32 experts is
// one contiguous slice; within it, the weights of expert 32g + l for inputs
// 4j .. 4j+3 are one 16-byte vector, lane l's in a row of 32.
__global__ void k_group_router(const float *in, float *out, int E, int d) {
    __shared__ float tile[32][33];
    const int i0 = blockIdx.x * 32, g = blockIdx.y;
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int e = g * 32 + k, i = i0 + threadIdx.x;
        tile[k][threadIdx.x] = (e < E && i < d) ? in[(size_t)e * d + i] : 0.0f;
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int i = i0 + k;
        if (i < d) out[(((size_t)g * (d / 4) + i / 4) * 32 + threadIdx.x) * 4 + (i & 3)] = tile[threadIdx.x][k];
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

void launch_transpose_router(const float *router, float *router_g, int E, int d,
                             cudaStream_t s) {
    dim3 grid((d + 31) / 32, (E + 31) / 32);
    k_group_router<<<grid, dim3(32, 8), 0, s>>>(router, router_g, E, d);
}

}  // namespace miag
