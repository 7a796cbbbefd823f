// noalloc.cu -- the MoE block with no memory allocation at call time.
//
// miag_moe_async grows the context's workspace with cudaMalloc when a call
// brings more tokens than any call before it.  Some callers must never see
// that: an engine that reserves all device memory up front under a fixed
// budget (the way motorIa sizes everything from its RAM budget), or a
// serving loop that cannot afford cudaMalloc's implicit device-wide
// synchronisation in the middle of a step.  miag_moe_noalloc gives them the
// same block with its scratch in a fixed array that is part of the loaded
// library: nothing is allocated, freed or grown by the call.
//
// The scratch is one file-scope __device__ array of kNoAllocScratchBytes.
// Every GPU that loads libmiag holds it until the process exits.  Its device
// address is looked up once per device, with that device current, and then
// reused; the first call on a device does that set-up, so it should come
// before any stream capture that contains later calls.
//
// All calls share the one array and it keeps whatever the last call left
// there.  Two things in it must start at zero: the router's per-token-group
// counters and the expert launches' SM-share claims, which sit first, at a
// fixed place for every batch size.  The array starts zeroed when the
// library loads and every call that runs to its end leaves them at zero
// again; when a call reports a device error (miag_sync, miag_moe), the
// library clears them once more on that device, so a call cut short cannot
// corrupt the next one.  Every other buffer of the block is written before it
// is read.  Two calls whose work overlaps on the GPU (other streams, other
// contexts on the same device) race on the array and must be serialised by
// the caller.  The address looked up at set-up is kept for the life of the
// process: a device reset (cudaDeviceReset) while libmiag is loaded is not
// supported.
#include <cstdio>
#include <mutex>

#include "../../include/miag/miag.h"
#include "kernels.cuh"

namespace miag {
int ctx_view(const miag_ctx *c, int layer, CtxView *v);
}

using namespace miag;

namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)11 << 20;  // 11 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void *g_scratch_dev[kMaxDevices];  // device address of g_noalloc_scratch, per device

void put_err(char *err, size_t errlen, const char *msg) {
    if (err && errlen) snprintf(err, errlen, "%s", msg);
}

// Looks up the array's device address for the current device (once).  In host
// code g_noalloc_scratch names a host-side stand-in, not device memory.
void *scratch_for(int device, char *err, size_t errlen) {
    if (device < 0 || device >= kMaxDevices) {
        put_err(err, errlen, "miag_moe_noalloc: device index beyond the set-up table");
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_dev[device]) {
        void *ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr) {
            if (err && errlen)
                snprintf(err, errlen, "miag_moe_noalloc: cudaGetSymbolAddress: %s",
                         cudaGetErrorString(e));
            return nullptr;
        }
        g_scratch_dev[device] = ptr;
    }
    return g_scratch_dev[device];
}

size_t bump(uint8_t *&p, size_t bytes) {
    const size_t off = (size_t)(reinterpret_cast<uintptr_t>(p));
    p += round_up_sz(bytes, 256);
    return off;
}

constexpr int kNoAllocGroups = 1024;  // token-group counters, at offset 0

// Lays the block's buffers for T tokens out from `base`; returns the bytes used.
size_t layout(const Dims &m, int T, uint8_t *base, Work *w) {
    const size_t P = (size_t)T * m.K;
    const int nchunks = (int)((P + kPermChunk - 1) / kPermChunk);
    const int xs = scale_pad(m.d / MIAG_QK);
    uint8_t *p = base;
    Work v{};
    v.T = T, v.P = (int)P, v.nchunks = nchunks;
    v.tg_count = reinterpret_cast<int32_t *>(bump(p, (size_t)kNoAllocGroups * 4));
    v.shares = reinterpret_cast<uint8_t *>(bump(p, kShareKinds * sizeof(ShareState)));  // fixed offset too
    v.xq = reinterpret_cast<int8_t *>(bump(p, (size_t)T * m.d));
    v.dx = reinterpret_cast<float *>(bump(p, (size_t)T * xs * 4));
    v.logits = reinterpret_cast<float *>(bump(p, (size_t)T * m.E * 4));
    v.idx = reinterpret_cast<int32_t *>(bump(p, P * 4));
    v.w = reinterpret_cast<float *>(bump(p, P * 4));
    v.rank = reinterpret_cast<int32_t *>(bump(p, P * 4));
    v.chunk_cnt = reinterpret_cast<int32_t *>(bump(p, (size_t)nchunks * m.E * 4));
    v.chunk_base = reinterpret_cast<int32_t *>(bump(p, (size_t)nchunks * m.E * 4));
    v.counts = reinterpret_cast<int32_t *>(bump(p, (size_t)m.E * 4));
    v.offsets = reinterpret_cast<int32_t *>(bump(p, (size_t)(m.E + 1) * 4));
    v.active = reinterpret_cast<int32_t *>(bump(p, (size_t)m.E * 4));
    v.n_active = reinterpret_cast<int32_t *>(bump(p, 4));
    v.chunk_pre = reinterpret_cast<int32_t *>(bump(p, (size_t)(m.E + 1) * 4));
    v.chunk_info = reinterpret_cast<int4 *>(bump(p, (P / kTokChunkNarrow + m.E + 1) * 16));
    v.max_chunk = reinterpret_cast<int32_t *>(bump(p, 4));
    v.chunk_done = reinterpret_cast<int32_t *>(bump(p, (P / kTokChunkNarrow + m.E + 1) * 4));
    v.perm = reinterpret_cast<int32_t *>(bump(p, P * 4));
    v.inv = reinterpret_cast<int32_t *>(bump(p, P * 4));
    v.h = reinterpret_cast<float *>(bump(p, P * 2 * m.eh * 4));
    v.hq = reinterpret_cast<int8_t *>(bump(p, P * m.eh));
    v.hs = reinterpret_cast<float *>(bump(p, P * scale_pad(m.eh / MIAG_QK) * 4));
    v.y = reinterpret_cast<float *>(bump(p, P * m.d * 4));
    if (w) *w = v;
    return (size_t)(p - base);
}

}  // namespace

namespace miag {
// Zeroes the counters at the head of the array on `device` (after a call
// reported a device error), if the array was ever set up there.  Enqueued on
// `s`; allocates nothing.
void noalloc_clear_counters(int device, cudaStream_t s) {
    if (device < 0 || device >= kMaxDevices) return;
    void *ptr;
    {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        ptr = g_scratch_dev[device];
    }
    if (!ptr) return;
    uint8_t *base = nullptr;
    Work w;
    layout(Dims{}, 0, base, &w);  // offsets of the counters from the array's start
    const size_t head = reinterpret_cast<size_t>(w.shares) + kShareKinds * sizeof(ShareState);
    cudaMemsetAsync(ptr, 0, head, s);
}
}  // namespace miag

extern "C" int miag_moe_noalloc(miag_ctx *c, int layer, float *x_dev, int n_tokens, void *stream,
                                char *err, size_t errlen) {
    CtxView v;
    if (ctx_view(c, layer, &v) != 0) {
        put_err(err, errlen, "miag_moe_noalloc: null context, bad layer, or layer not set");
        return -1;
    }
    if (n_tokens < 0 || (n_tokens > 0 && !x_dev) || ((uintptr_t)x_dev & 15u)) {
        put_err(err, errlen, "miag_moe_noalloc: bad token buffer (device pointer, 16-byte aligned)");
        return -1;
    }
    if (n_tokens == 0) return 0;
    const size_t need = layout(v.dims, n_tokens, nullptr, nullptr);
    if (need > kNoAllocScratchBytes || n_tokens > kNoAllocGroups) {
        if (err && errlen)
            snprintf(err, errlen,
                     "miag_moe_noalloc: %d tokens need %zu bytes of scratch, more than its fixed "
                     "%zu-byte array; use miag_moe_async for batches this large",
                     n_tokens, need, kNoAllocScratchBytes);
        return -1;
    }
    cudaError_t e = cudaSetDevice(v.device);
    if (e != cudaSuccess) {
        if (err && errlen) snprintf(err, errlen, "miag_moe_noalloc: cudaSetDevice: %s",
                                    cudaGetErrorString(e));
        return -1;
    }
    void *scratch = scratch_for(v.device, err, errlen);
    if (!scratch) return -1;
    Work w;
    layout(v.dims, n_tokens, static_cast<uint8_t *>(scratch), &w);
    const cudaStream_t s = stream ? (cudaStream_t)stream : v.stream;
    launch_route(v.dims, v.layer, x_dev, w, v.d_err, s);
    launch_permute(v.dims, w, v.d_err, s);
    launch_gateup(v.dims, v.lay, v.layer, w, v.num_sms, v.d_err, s);
    launch_down(v.dims, v.lay, v.layer, w, v.num_sms, v.d_err, s);
    launch_combine(v.dims, w, x_dev, v.d_err, s);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        if (err && errlen) snprintf(err, errlen, "miag_moe_noalloc: launch: %s",
                                    cudaGetErrorString(e));
        return -1;
    }
    return 0;
}
