// api.cu -- the libmiag C ABI (include/miag/miag.h): context, HBM expert
// store, workspace and the MoE block launch sequence.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <new>
#include <vector>

#include "../../include/miag/miag.h"
#include <algorithm>

#include "host_copy.h"
#include "kernels.cuh"

using namespace miag;

namespace {

struct LayerState {
    float *ffn_norm = nullptr;
    float *router_t = nullptr;
    float *bias = nullptr;
    bool has_bias = false;
    bool dense_set = false;
    uint8_t *experts = nullptr;
};

}  // namespace

struct miag_ctx {
    miag_shape shape;
    Dims dims;
    StoreLayout lay;
    int device = 0, num_sms = 0;
    cudaStream_t stream = nullptr;
    std::vector<LayerState> layers;
    size_t blob_bytes = 0;
    // workspace
    void *ws_mem = nullptr;
    size_t ws_bytes = 0;
    int ws_cap = 0;
    Work ws{};
    float *x_dev = nullptr;
    // miag_moe's transfer pipeline: a copy stream and per-chunk events
    cudaStream_t copy_stream = nullptr;
    std::vector<cudaEvent_t> pipe_events;
    int transfer_chunks = 4;  // miag_set_transfer_chunks
    // pageable callers: host threads copy through a pinned staging buffer
    // (miag_set_host_copy_threads; 0 = the driver's own pageable copies)
    int host_threads = -1;  // -1: not chosen yet (min(8, cores - 1))
    std::unique_ptr<CopyPool> copy_pool;
    float *pipe_host = nullptr;
    size_t pipe_host_bytes = 0;
    int *d_err = nullptr;
    int *h_err = nullptr;  // pinned: the error word, read back with a call's results
    // expert parallelism: this rank's exchange buffer (flags | CTA counter |
    // y rows) and the peers' buffers mapped here
    uint8_t *ep_buf = nullptr;
    size_t ep_rows = 0;
    int *ep_tiles = nullptr;  // the dispatch plan's per-tile counts
    int ep_tiles_cap = 0;
    std::vector<void *> ep_peers;
    const void *ep_owner = nullptr;  // the expert-parallel block using the exchange buffer
    int last_T = 0, last_launches = 0;
    // prefill-size batches on the tcgen05 kernels (tc.cu), else on the
    // mma.sync kernels of the decode regime (gemv.cu)
    bool prefill_tc = false;
    // upload staging
    uint8_t *stage_dev = nullptr, *stage_host = nullptr;
    size_t stage_bytes = 0;
    // per-kernel profiling: event pairs recorded around each stage
    bool profiling = false;
    std::vector<cudaEvent_t> event_pool;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> prof_events[16];
    int prof_launches[16] = {};
};

namespace {
enum Stage {
    kRoute = 0, kPermute, kGateUp, kDown, kCombine, kEpPlan, kEpPack, kGather, kSwiglu, kNumStages
};
const char *const kStageNames[kNumStages] = {"route",   "permute", "gateup", "down",  "combine",
                                             "ep_plan", "ep_pack", "gather", "swiglu"};

cudaEvent_t take_event(miag_ctx *c) {
    if (!c->event_pool.empty()) {
        cudaEvent_t e = c->event_pool.back();
        c->event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Runs one stage's launches, bracketed by events while profiling.
template <class F>
void run_stage(miag_ctx *c, int st, int launches, cudaStream_t s, F launch) {
    c->last_launches += launches;
    if (!c->profiling) {
        launch();
        return;
    }
    cudaEvent_t a = take_event(c), b = take_event(c);
    cudaEventRecord(a, s);
    launch();
    cudaEventRecord(b, s);
    c->prof_events[st].push_back({a, b});
    c->prof_launches[st] += launches;
}
}  // namespace

static void set_err(char *err, size_t errlen, const char *fmt, ...) {
    if (!err || errlen == 0) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
}

#define CU(call)                                                                          \
    do {                                                                                  \
        cudaError_t e_ = (call);                                                          \
        if (e_ != cudaSuccess) {                                                          \
            set_err(err, errlen, "%s: %s", #call, cudaGetErrorString(e_));                \
            return -1;                                                                    \
        }                                                                                 \
    } while (0)

// Bytes of a .mia expert blob that hold data: gate and up at 64-byte aligned
// offsets, then down (src/storage/mia_file.c:275-278).
static size_t mia_blob_content(const miag_shape *s) {
    const size_t mat = (size_t)s->expert_hidden * (s->dim / MIAG_QK) * 36;
    const size_t off_up = round_up_sz(mat, 64);
    const size_t down = (size_t)s->dim * (s->expert_hidden / MIAG_QK) * 36;
    return 2 * off_up + down;
}

// The blob padded to the 16 KiB expert alignment (tools/internal/mia/format.go:164).
static size_t mia_blob_bytes(const miag_shape *s) {
    return round_up_sz(mia_blob_content(s), 16384);
}

extern "C" size_t miag_blob_bytes(const miag_shape *shape) {
    return shape ? mia_blob_bytes(shape) : 0;
}

static int check_shape(const miag_shape *s, char *err, size_t errlen) {
    if (!s) {
        set_err(err, errlen, "null shape");
        return -1;
    }
    if (s->dim <= 0 || s->dim % MIAG_QK || s->expert_hidden <= 0 ||
        s->expert_hidden % MIAG_QK || s->n_experts <= 0 || s->n_experts > 1024 ||
        s->n_active <= 0 || s->n_active > s->n_experts || s->n_active > 64 ||
        s->n_layers <= 0) {
        set_err(err, errlen,
                "unsupported MoE shape (dim %d, expert_hidden %d, experts %d, active %d, layers %d)",
                s->dim, s->expert_hidden, s->n_experts, s->n_active, s->n_layers);
        return -1;
    }
    return 0;
}

extern "C" int miag_open(miag_ctx **out, const miag_shape *shape, int device, char *err,
                         size_t errlen) {
    if (!out) {
        set_err(err, errlen, "null output pointer");
        return -1;
    }
    *out = nullptr;
    if (check_shape(shape, err, errlen)) return -1;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        set_err(err, errlen, "no CUDA device: libmiag has no CPU path");
        return -1;
    }
    if (device < 0 || device >= ndev) {
        set_err(err, errlen, "device %d out of range (%d devices)", device, ndev);
        return -1;
    }
    CU(cudaSetDevice(device));
    cudaDeviceProp prop;
    CU(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) {
        set_err(err, errlen, "device %d is sm_%d%d; libmiag is built for sm_100a", device,
                prop.major, prop.minor);
        return -1;
    }
    miag_ctx *c = new (std::nothrow) miag_ctx();
    if (!c) {
        set_err(err, errlen, "out of host memory");
        return -1;
    }
    c->shape = *shape;
    c->dims = Dims{shape->dim, shape->expert_hidden, shape->n_experts, shape->n_active,
                   shape->norm_topk, shape->norm_eps};
    c->lay = make_layout(shape->dim, shape->expert_hidden);
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    c->blob_bytes = mia_blob_bytes(shape);
    c->layers.resize((size_t)shape->n_layers);
    auto fail = [&](const char *what, cudaError_t e) {
        set_err(err, errlen, "%s: %s", what, cudaGetErrorString(e));
        miag_close(c);
        return -1;
    };
    cudaError_t e;
    if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess)
        return fail("cudaStreamCreate", e);
    if ((e = cudaMalloc(&c->d_err, sizeof(int))) != cudaSuccess) return fail("cudaMalloc(err)", e);
    if ((e = cudaHostAlloc(&c->h_err, sizeof(int), cudaHostAllocDefault)) != cudaSuccess)
        return fail("cudaHostAlloc(err)", e);
    // Zero-fills go on the context stream: it is non-blocking, so a plain
    // cudaMemset (legacy default stream) would not be ordered with its kernels.
    if ((e = cudaMemsetAsync(c->d_err, 0, sizeof(int), c->stream)) != cudaSuccess)
        return fail("cudaMemset", e);
    const size_t E = (size_t)shape->n_experts, d = (size_t)shape->dim;
    for (auto &L : c->layers) {
        if ((e = cudaMalloc(&L.experts, E * c->lay.expert_bytes)) != cudaSuccess)
            return fail("cudaMalloc(expert store)", e);
        if ((e = cudaMemsetAsync(L.experts, 0, E * c->lay.expert_bytes, c->stream)) != cudaSuccess)
            return fail("cudaMemset(expert store)", e);
        if ((e = cudaMalloc(&L.ffn_norm, d * 4)) != cudaSuccess) return fail("cudaMalloc", e);
        const size_t Eg = (E + 31) / 32 * 32;  // router stored in 32-expert groups
        if ((e = cudaMalloc(&L.router_t, d * Eg * 4)) != cudaSuccess) return fail("cudaMalloc", e);
        if ((e = cudaMalloc(&L.bias, E * 4)) != cudaSuccess) return fail("cudaMalloc", e);
    }
    if (gemv_setup_attributes(c->dims, c->lay) != 0) {
        set_err(err, errlen, "expert GEMV tiles do not fit in shared memory for this shape");
        miag_close(c);
        return -1;
    }
    // The tcgen05 prefill kernels are built and exact, but the mma.sync ones
    // are still faster end to end (the tensor-memory epilogue issues about
    // twice the instructions its steps need): opt in with
    // miag_set_prefill_kernel(c, MIAG_PREFILL_TCGEN05).
    c->prefill_tc = false;
    if ((e = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("zero-fill", e);
    *out = c;
    return 0;
}

extern "C" void miag_close(miag_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (auto &L : c->layers) {
        cudaFree(L.experts);
        cudaFree(L.ffn_norm);
        cudaFree(L.router_t);
        cudaFree(L.bias);
    }
    for (auto &v : c->prof_events)
        for (auto &pr : v) c->event_pool.push_back(pr.first), c->event_pool.push_back(pr.second);
    for (cudaEvent_t e : c->event_pool) cudaEventDestroy(e);
    cudaFree(c->ws_mem);
    for (void *q : c->ep_peers) cudaIpcCloseMemHandle(q);
    cudaFree(c->ep_buf);
    cudaFree(c->ep_tiles);
    cudaFree(c->d_err);
    if (c->h_err) cudaFreeHost(c->h_err);
    cudaFree(c->stage_dev);
    if (c->stage_host) cudaFreeHost(c->stage_host);
    if (c->copy_stream) {
        cudaStreamSynchronize(c->copy_stream);
        cudaStreamDestroy(c->copy_stream);
    }
    for (cudaEvent_t e : c->pipe_events) cudaEventDestroy(e);
    c->copy_pool.reset();
    if (c->pipe_host) cudaFreeHost(c->pipe_host);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

static int check_layer(miag_ctx *c, int layer, char *err, size_t errlen) {
    if (!c) {
        set_err(err, errlen, "null context");
        return -1;
    }
    if (layer < 0 || layer >= c->shape.n_layers) {
        set_err(err, errlen, "layer %d out of range (%d layers)", layer, c->shape.n_layers);
        return -1;
    }
    return 0;
}

extern "C" int miag_set_layer(miag_ctx *c, int layer, const float *ffn_norm, const float *router,
                              const float *bias, char *err, size_t errlen) {
    if (check_layer(c, layer, err, errlen)) return -1;
    if (!ffn_norm || !router) {
        set_err(err, errlen, "ffn_norm and router are required");
        return -1;
    }
    CU(cudaSetDevice(c->device));
    LayerState &L = c->layers[(size_t)layer];
    const size_t E = (size_t)c->shape.n_experts, d = (size_t)c->shape.dim;
    float *tmp = nullptr;
    CU(cudaMalloc(&tmp, E * d * 4));
    cudaError_t e = cudaMemcpyAsync(tmp, router, E * d * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) {
        launch_transpose_router(tmp, L.router_t, (int)E, (int)d, c->stream);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(L.ffn_norm, ffn_norm, d * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess && bias)
        e = cudaMemcpyAsync(L.bias, bias, E * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) {
        set_err(err, errlen, "set_layer: %s", cudaGetErrorString(e));
        return -1;
    }
    L.has_bias = bias != nullptr;
    L.dense_set = true;
    return 0;
}

static int ensure_staging(miag_ctx *c, size_t bytes, char *err, size_t errlen) {
    if (c->stage_bytes >= bytes) return 0;
    cudaFree(c->stage_dev);
    if (c->stage_host) cudaFreeHost(c->stage_host);
    c->stage_dev = nullptr, c->stage_host = nullptr, c->stage_bytes = 0;
    CU(cudaMalloc(&c->stage_dev, bytes));
    CU(cudaMallocHost(&c->stage_host, bytes));
    c->stage_bytes = bytes;
    return 0;
}

static const int kUploadBatch = 16;  // experts per staging round

extern "C" int miag_upload_experts(miag_ctx *c, int layer, int first, int n, const void *blobs,
                                   size_t stride, char *err, size_t errlen) {
    if (check_layer(c, layer, err, errlen)) return -1;
    if (!blobs || n < 0 || first < 0 || first + n > c->shape.n_experts) {
        set_err(err, errlen, "bad expert range [%d, %d)", first, first + n);
        return -1;
    }
    const size_t need = mia_blob_content(&c->shape);
    if (stride < need) {
        set_err(err, errlen, "blob stride %zu smaller than the .mia blob (%zu)", stride, need);
        return -1;
    }
    CU(cudaSetDevice(c->device));
    if (ensure_staging(c, (size_t)kUploadBatch * stride, err, errlen)) return -1;
    LayerState &L = c->layers[(size_t)layer];
    for (int e0 = 0; e0 < n; e0 += kUploadBatch) {
        const int nb = n - e0 < kUploadBatch ? n - e0 : kUploadBatch;
        const uint8_t *src = (const uint8_t *)blobs + (size_t)e0 * stride;
        memcpy(c->stage_host, src, (size_t)nb * stride);
        CU(cudaMemcpyAsync(c->stage_dev, c->stage_host, (size_t)nb * stride, cudaMemcpyHostToDevice,
                           c->stream));
        launch_repack(c->dims, c->lay, c->stage_dev, stride, nb,
                      L.experts + (size_t)(first + e0) * c->lay.expert_bytes, c->stream);
        CU(cudaGetLastError());
        CU(cudaStreamSynchronize(c->stream));
    }
    return 0;
}

extern "C" int miag_upload_experts_device(miag_ctx *c, int layer, int first, int n,
                                          const void *blobs_dev, size_t stride, void *stream,
                                          char *err, size_t errlen) {
    if (check_layer(c, layer, err, errlen)) return -1;
    if (!blobs_dev || n < 0 || first < 0 || first + n > c->shape.n_experts) {
        set_err(err, errlen, "bad expert range [%d, %d)", first, first + n);
        return -1;
    }
    if (stride < mia_blob_content(&c->shape) || (stride & 3u) || ((uintptr_t)blobs_dev & 3u)) {
        set_err(err, errlen, "blob stride %zu: at least the .mia blob (%zu), 4-byte aligned", stride,
                mia_blob_content(&c->shape));
        return -1;
    }
    if (n == 0) return 0;
    CU(cudaSetDevice(c->device));
    LayerState &L = c->layers[(size_t)layer];
    launch_repack(c->dims, c->lay, (const uint8_t *)blobs_dev, stride, n,
                  L.experts + (size_t)first * c->lay.expert_bytes,
                  stream ? (cudaStream_t)stream : c->stream);
    CU(cudaGetLastError());
    return 0;
}

extern "C" int miag_load_experts(miag_ctx *c, miag_expert_loader load, void *load_ctx, char *err,
                                 size_t errlen) {
    if (!c || !load) {
        set_err(err, errlen, "null context or loader");
        return -1;
    }
    CU(cudaSetDevice(c->device));
    const size_t stride = c->blob_bytes;
    if (ensure_staging(c, (size_t)kUploadBatch * stride, err, errlen)) return -1;
    for (int l = 0; l < c->shape.n_layers; l++) {
        LayerState &L = c->layers[(size_t)l];
        for (int e0 = 0; e0 < c->shape.n_experts; e0 += kUploadBatch) {
            const int nb = c->shape.n_experts - e0 < kUploadBatch ? c->shape.n_experts - e0
                                                                   : kUploadBatch;
            // Wait for the previous batch's copy out of the pinned buffer.
            CU(cudaStreamSynchronize(c->stream));
            int ok = 0;
            for (int k = 0; k < nb; k++) {
                if (load(load_ctx, l, e0 + k, c->stage_host + (size_t)k * stride) != 0) {
                    set_err(err, errlen, "expert loader failed for layer %d expert %d", l, e0 + k);
                    break;
                }
                ok++;
            }
            // Experts that did load in this batch are still stored.
            if (ok > 0) {
                CU(cudaMemcpyAsync(c->stage_dev, c->stage_host, (size_t)ok * stride,
                                   cudaMemcpyHostToDevice, c->stream));
                launch_repack(c->dims, c->lay, c->stage_dev, stride, ok,
                              L.experts + (size_t)e0 * c->lay.expert_bytes, c->stream);
                CU(cudaGetLastError());
            }
            if (ok < nb) {
                cudaStreamSynchronize(c->stream);
                return -1;
            }
        }
    }
    CU(cudaStreamSynchronize(c->stream));
    return 0;
}

static void *bump(uint8_t *&p, size_t bytes) {
    void *r = p;
    p += round_up_sz(bytes, 256);
    return r;
}

static size_t ws_layout(miag_ctx *c, int T, uint8_t *base, Work *w, float **x_dev) {
    const Dims &m = c->dims;
    const size_t P = (size_t)T * m.K;
    const int nchunks = (int)((P + kPermChunk - 1) / kPermChunk);
    const int xs = scale_pad(m.d / MIAG_QK);
    uint8_t *p = base;
    Work v{};
    v.T = T, v.P = (int)P, v.nchunks = nchunks;
    v.tg_count = (int32_t *)bump(p, (size_t)T * 4);  // zeroed with the workspace, kept zero by the router
    v.shares = (uint8_t *)bump(p, kShareKinds * sizeof(ShareState));  // zero at creation
    v.tc_sched = (int32_t *)bump(p, 4 * sizeof(int32_t));             // zero at creation
    v.xq = (int8_t *)bump(p, (size_t)T * m.d);
    v.dx = (float *)bump(p, (size_t)T * xs * 4);
    v.logits = (float *)bump(p, (size_t)T * m.E * 4);
    v.idx = (int32_t *)bump(p, P * 4);
    v.w = (float *)bump(p, P * 4);
    v.rank = (int32_t *)bump(p, P * 4);
    v.chunk_cnt = (int32_t *)bump(p, (size_t)nchunks * m.E * 4);
    v.chunk_base = (int32_t *)bump(p, (size_t)nchunks * m.E * 4);
    v.counts = (int32_t *)bump(p, (size_t)m.E * 4);
    v.offsets = (int32_t *)bump(p, (size_t)(m.E + 1) * 4);
    v.active = (int32_t *)bump(p, (size_t)m.E * 4);
    v.n_active = (int32_t *)bump(p, 4);
    v.chunk_pre = (int32_t *)bump(p, (size_t)(m.E + 1) * 4);
    v.chunk_info = (int4 *)bump(p, (P / kTokChunkNarrow + m.E + 1) * 16);
    v.max_chunk = (int32_t *)bump(p, 4);
    v.chunk_done = (int32_t *)bump(p, (P / kTokChunkNarrow + m.E + 1) * 4);
    v.chunk_brow = (int32_t *)bump(p, (P / kTokChunkNarrow + m.E + 1) * 4);
    if (tc_supported(m)) {  // pair tiles of the tcgen05 prefill kernels
        v.bx = (uint8_t *)bump(p, tc_tile_bytes(m, (int)P, true));
        v.bh = (uint8_t *)bump(p, tc_tile_bytes(m, (int)P, false));
    }
    v.perm = (int32_t *)bump(p, P * 4);
    v.inv = (int32_t *)bump(p, P * 4);
    v.h = (float *)bump(p, P * 2 * m.eh * 4);
    v.hq = (int8_t *)bump(p, P * m.eh);
    v.hs = (float *)bump(p, P * scale_pad(m.eh / MIAG_QK) * 4);
    v.y = (float *)bump(p, P * m.d * 4);
    float *xd = (float *)bump(p, (size_t)T * m.d * 4);
    if (w) *w = v;
    if (x_dev) *x_dev = xd;
    return (size_t)(p - base);
}

// Sizes the workspace for at least T tokens.  Buffers are laid out for the
// capacity, so buffers keep their addresses while T varies; only the counts
// change with T.
static int ensure_ws(miag_ctx *c, int T, char *err, size_t errlen) {
    if (T > c->ws_cap) {
        int cap = c->ws_cap ? c->ws_cap : 64;
        while (cap < T) cap *= 2;
        const size_t bytes = ws_layout(c, cap, nullptr, nullptr, nullptr);
        cudaStreamSynchronize(c->stream);
        cudaFree(c->ws_mem);
        c->ws_mem = nullptr, c->ws_cap = 0;
        CU(cudaMalloc(&c->ws_mem, bytes));
        // on the context stream, finished before any stream (the caller's
        // included) can use the buffers
        CU(cudaMemsetAsync(c->ws_mem, 0, bytes, c->stream));
        CU(cudaStreamSynchronize(c->stream));
        c->ws_bytes = bytes;
        c->ws_cap = cap;
    }
    ws_layout(c, c->ws_cap, (uint8_t *)c->ws_mem, &c->ws, &c->x_dev);
    const int P = T * c->dims.K;
    c->ws.T = T, c->ws.P = P, c->ws.nchunks = (P + kPermChunk - 1) / kPermChunk;
    return 0;
}

// The regime of a call over w.P pairs: prefill-size batches (more than 8
// pairs per expert on average) on the tcgen05 kernels when the context uses
// them, in chunks of 128 pairs; otherwise the mma.sync kernels.
static void set_regime(const miag_ctx *c, Work &w) {
    w.tc = (c->prefill_tc && w.bx && w.bh && w.tc_sched && wide_batch(w.P, c->dims.E)) ? 1 : 0;
    w.chunk = w.tc ? kTcChunk : tok_chunk(w.P, c->dims.E);
}

// The expert products of a call: gate/up then down, each preceded on the
// tcgen05 path by the launch that lays its activations out as pair tiles.
template <class Run>
static void launch_experts(miag_ctx *c, const LayerDev &L, const Work &w, cudaStream_t s, Run run) {
    if (w.tc) {
        run(kGather, 1, [&] { launch_tc_gather(c->dims, c->lay, w, c->num_sms, c->d_err, s); });
        run(kGateUp, 1, [&] { launch_gateup_tc(c->dims, c->lay, L, w, c->num_sms, c->d_err, s); });
        run(kSwiglu, 1, [&] { launch_tc_swiglu(c->dims, c->lay, w, c->num_sms, c->d_err, s); });
        run(kDown, 1, [&] { launch_down_tc(c->dims, c->lay, L, w, c->num_sms, c->d_err, s); });
    } else {
        run(kGateUp, 1, [&] { launch_gateup(c->dims, c->lay, L, w, c->num_sms, c->d_err, s); });
        run(kDown, down_launches(c->dims, w.P),
            [&] { launch_down(c->dims, c->lay, L, w, c->num_sms, c->d_err, s); });
    }
}

static int enqueue_moe(miag_ctx *c, int layer, float *x_dev, int T, cudaStream_t s, char *err,
                       size_t errlen) {
    const LayerState &Ls = c->layers[(size_t)layer];
    if (!Ls.dense_set) {
        set_err(err, errlen, "layer %d has no router / ffn_norm (miag_set_layer)", layer);
        return -1;
    }
    LayerDev L{Ls.ffn_norm, Ls.router_t, Ls.has_bias ? Ls.bias : nullptr, Ls.experts};
    set_regime(c, c->ws);
    const Work &w = c->ws;
    c->last_launches = 0;
    run_stage(c, kRoute, 1, s, [&] { launch_route(c->dims, L, x_dev, w, c->d_err, s); });
    run_stage(c, kPermute, permute_launches(w.P, c->dims.E), s,
              [&] { launch_permute(c->dims, w, c->d_err, s); });
    launch_experts(c, L, w, s, [&](int st, int n, auto f) { run_stage(c, st, n, s, f); });
    run_stage(c, kCombine, 1, s, [&] { launch_combine(c->dims, w, x_dev, c->d_err, s); });
    c->last_T = T;
    CU(cudaGetLastError());
    return 0;
}

extern "C" int miag_moe_async(miag_ctx *c, int layer, float *x_dev, int n_tokens, void *stream,
                              char *err, size_t errlen) {
    if (check_layer(c, layer, err, errlen)) return -1;
    if (n_tokens < 0 || (n_tokens > 0 && !x_dev) || ((uintptr_t)x_dev & 15u)) {
        set_err(err, errlen, "bad token buffer (device pointer, 16-byte aligned)");
        return -1;
    }
    if (n_tokens == 0) {
        c->last_launches = 0;
        return 0;
    }
    CU(cudaSetDevice(c->device));
    if (ensure_ws(c, n_tokens, err, errlen)) return -1;
    return enqueue_moe(c, layer, x_dev, n_tokens, stream ? (cudaStream_t)stream : c->stream, err,
                       errlen);
}

// The error word, as a call that has just synchronised its stream left it:
// `code` when the caller already copied the word back with its results
// (pinned h_err, same stream), else read now.
static int read_device_error(miag_ctx *c, char *err, size_t errlen, int code = -1) {
    if (code < 0) CU(cudaMemcpy(&code, c->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (code == 0) return 0;
    CU(cudaMemsetAsync(c->d_err, 0, sizeof(int), c->stream));
    // A call cut short may have left counters that every call expects at
    // zero (the router's token-group counters, the SM-share claims): clear
    // them, in the workspace and in the no-allocation array of this device.
    if (c->ws_mem) {
        CU(cudaMemsetAsync(c->ws.tg_count, 0, (size_t)c->ws_cap * sizeof(int32_t), c->stream));
        CU(cudaMemsetAsync(c->ws.shares, 0, kShareKinds * sizeof(ShareState), c->stream));
        CU(cudaMemsetAsync(c->ws.tc_sched, 0, 4 * sizeof(int32_t), c->stream));
    }
    noalloc_clear_counters(c->device, c->stream);
    CU(cudaStreamSynchronize(c->stream));
    const char *what = code == kErrWaitFull    ? "a consumer timed out waiting for a staged tile"
                       : code == kErrWaitEmpty ? "the producer timed out waiting for a free stage"
                       : code == kErrBadExpert ? "a routing index was out of range"
                       : code == kErrItemList  ? "an expert launch's work list named a tile outside the store"
                       : code == kErrWaitPeer  ? "timed out waiting for another rank's expert results"
                                               : "unknown device error";
    set_err(err, errlen, "device error %d: %s", code, what);
    return -1;
}

// One thread waits, bounded, on an mbarrier that nothing arrives on: the
// same wait and error path the block's kernels take when a staged tile
// never lands, run on purpose.  No copy is in flight and the barrier lives
// in the CTA's own shared memory, so giving up leaves nothing behind.
static __global__ void k_wait_selftest(int *err, long long limit) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        if (!mbar_wait_for(&bar, 0, limit)) set_error(err, kErrWaitFull);
    }
}

extern "C" int miag_selftest_wait_timeout(miag_ctx *c, int timeout_us, char *err, size_t errlen) {
    if (!c || timeout_us <= 0 || timeout_us > 100000) {
        set_err(err, errlen, "miag_selftest_wait_timeout: null context or timeout outside 1..100000 us");
        return -1;
    }
    CU(cudaSetDevice(c->device));
    int khz = 0;
    CU(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, c->device));
    const long long limit = (long long)timeout_us * (khz / 1000);
    k_wait_selftest<<<1, 32, 0, c->stream>>>(c->d_err, limit);
    CU(cudaGetLastError());
    CU(cudaStreamSynchronize(c->stream));
    return read_device_error(c, err, errlen);
}

extern "C" int miag_sync(miag_ctx *c, void *stream, char *err, size_t errlen) {
    if (!c) {
        set_err(err, errlen, "null context");
        return -1;
    }
    CU(cudaSetDevice(c->device));
    CU(cudaStreamSynchronize(stream ? (cudaStream_t)stream : c->stream));
    return read_device_error(c, err, errlen);
}

// Batches of at least kPipeMin tokens move through miag_moe in
// transfer_chunks pieces (miag_set_transfer_chunks): the copy stream brings
// piece k + 1 in and takes piece k - 1 out while the block runs on piece k.
// Tokens are independent in the block (forward.c:167-197 is a per-token
// loop), so the results are those of one call over all of them, bit for bit.
// Pieces are enqueued in the order in(0), block(0), in(1), block(1), ... and
// the copies out last.
//
// A pageable caller buffer (the reference's m->x is malloc'd) goes through a
// pinned staging buffer in slices of about 2 MiB: host threads copy slice
// i + 1 into it while slice i crosses PCIe, and each piece's block waits for
// its last slice.  Results come back the same way: the host copies a slice
// out as soon as its device-to-host copy has landed.  A slice's staging
// region holds its inputs and then its results; the results are copied in
// only after the block, which follows the inputs' copy out of the region.
constexpr int kPipeMin = 2048, kPipeMaxChunks = 16;
constexpr size_t kStageMin = (size_t)1 << 20;    // smaller pageable buffers: the driver's copies
constexpr size_t kStageMax = (size_t)1 << 30;    // larger ones too (no staging buffer that big)
constexpr size_t kStageSlice = (size_t)2 << 20;  // bytes per staged slice

static bool host_pageable(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return true;
    }
    return a.type == cudaMemoryTypeUnregistered;
}

// The copy threads and a pinned staging buffer of `bytes`; false when either
// cannot be had, and the call then leaves its copies to the CUDA runtime.
static bool ensure_host_staging(miag_ctx *c, size_t bytes) {
    if (!c->copy_pool) {
        if (c->host_threads < 0) {
            const int cores = (int)std::thread::hardware_concurrency();
            c->host_threads = std::max(1, std::min(8, cores - 1));
        }
        try {
            c->copy_pool.reset(new CopyPool(c->host_threads - 1));
        } catch (...) {  // no threads to be had
            return false;
        }
    }
    if (c->pipe_host_bytes >= bytes) return true;
    if (c->pipe_host) cudaFreeHost(c->pipe_host);
    c->pipe_host = nullptr;
    c->pipe_host_bytes = 0;
    if (cudaHostAlloc((void **)&c->pipe_host, bytes, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        c->pipe_host = nullptr;
        return false;
    }
    c->pipe_host_bytes = bytes;
    return true;
}

static int moe_pipelined(miag_ctx *c, int layer, float *x, int n_tokens, int chunks, bool staged,
                         char *err, size_t errlen) {
    if (!c->copy_stream) {
        CU(cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking));
        for (int i = 0; i < 2 * kPipeMaxChunks; i++) {
            cudaEvent_t e;
            CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
            c->pipe_events.push_back(e);
        }
    }
    const size_t dim = (size_t)c->shape.dim, row = dim * sizeof(float);
    if (staged && !ensure_host_staging(c, (size_t)n_tokens * row)) staged = false;
    float *const src = staged ? c->pipe_host : x;  // what the copy engines read and write
    const std::vector<int> bound = piece_bounds(n_tokens, chunks);
    const int n_chunks = (int)bound.size() - 1;  // piece k: tokens [bound[k], bound[k + 1])
    // tokens per transfer: a slice of the staging buffer, or the whole piece
    const int slice = staged ? (int)std::max<size_t>(1, kStageSlice / row) : n_tokens;
    int n_slices = 0;
    for (int k = 0; k < n_chunks; k++) n_slices += (bound[k + 1] - bound[k] + slice - 1) / slice;
    while ((int)c->pipe_events.size() < 2 * kPipeMaxChunks + n_slices) {
        cudaEvent_t e;
        CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        c->pipe_events.push_back(e);
    }
    cudaEvent_t *const ev_in = c->pipe_events.data(), *const ev_block = ev_in + kPipeMaxChunks,
                       *const ev_out = ev_block + kPipeMaxChunks;
    int launches = 0;
    auto enqueue = [&]() -> int {
        for (int k = 0; k < n_chunks; k++) {
            const int t0 = bound[k], tk = bound[k + 1] - t0;
            for (int s0 = t0; s0 < t0 + tk; s0 += slice) {
                const size_t bytes = (size_t)std::min(slice, t0 + tk - s0) * row;
                if (staged) c->copy_pool->copy(src + s0 * dim, x + s0 * dim, bytes);
                CU(cudaMemcpyAsync(c->x_dev + s0 * dim, src + s0 * dim, bytes, cudaMemcpyHostToDevice,
                                   c->copy_stream));
            }
            CU(cudaEventRecord(ev_in[k], c->copy_stream));
            CU(cudaStreamWaitEvent(c->stream, ev_in[k], 0));
            if (ensure_ws(c, tk, err, errlen)) return -1;  // counts only: the buffers hold n_tokens
            if (enqueue_moe(c, layer, c->x_dev + t0 * dim, tk, c->stream, err, errlen)) return -1;
            launches += c->last_launches;
            CU(cudaEventRecord(ev_block[k], c->stream));
        }
        int j = 0;
        for (int k = 0; k < n_chunks; k++) {
            const int t0 = bound[k], tk = bound[k + 1] - t0;
            CU(cudaStreamWaitEvent(c->copy_stream, ev_block[k], 0));
            for (int s0 = t0; s0 < t0 + tk; s0 += slice) {
                CU(cudaMemcpyAsync(src + s0 * dim, c->x_dev + s0 * dim,
                                   (size_t)std::min(slice, t0 + tk - s0) * row, cudaMemcpyDeviceToHost,
                                   c->copy_stream));
                CU(cudaEventRecord(ev_out[j++], c->copy_stream));
            }
        }
        // after the last piece's block: the error word with the results
        CU(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, c->copy_stream));
        if (staged) {
            j = 0;
            for (int k = 0; k < n_chunks; k++) {
                const int t0 = bound[k], t1 = bound[k + 1];
                for (int s0 = t0; s0 < t1; s0 += slice) {
                    CU(cudaEventSynchronize(ev_out[j++]));
                    c->copy_pool->copy(x + s0 * dim, src + s0 * dim, (size_t)std::min(slice, t1 - s0) * row);
                }
            }
        }
        return 0;
    };
    if (enqueue() != 0) {
        // no copy enqueued may still land once the call has returned
        cudaStreamSynchronize(c->copy_stream);
        cudaStreamSynchronize(c->stream);
        return -1;
    }
    CU(cudaStreamSynchronize(c->copy_stream));
    c->last_launches = launches;
    return read_device_error(c, err, errlen, *c->h_err);
}

extern "C" int miag_moe(miag_ctx *c, int layer, float *x, int n_tokens, char *err, size_t errlen) {
    if (check_layer(c, layer, err, errlen)) return -1;
    if (n_tokens < 0 || (n_tokens > 0 && !x)) {
        set_err(err, errlen, "bad token buffer");
        return -1;
    }
    if (n_tokens == 0) {
        c->last_launches = 0;
        return 0;
    }
    CU(cudaSetDevice(c->device));
    if (ensure_ws(c, n_tokens, err, errlen)) return -1;
    const size_t bytes = (size_t)n_tokens * c->shape.dim * sizeof(float);
    const bool staged =
        c->host_threads != 0 && bytes >= kStageMin && bytes <= kStageMax && host_pageable(x);
    const int chunks = n_tokens >= kPipeMin ? c->transfer_chunks : 1;
    if (staged || chunks > 1) return moe_pipelined(c, layer, x, n_tokens, chunks, staged, err, errlen);
    CU(cudaMemcpyAsync(c->x_dev, x, bytes, cudaMemcpyHostToDevice, c->stream));
    if (enqueue_moe(c, layer, c->x_dev, n_tokens, c->stream, err, errlen)) return -1;
    CU(cudaMemcpyAsync(x, c->x_dev, bytes, cudaMemcpyDeviceToHost, c->stream));
    CU(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));  // one wait for the results and the error word
    return read_device_error(c, err, errlen, *c->h_err);
}

// ---- The block in three device steps, for callers that move pairs between
// GPUs in between (expert parallelism): route here, experts where they live,
// combine back here.

extern "C" int miag_route_async(miag_ctx *c, int layer, const float *x_dev, int n_tokens,
                                int32_t *idx, float *wts, int8_t *xq, float *dx, void *stream,
                                char *err, size_t errlen) {
    if (check_layer(c, layer, err, errlen)) return -1;
    if (n_tokens < 0 || (n_tokens > 0 && (!x_dev || !idx || !wts || !xq || !dx)) ||
        ((uintptr_t)x_dev & 15u) || ((uintptr_t)xq & 15u) || ((uintptr_t)dx & 15u)) {
        set_err(err, errlen, "bad buffers (device pointers; x, xq, dx 16-byte aligned)");
        return -1;
    }
    const LayerState &Ls = c->layers[(size_t)layer];
    if (!Ls.dense_set) {
        set_err(err, errlen, "layer %d has no router / ffn_norm (miag_set_layer)", layer);
        return -1;
    }
    c->last_launches = 0;
    if (n_tokens == 0) return 0;
    CU(cudaSetDevice(c->device));
    if (ensure_ws(c, n_tokens, err, errlen)) return -1;
    const cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    const LayerDev L{Ls.ffn_norm, Ls.router_t, Ls.has_bias ? Ls.bias : nullptr, Ls.experts};
    Work w = c->ws;  // logits and the token-group counters stay in the workspace
    w.idx = idx, w.w = wts, w.xq = xq, w.dx = dx;
    run_stage(c, kRoute, 1, s, [&] { launch_route(c->dims, L, x_dev, w, c->d_err, s); });
    CU(cudaGetLastError());
    return 0;
}

extern "C" int miag_experts_async(miag_ctx *c, int layer, const int8_t *xq, const float *dx,
                                  int n_rows, const int32_t *pair_row, const int32_t *pair_expert,
                                  int n_pairs, float *y, void *stream, char *err, size_t errlen) {
    if (check_layer(c, layer, err, errlen)) return -1;
    if (n_pairs < 0 || n_rows < 0 ||
        (n_pairs > 0 && (!xq || !dx || !pair_row || !pair_expert || !y || n_rows == 0)) ||
        ((uintptr_t)xq & 15u) || ((uintptr_t)dx & 15u)) {
        set_err(err, errlen, "bad buffers (device pointers; xq, dx 16-byte aligned)");
        return -1;
    }
    c->last_launches = 0;
    if (n_pairs == 0) return 0;
    CU(cudaSetDevice(c->device));
    // the workspace is laid out by tokens; size it for n_pairs pairs
    if (ensure_ws(c, (n_pairs + c->dims.K - 1) / c->dims.K, err, errlen)) return -1;
    const cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    const LayerState &Ls = c->layers[(size_t)layer];
    const LayerDev L{Ls.ffn_norm, Ls.router_t, Ls.has_bias ? Ls.bias : nullptr, Ls.experts};
    Work w = c->ws;
    w.P = n_pairs, w.nchunks = (n_pairs + kPermChunk - 1) / kPermChunk;
    w.idx = const_cast<int32_t *>(pair_expert);  // read only by the permutation
    w.xq = const_cast<int8_t *>(xq), w.dx = const_cast<float *>(dx);
    w.pair_row = pair_row, w.n_rows = n_rows, w.y = y;
    set_regime(c, w);
    run_stage(c, kPermute, permute_launches(w.P, c->dims.E), s,
              [&] { launch_permute(c->dims, w, c->d_err, s); });
    launch_experts(c, L, w, s, [&](int st, int n, auto f) { run_stage(c, st, n, s, f); });
    CU(cudaGetLastError());
    return 0;
}

// ---- Expert parallelism over peer memory: down stores each y row at the
// pair's origin rank, and a flag per rank says when all of them have landed.

namespace {
constexpr size_t kEpFlagsOff = 0, kEpDoneOff = 64, kEpRowsOff = 256;
}

extern "C" int miag_ep_buffer(miag_ctx *c, size_t y_rows, void **y_dev, unsigned **flags_dev,
                              void *ipc_handle, char *err, size_t errlen) {
    if (!c || !y_dev || !flags_dev || !ipc_handle) {
        set_err(err, errlen, "null argument");
        return -1;
    }
    CU(cudaSetDevice(c->device));
    if (!c->ep_buf || y_rows > c->ep_rows) {
        CU(cudaStreamSynchronize(c->stream));
        cudaFree(c->ep_buf);
        c->ep_buf = nullptr, c->ep_rows = 0;
        const size_t bytes = kEpRowsOff + y_rows * (size_t)c->dims.d * sizeof(float);
        CU(cudaMalloc(&c->ep_buf, bytes));
        CU(cudaMemset(c->ep_buf, 0, kEpRowsOff));  // flags and counter start at zero
        CU(cudaDeviceSynchronize());
        c->ep_rows = y_rows;
    }
    cudaIpcMemHandle_t h;
    CU(cudaIpcGetMemHandle(&h, c->ep_buf));
    memcpy(ipc_handle, &h, sizeof h);
    *y_dev = c->ep_buf + kEpRowsOff;
    *flags_dev = reinterpret_cast<unsigned *>(c->ep_buf + kEpFlagsOff);
    return 0;
}

extern "C" int miag_ep_open_peer(miag_ctx *c, const void *ipc_handle, void **y_dev,
                                 unsigned **flags_dev, char *err, size_t errlen) {
    if (!c || !ipc_handle || !y_dev || !flags_dev) {
        set_err(err, errlen, "null argument");
        return -1;
    }
    CU(cudaSetDevice(c->device));
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof h);
    void *q = nullptr;
    CU(cudaIpcOpenMemHandle(&q, h, cudaIpcMemLazyEnablePeerAccess));
    c->ep_peers.push_back(q);
    *y_dev = static_cast<uint8_t *>(q) + kEpRowsOff;
    *flags_dev = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(q) + kEpFlagsOff);
    return 0;
}

extern "C" int miag_ep_close_peers(miag_ctx *c, char *err, size_t errlen) {
    if (!c) {
        set_err(err, errlen, "null context");
        return -1;
    }
    CU(cudaSetDevice(c->device));
    CU(cudaStreamSynchronize(c->stream));
    for (void *q : c->ep_peers) CU(cudaIpcCloseMemHandle(q));
    c->ep_peers.clear();
    return 0;
}

namespace miag {
// miag_experts_to_ranks_async with the activation rows at any stride (the
// expert-parallel block of ep_comm.cu reads them straight from the received
// records: values then scales, one record a row).
int ctx_experts_to_ranks(miag_ctx *c, int layer, const int8_t *xq, size_t x_stride,
                         const float *dx, size_t dx_stride, int n_rows, const int32_t *pair_row,
                         const int32_t *pair_expert, int n_pairs, int n_ranks, int rank,
                         const int32_t *src_end, float *const *dst, unsigned *const *flags,
                         unsigned seq, cudaStream_t s, char *err, size_t errlen) {
    if (check_layer(c, layer, err, errlen)) return -1;
    if (n_ranks < 1 || n_ranks > kEpMaxRanks || rank < 0 || rank >= n_ranks || !src_end || !dst ||
        !flags || !c->ep_buf) {
        set_err(err, errlen, "bad ranks or routes (1..%d ranks; miag_ep_buffer first)", kEpMaxRanks);
        return -1;
    }
    if (n_pairs < 0 || n_rows < 0 ||
        (n_pairs > 0 && (!xq || !dx || !pair_row || !pair_expert || n_rows == 0)) ||
        ((uintptr_t)xq & 15u) || ((uintptr_t)dx & 15u) || (x_stride & 15u) || (dx_stride & 3u)) {
        set_err(err, errlen, "bad buffers (device pointers; xq, dx and row strides 16-byte aligned)");
        return -1;
    }
    YRoute yr{};
    yr.n = n_ranks, yr.me = rank, yr.seq = seq;
    yr.done = reinterpret_cast<unsigned *>(c->ep_buf + kEpDoneOff);
    int prev = 0;
    for (int r = 0; r < n_ranks; r++) {
        if (src_end[r] < prev || !flags[r] || (src_end[r] > prev && !dst[r])) {
            set_err(err, errlen, "rank %d: bad pair range or destination", r);
            return -1;
        }
        yr.end[r] = prev = src_end[r], yr.dst[r] = dst[r], yr.flags[r] = flags[r];
    }
    if (prev != n_pairs) {
        set_err(err, errlen, "the ranks' pair ranges cover %d pairs, not %d", prev, n_pairs);
        return -1;
    }
    c->last_launches = 0;
    CU(cudaSetDevice(c->device));
    if (n_pairs == 0) {  // nothing to compute: the other ranks still wait for this one
        launch_ep_signal(yr, s);
        c->last_launches = 1;
        CU(cudaGetLastError());
        return 0;
    }
    if (ensure_ws(c, (n_pairs + c->dims.K - 1) / c->dims.K, err, errlen)) return -1;
    const LayerState &Ls = c->layers[(size_t)layer];
    const LayerDev L{Ls.ffn_norm, Ls.router_t, Ls.has_bias ? Ls.bias : nullptr, Ls.experts};
    Work w = c->ws;
    w.P = n_pairs, w.nchunks = (n_pairs + kPermChunk - 1) / kPermChunk;
    w.idx = const_cast<int32_t *>(pair_expert);
    w.xq = const_cast<int8_t *>(xq), w.dx = const_cast<float *>(dx);
    w.x_stride = x_stride, w.dx_stride = dx_stride / sizeof(float);
    w.pair_row = pair_row, w.n_rows = n_rows, w.y = nullptr, w.yr = yr;
    set_regime(c, w);
    run_stage(c, kPermute, permute_launches(w.P, c->dims.E), s,
              [&] { launch_permute(c->dims, w, c->d_err, s); });
    launch_experts(c, L, w, s, [&](int st, int n, auto f) { run_stage(c, st, n, s, f); });
    CU(cudaGetLastError());
    return 0;
}

// The exchange buffer of a context belongs to at most one expert-parallel
// block (ep_comm.cu) at a time: its sequence numbers and peer mappings
// would otherwise interleave.
bool ctx_claim_ep(miag_ctx *c, const void *owner) {
    if (c->ep_owner && c->ep_owner != owner) return false;
    c->ep_owner = owner;
    return true;
}
void ctx_release_ep(miag_ctx *c, const void *owner) {
    if (c->ep_owner == owner) c->ep_owner = nullptr;
}
int ctx_device(const miag_ctx *c) { return c->device; }
const miag_shape *ctx_shape(const miag_ctx *c) { return &c->shape; }
cudaStream_t ctx_stream(const miag_ctx *c) { return c->stream; }
int ctx_num_sms(const miag_ctx *c) { return c->num_sms; }

// Sizes the workspace for batches of up to T tokens now, so that later
// calls of at most T tokens neither allocate nor synchronise (a captured
// launch sequence needs that).  The returned address changes whenever the
// workspace is re-allocated, which invalidates captured sequences.
const void *ctx_reserve(miag_ctx *c, int T, char *err, size_t errlen) {
    if (cudaSetDevice(c->device) != cudaSuccess) {
        set_err(err, errlen, "cudaSetDevice failed");
        return nullptr;
    }
    if (ensure_ws(c, T, err, errlen)) return nullptr;
    return c->ws_mem;
}
const void *ctx_workspace(const miag_ctx *c) { return c->ws_mem; }

// miag_set_layer from device memory (no bias): ffn_norm [d] and router
// [E][d] f32 may be freed once the stream has passed this point.
int ctx_set_layer_device(miag_ctx *c, int layer, const float *ffn_norm, const float *router,
                         cudaStream_t s, char *err, size_t errlen) {
    if (check_layer(c, layer, err, errlen)) return -1;
    CU(cudaSetDevice(c->device));
    LayerState &L = c->layers[(size_t)layer];
    const size_t E = (size_t)c->shape.n_experts, d = (size_t)c->shape.dim;
    launch_transpose_router(router, L.router_t, (int)E, (int)d, s);
    CU(cudaGetLastError());
    CU(cudaMemcpyAsync(L.ffn_norm, ffn_norm, d * 4, cudaMemcpyDeviceToDevice, s));
    L.has_bias = false;
    L.dense_set = true;
    return 0;
}
}  // namespace miag

extern "C" int miag_experts_to_ranks_async(miag_ctx *c, int layer, const int8_t *xq,
                                           const float *dx, int n_rows, const int32_t *pair_row,
                                           const int32_t *pair_expert, int n_pairs, int n_ranks,
                                           int rank, const int32_t *src_end, float *const *dst,
                                           unsigned *const *flags, unsigned seq, void *stream,
                                           char *err, size_t errlen) {
    if (!c) {
        set_err(err, errlen, "null context");
        return -1;
    }
    return ctx_experts_to_ranks(c, layer, xq, (size_t)c->dims.d, dx,
                                (size_t)scale_pad(c->dims.d / MIAG_QK) * sizeof(float), n_rows,
                                pair_row, pair_expert, n_pairs, n_ranks, rank, src_end, dst, flags,
                                seq, stream ? (cudaStream_t)stream : c->stream, err, errlen);
}

extern "C" int miag_ep_wait_async(miag_ctx *c, const unsigned *flags, int n_ranks, unsigned seq,
                                  void *stream, char *err, size_t errlen) {
    if (!c || !flags || n_ranks < 1 || n_ranks > kEpMaxRanks) {
        set_err(err, errlen, "bad flags or ranks (1..%d)", kEpMaxRanks);
        return -1;
    }
    CU(cudaSetDevice(c->device));
    const cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    launch_ep_wait(flags, n_ranks, seq, 2000000000LL, c->d_err, s);  // gives up after 2 s
    c->last_launches = 1;
    CU(cudaGetLastError());
    return 0;
}

extern "C" int miag_dx_stride(const miag_shape *s) {
    return s ? scale_pad(s->dim / MIAG_QK) : 0;
}

extern "C" int miag_combine_async(miag_ctx *c, float *x_dev, int n_tokens, const float *wts,
                                  const float *y, const int32_t *y_pos, void *stream, char *err,
                                  size_t errlen) {
    if (!c) {
        set_err(err, errlen, "null context");
        return -1;
    }
    if (n_tokens < 0 || (n_tokens > 0 && (!x_dev || !wts || !y)) || ((uintptr_t)x_dev & 15u) ||
        ((uintptr_t)y & 15u)) {
        set_err(err, errlen, "bad buffers (device pointers; x and y 16-byte aligned)");
        return -1;
    }
    c->last_launches = 0;
    if (n_tokens == 0) return 0;
    CU(cudaSetDevice(c->device));
    const cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    Work w{};
    w.T = n_tokens, w.w = const_cast<float *>(wts), w.y = const_cast<float *>(y), w.y_pos = y_pos;
    run_stage(c, kCombine, 1, s, [&] { launch_combine(c->dims, w, x_dev, c->d_err, s); });
    CU(cudaGetLastError());
    return 0;
}

extern "C" int miag_ep_plan_async(miag_ctx *c, const int32_t *idx, int n_tokens, int n_ranks,
                                  int experts_per_rank, int strided, int64_t *counts,
                                  int32_t *send_rows, int32_t *pair_meta, int32_t *y_pos,
                                  void *stream, char *err, size_t errlen) {
    if (!c) {
        set_err(err, errlen, "null context");
        return -1;
    }
    if (n_ranks < 1 || n_ranks > kEpMaxRanks || experts_per_rank < 1 ||
        (long)n_ranks * experts_per_rank != c->dims.E) {
        set_err(err, errlen, "%d ranks x %d experts: need 1..%d ranks holding all %d experts",
                n_ranks, experts_per_rank, kEpMaxRanks, c->dims.E);
        return -1;
    }
    if (c->dims.K > 32) {  // the plan's per-tile pair prefixes are 16-bit fields
        set_err(err, errlen, "expert parallelism supports at most 32 active experts");
        return -1;
    }
    if (n_tokens < 0 || !counts || (n_tokens > 0 && (!idx || !send_rows || !pair_meta || !y_pos)) ||
        ((uintptr_t)pair_meta & 7u)) {
        set_err(err, errlen, "bad buffers (device pointers; pair_meta 8-byte aligned)");
        return -1;
    }
    c->last_launches = 0;
    CU(cudaSetDevice(c->device));
    const cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    const int n_tiles = std::max(1, ep_plan_tiles(n_tokens));
    if (n_tiles > c->ep_tiles_cap) {
        CU(cudaStreamSynchronize(s));  // an earlier plan may still read the old counts
        cudaFree(c->ep_tiles);
        c->ep_tiles = nullptr, c->ep_tiles_cap = 0;
        CU(cudaMalloc(&c->ep_tiles, (size_t)n_tiles * 2 * kEpMaxRanks * sizeof(int)));
        c->ep_tiles_cap = n_tiles;
    }
    run_stage(c, kEpPlan, 2, s, [&] {
        launch_ep_plan(idx, n_tokens, c->dims.K, n_ranks, experts_per_rank, strided != 0,
                       c->ep_tiles, reinterpret_cast<long long *>(counts), send_rows, pair_meta,
                       y_pos, c->d_err, s);
    });
    CU(cudaGetLastError());
    return 0;
}

extern "C" int miag_ep_pack_async(miag_ctx *c, const int8_t *xq, const float *dx,
                                  const int32_t *send_rows, int n_rows, const int32_t *pair_meta,
                                  int n_pairs, const int64_t *all_counts, int rank, int n_ranks,
                                  uint8_t *rec, int32_t *meta_out, void *stream, char *err,
                                  size_t errlen) {
    if (!c) {
        set_err(err, errlen, "null context");
        return -1;
    }
    if (n_ranks < 1 || n_ranks > kEpMaxRanks || rank < 0 || rank >= n_ranks) {
        set_err(err, errlen, "rank %d of %d: need 1..%d ranks", rank, n_ranks, kEpMaxRanks);
        return -1;
    }
    if (n_rows < 0 || n_pairs < 0 || (n_rows > 0 && (!xq || !dx || !send_rows || !rec)) ||
        (n_pairs > 0 && (!pair_meta || !meta_out || !all_counts)) || ((uintptr_t)xq & 15u) ||
        ((uintptr_t)dx & 15u) || ((uintptr_t)rec & 15u) || ((uintptr_t)pair_meta & 7u) ||
        ((uintptr_t)meta_out & 7u)) {
        set_err(err, errlen,
                "bad buffers (device pointers; xq, dx, rec 16-byte and pair records 8-byte aligned)");
        return -1;
    }
    c->last_launches = 0;
    if (n_rows == 0 && n_pairs == 0) return 0;
    CU(cudaSetDevice(c->device));
    const cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    run_stage(c, kEpPack, 1, s, [&] {
        launch_ep_pack(xq, dx, c->dims.d, scale_pad(c->dims.d / MIAG_QK), send_rows, n_rows,
                       pair_meta, n_pairs, reinterpret_cast<const long long *>(all_counts), rank,
                       n_ranks, rec, meta_out, c->num_sms, s);
    });
    CU(cudaGetLastError());
    return 0;
}

extern "C" int miag_routing(miag_ctx *c, int32_t *idx, float *w, int32_t *counts, int32_t *offsets,
                            int32_t *perm, char *err, size_t errlen) {
    if (!c) {
        set_err(err, errlen, "null context");
        return -1;
    }
    CU(cudaSetDevice(c->device));
    CU(cudaStreamSynchronize(c->stream));
    const size_t P = (size_t)c->last_T * c->dims.K, E = (size_t)c->dims.E;
    if (idx) CU(cudaMemcpy(idx, c->ws.idx, P * 4, cudaMemcpyDeviceToHost));
    if (w) CU(cudaMemcpy(w, c->ws.w, P * 4, cudaMemcpyDeviceToHost));
    if (counts) CU(cudaMemcpy(counts, c->ws.counts, E * 4, cudaMemcpyDeviceToHost));
    if (offsets) CU(cudaMemcpy(offsets, c->ws.offsets, (E + 1) * 4, cudaMemcpyDeviceToHost));
    if (perm) CU(cudaMemcpy(perm, c->ws.perm, P * 4, cudaMemcpyDeviceToHost));
    return 0;
}

extern "C" int miag_router_logits(miag_ctx *c, float *logits, char *err, size_t errlen) {
    if (!c || !logits) {
        set_err(err, errlen, "null argument");
        return -1;
    }
    CU(cudaSetDevice(c->device));
    CU(cudaStreamSynchronize(c->stream));
    CU(cudaMemcpy(logits, c->ws.logits, (size_t)c->last_T * c->dims.E * 4,
                  cudaMemcpyDeviceToHost));
    return 0;
}

extern "C" int miag_last_launch_count(const miag_ctx *c) { return c ? c->last_launches : 0; }

extern "C" int miag_set_prefill_kernel(miag_ctx *c, int kind, char *err, size_t errlen) {
    if (!c || (kind != MIAG_PREFILL_MMA && kind != MIAG_PREFILL_TCGEN05)) {
        set_err(err, errlen, "null context or unknown prefill kernel %d", kind);
        return -1;
    }
    if (kind == MIAG_PREFILL_TCGEN05) {
        CU(cudaSetDevice(c->device));
        if (!tc_supported(c->dims) || tc_setup_attributes() != 0) {
            set_err(err, errlen, "the tcgen05 prefill kernels do not take this shape (dim and "
                                 "expert_hidden must be multiples of 256)");
            return -1;
        }
    }
    CU(cudaStreamSynchronize(c->stream));
    c->prefill_tc = kind == MIAG_PREFILL_TCGEN05;
    return 0;
}

extern "C" int miag_set_transfer_chunks(miag_ctx *c, int chunks) {
    if (!c || chunks < 1 || chunks > kPipeMaxChunks) return -1;
    c->transfer_chunks = chunks;
    return 0;
}

extern "C" int miag_set_host_copy_threads(miag_ctx *c, int threads) {
    if (!c || threads < 0 || threads > 64) return -1;
    if (threads != c->host_threads) c->copy_pool.reset();  // the next staged call makes the pool
    c->host_threads = threads;
    return 0;
}

extern "C" int miag_prefill_kernel(const miag_ctx *c) {
    return c && c->prefill_tc ? MIAG_PREFILL_TCGEN05 : MIAG_PREFILL_MMA;
}

extern "C" int miag_profile(miag_ctx *c, int enable) {
    if (!c) return -1;
    c->profiling = enable != 0;
    return 0;
}

extern "C" int miag_profile_stages(void) { return kNumStages; }

extern "C" const char *miag_profile_stage_name(int i) {
    return i >= 0 && i < kNumStages ? kStageNames[i] : nullptr;
}

extern "C" int miag_profile_read(miag_ctx *c, double *ms, int32_t *launches, char *err,
                                 size_t errlen) {
    if (!c) {
        set_err(err, errlen, "null context");
        return -1;
    }
    CU(cudaSetDevice(c->device));
    for (int st = 0; st < kNumStages; st++) {
        double total = 0.0;
        for (auto &pr : c->prof_events[st]) {
            CU(cudaEventSynchronize(pr.second));
            float t = 0.0f;
            CU(cudaEventElapsedTime(&t, pr.first, pr.second));
            total += t;
            c->event_pool.push_back(pr.first);
            c->event_pool.push_back(pr.second);
        }
        c->prof_events[st].clear();
        if (ms) ms[st] = total;
        if (launches) launches[st] = c->prof_launches[st];
        c->prof_launches[st] = 0;
    }
    return 0;
}

// Read-only view of a context's layer for other launch sequences (noalloc.cu).
namespace miag {
int ctx_view(const miag_ctx *c, int layer, CtxView *v) {
    if (!c || layer < 0 || layer >= c->shape.n_layers) return -1;
    const LayerState &Ls = c->layers[(size_t)layer];
    if (!Ls.dense_set) return -1;
    v->device = c->device;
    v->num_sms = c->num_sms;
    v->stream = c->stream;
    v->dims = c->dims;
    v->lay = c->lay;
    v->layer = LayerDev{Ls.ffn_norm, Ls.router_t, Ls.has_bias ? Ls.bias : nullptr, Ls.experts};
    v->d_err = c->d_err;
    return 0;
}
}  // namespace miag
