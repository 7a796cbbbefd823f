// ep_comm.cu -- the expert-parallel MoE block behind the C ABI: the ranks of
// an NCCL communicator (one GPU each, one node) each hold E / N experts and
// their own tokens, and miag_moe_ep_async runs the whole sharded block from
// C++ with no other runtime in the data path.
//
// The reference runs moe() (src/model/forward.c:167-197) on one device;
// sharding changes no arithmetic: every rank routes its own tokens
// (forward.c:174-181), each (token, expert) pair's expert products run
// where the expert lives (forward.c:186-193), and the results come back one
// f32 row per pair to be combined in top-k order (forward.c:194), so the
// outputs equal miag_moe's bit for bit.  One step:
//
//   1. route (the token rows' top-k, weights and Q8_0 form);
//   2. plan: per destination rank, the rows (once per token and rank) and
//      the (row, expert) pairs to send, and where each pair's result comes
//      back (ep.cu);
//   3. all-gather of the [src][dst] counts, read on the host: the single host
//      synchronisation of a step, since the sizes of what follows depend on it;
//   4. pack the send records (a row's int8 values then its f32 block scales)
//      and the pair records renumbered in the receiver's buffer (ep.cu);
//   5. one NCCL group of send/recv pairs carries rows and pair records;
//   6. the expert products read the received records in place (row strides)
//      and the down launch stores each result row straight into the origin
//      rank's exchange buffer over NVLink (peer memory), then raises this
//      rank's flag on every rank;
//   7. a bounded wait for every rank's flag, then the combine.
//
// NCCL is loaded at run time (libnccl.so.2; the one already in the process
// when there is one), so a single-GPU engine links nothing more.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "../../include/miag/miag.h"
#include "kernels.cuh"

namespace miag {
int ctx_experts_to_ranks(miag_ctx *c, int layer, const int8_t *xq, size_t x_stride,
                         const float *dx, size_t dx_stride, int n_rows, const int32_t *pair_row,
                         const int32_t *pair_expert, int n_pairs, int n_ranks, int rank,
                         const int32_t *src_end, float *const *dst, unsigned *const *flags,
                         unsigned seq, cudaStream_t s, char *err, size_t errlen);
bool ctx_claim_ep(miag_ctx *c, const void *owner);
void ctx_release_ep(miag_ctx *c, const void *owner);
int ctx_device(const miag_ctx *c);
const miag_shape *ctx_shape(const miag_ctx *c);
cudaStream_t ctx_stream(const miag_ctx *c);
}  // namespace miag

using namespace miag;

namespace {

void put_err(char *err, size_t errlen, const char *fmt, ...) {
    if (!err || !errlen) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
}

// ---- NCCL, resolved at run time

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommCount)(const ncclComm_t, int *);
    ncclResult_t (*CommUserRank)(const ncclComm_t, int *);
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t);
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                              ncclComm_t, cudaStream_t);
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    const char *(*GetErrorString)(ncclResult_t);
};

std::mutex g_nccl_mutex;
NcclApi g_nccl;
bool g_nccl_ok = false;

const NcclApi *nccl(char *err, size_t errlen) {
    std::lock_guard<std::mutex> lock(g_nccl_mutex);
    if (g_nccl_ok) return &g_nccl;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        put_err(err, errlen, "expert parallelism needs NCCL: libnccl.so.2 not found (%s)", dlerror());
        return nullptr;
    }
    NcclApi a;
#define MIAG_NCCL_SYM(field, name)                                                   \
    a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name));                   \
    if (!a.field) {                                                                  \
        put_err(err, errlen, "libnccl.so.2 has no %s", name);                        \
        return nullptr;                                                              \
    }
    MIAG_NCCL_SYM(GetUniqueId, "ncclGetUniqueId")
    MIAG_NCCL_SYM(CommInitRank, "ncclCommInitRank")
    MIAG_NCCL_SYM(CommDestroy, "ncclCommDestroy")
    MIAG_NCCL_SYM(CommCount, "ncclCommCount")
    MIAG_NCCL_SYM(CommUserRank, "ncclCommUserRank")
    MIAG_NCCL_SYM(AllGather, "ncclAllGather")
    MIAG_NCCL_SYM(AllReduce, "ncclAllReduce")
    MIAG_NCCL_SYM(Send, "ncclSend")
    MIAG_NCCL_SYM(Recv, "ncclRecv")
    MIAG_NCCL_SYM(GroupStart, "ncclGroupStart")
    MIAG_NCCL_SYM(GroupEnd, "ncclGroupEnd")
    MIAG_NCCL_SYM(GetErrorString, "ncclGetErrorString")
#undef MIAG_NCCL_SYM
    g_nccl = a;
    g_nccl_ok = true;
    return &g_nccl;
}

// Pair records [n][2] (row, expert) into the two arrays the expert launches
// read.
__global__ void k_split_pairs(const int2 *meta, int n, int32_t *rows, int32_t *experts) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int2 m = meta[i];
    rows[i] = m.x;
    experts[i] = m.y;
}

template <class T>
bool grow(T *&p, size_t &cap, size_t n, cudaStream_t s, char *err, size_t errlen, const char *what) {
    if (n <= cap && p) return true;
    cudaStreamSynchronize(s);  // work already enqueued may still read the old buffer
    cudaFree(p);
    p = nullptr, cap = 0;
    const size_t want = n > 0 ? n + n / 2 : 1;
    const cudaError_t e = cudaMalloc(&p, want * sizeof(T));
    if (e != cudaSuccess) {
        put_err(err, errlen, "expert parallelism: cudaMalloc(%s, %zu bytes): %s", what,
                want * sizeof(T), cudaGetErrorString(e));
        return false;
    }
    cap = want;
    return true;
}

}  // namespace

struct miag_ep {
    miag_ctx *c = nullptr;
    ncclComm_t comm = nullptr;
    const NcclApi *api = nullptr;
    int rank = 0, world = 1, per_rank = 0, strided = 0, device = 0;
    int d = 0, K = 0, xs = 0;
    size_t rec_w = 0;  // bytes of a send record: d int8 values, then xs f32 scales
    // per step (grown to the largest step so far)
    int32_t *idx = nullptr, *send_rows = nullptr, *pair_meta = nullptr, *y_pos = nullptr;
    float *w = nullptr, *dx = nullptr, *x_stage = nullptr;
    int8_t *xq = nullptr;
    size_t cap_idx = 0, cap_rows = 0, cap_meta = 0, cap_ypos = 0, cap_w = 0, cap_dx = 0,
           cap_xq = 0, cap_xstage = 0;
    long long *counts = nullptr, *all_counts = nullptr, *h_counts = nullptr;
    uint8_t *rec = nullptr, *rec_in = nullptr;
    size_t cap_rec = 0, cap_rec_in = 0;
    int32_t *meta_out = nullptr, *meta_in = nullptr, *pair_row = nullptr, *pair_exp = nullptr;
    size_t cap_meta_out = 0, cap_meta_in = 0, cap_prow = 0, cap_pexp = 0;
    // the peer exchange: this rank's y rows and flags, every rank's mapped
    size_t y_rows = 0;
    std::vector<float *> peer_y;
    std::vector<unsigned *> peer_flags;
    unsigned seq = 0;
    uint8_t *d_small = nullptr;  // device scratch for handle / uuid all-gathers (8 x 64 B each)
    int last_received_pairs = 0, last_received_rows = 0;
};

namespace {

int nccl_check(const miag_ep *ep, ncclResult_t r, const char *what, char *err, size_t errlen) {
    if (r == ncclSuccess) return 0;
    put_err(err, errlen, "%s: %s", what, ep->api->GetErrorString(r));
    return -1;
}

#define EPCU(call)                                                                        \
    do {                                                                                  \
        cudaError_t e_ = (call);                                                          \
        if (e_ != cudaSuccess) {                                                          \
            put_err(err, errlen, "%s: %s", #call, cudaGetErrorString(e_));                \
            return -1;                                                                    \
        }                                                                                 \
    } while (0)

// A barrier over the communicator, on `s` and then on the host.
int ep_barrier(miag_ep *ep, cudaStream_t s, char *err, size_t errlen) {
    int *one = reinterpret_cast<int *>(ep->d_small);
    if (nccl_check(ep, ep->api->AllReduce(one, one, 1, ncclInt32, ncclSum, ep->comm, s),
                   "ncclAllReduce (barrier)", err, errlen))
        return -1;
    EPCU(cudaStreamSynchronize(s));
    return 0;
}

// Exchange buffers of at least `rows` y rows on every rank, mapped by every
// peer.  Every rank calls this with the same `rows` (derived from the
// all-gathered counts), so all grow together.  Nothing is in flight then:
// every store into this rank's buffer landed before this rank's last
// combine, which every rank's count all-gather follows.
int ensure_exchange(miag_ep *ep, size_t rows, cudaStream_t s, char *err, size_t errlen) {
    rows = rows > 0 ? rows : 1;
    if (rows <= ep->y_rows) return 0;
    rows = rows > 2 * ep->y_rows ? rows : 2 * ep->y_rows;
    EPCU(cudaStreamSynchronize(s));
    if (ep->y_rows && miag_ep_close_peers(ep->c, err, errlen)) return -1;
    if (ep_barrier(ep, s, err, errlen)) return -1;  // nobody maps the old buffers now
    void *y = nullptr;
    unsigned *flags = nullptr;
    uint8_t handle[64];
    if (miag_ep_buffer(ep->c, rows, &y, &flags, handle, err, errlen)) return -1;
    uint8_t *dh = ep->d_small + 64;  // [world][64] handles
    EPCU(cudaMemcpyAsync(dh + 64 * ep->rank, handle, 64, cudaMemcpyHostToDevice, s));
    if (nccl_check(ep, ep->api->AllGather(dh + 64 * ep->rank, dh, 64, ncclUint8, ep->comm, s),
                   "ncclAllGather (exchange handles)", err, errlen))
        return -1;
    std::vector<uint8_t> all(64 * (size_t)ep->world);
    EPCU(cudaMemcpyAsync(all.data(), dh, all.size(), cudaMemcpyDeviceToHost, s));
    EPCU(cudaStreamSynchronize(s));
    ep->peer_y.assign((size_t)ep->world, nullptr);
    ep->peer_flags.assign((size_t)ep->world, nullptr);
    for (int r = 0; r < ep->world; r++) {
        if (r == ep->rank) {
            ep->peer_y[(size_t)r] = static_cast<float *>(y);
            ep->peer_flags[(size_t)r] = flags;
            continue;
        }
        void *py = nullptr;
        unsigned *pf = nullptr;
        if (miag_ep_open_peer(ep->c, all.data() + 64 * r, &py, &pf, err, errlen)) return -1;
        ep->peer_y[(size_t)r] = static_cast<float *>(py);
        ep->peer_flags[(size_t)r] = pf;
    }
    ep->y_rows = rows;
    return ep_barrier(ep, s, err, errlen);  // every rank mapped before anyone stores
}

}  // namespace

extern "C" int miag_nccl_unique_id(void *id, char *err, size_t errlen) {
    const NcclApi *a = nccl(err, errlen);
    if (!a) return -1;
    if (!id) {
        put_err(err, errlen, "null id buffer");
        return -1;
    }
    ncclUniqueId u;
    const ncclResult_t r = a->GetUniqueId(&u);
    if (r != ncclSuccess) {
        put_err(err, errlen, "ncclGetUniqueId: %s", a->GetErrorString(r));
        return -1;
    }
    memcpy(id, &u, sizeof u);
    return 0;
}

extern "C" int miag_nccl_comm_init(void **comm, int n_ranks, const void *id, int rank, int device,
                                   char *err, size_t errlen) {
    const NcclApi *a = nccl(err, errlen);
    if (!a) return -1;
    if (!comm || !id || n_ranks < 1 || rank < 0 || rank >= n_ranks) {
        put_err(err, errlen, "bad communicator arguments");
        return -1;
    }
    const cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        put_err(err, errlen, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
        return -1;
    }
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    ncclComm_t c = nullptr;
    const ncclResult_t r = a->CommInitRank(&c, n_ranks, u, rank);
    if (r != ncclSuccess) {
        put_err(err, errlen, "ncclCommInitRank: %s", a->GetErrorString(r));
        return -1;
    }
    *comm = c;
    return 0;
}

extern "C" void miag_nccl_comm_destroy(void *comm) {
    if (comm && g_nccl_ok) g_nccl.CommDestroy(static_cast<ncclComm_t>(comm));
}

extern "C" void miag_ep_close(miag_ep *ep) {
    if (!ep) return;
    if (ep->c) {
        cudaSetDevice(ep->device);
        cudaStreamSynchronize(ctx_stream(ep->c));
        if (ep->y_rows) miag_ep_close_peers(ep->c, nullptr, 0);
        ctx_release_ep(ep->c, ep);
    }
    cudaFree(ep->idx), cudaFree(ep->send_rows), cudaFree(ep->pair_meta), cudaFree(ep->y_pos);
    cudaFree(ep->w), cudaFree(ep->dx), cudaFree(ep->xq), cudaFree(ep->x_stage);
    cudaFree(ep->counts), cudaFree(ep->all_counts);
    if (ep->h_counts) cudaFreeHost(ep->h_counts);
    cudaFree(ep->rec), cudaFree(ep->rec_in), cudaFree(ep->meta_out), cudaFree(ep->meta_in);
    cudaFree(ep->pair_row), cudaFree(ep->pair_exp), cudaFree(ep->d_small);
    delete ep;
}

extern "C" int miag_ep_open(miag_ep **out, miag_ctx *c, void *nccl_comm, int strided, char *err,
                            size_t errlen) {
    if (!out || !c || !nccl_comm) {
        put_err(err, errlen, "null argument");
        return -1;
    }
    *out = nullptr;
    const NcclApi *a = nccl(err, errlen);
    if (!a) return -1;
    miag_ep *ep = new (std::nothrow) miag_ep();
    if (!ep) {
        put_err(err, errlen, "out of host memory");
        return -1;
    }
    ep->api = a;
    ep->comm = static_cast<ncclComm_t>(nccl_comm);
    const miag_shape *sh = ctx_shape(c);
    ep->device = ctx_device(c);
    auto fail = [&]() {
        ep->c = nullptr;  // not claimed
        miag_ep_close(ep);
        return -1;
    };
    if (a->CommCount(ep->comm, &ep->world) != ncclSuccess ||
        a->CommUserRank(ep->comm, &ep->rank) != ncclSuccess) {
        put_err(err, errlen, "not an NCCL communicator");
        return fail();
    }
    if (ep->world < 1 || ep->world > kEpMaxRanks || sh->n_experts % ep->world) {
        put_err(err, errlen, "%d ranks: need 1..%d ranks that split all %d experts evenly",
                ep->world, kEpMaxRanks, sh->n_experts);
        return fail();
    }
    if (sh->n_active > 32) {  // the plan's per-tile pair prefixes are 16-bit fields
        put_err(err, errlen, "expert parallelism supports at most 32 active experts");
        return fail();
    }
    if (!ctx_claim_ep(c, ep)) {
        put_err(err, errlen, "this context's exchange buffer already belongs to an expert-parallel block");
        return fail();
    }
    ep->c = c;
    ep->per_rank = sh->n_experts / ep->world;
    ep->strided = strided != 0;
    ep->d = sh->dim, ep->K = sh->n_active, ep->xs = miag_dx_stride(sh);
    ep->rec_w = (size_t)ep->d + 4 * (size_t)ep->xs;
    cudaError_t e;
    if ((e = cudaSetDevice(ep->device)) != cudaSuccess ||
        (e = cudaMalloc(&ep->counts, 2 * kEpMaxRanks * sizeof(long long))) != cudaSuccess ||
        (e = cudaMalloc(&ep->all_counts, 2 * kEpMaxRanks * kEpMaxRanks * sizeof(long long))) !=
            cudaSuccess ||
        (e = cudaHostAlloc(&ep->h_counts, 2 * kEpMaxRanks * kEpMaxRanks * sizeof(long long),
                           cudaHostAllocDefault)) != cudaSuccess ||
        (e = cudaMalloc(&ep->d_small, 64 * (kEpMaxRanks + 1))) != cudaSuccess) {
        put_err(err, errlen, "expert parallelism set-up: %s", cudaGetErrorString(e));
        return fail();
    }
    // One GPU per rank: the flag waits of two ranks must never share a GPU
    // (nothing guarantees such kernels run at the same time).
    const cudaStream_t s = ctx_stream(c);
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, ep->device)) != cudaSuccess) {
        put_err(err, errlen, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
        return fail();
    }
    uint8_t *du = ep->d_small + 64;
    std::vector<uint8_t> uu(16 * (size_t)ep->world);
    if ((e = cudaMemsetAsync(ep->d_small, 0, 64, s)) != cudaSuccess ||
        (e = cudaMemcpyAsync(du + 16 * ep->rank, &prop.uuid, 16, cudaMemcpyHostToDevice, s)) !=
            cudaSuccess) {
        put_err(err, errlen, "expert parallelism set-up: %s", cudaGetErrorString(e));
        return fail();
    }
    if (nccl_check(ep, a->AllGather(du + 16 * ep->rank, du, 16, ncclUint8, ep->comm, s),
                   "ncclAllGather (device ids)", err, errlen))
        return fail();
    if ((e = cudaMemcpyAsync(uu.data(), du, uu.size(), cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
        (e = cudaStreamSynchronize(s)) != cudaSuccess) {
        put_err(err, errlen, "expert parallelism set-up: %s", cudaGetErrorString(e));
        return fail();
    }
    for (int r = 0; r < ep->world; r++)
        for (int q = r + 1; q < ep->world; q++)
            if (!memcmp(uu.data() + 16 * r, uu.data() + 16 * q, 16)) {
                put_err(err, errlen, "ranks %d and %d share a GPU: expert parallelism needs one GPU a rank", r, q);
                return fail();
            }
    // d_small[0] holds the barrier's int 1
    const int one = 1;
    if ((e = cudaMemcpyAsync(ep->d_small, &one, sizeof one, cudaMemcpyHostToDevice, s)) !=
            cudaSuccess ||
        (e = cudaStreamSynchronize(s)) != cudaSuccess) {
        put_err(err, errlen, "expert parallelism set-up: %s", cudaGetErrorString(e));
        return fail();
    }
    *out = ep;
    return 0;
}

extern "C" int miag_ep_rank(const miag_ep *ep, int *rank, int *n_ranks, int *first_expert,
                            int *n_experts_here, int *stride) {
    if (!ep) return -1;
    if (rank) *rank = ep->rank;
    if (n_ranks) *n_ranks = ep->world;
    if (first_expert) *first_expert = ep->strided ? ep->rank : ep->rank * ep->per_rank;
    if (n_experts_here) *n_experts_here = ep->per_rank;
    if (stride) *stride = ep->strided ? ep->world : 1;
    return 0;
}

extern "C" int miag_ep_last_received(const miag_ep *ep, int *rows, int *pairs) {
    if (!ep) return -1;
    if (rows) *rows = ep->last_received_rows;
    if (pairs) *pairs = ep->last_received_pairs;
    return 0;
}

extern "C" int miag_moe_ep_async(miag_ep *ep, int layer, float *x_dev, int n_tokens, void *stream,
                                 char *err, size_t errlen) {
    if (!ep || !ep->c) {
        put_err(err, errlen, "null expert-parallel block");
        return -1;
    }
    if (n_tokens < 0 || (n_tokens > 0 && !x_dev) || ((uintptr_t)x_dev & 15u)) {
        put_err(err, errlen, "bad token buffer (device pointer, 16-byte aligned)");
        return -1;
    }
    EPCU(cudaSetDevice(ep->device));
    const cudaStream_t s = stream ? (cudaStream_t)stream : ctx_stream(ep->c);
    const int T = n_tokens, K = ep->K, G = ep->world, me = ep->rank;
    const size_t P = (size_t)T * K;
    // this step's buffers (every rank takes the same collective steps below,
    // with or without tokens)
    if (!grow(ep->idx, ep->cap_idx, P, s, err, errlen, "idx") ||
        !grow(ep->w, ep->cap_w, P, s, err, errlen, "weights") ||
        !grow(ep->xq, ep->cap_xq, (size_t)T * ep->d, s, err, errlen, "xq") ||
        !grow(ep->dx, ep->cap_dx, (size_t)T * ep->xs, s, err, errlen, "dx") ||
        !grow(ep->send_rows, ep->cap_rows, (size_t)T * G, s, err, errlen, "send rows") ||
        !grow(ep->pair_meta, ep->cap_meta, 2 * P, s, err, errlen, "pair records") ||
        !grow(ep->y_pos, ep->cap_ypos, P, s, err, errlen, "result places"))
        return -1;
    if (T > 0 && miag_route_async(ep->c, layer, x_dev, T, ep->idx, ep->w, ep->xq, ep->dx, s, err,
                                  errlen))
        return -1;
    if (miag_ep_plan_async(ep->c, ep->idx, T, G, ep->per_rank, ep->strided,
                           reinterpret_cast<int64_t *>(ep->counts), ep->send_rows, ep->pair_meta,
                           ep->y_pos, s, err, errlen))
        return -1;
    // every rank's (rows, pairs) per destination: the one host synchronisation
    if (nccl_check(ep, ep->api->AllGather(ep->counts, ep->all_counts, 2 * (size_t)G, ncclInt64,
                                          ep->comm, s),
                   "ncclAllGather (counts)", err, errlen))
        return -1;
    EPCU(cudaMemcpyAsync(ep->h_counts, ep->all_counts, 2 * (size_t)G * G * sizeof(long long),
                         cudaMemcpyDeviceToHost, s));
    EPCU(cudaStreamSynchronize(s));
    const long long *M = ep->h_counts;  // [src][dst][rows, pairs]
    auto rows_of = [&](int src, int dst) { return (size_t)M[2 * (src * G + dst)]; };
    auto pairs_of = [&](int src, int dst) { return (size_t)M[2 * (src * G + dst) + 1]; };
    size_t R_out = 0, R_in = 0, P_in = 0, max_sent = 0;
    for (int r = 0; r < G; r++) {
        R_out += rows_of(me, r), R_in += rows_of(r, me), P_in += pairs_of(r, me);
        size_t sent = 0;
        for (int q = 0; q < G; q++) sent += pairs_of(r, q);
        max_sent = sent > max_sent ? sent : max_sent;
    }
    if (!grow(ep->rec, ep->cap_rec, R_out * ep->rec_w, s, err, errlen, "send records") ||
        !grow(ep->meta_out, ep->cap_meta_out, 2 * P, s, err, errlen, "pair records out") ||
        !grow(ep->rec_in, ep->cap_rec_in, R_in * ep->rec_w, s, err, errlen, "received records") ||
        !grow(ep->meta_in, ep->cap_meta_in, 2 * P_in, s, err, errlen, "pair records in") ||
        !grow(ep->pair_row, ep->cap_prow, P_in, s, err, errlen, "pair rows") ||
        !grow(ep->pair_exp, ep->cap_pexp, P_in, s, err, errlen, "pair experts"))
        return -1;
    if (ensure_exchange(ep, max_sent, s, err, errlen)) return -1;
    if (miag_ep_pack_async(ep->c, ep->xq, ep->dx, ep->send_rows, (int)R_out, ep->pair_meta, (int)P,
                           reinterpret_cast<const int64_t *>(ep->all_counts), me, G, ep->rec,
                           ep->meta_out, s, err, errlen))
        return -1;
    // rows and pair records to the ranks that hold the experts, in one group
    if (nccl_check(ep, ep->api->GroupStart(), "ncclGroupStart", err, errlen)) return -1;
    size_t ro = 0, ri = 0, po = 0, pi = 0;
    for (int r = 0; r < G; r++) {
        const size_t rs = rows_of(me, r), rr = rows_of(r, me);
        const size_t ps = pairs_of(me, r), pr = pairs_of(r, me);
        ncclResult_t res = ncclSuccess;
        if (rs) res = ep->api->Send(ep->rec + ro * ep->rec_w, rs * ep->rec_w, ncclUint8, r, ep->comm, s);
        if (res == ncclSuccess && rr)
            res = ep->api->Recv(ep->rec_in + ri * ep->rec_w, rr * ep->rec_w, ncclUint8, r, ep->comm, s);
        if (res == ncclSuccess && ps)
            res = ep->api->Send(ep->meta_out + 2 * po, 2 * ps, ncclInt32, r, ep->comm, s);
        if (res == ncclSuccess && pr)
            res = ep->api->Recv(ep->meta_in + 2 * pi, 2 * pr, ncclInt32, r, ep->comm, s);
        if (res != ncclSuccess) {
            ep->api->GroupEnd();
            return nccl_check(ep, res, "ncclSend/ncclRecv (dispatch)", err, errlen);
        }
        ro += rs, ri += rr, po += ps, pi += pr;
    }
    if (nccl_check(ep, ep->api->GroupEnd(), "ncclGroupEnd (dispatch)", err, errlen)) return -1;
    if (P_in > 0) {
        k_split_pairs<<<(unsigned)((P_in + 255) / 256), 256, 0, s>>>(
            reinterpret_cast<const int2 *>(ep->meta_in), (int)P_in, ep->pair_row, ep->pair_exp);
        EPCU(cudaGetLastError());
    }
    // the expert products; each result row goes to its origin rank
    int32_t src_end[kEpMaxRanks];
    float *dst[kEpMaxRanks];
    size_t acc = 0;
    for (int r = 0; r < G; r++) {
        acc += pairs_of(r, me);
        src_end[r] = (int)acc;
        size_t before = 0;  // the pairs r sends to lower ranks come first in its y order
        for (int q = 0; q < me; q++) before += pairs_of(r, q);
        dst[r] = ep->peer_y[(size_t)r] + before * (size_t)ep->d;
    }
    ep->seq++;
    if (ctx_experts_to_ranks(ep->c, layer, reinterpret_cast<const int8_t *>(ep->rec_in), ep->rec_w,
                             reinterpret_cast<const float *>(ep->rec_in + ep->d), ep->rec_w,
                             (int)R_in, ep->pair_row, ep->pair_exp, (int)P_in, G, me, src_end, dst,
                             ep->peer_flags.data(), ep->seq, s, err, errlen))
        return -1;
    ep->last_received_rows = (int)R_in, ep->last_received_pairs = (int)P_in;
    // every rank's rows for this one have landed, then the combine
    if (miag_ep_wait_async(ep->c, ep->peer_flags[(size_t)me], G, ep->seq, s, err, errlen)) return -1;
    if (T > 0 && miag_combine_async(ep->c, x_dev, T, ep->w, ep->peer_y[(size_t)me], ep->y_pos, s,
                                    err, errlen))
        return -1;
    return 0;
}

extern "C" int miag_moe_ep(miag_ep *ep, int layer, float *x, int n_tokens, char *err,
                           size_t errlen) {
    if (!ep || !ep->c) {
        put_err(err, errlen, "null expert-parallel block");
        return -1;
    }
    if (n_tokens < 0 || (n_tokens > 0 && !x)) {
        put_err(err, errlen, "bad token buffer");
        return -1;
    }
    EPCU(cudaSetDevice(ep->device));
    const cudaStream_t s = ctx_stream(ep->c);
    const size_t bytes = (size_t)n_tokens * ep->d * sizeof(float);
    if (!grow(ep->x_stage, ep->cap_xstage, (size_t)n_tokens * ep->d, s, err, errlen, "x"))
        return -1;
    if (bytes) EPCU(cudaMemcpyAsync(ep->x_stage, x, bytes, cudaMemcpyHostToDevice, s));
    if (miag_moe_ep_async(ep, layer, ep->x_stage, n_tokens, s, err, errlen)) return -1;
    if (bytes) EPCU(cudaMemcpyAsync(x, ep->x_stage, bytes, cudaMemcpyDeviceToHost, s));
    return miag_sync(ep->c, s, err, errlen);
}
