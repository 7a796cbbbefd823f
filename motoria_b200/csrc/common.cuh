// common.cuh -- shared device helpers and layouts of libmiag (sm_100a).
//
// Numerics: nothing here is compiled with fast-math.  Every float operation
// whose rounding the reference fixes is written with an explicit
// round-to-nearest intrinsic (__fadd_rn, __fmul_rn, __fdiv_rn, ...), which
// the compiler never contracts into an FMA, so the GPU repeats the
// reference's x86 scalar arithmetic operation for operation.
#pragma once

#include <cstddef>
#include <cstdint>
#include <utility>
#include <cuda_runtime.h>

#define MIAG_QK 32

namespace miag {

// Device error codes written to the context's error word (first one wins).
enum : int {
    kErrNone = 0,
    kErrWaitFull = 1,     // a consumer gave up waiting for a staged tile
    kErrWaitEmpty = 2,    // the producer gave up waiting for a free stage
    kErrBadExpert = 3,    // a routing index outside [0, E)
    kErrItemList = 4,     // an expert launch's work list named a tile outside the store
    kErrWaitPeer = 5,     // a rank gave up waiting for another rank's expert results
};

// Bounded spin: about one second at B200 clocks.
constexpr long long kWaitCycles = 2000000000LL;

// ---------------------------------------------------------------------------
// HBM layout of one layer's expert store, repacked at upload from the .mia
// array of 36-byte {f32 d; int8 q[32]} blocks.  Per expert, two matrices:
//   GU: 2*eh rows x d columns, row 2i = gate row i, row 2i+1 = up row i
//   DN: d rows x eh columns (down)
// Each matrix is cut into tiles of 128 rows x 128 bytes of K (4 Q8_0
// blocks), stored [row tile][k tile], 16 KiB each.  Inside a tile, 8-row
// atoms of 8 x 128 B hold row r's 16-byte chunk c at chunk c ^ (r % 8): the
// 128-byte swizzle of the tensor-core K-major layout, which also makes eight
// rows' same-column chunks land in distinct shared-memory banks.  The scales
// of a tile, [128 rows][4 blocks] f32 (2 KiB), follow it directly: a unit of
// 18 KiB, so the k tiles a kernel streams, scales included, are one
// contiguous range (on B200 a bulk copy costs ~0.26 us of the copy engine
// whatever its size up to ~8 KiB, so separate scale copies cost a quarter of
// the bandwidth).  Rows and columns beyond the matrix are zero.
constexpr int kTileRows = 128;
constexpr int kTileK = 128;                       // bytes of K per tile = 4 blocks
constexpr int kTileBytes = kTileRows * kTileK;    // 16 KiB
constexpr int kTileScaleBytes = kTileRows * 4 * 4;  // 2 KiB
constexpr int kUnitBytes = kTileBytes + kTileScaleBytes;  // tile + its scales

struct StoreLayout {
    int d, eh;
    int gu_rt, gu_kt;  // GU row tiles, k tiles
    int dn_rt, dn_kt;
    uint32_t gu_off, dn_off;  // first unit of each matrix; unit (rt, kt) at + (rt*kt_count + kt) units
    size_t expert_bytes;
};

inline size_t round_up_sz(size_t n, size_t a) { return (n + a - 1) / a * a; }

inline StoreLayout make_layout(int d, int eh) {
    StoreLayout L;
    L.d = d, L.eh = eh;
    L.gu_rt = (2 * eh + kTileRows - 1) / kTileRows;
    L.gu_kt = (d + kTileK - 1) / kTileK;
    L.dn_rt = (d + kTileRows - 1) / kTileRows;
    L.dn_kt = (eh + kTileK - 1) / kTileK;
    size_t off = 0;
    L.gu_off = (uint32_t)off;
    off += (size_t)L.gu_rt * L.gu_kt * kUnitBytes;
    L.dn_off = (uint32_t)off;
    off += (size_t)L.dn_rt * L.dn_kt * kUnitBytes;
    L.expert_bytes = round_up_sz(off, 1024);
    return L;
}

// Byte offset of (row r, 16-byte chunk c) inside a 128 x 128 B swizzled tile.
__host__ __device__ inline uint32_t tile_chunk_offset(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Shared-memory row stride for a staged row of `bytes`: a multiple of 16
// whose 16-byte count is odd, so eight lanes reading 16 bytes at the same
// column of eight consecutive rows hit 32 distinct banks.
__host__ __device__ inline uint32_t smem_stride(uint32_t bytes) {
    uint32_t s = (bytes + 15u) & ~15u;
    if (((s >> 4) & 1u) == 0u) s += 16u;
    return s;
}

// Padded count of f32 scales per activation row (16-byte rows).
__host__ __device__ inline int scale_pad(int nblocks) { return (nblocks + 3) & ~3; }

// ---------------------------------------------------------------------------
// Correctly rounded expf: the float nearest CUDA's double-precision exp
// (documented max error 1 double ulp), i.e. the true e^x rounded to float
// except within ~2^-29 relative of a float rounding midpoint.
__device__ __forceinline__ float expf_cr(float x) {
    return __double2float_rn(exp((double)x));
}

// Reference SiLU-GLU element (forward.c:189-190): g / (1 + expf(-g)) * u.
__device__ __forceinline__ float swiglu_ref(float g, float u) {
    float e = expf_cr(-g);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, e)), u);
}

// ---------------------------------------------------------------------------
// mbarrier / bulk-copy (TMA 1-D) wrappers; every copy lands in this CTA's own
// shared memory.
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy accesses to shared memory
// before its later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// One bounded wait: the thread is suspended in hardware until the phase
// completes or the hint (10 ms) runs out, so waiting issues no instructions
// that would compete with the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(10000000u)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `parity` to complete; false after `limit` cycles.
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity, long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) return false;
    }
    return true;
}

// Waits for the phase of `parity` to complete; false after ~1 s.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    return mbar_wait_for(bar, parity, kWaitCycles);
}

// Global -> shared bulk copy completing on `bar` (16-B aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// 4 bytes from shared memory (a shared-window address).
__device__ __forceinline__ float lds32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// 16 bytes from shared memory (a shared-window address).
__device__ __forceinline__ float4 lds128(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ unsigned sm_id() {
    unsigned r;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// A flag between GPUs: stored with release, loaded with acquire, both at
// system scope (the other side may be a peer GPU).
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// bar.sync on a named barrier shared by `threads` threads (a multiple of 32).
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Programmatic dependent launch.  The block's kernels go out with
// launch_dependent, so each may start while the kernel before it in the
// stream still runs.  Before pdl_wait a kernel touches nothing an earlier
// kernel of the stream writes or reads (it may read the layer's constant
// weights and set up shared memory); pdl_wait returns once the previous
// kernel -- and so, since every kernel waits before it ends, every earlier
// one -- has finished and its writes are visible.  pdl_launch_dependents
// lets the next kernel's CTAs start their own prologues.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t s, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid, cfg.blockDim = block, cfg.dynamicSmemBytes = smem, cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr, cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__device__ __forceinline__ void set_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// One reference Q8_0 step: s += ((float)acc * dw) * dx (matmul.c:25).
__device__ __forceinline__ float q8_step(float s, int acc, float dw, float dx) {
    return __fadd_rn(s, __fmul_rn(__fmul_rn(__int2float_rn(acc), dw), dx));
}


// ---------------------------------------------------------------------------
// rmsnorm's scale (forward.c:75-81), certified equal to the reference's.

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
// lane 0 repeats the serial sum over x (shared memory).
__device__ __forceinline__ float rms_scale_certified(double ss, const float *x, int n, float eps, int lane) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const double rel = (2.02 * (double)n + 8.0) * 1.1102230246251565e-16;  // 2^-53
    // lanes 0 and 1 evaluate the two ends of the bracket at the same time
    const float end = rms_scale_of(ss * (lane == 0 ? 1.0 - rel : 1.0 + rel), n, eps);
    const float a = __shfl_sync(0xffffffffu, end, 0), b = __shfl_sync(0xffffffffu, end, 1);
    if (a == b) return a;
    float r = 0.0f;
    if (lane == 0) {
        double s2 = 0.0;
        for (int i = 0; i < n; i++) {
            const double v = (double)x[i];
            s2 = __dadd_rn(s2, __dmul_rn(v, v));
        }
        r = rms_scale_of(s2, n, eps);
    }
    return __shfl_sync(0xffffffffu, r, 0);
}

// ---------------------------------------------------------------------------
// Exact Q8_0 steps on int8 tensor-core dots.

// The int8 MMA accumulates onto kMagicBits, the bit pattern of 1.5 * 2^23.
// A Q8_0 block dot satisfies |dot| <= 32 * 127 * 127 < 2^22, so the int32
// result, read as a float, is exactly 12582912 + dot (same binade, unit ulp)
// and one exact subtraction gives (float)dot.  The conversion so runs on the
// FMA pipe; as an int-to-float conversion it saturated the conversion unit.
constexpr int kMagicBits = 0x4B400000;
constexpr float kMagic = 12582912.0f;

// Two f32 lanes in one 64-bit register: the packed FP32 instructions of
// sm_100 (FADD2, FMUL2, FFMA2) do one operation on both.
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
    uint64_t v;
    asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
    return v;
}
__device__ __forceinline__ uint64_t pack2i(int lo, int hi) {
    uint64_t v;
    asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(lo), "r"(hi));
    return v;
}
__device__ __forceinline__ float2 unpack2(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}

// The reference step s += ((float)dot * dw) * dx (matmul.c:25) for two
// accumulators at once, on magic MMA results m = kMagicBits + dot.  Each
// operation is rounded on its own, as in the reference: the dot is exact,
// then two rounded products.  The product is added as fma(v, one, s) with
// one = 1.0 from a kernel argument: v * 1 is exact, so this rounds once like
// the add -- and the compiler, which contracts a packed multiply feeding a
// packed add into one FFMA2 even when both are written with .rn (measured on
// sm_100a), finds no multiply-add pair here to contract.
__device__ __forceinline__ void q8_step_x2(uint64_t &s, uint64_t m, uint64_t w2, uint64_t x2,
                                           uint64_t neg_magic2, uint64_t one2) {
    uint64_t t;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(t) : "l"(m), "l"(neg_magic2));
    asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(t) : "l"(w2));
    asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(t) : "l"(x2));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(s) : "l"(t), "l"(one2));
}

}  // namespace miag
