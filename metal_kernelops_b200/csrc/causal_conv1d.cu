// Causal depthwise conv1d (the convolution in front of the scan in Mamba
// blocks) for sm_100a: prefill forward, analytic backward, decode update.
//
// Reference behaviour: src/metal_kernelops/cv/causal_conv1d.py --
// `causal_conv1d_fn` (:610-690), `_CausalConv1d` (:531-607) and
// `causal_conv1d_update` (:690-756).  With z = cat(initial_state, x) (zeros
// without a state) and taps = K - 1:
//     out[t]      = act(bias + sum_j w[j] z[t + j])          act = id or SiLU
//     final_state = z[L .. L + taps)
// and, with g[t] = dout[t] act'(pre[t]) for t < L,
//     dx[s]       = sum_j w[j] g[s + taps - j]
//     dinit[p]    = sum_{j <= p} w[j] g[p - j]                p < taps
//     dweight[j]  = sum_{b, t} g[t] z[t + j],   dbias = sum_{b, t} g[t]
//
// The work is bytes, not flops (2 K flops per element), so the kernels are
// built for HBM.  Rows of 16-byte aligned bytes stream through a ring of
// shared-memory stages filled by bulk asynchronous copies (the bulk-copy
// pipeline path below), computed with paired fp32 instructions; other rows
// take a plain path, a warp per 512-element segment with the taps-wide halos
// from the neighbouring lanes by shuffle.  The backward recomputes the
// pre-activation from x instead of saving it, and leaves dweight / dbias as
// partials that a second kernel folds per channel in a fixed order, so
// results are reproducible.
#include "common.cuh"
#include "tc.cuh"

namespace ssm {
namespace conv {

constexpr int kThreads = 256;
constexpr int kMaxWidth = 8;

struct Args {
    int64_t batch, channels, length, rows;    // rows = batch * channels
    int64_t nchunks, chunk;                   // chunks per row, elements per chunk
    int64_t slots;                            // dweight / dbias partials per chunk
    int64_t per;                              // bulk: items per CTA
    uint32_t flags;
    int64_t xs, ds;                           // channel-last: row strides of x and dout
    const void* x; const float* w; const float* bias; const void* init;
    void* out; void* final_state;
    const void* dout; void* dx; void* dinit;
    float* partial;                           // (rows, nchunks, slots, K + 1)
    int* status;                              // the call's optional status word
};

constexpr uint32_t kHasBias = SSM_HAS_BIAS, kSilu = SSM_CONV_SILU, kHasInit = SSM_HAS_INIT;

template <typename T, int V> struct Vec;
template <typename T> struct Vec<T, 1> {
    static __device__ __forceinline__ void ld(const T* p, float* v) { v[0] = ldf(p); }
    static __device__ __forceinline__ void st(T* p, const float* v) { stf(p, v[0]); }
};
template <> struct Vec<float, 8> {
    static __device__ __forceinline__ void ld(const float* p, float* v) {
        const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    static __device__ __forceinline__ void st(float* p, const float* v) {
        reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
};
template <typename H2, typename T> struct Vec16 {
    static __device__ __forceinline__ void ld(const T* p, float* v) {
        const uint4 r = *reinterpret_cast<const uint4*>(p);
        const H2* h = reinterpret_cast<const H2*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = Io2<T>::ld(reinterpret_cast<const T*>(&h[i]));
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
    static __device__ __forceinline__ void st(T* p, const float* v) {
        uint4 r;
        H2* h = reinterpret_cast<H2*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) Io2<T>::st(reinterpret_cast<T*>(&h[i]), make_float2(v[2 * i], v[2 * i + 1]));
        *reinterpret_cast<uint4*>(p) = r;
    }
};
template <> struct Vec<__nv_bfloat16, 8> : Vec16<__nv_bfloat162, __nv_bfloat16> {};
template <> struct Vec<__half, 8> : Vec16<__half2, __half> {};

// z at x-position p of one row: the initial state left of 0, zero past L.
template <typename T, int TAPS>
__device__ __forceinline__ float zval(const T* xr, const T* ir, int64_t p, int64_t L) {
    if (p < 0) return ir != nullptr ? ldf(ir + TAPS + p) : 0.0f;
    return p < L ? ldf(xr + p) : 0.0f;
}

// Each warp walks segments of 32 * E consecutive elements of its row, lane l
// owning E = U * V of them (U vectors of V).  The taps-wide halo left of a
// lane's elements is the previous lane's last taps values (a shuffle); lane 0
// reads it from memory, or from the initial state left of position 0.  Loops
// are warp-uniform so that every shuffle has all 32 lanes.
template <typename T, int V, int U, bool VEC>
__device__ __forceinline__ void load_run(const T* xr, int64_t t0, int64_t L, float* dst) {
    constexpr int E = U * V;
    if (VEC && t0 + E <= L) {
#pragma unroll
        for (int u = 0; u < U; ++u) Vec<T, V>::ld(xr + t0 + u * V, dst + u * V);
    } else {
#pragma unroll
        for (int i = 0; i < E; ++i) dst[i] = t0 + i < L ? ldf(xr + t0 + i) : 0.0f;
    }
}
template <typename T, int V, int U, bool VEC>
__device__ __forceinline__ void store_run(T* r, int64_t t0, int64_t L, const float* src) {
    constexpr int E = U * V;
    if (VEC && t0 + E <= L) {
#pragma unroll
        for (int u = 0; u < U; ++u) Vec<T, V>::st(r + t0 + u * V, src + u * V);
    } else {
#pragma unroll
        for (int i = 0; i < E; ++i)
            if (t0 + i < L) stf(r + t0 + i, src[i]);
    }
}

// (row, tile) and channel of a work item with 32-bit divisions: the host
// guarantees rows * nchunks < 2^31 (64-bit division is a long emulated
// sequence, and these run once per item and thread).
__device__ __forceinline__ void item_coords(const Args& a, int64_t it, int64_t& row, int64_t& tile, int64_t& c) {
    const uint32_t i = (uint32_t)it, nc = (uint32_t)a.nchunks;
    const uint32_t r = i / nc;
    row = r;
    tile = i - r * nc;
    c = r % (uint32_t)a.channels;
}

// One lane's backward over E positions: g over E + taps positions (dout on
// entry, times act'(pre) on exit), dx into o, and this lane's dweight/dbias.
// Positions past the row must arrive with g = 0.
template <typename T, int K, int E>
__device__ __forceinline__ void conv_bwd_lane(const float* w, float bv, bool silu, const float* z, float* g,
                                              float* o, float* dw) {
    constexpr int TAPS = K - 1, NG = E + TAPS;
    if (silu) {
#pragma unroll
        for (int u = 0; u < NG; ++u) {
            float pre = bv;
#pragma unroll
            for (int j = 0; j < K; ++j) pre = fmaf(w[j], z[u + j], pre);
            g[u] *= silu_grad_t<T>(pre);
        }
    }
#pragma unroll
    for (int i = 0; i < E; ++i) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < K; ++j) acc = fmaf(w[j], g[i + TAPS - j], acc);
        o[i] = acc;
    }
#pragma unroll
    for (int j = 0; j <= K; ++j) dw[j] = 0.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) {
        dw[K] += g[i];
#pragma unroll
        for (int j = 0; j < K; ++j) dw[j] = fmaf(g[i], z[i + j], dw[j]);
    }
}

// Gradient of the initial state of one row: dinit[p] = sum_{j <= p} w[j] g[p - j].
template <typename T, int K>
__device__ __forceinline__ void dinit_row(T* dir, const float* w, const float* g) {
#pragma unroll
    for (int p = 0; p < K - 1; ++p) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j <= p; ++j) acc = fmaf(w[j], g[p - j], acc);
        stf(dir + p, acc);
    }
}

// ------------------------------------------------------ plain (any layout) --
// Rows that are not 16-byte aligned: one warp per (row, 512-element segment)
// item, lane l owning 16 elements loaded one by one; the taps-wide halos come
// from the neighbouring lanes by shuffle (the warp's ends from memory).
constexpr int64_t kSeg = 32 * 16;

template <typename T, int K>
__global__ void __launch_bounds__(kThreads)
fwd_plain_kernel(const Args a) {
    constexpr int TAPS = K - 1, E = 16;
    const int lane = threadIdx.x & 31;
    const int64_t it = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
    if (it >= a.rows * a.nchunks) return;        // warp-uniform
    const int64_t L = a.length;
    int64_t row, seg, c;
    item_coords(a, it, row, seg, c);
    const int64_t t0 = seg * kSeg + (int64_t)lane * E;
    const T* xr = static_cast<const T*>(a.x) + row * L;
    const T* ir = (a.flags & kHasInit) ? static_cast<const T*>(a.init) + row * TAPS : nullptr;
    float w[K];
#pragma unroll
    for (int j = 0; j < K; ++j) w[j] = a.w[c * K + j];
    const float bv = (a.flags & kHasBias) ? a.bias[c] : 0.0f;
    float z[TAPS + E];
    load_run<T, 1, E, false>(xr, t0, L, z + TAPS);
#pragma unroll
    for (int i = 0; i < TAPS; ++i) {
        const float up = __shfl_up_sync(0xffffffffu, z[E + i], 1);
        z[i] = lane > 0 ? up : zval<T, TAPS>(xr, ir, t0 - TAPS + i, L);
    }
    float o[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
        float acc = bv;
#pragma unroll
        for (int j = 0; j < K; ++j) acc = fmaf(w[j], z[i + j], acc);
        o[i] = (a.flags & kSilu) ? silu_t<T>(acc) : acc;
    }
    if (t0 < L) store_run<T, 1, E, false>(static_cast<T*>(a.out) + row * L, t0, L, o);
    if (a.final_state != nullptr && seg == 0 && lane == 0) {
        T* fr = static_cast<T*>(a.final_state) + row * TAPS;
#pragma unroll
        for (int i = 0; i < TAPS; ++i) stf(fr + i, zval<T, TAPS>(xr, ir, L - TAPS + i, L));
    }
}

template <typename T, int K>
__global__ void __launch_bounds__(kThreads)
bwd_plain_kernel(const Args a) {
    constexpr int TAPS = K - 1, E = 16, NG = E + TAPS;
    const int lane = threadIdx.x & 31;
    const int64_t it = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
    if (it >= a.rows * a.nchunks) return;        // warp-uniform
    const int64_t L = a.length;
    int64_t row, seg, c;
    item_coords(a, it, row, seg, c);
    const int64_t t0 = seg * kSeg + (int64_t)lane * E;
    const T* xr = static_cast<const T*>(a.x) + row * L;
    const T* dr = static_cast<const T*>(a.dout) + row * L;
    const T* ir = (a.flags & kHasInit) ? static_cast<const T*>(a.init) + row * TAPS : nullptr;
    float w[K];
#pragma unroll
    for (int j = 0; j < K; ++j) w[j] = a.w[c * K + j];
    const float bv = (a.flags & kHasBias) ? a.bias[c] : 0.0f;
    float z[NG + TAPS], g[NG];
    load_run<T, 1, E, false>(xr, t0, L, z + TAPS);
    load_run<T, 1, E, false>(dr, t0, L, g);
#pragma unroll
    for (int i = 0; i < TAPS; ++i) {
        const float up = __shfl_up_sync(0xffffffffu, z[E + i], 1);
        const float xdn = __shfl_down_sync(0xffffffffu, z[TAPS + i], 1);
        const float gdn = __shfl_down_sync(0xffffffffu, g[i], 1);
        z[i] = lane > 0 ? up : zval<T, TAPS>(xr, ir, t0 - TAPS + i, L);
        const int64_t q = t0 + E + i;
        z[TAPS + E + i] = lane < 31 ? xdn : zval<T, TAPS>(xr, ir, q, L);
        g[E + i] = lane < 31 ? gdn : (q < L ? ldf(dr + q) : 0.0f);
    }
    float dw[K + 1];
    float o[E];
    conv_bwd_lane<T, K, E>(w, bv, a.flags & kSilu, z, g, o, dw);
    if (t0 < L) store_run<T, 1, E, false>(static_cast<T*>(a.dx) + row * L, t0, L, o);
#pragma unroll
    for (int j = 0; j <= K; ++j) {
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) dw[j] += __shfl_xor_sync(0xffffffffu, dw[j], o2);
    }
    if (lane == 0) {
#pragma unroll
        for (int j = 0; j <= K; ++j) a.partial[it * (K + 1) + j] = dw[j];
    }
    if (TAPS > 0 && t0 == 0 && a.dinit != nullptr) dinit_row<T, K>(static_cast<T*>(a.dinit) + row * TAPS, w, g);
}

// ------------------------------------------------- bulk-copy pipeline path --
// Rows whose bytes are 16-byte aligned: persistent CTAs walk (row, tile of
// kTile elements) items through a ring of kStages shared-memory stages.  A
// stage holds the item's tile (x, and dout for the backward) with up to kHalo
// elements of halo either side, landed by bulk asynchronous copies that
// complete on the stage's mbarrier.  The warps of a CTA never wait for one
// another: each polls the stage's mbarrier itself (bounded), reads its part,
// and counts itself off the stage; the last of the CTA's warps to finish a
// stage issues the copy of the stage's next item.  A wait that runs out
// records an error code (ssm_take_kernel_error) and the warp stops; the CTA
// then drains the copies it issued.
//
// Items are numbered channel-major, it = (c * batch + b) * nchunks + tile, and
// each CTA walks one contiguous range of `per` of them, so that it passes
// through few channels: a warp keeps the channel's weights, and in the
// backward its dweight / dbias sums, in registers across the channel's items
// and reduces the sums once per run of a channel.
//
// Thread t owns the 8-element groups at 8 t and kTile/2 + 8 t of a tile (each
// warp-wide 16-byte access covers 512 contiguous bytes), carried as the two
// lanes of float2 arithmetic.  Weights and bias are halved (exact) so that the
// pre-activation comes out as a / 2, the form the paired SiLU takes.
constexpr int kTile = kThreads * 16;   // 4096 elements
constexpr int kHalf = kTile / 2;
constexpr int kHalo = 8;
constexpr int kStages = 3;
constexpr int kWarps = kThreads / 32;

__device__ int g_conv_error;

// A bounded wait ran out: record the code in the device's flag and in the
// call's status word; the first failure wins.
__device__ __forceinline__ void report(const Args& a, int code) {
    atomicCAS(&g_conv_error, 0, code);
    if (a.status) atomicCAS(a.status, 0, code);
}

template <typename T, int NT>
struct BulkLayout {
    static constexpr int SPAN = kHalo + kTile + kHalo;             // elements per stage and tensor
    static constexpr size_t stage_bytes = (size_t)SPAN * sizeof(T) * NT;
    static constexpr size_t mbar_off = stage_bytes * kStages;      // kStages mbarriers
    static constexpr size_t done_off = mbar_off + 8 * kStages;     // kStages warp counters
    static constexpr size_t issued_off = done_off + 4 * kStages;   // kStages copies issued
    static constexpr size_t bytes = issued_off + 4 * kStages;
};

// A bulk item's (channel, batch, tile), stepped without divisions.  The host
// keeps rows * nchunks below 2^31.
struct Cursor {
    uint32_t c, b, tile;
    __device__ void set(const Args& a, int64_t it) {
        const uint32_t i = (uint32_t)it, nc = (uint32_t)a.nchunks, pc = (uint32_t)(a.batch * a.nchunks);
        c = i / pc;
        const uint32_t r = i - c * pc;
        b = r / nc;
        tile = r - b * nc;
    }
    __device__ void next(const Args& a) {
        if (++tile == (uint32_t)a.nchunks) {
            tile = 0;
            if (++b == (uint32_t)a.batch) { b = 0; ++c; }
        }
    }
    __device__ int64_t row(const Args& a) const { return (int64_t)b * a.channels + c; }
    __device__ int64_t t0() const { return (int64_t)tile * kTile; }
};

// Copy the item at `q` into stage `st`: elements [t0 - front, t0 + n + back)
// of the row land at stage offset kHalo - front.
template <typename T, int NT>
__device__ __forceinline__ void issue_tile(const Args& a, unsigned char* smem, int st, const Cursor& q,
                                           const void* s0, const void* s1) {
    using Lay = BulkLayout<T, NT>;
    const int64_t L = a.length, row = q.row(a), t0 = q.t0();
    const int64_t n = min64(kTile, L - t0);
    const int front = t0 >= kHalo ? kHalo : 0;
    const int back = NT > 1 ? (int)min64(kHalo, L - t0 - n) : 0;
    const uint32_t bytes = (uint32_t)((front + n + back) * sizeof(T));
    const uint32_t mbar = tc::smem_u32(smem + Lay::mbar_off + 8 * st);
    tc::mbar_expect_tx(mbar, bytes * NT);
    const void* src[2] = {s0, s1};
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        const T* g = static_cast<const T*>(src[k]) + row * L + t0 - front;
        unsigned char* dst = smem + st * Lay::stage_bytes + (size_t)k * Lay::SPAN * sizeof(T) +
                             (size_t)(kHalo - front) * sizeof(T);
        tc::bulk_load(tc::smem_u32(dst), g, bytes, mbar);
    }
    reinterpret_cast<int*>(smem + Lay::issued_off)[st] += 1;
}

// The stage ring of one CTA, whose items are [first, first + count).
template <typename T, int NT>
struct Ring {
    unsigned char* smem;
    int64_t first;
    int count;
    __device__ uint32_t mbar(int st) const { return tc::smem_u32(smem + BulkLayout<T, NT>::mbar_off + 8 * st); }
    __device__ void init(const Args& a, const void* s0, const void* s1) const {
        if (threadIdx.x == 0) {
            for (int s = 0; s < kStages; ++s) {
                tc::mbar_init(mbar(s), 1);
                reinterpret_cast<int*>(smem + BulkLayout<T, NT>::done_off)[s] = 0;
                reinterpret_cast<int*>(smem + BulkLayout<T, NT>::issued_off)[s] = 0;
            }
            tc::fence_mbar_init();
            Cursor q;
            q.set(a, first);
            for (int s = 0; s < kStages && s < count; ++s, q.next(a)) issue_tile<T, NT>(a, smem, s, q, s0, s1);
        }
        __syncthreads();
    }
    // every lane polls; warp-uniform result
    __device__ bool wait(int st, int use) const {
        const bool ok = tc::mbar_wait(mbar(st), (uint32_t)(use & 1));
        return __all_sync(0xffffffffu, ok);
    }
    // The calling warp is done reading stage `st` for its k-th item (the
    // stage's use-th); the CTA's last warp to get here issues the item
    // kStages further on, at `ahead`.
    __device__ void release(const Args& a, int st, int use, int k, const Cursor& ahead, const void* s0,
                            const void* s1) const {
        __syncwarp();
        if ((threadIdx.x & 31) == 0) {
            int* done = reinterpret_cast<int*>(smem + BulkLayout<T, NT>::done_off) + st;
            __threadfence_block();
            const int prev = atomicAdd(done, 1);
            if (prev == (use + 1) * kWarps - 1) {
                __threadfence_block();
                if (k + kStages < count) issue_tile<T, NT>(a, smem, st, ahead, s0, s1);
            }
        }
    }
    // After every warp has left its loop: wait (bounded) for the last copy
    // issued into each stage, so that none lands after the CTA exits.
    __device__ void drain() const {
        __syncthreads();
        if (threadIdx.x == 0)
            for (int s = 0; s < kStages; ++s) {
                const int m = reinterpret_cast<const int*>(smem + BulkLayout<T, NT>::issued_off)[s];
                if (m > 0) tc::mbar_wait(mbar(s), (uint32_t)((m - 1) & 1));
            }
    }
};

// v[i] = x at tile position p - 8 + i for i < 16 (the 8 elements before group p
// and the group), zero at or past n.  s points at tile position 0 of a stage
// (16-byte aligned, kHalo elements of front halo); p is a multiple of 8.
template <typename T>
__device__ __forceinline__ void load_span(const T* s, int p, int n, float* v) {
    if (p + 8 <= n) {
        Vec<T, 8>::ld(s + p - 8, v);
        Vec<T, 8>::ld(s + p, v + 8);
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = p - 8 + i < n ? ldf(s + p - 8 + i) : 0.0f;
    }
}
// The thread's two groups at p0 (lane .x) and p1 (lane .y): z[m] = x at
// p - TAPS + m for m < TAPS + 8.  Positions left of a row start are garbage
// here; the caller replaces them (they are read by thread 0 only).
template <typename T, int TAPS>
__device__ __forceinline__ void load_x_pair(const T* s, int p0, int p1, int n, float2* z) {
    float a[16], b[16];
    load_span<T>(s, p0, n, a);
    load_span<T>(s, p1, n, b);
#pragma unroll
    for (int m = 0; m < TAPS + 8; ++m) z[m] = make_float2(a[8 - TAPS + m], b[8 - TAPS + m]);
}
// g[i] = s at p + i for i < 8 (zero at or past n), both groups.
template <typename T>
__device__ __forceinline__ void load_pair8(const T* s, int p0, int p1, int n, float2* g) {
    float a[8], b[8];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int p = u ? p1 : p0;
        float* v = u ? b : a;
        if (p + 8 <= n) Vec<T, 8>::ld(s + p, v);
        else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = p + i < n ? ldf(s + p + i) : 0.0f;
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) g[i] = make_float2(a[i], b[i]);
}
template <typename T>
__device__ __forceinline__ void store_pair8(T* r, int p0, int p1, int n, const float2* o) {
    float a[8], b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) { a[i] = o[i].x; b[i] = o[i].y; }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int p = u ? p1 : p0;
        const float* v = u ? b : a;
        if (p + 8 <= n) Vec<T, 8>::st(r + p, v);
        else {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (p + i < n) stf(r + p + i, v[i]);
        }
    }
}

// A channel's halved weights and bias.
template <int K>
struct ChannelConst {
    float2 wh[K], bh;
    __device__ void load(const Args& a, uint32_t c) {
#pragma unroll
        for (int j = 0; j < K; ++j) wh[j] = f2(0.5f * a.w[(int64_t)c * K + j]);
        bh = f2((a.flags & kHasBias) ? 0.5f * a.bias[c] : 0.0f);
    }
};

// Thread 0 of a row-start item: the taps elements left of position 0 (the
// initial state, or zeros), loaded before the stage wait and put in place of
// the stage's unwritten front halo.
template <typename T, int TAPS>
struct RowStart {
    float v[TAPS > 0 ? TAPS : 1];
    __device__ void load(const Args& a, int64_t row, int64_t t0) {
        if (TAPS > 0 && t0 == 0 && threadIdx.x == 0) {
            const T* ir = (a.flags & kHasInit) ? static_cast<const T*>(a.init) + row * TAPS : nullptr;
#pragma unroll
            for (int i = 0; i < TAPS; ++i) v[i] = ir ? ldf(ir + i) : 0.0f;
        }
    }
    __device__ void apply(float2* z, int64_t t0) const {
        if (TAPS > 0 && t0 == 0 && threadIdx.x == 0) {
#pragma unroll
            for (int i = 0; i < TAPS; ++i) z[i].x = v[i];
        }
    }
};

template <typename T, int K>
__global__ void __launch_bounds__(kThreads)
fwd_bulk_kernel(const Args a) {
    constexpr int TAPS = K - 1;
    using Lay = BulkLayout<T, 1>;
    extern __shared__ __align__(128) unsigned char smem[];
    const int64_t items = a.rows * a.nchunks, L = a.length;
    const int64_t first = (int64_t)blockIdx.x * a.per;
    const Ring<T, 1> ring{smem, first, (int)max64(0, min64(a.per, items - first))};
    const int tid = threadIdx.x;
    ring.init(a, a.x, nullptr);
    const bool silu = a.flags & kSilu;
    const int p0 = tid * 8, p1 = kHalf + tid * 8;
    Cursor cur, ahead;
    cur.set(a, first);
    ahead.set(a, first + kStages);
    ChannelConst<K> cc;
    uint32_t wc = 0xffffffffu;
    int st = 0, use = 0;
    for (int k = 0; k < ring.count; ++k) {
        const int64_t row = cur.row(a), t0 = cur.t0();
        const int n = (int)min64(kTile, L - t0);
        if (cur.c != wc) {
            cc.load(a, cur.c);
            wc = cur.c;
        }
        RowStart<T, TAPS> rs;
        rs.load(a, row, t0);
        if (!ring.wait(st, use)) {
            if ((tid & 31) == 0) report(a, 61);
            break;
        }
        const T* xs = reinterpret_cast<const T*>(smem + st * Lay::stage_bytes) + kHalo;
        float2 z[TAPS + 8], o[8];
        load_x_pair<T, TAPS>(xs, p0, p1, n, z);
        ring.release(a, st, use, k, ahead, a.x, nullptr);
        rs.apply(z, t0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float2 hp = cc.bh;
#pragma unroll
            for (int j = 0; j < K; ++j) hp = fma2(cc.wh[j], z[i + j], hp);
            o[i] = silu ? silu2_half<T>(hp) : add2(hp, hp);
        }
        store_pair8<T>(static_cast<T*>(a.out) + row * L + t0, p0, p1, n, o);
        if (a.final_state != nullptr && t0 == 0 && tid == 0) {
            const T* xr = static_cast<const T*>(a.x) + row * L;
            const T* ir = (a.flags & kHasInit) ? static_cast<const T*>(a.init) + row * TAPS : nullptr;
            T* fr = static_cast<T*>(a.final_state) + row * TAPS;
#pragma unroll
            for (int i = 0; i < TAPS; ++i) stf(fr + i, zval<T, TAPS>(xr, ir, L - TAPS + i, L));
        }
        cur.next(a);
        ahead.next(a);
        if (++st == kStages) { st = 0; ++use; }
    }
    ring.drain();
}

// 2 dout silu'(pre) (or 2 dout without the activation) at tile positions q0
// (.x) and q1 (.y), read one by one from the stage; positions at or past
// `lim` give 0.  For the warp-boundary halo of the backward.
template <typename T, int K>
__device__ __forceinline__ float2 grad2_at(const T* xs, const T* ds, int q0, int q1, int lim, bool silu,
                                           const ChannelConst<K>& cc) {
    const bool v0 = q0 < lim, v1 = q1 < lim;
    const float2 d = make_float2(v0 ? ldf(ds + q0) : 0.0f, v1 ? ldf(ds + q1) : 0.0f);
    if (!silu) return add2(d, d);
    float2 hp = cc.bh;
#pragma unroll
    for (int j = 0; j < K; ++j) {
        const int o = j - (K - 1);
        hp = fma2(cc.wh[j], make_float2(v0 ? ldf(xs + q0 + o) : 0.0f, v1 ? ldf(xs + q1 + o) : 0.0f), hp);
    }
    return silu_grad2_half<T>(hp, d);
}

// One warp's dweight / dbias sums of a channel run (doubled, both lanes) into
// the partial slot of (run's first item, warp).
template <int K>
__device__ __forceinline__ void flush_run(const Args& a, int64_t run0, float2* acc) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* part = a.partial + (run0 * kWarps + warp) * (K + 1);
#pragma unroll
    for (int j = 0; j <= K; ++j) {
        float d = 0.5f * (acc[j].x + acc[j].y);
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o2);
        if (lane == 0) part[j] = d;
        acc[j] = f2(0.0f);
    }
}

// Backward over one stage, in the forward's thread layout and paired lanes.
// Phase 1 turns dout into the doubled gradient 2 g = 2 dout silu'(pre) of the
// thread's positions.  Each lane needs the taps positions right of its groups:
// the next lane's first ones (a shuffle) or, for lane 31, the positions after
// the warp's 256-element runs, which belong to the next warp, to the tile's
// second half or (last warp) to the next tile; lanes 32 - taps .. 31 compute
// those from the stage (zero past the row) and lane 31 takes them by shuffle.
// Phase 2 forms dx = sum_j (w_j / 2)(2 g) and accumulates the dweight / dbias
// products of the channel run.
template <typename T, int K>
__global__ void __launch_bounds__(kThreads)
bwd_bulk_kernel(const Args a) {
    constexpr int TAPS = K - 1;
    using Lay = BulkLayout<T, 2>;
    extern __shared__ __align__(128) unsigned char smem[];
    const int64_t items = a.rows * a.nchunks, L = a.length;
    const int64_t first = (int64_t)blockIdx.x * a.per;
    const Ring<T, 2> ring{smem, first, (int)max64(0, min64(a.per, items - first))};
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    ring.init(a, a.x, a.dout);
    const bool silu = a.flags & kSilu;
    const int p0 = tid * 8, p1 = kHalf + tid * 8;
    Cursor cur, ahead;
    cur.set(a, first);
    ahead.set(a, first + kStages);
    ChannelConst<K> cc;
    uint32_t wc = 0xffffffffu;
    int64_t run0 = first;
    float2 acc[K + 1];
#pragma unroll
    for (int j = 0; j <= K; ++j) acc[j] = f2(0.0f);
    int st = 0, use = 0;
    bool ok = true;
    for (int k = 0; k < ring.count; ++k) {
        const int64_t row = cur.row(a), t0 = cur.t0();
        const int n = (int)min64(kTile, L - t0);
        if (cur.c != wc) {
            if (k > 0) flush_run<K>(a, run0, acc);
            run0 = first + k;
            cc.load(a, cur.c);
            wc = cur.c;
        }
        RowStart<T, TAPS> rs;
        rs.load(a, row, t0);
        if (!ring.wait(st, use)) {
            if (lane == 0) report(a, 62);
            ok = false;
            break;
        }
        const T* xs = reinterpret_cast<const T*>(smem + st * Lay::stage_bytes) + kHalo;
        const T* ds = xs + Lay::SPAN;
        float2 z[TAPS + 8], g[8 + TAPS];
        load_x_pair<T, TAPS>(xs, p0, p1, n, z);
        load_pair8<T>(ds, p0, p1, n, g);
        float2 ex = f2(0.0f);                     // lane 32 - taps + i: right halo position i of the warp
        if (TAPS > 0 && lane >= 32 - TAPS) {
            // positions valid in the stage: the tile and, for a full tile, its
            // back halo up to the row's end
            const int lim = n + (int)min64(kHalo, L - t0 - n);
            const int q = 256 * (warp + 1) + lane - (32 - TAPS);
            ex = grad2_at<T, K>(xs, ds, q, kHalf + q, lim, silu, cc);
        }
        ring.release(a, st, use, k, ahead, a.x, a.dout);
        rs.apply(z, t0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (silu) {
                float2 hp = cc.bh;
#pragma unroll
                for (int j = 0; j < K; ++j) hp = fma2(cc.wh[j], z[i + j], hp);
                g[i] = silu_grad2_half<T>(hp, g[i]);
            } else {
                g[i] = add2(g[i], g[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < TAPS; ++i) {
            const float nx = __shfl_down_sync(0xffffffffu, g[i].x, 1), ny = __shfl_down_sync(0xffffffffu, g[i].y, 1);
            const float ax = __shfl_sync(0xffffffffu, ex.x, 32 - TAPS + i);
            const float ay = __shfl_sync(0xffffffffu, ex.y, 32 - TAPS + i);
            g[8 + i] = lane == 31 ? make_float2(ax, ay) : make_float2(nx, ny);
        }
        float2 o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float2 s = mul2(cc.wh[0], g[i + TAPS]);
#pragma unroll
            for (int j = 1; j < K; ++j) s = fma2(cc.wh[j], g[i + TAPS - j], s);
            o[i] = s;
        }
        store_pair8<T>(static_cast<T*>(a.dx) + row * L + t0, p0, p1, n, o);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            acc[K] = add2(acc[K], g[i]);
#pragma unroll
            for (int j = 0; j < K; ++j) acc[j] = fma2(g[i], z[i + j], acc[j]);
        }
        if (TAPS > 0 && t0 == 0 && tid == 0 && a.dinit != nullptr) {
            T* dir = static_cast<T*>(a.dinit) + row * TAPS;
#pragma unroll
            for (int p = 0; p < TAPS; ++p) {
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j <= p; ++j) s = fmaf(cc.wh[j].x, g[p - j].x, s);
                stf(dir + p, s);
            }
        }
        cur.next(a);
        ahead.next(a);
        if (++st == kStages) { st = 0; ++use; }
    }
    if (ok && ring.count > 0) flush_run<K>(a, run0, acc);
    ring.drain();
}

// dweight[c, j] and dbias[c]: partials of every (batch, chunk, slot) of channel
// c, summed in a fixed order.
template <int K>
__global__ void finalize_kernel(const Args a, float* dweight, float* dbias) {
    const int64_t total = a.channels * (K + 1);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = i / (K + 1);
        const int j = (int)(i - c * (K + 1));
        float s = 0.0f;
        for (int64_t b = 0; b < a.batch; ++b) {
            const int64_t m = a.nchunks * a.slots;
            const float* p = a.partial + ((b * a.channels + c) * m) * (K + 1) + j;
            for (int64_t k = 0; k < m; ++k) s += p[k * (K + 1)];
        }
        if (j < K) {
            if (dweight) dweight[c * K + j] = s;
        } else if (dbias) {
            dbias[c] = s;
        }
    }
}

// dweight / dbias of the bulk path: channel c's items [c B', (c + 1) B')
// (B' = batch * nchunks) fall into the ranges [k per, (k + 1) per) of one or
// more CTAs; each such run left one partial per warp at its first item.
// Summed in a fixed order.
template <int K>
__global__ void finalize_runs_kernel(const Args a, float* dweight, float* dbias) {
    const int64_t total = a.channels * (K + 1), bp = a.batch * a.nchunks;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = i / (K + 1);
        const int j = (int)(i - c * (K + 1));
        float s = 0.0f;
        for (int64_t r = c * bp; r < (c + 1) * bp; r = (r / a.per + 1) * a.per) {
#pragma unroll
            for (int w = 0; w < kWarps; ++w) s += a.partial[(r * kWarps + w) * (K + 1) + j];
        }
        if (j < K) {
            if (dweight) dweight[c * K + j] = s;
        } else if (dbias) {
            dbias[c] = s;
        }
    }
}

// ------------------------------------------------------- channel-last path --
// x, out, dout and dx stored (batch, length, channels) -- the layout a
// Mamba block's input projection produces, where the (batch, channels,
// length) operand is a transposed view: element (b, c, t) at
// (b length + t) rs + c, with rs the row stride (x and dout may be column
// slices of wider rows; out and dx are written densely).  A thread owns V
// consecutive channels (one 8-byte vector per row) and a run of kRun steps,
// which it walks in order with the taps-wide window of earlier rows in a ring
// of registers, so each row is read once (plus the taps rows before the run);
// a warp's 32 vectors are 256 contiguous bytes of a row.  A CTA is 32 lanes
// (32 V channels) x 8 warps (8 consecutive runs).  The ring slots are
// compile-time indices: the step loop is unrolled by K, and row t sits in slot
// (t - t_begin) mod K.
constexpr int kRun = 64;
constexpr int kClWarps = kThreads / 32;

template <typename T>
struct ClVec {
    static constexpr int V = 8 / (int)sizeof(T);   // channels per thread
    static constexpr int M = V / 2;                // channel pairs
    static __device__ __forceinline__ void ld(const T* p, float2* v) {
        const uint2 q = *reinterpret_cast<const uint2*>(p);
        if constexpr (sizeof(T) == 4) {
            v[0] = make_float2(__uint_as_float(q.x), __uint_as_float(q.y));
        } else {
            v[0] = Io2<T>::ld(reinterpret_cast<const T*>(&q.x));
            v[1] = Io2<T>::ld(reinterpret_cast<const T*>(&q.y));
        }
    }
    static __device__ __forceinline__ void from_raw(uint2 q, float2* v) {
        if constexpr (sizeof(T) == 4) {
            v[0] = make_float2(__uint_as_float(q.x), __uint_as_float(q.y));
        } else {
            v[0] = Io2<T>::ld(reinterpret_cast<const T*>(&q.x));
            v[1] = Io2<T>::ld(reinterpret_cast<const T*>(&q.y));
        }
    }
    static __device__ __forceinline__ void st(T* p, const float2* v) {
        uint2 q;
        if constexpr (sizeof(T) == 4) {
            q = make_uint2(__float_as_uint(v[0].x), __float_as_uint(v[0].y));
        } else {
            Io2<T>::st(reinterpret_cast<T*>(&q.x), v[0]);
            Io2<T>::st(reinterpret_cast<T*>(&q.y), v[1]);
        }
        *reinterpret_cast<uint2*>(p) = q;
    }
};

// Halved weights and bias of the thread's channel pairs.
template <typename T, int K>
__device__ __forceinline__ void cl_weights(const Args& a, int64_t c0, float2 (&wh)[K][ClVec<T>::M],
                                           float2 (&bh)[ClVec<T>::M]) {
#pragma unroll
    for (int m = 0; m < ClVec<T>::M; ++m) {
        const int64_t c = c0 + 2 * m;
#pragma unroll
        for (int j = 0; j < K; ++j) wh[j][m] = make_float2(0.5f * a.w[c * K + j], 0.5f * a.w[(c + 1) * K + j]);
        bh[m] = (a.flags & kHasBias) ? make_float2(0.5f * a.bias[c], 0.5f * a.bias[c + 1]) : f2(0.0f);
    }
}

// Each thread streams its rows through a private ring of kClDepth slots in
// shared memory, filled by 8-byte asynchronous copies issued kClDepth rows
// ahead of use (one commit group per row), so many rows are in flight
// without registers; a thread reads back only what it copied itself.
constexpr int kClDepth = 16;

template <typename T, int K>
__global__ void __launch_bounds__(kThreads)
fwd_cl_kernel(const Args a) {
    constexpr int M = ClVec<T>::M, V = ClVec<T>::V;
    extern __shared__ __align__(16) uint2 cl_stage[];       // [kClDepth][kThreads]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t c0 = ((int64_t)blockIdx.x * 32 + lane) * V;
    const int64_t b = blockIdx.z, L = a.length;
    const int64_t t_begin = ((int64_t)blockIdx.y * kClWarps + warp) * kRun;
    if (c0 >= a.channels || t_begin >= L) return;
    const int64_t t_end = min64(t_begin + kRun, L);
    const T* x = static_cast<const T*>(a.x) + b * L * a.xs + c0;
    T* out = static_cast<T*>(a.out) + b * L * a.channels + c0;
    auto slot = [&](int64_t t) { return tc::smem_u32(&cl_stage[(int)((t - t_begin) % kClDepth) * kThreads + tid]); };
#pragma unroll
    for (int i = 0; i < kClDepth; ++i) {
        if (t_begin + i < t_end) tc::cp_async8(slot(t_begin + i), x + (t_begin + i) * a.xs);
        tc::cp_async_commit();
    }
    float2 wh[K][M], bh[M];
    cl_weights<T, K>(a, c0, wh, bh);
    const bool silu = a.flags & kSilu;
    float2 ring[K][M];
#pragma unroll
    for (int i = 1; i < K; ++i) {          // rows t_begin - K + i in slot i
        const int64_t t = t_begin - K + i;
        if (t >= 0) ClVec<T>::ld(x + t * a.xs, ring[i]);
        else {
#pragma unroll
            for (int m = 0; m < M; ++m) ring[i][m] = f2(0.0f);
        }
    }
    for (int64_t t0 = t_begin; t0 < t_end; t0 += K) {
#pragma unroll
        for (int u = 0; u < K; ++u) {       // row t0 + u in slot u
            const int64_t t = t0 + u;
            if (t >= t_end) break;
            tc::cp_async_wait<kClDepth - 1>();
            const uint2 q = cl_stage[(int)((t - t_begin) % kClDepth) * kThreads + tid];
            ClVec<T>::from_raw(q, ring[u]);
            // refill the slot just read (its value is in registers now)
            if (t + kClDepth < t_end) tc::cp_async8(slot(t), x + (t + kClDepth) * a.xs);
            tc::cp_async_commit();
            float2 o[M];
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float2 hp = bh[m];
#pragma unroll
                for (int j = 0; j < K; ++j) hp = fma2(wh[j][m], ring[(u + 1 + j) % K][m], hp);   // row t - taps + j
                o[m] = silu ? silu2_half<T>(hp) : add2(hp, hp);
            }
            ClVec<T>::st(out + t * a.channels, o);
        }
    }
    tc::cp_async_wait<0>();
}

// Backward: for u = t_begin .. t_end + taps - 1 the thread forms the doubled
// gradient g(u) = 2 dout(u) silu'(pre(u)) (0 past the row) from the x ring
// (rows u - taps .. u) and keeps it in a ring of its own; dx(u - taps) =
// sum_j (w_j / 2) g(u - j) once u - taps >= t_begin, and the dweight / dbias
// products of the run's own steps.  x and dout rows stream through the
// thread's shared-memory ring like the forward's.  The CTA's warps add their
// sums in a fixed order (in the ring's space, after the loop) into one
// partial per (batch, CTA row block, channel).
template <typename T, int K>
__global__ void __launch_bounds__(kThreads, K <= 4 ? 2 : 1)
bwd_cl_kernel(const Args a) {
    constexpr int M = ClVec<T>::M, V = ClVec<T>::V, TAPS = K - 1;
    extern __shared__ __align__(16) uint2 cl_stage[];       // [kClDepth][2][kThreads]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t c0 = ((int64_t)blockIdx.x * 32 + lane) * V;
    const int64_t b = blockIdx.z, L = a.length;
    const int64_t t_begin = ((int64_t)blockIdx.y * kClWarps + warp) * kRun;
    const bool live = c0 < a.channels && t_begin < L;
    float2 acc[K + 1][M];
#pragma unroll
    for (int j = 0; j <= K; ++j)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[j][m] = f2(0.0f);
    if (live) {
        const int64_t t_end = min64(t_begin + kRun, L);
        const int64_t u_end = t_end + TAPS, u_load = min64(u_end, L);   // rows staged: [t_begin, u_load)
        const T* x = static_cast<const T*>(a.x) + b * L * a.xs + c0;
        const T* dout = static_cast<const T*>(a.dout) + b * L * a.ds + c0;
        T* dx = static_cast<T*>(a.dx) + b * L * a.channels + c0;
        auto sidx = [&](int64_t u, int k) { return ((int)((u - t_begin) % kClDepth) * 2 + k) * kThreads + tid; };
        auto issue = [&](int64_t u) {
            tc::cp_async8(tc::smem_u32(&cl_stage[sidx(u, 0)]), x + u * a.xs);
            tc::cp_async8(tc::smem_u32(&cl_stage[sidx(u, 1)]), dout + u * a.ds);
        };
#pragma unroll
        for (int i = 0; i < kClDepth; ++i) {
            if (t_begin + i < u_load) issue(t_begin + i);
            tc::cp_async_commit();
        }
        float2 wh[K][M], bh[M];
        cl_weights<T, K>(a, c0, wh, bh);
        const bool silu = a.flags & kSilu;
        float2 xr[K][M], gr[K][M];
#pragma unroll
        for (int i = 1; i < K; ++i) {
            const int64_t t = t_begin - K + i;
            if (t >= 0) ClVec<T>::ld(x + t * a.xs, xr[i]);
            else {
#pragma unroll
                for (int m = 0; m < M; ++m) xr[i][m] = f2(0.0f);
            }
#pragma unroll
            for (int m = 0; m < M; ++m) gr[i][m] = f2(0.0f);   // g before the run: unused
        }
        for (int64_t u0 = t_begin; u0 < u_end; u0 += K) {
#pragma unroll
            for (int k = 0; k < K; ++k) {   // step u = u0 + k in slot k
                const int64_t u = u0 + k;
                if (u >= u_end) break;
                float2 g[M];
                tc::cp_async_wait<kClDepth - 1>();
                if (u < L) {
                    ClVec<T>::from_raw(cl_stage[sidx(u, 0)], xr[k]);
                    ClVec<T>::from_raw(cl_stage[sidx(u, 1)], g);
                    if (u + kClDepth < u_load) issue(u + kClDepth);
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        if (silu) {
                            float2 hp = bh[m];
#pragma unroll
                            for (int j = 0; j < K; ++j) hp = fma2(wh[j][m], xr[(k + 1 + j) % K][m], hp);
                            g[m] = silu_grad2_half<T>(hp, g[m]);
                        } else {
                            g[m] = add2(g[m], g[m]);
                        }
                    }
                } else {
#pragma unroll
                    for (int m = 0; m < M; ++m) { g[m] = f2(0.0f); xr[k][m] = f2(0.0f); }
                }
                tc::cp_async_commit();
#pragma unroll
                for (int m = 0; m < M; ++m) gr[k][m] = g[m];
                if (u < t_end) {
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        acc[K][m] = add2(acc[K][m], g[m]);
#pragma unroll
                        for (int j = 0; j < K; ++j) acc[j][m] = fma2(g[m], xr[(k + 1 + j) % K][m], acc[j][m]);
                    }
                }
                if (u - TAPS >= t_begin) {
                    float2 o[M];
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        float2 s = mul2(wh[0][m], gr[k][m]);            // j = 0: g(u)
#pragma unroll
                        for (int j = 1; j < K; ++j) s = fma2(wh[j][m], gr[(k + K - j) % K][m], s);
                        o[m] = s;
                    }
                    ClVec<T>::st(dx + (u - TAPS) * a.channels, o);
                }
            }
        }
        tc::cp_async_wait<0>();
    }
    __syncthreads();                               // every ring is idle: its space takes the fold
    float* red = reinterpret_cast<float*>(cl_stage);   // [kClWarps][32 V][K + 1]
    constexpr int RW = 32 * V * (K + 1);
#pragma unroll
    for (int j = 0; j <= K; ++j)
#pragma unroll
        for (int m = 0; m < M; ++m) {
            red[warp * RW + (lane * V + 2 * m) * (K + 1) + j] = 0.5f * acc[j][m].x;
            red[warp * RW + (lane * V + 2 * m + 1) * (K + 1) + j] = 0.5f * acc[j][m].y;
        }
    __syncthreads();
    const int64_t nrb = (L + kClWarps * kRun - 1) / (kClWarps * kRun);
    float* part = a.partial + ((b * nrb + blockIdx.y) * a.channels + (int64_t)blockIdx.x * 32 * V) * (K + 1);
    for (int i = threadIdx.x; i < RW; i += kThreads) {
        const int cl = i / (K + 1);
        if ((int64_t)blockIdx.x * 32 * V + cl >= a.channels) continue;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kClWarps; ++w) s += red[w * RW + i];
        part[i] = s;
    }
}

// dweight / dbias of the channel-last backward: the partials of every
// (batch, row block) of channel c, in order.
template <int K>
__global__ void finalize_cl_kernel(const Args a, float* dweight, float* dbias) {
    const int64_t total = a.channels * (K + 1);
    const int64_t nrb = (a.length + kClWarps * kRun - 1) / (kClWarps * kRun);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        float s = 0.0f;
        for (int64_t k = 0; k < a.batch * nrb; ++k) s += a.partial[k * total + i];
        const int64_t c = i / (K + 1);
        const int j = (int)(i - c * (K + 1));
        if (j < K) {
            if (dweight) dweight[c * K + j] = s;
        } else if (dbias) {
            dbias[c] = s;
        }
    }
}

// ------------------------------------------------------------------- decode --
// One thread per (batch, channel): q new tokens against a rolling state of
// `span` >= taps columns addressed through its strides (a cache slice), then
// state <- cat(state, x)[..., -span:] in place, ascending so that every read of
// state[i + q] still sees the old value.
template <typename T, int K>
__global__ void update_kernel(T* state, const T* x, const float* wts, const float* bias, T* y,
                              int64_t channels, int64_t q, int64_t span, int64_t rows,
                              int64_t stride_b, int64_t stride_c, uint32_t flags) {
    constexpr int TAPS = K - 1;
    const int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const int64_t c = r % channels;
    T* st = state + (r / channels) * stride_b + c * stride_c;
    const T* xr = x + r * q;
    T* yr = y + r * q;
    float w[K];
#pragma unroll
    for (int j = 0; j < K; ++j) w[j] = wts[c * K + j];
    const float bv = (flags & kHasBias) ? bias[c] : 0.0f;
    const bool silu = flags & kSilu;
    for (int64_t t = 0; t < q; ++t) {
        float acc = bv;
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const int64_t p = span - TAPS + t + j;   // index into cat(state, x)
            acc = fmaf(w[j], p < span ? ldf(st + p) : ldf(xr + (p - span)), acc);
        }
        stf(yr + t, silu ? silu_t<T>(acc) : acc);
    }
    for (int64_t i = 0; i < span; ++i) {
        const int64_t src = i + q;
        const float v = src < span ? ldf(st + src) : ldf(xr + (src - span));
        stf(st + i, v);
    }
}

// ------------------------------------------------------------------- host ----
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int validate(const ssm_causal_conv1d_params* p) {
    if (p == nullptr) return fail(SSM_ERR_INVALID, "causal_conv1d: null params");
    if (p->batch < 0 || p->channels < 0 || p->length < 0)
        return fail(SSM_ERR_INVALID, "causal_conv1d: negative extent");
    if (p->width < 1 || p->width > kMaxWidth)
        return fail(SSM_ERR_UNSUPPORTED, "causal_conv1d: kernel width must be 1..8");
    if (p->dtype < SSM_F32 || p->dtype > SSM_F16) return fail(SSM_ERR_UNSUPPORTED, "causal_conv1d: dtype");
    if (p->batch * p->channels * ceil_div(max64(p->length, 1), kSeg) >= ((int64_t)1 << 31))
        return fail(SSM_ERR_UNSUPPORTED, "causal_conv1d: batch * channels * length too large");
    return SSM_OK;
}

// Rows of 16-byte aligned bytes take the bulk-copy path (items are kTile
// tiles); the rest the plain path (items are kSeg segments).
static bool bulk_ok(const ssm_causal_conv1d_params* p, bool bwd) {
    const int64_t esz = p->dtype == SSM_F32 ? 4 : 2;
    if ((p->length * esz) % 16 != 0 || !aligned16(p->x)) return false;
    return !bwd || aligned16(p->dout);
}

static void plan(const ssm_causal_conv1d_params* p, bool bulk, Args& a) {
    a.batch = p->batch;
    a.channels = p->channels;
    a.length = p->length;
    a.rows = p->batch * p->channels;
    a.chunk = bulk ? kTile : kSeg;
    a.nchunks = max64(1, ceil_div(p->length, a.chunk));
    a.slots = bulk ? kWarps : 1;
    a.xs = p->x_row_stride ? p->x_row_stride : p->channels;
    a.ds = p->dout_row_stride ? p->dout_row_stride : p->channels;
    a.flags = p->flags;
    a.x = p->x; a.w = p->weight; a.bias = p->bias; a.init = p->initial_state;
    a.out = p->out; a.final_state = p->final_state;
    a.dout = p->dout; a.dx = p->dx; a.dinit = p->dinitial;
    a.partial = nullptr;
    a.per = 0;
    a.status = p->status;
}

// Persistent grid: resident CTAs of the kernel on every SM, at most one per
// item; sets a.per, the items of each CTA's contiguous range.
template <typename F>
static unsigned persistent_grid(F kernel, size_t smem, Args& a) {
    int dev = 0, sms = 148, per = 1;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, kThreads, smem) != cudaSuccess || per < 1) {
        cudaGetLastError();
        per = 1;
    }
    const int64_t items = a.rows * a.nchunks;
    const int64_t grid = max64(1, min64((int64_t)sms * per, items));
    a.per = ceil_div(items, grid);
    return (unsigned)ceil_div(items, a.per);
}

template <typename T, int K>
static int launch_fwd(Args a, bool bulk, cudaStream_t st) {
    if (bulk) {
        const size_t sm = BulkLayout<T, 1>::bytes;
        auto k = fwd_bulk_kernel<T, K>;
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
            return check_launch("causal_conv1d fwd: smem attribute");
        const unsigned grid = persistent_grid(k, sm, a);
        k<<<grid, kThreads, sm, st>>>(a);
    } else {
        fwd_plain_kernel<T, K><<<(unsigned)ceil_div(a.rows * a.nchunks, kThreads / 32), kThreads, 0, st>>>(a);
    }
    return check_launch("causal_conv1d fwd");
}

template <typename T, int K>
static int launch_bwd(Args a, bool bulk, float* dweight, float* dbias, cudaStream_t st) {
    if (bulk) {
        const size_t sm = BulkLayout<T, 2>::bytes;
        auto k = bwd_bulk_kernel<T, K>;
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
            return check_launch("causal_conv1d bwd: smem attribute");
        const unsigned grid = persistent_grid(k, sm, a);
        k<<<grid, kThreads, sm, st>>>(a);
    } else {
        bwd_plain_kernel<T, K><<<(unsigned)ceil_div(a.rows * a.nchunks, kThreads / 32), kThreads, 0, st>>>(a);
    }
    if (int s = check_launch("causal_conv1d bwd")) return s;
    const int64_t total = a.channels * (K + 1);
    const unsigned fgrid = (unsigned)min64(ceil_div(total, 256), 148 * 8);
    if (bulk) finalize_runs_kernel<K><<<fgrid, 256, 0, st>>>(a, dweight, dbias);
    else finalize_kernel<K><<<fgrid, 256, 0, st>>>(a, dweight, dbias);
    return check_launch("causal_conv1d bwd finalize");
}

template <typename T, int K>
static int launch_update(const ssm_causal_conv1d_update_params* p, cudaStream_t st) {
    const int64_t rows = p->batch * p->channels;
    update_kernel<T, K><<<(unsigned)ceil_div(rows, 128), 128, 0, st>>>(
        static_cast<T*>(p->state), static_cast<const T*>(p->x), p->weight, p->bias, static_cast<T*>(p->out),
        p->channels, p->length, p->state_len, rows, p->state_stride_batch, p->state_stride_channel, p->flags);
    return check_launch("causal_conv1d update");
}

// dispatch on (dtype, K)
template <template <typename, int> class F, typename... Ts>
static int by_type_width(int dtype, int K, Ts... args) {
#define SSM_CONV_K(T)                                              \
    switch (K) {                                                   \
        case 1: return F<T, 1>::run(args...);                      \
        case 2: return F<T, 2>::run(args...);                      \
        case 3: return F<T, 3>::run(args...);                      \
        case 4: return F<T, 4>::run(args...);                      \
        case 5: return F<T, 5>::run(args...);                      \
        case 6: return F<T, 6>::run(args...);                      \
        case 7: return F<T, 7>::run(args...);                      \
        default: return F<T, 8>::run(args...);                     \
    }
    switch (dtype) {
        case SSM_F32: SSM_CONV_K(float)
        case SSM_BF16: SSM_CONV_K(__nv_bfloat16)
        default: SSM_CONV_K(__half)
    }
#undef SSM_CONV_K
}

template <typename T, int K> struct FwdRun {
    static int run(const Args* a, bool bulk, cudaStream_t st) { return launch_fwd<T, K>(*a, bulk, st); }
};
template <typename T, int K> struct BwdRun {
    static int run(const Args* a, bool bulk, float* dw, float* db, cudaStream_t st) {
        return launch_bwd<T, K>(*a, bulk, dw, db, st);
    }
};
template <typename T, int K>
static int launch_fwd_cl(const Args& a, cudaStream_t st) {
    constexpr int V = ClVec<T>::V;
    const dim3 grid((unsigned)ceil_div(a.channels, 32 * V), (unsigned)ceil_div(a.length, (int64_t)kClWarps * kRun),
                    (unsigned)a.batch);
    fwd_cl_kernel<T, K><<<grid, kThreads, (size_t)kClDepth * kThreads * 8, st>>>(a);
    return check_launch("causal_conv1d fwd (channel-last)");
}

template <typename T, int K>
static int launch_bwd_cl(const Args& a, float* dweight, float* dbias, cudaStream_t st) {
    constexpr int V = ClVec<T>::V;
    const dim3 grid((unsigned)ceil_div(a.channels, 32 * V), (unsigned)ceil_div(a.length, (int64_t)kClWarps * kRun),
                    (unsigned)a.batch);
    const size_t sm = (size_t)kClDepth * 2 * kThreads * 8;   // also holds the fold
    static_assert((size_t)kClDepth * 2 * kThreads * 8 >= (size_t)kClWarps * 32 * ClVec<T>::V * (K + 1) * 4,
                  "the dweight fold fits in the ring space");
    if (cudaFuncSetAttribute(bwd_cl_kernel<T, K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return check_launch("causal_conv1d bwd (channel-last): smem attribute");
    bwd_cl_kernel<T, K><<<grid, kThreads, sm, st>>>(a);
    if (int s = check_launch("causal_conv1d bwd (channel-last)")) return s;
    const int64_t total = a.channels * (K + 1);
    finalize_cl_kernel<K><<<(unsigned)min64(ceil_div(total, 256), 148 * 8), 256, 0, st>>>(a, dweight, dbias);
    return check_launch("causal_conv1d bwd (channel-last) finalize");
}

template <typename T, int K> struct ClFwdRun {
    static int run(const Args* a, cudaStream_t st) { return launch_fwd_cl<T, K>(*a, st); }
};
template <typename T, int K> struct ClBwdRun {
    static int run(const Args* a, float* dw, float* db, cudaStream_t st) { return launch_bwd_cl<T, K>(*a, dw, db, st); }
};
template <typename T, int K> struct UpdRun {
    static int run(const ssm_causal_conv1d_update_params* p, cudaStream_t st) { return launch_update<T, K>(p, st); }
};

}  // namespace conv
}  // namespace ssm

using namespace ssm;
using namespace ssm::conv;

// The channel-last layout's requirements (SSM_CHANNEL_LAST).
static int cl_check(const ssm_causal_conv1d_params* p, bool bwd) {
    const int64_t esz = p->dtype == SSM_F32 ? 4 : 2, v = 8 / esz;
    const int64_t xs = p->x_row_stride ? p->x_row_stride : p->channels;
    const int64_t ds = p->dout_row_stride ? p->dout_row_stride : p->channels;
    if ((p->flags & SSM_HAS_INIT) || p->final_state || (bwd && p->dinitial))
        return fail(SSM_ERR_UNSUPPORTED, "causal_conv1d channel-last: no initial or final state");
    if (p->channels % v || xs < p->channels || (bwd && ds < p->channels) || (xs * esz) % 8 || (ds * esz) % 8)
        return fail(SSM_ERR_UNSUPPORTED, "causal_conv1d channel-last: channels and row strides need 8-byte rows");
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 7) == 0; };
    if (!al(p->x) || (!bwd && !al(p->out)) || (bwd && (!al(p->dout) || !al(p->dx))))
        return fail(SSM_ERR_UNSUPPORTED, "causal_conv1d channel-last: pointers must be 8-byte aligned");
    if (ceil_div(max64(p->length, 1), (int64_t)kClWarps * kRun) > 65535 || p->batch > 65535)
        return fail(SSM_ERR_UNSUPPORTED, "causal_conv1d channel-last: length or batch too large");
    return SSM_OK;
}
static size_t cl_workspace(const ssm_causal_conv1d_params* p) {
    return (size_t)(p->batch * ceil_div(max64(p->length, 1), (int64_t)kClWarps * kRun) * p->channels *
                    (p->width + 1)) * 4;
}

extern "C" int ssm_causal_conv1d_sizes(const ssm_causal_conv1d_params* p, size_t* workspace_bytes) {
    if (int s = validate(p)) return s;
    if (p->flags & SSM_CHANNEL_LAST) {
        if (workspace_bytes) *workspace_bytes = cl_workspace(p);
        return SSM_OK;
    }
    Args a, b;
    plan(p, false, a);
    plan(p, true, b);
    const int64_t slots = max64(a.nchunks * a.slots, b.nchunks * b.slots);
    if (workspace_bytes) *workspace_bytes = (size_t)(a.rows * slots * (p->width + 1)) * 4;
    return SSM_OK;
}

int ssm_conv_take_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, ssm::conv::g_conv_error, sizeof(int)) != cudaSuccess) return -1;
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(ssm::conv::g_conv_error, &zero, sizeof(int));
    }
    return v;
}

extern "C" int ssm_causal_conv1d_fwd(const ssm_causal_conv1d_params* p, void* stream) {
    if (int s = validate(p)) return s;
    if (p->batch == 0 || p->channels == 0) return SSM_OK;
    if (!p->x || !p->weight || (!p->out && p->length) || ((p->flags & SSM_HAS_BIAS) && !p->bias) ||
        ((p->flags & SSM_HAS_INIT) && !p->initial_state))
        return fail(SSM_ERR_INVALID, "causal_conv1d fwd: null pointer");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (p->flags & SSM_CHANNEL_LAST) {
        if (int s = cl_check(p, false)) return s;
        if (p->length == 0) return SSM_OK;
        Args a;
        plan(p, false, a);
        return by_type_width<ClFwdRun>(p->dtype, (int)p->width, (const Args*)&a, st);
    }
    const bool bulk = bulk_ok(p, false);
    Args a;
    plan(p, bulk, a);
    if (p->length == 0) {
        // no outputs; the final state is the initial state (or zeros)
        if (p->final_state && p->width > 1) {
            const size_t bytes = (size_t)(a.rows * (p->width - 1)) * (p->dtype == SSM_F32 ? 4 : 2);
            const cudaError_t e = (p->flags & SSM_HAS_INIT)
                ? cudaMemcpyAsync(p->final_state, p->initial_state, bytes, cudaMemcpyDeviceToDevice, st)
                : cudaMemsetAsync(p->final_state, 0, bytes, st);
            if (e != cudaSuccess) return check_launch("causal_conv1d fwd: final state");
        }
        return SSM_OK;
    }
    return by_type_width<FwdRun>(p->dtype, (int)p->width, (const Args*)&a, bulk, st);
}

extern "C" int ssm_causal_conv1d_bwd(const ssm_causal_conv1d_params* p, void* stream) {
    if (int s = validate(p)) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool bulk = bulk_ok(p, true);
    Args a;
    plan(p, bulk, a);
    const int64_t K = p->width;
    if (p->batch == 0 || p->channels == 0 || p->length == 0) {
        if (p->dweight && p->channels && cudaMemsetAsync(p->dweight, 0, (size_t)(p->channels * K) * 4, st))
            return check_launch("causal_conv1d bwd: zero dweight");
        if (p->dbias && p->channels && cudaMemsetAsync(p->dbias, 0, (size_t)p->channels * 4, st))
            return check_launch("causal_conv1d bwd: zero dbias");
        if (p->dinitial && a.rows && K > 1 &&
            cudaMemsetAsync(p->dinitial, 0, (size_t)(a.rows * (K - 1)) * (p->dtype == SSM_F32 ? 4 : 2), st))
            return check_launch("causal_conv1d bwd: zero dinitial");
        return SSM_OK;
    }
    if (!p->x || !p->weight || !p->dout || !p->dx || ((p->flags & SSM_HAS_BIAS) && !p->bias) ||
        ((p->flags & SSM_HAS_INIT) && !p->initial_state))
        return fail(SSM_ERR_INVALID, "causal_conv1d bwd: null pointer");
    if (p->flags & SSM_CHANNEL_LAST) {
        if (int s = cl_check(p, true)) return s;
        if (p->workspace == nullptr || p->workspace_bytes < cl_workspace(p))
            return fail(SSM_ERR_WORKSPACE, "causal_conv1d bwd: workspace smaller than ssm_causal_conv1d_sizes");
        a.partial = static_cast<float*>(p->workspace);
        return by_type_width<ClBwdRun>(p->dtype, (int)K, (const Args*)&a, p->dweight,
                                       (p->flags & SSM_HAS_BIAS) ? p->dbias : nullptr, st);
    }
    const size_t need = (size_t)(a.rows * a.nchunks * a.slots * (K + 1)) * 4;
    if (p->workspace == nullptr || p->workspace_bytes < need)
        return fail(SSM_ERR_WORKSPACE, "causal_conv1d bwd: workspace smaller than ssm_causal_conv1d_sizes");
    a.partial = static_cast<float*>(p->workspace);
    if (!(p->flags & SSM_HAS_INIT)) a.dinit = nullptr;
    return by_type_width<BwdRun>(p->dtype, (int)K, (const Args*)&a, bulk, p->dweight,
                                 (p->flags & SSM_HAS_BIAS) ? p->dbias : nullptr, st);
}

extern "C" int ssm_causal_conv1d_update(const ssm_causal_conv1d_update_params* p, void* stream) {
    if (p == nullptr) return fail(SSM_ERR_INVALID, "causal_conv1d_update: null params");
    if (p->batch < 0 || p->channels < 0 || p->length < 0 || p->state_len < p->width - 1)
        return fail(SSM_ERR_INVALID, "causal_conv1d_update: extents");
    if (p->width < 1 || p->width > kMaxWidth)
        return fail(SSM_ERR_UNSUPPORTED, "causal_conv1d_update: kernel width must be 1..8");
    if (p->dtype < SSM_F32 || p->dtype > SSM_F16) return fail(SSM_ERR_UNSUPPORTED, "causal_conv1d_update: dtype");
    if (p->batch == 0 || p->channels == 0 || p->length == 0) return SSM_OK;
    // a width-1 kernel may come with a state of zero columns, which is never read
    if ((!p->state && p->state_len > 0) || !p->x || !p->weight || !p->out ||
        ((p->flags & SSM_HAS_BIAS) && !p->bias))
        return fail(SSM_ERR_INVALID, "causal_conv1d_update: null pointer");
    return by_type_width<UpdRun>(p->dtype, (int)p->width, p, static_cast<cudaStream_t>(stream));
}
