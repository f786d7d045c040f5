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
// built for HBM: persistent warps walk (row, 512-element segment) items, each
// lane owning 16 consecutive elements read and written as two 16-byte vectors
// (a scalar variant serves rows that are not 16-byte aligned), with the next
// item's loads issued before the current item is computed.  The taps-wide
// halos either side come from the neighbouring lanes by shuffle, so each
// element is loaded once.  The backward recomputes the pre-activation from x
// instead of saving it, and reduces dweight / dbias per item in a fixed order
// into partials that a second kernel folds per channel, so results are
// bit-reproducible.
#include "common.cuh"
#include "tc.cuh"

namespace ssm {
namespace conv {

constexpr int kThreads = 256;
constexpr int kMaxWidth = 8;

struct Args {
    int64_t batch, channels, length, rows;    // rows = batch * channels
    int64_t nchunks, chunk;                   // chunks per row, elements per chunk
    uint32_t flags;
    const void* x; const float* w; const float* bias; const void* init;
    void* out; void* final_state;
    const void* dout; void* dx; void* dinit;
    float* partial;                           // (rows, nchunks, K + 1)
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
// kTile elements) items.  One thread issues a bulk asynchronous copy of each
// item's tile -- with up to 8 elements of halo either side -- into one of
// kStages shared-memory stages, completing on the stage's mbarrier, so the next
// items' bytes stream in while the current tile is computed; every thread then
// owns 16 elements of the tile.  Waits are bounded: a wait that runs out
// records an error code (ssm_take_kernel_error) and the CTA stops after
// draining the copies it issued.
constexpr int kTile = kThreads * 16;   // 4096 elements
constexpr int kHalo = 8;
constexpr int kStages = 3;

__device__ int g_conv_error;

template <typename T, int NT>
struct BulkLayout {
    static constexpr int SPAN = kHalo + kTile + kHalo;             // elements per stage and tensor
    static constexpr size_t stage_bytes = (size_t)SPAN * sizeof(T) * NT;
    static constexpr size_t mbar_off = stage_bytes * kStages;
    static constexpr size_t bytes = mbar_off + 8 * kStages;
};

// Copy item `it`'s tile(s) into stage `st`: elements [t0 - front, t0 + n + back)
// of the row land at stage offset kHalo - front.
template <typename T, int NT>
__device__ __forceinline__ void issue_tile(const Args& a, unsigned char* smem, int st, int64_t it,
                                           const void* s0, const void* s1) {
    using Lay = BulkLayout<T, NT>;
    const int64_t L = a.length;
    int64_t row, tile, c;
    item_coords(a, it, row, tile, c);
    const int64_t t0 = tile * kTile;
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
}

template <typename T, int K>
__global__ void __launch_bounds__(kThreads)
fwd_bulk_kernel(const Args a) {
    constexpr int TAPS = K - 1;
    using Lay = BulkLayout<T, 1>;
    extern __shared__ __align__(128) unsigned char smem[];
    const int64_t items = a.rows * a.nchunks, L = a.length;
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) tc::mbar_init(tc::smem_u32(smem + Lay::mbar_off + 8 * s), 1);
        tc::fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < kStages; ++s) {
            const int64_t it = blockIdx.x + (int64_t)s * gridDim.x;
            if (it < items) issue_tile<T, 1>(a, smem, s, it, a.x, nullptr);
        }
    bool ok = true;
    int64_t k = 0;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x, ++k) {
        const int st = (int)(k % kStages);
        const uint32_t par = (uint32_t)((k / kStages) & 1);
        // one thread polls; the rest wait at the barrier without issuing
        if (tid == 0) ok = tc::mbar_wait(tc::smem_u32(smem + Lay::mbar_off + 8 * st), par);
        ok = __syncthreads_and(ok);
        if (!ok) { if (tid == 0) atomicCAS(&g_conv_error, 0, 61); break; }
        int64_t row, tl, c;
        item_coords(a, it, row, tl, c);
        const int64_t t0 = tl * kTile;
        const int64_t n = min64(kTile, L - t0);
        const T* tile = reinterpret_cast<const T*>(smem + st * Lay::stage_bytes) + kHalo;   // tile[p], p >= -front
        float w[K];
#pragma unroll
        for (int j = 0; j < K; ++j) w[j] = a.w[c * K + j];
        const float bv = (a.flags & kHasBias) ? a.bias[c] : 0.0f;
        const T* ir = (a.flags & kHasInit) ? static_cast<const T*>(a.init) + row * TAPS : nullptr;
        // thread tid owns the 8-element groups at 8 tid and kTile/2 + 8 tid, so
        // each warp-wide 16-byte store covers 512 contiguous bytes
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int p0 = u * (kTile / 2) + tid * 8;
            float z[TAPS + 8];
            const bool whole = p0 + 8 <= n;
            if (whole) {
                Vec<T, 8>::ld(tile + p0, z + TAPS);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) z[TAPS + i] = p0 + i < n ? ldf(tile + p0 + i) : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < TAPS; ++i) {
                const float up = __shfl_up_sync(0xffffffffu, z[8 + i], 1);
                float v;
                if (lane > 0) v = up;
                else if (t0 + p0 == 0) v = ir ? ldf(ir + i) : 0.0f;
                else v = ldf(tile + p0 - TAPS + i);
                z[i] = v;
            }
            if (p0 < n) {
                float o[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float acc = bv;
#pragma unroll
                    for (int j = 0; j < K; ++j) acc = fmaf(w[j], z[i + j], acc);
                    o[i] = (a.flags & kSilu) ? silu_t<T>(acc) : acc;
                }
                T* dst = static_cast<T*>(a.out) + row * L + t0 + p0;
                if (whole) Vec<T, 8>::st(dst, o);
                else {
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        if (p0 + i < n) stf(dst + i, o[i]);
                }
            }
        }
        if (a.final_state != nullptr && t0 == 0 && tid == 0) {
            const T* xr = static_cast<const T*>(a.x) + row * L;
            const T* ir = (a.flags & kHasInit) ? static_cast<const T*>(a.init) + row * TAPS : nullptr;
            T* fr = static_cast<T*>(a.final_state) + row * TAPS;
#pragma unroll
            for (int i = 0; i < TAPS; ++i) stf(fr + i, zval<T, TAPS>(xr, ir, L - TAPS + i, L));
        }
        __syncthreads();                          // every thread is done with the stage
        if (tid == 0) {
            const int64_t nit = it + (int64_t)kStages * gridDim.x;
            if (nit < items) issue_tile<T, 1>(a, smem, st, nit, a.x, nullptr);
        }
    }
    if (!ok && tid == 0) {
        // drain: wait (bounded) for every copy this CTA issued and has not consumed
        for (int64_t it = blockIdx.x + k * (int64_t)gridDim.x, j = k;
             it < items && j < k + kStages; it += gridDim.x, ++j)
            tc::mbar_wait(tc::smem_u32(smem + Lay::mbar_off + 8 * (j % kStages)), (uint32_t)((j / kStages) & 1));
    }
}

template <typename T, int K>
__global__ void __launch_bounds__(kThreads)
bwd_bulk_kernel(const Args a) {
    constexpr int TAPS = K - 1;
    using Lay = BulkLayout<T, 2>;
    __shared__ float red[kThreads / 32][K + 1];
    extern __shared__ __align__(128) unsigned char smem[];
    const int64_t items = a.rows * a.nchunks, L = a.length;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) tc::mbar_init(tc::smem_u32(smem + Lay::mbar_off + 8 * s), 1);
        tc::fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < kStages; ++s) {
            const int64_t it = blockIdx.x + (int64_t)s * gridDim.x;
            if (it < items) issue_tile<T, 2>(a, smem, s, it, a.x, a.dout);
        }
    bool ok = true;
    int64_t k = 0;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x, ++k) {
        const int st = (int)(k % kStages);
        const uint32_t par = (uint32_t)((k / kStages) & 1);
        // one thread polls; the rest wait at the barrier without issuing
        if (tid == 0) ok = tc::mbar_wait(tc::smem_u32(smem + Lay::mbar_off + 8 * st), par);
        ok = __syncthreads_and(ok);
        if (!ok) { if (tid == 0) atomicCAS(&g_conv_error, 0, 62); break; }
        int64_t row, tl, c;
        item_coords(a, it, row, tl, c);
        const int64_t t0 = tl * kTile;
        const int64_t n = min64(kTile, L - t0);
        const int64_t rem = L - t0;                // valid positions from the tile start
        const T* xt = reinterpret_cast<const T*>(smem + st * Lay::stage_bytes) + kHalo;
        const T* dt = xt + Lay::SPAN;
        float w[K];
#pragma unroll
        for (int j = 0; j < K; ++j) w[j] = a.w[c * K + j];
        const float bv = (a.flags & kHasBias) ? a.bias[c] : 0.0f;
        const T* ir = (a.flags & kHasInit) ? static_cast<const T*>(a.init) + row * TAPS : nullptr;
        float dw[K + 1];
#pragma unroll
        for (int j = 0; j <= K; ++j) dw[j] = 0.0f;
        // thread tid owns the 8-element groups at 8 tid and kTile/2 + 8 tid
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int p0 = u * (kTile / 2) + tid * 8;
            float z[8 + 2 * TAPS], g[8 + TAPS];
            const bool whole = p0 + 8 <= n;
            if (whole) {
                Vec<T, 8>::ld(xt + p0, z + TAPS);
                Vec<T, 8>::ld(dt + p0, g);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    z[TAPS + i] = p0 + i < n ? ldf(xt + p0 + i) : 0.0f;
                    g[i] = p0 + i < n ? ldf(dt + p0 + i) : 0.0f;
                }
            }
#pragma unroll
            for (int i = 0; i < TAPS; ++i) {
                const float up = __shfl_up_sync(0xffffffffu, z[8 + i], 1);
                const float xdn = __shfl_down_sync(0xffffffffu, z[TAPS + i], 1);
                const float gdn = __shfl_down_sync(0xffffffffu, g[i], 1);
                float v;
                if (lane > 0) v = up;
                else if (t0 + p0 == 0) v = ir ? ldf(ir + i) : 0.0f;
                else v = ldf(xt + p0 - TAPS + i);
                z[i] = v;
                // past this group: the next lane's group, or (last lane) the next
                // warp's, the back halo, or zero past the row
                const int q = p0 + 8 + i;
                const bool in = q < rem;
                z[TAPS + 8 + i] = lane < 31 ? xdn : (in ? ldf(xt + q) : 0.0f);
                g[8 + i] = lane < 31 ? gdn : (in ? ldf(dt + q) : 0.0f);
            }
            if (p0 < n) {
                float o[8], dwl[K + 1];
                conv_bwd_lane<T, K, 8>(w, bv, a.flags & kSilu, z, g, o, dwl);
#pragma unroll
                for (int j = 0; j <= K; ++j) dw[j] += dwl[j];
                T* dst = static_cast<T*>(a.dx) + row * L + t0 + p0;
                if (whole) Vec<T, 8>::st(dst, o);
                else {
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        if (p0 + i < n) stf(dst + i, o[i]);
                }
                if (TAPS > 0 && t0 + p0 == 0 && a.dinit != nullptr)
                    dinit_row<T, K>(static_cast<T*>(a.dinit) + row * TAPS, w, g);
            }
        }
#pragma unroll
        for (int j = 0; j <= K; ++j) {
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) dw[j] += __shfl_xor_sync(0xffffffffu, dw[j], o2);
            if (lane == 0) red[warp][j] = dw[j];
        }
        __syncthreads();                          // stage and red[] complete
        if (tid <= K) {
            float sum = 0.0f;
#pragma unroll
            for (int q = 0; q < kThreads / 32; ++q) sum += red[q][tid];
            a.partial[it * (K + 1) + tid] = sum;
        }
        if (tid == 0) {
            const int64_t nit = it + (int64_t)kStages * gridDim.x;
            if (nit < items) issue_tile<T, 2>(a, smem, st, nit, a.x, a.dout);
        }
        __syncthreads();                          // red[] is free again
    }
    if (!ok && tid == 0) {
        for (int64_t it = blockIdx.x + k * (int64_t)gridDim.x, j = k;
             it < items && j < k + kStages; it += gridDim.x, ++j)
            tc::mbar_wait(tc::smem_u32(smem + Lay::mbar_off + 8 * (j % kStages)), (uint32_t)((j / kStages) & 1));
    }
}

// dweight[c, j] and dbias[c]: partials of every (batch, chunk) of channel c.
template <int K>
__global__ void finalize_kernel(const Args a, float* dweight, float* dbias) {
    const int64_t total = a.channels * (K + 1);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = i / (K + 1);
        const int j = (int)(i - c * (K + 1));
        float s = 0.0f;
        for (int64_t b = 0; b < a.batch; ++b) {
            const float* p = a.partial + ((b * a.channels + c) * a.nchunks) * (K + 1) + j;
            for (int64_t k = 0; k < a.nchunks; ++k) s += p[k * (K + 1)];
        }
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
    a.flags = p->flags;
    a.x = p->x; a.w = p->weight; a.bias = p->bias; a.init = p->initial_state;
    a.out = p->out; a.final_state = p->final_state;
    a.dout = p->dout; a.dx = p->dx; a.dinit = p->dinitial;
    a.partial = nullptr;
}

// Persistent grid: resident CTAs of the kernel on every SM, at most one per item.
template <typename F>
static unsigned persistent_grid(F kernel, size_t smem, const Args& a) {
    int dev = 0, sms = 148, per = 1;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, kThreads, smem) != cudaSuccess || per < 1) {
        cudaGetLastError();
        per = 1;
    }
    return (unsigned)max64(1, min64((int64_t)sms * per, a.rows * a.nchunks));
}

template <typename T, int K>
static int launch_fwd(const Args& a, bool bulk, cudaStream_t st) {
    if (bulk) {
        const size_t sm = BulkLayout<T, 1>::bytes;
        auto k = fwd_bulk_kernel<T, K>;
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
            return check_launch("causal_conv1d fwd: smem attribute");
        k<<<persistent_grid(k, sm, a), kThreads, sm, st>>>(a);
    } else {
        fwd_plain_kernel<T, K><<<(unsigned)ceil_div(a.rows * a.nchunks, kThreads / 32), kThreads, 0, st>>>(a);
    }
    return check_launch("causal_conv1d fwd");
}

template <typename T, int K>
static int launch_bwd(const Args& a, bool bulk, float* dweight, float* dbias, cudaStream_t st) {
    if (bulk) {
        const size_t sm = BulkLayout<T, 2>::bytes;
        auto k = bwd_bulk_kernel<T, K>;
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
            return check_launch("causal_conv1d bwd: smem attribute");
        k<<<persistent_grid(k, sm, a), kThreads, sm, st>>>(a);
    } else {
        bwd_plain_kernel<T, K><<<(unsigned)ceil_div(a.rows * a.nchunks, kThreads / 32), kThreads, 0, st>>>(a);
    }
    if (int s = check_launch("causal_conv1d bwd")) return s;
    const int64_t total = a.channels * (K + 1);
    finalize_kernel<K><<<(unsigned)min64(ceil_div(total, 256), 148 * 8), 256, 0, st>>>(a, dweight, dbias);
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
template <typename T, int K> struct UpdRun {
    static int run(const ssm_causal_conv1d_update_params* p, cudaStream_t st) { return launch_update<T, K>(p, st); }
};

}  // namespace conv
}  // namespace ssm

using namespace ssm;
using namespace ssm::conv;

extern "C" int ssm_causal_conv1d_sizes(const ssm_causal_conv1d_params* p, size_t* workspace_bytes) {
    if (int s = validate(p)) return s;
    Args a;
    plan(p, false, a);   // the plain path has the most items
    if (workspace_bytes) *workspace_bytes = (size_t)(a.rows * a.nchunks * (p->width + 1)) * 4;
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
    const size_t need = (size_t)(a.rows * a.nchunks * (K + 1)) * 4;
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
