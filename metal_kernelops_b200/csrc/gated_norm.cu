// Gated RMSNorm (the normalisation after the SSD scan in Mamba-2 blocks) for
// sm_100a: fused forward and analytic backward.
//
// Reference behaviour: src/metal_kernelops/cv/gated_norm.py -- `rmsnorm_gated`
// (:647-686) over `_GatedRMSNorm` (:563-644), i.e. mamba_ssm's `rms_norm_ref`
// (restated by `rmsnorm_gated_reference`, :689-720).  Per row and group of G
// features, with gate = silu(z):
//     xb  = x * gate                    (norm_before_gate = False, z given)
//     r   = rsqrt(mean(xb^2) + eps)
//     y0  = xb * r * w + b
//     out = y0 * gate                   (norm_before_gate = True, z given)
// Backward, with xh = xb r, dy0 = dy * gate (after) or dy, dxh = dy0 w,
// c1 = mean(xh dxh) over the group:
//     dxb = r (dxh - xh c1);  dx = dxb * gate (before) or dxb
//     dz  = dxb x silu'(z) (before) or dy y0 silu'(z) (after)
//     dw  = sum_rows dy0 xh,  db = sum_rows dy0
// All arithmetic in fp32; x, z, out, dy, dx, dz in the activation dtype.
//
// Bytes, not flops: x and z (and dy) cross HBM once.  Groups of up to 1024
// bf16 / 512 fp32 elements (Mamba-2's groups are d_inner / ngroups, e.g. 640)
// take the warp path: one warp per (row, group), each lane owning a few
// 8- or 16-byte slots of the group, the sum of squares and c1 by shuffles, no
// block barrier; each warp stages its next row in shared memory with
// asynchronous copies while it computes the current one.  Each CTA's warps
// walk a block of rows of one group; the backward keeps each lane's dw column
// sums in registers, adding the warps in a fixed order into one partial per
// (row block, column).  Wider groups stream: one CTA per (row block, group)
// walks each row twice (the sum, then the outputs), the second pass
// re-reading the row from L1/L2, and adds its dw / db into its own partial
// slots.  A last kernel adds the partials in order, so the results are
// reproducible.
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "tc.cuh"

namespace ssm {
namespace gnorm {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kGateNone = 0, kGateBefore = 1, kGateAfter = 2;

struct Args {
    int64_t rows, features, group, ngroups;
    int64_t xs, zs;                       // row strides of x and z (elements)
    int64_t row_blocks, rows_per_block;
    float eps;
    int gate;
    bool has_bias;
    const void* x; const void* z; const float* w; const float* b;
    void* out; float* rstd;
    const void* dy; void* dx; void* dz;
    float* dw_part; float* db_part;       // (row_blocks, features)
};

template <typename T, int V> struct VecIo;
template <typename T> struct VecIo<T, 1> {
    static __device__ __forceinline__ void ld(const T* p, float* v) { v[0] = ldf(p); }
    static __device__ __forceinline__ void st(T* p, const float* v) { stf(p, v[0]); }
};
template <> struct VecIo<float, 4> {
    static __device__ __forceinline__ void ld(const float* p, float* v) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    }
    static __device__ __forceinline__ void st(float* p, const float* v) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
};
template <typename T> struct VecIo16 {
    static __device__ __forceinline__ void ld(const T* p, float* v) {
        const uint4 r = *reinterpret_cast<const uint4*>(p);
        const T* h = reinterpret_cast<const T*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = Io2<T>::ld(h + 2 * i);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
    static __device__ __forceinline__ void st(T* p, const float* v) {
        uint4 r;
        T* h = reinterpret_cast<T*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) Io2<T>::st(h + 2 * i, make_float2(v[2 * i], v[2 * i + 1]));
        *reinterpret_cast<uint4*>(p) = r;
    }
};
template <> struct VecIo<__nv_bfloat16, 8> : VecIo16<__nv_bfloat16> {};
template <> struct VecIo<__half, 8> : VecIo16<__half> {};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One element's backward given r and c1: dx, dz, and the dy0 / xh that feed
// dw and db.  sigmoid_t<T> picks the MUFU form by the data's storage type.
struct ElemGrad { float dx, dz, dy0, xh; };
template <typename T>
__device__ __forceinline__ ElemGrad elem_grad(float xv, float zv, float dv, float w, float b, float r, float c1,
                                              int gate) {
    const float sg = gate != kGateNone ? sigmoid_t<T>(zv) : 1.0f;
    const float gt = gate != kGateNone ? zv * sg : 1.0f;
    const float dsilu = sg * fmaf(zv, 1.0f - sg, 1.0f);
    const float xb = gate == kGateBefore ? xv * gt : xv;
    ElemGrad e;
    e.xh = xb * r;
    e.dy0 = gate == kGateAfter ? dv * gt : dv;
    const float dxb = r * (e.dy0 * w - e.xh * c1);
    e.dx = gate == kGateBefore ? dxb * gt : dxb;
    e.dz = gate == kGateBefore ? dxb * xv * dsilu : gate == kGateAfter ? dv * fmaf(e.xh, w, b) * dsilu : 0.0f;
    return e;
}
// Its contribution to c1 = mean(xh dy0 w).
template <typename T>
__device__ __forceinline__ float elem_c1(float xv, float zv, float dv, float w, float r, int gate) {
    const float gt = gate != kGateNone ? zv * sigmoid_t<T>(zv) : 1.0f;
    const float xh = (gate == kGateBefore ? xv * gt : xv) * r;
    const float dy0 = gate == kGateAfter ? dv * gt : dv;
    return xh * dy0 * w;
}

// ------------------------------------------------------------- warp path --
// One warp per (row, group): lane slot s = k * 32 + lane (k < NV) holds the
// V consecutive elements [s V, s V + V) of the group as raw words, V * size
// of T = 8 or 16 bytes, read and written with one vector access.  Elements
// are processed in adjacent pairs with the paired fp32 instructions; the gate
// mode is a template parameter.  Weight and bias sit in shared memory in
// natural order, so a slot's V floats are one or two 16-byte reads.

// V elements of T as 32-bit words.
template <typename T, int V>
struct Raw {
    static constexpr int W = V * (int)sizeof(T) / 4;
    uint32_t w[W];
    __device__ __forceinline__ void ld(const T* p) {
        if constexpr (W == 4) {
            const uint4 q = *reinterpret_cast<const uint4*>(p);
            w[0] = q.x; w[1] = q.y; w[2] = q.z; w[3] = q.w;
        } else {
            const uint2 q = *reinterpret_cast<const uint2*>(p);
            w[0] = q.x; w[1] = q.y;
        }
    }
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int i = 0; i < W; ++i) w[i] = 0u;
    }

    // elements (2m, 2m + 1)
    __device__ __forceinline__ float2 pair(int m) const {
        if constexpr (sizeof(T) == 4) {
            return make_float2(__uint_as_float(w[2 * m]), __uint_as_float(w[2 * m + 1]));
        } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            return make_float2(__uint_as_float(w[m] << 16), __uint_as_float(w[m] & 0xffff0000u));
        } else {
            __half2 h;
            memcpy(&h, &w[m], 4);
            return __half22float2(h);
        }
    }
    __device__ __forceinline__ void set(int m, float2 v) {
        if constexpr (sizeof(T) == 4) {
            w[2 * m] = __float_as_uint(v.x);
            w[2 * m + 1] = __float_as_uint(v.y);
        } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
            memcpy(&w[m], &h, 4);
        } else {
            const __half2 h = __floats2half2_rn(v.x, v.y);
            memcpy(&w[m], &h, 4);
        }
    }
    __device__ __forceinline__ void st(T* p) const {
        if constexpr (W == 4) *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
        else *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
    }
};

// silu(z) and sigmoid(z) of two elements, by the storage-type rules of
// sigmoid_t: fp32 data rcp(1 + 2^(-z log2 e)), 16-bit data (1 + tanh(z/2)) / 2.
struct Gate2 { float2 silu, sig; };
template <typename T>
__device__ __forceinline__ Gate2 gate2(float2 z) {
    if constexpr (sizeof(T) == 4) {
        const float2 m = mul2(z, f2(-kLog2e));
        const float2 d = add2(make_float2(exp2_mufu(m.x), exp2_mufu(m.y)), f2(1.0f));
        const float2 s = make_float2(rcp_mufu(d.x), rcp_mufu(d.y));
        return {mul2(z, s), s};
    } else {
        const float2 h = mul2(z, f2(0.5f));
        const float2 t = make_float2(tanh_mufu(h.x), tanh_mufu(h.y));
        return {fma2(h, t, h), fma2(t, f2(0.5f), f2(0.5f))};
    }
}
// silu'(z) = s (1 + z (1 - s))
__device__ __forceinline__ float2 dsilu2(float2 z, float2 s) {
    return mul2(s, fma2(z, fma2(s, f2(-1.0f), f2(1.0f)), f2(1.0f)));
}

// i, as a value the compiler cannot see through and that exists no earlier
// than `after`: loads indexed by it are issued again rather than merged with
// an earlier pass's loads of the same data, so that pass's registers die.
__device__ __forceinline__ int fresh(int i, float after) {
    int q;
    asm volatile("mov.b32 %0, %1;" : "=r"(q) : "r"(i), "f"(after));
    return q;
}

template <int V>
__device__ __forceinline__ float2 wpair(const float* ws, int e0, int m) {
    return *reinterpret_cast<const float2*>(ws + e0 + 2 * m);
}

template <int GP>
__device__ __forceinline__ void stage_wb(const Args& a, int64_t g, float* ws, float* bs) {
    for (int f = threadIdx.x; f < GP; f += kThreads) {
        const bool in = f < a.group;
        ws[f] = in ? a.w[g * a.group + f] : 0.0f;
        bs[f] = (in && a.has_bias) ? a.b[g * a.group + f] : 0.0f;
    }
}

// Per-warp ring of two row stages in shared memory: stage b holds NT tensors'
// GP elements of one (row, group), filled by per-lane asynchronous copies of
// the lane's own slots, so a warp loads row i + 1 while it computes row i and
// no registers hold data in flight.  A lane reads only what it copied itself,
// so its own cp.async wait makes the data visible.
template <typename T, int V, int NV, int NT>
struct RowRing {
    static constexpr int GP = 32 * NV * V;
    static constexpr size_t bytes = (size_t)2 * NT * GP * sizeof(T);   // per warp
    T* base;
    __device__ const T* at(int b, int t, int e0) const { return base + (b * NT + t) * GP + e0; }
    __device__ void issue(int b, const T* const* src, const int64_t* off, int64_t G) const {
        const int lane = threadIdx.x & 31;
        __syncwarp();                             // the lane's reads of stage b are done
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int e0 = (k * 32 + lane) * V;
            if (e0 < G) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const uint32_t d = tc::smem_u32(base + (b * NT + t) * GP + e0);
                    if constexpr (V * sizeof(T) == 16) tc::cp_async16(d, src[t] + off[t] + e0);
                    else tc::cp_async8(d, src[t] + off[t] + e0);
                }
            }
        }
        tc::cp_async_commit();
    }
};

// Forward: reduce the row's gated square sum, then write the outputs.
template <typename T, int V, int NV, int GATE>
__global__ void __launch_bounds__(kThreads)
fwd_kernel(const Args a) {
    constexpr int GP = 32 * NV * V, M = V / 2;
    constexpr int NT = GATE != kGateNone ? 2 : 1;
    using Ring = RowRing<T, V, NV, NT>;
    extern __shared__ __align__(16) unsigned char smraw[];
    float* ws = reinterpret_cast<float*>(smraw);
    float* bs = ws + GP;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const Ring ring{reinterpret_cast<T*>(smraw + 2 * GP * sizeof(float) + warp * Ring::bytes)};
    const int64_t g = blockIdx.y;
    const int64_t G = a.group, F = a.features;
    const int64_t r0 = blockIdx.x * a.rows_per_block;
    const int64_t r1 = min64(r0 + a.rows_per_block, a.rows);
    const T* const src[2] = {static_cast<const T*>(a.x), static_cast<const T*>(a.z)};
    T* out = static_cast<T*>(a.out);
    stage_wb<GP>(a, g, ws, bs);
    __syncthreads();
    const float inv_g = 1.0f / (float)G;
    // row offsets of x and z
    auto offs = [&](int64_t row, int64_t* o) { o[0] = row * a.xs + g * G; o[1] = row * a.zs + g * G; };
    int b = 0;
    int64_t off[2];
    if (r0 + warp < r1) { offs(r0 + warp, off); ring.issue(0, src, off, G); }
    for (int64_t row = r0 + warp; row < r1; row += kWarps, b ^= 1) {
        const int64_t base = row * F + g * G;
        if (row + kWarps < r1) { offs(row + kWarps, off); ring.issue(b ^ 1, src, off, G); }
        else tc::cp_async_commit();              // keep one group per row
        tc::cp_async_wait<1>();
        float2 xb[NV][M], gt[NV][M];
        float2 ss = f2(0.0f);
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int e0 = (k * 32 + lane) * V;
            Raw<T, V> xr, zr;
            if (e0 < G) {
                xr.ld(ring.at(b, 0, e0));
                if (GATE != kGateNone) zr.ld(ring.at(b, 1, e0));
            } else {
                xr.zero();
                zr.zero();
            }
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float2 v = xr.pair(m);
                if (GATE != kGateNone) {
                    gt[k][m] = gate2<T>(zr.pair(m)).silu;
                    if (GATE == kGateBefore) v = mul2(v, gt[k][m]);
                }
                xb[k][m] = v;
                ss = fma2(v, v, ss);
            }
        }
        const float r = rsqrtf(warp_sum(ss.x + ss.y) * inv_g + a.eps);
        if (a.rstd != nullptr && lane == 0) a.rstd[row * a.ngroups + g] = r;
        const float2 r2 = f2(r);
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int e0 = (k * 32 + lane) * V;
            if (e0 >= G) continue;
            Raw<T, V> o;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float2 y = mul2(mul2(xb[k][m], r2), wpair<V>(ws, e0, m));
                if (a.has_bias) y = add2(y, wpair<V>(bs, e0, m));
                if (GATE == kGateAfter) y = mul2(y, gt[k][m]);
                o.set(m, y);
            }
            o.st(out + base + e0);
        }
    }
    tc::cp_async_wait<0>();
}

// Backward.  Per row: r from the forward, c1 = mean(xh dy0 w) over the group
// (first pass over the staged row), then dx, dz and the dweight products
// (second pass over the same stage, recomputing the gate).  Each lane keeps
// the dweight sums of its own columns in registers across the CTA's rows
// (dbias, when there is a bias, in shared memory); at the end the warps' sums
// are added in a fixed order into one partial per (row block, column).
// Dynamic shared memory: w[GP], b[GP] floats, the warps' row rings (whose
// space then takes the dweight fold), and with a bias kWarps x GP floats of
// dbias sums.
template <typename T, int V, int NV, int GATE>
__global__ void __launch_bounds__(kThreads, 2)
bwd_kernel(const Args a) {
    constexpr int GP = 32 * NV * V, M = V / 2;
    constexpr int NT = GATE != kGateNone ? 3 : 2;
    using Ring = RowRing<T, V, NV, NT>;
    static_assert(Ring::bytes >= GP * sizeof(float), "the dweight fold reuses the rings");
    extern __shared__ __align__(16) unsigned char smraw[];
    float* ws = reinterpret_cast<float*>(smraw);
    float* bs = ws + GP;
    unsigned char* rings = smraw + 2 * GP * sizeof(float);
    float* fold = reinterpret_cast<float*>(rings);                       // after the row loop
    float* red_b = reinterpret_cast<float*>(rings + kWarps * Ring::bytes);   // with a bias only
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const Ring ring{reinterpret_cast<T*>(rings + warp * Ring::bytes)};
    const int64_t g = blockIdx.y;
    const int64_t G = a.group, F = a.features;
    const int64_t r0 = blockIdx.x * a.rows_per_block;
    const int64_t r1 = min64(r0 + a.rows_per_block, a.rows);
    // ring tensors: x, dy and (gated) z
    const T* const src[3] = {static_cast<const T*>(a.x), static_cast<const T*>(a.dy), static_cast<const T*>(a.z)};
    T* dx = static_cast<T*>(a.dx);
    T* dz = static_cast<T*>(a.dz);
    stage_wb<GP>(a, g, ws, bs);
    if (a.has_bias)
        for (int i = lane; i < GP; i += 32) red_b[warp * GP + i] = 0.0f;
    __syncthreads();
    const float inv_g = 1.0f / (float)G;
    float2 dwa[NV][M];
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
        for (int m = 0; m < M; ++m) dwa[k][m] = f2(0.0f);

    // row offsets of x, dy and z
    auto offs = [&](int64_t row, int64_t* o) {
        o[0] = row * a.xs + g * G;
        o[1] = row * F + g * G;
        o[2] = row * a.zs + g * G;
    };
    int b = 0;
    int64_t off[3];
    if (r0 + warp < r1) { offs(r0 + warp, off); ring.issue(0, src, off, G); }
    for (int64_t row = r0 + warp; row < r1; row += kWarps, b ^= 1) {
        const int64_t base = row * F + g * G;
        const float r = a.rstd[row * a.ngroups + g];
        if (row + kWarps < r1) { offs(row + kWarps, off); ring.issue(b ^ 1, src, off, G); }
        else tc::cp_async_commit();
        tc::cp_async_wait<1>();
        const float2 r2 = f2(r);
        float2 c1p = f2(0.0f);
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int e0 = (k * 32 + lane) * V;
            if (e0 >= G) continue;
            Raw<T, V> xr, dr, zr;
            xr.ld(ring.at(b, 0, e0));
            dr.ld(ring.at(b, 1, e0));
            if (GATE != kGateNone) zr.ld(ring.at(b, 2, e0));
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float2 xh = xr.pair(m), dy0 = dr.pair(m);
                if (GATE != kGateNone) {
                    const float2 gt = gate2<T>(zr.pair(m)).silu;
                    if (GATE == kGateBefore) xh = mul2(xh, gt);
                    else dy0 = mul2(dy0, gt);
                }
                xh = mul2(xh, r2);
                c1p = fma2(mul2(xh, dy0), wpair<V>(ws, e0, m), c1p);
            }
        }
        const float2 c1 = f2(warp_sum(c1p.x + c1p.y) * inv_g);
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int e0 = (k * 32 + lane) * V;
            if (e0 >= G) continue;
            Raw<T, V> xr, dr, zr, ox, oz;
            // the second read of the stage, ordered after c1 so that the first
            // pass's registers die
            const T* xs = ring.at(b, 0, fresh(e0, c1.x));
            xr.ld(xs);
            dr.ld(xs + GP);
            if (GATE != kGateNone) zr.ld(xs + 2 * GP);
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const float2 xv = xr.pair(m), dv = dr.pair(m), w2 = wpair<V>(ws, e0, m);
                float2 xh = xv, dy0 = dv, gt = f2(1.0f), sg = f2(0.0f), zv = f2(0.0f);
                if (GATE != kGateNone) {
                    zv = zr.pair(m);
                    const Gate2 gg = gate2<T>(zv);
                    gt = gg.silu;
                    sg = gg.sig;
                    if (GATE == kGateBefore) xh = mul2(xh, gt);
                    else dy0 = mul2(dy0, gt);
                }
                xh = mul2(xh, r2);
                // dxb = r (dy0 w - xh c1)
                const float2 dxb = mul2(r2, fma2(mul2(xh, f2(-1.0f)), c1, mul2(dy0, w2)));
                ox.set(m, GATE == kGateBefore ? mul2(dxb, gt) : dxb);
                if (GATE == kGateBefore) {
                    oz.set(m, mul2(mul2(dxb, xv), dsilu2(zv, sg)));
                } else if (GATE == kGateAfter) {
                    float2 y0 = mul2(xh, w2);
                    if (a.has_bias) y0 = add2(y0, wpair<V>(bs, e0, m));
                    oz.set(m, mul2(mul2(dv, y0), dsilu2(zv, sg)));
                }
                dwa[k][m] = fma2(dy0, xh, dwa[k][m]);
                if (a.has_bias) {
                    float2* bp = reinterpret_cast<float2*>(red_b + warp * GP + e0 + 2 * m);
                    *bp = add2(*bp, dy0);
                }
            }
            ox.st(dx + base + e0);
            if (GATE != kGateNone) oz.st(dz + base + e0);
        }
    }
    tc::cp_async_wait<0>();
    __syncthreads();                              // every ring is idle: its space takes the fold
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int e0 = (k * 32 + lane) * V;
#pragma unroll
        for (int m = 0; m < M; ++m) *reinterpret_cast<float2*>(fold + warp * GP + e0 + 2 * m) = dwa[k][m];
    }
    __syncthreads();
    // this row block's column partials: the warps' sums in a fixed order
    for (int f = threadIdx.x; f < G; f += kThreads) {
        float sw = 0.0f, sb = 0.0f;
#pragma unroll
        for (int q = 0; q < kWarps; ++q) {
            sw += fold[q * GP + f];
            if (a.has_bias) sb += red_b[q * GP + f];
        }
        a.dw_part[blockIdx.x * F + g * G + f] = sw;
        if (a.db_part != nullptr) a.db_part[blockIdx.x * F + g * G + f] = sb;
    }
}

// ------------------------------------------------------------ stream path --
// Groups wider than a warp's registers: one CTA per (row block, group), two
// passes per row over strided V-element chunks.
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    __syncthreads();                                  // red[] free
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) s += red[q];
    return s;
}

template <typename T, int V>
__global__ void __launch_bounds__(kThreads)
fwd_stream_kernel(const Args a) {
    __shared__ float red[kWarps];
    const int64_t g = blockIdx.y, G = a.group, F = a.features;
    const int64_t r0 = blockIdx.x * a.rows_per_block, r1 = min64(r0 + a.rows_per_block, a.rows);
    const T* x = static_cast<const T*>(a.x);
    const T* z = static_cast<const T*>(a.z);
    T* out = static_cast<T*>(a.out);
    for (int64_t row = r0; row < r1; ++row) {
        const int64_t base = row * F + g * G, xb = row * a.xs + g * G, zb = row * a.zs + g * G;
        float ss = 0.0f;
        for (int64_t e0 = (int64_t)threadIdx.x * V; e0 < G; e0 += (int64_t)kThreads * V) {
            float xv[V], zv[V];
            VecIo<T, V>::ld(x + xb + e0, xv);
            if (a.gate == kGateBefore) VecIo<T, V>::ld(z + zb + e0, zv);
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const float xb = a.gate == kGateBefore ? xv[i] * zv[i] * sigmoid_t<T>(zv[i]) : xv[i];
                ss = fmaf(xb, xb, ss);
            }
        }
        ss = block_sum(ss, red);
        const float r = rsqrtf(ss / (float)G + a.eps);
        if (a.rstd != nullptr && threadIdx.x == 0) a.rstd[row * a.ngroups + g] = r;
        for (int64_t e0 = (int64_t)threadIdx.x * V; e0 < G; e0 += (int64_t)kThreads * V) {
            float xv[V], zv[V], o[V];
            VecIo<T, V>::ld(x + xb + e0, xv);
            if (a.gate != kGateNone) VecIo<T, V>::ld(z + zb + e0, zv);
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const float gt = a.gate != kGateNone ? zv[i] * sigmoid_t<T>(zv[i]) : 1.0f;
                const float xb = a.gate == kGateBefore ? xv[i] * gt : xv[i];
                const int64_t f = g * G + e0 + i;
                const float y = fmaf(xb * r, a.w[f], a.has_bias ? a.b[f] : 0.0f);
                o[i] = a.gate == kGateAfter ? y * gt : y;
            }
            VecIo<T, V>::st(out + base + e0, o);
        }
    }
}

template <typename T, int V>
__global__ void __launch_bounds__(kThreads)
bwd_stream_kernel(const Args a) {
    __shared__ float red[kWarps];
    const int64_t g = blockIdx.y, G = a.group, F = a.features;
    const int64_t r0 = blockIdx.x * a.rows_per_block, r1 = min64(r0 + a.rows_per_block, a.rows);
    const T* x = static_cast<const T*>(a.x);
    const T* z = static_cast<const T*>(a.z);
    const T* dy = static_cast<const T*>(a.dy);
    T* dx = static_cast<T*>(a.dx);
    T* dz = static_cast<T*>(a.dz);
    float* dwp = a.dw_part + blockIdx.x * F + g * G;
    float* dbp = a.db_part != nullptr ? a.db_part + blockIdx.x * F + g * G : nullptr;
    for (int64_t e0 = (int64_t)threadIdx.x * V; e0 < G; e0 += (int64_t)kThreads * V)
#pragma unroll
        for (int i = 0; i < V; ++i) {
            dwp[e0 + i] = 0.0f;
            if (dbp) dbp[e0 + i] = 0.0f;
        }
    for (int64_t row = r0; row < r1; ++row) {
        const int64_t base = row * F + g * G, xb = row * a.xs + g * G, zb = row * a.zs + g * G;
        const float r = a.rstd[row * a.ngroups + g];
        float c1 = 0.0f;
        for (int64_t e0 = (int64_t)threadIdx.x * V; e0 < G; e0 += (int64_t)kThreads * V) {
            float xv[V], zv[V], dv[V];
            VecIo<T, V>::ld(x + xb + e0, xv);
            VecIo<T, V>::ld(dy + base + e0, dv);
            if (a.gate != kGateNone) VecIo<T, V>::ld(z + zb + e0, zv);
#pragma unroll
            for (int i = 0; i < V; ++i)
                c1 += elem_c1<T>(xv[i], a.gate != kGateNone ? zv[i] : 0.0f, dv[i], a.w[g * G + e0 + i], r, a.gate);
        }
        c1 = block_sum(c1, red) / (float)G;
        for (int64_t e0 = (int64_t)threadIdx.x * V; e0 < G; e0 += (int64_t)kThreads * V) {
            float xv[V], zv[V], dv[V], ox[V], oz[V];
            VecIo<T, V>::ld(x + xb + e0, xv);
            VecIo<T, V>::ld(dy + base + e0, dv);
            if (a.gate != kGateNone) VecIo<T, V>::ld(z + zb + e0, zv);
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const int64_t f = g * G + e0 + i;
                const ElemGrad e = elem_grad<T>(xv[i], a.gate != kGateNone ? zv[i] : 0.0f, dv[i], a.w[f],
                                                a.has_bias ? a.b[f] : 0.0f, r, c1, a.gate);
                ox[i] = e.dx;
                oz[i] = e.dz;
                dwp[e0 + i] = fmaf(e.dy0, e.xh, dwp[e0 + i]);     // this thread's own slots
                if (dbp) dbp[e0 + i] += e.dy0;
            }
            VecIo<T, V>::st(dx + base + e0, ox);
            if (a.gate != kGateNone) VecIo<T, V>::st(dz + base + e0, oz);
        }
    }
}

// dw[f], db[f]: partials of every row block, in order.
__global__ void reduce_kernel(const Args a, float* dw, float* db) {
    for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < a.features;
         f += (int64_t)gridDim.x * blockDim.x) {
        float sw = 0.0f, sb = 0.0f;
        for (int64_t k = 0; k < a.row_blocks; ++k) {
            sw += a.dw_part[k * a.features + f];
            if (a.db_part) sb += a.db_part[k * a.features + f];
        }
        if (dw) dw[f] = sw;
        if (db) db[f] = sb;
    }
}

// ------------------------------------------------------------------- host ----
static int validate(const ssm_gated_rmsnorm_params* p) {
    if (p == nullptr) return fail(SSM_ERR_INVALID, "rmsnorm_gated: null params");
    if (p->rows < 0 || p->features < 1 || p->group_size < 1 || p->features % p->group_size)
        return fail(SSM_ERR_INVALID, "rmsnorm_gated: group_size must divide features");
    if (p->dtype < SSM_F32 || p->dtype > SSM_F16) return fail(SSM_ERR_UNSUPPORTED, "rmsnorm_gated: dtype");
    if (p->gate < kGateNone || p->gate > kGateAfter) return fail(SSM_ERR_INVALID, "rmsnorm_gated: gate mode");
    if (p->features / p->group_size > 65535) return fail(SSM_ERR_UNSUPPORTED, "rmsnorm_gated: too many groups");
    if ((p->x_row_stride && p->x_row_stride < p->features) || (p->z_row_stride && p->z_row_stride < p->features))
        return fail(SSM_ERR_INVALID, "rmsnorm_gated: a row stride is below features");
    return SSM_OK;
}

// Warp path shape: V elements per slot (a 16- or 8-byte access) and NV slots
// per lane, the candidate covering the group with the least padding (V = 0:
// the group takes the stream path, whose vector width is `sv`, 16 bytes or 1).
struct Shape { int v, nv, sv; };
static bool aligned(const void* p, int64_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }
static bool ptrs_ok(const ssm_gated_rmsnorm_params* p, bool bwd, int64_t bytes) {
    if (!aligned(p->x, bytes) || (p->gate && !aligned(p->z, bytes))) return false;
    const int64_t esz = p->dtype == SSM_F32 ? 4 : 2;
    const int64_t xs = p->x_row_stride ? p->x_row_stride : p->features;
    const int64_t zs = p->z_row_stride ? p->z_row_stride : p->features;
    if ((xs * esz) % bytes || (p->gate && (zs * esz) % bytes) || (p->features * esz) % bytes) return false;
    if (!bwd) return aligned(p->out, bytes);
    return aligned(p->dy, bytes) && aligned(p->dx, bytes) && (!p->gate || aligned(p->dz, bytes));
}
static Shape shape_for(const ssm_gated_rmsnorm_params* p, bool bwd) {
    const int64_t esz = p->dtype == SSM_F32 ? 4 : 2, vmax = 16 / esz, G = p->group_size;
    Shape best{0, 0, 1};
    int64_t best_gp = 0;
    const int cand[5][2] = {{(int)vmax, 1}, {(int)vmax, 2}, {(int)vmax, 3}, {(int)vmax, 4}, {(int)vmax / 2, 5}};
    for (const auto& c : cand) {
        const int64_t gp = 32LL * c[0] * c[1];
        if (gp < G || G % c[0] || !ptrs_ok(p, bwd, c[0] * esz)) continue;
        if (best.v == 0 || gp < best_gp) { best = {c[0], c[1], 1}; best_gp = gp; }
    }
    if (best.v == 0) best.sv = ((G * esz) % 16 == 0 && ptrs_ok(p, bwd, 16)) ? (int)vmax : 1;
    return best;
}

template <typename T, int V, int NV, int GATE>
static void launch_warp(const Args& a, bool bwd, cudaStream_t st) {
    dim3 grid((unsigned)a.row_blocks, (unsigned)a.ngroups);
    constexpr int GP = 32 * NV * V;
    const size_t wb = 2 * GP * sizeof(float);
    if (bwd) {
        using Ring = RowRing<T, V, NV, GATE != kGateNone ? 3 : 2>;
        const size_t sm = wb + kWarps * Ring::bytes + (a.has_bias ? kWarps * GP * sizeof(float) : 0);
        auto k = bwd_kernel<T, V, NV, GATE>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        k<<<grid, kThreads, sm, st>>>(a);
    } else {
        using Ring = RowRing<T, V, NV, GATE != kGateNone ? 2 : 1>;
        const size_t sm = wb + kWarps * Ring::bytes;
        auto k = fwd_kernel<T, V, NV, GATE>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        k<<<grid, kThreads, sm, st>>>(a);
    }
}

template <typename T, int V, int NV>
static void launch_gate(const Args& a, bool bwd, cudaStream_t st) {
    switch (a.gate) {
        case kGateNone: launch_warp<T, V, NV, kGateNone>(a, bwd, st); break;
        case kGateBefore: launch_warp<T, V, NV, kGateBefore>(a, bwd, st); break;
        default: launch_warp<T, V, NV, kGateAfter>(a, bwd, st);
    }
}

template <typename T>
static int launch_t(const Args& a, const Shape& s, bool bwd, cudaStream_t st) {
    constexpr int VM = 16 / sizeof(T);
    dim3 grid((unsigned)a.row_blocks, (unsigned)a.ngroups);
    if (s.v == VM) {
        switch (s.nv) {
            case 1: launch_gate<T, VM, 1>(a, bwd, st); break;
            case 2: launch_gate<T, VM, 2>(a, bwd, st); break;
            case 3: launch_gate<T, VM, 3>(a, bwd, st); break;
            default: launch_gate<T, VM, 4>(a, bwd, st);
        }
    } else if (s.v == VM / 2) {
        launch_gate<T, VM / 2, 5>(a, bwd, st);
    } else if (s.sv == VM) {
        if (bwd) bwd_stream_kernel<T, VM><<<grid, kThreads, 0, st>>>(a);
        else fwd_stream_kernel<T, VM><<<grid, kThreads, 0, st>>>(a);
    } else {
        if (bwd) bwd_stream_kernel<T, 1><<<grid, kThreads, 0, st>>>(a);
        else fwd_stream_kernel<T, 1><<<grid, kThreads, 0, st>>>(a);
    }
    return check_launch(bwd ? "rmsnorm_gated bwd" : "rmsnorm_gated fwd");
}

// Row blocks: about four waves of (row block, group) CTAs, and at least one
// row per warp of a CTA.
static void plan(const ssm_gated_rmsnorm_params* p, Args& a) {
    a.rows = p->rows;
    a.features = p->features;
    a.group = p->group_size;
    a.ngroups = p->features / p->group_size;
    a.xs = p->x_row_stride ? p->x_row_stride : p->features;
    a.zs = p->z_row_stride ? p->z_row_stride : p->features;
    const int64_t want = 148 * 4 * 4;
    const int64_t per_group = max64(1, ceil_div(want, a.ngroups));
    a.rows_per_block = max64(kWarps, ceil_div(max64(a.rows, 1), per_group));
    a.row_blocks = max64(1, ceil_div(max64(a.rows, 1), a.rows_per_block));
    a.eps = p->eps;
    a.gate = p->gate;
    a.has_bias = p->flags & SSM_HAS_BIAS;
    a.x = p->x; a.z = p->z; a.w = p->weight; a.b = p->bias;
    a.out = p->out; a.rstd = p->rstd;
    a.dy = p->dy; a.dx = p->dx; a.dz = p->dz;
    a.dw_part = a.db_part = nullptr;
}

static int run(const ssm_gated_rmsnorm_params* p, const Args& a, bool bwd, cudaStream_t st) {
    const Shape s = shape_for(p, bwd);
    switch (p->dtype) {
        case SSM_F32: return launch_t<float>(a, s, bwd, st);
        case SSM_BF16: return launch_t<__nv_bfloat16>(a, s, bwd, st);
        default: return launch_t<__half>(a, s, bwd, st);
    }
}

}  // namespace gnorm
}  // namespace ssm

using namespace ssm;
using namespace ssm::gnorm;

extern "C" int ssm_gated_rmsnorm_sizes(const ssm_gated_rmsnorm_params* p, size_t* workspace_bytes) {
    if (int s = validate(p)) return s;
    Args a;
    plan(p, a);
    if (workspace_bytes) *workspace_bytes = (size_t)(2 * a.row_blocks * a.features) * 4;
    return SSM_OK;
}

extern "C" int ssm_gated_rmsnorm_fwd(const ssm_gated_rmsnorm_params* p, void* stream) {
    if (int s = validate(p)) return s;
    if (p->rows == 0) return SSM_OK;
    if (!p->x || !p->weight || !p->out || (p->gate && !p->z) || ((p->flags & SSM_HAS_BIAS) && !p->bias))
        return fail(SSM_ERR_INVALID, "rmsnorm_gated fwd: null pointer");
    Args a;
    plan(p, a);
    return run(p, a, false, static_cast<cudaStream_t>(stream));
}

extern "C" int ssm_gated_rmsnorm_bwd(const ssm_gated_rmsnorm_params* p, void* stream) {
    if (int s = validate(p)) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (p->rows == 0) {
        if (p->dweight && cudaMemsetAsync(p->dweight, 0, (size_t)p->features * 4, st))
            return check_launch("rmsnorm_gated bwd: zero dweight");
        if (p->dbias && cudaMemsetAsync(p->dbias, 0, (size_t)p->features * 4, st))
            return check_launch("rmsnorm_gated bwd: zero dbias");
        return SSM_OK;
    }
    if (!p->x || !p->weight || !p->dy || !p->dx || !p->rstd || (p->gate && (!p->z || !p->dz)) ||
        ((p->flags & SSM_HAS_BIAS) && !p->bias))
        return fail(SSM_ERR_INVALID, "rmsnorm_gated bwd: null pointer");
    Args a;
    plan(p, a);
    const size_t need = (size_t)(2 * a.row_blocks * a.features) * 4;
    if (!p->workspace || p->workspace_bytes < need)
        return fail(SSM_ERR_WORKSPACE, "rmsnorm_gated bwd: workspace smaller than ssm_gated_rmsnorm_sizes");
    a.dw_part = static_cast<float*>(p->workspace);
    a.db_part = (p->flags & SSM_HAS_BIAS) ? a.dw_part + a.row_blocks * a.features : nullptr;
    if (int s = run(p, a, true, st)) return s;
    reduce_kernel<<<(unsigned)min64(ceil_div(a.features, 256), 148 * 4), 256, 0, st>>>(
        a, p->dweight, (p->flags & SSM_HAS_BIAS) ? p->dbias : nullptr);
    return check_launch("rmsnorm_gated bwd: reduce");
}
