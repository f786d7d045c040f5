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
// Bytes, not flops: x and z (and dy) cross HBM once.  Groups of up to
// 32 * 4 vectors (1024 bf16 / 512 fp32 elements -- Mamba-2's groups are
// d_inner / ngroups, e.g. 640) are held in one warp's registers: one warp per
// (row, group), the sum of squares and c1 by shuffles, no block barrier.  Each
// CTA's warps walk a block of rows of one group; the group's weight and bias
// sit in shared memory, and the backward keeps each warp's dw / db column sums
// in shared memory too (every lane touches only its own columns), adding the
// warps in a fixed order into one partial per (row block, column).  Wider
// groups stream: one CTA per (row block, group) walks each row twice (the sum,
// then the outputs), the second pass re-reading the row from L1/L2, and adds
// its dw / db into its own partial slots.  A last kernel adds the partials in
// order, so the results are bit-reproducible.
#include "common.cuh"

namespace ssm {
namespace gnorm {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kGateNone = 0, kGateBefore = 1, kGateAfter = 2;

struct Args {
    int64_t rows, features, group, ngroups;
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
// Lane slot s = k * 32 + lane (k < NV) covers elements [s V, s V + V).  The
// group's weight and bias sit in shared memory (GP = 32 NV V floats each) in
// lane-major order -- element i of slot (k, lane) at (k V + i) * 32 + lane --
// so a warp's accesses to one (k, i) hit 32 consecutive banks.
template <int V>
__device__ __forceinline__ int lane_major(int f) {
    const int s = f / V, i = f - s * V;
    return ((s >> 5) * V + i) * 32 + (s & 31);
}
template <int V, int NV>
__device__ __forceinline__ void stage_wb(const Args& a, int64_t g, float* ws, float* bs) {
    constexpr int GP = 32 * NV * V;
    for (int f = threadIdx.x; f < GP; f += kThreads) {
        const bool in = f < a.group;
        ws[lane_major<V>(f)] = in ? a.w[g * a.group + f] : 0.0f;
        bs[lane_major<V>(f)] = (in && a.has_bias) ? a.b[g * a.group + f] : 0.0f;
    }
}

template <typename T, int V, int NV>
__global__ void __launch_bounds__(kThreads)
fwd_kernel(const Args a) {
    constexpr int GP = 32 * NV * V;
    __shared__ __align__(16) float ws[GP], bs[GP];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t g = blockIdx.y;
    const int64_t G = a.group, F = a.features;
    const int64_t r0 = blockIdx.x * a.rows_per_block;
    const int64_t r1 = min64(r0 + a.rows_per_block, a.rows);
    const T* x = static_cast<const T*>(a.x);
    const T* z = static_cast<const T*>(a.z);
    T* out = static_cast<T*>(a.out);
    stage_wb<V, NV>(a, g, ws, bs);
    __syncthreads();
    for (int64_t row = r0 + warp; row < r1; row += kWarps) {
        const int64_t base = row * F + g * G;
        float xv[NV][V], gt[NV][V];
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int e0 = (k * 32 + lane) * V;
            if (e0 < G) {
                VecIo<T, V>::ld(x + base + e0, xv[k]);
                if (a.gate != kGateNone) VecIo<T, V>::ld(z + base + e0, gt[k]);
            } else {
#pragma unroll
                for (int i = 0; i < V; ++i) { xv[k][i] = 0.0f; gt[k][i] = 0.0f; }
            }
#pragma unroll
            for (int i = 0; i < V; ++i) {
                if (a.gate != kGateNone) gt[k][i] *= sigmoid_t<T>(gt[k][i]);      // silu(z)
                if (a.gate == kGateBefore) xv[k][i] *= gt[k][i];
                ss = fmaf(xv[k][i], xv[k][i], ss);
            }
        }
        ss = warp_sum(ss);
        const float r = rsqrtf(ss / (float)G + a.eps);
        if (a.rstd != nullptr && lane == 0) a.rstd[row * a.ngroups + g] = r;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int e0 = (k * 32 + lane) * V;
            if (e0 >= G) continue;
            float o[V];
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const int q = (k * V + i) * 32 + lane;
                const float y = fmaf(xv[k][i] * r, ws[q], bs[q]);
                o[i] = a.gate == kGateAfter ? y * gt[k][i] : y;
            }
            VecIo<T, V>::st(out + base + e0, o);
        }
    }
}

// Backward warp path.  Dynamic shared memory: w[GP], b[GP], then per warp the
// dw and db column sums of its rows (acc[warp][2][GP]), all lane-major.
template <typename T, int V, int NV>
__global__ void __launch_bounds__(kThreads)
bwd_kernel(const Args a) {
    constexpr int GP = 32 * NV * V;
    extern __shared__ __align__(16) float sm[];
    float* ws = sm;
    float* bs = sm + GP;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* acc_w = sm + 2 * GP + warp * 2 * GP;
    float* acc_b = acc_w + GP;
    const int64_t g = blockIdx.y;
    const int64_t G = a.group, F = a.features;
    const int64_t r0 = blockIdx.x * a.rows_per_block;
    const int64_t r1 = min64(r0 + a.rows_per_block, a.rows);
    const T* x = static_cast<const T*>(a.x);
    const T* z = static_cast<const T*>(a.z);
    const T* dy = static_cast<const T*>(a.dy);
    T* dx = static_cast<T*>(a.dx);
    T* dz = static_cast<T*>(a.dz);
    stage_wb<V, NV>(a, g, ws, bs);
    for (int i = lane; i < 2 * GP; i += 32) acc_w[i] = 0.0f;
    __syncthreads();
    for (int64_t row = r0 + warp; row < r1; row += kWarps) {
        const int64_t base = row * F + g * G;
        const float r = a.rstd[row * a.ngroups + g];
        float xv[NV][V], zv[NV][V], dv[NV][V];
        float c1 = 0.0f;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int e0 = (k * 32 + lane) * V;
            if (e0 < G) {
                VecIo<T, V>::ld(x + base + e0, xv[k]);
                VecIo<T, V>::ld(dy + base + e0, dv[k]);
                if (a.gate != kGateNone) VecIo<T, V>::ld(z + base + e0, zv[k]);
                else {
#pragma unroll
                    for (int i = 0; i < V; ++i) zv[k][i] = 0.0f;
                }
            } else {
#pragma unroll
                for (int i = 0; i < V; ++i) { xv[k][i] = 0.0f; dv[k][i] = 0.0f; zv[k][i] = 0.0f; }
            }
#pragma unroll
            for (int i = 0; i < V; ++i)
                c1 += elem_c1<T>(xv[k][i], zv[k][i], dv[k][i], ws[(k * V + i) * 32 + lane], r, a.gate);
        }
        c1 = warp_sum(c1) / (float)G;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int e0 = (k * 32 + lane) * V;
            if (e0 >= G) continue;
            float ox[V], oz[V];
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const int q = (k * V + i) * 32 + lane;
                const ElemGrad e = elem_grad<T>(xv[k][i], zv[k][i], dv[k][i], ws[q], bs[q], r, c1, a.gate);
                ox[i] = e.dx;
                oz[i] = e.dz;
                acc_w[q] = fmaf(e.dy0, e.xh, acc_w[q]);
                acc_b[q] += e.dy0;
            }
            VecIo<T, V>::st(dx + base + e0, ox);
            if (a.gate != kGateNone) VecIo<T, V>::st(dz + base + e0, oz);
        }
    }
    __syncthreads();
    // this row block's column partials: the warps' sums in a fixed order
    for (int f = threadIdx.x; f < G; f += kThreads) {
        const int q0 = lane_major<V>(f);
        float sw = 0.0f, sb = 0.0f;
#pragma unroll
        for (int q = 0; q < kWarps; ++q) {
            sw += sm[2 * GP + q * 2 * GP + q0];
            sb += sm[2 * GP + q * 2 * GP + GP + q0];
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
        const int64_t base = row * F + g * G;
        float ss = 0.0f;
        for (int64_t e0 = (int64_t)threadIdx.x * V; e0 < G; e0 += (int64_t)kThreads * V) {
            float xv[V], zv[V];
            VecIo<T, V>::ld(x + base + e0, xv);
            if (a.gate == kGateBefore) VecIo<T, V>::ld(z + base + e0, zv);
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
            VecIo<T, V>::ld(x + base + e0, xv);
            if (a.gate != kGateNone) VecIo<T, V>::ld(z + base + e0, zv);
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
        const int64_t base = row * F + g * G;
        const float r = a.rstd[row * a.ngroups + g];
        float c1 = 0.0f;
        for (int64_t e0 = (int64_t)threadIdx.x * V; e0 < G; e0 += (int64_t)kThreads * V) {
            float xv[V], zv[V], dv[V];
            VecIo<T, V>::ld(x + base + e0, xv);
            VecIo<T, V>::ld(dy + base + e0, dv);
            if (a.gate != kGateNone) VecIo<T, V>::ld(z + base + e0, zv);
#pragma unroll
            for (int i = 0; i < V; ++i)
                c1 += elem_c1<T>(xv[i], a.gate != kGateNone ? zv[i] : 0.0f, dv[i], a.w[g * G + e0 + i], r, a.gate);
        }
        c1 = block_sum(c1, red) / (float)G;
        for (int64_t e0 = (int64_t)threadIdx.x * V; e0 < G; e0 += (int64_t)kThreads * V) {
            float xv[V], zv[V], dv[V], ox[V], oz[V];
            VecIo<T, V>::ld(x + base + e0, xv);
            VecIo<T, V>::ld(dy + base + e0, dv);
            if (a.gate != kGateNone) VecIo<T, V>::ld(z + base + e0, zv);
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
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int validate(const ssm_gated_rmsnorm_params* p) {
    if (p == nullptr) return fail(SSM_ERR_INVALID, "rmsnorm_gated: null params");
    if (p->rows < 0 || p->features < 1 || p->group_size < 1 || p->features % p->group_size)
        return fail(SSM_ERR_INVALID, "rmsnorm_gated: group_size must divide features");
    if (p->dtype < SSM_F32 || p->dtype > SSM_F16) return fail(SSM_ERR_UNSUPPORTED, "rmsnorm_gated: dtype");
    if (p->gate < kGateNone || p->gate > kGateAfter) return fail(SSM_ERR_INVALID, "rmsnorm_gated: gate mode");
    if (p->features / p->group_size > 65535) return fail(SSM_ERR_UNSUPPORTED, "rmsnorm_gated: too many groups");
    return SSM_OK;
}

// Vector width (elements per 16-byte access, or 1) and vectors per lane of
// the warp path (0: the group needs the stream path).
struct Shape { int v, nv; };
static Shape shape_for(const ssm_gated_rmsnorm_params* p, bool vec) {
    const int V = vec ? (p->dtype == SSM_F32 ? 4 : 8) : 1;
    const int64_t slots = ceil_div(p->group_size, V);
    for (int nv : {1, 2, 3, 4}) if (slots <= 32 * nv) return {V, nv};
    return {V, 0};
}

static bool vec_ok(const ssm_gated_rmsnorm_params* p, bool bwd) {
    const int64_t esz = p->dtype == SSM_F32 ? 4 : 2;
    if ((p->group_size * esz) % 16) return false;
    if (!aligned16(p->x) || (p->gate && !aligned16(p->z))) return false;
    if (!bwd) return aligned16(p->out);
    return aligned16(p->dy) && aligned16(p->dx) && (!p->gate || aligned16(p->dz));
}

template <typename T, int V, int NV>
static void launch_warp(const Args& a, bool bwd, cudaStream_t st) {
    dim3 grid((unsigned)a.row_blocks, (unsigned)a.ngroups);
    if (bwd) {
        constexpr int GP = 32 * NV * V;
        const size_t sm = (size_t)(2 * GP + kWarps * 2 * GP) * sizeof(float);
        auto k = bwd_kernel<T, V, NV>;
        if (sm > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        k<<<grid, kThreads, sm, st>>>(a);
    } else {
        fwd_kernel<T, V, NV><<<grid, kThreads, 0, st>>>(a);
    }
}

template <typename T, int V>
static void launch_v(const Args& a, int nv, bool bwd, cudaStream_t st) {
    switch (nv) {
        case 1: launch_warp<T, V, 1>(a, bwd, st); break;
        case 2: launch_warp<T, V, 2>(a, bwd, st); break;
        case 3: launch_warp<T, V, 3>(a, bwd, st); break;
        case 4: launch_warp<T, V, 4>(a, bwd, st); break;
        default: {
            dim3 grid((unsigned)a.row_blocks, (unsigned)a.ngroups);
            if (bwd) bwd_stream_kernel<T, V><<<grid, kThreads, 0, st>>>(a);
            else fwd_stream_kernel<T, V><<<grid, kThreads, 0, st>>>(a);
        }
    }
}

template <typename T>
static int launch_t(const Args& a, const Shape& s, bool bwd, cudaStream_t st) {
    if (s.v == 1) launch_v<T, 1>(a, s.nv, bwd, st);
    else launch_v<T, 16 / sizeof(T)>(a, s.nv, bwd, st);
    return check_launch(bwd ? "rmsnorm_gated bwd" : "rmsnorm_gated fwd");
}

// Row blocks: about four waves of (row block, group) CTAs, and at least one
// row per warp of a CTA.
static void plan(const ssm_gated_rmsnorm_params* p, Args& a) {
    a.rows = p->rows;
    a.features = p->features;
    a.group = p->group_size;
    a.ngroups = p->features / p->group_size;
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
    const Shape s = shape_for(p, vec_ok(p, bwd));
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
