// Mamba-2 decode state update (one token), forward and backward, for sm_100a.
//
// Reference behaviour: src/metal_kernelops/cv/mamba2_state.py:759-849.  One step
//
//     d  = softplus(dt + dt_bias)      (optional bias / softplus)
//     a  = exp(A_h * d)
//     s' = a * s + d * x * B[g]        (g = h / (nheads / ngroups))
//     y  = (<s', C[g]> + D * x) * silu(z)
//
// The state is (batch, nheads, headdim, dstate); each (b, h, p) is a "row" of
// dstate elements.  The op is a pure streaming read-modify-write of the fp32
// state, so the kernel is built for HBM bandwidth: one CTA per (batch, head),
// one warp per row with 16-byte vector accesses along dstate, four rows in
// flight per warp, B/C/dt/decay shared by the whole CTA.  new_state may alias
// state: every element is read and then written by the same thread.
//
// The backward (fp32, like the reference's, :71-75) keeps every reduction
// deterministic: per-(batch, head) partials of dB, dC, dA, d dt and dD are
// folded in registers and shared memory inside the CTA, then a second kernel
// adds them over heads / batch in a fixed order.  No atomics.
#include <mutex>
#include <string>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace ssm {
namespace supd {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct Args {
    int64_t batch, nheads, headdim, dstate, ngroups;
    uint32_t flags;
    const void* state; const void* x; const void* dt; const float* A; const void* B; const void* C;
    const float* D; const void* z; const float* dt_bias;
    void* new_state; void* y;
    const float* dy; const float* dnew;
    float* grad_state; float* dx; float* ddt; float* dz;
    float* dBp; float* dCp;         // (batch, nheads, dstate)
    float* dAp; float* dbp;         // (batch, nheads)
    float* dDp;                     // (batch, nheads) or (batch, nheads, headdim)
};

template <typename T, int VEC> struct Vec;
template <typename T> struct Vec<T, 1> {
    static __device__ __forceinline__ void ld(const T* p, float* v) { v[0] = ldf(p); }
    static __device__ __forceinline__ void st(T* p, const float* v) { stf(p, v[0]); }
};
template <> struct Vec<float, 4> {
    static __device__ __forceinline__ void ld(const float* p, float* v) {
        const float4 q = *reinterpret_cast<const float4*>(p);
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    }
    static __device__ __forceinline__ void st(float* p, const float* v) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
};
template <> struct Vec<__nv_bfloat16, 4> {
    static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float* v) {
        const uint2 q = *reinterpret_cast<const uint2*>(p);
        const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&q.x);
        const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&q.y);
        const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
        v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
    }
    static __device__ __forceinline__ void st(__nv_bfloat16* p, const float* v) {
        __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
        __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
        uint2 q;
        q.x = *reinterpret_cast<uint32_t*>(&a);
        q.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(p) = q;
    }
};
template <> struct Vec<__half, 4> {
    static __device__ __forceinline__ void ld(const __half* p, float* v) {
        const uint2 q = *reinterpret_cast<const uint2*>(p);
        const __half2 a = *reinterpret_cast<const __half2*>(&q.x);
        const __half2 b = *reinterpret_cast<const __half2*>(&q.y);
        const float2 fa = __half22float2(a), fb = __half22float2(b);
        v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
    }
    static __device__ __forceinline__ void st(__half* p, const float* v) {
        __half2 a = __floats2half2_rn(v[0], v[1]);
        __half2 b = __floats2half2_rn(v[2], v[3]);
        uint2 q;
        q.x = *reinterpret_cast<uint32_t*>(&a);
        q.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(p) = q;
    }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------------ forward --
// Phase 0: the first P threads compute each row's decay a = exp(A d) and input
// coefficient d x into shared memory (d per row or per head).  Phase 1: warp w
// owns rows w*kFwdRows ... and issues all of its state loads for one dstate
// slice before any arithmetic, so every thread keeps kFwdRows 16-byte loads in
// flight; the register cap (80) keeps three CTAs resident per SM, which puts
// about 96 KB of state reads in flight per SM.
constexpr int kFwdRows = 8;

// T: state, dt and y; TI: x, B, C and z (T, or 16-bit against an fp32 state).
template <typename T, typename TI, int VEC>
__global__ void __launch_bounds__(kThreads, 3)
fwd_kernel(const Args a) {
    extern __shared__ float s_rows[];   // [2][headdim]: decay, d*x
    const int64_t bh = blockIdx.x;
    const int64_t b = bh / a.nheads, h = bh % a.nheads;
    const int64_t g = h / (a.nheads / a.ngroups);
    const int P = (int)a.headdim, N = (int)a.dstate;   // one CTA's P*N fits in int
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool per_row = a.flags & SSM_DT_PER_ROW, has_bias = a.flags & SSM_HAS_BIAS;
    const bool softplus = a.flags & SSM_SOFTPLUS, has_d = a.flags & SSM_HAS_D;
    const bool d_per_head = a.flags & SSM_D_PER_HEAD, has_z = a.flags & SSM_HAS_Z;
    const T* st = reinterpret_cast<const T*>(a.state) + bh * (int64_t)P * N;
    T* ns = reinterpret_cast<T*>(a.new_state) + bh * (int64_t)P * N;
    const TI* Bg = reinterpret_cast<const TI*>(a.B) + (b * a.ngroups + g) * N;
    const TI* Cg = reinterpret_cast<const TI*>(a.C) + (b * a.ngroups + g) * N;
    const TI* xg = reinterpret_cast<const TI*>(a.x) + bh * (int64_t)P;
    const T* dtg = reinterpret_cast<const T*>(a.dt);
    const TI* zg = reinterpret_cast<const TI*>(a.z) + bh * (int64_t)P;
    T* yg = reinterpret_cast<T*>(a.y) + bh * (int64_t)P;
    const float Ah = a.A[h];
    const float bias = has_bias ? a.dt_bias[h] : 0.0f;
    float* s_decay = s_rows;
    float* s_dx = s_rows + P;

    for (int p = threadIdx.x; p < P; p += kThreads) {
        const float raw = ldf(per_row ? dtg + bh * (int64_t)P + p : dtg + bh) + bias;
        const float d = softplus ? softplus_f(raw) : raw;
        s_decay[p] = expf(Ah * d);
        s_dx[p] = d * ldf(xg + p);
    }
    __syncthreads();

    for (int p0 = warp * kFwdRows; p0 < P; p0 += kWarps * kFwdRows) {
        const int nr = min(kFwdRows, P - p0);
        float acc[kFwdRows];
#pragma unroll
        for (int r = 0; r < kFwdRows; ++r) acc[r] = 0.0f;
        for (int n = lane * VEC; n < N; n += 32 * VEC) {
            float sv[kFwdRows][VEC];
#pragma unroll
            for (int r = 0; r < kFwdRows; ++r)
                if (r < nr) Vec<T, VEC>::ld(st + (p0 + r) * N + n, sv[r]);
            float bv[VEC], cv[VEC];
            Vec<TI, VEC>::ld(Bg + n, bv);
            Vec<TI, VEC>::ld(Cg + n, cv);
#pragma unroll
            for (int r = 0; r < kFwdRows; ++r) {
                if (r < nr) {
                    const float dc = s_decay[p0 + r], dx = s_dx[p0 + r];
                    float out[VEC];
#pragma unroll
                    for (int k = 0; k < VEC; ++k) {
                        out[k] = fmaf(dc, sv[r][k], dx * bv[k]);
                        acc[r] = fmaf(out[k], cv[k], acc[r]);
                    }
                    Vec<T, VEC>::st(ns + (p0 + r) * N + n, out);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kFwdRows; ++r) acc[r] = warp_sum(acc[r]);
        // lane r finishes row p0 + r
        float tot = acc[0];
#pragma unroll
        for (int r = 1; r < kFwdRows; ++r)
            if (lane == r) tot = acc[r];
        if (lane < nr) {
            const int p = p0 + lane;
            float out = tot;
            if (has_d) out = fmaf(ldf(xg + p), d_per_head ? a.D[h * (int64_t)P + p] : a.D[h], out);
            if (has_z) {
                const float zv = ldf(zg + p);
                out *= zv * sigmoid_f(zv);
            }
            stf(yg + p, out);
        }
    }
}

// ----------------------------------------------------------------- backward --
// All inputs fp32 (the wrapper widens them).  One CTA per (batch, head).
template <int VEC>
__global__ void __launch_bounds__(kThreads)
bwd_kernel(const Args a) {
    extern __shared__ __align__(16) float sh[];   // [kWarps][2][N] + [kWarps][4]
    const int64_t bh = blockIdx.x;
    const int64_t b = bh / a.nheads, h = bh % a.nheads;
    const int64_t g = h / (a.nheads / a.ngroups);
    const int64_t P = a.headdim, N = a.dstate;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool per_row = a.flags & SSM_DT_PER_ROW, has_bias = a.flags & SSM_HAS_BIAS;
    const bool softplus = a.flags & SSM_SOFTPLUS, has_d = a.flags & SSM_HAS_D;
    const bool d_per_head = a.flags & SSM_D_PER_HEAD, has_z = a.flags & SSM_HAS_Z;
    const bool has_dy = a.flags & SSM_HAS_DY, has_dnew = a.flags & SSM_HAS_DSTATE;
    const float* st = reinterpret_cast<const float*>(a.state);
    const float* Bg = reinterpret_cast<const float*>(a.B) + (b * a.ngroups + g) * N;
    const float* Cg = reinterpret_cast<const float*>(a.C) + (b * a.ngroups + g) * N;
    const float* xg = reinterpret_cast<const float*>(a.x);
    const float* dtg = reinterpret_cast<const float*>(a.dt);
    const float* zg = reinterpret_cast<const float*>(a.z);
    const float Ah = a.A[h];
    const float bias = has_bias ? a.dt_bias[h] : 0.0f;
    float* shB = sh;                         // [kWarps][N]
    float* shC = sh + kWarps * N;            // [kWarps][N]
    float* shH = sh + 2 * kWarps * N;        // [kWarps][4]: dA, d dt (per head), dD (per head)

    float raw_head = 0.0f, d_head = 0.0f;
    if (!per_row) {
        raw_head = dtg[bh] + bias;
        d_head = softplus ? softplus_f(raw_head) : raw_head;
    }
    // per-lane dB/dC partial sums over this warp's rows
    constexpr int MAXE = 8;   // up to 32 * VEC * MAXE elements of dstate per lane
    float pB[MAXE][VEC], pC[MAXE][VEC];
#pragma unroll
    for (int e = 0; e < MAXE; ++e)
#pragma unroll
        for (int k = 0; k < VEC; ++k) { pB[e][k] = 0.0f; pC[e][k] = 0.0f; }
    float hA = 0.0f, hT = 0.0f, hD = 0.0f;   // per-warp sums of dA, d dt, dD (lane 0)

    for (int64_t p = warp; p < P; p += kWarps) {
        const int64_t row = bh * P + p;
        float raw = raw_head, d = d_head;
        if (per_row) {
            raw = dtg[row] + bias;
            d = softplus ? softplus_f(raw) : raw;
        }
        const float av = expf(Ah * d);
        const float xv = xg[row];
        const float dyv = has_dy ? a.dy[row] : 0.0f;
        float sg = 1.0f, zv = 0.0f, gate = 1.0f;
        if (has_z) { zv = zg[row]; sg = sigmoid_f(zv); gate = zv * sg; }
        const float dyp = dyv * gate;
        const float dv_skip = has_d ? (d_per_head ? a.D[h * P + p] : a.D[h]) : 0.0f;
        float sdx = 0.0f, sdd = 0.0f, sda = 0.0f, sy = 0.0f;
        int e = 0;
        for (int64_t n = (int64_t)lane * VEC; n < N; n += 32 * VEC, ++e) {
            float sv[VEC], bv[VEC], cv[VEC], dn[VEC], out[VEC];
            Vec<float, VEC>::ld(st + row * N + n, sv);
            Vec<float, VEC>::ld(Bg + n, bv);
            Vec<float, VEC>::ld(Cg + n, cv);
            if (has_dnew) Vec<float, VEC>::ld(a.dnew + row * N + n, dn);
            else {
#pragma unroll
                for (int k = 0; k < VEC; ++k) dn[k] = 0.0f;
            }
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                const float ns = fmaf(av, sv[k], d * xv * bv[k]);   // new state, recomputed
                const float qv = fmaf(dyp, cv[k], dn[k]);
                out[k] = qv * av;
                sdx = fmaf(qv, d * bv[k], sdx);
                sdd = fmaf(qv, xv * bv[k], sdd);
                sda = fmaf(qv, sv[k], sda);
                sy = fmaf(ns, cv[k], sy);
#pragma unroll
                for (int ee = 0; ee < MAXE; ++ee) {
                    if (ee == e) {
                        pB[ee][k] = fmaf(qv, d * xv, pB[ee][k]);
                        pC[ee][k] = fmaf(dyp, ns, pC[ee][k]);
                    }
                }
            }
            Vec<float, VEC>::st(a.grad_state + row * N + n, out);
        }
        sdx = warp_sum(sdx);
        sdd = warp_sum(sdd);
        sda = warp_sum(sda);
        sy = warp_sum(sy);
        if (lane == 0) {
            a.dx[row] = fmaf(dyp, dv_skip, sdx);
            const float dA_row = sda * av * d;
            float dd = fmaf(sda * av, Ah, sdd);
            hA += dA_row;
            const float dD_row = dyp * xv;
            if (has_d) {
                if (d_per_head) a.dDp[row] = dD_row;
                else hD += dD_row;
            }
            if (per_row) {
                if (softplus) dd *= softplus_grad_f(raw);
                a.ddt[row] = dd;
                hT += dd;
            } else {
                hT += dd;
            }
            if (has_z) {
                const float ypre = fmaf(xv, dv_skip, sy);
                a.dz[row] = dyv * ypre * sg * fmaf(zv, 1.0f - sg, 1.0f);
            }
        }
    }
    // fold the warps: dB/dC per (b, h), per-head scalars
    {
        int e = 0;
        for (int64_t n = (int64_t)lane * VEC; n < N; n += 32 * VEC, ++e) {
#pragma unroll
            for (int ee = 0; ee < MAXE; ++ee) {
                if (ee == e) {
#pragma unroll
                    for (int k = 0; k < VEC; ++k) {
                        shB[warp * N + n + k] = pB[ee][k];
                        shC[warp * N + n + k] = pC[ee][k];
                    }
                }
            }
        }
    }
    if (lane == 0) {
        shH[warp * 4 + 0] = hA;
        shH[warp * 4 + 1] = hT;
        shH[warp * 4 + 2] = hD;
    }
    __syncthreads();
    for (int64_t n = threadIdx.x; n < N; n += kThreads) {
        float sb = 0.0f, sc = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) { sb += shB[w * N + n]; sc += shC[w * N + n]; }
        a.dBp[bh * N + n] = sb;
        a.dCp[bh * N + n] = sc;
    }
    if (threadIdx.x == 0) {
        float sA = 0.0f, sT = 0.0f, sD = 0.0f;
        for (int w = 0; w < kWarps; ++w) { sA += shH[w * 4]; sT += shH[w * 4 + 1]; sD += shH[w * 4 + 2]; }
        a.dAp[bh] = sA;
        if (!per_row) {
            const float ddt = softplus ? sT * softplus_grad_f(raw_head) : sT;
            a.ddt[bh] = ddt;
            a.dbp[bh] = ddt;
        } else {
            a.dbp[bh] = sT;
        }
        if (has_d && !d_per_head) a.dDp[bh] = sD;
    }
}

// dB/dC over the heads of a group, dA / d dt_bias / dD over the batch.
__global__ void reduce_kernel(const Args a, float* dB, float* dC, float* dA, float* db, float* dD) {
    const int64_t H = a.nheads, N = a.dstate, P = a.headdim;
    const int64_t hpg = H / a.ngroups;
    const bool d_per_head = a.flags & SSM_D_PER_HEAD, has_d = a.flags & SSM_HAS_D;
    const int64_t nbc = a.batch * a.ngroups * N;
    const int64_t nd = has_d ? (d_per_head ? H * P : H) : 0;
    const int64_t total = nbc + 2 * H + nd;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (i < nbc) {
            const int64_t n = i % N, g = (i / N) % a.ngroups, b = i / (N * a.ngroups);
            float sb = 0.0f, sc = 0.0f;
            for (int64_t k = 0; k < hpg; ++k) {
                const int64_t off = (b * H + g * hpg + k) * N + n;
                sb += a.dBp[off];
                sc += a.dCp[off];
            }
            dB[i] = sb;
            dC[i] = sc;
        } else if (i < nbc + 2 * H) {
            const int64_t k = i - nbc;
            const bool is_a = k < H;
            const int64_t h = is_a ? k : k - H;
            const float* src = is_a ? a.dAp : a.dbp;
            float s = 0.0f;
            for (int64_t b = 0; b < a.batch; ++b) s += src[b * H + h];
            if (is_a) dA[h] = s;
            else if (db) db[h] = s;
        } else {
            const int64_t k = i - nbc - 2 * H;
            float s = 0.0f;
            for (int64_t b = 0; b < a.batch; ++b) s += a.dDp[b * nd + k];
            dD[k] = s;
        }
    }
}

// Per-head d dt (dt given per head) when dt is per row: nothing to do; the
// per-row ddt is written by bwd_kernel.

// mode: 0 = size query (inputs only), 1 = forward, 2 = backward
static int validate(const ssm_state_update_params* p, int mode) {
    const bool bwd = mode == 2;
    if (!p) return fail(SSM_ERR_INVALID, "null params");
    if (p->batch < 0 || p->nheads < 1 || p->headdim < 0 || p->dstate < 1 || p->ngroups < 1)
        return fail(SSM_ERR_INVALID, "state_update: bad sizes");
    if (p->nheads % p->ngroups) return fail(SSM_ERR_INVALID, "state_update: ngroups must divide nheads");
    if (p->dtype < 0 || p->dtype > 2) return fail(SSM_ERR_UNSUPPORTED, "state_update: unknown dtype");
    if ((p->flags & SSM_IO_DTYPE) && p->io_dtype != p->dtype) {
        if (mode != 1) return fail(SSM_ERR_UNSUPPORTED, "state_update: io_dtype is for the forward only");
        if (p->dtype != SSM_F32 || (p->io_dtype != SSM_BF16 && p->io_dtype != SSM_F16))
            return fail(SSM_ERR_UNSUPPORTED, "state_update: io_dtype must be bf16/f16 against an fp32 state");
    }
    if (p->dstate > 32 * 4 * 8) return fail(SSM_ERR_UNSUPPORTED, "state_update: dstate above 1024");
    if (p->batch * p->nheads > 0x7fffffffLL) return fail(SSM_ERR_UNSUPPORTED, "state_update: batch*nheads too large");
    const bool empty = p->batch == 0 || p->headdim == 0;
    if (!empty && (!p->state || !p->x || !p->dt || !p->A || !p->B || !p->C))
        return fail(SSM_ERR_INVALID, "state_update: null input");
    if (bwd && !empty && (!p->grad_state || !p->dx || !p->ddt || !p->dA || !p->dB || !p->dC))
        return fail(SSM_ERR_INVALID, "state_update bwd: null gradient pointer");
    if (mode == 1 && !empty && (!p->new_state || !p->y)) return fail(SSM_ERR_INVALID, "state_update: null output");
    return SSM_OK;
}

static void make_args(const ssm_state_update_params* p, Args& a) {
    a.batch = p->batch; a.nheads = p->nheads; a.headdim = p->headdim; a.dstate = p->dstate;
    a.ngroups = p->ngroups; a.flags = p->flags;
    a.state = p->state; a.x = p->x; a.dt = p->dt; a.A = p->A; a.B = p->B; a.C = p->C;
    a.D = p->D; a.z = p->z; a.dt_bias = p->dt_bias; a.new_state = p->new_state; a.y = p->y;
    a.dy = p->dy; a.dnew = p->dnew; a.grad_state = p->grad_state; a.dx = p->dx; a.ddt = p->ddt;
    a.dz = p->dz;
    a.dBp = a.dCp = a.dAp = a.dbp = a.dDp = nullptr;
}

struct Ws { size_t bc, h, dd, total; };
static Ws ws_layout(const ssm_state_update_params* p) {
    Ws w;
    w.bc = align_up((size_t)(p->batch * p->nheads * p->dstate) * 4, 256);
    w.h = align_up((size_t)(p->batch * p->nheads) * 4, 256);
    w.dd = align_up((size_t)(p->batch * p->nheads * p->headdim) * 4, 256);
    w.total = 2 * w.bc + 2 * w.h + w.dd;
    return w;
}

static bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

template <typename T, typename TI>
static int launch_fwd(const Args& a, bool vec, cudaStream_t s) {
    const unsigned grid = (unsigned)(a.batch * a.nheads);
    const size_t smem = 2 * (size_t)a.headdim * sizeof(float);
    if (vec) {
        if (smem > 48 * 1024) cudaFuncSetAttribute(fwd_kernel<T, TI, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        fwd_kernel<T, TI, 4><<<grid, kThreads, smem, s>>>(a);
    } else {
        if (smem > 48 * 1024) cudaFuncSetAttribute(fwd_kernel<T, TI, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        fwd_kernel<T, TI, 1><<<grid, kThreads, smem, s>>>(a);
    }
    return check_launch("state_update fwd");
}

}  // namespace supd
}  // namespace ssm

using namespace ssm;
using namespace ssm::supd;

extern "C" int ssm_state_update_sizes(const ssm_state_update_params* p, size_t* workspace_bytes) {
    if (int s = validate(p, 0)) return s;
    if (workspace_bytes) *workspace_bytes = ws_layout(p).total;
    return SSM_OK;
}

extern "C" int ssm_state_update_fwd(const ssm_state_update_params* p, void* stream) {
    if (int s = validate(p, 1)) return s;
    if (p->batch == 0 || p->headdim == 0) return SSM_OK;
    Args a;
    make_args(p, a);
    const int io = (p->flags & SSM_IO_DTYPE) ? p->io_dtype : p->dtype;
    const size_t esz = p->dtype == SSM_F32 ? 4 : 2, isz = io == SSM_F32 ? 4 : 2;
    // 4-element vectors need dstate % 4 == 0 and 4*size-byte aligned rows
    const bool vec = p->dstate % 4 == 0 &&
                     ((reinterpret_cast<uintptr_t>(p->state) | reinterpret_cast<uintptr_t>(p->new_state)) %
                      (4 * esz)) == 0 &&
                     ((reinterpret_cast<uintptr_t>(p->B) | reinterpret_cast<uintptr_t>(p->C)) % (4 * isz)) == 0;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (io != p->dtype) {   // validated: 16-bit inputs against an fp32 state
        if (io == SSM_BF16) return launch_fwd<float, __nv_bfloat16>(a, vec, s);
        return launch_fwd<float, __half>(a, vec, s);
    }
    switch (p->dtype) {
        case SSM_F32: return launch_fwd<float, float>(a, vec, s);
        case SSM_BF16: return launch_fwd<__nv_bfloat16, __nv_bfloat16>(a, vec, s);
        default: return launch_fwd<__half, __half>(a, vec, s);
    }
}

extern "C" int ssm_state_update_bwd(const ssm_state_update_params* p, void* stream) {
    if (int s = validate(p, 2)) return s;
    if (p->dtype != SSM_F32) return fail(SSM_ERR_UNSUPPORTED, "state_update bwd: inputs must be widened to fp32");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const bool has_d = p->flags & SSM_HAS_D, d_per_head = p->flags & SSM_D_PER_HEAD;
    if (p->batch == 0 || p->headdim == 0) {
        cudaMemsetAsync(p->dA, 0, (size_t)p->nheads * 4, s);
        if ((p->flags & SSM_HAS_BIAS) && p->ddt_bias) cudaMemsetAsync(p->ddt_bias, 0, (size_t)p->nheads * 4, s);
        if (has_d && p->dD)
            cudaMemsetAsync(p->dD, 0, (size_t)(d_per_head ? p->nheads * p->headdim : p->nheads) * 4, s);
        const size_t nbc = (size_t)(p->batch * p->ngroups * p->dstate) * 4;
        if (nbc) { cudaMemsetAsync(p->dB, 0, nbc, s); cudaMemsetAsync(p->dC, 0, nbc, s); }
        if (!(p->flags & SSM_DT_PER_ROW) && p->batch)
            cudaMemsetAsync(p->ddt, 0, (size_t)(p->batch * p->nheads) * 4, s);
        return check_launch("state_update bwd: memset");
    }
    Args a;
    make_args(p, a);
    const Ws w = ws_layout(p);
    if (!p->workspace || p->workspace_bytes < w.total)
        return fail(SSM_ERR_WORKSPACE, "state_update bwd: workspace too small");
    char* ws = reinterpret_cast<char*>(p->workspace);
    a.dBp = reinterpret_cast<float*>(ws);
    a.dCp = reinterpret_cast<float*>(ws + w.bc);
    a.dAp = reinterpret_cast<float*>(ws + 2 * w.bc);
    a.dbp = reinterpret_cast<float*>(ws + 2 * w.bc + w.h);
    a.dDp = reinterpret_cast<float*>(ws + 2 * w.bc + 2 * w.h);
    const bool vec = p->dstate % 4 == 0 && aligned16(p->state) && aligned16(p->B) && aligned16(p->C) &&
                     aligned16(p->grad_state) && (!(p->flags & SSM_HAS_DSTATE) || aligned16(p->dnew));
    const int64_t per_lane = ceil_div(p->dstate, 32 * (vec ? 4 : 1));
    if (per_lane > 8) return fail(SSM_ERR_UNSUPPORTED, "state_update bwd: dstate too large");
    const size_t smem = (2 * (size_t)kWarps * p->dstate + kWarps * 4) * 4;
    const unsigned grid = (unsigned)(p->batch * p->nheads);
    if (vec) {
        if (smem > 48 * 1024) cudaFuncSetAttribute(bwd_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        bwd_kernel<4><<<grid, kThreads, smem, s>>>(a);
    } else {
        if (smem > 48 * 1024) cudaFuncSetAttribute(bwd_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        bwd_kernel<1><<<grid, kThreads, smem, s>>>(a);
    }
    if (int st = check_launch("state_update bwd")) return st;
    const int64_t nd = has_d ? (d_per_head ? p->nheads * p->headdim : p->nheads) : 0;
    const int64_t total = p->batch * p->ngroups * p->dstate + 2 * p->nheads + nd;
    const int blocks = (int)min64(ceil_div(total, 256), 148 * 8);
    reduce_kernel<<<blocks, 256, 0, s>>>(a, p->dB, p->dC, p->dA,
                                         (p->flags & SSM_HAS_BIAS) ? p->ddt_bias : nullptr,
                                         has_d ? p->dD : nullptr);
    return check_launch("state_update bwd: reduce");
}

// ----------------------------------------------------------------------------
// Backward without any allocation.
//
// For callers that cannot call cudaMalloc (or any allocating routine) on the
// path where they run the decode backward -- for example a runtime whose memory
// is fully pre-planned and owned by someone else, or code that must not touch
// the device allocator at that point -- this entry point takes its scratch from
// one fixed array compiled into the library instead of from a caller-supplied
// workspace.  The array is a file-scope __device__ object: every GPU that loads
// the library holds its kStaticScratchBytes until the process exits.
//
// Only host code needs the array's device address.  In host code the symbol
// `g_static_scratch` names a host-side stand-in, not device memory, so its
// address is looked up with cudaGetSymbolAddress in the context current on the
// calling thread, on the first call made in that context, and cached under the
// context's unique id (cuCtxGetId: never reused within the process).  A new
// context -- after cudaDeviceReset, or a different context made current through
// the driver API -- therefore gets its own lookup instead of a stale address.
// The first call in a context should happen before any stream capture.
//
// All calls on a device share the one array, and it keeps whatever the last
// call left in it.  The backward writes every scratch element it later reads
// within the same call, so nothing needs clearing between calls.  Calls whose
// kernels overlap on the GPU (different streams, or concurrent host threads)
// race on the array: serialise them.
namespace ssm {
namespace supd {

constexpr size_t kStaticScratchBytes = SSM_STATE_UPDATE_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// (context id, device address of g_static_scratch in it); a fixed table, so
// the lookup allocates nothing either; when full, the oldest entry is replaced
constexpr int kCtxSlots = 64;
struct CtxAddr { unsigned long long id; void* addr; };
static std::mutex g_static_mu;
static CtxAddr g_static_addr[kCtxSlots];
static int g_static_used = 0, g_static_next = 0;

static PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
static PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;

// The unique id of the context current on this thread (0 when none is).
static int current_context_id(unsigned long long* id) {
    if (!g_ctx_current || !g_ctx_id) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !f)
            return fail(SSM_ERR_CUDA, "state_update bwd_noalloc: cuCtxGetCurrent unavailable");
        g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !f)
            return fail(SSM_ERR_CUDA, "state_update bwd_noalloc: cuCtxGetId unavailable");
        g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(f);
    }
    CUcontext ctx = nullptr;
    if (g_ctx_current(&ctx) != CUDA_SUCCESS)
        return fail(SSM_ERR_CUDA, "state_update bwd_noalloc: cuCtxGetCurrent failed");
    *id = 0;
    if (ctx && g_ctx_id(ctx, id) != CUDA_SUCCESS)
        return fail(SSM_ERR_CUDA, "state_update bwd_noalloc: cuCtxGetId failed");
    return SSM_OK;
}

static int static_scratch(void** out) {
    std::lock_guard<std::mutex> lock(g_static_mu);
    unsigned long long id = 0;
    if (int s = current_context_id(&id)) return s;
    for (int i = 0; id != 0 && i < g_static_used; ++i)
        if (g_static_addr[i].id == id) {
            *out = g_static_addr[i].addr;
            return SSM_OK;
        }
    // first call in this context (or none is current yet: the runtime makes the
    // device's primary context current during the lookup)
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_static_scratch);
    if (e != cudaSuccess || addr == nullptr)
        return fail(SSM_ERR_CUDA, std::string("state_update bwd_noalloc: cudaGetSymbolAddress: ") +
                                      cudaGetErrorString(e));
    if (id == 0 && (current_context_id(&id) != SSM_OK || id == 0)) {
        *out = addr;          // no context id to cache it under: use it uncached
        return SSM_OK;
    }
    const int slot = g_static_used < kCtxSlots ? g_static_used++ : (g_static_next++ % kCtxSlots);
    g_static_addr[slot] = {id, addr};
    *out = addr;
    return SSM_OK;
}

}  // namespace supd
}  // namespace ssm

extern "C" int ssm_state_update_bwd_noalloc(const ssm_state_update_params* p, void* stream) {
    if (int s = validate(p, 2)) return s;
    const size_t need = ws_layout(p).total;
    if (need > kStaticScratchBytes)
        return fail(SSM_ERR_UNSUPPORTED,
                    "state_update bwd_noalloc: this problem needs " + std::to_string(need) +
                        " bytes of scratch but the fixed array holds " + std::to_string(kStaticScratchBytes) +
                        "; call ssm_state_update_bwd with a workspace instead");
    void* scratch = nullptr;
    if (int s = static_scratch(&scratch)) return s;
    ssm_state_update_params q = *p;
    q.workspace = scratch;
    q.workspace_bytes = kStaticScratchBytes;
    return ssm_state_update_bwd(&q, stream);
}
