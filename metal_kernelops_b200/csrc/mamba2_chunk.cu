// Mamba-2 SSD chunk scan, forward and backward, for sm_100a.
//
// Reference behaviour: src/metal_kernelops/cv/mamba2_chunk.py:617-723.  For each
// (batch b, head h) with group g = h / (H / G):
//
//     d_t  = softplus(dt_t + dt_bias)                 (optional)
//     s_t  = exp(d_t A) s_{t-1} + d_t x_t B_t^T       s: (P, N), s_{-1} = initial
//     y_t  = s_t C_t + D x_t,  out_t = y_t * silu(z_t) final = s_{L-1}
//
// The sequence is cut into chunks of Q steps (an internal choice: the result
// does not depend on it).  With cs_l the within-chunk cumulative sum of d*A and
// H_c the state entering chunk c:
//
//     S_c      = sum_k exp(T - cs_k) d_k x_k B_k^T           (T = cs_{Q-1})
//     H_{c+1}  = exp(T_c) H_c + S_c
//     y_l      = sum_{k<=l} exp(cs_l - cs_k) d_k <C_l, B_k> x_k
//              + exp(cs_l) H_c C_l + D x_l
//
// Kernels (forward): prep_state (d, cs, S_c per (b,h,c)); state_pass (H_c,
// final, sequential over chunks per state element); out (one CTA per
// (b, g, c): <C_l, B_k> computed once and shared by the group's heads).
// Backward: out_bwd (intra-chunk and carried-state gradients, dHout_c),
// state_pass_bwd (reverse chunk recurrence: dS_c, d initial, dT partials),
// state_bwd (chunk-state gradients), dt_bwd (cumsum / softplus chain), reduce.
// Everything accumulates in fp32; every reduction has a fixed order, so the
// backward is deterministic.  This is the CUDA-core path that serves every
// dtype and shape; it is exact to fp32 rounding.  bf16/f16 inputs with headdim
// 64 and dstate 128 go to the tensor-core kernels of mamba2_chunk_tc.cu instead
// (unless the caller sets SSM_CUDA_CORES).
#include <string>

#include "common.cuh"
#include "ssd_tc.h"

namespace ssm {
namespace ssd {

constexpr int kThreads = 256;

struct Args {
    int64_t batch, length, nheads, headdim, ngroups, dstate;
    int64_t Q, nc, hpg;          // chunk, chunks, heads per group
    uint32_t flags;
    int dtype, dt_dtype;
    const void* x; const void* dt; const float* A; const void* B; const void* C;
    const float* D; const void* z; const float* dt_bias; const float* init;
    void* y; float* final_state;
    // saved by the forward: entering states (b,h,c,p,n), d and cs (b,h,c*Q)
    float* Hs; float* dsv; float* csv;
    // backward
    const void* dy; const float* dfinal;
    void* dx; float* ddt; float* dB; float* dC; void* dz; float* dinit;
    float* dHS;                  // (b,h,c,p,n): dHout_c, then dS_c
    float* dcs; float* ddd;      // (b,h,c*Q)
    float* dxf;                  // (b,L,h,p) fp32 intra part of dx
    float* dT_part;              // (b,h,c,ntile)
    int64_t ntile;
    float* dA_part; float* db_part; float* dD_part;   // (b,h,c) / (b,h,c[,p])
};

__device__ __forceinline__ int64_t xi(const Args& a, int64_t b, int64_t t, int64_t h, int64_t p) {
    return ((b * a.length + t) * a.nheads + h) * a.headdim + p;
}
__device__ __forceinline__ int64_t bci(const Args& a, int64_t b, int64_t t, int64_t g, int64_t n) {
    return ((b * a.length + t) * a.ngroups + g) * a.dstate + n;
}
__device__ __forceinline__ int64_t bhc(const Args& a, int64_t b, int64_t h, int64_t c) {
    return (b * a.nheads + h) * a.nc + c;
}

// -------------------------------------------------------------- forward ----
// d, cs for the chunk, and the chunk's own state S_c (into Hs).
__global__ void __launch_bounds__(kThreads) prep_state_kernel(const Args a) {
    extern __shared__ __align__(16) float sm[];
    const int64_t c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int64_t Q = a.Q, P = a.headdim, N = a.dstate;
    const int64_t g = h / a.hpg;
    float* ds = sm;              // [Q]
    float* cs = ds + Q;          // [Q]
    float* vs = cs + Q;          // [Q]
    float* xs = vs + Q;          // [Q][P]
    float* Bs = xs + Q * P;      // [Q][N]
    const int tid = threadIdx.x;
    const bool softplus = a.flags & SSM_SOFTPLUS, has_bias = a.flags & SSM_HAS_BIAS;
    const float bias = has_bias ? a.dt_bias[h] : 0.0f;
    const float Ah = a.A[h];
    for (int64_t l = tid; l < Q; l += kThreads) {
        const int64_t t = c * Q + l;
        float d = 0.0f;
        if (t < a.length) {
            const float raw = ld_any(a.dt, (b * a.length + t) * a.nheads + h, a.dt_dtype) + bias;
            d = softplus ? softplus_f(raw) : raw;
        }
        ds[l] = d;
    }
    for (int64_t i = tid; i < Q * P; i += kThreads) {
        const int64_t l = i / P, p = i % P, t = c * Q + l;
        xs[i] = t < a.length ? ld_any(a.x, xi(a, b, t, h, p), a.dtype) : 0.0f;
    }
    for (int64_t i = tid; i < Q * N; i += kThreads) {
        const int64_t l = i / N, n = i % N, t = c * Q + l;
        Bs[i] = t < a.length ? ld_any(a.B, bci(a, b, t, g, n), a.dtype) : 0.0f;
    }
    __syncthreads();
    if (tid == 0) {
        float run = 0.0f;
        for (int64_t l = 0; l < Q; ++l) {
            run += ds[l] * Ah;
            cs[l] = run;
        }
    }
    __syncthreads();
    const float T = cs[Q - 1];
    for (int64_t l = tid; l < Q; l += kThreads) {
        vs[l] = ds[l] * expf(T - cs[l]);
        a.dsv[bhc(a, b, h, c) * Q + l] = ds[l];
        a.csv[bhc(a, b, h, c) * Q + l] = cs[l];
    }
    __syncthreads();
    float* S = a.Hs + bhc(a, b, h, c) * P * N;
    for (int64_t i = tid; i < P * N; i += kThreads) {
        const int64_t p = i / N, n = i % N;
        float acc = 0.0f;
        for (int64_t l = 0; l < Q; ++l) acc = fmaf(vs[l] * xs[l * P + p], Bs[l * N + n], acc);
        S[i] = acc;
    }
}

// Turn S_c into the entering states H_c (in place) and write the final state.
__global__ void __launch_bounds__(kThreads) state_pass_kernel(const Args a) {
    const int64_t h = blockIdx.y, b = blockIdx.z;
    const int64_t PN = a.headdim * a.dstate;
    const int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x;
    if (i >= PN) return;
    float H = (a.flags & SSM_HAS_INIT) ? a.init[(b * a.nheads + h) * PN + i] : 0.0f;
    for (int64_t c = 0; c < a.nc; ++c) {
        float* slot = a.Hs + bhc(a, b, h, c) * PN + i;
        const float S = *slot;
        *slot = H;
        const float T = a.csv[bhc(a, b, h, c) * a.Q + a.Q - 1];
        H = fmaf(expf(T), H, S);
    }
    a.final_state[(b * a.nheads + h) * PN + i] = H;
}

// Output of one chunk for every head of one group.
__global__ void __launch_bounds__(kThreads) out_kernel(const Args a) {
    extern __shared__ __align__(16) float sm[];
    const int64_t c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int64_t Q = a.Q, P = a.headdim, N = a.dstate;
    const int tid = threadIdx.x;
    float* Cs = sm;              // [Q][N]
    float* Bs = Cs + Q * N;      // [Q][N]
    float* CB = Bs + Q * N;      // [Q][Q]
    float* W = CB + Q * Q;       // [Q][Q]
    float* ds = W + Q * Q;       // [Q]
    float* cs = ds + Q;          // [Q]
    float* xs = cs + Q;          // [Q][P]
    const bool has_d = a.flags & SSM_HAS_D, d_per_head = a.flags & SSM_D_PER_HEAD;
    const bool has_z = a.flags & SSM_HAS_Z;
    for (int64_t i = tid; i < Q * N; i += kThreads) {
        const int64_t l = i / N, n = i % N, t = c * Q + l;
        const bool ok = t < a.length;
        Cs[i] = ok ? ld_any(a.C, bci(a, b, t, g, n), a.dtype) : 0.0f;
        Bs[i] = ok ? ld_any(a.B, bci(a, b, t, g, n), a.dtype) : 0.0f;
    }
    __syncthreads();
    for (int64_t i = tid; i < Q * Q; i += kThreads) {
        const int64_t l = i / Q, k = i % Q;
        float acc = 0.0f;
        if (k <= l)
            for (int64_t n = 0; n < N; ++n) acc = fmaf(Cs[l * N + n], Bs[k * N + n], acc);
        CB[i] = acc;
    }
    for (int64_t hh = 0; hh < a.hpg; ++hh) {
        const int64_t h = g * a.hpg + hh;
        __syncthreads();
        for (int64_t l = tid; l < Q; l += kThreads) {
            ds[l] = a.dsv[bhc(a, b, h, c) * Q + l];
            cs[l] = a.csv[bhc(a, b, h, c) * Q + l];
        }
        for (int64_t i = tid; i < Q * P; i += kThreads) {
            const int64_t l = i / P, p = i % P, t = c * Q + l;
            xs[i] = t < a.length ? ld_any(a.x, xi(a, b, t, h, p), a.dtype) : 0.0f;
        }
        __syncthreads();
        for (int64_t i = tid; i < Q * Q; i += kThreads) {
            const int64_t l = i / Q, k = i % Q;
            W[i] = k <= l ? expf(cs[l] - cs[k]) * ds[k] * CB[i] : 0.0f;
        }
        __syncthreads();
        // carried-state term exp(cs_l) H_c C_l (H_c is L1-resident), intra-chunk term, skip, gate
        const float* Hc = a.Hs + bhc(a, b, h, c) * P * N;
        for (int64_t i = tid; i < Q * P; i += kThreads) {
            const int64_t l = i / P, p = i % P, t = c * Q + l;
            if (t >= a.length) continue;
            float off = 0.0f;
            for (int64_t n = 0; n < N; ++n) off = fmaf(Cs[l * N + n], Hc[p * N + n], off);
            float yv = off * expf(cs[l]);
            for (int64_t k = 0; k <= l; ++k) yv = fmaf(W[l * Q + k], xs[k * P + p], yv);
            if (has_d) yv = fmaf(d_per_head ? a.D[h * P + p] : a.D[h], xs[l * P + p], yv);
            if (has_z) {
                const float zv = ld_any(a.z, xi(a, b, t, h, p), a.dtype);
                yv *= zv * sigmoid_f(zv);
            }
            st_any(a.y, xi(a, b, t, h, p), a.dtype, yv);
        }
    }
}

// ------------------------------------------------------------- backward ----
// Intra-chunk and carried-state gradients for every head of one group:
// dz, dx (intra + skip, fp32), dC (complete), dB (intra part), dHout_c,
// d cs and d d (direct terms), dD partials.
__global__ void __launch_bounds__(kThreads) out_bwd_kernel(const Args a) {
    extern __shared__ __align__(16) float sm[];
    const int64_t c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int64_t Q = a.Q, P = a.headdim, N = a.dstate;
    const int tid = threadIdx.x;
    float* Cs = sm;              // [Q][N]
    float* Bs = Cs + Q * N;      // [Q][N]
    float* dCa = Bs + Q * N;     // [Q][N] accumulated over heads
    float* dBa = dCa + Q * N;    // [Q][N]
    float* CB = dBa + Q * N;     // [Q][Q]
    float* W = CB + Q * Q;       // [Q][Q]
    float* dW = W + Q * Q;       // [Q][Q]
    float* ds = dW + Q * Q;      // [Q]
    float* cs = ds + Q;
    float* dcs = cs + Q;
    float* ddd = dcs + Q;
    float* xs = ddd + Q;         // [Q][P]
    float* gs = xs + Q * P;      // [Q][P] gradient seen by y (dout * silu(z))
    float* yo = gs + Q * P;      // [Q][P] carried-state term exp(cs) H C
    const bool has_d = a.flags & SSM_HAS_D, d_per_head = a.flags & SSM_D_PER_HEAD;
    const bool has_z = a.flags & SSM_HAS_Z;
    for (int64_t i = tid; i < Q * N; i += kThreads) {
        const int64_t l = i / N, n = i % N, t = c * Q + l;
        const bool ok = t < a.length;
        Cs[i] = ok ? ld_any(a.C, bci(a, b, t, g, n), a.dtype) : 0.0f;
        Bs[i] = ok ? ld_any(a.B, bci(a, b, t, g, n), a.dtype) : 0.0f;
        dCa[i] = 0.0f;
        dBa[i] = 0.0f;
    }
    __syncthreads();
    for (int64_t i = tid; i < Q * Q; i += kThreads) {
        const int64_t l = i / Q, k = i % Q;
        float acc = 0.0f;
        if (k <= l)
            for (int64_t n = 0; n < N; ++n) acc = fmaf(Cs[l * N + n], Bs[k * N + n], acc);
        CB[i] = acc;
    }
    for (int64_t hh = 0; hh < a.hpg; ++hh) {
        const int64_t h = g * a.hpg + hh;
        const float* Hc = a.Hs + bhc(a, b, h, c) * P * N;
        __syncthreads();
        for (int64_t l = tid; l < Q; l += kThreads) {
            ds[l] = a.dsv[bhc(a, b, h, c) * Q + l];
            cs[l] = a.csv[bhc(a, b, h, c) * Q + l];
        }
        for (int64_t i = tid; i < Q * P; i += kThreads) {
            const int64_t l = i / P, p = i % P, t = c * Q + l;
            float xv = 0.0f, gv = 0.0f;
            if (t < a.length) {
                xv = ld_any(a.x, xi(a, b, t, h, p), a.dtype);
                gv = ld_any(a.dy, xi(a, b, t, h, p), a.dtype);
                if (has_z) {
                    const float zv = ld_any(a.z, xi(a, b, t, h, p), a.dtype);
                    gv *= zv * sigmoid_f(zv);
                }
            }
            xs[i] = xv;
            gs[i] = gv;
        }
        __syncthreads();
        for (int64_t i = tid; i < Q * Q; i += kThreads) {
            const int64_t l = i / Q, k = i % Q;
            W[i] = k <= l ? expf(cs[l] - cs[k]) * ds[k] * CB[i] : 0.0f;
        }
        for (int64_t i = tid; i < Q * P; i += kThreads) {
            const int64_t l = i / P, p = i % P;
            float s = 0.0f;
            for (int64_t n = 0; n < N; ++n) s = fmaf(Cs[l * N + n], Hc[p * N + n], s);
            yo[i] = s * expf(cs[l]);
        }
        __syncthreads();
        // dz, dx (intra + skip), dD partial
        float dDacc = 0.0f;
        for (int64_t i = tid; i < Q * P; i += kThreads) {
            const int64_t k = i / P, p = i % P, t = c * Q + k;
            if (t >= a.length) continue;
            const float Dv = has_d ? (d_per_head ? a.D[h * P + p] : a.D[h]) : 0.0f;
            float dxv = Dv * gs[i];
            for (int64_t l = k; l < Q; ++l) dxv = fmaf(W[l * Q + k], gs[l * P + p], dxv);
            a.dxf[xi(a, b, t, h, p)] = dxv;
            if (has_d) dDacc = fmaf(gs[i], xs[i], dDacc);
            if (has_z) {
                float ypre = yo[i] + Dv * xs[i];
                for (int64_t kk = 0; kk <= k; ++kk) ypre = fmaf(W[k * Q + kk], xs[kk * P + p], ypre);
                const float zv = ld_any(a.z, xi(a, b, t, h, p), a.dtype);
                const float go = ld_any(a.dy, xi(a, b, t, h, p), a.dtype);
                const float sg = sigmoid_f(zv);
                st_any(a.dz, xi(a, b, t, h, p), a.dtype, go * ypre * sg * fmaf(zv, 1.0f - sg, 1.0f));
            }
        }
        // dD partial sums: per head (block reduce) or per (head, p) (column sums)
        if (has_d) {
            if (d_per_head) {
                __syncthreads();
                for (int64_t p = tid; p < P; p += kThreads) {
                    float s = 0.0f;
                    for (int64_t l = 0; l < Q; ++l) s = fmaf(gs[l * P + p], xs[l * P + p], s);
                    a.dD_part[bhc(a, b, h, c) * P + p] = s;
                }
            } else {
                __shared__ float red[kThreads];
                red[tid] = dDacc;
                __syncthreads();
                for (int o = kThreads / 2; o > 0; o >>= 1) {
                    if (tid < o) red[tid] += red[tid + o];
                    __syncthreads();
                }
                if (tid == 0) a.dD_part[bhc(a, b, h, c)] = red[0];
            }
        }
        // dW = g x^T (lower triangle)
        for (int64_t i = tid; i < Q * Q; i += kThreads) {
            const int64_t l = i / Q, k = i % Q;
            float s = 0.0f;
            if (k <= l)
                for (int64_t p = 0; p < P; ++p) s = fmaf(gs[l * P + p], xs[k * P + p], s);
            dW[i] = s;
        }
        __syncthreads();
        // d cs and d d (direct), per position m
        for (int64_t m = tid; m < Q; m += kThreads) {
            float dc = 0.0f, dd = 0.0f;
            for (int64_t k = 0; k <= m; ++k) dc = fmaf(dW[m * Q + k], W[m * Q + k], dc);
            for (int64_t l = m; l < Q; ++l) {
                const float r = dW[l * Q + m] * W[l * Q + m];
                dc -= r;
                dd = fmaf(dW[l * Q + m], expf(cs[l] - cs[m]) * CB[l * Q + m], dd);
            }
            float go = 0.0f;
            for (int64_t p = 0; p < P; ++p) go = fmaf(gs[m * P + p], yo[m * P + p], go);
            dcs[m] = dc + go;
            ddd[m] = dd;
        }
        __syncthreads();   // every read of dW above completes before it is overwritten
        // dCB = dW * E * d  (in place in dW)
        for (int64_t i = tid; i < Q * Q; i += kThreads) {
            const int64_t l = i / Q, k = i % Q;
            dW[i] = k <= l ? dW[i] * expf(cs[l] - cs[k]) * ds[k] : 0.0f;
        }
        __syncthreads();
        for (int64_t l = tid; l < Q; l += kThreads) {
            a.dcs[bhc(a, b, h, c) * Q + l] = dcs[l];
            a.ddd[bhc(a, b, h, c) * Q + l] = ddd[l];
        }
        // dC += dCB B + exp(cs) g H ; dB += dCB^T C
        for (int64_t i = tid; i < Q * N; i += kThreads) {
            const int64_t l = i / N, n = i % N;
            float sc = 0.0f, sb = 0.0f;
            for (int64_t k = 0; k <= l; ++k) sc = fmaf(dW[l * Q + k], Bs[k * N + n], sc);
            for (int64_t k = l; k < Q; ++k) sb = fmaf(dW[k * Q + l], Cs[k * N + n], sb);
            float sh = 0.0f;
            for (int64_t p = 0; p < P; ++p) sh = fmaf(gs[l * P + p], Hc[p * N + n], sh);
            dCa[i] += fmaf(sh, expf(cs[l]), sc);
            dBa[i] += sb;
        }
        // dHout_c = sum_l exp(cs_l) g_l C_l^T
        float* dH = a.dHS + bhc(a, b, h, c) * P * N;
        for (int64_t i = tid; i < P * N; i += kThreads) {
            const int64_t p = i / N, n = i % N;
            float s = 0.0f;
            for (int64_t l = 0; l < Q; ++l) s = fmaf(gs[l * P + p] * expf(cs[l]), Cs[l * N + n], s);
            dH[i] = s;
        }
    }
    __syncthreads();
    for (int64_t i = tid; i < Q * N; i += kThreads) {
        const int64_t l = i / N, n = i % N, t = c * Q + l;
        if (t < a.length) {
            a.dC[bci(a, b, t, g, n)] = dCa[i];
            a.dB[bci(a, b, t, g, n)] = dBa[i];
        }
    }
}

// Reverse chunk recurrence per state element: dS_c (in place of dHout_c),
// d initial, and per-tile partial sums of dT_c.
__global__ void __launch_bounds__(kThreads) state_pass_bwd_kernel(const Args a) {
    __shared__ float red[kThreads];
    const int64_t tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int64_t PN = a.headdim * a.dstate;
    const int64_t i = tile * kThreads + threadIdx.x;
    const bool ok = i < PN;
    float lam = (ok && (a.flags & SSM_HAS_DSTATE)) ? a.dfinal[(b * a.nheads + h) * PN + i] : 0.0f;
    for (int64_t c = a.nc - 1; c >= 0; --c) {
        const float eT = expf(a.csv[bhc(a, b, h, c) * a.Q + a.Q - 1]);
        float contrib = 0.0f;
        if (ok) {
            float* slot = a.dHS + bhc(a, b, h, c) * PN + i;
            const float dHout = *slot;
            const float Hc = a.Hs[bhc(a, b, h, c) * PN + i];
            contrib = lam * eT * Hc;
            *slot = lam;                       // dS_c
            lam = fmaf(eT, lam, dHout);        // Lambda_c
        }
        red[threadIdx.x] = contrib;
        __syncthreads();
        for (int o = kThreads / 2; o > 0; o >>= 1) {
            if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
            __syncthreads();
        }
        if (threadIdx.x == 0) a.dT_part[bhc(a, b, h, c) * a.ntile + tile] = red[0];
        __syncthreads();
    }
    if (ok && a.dinit) a.dinit[(b * a.nheads + h) * PN + i] = lam;
}

// Chunk-state gradients for every head of one group: dx (adds the state term
// and writes dx in x's dtype), dB (adds), d cs, d d.
__global__ void __launch_bounds__(kThreads) state_bwd_kernel(const Args a) {
    extern __shared__ __align__(16) float sm[];
    const int64_t c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int64_t Q = a.Q, P = a.headdim, N = a.dstate;
    const int tid = threadIdx.x;
    float* Bs = sm;              // [Q][N]
    float* dBa = Bs + Q * N;     // [Q][N]
    float* Us = dBa + Q * N;     // [Q][P]  U = B dS^T
    float* xs = Us + Q * P;      // [Q][P]
    float* vs = xs + Q * P;      // [Q]
    float* dv = vs + Q;          // [Q]
    float* ds = dv + Q;
    float* cs = ds + Q;
    __shared__ float red[kThreads];
    for (int64_t i = tid; i < Q * N; i += kThreads) {
        const int64_t l = i / N, n = i % N, t = c * Q + l;
        Bs[i] = t < a.length ? ld_any(a.B, bci(a, b, t, g, n), a.dtype) : 0.0f;
        dBa[i] = 0.0f;
    }
    for (int64_t hh = 0; hh < a.hpg; ++hh) {
        const int64_t h = g * a.hpg + hh;
        const float* dS = a.dHS + bhc(a, b, h, c) * P * N;
        __syncthreads();
        for (int64_t l = tid; l < Q; l += kThreads) {
            ds[l] = a.dsv[bhc(a, b, h, c) * Q + l];
            cs[l] = a.csv[bhc(a, b, h, c) * Q + l];
        }
        for (int64_t i = tid; i < Q * P; i += kThreads) {
            const int64_t l = i / P, p = i % P, t = c * Q + l;
            xs[i] = t < a.length ? ld_any(a.x, xi(a, b, t, h, p), a.dtype) : 0.0f;
        }
        __syncthreads();
        const float T = cs[Q - 1];
        for (int64_t l = tid; l < Q; l += kThreads) vs[l] = ds[l] * expf(T - cs[l]);
        for (int64_t i = tid; i < Q * P; i += kThreads) {
            const int64_t k = i / P, p = i % P;
            float s = 0.0f;
            for (int64_t n = 0; n < N; ++n) s = fmaf(dS[p * N + n], Bs[k * N + n], s);
            Us[i] = s;
        }
        __syncthreads();
        // dx = dxf + v_k U_k (final, in x's dtype)
        for (int64_t i = tid; i < Q * P; i += kThreads) {
            const int64_t k = i / P, p = i % P, t = c * Q + k;
            if (t < a.length) {
                const int64_t o = xi(a, b, t, h, p);
                st_any(a.dx, o, a.dtype, fmaf(vs[k], Us[i], a.dxf[o]));
            }
        }
        // dv_k = x_k . U_k
        for (int64_t k = tid; k < Q; k += kThreads) {
            float s = 0.0f;
            for (int64_t p = 0; p < P; ++p) s = fmaf(xs[k * P + p], Us[k * P + p], s);
            dv[k] = s;
        }
        // dB += v_k dS^T x_k
        for (int64_t i = tid; i < Q * N; i += kThreads) {
            const int64_t k = i / N, n = i % N;
            float s = 0.0f;
            for (int64_t p = 0; p < P; ++p) s = fmaf(dS[p * N + n], xs[k * P + p], s);
            dBa[i] = fmaf(vs[k], s, dBa[i]);
        }
        __syncthreads();
        // dT_state = sum_k dv_k v_k ; d d_k += dv_k exp(T - cs_k) ; d cs_k -= dv_k v_k
        float part = 0.0f;
        for (int64_t k = tid; k < Q; k += kThreads) part = fmaf(dv[k], vs[k], part);
        red[tid] = part;
        __syncthreads();
        for (int o = kThreads / 2; o > 0; o >>= 1) {
            if (tid < o) red[tid] += red[tid + o];
            __syncthreads();
        }
        if (tid == 0) {
            float dT = red[0];
            for (int64_t j = 0; j < a.ntile; ++j) dT += a.dT_part[bhc(a, b, h, c) * a.ntile + j];
            a.dcs[bhc(a, b, h, c) * Q + Q - 1] += dT;
        }
        __syncthreads();
        for (int64_t k = tid; k < Q; k += kThreads) {
            float* dcs = a.dcs + bhc(a, b, h, c) * Q + k;
            *dcs -= dv[k] * vs[k];
            a.ddd[bhc(a, b, h, c) * Q + k] += dv[k] * expf(T - cs[k]);
        }
    }
    __syncthreads();
    for (int64_t i = tid; i < Q * N; i += kThreads) {
        const int64_t l = i / N, n = i % N, t = c * Q + l;
        if (t < a.length) a.dB[bci(a, b, t, g, n)] += dBa[i];
    }
}

// cs = cumsum(d*A): d d_j += A sum_{l>=j} dcs_l, dA += sum_l dcs_l sum_{j<=l} d_j;
// then softplus / bias chain and the per-chunk dA / d bias partials.
__global__ void __launch_bounds__(kThreads) dt_bwd_kernel(const Args a) {
    const int64_t c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    if (threadIdx.x != 0) return;
    const int64_t Q = a.Q;
    const float Ah = a.A[h];
    const bool softplus = a.flags & SSM_SOFTPLUS, has_bias = a.flags & SSM_HAS_BIAS;
    const float bias = has_bias ? a.dt_bias[h] : 0.0f;
    const int64_t base = bhc(a, b, h, c) * Q;
    // dA = sum_l dcs_l * sum_{j<=l} d_j (forward cumsum)
    float run_d = 0.0f, dA = 0.0f;
    for (int64_t l = 0; l < Q; ++l) {
        run_d += a.dsv[base + l];
        dA = fmaf(a.dcs[base + l], run_d, dA);
    }
    float suffix = 0.0f, db = 0.0f;
    for (int64_t j = Q - 1; j >= 0; --j) {
        suffix += a.dcs[base + j];
        const int64_t t = c * Q + j;
        if (t >= a.length) continue;
        const float dd = fmaf(Ah, suffix, a.ddd[base + j]);
        float g = dd;
        if (softplus) {
            const float raw = ld_any(a.dt, (b * a.length + t) * a.nheads + h, a.dt_dtype) + bias;
            g = dd * softplus_grad_f(raw);
        }
        a.ddt[(b * a.length + t) * a.nheads + h] = g;
        db += g;
    }
    a.dA_part[bhc(a, b, h, c)] = dA;
    a.db_part[bhc(a, b, h, c)] = db;
}

__global__ void reduce_kernel(const Args a, float* dA, float* dbias, float* dD) {
    const bool has_d = a.flags & SSM_HAS_D, d_per_head = a.flags & SSM_D_PER_HEAD;
    const int64_t H = a.nheads, P = a.headdim;
    const int64_t nd = has_d ? (d_per_head ? H * P : H) : 0;
    const int64_t total = 2 * H + nd;
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= total) return;
    if (i < 2 * H) {
        const bool is_a = i < H;
        const int64_t h = is_a ? i : i - H;
        const float* src = is_a ? a.dA_part : a.db_part;
        float s = 0.0f;
        for (int64_t b = 0; b < a.batch; ++b)
            for (int64_t c = 0; c < a.nc; ++c) s += src[(b * H + h) * a.nc + c];
        if (is_a) dA[h] = s;
        else if (dbias) dbias[h] = s;
    } else {
        const int64_t k = i - 2 * H;
        float s = 0.0f;
        if (d_per_head) {
            const int64_t h = k / P, p = k % P;
            for (int64_t b = 0; b < a.batch; ++b)
                for (int64_t c = 0; c < a.nc; ++c) s += a.dD_part[((b * H + h) * a.nc + c) * P + p];
        } else {
            for (int64_t b = 0; b < a.batch; ++b)
                for (int64_t c = 0; c < a.nc; ++c) s += a.dD_part[(b * H + k) * a.nc + c];
        }
        dD[k] = s;
    }
}

// ------------------------------------------------------------------ host ----
constexpr size_t kSmemCap = 200 * 1024;

static size_t smem_prep(int64_t Q, int64_t P, int64_t N) { return (3 * Q + Q * P + Q * N) * 4; }
static size_t smem_out(int64_t Q, int64_t P, int64_t N) {
    return (2 * Q * N + 2 * Q * Q + 2 * Q + Q * P) * 4;
}
static size_t smem_out_bwd(int64_t Q, int64_t P, int64_t N) {
    return (4 * Q * N + 3 * Q * Q + 4 * Q + 3 * Q * P) * 4;
}
static size_t smem_state_bwd(int64_t Q, int64_t P, int64_t N) { return (2 * Q * N + 2 * Q * P + 4 * Q) * 4; }

static int64_t pick_q(int64_t L, int64_t P, int64_t N) {
    for (int64_t q : {64, 32, 16, 8}) {
        if (q * P > 64 * 256) continue;
        if (smem_prep(q, P, N) <= kSmemCap && smem_out(q, P, N) <= kSmemCap &&
            smem_out_bwd(q, P, N) <= kSmemCap && smem_state_bwd(q, P, N) <= kSmemCap) {
            return q;
        }
    }
    return 0;
}

static int validate(const ssm_chunk_scan_params* p, int mode) {
    if (!p) return fail(SSM_ERR_INVALID, "null params");
    if (p->chunk_size < 1) return fail(SSM_ERR_INVALID, "chunk_scan: chunk_size must be positive");
    if (p->batch < 0 || p->length < 0 || p->nheads < 1 || p->headdim < 1 || p->ngroups < 1 || p->dstate < 1)
        return fail(SSM_ERR_INVALID, "chunk_scan: bad sizes");
    if (p->nheads % p->ngroups) return fail(SSM_ERR_INVALID, "chunk_scan: ngroups must divide nheads");
    if (p->dtype < 0 || p->dtype > 2 || p->dt_dtype < 0 || p->dt_dtype > 2)
        return fail(SSM_ERR_UNSUPPORTED, "chunk_scan: unknown dtype");
    if (!ssdtc::eligible(p) && pick_q(p->length, p->headdim, p->dstate) == 0)
        return fail(SSM_ERR_UNSUPPORTED, "chunk_scan: headdim/dstate too large for the kernels");
    const bool empty = p->batch == 0 || p->length == 0;
    if (mode >= 1 && !empty && (!p->x || !p->dt || !p->A || !p->B || !p->C))
        return fail(SSM_ERR_INVALID, "chunk_scan: null input");
    if (mode == 1 && !empty && (!p->y || !p->final_state))
        return fail(SSM_ERR_INVALID, "chunk_scan: null output");
    if (mode >= 1 && !empty && !p->saved)
        return fail(SSM_ERR_INVALID, "chunk_scan: null saved-state buffer");
    if (mode == 2 && !empty && (!p->dy || !p->dx || !p->ddt || !p->dA || !p->dB || !p->dC))
        return fail(SSM_ERR_INVALID, "chunk_scan bwd: null gradient pointer");
    const int64_t xd = p->nheads * p->headdim, bcd = p->ngroups * p->dstate;
    if ((p->x_token_stride && p->x_token_stride != xd) || (p->bc_token_stride && p->bc_token_stride != bcd)) {
        if (!ssdtc::eligible(p))
            return fail(SSM_ERR_UNSUPPORTED, "chunk_scan: token strides need the tensor-core path");
        const int64_t xs = p->x_token_stride ? p->x_token_stride : xd;
        const int64_t bs = p->bc_token_stride ? p->bc_token_stride : bcd;
        if (xs < xd || bs < bcd || xs % 8 || bs % 8)
            return fail(SSM_ERR_UNSUPPORTED, "chunk_scan: token strides must cover a token, in 16-byte steps");
    }
    return SSM_OK;
}

static void make_args(const ssm_chunk_scan_params* p, Args& a) {
    a.batch = p->batch; a.length = p->length; a.nheads = p->nheads; a.headdim = p->headdim;
    a.ngroups = p->ngroups; a.dstate = p->dstate;
    a.Q = pick_q(p->length, p->headdim, p->dstate);
    a.nc = ceil_div(p->length, a.Q);
    a.hpg = p->nheads / p->ngroups;
    a.flags = p->flags; a.dtype = p->dtype; a.dt_dtype = p->dt_dtype;
    a.x = p->x; a.dt = p->dt; a.A = p->A; a.B = p->B; a.C = p->C; a.D = p->D; a.z = p->z;
    a.dt_bias = p->dt_bias; a.init = p->initial_states;
    a.y = p->y; a.final_state = p->final_state;
    const int64_t BH = p->batch * p->nheads;
    float* sv = p->saved;
    a.Hs = sv;
    a.dsv = sv ? sv + BH * a.nc * p->headdim * p->dstate : nullptr;
    a.csv = sv ? a.dsv + BH * a.nc * a.Q : nullptr;
    a.dy = p->dy; a.dfinal = p->dfinal; a.dx = p->dx; a.ddt = p->ddt; a.dB = p->dB; a.dC = p->dC;
    a.dz = p->dz; a.dinit = p->dinitial;
    a.ntile = ceil_div(p->headdim * p->dstate, kThreads);
    a.dHS = a.dcs = a.ddd = a.dxf = a.dT_part = a.dA_part = a.db_part = a.dD_part = nullptr;
}

struct Ws { size_t hs, q, xf, tp, part, dd, total; };
static Ws ws_layout(const ssm_chunk_scan_params* p, int64_t Q, int64_t nc) {
    const int64_t BH = p->batch * p->nheads;
    Ws w;
    w.hs = align_up((size_t)(BH * nc * p->headdim * p->dstate) * 4, 256);
    w.q = align_up((size_t)(BH * nc * Q) * 4, 256);
    w.xf = align_up((size_t)(p->batch * p->length * p->nheads * p->headdim) * 4, 256);
    w.tp = align_up((size_t)(BH * nc * ceil_div(p->headdim * p->dstate, kThreads)) * 4, 256);
    w.part = align_up((size_t)(BH * nc) * 4, 256);
    w.dd = align_up((size_t)(BH * nc * p->headdim) * 4, 256);
    w.total = w.hs + 2 * w.q + w.xf + w.tp + 2 * w.part + w.dd;
    return w;
}

static int set_smem(const void* fn, size_t bytes) {
    if (bytes > 48 * 1024 &&
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
        return check_launch("chunk_scan: smem attribute");
    return SSM_OK;
}

}  // namespace ssd
}  // namespace ssm

using namespace ssm;
using namespace ssm::ssd;

extern "C" int ssm_chunk_scan_sizes(const ssm_chunk_scan_params* p, size_t* saved_bytes,
                                    size_t* workspace_bytes) {
    if (int s = validate(p, 0)) return s;
    if (ssdtc::eligible(p)) {
        ssdtc::sizes(p, saved_bytes, workspace_bytes);
        return SSM_OK;
    }
    const int64_t Q = pick_q(p->length, p->headdim, p->dstate);
    const int64_t nc = ceil_div(p->length, Q);
    const int64_t BH = p->batch * p->nheads;
    if (saved_bytes) *saved_bytes = (size_t)(BH * nc * (p->headdim * p->dstate + 2 * Q)) * 4;
    if (workspace_bytes) *workspace_bytes = ws_layout(p, Q, nc).total;
    return SSM_OK;
}

extern "C" int ssm_chunk_scan_fwd(const ssm_chunk_scan_params* p, void* stream) {
    if (int s = validate(p, 1)) return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t PN = p->headdim * p->dstate;
    if (p->batch == 0) return SSM_OK;
    if (p->length == 0) {
        // no steps: the final state is the initial state (or zero)
        const size_t bytes = (size_t)(p->batch * p->nheads * PN) * 4;
        if ((p->flags & SSM_HAS_INIT) && p->initial_states)
            cudaMemcpyAsync(p->final_state, p->initial_states, bytes, cudaMemcpyDeviceToDevice, st);
        else
            cudaMemsetAsync(p->final_state, 0, bytes, st);
        return check_launch("chunk_scan fwd: empty");
    }
    if (ssdtc::eligible(p)) return ssdtc::fwd(p, st);
    Args a;
    make_args(p, a);
    const int64_t Q = a.Q, P = p->headdim, N = p->dstate;
    if (int s = set_smem((const void*)prep_state_kernel, smem_prep(Q, P, N))) return s;
    if (int s = set_smem((const void*)out_kernel, smem_out(Q, P, N))) return s;
    prep_state_kernel<<<dim3((unsigned)a.nc, (unsigned)p->nheads, (unsigned)p->batch), kThreads,
                        smem_prep(Q, P, N), st>>>(a);
    if (int s = check_launch("chunk_scan fwd: prep")) return s;
    state_pass_kernel<<<dim3((unsigned)ceil_div(PN, kThreads), (unsigned)p->nheads, (unsigned)p->batch),
                        kThreads, 0, st>>>(a);
    if (int s = check_launch("chunk_scan fwd: state pass")) return s;
    out_kernel<<<dim3((unsigned)a.nc, (unsigned)p->ngroups, (unsigned)p->batch), kThreads,
                 smem_out(Q, P, N), st>>>(a);
    return check_launch("chunk_scan fwd: out");
}

extern "C" int ssm_chunk_scan_bwd(const ssm_chunk_scan_params* p, void* stream) {
    if (int s = validate(p, 2)) return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t H = p->nheads, P = p->headdim, N = p->dstate;
    const bool has_d = p->flags & SSM_HAS_D, d_per_head = p->flags & SSM_D_PER_HEAD;
    if (p->batch == 0 || p->length == 0) {
        cudaMemsetAsync(p->dA, 0, (size_t)H * 4, st);
        if ((p->flags & SSM_HAS_BIAS) && p->ddt_bias) cudaMemsetAsync(p->ddt_bias, 0, (size_t)H * 4, st);
        if (has_d && p->dD) cudaMemsetAsync(p->dD, 0, (size_t)(d_per_head ? H * P : H) * 4, st);
        if ((p->flags & SSM_HAS_INIT) && p->dinitial) {
            const size_t bytes = (size_t)(p->batch * H * P * N) * 4;
            if (p->flags & SSM_HAS_DSTATE)
                cudaMemcpyAsync(p->dinitial, p->dfinal, bytes, cudaMemcpyDeviceToDevice, st);
            else
                cudaMemsetAsync(p->dinitial, 0, bytes, st);
        }
        return check_launch("chunk_scan bwd: empty");
    }
    if (ssdtc::eligible(p)) return ssdtc::bwd(p, st);
    Args a;
    make_args(p, a);
    const int64_t Q = a.Q;
    const Ws w = ws_layout(p, Q, a.nc);
    if (!p->workspace || p->workspace_bytes < w.total)
        return fail(SSM_ERR_WORKSPACE, "chunk_scan bwd: workspace too small");
    char* ws = reinterpret_cast<char*>(p->workspace);
    a.dHS = reinterpret_cast<float*>(ws);
    a.dcs = reinterpret_cast<float*>(ws + w.hs);
    a.ddd = reinterpret_cast<float*>(ws + w.hs + w.q);
    a.dxf = reinterpret_cast<float*>(ws + w.hs + 2 * w.q);
    a.dT_part = reinterpret_cast<float*>(ws + w.hs + 2 * w.q + w.xf);
    a.dA_part = reinterpret_cast<float*>(ws + w.hs + 2 * w.q + w.xf + w.tp);
    a.db_part = reinterpret_cast<float*>(ws + w.hs + 2 * w.q + w.xf + w.tp + w.part);
    a.dD_part = reinterpret_cast<float*>(ws + w.hs + 2 * w.q + w.xf + w.tp + 2 * w.part);
    if (!(p->flags & SSM_HAS_INIT)) a.dinit = nullptr;
    const dim3 gg((unsigned)a.nc, (unsigned)p->ngroups, (unsigned)p->batch);
    const dim3 gh((unsigned)a.nc, (unsigned)H, (unsigned)p->batch);
    if (int s = set_smem((const void*)out_bwd_kernel, smem_out_bwd(Q, P, N))) return s;
    if (int s = set_smem((const void*)state_bwd_kernel, smem_state_bwd(Q, P, N))) return s;
    out_bwd_kernel<<<gg, kThreads, smem_out_bwd(Q, P, N), st>>>(a);
    if (int s = check_launch("chunk_scan bwd: out")) return s;
    state_pass_bwd_kernel<<<dim3((unsigned)a.ntile, (unsigned)H, (unsigned)p->batch), kThreads, 0, st>>>(a);
    if (int s = check_launch("chunk_scan bwd: state pass")) return s;
    state_bwd_kernel<<<gg, kThreads, smem_state_bwd(Q, P, N), st>>>(a);
    if (int s = check_launch("chunk_scan bwd: state")) return s;
    dt_bwd_kernel<<<gh, 32, 0, st>>>(a);
    if (int s = check_launch("chunk_scan bwd: dt")) return s;
    const int64_t total = 2 * H + (has_d ? (d_per_head ? H * P : H) : 0);
    reduce_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(
        a, p->dA, (p->flags & SSM_HAS_BIAS) ? p->ddt_bias : nullptr, has_d ? p->dD : nullptr);
    return check_launch("chunk_scan bwd: reduce");
}
