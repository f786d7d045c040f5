// Mamba-1 selective scan, forward and backward, for sm_100a.
//
// Reference behaviour: src/metal_kernelops/scan.py:295-320 (`selective_scan`)
// over `_Scan` (:236-280).  The reference runs the recurrence as three Metal
// passes over 64-step chunks (summarize -> boundaries -> outputs, MSL :60-127)
// with one thread per (batch, channel, chunk, state) and applies the bias,
// softplus, D skip and silu(z) gate as separate torch ops.  This file is a
// different design built for the B200:
//
//  * One thread owns one channel and NPT of its states (LPC lanes per channel);
//    time is walked sequentially, so every exp(delta*A) is evaluated exactly
//    once in the forward and the per-step output <x, C> is a register sum
//    (plus a log2(LPC) shuffle).  B and C of the channel's group are staged in
//    shared memory as fp32 [t][n] and read as broadcasts.
//  * Bias, softplus, the D skip and the silu(z) gate are fused into the same
//    kernel; y is written once.
//  * The forward stores the state entering every kTile-step chunk
//    (fp32, "checkpoints"); the backward walks the chunks in reverse, recomputes
//    the chunk from its checkpoint (pass A, which also produces dz, dC and the
//    output gradient seen by the scan), then replays each TS-step sub-block from
//    a shared-memory sub-checkpoint with the states and decays kept in
//    registers, and runs the adjoint recurrence backwards over it (pass B:
//    du, ddelta, dA, dB).
//  * The cross-channel sums dB/dC are reduced inside the warp with a butterfly
//    reduce-scatter, then across the CTA's warps in shared memory, and written
//    as one deterministic partial per CTA; a small kernel adds the partials and
//    the per-batch dA/dD/d_bias partials.  No float atomics (the reference uses
//    them, scan.py:226-227), so the backward is bit-reproducible.
#include "common.cuh"

namespace ssm {
namespace sscan {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 32;  // time steps per staged tile == checkpoint interval

struct Args {
    int64_t batch, dim, length, groups, dstate, per_group;
    int64_t ntiles;       // ceil(length / kTile)
    int64_t nct;          // channel tiles per group
    uint32_t flags;
    int bc_dtype;
    const void* u; const void* delta; const float* A; const void* B; const void* C;
    const float* D; const void* z; const float* delta_bias;
    void* y; float* ckpt;
    const void* dout; void* du; void* ddelta; void* dz;
    float* dB_part; float* dC_part;   // (batch*groups*nct, dstate, length)
    float* dA_part;                   // (batch, dim, dstate)
    float* dD_part; float* db_part;   // (batch, dim)
};

template <typename T> struct Pad { static constexpr int v = 4 / sizeof(T); };  // odd word stride

// Stage a [rows][kTile] tile of a (batch, dim, length) tensor into shared memory
// (row stride kTile + pad), zero-filling rows past `rows_valid` and steps past
// `len`.  Consecutive threads read consecutive steps of a row.
template <typename T, int ROWS>
__device__ __forceinline__ void load_act_tile(T* s, const T* g, int64_t row0, int rows_valid,
                                              int64_t L, int64_t t0, int len) {
    constexpr int RS = kTile + Pad<T>::v;
    for (int i = threadIdx.x; i < ROWS * kTile; i += kThreads) {
        const int r = i / kTile, t = i % kTile;
        T v;
        if (r < rows_valid && t < len) v = g[(row0 + r) * L + t0 + t];
        else v = T(0.0f);
        s[r * RS + t] = v;
    }
}

template <typename T, int ROWS>
__device__ __forceinline__ void store_act_tile(const T* s, T* g, int64_t row0, int rows_valid,
                                               int64_t L, int64_t t0, int len) {
    constexpr int RS = kTile + Pad<T>::v;
    for (int i = threadIdx.x; i < ROWS * kTile; i += kThreads) {
        const int r = i / kTile, t = i % kTile;
        if (r < rows_valid && t < len) g[(row0 + r) * L + t0 + t] = s[r * RS + t];
    }
}

// B or C of one (batch, group) as fp32 [kTile][NP] (NP >= dstate, zero padded).
template <int NP>
__device__ __forceinline__ void load_bc_tile(float* s, const void* g, int dtype, int64_t bg,
                                             int64_t N, int64_t L, int64_t t0, int len) {
    for (int i = threadIdx.x; i < NP * kTile; i += kThreads) {
        const int n = i / kTile, t = i % kTile;
        float v = 0.0f;
        if (n < N && t < len) v = ld_any(g, (bg * N + n) * L + t0 + t, dtype);
        s[t * NP + n] = v;
    }
}

// ------------------------------------------------------------------ forward --
template <typename T, int NPT, int LPC>
__global__ void __launch_bounds__(kThreads)
fwd_kernel(const Args a) {
    constexpr int CPW = 32 / LPC;
    constexpr int CPC = CPW * kWarps;
    constexpr int NP = NPT * LPC;
    constexpr int RS = kTile + Pad<T>::v;

    extern __shared__ __align__(16) unsigned char smem[];
    T* us = reinterpret_cast<T*>(smem);
    T* ds = us + CPC * RS;
    T* zs = ds + CPC * RS;
    T* ys = zs + CPC * RS;
    float* Bs = reinterpret_cast<float*>(ys + CPC * RS);
    Bs = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(Bs) + 15) & ~uintptr_t(15));
    float* Cs = Bs + kTile * NP;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cw = lane / LPC, sub = lane % LPC;
    const int c = warp * CPW + cw;
    const int64_t ct = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int64_t dl0 = ct * CPC;                       // first channel of the tile, within group
    const int rows = (int)min64(CPC, a.per_group - dl0);
    const int64_t d0 = g * a.per_group + dl0;           // first global channel
    const int64_t row0 = b * a.dim + d0;                // first (batch, channel) row
    const bool cvalid = c < rows;
    const int64_t d = d0 + c;
    const int64_t N = a.dstate, L = a.length;
    const bool has_d = a.flags & SSM_HAS_D, has_z = a.flags & SSM_HAS_Z;
    const bool has_bias = a.flags & SSM_HAS_BIAS, softplus = a.flags & SSM_SOFTPLUS;

    float An[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int n = sub * NPT + j;
        An[j] = (cvalid && n < N) ? a.A[d * N + n] : 0.0f;
    }
    const float Dd = (has_d && cvalid) ? a.D[d] : 0.0f;
    const float bias = (has_bias && cvalid) ? a.delta_bias[d] : 0.0f;
    float x[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) x[j] = 0.0f;

    const T* ug = reinterpret_cast<const T*>(a.u);
    const T* dg = reinterpret_cast<const T*>(a.delta);
    const T* zg = reinterpret_cast<const T*>(a.z);
    T* yg = reinterpret_cast<T*>(a.y);
    const int64_t bg = b * a.groups + g;

    for (int64_t tile = 0; tile < a.ntiles; ++tile) {
        const int64_t t0 = tile * kTile;
        const int len = (int)min64(kTile, L - t0);
        __syncthreads();
        load_act_tile<T, CPC>(us, ug, row0, rows, L, t0, len);
        load_act_tile<T, CPC>(ds, dg, row0, rows, L, t0, len);
        if (has_z) load_act_tile<T, CPC>(zs, zg, row0, rows, L, t0, len);
        load_bc_tile<NP>(Bs, a.B, a.bc_dtype, bg, N, L, t0, len);
        load_bc_tile<NP>(Cs, a.C, a.bc_dtype, bg, N, L, t0, len);
        __syncthreads();

        if (a.ckpt != nullptr && cvalid) {
            float* cp = a.ckpt + ((b * a.ntiles + tile) * a.dim + d) * N;
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int n = sub * NPT + j;
                if (n < N) cp[n] = x[j];
            }
        }

        for (int t = 0; t < len; ++t) {
            float dv = ldf(&ds[c * RS + t]) + bias;
            if (softplus) dv = softplus_f(dv);
            const float uv = ldf(&us[c * RS + t]);
            const float du = dv * uv;
            const float dl = dv * kLog2e;
            const float* Bt = Bs + t * NP + sub * NPT;
            const float* Ct = Cs + t * NP + sub * NPT;
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const float da = exp2_mufu(dl * An[j]);
                x[j] = fmaf(da, x[j], du * Bt[j]);
                acc = fmaf(x[j], Ct[j], acc);
            }
            acc = sum_low_lanes<LPC>(acc);
            if (sub == 0) {
                float out = fmaf(uv, Dd, acc);
                if (has_z) {
                    const float zv = ldf(&zs[c * RS + t]);
                    out *= zv * sigmoid_f(zv);
                }
                stf(&ys[c * RS + t], out);
            }
        }
        __syncthreads();
        store_act_tile<T, CPC>(ys, yg, row0, rows, L, t0, len);
    }
}

// ----------------------------------------------------------------- backward --
// Butterfly reduce-scatter of v[V] over the lanes that differ in lane bits
// [LO, 5).  Returns the first state index (within the thread's NPT) of the
// `V >> min(V_levels)` sums it ends up holding; `owner` is false on lanes whose
// sums duplicate another lane's (levels past log2(V) are plain all-reduces).
template <int V, int LO>
__device__ __forceinline__ int reduce_scatter(float (&v)[V], int lane, bool& owner) {
    int base = 0;
    owner = true;
    int cur = V;
#pragma unroll
    for (int bit = 4; bit >= LO; --bit) {
        const int o = 1 << bit;
        const bool hi = (lane >> bit) & 1;
        if (cur > 1) {
            const int half = cur / 2;
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                if (i < half) {
                    const float send = hi ? v[i] : v[half + i];
                    const float keep = hi ? v[half + i] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            if (hi) base += half;
            cur = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
            if (hi) owner = false;
        }
    }
    return base;
}

template <int V, int LO>
constexpr int scatter_kept() {
    int cur = V;
    for (int bit = 4; bit >= LO; --bit) if (cur > 1) cur /= 2;
    return cur;
}

template <typename T, int NPT, int LPC, int TS>
__global__ void __launch_bounds__(kThreads)
bwd_kernel(const Args a) {
    constexpr int CPW = 32 / LPC;
    constexpr int CPC = CPW * kWarps;
    constexpr int NP = NPT * LPC;
    constexpr int NPW = NP + 1;
    constexpr int RS = kTile + Pad<T>::v;
    constexpr int FS = kTile + 1;
    constexpr int LO = (LPC == 1) ? 0 : (LPC == 2) ? 1 : (LPC == 4) ? 2 : (LPC == 8) ? 3 : 4;
    constexpr int KEPT = scatter_kept<NPT, LO>();
    constexpr int NSB = kTile / TS;

    extern __shared__ __align__(16) unsigned char smem[];
    T* us = reinterpret_cast<T*>(smem);
    T* ds = us + CPC * RS;          // raw delta, overwritten by ddelta
    T* zs = ds + CPC * RS;          // z, overwritten by dz
    T* gs = zs + CPC * RS;          // dout, overwritten by du
    float* fbase = reinterpret_cast<float*>(
        (reinterpret_cast<uintptr_t>(gs + CPC * RS) + 15) & ~uintptr_t(15));
    float* dps = fbase;                     // delta after bias/softplus  [CPC][FS]
    float* gps = dps + CPC * FS;            // gradient seen by the scan  [CPC][FS]
    float* Bs = gps + CPC * FS;             // [kTile][NP]
    Bs = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(Bs) + 15) & ~uintptr_t(15));
    float* Cs = Bs + kTile * NP;
    float* dBw = Cs + kTile * NP;           // [kWarps][kTile][NPW]
    float* dCw = dBw + kWarps * kTile * NPW;
    float* sck = dCw + kWarps * kTile * NPW;  // [NSB][NPT][kThreads]

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int cw = lane / LPC, sub = lane % LPC;
    const int c = warp * CPW + cw;
    const int64_t ct = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int64_t dl0 = ct * CPC;
    const int rows = (int)min64(CPC, a.per_group - dl0);
    const int64_t d0 = g * a.per_group + dl0;
    const int64_t row0 = b * a.dim + d0;
    const bool cvalid = c < rows;
    const int64_t d = d0 + c;
    const int64_t N = a.dstate, L = a.length;
    const bool has_d = a.flags & SSM_HAS_D, has_z = a.flags & SSM_HAS_Z;
    const bool has_bias = a.flags & SSM_HAS_BIAS, softplus = a.flags & SSM_SOFTPLUS;

    float An[NPT], q[NPT], dA[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int n = sub * NPT + j;
        An[j] = (cvalid && n < N) ? a.A[d * N + n] : 0.0f;
        q[j] = 0.0f;
        dA[j] = 0.0f;
    }
    const float Dd = (has_d && cvalid) ? a.D[d] : 0.0f;
    const float bias = (has_bias && cvalid) ? a.delta_bias[d] : 0.0f;
    float dDacc = 0.0f, dbacc = 0.0f;

    const T* ug = reinterpret_cast<const T*>(a.u);
    const T* dg = reinterpret_cast<const T*>(a.delta);
    const T* zg = reinterpret_cast<const T*>(a.z);
    const T* gg = reinterpret_cast<const T*>(a.dout);
    const int64_t bg = b * a.groups + g;
    float* dBp = a.dB_part + (bg * a.nct + ct) * N * L;
    float* dCp = a.dC_part + (bg * a.nct + ct) * N * L;

    for (int64_t tile = a.ntiles - 1; tile >= 0; --tile) {
        const int64_t t0 = tile * kTile;
        const int len = (int)min64(kTile, L - t0);
        __syncthreads();
        load_act_tile<T, CPC>(us, ug, row0, rows, L, t0, len);
        load_act_tile<T, CPC>(ds, dg, row0, rows, L, t0, len);
        if (has_z) load_act_tile<T, CPC>(zs, zg, row0, rows, L, t0, len);
        load_act_tile<T, CPC>(gs, gg, row0, rows, L, t0, len);
        load_bc_tile<NP>(Bs, a.B, a.bc_dtype, bg, N, L, t0, len);
        load_bc_tile<NP>(Cs, a.C, a.bc_dtype, bg, N, L, t0, len);
        __syncthreads();

        // ---- pass A: forward recompute from the checkpoint ------------------
        float x[NPT];
        {
            const float* cp = a.ckpt + ((b * a.ntiles + tile) * a.dim + d) * N;
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int n = sub * NPT + j;
                x[j] = (cvalid && n < N) ? cp[n] : 0.0f;
            }
        }
        for (int t = 0; t < len; ++t) {
            if (t % TS == 0) {
#pragma unroll
                for (int j = 0; j < NPT; ++j) sck[((t / TS) * NPT + j) * kThreads + tid] = x[j];
            }
            const float raw = ldf(&ds[c * RS + t]) + bias;
            const float dv = softplus ? softplus_f(raw) : raw;
            const float uv = ldf(&us[c * RS + t]);
            const float du = dv * uv;
            const float dl = dv * kLog2e;
            const float* Bt = Bs + t * NP + sub * NPT;
            const float* Ct = Cs + t * NP + sub * NPT;
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const float da = exp2_mufu(dl * An[j]);
                x[j] = fmaf(da, x[j], du * Bt[j]);
                acc = fmaf(x[j], Ct[j], acc);
            }
            const float yv = sum_low_lanes<LPC>(acc);
            const float gv = ldf(&gs[c * RS + t]);
            float gpre = gv, dzv = 0.0f;
            if (has_z) {
                const float zv = ldf(&zs[c * RS + t]);
                const float sg = sigmoid_f(zv);
                gpre = gv * zv * sg;
                dzv = gv * fmaf(uv, Dd, yv) * sg * fmaf(zv, 1.0f - sg, 1.0f);
            }
            float v[NPT];
#pragma unroll
            for (int j = 0; j < NPT; ++j) v[j] = gpre * x[j];
            bool owner;
            const int base = reduce_scatter<NPT, LO>(v, lane, owner);
            if (owner) {
#pragma unroll
                for (int i = 0; i < KEPT; ++i) dCw[(warp * kTile + t) * NPW + sub * NPT + base + i] = v[i];
            }
            if (sub == 0) {
                dps[c * FS + t] = dv;
                gps[c * FS + t] = gpre;
                if (has_z) stf(&zs[c * RS + t], dzv);
                dDacc = fmaf(gpre, uv, dDacc);
            }
        }
        __syncwarp();

        // ---- pass B: reverse over sub-blocks --------------------------------
        for (int sb = (len - 1) / TS; sb >= 0; --sb) {
            const int tb = sb * TS;
            const int nb = min(TS, len - tb);
            float xh[TS][NPT], ah[TS][NPT];
#pragma unroll
            for (int j = 0; j < NPT; ++j) x[j] = sck[(sb * NPT + j) * kThreads + tid];
#pragma unroll
            for (int jj = 0; jj < TS; ++jj) {
                if (jj < nb) {
                    const int t = tb + jj;
                    const float dv = dps[c * FS + t];
                    const float du = dv * ldf(&us[c * RS + t]);
                    const float dl = dv * kLog2e;
                    const float* Bt = Bs + t * NP + sub * NPT;
#pragma unroll
                    for (int j = 0; j < NPT; ++j) {
                        const float da = exp2_mufu(dl * An[j]);
                        ah[jj][j] = da;
                        xh[jj][j] = x[j];
                        x[j] = fmaf(da, x[j], du * Bt[j]);
                    }
                }
            }
#pragma unroll
            for (int jj = TS - 1; jj >= 0; --jj) {
                if (jj < nb) {
                    const int t = tb + jj;
                    const float dv = dps[c * FS + t];
                    const float gpre = gps[c * FS + t];
                    const float uv = ldf(&us[c * RS + t]);
                    const float du = dv * uv;
                    const float* Bt = Bs + t * NP + sub * NPT;
                    const float* Ct = Cs + t * NP + sub * NPT;
                    float duacc = 0.0f, ddacc = 0.0f;
                    float v[NPT];
#pragma unroll
                    for (int j = 0; j < NPT; ++j) {
                        const float dh = fmaf(gpre, Ct[j], q[j]);
                        const float tmp = dh * (ah[jj][j] * xh[jj][j]);
                        ddacc = fmaf(tmp, An[j], ddacc);
                        dA[j] = fmaf(tmp, dv, dA[j]);
                        duacc = fmaf(dh, Bt[j], duacc);
                        v[j] = dh * du;
                        q[j] = dh * ah[jj][j];
                    }
                    duacc = sum_low_lanes<LPC>(duacc);
                    ddacc = sum_low_lanes<LPC>(ddacc);
                    bool owner;
                    const int base = reduce_scatter<NPT, LO>(v, lane, owner);
                    if (owner) {
#pragma unroll
                        for (int i = 0; i < KEPT; ++i) dBw[(warp * kTile + t) * NPW + sub * NPT + base + i] = v[i];
                    }
                    if (sub == 0) {
                        const float dut = fmaf(dv, duacc, gpre * Dd);
                        const float ddp = fmaf(uv, duacc, ddacc);
                        float ddt = ddp;
                        if (softplus) ddt = ddp * softplus_grad_f(ldf(&ds[c * RS + t]) + bias);
                        dbacc += ddt;
                        stf(&gs[c * RS + t], dut);
                        stf(&ds[c * RS + t], ddt);
                    }
                }
            }
        }
        __syncthreads();

        // ---- write the chunk's gradients ------------------------------------
        store_act_tile<T, CPC>(ds, reinterpret_cast<T*>(a.ddelta), row0, rows, L, t0, len);
        store_act_tile<T, CPC>(gs, reinterpret_cast<T*>(a.du), row0, rows, L, t0, len);
        if (has_z) store_act_tile<T, CPC>(zs, reinterpret_cast<T*>(a.dz), row0, rows, L, t0, len);
        for (int i = tid; i < N * len; i += kThreads) {
            const int n = i / len, t = i % len;
            float sb_ = 0.0f, sc_ = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                sb_ += dBw[(w * kTile + t) * NPW + n];
                sc_ += dCw[(w * kTile + t) * NPW + n];
            }
            dBp[n * L + t0 + t] = sb_;
            dCp[n * L + t0 + t] = sc_;
        }
    }

    if (cvalid) {
        float* dap = a.dA_part + (b * a.dim + d) * N;
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = sub * NPT + j;
            if (n < N) dap[n] = dA[j];
        }
        if (sub == 0) {
            a.dD_part[b * a.dim + d] = dDacc;
            a.db_part[b * a.dim + d] = dbacc;
        }
    }
}

// Sum the per-CTA dB/dC partials and the per-batch dA/dD/d_bias partials.
__global__ void reduce_kernel(const Args a, float* dB, float* dC, float* dA, float* dD, float* db) {
    const int64_t N = a.dstate, L = a.length;
    const int64_t nbc = a.batch * a.groups * N * L;
    const int64_t nda = a.dim * N;
    const int64_t total = nbc + nda + 2 * a.dim;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (i < nbc) {
            const int64_t t = i % L, n = (i / L) % N, bg = i / (L * N);
            float sb = 0.0f, sc = 0.0f;
            for (int64_t k = 0; k < a.nct; ++k) {
                const int64_t off = ((bg * a.nct + k) * N + n) * L + t;
                sb += a.dB_part[off];
                sc += a.dC_part[off];
            }
            dB[i] = sb;
            dC[i] = sc;
        } else if (i < nbc + nda) {
            const int64_t k = i - nbc;
            float s = 0.0f;
            for (int64_t bb = 0; bb < a.batch; ++bb) s += a.dA_part[bb * nda + k];
            dA[k] = s;
        } else {
            const int64_t k = i - nbc - nda;
            const bool is_d = k < a.dim;
            const int64_t ch = is_d ? k : k - a.dim;
            const float* src = is_d ? a.dD_part : a.db_part;
            float s = 0.0f;
            for (int64_t bb = 0; bb < a.batch; ++bb) s += src[bb * a.dim + ch];
            float* dst = is_d ? dD : db;
            if (dst) dst[ch] = s;
        }
    }
}

// ------------------------------------------------------------------- host ----
struct Cfg { int npt, lpc; };

static bool fwd_cfg(int64_t N, Cfg& c) {
    if (N <= 4) c = {4, 1};
    else if (N <= 8) c = {8, 1};
    else if (N <= 16) c = {16, 1};
    else if (N <= 32) c = {16, 2};
    else if (N <= 64) c = {16, 4};
    else return false;
    return true;
}
static bool bwd_cfg(int64_t N, Cfg& c) {
    if (N <= 4) c = {4, 1};
    else if (N <= 8) c = {8, 1};
    else if (N <= 16) c = {8, 2};
    else if (N <= 32) c = {8, 4};
    else if (N <= 64) c = {8, 8};
    else return false;
    return true;
}
constexpr int kTS = 8;

template <typename T>
static size_t fwd_smem(const Cfg& c) {
    const int cpc = 32 / c.lpc * kWarps, np = c.npt * c.lpc;
    const int rs = kTile + Pad<T>::v;
    return align_up(4 * (size_t)cpc * rs * sizeof(T), 16) + 2 * (size_t)kTile * np * 4 + 16;
}
template <typename T>
static size_t bwd_smem(const Cfg& c) {
    const int cpc = 32 / c.lpc * kWarps, np = c.npt * c.lpc;
    const int rs = kTile + Pad<T>::v;
    size_t s = align_up(4 * (size_t)cpc * rs * sizeof(T), 16);
    s += 2 * (size_t)cpc * (kTile + 1) * 4;
    s = align_up(s, 16);
    s += 2 * (size_t)kTile * np * 4;
    s += 2 * (size_t)kWarps * kTile * (np + 1) * 4;
    s += (size_t)(kTile / kTS) * c.npt * kThreads * 4;
    return s + 32;
}

// mode: 0 = size query (inputs only), 1 = forward, 2 = backward
static int validate(const ssm_selective_scan_params* p, int mode) {
    const bool bwd = mode == 2;
    if (!p) return fail(SSM_ERR_INVALID, "null params");
    if (p->batch < 0 || p->dim < 0 || p->length < 0 || p->groups < 1 || p->dstate < 1)
        return fail(SSM_ERR_INVALID, "selective_scan: negative size, groups < 1 or dstate < 1");
    if (p->dim % p->groups)
        return fail(SSM_ERR_INVALID, "selective_scan: dim must be divisible by groups");
    if (p->act_dtype < 0 || p->act_dtype > 2 || p->bc_dtype < 0 || p->bc_dtype > 2)
        return fail(SSM_ERR_UNSUPPORTED, "selective_scan: unknown dtype");
    Cfg c;
    if (!fwd_cfg(p->dstate, c))
        return fail(SSM_ERR_UNSUPPORTED, "selective_scan: dstate above 64 is not supported");
    const bool empty = p->batch == 0 || p->dim == 0 || p->length == 0;
    if (!empty) {
        if (!p->u || !p->delta || !p->A || !p->B || !p->C)
            return fail(SSM_ERR_INVALID, "selective_scan: null input pointer");
        if ((p->flags & SSM_HAS_D) && !p->D) return fail(SSM_ERR_INVALID, "selective_scan: D is null");
        if ((p->flags & SSM_HAS_Z) && !p->z) return fail(SSM_ERR_INVALID, "selective_scan: z is null");
        if ((p->flags & SSM_HAS_BIAS) && !p->delta_bias)
            return fail(SSM_ERR_INVALID, "selective_scan: delta_bias is null");
    }
    if (bwd) {
        if ((p->dim * p->dstate > 0 && !p->dA) || (!empty && (!p->dout || !p->du || !p->ddelta || !p->dB || !p->dC || !p->checkpoints)))
            return fail(SSM_ERR_INVALID, "selective_scan bwd: null gradient pointer");
        if ((p->flags & SSM_HAS_Z) && !empty && !p->dz) return fail(SSM_ERR_INVALID, "selective_scan bwd: dz is null");
    } else if (mode == 1 && !empty && !p->y) {
        return fail(SSM_ERR_INVALID, "selective_scan: y is null");
    }
    return SSM_OK;
}

static void make_args(const ssm_selective_scan_params* p, int cpc, Args& a) {
    a.batch = p->batch; a.dim = p->dim; a.length = p->length; a.groups = p->groups;
    a.dstate = p->dstate; a.per_group = p->dim / p->groups;
    a.ntiles = ceil_div(p->length, kTile);
    a.nct = ceil_div(a.per_group, cpc);
    a.flags = p->flags; a.bc_dtype = p->bc_dtype;
    a.u = p->u; a.delta = p->delta; a.A = p->A; a.B = p->B; a.C = p->C;
    a.D = p->D; a.z = p->z; a.delta_bias = p->delta_bias;
    a.y = p->y; a.ckpt = p->checkpoints;
    a.dout = p->dout; a.du = p->du; a.ddelta = p->ddelta; a.dz = p->dz;
    a.dB_part = a.dC_part = a.dA_part = a.dD_part = a.db_part = nullptr;
}

struct WsLayout { size_t bc, da, dd, total; };
static WsLayout ws_layout(const ssm_selective_scan_params* p, int64_t nct) {
    WsLayout w;
    w.bc = align_up((size_t)(p->batch * p->groups * nct * p->dstate * p->length) * 4, 256);
    w.da = align_up((size_t)(p->batch * p->dim * p->dstate) * 4, 256);
    w.dd = align_up((size_t)(p->batch * p->dim) * 4, 256);
    w.total = 2 * w.bc + w.da + 2 * w.dd;
    return w;
}

template <typename T, int NPT, int LPC>
static int launch_fwd(const Args& a, cudaStream_t st) {
    const Cfg c{NPT, LPC};
    const size_t sm = fwd_smem<T>(c);
    auto k = fwd_kernel<T, NPT, LPC>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return check_launch("selective_scan fwd: smem attribute");
    dim3 grid((unsigned)a.nct, (unsigned)a.groups, (unsigned)a.batch);
    k<<<grid, kThreads, sm, st>>>(a);
    return check_launch("selective_scan fwd");
}

template <typename T, int NPT, int LPC>
static int launch_bwd(const Args& a, cudaStream_t st) {
    const Cfg c{NPT, LPC};
    const size_t sm = bwd_smem<T>(c);
    auto k = bwd_kernel<T, NPT, LPC, kTS>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return check_launch("selective_scan bwd: smem attribute");
    dim3 grid((unsigned)a.nct, (unsigned)a.groups, (unsigned)a.batch);
    k<<<grid, kThreads, sm, st>>>(a);
    return check_launch("selective_scan bwd");
}

template <typename T>
static int dispatch_fwd(const Cfg& c, const Args& a, cudaStream_t st) {
    if (c.npt == 4) return launch_fwd<T, 4, 1>(a, st);
    if (c.npt == 8) return launch_fwd<T, 8, 1>(a, st);
    if (c.lpc == 1) return launch_fwd<T, 16, 1>(a, st);
    if (c.lpc == 2) return launch_fwd<T, 16, 2>(a, st);
    return launch_fwd<T, 16, 4>(a, st);
}
template <typename T>
static int dispatch_bwd(const Cfg& c, const Args& a, cudaStream_t st) {
    if (c.npt == 4) return launch_bwd<T, 4, 1>(a, st);
    if (c.lpc == 1) return launch_bwd<T, 8, 1>(a, st);
    if (c.lpc == 2) return launch_bwd<T, 8, 2>(a, st);
    if (c.lpc == 4) return launch_bwd<T, 8, 4>(a, st);
    return launch_bwd<T, 8, 8>(a, st);
}

}  // namespace sscan
}  // namespace ssm

using namespace ssm;
using namespace ssm::sscan;

extern "C" int ssm_selective_scan_sizes(const ssm_selective_scan_params* p,
                                        size_t* checkpoint_bytes, size_t* workspace_bytes) {
    if (int s = validate(p, 0)) return s;
    Cfg cb;
    bwd_cfg(p->dstate, cb);
    const int64_t nct = ceil_div(p->dim / p->groups, 32 / cb.lpc * kWarps);
    if (checkpoint_bytes)
        *checkpoint_bytes = (size_t)(p->batch * ceil_div(p->length, kTile) * p->dim * p->dstate) * 4;
    if (workspace_bytes) *workspace_bytes = ws_layout(p, nct).total;
    return SSM_OK;
}

extern "C" int ssm_selective_scan_fwd(const ssm_selective_scan_params* p, void* stream) {
    if (int s = validate(p, 1)) return s;
    if (p->batch == 0 || p->dim == 0 || p->length == 0) return SSM_OK;
    Cfg c;
    fwd_cfg(p->dstate, c);
    Args a;
    make_args(p, 32 / c.lpc * kWarps, a);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (p->act_dtype) {
        case SSM_F32: return dispatch_fwd<float>(c, a, st);
        case SSM_BF16: return dispatch_fwd<__nv_bfloat16>(c, a, st);
        default: return dispatch_fwd<__half>(c, a, st);
    }
}

extern "C" int ssm_selective_scan_bwd(const ssm_selective_scan_params* p, void* stream) {
    if (int s = validate(p, 2)) return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const bool empty = p->batch == 0 || p->dim == 0 || p->length == 0;
    if (empty) {
        // No steps: every parameter gradient is zero.
        if (p->dim && p->dstate && p->dA && cudaMemsetAsync(p->dA, 0, (size_t)(p->dim * p->dstate) * 4, st) != cudaSuccess)
            return check_launch("selective_scan bwd: memset");
        if (p->dD && p->dim) cudaMemsetAsync(p->dD, 0, (size_t)p->dim * 4, st);
        if (p->ddelta_bias && p->dim) cudaMemsetAsync(p->ddelta_bias, 0, (size_t)p->dim * 4, st);
        size_t nbc = (size_t)(p->batch * p->groups * p->dstate * p->length) * 4;
        if (nbc) { cudaMemsetAsync(p->dB, 0, nbc, st); cudaMemsetAsync(p->dC, 0, nbc, st); }
        return check_launch("selective_scan bwd: memset");
    }
    Cfg c;
    bwd_cfg(p->dstate, c);
    Args a;
    make_args(p, 32 / c.lpc * kWarps, a);
    const WsLayout w = ws_layout(p, a.nct);
    if (!p->workspace || p->workspace_bytes < w.total)
        return fail(SSM_ERR_WORKSPACE, "selective_scan bwd: workspace too small");
    char* ws = reinterpret_cast<char*>(p->workspace);
    a.dB_part = reinterpret_cast<float*>(ws);
    a.dC_part = reinterpret_cast<float*>(ws + w.bc);
    a.dA_part = reinterpret_cast<float*>(ws + 2 * w.bc);
    a.dD_part = reinterpret_cast<float*>(ws + 2 * w.bc + w.da);
    a.db_part = reinterpret_cast<float*>(ws + 2 * w.bc + w.da + w.dd);
    int s;
    switch (p->act_dtype) {
        case SSM_F32: s = dispatch_bwd<float>(c, a, st); break;
        case SSM_BF16: s = dispatch_bwd<__nv_bfloat16>(c, a, st); break;
        default: s = dispatch_bwd<__half>(c, a, st); break;
    }
    if (s) return s;
    const int64_t total = p->batch * p->groups * p->dstate * p->length + p->dim * p->dstate + 2 * p->dim;
    const int blocks = (int)min64(ceil_div(total, 256), 148 * 16);
    reduce_kernel<<<blocks, 256, 0, st>>>(a, p->dB, p->dC, p->dA,
                                          (p->flags & SSM_HAS_D) ? p->dD : nullptr,
                                          (p->flags & SSM_HAS_BIAS) ? p->ddelta_bias : nullptr);
    return check_launch("selective_scan bwd: reduce");
}
