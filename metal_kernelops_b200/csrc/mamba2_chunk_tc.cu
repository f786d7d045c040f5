// Mamba-2 SSD chunk scan on the sm_100a tensor cores (tcgen05 + TMEM).
//
// Reference behaviour: src/metal_kernelops/cv/mamba2_chunk.py:617-723 (the
// public op) and its chunk factorisation :15-31 / :447-533.  This path serves
// bf16 and f16 inputs whose headdim is a multiple of 8 up to 64, or 128 or
// 256, and whose dstate is a multiple of 8 up to 128; the tiles are
// 64 columns by 128 states (the Mamba-2 layer shape), smaller shapes fill them
// with zeros, and a wider head runs as several 64-column virtual heads.  Every
// other case runs the CUDA-core kernels of mamba2_chunk.cu.  The internal
// chunk is Q = 128 positions whatever chunk_size the caller asks for (the
// result does not depend on it).
//
// Per (batch b, head h, chunk c), with d_s the (softplus'd) step, cd_s its
// running sum inside the chunk, cs_s = A_h cd_s, T = cs_{Q-1}, G = C B^T:
//
//   Mh[l][s] = G[l][s] exp(cs_l - cs_s) d_s            (s <= l, else 0)
//   y_l      = (Mh X)_l + exp(cs_l) (C H_c^T)_l + D x_l          [* silu(z_l)]
//   H_{c+1}  = exp(T) H_c + sum_s exp(T - cs_s) d_s x_s B_s^T    (P x N)
//
// Kernels.  Forward: `states2` (one CTA per (b, h), sequential over chunks,
// warp-specialised) computes each chunk's own contribution B^T (w o X) on the
// tensor core into a TMEM buffer, ahead of the recurrence, while the CUDA
// cores carry H^T (dstate x headdim) in registers -- H_{c+1} = exp(T) H_c +
// B^T (w o X) -- and write every entering state H_c as a 16 KB operand image
// (bf16/f16, the shared-memory tile layout of tc.cuh), so that the consumers
// copy it linearly.  `outputs` (one CTA per (b, group, chunk))
// computes G once, then for each head of the group the decay-masked Mh into
// shared memory and the two output GEMMs Mh X and C H_c^T.
//
// Backward: `dstates` (one CTA per (b, h), reverse over chunks) carries dH^T in
// TMEM: dH_c = exp(T) dH_{c+1} + sum_l exp(cs_l) dy_l C_l^T, written as operand
// images; it also produces exp(T_c) <dH_{c+1}, H_c> and the per-position
// derivative of the inter-chunk output with respect to cs.  The derivative with
// respect to the chunk's total decay T_c is <dH_{c+1}, H_{c+1}> =
// exp(T_c) <dH_{c+1}, H_c> + sum_s d_s v_s (v_s = exp(T - cs_s) <x_s, dH_{c+1} B_s>);
// `grads` adds the second sum from the same v_s it subtracts at each position,
// so the two cancel exactly instead of leaving the rounding of two differently
// rounded state products (which dominated dA and d dt_bias in bf16).  `grads` (one CTA
// per (b, group, chunk)) runs eight GEMMs per head -- dY X^T, Mh^T dY,
// B dH^T, dG B, dYs H, dG^T C, (w o X) dH -- accumulating dB and dC for the
// whole group in TMEM, and finishes dx, d dt and the parameter partials.  Every
// reduction has a fixed order: the backward is deterministic.
//
// Operands are rounded to the input dtype before each GEMM (fp32 accumulate),
// so the result carries the input dtype's rounding, as the reference's own
// bf16/f16 runs do.
#include <mutex>
#include <string>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "ssd_tc.h"
#include "tc.cuh"

namespace ssm {
namespace ssdtc {

constexpr int Q = 128;        // chunk
constexpr int P = 64;         // headdim
constexpr int N = 128;        // dstate
constexpr int kThreads = 128;
constexpr int WX = P / 8;     // 16-byte chunks per row of an X-like tile (Q x P)
constexpr int WB = N / 8;     // per row of a B/C-like tile (Q x N)
constexpr int WH = P / 8;     // per row of an H^T tile (N x P)
constexpr uint32_t kTileX = Q * P * 2;
constexpr uint32_t kTileB = Q * N * 2;
constexpr uint32_t kTileH = N * P * 2;

__device__ int g_kernel_error;

struct Args {
    int64_t batch, length, nheads, ngroups, nc;
    int64_t b0;            // first batch row of this launch (grids cover a range of rows)
    // The tiles are P = 64 columns by N = 128 states.  A head whose headdim is a
    // multiple of 64 above 64 runs as pr "virtual heads" of 64 columns each
    // (columns of x, y and of the state are independent, and every gradient
    // that sums over columns is a sum of the virtual heads' parts); a smaller
    // headdim (a multiple of 8) and a dstate below 128 (a multiple of 8) fill
    // the tiles' leading columns / states, the rest reading as zeros.
    int64_t hv, pr;        // virtual heads (nheads * pr), virtual heads per head (1, 2 or 4)
    int prs;               // log2(pr): virtual head v belongs to head v >> prs
    int64_t hpg;           // virtual heads per group
    int64_t pa, pw, na;    // the caller's headdim, data columns per virtual head (min(pa, 64)), dstate
    int64_t xts;           // elements between tokens of x
    int fold;              // the tensor maps copy a whole tile per box (see encode_rows)
    uint32_t flags;
    int dt_dtype;
    const void* x; const void* dt; const float* A; const void* B; const void* C;
    const float* D; const void* z; const float* dt_bias; const float* init;
    void* y; float* final_state;
    unsigned char* Ht;     // (b, virtual head, c) H_c^T tiles, the state entering chunk c
    void* ypre;            // (b, l, virtual head, P) pre-gate output, saved when z is given
    const void* dy; const float* dfinal;
    void* dx; float* ddt; float* dB; float* dC; void* dz; float* dinit;
    unsigned char* dHt;    // (b, virtual head, c) dH_{c+1}^T tiles
    float* dcs_inter;      // (b, virtual head, nc * Q)
    float* dT;             // (b, virtual head, nc)
    float* dA_part; float* db_part; float* dD_part;   // (b, virtual head, nc) [x P]
    int* status;           // the call's optional status word (params.status)
    // TMA descriptors of x, dy (X-like rows) and B, C (B-like rows); see encode_rows()
    alignas(64) CUtensorMap tm_x;
    alignas(64) CUtensorMap tm_dy;
    alignas(64) CUtensorMap tm_B;
    alignas(64) CUtensorMap tm_C;
};

// ----------------------------------------------------------- element types --
template <typename T> struct Pk;
template <> struct Pk<__nv_bfloat16> {
    static constexpr uint32_t kFmt = 1;
    static __device__ __forceinline__ void unpack(const uint4& q, float* f) {
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
};
template <> struct Pk<__half> {
    static constexpr uint32_t kFmt = 0;
    static __device__ __forceinline__ void unpack(const uint4& q, float* f) {
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            f[2 * i] = v.x;
            f[2 * i + 1] = v.y;
        }
    }
    static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
        __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
};
template <typename T>
__device__ __forceinline__ uint4 pack8(const float* f) {
    return make_uint4(Pk<T>::pack2(f[0], f[1]), Pk<T>::pack2(f[2], f[3]), Pk<T>::pack2(f[4], f[5]),
                      Pk<T>::pack2(f[6], f[7]));
}

// Shape accessors.  PAD = false is the tile shape itself (headdim 64, dstate
// 128: compile-time constants, no virtual heads); PAD = true reads the
// caller's shape from the arguments.
template <bool PAD> __device__ __forceinline__ int pw_of(const Args& a) { return PAD ? (int)a.pw : P; }
template <bool PAD> __device__ __forceinline__ int64_t na_of(const Args& a) { return PAD ? a.na : N; }
template <bool PAD> __device__ __forceinline__ int64_t head_of(const Args& a, int64_t v) { return PAD ? v >> a.prs : v; }

// Element offsets of virtual head v.  Row of token t in a dense (b, l, heads,
// headdim) tensor (z, y, dy, dx, dz): virtual head v's columns start at v * pw.
template <bool PAD>
__device__ __forceinline__ int64_t row_off(const Args& a, int64_t b, int64_t t, int64_t v) {
    return (b * a.length + t) * a.nheads * (PAD ? a.pa : P) + v * pw_of<PAD>(a);
}
// Row of token t in the saved pre-gate output (internal, P columns per virtual head).
__device__ __forceinline__ int64_t prow_off(const Args& a, int64_t b, int64_t t, int64_t v) {
    return ((b * a.length + t) * a.hv + v) * P;
}
// Row p (p < pw) of virtual head v in a (b, heads, headdim, dstate) state tensor.
template <bool PAD>
__device__ __forceinline__ int64_t state_off(const Args& a, int64_t b, int64_t v, int64_t p) {
    return ((b * a.hv + v) * pw_of<PAD>(a) + p) * na_of<PAD>(a);
}

__device__ __forceinline__ float ld_dt(const Args& a, int64_t i) {
    switch (a.dt_dtype) {
        case SSM_F32: return reinterpret_cast<const float*>(a.dt)[i];
        case SSM_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.dt)[i]);
        default: return __half2float(reinterpret_cast<const __half*>(a.dt)[i]);
    }
}

// A bounded wait ran out (or a copy could not be issued): record the code in
// the device's flag and in the call's status word; the first failure wins.
__device__ __forceinline__ void report(int* status, int code) {
    atomicCAS(&g_kernel_error, 0, code);
    if (status) atomicCAS(status, 0, code);
}
__device__ __forceinline__ void report(const Args& a, int code) { report(a.status, code); }

// ------------------------------------------------------------ block helpers --
// Barrier over the whole CTA (NB = 0) or over the first NB threads only (named
// barrier 1), for kernels whose compute warps run beside an MMA-issuing warp.
template <int NB>
__device__ __forceinline__ void gsync() {
    if (NB) asm volatile("bar.sync 1, %0;" :: "n"(NB) : "memory");
    else __syncthreads();
}
// True on each of the first NB threads iff `v` is true on all of them.
template <int NB>
__device__ __forceinline__ bool cg_all(bool v) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, 1, %2, q;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}\n" : "=r"(r) : "r"((uint32_t)v), "n"(NB) : "memory");
    return r != 0;
}
// Warps taking part in a block-level helper.
template <int NB> constexpr int group_warps() { return (NB ? NB : kThreads) / 32; }

template <int NB = 0>
__device__ __forceinline__ float block_incl_scan(float v, float* sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    if (lane == 31) sh[w] = v;
    gsync<NB>();
    float off = 0.0f;
    for (int i = 0; i < w; ++i) off += sh[i];
    gsync<NB>();
    return v + off;
}
template <int NB = 0>
__device__ __forceinline__ float block_suffix_scan(float v, float* sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_down_sync(0xffffffffu, v, o);
        if (lane + o < 32) v += u;
    }
    if (lane == 0) sh[w] = v;
    gsync<NB>();
    float off = 0.0f;
    for (int i = group_warps<NB>() - 1; i > w; --i) off += sh[i];
    gsync<NB>();
    return v + off;
}
// Sum over the CTA; every thread gets the total (fixed order).
template <int NB = 0>
__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    gsync<NB>();
    float s = 0.0f;
    for (int i = 0; i < group_warps<NB>(); ++i) s += sh[i];
    gsync<NB>();
    return s;
}

// The same reductions over the first NB threads with two alternating scratch
// rows (`pp` is [2][16] floats, `k` a per-thread call counter that every
// thread advances alike): one barrier each.  A call writes the row its
// predecessor did not, and the call before that one has been read by every
// thread before any thread passed the barrier of the call in between.
template <int NB>
__device__ __forceinline__ float pp_sum(float v, float* pp, int& k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    float* row = pp + 16 * k;
    k ^= 1;
    if ((threadIdx.x & 31) == 0) row[threadIdx.x >> 5] = v;
    gsync<NB>();
    float s = 0.0f;
    for (int i = 0; i < group_warps<NB>(); ++i) s += row[i];
    return s;
}
// two sums at once (NB <= 256)
template <int NB>
__device__ __forceinline__ float2 pp_sum2(float2 v, float* pp, int& k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
        v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
    }
    float* row = pp + 16 * k;
    k ^= 1;
    if ((threadIdx.x & 31) == 0) {
        row[threadIdx.x >> 5] = v.x;
        row[8 + (threadIdx.x >> 5)] = v.y;
    }
    gsync<NB>();
    float2 s = make_float2(0.0f, 0.0f);
    for (int i = 0; i < group_warps<NB>(); ++i) {
        s.x += row[i];
        s.y += row[8 + i];
    }
    return s;
}
template <int NB>
__device__ __forceinline__ float pp_incl_scan(float v, float* pp, int& k) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    float* row = pp + 16 * k;
    k ^= 1;
    if (lane == 31) row[w] = v;
    gsync<NB>();
    float off = 0.0f;
    for (int i = 0; i < w; ++i) off += row[i];
    return v + off;
}
template <int NB>
__device__ __forceinline__ float pp_suffix_scan(float v, float* pp, int& k) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_down_sync(0xffffffffu, v, o);
        if (lane + o < 32) v += u;
    }
    float* row = pp + 16 * k;
    k ^= 1;
    if (lane == 0) row[w] = v;
    gsync<NB>();
    float off = 0.0f;
    for (int i = group_warps<NB>() - 1; i > w; --i) off += row[i];
    return v + off;
}

// Dynamic shared memory, rounded up to 128 bytes: TMA tile destinations need
// that alignment whatever the size of the kernel's static shared variables
// (the launches reserve kSmemPad extra bytes).
constexpr size_t kSmemPad = 128;
__device__ __forceinline__ unsigned char* aligned_smem(unsigned char* raw) {
    const uint32_t mis = tc::smem_u32(raw) & 127u;
    return raw + ((128u - mis) & 127u);
}

// The Q rows of chunk c of head / group hg of batch b, from a tensor map made by
// encode_rows(): with `fold`, one box that is the whole tile; otherwise Q/8
// boxes of 8 rows, each landing as the 8-row group of core matrices of the
// tile.  Rows past the sequence come back as zeros.  One thread issues; the
// bytes (Q * W * 16) complete on `mbar`.  (Each box costs the issuing thread
// tens of cycles: sixteen per tile kept the other warps of the CTA waiting at
// their next barrier.)
template <int W>
__device__ __forceinline__ void tma_rows(unsigned char* tile, const CUtensorMap& map, int64_t c, int64_t b,
                                         int64_t hg, uint32_t mbar, int* status, int fold) {
    if (reinterpret_cast<uintptr_t>(&map) & 63u) {   // descriptors must be 64-byte aligned: never issue
        report(status, 98);
        return;
    }
    const uint32_t st = tc::smem_u32(tile);
    if (fold) {
        tc::tma_load5(st, &map, 0, 0, (int)(hg * W), (int)(c * (Q / 8)), (int)b, mbar);
        return;
    }
#pragma unroll 4
    for (int k = 0; k < Q / 8; ++k)
        tc::tma_load5(st + k * W * 128, &map, 0, (int)(c * Q + 8 * k), 0, (int)b, (int)hg, mbar);
}
constexpr uint32_t kRowsX = Q * WX * 16;   // bytes of an X-like tile
constexpr uint32_t kRowsB = Q * WB * 16;   // bytes of a B-like tile

// Per-chunk step quantities of one head, thread s owning position s.
struct Steps {
    float raw;   // dt + bias (before the softplus)
    float d;     // step (0 beyond the sequence)
    float cd;    // running sum of d inside the chunk
    float cs;    // A * cd
};
// dt + bias of this thread's position of chunk c (0 beyond the sequence); h is
// a head of the caller's problem (not a virtual head).
__device__ __forceinline__ float raw_dt(const Args& a, int64_t b, int64_t h, int64_t c, float bias) {
    const int64_t t = c * Q + threadIdx.x;
    return t < a.length ? ld_dt(a, (b * a.length + t) * a.nheads + h) + bias : 0.0f;
}
template <int NB = 0>
__device__ __forceinline__ Steps steps_of(const Args& a, float raw, int64_t c, float Ah, float* scan_sh) {
    Steps s;
    const bool valid = threadIdx.x < Q && c * Q + threadIdx.x < a.length;
    s.raw = raw;
    s.d = valid ? ((a.flags & SSM_SOFTPLUS) ? softplus_f(raw) : raw) : 0.0f;
    s.cd = block_incl_scan<NB>(s.d, scan_sh);
    s.cs = Ah * s.cd;
    return s;
}

// dt + bias, A and D of up to kHeadsSh heads of a group for one chunk, loaded
// together so that their global latency is paid once, not once per head.
constexpr int kHeadsSh = 16;
struct HeadSh {
    float raw[kHeadsSh][Q + 1];     // dt + bias (padded row: conflict-free writes)
    float A[kHeadsSh], D[kHeadsSh];
};
template <int NT = kThreads>
__device__ __forceinline__ void stage_heads(const Args& a, HeadSh& hs, int64_t b, int64_t g, int64_t c,
                                            int64_t hh0, int n) {
    const int64_t h0 = g * a.hpg + hh0;       // first virtual head
    const bool has_bias = a.flags & SSM_HAS_BIAS;
    if ((int)threadIdx.x < n) {
        const int64_t h = (h0 + threadIdx.x) >> a.prs;
        hs.A[threadIdx.x] = a.A[h];
        hs.D[threadIdx.x] = ((a.flags & SSM_HAS_D) && !(a.flags & SSM_D_PER_HEAD)) ? a.D[h] : 0.0f;
    }
    for (int i = threadIdx.x; i < n * Q; i += NT) {
        const int pos = i / n, k = i % n;     // consecutive threads: consecutive heads of one position
        const int64_t t = c * Q + pos, h = (h0 + k) >> a.prs;
        float v = 0.0f;
        if (t < a.length) v = ld_dt(a, (b * a.length + t) * a.nheads + h) + (has_bias ? a.dt_bias[h] : 0.0f);
        hs.raw[k][pos] = v;
    }
}
template <int NB = 0>
__device__ __forceinline__ Steps staged_steps(const Args& a, const HeadSh& hs, int k, int64_t c, float* scan_sh) {
    return steps_of<NB>(a, threadIdx.x < Q ? hs.raw[k][threadIdx.x] : 0.0f, c, hs.A[k], scan_sh);
}
// staged_steps with the one-barrier scan (ping-pong scratch, see pp_sum)
template <int NB>
__device__ __forceinline__ Steps staged_steps_pp(const Args& a, const HeadSh& hs, int k, int64_t c, float* pp,
                                                 int& kk) {
    Steps s;
    const float raw = threadIdx.x < Q ? hs.raw[k][threadIdx.x] : 0.0f;
    const bool valid = threadIdx.x < Q && c * Q + threadIdx.x < a.length;
    s.raw = raw;
    s.d = valid ? ((a.flags & SSM_SOFTPLUS) ? softplus_f(raw) : raw) : 0.0f;
    s.cd = pp_incl_scan<NB>(s.d, pp, kk);
    s.cs = hs.A[k] * s.cd;
    return s;
}

// ===================================================================== F1b ==
// The forward state pass, warp-specialised, with the chunk-state GEMMs off the
// sequential chain.  One CTA per (b, h), chunks in order.  Four compute warps:
// thread n carries row n of H^T (64 fp32 values) in registers; per chunk c it
// scales its position's row of X_c in place to w o X_c, and then folds the
// previous chunk's contribution into H after emitting H_{c-1}:
// H_c = exp(T_{c-1}) H_{c-1} + S_{c-1}.  One producer warp issues every copy
// and GEMM: the tensor core computes each chunk's own S_c = B_c^T (w o X_c)
// into one of two TMEM buffers (64 columns each), so no GEMM waits on the
// recurrence and no compute warp waits on a copy being issued.  Hand-offs are
// mbarriers: tiles landed (copy -> compute, copy -> GEMM), w o X ready
// (compute -> GEMM, 128 arrivals), S ready (GEMM -> compute and -> the next
// copies into its buffers), S buffer read (compute -> GEMM, 128 arrivals).
// Two tile buffers for X and B (96 KB), 128 TMEM columns: two CTAs per SM.
constexpr int kStThreads = kThreads + 32;
constexpr size_t kSmemStates2 = 2 * kTileB + 2 * kTileX;

template <typename T, bool PAD>
__global__ void __launch_bounds__(kStThreads, 2) states2_kernel(const __grid_constant__ Args a) {
    extern __shared__ __align__(128) unsigned char sm_raw[];
    unsigned char* const sm = aligned_smem(sm_raw);
    unsigned char* const sB0 = sm;
    unsigned char* const sX0 = sm + 2 * kTileB;
    __shared__ float s_scan[4];
    __shared__ float s_T[2];
    __shared__ __align__(8) uint64_t lbx[2];    // X tile of buffer i landed
    __shared__ __align__(8) uint64_t lbb[2];    // B tile of buffer i landed
    __shared__ __align__(8) uint64_t xw[2];     // w o X of buffer i written (128 arrivals)
    __shared__ __align__(8) uint64_t sbar[2];   // the GEMM into S buffer i done
    __shared__ __align__(8) uint64_t sfree[2];  // S buffer i read by the compute warps (128 arrivals)
    __shared__ uint32_t tbase;
    __shared__ volatile int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5;
    const bool producer = warp == kThreads / 32;
    const int64_t h = blockIdx.x, b = blockIdx.y + a.b0, g = h / a.hpg;   // h: virtual head
    const int64_t H = a.hv, nc = a.nc;
    auto bar = [](uint64_t* m, int i) { return tc::smem_u32(&m[i]); };

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(bar(lbx, i), 1);
            tc::mbar_init(bar(lbb, i), 1);
            tc::mbar_init(bar(xw, i), kThreads);
            tc::mbar_init(bar(sbar, i), 1);
            tc::mbar_init(bar(sfree, i), kThreads);
        }
        s_abort = 0;
        tc::fence_mbar_init();
    }
    if (producer) tc::tmem_alloc(tc::smem_u32(&tbase), 128);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tm = tbase;

    if (producer) {
        if ((tid & 31) == 0) {
            const uint32_t id = tc::idesc_f16(Pk<T>::kFmt, 128, P, true, true);
            uint32_t xpend[2] = {~0u, ~0u}, bpend[2] = {~0u, ~0u}, mpend[2] = {~0u, ~0u};
            bool ok = true;
            auto load = [&](int64_t c) {
                const int buf = (int)(c & 1);
                const uint32_t par = (uint32_t)((c >> 1) & 1);
                tc::mbar_expect_tx(bar(lbx, buf), kRowsX);
                tma_rows<WX>(sX0 + buf * kTileX, a.tm_x, c, b, h, bar(lbx, buf), a.status, a.fold);
                tc::mbar_expect_tx(bar(lbb, buf), kRowsB);
                tma_rows<WB>(sB0 + buf * kTileB, a.tm_B, c, b, g, bar(lbb, buf), a.status, a.fold);
                xpend[buf] = bpend[buf] = par;
            };
            load(0);
            for (int64_t c = 0; c < nc && ok; ++c) {
                const int buf = (int)(c & 1);
                const uint32_t par = (uint32_t)((c >> 1) & 1);
                if (c + 1 < nc) {             // chunk c + 1's tiles, once the GEMM of c - 1 is done with its buffers
                    const int nb = buf ^ 1;
                    if (c >= 1) {
                        if (!tc::mbar_wait(bar(sbar, nb), (uint32_t)(((c - 1) >> 1) & 1))) { report(a, 81); ok = false; break; }
                        mpend[nb] = ~0u;
                    }
                    load(c + 1);
                }
                // the GEMM of c: w o X written, B landed, the S buffer read
                if (!tc::mbar_wait(bar(xw, buf), par)) { report(a, 82); ok = false; break; }
                xpend[buf] = ~0u;             // the compute warps waited for it
                if (!tc::mbar_wait(bar(lbb, buf), par)) { report(a, 83); ok = false; break; }
                bpend[buf] = ~0u;
                if (c >= 2 && !tc::mbar_wait(bar(sfree, buf), (uint32_t)(((c - 2) >> 1) & 1))) {
                    report(a, 84); ok = false; break;
                }
                tc::fence_after();
                const uint32_t aB = tc::smem_u32(sB0 + buf * kTileB), aX = tc::smem_u32(sX0 + buf * kTileX);
                const uint32_t dst = tm + (uint32_t)(buf * P);
#pragma unroll
                for (int ks = 0; ks < Q / 16; ++ks)
                    tc::mma_f16(dst, tc::desc_mn(aB, WB, 16 * ks), tc::desc_mn(aX, WX, 16 * ks), id, ks > 0);
                tc::commit(bar(sbar, buf));
                mpend[buf] = par;
                if (s_abort) { ok = false; break; }
            }
            if (!ok) s_abort = 1;
            // no copy may land and no GEMM may run after exit
            for (int i = 0; i < 2; ++i) {
                if (xpend[i] != ~0u) tc::mbar_wait(bar(lbx, i), xpend[i]);
                if (bpend[i] != ~0u) tc::mbar_wait(bar(lbb, i), bpend[i]);
                if (mpend[i] != ~0u) tc::mbar_wait(bar(sbar, i), mpend[i]);
            }
        }
        __syncwarp();
    } else {
        const int64_t hh = head_of<PAD>(a, h);  // the caller's head
        const float Ah = a.A[hh];
        const float bias = (a.flags & SSM_HAS_BIAS) ? a.dt_bias[hh] : 0.0f;
        const uint32_t row_addr = tm + ((uint32_t)(warp * 32) << 16);
        unsigned char* Hout = a.Ht + (size_t)(b * H + h) * nc * kTileH;
        const bool nrow = tid < na_of<PAD>(a);  // state n = tid exists (else its row stays 0)
        float hr[P];                            // row n = tid of H^T
#pragma unroll
        for (int p = 0; p < P; ++p)
            hr[p] = ((a.flags & SSM_HAS_INIT) && nrow && p < pw_of<PAD>(a)) ? a.init[state_off<PAD>(a, b, h, p) + tid] : 0.0f;
        bool ok = true;
        // emit H_c, then fold in S_c from TMEM buffer c & 1
        auto consume = [&](int64_t c) -> bool {
            const int buf = (int)(c & 1);
            if (!tc::mbar_wait(bar(sbar, buf), (uint32_t)((c >> 1) & 1))) { report(a, 85); return false; }
            tc::fence_after();
            unsigned char* out = Hout + (size_t)c * kTileH;
            const float eT = exp2_mufu(s_T[buf] * kLog2e);
            float sv[P / 16][16];
#pragma unroll
            for (int j = 0; j < P / 16; ++j) tc::tmem_ld16(row_addr + (uint32_t)(buf * P) + j * 16, sv[j]);
            tc::tmem_wait_ld(sv[0]);
#pragma unroll
            for (int j = 1; j < P / 16; ++j) tc::tmem_pin(sv[j]);
            tc::fence_before();
            tc::mbar_arrive(bar(sfree, buf));
#pragma unroll
            for (int j = 0; j < P / 16; ++j) {
                *reinterpret_cast<uint4*>(out + tc::tile_off(tid, 2 * j, WH)) = pack8<T>(hr + 16 * j);
                *reinterpret_cast<uint4*>(out + tc::tile_off(tid, 2 * j + 1, WH)) = pack8<T>(hr + 16 * j + 8);
#pragma unroll
                for (int k = 0; k < 16; ++k) hr[16 * j + k] = fmaf(eT, hr[16 * j + k], sv[j][k]);
            }
            return true;
        };
        float raw_next = raw_dt(a, b, hh, 0, bias);
        for (int64_t c = 0; c < nc && ok; ++c) {
            const int buf = (int)(c & 1);
            const float raw = raw_next;
            if (c + 1 < nc) raw_next = raw_dt(a, b, hh, c + 1, bias);   // in flight during this chunk
            const Steps st = steps_of<kThreads>(a, raw, c, Ah, s_scan);
            if (tid == Q - 1) s_T[buf] = st.cs;
            bool w_ok = tc::mbar_wait(bar(lbx, buf), (uint32_t)((c >> 1) & 1));
            if (!w_ok) report(a, 86);
            ok = cg_all<kThreads>(w_ok && !s_abort);   // also publishes s_T
            if (!ok) break;
            unsigned char* const sX = sX0 + buf * kTileX;
            const float w = exp2_mufu((s_T[buf] - st.cs) * kLog2e) * st.d;
#pragma unroll
            for (int j = 0; j < WX; ++j) {
                uint4* q = reinterpret_cast<uint4*>(sX + tc::tile_off(tid, j, WX));
                float f[8];
                Pk<T>::unpack(*q, f);
#pragma unroll
                for (int k = 0; k < 8; ++k) f[k] *= w;
                *q = pack8<T>(f);
            }
            tc::fence_async_smem();
            tc::mbar_arrive(bar(xw, buf));
            if (c > 0 && !consume(c - 1)) ok = false;
            ok = cg_all<kThreads>(ok && !s_abort);
        }
        if (ok) ok = consume(nc - 1);
        ok = cg_all<kThreads>(ok);
        if (ok && nrow) {
#pragma unroll
            for (int p = 0; p < P; ++p)
                if (p < pw_of<PAD>(a)) a.final_state[state_off<PAD>(a, b, h, p) + tid] = hr[p];
        } else if (!ok) {
            s_abort = 1;
        }
    }
    tc::fence_before();
    __syncthreads();
    if (producer) tc::tmem_dealloc(tm, 128);
}

// Decay factors for the mask of one head of one chunk, shared by the CTA:
// cs in log2 units, d, and cf_s = exp(cs_{e(s)} - cs_s) with e(s) the last
// position of s's 16-block.  For l past that block exp(cs_l - cs_s) =
// exp(cs_l - cs_{e(s)}) cf_s, and both factors are <= 1 when cs is
// non-increasing; the diagonal 16 x 16 blocks use direct exponentials.
struct __align__(16) MaskSh {   // 16-byte aligned: read as float2 pairs
    float cs2[Q];
    float d[Q];
    float cf[Q];
};
template <int NB = 0>
__device__ __forceinline__ void mask_factors(MaskSh& m, const Steps& st) {
    const int s = threadIdx.x;
    if (s < Q) {
        m.cs2[s] = st.cs * kLog2e;
        m.d[s] = st.d;
    }
    gsync<NB>();
    if (s < Q) m.cf[s] = exp2_mufu(m.cs2[s | 15] - m.cs2[s]);
    gsync<NB>();
}

// ====================================================================== F2 ==
// One CTA per (b, group, chunk), eight warps: warps w and w + 4 share TMEM lane
// quadrant w % 4 (rows l = 32 (w % 4) + lane) and split its work -- the mask
// pass by 16-column block parity (the lower-triangular mask gives quadrant q
// q + 1 blocks per warp instead of 2 q + 2 for a lone warp), the epilogue by
// column halves.  Threads 0..127 also own one chunk position each for the
// per-position scalars.  TMEM: G [0,128), Y intra [128,192), C H^T [192,256).
constexpr int kOutThreads = 256;

template <typename T, bool PAD>
__global__ void __launch_bounds__(kOutThreads, 2) outputs_kernel(const __grid_constant__ Args a) {
    extern __shared__ __align__(128) unsigned char sm_raw[];
    unsigned char* const sm = aligned_smem(sm_raw);
    unsigned char* sC = sm;
    unsigned char* sM = sm + kTileB;          // B, then Mh
    unsigned char* sX = sm + 2 * kTileB;
    unsigned char* sH = sX + kTileX;
    __shared__ MaskSh msh;
    __shared__ HeadSh hsh;
    __shared__ float s_scan[8];
    __shared__ __align__(8) uint64_t mbar;
    __shared__ __align__(8) uint64_t lbar;    // tile loads, one phase per load
    __shared__ uint32_t tbase;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q = warp & 3, hf = warp >> 2;   // TMEM lane quadrant, block parity / column half
    const int l = q * 32 + lane;              // TMEM row / chunk position of this thread
    const int64_t c = blockIdx.x, g = blockIdx.y, b = blockIdx.z + a.b0;
    const int64_t H = a.hv;
    const int64_t t0 = c * Q;
    const int valid = (int)min64(Q, a.length - t0);
    const int pw = pw_of<PAD>(a);
    const T* zg = reinterpret_cast<const T*>(a.z);
    T* yg = reinterpret_cast<T*>(a.y);
    T* ypg = reinterpret_cast<T*>(a.ypre);
    const bool has_z = a.flags & SSM_HAS_Z, has_d = a.flags & SSM_HAS_D;
    const bool d_per_head = a.flags & SSM_D_PER_HEAD;
    const uint32_t lb = tc::smem_u32(&lbar);
    uint32_t lpend = ~0u;                     // parity of a load still in flight (thread 0)

    if (warp == 0) tc::tmem_alloc(tc::smem_u32(&tbase), 256);
    if (tid == 0) {
        tc::mbar_init(tc::smem_u32(&mbar), 1);
        tc::mbar_init(lb, 1);
        tc::fence_mbar_init();
        tc::mbar_expect_tx(lb, 2 * kRowsB);
        tma_rows<WB>(sC, a.tm_C, c, b, g, lb, a.status, a.fold);
        tma_rows<WB>(sM, a.tm_B, c, b, g, lb, a.status, a.fold);
        lpend = 0;
    }
    __syncthreads();                          // the barriers are initialised before anyone waits
    bool lok = tc::mbar_wait(lb, 0);
    if (!lok) report(a, 23);
    else if (tid == 0) lpend = ~0u;
    tc::fence_before();
    lok = __syncthreads_and(lok);
    tc::fence_after();
    const uint32_t tm = tbase;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t aC = tc::smem_u32(sC), aM = tc::smem_u32(sM), aX = tc::smem_u32(sX), aH = tc::smem_u32(sH);
    if (tid == 0 && lok) {
        const uint32_t idg = tc::idesc_f16(Pk<T>::kFmt, 128, 128, false, false);
#pragma unroll
        for (int ks = 0; ks < N / 16; ++ks)
            tc::mma_f16(tm, tc::desc_k(aC, WB, 2 * ks), tc::desc_k(aM, WB, 2 * ks), idg, ks > 0);
        tc::commit(tc::smem_u32(&mbar));
    }
    uint32_t phase = 0;
    bool ok = lok && tc::mbar_wait(tc::smem_u32(&mbar), phase);
    if (lok && !ok) report(a, 21);
    phase ^= 1;
    tc::fence_after();
    ok = __syncthreads_and(ok);

    const uint32_t idy = tc::idesc_f16(Pk<T>::kFmt, 128, P, false, true);
    for (int64_t hh = 0; hh < a.hpg && ok; ++hh) {
        const int64_t h = g * a.hpg + hh;
        const uint32_t lpar = (uint32_t)((hh + 1) & 1);
        if (tid == 0) {   // the previous head's GEMMs and epilogue are done with sX and sH
            lpend = lpar;
            tc::mbar_expect_tx(lb, kRowsX + kTileH);
            tma_rows<WX>(sX, a.tm_x, c, b, h, lb, a.status, a.fold);
            tc::bulk_load(tc::smem_u32(sH), a.Ht + ((size_t)(b * H + h) * a.nc + c) * kTileH, kTileH, lb);
        }
        const int hk = (int)(hh % kHeadsSh);
        if (hk == 0) {
            stage_heads<kOutThreads>(a, hsh, b, g, c, hh, (int)min64(kHeadsSh, a.hpg - hh));
            __syncthreads();
        }
        const Steps st = staged_steps<kOutThreads>(a, hsh, hk, c, s_scan);
        mask_factors<kOutThreads>(msh, st);
        // Mh row l into sM (B is no longer needed once G is in TMEM): blocks
        // j = hf, hf + 2, ...; the quadrant's last live block is 2 q + 1, so
        // liveness is warp-uniform (tcgen05.ld is .sync.aligned)
        {
            const float csl = msh.cs2[l];
#pragma unroll 1
            for (int j = hf; j < Q / 16; j += 2) {
                uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
                if (j <= 2 * q + 1) {
                    float v[16];
                    tc::tmem_ld16(tm + lane_off + 16 * j, v);
                    tc::tmem_wait_ld(v);
                    if (16 * j <= l) {
                        if (16 * j + 15 < l) {
                            const float2 rf = f2(exp2_mufu(csl - msh.cs2[16 * j + 15]));
#pragma unroll
                            for (int k = 0; k < 16; k += 2) {   // v (rf cf d), in pairs
                                const float2 w = mul2(mul2(rf, *reinterpret_cast<const float2*>(&msh.cf[16 * j + k])),
                                                      *reinterpret_cast<const float2*>(&msh.d[16 * j + k]));
                                const float2 r = mul2(make_float2(v[k], v[k + 1]), w);
                                v[k] = r.x;
                                v[k + 1] = r.y;
                            }
                        } else {
#pragma unroll
                            for (int k = 0; k < 16; ++k) {
                                const int s = 16 * j + k;
                                v[k] = s <= l ? v[k] * exp2_mufu(csl - msh.cs2[s]) * msh.d[s] : 0.0f;
                            }
                        }
                        lo = pack8<T>(v);
                        hi = pack8<T>(v + 8);
                    }
                }
                *reinterpret_cast<uint4*>(sM + tc::tile_off(l, 2 * j, WB)) = lo;
                *reinterpret_cast<uint4*>(sM + tc::tile_off(l, 2 * j + 1, WB)) = hi;
            }
        }
        const bool lw = tc::mbar_wait(lb, lpar);      // this head's x and H_c
        if (!lw) report(a, 24);
        else if (tid == 0) lpend = ~0u;
        tc::fence_async_smem();
        tc::fence_before();
        if (!__syncthreads_and(lw)) { ok = false; break; }
        if (tid == 0) {
            tc::fence_after();
#pragma unroll
            for (int ks = 0; ks < Q / 16; ++ks)
                tc::mma_f16(tm + 128, tc::desc_k(aM, WB, 2 * ks), tc::desc_mn(aX, WX, 16 * ks), idy, ks > 0);
#pragma unroll
            for (int ks = 0; ks < N / 16; ++ks)
                tc::mma_f16(tm + 192, tc::desc_k(aC, WB, 2 * ks), tc::desc_mn(aH, WH, 16 * ks), idy, ks > 0);
            tc::commit(tc::smem_u32(&mbar));
        }
        // this row's gate inputs (its column half), loaded while the GEMMs run
        // (the waits below order every later memory access after them)
        const int64_t row = row_off<PAD>(a, b, t0 + l, h), prow = prow_off(a, b, t0 + l, h);
        constexpr int HALFC = P / 2;              // columns per thread
        const int col0 = hf * HALFC;
        uint4 zr[HALFC / 8];
        if (has_z && l < valid) {
#pragma unroll
            for (int u = 0; u < HALFC / 8; ++u)
                zr[u] = col0 + 8 * u < pw ? *reinterpret_cast<const uint4*>(zg + row + col0 + 8 * u) : make_uint4(0, 0, 0, 0);
        }
        if (!tc::mbar_wait(tc::smem_u32(&mbar), phase)) { report(a, 22); ok = false; }
        phase ^= 1;
        tc::fence_after();
        ok = __syncthreads_and(ok);
        if (ok) {
            const bool live = l < valid;
            const float el = exp2_mufu(msh.cs2[l]);
            const float Dh = hsh.D[hk];
#pragma unroll
            for (int jj = 0; jj < HALFC / 16; ++jj) {
                const int col = col0 + 16 * jj;
                float yi[16], ye[16];
                tc::tmem_ld16(tm + lane_off + 128 + col, yi);
                tc::tmem_ld16(tm + lane_off + 192 + col, ye);
                tc::tmem_wait_ld(yi);
                tc::tmem_pin(ye);
                if (!live) continue;
                float xv[16];
                Pk<T>::unpack(*reinterpret_cast<const uint4*>(sX + tc::tile_off(l, col / 8, WX)), xv);
                Pk<T>::unpack(*reinterpret_cast<const uint4*>(sX + tc::tile_off(l, col / 8 + 1, WX)), xv + 8);
                float yv[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const float Dk = has_d ? (d_per_head ? (col + k < pw ? a.D[h * pw + col + k] : 0.0f) : Dh)
                                           : 0.0f;
                    yv[k] = fmaf(el, ye[k], yi[k]) + Dk * xv[k];
                }
                if (has_z) {
                    if (ypg) {
                        *reinterpret_cast<uint4*>(ypg + prow + col) = pack8<T>(yv);
                        *reinterpret_cast<uint4*>(ypg + prow + col + 8) = pack8<T>(yv + 8);
                    }
                    float zv[16];
                    Pk<T>::unpack(zr[2 * jj], zv);
                    Pk<T>::unpack(zr[2 * jj + 1], zv + 8);
#pragma unroll
                    for (int k = 0; k < 16; ++k) yv[k] *= zv[k] * sigmoid_f(zv[k]);
                }
                if (col < pw) *reinterpret_cast<uint4*>(yg + row + col) = pack8<T>(yv);
                if (col + 8 < pw) *reinterpret_cast<uint4*>(yg + row + col + 8) = pack8<T>(yv + 8);
            }
        }
        tc::fence_before();
        __syncthreads();
    }
    if (tid == 0 && lpend != ~0u) tc::mbar_wait(lb, lpend);   // no copy may land after exit
    tc::fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tm, 256);
}

// ====================================================================== B1 ==
// One CTA per (b, h), chunks in reverse.  TMEM: dH^T [0,64), C H_c^T [64,128).
// GATED: z given (a separate instantiation, so that the ungated one carries no
// registers for the gate inputs it prefetches).
template <typename T, bool GATED, bool PAD>
__global__ void __launch_bounds__(kThreads) dstates_kernel(const __grid_constant__ Args a) {
    extern __shared__ __align__(128) unsigned char sm_raw[];
    unsigned char* const sm = aligned_smem(sm_raw);
    unsigned char* sC = sm;
    unsigned char* sH = sm + kTileB;
    unsigned char* sY = sm + kTileB + kTileH;   // dout, then exp(cs_l) dy_l
    __shared__ float s_scan[4];
    __shared__ float s_T;
    __shared__ __align__(8) uint64_t mbar;
    __shared__ __align__(8) uint64_t lbar;    // tile loads, one phase per chunk
    __shared__ uint32_t tbase;

    const int tid = threadIdx.x, warp = tid >> 5;
    const int64_t h = blockIdx.x, b = blockIdx.y + a.b0, g = h / a.hpg;   // h: virtual head
    const int64_t L = a.length, H = a.hv, hh = head_of<PAD>(a, h);   // hh: the caller's head
    const int pw = pw_of<PAD>(a);
    const bool nrow = tid < na_of<PAD>(a);    // state n = tid exists
    const float Ah = a.A[hh];
    const float bias = (a.flags & SSM_HAS_BIAS) ? a.dt_bias[hh] : 0.0f;
    const bool has_z = GATED;
    const T* zg = reinterpret_cast<const T*>(a.z);
    const T* ypg = reinterpret_cast<const T*>(a.ypre);
    T* dzg = reinterpret_cast<T*>(a.dz);
    const unsigned char* Hin = a.Ht + (size_t)(b * H + h) * a.nc * kTileH;
    unsigned char* dHout = a.dHt + (size_t)(b * H + h) * a.nc * kTileH;

    if (warp == 0) tc::tmem_alloc(tc::smem_u32(&tbase), 128);
    const uint32_t lb = tc::smem_u32(&lbar);
    uint32_t lpend = ~0u;                     // parity of a load still in flight (thread 0)
    if (tid == 0) {
        tc::mbar_init(tc::smem_u32(&mbar), 1);
        tc::mbar_init(lb, 1);
        tc::fence_mbar_init();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tm = tbase;
    const uint32_t row_addr = tm + ((uint32_t)(warp * 32) << 16);
    {
        float v[16];
        for (int j = 0; j < P / 16; ++j) {
#pragma unroll
            for (int k = 0; k < 16; ++k)
                v[k] = ((a.flags & SSM_HAS_DSTATE) && nrow && j * 16 + k < pw)
                           ? a.dfinal[state_off<PAD>(a, b, h, j * 16 + k) + tid] : 0.0f;
            tc::tmem_st16(row_addr + j * 16, v);
        }
        tc::tmem_wait_st();
    }
    const uint32_t idy = tc::idesc_f16(Pk<T>::kFmt, 128, P, false, true);
    const uint32_t idh = tc::idesc_f16(Pk<T>::kFmt, 128, P, true, true);
    const uint32_t aC = tc::smem_u32(sC), aY = tc::smem_u32(sY);
    uint32_t phase = 0;
    bool ok = true;
    float raw_next = raw_dt(a, b, hh, a.nc - 1, bias);
    for (int64_t c = a.nc - 1; c >= 0 && ok; --c) {
        const float raw = raw_next;
        if (c > 0) raw_next = raw_dt(a, b, hh, c - 1, bias);
        const int64_t t0 = c * Q;
        const int valid = (int)min64(Q, L - t0);
        const uint32_t lpar = (uint32_t)((a.nc - 1 - c) & 1);
        if (tid == 0) {   // the previous chunk's GEMMs and passes are done with these tiles
            tc::mbar_expect_tx(lb, kRowsB + kTileH + kRowsX);
            tma_rows<WB>(sC, a.tm_C, c, b, g, lb, a.status, a.fold);
            tc::bulk_load(tc::smem_u32(sH), Hin + (size_t)c * kTileH, kTileH, lb);
            tma_rows<WX>(sY, a.tm_dy, c, b, h, lb, a.status, a.fold);
            lpend = lpar;
        }
        const Steps st = steps_of(a, raw, c, Ah, s_scan);
        if (tid == Q - 1) s_T = st.cs;
        // the gate inputs of row l = tid, loaded while the tiles land
        const int64_t row = row_off<PAD>(a, b, t0 + tid, h), prow = prow_off(a, b, t0 + tid, h);
        uint4 zr[WX], ypr[WX];
        if (has_z && tid < valid) {
#pragma unroll
            for (int j = 0; j < WX; ++j) {
                zr[j] = 8 * j < pw ? *reinterpret_cast<const uint4*>(zg + row + 8 * j) : make_uint4(0, 0, 0, 0);
                if (dzg) ypr[j] = *reinterpret_cast<const uint4*>(ypg + prow + 8 * j);
            }
        }
        const bool lw = tc::mbar_wait(lb, lpar);
        if (!lw) report(a, 32);
        else if (tid == 0) lpend = ~0u;
        if (!__syncthreads_and(lw)) { ok = false; break; }
        const float Tc = s_T;
        // dy row l = tid: gate, then exp(cs_l) dy_l in place
        {
            const int l = tid;
            const float el = exp2_mufu(st.cs * kLog2e);
#pragma unroll
            for (int j = 0; j < WX; ++j) {
                float f[8];
                Pk<T>::unpack(*reinterpret_cast<const uint4*>(sY + tc::tile_off(l, j, WX)), f);
                if (has_z && l < valid) {
                    float zv[8], yp[8], dz[8];
                    Pk<T>::unpack(zr[j], zv);
                    if (dzg) Pk<T>::unpack(ypr[j], yp);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const float sg = sigmoid_f(zv[k]);
                        if (dzg) dz[k] = f[k] * yp[k] * sg * fmaf(zv[k], 1.0f - sg, 1.0f);
                        f[k] *= zv[k] * sg;
                    }
                    if (dzg && 8 * j < pw) *reinterpret_cast<uint4*>(dzg + row + 8 * j) = pack8<T>(dz);
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) f[k] *= el;
                *reinterpret_cast<uint4*>(sY + tc::tile_off(l, j, WX)) = pack8<T>(f);
            }
        }
        // dH_{c+1}: emit, <dH_{c+1}, H_c>, then dH^T <- exp(T) dH^T
        float dt_part = 0.0f;
        {
            unsigned char* out = dHout + (size_t)c * kTileH;
            const float eT = exp2_mufu(Tc * kLog2e);
            float v[P / 16][16];
#pragma unroll
            for (int j = 0; j < P / 16; ++j) tc::tmem_ld16(row_addr + j * 16, v[j]);
            tc::tmem_wait_ld(v[0]);
#pragma unroll
            for (int j = 1; j < P / 16; ++j) tc::tmem_pin(v[j]);
#pragma unroll
            for (int j = 0; j < P / 16; ++j) {
                float hv[16];
                *reinterpret_cast<uint4*>(out + tc::tile_off(tid, 2 * j, WH)) = pack8<T>(v[j]);
                *reinterpret_cast<uint4*>(out + tc::tile_off(tid, 2 * j + 1, WH)) = pack8<T>(v[j] + 8);
                Pk<T>::unpack(*reinterpret_cast<const uint4*>(sH + tc::tile_off(tid, 2 * j, WH)), hv);
                Pk<T>::unpack(*reinterpret_cast<const uint4*>(sH + tc::tile_off(tid, 2 * j + 1, WH)), hv + 8);
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    dt_part = fmaf(v[j][k], hv[k], dt_part);
                    v[j][k] *= eT;
                }
                tc::tmem_st16(row_addr + j * 16, v[j]);
            }
            tc::tmem_wait_st();
        }
        tc::fence_async_smem();
        tc::fence_before();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after();
            const uint32_t aH = tc::smem_u32(sH);
#pragma unroll
            for (int ks = 0; ks < N / 16; ++ks)
                tc::mma_f16(tm + 64, tc::desc_k(aC, WB, 2 * ks), tc::desc_mn(aH, WH, 16 * ks), idy, ks > 0);
#pragma unroll
            for (int ks = 0; ks < Q / 16; ++ks)
                tc::mma_f16(tm, tc::desc_mn(aC, WB, 16 * ks), tc::desc_mn(aY, WX, 16 * ks), idh, 1u);
            tc::commit(tc::smem_u32(&mbar));
        }
        const float dTc = block_sum(dt_part, s_scan);
        if (tid == 0) a.dT[(b * H + h) * a.nc + c] = exp2_mufu(Tc * kLog2e) * dTc;
        if (!tc::mbar_wait(tc::smem_u32(&mbar), phase)) { report(a, 31); ok = false; }
        phase ^= 1;
        tc::fence_after();
        ok = __syncthreads_and(ok);
        if (ok) {
            // d(loss)/d(cs_l) through the inter-chunk output: <exp(cs_l) dy_l, (C H_c^T)_l>
            const int l = tid;
            float acc = 0.0f;
            float ye4[P / 16][16];
#pragma unroll
            for (int j = 0; j < P / 16; ++j) tc::tmem_ld16(row_addr + 64 + 16 * j, ye4[j]);
            tc::tmem_wait_ld(ye4[0]);
#pragma unroll
            for (int j = 1; j < P / 16; ++j) tc::tmem_pin(ye4[j]);
#pragma unroll
            for (int j = 0; j < P / 16; ++j) {
                float yv[16];
                Pk<T>::unpack(*reinterpret_cast<const uint4*>(sY + tc::tile_off(l, 2 * j, WX)), yv);
                Pk<T>::unpack(*reinterpret_cast<const uint4*>(sY + tc::tile_off(l, 2 * j + 1, WX)), yv + 8);
#pragma unroll
                for (int k = 0; k < 16; ++k) acc = fmaf(yv[k], ye4[j][k], acc);
            }
            a.dcs_inter[(b * H + h) * a.nc * Q + t0 + l] = acc;
        }
        tc::fence_before();
        ok = __syncthreads_and(ok);
    }
    if (tid == 0 && lpend != ~0u) tc::mbar_wait(lb, lpend);   // no copy may land after exit
    if (ok && (a.flags & SSM_HAS_INIT) && a.dinit) {
        for (int j = 0; j < P / 16; ++j) {
            float v[16];
            tc::tmem_ld16(row_addr + j * 16, v);   // all lanes: .sync.aligned
            tc::tmem_wait_ld(v);
#pragma unroll
            for (int k = 0; k < 16; ++k)
                if (nrow && j * 16 + k < pw) a.dinit[state_off<PAD>(a, b, h, j * 16 + k) + tid] = v[k];
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tm, 128);
}

// Sum of 16 values over the 32 lanes of a warp, scattered: afterwards lane
// 2m and 2m+1 both hold the total of value index k(lane) =
// 8 b4 + 4 b3 + 2 b2 + b1 (b_i the bits of the lane).  Select-free halving.
__device__ __forceinline__ float warp_colsum16(float* v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int half = 8, off = 16; half >= 1; half >>= 1, off >>= 1) {
        const bool up = lane & off;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float keep = up ? v[half + i] : v[i];
            const float send = up ? v[i] : v[half + i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// ====================================================================== B2 ==
// One CTA per (b, group, chunk), warp-specialised: eight compute warps -- two
// per TMEM lane quadrant, splitting each row's columns -- and one warp that
// issues every tensor-core instruction.  Threads 0..127 also own one chunk
// position each for the per-position scalar work.
// TMEM: G [0,128), dB [128,256), dC [256,384), scratch S [384,512): dY X^T,
// then Mh^T dY [384,448) and B dH^T [448,512).
//
// Hand-offs (mbarriers, one phase per head):
//   bc   compute -> MMA   B and C tiles are in shared memory (once)
//   in   compute -> MMA   this head's tiles are ready and S is free
//   m1   MMA -> compute   dY X^T (and, for the first head, G) is in TMEM
//   mask compute -> MMA   Mh, dG, exp(cs) dy, w o x written; S read
//   m2   MMA -> compute   the eight GEMMs of the head are done
//   ep   compute -> MMA   the epilogue has read the dy tile
//   lh   copies -> compute  the head's x, dy, H and dH tiles landed
// While the eight GEMMs run, the compute warps fetch the epilogue's global
// inputs and compute the next head's step quantities.  The MMA warp copies
// the next head's x, H and dH tiles in as soon as the GEMMs are done with
// this head's (during the epilogue) and its dy tile once the epilogue has
// read this one, so the copies' latency hides behind the epilogue and the
// per-head scalar tail.
constexpr int kGC = 256;                       // compute threads
constexpr int kGradThreads = kGC + 32;

struct GradSh {
    MaskSh m;
    HeadSh hs;
    float col[4][Q];          // column sums of E per TMEM quadrant
    float rowp[2][Q];         // row sums of E d, per column half
    float vp[2][Q];           // <x_s, Z_s> per column half
    float scan[32];           // [2][16] ping-pong rows of the block reductions
    float T[2];
};

template <typename T, bool PAD>
__global__ void __launch_bounds__(kGradThreads, 1) grads_kernel(const __grid_constant__ Args a) {
    extern __shared__ __align__(128) unsigned char sm_raw[];
    unsigned char* const sm = aligned_smem(sm_raw);
    unsigned char* sB = sm;
    unsigned char* sC = sB + kTileB;
    unsigned char* sM = sC + kTileB;            // Mh
    unsigned char* sG = sM + kTileB;            // dG (masked)
    unsigned char* sX = sG + kTileB;            // x, then exp(cs) dy
    unsigned char* sY = sX + kTileX;            // dy (gated)
    unsigned char* sXW = sY + kTileX;           // w o x
    unsigned char* sH = sXW + kTileX;           // H_c^T
    unsigned char* sD = sH + kTileH;            // dH_{c+1}^T
    __shared__ GradSh sh;
    __shared__ __align__(8) uint64_t bars[7];
    __shared__ uint32_t tbase;
    enum { kBc = 0, kIn = 1, kM1 = 2, kMask = 3, kM2 = 4, kLh = 5, kEp = 6 };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool mma_warp = warp == kGC / 32;
    const int q = warp & 3, hf = (warp >> 2) & 1;      // TMEM quadrant, column half
    const int r = q * 32 + lane;                       // TMEM row / tile row of this thread
    const int64_t c = blockIdx.x, g = blockIdx.y, b = blockIdx.z + a.b0;
    const int64_t L = a.length, H = a.hv, G = a.ngroups;
    const int pw = pw_of<PAD>(a);
    const int64_t na = na_of<PAD>(a);
    const int64_t t0 = c * Q;
    const int valid = (int)min64(Q, L - t0);
    const T* xg = reinterpret_cast<const T*>(a.x);
    const T* zg = reinterpret_cast<const T*>(a.z);
    T* dxg = reinterpret_cast<T*>(a.dx);
    const bool has_z = a.flags & SSM_HAS_Z, has_d = a.flags & SSM_HAS_D;
    const bool d_per_head = a.flags & SSM_D_PER_HEAD;
    const uint32_t bar0 = tc::smem_u32(&bars[0]);
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };

    // parity of a head load still in flight: head 0's (issued by thread 0), the
    // later heads' (issued by lane 0 of the MMA warp)
    uint32_t lpend = ~0u;
    // one thread: the x, H and dH tiles of head hh, with the transaction count
    // of all four tiles, so that the phase also waits for load_y(hh)
    auto load_xhd = [&](int64_t hh) {
        const int64_t h = g * a.hpg + hh;
        const int64_t bhc = (b * H + h) * a.nc + c;
        tc::mbar_expect_tx(bar(kLh), 2 * kRowsX + 2 * kTileH);
        tma_rows<WX>(sX, a.tm_x, c, b, h, bar(kLh), a.status, a.fold);
        tc::bulk_load(tc::smem_u32(sH), a.Ht + (size_t)bhc * kTileH, kTileH, bar(kLh));
        tc::bulk_load(tc::smem_u32(sD), a.dHt + (size_t)bhc * kTileH, kTileH, bar(kLh));
        lpend = (uint32_t)(hh & 1);
    };
    auto load_y = [&](int64_t hh) {
        tma_rows<WX>(sY, a.tm_dy, c, b, g * a.hpg + hh, bar(kLh), a.status, a.fold);
    };

    if (mma_warp) tc::tmem_alloc(tc::smem_u32(&tbase), 512);
    if (tid == 0) {
        tc::mbar_init(bar(kBc), 1);
        tc::mbar_init(bar(kIn), kGC);
        tc::mbar_init(bar(kM1), 1);
        tc::mbar_init(bar(kMask), kGC);
        tc::mbar_init(bar(kM2), 1);
        tc::mbar_init(bar(kLh), 1);
        tc::mbar_init(bar(kEp), kGC);
        tc::fence_mbar_init();
        tc::mbar_expect_tx(bar(kBc), 2 * kRowsB);      // the MMA warp waits for these directly
        tma_rows<WB>(sC, a.tm_C, c, b, g, bar(kBc), a.status, a.fold);
        tma_rows<WB>(sB, a.tm_B, c, b, g, bar(kBc), a.status, a.fold);
        load_xhd(0);
        load_y(0);
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tm = tbase;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t tG = tm, tdB = tm + 128, tdC = tm + 256, tS = tm + 384;
    const uint32_t aB = tc::smem_u32(sB), aC = tc::smem_u32(sC), aM = tc::smem_u32(sM), aG = tc::smem_u32(sG);
    const uint32_t aX = tc::smem_u32(sX), aY = tc::smem_u32(sY), aXW = tc::smem_u32(sXW);
    const uint32_t aH = tc::smem_u32(sH), aD = tc::smem_u32(sD);
    constexpr uint32_t fmt = Pk<T>::kFmt;
    bool ok = true;

    if (mma_warp) {
        // ------------------------------------------------------- MMA warp --
        // lane 0 polls, the warp follows its outcome (uniform control flow)
        auto wait_warp = [&](int i, uint32_t par) {
            bool w = true;
            if (lane == 0) w = tc::mbar_wait(bar(i), par);
            return __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
        };
        ok = wait_warp(kBc, 0);
        tc::fence_after();
        if (ok && lane == 0) {
            const uint32_t idg = tc::idesc_f16(fmt, 128, 128, false, false);
#pragma unroll
            for (int ks = 0; ks < N / 16; ++ks)
                tc::mma_f16(tG, tc::desc_k(aC, WB, 2 * ks), tc::desc_k(aB, WB, 2 * ks), idg, ks > 0);
        }
        __syncwarp();
        for (int64_t hh = 0; hh < a.hpg && ok; ++hh) {
            const uint32_t par = (uint32_t)(hh & 1);
            if (!wait_warp(kIn, par)) { ok = false; break; }
            tc::fence_after();
            if (lane == 0) {
                const uint32_t idm = tc::idesc_f16(fmt, 128, 128, false, false);
#pragma unroll
                for (int ks = 0; ks < P / 16; ++ks)
                    tc::mma_f16(tS, tc::desc_k(aY, WX, 2 * ks), tc::desc_k(aX, WX, 2 * ks), idm, ks > 0);
                tc::commit(bar(kM1));
            }
            __syncwarp();
            if (!wait_warp(kMask, par)) { ok = false; break; }
            tc::fence_after();
            if (lane == 0) {
                const uint32_t i_mn_mn64 = tc::idesc_f16(fmt, 128, P, true, true);
                const uint32_t i_k_mn64 = tc::idesc_f16(fmt, 128, P, false, true);
                const uint32_t i_k_mn = tc::idesc_f16(fmt, 128, 128, false, true);
                const uint32_t i_k_k = tc::idesc_f16(fmt, 128, 128, false, false);
                const uint32_t i_mn_mn = tc::idesc_f16(fmt, 128, 128, true, true);
                const uint32_t first = hh == 0 ? 0u : 1u;
#pragma unroll
                for (int ks = 0; ks < Q / 16; ++ks)   // Mh^T dY
                    tc::mma_f16(tS, tc::desc_mn(aM, WB, 16 * ks), tc::desc_mn(aY, WX, 16 * ks), i_mn_mn64, ks > 0);
#pragma unroll
                for (int ks = 0; ks < N / 16; ++ks)   // B dH^T
                    tc::mma_f16(tS + 64, tc::desc_k(aB, WB, 2 * ks), tc::desc_mn(aD, WH, 16 * ks), i_k_mn64, ks > 0);
#pragma unroll
                for (int ks = 0; ks < Q / 16; ++ks)   // dC += dG B
                    tc::mma_f16(tdC, tc::desc_k(aG, WB, 2 * ks), tc::desc_mn(aB, WB, 16 * ks), i_k_mn, ks > 0 ? 1u : first);
#pragma unroll
                for (int ks = 0; ks < P / 16; ++ks)   // dC += (exp(cs) dy) H
                    tc::mma_f16(tdC, tc::desc_k(aX, WX, 2 * ks), tc::desc_k(aH, WH, 2 * ks), i_k_k, 1u);
#pragma unroll
                for (int ks = 0; ks < Q / 16; ++ks)   // dB += dG^T C
                    tc::mma_f16(tdB, tc::desc_mn(aG, WB, 16 * ks), tc::desc_mn(aC, WB, 16 * ks), i_mn_mn, ks > 0 ? 1u : first);
#pragma unroll
                for (int ks = 0; ks < P / 16; ++ks)   // dB += (w o x) dH
                    tc::mma_f16(tdB, tc::desc_k(aXW, WX, 2 * ks), tc::desc_k(aD, WH, 2 * ks), i_k_k, 1u);
                tc::commit(bar(kM2));
            }
            __syncwarp();
            if (hh + 1 < a.hpg) {
                // the next head's tiles: x, H and dH once the GEMMs are done with
                // this head's, dy once the epilogue has read this one
                if (!wait_warp(kM2, par)) { ok = false; break; }
                if (lane == 0) load_xhd(hh + 1);
                __syncwarp();
                const bool ep = wait_warp(kEp, par);
                if (lane == 0) load_y(hh + 1);   // also when the wait gave up: the phase must complete
                __syncwarp();
                if (!ep) { ok = false; break; }
            }
        }
        if (!ok && lane == 0) report(a, 44);
        if (lane == 0 && lpend != ~0u) tc::mbar_wait(bar(kLh), lpend);   // no copy may land after exit
    } else {
        // --------------------------------------------------- compute warps --
        const bool pos_thread = tid < Q;           // owns chunk position s = tid
        stage_heads<kGC>(a, sh.hs, b, g, c, 0, (int)min64(kHeadsSh, a.hpg));
        gsync<kGC>();
        int kpp = 0;                               // ping-pong row of the next block reduction
        Steps st = staged_steps_pp<kGC>(a, sh.hs, 0, c, sh.scan, kpp);
        if (tid == Q - 1) sh.T[0] = st.cs;
        mask_factors<kGC>(sh.m, st);
        const int j0 = hf * (WX / 2);              // this thread's half of an X-like row (chunks)
        float ddt_acc = 0.0f;
        (void)ddt_acc;
        for (int64_t hh = 0; hh < a.hpg; ++hh) {
            const uint32_t par = (uint32_t)(hh & 1);
            const int64_t h = g * a.hpg + hh;
            const int64_t bhc = (b * H + h) * a.nc + c;
            const int hk = (int)(hh % kHeadsSh);
            const float Ah = sh.hs.A[hk];
            const float Dh = sh.hs.D[hk];
            const float Tc = sh.T[hh & 1];
            const int64_t grow = row_off<PAD>(a, b, t0 + r, h);     // row r of dx / z
            const int64_t xrow = (b * L + t0 + r) * a.xts + h * pw;  // row r of x
            {
                const bool lw = tc::mbar_wait(bar(kLh), par);   // this head's tiles
                if (!lw) report(a, 45);
                else if (tid == 0) lpend = ~0u;
                ok = cg_all<kGC>(lw);
                if (!ok) break;
            }
            if (has_z && r < valid) {               // gate dy in place, own row half
                for (int j = j0; j < j0 + WX / 2 && 8 * j < pw; ++j) {
                    float f[8], zv[8];
                    Pk<T>::unpack(*reinterpret_cast<const uint4*>(sY + tc::tile_off(r, j, WX)), f);
                    Pk<T>::unpack(*reinterpret_cast<const uint4*>(zg + grow + 8 * j), zv);
#pragma unroll
                    for (int k = 0; k < 8; ++k) f[k] *= zv[k] * sigmoid_f(zv[k]);
                    *reinterpret_cast<uint4*>(sY + tc::tile_off(r, j, WX)) = pack8<T>(f);
                }
            }
            tc::fence_async_smem();
            tc::mbar_arrive(bar(kIn));
            if (has_z) gsync<kGC>();                // every gated row is in place before it is read
            // while dY X^T runs: w o x, and the D gradient partial <dy, x>
            float dD_head = 0.0f;
            {
                const float w = exp2_mufu(Tc * kLog2e - sh.m.cs2[r]) * sh.m.d[r];   // exp(T - cs_r) d_r
                for (int j = j0; j < j0 + WX / 2; ++j) {
                    float xv[8], yv[8];
                    Pk<T>::unpack(*reinterpret_cast<const uint4*>(sX + tc::tile_off(r, j, WX)), xv);
                    Pk<T>::unpack(*reinterpret_cast<const uint4*>(sY + tc::tile_off(r, j, WX)), yv);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        dD_head = fmaf(xv[k], yv[k], dD_head);
                        xv[k] *= w;
                    }
                    *reinterpret_cast<uint4*>(sXW + tc::tile_off(r, j, WX)) = pack8<T>(xv);
                }
            }
            if (has_d && d_per_head && tid < P) {
                const int p = tid;
                float s2 = 0.0f;
                for (int rr = 0; rr < Q; ++rr) {
                    const uint32_t off = tc::tile_off(rr, p >> 3, WX) + (p & 7) * 2;
                    s2 = fmaf(ldf(reinterpret_cast<const T*>(sX + off)), ldf(reinterpret_cast<const T*>(sY + off)), s2);
                }
                a.dD_part[bhc * P + p] = s2;
            }
            if (!tc::mbar_wait(bar(kM1), par)) { report(a, 42); ok = false; }
            tc::fence_after();
            ok = cg_all<kGC>(ok);                    // also: every thread is done reading sX
            if (!ok) break;
            // mask pass, row l = r: blocks of parity hf, up to the last one a row of this quadrant reaches
            {
                const int l = r;
                const float csl = sh.m.cs2[l];
                const int nj = min(Q / 16, 2 * q + 2);
                float rowsum = 0.0f;
                for (int j = hf; j < Q / 16; j += 2) {
                    uint4 m0 = make_uint4(0, 0, 0, 0), m1 = m0, g0 = m0, g1 = m0;
                    if (j < nj) {                              // warp-uniform
                        float gv[16], dm[16], E[16];
                        tc::tmem_ld16(tG + lane_off + 16 * j, gv);
                        tc::tmem_ld16(tS + lane_off + 16 * j, dm);
                        tc::tmem_wait_ld(gv);
                        tc::tmem_pin(dm);
                        float e[16];
                        if (16 * j + 15 < l) {
                            const float2 rf = f2(exp2_mufu(csl - sh.m.cs2[16 * j + 15]));
#pragma unroll
                            for (int k = 0; k < 16; k += 2) {
                                const float2 v = mul2(rf, *reinterpret_cast<const float2*>(&sh.m.cf[16 * j + k]));
                                e[k] = v.x;
                                e[k + 1] = v.y;
                            }
                        } else {
#pragma unroll
                            for (int k = 0; k < 16; ++k) {
                                const int s = 16 * j + k;
                                e[k] = s <= l ? exp2_mufu(csl - sh.m.cs2[s]) : 0.0f;
                            }
                        }
                        // the products in pairs (packed fp32, each rounded as alone)
                        float mh[16], dg[16];
#pragma unroll
                        for (int k = 0; k < 16; k += 2) {
                            const float2 e2 = make_float2(e[k], e[k + 1]);
                            const float2 g2 = make_float2(gv[k], gv[k + 1]);
                            const float2 m2 = make_float2(dm[k], dm[k + 1]);
                            const float2 ed = mul2(e2, *reinterpret_cast<const float2*>(&sh.m.d[16 * j + k]));
                            const float2 gd = mul2(g2, m2);
                            const float2 mv = mul2(g2, ed), dv = mul2(m2, ed), ev = mul2(gd, e2);
                            mh[k] = mv.x; mh[k + 1] = mv.y;
                            dg[k] = dv.x; dg[k + 1] = dv.y;
                            E[k] = ev.x; E[k + 1] = ev.y;
                            rowsum = fmaf(gd.x, ed.x, rowsum);
                            rowsum = fmaf(gd.y, ed.y, rowsum);
                        }
                        m0 = pack8<T>(mh); m1 = pack8<T>(mh + 8);
                        g0 = pack8<T>(dg); g1 = pack8<T>(dg + 8);
                        const float cs_sum = warp_colsum16(E);
                        if (!(lane & 1)) {
                            const int k = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 +
                                          ((lane >> 1) & 1);
                            sh.col[q][16 * j + k] = cs_sum;
                        }
                    } else if (lane < 16) {
                        sh.col[q][16 * j + lane] = 0.0f;
                    }
                    *reinterpret_cast<uint4*>(sM + tc::tile_off(l, 2 * j, WB)) = m0;
                    *reinterpret_cast<uint4*>(sM + tc::tile_off(l, 2 * j + 1, WB)) = m1;
                    *reinterpret_cast<uint4*>(sG + tc::tile_off(l, 2 * j, WB)) = g0;
                    *reinterpret_cast<uint4*>(sG + tc::tile_off(l, 2 * j + 1, WB)) = g1;
                }
                sh.rowp[hf][l] = rowsum;
                // exp(cs_l) dy_l into sX (row l, this thread's half)
                const float el = exp2_mufu(csl);
                for (int j = j0; j < j0 + WX / 2; ++j) {
                    float f[8];
                    Pk<T>::unpack(*reinterpret_cast<const uint4*>(sY + tc::tile_off(l, j, WX)), f);
#pragma unroll
                    for (int k = 0; k < 8; ++k) f[k] *= el;
                    *reinterpret_cast<uint4*>(sX + tc::tile_off(l, j, WX)) = pack8<T>(f);
                }
            }
            tc::fence_async_smem();
            tc::fence_before();
            tc::mbar_arrive(bar(kMask));
            // ---- while the eight GEMMs run ----
            uint4 xr[WX / 2];
            {
                const bool live = r < valid;
#pragma unroll
                for (int j = 0; j < WX / 2; ++j)
                    xr[j] = live && 8 * (j0 + j) < pw ? *reinterpret_cast<const uint4*>(xg + xrow + 8 * (j0 + j))
                                                      : make_uint4(0, 0, 0, 0);
            }
            const float dci = pos_thread ? a.dcs_inter[bhc * Q + tid] : 0.0f;
            const float dTc = tid == Q - 1 ? a.dT[bhc] : 0.0f;
            gsync<kGC>();                            // sh.col, sh.rowp complete
            float colsum = 0.0f, rowsum = 0.0f;
            if (pos_thread) {
#pragma unroll
                for (int w = 0; w < 4; ++w) colsum += sh.col[w][tid];
                rowsum = sh.rowp[0][tid] + sh.rowp[1][tid];
            }
            const float dD_sum = pp_sum<kGC>(dD_head, sh.scan, kpp);
            Steps st_next = st;
            if (hh + 1 < a.hpg) {
                const int hk1 = (int)((hh + 1) % kHeadsSh);
                if (hk1 == 0) {
                    stage_heads<kGC>(a, sh.hs, b, g, c, hh + 1, (int)min64(kHeadsSh, a.hpg - hh - 1));
                    gsync<kGC>();
                }
                st_next = staged_steps_pp<kGC>(a, sh.hs, hk1, c, sh.scan, kpp);
                if (tid == Q - 1) sh.T[(hh + 1) & 1] = st_next.cs;
            }
            if (!tc::mbar_wait(bar(kM2), par)) { report(a, 43); ok = false; }
            tc::fence_after();
            ok = cg_all<kGC>(ok);
            if (!ok) break;
            // epilogue, row s = r, columns [32 hf, 32 hf + 32): the TMEM part first
            {
                const int s = r;
                const float d_s = sh.m.d[s];
                const float eTs = exp2_mufu(Tc * kLog2e - sh.m.cs2[s]);
                float vpart = 0.0f;
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    const int col = 32 * hf + 16 * jj;
                    float di[16], zz[16], xv[16], yv[16];
                    tc::tmem_ld16(tS + lane_off + col, di);
                    tc::tmem_ld16(tS + lane_off + 64 + col, zz);
                    tc::tmem_wait_ld(di);
                    tc::tmem_pin(zz);
                    Pk<T>::unpack(xr[2 * jj], xv);
                    Pk<T>::unpack(xr[2 * jj + 1], xv + 8);
                    Pk<T>::unpack(*reinterpret_cast<const uint4*>(sY + tc::tile_off(s, col / 8, WX)), yv);
                    Pk<T>::unpack(*reinterpret_cast<const uint4*>(sY + tc::tile_off(s, col / 8 + 1, WX)), yv + 8);
                    float dxv[16];
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        vpart = fmaf(xv[k], zz[k], vpart);
                        const float Dk = has_d ? (d_per_head ? (col + k < pw ? a.D[h * pw + col + k] : 0.0f) : Dh) : 0.0f;
                        dxv[k] = fmaf(d_s * eTs, zz[k], di[k]) + Dk * yv[k];   // Mh already carries d_s
                    }
                    if (s < valid) {
                        if (col < pw) *reinterpret_cast<uint4*>(dxg + grow + col) = pack8<T>(dxv);
                        if (col + 8 < pw) *reinterpret_cast<uint4*>(dxg + grow + col + 8) = pack8<T>(dxv + 8);
                    }
                }
                sh.vp[hf][s] = vpart * eTs;
            }
            tc::mbar_arrive(bar(kEp));               // this thread is done with the dy tile
            tc::fence_before();                      // S read: the next head's dY X^T may overwrite it
            gsync<kGC>();                            // sh.vp complete
            if (hh + 1 < a.hpg) mask_factors<kGC>(sh.m, st_next);   // the scalars below use st, not sh.m
            float dcs = 0.0f, dd_direct = 0.0f, dv = 0.0f;
            if (pos_thread) {
                const float v_s = sh.vp[0][tid] + sh.vp[1][tid];
                dv = st.d * v_s;
                dcs = rowsum - st.d * colsum - dv + dci;
                dd_direct = colsum + v_s;
            }
            // d/dT_c = exp(T) <dH_{c+1}, H_c> + sum_s d_s v_s, added at the chunk's last position
            const float dv_sum = pp_sum<kGC>(dv, sh.scan, kpp);
            if (tid == Q - 1) dcs += dTc + dv_sum;
            const float suffix = pp_suffix_scan<kGC>(dcs, sh.scan, kpp);
            const float dd = fmaf(Ah, suffix, dd_direct);
            const float ddt = (a.flags & SSM_SOFTPLUS) ? dd * softplus_grad_f(st.raw) : dd;
            if constexpr (PAD) {
                // a head's virtual heads are consecutive here: their d dt parts add up
                const int64_t vk = h & (a.pr - 1);
                ddt_acc = vk == 0 ? ddt : ddt_acc + ddt;
                if (vk == a.pr - 1 && pos_thread && tid < valid)
                    a.ddt[(b * L + t0 + tid) * a.nheads + (h >> a.prs)] = ddt_acc;
            } else if (pos_thread && tid < valid) {
                a.ddt[(b * L + t0 + tid) * a.nheads + h] = ddt;
            }
            const float2 ab = pp_sum2<kGC>(make_float2(pos_thread ? dcs * st.cd : 0.0f,
                                                       pos_thread && tid < valid ? ddt : 0.0f), sh.scan, kpp);
            const float dA_sum = ab.x, db_sum = ab.y;
            if (tid == 0) {
                a.dA_part[bhc] = dA_sum;
                a.db_part[bhc] = db_sum;
                if (has_d && !d_per_head) a.dD_part[bhc] = dD_sum;
            }
            st = st_next;
        }
        if (ok) {
            // dC rows l, dB rows s (fp32, valid rows only), this thread's column half
            const bool live = r < valid;
            float* dCr = a.dC + ((b * L + t0 + (live ? r : 0)) * G + g) * na;
            float* dBr = a.dB + ((b * L + t0 + (live ? r : 0)) * G + g) * na;
            for (int jj = 0; jj < N / 32; ++jj) {
                const int col = 64 * hf + 16 * jj;
                float vc[16], vb[16];
                tc::tmem_ld16(tdC + lane_off + col, vc);   // all lanes: .sync.aligned
                tc::tmem_ld16(tdB + lane_off + col, vb);
                tc::tmem_wait_ld(vb);
                tc::tmem_pin(vc);
                if (live) {
#pragma unroll
                    for (int k = 0; k < 16; k += 4) {
                        if (col + k >= na) break;     // dstate is a multiple of 8
                        *reinterpret_cast<float4*>(dCr + col + k) = make_float4(vc[k], vc[k + 1], vc[k + 2], vc[k + 3]);
                        *reinterpret_cast<float4*>(dBr + col + k) = make_float4(vb[k], vb[k + 1], vb[k + 2], vb[k + 3]);
                    }
                }
            }
        }
        if (tid == 0) {                        // no copy may land after exit
            if (lpend != ~0u) tc::mbar_wait(bar(kLh), lpend);
            tc::mbar_wait(bar(kBc), 0);
        }
    }
    tc::fence_before();
    __syncthreads();
    if (mma_warp) tc::tmem_dealloc(tm, 512);
}

// dA, d dt_bias, dD over (batch, chunk, the head's virtual heads), fixed order.
__global__ void reduce_kernel(const Args a, float* dA, float* dbias, float* dD) {
    const int64_t H = a.nheads, HV = a.hv, pr = a.pr;
    const bool has_d = a.flags & SSM_HAS_D, d_per_head = a.flags & SSM_D_PER_HEAD;
    const int64_t nd = has_d ? (d_per_head ? H * a.pa : H) : 0;
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= 2 * H + nd) return;
    float s = 0.0f;
    if (i < 2 * H) {
        const int64_t h = i % H;
        const float* src = i < H ? a.dA_part : a.db_part;
        for (int64_t b = 0; b < a.batch; ++b)
            for (int64_t k = 0; k < pr; ++k)
                for (int64_t c = 0; c < a.nc; ++c) s += src[(b * HV + h * pr + k) * a.nc + c];
        if (i < H) dA[h] = s;
        else if (dbias) dbias[h] = s;
    } else {
        const int64_t k = i - 2 * H;
        if (d_per_head) {
            const int64_t h = k / a.pa, pc = k % a.pa;
            const int64_t v = h * pr + pc / a.pw, p = pc % a.pw;   // virtual head, its column
            for (int64_t b = 0; b < a.batch; ++b)
                for (int64_t c = 0; c < a.nc; ++c) s += a.dD_part[((b * HV + v) * a.nc + c) * P + p];
        } else {
            for (int64_t b = 0; b < a.batch; ++b)
                for (int64_t kk = 0; kk < pr; ++kk)
                    for (int64_t c = 0; c < a.nc; ++c) s += a.dD_part[(b * HV + k * pr + kk) * a.nc + c];
        }
        dD[k] = s;
    }
}

// ------------------------------------------------------------------ host ----
constexpr size_t kSmemOutputs = 2 * kTileB + kTileX + kTileH;
constexpr size_t kSmemDstates = kTileB + 2 * kTileH;
constexpr size_t kSmemGrads = 4 * kTileB + 3 * kTileX + 2 * kTileH;

// bf16 / f16 with a headdim that is a multiple of 8 up to 64, or 128 or 256
// (two or four virtual heads), and a dstate that is a multiple of 8 up to 128.
bool eligible(const ssm_chunk_scan_params* p) {
    const int64_t pa = p->headdim, na = p->dstate;
    const bool pd = (pa >= 8 && pa <= P && pa % 8 == 0) || pa == 2 * P || pa == 4 * P;
    return (p->dtype == SSM_BF16 || p->dtype == SSM_F16) && pd && na >= 8 && na <= N && na % 8 == 0 &&
           !(p->flags & SSM_CUDA_CORES);
}
static int64_t virt_per_head(const ssm_chunk_scan_params* p) { return p->headdim > P ? p->headdim / P : 1; }

static int64_t n_chunks(const ssm_chunk_scan_params* p) { return ceil_div(p->length, (int64_t)Q); }

struct Saved { size_t ht, yp, total; };
static Saved saved_layout(const ssm_chunk_scan_params* p) {
    Saved s;
    const int64_t BH = p->batch * p->nheads * virt_per_head(p);
    s.ht = align_up((size_t)(BH * n_chunks(p)) * kTileH, 256);
    s.yp = (p->flags & SSM_HAS_Z) ? align_up((size_t)(BH * p->length * P) * 2, 256) : 0;
    s.total = s.ht + s.yp;
    return s;
}
struct Ws { size_t dh, dci, dt, part, dd, total; };
static Ws ws_layout(const ssm_chunk_scan_params* p) {
    Ws w;
    const int64_t BH = p->batch * p->nheads * virt_per_head(p), nc = n_chunks(p);
    w.dh = align_up((size_t)(BH * nc) * kTileH, 256);
    w.dci = align_up((size_t)(BH * nc * Q) * 4, 256);
    w.dt = align_up((size_t)(BH * nc) * 4, 256);
    w.part = w.dt;
    w.dd = align_up((size_t)(BH * nc * P) * 4, 256);
    w.total = w.dh + w.dci + w.dt + 2 * w.part + w.dd;
    return w;
}

void sizes(const ssm_chunk_scan_params* p, size_t* saved_bytes, size_t* workspace_bytes) {
    if (saved_bytes) *saved_bytes = saved_layout(p).total;
    if (workspace_bytes) *workspace_bytes = ws_layout(p).total;
}

static void make_args(const ssm_chunk_scan_params* p, Args& a) {
    a.batch = p->batch; a.length = p->length; a.nheads = p->nheads; a.ngroups = p->ngroups;
    a.nc = n_chunks(p); a.b0 = 0;
    a.pr = virt_per_head(p); a.prs = a.pr == 4 ? 2 : a.pr == 2 ? 1 : 0;
    a.hv = p->nheads * a.pr; a.hpg = p->nheads / p->ngroups * a.pr;
    a.pa = p->headdim; a.pw = min64(p->headdim, P); a.na = p->dstate;
    a.flags = p->flags; a.dt_dtype = p->dt_dtype;
    a.xts = p->x_token_stride ? p->x_token_stride : p->nheads * p->headdim;
    a.fold = (p->headdim == P && p->dstate == N && p->length % 8 == 0) ? 1 : 0;
    a.x = p->x; a.dt = p->dt; a.A = p->A; a.B = p->B; a.C = p->C; a.D = p->D; a.z = p->z;
    a.dt_bias = p->dt_bias; a.init = p->initial_states;
    a.y = p->y; a.final_state = p->final_state;
    a.status = p->status;
    const Saved s = saved_layout(p);
    unsigned char* sv = reinterpret_cast<unsigned char*>(p->saved);
    a.Ht = sv;
    a.ypre = (sv && s.yp) ? sv + s.ht : nullptr;
    a.dy = p->dy; a.dfinal = p->dfinal; a.dx = p->dx; a.ddt = p->ddt; a.dB = p->dB; a.dC = p->dC;
    a.dz = p->dz; a.dinit = p->dinitial;
    a.dHt = nullptr; a.dcs_inter = a.dT = a.dA_part = a.db_part = a.dD_part = nullptr;
}

static bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime.
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// Tensor map over the rows of a (batch, length, heads, width) bf16/f16 tensor
// (x, dy: heads = virtual heads, width = their data columns; B, C: heads =
// ngroups, width = dstate) as the 5-D view (8 elements, row in the batch,
// 16-byte chunk, batch, head): a box of (8, 8, tile_width / 8, 1, 1) is one
// 8-row group of core matrices of a tile (tile_off layout); rows past
// `length` and chunks past `width` read as zeros.
//
// `fold` (width == tile_width and length a multiple of 8) splits the row into
// (row mod 8, row group) and merges the heads into the chunk axis instead:
// (8 elements, row mod 8, 16-byte chunk of the whole row, row group, batch),
// so one box of (8, 8, tile_width / 8, Q / 8, 1) lands a whole tile in the
// same layout.  Row groups past length / 8 read as zeros.
static int encode_rows(CUtensorMap* m, const void* base, int dtype, int64_t batch, int64_t length, int64_t heads,
                       int64_t width, int64_t tile_width, int64_t token_stride, bool fold) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(SSM_ERR_CUDA, "chunk_scan (tensor cores): cuTensorMapEncodeTiled unavailable");
    if (int s = ensure_context("chunk_scan (tensor cores)")) return s;
    const cuuint64_t es = 2;
    const int64_t ts = token_stride ? token_stride : heads * width;   // elements between tokens
    cuuint64_t dim[5] = {8, (cuuint64_t)length, (cuuint64_t)(width / 8), (cuuint64_t)batch, (cuuint64_t)heads};
    cuuint64_t str[4] = {(cuuint64_t)ts * es, 16, (cuuint64_t)(length * ts) * es, (cuuint64_t)width * es};
    cuuint32_t box[5] = {8, 8, (cuuint32_t)(tile_width / 8), 1, 1};
    if (fold) {
        if (width != tile_width || length % 8)
            return fail(SSM_ERR_INVALID, "chunk_scan (tensor cores): whole-tile map for a ragged shape");
        const cuuint64_t fdim[5] = {8, 8, (cuuint64_t)(heads * width / 8), (cuuint64_t)(length / 8), (cuuint64_t)batch};
        const cuuint64_t fstr[4] = {(cuuint64_t)ts * es, 16, (cuuint64_t)(8 * ts) * es, (cuuint64_t)(length * ts) * es};
        const cuuint32_t fbox[5] = {8, 8, (cuuint32_t)(tile_width / 8), (cuuint32_t)(Q / 8), 1};
        for (int i = 0; i < 5; ++i) { dim[i] = fdim[i]; box[i] = fbox[i]; }
        for (int i = 0; i < 4; ++i) str[i] = fstr[i];
    }
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUresult r = enc(m, dtype == SSM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                           const_cast<void*>(base), dim, str, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(SSM_ERR_CUDA, "chunk_scan (tensor cores): cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return SSM_OK;
}

static int set_smem(const void* fn, size_t bytes) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
        return check_launch("chunk_scan (tensor cores): smem attribute");
    return SSM_OK;
}

// One batch-row range [a.b0, a.b0 + rows) of the forward: the state pass, then
// the outputs of the same rows.
template <typename T, bool PAD>
static int run_fwd_rows(const Args& a, int64_t rows, cudaStream_t s) {
    states2_kernel<T, PAD><<<dim3((unsigned)a.hv, (unsigned)rows), kStThreads, kSmemStates2 + kSmemPad, s>>>(a);
    if (int e = check_launch("chunk_scan fwd (tensor cores): states")) return e;
    outputs_kernel<T, PAD><<<dim3((unsigned)a.nc, (unsigned)a.ngroups, (unsigned)rows), kOutThreads, kSmemOutputs + kSmemPad, s>>>(a);
    return check_launch("chunk_scan fwd (tensor cores): outputs");
}
// ... and of the backward (the parameter reduce runs once, over every row).
template <typename T, bool PAD>
static int run_bwd_rows(const Args& a, int64_t rows, cudaStream_t s) {
    if (a.flags & SSM_HAS_Z)
        dstates_kernel<T, true, PAD><<<dim3((unsigned)a.hv, (unsigned)rows), kThreads, kSmemDstates + kSmemPad, s>>>(a);
    else
        dstates_kernel<T, false, PAD><<<dim3((unsigned)a.hv, (unsigned)rows), kThreads, kSmemDstates + kSmemPad, s>>>(a);
    if (int e = check_launch("chunk_scan bwd (tensor cores): dstates")) return e;
    grads_kernel<T, PAD><<<dim3((unsigned)a.nc, (unsigned)a.ngroups, (unsigned)rows), kGradThreads, kSmemGrads + kSmemPad, s>>>(a);
    return check_launch("chunk_scan bwd (tensor cores): grads");
}

static int64_t sm_count_tc() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = 148;
    }
    return n;
}

// Up to kParts - 1 more non-blocking streams per device (created on first use,
// kept for the process), on which the later parts of the batch run.  Two parts
// at config 3: 5.42 -> 5.09 ms per fwd+bwd step; four and eight measured the
// same as two.
constexpr int kParts = 2;
static cudaStream_t side_stream(int i) {
    static std::mutex mu;
    static cudaStream_t streams[64][kParts] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!streams[dev][i] && cudaStreamCreateWithFlags(&streams[dev][i], cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        streams[dev][i] = nullptr;
    }
    return streams[dev][i];
}

// Runs `rows_fn(args, rows, stream)` over the whole batch.  The state kernels
// run one CTA per (batch row, head) through every chunk; when that grid needs
// more than one wave, the batch goes in up to kParts parts -- the first on the
// caller's stream, the others on side streams, forked from and joined back
// into the caller's stream by events -- so that the last, partly filled wave
// of one part's state kernel overlaps the other parts' kernels instead of
// leaving SMs idle.  Not while the caller's stream is being captured.
template <class F>
static int in_halves(const Args& a, cudaStream_t s, F&& rows_fn) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    const int parts = (int)min64(kParts, a.batch);
    if (parts < 2 || a.hv * a.batch <= 2 * sm_count_tc() ||
        cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return rows_fn(a, a.batch, s);
    }
    cudaStream_t st[kParts] = {s};
    cudaEvent_t fork = nullptr, join[kParts] = {};
    bool ok = cudaEventCreateWithFlags(&fork, cudaEventDisableTiming) == cudaSuccess;
    for (int i = 1; i < parts && ok; ++i) {
        st[i] = side_stream(i);
        ok = st[i] != nullptr && cudaEventCreateWithFlags(&join[i], cudaEventDisableTiming) == cudaSuccess;
    }
    if (!ok) {
        if (fork) cudaEventDestroy(fork);
        for (int i = 1; i < parts; ++i)
            if (join[i]) cudaEventDestroy(join[i]);
        cudaGetLastError();
        return rows_fn(a, a.batch, s);
    }
    int e = SSM_OK;
    if (cudaEventRecord(fork, s) != cudaSuccess) e = check_launch("chunk_scan (tensor cores): stream fork");
    for (int i = 1; i < parts && !e; ++i)
        if (cudaStreamWaitEvent(st[i], fork, 0) != cudaSuccess) e = check_launch("chunk_scan (tensor cores): stream fork");
    int64_t r0 = 0;
    for (int i = 0; i < parts && !e; ++i) {
        const int64_t r1 = a.batch * (i + 1) / parts;
        Args part = a;
        part.b0 = a.b0 + r0;
        e = rows_fn(part, r1 - r0, st[i]);
        r0 = r1;
    }
    // joined in every case, so that nothing later on the caller's stream runs ahead
    for (int i = 1; i < parts; ++i)
        if ((cudaEventRecord(join[i], st[i]) != cudaSuccess || cudaStreamWaitEvent(s, join[i], 0) != cudaSuccess) && !e)
            e = check_launch("chunk_scan (tensor cores): stream join");
    cudaEventDestroy(fork);
    for (int i = 1; i < parts; ++i) cudaEventDestroy(join[i]);
    return e;
}

template <typename T, bool PAD>
static int run_fwd(const Args& a, cudaStream_t s) {
    if (int e = set_smem((const void*)states2_kernel<T, PAD>, kSmemStates2 + kSmemPad)) return e;
    if (int e = set_smem((const void*)outputs_kernel<T, PAD>, kSmemOutputs + kSmemPad)) return e;
    return in_halves(a, s, [](const Args& r, int64_t rows, cudaStream_t st) { return run_fwd_rows<T, PAD>(r, rows, st); });
}

template <typename T, bool PAD>
static int run_bwd(const Args& a, const ssm_chunk_scan_params* p, cudaStream_t s) {
    if (int e = set_smem((const void*)dstates_kernel<T, false, PAD>, kSmemDstates + kSmemPad)) return e;
    if (int e = set_smem((const void*)dstates_kernel<T, true, PAD>, kSmemDstates + kSmemPad)) return e;
    if (int e = set_smem((const void*)grads_kernel<T, PAD>, kSmemGrads + kSmemPad)) return e;
    if (int e = in_halves(a, s, [](const Args& r, int64_t rows, cudaStream_t st) { return run_bwd_rows<T, PAD>(r, rows, st); }))
        return e;
    const bool has_d = p->flags & SSM_HAS_D, d_per_head = p->flags & SSM_D_PER_HEAD;
    const int64_t total = 2 * p->nheads + (has_d ? (d_per_head ? p->nheads * p->headdim : p->nheads) : 0);
    reduce_kernel<<<(unsigned)ceil_div(total, (int64_t)128), 128, 0, s>>>(
        a, p->dA, (p->flags & SSM_HAS_BIAS) ? p->ddt_bias : nullptr, has_d ? p->dD : nullptr);
    return check_launch("chunk_scan bwd (tensor cores): reduce");
}

// The tile shape itself (headdim 64, dstate 128) runs kernels with that shape
// compiled in; every other eligible shape the padded / virtual-head ones.
static bool padded(const Args& a) { return !(a.pa == P && a.na == N); }
template <typename T>
static int run_fwd_any(const Args& a, cudaStream_t s) {
    return padded(a) ? run_fwd<T, true>(a, s) : run_fwd<T, false>(a, s);
}
template <typename T>
static int run_bwd_any(const Args& a, const ssm_chunk_scan_params* p, cudaStream_t s) {
    return padded(a) ? run_bwd<T, true>(a, p, s) : run_bwd<T, false>(a, p, s);
}

int fwd(const ssm_chunk_scan_params* p, cudaStream_t s) {
    if (!p->saved) return fail(SSM_ERR_INVALID, "chunk_scan fwd (tensor cores): null saved buffer");
    if (!aligned16(p->x) || !aligned16(p->B) || !aligned16(p->C) || !aligned16(p->y) ||
        ((p->flags & SSM_HAS_Z) && !aligned16(p->z)) || !aligned16(p->saved))
        return fail(SSM_ERR_INVALID, "chunk_scan fwd (tensor cores): x, B, C, z, y and saved must be 16-byte aligned");
    Args a;
    make_args(p, a);
    if (int e = encode_rows(&a.tm_x, p->x, p->dtype, p->batch, p->length, a.hv, a.pw, P, a.xts, a.fold)) return e;
    if (int e = encode_rows(&a.tm_B, p->B, p->dtype, p->batch, p->length, p->ngroups, a.na, N, p->bc_token_stride, a.fold)) return e;
    if (int e = encode_rows(&a.tm_C, p->C, p->dtype, p->batch, p->length, p->ngroups, a.na, N, p->bc_token_stride, a.fold)) return e;
    return p->dtype == SSM_BF16 ? run_fwd_any<__nv_bfloat16>(a, s) : run_fwd_any<__half>(a, s);
}

int bwd(const ssm_chunk_scan_params* p, cudaStream_t s) {
    const Ws w = ws_layout(p);
    if (!p->workspace || p->workspace_bytes < w.total)
        return fail(SSM_ERR_WORKSPACE, "chunk_scan bwd: workspace too small");
    if (!aligned16(p->x) || !aligned16(p->B) || !aligned16(p->C) || !aligned16(p->dy) || !aligned16(p->dx) ||
        ((p->flags & SSM_HAS_Z) && (!aligned16(p->z) || !aligned16(p->dz))) || !aligned16(p->saved) ||
        !aligned16(p->dB) || !aligned16(p->dC))
        return fail(SSM_ERR_INVALID, "chunk_scan bwd (tensor cores): x, B, C, z, dy, dx, dz, dB, dC and saved must be 16-byte aligned");
    Args a;
    make_args(p, a);
    if (!(p->flags & SSM_HAS_INIT)) a.dinit = nullptr;
    char* ws = reinterpret_cast<char*>(p->workspace);
    a.dHt = reinterpret_cast<unsigned char*>(ws);
    a.dcs_inter = reinterpret_cast<float*>(ws + w.dh);
    a.dT = reinterpret_cast<float*>(ws + w.dh + w.dci);
    a.dA_part = reinterpret_cast<float*>(ws + w.dh + w.dci + w.dt);
    a.db_part = reinterpret_cast<float*>(ws + w.dh + w.dci + w.dt + w.part);
    a.dD_part = reinterpret_cast<float*>(ws + w.dh + w.dci + w.dt + 2 * w.part);
    if (int e = encode_rows(&a.tm_x, p->x, p->dtype, p->batch, p->length, a.hv, a.pw, P, a.xts, a.fold)) return e;
    if (int e = encode_rows(&a.tm_dy, p->dy, p->dtype, p->batch, p->length, a.hv, a.pw, P, p->nheads * p->headdim, a.fold)) return e;
    if (int e = encode_rows(&a.tm_B, p->B, p->dtype, p->batch, p->length, p->ngroups, a.na, N, p->bc_token_stride, a.fold)) return e;
    if (int e = encode_rows(&a.tm_C, p->C, p->dtype, p->batch, p->length, p->ngroups, a.na, N, p->bc_token_stride, a.fold)) return e;
    return p->dtype == SSM_BF16 ? run_bwd_any<__nv_bfloat16>(a, p, s) : run_bwd_any<__half>(a, p, s);
}

}  // namespace ssdtc
}  // namespace ssm

namespace ssm {
namespace ssdtc {
// The failure path of every bounded wait, exercised on purpose: one thread
// initialises an mbarrier that expects one arrival, nothing ever arrives and
// no copy is in flight, so tc::mbar_wait (the helper every pipeline here uses)
// runs out after `polls` polls; the kernel then records the code in the
// caller's status word and returns.
__global__ void selftest_wait_kernel(int* status, uint32_t polls) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    const uint32_t mb = tc::smem_u32(&bar);
    tc::mbar_init(mb, 1);
    if (!tc::mbar_wait(mb, 0, polls)) atomicCAS(status, 0, SSM_KERR_SELFTEST);
}
}  // namespace ssdtc
}  // namespace ssm

int ssm_conv_take_error();   // causal_conv1d.cu: the conv1d kernels' flag
int ssm_scan_take_error();   // selective_scan_tma.cu: the TMA scan kernels' flag

extern "C" int ssm_selftest_bounded_wait(int32_t* status, uint32_t polls, void* stream) {
    if (!status) return ssm::fail(SSM_ERR_INVALID, "selftest_bounded_wait: null status word");
    if (polls == 0 || polls > (1u << 20))
        return ssm::fail(SSM_ERR_INVALID, "selftest_bounded_wait: polls must be in 1..2^20");
    ssm::ssdtc::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, polls);
    return ssm::check_launch("selftest_bounded_wait");
}

extern "C" int ssm_take_kernel_error(void) {
    int v = 0;
    const cudaError_t e = cudaMemcpyFromSymbol(&v, ssm::ssdtc::g_kernel_error, sizeof(int));
    if (e != cudaSuccess) return -1;
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(ssm::ssdtc::g_kernel_error, &zero, sizeof(int));
    }
    const int c = ssm_conv_take_error();
    const int sc = ssm_scan_take_error();
    return v ? v : c ? c : sc;
}
