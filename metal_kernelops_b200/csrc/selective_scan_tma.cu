// Mamba-1 selective scan, TMA-staged forward and backward (sm_100a).
//
// Same algorithm and the same arithmetic, operation for operation, as the
// plain-staging kernels of selective_scan.cu (so both give identical results;
// the one exception is the dstate-16 backward of sscan_bwd2.cuh, whose sums
// over channels and states associate differently); what changes is how tiles
// reach and leave shared memory, and the per-chunk bookkeeping around the
// recurrence:
//
//  * Every activation tile (u, delta, z, dout, the saved scan output: CPC
//    channels x kChunk steps) and every B / C tile (NP states x kChunk steps)
//    arrives as ONE tensor copy (cp.async.bulk.tensor, issued by one thread,
//    completing on an mbarrier).  The tensor maps are 4-D (steps, channel in
//    group, group, batch) and 3-D (steps, state, batch*group), so channels past
//    the group and steps past the sequence land as zeros -- no per-element
//    bounds checks and no per-thread address arithmetic.
//  * The backward double-buffers those tiles: the copies of the next chunk
//    (walking backwards) are in flight while the current chunk computes.
//  * Outputs leave the same way: the forward writes y (and the saved scan
//    output) and the backward du, ddelta, dz in place over the tiles they were
//    computed from (each element is read and then written by one thread), and
//    one thread issues a tensor store per tile; the stores clip at the tensor
//    edges.
//  * The backward's saved states come through a two-slot ring of 16-byte
//    cp.async copies, one sub-block ahead, each warp copying its own channels'
//    states in contiguous 512-byte rows, so no thread waits on them.
//  * Every per-chunk loop runs a compile-time number of iterations with index
//    arithmetic in shifts and constant offsets.
//
// Conditions (checked on the host; otherwise the plain kernels run): the
// activations and B / C share one dtype, rows are 16-byte aligned (length *
// element size a multiple of 16, every base pointer 16-byte aligned), and the
// launch shape's state tile covers dstate exactly (dstate 4, 8, 16, 32, 64).
//
// Every wait on an mbarrier is bounded: a wait that runs out records a code
// (in the call's status word and a per-device flag), every thread drains its
// own copies in flight, and the CTA returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <string>
#include <type_traits>

#include "sscan.cuh"
#include "tc.cuh"

namespace ssm {
namespace sscan {

__device__ int g_scan_error;

__device__ __forceinline__ void report(const Args& a, int code) {
    atomicCAS(&g_scan_error, 0, code);
    if (a.status) atomicCAS(a.status, 0, code);
}

struct TmaArgs {
    Args a;
    // loads
    alignas(64) CUtensorMap m_u;
    alignas(64) CUtensorMap m_d;
    alignas(64) CUtensorMap m_z;
    alignas(64) CUtensorMap m_g;    // dout (backward)
    alignas(64) CUtensorMap m_ys;   // saved scan output (backward; forward: store)
    alignas(64) CUtensorMap m_B;
    alignas(64) CUtensorMap m_C;
    // stores: forward y; backward du, ddelta, dz
    alignas(64) CUtensorMap m_o0;
    alignas(64) CUtensorMap m_o1;
    alignas(64) CUtensorMap m_o2;
};

// ------------------------------------------------------------ tensor copies --
__device__ __forceinline__ void tma_load4(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                          uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4, %5}], [%6];"
        :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(mbar)
        : "memory");
}
__device__ __forceinline__ void tma_load3(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                          uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];"
        :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(mbar)
        : "memory");
}
__device__ __forceinline__ void tma_store4(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
        :: "l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the stores issued so far have finished reading shared memory
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// ... and have completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

constexpr size_t al128(size_t v) { return (v + 127) / 128 * 128; }
constexpr int log2c(int v) { return v <= 1 ? 0 : 1 + log2c(v / 2); }
constexpr uint32_t kPolls = 1u << 22;   // bounded mbarrier waits

// ------------------------------------------------------------------ forward --
template <typename T, int CPC, int NP>
struct FwdTmaLayout {
    static constexpr int K = kChunk;
    static constexpr int FS = K + 1;
    static constexpr size_t tile = al128((size_t)CPC * K * sizeof(T));   // [CPC][K] activation tile
    static constexpr size_t bct = al128((size_t)NP * K * sizeof(T));     // [NP][K] B or C tile
    static constexpr size_t o_u = 0, o_d = tile, o_z = 2 * tile;
    static constexpr size_t o_B = 3 * tile, o_C = o_B + bct;
    static constexpr size_t o_bc = o_C + bct;                             // fp32 [2][K][NP]
    static constexpr size_t o_dvu = o_bc + 2 * (size_t)K * NP * 4;        // [CPC][FS] float2
    static constexpr size_t o_ch = o_dvu + (size_t)CPC * FS * 8;          // [2][CPC] float
    static constexpr size_t o_bar = (o_ch + 2 * CPC * 4 + 7) / 8 * 8;
    static constexpr size_t bytes = o_bar + 16;
};

// One thread per (channel, NPT states) with LPC lanes per channel, kChunk-step
// chunks walked in order, one copy of every tile in flight per CTA (a tile's
// buffer holds its outputs until their stores have read it; nine CTAs share an
// SM, so copies of one overlap the compute of the others).
// LEAN: save only the state entering each chunk, and no scan output.
template <typename T, int NPT, int LPC, bool LEAN>
__global__ void __launch_bounds__(kThreads, NPT <= 8 ? 9 : 1)
fwd_tma_kernel(const __grid_constant__ TmaArgs ta) {
    const Args& a = ta.a;
    constexpr int CPW = 32 / LPC;
    constexpr int CPC = CPW * kWarps;
    constexpr int NP = NPT * LPC;
    constexpr int NH = NPT / 2;
    constexpr int K = kChunk;
    constexpr int FS = K + 1;
    using Lay = FwdTmaLayout<T, CPC, NP>;
    static_assert(NPT % 4 == 0 && kTS == 4 && K == 16 && CPC % 16 == 0, "launch shape");

    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((128u - (tc::smem_u32(smem_raw) & 127u)) & 127u);
    T* ru = reinterpret_cast<T*>(smem + Lay::o_u);
    T* rd = reinterpret_cast<T*>(smem + Lay::o_d);
    T* rz = reinterpret_cast<T*>(smem + Lay::o_z);
    const T* rB = reinterpret_cast<const T*>(smem + Lay::o_B);
    const T* rC = reinterpret_cast<const T*>(smem + Lay::o_C);
    float* Bs = reinterpret_cast<float*>(smem + Lay::o_bc);
    float* Cs = Bs + K * NP;
    float2* dvu = reinterpret_cast<float2*>(smem + Lay::o_dvu);   // (delta' log2e, delta' u) -> y in .x
    float* Dch = reinterpret_cast<float*>(smem + Lay::o_ch);
    float* bch = Dch + CPC;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Lay::o_bar);
    int* okp = reinterpret_cast<int*>(smem + Lay::o_bar + 8);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int cw = lane / LPC, sub = lane % LPC;
    const int c = warp * CPW + cw;
    const int64_t ct = blockIdx.x % a.nct, seg = blockIdx.x / a.nct, g = blockIdx.y, b = blockIdx.z;
    const int64_t dl0 = ct * CPC;
    const int rows = (int)min64(CPC, a.per_group - dl0);
    const int64_t d0 = g * a.per_group + dl0;
    const bool cvalid = c < rows;
    const int64_t d = d0 + c;
    const int64_t N = a.dstate, L = a.length;
    const bool has_d = a.flags & SSM_HAS_D, has_z = a.flags & SSM_HAS_Z;
    const bool has_bias = a.flags & SSM_HAS_BIAS, softplus = a.flags & SSM_SOFTPLUS;
    const bool save_y = a.ckpt != nullptr && has_z && !LEAN;
    const int64_t bg = b * a.groups + g;
    const int64_t sx = ((b * a.nseg + seg) * a.dim + d) * N;
    const uint32_t mb = tc::smem_u32(bar);
    const uint32_t tx = (uint32_t)((has_z ? 3 : 2) * CPC * K * sizeof(T) + 2 * NP * K * sizeof(T));

    auto issue = [&](int64_t tile) {   // thread 0: this chunk's input tiles
        const int t0 = (int)(tile * K);
        tc::mbar_expect_tx(mb, tx);
        tma_load4(tc::smem_u32(ru), &ta.m_u, t0, (int)dl0, (int)g, (int)b, mb);
        tma_load4(tc::smem_u32(rd), &ta.m_d, t0, (int)dl0, (int)g, (int)b, mb);
        if (has_z) tma_load4(tc::smem_u32(rz), &ta.m_z, t0, (int)dl0, (int)g, (int)b, mb);
        tma_load3(tc::smem_u32(rB), &ta.m_B, t0, 0, (int)bg, mb);
        tma_load3(tc::smem_u32(rC), &ta.m_C, t0, 0, (int)bg, mb);
    };

    const int64_t tile_lo = seg * a.seg_chunks;
    const int64_t tile_hi = min64(tile_lo + a.seg_chunks, a.nchunks);
    if (tid == 0) {
        tc::mbar_init(mb, 1);
        tc::fence_mbar_init();
        issue(tile_lo);
    }
    for (int i = tid; i < CPC; i += kThreads) {
        Dch[i] = (has_d && i < rows) ? a.D[d0 + i] : 0.0f;
        bch[i] = (has_bias && i < rows) ? a.delta_bias[d0 + i] : 0.0f;
    }
    float2 An2[NH], x2[NH];
    const bool from_seg = a.nseg > 1;
#pragma unroll
    for (int j = 0; j < NH; ++j) {
        const int n = sub * NPT + 2 * j;
        An2[j] = cvalid ? make_float2(a.A[d * N + n], a.A[d * N + n + 1]) : make_float2(0.0f, 0.0f);
        x2[j] = (from_seg && cvalid) ? make_float2(a.seg_x[sx + n], a.seg_x[sx + n + 1]) : make_float2(0.0f, 0.0f);
    }
    // this thread's saved states: (batch, sub-block, dim, dstate), 16-byte stores
    const int64_t sub_stride = a.dim * N;
    float* ck = a.ckpt ? a.ckpt + ((b * a.nsub + tile_lo * (LEAN ? 1 : K / kTS)) * a.dim + d) * N + sub * NPT
                       : nullptr;
    const bool save = a.ckpt != nullptr && cvalid;

    for (int64_t tile = tile_lo; tile < tile_hi; ++tile) {
        const int64_t t0 = tile * K;
        const int len = (int)min64(K, L - t0);
        if (tid == 0) okp[0] = tc::mbar_wait(mb, (uint32_t)((tile - tile_lo) & 1), kPolls) ? 1 : 0;
        __syncthreads();
        if (!okp[0]) {
            if (tid == 0) {
                report(a, 71);
                bulk_wait_all();
            }
            return;
        }

        // phase 0: per-step scalars (two steps per item) and B/C to fp32 [t][n]
#pragma unroll
        for (int k = 0; k < CPC / 16; ++k) {
            const int cc = (tid >> 3) + 16 * k, t = 2 * (tid & 7);
            const float2 dr = Io2<T>::ld(&rd[cc * K + t]);
            const float2 ur = Io2<T>::ld(&ru[cc * K + t]);
            float2 dv = add2(dr, f2(bch[cc]));
            if (softplus) dv = softplus2_fast(dv);
            const float2 dl = mul2(dv, f2(kLog2e)), du = mul2(dv, ur);
            dvu[cc * FS + t] = make_float2(dl.x, du.x);
            dvu[cc * FS + t + 1] = make_float2(dl.y, du.y);
        }
        for (int i = tid; i < NP * K; i += kThreads) {
            const int t = i / NP, n = i % NP;
            Bs[t * NP + n] = ldf(&rB[n * K + t]);
            Cs[t * NP + n] = ldf(&rC[n * K + t]);
        }
        __syncthreads();

        // phase 1: the recurrence, two states per packed instruction
        float2* vr = dvu + c * FS;
        auto step = [&](int t) {
            const float2 v = vr[t];
            const float2 dl2 = make_float2(v.x, v.x), du2 = make_float2(v.y, v.y);
            const float4* B4 = reinterpret_cast<const float4*>(Bs + t * NP + sub * NPT);
            const float4* C4 = reinterpret_cast<const float4*>(Cs + t * NP + sub * NPT);
            float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int q = 0; q < NPT / 4; ++q) {
                const float4 bq = B4[q], cq = C4[q];
                const float2 a0 = __fmul2_rn(dl2, An2[2 * q]);
                const float2 a1 = __fmul2_rn(dl2, An2[2 * q + 1]);
                const float2 e0 = make_float2(exp2_mufu(a0.x), exp2_mufu(a0.y));
                const float2 e1 = make_float2(exp2_mufu(a1.x), exp2_mufu(a1.y));
                x2[2 * q] = __ffma2_rn(e0, x2[2 * q], __fmul2_rn(du2, make_float2(bq.x, bq.y)));
                x2[2 * q + 1] = __ffma2_rn(e1, x2[2 * q + 1], __fmul2_rn(du2, make_float2(bq.z, bq.w)));
                acc0 = __ffma2_rn(x2[2 * q], make_float2(cq.x, cq.y), acc0);
                acc1 = __ffma2_rn(x2[2 * q + 1], make_float2(cq.z, cq.w), acc1);
            }
            float yv = (acc0.x + acc0.y) + (acc1.x + acc1.y);
            yv = sum_low_lanes<LPC>(yv);
            if (sub == 0) vr[t].x = yv;        // every lane of the channel has read vr[t]
        };
        auto store_ckpt = [&](int sb) {        // the state entering sub-block sb
            float* cp = ck + sb * sub_stride;
#pragma unroll
            for (int j = 0; j < NH; j += 2)
                __stcs(reinterpret_cast<float4*>(cp + 2 * j), make_float4(x2[j].x, x2[j].y, x2[j + 1].x, x2[j + 1].y));
        };
        if constexpr (LEAN) {                  // the state entering the chunk only
            if (save) store_ckpt(0);
            if (len == K) {
#pragma unroll
                for (int t = 0; t < K; ++t) step(t);
            } else {
#pragma unroll 1
                for (int t = 0; t < len; ++t) step(t);
            }
        } else if (len == K) {
#pragma unroll
            for (int t = 0; t < K; ++t) {
                if (t % kTS == 0 && save) store_ckpt(t / kTS);
                step(t);
            }
        } else {
#pragma unroll 1
            for (int t = 0; t < len; ++t) {
                if (t % kTS == 0 && save) store_ckpt(t / kTS);
                step(t);
            }
        }
        if (ck) ck += (LEAN ? 1 : K / kTS) * sub_stride;
        __syncthreads();

        // phase 2: skip and gate (two steps per item as paired lanes); y goes
        // over u, the saved scan output over delta (both dead for this chunk),
        // then one tensor store each
#pragma unroll
        for (int k = 0; k < CPC / 16; ++k) {
            const int cc = (tid >> 3) + 16 * k, t = 2 * (tid & 7);
            const float2 ur = Io2<T>::ld(&ru[cc * K + t]);
            const float2 yv = make_float2(dvu[cc * FS + t].x, dvu[cc * FS + t + 1].x);
            if (save_y) Io2<T>::st(&rd[cc * K + t], yv);
            float2 o = fma2(ur, f2(Dch[cc]), yv);
            if (has_z) {
                const float2 zr = Io2<T>::ld(&rz[cc * K + t]);
                o = mul2(o, mul2(zr, sigmoid2_t<T>(zr)));
            }
            Io2<T>::st(&ru[cc * K + t], o);
        }
        tc::fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tma_store4(&ta.m_o0, tc::smem_u32(ru), (int)t0, (int)dl0, (int)g, (int)b);
            if (save_y) tma_store4(&ta.m_ys, tc::smem_u32(rd), (int)t0, (int)dl0, (int)g, (int)b);
            bulk_commit();
            if (tile + 1 < tile_hi) {
                bulk_wait_read();              // the stores have read the tiles
                issue(tile + 1);
            }
        }
        (void)len;
    }
    if (tid == 0) bulk_wait_all();
}

// The forward's segment summary (nseg > 1, every segment but the last): the
// recurrence over this CTA's segment from a zero state, leaving the end state
// and the product of the decays, with the same arithmetic as the summary mode
// of the plain fwd_kernel.  Only u, delta and B are read.  Once phase 0 has
// turned a chunk's tiles into the fp32 step scalars and B, the tiles are dead,
// so the next chunk's copies are issued right then and land while this
// chunk's recurrence runs.
template <typename T, int NPT, int LPC>
__global__ void __launch_bounds__(kThreads, NPT <= 8 ? 9 : 1)
fwd_sum_tma_kernel(const __grid_constant__ TmaArgs ta) {
    const Args& a = ta.a;
    constexpr int CPW = 32 / LPC;
    constexpr int CPC = CPW * kWarps;
    constexpr int NP = NPT * LPC;
    constexpr int NH = NPT / 2;
    constexpr int K = kChunk;
    constexpr int FS = K + 1;
    using Lay = FwdTmaLayout<T, CPC, NP>;
    static_assert(NPT % 4 == 0 && K == 16 && CPC % 16 == 0, "launch shape");

    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((128u - (tc::smem_u32(smem_raw) & 127u)) & 127u);
    const T* ru = reinterpret_cast<const T*>(smem + Lay::o_u);
    const T* rd = reinterpret_cast<const T*>(smem + Lay::o_d);
    const T* rB = reinterpret_cast<const T*>(smem + Lay::o_B);
    float* Bs = reinterpret_cast<float*>(smem + Lay::o_bc);
    float2* dvu = reinterpret_cast<float2*>(smem + Lay::o_dvu);   // (delta' log2e, delta' u)
    float* bch = reinterpret_cast<float*>(smem + Lay::o_ch);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Lay::o_bar);
    int* okp = reinterpret_cast<int*>(smem + Lay::o_bar + 8);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int cw = lane / LPC, sub = lane % LPC;
    const int c = warp * CPW + cw;
    const int64_t ct = blockIdx.x % a.nct, seg = blockIdx.x / a.nct, g = blockIdx.y, b = blockIdx.z;
    const int64_t dl0 = ct * CPC;
    const int rows = (int)min64(CPC, a.per_group - dl0);
    const int64_t d0 = g * a.per_group + dl0;
    const bool cvalid = c < rows;
    const int64_t d = d0 + c;
    const int64_t N = a.dstate, L = a.length;
    const bool has_bias = a.flags & SSM_HAS_BIAS, softplus = a.flags & SSM_SOFTPLUS;
    const int64_t bg = b * a.groups + g;
    const int64_t sx = ((b * a.nseg + seg) * a.dim + d) * N;
    const uint32_t mb = tc::smem_u32(bar);
    const uint32_t tx = (uint32_t)(2 * CPC * K * sizeof(T) + NP * K * sizeof(T));

    auto issue = [&](int64_t tile) {   // thread 0: this chunk's u, delta and B tiles
        const int t0 = (int)(tile * K);
        tc::mbar_expect_tx(mb, tx);
        tma_load4(tc::smem_u32(ru), &ta.m_u, t0, (int)dl0, (int)g, (int)b, mb);
        tma_load4(tc::smem_u32(rd), &ta.m_d, t0, (int)dl0, (int)g, (int)b, mb);
        tma_load3(tc::smem_u32(rB), &ta.m_B, t0, 0, (int)bg, mb);
    };

    const int64_t tile_lo = seg * a.seg_chunks;
    const int64_t tile_hi = min64(tile_lo + a.seg_chunks, a.nchunks);
    if (tid == 0) {
        tc::mbar_init(mb, 1);
        tc::fence_mbar_init();
        issue(tile_lo);
    }
    for (int i = tid; i < CPC; i += kThreads) bch[i] = (has_bias && i < rows) ? a.delta_bias[d0 + i] : 0.0f;
    float2 An2[NH], x2[NH], p2[NH];
#pragma unroll
    for (int j = 0; j < NH; ++j) {
        const int n = sub * NPT + 2 * j;
        An2[j] = cvalid ? make_float2(a.A[d * N + n], a.A[d * N + n + 1]) : make_float2(0.0f, 0.0f);
        x2[j] = make_float2(0.0f, 0.0f);
        p2[j] = make_float2(1.0f, 1.0f);
    }

    for (int64_t tile = tile_lo; tile < tile_hi; ++tile) {
        const int len = (int)min64(K, L - tile * K);
        if (tid == 0) okp[0] = tc::mbar_wait(mb, (uint32_t)((tile - tile_lo) & 1), kPolls) ? 1 : 0;
        __syncthreads();                       // also: the previous chunk's recurrence is done
        if (!okp[0]) {
            if (tid == 0) report(a, 72);
            return;                            // the one copy in flight is the one this bounded wait gave up on
        }
        // phase 0: per-step scalars (two steps per item) and B to fp32 [t][n]
#pragma unroll
        for (int k = 0; k < CPC / 16; ++k) {
            const int cc = (tid >> 3) + 16 * k, t = 2 * (tid & 7);
            const float2 dr = Io2<T>::ld(&rd[cc * K + t]);
            const float2 ur = Io2<T>::ld(&ru[cc * K + t]);
            float2 dv = add2(dr, f2(bch[cc]));
            if (softplus) dv = softplus2_fast(dv);
            const float2 dl = mul2(dv, f2(kLog2e)), du = mul2(dv, ur);
            dvu[cc * FS + t] = make_float2(dl.x, du.x);
            dvu[cc * FS + t + 1] = make_float2(dl.y, du.y);
        }
        for (int i = tid; i < NP * K; i += kThreads) {
            const int t = i / NP, n = i % NP;
            Bs[t * NP + n] = ldf(&rB[n * K + t]);
        }
        __syncthreads();                       // the tiles are read: the next chunk's may land
        if (tid == 0 && tile + 1 < tile_hi) issue(tile + 1);

        // phase 1: the recurrence from a zero state, and the product of the decays
        const float2* vr = dvu + c * FS;
        auto step = [&](int t) {
            const float2 v = vr[t];
            const float2 dl2 = make_float2(v.x, v.x), du2 = make_float2(v.y, v.y);
            const float4* B4 = reinterpret_cast<const float4*>(Bs + t * NP + sub * NPT);
#pragma unroll
            for (int q = 0; q < NPT / 4; ++q) {
                const float4 bq = B4[q];
                const float2 a0 = __fmul2_rn(dl2, An2[2 * q]);
                const float2 a1 = __fmul2_rn(dl2, An2[2 * q + 1]);
                const float2 e0 = make_float2(exp2_mufu(a0.x), exp2_mufu(a0.y));
                const float2 e1 = make_float2(exp2_mufu(a1.x), exp2_mufu(a1.y));
                x2[2 * q] = __ffma2_rn(e0, x2[2 * q], __fmul2_rn(du2, make_float2(bq.x, bq.y)));
                x2[2 * q + 1] = __ffma2_rn(e1, x2[2 * q + 1], __fmul2_rn(du2, make_float2(bq.z, bq.w)));
                p2[2 * q] = __fmul2_rn(p2[2 * q], e0);
                p2[2 * q + 1] = __fmul2_rn(p2[2 * q + 1], e1);
            }
        };
        if (len == K) {
#pragma unroll
            for (int t = 0; t < K; ++t) step(t);
        } else {
#pragma unroll 1
            for (int t = 0; t < len; ++t) step(t);
        }
    }
    if (cvalid) {
#pragma unroll
        for (int j = 0; j < NH; ++j) {
            const int n = sub * NPT + 2 * j;
            a.seg_x[sx + n] = x2[j].x; a.seg_p[sx + n] = p2[j].x;
            a.seg_x[sx + n + 1] = x2[j].y; a.seg_p[sx + n + 1] = p2[j].y;
        }
    }
}

// The backward's segment summary (nseg > 1, every segment but the first): the
// adjoint recurrence q <- a_t (g_t C_t + q) over this CTA's segment, walked
// backwards from a zero adjoint at its end (g_t = dout_t, times the silu(z)
// gate), leaving the adjoint at the segment's start and the product of the
// decays, with the same arithmetic as the plain adj_kernel.  Reads delta,
// dout, z and C; like the forward summary, the copies of the chunk before this
// one are issued as soon as phase 0 has read this chunk's tiles.
template <typename T, int CPC, int NP>
struct AdjTmaLayout {
    static constexpr int K = kChunk;
    static constexpr int FS = K + 1;
    static constexpr size_t tile = al128((size_t)CPC * K * sizeof(T));
    static constexpr size_t bct = al128((size_t)NP * K * sizeof(T));
    static constexpr size_t o_d = 0, o_g = tile, o_z = 2 * tile, o_C = 3 * tile;
    static constexpr size_t o_c = o_C + bct;                              // fp32 [K][NP]
    static constexpr size_t o_dv = o_c + (size_t)K * NP * 4;              // [CPC][FS] float2
    static constexpr size_t o_ch = o_dv + (size_t)CPC * FS * 8;           // [CPC] float
    static constexpr size_t o_bar = (o_ch + CPC * 4 + 7) / 8 * 8;
    static constexpr size_t bytes = o_bar + 16;
};

template <typename T, int NPT, int LPC>
__global__ void __launch_bounds__(kThreads, NPT <= 8 ? 8 : 1)
adj_tma_kernel(const __grid_constant__ TmaArgs ta) {
    const Args& a = ta.a;
    constexpr int CPW = 32 / LPC;
    constexpr int CPC = CPW * kWarps;
    constexpr int NP = NPT * LPC;
    constexpr int NH = NPT / 2;
    constexpr int K = kChunk;
    constexpr int FS = K + 1;
    using Lay = AdjTmaLayout<T, CPC, NP>;
    static_assert(NPT % 4 == 0 && K == 16 && CPC % 16 == 0, "launch shape");

    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((128u - (tc::smem_u32(smem_raw) & 127u)) & 127u);
    const T* rd = reinterpret_cast<const T*>(smem + Lay::o_d);
    const T* rg = reinterpret_cast<const T*>(smem + Lay::o_g);
    const T* rz = reinterpret_cast<const T*>(smem + Lay::o_z);
    const T* rC = reinterpret_cast<const T*>(smem + Lay::o_C);
    float* Cs = reinterpret_cast<float*>(smem + Lay::o_c);
    float2* dv = reinterpret_cast<float2*>(smem + Lay::o_dv);     // (delta' log2e, g)
    float* bch = reinterpret_cast<float*>(smem + Lay::o_ch);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Lay::o_bar);
    int* okp = reinterpret_cast<int*>(smem + Lay::o_bar + 8);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int cw = lane / LPC, sub = lane % LPC;
    const int c = warp * CPW + cw;
    const int64_t ct = blockIdx.x % a.nct, seg = blockIdx.x / a.nct + 1, g = blockIdx.y, b = blockIdx.z;
    const int64_t dl0 = ct * CPC;
    const int rows = (int)min64(CPC, a.per_group - dl0);
    const int64_t d0 = g * a.per_group + dl0;
    const bool cvalid = c < rows;
    const int64_t d = d0 + c;
    const int64_t N = a.dstate, L = a.length;
    const bool has_z = a.flags & SSM_HAS_Z;
    const bool has_bias = a.flags & SSM_HAS_BIAS, softplus = a.flags & SSM_SOFTPLUS;
    const int64_t bg = b * a.groups + g;
    const int64_t sx = ((b * a.nseg + seg) * a.dim + d) * N;
    const uint32_t mb = tc::smem_u32(bar);
    const uint32_t tx = (uint32_t)((has_z ? 3 : 2) * CPC * K * sizeof(T) + NP * K * sizeof(T));

    auto issue = [&](int64_t tile) {   // thread 0: this chunk's delta, dout, z and C tiles
        const int t0 = (int)(tile * K);
        tc::mbar_expect_tx(mb, tx);
        tma_load4(tc::smem_u32(rd), &ta.m_d, t0, (int)dl0, (int)g, (int)b, mb);
        tma_load4(tc::smem_u32(rg), &ta.m_g, t0, (int)dl0, (int)g, (int)b, mb);
        if (has_z) tma_load4(tc::smem_u32(rz), &ta.m_z, t0, (int)dl0, (int)g, (int)b, mb);
        tma_load3(tc::smem_u32(rC), &ta.m_C, t0, 0, (int)bg, mb);
    };

    const int64_t tile_lo = seg * a.seg_chunks;
    const int64_t tile_hi = min64(tile_lo + a.seg_chunks, a.nchunks);
    if (tid == 0) {
        tc::mbar_init(mb, 1);
        tc::fence_mbar_init();
        issue(tile_hi - 1);
    }
    for (int i = tid; i < CPC; i += kThreads) bch[i] = (has_bias && i < rows) ? a.delta_bias[d0 + i] : 0.0f;
    float2 An2[NH], q2[NH], p2[NH];
#pragma unroll
    for (int j = 0; j < NH; ++j) {
        const int n = sub * NPT + 2 * j;
        An2[j] = cvalid ? make_float2(a.A[d * N + n], a.A[d * N + n + 1]) : make_float2(0.0f, 0.0f);
        q2[j] = make_float2(0.0f, 0.0f);
        p2[j] = make_float2(1.0f, 1.0f);
    }
    for (int64_t tile = tile_hi - 1; tile >= tile_lo; --tile) {
        const int len = (int)min64(K, L - tile * K);
        if (tid == 0) okp[0] = tc::mbar_wait(mb, (uint32_t)((tile_hi - 1 - tile) & 1), kPolls) ? 1 : 0;
        __syncthreads();                       // also: the later chunk's recurrence is done
        if (!okp[0]) {
            if (tid == 0) report(a, 73);
            return;                            // the one copy in flight is the one this bounded wait gave up on
        }
        // phase 0: per-step scalars (two steps per item) and C to fp32 [t][n]
#pragma unroll
        for (int k = 0; k < CPC / 16; ++k) {
            const int cc = (tid >> 3) + 16 * k, t = 2 * (tid & 7);
            const float2 dr = Io2<T>::ld(&rd[cc * K + t]);
            float2 go = Io2<T>::ld(&rg[cc * K + t]);
            float2 dl = add2(dr, f2(bch[cc]));
            if (softplus) dl = softplus2_fast(dl);
            if (has_z) {
                const float2 zr = Io2<T>::ld(&rz[cc * K + t]);
                go = mul2(go, mul2(zr, sigmoid2_t<T>(zr)));
            }
            dl = mul2(dl, f2(kLog2e));
            dv[cc * FS + t] = make_float2(dl.x, go.x);
            dv[cc * FS + t + 1] = make_float2(dl.y, go.y);
        }
        for (int i = tid; i < NP * K; i += kThreads) {
            const int t = i / NP, n = i % NP;
            Cs[t * NP + n] = ldf(&rC[n * K + t]);
        }
        __syncthreads();                       // the tiles are read: the earlier chunk's may land
        if (tid == 0 && tile > tile_lo) issue(tile - 1);

        const float2* vr = dv + c * FS;
        auto step = [&](int t) {
            const float2 v = vr[t];
            const float2 dl2 = make_float2(v.x, v.x), g2 = make_float2(v.y, v.y);
            const float4* C4 = reinterpret_cast<const float4*>(Cs + t * NP + sub * NPT);
#pragma unroll
            for (int q = 0; q < NPT / 4; ++q) {
                const float4 cq = C4[q];
                const float2 a0 = __fmul2_rn(dl2, An2[2 * q]);
                const float2 a1 = __fmul2_rn(dl2, An2[2 * q + 1]);
                const float2 e0 = make_float2(exp2_mufu(a0.x), exp2_mufu(a0.y));
                const float2 e1 = make_float2(exp2_mufu(a1.x), exp2_mufu(a1.y));
                q2[2 * q] = __fmul2_rn(__ffma2_rn(g2, make_float2(cq.x, cq.y), q2[2 * q]), e0);
                q2[2 * q + 1] = __fmul2_rn(__ffma2_rn(g2, make_float2(cq.z, cq.w), q2[2 * q + 1]), e1);
                p2[2 * q] = __fmul2_rn(p2[2 * q], e0);
                p2[2 * q + 1] = __fmul2_rn(p2[2 * q + 1], e1);
            }
        };
        if (len == K) {
#pragma unroll
            for (int t = K - 1; t >= 0; --t) step(t);
        } else {
#pragma unroll 1
            for (int t = len - 1; t >= 0; --t) step(t);
        }
    }
    if (cvalid) {
#pragma unroll
        for (int j = 0; j < NH; ++j) {
            const int n = sub * NPT + 2 * j;
            a.seg_x[sx + n] = q2[j].x; a.seg_p[sx + n] = p2[j].x;
            a.seg_x[sx + n + 1] = q2[j].y; a.seg_p[sx + n + 1] = p2[j].y;
        }
    }
}

// ----------------------------------------------------------------- backward --
template <typename T, int CPC, int NP, int NPT>
struct BwdTmaLayout {
    static constexpr int K = kChunk;
    static constexpr int FS = K + 1;
    static constexpr size_t tile = al128((size_t)CPC * K * sizeof(T));
    static constexpr size_t bct = al128((size_t)NP * K * sizeof(T));
    // one buffer: u, delta, z, dout, saved y, B, C
    static constexpr size_t o_u = 0, o_d = tile, o_z = 2 * tile, o_g = 3 * tile, o_y = 4 * tile;
    static constexpr size_t o_B = 5 * tile, o_C = o_B + bct;
    static constexpr size_t buf = o_C + bct;
    static constexpr size_t o_sck = 2 * buf;                                  // [2][NPT/4][kThreads] float4
    static constexpr int CS = K * NP + 16;                                    // permuted copy stride (floats)
    static constexpr size_t o_bc = o_sck + 2 * (size_t)NPT * kThreads * 4;    // fp32 [2][4][CS]
    static constexpr size_t o_dvu = o_bc + 2 * 4 * (size_t)CS * 4;            // [CPC][FS] float2
    static constexpr size_t o_f = o_dvu + (size_t)CPC * FS * 8;               // [3][CPC][FS] float
    static constexpr size_t o_w = o_f + 3 * (size_t)CPC * FS * 4;             // [2][kWarps][K][NP+1]
    static constexpr size_t o_ch = o_w + 2 * (size_t)kWarps * K * (NP + 1) * 4;   // [2][CPC]
    static constexpr size_t o_acc = o_ch + 2 * CPC * 4;                       // [2][CPC * K/2]
    static constexpr size_t o_bar = (o_acc + 2 * (size_t)CPC * (K / 2) * 4 + 7) / 8 * 8;
    static constexpr size_t bytes = o_bar + 32;
};

// LEAN: the forward saved only the state entering each chunk; each sub-block's
// entering state is replayed from it (0, 4, 8, 12 extra steps for the four
// sub-blocks of a chunk), and the scan output before the gate, which dz needs,
// is recomputed in the sub-block replay into the tile slot the saved output
// would have used.
template <typename T, int NPT, int LPC, bool LEAN>
__global__ void __launch_bounds__(kThreads, 3)
bwd_tma_kernel(const __grid_constant__ TmaArgs ta) {
    const Args& a = ta.a;
    constexpr int CPW = 32 / LPC;
    constexpr int CPC = CPW * kWarps;
    constexpr int NP = NPT * LPC;
    constexpr int NH = NPT / 2;
    constexpr int NQ = NPT / 4;          // 16-byte chunks of a lane's states
    constexpr int NPW = NP + 1;
    constexpr int K = kChunk;
    constexpr int FS = K + 1;
    constexpr int TS = kTS;
    constexpr int LO = log2c(LPC);
    using Sc = Scatter<NPT, LO>;
    constexpr int KEPT = Sc::kept();
    constexpr int HALF = K / 2;
    using Lay = BwdTmaLayout<T, CPC, NP, NPT>;
    static_assert(NPT % 4 == 0 && K == 16 && TS == 4 && CPC % 16 == 0, "launch shape");

    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((128u - (tc::smem_u32(smem_raw) & 127u)) & 127u);
    float2* dvu = reinterpret_cast<float2*>(smem + Lay::o_dvu);   // (delta', delta'*u)
    float* gs = reinterpret_cast<float*>(smem + Lay::o_f);        // gradient seen by the scan
    float* dua = gs + CPC * FS;                                   // sum_n dh*B
    float* dda = dua + CPC * FS;                                  // sum_n dh*a*x_prev*A
    constexpr int CS = Lay::CS;
    float* Bs = reinterpret_cast<float*>(smem + Lay::o_bc);       // [4 perms][CS]: [K][NP] + pad
    float* Cs = Bs + 4 * CS;
    float* dBw = reinterpret_cast<float*>(smem + Lay::o_w);
    float* dCw = dBw + kWarps * K * NPW;
    float* sck = reinterpret_cast<float*>(smem + Lay::o_sck);
    float* Dch = reinterpret_cast<float*>(smem + Lay::o_ch);
    float* bch = Dch + CPC;
    float* accD = reinterpret_cast<float*>(smem + Lay::o_acc);
    float* accb = accD + CPC * HALF;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Lay::o_bar);
    int* okp = reinterpret_cast<int*>(smem + Lay::o_bar + 16);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int cw = lane / LPC, sub = lane % LPC;
    const int c = warp * CPW + cw;
    const int64_t ct = blockIdx.x % a.nct, seg = blockIdx.x / a.nct, g = blockIdx.y, b = blockIdx.z;
    const int64_t dl0 = ct * CPC;
    const int rows = (int)min64(CPC, a.per_group - dl0);
    const int64_t d0 = g * a.per_group + dl0;
    const bool cvalid = c < rows;
    const int64_t d = d0 + c;
    const int64_t N = a.dstate, L = a.length;
    const bool has_d = a.flags & SSM_HAS_D, has_z = a.flags & SSM_HAS_Z;
    const bool has_bias = a.flags & SSM_HAS_BIAS, softplus = a.flags & SSM_SOFTPLUS;
    const int64_t bg = b * a.groups + g;
    const int64_t bs = b * a.nseg + seg;
    const int64_t sx = (bs * a.dim + d) * N;
    const int pm = Sc::mask(lane);
    const bool own = Sc::owner(lane);
    const float* Bp = Bs + (pm & 3) * CS + sub * NPT;
    const float* Cp = Cs + (pm & 3) * CS + sub * NPT;
    const int qx = pm >> 2;
    const uint32_t tx = (uint32_t)((has_z ? (LEAN ? 4 : 5) : 3) * CPC * K * sizeof(T) + 2 * NP * K * sizeof(T));

    auto bufp = [&](int buf, size_t off) { return smem + (size_t)buf * Lay::buf + off; };
    auto issue = [&](int64_t tile, int buf) {   // thread 0: one chunk's input tiles
        const uint32_t m = tc::smem_u32(&bar[buf]);
        const int t0 = (int)(tile * K);
        tc::mbar_expect_tx(m, tx);
        tma_load4(tc::smem_u32(bufp(buf, Lay::o_u)), &ta.m_u, t0, (int)dl0, (int)g, (int)b, m);
        tma_load4(tc::smem_u32(bufp(buf, Lay::o_d)), &ta.m_d, t0, (int)dl0, (int)g, (int)b, m);
        tma_load4(tc::smem_u32(bufp(buf, Lay::o_g)), &ta.m_g, t0, (int)dl0, (int)g, (int)b, m);
        if (has_z) {
            tma_load4(tc::smem_u32(bufp(buf, Lay::o_z)), &ta.m_z, t0, (int)dl0, (int)g, (int)b, m);
            if (!LEAN) tma_load4(tc::smem_u32(bufp(buf, Lay::o_y)), &ta.m_ys, t0, (int)dl0, (int)g, (int)b, m);
        }
        tma_load3(tc::smem_u32(bufp(buf, Lay::o_B)), &ta.m_B, t0, 0, (int)bg, m);
        tma_load3(tc::smem_u32(bufp(buf, Lay::o_C)), &ta.m_C, t0, 0, (int)bg, m);
    };

    const int64_t tile_lo = seg * a.seg_chunks;
    const int64_t tile_hi = min64(tile_lo + a.seg_chunks, a.nchunks);
    if (tid == 0) {
        tc::mbar_init(tc::smem_u32(&bar[0]), 1);
        tc::mbar_init(tc::smem_u32(&bar[1]), 1);
        tc::fence_mbar_init();
        issue(tile_hi - 1, 0);
    }

    // saved states: a two-slot ring of each thread's NPT states per sub-block
    // (16-byte chunk q of thread tid at [slot][q][tid]), filled one sub-block
    // ahead; sub-blocks are consumed in decreasing global order, from the CTA's
    // last one down to its first (tile_lo * K / TS)
    // (LEAN: one saved state per chunk, the same ring one chunk ahead).
    // Each warp copies its own channels' states, 512 contiguous bytes per copy
    // instruction: 16-byte piece k = q * 32 + lane of the warp's CPW x NP floats
    // goes to the slot of the lane that uses it (zeros for invalid channels).
    // Lanes then read copies other lanes made: a __syncwarp follows each wait,
    // and one precedes each refill of a slot the warp has read.
    const int last_len = (int)min64(K, L - (tile_hi - 1) * K);
    const int64_t s_first = LEAN ? tile_hi - 1 : (tile_hi - 1) * (K / TS) + (last_len + TS - 1) / TS - 1;
    int nleft = (int)(s_first - (LEAN ? tile_lo : tile_lo * (K / TS)));   // saved states still to fetch
    int slot = 0;
    const float* ckp = a.ckpt + ((b * a.nsub + s_first) * a.dim + d0) * N;   // the CTA's first channel
    auto fetch = [&](int sl) {              // the sub-block ckp points at, into slot sl
        constexpr int PPC = NP / 4;         // 16-byte pieces per channel
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const int k = q * 32 + lane;
            const int cwk = k / PPC, pc = k % PPC;
            const int ch = warp * CPW + cwk;
            const uint32_t dst = tc::smem_u32(
                sck + (((size_t)sl * NQ + pc % NQ) * kThreads + warp * 32 + cwk * LPC + pc / NQ) * 4);
            const bool ok = ch < rows;
            tc::cp_async16_zfill(dst, ckp + (ok ? ch * NP + 4 * pc : 0), ok ? 16u : 0u);
        }
        tc::cp_async_commit();
    };
    fetch(0);

    for (int i = tid; i < CPC; i += kThreads) {
        Dch[i] = (has_d && i < rows) ? a.D[d0 + i] : 0.0f;
        bch[i] = (has_bias && i < rows) ? a.delta_bias[d0 + i] : 0.0f;
    }
    for (int i = tid; i < CPC * HALF; i += kThreads) {
        accD[i] = 0.0f;
        accb[i] = 0.0f;
    }
    float2 An2[NH], q2[NH], dA2[NH];
#pragma unroll
    for (int j = 0; j < NH; ++j) {
        const int n0 = sub * NPT + ((2 * j) ^ pm), n1 = sub * NPT + ((2 * j + 1) ^ pm);
        An2[j] = cvalid ? make_float2(a.A[d * N + n0], a.A[d * N + n1]) : make_float2(0.0f, 0.0f);
        q2[j] = (a.nseg > 1 && cvalid) ? make_float2(a.seg_x[sx + n0], a.seg_x[sx + n1]) : make_float2(0.0f, 0.0f);
        dA2[j] = make_float2(0.0f, 0.0f);
    }

    const int64_t pofs = (bg * a.nct + ct) * N * L;        // this CTA's dB / dC partial tile

    int it = 0;
    for (int64_t tile = tile_hi - 1; tile >= tile_lo; --tile, ++it) {
        const int64_t t0 = tile * K;
        const int len = (int)min64(K, L - t0);
        const int buf = it & 1;
        __syncthreads();                       // the other buffer's readers are done
        if (tid == 0) {
            if (tile > tile_lo) {
                bulk_wait_read();              // its stores have read it
                issue(tile - 1, buf ^ 1);
            }
            okp[0] = tc::mbar_wait(tc::smem_u32(&bar[buf]), (uint32_t)((it >> 1) & 1), kPolls) ? 1 : 0;
        }
        __syncthreads();
        if (!okp[0]) {
            if (tid == 0) {
                report(a, 72);
                if (tile > tile_lo) tc::mbar_wait(tc::smem_u32(&bar[buf ^ 1]), (uint32_t)(((it + 1) >> 1) & 1), kPolls);
                bulk_wait_all();
            }
            tc::cp_async_wait<0>();
            return;
        }
        T* ru = reinterpret_cast<T*>(bufp(buf, Lay::o_u));
        T* rd = reinterpret_cast<T*>(bufp(buf, Lay::o_d));
        T* rz = reinterpret_cast<T*>(bufp(buf, Lay::o_z));
        const T* rg = reinterpret_cast<const T*>(bufp(buf, Lay::o_g));
        const T* ry = reinterpret_cast<const T*>(bufp(buf, Lay::o_y));
        const T* rB = reinterpret_cast<const T*>(bufp(buf, Lay::o_B));
        const T* rC = reinterpret_cast<const T*>(bufp(buf, Lay::o_C));

        // phase 0: per-step scalars, two steps per item as the lanes of paired
        // fp32 instructions (each lane rounds as the scalar form does)
#pragma unroll
        for (int k = 0; k < CPC / 16; ++k) {
            const int cc = (tid >> 3) + 16 * k, t = 2 * (tid & 7);
            const float2 dr = Io2<T>::ld(&rd[cc * K + t]);
            const float2 ur = Io2<T>::ld(&ru[cc * K + t]);
            float2 go = Io2<T>::ld(&rg[cc * K + t]);
            float2 dv = add2(dr, f2(bch[cc]));
            if (softplus) dv = softplus2_fast(dv);
            const float2 du = mul2(dv, ur);
            dvu[cc * FS + t] = make_float2(dv.x, du.x);
            dvu[cc * FS + t + 1] = make_float2(dv.y, du.y);
            if (has_z) {
                const float2 zr = Io2<T>::ld(&rz[cc * K + t]);
                go = mul2(go, mul2(zr, sigmoid2_t<T>(zr)));
            }
            gs[cc * FS + t] = go.x;
            gs[cc * FS + t + 1] = go.y;
        }
        // B/C as fp32 [t][n], in the four within-float4 orders (n & 3) ^ p:
        // one (array, step, 4-state group) per item, all four orders stored
        for (int i = tid; i < 2 * K * (NP / 4); i += kThreads) {
            const int arr = i / (K * (NP / 4)), r = i % (K * (NP / 4));
            const int t = r % K, nq = r / K;
            const T* src = (arr ? rC : rB) + nq * 4 * K + t;
            const float v0 = ldf(src), v1 = ldf(src + K), v2 = ldf(src + 2 * K), v3 = ldf(src + 3 * K);
            float* dst = (arr ? Cs : Bs) + t * NP + nq * 4;
            *reinterpret_cast<float4*>(dst) = make_float4(v0, v1, v2, v3);
            *reinterpret_cast<float4*>(dst + CS) = make_float4(v1, v0, v3, v2);
            *reinterpret_cast<float4*>(dst + 2 * CS) = make_float4(v2, v3, v0, v1);
            *reinterpret_cast<float4*>(dst + 3 * CS) = make_float4(v3, v2, v1, v0);
        }
        __syncthreads();

        T* const ryw = reinterpret_cast<T*>(bufp(buf, Lay::o_y));   // LEAN: recomputed scan output
        auto chunk_body = [&](auto full_tag) {
            constexpr bool FULL = decltype(full_tag)::value;
            float2 x2[NH];
            float2 x4[NH], x8[NH];            // LEAN, full chunk: the states entering steps TS and 2 TS
            const float2* vr = dvu + c * FS;
            const float* gr = gs + c * FS;
            int cslot = 0;
            (void)cslot;
            if constexpr (LEAN) {     // the chunk's entering state (the next chunk's copy started first)
                __syncwarp();
                if (nleft > 0) {
                    ckp -= a.ck_stride;
                    fetch(slot ^ 1);
                    --nleft;
                } else {
                    tc::cp_async_commit();
                }
                tc::cp_async_wait<1>();
                __syncwarp();
                cslot = slot;
                slot ^= 1;
            }

            for (int sb = ((FULL ? K : len) - 1) / TS; sb >= 0; --sb) {
                const int tb = sb * TS;
                const int nb = FULL ? TS : min(TS, len - tb);
                if constexpr (LEAN) {
                    // the chunk's entering state, replayed over the sub-blocks before
                    // sb; in a full chunk the states at steps TS and 2 TS, passed on
                    // the way to the last sub-block, are kept for the two before it
                    if (FULL && (sb == 2 || sb == 1)) {
#pragma unroll
                        for (int j = 0; j < NH; ++j) x2[j] = sb == 2 ? x8[j] : x4[j];
                    } else {
                    const float* src = sck + ((size_t)cslot * NQ * kThreads + tid) * 4;
#pragma unroll
                    for (int j = 0; j < NH; ++j) {
                        const int e0 = (2 * j) ^ pm, e1 = (2 * j + 1) ^ pm;
                        x2[j] = make_float2(src[(e0 >> 2) * kThreads * 4 + (e0 & 3)],
                                            src[(e1 >> 2) * kThreads * 4 + (e1 & 3)]);
                    }
                    for (int pb = 0; pb < sb; ++pb) {
#pragma unroll
                        for (int jj = 0; jj < TS; ++jj) {
                            const float2 v = vr[pb * TS + jj];
                            const float dl = v.x * kLog2e;
                            const float2 dl2 = make_float2(dl, dl), du2 = make_float2(v.y, v.y);
                            const float4* B4 = reinterpret_cast<const float4*>(Bp + (pb * TS + jj) * NP);
#pragma unroll
                            for (int qq = 0; qq < NPT / 4; ++qq) {
                                const float4 bq = B4[qq ^ qx];
                                const float2 a0 = __fmul2_rn(dl2, An2[2 * qq]);
                                const float2 a1 = __fmul2_rn(dl2, An2[2 * qq + 1]);
                                const float2 e0 = make_float2(exp2_mufu(a0.x), exp2_mufu(a0.y));
                                const float2 e1 = make_float2(exp2_mufu(a1.x), exp2_mufu(a1.y));
                                x2[2 * qq] = __ffma2_rn(e0, x2[2 * qq], __fmul2_rn(du2, make_float2(bq.x, bq.y)));
                                x2[2 * qq + 1] = __ffma2_rn(e1, x2[2 * qq + 1], __fmul2_rn(du2, make_float2(bq.z, bq.w)));
                            }
                        }
                        if (FULL && pb <= 1) {
#pragma unroll
                            for (int j = 0; j < NH; ++j) {
                                if (pb == 0) x4[j] = x2[j];
                                else x8[j] = x2[j];
                            }
                        }
                    }
                    }
                } else {
                // this sub-block's entering states (its copies are done: the
                // next sub-block's are started first)
                __syncwarp();
                if (nleft > 0) {
                    ckp -= a.ck_stride;
                    fetch(slot ^ 1);
                    --nleft;
                } else {
                    tc::cp_async_commit();
                }
                tc::cp_async_wait<1>();
                __syncwarp();
                {
                    const float* src = sck + ((size_t)slot * NQ * kThreads + tid) * 4;
#pragma unroll
                    for (int j = 0; j < NH; ++j) {
                        const int e0 = (2 * j) ^ pm, e1 = (2 * j + 1) ^ pm;
                        x2[j] = make_float2(src[(e0 >> 2) * kThreads * 4 + (e0 & 3)],
                                            src[(e1 >> 2) * kThreads * 4 + (e1 & 3)]);
                    }
                }
                slot ^= 1;
                }
                // the replay keeps the states entering each step; the
                // adjoint recomputes each step's decays (two exponentials per
                // element-state: a decay history would cost 32 more registers
                // and spill at this kernel's 3-CTA register budget)
                float2 xh[TS][NH];
#pragma unroll
                for (int jj = 0; jj < TS; ++jj) {
                    if (FULL || jj < nb) {
                        const float2 v = vr[tb + jj];
                        const float dl = v.x * kLog2e;
                        const float2 dl2 = make_float2(dl, dl), du2 = make_float2(v.y, v.y);
                        const float4* B4 = reinterpret_cast<const float4*>(Bp + (tb + jj) * NP);
#pragma unroll
                        for (int qq = 0; qq < NPT / 4; ++qq) {
                            const float4 bq = B4[qq ^ qx];
                            const float2 a0 = __fmul2_rn(dl2, An2[2 * qq]);
                            const float2 a1 = __fmul2_rn(dl2, An2[2 * qq + 1]);
                            const float2 e0 = make_float2(exp2_mufu(a0.x), exp2_mufu(a0.y));
                            const float2 e1 = make_float2(exp2_mufu(a1.x), exp2_mufu(a1.y));
                            xh[jj][2 * qq] = x2[2 * qq];
                            xh[jj][2 * qq + 1] = x2[2 * qq + 1];
                            x2[2 * qq] = __ffma2_rn(e0, x2[2 * qq], __fmul2_rn(du2, make_float2(bq.x, bq.y)));
                            x2[2 * qq + 1] = __ffma2_rn(e1, x2[2 * qq + 1], __fmul2_rn(du2, make_float2(bq.z, bq.w)));
                        }
                        if (LEAN && has_z) {   // the scan output <x_t, C_t> of this step, for dz
                            const float4* C4 = reinterpret_cast<const float4*>(Cp + (tb + jj) * NP);
                            float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
                            for (int qq = 0; qq < NPT / 4; ++qq) {
                                const float4 cq = C4[qq ^ qx];
                                acc = __ffma2_rn(x2[2 * qq], make_float2(cq.x, cq.y), acc);
                                acc = __ffma2_rn(x2[2 * qq + 1], make_float2(cq.z, cq.w), acc);
                            }
                            const float yv = sum_low_lanes<LPC>(acc.x + acc.y);
                            if (sub == 0) stf(&ryw[c * K + tb + jj], yv);
                        }
                    }
                }
#pragma unroll
                for (int jj = TS - 1; jj >= 0; --jj) {
                    if (FULL || jj < nb) {
                        const int t = tb + jj;
                        const float2 v = vr[t];
                        const float gv = gr[t];
                        const float2 g2 = make_float2(gv, gv), dv2 = make_float2(v.x, v.x);
                        const float2 du2 = make_float2(v.y, v.y);
                        const float4* B4 = reinterpret_cast<const float4*>(Bp + t * NP);
                        const float4* C4 = reinterpret_cast<const float4*>(Cp + t * NP);
                        float2 dua2 = make_float2(0.0f, 0.0f), dda2 = make_float2(0.0f, 0.0f);
                        const float dlr = v.x * kLog2e;
                        const float2 dlr2 = make_float2(dlr, dlr);
                        float w[NPT];
#pragma unroll
                        for (int qq = 0; qq < NPT / 4; ++qq) {
                            const float4 bq = B4[qq ^ qx], cq = C4[qq ^ qx];
                            const float2 bb[2] = {make_float2(bq.x, bq.y), make_float2(bq.z, bq.w)};
                            const float2 cc2[2] = {make_float2(cq.x, cq.y), make_float2(cq.z, cq.w)};
#pragma unroll
                            for (int r = 0; r < 2; ++r) {
                                const int j = 2 * qq + r;
                                const float2 ar = __fmul2_rn(dlr2, An2[j]);
                                const float2 aj = make_float2(exp2_mufu(ar.x), exp2_mufu(ar.y));
                                const float2 dh = __ffma2_rn(g2, cc2[r], q2[j]);
                                const float2 tmp = __fmul2_rn(dh, __fmul2_rn(aj, xh[jj][j]));
                                dda2 = __ffma2_rn(tmp, An2[j], dda2);
                                dA2[j] = __ffma2_rn(tmp, dv2, dA2[j]);
                                dua2 = __ffma2_rn(dh, bb[r], dua2);
                                const float2 wv = __fmul2_rn(dh, du2);
                                w[2 * j] = wv.x;
                                w[2 * j + 1] = wv.y;
                                q2[j] = __fmul2_rn(dh, aj);
                            }
                        }
                        const float duacc = sum_low_lanes<LPC>(dua2.x + dua2.y);
                        const float ddacc = sum_low_lanes<LPC>(dda2.x + dda2.y);
                        Sc::reduce(w);
                        if (own) {
#pragma unroll
                            for (int i = 0; i < KEPT; ++i) dBw[(warp * K + t) * NPW + sub * NPT + pm + i] = w[i];
                        }
                        const bool last = FULL ? (jj == TS - 1) : (jj == nb - 1);
#pragma unroll
                        for (int j = 0; j < NH; ++j) {
                            const float2 xt = (jj + 1 < TS && !last) ? xh[jj + 1 < TS ? jj + 1 : jj][j] : x2[j];
                            const float2 wv = __fmul2_rn(g2, xt);
                            w[2 * j] = wv.x;
                            w[2 * j + 1] = wv.y;
                        }
                        Sc::reduce(w);
                        if (own) {
#pragma unroll
                            for (int i = 0; i < KEPT; ++i) dCw[(warp * K + t) * NPW + sub * NPT + pm + i] = w[i];
                        }
                        if (sub == 0) {
                            dua[c * FS + t] = duacc;
                            dda[c * FS + t] = ddacc;
                        }
                    }
                }
            }
        };
        if (len == K) chunk_body(std::true_type{});
        else chunk_body(std::false_type{});
        __syncthreads();

        // phase C: element-wise gradients, written over the tiles they came
        // from (du over u, ddelta over delta, dz over z), then tensor stores
        // (two steps per item as the lanes of paired fp32 instructions; each
        // lane rounds as the plain-staging kernel's scalar form does)
#pragma unroll
        for (int k = 0; k < CPC / 16; ++k) {
            const int cc = (tid >> 3) + 16 * k, t = 2 * (tid & 7);
            const int i = tid + kThreads * k;
            const float2 ur = Io2<T>::ld(&ru[cc * K + t]);
            const float Dv = Dch[cc];
            const float2 dv = make_float2(dvu[cc * FS + t].x, dvu[cc * FS + t + 1].x);
            const float2 gv = make_float2(gs[cc * FS + t], gs[cc * FS + t + 1]);
            const float2 dsum = make_float2(dua[cc * FS + t], dua[cc * FS + t + 1]);
            const float2 o_du = fma2(dv, dsum, mul2(gv, f2(Dv)));
            float2 ddt = fma2(ur, dsum, make_float2(dda[cc * FS + t], dda[cc * FS + t + 1]));
            if (softplus) {                   // softplus' (threshold 20)
                const float2 xs = add2(Io2<T>::ld(&rd[cc * K + t]), f2(bch[cc]));
                const float2 sg = sigmoid2_t<T>(xs);
                ddt = mul2(ddt, make_float2(xs.x > 20.0f ? 1.0f : sg.x, xs.y > 20.0f ? 1.0f : sg.y));
            }
            float2 o_dz = make_float2(0.0f, 0.0f);
            if (has_z) {
                const float2 zr = Io2<T>::ld(&rz[cc * K + t]);
                const float2 sg = sigmoid2_t<T>(zr);
                const float2 pre = fma2(ur, f2(Dv), Io2<T>::ld(&ry[cc * K + t]));
                o_dz = mul2(mul2(mul2(Io2<T>::ld(&rg[cc * K + t]), pre), sg),
                            fma2(zr, fma2(sg, f2(-1.0f), f2(1.0f)), f2(1.0f)));
            }
            float pD = 0.0f, pb = 0.0f;
            if (cc < rows) {
                if (t < len) {
                    pD = fmaf(gv.x, ur.x, pD);
                    pb += ddt.x;
                }
                if (t + 1 < len) {
                    pD = fmaf(gv.y, ur.y, pD);
                    pb += ddt.y;
                }
            }
            Io2<T>::st(&ru[cc * K + t], o_du);
            Io2<T>::st(&rd[cc * K + t], ddt);
            if (has_z) Io2<T>::st(&rz[cc * K + t], o_dz);
            accD[i] += pD;                    // this thread's own slot
            accb[i] += pb;
        }
        // dB / dC of the chunk: the warps' partials added in order, one
        // partial per CTA
        if (len == K) {
#pragma unroll
            for (int k = 0; k < (NP * K + kThreads - 1) / kThreads; ++k) {
                const int i = tid + kThreads * k;
                if ((NP * K) % kThreads == 0 || i < NP * K) {
                    const int n = i / K, t = i % K;
                    float sb_ = 0.0f, sc_ = 0.0f;
#pragma unroll
                    for (int w = 0; w < kWarps; ++w) {
                        sb_ += dBw[(w * K + t) * NPW + n];
                        sc_ += dCw[(w * K + t) * NPW + n];
                    }
                    a.dB_part[pofs + n * L + t0 + t] = sb_;
                    a.dC_part[pofs + n * L + t0 + t] = sc_;
                }
            }
        } else {
            for (int i = tid; i < NP * len; i += kThreads) {
                const int n = i / len, t = i % len;
                float sb_ = 0.0f, sc_ = 0.0f;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) {
                    sb_ += dBw[(w * K + t) * NPW + n];
                    sc_ += dCw[(w * K + t) * NPW + n];
                }
                a.dB_part[pofs + n * L + t0 + t] = sb_;
                a.dC_part[pofs + n * L + t0 + t] = sc_;
            }
        }
        tc::fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tma_store4(&ta.m_o0, tc::smem_u32(ru), (int)t0, (int)dl0, (int)g, (int)b);
            tma_store4(&ta.m_o1, tc::smem_u32(rd), (int)t0, (int)dl0, (int)g, (int)b);
            if (has_z) tma_store4(&ta.m_o2, tc::smem_u32(rz), (int)t0, (int)dl0, (int)g, (int)b);
            bulk_commit();
        }
    }
    tc::cp_async_wait<0>();
    __syncthreads();

    if (cvalid) {
        float* dap = a.dA_part + (bs * a.dim + d) * N;
#pragma unroll
        for (int j = 0; j < NH; ++j) {
            const int n0 = sub * NPT + ((2 * j) ^ pm), n1 = sub * NPT + ((2 * j + 1) ^ pm);
            dap[n0] = dA2[j].x;
            dap[n1] = dA2[j].y;
        }
    }
    for (int i = tid; i < rows; i += kThreads) {
        float sd = 0.0f, sb = 0.0f;
#pragma unroll
        for (int h = 0; h < HALF; ++h) {
            sd += accD[i * HALF + h];
            sb += accb[i * HALF + h];
        }
        a.dD_part[bs * a.dim + d0 + i] = sd;
        a.db_part[bs * a.dim + d0 + i] = sb;
    }
    if (tid == 0) bulk_wait_all();
}

#include "sscan_bwd2.cuh"


// --------------------------------------------------------------------- host --
static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
        else
            cudaGetLastError();
    });
    return fn;
}

static CUtensorMapDataType tma_type(int dtype) {
    return dtype == SSM_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                            : dtype == SSM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// (batch, dim, length) activations as (steps, channel in group, group, batch);
// box: kChunk steps x cpc channels of one group of one batch row
static int encode_act(CUtensorMap* m, const void* base, const ssm_selective_scan_params* p, int cpc) {
    const int64_t es = p->act_dtype == SSM_F32 ? 4 : 2;
    const int64_t P = p->dim / p->groups;
    cuuint64_t dims[4] = {(cuuint64_t)p->length, (cuuint64_t)P, (cuuint64_t)p->groups, (cuuint64_t)p->batch};
    cuuint64_t strides[3] = {(cuuint64_t)(p->length * es), (cuuint64_t)(P * p->length * es),
                             (cuuint64_t)(p->dim * p->length * es)};
    cuuint32_t box[4] = {(cuuint32_t)kChunk, (cuuint32_t)cpc, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = encoder()(m, tma_type(p->act_dtype), 4, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? SSM_OK
                             : fail(SSM_ERR_CUDA, "selective_scan (TMA): cuTensorMapEncodeTiled failed (" +
                                                      std::to_string((int)r) + ")");
}

// (batch, groups, dstate, length) B or C as (steps, state, batch*group); box:
// kChunk steps x np states
static int encode_bc(CUtensorMap* m, const void* base, const ssm_selective_scan_params* p, int np) {
    const int64_t es = p->bc_dtype == SSM_F32 ? 4 : 2;
    cuuint64_t dims[3] = {(cuuint64_t)p->length, (cuuint64_t)p->dstate, (cuuint64_t)(p->batch * p->groups)};
    cuuint64_t strides[2] = {(cuuint64_t)(p->length * es), (cuuint64_t)(p->dstate * p->length * es)};
    cuuint32_t box[3] = {(cuuint32_t)kChunk, (cuuint32_t)np, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encoder()(m, tma_type(p->bc_dtype), 3, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? SSM_OK
                             : fail(SSM_ERR_CUDA, "selective_scan (TMA): cuTensorMapEncodeTiled failed (" +
                                                      std::to_string((int)r) + ")");
}

static bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

// The layout conditions of the TMA path (see the file comment).
static bool tma_ok(const ssm_selective_scan_params* p, const Cfg& c, bool bwd) {
    if ((p->flags & SSM_SCAN_PLAIN) || !encoder()) return false;
    if (p->act_dtype != p->bc_dtype || (int64_t)c.npt * c.lpc != p->dstate) return false;
    const int64_t es = p->act_dtype == SSM_F32 ? 4 : 2;
    if ((p->length * es) % 16) return false;
    if (p->length > (int64_t)INT32_MAX || p->dim > (int64_t)INT32_MAX) return false;
    if (!al16(p->u) || !al16(p->delta) || !al16(p->B) || !al16(p->C)) return false;
    if ((p->flags & SSM_HAS_Z) && !al16(p->z)) return false;
    if (!bwd) return al16(p->y) && (!p->checkpoints || al16(p->checkpoints));
    return al16(p->dout) && al16(p->du) && al16(p->ddelta) && al16(p->checkpoints) &&
           (!(p->flags & SSM_HAS_Z) || al16(p->dz));
}

template <typename T, int NPT, int LPC>
static int run_fwd_tma(const TmaArgs& ta, cudaStream_t st) {
    constexpr int CPC = 32 / LPC * kWarps;
    const size_t sm = FwdTmaLayout<T, CPC, NPT * LPC>::bytes + 128;
    auto k = ta.a.lean ? fwd_tma_kernel<T, NPT, LPC, true> : fwd_tma_kernel<T, NPT, LPC, false>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return check_launch("selective_scan fwd (TMA): smem attribute");
    const Args& a = ta.a;
    k<<<dim3((unsigned)(a.nct * a.nseg), (unsigned)a.groups, (unsigned)a.batch), kThreads, sm, st>>>(ta);
    return check_launch("selective_scan fwd (TMA)");
}

template <typename T, int NPT, int LPC>
static int run_fwd_sum_tma(const TmaArgs& ta, cudaStream_t st) {
    constexpr int CPC = 32 / LPC * kWarps;
    const size_t sm = FwdTmaLayout<T, CPC, NPT * LPC>::bytes + 128;
    auto k = fwd_sum_tma_kernel<T, NPT, LPC>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return check_launch("selective_scan fwd summary (TMA): smem attribute");
    const Args& a = ta.a;
    k<<<dim3((unsigned)(a.nct * (a.nseg - 1)), (unsigned)a.groups, (unsigned)a.batch), kThreads, sm, st>>>(ta);
    return check_launch("selective_scan fwd summary (TMA)");
}

template <typename T, int NPT, int LPC>
static int run_adj_tma(const TmaArgs& ta, cudaStream_t st) {
    constexpr int CPC = 32 / LPC * kWarps;
    const size_t sm = AdjTmaLayout<T, CPC, NPT * LPC>::bytes + 128;
    auto k = adj_tma_kernel<T, NPT, LPC>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return check_launch("selective_scan bwd summary (TMA): smem attribute");
    const Args& a = ta.a;
    k<<<dim3((unsigned)(a.nct * (a.nseg - 1)), (unsigned)a.groups, (unsigned)a.batch), kThreads, sm, st>>>(ta);
    return check_launch("selective_scan bwd summary (TMA)");
}

template <typename T, int NPT, int LPC>
static int run_bwd_tma(const TmaArgs& ta, cudaStream_t st) {
    constexpr int CPC = 32 / LPC * kWarps;
    const size_t sm = BwdTmaLayout<T, CPC, NPT * LPC, NPT>::bytes + 128;
    auto k = ta.a.lean ? bwd_tma_kernel<T, NPT, LPC, true> : bwd_tma_kernel<T, NPT, LPC, false>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return check_launch("selective_scan bwd (TMA): smem attribute");
    const Args& a = ta.a;
    k<<<dim3((unsigned)(a.nct * a.nseg), (unsigned)a.groups, (unsigned)a.batch), kThreads, sm, st>>>(ta);
    return check_launch("selective_scan bwd (TMA)");
}

// dstate 16 at 8 states x 2 lanes per channel: the two-channels-per-lane kernel
template <typename T>
static int run_bwd2_tma(const TmaArgs& ta, cudaStream_t st) {
    const size_t sm = BwdTmaLayout<T, 64, 16, 8>::bytes + 128;
    auto k = ta.a.lean ? bwd2_tma_kernel<T, true> : bwd2_tma_kernel<T, false>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return check_launch("selective_scan bwd (TMA): smem attribute");
    const Args& a = ta.a;
    k<<<dim3((unsigned)(a.nct * a.nseg), (unsigned)a.groups, (unsigned)a.batch), kThreads, sm, st>>>(ta);
    return check_launch("selective_scan bwd (TMA)");
}

template <typename T>
static int dispatch_fwd_tma(const Cfg& c, const TmaArgs& ta, cudaStream_t st) {
    switch (c.npt * 100 + c.lpc) {
        case 401: return run_fwd_tma<T, 4, 1>(ta, st);
        case 402: return run_fwd_tma<T, 4, 2>(ta, st);
        case 404: return run_fwd_tma<T, 4, 4>(ta, st);
        case 801: return run_fwd_tma<T, 8, 1>(ta, st);
        case 802: return run_fwd_tma<T, 8, 2>(ta, st);
        case 804: return run_fwd_tma<T, 8, 4>(ta, st);
        case 1602: return run_fwd_tma<T, 16, 2>(ta, st);
        case 1604: return run_fwd_tma<T, 16, 4>(ta, st);
        default: return SSM_ERR_UNSUPPORTED;
    }
}

template <typename T>
static int dispatch_fwd_sum_tma(const Cfg& c, const TmaArgs& ta, cudaStream_t st) {
    switch (c.npt * 100 + c.lpc) {
        case 401: return run_fwd_sum_tma<T, 4, 1>(ta, st);
        case 402: return run_fwd_sum_tma<T, 4, 2>(ta, st);
        case 404: return run_fwd_sum_tma<T, 4, 4>(ta, st);
        case 801: return run_fwd_sum_tma<T, 8, 1>(ta, st);
        case 802: return run_fwd_sum_tma<T, 8, 2>(ta, st);
        case 804: return run_fwd_sum_tma<T, 8, 4>(ta, st);
        case 1602: return run_fwd_sum_tma<T, 16, 2>(ta, st);
        case 1604: return run_fwd_sum_tma<T, 16, 4>(ta, st);
        default: return SSM_ERR_UNSUPPORTED;
    }
}

template <typename T>
static int dispatch_bwd_tma(const Cfg& c, const TmaArgs& ta, cudaStream_t st) {
    switch (c.npt * 100 + c.lpc) {
        case 401: return run_bwd_tma<T, 4, 1>(ta, st);
        case 404: return run_bwd_tma<T, 4, 4>(ta, st);
        case 801: return run_bwd_tma<T, 8, 1>(ta, st);
        case 802: return run_bwd2_tma<T>(ta, st);
        case 804: return run_bwd_tma<T, 8, 4>(ta, st);
        case 808: return run_bwd_tma<T, 8, 8>(ta, st);
        default: return SSM_ERR_UNSUPPORTED;
    }
}

int fwd_tma(const ssm_selective_scan_params* p, const Cfg& c, const Args& a, cudaStream_t st) {
    if (!tma_ok(p, c, false)) return SSM_ERR_UNSUPPORTED;
    if (int s = ensure_context("selective_scan fwd (TMA)")) return s;
    const int cpc = 32 / c.lpc * kWarps, np = c.npt * c.lpc;
    TmaArgs ta;
    ta.a = a;
    if (int s = encode_act(&ta.m_u, p->u, p, cpc)) return s;
    if (int s = encode_act(&ta.m_d, p->delta, p, cpc)) return s;
    if (int s = encode_act(&ta.m_z, (p->flags & SSM_HAS_Z) ? p->z : p->u, p, cpc)) return s;
    if (int s = encode_act(&ta.m_o0, p->y, p, cpc)) return s;
    const void* ys = (p->checkpoints && !a.lean) ? reinterpret_cast<const char*>(p->checkpoints) + a.ysave_off : p->y;
    if (int s = encode_act(&ta.m_ys, ys, p, cpc)) return s;
    if (int s = encode_bc(&ta.m_B, p->B, p, np)) return s;
    if (int s = encode_bc(&ta.m_C, p->C, p, np)) return s;
    switch (p->act_dtype) {
        case SSM_F32: return dispatch_fwd_tma<float>(c, ta, st);
        case SSM_BF16: return dispatch_fwd_tma<__nv_bfloat16>(c, ta, st);
        default: return dispatch_fwd_tma<__half>(c, ta, st);
    }
}

// The forward's segment summaries through TMA (SSM_ERR_UNSUPPORTED where the
// TMA conditions do not hold: the caller then runs the plain summary pass).
int fwd_sum_tma(const ssm_selective_scan_params* p, const Cfg& c, const Args& a, cudaStream_t st) {
    if (a.nseg < 2 || !tma_ok(p, c, false)) return SSM_ERR_UNSUPPORTED;
    if (int s = ensure_context("selective_scan fwd summary (TMA)")) return s;
    const int cpc = 32 / c.lpc * kWarps, np = c.npt * c.lpc;
    TmaArgs ta;
    ta.a = a;
    if (int s = encode_act(&ta.m_u, p->u, p, cpc)) return s;
    if (int s = encode_act(&ta.m_d, p->delta, p, cpc)) return s;
    if (int s = encode_bc(&ta.m_B, p->B, p, np)) return s;
    switch (p->act_dtype) {
        case SSM_F32: return dispatch_fwd_sum_tma<float>(c, ta, st);
        case SSM_BF16: return dispatch_fwd_sum_tma<__nv_bfloat16>(c, ta, st);
        default: return dispatch_fwd_sum_tma<__half>(c, ta, st);
    }
}

// The backward's segment summaries through TMA, for the launch shapes the TMA
// backward itself runs (SSM_ERR_UNSUPPORTED otherwise: the caller then runs
// the plain summary pass).
int bwd_sum_tma(const ssm_selective_scan_params* p, const Cfg& c, const Args& a, cudaStream_t st) {
    if (a.nseg < 2 || !tma_ok(p, c, true)) return SSM_ERR_UNSUPPORTED;
    if (int s = ensure_context("selective_scan bwd summary (TMA)")) return s;
    const int cpc = 32 / c.lpc * kWarps, np = c.npt * c.lpc;
    TmaArgs ta;
    ta.a = a;
    if (int s = encode_act(&ta.m_d, p->delta, p, cpc)) return s;
    if (int s = encode_act(&ta.m_g, p->dout, p, cpc)) return s;
    if (int s = encode_act(&ta.m_z, (p->flags & SSM_HAS_Z) ? p->z : p->delta, p, cpc)) return s;
    if (int s = encode_bc(&ta.m_C, p->C, p, np)) return s;
    const int key = c.npt * 100 + c.lpc;
    auto by = [&](auto tag) -> int {
        using T = decltype(tag);
        switch (key) {
            case 401: return run_adj_tma<T, 4, 1>(ta, st);
            case 404: return run_adj_tma<T, 4, 4>(ta, st);
            case 801: return run_adj_tma<T, 8, 1>(ta, st);
            case 802: return run_adj_tma<T, 8, 2>(ta, st);
            case 804: return run_adj_tma<T, 8, 4>(ta, st);
            case 808: return run_adj_tma<T, 8, 8>(ta, st);
            default: return SSM_ERR_UNSUPPORTED;
        }
    };
    switch (p->act_dtype) {
        case SSM_F32: return by(float{});
        case SSM_BF16: return by(__nv_bfloat16{});
        default: return by(__half{});
    }
}

int bwd_tma(const ssm_selective_scan_params* p, const Cfg& c, const Args& a, cudaStream_t st) {
    if (!tma_ok(p, c, true)) return SSM_ERR_UNSUPPORTED;
    if (int s = ensure_context("selective_scan bwd (TMA)")) return s;
    const int cpc = 32 / c.lpc * kWarps, np = c.npt * c.lpc;
    TmaArgs ta;
    ta.a = a;
    const bool z = p->flags & SSM_HAS_Z;
    if (int s = encode_act(&ta.m_u, p->u, p, cpc)) return s;
    if (int s = encode_act(&ta.m_d, p->delta, p, cpc)) return s;
    if (int s = encode_act(&ta.m_z, z ? p->z : p->u, p, cpc)) return s;
    if (int s = encode_act(&ta.m_g, p->dout, p, cpc)) return s;
    const void* ys = reinterpret_cast<const char*>(p->checkpoints) + a.ysave_off;
    if (int s = encode_act(&ta.m_ys, (z && !a.lean) ? ys : p->u, p, cpc)) return s;
    if (int s = encode_bc(&ta.m_B, p->B, p, np)) return s;
    if (int s = encode_bc(&ta.m_C, p->C, p, np)) return s;
    if (int s = encode_act(&ta.m_o0, p->du, p, cpc)) return s;
    if (int s = encode_act(&ta.m_o1, p->ddelta, p, cpc)) return s;
    if (int s = encode_act(&ta.m_o2, z ? p->dz : p->du, p, cpc)) return s;
    switch (p->act_dtype) {
        case SSM_F32: return dispatch_bwd_tma<float>(c, ta, st);
        case SSM_BF16: return dispatch_bwd_tma<__nv_bfloat16>(c, ta, st);
        default: return dispatch_bwd_tma<__half>(c, ta, st);
    }
}

}  // namespace sscan
}  // namespace ssm

// the TMA scan kernels' flag, read (and cleared) by ssm_take_kernel_error
int ssm_scan_take_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, ssm::sscan::g_scan_error, sizeof(int)) != cudaSuccess) return -1;
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(ssm::sscan::g_scan_error, &zero, sizeof(int));
    }
    return v;
}
