// Thin wrappers over the sm_100a fifth-generation tensor-core instructions
// (tcgen05.*), mbarriers and the shared-memory operand layout they read.
//
// Operand tiles live in shared memory in the "no swizzle" canonical layout:
// the tile is an array of 128-byte core matrices, each holding 8 rows of 16
// bytes (8 bf16/f16 values).  A tile with R rows of W 16-byte chunks stores
// chunk c of row r at
//
//     tile_off(r, c, W) = ((r / 8) * W + c) * 128 + (r % 8) * 16
//
// so a 16-byte global load lands in one 16-byte shared store.  The same tile
// can feed the tensor core in two ways:
//   * K-major: rows are the M (or N) index, chunks run along K.
//       leading offset (next 8 K values)  = 128 bytes
//       stride offset  (next 8 rows)      = W * 128 bytes
//   * MN-major: rows are the K index, chunks run along M (or N).
//       leading offset (next 8 K rows)    = W * 128 bytes
//       stride offset  (next 8 M/N values)= 128 bytes
// One MMA instruction consumes K = 16: two core matrices along K.
//
// Accumulators live in tensor memory (TMEM).  For M = 128 with one CTA, row m
// of the accumulator is TMEM lane m and column n is TMEM column base + n; warp
// w of a warpgroup may only touch lanes 32 (w % 4) ... 32 (w % 4) + 31.
#pragma once

#include <cstdint>

namespace ssm {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__host__ __device__ constexpr uint32_t tile_off(uint32_t r, uint32_t c, uint32_t W) {
    return ((r >> 3) * W + c) * 128u + (r & 7u) * 16u;
}

// Shared-memory matrix descriptor, no swizzle (layout type 0), version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}
// K-major view of a tile with W chunks per row, starting at K chunk kc.
__device__ __forceinline__ uint64_t desc_k(uint32_t tile, uint32_t W, uint32_t kc) {
    return sdesc(tile + kc * 128u, 128u, W * 128u);
}
// MN-major view of a tile with W chunks per row, starting at K row kr (multiple of 8).
__device__ __forceinline__ uint64_t desc_mn(uint32_t tile, uint32_t W, uint32_t kr) {
    return sdesc(tile + (kr >> 3) * W * 128u, W * 128u, 128u);
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
// bf16: fmt = 1, f16: fmt = 0.  a_mn / b_mn: operand is MN-major.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t fmt, uint32_t M, uint32_t N, bool a_mn, bool b_mn) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
           ((N >> 3) << 17) | ((M >> 4) << 24);
}

// D[tmem] (+)= A * B; issued by one thread.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        :: "r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accum));
}

// Arrive on an mbarrier once every previously issued MMA of this thread is done.
__device__ __forceinline__ void commit(uint32_t mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(mbar) : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Make this thread's generic-proxy shared-memory writes visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Whole warp: allocate ncols (power of two >= 32) TMEM columns; address to *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(dst_smem), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 16 columns: thread t of the warp gets columns [col, col+16) of lane 32w+t.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        :: "r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
           "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
           "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
           "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
           "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
           "r"(__float_as_uint(v[15]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The same wait, with the 16 registers a tmem_ld16 wrote passed through it: every
// use of them is ordered after the wait (the plain wait carries no dependency).
__device__ __forceinline__ void tmem_wait_ld(float* v) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]),
                   "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15])
                 :: "memory");
}
// Pin registers written by an earlier tcgen05.ld behind a wait that already ran.
__device__ __forceinline__ void tmem_pin(float* v) {
    asm volatile(""
                 : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]),
                   "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15])
                 :: "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint32_t mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(mbar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// One try_wait, with a suspend-time hint of 64 ns: the thread sleeps at most
// that long before it polls again.  Without a hint (the system's own limit)
// warps were seen resuming 300 to 1,500 cycles after the phase completed; with
// it the SSD backward at BASELINE config 3 ran 3.28 -> 3.17 ms (hints of 20 and
// 200 ns: 3.19, 3.18; polling with test_wait: no gain).  A call still returns
// false after the hint, so the callers' iteration limits keep every wait bounded.
__device__ __forceinline__ bool mbar_try_wait(uint32_t mbar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred P1;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2, 64;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}\n"
        : "=r"(done) : "r"(mbar), "r"(parity) : "memory");
    return done != 0;
}
// One arrival on an mbarrier.
__device__ __forceinline__ void mbar_arrive(uint32_t mbar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(mbar) : "memory");
}
// Bounded wait for the phase with the given parity to complete.  Returns false
// (and leaves the barrier alone) when the iteration limit runs out.
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity, uint32_t limit = 1u << 22) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(mbar, parity)) return true;
    return false;
}

// ------------------------------------------------------------ TMA copies --
// Arrive on an mbarrier and add `bytes` to the transaction count its current
// phase waits for (the copies below retire those bytes).
__device__ __forceinline__ void mbar_expect_tx(uint32_t mbar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(mbar), "r"(bytes) : "memory");
}
// Tiled 5-D tensor load (one box) into the issuing CTA's own shared memory.
// The innermost coordinate must keep 16-byte alignment (every caller passes 0).
__device__ __forceinline__ void tma_load5(uint32_t dst, const void* map, int c0, int c1, int c2, int c3, int c4,
                                          uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
        :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(mbar)
        : "memory");
}
// Contiguous global -> shared copy of `bytes` (multiple of 16, both ends 16-byte aligned).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "l"(src), "r"(bytes), "r"(mbar) : "memory");
}

// ------------------------------------------------------------ async copies --
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(saddr), "l"(g) : "memory");
}
// Zero-fill variant: copies src_bytes (0 or 16) and fills the rest with zeros.
__device__ __forceinline__ void cp_async16_zfill(uint32_t saddr, const void* g, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(saddr), "l"(g), "r"(src_bytes) : "memory");
}
// 8-byte copy through L1 (the 16-byte .cg form bypasses it; .ca takes 4, 8 or 16).
__device__ __forceinline__ void cp_async8(uint32_t saddr, const void* g) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" :: "r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

}  // namespace tc
}  // namespace ssm
