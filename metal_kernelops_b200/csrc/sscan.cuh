// Definitions shared by the selective-scan kernels: the plain-staging kernels
// of selective_scan.cu (every shape and dtype) and the TMA-staged kernels of
// selective_scan_tma.cu (16-byte aligned rows, one dtype for activations and
// B/C, one full state tile per lane group).
#pragma once

#include "common.cuh"

namespace ssm {
namespace sscan {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kChunk = 16;  // backward chunk (staged tile, walked in reverse)
constexpr int kFT = 16;     // forward tile
constexpr int kTS = 4;      // backward sub-block == interval of the saved states

struct Args {
    int64_t batch, dim, length, groups, dstate, per_group;
    int64_t nchunks;      // ceil(length / kChunk)
    int64_t nct;          // channel tiles per group
    // Sequence segments: blockIdx.x = segment * nct + channel tile.  With
    // nseg > 1 every segment of seg_chunks chunks runs as its own CTA, starting
    // from the state (forward) or adjoint (backward) that a summary pass and a
    // combine over segments left in seg_x: (batch, nseg, dim, dstate) fp32.
    int64_t nseg, seg_chunks;
    float* seg_x;
    float* seg_p;         // decay product over each segment, same layout
    uint32_t flags;
    int bc_dtype;
    bool fast;            // 16-byte aligned rows: asynchronous copies allowed
    const void* u; const void* delta; const float* A; const void* B; const void* C;
    const float* D; const void* z; const float* delta_bias;
    void* y; float* ckpt;
    int64_t nsub;         // sub-checkpoints per row: nchunks * kChunk / kTS
    int64_t ck_stride;    // floats between consecutive sub-checkpoints of a row: dim * dstate
    int ck_every;         // steps between saved states: kTS, or kChunk in the lean mode
    bool lean;            // SSM_SCAN_LEAN: states every chunk, no saved scan output
    int64_t ysave_off;    // bytes from ckpt to the saved scan output (activation dtype)
    const void* dout; void* du; void* ddelta; void* dz;
    float* dB_part; float* dC_part;   // (batch*groups*nct, dstate, length)
    float* dA_part;                   // (batch, dim, dstate)
    float* dD_part; float* db_part;   // (batch, dim)
    int* status;                      // the call's optional status word (params.status)
};

// The cross-channel sums dB[t][n] and dC[t][n] are butterfly reduce-scatters
// over the lanes that hold the same states of different channels (lane bits
// [LO, 5)).  Each lane stores its NPT states in a lane-dependent order -- slot
// i holds state (i XOR mask) -- chosen so that at every level both partners
// keep the LOWER half of their slots and send the upper half: a level is then
// one shuffle and one add per value, with no selects.  After the scatter
// levels slot i < kept holds the full sum for state (i + mask); the remaining
// levels (past log2(NPT)) are plain all-reduces, and `owner` marks the one
// lane of each duplicate set that writes.
template <int V, int LO>
struct Scatter {
    static constexpr int kept() {
        int cur = V;
        for (int bit = 4; bit >= LO; --bit)
            if (cur > 1) cur /= 2;
        return cur;
    }
    static __device__ __forceinline__ int mask(int lane) {
        int m = 0, cur = V;
#pragma unroll
        for (int bit = 4; bit >= LO; --bit) {
            if (cur > 1) {
                cur /= 2;
                if ((lane >> bit) & 1) m |= cur;
            }
        }
        return m;
    }
    static __device__ __forceinline__ bool owner(int lane) {
        int cur = V;
        bool own = true;
#pragma unroll
        for (int bit = 4; bit >= LO; --bit) {
            if (cur > 1) cur /= 2;
            else if ((lane >> bit) & 1) own = false;
        }
        return own;
    }
    // Levels that keep two or more values add them in pairs with one paired
    // fp32 add (each lane rounds exactly as the scalar add).
    static __device__ __forceinline__ void reduce(float (&v)[V]) {
        int cur = V;
#pragma unroll
        for (int bit = 4; bit >= LO; --bit) {
            const int o = 1 << bit;
            if (cur > 1) {
                const int h = cur / 2;
                if (h >= 2) {
#pragma unroll
                    for (int i = 0; i < V / 2; i += 2)
                        if (i + 1 < h) {
                            const float2 r = make_float2(__shfl_xor_sync(0xffffffffu, v[h + i], o),
                                                         __shfl_xor_sync(0xffffffffu, v[h + i + 1], o));
                            const float2 s = __fadd2_rn(make_float2(v[i], v[i + 1]), r);
                            v[i] = s.x;
                            v[i + 1] = s.y;
                        }
                } else {
                    v[0] += __shfl_xor_sync(0xffffffffu, v[1], o);
                }
                cur = h;
            } else {
                v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
            }
        }
    }
};

// Launch shape: states per thread and lanes per channel.
struct Cfg { int npt = 4, lpc = 4; };   // dstate > 64 is refused before use

// The TMA-staged kernels (selective_scan_tma.cu).  Each returns SSM_OK after
// launching, SSM_ERR_UNSUPPORTED (nothing launched, no error recorded) when the
// problem does not meet the TMA path's layout conditions, or another status
// on a CUDA failure.  The forward launches only the main pass (the segment
// summary and combine passes, when nseg > 1, are the caller's).
int fwd_tma(const ssm_selective_scan_params* p, const Cfg& c, const Args& a, cudaStream_t st);
int fwd_sum_tma(const ssm_selective_scan_params* p, const Cfg& c, const Args& a, cudaStream_t st);
int bwd_tma(const ssm_selective_scan_params* p, const Cfg& c, const Args& a, cudaStream_t st);
int bwd_sum_tma(const ssm_selective_scan_params* p, const Cfg& c, const Args& a, cudaStream_t st);

}  // namespace sscan
}  // namespace ssm
