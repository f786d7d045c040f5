// The TMA-staged selective-scan backward for dstate 16 with two channels per
// thread (included by selective_scan_tma.cu, which defines the tensor-copy
// helpers, TmaArgs and BwdTmaLayout).
//
// Thread mapping: lane = 4 * pg + sub.  The lane holds states 4 sub .. 4 sub + 3
// of the two channels c0 = 16 warp + 2 pg and c0 + 1 (a "channel pair"); the
// four lanes of a pair group hold all 16 states of both.  Compared with one
// channel of 8 states per lane (bwd_tma_kernel<T, 8, 2>):
//  * dB[t][n] and dC[t][n] (sums over the CTA's channels) are first summed over
//    the lane's two channels in registers, so the butterfly reduce-scatter over
//    the warp runs on 4 values and 3 lane levels instead of 8 values and 4
//    levels: half the shuffles;
//  * each step reads 4 states of B and C per lane (one 16-byte shared load each)
//    instead of 8;
//  * the per-channel sums over states (sum_n dh B and sum_n dh a x A, which
//    give du and ddelta) run over 4 lanes instead of 2.  Lanes with sub >= 2
//    keep the pair's channels in swapped order (their "first" channel is
//    c0 + 1), so the first level of that reduction sends one channel's sums
//    and keeps the other's with no select.
// Every per-element formula and the order of every per-channel recurrence are
// those of bwd_tma_kernel, except that dh a x_prev is formed as (dh a) x_prev
// from the carried adjoint dh a (one multiply fewer), and that the per-step
// scalar kept is delta' log2 e (the value the forward rounded its decays
// from) instead of delta': dA accumulates in log2 e units and is scaled back
// once, and du takes delta' as (delta' log2 e) ln 2.  These and the
// cross-channel and cross-state sums, which associate differently, make dA,
// dB, dC, du and ddelta differ from it in the last bits.
#pragma once

template <typename T, bool LEAN>
__global__ void __launch_bounds__(kThreads, 3)
bwd2_tma_kernel(const __grid_constant__ TmaArgs ta) {
    const Args& a = ta.a;
    constexpr int NPT = 4;               // states per channel per lane
    constexpr int CPW = 16;              // channels per warp
    constexpr int CPC = CPW * kWarps;
    constexpr int NP = 16;
    constexpr int K = kChunk;
    constexpr int FS = K + 1;
    constexpr int TS = kTS;
    constexpr int NPW = NP + 1;
    constexpr int HALF = K / 2;
    using Sc = Scatter<NPT, 2>;          // the reduce-scatter over lane bits 4, 3, 2
    using Lay = BwdTmaLayout<T, CPC, NP, 8>;   // 8 floats of saved state per lane, as NPT 8
    static_assert(Sc::kept() == 1 && K == 16 && TS == 4, "launch shape");

    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((128u - (tc::smem_u32(smem_raw) & 127u)) & 127u);
    float2* dvu = reinterpret_cast<float2*>(smem + Lay::o_dvu);   // (delta' log2 e, delta'*u)
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
    const int pg = lane >> 2, sub = lane & 3;
    const int sw = sub >> 1;                                      // 1: the pair is held swapped
    const int cf = warp * CPW + 2 * pg + sw, cs = warp * CPW + 2 * pg + 1 - sw;   // first, second channel
    const int64_t ct = blockIdx.x % a.nct, seg = blockIdx.x / a.nct, g = blockIdx.y, b = blockIdx.z;
    const int64_t dl0 = ct * CPC;
    const int rows = (int)min64(CPC, a.per_group - dl0);
    const int64_t d0 = g * a.per_group + dl0;
    const int cc2[2] = {cf, cs};
    const bool cvalid[2] = {cf < rows, cs < rows};
    const int64_t N = a.dstate, L = a.length;
    const bool has_d = a.flags & SSM_HAS_D, has_z = a.flags & SSM_HAS_Z;
    const bool has_bias = a.flags & SSM_HAS_BIAS, softplus = a.flags & SSM_SOFTPLUS;
    const int64_t bg = b * a.groups + g;
    const int64_t bs = b * a.nseg + seg;
    const int pm = Sc::mask(lane);
    const bool own = Sc::owner(lane);
    const float* Bp = Bs + pm * CS + sub * NPT;
    const float* Cp = Cs + pm * CS + sub * NPT;
    const uint32_t tx = (uint32_t)((has_z ? (LEAN ? 4 : 5) : 3) * CPC * K * sizeof(T) + 2 * NP * K * sizeof(T));
    // du / ddelta sums: after the two lane levels this lane holds channel cf's
    // sum_n dh B (sub even) or sum_n dh a x A (sub odd)
    float* const wsum = (sub & 1) ? dda : dua;

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

    // saved states: a two-slot ring, [slot][channel slot (first, second)][tid]
    // float4 (the lane's 4 states of that channel), filled one sub-block (LEAN:
    // one chunk) ahead.  Each warp copies its own 16 channels' states, 512
    // contiguous bytes per copy instruction, into the slots of the lanes that
    // use them; a __syncwarp follows each wait and precedes each refill.
    const int last_len = (int)min64(K, L - (tile_hi - 1) * K);
    const int64_t s_first = LEAN ? tile_hi - 1 : (tile_hi - 1) * (K / TS) + (last_len + TS - 1) / TS - 1;
    int nleft = (int)(s_first - (LEAN ? tile_lo : tile_lo * (K / TS)));   // saved states still to fetch
    int slot = 0;
    const float* ckp = a.ckpt + ((b * a.nsub + s_first) * a.dim + d0) * N;   // the CTA's first channel
    auto fetch = [&](int sl) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int k = q * 32 + lane;
            const int cwk = k >> 2, pc = k & 3;              // channel in the warp, its 16-byte piece
            const int user = 4 * (cwk >> 1) + pc;            // the lane holding those states
            const int qs = (cwk & 1) ^ (pc >> 1);            // ... in its first or second channel slot
            const int ch = warp * CPW + cwk;
            const uint32_t dst = tc::smem_u32(sck + (((size_t)sl * 2 + qs) * kThreads + warp * 32 + user) * 4);
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
    // per channel slot e (first, second): slot j of a pair holds states
    // 4 sub + ((2j) ^ pm), 4 sub + ((2j + 1) ^ pm)
    float2 An2[2][2], q2[2][2], dA2[2][2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const int64_t d = d0 + cc2[e];
        const int64_t sx = (bs * a.dim + d) * N;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int n0 = sub * NPT + ((2 * j) ^ pm), n1 = sub * NPT + ((2 * j + 1) ^ pm);
            An2[e][j] = cvalid[e] ? make_float2(a.A[d * N + n0], a.A[d * N + n1]) : make_float2(0.0f, 0.0f);
            q2[e][j] = (a.nseg > 1 && cvalid[e]) ? make_float2(a.seg_x[sx + n0], a.seg_x[sx + n1])
                                                 : make_float2(0.0f, 0.0f);
            dA2[e][j] = make_float2(0.0f, 0.0f);
        }
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
                report(a, 73);
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

        // phase 0: per-step scalars, two steps per item as paired lanes
#pragma unroll
        for (int k = 0; k < CPC / 16; ++k) {
            const int cc = (tid >> 3) + 16 * k, t = 2 * (tid & 7);
            const float2 dr = Io2<T>::ld(&rd[cc * K + t]);
            const float2 ur = Io2<T>::ld(&ru[cc * K + t]);
            float2 go = Io2<T>::ld(&rg[cc * K + t]);
            float2 dv = add2(dr, f2(bch[cc]));
            if (softplus) dv = softplus2_fast(dv);
            const float2 du = mul2(dv, ur);
            const float2 dl = mul2(dv, f2(kLog2e));   // the forward's rounding of delta' log2 e
            dvu[cc * FS + t] = make_float2(dl.x, du.x);
            dvu[cc * FS + t + 1] = make_float2(dl.y, du.y);
            if (has_z) {
                const float2 zr = Io2<T>::ld(&rz[cc * K + t]);
                go = mul2(go, mul2(zr, sigmoid2_t<T>(zr)));
            }
            gs[cc * FS + t] = go.x;
            gs[cc * FS + t + 1] = go.y;
        }
        // B/C as fp32 [t][n], in the four within-float4 orders (n & 3) ^ p
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
            float2 x2[2][2];
            float2 x8[2][2], x4[2][2];        // LEAN, full chunk: the states entering steps 2 TS and TS
            const float2* vr[2] = {dvu + cf * FS, dvu + cs * FS};
            const float* gr[2] = {gs + cf * FS, gs + cs * FS};
            // the lane's saved states of channel slot e, in its permuted order
            auto load_states = [&](int sl) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const float* src = sck + (((size_t)sl * 2 + e) * kThreads + tid) * 4;
#pragma unroll
                    for (int j = 0; j < 2; ++j)
                        x2[e][j] = make_float2(src[(2 * j) ^ pm], src[(2 * j + 1) ^ pm]);
                }
            };
            // one step of the forward recurrence for both channels
            auto replay = [&](int t) {
                const float4 bq = *reinterpret_cast<const float4*>(Bp + t * NP);
                const float2 bb[2] = {make_float2(bq.x, bq.y), make_float2(bq.z, bq.w)};
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const float2 v = vr[e][t];
                    const float dl = v.x;
                    const float2 dl2 = make_float2(dl, dl), du2 = make_float2(v.y, v.y);
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const float2 ar = __fmul2_rn(dl2, An2[e][j]);
                        const float2 ex = make_float2(exp2_mufu(ar.x), exp2_mufu(ar.y));
                        x2[e][j] = __ffma2_rn(ex, x2[e][j], __fmul2_rn(du2, bb[j]));
                    }
                }
            };
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
                    // sb; in a full chunk the state at step 2 TS, passed on the way to
                    // the last sub-block, is kept for the one before it (4 TS replayed
                    // steps per chunk instead of 6 TS)
                    if (FULL && (sb == 2 || sb == 1)) {
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            x2[e][0] = sb == 2 ? x8[e][0] : x4[e][0];
                            x2[e][1] = sb == 2 ? x8[e][1] : x4[e][1];
                        }
                    } else {
                        load_states(cslot);
                        for (int pb = 0; pb < sb; ++pb) {
#pragma unroll
                            for (int jj = 0; jj < TS; ++jj) replay(pb * TS + jj);
                            if (FULL && pb <= 1) {
#pragma unroll
                                for (int e = 0; e < 2; ++e) {
                                    if (pb == 0) { x4[e][0] = x2[e][0]; x4[e][1] = x2[e][1]; }
                                    else { x8[e][0] = x2[e][0]; x8[e][1] = x2[e][1]; }
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
                    load_states(slot);
                    slot ^= 1;
                }
                // the replay keeps the states entering each step; the adjoint
                // recomputes each step's decays
                float2 xh[TS][2][2];
#pragma unroll
                for (int jj = 0; jj < TS; ++jj) {
                    if (FULL || jj < nb) {
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            xh[jj][e][0] = x2[e][0];
                            xh[jj][e][1] = x2[e][1];
                        }
                        replay(tb + jj);
                        if (LEAN && has_z) {   // the scan output <x_t, C_t> of this step, for dz
                            const float4 cq = *reinterpret_cast<const float4*>(Cp + (tb + jj) * NP);
                            float ys[2];
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                float2 acc = __fmul2_rn(x2[e][0], make_float2(cq.x, cq.y));
                                acc = __ffma2_rn(x2[e][1], make_float2(cq.z, cq.w), acc);
                                ys[e] = acc.x + acc.y;
                            }
                            ys[0] += __shfl_xor_sync(0xffffffffu, ys[1], 2);
                            ys[0] += __shfl_xor_sync(0xffffffffu, ys[0], 1);
                            if ((sub & 1) == 0) stf(&ryw[cf * K + tb + jj], ys[0]);
                        }
                    }
                }
#pragma unroll
                for (int jj = TS - 1; jj >= 0; --jj) {
                    if (FULL || jj < nb) {
                        const int t = tb + jj;
                        const float4 bq = *reinterpret_cast<const float4*>(Bp + t * NP);
                        const float4 cq = *reinterpret_cast<const float4*>(Cp + t * NP);
                        const float2 bb[2] = {make_float2(bq.x, bq.y), make_float2(bq.z, bq.w)};
                        const float2 cc[2] = {make_float2(cq.x, cq.y), make_float2(cq.z, cq.w)};
                        const bool last = FULL ? (jj == TS - 1) : (jj == nb - 1);
                        float2 wb[2], wc[2];          // channel-summed dB / dC terms of the lane's states
                        float su[2], sd[2];           // per channel: sum over the lane's states
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const float2 v = vr[e][t];
                            const float gv = gr[e][t];
                            const float2 g2 = make_float2(gv, gv);
                            const float2 du2 = make_float2(v.y, v.y);
                            const float2 dlr2 = make_float2(v.x, v.x);   // delta' log2 e
                            float2 dua2 = make_float2(0.0f, 0.0f), dda2 = make_float2(0.0f, 0.0f);
#pragma unroll
                            for (int j = 0; j < 2; ++j) {
                                const float2 ar = __fmul2_rn(dlr2, An2[e][j]);
                                const float2 aj = make_float2(exp2_mufu(ar.x), exp2_mufu(ar.y));
                                const float2 dh = __ffma2_rn(g2, cc[j], q2[e][j]);
                                q2[e][j] = __fmul2_rn(dh, aj);
                                // dh a x_prev, as (dh a) x_prev: the carried adjoint times the state
                                const float2 tmp = __fmul2_rn(q2[e][j], xh[jj][e][j]);
                                dda2 = __ffma2_rn(tmp, An2[e][j], dda2);
                                dA2[e][j] = __ffma2_rn(tmp, dlr2, dA2[e][j]);   // in log2 e units
                                dua2 = __ffma2_rn(dh, bb[j], dua2);
                                wb[j] = e == 0 ? __fmul2_rn(dh, du2) : __ffma2_rn(dh, du2, wb[j]);
                                // the state after step t: the next step's entering state
                                const float2 xt = (jj + 1 < TS && !last) ? xh[jj + 1 < TS ? jj + 1 : jj][e][j] : x2[e][j];
                                wc[j] = e == 0 ? __fmul2_rn(g2, xt) : __ffma2_rn(g2, xt, wc[j]);
                            }
                            su[e] = dua2.x + dua2.y;
                            sd[e] = dda2.x + dda2.y;
                        }
                        // du / ddelta sums over the pair group's 4 lanes: keep the
                        // first channel's, send the second's (the partner holds
                        // them the other way round), then an all-reduce
                        su[0] += __shfl_xor_sync(0xffffffffu, su[1], 2);
                        sd[0] += __shfl_xor_sync(0xffffffffu, sd[1], 2);
                        su[0] += __shfl_xor_sync(0xffffffffu, su[0], 1);
                        sd[0] += __shfl_xor_sync(0xffffffffu, sd[0], 1);
                        float w[NPT] = {wb[0].x, wb[0].y, wb[1].x, wb[1].y};
                        Sc::reduce(w);
                        if (own) dBw[(warp * K + t) * NPW + sub * NPT + pm] = w[0];
                        float w2[NPT] = {wc[0].x, wc[0].y, wc[1].x, wc[1].y};
                        Sc::reduce(w2);
                        if (own) dCw[(warp * K + t) * NPW + sub * NPT + pm] = w2[0];
                        wsum[cf * FS + t] = (sub & 1) ? sd[0] : su[0];
                    }
                }
            }
        };
        if (len == K) chunk_body(std::true_type{});
        else chunk_body(std::false_type{});
        __syncthreads();

        // phase C: element-wise gradients (two steps per item as paired lanes),
        // written over the tiles they came from, then tensor stores
#pragma unroll
        for (int k = 0; k < CPC / 16; ++k) {
            const int cc = (tid >> 3) + 16 * k, t = 2 * (tid & 7);
            const int i = tid + kThreads * k;
            const float2 ur = Io2<T>::ld(&ru[cc * K + t]);
            const float Dv = Dch[cc];
            const float2 dv = mul2(make_float2(dvu[cc * FS + t].x, dvu[cc * FS + t + 1].x), f2(kLn2));
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

#pragma unroll
    for (int e = 0; e < 2; ++e) {
        if (!cvalid[e]) continue;
        float* dap = a.dA_part + (bs * a.dim + d0 + cc2[e]) * N;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float2 v = mul2(dA2[e][j], f2(kLn2));   // back from log2 e units
            dap[sub * NPT + ((2 * j) ^ pm)] = v.x;
            dap[sub * NPT + ((2 * j + 1) ^ pm)] = v.y;
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
