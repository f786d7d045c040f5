// Shared device/host helpers for the sm_100a SSM-scan kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <string>

#include "ssm_b200.h"

namespace ssm {

// ---------------------------------------------------------------- errors ----
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int check_launch(const char* what);
// Make the current device's primary context current on the calling thread
// (through the runtime) before a driver-API call that needs one, such as
// cuTensorMapEncodeTiled.  A thread whose first CUDA call is into this library
// -- torch runs backward passes on its own autograd thread -- has none yet.
int ensure_context(const char* what);

// ------------------------------------------------------------ dtype I/O ----
template <typename T> struct Io;
template <> struct Io<float> {
    static __device__ __forceinline__ float ld(const float* p) { return *p; }
    static __device__ __forceinline__ void st(float* p, float v) { *p = v; }
};
template <> struct Io<__nv_bfloat16> {
    static __device__ __forceinline__ float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
    static __device__ __forceinline__ void st(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};
template <> struct Io<__half> {
    static __device__ __forceinline__ float ld(const __half* p) { return __half2float(*p); }
    static __device__ __forceinline__ void st(__half* p, float v) { *p = __float2half_rn(v); }
};

template <typename T> __device__ __forceinline__ float ldf(const T* p) { return Io<T>::ld(p); }
template <typename T> __device__ __forceinline__ void stf(T* p, float v) { Io<T>::st(p, v); }

// Runtime-typed scalar load, for the small or cold operands (B/C staging).
__device__ __forceinline__ float ld_any(const void* base, int64_t i, int dtype) {
    if (dtype == SSM_F32) return reinterpret_cast<const float*>(base)[i];
    if (dtype == SSM_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
    return __half2float(reinterpret_cast<const __half*>(base)[i]);
}
__device__ __forceinline__ void st_any(void* base, int64_t i, int dtype, float v) {
    if (dtype == SSM_F32) reinterpret_cast<float*>(base)[i] = v;
    else if (dtype == SSM_BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half*>(base)[i] = __float2half_rn(v);
}

// ----------------------------------------------------------------- math ----
// 2^x on the MUFU pipe (PTX ex2.approx: ~2 ulp in fp32, flushes subnormals).
__device__ __forceinline__ float exp2_mufu(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;     // 1 / log2(e)

// torch.nn.functional.softplus with its default threshold: x > 20 -> x.
__device__ __forceinline__ float softplus_f(float x) {
    return x > 20.0f ? x : log1pf(expf(x));
}
// d softplus / dx, matching torch's backward (1 above the threshold).
__device__ __forceinline__ float softplus_grad_f(float x) {
    return x > 20.0f ? 1.0f : 1.0f / (1.0f + expf(-x));
}
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

// 1/x on the MUFU pipe (PTX rcp.approx: max error 2^-23 on [1, 2]).
__device__ __forceinline__ float rcp_mufu(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// sigmoid(x) = 1 / (1 + 2^(-x log2 e)): two MUFU ops, ~3e-7 relative error.
__device__ __forceinline__ float sigmoid_fast(float x) {
    return rcp_mufu(1.0f + exp2_mufu(-x * kLog2e));
}

// softplus(x) = max(x, 0) + log1p(exp(-|x|)), with torch's threshold rule
// (x > 20 returns x).  log1p(s) for s = exp(-|x|) in (0, 1] comes from the
// area-hyperbolic-tangent series
//   log(1 + s) = 2 artanh(w) = 2 (w + w^3/3 + w^5/5 + ...),  w = s / (2 + s) <= 1/3,
// truncated after the w^15 term (relative truncation error < 2e-9), so it keeps
// full relative accuracy for tiny s where log(1 + s) would lose it.  Every
// rounding step is an explicit intrinsic, so the paired form below rounds each
// lane exactly as this one does (no compiler contraction can differ between
// them).  Two MUFU ops and ~14 FMA-pipe instructions.
__device__ __forceinline__ float softplus_fast(float x) {
    const float e = exp2_mufu(__fmul_rn(-fabsf(x), kLog2e));
    const float w = __fmul_rn(e, rcp_mufu(__fadd_rn(2.0f, e)));
    const float w2 = __fmul_rn(w, w);
    float p = 1.0f / 15.0f;
    p = __fmaf_rn(p, w2, 1.0f / 13.0f);
    p = __fmaf_rn(p, w2, 1.0f / 11.0f);
    p = __fmaf_rn(p, w2, 1.0f / 9.0f);
    p = __fmaf_rn(p, w2, 1.0f / 7.0f);
    p = __fmaf_rn(p, w2, 1.0f / 5.0f);
    p = __fmaf_rn(p, w2, 1.0f / 3.0f);
    p = __fmaf_rn(p, w2, 1.0f);
    const float r = __fmaf_rn(__fadd_rn(w, w), p, fmaxf(x, 0.0f));
    return x > 20.0f ? x : r;
}
// d softplus / dx (torch's backward: 1 above the threshold).
__device__ __forceinline__ float softplus_grad_fast(float x) {
    return x > 20.0f ? 1.0f : sigmoid_fast(x);
}

// Sigmoid / SiLU / SiLU' chosen by the storage type T of the data they serve,
// no IEEE division.  fp32 data: sigmoid = rcp(1 + ex2(-a log2 e)) (two MUFU
// ops, ~3e-7 relative).  16-bit data, whose results are rounded to 8 or 11
// bits: sigmoid = (1 + tanh(a/2)) / 2 with PTX tanh.approx (one MUFU op,
// ~2^-11 relative), for kernels that are otherwise issue-bound.
__device__ __forceinline__ float tanh_mufu(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
template <typename T>
__device__ __forceinline__ float sigmoid_t(float a) {
    if constexpr (sizeof(T) == 4) return sigmoid_fast(a);
    else return fmaf(0.5f, tanh_mufu(0.5f * a), 0.5f);
}
template <typename T>
__device__ __forceinline__ float silu_t(float a) {
    if constexpr (sizeof(T) == 4) return a * sigmoid_fast(a);
    else {
        const float h = 0.5f * a;
        return fmaf(h, tanh_mufu(h), h);
    }
}
template <typename T>
__device__ __forceinline__ float silu_grad_t(float a) {
    const float s = sigmoid_t<T>(a);
    return s * fmaf(a, 1.0f - s, 1.0f);
}

// ---------------------------------------------------------- paired fp32 ----
// Two independent fp32 lanes per instruction (the sm_100 paired FMA / MUL /
// ADD): each lane is rounded exactly as the scalar fmaf, * or + rounds it, so a
// kernel that carries two independent element streams as the .x / .y of a
// float2 halves its FMA-pipe instructions without changing a result.
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

// softplus_fast of two lanes, each rounded exactly as the scalar form rounds it.
__device__ __forceinline__ float2 softplus2_fast(float2 x) {
    const float2 e = make_float2(exp2_mufu(__fmul_rn(-fabsf(x.x), kLog2e)),
                                 exp2_mufu(__fmul_rn(-fabsf(x.y), kLog2e)));
    const float2 den = add2(f2(2.0f), e);
    const float2 w = mul2(e, make_float2(rcp_mufu(den.x), rcp_mufu(den.y)));
    const float2 w2 = mul2(w, w);
    float2 p = f2(1.0f / 15.0f);
    p = fma2(p, w2, f2(1.0f / 13.0f));
    p = fma2(p, w2, f2(1.0f / 11.0f));
    p = fma2(p, w2, f2(1.0f / 9.0f));
    p = fma2(p, w2, f2(1.0f / 7.0f));
    p = fma2(p, w2, f2(1.0f / 5.0f));
    p = fma2(p, w2, f2(1.0f / 3.0f));
    p = fma2(p, w2, f2(1.0f));
    const float2 r = fma2(add2(w, w), p, make_float2(fmaxf(x.x, 0.0f), fmaxf(x.y, 0.0f)));
    return make_float2(x.x > 20.0f ? x.x : r.x, x.y > 20.0f ? x.y : r.y);
}

// sigmoid_t<T> of two lanes, each rounded exactly as the scalar form rounds it.
template <typename T>
__device__ __forceinline__ float2 sigmoid2_t(float2 a) {
    if constexpr (sizeof(T) == 4) {
        const float2 m = mul2(a, f2(-kLog2e));
        const float2 d = add2(f2(1.0f), make_float2(exp2_mufu(m.x), exp2_mufu(m.y)));
        return make_float2(rcp_mufu(d.x), rcp_mufu(d.y));
    } else {
        const float2 h = mul2(a, f2(0.5f));
        return fma2(f2(0.5f), make_float2(tanh_mufu(h.x), tanh_mufu(h.y)), f2(0.5f));
    }
}

// SiLU of two pre-activations given as halves hp = a / 2 (an exact power-of-two
// scaling): the values silu_t<T>(a) returns.
template <typename T>
__device__ __forceinline__ float2 silu2_half(float2 hp) {
    if constexpr (sizeof(T) == 4) {
        const float2 m = mul2(hp, f2(-2.0f * kLog2e));
        const float2 d = add2(make_float2(exp2_mufu(m.x), exp2_mufu(m.y)), f2(1.0f));
        return mul2(add2(hp, hp), make_float2(rcp_mufu(d.x), rcp_mufu(d.y)));
    } else {
        return fma2(hp, make_float2(tanh_mufu(hp.x), tanh_mufu(hp.y)), hp);
    }
}

// 2 g silu'(a) for two lanes from hp = a / 2, with silu'(a) = s (1 + a (1 - s)).
// 16-bit data: s = (1 + t) / 2 with t = tanh(hp), so the doubled gradient is
// g (1 + t) (1 + hp (1 - t)).  fp32 data: s = rcp(1 + 2^(-a log2 e)).
template <typename T>
__device__ __forceinline__ float2 silu_grad2_half(float2 hp, float2 g) {
    if constexpr (sizeof(T) == 4) {
        const float2 m = mul2(hp, f2(-2.0f * kLog2e));
        const float2 d = add2(make_float2(exp2_mufu(m.x), exp2_mufu(m.y)), f2(1.0f));
        const float2 s = make_float2(rcp_mufu(d.x), rcp_mufu(d.y));
        const float2 q = fma2(add2(hp, hp), fma2(s, f2(-1.0f), f2(1.0f)), f2(1.0f));
        return mul2(add2(g, g), mul2(s, q));
    } else {
        const float2 t = make_float2(tanh_mufu(hp.x), tanh_mufu(hp.y));
        const float2 q = fma2(hp, fma2(t, f2(-1.0f), f2(1.0f)), f2(1.0f));
        return mul2(mul2(g, add2(t, f2(1.0f))), q);
    }
}

// paired loads/stores of two consecutive elements as float2
template <typename T> struct Io2;
template <> struct Io2<float> {
    static __device__ __forceinline__ float2 ld(const float* p) { return *reinterpret_cast<const float2*>(p); }
    static __device__ __forceinline__ void st(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }
};
template <> struct Io2<__nv_bfloat16> {
    static __device__ __forceinline__ float2 ld(const __nv_bfloat16* p) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    }
    static __device__ __forceinline__ void st(__nv_bfloat16* p, float2 v) {
        *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v.x, v.y);
    }
};
template <> struct Io2<__half> {
    static __device__ __forceinline__ float2 ld(const __half* p) {
        return __half22float2(*reinterpret_cast<const __half2*>(p));
    }
    static __device__ __forceinline__ void st(__half* p, float2 v) {
        *reinterpret_cast<__half2*>(p) = __floats2half2_rn(v.x, v.y);
    }
};

// ---------------------------------------------------------- warp reduce ----
template <int WIDTH>
__device__ __forceinline__ float sum_low_lanes(float v) {
    // Sum over the WIDTH consecutive lanes sharing lane / WIDTH (WIDTH a power of two).
#pragma unroll
    for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace ssm
