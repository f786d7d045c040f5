// VMamba four-path 2D selective scan (ss2d) for sm_100a.
//
// Reference behaviour: src/metal_kernelops/cv/path_scan.py:546-576
// (`ss2d_scan`, `_PathScan` :383-543).  A (height, width) map is scanned along
// four paths -- row-major, column-major and their reverses -- with the Mamba-1
// recurrence, and the four outputs are added per pixel as (p0 + p2) + (p1 + p3)
// (cross-merge order of `ss2d_scan_reference`, :635-639), times 1 or 0.25.
//
// Design: the four paths become four blocks of channels (and of groups) of ONE
// Mamba-1 problem of 4 x channels rows over L = H*W steps, which the selective
// scan kernels (selective_scan.cu) run forward and backward unchanged; the
// reference's backward does the same with its scan kernels (:510-536).  Around
// them sit two kernels of this file:
//
//  * gather_kernel -- reads each (height, width) plane once, stages it in
//    shared memory (row pitch made odd so both the row-major and the
//    column-major reads are bank-conflict free) and writes the plane's four
//    path orders, every store coalesced.  Used for u, dt, B, C and dy.
//  * merge_kernel -- the inverse: for each output plane adds the four path
//    slices back at each pixel.  Paths 0 and 2 are read in place (coalesced);
//    paths 1 and 3 are added in column order into shared memory first (the
//    sum p1 + p3 at every pixel), then read transposed.
//
// The path orders need no index tables: step i of path 1 is pixel
// (i mod H, i div H), and paths 2/3 visit step i at L-1-i of paths 0/1.
#include <cstring>

#include "common.cuh"

namespace ssm {
namespace ss2d {

constexpr int kThreads = 256;
constexpr size_t kSmemLimit = 96 * 1024;   // planes above this read paths 1/3 from global

__host__ __device__ __forceinline__ int odd_pitch(int n) { return n | 1; }

// src: `planes` contiguous (H, W) planes; plane q = outer * per + inner.
// dst: stacked (outer, 4, per, L): path k of plane q at ((outer*4 + k)*per + inner)*L.
template <typename T, bool SMEM>
__global__ void __launch_bounds__(kThreads)
gather_kernel(const T* __restrict__ src, T* __restrict__ dst, int64_t planes, int64_t per,
              int H, int W, float scale) {
    extern __shared__ float plane[];
    const int L = H * W;
    const int pitch = odd_pitch(W);
    const int64_t ps = per * (int64_t)L;
    for (int64_t q = blockIdx.x; q < planes; q += gridDim.x) {
        const T* s = src + q * L;
        if (SMEM) {
            for (int i = threadIdx.x; i < L; i += kThreads) {
                const int h = i / W, w = i - h * W;
                plane[h * pitch + w] = ldf(s + i) * scale;
            }
            __syncthreads();
        }
        const int64_t outer = q / per, inner = q - outer * per;
        T* d = dst + (outer * 4 * per + inner) * (int64_t)L;
        for (int i = threadIdx.x; i < L; i += kThreads) {
            const int r = L - 1 - i;
            const int h0 = i / W, w0 = i - h0 * W;       // path 0: row-major step i
            const int w1 = i / H, h1 = i - w1 * H;       // path 1: column-major step i
            const int h2 = r / W, w2 = r - h2 * W;       // path 2: row-major step L-1-i
            const int w3 = r / H, h3 = r - w3 * H;       // path 3: column-major step L-1-i
            float v0, v1, v2, v3;
            if (SMEM) {
                v0 = plane[h0 * pitch + w0];
                v1 = plane[h1 * pitch + w1];
                v2 = plane[h2 * pitch + w2];
                v3 = plane[h3 * pitch + w3];
            } else {
                v0 = ldf(s + h0 * W + w0) * scale;
                v1 = ldf(s + h1 * W + w1) * scale;
                v2 = ldf(s + h2 * W + w2) * scale;
                v3 = ldf(s + h3 * W + w3) * scale;
            }
            stf(d + i, v0);
            stf(d + ps + i, v1);
            stf(d + 2 * ps + i, v2);
            stf(d + 3 * ps + i, v3);
        }
        if (SMEM) __syncthreads();
    }
}

// src: stacked (outer, 4, per, L) path slices; dst: (outer, per, H, W) planes.
// dst[p] = scale * ((s0[p] + s2[p]) + (s1[p] + s3[p])), s_k = path k at pixel p.
template <typename Tin, typename Tout, bool SMEM>
__global__ void __launch_bounds__(kThreads)
merge_kernel(const Tin* __restrict__ src, Tout* __restrict__ dst, int64_t planes, int64_t per,
             int H, int W, float scale) {
    extern __shared__ float cols[];              // [w][h], pitch odd_pitch(H): p1 + p3
    const int L = H * W;
    const int pitch = odd_pitch(H);
    const int64_t ps = per * (int64_t)L;
    for (int64_t q = blockIdx.x; q < planes; q += gridDim.x) {
        const int64_t outer = q / per, inner = q - outer * per;
        const Tin* s = src + (outer * 4 * per + inner) * (int64_t)L;
        if (SMEM) {
            // step j of path 1 is pixel (j mod H, j div H); path 3 visits it at L-1-j
            for (int j = threadIdx.x; j < L; j += kThreads) {
                const int w = j / H, h = j - w * H;
                cols[w * pitch + h] = ldf(s + ps + j) + ldf(s + 3 * ps + (L - 1 - j));
            }
            __syncthreads();
        }
        Tout* d = dst + q * (int64_t)L;
        for (int p = threadIdx.x; p < L; p += kThreads) {
            const int h = p / W, w = p - h * W;
            const float s02 = ldf(s + p) + ldf(s + 2 * ps + (L - 1 - p));
            float s13;
            if (SMEM) {
                s13 = cols[w * pitch + h];
            } else {
                const int j = w * H + h;
                s13 = ldf(s + ps + j) + ldf(s + 3 * ps + (L - 1 - j));
            }
            stf(d + p, scale * (s02 + s13));
        }
        if (SMEM) __syncthreads();
    }
}

// dA over the four path blocks of channels: (4, n) -> (n), (p0 + p2) + (p1 + p3).
__global__ void sum_paths_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = (src[i] + src[2 * n + i]) + (src[n + i] + src[3 * n + i]);
}

static int grid_for(int64_t planes) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return (int)min64(planes, (int64_t)sms * 8);
}

template <typename T>
static int gather_t(const void* src, void* dst, int64_t planes, int64_t per, int H, int W, float scale,
                    cudaStream_t st) {
    const size_t sm = (size_t)H * odd_pitch(W) * sizeof(float);
    const int grid = grid_for(planes);
    if (sm <= kSmemLimit) {
        auto k = gather_kernel<T, true>;
        if (sm > 48 * 1024 &&
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
            return check_launch("ss2d gather: smem attribute");
        k<<<grid, kThreads, sm, st>>>(static_cast<const T*>(src), static_cast<T*>(dst), planes, per, H, W, scale);
    } else {
        gather_kernel<T, false><<<grid, kThreads, 0, st>>>(static_cast<const T*>(src), static_cast<T*>(dst),
                                                          planes, per, H, W, scale);
    }
    return check_launch("ss2d gather");
}

static int gather(int dtype, const void* src, void* dst, int64_t planes, int64_t per, int H, int W,
                  float scale, cudaStream_t st) {
    if (planes == 0 || H == 0 || W == 0) return SSM_OK;
    switch (dtype) {
        case SSM_F32: return gather_t<float>(src, dst, planes, per, H, W, scale, st);
        case SSM_BF16: return gather_t<__nv_bfloat16>(src, dst, planes, per, H, W, scale, st);
        default: return gather_t<__half>(src, dst, planes, per, H, W, scale, st);
    }
}

template <typename Tin, typename Tout>
static int merge_t(const void* src, void* dst, int64_t planes, int64_t per, int H, int W, float scale,
                   cudaStream_t st) {
    const size_t sm = (size_t)W * odd_pitch(H) * sizeof(float);
    const int grid = grid_for(planes);
    if (sm <= kSmemLimit) {
        auto k = merge_kernel<Tin, Tout, true>;
        if (sm > 48 * 1024 &&
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
            return check_launch("ss2d merge: smem attribute");
        k<<<grid, kThreads, sm, st>>>(static_cast<const Tin*>(src), static_cast<Tout*>(dst), planes, per, H, W,
                                      scale);
    } else {
        merge_kernel<Tin, Tout, false><<<grid, kThreads, 0, st>>>(static_cast<const Tin*>(src),
                                                                 static_cast<Tout*>(dst), planes, per, H, W,
                                                                 scale);
    }
    return check_launch("ss2d merge");
}

// Path slices and the merged planes share a dtype (act dtype), or are fp32 (dB, dC).
static int merge(int dtype, const void* src, void* dst, int64_t planes, int64_t per, int H, int W, float scale,
                 cudaStream_t st) {
    if (planes == 0 || H == 0 || W == 0) return SSM_OK;
    switch (dtype) {
        case SSM_F32: return merge_t<float, float>(src, dst, planes, per, H, W, scale, st);
        case SSM_BF16: return merge_t<__nv_bfloat16, __nv_bfloat16>(src, dst, planes, per, H, W, scale, st);
        default: return merge_t<__half, __half>(src, dst, planes, per, H, W, scale, st);
    }
}

static size_t esize(int dtype) { return dtype == SSM_F32 ? 4 : 2; }

static bool empty_problem(const ssm_ss2d_scan_params* p) {
    return p->batch == 0 || p->channels == 0 || p->height == 0 || p->width == 0 || p->dstate == 0;
}

static int validate(const ssm_ss2d_scan_params* p) {
    if (p == nullptr) return fail(SSM_ERR_INVALID, "ss2d_scan: null params");
    if (p->batch < 0 || p->channels < 0 || p->height < 0 || p->width < 0 || p->groups < 0 || p->dstate < 0)
        return fail(SSM_ERR_INVALID, "ss2d_scan: negative extent");
    if (p->channels > 0 && (p->groups < 1 || p->channels % p->groups))
        return fail(SSM_ERR_INVALID, "ss2d_scan: groups must divide channels");
    if (p->act_dtype < SSM_F32 || p->act_dtype > SSM_F16 || p->bc_dtype < SSM_F32 || p->bc_dtype > SSM_F16)
        return fail(SSM_ERR_UNSUPPORTED, "ss2d_scan: dtype");
    if (p->height * p->width > (int64_t)1 << 30)
        return fail(SSM_ERR_UNSUPPORTED, "ss2d_scan: height * width too large");
    if (!(p->scale == 1.0f || p->scale == 0.25f))
        return fail(SSM_ERR_INVALID, "ss2d_scan: scale must be 1 (sum) or 0.25 (mean)");
    return SSM_OK;
}

// The Mamba-1 problem the four paths form: 4 x channels rows, 4 x groups groups.
static ssm_selective_scan_params stacked(const ssm_ss2d_scan_params* p) {
    ssm_selective_scan_params s;
    std::memset(&s, 0, sizeof(s));
    s.batch = p->batch;
    s.dim = 4 * p->channels;
    s.length = p->height * p->width;
    s.groups = 4 * p->groups;
    s.dstate = p->dstate;
    s.act_dtype = p->act_dtype;
    s.bc_dtype = p->bc_dtype;
    s.flags = 0;
    s.status = p->status;
    return s;
}

struct Layout {
    size_t su, sdt, sB, sC, A4, ypaths, fscan;   // forward (and the backward's first five)
    size_t sdy, dup, ddtp, dBp, dCp, dA4, scan;  // backward
    size_t fwd_bytes, bwd_bytes, scan_ws, scan_fws, ckpt;
};

static int layout(const ssm_ss2d_scan_params* p, Layout& o) {
    const int64_t L = p->height * p->width;
    const size_t act = (size_t)p->batch * 4 * p->channels * L * esize(p->act_dtype);
    const size_t bc = (size_t)p->batch * 4 * p->groups * p->dstate * L * esize(p->bc_dtype);
    const size_t bc32 = (size_t)p->batch * 4 * p->groups * p->dstate * L * 4;
    const size_t a4 = (size_t)4 * p->channels * p->dstate * 4;
    o.scan_ws = o.scan_fws = o.ckpt = 0;
    if (!empty_problem(p)) {
        ssm_selective_scan_params s = stacked(p);
        if (int st = ssm_selective_scan_sizes(&s, &o.ckpt, &o.scan_ws)) return st;
        if (int st = ssm_selective_scan_fwd_workspace(&s, &o.scan_fws)) return st;
    }
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t at = off; off = align_up(off + bytes, 256); return at; };
    o.su = take(act);
    o.sdt = take(act);
    o.sB = take(bc);
    o.sC = take(bc);
    o.A4 = take(a4);
    const size_t common_end = off;
    o.ypaths = take(act);
    o.fscan = take(o.scan_fws);
    o.fwd_bytes = off;
    off = common_end;
    o.sdy = take(act);
    o.dup = take(act);
    o.ddtp = take(act);
    o.dBp = take(bc32);
    o.dCp = take(bc32);
    o.dA4 = take(a4);
    o.scan = take(o.scan_ws);
    o.bwd_bytes = off;
    return SSM_OK;
}

// Stacked u, dt, B, C and A (four copies of A, one per path block of channels).
static int stage_inputs(const ssm_ss2d_scan_params* p, const Layout& o, unsigned char* ws, cudaStream_t st) {
    const int H = (int)p->height, W = (int)p->width;
    const int64_t planes = p->batch * p->channels, gplanes = p->batch * p->groups * p->dstate;
    const int64_t gper = p->groups * p->dstate;
    if (int s = gather(p->act_dtype, p->u, ws + o.su, planes, p->channels, H, W, 1.0f, st)) return s;
    if (int s = gather(p->act_dtype, p->dt, ws + o.sdt, planes, p->channels, H, W, 1.0f, st)) return s;
    if (int s = gather(p->bc_dtype, p->B, ws + o.sB, gplanes, gper, H, W, 1.0f, st)) return s;
    if (int s = gather(p->bc_dtype, p->C, ws + o.sC, gplanes, gper, H, W, 1.0f, st)) return s;
    const size_t abytes = (size_t)p->channels * p->dstate * 4;
    for (int k = 0; k < 4; ++k)
        if (cudaMemcpyAsync(ws + o.A4 + k * abytes, p->A, abytes, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return check_launch("ss2d: copy of A");
    return SSM_OK;
}

static void bind_inputs(ssm_selective_scan_params& s, const Layout& o, unsigned char* ws) {
    s.u = ws + o.su;
    s.delta = ws + o.sdt;
    s.B = ws + o.sB;
    s.C = ws + o.sC;
    s.A = reinterpret_cast<const float*>(ws + o.A4);
}

}  // namespace ss2d
}  // namespace ssm

using namespace ssm;
using namespace ssm::ss2d;

extern "C" int ssm_ss2d_scan_sizes(const ssm_ss2d_scan_params* p, size_t* checkpoint_bytes,
                                   size_t* fwd_workspace_bytes, size_t* bwd_workspace_bytes) {
    if (int s = validate(p)) return s;
    Layout o;
    if (int s = layout(p, o)) return s;
    if (checkpoint_bytes) *checkpoint_bytes = o.ckpt;
    if (fwd_workspace_bytes) *fwd_workspace_bytes = o.fwd_bytes;
    if (bwd_workspace_bytes) *bwd_workspace_bytes = o.bwd_bytes;
    return SSM_OK;
}

extern "C" int ssm_ss2d_scan_fwd(const ssm_ss2d_scan_params* p, void* stream) {
    if (int s = validate(p)) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t L = p->height * p->width;
    const size_t ybytes = (size_t)p->batch * p->channels * L * esize(p->act_dtype);
    if (empty_problem(p)) {
        if (ybytes && cudaMemsetAsync(p->y, 0, ybytes, st) != cudaSuccess) return check_launch("ss2d fwd: zero y");
        return SSM_OK;
    }
    Layout o;
    if (int s = layout(p, o)) return s;
    if (p->workspace == nullptr || p->workspace_bytes < o.fwd_bytes)
        return fail(SSM_ERR_WORKSPACE, "ss2d_scan fwd: workspace smaller than ssm_ss2d_scan_sizes");
    unsigned char* ws = static_cast<unsigned char*>(p->workspace);
    if (int s = stage_inputs(p, o, ws, st)) return s;
    ssm_selective_scan_params s = stacked(p);
    bind_inputs(s, o, ws);
    s.y = ws + o.ypaths;
    s.checkpoints = p->checkpoints;
    s.workspace = ws + o.fscan;
    s.workspace_bytes = o.scan_fws;
    if (int r = ssm_selective_scan_fwd(&s, stream)) return r;
    return merge(p->act_dtype, ws + o.ypaths, p->y, p->batch * p->channels, p->channels, (int)p->height,
                 (int)p->width, p->scale, st);
}

extern "C" int ssm_ss2d_scan_bwd(const ssm_ss2d_scan_params* p, void* stream) {
    if (int s = validate(p)) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t L = p->height * p->width;
    if (empty_problem(p)) {
        const size_t act = (size_t)p->batch * p->channels * L * esize(p->act_dtype);
        const size_t bc = (size_t)p->batch * p->groups * p->dstate * L * 4;
        const size_t a = (size_t)p->channels * p->dstate * 4;
        struct { void* ptr; size_t bytes; } outs[] = {{p->du, act}, {p->ddt, act}, {p->dA, a}, {p->dB, bc}, {p->dC, bc}};
        for (auto& x : outs)
            if (x.bytes && cudaMemsetAsync(x.ptr, 0, x.bytes, st) != cudaSuccess)
                return check_launch("ss2d bwd: zero gradients");
        return SSM_OK;
    }
    if (p->checkpoints == nullptr) return fail(SSM_ERR_INVALID, "ss2d_scan bwd: the forward saved no checkpoints");
    Layout o;
    if (int s = layout(p, o)) return s;
    if (p->workspace == nullptr || p->workspace_bytes < o.bwd_bytes)
        return fail(SSM_ERR_WORKSPACE, "ss2d_scan bwd: workspace smaller than ssm_ss2d_scan_sizes");
    unsigned char* ws = static_cast<unsigned char*>(p->workspace);
    const int H = (int)p->height, W = (int)p->width;
    const int64_t planes = p->batch * p->channels, gplanes = p->batch * p->groups * p->dstate;
    const int64_t gper = p->groups * p->dstate;
    if (int s = stage_inputs(p, o, ws, st)) return s;
    // every path receives the merged output's gradient times the merge scale
    if (int s = gather(p->act_dtype, p->dout, ws + o.sdy, planes, p->channels, H, W, p->scale, st)) return s;
    ssm_selective_scan_params s = stacked(p);
    bind_inputs(s, o, ws);
    s.checkpoints = p->checkpoints;
    s.dout = ws + o.sdy;
    s.du = ws + o.dup;
    s.ddelta = ws + o.ddtp;
    s.dA = reinterpret_cast<float*>(ws + o.dA4);
    s.dB = reinterpret_cast<float*>(ws + o.dBp);
    s.dC = reinterpret_cast<float*>(ws + o.dCp);
    s.workspace = ws + o.scan;
    s.workspace_bytes = o.scan_ws;
    if (int r = ssm_selective_scan_bwd(&s, stream)) return r;
    if (int r = merge(p->act_dtype, ws + o.dup, p->du, planes, p->channels, H, W, 1.0f, st)) return r;
    if (int r = merge(p->act_dtype, ws + o.ddtp, p->ddt, planes, p->channels, H, W, 1.0f, st)) return r;
    if (int r = merge(SSM_F32, ws + o.dBp, p->dB, gplanes, gper, H, W, 1.0f, st)) return r;
    if (int r = merge(SSM_F32, ws + o.dCp, p->dC, gplanes, gper, H, W, 1.0f, st)) return r;
    const int64_t n = p->channels * p->dstate;
    sum_paths_kernel<<<(int)min64(ceil_div(n, 256), 1024), 256, 0, st>>>(
        reinterpret_cast<const float*>(ws + o.dA4), p->dA, n);
    return check_launch("ss2d dA");
}
