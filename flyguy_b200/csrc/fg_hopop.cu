// The per-hop operator of the reference's CUDA path (flyguy/fly_cuda.py HopCuda, lines 78-115: kernels spmm_f /
// spmm_h / sddmm_f / sddmm_h at 25-54), on the caller's device buffers: no handle, no plan, no allocation beyond a
// 4-byte scratch word for the 16-bit gradient scale. States are [neurons, batch] with the batch a multiple of 32.
//
//   fg_hop_fwd: out[t, b] = sum over the edges e of row t (CSR by target: crow int64, col int32) of w[e] * h[col[e], b]
//   fg_hop_bwd: gw[e]     = sum_b gz[t(e), b] * h[col[e], b]
//               gh[s, b]  = sum over the edges of source s (CSR by source: tcrow int64, tcol int32, tperm int64 = the
//                           by-target position of each by-source edge) of w[tperm[i]] * gz[tcol[i], b]
// 16-bit mode (the reference's "cuda16": states read as fp16, sums in fp32): forward rounds h to fp16 as h.half()
// does; backward divides gz by scale = max|gz| (at least 1e-30), rounds it and h to fp16, sums in fp32 and multiplies
// the results by scale - the reference's own steps (fly_cuda.py:100-113).
//
// A warp owns one row (or one source, or one row's edges for gw) and 128 samples, 4 per lane; a row's edges are
// taken in CSR order, one fp32 FMA per edge and sample, as the reference's per-thread loop does. gw is a warp
// reduction per edge over the whole batch, written once (no atomics: the same value on every run).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <string>

#include "flyguy_b200.h"

namespace {

thread_local std::string g_hop_error;

constexpr int kHopWarps = 8;

__device__ __forceinline__ float r16(float v) { return __half2float(__float2half_rn(v)); }

// out[t, b..b+3] for warp row t = (crow, col, w[perm ? perm[e] : e]) x x; HALF: x read as fp16(x / scale)
template <bool HALF>
__global__ void __launch_bounds__(32 * kHopWarps) k_edge_spmm(const long long* __restrict__ crow,
                                                              const int* __restrict__ col, const float* __restrict__ w,
                                                              const long long* __restrict__ perm,
                                                              const float* __restrict__ x, float* __restrict__ out,
                                                              int n_rows, int B, const float* __restrict__ scale) {
    const int t = blockIdx.x * kHopWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int b = blockIdx.y * 128 + lane * 4;
    if (t >= n_rows || b >= B) return;
    const float sc = HALF && scale ? __ldg(scale) : 1.f;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    const long long e1 = __ldg(&crow[t + 1]);
    for (long long e = __ldg(&crow[t]); e < e1; ++e) {
        const float we = __ldg(&w[perm ? __ldg(&perm[e]) : e]);
        float4 v = __ldg(reinterpret_cast<const float4*>(x + (size_t)__ldg(&col[e]) * B + b));
        if (HALF) { v.x = r16(v.x / sc); v.y = r16(v.y / sc); v.z = r16(v.z / sc); v.w = r16(v.w / sc); }
        a0 = fmaf(we, v.x, a0); a1 = fmaf(we, v.y, a1); a2 = fmaf(we, v.z, a2); a3 = fmaf(we, v.w, a3);
    }
    *reinterpret_cast<float4*>(out + (size_t)t * B + b) = make_float4(a0 * sc, a1 * sc, a2 * sc, a3 * sc);
}

// gw[e] for the edges of warp row t: a dot product over the whole batch, reduced across the warp
template <bool HALF>
__global__ void __launch_bounds__(32 * kHopWarps) k_edge_sddmm(const long long* __restrict__ crow,
                                                               const int* __restrict__ col,
                                                               const float* __restrict__ gz,
                                                               const float* __restrict__ h, float* __restrict__ gw,
                                                               int n_rows, int B, const float* __restrict__ scale) {
    const int t = blockIdx.x * kHopWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= n_rows) return;
    const float sc = HALF ? __ldg(scale) : 1.f;
    const long long e1 = __ldg(&crow[t + 1]);
    for (long long e = __ldg(&crow[t]); e < e1; ++e) {
        const float* hs = h + (size_t)__ldg(&col[e]) * B;
        const float* gs = gz + (size_t)t * B;
        float s = 0.f;
        for (int b = lane * 4; b < B; b += 128) {
            float4 g = __ldg(reinterpret_cast<const float4*>(gs + b));
            float4 v = __ldg(reinterpret_cast<const float4*>(hs + b));
            if (HALF) {
                g.x = r16(g.x / sc); g.y = r16(g.y / sc); g.z = r16(g.z / sc); g.w = r16(g.w / sc);
                v.x = r16(v.x); v.y = r16(v.y); v.z = r16(v.z); v.w = r16(v.w);
            }
            s = fmaf(g.x, v.x, s); s = fmaf(g.y, v.y, s); s = fmaf(g.z, v.z, s); s = fmaf(g.w, v.w, s);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) gw[e] = s * sc;
    }
}

// max |x| over n values into *out (non-negative floats order as their bit patterns), at least 1e-30
__global__ void k_absmax(const float* __restrict__ x, long long n, unsigned* __restrict__ out) {
    float m = 0.f;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(__ldg(&x[i])));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(fmaxf(m, 1e-30f)));
}

struct HopErr {
    std::string msg;
};
#define HCK(call)                                                                                 \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess) throw HopErr{std::string(#call) + ": " + cudaGetErrorString(e_)};  \
    } while (0)

template <class F>
int hop_guard(F&& f) {
    try {
        f();
        g_hop_error.clear();
        return 0;
    } catch (const HopErr& e) {
        g_hop_error = e.msg;
    } catch (const std::exception& e) {
        g_hop_error = e.what();
    }
    return -1;
}

void check_shape(int n_rows, int n_src, int B) {
    if (n_rows < 0 || n_src < 0) throw HopErr{"fg_hop: negative row count"};
    if (B <= 0 || B % 32) throw HopErr{"fg_hop: the batch must be a positive multiple of 32"};
}
// states are read and written 4 samples (16 bytes) at a time
void check_aligned(const void* p, const char* what) {
    if (p && reinterpret_cast<uintptr_t>(p) % 16) throw HopErr{std::string("fg_hop: ") + what + " is not 16-byte aligned"};
}

// the 16-bit gradient scale: one word per device, kept for the process (the only device memory these calls own)
float* scale_word() {
    static thread_local int dev = -1;
    static thread_local float* p = nullptr;
    int d = 0;
    HCK(cudaGetDevice(&d));
    if (!p || d != dev) {
        HCK(cudaMalloc(&p, sizeof(float)));
        dev = d;
    }
    return p;
}

}  // namespace

extern "C" {

int fg_hop_fwd(const float* w, const float* h, const long long* crow, const int* col, int n_rows, int n_src, int B,
               int half, float* out, void* stream) {
    return hop_guard([&]() {
        check_shape(n_rows, n_src, B);
        if (!w || !h || !crow || !col || !out) throw HopErr{"fg_hop_fwd: null pointer"};
        check_aligned(h, "h");
        check_aligned(out, "out");
        if (!n_rows) return;
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        const dim3 g((unsigned)((n_rows + kHopWarps - 1) / kHopWarps), (unsigned)((B + 127) / 128));
        if (half) k_edge_spmm<true><<<g, 32 * kHopWarps, 0, st>>>(crow, col, w, nullptr, h, out, n_rows, B, nullptr);
        else k_edge_spmm<false><<<g, 32 * kHopWarps, 0, st>>>(crow, col, w, nullptr, h, out, n_rows, B, nullptr);
        HCK(cudaGetLastError());
    });
}

int fg_hop_bwd(const float* w, const float* h, const float* gz, const long long* crow, const int* col,
               const long long* tcrow, const int* tcol, const long long* tperm, int n_rows, int n_src, int B,
               int half, float* gw, float* gh, void* stream) {
    return hop_guard([&]() {
        check_shape(n_rows, n_src, B);
        if (!w || !h || !gz || !crow || !col) throw HopErr{"fg_hop_bwd: null pointer"};
        if (gh && (!tcrow || !tcol || !tperm)) throw HopErr{"fg_hop_bwd: gh needs the by-source CSR"};
        check_aligned(h, "h");
        check_aligned(gz, "gz");
        check_aligned(gh, "gh");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        float* sc = nullptr;
        if (half) {
            sc = scale_word();
            HCK(cudaMemsetAsync(sc, 0, sizeof(float), st));
            const long long n = (long long)n_rows * B;
            if (n) k_absmax<<<(unsigned)std::min<long long>((n + 255) / 256, 4096), 256, 0, st>>>(gz, n, reinterpret_cast<unsigned*>(sc));
            HCK(cudaGetLastError());
        }
        if (gw && n_rows) {
            const unsigned g = (unsigned)((n_rows + kHopWarps - 1) / kHopWarps);
            if (half) k_edge_sddmm<true><<<g, 32 * kHopWarps, 0, st>>>(crow, col, gz, h, gw, n_rows, B, sc);
            else k_edge_sddmm<false><<<g, 32 * kHopWarps, 0, st>>>(crow, col, gz, h, gw, n_rows, B, nullptr);
            HCK(cudaGetLastError());
        }
        if (gh && n_src) {
            const dim3 g((unsigned)((n_src + kHopWarps - 1) / kHopWarps), (unsigned)((B + 127) / 128));
            if (half) k_edge_spmm<true><<<g, 32 * kHopWarps, 0, st>>>(tcrow, tcol, w, tperm, gz, gh, n_src, B, sc);
            else k_edge_spmm<false><<<g, 32 * kHopWarps, 0, st>>>(tcrow, tcol, w, tperm, gz, gh, n_src, B, nullptr);
            HCK(cudaGetLastError());
        }
    });
}

const char* fg_hop_last_error(void) { return g_hop_error.c_str(); }

}  // extern "C"
