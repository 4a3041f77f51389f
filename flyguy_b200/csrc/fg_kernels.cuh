// flyguy_b200 device code: the hop path's kernels for sm_100a.
//
// Layout: every layer's states are neuron-major [rows][ld] (ld = the batch), so one warp reads 32*V consecutive
// samples of ONE source neuron as a single coalesced 16-byte-per-lane load (V = 4 fp32 or 8 bf16 values per lane).
// The forward and transposed products walk MERGED edge runs: the edges of one (destination, source) pair are folded
// into one weight once per weight version (k_fold_pairs), so a duplicate-heavy graph does each (row, source) product
// once. Reductions over the batch (neuron, plug and weight gradients) are owned by one CTA each and reduced in a
// fixed order - no float atomics, bit-reproducible for a given batch.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace fg {

constexpr int kWarps = 8;                 // warps per CTA of the row kernels
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxAct = 96;                // actions at most (the output plug's tiles pad to 96)

// First statement of every kernel. Launched with programmatic dependent launch (the library's step kernels), a kernel
// can start while the stream's previous kernel is still running: griddepcontrol.wait blocks until that grid has
// completed and its memory is visible, and launch_dependents lets the next kernel's launch begin once every CTA of
// this one has started. Launched without it, both are no-ops.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}


// ---- 16-byte vector loads / stores of V activations as fp32
__device__ __forceinline__ void ld_act(const float* p, float (&v)[4]) {
    float4 q = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
__device__ __forceinline__ void ld_act(const __nv_bfloat16* p, float (&v)[8]) {
    uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
    // bf16 -> fp32 is exact: the 16 bits become the high half of the fp32 word
    v[0] = __uint_as_float(q.x << 16); v[1] = __uint_as_float(q.x & 0xffff0000u);
    v[2] = __uint_as_float(q.y << 16); v[3] = __uint_as_float(q.y & 0xffff0000u);
    v[4] = __uint_as_float(q.z << 16); v[5] = __uint_as_float(q.z & 0xffff0000u);
    v[6] = __uint_as_float(q.w << 16); v[7] = __uint_as_float(q.w & 0xffff0000u);
}
__device__ __forceinline__ void ld_act(const __half* p, float (&v)[8]) {
    uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        v[2 * i] = f.x; v[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void st_act(float* p, const float (&v)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&b);
}
__device__ __forceinline__ void st_act(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 q;
    q.x = pack_bf16(v[0], v[1]); q.y = pack_bf16(v[2], v[3]);
    q.z = pack_bf16(v[4], v[5]); q.w = pack_bf16(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = q;
}
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
    __half2 b = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&b);
}
__device__ __forceinline__ void st_act(__half* p, const float (&v)[8]) {
    uint4 q;
    q.x = pack_f16(v[0], v[1]); q.y = pack_f16(v[2], v[3]);
    q.z = pack_f16(v[4], v[5]); q.w = pack_f16(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = q;
}
// V fp32 values stored as the layer's type (V = that type's vector width)
template <class TO, int V>
__device__ __forceinline__ void st_vals(TO* p, const float (&v)[V]);
template <>
__device__ __forceinline__ void st_vals<float, 8>(float* p, const float (&v)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
template <>
__device__ __forceinline__ void st_vals<float, 4>(float* p, const float (&v)[4]) { st_act(p, v); }
template <>
__device__ __forceinline__ void st_vals<__nv_bfloat16, 8>(__nv_bfloat16* p, const float (&v)[8]) { st_act(p, v); }
template <>
__device__ __forceinline__ void st_vals<__half, 8>(__half* p, const float (&v)[8]) { st_act(p, v); }
__device__ __forceinline__ void store2(float* p, float a, float b) { *reinterpret_cast<float2*>(p) = make_float2(a, b); }
__device__ __forceinline__ void store2(__nv_bfloat16* p, float a, float b) {
    *reinterpret_cast<uint32_t*>(p) = pack_bf16(a, b);
}
__device__ __forceinline__ void store2(__half* p, float a, float b) { *reinterpret_cast<uint32_t*>(p) = pack_f16(a, b); }
__device__ __forceinline__ float ld1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float ld1(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ float ld1(const __nv_bfloat16* p) { return __bfloat162float(*p); }

__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// sum of N values over the CTA (fixed order); result valid in every thread. `red` holds kWarps*N floats.
template <int N>
__device__ __forceinline__ void block_sum(float (&v)[N], float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = warp_sum(v[i]);
    __syncthreads();
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < N; ++i) red[i * kWarps + warp] = v[i];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < N; ++i) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += red[i * kWarps + w];
        v[i] = s;
    }
}

// ---------------------------------------------------------------- weight-version folds
// (one launch, k_fold in fg_outtc.cuh, runs the four folds side by side in separate block ranges)
// per row of every layer: its neuron's gain and threshold softplus(theta)
__device__ __forceinline__ void fold_neuron(int i, const int* __restrict__ nid, const float* __restrict__ gain,
                                            const float* __restrict__ theta, float* __restrict__ rgain,
                                            float* __restrict__ rthr, float* __restrict__ rsig, int n) {
    if (i >= n) return;
    int id = nid[i];
    float th = theta[id];
    rgain[i] = gain[id];
    rthr[i] = softplus_f(th);
    rsig[i] = sigmoid_f(th);
}
// merged pair weight = sum of the weights of its edges (edges of one (row, source) pair are contiguous)
// A warp owns 32 consecutive pairs: it gathers the weights of their edges (a contiguous range of gw) into shared memory
// with all lanes, 256 at a time, then each lane adds its own pair's edges from there. The sum is also
// written to the pair's place among the transposed pairs (tpos[p] >= 0) when there are any.
constexpr int kFoldBuf = 256;
__device__ __forceinline__ void fold_pairs(int blk, float (*buf)[kFoldBuf], const int* __restrict__ gptr,
                                           const int* __restrict__ gw, const float* __restrict__ W,
                                           int2* __restrict__ pairs, const int* __restrict__ tpos,
                                           int2* __restrict__ tpairs, int n) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p0 = (blk * kWarps + warp) * 32;
    if (p0 >= n) return;
    const int p = p0 + lane, pend = min(p0 + 32, n);
    const int e_lo = __ldg(&gptr[p0]), e_hi = __ldg(&gptr[pend]);
    const int my_lo = p < n ? __ldg(&gptr[p]) : e_hi, my_hi = p < n ? __ldg(&gptr[p + 1]) : e_hi;
    float* sb = buf[warp];
    float s = 0.f;
    for (int base = e_lo; base < e_hi; base += kFoldBuf) {
        const int cnt = min(kFoldBuf, e_hi - base);
#pragma unroll 8
        for (int i = lane; i < kFoldBuf; i += 32)
            if (i < cnt) sb[i] = __ldg(&W[__ldg(&gw[base + i])]);
        __syncwarp();
        // the lane's edges in this window into four interleaved sums, added pairwise (a fixed order: the same bits
        // in every run): a pair of many duplicate edges (hundreds on a hub source) waits on a quarter of the adds
        const int lo = max(my_lo, base) - base, hi = min(my_hi, base + cnt) - base;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int e = lo;
        for (; e + 4 <= hi; e += 4) {
            a0 += sb[e]; a1 += sb[e + 1]; a2 += sb[e + 2]; a3 += sb[e + 3];
        }
        if (e < hi) a0 += sb[e];
        if (e + 1 < hi) a1 += sb[e + 1];
        if (e + 2 < hi) a2 += sb[e + 2];
        if (lo < hi) s += (a0 + a1) + (a2 + a3);
        __syncwarp();
    }
    if (p < n) {
        pairs[p].y = __float_as_int(s);
        const int q = tpos ? __ldg(&tpos[p]) : -1;
        if (q >= 0) tpairs[q].y = __float_as_int(s);
    }
}


// ---------------------------------------------------------------- layout changes at the API boundary
// in [B, D] (sample-major, the caller's) -> out [D, ld] (neuron-major); 32x32 tiles through shared memory
__global__ void k_to_neuron_major(const float* __restrict__ in, float* __restrict__ out, int D, int B, int ld) {
    pdl_enter();
    __shared__ float tile[32][33];
    int b0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        int b = b0 + r, d = d0 + threadIdx.x;
        tile[r][threadIdx.x] = (b < B && d < D) ? in[(size_t)b * D + d] : 0.f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        int d = d0 + r, b = b0 + threadIdx.x;
        if (d < D && b < B) out[(size_t)d * ld + b] = tile[threadIdx.x][r];
    }
}

// ---------------------------------------------------------------- forward
// input plug + sensory activation: drive[s,b] = in_b[s] + sum_j in_w[s*fan+j] * x[col, b];
// h0 = relu(gain*drive - thr). A CTA stages x for a chunk of samples (all obs_dim rows; in the state type for 16-bit
// states - 128 samples - or fp32 - 64 samples) and its rows' plug columns and weights in shared memory, then every warp
// computes rows from there: lane l owns the chunk's samples [NS*l, NS*l + NS).
#ifndef FG_PLUG_THREADS
#define FG_PLUG_THREADS 768           // 24 warps: measured 1.24 ms vs 1.47 ms (512) and 1.32 ms (1024) at batch 65,536
#endif
constexpr int kPlugThreads = FG_PLUG_THREADS;
// samples per CTA chunk: 2 per lane for fp32 states, 4 for 16-bit states (517 obs rows x 64 or 128 = 132 KB staged)
template <class T> struct PlugCfg {
    static constexpr int cols = sizeof(T) == 4 ? 64 : 128;
    // rows a warp stages at a time (fewer for wide fans, so the slices fit beside the staged obs), and a warp's slice:
    // RW row records {bias, gain, threshold, -} and RW x F columns and weights
    __host__ __device__ static constexpr int rows(int F) { return F > 8 ? 16 : 32; }
    __host__ __device__ static constexpr int warp_bytes(int F) { return rows(F) * 16 + rows(F) * F * 8; }
};
__device__ __forceinline__ void cvt_store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void cvt_store4(__nv_bfloat16* p, float4 v) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
}
__device__ __forceinline__ void cvt_store4(__half* p, float4 v) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_f16(v.x, v.y), pack_f16(v.z, v.w));
}
// NS consecutive staged values as fp32 (NS = 2 for fp32, 4 for 16-bit types)
__device__ __forceinline__ void lds_ns(const float* p, float (&v)[2]) {
    const float2 q = *reinterpret_cast<const float2*>(p);
    v[0] = q.x; v[1] = q.y;
}
__device__ __forceinline__ void lds_ns(const __nv_bfloat16* p, float (&v)[4]) {
    const uint2 q = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(q.x << 16); v[1] = __uint_as_float(q.x & 0xffff0000u);
    v[2] = __uint_as_float(q.y << 16); v[3] = __uint_as_float(q.y & 0xffff0000u);
}
__device__ __forceinline__ void lds_ns(const __half* p, float (&v)[4]) {
    const uint2 q = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&q.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void st_ns(float* p, const float (&v)[2]) { *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]); }
__device__ __forceinline__ void st_ns(__nv_bfloat16* p, const float (&v)[4]) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
}
__device__ __forceinline__ void st_ns(__half* p, const float (&v)[4]) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_f16(v[0], v[1]), pack_f16(v[2], v[3]));
}

// relu(gain * drive - thr) of one lane's NS samples (as fp32 pairs), stored as the state type: 16-bit states round
// each pair first and take the max with zero on the packed pair (the same value as rounding after the relu)
template <class T, int NS>
__device__ __forceinline__ void plug_store(T* o, const float2 (&d)[NS / 2], float gn, float th) {
    const float2 g2 = make_float2(gn, gn), t2 = make_float2(-th, -th);
    if constexpr (sizeof(T) == 4) {
        static_assert(NS == 2, "fp32 states: two samples a lane");
        const float2 u = __ffma2_rn(g2, d[0], t2);
        *reinterpret_cast<float2*>(o) = make_float2(fmaxf(u.x, 0.f), fmaxf(u.y, 0.f));
    } else {
        static_assert(NS == 4, "16-bit states: four samples a lane");
        uint32_t q[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const float2 u = __ffma2_rn(g2, d[k], t2);
            if constexpr (std::is_same<T, __nv_bfloat16>::value) {
                __nv_bfloat162 b = __hmax2(__floats2bfloat162_rn(u.x, u.y), __float2bfloat162_rn(0.f));
                q[k] = *reinterpret_cast<uint32_t*>(&b);
            } else {
                __half2 b = __hmax2(__floats2half2_rn(u.x, u.y), __float2half2_rn(0.f));
                q[k] = *reinterpret_cast<uint32_t*>(&b);
            }
        }
        *reinterpret_cast<uint2*>(o) = make_uint2(q[0], q[1]);
    }
}

// A CTA owns one chunk of C samples and a block of rows: x for the chunk is staged once (as the state type for
// 16-bit states), then each warp takes RW consecutive rows at a time and stages, in its own slice of shared memory,
// their plug columns, weights and {bias, gain, threshold} with coalesced loads; the row loop then reads only shared
// memory (broadcast reads of the row's record, one 8-byte read of staged x per lane and column). FAN: the plug's
// fan-in (a multiple of 4 up to 16) or 0 for any fan (slower path).
template <class T, bool SAVE_DRIVE, int FAN>
__global__ void __launch_bounds__(kPlugThreads) k_plug_fwd(const int* __restrict__ in_col,
                                                           const float* __restrict__ in_w,
                                                           const float* __restrict__ in_b,
                                                           const float* __restrict__ rgain,
                                                           const float* __restrict__ rthr, const float* __restrict__ x,
                                                           float* __restrict__ drive, T* __restrict__ h0, int n_s,
                                                           int fan, int rows_per_cta, int obs_dim, int ld) {
    pdl_enter();
    constexpr int C = PlugCfg<T>::cols, NS = C / 32;
    constexpr int F = FAN > 0 ? FAN : 1;
    constexpr int kWarpsP = kPlugThreads / 32;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* xs = reinterpret_cast<T*>(smem_raw);                                               // [obs_dim][C]
    unsigned char* warp_base = smem_raw + ((size_t)obs_dim * C * sizeof(T) + 15) / 16 * 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int RW = PlugCfg<T>::rows(F);
    float4* rp = reinterpret_cast<float4*>(warp_base + (size_t)warp * PlugCfg<T>::warp_bytes(F));   // [RW] b, g, thr
    int* rc = reinterpret_cast<int*>(rp + RW);                                                       // [RW][F] cols
    float* rw = reinterpret_cast<float*>(rc + RW * F);                                               // [RW][F] weights
    const int b0 = blockIdx.y * C;
    const int r_lo = blockIdx.x * rows_per_cta, r_hi = min(n_s, r_lo + rows_per_cta);
    {                                                     // stage the chunk: four 16-byte loads in flight a thread
        constexpr int Q = C / 4, U = 4;
        const int total = obs_dim * Q;
        for (int i0 = threadIdx.x; i0 < total; i0 += U * blockDim.x) {
            float4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * blockDim.x, f = i / Q, q = (i - f * Q) * 4;
                v[u] = i < total && b0 + q < ld ? __ldg(reinterpret_cast<const float4*>(x + (size_t)f * ld + b0 + q))
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * blockDim.x, f = i / Q, q = (i - f * Q) * 4;
                if (i < total) cvt_store4(xs + f * C + q, v[u]);
            }
        }
    }
    __syncthreads();
    const int bl = NS * lane;
    const bool on = b0 + bl < ld;
    const T* xl = xs + bl;
    for (int r0 = r_lo + warp * RW; r0 < r_hi; r0 += kWarpsP * RW) {
        const int nrows = min(RW, r_hi - r0);
        __syncwarp();
        if (lane < nrows) {
            const int r = r0 + lane;
            rp[lane] = make_float4(__ldg(&in_b[r]), __ldg(&rgain[r]), __ldg(&rthr[r]), 0.f);
            if constexpr (FAN > 0) {
                const size_t e = (size_t)r * FAN;
#pragma unroll
                for (int j = 0; j < FAN; j += 4) {
                    *reinterpret_cast<int4*>(rc + lane * F + j) = __ldg(reinterpret_cast<const int4*>(in_col + e + j));
                    *reinterpret_cast<float4*>(rw + lane * F + j) = __ldg(reinterpret_cast<const float4*>(in_w + e + j));
                }
            }
        }
        __syncwarp();
        if (!on) continue;
        for (int i = 0; i < nrows; ++i) {
            const int row = r0 + i;
            const float4 prm = rp[i];
            float2 a2[NS / 2];
#pragma unroll
            for (int k = 0; k < NS / 2; ++k) a2[k] = make_float2(prm.x, prm.x);
            if constexpr (FAN > 0) {
#pragma unroll
                for (int j = 0; j < FAN; j += 4) {
                    const int4 cc = *reinterpret_cast<const int4*>(rc + i * F + j);
                    const float4 ww = *reinterpret_cast<const float4*>(rw + i * F + j);
                    const int cs[4] = {cc.x, cc.y, cc.z, cc.w};
                    const float ws[4] = {ww.x, ww.y, ww.z, ww.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        float v[NS];
                        lds_ns(xl + cs[u] * C, v);
                        const float2 w2 = make_float2(ws[u], ws[u]);
#pragma unroll
                        for (int k = 0; k < NS / 2; ++k)      // the same fp32 FMA per sample, two per instruction
                            a2[k] = __ffma2_rn(w2, make_float2(v[2 * k], v[2 * k + 1]), a2[k]);
                    }
                }
            } else {
                const size_t e0 = (size_t)row * fan;
                for (int j = 0; j < fan; ++j) {
                    float v[NS];
                    lds_ns(xl + __ldg(&in_col[e0 + j]) * C, v);
                    const float w = __ldg(&in_w[e0 + j]);
#pragma unroll
                    for (int k = 0; k < NS / 2; ++k) {
                        a2[k].x = fmaf(w, v[2 * k], a2[k].x);
                        a2[k].y = fmaf(w, v[2 * k + 1], a2[k].y);
                    }
                }
            }
            const size_t o = (size_t)row * ld + b0 + bl;
            if (SAVE_DRIVE) {
                if constexpr (NS == 2) *reinterpret_cast<float2*>(drive + o) = a2[0];
                else *reinterpret_cast<float4*>(drive + o) = make_float4(a2[0].x, a2[0].y, a2[1].x, a2[1].y);
            }
            plug_store<T, NS>(h0 + o, a2, prm.y, prm.z);
        }
    }
}

// one hop: z[t,b] = sum over merged pairs (src, w) of row t of w * hp[src, b] (+ drive[drow[t], b]);
// h = relu(gain*z - thr). One warp per (row, chunk of NG*32*V samples): each lane loads NG 16-byte groups of the
// source row per pair, the warp's loads of a group being one contiguous 512-byte run (group g of lane l: samples
// chunk + g*32V + l*V ... + V-1), so the pair record and its address math are shared by NG*V FMAs per lane; products
// use packed fp32x2 FMAs (sm_100). Rows run in degree-descending schedule order.
// TI: the source layer's type, TO: this layer's (the last layer of a 16-bit network is fp32).
__device__ __forceinline__ void unpack2(const __nv_bfloat16*, uint32_t x, float2& f) {
    f = make_float2(__uint_as_float(x << 16), __uint_as_float(x & 0xffff0000u));
}
__device__ __forceinline__ void unpack2(const __half*, uint32_t x, float2& f) {
    f = __half22float2(*reinterpret_cast<const __half2*>(&x));
}
// 16 bytes at p as float2 pairs (4 for 16-bit types, 2 for fp32)
template <class T>
__device__ __forceinline__ void ld16(const T* p, float2 (&v)[16 / sizeof(T) / 2]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    if constexpr (sizeof(T) == 4) {
        v[0] = make_float2(__uint_as_float(a.x), __uint_as_float(a.y));
        v[1] = make_float2(__uint_as_float(a.z), __uint_as_float(a.w));
    } else {
        unpack2(p, a.x, v[0]); unpack2(p, a.y, v[1]); unpack2(p, a.z, v[2]); unpack2(p, a.w, v[3]);
    }
}
template <class T> struct Vec16 { static constexpr int V = 16 / sizeof(T), H = V / 2; };

template <class TO, int V>
__device__ __forceinline__ void st16(TO* o, const float* hv) {
    if constexpr (sizeof(TO) == 4) {
#pragma unroll
        for (int i = 0; i < V; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(hv[i], hv[i + 1], hv[i + 2], hv[i + 3]);
    } else {
        float q[8] = {hv[0], hv[1], hv[2], hv[3], hv[4], hv[5], hv[6], hv[7]};
        st_act(o, q);
    }
}

// Per source-state type (measured at batch 65,536 bf16 / 16,384 and 4,096 fp32 on the Zipf graph; two pairs in flight
// beat the look-ahead record and one pair at a time for both types: bf16 hop forward 7.14 against 7.37 and 7.53 ms):
//   NG  16-byte groups per lane per pair - the pair record, its address and the loop are shared by NG x V samples
//       (16-bit: 4 -> 32 samples a lane, 1,024 a warp; fp32: 8 -> 32 samples a lane, 1,024 a warp);
//   PF  the next pair's record is loaded before this pair's gathers (fp32 only: with 16-bit states the extra
//       registers cost more than the shorter dependency chain saves);
//   UNR (without PF) pairs whose records and gathers are issued before any of their products;
//   min_blocks  resident CTAs per SM the register allocation is sized for (16-bit: 64 registers, fp32: 80).
#ifndef FG_HOP_NG16
#define FG_HOP_NG16 4
#endif
#ifndef FG_HOP_NG32
#define FG_HOP_NG32 8
#endif
#ifndef FG_HOP_PF16
#define FG_HOP_PF16 0
#endif
#ifndef FG_HOP_PF32
#define FG_HOP_PF32 0
#endif
#ifndef FG_HOP_UNR16
#define FG_HOP_UNR16 2
#endif
#ifndef FG_HOP_UNR32
#define FG_HOP_UNR32 2
#endif
#ifndef FG_HOP_MINB16
#define FG_HOP_MINB16 4
#endif
#ifndef FG_HOP_MINB32
#define FG_HOP_MINB32 3
#endif
// NARROW (fp32 states on a hop without hub sources, where the gathers miss L1): four groups (16 samples a lane,
// 512-sample warp chunks) at 64 registers and 4 CTAs a SM, more warps to cover the L2 latency - on the model.pt network
// the training step's hop forward took 13.0 ms against 14.1 with eight groups at 3 CTAs a SM; on the Zipf graph eight
// groups stay faster (2.96 against 3.12 ms)
template <class TI, bool NARROW = false> struct HopCfg {
    static constexpr bool W = NARROW && sizeof(TI) == 4;
    static constexpr int NG = W ? 4 : sizeof(TI) == 2 ? FG_HOP_NG16 : FG_HOP_NG32;
    static constexpr int UNR = sizeof(TI) == 2 ? FG_HOP_UNR16 : FG_HOP_UNR32;
    static constexpr bool PF = sizeof(TI) == 2 ? FG_HOP_PF16 : FG_HOP_PF32;
    static constexpr int min_blocks = W ? 4 : sizeof(TI) == 2 ? FG_HOP_MINB16 : FG_HOP_MINB32;
};
// states per lane per pair (the warp's chunk is 32 N samples)
template <class T, bool NARROW = false> struct Lane32 {
    static constexpr int N = HopCfg<T, NARROW>::NG * 16 / (int)sizeof(T);
};
// the 16 raw bytes of a gather, unpacked to fp32 and multiplied into a (same FMA per sample as one at a time)
template <class TI>
__device__ __forceinline__ void fma16(const uint4& r, float2 w, float2 (&a)[Vec16<TI>::H]) {
    if constexpr (sizeof(TI) == 4) {
        a[0] = __ffma2_rn(w, make_float2(__uint_as_float(r.x), __uint_as_float(r.y)), a[0]);
        a[1] = __ffma2_rn(w, make_float2(__uint_as_float(r.z), __uint_as_float(r.w)), a[1]);
    } else {
        const TI* tag = nullptr;
        float2 v[4];
        unpack2(tag, r.x, v[0]); unpack2(tag, r.y, v[1]); unpack2(tag, r.z, v[2]); unpack2(tag, r.w, v[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = __ffma2_rn(w, v[i], a[i]);
    }
}
__device__ __forceinline__ uint4 ldg16(const char* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
// byte offset of row r of a [rows][ld] array: a 32 x 32 -> 64-bit product (row_bytes = ld * element size < 2^32), so the
// address is one widening multiply-add instead of a 64-bit product
__device__ __forceinline__ const char* row_at(const char* base, int r, unsigned row_bytes) {
    return base + (unsigned long long)(unsigned)r * row_bytes;
}
// relu(gain * z - thr) of 16 bytes' worth of outputs, stored as the layer's type: 16-bit layers round each pair of
// values to the type first and take the max with zero on the packed pair (rounding is monotonic and keeps the sign, so
// this is the value rounded after the relu, as the oracle's emulation stores it)
template <class TO, int H>
__device__ __forceinline__ void act_store(TO* o, const float2 (&a)[H], float gn, float th) {
    const float2 g2 = make_float2(gn, gn), t2 = make_float2(-th, -th);
    if constexpr (sizeof(TO) == 4) {
#pragma unroll
        for (int i = 0; i < H; i += 2) {
            const float2 u = __ffma2_rn(g2, a[i], t2), v = __ffma2_rn(g2, a[i + 1], t2);
            *reinterpret_cast<float4*>(o + 2 * i) = make_float4(fmaxf(u.x, 0.f), fmaxf(u.y, 0.f), fmaxf(v.x, 0.f),
                                                                fmaxf(v.y, 0.f));
        }
    } else {
        static_assert(H == 4, "a 16-bit layer's 16 bytes are 8 values");
        uint32_t q[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 u = __ffma2_rn(g2, a[i], t2);
            if constexpr (std::is_same<TO, __nv_bfloat16>::value) {
                __nv_bfloat162 b = __hmax2(__floats2bfloat162_rn(u.x, u.y), __float2bfloat162_rn(0.f));
                q[i] = *reinterpret_cast<uint32_t*>(&b);
            } else {
                __half2 b = __hmax2(__floats2half2_rn(u.x, u.y), __float2half2_rn(0.f));
                q[i] = *reinterpret_cast<uint32_t*>(&b);
            }
        }
        *reinterpret_cast<uint4*>(o) = make_uint4(q[0], q[1], q[2], q[3]);
    }
}
// One warp's work: row `slot` of the schedule x sample chunk `chunk`. rows[slot] = {first pair, end, row t, 0}: three
// independent loads from one 16-byte record. drow[t]: the sensory row whose drive is added again, or -1 (drow is null
// for a network without sensory re-drive). FULL: the
// warp's whole chunk lies inside the batch (ld a multiple of 32 N): no per-group validity tests. SURV (the firing
// survey): also adds, per row, the number of samples whose state is positive to fired[t] and the sum of the squared
// pre-activations to sq[t] (per-lane atomics: lanes past the batch have already returned).
template <class TI, class TO, bool FULL, bool SURV = false, bool NARROW = false>
__device__ __forceinline__ void hop_row(int slot, int chunk, const int4* __restrict__ rows,
                                        const int2* __restrict__ pairs, const TI* __restrict__ hp,
                                        const float* __restrict__ rgain, const float* __restrict__ rthr,
                                        const int* __restrict__ drow, const float* __restrict__ drive,
                                        TO* __restrict__ h, int n_rows, int ld, int* __restrict__ fired = nullptr,
                                        float* __restrict__ sq = nullptr) {
    constexpr int V = Vec16<TI>::V, H = Vec16<TI>::H, NG = HopCfg<TI, NARROW>::NG, U = HopCfg<TI, NARROW>::UNR;
    constexpr bool PF = HopCfg<TI, NARROW>::PF;
    constexpr int GB = 32 * 16;                          // byte distance between a lane's groups
    const int lane = threadIdx.x & 31;
    if (slot >= n_rows) return;
    const int c0 = chunk * 32 * V * NG + lane * V;      // the lane's group g: samples c0 + 32 V g ...
    if (!FULL && c0 >= ld) return;
    const int t = __ldg(&rows[slot].z);
    // groups inside the batch (ld is a multiple of 32, so a group is either wholly inside or wholly outside)
    const int ng = FULL ? NG : min(NG, (ld - c0 + 32 * V - 1) / (32 * V));
    float2 a[NG][H];
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int i = 0; i < H; ++i) a[g][i] = make_float2(0.f, 0.f);
    const unsigned row_bytes = (unsigned)ld * (unsigned)sizeof(TI);
    const char* base = reinterpret_cast<const char*>(hp + c0);
    int e = __ldg(&rows[slot].x);
    const int e1 = __ldg(&rows[slot].y);
    if (FULL || ng == NG) {
        for (; !PF && e + U <= e1; e += U) {             // (with the look-ahead below, pairs go one at a time)
            int2 p[U];
            uint4 r[U][NG];
#pragma unroll
            for (int u = 0; u < U; ++u) p[u] = __ldg(&pairs[e + u]);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const char* ap = row_at(base, p[u].x, row_bytes);
#pragma unroll
                for (int g = 0; g < NG; ++g) r[u][g] = ldg16(ap + g * GB);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const float2 w = make_float2(__int_as_float(p[u].y), __int_as_float(p[u].y));
#pragma unroll
                for (int g = 0; g < NG; ++g) fma16<TI>(r[u][g], w, a[g]);
            }
        }
        // PF: the next pair's record is loaded before this pair's gathers (the pair array has one record past its end)
        int2 pn = PF && e < e1 ? __ldg(&pairs[e]) : make_int2(0, 0);
        for (; e < e1; ++e) {
            int2 p;
            if constexpr (PF) {
                p = pn;
                pn = __ldg(&pairs[e + 1]);
            } else {
                p = __ldg(&pairs[e]);
            }
            const char* ap = row_at(base, p.x, row_bytes);
            uint4 r[NG];
#pragma unroll
            for (int g = 0; g < NG; ++g) r[g] = ldg16(ap + g * GB);
            const float2 w = make_float2(__int_as_float(p.y), __int_as_float(p.y));
#pragma unroll
            for (int g = 0; g < NG; ++g) fma16<TI>(r[g], w, a[g]);
        }
    } else {                                              // the batch ends inside this chunk
        for (; e < e1; ++e) {
            const int2 p = __ldg(&pairs[e]);
            const char* ap = row_at(base, p.x, row_bytes);
            const float2 w = make_float2(__int_as_float(p.y), __int_as_float(p.y));
#pragma unroll
            for (int g = 0; g < NG; ++g)
                if (g < ng) fma16<TI>(ldg16(ap + g * GB), w, a[g]);
        }
    }
    if (drow) {                                          // (a network with sensory re-drive: z += drive[d])
        const int d = __ldg(&drow[t]);
        if (d >= 0) {
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                if (g >= ng) break;
                const float4* dr = reinterpret_cast<const float4*>(drive + (size_t)d * ld + c0 + g * 32 * V);
#pragma unroll
                for (int i = 0; i < H / 2; ++i) {
                    const float4 q = __ldg(dr + i);
                    a[g][2 * i].x += q.x; a[g][2 * i].y += q.y; a[g][2 * i + 1].x += q.z; a[g][2 * i + 1].y += q.w;
                }
            }
        }
    }
    const float gn = __ldg(&rgain[t]), th = __ldg(&rthr[t]);
    if constexpr (!SURV) {
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            if (g >= ng) break;
            act_store<TO, H>(h + (size_t)t * ld + c0 + g * 32 * V, a[g], gn, th);
        }
    } else {
        int n_on = 0;
        float s2 = 0.f;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            if (g >= ng) break;
            float hv[V];
#pragma unroll
            for (int i = 0; i < H; ++i) {
                hv[2 * i] = fmaxf(fmaf(gn, a[g][i].x, -th), 0.f);
                hv[2 * i + 1] = fmaxf(fmaf(gn, a[g][i].y, -th), 0.f);
                n_on += (hv[2 * i] > 0.f) + (hv[2 * i + 1] > 0.f);
                s2 = fmaf(a[g][i].x, a[g][i].x, fmaf(a[g][i].y, a[g][i].y, s2));
            }
            st16<TO, V>(h + (size_t)t * ld + c0 + g * 32 * V, hv);
        }
        atomicAdd(&fired[t], n_on);
        atomicAdd(&sq[t], s2);
    }
}

template <class TI, class TO, bool FULL, bool NARROW = false>
__global__ void __launch_bounds__(kThreads, HopCfg<TI, NARROW>::min_blocks) k_hop_fwd(const int4* __restrict__ rows,
                                                                               const int2* __restrict__ pairs,
                                                                               const TI* __restrict__ hp,
                                                                               const float* __restrict__ rgain,
                                                                               const float* __restrict__ rthr,
                                                                               const int* __restrict__ drow,
                                                                               const float* __restrict__ drive,
                                                                               TO* __restrict__ h, int n_rows, int ld) {
    pdl_enter();
    hop_row<TI, TO, FULL, false, NARROW>(blockIdx.x * kWarps + (threadIdx.x >> 5), blockIdx.y, rows, pairs, hp, rgain,
                                         rthr, drow, drive, h, n_rows, ld);
}
// the same forward hop for the firing survey (fired / sq: this hop's rows)
template <class TI, class TO, bool FULL>
__global__ void __launch_bounds__(kThreads) k_hop_fwd_surv(const int4* __restrict__ rows,
                                                           const int2* __restrict__ pairs, const TI* __restrict__ hp,
                                                           const float* __restrict__ rgain,
                                                           const float* __restrict__ rthr,
                                                           const int* __restrict__ drow,
                                                           const float* __restrict__ drive, TO* __restrict__ h,
                                                           int n_rows, int ld, int* __restrict__ fired,
                                                           float* __restrict__ sq) {
    pdl_enter();
    hop_row<TI, TO, FULL, true>(blockIdx.x * kWarps + (threadIdx.x >> 5), blockIdx.y, rows, pairs, hp, rgain, rthr,
                                drow, drive, h, n_rows, ld, fired, sq);
}
// the firing survey of the sensory layer: samples with a positive state per row (a warp per row)
template <class T>
__global__ void __launch_bounds__(kThreads) k_count_fired(const T* __restrict__ h0, int* __restrict__ fired, int n_s,
                                                          int B, int ld) {
    pdl_enter();
    const int r = blockIdx.x * kWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= n_s) return;
    int c = 0;
    for (int b = lane; b < B; b += 32) c += ld1(h0 + (size_t)r * ld + b) > 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) fired[r] += c;
}

// output plug: the forward and backward products are the tensor-core kernels of fg_outtc.cuh; kOutA is the padded
// action count of the forward's partial slabs
constexpr int kOutA = 96;
constexpr int kOutSlices = 8;                           // most split-K slices of the output plug's dn columns
// the slices' partial logits added in slice order + bias -> lg [n_act, ld] and/or out [B, n_act]; a CTA per 32 samples
__global__ void __launch_bounds__(256) k_out_reduce(const float* __restrict__ part, const float* __restrict__ ob,
                                                    float* __restrict__ lg, float* __restrict__ out, int slices,
                                                    int n_act, int B, int ld) {
    pdl_enter();
    __shared__ float st[32][kOutA + 1];
    const int b0 = blockIdx.x * 32;
    // every slice's partial of 4 (action, sample) items loaded before any is added (slices <= kOutSlices), so a
    // thread waits for memory once per 4 items, not once per partial; the sum is the bias, then slice 0, 1, ...
#pragma unroll 4
    for (int i = threadIdx.x; i < n_act * 32; i += 256) {
        const int a = i >> 5, bb = i & 31, b = b0 + bb;
        if (b >= B) continue;
        float p[kOutSlices];
#pragma unroll
        for (int s = 0; s < kOutSlices; ++s) p[s] = s < slices ? __ldg(&part[((size_t)s * kOutA + a) * ld + b]) : 0.f;
        float v = __ldg(&ob[a]);
#pragma unroll
        for (int s = 0; s < kOutSlices; ++s)
            if (s < slices) v += p[s];
        if (lg) lg[(size_t)a * ld + b] = v;
        st[bb][a] = v;
    }
    if (!out) return;
    __syncthreads();
    const int nbb = max(0, min(32, B - b0));
    float* o = out + (size_t)b0 * n_act;
    for (int i = threadIdx.x; i < nbb * n_act; i += 256) {
        const int bb = i / n_act, a = i - bb * n_act;
        o[i] = st[bb][a];
    }
}

// ---------------------------------------------------------------- loss
// per sample: p_t = softmax(teacher * it); kl = sum p_t (log p_t - log softmax(s)); dl = (softmax(s) - p_t) * inv_norm
// (inv_norm = 1 / the number of samples the loss averages over: the batch, or more when a batch comes in pieces);
// argmax agreement. teacher is the caller's [B, n_act]; lg and dl are neuron-major.
// A CTA owns kLossS samples: all its threads stage their logit rows ([a][b], coalesced) and teacher rows ([b][a],
// contiguous) in shared memory (teacher row stride n_act + 1 words: odd for n_act = 90, so the per-sample reads do not
// conflict), then a warp per sample computes it with its lanes over the actions and warp reductions (a short
// dependency chain at small batches, where one thread per sample running the passes in order took 26 us), writes dl
// into the staged logits, and the CTA stores dl back row by row. kLossS = 8 samples a CTA (one per warp; each staged row
// one 32-byte sector): a batch of 2,048 gives 256 CTAs for the 148 SMs, not 64.
#ifndef FG_LOSS_S
#define FG_LOSS_S 8
#endif
constexpr int kLossS = FG_LOSS_S, kLossT = 256;
__global__ void __launch_bounds__(kLossT) k_loss(const float* __restrict__ lg, const float* __restrict__ teacher,
                                                 float* __restrict__ dl, float* __restrict__ kl_s,
                                                 float* __restrict__ ag_s, int n_act, int B, int ld, float it,
                                                 float inv_norm) {
    pdl_enter();
    __shared__ float sl[kMaxAct * kLossS];
    __shared__ float stt[kLossS * (kMaxAct + 1)];
    const int b0 = blockIdx.x * kLossS, nb = min(kLossS, B - b0), tw = n_act + 1;
    const int j = threadIdx.x & (kLossS - 1), a0 = threadIdx.x / kLossS;
#pragma unroll 4
    for (int a = a0; a < n_act; a += kLossT / kLossS)
        if (j < nb) sl[a * kLossS + j] = __ldg(&lg[(size_t)a * ld + b0 + j]);
    const float* tb = teacher + (size_t)b0 * n_act;
#pragma unroll 4
    for (int i = threadIdx.x; i < nb * n_act; i += kLossT) {
        const int r = i / n_act;
        stt[r * tw + (i - r * n_act)] = __ldg(&tb[i]);
    }
    __syncthreads();
    // a warp per sample, the lanes over the actions (3 a lane for 90 actions): max with the
    // first index in action order on ties (the reference's strict '>' scan), the two log-sum-exps, the KL and dl
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int PA = kMaxAct / 32;
    for (int jj = warp; jj < nb; jj += kLossT / 32) {
        const float* t = stt + jj * tw;
        float sv[PA], tv[PA];
        float ms = -INFINITY, mt = -INFINITY;
        int as = n_act, at = n_act;
#pragma unroll
        for (int k = 0; k < PA; ++k) {
            const int a = lane + 32 * k;
            sv[k] = a < n_act ? sl[a * kLossS + jj] : -INFINITY;
            tv[k] = a < n_act ? t[a] * it : -INFINITY;
            if (a < n_act && (sv[k] > ms || as == n_act)) { ms = sv[k]; as = a; }
            if (a < n_act && (tv[k] > mt || at == n_act)) { mt = tv[k]; at = a; }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {                   // (value, first index) maxima over the warp
            const float ms2 = __shfl_xor_sync(0xffffffffu, ms, o), mt2 = __shfl_xor_sync(0xffffffffu, mt, o);
            const int as2 = __shfl_xor_sync(0xffffffffu, as, o), at2 = __shfl_xor_sync(0xffffffffu, at, o);
            if (ms2 > ms || (ms2 == ms && as2 < as)) { ms = ms2; as = as2; }
            if (mt2 > mt || (mt2 == mt && at2 < at)) { mt = mt2; at = at2; }
        }
        float zs = 0.f, zt = 0.f;
#pragma unroll
        for (int k = 0; k < PA; ++k)
            if (lane + 32 * k < n_act) { zs += expf(sv[k] - ms); zt += expf(tv[k] - mt); }
        zs = warp_sum(zs);
        zt = warp_sum(zt);
        const float ls = ms + logf(zs), lt = mt + logf(zt);
        float kl = 0.f;
#pragma unroll
        for (int k = 0; k < PA; ++k) {
            const int a = lane + 32 * k;
            if (a < n_act) {
                const float lps = sv[k] - ls, lpt = tv[k] - lt, pt = expf(lpt);
                kl += pt * (lpt - lps);
                sl[a * kLossS + jj] = (expf(lps) - pt) * inv_norm;
            }
        }
        kl = warp_sum(kl);
        if (lane == 0) {
            kl_s[b0 + jj] = kl;
            ag_s[b0 + jj] = as == at ? 1.f : 0.f;
        }
    }
    __syncthreads();
#pragma unroll 4
    for (int a = a0; a < n_act; a += kLossT / kLossS)
        if (j < nb) dl[(size_t)a * ld + b0 + j] = sl[a * kLossS + j];
}
// stats[0] += sum kl, stats[1] += sum agree: one CTA of 1,024 threads, 4 samples per thread step (B is a multiple of
// 32), warp sums then the 32 warp sums in warp order - a fixed order for a given batch
constexpr int kStatsT = 1024;
__global__ void __launch_bounds__(kStatsT) k_loss_stats(const float* __restrict__ kl_s, const float* __restrict__ ag_s,
                                                         float* __restrict__ stats, int B) {
    pdl_enter();
    __shared__ float red[2][kStatsT / 32];
    float v0 = 0.f, v1 = 0.f;
#pragma unroll 4
    for (int i = threadIdx.x; i < (B >> 2); i += kStatsT) {
        const float4 k = __ldg(reinterpret_cast<const float4*>(kl_s) + i);
        const float4 g = __ldg(reinterpret_cast<const float4*>(ag_s) + i);
        v0 += (k.x + k.y) + (k.z + k.w);
        v1 += (g.x + g.y) + (g.z + g.w);
    }
    v0 = warp_sum(v0);
    v1 = warp_sum(v1);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { red[0][w] = v0; red[1][w] = v1; }
    __syncthreads();
    if (w == 0) {
        v0 = warp_sum(red[0][lane]);
        v1 = warp_sum(red[1][lane]);
        if (lane == 0) { stats[0] += v0; stats[1] += v1; }
    }
}

// ---------------------------------------------------------------- backward: output plug
// G_out_w[a*n_dn + j] += sum_s part[s][a][j]; G_out_b[a] += sum_s part[s][a][n_dn]
__global__ void k_out_bwd_reduce(const float* __restrict__ part, float* __restrict__ gow, float* __restrict__ gob,
                                 int n_act, int n_dn, int splits) {
    pdl_enter();
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int n_col = n_dn + 1;
    if (i >= n_act * n_col) return;
    float s = 0.f;
#pragma unroll 8
    for (int k = 0; k < splits; ++k) s += part[(size_t)k * n_act * n_col + i];
    int a = i / n_col, j = i - a * n_col;
    if (j < n_dn) gow[(size_t)a * n_dn + j] += s; else gob[a] += s;
}

// ---------------------------------------------------------------- backward: through the neurons
// one CTA per listed row of the top layer: g = gh * [h > 0]; gz = g * gain -> gz; gain grad += sum g*z with z = (h + thr) / gain (exact where
// h > 0, the only place it counts); theta grad += sum -g * sigmoid(theta); gdrive[drow] += gz.
template <class T>
__global__ void __launch_bounds__(kThreads) k_act_bwd(const float* __restrict__ gh, const T* __restrict__ h,
                                                      const int* __restrict__ nid, const int* __restrict__ drow,
                                                      const float* __restrict__ rgain, const float* __restrict__ rthr,
                                                      const float* __restrict__ rsig, float* __restrict__ gz,
                                                      float* __restrict__ ggain, float* __restrict__ gtheta,
                                                      float* __restrict__ gdrive, const int* __restrict__ rows, int B,
                                                      int ld) {
    pdl_enter();
    __shared__ float red[3 * kWarps];
    const int t = __ldg(&rows[blockIdx.x]);             // a row whose gradient can be non-zero (an output-plug column)
    const float gn = rgain[t], th = rthr[t];
    const float inv_g = gn != 0.f ? 1.f / gn : 0.f;
    const int d = drow ? drow[t] : -1;
    const size_t o = (size_t)t * ld;
    float s[2] = {0.f, 0.f};                             // sum g*z, sum g
    for (int b = threadIdx.x * 4; b < B; b += kThreads * 4) {
        float4 q = __ldg(reinterpret_cast<const float4*>(gh + o + b));
        float hv[4] = {ld1(h + o + b), ld1(h + o + b + 1), ld1(h + o + b + 2), ld1(h + o + b + 3)};
        float gv[4] = {q.x, q.y, q.z, q.w};
        float zo[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float g = hv[i] > 0.f ? gv[i] : 0.f;
            s[0] = fmaf(g, (hv[i] + th) * inv_g, s[0]);
            s[1] += g;
            zo[i] = g * gn;
        }
        *reinterpret_cast<float4*>(gz + o + b) = make_float4(zo[0], zo[1], zo[2], zo[3]);
        if (d >= 0) {
            float4* gd = reinterpret_cast<float4*>(gdrive + (size_t)d * ld + b);
            float4 c = *gd;
            c.x += zo[0]; c.y += zo[1]; c.z += zo[2]; c.w += zo[3];
            *gd = c;
        }
    }
    block_sum<2>(s, red);
    if (threadIdx.x == 0) {
        const int id = nid[t];
        ggain[id] += s[0];
        gtheta[id] += -s[1] * rsig[t];
    }
}

// transposed hop: gh[s, b] = sum over merged pairs (dst, w) of source row s of w * gz[dst, b]. The source rows are
// cut into segments of at most a fixed number of pairs (hub sources have tens of thousands); a segment of a row that
// has one finishes the row, the others write partial rows that the last of them to finish adds up in slot order.
// One warp per (segment, 256-sample chunk); each lane owns two 4-sample groups 128 samples apart (every warp load is
// one contiguous 512-byte run); packed fp32x2 FMAs; segments longest first. seg = {row, first pair, end, slot or -1}.
// Chunk-major launch order and hub rows cut into short segments keep the few chunks in flight inside L2 (a hub row
// reaches every destination row, so each chunk reads its whole gz column slab).
// Finishing a row (EPI): the source layer's neuron backward is fused in - g = gh * [h > 0]; gz = g * gain is written
// (not gh), gdrive[drow] += gz, and the row's per-chunk sums of g*z (z = (h + thr) / gain where h > 0) and of g
// go to nsum[row][chunk][2] for k_neuron_reduce. Without EPI (the sensory layer) gh itself is written.
// The weight gradient (the reference's SDDMM, flyguy_train.cu:158-167) is fused in: the warp loads its source row's
// states for its chunk once (hs) and, per pair, adds gz[dst] * hs[src] over the chunk's 256 samples into
// wpart[chunk][pair] (two pairs' warp sums at once: each half-warp reduces one); k_sd_reduce then adds a pair's chunks
// in order into its edges' weight gradients. The gz rows each pair loads serve both products, and no source row is
// gathered per pair (the separate SDDMM gathered one per pair over the whole batch: on the model.pt network the
// training step went 56.6 -> 39.1 ms with the fusion, on the Zipf graph 5.08 -> 4.79 ms).
struct NeuronEpi {
    const float* h;          // the source layer's states [rows, ld]
    const float* rgain;      // per row
    const float* rthr;
    const int* drow;         // re-drive rows (nullable)
    float* gdrive;           // [n_s, ld]
    float* nsum;             // [rows][chunks][2]
    int chunks;
};
// one 4-sample group of a finished row: stores, and adds the group's neuron sums into sum[2]
template <bool EPI>
__device__ __forceinline__ void finish_group(int s, int c, int ld, const float (&a)[4], float* out,
                                             const NeuronEpi& ep, float gn, float th, float inv_g, float (&sum)[2]) {
    float* o = out + (size_t)s * ld + c;
    if (!EPI) {
        *reinterpret_cast<float4*>(o) = make_float4(a[0], a[1], a[2], a[3]);
        return;
    }
    const float4 hq = __ldg(reinterpret_cast<const float4*>(ep.h + (size_t)s * ld + c));
    const float hv[4] = {hq.x, hq.y, hq.z, hq.w};
    float gz[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float g = hv[i] > 0.f ? a[i] : 0.f;
        gz[i] = g * gn;
        sum[0] = fmaf(g, (hv[i] + th) * inv_g, sum[0]);
        sum[1] += g;
    }
    *reinterpret_cast<float4*>(o) = make_float4(gz[0], gz[1], gz[2], gz[3]);
    if (ep.drow) {
        const int d = __ldg(&ep.drow[s]);
        if (d >= 0) {
            float4* gd = reinterpret_cast<float4*>(ep.gdrive + (size_t)d * ld + c);
            float4 u = *gd;
            u.x += gz[0]; u.y += gz[1]; u.z += gz[2]; u.w += gz[3];
            *gd = u;
        }
    }
}
// the lane's two groups of a finished row (valid: in the batch); the warp then reduces the neuron sums
template <bool EPI>
__device__ __forceinline__ void finish_row(int s, int chunk, int c0, int c1, bool v0, bool v1, int ld,
                                           const float (&a0)[4], const float (&a1)[4], float* out,
                                           const NeuronEpi& ep) {
    float sum[2] = {0.f, 0.f};
    float gn = 0.f, th = 0.f, inv_g = 0.f;
    if (EPI) {
        gn = __ldg(&ep.rgain[s]);
        th = __ldg(&ep.rthr[s]);
        inv_g = gn != 0.f ? 1.f / gn : 0.f;
    }
    if (v0) finish_group<EPI>(s, c0, ld, a0, out, ep, gn, th, inv_g, sum);
    if (v1) finish_group<EPI>(s, c1, ld, a1, out, ep, gn, th, inv_g, sum);
    if (EPI) {
        sum[0] = warp_sum(sum[0]); sum[1] = warp_sum(sum[1]);
        if ((threadIdx.x & 31) == 0) {
            float* ns = ep.nsum + ((size_t)s * ep.chunks + chunk) * 2;
            ns[0] = sum[0]; ns[1] = sum[1];
        }
    }
}

// A segment of a split row writes its partial row to part[slot], then counts itself in done[red][chunk]; the last of
// the row's segments to arrive (no waiting: the others just leave) adds all the row's partials in slot order through
// L2 and finishes the row, then resets the counter for the next call. Deterministic: the sum order is fixed.
// (Four pairs' gathers in flight, 64 registers, 4 CTAs a SM: against two pairs at 5 CTAs (48 registers) the training
// step measured 38.1 / 38.8 ms on model.pt, 4.73 / 4.77 ms on the Zipf graph, 0.802 / 0.820 ms at batch 2,048; four
// pairs at 80 registers (3 CTAs) 40.7 ms on model.pt.)
template <bool EPI, bool FULL>
__global__ void __launch_bounds__(kThreads, 4) k_hop_bwd_t(const int4* __restrict__ segs, const int* __restrict__ seg_red,
                                                        const int4* __restrict__ reds, int* __restrict__ done,
                                                        const int2* __restrict__ tpairs, const float* __restrict__ gz,
                                                        float* __restrict__ out, float* __restrict__ part, int n_segs,
                                                        int ld, NeuronEpi ep, const float* __restrict__ hs,
                                                        float* __restrict__ wpart, int T) {
    pdl_enter();
    const int sidx = blockIdx.x * kWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (sidx >= n_segs) return;
    const int4 sg = __ldg(&segs[sidx]);
    const int chunk = blockIdx.y;
    const int c0 = chunk * 256 + lane * 4, c1 = c0 + 128;
    // lanes past the batch stay to the end (the epilogue reduces over the warp) but load and store nothing
    const bool v0 = FULL || c0 < ld, v1 = FULL || c1 < ld;
    float2 a0[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)}, a1[2] = {a0[0], a0[1]};
    const unsigned row_bytes = (unsigned)ld * 4u;
    const char* base = reinterpret_cast<const char*>(gz + (v0 ? c0 : 0));
    {
        // every lane runs every pair (the warp sums need the whole warp); lanes past the batch load nothing
        const float2 z2 = make_float2(0.f, 0.f);
        float2 h0[2] = {z2, z2}, h1[2] = {z2, z2};
        if (v0) ld16<float>(hs + (size_t)sg.x * ld + c0, h0);
        if (v1) ld16<float>(hs + (size_t)sg.x * ld + c1, h1);
        float* wp = wpart + (size_t)chunk * T;
        auto dot = [&](const float2 (&u0)[2], const float2 (&u1)[2]) {
            float2 d = __fmul2_rn(u0[0], h0[0]);
            d = __ffma2_rn(u0[1], h0[1], d);
            d = __ffma2_rn(u1[0], h1[0], d);
            d = __ffma2_rn(u1[1], h1[1], d);
            return d.x + d.y;
        };
        // the warp sums of two pairs' products at once: lanes 0-15 end with a's, 16-31 with b's
        auto sum2 = [&](float a, float b) {
            float v = lane < 16 ? a : b;
            v += __shfl_xor_sync(0xffffffffu, lane < 16 ? b : a, 16);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            return v;
        };
        int e = sg.y;
        for (; e + 4 <= sg.z; e += 4) {                  // four pairs' loads in flight
            int2 r[4];
            float2 x[4][2][2];
#pragma unroll
            for (int u = 0; u < 4; ++u) r[u] = __ldg(&tpairs[e + u]);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const char* ap = row_at(base, r[u].x, row_bytes);
                x[u][0][0] = x[u][0][1] = x[u][1][0] = x[u][1][1] = z2;
                if (v0) ld16<float>(reinterpret_cast<const float*>(ap), x[u][0]);
                if (v1) ld16<float>(reinterpret_cast<const float*>(ap + 512), x[u][1]);
            }
            float d[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float2 w2 = make_float2(__int_as_float(r[u].y), __int_as_float(r[u].y));
                a0[0] = __ffma2_rn(w2, x[u][0][0], a0[0]); a0[1] = __ffma2_rn(w2, x[u][0][1], a0[1]);
                a1[0] = __ffma2_rn(w2, x[u][1][0], a1[0]); a1[1] = __ffma2_rn(w2, x[u][1][1], a1[1]);
                d[u] = dot(x[u][0], x[u][1]);
            }
            const float v01 = sum2(d[0], d[1]), v23 = sum2(d[2], d[3]);
            if ((lane & 15) == 0) {
                wp[e + (lane >> 4)] = v01;
                wp[e + 2 + (lane >> 4)] = v23;
            }
        }
        for (; e + 2 <= sg.z; e += 2) {
            const int2 p = __ldg(&tpairs[e]), q = __ldg(&tpairs[e + 1]);
            const char* ap = row_at(base, p.x, row_bytes);
            const char* aq = row_at(base, q.x, row_bytes);
            float2 x0[2] = {z2, z2}, x1[2] = {z2, z2}, y0[2] = {z2, z2}, y1[2] = {z2, z2};
            if (v0) {
                ld16<float>(reinterpret_cast<const float*>(ap), x0);
                ld16<float>(reinterpret_cast<const float*>(aq), y0);
            }
            if (v1) {
                ld16<float>(reinterpret_cast<const float*>(ap + 512), x1);
                ld16<float>(reinterpret_cast<const float*>(aq + 512), y1);
            }
            const float2 wp2 = make_float2(__int_as_float(p.y), __int_as_float(p.y));
            const float2 wq2 = make_float2(__int_as_float(q.y), __int_as_float(q.y));
            a0[0] = __ffma2_rn(wp2, x0[0], a0[0]); a0[1] = __ffma2_rn(wp2, x0[1], a0[1]);
            a1[0] = __ffma2_rn(wp2, x1[0], a1[0]); a1[1] = __ffma2_rn(wp2, x1[1], a1[1]);
            a0[0] = __ffma2_rn(wq2, y0[0], a0[0]); a0[1] = __ffma2_rn(wq2, y0[1], a0[1]);
            a1[0] = __ffma2_rn(wq2, y1[0], a1[0]); a1[1] = __ffma2_rn(wq2, y1[1], a1[1]);
            const float v = sum2(dot(x0, x1), dot(y0, y1));
            if ((lane & 15) == 0) wp[e + (lane >> 4)] = v;
        }
        if (e < sg.z) {
            const int2 p = __ldg(&tpairs[e]);
            const char* ap = row_at(base, p.x, row_bytes);
            float2 x0[2] = {z2, z2}, x1[2] = {z2, z2};
            if (v0) ld16<float>(reinterpret_cast<const float*>(ap), x0);
            if (v1) ld16<float>(reinterpret_cast<const float*>(ap + 512), x1);
            const float2 wp2 = make_float2(__int_as_float(p.y), __int_as_float(p.y));
            a0[0] = __ffma2_rn(wp2, x0[0], a0[0]); a0[1] = __ffma2_rn(wp2, x0[1], a0[1]);
            a1[0] = __ffma2_rn(wp2, x1[0], a1[0]); a1[1] = __ffma2_rn(wp2, x1[1], a1[1]);
            const float v = warp_sum(dot(x0, x1));
            if (lane == 0) wp[e] = v;
        }
    }
    float r0[4] = {a0[0].x, a0[0].y, a0[1].x, a0[1].y}, r1[4] = {a1[0].x, a1[0].y, a1[1].x, a1[1].y};
    if (sg.w < 0) {
        finish_row<EPI>(sg.x, chunk, c0, c1, v0, v1, ld, r0, r1, out, ep);
        return;
    }
    {                                                      // a segment of a split row
        float* o = part + (size_t)sg.w * ld;
        if (v0) *reinterpret_cast<float4*>(o + c0) = make_float4(r0[0], r0[1], r0[2], r0[3]);
        if (v1) *reinterpret_cast<float4*>(o + c1) = make_float4(r1[0], r1[1], r1[2], r1[3]);
    }
    const int ri = __ldg(&seg_red[sidx]);
    const int4 rd = __ldg(&reds[ri]);
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(&done[(size_t)ri * gridDim.y + chunk], 1) == rd.z - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
#pragma unroll
    for (int i = 0; i < 4; ++i) { r0[i] = 0.f; r1[i] = 0.f; }
    for (int i = 0; i < rd.z; ++i) {
        const float* q = part + (size_t)(rd.y + i) * ld;
        if (v0) {
            const float4 u = __ldcg(reinterpret_cast<const float4*>(q + c0));
            r0[0] += u.x; r0[1] += u.y; r0[2] += u.z; r0[3] += u.w;
        }
        if (v1) {
            const float4 u = __ldcg(reinterpret_cast<const float4*>(q + c1));
            r1[0] += u.x; r1[1] += u.y; r1[2] += u.z; r1[3] += u.w;
        }
    }
    finish_row<EPI>(sg.x, chunk, c0, c1, v0, v1, ld, r0, r1, out, ep);
    if (lane == 0) done[(size_t)ri * gridDim.y + chunk] = 0;
}

// per live edge {j, q} of a hop (sde, in transposed-pair order): the weight gradient of its pair q = the sum of the
// pair's chunk partials in chunk order, added to the edge's weight gradient gW[gw[j]] - a thread per edge, so a pair
// of hundreds of duplicate edges (a hub source) is spread over as many threads; ATOMIC when a weight is used by more
// than one pair of the hop
template <bool ATOMIC>
__global__ void __launch_bounds__(256) k_sd_reduce(const float* __restrict__ wpart, int T, int chunks,
                                                   const int2* __restrict__ sde, int n, const int* __restrict__ gw,
                                                   float* __restrict__ gW) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int2 e = __ldg(&sde[i]);
    float v = 0.f;
#pragma unroll 8
    for (int c = 0; c < chunks; ++c) v += __ldg(&wpart[(size_t)c * T + e.y]);
    const int w = __ldg(&gw[e.x]);
    if (ATOMIC) atomicAdd(&gW[w], v); else gW[w] += v;
}

// packed gradient: buf[i] = g[idx[i]] (unpack: g[idx[i]] = buf[i])
__global__ void k_grad_pack(float* __restrict__ g, const int* __restrict__ idx, float* __restrict__ buf, int n,
                            int unpack) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int w = __ldg(&idx[i]);
    if (unpack) g[w] = buf[i]; else buf[i] = g[w];
}

// per listed row of a layer (the rows the transposed hop finished): gain grad += sum over chunks of g*z, theta grad +=
// -(sum of g) * sigmoid(theta)
__global__ void k_neuron_reduce(const float* __restrict__ nsum, const int* __restrict__ list,
                                const int* __restrict__ nid, const float* __restrict__ rsig,
                                float* __restrict__ ggain, float* __restrict__ gtheta, int n, int chunks) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int s = __ldg(&list[i]);
    float a = 0.f, b = 0.f;
    const float* p = nsum + (size_t)s * chunks * 2;
#pragma unroll 4
    for (int k = 0; k < chunks; ++k) { a += p[2 * k]; b += p[2 * k + 1]; }
    const int id = nid[s];
    ggain[id] += a;
    gtheta[id] += -b * rsig[s];
}

// sensory layer and plug, one warp per listed sensory row s (the rows with a possibly non-zero gradient) over the
// whole batch (4 samples per lane per step):
// g0 = gh0 * [h0 > 0]; gd = gdrive (re-drive from later hops) + g0 * gain; sums over the batch of g0 * drive, g0, gd and
// gd * x[col_e] for the row's fan edges (FAN of them, FAN <= 16; FAN 0: up to 16 in steps), reduced over the warp in
// a fixed order and added to the gradients of gain, theta, in_b and in_w. Without a saved drive (a network with no
// sensory re-drive keeps none) the pre-activation is recovered where it counts, h0 > 0: drive = (h0 + thr) / gain.
constexpr int kPlugFan = 16;
constexpr int kPlugSplits = 8;                   // most batch splits of the plug backward
template <int FAN>
__global__ void __launch_bounds__(kThreads) k_plug_bwd(const int* __restrict__ list, const int* __restrict__ gh_valid,
                                                       const float* __restrict__ gh0, const float* __restrict__ h0,
                                                       const float* __restrict__ drive, const float* __restrict__ gdrive,
                                                       const int* __restrict__ n0, const int* __restrict__ in_col,
                                                       const float* __restrict__ x, const float* __restrict__ rgain,
                                                       const float* __restrict__ rthr,
                                                       const float* __restrict__ rsig, float* __restrict__ ggain,
                                                       float* __restrict__ gtheta, float* __restrict__ gin_w,
                                                       float* __restrict__ gin_b, int n_list, int fan, int B, int ld,
                                                       float* __restrict__ part, int span) {
    pdl_enter();
    constexpr int F = FAN > 0 ? FAN : kPlugFan;
    const int i = blockIdx.x * kWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (i >= n_list) return;
    // part: the batch is split over gridDim.y warps a row (span samples each, a multiple of 128), each writing its
    // sums to part[(row * splits + split) * (fan + 3) ..] for k_plug_bwd_reduce to add in split order
    const int b_lo = part ? blockIdx.y * span : 0, b_hi = part ? min(B, b_lo + span) : B;
    const int s = __ldg(&list[i]);
    const bool ghv = __ldg(&gh_valid[s]) != 0;      // rows the transposed hop did not write have gh0 = 0
    const float gn = __ldg(&rgain[s]), th = __ldg(&rthr[s]), inv_g = gn != 0.f ? 1.f / gn : 0.f;
    const size_t o = (size_t)s * ld;
    const size_t e0 = (size_t)s * fan;
    for (int f0 = 0; f0 < fan || f0 == 0; f0 += F) {
        const int nf = min(F, fan - f0);
        const bool first = f0 == 0;
        const float* xr[F];
#pragma unroll
        for (int u = 0; u < F; ++u) xr[u] = x + (size_t)(u < nf ? __ldg(&in_col[e0 + f0 + u]) : 0) * ld;
        float v[F + 3];
#pragma unroll
        for (int u = 0; u < F + 3; ++u) v[u] = 0.f;
        // (two steps' loads in flight: a warp per live row is few warps a SM, so each waits on memory latency)
#pragma unroll 2
        for (int b = b_lo + lane * 4; b < b_hi; b += 128) {
            const float4 gh = ghv ? __ldg(reinterpret_cast<const float4*>(gh0 + o + b)) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 hh = __ldg(reinterpret_cast<const float4*>(h0 + o + b));
            const float4 gr = __ldg(reinterpret_cast<const float4*>(gdrive + o + b));
            const float g[4] = {hh.x > 0.f ? gh.x : 0.f, hh.y > 0.f ? gh.y : 0.f, hh.z > 0.f ? gh.z : 0.f,
                                hh.w > 0.f ? gh.w : 0.f};
            const float gd[4] = {fmaf(g[0], gn, gr.x), fmaf(g[1], gn, gr.y), fmaf(g[2], gn, gr.z),
                                 fmaf(g[3], gn, gr.w)};
            if (first) {
                const float4 dr = drive ? __ldg(reinterpret_cast<const float4*>(drive + o + b))
                                        : make_float4((hh.x + th) * inv_g, (hh.y + th) * inv_g, (hh.z + th) * inv_g,
                                                      (hh.w + th) * inv_g);
                v[F] += g[0] * dr.x + g[1] * dr.y + g[2] * dr.z + g[3] * dr.w;
                v[F + 1] += g[0] + g[1] + g[2] + g[3];
                v[F + 2] += gd[0] + gd[1] + gd[2] + gd[3];
            }
#pragma unroll
            for (int u = 0; u < F; ++u) {
                if (FAN > 0 || u < nf) {
                    const float4 xv = __ldg(reinterpret_cast<const float4*>(xr[u] + b));
                    v[u] += gd[0] * xv.x + gd[1] * xv.y + gd[2] * xv.z + gd[3] * xv.w;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < F + 3; ++u) v[u] = warp_sum(v[u]);
        if (part) {
            if (lane == 0) {
                float* pp = part + ((size_t)i * gridDim.y + blockIdx.y) * (fan + 3);
                for (int u = 0; u < nf; ++u) pp[f0 + u] = v[u];
                if (first) { pp[fan] = v[F]; pp[fan + 1] = v[F + 1]; pp[fan + 2] = v[F + 2]; }
            }
        } else if (lane == 0) {
            if (first) {
                const int id = __ldg(&n0[s]);
                ggain[id] += v[F];
                gtheta[id] += -v[F + 1] * __ldg(&rsig[s]);
                gin_b[s] += v[F + 2];
            }
            for (int u = 0; u < nf; ++u) gin_w[e0 + f0 + u] += v[u];
        }
        if (fan == 0) break;
    }
}

// the plug backward's per-split sums added in split order: a thread per (listed row, column of the row's fan + 3
// sums) - in_w of each plug column, then gain, theta and in_b
__global__ void __launch_bounds__(256) k_plug_bwd_reduce(const float* __restrict__ part, const int* __restrict__ list,
                                                         const int* __restrict__ n0, const float* __restrict__ rsig,
                                                         float* __restrict__ ggain, float* __restrict__ gtheta,
                                                         float* __restrict__ gin_w, float* __restrict__ gin_b,
                                                         int n_list, int fan, int splits) {
    pdl_enter();
    const int k = blockIdx.x * blockDim.x + threadIdx.x, w = fan + 3;
    if (k >= n_list * w) return;
    const int i = k / w, col = k - i * w;
    float v = 0.f;
    for (int sp = 0; sp < splits; ++sp) v += part[((size_t)i * splits + sp) * w + col];
    const int s = __ldg(&list[i]);
    if (col < fan) gin_w[(size_t)s * fan + col] += v;
    else if (col == fan) ggain[__ldg(&n0[s])] += v;
    else if (col == fan + 1) gtheta[__ldg(&n0[s])] += -v * __ldg(&rsig[s]);
    else gin_b[s] += v;
}

// ---------------------------------------------------------------- optimiser
// partial sums of squares of the flat gradient (one per CTA); the host or k_norm_final adds them in order
__global__ void k_sumsq(const float* __restrict__ g, long long n, float* __restrict__ part) {
    pdl_enter();
    __shared__ float red[kWarps];
    float v[1] = {0.f};
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        v[0] = fmaf(g[i], g[i], v[0]);
    block_sum<1>(v, red);
    if (threadIdx.x == 0) part[blockIdx.x] = v[0];
}
// norm[0] = sqrt(sum of part); norm[1] = gradient scale for clipping to max_norm (1 if not clipping)
__global__ void k_norm_final(const float* __restrict__ part, int n, float max_norm, float* __restrict__ norm) {
    pdl_enter();
    __shared__ float red[kWarps];
    float v[1] = {0.f};
    for (int i = threadIdx.x; i < n; i += blockDim.x) v[0] += part[i];
    block_sum<1>(v, red);
    if (threadIdx.x == 0) {
        float g = sqrtf(v[0]);
        norm[0] = g;
        norm[1] = (max_norm > 0.f && g > max_norm) ? max_norm / g : 1.f;
    }
}
// Adam over the flat parameter buffer: segments [0, seg1) at lr0 (strengths), [seg1, seg2) at lr1 (gain, theta),
// the rest at lr2 (plugs). Gradient scale from norm[1] when `scale` is given. Four elements per thread step (the
// buffers are separate 256-byte aligned allocations); each element's arithmetic is the scalar update.
__device__ __forceinline__ void adam1(float& p, float g, float& m, float& v, float& e, float lr, float c1, float c2,
                                      float decay) {
    const float mi = 0.9f * m + 0.1f * g, vi = 0.999f * v + 0.001f * g * g;
    m = mi; v = vi;
    p = p - lr * (mi / c1) / (sqrtf(vi / c2) + 1e-8f);
    e = decay * e + (1.f - decay) * p;
}
__global__ void k_adam(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                       float* __restrict__ ema, long long n, long long seg1, long long seg2, float lr0, float lr1,
                       float lr2, float c1, float c2, const float* __restrict__ scale, float decay) {
    pdl_enter();
    const float gs = scale ? scale[1] : 1.f;
    const long long n4 = n >> 2, stride = (long long)gridDim.x * blockDim.x;
    for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < n4; q += stride) {
        float4 P = reinterpret_cast<float4*>(p)[q], M = reinterpret_cast<float4*>(m)[q];
        float4 V = reinterpret_cast<float4*>(v)[q], E = reinterpret_cast<float4*>(ema)[q];
        const float4 G = __ldg(reinterpret_cast<const float4*>(g) + q);
        float* pp = &P.x; float* mm = &M.x; float* vv = &V.x; float* ee = &E.x;
        const float gg[4] = {G.x, G.y, G.z, G.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const long long i = 4 * q + k;
            adam1(pp[k], gg[k] * gs, mm[k], vv[k], ee[k], i < seg1 ? lr0 : (i < seg2 ? lr1 : lr2), c1, c2, decay);
        }
        reinterpret_cast<float4*>(p)[q] = P; reinterpret_cast<float4*>(m)[q] = M;
        reinterpret_cast<float4*>(v)[q] = V; reinterpret_cast<float4*>(ema)[q] = E;
    }
    for (long long i = 4 * n4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        adam1(p[i], g[i] * gs, m[i], v[i], ema[i], i < seg1 ? lr0 : (i < seg2 ? lr1 : lr2), c1, c2, decay);
}

}  // namespace fg
