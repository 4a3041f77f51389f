// Tensor-core hop forward for 16-bit states (sm_100a: tcgen05 MMA with TMEM accumulators, bulk async copies,
// mbarriers).
//
// A hop's merged pairs split into HUB pairs - pairs whose source is one of the hop's K most-read source rows (picked
// at plan time; on a Zipf-sourced graph a few dozen sources carry most pairs) - and TAIL pairs (the rest). For a tile
// of 128 rows x 256 samples:
//   z[row, s] = sum over hubs k of W[row, k] * x[hub_k, s]      (tensor cores: one dense 128 x 256 x K product)
//             + sum over the row's tail pairs of w * x[src, s]   (CUDA cores, in the epilogue)
//             + drive[drow[row], s];   h = relu(gain * z - thr)
// W[row, k] is the row's folded pair weight for hub k (0 where the row does not read the hub), held as two 16-bit
// terms hi + lo (lo = the rounding error of hi), so the product keeps ~16 mantissa bits of the fp32 weight; the
// states are already 16-bit; products accumulate in fp32 in TMEM.
//
// Operand layouts (both K-major, no swizzle, the canonical core-matrix layout of the MMA's shared-memory
// descriptors): an operand of R rows x K elements is R/8 x K/8 core matrices of 8 rows x 16 bytes, core matrix
// (i, kk) at byte (i * K/8 + kk) * 128, row r of it at + r * 16; so the K-direction core-matrix stride (LBO) is 128 B
// and the 8-row-group stride (SBO) is K/8 * 128 B. The weights are stored in HBM per row tile in exactly this layout
// (hi block then lo block) and the hub states per 256-sample tile (gathered each hop by k_gather_hub), so each tile
// arrives in shared memory with one bulk copy.
//
// CTA roles (1 CTA per SM, persistent over work items {row tile, range of sample tiles}):
//   warp 16, lane 0 - loads the row tile's weights, streams hub-state tiles into a double buffer, issues the MMAs
//                     into one of two TMEM accumulators (2 x 256 columns) and commits them to mbarriers;
//   warps 0..15     - epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its 32 rows: one row per thread) and
//                     columns 64 (w / 4) .. + 63 of the tile (its 64 samples), adds the tail pairs, drive and
//                     activation, and stores the states.
// Every wait is bounded (about 2 s): on expiry the CTA records an error code, stops issuing work and releases TMEM.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace fg {

constexpr int kTcRows = 128;            // rows per tile (MMA M; TMEM lanes)
constexpr int kTcCols = 256;            // samples per tile (MMA N; TMEM columns per accumulator)
constexpr int kTcEpiWarps = 16;
constexpr int kTcThreads = 32 * (kTcEpiWarps + 1);
constexpr int kHubMax = 128;            // hub columns per hop at most (a multiple of 16)
constexpr long long kTcWaitCycles = 4000000000LL;   // ~2 s at the B200's clock

// error codes written to the handle's device error word
constexpr int kTcErrWaitW = 1, kTcErrWaitX = 2, kTcErrWaitXEmpty = 3, kTcErrWaitAccEmpty = 4, kTcErrWaitAccFull = 5;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait for the phase with the given parity; false (and the CTA's abort flag set, the error recorded) when
// it does not complete within kTcWaitCycles or another role of the CTA has already given up
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, int* err, int code) {
    const long long t0 = clock64();
    while (!mbar_try(bar, parity)) {
        if (*abort) return false;
        if (clock64() - t0 > kTcWaitCycles) {
            *abort = 1;
            atomicCAS(err, 0, code);
            return false;
        }
    }
    return true;
}
// global -> shared bulk copy (16-byte aligned, size a multiple of 16) completing on an mbarrier
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// shared-memory matrix descriptor: K-major, no swizzle, start / LBO / SBO in bytes, descriptor version 1
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// instruction descriptor of kind::f16: fp32 accumulator, A and B both bf16 (fmt 1) or both f16 (fmt 0), both K-major
template <class T> struct MmaFmt { static constexpr uint32_t v = 1; };
template <> struct MmaFmt<__half> { static constexpr uint32_t v = 0; };
template <class T>
__device__ __forceinline__ constexpr uint32_t mma_idesc() {
    return (1u << 4) | (MmaFmt<T>::v << 7) | (MmaFmt<T>::v << 10) | ((uint32_t)(kTcCols >> 3) << 17) |
           ((uint32_t)(kTcRows >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// 32 lanes x 32 columns of fp32: thread l gets lane (base lane + l), columns col .. col + 31
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 columns of fp32: thread l gets lane (base lane + l), columns col .. col + 15 (complete after
// tmem_wait_ld)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- plan-time data kept per weight version
// the hub columns of the folded weights, split into hi + lo 16-bit terms, scattered into the per-row-tile operand
// layout: map[i] = {merged pair index, element offset of the hi term (the lo term is 128 K elements later)}
template <class T> __device__ __forceinline__ T to16(float v);
template <> __device__ __forceinline__ __nv_bfloat16 to16(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half to16(float v) { return __float2half_rn(v); }
template <class T> __device__ __forceinline__ float from16(T v);
template <> __device__ __forceinline__ float from16(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float from16(__half v) { return __half2float(v); }

template <class T>
__global__ void k_fold_hub(const int2* __restrict__ map, const int2* __restrict__ pairs, T* __restrict__ wt, int n,
                           int K) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int2 m = __ldg(&map[i]);
    const float w = __int_as_float(__ldg(&pairs[m.x]).y);
    const T hi = to16<T>(w);
    wt[m.y] = hi;
    wt[m.y + (size_t)kTcRows * K] = to16<T>(w - from16<T>(hi));
}

// hub states of one hop in the MMA's B-operand layout, per 256-sample tile: thread (sample s, group g of 8 hubs)
// writes the 16 bytes of row s of core matrix (s / 8, g). hubs[k] < 0 (padding) gives zeros.
template <class T>
__global__ void __launch_bounds__(256) k_gather_hub(const T* __restrict__ x, const int* __restrict__ hubs,
                                                    T* __restrict__ xh, int K, int ld) {
    const int tile = blockIdx.x, g = blockIdx.y, sl = threadIdx.x;
    const int s = tile * kTcCols + sl;
    uint16_t v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int hb = __ldg(&hubs[g * 8 + i]);
        v[i] = hb >= 0 ? __ldg(reinterpret_cast<const uint16_t*>(x) + (size_t)hb * ld + s) : (uint16_t)0;
    }
    uint4 q;
    q.x = v[0] | ((uint32_t)v[1] << 16); q.y = v[2] | ((uint32_t)v[3] << 16);
    q.z = v[4] | ((uint32_t)v[5] << 16); q.w = v[6] | ((uint32_t)v[7] << 16);
    T* dst = xh + (size_t)tile * kTcCols * K + ((size_t)(sl >> 3) * (K >> 3) + g) * 64 + (sl & 7) * 8;
    *reinterpret_cast<uint4*>(dst) = q;
}

struct TcHop {
    const void* wt;          // [row tiles][hi, lo][128 x K] operand layout
    const void* xh;          // [sample tiles][256 x K] operand layout
    const void* hp;          // source layer [n_src][ld], 16-bit
    const int2* pairs;       // this hop's merged pairs {src, folded weight}; a row's tail pairs come first
    const int* pptr;         // [rows + 1] first pair of each row
    const int* pmid;         // [rows] first hub pair of each row (= end of its tail pairs)
    const int* sched;        // [rows] row of each slot; a row tile is 128 consecutive slots
    const float* rgain;
    const float* rthr;
    const int* drow;         // nullptr or [rows]: sensory row re-driven into the row, or -1
    const float* drive;      // [n_s][ld]
    void* h;                 // this layer [rows][ld]
    int* err;
    int n_rows, ld, K, n_items, tiles_per_item, n_sample_tiles, items_per_row_tile;
};

// the tail pairs of one row for 32 samples (4 x 16 bytes of each source row) multiplied into v
template <class T>
__device__ __forceinline__ void tail32(const char* base, const int2* pairs, int e, int e1, unsigned row_bytes,
                                       float (&v)[32]) {
    for (; e + 2 <= e1; e += 2) {
        const int2 p = __ldg(&pairs[e]), q = __ldg(&pairs[e + 1]);
        const char* ap = base + (unsigned long long)(unsigned)p.x * row_bytes;
        const char* aq = base + (unsigned long long)(unsigned)q.x * row_bytes;
        uint4 ra[4], rb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) ra[i] = __ldg(reinterpret_cast<const uint4*>(ap) + i);
#pragma unroll
        for (int i = 0; i < 4; ++i) rb[i] = __ldg(reinterpret_cast<const uint4*>(aq) + i);
        const float2 wp = make_float2(__int_as_float(p.y), __int_as_float(p.y));
        const float2 wq = make_float2(__int_as_float(q.y), __int_as_float(q.y));
        const T* tag = nullptr;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t wa[4] = {ra[i].x, ra[i].y, ra[i].z, ra[i].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 f;
                unpack2(tag, wa[j], f);
                float2 acc = make_float2(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
                acc = __ffma2_rn(wp, f, acc);
                v[8 * i + 2 * j] = acc.x; v[8 * i + 2 * j + 1] = acc.y;
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t wb[4] = {rb[i].x, rb[i].y, rb[i].z, rb[i].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 f;
                unpack2(tag, wb[j], f);
                float2 acc = make_float2(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
                acc = __ffma2_rn(wq, f, acc);
                v[8 * i + 2 * j] = acc.x; v[8 * i + 2 * j + 1] = acc.y;
            }
        }
    }
    if (e < e1) {
        const int2 p = __ldg(&pairs[e]);
        const char* ap = base + (unsigned long long)(unsigned)p.x * row_bytes;
        uint4 ra[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) ra[i] = __ldg(reinterpret_cast<const uint4*>(ap) + i);
        const float2 wp = make_float2(__int_as_float(p.y), __int_as_float(p.y));
        const T* tag = nullptr;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t wa[4] = {ra[i].x, ra[i].y, ra[i].z, ra[i].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 f;
                unpack2(tag, wa[j], f);
                float2 acc = make_float2(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
                acc = __ffma2_rn(wp, f, acc);
                v[8 * i + 2 * j] = acc.x; v[8 * i + 2 * j + 1] = acc.y;
            }
        }
    }
}

// 32 activated states of one row: 16-bit (4 x 16 bytes) or fp32 (8 x 16 bytes)
__device__ __forceinline__ void store32(__nv_bfloat16* p, const float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
        reinterpret_cast<uint4*>(p)[i] = make_uint4(pack_bf16(v[8 * i], v[8 * i + 1]), pack_bf16(v[8 * i + 2], v[8 * i + 3]),
                                                    pack_bf16(v[8 * i + 4], v[8 * i + 5]), pack_bf16(v[8 * i + 6], v[8 * i + 7]));
}
__device__ __forceinline__ void store32(__half* p, const float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
        reinterpret_cast<uint4*>(p)[i] = make_uint4(pack_f16(v[8 * i], v[8 * i + 1]), pack_f16(v[8 * i + 2], v[8 * i + 3]),
                                                    pack_f16(v[8 * i + 4], v[8 * i + 5]), pack_f16(v[8 * i + 6], v[8 * i + 7]));
}
__device__ __forceinline__ void store32(float* p, const float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4*>(p)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// work item i: row tile i / items_per_row_tile, sample tiles [j * tiles_per_item, ...) with j = i % items_per_row_tile
__device__ __forceinline__ void tc_item(const TcHop& a, int i, int& rt, int& st0, int& st1) {
    rt = i / a.items_per_row_tile;
    st0 = (i - rt * a.items_per_row_tile) * a.tiles_per_item;
    st1 = min(a.n_sample_tiles, st0 + a.tiles_per_item);
}

template <class T, class TO>
__global__ void __launch_bounds__(kTcThreads, 1) k_hop_tc(const TcHop a) {
    extern __shared__ __align__(1024) unsigned char smem[];
    const int K = a.K;
    const uint32_t w_bytes = 2u * kTcRows * K * 2u;            // hi + lo operand blocks of one row tile
    const uint32_t x_bytes = (uint32_t)kTcCols * K * 2u;        // one sample tile of hub states
    unsigned char* sw = smem;                                   // weights
    unsigned char* sx = smem + w_bytes;                         // hub states, 2 buffers
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + w_bytes + 2 * x_bytes);
    // bars: 0 w_full, 1-2 x_full, 3-4 x_empty, 5-6 acc_full, 7-8 acc_empty
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t b0 = smem_u32(bars);
    auto bar = [&](int i) { return b0 + 8u * (uint32_t)i; };

    if (threadIdx.x == 0) {
        mbar_init(bar(0), 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar(1 + b), 1);
            mbar_init(bar(3 + b), 1);
            mbar_init(bar(5 + b), 1);
            mbar_init(bar(7 + b), kTcEpiWarps);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kTcEpiWarps) {                                  // the control warp owns the TMEM allocation
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * kTcCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kTcEpiWarps) {
        if (lane == 0) {
            const uint32_t idesc = mma_idesc<T>();
            const uint32_t sbo = (uint32_t)(K >> 3) * 128u;
            const uint32_t swa = smem_u32(sw), swl = swa + (uint32_t)kTcRows * K * 2u, sxa = smem_u32(sx);
            int it = 0, w_uses = 0, prev_rt = -1;
            bool ok = true;
            int item = blockIdx.x, rt = 0, st = 0, st1 = 0;
            if (item < a.n_items) {                           // the first tile's hub states
                tc_item(a, item, rt, st, st1);
                mbar_expect_tx(bar(1), x_bytes);
                bulk_g2s(sxa, reinterpret_cast<const char*>(a.xh) + (size_t)st * x_bytes, x_bytes, bar(1));
            }
            while (ok && item < a.n_items) {
                if (rt != prev_rt) {
                    // every MMA reading the old weights has completed once the last tile's accumulator is full
                    if (it > 0 && !mbar_wait(bar(5 + ((it - 1) & 1)), ((it - 1) >> 1) & 1, abort, a.err,
                                             kTcErrWaitAccFull)) { ok = false; break; }
                    mbar_expect_tx(bar(0), w_bytes);
                    bulk_g2s(swa, reinterpret_cast<const char*>(a.wt) + (size_t)rt * w_bytes, w_bytes, bar(0));
                    if (!mbar_wait(bar(0), w_uses & 1, abort, a.err, kTcErrWaitW)) { ok = false; break; }
                    ++w_uses;
                    prev_rt = rt;
                }
                const int b = it & 1, u = it >> 1;
                const uint32_t xb = sxa + (uint32_t)b * x_bytes;
                // the accumulator's previous tile has been read out, and this tile's hub states have landed
                if (it >= 2 && !mbar_wait(bar(7 + b), (u - 1) & 1, abort, a.err, kTcErrWaitAccEmpty)) { ok = false; break; }
                if (!mbar_wait(bar(1 + b), u & 1, abort, a.err, kTcErrWaitX)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * kTcCols);
                for (int kk = 0; kk < K / 16; ++kk)
                    mma_f16(d, smem_desc(swa + kk * 256u, 128u, sbo), smem_desc(xb + kk * 256u, 128u, sbo), idesc, kk > 0);
                for (int kk = 0; kk < K / 16; ++kk)
                    mma_f16(d, smem_desc(swl + kk * 256u, 128u, sbo), smem_desc(xb + kk * 256u, 128u, sbo), idesc, 1u);
                mma_commit(bar(3 + b));
                mma_commit(bar(5 + b));
                // next tile; its hub states go into the other buffer once the MMAs of the tile before this one are done
                ++it;
                if (++st == st1) {
                    item += gridDim.x;
                    if (item < a.n_items) tc_item(a, item, rt, st, st1);
                }
                if (item < a.n_items) {
                    const int b2 = it & 1, u2 = it >> 1;
                    if (it >= 2 && !mbar_wait(bar(3 + b2), (u2 - 1) & 1, abort, a.err, kTcErrWaitXEmpty)) { ok = false; break; }
                    mbar_expect_tx(bar(1 + b2), x_bytes);
                    bulk_g2s(sxa + (uint32_t)b2 * x_bytes, reinterpret_cast<const char*>(a.xh) + (size_t)st * x_bytes,
                             x_bytes, bar(1 + b2));
                }
            }
            // the last accumulator must be complete before the allocation is released
            if (ok && it > 0) mbar_wait(bar(5 + ((it - 1) & 1)), ((it - 1) >> 1) & 1, abort, a.err, kTcErrWaitAccFull);
        }
        __syncwarp();
    } else {
        const int q = warp & 3, c = warp >> 2;
        const unsigned row_bytes = (unsigned)a.ld * 2u;
        int it = 0;
        bool ok = true;
        for (int item = blockIdx.x; ok && item < a.n_items; item += gridDim.x) {
            int rt, st0, st1;
            tc_item(a, item, rt, st0, st1);
            const int slot = rt * kTcRows + q * 32 + lane;
            const bool valid = slot < a.n_rows;
            int t = 0, e0 = 0, e1 = 0, d = -1;
            float g = 0.f, th = 0.f;
            if (valid) {
                t = __ldg(&a.sched[slot]);
                e0 = __ldg(&a.pptr[t]);
                e1 = __ldg(&a.pmid[t]);
                g = __ldg(&a.rgain[t]);
                th = __ldg(&a.rthr[t]);
                if (a.drow) d = __ldg(&a.drow[t]);
            }
            for (int st = st0; st < st1; ++st, ++it) {
                const int b = it & 1, u = it >> 1;
                // the warp leaves together: tcgen05.ld below is warp-collective
                const bool full = mbar_wait(bar(5 + b), u & 1, abort, a.err, kTcErrWaitAccFull);
                if (!__all_sync(0xffffffffu, full)) { ok = false; break; }
                tc_fence_after();
#pragma unroll 1
                for (int half = 0; half < 2; ++half) {
                    float v[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * kTcCols + c * 64 + half * 32), v);
                    if (half == 1) {                          // this warp is done with the accumulator
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(bar(7 + b));
                    }
                    if (valid) {
                        const int s0 = st * kTcCols + c * 64 + half * 32;
                        tail32<T>(reinterpret_cast<const char*>(reinterpret_cast<const T*>(a.hp) + s0), a.pairs, e0, e1,
                                  row_bytes, v);
                        if (d >= 0) {
                            const float4* dr = reinterpret_cast<const float4*>(a.drive + (size_t)d * a.ld + s0);
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                const float4 z = __ldg(dr + i);
                                v[4 * i] += z.x; v[4 * i + 1] += z.y; v[4 * i + 2] += z.z; v[4 * i + 3] += z.w;
                            }
                        }
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = fmaxf(fmaf(g, v[i], -th), 0.f);
                        store32(reinterpret_cast<TO*>(a.h) + (size_t)t * a.ld + s0, v);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcEpiWarps) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTcCols) : "memory");
    }
}

}  // namespace fg
