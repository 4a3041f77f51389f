// Output plug forward on the tensor cores (sm_100a: tcgen05 kind::tf32 MMA, TMEM accumulator, bulk async copies,
// mbarriers): part[slice][a][b] = sum over the slice's dn columns j of out_w[a, j] * hK[dn[j], b] for one tile of 128
// samples x 96 actions (90 used, padded with zero weights), the slices' partials then added in order with the bias by
// k_out_reduce (the slice count is fixed by the graph, so a sample's logits do not depend on the batch it is in).
//
// fp32 accuracy from tf32 operands (3 x TF32): each fp32 operand x is split into hi = tf32(x) and lo = tf32(x - hi),
// and the product is accumulated as hi*hi + hi*lo + lo*hi (the dropped lo*lo term is ~2^-22 of the product); the
// tensor cores multiply tf32 values exactly and accumulate in fp32.
//
// MMA shape M = 128 samples, N = 96 actions, K = 8 columns per instruction, 32 columns (one chunk) per pipeline stage.
// Both operands are K-major in the canonical no-swizzle core-matrix layout: an operand of R rows x 32 tf32 columns is
// R/8 x 8 core matrices of 8 rows x 16 bytes (4 columns), core matrix (i, kk) at byte (i * 8 + kk) * 128, row r of it
// at + r * 16, so LBO (K direction) = 128 B and SBO (8-row groups) = 1024 B.
//   - out_w is folded into that layout once per weight version (k_fold_ow_tc: [chunk][hi, lo][96 x 32]) and arrives
//     in shared memory with one bulk copy per stage;
//   - hK's dn rows are gathered by 8 producer warps: warp w loads columns 4w .. 4w + 3 of the chunk (coalesced 128-byte
//     rows of 32 samples), splits them and writes each sample's 4 columns as one 16-byte core-matrix row (conflict-free
//     per quarter warp), then fences the writes for the tensor cores' (async proxy) reads.
// Warp 8, lane 0 issues the copies and the MMAs; the producer warps then read the accumulator out of TMEM (warp w:
// lanes 32 (w % 4) .., columns 48 (w / 4) ..) into the partial slab. Every wait is bounded (about 2 s): on expiry the
// CTA records an error code and stops.
#pragma once
#include "fg_kernels.cuh"
#include "fg_tcgen05.cuh"

namespace fg {

// Two stages (115 KB of shared memory) so that two CTAs share a SM and cover each other's gather latency: the forward
// output plug at batch 65,536 took 0.198 ms against 0.287 with three stages at one CTA a SM.
constexpr int kOtM = 128, kOtN = 96, kOtKC = 32, kOtStages = 2, kOtProd = 8;
constexpr int kOtThreads = 32 * (kOtProd + 1);
constexpr uint32_t kOtA = kOtM * kOtKC * 4;            // one term of a chunk of hK (16 KB)
constexpr uint32_t kOtB = kOtN * kOtKC * 4;            // one term of a chunk of out_w (12 KB)
constexpr uint32_t kOtStage = 2 * kOtA + 2 * kOtB;     // A hi, A lo, B hi, B lo
constexpr int kOtSmem = kOtStages * kOtStage + 128;
constexpr int kTcErrOutFull = 11, kTcErrOutEmpty = 12, kTcErrOutAcc = 13;

__device__ __forceinline__ uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
// kind::tf32 instruction descriptor: fp32 accumulator, A and B tf32 (format 2), both K-major, N = 96, M = 128
__device__ __forceinline__ constexpr uint32_t out_idesc() {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kOtN >> 3) << 17) | ((uint32_t)(kOtM >> 4) << 24);
}
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

// out_w [n_act][n_dn] -> wt [chunk][hi, lo][96 x 32] in the operand layout (zero past n_act actions and n_dn columns)
__device__ __forceinline__ void fold_ow_tc(int i, const float* __restrict__ ow, float* __restrict__ wt, int n_act,
                                           int n_dn, int chunks) {
    if (i >= chunks * kOtN * kOtKC) return;
    const int c = i / (kOtN * kOtKC), r = i - c * (kOtN * kOtKC), a = r / kOtKC, k = r - a * kOtKC;
    const int j = c * kOtKC + k;
    const float w = (a < n_act && j < n_dn) ? __ldg(&ow[(size_t)a * n_dn + j]) : 0.f;
    const uint32_t hi = to_tf32(w), lo = to_tf32(w - __uint_as_float(hi));
    const int off = ((a >> 3) * (kOtKC / 4) + (k >> 2)) * 32 + (a & 7) * 4 + (k & 3);
    float* base = wt + (size_t)c * 2 * kOtN * kOtKC;
    base[off] = __uint_as_float(hi);
    base[kOtN * kOtKC + off] = __uint_as_float(lo);
}

struct OutTc {
    const float* wt;         // folded out_w, [chunks][hi, lo][96 x 32]
    const int* dn;           // [n_dn] rows of hK read by the plug
    const float* hK;         // the top layer [rows][ld], fp32
    float* part;             // [slices][96][ld]
    int* err;
    int n_dn, B, ld, chunks, cps;    // cps: chunks per slice
};

__global__ void __launch_bounds__(kOtThreads, 2) k_out_tc(const OutTc a) {
    pdl_enter();
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOtStages * kOtStage);
    // bars: 0..2 stage full, 3..5 stage empty, 6 accumulator complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b0 = blockIdx.x * kOtM, slice = blockIdx.y;
    const int c0 = slice * a.cps, n = max(0, min(a.chunks, c0 + a.cps) - c0);
    const uint32_t bb = smem_u32(bars);
    auto bar = [&](int i) { return bb + 8u * (uint32_t)i; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kOtStages; ++s) {
            mbar_init(bar(s), kOtProd + 1);
            mbar_init(bar(kOtStages + s), 1);
        }
        mbar_init(bar(2 * kOtStages), 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kOtProd) {                                  // the control warp owns the TMEM allocation
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(128)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kOtProd) {
        if (lane == 0 && n > 0) {
            constexpr uint32_t idesc = out_idesc();
            bool ok = true;
            for (int i = 0; i < n; ++i) {
                const int s = i % kOtStages, u = i / kOtStages;
                if (i >= kOtStages && !mbar_wait(bar(kOtStages + s), (u - 1) & 1, abort, a.err, kTcErrOutEmpty)) {
                    ok = false;
                    break;
                }
                const uint32_t ah = smem_u32(smem + (size_t)s * kOtStage), al = ah + kOtA, bh = ah + 2 * kOtA,
                               bl = bh + kOtB;
                mbar_expect_tx(bar(s), 2 * kOtB);
                bulk_g2s(bh, a.wt + (size_t)(c0 + i) * 2 * kOtN * kOtKC, 2 * kOtB, bar(s));
                if (!mbar_wait(bar(s), u & 1, abort, a.err, kTcErrOutFull)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < kOtKC / 8; ++ks) {
                    const uint32_t o = (uint32_t)ks * 256u;
                    mma_tf32(tmem, smem_desc(ah + o, 128u, 1024u), smem_desc(bh + o, 128u, 1024u), idesc,
                             (i > 0 || ks > 0) ? 1u : 0u);
                    mma_tf32(tmem, smem_desc(ah + o, 128u, 1024u), smem_desc(bl + o, 128u, 1024u), idesc, 1u);
                    mma_tf32(tmem, smem_desc(al + o, 128u, 1024u), smem_desc(bh + o, 128u, 1024u), idesc, 1u);
                }
                mma_commit(bar(kOtStages + s));
            }
            if (ok) mma_commit(bar(2 * kOtStages));
        }
        __syncwarp();
    } else {
        bool ok = true;
        for (int i = 0; i < n; ++i) {
            const int s = i % kOtStages, u = i / kOtStages;
            if (i >= kOtStages) {
                const bool w_ok = mbar_wait(bar(kOtStages + s), (u - 1) & 1, abort, a.err, kTcErrOutEmpty);
                if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
            }
            unsigned char* st = smem + (size_t)s * kOtStage;
            const int j0 = (c0 + i) * kOtKC + 4 * warp;
            const float* rows[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
                rows[k] = j0 + k < a.n_dn ? a.hK + (size_t)__ldg(&a.dn[j0 + k]) * a.ld : nullptr;
            float v[4][4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int b = b0 + lane + 32 * m;
#pragma unroll
                for (int k = 0; k < 4; ++k) v[m][k] = (rows[k] && b < a.B) ? __ldg(rows[k] + b) : 0.f;
            }
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int sb = lane + 32 * m;
                uint4 hi, lo;
                hi.x = to_tf32(v[m][0]); lo.x = to_tf32(v[m][0] - __uint_as_float(hi.x));
                hi.y = to_tf32(v[m][1]); lo.y = to_tf32(v[m][1] - __uint_as_float(hi.y));
                hi.z = to_tf32(v[m][2]); lo.z = to_tf32(v[m][2] - __uint_as_float(hi.z));
                hi.w = to_tf32(v[m][3]); lo.w = to_tf32(v[m][3] - __uint_as_float(hi.w));
                const uint32_t off = ((uint32_t)(sb >> 3) * (kOtKC / 4) + (uint32_t)warp) * 128u + (uint32_t)(sb & 7) * 16u;
                *reinterpret_cast<uint4*>(st + off) = hi;
                *reinterpret_cast<uint4*>(st + kOtA + off) = lo;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> tensor-core reads
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(s));
        }
        // the accumulator into this slice's partial slab: thread = sample 32 (w % 4) + lane, 48 actions
        const int q = warp & 3, ch = warp >> 2;
        const int b = b0 + 32 * q + lane;
        float* pp = a.part + (size_t)slice * kOtN * a.ld + b;
        if (n == 0) {
            if (b < a.B)
                for (int c = 0; c < 48; ++c) pp[(size_t)(48 * ch + c) * a.ld] = 0.f;
        } else if (ok) {
            const bool full = mbar_wait(bar(2 * kOtStages), 0, abort, a.err, kTcErrOutAcc);
            if (__all_sync(0xffffffffu, full)) {
                tc_fence_after();
#pragma unroll
                for (int g = 0; g < 3; ++g) {
                    uint32_t r[16];
                    tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(48 * ch + 16 * g), r);
                    tmem_wait_ld();
                    if (b < a.B) {
#pragma unroll
                        for (int c = 0; c < 16; ++c) pp[(size_t)(48 * ch + 16 * g + c) * a.ld] = __uint_as_float(r[c]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kOtProd) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128) : "memory");
    }
}


// ---------------------------------------------------------------- output plug backward: gh = out_w^T dl
// gh[dn[j], b] = sum_a out_w[a, j] * dl[a, b] on the tensor cores, the same 3 x TF32 split: M = 128 samples, N = 128 dn
// columns per column tile, K = the 96 (padded) actions in 3 chunks of 32. A CTA owns one 128-sample tile and a run of
// column tiles: its 8 producer warps gather and split dl's rows once (the A operand, all 3 chunks, resident in shared
// memory; lane l loads samples 4l .. 4l + 3 of 4 action rows with 16-byte loads and writes each sample's 4 actions as
// one core-matrix row), the control thread streams each column tile's folded out_w (k_fold_owbt:
// [column tile][chunk][hi, lo][128 x 32]) through a 3-stage bulk-copy ring and issues the MMAs into one of two TMEM
// accumulators, and the same 8 warps then read each finished tile out (warp w: samples 32 (w % 4) .., columns
// 64 (w / 4) ..) and write its gh rows (a warp store = 32 consecutive samples of one row).
constexpr int kObN = 128, kObChunks = 3;
// dl^T's operand: 128 samples x 32 actions per chunk and term, 8-row groups 1040 B apart (one 16-byte pad each), so the
// 16-byte rows a quarter warp writes (lane l: samples 4l .. 4l + 3) fall in 8 different bank groups
constexpr uint32_t kObSBO = 8 * 128 + 16;
constexpr uint32_t kObA = 128 / 8 * kObSBO;
constexpr uint32_t kObB = kObN * kOtKC * 4;                     // one term of one chunk of out_w^T (16 KB)
constexpr uint32_t kObStage = 2 * kObB;
constexpr int kObSmem = kObChunks * 2 * kObA + 3 * kObStage + 128;
constexpr int kTcErrObA = 21, kTcErrObW = 22, kTcErrObEmpty = 23, kTcErrObAccEmpty = 24, kTcErrObAccFull = 25;
static_assert(kObChunks * kOtKC == 96, "the padded action count");

__device__ __forceinline__ constexpr uint32_t ob_idesc() {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kObN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// out_w [n_act][n_dn] -> wt [column tile][chunk][hi, lo][128 columns x 32 actions] in the K-major operand layout
__device__ __forceinline__ void fold_owbt(int i, const float* __restrict__ ow, float* __restrict__ wt, int n_act,
                                          int n_dn, int n_tiles) {
    if (i >= n_tiles * kObChunks * kObN * kOtKC) return;
    const int blk = i / (kObN * kOtKC), r = i - blk * (kObN * kOtKC);
    const int t = blk / kObChunks, c = blk - t * kObChunks;
    const int j = r / kOtKC, k = r - j * kOtKC;
    const int col = t * kObN + j, a = c * kOtKC + k;
    const float w = (a < n_act && col < n_dn) ? __ldg(&ow[(size_t)a * n_dn + col]) : 0.f;
    const uint32_t hi = to_tf32(w), lo = to_tf32(w - __uint_as_float(hi));
    const int off = ((j >> 3) * (kOtKC / 4) + (k >> 2)) * 32 + (j & 7) * 4 + (k & 3);
    float* base = wt + (size_t)blk * 2 * kObN * kOtKC;
    base[off] = __uint_as_float(hi);
    base[kObN * kOtKC + off] = __uint_as_float(lo);
}

struct OutBh {
    const float* wt;         // folded out_w^T
    const float* dl;         // [n_act][ld]
    const int* dn;
    float* gh;               // the top layer's gradient rows [rows][ld]; rows dn[j] are written
    int* err;
    int n_act, n_dn, B, ld, n_tiles, tpg;    // column tiles; column tiles per CTA
};

__global__ void __launch_bounds__(kOtThreads, 1) k_out_bwd_h_tc(const OutBh a) {
    pdl_enter();
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* sa = smem;                                      // A: [chunk][hi, lo] of kObA bytes
    unsigned char* sw = smem + kObChunks * 2 * kObA;               // W ring: 3 stages of [hi, lo]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sw + 3 * kObStage);
    // bars: 0 A ready, 1..3 W full, 4..6 W empty, 7..8 accumulator full, 9..10 accumulator empty
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b0 = blockIdx.x * 128, t0 = blockIdx.y * a.tpg;
    const int nt = max(0, min(a.n_tiles, t0 + a.tpg) - t0);
    const uint32_t bb = smem_u32(bars);
    auto bar = [&](int i) { return bb + 8u * (uint32_t)i; };

    if (threadIdx.x == 0) {
        mbar_init(bar(0), kOtProd);
        for (int s = 0; s < 3; ++s) {
            mbar_init(bar(1 + s), 1);
            mbar_init(bar(4 + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar(7 + b), 1);
            mbar_init(bar(9 + b), kOtProd);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kOtProd) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(256)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kOtProd) {
        if (lane == 0 && nt > 0) {
            constexpr uint32_t idesc = ob_idesc();
            const int n = nt * kObChunks;                          // chunks over all of this CTA's column tiles
            auto copy_w = [&](int g) {
                const int s = g % 3, t = t0 + g / kObChunks, c = g % kObChunks;
                mbar_expect_tx(bar(1 + s), kObStage);
                bulk_g2s(smem_u32(sw + (size_t)s * kObStage),
                         a.wt + ((size_t)t * kObChunks + c) * 2 * kObN * kOtKC, kObStage, bar(1 + s));
            };
            bool ok = true;
            for (int g = 0; g < min(n, 3); ++g) copy_w(g);
            if (!mbar_wait(bar(0), 0, abort, a.err, kTcErrObA)) ok = false;
            for (int g = 0; ok && g < n; ++g) {
                const int s = g % 3, c = g % kObChunks, it = g / kObChunks, ab = it & 1;
                if (c == 0 && it >= 2 &&
                    !mbar_wait(bar(9 + ab), ((it >> 1) - 1) & 1, abort, a.err, kTcErrObAccEmpty)) { ok = false; break; }
                if (!mbar_wait(bar(1 + s), (g / 3) & 1, abort, a.err, kTcErrObW)) { ok = false; break; }
                tc_fence_after();
                const uint32_t ah = smem_u32(sa + (size_t)c * 2 * kObA), al = ah + kObA;
                const uint32_t wh = smem_u32(sw + (size_t)s * kObStage), wl = wh + kObB;
                const uint32_t d = tmem + (uint32_t)(ab * kObN);
#pragma unroll
                for (int ks = 0; ks < kOtKC / 8; ++ks) {
                    const uint32_t o = (uint32_t)ks * 256u;
                    mma_tf32(d, smem_desc(ah + o, 128u, kObSBO), smem_desc(wh + o, 128u, 1024u), idesc,
                             (c > 0 || ks > 0) ? 1u : 0u);
                    mma_tf32(d, smem_desc(ah + o, 128u, kObSBO), smem_desc(wl + o, 128u, 1024u), idesc, 1u);
                    mma_tf32(d, smem_desc(al + o, 128u, kObSBO), smem_desc(wh + o, 128u, 1024u), idesc, 1u);
                }
                mma_commit(bar(4 + s));
                if (c == kObChunks - 1) mma_commit(bar(7 + ab));
                if (g >= 1 && g + 2 < n) {                         // refill the previous chunk's stage
                    const int sp = (g - 1) % 3;
                    if (!mbar_wait(bar(4 + sp), ((g - 1) / 3) & 1, abort, a.err, kTcErrObEmpty)) { ok = false; break; }
                    copy_w(g + 2);
                }
            }
        }
        __syncwarp();
    } else {
        // A: dl's rows for this sample tile, transposed and split; warp w: actions 4w .. 4w + 3 of each chunk
        const int bl = b0 + 4 * lane;
        const bool in = bl < a.B;
        for (int c = 0; c < kObChunks; ++c) {
            float4 v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int act = c * kOtKC + 4 * warp + k;
                v[k] = (in && act < a.n_act) ? __ldg(reinterpret_cast<const float4*>(a.dl + (size_t)act * a.ld + bl))
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            unsigned char* st = sa + (size_t)c * 2 * kObA;
            const float* f0 = &v[0].x;
            const float* f1 = &v[1].x;
            const float* f2 = &v[2].x;
            const float* f3 = &v[3].x;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int sb = 4 * lane + q;
                uint4 hi, lo;
                hi.x = to_tf32(f0[q]); lo.x = to_tf32(f0[q] - __uint_as_float(hi.x));
                hi.y = to_tf32(f1[q]); lo.y = to_tf32(f1[q] - __uint_as_float(hi.y));
                hi.z = to_tf32(f2[q]); lo.z = to_tf32(f2[q] - __uint_as_float(hi.z));
                hi.w = to_tf32(f3[q]); lo.w = to_tf32(f3[q] - __uint_as_float(hi.w));
                const uint32_t off = (uint32_t)(sb >> 3) * kObSBO + (uint32_t)warp * 128u + (uint32_t)(sb & 7) * 16u;
                *reinterpret_cast<uint4*>(st + off) = hi;
                *reinterpret_cast<uint4*>(st + kObA + off) = lo;
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(0));
        // epilogue: each finished column tile into gh
        const int q = warp & 3, ch = warp >> 2;
        const int b = b0 + 32 * q + lane;
        for (int it = 0; it < nt; ++it) {
            const int ab = it & 1;
            const bool full = mbar_wait(bar(7 + ab), (it >> 1) & 1, abort, a.err, kTcErrObAccFull);
            if (!__all_sync(0xffffffffu, full)) break;
            tc_fence_after();
            uint32_t r[4][16];
#pragma unroll
            for (int g = 0; g < 4; ++g)
                tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(ab * kObN + 64 * ch + 16 * g), r[g]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(9 + ab));
            const int j0 = (t0 + it) * kObN + 64 * ch;
            if (b < a.B) {
#pragma unroll
                for (int g = 0; g < 4; ++g)
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int j = j0 + 16 * g + e;
                        if (j < a.n_dn) a.gh[(size_t)__ldg(&a.dn[j]) * a.ld + b] = __uint_as_float(r[g][e]);
                    }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kOtProd) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
    }
}

// ---------------------------------------------------------------- output plug backward: gW = dl h^T
// part[slice][a][j] = sum over the slice's samples b of dl[a, b] * h[dn[j], b] (column j = n_dn is the bias: h = 1) on
// the tensor cores, the same 3 x TF32 split: M = 128 columns, N = 96 (padded) actions, K = the slice's samples in chunks
// of 32. Both operands are K-major as they lie in memory (rows of samples), so 8 producer warps only gather, split and
// place them: a warp load reads 4 rows x 32 samples (lane l: row l / 8, samples 4 (l % 8) ..), and each lane writes its
// 4 samples as one 16-byte core-matrix row. The K-direction stride is padded to 144 B (LBO; 8-row groups 1152 B apart),
// so the 8 rows a quarter warp writes (core matrices 0..7 along K) fall in 8 different bank groups. The loads of the
// next chunk are issued before this chunk is written. The slices' partials are added in order by k_out_bwd_reduce.
constexpr uint32_t kOwLBO = 144, kOwSBO = 8 * kOwLBO;
constexpr uint32_t kOwA = 128 / 8 * kOwSBO, kOwB = 96 / 8 * kOwSBO;
constexpr uint32_t kOwStage = 2 * kOwA + 2 * kOwB;
constexpr int kOwStages = 3, kOwRowGroups = (128 + 96) / 4;       // 4-row load groups per chunk (7 per warp)
constexpr int kOwSmem = kOwStages * kOwStage + 128;
constexpr int kTcErrOwFull = 31, kTcErrOwEmpty = 32, kTcErrOwAcc = 33;
static_assert(kOwRowGroups % kOtProd == 0, "row groups split evenly over the producer warps");

__device__ __forceinline__ constexpr uint32_t ow_idesc() {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(96 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

struct OutBw {
    const float* dl;         // [n_act][ld]
    const float* hK;         // the top layer [rows][ld]
    const int* dn;
    float* part;             // [slices][n_act][n_dn + 1]
    int* err;
    int n_act, n_dn, B, ld, slice_len;      // slice_len: a multiple of 32
};

__global__ void __launch_bounds__(kOtThreads, 1) k_out_bwd_w_tc(const OutBw a) {
    pdl_enter();
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOwStages * kOwStage);
    // bars: 0..2 stage full, 3..5 stage empty, 6 accumulator complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j0 = blockIdx.x * 128, slice = blockIdx.y;
    const int s0 = slice * a.slice_len, s1 = min(a.B, s0 + a.slice_len);
    const int n = max(0, (s1 - s0 + kOtKC - 1) / kOtKC);
    const uint32_t bb = smem_u32(bars);
    auto bar = [&](int i) { return bb + 8u * (uint32_t)i; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kOwStages; ++s) {
            mbar_init(bar(s), kOtProd);
            mbar_init(bar(kOwStages + s), 1);
        }
        mbar_init(bar(2 * kOwStages), 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kOtProd) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(128)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kOtProd) {
        if (lane == 0 && n > 0) {
            constexpr uint32_t idesc = ow_idesc();
            bool ok = true;
            for (int i = 0; i < n; ++i) {
                const int s = i % kOwStages, u = i / kOwStages;
                if (!mbar_wait(bar(s), u & 1, abort, a.err, kTcErrOwFull)) { ok = false; break; }
                tc_fence_after();
                const uint32_t ah = smem_u32(smem + (size_t)s * kOwStage), al = ah + kOwA, bh = ah + 2 * kOwA,
                               bl = bh + kOwB;
#pragma unroll
                for (int ks = 0; ks < kOtKC / 8; ++ks) {
                    const uint32_t o = (uint32_t)ks * 2u * kOwLBO;
                    mma_tf32(tmem, smem_desc(ah + o, kOwLBO, kOwSBO), smem_desc(bh + o, kOwLBO, kOwSBO), idesc,
                             (i > 0 || ks > 0) ? 1u : 0u);
                    mma_tf32(tmem, smem_desc(ah + o, kOwLBO, kOwSBO), smem_desc(bl + o, kOwLBO, kOwSBO), idesc, 1u);
                    mma_tf32(tmem, smem_desc(al + o, kOwLBO, kOwSBO), smem_desc(bh + o, kOwLBO, kOwSBO), idesc, 1u);
                }
                mma_commit(bar(kOwStages + s));
            }
            if (ok) mma_commit(bar(2 * kOwStages));
        }
        __syncwarp();
    } else {
        const int rsub = lane >> 3, kk = lane & 7;         // row within a load group, core matrix along K
        constexpr int kG = kOwRowGroups / kOtProd;         // 7 load groups per warp
        // this lane's rows: A rows 0..127 (columns j0 + row; dn gathered; the bias column reads ones), B rows 128..223
        // (actions)
        const float* src[kG];
        bool ones[kG];
#pragma unroll
        for (int g = 0; g < kG; ++g) {
            const int row = 4 * (warp + kOtProd * g) + rsub;
            src[g] = nullptr;
            ones[g] = false;
            if (row < 128) {
                const int j = j0 + row;
                if (j < a.n_dn) src[g] = a.hK + (size_t)__ldg(&a.dn[j]) * a.ld;
                else ones[g] = j == a.n_dn;
            } else if (row - 128 < a.n_act) {
                src[g] = a.dl + (size_t)(row - 128) * a.ld;
            }
        }
        auto load = [&](int i, float4 (&v)[kG]) {
            const int b = s0 + i * kOtKC + 4 * kk;
            const bool in = b < s1;
#pragma unroll
            for (int g = 0; g < kG; ++g)
                v[g] = (in && src[g]) ? __ldg(reinterpret_cast<const float4*>(src[g] + b))
                                      : (in && ones[g] ? make_float4(1.f, 1.f, 1.f, 1.f) : make_float4(0.f, 0.f, 0.f, 0.f));
        };
        bool ok = true;
        float4 cur[kG], nxt[kG];
        if (n > 0) load(0, cur);
        for (int i = 0; i < n; ++i) {
            const int s = i % kOwStages, u = i / kOwStages;
            if (i + 1 < n) load(i + 1, nxt);
            if (i >= kOwStages) {
                const bool w_ok = mbar_wait(bar(kOwStages + s), (u - 1) & 1, abort, a.err, kTcErrOwEmpty);
                if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
            }
            unsigned char* st = smem + (size_t)s * kOwStage;
#pragma unroll
            for (int g = 0; g < kG; ++g) {
                const int row = 4 * (warp + kOtProd * g) + rsub;
                const bool is_a = row < 128;
                const int r = is_a ? row : row - 128;
                uint4 hi, lo;
                hi.x = to_tf32(cur[g].x); lo.x = to_tf32(cur[g].x - __uint_as_float(hi.x));
                hi.y = to_tf32(cur[g].y); lo.y = to_tf32(cur[g].y - __uint_as_float(hi.y));
                hi.z = to_tf32(cur[g].z); lo.z = to_tf32(cur[g].z - __uint_as_float(hi.z));
                hi.w = to_tf32(cur[g].w); lo.w = to_tf32(cur[g].w - __uint_as_float(hi.w));
                const uint32_t off = (uint32_t)(r >> 3) * kOwSBO + (uint32_t)kk * kOwLBO + (uint32_t)(r & 7) * 16u;
                unsigned char* base = st + (is_a ? 0u : 2u * kOwA);
                const uint32_t term = is_a ? kOwA : kOwB;
                *reinterpret_cast<uint4*>(base + off) = hi;
                *reinterpret_cast<uint4*>(base + term + off) = lo;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(s));
#pragma unroll
            for (int g = 0; g < kG; ++g) cur[g] = nxt[g];
        }
        // the accumulator (lane = column j, TMEM column = action) into this slice's partials
        const int q = warp & 3, ch = warp >> 2;
        const int j = j0 + 32 * q + lane, n_col = a.n_dn + 1;
        float* pp = a.part + (size_t)slice * a.n_act * n_col + j;
        if (n == 0) {
            if (j < n_col)
                for (int c = 0; c < 48; ++c)
                    if (48 * ch + c < a.n_act) pp[(size_t)(48 * ch + c) * n_col] = 0.f;
        } else if (ok) {
            const bool full = mbar_wait(bar(2 * kOwStages), 0, abort, a.err, kTcErrOwAcc);
            if (__all_sync(0xffffffffu, full)) {
                tc_fence_after();
#pragma unroll
                for (int g = 0; g < 3; ++g) {
                    uint32_t r[16];
                    tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(48 * ch + 16 * g), r);
                    tmem_wait_ld();
                    if (j < n_col) {
#pragma unroll
                        for (int c = 0; c < 16; ++c) {
                            const int act = 48 * ch + 16 * g + c;
                            if (act < a.n_act) pp[(size_t)act * n_col] = __uint_as_float(r[c]);
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kOtProd) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128) : "memory");
    }
}

// ---------------------------------------------------------------- the folds of one weight version, one launch
// Block ranges, the longest first: merged pair weights (fold_pairs), per-row gain / threshold / sigmoid
// (fold_neuron), out_w in the forward's tensor-core operand layout (fold_ow_tc) and, when training, in the backward's
// (fold_owbt). The four read the weights only and write disjoint arrays.
struct FoldArgs {
    const int* nid; const float* gain; const float* theta; float* rgain; float* rthr; float* rsig; int n_rows;
    const int* gptr; const int* gw; const float* W; int2* pairs; const int* tpos; int2* tpairs; int n_pairs;
    const float* ow; float* ow_tc; float* ow_bt; int n_act, n_dn, chunks, ob_tiles;
    int nb_pairs, nb_rows, nb_ow;                    // blocks of each range (the rest: fold_owbt)
};
__global__ void __launch_bounds__(kThreads) k_fold(const FoldArgs a) {
    pdl_enter();
    __shared__ float buf[kWarps][kFoldBuf];
    int b = blockIdx.x;
    if (b < a.nb_pairs) {
        fold_pairs(b, buf, a.gptr, a.gw, a.W, a.pairs, a.tpos, a.tpairs, a.n_pairs);
        return;
    }
    b -= a.nb_pairs;
    if (b < a.nb_rows) {
        fold_neuron(b * kThreads + threadIdx.x, a.nid, a.gain, a.theta, a.rgain, a.rthr, a.rsig, a.n_rows);
        return;
    }
    b -= a.nb_rows;
    if (b < a.nb_ow) {
        fold_ow_tc(b * kThreads + threadIdx.x, a.ow, a.ow_tc, a.n_act, a.n_dn, a.chunks);
        return;
    }
    b -= a.nb_ow;
    if (a.ow_bt) fold_owbt(b * kThreads + threadIdx.x, a.ow, a.ow_bt, a.n_act, a.n_dn, a.ob_tiles);
}

}  // namespace fg
