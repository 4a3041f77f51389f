// flyguy_b200 host side: NET.bin loading, the merged-pair plans, device buffers and the C-ABI of
// include/flyguy_b200.h. The reference's equivalent is the host half of flyguy/native/flyguy_train.cu (load_net
// 230-256, alloc_batch 308-317, forward_logits 320-332, backward 339-359, fc_* 553-629).
#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <numeric>
#include <type_traits>
#include <stdexcept>
#include <string>
#include <vector>

#include "fg_kernels.cuh"
#include "fg_outtc.cuh"
#include "flyguy_b200.h"


using namespace fg;

namespace {

struct Err : std::runtime_error {
    using std::runtime_error::runtime_error;
};
#define CK(call)                                                                                      \
    do {                                                                                              \
        cudaError_t e_ = (call);                                                                      \
        if (e_ != cudaSuccess) throw Err(std::string(#call) + ": " + cudaGetErrorString(e_));         \
    } while (0)
#define LAUNCHED() CK(cudaGetLastError())

thread_local std::string g_create_error;    // fg_last_error(NULL): why the last create on this thread failed

struct Hop {
    int rows = 0, n_src = 0, E = 0, P = 0;
    long long wlo = 0, whi = 0;              // the strength indices this hop's edges use: [wlo, whi)
    long long pbase = 0;                     // first merged pair of this hop in the concatenated arrays
    long long rbase = 0;                     // first row of this hop's layer in the per-row arrays
    bool widx_unique = true, redrive = false;
    int *d_nid = nullptr, *d_drow = nullptr;
    int4* d_rows = nullptr;                      // forward schedule: per slot {first pair, end, row, 0}
    std::vector<int> h_psrc, h_pptr;             // host copies of the forward pairs (for the backward plan)
    long long tbase = 0;                         // first transposed pair of this hop in the concatenated arrays
    int T = 0;                                   // transposed pairs kept for the backward
    int *d_live_dst = nullptr, n_live_dst = 0;   // rows of this hop's layer whose gradient can be non-zero
    long long live_pairs = 0, live_edges = 0;    // merged pairs / edges of those rows (what the weight gradient visits)
    int *d_live_src = nullptr, n_live_src = 0;   // rows of the layer below that this hop's backward writes
    bool narrow = false;                         // no hub sources: narrow fp32 forward, longer transposed segments
    int2* d_sde = nullptr;                       // live edges {edge, transposed pair} in transposed-pair order
    int n_sde = 0;
    std::vector<int2> h_sde;                     // (host copy, until the packed-gradient list is built)
    int4 *d_segs = nullptr, *d_reds = nullptr;   // transposed product: segments of source rows, split-row reductions
    int* d_seg_red = nullptr;                    // per segment: its split row's reduction index, or -1
    int n_segs = 0, n_reds = 0, n_slots = 0;
    void* d_h = nullptr;                     // states [rows, ld]
    bool out_f32 = false;                    // this hop's layer is stored in fp32 (the last layer always is)
};

// pairs per transposed segment: short on a hop with hub sources (their long rows' CTAs retire fast), longer on a hop
// without (fewer split rows and partial rows: model.pt training 37.2 -> 35.5 -> 35.1 -> 34.9 ms with 128 / 256 / 512;
// with 128 everywhere the Zipf graph at batch 2,048 went 0.797 -> 0.822 ms, so hub hops keep 64)
constexpr int kSegLen = 64, kSegLenNarrow = 256;

// kernel classes timed by fg_timing (CUDA events around every launch of the class, on the handle's stream)
enum KClass { K_TRANSPOSE, K_FOLD, K_PLUG_FWD, K_HOP_FWD, K_OUT_FWD, K_LOSS, K_OUT_BWD, K_ACT_BWD, K_WGRAD, K_HOP_BWD,
              K_PLUG_BWD, K_ADAM, K_NORM, K_NCLASS };

struct Timer {
    unsigned mask = 0;                         // classes being timed (bit = KClass)
    std::vector<cudaEvent_t> pool;
    size_t used = 0;
    struct Rec { int cls; cudaEvent_t a, b; };
    std::vector<Rec> recs;
};

struct Core {
    int obs_dim = 0, n_act = 0, hops = 0, n_neurons = 0, n_w = 0, n_s = 0, fan = 0, n_dn = 0;
    std::vector<int> sizes;
    int maxB = 0, flags = 0;
    bool bf16 = false, f16 = false, train = true, redrive = false;
    float* out_part = nullptr;                           // the output plug's per-slice partial logits
    int out_slices = 1;                                  // split-K slices of the dn columns (fixed by the graph)
    float* ow_tc = nullptr;                              // out_w in the tensor-core operand layout (hi, lo terms)
    float* ow_bt = nullptr;                              // out_w^T in the backward's operand layout (training)
    int ob_tiles = 0;                                    // 128-column tiles of the dn columns
    int out_chunks = 0, out_cps = 0;                     // 32-column chunks of the dn columns; chunks per slice
    float* seg_part = nullptr;                           // partial rows of split transposed segments
    int* seg_done = nullptr;                             // arrival counters of split rows' segments [red][chunk]
    int *d_in_crow = nullptr, *d_in_col = nullptr, *d_n0 = nullptr, *d_dn = nullptr;
    std::vector<Hop> hop;
    long long R = 0, Ptot = 0, Etot = 0, Ttot = 0;
    int* d_plug_live = nullptr;                         // sensory rows the plug backward visits
    int* d_gh0_valid = nullptr;                         // per sensory row: 1 if the backward writes its gh0
    int n_plug_live = 0;
    int* d_row_nid = nullptr;
    float *d_rgain = nullptr, *d_rthr = nullptr, *d_rsig = nullptr;
    int2 *d_pairs = nullptr, *d_tpairs = nullptr;
    int *d_gptr = nullptr, *d_gw = nullptr, *d_tpos = nullptr;   // d_tpos: pair -> transposed pair, or -1
    float* sd_part = nullptr;                            // weight-gradient partials [256-sample chunk][transposed pair]
    float* plug_part = nullptr;                          // plug backward's per-split sums [live row][split][fan + 3]
    int* d_wlive = nullptr;                              // strengths a live edge can change, ascending (fg_grad_pack)
    int n_wlive = 0;
    long long off[8] = {0};                             // segment starts in the flat arrays (256-byte aligned)
    long long psize[7] = {0};                           // the seven arrays' true lengths
    float *P = nullptr, *G = nullptr, *M = nullptr, *V = nullptr, *EMA = nullptr;
    long long adam_t = 0;
    float *x = nullptr, *drive = nullptr, *lg = nullptr, *dl = nullptr;
    void* h0 = nullptr;
    float *gz_a = nullptr, *gz_b = nullptr, *gdrive = nullptr, *part = nullptr;
    float* nsum = nullptr;
    float *kl_s = nullptr, *ag_s = nullptr, *stats = nullptr, *norm_part = nullptr, *norm = nullptr;
    int out_splits = 1;
    float *obs_dev = nullptr, *logits_dev = nullptr;   // fg_forward_host staging
    cudaStream_t st = 0, h2d = nullptr, d2h = nullptr;
    int folded = -1;                                    // 0: derived arrays from P, 1: from EMA, -1: stale
    int lastB = 0;
    int status = 0;
    std::string err;
    std::vector<void*> allocs;
    int device = 0, n_sm = 148;
    int* d_err = nullptr;                               // device error word of the tensor-core kernels (0: none)
    int* sv_fired = nullptr;                            // during fg_survey: per-row firing counts and
    float* sv_sq = nullptr;                             //   sums of squared pre-activations (all layers' rows)
    long long launches = 0;
    Timer timer;
    // gradient buckets for an all-reduce that overlaps the backward: stage 0 = the output plug's gradient is final,
    // stage k + 1 = hop k's weight gradient is final; the caller's event for a stage is recorded when it is reached
    std::vector<cudaEvent_t> stage_ev;
};

cudaEvent_t pool_event(Core& c) {
    if (c.timer.used == c.timer.pool.size()) {
        cudaEvent_t e;
        CK(cudaEventCreate(&e));
        c.timer.pool.push_back(e);
    }
    return c.timer.pool[c.timer.used++];
}
// every kernel of the library goes through here: counted, and timed when fg_timing is on
template <class F>
void launch(Core& c, int cls, F&& f) {
    cudaEvent_t a = nullptr, b = nullptr;
    const bool timed = (c.timer.mask >> cls) & 1u;
    if (timed) {
        a = pool_event(c);
        b = pool_event(c);
        CK(cudaEventRecord(a, c.st));
    }
    f();
    CK(cudaGetLastError());
    ++c.launches;
    if (timed) {
        CK(cudaEventRecord(b, c.st));
        c.timer.recs.push_back({cls, a, b});
    }
}

// A kernel of the step on the handle's stream with programmatic dependent launch: the runtime may start its CTAs while
// the stream's previous kernel finishes its last wave; every kernel of the library begins with pdl_enter(), which
// waits for the previous grid to complete (its writes visible) before it reads anything, so only the launch and the
// CTAs' start-up overlap the previous kernel's tail. Stream operations that are not kernels (copies, memsets, event
// records) keep their ordinary ordering.
#ifndef FG_PDL
#define FG_PDL 1
#endif
template <class... KArgs, class... Args>
void pdl(Core& c, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = FG_PDL;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    CK(cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...));
}

template <class X>
X* dalloc(Core& c, size_t n) {
    void* p = nullptr;
    CK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(X)));
    c.allocs.push_back(p);
    return static_cast<X*>(p);
}
template <class X>
X* upload(Core& c, const std::vector<X>& v) {
    X* p = dalloc<X>(c, v.size());
    if (!v.empty()) CK(cudaMemcpy(p, v.data(), v.size() * sizeof(X), cudaMemcpyHostToDevice));
    return p;
}

// ---------------------------------------------------------------- NET.bin
struct Reader {
    std::vector<int> v;
    size_t at = 0;
    std::vector<int> take(long long n, const char* what) {
        if (n < 0 || at + (size_t)n > v.size()) throw Err(std::string("NET.bin too short reading ") + what);
        std::vector<int> out(v.begin() + at, v.begin() + at + n);
        at += n;
        return out;
    }
};

void check_range(const std::vector<int>& a, long long lo, long long hi, const char* what) {
    for (int x : a)
        if (x < lo || x >= hi) throw Err(std::string("NET.bin: ") + what + " index out of range");
}
void check_ptr(const std::vector<int>& p, long long n, const char* what) {
    if (p.empty() || p[0] != 0 || p.back() != n) throw Err(std::string("NET.bin: bad row pointer ") + what);
    for (size_t i = 1; i < p.size(); ++i)
        if (p[i] < p[i - 1]) throw Err(std::string("NET.bin: row pointer not ascending ") + what);
}

// merged pairs of one hop: pair = the edges of one (row, source); returns host arrays appended to the global ones
void build_hop_plan(Core& c, Hop& h, const std::vector<int>& crow, const std::vector<int>& col,
                    const std::vector<int>& widx, const std::vector<int>& drow, std::vector<int2>& pairs,
                    std::vector<int>& gptr, std::vector<int>& gw, std::vector<char>& mark) {
    const int rows = h.rows;
    std::vector<int> pptr(rows + 1, 0), order;
    const long long pbase = (long long)pairs.size();
    h.pbase = pbase;
    // a row's pairs by source (a pair = the row's edges from one source)
    std::vector<int> psrc;
    for (int t = 0; t < rows; ++t) {
        order.resize(crow[t + 1] - crow[t]);
        std::iota(order.begin(), order.end(), crow[t]);
        std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return col[a] < col[b]; });
        for (size_t i = 0; i < order.size(); ++i) {
            const int e = order[i];
            if (i == 0 || col[e] != col[order[i - 1]]) {
                psrc.push_back(col[e]);
                gptr.push_back((int)gw.size());
            }
            gw.push_back(widx[e]);
            if (mark[widx[e]]) h.widx_unique = false;
            mark[widx[e]] = 1;
        }
        pptr[t + 1] = (int)psrc.size();
    }
    for (int w : widx) mark[w] = 0;
    h.P = (int)psrc.size();
    for (int p = 0; p < h.P; ++p) pairs.push_back(make_int2(psrc[p], 0));
    {   // no hub sources (the 32 busiest carry under a fifth of the pairs): the narrow fp32 forward (HopCfg)
        std::vector<int> per_src(h.n_src, 0);
        for (int s : psrc) ++per_src[s];
        const int top = std::min<int>(32, (int)per_src.size());
        std::partial_sort(per_src.begin(), per_src.begin() + top, per_src.end(), std::greater<int>());
        const long long busy = std::accumulate(per_src.begin(), per_src.begin() + top, 0LL);
        h.narrow = h.P > 0 && busy * 5 < (long long)h.P;
    }
    // schedule: rows with most pairs first, so the long ones start early
    std::vector<int> sched(rows);
    std::iota(sched.begin(), sched.end(), 0);
    std::stable_sort(sched.begin(), sched.end(),
                     [&](int a, int b) { return pptr[a + 1] - pptr[a] > pptr[b + 1] - pptr[b]; });
    h.h_psrc = std::move(psrc);
    h.h_pptr = pptr;
    std::vector<int4> rows4(rows);
    for (int slot = 0; slot < rows; ++slot) {
        const int t = sched[slot];
        rows4[slot] = make_int4(pptr[t], pptr[t + 1], t, 0);
    }
    h.d_rows = upload(c, rows4);
}

// The backward plan. A row's gradient can be non-zero only if the row feeds a row whose gradient can be non-zero
// (the descending rows of the last layer start it): rows of the synthetic graph that no later row reads from get an
// exactly zero gradient, so the backward skips them - no transposed pairs into them, no weight gradients from them,
// nothing written for them (the reference skips zero gradients at run time, warp by warp). Then per hop: the
// transposed pairs into live rows, by source and destination, cut into segments of at most kSegLen pairs
// (kSegLenNarrow on a hop without hub sources).
void build_backward_plans(Core& c, const std::vector<std::vector<int>>& drows, const std::vector<int>& dn,
                          const std::vector<int>& gptr, long long n_edges, std::vector<int2>& tpairs,
                          std::vector<int>& tpi) {
    // edges of merged pair q (an index into the concatenated pair arrays)
    auto edges_of = [&](long long q) -> long long {
        return (q + 1 < (long long)gptr.size() ? gptr[q + 1] : n_edges) - gptr[q];
    };
    const int K = c.hops;
    std::vector<std::vector<char>> live(K + 1);
    live[K].assign(c.sizes[K], 0);
    for (int d : dn) live[K][d] = 1;
    for (int k = K; k >= 1; --k) {
        const Hop& h = c.hop[k - 1];
        live[k - 1].assign(c.sizes[k - 1], 0);
        for (int t = 0; t < h.rows; ++t)
            if (live[k][t])
                for (int p = h.h_pptr[t]; p < h.h_pptr[t + 1]; ++p) live[k - 1][h.h_psrc[p]] = 1;
    }
    // sensory rows: live through hop 1, or re-driven into a live row of a later layer
    std::vector<char> plug_live(live[0]);
    for (int k = 1; k <= K; ++k)
        for (int t = 0; t < c.sizes[k]; ++t)
            if (live[k][t] && drows[k - 1][t] >= 0) plug_live[drows[k - 1][t]] = 1;
    std::vector<int> pl;
    for (int s = 0; s < c.n_s; ++s) if (plug_live[s]) pl.push_back(s);
    c.n_plug_live = (int)pl.size();
    c.d_plug_live = upload(c, pl);
    c.d_gh0_valid = upload(c, std::vector<int>(live[0].begin(), live[0].end()));
    for (int k = 1; k <= K; ++k) {
        Hop& h = c.hop[k - 1];
        std::vector<int> ld, ls;
        for (int t = 0; t < h.rows; ++t) if (live[k][t]) ld.push_back(t);
        for (int s = 0; s < h.n_src; ++s) if (live[k - 1][s]) ls.push_back(s);
        h.n_live_dst = (int)ld.size();
        h.n_live_src = (int)ls.size();
        for (int t : ld) {
            h.live_pairs += h.h_pptr[t + 1] - h.h_pptr[t];
            for (int p = h.h_pptr[t]; p < h.h_pptr[t + 1]; ++p) h.live_edges += edges_of(h.pbase + p);
        }
        h.d_live_dst = upload(c, ld);
        h.d_live_src = upload(c, ls);
        // transposed pairs into live rows: by source, destinations ascending
        std::vector<int> tptr(h.n_src + 1, 0);
        for (int t = 0; t < h.rows; ++t)
            if (live[k][t])
                for (int p = h.h_pptr[t]; p < h.h_pptr[t + 1]; ++p) ++tptr[h.h_psrc[p] + 1];
        for (int s = 0; s < h.n_src; ++s) tptr[s + 1] += tptr[s];
        h.T = tptr[h.n_src];
        h.tbase = (long long)tpairs.size();
        std::vector<int> fill(tptr.begin(), tptr.end() - 1);
        std::vector<int2> tp(h.T);
        std::vector<int> ti(h.T);
        for (int t = 0; t < h.rows; ++t) {
            if (!live[k][t]) continue;
            for (int p = h.h_pptr[t]; p < h.h_pptr[t + 1]; ++p) {
                const int q = fill[h.h_psrc[p]]++;
                tp[q] = make_int2(t, 0);
                ti[q] = (int)(h.pbase + p);
            }
        }
        tpairs.insert(tpairs.end(), tp.begin(), tp.end());
        tpi.insert(tpi.end(), ti.begin(), ti.end());
        {   // the weight gradient's edges, pair by pair in transposed order
            std::vector<int2> sde;
            for (int q = 0; q < h.T; ++q)
                for (int j = gptr[ti[q]]; j < (ti[q] + 1 < (long long)gptr.size() ? gptr[ti[q] + 1] : (int)n_edges); ++j)
                    sde.push_back(make_int2(j, q));
            h.n_sde = (int)sde.size();
            if (h.n_sde) h.d_sde = upload(c, sde);
            h.h_sde = std::move(sde);
        }
        std::vector<int4> segs, reds;
        std::vector<int> seg_red;
        const int seg_len = h.narrow ? kSegLenNarrow : kSegLen;
        for (int s : ls) {
            const int n = tptr[s + 1] - tptr[s];
            if (n <= seg_len) {
                segs.push_back(make_int4(s, tptr[s], tptr[s + 1], -1));
                seg_red.push_back(-1);
                continue;
            }
            const int nseg = (n + seg_len - 1) / seg_len;
            for (int i = 0; i < nseg; ++i) {
                segs.push_back(make_int4(s, tptr[s] + i * seg_len,
                                         std::min(tptr[s + 1], tptr[s] + (i + 1) * seg_len), h.n_slots + i));
                seg_red.push_back((int)reds.size());
            }
            reds.push_back(make_int4(s, h.n_slots, nseg, 0));
            h.n_slots += nseg;
        }
        std::vector<int> by_len(segs.size());
        std::iota(by_len.begin(), by_len.end(), 0);
        std::stable_sort(by_len.begin(), by_len.end(),
                         [&](int a, int b) { return segs[a].z - segs[a].y > segs[b].z - segs[b].y; });
        std::vector<int4> segs_s(segs.size());
        std::vector<int> red_s(segs.size());
        for (size_t i = 0; i < by_len.size(); ++i) { segs_s[i] = segs[by_len[i]]; red_s[i] = seg_red[by_len[i]]; }
        h.n_segs = (int)segs.size();
        h.n_reds = (int)reds.size();
        h.d_segs = upload(c, segs_s);
        h.d_seg_red = upload(c, red_s);
        h.d_reds = upload(c, reds);
        std::vector<int>().swap(h.h_psrc);
        std::vector<int>().swap(h.h_pptr);
    }
}

// the file's arrays, read and checked on the host before anything touches the GPU
struct NetHost {
    std::vector<int> in_crow, in_col, n0, dn;
    std::vector<int> E;
    struct H { std::vector<int> nid, crow, col, widx, drow; };
    std::vector<H> hop;
};

NetHost parse_net(Core& c, const char* path) {
    FILE* f = fopen(path, "rb");
    if (!f) throw Err(std::string("cannot open ") + path);
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (sz < 36 || sz % 4) { fclose(f); throw Err("NET.bin: bad size"); }
    Reader r;
    r.v.resize(sz / 4);
    size_t got = fread(r.v.data(), 4, r.v.size(), f);
    fclose(f);
    if (got != r.v.size()) throw Err("NET.bin: short read");
    if (memcmp(r.v.data(), "FLY1", 4)) throw Err("NET.bin: not a FLY1 file");
    r.at = 1;
    auto hd = r.take(8, "header");
    c.obs_dim = hd[0]; c.n_act = hd[1]; c.hops = hd[2]; c.n_neurons = hd[3];
    c.n_w = hd[4]; c.n_s = hd[5]; c.fan = hd[6]; c.n_dn = hd[7];
    if (c.obs_dim <= 0 || c.n_act <= 0 || c.n_act > kMaxAct || c.hops <= 0 || c.hops > 32 || c.n_neurons <= 0 ||
        c.n_w < 0 || c.n_s <= 0 || c.fan < 0 || c.n_dn <= 0)
        throw Err("NET.bin: bad header");
    if ((long long)c.obs_dim * 64 * 4 > 220 * 1024) throw Err("obs_dim too large for the plug's staging");
    NetHost n;
    c.sizes = r.take(c.hops + 1, "sizes");
    n.E = r.take(c.hops, "edge counts");
    if (c.sizes[0] != c.n_s) throw Err("NET.bin: sizes[0] != n_s");
    for (int k = 0; k <= c.hops; ++k) if (c.sizes[k] <= 0) throw Err("NET.bin: empty layer");
    for (int k = 0; k < c.hops; ++k) if (n.E[k] < 0) throw Err("NET.bin: negative edge count");
    const long long e_in = (long long)c.n_s * c.fan;
    n.in_crow = r.take(c.n_s + 1, "in_crow");
    n.in_col = r.take(e_in, "in_col");
    r.take(c.obs_dim + 1, "in_tcrow"); r.take(e_in, "in_tcol"); r.take(e_in, "in_tperm");
    n.n0 = r.take(c.n_s, "n0");
    check_ptr(n.in_crow, e_in, "in_crow");
    check_range(n.in_col, 0, c.obs_dim, "in_col");
    check_range(n.n0, 0, c.n_neurons, "n0");
    n.hop.resize(c.hops);
    for (int k = 0; k < c.hops; ++k) {
        const int rows = c.sizes[k + 1], n_src = c.sizes[k], E = n.E[k];
        NetHost::H& h = n.hop[k];
        h.nid = r.take(rows, "nid");
        h.crow = r.take(rows + 1, "crow");
        h.col = r.take(E, "col");
        h.widx = r.take(E, "widx");
        r.take(n_src + 1, "tcrow"); r.take(E, "tcol"); r.take(E, "twidx");
        h.drow = r.take(rows, "drow");
        check_range(h.nid, 0, c.n_neurons, "nid");
        check_ptr(h.crow, E, "crow");
        check_range(h.col, 0, n_src, "col");
        check_range(h.widx, 0, c.n_w, "widx");
        check_range(h.drow, -1, c.n_s, "drow");
    }
    n.dn = r.take(c.n_dn, "dn_rows");
    check_range(n.dn, 0, c.sizes[c.hops], "dn_rows");
    r.take(c.n_w, "wmap");
    if (r.at != r.v.size()) throw Err("NET.bin: trailing bytes");
    return n;
}

void upload_net(Core& c, NetHost& n) {
    c.d_in_crow = upload(c, n.in_crow);
    c.d_in_col = upload(c, n.in_col);
    c.d_n0 = upload(c, n.n0);
    std::vector<int> row_nid(n.n0);
    std::vector<int2> pairs, tpairs;
    std::vector<int> gptr, gw, tpi;
    std::vector<char> mark(std::max(c.n_w, 1), 0);
    c.hop.resize(c.hops);
    long long rbase = c.n_s;
    for (int k = 0; k < c.hops; ++k) {
        Hop& h = c.hop[k];
        NetHost::H& src = n.hop[k];
        h.rows = c.sizes[k + 1]; h.n_src = c.sizes[k]; h.E = n.E[k]; h.rbase = rbase;
        for (int d : src.drow) if (d >= 0) h.redrive = true;
        c.redrive |= h.redrive;
        h.d_nid = upload(c, src.nid);
        h.d_drow = h.redrive ? upload(c, src.drow) : nullptr;
        row_nid.insert(row_nid.end(), src.nid.begin(), src.nid.end());
        build_hop_plan(c, h, src.crow, src.col, src.widx, src.drow, pairs, gptr, gw, mark);
        if (!src.widx.empty()) {
            const auto mm = std::minmax_element(src.widx.begin(), src.widx.end());
            h.wlo = *mm.first;
            h.whi = (long long)*mm.second + 1;
        }
        rbase += h.rows;
    }
    c.d_dn = upload(c, n.dn);
    {
        std::vector<std::vector<int>> drows;
        for (auto& hh : n.hop) drows.push_back(hh.drow);
        build_backward_plans(c, drows, n.dn, gptr, (long long)gw.size(), tpairs, tpi);
    }
    c.Ttot = (long long)tpairs.size();
    gptr.push_back((int)gw.size());
    c.R = (long long)row_nid.size();
    c.Ptot = (long long)pairs.size();
    c.Etot = (long long)gw.size();
    c.d_row_nid = upload(c, row_nid);
    c.d_rgain = dalloc<float>(c, c.R);
    c.d_rthr = dalloc<float>(c, c.R);
    c.d_rsig = dalloc<float>(c, c.R);
    pairs.push_back(make_int2(0, 0));       // one record past the end: the hop forward reads a pair ahead
    c.d_pairs = upload(c, pairs);
    c.d_tpairs = upload(c, tpairs);
    c.d_gptr = upload(c, gptr);
    c.d_gw = upload(c, gw);
    {   // the strengths whose gradient can be non-zero: those of the edges of pairs into live rows
        std::vector<char> on(std::max(c.n_w, 1), 0);
        for (const Hop& h : c.hop)
            for (const int2& e : h.h_sde) on[gw[e.x]] = 1;
        std::vector<int> wl;
        for (int w = 0; w < c.n_w; ++w) if (on[w]) wl.push_back(w);
        c.n_wlive = (int)wl.size();
        if (c.n_wlive) c.d_wlive = upload(c, wl);
        for (Hop& h : c.hop) std::vector<int2>().swap(h.h_sde);
    }
    if (c.Ttot) {
        std::vector<int> tpos(c.Ptot, -1);
        for (long long q = 0; q < c.Ttot; ++q) tpos[tpi[q]] = (int)q;
        c.d_tpos = upload(c, tpos);
    }
}

size_t act_bytes(const Core& c) { return (c.bf16 || c.f16) ? 2 : 4; }

void alloc_all(Core& c) {
    const long long ps[7] = {c.n_w, c.n_neurons, c.n_neurons, (long long)c.n_s * c.fan, c.n_s,
                             (long long)c.n_act * c.n_dn, c.n_act};
    c.off[0] = 0;
    for (int i = 0; i < 7; ++i) {
        c.psize[i] = ps[i];
        c.off[i + 1] = (c.off[i] + ps[i] + 63) / 64 * 64;   // every array starts on a 256-byte boundary
    }
    const long long n = c.off[7];
    c.P = dalloc<float>(c, n);
    c.EMA = dalloc<float>(c, n);
    CK(cudaMemset(c.P, 0, n * 4));
    CK(cudaMemset(c.EMA, 0, n * 4));
    if (c.train) {
        c.G = dalloc<float>(c, n); c.M = dalloc<float>(c, n); c.V = dalloc<float>(c, n);
        CK(cudaMemset(c.G, 0, n * 4)); CK(cudaMemset(c.M, 0, n * 4)); CK(cudaMemset(c.V, 0, n * 4));
    }
    const size_t B = c.maxB;
    int max_rows = c.n_s;
    for (auto& h : c.hop) max_rows = std::max(max_rows, h.rows);
    c.x = dalloc<float>(c, (size_t)c.obs_dim * B);
    if (c.redrive) c.drive = dalloc<float>(c, (size_t)c.n_s * B);   // the plug's pre-activation, for re-driven rows
    c.h0 = dalloc<char>(c, (size_t)c.n_s * B * act_bytes(c));
    for (size_t k = 0; k < c.hop.size(); ++k) {
        Hop& h = c.hop[k];
        h.out_f32 = act_bytes(c) == 4 || k + 1 == c.hop.size();
        h.d_h = dalloc<char>(c, (size_t)h.rows * B * (h.out_f32 ? 4 : act_bytes(c)));
    }
    c.d_err = dalloc<int>(c, 1);
    CK(cudaMemset(c.d_err, 0, sizeof(int)));
    CK(cudaDeviceGetAttribute(&c.n_sm, cudaDevAttrMultiProcessorCount, c.device));
    // The slice count depends on the graph only, never on the batch, so a sample's logits are the same bits whatever
    // batch (or piece of one) it is computed in: one slice per ~320 dn columns, at most 8.
    c.out_chunks = (c.n_dn + kOtKC - 1) / kOtKC;
    {
        const int want = std::max(1, std::min(kOutSlices, (c.n_dn + 319) / 320));
        c.out_cps = (c.out_chunks + want - 1) / want;
        c.out_slices = (c.out_chunks + c.out_cps - 1) / c.out_cps;
    }
    c.out_part = dalloc<float>(c, (size_t)c.out_slices * kOutA * B);
    c.ow_tc = dalloc<float>(c, (size_t)c.out_chunks * 2 * kOtN * kOtKC);
    c.ob_tiles = (c.n_dn + kObN - 1) / kObN;
    if (c.train) c.ow_bt = dalloc<float>(c, (size_t)c.ob_tiles * kObChunks * 2 * kObN * kOtKC);
    c.lg = dalloc<float>(c, (size_t)c.n_act * B);
    c.norm_part = dalloc<float>(c, 1024);
    c.norm = dalloc<float>(c, 4);
    c.stats = dalloc<float>(c, 4);
    if (c.train) {
        c.dl = dalloc<float>(c, (size_t)c.n_act * B);
        c.gz_a = dalloc<float>(c, (size_t)max_rows * B);
        c.gz_b = dalloc<float>(c, (size_t)max_rows * B);
        c.gdrive = dalloc<float>(c, (size_t)c.n_s * B);
        c.nsum = dalloc<float>(c, (size_t)max_rows * ((B + 255) / 256) * 2);
        c.out_splits = std::max(1, std::min(64, (int)(B / 128)));     // batch slices of the output-plug backward
        c.part = dalloc<float>(c, (size_t)c.out_splits * c.n_act * (c.n_dn + 1));
        c.kl_s = dalloc<float>(c, B);
        int slots = 0;
        for (auto& h : c.hop) slots = std::max(slots, h.n_slots);
        c.seg_part = dalloc<float>(c, (size_t)slots * B);
        long long tmax = 1;
        for (auto& h : c.hop) tmax = std::max<long long>(tmax, h.T);
        c.sd_part = dalloc<float>(c, (size_t)tmax * ((B + 255) / 256));
        c.plug_part = dalloc<float>(c, (size_t)std::max(1, c.n_plug_live) * kPlugSplits * (c.fan + 3));
        int reds = 0;
        for (auto& h : c.hop) reds = std::max(reds, h.n_reds);
        const size_t n_done = std::max<size_t>(1, (size_t)reds * ((B + 255) / 256));
        c.seg_done = dalloc<int>(c, n_done);
        CK(cudaMemset(c.seg_done, 0, n_done * sizeof(int)));
        c.ag_s = dalloc<float>(c, B);
    }
}

template <class T>
int plug_smem(const Core& c) {
    const int f = (c.fan % 4 == 0 && c.fan > 0 && c.fan <= 16) ? c.fan : 1;     // (the F the launch instantiates)
    return (c.obs_dim * PlugCfg<T>::cols * (int)sizeof(T) + 15) / 16 * 16 + (kPlugThreads / 32) * PlugCfg<T>::warp_bytes(f);
}

template <class T, bool SAVE>
void plug_limit(const Core& c) {
    const int smem = plug_smem<T>(c);
    if (smem > 232448)
        throw Err("input plug: obs_dim " + std::to_string(c.obs_dim) + " with fan " + std::to_string(c.fan) +
                  " needs " + std::to_string(smem) + " bytes of shared memory per CTA (at most 232448)");
    CK(cudaFuncSetAttribute(k_plug_fwd<T, SAVE, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    CK(cudaFuncSetAttribute(k_plug_fwd<T, SAVE, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    CK(cudaFuncSetAttribute(k_plug_fwd<T, SAVE, 12>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    CK(cudaFuncSetAttribute(k_plug_fwd<T, SAVE, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    CK(cudaFuncSetAttribute(k_plug_fwd<T, SAVE, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
}

void set_smem_limits(const Core& c) {
    CK(cudaFuncSetAttribute(k_out_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kOtSmem));
    CK(cudaFuncSetAttribute(k_out_bwd_h_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kObSmem));
    CK(cudaFuncSetAttribute(k_out_bwd_w_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kOwSmem));
    plug_limit<float, true>(c); plug_limit<float, false>(c);
    plug_limit<__nv_bfloat16, true>(c); plug_limit<__nv_bfloat16, false>(c);
    plug_limit<__half, true>(c); plug_limit<__half, false>(c);
}

inline unsigned blocks(long long n, int t = 256) { return (unsigned)((n + t - 1) / t); }
static_assert(kOtN == kOutA, "the tensor-core output plug writes the partial slabs k_out_reduce reads");

// derived per-version arrays: per-row gain / threshold / sigmoid, merged pair weights (forward and transposed)
void fold(Core& c, int which) {
    if (c.folded == which) return;
    const float* src = which ? c.EMA : c.P;
    FoldArgs f;
    f.nid = c.d_row_nid; f.gain = src + c.off[1]; f.theta = src + c.off[2];
    f.rgain = c.d_rgain; f.rthr = c.d_rthr; f.rsig = c.d_rsig; f.n_rows = (int)c.R;
    f.gptr = c.d_gptr; f.gw = c.d_gw; f.W = src + c.off[0]; f.pairs = c.d_pairs; f.tpos = c.d_tpos;
    f.tpairs = c.d_tpairs; f.n_pairs = (int)c.Ptot;
    f.ow = src + c.off[5]; f.ow_tc = c.ow_tc; f.ow_bt = c.ow_bt;
    f.n_act = c.n_act; f.n_dn = c.n_dn; f.chunks = c.out_chunks; f.ob_tiles = c.ob_tiles;
    f.nb_pairs = (int)blocks(c.Ptot, kWarps * 32);                     // a warp per 32 pairs
    f.nb_rows = (int)blocks(c.R, kThreads);
    f.nb_ow = (int)blocks((long long)c.out_chunks * kOtN * kOtKC, kThreads);
    const int nb_bt = c.ow_bt ? (int)blocks((long long)c.ob_tiles * kObChunks * kObN * kOtKC, kThreads) : 0;
    launch(c, K_FOLD, [&]() { pdl(c, k_fold, f.nb_pairs + f.nb_rows + f.nb_ow + nb_bt, kThreads, 0, f); });
    c.folded = which;
}

void check_batch(const Core& c, int B) {
    if (B <= 0 || B % 32 || B > c.maxB)
        throw Err("batch " + std::to_string(B) + " is not a positive multiple of 32 up to max_batch " +
                  std::to_string(c.maxB));
}

template <class T, bool SAVE>
void plug_launch(Core& c, const float* Pw, int B) {
    const int chunks = (B + PlugCfg<T>::cols - 1) / PlugCfg<T>::cols;
    // row blocks per chunk: the count whose whole waves of CTAs cost least, a CTA's time taken as its rows plus the
    // staging of its x chunk (about as long as 264 rows); at most one block per 64 rows
    const int smem = plug_smem<T>(c);
    const int per_sm = std::max(1, std::min(2048 / kPlugThreads, 233472 / (smem + 1024)));
    int nblk = 1;
    long long best = -1;
    for (int k = 1; k <= std::max(1, std::min(64, (c.n_s + 63) / 64)); ++k) {
        const long long waves = ((long long)chunks * k + (long long)c.n_sm * per_sm - 1) / ((long long)c.n_sm * per_sm);
        const long long cost = waves * ((c.n_s + k - 1) / k + 264);
        if (best < 0 || cost < best) { best = cost; nblk = k; }
    }
    const int rows = (c.n_s + nblk - 1) / nblk;
    const dim3 g(nblk, chunks);
    launch(c, K_PLUG_FWD, [&]() {
        if (c.fan == 8)
            pdl(c, k_plug_fwd<T, SAVE, 8>, g, kPlugThreads, smem, c.d_in_col, Pw + c.off[3], Pw + c.off[4],
                c.d_rgain, c.d_rthr, c.x, c.drive, (T*)c.h0, c.n_s, c.fan, rows, c.obs_dim, B);
        else if (c.fan == 16)
            pdl(c, k_plug_fwd<T, SAVE, 16>, g, kPlugThreads, smem, c.d_in_col, Pw + c.off[3], Pw + c.off[4],
                c.d_rgain, c.d_rthr, c.x, c.drive, (T*)c.h0, c.n_s, c.fan, rows, c.obs_dim, B);
        else if (c.fan == 4)
            pdl(c, k_plug_fwd<T, SAVE, 4>, g, kPlugThreads, smem, c.d_in_col, Pw + c.off[3], Pw + c.off[4],
                c.d_rgain, c.d_rthr, c.x, c.drive, (T*)c.h0, c.n_s, c.fan, rows, c.obs_dim, B);
        else if (c.fan == 12)
            pdl(c, k_plug_fwd<T, SAVE, 12>, g, kPlugThreads, smem, c.d_in_col, Pw + c.off[3], Pw + c.off[4],
                c.d_rgain, c.d_rthr, c.x, c.drive, (T*)c.h0, c.n_s, c.fan, rows, c.obs_dim, B);
        else
            pdl(c, k_plug_fwd<T, SAVE, 0>, g, kPlugThreads, smem, c.d_in_col, Pw + c.off[3], Pw + c.off[4],
                c.d_rgain, c.d_rthr, c.x, c.drive, (T*)c.h0, c.n_s, c.fan, rows, c.obs_dim, B);
    });
}

template <class TI, class TO>
void hop_launch(Core& c, const Hop& h, const void* hp, int B) {
    if (c.sv_fired) {                                     // the firing survey: CUDA-core hop with per-row counters
        constexpr int N = Lane32<TI>::N;
        const dim3 g((h.rows + kWarps - 1) / kWarps, (unsigned)((B + 32 * N - 1) / (32 * N)));
        launch(c, K_HOP_FWD, [&]() {
            if (B % (32 * N) == 0)
                pdl(c, k_hop_fwd_surv<TI, TO, true>, g, kThreads, 0, h.d_rows, c.d_pairs + h.pbase,
                    (const TI*)hp, c.d_rgain + h.rbase, c.d_rthr + h.rbase, h.d_drow, c.drive, (TO*)h.d_h, h.rows, B,
                    c.sv_fired + h.rbase, c.sv_sq + h.rbase);
            else
                pdl(c, k_hop_fwd_surv<TI, TO, false>, g, kThreads, 0, h.d_rows, c.d_pairs + h.pbase,
                    (const TI*)hp, c.d_rgain + h.rbase, c.d_rthr + h.rbase, h.d_drow, c.drive, (TO*)h.d_h, h.rows, B,
                    c.sv_fired + h.rbase, c.sv_sq + h.rbase);
        });
        return;
    }
    auto go = [&](auto narrow) {
        constexpr bool NW = decltype(narrow)::value;
        constexpr int N = Lane32<TI, NW>::N;             // samples per lane; the warp's chunk is 32 N
        const dim3 g((h.rows + kWarps - 1) / kWarps, (unsigned)((B + 32 * N - 1) / (32 * N)));
        const bool full = B % (32 * N) == 0;
        launch(c, K_HOP_FWD, [&]() {
            if (full)
                pdl(c, k_hop_fwd<TI, TO, true, NW>, g, kThreads, 0, h.d_rows, c.d_pairs + h.pbase, (const TI*)hp,
                    c.d_rgain + h.rbase, c.d_rthr + h.rbase, h.d_drow, c.drive, (TO*)h.d_h, h.rows, B);
            else
                pdl(c, k_hop_fwd<TI, TO, false, NW>, g, kThreads, 0, h.d_rows, c.d_pairs + h.pbase, (const TI*)hp,
                    c.d_rgain + h.rbase, c.d_rthr + h.rbase, h.d_drow, c.drive, (TO*)h.d_h, h.rows, B);
        });
    };
    if (sizeof(TI) == 4 && h.narrow) go(std::true_type{});
    else go(std::false_type{});
}

// obs == nullptr: the states start from c.x as it is
template <class T>
void forward_t(Core& c, const float* obs, int B, float* logits, int ema, bool keep_lg) {
    fold(c, ema ? 1 : 0);
    const float* Pw = ema ? c.EMA : c.P;
    if (obs) {
        launch(c, K_TRANSPOSE, [&]() {
            pdl(c, k_to_neuron_major, dim3((B + 31) / 32, (c.obs_dim + 31) / 32), dim3(32, 8), 0, obs, c.x, c.obs_dim,
                                                                                                B, B);
        });
    }
    if (c.drive) plug_launch<T, true>(c, Pw, B);
    else plug_launch<T, false>(c, Pw, B);
    const void* hp = c.h0;
    bool hp_f32 = std::is_same<T, float>::value;
    for (auto& h : c.hop) {
        if (hp_f32) hop_launch<float, float>(c, h, hp, B);
        else if (h.out_f32) hop_launch<T, float>(c, h, hp, B);
        else hop_launch<T, T>(c, h, hp, B);
        hp = h.d_h;
        hp_f32 = h.out_f32;
    }
    // tensor-core tiles of 128 samples x split-K slices of the dn columns, then k_out_reduce adds the bias and the
    // slices in order
    OutTc ot;
    ot.wt = c.ow_tc; ot.dn = c.d_dn; ot.hK = (const float*)hp; ot.part = c.out_part; ot.err = c.d_err;
    ot.n_dn = c.n_dn; ot.B = B; ot.ld = B; ot.chunks = c.out_chunks; ot.cps = c.out_cps;
    launch(c, K_OUT_FWD, [&]() {
        pdl(c, k_out_tc, dim3((B + kOtM - 1) / kOtM, c.out_slices), kOtThreads, kOtSmem, ot);
    });
    launch(c, K_OUT_FWD, [&]() {
        pdl(c, k_out_reduce, (B + 31) / 32, 256, 0, c.out_part, Pw + c.off[6], keep_lg ? c.lg : nullptr, logits,
                                                      c.out_slices, c.n_act, B, B);
    });
    c.lastB = B;
}

void forward(Core& c, const float* obs, int B, float* logits, int ema, bool keep_lg) {
    if (c.bf16) forward_t<__nv_bfloat16>(c, obs, B, logits, ema, keep_lg);
    else if (c.f16) forward_t<__half>(c, obs, B, logits, ema, keep_lg);
    else forward_t<float>(c, obs, B, logits, ema, keep_lg);
}

void record_stage(Core& c, int stage) {
    if (stage < (int)c.stage_ev.size() && c.stage_ev[stage]) CK(cudaEventRecord(c.stage_ev[stage], c.st));
}

// Ranges of the flat gradient that become final before the backward ends, and the stage at which each does: the
// output plug's arrays at stage 0; hop k's strengths [wlo, whi) at stage k + 1 when no hop the backward visits later
// (k - 1 .. 0) uses a strength inside that range (weights shared across hops - the shipped model.pt network - leave
// no such range). The rest of [0, flat length) is final at the end (stage -1).
std::vector<std::array<long long, 3>> grad_buckets(const Core& c) {
    std::vector<std::array<long long, 3>> early{{c.off[5], c.off[7], 0}};
    for (int k = c.hops - 1; k >= 0; --k) {
        const Hop& h = c.hop[k];
        if (h.whi <= h.wlo) continue;
        bool alone = true;
        for (int j = 0; j < k; ++j)
            if (c.hop[j].whi > c.hop[j].wlo && c.hop[j].wlo < h.whi && h.wlo < c.hop[j].whi) alone = false;
        if (alone) early.push_back({h.wlo, h.whi, k + 1});
    }
    std::vector<std::array<long long, 3>> out = early;
    std::vector<std::pair<long long, long long>> taken;
    for (auto& b : early) taken.push_back({b[0], b[1]});
    std::sort(taken.begin(), taken.end());
    long long at = 0;
    for (auto& t : taken) {
        if (t.first > at) out.push_back({at, t.first, -1});
        at = std::max(at, t.second);
    }
    if (at < c.off[7]) out.push_back({at, c.off[7], -1});
    return out;
}

// gradient of the loss whose d/dlogits is in c.dl [n_act, B], through the states of the last forward; ADDED to G.
// Per hop k (top down): the weight gradient of its merged pairs from gz_k and the states below, then the transposed
// product into the layer below with that layer's neuron backward fused in (for the sensory layer: gh0 for the plug).
void backward(Core& c, int B) {
    if (!c.train) throw Err("this handle was created for inference only");
    if (B != c.lastB) throw Err("fc_backward batch differs from the last forward's");
    fold(c, 0);
    CK(cudaMemsetAsync(c.gdrive, 0, (size_t)c.n_s * B * 4, c.st));
    const Hop& top = c.hop.back();
    const float* hK = (const float*)top.d_h;
    // weight gradient on the tensor cores: 128-column tiles x batch slices (multiples of 32 samples), about two
    // waves of CTAs; k_out_bwd_reduce adds the slices in order
    const int wtiles = (c.n_dn + 1 + 127) / 128;
    const int want = std::max(1, std::min({c.out_splits, (2 * c.n_sm + wtiles - 1) / wtiles, B / 32}));
    const int split_len = ((B + want - 1) / want + 31) / 32 * 32;
    const int splits = (B + split_len - 1) / split_len;
    {
        OutBw ow;
        ow.dl = c.dl; ow.hK = hK; ow.dn = c.d_dn; ow.part = c.part; ow.err = c.d_err;
        ow.n_act = c.n_act; ow.n_dn = c.n_dn; ow.B = B; ow.ld = B; ow.slice_len = split_len;
        launch(c, K_OUT_BWD, [&]() { pdl(c, k_out_bwd_w_tc, dim3(wtiles, splits), kOtThreads, kOwSmem, ow); });
    }
    launch(c, K_OUT_BWD, [&]() {
        pdl(c, k_out_bwd_reduce, blocks((long long)c.n_act * (c.n_dn + 1)), 256, 0, c.part, c.G + c.off[5],
                                                                                     c.G + c.off[6], c.n_act, c.n_dn,
                                                                                     splits);
    });
    record_stage(c, 0);
    float* gz = c.gz_a;                      // gz of the layer being processed
    float* nxt = c.gz_b;                     // gz (or gh0) of the layer below
    // only the output plug's columns of the top layer get a gradient; the other rows of gh / gz are never read
    {
        // gh = out_w^T dl on the tensor cores: 128-sample tiles x runs of 128-column tiles, about one CTA per SM
        OutBh ob;
        ob.wt = c.ow_bt; ob.dl = c.dl; ob.dn = c.d_dn; ob.gh = nxt; ob.err = c.d_err;
        ob.n_act = c.n_act; ob.n_dn = c.n_dn; ob.B = B; ob.ld = B; ob.n_tiles = c.ob_tiles;
        const int st = (B + 127) / 128;
        const int groups = std::max(1, std::min(c.ob_tiles, c.n_sm / st));
        ob.tpg = (c.ob_tiles + groups - 1) / groups;
        const int ng = (c.ob_tiles + ob.tpg - 1) / ob.tpg;
        launch(c, K_OUT_BWD, [&]() { pdl(c, k_out_bwd_h_tc, dim3(st, ng), kOtThreads, kObSmem, ob); });
    }
    if (top.n_live_dst)
    launch(c, K_ACT_BWD, [&]() {
        pdl(c, k_act_bwd<float>, top.n_live_dst, kThreads, 0, nxt, hK, top.d_nid, top.d_drow,
                                                                c.d_rgain + top.rbase, c.d_rthr + top.rbase,
                                                                c.d_rsig + top.rbase, gz, c.G + c.off[1],
                                                                c.G + c.off[2], c.gdrive, top.d_live_dst, B,
                                                                B);
    });
    const int chunks = (B + 255) / 256;
    for (int k = c.hops - 1; k >= 0; --k) {
        const Hop& h = c.hop[k];
        const float* hprev = k ? (const float*)c.hop[k - 1].d_h : (const float*)c.h0;
        const bool full = B % 256 == 0;
        // the transposed product, which also forms the weight gradient's per-chunk partials; k_sd_reduce then adds
        // them up into the edges' weight gradients
        auto transposed = [&](auto epi, const NeuronEpi& ep) {
            constexpr bool EPI = decltype(epi)::value;
            const dim3 gs((h.n_segs + kWarps - 1) / kWarps, chunks);
            if (h.n_segs == 0) return;
            launch(c, K_HOP_BWD, [&]() {
                if (full)
                    pdl(c, k_hop_bwd_t<EPI, true>, gs, kThreads, 0, h.d_segs, h.d_seg_red, h.d_reds, c.seg_done,
                        c.d_tpairs + h.tbase, gz, nxt, c.seg_part, h.n_segs, B, ep, hprev, c.sd_part, (int)h.T);
                else
                    pdl(c, k_hop_bwd_t<EPI, false>, gs, kThreads, 0, h.d_segs, h.d_seg_red, h.d_reds, c.seg_done,
                        c.d_tpairs + h.tbase, gz, nxt, c.seg_part, h.n_segs, B, ep, hprev, c.sd_part, (int)h.T);
            });
            if (h.n_sde) {
                launch(c, K_WGRAD, [&]() {
                    if (h.widx_unique)
                        pdl(c, k_sd_reduce<false>, blocks(h.n_sde), 256, 0, (const float*)c.sd_part, (int)h.T, chunks,
                            (const int2*)h.d_sde, h.n_sde, (const int*)c.d_gw, c.G + c.off[0]);
                    else
                        pdl(c, k_sd_reduce<true>, blocks(h.n_sde), 256, 0, (const float*)c.sd_part, (int)h.T, chunks,
                            (const int2*)h.d_sde, h.n_sde, (const int*)c.d_gw, c.G + c.off[0]);
                });
            }
        };
        if (k >= 1) {                        // the layer below is a hop's: its neuron backward rides along
            const Hop& lo = c.hop[k - 1];
            NeuronEpi ep{hprev, c.d_rgain + lo.rbase, c.d_rthr + lo.rbase, lo.d_drow, c.gdrive, c.nsum, chunks};
            transposed(std::true_type{}, ep);
            if (h.n_live_src)
            launch(c, K_ACT_BWD, [&]() {
                pdl(c, k_neuron_reduce, blocks(h.n_live_src), 256, 0, c.nsum, h.d_live_src, lo.d_nid,
                                                                       c.d_rsig + lo.rbase, c.G + c.off[1],
                                                                       c.G + c.off[2], h.n_live_src, chunks);
            });
        } else {
            NeuronEpi ep{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, chunks};
            transposed(std::false_type{}, ep);
        }
        record_stage(c, k + 1);                          // (hop k's weight gradient is final)
        std::swap(gz, nxt);
    }
    // gz now holds gh0 (the sensory layer's incoming gradient)
    if (c.n_plug_live)
    {
        // the batch split over up to 8 warps a row (2,048 samples or more each): a warp per live sensory row alone is
        // few warps a SM; the splits' sums are added in order by k_plug_bwd_reduce
        const int splits = std::max(1, std::min(kPlugSplits, B / 2048));
        const int span = ((B + splits - 1) / splits + 127) / 128 * 128;
        float* part = splits > 1 ? c.plug_part : nullptr;
        launch(c, K_PLUG_BWD, [&]() {
            const dim3 g((c.n_plug_live + kWarps - 1) / kWarps, splits);
            auto go = [&](auto kern) {
                pdl(c, kern, g, kThreads, 0, c.d_plug_live, c.d_gh0_valid, gz, (const float*)c.h0, c.drive, c.gdrive,
                    c.d_n0, c.d_in_col, c.x, c.d_rgain, c.d_rthr, c.d_rsig, c.G + c.off[1], c.G + c.off[2],
                    c.G + c.off[3], c.G + c.off[4], c.n_plug_live, c.fan, B, B, part, span);
            };
            if (c.fan == 8) go(k_plug_bwd<8>);
            else if (c.fan == 16) go(k_plug_bwd<16>);
            else go(k_plug_bwd<0>);
        });
        if (part)
            launch(c, K_PLUG_BWD, [&]() {
                pdl(c, k_plug_bwd_reduce, blocks((long long)c.n_plug_live * (c.fan + 3)), 256, 0, (const float*)part,
                    (const int*)c.d_plug_live, (const int*)c.d_n0, (const float*)c.d_rsig, c.G + c.off[1],
                    c.G + c.off[2], c.G + c.off[3], c.G + c.off[4], c.n_plug_live, c.fan, splits);
            });
    }
}

// the gradient norm and the clipping scale into c.norm (device)
void grad_norm_launch(Core& c, float max_norm) {
    const long long n = c.off[7];
    const int nb = (int)std::min<long long>(1024, std::max<long long>(1, blocks(n)));
    launch(c, K_NORM, [&]() { pdl(c, k_sumsq, nb, 256, 0, c.G, n, c.norm_part); });
    launch(c, K_NORM, [&]() { pdl(c, k_norm_final, 1, 256, 0, c.norm_part, nb, max_norm, c.norm); });
}
float read_norm(Core& c) {
    float g = 0.f;
    CK(cudaMemcpyAsync(&g, c.norm, 4, cudaMemcpyDeviceToHost, c.st));
    CK(cudaStreamSynchronize(c.st));
    return g;
}
float grad_norm(Core& c, float max_norm) {
    grad_norm_launch(c, max_norm);
    return read_norm(c);
}

float* flat(Core& c, int which) {
    switch (which) {
        case 0: return c.P;
        case 1: return c.EMA;
        case 2: return c.M;
        case 3: return c.V;
        case 4: return c.G;
    }
    return nullptr;
}

Core* as_core(void* h) { return static_cast<Core*>(h); }

template <class F>
auto guarded(void* h, F&& fn, decltype(fn()) fail) -> decltype(fn()) {
    Core* c = as_core(h);
    if (!c) { g_create_error = "null handle"; return fail; }
    if (c->status) return fail;
    try {
        CK(cudaSetDevice(c->device));
        return fn();
    } catch (const std::exception& e) {
        c->status = 1;
        c->err = e.what();
        return fail;
    }
}

void destroy(Core* c) {
    if (!c) return;
    if (c->allocs.empty() && !c->h2d && !c->d2h) { delete c; return; }
    cudaSetDevice(c->device);
    if (c->st) cudaStreamSynchronize(c->st);
    for (void* p : c->allocs) cudaFree(p);
    for (auto e : c->timer.pool) cudaEventDestroy(e);
    if (c->h2d) cudaStreamDestroy(c->h2d);
    if (c->d2h) cudaStreamDestroy(c->d2h);
    delete c;
}

void* create(const char* path, int max_batch, int flags) {
    Core* c = new Core;
    try {
        if (!path) throw Err("no network file");
        if (max_batch <= 0 || max_batch % 32) throw Err("max_batch must be a positive multiple of 32");
        // a state row of max_batch fp32 values must stay below 4 GiB (row offsets are 32 x 32 -> 64-bit products)
        if (max_batch > (1 << 28)) throw Err("max_batch must be at most 268435456");
        if (flags & ~(FG_ACT_BF16 | FG_INFER_ONLY | FG_ACT_F16)) throw Err("unknown flags " + std::to_string(flags));
        c->maxB = max_batch;
        c->flags = flags;
        c->bf16 = flags & FG_ACT_BF16;
        c->f16 = (flags & FG_ACT_F16) && !c->bf16;
        c->train = !(flags & (FG_ACT_BF16 | FG_ACT_F16 | FG_INFER_ONLY));
        NetHost n = parse_net(*c, path);     // (a bad file fails here, before the GPU is touched)
        // the hop kernels address a source row in 16-byte units with 32 bits: one layer of states at most 2^36 bytes
        for (int v : c->sizes)
            if ((double)v * max_batch * 4.0 >= 68719476736.0)
                throw Err("max_batch " + std::to_string(max_batch) + " makes a layer of " + std::to_string(v) +
                          " rows larger than 2^36 bytes");
        CK(cudaGetDevice(&c->device));
        upload_net(*c, n);
        alloc_all(*c);
        set_smem_limits(*c);
        CK(cudaDeviceSynchronize());
        return c;
    } catch (const std::exception& e) {
        g_create_error = e.what();
        destroy(c);
        return nullptr;
    }
}

}  // namespace

// ================================================================ C ABI
extern "C" {

void* fc_create(const char* net_path, int max_batch) { return create(net_path, max_batch, 0); }
void* fg_create(const char* net_path, int max_batch, int flags) { return create(net_path, max_batch, flags); }
void fg_destroy(void* h) { destroy(as_core(h)); }

int fg_status(void* h) { return h ? as_core(h)->status : (g_create_error.empty() ? 0 : 1); }
const char* fg_last_error(void* h) { return h ? as_core(h)->err.c_str() : g_create_error.c_str(); }
void fg_clear_error(void* h) {
    if (!h) { g_create_error.clear(); return; }
    as_core(h)->status = 0;
    as_core(h)->err.clear();
}

void fc_sizes(void* h, long long* out) {
    guarded(h, [&]() {
        Core& c = *as_core(h);
        for (int i = 0; i < 7; ++i) out[i] = c.psize[i];
        out[7] = c.obs_dim; out[8] = c.n_act; out[9] = c.maxB;
        return 0;
    }, 0);
}

void fg_offsets(void* h, long long* off) {
    guarded(h, [&]() { for (int i = 0; i < 8; ++i) off[i] = as_core(h)->off[i]; return 0; }, 0);
}

int fg_layout(void* h, int* sizes, long long* pairs) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        for (int k = 0; k <= c.hops; ++k) if (sizes) sizes[k] = c.sizes[k];
        for (int k = 0; k < c.hops; ++k) if (pairs) pairs[k] = c.hop[k].P;
        return c.hops;
    }, -1);
}

int fg_set_stage_event(void* h, int stage, void* event) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        if (stage < 0 || stage > c.hops) throw Err("fg_set_stage_event: stage " + std::to_string(stage) + " is not 0.." +
                                                   std::to_string(c.hops));
        if ((int)c.stage_ev.size() <= stage) c.stage_ev.resize(stage + 1, nullptr);
        c.stage_ev[stage] = static_cast<cudaEvent_t>(event);
        return 0;
    }, -1);
}

int fg_grad_buckets(void* h, long long* out, int n) {
    return guarded(h, [&]() {
        const auto b = grad_buckets(*as_core(h));
        for (int i = 0; i < n && i < (int)b.size(); ++i)
            for (int j = 0; j < 3; ++j) out[3 * i + j] = b[i][j];
        return (int)b.size();
    }, -1);
}

long long fg_grad_pack(void* h, float* buf, long long cap, int unpack) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        if (!c.train) throw Err("this handle was created for inference only");
        const long long tail = c.off[7] - c.off[1];
        const long long n = c.n_wlive + tail;
        if (!buf || cap == 0) return n;
        if (cap < n) throw Err("fg_grad_pack: the buffer holds " + std::to_string(cap) + " floats, the packed gradient " +
                               std::to_string(n));
        if (c.n_wlive)
            launch(c, K_NORM, [&]() {
                pdl(c, k_grad_pack, blocks(c.n_wlive), 256, 0, c.G, (const int*)c.d_wlive, buf, c.n_wlive, unpack);
            });
        float* g = c.G + c.off[1];
        float* b = buf + c.n_wlive;
        if (unpack) CK(cudaMemcpyAsync(g, b, (size_t)tail * 4, cudaMemcpyDeviceToDevice, c.st));
        else CK(cudaMemcpyAsync(b, g, (size_t)tail * 4, cudaMemcpyDeviceToDevice, c.st));
        return n;
    }, (long long)-1);
}

int fg_plan(void* h, long long* out, int n) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        std::vector<long long> v;
        for (const Hop& hp : c.hop) {
            const long long row[8] = {hp.rows, hp.n_src, hp.E, hp.P, hp.T, hp.n_live_dst, hp.n_live_src, hp.live_edges};
            v.insert(v.end(), row, row + 8);
        }
        const long long tail[4] = {c.n_plug_live, c.n_s, c.fan, c.n_dn};
        v.insert(v.end(), tail, tail + 4);
        for (int i = 0; i < n && i < (int)v.size(); ++i) out[i] = v[i];
        return (int)v.size();
    }, -1);
}

void fc_set_stream(void* h, void* stream) {
    guarded(h, [&]() { as_core(h)->st = static_cast<cudaStream_t>(stream); return 0; }, 0);
}

int fg_flat(void* h, int which, float** ptr, long long* n) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        float* p = flat(c, which);
        if (!p) throw Err("no such array in this handle (which " + std::to_string(which) + ")");
        *ptr = p;
        *n = c.off[7];
        if (which <= 1) c.folded = -1;       // the caller may write the weights through this pointer
        return 0;
    }, -1);
}

void fc_copy(void* h, int which, int to_core, float** ptrs) {
    guarded(h, [&]() {
        Core& c = *as_core(h);
        float* A = flat(c, which);
        if (!A) throw Err("fc_copy: no such array in this handle (which " + std::to_string(which) + ")");
        for (int i = 0; i < 7; ++i) {
            if (!ptrs[i]) continue;
            float* mine = A + c.off[i];
            const size_t bytes = (size_t)c.psize[i] * 4;
            if (to_core) CK(cudaMemcpyAsync(mine, ptrs[i], bytes, cudaMemcpyDeviceToDevice, c.st));
            else CK(cudaMemcpyAsync(ptrs[i], mine, bytes, cudaMemcpyDeviceToDevice, c.st));
        }
        if (to_core && which <= 1) c.folded = -1;
        return 0;
    }, 0);
}

void fc_forward(void* h, const float* obs, int B, float* logits, int ema) {
    guarded(h, [&]() {
        Core& c = *as_core(h);
        check_batch(c, B);
        forward(c, obs, B, logits, ema, c.train);
        return 0;
    }, 0);
}

void fc_zero_grad(void* h) {
    guarded(h, [&]() {
        Core& c = *as_core(h);
        if (!c.train) throw Err("this handle was created for inference only");
        CK(cudaMemsetAsync(c.G, 0, c.off[7] * 4, c.st));
        return 0;
    }, 0);
}

void fc_backward(void* h, const float* dlogits, int B) {
    guarded(h, [&]() {
        Core& c = *as_core(h);
        check_batch(c, B);
        if (!c.train) throw Err("this handle was created for inference only");
        launch(c, K_TRANSPOSE, [&]() { pdl(c, k_to_neuron_major, dim3((B + 31) / 32, (c.n_act + 31) / 32), dim3(32, 8), 0, dlogits, c.dl, c.n_act,
                                                                                            B, B); });
        backward(c, B);
        return 0;
    }, 0);
}

float fc_grad_norm(void* h) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        if (!c.train) throw Err("this handle was created for inference only");
        return grad_norm(c, 0.f);
    }, 0.f);
}

float fc_step(void* h, float lr, float lr_neuron, float lr_plug, float max_norm, float ema) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        if (!c.train) throw Err("this handle was created for inference only");
        const float* scale = nullptr;
        if (max_norm > 0) { grad_norm_launch(c, max_norm); scale = c.norm; }
        ++c.adam_t;
        const long long tc = std::min<long long>(c.adam_t, 100000);
        const float c1 = 1.f - (float)pow(0.9, (double)tc), c2 = 1.f - (float)pow(0.999, (double)tc);
        const long long n = c.off[7];
        launch(c, K_ADAM, [&]() { pdl(c, k_adam, (unsigned)std::min<long long>(blocks((n + 3) / 4), 148 * 8), 256, 0,
            c.P, c.G, c.M, c.V, c.EMA, n, c.off[1], c.off[3], lr, lr_neuron, lr_plug, c1, c2, scale, ema); });
        c.folded = -1;
        // the update is queued behind the norm on the device; the host reads the norm afterwards
        return max_norm > 0 ? read_norm(c) : 0.f;
    }, 0.f);
}

long long fc_adam_t(void* h, long long set) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        if (set >= 0) c.adam_t = set;
        return c.adam_t;
    }, (long long)0);
}

void fc_sync(void* h) {
    guarded(h, [&]() {
        Core& c = *as_core(h);
        CK(cudaStreamSynchronize(c.st));
        int e = 0;
        CK(cudaMemcpy(&e, c.d_err, sizeof(int), cudaMemcpyDeviceToHost));
        if (e) {
            CK(cudaMemset(c.d_err, 0, sizeof(int)));
            throw Err("tensor-core kernel: a wait expired (code " + std::to_string(e) + "); its results are not valid");
        }
        return 0;
    }, 0);
}

int fg_teach(void* h, const float* obs, const float* teacher, int B, float inv_temp, float* logits, double* stats) {
    return fg_teach_ex(h, obs, teacher, B, inv_temp, (float)B, logits, stats);
}

int fg_teach_ex(void* h, const float* obs, const float* teacher, int B, float inv_temp, float loss_norm, float* logits,
                double* stats) {
    return guarded(h, [&]() {
        if (!(loss_norm > 0.f)) throw Err("fg_teach_ex: loss_norm must be positive");
        Core& c = *as_core(h);
        check_batch(c, B);
        if (!c.train) throw Err("this handle was created for inference only");
        forward(c, obs, B, logits, 0, true);
        CK(cudaMemsetAsync(c.stats, 0, 16, c.st));
        launch(c, K_LOSS, [&]() { pdl(c, k_loss, blocks(B, kLossS), kLossT, 0, c.lg, teacher, c.dl, c.kl_s, c.ag_s, c.n_act, B, B, inv_temp, 1.f / loss_norm); });
        launch(c, K_LOSS, [&]() { pdl(c, k_loss_stats, 1, kStatsT, 0, c.kl_s, c.ag_s, c.stats, B); });
        backward(c, B);
        if (stats) {
            float s[2];
            CK(cudaMemcpyAsync(s, c.stats, 8, cudaMemcpyDeviceToHost, c.st));
            CK(cudaStreamSynchronize(c.st));
            stats[0] = s[0];
            stats[1] = s[1];
        }
        return 0;
    }, -1);
}

int fg_survey(void* h, const float* obs, const float* teacher, int B, int ema, int* fired, float* sq, double* stats) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        check_batch(c, B);
        if (!obs || !fired || !sq) throw Err("fg_survey: obs, fired and sq are required");
        const bool loss = teacher && stats;
        if (loss && !c.train) throw Err("fg_survey: the loss needs a handle made for training");
        c.sv_fired = fired;
        c.sv_sq = sq;
        try {
            forward(c, obs, B, nullptr, ema, loss);
        } catch (...) {
            c.sv_fired = nullptr;
            c.sv_sq = nullptr;
            throw;
        }
        c.sv_fired = nullptr;
        c.sv_sq = nullptr;
        launch(c, K_HOP_FWD, [&]() {
            const unsigned g = (unsigned)((c.n_s + kWarps - 1) / kWarps);
            if (c.bf16) pdl(c, k_count_fired<__nv_bfloat16>, g, kThreads, 0, (const __nv_bfloat16*)c.h0, fired, c.n_s, B, B);
            else if (c.f16) pdl(c, k_count_fired<__half>, g, kThreads, 0, (const __half*)c.h0, fired, c.n_s, B, B);
            else pdl(c, k_count_fired<float>, g, kThreads, 0, (const float*)c.h0, fired, c.n_s, B, B);
        });
        if (loss) {
            CK(cudaMemsetAsync(c.stats, 0, 16, c.st));
            launch(c, K_LOSS, [&]() { pdl(c, k_loss, blocks(B, kLossS), kLossT, 0, c.lg, teacher, c.dl, c.kl_s, c.ag_s, c.n_act, B, B, 1.f, 1.f / B); });
            launch(c, K_LOSS, [&]() { pdl(c, k_loss_stats, 1, kStatsT, 0, c.kl_s, c.ag_s, c.stats, B); });
            float s[2];
            CK(cudaMemcpyAsync(s, c.stats, 8, cudaMemcpyDeviceToHost, c.st));
            CK(cudaStreamSynchronize(c.st));
            stats[0] = s[0];
            stats[1] = s[1];
        }
        return 0;
    }, -1);
}

int fg_forward_host(void* h, const float* obs_host, int B, float* logits_host, int ema) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        check_batch(c, B);
        if (!c.obs_dev) {
            c.obs_dev = dalloc<float>(c, (size_t)c.maxB * c.obs_dim);
            c.logits_dev = dalloc<float>(c, (size_t)c.maxB * c.n_act);
            CK(cudaStreamCreateWithFlags(&c.h2d, cudaStreamNonBlocking));
            CK(cudaStreamCreateWithFlags(&c.d2h, cudaStreamNonBlocking));
        }
        // Pieces that grow threefold from a small first one (B/32 rounded up to 1,024, between 1,024 and 4,096) up to
        // 40,960 samples, multiples of 1,024 but the last: the first piece's upload is the only copy not hidden behind
        // compute, and each piece's upload (PCIe ~40-50 GB/s, ~2 KB a sample) takes less time than the forward of the
        // piece before it (~7.7K samples/ms at bf16). A sample's logits do not depend on the piece it is in.
        // Measured end to end (bf16, batch 65,536): 6.17M decisions/s with four equal pieces of 16,384, 6.65M with
        // 2,048 / 6,144 / 18,432 / 38,912; batch 8,192: 3.46M in one piece, 5.00M in 1,024 / 3,072 / 4,096; fp32
        // batch 4,096: 2.37M in one piece, 2.91M in 1,024 / 3,072.
        std::vector<std::pair<int, int>> pieces;           // (first sample, count)
        {
            auto up = [](long long v) { return (int)((v + 1023) / 1024 * 1024); };
            int sz = std::min(4096, std::max(1024, up(B / 32)));
            if (B <= 2 * sz) {
                pieces.emplace_back(0, B);
            } else {
                pieces.emplace_back(0, sz);
                for (int b0 = sz; b0 < B; b0 += sz) {
                    sz = std::min(40960, up(3LL * sz));
                    if (B - b0 - sz < sz / 2) sz = B - b0;      // a short remainder joins this piece
                    sz = std::min(sz, B - b0);
                    pieces.emplace_back(b0, sz);
                }
            }
        }
        std::vector<cudaEvent_t> ev;
        auto event = [&]() {
            cudaEvent_t e;
            CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
            ev.push_back(e);
            return e;
        };
        try {
            cudaEvent_t start = event();
            CK(cudaEventRecord(start, c.st));          // the copies start after the handle's earlier work
            CK(cudaStreamWaitEvent(c.h2d, start, 0));
            std::vector<cudaEvent_t> in_done, out_done;
            for (const auto& pc : pieces) {
                const int b0 = pc.first, n = pc.second;
                CK(cudaMemcpyAsync(c.obs_dev + (size_t)b0 * c.obs_dim, obs_host + (size_t)b0 * c.obs_dim,
                                   (size_t)n * c.obs_dim * 4, cudaMemcpyHostToDevice, c.h2d));
                cudaEvent_t e = event();
                CK(cudaEventRecord(e, c.h2d));
                in_done.push_back(e);
            }
            for (size_t i = 0; i < pieces.size(); ++i) {
                const int b0 = pieces[i].first, n = pieces[i].second;
                CK(cudaStreamWaitEvent(c.st, in_done[i], 0));
                forward(c, c.obs_dev + (size_t)b0 * c.obs_dim, n, c.logits_dev + (size_t)b0 * c.n_act, ema, false);
                cudaEvent_t e = event();
                CK(cudaEventRecord(e, c.st));
                CK(cudaStreamWaitEvent(c.d2h, e, 0));
                CK(cudaMemcpyAsync(logits_host + (size_t)b0 * c.n_act, c.logits_dev + (size_t)b0 * c.n_act,
                                   (size_t)n * c.n_act * 4, cudaMemcpyDeviceToHost, c.d2h));
            }
            cudaEvent_t done = event();
            CK(cudaEventRecord(done, c.d2h));
            CK(cudaStreamWaitEvent(c.st, done, 0));     // later work of the handle waits for the copies
            CK(cudaEventSynchronize(done));
        } catch (...) {
            for (auto e : ev) cudaEventDestroy(e);
            throw;
        }
        for (auto e : ev) cudaEventDestroy(e);
        c.lastB = 0;                                    // chunked states: no backward through them
        return 0;
    }, -1);
}

long long fg_launches(void* h) {
    return guarded(h, [&]() { return as_core(h)->launches; }, (long long)-1);
}

int fg_timing_classes(void* h, unsigned mask) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        if (!mask && !c.timer.recs.empty()) throw Err("fg_timing: read the recorded times (fg_timing_read) first");
        c.timer.mask = mask & ((1u << K_NCLASS) - 1u);
        return 0;
    }, -1);
}

int fg_timing(void* h, int on) { return fg_timing_classes(h, on ? ~0u : 0u); }

int fg_timing_read(void* h, double* ms, long long* count, int n) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        for (int i = 0; i < n; ++i) { ms[i] = 0.0; count[i] = 0; }
        CK(cudaStreamSynchronize(c.st));
        for (auto& r : c.timer.recs) {
            float t = 0.f;
            CK(cudaEventElapsedTime(&t, r.a, r.b));
            if (r.cls < n) { ms[r.cls] += t; ++count[r.cls]; }
        }
        c.timer.recs.clear();
        c.timer.used = 0;
        return (int)K_NCLASS;
    }, -1);
}

int fg_layer(void* h, int k, float* out, int B) {
    return guarded(h, [&]() {
        Core& c = *as_core(h);
        if (k < 0 || k > c.hops) throw Err("no such layer");
        if (B != c.lastB) throw Err("fg_layer: batch differs from the last forward's");
        const void* src = k ? c.hop[k - 1].d_h : c.h0;
        const size_t n = (size_t)c.sizes[k] * B;
        const bool f32 = act_bytes(c) == 4 || (k > 0 && c.hop[k - 1].out_f32);
        if (!f32 && c.f16) {
            std::vector<__half> hb(n);
            CK(cudaMemcpyAsync(hb.data(), src, n * 2, cudaMemcpyDeviceToHost, c.st));
            CK(cudaStreamSynchronize(c.st));
            std::vector<float> tmp(n);
            for (size_t i = 0; i < n; ++i) tmp[i] = __half2float(hb[i]);
            CK(cudaMemcpyAsync(out, tmp.data(), n * 4, cudaMemcpyHostToDevice, c.st));
            CK(cudaStreamSynchronize(c.st));
        } else if (f32) {
            CK(cudaMemcpyAsync(out, src, n * 4, cudaMemcpyDeviceToDevice, c.st));
        } else {
            std::vector<float> tmp;   // small layers in tests only: convert on the host
            std::vector<__nv_bfloat16> hb(n);
            CK(cudaMemcpyAsync(hb.data(), src, n * 2, cudaMemcpyDeviceToHost, c.st));
            CK(cudaStreamSynchronize(c.st));
            tmp.resize(n);
            for (size_t i = 0; i < n; ++i) tmp[i] = __bfloat162float(hb[i]);
            CK(cudaMemcpyAsync(out, tmp.data(), n * 4, cudaMemcpyHostToDevice, c.st));
            CK(cudaStreamSynchronize(c.st));
        }
        return 0;
    }, -1);
}

}  // extern "C"
