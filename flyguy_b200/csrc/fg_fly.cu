// The playing network's C interface of the reference (flyguy/native/fly_infer.cpp: fly_create, fly_set_plug,
// fly_set_hop, fly_set_out, fly_forward, fly_free, lines 31-99), on the GPU: the same names, arguments and host
// buffers, so FlyActor._native (flyguy/fly.py:187-241) loads this library by path. A decision for a few cars (the
// bot asks for 1-8 at a time) is latency, not throughput: the weights stay on the GPU; a call copies the observations
// in, runs the plug as a thread per (row, car), the hops as 4 lanes per (row, car) for up to 8 cars (else one), the
// output plug as a warp per (car, action), and
// copies the logits (and, when asked, the firing bytes of the first car - the visualizer's tap) back; the call is one
// CUDA graph per (cars, tap), with pinned staging buffers.
//
// Each hop's connections arrive by SOURCE neuron (tcrow / tcol, strengths in that order, as fly_infer.cpp walks them)
// and are regrouped by target row at set time, a row's connections ordered by (source, position) (one lane per (row,
// car) adds them in the order the reference's scatter does; several lanes add interleaved parts). tap: one byte per neuron state of car 0, layer
// after layer, 255 * tanh(1.5 * state) for a positive state, else 0 (fly_infer.cpp:31, 70-87).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <numeric>
#include <string>
#include <vector>

#include "flyguy_b200.h"

namespace {

thread_local std::string g_fly_error;

struct FlyErr {
    std::string msg;
};
#define FCK(call)                                                                                   \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess) throw FlyErr{std::string(#call) + ": " + cudaGetErrorString(e_)};   \
    } while (0)

template <class X>
struct DevArr {
    X* p = nullptr;
    size_t n = 0;
    void set(const X* host, size_t count) {
        if (p) cudaFree(p);
        p = nullptr;
        n = count;
        FCK(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(X)));
        if (count) FCK(cudaMemcpy(p, host, count * sizeof(X), cudaMemcpyHostToDevice));
    }
    void reserve(size_t count) {
        if (count <= n && p) return;
        if (p) cudaFree(p);
        p = nullptr;
        FCK(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(X)));
        n = count;
    }
    ~DevArr() {
        if (p) cudaFree(p);
    }
};

struct FlyHop {
    int rows = 0, src = 0;
    DevArr<int> crow, col, drow;       // by target: row pointers, source of each connection; sensory drive row or -1
    DevArr<float> w, g, t;             // strength per connection (by target), gain and threshold per row
};
struct Fly {
    int obs_dim = 0, n_act = 0, hops = 0, n_s = 0, n_dn = 0, max_rows = 0;
    DevArr<int> in_crow, in_col, dn;
    DevArr<float> in_w, in_b, g0, t0, out_w, out_b;
    std::vector<FlyHop> hop;
    DevArr<float> x, drive, sa, sb, lg;
    DevArr<unsigned char> tap;
    int cap = 0;                       // cars the buffers hold
    float *hx = nullptr, *hlg = nullptr;   // pinned staging of the observations and logits
    unsigned char* htap = nullptr;         // pinned staging of the firing bytes
    cudaStream_t st = nullptr;
    std::map<std::pair<int, bool>, cudaGraphExec_t> graphs;   // (cars, tap) -> the whole call as one graph
    void forget_graphs() {
        for (auto& g : graphs) cudaGraphExecDestroy(g.second);
        graphs.clear();
    }
    ~Fly() {
        forget_graphs();
        if (hx) cudaFreeHost(hx);
        if (hlg) cudaFreeHost(hlg);
        if (htap) cudaFreeHost(htap);
        if (st) cudaStreamDestroy(st);
    }
};

__device__ __forceinline__ unsigned char shade(float v) {
    return v > 0.f ? (unsigned char)(255.f * tanhf(1.5f * v)) : (unsigned char)0;
}

// sensory row r of car b: drive = in_b + sum in_w * obs, state = relu(g0 * drive - t0)
__global__ void k_fly_plug(const float* __restrict__ obs, const int* __restrict__ crow, const int* __restrict__ col,
                           const float* __restrict__ w, const float* __restrict__ bias, const float* __restrict__ g,
                           const float* __restrict__ t, float* __restrict__ drive, float* __restrict__ h,
                           unsigned char* __restrict__ tap, int n_s, int obs_dim, int B) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_s * B) return;
    const int r = i / B, b = i - r * B;
    const float* x = obs + (size_t)b * obs_dim;
    float acc = __ldg(&bias[r]);
    for (int e = __ldg(&crow[r]); e < __ldg(&crow[r + 1]); ++e) acc = fmaf(__ldg(&w[e]), __ldg(&x[__ldg(&col[e])]), acc);
    drive[i] = acc;
    const float v = fmaxf(fmaf(__ldg(&g[r]), acc, -__ldg(&t[r])), 0.f);
    h[i] = v;
    if (tap && b == 0) tap[r] = shade(v);
}
// hop row r of car b: the row's connections, + drive, relu(g * z - t); S lanes per (row, car) share the
// connections (lane k takes every S-th: S = 4 for a few cars, so a chain is a quarter of the row) and add up by shuffles
template <int S>
__global__ void k_fly_hop(const int* __restrict__ crow, const int* __restrict__ col, const float* __restrict__ w,
                          const float* __restrict__ g, const float* __restrict__ t, const int* __restrict__ drow,
                          const float* __restrict__ drive, const float* __restrict__ hp, float* __restrict__ h,
                          unsigned char* __restrict__ tap, int rows, int B) {
    const long long gi = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int i = (int)(gi / S), k = (int)(gi % S);
    const bool live = i < rows * B;
    const int r = live ? i / B : 0, b = live ? i - r * B : 0;
    float acc = 0.f;
    if (live) {
        const int e1 = __ldg(&crow[r + 1]);
#pragma unroll 4
        for (int e = __ldg(&crow[r]) + k; e < e1; e += S)
            acc = fmaf(__ldg(&w[e]), __ldg(&hp[(size_t)__ldg(&col[e]) * B + b]), acc);
    }
#pragma unroll
    for (int o = S / 2; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (!live || k) return;
    const int d = __ldg(&drow[r]);
    if (d >= 0) acc += __ldg(&drive[(size_t)d * B + b]);
    const float v = fmaxf(fmaf(__ldg(&g[r]), acc, -__ldg(&t[r])), 0.f);
    h[i] = v;
    if (tap && b == 0) tap[r] = shade(v);
}
// logits [B, n_act]: out_b + sum over descending rows of out_w * state; a warp per (car, action), lanes over the rows
// (a decision is latency: 1,332 terms as 32 chains of 42 and a shuffle reduction, not one chain of 1,332)
__global__ void k_fly_out(const float* __restrict__ w, const float* __restrict__ bias, const int* __restrict__ dn,
                          const float* __restrict__ h, float* __restrict__ lg, int n_act, int n_dn, int B) {
    const int i = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (i >= n_act * B) return;
    const int b = i / n_act, a = i - b * n_act;
    const float* wa = w + (size_t)a * n_dn;
    float acc = 0.f;
    for (int j = lane; j < n_dn; j += 32) acc = fmaf(__ldg(&wa[j]), __ldg(&h[(size_t)__ldg(&dn[j]) * B + b]), acc);
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) lg[i] = __ldg(&bias[a]) + acc;
}

template <class F>
void fly_guard(F&& f) {
    try {
        f();
        g_fly_error.clear();
    } catch (const FlyErr& e) {
        g_fly_error = e.msg;
    } catch (const std::exception& e) {
        g_fly_error = e.what();
    }
}

}  // namespace

extern "C" {

void* fly_create(int obs_dim, int n_act, int hops) {
    Fly* f = nullptr;
    fly_guard([&]() {
        if (obs_dim <= 0 || n_act <= 0 || hops <= 0 || hops > 64) throw FlyErr{"fly_create: bad sizes"};
        std::unique_ptr<Fly> nf(new Fly);
        nf->obs_dim = obs_dim;
        nf->n_act = n_act;
        nf->hops = hops;
        nf->hop.resize(hops);
        FCK(cudaStreamCreateWithFlags(&nf->st, cudaStreamNonBlocking));
        f = nf.release();
    });
    return f;
}

void fly_set_plug(void* p, int n_s, int E, const int* crow, const int* col, const float* w, const float* b,
                  const float* g0, const float* t0) {
    fly_guard([&]() {
        if (!p) throw FlyErr{"fly_set_plug: null handle"};
        Fly& f = *static_cast<Fly*>(p);
        f.forget_graphs();                               // (the graphs hold the old arrays' addresses)
        f.n_s = n_s;
        f.in_crow.set(crow, n_s + 1);
        f.in_col.set(col, E);
        f.in_w.set(w, E);
        f.in_b.set(b, n_s);
        f.g0.set(g0, n_s);
        f.t0.set(t0, n_s);
    });
}

void fly_set_hop(void* p, int k, int rows, int src, int E, const int* tcrow, const int* tcol, const float* w,
                 const float* g, const float* t, const int* drow) {
    fly_guard([&]() {
        if (!p) throw FlyErr{"fly_set_hop: null handle"};
        Fly& f = *static_cast<Fly*>(p);
        if (k < 0 || k >= f.hops) throw FlyErr{"fly_set_hop: hop index out of range"};
        f.forget_graphs();
        // by source -> by target, a row's connections in (source, position) order
        std::vector<int> cnt(rows + 1, 0);
        for (int e = 0; e < E; ++e) {
            if (tcol[e] < 0 || tcol[e] >= rows) throw FlyErr{"fly_set_hop: target row out of range"};
            ++cnt[tcol[e] + 1];
        }
        for (int r = 0; r < rows; ++r) cnt[r + 1] += cnt[r];
        std::vector<int> fill(cnt.begin(), cnt.end() - 1), col(E);
        std::vector<float> wt(E);
        for (int j = 0; j < src; ++j)
            for (int e = tcrow[j]; e < tcrow[j + 1]; ++e) {
                const int q = fill[tcol[e]]++;
                col[q] = j;
                wt[q] = w[e];
            }
        FlyHop& h = f.hop[k];
        h.rows = rows;
        h.src = src;
        h.crow.set(cnt.data(), rows + 1);
        h.col.set(col.data(), E);
        h.w.set(wt.data(), E);
        h.g.set(g, rows);
        h.t.set(t, rows);
        h.drow.set(drow, rows);
    });
}

void fly_set_out(void* p, int n_dn, const int* dn, const float* w, const float* b) {
    fly_guard([&]() {
        if (!p) throw FlyErr{"fly_set_out: null handle"};
        Fly& f = *static_cast<Fly*>(p);
        f.forget_graphs();
        f.n_dn = n_dn;
        f.dn.set(dn, n_dn);
        f.out_w.set(w, (size_t)f.n_act * n_dn);
        f.out_b.set(b, f.n_act);
        f.max_rows = f.n_s;
        for (auto& h : f.hop) f.max_rows = std::max(f.max_rows, h.rows);
        f.cap = 0;                                       // (the state buffers follow the largest layer)
    });
}

}  // extern "C"

namespace {
// one call's work on f.st: pinned observations up, plug, hops, output plug, pinned logits (and firing bytes) down
void enqueue(Fly& f, int batch, bool with_tap, size_t total) {
    unsigned char* tp = with_tap ? f.tap.p : nullptr;
    const cudaStream_t st = f.st;
    FCK(cudaMemcpyAsync(f.x.p, f.hx, (size_t)batch * f.obs_dim * 4, cudaMemcpyHostToDevice, st));
    auto blocks = [](long long n) { return (unsigned)((n + 127) / 128); };
    k_fly_plug<<<blocks((long long)f.n_s * batch), 128, 0, st>>>(f.x.p, f.in_crow.p, f.in_col.p, f.in_w.p, f.in_b.p,
                                                                  f.g0.p, f.t0.p, f.drive.p, f.sa.p, tp, f.n_s,
                                                                  f.obs_dim, batch);
    float *hp = f.sa.p, *hn = f.sb.p;
    size_t off = f.n_s;
    for (auto& h : f.hop) {
        if (batch <= 8)                                  // a few cars: 4 lanes per (row, car)
            k_fly_hop<4><<<blocks(4LL * h.rows * batch), 128, 0, st>>>(h.crow.p, h.col.p, h.w.p, h.g.p, h.t.p,
                                                                        h.drow.p, f.drive.p, hp, hn,
                                                                        tp ? tp + off : nullptr, h.rows, batch);
        else
            k_fly_hop<1><<<blocks((long long)h.rows * batch), 128, 0, st>>>(h.crow.p, h.col.p, h.w.p, h.g.p, h.t.p,
                                                                          h.drow.p, f.drive.p, hp, hn,
                                                                          tp ? tp + off : nullptr, h.rows, batch);
        off += h.rows;
        std::swap(hp, hn);
    }
    k_fly_out<<<(unsigned)((f.n_act * batch + 3) / 4), 128, 0, st>>>(f.out_w.p, f.out_b.p, f.dn.p, hp, f.lg.p,
                                                                      f.n_act, f.n_dn, batch);
    FCK(cudaGetLastError());
    FCK(cudaMemcpyAsync(f.hlg, f.lg.p, (size_t)batch * f.n_act * 4, cudaMemcpyDeviceToHost, st));
    if (with_tap) FCK(cudaMemcpyAsync(f.htap, f.tap.p, total, cudaMemcpyDeviceToHost, st));
}
}  // namespace

extern "C" {

void fly_forward(void* p, const float* obs, int batch, float* logits, unsigned char* tap) {
    bool ok = false;
    fly_guard([&]() {
        if (!p) throw FlyErr{"fly_forward: null handle"};
        Fly& f = *static_cast<Fly*>(p);
        if (batch <= 0) return;
        size_t total = f.n_s;
        for (auto& h : f.hop) total += h.rows;
        if (batch > f.cap || !f.htap) {
            f.forget_graphs();
            const int cap = std::max(batch, f.cap);
            f.x.reserve((size_t)cap * f.obs_dim);
            f.drive.reserve((size_t)cap * f.n_s);
            f.sa.reserve((size_t)cap * f.max_rows);
            f.sb.reserve((size_t)cap * f.max_rows);
            f.lg.reserve((size_t)cap * f.n_act);
            f.tap.reserve(total);
            if (f.hx) cudaFreeHost(f.hx);
            if (f.hlg) cudaFreeHost(f.hlg);
            if (f.htap) cudaFreeHost(f.htap);
            f.hx = f.hlg = nullptr;
            f.htap = nullptr;
            FCK(cudaMallocHost(&f.hx, (size_t)cap * f.obs_dim * 4));
            FCK(cudaMallocHost(&f.hlg, (size_t)cap * f.n_act * 4));
            FCK(cudaMallocHost(&f.htap, total));
            f.cap = cap;
        }
        memcpy(f.hx, obs, (size_t)batch * f.obs_dim * 4);
        // the call as one CUDA graph per (cars, tap): made on first use, replayed after (launch cost once, not 5x)
        const auto key = std::make_pair(batch, tap != nullptr);
        auto it = f.graphs.find(key);
        if (it == f.graphs.end()) {
            cudaGraph_t g = nullptr;
            cudaGraphExec_t ge = nullptr;
            FCK(cudaStreamBeginCapture(f.st, cudaStreamCaptureModeThreadLocal));
            try {
                enqueue(f, batch, tap != nullptr, total);
            } catch (...) {
                cudaStreamEndCapture(f.st, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            FCK(cudaStreamEndCapture(f.st, &g));
            const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
            cudaGraphDestroy(g);
            FCK(e);
            it = f.graphs.emplace(key, ge).first;
        }
        FCK(cudaGraphLaunch(it->second, f.st));
        FCK(cudaStreamSynchronize(f.st));
        memcpy(logits, f.hlg, (size_t)batch * f.n_act * 4);
        if (tap) memcpy(tap, f.htap, total);
        ok = true;
    });
    if (!ok && p && logits && batch > 0)             // (the interface has no status: a failed call answers NaN)
        std::fill(logits, logits + (size_t)batch * static_cast<Fly*>(p)->n_act, std::nanf(""));
}

void fly_free(void* p) { delete static_cast<Fly*>(p); }

const char* fg_fly_last_error(void) { return g_fly_error.c_str(); }

}  // extern "C"
