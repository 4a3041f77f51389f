// The standalone teaching trainer (the reference's flyguy/native/flyguy_train.cu main(), lines 631-788), on this
// library's public C-ABI: recorded teacher data in FLYD chunks kept on the GPU as 16-bit numbers, batches drawn and
// unpacked on the GPU, the fused teaching step (fg_teach_ex: forward, KL loss, backward) and Adam with the weights'
// running average (fc_step), the reference's learning-rate schedule (halved every --half-life steps, floored at
// --lr-min), FLYP / FLYO checkpoints, restart from the run's own save, a STOP file.
//
//   fg_train NET.bin PARAMS.bin DATA_DIR OUT_PREFIX [--batch 512] [--lr 3e-4] [--lr-neuron 1e-4] [--lr-plug 3e-4]
//            [--lr-min 3e-5] [--half-life 20000] [--ema 0.999] [--log 100] [--save-sec 120] [--steps 0] [--clip 0]
//            [--temp 1] [--ring 3] [--max-reuse -1] [--eval-batches 16] [--seed 12345] [--revive-every 0]
//            [--revive-batches 4] [--revive-target 0.4] [--revive-first 0]
//
// Data (flyguy/native/flyguy_train.cu:13-14, 366-417): DATA_DIR/chunk_*.bin = "FLYD", n (int64), obs_dim, n_act
// (int32), then n x obs_dim observations and n x n_act teacher logits as IEEE fp16. The newest --ring chunks form the
// ring every batch is drawn from (uniformly over their samples); chunks are picked up as they appear or are rewritten
// (the directory is looked at every --log steps); --max-reuse: at most that many draws per recorded sample before the
// trainer waits for new data (default 4 for an open-ended run, off with --steps). A new chunk is scored (KL and
// argmax agreement of the running average at temperature 1, --eval-batches batches) before it joins the ring.
// Saves OUT.bin and OUT.ema.bin (FLYP: "FLYP", step int64, the seven float32 arrays) and OUT.opt.bin (FLYO: "FLYO",
// step, adam_t, then M and V of each array) - export.py's formats; started from OUT.bin the run goes on from there with
// its running average and optimiser state. Eval lines (a new chunk, before it joins the ring) carry the running
// average's and the raw weights' KL and agreement, each layer's firing share and the silent neurons (fg_survey; the
// reference's survey() / firing_line(), flyguy_train.cu:437-471). --revive-every N [--revive-batches 4]
// [--revive-target 0.4] [--revive-first 0]: every N steps the neurons past the sensory layer that fire for none of
// the surveyed samples are brought back with the network's output unchanged (the reference's revive(), 486-551).
//
// Sample draws: sample i of step s is splitmix64(seed ^ (s * 2^32 + i)) modulo the ring's sample count (counter-based,
// so a Python re-run draws the same samples; the reference uses a sequential mt19937_64 stream).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <map>
#include <memory>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "flyguy_b200.h"

namespace {

namespace fs = std::filesystem;

struct TrainErr {
    std::string msg;
};
#define TCK(call)                                                                                   \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess) throw TrainErr{std::string(#call) + ": " + cudaGetErrorString(e_)};  \
    } while (0)

__host__ __device__ inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

constexpr int kMaxRing = 16;
struct RingDev {                 // the ring as the gather kernel sees it
    const __half* obs[kMaxRing];
    const __half* lg[kMaxRing];
    long long n[kMaxRing];
    int count;
    long long total;
};

// batch rows b: sample u = splitmix64(seed ^ (step << 32 | b)) mod total, found in the ring's chunks in order;
// obs [B, obs_dim] and teacher [B, n_act] fp32 (the layout fg_teach_ex takes). A warp per sample.
__global__ void k_draw_gather(RingDev r, uint64_t seed, long long step, int B, int obs_dim, int n_act, float* obs,
                              float* teacher) {
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= B) return;
    long long s = (long long)(splitmix64(seed ^ (((uint64_t)step << 32) | (uint64_t)b)) % (uint64_t)r.total);
    int c = 0;
    while (c + 1 < r.count && s >= r.n[c]) { s -= r.n[c]; ++c; }
    const __half* o = r.obs[c] + (size_t)s * obs_dim;
    const __half* l = r.lg[c] + (size_t)s * n_act;
    for (int i = lane; i < obs_dim; i += 32) obs[(size_t)b * obs_dim + i] = __half2float(o[i]);
    for (int i = lane; i < n_act; i += 32) teacher[(size_t)b * n_act + i] = __half2float(l[i]);
}

struct Chunk {
    std::string name;
    fs::file_time_type mtime;
    long long n = 0;
    __half *obs = nullptr, *lg = nullptr;
    ~Chunk() {
        if (obs) cudaFree(obs);
        if (lg) cudaFree(lg);
    }
};
using ChunkP = std::shared_ptr<Chunk>;

// a FLYD chunk read into GPU memory; nullptr if it is not (yet) a complete chunk of this network's sizes
ChunkP read_chunk(const fs::path& p, int obs_dim, int n_act) {
    FILE* f = fopen(p.string().c_str(), "rb");
    if (!f) return nullptr;
    char magic[4];
    long long n = 0;
    int od = 0, na = 0;
    bool ok = fread(magic, 1, 4, f) == 4 && !memcmp(magic, "FLYD", 4) && fread(&n, 8, 1, f) == 1 &&
              fread(&od, 4, 1, f) == 1 && fread(&na, 4, 1, f) == 1 && od == obs_dim && na == n_act && n > 0;
    std::vector<uint16_t> obs, lg;
    if (ok) {
        obs.resize((size_t)n * od);
        lg.resize((size_t)n * na);
        ok = fread(obs.data(), 2, obs.size(), f) == obs.size() && fread(lg.data(), 2, lg.size(), f) == lg.size();
    }
    fclose(f);
    if (!ok) return nullptr;
    auto c = std::make_shared<Chunk>();
    c->name = p.filename().string();
    c->n = n;
    TCK(cudaMalloc(&c->obs, obs.size() * 2));
    TCK(cudaMalloc(&c->lg, lg.size() * 2));
    TCK(cudaMemcpy(c->obs, obs.data(), obs.size() * 2, cudaMemcpyHostToDevice));
    TCK(cudaMemcpy(c->lg, lg.data(), lg.size() * 2, cudaMemcpyHostToDevice));
    return c;
}

struct Args {
    std::string net, params, data, out;
    int B = 512, log_every = 100, ring = 3, eval_batches = 16, revive_batches = 4, revive_first = 0;
    long long max_steps = 0, revive_every = 0;
    float revive_target = 0.4f;
    double save_sec = 120, half_life = 20000, max_reuse = -1;
    float lr = 3e-4f, lr_neuron = 1e-4f, lr_plug = 3e-4f, lr_min = 3e-5f, ema = 0.999f, clip = 0.f, temp = 1.f;
    uint64_t seed = 12345;
};

Args parse(int argc, const char* const* argv) {
    if (argc < 5) throw TrainErr{"usage: fg_train NET PARAMS DATA_DIR OUT_PREFIX [options]"};
    Args a;
    a.net = argv[1]; a.params = argv[2]; a.data = argv[3]; a.out = argv[4];
    for (int i = 5; i < argc; i += 2) {
        const std::string k = argv[i];
        if (i + 1 >= argc) throw TrainErr{"option " + k + " needs a value"};
        const double v = atof(argv[i + 1]);
        if (k == "--batch") a.B = (int)v;
        else if (k == "--lr") a.lr = (float)v;
        else if (k == "--lr-neuron") a.lr_neuron = (float)v;
        else if (k == "--lr-plug") a.lr_plug = (float)v;
        else if (k == "--lr-min") a.lr_min = (float)v;
        else if (k == "--half-life") a.half_life = v;
        else if (k == "--ema") a.ema = (float)v;
        else if (k == "--log") a.log_every = std::max(1, (int)v);
        else if (k == "--save-sec") a.save_sec = v;
        else if (k == "--steps") a.max_steps = (long long)v;
        else if (k == "--clip") a.clip = (float)v;
        else if (k == "--temp") a.temp = (float)v;
        else if (k == "--ring") a.ring = std::max(1, std::min(kMaxRing, (int)v));
        else if (k == "--max-reuse") a.max_reuse = v;
        else if (k == "--eval-batches") a.eval_batches = (int)v;
        else if (k == "--seed") a.seed = (uint64_t)strtoull(argv[i + 1], nullptr, 10);
        else if (k == "--revive-every") a.revive_every = (long long)v;
        else if (k == "--revive-batches") a.revive_batches = std::max(1, (int)v);
        else if (k == "--revive-target") a.revive_target = (float)v;
        else if (k == "--revive-first") a.revive_first = (int)v;
        else throw TrainErr{"unknown option " + k};
    }
    if (a.B <= 0 || a.B % 32) throw TrainErr{"--batch must be a positive multiple of 32"};
    if (!(a.temp > 0.f)) throw TrainErr{"--temp must be positive"};
    return a;
}

void check(void* h) {
    if (fg_status(h)) throw TrainErr{fg_last_error(h)};
}

struct Sizes {
    long long p[7];
    int obs_dim, n_act;
};
Sizes sizes_of(void* h) {
    long long s[10];
    fc_sizes(h, s);
    check(h);
    Sizes z;
    for (int i = 0; i < 7; ++i) z.p[i] = s[i];
    z.obs_dim = (int)s[7];
    z.n_act = (int)s[8];
    return z;
}

// the seven arrays between host vectors and the handle (which: 0 weights, 1 running average, 2 M, 3 V), through
// device staging buffers
void to_core(void* h, int which, const std::vector<std::vector<float>>& host, const Sizes& z) {
    float* dev[7];
    for (int i = 0; i < 7; ++i) {
        TCK(cudaMalloc(&dev[i], std::max<long long>(z.p[i], 1) * 4));
        TCK(cudaMemcpy(dev[i], host[i].data(), z.p[i] * 4, cudaMemcpyHostToDevice));
    }
    fc_copy(h, which, 1, dev);
    fc_sync(h);
    for (auto p : dev) cudaFree(p);
    check(h);
}
std::vector<std::vector<float>> from_core(void* h, int which, const Sizes& z) {
    float* dev[7];
    for (int i = 0; i < 7; ++i) TCK(cudaMalloc(&dev[i], std::max<long long>(z.p[i], 1) * 4));
    fc_copy(h, which, 0, dev);
    fc_sync(h);
    check(h);
    std::vector<std::vector<float>> out(7);
    for (int i = 0; i < 7; ++i) {
        out[i].resize(z.p[i]);
        TCK(cudaMemcpy(out[i].data(), dev[i], z.p[i] * 4, cudaMemcpyDeviceToHost));
        cudaFree(dev[i]);
    }
    return out;
}

// FLYP: "FLYP", step, the seven arrays (export.py; flyguy_train.cu:258-286)
bool read_flyp(const std::string& path, const Sizes& z, long long& step, std::vector<std::vector<float>>& v) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return false;
    char magic[4];
    bool ok = fread(magic, 1, 4, f) == 4 && !memcmp(magic, "FLYP", 4) && fread(&step, 8, 1, f) == 1;
    v.assign(7, {});
    for (int i = 0; ok && i < 7; ++i) {
        v[i].resize(z.p[i]);
        ok = fread(v[i].data(), 4, v[i].size(), f) == v[i].size();
    }
    fclose(f);
    return ok;
}
void write_atomic(const std::string& path, const std::vector<std::pair<const void*, size_t>>& parts) {
    const std::string tmp = path + ".tmp";
    FILE* f = fopen(tmp.c_str(), "wb");
    if (!f) throw TrainErr{"cannot write " + tmp};
    bool ok = true;
    for (auto& p : parts) ok = ok && fwrite(p.first, 1, p.second, f) == p.second;
    ok = fclose(f) == 0 && ok;
    if (!ok) throw TrainErr{"short write to " + tmp};
    std::error_code ec;
    fs::rename(tmp, path, ec);
    if (ec) {
        fs::remove(path, ec);
        fs::rename(tmp, path, ec);
        if (ec) throw TrainErr{"cannot rename " + tmp};
    }
}
void save_flyp(const std::string& path, long long step, const std::vector<std::vector<float>>& v) {
    std::vector<std::pair<const void*, size_t>> parts{{"FLYP", 4}, {&step, 8}};
    for (auto& a : v) parts.push_back({a.data(), a.size() * 4});
    write_atomic(path, parts);
}
// FLYO: "FLYO", step, adam_t, then M[i], V[i] for each array (flyguy_train.cu:288-307)
void save_flyo(const std::string& path, long long step, long long adam_t, const std::vector<std::vector<float>>& m,
               const std::vector<std::vector<float>>& v) {
    std::vector<std::pair<const void*, size_t>> parts{{"FLYO", 4}, {&step, 8}, {&adam_t, 8}};
    for (int i = 0; i < 7; ++i) {
        parts.push_back({m[i].data(), m[i].size() * 4});
        parts.push_back({v[i].data(), v[i].size() * 4});
    }
    write_atomic(path, parts);
}
bool read_flyo(const std::string& path, const Sizes& z, long long step, long long& adam_t,
               std::vector<std::vector<float>>& m, std::vector<std::vector<float>>& v) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return false;
    char magic[4];
    long long st = -1, at = 0;
    bool ok = fread(magic, 1, 4, f) == 4 && !memcmp(magic, "FLYO", 4) && fread(&st, 8, 1, f) == 1 &&
              fread(&at, 8, 1, f) == 1 && st == step;
    m.assign(7, {});
    v.assign(7, {});
    for (int i = 0; ok && i < 7; ++i) {
        m[i].resize(z.p[i]);
        v[i].resize(z.p[i]);
        ok = fread(m[i].data(), 4, m[i].size(), f) == m[i].size() && fread(v[i].data(), 4, v[i].size(), f) == v[i].size();
    }
    fclose(f);
    if (ok) adam_t = at;
    return ok;
}

double now() { return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count(); }

// what revival needs of NET.bin (export.py:9-16): per hop the rows' neuron ids and the connections (CSR by target,
// weight index per connection), the sensory neuron ids, the descending rows of the last layer
struct NetInfo {
    int obs_dim = 0, n_act = 0, hops = 0, n_neurons = 0, n_w = 0, n_s = 0, fan = 0, n_dn = 0;
    std::vector<int> sizes, n0, dn;
    struct H { std::vector<int> nid, crow, col, widx; };
    std::vector<H> hop;
};
NetInfo read_netinfo(const std::string& path) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) throw TrainErr{"cannot open " + path};
    auto ints = [&](size_t n) {
        std::vector<int> v(n);
        if (n && fread(v.data(), 4, n, f) != n) { fclose(f); throw TrainErr{"short NET.bin " + path}; }
        return v;
    };
    char magic[4];
    if (fread(magic, 1, 4, f) != 4 || memcmp(magic, "FLY1", 4)) { fclose(f); throw TrainErr{"not a NET.bin: " + path}; }
    NetInfo n;
    auto hd = ints(8);
    n.obs_dim = hd[0]; n.n_act = hd[1]; n.hops = hd[2]; n.n_neurons = hd[3]; n.n_w = hd[4]; n.n_s = hd[5];
    n.fan = hd[6]; n.n_dn = hd[7];
    n.sizes = ints(n.hops + 1);
    auto E = ints(n.hops);
    auto in_crow = ints(n.n_s + 1);
    const int e_in = in_crow.back();
    ints(e_in); ints(n.obs_dim + 1); ints(e_in); ints(e_in);     // plug: in_col, in_tcrow, in_tcol, in_tperm
    n.n0 = ints(n.n_s);
    for (int k = 0; k < n.hops; ++k) {
        NetInfo::H h;
        h.nid = ints(n.sizes[k + 1]);
        h.crow = ints(n.sizes[k + 1] + 1);
        h.col = ints(E[k]);
        h.widx = ints(E[k]);
        ints(n.sizes[k] + 1); ints(E[k]); ints(E[k]); ints(n.sizes[k + 1]);   // tcrow, tcol, twidx, drow
        n.hop.push_back(std::move(h));
    }
    n.dn = ints(n.n_dn);
    fclose(f);
    return n;
}

float median_positive(const std::vector<float>& v) {
    std::vector<float> p;
    for (float x : v) if (x > 0.f) p.push_back(x);
    if (p.empty()) return 0.f;
    std::nth_element(p.begin(), p.begin() + p.size() / 2, p.end());
    return p[p.size() / 2];
}

struct Surv {                   // a survey: per row of every layer, samples fired and summed squared input
    std::vector<int> cnt;
    std::vector<float> sq;
    double kl = 0, agree = 0, samples = 0;
};

struct Trainer {
    Args a;
    void* h = nullptr;
    Sizes z{};
    NetInfo net;
    int R = 0;                                          // rows of all layers
    int* d_fired = nullptr;
    float* d_sq = nullptr;
    std::vector<ChunkP> ring;
    std::map<std::string, fs::file_time_type> known;
    float *obs = nullptr, *teacher = nullptr;
    long long step = 0, ran = 0;

    ~Trainer() {
        if (obs) cudaFree(obs);
        if (teacher) cudaFree(teacher);
        if (d_fired) cudaFree(d_fired);
        if (d_sq) cudaFree(d_sq);
        ring.clear();
        if (h) fg_destroy(h);
    }
    RingDev ring_dev() const {
        RingDev r{};
        r.count = (int)ring.size();
        for (size_t i = 0; i < ring.size(); ++i) {
            r.obs[i] = ring[i]->obs;
            r.lg[i] = ring[i]->lg;
            r.n[i] = ring[i]->n;
            r.total += ring[i]->n;
        }
        return r;
    }
    // chunk files new or rewritten since they were read, oldest first
    std::vector<ChunkP> scan() {
        std::vector<std::pair<fs::file_time_type, fs::path>> files;
        std::error_code ec;
        for (auto& e : fs::directory_iterator(a.data, ec)) {
            const auto name = e.path().filename().string();
            if (name.rfind("chunk_", 0) != 0 || e.path().extension() != ".bin") continue;
            std::error_code e2;
            const auto mt = fs::last_write_time(e.path(), e2);
            if (e2) continue;
            auto k = known.find(name);
            if (k == known.end() || k->second != mt) files.push_back({mt, e.path()});
        }
        std::sort(files.begin(), files.end());
        std::vector<ChunkP> got;
        for (auto& fm : files) {
            ChunkP c = read_chunk(fm.second, z.obs_dim, z.n_act);
            if (!c) continue;                                  // being written: the next look has it
            c->mtime = fm.first;
            known[c->name] = fm.first;
            got.push_back(c);
        }
        return got;
    }
    void into_ring(const ChunkP& c) {
        ring.erase(std::remove_if(ring.begin(), ring.end(), [&](const ChunkP& o) { return o->name == c->name; }),
                   ring.end());
        ring.push_back(c);
        std::sort(ring.begin(), ring.end(), [](const ChunkP& x, const ChunkP& y) {
            return x->mtime != y->mtime ? x->mtime < y->mtime : x->name < y->name;
        });
        while ((int)ring.size() > a.ring) ring.erase(ring.begin());
    }
    void draw(const RingDev& r, uint64_t seed, long long s) {
        k_draw_gather<<<(a.B + 7) / 8, 256>>>(r, seed, s, a.B, z.obs_dim, z.n_act, obs, teacher);
        TCK(cudaGetLastError());
    }
    static RingDev ring_of(const std::vector<ChunkP>& src) {
        RingDev r{};
        r.count = (int)src.size();
        for (size_t i = 0; i < src.size(); ++i) {
            r.obs[i] = src[i]->obs; r.lg[i] = src[i]->lg; r.n[i] = src[i]->n; r.total += src[i]->n;
        }
        return r;
    }
    // `batches` batches from src (the same samples for the same seed) through the weights (ema 0) or their running
    // average (ema 1), no learning: loss and agreement at temperature 1, per row the samples fired and summed z^2
    Surv survey(int ema, const std::vector<ChunkP>& src, int batches, uint64_t seed) {
        TCK(cudaMemset(d_fired, 0, (size_t)R * 4));
        TCK(cudaMemset(d_sq, 0, (size_t)R * 4));
        Surv s;
        const RingDev r = ring_of(src);
        for (int i = 0; i < batches; ++i) {
            draw(r, seed, (long long)i);
            double st[2];
            if (fg_survey(h, obs, teacher, a.B, ema, d_fired, d_sq, st)) check(h);
            s.kl += st[0];
            s.agree += st[1];
        }
        s.cnt.resize(R);
        s.sq.resize(R);
        TCK(cudaMemcpy(s.cnt.data(), d_fired, (size_t)R * 4, cudaMemcpyDeviceToHost));
        TCK(cudaMemcpy(s.sq.data(), d_sq, (size_t)R * 4, cudaMemcpyDeviceToHost));
        s.samples = (double)a.B * batches;
        s.kl /= s.samples;
        s.agree /= s.samples;
        return s;
    }
    // per neuron (it can sit in several hops): how many times it fired; play = in a hop past the sensory layer
    void per_neuron(const Surv& s, std::vector<long long>& fired, std::vector<char>& play, std::vector<char>& sens) {
        fired.assign(net.n_neurons, 0);
        play.assign(net.n_neurons, 0);
        sens.assign(net.n_neurons, 0);
        for (int g : net.n0) sens[g] = 1;
        size_t off = net.n_s;
        for (auto& hh : net.hop) {
            for (size_t t = 0; t < hh.nid.size(); ++t) { play[hh.nid[t]] = 1; fired[hh.nid[t]] += s.cnt[off + t]; }
            off += hh.nid.size();
        }
    }
    std::string firing_line(const Surv& s, int& silent, int& in_play) {
        std::vector<long long> fired;
        std::vector<char> play, sens;
        per_neuron(s, fired, play, sens);
        silent = in_play = 0;
        for (int g = 0; g < net.n_neurons; ++g)
            if (play[g] && !sens[g]) { ++in_play; if (!fired[g]) ++silent; }
        std::string out;
        size_t off = 0;
        char buf[32];
        for (int k = 0; k <= net.hops; ++k) {
            const int rows = net.sizes[k];
            double c = 0;
            for (int t = 0; t < rows; ++t) c += s.cnt[off + t];
            snprintf(buf, sizeof buf, " %.3f", c / (rows * s.samples));
            out += buf;
            off += rows;
        }
        return out;
    }
    // the running average (what would be installed) and the raw weights on --eval-batches batches of one chunk
    void eval(const ChunkP& c, uint64_t seed, const char* what) {
        if (a.eval_batches <= 0) return;
        const std::vector<ChunkP> one{c};
        const Surv ev = survey(1, one, a.eval_batches, seed), raw = survey(0, one, a.eval_batches, seed);
        int silent = 0, in_play = 0;
        const std::string fl = firing_line(ev, silent, in_play);
        printf("eval step %lld | kl %.4f agree %.4f | raw kl %.4f agree %.4f | firing%s | silent %d of %d | %s %s\n",
               step, ev.kl, ev.agree, raw.kl, raw.agree, fl.c_str(), silent, in_play, c->name.c_str(), what);
        fflush(stdout);
    }
    // Silent neurons back to work with the network's output unchanged (the reference's revive(), flyguy_train.cu:
    // 479-551): every neuron past the sensory layer that fired for none of the surveyed samples gets its incoming
    // strengths' sizes with a random sign and one common factor that brings its input to `target` (rms, three
    // passes); gain 1 and threshold -4; its strengths onto live neurons and onto the actions become 0 - it sent
    // nothing before and sends nothing now, but it fires, so those can learn. The running average takes the new
    // values; Adam restarts for them at a typical scale.
    void revive(const std::vector<ChunkP>& src, uint64_t seed) {
        const Surv s0 = survey(0, src, a.revive_batches, seed);
        const int N = net.n_neurons, K = net.hops;
        std::vector<long long> fired;
        std::vector<char> play, sens, dead(N, 0);
        per_neuron(s0, fired, play, sens);
        int n_dead = 0, n_play = 0;
        for (int g = 0; g < N; ++g)
            if (play[g] && !sens[g]) { ++n_play; if (!fired[g]) { dead[g] = 1; ++n_dead; } }
        if (!n_dead) {
            printf("revive step %lld | no silent neuron among %d over %.0f samples\n", step, n_play, s0.samples);
            fflush(stdout);
            return;
        }
        auto P = from_core(h, 0, z);
        std::vector<float>&W = P[0], &gain = P[1], &theta = P[2], &ow = P[5];
        std::vector<char> mark(net.n_w, 0);            // 1: into a silent neuron (new sign); 2: from one into a live one
        std::mt19937_64 r(seed * 7919ULL + 17);
        long long n_in = 0, n_out = 0;
        for (int k = 0; k < K; ++k) {
            const auto& hh = net.hop[k];
            const std::vector<int>& below = k ? net.hop[k - 1].nid : net.n0;
            for (size_t t = 0; t < hh.nid.size(); ++t) {
                const bool dpost = dead[hh.nid[t]];
                for (int e = hh.crow[t]; e < hh.crow[t + 1]; ++e) {
                    const int wi = hh.widx[e];
                    if (mark[wi]) continue;
                    if (dpost) { W[wi] = std::max(fabsf(W[wi]), 1e-4f) * ((r() & 1) ? 1.f : -1.f); mark[wi] = 1; ++n_in; }
                    else if (dead[below[hh.col[e]]]) { W[wi] = 0.f; mark[wi] = 2; ++n_out; }
                }
            }
        }
        for (int g = 0; g < N; ++g) if (dead[g]) { gain[g] = 1.f; theta[g] = -4.f; }
        const auto& top = net.hop[K - 1];
        std::vector<char> dcol(net.n_dn, 0);
        int n_dn_dead = 0;
        for (int j = 0; j < net.n_dn; ++j)
            if (dead[top.nid[net.dn[j]]]) {
                dcol[j] = 1;
                ++n_dn_dead;
                for (int k2 = 0; k2 < net.n_act; ++k2) ow[(size_t)k2 * net.n_dn + j] = 0.f;
            }
        to_core(h, 0, P, z);
        for (int pass = 0; pass < 3; ++pass) {          // hop after hop the revived neurons' inputs come to the target
            const Surv s = survey(0, src, a.revive_batches, seed);
            std::vector<float> rms(N, 0.f);
            size_t off = net.n_s;
            for (auto& hh : net.hop) {
                for (size_t t = 0; t < hh.nid.size(); ++t)
                    rms[hh.nid[t]] = std::max(rms[hh.nid[t]], (float)std::sqrt(s.sq[off + t] / s.samples));
                off += hh.nid.size();
            }
            std::vector<char> done(net.n_w, 0);
            for (auto& hh : net.hop)
                for (size_t t = 0; t < hh.nid.size(); ++t) {
                    const int g = hh.nid[t];
                    if (!dead[g] || rms[g] <= 0.f) continue;
                    const float sc = std::min(200.f, std::max(0.02f, a.revive_target / rms[g]));
                    for (int e = hh.crow[t]; e < hh.crow[t + 1]; ++e) {
                        const int wi = hh.widx[e];
                        if (!done[wi]) { W[wi] *= sc; done[wi] = 1; }
                    }
                }
            to_core(h, 0, P, z);
        }
        const Surv s1 = survey(0, src, a.revive_batches, seed);
        per_neuron(s1, fired, play, sens);
        int still = 0;
        for (int g = 0; g < N; ++g) if (dead[g] && !fired[g]) ++still;
        {   // the running average and Adam follow
            auto E = from_core(h, 1, z), M = from_core(h, 2, z), V = from_core(h, 3, z);
            const float fill = median_positive(V[0]);
            for (int i = 0; i < net.n_w; ++i) if (mark[i]) { E[0][i] = W[i]; M[0][i] = 0.f; V[0][i] = fill; }
            for (int p = 1; p <= 2; ++p) {
                const float f2 = median_positive(V[p]);
                for (int g = 0; g < N; ++g) if (dead[g]) { E[p][g] = p == 1 ? 1.f : -4.f; M[p][g] = 0.f; V[p][g] = f2; }
            }
            for (int j = 0; j < net.n_dn; ++j)
                if (dcol[j])
                    for (int k2 = 0; k2 < net.n_act; ++k2) { E[5][(size_t)k2 * net.n_dn + j] = 0.f; M[5][(size_t)k2 * net.n_dn + j] = 0.f; }
            to_core(h, 1, E, z);
            to_core(h, 2, M, z);
            to_core(h, 3, V, z);
        }
        printf("revive step %lld | %d of %d neurons past the sensory layer silent over %.0f samples | new sign for %lld "
               "incoming strengths, zero for %lld outgoing and for %d descending neurons' action weights | %d still "
               "silent | kl %.5f -> %.5f (must be equal)\n",
               step, n_dead, n_play, s0.samples, n_in, n_out, n_dn_dead, still, s0.kl, s1.kl);
        fflush(stdout);
    }
    void save() {
        fc_sync(h);
        check(h);
        save_flyp(a.out + ".bin", step, from_core(h, 0, z));
        save_flyp(a.out + ".ema.bin", step, from_core(h, 1, z));
        const long long at = fc_adam_t(h, -1);
        save_flyo(a.out + ".opt.bin", step, at, from_core(h, 2, z), from_core(h, 3, z));
        printf("saved %s.bin, .ema.bin and .opt.bin at step %lld\n", a.out.c_str(), step);
        fflush(stdout);
    }

    int run() {
        h = fg_create(a.net.c_str(), a.B, 0);
        if (!h) throw TrainErr{fg_last_error(nullptr)};
        z = sizes_of(h);
        // a restart from this run's own save keeps the running average and the optimiser state
        const bool own = fs::path(a.params).lexically_normal() == fs::path(a.out + ".bin").lexically_normal();
        std::vector<std::vector<float>> P, E, M, V;
        if (!read_flyp(a.params, z, step, P)) throw TrainErr{"cannot read " + a.params + " (FLYP of this network)"};
        long long st_ema = 0;
        if (!(own && read_flyp(a.out + ".ema.bin", z, st_ema, E))) E = P;
        to_core(h, 0, P, z);
        to_core(h, 1, E, z);
        long long adam_t = 0;
        const bool opt = own && read_flyo(a.out + ".opt.bin", z, step, adam_t, M, V);
        if (opt) {
            to_core(h, 2, M, z);
            to_core(h, 3, V, z);
        }
        fc_adam_t(h, adam_t);
        check(h);
        TCK(cudaMalloc(&obs, (size_t)a.B * z.obs_dim * 4));
        TCK(cudaMalloc(&teacher, (size_t)a.B * z.n_act * 4));
        net = read_netinfo(a.net);
        R = 0;
        for (int v : net.sizes) R += v;
        TCK(cudaMalloc(&d_fired, (size_t)R * 4));
        TCK(cudaMalloc(&d_sq, (size_t)R * 4));
        printf("flyguy_b200 trainer: batch %d, lr %g (neurons %g, plugs %g), teacher temperature %g, ring of %d "
               "chunks, start step %lld%s\n",
               a.B, a.lr, a.lr_neuron, a.lr_plug, a.temp, a.ring, step, opt ? ", optimiser state restored" : "");
        fflush(stdout);
        for (;;) {
            auto got = scan();
            for (auto& c : got) into_ring(c);
            if (!ring.empty()) break;
            printf("waiting for data in %s\n", a.data.c_str());
            fflush(stdout);
            std::this_thread::sleep_for(std::chrono::seconds(5));
        }
        eval(ring.back(), 4242, "at the start");
        const double max_reuse = a.max_reuse < 0 ? (a.max_steps ? 0 : 4) : a.max_reuse;
        auto ring_total = [&]() { double s = 0; for (auto& c : ring) s += (double)c->n; return s; };
        double allow = max_reuse * ring_total();
        double t_log = now(), t_save = now(), kl = 0, ag = 0;
        long long last_revive = a.revive_first ? step - a.revive_every : step;
        long long since = 0;
        const float it = 1.f / a.temp;
        const std::string stop = a.out + ".STOP";
        while (!a.max_steps || ran < a.max_steps) {
            if (since == 0 || ran % a.log_every == 0) {
                for (auto& c : scan()) {                      // a new chunk: scored, then into the ring
                    eval(c, 1000003ULL * (uint64_t)step + 7, "unseen");
                    into_ring(c);
                    allow = std::min(allow + max_reuse * (double)c->n, max_reuse * ring_total());
                }
            }
            if (max_reuse > 0 && allow < a.B) {
                printf("step %lld | waiting for new data: every sample of the ring has been drawn %.0f times\n", step,
                       max_reuse);
                fflush(stdout);
                if (fs::exists(stop)) break;
                std::this_thread::sleep_for(std::chrono::seconds(1));
                since = 0;
                continue;
            }
            allow -= a.B;
            if (a.revive_every > 0 && step - last_revive >= a.revive_every) {
                revive(ring, 99991ULL * (uint64_t)step + 3);
                last_revive = step;
            }
            draw(ring_dev(), a.seed, step);                   // queued before the step on the same stream
            fc_zero_grad(h);                                  // each step's gradient is its batch's alone
            double s[2];
            if (fg_teach_ex(h, obs, teacher, a.B, it, (float)a.B, nullptr, s)) check(h);
            ++step; ++ran; ++since;
            kl += s[0];
            ag += s[1];
            const float sched = (float)std::pow(0.5, (double)step / a.half_life);
            auto rate = [&](float base) { return std::max(a.lr_min * base / a.lr, base * sched); };
            fc_step(h, rate(a.lr), rate(a.lr_neuron), rate(a.lr_plug), a.clip, a.ema);
            check(h);
            if (since >= a.log_every) {
                const double t = now();
                printf("step %lld | %.0f samples/s | kl %.4f agree %.4f | lr %.2e | ring %d, newest %s\n", step,
                       since * (double)a.B / (t - t_log), kl / ((double)a.B * since), ag / ((double)a.B * since),
                       std::max(a.lr_min, a.lr * sched), (int)ring.size(), ring.back()->name.c_str());
                fflush(stdout);
                t_log = t;
                since = 0;
                kl = ag = 0;
            }
            const bool stopping = fs::exists(stop);
            if (stopping || now() - t_save > a.save_sec) {
                save();
                t_save = now();
                if (stopping) break;
            }
        }
        save();
        if (fs::exists(stop)) {
            std::error_code ec;
            fs::rename(stop, stop + ".done", ec);
            printf("stopped on request at step %lld\n", step);
        } else {
            printf("done at step %lld\n", step);
        }
        fflush(stdout);
        return 0;
    }
};

}  // namespace

extern "C" int fg_train_main(int argc, const char* const* argv) {
    try {
        Trainer t;
        t.a = parse(argc, argv);
        return t.run();
    } catch (const TrainErr& e) {
        fprintf(stderr, "fg_train: %s\n", e.msg.c_str());
    } catch (const std::exception& e) {
        fprintf(stderr, "fg_train: %s\n", e.what());
    }
    return 1;
}
