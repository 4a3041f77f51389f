// fg_train: the standalone teaching trainer, written against this library's own C-ABI (fg_create, fg_teach_ex,
// fc_step, fg_survey, fc_copy). It is the B200 counterpart of the reference's flyguy_train program
// (flyguy/native/flyguy_train.cu:631-788): the same command line, data chunks and checkpoint files, learning-rate
// schedule, evaluation lines, revival of silent neurons and --check mode.
//
//   fg_train NET.bin PARAMS.bin DATA_DIR OUT_PREFIX [options]
//   fg_train --check NET.bin PARAMS.bin BATCH.bin
//
// Options (defaults): --batch 512  --lr 3e-4  --lr-neuron 1e-4  --lr-plug 3e-4  --lr-min 3e-5  --half-life 20000
//   --ema 0.999  --clip 0  --temp 1  --log 100  --save-sec 120  --steps 0 (no end)  --ring 3  --max-reuse -1
//   --eval-batches 16  --eval-every 0  --holdout 0  --seed 12345  --revive-every 0  --revive-batches 4
//   --revive-target 0.4  --revive-first 0  (--passes N is accepted and ignored, as by the reference)
//
// How a run goes, piece by piece:
//   DataDir    DATA_DIR/chunk_*.bin in the FLYD layout (flyguy_train.cu:13-14: "FLYD", n int64, obs_dim int32,
//              n_act int32, n x obs_dim observations then n x n_act teacher logits, IEEE fp16) are picked up when
//              they appear or are rewritten, and kept on the GPU as fp16.
//   Ring       the newest --ring chunks; every step's batch is drawn from all their samples on the GPU: sample i of
//              step s is splitmix64(seed ^ (s << 32 | i)) modulo the ring's sample count, counted through the chunks
//              oldest first (counter-based, so Python can redraw any batch; the reference uses one sequential
//              mt19937_64 stream), unpacked straight into the step's fp32 inputs. --max-reuse R: each sample may be
//              drawn R times on average before the run waits for new data (default 4 for an open-ended run, off with
//              --steps). --holdout 1: the newest chunk present at the start is kept out of the ring and only scored.
//   Step       zero the gradient, fg_teach_ex (forward, KL(teacher at 1/T || student) averaged over the batch,
//              backward), fc_step with each group's rate max(lr_min x base / lr, base x 0.5^(step / half-life)) -
//              teach.py's recipe - and the weights' running average.
//   Census     fg_survey over --eval-batches batches of a chunk, through the running average and through the raw
//              weights: loss and agreement at temperature 1, each layer's firing share, the silent neurons. A new
//              chunk is scored before it joins the ring; --eval-every N scores the held-out chunk (or the ring's
//              newest) every N steps.
//   Revival    --revive-every N: silent neurons (past the sensory layer, firing for none of --revive-batches
//              batches) are brought back with the network's output unchanged (the reference's revive(),
//              flyguy_train.cu:479-551; see revive() below for the steps).
//   Files      OUT.bin and OUT.ema.bin (FLYP: "FLYP", step int64, the seven float32 arrays) and OUT.opt.bin (FLYO:
//              "FLYO", step, adam_t, then M and V of each array), written every --save-sec seconds, at the end, and
//              on OUT.STOP (renamed OUT.STOP.done). Started from its own OUT.bin a run continues with its running
//              average and optimiser state.
//   --check    NET.bin PARAMS.bin BATCH.bin ("FLYB", n int32, n x obs_dim observations, n x n_act teacher logits,
//              float32 - export.py batch): one forward and backward, printing the loss and agreement, the first
//              sample's first five logits and every array's gradient norm and sum (what export.py batch prints for
//              the reference's PyTorch path).
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
#include <string>
#include <thread>
#include <vector>

#include "flyguy_b200.h"

namespace {

namespace fs = std::filesystem;

struct Fail {
    std::string msg;
};
#define TCK(call)                                                                                   \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess) throw Fail{std::string(#call) + ": " + cudaGetErrorString(e_)};      \
    } while (0)

__host__ __device__ inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

double seconds() { return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count(); }

// ---------------------------------------------------------------- options
struct Options {
    std::string net, params, data, out;
    int batch = 512, log_every = 100, ring = 3, eval_batches = 16, revive_batches = 4, revive_first = 0, holdout = 0;
    long long steps = 0, revive_every = 0, eval_every = 0;
    double save_sec = 120, half_life = 20000, max_reuse = -1;
    float lr = 3e-4f, lr_neuron = 1e-4f, lr_plug = 3e-4f, lr_min = 3e-5f, ema = 0.999f, clip = 0.f, temp = 1.f;
    float revive_target = 0.4f;
    uint64_t seed = 12345;
};

Options parse(int argc, const char* const* argv) {
    if (argc < 5) throw Fail{"usage: fg_train NET PARAMS DATA_DIR OUT_PREFIX [options] | --check NET PARAMS BATCH"};
    Options o;
    o.net = argv[1]; o.params = argv[2]; o.data = argv[3]; o.out = argv[4];
    struct Num { const char* name; double* d; float* f; int* i; long long* ll; };
    double seed_d = 0;                                       // (--seed is read as an unsigned 64-bit integer)
    const Num table[] = {
        {"--batch", nullptr, nullptr, &o.batch, nullptr}, {"--lr", nullptr, &o.lr, nullptr, nullptr},
        {"--lr-neuron", nullptr, &o.lr_neuron, nullptr, nullptr}, {"--lr-plug", nullptr, &o.lr_plug, nullptr, nullptr},
        {"--lr-min", nullptr, &o.lr_min, nullptr, nullptr}, {"--half-life", &o.half_life, nullptr, nullptr, nullptr},
        {"--ema", nullptr, &o.ema, nullptr, nullptr}, {"--clip", nullptr, &o.clip, nullptr, nullptr},
        {"--temp", nullptr, &o.temp, nullptr, nullptr}, {"--log", nullptr, nullptr, &o.log_every, nullptr},
        {"--save-sec", &o.save_sec, nullptr, nullptr, nullptr}, {"--steps", nullptr, nullptr, nullptr, &o.steps},
        {"--ring", nullptr, nullptr, &o.ring, nullptr}, {"--max-reuse", &o.max_reuse, nullptr, nullptr, nullptr},
        {"--eval-batches", nullptr, nullptr, &o.eval_batches, nullptr},
        {"--eval-every", nullptr, nullptr, nullptr, &o.eval_every}, {"--holdout", nullptr, nullptr, &o.holdout, nullptr},
        {"--revive-every", nullptr, nullptr, nullptr, &o.revive_every},
        {"--revive-batches", nullptr, nullptr, &o.revive_batches, nullptr},
        {"--revive-target", nullptr, &o.revive_target, nullptr, nullptr},
        {"--revive-first", nullptr, nullptr, &o.revive_first, nullptr}, {"--seed", &seed_d, nullptr, nullptr, nullptr},
        {"--passes", nullptr, nullptr, nullptr, nullptr}};
    for (int i = 5; i < argc; i += 2) {
        const std::string k = argv[i];
        if (i + 1 >= argc) throw Fail{"option " + k + " needs a value"};
        const Num* hit = nullptr;
        for (const Num& t : table) if (k == t.name) hit = &t;
        if (!hit) throw Fail{"unknown option " + k};
        char* end = nullptr;
        const double v = strtod(argv[i + 1], &end);
        if (!end || *end) throw Fail{"option " + k + ": not a number: " + argv[i + 1]};
        if (k == "--seed") { o.seed = strtoull(argv[i + 1], nullptr, 10); continue; }
        if (hit->d) *hit->d = v;
        if (hit->f) *hit->f = (float)v;
        if (hit->i) *hit->i = (int)v;
        if (hit->ll) *hit->ll = (long long)v;
    }
    if (o.batch <= 0 || o.batch % 32) throw Fail{"--batch must be a positive multiple of 32"};
    if (!(o.temp > 0.f)) throw Fail{"--temp must be positive"};
    o.log_every = std::max(1, o.log_every);
    o.revive_batches = std::max(1, o.revive_batches);
    if (o.ring < 1 || o.ring > 16) throw Fail{"--ring must be between 1 and 16"};
    return o;
}

// ---------------------------------------------------------------- the network handle and its arrays
void ok(void* h) {
    if (fg_status(h)) throw Fail{fg_last_error(h)};
}

using Arrays = std::vector<std::vector<float>>;          // the seven arrays W, gain, theta, in_w, in_b, out_w, out_b

struct Net {
    void* h = nullptr;
    long long len[7] = {0};
    int obs_dim = 0, n_act = 0;
    ~Net() { if (h) fg_destroy(h); }
    void open(const std::string& path, int batch) {
        h = fg_create(path.c_str(), batch, 0);
        if (!h) throw Fail{fg_last_error(nullptr)};
        long long s[10];
        fc_sizes(h, s);
        ok(h);
        std::copy(s, s + 7, len);
        obs_dim = (int)s[7];
        n_act = (int)s[8];
    }
    // which: 0 weights, 1 running average, 2 m, 3 v, 4 gradient. The library copies device to device, so the arrays
    // pass through one device staging block.
    Arrays get(int which) const {
        long long total = 0;
        for (long long n : len) total += n;
        float* d = nullptr;
        TCK(cudaMalloc(&d, std::max<long long>(total, 1) * 4));
        float* p[7];
        for (long long i = 0, at = 0; i < 7; at += len[i], ++i) p[i] = d + at;
        fc_copy(h, which, 0, p);
        fc_sync(h);
        Arrays out(7);
        for (int i = 0; i < 7; ++i) {
            out[i].resize(len[i]);
            TCK(cudaMemcpy(out[i].data(), p[i], len[i] * 4, cudaMemcpyDeviceToHost));
        }
        cudaFree(d);
        ok(h);
        return out;
    }
    void put(int which, const Arrays& a) const {
        long long total = 0;
        for (long long n : len) total += n;
        float* d = nullptr;
        TCK(cudaMalloc(&d, std::max<long long>(total, 1) * 4));
        float* p[7];
        for (long long i = 0, at = 0; i < 7; at += len[i], ++i) {
            p[i] = d + at;
            if (a[i].size() != (size_t)len[i]) { cudaFree(d); throw Fail{"array of the wrong length"}; }
            TCK(cudaMemcpy(p[i], a[i].data(), len[i] * 4, cudaMemcpyHostToDevice));
        }
        fc_copy(h, which, 1, p);
        fc_sync(h);
        cudaFree(d);
        ok(h);
    }
};

// ---------------------------------------------------------------- checkpoint files (export.py's layouts)
struct FileIn {
    FILE* f = nullptr;
    explicit FileIn(const std::string& p) : f(fopen(p.c_str(), "rb")) {}
    ~FileIn() { if (f) fclose(f); }
    bool read(void* dst, size_t bytes) { return f && fread(dst, 1, bytes, f) == bytes; }
    bool tag(const char* magic) { char m[4]; return read(m, 4) && !memcmp(m, magic, 4); }
};

bool read_arrays(FileIn& in, const Net& net, Arrays& a) {
    a.assign(7, {});
    for (int i = 0; i < 7; ++i) {
        a[i].resize(net.len[i]);
        if (!in.read(a[i].data(), a[i].size() * 4)) return false;
    }
    return true;
}
bool load_flyp(const std::string& path, const Net& net, long long& step, Arrays& a) {
    FileIn in(path);
    return in.tag("FLYP") && in.read(&step, 8) && read_arrays(in, net, a);
}
bool load_flyo(const std::string& path, const Net& net, long long want_step, long long& adam_t, Arrays& m, Arrays& v) {
    FileIn in(path);
    long long step = -1;
    if (!(in.tag("FLYO") && in.read(&step, 8) && in.read(&adam_t, 8)) || step != want_step) return false;
    m.assign(7, {});
    v.assign(7, {});
    for (int i = 0; i < 7; ++i) {
        m[i].resize(net.len[i]);
        v[i].resize(net.len[i]);
        if (!in.read(m[i].data(), m[i].size() * 4) || !in.read(v[i].data(), v[i].size() * 4)) return false;
    }
    return true;
}
// written to PATH.tmp, then renamed over PATH, so a reader never sees half a file
void store(const std::string& path, const std::vector<std::pair<const void*, size_t>>& parts) {
    const std::string tmp = path + ".tmp";
    FILE* f = fopen(tmp.c_str(), "wb");
    if (!f) throw Fail{"cannot write " + tmp};
    size_t bad = 0;
    for (auto& p : parts) bad += fwrite(p.first, 1, p.second, f) != p.second;
    if (fclose(f) != 0 || bad) throw Fail{"writing " + tmp + " failed"};
    std::error_code ec;
    fs::rename(tmp, path, ec);
    if (ec) {                                             // (a platform that will not rename over a file)
        fs::remove(path, ec);
        fs::rename(tmp, path, ec);
        if (ec) throw Fail{"cannot rename " + tmp + " to " + path};
    }
}
void save_flyp(const std::string& path, long long step, const Arrays& a) {
    std::vector<std::pair<const void*, size_t>> parts{{"FLYP", 4}, {&step, 8}};
    for (auto& x : a) parts.push_back({x.data(), x.size() * 4});
    store(path, parts);
}
void save_flyo(const std::string& path, long long step, long long adam_t, const Arrays& m, const Arrays& v) {
    std::vector<std::pair<const void*, size_t>> parts{{"FLYO", 4}, {&step, 8}, {&adam_t, 8}};
    for (int i = 0; i < 7; ++i) {
        parts.push_back({m[i].data(), m[i].size() * 4});
        parts.push_back({v[i].data(), v[i].size() * 4});
    }
    store(path, parts);
}

// ---------------------------------------------------------------- the wiring, as revival and the census need it
// NET.bin (export.py:9-16): per hop the rows' neuron ids and connections (CSR by row, weight index per connection),
// the sensory neuron ids, the descending rows of the last layer
struct Wiring {
    int hops = 0, n_neurons = 0, n_w = 0, n_s = 0, n_dn = 0, n_act = 0;
    std::vector<int> sizes, n0, dn;
    struct Hop { std::vector<int> nid, row_ptr, src, widx; };
    std::vector<Hop> hop;
    int rows_total() const { int r = 0; for (int s : sizes) r += s; return r; }
};
Wiring read_wiring(const std::string& path) {
    FileIn in(path);
    auto ints = [&](long long n) {
        std::vector<int> v((size_t)std::max<long long>(n, 0));
        if (n > 0 && !in.read(v.data(), v.size() * 4)) throw Fail{"NET.bin too short: " + path};
        return v;
    };
    if (!in.tag("FLY1")) throw Fail{"not a NET.bin: " + path};
    const std::vector<int> hd = ints(8);     // obs_dim n_act hops n_neurons n_w n_s fan n_dn
    Wiring w;
    w.n_act = hd[1]; w.hops = hd[2]; w.n_neurons = hd[3]; w.n_w = hd[4]; w.n_s = hd[5]; w.n_dn = hd[7];
    w.sizes = ints(w.hops + 1);
    const std::vector<int> E = ints(w.hops);
    const long long e_in = (long long)w.n_s * hd[6];
    ints(w.n_s + 1); ints(e_in); ints(hd[0] + 1); ints(e_in); ints(e_in);      // the plug's five arrays
    w.n0 = ints(w.n_s);
    for (int k = 0; k < w.hops; ++k) {
        Wiring::Hop h;
        h.nid = ints(w.sizes[k + 1]);
        h.row_ptr = ints(w.sizes[k + 1] + 1);
        h.src = ints(E[k]);
        h.widx = ints(E[k]);
        ints(w.sizes[k] + 1); ints(E[k]); ints(E[k]); ints(w.sizes[k + 1]);       // by-source arrays, drive rows
        w.hop.push_back(std::move(h));
    }
    w.dn = ints(w.n_dn);
    return w;
}

// ---------------------------------------------------------------- data: chunks on the GPU, the ring, batch draws
constexpr int kMaxChunks = 17;                              // --ring (at most 16) plus one held-out chunk
struct ChunkTable {                                         // what the draw kernel sees
    const __half* obs[kMaxChunks];
    const __half* teacher[kMaxChunks];
    long long n[kMaxChunks];
    int count;
    long long total;
};

// rows b < B: sample u = splitmix64(seed ^ (counter << 32 | b)) mod total, located in the chunks in table order,
// written as fp32 obs [B, obs_dim] and teacher [B, n_act]; a warp per row
__global__ void k_draw(ChunkTable t, uint64_t seed, long long counter, int B, int obs_dim, int n_act,
                       float* __restrict__ obs, float* __restrict__ teacher) {
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= B || t.total <= 0) return;
    long long u = (long long)(splitmix64(seed ^ (((uint64_t)counter << 32) | (uint64_t)b)) % (uint64_t)t.total);
    int c = 0;
    while (c + 1 < t.count && u >= t.n[c]) u -= t.n[c++];
    const __half* o = t.obs[c] + (size_t)u * obs_dim;
    const __half* l = t.teacher[c] + (size_t)u * n_act;
    for (int i = lane; i < obs_dim; i += 32) obs[(size_t)b * obs_dim + i] = __half2float(o[i]);
    for (int i = lane; i < n_act; i += 32) teacher[(size_t)b * n_act + i] = __half2float(l[i]);
}

struct Chunk {
    std::string name;
    fs::file_time_type mtime{};
    long long n = 0;
    __half *obs = nullptr, *teacher = nullptr;
    ~Chunk() {
        if (obs) cudaFree(obs);
        if (teacher) cudaFree(teacher);
    }
};
using ChunkP = std::shared_ptr<Chunk>;

// a FLYD file of this network's sizes, on the GPU; nullptr while it is incomplete or of other sizes
ChunkP load_chunk(const fs::path& p, int obs_dim, int n_act) {
    FileIn in(p.string());
    long long n = 0;
    int dims[2] = {0, 0};
    if (!(in.tag("FLYD") && in.read(&n, 8) && in.read(dims, 8)) || dims[0] != obs_dim || dims[1] != n_act || n <= 0)
        return nullptr;
    std::vector<uint16_t> o((size_t)n * obs_dim), t((size_t)n * n_act);
    if (!in.read(o.data(), o.size() * 2) || !in.read(t.data(), t.size() * 2)) return nullptr;
    auto c = std::make_shared<Chunk>();
    c->name = p.filename().string();
    c->n = n;
    TCK(cudaMalloc(&c->obs, o.size() * 2));
    TCK(cudaMalloc(&c->teacher, t.size() * 2));
    TCK(cudaMemcpy(c->obs, o.data(), o.size() * 2, cudaMemcpyHostToDevice));
    TCK(cudaMemcpy(c->teacher, t.data(), t.size() * 2, cudaMemcpyHostToDevice));
    return c;
}

// DATA_DIR, looked at on request: chunk files that are new or rewritten since the last look, oldest first
struct DataDir {
    std::string dir;
    int obs_dim = 0, n_act = 0;
    std::map<std::string, fs::file_time_type> seen;
    std::vector<ChunkP> poll() {
        std::vector<std::pair<fs::file_time_type, fs::path>> fresh;
        std::error_code ec;
        for (const auto& e : fs::directory_iterator(dir, ec)) {
            const std::string name = e.path().filename().string();
            if (name.rfind("chunk_", 0) != 0 || e.path().extension() != ".bin") continue;
            std::error_code e2;
            const auto mt = fs::last_write_time(e.path(), e2);
            if (e2) continue;
            const auto it = seen.find(name);
            if (it == seen.end() || it->second != mt) fresh.emplace_back(mt, e.path());
        }
        std::sort(fresh.begin(), fresh.end());
        std::vector<ChunkP> out;
        for (const auto& [mt, path] : fresh) {
            ChunkP c = load_chunk(path, obs_dim, n_act);
            if (!c) continue;                                 // still being written: the next look takes it
            c->mtime = mt;
            seen[c->name] = mt;
            out.push_back(c);
        }
        return out;
    }
};

// chunks in time order (oldest first), at most `cap` of them
struct Ring {
    int cap = 3;
    std::vector<ChunkP> chunks;
    void add(const ChunkP& c) {
        chunks.erase(std::remove_if(chunks.begin(), chunks.end(), [&](const ChunkP& x) { return x->name == c->name; }),
                     chunks.end());
        const auto at = std::upper_bound(chunks.begin(), chunks.end(), c, [](const ChunkP& a, const ChunkP& b) {
            return a->mtime != b->mtime ? a->mtime < b->mtime : a->name < b->name;
        });
        chunks.insert(at, c);
        if ((int)chunks.size() > cap) chunks.erase(chunks.begin(), chunks.end() - cap);
    }
    long long samples() const { long long s = 0; for (auto& c : chunks) s += c->n; return s; }
};
ChunkTable table_of(const std::vector<ChunkP>& cs) {
    ChunkTable t{};
    t.count = (int)std::min<size_t>(cs.size(), kMaxChunks);
    for (int i = 0; i < t.count; ++i) {
        t.obs[i] = cs[i]->obs;
        t.teacher[i] = cs[i]->teacher;
        t.n[i] = cs[i]->n;
        t.total += cs[i]->n;
    }
    return t;
}

// ---------------------------------------------------------------- census: fg_survey over a chunk, summed per neuron
struct Census {
    std::vector<int> fired;                  // per row of every layer: samples with a positive state
    std::vector<float> sq;                   // per row: summed squared pre-activation
    double kl = 0, agree = 0, samples = 0;   // per sample, at temperature 1
};

struct Trainer {
    Options o;
    Net net;
    Wiring wiring;
    DataDir data;
    Ring ring;
    ChunkP held;                                              // --holdout: scored, never learned from
    float *obs = nullptr, *teacher = nullptr;
    int* d_fired = nullptr;
    float* d_sq = nullptr;
    long long step = 0, ran = 0;

    ~Trainer() {
        cudaFree(obs); cudaFree(teacher); cudaFree(d_fired); cudaFree(d_sq);
    }
    void draw(const ChunkTable& t, uint64_t seed, long long counter) {
        k_draw<<<(o.batch + 7) / 8, 256>>>(t, seed, counter, o.batch, net.obs_dim, net.n_act, obs, teacher);
        TCK(cudaGetLastError());
    }
    // `batches` batches of `src` (the same samples for the same seed) through the weights (ema 0) or their running
    // average (ema 1), nothing learned
    Census census(int ema, const std::vector<ChunkP>& src, int batches, uint64_t seed) {
        const int R = wiring.rows_total();
        TCK(cudaMemset(d_fired, 0, (size_t)R * 4));
        TCK(cudaMemset(d_sq, 0, (size_t)R * 4));
        const ChunkTable t = table_of(src);
        Census c;
        for (int i = 0; i < batches; ++i) {
            draw(t, seed, i);
            double st[2] = {0, 0};
            if (fg_survey(net.h, obs, teacher, o.batch, ema, d_fired, d_sq, st)) ok(net.h);
            c.kl += st[0];
            c.agree += st[1];
        }
        c.fired.resize(R);
        c.sq.resize(R);
        TCK(cudaMemcpy(c.fired.data(), d_fired, (size_t)R * 4, cudaMemcpyDeviceToHost));
        TCK(cudaMemcpy(c.sq.data(), d_sq, (size_t)R * 4, cudaMemcpyDeviceToHost));
        c.samples = (double)o.batch * batches;
        c.kl /= c.samples;
        c.agree /= c.samples;
        return c;
    }
    // neurons that sit in a layer past the sensory one and are not sensory, and how often each fired (summed over
    // all its rows)
    void per_neuron(const Census& c, std::vector<char>& hidden, std::vector<long long>& fired) const {
        hidden.assign(wiring.n_neurons, 0);
        fired.assign(wiring.n_neurons, 0);
        size_t row = wiring.n_s;
        for (const auto& h : wiring.hop)
            for (int id : h.nid) { hidden[id] = 1; fired[id] += c.fired[row++]; }
        for (int id : wiring.n0) hidden[id] = 0;
    }
    void score(const ChunkP& c, uint64_t seed, const char* why) {
        if (o.eval_batches <= 0) return;
        const std::vector<ChunkP> one{c};
        const Census avg = census(1, one, o.eval_batches, seed), raw = census(0, one, o.eval_batches, seed);
        std::vector<char> hidden;
        std::vector<long long> fired;
        per_neuron(avg, hidden, fired);
        int silent = 0, n_hidden = 0;
        for (int g = 0; g < wiring.n_neurons; ++g)
            if (hidden[g]) { ++n_hidden; silent += fired[g] == 0; }
        std::string shares;
        size_t row = 0;
        for (int s : wiring.sizes) {
            long long f = 0;
            for (int t = 0; t < s; ++t) f += avg.fired[row++];
            char b[24];
            snprintf(b, sizeof b, "%s%.3f", shares.empty() ? "" : "/", s ? f / (s * avg.samples) : 0.0);
            shares += b;
        }
        printf("eval @%lld %s (%s) | average: kl %.4f agree %.4f | weights: kl %.4f agree %.4f | firing %s | "
               "silent %d/%d\n", step, c->name.c_str(), why, avg.kl, avg.agree, raw.kl, raw.agree, shares.c_str(),
               silent, n_hidden);
        fflush(stdout);
    }
    static float median_of_positive(const std::vector<float>& v) {
        std::vector<float> p;
        for (float x : v) if (x > 0.f) p.push_back(x);
        if (p.empty()) return 0.f;
        std::nth_element(p.begin(), p.begin() + p.size() / 2, p.end());
        return p[p.size() / 2];
    }
    // Revival of silent neurons with the network's output unchanged (the reference's revive(), flyguy_train.cu:
    // 479-551). A rectifying neuron whose input never turns positive passes no gradient, so it and its connections
    // never learn. For every neuron past the sensory layer that fired for none of the surveyed samples:
    //   1. each connection INTO it keeps its size (at least 1e-4) with a random sign - bit 0 of splitmix64(seed ^
    //      weight index), so the draw depends only on the weight - and each connection FROM it into a neuron that
    //      fires becomes 0; its gain and threshold parameter go back to 1 and -4; its action weights (if it is a
    //      descending neuron) become 0. It sent nothing before and sends nothing now, so the output is the same
    //      (the loss before and after is printed, and must be equal); but it fires, so all of those can learn.
    //   2. three times: a census, then each revived neuron's incoming strengths are scaled by one common factor
    //      clamp(target / rms input, 0.02, 200), so hop after hop their inputs come to the target size.
    //   3. the running average takes the new values; Adam's m restarts at 0 and v at the median positive v of the
    //      array for every changed strength, gain and threshold; the zeroed action weights' average and m become 0.
    void revive(uint64_t seed) {
        const Census before = census(0, ring.chunks, o.revive_batches, seed);
        std::vector<char> hidden;
        std::vector<long long> fired;
        per_neuron(before, hidden, fired);
        std::vector<char> silent(wiring.n_neurons, 0);
        int n_silent = 0, n_hidden = 0;
        for (int g = 0; g < wiring.n_neurons; ++g)
            if (hidden[g]) { ++n_hidden; if (!fired[g]) { silent[g] = 1; ++n_silent; } }
        if (!n_silent) {
            printf("revival @%lld: no silent neuron among %d past the sensory layer (%.0f samples)\n", step, n_hidden,
                   before.samples);
            fflush(stdout);
            return;
        }
        Arrays P = net.get(0);
        std::vector<char> touched(wiring.n_w, 0);            // 1: new sign (into a silent neuron), 2: zeroed
        long long n_in = 0, n_out = 0;
        for (int k = 0; k < wiring.hops; ++k) {
            const auto& h = wiring.hop[k];
            const std::vector<int>& below = k ? wiring.hop[k - 1].nid : wiring.n0;
            for (size_t t = 0; t < h.nid.size(); ++t)
                for (int e = h.row_ptr[t]; e < h.row_ptr[t + 1]; ++e) {
                    const int w = h.widx[e];
                    if (touched[w]) continue;
                    if (silent[h.nid[t]]) {
                        const float mag = std::max(std::fabs(P[0][w]), 1e-4f);
                        P[0][w] = (splitmix64(seed ^ (uint64_t)w) & 1u) ? mag : -mag;
                        touched[w] = 1;
                        ++n_in;
                    } else if (silent[below[h.src[e]]]) {
                        P[0][w] = 0.f;
                        touched[w] = 2;
                        ++n_out;
                    }
                }
        }
        for (int g = 0; g < wiring.n_neurons; ++g)
            if (silent[g]) { P[1][g] = 1.f; P[2][g] = -4.f; }
        const auto& top = wiring.hop.back();
        std::vector<char> dead_col(wiring.n_dn, 0);
        int n_cols = 0;
        for (int j = 0; j < wiring.n_dn; ++j)
            if (silent[top.nid[wiring.dn[j]]]) {
                dead_col[j] = 1;
                ++n_cols;
                for (int a = 0; a < wiring.n_act; ++a) P[5][(size_t)a * wiring.n_dn + j] = 0.f;
            }
        net.put(0, P);
        for (int pass = 0; pass < 3; ++pass) {
            const Census c = census(0, ring.chunks, o.revive_batches, seed);
            std::vector<float> rms(wiring.n_neurons, 0.f);
            size_t row = wiring.n_s;
            for (const auto& h : wiring.hop)
                for (int id : h.nid) { rms[id] = std::max(rms[id], (float)std::sqrt(c.sq[row] / c.samples)); ++row; }
            std::vector<char> scaled(wiring.n_w, 0);
            for (const auto& h : wiring.hop)
                for (size_t t = 0; t < h.nid.size(); ++t) {
                    const int g = h.nid[t];
                    if (!silent[g] || rms[g] <= 0.f) continue;
                    const float f = std::min(200.f, std::max(0.02f, o.revive_target / rms[g]));
                    for (int e = h.row_ptr[t]; e < h.row_ptr[t + 1]; ++e)
                        if (!scaled[h.widx[e]]) { P[0][h.widx[e]] *= f; scaled[h.widx[e]] = 1; }
                }
            net.put(0, P);
        }
        const Census after = census(0, ring.chunks, o.revive_batches, seed);
        per_neuron(after, hidden, fired);
        int still = 0;
        for (int g = 0; g < wiring.n_neurons; ++g) still += silent[g] && !fired[g];
        Arrays E = net.get(1), M = net.get(2), V = net.get(3);
        const float v_w = median_of_positive(V[0]);
        for (int w = 0; w < wiring.n_w; ++w)
            if (touched[w]) { E[0][w] = P[0][w]; M[0][w] = 0.f; V[0][w] = v_w; }
        for (int i = 1; i <= 2; ++i) {
            const float v_i = median_of_positive(V[i]);
            for (int g = 0; g < wiring.n_neurons; ++g)
                if (silent[g]) { E[i][g] = P[i][g]; M[i][g] = 0.f; V[i][g] = v_i; }
        }
        for (int j = 0; j < wiring.n_dn; ++j)
            if (dead_col[j])
                for (int a = 0; a < wiring.n_act; ++a) { E[5][(size_t)a * wiring.n_dn + j] = 0.f; M[5][(size_t)a * wiring.n_dn + j] = 0.f; }
        net.put(1, E);
        net.put(2, M);
        net.put(3, V);
        printf("revival @%lld: %d silent of %d past the sensory layer (%.0f samples); signs redrawn for %lld incoming "
               "strengths, %lld outgoing and %d action columns zeroed; still silent %d; kl %.5f -> %.5f\n",
               step, n_silent, n_hidden, before.samples, n_in, n_out, n_cols, still, before.kl, after.kl);
        fflush(stdout);
    }
    void save() {
        fc_sync(net.h);
        ok(net.h);
        save_flyp(o.out + ".bin", step, net.get(0));
        save_flyp(o.out + ".ema.bin", step, net.get(1));
        save_flyo(o.out + ".opt.bin", step, fc_adam_t(net.h, -1), net.get(2), net.get(3));
        printf("saved %s.bin, .ema.bin, .opt.bin @%lld\n", o.out.c_str(), step);
        fflush(stdout);
    }
    // each group's rate this step: the schedule factor rounded to float first, the product in float (teach.py's
    // arithmetic, so a run driven from Python with the same numbers takes the same steps)
    float rate(float base) const {
        const float sched = (float)std::pow(0.5, (double)step / o.half_life);
        const float floor = o.lr > 0.f ? o.lr_min * base / o.lr : 0.f;
        return std::max(floor, base * sched);
    }

    int run() {
        net.open(o.net, o.batch);
        wiring = read_wiring(o.net);
        Arrays P, E, M, V;
        if (!load_flyp(o.params, net, step, P)) throw Fail{"cannot read " + o.params + " as FLYP weights of this network"};
        // from this run's own OUT.bin: its running average and optimiser state come back too
        const bool own = fs::weakly_canonical(o.params) == fs::weakly_canonical(o.out + ".bin");
        long long ema_step = 0, adam_t = 0;
        if (!(own && load_flyp(o.out + ".ema.bin", net, ema_step, E))) E = P;
        const bool resumed = own && load_flyo(o.out + ".opt.bin", net, step, adam_t, M, V);
        net.put(0, P);
        net.put(1, E);
        if (resumed) { net.put(2, M); net.put(3, V); }
        fc_adam_t(net.h, adam_t);
        ok(net.h);
        TCK(cudaMalloc(&obs, (size_t)o.batch * net.obs_dim * 4));
        TCK(cudaMalloc(&teacher, (size_t)o.batch * net.n_act * 4));
        TCK(cudaMalloc(&d_fired, (size_t)wiring.rows_total() * 4));
        TCK(cudaMalloc(&d_sq, (size_t)wiring.rows_total() * 4));
        data.dir = o.data; data.obs_dim = net.obs_dim; data.n_act = net.n_act;
        ring.cap = o.ring;
        printf("fg_train: layers");
        for (int s : wiring.sizes) printf(" %d", s);
        printf(", batch %d, rates %g / %g / %g (floor %g, half-life %g), temperature %g, ring %d, from step %lld%s\n",
               o.batch, o.lr, o.lr_neuron, o.lr_plug, o.lr_min, o.half_life, o.temp, o.ring, step,
               resumed ? " with its optimiser state" : "");
        fflush(stdout);
        std::vector<ChunkP> first;
        while ((first = data.poll()).empty()) {
            printf("waiting for data in %s\n", o.data.c_str());
            fflush(stdout);
            std::this_thread::sleep_for(std::chrono::seconds(5));
        }
        if (o.holdout && first.size() > 1) {
            held = first.back();
            first.pop_back();
        }
        for (auto& c : first) ring.add(c);
        const uint64_t eval_seed = o.seed + 1;              // the same samples of a chunk at every evaluation
        if (held) score(held, eval_seed, "held out");
        else score(ring.chunks.back(), eval_seed, "at the start");
        const double reuse = o.max_reuse < 0 ? (o.steps ? 0.0 : 4.0) : o.max_reuse;
        double budget = reuse * (double)ring.samples();       // draws left before the run waits for new data
        long long revived_at = o.revive_first ? step - o.revive_every : step;
        double t_line = seconds(), t_saved = seconds(), kl = 0, agree = 0;
        long long in_line = 0;
        bool waiting = false;
        const std::string stop_file = o.out + ".STOP";
        const float inv_temp = 1.f / o.temp;
        int rc = 0;
        while (!o.steps || ran < o.steps) {
            if (waiting || in_line == 0 || ran % o.log_every == 0) {
                for (auto& c : data.poll()) {                    // new data: scored first, then learned from
                    score(c, o.seed + 2 + (uint64_t)step, "unseen");
                    ring.add(c);
                    budget = std::min(budget + reuse * (double)c->n, reuse * (double)ring.samples());
                }
            }
            if (reuse > 0 && budget < o.batch) {
                if (!waiting) {
                    printf("@%lld every sample of the ring has been drawn %g times: waiting for new data\n", step, reuse);
                    fflush(stdout);
                    waiting = true;
                }
                if (fs::exists(stop_file)) break;
                std::this_thread::sleep_for(std::chrono::seconds(1));
                t_line = seconds();
                in_line = 0;
                continue;
            }
            waiting = false;
            budget -= o.batch;
            if (o.revive_every > 0 && step - revived_at >= o.revive_every) {
                revive(o.seed + 3 + (uint64_t)step);
                revived_at = step;
            }
            draw(table_of(ring.chunks), o.seed, step);       // queued ahead of the step on the same stream
            fc_zero_grad(net.h);
            double st[2] = {0, 0};
            if (fg_teach_ex(net.h, obs, teacher, o.batch, inv_temp, (float)o.batch, nullptr, st)) ok(net.h);
            ++step; ++ran; ++in_line;
            kl += st[0];
            agree += st[1];
            fc_step(net.h, rate(o.lr), rate(o.lr_neuron), rate(o.lr_plug), o.clip, o.ema);
            ok(net.h);
            if (in_line >= o.log_every) {
                const double t = seconds();
                printf("step %lld | kl %.4f agree %.4f | lr %.2e | %.0f samples/s | ring %zu, newest %s\n", step,
                       kl / ((double)o.batch * in_line), agree / ((double)o.batch * in_line), rate(o.lr),
                       in_line * (double)o.batch / (t - t_line), ring.chunks.size(), ring.chunks.back()->name.c_str());
                fflush(stdout);
                t_line = t;
                in_line = 0;
                kl = agree = 0;
            }
            if (o.eval_every > 0 && step % o.eval_every == 0)
                score(held ? held : ring.chunks.back(), eval_seed, held ? "held out" : "newest in the ring");
            const bool stop = fs::exists(stop_file);
            if (stop || seconds() - t_saved > o.save_sec) {
                save();
                t_saved = seconds();
                if (stop) break;
            }
        }
        save();
        if (fs::exists(stop_file)) {
            std::error_code ec;
            fs::rename(stop_file, stop_file + ".done", ec);
            printf("stopped on request @%lld\n", step);
        } else {
            printf("finished @%lld\n", step);
        }
        fflush(stdout);
        return rc;
    }
};

// ---------------------------------------------------------------- --check
int check(const std::string& net_path, const std::string& params, const std::string& batch_path) {
    FileIn in(batch_path);
    int n = 0;
    if (!(in.tag("FLYB") && in.read(&n, 4)) || n <= 0) throw Fail{batch_path + " is not a FLYB batch"};
    const int B = (n + 31) / 32 * 32;                        // the library's batches are multiples of 32
    Net net;
    net.open(net_path, B);
    std::vector<float> x((size_t)n * net.obs_dim), t((size_t)n * net.n_act);
    if (!in.read(x.data(), x.size() * 4) || !in.read(t.data(), t.size() * 4)) throw Fail{batch_path + " is too short"};
    long long step = 0;
    Arrays P;
    if (!load_flyp(params, net, step, P)) throw Fail{"cannot read " + params + " as FLYP weights of this network"};
    net.put(0, P);
    net.put(1, P);
    const std::vector<float> last(x.end() - net.obs_dim, x.end());
    for (int r = n; r < B; ++r) x.insert(x.end(), last.begin(), last.end());   // padding: their loss gradient is 0
    float *d_x = nullptr, *d_lg = nullptr, *d_dl = nullptr;
    TCK(cudaMalloc(&d_x, x.size() * 4));
    TCK(cudaMalloc(&d_lg, (size_t)B * net.n_act * 4));
    TCK(cudaMalloc(&d_dl, (size_t)B * net.n_act * 4));
    TCK(cudaMemcpy(d_x, x.data(), x.size() * 4, cudaMemcpyHostToDevice));
    fc_forward(net.h, d_x, B, d_lg, 0);
    fc_sync(net.h);
    ok(net.h);
    std::vector<float> lg((size_t)B * net.n_act), dl((size_t)B * net.n_act, 0.f);
    TCK(cudaMemcpy(lg.data(), d_lg, lg.size() * 4, cudaMemcpyDeviceToHost));
    // KL(softmax(teacher) || softmax(logits)) per sample, averaged over the n real samples, and its gradient
    double kl = 0, agree = 0;
    const int A = net.n_act;
    for (int b = 0; b < n; ++b) {
        const float *s = &lg[(size_t)b * A], *q = &t[(size_t)b * A];
        const int as = (int)(std::max_element(s, s + A) - s), at = (int)(std::max_element(q, q + A) - q);
        const double ms = s[as], mt = q[at];
        double zs = 0, zt = 0;
        for (int a = 0; a < A; ++a) { zs += std::exp(s[a] - ms); zt += std::exp(q[a] - mt); }
        for (int a = 0; a < A; ++a) {
            const double lps = s[a] - ms - std::log(zs), lpt = q[a] - mt - std::log(zt), pt = std::exp(lpt);
            kl += pt * (lpt - lps);
            dl[(size_t)b * A + a] = (float)((std::exp(lps) - pt) / n);
        }
        agree += as == at;
    }
    TCK(cudaMemcpy(d_dl, dl.data(), dl.size() * 4, cudaMemcpyHostToDevice));
    fc_zero_grad(net.h);
    fc_backward(net.h, d_dl, B);
    fc_sync(net.h);
    ok(net.h);
    const Arrays G = net.get(4);
    printf("fg_train --check: %d samples | loss %.6f agree %.4f\n   logits[0][:5]", n, kl / n, agree / n);
    for (int a = 0; a < std::min(5, A); ++a) printf(" %.6f", lg[a]);
    printf("\n");
    const char* names[7] = {"W", "gain", "theta", "in_w", "in_b", "out_w", "out_b"};
    for (int i = 0; i < 7; ++i) {
        double ss = 0, sum = 0;
        for (float v : G[i]) { ss += (double)v * v; sum += v; }
        printf("   grad %-6s norm %.6e sum %+.6e\n", names[i], std::sqrt(ss), sum);
    }
    fflush(stdout);
    cudaFree(d_x); cudaFree(d_lg); cudaFree(d_dl);
    return 0;
}

}  // namespace

extern "C" int fg_train_main(int argc, const char* const* argv) {
    try {
        if (argc >= 2 && !strcmp(argv[1], "--check")) {
            if (argc != 5) throw Fail{"usage: fg_train --check NET.bin PARAMS.bin BATCH.bin"};
            return check(argv[2], argv[3], argv[4]);
        }
        Trainer t;
        t.o = parse(argc, argv);
        return t.run();
    } catch (const Fail& e) {
        fprintf(stderr, "fg_train: %s\n", e.msg.c_str());
    } catch (const std::exception& e) {
        fprintf(stderr, "fg_train: %s\n", e.what());
    }
    return 1;
}
