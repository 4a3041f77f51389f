/* CPU ORACLE for the flyguy hop path - TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's arithmetic, used by tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg as the checker. The product (flyguy_b200/libflyguy_b200.so) never links or calls this file.
 *
 * What it restates (paths inside the reference project adventure-gpt/flyguy):
 *   forward   flyguy/fly.py:295-305 (plug, hops with sensory re-drive, relu(gain*z - softplus(theta)), out plug);
 *             the same math as flyguy/native/flyguy_train.cu:73-101 (k_plug, k_act0, k_hop, k_logits)
 *   loss      flyguy/native/flyguy_train.cu:104-123 (KL(teacher^(1/T) || student), dl = (softmax(s) - p_t) / B);
 *             flyguy/teach.py:151-153
 *   backward  flyguy/native/flyguy_train.cu:125-179, 339-359 (out plug, relu/gain/theta, per-edge weight
 *             gradient, transposed product, plug); torch autograd of flyguy/fly.py:286-305 computes the same
 *   adam      flyguy/native/flyguy_train.cu:194-203, 610-627 (fc_grad_norm, fc_step: betas 0.9/0.999, eps 1e-8
 *             outside the sqrt, bias corrections capped at t=100000, clipping, EMA of the weights)
 *
 * Sums are accumulated in double, one sample at a time, in CSR order; samples run in parallel (OpenMP) and the
 * backward keeps one double gradient buffer per thread, added in thread order (deterministic for a thread count).
 * Pinned against the reference's own outputs by tests/golden (fixtures written by tests/golden/make_golden.py
 * from the reference's FlyActor in this container).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
    int obs_dim, n_act, hops, n_neurons, n_w, n_s, fan, n_dn;
    const int* sizes;                       /* hops + 1 */
    const int* in_crow;                     /* n_s + 1 */
    const int* in_col;                      /* n_s * fan */
    const int* n0;                          /* n_s */
    const int* dn_rows;                     /* n_dn */
    const int* const* nid;                  /* per hop: rows */
    const int* const* crow;                 /* per hop: rows + 1 */
    const int* const* col;                  /* per hop: E */
    const int* const* widx;                 /* per hop: E */
    const int* const* drow;                 /* per hop: rows */
} fo_net;

/* 16-bit state emulation (fo_forward_q): the value a kernel stores for a state of the given format - the fp32 result
 * rounded to the 16-bit type, round to nearest even. qmode bits 0-1: 0 keep fp32, 1 bf16, 2 fp16; bit 4: the plug's
 * observation values are rounded to that type as well (a kernel that stages obs in the state type). */
enum { FO_Q_NONE = 0, FO_Q_BF16 = 1, FO_Q_F16 = 2, FO_Q_OBS = 16, FO_PRE = 32 };
static float q16(float f, int qmode) {
    switch (qmode & 3) {
        case FO_Q_BF16: {
            uint32_t u;
            memcpy(&u, &f, 4);
            if ((u & 0x7fffffffu) > 0x7f800000u) return f;                 /* NaN stays NaN */
            u += 0x7fffu + ((u >> 16) & 1u);
            u &= 0xffff0000u;
            memcpy(&f, &u, 4);
            return f;
        }
        case FO_Q_F16: return (float)(_Float16)f;
        default: return f;
    }
}

/* q16 over an array (so tests can pin the rounding against other implementations) */
void fo_round16(const float* in, float* out, long long n, int qmode) {
    for (long long i = 0; i < n; ++i) out[i] = q16(in[i], qmode);
}

static double softplus_d(double x) { return x > 20.0 ? x : log1p(exp(x)); }
static double sigmoid_d(double x) { return 1.0 / (1.0 + exp(-x)); }

static int max_rows(const fo_net* n) {
    int m = n->n_s;
    for (int k = 1; k <= n->hops; ++k) if (n->sizes[k] > m) m = n->sizes[k];
    return m;
}
static size_t total_rows(const fo_net* n) {
    size_t t = 0;
    for (int k = 0; k <= n->hops; ++k) t += (size_t)n->sizes[k];
    return t;
}

/* one sample forward; fills drive[n_s], h (all layers back to back: h0, h1, ..., hK) and z (layers 1..K back to
 * back); returns logits[n_act] */
static void fwd_one_q(const fo_net* n, const float* const* P, const float* x, double* drive, double* h, double* z,
                      float* lg, int qmode) {
    const float *W = P[0], *gain = P[1], *theta = P[2], *in_w = P[3], *in_b = P[4], *ow = P[5], *ob = P[6];
    for (int s = 0; s < n->n_s; ++s) {
        double acc = in_b[s];
        for (int e = n->in_crow[s]; e < n->in_crow[s + 1]; ++e) {
            const float xv = (qmode & FO_Q_OBS) ? q16(x[n->in_col[e]], qmode) : x[n->in_col[e]];
            acc += (double)in_w[e] * xv;
        }
        drive[s] = acc;
        int id = n->n0[s];
        double v = (double)gain[id] * acc - softplus_d(theta[id]);
        h[s] = v > 0.0 ? v : 0.0;
        if (qmode & 3) h[s] = q16((float)h[s], qmode);
    }
    size_t off_prev = 0, off = n->n_s, zoff = 0;
    for (int k = 0; k < n->hops; ++k) {
        int rows = n->sizes[k + 1];
        const int *crow = n->crow[k], *col = n->col[k], *widx = n->widx[k], *nid = n->nid[k], *drow = n->drow[k];
        const double* hp = h + off_prev;
        for (int t = 0; t < rows; ++t) {
            double acc = 0.0;
            for (int e = crow[t]; e < crow[t + 1]; ++e) acc += (double)W[widx[e]] * hp[col[e]];
            if (drow[t] >= 0) acc += drive[drow[t]];
            z[zoff + t] = acc;
            int id = nid[t];
            double v = (double)gain[id] * acc - softplus_d(theta[id]);
            h[off + t] = v > 0.0 ? v : 0.0;
            if ((qmode & 3) && k + 1 < n->hops) h[off + t] = q16((float)h[off + t], qmode);   /* last layer: fp32 */
        }
        off_prev = off; off += rows; zoff += rows;
    }
    const double* hK = h + off_prev;
    for (int a = 0; a < n->n_act; ++a) {
        double acc = ob[a];
        for (int j = 0; j < n->n_dn; ++j) acc += (double)ow[(size_t)a * n->n_dn + j] * hK[n->dn_rows[j]];
        lg[a] = (float)acc;
    }
}

static void fwd_one(const fo_net* n, const float* const* P, const float* x, double* drive, double* h, double* z,
                    float* lg) {
    fwd_one_q(n, P, x, drive, h, z, lg, FO_Q_NONE);
}

/* obs [B, obs_dim] -> logits [B, n_act]; layers (nullable): [B, n_s + sum rows] fp32 = h0, h1, ..., hK.
 * qmode: FO_Q_NONE (the reference's fp32 forward) or a 16-bit state emulation (q16 above): every layer but the last
 * rounded to the 16-bit type where it is stored, sums still in double. With FO_PRE, layers receives the
 * pre-activations instead of the states: the plug's drive for layer 0, z (sum over the edges + re-drive) for the hop
 * layers. */
int fo_forward_q(const fo_net* n, const float* const* P, const float* obs, int B, float* logits, float* layers,
                 int threads, int qmode) {
    size_t R = total_rows(n);
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
    int bad = 0;
#pragma omp parallel reduction(| : bad)
    {
        double* drive = malloc(sizeof(double) * (size_t)n->n_s);
        double* h = malloc(sizeof(double) * R);
        double* z = malloc(sizeof(double) * R);
        if (!drive || !h || !z) bad = 1;
        else {
#pragma omp for schedule(static)
            for (int b = 0; b < B; ++b) {
                fwd_one_q(n, P, obs + (size_t)b * n->obs_dim, drive, h, z, logits + (size_t)b * n->n_act, qmode);
                if (layers && (qmode & FO_PRE)) {
                    for (int i = 0; i < n->n_s; ++i) layers[(size_t)b * R + i] = (float)drive[i];
                    for (size_t i = (size_t)n->n_s; i < R; ++i) layers[(size_t)b * R + i] = (float)z[i - n->n_s];
                } else if (layers) {
                    for (size_t i = 0; i < R; ++i) layers[(size_t)b * R + i] = (float)h[i];
                }
            }
        }
        free(drive); free(h); free(z);
    }
    return bad ? -1 : 0;
}

int fo_forward(const fo_net* n, const float* const* P, const float* obs, int B, float* logits, float* layers,
               int threads) {
    return fo_forward_q(n, P, obs, B, logits, layers, threads, FO_Q_NONE);
}

/* KL(softmax(teacher * inv_temp) || softmax(logits)) summed over the batch (kl_sum), argmax agreements (agree),
 * and dl = (softmax(logits) - p_t) / B   [B, n_act] */
void fo_loss(const float* logits, const float* teacher, int B, int n_act, float inv_temp, float* dl, double* kl_sum,
             double* agree) {
    double kl_all = 0.0, ag = 0.0;
    for (int b = 0; b < B; ++b) {
        const float *s = logits + (size_t)b * n_act, *t = teacher + (size_t)b * n_act;
        double ms = -1e300, mt = -1e300;
        int as = 0, at = 0;
        for (int a = 0; a < n_act; ++a) {
            double tv = (double)t[a] * inv_temp;
            if (s[a] > ms) { ms = s[a]; as = a; }
            if (tv > mt) { mt = tv; at = a; }
        }
        double zs = 0.0, zt = 0.0;
        for (int a = 0; a < n_act; ++a) { zs += exp(s[a] - ms); zt += exp((double)t[a] * inv_temp - mt); }
        double ls = ms + log(zs), lt = mt + log(zt), kl = 0.0;
        for (int a = 0; a < n_act; ++a) {
            double lps = s[a] - ls, lpt = (double)t[a] * inv_temp - lt, pt = exp(lpt);
            kl += pt * (lpt - lps);
            dl[(size_t)b * n_act + a] = (float)((exp(lps) - pt) / B);
        }
        kl_all += kl;
        ag += as == at ? 1.0 : 0.0;
    }
    *kl_sum = kl_all;
    *agree = ag;
}

/* gradients of sum_b <dlogits[b], logits[b]> ADDED to G[7] (float) - what fc_backward does; obs [B, obs_dim],
 * dlogits [B, n_act] */
int fo_backward(const fo_net* n, const float* const* P, const float* obs, const float* dlogits, int B, float* const* G,
                int threads) {
    const float *W = P[0], *gain = P[1], *theta = P[2], *ow = P[5];
    size_t R = total_rows(n);
    size_t ps[7] = {(size_t)n->n_w, (size_t)n->n_neurons, (size_t)n->n_neurons, (size_t)n->n_s * n->fan,
                    (size_t)n->n_s, (size_t)n->n_act * n->n_dn, (size_t)n->n_act};
    size_t gtot = 0, goff[8];
    for (int i = 0; i < 7; ++i) { goff[i] = gtot; gtot += ps[i]; }
    goff[7] = gtot;
    int nthr = 1;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
    nthr = omp_get_max_threads();
#endif
    double** acc = calloc((size_t)nthr, sizeof(double*));
    if (!acc) return -1;
    int bad = 0;
    int mr = max_rows(n);
#pragma omp parallel reduction(| : bad)
    {
        int me = 0;
#ifdef _OPENMP
        me = omp_get_thread_num();
#endif
        double* g = calloc(gtot, sizeof(double));
        double* drive = malloc(sizeof(double) * (size_t)n->n_s);
        double* h = malloc(sizeof(double) * R);
        double* z = malloc(sizeof(double) * R);
        double* gh = malloc(sizeof(double) * R);
        double* gdrive = malloc(sizeof(double) * (size_t)n->n_s);
        float* lg = malloc(sizeof(float) * (size_t)n->n_act);
        acc[me] = g;
        if (!g || !drive || !h || !z || !gh || !gdrive || !lg) bad = 1;
        else {
            double *gW = g + goff[0], *ggain = g + goff[1], *gth = g + goff[2], *gin_w = g + goff[3],
                   *gin_b = g + goff[4], *gow = g + goff[5], *gob = g + goff[6];
            (void)mr;
#pragma omp for schedule(static)
            for (int b = 0; b < B; ++b) {
                const float* x = obs + (size_t)b * n->obs_dim;
                const float* dl = dlogits + (size_t)b * n->n_act;
                fwd_one(n, P, x, drive, h, z, lg);
                memset(gh, 0, sizeof(double) * R);
                memset(gdrive, 0, sizeof(double) * (size_t)n->n_s);
                /* layer offsets */
                size_t off[64], zoff[64];
                off[0] = 0;
                for (int k = 1; k <= n->hops; ++k) off[k] = off[k - 1] + (size_t)n->sizes[k - 1];
                zoff[1] = 0;
                for (int k = 2; k <= n->hops; ++k) zoff[k] = zoff[k - 1] + (size_t)n->sizes[k - 1];
                const double* hK = h + off[n->hops];
                double* ghK = gh + off[n->hops];
                for (int a = 0; a < n->n_act; ++a) {
                    double d = dl[a];
                    gob[a] += d;
                    for (int j = 0; j < n->n_dn; ++j) {
                        int r = n->dn_rows[j];
                        gow[(size_t)a * n->n_dn + j] += d * hK[r];
                        ghK[r] += (double)ow[(size_t)a * n->n_dn + j] * d;
                    }
                }
                for (int k = n->hops; k >= 1; --k) {
                    int rows = n->sizes[k];
                    const int *crow = n->crow[k - 1], *col = n->col[k - 1], *widx = n->widx[k - 1],
                              *nid = n->nid[k - 1], *drow = n->drow[k - 1];
                    const double *hk = h + off[k], *zk = z + zoff[k], *hp = h + off[k - 1];
                    const double* ghk = gh + off[k];
                    double* ghp = gh + off[k - 1];
                    for (int t = 0; t < rows; ++t) {
                        double gg = hk[t] > 0.0 ? ghk[t] : 0.0;
                        if (gg == 0.0) continue;
                        int id = nid[t];
                        double gz = gg * gain[id];
                        ggain[id] += gg * zk[t];
                        gth[id] += -gg * sigmoid_d(theta[id]);
                        if (drow[t] >= 0) gdrive[drow[t]] += gz;
                        for (int e = crow[t]; e < crow[t + 1]; ++e) {
                            gW[widx[e]] += gz * hp[col[e]];
                            ghp[col[e]] += (double)W[widx[e]] * gz;
                        }
                    }
                }
                for (int s = 0; s < n->n_s; ++s) {
                    double gg = h[s] > 0.0 ? gh[s] : 0.0;
                    int id = n->n0[s];
                    if (gg != 0.0) {
                        ggain[id] += gg * drive[s];
                        gth[id] += -gg * sigmoid_d(theta[id]);
                        gdrive[s] += gg * gain[id];
                    }
                    double gd = gdrive[s];
                    gin_b[s] += gd;
                    for (int e = n->in_crow[s]; e < n->in_crow[s + 1]; ++e) gin_w[e] += gd * x[n->in_col[e]];
                }
            }
        }
        free(drive); free(h); free(z); free(gh); free(gdrive); free(lg);
    }
    if (!bad) {
        for (int i = 0; i < 7; ++i) {
            for (size_t j = 0; j < ps[i]; ++j) {
                double s = 0.0;
                for (int t = 0; t < nthr; ++t) if (acc[t]) s += acc[t][goff[i] + j];
                G[i][j] += (float)s;
            }
        }
    }
    for (int t = 0; t < nthr; ++t) free(acc[t]);
    free(acc);
    return bad ? -1 : 0;
}

/* sqrt(sum of squares) of the seven gradient arrays (fc_grad_norm) */
double fo_grad_norm(float* const* G, const long long* sizes) {
    double ss = 0.0;
    for (int i = 0; i < 7; ++i) for (long long j = 0; j < sizes[i]; ++j) ss += (double)G[i][j] * G[i][j];
    return sqrt(ss);
}

/* one Adam step over the seven arrays (fc_step); t is the step count AFTER the increment; returns the pre-clip
 * norm (0 when max_norm <= 0, as the reference) */
double fo_adam(float* const* P, float* const* G, float* const* M, float* const* V, float* const* EMA,
               const long long* sizes, long long t, float lr, float lr_neuron, float lr_plug, float max_norm,
               float ema) {
    double g = max_norm > 0 ? fo_grad_norm(G, sizes) : 0.0;
    float gs = (max_norm > 0 && g > max_norm) ? (float)(max_norm / g) : 1.0f;
    long long tc = t < 100000 ? t : 100000;
    float c1 = 1.0f - (float)pow(0.9, (double)tc), c2 = 1.0f - (float)pow(0.999, (double)tc);
    for (int i = 0; i < 7; ++i) {
        float l = i == 0 ? lr : (i <= 2 ? lr_neuron : lr_plug);
        for (long long j = 0; j < sizes[i]; ++j) {
            float gr = G[i][j] * gs;
            float mi = 0.9f * M[i][j] + 0.1f * gr, vi = 0.999f * V[i][j] + 0.001f * gr * gr;
            M[i][j] = mi; V[i][j] = vi;
            float pi = P[i][j] - l * (mi / c1) / (sqrtf(vi / c2) + 1e-8f);
            P[i][j] = pi;
            EMA[i][j] = ema * EMA[i][j] + (1.0f - ema) * pi;
        }
    }
    return g;
}
