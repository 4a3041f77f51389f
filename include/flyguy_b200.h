/* flyguy_b200 - the connectome hop path of flyguy on B200 (sm_100a), as a C-ABI shared library.
 *
 * libflyguy_b200.so replaces the reference's whole-network GPU library `fc_*` (adventure-gpt/flyguy,
 * flyguy/native/flyguy_train.cu:553-629, built with -DFLYGUY_CORE, loaded by ctypes in flyguy/fly_native.py:127-159).
 * Every fc_* entry point below keeps the reference's name, argument order and meaning, so the reference's ctypes
 * binding loads this library by path alone. The fg_* entry points are additions (status codes instead of exiting
 * the process, an explicit stream, bf16 activations, zero-copy gradient for the data-parallel all-reduce, the fused
 * teaching step, host-buffer forward).
 *
 * Conventions (all entry points):
 *  - Pointers named obs / logits / dlogits / teacher are DEVICE memory owned by the caller (torch tensors), fp32,
 *    row-major [B, obs_dim] / [B, n_act], contiguous - except fg_forward_host, which takes HOST memory.
 *  - B is a multiple of 32 and at most the max_batch given at creation.
 *  - Work is queued on the handle's stream (fc_set_stream; default: the legacy default stream) in order; calls return
 *    before the GPU finishes unless they return a value that needs the GPU (fc_grad_norm, fc_step with max_norm > 0,
 *    fg_teach with stats != NULL).
 *  - Errors never end the process: a failing call records a message in the handle, later calls on the handle
 *    return at once, and fg_status / fg_last_error report it. A NULL handle from create: fg_last_error(NULL).
 *  - A handle is not thread-safe; use one per thread.
 */
#ifndef FLYGUY_B200_H
#define FLYGUY_B200_H

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference-compatible entry points (flyguy/native/flyguy_train.cu) ---------------------------------------- */

/* Loads NET.bin ("FLY1", flyguy/native/export.py:9-16) and allocates weights, gradient, Adam state, running average
 * and fp32 states for batches up to max_batch. Replaces fc_create (flyguy_train.cu:569-575). NULL on failure. */
void* fc_create(const char* net_path, int max_batch);

/* out[0..6]: lengths of the seven weight arrays (W in play, gain, theta, in_w, in_b, out_w, out_b); out[7] obs_dim,
 * out[8] n_act, out[9] max_batch. Replaces fc_sizes (flyguy_train.cu:577-581). */
void fc_sizes(void* h, long long* out);

/* which: 0 weights, 1 running average, 2 / 3 Adam's first / second moments, 4 gradient. ptrs: seven device arrays
 * (NULL = skip). to_core 1: read them into the library; 0: write the library's arrays into them.
 * Replaces fc_copy (flyguy_train.cu:584-589). */
void fc_copy(void* h, int which, int to_core, float** ptrs);

/* obs [B, obs_dim] -> logits [B, n_act] with the weights (ema 0) or their running average (ema 1). The states stay
 * for fc_backward. Replaces fc_forward (flyguy_train.cu:592-598). */
void fc_forward(void* h, const float* obs, int B, float* logits, int ema);

/* gradient = 0. Replaces fc_zero_grad (flyguy_train.cu:599-602). */
void fc_zero_grad(void* h);

/* dlogits [B, n_act]: gradient of a loss w.r.t. the logits of the batch the last fc_forward(.., ema 0) went through;
 * the weights' gradients are ADDED to the library's gradient. Replaces fc_backward (flyguy_train.cu:604-609). */
void fc_backward(void* h, const float* dlogits, int B);

/* Euclidean norm of the whole gradient (waits for the GPU). Replaces fc_grad_norm (flyguy_train.cu:610-616). */
float fc_grad_norm(void* h);

/* One Adam step (betas 0.9 / 0.999, eps 1e-8) from the gradient; strengths at lr, gain / theta at lr_neuron, plugs
 * at lr_plug; the gradient is scaled to max_norm first if longer (0 = no clipping); the running average follows with
 * decay `ema`. Returns the gradient norm before clipping (0 when max_norm is 0).
 * Replaces fc_step (flyguy_train.cu:619-627). */
float fc_step(void* h, float lr, float lr_neuron, float lr_plug, float max_norm, float ema);

/* Adam's step count; set >= 0 sets it. Replaces fc_adam_t (flyguy_train.cu:628). */
long long fc_adam_t(void* h, long long set);

/* Waits for the handle's stream. Replaces fc_sync (flyguy_train.cu:629). */
void fc_sync(void* h);

/* ---- additions ------------------------------------------------------------------------------------------------ */

#define FG_ACT_BF16 1     /* states stored as bf16 (fp32 accumulation, fp32 weights); forward only */
#define FG_INFER_ONLY 2   /* no gradient / optimiser buffers: fc_backward and fc_step fail */
#define FG_ACT_F16 4      /* states stored as IEEE fp16 (the reference's 16-bit "cuda16" states); forward only */
/* In both 16-bit modes every layer but the last is stored in the 16-bit type, rounded to nearest even where it is
   written; the last layer (the descending neurons the output plug reads) stays fp32, and the input plug reads the
   observation values rounded to the same 16-bit type. Sums are fp32 throughout. */

/* fc_create with flags (FG_ACT_BF16 and FG_ACT_F16 imply FG_INFER_ONLY). */
void* fg_create(const char* net_path, int max_batch, int flags);
/* Frees the handle and its device memory (the reference never frees its handle). */
void fg_destroy(void* h);
/* 0 = fine; otherwise the handle is in error and fg_last_error says why. */
int fg_status(void* h);
const char* fg_last_error(void* h);
/* Clears a recorded error (after the caller handled it). */
void fg_clear_error(void* h);
/* All later work of the handle goes to this cudaStream_t (e.g. torch.cuda.current_stream().cuda_stream). */
void fc_set_stream(void* h, void* stream);
/* Device pointer and length of one flat array (which as in fc_copy): the seven arrays in fc_sizes order, each
 * starting on a 256-byte boundary (fg_offsets; the gaps stay zero). The gradient (which 4) is what a data-parallel
 * trainer all-reduces in place before fc_step. */
int fg_flat(void* h, int which, float** ptr, long long* n);
/* The seven arrays' offsets into the flat arrays, in floats: off[0..7] (off[7] = the flat length). */
void fg_offsets(void* h, long long* off);
/* Layer sizes: sizes[0..hops] (returns hops); merged (destination, source) pairs per hop into pairs[0..hops-1]. */
int fg_layout(void* h, int* sizes, long long* pairs);
/* The work plan's counts, for roofline arithmetic: per hop 8 values {rows, source rows, edges, merged pairs,
   transposed pairs kept for the backward, rows whose gradient can be non-zero, source rows the backward writes, edges
   of the live rows' pairs}, then {sensory rows the plug backward visits, sensory rows, plug fan, descending rows}.
   Writes min(n, count) values into out; returns the count (8 * hops + 4), or -1 on error. */
int fg_plan(void* h, long long* out, int n);
/* Gradient buckets for a data-parallel all-reduce that overlaps the backward (the reference all-reduces after the
   whole backward: NativeAdam.step -> dist.mean_, fly_native.py:78-81). Writes up to n triples {first, end, stage} of the
   flat gradient (fg_flat 4) into out and returns their count: stage 0 = final once the output plug's backward is
   done, stage k + 1 = final once hop k's weight gradient is done, -1 = final when the backward returns. The ranges
   cover [0, flat length) once. */
int fg_grad_buckets(void* h, long long* out, int n);
/* The caller's cudaEvent_t (NULL: none) that the backward records on the handle's stream when it reaches `stage`
   (0..hops, as in fg_grad_buckets); a side stream that waits on it can start that bucket's all-reduce. Returns 0, or
   -1 for a stage out of range. */
int fg_set_stage_event(void* h, int stage, void* event);
/* The gradient packed without its structural zeros, for a smaller data-parallel all-reduce: the connection strengths
   that a live edge can change (every other strength's gradient is exactly zero on every rank: the backward never
   writes it after fc_zero_grad), then the other six arrays whole. unpack = 0: buf (device, cap floats) <- the
   gradient; unpack = 1: the gradient <- buf (the strengths outside the packed set keep their zero). Queued on the
   handle's stream. Returns the packed length (buf NULL or cap 0: the length only), or -1. */
long long fg_grad_pack(void* h, float* buf, long long cap, int unpack);

/* The distillation step's device half, fused: forward with the weights, KL(softmax(teacher * inv_temp) ||
 * softmax(logits)) averaged over the batch, its gradient through the network ADDED to the gradient.
 * obs [B, obs_dim], teacher [B, n_act] device; logits [B, n_act] device or NULL. stats: host double[2] (sum of KL over
 * the batch, number of argmax agreements), or NULL to not wait for the GPU. Returns 0 or -1 (see fg_last_error). */
int fg_teach(void* h, const float* obs, const float* teacher, int B, float inv_temp, float* logits, double* stats);
/* fg_teach with the loss averaged over loss_norm samples instead of B: a batch larger than max_batch goes through in
 * pieces (each adds its share of the gradient of the mean over all loss_norm samples). fg_teach = loss_norm B. */
int fg_teach_ex(void* h, const float* obs, const float* teacher, int B, float inv_temp, float loss_norm, float* logits,
                double* stats);

/* Forward from HOST memory: obs_host [B, obs_dim] -> logits_host [B, n_act], host<->device copies overlapped with the
 * compute in chunks (pinned host memory makes the copies asynchronous). Waits for the result. Returns 0 or -1. */
int fg_forward_host(void* h, const float* obs_host, int B, float* logits_host, int ema);

/* Neuron-major states of layer k (0 = sensory ... hops) of the last forward: [sizes[k], B] fp32, device. */
int fg_layer(void* h, int k, float* out, int B);

/* Number of kernels this handle has launched so far. */
long long fg_launches(void* h);
/* on 1: every later kernel launch is bracketed by CUDA events on the handle's stream (for live per-kernel timing);
 * on 0: stop (after reading). */
int fg_timing(void* h, int on);
/* Like fg_timing, for the classes whose bit (1 << class, classes as for fg_timing_read) is set in mask only; the other
 * launches run without events. mask 0: stop (after reading). */
int fg_timing_classes(void* h, unsigned mask);
/* Waits for the stream; sums the recorded times per kernel class into ms[0..n-1] (milliseconds) and count[0..n-1]
 * (launches), then forgets them. Classes: 0 layout change, 1 weight folds, 2 input plug, 3 hop forward, 4 output
 * plug, 5 loss, 6 output-plug backward, 7 neuron backward, 8 weight gradient, 9 transposed hop, 10 plug backward,
 * 11 Adam, 12 gradient norm. Returns the number of classes. */
int fg_timing_read(void* h, double* ms, long long* count, int n);

/* No counterpart in the reference. KL(softmax(teacher * inv_temp) || softmax(logits)) over a batch and its gradient
 * for callers that cannot allocate device memory (for example a trainer embedded in a host application that only
 * hands over pointers into memory it reserved up front). logits, teacher, dlogits: [B, n_act] device, fp32;
 * dlogits = (softmax(logits) - p_teacher) / B; stats: device float[2] = sum of KL over the batch, number of argmax
 * agreements. Allocates nothing: its scratch is a fixed 512 KiB array inside the library, so B is at most 65,536
 * (larger batches are refused with -1). The first call on a device looks up that array and should come before any
 * stream capture; calls that overlap on the GPU share the array and race. Queued on `stream`; returns 0 or -1
 * (fg_noalloc_last_error says why). */
int fg_kl_loss_noalloc(const float* logits, const float* teacher, int B, int n_act, float inv_temp, float* dlogits,
                       float* stats, void* stream);
const char* fg_noalloc_last_error(void);

/* The firing survey (the reference trainer's survey(), flyguy_train.cu:437-454, kernel k_fired at 180-187): one
 * forward of obs [B, obs_dim] (device) with the weights (ema 0) or their running average (ema 1) that ADDS, for every
 * row of every layer (the sensory rows, then each hop's rows in order: fg_layout), the number of samples whose state
 * is positive to fired[row] and the sum of the squared pre-activations (sensory rows: 0) to sq[row] (device arrays).
 * teacher [B, n_act] and stats non-NULL (training handles): stats[0] = sum of KL at temperature 1 over the batch,
 * stats[1] = argmax agreements (waits for the GPU). Returns 0 or -1. */
int fg_survey(void* h, const float* obs, const float* teacher, int B, int ema, int* fired, float* sq, double* stats);

/* ---- the per-hop operator (replaces the reference's HopCuda, flyguy/fly_cuda.py:78-115) ------------------------
 * Handle-free, on the caller's device buffers and stream (NULL = the legacy default stream); states are
 * [neurons, batch] fp32, 16-byte aligned, batch a multiple of 32; CSR index arrays as the reference's FlyActor buffers
 * (crow/tcrow/tperm int64, col/tcol int32). Return 0, or -1 with the reason in fg_hop_last_error(). */

/* HopCuda.forward (fly_cuda.py:83-92, kernels spmm_f / spmm_h at 25-39): out[t, b] = sum over the edges e of row t of
 * w[e] * h[col[e], b]. half != 0: h read rounded to fp16 (h.half()), sums in fp32. */
int fg_hop_fwd(const float* w, const float* h, const long long* crow, const int* col, int n_rows, int n_src, int B,
               int half, float* out, void* stream);
/* HopCuda.backward (fly_cuda.py:94-115, kernels sddmm_f / sddmm_h at 44-54): gw[e] = sum_b gz[t(e), b] * h[col[e], b]
 * (gw NULL: skipped); gh[s, b] = sum over the by-source edges i of s of w[tperm[i]] * gz[tcol[i], b] (gh NULL:
 * skipped). half != 0: gz / max|gz| and h read rounded to fp16, sums in fp32, results times max|gz| (fly_cuda.py:100-113). */
int fg_hop_bwd(const float* w, const float* h, const float* gz, const long long* crow, const int* col,
               const long long* tcrow, const int* tcol, const long long* tperm, int n_rows, int n_src, int B,
               int half, float* gw, float* gh, void* stream);
/* Why the calling thread's last fg_hop_* call failed ("" after a success). */
const char* fg_hop_last_error(void);

/* ---- the playing network's interface (replaces the reference's CPU library flyguy/native/fly_infer.cpp, loaded by
 * FlyActor._native, flyguy/fly.py:187-241): the same names, arguments and HOST buffers; the forward runs on the GPU.
 * Errors: fg_fly_last_error() (the interface itself has no status; a failed fly_forward answers NaN logits). */

/* fly_infer.cpp:33-36. */
void* fly_create(int obs_dim, int n_act, int hops);
/* fly_infer.cpp:37-42: the plug, CSR by sensory row; gain g0 and threshold t0 (softplus(theta)) per sensory row. */
void fly_set_plug(void* p, int n_s, int E, const int* crow, const int* col, const float* w, const float* b,
                  const float* g0, const float* t0);
/* fly_infer.cpp:43-47: hop k's connections by SOURCE neuron (tcrow[src + 1], tcol = target row, w in that order),
 * gain g and threshold t per target row, drow = the sensory row re-driven into a target row or -1. */
void fly_set_hop(void* p, int k, int rows, int src, int E, const int* tcrow, const int* tcol, const float* w,
                 const float* g, const float* t, const int* drow);
/* fly_infer.cpp:48-54: the output plug, w [n_act, n_dn] row = action. */
void fly_set_out(void* p, int n_dn, const int* dn, const float* w, const float* b);
/* fly_infer.cpp:55-97: obs [batch, obs_dim] -> logits [batch, n_act] (host); tap (or NULL): one byte per neuron
 * state of the first car, layer after layer, 255 * tanh(1.5 * state). */
void fly_forward(void* p, const float* obs, int batch, float* logits, unsigned char* tap);
/* fly_infer.cpp:98. */
void fly_free(void* p);
/* Why the calling thread's last fly_* call failed ("" after a success). */
const char* fg_fly_last_error(void);

/* ---- the standalone teaching trainer (replaces the reference's flyguy_train executable, flyguy/native/
 * flyguy_train.cu main() at 631-788): argv as the command line "fg_train NET.bin PARAMS.bin DATA_DIR OUT_PREFIX
 * [options]" (options and file formats in csrc/fg_train.cu). Returns the process exit status (0: done or stopped). */
int fg_train_main(int argc, const char* const* argv);

#ifdef __cplusplus
}
#endif
#endif
