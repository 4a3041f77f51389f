// fg_kl_loss_noalloc: the distillation loss and its gradient for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc or any allocating routine: a trainer embedded in a host
// application that hands the library only pointers into memory it reserved up front, or a process running under a
// fixed device-memory budget shared with a simulator. This entry point computes, for logits a caller already has,
// KL(softmax(teacher * inv_temp) || softmax(logits)) and its gradient without any allocation: its per-sample scratch
// lives in a file-scope __device__ array (g_loss_scratch below, kNoAllocMaxBatch samples, 512 KiB), which every GPU
// that loads the library holds until the process exits.
//
// Set-up: the first call on a device looks up that array's device address (cudaGetSymbolAddress, with the device
// current) and keeps it; make that first call before any stream capture. Every later call on the device reuses the
// same array, so calls whose work overlaps on the GPU (different streams, not ordered) race on it; the array keeps
// the last call's values, and each call overwrites every entry it reads, so nothing needs clearing.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>
#include <string>

#include "flyguy_b200.h"

namespace {

constexpr int kNoAllocMaxBatch = 65536;
constexpr int kNoAllocMaxDevices = 64;

// per-sample KL and argmax agreement of the last call (2 x kNoAllocMaxBatch floats)
static __device__ __align__(256) float g_loss_scratch[2 * kNoAllocMaxBatch];

float* g_scratch_ptr[kNoAllocMaxDevices] = {};
std::mutex g_mu;
thread_local std::string g_err;

// one thread per sample, the caller's [B, n_act] rows: the same arithmetic as the fused step's loss
__global__ void k_loss_rows(const float* __restrict__ lg, const float* __restrict__ teacher, float* __restrict__ dl,
                            float* __restrict__ scratch, int n_act, int B, float it) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const float* s = lg + (size_t)b * n_act;
    const float* t = teacher + (size_t)b * n_act;
    float ms = -INFINITY, mt = -INFINITY;
    int as = 0, at = 0;
    for (int a = 0; a < n_act; ++a) {
        const float tv = t[a] * it;
        if (s[a] > ms) { ms = s[a]; as = a; }
        if (tv > mt) { mt = tv; at = a; }
    }
    float zs = 0.f, zt = 0.f;
    for (int a = 0; a < n_act; ++a) { zs += expf(s[a] - ms); zt += expf(t[a] * it - mt); }
    const float ls = ms + logf(zs), lt = mt + logf(zt), inv_b = 1.f / (float)B;
    float kl = 0.f;
    for (int a = 0; a < n_act; ++a) {
        const float lps = s[a] - ls, lpt = t[a] * it - lt, pt = expf(lpt);
        kl += pt * (lpt - lps);
        dl[(size_t)b * n_act + a] = (expf(lps) - pt) * inv_b;
    }
    scratch[b] = kl;
    scratch[kNoAllocMaxBatch + b] = as == at ? 1.f : 0.f;
}

// stats[0] = sum of KL, stats[1] = argmax agreements; one CTA adds the per-sample values in a fixed order
__global__ void k_loss_rows_stats(const float* __restrict__ scratch, float* __restrict__ stats, int B) {
    __shared__ float red[2][32];
    float k = 0.f, a = 0.f;
    for (int b = threadIdx.x; b < B; b += blockDim.x) { k += scratch[b]; a += scratch[kNoAllocMaxBatch + b]; }
    for (int o = 16; o; o >>= 1) {
        k += __shfl_xor_sync(0xffffffffu, k, o);
        a += __shfl_xor_sync(0xffffffffu, a, o);
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { red[0][w] = k; red[1][w] = a; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float sk = 0.f, sa = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { sk += red[0][i]; sa += red[1][i]; }
        stats[0] = sk;
        stats[1] = sa;
    }
}

// the device address of g_loss_scratch on the current device, looked up once per device
float* scratch_of_current_device() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { g_err = std::string("cudaGetDevice: ") + cudaGetErrorString(e); return nullptr; }
    if (dev < 0 || dev >= kNoAllocMaxDevices) { g_err = "device index out of range"; return nullptr; }
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
        float* p = nullptr;
        e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_loss_scratch);
        if (e != cudaSuccess) {
            g_err = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e);
            return nullptr;
        }
        g_scratch_ptr[dev] = p;
    }
    return g_scratch_ptr[dev];
}

}  // namespace

extern "C" {

int fg_kl_loss_noalloc(const float* logits, const float* teacher, int B, int n_act, float inv_temp, float* dlogits,
                       float* stats, void* stream) {
    if (B <= 0 || B > kNoAllocMaxBatch) {
        g_err = "fg_kl_loss_noalloc: batch " + std::to_string(B) + " is outside 1.." + std::to_string(kNoAllocMaxBatch) +
                " (the size of its fixed scratch)";
        return -1;
    }
    if (n_act <= 0 || !logits || !teacher || !dlogits || !stats) {
        g_err = "fg_kl_loss_noalloc: bad arguments";
        return -1;
    }
    float* scratch = scratch_of_current_device();
    if (!scratch) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    k_loss_rows<<<(B + 255) / 256, 256, 0, st>>>(logits, teacher, dlogits, scratch, n_act, B, inv_temp);
    k_loss_rows_stats<<<1, 256, 0, st>>>(scratch, stats, B);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_err = std::string("fg_kl_loss_noalloc: ") + cudaGetErrorString(e);
        return -1;
    }
    return 0;
}

const char* fg_noalloc_last_error(void) { return g_err.c_str(); }

}  // extern "C"
