// af_argmax.cu -- single-launch greedy argmax over FP32 logits, plus the
// library's small runtime entry points (status strings, workspace reset,
// device queries).
//
// Reference: src/kernel/argmax.cu:23-119 (two launches; phase 2 reads only
// the first 256 of ceil(V/256) block results, so ids >= 65536 never win,
// argmax.cu:72-73,115-117).  AF_ARGMAX_TRUE returns the true argmax;
// AF_ARGMAX_REF_COMPAT reproduces the reference's restriction.  Ties resolve
// to the lowest index in both, as the reference's strict '>' tree does.
//
// Here: CTAs reduce grid-strided slices with 128-bit loads, write one
// (value, index) candidate each, and the last CTA to arrive (arrival counter
// in the caller's workspace) reduces the candidates and re-zeroes the counter.

#include <cfloat>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "af_common.cuh"
#include "af_internal.h"

namespace af {

constexpr int kArgThreads = 512;
constexpr int kArgMaxBlocks = 1024;

struct ArgmaxWs {
    int* done;
    float* val;
    int* idx;
};

__device__ __forceinline__ void warp_best(float& v, int& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (argmax_better(ov, oi, v, i)) { v = ov; i = oi; }
    }
}

// Block-wide (value, index) reduction; result valid in thread 0.
__device__ __forceinline__ void block_best(float& v, int& i) {
    __shared__ float sv[kArgThreads / 32];
    __shared__ int si[kArgThreads / 32];
    warp_best(v, i);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { sv[warp] = v; si[warp] = i; }
    __syncthreads();
    if (warp == 0) {
        v = lane < kArgThreads / 32 ? sv[lane] : 0.f;
        i = lane < kArgThreads / 32 ? si[lane] : -1;
        warp_best(v, i);
    }
}

__global__ void __launch_bounds__(kArgThreads) argmax_kernel(const float* __restrict__ logits, int n,
                                                             int* out, ArgmaxWs ws) {
    pdl_wait();
    pdl_launch_dependents();
    float v = 0.f;
    int i = -1;
    const int stride = gridDim.x * kArgThreads;
    const bool vec = (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
    const int n4 = vec ? n / 4 : 0;
    for (int q = blockIdx.x * kArgThreads + threadIdx.x; q < n4; q += stride) {
        const float4 f = ldcg_f4(logits + 4 * q);
        if (argmax_better(f.x, 4 * q + 0, v, i)) { v = f.x; i = 4 * q + 0; }
        if (argmax_better(f.y, 4 * q + 1, v, i)) { v = f.y; i = 4 * q + 1; }
        if (argmax_better(f.z, 4 * q + 2, v, i)) { v = f.z; i = 4 * q + 2; }
        if (argmax_better(f.w, 4 * q + 3, v, i)) { v = f.w; i = 4 * q + 3; }
    }
    for (int q = 4 * n4 + blockIdx.x * kArgThreads + threadIdx.x; q < n; q += stride) {
        const float f = ldcg_f32(logits + q);
        if (argmax_better(f, q, v, i)) { v = f; i = q; }
    }
    block_best(v, i);
    __shared__ int s_last;
    if (threadIdx.x == 0) {
        __stcg(ws.val + blockIdx.x, v);
        __stcg(ws.idx + blockIdx.x, i);
        __threadfence();
        s_last = (atomicAdd(ws.done, 1) == (int)gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    v = 0.f;
    i = -1;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += kArgThreads) {
        const float bv = ldcg_f32(ws.val + b);
        const int bi = ldcg_s32(ws.idx + b);
        if (argmax_better(bv, bi, v, i)) { v = bv; i = bi; }
        __stcg(ws.val + b, 0.f);   // leave the workspace all-zero: any op may reuse it next
        __stcg(ws.idx + b, 0);
    }
    block_best(v, i);
    if (threadIdx.x == 0) {
        *out = i;
        *ws.done = 0;
    }
}

namespace {
int argmax_blocks(int n, int sms) {
    int b = (n + kArgThreads * 8 - 1) / (kArgThreads * 8);
    if (b > 2 * sms) b = 2 * sms;
    if (b > kArgMaxBlocks) b = kArgMaxBlocks;
    if (b < 1) b = 1;
    return b;
}
}  // namespace

// ------------------------------------------------------------- runtime ---

static thread_local char g_cuda_err[256] = "";

af_status cuda_fail(cudaError_t e, const char* where) {
    snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s (%d)", where, cudaGetErrorString(e), (int)e);
    return AF_ERR_CUDA;
}

int device_sm_count(int* device_out) {
    static int cache[kMaxDevices] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    if (device_out) *device_out = dev;
    if (dev < 0 || dev >= kMaxDevices) return -1;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace af

using namespace af;

extern "C" const char* af_status_string(af_status s) {
    switch (s) {
        case AF_OK: return "ok";
        case AF_ERR_INVALID: return "invalid argument";
        case AF_ERR_UNSUPPORTED: return "unsupported";
        case AF_ERR_PEER_TIMEOUT: return "peer timeout";
        case AF_ERR_CUDA: return "cuda error";
        case AF_ERR_WORKSPACE: return "workspace missing or too small";
    }
    return "unknown status";
}

extern "C" const char* af_last_cuda_error(void) { return g_cuda_err; }

extern "C" int af_version(void) { return 110; }

extern "C" af_status af_device_faults(unsigned* out, int clear) {
    if (out == nullptr) return AF_ERR_INVALID;
    cudaError_t e1 = cudaSuccess, e2 = cudaSuccess, e3 = cudaSuccess, e4 = cudaSuccess;
    const unsigned v = gemv_faults(clear != 0, &e1) | decode_faults(clear != 0, &e2) | chain_faults(clear != 0, &e3) |
                       tc_faults(clear != 0, &e4);
    for (cudaError_t e : {e1, e2, e3, e4})
        if (e != cudaSuccess) return cuda_fail(e, "af_device_faults");
    *out = v;
    return AF_OK;
}

extern "C" af_status af_workspace_reset(void* workspace, size_t workspace_bytes, void* stream) {
    if (workspace == nullptr) return workspace_bytes == 0 ? AF_OK : AF_ERR_INVALID;
    cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "af_workspace_reset");
}

extern "C" size_t af_argmax_workspace_bytes(int V) {
    const int sms = device_sm_count();
    if (sms <= 0) return 0;
    const int b = argmax_blocks(V > 0 ? V : 1, sms);
    return round_up(256 + round_up((size_t)b * 4, 256) * 2, 256);
}

extern "C" af_status af_argmax_f32(const float* logits, int V, int* d_out, af_argmax_mode mode,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    if (V <= 0 || logits == nullptr || d_out == nullptr) return AF_ERR_INVALID;
    if (mode != AF_ARGMAX_TRUE && mode != AF_ARGMAX_REF_COMPAT) return AF_ERR_INVALID;
    const int sms = device_sm_count();
    if (sms <= 0) return AF_ERR_CUDA;
    const int n = (mode == AF_ARGMAX_REF_COMPAT && V > 65536) ? 65536 : V;
    const int blocks = argmax_blocks(n, sms);
    const size_t need = af_argmax_workspace_bytes(V);
    if (workspace == nullptr || workspace_bytes < need) return AF_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return AF_ERR_INVALID;
    unsigned char* b = static_cast<unsigned char*>(workspace);
    ArgmaxWs ws{reinterpret_cast<int*>(b), reinterpret_cast<float*>(b + 256),
                reinterpret_cast<int*>(b + 256 + round_up((size_t)blocks * 4, 256))};
    cudaError_t e = launch_pdl(argmax_kernel, dim3(blocks), dim3(kArgThreads), 0,
                               static_cast<cudaStream_t>(stream), logits, n, d_out, ws);
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "argmax_kernel");
}

// ------------------------------------------------------ no-allocation argmax ---
//
// Some callers cannot allocate device memory at all -- code that runs where
// cudaMalloc is forbidden or unavailable (a host that owns every allocation
// and hands out only input/output buffers, or an allocator-free deployment) --
// and so cannot provide the workspace af_argmax_f32 needs.  For them the same
// kernel runs on a scratch block that lives inside this library image: a
// file-scope __device__ array of kNoAllocScratchBytes, present on every GPU
// that loads the library until the process exits.
//
// The array's name in host code is only a host-side handle, not a device
// address; the device address is looked up with cudaGetSymbolAddress, once per
// device with that device current, on the first call made on that device.
// That first call should therefore come before any stream capture.  All calls
// share the one array: calls that can overlap on the GPU (different streams
// without ordering between them) race on it.

namespace af {
constexpr int kNoAllocBlocks = 256;                 // candidate slots in the scratch
constexpr int kNoAllocMaxV = 1 << 28;               // largest V accepted
constexpr size_t kNoAllocScratchBytes = 256 + 2 * kNoAllocBlocks * 4;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
unsigned char* noalloc_scratch_ptr(af_status* st) {
    static std::once_flag flags[kMaxDevices];
    static unsigned char* ptrs[kMaxDevices] = {nullptr};
    static cudaError_t errs[kMaxDevices];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *st = cuda_fail(e != cudaSuccess ? e : cudaErrorInvalidDevice, "af_argmax_f32_noalloc: device");
        return nullptr;
    }
    std::call_once(flags[dev], [&] {
        void* p = nullptr;
        errs[dev] = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        ptrs[dev] = static_cast<unsigned char*>(p);
    });
    if (errs[dev] != cudaSuccess || ptrs[dev] == nullptr) {
        *st = cuda_fail(errs[dev] != cudaSuccess ? errs[dev] : cudaErrorInvalidSymbol,
                        "af_argmax_f32_noalloc: cudaGetSymbolAddress");
        return nullptr;
    }
    *st = AF_OK;
    return ptrs[dev];
}
}  // namespace
}  // namespace af

extern "C" af_status af_argmax_f32_noalloc(const float* logits, int V, int* d_out, af_argmax_mode mode,
                                           void* stream) {
    if (V <= 0 || logits == nullptr || d_out == nullptr) return AF_ERR_INVALID;
    if (mode != AF_ARGMAX_TRUE && mode != AF_ARGMAX_REF_COMPAT) return AF_ERR_INVALID;
    if (V > kNoAllocMaxV) {
        snprintf(g_cuda_err, sizeof(g_cuda_err),
                 "af_argmax_f32_noalloc: V = %d exceeds the built-in scratch limit of %d logits", V,
                 kNoAllocMaxV);
        return AF_ERR_UNSUPPORTED;
    }
    const int sms = device_sm_count();
    if (sms <= 0) return AF_ERR_CUDA;
    af_status st = AF_OK;
    unsigned char* b = noalloc_scratch_ptr(&st);
    if (b == nullptr) return st;
    const int n = (mode == AF_ARGMAX_REF_COMPAT && V > 65536) ? 65536 : V;
    int blocks = argmax_blocks(n, sms);
    if (blocks > kNoAllocBlocks) blocks = kNoAllocBlocks;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The arrival counter must start at zero; the kernel leaves it (and the
    // candidates) zeroed, but clear it anyway in case an earlier call was cut short.
    cudaError_t e = cudaMemsetAsync(b, 0, 4, s);
    if (e != cudaSuccess) return cuda_fail(e, "af_argmax_f32_noalloc: clear");
    ArgmaxWs ws{reinterpret_cast<int*>(b), reinterpret_cast<float*>(b + 256),
                reinterpret_cast<int*>(b + 256 + kNoAllocBlocks * 4)};
    e = launch_pdl(argmax_kernel, dim3(blocks), dim3(kArgThreads), 0, s, logits, n, d_out, ws);
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "af_argmax_f32_noalloc: launch");
}
