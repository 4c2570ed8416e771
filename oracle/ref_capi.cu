// ref_capi.cu -- C entry points around the REFERENCE's own kernels, for tests
// and for bench.py's reference arm.  TEST INFRASTRUCTURE ONLY.
//
// Linked, by oracle/Makefile, with the unmodified AtomFlow sources
// src/kernel/qkv_gemm.cu and src/kernel/argmax.cu, compiled in place with the
// reference's release flags (-O3 --use_fast_math -DNDEBUG, CMakeLists.txt
// :12-14,117-131) for sm_100a.  Nothing here re-implements the reference; each
// function builds the reference's Views and calls its launcher.
#include <cuda_runtime.h>
#include <cublas_v2.h>

#include "core/view.h"
#include "ops/kernel.h"

extern "C" int afref_w8a16_gemv(const void* x, const void* w, const void* s, void* y, int N,
                                int K, void* stream) {
    // The engine's Views for one GEMV: act [1,K], weight [N,K], scales [N,K/128],
    // output [1,N] (src/core/engine.cu:110-139,175-182).
    View ax = create_contiguous_view(const_cast<void*>(x), DataType::FP16, {1, K});
    View wv = create_contiguous_view(const_cast<void*>(w), DataType::FP8_E4M3, {N, K});
    View sv = create_contiguous_view(const_cast<void*>(s), DataType::FP16, {N, K / 128});
    View yv = create_contiguous_view(y, DataType::FP16, {1, N});
    launch_w8a16_gemv(ax, wv, sv, yv, 128, static_cast<cudaStream_t>(stream));
    return (int)cudaGetLastError();
}

extern "C" int afref_argmax(const float* logits, int V, int* out, void* stream) {
    View lv = create_contiguous_view(const_cast<float*>(logits), DataType::FP32, {1, V});
    launch_argmax(lv, out, static_cast<cudaStream_t>(stream));
    return (int)cudaGetLastError();
}

// The engine's lm_head call, argument for argument (src/core/engine.cu:498-512).
extern "C" int afref_lm_head(const void* w, const void* x, float* logits, int V, int D,
                             void* stream) {
    static cublasHandle_t handle[64] = {nullptr};
    int dev = 0;
    cudaGetDevice(&dev);
    if (handle[dev] == nullptr && cublasCreate(&handle[dev]) != CUBLAS_STATUS_SUCCESS) return -1;
    cublasSetStream(handle[dev], static_cast<cudaStream_t>(stream));
    float alpha = 1.0f, beta = 0.0f;
    cublasStatus_t st = cublasGemmEx(handle[dev], CUBLAS_OP_T, CUBLAS_OP_N, V, 1, D, &alpha, w,
                                     CUDA_R_16F, D, x, CUDA_R_16F, D, &beta, logits, CUDA_R_32F, V,
                                     CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    return st == CUBLAS_STATUS_SUCCESS ? (int)cudaGetLastError() : -(int)st;
}
