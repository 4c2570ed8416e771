// ref_capi.cu -- C entry points around the REFERENCE's own kernels, for tests
// and for bench.py's reference arm.  TEST INFRASTRUCTURE ONLY.
//
// Linked, by oracle/Makefile, with the unmodified AtomFlow sources
// src/kernel/{qkv_gemm,argmax,rmsnorm,swiglu,residual_add}.cu, compiled in place with the
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

// The engine's RMSNorm call (src/core/engine.cu:294,409): FP16 [1,D] in, FP32 weight, eps 1e-5.
extern "C" int afref_rms_norm(const void* x, const float* w, void* out, int D, float eps, void* stream) {
    View xv = create_contiguous_view(const_cast<void*>(x), DataType::FP16, {1, D});
    View wv = create_contiguous_view(const_cast<float*>(w), DataType::FP32, {D});
    View ov = create_contiguous_view(out, DataType::FP16, {1, D});
    launch_rms_norm(xv, wv, ov, eps, static_cast<cudaStream_t>(stream));
    return (int)cudaGetLastError();
}

// src/core/engine.cu:448: out = silu(gate) * up (FP16), in place over gate there.
extern "C" int afref_swiglu(const void* gate, const void* up, void* out, int N, void* stream) {
    View gv = create_contiguous_view(const_cast<void*>(gate), DataType::FP16, {1, N});
    View uv = create_contiguous_view(const_cast<void*>(up), DataType::FP16, {1, N});
    View ov = create_contiguous_view(out, DataType::FP16, {1, N});
    launch_swiglu(gv, uv, ov, static_cast<cudaStream_t>(stream));
    return (int)cudaGetLastError();
}

// src/core/engine.cu:401,483: inout += sub (FP16, in place).
extern "C" int afref_residual_add(void* inout, const void* sub, int N, void* stream) {
    View iv = create_contiguous_view(inout, DataType::FP16, {1, N});
    View sv = create_contiguous_view(const_cast<void*>(sub), DataType::FP16, {1, N});
    launch_residual_add(iv, sv, static_cast<cudaStream_t>(stream));
    return (int)cudaGetLastError();
}

// RoPE on one token at a position (engine.cu:334-346: cos/sin pointers offset by the position, seq 1),
// then the KV-cache write (engine.cu:350-355).
extern "C" int afref_rope_kv(void* qkv, const float* d_cos, const float* d_sin, void* k_cache, void* v_cache,
                             int pos, int NH, int NKV, int HD, void* stream) {
    const int q_dim = NH * HD, kv_dim = NKV * HD;
    half* base = static_cast<half*>(qkv);
    View qv = create_contiguous_view(base, DataType::FP16, {1, q_dim});
    View kv = create_contiguous_view(base + q_dim, DataType::FP16, {1, kv_dim});
    launch_rope(qv, kv, d_cos + (size_t)pos * (HD / 2), d_sin + (size_t)pos * (HD / 2), 1, NKV, NH, HD,
                static_cast<cudaStream_t>(stream));
    View all = create_contiguous_view(qkv, DataType::FP16, {1, q_dim + 2 * kv_dim});
    View kc = create_contiguous_view(k_cache, DataType::FP16, {2048, kv_dim});
    View vc = create_contiguous_view(v_cache, DataType::FP16, {2048, kv_dim});
    launch_write_kv_cache(all, kc, vc, pos, q_dim, kv_dim, static_cast<cudaStream_t>(stream));
    return (int)cudaGetLastError();
}

extern "C" int afref_rope_cache(float* d_cos, float* d_sin, int max_seq, int HD, float base, void* stream) {
    build_rope_cache(d_cos, d_sin, max_seq, HD, base, static_cast<cudaStream_t>(stream));
    return (int)cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
}

extern "C" int afref_cached_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                                      int seq_len, int HD, int NH, int NKV, void* stream) {
    launch_cached_attention(static_cast<const half*>(q), static_cast<const half*>(k_cache),
                            static_cast<const half*>(v_cache), static_cast<half*>(out), seq_len, HD, NH, NKV,
                            static_cast<cudaStream_t>(stream));
    return (int)cudaGetLastError();
}
