// ref_engine.cu -- C entry points around the REFERENCE's decode engine
// (AtomFlowEngine, src/core/engine.cu), for the decode-step parity test and
// bench.py's reference arm.  TEST INFRASTRUCTURE ONLY.  Linked by
// oracle/Makefile with the reference's unmodified engine and kernel sources.
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <string>
#include <vector>

// The logits View is a private member; the checker reads it (for the top-2
// margin of a divergent step) without changing the engine's code.
#define private public
#include "core/engine.h"
#undef private

extern "C" void* afref_engine_create(const char* path) {
    AtomFlowEngine* e = new AtomFlowEngine();
    e->initialize(path);
    return e;
}

extern "C" void afref_engine_destroy(void* h) { delete static_cast<AtomFlowEngine*>(h); }

// One greedy step as main.cu's autoregressive loop does it (main.cu:235-245).
extern "C" int afref_engine_step(void* h, int token, int pos) {
    AtomFlowEngine* e = static_cast<AtomFlowEngine*>(h);
    e->current_pos_ = pos;
    e->inject_token(token);
    e->forward_pass();
    return e->get_output_token();
}

// Device pointer of the engine's FP32 logits [V] (ActBuffers::logits) and V.
extern "C" const void* afref_engine_logits(void* h, int* vocab) {
    AtomFlowEngine* e = static_cast<AtomFlowEngine*>(h);
    if (vocab) *vocab = e->V;
    return e->act_.logits.data_ptr;
}

// TPOT as main.cu measures it (main.cu:92-150): forward_pass at a fixed
// position captured into one CUDA graph, replayed; CUDA events around
// `iters` replays after `warmup`.  Returns ms per step.
extern "C" float afref_engine_tpot_ms(void* h, int pos, int iters, int warmup) {
    AtomFlowEngine* e = static_cast<AtomFlowEngine*>(h);
    e->current_pos_ = pos;
    cudaStream_t st = e->stream();
    e->forward_pass();   // eager warm-up
    cudaStreamSynchronize(st);
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeGlobal) != cudaSuccess) return -1.f;
    e->forward_pass();
    if (cudaStreamEndCapture(st, &g) != cudaSuccess) return -2.f;
    if (cudaGraphInstantiate(&ge, g, nullptr, nullptr, 0) != cudaSuccess) return -3.f;
    for (int i = 0; i < warmup; ++i) cudaGraphLaunch(ge, st);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, st);
    for (int i = 0; i < iters; ++i) cudaGraphLaunch(ge, st);
    cudaEventRecord(b, st);
    cudaEventSynchronize(b);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaGraphExecDestroy(ge);
    cudaGraphDestroy(g);
    return ms / iters;
}
