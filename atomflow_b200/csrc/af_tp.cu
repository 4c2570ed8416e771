// af_tp.cu -- lifecycle of the tensor-parallel exchange buffers used by
// af_w8a16_gemv_allreduce (the kernel side lives in af_gemv.cu).
//
// Each rank allocates one buffer at setup (never per call), zero-fills it and
// exports it with CUDA IPC; each rank maps every peer's buffer.  Only plain
// peer stores and loads touch peer memory -- no multicast of any kind.

#include <cuda_runtime.h>
#include <cstdlib>
#include <cstring>
#include <new>

#include "af_internal.h"

using namespace af;

extern "C" size_t af_tp_buffer_bytes(int max_n) { return max_n > 0 ? TpLayout::bytes(max_n) : 0; }

extern "C" af_status af_tp_create(int rank, int world, int max_n, af_tp_comm** out) {
    if (out == nullptr || world < 1 || world > kTpMaxRanks || rank < 0 || rank >= world || max_n <= 0)
        return AF_ERR_INVALID;
    *out = nullptr;
    af_tp_comm* c = new (std::nothrow) af_tp_comm();
    if (c == nullptr) return AF_ERR_INVALID;
    c->rank = rank;
    c->world = world;
    c->nmax = max_n;
    c->wait_ns = 2000000000ull;
    cudaError_t e = cudaGetDevice(&c->device);
    if (e == cudaSuccess) e = cudaMalloc(&c->buf, TpLayout::bytes(max_n));
    if (e == cudaSuccess) e = cudaMemset(c->buf, 0, TpLayout::bytes(max_n));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (c->buf) cudaFree(c->buf);
        delete c;
        return cuda_fail(e, "af_tp_create");
    }
    c->peer[rank] = c->buf;
    *out = c;
    return AF_OK;
}

extern "C" af_status af_tp_ipc_handle(const af_tp_comm* c, void* handle64) {
    if (c == nullptr || handle64 == nullptr) return AF_ERR_INVALID;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, c->buf);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    memcpy(handle64, &h, 64);
    return AF_OK;
}

extern "C" af_status af_tp_open_peers(af_tp_comm* c, const void* handles) {
    if (c == nullptr || handles == nullptr) return AF_ERR_INVALID;
    for (int r = 0; r < c->world; ++r) {
        if (r == c->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const unsigned char*>(handles) + (size_t)r * 64, 64);
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
        c->peer[r] = static_cast<unsigned char*>(p);
        c->ipc_opened[r] = true;
    }
    return AF_OK;
}

extern "C" af_status af_tp_set_peer(af_tp_comm* c, int r, void* buf) {
    if (c == nullptr || r < 0 || r >= c->world || r == c->rank || buf == nullptr) return AF_ERR_INVALID;
    c->peer[r] = static_cast<unsigned char*>(buf);
    c->ipc_opened[r] = false;
    return AF_OK;
}

extern "C" void* af_tp_buffer(const af_tp_comm* c) { return c ? c->buf : nullptr; }

extern "C" af_status af_tp_set_wait_limit_ms(af_tp_comm* c, int ms) {
    if (c == nullptr || ms < 1) return AF_ERR_INVALID;
    c->wait_ns = (unsigned long long)ms * 1000000ull;
    return AF_OK;
}

extern "C" af_status af_tp_status(const af_tp_comm* c, int* status) {
    if (c == nullptr || status == nullptr) return AF_ERR_INVALID;
    cudaError_t e = cudaMemcpy(status, c->buf + TpLayout::status, 4, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "af_tp_status");
}

extern "C" af_status af_tp_destroy(af_tp_comm* c) {
    if (c == nullptr) return AF_OK;
    for (int r = 0; r < c->world; ++r)
        if (c->ipc_opened[r]) cudaIpcCloseMemHandle(c->peer[r]);
    if (c->buf) cudaFree(c->buf);
    delete c;
    return AF_OK;
}
