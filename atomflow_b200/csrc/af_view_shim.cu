// af_view_shim.cu -- the reference's View-based launchers (include/ops/kernel.h)
// implemented on this library's C ABI.  See include/atomflow_view_ops.h for the
// ABI contract (exact mangled names, View layout, error behaviour).

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <atomic>
#include <mutex>

#include "../../include/atomflow_b200.h"
#include "../../include/atomflow_view_ops.h"
#include "af_internal.h"

// The reference View (include/core/view.h:22-39) as laid out by g++ on x86-64.
static_assert(sizeof(View) == 56, "View must keep the reference's 56-byte layout");
static_assert(offsetof(View, data_ptr) == 8, "View::data_ptr offset");
static_assert(offsetof(View, dims) == 16, "View::dims offset");
static_assert(offsetof(View, strides) == 32, "View::strides offset");
static_assert(offsetof(View, num_dims) == 48, "View::num_dims offset");

namespace {

thread_local int g_last_status = AF_OK;

void report(af_status st, const char* op) {
    g_last_status = st;
    if (st == AF_OK) return;
    std::fprintf(stderr, "[atomflow_b200] %s failed: %s %s\n", op, af_status_string(st),
                 st == AF_ERR_CUDA ? af_last_cuda_error() : "");
    static const bool abort_on_error = [] {
        const char* e = std::getenv("AF_VIEW_ABORT");
        return e != nullptr && e[0] == '1';
    }();
    if (abort_on_error) std::abort();
}

// Rows of an activation View: the product of all but the last dim
// (calculate_rows, include/ops/kernel.h:11-18).
int rows_of(const View& v) {
    if (v.num_dims < 2) return 1;
    int r = 1;
    for (int i = 0; i < v.num_dims - 1; ++i) r *= v.dims[i];
    return r;
}

int last_dim(const View& v) { return v.num_dims >= 1 ? v.dims[v.num_dims - 1] : 0; }

// A workspace per device that only grows; allocated on an eager call (the
// reference's own argmax scratch is allocated the same way).
struct DeviceWs {
    std::mutex mu;
    void* ptr = nullptr;
    size_t bytes = 0;
};
DeviceWs g_ws[af::kMaxDevices];

af_status workspace_for(size_t need, cudaStream_t stream, void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return af::cuda_fail(e, "cudaGetDevice");
    DeviceWs& w = g_ws[dev % af::kMaxDevices];
    std::lock_guard<std::mutex> lock(w.mu);
    if (w.bytes < need) {
        if (w.ptr != nullptr) {
            e = cudaStreamSynchronize(stream);
            if (e != cudaSuccess) return af::cuda_fail(e, "cudaStreamSynchronize");
            cudaFree(w.ptr);
            w.ptr = nullptr;
            w.bytes = 0;
        }
        const size_t bytes = af::round_up(need, 1 << 20);
        e = cudaMalloc(&w.ptr, bytes);
        if (e != cudaSuccess) return af::cuda_fail(e, "cudaMalloc(workspace)");
        e = cudaMemset(w.ptr, 0, bytes);
        if (e != cudaSuccess) return af::cuda_fail(e, "cudaMemset(workspace)");
        w.bytes = bytes;
    }
    *out = w.ptr;
    return AF_OK;
}

}  // namespace

extern "C" int af_view_last_status(void) { return g_last_status; }

static std::atomic<int> g_argmax_mode{AF_ARGMAX_REF_COMPAT};

extern "C" int af_view_set_argmax_mode(int mode) {
    if (mode != AF_ARGMAX_TRUE && mode != AF_ARGMAX_REF_COMPAT) return -1;
    return g_argmax_mode.exchange(mode);
}

void launch_w8a16_gemv(const View& act_x, const View& weight, const View& scales, View& output,
                       int group_size, cudaStream_t stream) {
    // Same shape source as the reference launcher (qkv_gemm.cu:137-139): N and K
    // come from the weight View; M from the activation's leading dims.
    if (weight.num_dims != 2 || weight.dtype != DataType::FP8_E4M3 ||
        act_x.dtype != DataType::FP16 || scales.dtype != DataType::FP16 ||
        output.dtype != DataType::FP16) {
        report(AF_ERR_INVALID, "launch_w8a16_gemv");
        return;
    }
    const int N = weight.dims[0];
    const int K = weight.dims[1];
    const int M = rows_of(act_x);
    if (last_dim(act_x) != K || rows_of(output) != M || last_dim(output) != N) {
        report(AF_ERR_INVALID, "launch_w8a16_gemv");
        return;
    }
    if (M == 1 && group_size == 128 && af::chain_ok(act_x.data_ptr, weight.data_ptr, scales.data_ptr, K) &&
        af::aligned(output.data_ptr, 2)) {
        // the reference's decode GEMV: the exact chain kernel, bit-identical to
        // w8a16_gemv_kernel, so an engine linked against this library produces
        // the unmodified build's outputs
        af_chain_op op{};
        op.kind = AF_OP_GEMV;
        op.N = N;
        op.K = K;
        op.x = act_x.data_ptr;
        op.w = weight.data_ptr;
        op.scales = scales.data_ptr;
        op.y = output.data_ptr;
        report(af::chain_launch(&op, 1, nullptr, 0, stream, true, true), "launch_w8a16_gemv");
        return;
    }
    void* ws = nullptr;
    af_status st = workspace_for(af_w8a16_gemv_workspace_bytes(M, N, K, AF_SCALE_GROUP_F16),
                                 stream, &ws);
    if (st == AF_OK) {
        st = af_w8a16_gemv(act_x.data_ptr, weight.data_ptr, scales.data_ptr, output.data_ptr, M, N,
                           K, group_size, AF_SCALE_GROUP_F16, ws,
                           af_w8a16_gemv_workspace_bytes(M, N, K, AF_SCALE_GROUP_F16), stream);
    }
    report(st, "launch_w8a16_gemv");
}

void launch_argmax(const View& logits, int* out_token_id, cudaStream_t stream) {
    // argmax.cu:93 takes V from the last dim.  The mode is the reference's
    // (ids < 65536) unless af_view_set_argmax_mode chose the true argmax.
    if (logits.dtype != DataType::FP32) {
        report(AF_ERR_INVALID, "launch_argmax");
        return;
    }
    const int V = last_dim(logits);
    void* ws = nullptr;
    const size_t need = af_argmax_workspace_bytes(V);
    af_status st = workspace_for(need, stream, &ws);
    if (st == AF_OK)
        st = af_argmax_f32(static_cast<const float*>(logits.data_ptr), V, out_token_id,
                           static_cast<af_argmax_mode>(g_argmax_mode.load()), ws, need, stream);
    report(st, "launch_argmax");
}

void launch_linear_gemm(const View& input, const View& weight, View& output, cublasHandle_t,
                        cudaStream_t stream) {
    // qkv_gemm.cu:156-181: FP8 weight [N, K] x FP16 input [M, K] -> FP16 [M, N], no scales.
    if (weight.num_dims != 2 || weight.dtype != DataType::FP8_E4M3 ||
        input.dtype != DataType::FP16 || output.dtype != DataType::FP16) {
        report(AF_ERR_INVALID, "launch_linear_gemm");
        return;
    }
    const int N = weight.dims[0];
    const int K = weight.dims[1];
    const int M = rows_of(input);
    if (last_dim(input) != K || rows_of(output) != M || last_dim(output) != N) {
        report(AF_ERR_INVALID, "launch_linear_gemm");
        return;
    }
    void* ws = nullptr;
    const size_t need = af_w8a16_gemv_workspace_bytes(M, N, K, AF_SCALE_NONE);
    af_status st = workspace_for(need, stream, &ws);
    if (st == AF_OK)
        st = af_w8a16_gemv(input.data_ptr, weight.data_ptr, nullptr, output.data_ptr, M, N, K, 128,
                           AF_SCALE_NONE, ws, need, stream);
    report(st, "launch_linear_gemm");
}
