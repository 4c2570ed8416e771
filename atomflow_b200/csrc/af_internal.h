// af_internal.h -- host-side plumbing shared by the launchers (not installed).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "../../include/atomflow_b200.h"

namespace af {

constexpr int kMaxDevices = 64;

// Streaming multiprocessors of the current device (cached per device).
int device_sm_count(int* device_out = nullptr);

// Record a CUDA failure for af_last_cuda_error() and map it to AF_ERR_CUDA.
af_status cuda_fail(cudaError_t e, const char* where);

// CTAs launched per SM by the streaming kernels.
constexpr int ctas_per_sm() { return 1; }

// Fault bits recorded on the current device by the GEMV (af_gemv.cu) and
// decode-step (af_decode.cu) kernels; `clear` resets them.  Synchronous.
unsigned gemv_faults(bool clear, cudaError_t* err);
unsigned decode_faults(bool clear, cudaError_t* err);
unsigned chain_faults(bool clear, cudaError_t* err);
unsigned tc_faults(bool clear, cudaError_t* err);
// 8+ token FP8 projections on the tcgen05 tensor cores (af_gemv_tc.cu)
bool tc_ok(int M, int K, bool row_scale, const void* x, const void* w, const void* s, const void* y);
af_status tc_launch(const void* x, const void* w, const void* s, bool row_scale, void* y, int M, int N, int K,
                    cudaStream_t st);


inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// The persistent projection-chain kernel (af_chain.cu).  `single`: a one-op
// call (shallower ring, two CTAs per SM, programmatic dependent launch).
constexpr int kChainMaxK = 16384;
af_status chain_launch(const af_chain_op* ops, int n_ops, void* workspace, size_t ws_bytes, cudaStream_t st,
                       bool single, bool exact);
inline bool chain_ok(const void* x, const void* w, const void* s, int K) {
    return K > 0 && K % 128 == 0 && K <= kChainMaxK && x != nullptr && w != nullptr && s != nullptr &&
           aligned(x, 16) && aligned(w, 16) && aligned(s, 2);
}

// Launch `kernel` with programmatic stream serialization, so it may begin
// while the previous kernel of the stream drains; the kernel itself calls
// griddepcontrol.wait before touching data that kernel may have written.
template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace af

// ---- tensor-parallel all-reduce state (af_tp.cu) ----
namespace af {
constexpr int kTpMaxRanks = 8;
constexpr int kTpMaxCtas = 256;

// One rank's exchange buffer; every rank's buffer has the same layout and
// size, and each rank maps all of them (CUDA IPC or same-process pointers):
//   [0, 256)            status word (bit 0: a bounded wait gave up) at 0; lm_head
//                       argmax exchange epoch at 4
//   [256, +1 KB)        unused
//   [1280, +256)        lm_head argmax pairs [epoch parity][source rank] as two
//                       64-bit words {epoch, FP32 max} {epoch, global index}
//   [.., +2*8*nmax*8)   partials [epoch parity][source rank][nmax], each a 64-bit
//                       word {launch epoch : 32, FP32 bits : 32}: the data carries
//                       its own flag, so a reader polls the word itself and no
//                       fence or separate flag store is needed
//   [.., +nmax*4)       per-row epoch of this rank: how many all-reduces row r
//                       has taken part in.  Keyed by row, not by CTA, so the tag
//                       of a row alternates parity on every launch that touches
//                       it whatever grid each launch uses
struct TpLayout {
    static constexpr size_t status = 0;
    static constexpr size_t lm_epoch = 4;
    static constexpr size_t lm_pair = 256 + kTpMaxCtas * 4;
    static constexpr size_t part = lm_pair + 2 * kTpMaxRanks * 16;
    __host__ __device__ static size_t row_epoch(int nmax) { return part + (size_t)2 * kTpMaxRanks * nmax * 8; }
    __host__ __device__ static size_t bytes(int nmax) { return row_epoch(nmax) + (((size_t)nmax * 4 + 15) & ~(size_t)15); }
};
}  // namespace af

struct af_tp_comm {
    int rank, world, nmax, device;
    unsigned char* buf;                       // this rank's buffer (owned)
    unsigned char* peer[af::kTpMaxRanks];     // every rank's buffer as mapped here
    bool ipc_opened[af::kTpMaxRanks];
    unsigned long long wait_ns;
};
