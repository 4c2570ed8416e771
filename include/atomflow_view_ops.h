/*
 * atomflow_view_ops.h -- the reference's View-based operator launchers,
 * re-implemented on the B200 kernels of atomflow_b200.h.
 *
 * These are C++ symbols, not C: their names and parameter types must mangle
 * exactly like the declarations in the reference's include/ops/kernel.h so
 * that the reference engine (src/core/engine.cu) links against this library
 * in place of src/kernel/qkv_gemm.cu and src/kernel/argmax.cu without a
 * source change.  `View`/`DataType` below therefore keep the reference
 * layout of include/core/view.h:15-39 (56 bytes: dtype @0, data_ptr @8,
 * dims @16, strides @32, num_dims @48); the static_asserts in the shim pin it.
 * A translation unit that already includes the reference's core/view.h must
 * define AF_HAVE_REFERENCE_VIEW before including this header.
 *
 * Error behaviour: the reference launchers return void and abort only in
 * debug builds (include/utils/utils.h:95-116).  These launchers validate
 * their arguments, record a sticky status readable through
 * af_view_last_status(), print a one-line diagnostic to stderr, and launch
 * nothing on failure.  Defining AF_VIEW_ABORT=1 in the environment makes a
 * failure abort like the reference's debug build.
 *
 * Scratch memory: the reference lazily cudaMallocs argmax scratch on first
 * use (src/kernel/argmax.cu:98-103).  These launchers do the same for their
 * split-K and argmax workspaces, so the first call on a device (made eagerly,
 * as the reference's warm-up does before graph capture, src/main.cu:67-73)
 * must precede any stream capture.
 */
#ifndef ATOMFLOW_VIEW_OPS_H
#define ATOMFLOW_VIEW_OPS_H

#include <cstdint>
#include <cstddef>

struct CUstream_st;
typedef CUstream_st* cudaStream_t;
struct cublasContext;
typedef cublasContext* cublasHandle_t;

#ifndef AF_HAVE_REFERENCE_VIEW
enum class DataType { FP32, FP16, BF16, FP8_E4M3 };
struct View {
    DataType dtype;
    void* data_ptr;
    int32_t dims[4];
    int32_t strides[4];
    int8_t num_dims;
};
#endif

/* include/ops/kernel.h:138-145 -- W8A16 GEMV.  act_x FP16 [M, K] (M from the
 * leading dims, as calculate_rows, kernel.h:11-18), weight FP8 [N, K], scales
 * FP16 [N, K/group_size], output FP16 [M, N].  One token (the reference's
 * case) is bit-identical to the reference's w8a16_gemv_kernel. */
void launch_w8a16_gemv(const View& act_x, const View& weight, const View& scales,
                       View& output, int group_size, cudaStream_t stream);

/* include/ops/kernel.h:155-159 -- greedy argmax of FP32 logits [.., V].
 * By default it gives the reference launcher's result: only ids below 65,536
 * are candidates (src/kernel/argmax.cu:72-73, 115-117 read 256 of the 501
 * per-block partials), so an engine linked against this library emits the same
 * tokens as the unmodified build.  af_view_set_argmax_mode(AF_ARGMAX_TRUE = 0)
 * switches this process to the true argmax over all V ids. */
void launch_argmax(const View& logits, int* out_token_id, cudaStream_t stream);

/* include/ops/kernel.h:53-59 -- FP8 weight x FP16 activation linear layer
 * without scales (the reference declares it; its engine never calls it).
 * The cuBLAS handle is accepted and ignored. */
void launch_linear_gemm(const View& input, const View& weight, View& output,
                        cublasHandle_t handle, cudaStream_t stream);

extern "C" int af_view_last_status(void);
/* Mode of launch_argmax for the whole process: 1 (AF_ARGMAX_REF_COMPAT, the
 * default) or 0 (AF_ARGMAX_TRUE).  Returns the previous mode, or -1 for an
 * unknown mode (nothing changes). */
extern "C" int af_view_set_argmax_mode(int mode);

#endif /* ATOMFLOW_VIEW_OPS_H */
