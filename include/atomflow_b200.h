/*
 * atomflow_b200.h -- C ABI of the B200 (sm_100a) W8A16 decode hot path.
 *
 * Plain pointers and sizes only.  Every device pointer is owned by the caller;
 * no entry point allocates device memory.  Every entry point is asynchronous
 * on `stream` (a cudaStream_t passed as void*, NULL = legacy default stream)
 * and safe to record under CUDA stream capture once the library has run one
 * eager call on the device (the first call sets per-kernel attributes).
 *
 * Reference interfaces replaced (paths relative to the AtomFlow source tree):
 *   af_w8a16_gemv    <- launch_w8a16_gemv   include/ops/kernel.h:138-145,
 *                       src/kernel/qkv_gemm.cu:129-150 (kernel :32-111)
 *   af_lm_head_gemv  <- the inline cublasGemmEx vocab projection
 *                       src/core/engine.cu:494-513, fused with the argmax
 *                       launch at src/core/engine.cu:521
 *   af_argmax_f32    <- launch_argmax       include/ops/kernel.h:155-159,
 *                       src/kernel/argmax.cu:92-119
 * The View-based C++ launchers with the reference's exact signatures are in
 * atomflow_view_ops.h and forward to these functions.
 */
#ifndef ATOMFLOW_B200_H
#define ATOMFLOW_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum af_status {
    AF_OK = 0,
    AF_ERR_INVALID = 1,       /* bad shape, dtype, pointer or alignment */
    AF_ERR_UNSUPPORTED = 2,   /* valid request this build does not implement */
    AF_ERR_PEER_TIMEOUT = 3,  /* a bounded wait on another rank gave up */
    AF_ERR_CUDA = 4,          /* a CUDA runtime call failed (see af_last_cuda_error) */
    AF_ERR_WORKSPACE = 5      /* workspace NULL or smaller than *_workspace_bytes() */
} af_status;

/* How the FP8 weight rows are scaled. */
typedef enum af_scale_kind {
    AF_SCALE_GROUP_F16 = 0,   /* FP16 scales [N, K/group_size], group_size == 128 (reference format) */
    AF_SCALE_ROW_F32 = 1,     /* FP32 scale per output row [N] */
    AF_SCALE_NONE = 2         /* no scale (scale 1); `scales` must be NULL */
} af_scale_kind;

typedef enum af_weight_dtype {
    AF_W_F16 = 0,             /* FP16 weights (the reference lm_head) */
    AF_W_FP8_E4M3 = 1         /* FP8-E4M3 weights (OCP E4M3, max 448) */
} af_weight_dtype;

typedef enum af_argmax_mode {
    AF_ARGMAX_TRUE = 0,       /* index of the largest logit, ties -> lowest index, NaN ignored */
    AF_ARGMAX_REF_COMPAT = 1  /* the reference's result: only ids < 65536 are candidates */
} af_argmax_mode;

/* Fault bits a kernel records on its device instead of faulting the GPU. */
typedef enum af_fault_bits {
    AF_FAULT_X_COPY = 1,      /* a GEMV's bounded wait for its x copy ran out (that y is invalid) */
    AF_FAULT_POSITION = 2,    /* a decode kernel read a position outside [0, max_seq) and skipped its work */
    AF_FAULT_CHAIN_WAIT = 4,  /* a projection chain's bounded wait ran out (that launch's outputs are invalid) */
    AF_FAULT_TC_WAIT = 8      /* an af_w8a16_gemm_tc bounded wait ran out (its outputs are invalid) */
} af_fault_bits;

const char* af_status_string(af_status s);
/* The AF_FAULT_* bits recorded on the current device since the last clear (0:
 * none); clear != 0 resets them.  Synchronous (reads device memory), so call it
 * outside stream capture, e.g. after a run of graph replays. */
af_status af_device_faults(unsigned* out, int clear);
/* Error string of the last CUDA failure seen by this library on this thread. */
const char* af_last_cuda_error(void);
int af_version(void);

/* Zero-fills a workspace.  Required once before its first use: every kernel
 * returns all the workspace bytes it touched to zero before it exits (unless a
 * bounded wait gave up -- then word 0 holds a non-zero error code), so one
 * workspace serves any sequence of calls, ops and shapes, graph replays
 * included, provided the calls cannot overlap on the GPU (same stream). */
af_status af_workspace_reset(void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- GEMV ---
 * y[m, n] = sum_k dequant(W[n, k]) * x[m, k]   for m < M, n < N
 *   x : FP16 [M, K] row-major          w : FP8-E4M3 [N, K] row-major
 *   y : FP16 [M, N] row-major          scales: see af_scale_kind
 * FP32 accumulation, FP16 round-to-nearest output.  M = 1 is the decode
 * case of the reference; 1 <= M <= 16 runs in one pass over W, larger M in
 * ceil(M/16) passes (tensor-core math, within FP16 rounding of FP64; the
 * bit-identical form of the reference kernel is af_gemv_chain, and the View
 * launcher launch_w8a16_gemv uses it).  Returns AF_ERR_INVALID for group_size != 128 with
 * AF_SCALE_GROUP_F16, or K % 128 != 0 with group scales (the reference kernel
 * hard-codes 128-wide groups, qkv_gemm.cu:70). */
size_t af_w8a16_gemv_workspace_bytes(int M, int N, int K, af_scale_kind kind);
af_status af_w8a16_gemv(const void* x, const void* w, const void* scales, void* y,
                        int M, int N, int K, int group_size, af_scale_kind kind,
                        void* workspace, size_t workspace_bytes, void* stream);
/* The same projection for any M on the tcgen05 tensor cores (the batched /
 * prefill shape that launch_linear_gemm declares, include/ops/kernel.h:53-59,
 * with the reference's scales; its kernel is single-token only,
 * src/kernel/qkv_gemm.cu:32-150).  128 weight rows form the MMA's M and 16
 * tokens its N; FP8 is widened to FP16 in shared memory and each K=16 MMA
 * accumulates from zero in its own TMEM block, the group scale applied to each
 * 128-position partial sum; the CTAs that split one row tile's K form a
 * thread-block cluster and merge in distributed shared memory (no workspace,
 * no allocation).  FP8 group (group_size 128) or FP32 row scales, K % 128 == 0,
 * 16-byte aligned x and w.  Within FP16 rounding of FP64, deterministic.  Its
 * throughput is bounded by the FP8 -> FP16 widening (about 1 TB/s at M = 8 to
 * 16), below af_w8a16_gemv's tokens-in-MMA-columns path, which therefore stays
 * the default. */
af_status af_w8a16_gemm_tc(const void* x, const void* w, const void* scales, void* y, int M, int N, int K,
                           int group_size, af_scale_kind kind, void* stream);

/* ------------------------------------------------------------ lm_head ---
 * logits[v] = sum_d W[v, d] * x[d]  (FP32 out, one token), optionally
 * followed by a fused greedy argmax written to *d_argmax (device int).
 *   w_dtype AF_W_F16      : W FP16 [V, D], row_scale must be NULL
 *   w_dtype AF_W_FP8_E4M3 : W FP8 [V, D], row_scale FP32 [V]
 * `logits` may be NULL when only the argmax is wanted; d_argmax may be NULL. */
size_t af_lm_head_workspace_bytes(int V, int D, af_weight_dtype w_dtype);
af_status af_lm_head_gemv(const void* x, const void* w, af_weight_dtype w_dtype,
                          const float* row_scale, float* logits, int V, int D,
                          int* d_argmax, af_argmax_mode mode,
                          void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------- argmax ---
 * *d_out = argmax(logits[0:V]) (FP32), single launch. */
size_t af_argmax_workspace_bytes(int V);
af_status af_argmax_f32(const float* logits, int V, int* d_out, af_argmax_mode mode,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------ tensor parallelism (NVLink) ---
 * Row-parallel projections (O, down) of Megatron tensor parallelism: each of
 * `world` ranks (one process or one device each) holds a K-shard of W and x
 * and needs y = sum over ranks of W_r x_r.  af_w8a16_gemv_allreduce computes
 * its shard and sums across ranks in the same kernel: every CTA stores its
 * rows' FP32 partials, tagged with the launch epoch, straight into each
 * peer's exchange buffer over NVLink, polls (bounded) until every rank's
 * words for its rows carry that epoch, and sums in rank order (deterministic,
 * identical on every rank).  No counterpart in the reference (it is
 * single-GPU); this replaces GEMV + NCCL all-reduce.
 *
 * Setup is collective: every rank calls af_tp_create, exports its buffer with
 * af_tp_ipc_handle (64 bytes), exchanges the handles by any transport, and
 * calls af_tp_open_peers with all `world` handles in rank order.  A process
 * that drives several GPUs itself can instead call af_tp_set_peer with device
 * pointers it can reach (peer access enabled).  All ranks must issue the same
 * sequence of allreduce calls; a wait that runs out (default 2 s,
 * af_tp_set_wait_limit_ms) sets bit 0 of the status word that af_tp_status
 * reads, and the kernel finishes with undefined y instead of hanging. */
typedef struct af_tp_comm af_tp_comm;
af_status af_tp_create(int rank, int world, int max_n, af_tp_comm** out);
af_status af_tp_ipc_handle(const af_tp_comm* comm, void* handle64);
af_status af_tp_open_peers(af_tp_comm* comm, const void* handles /* world x 64 bytes */);
af_status af_tp_set_peer(af_tp_comm* comm, int peer_rank, void* peer_buffer);
size_t af_tp_buffer_bytes(int max_n);
void* af_tp_buffer(const af_tp_comm* comm);
af_status af_tp_set_wait_limit_ms(af_tp_comm* comm, int ms);
af_status af_tp_status(const af_tp_comm* comm, int* status);   /* synchronous read */
af_status af_tp_destroy(af_tp_comm* comm);
/* One token (M = 1), FP8 weights, K % 128 == 0, x 16-byte aligned, N <= max_n. */
af_status af_w8a16_gemv_allreduce(const void* x, const void* w, const void* scales, void* y, int N, int K,
                                  int group_size, af_scale_kind kind, af_tp_comm* comm, void* stream);
/* Vocab-parallel lm_head + greedy argmax: rank r holds rows [vocab_offset,
 * vocab_offset + V_local) of the lm_head weight (any split; offsets
 * increasing with rank).  Each rank projects its rows (local logits to
 * `logits` when not NULL) and takes its local argmax; the last CTA pushes the
 * (max, global index) pair to every rank and reduces all ranks' pairs, so
 * *d_argmax (device int, required) holds the same global token on every
 * rank, ties to the lowest index.  AF_ARGMAX_REF_COMPAT limits candidates to
 * global ids < 65536.  Same weight formats as af_lm_head_gemv; one-token
 * kernel only (16-byte aligned x and W, D % 128 == 0 for FP8, D % 64 for FP16). */
af_status af_lm_head_gemv_tp(const void* x, const void* w, af_weight_dtype w_dtype, const float* row_scale,
                             float* logits, int V_local, int D, int vocab_offset, int* d_argmax,
                             af_argmax_mode mode, void* workspace, size_t workspace_bytes, af_tp_comm* comm,
                             void* stream);

/* ------------------------------------------------ fused decode-layer ops ---
 * The reference runs RMSNorm, GEMV, SwiGLU and residual add as separate
 * kernels (src/core/engine.cu:292-483; src/kernel/rmsnorm.cu, swiglu.cu,
 * residual_add.cu).  These fold the element-wise work into the one-token
 * GEMV, with the reference's rounding points kept (the normalised x, gate and
 * up, and the GEMV output are rounded to FP16 where the reference stores them):
 *   af_rmsnorm_w8a16_gemv    y = W . half(rmsnorm(x) * norm_w)     (QKV)
 *   af_w8a16_gemv_residual   inout = half(inout + half(W . x))     (O, down)
 *   af_rmsnorm_w8a16_swiglu  h = half(silu(half(Wg . xn)) * half(Wu . xn)),
 *                            xn = rmsnorm(x) (norm_w NULL: xn = x) (gate/up)
 * RMSNorm: r = 1 / sqrt(sum(x^2) / K + eps), xn = half(x * r * norm_w), norm_w
 * FP32 [K] 16-byte aligned.  Optional outputs for checking each stage:
 * x_norm_out FP16 [K], y_out FP16 [N] (before the residual), gate_up_out FP16
 * [2N] (gate then up).  One token, FP8 weights, K % 128 == 0, x and W 16-byte
 * aligned (else AF_ERR_UNSUPPORTED); SwiGLU needs FP16 group scales. */
af_status af_rmsnorm_w8a16_gemv(const void* x, const float* norm_w, float eps, const void* w, const void* scales,
                                void* y, int N, int K, int group_size, af_scale_kind kind, void* x_norm_out,
                                void* stream);
af_status af_w8a16_gemv_residual(const void* x, const void* w, const void* scales, void* inout, int N, int K,
                                 int group_size, af_scale_kind kind, void* y_out, void* stream);
af_status af_rmsnorm_w8a16_swiglu(const void* x, const float* norm_w, float eps, const void* w_gate,
                                  const void* s_gate, const void* w_up, const void* s_up, void* h, int N, int K,
                                  int group_size, af_scale_kind kind, void* gate_up_out, void* x_norm_out,
                                  void* stream);
/* Row-parallel projection + all-reduce + residual in one kernel:
 * inout = half(inout + half(sum over ranks of W_r x_r)). */
af_status af_w8a16_gemv_allreduce_residual(const void* x, const void* w, const void* scales, void* inout, int N,
                                           int K, int group_size, af_scale_kind kind, af_tp_comm* comm,
                                           void* stream);

/* ------------------------------------------------- rest of a decode step ---
 * With these and the projections above, a whole greedy decode step (embedding
 * .. argmax) runs on device-side state -- the token id and the position live
 * in device ints -- so consecutive steps replay one captured CUDA graph.
 * Layouts are the reference engine's: qkv FP16 [NH*HD | NKV*HD | NKV*HD]
 * (engine.cu:315), caches FP16 [max_seq, NKV*HD] per layer (engine.cu:196-209),
 * RoPE tables FP32 [max_seq, HD/2].
 *   af_embed_lookup      x = half(table[*d_token])      (helpers.cu k_embed_lookup_kernel)
 *   af_rope_tables       host: cos/sin tables, the reference's float formula
 *                        (helpers.cu build_rope_cache), base 500000 for Llama 3
 *   af_rope_kv_write     rotate q and k in qkv at *d_pos, write k and v to row
 *                        *d_pos of the caches (rope.cu; helpers.cu k_write_kv_cache)
 *   af_decode_attention  softmax(q k^T / sqrt(HD)) v over positions 0..*d_pos,
 *                        GQA (NH % NKV == 0, NH/NKV <= 8), HD = 128; bit-identical
 *                        to the reference's gqa_cached_attention_kernel
 *                        (tiled_attention.cu:196-269).  Workspace:
 *                        af_decode_attention_workspace_bytes(NH, NKV, max_seq),
 *                        zeroed once (af_workspace_reset), one per stream; every
 *                        call leaves its counters at zero.
 *   af_rmsnorm           the reference's rms_norm arithmetic, one vector
 *   af_decode_advance    *d_pos += by (the step's last launch)
 * max_seq is the caches' and tables' row count: a kernel that reads *d_pos
 * outside [0, max_seq) writes and reads nothing, leaves its outputs as they
 * were and sets AF_FAULT_POSITION (af_device_faults).
 */
af_status af_embed_lookup(const float* table, const int* d_token, void* x, int D, void* stream);
af_status af_rope_tables(float* cos_out, float* sin_out, int max_seq, int head_dim, float base);
af_status af_rope_kv_write(void* qkv, const float* cos_tab, const float* sin_tab, const int* d_pos, void* k_cache,
                           void* v_cache, int n_heads, int n_kv_heads, int head_dim, int max_seq, void* stream);
size_t af_decode_attention_workspace_bytes(int n_heads, int n_kv_heads, int max_seq);
af_status af_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int* d_pos, void* out,
                              int n_heads, int n_kv_heads, int head_dim, int max_seq, void* workspace,
                              size_t workspace_bytes, void* stream);
/* RoPE + KV-cache write + attention in one launch: q, k, v read from the raw qkv vector; the same
 * results, bit for bit, as af_rope_kv_write followed by af_decode_attention (qkv itself is left
 * unrotated). */
af_status af_decode_rope_attention(void* qkv, const float* cos_tab, const float* sin_tab, const int* d_pos,
                                   void* k_cache, void* v_cache, void* out, int n_heads, int n_kv_heads,
                                   int head_dim, int max_seq, void* workspace, size_t workspace_bytes, void* stream);
/* The same step as af_decode_rope_attention with an online softmax split over
 * one 8-CTA thread-block cluster per kv head (partials merged in distributed
 * shared memory): the KV-cache rows written are bit-identical, every output is
 * within 2 FP16 ulp / 2e-3 relative of FP64, not the reference's summation
 * order.  A fast form for throughput; it uses no workspace (the arguments are
 * accepted and ignored). */
af_status af_decode_rope_attention_fast(void* qkv, const float* cos_tab, const float* sin_tab, const int* d_pos,
                                        void* k_cache, void* v_cache, void* out, int n_heads, int n_kv_heads,
                                        int head_dim, int max_seq, void* workspace, size_t workspace_bytes,
                                        void* stream);
af_status af_rmsnorm(const void* x, const float* norm_w, float eps, void* out, int K, void* stream);
af_status af_decode_advance(int* d_pos, int by, void* stream);

/* ---------------------------------------------------- projection chains ---
 * A sequence of one-token FP8 projections -- a decode layer's, or a whole
 * step's -- in ONE persistent launch (one CTA per SM).  Outputs are
 * bit-identical to the reference's w8a16_gemv_kernel (src/kernel/qkv_gemm.cu:
 * 32-111: its per-thread FMA chains, shuffle tree and warp-order sum are
 * reproduced exactly) followed by its element-wise kernels (rmsnorm.cu,
 * swiglu.cu, residual_add.cu), so a chain computes what the reference's
 * engine.cu:292-483 computes, without the kernel boundaries: while op i
 * waits for op i-1's output, the weights of op i are already streaming.
 *   AF_OP_GEMV           y = half(W x)
 *   AF_OP_GEMV_RESIDUAL  y = half(y + half(W x))                       (O, down)
 *   AF_OP_RMSNORM_GEMV   xn = half(x * r * norm_w), y = half(W xn)       (QKV)
 *   AF_OP_RMSNORM_SWIGLU y = half(silu(half(W xn)) * half(W2 xn))        (gate/up)
 *     r = 1 / sqrt(sum(x^2) / K + eps) in the reference's arithmetic.
 * Each op: FP8-E4M3 W [N, K] with FP16 group scales [N, K/128]; x FP16 [K];
 * y FP16 [N]; K % 128 == 0, K <= 16384; x, W (and W2) 16-byte aligned, scales
 * and y 2-byte aligned, norm_w FP32 [K] 4-byte aligned, xn_out and aux
 * (optional stage outputs, for checking) 2-byte aligned.  wait_prev != 0: the op
 * reads data an earlier op of the chain writes, so it starts only when every
 * CTA has finished the previous op (a device-side counter; ops before it
 * complete first).  x may alias an earlier op's y; y of a residual op is read
 * and written in place.  At most 320 ops per call.
 * Workspace: af_chain_workspace_bytes(n_ops) bytes, zeroed once
 * (af_workspace_reset) and left zeroed by every launch; needed only when some
 * op waits (else NULL).  Calls sharing a workspace must not overlap on the GPU.
 * Every wait is bounded: AF_FAULT_CHAIN_WAIT (af_device_faults) marks a launch
 * whose outputs are invalid. */
typedef enum af_op_kind {
    AF_OP_GEMV = 0,
    AF_OP_GEMV_RESIDUAL = 1,
    AF_OP_RMSNORM_GEMV = 2,
    AF_OP_RMSNORM_SWIGLU = 3
} af_op_kind;
typedef struct af_chain_op {
    int kind;                 /* af_op_kind */
    int N, K;
    int wait_prev;
    const void* x;
    const void* w;
    const void* scales;
    const void* w2;           /* SwiGLU: the up projection's weights and scales */
    const void* scales2;
    const float* norm_w;      /* RMSNorm ops */
    float eps;
    void* y;
    void* xn_out;             /* RMSNorm ops, optional: the normalised x FP16 [K] */
    void* aux;                /* optional: residual op: half(W x) [N] before the add;
                                 SwiGLU: half(gate) [N] then half(up) [N] */
} af_chain_op;
size_t af_chain_workspace_bytes(int n_ops);
af_status af_gemv_chain(const af_chain_op* ops, int n_ops, void* workspace, size_t workspace_bytes, void* stream);
/* The same chain with the dot products on the tensor cores (FP8 -> FP16
 * packed conversion, m16n8k16 MMAs, FP32 accumulation, the group scale applied
 * to each 128-position group sum): deterministic, every output within 2 FP16
 * ulp / 2e-3 relative of FP64 (the reference kernel's own tolerance), but not
 * its summation order, so not bit-identical to it.  Same arguments. */
af_status af_gemv_chain_fast(const af_chain_op* ops, int n_ops, void* workspace, size_t workspace_bytes,
                             void* stream);

/* -------------------------------------------------------- decode engine ---
 * A whole greedy decode step of a model in the reference's .bin format
 * (tools/quantize_weights.py:320-427; read as include/memory/weight_loader.h
 * and src/core/engine.cu:103-147 read it), driven from C++ with no Python:
 * the interface of the reference's AtomFlowEngine (include/core/engine.h:
 * initialize / inject_token / forward_pass / get_output_token / current_pos_),
 * with the token id and the position kept in device ints so that a captured
 * step replays token after token.  The engine is the one part of this library
 * that allocates device memory: at create, its weight arena (the file, copied
 * once), KV cache, activations and workspaces -- as the reference engine's
 * initialize does (engine.cu:56-234); nothing allocates afterwards.
 *   AF_ENGINE_EXACT  every kernel bit-identical to the reference's: projection
 *                    chains (af_gemv_chain), attention, norms, SwiGLU,
 *                    residual, RoPE, embedding; lm_head + argmax as
 *                    af_lm_head_gemv (the reference's is a cuBLAS call)
 *   AF_ENGINE_FAST   the fused tensor-core projections and the cluster
 *                    attention (af_decode_rope_attention_fast)
 * argmax_mode: AF_ARGMAX_REF_COMPAT (the reference's ids < 65536) or TRUE.
 * One engine per host thread at a time; calls are ordered on its stream. */
typedef struct af_engine af_engine;
typedef enum af_engine_mode { AF_ENGINE_EXACT = 0, AF_ENGINE_FAST = 1 } af_engine_mode;
af_status af_engine_create(const char* bin_path, int max_seq, af_engine_mode mode, af_argmax_mode argmax_mode,
                           af_engine** out);
af_status af_engine_destroy(af_engine* e);
/* Tensor-parallel engine: rank comm->rank of comm->world (af_tp_create /
 * af_tp_open_peers, max_n >= dim), one process per GPU with that GPU current.
 * Megatron split: QKV by heads, gate/up by rows, O and down along K with the
 * partial outputs summed over the ranks inside the projection kernel over
 * NVLink peer memory (af_w8a16_gemv_allreduce_residual), the lm_head by
 * vocabulary rows with the argmax exchanged in its kernel (af_lm_head_gemv_tp):
 * every rank ends the step with the same token.  Fast mode only (a sum split
 * over ranks cannot keep the reference's summation order). */
af_status af_engine_create_tp(const char* bin_path, int max_seq, af_argmax_mode argmax_mode, af_tp_comm* comm,
                              af_engine** out);
/* dims[9]: dim, ffn, layers, heads, kv heads, vocab, max_seq, launches per step (without the
 * position advance), file size in MiB. */
af_status af_engine_info(const af_engine* e, int* dims);
af_status af_engine_set_position(af_engine* e, int pos);
af_status af_engine_get_position(af_engine* e, int* pos);
af_status af_engine_inject_token(af_engine* e, int token);
af_status af_engine_output_token(af_engine* e, int* token);
/* One step launched eagerly (advance != 0: then *d_pos += 1 on the device). */
af_status af_engine_step(af_engine* e, int advance);
/* Captures one step (advance != 0: with the position increment) as a CUDA graph
 * owned by the engine (replacing any earlier one); the first eager step must
 * have run.  af_engine_replay launches it n times on the engine's stream. */
af_status af_engine_capture(af_engine* e, int advance);
af_status af_engine_replay(af_engine* e, int n);
af_status af_engine_synchronize(af_engine* e);
/* The engine's stream (cudaStream_t), device token / position ints, FP32 logits [vocab]. */
void* af_engine_stream(af_engine* e);
int* af_engine_device_token(af_engine* e);
int* af_engine_device_position(af_engine* e);
const float* af_engine_logits(af_engine* e);

/* ----------------------------------------------- argmax, no allocation ---
 * No counterpart in the reference.  The same argmax as af_argmax_f32 for
 * callers that cannot allocate device memory (no cudaMalloc available or
 * allowed, so no workspace to pass): its scratch is a fixed ~2.3 KB block
 * inside the library, resident on every GPU that loads it until exit.
 *   - V above 268,435,456 (1 << 28) returns AF_ERR_UNSUPPORTED, launching nothing.
 *   - The first call on a device looks up that block's device address; make it
 *     before any stream capture.
 *   - All calls share the block: calls that may overlap on the GPU race.
 * It allocates nothing and calls no allocating routine. */
af_status af_argmax_f32_noalloc(const float* logits, int V, int* d_out, af_argmax_mode mode, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ATOMFLOW_B200_H */
