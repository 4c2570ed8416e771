// af_gemv.cu -- streaming W8A16 GEMV and lm_head vocab projection for sm_100a.
//
// Reference behaviour (AtomFlow):
//   src/kernel/qkv_gemm.cu:32-111  w8a16_gemv_kernel: y[n] = sum_k fp8(W[n,k]) *
//                                  half(S[n,k/128]) * x[k], FP32 accumulate, FP16 out
//   src/kernel/qkv_gemm.cu:129-150 launch_w8a16_gemv (N, K from weight.dims)
//   src/core/engine.cu:494-513     lm_head: cublasGemmEx FP16 W[V,D] x FP16 x[D] -> FP32 logits
//   src/kernel/argmax.cu:23-119    greedy argmax of the logits
//
// Design (one kernel family, three weight formats):
//   * One CTA per SM.  CTA i owns the rows [i*N/G, (i+1)*N/G): shares differ
//     by at most one row, so every SM streams the same number of bytes, and no
//     output row is split between CTAs (no cross-CTA reduction, no fences, no
//     device scratch).  A CTA's rows form 16-row tiles (the last one partial;
//     rows past the share are neither loaded nor stored), and each tile's K
//     range is cut into "chunks" of 64 FP8 / 32 FP16 positions (64 B per row).
//   * The CTA's tiles x chunks list is split into equal contiguous ranges, one
//     per warp.  A lane streams exactly the bytes it consumes -- 16 B of each
//     of two rows (g, g+8) per chunk -- with 16-byte asynchronous copies
//     (cp.async, L2 only) into its own places of a 10-chunk shared-memory ring
//     (160 KB per SM in flight), one commit group per chunk; the CTA's group
//     scales are staged the same way.  No lane reads another lane's bytes, so
//     the ring needs no barriers.  The ring is filled before
//     griddepcontrol.wait: with programmatic dependent launch a config-sized
//     GEMV's whole weight share is requested while the previous kernel of the
//     stream drains, and the stream costs one DRAM round trip, not one per
//     batch.
//   * FP8 bytes become FP16 with the packed cvt (exact) and the dot products
//     run on the tensor cores as m16n8k16 MMAs: W rows are the MMA's M, tokens
//     its N (M = 1 uses one column; up to 16 tokens share one pass over W).
//     Every MMA starts from a zero accumulator and its result is added in FP32
//     registers, keeping cancellation error at the level of an FFMA chain.
//     The activations are staged once per CTA in shared memory.
//   * Group scales are applied to each 64-position chunk sum (a scale group
//     never straddles a chunk); row scales after the reduction.
//   * A tile whose chunks all fall in one warp's range is finished by that
//     warp; tiles split between warps are summed through shared memory after
//     the stream, in warp order -- results are deterministic.
//   * The lm_head variant writes FP32 logits and folds the greedy argmax into
//     the epilogue (per-CTA candidates in the caller's workspace, the last CTA
//     reduces them and returns the workspace to zero).

#include <algorithm>
#include <cuda_fp8.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "af_common.cuh"
#include "af_internal.h"

namespace af {

enum WKind { W_FP8_GROUP = 0, W_FP8_ROW = 1, W_F16 = 2 };

constexpr int kXsPad = 32;              // halves of padding per staged x row (bank spread)
constexpr size_t kSmemMax = 227 * 1024;

struct GemvParams {
    const uint8_t* w;
    const void* s;        // FP16 [N,G] group scales | FP32 [N] row scales | null
    const __half* x;      // [M, K]
    void* y;              // [M, N] FP16 or FP32 (null: no store)
    int M, N, K, G;
    int cpt;              // chunks per 16-row tile
    int xs_stride;        // staged x row stride in halves (0: read x from global)
    int xs_bytes;         // shared bytes reserved for x
    int sc_bytes;         // shared bytes reserved for staged group scales (0: read from L2)
    int y_f32;
    int* arg_out;         // fused argmax result (null: off)
    float* arg_val;       // [CTAs]
    int* arg_idx;         // [CTAs]
    int* arg_done;        // [1]
    int arg_limit;        // rows >= arg_limit are not argmax candidates
    int pre;              // one-token kernel: ring slots requested before griddepcontrol.wait
    // tensor-parallel all-reduce epilogue of the one-token kernel (tp_world <= 1: off)
    int tp_world, tp_rank, tp_nmax;
    // fused prologue / epilogues of the one-token kernel (all null: a plain GEMV)
    const float* norm_w;  // RMSNorm weight FP32 [K]: x is normalised in shared memory first
    float norm_eps;
    int gam_bytes;        // shared bytes reserved for the staged norm weight
    __half* xn_out;       // optional: the normalised x (CTA 0 writes it)
    const __half* res;    // residual FP16 [N]: y = half(res + half(Wx)) (may alias y)
    __half* aux;          // optional: residual mode -> half(Wx) [N]; gate/up mode -> [gate | up] FP16 [2N]
    const uint8_t* w2;    // gate/up mode: the up weights (p.w: gate), y = half(silu(gate) * up)
    const void* s2;       // gate/up mode: the up scales
    int tp_arg;           // 1: the exchange is the argmax pair (vocab-parallel lm_head), not the rows
    int arg_off;          // global index of this rank's row 0 (vocab-parallel lm_head)
    unsigned char* tp_buf[kTpMaxRanks];   // every rank's exchange buffer (TpLayout)
    unsigned long long tp_wait_ns;
};

__device__ __forceinline__ uint32_t u4w(const uint4& v, int t) {
    return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}


// Owner of chunk `c` of a range of `n` chunks split into `parts` equal
// contiguous pieces (parts <= n): the largest i with floor(i*n/parts) <= c.
__device__ __forceinline__ long long owner_of(long long c, long long n, long long parts) {
    return ((c + 1) * parts - 1) / n;
}

template <int WK, int NT, int kWarps, int kS>
__global__ void __launch_bounds__(kWarps * 32, 1) gemv_stream_kernel(const GemvParams p) {
    constexpr int kThreads = kWarps * 32;
    constexpr int POS = (WK == W_F16) ? 32 : 64;   // positions per chunk
    constexpr int LPOS = POS / 4;                  // positions per lane per row
    constexpr int ESZ = (WK == W_F16) ? 2 : 1;     // weight bytes per element
    constexpr int XU4 = LPOS / 8;                  // uint4 of x per lane per chunk
    constexpr int PF = 4 * NT;                     // partial floats per lane

    pdl_launch_dependents();
    extern __shared__ __align__(128) unsigned char smem[];
    // [ring: kWarps x kS chunk slots of 1 KB][x: xs_bytes][scales: sc_bytes][warp partials]
    unsigned char* ring = smem;
    __half* xs = reinterpret_cast<__half*>(smem + (size_t)kWarps * kS * 1024);
    unsigned char* scs = smem + (size_t)kWarps * kS * 1024 + p.xs_bytes;
    float* wslots = reinterpret_cast<float*>(scs + p.sc_bytes);   // [kWarps][2][32][PF]
    __shared__ float s_best_v[kWarps];
    __shared__ int s_best_i[kWarps];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int g = lane >> 2;
    const int c = lane & 3;
    // This CTA's rows [row0, row1): an equal share of N (shares differ by at
    // most one row), processed as 16-row tiles, the last one partial.
    const int G = gridDim.x;
    const int cta = blockIdx.x;
    const int row0 = (int)((long long)cta * p.N / G);
    const int row1 = (int)((long long)(cta + 1) * p.N / G);
    const int T = (row1 - row0 + 15) >> 4;
    const int L = T * p.cpt;                      // this CTA's chunks
    const int We = L < kWarps ? L : kWarps;       // warps that own chunks
    const int wc0 = warp < We ? (int)((long long)warp * L / We) : L;
    const int wc1 = warp < We ? (int)((long long)(warp + 1) * L / We) : L;
    const size_t row_bytes = (size_t)p.K * ESZ;
    const uint16_t* s16 = static_cast<const uint16_t*>(p.s);

    // The CTA's group scales are one contiguous block of the [N, G] array:
    // stage it (16-byte pieces covering it) when the caller's layout allows.
    const size_t sc_lo = p.sc_bytes ? ((size_t)row0 * p.G * 2) & ~(size_t)15 : 0;
    if (WK == W_FP8_GROUP && p.sc_bytes) {
        const size_t sc_hi = ((size_t)row1 * p.G * 2 + 15) & ~(size_t)15;
        const unsigned char* sb = static_cast<const unsigned char*>(p.s);
        for (size_t o = sc_lo + (size_t)threadIdx.x * 16; o < sc_hi; o += (size_t)kThreads * 16)
            cp_async16(smem_u32(scs + (o - sc_lo)), sb + o);
    }
    cp_async_commit();

    // Each lane streams exactly the bytes it consumes: per chunk 16 B of row g
    // and 16 B of row g+8 into its own places of a kS-slot ring, one commit
    // group per chunk.  Rows past row1 are not loaded.
    unsigned char* my_ring = ring + (size_t)warp * kS * 1024;
    // Issue cursor: next chunk to request (tile, chunk-in-tile, ring slot),
    // advanced incrementally -- no divisions in the stream loop.
    int i_left = wc1 - wc0;
    int i_tile = wc0 / p.cpt, i_kc = wc0 - (wc0 / p.cpt) * p.cpt, i_slot = 0;
    const uint8_t* i_p0 = nullptr;
    const uint8_t* i_p1 = nullptr;
    auto i_rows = [&]() {   // per-tile row pointers (null: row past row1)
        const int r0 = row0 + i_tile * 16 + g;
        i_p0 = r0 < row1 ? p.w + (size_t)r0 * row_bytes + (size_t)c * LPOS * ESZ : nullptr;
        i_p1 = r0 + 8 < row1 ? p.w + (size_t)(r0 + 8) * row_bytes + (size_t)c * LPOS * ESZ : nullptr;
    };
    i_rows();
    auto issue = [&]() {
        if (i_left > 0) {
            unsigned char* slot = my_ring + (size_t)i_slot * 1024;
            const size_t off = (size_t)i_kc * POS * ESZ;
            if (i_p0) cp_async16(smem_u32(slot + lane * 16), i_p0 + off);
            if (i_p1) cp_async16(smem_u32(slot + 512 + lane * 16), i_p1 + off);
            --i_left;
            if (++i_slot == kS) i_slot = 0;
            if (++i_kc == p.cpt) {
                i_kc = 0;
                ++i_tile;
                i_rows();
            }
        }
        cp_async_commit();   // empty groups past the end keep the count uniform
    };
#pragma unroll 1
    for (int q = 0; q < kS; ++q) issue();

    // Everything above touched only weights.  From here on we read the
    // activations and write outputs, which the previous kernel may own.
    pdl_wait();

    if (p.xs_stride > 0) {
        const int k8 = p.K >> 3;
        const int total = p.M * k8;
        for (int i = threadIdx.x; i < total; i += kThreads) {
            const int tok = i / k8;
            const int kk = (i - tok * k8) * 8;
            *reinterpret_cast<uint4*>(xs + (size_t)tok * p.xs_stride + kk) = ldcg_u4(p.x + (size_t)tok * p.K + kk);
        }
    }
    cp_async_wait<kS>();   // the scale group (the oldest) has landed
    __syncthreads();

    auto load_x = [&](int tok, int pos, uint32_t (&xf)[LPOS / 2]) {
#pragma unroll
        for (int u = 0; u < XU4; ++u) {
            uint4 v;
            if (p.xs_stride > 0)
                v = *reinterpret_cast<const uint4*>(xs + (size_t)tok * p.xs_stride + pos + u * 8);
            else
                v = ldcg_u4(p.x + (size_t)tok * p.K + pos + u * 8);
            xf[u * 4 + 0] = v.x;
            xf[u * 4 + 1] = v.y;
            xf[u * 4 + 2] = v.z;
            xf[u * 4 + 3] = v.w;
        }
    };

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[nt][k] = 0.f;

    auto scale_pair = [&](int r0, int r1, int grp) -> uint32_t {
        uint32_t lo = 0, hi = 0;
        if (p.sc_bytes) {
            if (r0 < row1) lo = *reinterpret_cast<const uint16_t*>(scs + ((size_t)r0 * p.G + grp) * 2 - sc_lo);
            if (r1 < row1) hi = *reinterpret_cast<const uint16_t*>(scs + ((size_t)r1 * p.G + grp) * 2 - sc_lo);
        } else {
            if (r0 < row1) lo = __ldg(s16 + (size_t)r0 * p.G + grp);
            if (r1 < row1) hi = __ldg(s16 + (size_t)r1 * p.G + grp);
        }
        return lo | (hi << 16);
    };

    // Chunk at (tile, kc, slot): its data landed (wait_group); compute, then
    // refill the slot with the chunk kS further on.
    auto compute = [&](int tile, int kc, int slot_i) {
        const int r0 = row0 + tile * 16 + g;
        const int r1 = r0 + 8;
        const unsigned char* slot = my_ring + (size_t)slot_i * 1024;
        cp_async_wait<kS - 1>();
        const uint4 w0 = r0 < row1 ? *reinterpret_cast<const uint4*>(slot + lane * 16) : make_uint4(0, 0, 0, 0);
        const uint4 w1 = r1 < row1 ? *reinterpret_cast<const uint4*>(slot + 512 + lane * 16) : make_uint4(0, 0, 0, 0);
        const uint32_t scp = (WK == W_FP8_GROUP) ? scale_pair(r0, r1, kc >> 1) : 0u;
        const int pos = kc * POS + c * LPOS;
        float d[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int k = 0; k < 4; ++k) d[nt][k] = 0.f;
        uint32_t xf[NT][LPOS / 2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) load_x(min(nt * 8 + g, p.M - 1), pos, xf[nt]);
        constexpr int KSTEPS = (WK == W_F16) ? 2 : 4;
#pragma unroll
        for (int t = 0; t < KSTEPS; ++t) {
            uint32_t a0, a1, a2, a3;
            if (WK == W_F16) {
                a0 = u4w(w0, 2 * t);
                a1 = u4w(w1, 2 * t);
                a2 = u4w(w0, 2 * t + 1);
                a3 = u4w(w1, 2 * t + 1);
            } else {
                const uint32_t b0 = u4w(w0, t), b1 = u4w(w1, t);
                a0 = e4m3x2_lo(b0);
                a1 = e4m3x2_lo(b1);
                a2 = e4m3x2_hi(b0);
                a3 = e4m3x2_hi(b1);
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float e[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(e, a0, a1, a2, a3, xf[nt][2 * t], xf[nt][2 * t + 1]);
#pragma unroll
                for (int k = 0; k < 4; ++k) d[nt][k] += e[k];
            }
        }
        // the slot's bytes are in registers and used: refill it
        issue();
        if (WK == W_FP8_GROUP) {
            const float s0 = half_bits_to_float((uint16_t)(scp & 0xffffu));
            const float s1 = half_bits_to_float((uint16_t)(scp >> 16));
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                acc[nt][0] = fmaf(s0, d[nt][0], acc[nt][0]);
                acc[nt][1] = fmaf(s0, d[nt][1], acc[nt][1]);
                acc[nt][2] = fmaf(s1, d[nt][2], acc[nt][2]);
                acc[nt][3] = fmaf(s1, d[nt][3], acc[nt][3]);
            }
        } else {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[nt][k] += d[nt][k];
        }
    };

    float best_v = 0.f;   // fused argmax: running best of this lane
    int best_i = -1;

    auto emit = [&](int tile, float (&v)[NT][4]) {
        const int r0 = row0 + tile * 16 + g;
        const int r1 = r0 + 8;
        if (WK == W_FP8_ROW && p.s != nullptr) {
            const float* s32 = static_cast<const float*>(p.s);
            const float s0 = r0 < row1 ? __ldg(s32 + r0) : 0.f;
            const float s1 = r1 < row1 ? __ldg(s32 + r1) : 0.f;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                v[nt][0] *= s0;
                v[nt][1] *= s0;
                v[nt][2] *= s1;
                v[nt][3] *= s1;
            }
        }
        if (p.y != nullptr) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    const int tok = nt * 8 + 2 * c + jj;
                    if (tok < p.M) {
                        if (p.y_f32) {
                            float* y = static_cast<float*>(p.y) + (size_t)tok * p.N;
                            if (r0 < row1) y[r0] = v[nt][jj];
                            if (r1 < row1) y[r1] = v[nt][2 + jj];
                        } else {
                            __half* y = static_cast<__half*>(p.y) + (size_t)tok * p.N;
                            if (r0 < row1) y[r0] = __float2half_rn(v[nt][jj]);
                            if (r1 < row1) y[r1] = __float2half_rn(v[nt][2 + jj]);
                        }
                    }
                }
            }
        }
        if (p.arg_out != nullptr && c == 0) {
            const int lim = min(row1, p.arg_limit);
            if (r0 < lim && argmax_better(v[0][0], r0, best_v, best_i)) { best_v = v[0][0]; best_i = r0; }
            if (r1 < lim && argmax_better(v[0][2], r1, best_v, best_i)) { best_v = v[0][2]; best_i = r1; }
        }
    };

    // A warp's range has at most two partial tile segments: its first (slot 0)
    // and its last (slot 1); a range inside one tile uses slot 0.
    const int first_tile = wc0 < wc1 ? wc0 / p.cpt : -1;

    auto segment_end = [&](int tile, int seg_lo, int seg_hi) {
        if (seg_lo == tile * p.cpt && seg_hi == (tile + 1) * p.cpt) {
            emit(tile, acc);   // the whole tile lies in this warp's range
        } else {
            float* dst = wslots + ((size_t)(warp * 2 + (tile == first_tile ? 0 : 1)) * 32 + lane) * PF;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
                *reinterpret_cast<float4*>(dst + 4 * nt) = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[nt][k] = 0.f;
    };

    int seg_lo = wc0;
    int c_tile = wc0 < wc1 ? wc0 / p.cpt : 0;
    int c_kc = wc0 - c_tile * p.cpt, c_slot = 0;
#pragma unroll 2
    for (int j = wc0; j < wc1; ++j) {
        compute(c_tile, c_kc, c_slot);
        if (++c_slot == kS) c_slot = 0;
        const bool tile_done = ++c_kc == p.cpt;
        if (j + 1 == wc1 || tile_done) {
            segment_end(c_tile, seg_lo, j + 1);
            seg_lo = j + 1;
        }
        if (tile_done) {
            c_kc = 0;
            ++c_tile;
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    // Tiles split between warps: sum the warps' partials in warp order.
    for (int t = warp; t < T; t += kWarps) {
        const int lo = t * p.cpt, hi = (t + 1) * p.cpt;
        const int wa_ = (int)owner_of(lo, L, We);
        const int wb_ = (int)owner_of(hi - 1, L, We);
        if (wa_ == wb_) continue;   // finished by its warp already
        float v[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int k = 0; k < 4; ++k) v[nt][k] = 0.f;
        for (int w = wa_; w <= wb_; ++w) {
            const int w0 = (int)((long long)w * L / We);
            const int slot = (t == w0 / p.cpt) ? 0 : 1;
            const float* src = wslots + ((size_t)(w * 2 + slot) * 32 + lane) * PF;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float4 f = *reinterpret_cast<const float4*>(src + 4 * nt);
                v[nt][0] += f.x;
                v[nt][1] += f.y;
                v[nt][2] += f.z;
                v[nt][3] += f.w;
            }
        }
        emit(t, v);
    }

    if (p.arg_out != nullptr) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (argmax_better(ov, oi, best_v, best_i)) { best_v = ov; best_i = oi; }
        }
        if (lane == 0) {
            s_best_v[warp] = best_v;
            s_best_i[warp] = best_i;
        }
        __syncthreads();
        if (warp == 0) {
            best_v = lane < kWarps ? s_best_v[lane] : 0.f;
            best_i = lane < kWarps ? s_best_i[lane] : -1;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
                if (argmax_better(ov, oi, best_v, best_i)) { best_v = ov; best_i = oi; }
            }
            int last = 0;
            if (lane == 0) {
                __stcg(p.arg_val + cta, best_v);
                __stcg(p.arg_idx + cta, best_i);
                __threadfence();
                last = (atomicAdd(p.arg_done, 1) == G - 1);
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
                float bv = 0.f;
                int bi = -1;
                for (int i = lane; i < G; i += 32) {
                    const float v = ldcg_f32(p.arg_val + i);
                    const int ix = ldcg_s32(p.arg_idx + i);
                    if (argmax_better(v, ix, bv, bi)) { bv = v; bi = ix; }
                    __stcg(p.arg_val + i, 0.f);   // leave the workspace all-zero
                    __stcg(p.arg_idx + i, 0);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (argmax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                }
                if (lane == 0) {
                    *p.arg_out = bi;
                    *p.arg_done = 0;
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// One token, FP8 weights, K % 128 == 0: the decode case of the reference
// (every launch_w8a16_gemv of engine.cu, and an FP8 lm_head).  Same row split
// and warp ranges as gemv_stream_kernel, tuned for a chain of dependent GEMVs:
//   * a chunk is a whole 128-wide scale group (a lane streams 32 B of rows g
//     and g+8: bytes [16c, 16c+16) and [64+16c, 64+16c+16), so that each load
//     instruction covers whole 32-byte sectors), all per-tile addressing is
//     hoisted out of the chunk loop;
//   * 8 warps and <= 113 KB of shared memory per CTA, so that the CTA of the
//     NEXT GEMV of the stream sits on the same SM and fills its own ring
//     (cp.async, before its griddepcontrol.wait) while this one computes --
//     the SM's memory pipe never idles between kernels;
//   * x arrives by one bulk copy on the TMA engine straight into shared memory,
//     so it does not queue behind the co-resident CTA's weight requests.
//   * PAIR (gate/up + SwiGLU): a 16-row MMA tile holds 8 gate rows and the same
//     8 up rows, so each lane owns gate[r] and up[r] and applies the
//     activation in registers.
//   * MT = 8 (2..8 tokens): the MMA's 8 columns carry 8 tokens -- lane (g, c)
//     feeds token g's x -- so a batch costs the MMA instructions of one token;
//     x rows sit in shared memory 16 bytes apart modulo 128 (bank-conflict free).
//     MT = 16 (9..16 tokens): a second MMA per k-step on the same converted
//     weights for tokens 8..15.
// Fault bits (AF_FAULT_*) of this device's GEMV kernels, read by af_device_faults.
__device__ unsigned int g_gemv_faults;

template <bool GROUP, bool F16, int kWarps, int kS, int kMinCtas, bool PAIR, int MT = 1>
__global__ void __launch_bounds__(kWarps * 32, kMinCtas) gemv_fp8_m1_kernel(const GemvParams p) {
    constexpr int kThreads = kWarps * 32;
    constexpr int kSlot = 2048;
    constexpr int NQ = MT == 16 ? 8 : 4;   // accumulators per lane
    pdl_launch_dependents();
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* ring = smem;
    __half* xs = reinterpret_cast<__half*>(smem + (size_t)kWarps * kS * kSlot);   // x: K halves
    unsigned char* scs = reinterpret_cast<unsigned char*>(xs) + p.xs_bytes;       // staged scales
    // warp partials [kWarps][2][32][4] reuse the ring once every warp has finished streaming
    float* wslots = reinterpret_cast<float*>(ring);
    __shared__ __align__(8) uint64_t s_xbar;
    __shared__ float s_red[kWarps];
    __shared__ int s_redi[kWarps];
    __shared__ int s_wstart[kWarps + 1];   // first chunk of each warp; [kWarps] = L

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
    const int G = gridDim.x, cta = blockIdx.x;
    const int row0 = (int)((long long)cta * p.N / G);
    const int row1 = (int)((long long)(cta + 1) * p.N / G);
    constexpr int ESZ = F16 ? 2 : 1;              // weight bytes per element
    constexpr int CPOS = 128 / ESZ;               // positions per 128-byte chunk
    const int cpt = (p.K * ESZ) >> 7;             // chunks (FP8: scale groups) per row
    constexpr int TR = PAIR ? 8 : 16;             // output rows per MMA tile
    const int T = (row1 - row0 + TR - 1) / TR;
    const int L = T * cpt;
    const int We = L < kWarps ? L : kWarps;
    const int wc0 = warp < We ? (int)((long long)warp * L / We) : L;
    const int wc1 = warp < We ? (int)((long long)(warp + 1) * L / We) : L;

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&s_xbar), 1);
        mbar_init_fence();
        s_wstart[kWarps] = L;
    }
    if (lane == 0) s_wstart[warp] = wc0;
    __syncthreads();

    // staged scales: bytes [sc_lo, ...) of the [N, G] FP16 array
    const size_t sc_lo = p.sc_bytes ? ((size_t)row0 * cpt * 2) & ~(size_t)15 : 0;
    const int sc_half = PAIR ? p.sc_bytes / 2 : 0;   // gate/up mode: up scales at scs + sc_half
    if (GROUP && p.sc_bytes) {
        const size_t sc_hi = ((size_t)row1 * cpt * 2 + 15) & ~(size_t)15;
#pragma unroll
        for (int m = 0; m < (PAIR ? 2 : 1); ++m) {
            const unsigned char* sb = static_cast<const unsigned char*>(m ? p.s2 : p.s);
            for (size_t o = sc_lo + (size_t)threadIdx.x * 16; o < sc_hi; o += (size_t)kThreads * 16)
                cp_async16(smem_u32(scs + m * sc_half + (o - sc_lo)), sb + o);
        }
    }
    // RMSNorm weight (a constant: staged before the wait)
    float* gam = reinterpret_cast<float*>(scs + p.sc_bytes);
    if (p.norm_w != nullptr) {
        const unsigned char* gb = reinterpret_cast<const unsigned char*>(p.norm_w);
        for (int o = threadIdx.x * 16; o < p.K * 4; o += kThreads * 16)
            cp_async16(smem_u32(reinterpret_cast<unsigned char*>(gam) + o), gb + o);
    }
    cp_async_commit();

    // ---- issue cursor (weights only: runs before griddepcontrol.wait) ----
    // Slot layout: [row g bytes 0-15 | row g 16-31 | row g+8 0-15 | row g+8 16-31],
    // 512 B each, lane-major: conflict-free 128-bit shared loads.
    const uint32_t my_ring = smem_u32(ring + (size_t)warp * kS * kSlot) + lane * 16;
    int i_left = wc1 - wc0;
    int i_tile = wc0 / (cpt > 0 ? cpt : 1);
    int i_kc = wc0 - i_tile * cpt, i_slot = 0;
    const uint8_t* i_p0 = nullptr;
    const uint8_t* i_p1 = nullptr;
    auto i_rows = [&]() {
        const int r0 = row0 + i_tile * TR + g;
        if (PAIR) {
            i_p0 = r0 < row1 ? p.w + (size_t)r0 * p.K + c * 16 : nullptr;
            i_p1 = r0 < row1 ? p.w2 + (size_t)r0 * p.K + c * 16 : nullptr;
        } else {
            i_p0 = r0 < row1 ? p.w + (size_t)r0 * p.K * ESZ + c * 16 : nullptr;
            i_p1 = r0 + 8 < row1 ? p.w + (size_t)(r0 + 8) * p.K * ESZ + c * 16 : nullptr;
        }
    };
    i_rows();
    auto issue = [&]() {
        if (i_left > 0) {
            const uint32_t d = my_ring + i_slot * kSlot;
            const int off = i_kc << 7;
            // lanes c = 0..3 of a row cover 64 contiguous bytes per instruction
            if (i_p0) {
                cp_async16(d, i_p0 + off);
                cp_async16(d + 512, i_p0 + off + 64);
            }
            if (i_p1) {
                cp_async16(d + 1024, i_p1 + off);
                cp_async16(d + 1536, i_p1 + off + 64);
            }
            --i_left;
            if (++i_slot == kS) i_slot = 0;
            if (++i_kc == cpt) {
                i_kc = 0;
                ++i_tile;
                i_rows();
            }
        }
        cp_async_commit();
    };
    // Only part of the ring is requested before griddepcontrol.wait (p.pre slots);
    // the rest after x has landed, so that the previous kernel's x/y traffic and
    // our own x fetch do not wait behind a full prefetch.
#pragma unroll 1
    for (int q = 0; q < p.pre; ++q) issue();
    // x may be written by the kernel this one waits for, so it is read only
    // after the wait; an L2 prefetch now is only a hint (L2 is the point of
    // coherence) and turns that read into an L2 hit when x was not just written.
    if (threadIdx.x == 32) bulk_prefetch_l2(p.x, (uint32_t)p.M * p.K * 2u);

    pdl_wait();
    // x by one bulk copy on the TMA engine (see above)
    if (threadIdx.x == 0) {
        if (MT == 1) {
            mbar_arrive_expect_tx(smem_u32(&s_xbar), (uint32_t)p.K * 2u);
            bulk_g2s(smem_u32(xs), p.x, (uint32_t)p.K * 2u, smem_u32(&s_xbar));
        } else {
            mbar_arrive_expect_tx(smem_u32(&s_xbar), (uint32_t)p.M * p.K * 2u);
            for (int m = 0; m < p.M; ++m)
                bulk_g2s(smem_u32(xs + (size_t)m * p.xs_stride), p.x + (size_t)m * p.K, (uint32_t)p.K * 2u,
                         smem_u32(&s_xbar));
        }
    }
    // tensor-parallel epilogue: row r's tag this launch is its epoch + 1
    const unsigned* row_ep = p.tp_world > 1
        ? reinterpret_cast<const unsigned*>(p.tp_buf[p.tp_rank] + TpLayout::row_epoch(p.tp_nmax)) : nullptr;
    cp_async_wait<0>();    // staged scales (and the early ring slots) have landed
    __syncthreads();       // everyone's staged scales are visible
    if (!mbar_wait_bounded(smem_u32(&s_xbar), 0, 2000000000ull))
        atomicOr(&g_gemv_faults, (unsigned)AF_FAULT_X_COPY);   // y is not valid: the host sees the fault bit
    if (MT == 1 && p.norm_w != nullptr) {
        // RMSNorm of x in place, in the reference's arithmetic order
        // (src/kernel/rmsnorm.cu:9-67, 128 threads): per-thread strided FMA
        // sums, each warp's shuffle-down tree, the warps' sums in order, then
        // rsqrt(sum / K + eps) and half(x * r * w).
        __shared__ float s_nrm[4];
        __shared__ float s_rms;
        if (threadIdx.x < 128) {
            float ss = 0.f;
            for (int i = threadIdx.x; i < p.K; i += 128) {
                const float v = __half2float(xs[i]);
                ss = fmaf(v, v, ss);
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) ss += __shfl_down_sync(0xffffffffu, ss, o);
            if (lane == 0) s_nrm[warp] = ss;
        }
        __syncthreads();
        if (threadIdx.x == 0)
            s_rms = rms_scale_ref(((s_nrm[0] + s_nrm[1]) + s_nrm[2]) + s_nrm[3], p.K, p.norm_eps);
        __syncthreads();
        const float r = s_rms;
        for (int i = threadIdx.x; i < p.K; i += kThreads) xs[i] = __float2half_rn(__half2float(xs[i]) * r * gam[i]);
        __syncthreads();
        if (p.xn_out != nullptr && cta == 0)
            for (int i = threadIdx.x; i < p.K; i += kThreads) p.xn_out[i] = xs[i];
    }
#pragma unroll 1
    for (int q = p.pre; q < kS; ++q) issue();

    // ---- compute cursor ----
    const unsigned char* my_ring_p = ring + (size_t)warp * kS * kSlot + lane * 16;
    // MT = 8: lane (g, c) feeds token g (tokens >= M read zeros)
    const bool x_on = MT == 1 || g < p.M;
    const __half* my_x = xs + (MT == 1 ? 0 : (size_t)(x_on ? g : 0) * p.xs_stride) + c * (16 / ESZ);
    const bool x_on1 = MT == 16 && g + 8 < p.M;   // second token group (MT = 16)
    const __half* my_x1 = xs + (MT == 16 ? (size_t)(x_on1 ? g + 8 : 0) * p.xs_stride : 0) + c * (16 / ESZ);
    const uint16_t* s16 = static_cast<const uint16_t*>(p.s);
    const float* rs = static_cast<const float*>(p.s);
    int c_tile = wc0 / (cpt > 0 ? cpt : 1);
    int c_kc = wc0 - c_tile * cpt, c_slot = 0;
    bool v0 = false, v1 = false;
    const uint16_t* sp0 = nullptr;   // scales of rows g, g+8 (shared or global)
    const uint16_t* sp1 = nullptr;
    auto c_rows = [&]() {
        const int r0 = row0 + c_tile * TR + g;
        v0 = r0 < row1;
        v1 = PAIR ? v0 : r0 + 8 < row1;
        if (PAIR) {
            const int a0 = v0 ? r0 : row0;
            if (p.sc_bytes) {
                sp0 = reinterpret_cast<const uint16_t*>(scs + (size_t)a0 * cpt * 2 - sc_lo);
                sp1 = reinterpret_cast<const uint16_t*>(scs + sc_half + (size_t)a0 * cpt * 2 - sc_lo);
            } else {
                sp0 = s16 + (size_t)a0 * cpt;
                sp1 = static_cast<const uint16_t*>(p.s2) + (size_t)a0 * cpt;
            }
        } else if (GROUP) {
            const int a0 = v0 ? r0 : row0, a1 = v1 ? r0 + 8 : row0;
            if (p.sc_bytes) {
                sp0 = reinterpret_cast<const uint16_t*>(scs + (size_t)a0 * cpt * 2 - sc_lo);
                sp1 = reinterpret_cast<const uint16_t*>(scs + (size_t)a1 * cpt * 2 - sc_lo);
            } else {
                sp0 = s16 + (size_t)a0 * cpt;
                sp1 = s16 + (size_t)a1 * cpt;
            }
        }
    };
    c_rows();

    float acc[NQ], part0[NQ], part1[NQ];
#pragma unroll
    for (int k = 0; k < NQ; ++k) acc[k] = part0[k] = part1[k] = 0.f;
    const int first_tile = wc0 < wc1 ? c_tile : -1;
    float best_v = 0.f;
    int best_i = -1;

    auto emit = [&](int tile, const float (&v)[NQ]) {
        if (MT > 1) {
            // lane (g, c) holds rows g, g+8 for tokens 2c, 2c+1 (and 8+2c, 9+2c)
            const int r0 = row0 + tile * 16 + g, r1 = r0 + 8;
#pragma unroll
            for (int j = 0; j < NQ / 2; ++j) {
                const int tok = (j >> 1) * 8 + 2 * c + (j & 1);
                if (tok >= p.M) continue;
                float a = v[(j >> 1) * 4 + (j & 1)], b = v[(j >> 1) * 4 + 2 + (j & 1)];
                if (!GROUP && rs != nullptr) {
                    a *= r0 < row1 ? __ldg(rs + r0) : 0.f;
                    b *= r1 < row1 ? __ldg(rs + r1) : 0.f;
                }
                if (p.y_f32) {
                    float* yo = static_cast<float*>(p.y) + (size_t)tok * p.N;
                    if (r0 < row1) yo[r0] = a;
                    if (r1 < row1) yo[r1] = b;
                } else {
                    __half* yo = static_cast<__half*>(p.y) + (size_t)tok * p.N;
                    if (r0 < row1) yo[r0] = __float2half_rn(a);
                    if (r1 < row1) yo[r1] = __float2half_rn(b);
                }
            }
            return;
        }
        if (c != 0) return;   // token 0 sits in MMA column 0 (lanes c == 0)
        const int r0 = row0 + tile * TR + g, r1 = r0 + 8;
        float a = v[0], b = v[2];
        if (PAIR) {
            // gate and up rounded to FP16 as the reference stores them, then its
            // SwiGLU (src/kernel/swiglu.cu:12-26): half(g / (1 + e^-g) * u)
            if (r0 < row1) {
                const __half gh = __float2half_rn(a), uh = __float2half_rn(b);
                const float gf = __half2float(gh);
                const float silu = fdiv_full_ftz(gf, 1.0f + __expf(-gf));
                static_cast<__half*>(p.y)[r0] = __float2half_rn(silu * __half2float(uh));
                if (p.aux != nullptr) {
                    p.aux[r0] = gh;
                    p.aux[p.N + r0] = uh;
                }
            }
            return;
        }
        if (!GROUP && rs != nullptr) {
            a *= r0 < row1 ? __ldg(rs + r0) : 0.f;
            b *= r1 < row1 ? __ldg(rs + r1) : 0.f;
        }
        if (p.tp_world > 1 && !p.tp_arg) {
            // this rank's partial of rows r0, r1, tagged with each row's
            // epoch, into every rank's buffer (NVLink stores to the peers)
            const unsigned ea = r0 < row1 ? __ldcg(row_ep + r0) + 1u : 0u;
            const unsigned eb = r1 < row1 ? __ldcg(row_ep + r1) + 1u : 0u;
            const size_t sa = ((size_t)(ea & 1) * kTpMaxRanks + p.tp_rank) * p.tp_nmax;
            const size_t sb = ((size_t)(eb & 1) * kTpMaxRanks + p.tp_rank) * p.tp_nmax;
            const unsigned long long ta = ((unsigned long long)ea << 32) | __float_as_uint(a);
            const unsigned long long tb = ((unsigned long long)eb << 32) | __float_as_uint(b);
            for (int rr = 0; rr < p.tp_world; ++rr) {
                unsigned long long* part = reinterpret_cast<unsigned long long*>(p.tp_buf[rr] + TpLayout::part);
                if (r0 < row1) st_relaxed_sys_u64(part + sa + r0, ta);
                if (r1 < row1) st_relaxed_sys_u64(part + sb + r1, tb);
            }
        } else if (p.y != nullptr) {
            if (p.y_f32) {
                if (r0 < row1) static_cast<float*>(p.y)[r0] = a;
                if (r1 < row1) static_cast<float*>(p.y)[r1] = b;
            } else {
                // residual: half(res + half(Wx)) as the reference's residual add
                // (src/kernel/residual_add.cu:11-20) applied to the stored output
                __half ya = __float2half_rn(a), yb = __float2half_rn(b);
                if (p.aux != nullptr) {
                    if (r0 < row1) p.aux[r0] = ya;
                    if (r1 < row1) p.aux[r1] = yb;
                }
                if (p.res != nullptr) {
                    if (r0 < row1) ya = __float2half_rn(__half2float(p.res[r0]) + __half2float(ya));
                    if (r1 < row1) yb = __float2half_rn(__half2float(p.res[r1]) + __half2float(yb));
                }
                if (r0 < row1) static_cast<__half*>(p.y)[r0] = ya;
                if (r1 < row1) static_cast<__half*>(p.y)[r1] = yb;
            }
        }
        if (p.arg_out != nullptr) {
            const int lim = min(row1, p.arg_limit);
            if (r0 < lim && argmax_better(a, r0, best_v, best_i)) { best_v = a; best_i = r0; }
            if (r1 < lim && argmax_better(b, r1, best_v, best_i)) { best_v = b; best_i = r1; }
        }
    };

    int seg_lo = wc0;
#pragma unroll 1
    for (int j = wc0; j < wc1; ++j) {
        cp_async_wait<kS - 1>();
        const unsigned char* sl = my_ring_p + c_slot * kSlot;
        const uint4 z = make_uint4(0, 0, 0, 0);
        uint4 wg[2], wh[2];
        wg[0] = v0 ? *reinterpret_cast<const uint4*>(sl) : z;
        wg[1] = v0 ? *reinterpret_cast<const uint4*>(sl + 512) : z;
        wh[0] = v1 ? *reinterpret_cast<const uint4*>(sl + 1024) : z;
        wh[1] = v1 ? *reinterpret_cast<const uint4*>(sl + 1536) : z;
        // the lane's 32 positions: [16c, 16c+16) and [64+16c, 64+16c+16) of the chunk
        // FP16 weights: the lane's 16 positions [8c, 8c+8) and [32+8c, 32+8c+8)
        const __half* xp_ = my_x + c_kc * CPOS;
        uint4 xv[4];
        if (F16) {
            xv[0] = *reinterpret_cast<const uint4*>(xp_);
            xv[1] = *reinterpret_cast<const uint4*>(xp_ + 32);
        } else {
            xv[0] = *reinterpret_cast<const uint4*>(xp_);
            xv[1] = *reinterpret_cast<const uint4*>(xp_ + 8);
            xv[2] = *reinterpret_cast<const uint4*>(xp_ + 64);
            xv[3] = *reinterpret_cast<const uint4*>(xp_ + 72);
        }
        if (MT > 1 && !x_on) xv[0] = xv[1] = xv[2] = xv[3] = make_uint4(0, 0, 0, 0);
        uint4 xw[4];   // tokens 8..15 (MT = 16)
        if (MT == 16) {
            const __half* xq = my_x1 + c_kc * CPOS;
            xw[0] = *reinterpret_cast<const uint4*>(xq);
            xw[1] = *reinterpret_cast<const uint4*>(xq + 8);
            xw[2] = *reinterpret_cast<const uint4*>(xq + 64);
            xw[3] = *reinterpret_cast<const uint4*>(xq + 72);
            if (!x_on1) xw[0] = xw[1] = xw[2] = xw[3] = make_uint4(0, 0, 0, 0);
        }
        float s0 = 1.f, s1 = 1.f;
        if (GROUP) {
            s0 = half_bits_to_float(sp0[c_kc]);
            s1 = half_bits_to_float(sp1[c_kc]);
        }
        issue();   // this slot's bytes are in registers: refill it
        float d[NQ];
#pragma unroll
        for (int k = 0; k < NQ; ++k) d[k] = 0.f;
        // lane (g, c): bytes 4t..4t+3 of its 32 row bytes are MMA k-step t; its
        // x halves are in the same order, so the permutation of k cancels
#pragma unroll
        for (int t = 0; t < (F16 ? 4 : 8); ++t) {
            uint32_t a0, a1, a2, a3;
            if (F16) {   // halves 4t..4t+3 of the lane's 16
                a0 = u4w(wg[t >> 1], (t & 1) * 2);
                a1 = u4w(wh[t >> 1], (t & 1) * 2);
                a2 = u4w(wg[t >> 1], (t & 1) * 2 + 1);
                a3 = u4w(wh[t >> 1], (t & 1) * 2 + 1);
            } else {     // bytes 4t..4t+3 of the lane's 32
                const uint32_t b0 = u4w(wg[t >> 2], t & 3), b1 = u4w(wh[t >> 2], t & 3);
                a0 = e4m3x2_lo(b0);
                a1 = e4m3x2_lo(b1);
                a2 = e4m3x2_hi(b0);
                a3 = e4m3x2_hi(b1);
            }
            float e[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(e, a0, a1, a2, a3, u4w(xv[t >> 1], (t & 1) * 2), u4w(xv[t >> 1], (t & 1) * 2 + 1));
#pragma unroll
            for (int k = 0; k < 4; ++k) d[k] += e[k];
            if (MT == 16) {
                float e1[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(e1, a0, a1, a2, a3, u4w(xw[t >> 1], (t & 1) * 2), u4w(xw[t >> 1], (t & 1) * 2 + 1));
#pragma unroll
                for (int k = 0; k < 4; ++k) d[4 + k] += e1[k];
            }
        }
#pragma unroll
        for (int k = 0; k < NQ; ++k) acc[k] = fmaf((k & 2) ? s1 : s0, d[k], acc[k]);
        if (++c_slot == kS) c_slot = 0;
        const bool tile_done = ++c_kc == cpt;
        if (j + 1 == wc1 || tile_done) {
            if (seg_lo == c_tile * cpt && j + 1 == (c_tile + 1) * cpt) {
                emit(c_tile, acc);
            } else {
                float* dst = c_tile == first_tile ? part0 : part1;   // registers until the ring is free
#pragma unroll
                for (int k = 0; k < NQ; ++k) dst[k] = acc[k];
            }
#pragma unroll
            for (int k = 0; k < NQ; ++k) acc[k] = 0.f;
            seg_lo = j + 1;
        }
        if (tile_done) {
            c_kc = 0;
            ++c_tile;
            c_rows();
        }
    }
    cp_async_wait<0>();
    __syncthreads();   // every warp is done with the ring
#pragma unroll
    for (int q = 0; q < NQ / 4; ++q) {
        *reinterpret_cast<float4*>(wslots + ((size_t)(warp * 2 + 0) * 32 + lane) * NQ + 4 * q) =
            make_float4(part0[4 * q], part0[4 * q + 1], part0[4 * q + 2], part0[4 * q + 3]);
        *reinterpret_cast<float4*>(wslots + ((size_t)(warp * 2 + 1) * 32 + lane) * NQ + 4 * q) =
            make_float4(part1[4 * q], part1[4 * q + 1], part1[4 * q + 2], part1[4 * q + 3]);
    }
    __syncthreads();

    // Tiles split between warps: sum the owners' partials in warp order.  The
    // owners come from the warp-start table (no divisions on this serial tail).
    for (int t = warp; t < T; t += kWarps) {
        const int lo = t * cpt, hi = lo + cpt;
        float v[NQ];
#pragma unroll
        for (int k = 0; k < NQ; ++k) v[k] = 0.f;
        int owners = 0;
        for (int w = 0; w < kWarps; ++w) {
            const int a = s_wstart[w], b = s_wstart[w + 1];
            if (a >= b || a >= hi || b <= lo) continue;
            ++owners;
            const int slot = a >= lo ? 0 : 1;   // t is w's first tile -> part0
#pragma unroll
            for (int q = 0; q < NQ / 4; ++q) {
                const float4 f =
                    *reinterpret_cast<const float4*>(wslots + ((size_t)(w * 2 + slot) * 32 + lane) * NQ + 4 * q);
                v[4 * q] += f.x;
                v[4 * q + 1] += f.y;
                v[4 * q + 2] += f.z;
                v[4 * q + 3] += f.w;
            }
        }
        if (owners < 2) continue;   // one owner: emitted from the main loop
        emit(t, v);
    }

    if (p.tp_world > 1 && !p.tp_arg) {
        // Sum this CTA's rows over the ranks, in rank order: each word is
        // polled (bounded) until it carries the row's epoch.  A peer is at
        // most one launch ahead on any row (it cannot finish a launch without
        // our partials of it), so the other parity half is never overwritten
        // early.  The barrier orders every emitting thread's epoch read before
        // the thread that owns the row here bumps it.
        __syncthreads();
        unsigned* my_ep = reinterpret_cast<unsigned*>(p.tp_buf[p.tp_rank] + TpLayout::row_epoch(p.tp_nmax));
        const unsigned long long* part = reinterpret_cast<const unsigned long long*>(p.tp_buf[p.tp_rank] + TpLayout::part);
        bool late = false;
        for (int r = row0 + threadIdx.x; r < row1; r += kThreads) {
            const unsigned ep = __ldcg(my_ep + r) + 1u;
            const unsigned long long* half_r = part + (size_t)(ep & 1) * kTpMaxRanks * p.tp_nmax + r;
            float acc_r = 0.f;
            for (int rr = 0; rr < p.tp_world; ++rr) {
                const unsigned long long* wp = half_r + (size_t)rr * p.tp_nmax;
                unsigned long long v = ld_relaxed_sys_u64(wp);
                if ((unsigned)(v >> 32) != ep && !late) {
                    const uint64_t t0 = globaltimer_ns();
                    do {
                        v = ld_relaxed_sys_u64(wp);
                        if (globaltimer_ns() - t0 > p.tp_wait_ns) { late = true; break; }
                    } while ((unsigned)(v >> 32) != ep);
                }
                acc_r += __uint_as_float((unsigned)v);
            }
            __stcg(my_ep + r, ep);
            __half yh = __float2half_rn(acc_r);
            if (p.aux != nullptr) p.aux[r] = yh;
            if (p.res != nullptr) yh = __float2half_rn(__half2float(p.res[r]) + __half2float(yh));
            static_cast<__half*>(p.y)[r] = yh;
        }
        if (late) atomicOr(reinterpret_cast<int*>(p.tp_buf[p.tp_rank] + TpLayout::status), 1);
    }

    if (p.arg_out != nullptr) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (argmax_better(ov, oi, best_v, best_i)) { best_v = ov; best_i = oi; }
        }
        if (lane == 0) {
            s_red[warp] = best_v;
            s_redi[warp] = best_i;
        }
        __syncthreads();
        if (warp == 0) {
            best_v = lane < kWarps ? s_red[lane] : 0.f;
            best_i = lane < kWarps ? s_redi[lane] : -1;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
                if (argmax_better(ov, oi, best_v, best_i)) { best_v = ov; best_i = oi; }
            }
            int last = 0;
            if (lane == 0) {
                __stcg(p.arg_val + cta, best_v);
                __stcg(p.arg_idx + cta, best_i);
                __threadfence();
                last = (atomicAdd(p.arg_done, 1) == G - 1);
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
                float bv = 0.f;
                int bi = -1;
                for (int i = lane; i < G; i += 32) {
                    const float v = ldcg_f32(p.arg_val + i);
                    const int ix = ldcg_s32(p.arg_idx + i);
                    if (argmax_better(v, ix, bv, bi)) { bv = v; bi = ix; }
                    __stcg(p.arg_val + i, 0.f);   // leave the workspace all-zero
                    __stcg(p.arg_idx + i, 0);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (argmax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                }
                if (p.tp_world > 1 && p.tp_arg) {
                    // vocab-parallel: push (max, global index) to every rank, then
                    // reduce all ranks' pairs (lane r polls rank r, bounded)
                    const unsigned ep = (unsigned)ldcg_s32(reinterpret_cast<const int*>(
                                            p.tp_buf[p.tp_rank] + TpLayout::lm_epoch)) + 1u;
                    const size_t pslot = ((size_t)(ep & 1) * kTpMaxRanks + p.tp_rank) * 2;
                    const int gi = bi >= 0 ? bi + p.arg_off : -1;
                    if (lane < p.tp_world) {
                        unsigned long long* dst =
                            reinterpret_cast<unsigned long long*>(p.tp_buf[lane] + TpLayout::lm_pair) + pslot;
                        st_relaxed_sys_u64(dst, ((unsigned long long)ep << 32) | __float_as_uint(bv));
                        st_relaxed_sys_u64(dst + 1, ((unsigned long long)ep << 32) | (unsigned)gi);
                    }
                    float rv = 0.f;
                    int ri = -1;
                    if (lane < p.tp_world) {
                        const unsigned long long* src =
                            reinterpret_cast<const unsigned long long*>(p.tp_buf[p.tp_rank] + TpLayout::lm_pair) +
                            ((size_t)(ep & 1) * kTpMaxRanks + lane) * 2;
                        unsigned long long a = ld_relaxed_sys_u64(src), b = ld_relaxed_sys_u64(src + 1);
                        if ((unsigned)(a >> 32) != ep || (unsigned)(b >> 32) != ep) {
                            const uint64_t t0 = globaltimer_ns();
                            bool late = false;
                            do {
                                a = ld_relaxed_sys_u64(src);
                                b = ld_relaxed_sys_u64(src + 1);
                                if (globaltimer_ns() - t0 > p.tp_wait_ns) { late = true; break; }
                            } while ((unsigned)(a >> 32) != ep || (unsigned)(b >> 32) != ep);
                            if (late) atomicOr(reinterpret_cast<int*>(p.tp_buf[p.tp_rank] + TpLayout::status), 1);
                        }
                        const bool fresh = (unsigned)(a >> 32) == ep && (unsigned)(b >> 32) == ep;
                        rv = fresh ? __uint_as_float((unsigned)a) : 0.f;   // a late rank is no candidate
                        ri = fresh ? (int)(unsigned)b : -1;
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, rv, o);
                        const int oi = __shfl_xor_sync(0xffffffffu, ri, o);
                        if (argmax_better(ov, oi, rv, ri)) { rv = ov; ri = oi; }
                    }
                    bi = ri;
                    if (lane == 0) reinterpret_cast<unsigned*>(p.tp_buf[p.tp_rank] + TpLayout::lm_epoch)[0] = ep;
                }
                if (lane == 0) {
                    *p.arg_out = bi;
                    *p.arg_done = 0;
                }
            }
        }
    }
}

// Any alignment, any K: one warp per (row, token), scalar decode.  Used when a
// pointer or K does not meet the streaming kernel's 16-byte layout rules.
__device__ __forceinline__ uint16_t ld_u16_bytes(const void* base, size_t byte_off) {
    const uint8_t* b = static_cast<const uint8_t*>(base) + byte_off;
    return (uint16_t)(b[0] | (b[1] << 8));
}

__global__ void gemv_simple_kernel(const uint8_t* w, int w_f16, const void* s, int skind, int G,
                                   const __half* x, void* y, int y_f32, int M, int N, int K) {
    pdl_wait();
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * (blockDim.x >> 5) + warp;
    const int m = blockIdx.y;
    if (n >= N || m >= M) return;
    float acc = 0.f;
    for (int k = lane; k < K; k += 32) {
        float wv;
        if (w_f16) {
            wv = half_bits_to_float(ld_u16_bytes(w, ((size_t)n * K + k) * 2));
        } else {
            const __half_raw hr = __nv_cvt_fp8_to_halfraw(w[(size_t)n * K + k], __NV_E4M3);
            wv = __half2float(__half(hr));
        }
        if (skind == AF_SCALE_GROUP_F16) wv *= half_bits_to_float(ld_u16_bytes(s, ((size_t)n * G + k / 128) * 2));
        acc = fmaf(wv, half_bits_to_float(ld_u16_bytes(x, ((size_t)m * K + k) * 2)), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
        if (skind == AF_SCALE_ROW_F32 && s != nullptr) {
            const uint8_t* sb = static_cast<const uint8_t*>(s) + (size_t)n * 4;
            acc *= __uint_as_float((uint32_t)sb[0] | ((uint32_t)sb[1] << 8) | ((uint32_t)sb[2] << 16) |
                                   ((uint32_t)sb[3] << 24));
        }
        // outputs are required aligned (FP16: 2 B, FP32: 4 B): typed stores
        if (y_f32)
            static_cast<float*>(y)[(size_t)m * N + n] = acc;
        else
            static_cast<__half*>(y)[(size_t)m * N + n] = __float2half_rn(acc);
    }
}

// ----------------------------------------------------------------- host ---

namespace {

struct Plan {
    int grid;
    int nt;
    int cpt;
    size_t off_done, off_argv, off_argi, total;
};

// The GEMV itself needs no device scratch (rows are split between CTAs, and
// warps of a CTA combine through shared memory).  Only the fused argmax does:
// one counter and one (value, index) candidate per CTA.  Word 0 is reserved.
Plan make_plan(int nt, int N, int K, int wk, int sms, bool argmax) {
    Plan pl{};
    pl.nt = nt;
    pl.grid = sms * ctas_per_sm();
    if (pl.grid > N) pl.grid = N;   // every CTA owns >= 1 row
    if (pl.grid < 1) pl.grid = 1;
    const int pos = (wk == W_F16) ? 32 : 64;
    pl.cpt = K / pos;
    size_t off = 256;
    pl.off_done = off;
    off = round_up(off + 4, 256);
    pl.off_argv = off;
    off = round_up(off + (size_t)pl.grid * 4, 256);
    pl.off_argi = off;
    off = round_up(off + (size_t)pl.grid * 4, 256);
    pl.total = argmax ? off : 0;
    return pl;
}

constexpr int kWarpsPerCta = 16;
constexpr int kRingSlots = 10;   // chunk slots per warp (1 KB each)

template <int WK, int NT>
cudaError_t launch_stream(const GemvParams& prm, const Plan& pl, size_t smem, cudaStream_t st) {
    auto kern = gemv_stream_kernel<WK, NT, kWarpsPerCta, kRingSlots>;
    static std::once_flag flags[kMaxDevices];
    static cudaError_t attr_err[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(flags[dev % kMaxDevices], [&] {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemMax - 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared);
        attr_err[dev % kMaxDevices] = e;
    });
    if (attr_err[dev % kMaxDevices] != cudaSuccess) return attr_err[dev % kMaxDevices];
    return launch_pdl(kern, dim3(pl.grid), dim3(kWarpsPerCta * 32), smem, st, prm);
}

template <bool GROUP, bool F16, int NW, int NS, bool PAIR = false, int MT = 1>
cudaError_t launch_m1(const GemvParams& prm, const Plan& pl, size_t smem, cudaStream_t st) {
    // a ring past ~100 KB means one CTA per SM: registers may grow
    auto kern = gemv_fp8_m1_kernel<GROUP, F16, NW, NS, (NW * NS * 2 > 100) ? 1 : (NW <= 6 ? 3 : 2), PAIR, MT>;
    static std::once_flag flags[kMaxDevices];
    static cudaError_t attr_err[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(flags[dev % kMaxDevices], [&] {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemMax - 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared);
        attr_err[dev % kMaxDevices] = e;
    });
    if (attr_err[dev % kMaxDevices] != cudaSuccess) return attr_err[dev % kMaxDevices];
    return launch_pdl(kern, dim3(pl.grid), dim3(NW * 32), smem, st, prm);
}

cudaError_t dispatch(int wk, const GemvParams& prm, const Plan& pl, size_t smem, cudaStream_t st) {
    const bool two = pl.nt == 2;
    switch (wk) {
        case W_FP8_GROUP:
            return two ? launch_stream<W_FP8_GROUP, 2>(prm, pl, smem, st) : launch_stream<W_FP8_GROUP, 1>(prm, pl, smem, st);
        case W_FP8_ROW:
            return two ? launch_stream<W_FP8_ROW, 2>(prm, pl, smem, st) : launch_stream<W_FP8_ROW, 1>(prm, pl, smem, st);
        default:
            return two ? launch_stream<W_F16, 2>(prm, pl, smem, st) : launch_stream<W_F16, 1>(prm, pl, smem, st);
    }
}

// Whether the streaming kernel's layout rules hold; otherwise the scalar kernel runs.
bool stream_ok(int wk, const void* x, const void* w, const void* s, const void* y, int K, int y_f32) {
    const int pos = (wk == W_F16) ? 32 : 64;
    if (K <= 0 || K % pos != 0) return false;
    if (!aligned(x, 16) || !aligned(w, 16)) return false;
    if (y != nullptr && !aligned(y, y_f32 ? 4 : 2)) return false;
    if (wk == W_FP8_GROUP && !aligned(s, 2)) return false;
    if (wk == W_FP8_ROW && s != nullptr && !aligned(s, 4)) return false;
    return true;
}

// Runs one pass of <= 16 tokens.
// Fused prologue / epilogues of the one-token kernel (GemvParams has the meaning).
struct Fused {
    const float* norm_w = nullptr;
    float eps = 0.f;
    __half* xn_out = nullptr;
    const __half* res = nullptr;
    __half* aux = nullptr;
    const uint8_t* w2 = nullptr;   // non-null: gate/up + SwiGLU
    const void* s2 = nullptr;
};

af_status run_gemv(int wk, const __half* x, const uint8_t* w, const void* s, void* y, int y_f32, int M, int N,
                   int K, int* arg_out, int arg_limit, void* ws, size_t ws_bytes, cudaStream_t st,
                   const af_tp_comm* tp = nullptr, int tp_arg_off = 0, const Fused* fz = nullptr) {
    const bool pair = fz != nullptr && fz->w2 != nullptr;
    int sms = device_sm_count();
    if (sms <= 0) return AF_ERR_CUDA;
    if (!stream_ok(wk, x, w, s, y, K, y_f32) || (arg_out != nullptr && M != 1)) {
        if (arg_out != nullptr || tp != nullptr || fz != nullptr) return AF_ERR_UNSUPPORTED;
        const int skind = (wk == W_FP8_GROUP) ? AF_SCALE_GROUP_F16 : (wk == W_FP8_ROW) ? AF_SCALE_ROW_F32 : AF_SCALE_NONE;
        dim3 grid((N + 7) / 8, M);
        cudaError_t e = launch_pdl(gemv_simple_kernel, grid, dim3(256), 0, st, w, (int)(wk == W_F16), s, skind,
                                   K / 128, x, y, y_f32, M, N, K);
        return e == cudaSuccess ? AF_OK : cuda_fail(e, "gemv_simple_kernel");
    }
    const int nt = (M <= 8) ? 1 : 2;
    Plan pl = make_plan(nt, N, K, wk, sms, arg_out != nullptr);
    if (pl.total > 0) {
        if (ws == nullptr || ws_bytes < pl.total) return AF_ERR_WORKSPACE;
        if (!aligned(ws, 256)) return AF_ERR_INVALID;
    }
    unsigned char* wsb = static_cast<unsigned char*>(ws);
    GemvParams prm{};
    prm.w = w;
    prm.s = s;
    prm.x = x;
    prm.y = y;
    prm.M = M;
    prm.N = N;
    prm.K = K;
    prm.G = K / 128;
    prm.cpt = pl.cpt;
    prm.y_f32 = y_f32;
    prm.arg_out = arg_out;
    if (arg_out != nullptr) {
        prm.arg_val = reinterpret_cast<float*>(wsb + pl.off_argv);
        prm.arg_idx = reinterpret_cast<int*>(wsb + pl.off_argi);
        prm.arg_done = reinterpret_cast<int*>(wsb + pl.off_done);
    }
    prm.arg_limit = arg_limit;
    if (fz != nullptr) {
        prm.norm_w = fz->norm_w;
        prm.norm_eps = fz->eps;
        prm.xn_out = fz->xn_out;
        prm.res = fz->res;
        prm.aux = fz->aux;
        prm.w2 = fz->w2;
        prm.s2 = fz->s2;
    }
    if (tp != nullptr) {
        prm.tp_world = tp->world;
        prm.tp_rank = tp->rank;
        prm.tp_nmax = tp->nmax;
        prm.tp_wait_ns = tp->wait_ns;
        prm.tp_arg = arg_out != nullptr;
        prm.arg_off = tp_arg_off;
        for (int r = 0; r < tp->world; ++r) prm.tp_buf[r] = tp->peer[r];
        if (arg_out == nullptr && N > tp->nmax) return AF_ERR_UNSUPPORTED;
    }
    // Shared memory: the ring, staged x and scales (when they fit), warp partials.
    const size_t ring = (size_t)kWarpsPerCta * kRingSlots * 1024;
    const size_t slots = (size_t)kWarpsPerCta * 2 * 32 * 4 * nt * sizeof(float);
    const size_t budget = kSmemMax - 1024;   // static shared and alignment
    size_t sc = 0;
    if (wk == W_FP8_GROUP && aligned(s, 16) && ((size_t)N * (K / 128) * 2) % 16 == 0 &&
        (!pair || aligned(fz->s2, 16))) {
        const size_t rows = (size_t)(N + pl.grid - 1) / pl.grid;
        sc = round_up(rows * (K / 128) * 2 + 32, 128) * (pair ? 2 : 1);
        if (ring + slots + sc > budget || sc > 32 * 1024) sc = 0;
    }
    const size_t gam = (fz != nullptr && fz->norm_w != nullptr) ? round_up((size_t)K * 4, 128) : 0;
    // 2..8 tokens: the one-token kernel with the tokens in the MMA's columns.
    if (M >= 2 && M <= 16 && fz == nullptr && tp == nullptr && arg_out == nullptr && wk != W_F16 &&
        K % 128 == 0 && aligned(x, 16)) {
        const size_t stride = (size_t)K + 8;   // halves: token rows 16 B apart modulo 128
        const size_t xs1 = round_up((size_t)M * stride * 2, 128);
        const size_t sc1 = (sc && sc <= 16 * 1024) ? sc : 0;
        struct Opt { int ns; size_t cap; };
        const Opt opts[4] = {{5, 113 * 1024}, {3, 113 * 1024}, {5, kSmemMax - 1024}, {3, kSmemMax - 1024}};
        for (const Opt& o : opts) {
            for (size_t scx : {sc1, (size_t)0}) {
                const size_t smem1 = (size_t)8 * o.ns * 2048 + xs1 + scx;
                if (smem1 > o.cap) continue;
                prm.xs_stride = (int)stride;
                prm.pre = o.ns;
                prm.xs_bytes = (int)xs1;
                prm.sc_bytes = (int)scx;
                cudaError_t e;
#define AF_MT(NS, T) (wk == W_FP8_GROUP ? launch_m1<true, false, 8, NS, false, T>(prm, pl, smem1, st) \
                                       : launch_m1<false, false, 8, NS, false, T>(prm, pl, smem1, st))
                if (M > 8) e = o.ns == 5 ? AF_MT(5, 16) : AF_MT(3, 16);
                else e = o.ns == 5 ? AF_MT(5, 8) : AF_MT(3, 8);
#undef AF_MT
                return e == cudaSuccess ? AF_OK : cuda_fail(e, "gemv_fp8_m1_kernel (tokens in MMA columns)");
            }
        }
    }
    // The decode case -- one token, FP8 weights, whole 128-wide groups -- has
    // its own kernel, sized so that two CTAs (of consecutive GEMVs) share an SM.
    if (M == 1 && (wk == W_F16 ? K % 64 : K % 128) == 0 && aligned(x, 16)) {
        // (warps, ring slots): 8 warps with a 5-slot ring (80 KB, two CTAs per SM),
        // or 3 slots when the staged x / scales / norm weight need the room.
        struct Cfg { int nw, ns; };
        const Cfg cfgs[2] = {{8, 5}, {8, 3}};
        const size_t xs1 = round_up((size_t)K * 2, 128);
        const size_t sc1 = (sc && sc <= (pair ? 32 : 16) * 1024) ? sc : 0;
        for (const Cfg& cf : cfgs) {
            const size_t cap = 113 * 1024;   // two CTAs per SM
            const size_t slots1 = 0;   // the warp partials reuse the ring
            const size_t ring1 = (size_t)cf.nw * cf.ns * 2048;   // >= the 1 KB per warp the partials need
            for (size_t scx : {sc1, (size_t)0}) {
                if (ring1 + slots1 + xs1 + scx + gam > cap) continue;
                prm.xs_stride = 0;
                prm.pre = cf.ns;
                prm.xs_bytes = (int)xs1;
                prm.sc_bytes = (int)scx;
                prm.gam_bytes = (int)gam;
                const size_t smem1 = ring1 + xs1 + scx + gam + slots1;
                cudaError_t e;
                const bool grp = wk == W_FP8_GROUP, f16 = wk == W_F16;
#define AF_M1(NW, NS) (pair ? launch_m1<true, false, NW, NS, true>(prm, pl, smem1, st) \
                       : grp ? launch_m1<true, false, NW, NS>(prm, pl, smem1, st) \
                       : f16 ? launch_m1<false, true, NW, NS>(prm, pl, smem1, st) \
                             : launch_m1<false, false, NW, NS>(prm, pl, smem1, st))
                e = cf.ns == 5 ? AF_M1(8, 5) : AF_M1(8, 3);
#undef AF_M1
                return e == cudaSuccess ? AF_OK : cuda_fail(e, "gemv_fp8_m1_kernel");
            }
        }
    }
    // the all-reduce and the fused prologue / epilogues are the one-token kernel's
    if (tp != nullptr || fz != nullptr) return AF_ERR_UNSUPPORTED;
    const size_t stride = (size_t)K + kXsPad;
    size_t xs = round_up((size_t)M * stride * sizeof(__half), 128);
    if (ring + slots + sc + xs > budget) sc = 0;   // scales from L2 before giving up staged x
    if (ring + slots + sc + xs > budget) xs = 0;   // then x from L2
    prm.xs_stride = xs ? (int)stride : 0;
    prm.xs_bytes = (int)xs;
    prm.sc_bytes = (int)sc;
    cudaError_t e = dispatch(wk, prm, pl, ring + xs + sc + slots, st);
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "gemv_stream_kernel");
}

int wkind_of(af_scale_kind kind) { return kind == AF_SCALE_GROUP_F16 ? W_FP8_GROUP : W_FP8_ROW; }

}  // namespace
}  // namespace af

unsigned af::gemv_faults(bool clear, cudaError_t* err) {
    unsigned v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemv_faults, sizeof(v));
    if (e == cudaSuccess && clear && v != 0) {
        const unsigned z = 0;
        e = cudaMemcpyToSymbol(g_gemv_faults, &z, sizeof(z));
    }
    *err = e;
    return v;
}

using namespace af;

extern "C" size_t af_w8a16_gemv_workspace_bytes(int M, int N, int K, af_scale_kind kind) {
    // The GEMV needs no device scratch; the size query stays part of the ABI.
    (void)M, (void)N, (void)K, (void)kind;
    return 0;
}

extern "C" af_status af_w8a16_gemv(const void* x, const void* w, const void* scales, void* y,
                                   int M, int N, int K, int group_size, af_scale_kind kind,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    if (M < 0 || N < 0 || K < 0) return AF_ERR_INVALID;
    if (kind != AF_SCALE_GROUP_F16 && kind != AF_SCALE_ROW_F32 && kind != AF_SCALE_NONE)
        return AF_ERR_INVALID;
    if (kind == AF_SCALE_GROUP_F16 && (group_size != 128 || K % 128 != 0)) return AF_ERR_INVALID;
    if (kind == AF_SCALE_NONE && scales != nullptr) return AF_ERR_INVALID;
    if (M == 0 || N == 0) return AF_OK;
    if (x == nullptr || w == nullptr || y == nullptr) return AF_ERR_INVALID;
    if (kind != AF_SCALE_NONE && scales == nullptr) return AF_ERR_INVALID;
    if (!aligned(y, 2)) return AF_ERR_INVALID;   // an FP16 output is 2-byte aligned
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int wk = wkind_of(kind);
    for (int m0 = 0; m0 < M; m0 += 16) {
        const int mb = (M - m0 < 16) ? (M - m0) : 16;
        af_status r = run_gemv(wk, static_cast<const __half*>(x) + (size_t)m0 * K,
                               static_cast<const uint8_t*>(w), scales,
                               static_cast<__half*>(y) + (size_t)m0 * N, 0, mb, N, K, nullptr, 0,
                               workspace, workspace_bytes, st);
        if (r != AF_OK) return r;
    }
    return AF_OK;
}

extern "C" size_t af_lm_head_workspace_bytes(int V, int D, af_weight_dtype w_dtype) {
    if (V <= 0 || D <= 0) return 256;
    const int sms = device_sm_count();
    if (sms <= 0) return 0;
    const int wk = (w_dtype == AF_W_F16) ? W_F16 : W_FP8_ROW;
    const int pos = (wk == W_F16) ? 32 : 64;
    // The unaligned fallback runs the standalone argmax in the same workspace.
    const size_t arg = af_argmax_workspace_bytes(V);
    if (D % pos != 0) return arg;
    const size_t t = make_plan(1, V, D, wk, sms, true).total;
    return t > arg ? t : arg;
}

extern "C" af_status af_lm_head_gemv(const void* x, const void* w, af_weight_dtype w_dtype,
                                     const float* row_scale, float* logits, int V, int D,
                                     int* d_argmax, af_argmax_mode mode, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    if (V < 0 || D < 0) return AF_ERR_INVALID;
    if (w_dtype != AF_W_F16 && w_dtype != AF_W_FP8_E4M3) return AF_ERR_INVALID;
    if (w_dtype == AF_W_F16 && row_scale != nullptr) return AF_ERR_INVALID;
    if (w_dtype == AF_W_FP8_E4M3 && row_scale == nullptr) return AF_ERR_INVALID;
    if (mode != AF_ARGMAX_TRUE && mode != AF_ARGMAX_REF_COMPAT) return AF_ERR_INVALID;
    if (V == 0) return AF_OK;
    if (x == nullptr || w == nullptr || (logits == nullptr && d_argmax == nullptr))
        return AF_ERR_INVALID;
    if ((logits != nullptr && !aligned(logits, 4)) || (d_argmax != nullptr && !aligned(d_argmax, 4)))
        return AF_ERR_INVALID;
    const int wk = (w_dtype == AF_W_F16) ? W_F16 : W_FP8_ROW;
    const int limit = (mode == AF_ARGMAX_REF_COMPAT && V > 65536) ? 65536 : V;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (D == 0 || !stream_ok(wk, x, w, row_scale, logits, D, 1)) {
        // Unaligned or ragged D: scalar projection, then the standalone argmax.
        if (logits == nullptr) return AF_ERR_INVALID;
        af_status r = run_gemv(wk, static_cast<const __half*>(x), static_cast<const uint8_t*>(w),
                               row_scale, logits, 1, 1, V, D, nullptr, 0, workspace,
                               workspace_bytes, st);
        if (r != AF_OK || d_argmax == nullptr) return r;
        return af_argmax_f32(logits, V, d_argmax, mode, workspace, workspace_bytes, stream);
    }
    return run_gemv(wk, static_cast<const __half*>(x), static_cast<const uint8_t*>(w), row_scale,
                    logits, 1, 1, V, D, d_argmax, limit, workspace, workspace_bytes, st);
}

extern "C" af_status af_w8a16_gemv_allreduce(const void* x, const void* w, const void* scales, void* y, int N,
                                             int K, int group_size, af_scale_kind kind, af_tp_comm* comm,
                                             void* stream) {
    if (comm == nullptr || N <= 0 || K <= 0) return AF_ERR_INVALID;
    if (kind != AF_SCALE_GROUP_F16 && kind != AF_SCALE_ROW_F32) return AF_ERR_INVALID;
    if (kind == AF_SCALE_GROUP_F16 && (group_size != 128 || K % 128 != 0)) return AF_ERR_INVALID;
    if (x == nullptr || w == nullptr || y == nullptr || scales == nullptr || !aligned(y, 2)) return AF_ERR_INVALID;
    for (int r = 0; r < comm->world; ++r)
        if (comm->peer[r] == nullptr) return AF_ERR_INVALID;   // peers not opened
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) return AF_ERR_INVALID;
    if (comm->world == 1)
        return af_w8a16_gemv(x, w, scales, y, 1, N, K, group_size, kind, nullptr, 0, stream);
    if (K % 128 != 0 || !aligned(x, 16) || !aligned(w, 16)) return AF_ERR_UNSUPPORTED;
    return run_gemv(wkind_of(kind), static_cast<const __half*>(x), static_cast<const uint8_t*>(w), scales, y, 0, 1,
                    N, K, nullptr, 0, nullptr, 0, static_cast<cudaStream_t>(stream), comm);
}

extern "C" af_status af_lm_head_gemv_tp(const void* x, const void* w, af_weight_dtype w_dtype, const float* row_scale,
                                        float* logits, int V_local, int D, int vocab_offset, int* d_argmax,
                                        af_argmax_mode mode, void* workspace, size_t workspace_bytes,
                                        af_tp_comm* comm, void* stream) {
    if (comm == nullptr || V_local <= 0 || D <= 0 || vocab_offset < 0 || d_argmax == nullptr) return AF_ERR_INVALID;
    if (w_dtype != AF_W_F16 && w_dtype != AF_W_FP8_E4M3) return AF_ERR_INVALID;
    if ((w_dtype == AF_W_F16) != (row_scale == nullptr)) return AF_ERR_INVALID;
    if (mode != AF_ARGMAX_TRUE && mode != AF_ARGMAX_REF_COMPAT) return AF_ERR_INVALID;
    if (x == nullptr || w == nullptr || !aligned(d_argmax, 4) || (logits != nullptr && !aligned(logits, 4)))
        return AF_ERR_INVALID;
    for (int r = 0; r < comm->world; ++r)
        if (comm->peer[r] == nullptr) return AF_ERR_INVALID;   // peers not opened
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) return AF_ERR_INVALID;
    if (comm->world == 1)
        return af_lm_head_gemv(x, w, w_dtype, row_scale, logits, V_local, D, d_argmax, mode, workspace,
                               workspace_bytes, stream);
    const int wk = (w_dtype == AF_W_F16) ? W_F16 : W_FP8_ROW;
    if ((wk == W_F16 ? D % 64 : D % 128) != 0 || !aligned(x, 16) || !aligned(w, 16))
        return AF_ERR_UNSUPPORTED;
    // ref-compat: only global ids < 65536 are candidates
    long long lim = V_local;
    if (mode == AF_ARGMAX_REF_COMPAT) lim = std::max(0ll, std::min<long long>(V_local, 65536ll - vocab_offset));
    return run_gemv(wk, static_cast<const __half*>(x), static_cast<const uint8_t*>(w), row_scale, logits, 1, 1,
                    V_local, D, d_argmax, (int)lim, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                    comm, vocab_offset);
}

// ------------------------------------------------- fused decode-layer ops
namespace {
af_status fused_checks(const void* x, const void* w, const void* scales, const void* y, int N, int K,
                       int group_size, af_scale_kind kind) {
    if (N <= 0 || K <= 0 || x == nullptr || w == nullptr || y == nullptr || scales == nullptr) return AF_ERR_INVALID;
    if (kind != AF_SCALE_GROUP_F16 && kind != AF_SCALE_ROW_F32) return AF_ERR_INVALID;
    if (kind == AF_SCALE_GROUP_F16 && group_size != 128) return AF_ERR_INVALID;
    if (K % 128 != 0 || !aligned(y, 2)) return AF_ERR_INVALID;
    if (!aligned(x, 16) || !aligned(w, 16)) return AF_ERR_UNSUPPORTED;
    return AF_OK;
}
}  // namespace

extern "C" af_status af_rmsnorm_w8a16_gemv(const void* x, const float* norm_w, float eps, const void* w,
                                          const void* scales, void* y, int N, int K, int group_size,
                                          af_scale_kind kind, void* x_norm_out, void* stream) {
    af_status r = fused_checks(x, w, scales, y, N, K, group_size, kind);
    if (r != AF_OK) return r;
    if (norm_w == nullptr || !aligned(norm_w, 16) || (x_norm_out != nullptr && !aligned(x_norm_out, 2)))
        return AF_ERR_INVALID;
    Fused fz;
    fz.norm_w = norm_w;
    fz.eps = eps;
    fz.xn_out = static_cast<__half*>(x_norm_out);
    return run_gemv(wkind_of(kind), static_cast<const __half*>(x), static_cast<const uint8_t*>(w), scales, y, 0, 1,
                    N, K, nullptr, 0, nullptr, 0, static_cast<cudaStream_t>(stream), nullptr, 0, &fz);
}

extern "C" af_status af_w8a16_gemv_residual(const void* x, const void* w, const void* scales, void* inout, int N,
                                           int K, int group_size, af_scale_kind kind, void* y_out, void* stream) {
    af_status r = fused_checks(x, w, scales, inout, N, K, group_size, kind);
    if (r != AF_OK) return r;
    if (y_out != nullptr && !aligned(y_out, 2)) return AF_ERR_INVALID;
    Fused fz;
    fz.res = static_cast<const __half*>(inout);
    fz.aux = static_cast<__half*>(y_out);
    return run_gemv(wkind_of(kind), static_cast<const __half*>(x), static_cast<const uint8_t*>(w), scales, inout, 0,
                    1, N, K, nullptr, 0, nullptr, 0, static_cast<cudaStream_t>(stream), nullptr, 0, &fz);
}

extern "C" af_status af_rmsnorm_w8a16_swiglu(const void* x, const float* norm_w, float eps, const void* w_gate,
                                            const void* s_gate, const void* w_up, const void* s_up, void* h, int N,
                                            int K, int group_size, af_scale_kind kind, void* gate_up_out,
                                            void* x_norm_out, void* stream) {
    af_status r = fused_checks(x, w_gate, s_gate, h, N, K, group_size, kind);
    if (r != AF_OK) return r;
    if (w_up == nullptr || s_up == nullptr) return AF_ERR_INVALID;
    if (kind != AF_SCALE_GROUP_F16 || !aligned(w_up, 16)) return AF_ERR_UNSUPPORTED;
    if (norm_w != nullptr && !aligned(norm_w, 16)) return AF_ERR_INVALID;
    if ((gate_up_out != nullptr && !aligned(gate_up_out, 2)) || (x_norm_out != nullptr && !aligned(x_norm_out, 2)))
        return AF_ERR_INVALID;
    if (norm_w == nullptr && x_norm_out != nullptr) return AF_ERR_INVALID;
    Fused fz;
    fz.norm_w = norm_w;
    fz.eps = eps;
    fz.xn_out = static_cast<__half*>(x_norm_out);
    fz.aux = static_cast<__half*>(gate_up_out);
    fz.w2 = static_cast<const uint8_t*>(w_up);
    fz.s2 = s_up;
    return run_gemv(W_FP8_GROUP, static_cast<const __half*>(x), static_cast<const uint8_t*>(w_gate), s_gate, h, 0,
                    1, N, K, nullptr, 0, nullptr, 0, static_cast<cudaStream_t>(stream), nullptr, 0, &fz);
}

extern "C" af_status af_w8a16_gemv_allreduce_residual(const void* x, const void* w, const void* scales, void* inout,
                                                     int N, int K, int group_size, af_scale_kind kind,
                                                     af_tp_comm* comm, void* stream) {
    if (comm == nullptr) return AF_ERR_INVALID;
    af_status r = fused_checks(x, w, scales, inout, N, K, group_size, kind);
    if (r != AF_OK) return r;
    for (int q = 0; q < comm->world; ++q)
        if (comm->peer[q] == nullptr) return AF_ERR_INVALID;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) return AF_ERR_INVALID;
    Fused fz;
    fz.res = static_cast<const __half*>(inout);
    return run_gemv(wkind_of(kind), static_cast<const __half*>(x), static_cast<const uint8_t*>(w), scales, inout, 0,
                    1, N, K, nullptr, 0, nullptr, 0, static_cast<cudaStream_t>(stream),
                    comm->world > 1 ? comm : nullptr, 0, &fz);
}
