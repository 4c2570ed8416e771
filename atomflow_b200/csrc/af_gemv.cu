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
//   * The weight matrix is cut into 16-row tiles and each tile's K range into
//     "chunks" (64 FP8 or 32 FP16 positions = 64 B of each of the 16 rows).
//     The grid is one CTA per SM; the tiles*chunks list is split into equal
//     contiguous ranges, one per CTA, so every SM streams the same number of
//     bytes whatever N and K are.  Split-K happens wherever a range boundary
//     falls inside a tile.
//   * Each CTA is one producer warp and eight consumer warps.  The producer
//     streams "stages" (16 rows x up to 16 chunks = up to 16 KB) into a ring
//     of shared-memory slots with 1-D bulk copies (cp.async.bulk, one per row)
//     that complete on per-slot mbarriers.  The producer never reads anything
//     a previous kernel writes, so it runs ahead of griddepcontrol.wait: with
//     programmatic dependent launch a GEMV fills its ring (~100 KB per SM, a
//     whole 3072x3072 GEMV) while the previous kernel of the stream drains.
//     Two CTAs fit per SM (<= 113 KB shared memory each), one from each of two
//     consecutive kernels.
//   * Consumers wait for griddepcontrol.wait, stage x in shared memory, then
//     take two chunks of every stage each.  FP8 bytes become FP16 with the
//     packed cvt (exact) and the dot products run on the tensor cores as
//     m16n8k16 MMAs: W rows are the MMA's M, tokens its N (M = 1 uses one
//     column; up to 16 tokens share one pass over W).  Every MMA starts from a
//     zero accumulator and its result is added in FP32 registers, which keeps
//     cancellation error at the level of an FFMA chain.
//   * Group scales are applied to each 64-position chunk sum (a scale group
//     never straddles a chunk); row scales after the reduction.
//   * At the end of a tile segment the eight warps' partials are summed in
//     shared memory in warp order.  Segments of a tile split across CTAs leave
//     FP32 partials in a workspace; the last CTA to finish the tile
//     (per-tile arrival counter) sums them in slot order -- so results are
//     deterministic -- stores the output and resets the counter for the next
//     call / graph replay.
//   * The lm_head variant writes FP32 logits and folds the greedy argmax into
//     the epilogue (per-CTA candidates, the last CTA reduces).
//   * Every mbarrier wait is bounded (globaltimer); a wait that gives up sets a
//     sticky error word in the workspace and the kernel unwinds without
//     breaking its barrier protocol.

#include <cuda_fp8.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "af_common.cuh"
#include "af_internal.h"

namespace af {

enum WKind { W_FP8_GROUP = 0, W_FP8_ROW = 1, W_F16 = 2 };

constexpr int kCW = 8;                       // consumer warps
constexpr int kThreads = (kCW + 1) * 32;     // + one producer warp
constexpr int kStageChunks = 16;             // chunks per stage
constexpr int kRowPitch = kStageChunks * 64 + 64;   // staged row pitch: == 64 (mod 128) -> conflict-free LDS.128
constexpr int kSlotBytes = 16 * kRowPitch;   // one stage: 16 rows
constexpr int kXsPad = 32;                   // halves of padding per staged x row (bank spread)
constexpr int kMaxStages = 8;

struct GemvParams {
    const uint8_t* w;
    const void* s;        // FP16 [N,G] group scales | FP32 [N] row scales | null
    const __half* x;      // [M, K]
    void* y;              // [M, N] FP16 or FP32 (null: no store)
    int M, N, K, G;
    int tiles, cpt;       // 16-row tiles, chunks per tile
    long long C;          // tiles * cpt
    int ms;               // partial slots per tile
    int ns;               // ring stages
    int xs_stride;        // staged x row stride in halves (0: read x from global)
    int xs_bytes;         // shared bytes reserved for x
    int y_f32;
    int* cnt;             // [tiles] arrival counters (zero between calls)
    float* part;          // [tiles][ms][32 lanes][4*NT]
    int* arg_out;         // fused argmax result (null: off)
    float* arg_val;       // [CTAs]
    int* arg_idx;         // [CTAs]
    int* arg_done;        // [1]
    int arg_limit;        // rows >= arg_limit are not argmax candidates
    int* status;          // sticky error word (bit 0: a bounded wait gave up)
    unsigned long long wait_ns;
};

__device__ __forceinline__ uint32_t u4w(const uint4& v, int t) {
    return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}

struct Stage {
    long long cur;   // first chunk (global index)
    int tile, kc0, n;
};

__device__ __forceinline__ Stage stage_at(long long cur, long long c1, int cpt) {
    Stage st;
    st.cur = cur;
    st.tile = (int)(cur / cpt);
    st.kc0 = (int)(cur - (long long)st.tile * cpt);
    int n = kStageChunks;
    if (cpt - st.kc0 < n) n = cpt - st.kc0;
    if (c1 - cur < n) n = (int)(c1 - cur);
    st.n = n;
    return st;
}

template <int WK, int NT>
__global__ void __launch_bounds__(kThreads, 2) gemv_stream_kernel(const GemvParams p) {
    constexpr int POS = (WK == W_F16) ? 32 : 64;   // positions per chunk
    constexpr int LPOS = POS / 4;                  // positions per lane per row
    constexpr int XU4 = LPOS / 8;                  // uint4 of x per lane per chunk
    constexpr int MT = 8 * NT;                     // token columns

    pdl_launch_dependents();
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* ring = smem;
    __half* xs = reinterpret_cast<__half*>(smem + (size_t)p.ns * kSlotBytes);
    float* red = reinterpret_cast<float*>(smem + (size_t)p.ns * kSlotBytes + p.xs_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(red) +
                                                 (size_t)kCW * 16 * MT * sizeof(float));
    volatile int* s_abort = reinterpret_cast<volatile int*>(bars + 2 * p.ns);
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + p.ns);

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int g = lane >> 2;
    const int c = lane & 3;
    const long long G = gridDim.x;
    const long long Ge = G < p.C ? G : p.C;   // CTAs that own chunks (each owns >= 1)
    const long long cta = blockIdx.x;
    const long long c0 = cta < Ge ? cta * p.C / Ge : p.C;
    const long long c1 = cta < Ge ? (cta + 1) * p.C / Ge : p.C;
    const size_t row_bytes = (size_t)p.K * ((WK == W_F16) ? 2 : 1);

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.ns; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kCW);
        }
        *s_abort = 0;
        mbar_init_fence();
    }
    __syncthreads();

    auto wait = [&](uint32_t bar, uint32_t parity) {
        const uint64_t lim = *s_abort ? 0ull : p.wait_ns;
        if (!mbar_wait_bounded(bar, parity, lim)) {
            if (!*s_abort) {
                *s_abort = 1;
                atomicOr(p.status, 1);
            }
        }
    };

    if (warp == kCW) {
        // ------------------------------------------------------ producer ---
        long long cur = c0;
        int j = 0;
        while (cur < c1) {
            const Stage st = stage_at(cur, c1, p.cpt);
            const int s = j % p.ns;
            const int round = j / p.ns;
            if (round > 0) wait(empty0 + 8 * s, (round - 1) & 1);
            if (*s_abort) break;
            const uint32_t bytes = (uint32_t)st.n * 64u;
            if (lane == 0) mbar_arrive_expect_tx(full0 + 8 * s, 16u * bytes);
            __syncwarp();
            if (lane < 16) {
                const int row = min(st.tile * 16 + lane, p.N - 1);
                const uint8_t* src = p.w + (size_t)row * row_bytes + (size_t)st.kc0 * 64;
                bulk_g2s(smem_u32(ring + (size_t)s * kSlotBytes + lane * kRowPitch), src, bytes, full0 + 8 * s);
            }
            cur += st.n;
            ++j;
        }
        // Do not leave while copies into this CTA's shared memory may still land.
        for (int k = (j > p.ns ? j - p.ns : 0); k < j; ++k) wait(full0 + 8 * (k % p.ns), (k / p.ns) & 1);
        return;
    }

    // -------------------------------------------------------- consumers ---
    const uint16_t* s16 = static_cast<const uint16_t*>(p.s);

    auto load_scales = [&](const Stage& st, uint32_t (&sc)[2]) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int i = warp + q * kCW;
            sc[q] = 0;
            if (WK == W_FP8_GROUP && i < st.n) {
                const int grp = (st.kc0 + i) >> 1;
                const int r0 = min(st.tile * 16 + g, p.N - 1);
                const int r1 = min(st.tile * 16 + g + 8, p.N - 1);
                sc[q] = (uint32_t)__ldg(s16 + (size_t)r0 * p.G + grp) |
                        ((uint32_t)__ldg(s16 + (size_t)r1 * p.G + grp) << 16);
            }
        }
    };

    Stage st{};
    uint32_t sc[2] = {0, 0};
    if (c0 < c1) {
        st = stage_at(c0, c1, p.cpt);
        load_scales(st, sc);
    }

    // Everything above touched only weights.  From here on we read the
    // activations and the workspace, which the previous kernel may own.
    pdl_wait();

    if (p.xs_stride > 0) {
        const int k8 = p.K >> 3;
        const int total = p.M * k8;
        for (int i = threadIdx.x; i < total; i += kCW * 32) {
            const int tok = i / k8;
            const int kk = (i - tok * k8) * 8;
            *reinterpret_cast<uint4*>(xs + (size_t)tok * p.xs_stride + kk) = ldcg_u4(p.x + (size_t)tok * p.K + kk);
        }
        named_bar_sync(1, kCW * 32);
    }

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

    // One chunk of a staged slot: rows g and g+8, 16 bytes each.
    auto do_chunk = [&](const unsigned char* slot, int i, int kc, uint32_t scp) {
        const uint4 w0 = *reinterpret_cast<const uint4*>(slot + g * kRowPitch + i * 64 + c * 16);
        const uint4 w1 = *reinterpret_cast<const uint4*>(slot + (g + 8) * kRowPitch + i * 64 + c * 16);
        const int pos = kc * POS + c * LPOS;
        uint32_t xf[NT][LPOS / 2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) load_x(min(nt * 8 + g, p.M - 1), pos, xf[nt]);
        float d[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int k = 0; k < 4; ++k) d[nt][k] = 0.f;
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

    float best_v = 0.f;   // fused argmax: running best of this lane (warp 0)
    int best_i = -1;

    auto emit = [&](int tile, float (&v)[NT][4]) {
        const int r0 = tile * 16 + g;
        const int r1 = r0 + 8;
        if (WK == W_FP8_ROW && p.s != nullptr) {
            const float* s32 = static_cast<const float*>(p.s);
            const float s0 = __ldg(s32 + min(r0, p.N - 1));
            const float s1 = __ldg(s32 + min(r1, p.N - 1));
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
                            if (r0 < p.N) y[r0] = v[nt][jj];
                            if (r1 < p.N) y[r1] = v[nt][2 + jj];
                        } else {
                            __half* y = static_cast<__half*>(p.y) + (size_t)tok * p.N;
                            if (r0 < p.N) y[r0] = __float2half_rn(v[nt][jj]);
                            if (r1 < p.N) y[r1] = __float2half_rn(v[nt][2 + jj]);
                        }
                    }
                }
            }
        }
        if (p.arg_out != nullptr && c == 0) {
            const int lim = min(p.N, p.arg_limit);
            if (r0 < lim && argmax_better(v[0][0], r0, best_v, best_i)) { best_v = v[0][0]; best_i = r0; }
            if (r1 < lim && argmax_better(v[0][2], r1, best_v, best_i)) { best_v = v[0][2]; best_i = r1; }
        }
    };

    // Warp 0 only: combine this CTA's sum for `tile` with other CTAs' segments.
    auto finish_tile = [&](int tile, float (&v)[NT][4]) {
        const long long start = (long long)tile * p.cpt;
        const long long end = start + p.cpt;
        const long long own_a = ((start + 1) * Ge - 1) / p.C;   // CTA owning chunk `start`
        const long long own_b = (end * Ge - 1) / p.C;           // CTA owning chunk `end - 1`
        const int count = (int)(own_b - own_a + 1);
        if (count == 1) {
            emit(tile, v);
            return;
        }
        const int slot = (int)(cta - own_a);
        float* dst = p.part + (((size_t)tile * p.ms + slot) * 32 + lane) * 4 * NT;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            __stcg(reinterpret_cast<float4*>(dst + 4 * nt), make_float4(v[nt][0], v[nt][1], v[nt][2], v[nt][3]));
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = (atomicAdd(p.cnt + tile, 1) == count - 1);
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) return;
        __threadfence();
        float r[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int k = 0; k < 4; ++k) r[nt][k] = 0.f;
        for (int sl = 0; sl < count; ++sl) {
            float* src = p.part + (((size_t)tile * p.ms + sl) * 32 + lane) * 4 * NT;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float4 f = ldcg_f4(src + 4 * nt);
                r[nt][0] += f.x;
                r[nt][1] += f.y;
                r[nt][2] += f.z;
                r[nt][3] += f.w;
                // leave the workspace all-zero: any op may reuse it next
                __stcg(reinterpret_cast<float4*>(src + 4 * nt), make_float4(0.f, 0.f, 0.f, 0.f));
            }
        }
        if (lane == 0) p.cnt[tile] = 0;
        emit(tile, r);
    };

    // All consumer warps: sum the eight warps' partials of `tile` in warp order.
    auto tile_end = [&](int tile) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const int tok = nt * 8 + 2 * c + jj;
                red[(warp * 16 + g) * MT + tok] = acc[nt][jj];
                red[(warp * 16 + g + 8) * MT + tok] = acc[nt][2 + jj];
            }
        named_bar_sync(1, kCW * 32);
        float v[NT][4];
        if (warp == 0) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    const int tok = nt * 8 + 2 * c + jj;
                    float a = 0.f, b = 0.f;
                    for (int w = 0; w < kCW; ++w) {
                        a += red[(w * 16 + g) * MT + tok];
                        b += red[(w * 16 + g + 8) * MT + tok];
                    }
                    v[nt][jj] = a;
                    v[nt][2 + jj] = b;
                }
        }
        named_bar_sync(1, kCW * 32);
        if (warp == 0) finish_tile(tile, v);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[nt][k] = 0.f;
    };

    long long cur = c0;
    int j = 0;
    while (cur < c1) {
        Stage nx{};
        uint32_t scn[2] = {0, 0};
        const bool has_next = cur + st.n < c1;
        if (has_next) {
            nx = stage_at(cur + st.n, c1, p.cpt);
            load_scales(nx, scn);   // one stage ahead: hides the scale loads' latency
        }
        const int s = j % p.ns;
        wait(full0 + 8 * s, (j / p.ns) & 1);
        const unsigned char* slot = ring + (size_t)s * kSlotBytes;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int i = warp + q * kCW;
            if (i < st.n) do_chunk(slot, i, st.kc0 + i, sc[q]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);
        if (st.kc0 + st.n == p.cpt || cur + st.n == c1) tile_end(st.tile);
        cur += st.n;
        ++j;
        st = nx;
        sc[0] = scn[0];
        sc[1] = scn[1];
    }

    if (p.arg_out != nullptr && warp == 0) {
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
            last = (atomicAdd(p.arg_done, 1) == (int)G - 1);
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence();
            float bv = 0.f;
            int bi = -1;
            for (long long i = lane; i < G; i += 32) {
                const float v = ldcg_f32(p.arg_val + i);
                const int ix = ldcg_s32(p.arg_idx + i);
                if (argmax_better(v, ix, bv, bi)) { bv = v; bi = ix; }
                __stcg(p.arg_val + i, 0.f);
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
        uint8_t* yb = static_cast<uint8_t*>(y);
        if (y_f32) {
            const uint32_t b = __float_as_uint(acc);
            uint8_t* dst = yb + ((size_t)m * N + n) * 4;
            dst[0] = b & 0xff;
            dst[1] = (b >> 8) & 0xff;
            dst[2] = (b >> 16) & 0xff;
            dst[3] = b >> 24;
        } else {
            const uint16_t b = __half_as_ushort(__float2half_rn(acc));
            uint8_t* dst = yb + ((size_t)m * N + n) * 2;
            dst[0] = b & 0xff;
            dst[1] = b >> 8;
        }
    }
}

// ----------------------------------------------------------------- host ---

namespace {

struct Plan {
    int grid;
    int nt;
    int tiles, cpt;
    long long C;
    int ms;
    size_t off_status, off_cnt, off_done, off_argv, off_argi, off_part, total;
};

Plan make_plan(int nt, int N, int K, int wk, int sms) {
    Plan pl{};
    pl.nt = nt;
    pl.grid = sms * ctas_per_sm();
    const long long G = pl.grid;
    const int pos = (wk == W_F16) ? 32 : 64;
    pl.tiles = (N + 15) / 16;
    pl.cpt = K / pos;
    pl.C = (long long)pl.tiles * pl.cpt;
    // Every active CTA owns q or q+1 chunks (q >= 1), so a tile of cpt chunks
    // is split among at most 1 + ceil((cpt - 1) / q) CTAs.
    const long long Ge = G < pl.C ? G : (pl.C > 0 ? pl.C : 1);
    const long long q = pl.C / Ge;
    long long ms = q > 0 ? 1 + (pl.cpt - 1 + q - 1) / q : pl.cpt;
    pl.ms = (int)(ms < pl.cpt ? ms : pl.cpt);
    if (pl.ms < 1) pl.ms = 1;
    size_t off = 0;
    pl.off_status = off;
    off = round_up(off + 4, 256);
    pl.off_cnt = off;
    off = round_up(off + (size_t)pl.tiles * 4, 256);
    pl.off_done = off;
    off = round_up(off + 4, 256);
    pl.off_argv = off;
    off = round_up(off + (size_t)G * 4, 256);
    pl.off_argi = off;
    off = round_up(off + (size_t)G * 4, 256);
    pl.off_part = off;
    off = round_up(off + (size_t)pl.tiles * pl.ms * 32 * 4 * nt * sizeof(float), 256);
    pl.total = off;
    return pl;
}

// Shared memory per CTA: two CTAs (of consecutive kernels) must fit on one SM.
size_t smem_budget() {
    static size_t v = [] {
        const char* e = getenv("AF_SMEM_BUDGET_KB");
        long k = e ? atol(e) : 113;
        if (k < 40 || k > 226) k = 113;
        return (size_t)k * 1024;
    }();
    return v;
}

unsigned long long wait_limit_ns() {
    static unsigned long long v = [] {
        const char* e = getenv("AF_WAIT_LIMIT_MS");
        long long ms = e ? atoll(e) : 2000;
        if (ms < 1) ms = 2000;
        return (unsigned long long)ms * 1000000ull;
    }();
    return v;
}

template <int WK, int NT>
cudaError_t launch_stream(const GemvParams& prm, const Plan& pl, size_t smem, cudaStream_t st) {
    auto kern = gemv_stream_kernel<WK, NT>;
    static std::once_flag flags[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    static cudaError_t attr_err[kMaxDevices];
    std::call_once(flags[dev % kMaxDevices], [&] {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared);
        attr_err[dev % kMaxDevices] = e;
    });
    if (attr_err[dev % kMaxDevices] != cudaSuccess) return attr_err[dev % kMaxDevices];
    return launch_pdl(kern, dim3(pl.grid), dim3(kThreads), smem, st, prm);
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
af_status run_gemv(int wk, const __half* x, const uint8_t* w, const void* s, void* y, int y_f32, int M, int N,
                   int K, int* arg_out, int arg_limit, void* ws, size_t ws_bytes, cudaStream_t st) {
    int sms = device_sm_count();
    if (sms <= 0) return AF_ERR_CUDA;
    if (!stream_ok(wk, x, w, s, y, K, y_f32) || (arg_out != nullptr && M != 1)) {
        if (arg_out != nullptr) return AF_ERR_UNSUPPORTED;
        const int skind = (wk == W_FP8_GROUP) ? AF_SCALE_GROUP_F16 : (wk == W_FP8_ROW) ? AF_SCALE_ROW_F32 : AF_SCALE_NONE;
        dim3 grid((N + 7) / 8, M);
        cudaError_t e = launch_pdl(gemv_simple_kernel, grid, dim3(256), 0, st, w, (int)(wk == W_F16), s, skind,
                                   K / 128, x, y, y_f32, M, N, K);
        return e == cudaSuccess ? AF_OK : cuda_fail(e, "gemv_simple_kernel");
    }
    const int nt = (M <= 8) ? 1 : 2;
    Plan pl = make_plan(nt, N, K, wk, sms);
    if (ws == nullptr || ws_bytes < pl.total) return AF_ERR_WORKSPACE;
    if (!aligned(ws, 256)) return AF_ERR_INVALID;
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
    prm.tiles = pl.tiles;
    prm.cpt = pl.cpt;
    prm.C = pl.C;
    prm.ms = pl.ms;
    prm.y_f32 = y_f32;
    prm.status = reinterpret_cast<int*>(wsb + pl.off_status);
    prm.cnt = reinterpret_cast<int*>(wsb + pl.off_cnt);
    prm.part = reinterpret_cast<float*>(wsb + pl.off_part);
    prm.arg_out = arg_out;
    prm.arg_val = reinterpret_cast<float*>(wsb + pl.off_argv);
    prm.arg_idx = reinterpret_cast<int*>(wsb + pl.off_argi);
    prm.arg_done = reinterpret_cast<int*>(wsb + pl.off_done);
    prm.arg_limit = arg_limit;
    prm.wait_ns = wait_limit_ns();
    // Shared memory: ring stages, staged x (when it leaves room for >= 3 stages),
    // the cross-warp reduction buffer and the mbarriers.
    const size_t budget = smem_budget();
    const size_t red = (size_t)kCW * 16 * (8 * nt) * sizeof(float);
    const size_t fixed = red + 2 * kMaxStages * 8 + 16;
    size_t xs = round_up((size_t)M * (K + kXsPad) * sizeof(__half), 128);
    if (fixed + xs + 3 * (size_t)kSlotBytes > budget) xs = 0;
    size_t ns = (budget - fixed - xs) / kSlotBytes;
    if (ns > (size_t)kMaxStages) ns = kMaxStages;
    if (ns < 2) return AF_ERR_UNSUPPORTED;
    prm.ns = (int)ns;
    prm.xs_stride = xs ? K + kXsPad : 0;
    prm.xs_bytes = (int)xs;
    const size_t smem = ns * kSlotBytes + xs + red + 2 * ns * 8 + 16;
    cudaError_t e = dispatch(wk, prm, pl, smem, st);
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "gemv_stream_kernel");
}

int wkind_of(af_scale_kind kind) { return kind == AF_SCALE_GROUP_F16 ? W_FP8_GROUP : W_FP8_ROW; }

}  // namespace
}  // namespace af

using namespace af;

extern "C" size_t af_w8a16_gemv_workspace_bytes(int M, int N, int K, af_scale_kind kind) {
    if (M <= 0 || N <= 0 || K <= 0) return 256;
    const int sms = device_sm_count();
    if (sms <= 0) return 0;
    const int nt = (M <= 8) ? 1 : 2;
    const int wk = wkind_of(kind);
    const int pos = 64;
    if (K % pos != 0) return 256;
    return make_plan(nt, N, K, wk, sms).total;
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
    const size_t t = make_plan(1, V, D, wk, sms).total;
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
