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
//     "chunks" (64 FP8 or 32 FP16 positions = 1 KB of one tile).  The grid is
//     one CTA of 8 warps per SM; the tiles*chunks list is split into equal
//     contiguous ranges, one per warp, so every warp streams the same number
//     of bytes whatever N and K are (split-K happens wherever a range boundary
//     falls inside a tile).
//   * A lane streams 16 B of two rows per chunk with L1-bypassing 128-bit
//     loads, four chunks per batch, double-buffered in registers.  The first
//     batch is issued before griddepcontrol.wait, so with programmatic
//     dependent launch a GEMV's weight stream starts while the previous kernel
//     of the stream is still running.
//   * FP8 bytes become FP16 with the packed cvt (exact), and the dot products
//     run on the tensor cores as m16n8k16 MMAs with FP32 accumulation: W rows
//     are the MMA's M, tokens the MMA's N (M = 1 uses column 0; up to 16
//     tokens share one pass over W).  This leaves ~1 ALU op per weight byte,
//     far under the issue budget at HBM rate, instead of the reference's
//     scalar convert-and-FMA chain.
//   * Group scales are applied to each 64-position partial (one scale group
//     never straddles a chunk); row scales after the reduction.
//   * Range boundaries inside a tile leave FP32 partials in a workspace;
//     the last warp to finish a tile (per-tile arrival counter) sums them in
//     slot order, so the result is deterministic, converts and stores, and
//     resets the counter for the next call / graph replay.
//   * The lm_head variant writes FP32 logits and folds the greedy argmax into
//     the epilogue (per-warp candidates, last warp reduces).

#include <cuda_fp8.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "af_common.cuh"
#include "af_internal.h"

namespace af {

enum WKind { W_FP8_GROUP = 0, W_FP8_ROW = 1, W_F16 = 2 };

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kNB = 4;                 // chunks per register batch
constexpr int kXsPad = 32;             // halves of padding per staged x row (bank spread)
constexpr size_t kXsMaxBytes = 100 * 1024;

struct GemvParams {
    const uint8_t* w;
    const void* s;        // FP16 [N,G] group scales | FP32 [N] row scales | null
    const __half* x;      // [M, K]
    void* y;              // [M, N] FP16 or FP32 (null: no store)
    int M, N, K, G;
    int tiles, cpt;       // 16-row tiles, chunks per tile
    long long C;          // tiles * cpt
    int ms;               // partial slots per tile
    int xs_stride;        // staged x row stride (halves)
    int y_f32;
    int* cnt;             // [tiles] arrival counters (zero between calls)
    float* part;          // [tiles][ms][32 lanes][4*NT]
    int* arg_out;         // fused argmax result (null: off)
    float* arg_val;       // [total warps]
    int* arg_idx;         // [total warps]
    int* arg_done;        // [1]
    int arg_limit;        // rows >= arg_limit are not argmax candidates
};

__device__ __forceinline__ uint32_t u4w(const uint4& v, int t) {
    return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}

template <int WK, int NT, bool XS>
__global__ void __launch_bounds__(kThreads, 2) gemv_stream_kernel(const GemvParams p) {
    constexpr int POS = (WK == W_F16) ? 32 : 64;   // positions per chunk
    constexpr int LPOS = POS / 4;                  // positions per lane per row
    constexpr int ESZ = (WK == W_F16) ? 2 : 1;     // weight bytes per element
    constexpr int XU4 = LPOS / 8;                  // uint4 of x per lane per chunk

    pdl_launch_dependents();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* xs = reinterpret_cast<__half*>(smem_raw);

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int g = lane >> 2;
    const int c = lane & 3;
    const long long GW = (long long)gridDim.x * kWarps;
    const long long gw = (long long)blockIdx.x * kWarps + warp;
    // Partition over GWe = min(warps, chunks) warps so that every warp that owns
    // part of a tile owns at least one chunk of it (the per-tile arrival count
    // below relies on this); warps beyond GWe stream nothing.
    const long long GWe = GW < p.C ? GW : p.C;
    const long long c0 = gw < GWe ? gw * p.C / GWe : p.C;
    const long long c1 = gw < GWe ? (gw + 1) * p.C / GWe : p.C;
    const size_t row_bytes = (size_t)p.K * ESZ;
    const uint16_t* s16 = static_cast<const uint16_t*>(p.s);

    uint4 wa[kNB][2], wb[kNB][2];
    uint32_t sa[kNB], sb[kNB];   // FP16 scales of rows g (low) and g+8 (high)

    auto issue = [&](uint4 (&wbuf)[kNB][2], uint32_t (&sbuf)[kNB], long long cur, int& n,
                     int& tile, int& kc0) {
        tile = (int)(cur / p.cpt);
        kc0 = (int)(cur - (long long)tile * p.cpt);
        long long left = c1 - cur;
        n = kNB;
        if (p.cpt - kc0 < n) n = p.cpt - kc0;
        if (left < n) n = (int)left;
        const int r0 = min(tile * 16 + g, p.N - 1);
        const int r1 = min(tile * 16 + g + 8, p.N - 1);
        const uint8_t* p0 = p.w + (size_t)r0 * row_bytes + (size_t)(kc0 * POS + c * LPOS) * ESZ;
        const uint8_t* p1 = p.w + (size_t)r1 * row_bytes + (size_t)(kc0 * POS + c * LPOS) * ESZ;
#pragma unroll
        for (int i = 0; i < kNB; ++i) {
            if (i < n) {
                wbuf[i][0] = ldg_stream(p0 + (size_t)i * POS * ESZ);
                wbuf[i][1] = ldg_stream(p1 + (size_t)i * POS * ESZ);
                if (WK == W_FP8_GROUP) {
                    const int grp = (kc0 + i) >> 1;   // 64-position chunk -> 128-wide group
                    sbuf[i] = (uint32_t)__ldg(s16 + (size_t)r0 * p.G + grp) |
                              ((uint32_t)__ldg(s16 + (size_t)r1 * p.G + grp) << 16);
                }
            }
        }
    };

    auto load_x = [&](int tok, int pos, uint32_t (&xf)[2 * LPOS / 4]) {
        // 2*LPOS/4 = LPOS/2 half2 registers = positions [pos, pos + LPOS)
#pragma unroll
        for (int u = 0; u < XU4; ++u) {
            uint4 v;
            if (XS)
                v = *reinterpret_cast<const uint4*>(xs + (size_t)tok * p.xs_stride + pos + u * 8);
            else
                v = ldcg_u4(p.x + (size_t)tok * p.K + pos + u * 8);
            xf[u * 4 + 0] = v.x;
            xf[u * 4 + 1] = v.y;
            xf[u * 4 + 2] = v.z;
            xf[u * 4 + 3] = v.w;
        }
    };

    auto compute = [&](const uint4 (&wbuf)[kNB][2], const uint32_t (&sbuf)[kNB], int n, int kc0,
                       float (&acc)[NT][4]) {
#pragma unroll
        for (int i = 0; i < kNB; ++i) {
            if (i < n) {
                const int pos = (kc0 + i) * POS + c * LPOS;
                uint32_t xf[NT][LPOS / 2];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) load_x(min(nt * 8 + g, p.M - 1), pos, xf[nt]);
                if (WK == W_F16) {
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        const uint32_t a0 = u4w(wbuf[i][0], 2 * t), a1 = u4w(wbuf[i][1], 2 * t);
                        const uint32_t a2 = u4w(wbuf[i][0], 2 * t + 1), a3 = u4w(wbuf[i][1], 2 * t + 1);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
                            mma16816(acc[nt], a0, a1, a2, a3, xf[nt][2 * t], xf[nt][2 * t + 1]);
                    }
                } else {
                    float d[NT][4];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int j = 0; j < 4; ++j) d[nt][j] = 0.f;
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const uint32_t w0 = u4w(wbuf[i][0], t), w1 = u4w(wbuf[i][1], t);
                        const uint32_t a0 = e4m3x2_lo(w0), a1 = e4m3x2_lo(w1);
                        const uint32_t a2 = e4m3x2_hi(w0), a3 = e4m3x2_hi(w1);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
                            mma16816(d[nt], a0, a1, a2, a3, xf[nt][2 * t], xf[nt][2 * t + 1]);
                    }
                    if (WK == W_FP8_GROUP) {
                        const float s0 = half_bits_to_float((uint16_t)(sbuf[i] & 0xffffu));
                        const float s1 = half_bits_to_float((uint16_t)(sbuf[i] >> 16));
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
                            for (int j = 0; j < 4; ++j) acc[nt][j] += d[nt][j];
                    }
                }
            }
        }
    };

    // Fused-argmax running best of this lane.
    float best_v = 0.f;
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
                for (int j = 0; j < 2; ++j) {
                    const int tok = nt * 8 + 2 * c + j;
                    if (tok < p.M) {
                        if (p.y_f32) {
                            float* y = static_cast<float*>(p.y) + (size_t)tok * p.N;
                            if (r0 < p.N) y[r0] = v[nt][j];
                            if (r1 < p.N) y[r1] = v[nt][2 + j];
                        } else {
                            __half* y = static_cast<__half*>(p.y) + (size_t)tok * p.N;
                            if (r0 < p.N) y[r0] = __float2half_rn(v[nt][j]);
                            if (r1 < p.N) y[r1] = __float2half_rn(v[nt][2 + j]);
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

    auto finish_tile = [&](int tile, float (&acc)[NT][4]) {
        const long long start = (long long)tile * p.cpt;
        const long long end = start + p.cpt;
        const long long own_a = ((start + 1) * GWe - 1) / p.C;   // warp owning chunk `start`
        const long long own_b = (end * GWe - 1) / p.C;           // warp owning chunk `end - 1`
        const int count = (int)(own_b - own_a + 1);
        if (count == 1) {
            emit(tile, acc);
            return;
        }
        const int slot = (int)(gw - own_a);
        float* dst = p.part + (((size_t)tile * p.ms + slot) * 32 + lane) * 4 * NT;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            __stcg(reinterpret_cast<float4*>(dst + 4 * nt),
                   make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]));
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = (atomicAdd(p.cnt + tile, 1) == count - 1);
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) return;
        __threadfence();
        float v[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 4; ++j) v[nt][j] = 0.f;
        for (int s = 0; s < count; ++s) {
            const float* src = p.part + (((size_t)tile * p.ms + s) * 32 + lane) * 4 * NT;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float4 f = ldcg_f4(src + 4 * nt);
                v[nt][0] += f.x;
                v[nt][1] += f.y;
                v[nt][2] += f.z;
                v[nt][3] += f.w;
            }
        }
        if (lane == 0) p.cnt[tile] = 0;
        emit(tile, v);
    };

    long long cur = c0;
    int nA = 0, tA = 0, kA = 0, nB = 0, tB = 0, kB = 0;
    if (cur < c1) issue(wa, sa, cur, nA, tA, kA);

    // Everything above touched only weights and scales.  From here on we read
    // the activations and the workspace, which the previous kernel may own.
    pdl_wait();

    if (XS) {
        const int k8 = p.K >> 3;
        const int total = p.M * k8;
        for (int i = threadIdx.x; i < total; i += kThreads) {
            const int tok = i / k8;
            const int kk = (i - tok * k8) * 8;
            *reinterpret_cast<uint4*>(xs + (size_t)tok * p.xs_stride + kk) =
                ldcg_u4(p.x + (size_t)tok * p.K + kk);
        }
        __syncthreads();
    }

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[nt][j] = 0.f;

    auto reset_acc = [&]() {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[nt][j] = 0.f;
    };

    while (cur < c1) {
        long long nxt = cur + nA;
        if (nxt < c1) issue(wb, sb, nxt, nB, tB, kB);
        compute(wa, sa, nA, kA, acc);
        if (nxt == c1 || kA + nA == p.cpt) {
            finish_tile(tA, acc);
            reset_acc();
        }
        cur = nxt;
        if (cur >= c1) break;
        nxt = cur + nB;
        if (nxt < c1) issue(wa, sa, nxt, nA, tA, kA);
        compute(wb, sb, nB, kB, acc);
        if (nxt == c1 || kB + nB == p.cpt) {
            finish_tile(tB, acc);
            reset_acc();
        }
        cur = nxt;
    }

    if (p.arg_out != nullptr) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (argmax_better(ov, oi, best_v, best_i)) { best_v = ov; best_i = oi; }
        }
        int last = 0;
        if (lane == 0) {
            __stcg(p.arg_val + gw, best_v);
            __stcg(p.arg_idx + gw, best_i);
            __threadfence();
            last = (atomicAdd(p.arg_done, 1) == (int)GW - 1);
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence();
            float bv = 0.f;
            int bi = -1;
            for (long long i = lane; i < GW; i += 32) {
                const float v = ldcg_f32(p.arg_val + i);
                const int ix = ldcg_s32(p.arg_idx + i);
                if (argmax_better(v, ix, bv, bi)) { bv = v; bi = ix; }
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
            __half h;
            memcpy(&h, w + ((size_t)n * K + k) * 2, 2);
            wv = __half2float(h);
        } else {
            const __half_raw hr = __nv_cvt_fp8_to_halfraw(w[(size_t)n * K + k], __NV_E4M3);
            wv = __half2float(__half(hr));
        }
        if (skind == AF_SCALE_GROUP_F16) {
            uint16_t sb;
            memcpy(&sb, static_cast<const uint8_t*>(s) + ((size_t)n * G + k / 128) * 2, 2);
            wv *= half_bits_to_float(sb);
        }
        __half xh;
        memcpy(&xh, reinterpret_cast<const uint8_t*>(x) + ((size_t)m * K + k) * 2, 2);
        acc = fmaf(wv, __half2float(xh), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
        if (skind == AF_SCALE_ROW_F32 && s != nullptr) {
            float sv;
            memcpy(&sv, static_cast<const uint8_t*>(s) + (size_t)n * 4, 4);
            acc *= sv;
        }
        if (y_f32) {
            uint8_t* dst = static_cast<uint8_t*>(y) + ((size_t)m * N + n) * 4;
            memcpy(dst, &acc, 4);
        } else {
            const __half h = __float2half_rn(acc);
            uint8_t* dst = static_cast<uint8_t*>(y) + ((size_t)m * N + n) * 2;
            memcpy(dst, &h, 2);
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
    size_t off_cnt, off_done, off_argv, off_argi, off_part, total;
};

Plan make_plan(int nt, int N, int K, int wk, int sms) {
    Plan pl{};
    pl.nt = nt;
    pl.grid = sms * ctas_per_sm();
    const long long GW = (long long)pl.grid * kWarps;
    const int pos = (wk == W_F16) ? 32 : 64;
    pl.tiles = (N + 15) / 16;
    pl.cpt = K / pos;
    pl.C = (long long)pl.tiles * pl.cpt;
    // Every active warp owns q or q+1 chunks (q >= 1), so a tile of cpt chunks
    // is split among at most 1 + ceil((cpt - 1) / q) warps.
    const long long GWe = GW < pl.C ? GW : (pl.C > 0 ? pl.C : 1);
    const long long q = pl.C / GWe;
    long long ms = q > 0 ? 1 + (pl.cpt - 1 + q - 1) / q : pl.cpt;
    pl.ms = (int)(ms < pl.cpt ? ms : pl.cpt);
    if (pl.ms < 1) pl.ms = 1;
    size_t off = 0;
    pl.off_cnt = off;
    off = round_up(off + (size_t)pl.tiles * 4, 256);
    pl.off_done = off;
    off = round_up(off + 4, 256);
    pl.off_argv = off;
    off = round_up(off + (size_t)GW * 4, 256);
    pl.off_argi = off;
    off = round_up(off + (size_t)GW * 4, 256);
    pl.off_part = off;
    off = round_up(off + (size_t)pl.tiles * pl.ms * 32 * 4 * nt * sizeof(float), 256);
    pl.total = off;
    return pl;
}

template <int WK, int NT, bool XS>
cudaError_t launch_stream(const GemvParams& prm, const Plan& pl, size_t smem, cudaStream_t st) {
    auto kern = gemv_stream_kernel<WK, NT, XS>;
    static std::once_flag flags[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t attr_err = cudaSuccess;
    std::call_once(flags[dev % kMaxDevices], [&] {
        attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kXsMaxBytes + 1024);
    });
    if (attr_err != cudaSuccess) return attr_err;
    return launch_pdl(kern, dim3(pl.grid), dim3(kThreads), smem, st, prm);
}

template <int WK>
cudaError_t dispatch_stream(const GemvParams& prm, const Plan& pl, bool xs, size_t smem,
                            cudaStream_t st) {
    if (pl.nt == 1)
        return xs ? launch_stream<WK, 1, true>(prm, pl, smem, st)
                  : launch_stream<WK, 1, false>(prm, pl, 0, st);
    return xs ? launch_stream<WK, 2, true>(prm, pl, smem, st)
              : launch_stream<WK, 2, false>(prm, pl, 0, st);
}

cudaError_t dispatch(int wk, const GemvParams& prm, const Plan& pl, bool xs, size_t smem,
                     cudaStream_t st) {
    switch (wk) {
        case W_FP8_GROUP: return dispatch_stream<W_FP8_GROUP>(prm, pl, xs, smem, st);
        case W_FP8_ROW: return dispatch_stream<W_FP8_ROW>(prm, pl, xs, smem, st);
        default: return dispatch_stream<W_F16>(prm, pl, xs, smem, st);
    }
}

// Whether the streaming kernel's layout rules hold; otherwise the scalar kernel runs.
bool stream_ok(int wk, const void* x, const void* w, const void* s, const void* y, int K,
               int y_f32) {
    const int pos = (wk == W_F16) ? 32 : 64;
    if (K <= 0 || K % pos != 0) return false;
    if (!aligned(x, 16) || !aligned(w, 16)) return false;
    if (y != nullptr && !aligned(y, y_f32 ? 4 : 2)) return false;
    if (wk == W_FP8_GROUP && !aligned(s, 2)) return false;
    if (wk == W_FP8_ROW && s != nullptr && !aligned(s, 4)) return false;
    return true;
}

// Runs one pass of <= 16 tokens.
af_status run_gemv(int wk, const __half* x, const uint8_t* w, const void* s, void* y, int y_f32,
                   int M, int N, int K, int* arg_out, int arg_limit, void* ws, size_t ws_bytes,
                   cudaStream_t st) {
    int sms = device_sm_count();
    if (sms <= 0) return AF_ERR_CUDA;
    if (!stream_ok(wk, x, w, s, y, K, y_f32) || (arg_out != nullptr && M != 1)) {
        if (arg_out != nullptr) return AF_ERR_UNSUPPORTED;
        const int skind = (wk == W_FP8_GROUP) ? AF_SCALE_GROUP_F16
                          : (wk == W_FP8_ROW) ? AF_SCALE_ROW_F32 : AF_SCALE_NONE;
        dim3 grid((N + 7) / 8, M);
        cudaError_t e = launch_pdl(gemv_simple_kernel, grid, dim3(256), 0, st, w, (int)(wk == W_F16),
                                   s, skind, K / 128, x, y, y_f32, M, N, K);
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
    prm.xs_stride = K + kXsPad;
    prm.y_f32 = y_f32;
    prm.cnt = reinterpret_cast<int*>(wsb + pl.off_cnt);
    prm.part = reinterpret_cast<float*>(wsb + pl.off_part);
    prm.arg_out = arg_out;
    prm.arg_val = reinterpret_cast<float*>(wsb + pl.off_argv);
    prm.arg_idx = reinterpret_cast<int*>(wsb + pl.off_argi);
    prm.arg_done = reinterpret_cast<int*>(wsb + pl.off_done);
    prm.arg_limit = arg_limit;
    const size_t smem = (size_t)M * (K + kXsPad) * sizeof(__half);
    const bool xs = smem <= kXsMaxBytes;
    cudaError_t e = dispatch(wk, prm, pl, xs, xs ? smem : 0, st);
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
