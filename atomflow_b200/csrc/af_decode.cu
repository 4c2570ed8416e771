// af_decode.cu -- the rest of a decode step around the projections: token
// embedding, RoPE + KV-cache write, cached GQA attention, standalone RMSNorm,
// and the position counter.  Positions and tokens live in device memory, so a
// whole autoregressive step (embedding .. argmax) replays as one CUDA graph.
//
// Reference counterparts: src/kernel/helpers.cu (k_embed_lookup_kernel,
// build_rope_cache, k_write_kv_cache), src/kernel/rope.cu (rope_kernel),
// src/kernel/tiled_attention.cu:183-269 (gqa_cached_attention_kernel),
// src/kernel/rmsnorm.cu (rms_norm_kernel); order of use src/core/engine.cu:262-521.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstdlib>
#include <cstdint>

#include "af_common.cuh"
#include "af_internal.h"

using namespace af;

// Fault bits (AF_FAULT_*) of this device's decode kernels, read by af_device_faults.
__device__ unsigned int g_decode_faults;

namespace {

// A position outside the KV cache: record it once and skip the launch's work
// (every CTA sees the same *d_pos, so all of them return).
__device__ __forceinline__ bool pos_out_of_range(int pos, int max_seq) {
    if (pos >= 0 && pos < max_seq) return false;
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) atomicOr(&g_decode_faults, (unsigned)AF_FAULT_POSITION);
    return true;
}

// ---------------------------------------------------------------- embedding
// x[i] = half(table[token * D + i])  (helpers.cu k_embed_lookup_kernel)
__global__ void embed_kernel(const float* __restrict__ table, const int* __restrict__ d_token,
                             __half* __restrict__ x, int D) {
    const int tok = *d_token;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < D; i += gridDim.x * blockDim.x)
        x[i] = __float2half_rn(table[(size_t)tok * D + i]);
}

// ------------------------------------------------------- RoPE + KV write
// Blocks 0..NH-1 rotate q heads, NH..NH+NKV-1 rotate k heads and write k and v
// to the caches at row *d_pos.  Pair (d, d + HD/2) rotates by the position's
// angle (rope.cu:9-41).  The reference is built with --use_fast_math, which
// contracts x*c - y*s into one fused multiply-add; `form` picks the operand
// order of that contraction.
__device__ __forceinline__ void rope_pair(float x, float y, float c, float s, int form, float& o0, float& o1) {
    if (form == 0) {
        o0 = fmaf(x, c, -(y * s));
        o1 = fmaf(x, s, y * c);
    } else {
        o0 = fmaf(-y, s, x * c);
        o1 = fmaf(y, c, x * s);
    }
}

__global__ void rope_kv_kernel(__half* __restrict__ qkv, const float* __restrict__ cos_tab,
                               const float* __restrict__ sin_tab, const int* __restrict__ d_pos,
                               __half* __restrict__ k_cache, __half* __restrict__ v_cache, int NH, int NKV, int HD,
                               int form, int max_seq) {
    const int pos = *d_pos;
    if (pos_out_of_range(pos, max_seq)) return;
    const int h = blockIdx.x, half_hd = HD / 2;
    const int q_dim = NH * HD, kv_dim = NKV * HD;
    for (int d = threadIdx.x; d < half_hd; d += blockDim.x) {
        const float c = cos_tab[(size_t)pos * half_hd + d], s = sin_tab[(size_t)pos * half_hd + d];
        __half* base = h < NH ? qkv + (size_t)h * HD : qkv + q_dim + (size_t)(h - NH) * HD;
        float o0, o1;
        rope_pair(__half2float(base[d]), __half2float(base[d + half_hd]), c, s, form, o0, o1);
        const __half r0 = __float2half_rn(o0), r1 = __float2half_rn(o1);
        base[d] = r0;
        base[d + half_hd] = r1;
        if (h >= NH) {   // write_kv_cache (helpers.cu k_write_kv_cache): rotated k and v
            const size_t row = (size_t)pos * kv_dim + (size_t)(h - NH) * HD;
            k_cache[row + d] = r0;
            k_cache[row + d + half_hd] = r1;
            const __half* v = qkv + q_dim + kv_dim + (size_t)(h - NH) * HD;
            v_cache[row + d] = v[d];
            v_cache[row + d + half_hd] = v[d + half_hd];
        }
    }
}

// ------------------------------------------------------ cached attention
// GQA attention for one token, bit-identical to the reference's
// gqa_cached_attention_kernel (src/kernel/tiled_attention.cu:196-269, built
// with --use_fast_math), whose arithmetic per query head is:
//   score[t] = tree_sum_d(q[d] * k[t][d]) * rsqrtf(HD)   (pairwise tree, strides 64..1)
//   m = max_t score[t];  e[t] = expf(score[t] - m);  sum = e[0] + e[1] + ... (in t order)
//   p[t] = e[t] * (1 / sum);  out[d] = half(sum_t p[t] * v[t][d])   (FMA chain in t order)
// The scores are independent per position, so they are spread over the GPU:
// CTA (chunk, kv head) scores positions [t0, t1) of the cache for the G query
// heads sharing the kv head (one warp per position; lane l holds dims l, l+32,
// l+64, l+96, so the reference's strides 64 and 32 are in-lane adds and
// strides 16..1 a shuffle butterfly -- FP addition is commutative, so every
// partial sum is the reference's).  The two order-bound sums (the softmax
// denominator, and each output dim's chain over t) cannot be split without
// changing the rounding: the last CTA of each kv head runs them, one
// 128-thread group per query head, reading the scores back from the workspace.
constexpr int kAttnChunks = 16;
constexpr int kAttnMaxG = 8;
constexpr int kVChunk = 64;   // V rows per shared-memory window of the P.V phase
constexpr int kVBufs = 4;     // windows in flight: V streams kVBufs - 1 windows ahead of the FMA chains
constexpr size_t kAttnSmemMax = 200 * 1024;

// Dynamic shared memory of attention_kernel<G>: the G heads' scores and two V windows.
inline size_t attn_smem(int G, int max_seq) {
    return (size_t)G * max_seq * 4 + (size_t)kVBufs * kVChunk * 128 * 2;
}

// Operand order of the RoPE contraction (see rope_pair): form 0 reproduces the
// reference's rope kernel bit for bit (tests/test_decode_gpu.py pins it; form 1
// is the other order, kept in rope_pair for that comparison).
constexpr int kRopeForm = 0;
// 1 / sum in the reference's fast-math build: the approximate reciprocal
// (form 0) or the full-range approximate division 1 / x (form 1).
constexpr int kRecipForm = 0;

__device__ __forceinline__ float recip_ref(float x) {
    return kRecipForm == 0 ? rcp_approx_ftz(x) : fdiv_full_ftz(1.0f, x);
}

// (a0, a1) = (fma(p, v0, a0), fma(p, v1, a1)) in one packed FP32 FMA.
__device__ __forceinline__ void fma2(float& a0, float& a1, float p, float v0, float v1) {
    unsigned long long av, pv, vv;
    asm("mov.b64 %0, {%1,%2};" : "=l"(av) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1,%1};" : "=l"(pv) : "f"(p));
    asm("mov.b64 %0, {%1,%2};" : "=l"(vv) : "f"(v0), "f"(v1));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(av) : "l"(pv), "l"(vv));
    asm("mov.b64 {%0,%1}, %2;" : "=f"(a0), "=f"(a1) : "l"(av));
}

template <int G>
__global__ void __launch_bounds__(G * 128) attention_kernel(
    const __half* __restrict__ q, const __half* __restrict__ k_cache, const __half* __restrict__ v_cache,
    const int* __restrict__ d_pos, __half* __restrict__ out, int NKV, float* __restrict__ scores,
    int* __restrict__ counters, const float* __restrict__ cos_tab, const float* __restrict__ sin_tab, int NH,
    int max_seq, int head_dim, __half* k_wr, __half* v_wr) {
    // cos_tab != null: RoPE + KV write fused in.  q then points at the raw qkv
    // vector: every CTA rotates its own query heads (rounded to FP16, as the
    // reference stores them), the current position's k (rotated) and v come
    // from qkv, and the CTA whose range holds that position writes them to the
    // caches.
    constexpr int HD = 128;
    constexpr int NW = G * 4;
    const int pos = *d_pos;
    if (pos_out_of_range(pos, max_seq)) return;
    const int seq = pos + 1;
    const int chunk = blockIdx.x, kvh = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int kv_dim = NKV * HD;
    const bool fused = cos_tab != nullptr;

    float rc[2] = {0.f, 0.f}, rs[2] = {0.f, 0.f};   // pair indices lane and lane + 32
    if (fused) {
        rc[0] = cos_tab[(size_t)pos * (HD / 2) + lane];
        rs[0] = sin_tab[(size_t)pos * (HD / 2) + lane];
        rc[1] = cos_tab[(size_t)pos * (HD / 2) + lane + 32];
        rs[1] = sin_tab[(size_t)pos * (HD / 2) + lane + 32];
    }
    auto ld4 = [&](const __half* base, float (&v)[4]) {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __half2float(base[lane + 32 * i]);
    };
    auto rot = [&](float (&v)[4]) {   // pairs (d, d + 64): (v0, v2) and (v1, v3)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            float o0, o1;
            rope_pair(v[i], v[i + 2], rc[i], rs[i], kRopeForm, o0, o1);
            v[i] = __half2float(__float2half_rn(o0));
            v[i + 2] = __half2float(__float2half_rn(o1));
        }
    };
    float qv[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        ld4(q + (size_t)(kvh * G + g) * HD, qv[g]);
        if (fused) rot(qv[g]);
    }
    const int per = (seq + kAttnChunks - 1) / kAttnChunks;
    const int t0 = min(seq, chunk * per), t1 = min(seq, t0 + per);
    float kcur[4] = {0.f, 0.f, 0.f, 0.f};
    if (fused) {
        const __half* kq = q + (size_t)NH * HD + (size_t)kvh * HD;
        ld4(kq, kcur);
        rot(kcur);
        if (warp == 0 && t0 <= pos && pos < t1) {
            float vcur[4];
            ld4(kq + kv_dim, vcur);
            const size_t row = (size_t)pos * kv_dim + (size_t)kvh * HD + lane;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                k_wr[row + 32 * i] = __float2half_rn(kcur[i]);
                v_wr[row + 32 * i] = __float2half_rn(vcur[i]);
            }
        }
    }
    // rsqrtf of the runtime head dim, as the reference computes it
    // (tiled_attention.cu:211); this file is built with --use_fast_math like the
    // reference, which is what makes the value and its use round identically
    const float inv_sqrt = rsqrtf(static_cast<float>(head_dim));
    // ---- scores of positions [t0, t1): one warp per position, four positions'
    // keys loaded before any is reduced (the loads overlap)
    constexpr int kU = 4;
    for (int tb = t0 + warp * kU; tb < t1; tb += NW * kU) {
        float kf[kU][4];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int t = tb + u;
            if (t < t1 && !(fused && t == pos)) ld4(k_cache + (size_t)t * kv_dim + (size_t)kvh * HD, kf[u]);
            else
#pragma unroll
                for (int i = 0; i < 4; ++i) kf[u][i] = kcur[i];
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int t = tb + u;
            if (t >= t1) break;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                // strides 64 (dims l and l + 32) and 32 in-lane, then 16 .. 1 across lanes
                const float a = __fadd_rn(__fmul_rn(qv[g][0], kf[u][0]), __fmul_rn(qv[g][2], kf[u][2]));
                const float b = __fadd_rn(__fmul_rn(qv[g][1], kf[u][1]), __fmul_rn(qv[g][3], kf[u][3]));
                float c = a + b;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
                if (lane == g) __stcg(scores + (size_t)(kvh * G + g) * max_seq + t, c * inv_sqrt);
            }
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (threadIdx.x == 0) s_last = atomicAdd(counters + kvh, 1) == kAttnChunks - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // ---- the last CTA of this kv head: softmax and P.V, one 128-thread group per
    // query head, on the scores copied into shared memory; V streams through a
    // double-buffered shared-memory window of kVChunk positions (cp.async)
    constexpr int NT = G * 128;
    extern __shared__ __align__(16) float dsm[];
    float* es = dsm;                                                   // [G][max_seq]
    __half* vbuf = reinterpret_cast<__half*>(dsm + (size_t)G * max_seq);  // [kVBufs][kVChunk][HD]
    const int g = threadIdx.x >> 7, d = threadIdx.x & 127, gw = (threadIdx.x >> 5) & 3;
    const unsigned char* vsrc = reinterpret_cast<const unsigned char*>(v_cache + (size_t)kvh * HD);
    const int nch = (seq + kVChunk - 1) / kVChunk;
    auto issue_v = [&](int c) {   // rows [c*kVChunk, ...) of this kv head's V: 256 bytes each, 16 per thread-copy
        unsigned char* dst = reinterpret_cast<unsigned char*>(vbuf + (size_t)(c % kVBufs) * kVChunk * HD);
        const int r0 = c * kVChunk, nr = min(kVChunk, seq - r0);
        for (int i = threadIdx.x; i < nr * 16; i += NT) {
            const int r = i >> 4, piece = i & 15;
            cp_async16(smem_u32(dst + r * 256 + piece * 16), vsrc + (size_t)(r0 + r) * kv_dim * 2 + piece * 16);
        }
        cp_async_commit();
    };
    // the first windows of V load while the softmax runs (an empty commit group
    // past the end keeps the group count uniform)
    for (int c = 0; c < kVBufs - 1; ++c) {
        if (c < nch) issue_v(c);
        else cp_async_commit();
    }
    for (int gg = 0; gg < G; ++gg)
        for (int t = threadIdx.x; t < seq; t += NT) es[gg * max_seq + t] = __ldcg(scores + (size_t)(kvh * G + gg) * max_seq + t);
    __syncthreads();
    float* e = es + (size_t)g * max_seq;
    __shared__ float s_max[G][4];
    __shared__ float s_inv[G];
    float m = -1e38f;   // the reference's initial value
    for (int t = d; t < seq; t += 128) m = fmaxf(m, e[t]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) s_max[g][gw] = m;
    named_bar_sync(1 + g, 128);
    m = fmaxf(fmaxf(s_max[g][0], s_max[g][1]), fmaxf(s_max[g][2], s_max[g][3]));
    for (int t = d; t < seq; t += 128) e[t] = __expf(e[t] - m);
    named_bar_sync(1 + g, 128);
    if (d == 0) {
        // the denominator in t order: a serial chain over shared memory
        float sum = 0.f;
        int t = 0;
        for (; t + 32 <= seq; t += 32) {
            float v32[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v32[i] = e[t + i];
#pragma unroll
            for (int i = 0; i < 32; ++i) sum += v32[i];
        }
        for (; t < seq; ++t) sum += e[t];
        s_inv[g] = recip_ref(sum);
    }
    __syncthreads();
    // p[t] = e[t] * (1 / sum), the reference's normalised scores, once per head
    {
        const float inv = s_inv[g];
        for (int t = d; t < seq; t += 128) e[t] = __fmul_rn(e[t], inv);
    }
    __syncthreads();
    // out[d] = sum_t p[t] * v[t][d], an FMA chain in t order per dim; a thread
    // runs two dims' chains in one packed FMA (two independent FMAs)
    const bool pv_lane = d < 64;
    float acc0 = 0.f, acc1 = 0.f;
    for (int c = 0; c < nch; ++c) {
        // window c + kVBufs - 1 reuses the buffer of window c - 1: every thread is past it
        if (c + kVBufs - 1 < nch) issue_v(c + kVBufs - 1);
        else cp_async_commit();
        cp_async_wait<kVBufs - 1>();   // window c has landed
        __syncthreads();
        if (pv_lane) {
            const __half2* vb = reinterpret_cast<const __half2*>(vbuf + (size_t)(c % kVBufs) * kVChunk * HD) + d;
            const float* pc = e + c * kVChunk;
            const int nr = min(kVChunk, seq - c * kVChunk);
            if (nr == kVChunk) {
                // software-pipelined: batch b + 1's loads are in flight while batch b accumulates
                constexpr int B = 8;
                float pa[B], pb[B];
                __half2 va[B], vbb[B];
#pragma unroll
                for (int k = 0; k < B; ++k) {
                    pa[k] = pc[k];
                    va[k] = vb[k * (HD / 2)];
                }
#pragma unroll
                for (int i = 0; i < kVChunk; i += B) {
                    if (i + B < kVChunk) {
#pragma unroll
                        for (int k = 0; k < B; ++k) {
                            pb[k] = pc[i + B + k];
                            vbb[k] = vb[(i + B + k) * (HD / 2)];
                        }
                    }
#pragma unroll
                    for (int k = 0; k < B; ++k) {
                        const float2 vf = __half22float2(va[k]);
                        fma2(acc0, acc1, pa[k], vf.x, vf.y);
                    }
#pragma unroll
                    for (int k = 0; k < B; ++k) {
                        pa[k] = pb[k];
                        va[k] = vbb[k];
                    }
                }
            } else {
                for (int i = 0; i < nr; ++i) {
                    const float2 vf = __half22float2(vb[i * (HD / 2)]);
                    fma2(acc0, acc1, pc[i], vf.x, vf.y);
                }
            }
        }
        __syncthreads();
    }
    if (pv_lane) {
        out[(size_t)(kvh * G + g) * HD + 2 * d] = __float2half_rn(acc0);
        out[(size_t)(kvh * G + g) * HD + 2 * d + 1] = __float2half_rn(acc1);
    }
    __syncthreads();
    if (threadIdx.x == 0) counters[kvh] = 0;   // leave the workspace counter at zero
}

// ------------------------------------------- cached attention, fast form
// Within FP16 rounding of FP64 (online softmax: not the reference's summation
// order, so not bit-identical to it).  One thread-block cluster per kv head.
// The kv head's positions are cut into kClus contiguous ranges, one per CTA of
// the cluster, and each CTA's into per-warp strided positions.  Every warp
// issues the K/V loads of up to kClusBatch positions before it does anything
// else with them (right after reading the position), so a CTA pays about one
// DRAM round trip per batch; the query heads are rotated while those loads fly.
// Each warp keeps an online softmax (running max, sum and P.V), the warps
// merge through shared memory, and the cluster's CTAs merge their partials in
// rank order through distributed shared memory -- no global workspace, fence
// or counter.  Results are deterministic (fixed merge order).
constexpr int kClus = 8;
constexpr int kClusBatch = 16;

template <int G>
__global__ void __cluster_dims__(kClus, 1, 1) __launch_bounds__(256) attention_cluster_kernel(
    const __half* __restrict__ q, const __half* k_cache, const __half* v_cache, const int* __restrict__ d_pos,
    __half* __restrict__ out, int NKV, const float* __restrict__ cos_tab, const float* __restrict__ sin_tab, int NH,
    int form, __half* k_wr, __half* v_wr, int max_seq) {
    constexpr int HD = 128, W = 8, rec = 2 + HD;
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int split = (int)cluster.block_rank(), kvh = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int pos = *d_pos;
    if (pos_out_of_range(pos, max_seq)) return;   // every CTA of the cluster reads the same d_pos
    const int seq = pos + 1;
    const int chunk = (seq + kClus - 1) / kClus;
    const int t0 = min(seq, split * chunk), t1 = min(seq, t0 + chunk);
    const int kv_dim = NKV * HD;
    const size_t col = (size_t)kvh * HD + lane * 4;
    const bool fused = cos_tab != nullptr;

    uint2 kr[kClusBatch], vr[kClusBatch];
    auto fetch = [&](int tb) {
#pragma unroll
        for (int i = 0; i < kClusBatch; ++i) {
            const int t = tb + warp + i * W;
            if (t < t1 && !(fused && t == pos)) {
                kr[i] = *reinterpret_cast<const uint2*>(k_cache + (size_t)t * kv_dim + col);
                vr[i] = *reinterpret_cast<const uint2*>(v_cache + (size_t)t * kv_dim + col);
            } else {
                kr[i] = vr[i] = make_uint2(0u, 0u);
            }
        }
    };
    fetch(t0);

    auto unpack4 = [](const uint2 raw, float (&v)[4]) {
        const __half2 a = *reinterpret_cast<const __half2*>(&raw.x), b = *reinterpret_cast<const __half2*>(&raw.y);
        v[0] = __low2float(a);
        v[1] = __high2float(a);
        v[2] = __low2float(b);
        v[3] = __high2float(b);
    };
    float rc[4], rs[4];
    if (fused) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = (lane & 15) * 4 + e;
            rc[e] = cos_tab[(size_t)pos * (HD / 2) + d];
            rs[e] = sin_tab[(size_t)pos * (HD / 2) + d];
        }
    }
    auto rotate = [&](float (&v)[4]) {   // v: this lane's 4 dims -> rotated, rounded to FP16
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float other = __shfl_xor_sync(0xffffffffu, v[e], 16);
            float o0, o1;
            if (lane < 16) rope_pair(v[e], other, rc[e], rs[e], form, o0, o1);
            else rope_pair(other, v[e], rc[e], rs[e], form, o0, o1);
            v[e] = __half2float(__float2half_rn(lane < 16 ? o0 : o1));
        }
    };
    float qv[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        unpack4(*reinterpret_cast<const uint2*>(q + (size_t)(kvh * G + g) * HD + lane * 4), qv[g]);
        if (fused) rotate(qv[g]);
    }
    float kcur[4] = {0.f, 0.f, 0.f, 0.f}, vcur[4] = {0.f, 0.f, 0.f, 0.f};
    if (fused) {
        const __half* kq = q + (size_t)NH * HD + (size_t)kvh * HD + lane * 4;
        unpack4(*reinterpret_cast<const uint2*>(kq), kcur);
        rotate(kcur);
        unpack4(*reinterpret_cast<const uint2*>(kq + (size_t)NKV * HD), vcur);
        if (warp == 0 && t0 <= pos && pos < t1) {   // this CTA's range holds the new row: store it
            const size_t row = (size_t)pos * kv_dim + col;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                k_wr[row + e] = __float2half_rn(kcur[e]);
                v_wr[row + e] = __float2half_rn(vcur[e]);
            }
        }
    }
    const float scale = rsqrtf((float)HD);
    float m[G], l[G], o[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
        o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
    }
    for (int tb = t0; tb < t1; tb += kClusBatch * W) {
        if (tb != t0) fetch(tb);
#pragma unroll
        for (int i = 0; i < kClusBatch; ++i) {
            const int t = tb + warp + i * W;
            if (t >= t1) break;
            float kf[4], vf[4];
            if (fused && t == pos) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    kf[e] = kcur[e];
                    vf[e] = vcur[e];
                }
            } else {
                unpack4(kr[i], kf);
                unpack4(vr[i], vf);
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float sdot = qv[g][0] * kf[0];
                sdot = fmaf(qv[g][1], kf[1], sdot);
                sdot = fmaf(qv[g][2], kf[2], sdot);
                sdot = fmaf(qv[g][3], kf[3], sdot);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) sdot += __shfl_xor_sync(0xffffffffu, sdot, off);
                const float sc = sdot * scale;
                const float mn = fmaxf(m[g], sc);
                const float corr = __expf(m[g] - mn);   // 0 on the first position (m = -inf)
                const float pw = __expf(sc - mn);
                l[g] = l[g] * corr + pw;
#pragma unroll
                for (int e = 0; e < 4; ++e) o[g][e] = fmaf(pw, vf[e], o[g][e] * corr);
                m[g] = mn;
            }
        }
    }
    // the warps' partials -> this CTA's partial (m, l, o[HD]) per query head
    __shared__ float s_m[W][G], s_l[W][G];
    __shared__ float s_o[W][G][HD];
    __shared__ float s_part[G * rec];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) {
            s_m[warp][g] = m[g];
            s_l[warp][g] = l[g];
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) s_o[warp][g][lane * 4 + e] = o[g][e];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const int g = i / HD, d = i % HD;
        float mm = -INFINITY;
#pragma unroll
        for (int w = 0; w < W; ++w) mm = fmaxf(mm, s_m[w][g]);
        float ll = 0.f, oo = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) {
            const float f = s_m[w][g] == -INFINITY ? 0.f : __expf(s_m[w][g] - mm);
            ll = fmaf(s_l[w][g], f, ll);
            oo = fmaf(s_o[w][g][d], f, oo);
        }
        s_part[g * rec + 2 + d] = oo;
        if (d == 0) {
            s_part[g * rec] = mm;
            s_part[g * rec + 1] = ll;
        }
    }
    cluster.sync();   // every CTA's partial is visible to the cluster
    if (split == 0) {
        const float* parts[kClus];
#pragma unroll
        for (int r = 0; r < kClus; ++r) parts[r] = cluster.map_shared_rank(s_part, r);
        for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
            const int g = i / HD, d = i % HD;
            float ms[kClus], ls[kClus], os[kClus];
#pragma unroll
            for (int r = 0; r < kClus; ++r) {
                ms[r] = parts[r][g * rec];
                ls[r] = parts[r][g * rec + 1];
                os[r] = parts[r][g * rec + 2 + d];
            }
            float mm = -INFINITY;
#pragma unroll
            for (int r = 0; r < kClus; ++r) mm = fmaxf(mm, ms[r]);
            float ll = 0.f, oo = 0.f;
#pragma unroll
            for (int r = 0; r < kClus; ++r) {   // rank order: deterministic
                const float f = ms[r] == -INFINITY ? 0.f : __expf(ms[r] - mm);   // empty ranges add nothing
                ll = fmaf(ls[r], f, ll);
                oo = fmaf(os[r], f, oo);
            }
            out[(size_t)(kvh * G + g) * HD + d] = __float2half_rn(oo / ll);
        }
    }
    cluster.sync();   // no CTA leaves while rank 0 still reads its shared memory
}

// ------------------------------------------------------------- RMSNorm
// The reference's rms_norm_kernel<half, 128> arithmetic (rmsnorm.cu:9-67):
// 128 threads, strided FMA sums, each warp's shuffle-down tree, the four warp
// sums in order, the reference build's rsqrt(sum / K + eps) (rms_scale_ref), and
// half(x * r * w).
__global__ void __launch_bounds__(128) rmsnorm_kernel(const __half* __restrict__ x, const float* __restrict__ w,
                                                      float eps, __half* __restrict__ out, int K) {
    __shared__ float s_nrm[4];
    __shared__ float s_r;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float ss = 0.f;
    for (int i = threadIdx.x; i < K; i += 128) {
        const float v = __half2float(x[i]);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) ss += __shfl_down_sync(0xffffffffu, ss, o);
    if (lane == 0) s_nrm[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0)
        s_r = rms_scale_ref(((s_nrm[0] + s_nrm[1]) + s_nrm[2]) + s_nrm[3], K, eps);
    __syncthreads();
    const float r = s_r;
    for (int i = threadIdx.x; i < K; i += 128) out[i] = __float2half_rn(__half2float(x[i]) * r * w[i]);
}

__global__ void advance_kernel(int* d_pos, int by) { *d_pos += by; }

}  // namespace

extern "C" af_status af_embed_lookup(const float* table, const int* d_token, void* x, int D, void* stream) {
    if (table == nullptr || d_token == nullptr || x == nullptr || D <= 0 || !aligned(x, 2)) return AF_ERR_INVALID;
    embed_kernel<<<(D + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        table, d_token, static_cast<__half*>(x), D);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "embed_kernel");
}

extern "C" af_status af_rope_tables(float* cos_out, float* sin_out, int max_seq, int head_dim, float base) {
    if (cos_out == nullptr || sin_out == nullptr || max_seq <= 0 || head_dim <= 0 || head_dim % 2) return AF_ERR_INVALID;
    // the reference's host formula (helpers.cu build_rope_cache), in float
    const int half_dim = head_dim / 2;
    for (int s = 0; s < max_seq; ++s)
        for (int i = 0; i < half_dim; ++i) {
            const float theta = s / std::pow(base, 2.0f * i / head_dim);
            cos_out[(size_t)s * half_dim + i] = std::cos(theta);
            sin_out[(size_t)s * half_dim + i] = std::sin(theta);
        }
    return AF_OK;
}

extern "C" af_status af_rope_kv_write(void* qkv, const float* cos_tab, const float* sin_tab, const int* d_pos,
                                     void* k_cache, void* v_cache, int n_heads, int n_kv_heads, int head_dim,
                                     int max_seq, void* stream) {
    if (max_seq <= 0) return AF_ERR_INVALID;
    if (qkv == nullptr || cos_tab == nullptr || sin_tab == nullptr || d_pos == nullptr || k_cache == nullptr ||
        v_cache == nullptr || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || head_dim % 2)
        return AF_ERR_INVALID;
    rope_kv_kernel<<<n_heads + n_kv_heads, 64, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<__half*>(qkv), cos_tab, sin_tab, d_pos, static_cast<__half*>(k_cache),
        static_cast<__half*>(v_cache), n_heads, n_kv_heads, head_dim, kRopeForm, max_seq);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "rope_kv_kernel");
}


extern "C" size_t af_decode_attention_workspace_bytes(int n_heads, int n_kv_heads, int max_seq) {
    if (n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads || max_seq <= 0) return 0;
    // the exact form's scores [NH][max_seq] (the fast form needs none)
    return 256 + round_up((size_t)n_kv_heads * 4, 256) + (size_t)n_heads * max_seq * 4;
}

static af_status attention_launch(const void* q, const void* k_cache, const void* v_cache, const int* d_pos,
                                  void* out, int n_heads, int n_kv_heads, int head_dim, int max_seq, void* workspace,
                                  size_t workspace_bytes, void* stream, const float* cos_tab, const float* sin_tab) {
    if (max_seq <= 0) return AF_ERR_INVALID;
    if (q == nullptr || k_cache == nullptr || v_cache == nullptr || d_pos == nullptr || out == nullptr ||
        n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads)
        return AF_ERR_INVALID;
    if (head_dim != 128 || n_heads / n_kv_heads > kAttnMaxG) return AF_ERR_UNSUPPORTED;
    if (!aligned(q, 2) || !aligned(k_cache, 2) || !aligned(v_cache, 2) || !aligned(out, 2)) return AF_ERR_INVALID;
    const size_t need = af_decode_attention_workspace_bytes(n_heads, n_kv_heads, max_seq);
    if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 256)) return AF_ERR_WORKSPACE;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    int* counters = reinterpret_cast<int*>(ws + 256);
    float* scores = reinterpret_cast<float*>(ws + 256 + round_up((size_t)n_kv_heads * 4, 256));
    const dim3 grid(kAttnChunks, n_kv_heads);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    const __half *qh = static_cast<const __half*>(q), *kh = static_cast<const __half*>(k_cache),
                 *vh = static_cast<const __half*>(v_cache);
    __half* oh = static_cast<__half*>(out);
    // fused RoPE mode writes the current row of the caches (the caller's buffers are writable)
    __half* kw = cos_tab ? const_cast<__half*>(kh) : nullptr;
    __half* vw = cos_tab ? const_cast<__half*>(vh) : nullptr;
    const size_t smem = attn_smem(n_heads / n_kv_heads, max_seq);
    if (smem > kAttnSmemMax) return AF_ERR_UNSUPPORTED;   // the scores of the whole cache live in shared memory
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AF_ERR_CUDA;
    static bool attr_set[kMaxDevices][kAttnMaxG + 1] = {};
    switch (n_heads / n_kv_heads) {
#define AF_ATTN(GG)                                                                                       \
    case GG: {                                                                                            \
        if (!attr_set[dev][GG]) {                                                                         \
            cudaError_t ea = cudaFuncSetAttribute(attention_kernel<GG>,                                   \
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnSmemMax); \
            if (ea != cudaSuccess) return cuda_fail(ea, "attention_kernel attributes");                   \
            attr_set[dev][GG] = true;                                                                     \
        }                                                                                                 \
        attention_kernel<GG><<<grid, GG * 128, smem, cs>>>(qh, kh, vh, d_pos, oh, n_kv_heads, scores, counters, \
                                                           cos_tab, sin_tab, n_heads, max_seq, head_dim, kw, vw); \
        break;                                                                                            \
    }
        AF_ATTN(1) AF_ATTN(2) AF_ATTN(3) AF_ATTN(4) AF_ATTN(5) AF_ATTN(6) AF_ATTN(7) AF_ATTN(8)
#undef AF_ATTN
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "attention_kernel");
}

static af_status attention_fast_launch(const void* q, const void* k_cache, const void* v_cache, const int* d_pos,
                                        void* out, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                                        void* workspace, size_t workspace_bytes, void* stream, const float* cos_tab,
                                        const float* sin_tab) {
    if (max_seq <= 0) return AF_ERR_INVALID;
    if (q == nullptr || k_cache == nullptr || v_cache == nullptr || d_pos == nullptr || out == nullptr ||
        n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads)
        return AF_ERR_INVALID;
    if (head_dim != 128 || n_heads / n_kv_heads > kAttnMaxG) return AF_ERR_UNSUPPORTED;
    if (!aligned(q, 8) || !aligned(k_cache, 8) || !aligned(v_cache, 8) || !aligned(out, 2)) return AF_ERR_INVALID;
    (void)workspace;   // the cluster form merges in distributed shared memory: no workspace
    (void)workspace_bytes;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    const __half *qh = static_cast<const __half*>(q), *kh = static_cast<const __half*>(k_cache),
                 *vh = static_cast<const __half*>(v_cache);
    __half* oh = static_cast<__half*>(out);
    __half* kw = cos_tab ? const_cast<__half*>(kh) : nullptr;
    __half* vw = cos_tab ? const_cast<__half*>(vh) : nullptr;
    const dim3 cgrid(kClus, n_kv_heads);
    switch (n_heads / n_kv_heads) {
#define AF_ATTN(GG)                                                                                            \
    case GG:                                                                                                  \
        attention_cluster_kernel<GG><<<cgrid, 256, 0, cs>>>(qh, kh, vh, d_pos, oh, n_kv_heads, cos_tab, sin_tab, \
                                                            n_heads, kRopeForm, kw, vw, max_seq);             \
        break;
        AF_ATTN(1) AF_ATTN(2) AF_ATTN(3) AF_ATTN(4) AF_ATTN(5) AF_ATTN(6) AF_ATTN(7) AF_ATTN(8)
#undef AF_ATTN
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "attention_cluster_kernel");
}

extern "C" af_status af_decode_rope_attention_fast(void* qkv, const float* cos_tab, const float* sin_tab,
                                                  const int* d_pos, void* k_cache, void* v_cache, void* out,
                                                  int n_heads, int n_kv_heads, int head_dim, int max_seq,
                                                  void* workspace, size_t workspace_bytes, void* stream) {
    if (cos_tab == nullptr || sin_tab == nullptr) return AF_ERR_INVALID;
    return attention_fast_launch(qkv, k_cache, v_cache, d_pos, out, n_heads, n_kv_heads, head_dim, max_seq,
                                  workspace, workspace_bytes, stream, cos_tab, sin_tab);
}

extern "C" af_status af_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int* d_pos,
                                        void* out, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                                        void* workspace, size_t workspace_bytes, void* stream) {
    return attention_launch(q, k_cache, v_cache, d_pos, out, n_heads, n_kv_heads, head_dim, max_seq, workspace,
                            workspace_bytes, stream, nullptr, nullptr);
}

extern "C" af_status af_decode_rope_attention(void* qkv, const float* cos_tab, const float* sin_tab, const int* d_pos,
                                             void* k_cache, void* v_cache, void* out, int n_heads, int n_kv_heads,
                                             int head_dim, int max_seq, void* workspace, size_t workspace_bytes,
                                             void* stream) {
    if (cos_tab == nullptr || sin_tab == nullptr) return AF_ERR_INVALID;
    return attention_launch(qkv, k_cache, v_cache, d_pos, out, n_heads, n_kv_heads, head_dim, max_seq, workspace,
                            workspace_bytes, stream, cos_tab, sin_tab);
}

extern "C" af_status af_rmsnorm(const void* x, const float* norm_w, float eps, void* out, int K, void* stream) {
    if (x == nullptr || norm_w == nullptr || out == nullptr || K <= 0 || !aligned(x, 2) || !aligned(out, 2))
        return AF_ERR_INVALID;
    rmsnorm_kernel<<<1, 128, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const __half*>(x), norm_w, eps,
                                                                    static_cast<__half*>(out), K);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "rmsnorm_kernel");
}

extern "C" af_status af_decode_advance(int* d_pos, int by, void* stream) {
    if (d_pos == nullptr) return AF_ERR_INVALID;
    advance_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(d_pos, by);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "advance_kernel");
}

unsigned af::decode_faults(bool clear, cudaError_t* err) {
    unsigned v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_decode_faults, sizeof(v));
    if (e == cudaSuccess && clear && v != 0) {
        const unsigned z = 0;
        e = cudaMemcpyToSymbol(g_decode_faults, &z, sizeof(z));
    }
    *err = e;
    return v;
}
