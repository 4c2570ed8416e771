// af_chain.cu -- the one-token W8A16 projections of a decode step as ONE
// persistent kernel, bit-identical to the reference's GEMV.
//
// Reference behaviour (AtomFlow):
//   src/kernel/qkv_gemm.cu:32-111   w8a16_gemv_kernel<256>: thread t of the
//       row's block sums (float(W) * float(S)) * float(x) over positions
//       4t + 1024j + v (j = 0.., v = 0..3) in that order, FMUL then FFMA;
//       then __shfl_down 16, 8, 4, 2, 1; then thread 0 adds the 8 warp sums in
//       order (starting from 0.0f) and rounds to FP16.
//   src/kernel/rmsnorm.cu, swiglu.cu, residual_add.cu: the element-wise work
//       around the projections (src/core/engine.cu:292-483), fused here as a
//       prologue (RMSNorm of x) or an epilogue (SwiGLU of gate/up, residual add).
//
// Arithmetic: every output equals the reference kernel's, bit for bit.  Each
// of the 256 consumer threads of a CTA plays the reference's thread t for 16
// rows at once: a stage holds 16 rows x 1024 positions, which is exactly one
// j-step of every t, so thread t's FFMA chain per row runs over the stages in
// the reference's order.  float(W) * float(S) is exact in FP32 (4 + 11
// significant bits), computed by one mixed-precision FMA from the FP16 forms
// (the packed e4m3x2 -> f16x2 conversion is exact); the chains of two rows
// share one packed f32x2 FMA (two independent, identically rounded FMAs).
// The warp tree is the reference's shuffle-down tree evaluated as a
// transpose-reduce (each lane ends with one row's sum; FP addition is
// commutative, so every partial sum is the reference's), then the warp sums
// are added in warp order.
//
// Data movement (sm_100a): one producer warp streams the weight rows with
// 1-D TMA bulk copies (cp.async.bulk, global -> shared, completion on an
// mbarrier) into a ring of 16 KB stages; 8 consumer warps compute.  The ring
// never drains across projections: while the consumers wait for the previous
// projection's output (a grid-wide completion counter in the caller's
// workspace, polled with a bound), the producer keeps filling the ring with
// the next projection's weights, which depend on nothing.  A decode layer's
// chain -- RMSNorm+QKV, O+residual, RMSNorm+gate/up+SwiGLU, down+residual --
// or a whole step's projections run in one launch with no kernel boundary.
//
// Every wait is bounded (%globaltimer): on expiry the kernel records
// AF_FAULT_CHAIN_WAIT, stops issuing copies, lets every thread run to the end
// without waiting again, waits (bounded) for its own copies in flight and
// returns -- the results are then invalid, the context stays usable.

#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "af_common.cuh"
#include "af_internal.h"

// Fault bits (AF_FAULT_*) of this device's chain kernels, read by af_device_faults.
__device__ unsigned int g_chain_faults;

namespace af {
namespace {

constexpr int kCWarps = 8;                  // consumer warps: the reference's 256 threads
constexpr int kThreads = (kCWarps + 1) * 32;  // + one producer warp
constexpr int kRows = 16;                   // rows per stage
constexpr int kBlk = 1024;                  // positions per stage (the reference's j-stride)
constexpr int kStage = kRows * kBlk;        // bytes per stage
constexpr int kMaxOps = 320;
constexpr int kMaxK = 16384;
constexpr size_t kSmemCap = 227 * 1024;

enum OpKind { OP_GEMV = 0, OP_GEMV_RESIDUAL = 1, OP_RMSNORM_GEMV = 2, OP_RMSNORM_SWIGLU = 3 };

struct Op {
    const __half* x;
    const uint8_t* w;
    const uint16_t* s;
    const uint8_t* w2;
    const uint16_t* s2;
    const float* norm_w;
    __half* y;
    __half* xn_out;
    __half* aux;
    int kind, N, K, wait;
    float eps;
};

struct Params {
    int n_ops;
    int stages;                 // ring stages
    int x_bytes, sc_bytes;      // shared carve-up: x [K] FP16, one scale buffer
    int* counters;              // [n_ops + 1] completion counters (null: no op waits)
    unsigned long long wait_ns;
    Op ops[kMaxOps];
};

static_assert(sizeof(Params) <= 32764, "the op table must fit the kernel parameter space");

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// W * S exactly, as an FP32: a mixed-precision FMA of the two FP16 values
// (the product has at most 15 significant bits) plus -0 (keeps the sign of zero).
__device__ __forceinline__ float mul_f16_exact(uint16_t a, uint16_t b) {
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(-0.0f));
    return d;
}

// (s0, s1) = fma((a0, a1), (x, x), (s0, s1)): two FP32 FMAs in one packed instruction.
__device__ __forceinline__ void fma_pair(float& s0, float& s1, float a0, float a1, float x) {
    unsigned long long sv, av, xv;
    asm("mov.b64 %0, {%1,%2};" : "=l"(sv) : "f"(s0), "f"(s1));
    asm("mov.b64 %0, {%1,%2};" : "=l"(av) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1,%1};" : "=l"(xv) : "f"(x));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(sv) : "l"(av), "l"(xv));
    asm("mov.b64 {%0,%1}, %2;" : "=f"(s0), "=f"(s1) : "l"(sv));
}

// Bounded mbarrier wait that gives up at once when the CTA has aborted.
__device__ __forceinline__ void chain_wait(uint32_t bar, uint32_t parity, unsigned long long limit,
                                           volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return;
    if (*abort_flag) return;
    if (!mbar_wait_bounded(bar, parity, limit)) {
        atomicOr(&g_chain_faults, (unsigned)AF_FAULT_CHAIN_WAIT);
        *abort_flag = 1;
    }
}

struct RowSplit {
    int r0, r1, tr;   // this CTA's output rows [r0, r1); output rows per 16-row stage
};
__device__ __forceinline__ RowSplit row_split(const Op& op) {
    RowSplit rs;
    rs.r0 = (int)((long long)blockIdx.x * op.N / gridDim.x);
    rs.r1 = (int)((long long)(blockIdx.x + 1) * op.N / gridDim.x);
    rs.tr = op.kind == OP_RMSNORM_SWIGLU ? 8 : 16;   // SwiGLU: 8 gate rows + the same 8 up rows
    return rs;
}

// Where an op's staged scales sit in a scale buffer: matrix m (gate, then up
// for SwiGLU) at byte off[m], whose value modulo 16 equals the source block's
// address modulo 16.
struct ScaleLayout {
    int off[2];
};
__device__ __forceinline__ ScaleLayout scale_layout(const Op& op, const RowSplit& rs, int G) {
    ScaleLayout sl;
    const int cnt = (rs.r1 - rs.r0) * G;
    sl.off[0] = (int)(reinterpret_cast<uintptr_t>(op.s + (size_t)rs.r0 * G) & 15);
    sl.off[1] = 0;
    if (op.kind == OP_RMSNORM_SWIGLU)
        sl.off[1] = ((sl.off[0] + cnt * 2 + 15) & ~15) + (int)(reinterpret_cast<uintptr_t>(op.s2 + (size_t)rs.r0 * G) & 15);
    return sl;
}

__global__ void __launch_bounds__(kThreads, 1) chain_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    const int S = p.stages;
    unsigned char* ring = smem;
    __half* xs = reinterpret_cast<__half*>(smem + (size_t)S * kStage);
    unsigned char* scb = reinterpret_cast<unsigned char*>(xs) + p.x_bytes;
    __shared__ __align__(8) uint64_t full[16], empty[16], sc_full[2], sc_empty[2];
    __shared__ float part[2][kCWarps][kRows];
    __shared__ float s_nrm[4];
    __shared__ float s_r;
    __shared__ volatile int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(smem_u32(&full[i]), 1);
            mbar_init(smem_u32(&empty[i]), kCWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&sc_full[b]), 32);
            mbar_init(smem_u32(&sc_empty[b]), kCWarps);
        }
        s_abort = 0;
        mbar_init_fence();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kCWarps) {
        // ------------------------------------------------------------ producer
        int slot = 0;
        uint32_t phase = 0;
        int issued = 0;
        for (int o = 0; o < p.n_ops && !s_abort; ++o) {
            const Op& op = p.ops[o];
            const RowSplit rs = row_split(op);
            const bool pair = op.kind == OP_RMSNORM_SWIGLU;
            const int G = op.K >> 7;
            // this CTA's group scales (FP16 [rows, G]; SwiGLU: gate's, then up's) -> buffer o & 1
            const int b = o & 1;
            chain_wait(smem_u32(&sc_empty[b]), ((o >> 1) & 1) ^ 1, p.wait_ns, &s_abort);
            {
                // The block's 16-byte-aligned middle by one bulk copy, its ragged
                // ends (< 8 values each) by plain loads; the staged copy keeps the
                // block's address modulo 16 so that the bulk part lands aligned.
                unsigned char* sc = scb + (size_t)b * p.sc_bytes;
                const int cnt = (rs.r1 - rs.r0) * G;
                const uint32_t scf = smem_u32(&sc_full[b]);
                uint32_t tx = 0;
                ScaleLayout sl = scale_layout(op, rs, G);
                for (int m = 0; m < (pair ? 2 : 1); ++m) {
                    const uint16_t* src = (m ? op.s2 : op.s) + (size_t)rs.r0 * G;
                    const uintptr_t a0 = reinterpret_cast<uintptr_t>(src), a1 = a0 + (uintptr_t)cnt * 2;
                    const uintptr_t m0 = (a0 + 15) & ~(uintptr_t)15, m1 = a1 & ~(uintptr_t)15;
                    unsigned char* dst = sc + sl.off[m];
                    if (m1 > m0) {
                        if (lane == 0) {
                            mbar_expect_tx(scf, (uint32_t)(m1 - m0));
                            bulk_g2s(smem_u32(dst + (m0 - a0)), reinterpret_cast<const void*>(m0), (uint32_t)(m1 - m0),
                                     scf);
                        }
                        tx += (uint32_t)(m1 - m0);
                        for (uintptr_t a = a0 + 2 * lane; a < m0; a += 64)
                            *reinterpret_cast<uint16_t*>(dst + (a - a0)) = __ldg(reinterpret_cast<const uint16_t*>(a));
                        for (uintptr_t a = m1 + 2 * lane; a < a1; a += 64)
                            *reinterpret_cast<uint16_t*>(dst + (a - a0)) = __ldg(reinterpret_cast<const uint16_t*>(a));
                    } else {
                        for (uintptr_t a = a0 + 2 * lane; a < a1; a += 64)
                            *reinterpret_cast<uint16_t*>(dst + (a - a0)) = __ldg(reinterpret_cast<const uint16_t*>(a));
                    }
                }
                (void)tx;
                mbar_arrive(scf);   // 32 arrivals, each lane after its own stores; plus the bulk bytes
            }

            const int nblk = (op.K + kBlk - 1) / kBlk;
            for (int tr = rs.r0; tr < rs.r1; tr += rs.tr) {
                const int nv = min(rs.tr, rs.r1 - tr);
                for (int j = 0; j < nblk; ++j) {
                    chain_wait(smem_u32(&empty[slot]), phase ^ 1, p.wait_ns, &s_abort);
                    if (s_abort) break;
                    const int bb = min(kBlk, op.K - j * kBlk);
                    const uint32_t fb = smem_u32(&full[slot]);
                    if (lane == 0) mbar_arrive_expect_tx(fb, (uint32_t)((pair ? 2 * nv : nv) * bb));
                    __syncwarp();
                    if (lane < kRows) {
                        const uint8_t* src = nullptr;
                        if (pair) {
                            const int r = lane & 7;
                            if (r < nv) src = (lane < 8 ? op.w : op.w2) + (size_t)(tr + r) * op.K + (size_t)j * kBlk;
                        } else if (lane < nv) {
                            src = op.w + (size_t)(tr + lane) * op.K + (size_t)j * kBlk;
                        }
                        if (src) bulk_g2s(smem_u32(ring + (size_t)slot * kStage + lane * kBlk), src, (uint32_t)bb, fb);
                    }
                    ++issued;
                    if (++slot == S) {
                        slot = 0;
                        phase ^= 1;
                    }
                }
                if (s_abort) break;
            }
        }
        if (s_abort && lane == 0) {
            // a wait gave up: the copies already issued still land in this CTA's
            // shared memory -- wait for them (bounded) before the CTA may exit
            const unsigned long long t0 = globaltimer_ns();
            for (int q = max(0, issued - S); q < issued; ++q) {
                const int sl = q % S;
                const uint32_t ph = (uint32_t)((q / S) & 1);
                while (!mbar_try_wait(smem_u32(&full[sl]), ph))
                    if (globaltimer_ns() - t0 > p.wait_ns) break;
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        const int t = threadIdx.x;   // the reference's thread index
        pdl_wait();                  // x / residual inputs of the first ops may come from the previous kernel
        int slot = 0;
        uint32_t phase = 0;
        int tb = 0;
        for (int o = 0; o < p.n_ops; ++o) {
            const Op& op = p.ops[o];
            const RowSplit rs = row_split(op);
            const bool pair = op.kind == OP_RMSNORM_SWIGLU;
            const int G = op.K >> 7;
            const int K = op.K;
            if (op.wait && o > 0 && p.counters != nullptr) {
                // op o reads what op o-1 wrote: wait until every CTA has finished it
                if (t == 0 && !s_abort) {
                    const unsigned long long t0 = globaltimer_ns();
                    while (ld_acquire_gpu(p.counters + o - 1) < (int)gridDim.x) {
                        if (globaltimer_ns() - t0 > p.wait_ns) {
                            atomicOr(&g_chain_faults, (unsigned)AF_FAULT_CHAIN_WAIT);
                            s_abort = 1;
                            break;
                        }
                    }
                }
                named_bar_sync(1, kCWarps * 32);
            }
            // x -> shared (L2-coherent loads: another CTA may have written it)
            for (int i = t * 8; i < K; i += kCWarps * 32 * 8)
                *reinterpret_cast<uint4*>(xs + i) = ldcg_u4(op.x + i);
            named_bar_sync(1, kCWarps * 32);
            if (op.kind == OP_RMSNORM_GEMV || op.kind == OP_RMSNORM_SWIGLU) {
                // RMSNorm of x in the reference's arithmetic (src/kernel/rmsnorm.cu:9-67,
                // 128 threads): strided FMA sums, shuffle-down tree 1..16, the four
                // warp sums in order, rsqrt(sum / K + eps) as its fast-math build
                // evaluates it, then half(x * r * w).
                if (t < 128) {
                    float ss = 0.f;
                    for (int i = t; i < K; i += 128) {
                        const float v = __half2float(xs[i]);
                        ss = fmaf(v, v, ss);
                    }
#pragma unroll
                    for (int off = 1; off < 32; off <<= 1) ss += __shfl_down_sync(0xffffffffu, ss, off);
                    if (lane == 0) s_nrm[warp] = ss;
                }
                named_bar_sync(1, kCWarps * 32);
                if (t == 0) s_r = rms_scale_ref(((s_nrm[0] + s_nrm[1]) + s_nrm[2]) + s_nrm[3], K, op.eps);
                named_bar_sync(1, kCWarps * 32);
                const float r = s_r;
                for (int i = t; i < K; i += kCWarps * 32)
                    xs[i] = __float2half_rn(__half2float(xs[i]) * r * __ldg(op.norm_w + i));
                named_bar_sync(1, kCWarps * 32);
                if (op.xn_out != nullptr && blockIdx.x == 0)
                    for (int i = t; i < K; i += kCWarps * 32) op.xn_out[i] = xs[i];
            }
            const int b = o & 1;
            chain_wait(smem_u32(&sc_full[b]), (o >> 1) & 1, p.wait_ns, &s_abort);
            const ScaleLayout sl = scale_layout(op, rs, G);
            const uint16_t* sc = reinterpret_cast<const uint16_t*>(scb + (size_t)b * p.sc_bytes + sl.off[0]);
            const int up_base = (sl.off[1] - sl.off[0]) / 2;   // halves from gate's block to up's

            const int nblk = (K + kBlk - 1) / kBlk;
            for (int tr = rs.r0; tr < rs.r1; tr += rs.tr) {
                const int nv = min(rs.tr, rs.r1 - tr);
                // the 16 stage rows' scale rows in the staged block (invalid rows: row 0's)
                int srow[kRows];
#pragma unroll
                for (int i = 0; i < kRows; ++i) {
                    const int r = pair ? (i & 7) : i;
                    const int rr = (r < nv ? tr + r : tr) - rs.r0;
                    srow[i] = (pair && i >= 8 ? up_base : 0) + rr * G;
                }
                float acc[kRows];
#pragma unroll
                for (int i = 0; i < kRows; ++i) acc[i] = 0.f;
                for (int j = 0; j < nblk; ++j) {
                    chain_wait(smem_u32(&full[slot]), phase, p.wait_ns, &s_abort);
                    const int kp = j * kBlk + 4 * t;
                    if (kp < K) {
                        const uint2 xr = *reinterpret_cast<const uint2*>(xs + kp);
                        const float2 x01 = __half22float2(*reinterpret_cast<const __half2*>(&xr.x));
                        const float2 x23 = __half22float2(*reinterpret_cast<const __half2*>(&xr.y));
                        const int gidx = kp >> 7;
                        const unsigned char* st = ring + (size_t)slot * kStage + 4 * t;
#pragma unroll
                        for (int i = 0; i < kRows; i += 2) {
                            const uint32_t w0 = *reinterpret_cast<const uint32_t*>(st + i * kBlk);
                            const uint32_t w1 = *reinterpret_cast<const uint32_t*>(st + (i + 1) * kBlk);
                            const uint16_t s0 = sc[srow[i] + gidx], s1 = sc[srow[i + 1] + gidx];
                            const uint32_t h0a = e4m3x2_lo(w0), h0b = e4m3x2_hi(w0);
                            const uint32_t h1a = e4m3x2_lo(w1), h1b = e4m3x2_hi(w1);
                            fma_pair(acc[i], acc[i + 1], mul_f16_exact((uint16_t)h0a, s0),
                                     mul_f16_exact((uint16_t)h1a, s1), x01.x);
                            fma_pair(acc[i], acc[i + 1], mul_f16_exact((uint16_t)(h0a >> 16), s0),
                                     mul_f16_exact((uint16_t)(h1a >> 16), s1), x01.y);
                            fma_pair(acc[i], acc[i + 1], mul_f16_exact((uint16_t)h0b, s0),
                                     mul_f16_exact((uint16_t)h1b, s1), x23.x);
                            fma_pair(acc[i], acc[i + 1], mul_f16_exact((uint16_t)(h0b >> 16), s0),
                                     mul_f16_exact((uint16_t)(h1b >> 16), s1), x23.y);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&empty[slot]));
                    if (++slot == S) {
                        slot = 0;
                        phase ^= 1;
                    }
                }
                // warp tree: the reference's shuffle-down tree 16, 8, 4, 2, 1 as a
                // transpose-reduce; lane l ends with the warp sum of row rowof(l)
                float v8[8], v4[4], v2[2], v1;
                {
                    const bool hi = lane & 16;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float send = hi ? acc[i] : acc[8 + i];
                        const float keep = hi ? acc[8 + i] : acc[i];
                        v8[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                    }
                }
                {
                    const bool hi = lane & 8;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float send = hi ? v8[i] : v8[4 + i];
                        const float keep = hi ? v8[4 + i] : v8[i];
                        v4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                    }
                }
                {
                    const bool hi = lane & 4;
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const float send = hi ? v4[i] : v4[2 + i];
                        const float keep = hi ? v4[2 + i] : v4[i];
                        v2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
                    }
                }
                {
                    const bool hi = lane & 2;
                    const float send = hi ? v2[0] : v2[1];
                    const float keep = hi ? v2[1] : v2[0];
                    v1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
                }
                v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
                const int rowof = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 +
                                  ((lane >> 1) & 1);
                if ((lane & 1) == 0) part[tb][warp][rowof] = v1;
                named_bar_sync(1, kCWarps * 32);
                // the warp sums in warp order, from 0.0f, then the op's epilogue
                if (t < (pair ? 8 : 16) && t < nv) {
                    float tot = 0.f;
#pragma unroll
                    for (int w = 0; w < kCWarps; ++w) tot += part[tb][w][t];
                    const int row = tr + t;
                    if (pair) {
                        float up = 0.f;
#pragma unroll
                        for (int w = 0; w < kCWarps; ++w) up += part[tb][w][8 + t];
                        // swiglu.cu:12-26 on the FP16 gate / up outputs
                        const __half gh = __float2half_rn(tot), uh = __float2half_rn(up);
                        if (op.aux != nullptr) {
                            op.aux[row] = gh;
                            op.aux[op.N + row] = uh;
                        }
                        const float g = __half2float(gh);
                        const float u = __half2float(uh);
                        const float silu = fdiv_full_ftz(g, 1.0f + __expf(-g));
                        op.y[row] = __float2half_rn(silu * u);
                    } else if (op.kind == OP_GEMV_RESIDUAL) {
                        // residual_add.cu:11-20: half(float(x) + float(half(Wx)))
                        const unsigned short old = __ldcg(reinterpret_cast<const unsigned short*>(op.y) + row);
                        const __half oh = __float2half_rn(tot);
                        if (op.aux != nullptr) op.aux[row] = oh;
                        const float o16 = __half2float(oh);
                        op.y[row] = __float2half_rn(half_bits_to_float(old) + o16);
                    } else {
                        op.y[row] = __float2half_rn(tot);
                    }
                }
                tb ^= 1;
            }
            named_bar_sync(1, kCWarps * 32);   // every row of this op is stored
            if (t == 0 && p.counters != nullptr) {
                __threadfence();
                atomicAdd(p.counters + o, 1);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&sc_empty[b]));
        }
    }
    __syncthreads();
    // the last CTA to finish returns the counters to zero for the next launch
    if (threadIdx.x == 0 && p.counters != nullptr) {
        __threadfence();
        if (atomicAdd(p.counters + p.n_ops, 1) == (int)gridDim.x - 1) {
            for (int i = 0; i <= p.n_ops; ++i) p.counters[i] = 0;
            __threadfence();
        }
    }
}

}  // namespace

unsigned chain_faults(bool clear, cudaError_t* err) {
    unsigned v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_chain_faults, sizeof(v));
    if (e == cudaSuccess && clear && v != 0) {
        const unsigned z = 0;
        e = cudaMemcpyToSymbol(g_chain_faults, &z, sizeof(z));
    }
    *err = e;
    return v;
}

namespace {

bool al(const void* p, size_t a) { return p != nullptr && aligned(p, a); }

// Validates one op and returns its staged-scale bytes (0: invalid).
size_t op_scale_bytes(const af_chain_op& op, int grid) {
    if (op.kind < AF_OP_GEMV || op.kind > AF_OP_RMSNORM_SWIGLU) return 0;
    if (op.N <= 0 || op.K <= 0 || op.K % 128 != 0 || op.K > kMaxK) return 0;
    if (!al(op.x, 16) || !al(op.w, 16) || !al(op.scales, 2) || !al(op.y, 2)) return 0;
    const bool norm = op.kind == AF_OP_RMSNORM_GEMV || op.kind == AF_OP_RMSNORM_SWIGLU;
    if (norm && !al(op.norm_w, 4)) return 0;
    if (!aligned(op.xn_out, 2) || !aligned(op.aux, 2)) return 0;
    if (op.kind == AF_OP_RMSNORM_SWIGLU && (!al(op.w2, 16) || !al(op.scales2, 2))) return 0;
    const size_t rows = ((size_t)op.N + grid - 1) / grid + 1;
    return (rows * (op.K / 128) * 2 + 32) * (op.kind == AF_OP_RMSNORM_SWIGLU ? 2 : 1);
}

struct Attr {
    std::once_flag once;
    cudaError_t err = cudaSuccess;
};
Attr g_attr[kMaxDevices];

}  // namespace

af_status chain_launch(const af_chain_op* ops, int n_ops, void* workspace, size_t ws_bytes, cudaStream_t st,
                       bool single) {
    if (ops == nullptr || n_ops <= 0 || n_ops > kMaxOps) return n_ops > kMaxOps ? AF_ERR_UNSUPPORTED : AF_ERR_INVALID;
    int dev = 0;
    const int sms = device_sm_count(&dev);
    if (sms <= 0) return AF_ERR_CUDA;
    static Params prm;   // 28 KB: not on the stack; the launch copies it
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    bool waits = false;
    size_t scb = 16, xb = 16;
    for (int o = 0; o < n_ops; ++o) {
        const size_t s = op_scale_bytes(ops[o], sms);
        if (s == 0) return AF_ERR_INVALID;
        scb = std::max(scb, s);
        xb = std::max(xb, (size_t)ops[o].K * 2);
        waits |= (o > 0 && ops[o].wait_prev != 0);
    }
    scb = round_up(scb, 128);
    xb = round_up(xb, 128);
    if (waits) {
        if (workspace == nullptr || ws_bytes < af_chain_workspace_bytes(n_ops)) return AF_ERR_WORKSPACE;
        if (!aligned(workspace, 4)) return AF_ERR_INVALID;
    }
    const size_t fixed = xb + 2 * scb + 2048;   // + static shared memory and alignment
    if (fixed + 2 * (size_t)kStage > kSmemCap) return AF_ERR_UNSUPPORTED;
    // one projection: a 5-stage ring (two CTAs per SM, so the next kernel's CTA
    // starts streaming under programmatic dependent launch); a chain: the
    // deepest ring that fits (one CTA per SM)
    int stages = (int)std::min<size_t>(16, (kSmemCap - fixed) / kStage);
    if (single) stages = std::min(stages, 5);
    prm.n_ops = n_ops;
    prm.stages = stages;
    prm.x_bytes = (int)xb;
    prm.sc_bytes = (int)scb;
    prm.counters = waits ? static_cast<int*>(workspace) : nullptr;
    prm.wait_ns = 2000000000ull;
    for (int o = 0; o < n_ops; ++o) {
        const af_chain_op& a = ops[o];
        Op& d = prm.ops[o];
        d.x = static_cast<const __half*>(a.x);
        d.w = static_cast<const uint8_t*>(a.w);
        d.s = static_cast<const uint16_t*>(a.scales);
        d.w2 = static_cast<const uint8_t*>(a.w2);
        d.s2 = static_cast<const uint16_t*>(a.scales2);
        d.norm_w = a.norm_w;
        d.y = static_cast<__half*>(a.y);
        d.xn_out = static_cast<__half*>(a.xn_out);
        d.aux = static_cast<__half*>(a.aux);
        d.kind = a.kind;
        d.N = a.N;
        d.K = a.K;
        d.wait = a.wait_prev != 0;
        d.eps = a.eps;
    }
    Attr& at = g_attr[dev % kMaxDevices];
    std::call_once(at.once, [&] {
        at.err = cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap - 2048);
        if (at.err == cudaSuccess)
            at.err = cudaFuncSetAttribute(chain_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                          (int)cudaSharedmemCarveoutMaxShared);
    });
    if (at.err != cudaSuccess) return cuda_fail(at.err, "chain_kernel attributes");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)stages * kStage + xb + 2 * scb;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (waits) {
        // CTAs wait for one another: all of them must be resident at once
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
    } else {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, chain_kernel, prm);
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "chain_kernel");
}

}  // namespace af

extern "C" size_t af_chain_workspace_bytes(int n_ops) {
    if (n_ops <= 0) return 0;
    return af::round_up((size_t)(n_ops + 1) * 4, 256);
}

extern "C" af_status af_gemv_chain(const af_chain_op* ops, int n_ops, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    return af::chain_launch(ops, n_ops, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), n_ops == 1);
}
