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

constexpr int kRefWarps = 8;                // the reference kernel's 256 threads
constexpr int kCWarps = 8;                  // consumer warps: thread t plays the reference's thread t
constexpr int kThreads = (kCWarps + 1) * 32;  // + one producer warp
constexpr int kRows = 16;                   // rows per stage
constexpr int kBlk = 1024;                  // the reference's j-stride (positions)
constexpr int kBPS = 3;                     // j-blocks per stage: 3 KB row copies (TMA bulk copies of
                                            // 1-2 KB cannot keep HBM busy; >= 3 KB per copy can)
constexpr int kRowB = kBlk * kBPS;          // bytes of a row in a stage
// stage row pitch: the exact consumers read 4 consecutive bytes per lane (any
// pitch is conflict-free); the tensor-core consumers read 16-byte pieces of rows
// g and g + 1 in one quarter-warp, so their rows sit 16 bytes apart modulo 128
template <bool EXACT>
__host__ __device__ constexpr int pitch() { return EXACT ? kRowB : kRowB + 16; }
template <bool EXACT>
__host__ __device__ constexpr int stage_bytes() { return kRows * pitch<EXACT>(); }
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
    int unused;
    float eps;
};

struct Params {
    int n_ops;
    int stages;                 // ring stages
    int x_bytes, sc_bytes;      // shared carve-up: x [K] FP16 (two of them), one staged-scale buffer (two of them),
    int sct_bytes;              // and the transposed scales of the current op
    int* counters;              // [n_ops + 1] completion counters (null: no op waits)
    unsigned long long wait_ns;
    Op ops[kMaxOps];
};

static_assert(sizeof(Params) <= 32764, "the op table must fit the kernel parameter space");

// One more finished tile: a release add, so the tile's output rows (stored by
// this warp before the __syncwarp that precedes it) are visible to whoever
// acquires the count.
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

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

// Shared-memory loads by 32-bit shared address (volatile: a ring slot's
// contents change between the mbarrier phases that guard it).
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint16_t lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
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

// EXACT: the reference's arithmetic, bit for bit.  !EXACT: the same data flow
// with the dot products on the tensor cores (FP8 -> FP16 packed conversion,
// m16n8k16 MMAs with FP32 accumulation, the group scale applied to each
// 128-position group sum, warps combined in a fixed order): deterministic, and
// within the FP16 rounding of FP64, but not the reference's summation order.
template <bool EXACT>
__global__ void __launch_bounds__(kThreads, 1) chain_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    constexpr int kStage = stage_bytes<EXACT>();
    constexpr int kPitch = pitch<EXACT>();
    const int S = p.stages;
    unsigned char* ring = smem;
    // x of op o sits in buffer o & 1: an op that does not wait for the previous
    // one has its x fetched (cp.async) while the previous op computes
    unsigned char* const xbase = smem + (size_t)S * kStage;
    auto xbuf = [&](int o) { return reinterpret_cast<__half*>(xbase + (size_t)(o & 1) * p.x_bytes); };
    unsigned char* scb = smem + (size_t)S * kStage + 2 * (size_t)p.x_bytes;
    uint16_t* sct = reinterpret_cast<uint16_t*>(scb + 2 * (size_t)p.sc_bytes);   // [m][G][rows_pad]
    __shared__ __align__(8) uint64_t full[16], empty[16], sc_full[2], sc_empty[2];
    // warp sums of the last 8 tiles: consumer warps run at most one ring (<= 6
    // stages, >= 1 stage per tile) apart, so a tile's buffer is free again
    // before any warp reaches the tile 8 later
    __shared__ float part[8][kRefWarps][kRows];
    __shared__ int s_tcnt[8];                       // warps done with each of them
    __shared__ int s_opdone[2];                     // tiles of the current op finished (op parity)
    __shared__ __align__(16) uint32_t s_zero[64];   // B fragments of the MMA columns that carry no token
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
        for (int i = 0; i < 8; ++i) s_tcnt[i] = 0;
        s_opdone[0] = s_opdone[1] = 0;
        for (int i = 0; i < 64; ++i) s_zero[i] = 0;
        mbar_init_fence();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kCWarps) {
        // ------------------------------------------------------------ producer
        int slot = 0;
        uint32_t phase = 0;
        int issued = 0;
        // this CTA's group scales of op o -> scale buffer o & 1 (issued one op
        // ahead, so that waiting on its plain loads never holds up the weights)
        auto stage_scales = [&](int o) {
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
        };
        stage_scales(0);
        for (int o = 0; o < p.n_ops && !s_abort; ++o) {
            const Op& op = p.ops[o];
            const RowSplit rs = row_split(op);
            const bool pair = op.kind == OP_RMSNORM_SWIGLU;

            const int nst = (op.K + kRowB - 1) / kRowB;   // stages per 16-row tile
            for (int tr = rs.r0; tr < rs.r1; tr += rs.tr) {
                const int nv = min(rs.tr, rs.r1 - tr);
                for (int j = 0; j < nst; ++j) {
                    chain_wait(smem_u32(&empty[slot]), phase ^ 1, p.wait_ns, &s_abort);
                    if (s_abort) break;
                    const int bb = min(kRowB, op.K - j * kRowB);
                    const uint32_t fb = smem_u32(&full[slot]);
                    if (lane == 0) mbar_arrive_expect_tx(fb, (uint32_t)((pair ? 2 * nv : nv) * bb));
                    __syncwarp();
                    if (lane < kRows) {
                        const uint8_t* src = nullptr;
                        if (pair) {
                            const int r = lane & 7;
                            if (r < nv) src = (lane < 8 ? op.w : op.w2) + (size_t)(tr + r) * op.K + (size_t)j * kRowB;
                        } else if (lane < nv) {
                            src = op.w + (size_t)(tr + lane) * op.K + (size_t)j * kRowB;
                        }
                        if (src) bulk_g2s(smem_u32(ring + (size_t)slot * kStage + lane * kPitch), src, (uint32_t)bb, fb);
                    }
                    ++issued;
                    if (++slot == S) {
                        slot = 0;
                        phase ^= 1;
                    }
                }
                if (s_abort) break;
            }
            if (o + 1 < p.n_ops && !s_abort) stage_scales(o + 1);
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
        const int ct = threadIdx.x;                 // consumer thread
        const int t = ct;                           // = the reference's thread index
        pdl_wait();                  // x / residual inputs of the first ops may come from the previous kernel
        int slot = 0;
        uint32_t phase = 0;
        int tb = 0;
        bool ready = false;   // the next stage's full barrier tested complete
        bool x_pref = false;  // this op's x was fetched during the previous op
        for (int o = 0; o < p.n_ops; ++o) {
            const Op& op = p.ops[o];
            const RowSplit rs = row_split(op);
            const bool pair = op.kind == OP_RMSNORM_SWIGLU;
            const int G = op.K >> 7;
            const int K = op.K;
            if (o > 0) named_bar_sync(1, kCWarps * 32);   // every warp is done with the previous op's x and scales
            // this CTA's scales of the op: [rows][G] -> [G][rows_pad] (gate's, then up's), so
            // that a thread's 16 stage rows at one group are 32 contiguous bytes -- done
            // before the dependency wait, which it does not need
            const int b = o & 1;
            chain_wait(smem_u32(&sc_full[b]), (o >> 1) & 1, p.wait_ns, &s_abort);
            const ScaleLayout sl = scale_layout(op, rs, G);
            const int rows = rs.r1 - rs.r0, rows_pad = (rows + 15) & ~15;
            for (int m = 0; m < (pair ? 2 : 1); ++m) {
                const uint16_t* src = reinterpret_cast<const uint16_t*>(scb + (size_t)b * p.sc_bytes + sl.off[m]);
                uint16_t* dst = sct + (size_t)m * G * rows_pad;
                for (int i = ct; i < rows * G; i += kCWarps * 32) {
                    const int r = i / G, gg = i - r * G;
                    dst[gg * rows_pad + r] = src[i];
                }
            }
            if (op.wait && o > 0 && p.counters != nullptr && ct == 0 && !s_abort) {
                // op o reads what op o-1 wrote: wait until every CTA has finished it
                const unsigned long long t0 = globaltimer_ns();
                while (ld_acquire_gpu(p.counters + o - 1) < (int)gridDim.x) {
                    if (globaltimer_ns() - t0 > p.wait_ns) {
                        atomicOr(&g_chain_faults, (unsigned)AF_FAULT_CHAIN_WAIT);
                        s_abort = 1;
                        break;
                    }
                }
            }
            if (x_pref) cp_async_wait<0>();   // this op's x, fetched during the previous op
            named_bar_sync(1, kCWarps * 32);
            __half* xs = xbuf(o);
            if (!x_pref) {
                // x -> shared (L2-coherent loads: another CTA may have written it)
                for (int i = ct * 8; i < K; i += kCWarps * 32 * 8)
                    *reinterpret_cast<uint4*>(xs + i) = ldcg_u4(op.x + i);
                named_bar_sync(1, kCWarps * 32);
            }
            // The next op's x, if that op reads nothing this one writes (it does
            // not wait): its buffer was last read by op o - 1, which every warp
            // has finished (the barrier at this op's start), and any op it might
            // depend on further back finished before this op's wait above.
            x_pref = false;
            if (o + 1 < p.n_ops && !p.ops[o + 1].wait) {   // uniform: every thread takes the same branch
                const Op& nx = p.ops[o + 1];
                const uint32_t xd = smem_u32(xbuf(o + 1));
                for (int i = ct * 8; i < nx.K; i += kCWarps * 32 * 8) cp_async16(xd + 2 * i, nx.x + i);
                cp_async_commit();
                x_pref = true;
            }
            if (op.kind == OP_RMSNORM_GEMV || op.kind == OP_RMSNORM_SWIGLU) {
                // RMSNorm of x in the reference's arithmetic (src/kernel/rmsnorm.cu:9-67,
                // 128 threads): strided FMA sums, shuffle-down tree 1..16, the four
                // warp sums in order, rsqrt(sum / K + eps) as its fast-math build
                // evaluates it, then half(x * r * w).
                if (ct < 128) {
                    float ss = 0.f;
                    for (int i = ct; i < K; i += 128) {
                        const float v = __half2float(xs[i]);
                        ss = fmaf(v, v, ss);
                    }
#pragma unroll
                    for (int off = 1; off < 32; off <<= 1) ss += __shfl_down_sync(0xffffffffu, ss, off);
                    if (lane == 0) s_nrm[warp] = ss;
                }
                named_bar_sync(1, kCWarps * 32);
                if (ct == 0) s_r = rms_scale_ref(((s_nrm[0] + s_nrm[1]) + s_nrm[2]) + s_nrm[3], K, op.eps);
                named_bar_sync(1, kCWarps * 32);
                const float r = s_r;
                for (int i = ct; i < K; i += kCWarps * 32)
                    xs[i] = __float2half_rn(__half2float(xs[i]) * r * __ldg(op.norm_w + i));
                named_bar_sync(1, kCWarps * 32);
                if (op.xn_out != nullptr && blockIdx.x == 0)
                    for (int i = ct; i < K; i += kCWarps * 32) op.xn_out[i] = xs[i];
            }
            const uint32_t sct_u = smem_u32(sct);
            const uint32_t up_off = (uint32_t)G * rows_pad * 2;   // bytes from gate's block to up's
            const uint32_t ring_u = smem_u32(ring) + 4 * t;   // exact path: thread t's 4 bytes of a row
            const uint32_t ring_m = smem_u32(ring);
            const uint32_t xs_u = smem_u32(xs);

            for (int tr = rs.r0; tr < rs.r1; tr += rs.tr) {
                const int nv = min(rs.tr, rs.r1 - tr);
                const uint32_t toff = (uint32_t)(tr - rs.r0) * 2;   // this tile's rows in a transposed group row
                if constexpr (EXACT) {
                float acc[kRows];
#pragma unroll
                for (int i = 0; i < kRows; ++i) acc[i] = 0.f;
                const int nst = (K + kRowB - 1) / kRowB;
                for (int j = 0; j < nst; ++j) {
                    // the stage's full barrier was tested (non-blocking) while the
                    // previous stage was computed; wait only if it was not complete
                    if (!ready) chain_wait(smem_u32(&full[slot]), phase, p.wait_ns, &s_abort);
                    {
                        const int ns = slot + 1 == S ? 0 : slot + 1;
                        ready = mbar_test_wait(smem_u32(&full[ns]), ns == 0 ? phase ^ 1 : phase);
                    }
                    const uint32_t st = ring_u + (uint32_t)slot * kStage;
#pragma unroll
                    for (int jb = 0; jb < kBPS; ++jb) {
                        const int kp = (j * kBPS + jb) * kBlk + 4 * t;   // the reference's kv for this j
                        if (kp < K) {
                            const uint2 xr = lds64(xs_u + 2 * kp);
                            const float2 x01 = __half22float2(*reinterpret_cast<const __half2*>(&xr.x));
                            const float2 x23 = __half22float2(*reinterpret_cast<const __half2*>(&xr.y));
                            const uint32_t sa = sct_u + (uint32_t)(kp >> 7) * rows_pad * 2 + toff;
                            const uint4 sv0 = lds128(sa);                          // rows 0-7 (gate's for SwiGLU)
                            const uint4 sv1 = lds128(pair ? sa + up_off : sa + 16);  // rows 8-15 (up's for SwiGLU)
                            const uint32_t sw[8] = {sv0.x, sv0.y, sv0.z, sv0.w, sv1.x, sv1.y, sv1.z, sv1.w};
#pragma unroll
                            for (int i = 0; i < kRows; i += 2) {
                                const uint32_t w0 = lds32(st + i * kRowB + jb * kBlk);
                                const uint32_t w1 = lds32(st + (i + 1) * kRowB + jb * kBlk);
                                const uint16_t s0 = (uint16_t)(sw[i >> 1] & 0xffffu), s1 = (uint16_t)(sw[i >> 1] >> 16);
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
                } else {
                // tensor-core path: warp w takes positions [384 w, 384 w + 384) of
                // each stage (three scale groups); lane (g, c) feeds rows g and g + 8
                const int g = lane >> 2, c = lane & 3;
                float acc0 = 0.f, acc1 = 0.f;   // rows g, g + 8 (column 0 of the MMA: lanes c == 0)
                const uint32_t xlane = g == 0 ? xs_u + 64 * c : smem_u32(s_zero);   // columns 1..7 carry zeros
                const uint32_t xstep = g == 0 ? 1u : 0u;
                const uint32_t srow0 = toff + 2 * g;                         // row g's scale in a transposed group row
                const uint32_t srow1 = pair ? up_off + toff + 2 * g : toff + 2 * (g + 8);
                const int nst = (K + kRowB - 1) / kRowB;
                for (int j = 0; j < nst; ++j) {
                    if (!ready) chain_wait(smem_u32(&full[slot]), phase, p.wait_ns, &s_abort);
                    {
                        const int ns = slot + 1 == S ? 0 : slot + 1;
                        ready = mbar_test_wait(smem_u32(&full[ns]), ns == 0 ? phase ^ 1 : phase);
                    }
                    const uint32_t rowg =
                        ring_m + (uint32_t)slot * kStage + (uint32_t)g * kPitch + warp * (kBPS * 128) + c * 32;
#pragma unroll
                    for (int gg = 0; gg < kBPS; ++gg) {
                        const int gp = j * kRowB + warp * (kBPS * 128) + gg * 128;   // the group's first position
                        if (gp < K) {
                            const uint32_t ra = rowg + gg * 128;
                            const uint4 r0a = lds128(ra), r0b = lds128(ra + 16);
                            const uint4 r1a = lds128(ra + 8 * kPitch), r1b = lds128(ra + 8 * kPitch + 16);
                            const uint32_t xa = xlane + xstep * 2u * (uint32_t)gp;
                            const uint4 xq0 = lds128(xa), xq1 = lds128(xa + 16), xq2 = lds128(xa + 32),
                                        xq3 = lds128(xa + 48);
                            const uint32_t w0[8] = {r0a.x, r0a.y, r0a.z, r0a.w, r0b.x, r0b.y, r0b.z, r0b.w};
                            const uint32_t w1[8] = {r1a.x, r1a.y, r1a.z, r1a.w, r1b.x, r1b.y, r1b.z, r1b.w};
                            const uint32_t xw[16] = {xq0.x, xq0.y, xq0.z, xq0.w, xq1.x, xq1.y, xq1.z, xq1.w,
                                                     xq2.x, xq2.y, xq2.z, xq2.w, xq3.x, xq3.y, xq3.z, xq3.w};
                            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                            for (int m = 0; m < 8; ++m)
                                mma16816(d, e4m3x2_lo(w0[m]), e4m3x2_lo(w1[m]), e4m3x2_hi(w0[m]), e4m3x2_hi(w1[m]),
                                         xw[2 * m], xw[2 * m + 1]);
                            const uint32_t sg = sct_u + (uint32_t)(gp >> 7) * rows_pad * 2;
                            acc0 = fmaf(half_bits_to_float(lds16(sg + srow0)), d[0], acc0);
                            acc1 = fmaf(half_bits_to_float(lds16(sg + srow1)), d[2], acc1);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&empty[slot]));
                    if (++slot == S) {
                        slot = 0;
                        phase ^= 1;
                    }
                }
                if (c == 0) {
                    part[tb][warp][g] = acc0;
                    part[tb][warp][g + 8] = acc1;
                }
                }
                // the last warp done with the tile finishes it (no CTA-wide barrier per tile)
                __syncwarp();
                int last = 0;
                if (lane == 0) {
                    __threadfence_block();
                    last = atomicAdd(&s_tcnt[tb], 1) == kCWarps - 1;
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence_block();
                    if (lane < (pair ? 8 : 16) && lane < nv) {
                        // the warp sums in warp order, from 0.0f, then the op's epilogue
                        float tot = 0.f;
#pragma unroll
                        for (int w = 0; w < kRefWarps; ++w) tot += part[tb][w][lane];
                        const int row = tr + lane;
                        if (pair) {
                            float up = 0.f;
#pragma unroll
                            for (int w = 0; w < kRefWarps; ++w) up += part[tb][w][8 + lane];
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
                    __syncwarp();   // the tile's rows are stored
                    if (lane == 0) {
                        s_tcnt[tb] = 0;
                        // count the tile in the CTA (release at CTA scope: the warp's row
                        // stores come first); the CTA's last tile of the op publishes the
                        // CTA's rows with one GPU-scope release add
                        __threadfence_block();
                        const int ntiles = (rs.r1 - rs.r0 + rs.tr - 1) / rs.tr;
                        if (atomicAdd(&s_opdone[o & 1], 1) == ntiles - 1) {
                            __threadfence_block();   // acquire the CTA's other tiles
                            s_opdone[o & 1] = 0;
                            if (p.counters != nullptr) red_release_gpu_add(p.counters + o, 1);
                        }
                    }
                }
                tb = (tb + 1) & 7;
            }
            // a CTA without rows in this op still reports it done
            if (rs.r1 == rs.r0 && ct == 0 && p.counters != nullptr) red_release_gpu_add(p.counters + o, 1);
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
Attr g_attr[kMaxDevices * 2];

}  // namespace

af_status chain_launch(const af_chain_op* ops, int n_ops, void* workspace, size_t ws_bytes, cudaStream_t st,
                       bool single, bool exact) {
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
    size_t sctb = 128;
    for (int o = 0; o < n_ops; ++o) {
        const size_t rows = ((size_t)ops[o].N + sms - 1) / sms;
        sctb = std::max(sctb, ((rows + 15) / 16 * 16) * (ops[o].K / 128) * 2 *
                                  (ops[o].kind == AF_OP_RMSNORM_SWIGLU ? 2 : 1));
    }
    sctb = round_up(sctb, 128);
    if (waits) {
        if (workspace == nullptr || ws_bytes < af_chain_workspace_bytes(n_ops)) return AF_ERR_WORKSPACE;
        if (!aligned(workspace, 4)) return AF_ERR_INVALID;
    }
    const size_t fixed = 2 * xb + 2 * scb + sctb + 6144;   // + static shared memory and alignment
    const size_t kStage = exact ? stage_bytes<true>() : stage_bytes<false>();
    if (fixed + 2 * kStage > kSmemCap) return AF_ERR_UNSUPPORTED;
    // one projection: a 3-stage ring (two CTAs per SM, so the next kernel's CTA
    // starts streaming under programmatic dependent launch); a chain: the
    // deepest ring that fits (one CTA per SM)
    int stages = (int)std::min<size_t>(6, (kSmemCap - fixed) / kStage);
    if (single) stages = std::min(stages, 3);
    prm.n_ops = n_ops;
    prm.stages = stages;
    prm.x_bytes = (int)xb;
    prm.sc_bytes = (int)scb;
    prm.sct_bytes = (int)sctb;
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
    auto kern = exact ? chain_kernel<true> : chain_kernel<false>;
    Attr& at = g_attr[(dev % kMaxDevices) * 2 + (exact ? 1 : 0)];
    std::call_once(at.once, [&] {
        at.err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap - 6144);
        if (at.err == cudaSuccess)
            at.err = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                          (int)cudaSharedmemCarveoutMaxShared);
    });
    if (at.err != cudaSuccess) return cuda_fail(at.err, "chain_kernel attributes");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)stages * kStage + 2 * xb + 2 * scb + sctb;
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
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, prm);
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "chain_kernel");
}

}  // namespace af

extern "C" size_t af_chain_workspace_bytes(int n_ops) {
    if (n_ops <= 0) return 0;
    return af::round_up((size_t)(n_ops + 1) * 4, 256);
}

extern "C" af_status af_gemv_chain(const af_chain_op* ops, int n_ops, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    return af::chain_launch(ops, n_ops, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), n_ops == 1,
                            true);
}

extern "C" af_status af_gemv_chain_fast(const af_chain_op* ops, int n_ops, void* workspace, size_t workspace_bytes,
                                        void* stream) {
    return af::chain_launch(ops, n_ops, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), n_ops == 1,
                            false);
}
