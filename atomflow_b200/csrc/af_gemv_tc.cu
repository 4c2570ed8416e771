// af_gemv_tc.cu -- the W8A16 projection for any number of tokens on the tcgen05
// tensor cores (af_w8a16_gemm_tc: the batched shape launch_linear_gemm declares,
// include/ops/kernel.h:53-59, with the reference's scales; the reference kernel
// handles one token per launch: src/kernel/qkv_gemm.cu:32-150).
//
// Swap-AB: 128 weight rows form the MMA's M, 16 tokens its N, and the
// FP32 accumulators live in tensor memory (TMEM).
//   * Work: a CTA owns one 128-row tile and one contiguous range of the K
//     dimension's 128-position scale groups; the CTAs that split one tile's K
//     form a thread-block cluster (<= 8) and merge their partial sums in rank
//     order through distributed shared memory -- no global workspace, so the
//     drop-in launcher needs no allocation.  Tokens beyond 16 take further
//     grid slices (blockIdx.z).
//   * Warps 4-7 stream: eight lanes fetch one weight row's 128 FP8 bytes of a
//     group (a warp instruction covers four whole rows) with 16-byte cp.async
//     into a ring, plus x's tile; every thread converts exactly the bytes it
//     fetched to FP16 (E4M3 -> FP16 is exact) straight into the MMA's canonical
//     K-major layout (8-row x 16-byte core matrices, no swizzle).  x is copied
//     into the same layout as it arrives, so the MMA reads it in place.
//   * Warp 8 issues, per group, eight K=16 `tcgen05.mma.kind::f16`, each from
//     a zero accumulator into its own TMEM column block (two sets of eight,
//     alternating between groups), and commits them to an mbarrier.
//   * Warps 0-3 drain each finished set (`tcgen05.ld`, one weight row per
//     thread): the eight K=16 partial sums are added in FP32 registers, then
//     multiplied by the row's FP16 group scale and added to the total -- the
//     scale once per 128-position partial sum, and no accumulation inside the
//     tensor core across K steps (its FP32 accumulation truncates; sums that
//     cancel to almost nothing then lose more than the FP16 output can
//     tolerate), as the one-token kernels do.  FP32 row scales multiply the
//     final sum.
//   * Every mbarrier wait is bounded (%globaltimer); a wait that runs out sets
//     AF_FAULT_TC_WAIT, the kernel finishes without waiting further (its
//     outputs invalid) and frees its TMEM.
// No TMA or bulk copy is used, so nothing here can multicast.

#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "af_common.cuh"
#include "af_internal.h"

// Fault bits of this device's tensor-core projections, read by af_device_faults.
__device__ unsigned int g_tc_faults;

namespace af {
namespace {

constexpr int kTcRows = 128;               // weight rows per tile = the MMA's M
constexpr int kTcThreads = 288;            // 4 drain warps, 4 streaming warps, 1 MMA warp
constexpr int kRawGroup = kTcRows * 128;   // FP8 bytes of one tile's group (16 KB)
constexpr int kATile = kTcRows * 256;      // the group as FP16 in the MMA layout (32 KB)
constexpr int kCoreRowGroup = 2048;        // bytes between 8-row core-matrix groups (16 chunks x 128 B)
constexpr uint64_t kTcWaitNs = 2000000000ull;
constexpr size_t kSmemMax = 227 * 1024;    // dynamic shared memory a CTA may opt into

struct TcParams {
    const __half* x;
    const uint8_t* w;
    const void* s;
    __half* y;
    int M, N, K, G;       // tokens, rows, positions, scale groups (K / 128)
    int row_scale;        // 0: FP16 group scales [N][G]; 1: FP32 row scales [N]
    int splits;           // CTAs per row tile along K (the cluster's size)
    int stages;           // ring slots
    int gs_max;           // groups a CTA owns at most
    uint32_t idesc;       // the MMA's instruction descriptor
};

// ---- tcgen05 / async-proxy primitives (PTX ISA, tcgen05 family) ----
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, uint32_t n) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_alloc(uint32_t dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
// 128 consecutive FP32 columns of this warp's 32 TMEM lanes in one load; waits for it.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&r)[128]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
        : "r"(taddr)
        : "memory");
}
// Shared-memory matrix descriptor: K-major, no swizzle; lbo = bytes between the
// two 16-byte core-matrix columns of one K=16 step, sbo = bytes between 8-row
// groups; version 1 (bits 46-47) as tcgen05 requires; layout type 0 (none).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

// cp.async.wait_group with a run-time count (the instruction takes an immediate)
__device__ __forceinline__ void cp_async_wait_dyn(int n) {
    switch (n) {
        case 0: cp_async_wait<0>(); break;
        case 1: cp_async_wait<1>(); break;
        case 2: cp_async_wait<2>(); break;
        case 3: cp_async_wait<3>(); break;
        case 4: cp_async_wait<4>(); break;
        case 5: cp_async_wait<5>(); break;
        default: cp_async_wait<6>(); break;
    }
}

// Bounded mbarrier wait: false once the limit has passed (the fault bit is set).
__device__ __forceinline__ bool tc_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    if (*abort) return false;
    if (mbar_wait_bounded(bar, parity, kTcWaitNs)) return true;
    atomicOr(&g_tc_faults, (unsigned)AF_FAULT_TC_WAIT);
    *abort = 1;
    return false;
}

template <int NT>
__global__ void __launch_bounds__(kTcThreads, 1) gemv_tc_kernel(const TcParams p) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ __align__(8) uint64_t a_full[2], mma_done[2], tmem_empty[2];
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_abort;

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int tile = blockIdx.y;
    const int tok0 = blockIdx.z * NT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g0 = (int)((long long)rank * p.G / p.splits);
    const int g1 = (int)((long long)(rank + 1) * p.G / p.splits);
    const int ng = g1 - g0;
    const int S = p.stages, D = p.stages - 2;

    unsigned char* a_buf = smem;                                   // 2 x 32 KB FP16 A tiles
    unsigned char* x_ring = smem + 2 * kATile;                     // S x NT x 256 B
    unsigned char* raw_ring = x_ring + (size_t)S * NT * 256;       // S x 16 KB FP8
    uint16_t* sc_s = reinterpret_cast<uint16_t*>(raw_ring + (size_t)S * kRawGroup);   // [gs][128]
    constexpr uint32_t kTmemCols = 2 * 8 * NT;   // two sets of eight K=16 blocks

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&a_full[b]), 128);
            mbar_init(smem_u32(&mma_done[b]), 1);
            mbar_init(smem_u32(&tmem_empty[b]), 128);
        }
        s_abort = 0;
        mbar_init_fence();
    }
    if (warp == 8) {
        tmem_alloc(smem_u32(&s_tmem), kTmemCols);
        tmem_relinquish();
    }
    // this CTA's group scales, transposed to [group][row] (FP16 bits; rows past N: 0)
    if (warp < 4 && !p.row_scale) {
        const int r = threadIdx.x;
        const int row = tile * kTcRows + r;
        const uint16_t* src = static_cast<const uint16_t*>(p.s) + (size_t)row * p.G + g0;
        for (int j = 0; j < ng; ++j) sc_s[j * kTcRows + r] = row < p.N ? __ldg(src + j) : (uint16_t)0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp >= 4 && warp < 8) {
        // ---------------------------------------------------- stream + dequantise
        // chunk i = d + 128 k (k < 8) of a group: row i >> 3, 16-byte piece i & 7 --
        // eight lanes read one row's 128 contiguous bytes, a warp four rows
        const int d = threadIdx.x - 128;
        auto issue = [&](int j) {   // group j of this CTA -> ring slot j % S
            const int slot = j % S;
            const size_t kpos = (size_t)(g0 + j) * 128;
            const uint32_t raw = smem_u32(raw_ring + (size_t)slot * kRawGroup);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int i = d + 128 * k, rr = i >> 3, row = tile * kTcRows + rr;
                const bool ok = row < p.N;
                cp_async16_zfill(raw + i * 16, p.w + (ok ? (size_t)row * p.K + kpos + (i & 7) * 16 : 0),
                                 ok ? 16u : 0u);
            }
            const uint32_t xs = smem_u32(x_ring + (size_t)slot * NT * 256);
            for (int i = d; i < NT * 16; i += 128) {
                const int t = i >> 4, kc = i & 15;
                const bool ok = tok0 + t < p.M;
                const __half* src = p.x + (ok ? (size_t)(tok0 + t) * p.K + kpos + kc * 8 : 0);
                cp_async16_zfill(xs + (t >> 3) * kCoreRowGroup + kc * 128 + (t & 7) * 16, src, ok ? 16u : 0u);
            }
        };
        for (int j = 0; j < D; ++j) {
            if (j < ng) issue(j);
            cp_async_commit();
        }
        for (int j = 0; j < ng; ++j) {
            // A[j & 1] and ring slot (j + D) % S were last read by group j - 2's MMAs
            if (j >= 2) tc_wait(smem_u32(&mma_done[j & 1]), ((j - 2) >> 1) & 1, &s_abort);
            if (j + D < ng) issue(j + D);
            cp_async_commit();
            cp_async_wait_dyn(D);   // this thread's copies of group j have landed
            const unsigned char* raw = raw_ring + (size_t)(j % S) * kRawGroup;
            unsigned char* a = a_buf + (size_t)(j & 1) * kATile;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                // this thread's own piece: 16 FP8 of row rr at positions 16c..16c+15 ->
                // the two FP16 core-matrix columns 2c, 2c + 1 of that row
                const int i = d + 128 * k, rr = i >> 3, c = i & 7;
                const uint4 q = *reinterpret_cast<const uint4*>(raw + i * 16);
                uint4 lo, hi;
                lo.x = e4m3x2_lo(q.x);
                lo.y = e4m3x2_hi(q.x);
                lo.z = e4m3x2_lo(q.y);
                lo.w = e4m3x2_hi(q.y);
                hi.x = e4m3x2_lo(q.z);
                hi.y = e4m3x2_hi(q.z);
                hi.z = e4m3x2_lo(q.w);
                hi.w = e4m3x2_hi(q.w);
                unsigned char* ar = a + (size_t)(rr >> 3) * kCoreRowGroup + (rr & 7) * 16;
                *reinterpret_cast<uint4*>(ar + (2 * c) * 128) = lo;
                *reinterpret_cast<uint4*>(ar + (2 * c + 1) * 128) = hi;
            }
            fence_async_smem();   // the A tile and x's cp.async bytes become visible to the MMA
            mbar_arrive(smem_u32(&a_full[j & 1]));
        }
        cp_async_wait<0>();
    } else if (warp == 8) {
        // ------------------------------------------------------------- MMA issue
        for (int j = 0; j < ng; ++j) {
            tc_wait(smem_u32(&a_full[j & 1]), (j >> 1) & 1, &s_abort);
            if (j >= 2) tc_wait(smem_u32(&tmem_empty[j & 1]), ((j - 2) >> 1) & 1, &s_abort);
            tc_fence_after();
            if (lane == 0 && !s_abort) {
                const uint32_t a0 = smem_u32(a_buf + (size_t)(j & 1) * kATile);
                const uint32_t b0 = smem_u32(x_ring + (size_t)(j % S) * NT * 256);
                const uint32_t dcol = tmem + (uint32_t)(j & 1) * 8 * NT;
#pragma unroll
                for (int s = 0; s < 8; ++s)
                    tc_mma(dcol + s * NT, smem_desc(a0 + s * 256, 128, kCoreRowGroup),
                           smem_desc(b0 + s * 256, 128, kCoreRowGroup), p.idesc, 0u);
                tc_commit(smem_u32(&mma_done[j & 1]));
            }
            __syncwarp();
        }
        // every MMA has finished before the TMEM is freed below
        if (ng > 0) tc_wait(smem_u32(&mma_done[(ng - 1) & 1]), ((ng - 1) >> 1) & 1, &s_abort);
    }

    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    const int r = threadIdx.x;   // drain warps: this thread's row of the tile (TMEM lane)
    if (warp < 4) {
        // ------------------------------------------------------------ drain
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        for (int j = 0; j < ng; ++j) {
            const bool ok = tc_wait(smem_u32(&mma_done[j & 1]), (j >> 1) & 1, &s_abort);
            tc_fence_after();
            if (ok) {
                const float sc = p.row_scale ? 1.f : half_bits_to_float(sc_s[j * kTcRows + r]);
                // the set's 8 x NT columns (k-step s, token t at column s * NT + t) in
                // 128-column loads; each group's K=16 partial sums are added in K order
                float gsum[NT];
                constexpr int kLd = 128;   // columns per load: the whole set
                static_assert(8 * NT % kLd == 0, "whole loads per set");
#pragma unroll
                for (int h = 0; h < 8 * NT / kLd; ++h) {
                    uint32_t v[kLd];
                    tmem_ld128(lane_base + (uint32_t)(j & 1) * 8 * NT + h * kLd, v);
#pragma unroll
                    for (int c = 0; c < kLd; ++c) {
                        const int col = h * kLd + c, st = col / NT, t = col % NT;
                        gsum[t] = st == 0 ? __uint_as_float(v[c]) : gsum[t] + __uint_as_float(v[c]);
                    }
                }
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[t] = fmaf(sc, gsum[t], acc[t]);
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&tmem_empty[j & 1]));
        }
        const int row = tile * kTcRows + r;
        if (p.row_scale && row < p.N) {
            const float rs = __ldg(static_cast<const float*>(p.s) + row);
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t] *= rs;
        }
    }
    // the ring is idle now (every copy landed, every MMA finished): partial sums go there
    __syncthreads();
    float* part = reinterpret_cast<float*>(raw_ring);   // [NT][128]
    if (warp < 4) {
#pragma unroll
        for (int t = 0; t < NT; ++t) part[t * kTcRows + r] = acc[t];
    }
    cluster.sync();   // every CTA's partial is visible to the cluster
    if (rank == 0 && warp < 4) {
        const int row = tile * kTcRows + r;
        if (row < p.N) {
            for (int t = 0; t < NT && tok0 + t < p.M; ++t) {
                float sum = 0.f;
                for (int q = 0; q < p.splits; ++q)   // rank order: deterministic
                    sum += cluster.map_shared_rank(part, q)[t * kTcRows + r];
                p.y[(size_t)(tok0 + t) * p.N + row] = __float2half_rn(sum);
            }
        }
    }
    tc_fence_before();
    cluster.sync();   // no CTA leaves while rank 0 reads its partial
    if (warp == 8) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

struct TcAttr {
    std::once_flag once;
    cudaError_t err = cudaSuccess;
};
TcAttr g_tc_attr[kMaxDevices];

template <int NT>
cudaError_t tc_launch_nt(const TcParams& prm, dim3 grid, size_t smem, cudaStream_t st, int dev) {
    auto kern = gemv_tc_kernel<NT>;
    TcAttr& at = g_tc_attr[dev % kMaxDevices];
    std::call_once(at.once, [&] {
        at.err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kSmemMax - 2048));
        if (at.err == cudaSuccess)
            at.err = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                          (int)cudaSharedmemCarveoutMaxShared);
    });
    if (at.err != cudaSuccess) return at.err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = grid.x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, prm);
}

// Clusters of `splits` CTAs that fit on the device at once (cached per device and size).
int tc_max_clusters(int dev, int splits, size_t smem) {
    static std::mutex mu;
    static int cache[kMaxDevices][9];
    std::lock_guard<std::mutex> lock(mu);
    int& c = cache[dev % kMaxDevices][splits];
    if (c > 0) return c;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, 1, 1);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemv_tc_kernel<16>, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = 1;
    }
    c = n;
    return n;
}

}  // namespace

bool tc_ok(int M, int K, bool row_scale, const void* x, const void* w, const void* s, const void* y) {
    if (M < 1 || K <= 0 || K % 128 != 0) return false;
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 2)) return false;
    return row_scale ? aligned(s, 4) : aligned(s, 2);
}

af_status tc_launch(const void* x, const void* w, const void* s, bool row_scale, void* y, int M, int N, int K,
                    cudaStream_t st) {
    int dev = 0;
    const int sms = device_sm_count(&dev);
    if (sms <= 0) return AF_ERR_CUDA;
    constexpr int NT = 16;   // tokens per pass (32 would spill the drain's registers)
    const int G = K / 128;
    const int tiles = (N + kTcRows - 1) / kTcRows;
    const int zb = (M + NT - 1) / NT;
    const size_t slot = (size_t)kRawGroup + (size_t)NT * 256;
    const size_t cap = kSmemMax - 2048;
    // K split over the largest cluster whose clusters all fit on the GPU at once
    int splits = std::max(1, std::min(std::min(sms / std::max(1, tiles * zb), 8), G));
    int stages = 0, gs_max = 0;
    size_t smem = 0;
    for (; splits >= 1; --splits) {
        gs_max = (G + splits - 1) / splits;
        const size_t fixed = 2 * (size_t)kATile + (size_t)gs_max * kTcRows * 2 + 1024;
        if (fixed + 4 * slot > cap) continue;
        stages = (int)std::min<size_t>(8, (cap - fixed) / slot);
        smem = 2 * (size_t)kATile + (size_t)stages * slot + (size_t)gs_max * kTcRows * 2;
        if (splits == 1 || tiles * zb <= tc_max_clusters(dev, splits, smem)) break;
    }
    if (splits < 1 || stages < 4) return AF_ERR_UNSUPPORTED;
    TcParams prm{};
    prm.x = static_cast<const __half*>(x);
    prm.w = static_cast<const uint8_t*>(w);
    prm.s = s;
    prm.y = static_cast<__half*>(y);
    prm.M = M;
    prm.N = N;
    prm.K = K;
    prm.G = G;
    prm.row_scale = row_scale ? 1 : 0;
    prm.splits = splits;
    prm.stages = stages;
    prm.gs_max = gs_max;
    // instruction descriptor (kind::f16): FP32 accumulator (bits 4-5 = 1), A and
    // B FP16 (formats 0), both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28
    prm.idesc = (1u << 4) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
    const dim3 grid(splits, tiles, zb);
    cudaError_t e = tc_launch_nt<NT>(prm, grid, smem, st, dev);
    return e == cudaSuccess ? AF_OK : cuda_fail(e, "gemv_tc_kernel");
}

unsigned tc_faults(bool clear, cudaError_t* err) {
    unsigned v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_faults, sizeof(v));
    if (e == cudaSuccess && clear && v != 0) {
        const unsigned z = 0;
        e = cudaMemcpyToSymbol(g_tc_faults, &z, sizeof(z));
    }
    *err = e;
    return v;
}

}  // namespace af

extern "C" af_status af_w8a16_gemm_tc(const void* x, const void* w, const void* scales, void* y, int M, int N, int K,
                                     int group_size, af_scale_kind kind, void* stream) {
    if (M <= 0 || N <= 0 || K <= 0) return (M == 0 || N == 0) ? AF_OK : AF_ERR_INVALID;
    if (x == nullptr || w == nullptr || y == nullptr || scales == nullptr) return AF_ERR_INVALID;
    if (kind == AF_SCALE_GROUP_F16 && group_size != 128) return AF_ERR_INVALID;
    if (kind != AF_SCALE_GROUP_F16 && kind != AF_SCALE_ROW_F32) return AF_ERR_INVALID;
    if (!af::tc_ok(M, K, kind == AF_SCALE_ROW_F32, x, w, scales, y)) return AF_ERR_INVALID;
    return af::tc_launch(x, w, scales, kind == AF_SCALE_ROW_F32, y, M, N, K, static_cast<cudaStream_t>(stream));
}
