/*
 * af_oracle.c -- CPU restatement of AtomFlow's W8A16 decode-path arithmetic.
 * TEST INFRASTRUCTURE ONLY (see af_oracle.h): the checker, never the product.
 *
 * Built with -ffp-contract=off so every FP32 operation rounds exactly where
 * this source says; fmaf() is used where the reference kernel's nvcc build
 * fuses a multiply into an add.
 */
#include "af_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ formats --- */

float af_oracle_e4m3_to_float(uint8_t b) {
    /* OCP E4M3: s eeee mmm, bias 7; e == 0 subnormal (m * 2^-9); S.1111.111 NaN. */
    const int sign = b >> 7, e = (b >> 3) & 15, m = b & 7;
    float v;
    if (e == 15 && m == 7)
        v = NAN;
    else if (e == 0)
        v = ldexpf((float)m, -9);
    else
        v = ldexpf((float)(8 + m), e - 10);
    return sign ? -v : v;
}

uint8_t af_oracle_float_to_e4m3_rn(float f) {
    /* Round to nearest, ties to even, on the E4M3 grid; |f| >= 480 (where the
     * rounded value would leave the format) -> NaN, as torch's float8_e4m3fn. */
    if (isnan(f)) return 0x7F;
    const uint8_t sign = signbit(f) ? 0x80 : 0x00;
    float a = fabsf(f);
    if (a >= 480.0f) return sign | 0x7F;
    if (a == 0.0f) return sign;
    int e;
    frexpf(a, &e);              /* a = fr * 2^e, fr in [0.5, 1) -> unbiased exponent e-1 */
    int ue = e - 1;
    if (ue < -6) ue = -6;       /* subnormal range shares the 2^-6 binade's quantum */
    const float quantum = ldexpf(1.0f, ue - 3);
    float r = nearbyintf(a / quantum) * quantum; /* a/quantum exact (power of 2) */
    if (r == 0.0f) return sign;
    if (r > 448.0f) return sign | 0x7F;
    int e2;
    frexpf(r, &e2);
    int ue2 = e2 - 1;
    if (ue2 < -6) {
        /* subnormal: r = m * 2^-9 */
        const int m = (int)ldexpf(r, 9);
        return sign | (uint8_t)m;
    }
    const int m = (int)(ldexpf(r, -ue2) * 8.0f) - 8;
    return sign | (uint8_t)(((ue2 + 7) << 3) | m);
}

float af_oracle_half_to_float(uint16_t h) {
    const int sign = h >> 15, e = (h >> 10) & 31, m = h & 1023;
    float v;
    if (e == 31)
        v = m ? NAN : INFINITY;
    else if (e == 0)
        v = ldexpf((float)m, -24);
    else
        v = ldexpf((float)(1024 + m), e - 25);
    return sign ? -v : v;
}

uint16_t af_oracle_float_to_half_rn(float f) {
    if (isnan(f)) return 0x7E00;
    const uint16_t sign = signbit(f) ? 0x8000 : 0;
    float a = fabsf(f);
    if (a == 0.0f) return sign;
    if (a >= 65520.0f) return sign | 0x7C00; /* rounds past 65504 -> inf */
    int e;
    frexpf(a, &e);
    int ue = e - 1;
    if (ue < -14) ue = -14;
    const float quantum = ldexpf(1.0f, ue - 10);
    const float r = nearbyintf(a / quantum) * quantum;
    if (r == 0.0f) return sign;
    int e2;
    frexpf(r, &e2);
    const int ue2 = e2 - 1;
    if (ue2 < -14) return sign | (uint16_t)ldexpf(r, 24);
    const int m = (int)(ldexpf(r, -ue2) * 1024.0f) - 1024;
    return sign | (uint16_t)(((ue2 + 15) << 10) | m);
}

/* ---------------------------------------------------------- quantiser --- */

void af_oracle_quantize_gs128(const float* w, int N, int K, uint8_t* q, uint16_t* s) {
    const int G = K / 128;
    for (int n = 0; n < N; ++n) {
        for (int g = 0; g < G; ++g) {
            const float* src = w + (size_t)n * K + (size_t)g * 128;
            float mx = 0.0f;
            for (int k = 0; k < 128; ++k) {
                const float a = fabsf(src[k]);
                if (a > mx) mx = a;
            }
            const float scale = mx > 0.0f ? mx / 448.0f : 1.0f;
            for (int k = 0; k < 128; ++k) {
                float t = src[k] / scale;
                if (t > 448.0f) t = 448.0f;
                if (t < -448.0f) t = -448.0f;
                q[(size_t)n * K + (size_t)g * 128 + k] = af_oracle_float_to_e4m3_rn(t);
            }
            s[(size_t)n * G + g] = af_oracle_float_to_half_rn(scale);
        }
    }
}

void af_oracle_quantize_row(const float* w, int N, int K, uint8_t* q, float* s) {
    for (int n = 0; n < N; ++n) {
        const float* src = w + (size_t)n * K;
        float mx = 0.0f;
        for (int k = 0; k < K; ++k) {
            const float a = fabsf(src[k]);
            if (a > mx) mx = a;
        }
        const float scale = mx > 0.0f ? mx / 448.0f : 1.0f;
        for (int k = 0; k < K; ++k) {
            float t = src[k] / scale;
            if (t > 448.0f) t = 448.0f;
            if (t < -448.0f) t = -448.0f;
            q[(size_t)n * K + k] = af_oracle_float_to_e4m3_rn(t);
        }
        s[n] = scale;
    }
}

/* -------------------------------------------------------------- GEMV --- */

void af_oracle_gemv_f64(const uint16_t* x, const void* w, const void* s, int kind, int M, int N,
                        int K, double* y) {
    af_oracle_gemv_f64_l2(x, w, s, kind, M, N, K, y, NULL);
}

void af_oracle_gemv_f64_l2(const uint16_t* x, const void* w, const void* s, int kind, int M, int N,
                           int K, double* y, double* l2) {
    const uint8_t* w8 = (const uint8_t*)w;
    const uint16_t* w16 = (const uint16_t*)w;
    const uint16_t* sg = (const uint16_t*)s;
    const float* sr = (const float*)s;
    const int G = K / 128;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        for (int m = 0; m < M; ++m) {
            double acc = 0.0, sq = 0.0;
            for (int k = 0; k < K; ++k) {
                double wv;
                if (kind == 3)
                    wv = af_oracle_half_to_float(w16[(size_t)n * K + k]);
                else
                    wv = af_oracle_e4m3_to_float(w8[(size_t)n * K + k]);
                if (kind == 0) wv *= af_oracle_half_to_float(sg[(size_t)n * G + k / 128]);
                const double t = wv * (double)af_oracle_half_to_float(x[(size_t)m * K + k]);
                acc += t;
                sq += t * t;
            }
            if (kind == 1) {
                acc *= (double)sr[n];
                sq *= (double)sr[n] * (double)sr[n];
            }
            y[(size_t)m * N + n] = acc;
            if (l2) l2[(size_t)m * N + n] = sqrt(sq);
        }
    }
}

/* qkv_gemm.cu:32-111 with BLOCK_DIM = 256, VEC = 4. */
static uint16_t refmath_row(const uint16_t* x, const uint8_t* wrow, const uint16_t* srow, int K) {
    enum { BLOCK = 256, VEC = 4, WARPS = BLOCK / 32 };
    float lane_sum[BLOCK];
    for (int tid = 0; tid < BLOCK; ++tid) {
        float sum = 0.0f;
        for (int kv = tid * VEC; kv < K; kv += BLOCK * VEC) {         /* :58 */
            const float sc = af_oracle_half_to_float(srow[kv / 128]); /* :70 */
            for (int v = 0; v < VEC; ++v) {
                const float wv = af_oracle_e4m3_to_float(wrow[kv + v]);
                const float xv = af_oracle_half_to_float(x[kv + v]);
                /* :82 sum += (w_val * s) * x_val -> FMUL then FFMA */
                sum = fmaf(wv * sc, xv, sum);
            }
        }
        lane_sum[tid] = sum;
    }
    float warp_sum[WARPS];
    for (int wp = 0; wp < WARPS; ++wp) {
        float l[32], nx[32];
        memcpy(l, lane_sum + wp * 32, sizeof(l));
        for (int off = 16; off > 0; off >>= 1) { /* :88-89 __shfl_down_sync */
            for (int i = 0; i < 32; ++i) nx[i] = l[i] + (i + off < 32 ? l[i + off] : l[i]);
            memcpy(l, nx, sizeof(l));
        }
        warp_sum[wp] = l[0];
    }
    float total = 0.0f; /* :104-108 serial sum of the warp sums */
    for (int wp = 0; wp < WARPS; ++wp) total = total + warp_sum[wp];
    return af_oracle_float_to_half_rn(total); /* :109 __float2half */
}

void af_oracle_gemv_refmath(const uint16_t* x, const uint8_t* w, const uint16_t* s, int N, int K,
                            uint16_t* y, int nthreads) {
    const int G = K / 128;
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (int n = 0; n < N; ++n)
        y[n] = refmath_row(x, w + (size_t)n * K, s + (size_t)n * G, K);
}

/* The same arithmetic as af_oracle_gemv_refmath (bit-identical output) with
 * table decode, x converted once, and the 256 kernel "threads" of a row laid
 * side by side so the compiler can vectorise across them: the timed CPU
 * baseline of the benchmark. */
void af_oracle_gemv_cpu_baseline(const uint16_t* x, const uint8_t* w, const uint16_t* s, int N,
                                 int K, uint16_t* y, int nthreads) {
    enum { BLOCK = 256, VEC = 4, WARPS = BLOCK / 32 };
    static float lut8[256];
    static int lut_ready = 0;
    if (!lut_ready) {
        for (int i = 0; i < 256; ++i) lut8[i] = af_oracle_e4m3_to_float((uint8_t)i);
        lut_ready = 1;
    }
    float* xf = (float*)malloc(sizeof(float) * (size_t)K);
    for (int k = 0; k < K; ++k) xf[k] = af_oracle_half_to_float(x[k]);
    const int G = K / 128;
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (int n = 0; n < N; ++n) {
        const uint8_t* wr = w + (size_t)n * K;
        const uint16_t* sr = s + (size_t)n * G;
        float sg[512];
        float lane[BLOCK];
        for (int g = 0; g < G && g < 512; ++g) sg[g] = af_oracle_half_to_float(sr[g]);
        for (int t = 0; t < BLOCK; ++t) lane[t] = 0.0f;
        for (int base = 0; base < K; base += BLOCK * VEC) {
            const int lim = (K - base) / VEC < BLOCK ? (K - base) / VEC : BLOCK;
            for (int t = 0; t < lim; ++t) {
                const int kv = base + t * VEC;
                const float sc = G <= 512 ? sg[kv / 128] : af_oracle_half_to_float(sr[kv / 128]);
                float a = lane[t];
                a = fmaf(lut8[wr[kv + 0]] * sc, xf[kv + 0], a);
                a = fmaf(lut8[wr[kv + 1]] * sc, xf[kv + 1], a);
                a = fmaf(lut8[wr[kv + 2]] * sc, xf[kv + 2], a);
                a = fmaf(lut8[wr[kv + 3]] * sc, xf[kv + 3], a);
                lane[t] = a;
            }
        }
        float total = 0.0f;
        for (int wp = 0; wp < WARPS; ++wp) {
            float l[32], nx[32];
            memcpy(l, lane + wp * 32, sizeof(l));
            for (int off = 16; off > 0; off >>= 1) {
                for (int i = 0; i < 32; ++i) nx[i] = l[i] + (i + off < 32 ? l[i + off] : l[i]);
                memcpy(l, nx, sizeof(l));
            }
            total = total + l[0];
        }
        y[n] = af_oracle_float_to_half_rn(total);
    }
    free(xf);
}

/* ------------------------------------------------------------ argmax --- */

int af_oracle_argmax(const float* v, int n, int mode) {
    if (mode == 1 && n > 65536) n = 65536;
    int bi = -1;
    float bv = 0.0f;
    for (int i = 0; i < n; ++i) {
        if (isnan(v[i])) continue;
        if (bi < 0 || v[i] > bv) {
            bv = v[i];
            bi = i;
        }
    }
    return bi;
}
