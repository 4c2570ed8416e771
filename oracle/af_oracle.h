/*
 * af_oracle.h -- CPU restatement of AtomFlow's W8A16 decode-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This code is the parity checker for the CUDA
 * library in atomflow_b200/ and the timed CPU baseline of bench.py.  Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs
 * may load it; the product path never does.
 *
 * Pinning: the bit-exact restatement af_oracle_gemv_refmath() is checked
 * against golden vectors that the reference's own w8a16_gemv_kernel produced
 * on a B200 (tests/golden/, generator script beside them), and the quantiser
 * against vectors made by the reference's own tools/quantize_weights.py.
 */
#ifndef AF_ORACLE_H
#define AF_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Number formats (OCP FP8 E4M3 "fn" variant: bias 7, no inf, 0x7F/0xFF NaN, max 448;
 * IEEE binary16). */
float af_oracle_e4m3_to_float(uint8_t b);
uint8_t af_oracle_float_to_e4m3_rn(float f);
float af_oracle_half_to_float(uint16_t h);
uint16_t af_oracle_float_to_half_rn(float f);

/* tools/quantize_weights.py:220-268 quantize_fp8_gs128: per 128-wide group,
 * scale = absmax/448 (1 for an all-zero group) in FP32, q = e4m3(clamp(w/scale,
 * +-448)), stored scale = half(scale).  w FP32 [N,K]; q [N,K]; s FP16 bits [N,K/128]. */
void af_oracle_quantize_gs128(const float* w, int N, int K, uint8_t* q, uint16_t* s);
/* The per-output-row variant of the benchmark configs: scale = rowabsmax/448 (FP32). */
void af_oracle_quantize_row(const float* w, int N, int K, uint8_t* q, float* s);

/* y[m,n] = sum_k W[n,k]*scale*x[m,k] in FP64.
 * kind 0: FP8 W, FP16 group scales [N,K/128]; 1: FP8 W, FP32 row scales [N];
 * kind 2: FP8 W, no scale; 3: FP16 W (bits), no scale. */
void af_oracle_gemv_f64(const uint16_t* x, const void* w, const void* s, int kind, int M, int N,
                        int K, double* y);
/* As af_oracle_gemv_f64, also returning l2[m,n] = sqrt(sum_k (W[n,k]*scale*x[m,k])^2),
 * the natural scale of the FP32 rounding noise of any FP32-accumulated result. */
void af_oracle_gemv_f64_l2(const uint16_t* x, const void* w, const void* s, int kind, int M, int N,
                           int K, double* y, double* l2);

/* Bit-exact restatement of src/kernel/qkv_gemm.cu:32-111 (w8a16_gemv_kernel<256>)
 * for one token: FP32 fused multiply-add per element in the kernel's thread /
 * stride order, the __shfl_down tree, the serial sum of 8 warp sums, FP16 RN.
 * Rows are independent, so `nthreads` OpenMP threads split them. */
void af_oracle_gemv_refmath(const uint16_t* x, const uint8_t* w, const uint16_t* s, int N, int K,
                            uint16_t* y, int nthreads);

/* Identical output to af_oracle_gemv_refmath; table decode and a loop order
 * the compiler vectorises.  The benchmark's timed CPU baseline. */
void af_oracle_gemv_cpu_baseline(const uint16_t* x, const uint8_t* w, const uint16_t* s, int N,
                                 int K, uint16_t* y, int nthreads);

/* argmax of FP32 values: mode 0 true argmax (ties -> lowest index, NaN never
 * wins); mode 1 the reference's (src/kernel/argmax.cu: only ids < 65536). */
int af_oracle_argmax(const float* v, int n, int mode);

#ifdef __cplusplus
}
#endif
#endif
