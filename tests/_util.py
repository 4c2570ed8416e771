"""Seeded inputs and the parity criterion shared by the tests."""
import numpy as np

import oracle


def normal_f32(seed, shape, std=1.0):
    return (np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(std))


def fp16_bits(a):
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def make_gemv_case(seed, M, N, K, kind="group", x_std=1.0, w_std=0.02):
    """BASELINE config-0 recipe: W ~ N(0, 0.02) FP32 quantised to E4M3 (group or row
    scales), x ~ N(0, 1) FP16.  Returns numpy arrays (x as fp16 bits)."""
    w = normal_f32(seed, (N, K), w_std)
    if kind == "group":
        q, s = oracle.quantize_gs128(w)
    elif kind == "row":
        q, s = oracle.quantize_row(w)
    else:
        q, _ = oracle.quantize_row(w)
        s = None
    x = fp16_bits(normal_f32(seed + 1_000_003, (M, K), x_std))
    return x, q, s


def assert_fp16_parity(y_bits, ref_f64, what="", ref_kernel_bits=None):
    """BASELINE tolerance, per output: |y - r| <= 2 FP16 ulp where r is the
    reference kernel's own output (ulp at r's binade), OR relative error
    <= 2e-3 against FP64 -- whichever is looser.  `ref_kernel_bits` is the
    reference w8a16_gemv_kernel's output (its bit-exact restatement,
    oracle.gemv_refmath, pinned to the kernel by golden vectors); where the
    reference kernel has no such path (row scales, M > 1) the FP64 value
    stands in for r.  Returns the largest error in FP16 ulps vs FP64."""
    y = np.asarray(y_bits, np.uint16).view(np.float16).astype(np.float64).reshape(ref_f64.shape)
    ref16 = fp16_bits(ref_f64.astype(np.float32))
    ulp = oracle.half_ulp(ref16)
    err = np.abs(y - ref_f64)
    ok = (err <= 2.0 * ulp) | (err <= 2e-3 * np.abs(ref_f64))
    if ref_kernel_bits is not None:
        rk = np.asarray(ref_kernel_bits, np.uint16).reshape(ref_f64.shape)
        rv = rk.view(np.float16).astype(np.float64)
        ok |= np.abs(y - rv) <= 2.0 * oracle.half_ulp(rk)
    if not ok.all():
        i = np.flatnonzero(~ok)[:5]
        raise AssertionError(f"{what}: {int((~ok).sum())} of {ok.size} outputs out of tolerance; "
                             f"first at {i.tolist()}: got {y.ravel()[i]}, ref {ref_f64.ravel()[i]}")
    return float((err / ulp).max())


def assert_fp32_close(y, ref_f64, what="", rel=1e-4):
    """FP32 outputs (logits): |y - ref| <= rel * (|ref| + rms(ref))."""
    y = np.asarray(y, np.float64)
    tol = rel * (np.abs(ref_f64) + np.sqrt(np.mean(ref_f64 ** 2)))
    err = np.abs(y - ref_f64)
    if not (err <= tol).all():
        i = np.flatnonzero(err > tol)[:5]
        raise AssertionError(f"{what}: {int((err > tol).sum())} logits out of tolerance; first {i.tolist()}")
