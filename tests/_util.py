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


FP32_NOISE_ULPS = 4.0


def assert_fp16_parity(y_bits, ref, what="", ref_kernel_bits=None, noise_ulps=None):
    """BASELINE tolerance, per output: |y - r| <= 2 FP16 ulp where r is the
    reference kernel's own output (ulp at r's binade), OR relative error
    <= 2e-3 against FP64 -- whichever is looser.

    `ref` is the FP64 oracle's (y, l2) pair (oracle.gemv_f64(..., with_l2=True))
    or a plain FP64 array.  `ref_kernel_bits` is the reference
    w8a16_gemv_kernel's output (its bit-exact restatement oracle.gemv_refmath,
    pinned to the kernel by golden vectors); where the reference kernel has no
    such path (row scales, no scales) only the FP64 leg applies.

    One more leg covers outputs that cancel to almost nothing: |y - FP64| <=
    4 * 2^-24 * l2, l2 = ||(w*s*x)_k||_2, i.e. four FP32 rounding steps at the
    natural scale of the output's terms.  Any FP32-accumulated dot product --
    the reference kernel's included, see
    tests/test_oracle.py::test_reference_kernel_needs_the_fp32_noise_floor --
    differs from FP64 by about that much, which exceeds 2 FP16 ulp once |y| is
    below ~1e-4 * l2.  Returns the largest error in FP16 ulps vs FP64."""
    if isinstance(ref, tuple):
        ref_f64, l2 = ref
    else:
        ref_f64, l2 = ref, None
    y = np.asarray(y_bits, np.uint16).view(np.float16).astype(np.float64).reshape(ref_f64.shape)
    ref16 = fp16_bits(ref_f64.astype(np.float32))
    ulp = oracle.half_ulp(ref16)
    err = np.abs(y - ref_f64)
    ok = (err <= 2.0 * ulp) | (err <= 2e-3 * np.abs(ref_f64))
    if ref_kernel_bits is not None:
        rk = np.asarray(ref_kernel_bits, np.uint16).reshape(ref_f64.shape)
        rv = rk.view(np.float16).astype(np.float64)
        ok |= np.abs(y - rv) <= 2.0 * oracle.half_ulp(rk)
    if l2 is not None:
        ok |= err <= (noise_ulps or FP32_NOISE_ULPS) * 2.0 ** -24 * l2.reshape(ref_f64.shape)
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
