"""The batched W8A16 projection on the tcgen05 tensor cores (af_gemv_tc.cu),
called through its C ABI entry point af_w8a16_gemm_tc.

The reference kernel is one token per launch (src/kernel/qkv_gemm.cu:32-150),
so every token row is also checked against its bit-exact restatement: each
output meets the tolerance of the one-token path (2 FP16 ulp of the reference
kernel's own value, or 2e-3 relative against FP64).  The noise-floor leg for
outputs that cancel to almost nothing is 8 (not 4) FP32 rounding steps at the
scale of the output's terms: the tensor core's FP32 accumulation of each K=16
product block does not round to nearest, which costs about one more step
(worst case seen: 4.3 steps, one output in 1M at M = 128).
"""
import numpy as np
import pytest

import oracle
from tests._util import assert_fp16_parity as _parity, make_gemv_case
from tests.test_gemv_gpu import dev, gemv_np, lib

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def assert_fp16_parity(*a, **k):
    return _parity(*a, noise_ulps=8, **k)


KIND = {"group": 0, "row": 1}


def run_tc(x, q, s, kind="group", out=None, xd=None, qd=None, sd=None, stream=None):
    M, K = x.shape
    N = q.shape[0]
    xd = dev(x) if xd is None else xd
    qd = dev(q) if qd is None else qd
    sd = dev(s) if sd is None else sd
    y = out if out is not None else torch.zeros(M, N, dtype=torch.int16, device="cuda")
    st = (stream or torch.cuda.current_stream()).cuda_stream
    rc = lib().af_w8a16_gemm_tc(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), y.data_ptr(), M, N, K, 128, KIND[kind],
                                st)
    return rc, y


def tc_np(x, q, s, kind="group"):
    rc, y = run_tc(x, q, s, kind)
    torch.cuda.synchronize()
    assert rc == 0, lib().af_status_string(rc)
    return y.cpu().numpy().view(np.uint16)


def _faults():
    import ctypes
    v = ctypes.c_uint(0)
    assert lib().af_device_faults(ctypes.byref(v), 1) == 0
    return v.value


@pytest.mark.parametrize("M", [1, 8, 16, 33, 128])
@pytest.mark.parametrize("N,K", [(8192, 3072), (3072, 8192)])
def test_tc_config_shapes(M, N, K):
    x, q, s = make_gemv_case(4000 + M + N % 7, M, N, K)
    y = tc_np(x, q, s)
    ref = oracle.gemv_f64(x, q, s, "group", with_l2=True)
    rows = sorted({0, M // 2, M - 1})   # the reference kernel's restatement on a few token rows
    rk = np.stack([oracle.gemv_refmath(x[m], q, s, 8) for m in rows])
    assert_fp16_parity(y[rows], (ref[0][rows], ref[1][rows]), f"M={M} {N}x{K} (ref rows)", rk)
    assert_fp16_parity(y, ref, f"M={M} {N}x{K}")
    assert _faults() == 0


@pytest.mark.parametrize("M,N,K", [(8, 100, 640), (9, 129, 1152), (24, 1000, 256), (16, 5120, 3072),
                                   (40, 4099, 512), (8, 300, 14336), (17, 6144, 4096), (12, 1, 128)])
def test_tc_ragged_shapes(M, N, K):
    """Row tiles past N, token slices past M, K of one group, K split over 8 CTAs."""
    x, q, s = make_gemv_case(77 + M + N + K, M, N, K)
    assert_fp16_parity(tc_np(x, q, s), oracle.gemv_f64(x, q, s, "group", with_l2=True), f"M={M} {N}x{K}")


@pytest.mark.parametrize("M,N,K", [(8, 3072, 8192), (16, 8192, 3072), (33, 777, 384)])
def test_tc_row_scales(M, N, K):
    x, q, s = make_gemv_case(31 + M + N, M, N, K, kind="row")
    assert_fp16_parity(tc_np(x, q, s, "row"), oracle.gemv_f64(x, q, s, "row", with_l2=True), f"row M={M} {N}x{K}")


def test_tc_deterministic_no_overwrite_and_graph():
    """Repeats are bit-identical (the cluster merges its partials in rank order),
    nothing past y is written, and a captured launch replays to the same bits."""
    M, N, K = 16, 3072, 8192
    x, q, s = make_gemv_case(5, M, N, K)
    xd, qd, sd = dev(x), dev(q), dev(s)
    L = lib()
    canary = torch.full((M * N + 64,), 0x5A5A, dtype=torch.int16, device="cuda")
    outs = []
    for _ in range(3):
        rc, _ = run_tc(x, q, s, out=canary, xd=xd, qd=qd, sd=sd)
        assert rc == 0
        torch.cuda.synchronize()
        c = canary.cpu().numpy().view(np.uint16)
        assert (c[M * N:] == 0x5A5A).all()
        outs.append(c[:M * N].copy())
    np.testing.assert_array_equal(outs[0], outs[1])
    np.testing.assert_array_equal(outs[0], outs[2])
    y = torch.zeros(M, N, dtype=torch.int16, device="cuda")
    st = torch.cuda.Stream()

    def call():
        return L.af_w8a16_gemm_tc(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), y.data_ptr(), M, N, K, 128, 0,
                                  st.cuda_stream)

    assert call() == 0   # first call outside capture
    st.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        assert call() == 0
    for _ in range(2):
        y.zero_()
        g.replay()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy().view(np.uint16).reshape(-1), outs[0])
    assert _faults() == 0


def test_tc_matches_one_token_path():
    """Each token of a batch agrees with the same token through the one-token kernel."""
    M, N, K = 8, 5120, 3072
    x, q, s = make_gemv_case(12, M, N, K)
    yb = tc_np(x, q, s).view(np.float16).astype(np.float64)
    ref = oracle.gemv_f64(x, q, s, "group", with_l2=True)
    for m in range(M):
        y1 = gemv_np(x[m:m + 1], q, s).view(np.float16).astype(np.float64)[0]
        # both within the tolerance of FP64, so within twice of it of each other
        scale = np.abs(ref[0][m]) + np.sqrt(np.mean(ref[0][m] ** 2))
        assert np.abs(yb[m] - y1).max() <= 4e-3 * scale.max()


def test_tc_argument_errors():
    x, q, s = make_gemv_case(9, 8, 32, 256)
    xd, qd, sd = dev(x), dev(q), dev(s)
    y = torch.zeros(8, 32, dtype=torch.int16, device="cuda")
    L = lib()
    st = torch.cuda.current_stream().cuda_stream
    assert L.af_w8a16_gemm_tc(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), y.data_ptr(), 8, 32, 256, 64, 0, st) == 1
    assert L.af_w8a16_gemm_tc(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), y.data_ptr(), 8, 32, 200, 128, 0, st) == 1
    assert L.af_w8a16_gemm_tc(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), y.data_ptr(), 8, 32, 256, 128, 2, st) == 1
    assert L.af_w8a16_gemm_tc(xd.data_ptr() + 2, qd.data_ptr(), sd.data_ptr(), y.data_ptr(), 8, 32, 256, 128, 0,
                              st) == 1
    assert L.af_w8a16_gemm_tc(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), y.data_ptr(), 0, 32, 256, 128, 0, st) == 0
