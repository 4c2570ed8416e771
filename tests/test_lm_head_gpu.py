"""GPU parity of the lm_head projection (FP16 and FP8-row variants) with the
fused argmax, and of the standalone argmax, through the C ABI."""
import numpy as np
import pytest

import oracle
from tests._util import assert_fp32_close, fp16_bits, normal_f32

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def lib():
    from atomflow_b200 import lib as _l
    return _l()


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).cuda()


def lm_head(x, w, wdt, rs=None, mode=0, want_logits=True):
    L = lib()
    V, D = w.shape
    ws = torch.zeros(L.af_lm_head_workspace_bytes(V, D, wdt), dtype=torch.uint8, device="cuda")
    logits = torch.zeros(V, dtype=torch.float32, device="cuda") if want_logits else None
    idx = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    xd, wd = dev(x), dev(w)
    rsd = dev(rs) if rs is not None else None
    rc = L.af_lm_head_gemv(xd.data_ptr(), wd.data_ptr(), wdt, rsd.data_ptr() if rsd is not None else None,
                           logits.data_ptr() if logits is not None else None, V, D, idx.data_ptr(), mode,
                           ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, L.af_status_string(rc)
    return (logits.cpu().numpy() if logits is not None else None), int(idx.item())


def f16_case(seed, V, D):
    w = fp16_bits(normal_f32(seed, (V, D), 0.02))
    x = fp16_bits(normal_f32(seed + 1, (1, D)))
    return x, w


@pytest.mark.parametrize("V,D", [(128256, 3072), (1000, 3072), (77, 64), (5, 32)])
def test_lm_head_f16(V, D):
    x, w = f16_case(V + D, V, D)
    logits, idx = lm_head(x, w, 0)
    ref = oracle.gemv_f64(x, w, None, "f16")[0]
    assert_fp32_close(logits, ref, f"lm_head f16 {V}x{D}")
    assert idx == oracle.argmax(logits)
    assert idx == int(np.argmax(ref))


@pytest.mark.parametrize("V,D", [(128256, 3072), (999, 640)])
def test_lm_head_fp8_row(V, D):
    wf = normal_f32(V, (V, D), 0.02)
    q, rs = oracle.quantize_row(wf)
    x = fp16_bits(normal_f32(V + 1, (1, D)))
    logits, idx = lm_head(x, q, 1, rs)
    ref = oracle.gemv_f64(x, q, rs, "row")[0]
    assert_fp32_close(logits, ref, f"lm_head fp8 {V}x{D}")
    assert idx == oracle.argmax(logits)


def test_lm_head_argmax_only_and_ref_compat_mode():
    V, D = 128256, 3072
    x, w = f16_case(42, V, D)
    # plant the winner above 65535 and a runner-up below it
    wv = w.view(np.float16).copy()
    wv[100000] = (np.abs(wv[100000]) * np.sign(x.view(np.float16)[0])).astype(np.float16) * 4
    wv[1234] = (np.abs(wv[1234]) * np.sign(x.view(np.float16)[0])).astype(np.float16) * 3
    w = wv.view(np.uint16)
    _, i_true = lm_head(x, w, 0, want_logits=False)
    logits, i_compat = lm_head(x, w, 0, mode=1)
    assert i_true == 100000
    assert i_compat == oracle.argmax(logits, 1) == 1234


def test_lm_head_matches_reference_cublas_and_argmax():
    R = oracle.ref()
    if R is None:
        pytest.skip("oracle/_ref/libafref.so not built")
    V, D = 128256, 3072
    x, w = f16_case(5, V, D)
    xd, wd = dev(x), dev(w)
    lr = torch.zeros(V, dtype=torch.float32, device="cuda")
    ir = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert R.afref_lm_head(wd.data_ptr(), xd.data_ptr(), lr.data_ptr(), V, D, st) == 0
    assert R.afref_argmax(lr.data_ptr(), V, ir.data_ptr(), st) == 0
    torch.cuda.synchronize()
    lref = lr.cpu().numpy()
    logits, _ = lm_head(x, w, 0)
    _, icompat = lm_head(x, w, 0, mode=1)
    assert_fp32_close(logits, lref.astype(np.float64), "vs reference cuBLAS", rel=2e-4)
    assert int(ir.item()) == icompat == oracle.argmax(lref, 1)


@pytest.mark.parametrize("V", [1, 31, 4096, 65536, 65537, 128256, 1 << 20])
def test_argmax_standalone(V):
    L = lib()
    v = normal_f32(V, V)
    v[V // 3] = 9.0
    v[(2 * V) // 3] = 9.0          # tie -> lower index
    if V > 10:
        v[7] = np.nan
    vd = torch.from_numpy(v).cuda()
    for mode in (0, 1):
        ws = torch.zeros(L.af_argmax_workspace_bytes(V), dtype=torch.uint8, device="cuda")
        out = torch.full((1,), -5, dtype=torch.int32, device="cuda")
        for _ in range(2):   # second call checks the self-reset counter
            assert L.af_argmax_f32(vd.data_ptr(), V, out.data_ptr(), mode, ws.data_ptr(), ws.numel(),
                                   torch.cuda.current_stream().cuda_stream) == 0
            torch.cuda.synchronize()
            assert int(out.item()) == oracle.argmax(v, mode)


def test_lm_head_needs_its_argmax_workspace():
    L = lib()
    V, D = 4096, 3072
    x, w = f16_case(3, V, D)
    xd, wd = dev(x), dev(w)
    logits = torch.zeros(V, dtype=torch.float32, device="cuda")
    idx = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.af_lm_head_workspace_bytes(V, D, 0) > 0
    rc = L.af_lm_head_gemv(xd.data_ptr(), wd.data_ptr(), 0, None, logits.data_ptr(), V, D, idx.data_ptr(), 0,
                           None, 0, st)
    assert rc == 5   # AF_ERR_WORKSPACE
