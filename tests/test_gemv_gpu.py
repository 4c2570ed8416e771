"""GPU parity of the W8A16 GEMV, called through the C ABI (af_w8a16_gemv),
against the FP64 oracle, the bit-exact restatement and the reference's own
kernel (oracle/_ref)."""
import ctypes

import numpy as np
import pytest

import oracle
from tests._util import assert_fp16_parity, fp16_bits, make_gemv_case

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


class Ws:
    def __init__(self, nbytes):
        self.t = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device="cuda")


KIND = {"group": 0, "row": 1, "none": 2}


def run_gemv(x, q, s, kind="group", ws=None, out=None, stream=None, M=None, N=None, K=None,
             group_size=128, xd=None, qd=None):
    L = lib()
    M = M if M is not None else x.shape[0]
    N = N if N is not None else q.shape[0]
    K = K if K is not None else q.shape[1]
    xd = dev(x) if xd is None else xd
    qd = dev(q) if qd is None else qd
    sd = dev(s) if s is not None else None
    need = L.af_w8a16_gemv_workspace_bytes(M, N, K, KIND[kind])
    ws = ws or Ws(need)
    y = out if out is not None else torch.zeros(M, N, dtype=torch.int16, device="cuda")
    st = (stream or torch.cuda.current_stream()).cuda_stream
    rc = L.af_w8a16_gemv(xd.data_ptr(), qd.data_ptr(), sd.data_ptr() if sd is not None else None,
                         y.data_ptr(), M, N, K, group_size, KIND[kind], ws.t.data_ptr(),
                         ws.t.numel(), st)
    return rc, y


def gemv_np(x, q, s, kind="group"):
    rc, y = run_gemv(x, q, s, kind)
    torch.cuda.synchronize()
    assert rc == 0, lib().af_status_string(rc)
    return y.cpu().numpy().view(np.uint16)


# BASELINE shapes: config 0, the five config-1 projections, the 8B TP shapes (config 4)
SHAPES = [(3072, 3072), (5120, 3072), (8192, 3072), (3072, 8192),
          (6144, 4096), (14336, 4096), (4096, 14336)]


@pytest.mark.parametrize("N,K", SHAPES)
def test_gemv_m1_group_full_shapes(N, K):
    x, q, s = make_gemv_case(100 + N % 97 + K % 89, 1, N, K)
    y = gemv_np(x, q, s)
    assert_fp16_parity(y, oracle.gemv_f64(x, q, s, "group", with_l2=True), f"{N}x{K}", oracle.gemv_refmath(x, q, s, 8))


@pytest.mark.parametrize("N,K", [(1, 128), (3, 128), (17, 256), (31, 384), (1000, 640),
                                 (129, 1152), (4099, 512), (2, 8192), (300, 14336)])
def test_gemv_ragged_shapes(N, K):
    x, q, s = make_gemv_case(7 + N + K, 1, N, K)
    assert_fp16_parity(gemv_np(x, q, s), oracle.gemv_f64(x, q, s, "group", with_l2=True), f"{N}x{K}",
                       oracle.gemv_refmath(x, q, s, 8))


@pytest.mark.parametrize("M", [1, 2, 3, 4, 7, 8, 9, 12, 16, 17, 33])
@pytest.mark.parametrize("N,K", [(8192, 3072), (3072, 8192), (100, 640)])
def test_gemv_batched_tokens(M, N, K):
    x, q, s = make_gemv_case(900 + M, M, N, K)
    # the reference kernel is M = 1 only: each token row through its restatement
    rk = np.stack([oracle.gemv_refmath(x[m], q, s, 8) for m in range(M)])
    assert_fp16_parity(gemv_np(x, q, s), oracle.gemv_f64(x, q, s, "group", with_l2=True), f"M={M} {N}x{K}", rk)


@pytest.mark.parametrize("kind", ["row", "none"])
@pytest.mark.parametrize("M,N,K", [(1, 3072, 3072), (1, 8192, 3072), (5, 777, 192), (16, 512, 4096),
                                   (4, 1000, 1024), (8, 3072, 8192)])
def test_gemv_row_scale_and_unscaled(kind, M, N, K):
    x, q, s = make_gemv_case(31 + M + N, M, N, K, kind=kind)
    y = gemv_np(x, q, s, kind)
    assert_fp16_parity(y, oracle.gemv_f64(x, q, s, kind, with_l2=True), f"{kind} M={M} {N}x{K}")


@pytest.mark.parametrize("x_std", [1e-3, 40.0, 250.0])
def test_gemv_heavy_tailed_and_small_activations(x_std):
    x, q, s = make_gemv_case(55, 1, 3072, 3072, x_std=x_std)
    x = x.copy()
    x[0, ::97] = fp16_bits(np.float32(287.8))      # outliers like gt_layer27_mlp_out
    x[0, 5::211] = 0
    assert_fp16_parity(gemv_np(x, q, s), oracle.gemv_f64(x, q, s, "group", with_l2=True), f"x_std={x_std}",
                       oracle.gemv_refmath(x, q, s, 8))


def test_gemv_matches_reference_kernel_and_pins_refmath():
    R = oracle.ref()
    if R is None:
        pytest.skip("oracle/_ref/libafref.so not built")
    for (N, K) in [(3072, 3072), (5120, 3072), (8192, 3072), (3072, 8192), (77, 640)]:
        x, q, s = make_gemv_case(N + K, 1, N, K)
        xd, qd, sd = dev(x), dev(q), dev(s)
        yr = torch.zeros(N, dtype=torch.int16, device="cuda")
        assert R.afref_w8a16_gemv(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), yr.data_ptr(), N, K,
                                  torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        yref = yr.cpu().numpy().view(np.uint16)
        # the oracle restates the reference kernel bit for bit
        np.testing.assert_array_equal(oracle.gemv_refmath(x, q, s), yref)
        # and ours is within 2 FP16 ulp of the reference kernel's output as well as of FP64
        y = gemv_np(x, q, s)
        ref64 = oracle.gemv_f64(x, q, s, "group", with_l2=True)
        assert_fp16_parity(y, ref64, "vs reference kernel / f64", yref)
        yv = y.view(np.float16).astype(np.float64)
        rv = yref.view(np.float16).astype(np.float64)
        assert (np.abs(yv - rv) <= 2 * oracle.half_ulp(yref) + 2 * oracle.half_ulp(y)).all()


def test_gemv_deterministic_and_no_overwrite():
    """Bit-identical repeats (fixed-order split-K reduction) and canary-padded output."""
    N, K = 5120, 3072
    x, q, s = make_gemv_case(3, 1, N, K)
    L = lib()
    ws = Ws(L.af_w8a16_gemv_workspace_bytes(1, N, K, 0))
    canary = torch.full((N + 64,), 0x5A5A, dtype=torch.int16, device="cuda")
    outs = []
    for _ in range(3):
        rc, _ = run_gemv(x, q, s, ws=ws, out=canary)
        assert rc == 0
        torch.cuda.synchronize()
        c = canary.cpu().numpy().view(np.uint16)
        assert (c[N:] == 0x5A5A).all()
        outs.append(c[:N].copy())
    np.testing.assert_array_equal(outs[0], outs[1])
    np.testing.assert_array_equal(outs[0], outs[2])
    # the workspace counters are back to zero after every call
    assert int(ws.t.abs().sum()) == 0


def test_gemv_linearity_full_size():
    """Size-independent property at the largest BASELINE shape: W(x1+x2) = Wx1 + Wx2."""
    N, K = 14336, 4096
    x, q, s = make_gemv_case(4, 2, N, K, x_std=0.5)
    x3 = fp16_bits(x.view(np.float16).astype(np.float32).sum(0, keepdims=True))
    xa = np.concatenate([x, x3])
    y = gemv_np(xa, q, s).view(np.float16).astype(np.float64)
    ref = oracle.gemv_f64(xa, q, s, "group", with_l2=True)
    rk = np.stack([oracle.gemv_refmath(xa[m], q, s, 8) for m in range(3)])
    assert_fp16_parity(y.astype(np.float16).view(np.uint16), ref, "linearity", rk)
    lhs, rhs = y[2], y[0] + y[1]
    scale = np.sqrt(np.mean(ref[0][2] ** 2))
    assert np.abs(lhs - rhs).max() <= 0.01 * scale


def test_gemv_fallback_paths_unaligned():
    """Unaligned x / W pointers take the scalar kernel and still match."""
    N, K = 40, 256
    x, q, s = make_gemv_case(8, 1, N, K)
    xbuf = torch.zeros(K + 8, dtype=torch.int16, device="cuda")
    xbuf[1:K + 1] = dev(x)[0]
    qbuf = torch.zeros(N * K + 16, dtype=torch.uint8, device="cuda")
    qbuf[3:3 + N * K] = dev(q).view(-1)
    rc, y = run_gemv(x, q, s, xd=xbuf[1:], qd=qbuf[3:])
    torch.cuda.synchronize()
    assert rc == 0
    assert_fp16_parity(y.cpu().numpy().view(np.uint16), oracle.gemv_f64(x, q, s, "group", with_l2=True), "unaligned",
                       oracle.gemv_refmath(x, q, s))


def test_gemv_argument_errors():
    x, q, s = make_gemv_case(9, 1, 32, 256)
    assert run_gemv(x, q, s, group_size=64)[0] == 1                      # INVALID
    assert run_gemv(x, q, s, ws=Ws(0))[0] == 0                           # the GEMV needs no scratch

    assert run_gemv(x, q, s, M=0)[0] == 0 and run_gemv(x, q, s, N=0)[0] == 0
    assert run_gemv(x[:, :200], q[:, :200], s, K=200)[0] == 1            # K % 128 with groups


def test_gemv_graph_replay_and_pdl_chain():
    """A CUDA graph of 140 dependent launches (one config-1 layer set x 28
    scaled down to 4 layers here) replays to the same bits as eager calls."""
    shapes = [(5120, 3072), (3072, 3072), (8192, 3072), (8192, 3072), (3072, 8192)] * 4
    cases = [make_gemv_case(500 + i, 1, N, K) for i, (N, K) in enumerate(shapes)]
    L = lib()
    ws = Ws(max(L.af_w8a16_gemv_workspace_bytes(1, N, K, 0) for N, K in shapes))
    dx = [dev(c[0]) for c in cases]
    dq = [dev(c[1]) for c in cases]
    ds = [dev(c[2]) for c in cases]
    outs = [torch.zeros(1, N, dtype=torch.int16, device="cuda") for N, _ in shapes]
    st = torch.cuda.Stream()

    def step():
        for i, (N, K) in enumerate(shapes):
            rc = L.af_w8a16_gemv(dx[i].data_ptr(), dq[i].data_ptr(), ds[i].data_ptr(), outs[i].data_ptr(),
                                 1, N, K, 128, 0, ws.t.data_ptr(), ws.t.numel(), st.cuda_stream)
            assert rc == 0

    with torch.cuda.stream(st):
        step()
    st.synchronize()
    eager = [o.cpu().numpy().copy() for o in outs]
    for o in outs:
        o.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        step()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        np.testing.assert_array_equal(o.cpu().numpy(), eager[i])
    y0 = eager[0].view(np.uint16)
    assert_fp16_parity(y0, oracle.gemv_f64(cases[0][0], cases[0][1], cases[0][2], "group", with_l2=True), "graph",
                       oracle.gemv_refmath(cases[0][0], cases[0][1], cases[0][2]))
