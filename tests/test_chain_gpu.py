"""The persistent projection chain (af_gemv_chain) against the reference's own
kernels, bit for bit.

  * one projection (af_w8a16_gemv, M = 1, group scales, which runs the chain
    kernel): every output bit-identical to the reference's w8a16_gemv_kernel
    (compiled from its sources into oracle/_ref) at the BASELINE shapes and at
    ragged ones (K not a multiple of 1024, N below the CTA count);
  * decode layers without attention -- RMSNorm+QKV, O+residual,
    RMSNorm+gate/up+SwiGLU, down+residual, with each op waiting for the one
    before -- as one launch: the residual stream, QKV and the SwiGLU output
    bit-identical to the reference's ten-kernel sequence of engine.cu:292-483
    (rms_norm, w8a16_gemv x5, residual_add x2, swiglu);
  * repeated launches and CUDA-graph replays reproduce the eager result (the
    completion counters return to zero after every launch);
  * invalid arguments launch nothing.
"""
import ctypes

import numpy as np
import pytest

import oracle
from tests._util import make_gemv_case

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

EPS = 1e-5
D, FFN, QKV = 3072, 8192, 5120


def L():
    from atomflow_b200 import lib
    return lib()


def R():
    r = oracle.ref()
    if r is None:
        pytest.skip("oracle/_ref/libafref.so not built")
    return r


def st():
    return torch.cuda.current_stream().cuda_stream


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).cuda()


@pytest.mark.parametrize("N,K", [(3072, 3072), (5120, 3072), (8192, 3072), (3072, 8192), (6144, 4096),
                                 (4096, 14336), (1, 128), (3, 128), (17, 256), (31, 384), (77, 640),
                                 (129, 1152), (1000, 1536), (4099, 512), (2, 8192), (300, 16384)])
def test_gemv_bit_identical_to_reference_kernel(N, K):
    x, q, s = make_gemv_case(N * 7 + K, 1, N, K)
    xd, qd, sd = dev(x), dev(q), dev(s)
    ours = torch.zeros(N, dtype=torch.int16, device="cuda")
    theirs = torch.zeros(N, dtype=torch.int16, device="cuda")
    from atomflow_b200._lib import ChainOp, OpKind
    op = ChainOp(kind=OpKind.GEMV, N=N, K=K, x=xd.data_ptr(), w=qd.data_ptr(), scales=sd.data_ptr(),
                 y=ours.data_ptr())
    assert L().af_gemv_chain(ctypes.byref(op), 1, None, 0, st()) == 0
    assert R().afref_w8a16_gemv(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), theirs.data_ptr(), N, K, st()) == 0
    torch.cuda.synchronize()
    a, b = ours.cpu().numpy(), theirs.cpu().numpy()
    bad = np.flatnonzero(a != b)
    assert bad.size == 0, f"{bad.size} of {N} outputs differ from the reference kernel, first at {bad[:5].tolist()}"
    if N * K <= 4_000_000:   # and the CPU restatement agrees
        np.testing.assert_array_equal(oracle.gemv_refmath(x, q, s, 8), a.view(np.uint16))


def _weights(g, N, K):
    from atomflow_b200.quant import quantize_gs128
    q, s = quantize_gs128(torch.randn(N, K, generator=g, device="cuda") * 0.02)
    return q.view(torch.uint8).contiguous(), s.contiguous()


def _layers(n, seed=5):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    out = []
    for _ in range(n):
        ly = {nm: _weights(g, N, K) for nm, N, K in (("qkv", QKV, D), ("o", D, D), ("gate", FFN, D),
                                                      ("up", FFN, D), ("down", D, FFN))}
        ly["g_attn"] = (1 + 0.1 * torch.randn(D, generator=g, device="cuda")).float()
        ly["g_mlp"] = (1 + 0.1 * torch.randn(D, generator=g, device="cuda")).float()
        out.append(ly)
    x0 = torch.randn(D, generator=g, device="cuda").half()
    return out, x0


def _chain_ops(layers, b):
    from atomflow_b200._lib import ChainOp, OpKind
    p = lambda t: t.data_ptr()  # noqa: E731
    ops = []
    for ly in layers:
        (wq, sq), (wo, so), (wg, sg), (wu, su), (wd, sd) = (ly[k] for k in ("qkv", "o", "gate", "up", "down"))
        ops.append(ChainOp(kind=OpKind.RMSNORM_GEMV, N=QKV, K=D, wait_prev=1, x=p(b["x"]), w=p(wq), scales=p(sq),
                           norm_w=p(ly["g_attn"]), eps=EPS, y=p(b["qkv"])))
        # O reads the first D entries of QKV in place of the attention output
        ops.append(ChainOp(kind=OpKind.GEMV_RESIDUAL, N=D, K=D, wait_prev=1, x=p(b["qkv"]), w=p(wo), scales=p(so),
                           y=p(b["x"])))
        ops.append(ChainOp(kind=OpKind.RMSNORM_SWIGLU, N=FFN, K=D, wait_prev=1, x=p(b["x"]), w=p(wg), scales=p(sg),
                           w2=p(wu), scales2=p(su), norm_w=p(ly["g_mlp"]), eps=EPS, y=p(b["h"])))
        ops.append(ChainOp(kind=OpKind.GEMV_RESIDUAL, N=D, K=FFN, wait_prev=1, x=p(b["h"]), w=p(wd), scales=p(sd),
                           y=p(b["x"])))
    return (ChainOp * len(ops))(*ops), len(ops)


def _bufs():
    z = lambda n: torch.zeros(n, dtype=torch.float16, device="cuda")  # noqa: E731
    return {"x": z(D), "qkv": z(QKV), "h": z(FFN), "xn": z(D), "o": z(D), "g": z(FFN), "u": z(FFN)}


def _reference_chain(layers, b):
    r, s = R(), st()
    p = lambda t: t.data_ptr()  # noqa: E731
    for ly in layers:
        (wq, sq), (wo, so), (wg, sg), (wu, su), (wd, sd) = (ly[k] for k in ("qkv", "o", "gate", "up", "down"))
        rc = r.afref_rms_norm(p(b["x"]), p(ly["g_attn"]), p(b["xn"]), D, EPS, s)
        rc |= r.afref_w8a16_gemv(p(b["xn"]), p(wq), p(sq), p(b["qkv"]), QKV, D, s)
        rc |= r.afref_w8a16_gemv(p(b["qkv"]), p(wo), p(so), p(b["o"]), D, D, s)
        rc |= r.afref_residual_add(p(b["x"]), p(b["o"]), D, s)
        rc |= r.afref_rms_norm(p(b["x"]), p(ly["g_mlp"]), p(b["xn"]), D, EPS, s)
        rc |= r.afref_w8a16_gemv(p(b["xn"]), p(wg), p(sg), p(b["g"]), FFN, D, s)
        rc |= r.afref_w8a16_gemv(p(b["xn"]), p(wu), p(su), p(b["u"]), FFN, D, s)
        rc |= r.afref_swiglu(p(b["g"]), p(b["u"]), p(b["h"]), FFN, s)
        rc |= r.afref_w8a16_gemv(p(b["h"]), p(wd), p(sd), p(b["o"]), D, FFN, s)
        rc |= r.afref_residual_add(p(b["x"]), p(b["o"]), D, s)
        assert rc == 0


def _run_chain(ops, n, ws):
    return L().af_gemv_chain(ops, n, ws.data_ptr(), ws.numel(), st())


def test_layer_chain_bit_identical_to_reference_kernels():
    layers, x0 = _layers(3)
    ours, theirs = _bufs(), _bufs()
    ours["x"].copy_(x0)
    theirs["x"].copy_(x0)
    ops, n = _chain_ops(layers, ours)
    ws = torch.zeros(L().af_chain_workspace_bytes(n), dtype=torch.uint8, device="cuda")
    assert _run_chain(ops, n, ws) == 0
    _reference_chain(layers, theirs)
    torch.cuda.synchronize()
    flt = ctypes.c_uint(0)
    assert L().af_device_faults(ctypes.byref(flt), 1) == 0 and flt.value == 0
    for k in ("x", "qkv", "h"):
        a, b = ours[k].view(torch.int16), theirs[k].view(torch.int16)
        nbad = int((a != b).sum())
        assert nbad == 0, f"{k}: {nbad} of {a.numel()} values differ from the reference kernel sequence"
    assert not torch.equal(ours["x"], x0)
    assert int(ws.count_nonzero()) == 0   # counters back at zero


def test_chain_repeat_and_graph_replay():
    layers, x0 = _layers(2, seed=9)
    b = _bufs()
    ops, n = _chain_ops(layers, b)
    ws = torch.zeros(L().af_chain_workspace_bytes(n), dtype=torch.uint8, device="cuda")
    res = []
    for _ in range(3):
        b["x"].copy_(x0)
        assert _run_chain(ops, n, ws) == 0
        res.append(b["x"].clone())
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        b["x"].copy_(x0)
        assert L().af_gemv_chain(ops, n, ws.data_ptr(), ws.numel(), s.cuda_stream) == 0
    for _ in range(3):
        with torch.cuda.stream(s):
            g.replay()
        s.synchronize()
        res.append(b["x"].clone())
    torch.cuda.synchronize()
    for r in res[1:]:
        assert torch.equal(r, res[0])
    assert int(ws.count_nonzero()) == 0


def test_chain_independent_ops_match_single_calls():
    """A layer-set chain (independent x per op, no waits) equals one launch per op."""
    from atomflow_b200._lib import ChainOp, OpKind
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    items = []
    for N, K in ((QKV, D), (D, D), (FFN, D), (FFN, D), (D, FFN)) * 2:
        q, s = _weights(g, N, K)
        x = torch.randn(K, generator=g, device="cuda").half()
        items.append((N, K, q, s, x, torch.zeros(N, dtype=torch.float16, device="cuda"),
                      torch.zeros(N, dtype=torch.float16, device="cuda")))
    ops = (ChainOp * len(items))(*[ChainOp(kind=OpKind.GEMV, N=N, K=K, wait_prev=0, x=x.data_ptr(), w=q.data_ptr(),
                                           scales=s.data_ptr(), y=y.data_ptr())
                                   for (N, K, q, s, x, y, _) in items])
    assert L().af_gemv_chain(ops, len(items), None, 0, st()) == 0
    for (N, K, q, s, x, _, y1) in items:
        one = ChainOp(kind=OpKind.GEMV, N=N, K=K, x=x.data_ptr(), w=q.data_ptr(), scales=s.data_ptr(),
                      y=y1.data_ptr())
        assert L().af_gemv_chain(ctypes.byref(one), 1, None, 0, st()) == 0
    torch.cuda.synchronize()
    for (N, K, q, s, x, y, y1) in items:
        assert torch.equal(y.view(torch.int16), y1.view(torch.int16)), (N, K)


def test_chain_rejects_bad_arguments():
    from atomflow_b200._lib import ChainOp, OpKind
    q = torch.zeros(64, 3072, dtype=torch.uint8, device="cuda")
    s = torch.ones(64, 24, dtype=torch.float16, device="cuda")
    x = torch.zeros(3072, dtype=torch.float16, device="cuda")
    y = torch.zeros(64, dtype=torch.float16, device="cuda")
    good = dict(kind=OpKind.GEMV, N=64, K=3072, wait_prev=0, x=x.data_ptr(), w=q.data_ptr(), scales=s.data_ptr(),
                y=y.data_ptr())
    for bad in (dict(K=3000), dict(K=0), dict(N=0), dict(kind=9), dict(x=x.data_ptr() + 2), dict(w=None),
                dict(kind=OpKind.RMSNORM_GEMV), dict(kind=OpKind.RMSNORM_SWIGLU, norm_w=s.data_ptr()),
                dict(K=32768)):
        op = ChainOp(**{**good, **bad})
        assert L().af_gemv_chain(ctypes.byref(op), 1, None, 0, st()) == 1, bad
    two = (ChainOp * 2)(ChainOp(**good), ChainOp(**{**good, "wait_prev": 1}))
    assert L().af_gemv_chain(two, 2, None, 0, st()) == 5       # waits need the workspace
    assert L().af_gemv_chain(two, 0, None, 0, st()) == 1
    torch.cuda.synchronize()


# ---------------------------------------------------------------- fast path

@pytest.mark.parametrize("N,K", [(3072, 3072), (5120, 3072), (8192, 3072), (3072, 8192), (4096, 14336), (1, 128),
                                 (17, 256), (77, 640), (1000, 1536), (4099, 512), (300, 16384)])
def test_fast_chain_gemv_within_tolerance(N, K):
    from atomflow_b200._lib import ChainOp, OpKind
    from tests._util import assert_fp16_parity
    x, q, s = make_gemv_case(N * 3 + K, 1, N, K)
    xd, qd, sd = dev(x), dev(q), dev(s)
    y = torch.zeros(N, dtype=torch.int16, device="cuda")
    op = ChainOp(kind=OpKind.GEMV, N=N, K=K, x=xd.data_ptr(), w=qd.data_ptr(), scales=sd.data_ptr(), y=y.data_ptr())
    assert L().af_gemv_chain_fast(ctypes.byref(op), 1, None, 0, st()) == 0
    torch.cuda.synchronize()
    yb = y.cpu().numpy().view(np.uint16)
    assert_fp16_parity(yb, oracle.gemv_f64(x, q, s, "group", with_l2=True), f"fast {N}x{K}",
                       oracle.gemv_refmath(x, q, s, 8) if N * K <= 4_000_000 else None)
    # deterministic
    y2 = torch.zeros_like(y)
    op.y = y2.data_ptr()
    assert L().af_gemv_chain_fast(ctypes.byref(op), 1, None, 0, st()) == 0
    torch.cuda.synchronize()
    assert torch.equal(y, y2)


def test_fast_layer_chain_matches_exact_within_rounding():
    """The tensor-core chain and the exact chain on the same 3 decode layers: the
    residual stream agrees to FP16 rounding (each op's error is within the GEMV
    tolerance; through 12 ops they compound only to a few FP16 ulp)."""
    layers, x0 = _layers(3, seed=13)
    fast, exact = _bufs(), _bufs()
    fast["x"].copy_(x0)
    exact["x"].copy_(x0)
    ops_f, n = _chain_ops(layers, fast)
    ops_e, _ = _chain_ops(layers, exact)
    ws = torch.zeros(L().af_chain_workspace_bytes(n), dtype=torch.uint8, device="cuda")
    assert L().af_gemv_chain_fast(ops_f, n, ws.data_ptr(), ws.numel(), st()) == 0
    assert L().af_gemv_chain(ops_e, n, ws.data_ptr(), ws.numel(), st()) == 0
    torch.cuda.synchronize()
    a, b = fast["x"].float(), exact["x"].float()
    rms = float(b.pow(2).mean().sqrt())
    err = (a - b).abs()
    assert float(err.max()) <= 1e-2 * rms + 4 * 2.0 ** -10 * float(b.abs().max()), (float(err.max()), rms)
    assert int(ws.count_nonzero()) == 0
