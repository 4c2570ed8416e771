"""The decode-step kernels (af_decode.cu) and the decode engine against the
reference's own kernels and engine (compiled from its sources into oracle/_ref):

  * RoPE tables, RoPE + KV-cache write, RMSNorm, embedding: bit-identical;
  * cached attention: within FP16 rounding of an FP64 oracle, like the
    reference kernel (different summation order, so not bitwise);
  * a whole model: the greedy tokens of DecodeEngine and the reference's
    AtomFlowEngine on the same random-init `.bin` file.
"""
import ctypes

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

NH, NKV, HD, MAXSEQ = 24, 8, 128, 2048


def lib():
    from atomflow_b200 import lib as _l
    return _l()


def ref():
    r = oracle.ref()
    if r is None:
        pytest.skip("oracle/_ref/libafref.so not built")
    return r


def st():
    return torch.cuda.current_stream().cuda_stream


def half_ulp(v):
    return oracle.half_ulp(np.asarray(v, np.float32).astype(np.float16).view(np.uint16)).reshape(np.shape(v))


def test_rope_tables_match_reference():
    L = lib()
    cos = np.empty((MAXSEQ, HD // 2), np.float32)
    sin = np.empty_like(cos)
    assert L.af_rope_tables(cos.ctypes.data_as(ctypes.c_void_p), sin.ctypes.data_as(ctypes.c_void_p), MAXSEQ, HD,
                            500000.0) == 0
    dc = torch.zeros(MAXSEQ * HD // 2, device="cuda")
    ds = torch.zeros_like(dc)
    assert ref().afref_rope_cache(dc.data_ptr(), ds.data_ptr(), MAXSEQ, HD, 500000.0, st()) == 0
    assert np.array_equal(dc.cpu().numpy(), cos.ravel())
    assert np.array_equal(ds.cpu().numpy(), sin.ravel())


def _tables():
    cos = np.empty((MAXSEQ, HD // 2), np.float32)
    sin = np.empty_like(cos)
    lib().af_rope_tables(cos.ctypes.data_as(ctypes.c_void_p), sin.ctypes.data_as(ctypes.c_void_p), MAXSEQ, HD,
                         500000.0)
    return torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()


def test_rope_kv_write_matches_reference():
    L = lib()
    cos, sin = _tables()
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    qd, kvd = NH * HD, NKV * HD
    ok = True
    for pos in (0, 5, 1000, 2047):
        qkv = (torch.randn(qd + 2 * kvd, generator=g, device="cuda") * 3).half()
        a, b = qkv.clone(), qkv.clone()
        kc_a = torch.zeros(MAXSEQ, kvd, dtype=torch.float16, device="cuda")
        vc_a, kc_b, vc_b = kc_a.clone(), kc_a.clone(), kc_a.clone()
        dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        assert L.af_rope_kv_write(a.data_ptr(), cos.data_ptr(), sin.data_ptr(), dpos.data_ptr(), kc_a.data_ptr(),
                                  vc_a.data_ptr(), NH, NKV, HD, MAXSEQ, st()) == 0
        assert ref().afref_rope_kv(b.data_ptr(), cos.data_ptr(), sin.data_ptr(), kc_b.data_ptr(), vc_b.data_ptr(),
                                   pos, NH, NKV, HD, st()) == 0
        torch.cuda.synchronize()
        ok &= torch.equal(a.view(torch.int16), b.view(torch.int16))
        ok &= torch.equal(kc_a.view(torch.int16), kc_b.view(torch.int16))
        ok &= torch.equal(vc_a.view(torch.int16), vc_b.view(torch.int16))
    assert ok, "RoPE + KV write differs from the reference kernels"


def test_embed_and_rmsnorm_match_reference():
    L = lib()
    V, D = 1000, 3072
    table = torch.randn(V, D, device="cuda") * 0.02
    tok = torch.tensor([777], dtype=torch.int32, device="cuda")
    x = torch.zeros(D, dtype=torch.float16, device="cuda")
    assert L.af_embed_lookup(table.data_ptr(), tok.data_ptr(), x.data_ptr(), D, st()) == 0
    torch.cuda.synchronize()
    assert torch.equal(x, table[777].half())
    gen = torch.Generator(device="cuda")
    gen.manual_seed(123)
    # many vectors: a wrong rounding form of the norm shows on about 1 vector in 80
    for it in range(300):
        K, scale = ((3072, 1.0), (1024, 40.0), (200, 0.01), (4096, 3.0))[it % 4]
        xx = (torch.randn(K, generator=gen, device="cuda") * scale).half()
        w = (1 + 0.1 * torch.randn(K, generator=gen, device="cuda")).float()
        a = torch.zeros(K, dtype=torch.float16, device="cuda")
        b = torch.zeros_like(a)
        assert L.af_rmsnorm(xx.data_ptr(), w.data_ptr(), 1e-5, a.data_ptr(), K, st()) == 0
        assert ref().afref_rms_norm(xx.data_ptr(), w.data_ptr(), b.data_ptr(), K, 1e-5, st()) == 0
        torch.cuda.synchronize()
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), K


def _attention_f64(q, kc, vc, seq):
    qf = q.cpu().double().numpy().reshape(NH, HD)
    k = kc[:seq].cpu().double().numpy().reshape(seq, NKV, HD)
    v = vc[:seq].cpu().double().numpy().reshape(seq, NKV, HD)
    out = np.empty((NH, HD))
    for h in range(NH):
        kv = h * NKV // NH
        s = k[:, kv, :] @ qf[h] / np.sqrt(HD)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h] = p @ v[:, kv, :]
    return out.ravel()


def test_decode_attention_parity():
    L = lib()
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    kc = torch.randn(MAXSEQ, NKV * HD, generator=g, device="cuda").half()
    vc = torch.randn(MAXSEQ, NKV * HD, generator=g, device="cuda").half()
    ws = torch.zeros(L.af_decode_attention_workspace_bytes(NH, NKV, MAXSEQ), dtype=torch.uint8, device="cuda")
    for pos in (0, 1, 7, 31, 100, 1024, 2047):
        q = (torch.randn(NH * HD, generator=g, device="cuda") * 2).half()
        dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        outs = []
        for _ in range(2):   # two calls in a row: the workspace is left zeroed
            o = torch.zeros(NH * HD, dtype=torch.float16, device="cuda")
            assert L.af_decode_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), dpos.data_ptr(), o.data_ptr(),
                                         NH, NKV, HD, MAXSEQ, ws.data_ptr(), ws.numel(), st()) == 0
            outs.append(o)
        o_ref = torch.zeros(NH * HD, dtype=torch.float16, device="cuda")
        assert ref().afref_cached_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), o_ref.data_ptr(), pos + 1, HD,
                                            NH, NKV, st()) == 0
        torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1])
        # bit for bit the reference kernel's output
        nbad = int((outs[0].view(torch.int16) != o_ref.view(torch.int16)).sum())
        assert nbad == 0, f"pos {pos}: {nbad} of {NH * HD} outputs differ from the reference attention kernel"
        want = _attention_f64(q, kc, vc, pos + 1)
        for name, got in (("ours", outs[0]), ("reference", o_ref)):
            y = got.float().cpu().numpy().astype(np.float64)
            err = np.abs(y - want)
            ok = (err <= 2 * half_ulp(want)) | (err <= 2e-3 * np.abs(want)) | (err <= 1e-4)
            assert ok.all(), f"{name} pos {pos}: {int((~ok).sum())} outputs off, max err {err.max():.3g}"


def test_fused_rope_attention_equals_the_two_kernels():
    L = lib()
    cos, sin = _tables()
    g = torch.Generator(device="cuda")
    g.manual_seed(17)
    qd, kvd = NH * HD, NKV * HD
    ws_a = torch.zeros(L.af_decode_attention_workspace_bytes(NH, NKV, MAXSEQ), dtype=torch.uint8, device="cuda")
    ws_b = torch.zeros_like(ws_a)
    kc = torch.randn(MAXSEQ, kvd, generator=g, device="cuda").half()
    vc = torch.randn(MAXSEQ, kvd, generator=g, device="cuda").half()
    for pos in (0, 1, 33, 1024, 2047):
        qkv = (torch.randn(qd + 2 * kvd, generator=g, device="cuda") * 2).half()
        dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        ka, va, kb, vb = kc.clone(), vc.clone(), kc.clone(), vc.clone()
        oa = torch.zeros(qd, dtype=torch.float16, device="cuda")
        ob = torch.zeros_like(oa)
        a = qkv.clone()
        assert L.af_rope_kv_write(a.data_ptr(), cos.data_ptr(), sin.data_ptr(), dpos.data_ptr(), ka.data_ptr(),
                                  va.data_ptr(), NH, NKV, HD, MAXSEQ, st()) == 0
        assert L.af_decode_attention(a.data_ptr(), ka.data_ptr(), va.data_ptr(), dpos.data_ptr(), oa.data_ptr(), NH,
                                     NKV, HD, MAXSEQ, ws_a.data_ptr(), ws_a.numel(), st()) == 0
        b = qkv.clone()
        assert L.af_decode_rope_attention(b.data_ptr(), cos.data_ptr(), sin.data_ptr(), dpos.data_ptr(), kb.data_ptr(),
                                          vb.data_ptr(), ob.data_ptr(), NH, NKV, HD, MAXSEQ, ws_b.data_ptr(), ws_b.numel(),
                                          st()) == 0
        torch.cuda.synchronize()
        assert torch.equal(oa.view(torch.int16), ob.view(torch.int16)), pos
        assert torch.equal(ka.view(torch.int16), kb.view(torch.int16)), pos
        assert torch.equal(va.view(torch.int16), vb.view(torch.int16)), pos
        assert torch.equal(b, qkv)   # the fused kernel leaves qkv unrotated


def _attention_f64_g(q, kc, vc, seq, nh, nkv):
    qf = q.cpu().double().numpy().reshape(nh, HD)
    k = kc[:seq].cpu().double().numpy().reshape(seq, nkv, HD)
    v = vc[:seq].cpu().double().numpy().reshape(seq, nkv, HD)
    out = np.empty((nh, HD))
    for h in range(nh):
        kv = h // (nh // nkv)
        s = k[:, kv, :] @ qf[h] / np.sqrt(HD)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h] = p @ v[:, kv, :]
    return out.ravel()


@pytest.mark.parametrize("nh,nkv", [(24, 8), (32, 8), (8, 8), (16, 2), (12, 4)])
def test_fast_rope_attention(nh, nkv):
    """af_decode_rope_attention_fast (one thread-block cluster per kv head):
    the KV-cache rows it writes are bit-identical to the exact RoPE kernel's,
    its output is within FP16 rounding of an FP64 softmax over the same rotated
    q and caches, and two calls in a row give the same bits."""
    L = lib()
    cos, sin = _tables()
    g = torch.Generator(device="cuda")
    g.manual_seed(23 + nh + nkv)
    qd, kvd = nh * HD, nkv * HD
    ws = torch.zeros(L.af_decode_attention_workspace_bytes(nh, nkv, MAXSEQ), dtype=torch.uint8, device="cuda")
    kc = torch.randn(MAXSEQ, kvd, generator=g, device="cuda").half()
    vc = torch.randn(MAXSEQ, kvd, generator=g, device="cuda").half()
    for pos in (0, 1, 7, 33, 130, 1024, MAXSEQ - 1):
        qkv = (torch.randn(qd + 2 * kvd, generator=g, device="cuda") * 2).half()
        dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        ka, va = kc.clone(), vc.clone()
        a = qkv.clone()
        assert L.af_rope_kv_write(a.data_ptr(), cos.data_ptr(), sin.data_ptr(), dpos.data_ptr(), ka.data_ptr(),
                                  va.data_ptr(), nh, nkv, HD, MAXSEQ, st()) == 0
        outs = []
        for _ in range(2):
            kb, vb = kc.clone(), vc.clone()
            b = qkv.clone()
            ob = torch.zeros(qd, dtype=torch.float16, device="cuda")
            assert L.af_decode_rope_attention_fast(b.data_ptr(), cos.data_ptr(), sin.data_ptr(), dpos.data_ptr(),
                                                   kb.data_ptr(), vb.data_ptr(), ob.data_ptr(), nh, nkv, HD, MAXSEQ,
                                                   ws.data_ptr(), ws.numel(), st()) == 0
            torch.cuda.synchronize()
            assert torch.equal(ka.view(torch.int16), kb.view(torch.int16)), pos
            assert torch.equal(va.view(torch.int16), vb.view(torch.int16)), pos
            assert torch.equal(b, qkv)
            outs.append(ob)
        assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16)), pos
        want = _attention_f64_g(a[:qd], ka, va, pos + 1, nh, nkv)
        y = outs[0].float().cpu().numpy().astype(np.float64)
        err = np.abs(y - want)
        ok = (err <= 2 * half_ulp(want)) | (err <= 2e-3 * np.abs(want)) | (err <= 1e-4)
        assert ok.all(), f"pos {pos}: {int((~ok).sum())} outputs off, max err {err.max():.3g}"


def test_position_outside_the_cache_is_skipped_and_flagged():
    """A device-side position at or past max_seq (a replayed step that ran past
    the cache) must write nothing and set AF_FAULT_POSITION, not write out of
    bounds."""
    L = lib()
    cos, sin = _tables()
    qd, kvd = NH * HD, NKV * HD
    flt = ctypes.c_uint(0)
    assert L.af_device_faults(ctypes.byref(flt), 1) == 0
    ws = torch.zeros(L.af_decode_attention_workspace_bytes(NH, NKV, MAXSEQ), dtype=torch.uint8, device="cuda")
    qkv = torch.randn(qd + 2 * kvd, device="cuda").half()
    small = 64   # caches with 64 rows; the buffers run on past them, so a stray write would show
    kc = torch.zeros(2 * small, kvd, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    o = torch.full((qd,), 7.0, dtype=torch.float16, device="cuda")
    for pos in (small, small + 5, -1):
        dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        assert L.af_decode_rope_attention(qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), dpos.data_ptr(),
                                          kc.data_ptr(), vc.data_ptr(), o.data_ptr(), NH, NKV, HD, small,
                                          ws.data_ptr(), ws.numel(), st()) == 0
        assert L.af_rope_kv_write(qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), dpos.data_ptr(), kc.data_ptr(),
                                  vc.data_ptr(), NH, NKV, HD, small, st()) == 0
        torch.cuda.synchronize()
        assert not kc.any() and not vc.any() and bool((o == 7.0).all()), pos
        assert L.af_device_faults(ctypes.byref(flt), 1) == 0
        assert flt.value & 2, pos
    assert L.af_device_faults(ctypes.byref(flt), 0) == 0 and flt.value == 0
    # the workspace is still usable: an in-range call afterwards matches a fresh workspace
    dpos = torch.tensor([small - 1], dtype=torch.int32, device="cuda")
    outs = []
    for w in (ws, torch.zeros_like(ws)):
        oo = torch.zeros(qd, dtype=torch.float16, device="cuda")
        assert L.af_decode_attention(qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(), dpos.data_ptr(), oo.data_ptr(),
                                     NH, NKV, HD, small, w.data_ptr(), w.numel(), st()) == 0
        outs.append(oo)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def test_decode_engine_tokens_match_reference(tmp_path):
    R = oracle.ref_engine()
    if R is None:
        pytest.skip("oracle/_ref/libafref_engine.so not built")
    from atomflow_b200.decode import DecodeEngine
    from atomflow_b200.weights_bin import ModelShape, write_synthetic_bin
    shape = ModelShape(dim=1024, ffn=2048, n_layers=4, n_heads=8, n_kv_heads=2, vocab=128256, max_seq_len=2048)
    path = tmp_path / "tiny.bin"
    write_synthetic_bin(path, shape, seed=21, device="cuda")
    ours = DecodeEngine(path)
    theirs = R.afref_engine_create(str(path).encode())
    try:
        rng = np.random.default_rng(5)
        prompt = rng.integers(0, 65536, 16).tolist()
        tok_a = tok_b = None
        seq_a, seq_b = [], []
        for pos in range(16 + 48):
            feed_a = prompt[pos] if pos < 16 else tok_a
            feed_b = prompt[pos] if pos < 16 else tok_b
            ours.current_pos = pos
            ours.inject_token(feed_a)
            ours.forward_pass()
            tok_a = ours.get_output_token()
            tok_b = R.afref_engine_step(theirs, feed_b, pos)
            if pos >= 15:
                seq_a.append(tok_a)
                seq_b.append(tok_b)
        same = sum(a == b for a, b in zip(seq_a, seq_b))
        print(f"greedy tokens identical: {same} of {len(seq_a)}; ours {seq_a[:8]} reference {seq_b[:8]}")
        assert seq_a[0] == seq_b[0]
        assert seq_a == seq_b
        # the same steps replayed as one graph per step give the same tokens
        ours.current_pos = 16
        ours.inject_token(seq_a[0])
        g = ours.capture(advance=True)
        ours.current_pos = 16
        ours.inject_token(seq_a[0])
        for i in range(8):
            ours.replay(g)
            assert ours.get_output_token() == seq_a[i + 1]
    finally:
        R.afref_engine_destroy(theirs)
