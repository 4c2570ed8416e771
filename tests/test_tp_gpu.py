"""af_w8a16_gemv_allreduce on GPUs.

* Two GPUs (skipped with fewer): one process per GPU, IPC handles exchanged
  over gloo; each rank holds a K-shard of a row-parallel projection; the fused
  GEMV + NVLink all-reduce must equal the unsharded FP64 oracle on every rank,
  bit-identically across ranks, over repeated calls and a graph replay.
* Vocab-parallel lm_head (two GPUs): each rank projects its slice of the
  vocabulary; the exchanged argmax must equal the argmax of all ranks' local
  logits (gathered), on every rank, in true and reference-compatible modes.
* One GPU: a peer that never arrives (its flags are never set) makes the
  bounded wait run out; the kernel must finish, set the status word, and
  leave the GPU usable.  No second waiting kernel runs anywhere.
"""
import ctypes
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, out_q):
    import torch.distributed as dist
    import oracle
    from atomflow_b200.quant import quantize_gs128
    from atomflow_b200.tp import TpComm, shard
    from tests._util import assert_fp16_parity
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = TpComm(rank, world, 8192)
    st = torch.cuda.Stream()
    results = {}
    for name, N, K in [("o", 3072, 3072), ("down", 3072, 8192), ("odd", 1000, 1024)]:
        g = torch.Generator().manual_seed(N + K)
        w = torch.randn(N, K, generator=g) * 0.02
        x = torch.randn(1, K, generator=g).half()
        qf, sf = quantize_gs128(w)
        ws, xs = shard(w, x, "row", rank, world)
        q, s = quantize_gs128(ws.contiguous())
        qd, sd, xd = q.view(torch.uint8).cuda(), s.cuda(), xs.contiguous().cuda()
        ys = [torch.zeros(1, N, dtype=torch.float16, device="cuda") for _ in range(3)]
        with torch.cuda.stream(st):
            for y in ys[:2]:   # two calls in a row: epochs advance, parities alternate
                assert comm.gemv_allreduce(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), y.data_ptr(), N,
                                           K // world, st.cuda_stream) == 0
        st.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=st):
            assert comm.gemv_allreduce(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), ys[2].data_ptr(), N,
                                       K // world, st.cuda_stream) == 0
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        ref = oracle.gemv_f64(x.view(torch.int16).numpy().view(np.uint16), qf.view(torch.uint8).numpy(),
                              sf.view(torch.int16).numpy().view(np.uint16), "group", with_l2=True)
        outs = [y.cpu().numpy().view(np.uint16) for y in ys]
        for o in outs:
            assert_fp16_parity(o, ref, f"{name} rank {rank}")
        assert all(np.array_equal(outs[0], o) for o in outs[1:])
        # the same all-reduce with the residual add folded in
        res = (torch.randn(1, N, generator=g) * 2).half()
        inout = res.cuda()
        with torch.cuda.stream(st):
            assert comm.L.af_w8a16_gemv_allreduce_residual(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(),
                                                           inout.data_ptr(), N, K // world, 128, 0, comm.h,
                                                           st.cuda_stream) == 0
        st.synchronize()
        want = (res.float() + torch.from_numpy(outs[0].view(np.float16).astype(np.float32))).half()
        assert torch.equal(inout.cpu().view(torch.int16), want.view(torch.int16))
        results[name] = outs[0].tobytes()
    gathered = [None] * world
    dist.all_gather_object(gathered, results)
    assert comm.status() == 0
    if rank == 0:
        for name in results:
            assert all(gathered[r][name] == gathered[0][name] for r in range(world)), name
        out_q.put("ok")
    dist.barrier()
    os._exit(0)


def _lm_rank_main(rank, world, port, out_q):
    import torch.distributed as dist
    import oracle
    from atomflow_b200 import lib
    from atomflow_b200.tp import TpComm
    from tests._util import assert_fp32_close
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    L = lib()
    comm = TpComm(rank, world, 64)
    st = torch.cuda.Stream()
    checked = []
    # (V, D, fp8, split point): uneven splits; the FP8 case straddles id 65536
    for V, D, fp8, cut in [(20000, 3072, False, 12345), (70016, 1024, True, 40000)]:
        g = torch.Generator().manual_seed(V)
        w = torch.randn(V, D, generator=g) * 0.02
        x = torch.randn(1, D, generator=g).half()
        if fp8:
            rs = (w.abs().amax(1) / 448).clamp_min(1e-12)
            q = (w / rs[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
            wfull, sfull = q, rs.float()
        else:
            wfull, sfull = w.half(), None
        lo, hi = (0, cut) if rank == 0 else (cut, V)
        wd = wfull[lo:hi].contiguous().cuda()
        sd = sfull[lo:hi].contiguous().cuda() if fp8 else None
        xd = x.cuda()
        logits = torch.zeros(hi - lo, dtype=torch.float32, device="cuda")
        ws = torch.zeros(L.af_lm_head_workspace_bytes(hi - lo, D, 1 if fp8 else 0), dtype=torch.uint8, device="cuda")
        for mode in (0, 1):
            idx = torch.full((1,), -7, dtype=torch.int32, device="cuda")
            with torch.cuda.stream(st):
                for _ in range(3):   # repeated calls: the exchange epoch advances
                    rc = comm.lm_head_argmax(xd.data_ptr(), wd.data_ptr(), fp8, sd.data_ptr() if fp8 else None,
                                             logits.data_ptr(), hi - lo, D, lo, idx.data_ptr(), mode, ws.data_ptr(),
                                             ws.numel(), st.cuda_stream)
                    assert rc == 0, rc
            st.synchronize()
            parts = [None] * world
            dist.all_gather_object(parts, logits.cpu().numpy())
            full = np.concatenate(parts)
            want = oracle.argmax(full, mode)
            assert int(idx.item()) == want, (V, mode, int(idx.item()), want)
            checked.append(int(idx.item()))
        # local logits against the FP64 oracle
        xb = x.view(torch.int16).numpy().view(np.uint16)
        if fp8:
            ref = oracle.gemv_f64(xb, wfull[lo:hi].numpy(), sfull[lo:hi].numpy(), "row")
        else:
            ref = oracle.gemv_f64(xb, wfull[lo:hi].view(torch.int16).numpy().view(np.uint16), None, "f16")
        assert_fp32_close(logits.cpu().numpy(), ref.ravel(), f"lm_head V={V} rank {rank}")
    assert comm.status() == 0
    gathered = [None] * world
    dist.all_gather_object(gathered, checked)
    if rank == 0:
        assert gathered[0] == gathered[1]
        out_q.put("ok")
    dist.barrier()
    os._exit(0)


def _spawn(target, world=2):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    assert q.get(timeout=5) == "ok"


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_lm_head_vocab_parallel_two_gpus():
    _spawn(_lm_rank_main)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gemv_allreduce_two_gpus():
    _spawn(_rank_main)


def test_gemv_allreduce_missing_peer_times_out_with_status():
    from atomflow_b200 import lib
    from tests._util import make_gemv_case
    L = lib()
    h = ctypes.c_void_p()
    assert L.af_tp_create(0, 2, 4096, ctypes.byref(h)) == 0
    # "rank 1" is a second buffer on this GPU that no kernel ever flags
    ghost = torch.zeros(L.af_tp_buffer_bytes(4096), dtype=torch.uint8, device="cuda")
    assert L.af_tp_set_peer(h, 1, ghost.data_ptr()) == 0
    assert L.af_tp_set_wait_limit_ms(h, 50) == 0
    x, q, s = make_gemv_case(1, 1, 1024, 1024)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    qd = torch.from_numpy(q).cuda()
    sd = torch.from_numpy(s.view(np.int16)).cuda()
    y = torch.zeros(1, 1024, dtype=torch.float16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.af_w8a16_gemv_allreduce(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), y.data_ptr(), 1024, 1024, 128, 0,
                                     h, st) == 0
    torch.cuda.synchronize()
    status = ctypes.c_int(0)
    assert L.af_tp_status(h, ctypes.byref(status)) == 0
    assert status.value & 1
    # the context is still usable
    yy = torch.zeros(1, 1024, dtype=torch.float16, device="cuda")
    assert L.af_w8a16_gemv(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), yy.data_ptr(), 1, 1024, 1024, 128, 0, None, 0,
                           st) == 0
    torch.cuda.synchronize()
    assert L.af_tp_destroy(h) == 0


def test_gemv_allreduce_argument_errors():
    from atomflow_b200 import lib
    L = lib()
    h = ctypes.c_void_p()
    assert L.af_tp_create(0, 9, 64, ctypes.byref(h)) == 1           # world > 8
    assert L.af_tp_create(0, 2, 4096, ctypes.byref(h)) == 0
    # peers not opened yet
    assert L.af_w8a16_gemv_allreduce(16, 16, 16, 16, 64, 128, 128, 0, h, None) == 1
    assert L.af_tp_destroy(h) == 0


def test_lm_head_tp_missing_peer_times_out_with_status():
    from atomflow_b200 import lib
    L = lib()
    h = ctypes.c_void_p()
    assert L.af_tp_create(0, 2, 64, ctypes.byref(h)) == 0
    ghost = torch.zeros(L.af_tp_buffer_bytes(64), dtype=torch.uint8, device="cuda")
    assert L.af_tp_set_peer(h, 1, ghost.data_ptr()) == 0
    assert L.af_tp_set_wait_limit_ms(h, 50) == 0
    V, D = 4096, 1024
    w = (torch.randn(V, D, device="cuda") * 0.02).half()
    x = torch.randn(1, D, device="cuda").half()
    ws = torch.zeros(L.af_lm_head_workspace_bytes(V, D, 0), dtype=torch.uint8, device="cuda")
    idx = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.af_lm_head_gemv_tp(x.data_ptr(), w.data_ptr(), 0, None, None, V, D, 0, idx.data_ptr(), 0,
                                ws.data_ptr(), ws.numel(), h, st) == 0
    torch.cuda.synchronize()
    status = ctypes.c_int(0)
    assert L.af_tp_status(h, ctypes.byref(status)) == 0
    assert status.value & 1
    assert 0 <= int(idx.item()) < V   # the local candidate survives a missing peer
    assert L.af_tp_destroy(h) == 0
