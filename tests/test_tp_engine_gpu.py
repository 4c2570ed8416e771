"""Tensor-parallel decode engine on two GPUs (skipped with fewer).

One process per GPU; IPC handles of the exchange buffers travel over gloo.  On
a random-init model file, 32 teacher-forced steps then 32 greedy steps:
  * both ranks hold the same token after every step;
  * every teacher-forced token equals the one-GPU exact engine's (the
    reference's arithmetic), except where that engine's two best logits are
    closer than rounding can separate (a near tie), and the gathered TP logits
    stay within FP16-level rounding of the one-GPU logits;
  * no bounded peer wait runs out (status word clear).
"""
import ctypes
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TF, GREEDY = 32, 32
NEAR_TIE = 2e-2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _logits(eng, n):
    out = np.empty(n, np.float32)
    cudart = ctypes.CDLL("libcudart.so.12")
    eng.synchronize()
    assert cudart.cudaMemcpy(out.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(eng.logits_ptr),
                             ctypes.c_size_t(out.nbytes), 2) == 0
    return out


def _run(eng, prompt, nl):
    eng.capture(advance=True)
    eng.current_pos = 0
    toks, logits = [], []
    for p in range(TF + GREEDY):
        if p < TF:
            eng.inject_token(prompt[p])
        eng.replay()
        toks.append(eng.get_output_token())
        if p < TF:
            logits.append(_logits(eng, nl))
    return toks, logits


def _rank_main(rank, world, port, path, out_q):
    import datetime
    import torch.distributed as dist
    from atomflow_b200.decode import DecodeEngine
    from atomflow_b200.tp import TpComm
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=180))
    prompt = np.random.default_rng(4).integers(0, 65536, TF).tolist()
    try:
        single = None
        if rank == 0:
            e1 = DecodeEngine(path, mode="exact", max_seq_len=1024)
            single = _run(e1, prompt, e1.V)
            e1.close()
        comm = TpComm(rank, world, 1024)
        eng = DecodeEngine(path, mode="fast", max_seq_len=1024, comm=comm)
        toks, logits = _run(eng, prompt, eng.V // world)
        assert comm.status() == 0
        gathered = [None] * world
        dist.all_gather_object(gathered, (toks, logits))
        if rank == 0:
            assert gathered[0][0] == gathered[1][0], "the ranks disagree on the token"
            s_toks, s_logits = single
            report = []
            for p in range(TF):
                full = np.concatenate([gathered[r][1][p] for r in range(world)]).astype(np.float64)
                ref = s_logits[p].astype(np.float64)
                rms = np.sqrt(np.mean(ref ** 2))
                err = np.abs(full - ref).max()
                assert err <= 2e-2 * rms, f"step {p}: TP logits off by {err:.4g} (rms {rms:.4g})"
                if toks[p] != s_toks[p]:
                    top = np.sort(ref[:65536])[-2:]
                    report.append((p, float(top[1] - top[0])))
            assert all(m < NEAR_TIE for _, m in report), report
            out_q.put("ok")
        dist.barrier()
    except Exception as ex:   # noqa: BLE001
        out_q.put(f"rank {rank}: {ex!r}")
        raise
    finally:
        os._exit(0)


def test_tp_engine_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from atomflow_b200.weights_bin import ModelShape, write_synthetic_bin
    shape = ModelShape(dim=1024, ffn=2048, n_layers=4, n_heads=8, n_kv_heads=2, vocab=128256, max_seq_len=1024)
    path = tmp_path / "tp.bin"
    write_synthetic_bin(path, shape, seed=5, device="cuda")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(path), q), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    try:
        msg = q.get(timeout=400)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():   # a rank still waiting on its peer: end it, not the run
                p.kill()
    assert msg == "ok", msg
