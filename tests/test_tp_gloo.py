"""Tensor-parallel split of the layer set, world size 2 over gloo on CPU.

Each rank quantises its shard (atomflow_b200.tp.shard + quant.quantize_gs128),
computes its partial GEMV with the FP64 oracle, and the partials of
row-parallel projections are summed with all_reduce, as bench.py does with
NCCL on GPUs.  The result must equal the unsharded projection, and the shard
bytes/scales must equal slices of the unsharded quantisation."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


SHAPES = [("qkv", 640, 512, "col"), ("o", 256, 512, "row"), ("down", 256, 1024, "row")]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import oracle
    from atomflow_b200.quant import quantize_gs128
    from atomflow_b200.tp import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    out = {}
    for i, (name, N, K, split) in enumerate(SHAPES):
        g = torch.Generator().manual_seed(100 + i)
        w = torch.randn(N, K, generator=g) * 0.02
        x = torch.randn(1, K, generator=g).half()
        ws, xs = shard(w, x, split, rank, world)
        qs, ss = quantize_gs128(ws.contiguous())
        qfull, sfull = quantize_gs128(w)
        # shard quantisation == slice of the full quantisation
        if split == "col":
            ref_q = qfull.chunk(world, 0)[rank]
            ref_s = sfull.chunk(world, 0)[rank]
        else:
            ref_q = qfull.chunk(world, 1)[rank]
            ref_s = sfull.chunk(world, 1)[rank]
        assert torch.equal(qs.view(torch.uint8), ref_q.contiguous().view(torch.uint8)), name
        assert torch.equal(ss, ref_s.contiguous()), name
        y = oracle.gemv_f64(xs.contiguous().view(torch.int16).numpy().view(np.uint16),
                            qs.view(torch.uint8).numpy(), ss.view(torch.int16).numpy().view(np.uint16), "group")
        yt = torch.from_numpy(y)
        if split == "row":
            dist.all_reduce(yt)
        else:
            parts = [torch.zeros_like(yt) for _ in range(world)]
            dist.all_gather(parts, yt)
            yt = torch.cat(parts, dim=1)
        full = oracle.gemv_f64(x.view(torch.int16).numpy().view(np.uint16), qfull.view(torch.uint8).numpy(),
                               sfull.view(torch.int16).numpy().view(np.uint16), "group")
        out[name] = float(np.abs(yt.numpy() - full).max() / (np.abs(full).max() + 1e-30))
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        q.put(out)


def test_tp_world2_gloo_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    out = q.get(timeout=10)
    for name, rel in out.items():
        assert rel < 1e-12, (name, rel)


def test_shard_rejects_unaligned_row_split():
    from atomflow_b200.tp import shard
    with pytest.raises(ValueError):
        shard(torch.zeros(8, 384), torch.zeros(1, 384), "row", 0, 2)
