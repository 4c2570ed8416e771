"""Tensor parallelism of the decode projections.

* `shard`: Megatron split.  Column-parallel projections (fused QKV, gate, up)
  split the output rows N; row-parallel ones (O, down) split K and need the
  partial outputs summed across ranks.  K / world stays a multiple of 128 for
  every shape used here (3072/8 = 384, 8192/8 = 1024, 4096/8 = 512,
  14336/8 = 1792), so the 128-wide scale groups of a K shard are exactly the
  full matrix's groups.
* `TpComm`: the exchange buffers of af_w8a16_gemv_allreduce (GEMV + all-reduce
  over NVLink peer memory in one kernel), set up over a torch.distributed
  group (any backend; only 64-byte IPC handles travel).
"""
import ctypes

import numpy as np

from ._lib import check, lib


def shard(w, x, split, rank, world):
    """(w [N, K], x [M, K]) -> this rank's (w, x).  split: 'col' or 'row'."""
    if world == 1:
        return w, x
    if split == "col":
        n = w.shape[0]
        if n % world:
            raise ValueError(f"N={n} is not divisible by world={world}")
        return w.chunk(world, 0)[rank], x
    k = w.shape[1]
    if k % (128 * world):
        raise ValueError(f"K={k} must split into multiples of 128 over {world} ranks")
    return w.chunk(world, 1)[rank], x.chunk(world, x.dim() - 1)[rank]


class TpComm:
    """One rank's exchange buffer, with every peer's buffer mapped (CUDA IPC)."""

    def __init__(self, rank, world, max_n, group=None):
        import torch.distributed as dist
        L = lib()
        self.L = L
        self.rank, self.world = rank, world
        self.h = ctypes.c_void_p()
        check(L.af_tp_create(rank, world, max_n, ctypes.byref(self.h)), "af_tp_create")
        mine = (ctypes.c_uint8 * 64)()
        check(L.af_tp_ipc_handle(self.h, mine), "af_tp_ipc_handle")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(mine), group=group)
        flat = np.frombuffer(b"".join(handles), dtype=np.uint8).copy()
        check(L.af_tp_open_peers(self.h, flat.ctypes.data_as(ctypes.c_void_p)), "af_tp_open_peers")

    def gemv_allreduce(self, x, w, s, y, N, K, stream):
        """y = sum over ranks of this rank's shard W x (FP16), in one kernel."""
        return self.L.af_w8a16_gemv_allreduce(x, w, s, y, N, K, 128, 0, self.h, stream)

    def lm_head_argmax(self, x, w, fp8, row_scale, logits, V_local, D, vocab_offset, d_argmax, mode, ws, ws_bytes,
                       stream):
        """Vocab-parallel lm_head: this rank's rows [vocab_offset, +V_local); the
        global greedy token lands in d_argmax on every rank."""
        return self.L.af_lm_head_gemv_tp(x, w, 1 if fp8 else 0, row_scale, logits, V_local, D, vocab_offset,
                                         d_argmax, mode, ws, ws_bytes, self.h, stream)

    def status(self):
        v = ctypes.c_int(0)
        check(self.L.af_tp_status(self.h, ctypes.byref(v)), "af_tp_status")
        return v.value
