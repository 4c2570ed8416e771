"""Python front of the C++ decode engine (af_engine_*, atomflow_b200/csrc/af_engine.cu).

A greedy decode step of a model in the reference's `.bin` format runs in the
library: the engine maps the file, owns the device arenas, launches the step
and captures it as a CUDA graph -- no PyTorch or Python on that path.  This
class mirrors the reference engine's interface (include/core/engine.h:
initialize / inject_token / forward_pass / get_output_token / current_pos_)
for tests and the benchmark.

Modes: "exact" -- every kernel bit-identical to the reference's (projection
chains, attention, norms, RoPE, SwiGLU, residual, embedding; the lm_head is
the library's, the reference's is a cuBLAS call); "fast" -- fused tensor-core
projections and cluster attention, within FP16 rounding of FP64.  The
argmax is the reference's (ids < 65536, its launch_argmax behaviour) unless
`true_argmax` is set.
"""
from __future__ import annotations

import ctypes

from ._lib import check, lib
from .weights_bin import BinFile

MAX_SEQ_LEN = 4096   # KV-cache rows: BASELINE config 3 (the reference engine has 2048, engine.h:41)
MODES = {"exact": 0, "fast": 1}


class DecodeEngine:
    def __init__(self, path, device="cuda", max_seq_len=MAX_SEQ_LEN, true_argmax=False, mode="exact", comm=None):
        """comm: an atomflow_b200.tp.TpComm -- this process's rank of a
        tensor-parallel engine (fast mode; every rank ends each step with the
        same token)."""
        import torch
        self.L = lib()
        if mode not in MODES:
            raise ValueError(f"mode must be one of {list(MODES)}")
        dev = torch.device(device)
        if dev.index is not None:   # a bare "cuda" keeps the current device (one process per GPU)
            torch.cuda.set_device(dev)
        b = BinFile(path)
        self.shape = b.shape
        b.close()
        s = self.shape
        self.D, self.FFN, self.V, self.NL = s.dim, s.ffn, s.vocab, s.n_layers
        self.NH, self.NKV, self.HD = s.n_heads, s.n_kv_heads, s.head_dim
        self.QD, self.KVD = self.NH * self.HD, self.NKV * self.HD
        self.max_seq = max_seq_len
        self.mode = mode
        h = ctypes.c_void_p()
        amode = 0 if true_argmax else 1
        if comm is not None and comm.world > 1:
            if mode != "fast":
                raise ValueError("a tensor-parallel engine runs the fast mode")
            check(self.L.af_engine_create_tp(str(path).encode(), max_seq_len, amode, comm.h, ctypes.byref(h)),
                  "af_engine_create_tp")
        else:
            check(self.L.af_engine_create(str(path).encode(), max_seq_len, MODES[mode], amode, ctypes.byref(h)),
                  "af_engine_create")
        self.comm = comm
        self.h = h
        self.stream = torch.cuda.ExternalStream(self.L.af_engine_stream(h), device=torch.cuda.current_device())
        self.launches_per_step = None

    def close(self):
        if self.h:
            self.L.af_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- the reference engine's interface
    @property
    def current_pos(self) -> int:
        v = ctypes.c_int(0)
        check(self.L.af_engine_get_position(self.h, ctypes.byref(v)), "af_engine_get_position")
        return v.value

    @current_pos.setter
    def current_pos(self, p: int):
        if not 0 <= p < self.max_seq:
            raise ValueError(f"position {p} outside the KV cache (max {self.max_seq})")
        check(self.L.af_engine_set_position(self.h, int(p)), "af_engine_set_position")

    def inject_token(self, token: int):
        check(self.L.af_engine_inject_token(self.h, int(token)), "af_engine_inject_token")

    def get_output_token(self) -> int:
        v = ctypes.c_int(0)
        check(self.L.af_engine_output_token(self.h, ctypes.byref(v)), "af_engine_output_token")
        return v.value

    def forward_pass(self):
        check(self.L.af_engine_step(self.h, 0), "af_engine_step")
        self._info()

    def capture(self, advance=True):
        """One step (plus the position increment when `advance`) as the engine's CUDA graph."""
        pos = self.current_pos
        self.forward_pass()   # the first calls on the device happen outside capture
        self.current_pos = pos
        check(self.L.af_engine_capture(self.h, 1 if advance else 0), "af_engine_capture")
        return self   # a handle for replay(); the engine holds one graph

    def replay(self, g=None, n=1):
        check(self.L.af_engine_replay(self.h, int(n)), "af_engine_replay")

    def synchronize(self):
        check(self.L.af_engine_synchronize(self.h), "af_engine_synchronize")

    @property
    def d_token(self) -> int:
        """Device address of the engine's token int."""
        return self.L.af_engine_device_token(self.h)

    @property
    def logits_ptr(self) -> int:
        return self.L.af_engine_logits(self.h)

    def _info(self):
        dims = (ctypes.c_int * 9)()
        check(self.L.af_engine_info(self.h, dims), "af_engine_info")
        self.launches_per_step = dims[7]

    def weight_bytes(self) -> int:
        """Bytes a step must read at least: every weight, scale and norm, the
        embedding row, and the lm_head."""
        s = self.shape
        b = sum(n * k + n * (k // 128) * 2 for _, n, k in s.linears()) * self.NL
        b += (2 * self.D * 4) * self.NL + self.D * 4 + self.V * self.D * 2 + self.D * 4
        return b

    def kv_bytes(self, pos: int) -> int:
        return 2 * (pos + 1) * self.KVD * 2 * self.NL
