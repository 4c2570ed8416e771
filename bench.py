"""Benchmark of the W8A16 decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload layerset|layerset8b|layerchain|gemv:N:K[:M]|lmhead:f16|lmhead:fp8]

Default workload: the Llama-3.2-3B-shaped projection set
at M = 1 -- fused QKV [5120x3072], O [3072x3072], gate and up [8192x3072],
down [3072x8192] -- for 28 independent layers (2.82 GB of FP8 weights plus
FP16 group scales, far larger than the 126 MB L2, so no flush is needed).
One step = the 140 GEMVs in layer order, one CUDA-graph replay.  The metric is
achieved HBM GB/s over the algorithmic bytes (W + scales + x + y).

Arms
  ours       this library through its C ABI (af_w8a16_gemv), graph-captured.
  reference  the reference's own w8a16_gemv_kernel (src/kernel/qkv_gemm.cu,
             compiled from its sources into oracle/_ref/libafref.so) on the
             same data, graph-captured like the reference's main.cu.  The
             reference's path is CUDA, so this arm runs on the GPU.

N > 1 ranks (torchrun): Megatron tensor parallelism of the same layer set --
QKV/gate/up column-split, O/down row-split with the partial outputs summed over
the ranks inside the same kernel through NVLink peer memory
(af_w8a16_gemv_allreduce; --tp-comm nccl uses a separate NCCL all-reduce).  Total work is fixed (strong scaling); `value` counts the
bytes all ranks stream divided by the slowest rank's time.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from atomflow_b200 import lib as af_lib  # noqa: E402
from atomflow_b200.quant import quantize_gs128, quantize_row  # noqa: E402
from atomflow_b200.tp import shard  # noqa: E402

D, FFN, QKV = 3072, 8192, 5120
NLAYERS = 28
PROJ = [("qkv", QKV, D, "col"), ("o", D, D, "row"), ("gate", FFN, D, "col"),
        ("up", FFN, D, "col"), ("down", D, FFN, "row")]
# BASELINE config 4's 8B-shaped layer: hidden 4096, intermediate 14336, GQA 32 Q / 8 KV heads of 128
D8, FFN8, QKV8, NLAYERS8 = 4096, 14336, 4096 + 2 * 8 * 128, 32
PROJ8 = [("qkv", QKV8, D8, "col"), ("o", D8, D8, "row"), ("gate", FFN8, D8, "col"),
         ("up", FFN8, D8, "col"), ("down", D8, FFN8, "row")]
FALLBACK_HBM_GBS = 6650.0


# ------------------------------------------------------------------ utils

def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in the background."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.samples = []
        self.proc = None
        self.ok = True
        try:
            bus = torch.cuda.get_device_properties(device_index).pci_bus_id
            ident = ["--id=" + bus] if bus else []
        except Exception:
            ident = []
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                                          "-lms", "200", *ident], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.ok = False
            return
        self.marks = []
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [c.strip() for c in line.split(",")]))

    def wait_first(self, limit_s=5.0):
        """Block until nvidia-smi has printed a sample (it needs ~1 s to start),
        so that a short timed region still has samples within 250 ms of it."""
        t_end = time.time() + limit_s
        while self.ok and not self.samples and time.time() < t_end:
            time.sleep(0.05)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0, t1):
        rows = [r for (t, r) in self.samples if t0 - 0.25 <= t <= t1 + 0.25] or [r for _, r in self.samples]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "power_w_max": max(pw) if pw else None, "samples": len(rows)}


def algorithmic_bytes(N, K, M=1, scale="group"):
    sb = N * (K // 128) * 2 if scale == "group" else (N * 4 if scale == "row" else 0)
    return N * K + sb + M * K * 2 + M * N * 2


# --------------------------------------------------------------- workload

def make_layerset(device, rank, world, seed=1234, layers=NLAYERS, proj=PROJ):
    """Config-1 weights: per (layer, projection) W ~ N(0, 0.02) quantised to E4M3
    with FP16 group scales (the reference's format); x ~ N(0, 1) FP16.  Under TP
    each rank keeps its shard of every projection."""
    items = []
    g = torch.Generator(device=device)
    for layer in range(layers):
        for pi, (name, N, K, split) in enumerate(proj):
            g.manual_seed(seed + 1000 * layer + pi)
            w = torch.randn(N, K, generator=g, device=device, dtype=torch.float32) * 0.02
            x = torch.randn(1, K, generator=g, device=device, dtype=torch.float32).half()
            w, x = shard(w, x, split, rank, world)
            q, s = quantize_gs128(w.contiguous())
            del w
            items.append(dict(name=name, layer=layer, N=q.shape[0], K=q.shape[1], split=split,
                              q=q.view(torch.uint8).contiguous(), s=s.contiguous(), x=x.contiguous(),
                              y=torch.zeros(1, q.shape[0], dtype=torch.float16, device=device)))
    return items


NORM_EPS = 1e-5


def make_layerchain(device, rank, world, seed=1234, layers=NLAYERS):
    """The decode layer without attention, in the reference's order
    (src/core/engine.cu:292-483): RMSNorm -> QKV, O (input: the first K_o
    entries of QKV, standing in for attention) -> residual, RMSNorm -> gate, up
    -> SwiGLU -> down -> residual, for 28 layers of config-1 weights.  FP32 norm
    weights 1 + N(0, 0.1); the residual stream x ~ N(0, 1) is reset every step."""
    items = make_layerset(device, rank, world, seed, layers)
    g = torch.Generator(device=device)
    g.manual_seed(seed + 77)
    nlayers, layers = layers, []
    for l in range(nlayers):
        p = {it["name"]: it for it in items[5 * l:5 * l + 5]}
        for it in p.values():
            it.pop("x", None)
            it.pop("y", None)
        layers.append(dict(p, layer=l, name=f"layer{l}", split="chain",
                           g_attn=(1 + 0.1 * torch.randn(D, generator=g, device=device)).float().contiguous(),
                           g_mlp=(1 + 0.1 * torch.randn(D, generator=g, device=device)).float().contiguous()))
    qkv_n, ffn_n = layers[0]["qkv"]["N"], layers[0]["gate"]["N"]
    bufs = dict(x0=torch.randn(1, D, generator=g, device=device).half(),
                x=torch.zeros(1, D, dtype=torch.float16, device=device),
                qkv=torch.zeros(1, qkv_n, dtype=torch.float16, device=device),
                h=torch.zeros(1, ffn_n, dtype=torch.float16, device=device),
                # reference arm intermediates (it stores every stage, as engine.cu does)
                xn=torch.zeros(1, D, dtype=torch.float16, device=device),
                o=torch.zeros(1, D, dtype=torch.float16, device=device),
                up=torch.zeros(1, ffn_n, dtype=torch.float16, device=device))
    return layers, bufs


def chain_bytes(layers, tp):
    """Algorithmic bytes of one step on one rank: every projection's weights,
    scales and x/y, the norm weights and x, and the residual reads."""
    b = 0
    for ly in layers:
        for nm in ("qkv", "o", "gate", "up", "down"):
            b += algorithmic_bytes(ly[nm]["N"], ly[nm]["K"])
        b += 2 * (D * 4 + D * 2)        # two RMSNorms: weight + x
        b += 2 * D * 2                  # two residual reads
    return b


class OursChain:
    """4 launches per layer: af_rmsnorm_w8a16_gemv (QKV), af_w8a16_gemv_residual
    (O), af_rmsnorm_w8a16_swiglu (gate/up), af_w8a16_gemv_residual (down); at
    N > 1 the row-split O/down are af_w8a16_gemv_allreduce_residual."""
    launches_per_layer = 4

    def __init__(self, bufs, as_chain=False, exact=False):
        self.L = af_lib()
        self.b = bufs
        self.comm = None
        self.fn = self.L.af_gemv_chain if exact else self.L.af_gemv_chain_fast
        if as_chain:
            from atomflow_b200._lib import ChainOp
            self.ChainOp = ChainOp
            self.launch_all = self._launch_all
            self.ws = torch.zeros(self.L.af_chain_workspace_bytes(4 * NLAYERS), dtype=torch.uint8,
                                  device=bufs["x"].device)

    def _launch_all(self, stream, layers):
        """All layers' 4 fused projections as ONE persistent launch (af_gemv_chain)."""
        b, C = self.b, self.ChainOp
        p = lambda t: t.data_ptr()  # noqa: E731
        ops = []
        for ly in layers:
            q, o, ga, up, dn = (ly[k] for k in ("qkv", "o", "gate", "up", "down"))
            ops += [C(kind=2, N=q["N"], K=q["K"], wait_prev=1, x=p(b["x"]), w=p(q["q"]), scales=p(q["s"]),
                      norm_w=p(ly["g_attn"]), eps=NORM_EPS, y=p(b["qkv"])),
                    C(kind=1, N=o["N"], K=o["K"], wait_prev=1, x=p(b["qkv"]), w=p(o["q"]), scales=p(o["s"]),
                      y=p(b["x"])),
                    C(kind=3, N=ga["N"], K=ga["K"], wait_prev=1, x=p(b["x"]), w=p(ga["q"]), scales=p(ga["s"]),
                      w2=p(up["q"]), scales2=p(up["s"]), norm_w=p(ly["g_mlp"]), eps=NORM_EPS, y=p(b["h"])),
                    C(kind=1, N=dn["N"], K=dn["K"], wait_prev=1, x=p(b["h"]), w=p(dn["q"]), scales=p(dn["s"]),
                      y=p(b["x"]))]
        arr = (C * len(ops))(*ops)
        self._check(self.fn(arr, len(ops), self.ws.data_ptr(), self.ws.numel(), stream.cuda_stream), "af_gemv_chain")

    def _check(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"{what}: {self.L.af_status_string(rc).decode()}")

    def _row(self, stream, it, xptr):
        xo = self.b["x"].data_ptr()
        if self.comm is not None:
            self._check(self.L.af_w8a16_gemv_allreduce_residual(xptr, it["q"].data_ptr(), it["s"].data_ptr(), xo,
                                                                 it["N"], it["K"], 128, 0, self.comm.h,
                                                                 stream.cuda_stream), "allreduce_residual")
        else:
            self._check(self.L.af_w8a16_gemv_residual(xptr, it["q"].data_ptr(), it["s"].data_ptr(), xo, it["N"],
                                                      it["K"], 128, 0, None, stream.cuda_stream), "gemv_residual")

    def launch(self, stream, ly, xptr=None, yptr=None):
        b, L, st = self.b, self.L, stream.cuda_stream
        q = ly["qkv"]
        self._check(L.af_rmsnorm_w8a16_gemv(b["x"].data_ptr(), ly["g_attn"].data_ptr(), NORM_EPS, q["q"].data_ptr(),
                                            q["s"].data_ptr(), b["qkv"].data_ptr(), q["N"], q["K"], 128, 0, None,
                                            st), "rmsnorm_gemv")
        self._row(stream, ly["o"], b["qkv"].data_ptr())
        ga, up = ly["gate"], ly["up"]
        self._check(L.af_rmsnorm_w8a16_swiglu(b["x"].data_ptr(), ly["g_mlp"].data_ptr(), NORM_EPS, ga["q"].data_ptr(),
                                              ga["s"].data_ptr(), up["q"].data_ptr(), up["s"].data_ptr(),
                                              b["h"].data_ptr(), ga["N"], ga["K"], 128, 0, None, None, st),
                    "rmsnorm_swiglu")
        self._row(stream, ly["down"], b["h"].data_ptr())


class RefChain:
    """The reference's own kernels in engine.cu's order, 10 launches per layer:
    rms_norm, gemv QKV, gemv O, residual_add, rms_norm, gemv gate, gemv up,
    swiglu, gemv down, residual_add (oracle/_ref, compiled from its sources)."""
    launches_per_layer = 10

    def __init__(self, bufs):
        import oracle
        self.R = oracle.ref()
        if self.R is None:
            raise FileNotFoundError("oracle/_ref/libafref.so")
        self.b = bufs

    def launch(self, stream, ly, xptr=None, yptr=None):
        R, b, st = self.R, self.b, stream.cuda_stream
        x, xn, o, h, up = (b[k].data_ptr() for k in ("x", "xn", "o", "h", "up"))
        rc = R.afref_rms_norm(x, ly["g_attn"].data_ptr(), xn, D, NORM_EPS, st)
        q = ly["qkv"]
        rc |= R.afref_w8a16_gemv(xn, q["q"].data_ptr(), q["s"].data_ptr(), b["qkv"].data_ptr(), q["N"], q["K"], st)
        oo = ly["o"]
        rc |= R.afref_w8a16_gemv(b["qkv"].data_ptr(), oo["q"].data_ptr(), oo["s"].data_ptr(), o, oo["N"], oo["K"], st)
        rc |= R.afref_residual_add(x, o, D, st)
        rc |= R.afref_rms_norm(x, ly["g_mlp"].data_ptr(), xn, D, NORM_EPS, st)
        ga, uu, dd = ly["gate"], ly["up"], ly["down"]
        rc |= R.afref_w8a16_gemv(xn, ga["q"].data_ptr(), ga["s"].data_ptr(), h, ga["N"], ga["K"], st)
        rc |= R.afref_w8a16_gemv(xn, uu["q"].data_ptr(), uu["s"].data_ptr(), up, uu["N"], uu["K"], st)
        rc |= R.afref_swiglu(h, up, h, ga["N"], st)
        rc |= R.afref_w8a16_gemv(h, dd["q"].data_ptr(), dd["s"].data_ptr(), o, dd["N"], dd["K"], st)
        rc |= R.afref_residual_add(x, o, D, st)
        if rc != 0:
            raise RuntimeError(f"reference chain launch failed ({rc})")


def make_single(device, N, K, M, seed=99):
    """One GEMV shape, with enough rotating weight copies to exceed 4x L2."""
    copies = max(2, int(np.ceil(4 * 128e6 / (N * K))))
    items = []
    g = torch.Generator(device=device)
    for i in range(copies):
        g.manual_seed(seed + i)
        w = torch.randn(N, K, generator=g, device=device) * 0.02
        q, s = quantize_gs128(w)
        x = torch.randn(M, K, generator=g, device=device).half()
        items.append(dict(name=f"gemv{i}", layer=i, N=N, K=K, split="col", q=q.view(torch.uint8), s=s, x=x,
                          y=torch.zeros(M, N, dtype=torch.float16, device=device)))
    return items


def make_lmhead(device, fp8, rank=0, world=1, V=128256, D=3072, seed=7):
    """W [128256 x 3072] ~ N(0, 0.02) as FP16, or FP8-E4M3 with an
    FP32 per-row scale; x ~ N(0, 1) FP16; FP32 logits plus the greedy argmax.
    world > 1: this rank's vocab rows [rank*V/world, (rank+1)*V/world)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = torch.randn(V, D, generator=g, device=device) * 0.02
    x = torch.randn(1, D, generator=g, device=device).half()
    if fp8:
        q, rs = quantize_row(w)
        del w
        wq, scale = q.view(torch.uint8).contiguous(), rs.contiguous()
    else:
        wq, scale = w.half().contiguous(), None
        del w
    lo, hi = rank * V // world, (rank + 1) * V // world
    if world > 1:
        wq = wq[lo:hi].contiguous()
        scale = scale[lo:hi].contiguous() if scale is not None else None
    return [dict(name="lm_head", layer=0, N=hi - lo, K=D, off=lo, split="col", q=wq, s=scale, x=x, fp8=fp8,
                 y=torch.zeros(1, hi - lo, dtype=torch.float32, device=device),
                 idx=torch.zeros(1, dtype=torch.int32, device=device))]


def lm_bytes(it):
    V, D = it["N"], it["K"]
    return V * D * (1 if it["fp8"] else 2) + (V * 4 if it["fp8"] else 0) + D * 2 + V * 4


# ------------------------------------------------------------------- arms

class OursGemv:
    def __init__(self, items, device):
        self.L = af_lib()
        self.items = items
        need = max(self.L.af_w8a16_gemv_workspace_bytes(it["x"].shape[0], it["N"], it["K"], 0) for it in items)
        self.ws = torch.zeros(need, dtype=torch.uint8, device=device)

        self.comm = None

    def launch(self, stream, it, xptr=None, yptr=None):
        if self.comm is not None and it["split"] == "row":
            rc = self.comm.gemv_allreduce(xptr or it["x"].data_ptr(), it["q"].data_ptr(), it["s"].data_ptr(),
                                          yptr or it["y"].data_ptr(), it["N"], it["K"], stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(f"af_w8a16_gemv_allreduce: {self.L.af_status_string(rc).decode()}")
            return
        rc = self.L.af_w8a16_gemv(xptr or it["x"].data_ptr(), it["q"].data_ptr(), it["s"].data_ptr(),
                                  yptr or it["y"].data_ptr(), it["x"].shape[0], it["N"], it["K"], 128, 0,
                                  self.ws.data_ptr(), self.ws.numel(), stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"af_w8a16_gemv: {self.L.af_status_string(rc).decode()}")


class OursGemmTc(OursGemv):
    """The batched projection through af_w8a16_gemm_tc (tcgen05 tensor cores)."""

    def launch(self, stream, it, xptr=None, yptr=None):
        rc = self.L.af_w8a16_gemm_tc(xptr or it["x"].data_ptr(), it["q"].data_ptr(), it["s"].data_ptr(),
                                     yptr or it["y"].data_ptr(), it["x"].shape[0], it["N"], it["K"], 128, 0,
                                     stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"af_w8a16_gemm_tc: {self.L.af_status_string(rc).decode()}")


class OursChainSet:
    """The layer set as ONE persistent launch (af_gemv_chain): every GEMV of the
    step in order, each waiting for the previous one to finish on every CTA --
    the same ordering the reference's 140 dependent launches have -- while the
    next GEMV's weights stream in."""
    launches_per_item = 1 / 140

    def __init__(self, items, device, wait=True, exact=False):
        from atomflow_b200._lib import ChainOp
        self.L = af_lib()
        self.wait = wait
        self.fn = self.L.af_gemv_chain if exact else self.L.af_gemv_chain_fast
        self.ChainOp = ChainOp
        self.ws = torch.zeros(self.L.af_chain_workspace_bytes(len(items)), dtype=torch.uint8, device=device)

    def ops(self, items, xptrs=None, yptrs=None):
        return (self.ChainOp * len(items))(*[
            self.ChainOp(kind=0, N=it["N"], K=it["K"], wait_prev=int(self.wait and i > 0),
                         x=xptrs[i] if xptrs else it["x"].data_ptr(), w=it["q"].data_ptr(), scales=it["s"].data_ptr(),
                         y=yptrs[i] if yptrs else it["y"].data_ptr())
            for i, it in enumerate(items)])

    def launch_all(self, stream, items, xptrs=None, yptrs=None):
        ops = self.ops(items, xptrs, yptrs)
        rc = self.fn(ops, len(items), self.ws.data_ptr(), self.ws.numel(), stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"af_gemv_chain: {self.L.af_status_string(rc).decode()}")


class RefGemv:
    def __init__(self, items, device):
        sys.path.insert(0, str(ROOT))
        import oracle
        self.L = oracle.ref()
        if self.L is None:
            raise FileNotFoundError("oracle/_ref/libafref.so")
        self.items = items

    def launch(self, stream, it, xptr=None, yptr=None):
        # The reference kernel computes one token per launch (qkv_gemm.cu:129-150 ignores M),
        # so M tokens are M launches, one per row of x and y.
        M, K, N = it["x"].shape[0], it["K"], it["N"]
        x0, y0 = xptr or it["x"].data_ptr(), yptr or it["y"].data_ptr()
        for m in range(M):
            rc = self.L.afref_w8a16_gemv(x0 + m * K * 2, it["q"].data_ptr(), it["s"].data_ptr(), y0 + m * N * 2, N, K,
                                         stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(f"reference launch failed ({rc})")


class OursLmHead:
    def __init__(self, items, device):
        self.L = af_lib()
        it = items[0]
        self.ws = torch.zeros(self.L.af_lm_head_workspace_bytes(it["N"], it["K"], int(it["fp8"])),
                              dtype=torch.uint8, device=device)
        self.comm = None

    def launch(self, stream, it, xptr=None, yptr=None):
        if self.comm is not None:   # vocab-parallel: the argmax pairs cross NVLink in the same kernel
            rc = self.comm.lm_head_argmax(xptr or it["x"].data_ptr(), it["q"].data_ptr(), it["fp8"],
                                          it["s"].data_ptr() if it["s"] is not None else None,
                                          yptr or it["y"].data_ptr(), it["N"], it["K"], it["off"],
                                          it["idx"].data_ptr(), 0, self.ws.data_ptr(), self.ws.numel(),
                                          stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(f"af_lm_head_gemv_tp: {self.L.af_status_string(rc).decode()}")
            return
        rc = self.L.af_lm_head_gemv(xptr or it["x"].data_ptr(), it["q"].data_ptr(), int(it["fp8"]),
                                    it["s"].data_ptr() if it["s"] is not None else None, yptr or it["y"].data_ptr(),
                                    it["N"], it["K"], it["idx"].data_ptr(), 0, self.ws.data_ptr(), self.ws.numel(),
                                    stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"af_lm_head_gemv: {self.L.af_status_string(rc).decode()}")


class RefLmHead:
    """The reference's lm_head: its exact cublasGemmEx call (engine.cu:498-512) and its
    launch_argmax (argmax.cu:92-119), compiled from its sources (oracle/_ref)."""

    def __init__(self, items, device):
        import oracle
        self.L = oracle.ref()
        if self.L is None:
            raise FileNotFoundError("oracle/_ref/libafref.so (needs the reference sources)")

    def launch(self, stream, it, xptr=None, yptr=None):
        st = stream.cuda_stream
        rc = self.L.afref_lm_head(it["q"].data_ptr(), xptr or it["x"].data_ptr(), yptr or it["y"].data_ptr(),
                                  it["N"], it["K"], st)
        rc = rc or self.L.afref_argmax(yptr or it["y"].data_ptr(), it["N"], it["idx"].data_ptr(), st)
        if rc != 0:
            raise RuntimeError(f"reference lm_head failed ({rc})")


def capture_step(arm, items, stream, allreduce=None, pre=None, post=None):
    def step():
        if pre:
            pre()
        if hasattr(arm, "launch_all"):
            arm.launch_all(stream, items)
        else:
            for it in items:
                arm.launch(stream, it)
                if allreduce is not None and it["split"] == "row":
                    allreduce(it["y"])
        if post:
            post()

    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        step()     # one eager pass (sets kernel attributes, NCCL warm-up) before capture
    stream.synchronize()
    with torch.cuda.graph(g, stream=stream):
        step()
    return g


def time_graph(g, stream, steps, warmup, dist_on):
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(steps):
            g.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    t1 = time.time()
    ms = ev0.elapsed_time(ev1)
    if dist_on:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
    return ms, t0, t1


# ------------------------------------------------------------ CPU baseline

def cpu_baseline(items, budget_s=10.0):
    """The reference's GEMV arithmetic as a host loop (oracle, OpenMP over rows,
    bit-identical to the reference kernel) on a bounded sample of the workload:
    the first layer's five projections, repeated until ~budget_s have passed."""
    import oracle
    L = oracle.cpu()
    L.af_oracle_gemv_cpu_baseline.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 2 + [ctypes.c_void_p, ctypes.c_int]
    sample = items[:5]
    host = [(it["x"].cpu().numpy().view(np.uint16).copy(), it["q"].cpu().numpy().copy(),
             it["s"].cpu().numpy().view(np.uint16).copy(), np.empty(it["N"], np.uint16), it["N"], it["K"])
            for it in sample]
    cores = os.cpu_count() or 1
    nbytes = sum(algorithmic_bytes(N, K) for (_, _, _, _, N, K) in host)
    reps, t0 = 0, time.perf_counter()
    while True:
        for x, q, s, y, N, K in host:
            L.af_oracle_gemv_cpu_baseline(x.ctypes.data, q.ctypes.data, s.ctypes.data, N, K, y.ctypes.data, cores)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(nbytes * reps / dt / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"layer 0's 5 projections (M=1, {nbytes / 1e6:.1f} MB algorithmic) x {reps} passes, "
                      f"{dt:.1f} s, {cores} OpenMP threads"}


# -------------------------------------------------------------------- main

DECODE_POS = 1024
TOKEN_CHECK_STEPS = 64


def decode_model_path():
    """BASELINE config 3's random-init model in the reference's .bin format,
    written once per box (generated on the GPU) and shared by both arms."""
    from atomflow_b200.weights_bin import ModelShape, synthetic_model_file
    return synthetic_model_file(ModelShape(), seed=0)


def run_decode(args, device, local):
    """Greedy decode of a Llama-3.2-3B-shaped model (config 3): KV cache
    prefilled to 1024 positions by teacher-forced steps with seeded random
    tokens, then `steps` greedy steps.  Ours: DecodeEngine, one CUDA-graph
    replay per token, position and token kept on the device.  Reference: its
    own AtomFlowEngine (oracle/_ref), TPOT as its main.cu measures it -- one
    graph of forward_pass at position 1024, replayed."""
    world = int(os.environ.get("WORLD_SIZE", "1")) if args.impl == "ours" else 1
    rank = int(os.environ.get("RANK", "0")) if world > 1 else 0
    if world > 1 and rank != 0:
        torch.distributed.barrier()          # rank 0 writes the model file once
    path = decode_model_path()
    if world > 1 and rank == 0:
        torch.distributed.barrier()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.wait_first()
    peak, peak_kind = measured_peaks()
    config = {"workload": "llama3.2-3b-shaped greedy decode, 28 layers, random-init weights in the reference .bin "
                          "format (BASELINE config 3)", "position": DECODE_POS, "M": 1,
              "kv_cache": f"prefilled to {DECODE_POS} positions by teacher-forced steps (seeded random tokens)",
              "l2": "3.8 GB read per step (weights, lm_head, KV cache) >> 126 MB L2 (no flush needed)", "parallelism": f"tp{world}" if world > 1 else "single"}
    out = {"metric": "decode tok/s (Llama-3.2-3B-shaped, M=1, KV cache at 1024 positions)", "unit": "tok/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "fp8e4m3 weights x fp16 act, fp32 accum", "data": "synthetic seeded",
           "config": config}
    if args.impl == "reference":
        import oracle
        R = oracle.ref_engine()
        if R is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libafref_engine.so not built"}))
            return 0
        h = R.afref_engine_create(str(path).encode())
        t0 = time.time()
        ms = float(R.afref_engine_tpot_ms(h, DECODE_POS, args.steps, args.warmup))
        t1 = time.time()
        sampler.stop()
        if ms <= 0:
            raise RuntimeError(f"reference TPOT measurement failed ({ms})")
        out.update({"impl": "reference", "value": round(1000.0 / ms, 2), "ms_per_step": round(ms, 5),
                    "clocks": sampler.summary(t0, t1), "gpu_launches": 0,
                    "e2e": {"value": round(1000.0 / ms, 2), "unit": "tok/s", "h2d_bytes_per_step": 0,
                            "d2h_bytes_per_step": 0},
                    "cpu_baseline": {"value": round(1000.0 / ms, 2), "unit": "tok/s", "cores": None,
                                     "kind": "reference", "sample": "the reference's AtomFlowEngine (CUDA, compiled "
                                     "from its sources), graph of forward_pass at position 1024, on this GPU"}})
        print(json.dumps(out))
        R.afref_engine_destroy(h)
        return 0
    from atomflow_b200.decode import DecodeEngine
    comm = None
    if world > 1:
        from atomflow_b200.tp import TpComm
        if args.decode_mode != "fast":
            raise SystemExit("tensor-parallel decode runs the fast mode")
        from atomflow_b200.weights_bin import BinFile
        b = BinFile(path)
        comm = TpComm(rank, world, b.shape.dim)
        b.close()
    eng = DecodeEngine(path, mode=args.decode_mode, comm=comm)
    config["engine"] = (f"C++ af_engine, {args.decode_mode} mode: " +
                        ("every kernel bit-identical to the reference's" if args.decode_mode == "exact" else
                         "fused tensor-core projections, cluster attention (one 8-CTA cluster per kv head)"))
    if world > 1:
        config["engine"] += (f"; Megatron tensor parallel over {world} GPUs: QKV/gate/up column-split, O/down "
                             "row-split with the all-reduce and residual fused into the GEMV over NVLink peer "
                             "memory, vocab-parallel lm_head with the argmax pairs exchanged in-kernel")

    def sync_all():
        eng.stream.synchronize()
        if world > 1:
            torch.distributed.barrier()
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, 65536, DECODE_POS).tolist()
    g = eng.capture(advance=True)
    eng.current_pos = 0
    if os.environ.get("AF_DECODE_PREFILL", "1") != "0":   # "0": profiling runs only (the cache's
        for t in prompt:                                  # contents change no kernel's work)
            eng.inject_token(t)
            eng.replay(g)
    else:
        config["kv_cache"] = "not prefilled (profiling run)"
        eng.current_pos = DECODE_POS
    eng.stream.synchronize()
    assert eng.current_pos == DECODE_POS
    first_token = eng.get_output_token()  # the prefill's last output: the first greedy step's input
    if DECODE_POS + max(args.warmup, args.steps + 3, TOKEN_CHECK_STEPS) >= eng.max_seq:
        raise SystemExit(f"--steps/--warmup would run past the {eng.max_seq}-row KV cache")
    for _ in range(args.warmup):          # greedy warm-up steps, then rewind
        eng.replay(g)
    eng.current_pos = DECODE_POS
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sync_all()
    t0 = time.time()
    ev0.record(eng.stream)
    for _ in range(args.steps):
        eng.replay(g)
    ev1.record(eng.stream)
    sync_all()
    t1 = time.time()
    ms = max_over_ranks(ev0.elapsed_time(ev1), world) / args.steps
    clocks = sampler.summary(t0, t1) if sampler else None
    # end to end: each step the host sends the token from pinned memory, the
    # captured step runs, and the next token returns to pinned memory
    cudart = ctypes.CDLL("libcudart.so.12")
    cudart.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    cudart.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    tok_h = torch.zeros(1, dtype=torch.int32).pin_memory()
    tok_back = torch.zeros(1, dtype=torch.int32).pin_memory()
    est = eng.stream.cuda_stream

    def e2e_step():
        cudart.cudaMemcpyAsync(eng.d_token, tok_h.data_ptr(), 4, 1, est)
        eng.replay(g)
        cudart.cudaMemcpyAsync(tok_back.data_ptr(), eng.d_token, 4, 2, est)

    eng.current_pos = DECODE_POS
    for _ in range(3):
        e2e_step()
    eng.current_pos = DECODE_POS
    sync_all()
    ev0.record(eng.stream)
    for _ in range(args.steps):
        e2e_step()
    ev1.record(eng.stream)
    sync_all()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1), world) / args.steps
    if sampler:
        sampler.stop()
    # greedy tokens from position DECODE_POS, checked against the reference engine's
    eng.current_pos = DECODE_POS
    eng.inject_token(first_token)
    ours_toks = []
    for _ in range(TOKEN_CHECK_STEPS):
        eng.replay(g)
        ours_toks.append(eng.get_output_token())
    tokens = {"greedy_steps": TOKEN_CHECK_STEPS, "from_position": DECODE_POS, "ours": ours_toks}
    if comm is not None and comm.status() != 0:
        raise RuntimeError("tensor-parallel decode: a peer wait ran out (status word set)")
    launches = eng.launches_per_step * args.steps
    if world > 1:
        sync_all()
        eng.close()
        if rank != 0:
            return finish(True)
    import oracle
    R = oracle.ref_engine() if not args.no_token_check and config["kv_cache"].startswith("prefilled") else None
    if R is not None:
        h = R.afref_engine_create(str(path).encode())
        tok = None
        ref_toks, margins = [], []
        nv = ctypes.c_int(0)
        for pos in range(DECODE_POS + TOKEN_CHECK_STEPS):
            tok = R.afref_engine_step(h, int(prompt[pos]) if pos < DECODE_POS else tok, pos)
            if pos >= DECODE_POS:
                ref_toks.append(tok)
                # the reference's two best candidate logits (ids < 65536, as its argmax)
                torch.cuda.synchronize()
                src = R.afref_engine_logits(h, ctypes.byref(nv))
                t = torch.empty(eng.V, dtype=torch.float32, device="cuda")
                torch.cuda.synchronize()
                cudart.cudaMemcpy(ctypes.c_void_p(t.data_ptr()), ctypes.c_void_p(src), ctypes.c_size_t(4 * eng.V), 3)
                top = torch.topk(t[:65536], 2).values.tolist()
                margins.append(top[0] - top[1])
        R.afref_engine_destroy(h)
        div = [i for i, (a, b) in enumerate(zip(ours_toks, ref_toks)) if a != b]
        tokens.update({"reference": ref_toks, "match_reference": not div,
                       "first_divergence": (DECODE_POS + div[0]) if div else None})
        if div:
            # a greedy sequence after a divergence is a different sequence: what
            # matters is whether the first divergence is a near tie in the
            # reference's own logits (two candidates closer than rounding)
            tokens["reference_top2_margin_at_divergence"] = round(margins[div[0]], 6)
            tokens["reference_min_top2_margin"] = round(min(margins), 6)
    else:
        tokens["match_reference"] = None
    step_bytes = eng.weight_bytes() + eng.kv_bytes(DECODE_POS + args.steps // 2)
    achieved = step_bytes / (ms / 1e3) / 1e9
    out.update({"value": round(1000.0 / ms, 2), "ms_per_step": round(ms, 5), "clocks": clocks,
                "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                             "frac": round(achieved / peak, 4),
                             "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                             "traffic": None, "kernel": "whole step (GEMV kernels carry 94% of the bytes)",
                             "per_launch": f"{step_bytes / 1e9:.3f} GB per step (weights, scales, norms, lm_head, "
                                           f"embedding row, KV cache) over {ms * 1e3:.1f} us"},
                "gpu_launches": launches, "tokens": tokens,
                "e2e": {"value": round(1000.0 / e2e_ms, 2), "unit": "tok/s", "ms_per_step": round(e2e_ms, 5),
                        "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                        "path": "af_engine (C++) over the C ABI: token H2D from pinned memory, the captured step, next "
                                "token D2H to pinned memory, every step"}})
    if world > 1:
        out["roofline"]["achieved"] = round(achieved / world, 2)   # per GPU: each reads 1/world of the bytes
        out["roofline"]["frac"] = round(achieved / world / peak, 4)
        out["roofline"]["per_launch"] += f"; {world} GPUs, each reading about 1/{world} of it"
    out["roofline"]["traffic"] = traffic_from_profiles("decode", 1)
    if not args.no_cpu_baseline and world == 1:
        out["cpu_baseline"] = decode_cpu_baseline(path)
    print(json.dumps(out))
    return finish(world > 1)


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def decode_cpu_baseline(path, budget_s=15.0):
    """The reference's GEMV arithmetic as a host loop (oracle, OpenMP over
    rows) over the model file's own projections, layer after layer until
    ~budget_s pass, scaled to tokens/s for the step's 28 layers of projections
    plus the FP16 lm_head at the same bytes/s.  Attention and the small
    elementwise kernels are left out, so this is an upper bound on the host's
    token rate."""
    import oracle
    from atomflow_b200.weights_bin import BinFile
    L = oracle.cpu()
    L.af_oracle_gemv_cpu_baseline.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 2 + [ctypes.c_void_p, ctypes.c_int]
    b = BinFile(path)
    s = b.shape
    cores = os.cpu_count() or 1
    x = np.random.default_rng(1).standard_normal(max(s.dim, s.ffn)).astype(np.float16).view(np.uint16)
    y = np.empty(max(s.qkv_out, s.ffn), np.uint16)
    done_layers, nbytes, t0 = 0, 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        for name, N, K in s.linears():
            q, sc = b.linear(done_layers % s.n_layers, name)
            L.af_oracle_gemv_cpu_baseline(x.ctypes.data, q.ctypes.data, sc.ctypes.data, N, K, y.ctypes.data, cores)
            nbytes += algorithmic_bytes(N, K)
        done_layers += 1
    dt = time.perf_counter() - t0
    b.close()
    rate = nbytes / dt                                   # bytes/s of the host loop
    layer_b = sum(algorithmic_bytes(N, K) for _, N, K in s.linears())
    step_b = layer_b * s.n_layers + s.vocab * s.dim * 2  # projections + FP16 lm_head
    return {"value": round(rate / step_b, 3), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{done_layers} layer passes over the model file's 28 layers x 5 projections "
                      f"({nbytes / 1e9:.2f} GB algorithmic) in {dt:.1f} s on {cores} OpenMP threads "
                      f"({rate / 1e9:.2f} GB/s), scaled to one step's projections + lm_head; attention excluded"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="layerset")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--math", choices=["fast", "exact"], default="fast",
                    help="chain: tensor-core dot products (fast) or the reference kernel's FP32 FMA order (exact)")
    ap.add_argument("--launch", choices=["chain", "per-gemv"], default=None,
                    help="one-token GEMVs on one GPU: one persistent launch per step (chain; default for the "
                         "layer set) or one launch per GEMV (per-gemv; default elsewhere)")
    ap.add_argument("--order", choices=["dependent", "independent"], default="independent",
                    help="layer set as one chain launch: each GEMV waits for the previous one (dependent, the "
                         "order of the reference's launches) or not (independent: the layer set's GEMVs share no data)")
    ap.add_argument("--decode-mode", choices=["exact", "fast"], default="fast",
                    help="decode: kernels bit-identical to the reference's (exact) or the fused fast forms")
    ap.add_argument("--no-token-check", action="store_true",
                    help="decode: skip comparing 64 greedy tokens with the reference engine")
    ap.add_argument("--layers", type=int, default=NLAYERS,
                    help="layers of the layerset / layerchain workloads (default 28; fewer only for profiling)")
    ap.add_argument("--tp-comm", choices=["fused", "nccl"], default="fused",
                    help="N > 1: all-reduce of row-split outputs inside the GEMV kernel (fused) or by NCCL")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist_on = world > 1 and args.impl == "ours"
    if args.impl == "reference" and world > 1 and rank != 0:
        return 0                     # the reference arm runs on rank 0 alone
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if dist_on and args.impl == "ours":
        torch.distributed.init_process_group("nccl", device_id=device)
    tp = world if (dist_on and args.impl == "ours") else 1
    trank = rank if tp > 1 else 0

    wl = args.workload
    if wl == "decode":
        return run_decode(args, device, local)
    if wl == "layerset":
        items = make_layerset(device, trank, tp, layers=args.layers)
        config = {"workload": f"llama3.2-3b layer-set x{args.layers} (BASELINE config 1)", "M": 1,
                  "shapes": "qkv 5120x3072, o 3072x3072, gate/up 8192x3072, down 3072x8192",
                  "scales": "fp16 per 128-group (reference format)", "gemvs_per_step": len(items),
                  "weights_gb": round(sum(it["q"].numel() for it in items) * tp / 1e9, 3),
                  "l2": "inputs 2.8 GB >> 126 MB L2 (no flush needed)",
                  "parallelism": f"tp{tp}" if tp > 1 else "single"}
    elif wl == "layerset8b":
        nl = NLAYERS8 if args.layers == NLAYERS else args.layers
        items = make_layerset(device, trank, tp, layers=nl, proj=PROJ8)
        config = {"workload": f"llama3-8b-shaped layer-set x{nl} (BASELINE config 4, TP sharding)", "M": 1,
                  "shapes": "qkv 6144x4096, o 4096x4096, gate/up 14336x4096, down 4096x14336",
                  "scales": "fp16 per 128-group (reference format)", "gemvs_per_step": len(items),
                  "weights_gb": round(sum(it["q"].numel() for it in items) * tp / 1e9, 3),
                  "l2": "inputs >> 126 MB L2 (no flush needed)",
                  "parallelism": f"tp{tp}" if tp > 1 else "single"}
    elif wl == "layerchain":
        items, cbufs = make_layerchain(device, trank, tp, layers=args.layers)
        config = {"workload": f"llama3.2-3b decode layer without attention x{args.layers} (RMSNorm, QKV, O + residual, "
                              "RMSNorm, gate/up + SwiGLU, down + residual)", "M": 1,
                  "attention": "out of scope: O reads the first K_o entries of QKV in its place",
                  "scales": "fp16 per 128-group (reference format)", "layers": args.layers,
                  "l2": "inputs 2.8 GB >> 126 MB L2 (no flush needed)",
                  "parallelism": f"tp{tp}" if tp > 1 else "single"}
    elif wl.startswith("gemv:") or wl.startswith("gemmtc:"):
        parts = [int(v) for v in wl.split(":")[1:]]
        N, K = parts[0], parts[1]
        M = parts[2] if len(parts) > 2 else 1
        items = make_single(device, N, K, M)
        config = {"workload": f"single GEMV {N}x{K} M={M}" + (" (af_w8a16_gemm_tc)" if wl.startswith("gemmtc") else ""),
                  "M": M, "copies": len(items),
                  "l2": f"{len(items)} rotating weight copies ({len(items) * N * K / 1e6:.0f} MB) > 4x L2",
                  "parallelism": "single"}
    elif wl in ("lmhead:f16", "lmhead:fp8"):
        items = make_lmhead(device, wl.endswith("fp8"), trank, tp)
        config = {"workload": f"lm_head vocab projection 128256x3072 {wl.split(':')[1].upper()} + greedy argmax "
                              "(BASELINE config 2)", "M": 1,
                  "l2": "788 / 394 MB of weights >> 126 MB L2 (no flush needed)",
                  "parallelism": f"vocab-parallel tp{tp}" if tp > 1 else "single"}
    else:
        raise SystemExit(f"unknown workload {wl}")

    lm = wl.startswith("lmhead")
    chain = wl == "layerchain"
    # one token per GEMV on one GPU: the whole step as one persistent launch (af_gemv_chain)
    if args.launch is None:
        args.launch = "chain" if wl == "layerset" else "per-gemv"
    use_chain = (args.impl == "ours" and tp == 1 and not lm and args.launch == "chain" and
                 all(it["x"].shape[0] == 1 for it in items if not chain))
    exact = args.math == "exact"
    if use_chain:
        config["launch"] = ("one persistent launch per step, every GEMV waits for the previous one"
                            if args.order == "dependent" or chain else
                            "one persistent launch per step over the 140 independent GEMVs (no waits between them)")
        config["math"] = ("exact: the reference kernel's FP32 FMA order, bit-identical" if exact else
                          "fast: tensor-core MMAs, FP32 accumulation, within FP16 rounding of FP64")
    if chain:
        arm = OursChain(cbufs, as_chain=use_chain, exact=exact) if args.impl == "ours" else None
    elif use_chain:
        arm = OursChainSet(items, device, wait=args.order == "dependent", exact=exact)
    else:
        arm = ((OursLmHead(items, device) if lm else OursGemmTc(items, device) if wl.startswith("gemmtc") else
                OursGemv(items, device)) if args.impl == "ours" else None)
    if args.impl == "reference":
        try:
            if lm and wl.endswith("fp8"):
                raise FileNotFoundError("an FP8 lm_head (the reference's lm_head is FP16 cuBLAS only)")
            arm = RefChain(cbufs) if chain else (RefLmHead(items, device) if lm else RefGemv(items, device))
        except FileNotFoundError as e:
            print(json.dumps({"impl": "reference", "unavailable": f"no reference arm: {e}"}))
            return 0
    stream = torch.cuda.Stream(device)
    allreduce = None
    comm = None
    if tp > 1 and (lm or chain) and args.tp_comm == "nccl":
        raise SystemExit("the lm_head and layer-chain workloads exchange inside their kernels (--tp-comm fused)")
    if tp > 1 and args.tp_comm == "nccl":
        def allreduce(y):
            torch.distributed.all_reduce(y)
    elif tp > 1:
        # row-split projections: one kernel computes the partial GEMV and sums it
        # over the ranks through NVLink peer memory (af_w8a16_gemv_allreduce)
        from atomflow_b200.tp import TpComm
        comm = TpComm(trank, tp, D if chain else (max(it["N"] for it in items) if not lm else 64))
        arm.comm = comm

    step_bytes = (sum(lm_bytes(it) for it in items) if lm else chain_bytes(items, tp) if chain else
                  sum(algorithmic_bytes(it["N"], it["K"], it["x"].shape[0]) for it in items))
    total_bytes = step_bytes * tp
    sampler = ClockSampler(local) if rank == 0 else None
    reset = (lambda: cbufs["x"].copy_(cbufs["x0"])) if chain else None
    g = capture_step(arm, items, stream, allreduce, pre=reset)
    if sampler:
        sampler.wait_first()
    ms, t0, t1 = time_graph(g, stream, args.steps, args.warmup, dist_on)
    clocks = sampler.summary(t0, t1) if sampler else None
    ms_step = ms / args.steps
    value = total_bytes / (ms_step / 1e3) / 1e9
    if use_chain and not chain:
        # the same GEMVs as one launch each (the reference's launch pattern), for comparison
        gp = capture_step(OursGemv(items, device), items, stream)
        pms, _, _ = time_graph(gp, stream, args.steps, args.warmup, dist_on)
        gp = None
        pv = total_bytes / (pms / args.steps / 1e3) / 1e9
        peak_pg, _ = measured_peaks()
        config["per_gemv_launch"] = {"value": round(pv, 2), "unit": "GB/s", "ms_per_step": round(pms / args.steps, 5),
                                     "frac": round(pv / peak_pg, 4),
                                     "kernel": "gemv_fp8_m1_kernel, one launch per GEMV (af_w8a16_gemv)"}
    if use_chain:
        launches = args.steps            # one persistent launch per step
    else:
        launches = len(items) * args.steps * (arm.launches_per_layer if chain else 1)

    e2e = None
    if not args.no_e2e and chain:
        # End to end through the C ABI: each step takes the residual stream from
        # pinned host memory and returns it there (a decode step's real I/O).
        x_host = cbufs["x0"].cpu().pin_memory()
        x_back = torch.empty_like(x_host).pin_memory()
        ge = capture_step(arm, items, stream, allreduce, lambda: cbufs["x"].copy_(x_host, non_blocking=True),
                          lambda: x_back.copy_(cbufs["x"], non_blocking=True))
        ems, _, _ = time_graph(ge, stream, args.steps, args.warmup, dist_on)
        e2e = {"value": round(total_bytes / (ems / args.steps / 1e3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(ems / args.steps, 5), "h2d_bytes_per_step": int(x_host.numel() * 2),
               "d2h_bytes_per_step": int(x_back.numel() * 2),
               "path": ("af_gemv_chain (one launch)" if use_chain else "af_rmsnorm_w8a16_gemv / af_w8a16_gemv_residual / af_rmsnorm_w8a16_swiglu") + " C ABI; residual "
                       "stream pinned host -> device -> pinned host each step; CUDA graph"}
    elif not args.no_e2e:
        # End to end through the C ABI with host buffers: every step copies all
        # 140 activation vectors from pinned host memory, runs the GEMVs and
        # copies every output back; graph-captured like the reference's decode.
        xs_host = torch.cat([it["x"].reshape(-1) for it in items]).cpu().pin_memory()
        ys_n = sum(it["y"].numel() for it in items)
        ydt = items[0]["y"].dtype
        ys_host = torch.empty(ys_n, dtype=ydt).pin_memory()
        xs_dev = torch.empty_like(xs_host, device=device)
        ys_dev = torch.empty(ys_n, dtype=ydt, device=device)
        xo, yo = [], []
        ox = oy = 0
        for it in items:
            xo.append(ox)
            yo.append(oy)
            ox += it["x"].numel()
            oy += it["y"].numel()

        class E2E:
            def launch(self_, stream_, it):
                i = it["_i"]
                arm.launch(stream_, it, xs_dev[xo[i]:].data_ptr(), ys_dev[yo[i]:].data_ptr())

        if use_chain:
            def _all(stream_, items_):
                arm.launch_all(stream_, items_, [xs_dev[xo[i]:].data_ptr() for i in range(len(items_))],
                               [ys_dev[yo[i]:].data_ptr() for i in range(len(items_))])
            E2E.launch_all = lambda self_, stream_, items_: _all(stream_, items_)

        for i, it in enumerate(items):
            it["_i"] = i

        def pre():
            xs_dev.copy_(xs_host, non_blocking=True)

        def post():
            ys_host.copy_(ys_dev, non_blocking=True)

        ge = capture_step(E2E(), items, stream, allreduce, pre, post)
        ems, _, _ = time_graph(ge, stream, args.steps, args.warmup, dist_on)
        e2e = {"value": round(total_bytes / (ems / args.steps / 1e3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(ems / args.steps, 5),
               "h2d_bytes_per_step": int(xs_host.numel() * 2), "d2h_bytes_per_step": int(ys_n * ys_host.element_size()),
               "path": ("af_lm_head_gemv" if lm else "af_gemv_chain" if use_chain else "af_w8a16_gemv") +
                       " C ABI; pinned-host x -> device, every GEMV of the step, outputs -> pinned host; CUDA graph"}
    if sampler:
        sampler.stop()
    if comm is not None and comm.status() != 0:
        raise RuntimeError("af_w8a16_gemv_allreduce: a peer wait ran out (status word set)")
    if tp > 1:
        config["tp_allreduce"] = (("argmax (max, index) pairs exchanged inside the lm_head kernel over NVLink"
                                   if lm else "fused into the GEMV over NVLink peer memory") if comm is not None
                                  else "NCCL all_reduce after the GEMV")

    g = ge = None          # graphs (and any NCCL work they captured) go before the process group
    torch.cuda.synchronize()
    if rank != 0:
        return finish(dist_on)

    peak, peak_kind = measured_peaks()
    per_rank_gbs = step_bytes / (ms_step / 1e3) / 1e9
    out = {
        "metric": ("lm_head vocab projection + argmax achieved HBM GB/s" if lm else
                   "decode-layer chain achieved HBM GB/s (Llama-3.2-3B, M=1, attention excluded)" if chain else
                   "W8A16 GEMV achieved HBM GB/s (Llama-3-8B-shaped layer-set stream, M=1)" if wl == "layerset8b" else
                   "W8A16 GEMV achieved HBM GB/s (Llama-3.2-3B layer-set stream, M=1)"),
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp8e4m3 weights x fp16 act, fp32 accum",
        "data": "synthetic seeded (W~N(0,0.02) quantised per BASELINE config 0 recipe, x~N(0,1))",
        "config": config,
        "roofline": {"bound": "hbm", "achieved": round(per_rank_gbs, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(per_rank_gbs / peak, 4), "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                     if peak_kind == "measured" else "fallback 6.65 TB/s",
                     "traffic": traffic_from_profiles("layerset_chain" if use_chain and wl == "layerset" else wl, len(items))
                     if args.impl == "ours" else None,
                     "kernel": ({"ours": "gemv_stream_kernel (FP16 W) / gemv_fp8_m1_kernel (FP8 W)",
                                 "reference": "cublasGemmEx + argmax (reference)"} if lm else
                                {"ours": f"chain_kernel<{'exact' if exact else 'fast'}> (one persistent launch per step)" if use_chain
                                 else "chain_kernel / gemv_fp8_m1_kernel (one launch per GEMV)",
                                 "reference": "w8a16_gemv_kernel (reference)"})[args.impl],
                     "per_launch": f"{step_bytes / (launches / args.steps) / 1e6:.2f} MB avg algorithmic bytes / launch "
                                   f"over {ms_step * 1e3 / (launches / args.steps):.2f} us avg launch (CUDA events "
                                   f"over the timed region)"},
        "gpu_launches": launches if args.impl == "ours" else 0,
        "clocks": clocks,
    }
    if args.impl == "ours":
        out["e2e"] = e2e
        if not args.no_cpu_baseline and world == 1 and wl == "layerset":
            out["cpu_baseline"] = cpu_baseline(items)
    else:
        out["impl"] = "reference"
        out["e2e"] = {"value": out["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
        out["cpu_baseline"] = {"value": out["value"], "unit": "GB/s", "cores": None, "kind": "reference",
                               "sample": "full workload; the reference's path is CUDA (src/kernel/qkv_gemm.cu "
                                         "w8a16_gemv_kernel, compiled from its sources), run on this GPU"}
        out["reference_kernel_launches"] = launches * (items[0]["x"].shape[0] if wl.startswith("gemv:") else 1)
    print(json.dumps(out))
    return finish(dist_on)


def finish(dist_on):
    """Normal exit: all ranks meet at a barrier (no rank leaves with work in
    flight), then the process group is destroyed and main returns."""
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
        torch.cuda.synchronize()
        torch.distributed.destroy_process_group()
    sys.stdout.flush()
    sys.stderr.flush()
    return 0


def traffic_from_profiles(workload, launches_per_step):
    """DRAM bytes (read + write) per launch from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(workload)
    except Exception:
        return None


if __name__ == "__main__":
    sys.exit(main())
