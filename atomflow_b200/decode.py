"""A greedy decode step on this library's kernels, for models in the
reference's `.bin` format.

Mirrors the reference engine's interface (include/core/engine.h:
initialize / inject_token / forward_pass / get_output_token / current_pos)
and its order of work (src/core/engine.cu:262-521), with the layer's
element-wise work fused into the projections:

  embedding lookup                        af_embed_lookup
  per layer:
    RMSNorm + QKV                         af_rmsnorm_w8a16_gemv
    RoPE + KV-cache write + attention     af_decode_rope_attention
    O + residual                          af_w8a16_gemv_residual
    RMSNorm + gate/up + SwiGLU            af_rmsnorm_w8a16_swiglu
    down + residual                       af_w8a16_gemv_residual
  final RMSNorm                           af_rmsnorm
  lm_head (FP16) + greedy argmax          af_lm_head_gemv

The token id and the position are device ints: `forward_pass` launches one
step eagerly; `capture()` records one step (optionally followed by the
position increment) as a CUDA graph whose replays generate token after token
without the host.  The argmax is the reference's (ids < 65536, its
launch_argmax behaviour) unless `true_argmax` is set.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from ._lib import check, lib
from .weights_bin import BinFile

NORM_EPS = 1e-5
ROPE_BASE = 500000.0
MAX_SEQ_LEN = 4096   # KV-cache rows: BASELINE config 3 (the reference engine has 2048, engine.h:41)


class DecodeEngine:
    def __init__(self, path, device="cuda", max_seq_len=MAX_SEQ_LEN, true_argmax=False):
        self.L = lib()
        self.dev = torch.device(device)
        self.mode = 0 if true_argmax else 1
        b = BinFile(path)
        s = self.shape = b.shape
        self.D, self.FFN, self.V, self.NL = s.dim, s.ffn, s.vocab, s.n_layers
        self.NH, self.NKV, self.HD = s.n_heads, s.n_kv_heads, s.head_dim
        self.QD, self.KVD = self.NH * self.HD, self.NKV * self.HD
        self.max_seq = max_seq_len

        def up(a, dt=None):
            t = torch.from_numpy(np.ascontiguousarray(a))
            if dt is not None:
                t = t.view(dt)
            return t.to(self.dev)

        self.embed = up(b.block("embed"))
        self.layers = []
        for i in range(self.NL):
            ly = {"in_norm": up(b.block(f"layers.{i}.input_norm")), "post_norm": up(b.block(f"layers.{i}.post_norm"))}
            for name, _, _ in s.linears():
                q, sc = b.linear(i, name)
                ly[name] = (up(q), up(sc.view(np.int16)))
            ly["k_cache"] = torch.zeros(max_seq_len, self.KVD, dtype=torch.float16, device=self.dev)
            ly["v_cache"] = torch.zeros(max_seq_len, self.KVD, dtype=torch.float16, device=self.dev)
            self.layers.append(ly)
        self.final_norm = up(b.block("final_norm"))
        self.lm_head = up(b.block("lm_head").view(np.int16))
        b.close()

        cos = np.empty((max_seq_len, self.HD // 2), np.float32)
        sin = np.empty_like(cos)
        check(self.L.af_rope_tables(cos.ctypes.data_as(ctypes.c_void_p), sin.ctypes.data_as(ctypes.c_void_p),
                                    max_seq_len, self.HD, ROPE_BASE), "af_rope_tables")
        self.cos, self.sin = up(cos), up(sin)

        z = lambda n, dt=torch.float16: torch.zeros(n, dtype=dt, device=self.dev)  # noqa: E731
        self.x, self.xn = z(self.D), z(self.D)
        self.qkv, self.attn = z(self.QD + 2 * self.KVD), z(self.QD)
        self.h = z(self.FFN)
        self.logits = z(self.V, torch.float32)
        self.d_token = z(1, torch.int32)
        self.d_pos = z(1, torch.int32)
        aw = self.L.af_decode_attention_workspace_bytes(self.NH, self.NKV, max_seq_len)
        self.attn_ws = z(aw, torch.uint8)
        lw = self.L.af_lm_head_workspace_bytes(self.V, self.D, 0)
        self.lm_ws = z(lw, torch.uint8)
        self.stream = torch.cuda.Stream(self.dev)
        self.stream.wait_stream(torch.cuda.current_stream(self.dev))   # the uploads above

    # ---- the reference engine's interface
    # (host reads and writes of the device ints go through the engine's stream,
    # so they are ordered with the steps)
    @property
    def current_pos(self) -> int:
        self.stream.synchronize()
        return int(self.d_pos.item())

    @current_pos.setter
    def current_pos(self, p: int):
        if not 0 <= p < self.max_seq:
            raise ValueError(f"position {p} outside the KV cache (max {self.max_seq})")
        with torch.cuda.stream(self.stream):
            self.d_pos.fill_(p)

    def inject_token(self, token: int):
        with torch.cuda.stream(self.stream):
            self.d_token.fill_(int(token))

    def get_output_token(self) -> int:
        self.stream.synchronize()
        return int(self.d_token.item())

    def forward_pass(self):
        with torch.cuda.stream(self.stream):
            self._launch_step(self.stream.cuda_stream, advance=False)

    def capture(self, advance=True) -> torch.cuda.CUDAGraph:
        """One step (plus the position increment when `advance`) as a CUDA graph."""
        self.forward_pass()   # first calls on the device happen outside capture
        self.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self._launch_step(self.stream.cuda_stream, advance=advance)
        return g

    def replay(self, g: torch.cuda.CUDAGraph):
        """Replay a captured step on the engine's stream (CUDAGraph.replay
        alone would launch on torch's current stream, unordered with the
        engine's token and position writes)."""
        with torch.cuda.stream(self.stream):
            g.replay()

    launches_per_step = None   # set on the first step

    # ---- one step
    def _launch_step(self, st, advance):
        L, p = self.L, (lambda t: t.data_ptr())
        n = 0
        check(L.af_embed_lookup(p(self.embed), p(self.d_token), p(self.x), self.D, st), "af_embed_lookup")
        n += 1
        for ly in self.layers:
            wq, sq = ly["qkv"]
            check(L.af_rmsnorm_w8a16_gemv(p(self.x), p(ly["in_norm"]), NORM_EPS, p(wq), p(sq), p(self.qkv),
                                          self.QD + 2 * self.KVD, self.D, 128, 0, None, st), "rmsnorm_gemv")
            check(L.af_decode_rope_attention(p(self.qkv), p(self.cos), p(self.sin), p(self.d_pos), p(ly["k_cache"]),
                                             p(ly["v_cache"]), p(self.attn), self.NH, self.NKV, self.HD, self.max_seq,
                                             p(self.attn_ws), self.attn_ws.numel(), st), "rope_attention")
            wo, so = ly["o"]
            check(L.af_w8a16_gemv_residual(p(self.attn), p(wo), p(so), p(self.x), self.D, self.QD, 128, 0, None, st),
                  "o + residual")
            (wg, sg), (wu, su) = ly["gate"], ly["up"]
            check(L.af_rmsnorm_w8a16_swiglu(p(self.x), p(ly["post_norm"]), NORM_EPS, p(wg), p(sg), p(wu), p(su),
                                            p(self.h), self.FFN, self.D, 128, 0, None, None, st), "rmsnorm_swiglu")
            wd, sd = ly["down"]
            check(L.af_w8a16_gemv_residual(p(self.h), p(wd), p(sd), p(self.x), self.D, self.FFN, 128, 0, None, st),
                  "down + residual")
            n += 5
        check(L.af_rmsnorm(p(self.x), p(self.final_norm), NORM_EPS, p(self.xn), self.D, st), "final rmsnorm")
        check(L.af_lm_head_gemv(p(self.xn), p(self.lm_head), 0, None, p(self.logits), self.V, self.D,
                                p(self.d_token), self.mode, p(self.lm_ws), self.lm_ws.numel(), st), "lm_head")
        n += 2
        if advance:
            check(L.af_decode_advance(p(self.d_pos), 1, st), "advance")
            n += 1
        self.launches_per_step = n

    def weight_bytes(self) -> int:
        """Bytes a step must read at least: every weight, scale and norm, the
        embedding row, and the KV cache up to the current position."""
        s = self.shape
        b = sum(n * k + n * (k // 128) * 2 for _, n, k in s.linears()) * self.NL
        b += (2 * self.D * 4) * self.NL + self.D * 4 + self.V * self.D * 2 + self.D * 4
        return b

    def kv_bytes(self, pos: int) -> int:
        return 2 * (pos + 1) * self.KVD * 2 * self.NL
