"""Random-init model files in the reference's `.bin` weight format.

The reference engine loads one file (tools/quantize_weights.py:320-427 writes
it; include/memory/weight_loader.h:19-30,91-99 and src/core/engine.cu:103-147
read it).  Without the real checkpoint, a decode step on the reference engine
needs a file of the same layout with seeded random weights; this module writes
one and reads any such file back.

Layout (little-endian; every block padded to a multiple of 256 bytes):
  header, 256 bytes: "ATOM", version 1, group size 128, dim, ffn, n_layers,
      n_heads, n_kv_heads, vocab, max_seq_len (int32 each), zero padding
  embedding          FP32 [vocab, dim]
  per layer:         input norm FP32 [dim], post-attention norm FP32 [dim],
                     then for qkv [(n_heads + 2 n_kv) * head_dim, dim], o [dim, dim],
                     gate [ffn, dim], up [ffn, dim], down [dim, ffn]:
                     FP8-E4M3 weights, then FP16 group scales [N, K/128]
  final norm         FP32 [dim]
  lm_head            FP16 [vocab, dim]

Values: linear weights N(0, 0.02) quantised per 128-wide
group exactly as the reference exporter does (atomflow_b200.quant); the
embedding, norms and lm_head are FP16 values (embedding and lm_head N(0,
0.02), norms 1 + N(0, 0.1) rounded to FP16), stored as FP32 where the format
wants FP32, so FP16 and FP32 readings agree.  Every tensor has its own seed,
so the file is reproducible block by block.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from .quant import GROUP, quantize_gs128

ALIGN = 256
MAGIC = b"ATOM"


@dataclass(frozen=True)
class ModelShape:
    dim: int = 3072
    ffn: int = 8192
    n_layers: int = 28
    n_heads: int = 24
    n_kv_heads: int = 8
    vocab: int = 128256
    max_seq_len: int = 4096

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @property
    def qkv_out(self) -> int:
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim

    def linears(self):
        """(name, N, K) of a layer's five projections, in file order."""
        d, f = self.dim, self.ffn
        return [("qkv", self.qkv_out, d), ("o", d, d), ("gate", f, d), ("up", f, d), ("down", d, f)]


def _pad(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def block_plan(shape: ModelShape):
    """[(name, dtype, shape, offset, nbytes)] of every block, in file order --
    the offsets weight_loader.h's next_block() arrives at."""
    plan, off = [], ALIGN

    def add(name, dtype, dims):
        nonlocal off
        nbytes = int(np.prod(dims)) * np.dtype(dtype).itemsize
        plan.append((name, dtype, tuple(dims), off, nbytes))
        off += _pad(nbytes)

    add("embed", np.float32, (shape.vocab, shape.dim))
    for i in range(shape.n_layers):
        add(f"layers.{i}.input_norm", np.float32, (shape.dim,))
        add(f"layers.{i}.post_norm", np.float32, (shape.dim,))
        for name, n, k in shape.linears():
            add(f"layers.{i}.{name}", np.uint8, (n, k))
            add(f"layers.{i}.{name}_scales", np.uint16, (n, k // GROUP))
    add("final_norm", np.float32, (shape.dim,))
    add("lm_head", np.uint16, (shape.vocab, shape.dim))
    return plan, off


def _header(shape: ModelShape) -> bytes:
    h = struct.pack("<4sii7i", MAGIC, 1, GROUP, shape.dim, shape.ffn, shape.n_layers, shape.n_heads,
                    shape.n_kv_heads, shape.vocab, shape.max_seq_len)
    return h + b"\0" * (ALIGN - len(h))


def _rng(seed: int, tag: str, device="cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + sum((i + 1) * ord(ch) for i, ch in enumerate(tag))) % (2**63))
    return g


def tensor_values(shape: ModelShape, name: str, seed: int = 0, device="cpu"):
    """The values written for block `name` (numpy, in the stored dtype); a
    linear weight and its scales come together from `name` = layers.i.proj.
    The draw depends on the generating device (device="cuda" is much faster
    for full-size files); a given (seed, device) always gives the same file."""
    g = _rng(seed, name, device)
    kw = dict(generator=g, device=device)
    if name in ("embed", "lm_head"):
        v = (torch.randn(shape.vocab, shape.dim, **kw) * 0.02).half().cpu()
        return v.float().numpy() if name == "embed" else v.view(torch.int16).numpy().view(np.uint16)
    if name.endswith("norm"):
        return (1.0 + 0.1 * torch.randn(shape.dim, **kw)).half().float().cpu().numpy()
    proj = name.split(".")[-1]
    n, k = {nm: (n, k) for nm, n, k in shape.linears()}[proj]
    q, s = quantize_gs128(torch.randn(n, k, **kw) * 0.02)
    return q.view(torch.uint8).cpu().numpy(), s.view(torch.int16).cpu().numpy().view(np.uint16)


def write_synthetic_bin(path, shape: ModelShape = ModelShape(), seed: int = 0, device="cpu") -> int:
    """Write a random-init model file; returns its size in bytes."""
    plan, total = block_plan(shape)
    path = Path(path)
    with open(path, "wb") as f:
        f.write(_header(shape))
        for name, dtype, dims, off, nbytes in plan:
            if name.endswith("_scales"):
                continue   # written together with its weights
            assert f.tell() == off, (name, f.tell(), off)
            v = tensor_values(shape, name, seed, device)
            blobs = v if isinstance(v, tuple) else (v,)
            for b in blobs:
                raw = np.ascontiguousarray(b).tobytes()
                f.write(raw)
                f.write(b"\0" * (_pad(len(raw)) - len(raw)))
        assert f.tell() == total
    return total


def synthetic_model_file(shape: ModelShape = ModelShape(), seed: int = 0, directory=None) -> Path:
    """A random-init model file of `shape`, written once (values drawn on the
    GPU) under `directory` (default: the system temp dir, or $AF_MODEL_DIR)
    and reused by later calls with the same shape and seed."""
    import os
    import tempfile
    d = Path(directory or os.environ.get("AF_MODEL_DIR") or tempfile.gettempdir())
    tag = "-".join(str(v) for v in (shape.dim, shape.ffn, shape.n_layers, shape.n_heads, shape.n_kv_heads,
                                    shape.vocab, shape.max_seq_len))
    path = d / f"af_synthetic_{tag}_seed{seed}.bin"
    if not path.exists() or path.stat().st_size != block_plan(shape)[1]:
        tmp = path.with_suffix(f".part{os.getpid()}")
        write_synthetic_bin(tmp, shape, seed=seed, device="cuda")
        os.replace(tmp, path)
    return path


class BinFile:
    """Read-only view of a `.bin` model file (mmap), block by block."""

    def __init__(self, path):
        self._f = open(path, "rb")
        self._m = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        magic, version, gs, *dims = struct.unpack_from("<4sii7i", self._m, 0)
        if magic != MAGIC:
            raise ValueError("not an AtomFlow .bin file (magic)")
        if version != 1 or gs != GROUP:
            raise ValueError(f"unsupported .bin version {version} / group size {gs}")
        self.shape = ModelShape(*dims)
        self.plan, self.expected_size = block_plan(self.shape)
        if len(self._m) < self.expected_size:
            raise ValueError(f"file has {len(self._m)} bytes, the layout needs {self.expected_size}")
        self._index = {p[0]: p for p in self.plan}

    def block(self, name: str) -> np.ndarray:
        _, dtype, dims, off, nbytes = self._index[name]
        return np.frombuffer(self._m, dtype=dtype, count=nbytes // np.dtype(dtype).itemsize,
                             offset=off).reshape(dims)

    def linear(self, layer: int, proj: str):
        """(FP8 weights uint8 [N, K], FP16 group scales as uint16 bits [N, K/128])."""
        return self.block(f"layers.{layer}.{proj}"), self.block(f"layers.{layer}.{proj}_scales")

    def close(self):
        """Release the file.  While arrays returned by block() are alive the
        mapping stays open and is released with the last of them."""
        try:
            self._m.close()
        except BufferError:
            pass
        self._f.close()


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description="write a random-init AtomFlow .bin model file")
    ap.add_argument("path")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--layers", type=int, default=28)
    a = ap.parse_args()
    size = write_synthetic_bin(a.path, ModelShape(n_layers=a.layers), a.seed)
    print(f"{a.path}: {size / 2**30:.2f} GiB")
