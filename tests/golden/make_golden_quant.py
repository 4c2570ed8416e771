"""Generate tests/golden/quant_gs128.npz from the REFERENCE's own quantiser.

Imports quantize_fp8_gs128 from the reference checkout (tools/quantize_weights.py
:220-268) and records its output on seeded inputs, so the CPU tests can pin the
oracle's and the library's quantisers to it without the reference present.

    python tests/golden/make_golden_quant.py [/path/to/reference]
"""
import sys
from pathlib import Path

import numpy as np
import torch

REF = Path(sys.argv[1]) if len(sys.argv) > 1 else sys.exit("usage: make_golden_quant.py <reference checkout>")
sys.path.insert(0, str(REF / "tools"))
from quantize_weights import quantize_fp8_gs128  # noqa: E402

OUT = Path(__file__).resolve().parent / "quant_gs128.npz"


def case(seed, N, K, std):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * std
    if seed == 2:          # an all-zero group and a clamp-edge value
        w[0, :128] = 0.0
        w[1, 5] = 3.0
    q, s = quantize_fp8_gs128(w)
    return (w.numpy().astype(np.float32), np.frombuffer(q, np.uint8).reshape(N, K).copy(),
            np.frombuffer(s, np.uint16).reshape(N, K // 128).copy())


arrays = {}
for i, (seed, N, K, std) in enumerate([(0, 16, 256, 0.02), (1, 7, 384, 1.0), (2, 5, 640, 0.05)]):
    w, q, s = case(seed, N, K, std)
    arrays[f"w{i}"], arrays[f"q{i}"], arrays[f"s{i}"] = w, q, s
np.savez_compressed(OUT, **arrays)
print(OUT, {k: v.shape for k, v in arrays.items()})
