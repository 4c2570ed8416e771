"""Offline weight quantisation into the formats the kernels consume.

Follows the reference exporter, tools/quantize_weights.py:220-268
(quantize_fp8_gs128): per 128-wide group along K, scale = absmax/448 (1 for an
all-zero group) in FP32, q = float8_e4m3fn(clamp(w/scale, +-448)) with
round-to-nearest-even, scale stored as FP16.  `quantize_row` is the
per-output-row FP32-scale variant.  Runs on any torch device, so benchmark
weights can be made on the GPU.
"""
import torch

FP8_MAX = 448.0
GROUP = 128


def quantize_gs128(w: torch.Tensor):
    """w [N, K] float -> (q float8_e4m3fn [N, K], scales float16 [N, K/128])."""
    t = w.detach().float()
    N, K = t.shape
    if K % GROUP:
        raise ValueError(f"K={K} is not a multiple of {GROUP}")
    tg = t.view(N, K // GROUP, GROUP)
    mx = tg.abs().amax(dim=2)
    sc = torch.where(mx > 0, mx / FP8_MAX, torch.ones_like(mx))
    q = (tg / sc.unsqueeze(2)).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.view(N, K), sc.to(torch.float16)


def quantize_row(w: torch.Tensor):
    """w [N, K] float -> (q float8_e4m3fn [N, K], scales float32 [N])."""
    t = w.detach().float()
    mx = t.abs().amax(dim=1)
    sc = torch.where(mx > 0, mx / FP8_MAX, torch.ones_like(mx))
    q = (t / sc.unsqueeze(1)).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q, sc
