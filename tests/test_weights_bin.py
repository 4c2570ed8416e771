"""The random-init `.bin` writer/reader (atomflow_b200.weights_bin) against the
reference's file layout: block offsets pinned by the reference's own weight
loader (tests/golden/bin_layout_tiny.json, made by make_golden_bin_layout.py),
header fields, zero padding, and value round trips."""
import json
import struct
from pathlib import Path

import numpy as np
import pytest
import torch

from atomflow_b200.weights_bin import BinFile, ModelShape, block_plan, tensor_values, write_synthetic_bin

GOLD = json.loads((Path(__file__).parent / "golden" / "bin_layout_tiny.json").read_text())
TINY = ModelShape(**GOLD["shape"])


def test_offsets_match_the_reference_loader(tmp_path):
    plan, total = block_plan(TINY)
    starts = [p[3] for p in plan]
    # the reference walker marks the cursor after the header and after every block
    assert [256] + [s for s in starts[1:]] + [total] == GOLD["offsets"]
    size = write_synthetic_bin(tmp_path / "m.bin", TINY, seed=3)
    assert size == total == GOLD["file_size"] == (tmp_path / "m.bin").stat().st_size


def test_header_and_padding(tmp_path):
    p = tmp_path / "m.bin"
    write_synthetic_bin(p, TINY, seed=1)
    raw = p.read_bytes()
    assert raw[:4] == b"ATOM"
    assert list(struct.unpack_from("<9i", raw, 4)) == GOLD["header"]
    assert raw[40:256] == b"\0" * 216
    plan, _ = block_plan(TINY)
    for name, dtype, dims, off, nbytes in plan:
        assert off % 256 == 0
        end = off + nbytes
        pad_end = (end + 255) // 256 * 256
        assert raw[end:pad_end] == b"\0" * (pad_end - end), name


def test_values_round_trip_and_quantisation(tmp_path):
    p = tmp_path / "m.bin"
    write_synthetic_bin(p, TINY, seed=5)
    b = BinFile(p)
    assert b.shape == TINY
    np.testing.assert_array_equal(b.block("embed"), tensor_values(TINY, "embed", 5))
    np.testing.assert_array_equal(b.block("lm_head"), tensor_values(TINY, "lm_head", 5))
    # FP16-valued norms and embedding: FP32 and FP16 readings agree
    e = b.block("embed")
    assert np.array_equal(e, e.astype(np.float16).astype(np.float32))
    n = b.block("layers.1.post_norm")
    assert np.array_equal(n, n.astype(np.float16).astype(np.float32)) and abs(n.mean() - 1) < 0.05
    for name, nn, k in TINY.linears():
        q, s = b.linear(1, name)
        assert q.shape == (nn, k) and s.shape == (nn, k // 128)
        q0, s0 = tensor_values(TINY, f"layers.1.{name}", 5)
        np.testing.assert_array_equal(q, q0)
        np.testing.assert_array_equal(s, s0)
        # dequantised weights are the N(0, 0.02) draw within E4M3 rounding
        w = torch.from_numpy(q.copy()).view(torch.float8_e4m3fn).float().view(nn, k // 128, 128)
        w = (w * torch.from_numpy(s.view(np.float16).astype(np.float32))[..., None]).view(nn, k)
        assert 0.015 < float(w.std()) < 0.025
    b.close()


def test_default_shape_is_llama_3_2_3b():
    s = ModelShape()
    assert (s.qkv_out, s.head_dim) == (5120, 128)
    _, total = block_plan(s)
    # 2.82 GB FP8 + 44 MB scales + FP32 embedding 1.58 GB + FP16 lm_head 0.79 GB + norms
    assert 5.2e9 < total < 5.3e9


@pytest.mark.gpu
def test_file_weights_feed_the_gemv(tmp_path):
    """Layer 0's projections, read from a written file, through af_w8a16_gemv."""
    import oracle
    from atomflow_b200 import lib
    from tests._util import assert_fp16_parity, fp16_bits, normal_f32
    shape = ModelShape(dim=1024, ffn=2048, n_layers=1, n_heads=8, n_kv_heads=2, vocab=512, max_seq_len=64)
    p = tmp_path / "m.bin"
    write_synthetic_bin(p, shape, seed=9)
    b = BinFile(p)
    L = lib()
    for name, n, k in shape.linears():
        q, s = b.linear(0, name)
        x = fp16_bits(normal_f32(n + k, (1, k)))
        xd = torch.from_numpy(x.view(np.int16)).cuda()
        qd = torch.from_numpy(q.copy()).cuda()
        sd = torch.from_numpy(s.view(np.int16).copy()).cuda()
        y = torch.zeros(n, dtype=torch.int16, device="cuda")
        assert L.af_w8a16_gemv(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), y.data_ptr(), 1, n, k, 128, 0, None, 0,
                               torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert_fp16_parity(y.cpu().numpy().view(np.uint16), oracle.gemv_f64(x, q, s, "group", with_l2=True),
                           f"file layer 0 {name}")
    b.close()

