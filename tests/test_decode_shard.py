"""Tensor-parallel sharding of a decode layer (atomflow_b200.decode.shard_linear):
the ranks' shards reassemble every projection exactly, QKV shards keep whole
heads ([Q_r | K_r | V_r]) and K-splits keep whole 128-wide scale groups."""
import numpy as np
import pytest

from atomflow_b200.decode import shard_linear
from atomflow_b200.weights_bin import ModelShape

SHAPE = ModelShape(dim=1024, ffn=2048, n_layers=1, n_heads=8, n_kv_heads=4, vocab=1000, max_seq_len=64)


def _fake(n, k, seed):
    rng = np.random.default_rng(seed)
    return rng.integers(0, 255, (n, k), dtype=np.uint8), rng.integers(0, 60000, (n, k // 128), dtype=np.uint16)


@pytest.mark.parametrize("world", [2, 4])
def test_shards_reassemble(world):
    hd, nh, nkv = SHAPE.head_dim, SHAPE.n_heads, SHAPE.n_kv_heads
    for name, n, k in SHAPE.linears():
        q, s = _fake(n, k, n + k)
        parts = [shard_linear(name, q, s, SHAPE, r, world) for r in range(world)]
        if name == "qkv":
            hq, hk = nh // world, nkv // world
            for r, (qr, sr) in enumerate(parts):
                assert qr.shape == ((hq + 2 * hk) * hd, k) and sr.shape == (qr.shape[0], k // 128)
                np.testing.assert_array_equal(qr[:hq * hd], q[r * hq * hd:(r + 1) * hq * hd])
                np.testing.assert_array_equal(qr[hq * hd:(hq + hk) * hd], q[nh * hd + r * hk * hd:nh * hd + (r + 1) * hk * hd])
                np.testing.assert_array_equal(qr[(hq + hk) * hd:], q[(nh + nkv) * hd + r * hk * hd:(nh + nkv) * hd + (r + 1) * hk * hd])
            # every row of the full matrix appears in exactly one rank's shard
            assert sum(p[0].shape[0] for p in parts) == n
        elif name in ("gate", "up"):
            np.testing.assert_array_equal(np.concatenate([p[0] for p in parts]), q)
            np.testing.assert_array_equal(np.concatenate([p[1] for p in parts]), s)
        else:
            np.testing.assert_array_equal(np.concatenate([p[0] for p in parts], axis=1), q)
            np.testing.assert_array_equal(np.concatenate([p[1] for p in parts], axis=1), s)
            for qr, sr in parts:
                assert qr.shape[1] % 128 == 0 and sr.shape[1] == qr.shape[1] // 128


def test_o_split_follows_the_heads():
    # O's K dims of rank r are exactly the output dims of its query heads
    world, hd = 2, SHAPE.head_dim
    q, s = _fake(SHAPE.dim, SHAPE.n_heads * hd, 3)
    q0, _ = shard_linear("o", q, s, SHAPE, 0, world)
    np.testing.assert_array_equal(q0, q[:, :SHAPE.n_heads // world * hd])


def test_unsplittable_models_are_rejected():
    q, s = _fake(1024, 1024, 1)
    with pytest.raises(ValueError):
        shard_linear("qkv", q, s, ModelShape(dim=1024, ffn=2048, n_heads=8, n_kv_heads=2), 0, 4)  # 2 kv heads / 4
