"""bench.py's byte accounting -- the numerator of every GB/s it reports --
against the algorithmic figures of the path: W + scales + x + y per GEMV."""
import importlib.util
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_gemv_bytes():
    b = _bench()
    # 8192 x 3072 FP8 + FP16 group scales + x + y
    assert b.algorithmic_bytes(8192, 3072) == 8192 * 3072 + 8192 * 24 * 2 + 3072 * 2 + 8192 * 2 == 25_581_568
    assert b.algorithmic_bytes(3072, 8192) == 25_581_568
    # row scales: 4 bytes per row; M tokens: M rows of x and y
    assert b.algorithmic_bytes(3072, 3072, 1, "row") == 3072 * 3072 + 3072 * 4 + 3072 * 2 * 2
    assert b.algorithmic_bytes(3072, 3072, 8) - b.algorithmic_bytes(3072, 3072, 1) == 7 * (3072 * 2 * 2)


def test_layer_set_step_bytes():
    b = _bench()
    per_layer = sum(b.algorithmic_bytes(n, k) for _, n, k, _ in b.PROJ)
    step = per_layer * b.NLAYERS
    # 2.819 GB of FP8 weights + 44.0 MB of scales + activations ~ 2.865 GB per step
    assert 2.86e9 < step < 2.87e9
    fp8 = sum(n * k for _, n, k, _ in b.PROJ) * b.NLAYERS
    assert fp8 == 2_818_572_288


def test_lm_head_bytes():
    b = _bench()
    it16 = {"N": 128256, "K": 3072, "fp8": False}
    it8 = {"N": 128256, "K": 3072, "fp8": True}
    assert b.lm_bytes(it16) == 128256 * 3072 * 2 + 3072 * 2 + 128256 * 4   # 788.5 MB
    assert b.lm_bytes(it8) == 128256 * 3072 + 128256 * 4 + 3072 * 2 + 128256 * 4
