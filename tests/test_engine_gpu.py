"""The C++ decode engine (af_engine_*) and its command-line driver af_generate.

  * exact mode: greedy tokens identical to the reference's own AtomFlowEngine
    (compiled from its sources into oracle/_ref) on a random-init model file,
    teacher-forced positions and free greedy steps alike -- every kernel of
    the step is bit-identical to the reference's, so identity is guaranteed,
    not likely;
  * fast mode: its logits within FP16-level rounding of the exact mode's;
  * af_generate (C++, no Python in the loop) emits the same tokens as the engine
    driven through the Python front and as the reference engine;
  * bad model files and out-of-range positions are rejected.
"""
import ctypes
import subprocess

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

PROMPT, GREEDY = 16, 48


@pytest.fixture(scope="module")
def tiny_model(tmp_path_factory):
    from atomflow_b200.weights_bin import ModelShape, write_synthetic_bin
    shape = ModelShape(dim=1024, ffn=2048, n_layers=4, n_heads=8, n_kv_heads=2, vocab=128256, max_seq_len=2048)
    path = tmp_path_factory.mktemp("engine") / "tiny.bin"
    write_synthetic_bin(path, shape, seed=33, device="cuda")
    return path


def _prompt():
    return np.random.default_rng(9).integers(0, 65536, PROMPT).tolist()


def _engine_tokens(path, mode):
    from atomflow_b200.decode import DecodeEngine
    eng = DecodeEngine(path, mode=mode, max_seq_len=2048)
    eng.capture(advance=True)
    eng.current_pos = 0
    toks = []
    for p in range(PROMPT + GREEDY):
        if p < PROMPT:
            eng.inject_token(_prompt()[p])
        eng.replay()
        toks.append(eng.get_output_token())
    eng.close()
    return toks


def _reference_tokens(path):
    R = oracle.ref_engine()
    if R is None:
        pytest.skip("oracle/_ref/libafref_engine.so not built")
    h = R.afref_engine_create(str(path).encode())
    toks, tok = [], None
    for p in range(PROMPT + GREEDY):
        tok = R.afref_engine_step(h, _prompt()[p] if p < PROMPT else tok, p)
        toks.append(tok)
    R.afref_engine_destroy(h)
    return toks


def test_exact_engine_tokens_identical_to_reference(tiny_model):
    assert _engine_tokens(tiny_model, "exact") == _reference_tokens(tiny_model)


def test_fast_engine_logits_close_to_exact(tiny_model):
    from atomflow_b200.decode import DecodeEngine
    out = {}
    for mode in ("exact", "fast"):
        eng = DecodeEngine(tiny_model, mode=mode, max_seq_len=2048)
        eng.current_pos = 0
        for p in range(8):
            eng.inject_token(_prompt()[p])
            eng.current_pos = p
            eng.forward_pass()
        eng.synchronize()
        lg = np.empty(eng.V, np.float32)
        cudart = ctypes.CDLL("libcudart.so.12")
        assert cudart.cudaMemcpy(lg.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(eng.logits_ptr),
                                 ctypes.c_size_t(lg.nbytes), 2) == 0
        out[mode] = lg
        eng.close()
    a, b = out["fast"].astype(np.float64), out["exact"].astype(np.float64)
    rms = np.sqrt(np.mean(b ** 2))
    assert np.abs(a - b).max() <= 2e-2 * rms, (np.abs(a - b).max(), rms)


def test_af_generate_cli_matches_engine_and_reference(tiny_model, tmp_path):
    from atomflow_b200._lib import lib_path
    cli = lib_path().parent / "af_generate"
    assert cli.exists(), "af_generate is built beside the library"
    pf = tmp_path / "prompt.txt"
    pf.write_text(" ".join(str(t) for t in _prompt()))
    r = subprocess.run([str(cli), "--model", str(tiny_model), "--prompt", str(pf), "--steps", str(GREEDY),
                        "--max-seq", "2048", "--tpot-steps", "20"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.split()
    toks = [int(v) for v in r.stdout.splitlines() if not v.startswith("tpot_ms")]
    assert "tpot_ms" in lines and float(lines[lines.index("tpot_ms") + 1]) > 0
    ref = _reference_tokens(tiny_model)
    # the CLI prints the greedy tokens: the output of the last prompt step, then GREEDY - 1 more
    assert toks == ref[PROMPT - 1:PROMPT - 1 + GREEDY]
    assert toks == _engine_tokens(tiny_model, "exact")[PROMPT - 1:PROMPT - 1 + GREEDY]


def test_engine_rejects_bad_input(tiny_model, tmp_path):
    from atomflow_b200 import lib
    L = lib()
    h = ctypes.c_void_p()
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"NOPE" + bytes(1020))
    assert L.af_engine_create(str(bad).encode(), 2048, 0, 1, ctypes.byref(h)) == 1
    trunc = tmp_path / "trunc.bin"
    trunc.write_bytes(tiny_model.read_bytes()[:1 << 20])
    assert L.af_engine_create(str(trunc).encode(), 2048, 0, 1, ctypes.byref(h)) == 1
    assert L.af_engine_create(str(tiny_model).encode(), 0, 0, 1, ctypes.byref(h)) == 1
    assert L.af_engine_create(str(tiny_model).encode(), 2048, 0, 1, ctypes.byref(h)) == 0
    assert L.af_engine_set_position(h, 2048) == 1 and L.af_engine_set_position(h, -1) == 1
    assert L.af_engine_inject_token(h, 128256) == 1
    assert L.af_engine_replay(h, 1) == 1      # nothing captured yet
    assert L.af_engine_destroy(h) == 0
