"""CPU tests of the oracle (the parity checker) against independent decoders,
the reference's own quantiser output, and the reference kernel's own outputs."""
from pathlib import Path

import ml_dtypes
import numpy as np
import pytest

import oracle
from tests._util import assert_fp16_parity, make_gemv_case, normal_f32

GOLD = Path(__file__).resolve().parent / "golden"


def test_e4m3_decode_matches_ml_dtypes():
    L = oracle.cpu()
    b = np.arange(256, dtype=np.uint8)
    want = b.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    got = np.array([L.af_oracle_e4m3_to_float(int(i)) for i in b], np.float32)
    np.testing.assert_array_equal(np.isnan(want), np.isnan(got))
    np.testing.assert_array_equal(want[~np.isnan(want)], got[~np.isnan(got)])
    # known answers: smallest subnormal, max normal, NaN
    assert got[0x01] == 2.0 ** -9 and got[0x7E] == 448.0 and np.isnan(got[0x7F])


def test_e4m3_encode_round_to_nearest_even():
    L = oracle.cpu()
    rng = np.random.default_rng(7)
    f = np.concatenate([rng.normal(0, 100, 4000), rng.normal(0, 1e-2, 4000),
                        rng.uniform(-448, 448, 4000), [0.0, -0.0, 2.0 ** -10, 3 * 2.0 ** -11,
                                                       448.0, -448.0, 464.0]]).astype(np.float32)
    want = f.astype(ml_dtypes.float8_e4m3fn).view(np.uint8)
    got = np.array([L.af_oracle_float_to_e4m3_rn(float(v)) for v in f], np.uint8)
    np.testing.assert_array_equal(want, got)


def test_half_conversions_match_numpy():
    L = oracle.cpu()
    hb = np.arange(0, 65536, 7, dtype=np.uint16)
    want = hb.view(np.float16).astype(np.float32)
    got = np.array([L.af_oracle_half_to_float(int(i)) for i in hb], np.float32)
    np.testing.assert_array_equal(np.isnan(want), np.isnan(got))
    np.testing.assert_array_equal(want[~np.isnan(want)], got[~np.isnan(got)])
    f = np.concatenate([normal_f32(3, 5000, 3000.0), normal_f32(4, 5000, 1e-5)])
    got = np.array([L.af_oracle_float_to_half_rn(float(v)) for v in f], np.uint16)
    np.testing.assert_array_equal(f.astype(np.float16).view(np.uint16), got)


@pytest.mark.parametrize("i", [0, 1, 2])
def test_quantizer_matches_reference_exporter(i):
    """Golden vectors produced by the reference's quantize_fp8_gs128
    (tools/quantize_weights.py:220-268), see golden/make_golden_quant.py."""
    d = np.load(GOLD / "quant_gs128.npz")
    q, s = oracle.quantize_gs128(d[f"w{i}"])
    np.testing.assert_array_equal(q, d[f"q{i}"])
    np.testing.assert_array_equal(s, d[f"s{i}"])


def test_library_quantizer_matches_reference_exporter():
    torch = pytest.importorskip("torch")
    from atomflow_b200 import quant
    d = np.load(GOLD / "quant_gs128.npz")
    for i in range(3):
        q, s = quant.quantize_gs128(torch.from_numpy(d[f"w{i}"]))
        np.testing.assert_array_equal(q.view(torch.uint8).numpy(), d[f"q{i}"])
        np.testing.assert_array_equal(s.view(torch.int16).numpy().view(np.uint16), d[f"s{i}"])


@pytest.mark.parametrize("N,K", [(64, 3072), (33, 1024), (8, 128), (5, 640)])
def test_refmath_within_tolerance_of_f64(N, K):
    x, q, s = make_gemv_case(11, 1, N, K)
    y = oracle.gemv_refmath(x, q, s)
    ref, l2 = oracle.gemv_f64(x, q, s, "group", with_l2=True)
    assert_fp16_parity(y, (ref[0], l2[0]), "refmath vs f64")


def test_refmath_threads_do_not_change_bits():
    x, q, s = make_gemv_case(12, 1, 200, 2048)
    np.testing.assert_array_equal(oracle.gemv_refmath(x, q, s, 1), oracle.gemv_refmath(x, q, s, 4))


def test_f64_oracle_kinds_agree():
    """Group scales that are all equal to a row scale give the row-scale result."""
    x, q, _ = make_gemv_case(13, 2, 16, 256, kind="none")
    s_row = np.full(16, 0.5, np.float32)
    s_grp = np.full((16, 2), np.float16(0.5).view(np.uint16), np.uint16)
    a = oracle.gemv_f64(x, q, s_row, "row")
    b = oracle.gemv_f64(x, q, s_grp, "group")
    np.testing.assert_allclose(a, b, rtol=0, atol=0)


def test_argmax_oracle():
    v = np.array([1.0, 3.0, 3.0, np.nan, -1.0], np.float32)
    assert oracle.argmax(v) == 1
    big = np.zeros(70000, np.float32)
    big[69000] = 5.0
    big[100] = 4.0
    assert oracle.argmax(big, 0) == 69000
    assert oracle.argmax(big, 1) == 100      # the reference only sees ids < 65536


def test_refmath_matches_reference_kernel_golden():
    """Pin: outputs of the reference's own w8a16_gemv_kernel, run on a B200
    (golden/make_golden_ref.py), equal the bit-exact restatement."""
    path = GOLD / "ref_gemv.npz"
    if not path.exists():
        pytest.fail("golden/ref_gemv.npz missing: run golden/make_golden_ref.py on a GPU box")
    d = np.load(path)
    n = int(d["ncases"])
    for i in range(n):
        y = oracle.gemv_refmath(d[f"x{i}"], d[f"q{i}"], d[f"s{i}"])
        np.testing.assert_array_equal(y, d[f"y{i}"], err_msg=f"case {i} {d[f'q{i}'].shape}")


def test_reference_kernel_needs_the_fp32_noise_floor():
    """The reference kernel's own outputs (its bit-exact restatement) break the
    bare '2 FP16 ulp or 2e-3 relative vs FP64' rule on outputs that cancel to
    ~1e-6, and stay inside the FP32 noise floor the parity tests add."""
    x, q, s = make_gemv_case(900 + 33, 33, 3072, 8192)
    ref, l2 = oracle.gemv_f64(x, q, s, "group", with_l2=True)
    y = np.stack([oracle.gemv_refmath(x[m], q, s, 8) for m in range(33)])
    with pytest.raises(AssertionError):
        assert_fp16_parity(y, ref, "reference kernel, bare rule")
    assert_fp16_parity(y, (ref, l2), "reference kernel, with the FP32 floor")
