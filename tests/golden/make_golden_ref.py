"""Generate tests/golden/ref_gemv.npz by running the REFERENCE's own
w8a16_gemv_kernel (oracle/_ref/libafref.so, compiled from the reference's
src/kernel/qkv_gemm.cu) on a GPU, on seeded inputs.

    python tests/golden/make_golden_ref.py [out.npz]

The CPU test tests/test_oracle.py::test_refmath_matches_reference_kernel_golden
then pins the oracle's bit-exact restatement to these outputs.
"""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
import oracle  # noqa: E402
from tests._util import make_gemv_case  # noqa: E402

CASES = [  # (seed, N, K, x_std): config-0 shape, a ragged N, the K range, a heavy-tailed x
    (0, 48, 3072, 1.0), (1, 37, 1024, 1.0), (2, 16, 128, 1.0), (3, 9, 640, 1.0),
    (4, 24, 8192, 1.0), (5, 32, 3072, 40.0), (6, 16, 4096, 1e-3),
]


def main(out):
    R = oracle.ref()
    assert R is not None, "oracle/_ref/libafref.so not built"
    arrays = {"ncases": np.array(len(CASES))}
    for i, (seed, N, K, xs) in enumerate(CASES):
        x, q, s = make_gemv_case(seed, 1, N, K, x_std=xs)
        xd = torch.from_numpy(x.view(np.int16)).cuda()
        qd = torch.from_numpy(q).cuda()
        sd = torch.from_numpy(s.view(np.int16)).cuda()
        yd = torch.zeros(N, dtype=torch.int16, device="cuda")
        rc = R.afref_w8a16_gemv(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), yd.data_ptr(), N, K,
                                torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert rc == 0, rc
        arrays.update({f"x{i}": x, f"q{i}": q, f"s{i}": s,
                       f"y{i}": yd.cpu().numpy().view(np.uint16)})
    np.savez_compressed(out, **arrays)
    print("wrote", out)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(Path(__file__).with_name("ref_gemv.npz")))
