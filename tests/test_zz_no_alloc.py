"""The argmax entry point that allocates nothing, af_argmax_f32_noalloc.

It exists for callers that cannot allocate device memory -- hosts where
cudaMalloc is unavailable or not allowed, which therefore cannot hand the
library a workspace.  Its scratch is a fixed block inside the library.  These
tests call it through the C ABI and check it against af_argmax_f32 (the
workspace-taking entry point) -- argmax indices, compared exactly -- on two
calls in a row, since the second call reuses the scratch the first one left.

This file is collected last on purpose; it must pass alone in a fresh process
as well as after the other tests.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _lib():
    from atomflow_b200 import lib
    return lib()


def _reference_argmax(L, vd, V, mode, st):
    ws = torch.zeros(L.af_argmax_workspace_bytes(V), dtype=torch.uint8, device="cuda")
    out = torch.full((1,), -3, dtype=torch.int32, device="cuda")
    assert L.af_argmax_f32(vd.data_ptr(), V, out.data_ptr(), mode, ws.data_ptr(), ws.numel(), st) == 0
    return out


@pytest.mark.parametrize("V", [1, 1000, 65537, 128256, 3_000_000])
@pytest.mark.parametrize("mode", [0, 1])
def test_noalloc_matches_workspace_argmax_two_calls(V, mode):
    L = _lib()
    st = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(V + 17 * mode)
    for call in range(2):
        v = rng.standard_normal(V).astype(np.float32)
        if V > 70000:
            v[V - 5] = 50.0 + call        # a winner above id 65535 (REF_COMPAT ignores it)
            v[123 + call] = 40.0
        vd = torch.from_numpy(v).cuda()
        out = torch.full((1,), -7, dtype=torch.int32, device="cuda")
        assert L.af_argmax_f32_noalloc(vd.data_ptr(), V, out.data_ptr(), mode, st) == 0
        ref = _reference_argmax(L, vd, V, mode, st)
        torch.cuda.synchronize()
        assert int(out.item()) == int(ref.item()), (call, int(out.item()), int(ref.item()))


def test_noalloc_rejects_oversized_and_bad_arguments():
    L = _lib()
    st = torch.cuda.current_stream().cuda_stream
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    vd = torch.zeros(16, dtype=torch.float32, device="cuda")
    assert L.af_argmax_f32_noalloc(vd.data_ptr(), (1 << 28) + 1, out.data_ptr(), 0, st) == 2   # UNSUPPORTED
    assert b"scratch limit" in L.af_last_cuda_error()
    assert L.af_argmax_f32_noalloc(vd.data_ptr(), 0, out.data_ptr(), 0, st) == 1               # INVALID
    assert L.af_argmax_f32_noalloc(vd.data_ptr(), 16, out.data_ptr(), 9, st) == 1
