"""Host-side operators over the C ABI, for callers that hold torch CUDA tensors.

PyTorch here is plumbing (device memory, the current stream); all arithmetic
runs in libatomflow_b200.so.  Each op mirrors a reference launcher:

  w8a16_gemv  <- launch_w8a16_gemv   (include/ops/kernel.h:138-145)
  lm_head     <- engine.cu:494-513 cublasGemmEx + argmax launch (engine.cu:521)
  argmax      <- launch_argmax       (include/ops/kernel.h:155-159)
"""
import torch

from ._lib import ArgmaxMode, ScaleKind, WeightDtype, check, lib


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class Workspace:
    """Zero-initialised device scratch that grows on demand.  Kernels leave it
    zeroed again, so one Workspace serves every call issued on one stream."""

    def __init__(self, device=None, nbytes=1 << 20):
        self.device = torch.device(device or "cuda")
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)

    def get(self, nbytes):
        if self.buf.numel() < nbytes:
            torch.cuda.current_stream(self.device).synchronize()
            self.buf = torch.zeros(max(nbytes, 2 * self.buf.numel()), dtype=torch.uint8,
                                   device=self.device)
        return self.buf.data_ptr(), self.buf.numel()


_default_ws = {}


def default_workspace(device) -> Workspace:
    d = torch.device(device)
    key = d.index if d.index is not None else torch.cuda.current_device()
    if key not in _default_ws:
        _default_ws[key] = Workspace(torch.device("cuda", key))
    return _default_ws[key]


def _need(t, dtype, name):
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor")


def w8a16_gemv(x, w, scales=None, out=None, *, scale_kind="group", group_size=128,
               workspace=None, stream=None):
    """y[M, N] (fp16) = dequant(w[N, K] fp8) @ x[M, K] (fp16)^T, FP32 accumulation."""
    kind = {"group": ScaleKind.GROUP_F16, "row": ScaleKind.ROW_F32, "none": ScaleKind.NONE}[scale_kind]
    x2 = x.reshape(-1, x.shape[-1])
    M, K = x2.shape
    N = w.shape[0]
    _need(x2, torch.float16, "x")
    if w.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise ValueError("w must be float8_e4m3fn (or its uint8 bytes)")
    if out is None:
        out = torch.empty(M, N, dtype=torch.float16, device=x.device)
    _need(out, torch.float16, "out")
    L = lib()
    ws = workspace or default_workspace(x.device)
    need = L.af_w8a16_gemv_workspace_bytes(M, N, K, int(kind))
    ptr, nb = ws.get(need)
    check(L.af_w8a16_gemv(x2.data_ptr(), w.data_ptr(), scales.data_ptr() if scales is not None else None,
                          out.data_ptr(), M, N, K, group_size, int(kind), ptr, nb, _stream(stream)),
          "af_w8a16_gemv")
    return out


def lm_head(x, w, row_scale=None, logits=None, *, want_logits=True, want_argmax=True,
            mode="true", workspace=None, stream=None):
    """FP32 logits[V] = w[V, D] @ x[D]; optional fused greedy argmax (device int32[1])."""
    V, D = w.shape
    wdt = WeightDtype.F16 if w.dtype == torch.float16 else WeightDtype.FP8_E4M3
    if want_logits and logits is None:
        logits = torch.empty(V, dtype=torch.float32, device=x.device)
    idx = torch.empty(1, dtype=torch.int32, device=x.device) if want_argmax else None
    L = lib()
    ws = workspace or default_workspace(x.device)
    ptr, nb = ws.get(L.af_lm_head_workspace_bytes(V, D, int(wdt)))
    m = ArgmaxMode.TRUE if mode == "true" else ArgmaxMode.REF_COMPAT
    check(L.af_lm_head_gemv(x.data_ptr(), w.data_ptr(), int(wdt),
                            row_scale.data_ptr() if row_scale is not None else None,
                            logits.data_ptr() if want_logits else None, V, D,
                            idx.data_ptr() if idx is not None else None, int(m), ptr, nb,
                            _stream(stream)), "af_lm_head_gemv")
    return logits, idx


def argmax(logits, *, mode="true", out=None, workspace=None, stream=None):
    V = logits.shape[-1]
    _need(logits, torch.float32, "logits")
    if out is None:
        out = torch.empty(1, dtype=torch.int32, device=logits.device)
    L = lib()
    ws = workspace or default_workspace(logits.device)
    ptr, nb = ws.get(L.af_argmax_workspace_bytes(V))
    m = ArgmaxMode.TRUE if mode == "true" else ArgmaxMode.REF_COMPAT
    check(L.af_argmax_f32(logits.data_ptr(), V, out.data_ptr(), int(m), ptr, nb, _stream(stream)),
          "af_argmax_f32")
    return out
