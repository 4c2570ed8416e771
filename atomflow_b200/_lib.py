"""ctypes binding of the C ABI in include/atomflow_b200.h.

The CUDA library is required: importing an op when libatomflow_b200.so is
missing or fails to load raises immediately -- there is no CPU fallback.
"""
import ctypes
import enum
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libatomflow_b200.so"


class Status(enum.IntEnum):
    OK = 0
    INVALID = 1
    UNSUPPORTED = 2
    PEER_TIMEOUT = 3
    CUDA = 4
    WORKSPACE = 5


class ScaleKind(enum.IntEnum):
    GROUP_F16 = 0
    ROW_F32 = 1
    NONE = 2


class WeightDtype(enum.IntEnum):
    F16 = 0
    FP8_E4M3 = 1


class ArgmaxMode(enum.IntEnum):
    TRUE = 0
    REF_COMPAT = 1


class AtomflowError(RuntimeError):
    def __init__(self, status, where=""):
        self.status = Status(status)
        msg = f"{where}: {lib().af_status_string(int(status)).decode()}"
        if self.status == Status.CUDA:
            msg += f" ({lib().af_last_cuda_error().decode()})"
        super().__init__(msg)


class ChainOp(ctypes.Structure):
    """af_chain_op (include/atomflow_b200.h)."""
    _fields_ = [("kind", ctypes.c_int), ("N", ctypes.c_int), ("K", ctypes.c_int), ("wait_prev", ctypes.c_int),
                ("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("w2", ctypes.c_void_p), ("scales2", ctypes.c_void_p), ("norm_w", ctypes.c_void_p),
                ("eps", ctypes.c_float), ("y", ctypes.c_void_p), ("xn_out", ctypes.c_void_p),
                ("aux", ctypes.c_void_p)]


class OpKind(enum.IntEnum):
    GEMV = 0
    GEMV_RESIDUAL = 1
    RMSNORM_GEMV = 2
    RMSNORM_SWIGLU = 3


# Every symbol include/atomflow_b200.h and include/atomflow_view_ops.h declare,
# with its ctypes signature (restype, argtypes).
_vp, _sz, _i, _fp = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p
C_SYMBOLS = {
    "af_status_string": (ctypes.c_char_p, [_i]),
    "af_last_cuda_error": (ctypes.c_char_p, []),
    "af_version": (_i, []),
    "af_workspace_reset": (_i, [_vp, _sz, _vp]),
    "af_w8a16_gemv_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "af_w8a16_gemv": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "af_w8a16_gemm_tc": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "af_lm_head_workspace_bytes": (_sz, [_i, _i, _i]),
    "af_lm_head_gemv": (_i, [_vp, _vp, _i, _vp, _vp, _i, _i, _vp, _i, _vp, _sz, _vp]),
    "af_argmax_workspace_bytes": (_sz, [_i]),
    "af_argmax_f32": (_i, [_vp, _i, _vp, _i, _vp, _sz, _vp]),
    "af_argmax_f32_noalloc": (_i, [_vp, _i, _vp, _i, _vp]),
    "af_tp_create": (_i, [_i, _i, _i, ctypes.POINTER(ctypes.c_void_p)]),
    "af_tp_ipc_handle": (_i, [_vp, _vp]),
    "af_tp_open_peers": (_i, [_vp, _vp]),
    "af_tp_set_peer": (_i, [_vp, _i, _vp]),
    "af_tp_buffer_bytes": (_sz, [_i]),
    "af_tp_buffer": (_vp, [_vp]),
    "af_tp_set_wait_limit_ms": (_i, [_vp, _i]),
    "af_tp_status": (_i, [_vp, ctypes.POINTER(ctypes.c_int)]),
    "af_tp_destroy": (_i, [_vp]),
    "af_w8a16_gemv_allreduce": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "af_lm_head_gemv_tp": (_i, [_vp, _vp, _i, _vp, _vp, _i, _i, _i, _vp, _i, _vp, _sz, _vp, _vp]),
    "af_rmsnorm_w8a16_gemv": (_i, [_vp, _vp, ctypes.c_float, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "af_w8a16_gemv_residual": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "af_rmsnorm_w8a16_swiglu": (_i, [_vp, _vp, ctypes.c_float, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    "af_w8a16_gemv_allreduce_residual": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "af_embed_lookup": (_i, [_vp, _vp, _vp, _i, _vp]),
    "af_rope_tables": (_i, [_vp, _vp, _i, _i, ctypes.c_float]),
    "af_rope_kv_write": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "af_decode_attention_workspace_bytes": (_sz, [_i, _i, _i]),
    "af_decode_attention": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    "af_decode_rope_attention": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    "af_device_faults": (_i, [ctypes.POINTER(ctypes.c_uint), _i]),
    "af_decode_rope_attention_fast": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    "af_rmsnorm": (_i, [_vp, _vp, ctypes.c_float, _vp, _i, _vp]),
    "af_decode_advance": (_i, [_vp, _i, _vp]),
    "af_chain_workspace_bytes": (_sz, [_i]),
    "af_gemv_chain": (_i, [ctypes.c_void_p, _i, _vp, _sz, _vp]),
    "af_gemv_chain_fast": (_i, [ctypes.c_void_p, _i, _vp, _sz, _vp]),
    "af_engine_create": (_i, [ctypes.c_char_p, _i, _i, _i, ctypes.POINTER(ctypes.c_void_p)]),
    "af_engine_create_tp": (_i, [ctypes.c_char_p, _i, _i, _vp, ctypes.POINTER(ctypes.c_void_p)]),
    "af_engine_destroy": (_i, [_vp]),
    "af_engine_info": (_i, [_vp, ctypes.POINTER(ctypes.c_int)]),
    "af_engine_set_position": (_i, [_vp, _i]),
    "af_engine_get_position": (_i, [_vp, ctypes.POINTER(ctypes.c_int)]),
    "af_engine_inject_token": (_i, [_vp, _i]),
    "af_engine_output_token": (_i, [_vp, ctypes.POINTER(ctypes.c_int)]),
    "af_engine_step": (_i, [_vp, _i]),
    "af_engine_capture": (_i, [_vp, _i]),
    "af_engine_replay": (_i, [_vp, _i]),
    "af_engine_synchronize": (_i, [_vp]),
    "af_engine_stream": (_vp, [_vp]),
    "af_engine_device_token": (_vp, [_vp]),
    "af_engine_device_position": (_vp, [_vp]),
    "af_engine_logits": (_vp, [_vp]),
    "af_view_last_status": (_i, []),
    "af_view_set_argmax_mode": (_i, [_i]),
}
# C++ launchers with the reference's signatures (include/ops/kernel.h); references are pointers.
CXX_SYMBOLS = {
    "launch_w8a16_gemv": ("_Z17launch_w8a16_gemvRK4ViewS1_S1_RS_iP11CUstream_st",
                          None, [_vp, _vp, _vp, _vp, _i, _vp]),
    "launch_argmax": ("_Z13launch_argmaxRK4ViewPiP11CUstream_st", None, [_vp, _vp, _vp]),
    "launch_linear_gemm": ("_Z18launch_linear_gemmRK4ViewS1_RS_P13cublasContextP11CUstream_st",
                           None, [_vp, _vp, _vp, _vp, _vp]),
}

_lib = None


def lib_path() -> Path:
    return _LIB_PATH


def lib():
    """Load libatomflow_b200.so (raises if it is missing -- no fallback)."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise ImportError(f"{_LIB_PATH} is missing; build it with `python -m atomflow_b200.build`")
        h = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in C_SYMBOLS.items():
            f = getattr(h, name)
            f.restype, f.argtypes = res, args
        for name, (mangled, res, args) in CXX_SYMBOLS.items():
            f = getattr(h, mangled)
            f.restype, f.argtypes = res, args
            setattr(h, name, f)
        _lib = h
    return _lib


def check(status, where):
    if status != 0:
        raise AtomflowError(status, where)


class View(ctypes.Structure):
    """The reference's View (include/core/view.h:22-39): 56 bytes."""
    _fields_ = [("dtype", ctypes.c_int), ("data_ptr", ctypes.c_void_p),
                ("dims", ctypes.c_int32 * 4), ("strides", ctypes.c_int32 * 4),
                ("num_dims", ctypes.c_int8)]


class DataType(enum.IntEnum):
    FP32 = 0
    FP16 = 1
    BF16 = 2
    FP8_E4M3 = 3


def make_view(ptr: int, dtype: DataType, dims) -> View:
    """create_contiguous_view (include/core/view.h:41-55)."""
    v = View()
    v.dtype = int(dtype)
    v.data_ptr = ptr
    v.num_dims = len(dims)
    for i, d in enumerate(dims):
        v.dims[i] = d
    st = 1
    for i in reversed(range(len(dims))):
        v.strides[i] = st
        st *= dims[i]
    return v


assert ctypes.sizeof(View) == 56
