"""Python handle on the checkers.  TEST INFRASTRUCTURE ONLY.

  oracle.cpu()  -- liboracle.so, the C restatement of the reference arithmetic
  oracle.ref()  -- _ref/libafref.so, the reference's own CUDA kernels compiled
                   from its sources (None when it was not built)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and reference
legs use this package; the product (atomflow_b200/) never imports it.
"""
import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_cpu = None
_ref = None


def build(ref_sources=None):
    """Compile liboracle.so; also the reference's own kernels and engine into
    _ref/ when `ref_sources` names a reference checkout."""
    subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    if ref_sources is not None and (Path(ref_sources) / "src" / "kernel" / "qkv_gemm.cu").exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={ref_sources}"], check=True)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def cpu():
    global _cpu
    if _cpu is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            build()
        L = ctypes.CDLL(str(path))
        vp, i = ctypes.c_void_p, ctypes.c_int
        L.af_oracle_e4m3_to_float.restype = ctypes.c_float
        L.af_oracle_e4m3_to_float.argtypes = [ctypes.c_uint8]
        L.af_oracle_float_to_e4m3_rn.restype = ctypes.c_uint8
        L.af_oracle_float_to_e4m3_rn.argtypes = [ctypes.c_float]
        L.af_oracle_half_to_float.restype = ctypes.c_float
        L.af_oracle_half_to_float.argtypes = [ctypes.c_uint16]
        L.af_oracle_float_to_half_rn.restype = ctypes.c_uint16
        L.af_oracle_float_to_half_rn.argtypes = [ctypes.c_float]
        L.af_oracle_quantize_gs128.argtypes = [vp, i, i, vp, vp]
        L.af_oracle_quantize_row.argtypes = [vp, i, i, vp, vp]
        L.af_oracle_gemv_f64.argtypes = [vp, vp, vp, i, i, i, i, vp]
        L.af_oracle_gemv_f64_l2.argtypes = [vp, vp, vp, i, i, i, i, vp, vp]
        L.af_oracle_gemv_refmath.argtypes = [vp, vp, vp, i, i, vp, i]
        L.af_oracle_argmax.restype = i
        L.af_oracle_argmax.argtypes = [vp, i, i]
        _cpu = L
    return _cpu


_ref_engine = {}


def ref_engine(shim=False):
    """The reference's decode engine (GPU), or None if its library is absent.
    shim=True: the same unmodified engine.cu linked against this library's View
    launchers in place of the reference's GEMV and argmax
    (_ref/libafref_engine_shim.so)."""
    name = "libafref_engine_shim.so" if shim else "libafref_engine.so"
    if name not in _ref_engine:
        path = HERE / "_ref" / name
        if not path.exists():
            return None
        L = ctypes.CDLL(str(path))
        vp, i = ctypes.c_void_p, ctypes.c_int
        L.afref_engine_create.restype = vp
        L.afref_engine_create.argtypes = [ctypes.c_char_p]
        L.afref_engine_destroy.restype = None
        L.afref_engine_destroy.argtypes = [vp]
        L.afref_engine_step.restype = i
        L.afref_engine_step.argtypes = [vp, i, i]
        L.afref_engine_tpot_ms.restype = ctypes.c_float
        L.afref_engine_tpot_ms.argtypes = [vp, i, i, i]
        L.afref_engine_logits.restype = vp
        L.afref_engine_logits.argtypes = [vp, ctypes.POINTER(ctypes.c_int)]
        _ref_engine[name] = L
    return _ref_engine[name]


def ref():
    """The reference's kernels (GPU), or None if _ref/libafref.so is absent."""
    global _ref
    if _ref is None:
        path = HERE / "_ref" / "libafref.so"
        if not path.exists():
            return None
        L = ctypes.CDLL(str(path))
        vp, i = ctypes.c_void_p, ctypes.c_int
        L.afref_w8a16_gemv.restype = i
        L.afref_w8a16_gemv.argtypes = [vp, vp, vp, vp, i, i, vp]
        L.afref_argmax.restype = i
        L.afref_argmax.argtypes = [vp, i, vp, vp]
        L.afref_lm_head.restype = i
        L.afref_lm_head.argtypes = [vp, vp, vp, i, i, vp]
        L.afref_rms_norm.restype = i
        L.afref_rms_norm.argtypes = [vp, vp, vp, i, ctypes.c_float, vp]
        L.afref_swiglu.restype = i
        L.afref_swiglu.argtypes = [vp, vp, vp, i, vp]
        L.afref_residual_add.restype = i
        L.afref_residual_add.argtypes = [vp, vp, i, vp]
        L.afref_rope_kv.restype = i
        L.afref_rope_kv.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, vp]
        L.afref_rope_cache.restype = i
        L.afref_rope_cache.argtypes = [vp, vp, i, i, ctypes.c_float, vp]
        L.afref_cached_attention.restype = i
        L.afref_cached_attention.argtypes = [vp, vp, vp, vp, i, i, i, i, vp]
        _ref = L
    return _ref


# ----------------------------------------------------------- numpy wrappers

def quantize_gs128(w):
    """w float32 [N, K] -> (q uint8 [N, K], s uint16 (fp16 bits) [N, K/128])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    q = np.empty((N, K), np.uint8)
    s = np.empty((N, K // 128), np.uint16)
    cpu().af_oracle_quantize_gs128(_p(w), N, K, _p(q), _p(s))
    return q, s


def quantize_row(w):
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    q = np.empty((N, K), np.uint8)
    s = np.empty((N,), np.float32)
    cpu().af_oracle_quantize_row(_p(w), N, K, _p(q), _p(s))
    return q, s


KIND = {"group": 0, "row": 1, "none": 2, "f16": 3}


def gemv_f64(x, w, s, kind, with_l2=False):
    """x fp16-bits uint16 [M, K]; w uint8 [N, K] (or uint16 fp16 bits for kind 'f16').
    Returns y [M, N] in FP64 (and, with_l2, the l2 norm of each output's terms)."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    x = x.reshape(-1, x.shape[-1])
    w = np.ascontiguousarray(w)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), np.float64)
    l2 = np.empty((M, N), np.float64) if with_l2 else None
    s = np.ascontiguousarray(s) if s is not None else None
    cpu().af_oracle_gemv_f64_l2(_p(x), _p(w), _p(s) if s is not None else None, KIND[kind], M, N, K,
                                _p(y), _p(l2) if with_l2 else None)
    return (y, l2) if with_l2 else y


def gemv_refmath(x, w, s, nthreads=1):
    """Bit-exact restatement of the reference kernel: returns fp16 bits uint16 [N]."""
    x = np.ascontiguousarray(x, dtype=np.uint16).reshape(-1)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.uint16)
    N, K = w.shape
    y = np.empty((N,), np.uint16)
    cpu().af_oracle_gemv_refmath(_p(x), _p(w), _p(s), N, K, _p(y), nthreads)
    return y


def argmax(v, mode=0):
    v = np.ascontiguousarray(v, dtype=np.float32)
    return cpu().af_oracle_argmax(_p(v), v.size, mode)


def half_ulp(ref_f16_bits):
    """Size of one FP16 ulp at the binade of each reference value (fp16 bits)."""
    e = (np.asarray(ref_f16_bits, np.uint16) >> 10) & 31
    e = np.maximum(e.astype(np.int32), 1)
    return np.ldexp(1.0, e - 25)
