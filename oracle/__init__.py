"""CPU oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this package, as the checker of the
device results or as the timed CPU baseline. It wraps two libraries built by oracle/Makefile:

  liboracle.so          the C restatement in oracle/oracle.c of the reference's CPU arithmetic for the decode hot
                        path (fpga/src/gemvq_ref.h) and of the command-list semantics (fpga/src/gemvqc16.h:24-121);
  _ref/libgemvq_ref.so  the reference's own gemvq_ref.h compiled from its sources (oracle/ref_shim.cpp), used to
                        pin the restatement and as the "reference" CPU baseline.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libgemvq_ref.so")

_P = ctypes.c_void_p
_orc = None
_ref = None


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def orc() -> ctypes.CDLL:
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_PATH):
            raise RuntimeError(f"{ORACLE_PATH} missing: make -C oracle")
        L = ctypes.CDLL(ORACLE_PATH)
        U, F, SZ = ctypes.c_uint, ctypes.c_float, ctypes.c_size_t
        L.orc_gemv.argtypes = [_P, _P, U, U, U, _P, _P]
        L.orc_block_sums.argtypes = [_P, _P, U, U, U, _P]
        L.orc_quantize_q8_0.argtypes = [_P, U, _P, _P, _P]
        L.orc_quantize_q8_1.argtypes = [_P, U, _P, _P, _P]
        L.orc_quantize_q8_k.argtypes = [_P, U, _P, _P, _P]
        L.orc_half_to_float.argtypes = [ctypes.c_uint16]
        L.orc_half_to_float.restype = F
        L.orc_float_to_half.argtypes = [F]
        L.orc_float_to_half.restype = ctypes.c_uint16
        L.orc_rownorm.argtypes = [_P, _P, U, U, U, F, U, _P]
        L.orc_norm_scale.argtypes = [_P, U, F, U]
        L.orc_norm_scale.restype = F
        L.orc_unary1.argtypes = [F, U]
        L.orc_unary1.restype = F
        L.orc_silu_mul1.argtypes = [F, F, U]
        L.orc_silu_mul1.restype = F
        L.orc_conv.argtypes = [_P, _P, _P, U, U, _P, _P]
        L.orc_rope.argtypes = [_P, _P, U, U, U, _P]
        L.orc_gdn.argtypes = [_P, _P, _P, _P, _P, _P, U, U, F, _P, _P, _P]
        L.orc_attn.argtypes = [_P, _P, _P, U, U, U, U, U, F, _P]
        L.orc_dequantize_row.argtypes = [_P, U, U, _P]
        L.orc_row_bytes.argtypes = [U, U]
        L.orc_row_bytes.restype = SZ
        L.orc_run_list.argtypes = [_P, SZ, _P, SZ, _P, U, _P, SZ, U, _P, U]
        L.orc_run_list.restype = ctypes.c_int
        _orc = L
    return _orc


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not os.path.exists(REF_PATH):
            raise RuntimeError(f"{REF_PATH} missing: make -C oracle (needs the reference sources)")
        L = ctypes.CDLL(REF_PATH)
        U, F = ctypes.c_uint, ctypes.c_float
        L.ref_gemv.argtypes = [_P, _P, U, U, U, _P, _P]
        L.ref_gemv_rows_omp.argtypes = [_P, _P, U, U, U, _P, ctypes.c_int]
        L.ref_quantize_q8_k.argtypes = [_P, U, _P, _P]
        L.ref_half_to_float.argtypes = [ctypes.c_uint16]
        L.ref_half_to_float.restype = F
        L.ref_float_to_half.argtypes = [F]
        L.ref_float_to_half.restype = ctypes.c_uint16
        L.ref_rownorm.argtypes = [_P, _P, U, U, F, U, _P]
        L.ref_rmsnorm.argtypes = [_P, _P, U, F, _P]
        L.ref_silu_mul.argtypes = [_P, _P, U, _P]
        L.ref_unary.argtypes = [_P, U, U, _P]
        L.ref_add.argtypes = [_P, _P, U, _P]
        L.ref_mul.argtypes = [_P, _P, U, _P]
        L.ref_conv.argtypes = [_P, _P, _P, U, ctypes.c_int, _P, _P]
        L.ref_gdn.argtypes = [_P, _P, _P, _P, _P, _P, U, U, F, _P, _P, _P]
        L.ref_within_tolerance.argtypes = [F, F, ctypes.c_double]
        L.ref_within_elementwise.argtypes = [F, F]
        _ref = L
    return _ref


# ---- restatement ---------------------------------------------------------------------------------------------------
def quantize_q8_0(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    q, d, b = np.zeros(n, np.int8), np.zeros(n // 32, np.uint16), np.zeros(n // 32, np.int32)
    orc().orc_quantize_q8_0(_ptr(x), n, _ptr(q), _ptr(d), _ptr(b))
    return q, d, b


def quantize_q8_1(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    q, ds, b = np.zeros(n, np.int8), np.zeros(n // 16, np.uint16), np.zeros(n // 32, np.int32)
    orc().orc_quantize_q8_1(_ptr(x), n, _ptr(q), _ptr(ds), _ptr(b))
    return q, ds, b


def quantize_q8_k(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    q, d, b = np.zeros(n, np.int8), np.zeros(n // 256, np.float32), np.zeros(n // 16, np.int32)
    orc().orc_quantize_q8_k(_ptr(x), n, _ptr(q), _ptr(d), _ptr(b))
    return q, d, b


def gemv(w: np.ndarray, x: np.ndarray, rows: int, cols: int, fmt: int):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y, mag = np.zeros(rows, np.float32), np.zeros(rows, np.float64)
    if orc().orc_gemv(_ptr(w), _ptr(x), rows, cols, fmt, _ptr(y), _ptr(mag)) != 0:
        raise ValueError("unsupported format")
    return y, mag


def block_sums(w: np.ndarray, q: np.ndarray, rows: int, cols: int, fmt: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    q = np.ascontiguousarray(q, dtype=np.int8)
    n = rows * (cols // 256) * 9 if fmt in (13, 14) else rows * (cols // 32)
    out = np.zeros(n, np.int32)
    orc().orc_block_sums(_ptr(w), _ptr(q), rows, cols, fmt, _ptr(out))
    return out


def rownorm(x, w, n, rows, eps, flags, stride=0):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w if w is not None else np.zeros(n), dtype=np.float32)
    y = np.zeros(n * rows, np.float32)
    orc().orc_rownorm(_ptr(x), _ptr(w), n, rows, stride, eps, flags, _ptr(y))
    return y


def dequantize_row(row: np.ndarray, cols: int, fmt: int) -> np.ndarray:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    y = np.zeros(cols, np.float32)
    orc().orc_dequantize_row(_ptr(row), cols, fmt, _ptr(y))
    return y


def gdn(state, q, k, v, g, beta, hv, hk, scale):
    st = np.ascontiguousarray(state, dtype=np.float32).copy()
    y = np.zeros(hv * 128, np.float32)
    ym, sm = np.zeros(hv * 128, np.float64), np.zeros(st.size, np.float64)
    args = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, g, beta)]
    orc().orc_gdn(_ptr(st), *[_ptr(a) for a in args], hv, hk, scale, _ptr(y), _ptr(ym), _ptr(sm))
    return st, y, ym, sm


class _Weight(ctypes.Structure):
    _fields_ = [("handle", ctypes.c_uint64), ("data", ctypes.c_void_p), ("rows", ctypes.c_uint),
                ("cols", ctypes.c_uint), ("format", ctypes.c_uint)]


def run_list(act: np.ndarray, cmds: np.ndarray, weights: dict, state: np.ndarray | None = None,
             kv: np.ndarray | None = None, kv_ctx: int = 0) -> int:
    """Runs a command list on the CPU in place on act / state / kv; weights: {handle: (gguf_bytes, rows, cols, fmt)}.
    Returns the status word the reference kernel would return."""
    assert act.dtype == np.float32 and act.flags.c_contiguous
    ws = (_Weight * max(1, len(weights)))()
    keep = []
    for i, (h, (data, rows, cols, fmt)) in enumerate(weights.items()):
        d = np.ascontiguousarray(data, dtype=np.uint8)
        keep.append(d)
        ws[i] = _Weight(h, d.ctypes.data, rows, cols, fmt)
    c = np.ascontiguousarray(cmds, dtype=np.uint32)
    st = state if state is not None else np.zeros(128, np.float32)
    kvb = kv if kv is not None else np.zeros(8, np.uint16)
    return orc().orc_run_list(_ptr(act), act.size, _ptr(st), st.size // 128, ws, len(weights), _ptr(kvb),
                              kvb.nbytes if kv is not None else 0, kv_ctx, _ptr(c), len(c) // 8)


# tolerances of the reference (gemvq_ref.h:267-272, 399-402)
def within_tolerance(got, ref, mag) -> np.ndarray:
    got, ref, mag = (np.asarray(a, dtype=np.float64) for a in (got, ref, mag))
    return np.abs(got - ref) <= 1e-6 + 1e-5 * np.abs(ref) + 1e-6 * mag


def within_elementwise(got, ref) -> np.ndarray:
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return np.abs(got - ref) <= 1e-6 + 2e-5 * np.abs(ref)


# ---- the reference's own build -------------------------------------------------------------------------------------
def ref_gemv(w, x, rows, cols, fmt):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y, mag = np.zeros(rows, np.float32), np.zeros(rows, np.float64)
    ref().ref_gemv(_ptr(w), _ptr(x), rows, cols, fmt, _ptr(y), _ptr(mag))
    return y, mag


def ref_gemv_omp(w, x, rows, cols, fmt, slices):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, np.float32)
    ref().ref_gemv_rows_omp(_ptr(w), _ptr(x), rows, cols, fmt, _ptr(y), slices)
    return y
