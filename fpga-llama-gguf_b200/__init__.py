"""Python binding of libb200q (include/b200q.h): the B200 decode hot path behind the reference's command-list
interface (fpga/src/gemvqc16.h). This module is a thin ctypes layer over the C ABI; the host logic (planning,
validation, launches, CUDA Graphs, NCCL) and the kernels live in the shared library.

Command builders mirror the reference ISA word for word (fpga/src/gemvqc16.h:24-98): a list is a numpy uint32 array
of 8-word commands; `Context.run` returns what the reference's gemvqc16 returns (0, or the 1-based index of the first
invalid command, or 129 for more than 128 commands), and raises `B200QError` for host / CUDA failures.

The package directory name contains dashes, so import it with `load_package()` from the repository's tests / bench,
or by path with importlib.
"""
from __future__ import annotations

import ctypes
import os
import struct

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libb200q.so")

# ---- command ISA (reference fpga/src/gemvqc16.h:100-135) -------------------------------------------------------
CMD_WORDS = 8
MAX_CMDS = 128
OP_GEMV, OP_RMSNORM, OP_ADD, OP_SILU_MUL, OP_MUL, OP_UNARY, OP_GDN, OP_CONV = 1, 2, 3, 4, 5, 6, 7, 8
OP_STATE_LOAD, OP_ROPE, OP_TRACE = 9, 10, 11
OP_ATTN, OP_ARGMAX, OP_GET_ROW, OP_ALLREDUCE, OP_ALLGATHER = 12, 13, 14, 15, 16  # extensions of this library
OP_GEMV_BATCH = 17
BATCH_MAX = 8  # activation rows of one gemv_batch_kernel launch (more: the tensor-core GEMM)
GEMV_SWIGLU, GEMV_CONV, GEMV_ADD = 0x100, 0x200, 0x400
GDN_WITH_GEMV, GDN_L2_QK, GDN_GATED, GDN_GATES, GDN_WITH_OUT = 1, 2, 4, 8, 16
NORM_L2, NORM_NO_WEIGHT, NORM_DEFER = 1, 2, 4
UNARY_SILU, UNARY_SIGMOID, UNARY_SOFTPLUS, UNARY_COPY = 1, 2, 3, 4
SILU_MUL_SIGMOID = 1
Q4_0, Q4_1, Q8_0, Q5_K, Q6_K = 2, 3, 8, 13, 14
FEATURES = (0x6B51FFFF, 0x6B520001, 0x6B53007F)
COMM_EXPLICIT = 1
UPLOAD_REPLICATE = 1
UPLOAD_SRC_Q4_0X8 = 2


def UPLOAD_PASS_ROWS(n: int) -> int:
    """Upload flag: the matrix joins a multi-output pass of n rows in all (panel height chosen for the pass)."""
    return int(n) << 8

ERR = {-1: "bad argument", -2: "CUDA failure", -3: "out of memory", -4: "context disabled", -5: "NCCL failure",
       -6: "call out of order", -7: "bounded wait ran out", -8: "runtime verification failed"}


class B200QError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"b200q error {code} ({ERR.get(code, '?')}): {msg}")
        self.code = code


def fbits(x: float) -> int:
    """FP32 bits of x as an unsigned command word."""
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def cmd(*words: int) -> np.ndarray:
    w = list(words) + [0] * (CMD_WORDS - len(words))
    if len(w) != CMD_WORDS:
        raise ValueError("a command has 8 words")
    return np.array([int(v) & 0xFFFFFFFF for v in w], dtype=np.uint32)


def cmd_list(*cmds: np.ndarray) -> np.ndarray:
    return np.concatenate([np.asarray(c, dtype=np.uint32).reshape(-1) for c in cmds]) if cmds else \
        np.zeros(0, dtype=np.uint32)


def gemv(fmt: int, rows: int, cols: int, w_off: int, x_off: int, y_off: int, flags: int = 0) -> np.ndarray:
    return cmd(OP_GEMV, fmt | flags, rows, cols, w_off & 0xFFFFFFFF, w_off >> 32, x_off, y_off)


def rmsnorm(n: int, x_off: int, w_off: int, y_off: int, eps: float, rows: int = 0, flags: int = 0,
            stride_words: int = 0) -> np.ndarray:
    return cmd(OP_RMSNORM, n, x_off, w_off, y_off, fbits(eps), rows, flags | (stride_words << 8))


def add(n: int, a: int, b: int, y: int) -> np.ndarray:
    return cmd(OP_ADD, n, a, b, y)


def mul(n: int, a: int, b: int, y: int) -> np.ndarray:
    return cmd(OP_MUL, n, a, b, y)


def silu_mul(n: int, g: int, u: int, y: int, sigmoid: bool = False, row: int = 0, stride: int = 0) -> np.ndarray:
    return cmd(OP_SILU_MUL, n, g, u, y, SILU_MUL_SIGMOID if sigmoid else 0, row, stride)


def unary(n: int, x: int, kind: int, y: int, row: int = 0, stride: int = 0) -> np.ndarray:
    return cmd(OP_UNARY, n, x, kind, y, row, stride)


def conv(ch: int, x: int, w: int, y: int, s_src: int, s_dst: int, use_silu: bool = True) -> np.ndarray:
    return cmd(OP_CONV, ch, x, w, y, s_src, s_dst, 1 if use_silu else 0)


def rope(n_dims: int, x: int, cs: int, y: int, ne0: int, rows: int) -> np.ndarray:
    return cmd(OP_ROPE, n_dims, x, cs, y, ne0, rows)


def state_load(hv: int, src_row: int) -> np.ndarray:
    return cmd(OP_STATE_LOAD, hv, src_row)


def trace(log_off: int) -> np.ndarray:
    return cmd(OP_TRACE, log_off)


def gdn(hv: int, hk: int, q: int, k: int, v: int, g: int, beta: int, y: int, src_row: int, dst_row: int,
        scale: float, flags: int = 0, l2_eps: float = 1e-6, rms_eps: float = 1e-6, w_off: int = 0, z_off: int = 0,
        dt_off: int = 0, a_off: int = 0) -> np.ndarray:
    """GDN step: two slots, or three with GDN_GATES (reference gemvqc16.h:60-81)."""
    slots = [cmd(OP_GDN, hv | (hk << 16), q, k, v, g, beta, y),
             cmd(src_row, dst_row, fbits(scale), flags, fbits(l2_eps), fbits(rms_eps), w_off, z_off)]
    if flags & GDN_GATES:
        slots.append(cmd(dt_off, a_off))
    return cmd_list(*slots)


def attn(n_head: int, n_kv: int, head_dim: int, q: int, k: int, v: int, y: int, pos_off: int, slot: int) -> np.ndarray:
    """ATTN extension; the token position is read from act[pos_off] (uint32 bits)."""
    return cmd(OP_ATTN, n_head | (n_kv << 8) | ((head_dim // 16) << 16), q, k, v, y, pos_off, slot)


def argmax(n: int, x: int, y: int) -> np.ndarray:
    return cmd(OP_ARGMAX, n, x, y)


def get_row(fmt: int, cols: int, w_off: int, idx_off: int, y_off: int) -> np.ndarray:
    return cmd(OP_GET_ROW, fmt, cols, w_off & 0xFFFFFFFF, w_off >> 32, idx_off, y_off)


def allreduce(n: int, x_off: int, y_off: int) -> np.ndarray:
    """ALLREDUCE extension: y = the sum over the communicator's ranks of their x (one rank: y = x)."""
    return cmd(OP_ALLREDUCE, n, x_off, y_off)


def allgather(n: int, x_off: int, y_off: int) -> np.ndarray:
    """ALLGATHER extension: y[r n .. r n + n) = x of rank r (one rank: y = x)."""
    return cmd(OP_ALLGATHER, n, x_off, y_off)


def gemv_batch(fmt: int, rows: int, cols: int, w_off: int, x_off: int, y_off: int, batch: int,
               flags: int = 0) -> np.ndarray:
    """GEMV_BATCH extension: y_m = W x_m (flags GEMV_ADD: + y_m) for m < batch <= 65536; x rows `cols` floats apart
    from x_off, y rows round16(rows) floats apart from y_off. Up to BATCH_MAX rows one kernel reads the weights once
    for all rows; more rows run as the tensor-core GEMM (prefill)."""
    return cmd(OP_GEMV_BATCH, fmt | flags | ((batch - 1) << 16), rows, cols, w_off & 0xFFFFFFFF, w_off >> 32,
               x_off, y_off)


# ---- library ---------------------------------------------------------------------------------------------------
class _Config(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("weight_bytes", ctypes.c_size_t), ("act_floats", ctypes.c_size_t),
                ("state_rows", ctypes.c_size_t), ("kv_bytes", ctypes.c_size_t), ("kv_ctx", ctypes.c_uint)]


class _PassInfo(ctypes.Structure):
    _fields_ = [("first_cmd", ctypes.c_uint32), ("n_cmds", ctypes.c_uint32), ("kind", ctypes.c_uint32),
                ("n_members", ctypes.c_uint32), ("fused_norm", ctypes.c_uint32)]


PASS_KINDS = {1: "gemv", 2: "elementwise", 3: "gdn", 4: "nop", 5: "ext"}

_lib = None


class VerifyView(ctypes.Structure):
    """b200q_verify_view: what a runtime-verification checker receives."""
    _fields_ = [("cmds", ctypes.POINTER(ctypes.c_uint32)), ("n_cmds", ctypes.c_uint), ("status", ctypes.c_int),
                ("act_before", ctypes.POINTER(ctypes.c_float)), ("act_after", ctypes.POINTER(ctypes.c_float)),
                ("act_floats", ctypes.c_size_t), ("state_before", ctypes.POINTER(ctypes.c_float)),
                ("state_after", ctypes.POINTER(ctypes.c_float)), ("state_rows", ctypes.c_size_t),
                ("kv_before", ctypes.c_void_p), ("kv_after", ctypes.c_void_p), ("kv_bytes", ctypes.c_size_t),
                ("kv_ctx", ctypes.c_uint)]


VERIFY_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(VerifyView), ctypes.c_void_p, ctypes.c_uint)
MASK_GROUPS, MASK_DEFER_NORM, MASK_GDN_OUT = 1 << 3, 1 << 9, 1 << 15
MASK_X_IMAGE, MASK_NORM_PARTIALS, MASK_PDL, MASK_ROW_OPS, MASK_ATTN_GATE = 1 << 16, 1 << 17, 1 << 18, 1 << 19, 1 << 20
MASK_CHAINS = 1 << 21
DEFAULT_FEATURE_MASK = 0xFFFFFFFF & ~MASK_CHAINS
ERR_VERIFY = -8


def lib() -> ctypes.CDLL:
    """The loaded libb200q.so; raises if it has not been built (there is no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python __graft_entry__.py` or make -C csrc")
    L = ctypes.CDLL(LIB_PATH)
    P, U32, U, I, SZ = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint, ctypes.c_int, ctypes.c_size_t
    sig = {
        "b200q_create": (I, [ctypes.POINTER(_Config), ctypes.POINTER(P)]),
        "b200q_destroy": (None, [P]),
        "b200q_last_error": (ctypes.c_char_p, [P]),
        "b200q_stream": (P, [P]),
        "b200q_synchronize": (I, [P]),
        "b200q_act_device_ptr": (P, [P]),
        "b200q_state_device_ptr": (P, [P]),
        "b200q_kv_device_ptr": (P, [P]),
        "b200q_features": (None, [P]),
        "b200q_upload_weight": (I, [P, P, U, U, U, U, ctypes.POINTER(ctypes.c_uint64)]),
        "b200q_upload_weight_ex": (I, [P, P, U, U, U, U, U, ctypes.POINTER(ctypes.c_uint64)]),
        "b200q_weight_device_bytes": (SZ, [U, U, U]),
        "b200q_weight_device_bytes_ex": (SZ, [U, U, U, U]),
        "b200q_gguf_row_bytes": (SZ, [U, U]),
        "b200q_weights_reset": (I, [P]),
        "b200q_act_write": (I, [P, SZ, P, SZ]),
        "b200q_act_read": (I, [P, SZ, P, SZ]),
        "b200q_act_fill": (I, [P, SZ, ctypes.c_float, SZ]),
        "b200q_act_write_async": (I, [P, SZ, P, SZ]),
        "b200q_act_read_async": (I, [P, SZ, P, SZ]),
        "b200q_state_write": (I, [P, SZ, P, SZ]),
        "b200q_state_read": (I, [P, SZ, P, SZ]),
        "b200q_kv_write": (I, [P, SZ, P, SZ]),
        "b200q_run": (I, [P, P, U]),
        "b200q_run_async": (I, [P, P, U]),
        "b200q_graph_create": (I, [P, P, U, ctypes.POINTER(P)]),
        "b200q_graph_launch": (I, [P, P]),
        "b200q_graph_destroy": (None, [P]),
        "b200q_graph_kernel_count": (U, [P]),
        "b200q_graph_launch_many": (I, [P, P, U, U]),
        "b200q_plan": (I, [P, U, P, U, ctypes.POINTER(U)]),
        "b200q_debug_quantize": (I, [P, U, SZ, U, U32, ctypes.c_float, U, P, P, P]),
        "b200q_debug_block_sums": (I, [P, P, P]),
        "b200q_quantize_noalloc": (I, [I, P, U, U, P, ctypes.c_float, U, P, P, P, P, ctypes.c_char_p, U]),
        "b200q_comm_unique_id": (I, [P]),
        "b200q_comm_init": (I, [P, I, I, P]),
        "b200q_comm_init_ex": (I, [P, I, I, P, U]),
        "b200q_comm_world": (I, [P]),
        "b200q_row_slice": (I, [U, U, I, I, ctypes.POINTER(U), ctypes.POINTER(U)]),
        "b200q_layout": (I, [U, U, U, U, P]),
        "b200q_layout_ex": (I, [U, U, U, U, U, P]),
        "b200q_repack_host": (I, [P, U, U, U, U, P]),
        "b200q_unpack_row_host": (I, [P, U, U, U, U, U, P]),
        "b200q_gguf_open": (I, [ctypes.c_char_p, ctypes.POINTER(P), ctypes.c_char_p, U]),
        "b200q_gguf_close": (None, [P]),
        "b200q_gguf_version": (U32, [P]),
        "b200q_gguf_n_tensors": (ctypes.c_uint64, [P]),
        "b200q_gguf_n_kv": (ctypes.c_uint64, [P]),
        "b200q_gguf_tensor": (I, [P, ctypes.c_uint64, P]),
        "b200q_gguf_find_tensor": (I, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)]),
        "b200q_gguf_kv": (I, [P, ctypes.c_uint64, P]),
        "b200q_gguf_find_kv": (I, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)]),
        "b200q_gguf_get_int": (I, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]),
        "b200q_gguf_get_float": (I, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
        "b200q_upload_gguf_tensor": (I, [P, P, ctypes.c_uint64, U, U, ctypes.POINTER(ctypes.c_uint64)]),
        "b200q_q4_0x8_to_q4_0": (I, [P, U, U, P]),
        "b200q_set_feature_mask": (I, [P, U32]),
        "b200q_feature_mask": (U32, [P]),
        "b200q_set_verify": (I, [P, VERIFY_FN, P, I]),
        "b200q_lower": (I, [P, U, U32, ctypes.POINTER(P), ctypes.c_char_p, U]),
        "b200q_lowering_free": (None, [P]),
        "b200q_lowering_lists": (U, [P]),
        "b200q_lowering_list": (ctypes.POINTER(U32), [P, U, ctypes.POINTER(U)]),
        "b200q_lowering_offset": (SZ, [P, U]),
        "b200q_lowering_act_floats": (SZ, [P]),
        "b200q_node_supported": (I, [P, U]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


EXPORTED = ["b200q_create", "b200q_destroy", "b200q_last_error", "b200q_stream", "b200q_synchronize",
            "b200q_act_device_ptr", "b200q_state_device_ptr", "b200q_kv_device_ptr", "b200q_features",
            "b200q_upload_weight", "b200q_upload_weight_ex", "b200q_weight_device_bytes", "b200q_weight_device_bytes_ex",
            "b200q_gguf_row_bytes",
            "b200q_weights_reset", "b200q_act_write", "b200q_act_read", "b200q_act_fill", "b200q_act_write_async",
            "b200q_act_read_async", "b200q_state_write",
            "b200q_state_read", "b200q_kv_write", "b200q_run", "b200q_run_async", "b200q_graph_create",
            "b200q_graph_launch", "b200q_graph_launch_many", "b200q_graph_destroy", "b200q_graph_kernel_count", "b200q_plan",
            "b200q_debug_quantize", "b200q_debug_block_sums", "b200q_quantize_noalloc", "b200q_comm_unique_id",
            "b200q_comm_init",
            "b200q_comm_world", "b200q_row_slice", "b200q_layout", "b200q_layout_ex", "b200q_repack_host", "b200q_unpack_row_host",
            "b200q_gguf_open", "b200q_gguf_close", "b200q_gguf_version", "b200q_gguf_n_tensors", "b200q_gguf_n_kv",
            "b200q_gguf_tensor", "b200q_gguf_find_tensor", "b200q_gguf_kv", "b200q_gguf_find_kv", "b200q_gguf_get_int",
            "b200q_gguf_get_float", "b200q_upload_gguf_tensor", "b200q_q4_0x8_to_q4_0", "b200q_set_feature_mask",
            "b200q_feature_mask", "b200q_set_verify", "b200q_comm_init_ex", "b200q_lower", "b200q_lowering_free",
            "b200q_lowering_lists", "b200q_lowering_list", "b200q_lowering_offset", "b200q_lowering_act_floats",
            "b200q_node_supported"]


class _LayoutInfo(ctypes.Structure):
    _fields_ = [("rows_per_tile", ctypes.c_uint32), ("blocks_per_tile", ctypes.c_uint32),
                ("tiles_per_row_tile", ctypes.c_uint32), ("row_tiles", ctypes.c_uint32),
                ("tile_bytes", ctypes.c_uint32), ("total_bytes", ctypes.c_uint64)]


def layout(rows: int, cols: int, fmt: int, sms: int = 148, flags: int = 0) -> dict:
    info = _LayoutInfo()
    if lib().b200q_layout_ex(rows, cols, fmt, sms, flags, ctypes.byref(info)) != 0:
        raise ValueError("unsupported shape or format")
    return {f: int(getattr(info, f)) for f, _ in _LayoutInfo._fields_}


def repack_host(gguf: np.ndarray, rows: int, cols: int, fmt: int, sms: int = 148) -> np.ndarray:
    src = np.ascontiguousarray(gguf, dtype=np.uint8)
    out = np.zeros(layout(rows, cols, fmt, sms)["total_bytes"], dtype=np.uint8)
    if lib().b200q_repack_host(src.ctypes.data_as(ctypes.c_void_p), rows, cols, fmt, sms,
                               out.ctypes.data_as(ctypes.c_void_p)) != 0:
        raise ValueError("repack failed")
    return out


def unpack_row_host(dev: np.ndarray, rows: int, cols: int, fmt: int, row: int, sms: int = 148) -> np.ndarray:
    out = np.zeros(gguf_row_bytes(cols, fmt), dtype=np.uint8)
    d = np.ascontiguousarray(dev, dtype=np.uint8)
    if lib().b200q_unpack_row_host(d.ctypes.data_as(ctypes.c_void_p), rows, cols, fmt, sms, row,
                                   out.ctypes.data_as(ctypes.c_void_p)) != 0:
        raise ValueError("unpack failed")
    return out


def features() -> tuple:
    out = (ctypes.c_uint32 * 3)()
    lib().b200q_features(out)
    return tuple(out)


def plan(cmds: np.ndarray, max_passes: int = 256):
    """Host-only planning (no GPU): (status, [pass dicts]) as the device run would execute the list."""
    c = np.ascontiguousarray(cmds, dtype=np.uint32)
    infos = (_PassInfo * max_passes)()
    n = ctypes.c_uint(0)
    st = lib().b200q_plan(c.ctypes.data_as(ctypes.c_void_p), len(c) // CMD_WORDS, infos, max_passes,
                          ctypes.byref(n))
    passes = [dict(first=p.first_cmd, count=p.n_cmds, kind=PASS_KINDS.get(p.kind, "?"), members=p.n_members,
                   fused_norm=bool(p.fused_norm), stored_norm=p.fused_norm == 2)
              for p in infos[: min(n.value, max_passes)]]
    return st, passes


NOALLOC_MAX_N = 16384


def quantize_noalloc(device: int, x_ptr: int, n: int, fmt: int, norm_w_ptr: int | None = None, eps: float = 0.0,
                     norm_flags: int = 0, stream: int | None = None):
    """b200q_quantize_noalloc: n device floats at x_ptr quantized as a GEMV pass of format `fmt` would, without a
    context and without allocating device memory (n <= NOALLOC_MAX_N). Returns (q, scales, bsums) as
    Context.debug_quantize does."""
    q = np.zeros(n, dtype=np.int8)
    act = 2 if fmt in (Q5_K, Q6_K) else (1 if fmt == Q4_1 else 0)
    if act == 2:
        scales = np.zeros(max(n // 256, 1), dtype=np.float32)
        bs = np.zeros(max(n // 16, 1), dtype=np.int32)
    else:
        scales = np.zeros(max(n // 32, 1) * (2 if act == 1 else 1), dtype=np.uint16)
        bs = np.zeros(max(n // 32, 1), dtype=np.int32)
    err = ctypes.create_string_buffer(256)
    rc = lib().b200q_quantize_noalloc(device, x_ptr, n, fmt, norm_w_ptr, eps, norm_flags, stream,
                                      q.ctypes.data_as(ctypes.c_void_p), scales.ctypes.data_as(ctypes.c_void_p),
                                      bs.ctypes.data_as(ctypes.c_void_p), err, len(err))
    if rc != 0:
        raise B200QError(rc, err.value.decode() or ERR.get(rc, str(rc)))
    return q, scales, bs


def row_slice(rows: int, world: int, rank: int, flags: int = 0) -> tuple:
    """The rows (r0, r1) of a matrix that `rank` keeps in a row-sharded context of `world` ranks (host only)."""
    r0, r1 = ctypes.c_uint(), ctypes.c_uint()
    rc = lib().b200q_row_slice(rows, flags, world, rank, ctypes.byref(r0), ctypes.byref(r1))
    if rc != 0:
        raise B200QError(rc, "bad world / rank")
    return int(r0.value), int(r1.value)


class _GgufTensorInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_uint32), ("n_dims", ctypes.c_uint32),
                ("ne", ctypes.c_uint64 * 4), ("offset", ctypes.c_uint64), ("bytes", ctypes.c_uint64),
                ("data", ctypes.c_void_p)]


class _GgufKvInfo(ctypes.Structure):
    _fields_ = [("key", ctypes.c_char_p), ("type", ctypes.c_uint32), ("array_type", ctypes.c_uint32),
                ("count", ctypes.c_uint64), ("value", ctypes.c_void_p), ("str_len", ctypes.c_uint64)]


class GgufFile:
    """A .gguf file opened by the library's reader (b200q_gguf_open): tensor table, metadata, and tensor data as
    numpy views of the read-only mapping (valid until close)."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        rc = lib().b200q_gguf_open(os.fsencode(path), ctypes.byref(h), err, len(err))
        if rc != 0:
            raise B200QError(rc, err.value.decode())
        self.h = h

    def close(self):
        if self.h:
            lib().b200q_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def version(self) -> int:
        return int(lib().b200q_gguf_version(self.h))

    def tensor(self, index: int) -> dict:
        t = _GgufTensorInfo()
        if lib().b200q_gguf_tensor(self.h, index, ctypes.byref(t)) != 0:
            raise IndexError(index)
        data = None
        if t.data and t.bytes:
            data = np.ctypeslib.as_array(ctypes.cast(t.data, ctypes.POINTER(ctypes.c_uint8)), shape=(t.bytes,))
        return {"name": t.name.decode(), "type": t.type, "n_dims": t.n_dims, "ne": list(t.ne)[:max(1, t.n_dims)],
                "offset": t.offset, "bytes": t.bytes, "data": data}

    def tensors(self) -> list:
        return [self.tensor(i) for i in range(int(lib().b200q_gguf_n_tensors(self.h)))]

    def find(self, name: str) -> int:
        i = ctypes.c_uint64()
        if lib().b200q_gguf_find_tensor(self.h, name.encode(), ctypes.byref(i)) != 0:
            raise KeyError(name)
        return int(i.value)

    def keys(self) -> list:
        out = []
        for i in range(int(lib().b200q_gguf_n_kv(self.h))):
            kv = _GgufKvInfo()
            lib().b200q_gguf_kv(self.h, i, ctypes.byref(kv))
            out.append(kv.key.decode())
        return out

    def get_int(self, key: str) -> int:
        v = ctypes.c_int64()
        if lib().b200q_gguf_get_int(self.h, key.encode(), ctypes.byref(v)) != 0:
            raise KeyError(key)
        return int(v.value)

    def get_float(self, key: str) -> float:
        v = ctypes.c_double()
        if lib().b200q_gguf_get_float(self.h, key.encode(), ctypes.byref(v)) != 0:
            raise KeyError(key)
        return float(v.value)

    def get_str(self, key: str) -> str:
        i = ctypes.c_uint64()
        if lib().b200q_gguf_find_kv(self.h, key.encode(), ctypes.byref(i)) != 0:
            raise KeyError(key)
        kv = _GgufKvInfo()
        lib().b200q_gguf_kv(self.h, i.value, ctypes.byref(kv))
        if kv.type != 8:
            raise TypeError(f"{key} is not a string")
        return ctypes.string_at(kv.value, kv.str_len).decode()


def q4_0x8_to_q4_0(src: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Q4_0 rows back from ggml's CPU_REPACK block_q4_0x8 layout (b200q_q4_0x8_to_q4_0)."""
    src = np.ascontiguousarray(src, dtype=np.uint8).reshape(-1)
    out = np.zeros((rows, cols // 32 * 18), np.uint8)
    rc = lib().b200q_q4_0x8_to_q4_0(src.ctypes.data_as(ctypes.c_void_p), rows, cols,
                                    out.ctypes.data_as(ctypes.c_void_p))
    if rc != 0:
        raise B200QError(rc, "q4_0x8_to_q4_0: rows must be a multiple of 8, cols of 32")
    return out


def gguf_row_bytes(cols: int, fmt: int) -> int:
    return int(lib().b200q_gguf_row_bytes(cols, fmt))


def weight_device_bytes(rows: int, cols: int, fmt: int, flags: int = 0) -> int:
    """Device bytes of one uploaded matrix (its repacked layout), before the arena's 256-byte rounding."""
    return int(lib().b200q_weight_device_bytes_ex(rows, cols, fmt, flags))


class Graph:
    def __init__(self, ctx: "Context", handle: int):
        self.ctx, self.handle = ctx, handle

    @property
    def kernels(self) -> int:
        return int(lib().b200q_graph_kernel_count(self.handle))

    def launch(self):
        self.ctx._check(lib().b200q_graph_launch(self.ctx.h, self.handle))

    def close(self):
        if self.handle:
            lib().b200q_graph_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Context:
    """One device context: weight arena, act (FP32 activations), DeltaNet state rows, F16 KV cache, stream."""

    def __init__(self, device: int = 0, weight_bytes: int = 1 << 30, act_floats: int = 1 << 20,
                 state_rows: int = 0, kv_bytes: int = 0, kv_ctx: int = 0):
        cfg = _Config(device, weight_bytes, act_floats, state_rows, kv_bytes, kv_ctx)
        h = ctypes.c_void_p()
        rc = lib().b200q_create(ctypes.byref(cfg), ctypes.byref(h))
        if rc != 0:
            raise B200QError(rc, "b200q_create failed")
        self.h = h.value
        self.act_floats, self.state_rows, self.kv_bytes, self.kv_ctx = act_floats, state_rows, kv_bytes, kv_ctx

    def close(self):
        if getattr(self, "h", None):
            lib().b200q_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def last_error(self) -> str:
        s = lib().b200q_last_error(self.h)
        return s.decode() if s else ""

    def _check(self, rc: int) -> int:
        if rc < 0:
            raise B200QError(rc, self.last_error())
        return rc

    # buffers
    @property
    def stream(self) -> int:
        return int(lib().b200q_stream(self.h) or 0)

    @property
    def act_ptr(self) -> int:
        return int(lib().b200q_act_device_ptr(self.h))

    @property
    def kv_ptr(self) -> int:
        return int(lib().b200q_kv_device_ptr(self.h) or 0)

    def synchronize(self):
        self._check(lib().b200q_synchronize(self.h))

    def launch_many(self, graphs, launches: int) -> None:
        """graphs[i % len(graphs)] for i < launches, launched from C on the context stream."""
        arr = (ctypes.c_void_p * len(graphs))(*[g.handle for g in graphs])
        self._check(lib().b200q_graph_launch_many(self.h, arr, len(graphs), launches))

    def upload(self, gguf: np.ndarray, rows: int, cols: int, fmt: int, block_cols: int = 0, flags: int = 0) -> int:
        data = np.ascontiguousarray(gguf, dtype=np.uint8)
        if data.size != rows * gguf_row_bytes(cols, fmt):  # (a Q4_0x8 source has the same byte count)
            raise ValueError("GGUF byte count does not match rows x cols of the format")
        off = ctypes.c_uint64()
        self._check(lib().b200q_upload_weight_ex(self.h, data.ctypes.data_as(ctypes.c_void_p), rows, cols, fmt,
                                                 block_cols, flags, ctypes.byref(off)))
        return int(off.value)

    def upload_gguf(self, f: "GgufFile", name: str, block_cols: int = 0, flags: int = 0) -> int:
        """b200q_upload_gguf_tensor: the named 2-D tensor of an open GGUF file, uploaded straight from its mapping."""
        off = ctypes.c_uint64()
        self._check(lib().b200q_upload_gguf_tensor(self.h, f.h, f.find(name), block_cols, flags, ctypes.byref(off)))
        return int(off.value)

    def reset_weights(self):
        self._check(lib().b200q_weights_reset(self.h))

    def set_feature_mask(self, mask: int) -> None:
        """b200q_set_feature_mask: hide fused forms from the feature probe and switch the executor's fusions off."""
        self._check(lib().b200q_set_feature_mask(self.h, mask & 0xFFFFFFFF))

    @property
    def feature_mask(self) -> int:
        return int(lib().b200q_feature_mask(self.h))

    def set_verify(self, checker, n_calls: int) -> None:
        """b200q_set_verify: checker(view: VerifyView) -> (ok: bool, message: str) is called after each of the next
        n_calls lists (b200q_run or graph replays) with host copies of act / state / KV before and after; checker None
        turns verification off."""
        if checker is None:
            self._verify_cb = None
            self._check(lib().b200q_set_verify(self.h, VERIFY_FN(), None, 0))
            return

        def cb(_user, view, msg, msg_len):
            try:
                ok, text = checker(view.contents)
            except Exception as e:  # a checker that raises counts as a disagreement
                ok, text = False, f"checker raised {e!r}"
            if not ok:
                data = text.encode()[: max(0, msg_len - 1)] + b"\0"
                ctypes.memmove(msg, data, len(data))
            return 0 if ok else 1

        self._verify_cb = VERIFY_FN(cb)  # kept alive as long as the context may call it
        self._check(lib().b200q_set_verify(self.h, self._verify_cb, None, n_calls))

    def write(self, off: int, x) -> None:
        a = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        self._check(lib().b200q_act_write(self.h, off, a.ctypes.data_as(ctypes.c_void_p), a.size))

    def read(self, off: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self._check(lib().b200q_act_read(self.h, off, out.ctypes.data_as(ctypes.c_void_p), n))
        return out

    def write_async(self, off: int, host_ptr: int, n: int) -> None:
        """Stream-ordered copy of n floats at host_ptr (page-locked memory for no wait) into act[off:]; the buffer
        must stay untouched until synchronize()."""
        self._check(lib().b200q_act_write_async(self.h, off, host_ptr, n))

    def read_async(self, off: int, host_ptr: int, n: int) -> None:
        """Stream-ordered copy of act[off:off + n] to host_ptr; valid after synchronize()."""
        self._check(lib().b200q_act_read_async(self.h, off, host_ptr, n))

    def fill(self, off: int, value: float, n: int) -> None:
        self._check(lib().b200q_act_fill(self.h, off, value, n))

    def write_state(self, row: int, s) -> None:
        a = np.ascontiguousarray(s, dtype=np.float32).reshape(-1)
        if a.size % 128:
            raise ValueError("state rows are 128 floats")
        self._check(lib().b200q_state_write(self.h, row, a.ctypes.data_as(ctypes.c_void_p), a.size // 128))

    def read_state(self, row: int, rows: int) -> np.ndarray:
        out = np.empty(rows * 128, dtype=np.float32)
        self._check(lib().b200q_state_read(self.h, row, out.ctypes.data_as(ctypes.c_void_p), rows))
        return out

    def write_kv(self, byte_off: int, data: np.ndarray) -> None:
        a = np.ascontiguousarray(data)
        self._check(lib().b200q_kv_write(self.h, byte_off, a.ctypes.data_as(ctypes.c_void_p), a.nbytes))

    # lists
    def run(self, cmds: np.ndarray) -> int:
        c = np.ascontiguousarray(cmds, dtype=np.uint32)
        return self._check(lib().b200q_run(self.h, c.ctypes.data_as(ctypes.c_void_p), len(c) // CMD_WORDS))

    def run_async(self, cmds: np.ndarray) -> int:
        c = np.ascontiguousarray(cmds, dtype=np.uint32)
        return self._check(lib().b200q_run_async(self.h, c.ctypes.data_as(ctypes.c_void_p), len(c) // CMD_WORDS))

    def graph(self, cmds: np.ndarray) -> Graph:
        c = np.ascontiguousarray(cmds, dtype=np.uint32)
        g = ctypes.c_void_p()
        rc = self._check(lib().b200q_graph_create(self.h, c.ctypes.data_as(ctypes.c_void_p), len(c) // CMD_WORDS,
                                                  ctypes.byref(g)))
        if rc != 0:
            raise B200QError(-1, f"list rejected at command {rc}: {self.last_error()}")
        return Graph(self, g.value)

    # bit-exact intermediate values
    def debug_quantize(self, fmt: int, x_off: int, n: int, norm_w_off: int | None = None, eps: float = 0.0,
                       norm_flags: int = 0):
        q = np.zeros(n, dtype=np.int8)
        act = 2 if fmt in (Q5_K, Q6_K) else (1 if fmt == Q4_1 else 0)
        if act == 2:
            scales = np.zeros(n // 256, dtype=np.float32)
            bs = np.zeros(n // 16, dtype=np.int32)
        else:
            scales = np.zeros(n // 32 * (2 if act == 1 else 1), dtype=np.uint16)
            bs = np.zeros(n // 32, dtype=np.int32)
        self._check(lib().b200q_debug_quantize(
            self.h, fmt, x_off, n, 0xFFFFFFFF if norm_w_off is None else norm_w_off, eps, norm_flags,
            q.ctypes.data_as(ctypes.c_void_p), scales.ctypes.data_as(ctypes.c_void_p),
            bs.ctypes.data_as(ctypes.c_void_p)))
        return q, scales, bs

    def debug_block_sums(self, command: np.ndarray) -> np.ndarray:
        """Integer block sums of one GEMV command (rows x blocks), or of a GEMV_BATCH command of more than
        BATCH_MAX rows: block 0 of weight rows 0..127 x batch rows 0..127 (a 128 x 128 array, the GEMM's MMA)."""
        c = np.ascontiguousarray(command, dtype=np.uint32)
        fmt, rows, cols = int(c[1]) & 0xFF, int(c[2]), int(c[3])
        if int(c[0]) == OP_GEMV_BATCH and (int(c[1]) >> 16) + 1 > BATCH_MAX:
            out = np.zeros(128 * 128, dtype=np.int32)
            self._check(lib().b200q_debug_block_sums(self.h, c.ctypes.data_as(ctypes.c_void_p),
                                                     out.ctypes.data_as(ctypes.c_void_p)))
            return out.reshape(128, 128)
        n = rows * (cols // 256) * 9 if fmt in (Q5_K, Q6_K) else rows * (cols // 32)
        out = np.zeros(n, dtype=np.int32)
        self._check(lib().b200q_debug_block_sums(self.h, c.ctypes.data_as(ctypes.c_void_p),
                                                 out.ctypes.data_as(ctypes.c_void_p)))
        return out

    # multi-GPU
    @staticmethod
    def unique_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        rc = lib().b200q_comm_unique_id(buf)
        if rc != 0:
            raise B200QError(rc, "ncclGetUniqueId failed")
        return bytes(buf)

    def comm_init(self, world: int, rank: int, uid: bytes, flags: int = 0) -> None:
        """b200q_comm_init_ex: flags 0 row-shards uploads and gathers outputs by itself; COMM_EXPLICIT takes each
        rank's own lists (ALLREDUCE / ALLGATHER commands)."""
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
        self._check(lib().b200q_comm_init_ex(self.h, world, rank, buf, flags))
