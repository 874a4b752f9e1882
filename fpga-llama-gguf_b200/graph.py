"""Op graphs lowered to command lists (b200q_lower): a node builder over the library's b200q_node and the lowering's
result (lists, the act offset of every tensor, the act size). The graph is the form a framework holds a model's
token in (the reference's backend receives a ggml graph and does this step itself, ggml-xrt.cpp:1815-2745); the
lowering finds the fusions of the command ISA and places the tensors.

    g = Graph()
    x = g.input(2560)
    w = g.param(2560)
    xn = g.mul(g.rms_norm(x, 1e-6), w)            # a weighted norm; deferred into the GEMVs that read it
    y = g.mul_mat(xn, handle, Q4_0, 9216, 2560)
    low = g.lower()                               # low.lists, low.offset(x), low.act_floats
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import B200QError, lib

NODE_INPUT, NODE_PARAM, NODE_VIEW, NODE_MUL_MAT, NODE_RMS_NORM, NODE_L2_NORM, NODE_MUL, NODE_ADD, NODE_SWIGLU, \
    NODE_UNARY, NODE_CONV, NODE_GDN, NODE_ROPE, NODE_ATTN, NODE_GET_ROWS, NODE_ARGMAX, NODE_ALLREDUCE, \
    NODE_ALLGATHER = range(1, 19)
SEGMENT_END, OUTPUT, LIST_END = 1, 2, 4
SRCS = 6
ALL_FEATURES = 0x1FFFF  # word 0 bits 0..15 and the SIGMOID_MUL bit of word 1


class _Node(ctypes.Structure):
    _fields_ = [("op", ctypes.c_uint32), ("flags", ctypes.c_uint32), ("src", ctypes.c_int32 * SRCS),
                ("dst", ctypes.c_int32), ("n", ctypes.c_uint32), ("fmt", ctypes.c_uint32), ("rows", ctypes.c_uint32),
                ("cols", ctypes.c_uint32), ("weight", ctypes.c_uint64), ("eps", ctypes.c_float),
                ("u", ctypes.c_uint32 * 4)]


class Lowering:
    """The lists (uint32 arrays of 8-word commands), the act offset of each node (None when the tensor lives only
    inside a command) and the act floats the lists use."""

    def __init__(self, lists, offsets, act_floats):
        self.lists, self._off, self.act_floats = lists, offsets, act_floats

    def offset(self, node: int):
        return self._off[node]


class Graph:
    def __init__(self):
        self.nodes: list[dict] = []

    def _add(self, op, n, srcs=(), dst=-1, fmt=0, rows=0, cols=0, weight=0, eps=0.0, u=(), flags=0) -> int:
        self.nodes.append(dict(op=op, n=int(n), src=list(srcs), dst=dst, fmt=fmt, rows=rows, cols=cols,
                               weight=int(weight), eps=float(eps), u=list(u), flags=flags))
        return len(self.nodes) - 1

    def n(self, i: int) -> int:
        return self.nodes[i]["n"]

    # leaves and views
    def input(self, n: int) -> int:
        return self._add(NODE_INPUT, n)

    def param(self, n: int) -> int:
        return self._add(NODE_PARAM, n)

    def view(self, src: int, offset: int, row: int, stride: int = 0, rows: int = 1) -> int:
        return self._add(NODE_VIEW, row * rows, [src], u=[offset, row, stride or row, rows])

    # ops
    def mul_mat(self, x: int, weight: int, fmt: int, rows: int, cols: int, dst: int = -1, batch: int = 1) -> int:
        """y = W x; with batch > 1, x holds `batch` rows of cols floats and y `batch` rows of round16(rows) floats
        (one GEMV_BATCH command: the prompt's rows, on the tensor cores beyond 8)."""
        if batch > 1:
            return self._add(NODE_MUL_MAT, batch * ((rows + 15) // 16 * 16), [x], dst=dst, fmt=fmt, rows=rows,
                             cols=cols, weight=weight, u=[batch])
        return self._add(NODE_MUL_MAT, rows, [x], dst=dst, fmt=fmt, rows=rows, cols=cols, weight=weight)

    def rms_norm(self, x: int, eps: float, rows: int = 1) -> int:
        return self._add(NODE_RMS_NORM, self.n(x), [x], rows=rows, eps=eps)

    def l2_norm(self, x: int, eps: float, rows: int = 1) -> int:
        return self._add(NODE_L2_NORM, self.n(x), [x], rows=rows, eps=eps)

    def mul(self, a: int, b: int) -> int:
        return self._add(NODE_MUL, max(self.n(a), self.n(b)), [a, b])

    def add(self, a: int, b: int) -> int:
        return self._add(NODE_ADD, self.n(a), [a, b])

    def swiglu(self, g: int, u: int) -> int:
        return self._add(NODE_SWIGLU, self.n(g), [g, u])

    def unary(self, x: int, kind: int) -> int:
        return self._add(NODE_UNARY, self.n(x), [x], u=[kind])

    def conv(self, x: int, w: int, state: int, silu: bool = True) -> int:
        return self._add(NODE_CONV, self.n(x), [x, w, state], u=[1 if silu else 0])

    def gdn(self, q: int, k: int, v: int, g: int, beta: int, hv: int, hk: int, state_row: int, scale: float) -> int:
        return self._add(NODE_GDN, hv * 128, [q, k, v, g, beta], eps=scale, u=[hv, hk, state_row])

    def rope(self, x: int, cs: int, dims: int, row: int, rows: int) -> int:
        return self._add(NODE_ROPE, row * rows, [x, cs], u=[dims, row, rows])

    def attn(self, q: int, k: int, v: int, pos: int, n_head: int, n_kv: int, head_dim: int, slot: int) -> int:
        return self._add(NODE_ATTN, n_head * head_dim, [q, k, v, pos], u=[n_head, n_kv, head_dim, slot])

    def get_rows(self, idx: int, weight: int, fmt: int, cols: int, dst: int = -1) -> int:
        return self._add(NODE_GET_ROWS, cols, [idx], dst=dst, fmt=fmt, cols=cols, weight=weight)

    def argmax(self, x: int, dst: int = -1) -> int:
        return self._add(NODE_ARGMAX, 2, [x], dst=dst)

    def allreduce(self, x: int) -> int:
        return self._add(NODE_ALLREDUCE, self.n(x), [x])

    def allgather(self, x: int, world: int, dst: int = -1) -> int:
        return self._add(NODE_ALLGATHER, self.n(x) * world, [x], dst=dst)

    def end_segment(self) -> None:
        """The last node so far closes a segment (lists are cut between segments only)."""
        self.nodes[-1]["flags"] |= SEGMENT_END

    def end_list(self) -> None:
        """The last node so far closes a segment and the list (ranks of a tensor-parallel run cut at the same places)."""
        self.nodes[-1]["flags"] |= SEGMENT_END | LIST_END

    def mark_output(self, i: int) -> int:
        self.nodes[i]["flags"] |= OUTPUT
        return i

    def _array(self):
        arr = (_Node * len(self.nodes))()
        for i, d in enumerate(self.nodes):
            a = arr[i]
            a.op, a.flags, a.dst, a.n = d["op"], d["flags"], d["dst"], d["n"]
            for k in range(SRCS):
                a.src[k] = d["src"][k] if k < len(d["src"]) else -1
            a.fmt, a.rows, a.cols, a.weight, a.eps = d["fmt"], d["rows"], d["cols"], d["weight"], d["eps"]
            for k, v in enumerate(d["u"]):
                a.u[k] = v
        return arr

    def supported(self, i: int) -> bool:
        return bool(lib().b200q_node_supported(ctypes.cast(self._array(), ctypes.c_void_p), i))

    def lower(self, features: int = ALL_FEATURES) -> Lowering:
        arr = self._array()
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        rc = lib().b200q_lower(ctypes.cast(arr, ctypes.c_void_p), len(self.nodes), features, ctypes.byref(h), err, 512)
        if rc != 0:
            raise B200QError(rc, err.value.decode())
        try:
            L = lib()
            lists = []
            for i in range(L.b200q_lowering_lists(h)):
                n = ctypes.c_uint(0)
                p = L.b200q_lowering_list(h, i, ctypes.byref(n))
                lists.append(np.ctypeslib.as_array(p, shape=(n.value * 8,)).copy())
            none = ctypes.c_size_t(-1).value
            offs = [L.b200q_lowering_offset(h, i) for i in range(len(self.nodes))]
            offs = [None if o == none else int(o) for o in offs]
            return Lowering(lists, offs, int(L.b200q_lowering_act_floats(h)))
        finally:
            lib().b200q_lowering_free(h)
