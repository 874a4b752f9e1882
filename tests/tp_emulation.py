"""Runs the lists of several tensor-parallel ranks on the CPU oracle in lock step, doing their ALLREDUCE / ALLGATHER
commands between the lists' other commands (the oracle itself treats a collective as one rank's copy). Test helper
(TEST INFRASTRUCTURE ONLY): ALLREDUCE adds the ranks' x in rank order in FP32, ALLGATHER places rank r's x at
r * n."""
from __future__ import annotations

import numpy as np

OP_ALLREDUCE, OP_ALLGATHER = 15, 16


def split_at_collectives(cl: np.ndarray):
    """[(commands before a collective, the collective's 8 words or None), ...] of one list."""
    cmds = np.asarray(cl, np.uint32).reshape(-1, 8)
    out, start = [], 0
    for i, c in enumerate(cmds):
        if c[0] in (OP_ALLREDUCE, OP_ALLGATHER):
            out.append((cmds[start:i].reshape(-1), c))
            start = i + 1
    out.append((cmds[start:].reshape(-1), None))
    return out


def collective(cs, acts):
    """cs[r]: rank r's collective command (the same opcode and n on every rank; x and y are offsets in the rank's own
    act, which may differ between ranks whose lists place their tensors differently)."""
    op, n = int(cs[0][0]), int(cs[0][1])
    xs, ys = [int(c[2]) for c in cs], [int(c[3]) for c in cs]
    if op == OP_ALLREDUCE:
        s = acts[0][xs[0]:xs[0] + n].copy()
        for a, x in zip(acts[1:], xs[1:]):
            s = (s + a[x:x + n]).astype(np.float32)
        for a, y in zip(acts, ys):
            a[y:y + n] = s
    else:
        parts = [a[x:x + n].copy() for a, x in zip(acts, xs)]
        for a, y in zip(acts, ys):
            for r, p in enumerate(parts):
                a[y + r * n:y + (r + 1) * n] = p


def run_lists(orc, lists_per_rank, acts, ws, states, kvs, kv_ctx: int) -> None:
    """lists_per_rank[r]: rank r's lists (the same structure on every rank); acts / ws / states / kvs per rank."""
    for li in range(len(lists_per_rank[0])):
        segs = [split_at_collectives(lists[li]) for lists in lists_per_rank]
        assert len({len(s) for s in segs}) == 1, "ranks' lists differ in their collectives"
        for si in range(len(segs[0])):
            for r, sg in enumerate(segs):
                if sg[si][0].size:
                    st = orc.run_list(acts[r], sg[si][0], ws[r], state=states[r], kv=kvs[r], kv_ctx=kv_ctx)
                    assert st == 0, (r, li, si, st)
            cs = [sg[si][1] for sg in segs]
            if cs[0] is not None:
                assert all(c is not None and np.array_equal(c[[0, 1]], cs[0][[0, 1]]) for c in cs), "collectives differ"
                collective(cs, acts)
