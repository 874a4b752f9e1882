"""Host planner (no GPU): list validation gives the status the reference command processor gives
(fpga/src/gemvqc16.cpp:553-958), checked against the oracle's command-by-command interpreter; pass structure
(GEMV groups, SwiGLU pairs, epilogues, deferred norm, GDN slots)."""
import numpy as np
import pytest

from conftest import rng

X, Y, Z = 0, 4096, 8192


def weights(synth):
    r = rng(30)
    ws = {}
    for h, (fmt, rows, cols) in enumerate([(2, 64, 256), (2, 64, 256), (8, 64, 256), (3, 32, 256),
                                           (13, 48, 512), (14, 48, 512), (2, 32, 256)]):
        ws[1000 + 4096 * h] = (synth.matrix(fmt, r, rows, cols).reshape(-1), rows, cols, fmt)
    return ws


def oracle_status(orc, cmds, ws):
    act = rng(31).normal(0, 1, 1 << 15).astype(np.float32)
    state = np.zeros(64 * 128 * 128 // 128 * 128, np.float32)
    return orc.run_list(act, cmds, ws, state=state)


def test_group_pair_epilogue_structure(b2):
    g = b2.gemv
    cl = b2.cmd_list(
        b2.rmsnorm(256, X, 256, 512, 1e-6, flags=b2.NORM_DEFER),
        g(2, 64, 256, 1000, 512, Y, b2.GEMV_SWIGLU), g(2, 64, 256, 5096, 512, Y + 64),
        g(8, 64, 256, 9192, 512, Y + 128), g(2, 32, 256, 25576, 512, Y + 192),
        g(2, 64, 256, 1000, Y + 64, Z, b2.GEMV_ADD), b2.add(64, Z, 256, Z + 64),
        g(2, 64, 256, 1000, 0, Z + 128, b2.GEMV_CONV), b2.conv(64, Z + 128, 1024, Z + 256, 2048, 2048))
    st, passes = b2.plan(cl)
    assert st == 0
    kinds = [(p["kind"], p["first"], p["count"], p["members"]) for p in passes]
    assert kinds[0] == ("nop", 0, 1, 0)
    assert kinds[1] == ("gemv", 1, 4, 4) and passes[1]["fused_norm"]
    assert kinds[2] == ("gemv", 5, 2, 1)
    assert kinds[3] == ("gemv", 7, 2, 1)


def test_unpaired_swiglu_in_front_is_invalid(b2):
    cl = b2.cmd_list(b2.gemv(2, 64, 256, 1000, 0, Y, b2.GEMV_SWIGLU), b2.gemv(2, 32, 256, 5096, 0, Y + 64))
    assert b2.plan(cl)[0] == 1
    # an unpaired g at the end of a full group starts the next group instead
    g = b2.gemv
    cl = b2.cmd_list(g(2, 64, 256, 1000, 0, Y), g(2, 64, 256, 1000, 0, Y + 64), g(2, 64, 256, 1000, 0, Y + 128),
                     g(2, 64, 256, 1000, 0, Y + 192, b2.GEMV_SWIGLU), g(2, 64, 256, 1000, 0, Y + 256))
    st, passes = b2.plan(cl)
    assert st == 0 and [p["members"] for p in passes] == [3, 2]


def test_group_ends_after_y_overlapping_x(b2):
    g = b2.gemv
    cl = b2.cmd_list(g(2, 64, 256, 1000, 0, 128), g(2, 64, 256, 1000, 0, Y))
    st, passes = b2.plan(cl)
    assert st == 0 and [p["members"] for p in passes] == [1, 1]


def test_too_many_commands(b2):
    cl = b2.cmd_list(*[b2.add(16, 0, 16, 32)] * 129)
    assert b2.plan(cl)[0] == 129


def test_gdn_slots(b2):
    cl = b2.cmd_list(b2.gdn(4, 2, 0, 256, 512, 1024, 1040, 2048, 0, 0, 0.088, flags=b2.GDN_GATES | b2.GDN_L2_QK,
                            dt_off=1056, a_off=1072),
                     b2.gemv(2, 64, 512, 1000, 2048, Y, b2.GEMV_ADD), b2.add(64, Y, 3072, 3072))
    st, passes = b2.plan(cl)
    assert st == 0 and passes[0]["kind"] == "gdn" and passes[0]["count"] == 3
    cl2 = b2.cmd_list(b2.gdn(4, 2, 0, 256, 512, 1024, 1040, 2048, 0, 0, 0.088, flags=b2.GDN_WITH_OUT),
                      b2.gemv(2, 64, 512, 1000, 2048, Y, b2.GEMV_ADD), b2.add(64, Y, 3072, 3072))
    st, passes = b2.plan(cl2)
    assert st == 0 and passes[0]["count"] == 4 and passes[0]["members"] == 1
    bad = cl2.copy()
    bad[16 + 6] = 16  # the WITH_OUT GEMV must read the step's output
    assert b2.plan(bad)[0] == 1


def _random_list(b2, r, ws):
    handles = list(ws.keys())
    out = []
    for _ in range(int(r.integers(1, 12))):
        k = int(r.integers(0, 9))
        off = lambda: int(r.integers(0, 64)) * 16 + (int(r.integers(0, 40)) == 0)  # sometimes misaligned
        if k <= 2:
            h = handles[int(r.integers(0, len(handles)))]
            _, rows, cols, fmt = ws[h]
            fl = [0, 0, 0, b2.GEMV_SWIGLU, b2.GEMV_ADD, b2.GEMV_CONV][int(r.integers(0, 6))]
            out.append(b2.gemv(fmt, rows, cols, h, 0 if r.integers(0, 3) else 512,
                               off(), fl))
        elif k == 3:
            out.append(b2.add(int(r.integers(1, 5)) * 16 + (r.integers(0, 20) == 0), off(), off(), off()))
        elif k == 4:
            out.append(b2.rmsnorm(int(r.integers(1, 17)) * 16, off(), off(), off(), 1e-6,
                                  flags=[0, 1, 2, 3, 4, 8][int(r.integers(0, 6))]))
        elif k == 5:
            out.append(b2.conv(64, off(), off(), off(), off(), off(), bool(r.integers(0, 2))))
        elif k == 6:
            out.append(b2.unary(int(r.integers(1, 5)) * 16, off(), int(r.integers(0, 6)), off()))
        elif k == 7:
            out.append(b2.rope(int(r.integers(0, 5)) * 32, off(), off(), off(), 128, int(r.integers(0, 3))))
        else:
            out.append(b2.silu_mul(int(r.integers(1, 5)) * 16, off(), off(), off(), bool(r.integers(0, 2))))
    return b2.cmd_list(*out)


def test_random_lists_status_matches_oracle(b2, synth, orc):
    ws = weights(synth)
    r = rng(32)
    agree = 0
    for trial in range(400):
        cl = _random_list(b2, r, ws)
        st_plan, _ = b2.plan(cl)
        st_orc = oracle_status(orc, cl, ws)
        assert st_plan == st_orc, (trial, cl.reshape(-1, 8))
        agree += 1
    assert agree == 400


def test_deferred_norm_stored_only_when_x_changes_before_a_consumer(b2):
    """A deferred RMSNORM is computed inside its consumer GEMV pass unless its x or weight changes between the
    command and a consumer (an earlier pass, or the consumer itself writing them): then it is stored at the
    command. Writes after the last consumer (the residual ADD of a layer) leave it fused."""
    g = b2.gemv
    norm = b2.rmsnorm(256, X, 256, 512, 1e-6, flags=b2.NORM_DEFER)
    cases = {
        "write after the consumer": (b2.cmd_list(norm, g(2, 64, 256, 1000, 512, Y), b2.add(256, X, Z, X)), False),
        "x written before": (b2.cmd_list(norm, b2.add(256, X, Z, X), g(2, 64, 256, 1000, 512, Y)), True),
        "weight written before": (b2.cmd_list(norm, b2.add(256, 256, Z, 256), g(2, 64, 256, 1000, 512, Y)), True),
        "consumer writes x": (b2.cmd_list(norm, g(2, 64, 256, 1000, 512, X)), True),
        "unrelated write": (b2.cmd_list(norm, b2.add(256, Z, Z, Z + 256), g(2, 64, 256, 1000, 512, Y)), False),
    }
    for name, (cl, stored) in cases.items():
        st, passes = b2.plan(cl)
        assert st == 0, name
        gp = [p for p in passes if p["kind"] == "gemv"][0]
        assert gp["fused_norm"] and gp["stored_norm"] == stored, name


def test_small_passes_fuse_into_one_launch(b2):
    """Consecutive stored RMSNORM / ROPE commands run as one launch when independent (a ROPE of a norm's stored rows
    joins that norm), and ATTN takes a following sigmoid SILU_MUL of its output into its merge; a ROPE that reads rows
    another job of the run writes ends the run."""
    nh, nkv, hd = 4, 2, 128
    QG, K, QN, KN, QR, KR, CS, YA, YG, POS = 0, 1024, 1280, 1792, 2048, 2560, 2816, 3072, 3584, 4096
    W = 4352
    layer = b2.cmd_list(
        b2.rmsnorm(hd, QG, W, QN, 1e-6, rows=nh, stride_words=2 * hd // 16),
        b2.rmsnorm(hd, K, W, KN, 1e-6, rows=nkv),
        b2.rope(32, QN, CS, QR, hd, nh), b2.rope(32, KN, CS, KR, hd, nkv),
        b2.attn(nh, nkv, hd, QR, KR, K, YA, POS, 0),
        b2.silu_mul(nh * hd, QG + hd, YA, YG, sigmoid=True, row=hd, stride=2 * hd))
    st, passes = b2.plan(layer)
    assert st == 0
    assert [(p["kind"], p["first"], p["count"]) for p in passes] == [("elementwise", 0, 4), ("ext", 4, 2)]
    # the second ROPE reads the rows the first norm writes: the run stops before it
    clash = b2.cmd_list(
        b2.rmsnorm(hd, QG, W, QN, 1e-6, rows=nh, stride_words=2 * hd // 16),
        b2.rope(32, K, CS, KR, hd, nkv), b2.rope(32, QN, CS, QN, hd, nkv))
    st, passes = b2.plan(clash)
    assert st == 0 and [(p["first"], p["count"]) for p in passes] == [(0, 2), (2, 1)]
    # a gate whose g rows meet the attention output stays a separate pass
    st, passes = b2.plan(b2.cmd_list(b2.attn(nh, nkv, hd, QR, KR, K, YA, POS, 0),
                                     b2.silu_mul(nh * hd, YA, YA, YG, sigmoid=True)))
    assert st == 0 and [p["count"] for p in passes] == [1, 1]
