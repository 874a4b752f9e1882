"""GEMV_BATCH (opcode 17, no GPU): the host planner's validation agrees with the oracle's interpreter on valid and
invalid commands, and the oracle's batch command is, row by row, the GEMV command on each activation row (with the
ADD flag: plus the old y row; y rows zero-padded to a multiple of 16), for a few rows and for more than 8 (the
batch field is 16 bits wide; the GPU runs those as the tensor-core GEMM). The GPU kernel is held to the same in
tests/test_gpu_batch.py."""
import numpy as np
import pytest

from conftest import rng

X, Y = 0, 65536
H1, H2, H3 = 4096, 1 << 24, 2 << 24


def _weights(synth):
    r = rng(120)
    return {H1: (synth.q4_0(r, 100, 256).reshape(-1), 100, 256, 2),
            H2: (synth.q8_0(r, 64, 512).reshape(-1), 64, 512, 8),
            H3: (synth.q4_1(r, 48, 384).reshape(-1), 48, 384, 3)}


def _act(n=1 << 17, seed=0):
    return rng(121, seed).normal(0, 1, n).astype(np.float32)


@pytest.mark.parametrize("h,batch", [(H1, 1), (H1, 5), (H2, 8), (H3, 3), (H1, 9), (H2, 40), (H3, 130)])
@pytest.mark.parametrize("add", [False, True])
def test_oracle_batch_is_the_gemv_of_every_row(b2, orc, synth, h, batch, add):
    ws = _weights(synth)
    _, rows, cols, fmt = ws[h]
    ys = (rows + 15) // 16 * 16
    act = _act(seed=batch)
    ref = act.copy()
    flags = b2.GEMV_ADD if add else 0
    assert orc.run_list(act, b2.cmd_list(b2.gemv_batch(fmt, rows, cols, h, X, Y, batch, flags)), ws) == 0
    for m in range(batch):
        y, _ = orc.gemv(ws[h][0], ref[X + m * cols:X + (m + 1) * cols], rows, cols, fmt)
        want = (y + ref[Y + m * ys:Y + m * ys + rows]).astype(np.float32) if add else y
        got = act[Y + m * ys:Y + (m + 1) * ys]
        assert np.array_equal(got[:rows].view(np.uint32), want.view(np.uint32)), m
        assert not got[rows:].any()
    # rows past the batch keep their values
    assert np.array_equal(act[Y + batch * ys:Y + batch * ys + 64], ref[Y + batch * ys:Y + batch * ys + 64])


def _status(b2, orc, ws, cmd):
    cl = b2.cmd_list(b2.gemv(2, 100, 256, H1, X, 8192), cmd)
    return b2.plan(cl)[0], orc.run_list(_act(), cl, ws)


def test_planner_and_oracle_agree_on_valid_and_invalid_batches(b2, orc, synth):
    ws = _weights(synth)
    gb = b2.gemv_batch
    valid = [gb(2, 100, 256, H1, X, Y, 8), gb(8, 64, 512, H2, X, Y, 2, b2.GEMV_ADD), gb(3, 48, 384, H3, 256, Y, 1),
             gb(2, 100, 256, H1, X, Y, 9), gb(8, 64, 512, H2, X, Y, 100)]  # more than 8 rows: the GEMM
    for cmd in valid:
        assert _status(b2, orc, ws, cmd) == (0, 0)
    invalid = [
        gb(2, 100, 256, H1, X, Y, 300),                  # 300 rows of x reach into y
        gb(2, 100, 256, H1, X, 512, 4),                  # y overlaps x
        gb(2, 100, 256, H1, X, Y, 2, b2.GEMV_SWIGLU),    # no epilogue but ADD
        gb(2, 100, 256, H1, 8, Y, 2),                    # x not 16-aligned
        gb(14, 48, 512, H1, X, Y, 2),                    # K-quants are not batched
        gb(2, 100, 192, H1, X, Y, 2),                    # cols not a multiple of 128
    ]
    for cmd in invalid:
        st = _status(b2, orc, ws, cmd)
        assert st == (2, 2), (cmd, st)
    # weights of another shape, y past the end of act: only the oracle (which knows the weights and act) and a device
    # context can see these; host-only planning knows neither
    assert _status(b2, orc, ws, gb(2, 64, 256, H1, X, Y, 2))[1] == 2
    assert _status(b2, orc, ws, gb(2, 100, 256, H1, X, (1 << 17) - 64, 2))[1] == 2


def test_batch_is_one_pass_and_writes_its_rows(b2):
    cl = b2.cmd_list(b2.rmsnorm(256, X, 256, 512, 1e-6, flags=b2.NORM_DEFER),
                     b2.gemv_batch(2, 100, 256, H1, 1024, Y, 4), b2.gemv(2, 100, 256, H1, 512, 8192))
    st, passes = b2.plan(cl)
    assert st == 0
    assert [p["kind"] for p in passes] == ["nop", "ext", "gemv"]
    # the batch does not write the norm's x or weight: the norm stays deferred into the GEMV
    assert passes[2]["fused_norm"] and not passes[2]["stored_norm"]
