"""GEMV_BATCH on the GPU (gemv_batch_kernel): every output row has the bits of the GEMV command on its activation row
and of the oracle, for Q4_0 / Q8_0 / Q4_1, 1 to 8 rows, the configs' shapes, rows that are not a multiple of 32,
the ADD flag, the zero padding of y, a 16384-column matrix whose rows need several launches (the images and term
buffers of 8 rows do not fit one CTA), and graph replays."""
import numpy as np
import pytest

from conftest import rng

pytestmark = pytest.mark.gpu

X, Y, YS = 0, 1 << 18, 1 << 20


def _setup(ctx, synth, fmt, rows, cols, batch, seed):
    ctx.reset_weights()
    r = rng(125, fmt, rows, cols, batch, seed)
    w = synth.matrix(fmt, r, rows, cols)
    h = ctx.upload(w, rows, cols, fmt)
    xs = np.stack([synth.activation(r, cols) * (1 + m) for m in range(batch)]).astype(np.float32)
    return w, h, xs


@pytest.mark.parametrize("fmt,rows,cols", [(2, 9216, 2560), (8, 9216, 2560), (2, 2560, 9216), (8, 2560, 9216),
                                           (3, 1000, 2560), (2, 4096, 16384)])
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_batch_rows_are_the_gemv_and_the_oracle(ctx, b2, synth, orc, fmt, rows, cols, batch):
    w, h, xs = _setup(ctx, synth, fmt, rows, cols, batch, 0)
    ys = (rows + 15) // 16 * 16
    ctx.write(X, xs.reshape(-1))
    ctx.fill(Y, 7.0, batch * ys + 16)  # padding must come back zero, the row past the batch untouched
    assert ctx.run(b2.cmd_list(b2.gemv_batch(fmt, rows, cols, h, X, Y, batch))) == 0, ctx.last_error()
    got = ctx.read(Y, batch * ys + 16)
    singles = b2.cmd_list(*[b2.gemv(fmt, rows, cols, h, X + m * cols, YS + m * ys) for m in range(batch)])
    assert ctx.run(singles) == 0
    one = ctx.read(YS, batch * ys)
    for m in range(batch):
        g = got[m * ys:(m + 1) * ys]
        assert np.array_equal(g[:rows].view(np.uint32), one[m * ys:m * ys + rows].view(np.uint32)), m
        assert not g[rows:].any()
        if m in (0, batch - 1):
            y, _ = orc.gemv(w, xs[m], rows, cols, fmt)
            assert np.array_equal(g[:rows].view(np.uint32), y.view(np.uint32)), m
    assert np.all(got[batch * ys:] == 7.0)


def test_batch_add_and_graph_replays(ctx, b2, synth, orc):
    fmt, rows, cols, batch = 2, 2560, 9216, 4
    w, h, xs = _setup(ctx, synth, fmt, rows, cols, batch, 1)
    res = rng(126).normal(0, 1, (batch, rows)).astype(np.float32)
    cl = b2.cmd_list(b2.gemv_batch(fmt, rows, cols, h, X, Y, batch, b2.GEMV_ADD))
    ctx.write(X, xs.reshape(-1))
    g = ctx.graph(cl)
    assert g.kernels == 1  # the rows' quantization is part of the one batch launch
    outs = []
    for _ in range(3):
        ctx.write(Y, res.reshape(-1))
        ctx.launch_many([g], 1)
        ctx.synchronize()
        outs.append(ctx.read(Y, batch * rows))
    g.close()
    for o in outs[1:]:
        assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32))
    act = np.zeros(Y + batch * rows + 16, np.float32)
    act[X:X + batch * cols] = xs.reshape(-1)
    act[Y:Y + batch * rows] = res.reshape(-1)
    assert orc.run_list(act, cl, {h: (w.reshape(-1), rows, cols, fmt)}) == 0
    assert np.array_equal(outs[0].view(np.uint32), act[Y:Y + batch * rows].view(np.uint32))


def test_invalid_batch_is_rejected_with_its_index(ctx, b2, synth):
    fmt, rows, cols = 8, 1024, 2560
    _, h, _ = _setup(ctx, synth, fmt, rows, cols, 1, 2)
    bad = b2.cmd_list(b2.gemv(fmt, rows, cols, h, X, YS), b2.gemv_batch(fmt, rows + 32, cols, h, X, Y, 2))
    assert ctx.run(bad) == 2  # a weight of another shape: the context knows its weights
