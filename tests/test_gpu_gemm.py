"""GEMV_BATCH commands of more than 8 rows on the GPU: the prefill GEMM on the tensor cores (gemm_tc_kernel, int8
tcgen05.mma per 32-value block, FP32 block terms in block order). The MMA's integer sums of one block are the oracle's
block dots; every output row has the bits of the GEMV of its activation row (checked against the batch kernel of up
to 8 rows, itself bit-identical to the GEMV, and against the oracle); Q4_0 / Q8_0 / Q4_1, weight rows that are not a
multiple of 128, token counts that are not a multiple of 128, the ADD flag, the zero padding of y, graph replays."""
import numpy as np
import pytest

from conftest import has_gpu, rng

pytestmark = pytest.mark.gpu

X, Y, YB = 0, 1 << 22, 1 << 23


@pytest.fixture(scope="module")
def ctx(b2):
    if not has_gpu():
        pytest.skip("no GPU")
    c = b2.Context(device=0, weight_bytes=1 << 30, act_floats=1 << 24)
    yield c
    c.close()


def _setup(ctx, synth, fmt, rows, cols, tokens, seed):
    ctx.reset_weights()
    r = rng(127, fmt, rows, cols, tokens, seed)
    w = synth.matrix(fmt, r, rows, cols)
    h = ctx.upload(w, rows, cols, fmt)
    xs = np.stack([synth.activation(r, cols) * (1 + (t % 7) * 0.25) for t in range(tokens)]).astype(np.float32)
    return w, h, xs


def _quantized(orc, fmt, x):
    return (orc.quantize_q8_1 if fmt == 3 else orc.quantize_q8_0)(x)[0]


@pytest.mark.parametrize("fmt", [2, 8, 3])
def test_mma_block_sums_are_the_integer_block_dots(ctx, b2, synth, orc, fmt):
    rows, cols, tokens = 256, 512, 128
    w, h, xs = _setup(ctx, synth, fmt, rows, cols, tokens, 0)
    ctx.write(X, xs.reshape(-1))
    got = ctx.debug_block_sums(b2.gemv_batch(fmt, rows, cols, h, X, Y, tokens))
    nb = cols // 32
    want = np.zeros((128, tokens), np.int64)
    for t in range(tokens):
        want[:, t] = orc.block_sums(w, _quantized(orc, fmt, xs[t]), rows, cols, fmt).reshape(rows, nb)[:128, 0]
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)
        same_t = np.array_equal(got, want.T)
        raise AssertionError(f"{len(bad)} of {got.size} sums differ (first {bad[:4].tolist()}: got "
                             f"{[int(got[i, j]) for i, j in bad[:4]]} want {[int(want[i, j]) for i, j in bad[:4]]}); "
                             f"transposed equal: {same_t}; got row 0 {got[0, :8].tolist()} col 0 {got[:8, 0].tolist()}; "
                             f"want row 0 {want[0, :8].tolist()} col 0 {want[:8, 0].tolist()}")


@pytest.mark.parametrize("fmt,rows,cols", [(2, 9216, 2560), (8, 2560, 9216), (3, 1000, 2560), (2, 2560, 2560)])
@pytest.mark.parametrize("tokens", [9, 200])
def test_gemm_rows_are_the_gemv_and_the_oracle(ctx, b2, synth, orc, fmt, rows, cols, tokens):
    w, h, xs = _setup(ctx, synth, fmt, rows, cols, tokens, 1)
    ys = (rows + 15) // 16 * 16
    ctx.write(X, xs.reshape(-1))
    ctx.fill(Y, 7.0, tokens * ys + 16)  # padding must come back zero, the row past the batch untouched
    assert ctx.run(b2.cmd_list(b2.gemv_batch(fmt, rows, cols, h, X, Y, tokens))) == 0, ctx.last_error()
    got = ctx.read(Y, tokens * ys + 16)
    # the same rows through the batch kernel (up to 8 rows per command, bit-identical to the GEMV)
    per = b2.BATCH_MAX
    chunks = [b2.gemv_batch(fmt, rows, cols, h, X + m * cols, YB + m * ys, min(per, tokens - m))
              for m in range(0, tokens, per)]
    for i in range(0, len(chunks), 100):
        assert ctx.run(b2.cmd_list(*chunks[i:i + 100])) == 0, ctx.last_error()
    one = ctx.read(YB, tokens * ys)
    got_rows = got[:tokens * ys].reshape(tokens, ys)
    bad = [t for t in range(tokens)
           if not np.array_equal(got_rows[t, :rows].view(np.uint32), one[t * ys:t * ys + rows].view(np.uint32))]
    assert not bad, f"tokens {bad[:8]} differ from the batch kernel"
    assert not got_rows[:, rows:].any()
    assert np.all(got[tokens * ys:] == 7.0)
    for t in (0, tokens - 1):
        y, _ = orc.gemv(w, xs[t], rows, cols, fmt)
        assert np.array_equal(got_rows[t, :rows].view(np.uint32), y.view(np.uint32)), t


def test_gemm_add_graph_replays_and_kernel_count(ctx, b2, synth, orc):
    fmt, rows, cols, tokens = 8, 384, 1024, 130
    w, h, xs = _setup(ctx, synth, fmt, rows, cols, tokens, 2)
    res = rng(128).normal(0, 1, (tokens, rows)).astype(np.float32)
    cl = b2.cmd_list(b2.gemv_batch(fmt, rows, cols, h, X, Y, tokens, b2.GEMV_ADD))
    ctx.write(X, xs.reshape(-1))
    g = ctx.graph(cl)
    assert g.kernels == 2  # the tokens' quantizer and the GEMM
    outs = []
    for _ in range(3):
        ctx.write(Y, res.reshape(-1))
        ctx.launch_many([g], 1)
        ctx.synchronize()
        outs.append(ctx.read(Y, tokens * rows))
    g.close()
    for o in outs[1:]:
        assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32))
    act = np.zeros(Y + tokens * rows + 16, np.float32)
    act[X:X + tokens * cols] = xs.reshape(-1)
    act[Y:Y + tokens * rows] = res.reshape(-1)
    assert orc.run_list(act, cl, {h: (w.reshape(-1), rows, cols, fmt)}) == 0
    assert np.array_equal(outs[0].view(np.uint32), act[Y:Y + tokens * rows].view(np.uint32))
