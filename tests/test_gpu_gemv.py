"""GEMV passes on the GPU against the CPU oracle (itself pinned to the reference's gemvq_ref.h): activation quants,
fp16 scales and per-block integer sums bit-exact; FP32 outputs bit-exact (the kernels fold the block terms in the
CPU's order); padding lanes zero."""
import numpy as np
import pytest

from conftest import rng

pytestmark = pytest.mark.gpu

SHAPES = [(2, 9216, 2560), (8, 2560, 9216), (3, 300, 512), (13, 9216, 2560), (14, 1000, 2560),
          (2, 17, 128), (8, 33, 384), (14, 7, 256), (13, 5, 512)]


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("fmt,rows,cols", SHAPES)
def test_single_gemv_bit_exact(ctx, b2, synth, orc, fmt, rows, cols):
    r = rng(40, fmt, rows, cols)
    w = synth.matrix(fmt, r, rows, cols)
    x = synth.activation(r, cols)
    ctx.reset_weights()
    h = ctx.upload(w, rows, cols, fmt)
    X, Y = 0, 16384
    ctx.write(X, x)
    ctx.fill(Y, 7.0, rows + 32)
    assert ctx.run(b2.gemv(fmt, rows, cols, h, X, Y)) == 0
    got = ctx.read(Y, rows + 32)
    ref, mag = orc.gemv(w, x, rows, cols, fmt)
    assert np.array_equal(_bits(got[:rows]), _bits(ref)), \
        f"{np.sum(_bits(got[:rows]) != _bits(ref))} rows differ; within tol: {orc.within_tolerance(got[:rows], ref, mag).all()}"
    pad = (rows + 15) // 16 * 16
    assert np.all(got[rows:pad] == 0.0) and np.all(got[pad:] == 7.0)


@pytest.mark.parametrize("fmt,n", [(2, 2560), (8, 9216), (3, 512), (14, 2560), (13, 16384)])
def test_quantized_activation_bit_exact(ctx, b2, orc, fmt, n):
    x = np.concatenate([rng(41, n).normal(0, 1, n - 256), np.zeros(128), rng(42).normal(0, 1e-4, 128)]).astype(np.float32)
    ctx.write(0, x)
    q, scales, bs = ctx.debug_quantize(fmt, 0, n)
    if fmt in (13, 14):
        qr, dr, br = orc.quantize_q8_k(x)
        assert np.array_equal(_bits(scales), _bits(dr))
    elif fmt == 3:
        qr, dr, br = orc.quantize_q8_1(x)
        assert np.array_equal(scales, dr)
    else:
        qr, dr, br = orc.quantize_q8_0(x)
        assert np.array_equal(scales, dr)
    assert np.array_equal(q, qr) and np.array_equal(bs, br)


@pytest.mark.parametrize("flags", [0, 1, 2, 3])
def test_fused_norm_quantizer_bit_exact(ctx, b2, orc, flags):
    n = 2560
    x = rng(43, flags).normal(0, 1, n).astype(np.float32)
    g = rng(44).normal(1, 0.1, n).astype(np.float32)
    ctx.write(0, x)
    ctx.write(n, g)
    q, scales, bs = ctx.debug_quantize(8, 0, n, norm_w_off=n, eps=1e-6, norm_flags=flags)
    xn = orc.rownorm(x, g, n, 1, 1e-6, flags)
    qr, dr, br = orc.quantize_q8_0(xn)
    assert np.array_equal(q, qr) and np.array_equal(scales, dr) and np.array_equal(bs, br)


@pytest.mark.parametrize("fmt,rows,cols", [(2, 9216, 2560), (8, 300, 1024), (3, 64, 256), (13, 96, 512),
                                           (14, 200, 2560)])
def test_block_sums_bit_exact(ctx, b2, synth, orc, fmt, rows, cols):
    r = rng(45, fmt)
    w = synth.matrix(fmt, r, rows, cols)
    x = synth.activation(r, cols)
    ctx.reset_weights()
    h = ctx.upload(w, rows, cols, fmt)
    ctx.write(0, x)
    got = ctx.debug_block_sums(b2.gemv(fmt, rows, cols, h, 0, 16384))
    if fmt in (13, 14):
        q = orc.quantize_q8_k(x)[0]
    elif fmt == 3:
        q = orc.quantize_q8_1(x)[0]
    else:
        q = orc.quantize_q8_0(x)[0]
    ref = orc.block_sums(w, q, rows, cols, fmt)
    assert np.array_equal(got, ref)


def _weights_and_list(b2, synth, ctx, specs, r):
    ws = {}
    for fmt, rows, cols in specs:
        w = synth.matrix(fmt, r, rows, cols)
        h = ctx.upload(w, rows, cols, fmt)
        ws[h] = (w.reshape(-1), rows, cols, fmt)
    return ws


def _compare_list(ctx, orc, cl, ws, act_init, n_act, state=None, exact=True):
    ctx.write(0, act_init)
    if state is not None:
        ctx.write_state(0, state)
    st = ctx.run(cl)
    got = ctx.read(0, n_act)
    act = act_init.copy()
    st_ref = orc.run_list(act, cl, ws, state=state.copy() if state is not None else None)
    assert st == st_ref
    if exact:
        diff = np.nonzero(_bits(got) != _bits(act[:n_act]))[0]
        assert diff.size == 0, f"{diff.size} floats differ, first at {diff[:8]}"
    return got, act


def test_group_with_swiglu_conv_add_epilogues(ctx, b2, synth, orc):
    ctx.reset_weights()
    r = rng(46)
    ws = _weights_and_list(b2, synth, ctx, [(2, 256, 512), (2, 256, 512), (8, 64, 512), (2, 128, 512),
                                            (2, 96, 512)], r)
    h = list(ws)
    X, N = 0, 1 << 15
    act = r.normal(0, 1, N).astype(np.float32)
    g = b2.gemv
    cl = b2.cmd_list(
        g(2, 256, 512, h[0], X, 4096, b2.GEMV_SWIGLU), g(2, 256, 512, h[1], X, 4608),   # SwiGLU pair -> 4608
        g(8, 64, 512, h[2], X, 5120, b2.GEMV_CONV), b2.conv(64, 5120, 6144, 5200, 7000, 7000, True),  # conv in place
        g(2, 128, 512, h[3], X, 8192, b2.GEMV_ADD), b2.add(128, 9000, 8192, 9216),      # residual add
        g(2, 96, 512, h[4], X, 10000))                                                   # plain, padded to 96
    _compare_list(ctx, orc, cl, ws, act, N)


def test_pass_rows_hint_changes_layout_not_results(ctx, b2, synth, orc):
    """The DeltaNet q/k/v, z, beta, alpha rows on one normed x (4 members, 8224 rows): uploaded with
    B200Q_UPLOAD_PASS_ROWS they take 32-row panels (one wave), without it 16 / 8 / 2-row panels (two waves); the
    outputs are the same bits, and the oracle's."""
    r = rng(47)
    H = 2560
    shapes = [(6144, H), (2048, H), (16, H), (16, H)]
    mats = [synth.q4_0(r, rows, cols) for rows, cols in shapes]
    act = np.zeros(1 << 15, np.float32)
    act[:H] = r.normal(0, 1, H)
    act[H:2 * H] = r.normal(1, 0.1, H)
    XN, Y = 2 * H, 3 * H
    outs = []
    for flags in (0, b2.UPLOAD_PASS_ROWS(8224)):
        ctx.reset_weights()
        hs = [ctx.upload(m, rows, cols, b2.Q4_0, flags=flags) for m, (rows, cols) in zip(mats, shapes)]
        offs = [Y, Y + 6144, Y + 8192, Y + 8208]
        cl = b2.cmd_list(b2.rmsnorm(H, 0, H, XN, 1e-6, flags=b2.NORM_DEFER),
                         *[b2.gemv(b2.Q4_0, rows, cols, h, XN, o) for h, (rows, cols), o in zip(hs, shapes, offs)])
        ctx.write(0, act)
        assert ctx.run(cl) == 0
        outs.append(ctx.read(Y, 8224))
        if flags:
            ws = {h: (m.reshape(-1), rows, cols, b2.Q4_0) for h, m, (rows, cols) in zip(hs, mats, shapes)}
            ref = act.copy()
            assert orc.run_list(ref, cl, ws) == 0
            assert np.array_equal(_bits(outs[-1]), _bits(ref[Y:Y + 8224]))
    assert b2.layout(2048, H, b2.Q4_0)["rows_per_tile"] != b2.layout(2048, H, b2.Q4_0, flags=b2.UPLOAD_PASS_ROWS(8224))["rows_per_tile"]
    assert np.array_equal(_bits(outs[0]), _bits(outs[1]))


def test_fused_ffn_block_config1(ctx, b2, synth, orc):
    """Config 1: RMSNorm (deferred) -> Q8_0 gate+up in one pass -> SwiGLU -> down -> residual add."""
    ctx.reset_weights()
    r = rng(47)
    H, F = 2560, 9216
    ws = _weights_and_list(b2, synth, ctx, [(8, F, H), (8, F, H), (8, H, F)], r)
    hg, hu, hd = list(ws)
    XIN, GAIN, XN, FF, OUT = 0, H, 2 * H, 4 * H, 4 * H + F
    act = np.zeros(OUT + H, np.float32)
    act[XIN:XIN + H] = synth.activation(r, H)
    act[GAIN:GAIN + H] = r.normal(1, 0.1, H).astype(np.float32)
    cl = b2.cmd_list(
        b2.rmsnorm(H, XIN, GAIN, XN, 1e-6, flags=b2.NORM_DEFER),
        b2.gemv(8, F, H, hg, XN, FF, b2.GEMV_SWIGLU), b2.gemv(8, F, H, hu, XN, FF),
        b2.gemv(8, H, F, hd, FF, OUT, b2.GEMV_ADD), b2.add(H, OUT, XIN, OUT))
    st, passes = b2.plan(cl)
    assert st == 0 and passes[1]["fused_norm"] and passes[1]["members"] == 2
    got, ref = _compare_list(ctx, orc, cl, ws, act, act.size, exact=False)
    # SwiGLU uses exp(): CUDA's and glibc's FP32 exp may differ in the last bit; the rest is bit-exact
    rel = np.abs(got[OUT:] - ref[OUT:]) / np.maximum(np.abs(ref[OUT:]), 1e-30)
    assert rel.max() <= 1e-4
    assert np.array_equal(_bits(got[XIN:XN]), _bits(ref[XIN:XN]))


def test_deferred_norm_of_a_row_that_changes_before_its_consumer(ctx, b2, synth, orc):
    """RMSNORM (deferred) of x, then an ADD that rewrites x, then the GEMV that reads the norm: the norm is the one of
    x at the RMSNORM command (stored there), as the reference's on-chip row is."""
    ctx.reset_weights()
    r = rng(56)
    H, R = 2560, 2048
    ws = _weights_and_list(b2, synth, ctx, [(2, R, H)], r)
    (h,) = list(ws)
    XIN, GAIN, OTHER, XN, Y = 0, H, 2 * H, 3 * H, 4 * H
    act = np.zeros(Y + R, np.float32)
    act[XIN:XIN + H] = synth.activation(r, H)
    act[GAIN:GAIN + H] = r.normal(1, 0.1, H).astype(np.float32)
    act[OTHER:OTHER + H] = synth.activation(r, H)
    cl = b2.cmd_list(b2.rmsnorm(H, XIN, GAIN, XN, 1e-6, flags=b2.NORM_DEFER), b2.add(H, XIN, OTHER, XIN),
                     b2.gemv(2, R, H, h, XN, Y))
    st, passes = b2.plan(cl)
    assert st == 0 and passes[-1]["stored_norm"]
    got, ref = _compare_list(ctx, orc, cl, ws, act, act.size, exact=True)
    assert np.array_equal(_bits(got[Y:Y + R]), _bits(ref[Y:Y + R]))


CHAINS = ["q8_0-to-q4_0", "q4_0-add-to-q4_1", "p8-to-q8_0", "q8_0-norm-to-q4_0", "q4_0-l2norm-to-q4_1"]


@pytest.mark.parametrize("chain", CHAINS)
def test_gemv_chain_hands_over_quantized_x(ctx, b2, synth, orc, chain):
    """A GEMV pass whose output is the next GEMV pass's whole x writes that pass's quantized x itself when its output
    rows are in 32-row panels (the first two chains; a Q4_1 consumer takes a Q8_1 image, with the s terms); outputs
    in smaller panels, and outputs the next pass reads through a deferred RMSNORM (weighted, and L2 without weight),
    are quantized by the next pass. Every chain stays bit-exact against the CPU path (no exp in it)."""
    ctx.reset_weights()
    r = rng(49, CHAINS.index(chain))
    H, F, K = 2560, 9216, 1024
    if chain == "p8-to-q8_0":  # [2560 x 9216] is laid out in 8-row panels
        ws = _weights_and_list(b2, synth, ctx, [(8, H, F), (8, K, H)], r)
        h1, h2 = list(ws)
        X, Y1, Y2 = 0, F, F + H
        act = np.zeros(Y2 + K, np.float32)
        act[X:X + F] = synth.activation(r, F)
        cl = b2.cmd_list(b2.gemv(8, H, F, h1, X, Y1), b2.gemv(8, K, H, h2, Y1, Y2))
    elif chain in ("q8_0-norm-to-q4_0", "q4_0-l2norm-to-q4_1"):
        f1, f2, flags = (8, 2, b2.NORM_DEFER) if chain == "q8_0-norm-to-q4_0" else (2, 3, b2.NORM_DEFER | 1 | 2)
        ws = _weights_and_list(b2, synth, ctx, [(f1, H, F), (f2, K, H)], r)
        h1, h2 = list(ws)
        X, R, Y1, G, XN, Y2 = 0, F, F + H, F + 2 * H, F + 3 * H, F + 4 * H
        act = np.zeros(Y2 + K, np.float32)
        act[X:X + F] = synth.activation(r, F)
        act[R:R + H] = synth.activation(r, H)
        act[G:G + H] = r.normal(1, 0.1, H).astype(np.float32)
        cl = b2.cmd_list(b2.gemv(f1, H, F, h1, X, Y1, b2.GEMV_ADD), b2.add(H, Y1, R, Y1),
                         b2.rmsnorm(H, Y1, G, XN, 1e-6, flags=flags), b2.gemv(f2, K, H, h2, XN, Y2))
    elif chain == "q8_0-to-q4_0":
        ws = _weights_and_list(b2, synth, ctx, [(8, F, H), (2, H, F)], r)
        h1, h2 = list(ws)
        X, Y1, Y2 = 0, H, H + F
        act = np.zeros(Y2 + H, np.float32)
        act[X:X + H] = synth.activation(r, H)
        cl = b2.cmd_list(b2.gemv(8, F, H, h1, X, Y1), b2.gemv(2, H, F, h2, Y1, Y2))
    else:
        ws = _weights_and_list(b2, synth, ctx, [(2, F, H), (3, K, F)], r)
        h1, h2 = list(ws)
        X, R, Y1, Y2 = 0, H, H + F, H + 2 * F
        act = np.zeros(Y2 + K, np.float32)
        act[X:X + H] = synth.activation(r, H)
        act[R:R + F] = synth.activation(r, F)
        cl = b2.cmd_list(b2.gemv(2, F, H, h1, X, Y1, b2.GEMV_ADD), b2.add(F, Y1, R, Y1), b2.gemv(3, K, F, h2, Y1, Y2))
    st, passes = b2.plan(cl)
    assert st == 0 and sum(p["kind"] == "gemv" for p in passes) == 2
    _compare_list(ctx, orc, cl, ws, act, act.size)


@pytest.mark.parametrize("fmt", [8, 2])
def test_two_layer_ffn_stack(ctx, b2, synth, orc, fmt):
    """Two FFN blocks in one list, the second reading the residual the first wrote through its deferred RMSNORM
    (each gate+up pass hands its down pass the quantized SwiGLU output; with Q4_0 the first down pass also hands the
    second gate+up pass its per-panel sums of squares for the norm)."""
    ctx.reset_weights()
    r = rng(55, fmt)
    H, F = 2560, 9216
    ws = _weights_and_list(b2, synth, ctx, [(fmt, F, H), (fmt, F, H), (fmt, H, F)] * 2, r)
    hs = list(ws)
    R0, GAIN, XN, FF, R1 = 0, H, 2 * H, 4 * H, 4 * H + F
    act = np.zeros(R1 + H, np.float32)
    act[R0:R0 + H] = synth.activation(r, H)
    act[GAIN:GAIN + H] = r.normal(1, 0.1, H).astype(np.float32)
    cmds = []
    for layer, (xin, out) in enumerate(((R0, R1), (R1, R0))):
        hg, hu, hd = hs[3 * layer:3 * layer + 3]
        cmds += [b2.rmsnorm(H, xin, GAIN, XN, 1e-6, flags=b2.NORM_DEFER),
                 b2.gemv(fmt, F, H, hg, XN, FF, b2.GEMV_SWIGLU), b2.gemv(fmt, F, H, hu, XN, FF),
                 b2.gemv(fmt, H, F, hd, FF, out, b2.GEMV_ADD), b2.add(H, out, xin, out)]
    cl = b2.cmd_list(*cmds)
    got, ref = _compare_list(ctx, orc, cl, ws, act, act.size, exact=False)
    rel = np.abs(got[R0:R0 + H] - ref[R0:R0 + H]) / np.maximum(np.abs(ref[R0:R0 + H]), 1e-30)
    assert rel.max() <= 1e-4, rel.max()


def test_q6k_output_head_config2(ctx, b2, synth, orc):
    """The Q6_K output head [151936 x 2560]: GEMV commands hold at most 65536 rows (reference MAX_ROWS), so the head
    goes in 65520-row pieces as the reference backend emits it (ggml-xrt.cpp:133-139, 1536-1554) — here three
    GEMVs on one x, one pass."""
    ctx.reset_weights()
    r = rng(48)
    rows, cols = 151936, 2560
    w = synth.q6_k(r, rows, cols)
    x = synth.activation(r, cols)
    rb = b2.gguf_row_bytes(cols, 14)
    pieces, cmds, r0 = [], [], 0
    while r0 < rows:
        n = min(65520, rows - r0)
        h = ctx.upload(w.reshape(-1)[r0 * rb:(r0 + n) * rb], n, cols, 14)
        cmds.append(b2.gemv(14, n, cols, h, 0, 4096 + r0))
        r0 += n
    ctx.write(0, x)
    cl = b2.cmd_list(*cmds)
    st, passes = b2.plan(cl)
    assert st == 0 and len(passes) == 1 and passes[0]["members"] == 3
    assert ctx.run(cl) == 0
    got = ctx.read(4096, rows)
    ref, _ = orc.gemv(w, x, rows, cols, 14)
    assert np.array_equal(_bits(got), _bits(ref))
    assert ctx.run(b2.gemv(14, rows, cols, 0, 0, 4096)) == 1  # one command of more than 65536 rows is invalid


def test_graph_replay_matches_run(ctx, b2, synth, orc):
    ctx.reset_weights()
    r = rng(49)
    w = synth.q4_0(r, 2048, 2560)
    h = ctx.upload(w, 2048, 2560, 2)
    cl = b2.cmd_list(b2.gemv(2, 2048, 2560, h, 0, 4096))
    g = ctx.graph(cl)
    assert g.kernels >= 1
    for i in range(3):
        x = synth.activation(rng(50, i), 2560)
        ctx.write(0, x)
        g.launch()
        ctx.synchronize()
        got = ctx.read(4096, 2048)
        ref, _ = orc.gemv(w, x, 2048, 2560, 2)
        assert np.array_equal(_bits(got), _bits(ref))
    g.close()


def test_feature_probe(ctx, b2):
    ctx.fill(0, 0.0, 16)
    assert ctx.run(np.zeros(0, np.uint32)) == 0
    got = ctx.read(0, 3).view(np.uint32)
    assert tuple(int(v) for v in got) == b2.FEATURES
