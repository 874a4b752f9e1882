"""Persistent GEMV chains (gemv_chain_kernel, feature-mask bit 21, off by default): runs of Q4_0 / Q8_0 GEMV passes
that one persistent kernel executes. Every chained list gives the bits of the same list run pass by pass (bit 21
off), and the oracle's values; replays of the same graph (the chain's counters reset by each launch) and several chains in one list (one
counter block each) too."""
import numpy as np
import pytest

from conftest import rng

pytestmark = pytest.mark.gpu

H, F = 2560, 9216
XIN, GAIN, XN, FF, OUT = 0, H, 2 * H, 4 * H, 4 * H + F
ALL = 0xFFFFFFFF


def _run(ctx, cl, act, mask, replays=1):
    ctx.set_feature_mask(mask)
    try:
        ctx.write(0, act)
        g = ctx.graph(cl)
        kernels = g.kernels
        outs = []
        for _ in range(replays):
            ctx.write(0, act)
            ctx.launch_many([g], 1)
            ctx.synchronize()
            outs.append(ctx.read(0, act.size))
        g.close()
    finally:
        ctx.set_feature_mask(b2_default())
    return outs, kernels


def b2_default():
    import fpga_llama_gguf_b200 as b2
    return b2.DEFAULT_FEATURE_MASK


@pytest.mark.parametrize("fmt", [2, 8])
def test_layer_stack_chain_matches_passes_and_oracle(ctx, b2, synth, orc, fmt):
    """Four FFN layers (deferred norm -> gate+up SwiGLU -> down + residual), residual rows alternating: one chain."""
    ctx.reset_weights()
    r = rng(110, fmt)
    gen = synth.q8_0 if fmt == 8 else synth.q4_0
    layers, ws, cmds = [], {}, []
    res = (XIN, OUT)
    for c in range(4):
        mats = (gen(r, F, H), gen(r, F, H), gen(r, H, F))
        hs = [ctx.upload(m, rows, cols, fmt) for m, rows, cols in zip(mats, (F, F, H), (H, H, F))]
        for h, m, rows, cols in zip(hs, mats, (F, F, H), (H, H, F)):
            ws[h] = (m.reshape(-1), rows, cols, fmt)
        xi, xo = res[c % 2], res[(c + 1) % 2]
        cmds += [b2.rmsnorm(H, xi, GAIN, XN, 1e-6, flags=b2.NORM_DEFER),
                 b2.gemv(fmt, F, H, hs[0], XN, FF, b2.GEMV_SWIGLU), b2.gemv(fmt, F, H, hs[1], XN, FF),
                 b2.gemv(fmt, H, F, hs[2], FF, xo, b2.GEMV_ADD), b2.add(H, xo, xi, xo)]
    cl = b2.cmd_list(*cmds)
    act = np.zeros(1 << 16, np.float32)
    act[XIN:XIN + H] = synth.activation(r, H)
    act[GAIN:GAIN + H] = r.normal(1, 0.1, H)
    (chained,), k1 = _run(ctx, cl, act, ALL)
    (passes,), k2 = _run(ctx, cl, act, ALL & ~b2.MASK_CHAINS)
    assert k1 == 1 and k2 == 8
    assert np.array_equal(chained.view(np.uint32), passes.view(np.uint32))
    ref = act.copy()
    assert orc.run_list(ref, cl, ws) == 0
    out = slice(XIN, XIN + H)  # four layers: the residual is back in its first row
    rel = np.abs(chained[out] - ref[out]) / np.maximum(np.abs(ref[out]), 1e-3)
    assert rel.max() <= 1e-4


def test_chain_variants_replays_and_two_chains_per_list(ctx, b2, synth, orc):
    """Plain x quantized in the kernel, a pass reading the previous pass's image, a residual added in place, rows not
    a multiple of 32 (no image), a 9216-column pass; then a SILU_MUL that ends the first chain and a second chain.
    Three replays of the graph: the same bits each time, as the passes one by one."""
    ctx.reset_weights()
    r = rng(111)
    A = 1 << 16
    specs = [(2, 4096, 2560), (2, 2560, 4096), (8, 1000, 2560), (8, 9216, 2560), (2, 2560, 9216)]
    hs, ws = [], {}
    for fmt, rows, cols in specs:
        m = synth.matrix(fmt, r, rows, cols)
        h = ctx.upload(m, rows, cols, fmt)
        hs.append(h)
        ws[h] = (m.reshape(-1), rows, cols, fmt)
    X0, Y1, Y2, Y3, Y4, Y5, G = 0, 4096, 8192, 12288, 14336, 24576, 36864
    cl = b2.cmd_list(
        b2.gemv(2, 4096, 2560, hs[0], X0, Y1),                       # x from act
        b2.gemv(2, 2560, 4096, hs[1], Y1, X0, b2.GEMV_ADD),          # x = the image of Y1; X0 += W x (in place)
        b2.add(2560, X0, X0, X0),
        b2.gemv(8, 1000, 2560, hs[2], X0, Y2),                       # 1000 rows
        b2.silu_mul(1008, Y2, Y2, Y3),                               # not a GEMV: the first chain ends
        b2.gemv(8, 9216, 2560, hs[3], X0, Y4),
        b2.gemv(2, 2560, 9216, hs[4], Y4, Y5))                       # 9216 columns, x = the image of Y4
    act = np.zeros(A, np.float32)
    act[X0:X0 + 2560] = synth.activation(r, 2560)
    outs, k1 = _run(ctx, cl, act, ALL, replays=3)
    (passes,), k2 = _run(ctx, cl, act, ALL & ~b2.MASK_CHAINS)
    assert k1 < k2
    for o in outs:
        assert np.array_equal(o.view(np.uint32), passes.view(np.uint32))
    ref = act.copy()
    assert orc.run_list(ref, cl, ws) == 0
    for off, n in ((Y1, 4096), (X0, 2560), (Y2, 1000), (Y4, 9216), (Y5, 2560)):
        assert np.array_equal(outs[0][off:off + n].view(np.uint32), ref[off:off + n].view(np.uint32)), off
