"""Diagnostic modes on the GPU: the feature mask (B200Q_FEATURE_MASK / b200q_set_feature_mask) and runtime
verification (B200Q_VERIFY_CALLS / b200q_set_verify).

Feature mask: every fused form of this library gives the same values as its plain form, so a decode with any of the
executor's fusions switched off (multi-output passes, deferred norms in the GEMV prologue, the DeltaNet y image, the
pass-to-pass x image, the norm partials, programmatic dependent launch, fused norm / RoPE launches, the fused
attention gate, persistent GEMV chains; one at a time and all at once) gives bit-identical tokens, logits, act and states. The feature probe
reports the masked word, the format bits kept.

Runtime verification: a checker built on the CPU oracle sees the first n lists (direct runs and graph replays) with
act and state before and after, and agrees; a checker that disagrees (a mistake planted in the checker's copy of a
weight, on the CPU) makes the call fail with B200Q_ERR_VERIFY and disables the context."""
import numpy as np
import pytest

from conftest import rng

pytestmark = pytest.mark.gpu


def _shape(D):
    # the 4B-like layer shapes (so the fusions that depend on 32-row panels take part), 4 layers, a small vocabulary
    return D.Shape(n_layers=4, vocab=16384, head_piece=16384)


def _decode(b2, D, m, mask, tokens=2):
    with b2.Context(device=0, **m.context_config()) as ctx:
        ctx.set_feature_mask(mask)
        m.load(ctx)
        graphs = [ctx.graph(cl) for cl in m.token_lists()]
        kernels = sum(g.kernels for g in graphs)
        toks = []
        for t in range(tokens):
            ctx.write(m.L.REC, m.record(m.s.prefill + t))
            ctx.launch_many(graphs, len(graphs))
            toks.append(int(ctx.read(m.L.TOK, 1).view(np.uint32)[0]))
        act = ctx.read(0, m.L.size)
        state = ctx.read_state(0, m.s.n_gdn * m.s.gdn_rows)
        for g in graphs:
            g.close()
    return toks, act, state, kernels


def test_feature_probe_reports_the_mask(ctx, b2):
    full = b2.features()[0]
    ctx.set_feature_mask(~(b2.MASK_GROUPS | b2.MASK_DEFER_NORM | 1 | 0x2000) & 0xFFFFFFFF)
    try:
        ctx.fill(0, 0.0, 16)
        assert ctx.run(np.zeros(0, np.uint32)) == 0
        word = int(ctx.read(0, 1).view(np.uint32)[0])
        assert word == full & ~(b2.MASK_GROUPS | b2.MASK_DEFER_NORM)  # format / layout bits 0 and 13 stay
    finally:
        ctx.set_feature_mask(0xFFFFFFFF)
    assert ctx.feature_mask == 0xFFFFFFFF
    ctx.set_feature_mask(b2.DEFAULT_FEATURE_MASK)


def test_decode_is_bit_identical_under_every_feature_mask(b2):
    import fpga_llama_gguf_b200.decode as D
    m = D.HybridDecoder(_shape(D), seed=6)
    base = _decode(b2, D, m, 0xFFFFFFFF)  # every fusion on, the persistent chains too
    masks = {"groups": b2.MASK_GROUPS, "defer_norm": b2.MASK_DEFER_NORM, "gdn_out": b2.MASK_GDN_OUT,
             "x_image": b2.MASK_X_IMAGE, "norm_partials": b2.MASK_NORM_PARTIALS, "pdl": b2.MASK_PDL,
             "row_ops": b2.MASK_ROW_OPS, "attn_gate": b2.MASK_ATTN_GATE, "chains": b2.MASK_CHAINS}
    masks["all"] = sum(masks.values())
    for name, bits in masks.items():
        got = _decode(b2, D, m, ~bits & 0xFFFFFFFF)
        assert got[0] == base[0], name
        assert np.array_equal(got[1].view(np.uint32), base[1].view(np.uint32)), name
        assert np.array_equal(got[2].view(np.uint32), base[2].view(np.uint32)), name
        if name in ("groups", "defer_norm", "row_ops", "attn_gate", "chains", "all"):
            assert got[3] > base[3], name  # the plain forms take more launches


ACT = 32768  # the block's rows: x, gain, norm row, FF [9216], out


def _ffn_block(b2, synth, ctx, seed):
    H, F = 2560, 9216
    r = rng(95, seed)
    wg, wu, wd = synth.q4_0(r, F, H), synth.q4_0(r, F, H), synth.q4_0(r, H, F)
    hs = [ctx.upload(w, rows, cols, b2.Q4_0) for w, rows, cols in ((wg, F, H), (wu, F, H), (wd, H, F))]
    ws = {h: (w.reshape(-1), rows, cols, b2.Q4_0) for h, w, rows, cols in zip(hs, (wg, wu, wd), (F, F, H), (H, H, F))}
    cl = b2.cmd_list(
        b2.rmsnorm(H, 0, H, 2 * H, 1e-6, flags=b2.NORM_DEFER),
        b2.gemv(b2.Q4_0, F, H, hs[0], 2 * H, 4 * H, b2.GEMV_SWIGLU), b2.gemv(b2.Q4_0, F, H, hs[1], 2 * H, 4 * H),
        b2.gemv(b2.Q4_0, H, F, hs[2], 4 * H, 4 * H + F, b2.GEMV_ADD), b2.add(H, 4 * H + F, 0, 4 * H + F))
    act = np.zeros(ACT, np.float32)
    act[0:H] = synth.activation(r, H)
    act[H:2 * H] = r.normal(1, 0.1, H)
    return cl, ws, act


def _oracle_checker(orc, ws, seen):
    def check(view):
        n = view.act_floats
        before = np.ctypeslib.as_array(view.act_before, shape=(n,)).copy()
        after = np.ctypeslib.as_array(view.act_after, shape=(n,))
        cmds = np.ctypeslib.as_array(view.cmds, shape=(view.n_cmds * 8,)).copy()
        st = orc.run_list(before, cmds, ws)
        seen.append(view.n_cmds)
        if st != view.status or st != 0:
            return False, f"status {view.status} vs {st}"
        # GEMV outputs are bit-exact; SwiGLU (expf on the CPU, a once-rounded exp on the GPU) within 1e-4 relative
        bad = np.abs(after - before) > 1e-4 * np.maximum(np.abs(before), 1e-3)
        return (not bad.any()), f"{int(bad.sum())} values outside the tolerance"
    return check


def test_verify_calls_check_the_first_lists_against_the_oracle(ctx, b2, synth, orc):
    ctx.reset_weights()
    cl, ws, act = _ffn_block(b2, synth, ctx, 0)
    ctx.write(0, act)
    seen = []
    ctx.set_verify(_oracle_checker(orc, ws, seen), 3)
    try:
        for _ in range(2):
            assert ctx.run(cl) == 0
        g = ctx.graph(cl)
        ctx.launch_many([g], 3)  # the third verified list is the first replay; the rest run unchecked
        ctx.synchronize()
        g.close()
    finally:
        ctx.set_verify(None, 0)
    assert seen == [cl.size // 8] * 3


def test_a_disagreeing_checker_disables_the_context(b2, synth, orc):
    with b2.Context(device=0, weight_bytes=256 << 20, act_floats=ACT) as c:
        cl, ws, act = _ffn_block(b2, synth, c, 1)
        # the checker's copy of the down projection has one quant byte changed (a mistake planted on the CPU)
        h_down = max(ws)
        w = ws[h_down][0].copy()
        w[2] ^= 0x11
        ws[h_down] = (w,) + ws[h_down][1:]
        c.write(0, act)
        seen = []
        c.set_verify(_oracle_checker(orc, ws, seen), 1)
        with pytest.raises(b2.B200QError) as e:
            c.run(cl)
        assert e.value.code == b2.ERR_VERIFY and "outside the tolerance" in str(e.value)
        with pytest.raises(b2.B200QError) as e:
            c.run(cl)
        assert e.value.code == -4  # disabled
