"""Graph lowering (b200q_lower, host only): op graphs to command lists, the step the reference's backend does on its
ggml graph (plan / fusion analysis and emission, ggml-xrt.cpp:1815-2745).

  - an FFN block lowers to the fused commands (deferred weighted RMSNORM, SwiGLU GEMV pair, ADD epilogue), and with
    every feature bit cleared to the plain ones; both run on the oracle to the same values;
  - the synthetic hybrid decoder's token, written as an op graph (HybridDecoder.token_graph), lowers to the same
    command sequence as the hand-built lists (opcodes and flags, list by list) and decodes, on the oracle, the same
    tokens with bit-identical logits, DeltaNet states and KV cache;
  - tensor parallel: every rank's graph (ALLREDUCE / ALLGATHER nodes) lowers to that rank's hand-built lists, and the
    ranks' lowered lists, run in lock step, decode as the hand-built ones;
  - invalid graphs fail with the node named; b200q_node_supported follows the command limits;
  - random graphs: every lowering is refused cleanly or planner-valid, and random graphs of the fusable patterns give
    bit-identical outputs with every fusion and with none;
  - batched MUL_MATs (the prompt's rows) lower to GEMV_BATCH commands, and a batched FFN block gives, row by row,
    the bits of the one-row block."""
import numpy as np
import pytest

from conftest import rng


def _small_shape(D):
    return D.Shape(hidden=1024, ffn=2048, n_layers=4, vocab=4096, gdn_heads=4, n_head=4, n_kv_head=2, head_dim=128,
                   rope_dims=32, kv_ctx=128, prefill=64, head_piece=2048)


def _ops(cl):
    """(opcode, flags word) of each command, the GDN's extension slots skipped."""
    c = np.asarray(cl).reshape(-1, 8)
    out, i = [], 0
    while i < len(c):
        out.append((int(c[i][0]), int(c[i][1]) if c[i][0] in (1, 7, 12) else int(c[i][7] if c[i][0] == 2 else 0)))
        if c[i][0] == 7:
            out.append(("gdn-flags", int(c[i + 1][3])))
            i += 3 if c[i + 1][3] & 8 else 2
        else:
            i += 1
    return out


def _ffn_graph(G, b2, hs, H=1024, F=2048):
    g = G.Graph()
    x, w = g.input(H), g.param(H)
    xn = g.mul(g.rms_norm(x, 1e-6), w)
    ff = g.swiglu(g.mul_mat(xn, hs[0], b2.Q4_0, F, H), g.mul_mat(xn, hs[1], b2.Q4_0, F, H))
    y = g.add(g.mul_mat(ff, hs[2], b2.Q4_0, H, F), x)
    g.mark_output(y)
    g.end_segment()
    return g, x, w, y


def test_ffn_block_fuses_and_matches_the_plain_form(b2, orc, synth):
    import fpga_llama_gguf_b200.graph as G
    H, F = 1024, 2048
    r = rng(130)
    mats = [synth.q4_0(r, F, H), synth.q4_0(r, F, H), synth.q4_0(r, H, F)]
    hs = [4096, 8192, 12288]
    ws = {h: (m.reshape(-1), rows, cols, b2.Q4_0) for h, m, rows, cols in zip(hs, mats, (F, F, H), (H, H, F))}
    g, x, w, y = _ffn_graph(G, b2, hs)
    fused, plain = g.lower(), g.lower(features=0)
    assert [len(cl) // 8 for cl in fused.lists] == [5]
    assert _ops(fused.lists[0]) == [(2, b2.NORM_DEFER), (1, b2.Q4_0 | b2.GEMV_SWIGLU), (1, b2.Q4_0),
                                    (1, b2.Q4_0 | b2.GEMV_ADD), (3, 0)]
    assert _ops(plain.lists[0]) == [(2, 0), (1, b2.Q4_0), (1, b2.Q4_0), (4, 0), (1, b2.Q4_0), (3, 0)]
    for low in (fused, plain):
        assert b2.plan(low.lists[0])[0] == 0
    outs = []
    xv, wv = synth.activation(r, H), r.normal(1, 0.1, H).astype(np.float32)
    for low in (fused, plain):
        act = np.zeros(low.act_floats, np.float32)
        act[low.offset(x):low.offset(x) + H] = xv
        act[low.offset(w):low.offset(w) + H] = wv
        assert orc.run_list(act, low.lists[0], ws) == 0
        outs.append(act[low.offset(y):low.offset(y) + H].copy())
    # the SwiGLU epilogue and SILU_MUL apply the same arithmetic: the block gives the same bits either way
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_decoder_graph_lowers_to_the_hand_built_lists(b2, orc):
    import fpga_llama_gguf_b200.decode as D
    shape = _small_shape(D)
    m = D.HybridDecoder(shape, seed=5)
    ws = {}
    m.upload(lambda g_, rows, cols, fmt, bc, fl: (len(ws) + 1) * 4096, keep=ws)
    g, names = m.token_graph()
    low = g.lower()
    ref = m.token_lists()
    assert len(low.lists) == len(ref)
    for a, b in zip(low.lists, ref):
        assert _ops(a) == _ops(b)
        assert b2.plan(a)[0] == 0
    # the same decode on the oracle
    act1, st1, kv1 = m.initial_act(), m.initial_state(), m.initial_kv()
    act2, st2, kv2 = m.graph_act(names, low), st1.copy(), kv1.copy()
    for t in range(2):
        rec = m.record(shape.prefill + t)
        act1[m.L.REC:m.L.REC + D.RECORD] = rec
        r0 = low.offset(names["rec"])
        act2[r0:r0 + D.RECORD] = rec
        for cl in m.token_lists():
            assert orc.run_list(act1, cl, ws, state=st1, kv=kv1, kv_ctx=shape.kv_ctx) == 0
        for cl in low.lists:
            assert orc.run_list(act2, cl, ws, state=st2, kv=kv2, kv_ctx=shape.kv_ctx) == 0
        t1, t2 = m.L.TOK, low.offset(names["tok"])
        assert act1[t1:t1 + 2].view(np.uint32)[0] == act2[t2:t2 + 2].view(np.uint32)[0]
    l1, l2 = m.L.LOGITS, low.offset(names["logits"])
    assert np.array_equal(act1[l1:l1 + shape.vocab].view(np.uint32), act2[l2:l2 + shape.vocab].view(np.uint32))
    assert np.array_equal(st1.view(np.uint32), st2.view(np.uint32))
    assert np.array_equal(kv1, kv2)


def test_invalid_graphs_name_the_node(b2):
    import fpga_llama_gguf_b200.graph as G
    g = G.Graph()
    x = g.input(100)
    g.mul_mat(x, 4096, b2.Q4_0, 64, 100)  # 100 columns: not a multiple of 128
    with pytest.raises(b2.B200QError, match="node 1"):
        g.lower()
    assert not g.supported(1) and g.supported(0)
    g = G.Graph()
    x = g.input(1024)
    for _ in range(130):  # one segment of 130 commands does not fit a list
        x = g.add(x, x)
    with pytest.raises(b2.B200QError, match="segment 0 has 130 commands"):
        g.lower()
    g = G.Graph()
    x = g.input(1024)
    g.nodes.append(dict(op=G.NODE_ADD, n=1024, src=[x, 5], dst=-1, fmt=0, rows=0, cols=0, weight=0, eps=0.0, u=[],
                        flags=0))
    with pytest.raises(b2.B200QError, match="not an earlier node"):
        g.lower()


def test_segments_pack_into_lists_of_at_most_128_commands(b2):
    import fpga_llama_gguf_b200.graph as G
    g = G.Graph()
    x = g.input(1024)
    for s in range(5):  # five segments of 40 ADDs: 40 + 40 + 40, then 40 + 40
        for _ in range(40):
            x = g.add(x, x)
        g.end_segment()
    low = g.lower()
    assert [len(cl) // 8 for cl in low.lists] == [120, 80]


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_graphs_lower_to_the_hand_built_rank_lists(b2, orc, world):
    """Each rank's token graph (its slices, ALLREDUCE after every projection back to the hidden size, ALLGATHER of the
    logits) lowers to that rank's hand-built command sequence; run in lock step on the oracle (the collectives done
    between lists, tests/tp_emulation.py), the lowered lists of all ranks decode the same tokens with bit-identical
    logits as the hand-built ones."""
    import fpga_llama_gguf_b200.decode as D
    import tp_emulation as tp
    from test_tensor_parallel_cpu import _decoder_state, _shape
    shape = _shape(D, world)
    ranks = [D.HybridDecoder(shape, seed=7, world=world, rank=r) for r in range(world)]
    per = [_decoder_state(m) for m in ranks]
    ws = [p[0] for p in per]
    lowered = [m.token_graph() for m in ranks]
    lows = [g.lower() for g, _ in lowered]
    for m, low in zip(ranks, lows):
        ref = m.token_lists()
        assert len(low.lists) == len(ref)
        for a, b in zip(low.lists, ref):
            assert _ops(a) == _ops(b)
    acts1, states1, kvs1 = [p[1] for p in per], [p[2] for p in per], [p[3] for p in per]
    acts2 = [m.graph_act(names, low) for m, (_, names), low in zip(ranks, lowered, lows)]
    states2, kvs2 = [s.copy() for s in states1], [k.copy() for k in kvs1]
    for t in range(2):
        rec = ranks[0].record(shape.prefill + t)
        for m, a, (_, names), low in zip(ranks, acts1, lowered, lows):
            a[m.L.REC:m.L.REC + D.RECORD] = rec
        for a, (_, names), low in zip(acts2, lowered, lows):
            a[low.offset(names["rec"]):low.offset(names["rec"]) + D.RECORD] = rec
        tp.run_lists(orc, [m.token_lists() for m in ranks], acts1, ws, states1, kvs1, shape.kv_ctx)
        tp.run_lists(orc, [low.lists for low in lows], acts2, ws, states2, kvs2, shape.kv_ctx)
        for m, a1, a2, (_, names), low in zip(ranks, acts1, acts2, lowered, lows):
            assert a1[m.L.TOK:m.L.TOK + 1].view(np.uint32)[0] == \
                a2[low.offset(names["tok"]):low.offset(names["tok"]) + 1].view(np.uint32)[0]
    for m, a1, a2, (_, names), low in zip(ranks, acts1, acts2, lowered, lows):
        l1, l2 = m.L.LOGITS, low.offset(names["logits"])
        assert np.array_equal(a1[l1:l1 + shape.vocab].view(np.uint32), a2[l2:l2 + shape.vocab].view(np.uint32))


def test_random_graphs_either_fail_cleanly_or_give_valid_lists(b2):
    """Random graphs (ops and operands drawn at random, mostly well-formed, some not): the lowering either refuses with
    a message or returns lists the planner accepts; it never crashes."""
    import fpga_llama_gguf_b200.graph as G
    r = rng(131)
    sizes = [128, 256, 512, 1024, 2048]
    lowered = 0
    for trial in range(300):
        g = G.Graph()
        g.input(int(r.choice(sizes)))
        g.param(int(r.choice(sizes)))
        for _ in range(int(r.integers(1, 24))):
            k = len(g.nodes)
            x = int(r.integers(0, k))
            same = [i for i in range(k) if g.n(i) == g.n(x)]
            y = int(r.choice(same))
            kind = r.random()
            if kind < 0.25:
                fmt = int(r.choice([2, 3, 8]))
                if g.n(x) % 128 == 0:
                    g.mul_mat(x, 4096 * (1 + int(r.integers(0, 8))), fmt, int(r.choice(sizes)), g.n(x))
                else:
                    g.unary(x, 1)
            elif kind < 0.4:
                g.add(x, y)
            elif kind < 0.5:
                g.mul(x, y)
            elif kind < 0.6:
                g.swiglu(x, y)
            elif kind < 0.7:
                g.unary(x, int(r.integers(1, 5)))
            elif kind < 0.8:
                (g.rms_norm if r.random() < 0.7 else g.l2_norm)(x, 1e-6)
            elif kind < 0.85:
                base = x if g.nodes[x]["op"] != G.NODE_VIEW else g.nodes[x]["src"][0]
                g.view(base, 0, g.n(base))
            else:  # anything: random op, operands and sizes (mostly refused)
                op = int(r.integers(1, 19))
                g.nodes.append(dict(op=op, n=int(r.choice(sizes)), src=[int(r.integers(-1, k)) for _ in range(5)],
                                    dst=int(r.integers(-1, k)) if r.random() < 0.2 else -1, fmt=int(r.choice([2, 14])),
                                    rows=int(r.choice([0, 1, 4])), cols=int(r.choice(sizes)), weight=4096, eps=1e-6,
                                    u=[int(r.choice([0, 1, 2, 16, 128])) for _ in range(4)],
                                    flags=int(r.integers(0, 4))))
            if r.random() < 0.2:
                g.end_segment()
        try:
            low = g.lower(features=int(r.choice([0, G.ALL_FEATURES])))
        except b2.B200QError as e:
            assert "node" in str(e) or "segment" in str(e)
            continue
        lowered += 1
        for cl in low.lists:
            assert b2.plan(cl)[0] == 0, (trial, cl.reshape(-1, 8)[:4])
    assert lowered > 50, lowered


def test_random_graphs_compute_the_same_with_and_without_fusions(b2, orc, synth):
    """Random well-formed graphs built from the fusable patterns (norm x weight read by GEMVs, SwiGLU of two GEMVs on one
    x, GEMV + residual ADD, MUL by SILU / SIGMOID) and plain ops, lowered with every fusion and with none, give on the
    oracle bit-identical values for every tensor the caller marks as an output (outputs are never fused away)."""
    import fpga_llama_gguf_b200.graph as G
    r = rng(132)
    sizes = [256, 512, 1024]
    checked = fused_trials = 0
    for trial in range(60):
        g = G.Graph()
        ws = {}
        leaves = [g.input(int(r.choice(sizes))), g.param(int(r.choice(sizes)))]

        def mm(x, rows):
            fmt = int(r.choice([2, 8]))
            h = 4096 * (len(ws) + 1)
            ws[h] = (synth.matrix(fmt, r, rows, g.n(x)).reshape(-1), rows, g.n(x), fmt)
            return g.mul_mat(x, h, fmt, rows, g.n(x))

        for _ in range(int(r.integers(3, 10))):
            k = len(g.nodes)
            x = int(r.integers(0, k))
            same = [i for i in range(k) if g.n(i) == g.n(x)]
            y = int(r.choice(same))
            kind = r.random()
            if kind < 0.25:    # norm x weight, read by one to three GEMVs
                w = g.param(g.n(x))
                leaves.append(w)
                xn = g.mul(g.rms_norm(x, 1e-6), w)
                for _ in range(int(r.integers(1, 4))):
                    mm(xn, int(r.choice(sizes)))
            elif kind < 0.4:   # SwiGLU of two GEMVs on one x
                rows = int(r.choice(sizes))
                g.swiglu(mm(x, rows), mm(x, rows))
            elif kind < 0.55:  # GEMV + residual
                g.add(mm(x, g.n(y)), y)
            elif kind < 0.65:  # MUL by SILU / SIGMOID
                g.mul(x, g.unary(y, int(r.choice([1, 2]))))
            elif kind < 0.75:
                mm(x, int(r.choice(sizes)))
            elif kind < 0.85:
                g.add(x, y)
            elif kind < 0.95:
                g.unary(x, int(r.integers(1, 4)))
            else:
                base = x if g.nodes[x]["op"] != G.NODE_VIEW else g.nodes[x]["src"][0]
                g.view(base, 0, g.n(base))
            if r.random() < 0.3:
                g.mark_output(len(g.nodes) - 1)
        g.mark_output(len(g.nodes) - 1)
        outs = [i for i, d in enumerate(g.nodes) if d["flags"] & G.OUTPUT and d["op"] != G.NODE_VIEW]
        values = {i: r.normal(0, 1, g.n(i)).astype(np.float32) for i in leaves}
        results, shapes = [], []
        for feats in (G.ALL_FEATURES, 0):
            low = g.lower(features=feats)
            shapes.append([tuple(c.reshape(-1, 8)[:, :2].reshape(-1)) for c in low.lists])
            act = np.zeros(low.act_floats, np.float32)
            for i, v in values.items():
                act[low.offset(i):low.offset(i) + v.size] = v
            for cl in low.lists:
                assert b2.plan(cl)[0] == 0
                assert orc.run_list(act, cl, ws) == 0, trial
            results.append({i: act[low.offset(i):low.offset(i) + g.n(i)].copy() for i in outs})
        fused_trials += shapes[0] != shapes[1]
        for i in outs:
            assert np.array_equal(results[0][i].view(np.uint32), results[1][i].view(np.uint32)), (trial, i)
            checked += 1
    assert checked > 60 and fused_trials > 40, (checked, fused_trials)


def test_batched_ffn_block_is_the_one_row_block_for_every_row(b2, orc, synth):
    """The prompt's form of the FFN block: T rows through a multi-row RMS_NORM, batched MUL_MATs (one GEMV_BATCH
    command each, joining no fusion; more than 8 rows run as the tensor-core GEMM on the GPU), SWIGLU and ADD over all
    rows. On the oracle every output row has the bits of the one-row block on that row."""
    import fpga_llama_gguf_b200.graph as G
    H, F, T = 256, 512, 12
    r = rng(131)
    mats = [synth.q4_0(r, F, H), synth.q8_0(r, F, H), synth.q4_1(r, H, F)]
    fmts = [b2.Q4_0, b2.Q8_0, b2.Q4_1]
    hs = [4096, 8192, 12288]
    ws = {h: (m.reshape(-1), rows, cols, f) for h, m, rows, cols, f in zip(hs, mats, (F, F, H), (H, H, F), fmts)}
    g = G.Graph()
    x, w = g.input(T * H), g.param(H)
    xn = g.mul(g.rms_norm(x, 1e-6, rows=T), w)
    ff = g.swiglu(g.mul_mat(xn, hs[0], fmts[0], F, H, batch=T), g.mul_mat(xn, hs[1], fmts[1], F, H, batch=T))
    y = g.add(g.mul_mat(ff, hs[2], fmts[2], H, F, batch=T), x)
    g.mark_output(y)
    g.end_segment()
    low = g.lower()
    ops = [int(c) for c in np.asarray(low.lists[0]).reshape(-1, 8)[:, 0]]
    assert ops.count(17) == 3 and 1 not in ops, ops
    assert b2.plan(low.lists[0])[0] == 0
    xv = np.concatenate([synth.activation(r, H) * (1 + t % 3) for t in range(T)]).astype(np.float32)
    wv = r.normal(1, 0.1, H).astype(np.float32)
    act = np.zeros(low.act_floats, np.float32)
    act[low.offset(x):low.offset(x) + T * H] = xv
    act[low.offset(w):low.offset(w) + H] = wv
    assert orc.run_list(act, low.lists[0], ws) == 0
    got = act[low.offset(y):low.offset(y) + T * H].reshape(T, H)
    # the one-row block, every feature off (plain commands), row by row
    g1 = G.Graph()
    x1, w1 = g1.input(H), g1.param(H)
    xn1 = g1.mul(g1.rms_norm(x1, 1e-6), w1)
    ff1 = g1.swiglu(g1.mul_mat(xn1, hs[0], fmts[0], F, H), g1.mul_mat(xn1, hs[1], fmts[1], F, H))
    y1 = g1.add(g1.mul_mat(ff1, hs[2], fmts[2], H, F), x1)
    g1.mark_output(y1)
    g1.end_segment()
    one = g1.lower(features=0)
    for t in range(T):
        a1 = np.zeros(one.act_floats, np.float32)
        a1[one.offset(x1):one.offset(x1) + H] = xv[t * H:(t + 1) * H]
        a1[one.offset(w1):one.offset(w1) + H] = wv
        assert orc.run_list(a1, one.lists[0], ws) == 0
        assert np.array_equal(got[t].view(np.uint32), a1[one.offset(y1):one.offset(y1) + H].view(np.uint32)), t


def test_batched_mul_mat_limits(b2):
    import fpga_llama_gguf_b200.graph as G
    g = G.Graph()
    x = g.input(4 * 256)
    ok = g.mul_mat(x, 4096, b2.Q4_0, 100, 256, batch=4)
    kq = g.mul_mat(x, 4096, b2.Q6_K, 100, 256, batch=4)     # K-quants are not batched
    assert g.supported(ok) and not g.supported(kq)
    assert g.n(ok) == 4 * 112                               # rows padded to 16 floats, row by row
    g = G.Graph()
    x = g.input(4 * 256)
    v = g.view(x, 0, 128, 256, 4)                            # rows of 128 floats every 256: not contiguous
    g.mul_mat(v, 4096, b2.Q4_0, 100, 128, batch=4)
    g.end_segment()
    with pytest.raises(b2.B200QError, match="contiguous"):
        g.lower()
