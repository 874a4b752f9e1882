"""The synthetic hybrid decoder (Qwen3.5-like token lists): list structure and byte accounting on the CPU, the
oracle's token loop on the CPU, and on the GPU the per-token CUDA Graph replay against the oracle's token loop on
the same seeded model."""
import numpy as np
import pytest

from conftest import load_package

b2 = load_package()
import fpga_llama_gguf_b200.decode as D  # noqa: E402

# a small model of the same structure (3 DeltaNet layers + 1 attention layer) for loops the oracle runs in seconds
SMALL = D.Shape(hidden=1024, ffn=2048, n_layers=4, vocab=4096, gdn_heads=4, n_head=4, n_kv_head=2, head_dim=128,
                rope_dims=32, kv_ctx=640, prefill=64, head_piece=2048)


def _fake_upload():
    nxt = [256]

    def up(g, rows, cols, fmt, bc, fl):
        h = nxt[0]
        nxt[0] += 256
        return h
    return up


def _oracle_tokens(orc, m, ws, n_tokens, act=None, state=None, kv=None):
    s, L = m.s, m.L
    act = m.initial_act() if act is None else act
    state = m.initial_state() if state is None else state
    kv = m.initial_kv() if kv is None else kv
    lists = m.token_lists()
    toks, logits = [], []
    for t in range(n_tokens):
        act[L.REC:L.REC + D.RECORD] = m.record(s.prefill + t)
        for cl in lists:
            assert orc.run_list(act, cl, ws, state=state, kv=kv, kv_ctx=s.kv_ctx) == 0
        toks.append(int(act[L.TOK:L.TOK + 1].view(np.uint32)[0]))
        logits.append(act[L.LOGITS:L.LOGITS + s.vocab].copy())
    return toks, logits, act, state, kv


def test_byte_counts_and_list_structure():
    """Bytes per token of the 4B-like and 9B-like shapes (layers + Q6_K head + KV at 512 + DeltaNet state r/w), and
    every token list plans with status 0 in at most 128 commands, with the fusions the model relies on."""
    assert D.SHAPE_4B.bytes_per_token() == 2_180_345_344
    assert D.SHAPE_9B.bytes_per_token() == 4_127_764_480
    for shape in (D.SHAPE_4B, D.SHAPE_9B, SMALL):
        m = D.HybridDecoder(shape)
        m.handles = {name: (k + 1) * 256 for k, (name, *_) in enumerate(m.matrices())}
        lists = m.token_lists()
        assert sum(len(c) // 8 for c in lists) == 1 + 16 * shape.n_gdn + 17 * shape.n_attn + 2 + len(shape.head_pieces())
        kinds = {}
        for cl in lists:
            assert len(cl) // 8 <= 128
            st, passes = b2.plan(cl)
            assert st == 0
            for p in passes:
                kinds[p["kind"]] = kinds.get(p["kind"], 0) + 1
                if p["kind"] == "gemv" and p["members"] == 4:
                    assert p["fused_norm"]  # qkv/z/beta/alpha on the deferred norm
                assert not p["stored_norm"]  # residual writes come after each norm's consumer
        # per DeltaNet layer: one 4-member group, the step with ssm_out fused, gate+up, down
        assert kinds["gdn"] == shape.n_gdn
        assert kinds["gemv"] == 3 * shape.n_gdn + 4 * shape.n_attn + 1


def test_small_model_oracle_token_loop():
    """Three tokens of the small model through the oracle: every list valid, tokens in range, each token's K/V row
    stored at its position of every attention slot, the DeltaNet states changed, and the next token's embedding is
    the row of the previous argmax."""
    import oracle as orc
    m = D.HybridDecoder(SMALL, seed=7)
    ws = {}
    m.upload(_fake_upload(), keep=ws)
    kv0 = m.initial_kv()
    state0 = m.initial_state()
    toks, logits, act, state, kv = _oracle_tokens(orc, m, ws, 3, state=state0.copy(), kv=kv0.copy())
    assert all(0 <= t < SMALL.vocab for t in toks)
    assert [int(np.argmax(lg)) for lg in logits] == toks
    s = SMALL
    slot = kv.view(np.float16).reshape(s.n_attn, 2, s.n_kv_head, s.kv_ctx, s.head_dim)
    for t in range(3):
        assert np.any(slot[:, :, :, s.prefill + t, :] != 0)
    assert not np.any(slot[:, :, :, s.prefill + 3:, :])
    assert np.array_equal(slot[:, :, :, :s.prefill, :],
                          kv0.view(np.float16).reshape(slot.shape)[:, :, :, :s.prefill, :])
    assert not np.array_equal(state, state0)
    emb = ws[m.handles["tok_embd"]][0].reshape(s.vocab, -1)
    want = orc.dequantize_row(emb[toks[-2]], s.hidden, b2.Q4_0)
    a2 = act.copy()
    a2[m.L.TOK] = np.array([toks[-2]], np.uint32).view(np.float32)[0]
    assert orc.run_list(a2, m.token_lists()[0][:8], ws, state=state.copy(), kv=kv.copy(), kv_ctx=s.kv_ctx) == 0
    assert np.array_equal(a2[m.L.X:m.L.X + s.hidden], want)


@pytest.mark.gpu
def test_small_model_graph_decode_matches_oracle(ctx, orc):
    """Eight tokens of the small model, each token the replay of its captured lists after a stream-ordered record
    write: the same greedy tokens as the oracle's loop, logits and DeltaNet states within 1e-4 relative (of the
    largest magnitude)."""
    ctx.reset_weights()
    m = D.HybridDecoder(SMALL, seed=8)
    ws = {}
    m.load(ctx, keep=ws)
    s, L = SMALL, m.L
    graphs = [ctx.graph(cl) for cl in m.token_lists()]
    rec = np.stack([m.record(s.prefill + t) for t in range(8)])
    out = np.zeros((8, 2), np.float32)
    for t in range(8):
        ctx.write_async(L.REC, rec[t].ctypes.data, D.RECORD)
        ctx.launch_many(graphs, len(graphs))
        ctx.read_async(L.TOK, out[t].ctypes.data, 2)
    ctx.synchronize()
    got_toks = [int(v) for v in out[:, 0].view(np.uint32)]
    toks, logits, act, state, kv = _oracle_tokens(orc, m, ws, 8)
    assert got_toks == toks
    got = ctx.read(0, L.size)
    lg, rl = got[L.LOGITS:L.LOGITS + s.vocab], act[L.LOGITS:L.LOGITS + s.vocab]
    assert np.abs(lg - rl).max() <= 1e-4 * np.abs(rl).max()
    gs = ctx.read_state(0, s.n_gdn * s.gdn_rows)
    assert np.abs(gs - state).max() <= 1e-4 * np.abs(state).max()
    for g in graphs:
        g.close()
