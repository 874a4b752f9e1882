"""Tensor-parallel decode lists (HybridDecoder with world > 1) on the CPU oracle: the ranks' slices of the one model,
run in lock step with their ALLREDUCE / ALLGATHER commands done between lists (tests/tp_emulation.py), decode the same
greedy tokens as the one-rank lists, with logits within 1e-4 of the largest logit and every rank's DeltaNet state
slice within 1e-4 (relative, floor 1e-3) of the one-rank state's rows for its heads. (Not bit for bit: the projections
split by columns add their partial sums in another order than the one-rank GEMV.)"""
import numpy as np
import pytest

import tp_emulation as tp


def _shape(D, world: int = 2):
    # 8 DeltaNet heads and 8 query heads over 2 KV heads: at 4 ranks two heads each and one KV head per two ranks;
    # 8 ranks: 16 heads of each kind over 4 KV heads (the 4B-like head counts), two per rank, one KV head per two ranks
    h, kv = (16, 4) if world == 8 else (8, 2)
    return D.Shape(hidden=1024, ffn=2048, n_layers=4, vocab=4096, gdn_heads=h, n_head=h, n_kv_head=kv, head_dim=128,
                   rope_dims=32, kv_ctx=128, prefill=64, head_piece=1536)


def _decoder_state(m):
    ws = {}
    m.upload(lambda g, rows, cols, fmt, bc, fl: len(ws) * 4096, keep=ws)
    return ws, m.initial_act(), m.initial_state(), m.initial_kv()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_lists_decode_as_one_rank(b2, orc, world):
    import fpga_llama_gguf_b200.decode as D
    shape = _shape(D, world)
    one = D.HybridDecoder(shape, seed=7)
    ws1, act1, st1, kv1 = _decoder_state(one)
    ranks = [D.HybridDecoder(shape, seed=7, world=world, rank=r) for r in range(world)]
    per = [_decoder_state(m) for m in ranks]
    ws = [p[0] for p in per]
    acts, states, kvs = [p[1] for p in per], [p[2] for p in per], [p[3] for p in per]
    toks, toks1 = [], []
    for t in range(2):
        rec = one.record(shape.prefill + t)
        act1[one.L.REC:one.L.REC + D.RECORD] = rec
        for cl in one.token_lists():
            assert orc.run_list(act1, cl, ws1, state=st1, kv=kv1, kv_ctx=shape.kv_ctx) == 0
        toks1.append(int(act1[one.L.TOK:one.L.TOK + 1].view(np.uint32)[0]))
        for m, a in zip(ranks, acts):
            a[m.L.REC:m.L.REC + D.RECORD] = rec
        tp.run_lists(orc, [m.token_lists() for m in ranks], acts, ws, states, kvs, shape.kv_ctx)
        got = {int(a[m.L.TOK:m.L.TOK + 1].view(np.uint32)[0]) for m, a in zip(ranks, acts)}
        assert len(got) == 1
        toks.append(got.pop())
    assert toks == toks1
    L1, L = one.L, ranks[0].L
    ref = act1[L1.LOGITS:L1.LOGITS + shape.vocab]
    for m, a in zip(ranks, acts):
        lg = a[L.LOGITS:L.LOGITS + shape.vocab]
        assert np.abs(lg - ref).max() <= 1e-4 * np.abs(ref).max()
        x = a[L.X:L.X + shape.hidden]
        x1 = act1[L1.X:L1.X + shape.hidden]
        assert (np.abs(x - x1) <= 1e-4 * np.maximum(np.abs(x1), 1e-3)).all()
    # every rank's DeltaNet heads against the one-rank state's rows for those heads
    S = D.GDN_DIM * D.GDN_DIM
    full = st1.reshape(shape.n_gdn, shape.gdn_heads, S)
    for m, st in zip(ranks, states):
        h0, h1 = m._gdn_heads()
        want = full[:, h0:h1].reshape(-1)
        rel = np.abs(st - want) / np.maximum(np.abs(want), 1e-3)
        assert rel.max() <= 1e-4, rel.max()


def test_tp_lists_split_the_model(b2):
    """Every rank's matrices together hold the one-rank model's bytes: row slices side by side, column slices of the
    projections, the embedding on every rank; each list's collectives are the same on every rank."""
    import fpga_llama_gguf_b200.decode as D
    shape = _shape(D)
    world = 2
    one = {m[0]: m for m in D.HybridDecoder(shape, seed=8).matrices()}
    ranks = [D.HybridDecoder(shape, seed=8, world=world, rank=r) for r in range(world)]
    mats = [{m[0]: m for m in r.matrices()} for r in ranks]
    for name in ("0.gate", "0.down", "0.wqkv", "0.ssm_out", "3.wo", "3.wk", "tok_embd"):
        full = one[name][6]().reshape(one[name][2], -1)
        parts = [mm[name][6]().reshape(mm[name][2], -1) for mm in mats]
        if name in ("0.down", "0.ssm_out", "3.wo"):
            assert np.array_equal(np.concatenate(parts, axis=1), full), name
        elif name == "tok_embd":
            assert all(np.array_equal(p, full) for p in parts)
        elif name == "3.wk":  # 2 KV heads, 2 ranks: one each
            assert np.array_equal(np.concatenate(parts), full)
        elif name == "0.wqkv":
            d = shape.gdn_rows
            for r, p in enumerate(parts):
                h = d // world
                want = np.concatenate([full[g * d + r * h:g * d + (r + 1) * h] for g in range(3)])
                assert np.array_equal(p, want)
        else:
            assert np.array_equal(np.concatenate(parts), full), name
    head1 = np.concatenate([one[f"output.{j}"][6]().reshape(-1) for j in range(len(shape.head_pieces()))])
    head = np.concatenate([mm[k][6]().reshape(-1) for mm in mats for k in sorted(mm) if k.startswith("output.")])
    assert np.array_equal(head, head1)
    for r in ranks:
        r.handles = {m[0]: 0 for m in r.matrices()}
    lists = [r.token_lists() for r in ranks]
    n_coll = [sum(1 for cl in ls for c in np.asarray(cl).reshape(-1, 8) if c[0] in (15, 16)) for ls in lists]
    assert n_coll[0] == n_coll[1] == 2 * shape.n_layers + 1
