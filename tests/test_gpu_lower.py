"""Lists lowered from an op graph (b200q_lower) on the GPU: the synthetic hybrid decoder's token graph, lowered, fused
and placed by the library, decodes the same tokens with bit-identical logits and DeltaNet states as the hand-built
lists, replayed as CUDA graphs."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _small_shape(D):
    return D.Shape(hidden=1024, ffn=2048, n_layers=4, vocab=4096, gdn_heads=4, n_head=4, n_kv_head=2, head_dim=128,
                   rope_dims=32, kv_ctx=128, prefill=64, head_piece=2048)


def test_lowered_graph_decodes_as_the_hand_built_lists(b2):
    import fpga_llama_gguf_b200.decode as D
    m = D.HybridDecoder(_small_shape(D), seed=5)
    cfg = m.context_config()
    cfg["act_floats"] = 4 * cfg["act_floats"]
    results = []
    for lowered in (False, True):
        with b2.Context(device=0, **cfg) as ctx:
            m.load(ctx)
            if lowered:
                g, names = m.token_graph()
                low = g.lower()
                assert low.act_floats <= cfg["act_floats"]
                ctx.write(0, m.graph_act(names, low))
                lists, rec_off, tok_off, lg_off = low.lists, low.offset(names["rec"]), low.offset(names["tok"]), \
                    low.offset(names["logits"])
            else:
                lists, rec_off, tok_off, lg_off = m.token_lists(), m.L.REC, m.L.TOK, m.L.LOGITS
            graphs = [ctx.graph(cl) for cl in lists]
            toks = []
            for t in range(3):
                ctx.write(rec_off, m.record(m.s.prefill + t))
                ctx.launch_many(graphs, len(graphs))
                toks.append(int(ctx.read(tok_off, 1).view(np.uint32)[0]))
            kernels = sum(gr.kernels for gr in graphs)
            logits = ctx.read(lg_off, m.s.vocab)
            state = ctx.read_state(0, m.s.n_gdn * m.s.gdn_rows)
            for gr in graphs:
                gr.close()
        results.append((toks, logits, state, kernels))
    (t1, l1, s1, k1), (t2, l2, s2, k2) = results
    assert t1 == t2
    assert np.array_equal(l1.view(np.uint32), l2.view(np.uint32))
    assert np.array_equal(s1.view(np.uint32), s2.view(np.uint32))
    print(f"kernels per token: hand-built {k1}, lowered {k2}")
