"""Weights loaded from a GGUF file through the library's reader, on the GPU: a small synthetic hybrid model written to
a .gguf file by the `gguf` package and loaded with b200q_upload_gguf_tensor decodes the same tokens, with bit-identical
logits, as the same model uploaded from memory; a Q4_0 matrix uploaded from ggml's CPU_REPACK layout
(B200Q_UPLOAD_SRC_Q4_0X8) gives the bit-identical GEMV of the plain upload and of the oracle."""
import numpy as np
import pytest

from conftest import rng
from test_gguf import to_q4_0x8, write_gguf

pytestmark = pytest.mark.gpu
gguf = pytest.importorskip("gguf")


def _small_shape(D):
    return D.Shape(hidden=1024, ffn=2048, n_layers=4, vocab=4096, gdn_heads=4, n_head=4, n_kv_head=2, head_dim=128,
                   rope_dims=32, kv_ctx=128, prefill=64, head_piece=2048)


def _decode(b2, D, m, load, tokens=3):
    with b2.Context(device=0, **m.context_config()) as ctx:
        load(ctx)
        graphs = [ctx.graph(cl) for cl in m.token_lists()]
        toks = []
        for t in range(tokens):
            ctx.write(m.L.REC, m.record(m.s.prefill + t))
            ctx.launch_many(graphs, len(graphs))
            toks.append(int(ctx.read(m.L.TOK, 1).view(np.uint32)[0]))
        logits = ctx.read(m.L.LOGITS, m.s.vocab)
        for g in graphs:
            g.close()
    return toks, logits


def test_model_from_a_gguf_file_decodes_as_from_memory(b2, tmp_path):
    import fpga_llama_gguf_b200.decode as D
    m = D.HybridDecoder(_small_shape(D), seed=5)
    ts = {name: (fmt, gen().reshape(rows, -1)) for name, fmt, rows, cols, bc, fl, gen in m.matrices()}
    path = str(tmp_path / "hybrid.gguf")
    write_gguf(path, ts, {"hybrid.block_count": m.s.n_layers})
    want = _decode(b2, D, m, m.load)
    with b2.GgufFile(path) as f:
        assert f.get_int("hybrid.block_count") == m.s.n_layers
        m2 = D.HybridDecoder(m.s, seed=5)
        got = _decode(b2, D, m2, lambda ctx: m2.load_gguf(ctx, f))
    assert got[0] == want[0]
    assert np.array_equal(got[1].view(np.uint32), want[1].view(np.uint32))


def test_q4_0x8_source_upload_matches_plain_upload_and_oracle(ctx, b2, synth, orc):
    ctx.reset_weights()
    rows, cols = 1024, 2560
    r = rng(93)
    w = synth.q4_0(r, rows, cols)
    x = synth.activation(r, cols)
    h_plain = ctx.upload(w, rows, cols, b2.Q4_0)
    h_x8 = ctx.upload(to_q4_0x8(w, rows, cols), rows, cols, b2.Q4_0, flags=b2.UPLOAD_SRC_Q4_0X8)
    ctx.write(0, x)
    assert ctx.run(b2.cmd_list(b2.gemv(b2.Q4_0, rows, cols, h_plain, 0, 4096),
                               b2.gemv(b2.Q4_0, rows, cols, h_x8, 0, 8192))) == 0
    a, b = ctx.read(4096, rows), ctx.read(8192, rows)
    y, _ = orc.gemv(w, x, rows, cols, b2.Q4_0)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert np.array_equal(b.view(np.uint32), y.view(np.uint32))
