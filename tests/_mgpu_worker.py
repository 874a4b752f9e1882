"""Worker process of the multi-GPU tests: one rank on cuda:<rank>. It decodes tokens of the small hybrid model (the
same seeded weights on every rank) and rank 0 saves the greedy tokens, the act buffer and the DeltaNet states to
<out>/rank0.npz. Started by tests/test_multi_gpu.py with RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT in the
environment; the NCCL id for b200q travels through a gloo process group. MGPU_MODE: "rows" (default) a row-sharded
context that runs the one-rank lists; "tp" a tensor-parallel rank (COMM_EXPLICIT) running its own slice's lists.
MGPU_SHAPE: "small" (default) or "small8" (8 DeltaNet / query heads, which split over 4 ranks)."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))

from conftest import load_package  # noqa: E402


def main():
    import torch.distributed as dist
    from datetime import timedelta
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    out, n_tokens = sys.argv[1], int(sys.argv[2])
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    b2 = load_package()
    import fpga_llama_gguf_b200.decode as D
    from test_decode import SMALL
    shape = SMALL if os.environ.get("MGPU_SHAPE", "small") == "small" else D.Shape(
        hidden=1024, ffn=2048, n_layers=4, vocab=4096, gdn_heads=8, n_head=8, n_kv_head=2, head_dim=128, rope_dims=32,
        kv_ctx=640, prefill=64, head_piece=1536)
    tp = os.environ.get("MGPU_MODE", "rows") == "tp"
    ctx = b2.Context(device=rank, weight_bytes=1 << 30, act_floats=1 << 21, state_rows=8192, kv_bytes=64 << 20,
                     kv_ctx=shape.kv_ctx)
    obj = [b2.Context.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    if world > 1:
        ctx.comm_init(world, rank, obj[0], b2.COMM_EXPLICIT if tp else 0)
    m = D.HybridDecoder(shape, seed=9, world=world if tp else 1, rank=rank if tp else 0)
    SMALL = shape
    m.load(ctx)
    graphs = [ctx.graph(cl) for cl in m.token_lists()]
    toks = []
    for t in range(n_tokens):
        ctx.write(m.L.REC, m.record(SMALL.prefill + t))
        ctx.launch_many(graphs, len(graphs))
        toks.append(int(ctx.read(m.L.TOK, 1).view(np.uint32)[0]))
    act = ctx.read(0, m.L.size)
    state = ctx.read_state(0, SMALL.n_gdn * m.ls.gdn_rows)
    for g in graphs:
        g.close()
    ctx.close()
    if rank == 0:
        np.savez(os.path.join(out, "rank0.npz"), toks=np.array(toks), act=act, state=state,
                 logits=act[m.L.LOGITS:m.L.LOGITS + SMALL.vocab], x=act[m.L.X:m.L.X + SMALL.hidden])
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
