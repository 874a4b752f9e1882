"""Worker process of the multi-GPU tests: one rank of a row-sharded context on cuda:<rank>. It decodes tokens of the
small hybrid model (the same seeded weights on every rank) and rank 0 saves the greedy tokens, the act buffer and
the DeltaNet states to <out>/rank0.npz. Started by tests/test_multi_gpu.py with RANK / WORLD_SIZE / MASTER_ADDR /
MASTER_PORT in the environment; the NCCL id for b200q travels through a gloo process group."""
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
    ctx = b2.Context(device=rank, weight_bytes=1 << 30, act_floats=1 << 21, state_rows=8192, kv_bytes=64 << 20,
                     kv_ctx=SMALL.kv_ctx)
    obj = [b2.Context.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    if world > 1:
        ctx.comm_init(world, rank, obj[0])
    m = D.HybridDecoder(SMALL, seed=9)
    m.load(ctx)
    graphs = [ctx.graph(cl) for cl in m.token_lists()]
    toks = []
    for t in range(n_tokens):
        ctx.write(m.L.REC, m.record(SMALL.prefill + t))
        ctx.launch_many(graphs, len(graphs))
        toks.append(int(ctx.read(m.L.TOK, 1).view(np.uint32)[0]))
    act = ctx.read(0, m.L.size)
    state = ctx.read_state(0, SMALL.n_gdn * SMALL.gdn_rows)
    for g in graphs:
        g.close()
    ctx.close()
    if rank == 0:
        np.savez(os.path.join(out, "rank0.npz"), toks=np.array(toks), act=act, state=state)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
