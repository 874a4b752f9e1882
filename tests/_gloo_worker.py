"""Worker of tests/test_multi_rank_cpu.py: one gloo rank on the CPU. It runs the config-1 FFN block the way a
row-sharded context does — each GEMV's rows split by the library's own rule (b200q_row_slice), this rank's rows
computed by the oracle from its slice of the GGUF bytes, the slices all-gathered — and rank 0 saves the result."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))

from conftest import load_package, rng  # noqa: E402


def main():
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import oracle
    b2 = load_package()
    import fpga_llama_gguf_b200.synth as synth
    out = sys.argv[1]
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    r = rng(70)
    H, F = 512, 1024
    wg, wu, wd = synth.q8_0(r, F, H), synth.q8_0(r, F, H), synth.q8_0(r, H, F)
    x = synth.activation(r, H)
    gain = r.normal(1, 0.1, H).astype(np.float32)

    def sharded_gemv(w, xv, rows, cols):
        r0, r1 = b2.row_slice(rows, world, rank)
        rb = b2.gguf_row_bytes(cols, 8)
        mine, _ = oracle.gemv(w.reshape(-1)[r0 * rb:r1 * rb], xv, r1 - r0, cols, 8)
        parts = [torch.zeros(r1 - r0, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(mine)))
        return np.concatenate([p.numpy() for p in parts]) if (r1 - r0) != rows else mine

    xn = oracle.rownorm(x, gain, H, 1, 1e-6, 0)
    g, u = sharded_gemv(wg, xn, F, H), sharded_gemv(wu, xn, F, H)
    L = oracle.orc()
    h = np.array([L.orc_silu_mul1(float(a), float(b), 0) for a, b in zip(g, u)], np.float32)
    d = sharded_gemv(wd, h, H, F)
    y = (d + x).astype(np.float32)
    if rank == 0:
        np.savez(os.path.join(out, "sharded.npz"), y=y, x=x, gain=gain, wg=wg, wu=wu, wd=wd)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
