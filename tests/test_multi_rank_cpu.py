"""The multi-rank host paths on the CPU with world_size-2 gloo process groups: the row-slice rule and its composition
(the FFN block computed rank by rank from the library's row slices and all-gathered equals the unsharded oracle
list bit for bit), and the bench's reference arm under torchrun (rank 0 alone prints its line)."""
import json
import os
import socket
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_row_slice_rule(b2):
    assert b2.row_slice(9216, 2, 1) == (4608, 9216)
    assert b2.row_slice(9216, 8, 3) == (3456, 4608)
    assert b2.row_slice(16, 2, 0) == (0, 16)                          # rows not divisible by 16 x world: replicated
    assert b2.row_slice(151936, 8, 7, b2.UPLOAD_REPLICATE) == (0, 151936)
    assert b2.row_slice(1000, 1, 0) == (0, 1000)
    # every rank's slice together covers the rows exactly once
    for rows, world in ((6144, 2), (6144, 4), (50688, 8), (2560, 8)):
        cover = [b2.row_slice(rows, world, k) for k in range(world)]
        assert cover[0][0] == 0 and cover[-1][1] == rows
        assert all(cover[k][1] == cover[k + 1][0] for k in range(world - 1))


def test_two_rank_row_sharded_ffn_block_is_bit_identical(b2, orc, scratch):
    port = _port()
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "_gloo_worker.py"), scratch],
                              env=dict(os.environ, RANK=str(k), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                                       MASTER_PORT=str(port), TMPDIR=scratch),
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT) for k in range(2)]
    logs = [p.communicate(timeout=180)[0].decode(errors="replace") for p in procs]
    assert all(p.returncode == 0 for p in procs), "\n".join(logs)[-3000:]
    z = np.load(os.path.join(scratch, "sharded.npz"))
    H, F = 512, 1024
    XIN, GAIN, XN, FF, OUT = 0, H, 2 * H, 4 * H, 4 * H + F
    act = np.zeros(OUT + H, np.float32)
    act[XIN:XIN + H], act[GAIN:GAIN + H] = z["x"], z["gain"]
    ws = {1 << 8: (z["wg"].reshape(-1), F, H, 8), 2 << 8: (z["wu"].reshape(-1), F, H, 8),
          3 << 8: (z["wd"].reshape(-1), H, F, 8)}
    cl = b2.cmd_list(
        b2.rmsnorm(H, XIN, GAIN, XN, 1e-6, flags=b2.NORM_DEFER),
        b2.gemv(8, F, H, 1 << 8, XN, FF, b2.GEMV_SWIGLU), b2.gemv(8, F, H, 2 << 8, XN, FF),
        b2.gemv(8, H, F, 3 << 8, FF, OUT, b2.GEMV_ADD), b2.add(H, OUT, XIN, OUT))
    assert orc.run_list(act, cl, ws) == 0
    assert np.array_equal(act[OUT:OUT + H].view(np.uint32), z["y"].view(np.uint32))


def test_reference_arm_under_torchrun_prints_one_line(scratch):
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", str(_port()), os.path.join(ROOT, "bench.py"),
                          "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1", "--cpu-budget", "0.5"],
                         capture_output=True, text=True, timeout=300,
                         env=dict(os.environ, OMP_NUM_THREADS="2", TMPDIR=scratch))
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["cpu_baseline"]["value"] > 0
