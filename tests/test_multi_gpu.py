"""Row-sharded decode on two GPUs (each rank stores its GEMV rows into the peer's act over NVLink, no collective)
against the same decode on one GPU: every row is computed by the same arithmetic on whichever rank holds it, so the
greedy tokens, the act buffer and the DeltaNet states are bit-identical. Needs two GPUs; skipped otherwise (the
single-GPU round-end run skips it)."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world: int, out: str, n_tokens: int, extra_env=None):
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                   NCCL_NVLS_ENABLE="0", TMPDIR=out, **(extra_env or {}))
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "_mgpu_worker.py"), out, str(n_tokens)],
                                      env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    logs = []
    for p in procs:
        try:
            o, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            p.kill()
            o, _ = p.communicate()
        logs.append(o.decode(errors="replace"))
    assert all(p.returncode == 0 for p in procs), "\n".join(logs)[-4000:]
    return np.load(os.path.join(out, "rank0.npz"))


@pytest.mark.gpu
@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["peer", "nccl"])
def test_two_gpu_sharded_decode_is_bit_identical_to_one_gpu(scratch, mode):
    one, two = os.path.join(scratch, "one"), os.path.join(scratch, "two")
    os.makedirs(one)
    os.makedirs(two)
    a = _run(1, str(one), 6)
    b = _run(2, str(two), 6, {"B200Q_PEER": "1" if mode == "peer" else "0"})
    assert list(a["toks"]) == list(b["toks"])
    assert np.array_equal(a["act"].view(np.uint32), b["act"].view(np.uint32))
    assert np.array_equal(a["state"].view(np.uint32), b["state"].view(np.uint32))
