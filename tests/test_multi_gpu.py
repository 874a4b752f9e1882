"""Decode on two (and four) GPUs against the same decode on one GPU. Needs two GPUs; skipped otherwise (the
single-GPU round-end run skips it).

Row-sharded (each rank's GEMV rows gathered by NCCL or stored into the peer's act over NVLink): every row is computed
by the same arithmetic on whichever rank holds it, so the greedy tokens, the act buffer and the DeltaNet states are
bit-identical to one GPU whose deferred norms also sum x's squares from x itself (the feature mask switches off the
per-panel partials a one-GPU run hands between passes, whose sum takes another fixed order).

Tensor parallel (each rank its own heads, FFN rows and column slices; ALLREDUCE per projection, by NCCL or by the
peer kernel): the same greedy tokens, logits within 1e-4 of the largest, the residual stream within 1e-4 (relative,
floor 1e-3), rank 0's DeltaNet states within 1e-4 of the one-GPU rows of its heads."""
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
    a = _run(1, str(one), 6, {"B200Q_FEATURE_MASK": str(0xFFFFFFFF & ~(1 << 17))})
    b = _run(2, str(two), 6, {"B200Q_PEER": "1" if mode == "peer" else "0"})
    assert list(a["toks"]) == list(b["toks"])
    assert np.array_equal(a["act"].view(np.uint32), b["act"].view(np.uint32))
    assert np.array_equal(a["state"].view(np.uint32), b["state"].view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("world,mode", [(2, "peer"), (2, "nccl"), (4, "peer")])
def test_tensor_parallel_decode_matches_one_gpu(scratch, world, mode):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    one, many = os.path.join(scratch, "one"), os.path.join(scratch, "many")
    os.makedirs(one)
    os.makedirs(many)
    env = {"MGPU_SHAPE": "small8"}
    a = _run(1, str(one), 6, env)
    b = _run(world, str(many), 6, dict(env, MGPU_MODE="tp", B200Q_PEER="1" if mode == "peer" else "0"))
    assert list(a["toks"]) == list(b["toks"])
    assert np.abs(a["logits"] - b["logits"]).max() <= 1e-4 * np.abs(a["logits"]).max()
    assert (np.abs(a["x"] - b["x"]) <= 1e-4 * np.maximum(np.abs(a["x"]), 1e-3)).all()
    # rank 0 holds the first heads of every DeltaNet layer
    n_gdn, heads, S = 3, 8, 128 * 128
    want = a["state"].reshape(n_gdn, heads, S)[:, :heads // world].reshape(-1)
    assert (np.abs(b["state"] - want) <= 1e-4 * np.maximum(np.abs(want), 1e-3)).all()
