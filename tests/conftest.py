"""Shared test setup: the `gpu` marker, the package loader (its directory name has dashes) and seeded inputs."""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_package():
    name = "fpga_llama_gguf_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = os.path.join(ROOT, "fpga-llama-gguf_b200")
    spec = importlib.util.spec_from_file_location(name, os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libb200q.so")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def b2():
    return load_package()


@pytest.fixture(scope="session")
def synth(b2):
    import fpga_llama_gguf_b200.synth as s
    return s


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle


@pytest.fixture(scope="module")
def ctx(b2):
    if not has_gpu():
        pytest.skip("no GPU")
    c = b2.Context(device=0, weight_bytes=3 << 30, act_floats=1 << 22, state_rows=64 * 128, kv_bytes=64 << 20,
                   kv_ctx=640)
    yield c
    c.close()


@pytest.fixture
def scratch(request):
    """A fresh directory under tests/_scratch (git-ignored) for files the test's child processes exchange; also the
    TMPDIR of those processes. Removed after the test."""
    import shutil
    d = os.path.join(ROOT, "tests", "_scratch", f"{request.node.name}-{os.getpid()}".replace("/", "_"))
    shutil.rmtree(d, ignore_errors=True)
    os.makedirs(d)
    yield d
    shutil.rmtree(d, ignore_errors=True)


def rng(*salt):
    return np.random.default_rng([0x5EED, *salt])
