"""The oracle restatement against the committed golden vectors that tests/golden/make_golden.py produced with the
reference's own gemvq_ref.h (runs without the reference tree, e.g. on the GPU box). CPU only; bit-exact."""
import ctypes
import glob
import os

import numpy as np
import pytest

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
P = ctypes.c_void_p


def load(name):
    return np.load(os.path.join(HERE, f"{name}.npz"))


def _eq(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def test_fixture_set_present():
    assert len(glob.glob(os.path.join(HERE, "*.npz"))) == 15


@pytest.mark.parametrize("fmt", [2, 8, 3, 13, 14])
def test_gemv_golden(orc, fmt):
    g = load(f"gemv_{fmt}")
    rows, cols, f = (int(v) for v in g["shape"])
    y, mag = orc.gemv(g["w"], g["x"], rows, cols, f)
    assert _eq(y, g["y"])
    np.testing.assert_allclose(mag, g["mag"], rtol=1e-12)


def test_q8k_golden(orc):
    g = load("q8k")
    q, d, _ = orc.quantize_q8_k(g["x"])
    assert np.array_equal(q, g["q"]) and _eq(d, g["d"])


@pytest.mark.parametrize("flags", [0, 1, 3])
def test_rownorm_golden(orc, flags):
    g = load(f"rownorm_{flags}")
    y = orc.rownorm(g["x"], g["w"], 256, 2, 1e-6, flags)
    assert _eq(y, g["y"])


def test_elementwise_golden(orc):
    L = orc.orc()
    g = load("silu_mul")
    y = np.array([L.orc_silu_mul1(float(a), float(b), 0) for a, b in zip(g["g"], g["u"])], np.float32)
    assert _eq(y, g["y"])
    for kind in (1, 2, 3):
        g = load(f"unary_{kind}")
        y = np.array([L.orc_unary1(float(v), kind) for v in g["x"]], np.float32)
        assert _eq(y, g["y"])
    g = load("conv")
    y, ns = np.zeros(64, np.float32), np.zeros(192, np.float32)
    L.orc_conv(g["state"].ctypes.data_as(P), g["x"].ctypes.data_as(P), g["w"].ctypes.data_as(P), 64, 1,
               y.ctypes.data_as(P), ns.ctypes.data_as(P))
    assert _eq(y, g["y"]) and _eq(ns, g["new_state"])


def test_gdn_golden(orc):
    g = load("gdn")
    st, y, _, _ = orc.gdn(g["state"], g["q"], g["k"], g["v"], g["g"], g["beta"], 2, 1, 128 ** -0.5)
    assert _eq(st, g["new_state"]) and _eq(y, g["y"])
