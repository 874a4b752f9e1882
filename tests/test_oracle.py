"""The oracle restatement (oracle/oracle.c) against the reference's own gemvq_ref.h built from its sources
(oracle/_ref), and against the gguf package's Q8_0 quantizer. CPU only."""
import numpy as np
import pytest

from conftest import rng

FORMATS = [(2, 128 * 3), (8, 128 * 5), (3, 128 * 2), (13, 256 * 3), (14, 256 * 4)]


def _need_ref(orc):
    if not orc.ref_available():
        pytest.skip("reference build absent")


@pytest.mark.parametrize("fmt,cols", FORMATS)
def test_gemv_matches_reference_build_bitwise(orc, synth, fmt, cols):
    _need_ref(orc)
    r = rng(1, fmt)
    rows = 37
    w = synth.matrix(fmt, r, rows, cols)
    x = synth.activation(r, cols)
    y, mag = orc.gemv(w, x, rows, cols, fmt)
    yr, magr = orc.ref_gemv(w, x, rows, cols, fmt)
    assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))
    np.testing.assert_allclose(mag, magr, rtol=1e-12)


@pytest.mark.parametrize("fmt", [2, 8])
def test_gemv_edge_inputs(orc, synth, fmt):
    _need_ref(orc)
    r = rng(2, fmt)
    rows, cols = 16, 256
    w = synth.matrix(fmt, r, rows, cols)
    for x in (np.zeros(cols, np.float32),                       # all-zero blocks: d = 0, id = 0
              np.full(cols, 1e-30, np.float32),                  # fp16 scale underflows to 0
              np.where(np.arange(cols) % 2 == 0, 1.0, -1.0).astype(np.float32),  # ties of |x|
              (np.arange(cols, dtype=np.float32) - 128) * 1e-5):  # subnormal fp16 scales
        y, _ = orc.gemv(w, x, rows, cols, fmt)
        yr, _ = orc.ref_gemv(w, x, rows, cols, fmt)
        assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))


def test_quantize_q8_0_matches_gguf_package(orc):
    gguf = pytest.importorskip("gguf")
    from gguf.quants import quantize
    x = np.concatenate([rng(3).normal(0, 1, 2560), rng(4).normal(0, 0.001, 512),
                        np.zeros(64)]).astype(np.float32)
    q, d, _ = orc.quantize_q8_0(x)
    blocks = quantize(x.reshape(1, -1), gguf.GGMLQuantizationType.Q8_0).reshape(-1, 34)
    assert np.array_equal(blocks[:, :2].copy().view(np.uint16).reshape(-1), d)
    assert np.array_equal(blocks[:, 2:].view(np.int8).reshape(-1), q)


def test_quantize_q8_k_matches_reference_build(orc):
    _need_ref(orc)
    import ctypes
    x = np.concatenate([rng(5).normal(0, 1, 2560), np.zeros(256),
                        np.tile([3.0, -3.0, 1.0, 0.5], 64)]).astype(np.float32)  # zero block, tie +3/-3
    q, d, _ = orc.quantize_q8_k(x)
    qr, dr = np.zeros_like(q), np.zeros_like(d)
    orc.ref().ref_quantize_q8_k(x.ctypes.data_as(ctypes.c_void_p), x.size, qr.ctypes.data_as(ctypes.c_void_p),
                                dr.ctypes.data_as(ctypes.c_void_p))
    assert np.array_equal(q, qr) and np.array_equal(d.view(np.uint32), dr.view(np.uint32))


def test_half_conversions_match_reference(orc):
    _need_ref(orc)
    L, R = orc.orc(), orc.ref()
    vals = np.concatenate([rng(6).normal(0, 1e-5, 2000), rng(7).normal(0, 100, 2000),
                           [0.0, -0.0, 65504.0, 65520.0, 1e-8, 2.0 ** -25, 2.0 ** -24, 3 * 2.0 ** -26]])
    for v in vals.astype(np.float32):
        assert L.orc_float_to_half(v) == R.ref_float_to_half(v)
    for h in range(0, 65536, 7):
        a, b = L.orc_half_to_float(h), R.ref_half_to_float(h)
        assert (np.isnan(a) and np.isnan(b)) or np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)


def test_rownorm_matches_reference(orc):
    _need_ref(orc)
    import ctypes
    P = ctypes.c_void_p
    n, rows = 256, 3
    x = rng(8).normal(0, 1, n * rows).astype(np.float32)
    w = rng(9).normal(1, 0.1, n).astype(np.float32)
    for flags in (0, 1, 2, 3):
        y = orc.rownorm(x, w, n, rows, 1e-6, flags)
        yr = np.zeros_like(y)
        orc.ref().ref_rownorm(x.ctypes.data_as(P), w.ctypes.data_as(P), n, rows, 1e-6, flags, yr.ctypes.data_as(P))
        assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))


def test_gdn_matches_reference(orc):
    _need_ref(orc)
    import ctypes
    P = ctypes.c_void_p
    hv, hk = 4, 2
    r = rng(10)
    st = r.normal(0, 0.1, hv * 128 * 128).astype(np.float32)
    q, k = r.normal(0, 1, hk * 128).astype(np.float32), r.normal(0, 1, hk * 128).astype(np.float32)
    v = r.normal(0, 1, hv * 128).astype(np.float32)
    g = -np.log1p(np.exp(r.normal(0, 1, hv))).astype(np.float32)
    beta = (1 / (1 + np.exp(-r.normal(0, 1, hv)))).astype(np.float32)
    st2, y, _, _ = orc.gdn(st, q, k, v, g, beta, hv, hk, 128 ** -0.5)
    str_ = st.copy()
    yr = np.zeros(hv * 128, np.float32)
    orc.ref().ref_gdn(str_.ctypes.data_as(P), *[a.ctypes.data_as(P) for a in (q, k, v, g, beta)], hv, hk,
                      np.float32(128 ** -0.5), yr.ctypes.data_as(P), None, None)
    assert np.array_equal(st2.view(np.uint32), str_.view(np.uint32))
    assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))


def test_elementwise_match_reference(orc):
    _need_ref(orc)
    import ctypes
    P = ctypes.c_void_p
    n = 512
    a = rng(11).normal(0, 3, n).astype(np.float32)
    b = rng(12).normal(0, 3, n).astype(np.float32)
    L = orc.orc()
    y = np.array([L.orc_silu_mul1(float(g), float(u), 0) for g, u in zip(a, b)], np.float32)
    yr = np.zeros(n, np.float32)
    orc.ref().ref_silu_mul(a.ctypes.data_as(P), b.ctypes.data_as(P), n, yr.ctypes.data_as(P))
    assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))
    for kind in (1, 2, 3):
        y = np.array([L.orc_unary1(float(v), kind) for v in a * 10], np.float32)
        a10 = (a * 10).astype(np.float32)
        orc.ref().ref_unary(a10.ctypes.data_as(P), n, kind, yr.ctypes.data_as(P))
        assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))
    ch = 64
    st = rng(13).normal(0, 1, 3 * ch).astype(np.float32)
    x = rng(14).normal(0, 1, ch).astype(np.float32)
    w = rng(15).normal(0, 1, 4 * ch).astype(np.float32)
    y1, ns1 = np.zeros(ch, np.float32), np.zeros(3 * ch, np.float32)
    y2, ns2 = np.zeros(ch, np.float32), np.zeros(3 * ch, np.float32)
    L.orc_conv(st.ctypes.data_as(P), x.ctypes.data_as(P), w.ctypes.data_as(P), ch, 1, y1.ctypes.data_as(P),
               ns1.ctypes.data_as(P))
    orc.ref().ref_conv(st.ctypes.data_as(P), x.ctypes.data_as(P), w.ctypes.data_as(P), ch, 1, y2.ctypes.data_as(P),
                       ns2.ctypes.data_as(P))
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32)) and np.array_equal(ns1, ns2)
