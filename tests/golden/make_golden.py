"""Generates tests/golden/*.npz: seeded small cases run through the reference's OWN CPU arithmetic
(fpga/src/gemvq_ref.h compiled from the reference sources into oracle/_ref/libgemvq_ref.so by oracle/Makefile).
The fixtures pin the oracle restatement where the reference tree is absent (the GPU box).

Run from the repository root:  python tests/golden/make_golden.py
"""
import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from conftest import load_package  # noqa: E402

import oracle  # noqa: E402

P = ctypes.c_void_p
OUT = os.path.dirname(os.path.abspath(__file__))


def ptr(a):
    return a.ctypes.data_as(P)


def main():
    load_package()
    import fpga_llama_gguf_b200.synth as synth
    R = oracle.ref()
    cases = {}
    for fmt, rows, cols in [(2, 48, 512), (8, 40, 384), (3, 24, 256), (13, 20, 512), (14, 20, 512)]:
        r = np.random.default_rng([0x601D, fmt])
        w = synth.matrix(fmt, r, rows, cols)
        x = synth.activation(r, cols)
        y, mag = oracle.ref_gemv(w, x, rows, cols, fmt)
        cases[f"gemv_{fmt}"] = dict(w=w, x=x, y=y, mag=mag, shape=np.array([rows, cols, fmt]))
    r = np.random.default_rng([0x601D, 100])
    x = np.concatenate([r.normal(0, 1, 1024), np.zeros(256), np.tile([2.0, -2.0], 128)]).astype(np.float32)
    q, d = np.zeros(x.size, np.int8), np.zeros(x.size // 256, np.float32)
    R.ref_quantize_q8_k(ptr(x), x.size, ptr(q), ptr(d))
    cases["q8k"] = dict(x=x, q=q, d=d)
    n, rows = 256, 2
    xn = r.normal(0, 1, n * rows).astype(np.float32)
    wn = r.normal(1, 0.1, n).astype(np.float32)
    for flags in (0, 1, 3):
        y = np.zeros(n * rows, np.float32)
        R.ref_rownorm(ptr(xn), ptr(wn), n, rows, np.float32(1e-6), flags, ptr(y))
        cases[f"rownorm_{flags}"] = dict(x=xn, w=wn, y=y, flags=np.array([flags]))
    g, u = r.normal(0, 3, 512).astype(np.float32), r.normal(0, 3, 512).astype(np.float32)
    y = np.zeros(512, np.float32)
    R.ref_silu_mul(ptr(g), ptr(u), 512, ptr(y))
    cases["silu_mul"] = dict(g=g, u=u, y=y)
    for kind in (1, 2, 3):
        y = np.zeros(512, np.float32)
        g10 = (g * 10).astype(np.float32)
        R.ref_unary(ptr(g10), 512, kind, ptr(y))
        cases[f"unary_{kind}"] = dict(x=g10, y=y)
    ch = 64
    st, xc, wc = (r.normal(0, 1, k * ch).astype(np.float32) for k in (3, 1, 4))
    y, ns = np.zeros(ch, np.float32), np.zeros(3 * ch, np.float32)
    R.ref_conv(ptr(st), ptr(xc), ptr(wc), ch, 1, ptr(y), ptr(ns))
    cases["conv"] = dict(state=st, x=xc, w=wc, y=y, new_state=ns)
    hv, hk = 2, 1
    s0 = r.normal(0, 0.1, hv * 128 * 128).astype(np.float32)
    q, k, v = (r.normal(0, 1, n_ * 128).astype(np.float32) for n_ in (hk, hk, hv))
    q /= np.linalg.norm(q)
    k /= np.linalg.norm(k)
    gg = (-np.log1p(np.exp(r.normal(0, 1, hv)))).astype(np.float32)
    bb = (1 / (1 + np.exp(-r.normal(0, 1, hv)))).astype(np.float32)
    s1 = s0.copy()
    yg = np.zeros(hv * 128, np.float32)
    R.ref_gdn(ptr(s1), ptr(q), ptr(k), ptr(v), ptr(gg), ptr(bb), hv, hk, np.float32(128 ** -0.5), ptr(yg), None, None)
    cases["gdn"] = dict(state=s0, q=q, k=k, v=v, g=gg, beta=bb, y=yg, new_state=s1)
    for name, arrays in cases.items():
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **arrays)
    print(f"wrote {len(cases)} fixtures to {OUT}")


if __name__ == "__main__":
    main()
