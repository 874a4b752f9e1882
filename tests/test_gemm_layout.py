"""The prefill GEMM's weight addressing, restated on the CPU (no GPU): gemm_tc_kernel's loader thread for weight row r
of a 128-row tile reads block b of that row out of the device layout at unit u = (row % P) * C + b % C of tile
(row / P, b / C), and its expand step writes it into the MMA's canonical K-major layout. Here the same addressing runs
over the bytes the library's own repack produces (b200q_repack_host), for every panel height P the layout picks
(1 to 32 rows, C = 32 / P blocks per tile), and must give back every quant and scale of every GGUF row; the canonical
placement must be the layout the MMA's shared-memory descriptor describes (leading byte offset 128, stride byte
offset 256); and the decomposition itself (one integer product per block, FP32 terms folded in block order) gives
the oracle GEMV's bits. The GPU tests (test_gpu_gemm.py) check the kernel's results themselves."""
import numpy as np
import pytest

from conftest import rng


def _gguf_blocks(w, rows, cols, fmt):
    """Per row and block: the 32 int8 values the MMA must see, d (FP16 bits) and, for Q4_1, m."""
    nb = cols // 32
    bb = {2: 18, 8: 34, 3: 20}[fmt]
    b = np.asarray(w, np.uint8).reshape(rows, nb, bb)
    d = b[:, :, 0].astype(np.uint16) | (b[:, :, 1].astype(np.uint16) << 8)
    m = None
    if fmt == 8:
        q = b[:, :, 2:34].view(np.int8).astype(np.int32)
    else:
        qs = b[:, :, 4:20] if fmt == 3 else b[:, :, 2:18]
        lo, hi = (qs & 0x0F).astype(np.int32), (qs >> 4).astype(np.int32)
        q = np.concatenate([lo, hi], axis=2) - (8 if fmt == 2 else 0)
        if fmt == 3:
            m = b[:, :, 2].astype(np.uint16) | (b[:, :, 3].astype(np.uint16) << 8)
    return q, d, m


def _kernel_reads(dev, L, rows, cols, fmt):
    """What the loader threads of every 128-row tile read, block by block (rows past the panels: zero)."""
    P, C, KC, tb = L["rows_per_tile"], L["blocks_per_tile"], L["tiles_per_row_tile"], L["tile_bytes"]
    n_rt, nb = L["row_tiles"], cols // 32
    qs_part = 32 * (32 if fmt == 8 else 16)
    db = 4 if fmt == 3 else 2
    tiles = (rows + 127) // 128
    grow = np.arange(tiles * 128)
    pnl, rr = grow // P, grow % P
    have = pnl < n_rt
    q = np.zeros((tiles * 128, nb, 32), np.int32)
    d = np.zeros((tiles * 128, nb), np.uint16)
    m = np.zeros((tiles * 128, nb), np.uint16)
    g = grow[have]
    for b in range(nb):
        u = rr[have] * C + b % C
        tile = (pnl[have] * KC + b // C) * tb
        q0 = dev[(tile + u * 16)[:, None] + np.arange(16)]
        if fmt == 8:
            q1 = dev[(tile + 512 + u * 16)[:, None] + np.arange(16)]
            q[g, b] = np.concatenate([q0, q1], axis=1).view(np.int8).astype(np.int32)
        else:
            lo, hi = (q0 & 0x0F).astype(np.int32), (q0 >> 4).astype(np.int32)
            q[g, b] = np.concatenate([lo, hi], axis=1) - (8 if fmt == 2 else 0)
        w = tile + qs_part + ((u * db) & ~3)  # the 4-byte scale word the loader copies
        word = (dev[w].astype(np.uint32) | (dev[w + 1].astype(np.uint32) << 8) | (dev[w + 2].astype(np.uint32) << 16)
                | (dev[w + 3].astype(np.uint32) << 24))
        if fmt == 3:
            d[g, b], m[g, b] = word & 0xFFFF, word >> 16
        else:
            d[g, b] = np.where(u & 1, word >> 16, word & 0xFFFF)
    return q, d, m, have


@pytest.mark.parametrize("fmt", [2, 8, 3])
def test_loader_addressing_reads_every_block_for_every_panel_height(b2, synth, fmt):
    heights = set()
    shapes = [(256, 512), (600, 256), (1000, 512), (2560, 256), (4096, 256), (9216, 256), (100, 384), (300, 1024), (2561, 256)]
    for rows, cols in shapes:
        L = b2.layout(rows, cols, fmt)
        heights.add(L["rows_per_tile"])
        w = synth.matrix(fmt, rng(132, fmt, rows, cols), rows, cols)
        dev = b2.repack_host(w, rows, cols, fmt)
        q, d, m, have = _kernel_reads(dev, L, rows, cols, fmt)
        wq, wd, wm = _gguf_blocks(w, rows, cols, fmt)
        assert np.array_equal(q[:rows], wq), (rows, cols)
        assert np.array_equal(d[:rows], wd), (rows, cols)
        if fmt == 3:
            assert np.array_equal(m[:rows], wm), (rows, cols)
        # rows past the matrix inside the last panel are zero bytes in the layout (scale 0; Q4_0's zero nibbles enter
        # the MMA as -8), and the kernel stores no output for them; rows past the panels are not loaded
        pad = have[rows:]
        assert not d[rows:][pad].any() and np.all(q[rows:][pad] == (-8 if fmt == 2 else 0))
    assert heights == {1, 2, 4, 8, 16, 32}, heights


def test_canonical_placement_is_the_descriptors_layout():
    """expand writes row r's K half h at (r >> 3) * 256 + h * 128 + (r & 7) * 16; the descriptor (no swizzle,
    K-major) reads element (row m, k) at (m % 8) * 16 + (m // 8) * SBO + (k // 16) * LBO + k % 16."""
    lbo, sbo = 128, 256
    buf = np.full(4096, -1, np.int32)
    for r in range(128):
        for h in range(2):
            base = (r >> 3) * 256 + h * 128 + (r & 7) * 16
            buf[base:base + 16] = r * 32 + h * 16 + np.arange(16)
    m, k = np.meshgrid(np.arange(128), np.arange(32), indexing="ij")
    addr = (m % 8) * 16 + (m // 8) * sbo + (k // 16) * lbo + k % 16
    assert np.array_equal(buf[addr], m * 32 + k)
    assert np.array_equal(np.sort(addr.reshape(-1)), np.arange(4096))  # the 4 KB tile, each byte once


@pytest.mark.parametrize("fmt", [2, 8, 3])
def test_block_matmul_and_ordered_fold_is_the_oracle_gemv(b2, synth, orc, fmt):
    """The GEMM's decomposition, restated in numpy: per 32-value block one integer matrix product of the weight
    quants (Q4_0 nibbles - 8) with the tokens' Q8_0 / Q8_1 quants (what one int8 MMA computes for a tile), then the
    FP32 terms float(sumi) * (d_w * d_x) [Q4_1: (d_w * d_x) * float(sumi) + m_w * s_x] added in block order from 0,
    each operation rounded once. Every output has the oracle GEMV's bits."""
    rows, cols, T = 200, 512, 20
    r = rng(133, fmt)
    w = synth.matrix(fmt, r, rows, cols)
    xs = np.stack([synth.activation(r, cols) * (1 + t % 5) for t in range(T)]).astype(np.float32)
    wq, wd, wm = _gguf_blocks(w, rows, cols, fmt)
    dw = wd.view(np.float16).astype(np.float32)
    nb = cols // 32
    xq = np.zeros((T, nb, 32), np.int32)
    xd = np.zeros((T, nb), np.float32)
    xsum = np.zeros((T, nb), np.float32)
    for t in range(T):
        if fmt == 3:
            q, ds, _ = orc.quantize_q8_1(xs[t])
            pair = ds.reshape(nb, 2).view(np.float16).astype(np.float32)
            xd[t], xsum[t] = pair[:, 0], pair[:, 1]
        else:
            q, d, _ = orc.quantize_q8_0(xs[t])
            xd[t] = d.view(np.float16).astype(np.float32)
        xq[t] = q.reshape(nb, 32)
    acc = np.zeros((rows, T), np.float32)
    for b in range(nb):
        sumi = (wq[:, b, :] @ xq[:, b, :].T).astype(np.float32)  # exact: |sumi| < 2^24
        p = (dw[:, b, None] * xd[None, :, b]).astype(np.float32)
        if fmt == 3:
            mw = wm.view(np.float16).astype(np.float32)
            term = (p * sumi).astype(np.float32) + (mw[:, b, None] * xsum[None, :, b]).astype(np.float32)
        else:
            term = (sumi * p).astype(np.float32)
        acc = (acc + term.astype(np.float32)).astype(np.float32)
    for t in range(T):
        y, _ = orc.gemv(w, xs[t], rows, cols, fmt)
        assert np.array_equal(acc[:, t].view(np.uint32), y.view(np.uint32)), t
