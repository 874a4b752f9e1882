"""The C-ABI library loads and exports every entry point include/b200q.h declares; the host-only layout repack keeps
every bit (no GPU needed)."""
import os
import re

import numpy as np
import pytest

from conftest import ROOT, rng


def test_exports_every_declared_symbol(b2):
    header = open(os.path.join(ROOT, "include", "b200q.h")).read()
    declared = set(re.findall(r"B200Q_API[^;(]*?\b(b200q_\w+)\s*\(", header))
    assert len(declared) >= 30
    L = b2.lib()
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing
    assert declared == set(b2.EXPORTED)


def test_features(b2):
    assert b2.features() == b2.FEATURES
    f = b2.features()
    assert f[0] >> 16 == 0x6B51 and f[1] >> 16 == 0x6B52 and f[2] >> 16 == 0x6B53


@pytest.mark.parametrize("fmt,cols", [(2, 2560), (2, 128), (8, 9216), (3, 384), (13, 2560), (14, 2560), (14, 256)])
@pytest.mark.parametrize("rows", [1, 17, 300])
def test_repack_roundtrip_keeps_bits(b2, synth, fmt, cols, rows):
    w = synth.matrix(fmt, rng(20, fmt, rows), rows, cols)
    dev = b2.repack_host(w, rows, cols, fmt)
    lay = b2.layout(rows, cols, fmt)
    assert dev.size == lay["total_bytes"] and lay["tile_bytes"] % 16 == 0
    for r in sorted({0, rows // 2, rows - 1}):
        assert np.array_equal(b2.unpack_row_host(dev, rows, cols, fmt, r), w[r])
    # the repack only moves bytes around: the multiset of bits is unchanged for the byte-aligned formats
    if fmt in (2, 8, 3):
        assert np.unpackbits(dev).sum() == np.unpackbits(w).sum()


def test_layout_panels_fill_the_warps(b2):
    # Q8_0 family: tiles of 32 units (P rows x 32 / P blocks, one warp step); P the largest whose panels (one per
    # CTA) fill between half and all of the 3 x 148 CTA slots, with at most 15% padding
    for rows, cols, fmt, P in [(9216, 2560, 8, 32), (2560, 9216, 8, 8), (9216, 2560, 2, 32), (4096, 2560, 2, 16),
                               (151936, 2560, 2, 32), (300, 512, 3, 2), (1024, 2560, 2, 4)]:
        lay = b2.layout(rows, cols, fmt)
        qb, db = {2: (16, 2), 8: (32, 2), 3: (16, 4)}[fmt]
        assert lay["rows_per_tile"] == P and lay["rows_per_tile"] * lay["blocks_per_tile"] == 32, (rows, lay)
        assert lay["tile_bytes"] == 32 * (qb + db)
        assert lay["tiles_per_row_tile"] == -(-cols // 32 // lay["blocks_per_tile"])
        assert lay["row_tiles"] == -(-rows // P)
    # K-quants: tiles of 32 rows (a lane each) x C super-blocks, C the largest divisor of the row's super-blocks up
    # to 8 whose tile is at most 34 KB; per row and super-block the packed quants, 16 scale bytes and d (Q5_K: d, dmin)
    for rows, cols, fmt, C in [(65520, 2560, 14, 5), (9216, 2560, 13, 5), (50688, 4096, 14, 4), (300, 9216, 13, 6),
                               (7, 256, 14, 1), (64, 2048, 13, 4), (64, 8192, 14, 4)]:
        lay = b2.layout(rows, cols, fmt)
        qb, dd = {14: (192, 2), 13: (160, 4)}[fmt]
        assert lay["rows_per_tile"] == 32 and lay["blocks_per_tile"] == C, (rows, cols, lay)
        assert lay["tile_bytes"] == 32 * C * (qb + 16) + -(-32 * C * dd // 16) * 16
        assert lay["row_tiles"] == -(-rows // 32) and lay["tiles_per_row_tile"] == cols // 256 // C


def test_layout_pass_hint(b2):
    # members of a multi-output pass (here the DeltaNet q/k/v, z, beta, alpha rows on one x: 8224 rows) take the
    # panel height of the whole pass, so that their panels make one wave of CTAs
    hint = b2.UPLOAD_PASS_ROWS(8224)
    for rows, alone in [(6144, 16), (2048, 8), (16, 2)]:
        assert b2.layout(rows, 2560, b2.Q4_0)["rows_per_tile"] == alone
        lay = b2.layout(rows, 2560, b2.Q4_0, flags=hint)
        assert lay["rows_per_tile"] == 32 and lay["row_tiles"] == -(-rows // 32)
        assert b2.weight_device_bytes(rows, 2560, b2.Q4_0, hint) == lay["total_bytes"]
    # K-quant tiles do not depend on the hint
    assert b2.layout(65520, 2560, 14, flags=hint) == b2.layout(65520, 2560, 14)


def test_device_bytes_and_row_bytes(b2):
    assert b2.gguf_row_bytes(2560, 2) == 80 * 18
    assert b2.gguf_row_bytes(2560, 14) == 10 * 210
    assert b2.lib().b200q_weight_device_bytes(9216, 2560, 2) >= 9216 * 80 * 18
