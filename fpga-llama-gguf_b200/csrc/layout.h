// One-time load-time repack of GGUF weight rows into the device layout of the GEMV kernels. Same role as the
// reference's gemvqw_layout::repack (fpga/src/gemvqw_layout.h:137-152), for a different machine: the reference
// groups scales and quants into 64-byte words for 20 FPGA engines; here a matrix becomes a sequence of tiles of
// R rows x C blocks, each tile one contiguous run of bytes:
//
//   tile (t, k) = rows [t R, t R + R) x blocks [k C, k C + C), at byte (t * KC + k) * tile_bytes
//
// Q8_0 family (Q4_0, Q8_0, Q4_1): R x C = 32 units (R = P rows of a panel, C = 32 / P blocks), so one tile is
// one step of one warp, lane i = unit (i / C, i % C) reading 16-byte words at lane * 16 (coalesced 512 bytes):
//     [ quants : 32 x 16 bytes (Q8_0: first halves, then the second halves 512 bytes further) ]
//     [ scales : 32 x DB bytes ]
//   Q4_0: 16 quant bytes = GGUF bytes 2..17 of the block, DB 2 = FP16 d (GGUF bytes 0..1)
//   Q8_0: 2 x 16 quant bytes = GGUF bytes 2..17 and 18..33, DB 2 = FP16 d
//   Q4_1: 16 quant bytes = GGUF bytes 4..19, DB 4 = FP16 d, FP16 m (GGUF bytes 0..3)
//   KC = ceil(blocks / C): units past the last block, and rows past the matrix, are zero.
// K-quants (Q5_K, Q6_K): tiles of R = 32 rows x C super-blocks (C the largest divisor of the row's super-blocks
// up to 8 with C x 32 x (QB + DB + DD) <= kKqTileCap), each moved by one bulk copy (TMA) into shared memory; lane i
// of a compute warp owns row i:
//     [ quants : C steps x QB / 16 words x 32 rows x 16 bytes (word q of row i, step c at (c QB/16 + q) 512 + 16 i) ]
//     [ scales : C x R x DB bytes, (step, row) order ]
//     [ d/dmin : C x R x DD bytes, (step, row) order, padded to 16 ]
//   Q6_K: QB 192 = ql/qh fields permuted per super-block, DB 16 = int8 scales (GGUF 192..207), DD 2 = FP16 d
//   Q5_K: QB 160 = qs/qh fields permuted per super-block, DB 16 = packed scales (GGUF 4..15) + 4 zero bytes,
//         DD 4 = FP16 d, FP16 dmin (GGUF 0..3)
// Every scale and quant keeps its bits; the K-quant quant fields change position only (so one decoded 32-bit
// word feeds one dp4a / dp2a).
#pragma once
#include <cstddef>
#include <cstdint>

namespace b200q {

struct DeviceLayout {
    unsigned format = 0, rows = 0, cols = 0;
    unsigned blocks = 0;      // blocks (32) or super-blocks (256) per row
    unsigned qb = 0, db = 0, dd = 0;
    unsigned rt = 1;          // R: rows per tile (Q8_0 family: P, rows per panel)
    unsigned ct = 1;          // C: blocks per tile (Q8_0 family: 32 / P)
    unsigned kc = 1;          // tiles per row tile (ceil(blocks / C))
    unsigned n_rt = 0;        // row tiles
    unsigned qs_part = 0, dm_part = 0, dd_part = 0, tile_bytes = 0;
    size_t total = 0;         // all tiles, rounded up to 256 bytes
};

bool format_supported(unsigned format);
size_t gguf_row_bytes(unsigned cols, unsigned format);
// Tiling for `rows` rows on a GPU with `sms` multiprocessors: Q8_0-family panels for one wave of
// kPanelCtasPerSm CTAs per SM; K-quant tiles of 32 rows x up to 8 super-blocks, at most kKqTileCap bytes.
constexpr unsigned kPanelCtasPerSm = 3;
constexpr unsigned kKqTileCap = 34 * 1024;
// pass_rows: rows of the whole multi-output pass the matrix joins (its members' panels share one wave of CTAs), or 0
// for a matrix that is a pass of its own.
DeviceLayout device_layout(unsigned rows, unsigned cols, unsigned format, unsigned sms = 148, unsigned pass_rows = 0);
// Repacks GGUF rows [row_begin, row_end) into dst (a layout L made for row_end - row_begin rows).
void repack_rows(const uint8_t *gguf, unsigned row_begin, unsigned row_end, const DeviceLayout &L, uint8_t *dst);
// Inverse for one row (tests: the repack keeps every bit).
void unpack_row(const uint8_t *dev, const DeviceLayout &L, unsigned row, uint8_t *gguf_row);

}  // namespace b200q
