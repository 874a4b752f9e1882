// One-time load-time repack of GGUF weight rows into the device layout of the GEMV kernels. Same role as the
// reference's gemvqw_layout::repack (fpga/src/gemvqw_layout.h:137-152), for a different machine: the reference
// groups scales and quants into 64-byte words for 20 FPGA engines; here a matrix becomes a sequence of tiles of
// R rows x C blocks, each tile one contiguous run of bytes that a single bulk copy (TMA) moves into shared memory:
//
//   tile (t, k) = rows [t R, t R + R) x blocks [k C, k C + C), at byte (t * KC + k) * tile_bytes, KC = blocks / C
//     [ quants : R x C x QB bytes, row-major (row, block) ]
//     [ scales : R x C x DB bytes, row-major, padded to 16 ]
//     [ K-quant d/dmin : R x C x DD bytes, row-major, padded to 16 ]
//
//   Q4_0: QB 16 = GGUF bytes 2..17 of the block, DB 2 = FP16 d (GGUF bytes 0..1)
//   Q8_0: QB 32 = GGUF bytes 2..33,              DB 2 = FP16 d
//   Q4_1: QB 16 = GGUF bytes 4..19,              DB 4 = FP16 d, FP16 m (GGUF bytes 0..3)
//   Q6_K: QB 192 = ql/qh fields permuted per super-block, DB 16 = int8 scales (GGUF 192..207), DD 2 = FP16 d
//   Q5_K: QB 160 = qs/qh fields permuted per super-block, DB 16 = packed scales (GGUF 4..15) + 4 zero bytes,
//         DD 4 = FP16 d, FP16 dmin (GGUF 0..3)
// Rows past the matrix in the last row tile are zero. Every scale and quant keeps its bits; the K-quant quant
// fields change position only (so one decoded 32-bit word feeds one dp4a / dp2a).
#pragma once
#include <cstddef>
#include <cstdint>

namespace b200q {

struct DeviceLayout {
    unsigned format = 0, rows = 0, cols = 0;
    unsigned blocks = 0;      // blocks (32) or super-blocks (256) per row
    unsigned qb = 0, db = 0, dd = 0;
    unsigned rt = 1;          // R: rows per tile
    unsigned ct = 1;          // C: blocks per tile
    unsigned kc = 1;          // tiles per row tile (blocks / C)
    unsigned n_rt = 0;        // row tiles
    unsigned qs_part = 0, dm_part = 0, dd_part = 0, tile_bytes = 0;
    size_t total = 0;         // all tiles, rounded up to 256 bytes
};

bool format_supported(unsigned format);
size_t gguf_row_bytes(unsigned cols, unsigned format);
// Tiling for `rows` rows on a GPU with `sms` multiprocessors: enough row tiles to balance the SMs, tiles of at
// most kTileTarget bytes.
constexpr unsigned kTileTarget = 12288, kTileTargetK = 16384;
DeviceLayout device_layout(unsigned rows, unsigned cols, unsigned format, unsigned sms = 148);
// Repacks GGUF rows [row_begin, row_end) into dst (a layout L made for row_end - row_begin rows).
void repack_rows(const uint8_t *gguf, unsigned row_begin, unsigned row_end, const DeviceLayout &L, uint8_t *dst);
// Inverse for one row (tests: the repack keeps every bit).
void unpack_row(const uint8_t *dev, const DeviceLayout &L, unsigned row, uint8_t *gguf_row);

}  // namespace b200q
