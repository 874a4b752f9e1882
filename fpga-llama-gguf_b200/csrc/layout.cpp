// Repack of GGUF rows into the device layout (see layout.h and kernel_args.h).
#include "layout.h"

#include <cstring>
#include <vector>

namespace b200q {
namespace {

// Q6_K element decode of one GGUF super-block (gemvq_ref.h:157-165): 6-bit value = low4 | high2 << 4.
void q6k_fields(const uint8_t *blk, uint8_t lo4[256], uint8_t hi2[256]) {
    const uint8_t *ql = blk, *qh = blk + 128;
    for (unsigned n = 0; n < 2; ++n)
        for (unsigned l = 0; l < 32; ++l) {
            const uint8_t h = qh[32 * n + l];
            lo4[128 * n + l] = ql[64 * n + l] & 0xF;
            hi2[128 * n + l] = (h >> 0) & 3;
            lo4[128 * n + l + 32] = ql[64 * n + l + 32] & 0xF;
            hi2[128 * n + l + 32] = (h >> 2) & 3;
            lo4[128 * n + l + 64] = ql[64 * n + l] >> 4;
            hi2[128 * n + l + 64] = (h >> 4) & 3;
            lo4[128 * n + l + 96] = ql[64 * n + l + 32] >> 4;
            hi2[128 * n + l + 96] = (h >> 6) & 3;
        }
}

void q6k_fields_inverse(const uint8_t lo4[256], const uint8_t hi2[256], uint8_t *blk) {
    uint8_t *ql = blk, *qh = blk + 128;
    std::memset(blk, 0, 192);
    for (unsigned n = 0; n < 2; ++n)
        for (unsigned l = 0; l < 32; ++l) {
            ql[64 * n + l] = uint8_t(lo4[128 * n + l] | lo4[128 * n + l + 64] << 4);
            ql[64 * n + l + 32] = uint8_t(lo4[128 * n + l + 32] | lo4[128 * n + l + 96] << 4);
            qh[32 * n + l] = uint8_t(hi2[128 * n + l] | hi2[128 * n + l + 32] << 2 | hi2[128 * n + l + 64] << 4 |
                                     hi2[128 * n + l + 96] << 6);
        }
}

// Device element of Q6_K decoded word G(j, p) byte b: the pairs (e, e + 8) of one 16-element sub-block j.
unsigned q6k_elem(unsigned j, unsigned p, unsigned b) {
    static const unsigned off[4] = {0, 8, 1, 9};
    return 16 * j + 2 * p + off[b];
}

// Device quant region of one Q6_K super-block: QL words 2j+h (low nibble G(j,2h), high nibble G(j,2h+1)),
// QH words j (bits 2p..2p+1 of byte b: G(j,p) byte b's high 2 bits).
void q6k_pack(const uint8_t lo4[256], const uint8_t hi2[256], uint8_t *qs) {
    std::memset(qs, 0, 192);
    for (unsigned j = 0; j < 16; ++j)
        for (unsigned p = 0; p < 4; ++p)
            for (unsigned b = 0; b < 4; ++b) {
                const unsigned e = q6k_elem(j, p, b);
                uint8_t &l = qs[4 * (2 * j + p / 2) + b];
                l |= uint8_t((p & 1) ? lo4[e] << 4 : lo4[e]);
                qs[128 + 4 * j + b] |= uint8_t(hi2[e] << (2 * p));
            }
}

void q6k_unpack(const uint8_t *qs, uint8_t lo4[256], uint8_t hi2[256]) {
    for (unsigned j = 0; j < 16; ++j)
        for (unsigned p = 0; p < 4; ++p)
            for (unsigned b = 0; b < 4; ++b) {
                const unsigned e = q6k_elem(j, p, b);
                const uint8_t l = qs[4 * (2 * j + p / 2) + b];
                lo4[e] = (p & 1) ? l >> 4 : l & 0xF;
                hi2[e] = (qs[128 + 4 * j + b] >> (2 * p)) & 3;
            }
}

// Q5_K (gemvq_ref.h:99-107): element 32s + e: low4 from qs[32 (s/2) + e] (nibble s & 1), high bit qh[e] bit s.
void q5k_fields(const uint8_t *blk, uint8_t lo4[256], uint8_t hb[256]) {
    const uint8_t *qh = blk + 16, *qs = blk + 48;
    for (unsigned s = 0; s < 8; ++s)
        for (unsigned e = 0; e < 32; ++e) {
            const uint8_t byte = qs[32 * (s / 2) + e];
            lo4[32 * s + e] = (s & 1) ? byte >> 4 : byte & 15;
            hb[32 * s + e] = (qh[e] >> s) & 1;
        }
}

void q5k_fields_inverse(const uint8_t lo4[256], const uint8_t hb[256], uint8_t *blk) {
    uint8_t *qh = blk + 16, *qs = blk + 48;
    std::memset(qh, 0, 32);
    std::memset(qs, 0, 128);
    for (unsigned s = 0; s < 8; ++s)
        for (unsigned e = 0; e < 32; ++e) {
            qs[32 * (s / 2) + e] |= uint8_t((s & 1) ? lo4[32 * s + e] << 4 : lo4[32 * s + e]);
            qh[e] |= uint8_t(hb[32 * s + e] << s);
        }
}

// Device Q5_K element of decoded word W(j, l) byte b: element 32j + l + 8b (the 4 elements with index % 8 == l).
// QL words 8(j/2) + l: low nibble W(2p, l), high nibble W(2p+1, l); QH words l: byte b bit j = high bit of W(j,l)[b].
void q5k_pack(const uint8_t lo4[256], const uint8_t hb[256], uint8_t *qs) {
    std::memset(qs, 0, 160);
    for (unsigned j = 0; j < 8; ++j)
        for (unsigned l = 0; l < 8; ++l)
            for (unsigned b = 0; b < 4; ++b) {
                const unsigned e = 32 * j + l + 8 * b;
                qs[4 * (8 * (j / 2) + l) + b] |= uint8_t((j & 1) ? lo4[e] << 4 : lo4[e]);
                qs[128 + 4 * l + b] |= uint8_t(hb[e] << j);
            }
}

void q5k_unpack(const uint8_t *qs, uint8_t lo4[256], uint8_t hb[256]) {
    for (unsigned j = 0; j < 8; ++j)
        for (unsigned l = 0; l < 8; ++l)
            for (unsigned b = 0; b < 4; ++b) {
                const unsigned e = 32 * j + l + 8 * b;
                const uint8_t v = qs[4 * (8 * (j / 2) + l) + b];
                lo4[e] = (j & 1) ? v >> 4 : v & 0xF;
                hb[e] = (qs[128 + 4 * l + b] >> j) & 1;
            }
}

}  // namespace

bool format_supported(unsigned f) { return f == 2 || f == 3 || f == 8 || f == 13 || f == 14; }

size_t gguf_row_bytes(unsigned cols, unsigned f) {
    switch (f) {
    case 2: return size_t(cols / 32) * 18;
    case 3: return size_t(cols / 32) * 20;
    case 8: return size_t(cols / 32) * 34;
    case 13: return size_t(cols / 256) * 176;
    case 14: return size_t(cols / 256) * 210;
    default: return 0;
    }
}

namespace {
unsigned align16(unsigned v) { return (v + 15u) & ~15u; }
}

DeviceLayout device_layout(unsigned rows, unsigned cols, unsigned f, unsigned sms, unsigned pass_rows) {
    DeviceLayout L;
    L.format = f;
    L.rows = rows;
    L.cols = cols;
    switch (f) {
    case 2: L.blocks = cols / 32; L.qb = 16; L.db = 2; break;
    case 3: L.blocks = cols / 32; L.qb = 16; L.db = 4; break;
    case 8: L.blocks = cols / 32; L.qb = 32; L.db = 2; break;
    case 13: L.blocks = cols / 256; L.qb = 160; L.db = 16; L.dd = 4; break;
    case 14: L.blocks = cols / 256; L.qb = 192; L.db = 16; L.dd = 2; break;
    default: return L;
    }
    if (rows == 0 || L.blocks == 0) return L;
    if (f == 2 || f == 3 || f == 8) {
        // Panels of P rows (one per CTA of a pass), streamed as steps of 32 units (P rows x J = 32 / P blocks; the
        // last step of a panel is zero-padded when J does not divide the blocks). P: the largest for which the
        // panels of the pass (of this matrix, or of all members of the multi-output pass it joins) fill between half
        // and all of the CTA slots of the GPU (one wave), with at most 15% padding; passes too large for one wave
        // take P = 32, too small ones the smallest P (most panels).
        const unsigned slots = (sms ? sms : 148u) * kPanelCtasPerSm;
        const unsigned fill_rows = pass_rows > rows ? pass_rows : rows;
        auto panels = [&](unsigned P) { return (fill_rows + P - 1) / P; };
        auto padded_ok = [&](unsigned P) {
            const unsigned J = 32u / P;
            return double((L.blocks + J - 1) / J * J) <= 1.15 * double(L.blocks);
        };
        unsigned P = 0;
        for (unsigned p = 32; p >= 1 && !P; p /= 2)
            if (2 * panels(p) >= slots && panels(p) <= slots && padded_ok(p)) P = p;
        if (!P && panels(32) > slots) P = 32;
        if (!P)
            for (unsigned p = 32; p >= 1; p /= 2)
                if (padded_ok(p)) P = p;
        if (!P) P = 1;
        L.rt = P;
        L.ct = 32u / P;
        L.kc = (L.blocks + L.ct - 1) / L.ct;
        L.n_rt = (rows + P - 1) / P;
        L.qs_part = 32u * L.qb;
        L.dm_part = 32u * L.db;
        L.dd_part = 0;
        L.tile_bytes = L.qs_part + L.dm_part;
        L.total = (size_t(L.n_rt) * L.kc * L.tile_bytes + 255) & ~size_t(255);
        return L;
    }
    // K-quants: row tiles of 32 rows (one per lane of a compute warp), tiles of C super-blocks (C the largest
    // divisor of the row's super-blocks up to 8 whose tile stays within kKqTileCap, so two stages and two CTAs fit
    // an SM; the compute warps share a tile's super-blocks out in parts). Inside a tile, step c (super-block c) holds
    // the 32 rows' packed quants word-interleaved (16-byte word q of row i at (c * qb / 16 + q) * 512 + 16 i, so a
    // warp reading word q of its 32 rows reads 512 contiguous bytes), then all steps' scales (16 bytes per row and
    // step), then their d (Q6_K) / d and dmin (Q5_K).
    L.rt = 32;
    unsigned C = 1;
    const unsigned per_sb = 32u * (L.qb + L.db + L.dd);
    for (unsigned c = 8; c > 1; --c)
        if (L.blocks % c == 0 && c * per_sb <= kKqTileCap) { C = c; break; }
    L.ct = C;
    L.kc = L.blocks / C;
    L.n_rt = (rows + 31) / 32;
    L.qs_part = 32 * C * L.qb;
    L.dm_part = 32 * C * L.db;
    L.dd_part = align16(32 * C * L.dd);
    L.tile_bytes = L.qs_part + L.dm_part + L.dd_part;
    L.total = (size_t(L.n_rt) * L.kc * L.tile_bytes + 255) & ~size_t(255);
    return L;
}

namespace {
// Byte addresses of block (row r, block b) of a layout.
struct BlockAt {
    size_t qs, dm, dd;
};
BlockAt block_at(const DeviceLayout &L, unsigned r, unsigned b) {
    const unsigned t = r / L.rt, rr = r % L.rt, k = b / L.ct, cc = b % L.ct;
    const size_t tile = (size_t(t) * L.kc + k) * L.tile_bytes;
    if (L.format == 13 || L.format == 14) {  // quant word q of this (row, super-block) at qs + q * 512
        const size_t i = size_t(cc) * 32 + rr;
        return {tile + size_t(cc) * (L.qb / 16) * 512 + size_t(rr) * 16, tile + L.qs_part + i * L.db,
                tile + L.qs_part + L.dm_part + i * L.dd};
    }
    const size_t i = size_t(rr) * L.ct + cc;
    return {tile + i * 16u, tile + L.qs_part + i * L.db, tile + L.qs_part + L.dm_part + i * L.dd};
}
// the packed quant words of a K-quant (row, super-block) to / from their interleaved places
void scatter_words(const uint8_t *packed, unsigned qb, uint8_t *qs) {
    for (unsigned q = 0; q < qb / 16; ++q) std::memcpy(qs + size_t(q) * 512, packed + 16 * q, 16);
}
void gather_words(const uint8_t *qs, unsigned qb, uint8_t *packed) {
    for (unsigned q = 0; q < qb / 16; ++q) std::memcpy(packed + 16 * q, qs + size_t(q) * 512, 16);
}
}  // namespace

void repack_rows(const uint8_t *gguf, unsigned row_begin, unsigned row_end, const DeviceLayout &L, uint8_t *dst) {
    const unsigned rows = row_end - row_begin, f = L.format;
    const size_t rb = gguf_row_bytes(L.cols, f);
    std::memset(dst, 0, L.total);
    uint8_t lo[256], hi[256], packed[192];
    for (unsigned r = 0; r < rows; ++r) {
        const uint8_t *row = gguf + size_t(row_begin + r) * rb;
        for (unsigned b = 0; b < L.blocks; ++b) {
            const BlockAt a = block_at(L, r, b);
            if (f == 2) {
                std::memcpy(dst + a.dm, row + size_t(b) * 18, 2);
                std::memcpy(dst + a.qs, row + size_t(b) * 18 + 2, 16);
            } else if (f == 8) {  // quant halves 512 bytes apart (32 units x 16 bytes)
                std::memcpy(dst + a.dm, row + size_t(b) * 34, 2);
                std::memcpy(dst + a.qs, row + size_t(b) * 34 + 2, 16);
                std::memcpy(dst + a.qs + 512, row + size_t(b) * 34 + 18, 16);
            } else if (f == 3) {
                std::memcpy(dst + a.dm, row + size_t(b) * 20, 4);
                std::memcpy(dst + a.qs, row + size_t(b) * 20 + 4, 16);
            } else if (f == 14) {
                const uint8_t *blk = row + size_t(b) * 210;
                q6k_fields(blk, lo, hi);
                q6k_pack(lo, hi, packed);
                scatter_words(packed, 192, dst + a.qs);
                std::memcpy(dst + a.dm, blk + 192, 16);
                std::memcpy(dst + a.dd, blk + 208, 2);
            } else {  // 13
                const uint8_t *blk = row + size_t(b) * 176;
                q5k_fields(blk, lo, hi);
                q5k_pack(lo, hi, packed);
                scatter_words(packed, 160, dst + a.qs);
                std::memcpy(dst + a.dm, blk + 4, 12);
                std::memcpy(dst + a.dd, blk, 4);
            }
        }
    }
}

void unpack_row(const uint8_t *dev, const DeviceLayout &L, unsigned r, uint8_t *out) {
    const unsigned f = L.format;
    uint8_t lo[256], hi[256], packed[192];
    for (unsigned b = 0; b < L.blocks; ++b) {
        const BlockAt a = block_at(L, r, b);
        if (f == 2) {
            std::memcpy(out + size_t(b) * 18, dev + a.dm, 2);
            std::memcpy(out + size_t(b) * 18 + 2, dev + a.qs, 16);
        } else if (f == 8) {
            std::memcpy(out + size_t(b) * 34, dev + a.dm, 2);
            std::memcpy(out + size_t(b) * 34 + 2, dev + a.qs, 16);
            std::memcpy(out + size_t(b) * 34 + 18, dev + a.qs + 512, 16);
        } else if (f == 3) {
            std::memcpy(out + size_t(b) * 20, dev + a.dm, 4);
            std::memcpy(out + size_t(b) * 20 + 4, dev + a.qs, 16);
        } else if (f == 14) {
            uint8_t *blk = out + size_t(b) * 210;
            gather_words(dev + a.qs, 192, packed);
            q6k_unpack(packed, lo, hi);
            q6k_fields_inverse(lo, hi, blk);
            std::memcpy(blk + 192, dev + a.dm, 16);
            std::memcpy(blk + 208, dev + a.dd, 2);
        } else {
            uint8_t *blk = out + size_t(b) * 176;
            std::memcpy(blk, dev + a.dd, 4);
            std::memcpy(blk + 4, dev + a.dm, 12);
            gather_words(dev + a.qs, 160, packed);
            q5k_unpack(packed, lo, hi);
            q5k_fields_inverse(lo, hi, blk);
        }
    }
}

}  // namespace b200q
