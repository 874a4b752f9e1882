// GEMV pass for the K-quant weight formats Q5_K and Q6_K against Q8_K activations (up to four members on one x),
// bit-exact with ggml_vec_dot_q5_K_q8_K / q6_K_q8_K generic as restated in gemvq_ref.h:94-192:
//   per super-block the 8 integer lane sums aux[l] = sum over elements with (index % 8) == l of scale * y * w,
//   plus (Q5_K) the mins sum sum_j bsum16_j * m_(j/2); per row, in super-block order,
//   sums[l] += (d_w * d_x) * float(aux[l]), Q5_K: sumf -= (dmin_w * d_x) * float(mins); then sumf += sums[0..7].
//
// A producer warp streams tiles (32 rows x C super-blocks, layout.h) with bulk copies into a stage ring (and asks
// L2 for the next tiles ahead of it); compute warp w takes super-block w of the tile (C <= 4: half super-block w,
// so eight warps share four super-blocks) and each of its lanes one row: the lane forms the super-block's integer
// sums from the packed quant words (dp2a / dp4a; every lane of the warp reads the same activation words, a
// shared-memory broadcast) and writes them as one record; the fold warp adds each row's records (two halves: their
// integer sums) in super-block order. (An earlier mapping of 8 threads per super-block with shuffle reductions was
// instruction-bound at ~2 TB/s; splitting every super-block in eighths added through shared-memory atomics ran
// 25% slower than whole super-blocks at C = 5.)
//
// Roofline: HBM bandwidth, 176 (Q5_K) / 210 (Q6_K) bytes per 256 weights.
#include "gemv_common.cuh"
#include "launch.h"

namespace b200q {

constexpr unsigned kRecWords = 11;  // per (row, super-block): aux[8], mins, d | dmin << 16, pad (odd stride)

// y5: per (sb, j, l) int8x4 (y[32j+l], y[32j+l+8], y[32j+l+16], y[32j+l+24]); y6: per (sb, j, l) int16x2
// (y[16j+l], y[16j+l+8]). Word order inside a super-block: the 4-word groups that the eight parts of one
// (row, super-block) read together are adjacent, so a quarter-warp's 128-bit loads hit 32 distinct banks:
// y5 [sb][half h][part j][t] holds word (j, l = 4h + t); y6 [sb][jj][half h][part p][t] holds (j = 2p + jj, 4h + t).
__device__ __forceinline__ unsigned y5_word(unsigned j, unsigned l) { return ((l / 4) * 8 + j) * 4 + l % 4; }
__device__ __forceinline__ unsigned y6_word(unsigned j, unsigned l) {
    return (((j % 2) * 2 + l / 4) * 8 + j / 2) * 4 + l % 4;
}

__device__ __forceinline__ void build_transposed(const XImage &X, unsigned cols, bool need5, bool need6, uint32_t *y5,
                                                 uint32_t *y6) {
    const unsigned nsb = cols / 256, t = threadIdx.x - 32;
    if (need5) {
        for (unsigned i = t; i < nsb * 64; i += kXThreads) {
            const unsigned sb = i / 64, j = (i / 8) % 8, l = i % 8;
            const int8_t *y = X.q + sb * 256 + 32 * j + l;
            y5[sb * 64 + y5_word(j, l)] = uint32_t(uint8_t(y[0])) | uint32_t(uint8_t(y[8])) << 8 |
                                          uint32_t(uint8_t(y[16])) << 16 | uint32_t(uint8_t(y[24])) << 24;
        }
    }
    if (need6) {
        for (unsigned i = t; i < nsb * 128; i += kXThreads) {
            const unsigned sb = i / 128, j = (i / 8) % 16, l = i % 8;
            const int8_t *y = X.q + sb * 256 + 16 * j + l;
            y6[sb * 128 + y6_word(j, l)] = uint32_t(uint16_t(int16_t(y[0]))) | uint32_t(uint16_t(int16_t(y[8]))) << 16;
        }
    }
    named_sync_x();
}

// get_scale_min_k4 (gemvq_ref.h:83-92) on the 12 packed bytes
__device__ __forceinline__ void scale_min_k4_bytes(unsigned j, const uint8_t *q, int &sc, int &m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Q6_K super-block of one row: packed quant words at q + 512 k (k = 0..11; QL words 0..31, QH words 32..47, layout.cpp
// q6k_pack), 16 int8 scales at sc. Group j (16 elements): QL words 2j, 2j + 1 and QH word j give the four dp2a words
// G(j, p) holding elements (2p, 2p + 8, 2p + 1, 2p + 9) of the group, as 6-bit values minus 32.
__device__ __forceinline__ void sb_q6k(const uint8_t *q, const uint8_t *sc, unsigned sb, const uint32_t *y6,
                                       int aux[8]) {
    const uint32_t m4 = 0x0F0F0F0Fu, m2 = 0x30303030u;
    uint32_t QH[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint4 h = *reinterpret_cast<const uint4 *>(q + (8 + k) * 512);
        QH[4 * k] = h.x, QH[4 * k + 1] = h.y, QH[4 * k + 2] = h.z, QH[4 * k + 3] = h.w;
    }
    const uint4 s4 = *reinterpret_cast<const uint4 *>(sc);
    const uint32_t SW[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
    for (int l = 0; l < 8; ++l) aux[l] = 0;
#pragma unroll
    for (int jp = 0; jp < 8; ++jp) {
        const uint4 ql = *reinterpret_cast<const uint4 *>(q + jp * 512);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const int j = 2 * jp + jj;
            const uint32_t l0 = jj ? ql.z : ql.x, l1 = jj ? ql.w : ql.y, h = QH[j];
            const int scj = int(int8_t(SW[j / 4] >> (8 * (j % 4))));
            const uint4 ya = *reinterpret_cast<const uint4 *>(y6 + sb * 128 + y6_word(j, 0));
            const uint4 yb = *reinterpret_cast<const uint4 *>(y6 + sb * 128 + y6_word(j, 4));
            const uint32_t Y[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
            uint32_t g[4];
            g[0] = (l0 & m4) | ((h << 4) & m2);
            g[1] = ((l0 >> 4) & m4) | ((h << 2) & m2);
            g[2] = (l1 & m4) | (h & m2);
            g[3] = ((l1 >> 4) & m4) | ((h >> 2) & m2);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const int a = int(__vsub4(g[p], 0x20202020u));  // bytes w - 32 in -32..31
                aux[2 * p] += scj * __dp2a_lo(int(Y[2 * p]), a, 0);
                aux[2 * p + 1] += scj * __dp2a_hi(int(Y[2 * p + 1]), a, 0);
            }
        }
    }
}

// Q5_K super-block of one row: packed quant words at q + 512 k (k = 0..9; QL words 0..31, QH words 32..39, layout.cpp
// q5k_pack), 12 packed 6-bit scales / mins at dm. Sub-block j, class l: the 4 elements 32j + l + 8b, 5-bit values.
__device__ __forceinline__ void sb_q5k(const uint8_t *q, const uint8_t *dm, unsigned sb, const XImage &X,
                                       const uint32_t *y5, int aux[8], int &mins) {
    const uint32_t m4 = 0x0F0F0F0Fu;
    uint32_t QH[8];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint4 h = *reinterpret_cast<const uint4 *>(q + (8 + k) * 512);
        QH[4 * k] = h.x, QH[4 * k + 1] = h.y, QH[4 * k + 2] = h.z, QH[4 * k + 3] = h.w;
    }
    uint8_t sc12[12];
    {
        const uint4 d4 = *reinterpret_cast<const uint4 *>(dm);
        const uint32_t w[3] = {d4.x, d4.y, d4.z};
#pragma unroll
        for (int i = 0; i < 12; ++i) sc12[i] = uint8_t(w[i / 4] >> (8 * (i % 4)));
    }
#pragma unroll
    for (int l = 0; l < 8; ++l) aux[l] = 0;
    mins = 0;
#pragma unroll
    for (int jp = 0; jp < 4; ++jp) {  // sub-blocks 2jp (low nibbles) and 2jp + 1 (high nibbles) share QL words
        const uint4 qa = *reinterpret_cast<const uint4 *>(q + (2 * jp) * 512);
        const uint4 qb = *reinterpret_cast<const uint4 *>(q + (2 * jp + 1) * 512);
        const uint32_t QL[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const int j = 2 * jp + jj;
            int scj, mj;
            scale_min_k4_bytes(j, sc12, scj, mj);
            const uint4 ya = *reinterpret_cast<const uint4 *>(y5 + sb * 64 + y5_word(j, 0));
            const uint4 yb = *reinterpret_cast<const uint4 *>(y5 + sb * 64 + y5_word(j, 4));
            const uint32_t Y[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
#pragma unroll
            for (int l = 0; l < 8; ++l) {
                const uint32_t lo = jj ? ((QL[l] >> 4) & m4) : (QL[l] & m4);
                const uint32_t hi = ((QH[l] >> j) & 0x01010101u) << 4;
                aux[l] += scj * __dp4a(int(lo | hi), int(Y[l]), 0);
            }
            mins += (X.b[sb * 16 + 2 * j] + X.b[sb * 16 + 2 * j + 1]) * mj;
        }
    }
}

// Parts of a super-block (the integer lane sums of a super-block are the exact sums of its parts'):
// Q6_K part jp = groups 2jp, 2jp + 1 of 16 elements, Q5_K part jp = sub-blocks 2jp, 2jp + 1 of 32 elements.
// Q6_K part jp of one row's super-block: packed quant words at q + 512 k (k = 0..11; QL words 0..31, QH words
// 32..47, layout.cpp q6k_pack), 16 int8 scales at sc. Group j (16 elements): QL words 2j, 2j + 1 and QH word j give
// the four dp2a words G(j, p) holding elements (2p, 2p + 8, 2p + 1, 2p + 9) of the group, as 6-bit values minus 32.
__device__ __forceinline__ void part_q6k(const uint8_t *q, const uint8_t *sc, unsigned sb, unsigned jp,
                                         const uint32_t *y6, int aux[8]) {
    const uint32_t m4 = 0x0F0F0F0Fu, m2 = 0x30303030u;
    const uint4 ql = *reinterpret_cast<const uint4 *>(q + jp * 512);
    const uint2 qh = *reinterpret_cast<const uint2 *>(q + (8 + jp / 2) * 512 + (jp % 2) * 8);
    const uint32_t s2 = *reinterpret_cast<const uint16_t *>(sc + 2 * jp);
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
        const unsigned j = 2 * jp + jj;
        const uint32_t l0 = jj ? ql.z : ql.x, l1 = jj ? ql.w : ql.y, h = jj ? qh.y : qh.x;
        const int scj = int(int8_t(uint8_t(s2 >> (8 * jj))));
        const uint4 ya = *reinterpret_cast<const uint4 *>(y6 + sb * 128 + y6_word(j, 0));
        const uint4 yb = *reinterpret_cast<const uint4 *>(y6 + sb * 128 + y6_word(j, 4));
        const uint32_t Y[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
        uint32_t g[4];
        g[0] = (l0 & m4) | ((h << 4) & m2);
        g[1] = ((l0 >> 4) & m4) | ((h << 2) & m2);
        g[2] = (l1 & m4) | (h & m2);
        g[3] = ((l1 >> 4) & m4) | ((h >> 2) & m2);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const int a = int(__vsub4(g[p], 0x20202020u));  // bytes w - 32 in -32..31
            aux[2 * p] += scj * __dp2a_lo(int(Y[2 * p]), a, 0);
            aux[2 * p + 1] += scj * __dp2a_hi(int(Y[2 * p + 1]), a, 0);
        }
    }
}

// get_scale_min_k4 (gemvq_ref.h:83-92) for sub-block j = 4 hi + t of the 12 packed bytes w0 | w1 | w2
__device__ __forceinline__ void scale_min_k4(bool hi, unsigned t, uint32_t w0, uint32_t w1, uint32_t w2, int &sc,
                                             int &m) {
    const int b0 = int((w0 >> (8 * t)) & 0xffu), b1 = int((w1 >> (8 * t)) & 0xffu), b2 = int((w2 >> (8 * t)) & 0xffu);
    sc = hi ? ((b2 & 0xF) | ((b0 >> 6) << 4)) : (b0 & 63);
    m = hi ? ((b2 >> 4) | ((b1 >> 6) << 4)) : (b1 & 63);
}

// Q5_K part jp of one row's super-block: packed quant words at q + 512 k (k = 0..9; QL words 0..31, QH words
// 32..39, layout.cpp q5k_pack), 12 packed 6-bit scales / mins at dm. Sub-block j, class l: the 4 elements
// 32j + l + 8b, 5-bit values; sub-blocks 2jp (low nibbles) and 2jp + 1 (high nibbles) share QL words.
__device__ __forceinline__ void part_q5k(const uint8_t *q, const uint8_t *dm, unsigned sb, unsigned jp,
                                         const XImage &X, const uint32_t *y5, int aux[8], int &mins) {
    const uint32_t m4 = 0x0F0F0F0Fu;
    const uint4 h0 = *reinterpret_cast<const uint4 *>(q + 8 * 512), h1 = *reinterpret_cast<const uint4 *>(q + 9 * 512);
    const uint32_t QH[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const uint4 qa = *reinterpret_cast<const uint4 *>(q + (2 * jp) * 512);
    const uint4 qb = *reinterpret_cast<const uint4 *>(q + (2 * jp + 1) * 512);
    const uint32_t QL[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const uint4 d4 = *reinterpret_cast<const uint4 *>(dm);
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
        const unsigned j = 2 * jp + jj;
        int scj, mj;
        scale_min_k4(j >= 4, j & 3u, d4.x, d4.y, d4.z, scj, mj);
        const uint4 ya = *reinterpret_cast<const uint4 *>(y5 + sb * 64 + y5_word(j, 0));
        const uint4 yb = *reinterpret_cast<const uint4 *>(y5 + sb * 64 + y5_word(j, 4));
        const uint32_t Y[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t lo = jj ? ((QL[l] >> 4) & m4) : (QL[l] & m4);
            const uint32_t hi = ((QH[l] >> j) & 0x01010101u) << 4;
            aux[l] += scj * __dp4a(int(lo | hi), int(Y[l]), 0);
        }
        mins += (X.b[sb * 16 + 2 * j] + X.b[sb * 16 + 2 * j + 1]) * mj;
    }
}

// Records in a result buffer: (half h, super-block c, row) at word ((h C + c) 32 + row) kRecWords (an odd stride,
// so the 32 rows of a warp hit 32 banks): aux[8], mins, d | dmin << 16. Half 1 is used when the tile's super-blocks
// are split in halves (below); a row's sums are then the exact integer sums of its two halves'.
__host__ __device__ inline bool kq_halves(unsigned C) { return 2 * C <= kComputeWarps; }
// rows of records per super-block of a member's tile: 32, twice over with halves
__host__ __device__ inline unsigned kq_rec_rows(unsigned C) { return kq_halves(C) ? 64u : 32u; }

__device__ __forceinline__ void kq_store(uint32_t *o, const int aux[8], int mins, bool dd_too, uint32_t dd) {
#pragma unroll
    for (int l = 0; l < 8; ++l) o[l] = uint32_t(aux[l]);
    o[8] = uint32_t(mins);
    if (dd_too) o[9] = dd;
}

// One tile (32 rows x C super-blocks), lane i of a compute warp on row i. With C >= 5 compute warp w takes whole
// super-blocks w, w + 8, ...; with C <= 4 the 2 C half super-blocks (Q6_K groups 8h..8h+7, Q5_K sub-blocks
// 4h..4h+3) go one to a warp, so the tile's work is spread over twice as many warps.
__device__ __forceinline__ void compute_tile_kq(const uint8_t *tile, const MatrixView &w, unsigned nr, unsigned k,
                                                const XImage &X, const uint32_t *y5, const uint32_t *y6,
                                                uint32_t *rec) {
    const bool q5 = w.format == 13;
    const unsigned C = w.ct, QW = q5 ? 10u : 12u;
    const unsigned cw = threadIdx.x / 32 - 2, lane = threadIdx.x % 32;
    const uint8_t *scp = tile + w.qs_part, *ddp = tile + w.qs_part + w.dm_part;
    if (lane >= nr) return;
    auto dd_of = [&](unsigned r) {
        return q5 ? *reinterpret_cast<const uint32_t *>(ddp + r * 4)
                  : uint32_t(*reinterpret_cast<const uint16_t *>(ddp + r * 2));
    };
    if (!kq_halves(C)) {
        for (unsigned c = cw; c < C; c += kComputeWarps) {
            const unsigned sb = k * C + c, r = c * 32 + lane;
            const uint8_t *q = tile + size_t(c) * QW * 512 + lane * 16;
            int aux[8];
            int mins = 0;
            if (q5) sb_q5k(q, scp + r * 16, sb, X, y5, aux, mins);
            else sb_q6k(q, scp + r * 16, sb, y6, aux);
            kq_store(rec + r * kRecWords, aux, mins, true, dd_of(r));
        }
        return;
    }
    if (cw >= 2 * C) return;
    const unsigned c = cw / 2, h = cw % 2, sb = k * C + c, r = c * 32 + lane;
    const uint8_t *q = tile + size_t(c) * QW * 512 + lane * 16;
    int aux[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int mins = 0;
    if (q5) {
#pragma unroll
        for (unsigned t = 0; t < 2; ++t) part_q5k(q, scp + r * 16, sb, 2 * h + t, X, y5, aux, mins);
    } else {
#pragma unroll
        for (unsigned t = 0; t < 4; ++t) part_q6k(q, scp + r * 16, sb, 4 * h + t, y6, aux);
    }
    kq_store(rec + ((h * C + c) * 32 + lane) * kRecWords, aux, mins, h == 0, h == 0 ? dd_of(r) : 0u);
}

struct KqAcc {
    float sums[8];
    float sumf;
};

__device__ __forceinline__ void kq_reset(KqAcc &A) {
#pragma unroll
    for (int l = 0; l < 8; ++l) A.sums[l] = 0.0f;
    A.sumf = 0.0f;
}

// Integer sums of (row, super-block c) from its record(s): word l of half 0, plus half 1's when halves are used.
__device__ __forceinline__ int kq_sum(const uint32_t *rec, unsigned half_off, unsigned l) {
    return int32_t(rec[l]) + (half_off ? int32_t(rec[half_off + l]) : 0);
}

// The row's super-blocks of one tile, in order (gemvq_ref.h:122-131, 170-175); rec: the row's record of c = 0.
__device__ __forceinline__ void kq_fold(KqAcc &A, const uint32_t *rec, unsigned C, unsigned k, unsigned format,
                                        const XImage &X) {
    const unsigned ho = kq_halves(C) ? C * 32 * kRecWords : 0u;
    for (unsigned c = 0; c < C; ++c, rec += 32 * kRecWords) {
        const float dx = X.d[k * C + c];
        const float d = fmul(half_bits_to_float(uint16_t(rec[9] & 0xffffu)), dx);
#pragma unroll
        for (int l = 0; l < 8; ++l) A.sums[l] = fadd(A.sums[l], fmul(d, float(kq_sum(rec, ho, l))));
        if (format == 13) {
            const float dmin = fmul(half_bits_to_float(uint16_t(rec[9] >> 16)), dx);
            A.sumf = fsub(A.sumf, fmul(dmin, float(kq_sum(rec, ho, 8))));
        }
    }
}

// Debug pass: the exact integer sums of each (row, super-block) of the tile, 9 per super-block (mins last, 0 for
// Q6_K), instead of the rows.
__device__ __forceinline__ void kq_dump(int32_t *dbg, const uint32_t *rec, const MatrixView &w, unsigned row,
                                        unsigned k) {
    const unsigned C = w.ct, ho = kq_halves(C) ? C * 32 * kRecWords : 0u;
    for (unsigned c = 0; c < C; ++c, rec += 32 * kRecWords) {
        int32_t *d = dbg + (size_t(w.row0 + row) * (w.kc * C) + k * C + c) * 9;
#pragma unroll
        for (int l = 0; l < 8; ++l) d[l] = kq_sum(rec, ho, l);
        d[8] = w.format == 13 ? kq_sum(rec, ho, 8) : 0;
    }
}

__device__ __forceinline__ float kq_final(const KqAcc &A) {
    float s = A.sumf;
#pragma unroll
    for (int l = 0; l < 8; ++l) s = fadd(s, A.sums[l]);
    return s;
}

// PEERS: a row-sharded multi-GPU launch (rows also stored into the peers, ready / data flags).
template <bool PEERS>
__global__ void __launch_bounds__(kPassThreads, 2) gemv_kq_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const PassSmem P = carve_pass(smem, a);
    const XImage X = carve_ximage(P.ximg, a.cols);
    bool need5 = false, need6 = false;
    for (unsigned i = 0; i < a.n_members; ++i) {
        need5 |= a.m[i].w.format == 13;
        need6 |= a.m[i].w.format == 14;
    }
    // the activation tables: y5 (cols bytes) when a member is Q5_K, then y6 (2 cols bytes) when one is Q6_K
    uint32_t *y5 = reinterpret_cast<uint32_t *>(P.extra);
    uint32_t *y6 = y5 + (need5 ? a.cols / 4 : 0u);
    const unsigned warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) init_pass_barriers(a, P);
    __syncthreads();
    pdl_launch_dependents();
    if (warp == 0) {
        if (lane == 0) producer_loop(a, P);
        return;
    }
    pdl_wait();
    if (a.pw.n) {  // rows of earlier sharded launches: wait for the peers' (the x warps only; warp 0 streams)
        if (threadIdx.x == 32) peer_wait_rows(a.pw);
        named_sync_x();
    }
    prepare_x(a, P, X, 2);
    build_transposed(X, a.cols, need5, need6, y5, y6);
    TileIt it = tile_first(a);
    unsigned seq = 0;
    if (warp >= 2) {  // compute
        while (tile_valid(a, it)) {
            const unsigned s = seq % a.n_stages, b = seq % kNR;
            const bool ok = compute_acquire(P, seq, a.n_stages);
            if (!ok) {
                fail_pass(a, P.abort);
                break;
            }
            const GemvMemberArgs &M0 = unit_member(a, it.unit);
            const int pair = a.unit_pair[it.unit];
            const unsigned t = it.item - a.item_start[it.unit];
            const unsigned R = M0.w.rt, C = M0.w.ct;
            const unsigned r0 = t * R, nr = min(R, M0.w.rows - r0);
            uint32_t *rec = reinterpret_cast<uint32_t *>((b ? P.res[1] : P.res[0]));
            const uint8_t *stage = P.stages + size_t(s) * a.stage_bytes;
            compute_tile_kq(stage, M0.w, nr, it.k, X, y5, y6, rec);
            if (pair >= 0)
                compute_tile_kq(stage + pair_offset(M0.w.tile_bytes), a.m[pair].w, nr, it.k, X, y5, y6,
                                rec + size_t(kq_rec_rows(C)) * C * kRecWords);
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&P.empty[s]);
                mbar_arrive(&P.rfull[b]);
            }
            ++seq;
            tile_next(a, it);
        }
        return;
    }
    // fold (warp 1)
    constexpr bool peers = PEERS;
    if (peers && blockIdx.x == 0 && lane == 0) peer_announce(a.ps);
    const PeerSync *ps = nullptr;  // set once every peer has reached this launch (before the first store)
    if (peers) {
        const bool ok = __shfl_sync(0xffffffffu, lane == 0 ? peer_wait_ready(a.ps) : false, 0);
        if (ok) ps = &a.ps;
        else if (lane == 0 && a.err) atomicExch(a.err, 1u);
    }
    KqAcc A0, A1;
    kq_reset(A0);
    kq_reset(A1);
    while (tile_valid(a, it)) {
        const unsigned b = seq % kNR;
        if (!role_wait(&P.rfull[b], (seq / kNR) & 1u, P.abort)) {
            fail_pass(a, P.abort);
            break;
        }
        const GemvMemberArgs &M0 = unit_member(a, it.unit);
        const int pair = a.unit_pair[it.unit];
        const unsigned t = it.item - a.item_start[it.unit];
        const unsigned R = M0.w.rt, C = M0.w.ct;
        const unsigned r0 = t * R, nr = min(R, M0.w.rows - r0);
        const uint32_t *rec = reinterpret_cast<const uint32_t *>((b ? P.res[1] : P.res[0]));
        const uint32_t *rec_a = rec + lane * kRecWords, *rec_b = rec + (size_t(kq_rec_rows(C)) * C + lane) * kRecWords;
        if (a.dbg) {
            if (lane < nr) kq_dump(a.dbg, rec_a, M0.w, r0 + lane, it.k);
        } else {
            const bool last = it.k + 1 == M0.w.kc;
            if (lane < nr) {
                kq_fold(A0, rec_a, C, it.k, M0.w.format, X);
                if (pair >= 0) kq_fold(A1, rec_b, C, it.k, a.m[pair].w.format, X);
                if (last) {
                    const unsigned gr = M0.w.row0 + r0 + lane;
                    if (pair >= 0) write_row(a.m[pair], gr, kq_final(A1), kq_final(A0), nullptr, ps);
                    else write_row(M0, gr, kq_final(A0), 0.0f, nullptr, ps);
                    kq_reset(A0);
                    kq_reset(A1);
                }
            }
            if (last) write_padding(pair >= 0 ? a.m[pair] : M0, M0.w.row0 + r0 + nr, lane, ps);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&P.rempty[b]);
        ++seq;
        tile_next(a, it);
    }
    if (peers) {  // this CTA's rows are in every peer: count it; the last CTA raises the data flags
        __syncwarp();
        if (lane == 0) peer_signal(a.ps, gridDim.x);
    }
}

void plan_gemv_kq(GemvArgs &a, size_t &smem) {
    unsigned stage = 0, res = 0;
    for (unsigned u = 0; u < a.n_units; ++u) {
        const MatrixView &w = a.m[a.unit_member[u]].w;
        const bool pair = a.unit_pair[u] >= 0;
        const unsigned sb = pair ? pair_offset(w.tile_bytes) + w.tile_bytes : w.tile_bytes;
        stage = stage > sb ? stage : sb;
        const unsigned rb = (pair ? 2u : 1u) * kq_rec_rows(w.ct) * w.ct * kRecWords * 4u;
        res = res > rb ? res : rb;
    }
    a.stage_bytes = (stage + 127u) & ~127u;
    a.res_bytes = (res + 127u) & ~127u;
    bool need5 = false, need6 = false;
    for (unsigned i = 0; i < a.n_members; ++i) {
        need5 |= a.m[i].w.format == 13;
        need6 |= a.m[i].w.format == 14;
    }
    const size_t extra = (need5 ? size_t(a.cols) : 0u) + (need6 ? 2 * size_t(a.cols) : 0u);
    // as many stages as keep two CTAs per SM; then the norm weights in shared memory if they still fit
    a.wraw = 0;
    unsigned ns = kMaxStages;
    while (ns > 2 && pass_smem_bytes(ns, a.stage_bytes, a.res_bytes, a.cols, false, extra) > 113 * 1024) --ns;
    const bool norm_w = (a.norm_mode & 8u) && !(a.norm_mode & 2u) && !a.xq;
    if (norm_w && pass_smem_bytes(ns, a.stage_bytes, a.res_bytes, a.cols, true, extra) <= 113 * 1024) a.wraw = 1;
    a.n_stages = ns;
    smem = pass_smem_bytes(ns, a.stage_bytes, a.res_bytes, a.cols, a.wraw, extra);
}

cudaError_t launch_gemv_kq(const GemvArgs &a, unsigned grid, size_t smem, cudaStream_t st, bool pdl) {
    const void *k = a.ps.world > 1 ? reinterpret_cast<const void *>(gemv_kq_kernel<true>)
                                   : reinterpret_cast<const void *>(gemv_kq_kernel<false>);
    const cudaError_t e = ensure_smem_attr(k, 227 * 1024);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kPassThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return a.ps.world > 1 ? cudaLaunchKernelEx(&cfg, gemv_kq_kernel<true>, a)
                          : cudaLaunchKernelEx(&cfg, gemv_kq_kernel<false>, a);
}

}  // namespace b200q
