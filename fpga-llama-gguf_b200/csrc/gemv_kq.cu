// GEMV pass for the K-quant weight formats Q5_K and Q6_K against Q8_K activations (up to four members on one x),
// bit-exact with ggml_vec_dot_q5_K_q8_K / q6_K_q8_K generic as restated in gemvq_ref.h:94-192:
//   per super-block the 8 integer lane sums aux[l] = sum over elements with (index % 8) == l of scale * y * w,
//   plus (Q5_K) the mins sum sum_j bsum16_j * m_(j/2); per row, in super-block order,
//   sums[l] += (d_w * d_x) * float(aux[l]), Q5_K: sumf -= (dmin_w * d_x) * float(mins); then sumf += sums[0..7].
//
// Same tile pipeline as gemv_q8.cu (bulk copies into a stage ring, issued before the wait on the previous kernel).
// Eight threads share one (row, super-block): each takes 1/8 of it (Q5_K: one 32-element sub-block, Q6_K: two
// 16-element sub-blocks), computes partial lane sums with dp4a / dp2a on the permuted quant words of the device
// layout, and the eight partials are added exactly with shuffles (lane p ends with aux[p]). One thread per row then
// applies the FP32 fold in super-block order.
//
// Roofline: HBM bandwidth, 176 (Q5_K) / 210 (Q6_K) bytes per 256 weights.
#include "gemv_common.cuh"
#include "launch.h"

namespace b200q {

constexpr unsigned kRecWords = 12;  // per (row, super-block): aux[8], mins, d | dmin << 16, pad

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
__device__ __forceinline__ void scale_min_k4(unsigned j, const uint8_t *q, int &sc, int &m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Exact sum of the 8 partial lane-sum vectors of an aligned group of 8 lanes; lane p of the group gets aux[p].
__device__ __forceinline__ int reduce8(int v[8]) {
    const unsigned lane = threadIdx.x & 7u;
    int a1[4], a2[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const bool up = (lane & 4u) != 0;
        const int mine = up ? v[i + 4] : v[i], other = up ? v[i] : v[i + 4];
        a1[i] = mine + __shfl_xor_sync(0xffffffffu, other, 4);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const bool up = (lane & 2u) != 0;
        const int mine = up ? a1[i + 2] : a1[i], other = up ? a1[i] : a1[i + 2];
        a2[i] = mine + __shfl_xor_sync(0xffffffffu, other, 2);
    }
    const bool up = (lane & 1u) != 0;
    const int mine = up ? a2[1] : a2[0], other = up ? a2[0] : a2[1];
    return mine + __shfl_xor_sync(0xffffffffu, other, 1);
}

// Q5_K part p = sub-block j of (row, super-block) item i of the tile.
__device__ __forceinline__ void part_q5k(const uint8_t *qs, const uint8_t *dm, unsigned j, unsigned sb,
                                         const XImage &X, const uint32_t *y5, int aux[8], int &mins) {
    const uint4 l0 = *reinterpret_cast<const uint4 *>(qs + 32 * (j / 2));
    const uint4 l1 = *reinterpret_cast<const uint4 *>(qs + 32 * (j / 2) + 16);
    const uint4 h0 = *reinterpret_cast<const uint4 *>(qs + 128);
    const uint4 h1 = *reinterpret_cast<const uint4 *>(qs + 144);
    const uint32_t QL[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
    const uint32_t QH[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const uint4 ya = *reinterpret_cast<const uint4 *>(y5 + sb * 64 + y5_word(j, 0));
    const uint4 yb = *reinterpret_cast<const uint4 *>(y5 + sb * 64 + y5_word(j, 4));
    const uint32_t Y[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
    int sc, m;
    scale_min_k4(j, dm, sc, m);
#pragma unroll
    for (int l = 0; l < 8; ++l) {
        const uint32_t lo = (j & 1) ? ((QL[l] >> 4) & 0x0F0F0F0Fu) : (QL[l] & 0x0F0F0F0Fu);
        const uint32_t hi = ((QH[l] >> j) & 0x01010101u) << 4;
        aux[l] = sc * __dp4a(int(lo | hi), int(Y[l]), 0);
    }
    mins = (X.b[sb * 16 + 2 * j] + X.b[sb * 16 + 2 * j + 1]) * m;
}

// Q6_K part p = sub-blocks 2p, 2p + 1 of (row, super-block).
__device__ __forceinline__ void part_q6k(const uint8_t *qs, const uint8_t *dm, unsigned p, unsigned sb,
                                         const uint32_t *y6, int aux[8]) {
    const uint4 lw = *reinterpret_cast<const uint4 *>(qs + 16 * p);       // QL words 4p .. 4p + 3
    const uint2 hw = *reinterpret_cast<const uint2 *>(qs + 128 + 8 * p);  // QH words 2p, 2p + 1
    const uint16_t scw = *reinterpret_cast<const uint16_t *>(dm + 2 * p);
    const uint32_t m4 = 0x0F0F0F0Fu, m2 = 0x30303030u;
#pragma unroll
    for (int l = 0; l < 8; ++l) aux[l] = 0;
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
        const unsigned j = 2 * p + jj;
        const int sc = int(int8_t(scw >> (8 * jj)));
        const uint32_t l0 = jj ? lw.z : lw.x, l1 = jj ? lw.w : lw.y, h = jj ? hw.y : hw.x;
        const uint4 ya = *reinterpret_cast<const uint4 *>(y6 + sb * 128 + y6_word(j, 0));
        const uint4 yb = *reinterpret_cast<const uint4 *>(y6 + sb * 128 + y6_word(j, 4));
        const uint32_t Y[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
        uint32_t g[4];
        g[0] = (l0 & m4) | ((h << 4) & m2);
        g[1] = ((l0 >> 4) & m4) | ((h << 2) & m2);
        g[2] = (l1 & m4) | (h & m2);
        g[3] = ((l1 >> 4) & m4) | ((h >> 2) & m2);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int a = int(__vsub4(g[q], 0x20202020u));  // bytes w - 32 in -32..31
            aux[2 * q] += sc * __dp2a_lo(int(Y[2 * q]), a, 0);
            aux[2 * q + 1] += sc * __dp2a_hi(int(Y[2 * q + 1]), a, 0);
        }
    }
}

// One tile: items (row, super-block) x 8 parts.
__device__ __forceinline__ void compute_tile_kq(const uint8_t *tile, const MatrixView &w, unsigned nr, unsigned k,
                                                const XImage &X, const uint32_t *y5, const uint32_t *y6,
                                                uint32_t *rec, int32_t *dbg, unsigned r0) {
    const unsigned C = w.ct, items = nr * C * 8;
    const unsigned QB = w.format == 13 ? 160u : 192u;
    const unsigned DD = w.format == 13 ? 4u : 2u;
    const uint8_t *dmp = tile + w.qs_part, *ddp = tile + w.qs_part + w.dm_part;
    // items beyond the tile run the shuffles with zero work (the whole warp takes part in every round)
    const unsigned rounds = (items + kComputeThreads - 1) / kComputeThreads, ct = threadIdx.x - 64;
    for (unsigned rd = 0; rd < rounds; ++rd) {
        const unsigned idx = rd * kComputeThreads + ct;
        const bool live = idx < items;
        const unsigned i = live ? idx / 8 : 0, p = idx & 7u;  // i = r * C + c
        const unsigned c = i % C, sb = k * C + c;
        int aux[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int mins = 0;
        if (live) {
            const uint8_t *qs = tile + size_t(i) * QB, *dm = dmp + size_t(i) * 16;
            if (w.format == 13) part_q5k(qs, dm, p, sb, X, y5, aux, mins);
            else part_q6k(qs, dm, p, sb, y6, aux);
        }
        const int mine = reduce8(aux);
        mins += __shfl_xor_sync(0xffffffffu, mins, 4);
        mins += __shfl_xor_sync(0xffffffffu, mins, 2);
        mins += __shfl_xor_sync(0xffffffffu, mins, 1);
        if (live) {
            uint32_t *o = rec + size_t(i) * kRecWords;
            o[p] = uint32_t(mine);
            if (p == 0) {
                o[8] = uint32_t(mins);
                o[9] = DD == 4 ? *reinterpret_cast<const uint32_t *>(ddp + size_t(i) * 4)
                               : uint32_t(*reinterpret_cast<const uint16_t *>(ddp + size_t(i) * 2));
            }
            if (dbg) {
                int32_t *d = dbg + (size_t(w.row0 + r0 + i / C) * (w.kc * C) + sb) * 9;
                d[p] = mine;
                if (p == 0) d[8] = w.format == 13 ? mins : 0;
            }
        }
    }
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

// The row's super-blocks of one tile, in order (gemvq_ref.h:122-131, 170-175).
__device__ __forceinline__ void kq_fold(KqAcc &A, const uint32_t *rec, unsigned C, unsigned k, unsigned format,
                                        const XImage &X) {
    for (unsigned c = 0; c < C; ++c, rec += kRecWords) {
        const float dx = X.d[k * C + c];
        const float d = fmul(half_bits_to_float(uint16_t(rec[9] & 0xffffu)), dx);
#pragma unroll
        for (int l = 0; l < 8; ++l) A.sums[l] = fadd(A.sums[l], fmul(d, float(int32_t(rec[l]))));
        if (format == 13) {
            const float dmin = fmul(half_bits_to_float(uint16_t(rec[9] >> 16)), dx);
            A.sumf = fsub(A.sumf, fmul(dmin, float(int32_t(rec[8]))));
        }
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
    uint32_t *y5 = reinterpret_cast<uint32_t *>(P.extra);
    uint32_t *y6 = y5 + a.cols / 4;
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
    bool need5 = false, need6 = false;
    for (unsigned i = 0; i < a.n_members; ++i) {
        need5 |= a.m[i].w.format == 13;
        need6 |= a.m[i].w.format == 14;
    }
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
            compute_tile_kq(stage, M0.w, nr, it.k, X, y5, y6, rec, a.dbg, r0);
            if (pair >= 0)
                compute_tile_kq(stage + pair_offset(M0.w.tile_bytes), a.m[pair].w, nr, it.k, X, y5, y6,
                                rec + size_t(R) * C * kRecWords, nullptr, r0);
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
        if (!a.dbg) {
            const bool last = it.k + 1 == M0.w.kc;
            if (lane < nr) {
                kq_fold(A0, rec + size_t(lane) * C * kRecWords, C, it.k, M0.w.format, X);
                if (pair >= 0) kq_fold(A1, rec + size_t(R + lane) * C * kRecWords, C, it.k, a.m[pair].w.format, X);
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
        const unsigned rb = (pair ? 2u : 1u) * w.rt * w.ct * kRecWords * 4u;
        res = res > rb ? res : rb;
    }
    a.stage_bytes = (stage + 127u) & ~127u;
    a.res_bytes = (res + 127u) & ~127u;
    const bool norm_w = (a.norm_mode & 8u) && !(a.norm_mode & 2u) && !a.xq;
    a.wraw = norm_w && a.cols <= 4096 ? 1u : 0u;
    const size_t extra = size_t(a.cols) / 4 * 4 + size_t(a.cols) / 2 * 4;
    unsigned ns = kMaxStages;
    while (ns > 2 && pass_smem_bytes(ns, a.stage_bytes, a.res_bytes, a.cols, a.wraw, extra) > 113 * 1024) --ns;
    a.n_stages = ns;
    smem = pass_smem_bytes(ns, a.stage_bytes, a.res_bytes, a.cols, a.wraw, extra);
}

cudaError_t launch_gemv_kq(const GemvArgs &a, unsigned grid, size_t smem, cudaStream_t st, bool pdl) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(gemv_kq_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        cudaFuncSetAttribute(gemv_kq_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        attr_set = true;
    }
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
