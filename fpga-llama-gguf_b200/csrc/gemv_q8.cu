// GEMV pass for the Q8_0-activation weight formats (Q4_0, Q8_0) and Q4_1 (Q8_1 activations): up to four GEMVs on
// one shared x in one launch, with the SwiGLU / residual ADD / causal CONV epilogues of the reference's result
// writer (fpga/src/gemvqc16.cpp:203-316).
//
// Per CTA (persistent over its row tiles):
//   1. thread 0 starts bulk copies of the first weight tiles into a ring of shared-memory stages — before the
//      wait on the previous kernel (programmatic dependent launch), since weights never change within a list;
//   2. after the wait, x is quantized into shared memory (optionally through the deferred RMSNORM);
//   3. per stage: every thread takes (row, block) items of the tile: an exact integer block dot with dp4a and
//      the block term float(sumi) * (d_w * d_x) (two IEEE roundings, as the CPU path); then one thread per row adds
//      the row's terms in block order into its running sum (sum += term), reproducing the CPU's FP32 sum bit for
//      bit (gemvq_ref.h:248-262); after the row's last tile it applies the epilogue and writes y.
//
// Roofline: HBM bandwidth. Bytes per row: cols/32 * (16 + 2) for Q4_0, * (32 + 2) for Q8_0, * (16 + 4) for Q4_1.
#include "gemv_common.cuh"
#include "launch.h"

namespace b200q {

__host__ __device__ inline unsigned res_stride(unsigned C) { return C + ((36u - C % 32u) % 32u); }

// One tile (R rows x C blocks, C a power of two <= 32) by the 8 compute warps: a warp instruction covers 32 / C
// rows x C blocks (lane = row sub-index * C + block), so a lane's x block (and its scale and sum) is loaded once per
// tile; the warp walks its row groups two at a time. Per item: exact integer block dot (dp4a), FP32 term
// float(sumi) * (d_w * d_x), stored to the result buffer (row stride cs).
template <unsigned FMT>
__device__ __forceinline__ void compute_tile(uint32_t s_tile, uint32_t qs_part, unsigned C, unsigned nr, unsigned kC,
                                             uint32_t s_xq, uint32_t s_xd, uint32_t s_xs, uint32_t s_xb,
                                             uint32_t s_res, unsigned cs, int32_t *dbg, size_t dbg_row0,
                                             unsigned nb) {
    constexpr unsigned QB = FMT == 8 ? 32 : 16;
    constexpr unsigned DB = FMT == 3 ? 4 : 2;
    const unsigned warp = threadIdx.x / 32 - 2, lane = threadIdx.x % 32;
    const unsigned c = lane & (C - 1), rsub = lane / C, rows_per_group = 32 / C;
    const unsigned groups = (nr + rows_per_group - 1) / rows_per_group;
    const unsigned blk = kC + c;
    const uint32_t s_dm = s_tile + qs_part;
    // this lane's x block, for all rows of the tile
    const uint4 x0 = lds128(s_xq + blk * 32), x1 = lds128(s_xq + blk * 32 + 16);
    const float xd = ldsf(s_xd + blk * 4);
    const int xcorr = FMT == 2 ? 8 * int(lds32(s_xb + blk * 4)) : 0;
    const float xs = FMT == 3 ? ldsf(s_xs + blk * 4) : 0.0f;
    auto item = [&](unsigned r) {
        const unsigned i = r * C + c;
        int d0 = 0, d1 = 0;
        if (FMT == 8) {
            const uint4 w0 = lds128(s_tile + i * QB), w1 = lds128(s_tile + i * QB + 16);
            d0 = __dp4a(int(w0.x), int(x0.x), d0);
            d1 = __dp4a(int(w1.x), int(x1.x), d1);
            d0 = __dp4a(int(w0.y), int(x0.y), d0);
            d1 = __dp4a(int(w1.y), int(x1.y), d1);
            d0 = __dp4a(int(w0.z), int(x0.z), d0);
            d1 = __dp4a(int(w1.z), int(x1.z), d1);
            d0 = __dp4a(int(w0.w), int(x0.w), d0);
            d1 = __dp4a(int(w1.w), int(x1.w), d1);
        } else {
            // byte j: low nibble = element j, high nibble = element j + 16
            const uint4 wv = lds128(s_tile + i * QB);
            const uint32_t m = 0x0F0F0F0Fu;
            d0 = __dp4a(int(wv.x & m), int(x0.x), d0);
            d1 = __dp4a(int((wv.x >> 4) & m), int(x1.x), d1);
            d0 = __dp4a(int(wv.y & m), int(x0.y), d0);
            d1 = __dp4a(int((wv.y >> 4) & m), int(x1.y), d1);
            d0 = __dp4a(int(wv.z & m), int(x0.z), d0);
            d1 = __dp4a(int((wv.z >> 4) & m), int(x1.z), d1);
            d0 = __dp4a(int(wv.w & m), int(x0.w), d0);
            d1 = __dp4a(int((wv.w >> 4) & m), int(x1.w), d1);
        }
        const int sumi = d0 + d1 - xcorr;  // Q4_0: sum (w - 8) q = sum w q - 8 sum q
        float term;
        if (FMT == 3) {
            // (d_w * d_8) * sumi + m_w * s_8 (gemvq_ref.h:221-223)
            const uint32_t dmv = lds32(s_dm + i * 4);
            const float dw = half_bits_to_float(uint16_t(dmv & 0xffffu)), mw = half_bits_to_float(uint16_t(dmv >> 16));
            term = fadd(fmul(fmul(dw, xd), float(sumi)), fmul(mw, xs));
        } else {
            const float dw = half_bits_to_float(lds16(s_dm + i * DB));
            term = fmul(float(sumi), fmul(dw, xd));
        }
        stsf(s_res + (r * cs + c) * 4, term);
        if (dbg) dbg[(dbg_row0 + r) * nb + blk] = sumi;
    };
    unsigned g = warp;
    for (; g + kComputeWarps < groups; g += 2 * kComputeWarps) {
        const unsigned ra = g * rows_per_group + rsub, rb = (g + kComputeWarps) * rows_per_group + rsub;
        if (ra < nr) item(ra);
        if (rb < nr) item(rb);
    }
    if (g < groups) {
        const unsigned ra = g * rows_per_group + rsub;
        if (ra < nr) item(ra);
    }
}

__device__ __forceinline__ void compute_tile_any(const uint8_t *tile, const MatrixView &w, unsigned nr, unsigned k,
                                                 const XImage &X, float *res, unsigned cs, int32_t *dbg, unsigned r0) {
    const uint32_t st = smem_addr(tile), sq = smem_addr(X.q), sd = smem_addr(X.d), ss = smem_addr(X.s);
    const uint32_t sb = smem_addr(X.b), sr = smem_addr(res);
    const unsigned C = w.ct, nb = w.kc * w.ct;
    const size_t drow = size_t(w.row0) + r0;
    switch (w.format) {
    case 2: compute_tile<2>(st, w.qs_part, C, nr, k * C, sq, sd, ss, sb, sr, cs, dbg, drow, nb); break;
    case 8: compute_tile<8>(st, w.qs_part, C, nr, k * C, sq, sd, ss, sb, sr, cs, dbg, drow, nb); break;
    default: compute_tile<3>(st, w.qs_part, C, nr, k * C, sq, sd, ss, sb, sr, cs, dbg, drow, nb); break;
    }
}

// sum += term over one tile's C terms, in block order (row at shared address a, 16-byte aligned)
__device__ __forceinline__ float fold_terms(float s, uint32_t a, unsigned C) {
    unsigned c = 0;
    for (; c + 4 <= C; c += 4) {
        const uint4 v = lds128(a + c * 4);
        s = fadd(s, __uint_as_float(v.x));
        s = fadd(s, __uint_as_float(v.y));
        s = fadd(s, __uint_as_float(v.z));
        s = fadd(s, __uint_as_float(v.w));
    }
    for (; c < C; ++c) s = fadd(s, ldsf(a + c * 4));
    return s;
}

__global__ void __launch_bounds__(kPassThreads, 2) gemv_q8_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const PassSmem P = carve_pass(smem, a);
    const XImage X = carve_ximage(P.ximg, a.cols);
    const unsigned warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) init_pass_barriers(a, P);
    __syncthreads();
    pdl_launch_dependents();  // the next kernel may start its own weight copies as SMs free up
    if (warp == 0) {
        if (lane == 0) producer_loop(a, P);
        return;
    }
    pdl_wait();
    prepare_x(a, P, X, a.m[0].w.format == 3 ? 1u : 0u);
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
            const unsigned R = M0.w.rt, cs = res_stride(M0.w.ct);
            const unsigned r0 = t * R, nr = min(R, M0.w.rows - r0);
            float *res = reinterpret_cast<float *>((b ? P.res[1] : P.res[0]));
            const uint8_t *stage = P.stages + size_t(s) * a.stage_bytes;
            compute_tile_any(stage, M0.w, nr, it.k, X, res, cs, a.dbg, r0);
            if (pair >= 0)
                compute_tile_any(stage + pair_offset(M0.w.tile_bytes), a.m[pair].w, nr, it.k, X, res + R * cs, cs,
                                 nullptr, r0);
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
    // fold (warp 1): lane r adds row r's terms in block order
    float acc0 = 0.0f, acc1 = 0.0f;
    while (tile_valid(a, it)) {
        const unsigned b = seq % kNR;
        if (!role_wait(&P.rfull[b], (seq / kNR) & 1u, P.abort)) {
            fail_pass(a, P.abort);
            break;
        }
        const GemvMemberArgs &M0 = unit_member(a, it.unit);
        const int pair = a.unit_pair[it.unit];
        const unsigned t = it.item - a.item_start[it.unit];
        const unsigned R = M0.w.rt, C = M0.w.ct, cs = res_stride(C);
        const unsigned r0 = t * R, nr = min(R, M0.w.rows - r0);
        const uint32_t res = smem_addr((b ? P.res[1] : P.res[0]));
        if (!a.dbg) {
            const bool last = it.k + 1 == M0.w.kc;
            if (lane < nr) {
                acc0 = fold_terms(acc0, res + lane * cs * 4, C);
                if (pair >= 0) acc1 = fold_terms(acc1, res + (R + lane) * cs * 4, C);
                if (last) {
                    const unsigned gr = M0.w.row0 + r0 + lane;
                    if (pair >= 0) write_row(a.m[pair], gr, acc1, acc0);
                    else write_row(M0, gr, acc0, 0.0f);
                    acc0 = acc1 = 0.0f;
                }
            }
            if (last) write_padding(pair >= 0 ? a.m[pair] : M0, M0.w.row0 + r0 + nr, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&P.rempty[b]);
        ++seq;
        tile_next(a, it);
    }
}

__global__ void __launch_bounds__(256) quantize_kernel(const QuantArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const XImage X = carve_ximage(smem, a.n);
    pdl_wait();
    quantize_cta(a.x, a.n, a.act, a.norm_w, a.norm_eps, a.norm_mode, X);
    for (unsigned i = threadIdx.x; i < a.n / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(a.q)[i] = reinterpret_cast<const uint4 *>(X.q)[i];
    const unsigned nd = a.act == 2 ? a.n / 256 : a.n / 32, nbs = a.act == 2 ? a.n / 16 : a.n / 32;
    for (unsigned i = threadIdx.x; i < nd; i += blockDim.x) {
        a.d[i] = X.d[i];
        if (a.act == 1 && a.s) a.s[i] = X.s[i];
        if (a.d16) {
            if (a.act == 0) {
                a.d16[i] = float_to_half_bits(X.d[i]);
            } else if (a.act == 1) {
                a.d16[2 * i] = float_to_half_bits(X.d[i]);
                a.d16[2 * i + 1] = float_to_half_bits(X.s[i]);
            }
        }
    }
    for (unsigned i = threadIdx.x; i < nbs; i += blockDim.x) a.b[i] = X.b[i];
}

// Shared memory plan of a Q8 pass (see PassSmem): stage = the largest unit tile (x2 for a pair), results = the
// largest R x stride terms (x2 for a pair); as many stages as fit two CTAs per SM.
void plan_gemv_q8(GemvArgs &a, size_t &smem) {
    unsigned stage = 0, res = 0;
    for (unsigned u = 0; u < a.n_units; ++u) {
        const MatrixView &w = a.m[a.unit_member[u]].w;
        const bool pair = a.unit_pair[u] >= 0;
        const unsigned sb = pair ? pair_offset(w.tile_bytes) + w.tile_bytes : w.tile_bytes;
        stage = stage > sb ? stage : sb;
        const unsigned rb = (pair ? 2u : 1u) * w.rt * res_stride(w.ct) * 4u;
        res = res > rb ? res : rb;
    }
    a.stage_bytes = (stage + 127u) & ~127u;
    a.res_bytes = (res + 127u) & ~127u;
    const bool norm_w = (a.norm_mode & 8u) && !(a.norm_mode & 2u) && !a.xq;
    a.wraw = norm_w && a.cols <= 4096 ? 1u : 0u;
    unsigned ns = kMaxStages;
    while (ns > 2 && pass_smem_bytes(ns, a.stage_bytes, a.res_bytes, a.cols, a.wraw, 0) > 113 * 1024) --ns;
    a.n_stages = ns;
    smem = pass_smem_bytes(ns, a.stage_bytes, a.res_bytes, a.cols, a.wraw, 0);
}

cudaError_t launch_gemv_q8(const GemvArgs &a, unsigned grid, size_t smem, cudaStream_t st, bool pdl) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(gemv_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
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
    return cudaLaunchKernelEx(&cfg, gemv_q8_kernel, a);
}

cudaError_t launch_quantize(const QuantArgs &a, cudaStream_t st) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(quantize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        attr_set = true;
    }
    const size_t smem = (ximage_bytes(a.n) + 127) & ~size_t(127);
    quantize_kernel<<<1, 256, smem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace b200q
