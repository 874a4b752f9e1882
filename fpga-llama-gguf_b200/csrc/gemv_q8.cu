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

template <unsigned FMT>
__device__ __forceinline__ void compute_tile(const uint8_t *tile, const MatrixView &w, unsigned nr, unsigned k,
                                             const XImage &X, float *res, unsigned cs, int32_t *dbg, unsigned r0) {
    constexpr unsigned DB = FMT == 3 ? 4 : 2;
    const unsigned C = w.ct, items = nr * C;
    const uint8_t *qs = tile, *dm = tile + w.qs_part;
    unsigned r = threadIdx.x / C, c = threadIdx.x % C;
    const unsigned dr = kPassThreads / C, dc = kPassThreads % C;
    for (unsigned idx = threadIdx.x; idx < items; idx += kPassThreads) {
        const unsigned i = r * C + c, blk = k * C + c;
        const int4 x0 = *reinterpret_cast<const int4 *>(X.q + blk * 32);
        const int4 x1 = *reinterpret_cast<const int4 *>(X.q + blk * 32 + 16);
        int dot = 0;
        if (FMT == 8) {
            const int4 w0 = *reinterpret_cast<const int4 *>(qs + i * 32);
            const int4 w1 = *reinterpret_cast<const int4 *>(qs + i * 32 + 16);
            dot = __dp4a(w0.x, x0.x, dot);
            dot = __dp4a(w0.y, x0.y, dot);
            dot = __dp4a(w0.z, x0.z, dot);
            dot = __dp4a(w0.w, x0.w, dot);
            dot = __dp4a(w1.x, x1.x, dot);
            dot = __dp4a(w1.y, x1.y, dot);
            dot = __dp4a(w1.z, x1.z, dot);
            dot = __dp4a(w1.w, x1.w, dot);
        } else {
            // byte j: low nibble = element j, high nibble = element j + 16
            const uint4 wv = *reinterpret_cast<const uint4 *>(qs + i * 16);
            const uint32_t m = 0x0F0F0F0Fu;
            dot = __dp4a(int(wv.x & m), x0.x, dot);
            dot = __dp4a(int(wv.y & m), x0.y, dot);
            dot = __dp4a(int(wv.z & m), x0.z, dot);
            dot = __dp4a(int(wv.w & m), x0.w, dot);
            dot = __dp4a(int((wv.x >> 4) & m), x1.x, dot);
            dot = __dp4a(int((wv.y >> 4) & m), x1.y, dot);
            dot = __dp4a(int((wv.z >> 4) & m), x1.z, dot);
            dot = __dp4a(int((wv.w >> 4) & m), x1.w, dot);
        }
        int sumi = dot;
        if (FMT == 2) sumi -= 8 * X.b[blk];  // sum (w - 8) q = sum w q - 8 sum q
        float term;
        if (FMT == 3) {
            // (d_w * d_8) * sumi + m_w * s_8 (gemvq_ref.h:221-223)
            const uint32_t dmv = *reinterpret_cast<const uint32_t *>(dm + i * 4);
            const float dw = half_bits_to_float(uint16_t(dmv & 0xffffu)), mw = half_bits_to_float(uint16_t(dmv >> 16));
            term = fadd(fmul(fmul(dw, X.d[blk]), float(sumi)), fmul(mw, X.s[blk]));
        } else {
            const float dw = half_bits_to_float(*reinterpret_cast<const uint16_t *>(dm + i * DB));
            term = fmul(float(sumi), fmul(dw, X.d[blk]));
        }
        res[r * cs + c] = term;
        if (dbg) dbg[size_t(w.row0 + r0 + r) * (w.kc * C) + blk] = sumi;
        r += dr;
        c += dc;
        if (c >= C) { c -= C; ++r; }
    }
}

__device__ __forceinline__ void compute_tile_any(const uint8_t *tile, const MatrixView &w, unsigned nr, unsigned k,
                                                 const XImage &X, float *res, unsigned cs, int32_t *dbg, unsigned r0) {
    switch (w.format) {
    case 2: compute_tile<2>(tile, w, nr, k, X, res, cs, dbg, r0); break;
    case 8: compute_tile<8>(tile, w, nr, k, X, res, cs, dbg, r0); break;
    default: compute_tile<3>(tile, w, nr, k, X, res, cs, dbg, r0); break;
    }
}

// sum += term over one tile's C terms, in block order
__device__ __forceinline__ float fold_terms(float s, const float *row, unsigned C) {
    unsigned c = 0;
    for (; c + 4 <= C; c += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(row + c);
        s = fadd(s, v.x);
        s = fadd(s, v.y);
        s = fadd(s, v.z);
        s = fadd(s, v.w);
    }
    for (; c < C; ++c) s = fadd(s, row[c]);
    return s;
}

__global__ void __launch_bounds__(kPassThreads, 2) gemv_q8_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const PassSmem P = carve_pass(smem, a);
    const XImage X = carve_ximage(P.ximg, a.cols);
    const uint64_t policy = evict_first_policy();
    TileIt issue = tile_first(a);
    unsigned issued = pass_prologue(a, P, issue, policy);  // copies started (thread 0's count)
    pdl_launch_dependents();  // the next kernel may start its own weight copies as SMs free up
    pdl_wait();
    const unsigned act = a.m[0].w.format == 3 ? 1u : 0u;
    if (a.xq) load_quant_cta(a.xq, a.xd, a.xs, a.xb, a.cols, act, X);
    else quantize_cta(a.x, a.cols, act, a.norm_w, a.norm_eps, a.norm_mode, X);
    TileIt it = tile_first(a);
    float acc0 = 0.0f, acc1 = 0.0f;
    unsigned seq = 0;
    bool failed = false;
    while (tile_valid(a, it)) {
        const unsigned s = seq % a.n_stages;
        const bool ok = mbar_wait(&P.bar[s], (seq / a.n_stages) & 1u);
        const GemvMemberArgs &M0 = unit_member(a, it.unit);
        const int pair = a.unit_pair[it.unit];
        const unsigned t = it.item - a.item_start[it.unit];
        const unsigned R = M0.w.rt, C = M0.w.ct, cs = res_stride(C);
        const unsigned r0 = t * R, nr = min(R, M0.w.rows - r0);
        float *res = reinterpret_cast<float *>(P.res[seq & 1u]);
        const uint8_t *stage = P.stages + size_t(s) * a.stage_bytes;
        if (ok) {
            compute_tile_any(stage, M0.w, nr, it.k, X, res, cs, a.dbg, r0);
            if (pair >= 0)
                compute_tile_any(stage + pair_offset(M0.w.tile_bytes), a.m[pair].w, nr, it.k, X, res + R * cs, cs,
                                 nullptr, r0);
        }
        if (__syncthreads_or(!ok)) {
            failed = true;
            break;
        }
        // the stage is consumed: refill it with the tile n_stages positions ahead
        if (threadIdx.x == 0 && tile_valid(a, issue)) {
            issue_stage(a, issue, P.stages + size_t(s) * a.stage_bytes, &P.bar[s], policy);
            tile_next(a, issue);
            ++issued;
        }
        if (!a.dbg) {
            const bool last = it.k + 1 == M0.w.kc;
            if (threadIdx.x < nr) {
                acc0 = fold_terms(acc0, res + threadIdx.x * cs, C);
                if (pair >= 0) acc1 = fold_terms(acc1, res + (R + threadIdx.x) * cs, C);
                if (last) {
                    const unsigned gr = M0.w.row0 + r0 + threadIdx.x;
                    if (pair >= 0) write_row(a.m[pair], gr, acc1, acc0);
                    else write_row(M0, gr, acc0, 0.0f);
                    acc0 = acc1 = 0.0f;
                }
            }
            if (last && threadIdx.x >= 32 && threadIdx.x < 48)
                write_padding(pair >= 0 ? a.m[pair] : M0, M0.w.row0 + r0 + nr, threadIdx.x - 32);
        }
        ++seq;
        tile_next(a, it);
    }
    if (failed) {
        // a copy did not arrive in time: report, then wait (bounded) for the copies still in flight
        if (threadIdx.x == 0) {
            if (a.err) atomicExch(a.err, 1u);
            for (unsigned q = seq; q < issued; ++q) mbar_wait(&P.bar[q % a.n_stages], (q / a.n_stages) & 1u);
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kPassThreads) quantize_kernel(const QuantArgs a) {
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
// largest R x stride terms (x2 for a pair).
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
    const size_t xb = (ximage_bytes(a.cols) + 127) & ~size_t(127);
    // as many stages as fit two CTAs per SM (<= 113 KB each), at least 2, at most 4
    unsigned ns = 4;
    while (ns > 2 && pass_smem_bytes(ns, a.stage_bytes, a.res_bytes, xb) > 113 * 1024) --ns;
    a.n_stages = ns;
    smem = pass_smem_bytes(ns, a.stage_bytes, a.res_bytes, xb);
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
    quantize_kernel<<<1, kPassThreads, smem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace b200q
