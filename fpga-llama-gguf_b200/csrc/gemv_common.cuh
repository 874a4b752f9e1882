// Warp-specialized pass framework shared by the two GEMV kernels (gemv_q8.cu, gemv_kq.cu).
//
// A CTA (two per SM) walks its weight tiles (row tiles of the pass's units, round-robin over the grid; each row
// tile streamed as kc tiles of R rows x C blocks) with three roles:
//   warp 0    producer: bulk copies (cp.async.bulk) of tiles into a ring of n_stages shared-memory stages; the
//             first stages start before the wait on the previous kernel (weights never change within a list);
//   warps 2-9 compute: per tile, the exact integer block dots and the FP32 block terms, into a result buffer;
//   warp 1    fold: per row (lane), the row's block terms added in block order — the CPU's FP32 sum, bit for bit —
//             and after the row's last tile the epilogue (SwiGLU / residual add / conv1d) and the store of y.
// Hand-offs go through mbarriers (full/empty per stage, rfull/rempty per result buffer), so the copies, the integer
// work and the sequential fold of different tiles overlap. Every wait is bounded; a wait that runs out sets the
// CTA's abort flag and the pass's error word, and all roles leave (the producer first waits, bounded, for the
// copies it started).
#pragma once
#include "kernel_args.h"
#include "peer.cuh"
#include "pipeline.cuh"
#include "plan.h"
#include "quant.cuh"

namespace b200q {

constexpr unsigned kComputeWarps = 8;
constexpr unsigned kPassThreads = 32 * (2 + kComputeWarps);  // producer + fold + compute
constexpr unsigned kComputeThreads = 32 * kComputeWarps;
constexpr unsigned kXThreads = kPassThreads - 32;              // fold + compute warps prepare x
constexpr unsigned kNR = 2;                                     // result buffers
constexpr unsigned kMaxStages = 6;
constexpr unsigned kL2Ahead = 2;                                // tiles asked of L2 beyond the stage ring

// Position in the tile sequence of one CTA: items (row tiles of units) blockIdx.x, blockIdx.x + gridDim.x, ...;
// each item is streamed as its unit's kc tiles.
struct TileIt {
    unsigned item, k, unit;
};

__device__ __forceinline__ unsigned unit_of(const GemvArgs &a, unsigned item) {
    unsigned u = 0;
    while (u + 1 < a.n_units && item >= a.item_start[u + 1]) ++u;
    return u;
}

__device__ __forceinline__ const GemvMemberArgs &unit_member(const GemvArgs &a, unsigned u) {
    return a.m[a.unit_member[u]];
}

__device__ __forceinline__ TileIt tile_first(const GemvArgs &a) {
    TileIt it{blockIdx.x, 0, 0};
    if (it.item < a.item_start[a.n_units]) it.unit = unit_of(a, it.item);
    return it;
}

__device__ __forceinline__ bool tile_valid(const GemvArgs &a, const TileIt &it) {
    return it.item < a.item_start[a.n_units];
}

__device__ __forceinline__ void tile_next(const GemvArgs &a, TileIt &it) {
    if (++it.k == unit_member(a, it.unit).w.kc) {
        it.k = 0;
        it.item += gridDim.x;
        if (it.item < a.item_start[a.n_units]) it.unit = unit_of(a, it.item);
    }
}

__device__ __forceinline__ const uint8_t *tile_src(const MatrixView &w, unsigned t, unsigned k) {
    return w.base + (size_t(t) * w.kc + k) * w.tile_bytes;
}

// Pair tile offset inside a stage.
__host__ __device__ inline unsigned pair_offset(unsigned tile_bytes) { return (tile_bytes + 127u) & ~127u; }

// Bulk copies of one stage (the unit's tile, and for a pair the u tile of the same rows and columns).
__device__ __forceinline__ void issue_stage(const GemvArgs &a, const TileIt &it, uint8_t *stage, uint64_t *bar,
                                            uint64_t policy) {
    const GemvMemberArgs &M = unit_member(a, it.unit);
    const unsigned t = it.item - a.item_start[it.unit];
    const int pair = a.unit_pair[it.unit];
    const unsigned bytes = M.w.tile_bytes;
    mbar_expect_tx(bar, pair >= 0 ? 2 * bytes : bytes);
    bulk_copy(stage, tile_src(M.w, t, it.k), bytes, bar, policy);
    if (pair >= 0) bulk_copy(stage + pair_offset(bytes), tile_src(a.m[pair].w, t, it.k), bytes, bar, policy);
}

// Result writer for one output row: SwiGLU silu(g) * u (silu_mul_f), residual add (add_mul_f), conv1d + SiLU +
// state shift (conv_chan, silu_f), else the row value (fpga/src/gemvqc16.cpp:203-316).
// The value the writer stores for row gr (every epilogue but CONV).
__device__ __forceinline__ float row_value(const GemvMemberArgs &M, unsigned gr, float v, float g,
                                           const float *res_pre = nullptr) {
    switch (M.epi) {
    case EpiSwigluU: return fmul(silu_f32(g), v);
    case EpiAdd: return fadd(v, res_pre ? *res_pre : M.res[gr]);
    default: return v;
    }
}

// ps (multi-GPU): the rows of a sharded member (its local rows are fewer than its total rows) also go to the peers.
__device__ __forceinline__ void write_row(const GemvMemberArgs &M, unsigned gr, float v, float g,
                                          const float *res_pre = nullptr, const PeerSync *ps = nullptr) {
    const PeerSync *pp = (ps && M.w.rows != M.total_rows) ? ps : nullptr;
    switch (M.epi) {
    case EpiSwigluU: peer_store(pp, M.y + gr, row_value(M, gr, v, g)); break;
    case EpiAdd: peer_store(pp, M.y + gr, row_value(M, gr, v, g, res_pre)); break;
    case EpiConv: {
        const float s0 = M.cs[3 * gr], s1 = M.cs[3 * gr + 1], s2 = M.cs[3 * gr + 2];
        float sum = 0.0f;
        sum = fadd(sum, fmul(s0, M.cw[4 * gr]));
        sum = fadd(sum, fmul(s1, M.cw[4 * gr + 1]));
        sum = fadd(sum, fmul(s2, M.cw[4 * gr + 2]));
        sum = fadd(sum, fmul(v, M.cw[4 * gr + 3]));
        peer_store(pp, M.y + gr, M.csilu ? silu_f32(sum) : sum);
        peer_store(pp, M.cd + 3 * gr, s1);
        peer_store(pp, M.cd + 3 * gr + 1, s2);
        peer_store(pp, M.cd + 3 * gr + 2, v);
        break;
    }
    default: peer_store(pp, M.y + gr, v); break;
    }
}

// Zero padding of y up to a multiple of 16 rows (the reference writes y rounded up to 16 floats), by the CTA that
// writes the matrix's last row.
__device__ __forceinline__ void write_padding(const GemvMemberArgs &OUT, unsigned end_row, unsigned lane,
                                              const PeerSync *ps = nullptr) {
    if (end_row == OUT.total_rows && OUT.epi != EpiConv && OUT.epi != EpiAdd) {
        const unsigned pad = round16(end_row) - end_row;
        const PeerSync *pp = (ps && OUT.w.rows != OUT.total_rows) ? ps : nullptr;
        if (lane < pad) peer_store(pp, OUT.y + end_row + lane, 0.0f);
    }
}

// ---- shared memory of a pass ------------------------------------------------------------------------------------
// [256 B: full[NS] empty[NS] rfull[2] rempty[2] abort go][stages][results x 2][x image][raw x][raw norm weight][extra]
constexpr unsigned kBarRegion = 256;
static_assert((2 * kMaxStages + 2 * kNR) * 8 + 12 <= kBarRegion, "barriers and the flags fit their region");
struct PassSmem {
    uint64_t *full, *empty, *rfull, *rempty;
    unsigned *abort;
    unsigned *go;  // the lead compute warp's verdicts for the other compute warps (two, alternating)
    uint8_t *stages;
    uint8_t *res[kNR];
    unsigned char *ximg;
    float *xraw, *wraw;
    unsigned char *extra;
};

__host__ __device__ inline size_t align128(size_t v) { return (v + 127) & ~size_t(127); }

__host__ __device__ inline size_t pass_smem_bytes(unsigned n_stages, unsigned stage_bytes, unsigned res_bytes,
                                                  unsigned cols, bool wraw, size_t extra) {
    return kBarRegion + size_t(n_stages) * stage_bytes + kNR * size_t(res_bytes) + align128(ximage_bytes(cols)) +
           align128(size_t(cols) * 4) + (wraw ? align128(size_t(cols) * 4) : 0) + extra;
}

__device__ __forceinline__ PassSmem carve_pass(unsigned char *smem, const GemvArgs &a) {
    PassSmem P;
    uint64_t *b = reinterpret_cast<uint64_t *>(smem);
    P.full = b;
    P.empty = b + a.n_stages;
    P.rfull = b + 2 * a.n_stages;
    P.rempty = P.rfull + kNR;
    P.abort = reinterpret_cast<unsigned *>(P.rempty + kNR);
    P.go = P.abort + 1;
    unsigned char *p = smem + kBarRegion;
    P.stages = p;
    p += size_t(a.n_stages) * a.stage_bytes;
    for (unsigned i = 0; i < kNR; ++i) {
        P.res[i] = p;
        p += a.res_bytes;
    }
    P.ximg = p;
    p += align128(ximage_bytes(a.cols));
    P.xraw = reinterpret_cast<float *>(p);
    p += align128(size_t(a.cols) * 4);
    P.wraw = nullptr;
    if (a.wraw) {
        P.wraw = reinterpret_cast<float *>(p);
        p += align128(size_t(a.cols) * 4);
    }
    P.extra = p;
    return P;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// A bounded wait that also gives up once another role set the abort flag.
__device__ __forceinline__ bool role_wait(uint64_t *bar, unsigned parity, volatile unsigned *abort) {
    const uint32_t a = smem_addr(bar);
    unsigned long long start = 0;
    for (unsigned i = 0;; ++i) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(a), "r"(parity), "r"(kSuspendHintNs)
            : "memory");
        if (done) return true;
        if ((i & 1023u) == 0) {
            if (*abort) return false;
            const unsigned long long now = global_ns();
            if (start == 0) start = now;
            else if (now - start > kWaitLimitNs) return false;
        }
    }
}

__device__ __forceinline__ void fail_pass(const GemvArgs &a, volatile unsigned *abort) {
    *abort = 1u;
    if (a.err) atomicExch(a.err, 1u);
}

// Thread 0: barrier init (full: the producer's arrival + bytes; empty / rfull: one arrival per compute warp;
// rempty: the fold warp).
__device__ __forceinline__ void init_pass_barriers(const GemvArgs &a, const PassSmem &P) {
    for (unsigned s = 0; s < a.n_stages; ++s) {
        mbar_init(&P.full[s], 1);
        mbar_init(&P.empty[s], kComputeWarps);
    }
    for (unsigned b = 0; b < kNR; ++b) {
        mbar_init(&P.rfull[b], kComputeWarps);
        mbar_init(&P.rempty[b], 1);
    }
    *P.abort = 0u;
    mbar_fence_init();
}

// L2 prefetch of the bytes issue_stage copies for one tile (no data returns to the SM).
__device__ __forceinline__ void prefetch_stage(const GemvArgs &a, const TileIt &it) {
    const GemvMemberArgs &M = unit_member(a, it.unit);
    const unsigned t = it.item - a.item_start[it.unit];
    const int pair = a.unit_pair[it.unit];
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(tile_src(M.w, t, it.k)), "r"(M.w.tile_bytes)
                 : "memory");
    if (pair >= 0)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(tile_src(a.m[pair].w, t, it.k)),
                     "r"(M.w.tile_bytes)
                     : "memory");
}

// Producer (one thread): streams the CTA's tiles through the stage ring. The kL2Ahead tiles after the ring's are
// asked of L2 ahead of their copies, so HBM keeps streaming while every stage waits for its compute.
__device__ __forceinline__ void producer_loop(const GemvArgs &a, const PassSmem &P) {
    const uint64_t policy = evict_first_policy();
    TileIt it = tile_first(a), pf = it;
    for (unsigned i = 0; i < a.n_stages && tile_valid(a, pf); ++i) tile_next(a, pf);
    for (unsigned i = 0; i < kL2Ahead && tile_valid(a, pf); ++i) {
        prefetch_stage(a, pf);
        tile_next(a, pf);
    }
    unsigned seq = 0;
    bool failed = false;
    while (tile_valid(a, it)) {
        const unsigned s = seq % a.n_stages;
        if (seq >= a.n_stages && !role_wait(&P.empty[s], ((seq / a.n_stages) - 1u) & 1u, P.abort)) {
            failed = true;
            break;
        }
        issue_stage(a, it, P.stages + size_t(s) * a.stage_bytes, &P.full[s], policy);
        if (seq >= a.n_stages && tile_valid(a, pf)) {
            prefetch_stage(a, pf);
            tile_next(a, pf);
        }
        tile_next(a, it);
        ++seq;
    }
    if (failed) {
        fail_pass(a, P.abort);
        // the last issued copy of every stage: wait (bounded) until it has landed before the CTA may exit
        const unsigned from = seq > a.n_stages ? seq - a.n_stages : 0u;
        for (unsigned q = from; q < seq; ++q) mbar_wait(&P.full[q % a.n_stages], (q / a.n_stages) & 1u);
    }
}

__device__ __forceinline__ void named_sync_x() { asm volatile("bar.sync 1, %0;" ::"n"(kXThreads) : "memory"); }
// The 8 compute warps: the lead warp waits on the mbarriers, the others sleep on this hardware barrier.
__device__ __forceinline__ void named_sync_compute() {
    asm volatile("bar.sync 2, %0;" ::"n"(kComputeThreads) : "memory");
}

// Compute warps: wait until stage s holds the tile and result buffer b is free. The lead warp polls; the others
// sleep on the named barrier, then take their own (already complete, so non-blocking) acquire of the stage.
// The verdict alternates between two flags, so the lead never overwrites one another warp has not read yet.
// False (for every compute warp) if a wait gave up.
__device__ __forceinline__ bool compute_acquire(const PassSmem &P, unsigned seq, unsigned n_stages) {
    const unsigned warp = threadIdx.x / 32, s = seq % n_stages, b = seq % kNR;
    volatile unsigned *flag = P.go + (seq & 1u);
    if (warp == 2) {
        bool ok = role_wait(&P.full[s], (seq / n_stages) & 1u, P.abort);
        if (ok && seq >= kNR) ok = role_wait(&P.rempty[b], ((seq / kNR) - 1u) & 1u, P.abort);
        if (threadIdx.x == 64) *flag = ok ? 1u : 0u;
    }
    named_sync_compute();
    const bool ok = *flag != 0u;
    if (ok && warp != 2) role_wait(&P.full[s], (seq / n_stages) & 1u, P.abort);
    return ok;
}

template <unsigned NT>
__device__ __forceinline__ void x_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }

// Index of element e (0..31) of 32-block b in the x image: contiguous 32-byte blocks, or (split) the first 16
// bytes of every block in one run and the second 16 bytes in another, so that lanes reading consecutive blocks'
// 16-byte halves hit consecutive banks.
template <bool SPLIT>
__device__ __forceinline__ unsigned xq_index(unsigned b, unsigned e, unsigned n) {
    return SPLIT ? (e / 16) * (n / 2) + b * 16 + (e & 15) : b * 32 + e;
}

// x into shared memory (coalesced), then quantized by warps: NT threads from thread OFF on, barrier 1 among them.
template <unsigned NT, unsigned OFF, bool SPLIT>
__device__ __forceinline__ void prepare_x_t(const GemvArgs &a, float *xraw, float *wraw_buf, const XImage &X,
                                            unsigned act) {
    const unsigned t = threadIdx.x - OFF, warp = t / 32, lane = t % 32, nw = NT / 32;
    const unsigned n = a.cols;
    if (a.xq) {
        for (unsigned i = t; i < n / 16; i += NT) {
            const unsigned dst = SPLIT ? (i & 1u) * (n / 32) + i / 2 : i;
            reinterpret_cast<uint4 *>(X.q)[dst] = reinterpret_cast<const uint4 *>(a.xq)[i];
        }
        const unsigned nd = act == 2 ? n / 256 : n / 32, nb = act == 2 ? n / 16 : n / 32;
        for (unsigned i = t; i < nd; i += NT) {
            X.d[i] = a.xd[i];
            if (act == 1) X.s[i] = a.xs[i];
        }
        for (unsigned i = t; i < nb; i += NT) X.b[i] = a.xb[i];
        x_sync<NT>();
        return;
    }
    const bool norm = (a.norm_mode & 8u) != 0, weighted = (a.norm_mode & 2u) == 0;
    const float4 *x4 = reinterpret_cast<const float4 *>(a.x);
    float4 *xr4 = reinterpret_cast<float4 *>(xraw);
    double acc = 0.0;
    for (unsigned i = t; i < n / 4; i += NT) {
        const float4 v = x4[i];
        xr4[i] = v;
        if (norm) {
            acc += double(fmul(v.x, v.x));
            acc += double(fmul(v.y, v.y));
            acc += double(fmul(v.z, v.z));
            acc += double(fmul(v.w, v.w));
        }
    }
    float *wraw = (norm && weighted) ? wraw_buf : nullptr;
    if (wraw) {
        const float4 *w4 = reinterpret_cast<const float4 *>(a.norm_w);
        for (unsigned i = t; i < n / 4; i += NT) reinterpret_cast<float4 *>(wraw)[i] = w4[i];
    }
    float scale = 1.0f;
    if (norm) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) X.red[warp] = acc;
        x_sync<NT>();
        if (t == 0) {
            double sum = 0.0;
            for (unsigned w = 0; w < nw; ++w) sum += X.red[w];
            float sc;
            if (a.norm_mode & 1u) sc = fdiv(1.0f, fmaxf(__fsqrt_rn(__double2float_rn(sum)), a.norm_eps));
            else sc = fdiv(1.0f, __fsqrt_rn(fadd(__double2float_rn(__ddiv_rn(sum, double(n))), a.norm_eps)));
            *X.scale = sc;
        }
    }
    x_sync<NT>();
    if (norm) scale = *X.scale;
    const float *wn = wraw ? wraw : a.norm_w;
    if (act == 2) {
        for (unsigned sb = warp; sb < n / 256; sb += nw) {
            float v[8];
            float amax = 0.0f, mx = 0.0f;
            int idx = 0x7fffffff;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const unsigned e = sb * 256 + lane + 32 * k;
                v[k] = norm_value(xraw, e, norm, scale, wn, weighted);
                const float av = fabsf(v[k]);
                if (av > amax) { amax = av; mx = v[k]; idx = int(lane + 32 * k); }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {  // largest magnitude, first index on ties (gemvq_ref.h:68-75)
                const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
                const float om = __shfl_xor_sync(0xffffffffu, mx, o);
                const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
                if (oa > amax || (oa == amax && oi < idx)) { amax = oa; mx = om; idx = oi; }
            }
            const float iscale = amax != 0.0f ? fdiv(-127.0f, mx) : 0.0f;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                int q = 0;
                if (amax != 0.0f) {
                    q = __float2int_rn(fmul(iscale, v[k]));
                    q = q < 127 ? q : 127;
                }
                X.q[sb * 256 + lane + 32 * k] = int8_t(q);
                int part = q;  // sums of 16: lanes 0..15 -> group 2k, lanes 16..31 -> group 2k + 1
                part += __shfl_xor_sync(0xffffffffu, part, 8);
                part += __shfl_xor_sync(0xffffffffu, part, 4);
                part += __shfl_xor_sync(0xffffffffu, part, 2);
                part += __shfl_xor_sync(0xffffffffu, part, 1);
                if (lane == 0) X.b[sb * 16 + 2 * k] = part;
                if (lane == 16) X.b[sb * 16 + 2 * k + 1] = part;
            }
            if (lane == 0) X.d[sb] = amax != 0.0f ? fdiv(1.0f, iscale) : 0.0f;
        }
    } else {
        // four lanes per 32-block, eight elements each: lane j of the quad of block b takes the elements
        // (8j + e + b) % 32, e < 8, so the 32 lanes of a warp (8 blocks) read 32 different banks; amax and the sum
        // over the quad by shuffles. The loop runs warp-uniformly (whole warps per round).
        const unsigned nq = n / 32 * 4;
        for (unsigned wbase = t & ~31u; wbase < nq; wbase += NT) {
            const unsigned item = wbase + (t & 31u), b = item / 4, j = item & 3u;
            const bool live = item < nq;
            float v[8];
            float amax = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const unsigned off = (8u * j + unsigned(e) + b) & 31u;
                v[e] = live ? norm_value(xraw, b * 32 + off, norm, scale, wn, weighted) : 0.0f;
                amax = fmaxf(amax, fabsf(v[e]));
            }
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            const float s = fdiv(amax, 127.0f);
            const float id = s != 0.0f ? fdiv(1.0f, s) : 0.0f;
            int sum = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int q = int(roundf(fmul(v[e], id)));
                sum += q;
                const unsigned off = (8u * j + unsigned(e) + b) & 31u;
                if (live) X.q[xq_index<SPLIT>(b, off, n)] = int8_t(q);
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            if (live && j == 0) {
                X.d[b] = half_bits_to_float(float_to_half_bits(s));
                X.b[b] = sum;
                if (act == 1) X.s[b] = half_bits_to_float(float_to_half_bits(fmul(float(sum), s)));
            }
        }
    }
    x_sync<NT>();
}


// The K-quant pass: fold + compute warps (threads 32..319) prepare x.
__device__ __forceinline__ void prepare_x(const GemvArgs &a, const PassSmem &P, const XImage &X, unsigned act) {
    prepare_x_t<kXThreads, 32, false>(a, P.xraw, P.wraw, X, act);
}

}  // namespace b200q
