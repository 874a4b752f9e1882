// Pieces shared by the two GEMV pass kernels (gemv_q8.cu, gemv_kq.cu): the walk over a CTA's weight tiles, the
// bulk-copy issue into the stage ring, and the result writer (epilogues of fpga/src/gemvqc16.cpp:203-316).
#pragma once
#include "kernel_args.h"
#include "pipeline.cuh"
#include "plan.h"
#include "quant.cuh"

namespace b200q {

constexpr unsigned kPassThreads = 256;

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

// Thread 0: bulk copies of one stage (the unit's tile, and for a pair the u tile of the same rows and columns).
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
// state shift (conv_chan, silu_f), else the row value.
__device__ __forceinline__ void write_row(const GemvMemberArgs &M, unsigned gr, float v, float g) {
    switch (M.epi) {
    case EpiSwigluU: M.y[gr] = fmul(silu_f32(g), v); break;
    case EpiAdd: M.y[gr] = fadd(v, M.res[gr]); break;
    case EpiConv: {
        const float s0 = M.cs[3 * gr], s1 = M.cs[3 * gr + 1], s2 = M.cs[3 * gr + 2];
        float sum = 0.0f;
        sum = fadd(sum, fmul(s0, M.cw[4 * gr]));
        sum = fadd(sum, fmul(s1, M.cw[4 * gr + 1]));
        sum = fadd(sum, fmul(s2, M.cw[4 * gr + 2]));
        sum = fadd(sum, fmul(v, M.cw[4 * gr + 3]));
        M.y[gr] = M.csilu ? silu_f32(sum) : sum;
        M.cd[3 * gr] = s1;
        M.cd[3 * gr + 1] = s2;
        M.cd[3 * gr + 2] = v;
        break;
    }
    default: M.y[gr] = v; break;
    }
}

// Zero padding of y up to a multiple of 16 rows (the reference writes y rounded up to 16 floats), by the CTA that
// writes the matrix's last row.
__device__ __forceinline__ void write_padding(const GemvMemberArgs &OUT, unsigned end_row, unsigned lane) {
    if (end_row == OUT.total_rows && OUT.epi != EpiConv && OUT.epi != EpiAdd) {
        const unsigned pad = round16(end_row) - end_row;
        if (lane < pad) OUT.y[end_row + lane] = 0.0f;
    }
}

// Shared memory of a pass: [mbarriers 64 B][stages][results x 2][x image]
struct PassSmem {
    uint64_t *bar;
    uint8_t *stages;
    uint8_t *res[2];
    unsigned char *ximg;
};

__host__ __device__ inline size_t pass_smem_bytes(unsigned n_stages, unsigned stage_bytes, unsigned res_bytes,
                                                  size_t extra) {
    return 64 + size_t(n_stages) * stage_bytes + 2 * size_t(res_bytes) + extra;
}

__device__ __forceinline__ PassSmem carve_pass(unsigned char *smem, const GemvArgs &a) {
    PassSmem P;
    P.bar = reinterpret_cast<uint64_t *>(smem);
    P.stages = smem + 64;
    P.res[0] = P.stages + size_t(a.n_stages) * a.stage_bytes;
    P.res[1] = P.res[0] + a.res_bytes;
    P.ximg = P.res[1] + a.res_bytes;
    return P;
}

// Thread 0: mbarrier init; then the first stages are issued (weights never change during a list, so this runs
// before the wait on the previous kernel).
__device__ __forceinline__ unsigned pass_prologue(const GemvArgs &a, const PassSmem &P, TileIt &issue,
                                                  uint64_t policy) {
    unsigned issued = 0;
    if (threadIdx.x == 0) {
        for (unsigned s = 0; s < a.n_stages; ++s) mbar_init(&P.bar[s], 1);
        mbar_fence_init();
        while (issued < a.n_stages && tile_valid(a, issue)) {
            issue_stage(a, issue, P.stages + size_t(issued) * a.stage_bytes, &P.bar[issued], policy);
            tile_next(a, issue);
            ++issued;
        }
    }
    __syncthreads();
    return issued;
}

}  // namespace b200q
