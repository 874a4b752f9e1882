// GEMV pass for the Q8_0-activation weight formats (Q4_0, Q8_0) and Q4_1 (Q8_1 activations): up to four GEMVs on
// one shared x in one launch, with the SwiGLU / residual ADD / causal CONV epilogues of the reference's result
// writer (fpga/src/gemvqc16.cpp:203-316).
//
// A CTA takes one panel at a time (P rows x all blocks of one matrix, or of a SwiGLU g/u pair; one wave of CTAs
// covers the pass when it fits) and splits the panel's steps over its 8 warps (warp w: steps w, w + 8, ...):
//   1. before the wait on the previous kernel (programmatic dependent launch) the CTA bulk-copies the leading steps
//      of its first panel into shared memory and asks L2 for the rest of it (weights never change within a list),
//      so HBM streams while the previous kernel ends and while x is prepared;
//   2. the CTA quantizes x into shared memory once (optionally through the deferred RMSNORM);
//   3. per step (one 32-unit tile: P rows x 32 / P blocks, lane = unit) each lane loads its unit's 16-byte quant
//      words and scale with coalesced 128-bit loads, several steps ahead in registers, forms the exact integer
//      block dot (dp4a) and the block term float(sumi) * (d_w * d_x) (two IEEE roundings, as the CPU path), and
//      stores the term to the panel's term buffer in shared memory (row-major: a row's terms contiguous);
//   4. after the panel, one lane per row adds the row's terms in block order, reproducing the CPU's FP32 sum bit
//      for bit (gemvq_ref.h:248-262), applies the epilogue and writes y.
//
// Roofline: HBM bandwidth. Bytes per row: cols/32 * (16 + 2) for Q4_0, * (32 + 2) for Q8_0, * (16 + 4) for Q4_1.
#include <algorithm>

#include "gemv_common.cuh"
#include "launch.h"

namespace b200q {

constexpr unsigned kPanelWarps = 8, kPanelThreads = 32 * kPanelWarps;

// Term buffer of a panel: row i's block terms contiguous at word i * term_stride(blocks), blocks = the row's units over
// all steps (zero padding included). The stride is a multiple of 4 with stride / 4 odd, so the 16-byte loads of 8
// consecutive rows hit 8 distinct bank groups (and a P = 8 step's 32 stores hit 32 banks).
__host__ __device__ inline unsigned term_stride(unsigned blocks) {
    const unsigned s = (blocks + 3u) & ~3u;
    return (s / 4u) % 2u ? s : s + 4u;
}

// ---- one lane's share of one step ---------------------------------------------------------------------------------
template <unsigned FMT>
struct Step {
    uint4 q0, q1;  // quant words (q1: Q8_0 only)
    uint32_t d;    // FP16 d (Q4_1: d | m << 16)
};

__device__ __forceinline__ uint4 ldw128(const uint8_t *p, uint64_t pol) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ uint32_t ldw32(const uint8_t *p, uint64_t pol) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ uint32_t ldw16(const uint8_t *p, uint64_t pol) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u16 %0, [%1], %2;" : "=h"(v) : "l"(p), "l"(pol));
    return v;
}

// Step tile layout (layout.h): quants at lane * 16 (Q8_0: + 512 for the second half), scales at 512 (Q8_0: 1024).
template <unsigned FMT>
__device__ __forceinline__ void load_step(Step<FMT> &v, const uint8_t *tile, unsigned lane, uint64_t pol) {
    v.q0 = ldw128(tile + lane * 16, pol);
    if (FMT == 8) {
        v.q1 = ldw128(tile + 512 + lane * 16, pol);
        v.d = ldw16(tile + 1024 + lane * 2, pol);
    } else if (FMT == 2) {
        v.d = ldw16(tile + 512 + lane * 2, pol);
    } else {
        v.d = ldw32(tile + 512 + lane * 4, pol);
    }
}

// x block of a lane: the split image (first 16 quant bytes of block b at q0 + 16 b, the second 16 at q1 + 16 b)
// and the block's meta word {d, s (Q8_1), sum of q, 0} at meta + 16 b.
struct XBlock {
    uint4 q0, q1;
    float d, s;
    int bsum;
};

// ---- the RMSNORM scale of x, in the order both quantizer paths use ------------------------------------------------
// Thread t of a CTA owns values 16 (t & 1) .. +15 of block 128 r + t / 2 in round r (the values it quantizes); it adds
// their FP32 squares in FP64 in order, rounds in order; then a shuffle tree over the warp, then the warps in order.
// The reference adds the same FP64 terms left to right; both round to the same FP32 mean unless the exact sum lies
// within ~1e-13 (relative) of an FP32 rounding boundary.
__device__ __forceinline__ double sumsq16(const float4 (&v)[4]) {
    double acc = 0.0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc += double(fmul(v[i].x, v[i].x));
        acc += double(fmul(v[i].y, v[i].y));
        acc += double(fmul(v[i].z, v[i].z));
        acc += double(fmul(v[i].w, v[i].w));
    }
    return acc;
}

// The 16 values of thread t in round r (zeros past the end); cg: read through L2 only.
__device__ __forceinline__ void load16(const float *x, unsigned n, unsigned r, bool cg, float4 (&v)[4]) {
    const unsigned b = r * (kPanelThreads / 2) + threadIdx.x / 2, h = threadIdx.x & 1u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (b < n / 32) {
            const float4 *p = reinterpret_cast<const float4 *>(x + b * 32 + h * 16) + i;
            v[i] = cg ? __ldcg(p) : *p;
        }
    }
}

// Completes the sum from each thread's partial (every thread of the CTA calls it) and returns the RMSNORM scale.
__device__ __forceinline__ float norm_scale(double acc, unsigned n, float eps, unsigned l2, double *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = acc;
    __syncthreads();
    double sum = 0.0;
    for (unsigned w = 0; w < kPanelWarps; ++w) sum += red[w];
    if (l2) return fdiv(1.0f, fmaxf(__fsqrt_rn(__double2float_rn(sum)), eps));
    return fdiv(1.0f, __fsqrt_rn(fadd(__double2float_rn(__ddiv_rn(sum, double(n))), eps)));
}

struct XSmem {
    const uint4 *q0, *q1, *meta;
};

// Plain C++ shared-memory loads (not volatile asm): the compiler may issue them early and overlap them.
__device__ __forceinline__ XBlock load_xblock(const XSmem &xs, unsigned b) {
    XBlock x;
    x.q0 = xs.q0[b];
    x.q1 = xs.q1[b];
    const uint4 m = xs.meta[b];
    x.d = __uint_as_float(m.x);
    x.s = __uint_as_float(m.y);
    x.bsum = int(m.z);
    return x;
}

// Exact integer block dot and the FP32 block term (the CPU path's arithmetic, gemvq_ref.h:215-262).
template <unsigned FMT>
__device__ __forceinline__ float block_term(const Step<FMT> &w, const XBlock &x, int &sumi) {
    int d0 = 0, d1 = 0;
    if (FMT == 8) {
        d0 = __dp4a(int(w.q0.x), int(x.q0.x), d0);
        d1 = __dp4a(int(w.q1.x), int(x.q1.x), d1);
        d0 = __dp4a(int(w.q0.y), int(x.q0.y), d0);
        d1 = __dp4a(int(w.q1.y), int(x.q1.y), d1);
        d0 = __dp4a(int(w.q0.z), int(x.q0.z), d0);
        d1 = __dp4a(int(w.q1.z), int(x.q1.z), d1);
        d0 = __dp4a(int(w.q0.w), int(x.q0.w), d0);
        d1 = __dp4a(int(w.q1.w), int(x.q1.w), d1);
    } else {
        // byte j: low nibble = element j, high nibble = element j + 16
        const uint32_t m = 0x0F0F0F0Fu;
        d0 = __dp4a(int(w.q0.x & m), int(x.q0.x), d0);
        d1 = __dp4a(int((w.q0.x >> 4) & m), int(x.q1.x), d1);
        d0 = __dp4a(int(w.q0.y & m), int(x.q0.y), d0);
        d1 = __dp4a(int((w.q0.y >> 4) & m), int(x.q1.y), d1);
        d0 = __dp4a(int(w.q0.z & m), int(x.q0.z), d0);
        d1 = __dp4a(int((w.q0.z >> 4) & m), int(x.q1.z), d1);
        d0 = __dp4a(int(w.q0.w & m), int(x.q0.w), d0);
        d1 = __dp4a(int((w.q0.w >> 4) & m), int(x.q1.w), d1);
    }
    sumi = d0 + d1 - (FMT == 2 ? 8 * x.bsum : 0);  // Q4_0: sum (w - 8) q = sum w q - 8 sum q
    if (FMT == 3) {
        // (d_w * d_8) * sumi + m_w * s_8 (gemvq_ref.h:221-223)
        const float dw = half_bits_to_float(uint16_t(w.d & 0xffffu)), mw = half_bits_to_float(uint16_t(w.d >> 16));
        return fadd(fmul(fmul(dw, x.d), float(sumi)), fmul(mw, x.s));
    }
    return fmul(float(sumi), fmul(half_bits_to_float(uint16_t(w.d)), x.d));
}

// L2 prefetch of [p, p + bytes) (bulk, 16-byte multiples; no data returns to the SM).
__device__ __forceinline__ void l2_prefetch(const uint8_t *p, unsigned long long bytes) {
    while (bytes) {
        const unsigned n = bytes > (1u << 20) ? (1u << 20) : unsigned(bytes);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(n) : "memory");
        p += n;
        bytes -= n;
    }
}

// Steps [from, kc) of an item into L2, in step order (a pair: its g and u panels in alternating 16 KB pieces), so
// the earlier steps arrive first. One thread.
__device__ __forceinline__ void prefetch_panel(const GemvArgs &a, unsigned item, unsigned from) {
    if (item >= a.item_start[a.n_units]) return;
    const unsigned u = unit_of(a, item), pnl = item - a.item_start[u];
    const int pair = a.unit_pair[u];
    const MatrixView &g = unit_member(a, u).w;
    const unsigned ga = from * g.tile_bytes, gb = g.kc * g.tile_bytes;
    const uint8_t *pg = g.base + size_t(pnl) * gb;
    const MatrixView &v = pair >= 0 ? a.m[pair].w : g;
    const unsigned va = pair >= 0 ? from * v.tile_bytes : 0u, vb = pair >= 0 ? v.kc * v.tile_bytes : 0u;
    const uint8_t *pv = v.base + size_t(pnl) * vb;
    constexpr unsigned kPiece = 16384;
    for (unsigned k = 0; ga + k < gb || va + k < vb; k += kPiece) {
        if (ga + k < gb) l2_prefetch(pg + ga + k, min(kPiece, gb - ga - k));
        if (va + k < vb) l2_prefetch(pv + va + k, min(kPiece, vb - va - k));
    }
}

// ---- x preparation, split over a cluster of kXCluster CTAs ---------------------------------------------------------
__device__ __forceinline__ float4 ldg_act4(const float *p) {
    return *reinterpret_cast<const float4 *>(p);
}

// Shared-memory image of the quantized x of a Q8 pass: the RMSNORM partial sums, the quants as two runs of
// 16-byte halves, one meta word {d, s, sum of q, 0} per 32-block.
struct QImage {
    double *red;
    uint8_t *q;
    uint4 *meta;
};
__host__ __device__ inline size_t qimage_bytes(unsigned cols) { return 256 + size_t(cols) + size_t(cols / 32) * 16; }
__device__ __forceinline__ QImage carve_qimage(unsigned char *p, unsigned cols) {
    QImage X;
    X.red = reinterpret_cast<double *>(p);
    X.q = p + 256;
    X.meta = reinterpret_cast<uint4 *>(p + 256 + cols);
    return X;
}

// Q8_0 / Q8_1 image of x (optionally through the deferred RMSNORM) in the shared memory of every CTA of the
// cluster: CTA `rank` quantizes the blocks [rank * per, rank * per + per) (per <= 128), two lanes per block (16
// values each, straight from global memory; lane h of the pair owns the block's h-th 16 quant bytes) and stores
// each block into all kXCluster images (distributed shared memory, 16-byte stores). The RMSNORM sum of squares
// over the whole x: every CTA computes it in the same fixed order (per thread, then a shuffle tree, then the warps
// in order), so all CTAs get the same scale. Same arithmetic as the reference CPU quantizer (quant.cuh,
// gemvq_ref.h:196-245). The caller arrived on the cluster barrier at the kernel's start; the wait here (every peer
// has started, its x_bar initialised) precedes the first store into a peer. Afterwards every image is complete: with
// ASYNC each block goes to every CTA by st.async, which counts its bytes on that CTA's x_bar, and a CTA waits until
// its x_bar has counted them all (no closing cluster barrier); otherwise plain DSMEM stores and a cluster barrier.
// (Measured on the same box: ASYNC made the Q4_0 decode ~1.3% faster and the Q8_0 stack ~0.6% slower, hence its
// use for every format but Q8_0.)
constexpr unsigned kXCluster = 4;
static_assert(kMaxQuantCols / 32 / kXCluster <= kPanelThreads / 2, "one round of two lanes per block");
template <bool ASYNC, class Hook>
__device__ __forceinline__ void prepare_x_cluster(const GemvArgs &a, const QImage &X, unsigned act, uint64_t *x_bar,
                                                  Hook after_loads) {
    const unsigned n = a.cols, nb = n / 32, rank = cluster_rank();
    const unsigned per = (nb + kXCluster - 1) / kXCluster, b0 = rank * per, b1 = min(nb, b0 + per);
    const bool norm = (a.norm_mode & 8u) != 0, weighted = (a.norm_mode & 2u) == 0;
    const unsigned t = threadIdx.x, h = t & 1u, b = b0 + (t >> 1);
    const bool live = b < b1;
    float v[16], w16[16];
#pragma unroll
    for (unsigned i = 0; i < 4; ++i) {
        float4 xv = make_float4(0.f, 0.f, 0.f, 0.f), wv = make_float4(1.f, 1.f, 1.f, 1.f);
        if (live) {
            xv = ldg_act4(a.x + b * 32 + h * 16 + i * 4);
            if (norm && weighted) wv = ldg_act4(a.norm_w + b * 32 + h * 16 + i * 4);
        }
        v[4 * i] = xv.x, v[4 * i + 1] = xv.y, v[4 * i + 2] = xv.z, v[4 * i + 3] = xv.w;
        w16[4 * i] = wv.x, w16[4 * i + 1] = wv.y, w16[4 * i + 2] = wv.z, w16[4 * i + 3] = wv.w;
    }
    // the RMSNORM sum: from the previous pass's per-panel partials when it wrote them (in panel order, then the
    // fixed tree), else from the whole x (canonical order); either is requested before the hook
    const bool partials = ASYNC && norm && a.nsq_in;  // (never handed to Q8_0 passes: compiled out of those)
    float4 nv[4];
    double pa = 0.0;
    if (partials) {
        const double p0 = threadIdx.x < a.nsq_n ? __ldcg(a.nsq_in + threadIdx.x) : 0.0;
        const double p1 = threadIdx.x + kPanelThreads < a.nsq_n ? __ldcg(a.nsq_in + threadIdx.x + kPanelThreads) : 0.0;
        pa = p0 + p1;
    } else if (norm) {
        load16(a.x, n, 0, false, nv);
    }
    after_loads();
    float scale = 1.0f;
    if (norm) {
        double acc = pa;
        if (partials) {
            for (unsigned i = threadIdx.x + 2 * kPanelThreads; i < a.nsq_n; i += kPanelThreads) acc += __ldcg(a.nsq_in + i);
        } else {
            acc = sumsq16(nv);
            for (unsigned r = 1; r * (kPanelThreads / 2) < nb; ++r) {
                load16(a.x, n, r, false, nv);
                acc += sumsq16(nv);
            }
        }
        scale = norm_scale(acc, n, a.norm_eps, a.norm_mode & 1u, X.red);
    }
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        if (norm) v[e] = weighted ? fmul(fmul(v[e], scale), w16[e]) : fmul(v[e], scale);
        amax = fmaxf(amax, fabsf(v[e]));
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    const float s = fdiv(amax, 127.0f);
    const float id = s != 0.0f ? fdiv(1.0f, s) : 0.0f;
    int sum = 0;
    uint32_t word[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        const int q = int(roundf(fmul(v[e], id)));
        sum += q;
        word[e / 4] |= uint32_t(q & 0xff) << (8 * (e % 4));
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    cluster_wait();  // every CTA of the cluster has started (the arrive is at the kernel's start)
    // ASYNC: this CTA's image is complete when its x_bar has counted every block's bytes, from all four CTAs
    if (ASYNC && threadIdx.x == 0) mbar_expect_tx(x_bar, n + nb * 16);
    if (live) {
        const uint32_t qa = smem_addr(X.q) + h * (n / 2) + b * 16, ma = smem_addr(X.meta) + b * 16;
        const uint4 qw = make_uint4(word[0], word[1], word[2], word[3]);
        const float dh = half_bits_to_float(float_to_half_bits(s));
        const float sh = act == 1 ? half_bits_to_float(float_to_half_bits(fmul(float(sum), s))) : 0.0f;
        const uint4 m = make_uint4(__float_as_uint(dh), __float_as_uint(sh), uint32_t(sum), 0u);
#pragma unroll
        for (unsigned k = 0; k < kXCluster; ++k) {
            if (ASYNC) {
                const uint32_t pb = peer_smem(smem_addr(x_bar), k);
                st_async_v4(peer_smem(qa, k), qw, pb);
                if (h == 0) st_async_v4(peer_smem(ma, k), m, pb);
            } else {
                st_cluster_v4(peer_smem(qa, k), qw);
                if (h == 0) st_cluster_v4(peer_smem(ma, k), m);
            }
        }
    }
    if (ASYNC) {
        if (!mbar_wait(x_bar, 0) && threadIdx.x == 0 && a.err) atomicExch(a.err, 1u);
    } else {
        cluster_sync();
    }
}

// Copy of a pre-quantized x (scratch of a separate quantize launch) into the image.
__device__ __forceinline__ void load_xq(const GemvArgs &a, const QImage &X, unsigned act) {
    const unsigned n = a.cols, nb = n / 32;
    for (unsigned i = threadIdx.x; i < n / 16; i += kPanelThreads)
        reinterpret_cast<uint4 *>(X.q)[(i & 1u) * (n / 32) + i / 2] = reinterpret_cast<const uint4 *>(a.xq)[i];
    for (unsigned i = threadIdx.x; i < nb; i += kPanelThreads)
        X.meta[i] = make_uint4(__float_as_uint(a.xd[i]), act == 1 ? __float_as_uint(a.xs[i]) : 0u, uint32_t(a.xb[i]), 0u);
    __syncthreads();
}

// Copy of an x image written by the previous pass (same layout as the shared-memory image: quants, then meta). The
// loads go out before the hook (the weight staging copy), so they are not queued behind it.
template <class Hook>
__device__ __forceinline__ void load_qimage(const GemvArgs &a, const QImage &X, Hook after_loads) {
    const unsigned n = a.cols, words = (n + n / 32 * 16) / 16;
    const uint4 *src = reinterpret_cast<const uint4 *>(a.qin);
    uint4 *dst = reinterpret_cast<uint4 *>(X.q);
    constexpr unsigned kPre = (kQImageBytes / 16 + kPanelThreads - 1) / kPanelThreads;
    uint4 v[kPre];
#pragma unroll
    for (unsigned k = 0; k < kPre; ++k) {
        const unsigned i = threadIdx.x + k * kPanelThreads;
        if (i < words) v[k] = __ldcg(src + i);
    }
    after_loads();
#pragma unroll
    for (unsigned k = 0; k < kPre; ++k) {
        const unsigned i = threadIdx.x + k * kPanelThreads;
        if (i < words) dst[i] = v[k];
    }
    __syncthreads();
}



// ---- staged leading steps, compute, fold --------------------------------------------------------------------------
// Bounded spin (kWaitLimitNs) on the completion of phase `parity` of `bar` (non-blocking test).
__device__ __forceinline__ bool mbar_spin(uint64_t *bar, unsigned parity) {
    const uint32_t a = smem_addr(bar);
    unsigned long long start = 0;
    for (unsigned i = 0;; ++i) {
        uint32_t done;
        asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                     : "=r"(done)
                     : "r"(a), "r"(parity)
                     : "memory");
        if (done) return true;
        if ((i & 1023u) == 1023u) {
            const unsigned long long now = global_ns();
            if (start == 0) start = now;
            else if (now - start > kWaitLimitNs) return false;
        }
    }
}

// Weights of the first steps of a CTA's first panel, staged in shared memory by one bulk copy (per matrix) issued
// with the x loads: [A: k steps][B: k steps (pairs)].
struct Staging {
    const uint8_t *base;  // A's first staged step
    unsigned k;           // staged steps (0: none)
    uint32_t b_off;       // offset of B's part
};

template <unsigned FMT>
__device__ __forceinline__ void load_step_smem(Step<FMT> &v, const uint8_t *tile, unsigned lane) {
    v.q0 = reinterpret_cast<const uint4 *>(tile)[lane];
    if (FMT == 8) {
        v.q1 = reinterpret_cast<const uint4 *>(tile + 512)[lane];
        v.d = reinterpret_cast<const uint16_t *>(tile + 1024)[lane];
    } else if (FMT == 2) {
        v.d = reinterpret_cast<const uint16_t *>(tile + 512)[lane];
    } else {
        v.d = reinterpret_cast<const uint32_t *>(tile + 512)[lane];
    }
}

// Warp w: steps w, w + 8, ... of one panel, block terms into the term buffers (row s = step s, 32 floats). FA alone
// (FB == 0) or the SwiGLU pair g (FA) / u (FB) over the same rows and steps. U steps in flight; staged steps come
// from shared memory. False if the wait for the staged steps gave up.
template <unsigned FA, unsigned FB, unsigned U>
__device__ __forceinline__ bool compute_steps(const GemvArgs &a, const GemvMemberArgs &MA, const GemvMemberArgs &MB,
                                              unsigned pnl, const XSmem &xs, unsigned warp, unsigned lane,
                                              uint64_t pol, float *term_a, float *term_b, const Staging &stg,
                                              uint64_t *stage_bar) {
    const MatrixView &w = MA.w;
    const unsigned J = w.ct, S = w.kc, nb = a.cols / 32, TS = term_stride(S * J);
    const unsigned j = lane & (J - 1u), lrow = pnl * w.rt + lane / J;
    const unsigned tslot = (lane / J) * TS + j;  // + s J: the term of (row lane / J, block s J + j)
    const unsigned TA = w.tile_bytes, TB = FB ? MB.w.tile_bytes : 0u;
    const uint8_t *ta = w.base + size_t(pnl) * S * TA;
    const uint8_t *tb = FB ? MB.w.base + size_t(pnl) * S * TB : nullptr;
    constexpr unsigned FB_ = FB ? FB : FA;
    constexpr unsigned NW = kPanelWarps;
    const unsigned n_my = S > warp ? (S - warp + NW - 1) / NW : 0u;
    // this warp's steps i < i_g are staged (step warp + 8 i < k), the rest stream from global memory
    const unsigned i_g = min(n_my, stg.k > warp ? (stg.k - warp + NW - 1) / NW : 0u);
    int32_t *dbg = a.dbg && lrow < w.rows ? a.dbg + size_t(w.row0 + lrow) * nb : nullptr;
    auto step = [&](const Step<FA> &ca, const Step<FB_> &cb, unsigned i) {
        const unsigned s = warp + NW * i;
        const unsigned b = s * J + j, bc = b < nb ? b : 0u;
        const XBlock x = load_xblock(xs, bc);
        int sumi;
        term_a[tslot + s * J] = block_term<FA>(ca, x, sumi);
        if (dbg && b < nb) dbg[b] = sumi;
        if (FB) {
            int su;
            term_b[tslot + s * J] = block_term<FB_>(cb, x, su);
        }
    };
    Step<FA> ba[U];
    Step<FB_> bb[U];
#pragma unroll
    for (unsigned k = 0; k < U; ++k) {
        const unsigned i = i_g + k;
        if (i < n_my) {
            load_step<FA>(ba[k], ta + (warp + NW * i) * TA, lane, pol);
            if (FB) load_step<FB_>(bb[k], tb + (warp + NW * i) * TB, lane, pol);
        }
    }
    const bool ok = i_g == 0 || mbar_spin(stage_bar, 0);
    for (unsigned i = 0; ok && i < i_g; ++i) {
        const unsigned s = warp + NW * i;
        Step<FA> ca;
        Step<FB_> cb;
        load_step_smem<FA>(ca, stg.base + s * TA, lane);
        if (FB) load_step_smem<FB_>(cb, stg.base + stg.b_off + s * TB, lane);
        step(ca, cb, i);
    }
    for (unsigned i0 = i_g; ok && i0 < n_my; i0 += U) {
#pragma unroll
        for (unsigned k = 0; k < U; ++k) {
            const unsigned i = i0 + k;
            if (i < n_my) {
                step(ba[k], bb[k], i);  // then the slot takes step i + U
                if (i + U < n_my) {
                    const unsigned s2 = warp + NW * (i + U);
                    load_step<FA>(ba[k], ta + s2 * TA, lane, pol);
                    if (FB) load_step<FB_>(bb[k], tb + s2 * TB, lane, pol);
                }
            }
        }
    }
    return ok;
}

// Row r's terms in block order, sum += term from 0: the CPU's sequential FP32 sum (gemvq_ref.h:248-262). The terms
// of row r are contiguous at terms[r TS ..] (term_stride), read 16 at a time with 16-byte loads ahead of their
// additions, so the dependent chain of additions is the only wait.
__device__ __forceinline__ float fold_row(const float *terms, unsigned r, unsigned TS, unsigned nb) {
    const float *t = terms + r * TS;
    const float4 *t4 = reinterpret_cast<const float4 *>(t);
    float acc = 0.0f;
    unsigned k = 0;
#pragma unroll 2
    for (; k + 16 <= nb; k += 16) {
        float4 v[4];
#pragma unroll
        for (unsigned e = 0; e < 4; ++e) v[e] = t4[k / 4 + e];
#pragma unroll
        for (unsigned e = 0; e < 4; ++e) {
            acc = fadd(acc, v[e].x);
            acc = fadd(acc, v[e].y);
            acc = fadd(acc, v[e].z);
            acc = fadd(acc, v[e].w);
        }
    }
    for (; k < nb; ++k) acc = fadd(acc, t[k]);
    return acc;
}

// One launch serves the units of one format combination: FA alone (FB == 0) or SwiGLU pairs FA / FB. Clusters
// of kXCluster CTAs share the x preparation.
//   shared memory: [x image][terms A][terms B (pairs)][staging mbarrier, u sums][staged steps]
// PEERS: a row-sharded multi-GPU launch (rows also stored into the peers, ready / data flags); a separate
// instantiation so single-GPU launches carry none of it.
template <unsigned FA, unsigned FB, unsigned U, bool PEERS>
__global__ void __cluster_dims__(kXCluster, 1, 1) __launch_bounds__(kPanelThreads, 3)
    gemv_q8_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char *p = smem;
    const QImage X = carve_qimage(p, a.cols);
    p += align128(qimage_bytes(a.cols));
    float *term_a = reinterpret_cast<float *>(p), *term_b = reinterpret_cast<float *>(p + (FB ? a.term_bytes : 0u));
    p += (FB ? 2u : 1u) * a.term_bytes;
    uint64_t *stage_bar = reinterpret_cast<uint64_t *>(p);
    float *usum = reinterpret_cast<float *>(p + 128);  // 32 floats
    p += 256;
    const unsigned warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const unsigned total = a.item_start[a.n_units];
    uint64_t *x_bar = stage_bar + 1;  // the x image's arrival (bytes from the cluster's CTAs)
    if (threadIdx.x == 0) {
        mbar_init(stage_bar, 1);
        mbar_init(x_bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    // the first steps of the first panel into shared memory: one bulk copy per matrix
    Staging stg{p, 0u, 0u};
    unsigned u0 = 0, pnl0 = 0;
    if (blockIdx.x < total && a.n_stages) {
        u0 = unit_of(a, blockIdx.x);
        pnl0 = blockIdx.x - a.item_start[u0];
        const MatrixView &g = unit_member(a, u0).w;
        stg.k = min(a.n_stages, g.kc);
        stg.b_off = stg.k * g.tile_bytes;
    }
    auto issue_staging = [&]() {
        if (threadIdx.x != 0 || stg.k == 0) return;
        const uint64_t pol = evict_first_policy();
        const MatrixView &g = unit_member(a, u0).w;
        const MatrixView *v = FB ? &a.m[a.unit_pair[u0]].w : nullptr;
        const unsigned bytes_b = v ? stg.k * v->tile_bytes : 0u;
        mbar_expect_tx(stage_bar, stg.b_off + bytes_b);
        bulk_copy(p, g.base + size_t(pnl0) * g.kc * g.tile_bytes, stg.b_off, stage_bar, pol);
        if (v) bulk_copy(p + stg.b_off, v->base + size_t(pnl0) * v->kc * v->tile_bytes, bytes_b, stage_bar, pol);
    };
    // x prepared across the cluster: announce that this CTA has started (its shared memory may be written by the
    // others); the matching wait comes before the first store into a peer
    const bool cluster_x = !a.qin && !a.xq;
    if (cluster_x) cluster_arrive_relaxed();
    pdl_launch_dependents();  // the next kernel may start as SMs free up
    // weights never change within a list: a CTA that is resident before the previous kernel completes starts its
    // staging copy now, and asks L2 for the rest of its first panel, so HBM streams while that kernel finishes and
    // while x is prepared. (Issued after the wait, the L2 requests held up thread 0's warp behind the staging copies
    // in the copy engine's queue for ~1.5 us; later panels are not prefetched: that cost more than it saved.)
    issue_staging();
    if (threadIdx.x == 0 && blockIdx.x < total) prefetch_panel(a, blockIdx.x, stg.k);
    pdl_wait();
    constexpr bool peers = PEERS;
    if (peers && blockIdx.x == 0 && threadIdx.x == 0) peer_announce(a.ps);
    peer_wait_rows_cta(a.pw);
    if (a.qin) {
        load_qimage(a, X, [] {});
    } else if (a.xq) {
        load_xq(a, X, FA == 3 ? 1u : 0u);
    } else {
        prepare_x_cluster<FA != 8>(a, X, FA == 3 ? 1u : 0u, x_bar, [] {});
    }
    const unsigned n = a.cols, nb = n / 32;
    const XSmem xs{reinterpret_cast<const uint4 *>(X.q), reinterpret_cast<const uint4 *>(X.q + n / 2), X.meta};
    const uint64_t pol = evict_first_policy();
    bool failed = false;
    const PeerSync *ps = nullptr;  // set once every peer has reached this launch (before the first store)
    unsigned np = 0;
    for (unsigned it = blockIdx.x; it < total; it += gridDim.x, ++np) {
        const unsigned u = unit_of(a, it), pnl = it - a.item_start[u];
        const GemvMemberArgs &MA = unit_member(a, u);
        const GemvMemberArgs &MB = FB ? a.m[a.unit_pair[u]] : MA;
        const MatrixView &w = MA.w;
        const unsigned P = w.rt, lrow = pnl * P + lane;
        const bool mine = lane < P && lrow < w.rows;
        const GemvMemberArgs &OUT = FB ? MB : MA;
        float res = 0.0f;  // residual of the row, loaded before the steps (off the tail)
        if (warp == 0 && mine && OUT.epi == EpiAdd && !a.dbg) res = OUT.res[w.row0 + lrow];
        const Staging none{nullptr, 0u, 0u};
        if (!compute_steps<FA, FB, U>(a, MA, MB, pnl, xs, warp, lane, pol, term_a, term_b, np == 0 ? stg : none,
                                      stage_bar)) {
            failed = true;
            if (lane == 0 && a.err) atomicExch(a.err, 1u);
        }
        if (__syncthreads_or(failed)) break;
        if (!a.dbg) {
            // the row sums: warp 0 folds the g (or only) terms while warp 1 folds a pair's u terms
            const unsigned out_member = FB ? unsigned(a.unit_pair[u]) : a.unit_member[u];
            const bool handoff = a.qout && out_member == a.qout_member && P == 32;
            const unsigned TS = term_stride(w.kc * w.ct);
            float acc = 0.0f;
            if (warp == 0 && (handoff || mine)) acc = fold_row(term_a, lane, TS, nb);
            if (FB && warp == 1 && lane < P) usum[lane] = fold_row(term_b, lane, TS, nb);
            if (FB) __syncthreads();
            if (warp == 0) {
                if (peers && np == 0) {
                    const bool ok = __shfl_sync(0xffffffffu, lane == 0 ? peer_wait_ready(a.ps) : false, 0);
                    if (ok) ps = &a.ps;
                    else if (lane == 0 && a.err) atomicExch(a.err, 1u);
                }
                if (handoff) {
                    // this panel is block pnl of the next pass's x: every lane holds a row (rows % 32 == 0)
                    const float val = FB ? row_value(MB, w.row0 + lrow, usum[lane], acc)
                                         : row_value(MA, w.row0 + lrow, acc, 0.0f, &res);
                    OUT.y[w.row0 + lrow] = val;
                    write_image_block(a.qout, OUT.total_rows, pnl, val, lane, a.qout_act);
                } else if (mine) {
                    if (FB) write_row(MB, w.row0 + lrow, usum[lane], acc, nullptr, ps);
                    else write_row(MA, w.row0 + lrow, acc, 0.0f, &res, ps);
                }
                if (a.nsq_out && out_member == a.nsq_member) {
                    // the next pass's deferred-norm sum: this panel's stored values squared, summed in a fixed tree
                    const float v = !mine ? 0.0f
                                          : (FB ? row_value(MB, w.row0 + lrow, usum[lane], acc)
                                                : row_value(MA, w.row0 + lrow, acc, 0.0f, &res));
                    double sq = double(fmul(v, v));
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                    if (lane == 0) a.nsq_out[pnl] = sq;
                }
                const unsigned end = min((pnl + 1) * P, w.rows);
                if (end == w.rows) write_padding(OUT, w.row0 + end, lane, ps);
            }
        }
        __syncthreads();  // the term buffers are reused by the next panel
    }
    // a staging copy that no warp waited for (a failure): let it land before the CTA exits
    if (threadIdx.x == 0 && stg.k && failed) mbar_spin(stage_bar, 0);
    if (peers && warp == 0) {  // this CTA's rows are in every peer: count it; the last CTA raises the data flags
        __syncwarp();
        if (lane == 0) peer_signal(a.ps, gridDim.x);
    }
}

using GemvKernel = void (*)(GemvArgs);

// The kernel of a format combination (fb = 0: single members), or null.
template <bool PEERS>
static GemvKernel q8_kernel_of(unsigned fa, unsigned fb) {
    if (fb == 0) {
        if (fa == 8) return gemv_q8_kernel<8, 0, 4, PEERS>;
        if (fa == 2) return gemv_q8_kernel<2, 0, 6, PEERS>;
        if (fa == 3) return gemv_q8_kernel<3, 0, 6, PEERS>;
    } else {
        if (fa == 8 && fb == 8) return gemv_q8_kernel<8, 8, 2, PEERS>;
        if (fa == 2 && fb == 2) return gemv_q8_kernel<2, 2, 3, PEERS>;
        if (fa == 8 && fb == 2) return gemv_q8_kernel<8, 2, 2, PEERS>;
        if (fa == 2 && fb == 8) return gemv_q8_kernel<2, 8, 2, PEERS>;
        if (fa == 3 && fb == 3) return gemv_q8_kernel<3, 3, 3, PEERS>;
    }
    return nullptr;
}
static GemvKernel q8_kernel_for(unsigned fa, unsigned fb, bool peers = false) {
    return peers ? q8_kernel_of<true>(fa, fb) : q8_kernel_of<false>(fa, fb);
}

__global__ void __launch_bounds__(256) quantize_kernel(const QuantArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const XImage X = carve_ximage(smem, a.n);
    pdl_wait();
    pdl_launch_dependents();
    peer_wait_rows_cta(a.pw);
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

// Shared memory of a Q8 pass: the x image (split halves), the term buffers of one panel (two for a pair), the
// staging mbarrier and the u sums, and as many staged leading steps of the first panel as keep three CTAs per SM.
void plan_gemv_q8(GemvArgs &a, size_t &smem) {
    a.wraw = 0;
    a.res_bytes = 0;
    unsigned steps = 0, stage_step_bytes = 0;
    bool pair = false;
    for (unsigned u = 0; u < a.n_units; ++u) {
        const MatrixView &g = a.m[a.unit_member[u]].w;
        steps = steps > g.kc ? steps : g.kc;
        unsigned sb = g.tile_bytes;
        if (a.unit_pair[u] >= 0) {
            pair = true;
            sb += a.m[a.unit_pair[u]].w.tile_bytes;
        }
        stage_step_bytes = stage_step_bytes > sb ? stage_step_bytes : sb;
    }
    unsigned tb = 0;
    for (unsigned u = 0; u < a.n_units; ++u) {
        const MatrixView &g = a.m[a.unit_member[u]].w;
        const unsigned b = g.rt * term_stride(g.kc * g.ct) * 4u;
        tb = tb > b ? tb : b;
    }
    a.term_bytes = unsigned(align128(tb));
    const size_t fixed = align128(qimage_bytes(a.cols)) + (pair ? 2u : 1u) * size_t(a.term_bytes) + 256;
    // staged leading steps: what is left of a third of the SM's shared memory (three CTAs per SM)
    const size_t per_cta = 227 * 1024 / 3 - 1024;
    const size_t room = per_cta > fixed ? per_cta - fixed : 0;
    a.n_stages = stage_step_bytes ? unsigned(std::min<size_t>(room / stage_step_bytes, steps)) : 0u;
    a.stage_bytes = unsigned(align128(size_t(a.n_stages) * stage_step_bytes));
    smem = fixed + a.stage_bytes;
}

unsigned gemv_q8_warps_per_cta() { return kPanelWarps; }

bool gemv_q8_supported(unsigned fa, unsigned fb) { return q8_kernel_for(fa, fb) != nullptr; }

// CTAs of the kernel of (fa, fb) with `smem` bytes of shared memory that are resident at once on the GPU (whole
// clusters of kXCluster).
unsigned gemv_q8_resident_ctas(unsigned fa, unsigned fb, size_t smem, cudaStream_t st) {
    const GemvKernel k = q8_kernel_for(fa, fb);
    if (!k) return kXCluster;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kXCluster * 148);
    cfg.blockDim = dim3(kPanelThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, k, &cfg) != cudaSuccess || clusters < 1) {
        cudaGetLastError();
        clusters = 1;
    }
    return unsigned(clusters) * kXCluster;
}

unsigned gemv_q8_cluster() { return kXCluster; }

cudaError_t launch_gemv_q8(const GemvArgs &a, unsigned fa, unsigned fb, unsigned grid, size_t smem, cudaStream_t st,
                           bool pdl) {
    const bool peers = a.ps.world > 1;
    const GemvKernel k = q8_kernel_for(fa, fb, peers);
    if (!k) return cudaErrorInvalidValue;
    if (peers) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kPanelThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, a);
}

// The quantizer's shared memory stays under the 48 KB every kernel may use without an attribute, for every n the
// library accepts, so no per-device function attribute is needed.
static_assert(ximage_bytes(kMaxQuantCols) + 127 <= 48 * 1024, "quantize_kernel's image fits the default shared memory");

cudaError_t launch_quantize(const QuantArgs &a, cudaStream_t st) {
    const size_t smem = (ximage_bytes(a.n) + 127) & ~size_t(127);
    quantize_kernel<<<1, 256, smem, st>>>(a);
    return cudaGetLastError();
}


// ==== persistent GEMV chain =========================================================================================
// One launch runs a chain of consecutive Q4_0 / Q8_0 passes (ChainArgs): the layer stack's norm -> gate+up (SwiGLU)
// -> down (+residual) -> norm -> ..., without a kernel boundary between the passes. One CTA per SM (any grid works:
// work is taken, not assigned, so no CTA waits for one that is not resident), 11 warps:
//   warp 8 (producer): takes the chain's items (row panels, numbered pass by pass) one at a time from a global
//     counter and streams each item's steps (one 32-unit tile per matrix), 8 consecutive steps of a pair or 16 of a
//     single matrix per stage (one bulk copy per matrix), into a ring of shared-memory stages. Weights never change, so it runs ahead into the
//     next pass while that pass still waits for its x: HBM keeps streaming through every dependency between passes
//     (the stall a kernel boundary costs).
//   warps 9, 10 (fold): per item, add each row's terms in block order (the CPU's FP32 sum, bit for bit; warp 10 a
//     pair's u terms) and write the row, while the consumers already fill the other of two term buffers;
//   warps 0-7 (consumers): per item, warp w takes steps w, w + 8, ... of every stage (lane = unit: the exact
//     integer block dot and the FP32 block term, as gemv_q8_kernel) into a term buffer; before an item of a new pass
//     they wait until every item of the previous pass is finished (a global counter per pass) and prepare that pass's
//     x: the previous pass's quantized image, or act x (through the deferred RMSNORM) quantized by the same
//     arithmetic as the single-pass kernel.
// Stage / queue hand-offs are mbarriers; every wait is bounded (kWaitLimitNs): on expiry the CTA sets the error word,
// stops, and lets its own bulk copies land before it exits. The launch's last CTA leaves the counters at zero. The
// kernel never triggers the next kernel's early launch, so the next chain launch finds its counters reset.
// Activations written inside the launch (x, the residual, the images) are read through L2 only (ld.global.cg).
constexpr unsigned kChainConsumers = 8, kChainThreads = 32 * (kChainConsumers + 3), kChainQueue = 8;
constexpr unsigned kChainEnd = 0xffffffffu;
constexpr unsigned kChainBarBytes = 2048;  // mbarriers, the item queue and words, the abort flag, 2 x 32 u sums
static_assert(sizeof(ChainArgs) <= 32000, "the chain's arguments fit the kernel parameter space");

// the consumer warps' barrier (named barrier 1; the producer warp never joins it)
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kChainConsumers) : "memory");
}
// ... and the same barrier returning, to every consumer thread, whether any of them passed true
__device__ __forceinline__ bool consumers_any(bool v) {
    uint32_t r;
    asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
                 : "=r"(r)
                 : "r"(unsigned(v)), "n"(32 * kChainConsumers)
                 : "memory");
    return r != 0;
}
__device__ __forceinline__ void fold_pair_sync() { asm volatile("bar.sync 2, 64;" ::: "memory"); }

__device__ __forceinline__ void red_release_gpu(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// A stage holds the consecutive steps of one item: kChainConsumers of a SwiGLU pair ([g steps][u steps at
// chain_pair_offset]) or twice as many of a single matrix, so that both fill the same bytes (each consumer warp
// takes one pair step or two single steps of a stage).
constexpr unsigned kChainPairSteps = kChainConsumers;
__host__ __device__ inline unsigned chain_stage_steps(unsigned pair) { return pair ? kChainPairSteps : 2 * kChainPairSteps; }
__host__ __device__ inline unsigned chain_pair_offset(unsigned tile_bytes) {
    return (kChainPairSteps * tile_bytes + 127u) & ~127u;
}

__device__ __forceinline__ unsigned chain_pass_of(const ChainArgs &a, unsigned g) {
    unsigned k = 0;
    while (k + 1 < a.n_passes && g >= a.p[k + 1].item0) ++k;
    return k;
}
__device__ __forceinline__ unsigned chain_items(const ChainArgs &a, unsigned k) {
    return (k + 1 < a.n_passes ? a.p[k + 1].item0 : a.total_items) - a.p[k].item0;
}

// The RMSNORM scale from each consumer thread's FP64 partial: the order of norm_scale (a shuffle tree per warp, then
// the warps in order), with the consumers' barrier.
__device__ __forceinline__ float chain_norm_scale(double acc, unsigned n, float eps, unsigned l2, double *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = acc;
    consumers_sync();
    double sum = 0.0;
    for (unsigned w = 0; w < kChainConsumers; ++w) sum += red[w];
    if (l2) return fdiv(1.0f, fmaxf(__fsqrt_rn(__double2float_rn(sum)), eps));
    return fdiv(1.0f, __fsqrt_rn(fadd(__double2float_rn(__ddiv_rn(sum, double(n))), eps)));
}

// x of pass P into the image (quants at q, meta words at q + cols), by the 256 consumer threads (x_kind 0 / 1): per
// 32-block the arithmetic of prepare_x_cluster (the same per-thread ownership of 16 values, the same FP64 norm sum
// order), every block by this CTA.
__device__ __forceinline__ void chain_prepare_x(const ChainPass &P, uint8_t *q, double *red) {
    const unsigned n = P.cols, nb = n / 32, t = threadIdx.x, h = t & 1u;
    uint4 *meta = reinterpret_cast<uint4 *>(q + n);
    const bool norm = P.x_kind == 1, weighted = (P.norm_mode & 2u) == 0;
    // round 0's x and weight values stay in registers from the one load both the norm sum and the quantizer use
    // (thread t owns the same 16 values in both); later rounds (more than 4096 columns) load again
    float4 x0[4], w0[4];
#pragma unroll
    for (unsigned i = 0; i < 4; ++i) {
        const unsigned b = t >> 1;
        x0[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        w0[i] = make_float4(1.f, 1.f, 1.f, 1.f);
        if (b < nb) {
            x0[i] = __ldcg(reinterpret_cast<const float4 *>(P.x + b * 32 + h * 16) + i);
            if (norm && weighted) w0[i] = __ldcg(reinterpret_cast<const float4 *>(P.norm_w + b * 32 + h * 16) + i);
        }
    }
    float scale = 1.0f;
    if (norm) {
        double acc = sumsq16(x0);
        for (unsigned r = 1; r * (kPanelThreads / 2) < nb; ++r) {
            float4 nv[4];
            load16(P.x, n, r, true, nv);
            acc += sumsq16(nv);
        }
        scale = chain_norm_scale(acc, n, P.norm_eps, P.norm_mode & 1u, red);
    }
    for (unsigned r = 0; r * (kPanelThreads / 2) < nb; ++r) {
        const unsigned b = r * (kPanelThreads / 2) + (t >> 1);
        const bool live = b < nb;
        float v[16];
#pragma unroll
        for (unsigned i = 0; i < 4; ++i) {
            float4 xv = x0[i], wv = w0[i];
            if (r > 0) {
                xv = make_float4(0.f, 0.f, 0.f, 0.f);
                wv = make_float4(1.f, 1.f, 1.f, 1.f);
                if (live) {
                    xv = __ldcg(reinterpret_cast<const float4 *>(P.x + b * 32 + h * 16) + i);
                    if (norm && weighted)
                        wv = __ldcg(reinterpret_cast<const float4 *>(P.norm_w + b * 32 + h * 16) + i);
                }
            }
            const float xs[4] = {xv.x, xv.y, xv.z, xv.w}, ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (unsigned e = 0; e < 4; ++e)
                v[4 * i + e] = !norm ? xs[e] : (weighted ? fmul(fmul(xs[e], scale), ws[e]) : fmul(xs[e], scale));
        }
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[e]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        const float s = fdiv(amax, 127.0f);
        const float id = s != 0.0f ? fdiv(1.0f, s) : 0.0f;
        int sum = 0;
        uint32_t word[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const int qv = int(roundf(fmul(v[e], id)));
            sum += qv;
            word[e / 4] |= uint32_t(qv & 0xff) << (8 * (e % 4));
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        if (live) {
            *reinterpret_cast<uint4 *>(q + h * (n / 2) + b * 16) = make_uint4(word[0], word[1], word[2], word[3]);
            if (h == 0) {
                const float dh = half_bits_to_float(float_to_half_bits(s));
                meta[b] = make_uint4(__float_as_uint(dh), 0u, uint32_t(sum), 0u);
            }
        }
    }
}

// The image the previous pass wrote (x_kind 2): quants, then the meta words, as they lie in shared memory.
__device__ __forceinline__ void chain_copy_image(const ChainPass &P, uint8_t *q) {
    const unsigned n = P.cols, words = (n + n / 32 * 16) / 16;
    const uint4 *src = reinterpret_cast<const uint4 *>(P.qin);
    uint4 *dst = reinterpret_cast<uint4 *>(q);
    for (unsigned i = threadIdx.x; i < words; i += 32 * kChainConsumers) dst[i] = __ldcg(src + i);
}

// Warp `warp`'s steps of one item: stage (s_base + c) % S holds steps M c .. M c + M - 1 (M = chain_stage_steps),
// and the warp takes steps M c + warp (+ 8) of each (every warp releases every stage once, as soon as its loads are
// in registers): steps warp, warp + 8, ... of the item. False if a wait gave up.
template <unsigned FMT, bool PAIR>
__device__ __forceinline__ bool chain_steps(const ChainPass &P, const XSmem &xs, unsigned warp, unsigned lane,
                                            const uint8_t *stages, unsigned stage_bytes, unsigned S, uint64_t *full,
                                            uint64_t *empty, unsigned s_base, float *term_a, float *term_b,
                                            volatile unsigned *abort) {
    constexpr unsigned M = PAIR ? kChainPairSteps : 2 * kChainPairSteps, R = M / kChainConsumers;
    const MatrixView &w = P.wa;
    const unsigned J = w.ct, K = w.kc, nb = P.cols / 32, TS = term_stride(K * J);
    const unsigned j = lane & (J - 1u), tslot = (lane / J) * TS + j;
    const unsigned boff = chain_pair_offset(w.tile_bytes);
    for (unsigned c = 0; c * M < K; ++c) {
        const unsigned gs = s_base + c, st = gs % S;
        if (!role_wait(full + st, (gs / S) & 1u, abort)) return false;
        const uint8_t *stage = stages + size_t(st) * stage_bytes;
        Step<FMT> ca[R], cb[R];
#pragma unroll
        for (unsigned r = 0; r < R; ++r) {
            const unsigned m = warp + kChainConsumers * r;
            if (c * M + m < K) {
                load_step_smem<FMT>(ca[r], stage + m * w.tile_bytes, lane);
                if (PAIR) load_step_smem<FMT>(cb[r], stage + boff + m * P.wb.tile_bytes, lane);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + st);
#pragma unroll
        for (unsigned r = 0; r < R; ++r) {
            const unsigned i = c * M + warp + kChainConsumers * r;
            if (i >= K) break;
            const unsigned b = i * J + j, bc = b < nb ? b : 0u;
            const XBlock x = load_xblock(xs, bc);
            int sumi;
            term_a[tslot + i * J] = block_term<FMT>(ca[r], x, sumi);
            if (PAIR) {
                int su;
                term_b[tslot + i * J] = block_term<FMT>(cb[r], x, su);
            }
        }
    }
    return true;
}

__device__ __forceinline__ bool chain_steps_any(const ChainPass &P, const XSmem &xs, unsigned warp, unsigned lane,
                                                const uint8_t *stages, unsigned stage_bytes, unsigned S,
                                                uint64_t *full, uint64_t *empty, unsigned s_base, float *term_a,
                                                float *term_b, volatile unsigned *abort) {
    if (P.fmt == 8)
        return P.pair ? chain_steps<8, true>(P, xs, warp, lane, stages, stage_bytes, S, full, empty, s_base, term_a,
                                             term_b, abort)
                      : chain_steps<8, false>(P, xs, warp, lane, stages, stage_bytes, S, full, empty, s_base, term_a,
                                              term_b, abort);
    return P.pair ? chain_steps<2, true>(P, xs, warp, lane, stages, stage_bytes, S, full, empty, s_base, term_a,
                                         term_b, abort)
                  : chain_steps<2, false>(P, xs, warp, lane, stages, stage_bytes, S, full, empty, s_base, term_a,
                                          term_b, abort);
}

// Bounded wait until a pass's items are all finished (one thread).
__device__ __forceinline__ bool chain_wait_pass(const unsigned *done, unsigned items) {
    unsigned long long t0 = 0;
    for (unsigned i = 0; ld_acquire_gpu(done) < items; ++i) {
        if ((i & 255u) == 255u) {
            const unsigned long long now = global_ns();
            if (t0 == 0) t0 = now;
            else if (now - t0 > kWaitLimitNs) return false;
        }
    }
    return true;
}

__global__ void __launch_bounds__(kChainThreads, 1) gemv_chain_kernel(const __grid_constant__ ChainArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const unsigned S = a.n_stages, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + S;
    uint64_t *qfull = empty + S, *qempty = qfull + kChainQueue;
    uint64_t *tready = qempty + kChainQueue, *tfree = tready + 2;  // per term buffer: terms written / folded
    unsigned *queue = reinterpret_cast<unsigned *>(tfree + 2);
    unsigned *info = queue + kChainQueue;  // per term buffer: the item whose terms it holds (kChainEnd: none left)
    volatile unsigned *abort = info + 2;
    float *usum = reinterpret_cast<float *>(smem + kChainBarBytes - 256);  // [2 buffers][32]
    unsigned char *p = smem + kChainBarBytes;
    double *red = reinterpret_cast<double *>(p);  // 256 bytes of norm partials, then the x image
    uint8_t *xq = p + 256;
    p += a.ximg_bytes;
    float *terms = reinterpret_cast<float *>(p);  // [2 buffers][a, b] of term_bytes each
    p += 4 * size_t(a.term_bytes);
    uint8_t *stages = p;
    if (threadIdx.x == 0) {
        for (unsigned i = 0; i < S; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, kChainConsumers);  // every consumer warp releases every stage
        }
        for (unsigned i = 0; i < kChainQueue; ++i) {
            mbar_init(qfull + i, 1);
            mbar_init(qempty + i, 1);
        }
        for (unsigned i = 0; i < 2; ++i) {
            mbar_init(tready + i, kChainConsumers);
            mbar_init(tfree + i, 1);
        }
        *abort = 0u;
        mbar_fence_init();
    }
    __syncthreads();
    unsigned *taken = a.counters, *finished = a.counters + 1, *done = a.counters + 2;
    const unsigned tw = a.term_bytes / 4;  // floats of one term buffer

    if (warp == kChainConsumers) {
        // ---- producer: weights only, so it starts before the wait on the previous kernel
        if (lane == 0) {
            const uint64_t pol = evict_first_policy();
            unsigned s = 0;
            bool ok = true;
            for (unsigned n = 0;; ++n) {
                const unsigned g = atomicAdd(taken, 1u);
                const unsigned q = n % kChainQueue;
                if (n >= kChainQueue && !role_wait(qempty + q, ((n / kChainQueue) - 1u) & 1u, abort)) ok = false;
                queue[q] = ok && g < a.total_items ? g : kChainEnd;
                mbar_arrive(qfull + q);
                if (ok && g < a.total_items) {
                    const ChainPass &P = a.p[chain_pass_of(a, g)];
                    const unsigned t = g - P.item0, K = P.wa.kc, ta = P.wa.tile_bytes, tb = P.wb.tile_bytes;
                    const uint8_t *src_a = P.wa.base + size_t(t) * K * ta;
                    const uint8_t *src_b = P.pair ? P.wb.base + size_t(t) * K * tb : nullptr;
                    const unsigned M = chain_stage_steps(P.pair);
                    for (unsigned i = 0; i < K; i += M, ++s) {
                        const unsigned st = s % S, m = min(M, K - i);
                        if (s >= S && !role_wait(empty + st, ((s / S) - 1u) & 1u, abort)) {
                            ok = false;
                            break;
                        }
                        uint8_t *dst = stages + size_t(st) * a.stage_bytes;
                        mbar_expect_tx(full + st, m * (P.pair ? ta + tb : ta));
                        bulk_copy(dst, src_a + size_t(i) * ta, m * ta, full + st, pol);
                        if (P.pair)
                            bulk_copy(dst + chain_pair_offset(ta), src_b + size_t(i) * tb, m * tb, full + st, pol);
                    }
                }
                if (!ok) {
                    if (a.err) atomicExch(a.err, 1u);
                    *abort = 1u;
                    // the copies already issued land before the CTA's shared memory goes away
                    for (unsigned k2 = s > S ? s - S : 0u; k2 < s; ++k2) mbar_spin(full + k2 % S, (k2 / S) & 1u);
                    break;
                }
                if (g >= a.total_items) break;
            }
        }
        return;
    }

    if (warp > kChainConsumers) {
        // ---- fold warps: warp 9 adds each row's (g) terms in block order and writes the row, warp 10 a pair's u
        // terms; per item, while the consumers already compute the next item's terms in the other buffer
        const bool gw = warp == kChainConsumers + 1;
        pdl_wait();
        for (unsigned n = 0;; ++n) {
            const unsigned b = n & 1u;
            if (!role_wait(tready + b, (n >> 1) & 1u, abort)) break;
            const unsigned g = info[b];
            if (g == kChainEnd) break;
            const unsigned k = chain_pass_of(a, g);
            const ChainPass &P = a.p[k];
            const unsigned t = g - P.item0, R = P.wa.rt, lrow = t * R + lane, nb = P.cols / 32;
            const unsigned TS = term_stride(P.wa.kc * P.wa.ct);
            const float *ta = terms + size_t(2 * b) * tw, *tb = ta + tw;
            const bool mine = lane < R && lrow < P.wa.rows;
            if (!gw) {
                if (P.pair) {
                    if (lane < R) usum[32 * b + lane] = fold_row(tb, lane, TS, nb);
                    fold_pair_sync();
                }
                continue;
            }
            const GemvMemberArgs &O = P.out;
            const bool image = P.qout != nullptr;  // 32-row panels: this panel is block t of the next pass's x
            float acc = 0.0f, val = 0.0f;
            if (mine || image) acc = fold_row(ta, lane, TS, nb);
            if (P.pair) fold_pair_sync();
            if (mine || image) {
                if (P.pair) val = fmul(silu_f32(acc), usum[32 * b + lane]);
                else if (O.epi == EpiAdd) val = fadd(acc, __ldcg(O.res + lrow));
                else val = acc;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(tfree + b);  // the terms (and u sums) of this buffer are read
            if (mine) O.y[lrow] = val;
            if (image) write_image_block(P.qout, O.total_rows, t, mine ? val : 0.0f, lane, P.qout_act);
            const unsigned end = min((t + 1) * R, P.wa.rows);
            if (end == P.wa.rows) write_padding(O, end, lane);
            __threadfence();
            __syncwarp();
            if (lane == 0) red_release_gpu(done + k, 1u);
        }
        // the launch's last CTA leaves the counters at zero for the next launch (the fold warp finishes last)
        if (gw && lane == 0) {
            __threadfence();
            if (atomicAdd(finished, 1u) == gridDim.x - 1) {
                for (unsigned i = 0; i < kChainCounters; ++i) a.counters[i] = 0u;
                __threadfence();
            }
        }
        return;
    }

    // ---- consumers
    pdl_wait();
    int cur = -1;
    unsigned s_base = 0;
    for (unsigned n = 0;; ++n) {
        const unsigned q = n % kChainQueue, b = n & 1u;
        bool bad = false;
        if (threadIdx.x == 0) bad = !role_wait(qfull + q, (n / kChainQueue) & 1u, abort);
        if (consumers_any(bad || *abort)) {
            if (threadIdx.x == 0 && a.err) atomicExch(a.err, 1u);
            *abort = 1u;
            break;
        }
        const unsigned g = queue[q];
        consumers_sync();
        if (threadIdx.x == 0) mbar_arrive(qempty + q);
        if (g == kChainEnd) {
            // the fold warps' last buffer: none left (the buffer's previous item was folded first)
            const bool ok = n < 2 || role_wait(tfree + b, ((n >> 1) - 1u) & 1u, abort);
            if (threadIdx.x == 0) info[b] = kChainEnd;
            __syncwarp();
            if (lane == 0 && ok) mbar_arrive(tready + b);
            break;
        }
        const unsigned k = chain_pass_of(a, g);
        const ChainPass &P = a.p[k];
        if (int(k) != cur) {
            // every item of the previous pass is finished (its rows, its image) before this pass's x is read
            bad = false;
            if (k > 0 && threadIdx.x == 0) bad = !chain_wait_pass(done + (k - 1), chain_items(a, k - 1));
            if (consumers_any(bad)) {
                if (threadIdx.x == 0 && a.err) atomicExch(a.err, 1u);
                *abort = 1u;
                break;
            }
            if (P.x_kind == 2) chain_copy_image(P, xq);
            else chain_prepare_x(P, xq, red);
            consumers_sync();
            cur = int(k);
        }
        // this buffer's previous item (n - 2) has been folded
        bool ok = n < 2 || role_wait(tfree + b, ((n >> 1) - 1u) & 1u, abort);
        const XSmem xs{reinterpret_cast<const uint4 *>(xq), reinterpret_cast<const uint4 *>(xq + P.cols / 2),
                       reinterpret_cast<const uint4 *>(xq + P.cols)};
        float *ta = terms + size_t(2 * b) * tw, *tb = ta + tw;
        if (ok) ok = chain_steps_any(P, xs, warp, lane, stages, a.stage_bytes, S, full, empty, s_base, ta, tb, abort);
        if (!ok) {
            if (lane == 0 && a.err) atomicExch(a.err, 1u);
            *abort = 1u;
        }
        if (threadIdx.x == 0) info[b] = g;
        __syncwarp();
        if (lane == 0) mbar_arrive(tready + b);  // this warp's terms of the item are written
        if (consumers_any(!ok)) break;
        s_base += (P.wa.kc + chain_stage_steps(P.pair) - 1) / chain_stage_steps(P.pair);
    }
}

bool plan_gemv_chain(ChainArgs &a, size_t &smem) {
    unsigned stage = 0, tb = 0, cols = 0;
    for (unsigned k = 0; k < a.n_passes; ++k) {
        const ChainPass &P = a.p[k];
        const unsigned sb = P.pair ? chain_pair_offset(P.wa.tile_bytes) + kChainPairSteps * P.wb.tile_bytes
                                   : chain_stage_steps(0) * P.wa.tile_bytes;
        stage = std::max(stage, sb);
        tb = std::max(tb, P.wa.rt * term_stride(P.wa.kc * P.wa.ct) * 4u);
        cols = std::max(cols, P.cols);
    }
    a.stage_bytes = unsigned(align128(stage));
    a.term_bytes = unsigned(align128(tb));
    a.ximg_bytes = unsigned(align128(qimage_bytes(cols)));
    const size_t fixed = kChainBarBytes + a.ximg_bytes + 4 * size_t(a.term_bytes);
    const size_t room = 227 * 1024 > fixed ? 227 * 1024 - fixed : 0;
    // full + empty mbarriers per stage; the queue's and the term buffers' mbarriers, the queue, the item words and the
    // abort word; the u sums at the end
    const unsigned max_stages = (kChainBarBytes - 256 - 16 * kChainQueue - 32 - 4 * (kChainQueue + 3)) / 16;
    a.n_stages = unsigned(std::min<size_t>(room / a.stage_bytes, max_stages));
    smem = fixed + size_t(a.n_stages) * a.stage_bytes;
    return a.n_stages >= 4;
}

cudaError_t launch_gemv_chain(const ChainArgs &a, unsigned grid, size_t smem, cudaStream_t st, bool pdl) {
    cudaError_t e = cudaFuncSetAttribute(gemv_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kChainThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_chain_kernel, a);
}


// ==== GEMV_BATCH: y_m = W x_m for up to kBatchMax activation rows on one read of the weights =========================
// The batch path of the reference's roadmap (docs/ROADMAP.md:80-96, P2: one weight word for M input vectors), for
// speculative-decode checks and several sequences per pass. One launch, 8 consumer warps + 1 producer warp per CTA;
// CTAs take the matrix's panels (P rows x all blocks) as gemv_q8_kernel does:
//   producer   one bulk copy per round of 16 consecutive steps (tiles) of the CTA's panels into a ring of shared-memory
//              stages (full / empty mbarriers, bounded waits); the first stages are issued before the wait on the
//              previous kernel, as the weights never change within a list;
//   consumers  after the wait, quantize the activation rows into shared-memory images (one thread per 32-value
//              block, the arithmetic of the GEMV pass's quantizer), then per round: lane = unit, two steps per warp,
//              the unit's exact integer block dot with the same block of every row and the FP32 block term
//              float(sumi) * (d_w * d_x) into the round's term buffer; one barrier; then one thread per (activation
//              row, panel row) adds the round's terms of its row in block order to its running sum (from 0 per panel).
// Every output row has the bits of the single GEMV of its activation row: the same terms (block_term), added in the
// same order (gemvq_ref.h:248-262). Roofline: HBM bandwidth (the weights once per launch); every CTA quantizes the
// rows itself (batch x cols x 4 bytes from L2). When the images, term buffers and a ring of two stages do not fit
// one CTA's shared memory, the host splits the rows over several launches (each reads the weights once).

constexpr unsigned kBatchChunk = 16;  // steps per round (one ring stage): two per consumer warp
constexpr unsigned kBatchThreads = kPanelThreads + 32;  // 8 consumer warps + the producer warp
constexpr unsigned kBatchBarBytes = 256;

__host__ __device__ inline size_t batch_img_smem(unsigned cols, unsigned mn) {
    return align128(size_t(mn) * (cols / 32) * kBatchImgBlockBytes);
}
// Term buffer of one round, per activation row: the round's blocks (kBatchChunk steps x C) x P rows, row fastest (a
// step's 32 stores are 32 consecutive words), plus P words of padding so that the P-row groups of the activation rows
// a warp folds at once start in different banks.
__host__ __device__ inline unsigned batch_row_stride(unsigned p) { return kBatchChunk * 32 + p; }
__host__ __device__ inline size_t batch_term_smem(const MatrixView &w, unsigned mn) {
    return align128(2 * size_t(mn) * batch_row_stride(w.rt) * 4);  // two rounds in flight
}
__host__ __device__ inline size_t batch_stage_bytes(const MatrixView &w) {
    return align128(size_t(kBatchChunk) * w.tile_bytes);
}
__host__ __device__ inline size_t batch_fixed_smem(const MatrixView &w, unsigned cols, unsigned mn) {
    return kBatchBarBytes + batch_img_smem(cols, mn) + batch_term_smem(w, mn);
}

template <unsigned FMT>
__global__ void __launch_bounds__(kBatchThreads) gemv_batch_kernel(const BatchArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const MatrixView &W = a.w;
    const unsigned mn = a.mn, nb = a.cols / 32, P = W.rt, C = W.ct, KC = W.kc, NS = a.n_stages;
    const unsigned rs = batch_row_stride(P);
    const unsigned rounds = (KC + kBatchChunk - 1) / kBatchChunk;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem), *empty = full + NS;
    uint8_t *img = smem + kBatchBarBytes;
    float *terms = reinterpret_cast<float *>(img + batch_img_smem(a.cols, mn));
    uint8_t *ring = reinterpret_cast<uint8_t *>(terms) + batch_term_smem(W, mn);
    const unsigned warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    // the CTA's work: rounds of its panels blockIdx.x, blockIdx.x + gridDim.x, ..., in order
    const unsigned my_panels = blockIdx.x < W.n_rt ? (W.n_rt - blockIdx.x + gridDim.x - 1) / gridDim.x : 0u;
    const unsigned items = my_panels * rounds;
    if (threadIdx.x == kPanelThreads) {
        for (unsigned s = 0; s < NS; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kPanelWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();
    if (warp == kPanelWarps) {
        // ---- producer: one bulk copy per round (its steps are consecutive tiles of the panel). The weights never
        // change within a list, so the first NS rounds are issued before the wait on the quantizer.
        if (lane != 0) return;
        const uint64_t pol = evict_first_policy();
        auto issue = [&](unsigned it) {
            const unsigned pnl = blockIdx.x + (it / rounds) * gridDim.x, k0 = (it % rounds) * kBatchChunk;
            const unsigned bytes = min(kBatchChunk, KC - k0) * W.tile_bytes;
            const unsigned s = it % NS;
            mbar_expect_tx(full + s, bytes);
            bulk_copy(ring + size_t(s) * a.stage_bytes, W.base + (size_t(pnl) * KC + k0) * W.tile_bytes, bytes,
                      full + s, pol);
        };
        unsigned it = 0;
        for (; it < items && it < NS; ++it) issue(it);
        pdl_wait();
        pdl_launch_dependents();
        bool ok = true;
        for (; it < items; ++it) {
            // stage it % NS was filled for item it - NS; its consumers release it once per use
            if (!mbar_wait(empty + it % NS, ((it / NS) - 1) & 1u)) {
                ok = false;
                break;
            }
            issue(it);
        }
        if (!ok) {
            if (a.err) atomicExch(a.err, 1u);
            // copies still in flight land before the CTA exits (bounded)
            for (unsigned j = it > NS ? it - NS : 0u; j < it; ++j) mbar_wait(full + j % NS, (j / NS) & 1u);
        }
        return;
    }
    // ---- consumers (warps 0..7): the rows' images, quantized once per CTA while the ring fills
    pdl_wait();
    pdl_launch_dependents();
    for (unsigned i = threadIdx.x; i < mn * nb; i += kPanelThreads) {
        const unsigned m = i / nb, b = i % nb;
        uint4 q0, q1, meta;
        batch_quant_block(a.x + size_t(a.m0 + m) * a.cols + size_t(b) * 32, a.act == 1, q0, q1, meta);
        uint4 *im = reinterpret_cast<uint4 *>(img + (size_t(m) * nb + b) * kBatchImgBlockBytes);
        im[0] = q0;
        im[1] = q1;
        im[2] = meta;
    }
    consumers_sync();
    // fold ownership: thread t < mn * P adds the terms of (activation row t / P, panel row t % P), in block order
    const bool owner = threadIdx.x < mn * P;
    const unsigned om = owner ? threadIdx.x / P : 0u, orow = threadIdx.x % P;
    const unsigned r_in = lane / C, b_in = lane % C;  // the lane's unit: panel row, block within the step
    float acc = 0.0f;
    bool failed = false;
    for (unsigned it = 0; it < items; ++it) {
        const unsigned pnl = blockIdx.x + (it / rounds) * gridDim.x, rd = it % rounds, k0 = rd * kBatchChunk;
        const unsigned s = it % NS;
        if (rd == 0) acc = 0.0f;
        const bool landed = mbar_wait(full + s, (it / NS) & 1u);
        float *tb = terms + size_t(it & 1u) * mn * rs;
        const uint8_t *stage = ring + size_t(s) * a.stage_bytes;
        if (landed) {
#pragma unroll
            for (unsigned u = 0; u < 2; ++u) {
                const unsigned j = warp + u * kPanelWarps;  // the step within the round
                const unsigned k = k0 + j;
                if (k >= KC) break;
                const uint8_t *tile = stage + size_t(j) * W.tile_bytes;
                Step<FMT> st;
                st.q0 = *reinterpret_cast<const uint4 *>(tile + lane * 16);
                if (FMT == 8) {
                    st.q1 = *reinterpret_cast<const uint4 *>(tile + 512 + lane * 16);
                    st.d = *reinterpret_cast<const uint16_t *>(tile + 1024 + lane * 2);
                } else if (FMT == 2) {
                    st.d = *reinterpret_cast<const uint16_t *>(tile + 512 + lane * 2);
                } else {
                    st.d = *reinterpret_cast<const uint32_t *>(tile + 512 + lane * 4);
                }
                const unsigned b = k * C + b_in;
                float *tslot = tb + (j * C + b_in) * P + r_in;
                if (b >= nb) {  // a padding unit past the row's last block: its term is never folded
                    continue;
                }
                // the unit's weight words, unpacked once for all rows (block_term's arithmetic, split)
                uint4 wl, wh;
                if (FMT == 8) {
                    wl = st.q0;
                    wh = st.q1;
                } else {
                    const uint32_t mk = 0x0F0F0F0Fu;
                    wl = make_uint4(st.q0.x & mk, st.q0.y & mk, st.q0.z & mk, st.q0.w & mk);
                    wh = make_uint4((st.q0.x >> 4) & mk, (st.q0.y >> 4) & mk, (st.q0.z >> 4) & mk, (st.q0.w >> 4) & mk);
                }
                const float dw = half_bits_to_float(uint16_t(st.d & 0xffffu));
                const float mw = FMT == 3 ? half_bits_to_float(uint16_t(st.d >> 16)) : 0.0f;
                const uint8_t *xb = img + size_t(b) * kBatchImgBlockBytes;
#pragma unroll
                for (unsigned m = 0; m < kBatchMax; ++m) {
                    if (m >= mn) break;
                    const uint8_t *xm = xb + size_t(m) * nb * kBatchImgBlockBytes;
                    const uint4 x0 = *reinterpret_cast<const uint4 *>(xm);
                    const uint4 x1 = *reinterpret_cast<const uint4 *>(xm + 16);
                    const uint4 meta = *reinterpret_cast<const uint4 *>(xm + 32);
                    int d0 = __dp4a(int(wl.x), int(x0.x), 0);
                    int d1 = __dp4a(int(wh.x), int(x1.x), 0);
                    d0 = __dp4a(int(wl.y), int(x0.y), d0);
                    d1 = __dp4a(int(wh.y), int(x1.y), d1);
                    d0 = __dp4a(int(wl.z), int(x0.z), d0);
                    d1 = __dp4a(int(wh.z), int(x1.z), d1);
                    d0 = __dp4a(int(wl.w), int(x0.w), d0);
                    d1 = __dp4a(int(wh.w), int(x1.w), d1);
                    const int sumi = d0 + d1 - (FMT == 2 ? 8 * int(meta.z) : 0);
                    const float xd = __uint_as_float(meta.x);
                    float t;
                    if (FMT == 3) t = fadd(fmul(fmul(dw, xd), float(sumi)), fmul(mw, __uint_as_float(meta.y)));
                    else t = fmul(float(sumi), fmul(dw, xd));
                    tslot[m * rs] = t;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + s);  // this warp has read the stage
        // one barrier (with a vote) per round: this round's terms before their fold; the buffer written above was
        // last read by the fold of round it - 2, which every consumer finished before the barrier of round it - 1
        if (consumers_any(!landed)) {
            failed = true;
            break;
        }
        if (owner) {
            const unsigned j1 = min(kBatchChunk * C, nb > k0 * C ? nb - k0 * C : 0u);
            const float *t = tb + om * rs + orow;
            for (unsigned j = 0; j < j1; ++j) acc = fadd(acc, t[j * P]);
            const unsigned row = pnl * P + orow;
            if (rd + 1 == rounds && row < W.rows) {
                float *y = a.y + size_t(a.m0 + om) * a.ystride + W.row0 + row;
                *y = a.add ? fadd(acc, *y) : acc;
            }
        }
    }
    if (failed) {
        if (threadIdx.x == 0 && a.err) atomicExch(a.err, 1u);
        return;
    }
    // zero padding of every output row up to a multiple of 16 floats (the GEMV's padding rule)
    if (blockIdx.x == 0) {
        const unsigned pad = a.ystride - W.rows;
        for (unsigned i = threadIdx.x; i < mn * pad; i += kPanelThreads)
            a.y[size_t(a.m0 + i / pad) * a.ystride + W.rows + i % pad] = 0.0f;
    }
}

static void (*batch_kernel_for(unsigned fmt))(BatchArgs) {
    switch (fmt) {
    case 2: return gemv_batch_kernel<2>;
    case 3: return gemv_batch_kernel<3>;
    case 8: return gemv_batch_kernel<8>;
    default: return nullptr;
    }
}

// Rows per launch: as many as leave room for a ring of at least two stages in one CTA's shared memory.
unsigned gemv_batch_rows_per_launch(const MatrixView &w, unsigned cols) {
    for (unsigned mn = kBatchMax; mn >= 1; --mn)
        if (batch_fixed_smem(w, cols, mn) + 2 * batch_stage_bytes(w) <= 227 * 1024) return mn;
    return 0;
}

cudaError_t launch_gemv_batch(const BatchArgs &args, unsigned sms, cudaStream_t st, bool pdl) {
    const auto k = batch_kernel_for(args.w.format);
    const unsigned per = gemv_batch_rows_per_launch(args.w, args.cols);
    if (!k || per == 0 || args.batch == 0 || args.batch > kBatchMax) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    const size_t stage = batch_stage_bytes(args.w);
    for (unsigned m0 = 0; m0 < args.batch; m0 += per) {
        BatchArgs a = args;
        a.m0 = m0;
        a.mn = std::min(per, args.batch - m0);
        a.stage_bytes = unsigned(stage);
        const size_t fixed = batch_fixed_smem(a.w, a.cols, a.mn);
        // two CTAs per SM when a ring of four stages still fits half the shared memory, else one with a deeper ring;
        // at most 16 stages (the mbarriers' room)
        const size_t half = 227 * 1024 / 2 - 1024;
        const unsigned per_sm = fixed + 4 * stage <= half ? 2u : 1u;
        const size_t budget = per_sm == 2 ? half : 227 * 1024;
        a.n_stages = unsigned(std::min<size_t>((budget - fixed) / stage, kBatchBarBytes / 16));
        const size_t smem = fixed + size_t(a.n_stages) * stage;
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(std::min(a.w.n_rt, sms * per_sm));
        cfg.blockDim = dim3(kBatchThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        e = cudaLaunchKernelEx(&cfg, k, a);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace b200q
