// Prefill GEMM: GEMV_BATCH commands of more than kBatchMax activation rows ("tokens"), Y = W X on the fifth-
// generation tensor cores (tcgen05, TMEM accumulators), every output with the bits of one GEMV per token.
//
// The reference's dot of a weight row with a quantized x (gemvq_ref.h:248-262) is, per 32-value block b, an exact
// integer sum sumi_b of weight quants times x quants, then the FP32 terms float(sumi_b) * (d_w * d_x) added in block
// order (Q4_1 x Q8_1: (d_w * d_x) * float(sumi_b) + m_w * s_x, gemvq_ref.h:194-229). One tcgen05.mma of kind::i8 with
// K = 32 is exactly one block for a tile of rows x tokens: D[row][token] = sumi_b in TMEM, as int32. The FP32 part
// (scales, products, the ordered sum) runs on the CUDA cores, so every output keeps the GEMV's bits. Q4_0 nibbles
// enter the MMA as q - 8 (sum of (q - 8) x = sum q x - 8 sum x, the GEMV's corrected sum), Q4_1 nibbles as they are.
//
// Launches: gemm_quantize_kernel writes the tokens' Q8_0 / Q8_1 image (kernel_args.h) once, with the GEMV
// quantizer's arithmetic; gemm_tc_kernel takes one tile of kGemmRows weight rows x kGemmTokens tokens per CTA
// (tiles of one row range adjacent, so they share the weights through L2), 8 warps, two TMEM slots of 128 int32
// columns (256 columns: two CTAs per SM). Per block b:
//   load    thread r < 128 copies weight row r's unit of block b out of the device layout (16 or 32 quant bytes and
//           the scale word), thread 128 + t token t's block out of the image (32 quant bytes, d, s), by cp.async
//           into its own slot of a ring of kGemmStages raw stages, kGemmStages - 1 blocks ahead;
//   expand  the same thread writes its row into the MMA's canonical K-major layout without swizzle (core matrices
//           of 8 rows x 16 bytes; K halves 128 bytes apart, 8-row groups 256 bytes apart) as int8, and its scales as
//           FP32, into canonical buffer b % 2; then fence.proxy.async (generic stores -> tensor-core reads);
//   mma     after a CTA barrier, thread 0 issues the MMA (M 128, N 128, K 32, s8 x s8 -> s32) into TMEM slot b % 2
//           and commits it to that slot's mbarrier;
//   fold    meanwhile every thread folds block b - 1: wait for its MMA, tcgen05.ld of the slot (32 columns at a
//           time), the FP32 terms added to its 64 running sums (thread = TMEM lane = weight row, warp / 4 = which
//           64 tokens); a second CTA barrier frees the slot and the canonical buffer for block b + 1.
// Bounds: the wait on an MMA is bounded (pipeline.cuh); when one runs out the CTA sets the error word, stores
// nothing and returns after freeing its TMEM. No cluster, no multicast, one GPU's memory.
#include <algorithm>

#include "common.cuh"
#include "kernel_args.h"
#include "launch.h"
#include "pipeline.cuh"
#include "quant.cuh"

namespace b200q {
namespace {

constexpr unsigned kGemmThreads = 256;
constexpr unsigned kGemmStages = 4;
constexpr unsigned kGemmRaw = 48;         // raw bytes per thread and stage: 16 + 16 quant bytes, two scale words
constexpr unsigned kGemmTmemCols = 2 * kGemmTokens;
// canonical buffer: A (weights, 128 x 32 int8) | B (tokens, 128 x 32 int8) | d_w | m_w | d_x | s_x (128 FP32 each)
constexpr unsigned kCanA = 0, kCanB = 4096, kCanDw = 8192, kCanMw = 8704, kCanDx = 9216, kCanSx = 9728;
constexpr unsigned kCanonBytes = 10240;
constexpr unsigned kRawBytes = kGemmStages * kGemmThreads * kGemmRaw;
constexpr unsigned kBarOff = kRawBytes + 2 * kCanonBytes;
constexpr unsigned kGemmSmem = kBarOff + 64;
static_assert(kGemmRows == 128 && kGemmTokens == 128, "the MMA shape and the thread mapping assume 128 x 128 tiles");
static_assert(kRawBytes % 1024 == 0 && kCanonBytes % 1024 == 0, "canonical buffers start on 1024-byte boundaries");

// Instruction descriptor of tcgen05.mma kind::i8: D s32 (bits 4-5 = 2), A and B signed 8-bit (bits 7-9, 10-12 = 1),
// both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((kGemmTokens >> 3) << 17) | ((kGemmRows >> 4) << 24);

// Shared-memory matrix descriptor of a 128 x 32-byte K-major operand without swizzle: start address >> 4 (bits
// 0-13), leading byte offset (between the two 16-byte K halves) 128 >> 4 (bits 16-29), stride byte offset (between
// 8-row groups) 256 >> 4 (bits 32-45), descriptor version 1 (bits 46-47), base offset 0, layout type 0 (bits 61-63).
__device__ __forceinline__ uint64_t operand_desc(uint32_t addr) {
    return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t(128u >> 4) << 16) | (uint64_t(256u >> 4) << 32) |
           (uint64_t(1) << 46);
}

__device__ __forceinline__ void tmem_alloc(uint32_t *dst, unsigned cols) {  // whole warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, unsigned cols) {  // whole warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D (TMEM) = A B^T for one 32-value block: A 128 weight rows, B 128 tokens, both 32 int8 per row.
__device__ __forceinline__ void mma_block(uint32_t d, uint64_t adesc, uint64_t bdesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(0u)
        : "memory");
}
// The mbarrier receives one arrival when every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 consecutive int32 columns of this warp's 32 TMEM lanes (lane i of the warp gets TMEM lane base + i), with the
// wait for the load in the same statement so that no use of v can be scheduled before it.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_ring() {
    asm volatile("cp.async.wait_group %0;" ::"n"(kGemmStages - 1) : "memory");
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// The 16 low (values 0..15) or high (values 16..31) nibbles of a Q4 block's 16 bytes as int8, minus 8 for Q4_0.
__device__ __forceinline__ uint4 nibbles(uint4 q, unsigned shift, bool minus8) {
    const uint32_t m = 0x0F0F0F0Fu;
    uint4 r = make_uint4((q.x >> shift) & m, (q.y >> shift) & m, (q.z >> shift) & m, (q.w >> shift) & m);
    if (minus8) r = make_uint4(__vsub4(r.x, 0x08080808u), __vsub4(r.y, 0x08080808u), __vsub4(r.z, 0x08080808u),
                               __vsub4(r.w, 0x08080808u));
    return r;
}

// One thread per (token, block) of the image: the GEMV quantizer's block arithmetic (batch_quant_block); tokens past
// `tokens` get zero quants and scales.
__global__ void __launch_bounds__(256) gemm_quantize_kernel(const GemmArgs a) {
    pdl_wait();
    pdl_launch_dependents();
    const unsigned nb = a.cols / 32;
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(nb) * a.tpad) return;
    const unsigned t = unsigned(i % a.tpad), b = unsigned(i / a.tpad);
    uint4 q0 = make_uint4(0u, 0u, 0u, 0u), q1 = q0, meta = q0;
    if (t < a.tokens) batch_quant_block(a.x + size_t(t) * a.cols + size_t(b) * 32, a.act == 1, q0, q1, meta);
    uint4 *q = reinterpret_cast<uint4 *>(a.xq + i * 32);
    q[0] = q0;
    q[1] = q1;
    a.xd[i] = __uint_as_float(meta.x);
    a.xs[i] = __uint_as_float(meta.y);
}

template <unsigned FMT>
__global__ void __launch_bounds__(kGemmThreads, 2) gemm_tc_kernel(const GemmArgs a) {
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t *mma_bar = reinterpret_cast<uint64_t *>(smem + kBarOff);
    uint32_t *tmem_base = reinterpret_cast<uint32_t *>(smem + kBarOff + 16);
    const unsigned tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const MatrixView &W = a.w;
    const unsigned nb = a.cols / 32, n_tt = a.tpad / kGemmTokens;
    const unsigned m0 = (blockIdx.x / n_tt) * kGemmRows, t0 = (blockIdx.x % n_tt) * kGemmTokens;

    if (warp == 0) {
        tmem_alloc(tmem_base, kGemmTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(mma_bar, 1);
        mbar_init(mma_bar + 1, 1);
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_base;

    // the loads of this thread: weight row m0 + tid (tid < 128) or token t0 + tid - 128
    const bool wt = tid < kGemmRows;
    const unsigned r = tid & (kGemmRows - 1u);
    const unsigned grow = m0 + r, P = W.rt, C = W.ct;
    const unsigned pnl = grow / P, rr = grow % P;
    const bool have = wt ? pnl < W.n_rt : true;  // rows of a panel past the matrix are zero in the layout
    constexpr unsigned DB = FMT == 3 ? 4u : 2u;
    const uint32_t raw0 = smem_addr(smem) + tid * kGemmRaw;
    auto issue = [&](unsigned b) {  // block b into raw stage b % kGemmStages (an empty group past the last block)
        const uint32_t dst = raw0 + (b % kGemmStages) * (kGemmThreads * kGemmRaw);
        if (b < nb && have) {
            if (wt) {
                const unsigned u = rr * C + b % C;
                const uint8_t *tile = W.base + (size_t(pnl) * W.kc + b / C) * W.tile_bytes;
                cp_async16(dst, tile + u * 16);
                if (FMT == 8) cp_async16(dst + 16, tile + 512 + u * 16);
                cp_async4(dst + 32, tile + W.qs_part + ((u * DB) & ~3u));
            } else {
                const size_t i = size_t(b) * a.tpad + t0 + r;
                cp_async16(dst, a.xq + i * 32);
                cp_async16(dst + 16, a.xq + i * 32 + 16);
                cp_async4(dst + 32, a.xd + i);
                if (FMT == 3) cp_async4(dst + 36, a.xs + i);
            }
        }
        cp_async_commit();
    };
    auto expand = [&](unsigned b) {  // raw stage of block b -> canonical buffer b % 2
        const uint32_t src = raw0 + (b % kGemmStages) * (kGemmThreads * kGemmRaw);
        const uint32_t cb = smem_addr(smem + kRawBytes + (b & 1u) * kCanonBytes);
        uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
        float s0 = 0.0f, s1 = 0.0f;
        if (have) {
            const uint4 q0 = lds128(src);
            const uint32_t sw = lds32(src + 32);
            if (wt) {
                const unsigned u = rr * C + b % C;
                const uint16_t dbits = FMT == 3 ? uint16_t(sw & 0xffffu) : uint16_t((u & 1u) ? sw >> 16 : sw & 0xffffu);
                s0 = half_bits_to_float(dbits);
                if (FMT == 3) s1 = half_bits_to_float(uint16_t(sw >> 16));
                if (FMT == 8) {
                    lo = q0;
                    hi = lds128(src + 16);
                } else {
                    lo = nibbles(q0, 0, FMT == 2);
                    hi = nibbles(q0, 4, FMT == 2);
                }
            } else {
                lo = q0;
                hi = lds128(src + 16);
                s0 = __uint_as_float(sw);
                if (FMT == 3) s1 = ldsf(src + 36);
            }
        }
        const uint32_t op = cb + (wt ? kCanA : kCanB) + (r >> 3) * 256 + (r & 7u) * 16;
        sts128(op, lo);
        sts128(op + 128, hi);
        stsf(cb + (wt ? kCanDw : kCanDx) + r * 4, s0);
        stsf(cb + (wt ? kCanMw : kCanSx) + r * 4, s1);
    };

    // epilogue mapping: TMEM lane (= weight row) q * 32 + lane, tokens h * 64 .. h * 64 + 63 of the tile
    const unsigned q = warp & 3u, h = warp >> 2, row = q * 32 + lane;
    float acc[64];
#pragma unroll
    for (unsigned j = 0; j < 64; ++j) acc[j] = 0.0f;
    auto fold = [&](unsigned b) -> bool {
        if (!mbar_wait(mma_bar + (b & 1u), (b >> 1) & 1u)) return false;
        tc_fence_after();
        const unsigned char *cb = smem + kRawBytes + (b & 1u) * kCanonBytes;
        const float dw = reinterpret_cast<const float *>(cb + kCanDw)[row];
        const float mw = FMT == 3 ? reinterpret_cast<const float *>(cb + kCanMw)[row] : 0.0f;
        const float *dx = reinterpret_cast<const float *>(cb + kCanDx) + h * 64;
        const float *sx = reinterpret_cast<const float *>(cb + kCanSx) + h * 64;
#pragma unroll
        for (unsigned ch = 0; ch < 2; ++ch) {
            if (t0 + h * 64 + ch * 32 >= a.tokens) continue;  // warp-uniform: no token of this chunk
            uint32_t v[32];
            tmem_load32(tmem + ((q * 32u) << 16) + (b & 1u) * kGemmTokens + h * 64 + ch * 32, v);
            if (a.sums && b == 0 && blockIdx.x == 0) {
#pragma unroll
                for (unsigned j = 0; j < 32; ++j) a.sums[row * kGemmTokens + h * 64 + ch * 32 + j] = int32_t(v[j]);
            }
#pragma unroll
            for (unsigned j = 0; j < 32; j += 4) {
                const float4 d4 = *reinterpret_cast<const float4 *>(dx + ch * 32 + j);
                const float xd[4] = {d4.x, d4.y, d4.z, d4.w};
                float xs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (FMT == 3) {
                    const float4 s4 = *reinterpret_cast<const float4 *>(sx + ch * 32 + j);
                    xs[0] = s4.x;
                    xs[1] = s4.y;
                    xs[2] = s4.z;
                    xs[3] = s4.w;
                }
#pragma unroll
                for (unsigned e = 0; e < 4; ++e) {
                    const float si = __int2float_rn(int(v[j + e]));
                    float t;
                    if (FMT == 3) t = fadd(fmul(fmul(dw, xd[e]), si), fmul(mw, xs[e]));
                    else t = fmul(si, fmul(dw, xd[e]));
                    acc[ch * 32 + j + e] = fadd(acc[ch * 32 + j + e], t);
                }
            }
        }
        return true;
    };

    // weights never change within a list: their first copies go out before the wait on the previous kernel
    if (wt)
        for (unsigned b = 0; b + 1 < kGemmStages; ++b) issue(b);
    pdl_wait();
    if (!wt)
        for (unsigned b = 0; b + 1 < kGemmStages; ++b) issue(b);

    bool failed = false;
    for (unsigned b = 0; b < nb; ++b) {
        issue(b + kGemmStages - 1);
        cp_async_wait_ring();  // this thread's copies of block b have landed
        expand(b);
        fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t cb = smem_addr(smem + kRawBytes + (b & 1u) * kCanonBytes);
            mma_block(tmem + (b & 1u) * kGemmTokens, operand_desc(cb + kCanA), operand_desc(cb + kCanB));
            mma_commit(mma_bar + (b & 1u));
        }
        const bool ok = b == 0 || fold(b - 1);
        tc_fence_before();
        if (__syncthreads_or(!ok)) {
            failed = true;
            break;
        }
    }
    if (!failed && nb > 0) failed = __syncthreads_or(!fold(nb - 1));
    asm volatile("cp.async.wait_all;" ::: "memory");

    if (failed) {
        if (tid == 0 && a.err) atomicExch(a.err, 1u);
    } else {
        const unsigned gr = m0 + row;
#pragma unroll
        for (unsigned j = 0; j < 64; ++j) {
            const unsigned tok = t0 + h * 64 + j;
            if (tok >= a.tokens) continue;
            float *yt = a.y + size_t(tok) * a.ystride;
            if (gr < W.rows) {
                float *y = yt + W.row0 + gr;
                *y = a.add ? fadd(acc[j], *y) : acc[j];
            } else if (gr < a.ystride) {
                yt[gr] = 0.0f;  // zero padding up to a multiple of 16 floats (the GEMV's rule)
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kGemmTmemCols);
    }
}

void (*gemm_kernel_for(unsigned fmt))(GemmArgs) {
    switch (fmt) {
    case 2: return gemm_tc_kernel<2>;
    case 3: return gemm_tc_kernel<3>;
    case 8: return gemm_tc_kernel<8>;
    default: return nullptr;
    }
}

}  // namespace

size_t gemm_image_bytes(unsigned cols, unsigned tokens) {
    const size_t tpad = (size_t(tokens) + kGemmTokens - 1) / kGemmTokens * kGemmTokens;
    return size_t(cols / 32) * tpad * (32 + 2 * sizeof(float));
}

cudaError_t launch_gemm(GemmArgs a, cudaStream_t st, bool pdl) {
    const auto k = gemm_kernel_for(a.w.format);
    if (!k || a.tokens == 0 || a.cols == 0 || a.cols % 32 || !a.xq) return cudaErrorInvalidValue;
    a.tpad = (a.tokens + kGemmTokens - 1) / kGemmTokens * kGemmTokens;
    const size_t nbt = size_t(a.cols / 32) * a.tpad;
    a.xd = reinterpret_cast<float *>(a.xq + nbt * 32);
    a.xs = a.xd + nbt;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned((nbt + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_quantize_kernel, a);
    if (e != cudaSuccess) return e;
    if ((e = ensure_smem_attr(reinterpret_cast<const void *>(k), int(kGemmSmem))) != cudaSuccess) return e;
    const unsigned row_tiles = (a.w.rows + kGemmRows - 1) / kGemmRows;
    cfg.gridDim = dim3(row_tiles * (a.tpad / kGemmTokens));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = kGemmSmem;
    // with PDL the GEMM's prologue (TMEM, barriers, first weight copies) overlaps the quantizer
    return cudaLaunchKernelEx(&cfg, k, a);
}

}  // namespace b200q
