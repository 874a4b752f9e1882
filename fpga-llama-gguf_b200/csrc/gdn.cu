// Gated DeltaNet decode step (ggml GATED_DELTA_NET, one token, scalar gate, head size 128): the reference's GDN
// opcode (fpga/src/gemvqc16.cpp:801-904, gemvqc_gdn.h:74-346) with its CPU arithmetic (gemvq_ref.h:360-397):
// per value head h (key head h % H_k) and state row j (column j of S):
//   x = S_j * exp(g);  delta = (v_j - x . k) * beta;  S_j' = x + k * delta;  y_j = (S_j' . q) * scale
// optionally with q/k L2-normalized per head (RMSNORM with flags 3), the gates beta = sigmoid(beta),
// g = softplus(g + dt) * a, and the gated output (RMSNORM(y) * w) * silu(z) per head.
//
// One cluster of 4 CTAs per value head, 32 state rows per CTA, eight threads per state row: each thread holds a
// 16-float segment of its row in registers for the whole step (read once, written once). A row's dot products are
// summed as four 32-float quarters, each in index order — the even thread of a pair adds its 16 products, the odd
// thread continues from that sum with its own 16 — and the quarters are added as (q0 + q1) + (q2 + q3). (One thread
// per row, the CPU's fully sequential order, left a single warp per SM running ~1800 dependent instructions: ~8 us
// per step; the quarters held by four threads per row, 128 threads per CTA, gave the same sums with half the warps
// and loads in flight.) The result is within the reference's tolerance, not bit-exact. The per-head sums of squares (L2 of q and k, RMS of y)
// are four 32-value shuffle-tree sums added in row order, as the CPU oracle is checked against; each CTA forms the
// q / k sums itself and the y sum from the four CTAs' parts, exchanged through distributed shared memory. When the
// step's WITH_OUT GEMV follows, each CTA also quantizes its 32 outputs (one Q8_0 block) into that GEMV's x image.
#include "launch.h"
#include "peer.cuh"
#include "pipeline.cuh"
#include "quant.cuh"

namespace b200q {

constexpr unsigned kGdnSplit = 4;      // CTAs per head (one cluster), 32 state rows each
constexpr unsigned kGdnPerRow = 8;     // threads per state row
constexpr unsigned kGdnSeg = 128 / kGdnPerRow;  // floats of a row per thread
constexpr unsigned kGdnThreads = 32 * kGdnPerRow;

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// A row's sum from the products its eight threads hold (prod: this thread's 16, in index order): quarter t (32
// floats) is the in-order sum of threads 2t and 2t + 1 — the odd thread continues from the even thread's sum — and
// the row's sum is (q0 + q1) + (q2 + q3); every thread of the row gets the same bits.
__device__ __forceinline__ float row_sum(const float (&prod)[kGdnSeg], unsigned seg) {
    float acc = 0.0f;
    if ((seg & 1u) == 0) {
#pragma unroll
        for (int i = 0; i < int(kGdnSeg); ++i) acc = fadd(acc, prod[i]);
    }
    acc = __shfl_xor_sync(0xffffffffu, acc, 1);  // odd threads: the even thread's sum
    if (seg & 1u) {
#pragma unroll
        for (int i = 0; i < int(kGdnSeg); ++i) acc = fadd(acc, prod[i]);
    }
    // the quarters sit in the odd threads 1, 3, 5, 7 of the row's eight: q0 + q1 and q2 + q3, then their sum
    float qsum = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
    qsum = fadd(qsum, __shfl_xor_sync(0xffffffffu, qsum, 4));
    return __shfl_sync(0xffffffffu, qsum, (threadIdx.x % 32) | 1u);
}

__global__ void __cluster_dims__(kGdnSplit, 1, 1) __launch_bounds__(kGdnThreads) gdn_kernel(const GdnArgs a) {
    __shared__ __align__(16) float qs[128], ks[128];
    __shared__ float ycta[32], yout[32];
    __shared__ double red[4];
    __shared__ double ysum[kGdnSplit];  // part p of the head's sum of y^2, written by CTA p into every CTA
    __shared__ float gate[2];
    cluster_arrive_relaxed();
    pdl_wait();
    pdl_launch_dependents();  // the next kernel may stage its weights while this one runs
    peer_wait_rows_cta(a.pw);
    const unsigned part = cluster_rank(), h = blockIdx.x / kGdnSplit, kh = h % a.hk;
    const unsigned tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const unsigned rloc = tid / kGdnPerRow, seg = tid % kGdnPerRow, j = part * 32 + rloc;
    // this thread's segment of state row j: issue the loads first
    const float4 *src = reinterpret_cast<const float4 *>(a.state_in + (size_t(h) * 128 + j) * 128 + seg * kGdnSeg);
    float row[kGdnSeg];
#pragma unroll
    for (int i = 0; i < int(kGdnSeg / 4); ++i) {
        const float4 v = src[i];
        row[4 * i] = v.x;
        row[4 * i + 1] = v.y;
        row[4 * i + 2] = v.z;
        row[4 * i + 3] = v.w;
    }
    // threads 0..127 hold one value each of the head's q and k (warps 0..3)
    const bool qk = tid < 128;
    float qv = qk ? a.q[kh * 128 + tid] : 0.0f, kv = qk ? a.k[kh * 128 + tid] : 0.0f;
    // every other input of the step now, so no load waits in the middle of the dependent chain
    const float vj = a.v[h * 128 + j];
    const float zj = a.z ? a.z[h * 128 + j] : 0.0f, wj = a.z ? a.wn[j] : 0.0f;
    float g_in = 0.0f, b_in = 0.0f, dt_in = 0.0f, a_in = 0.0f;
    if (tid == 0) {
        g_in = a.g[h];
        b_in = a.beta[h];
        if (a.dt) {
            dt_in = a.dt[h];
            a_in = a.a[h];
        }
    }
    if (a.l2) {  // 1 / fmaxf(sqrtf(float(sum x^2)), eps), x * scale (gemvq_ref.h:309-324 with flags 3)
        const double sq = warp_sum_d(double(fmul(qv, qv))), sk = warp_sum_d(double(fmul(kv, kv)));
        if (lane == 0 && qk) red[warp] = sq;
        __syncthreads();
        const double tq = ((red[0] + red[1]) + red[2]) + red[3];
        __syncthreads();
        if (lane == 0 && qk) red[warp] = sk;
        __syncthreads();
        const double tk = ((red[0] + red[1]) + red[2]) + red[3];
        qv = fmul(qv, fdiv(1.0f, fmaxf(__fsqrt_rn(__double2float_rn(tq)), a.l2_eps)));
        kv = fmul(kv, fdiv(1.0f, fmaxf(__fsqrt_rn(__double2float_rn(tk)), a.l2_eps)));
    }
    if (qk) {
        qs[tid] = qv;
        ks[tid] = kv;
    }
    if (tid == 0) {
        float g = g_in, b = b_in;
        if (a.dt) {  // gemvqc_gdn.h:265-280: g = softplus(g + dt) * a, beta = sigmoid(beta)
            g = fmul(softplus_f32(fadd(g, dt_in)), a_in);
            b = sigmoid_f32(b);
        }
        gate[0] = exp_f32(g);
        gate[1] = b;
    }
    __syncthreads();
    const float decay = gate[0], beta = gate[1];
    float kseg[kGdnSeg];
#pragma unroll
    for (int i = 0; i < int(kGdnSeg / 4); ++i) {
        const float4 k4 = reinterpret_cast<const float4 *>(ks + seg * kGdnSeg)[i];
        kseg[4 * i] = k4.x;
        kseg[4 * i + 1] = k4.y;
        kseg[4 * i + 2] = k4.z;
        kseg[4 * i + 3] = k4.w;
    }
    float prod[kGdnSeg];
#pragma unroll
    for (int i = 0; i < int(kGdnSeg); ++i) {
        row[i] = fmul(row[i], decay);
        prod[i] = fmul(row[i], kseg[i]);
    }
    const float dot = row_sum(prod, seg);
    const float delta = fmul(fsub(vj, dot), beta);
#pragma unroll
    for (int i = 0; i < int(kGdnSeg); ++i) {
        row[i] = fadd(row[i], fmul(kseg[i], delta));
        prod[i] = fmul(row[i], qs[seg * kGdnSeg + i]);
    }
    const float out = row_sum(prod, seg);
    float4 *dst = reinterpret_cast<float4 *>(a.state_out + (size_t(h) * 128 + j) * 128 + seg * kGdnSeg);
#pragma unroll
    for (int i = 0; i < int(kGdnSeg / 4); ++i)
        dst[i] = make_float4(row[4 * i], row[4 * i + 1], row[4 * i + 2], row[4 * i + 3]);
    float yv = fmul(out, a.scale);
    cluster_wait();  // every CTA of the cluster has started: its shared memory may be written
    if (a.z) {  // (y * rms scale) * w, then silu(z) * that (RMSNORM + SILU_MUL, gemvqc_gdn.h:284-346)
        if (seg == 0) ycta[rloc] = yv;
        __syncthreads();
        if (warp == 0) {
            const double mine = warp_sum_d(double(fmul(ycta[lane], ycta[lane])));
            if (lane < kGdnSplit) st_cluster_f64(peer_smem(smem_addr(&ysum[part]), lane), mine);
        }
        cluster_sync();
        const double s = ((ysum[0] + ysum[1]) + ysum[2]) + ysum[3];
        const float sc = fdiv(1.0f, __fsqrt_rn(fadd(__double2float_rn(__ddiv_rn(s, 128.0)), a.rms_eps)));
        const float nv = fmul(fmul(yv, sc), wj);
        yv = fmul(silu_f32(zj), nv);
    }
    if (seg == 0) a.y[h * 128 + j] = yv;
    if (a.img) {  // this CTA's 32 rows are block 4 h + part of the next GEMV's x: its image block, as that pass would
        if (seg == 0) yout[rloc] = yv;
        __syncthreads();
        if (warp == 0) write_image_block(a.img, a.hv * 128, h * kGdnSplit + part, yout[lane], lane, a.img_act);
    }
}

cudaError_t launch_gdn(const GdnArgs &a, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.hv * kGdnSplit);
    cfg.blockDim = dim3(kGdnThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gdn_kernel, a);
}

}  // namespace b200q
