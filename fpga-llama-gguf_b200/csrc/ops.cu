// Element-wise commands of the reference ISA and the extension opcodes, one kernel each:
//   RMSNORM (fpga/src/gemvqc_ops.h:169-234, CPU gemvq_ref.h:309-324), ADD/MUL (:314-336), SILU_MUL (:338-361),
//   UNARY (:363-385), CONV (:387-431, CPU gemvq_ref.h:344-358), ROPE (:275-312), ARGMAX, GET_ROW.
// All FP32 arithmetic uses the _rn intrinsics in the CPU reference's operation order, so results match the CPU
// bit for bit except where exp/log are involved (see common.cuh). Bandwidth-bound and tiny (<= 65536 floats).
#include "launch.h"
#include "peer.cuh"
#include "quant.cuh"

namespace b200q {

// ---- RMSNORM rows: one CTA per row --------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *x, const float *w, float *y, unsigned n,
                                                       unsigned stride, float eps, unsigned flags, const PeerWait pw) {
    __shared__ double red[32];
    __shared__ float scale_s;
    pdl_wait();
    pdl_launch_dependents();  // the next kernel may stage its weights while this one runs
    peer_wait_rows_cta(pw);
    const float *xr = x + size_t(blockIdx.x) * stride;
    float *yr = y + size_t(blockIdx.x) * n;
    const float s = cta_norm_scale(xr, n, eps, flags & 1u, red, &scale_s);
    for (unsigned i = threadIdx.x; i < n; i += blockDim.x) {
        const float t = fmul(xr[i], s);
        yr[i] = (flags & 2u) ? t : fmul(t, w[i]);
    }
}

// ---- ADD / MUL / SILU_MUL / UNARY ---------------------------------------------------------------------------------
__global__ void ew_kernel(const EwArgs a) {
    pdl_wait();
    pdl_launch_dependents();  // the next kernel may stage its weights while this one runs
    peer_wait_rows_cta(a.pw);
    for (unsigned e = blockIdx.x * blockDim.x + threadIdx.x; e < a.n; e += gridDim.x * blockDim.x) {
        const size_t ai = a.row ? size_t(e / a.row) * a.stride + e % a.row : e;
        const float av = a.a[ai];
        float r;
        switch (a.op) {
        case 3: r = fadd(av, a.b[e]); break;
        case 5: r = fmul(av, a.b[e]); break;
        case 4: r = a.sigmoid ? fmul(sigmoid_f32(av), a.b[e]) : fmul(silu_f32(av), a.b[e]); break;
        default:
            r = a.kind == 1 ? silu_f32(av) : a.kind == 2 ? sigmoid_f32(av) : a.kind == 3 ? softplus_f32(av) : av;
            break;
        }
        a.y[e] = r;
    }
}

// ---- CONV (ggml_ssm_conv, one token, d_conv 4) --------------------------------------------------------------------
__global__ void conv_kernel(const float *x, const float *w, float *y, const float *s_src, float *s_dst, unsigned ch,
                            unsigned use_silu, const PeerWait pw) {
    pdl_wait();
    pdl_launch_dependents();  // the next kernel may stage its weights while this one runs
    peer_wait_rows_cta(pw);
    const unsigned c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= ch) return;
    const float s0 = s_src[3 * c], s1 = s_src[3 * c + 1], s2 = s_src[3 * c + 2], xv = x[c];
    float sum = 0.0f;
    sum = fadd(sum, fmul(s0, w[4 * c]));
    sum = fadd(sum, fmul(s1, w[4 * c + 1]));
    sum = fadd(sum, fmul(s2, w[4 * c + 2]));
    sum = fadd(sum, fmul(xv, w[4 * c + 3]));
    y[c] = use_silu ? silu_f32(sum) : sum;
    s_dst[3 * c] = s1;
    s_dst[3 * c + 1] = s2;
    s_dst[3 * c + 2] = xv;
}

// ---- ROPE, NEOX pairing --------------------------------------------------------------------------------------------
__global__ void rope_kernel(const float *x, const float *cs, float *y, unsigned n_dims, unsigned ne0, unsigned rows,
                            const PeerWait pw) {
    pdl_wait();
    pdl_launch_dependents();  // the next kernel may stage its weights while this one runs
    peer_wait_rows_cta(pw);
    const unsigned half = n_dims / 2;
    const unsigned per_row = half + (ne0 - n_dims);
    for (unsigned t = blockIdx.x * blockDim.x + threadIdx.x; t < rows * per_row; t += gridDim.x * blockDim.x) {
        const unsigned r = t / per_row, i = t % per_row;
        const float *xr = x + size_t(r) * ne0;
        float *yr = y + size_t(r) * ne0;
        if (i < half) {
            const float x0 = xr[i], x1 = xr[i + half], c = cs[2 * i], s = cs[2 * i + 1];
            const float a = fsub(fmul(x0, c), fmul(x1, s));
            const float b = fadd(fmul(x0, s), fmul(x1, c));
            yr[i] = a;
            yr[i + half] = b;
        } else {
            const unsigned k = n_dims + (i - half);
            yr[k] = xr[k];
        }
    }
}

// ---- ARGMAX (extension): first index of the maximum ---------------------------------------------------------------
// Order-preserving key of a float (NaN lowest, so it never wins) packed with the complement of the index: the
// largest packed value is the largest value at its first index.
__device__ __forceinline__ unsigned long long argmax_key(float v, unsigned i) {
    const unsigned u = v == 0.0f ? 0u : __float_as_uint(v);  // -0 and +0 compare equal
    const unsigned key = isnan(v) ? 0u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
    return (static_cast<unsigned long long>(key) << 32) | (0xffffffffu - i);
}

// Each CTA reduces a strided share of x to one packed key and folds it into the combine slot with a 64-bit
// atomicMax; the last CTA to finish (counter) writes the result and clears slot and counter for the next launch.
// Like a scalar scan with `>` from index 0: a NaN at index 0 keeps index 0, other NaNs are skipped.
__global__ void __launch_bounds__(256) argmax_kernel(const float *x, unsigned n, float *y, unsigned long long *slot,
                                                     unsigned *counter, const PeerWait pw) {
    __shared__ unsigned long long red[8];
    __shared__ bool last_s;
    pdl_wait();
    pdl_launch_dependents();  // the next kernel may stage its weights while this one runs
    peer_wait_rows_cta(pw);
    unsigned long long best = 0;
    const unsigned n4 = n / 4, stride = gridDim.x * blockDim.x;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 v = __ldg(x4 + i);
        best = max(best, argmax_key(v.x, 4 * i));
        best = max(best, argmax_key(v.y, 4 * i + 1));
        best = max(best, argmax_key(v.z, 4 * i + 2));
        best = max(best, argmax_key(v.w, 4 * i + 3));
    }
    for (unsigned i = 4 * n4 + blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        best = max(best, argmax_key(x[i], i));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (unsigned w = 1; w < blockDim.x / 32; ++w) best = max(best, red[w]);
        atomicMax(slot, best);
        __threadfence();
        last_s = atomicAdd(counter, 1u) == gridDim.x - 1;
        if (last_s) {
            __threadfence();
            const unsigned long long r = atomicExch(slot, 0ull);
            *counter = 0;
            unsigned idx = 0xffffffffu - unsigned(r & 0xffffffffu);
            if (isnan(x[0]) || r == 0) idx = 0;  // NaN first (or every value NaN): index 0, as the scan keeps it
            const float v = x[idx];
            y[0] = __uint_as_float(idx);
            y[1] = v;
        }
    }
}

// ---- GET_ROW (extension): one dequantized row, index read from act (ggml dequantize_row_q4_0 / q8_0) -------------
__global__ void get_row_kernel(const MatrixView w, unsigned cols, const float *idx_f, float *y, unsigned *status,
                               const PeerWait pw) {
    pdl_wait();
    pdl_launch_dependents();  // the next kernel may stage its weights while this one runs
    peer_wait_rows_cta(pw);
    const unsigned row = __float_as_uint(*idx_f);
    if (row < w.row0 || row >= w.row0 + w.rows) {
        if (blockIdx.x == 0 && threadIdx.x == 0 && status) atomicExch(status, 1u);
        return;
    }
    const unsigned r = row - w.row0;
    for (unsigned e = blockIdx.x * blockDim.x + threadIdx.x; e < cols; e += gridDim.x * blockDim.x) {
        const unsigned b = e / 32, j = e % 32;
        // panel layout: tile (r / P, b / C), unit (r % P) * C + b % C; 16 quant bytes per unit (Q8_0: two
        // halves 512 bytes apart), then the 32 FP16 scales
        const uint8_t *tile = w.base + (size_t(r / w.rt) * w.kc + b / w.ct) * w.tile_bytes;
        const unsigned i = (r % w.rt) * w.ct + b % w.ct;
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(tile + w.qs_part + i * 2));
        int q;
        if (w.format == 2) {
            const uint8_t byte = tile[i * 16 + (j & 15)];
            q = int(j < 16 ? (byte & 0xF) : (byte >> 4)) - 8;
        } else {
            q = int(int8_t(tile[(j / 16) * 512 + i * 16 + (j & 15)]));
        }
        y[e] = fmul(float(q), d);
    }
}

// ---- RMSNORM / ROPE runs in one launch (same arithmetic as rmsnorm_kernel and rope_kernel) ------------------------
__global__ void __launch_bounds__(256) rowops_kernel(const RowOpsArgs a) {
    __shared__ double red[32];
    __shared__ float scale_s;
    pdl_wait();
    pdl_launch_dependents();  // the next kernel may stage its weights while this one runs
    peer_wait_rows_cta(a.pw);
    unsigned j = 0;
    while (j + 1 < a.n_jobs && a.job[j + 1].row0 <= blockIdx.x) ++j;
    const RowJobArgs &J = a.job[j];
    const unsigned r = blockIdx.x - J.row0;
    if (J.norm) {
        const float *xr = J.x + size_t(r) * J.xstride;
        float *yr = J.y + size_t(r) * J.n;
        const float s = cta_norm_scale(xr, J.n, J.eps, J.flags & 1u, red, &scale_s);
        for (unsigned i = threadIdx.x; i < J.n; i += blockDim.x) {
            const float t = fmul(xr[i], s);
            yr[i] = (J.flags & 2u) ? t : fmul(t, J.w[i]);
        }
        __syncthreads();
    }
    if (J.nd) {
        const float *xr = J.rx + size_t(r) * J.ne0;
        float *yr = J.ry + size_t(r) * J.ne0;
        const unsigned half = J.nd / 2, per_row = half + (J.ne0 - J.nd);
        for (unsigned i = threadIdx.x; i < per_row; i += blockDim.x) {
            if (i < half) {
                const float x0 = xr[i], x1 = xr[i + half], c = J.cs[2 * i], sn = J.cs[2 * i + 1];
                const float va = fsub(fmul(x0, c), fmul(x1, sn));
                const float vb = fadd(fmul(x0, sn), fmul(x1, c));
                yr[i] = va;
                yr[i + half] = vb;
            } else {
                const unsigned k = J.nd + (i - half);
                yr[k] = xr[k];
            }
        }
    }
}

// ---- row-sharded passes: the wait for the peers' rows as a kernel of its own ----------------------------------------
// (before a copy or a host read of act that no kernel in between covers)
__global__ void peer_wait_kernel(const PeerWait pw) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0) peer_wait_rows(pw);
}

// ---- launchers ------------------------------------------------------------------------------------------------------
static cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                                   cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

cudaError_t launch_rmsnorm(const float *x, const float *w, float *y, unsigned n, unsigned rows, unsigned stride,
                           float eps, unsigned flags, const PeerWait &pw, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(rows), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, rmsnorm_kernel, x, w, y, n, stride, eps, flags, pw);
}

cudaError_t launch_ew(const EwArgs &a, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute attr[1];
    const unsigned grid = (a.n + 255) / 256 < 296 ? (a.n + 255) / 256 : 296;
    cudaLaunchConfig_t cfg = make_cfg(dim3(grid), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, ew_kernel, a);
}

cudaError_t launch_conv(const float *x, const float *w, float *y, const float *s_src, float *s_dst, unsigned ch,
                        unsigned use_silu, const PeerWait &pw, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3((ch + 127) / 128), dim3(128), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, conv_kernel, x, w, y, s_src, s_dst, ch, use_silu, pw);
}

cudaError_t launch_rope(const float *x, const float *cs, float *y, unsigned n_dims, unsigned ne0, unsigned rows,
                        const PeerWait &pw, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute attr[1];
    const unsigned work = rows * (n_dims / 2 + ne0 - n_dims);
    const unsigned grid = (work + 255) / 256 < 148 ? (work + 255) / 256 : 148;
    cudaLaunchConfig_t cfg = make_cfg(dim3(grid), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, rope_kernel, x, cs, y, n_dims, ne0, rows, pw);
}

cudaError_t launch_argmax(const float *x, unsigned n, float *y, unsigned long long *slot, unsigned *counter,
                          const PeerWait &pw, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute attr[1];
    const unsigned per_cta = 256 * 4 * 4;  // about four float4 per thread
    unsigned grid = (n + per_cta - 1) / per_cta;
    grid = grid < 1 ? 1 : (grid > 148 ? 148 : grid);
    cudaLaunchConfig_t cfg = make_cfg(dim3(grid), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, argmax_kernel, x, n, y, slot, counter, pw);
}

cudaError_t launch_get_row(const MatrixView &w, unsigned cols, const float *idx, float *y, unsigned *status,
                           const PeerWait &pw, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3((cols + 255) / 256), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, get_row_kernel, w, cols, idx, y, status, pw);
}

cudaError_t launch_peer_wait(const PeerWait &pw, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(32), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, peer_wait_kernel, pw);
}

cudaError_t launch_rowops(const RowOpsArgs &a, cudaStream_t st, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(a.total_rows), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, rowops_kernel, a);
}

}  // namespace b200q
