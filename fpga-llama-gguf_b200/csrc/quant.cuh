// Activation quantizers of the GEMV passes, CTA-cooperative, with the deferred RMSNORM fused in front.
//
// Bit-exact restatements of the reference's CPU arithmetic:
//   Q8_0 (gemvq_ref.h:239-245): per 32 values amax, s = amax / 127, id = s ? 1 / s : 0, d = fp16(s),
//        q = roundf(x * id) (half away from zero);
//   Q8_1 (gemvq_ref.h:196-212): as Q8_0 plus s8 = fp16(sum(q) * d) with the unrounded d;
//   Q8_K (gemvq_ref.h:62-81): per 256 values the value of largest magnitude, the first one on ties, gives
//        iscale = -127 / max, q = min(127, rne(iscale * x)), d = 1 / iscale;
//   RMSNORM (gemvq_ref.h:309-324): squares in FP32, their sum in FP64, RMS scale = 1 / sqrtf(float(sum / n) + eps)
//        or L2 scale = 1 / fmaxf(sqrtf(float(sum)), eps), value = (x * scale) * w.
// The FP64 sum is reduced in a fixed tree instead of the CPU's left-to-right order; both round to the same FP32
// mean unless the exact sum lies within ~1e-13 (relative) of an FP32 rounding boundary.
#pragma once
#include "common.cuh"

namespace b200q {

constexpr unsigned kMaxQuantCols = 16384;

// Shared-memory image of a quantized x, carved from dynamic shared memory for `cols` values.
struct XImage {
    int8_t *q;      // cols int8
    float *d;       // Q8_0/Q8_1: d (FP16-rounded) per 32-block; Q8_K: d per 256
    float *s;       // Q8_1: s per 32-block
    int32_t *b;     // Q8_0/Q8_1: sum of q per 32-block; Q8_K: sums of 16
    double *red;    // 32 partial sums
    float *scale;   // the norm scale
};

__host__ __device__ constexpr size_t ximage_bytes(unsigned cols) {
    return size_t(cols) + 4 * size_t(cols / 32) * 2 + 4 * size_t(cols / 16) + 32 * 8 + 16;
}

__device__ __forceinline__ XImage carve_ximage(unsigned char *p, unsigned cols) {
    XImage X;
    X.red = reinterpret_cast<double *>(p);
    p += 32 * 8;
    X.scale = reinterpret_cast<float *>(p);
    p += 16;
    X.q = reinterpret_cast<int8_t *>(p);
    p += cols;
    X.d = reinterpret_cast<float *>(p);
    p += 4 * (cols / 32);
    X.s = reinterpret_cast<float *>(p);
    p += 4 * (cols / 32);
    X.b = reinterpret_cast<int32_t *>(p);
    return X;
}

// Norm scale of x[0..n) by the RMSNORM arithmetic; every thread of the CTA gets it.
__device__ __forceinline__ float cta_norm_scale(const float *x, unsigned n, float eps, unsigned l2, double *red,
                                                float *out) {
    double acc = 0.0;
    for (unsigned i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        acc += double(fmul(v, v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    const unsigned warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = (blockDim.x + 31) / 32;
    __syncthreads();
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double sum = 0.0;
        for (unsigned w = 0; w < nw; ++w) sum += red[w];
        float scale;
        if (l2) scale = fdiv(1.0f, fmaxf(__fsqrt_rn(__double2float_rn(sum)), eps));
        else scale = fdiv(1.0f, __fsqrt_rn(fadd(__double2float_rn(__ddiv_rn(sum, double(n))), eps)));
        *out = scale;
    }
    __syncthreads();
    return *out;
}

// The value the quantizer sees at index i: x, or the deferred norm's (x * scale) * w / x * scale.
__device__ __forceinline__ float norm_value(const float *x, unsigned i, bool norm, float scale, const float *w,
                                            bool weighted) {
    const float v = x[i];
    if (!norm) return v;
    const float t = fmul(v, scale);
    return weighted ? fmul(t, w[i]) : t;
}

// Q8_0 / Q8_1 block b of the (normalized) x into the image.
__device__ __forceinline__ void quant_block_q80(const float *x, unsigned b, bool norm, float scale, const float *w,
                                                bool weighted, bool q81, const XImage &X) {
    float amax = 0.0f;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(norm_value(x, b * 32 + j, norm, scale, w, weighted)));
    const float s = fdiv(amax, 127.0f);
    const float id = s != 0.0f ? fdiv(1.0f, s) : 0.0f;
    int sum = 0;
    uint32_t *dst = reinterpret_cast<uint32_t *>(X.q + b * 32);
#pragma unroll 2
    for (int k = 0; k < 8; ++k) {
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int q = int(roundf(fmul(norm_value(x, b * 32 + k * 4 + e, norm, scale, w, weighted), id)));
            sum += q;
            word |= uint32_t(q & 0xff) << (8 * e);
        }
        dst[k] = word;
    }
    X.d[b] = half_bits_to_float(float_to_half_bits(s));
    X.b[b] = sum;
    if (q81) X.s[b] = half_bits_to_float(float_to_half_bits(fmul(float(sum), s)));
}

// Q8_K super-block sb (256 values) by one warp.
__device__ __forceinline__ void quant_superblock_q8k(const float *x, unsigned sb, bool norm, float scale,
                                                     const float *w, bool weighted, const XImage &X) {
    const unsigned lane = threadIdx.x % 32;
    float v[8];
    float amax = 0.0f;
    int idx = 0x7fffffff;
    float mx = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        v[j] = norm_value(x, sb * 256 + lane * 8 + j, norm, scale, w, weighted);
        const float a = fabsf(v[j]);
        if (a > amax) { amax = a; mx = v[j]; idx = int(lane * 8 + j); }
    }
    // first index of the largest magnitude
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const float om = __shfl_xor_sync(0xffffffffu, mx, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (oa > amax || (oa == amax && oi < idx)) { amax = oa; mx = om; idx = oi; }
    }
    uint32_t lo = 0, hi = 0;
    int s0 = 0, s1 = 0;
    if (amax != 0.0f) {
        const float iscale = fdiv(-127.0f, mx);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int q = __float2int_rn(fmul(iscale, v[j]));
            q = q < 127 ? q : 127;
            if (j < 4) { lo |= uint32_t(q & 0xff) << (8 * j); s0 += q; }
            else { hi |= uint32_t(q & 0xff) << (8 * (j - 4)); s1 += q; }
        }
        if (lane == 0) X.d[sb] = fdiv(1.0f, iscale);
    } else if (lane == 0) {
        X.d[sb] = 0.0f;
    }
    reinterpret_cast<uint2 *>(X.q + sb * 256)[lane] = make_uint2(lo, hi);
    // sums of 16: lanes 2g and 2g+1 hold group g
    int part = s0 + s1;
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    if ((lane & 1) == 0) X.b[sb * 16 + lane / 2] = part;
}

// The whole x quantized into X by the CTA. act: 0 Q8_0, 1 Q8_1, 2 Q8_K. Ends with __syncthreads().
__device__ __forceinline__ void quantize_cta(const float *x, unsigned n, unsigned act, const float *norm_w,
                                             float norm_eps, unsigned norm_mode, const XImage &X) {
    const bool norm = (norm_mode & 8u) != 0;
    const bool weighted = (norm_mode & 2u) == 0;
    float scale = 1.0f;
    if (norm) scale = cta_norm_scale(x, n, norm_eps, norm_mode & 1u, X.red, X.scale);
    if (act == 2) {
        const unsigned warp = threadIdx.x / 32, nw = blockDim.x / 32;
        for (unsigned sb = warp; sb < n / 256; sb += nw) quant_superblock_q8k(x, sb, norm, scale, norm_w, weighted, X);
    } else {
        for (unsigned b = threadIdx.x; b < n / 32; b += blockDim.x)
            quant_block_q80(x, b, norm, scale, norm_w, weighted, act == 1, X);
    }
    __syncthreads();
}

// Copy of a pre-quantized x (scratch) into X.
__device__ __forceinline__ void load_quant_cta(const int8_t *q, const float *d, const float *s, const int32_t *b,
                                               unsigned n, unsigned act, const XImage &X) {
    for (unsigned i = threadIdx.x; i < n / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(X.q)[i] = reinterpret_cast<const uint4 *>(q)[i];
    const unsigned nd = act == 2 ? n / 256 : n / 32, nb = act == 2 ? n / 16 : n / 32;
    for (unsigned i = threadIdx.x; i < nd; i += blockDim.x) {
        X.d[i] = d[i];
        if (act == 1) X.s[i] = s[i];
    }
    for (unsigned i = threadIdx.x; i < nb; i += blockDim.x) X.b[i] = b[i];
    __syncthreads();
}

// Image block b (32 values, lane r holding value r) of a next pass's x, written by a warp: the reference's Q8_0 /
// Q8_1 arithmetic (gemvq_ref.h:196-245), the same as the x preparation. n: the values of the whole x.
__device__ __forceinline__ void write_image_block(uint8_t *img, unsigned n, unsigned b, float y, unsigned lane,
                                                  unsigned act) {
    const float amax = warp_max(fabsf(y));
    const float s = fdiv(amax, 127.0f);
    const float id = s != 0.0f ? fdiv(1.0f, s) : 0.0f;
    const int q = int(roundf(fmul(y, id)));
    const int sum = warp_sum_i(q);
    const uint32_t qb = uint32_t(q & 0xff);
    const uint32_t w = qb | (__shfl_down_sync(0xffffffffu, qb, 1) << 8) | (__shfl_down_sync(0xffffffffu, qb, 2) << 16) |
                       (__shfl_down_sync(0xffffffffu, qb, 3) << 24);
    if ((lane & 3u) == 0) {  // bytes 4k .. 4k + 3: half k / 4, word k % 4
        const unsigned k = lane / 4;
        *reinterpret_cast<uint32_t *>(img + (k / 4) * (n / 2) + b * 16 + (k % 4) * 4) = w;
    }
    if (lane == 0) {
        const float dh = half_bits_to_float(float_to_half_bits(s));
        const float sh = act == 1 ? half_bits_to_float(float_to_half_bits(fmul(float(sum), s))) : 0.0f;
        *reinterpret_cast<uint4 *>(img + n + b * 16) =
            make_uint4(__float_as_uint(dh), __float_as_uint(sh), uint32_t(sum), 0u);
    }
}

// One 32-value block of an activation row quantized to Q8_0 / Q8_1 by one thread from registers: the arithmetic of
// quant_block_q80 (gemvq_ref.h:196-245), the image words of an XBlock (values 0..15, 16..31, {d, s, sum of q, 0}).
__device__ __forceinline__ void batch_quant_block(const float *x32, bool q81, uint4 &q0, uint4 &q1, uint4 &meta) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = reinterpret_cast<const float4 *>(x32)[i];
        v[4 * i] = f.x;
        v[4 * i + 1] = f.y;
        v[4 * i + 2] = f.z;
        v[4 * i + 3] = f.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    const float sc = fdiv(amax, 127.0f);
    const float id = sc != 0.0f ? fdiv(1.0f, sc) : 0.0f;
    uint32_t w[8];
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int q = int(roundf(fmul(v[4 * k + e], id)));
            sum += q;
            word |= uint32_t(q & 0xff) << (8 * e);
        }
        w[k] = word;
    }
    q0 = make_uint4(w[0], w[1], w[2], w[3]);
    q1 = make_uint4(w[4], w[5], w[6], w[7]);
    const float d = half_bits_to_float(float_to_half_bits(sc));
    const float s8 = q81 ? half_bits_to_float(float_to_half_bits(fmul(float(sum), sc))) : 0.0f;
    meta = make_uint4(__float_as_uint(d), __float_as_uint(s8), uint32_t(sum), 0u);
}

}  // namespace b200q
