/*
 * CPU oracle for the b200q decode hot path — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this library, and only as the
 * checker or the timed CPU baseline; the product (libb200q.so) never links or calls it.
 *
 * What it restates: the reference's CPU path for the decode hot path, i.e. the generic ggml arithmetic the
 * reference verifies its FPGA kernel against (fpga/src/gemvq_ref.h, which states that it follows ggml's generic
 * quantize_row_q8_0 / quantize_row_q8_K_ref / ggml_vec_dot_*_generic), plus the command-list semantics of the
 * reference ISA (fpga/src/gemvqc16.h:24-121) executed command by command ("the result of running the commands one
 * by one", gemvqc16.h:44-45, 80-81). ggml itself (llama.cpp @ c92e806d) is not available here; the reference's own
 * gemvq_ref.h is compiled beside this file (oracle/_ref) and the tests check this restatement against it.
 *
 * Floating point: compiled with -ffp-contract=off and without -march=native, so every a*b+c rounds twice as the
 * C source reads (ISO semantics); the device kernels use __fmul_rn/__fadd_rn for the same reason.
 *
 * Parity pins: outputs of the reference's gemvq_ref.h built from its sources (oracle/_ref) and the golden vectors
 * under tests/golden/ that tests/golden/make_golden.py generated from it.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------------------------------------------------------
 * FP16 <-> FP32 (gemvq_ref.h:16-52: exact widening; RNE narrowing incl. subnormals, overflow to inf)
 * ------------------------------------------------------------------------------------------------------------- */
ORC_API float orc_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int shift = 0;
            while (!(m & 0x400u)) { m <<= 1; ++shift; }
            bits = sign | (uint32_t)(113 - shift) << 23 | (m & 0x3ffu) << 13;
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | m << 13;
    } else {
        bits = sign | (e + 112u) << 23 | m << 13;
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

ORC_API uint16_t orc_float_to_half(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int e = (int)((bits >> 23) & 0xff) - 112; /* half exponent field */
    uint32_t m = bits & 0x7fffffu;
    if (e >= 31) return sign | 0x7c00u;
    if (e <= 0) {
        if (e < -10) return sign;
        m |= 0x800000u;
        int shift = 14 - e;
        uint32_t r = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return sign | (uint16_t)r;
    }
    uint32_t r = ((uint32_t)e << 10) | (m >> 13), rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r; /* carry into the exponent is the right result */
    return sign | (uint16_t)r;
}

/* ggml nearest_int: round half to even by adding 1.5 * 2^23 (gemvq_ref.h:54-60) */
static int nearest_int(float v) {
    float biased = v + 12582912.f;
    int32_t b;
    memcpy(&b, &biased, 4);
    return (b & 0x007fffff) - 0x00400000;
}

/* ---------------------------------------------------------------------------------------------------------------
 * Activation quantizers
 * ------------------------------------------------------------------------------------------------------------- */
/* Q8_0 (gemvq_ref.h:239-245, ggml quantize_row_q8_0 generic): per 32 values amax, s = amax / 127,
 * id = s ? 1 / s : 0, d = fp16(s), q = roundf(x * id). bsum: sum of the block's q (ints, for the kernels' checks). */
ORC_API void orc_quantize_q8_0(const float *x, unsigned n, int8_t *q, uint16_t *d, int32_t *bsum) {
    for (unsigned b = 0; b < n / 32; ++b) {
        float amax = 0.0f;
        for (unsigned j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[b * 32 + j]));
        const float s = amax / 127.0f, id = s != 0.0f ? 1.0f / s : 0.0f;
        d[b] = orc_float_to_half(s);
        int32_t sum = 0;
        for (unsigned j = 0; j < 32; ++j) {
            q[b * 32 + j] = (int8_t)roundf(x[b * 32 + j] * id);
            sum += q[b * 32 + j];
        }
        if (bsum) bsum[b] = sum;
    }
}

/* Q8_1 (gemvq_ref.h:194-212, quantize_row_q8_1_ref): as Q8_0, plus s = fp16(sum(q) * d_unrounded). ds: 2 halves
 * per block (d, s). */
ORC_API void orc_quantize_q8_1(const float *x, unsigned n, int8_t *q, uint16_t *ds, int32_t *bsum) {
    for (unsigned b = 0; b < n / 32; ++b) {
        float amax = 0.0f;
        for (unsigned j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[b * 32 + j]));
        const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
        int32_t sum = 0;
        for (unsigned j = 0; j < 32; ++j) {
            q[b * 32 + j] = (int8_t)roundf(x[b * 32 + j] * id);
            sum += q[b * 32 + j];
        }
        ds[2 * b] = orc_float_to_half(d);
        ds[2 * b + 1] = orc_float_to_half((float)sum * d);
        if (bsum) bsum[b] = sum;
    }
}

/* Q8_K (gemvq_ref.h:62-81, quantize_row_q8_K_ref): per 256 values the value of largest magnitude (the first one on
 * ties) gives iscale = -127 / max, q = min(127, nearest_int(iscale * x)), d = 1 / iscale (0 for an all-zero block);
 * bsums: the 16 sums of 16 q per super-block. */
ORC_API void orc_quantize_q8_k(const float *x, unsigned n, int8_t *q, float *d, int32_t *bsums) {
    for (unsigned b = 0; b < n / 256; ++b) {
        const float *xb = x + b * 256;
        float max = 0.0f, amax = 0.0f;
        for (unsigned j = 0; j < 256; ++j) {
            const float ax = fabsf(xb[j]);
            if (ax > amax) { amax = ax; max = xb[j]; }
        }
        if (amax == 0.0f) {
            d[b] = 0.0f;
            memset(q + b * 256, 0, 256);
        } else {
            const float iscale = -127.0f / max;
            for (unsigned j = 0; j < 256; ++j) {
                int v = nearest_int(iscale * xb[j]);
                q[b * 256 + j] = (int8_t)(v < 127 ? v : 127);
            }
            d[b] = 1.0f / iscale;
        }
        if (bsums) {
            for (unsigned g = 0; g < 16; ++g) {
                int32_t s = 0;
                for (unsigned j = 0; j < 16; ++j) s += q[b * 256 + g * 16 + j];
                bsums[b * 16 + g] = s;
            }
        }
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * GEMV rows (one row of GGUF blocks against quantized x)
 * ------------------------------------------------------------------------------------------------------------- */
static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | p[1] << 8); }

ORC_API size_t orc_row_bytes(unsigned cols, unsigned format) {
    switch (format) {
    case 2: return (size_t)(cols / 32) * 18;
    case 3: return (size_t)(cols / 32) * 20;
    case 8: return (size_t)(cols / 32) * 34;
    case 13: return (size_t)(cols / 256) * 176;
    case 14: return (size_t)(cols / 256) * 210;
    default: return 0;
    }
}

/* Q4_0 / Q8_0 block integer dot (gemvq_ref.h:251-257): Q4_0 element j < 16 is the low nibble of byte j, j >= 16
 * the high nibble of byte j - 16, minus 8; Q8_0 elements are int8. */
static int32_t dot_block_q40_q80(const uint8_t *blk, unsigned format, const int8_t *q) {
    int32_t s = 0;
    for (unsigned j = 0; j < 32; ++j) {
        int w = format == 2 ? (int)(j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4)) - 8 : (int)(int8_t)blk[2 + j];
        s += w * q[j];
    }
    return s;
}

/* Q4_0 / Q8_0 row (gemvq_ref.h:248-263): sum += float(sumi) * (d_w * d_x) in block order. */
static float row_q40_q80(const uint8_t *row, unsigned format, unsigned nb, const int8_t *q, const float *dx,
                         double *mag) {
    const unsigned bb = format == 2 ? 18 : 34;
    float sum = 0.0f;
    double m = 0.0;
    for (unsigned b = 0; b < nb; ++b) {
        const uint8_t *blk = row + (size_t)b * bb;
        const int32_t sumi = dot_block_q40_q80(blk, format, q + b * 32);
        const float term = (float)sumi * (orc_half_to_float(rd16(blk)) * dx[b]);
        sum += term;
        m += fabs((double)term);
    }
    if (mag) *mag = m;
    return sum;
}

/* Q4_1 row against Q8_1 (gemvq_ref.h:213-227): sum += (d4 * d8) * sumi + m4 * s8. */
static float row_q41_q81(const uint8_t *row, unsigned nb, const int8_t *q, const float *d8, const float *s8,
                         double *mag) {
    float sum = 0.0f;
    double m = 0.0;
    for (unsigned b = 0; b < nb; ++b) {
        const uint8_t *blk = row + (size_t)b * 20;
        int32_t sumi = 0;
        for (unsigned j = 0; j < 16; ++j)
            sumi += (blk[4 + j] & 0x0F) * q[b * 32 + j] + (blk[4 + j] >> 4) * q[b * 32 + j + 16];
        const float dw = orc_half_to_float(rd16(blk)), mw = orc_half_to_float(rd16(blk + 2));
        const float a = (dw * d8[b]) * (float)sumi, c = mw * s8[b];
        sum += a + c;
        m += (double)(fabsf(a) + fabsf(c));  /* float sum, as gemvq_ref.h:224 */
    }
    if (mag) *mag = m;
    return sum;
}

/* get_scale_min_k4 (gemvq_ref.h:83-92) */
static void scale_min_k4(unsigned j, const uint8_t *s, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* The integer parts of one Q5_K super-block (gemvq_ref.h:98-121): aux[l] = sum over i % 8 == l of sc * q8 * w,
 * mins = sum_j bsum_j * m_j. */
static void q5k_sb_ints(const uint8_t *blk, const int8_t *y, int32_t aux[8], int32_t *mins) {
    const uint8_t *scales = blk + 4, *qh = blk + 16, *qs = blk + 48;
    int a[256];
    for (unsigned s = 0; s < 8; ++s)
        for (unsigned e = 0; e < 32; ++e) {
            const uint8_t byte = qs[32 * (s / 2) + e];
            a[32 * s + e] = ((s & 1) ? (byte >> 4) : (byte & 15)) + (((qh[e] >> s) & 1) ? 16 : 0);
        }
    int32_t sumi = 0;
    for (unsigned j = 0; j < 16; ++j) {
        int bs = 0, sc, m;
        for (unsigned i = 0; i < 16; ++i) bs += y[16 * j + i];
        scale_min_k4(j / 2, scales, &sc, &m);
        sumi += bs * m;
    }
    for (unsigned l = 0; l < 8; ++l) aux[l] = 0;
    for (unsigned j = 0; j < 8; ++j) {
        int sc, m;
        scale_min_k4(j, scales, &sc, &m);
        for (unsigned i = 0; i < 32; ++i) aux[i % 8] += sc * (y[32 * j + i] * a[32 * j + i]);
    }
    *mins = sumi;
}

/* Q6_K super-block ints (gemvq_ref.h:152-169) */
static void q6k_sb_ints(const uint8_t *blk, const int8_t *y, int32_t aux[8]) {
    const uint8_t *ql = blk, *qh = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    int a[256];
    for (unsigned n = 0; n < 2; ++n)
        for (unsigned l = 0; l < 32; ++l) {
            const uint8_t h = qh[32 * n + l];
            a[128 * n + l] = (int8_t)((ql[64 * n + l] & 0xF) | (((h >> 0) & 3) << 4)) - 32;
            a[128 * n + l + 32] = (int8_t)((ql[64 * n + l + 32] & 0xF) | (((h >> 2) & 3) << 4)) - 32;
            a[128 * n + l + 64] = (int8_t)((ql[64 * n + l] >> 4) | (((h >> 4) & 3) << 4)) - 32;
            a[128 * n + l + 96] = (int8_t)((ql[64 * n + l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32;
        }
    for (unsigned l = 0; l < 8; ++l) aux[l] = 0;
    for (unsigned j = 0; j < 16; ++j)
        for (unsigned i = 0; i < 16; ++i) aux[i % 8] += sc[j] * (y[16 * j + i] * a[16 * j + i]);
}

/* Q5_K row (gemvq_ref.h:95-134): sums[l] += d * aux[l] per super-block, sumf -= dmin * mins, then sumf += sums[l]. */
static float row_q5k(const uint8_t *row, unsigned nsb, const int8_t *q8, const float *d8, double *mag) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0}, sumf = 0.0f;
    double m = 0.0;
    for (unsigned sb = 0; sb < nsb; ++sb) {
        const uint8_t *blk = row + (size_t)sb * 176;
        int32_t aux[8], mins;
        q5k_sb_ints(blk, q8 + sb * 256, aux, &mins);
        const float d = orc_half_to_float(rd16(blk)) * d8[sb];
        double part = 0.0;
        for (unsigned l = 0; l < 8; ++l) {
            sums[l] += d * (float)aux[l];
            part += (double)aux[l];
        }
        const float dmin = orc_half_to_float(rd16(blk + 2)) * d8[sb];
        sumf -= dmin * (float)mins;
        m += fabs((double)d * part) + fabs((double)dmin * mins);
    }
    for (unsigned l = 0; l < 8; ++l) sumf += sums[l];
    if (mag) *mag = m;
    return sumf;
}

/* Q6_K row (gemvq_ref.h:149-181) */
static float row_q6k(const uint8_t *row, unsigned nsb, const int8_t *q8, const float *d8, double *mag) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    double m = 0.0;
    for (unsigned sb = 0; sb < nsb; ++sb) {
        const uint8_t *blk = row + (size_t)sb * 210;
        int32_t aux[8];
        q6k_sb_ints(blk, q8 + sb * 256, aux);
        const float d = orc_half_to_float(rd16(blk + 208)) * d8[sb];
        double part = 0.0;
        for (unsigned l = 0; l < 8; ++l) {
            sums[l] += d * (float)aux[l];
            part += (double)aux[l];
        }
        m += fabs((double)d * part);
    }
    float sumf = 0.0f;
    for (unsigned l = 0; l < 8; ++l) sumf += sums[l];
    if (mag) *mag = m;
    return sumf;
}

/* Full GEMV y = W x on GGUF rows, x quantized as the format's ggml vec_dot type (gemvq_ref.h:231-265, 137-146,
 * 183-192, 196-229). mag (optional): per row the sum of |block terms| (tolerance of gemvq_ref.h:269-272).
 * Rows are independent; OpenMP splits them (the timed CPU baseline uses that). */
ORC_API int orc_gemv(const uint8_t *w, const float *x, unsigned rows, unsigned cols, unsigned format, float *y,
                     double *mag) {
    const size_t rb = orc_row_bytes(cols, format);
    if (rb == 0) return -1;
    int8_t *q = (int8_t *)malloc(cols);
    float *d = (float *)malloc(sizeof(float) * (cols / 32 + 1));
    float *s = (float *)malloc(sizeof(float) * (cols / 32 + 1));
    if (format == 13 || format == 14) {
        orc_quantize_q8_k(x, cols, q, d, NULL);
    } else if (format == 3) {
        uint16_t *ds = (uint16_t *)malloc(sizeof(uint16_t) * 2 * (cols / 32));
        orc_quantize_q8_1(x, cols, q, ds, NULL);
        for (unsigned b = 0; b < cols / 32; ++b) {
            d[b] = orc_half_to_float(ds[2 * b]);
            s[b] = orc_half_to_float(ds[2 * b + 1]);
        }
        free(ds);
    } else {
        uint16_t *d16 = (uint16_t *)malloc(sizeof(uint16_t) * (cols / 32));
        orc_quantize_q8_0(x, cols, q, d16, NULL);
        for (unsigned b = 0; b < cols / 32; ++b) d[b] = orc_half_to_float(d16[b]);
        free(d16);
    }
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)rows; ++r) {
        const uint8_t *row = w + (size_t)r * rb;
        double m = 0.0;
        float v;
        if (format == 13) v = row_q5k(row, cols / 256, q, d, &m);
        else if (format == 14) v = row_q6k(row, cols / 256, q, d, &m);
        else if (format == 3) v = row_q41_q81(row, cols / 32, q, d, s, &m);
        else v = row_q40_q80(row, format, cols / 32, q, d, &m);
        y[r] = v;
        if (mag) mag[r] = m;
    }
    free(q);
    free(d);
    free(s);
    return 0;
}

/* Per-block integer sums of a GEMV against already-quantized x (the "per-block int32 dot sums" of the bit-exact
 * contract). Q4_0/Q8_0: rows x nb sumi; Q4_1: rows x nb; Q5_K/Q6_K: rows x nsb x 9 (aux[0..7], mins). */
ORC_API int orc_block_sums(const uint8_t *w, const int8_t *q, unsigned rows, unsigned cols, unsigned format,
                           int32_t *out) {
    const size_t rb = orc_row_bytes(cols, format);
    if (rb == 0) return -1;
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)rows; ++r) {
        const uint8_t *row = w + (size_t)r * rb;
        if (format == 13 || format == 14) {
            for (unsigned sb = 0; sb < cols / 256; ++sb) {
                int32_t *o = out + ((size_t)r * (cols / 256) + sb) * 9;
                if (format == 13) q5k_sb_ints(row + (size_t)sb * 176, q + sb * 256, o, &o[8]);
                else { q6k_sb_ints(row + (size_t)sb * 210, q + sb * 256, o); o[8] = 0; }
            }
        } else if (format == 3) {
            for (unsigned b = 0; b < cols / 32; ++b) {
                const uint8_t *blk = row + (size_t)b * 20;
                int32_t s = 0;
                for (unsigned j = 0; j < 16; ++j)
                    s += (blk[4 + j] & 0x0F) * q[b * 32 + j] + (blk[4 + j] >> 4) * q[b * 32 + j + 16];
                out[(size_t)r * (cols / 32) + b] = s;
            }
        } else {
            const unsigned bb = format == 2 ? 18 : 34;
            for (unsigned b = 0; b < cols / 32; ++b)
                out[(size_t)r * (cols / 32) + b] = dot_block_q40_q80(row + (size_t)b * bb, format, q + b * 32);
        }
    }
    return 0;
}

/* ---------------------------------------------------------------------------------------------------------------
 * Element-wise ops (gemvq_ref.h:286-358; RoPE after fpga/src/gemvqc_ops.h:275-312 / ggml's NEOX rope)
 * ------------------------------------------------------------------------------------------------------------- */
/* silu(x) = x / (1 + expf(-x)) (gemvq_ref.h:286-287, 303-307) */
static float silu(float v) { return v / (1.0f + expf(-v)); }

/* Row norm of the RMSNORM opcode (gemvq_ref.h:309-324, ggml rms_norm / l2_norm): squares in float, summed in
 * double; RMS: scale = 1 / sqrtf(float(sum / n) + eps); L2: scale = 1 / fmaxf(sqrtf(float(sum)), eps);
 * y = (x * scale) * w, or x * scale without weight. */
ORC_API float orc_norm_scale(const float *x, unsigned n, float eps, unsigned l2) {
    double sum = 0.0;
    for (unsigned i = 0; i < n; ++i) sum += (double)(x[i] * x[i]);
    return l2 ? 1.0f / fmaxf(sqrtf((float)sum), eps) : 1.0f / sqrtf((float)(sum / n) + eps);
}

ORC_API void orc_rownorm(const float *x, const float *w, unsigned n, unsigned rows, unsigned stride, float eps,
                         unsigned flags, float *y) {
    for (unsigned r = 0; r < rows; ++r) {
        const float *xr = x + (size_t)r * (stride ? stride : n);
        const float scale = orc_norm_scale(xr, n, eps, flags & 1u);
        for (unsigned i = 0; i < n; ++i) y[(size_t)r * n + i] = (flags & 2u) ? xr[i] * scale : (xr[i] * scale) * w[i];
    }
}

/* UNARY kinds 1 SiLU, 2 sigmoid, 3 softplus (x > 20 ? x : log(1 + e^x)) (gemvq_ref.h:332-342) */
ORC_API float orc_unary1(float v, unsigned kind) {
    if (kind == 1) return v / (1.0f + expf(-v));
    if (kind == 2) return 1.0f / (1.0f + expf(-v));
    if (kind == 3) return v > 20.0f ? v : logf(1.0f + expf(v));
    return v;
}

/* SILU_MUL: silu(g) * u, or with the sigmoid flag sigmoid(g) * u (gemvq_ref.h:303-307; gemvqc_ops.h:94-99) */
ORC_API float orc_silu_mul1(float g, float u, unsigned sigmoid) {
    return sigmoid ? (1.0f / (1.0f + expf(-g))) * u : silu(g) * u;
}

/* ggml_ssm_conv, one token, d_conv 4 (gemvq_ref.h:344-358): window [state[3c..3c+2], x[c]] (channel-major state),
 * kernel w[4c..4c+3]; sum from t = 0; new state = window[1..3]. Safe when s_dst == s_src. */
ORC_API void orc_conv(const float *state, const float *x, const float *w, unsigned ch, unsigned use_silu, float *y,
                      float *new_state) {
    for (unsigned c = 0; c < ch; ++c) {
        const float in[4] = {state[c * 3], state[c * 3 + 1], state[c * 3 + 2], x[c]};
        float sum = 0.0f;
        for (unsigned t = 0; t < 4; ++t) sum += in[t] * w[c * 4 + t];
        y[c] = use_silu ? silu(sum) : sum;
        for (unsigned t = 0; t < 3; ++t) new_state[c * 3 + t] = in[t + 1];
    }
}

/* NEOX RoPE (gemvqc_ops.h:275-312): pairs (i, i + n_dims/2) rotated by cos/sin at cs[2i], cs[2i+1]; floats from
 * n_dims on copied. */
ORC_API void orc_rope(const float *x, const float *cs, unsigned n_dims, unsigned ne0, unsigned rows, float *y) {
    const unsigned half = n_dims / 2;
    for (unsigned r = 0; r < rows; ++r) {
        const float *xr = x + (size_t)r * ne0;
        float *yr = y + (size_t)r * ne0;
        for (unsigned i = n_dims; i < ne0; ++i) yr[i] = xr[i];
        for (unsigned i = 0; i < half; ++i) {
            const float x0 = xr[i], x1 = xr[i + half], c = cs[2 * i], s = cs[2 * i + 1];
            yr[i] = x0 * c - x1 * s;
            yr[i + half] = x0 * s + x1 * c;
        }
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * Gated DeltaNet step (gemvq_ref.h:360-397; ggml GATED_DELTA_NET, one token, scalar gate, head size 128).
 * state[h][j][i]: row j of head h holds column j of S. Key head of value head h is h % hk. Updates the state in
 * place, writes y[hv][128]; s_mag / y_mag (optional) are the term magnitudes of the reference's tolerance.
 * ------------------------------------------------------------------------------------------------------------- */
ORC_API void orc_gdn(float *state, const float *q, const float *k, const float *v, const float *g, const float *beta,
                     unsigned hv, unsigned hk, float scale, float *y, double *y_mag, double *s_mag) {
    const unsigned S = 128;
    for (unsigned h = 0; h < hv; ++h) {
        const float *qh = q + (h % hk) * S, *kh = k + (h % hk) * S;
        const float decay = expf(g[h]);
        for (unsigned j = 0; j < S; ++j) {
            float *row = state + ((size_t)h * S + j) * S;
            double dmag = 0.0;
            float dot = 0.0f;
            for (unsigned i = 0; i < S; ++i) {
                row[i] *= decay;
                dot += row[i] * kh[i];
                dmag += fabs((double)row[i] * kh[i]);
            }
            const float delta = (v[h * S + j] - dot) * beta[h];
            const double delta_mag = (fabs((double)v[h * S + j]) + dmag) * fabs((double)beta[h]);
            float out = 0.0f;
            double omag = 0.0;
            for (unsigned i = 0; i < S; ++i) {
                if (s_mag) s_mag[((size_t)h * S + j) * S + i] = fabs((double)row[i]) + fabs((double)kh[i]) * delta_mag;
                row[i] += kh[i] * delta;
                out += row[i] * qh[i];
                omag += (fabs((double)row[i]) + fabs((double)kh[i]) * delta_mag) * fabs((double)qh[i]);
            }
            y[h * S + j] = out * scale;
            if (y_mag) y_mag[h * S + j] = omag * scale;
        }
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * Decode attention over an F16 KV cache (extension opcode 12; the reference runs this on the CPU through ggml's
 * F16 path: scores = q . k (k widened from F16), scaled, softmax with the max subtracted, y = sum p * v).
 * kv layout: K then V, each [n_kv_head][n_ctx][head_dim] F16; GQA: q head h reads kv head h / (n_head/n_kv_head).
 * ------------------------------------------------------------------------------------------------------------- */
ORC_API void orc_attn(const float *q, const uint16_t *kcache, const uint16_t *vcache, unsigned n_head,
                      unsigned n_kv_head, unsigned head_dim, unsigned n_ctx, unsigned n_past, float scale, float *y) {
    const unsigned group = n_head / n_kv_head;
    float *p = (float *)malloc(sizeof(float) * (n_past ? n_past : 1));
    for (unsigned h = 0; h < n_head; ++h) {
        const unsigned kvh = h / group;
        const float *qh = q + (size_t)h * head_dim;
        float mx = -INFINITY;
        for (unsigned t = 0; t < n_past; ++t) {
            const uint16_t *kr = kcache + ((size_t)kvh * n_ctx + t) * head_dim;
            double s = 0.0;
            for (unsigned i = 0; i < head_dim; ++i) s += (double)qh[i] * (double)orc_half_to_float(kr[i]);
            p[t] = (float)s * scale;
            if (p[t] > mx) mx = p[t];
        }
        double sum = 0.0;
        for (unsigned t = 0; t < n_past; ++t) {
            p[t] = expf(p[t] - mx);
            sum += p[t];
        }
        for (unsigned i = 0; i < head_dim; ++i) {
            double acc = 0.0;
            for (unsigned t = 0; t < n_past; ++t)
                acc += (double)p[t] * (double)orc_half_to_float(vcache[((size_t)kvh * n_ctx + t) * head_dim + i]);
            y[(size_t)h * head_dim + i] = (float)(acc / sum);
        }
    }
    free(p);
}

/* Dequantize one GGUF row (ggml dequantize_row_q4_0 / q8_0: y = float(q - 8) * d, y = float(q) * d). */
ORC_API int orc_dequantize_row(const uint8_t *row, unsigned cols, unsigned format, float *y) {
    for (unsigned b = 0; b < cols / 32; ++b) {
        if (format == 2) {
            const uint8_t *blk = row + (size_t)b * 18;
            const float d = orc_half_to_float(rd16(blk));
            for (unsigned j = 0; j < 16; ++j) {
                y[b * 32 + j] = (float)((blk[2 + j] & 0x0F) - 8) * d;
                y[b * 32 + j + 16] = (float)((blk[2 + j] >> 4) - 8) * d;
            }
        } else if (format == 8) {
            const uint8_t *blk = row + (size_t)b * 34;
            const float d = orc_half_to_float(rd16(blk));
            for (unsigned j = 0; j < 32; ++j) y[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
        } else {
            return -1;
        }
    }
    return 0;
}

/* ---------------------------------------------------------------------------------------------------------------
 * Command-list interpreter: the reference ISA (gemvqc16.h:24-121) executed command by command, fused forms as the
 * plain sequences they stand for. Weights: table of (handle, GGUF bytes, rows, cols, format). State: rows of 128
 * floats. Returns 0, or the 1-based index of the first command it rejects (validation mirrors
 * fpga/src/gemvqc16.cpp:455-913), or 129 for more than 128 commands.
 * ------------------------------------------------------------------------------------------------------------- */
typedef struct orc_weight {
    uint64_t handle;
    const uint8_t *data;
    unsigned rows, cols, format;
} orc_weight;

static const orc_weight *find_w(const orc_weight *ws, unsigned nw, uint64_t h) {
    for (unsigned i = 0; i < nw; ++i)
        if (ws[i].handle == h) return &ws[i];
    return NULL;
}

static float bits_f(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}

typedef struct {
    float *act;
    size_t act_floats;
    float *state;
    size_t state_rows;
    const orc_weight *ws;
    unsigned nw;
    const uint16_t *kv;
    size_t kv_bytes;
    unsigned kv_ctx; /* tokens per KV slot (ATTN extension) */
    /* deferred norm: the normalized row the following GEMVs read instead of act at nd_y */
    int nd_valid;
    unsigned nd_y, nd_n;
    float *nd_row;
} orc_machine;

static int in_act(const orc_machine *m, size_t off, size_t n) { return off + n <= m->act_floats; }

/* GEMV command: y (rounded up to 16 floats, padding 0) = W x; x from the deferred norm if it matches. */
static int exec_gemv(orc_machine *m, const uint32_t *c, float *out_override, int allow_nd) {
    const unsigned fmt = c[1] & 0xff, rows = c[2], cols = c[3], x_off = c[6], y_off = c[7];
    const uint64_t h = (uint64_t)c[4] | ((uint64_t)c[5] << 32);
    const orc_weight *w = find_w(m->ws, m->nw, h);
    if (!w || w->format != fmt || w->cols != cols || w->rows < rows) return -1;
    if (!in_act(m, x_off, cols)) return -1;
    const float *x = (allow_nd && m->nd_valid && x_off == m->nd_y && cols == m->nd_n) ? m->nd_row : m->act + x_off;
    float *tmp = (float *)malloc(sizeof(float) * rows);
    orc_gemv(w->data, x, rows, cols, fmt, tmp, NULL);
    if (out_override) {
        memcpy(out_override, tmp, sizeof(float) * rows);
    } else {
        const unsigned pad = (rows + 15) / 16 * 16;
        if (!in_act(m, y_off, pad)) { free(tmp); return -1; }
        memcpy(m->act + y_off, tmp, sizeof(float) * rows);
        for (unsigned r = rows; r < pad; ++r) m->act[y_off + r] = 0.0f;
    }
    free(tmp);
    return 0;
}

static int gemv_valid(const uint32_t *c) {
    const unsigned fmt = c[1] & 0xff, rows = c[2], cols = c[3], flags = c[1] & ~0xffu;
    const int kq = fmt == 13 || fmt == 14;
    return c[0] == 1 && (flags & ~(0x100u | 0x200u | 0x400u)) == 0 && (flags & (flags - 1u)) == 0 && rows != 0 &&
           rows <= 65536 && cols != 0 && cols <= 16384 && cols % (kq ? 256u : 128u) == 0 &&
           (fmt == 2 || fmt == 3 || fmt == 8 || kq) && c[6] % 16 == 0 && c[7] % 16 == 0;
}

static unsigned act_type(unsigned fmt) { return (fmt == 13 || fmt == 14) ? 2u : (fmt == 3 ? 1u : 0u); }

ORC_API int orc_run_list(float *act, size_t act_floats, float *state, size_t state_rows, const orc_weight *ws,
                         unsigned nw, const uint16_t *kv, size_t kv_bytes, unsigned kv_ctx, const uint32_t *cmds,
                         unsigned n_cmds) {
    if (n_cmds == 0) {
        /* feature probe (gemvqc16.h:124-134): the features this library reports */
        const uint32_t f[3] = {0x6B51FFFFu, 0x6B520001u, 0x6B53007Fu};
        memcpy(act, f, sizeof(f));
        return 0;
    }
    if (n_cmds > 128) return 129;
    orc_machine M = {act, act_floats, state, state_rows, ws, nw, kv, kv_bytes, kv_ctx, 0, 0, 0, NULL};
    M.nd_row = (float *)malloc(sizeof(float) * 16384);
    int status = 0;
    unsigned i = 0;
    while (i < n_cmds && status == 0) {
        const uint32_t *c = cmds + (size_t)i * 8;
        const uint32_t op = c[0];
        unsigned adv = 1;
        if (op == 1) { /* GEMV, possibly with an epilogue command behind it */
            const uint32_t fl = c[1] & ~0xffu;
            if (!gemv_valid(c)) { status = (int)i + 1; break; }
            if (fl & 0x100u) { /* SwiGLU pair: g here, u next (same x, rows; no epilogue bits) */
                const uint32_t *u = cmds + (size_t)(i + 1) * 8;
                /* a group ends after a member whose y (rounded to 16) overlaps x, so such a g has no u
                 * (gemvqc16.cpp:468-474, 700-719) */
                const unsigned gyr = (c[2] + 15) / 16 * 16;
                const int g_over_x = c[7] < c[6] + c[3] && c[6] < c[7] + gyr;
                if (i + 1 >= n_cmds || g_over_x || !gemv_valid(u) || u[2] != c[2] || (u[1] & ~0xffu) != 0 ||
                    u[6] != c[6] || u[3] != c[3] || act_type(u[1] & 0xff) != act_type(c[1] & 0xff) || c[2] > 16384) {
                    status = (int)i + 1;
                    break;
                }
                const unsigned rows = c[2], pad = (rows + 15) / 16 * 16;
                float *g = (float *)malloc(sizeof(float) * rows), *uu = (float *)malloc(sizeof(float) * rows);
                if (exec_gemv(&M, c, g, 1) || exec_gemv(&M, u, uu, 1) || !in_act(&M, u[7], pad)) {
                    free(g); free(uu); status = (int)i + 1; break;
                }
                for (unsigned r = 0; r < rows; ++r) M.act[u[7] + r] = orc_silu_mul1(g[r], uu[r], 0);
                for (unsigned r = rows; r < pad; ++r) M.act[u[7] + r] = 0.0f;
                free(g); free(uu);
                adv = 2;
            } else if (fl & 0x200u) { /* CONV epilogue: next command is CONV on this y */
                const uint32_t *cv = cmds + (size_t)(i + 1) * 8;
                if (i + 1 >= n_cmds || cv[0] != 8 || cv[1] != c[2] || cv[2] != c[7] || cv[1] % 16 || cv[1] > 16384 ||
                    cv[3] % 16 || cv[4] % 16 || cv[5] % 16 || cv[6] % 16 || cv[7] > 1) {
                    status = (int)i + 1;
                    break;
                }
                const unsigned ch = c[2];
                float *t = (float *)malloc(sizeof(float) * ch), *ns = (float *)malloc(sizeof(float) * ch * 3);
                if (exec_gemv(&M, c, t, 1) || !in_act(&M, cv[3], 4 * ch) || !in_act(&M, cv[4], ch) ||
                    !in_act(&M, cv[5], 3 * ch) || !in_act(&M, cv[6], 3 * ch)) {
                    free(t); free(ns); status = (int)i + 1; break;
                }
                orc_conv(M.act + cv[5], t, M.act + cv[3], ch, cv[7] & 1u, M.act + cv[4], ns);
                memcpy(M.act + cv[6], ns, sizeof(float) * ch * 3);
                free(t); free(ns);
                adv = 2;
            } else if (fl & 0x400u) { /* ADD epilogue */
                const uint32_t *ad = cmds + (size_t)(i + 1) * 8;
                const unsigned rows = c[2];
                if (i + 1 >= n_cmds || ad[0] != 3 || ad[1] != rows || (ad[2] != c[7] && ad[3] != c[7]) || rows % 16 ||
                    rows > 16384 || ad[2] % 16 || ad[3] % 16 || ad[4] % 16) {
                    status = (int)i + 1;
                    break;
                }
                const unsigned r_off = ad[2] == c[7] ? ad[3] : ad[2];
                float *t = (float *)malloc(sizeof(float) * rows);
                if (exec_gemv(&M, c, t, 1) || !in_act(&M, r_off, rows) || !in_act(&M, ad[4], rows)) {
                    free(t); status = (int)i + 1; break;
                }
                for (unsigned r = 0; r < rows; ++r) M.act[ad[4] + r] = t[r] + M.act[r_off + r];
                free(t);
                adv = 2;
            } else if (exec_gemv(&M, c, NULL, 1)) {
                status = (int)i + 1;
                break;
            }
        } else if (op == 2) { /* RMSNORM */
            const unsigned n = c[1], xo = c[2], wo = c[3], yo = c[4], rows = c[6] ? c[6] : 1u, fl = c[7];
            const unsigned stride = (fl >> 8) & 0xffffu, defer = (fl & 4u) != 0;
            if (n == 0 || n % 16 || rows > 4096 || (size_t)(n / 16) * rows > 4096 || xo % 16 || wo % 16 || yo % 16 ||
                (fl & 0xff0000f8u) || (stride != 0 && stride < n / 16) || (defer && (rows != 1 || n > 16384))) {
                status = (int)i + 1;
                break;
            }
            const size_t span = stride ? (size_t)(rows - 1) * stride * 16 + n : (size_t)rows * n;
            if (!in_act(&M, xo, span) || ((fl & 2u) == 0 && !in_act(&M, wo, n)) || !in_act(&M, yo, (size_t)rows * n)) {
                status = (int)i + 1;
                break;
            }
            if (defer) {
                orc_rownorm(M.act + xo, M.act + wo, n, 1, 0, bits_f(c[5]), fl & 3u, M.nd_row);
                M.nd_valid = 1;
                M.nd_y = yo;
                M.nd_n = n;
            } else {
                float *t = (float *)malloc(sizeof(float) * (size_t)rows * n);
                orc_rownorm(M.act + xo, M.act + wo, n, rows, stride * 16, bits_f(c[5]), fl & 3u, t);
                memcpy(M.act + yo, t, sizeof(float) * (size_t)rows * n);
                free(t);
            }
        } else if (op == 3 || op == 4 || op == 5 || op == 6) { /* ADD SILU_MUL MUL UNARY */
            const unsigned n = c[1], a = c[2], b = c[3], yo = c[4];
            const int unary = op == 6, sm = op == 4;
            const unsigned row = unary ? c[5] : (sm ? c[6] : 0u), stride = unary ? c[6] : c[7];
            if (n == 0 || n > 65536 || n % 16 || a % 16 || yo % 16 || (unary ? (b == 0 || b > 4) : (b % 16 != 0)) ||
                (sm && (c[5] & ~1u)) || (row != 0 && (row % 16 || n % row || stride % 16 || stride < row))) {
                status = (int)i + 1;
                break;
            }
            const size_t span = row ? (size_t)(n / row - 1) * stride + row : n;
            if (!in_act(&M, a, span) || (!unary && !in_act(&M, b, n)) || !in_act(&M, yo, n)) {
                status = (int)i + 1;
                break;
            }
            float *t = (float *)malloc(sizeof(float) * n);
            for (unsigned e = 0; e < n; ++e) {
                const size_t ai = row ? (size_t)(e / row) * stride + e % row : e;
                const float av = M.act[a + ai];
                if (op == 3) t[e] = av + M.act[b + e];
                else if (op == 5) t[e] = av * M.act[b + e];
                else if (op == 4) t[e] = orc_silu_mul1(av, M.act[b + e], c[5] & 1u);
                else t[e] = b == 4 ? av : orc_unary1(av, b);
            }
            memcpy(M.act + yo, t, sizeof(float) * n);
            free(t);
        } else if (op == 8) { /* CONV */
            const unsigned ch = c[1];
            if (ch == 0 || ch > 16384 || ch % 16 || c[2] % 16 || c[3] % 16 || c[4] % 16 || c[5] % 16 || c[6] % 16 ||
                c[7] > 1) {
                status = (int)i + 1;
                break;
            }
            if (!in_act(&M, c[2], ch) || !in_act(&M, c[3], 4 * ch) || !in_act(&M, c[4], ch) ||
                !in_act(&M, c[5], 3 * ch) || !in_act(&M, c[6], 3 * ch)) {
                status = (int)i + 1;
                break;
            }
            float *t = (float *)malloc(sizeof(float) * ch), *ns = (float *)malloc(sizeof(float) * 3 * ch);
            orc_conv(M.act + c[5], M.act + c[2], M.act + c[3], ch, c[7] & 1u, t, ns);
            memcpy(M.act + c[4], t, sizeof(float) * ch);
            memcpy(M.act + c[6], ns, sizeof(float) * 3 * ch);
            free(t); free(ns);
        } else if (op == 10) { /* ROPE */
            const unsigned nd = c[1], xo = c[2], cs = c[3], yo = c[4], ne0 = c[5], rows = c[6];
            if (nd == 0 || nd % 32 || nd > 128 || nd > ne0 || ne0 % 16 || rows == 0 || (size_t)(ne0 / 16) * rows > 4096 ||
                xo % 16 || cs % 16 || yo % 16 || c[7] != 0 || !in_act(&M, xo, (size_t)ne0 * rows) ||
                !in_act(&M, cs, nd) || !in_act(&M, yo, (size_t)ne0 * rows)) {
                status = (int)i + 1;
                break;
            }
            float *t = (float *)malloc(sizeof(float) * ne0 * rows);
            orc_rope(M.act + xo, M.act + cs, nd, ne0, rows, t);
            memcpy(M.act + yo, t, sizeof(float) * ne0 * rows);
            free(t);
        } else if (op == 11) { /* TRACE: timing only; no values to check */
            if (c[1] % 16 || (c[2] | c[3] | c[4] | c[5] | c[6] | c[7])) { status = (int)i + 1; break; }
        } else if (op == 9) { /* STATE_LOAD: a prefetch hint, no effect on values */
            if (c[1] == 0 || c[1] > 32 || c[2] % 4) { status = (int)i + 1; break; }
        } else if (op == 7) { /* GDN (gemvqc16.cpp:801-913 validation; gemvqc_gdn.h:223-346 arithmetic) */
            const unsigned hv = c[1] & 0xffffu, hk = c[1] >> 16;
            const uint32_t *e = cmds + (size_t)(i + 1) * 8;
            const uint32_t zero[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (i + 1 >= n_cmds) e = zero;
            const unsigned fl = e[3];
            const int gates = (fl & 8u) != 0;
            const unsigned slots = gates ? 3u : 2u;
            const uint32_t *e2 = (i + 2 < n_cmds) ? cmds + (size_t)(i + 2) * 8 : zero;
            if (i + slots > n_cmds || hv == 0 || hv > 32 || hk == 0 || hk > hv || hv % hk || c[2] % 16 || c[3] % 16 ||
                c[4] % 16 || c[5] % 16 || c[6] % 16 || c[7] % 16 || e[0] % 4 || e[1] % 4 || fl > 31u ||
                ((fl & 4u) && (e[6] % 16 || e[7] % 16)) || (gates && (e2[0] % 16 || e2[1] % 16))) {
                status = (int)i + 1;
                break;
            }
            const unsigned S = 128, rows = hv * S;
            if ((size_t)e[0] + rows > M.state_rows || (size_t)e[1] + rows > M.state_rows ||
                !in_act(&M, c[2], hk * S) || !in_act(&M, c[3], hk * S) || !in_act(&M, c[4], hv * S) ||
                !in_act(&M, c[5], hv) || !in_act(&M, c[6], hv) || !in_act(&M, c[7], hv * S)) {
                status = (int)i + 1;
                break;
            }
            /* a WITH_OUT GEMV (and its ADD) must be valid before anything runs (gemvqc16.cpp:874-895) */
            unsigned out_adv = 0;
            if (fl & 16u) {
                const uint32_t *nx = (i + slots < n_cmds) ? cmds + (size_t)(i + slots) * 8 : zero;
                const unsigned nfl = nx[1] & ~0xffu;
                int ok = (fl & 1u) == 0 && gemv_valid(nx) && (nfl & 0x300u) == 0 && nx[6] == c[7] && nx[3] == rows &&
                         rows % 256 == 0 && nx[2] <= 512u * 20u;
                if (ok && (nfl & 0x400u)) {
                    const uint32_t *ad = (i + slots + 1 < n_cmds) ? cmds + (size_t)(i + slots + 1) * 8 : zero;
                    const unsigned r_off = ad[2] == nx[7] ? ad[3] : ad[2];
                    ok = ad[0] == 3 && ad[1] == nx[2] && (ad[2] == nx[7] || ad[3] == nx[7]) && nx[2] % 16 == 0 &&
                         nx[2] <= 16384 && ad[2] % 16 == 0 && ad[3] % 16 == 0 && ad[4] % 16 == 0 &&
                         !(r_off < c[7] + rows && c[7] < r_off + nx[2]);
                }
                if (!ok) { status = (int)i + 1; break; }
                out_adv = (nfl & 0x400u) ? 2u : 1u;
            }
            float *q = (float *)malloc(sizeof(float) * hk * S), *k = (float *)malloc(sizeof(float) * hk * S);
            float gg[32], bb[32];
            memcpy(q, M.act + c[2], sizeof(float) * hk * S);
            memcpy(k, M.act + c[3], sizeof(float) * hk * S);
            if (fl & 2u) { /* L2-normalize q and k per head (RMSNORM with flags 3) */
                const float eps = bits_f(e[4]);
                for (unsigned h = 0; h < hk; ++h) {
                    orc_rownorm(M.act + c[2] + h * S, NULL, S, 1, 0, eps, 3u, q + h * S);
                    orc_rownorm(M.act + c[3] + h * S, NULL, S, 1, 0, eps, 3u, k + h * S);
                }
            }
            for (unsigned h = 0; h < hv; ++h) {
                const float gr = M.act[c[5] + h], br = M.act[c[6] + h];
                if (gates) { /* beta = sigmoid(beta), g = softplus(g + dt) * a (gemvqc_gdn.h:265-280) */
                    const float dt = M.act[e2[0] + h], a = M.act[e2[1] + h];
                    gg[h] = orc_unary1(gr + dt, 3) * a;
                    bb[h] = orc_unary1(br, 2);
                } else {
                    gg[h] = gr;
                    bb[h] = br;
                }
            }
            float *st = (float *)malloc(sizeof(float) * rows * S), *y = (float *)malloc(sizeof(float) * rows);
            memcpy(st, M.state + (size_t)e[0] * S, sizeof(float) * rows * S);
            /* z for the gated norm is read when the step starts (gemvqc16.h:70-71) */
            float *z = NULL, *wg = NULL;
            if (fl & 4u) {
                z = (float *)malloc(sizeof(float) * rows);
                wg = (float *)malloc(sizeof(float) * S);
                memcpy(z, M.act + e[7], sizeof(float) * rows);
                memcpy(wg, M.act + e[6], sizeof(float) * S);
            }
            orc_gdn(st, q, k, M.act + c[4], gg, bb, hv, hk, bits_f(e[2]), y, NULL, NULL);
            memcpy(M.state + (size_t)e[1] * S, st, sizeof(float) * rows * S);
            if (fl & 4u) { /* per head (y * rms scale) * w * silu(z): RMSNORM with weight, then SILU_MUL(z, .) */
                const float eps = bits_f(e[5]);
                float nrm[128];
                for (unsigned h = 0; h < hv; ++h) {
                    orc_rownorm(y + h * S, wg, S, 1, 0, eps, 0u, nrm);
                    for (unsigned j = 0; j < S; ++j) y[h * S + j] = orc_silu_mul1(z[h * S + j], nrm[j], 0);
                }
                free(z); free(wg);
            }
            /* WITH_GEMV: the next GEMV runs in the same pass; its x was read before the step unless it touches y */
            float *xcopy = NULL;
            const uint32_t *wg_cmd = NULL;
            if ((fl & 1u) && i + slots < n_cmds) {
                const uint32_t *nx = cmds + (size_t)(i + slots) * 8;
                const unsigned nyr = (nx[2] + 15) / 16 * 16;
                if (gemv_valid(nx) && (nx[1] & ~0xffu) == 0 && !(nx[6] < c[7] + rows && c[7] < nx[6] + nx[3]) &&
                    !(nx[7] < c[7] + rows && c[7] < nx[7] + nyr))
                    wg_cmd = nx;
            }
            (void)xcopy;
            memcpy(M.act + c[7], y, sizeof(float) * rows);
            free(q); free(k); free(st); free(y);
            adv = slots;
            if (wg_cmd) { /* disjoint from the step's y: same values as running it after the step */
                if (exec_gemv(&M, wg_cmd, NULL, 1)) { status = (int)i + 1; break; }
                adv = slots + 1;
            }
            if (out_adv) { /* the GEMV on the step's output (and its ADD) */
                const uint32_t *nx = cmds + (size_t)(i + slots) * 8;
                const unsigned orow = nx[2];
                if ((nx[1] & 0x400u) == 0) {
                    if (exec_gemv(&M, nx, NULL, 0)) { status = (int)i + 1; break; }
                } else {
                    const uint32_t *ad = cmds + (size_t)(i + slots + 1) * 8;
                    const unsigned r_off = ad[2] == nx[7] ? ad[3] : ad[2];
                    float *t = (float *)malloc(sizeof(float) * orow);
                    if (exec_gemv(&M, nx, t, 0)) { free(t); status = (int)i + 1; break; }
                    for (unsigned r = 0; r < orow; ++r) M.act[ad[4] + r] = t[r] + M.act[r_off + r];
                    free(t);
                }
                adv = slots + out_adv;
            }
        } else if (op == 12) { /* ATTN extension: pos = act[pos_off] (uint32 bits); store this token's k, v (F16) at
                                 pos, attend over pos + 1 */
            const unsigned nh = c[1] & 0xffu, nkv = (c[1] >> 8) & 0xffu, hd = (c[1] >> 16) * 16u;
            const unsigned slot = c[7];
            unsigned pos = 0xffffffffu;
            if (in_act(&M, c[6], 1)) memcpy(&pos, &M.act[c[6]], 4);
            const size_t slot_elems = (size_t)nkv * kv_ctx * hd; /* K, then V */
            if (nh == 0 || nkv == 0 || nh % nkv || nh / nkv > 16 || hd == 0 || hd > 512 || c[2] % 16 || c[3] % 16 || c[4] % 16 ||
                c[5] % 16 || c[6] % 16 || pos >= kv_ctx || !in_act(&M, c[2], (size_t)nh * hd) || !in_act(&M, c[3], (size_t)nkv * hd) ||
                !in_act(&M, c[4], (size_t)nkv * hd) || !in_act(&M, c[5], (size_t)nh * hd) ||
                ((size_t)slot + 1) * slot_elems * 2 * sizeof(uint16_t) > kv_bytes) {
                status = (int)i + 1;
                break;
            }
            uint16_t *kc = (uint16_t *)kv + (size_t)slot * slot_elems * 2, *vc = kc + slot_elems;
            for (unsigned h = 0; h < nkv; ++h)
                for (unsigned e = 0; e < hd; ++e) {
                    kc[((size_t)h * kv_ctx + pos) * hd + e] = orc_float_to_half(M.act[c[3] + h * hd + e]);
                    vc[((size_t)h * kv_ctx + pos) * hd + e] = orc_float_to_half(M.act[c[4] + h * hd + e]);
                }
            float *t = (float *)malloc(sizeof(float) * nh * hd);
            orc_attn(M.act + c[2], kc, vc, nh, nkv, hd, kv_ctx, pos + 1, 1.0f / sqrtf((float)hd), t);
            memcpy(M.act + c[5], t, sizeof(float) * nh * hd);
            free(t);
        } else if (op == 13) { /* ARGMAX extension: first index of the maximum */
            const unsigned n = c[1];
            if (n == 0 || c[2] % 16 || c[3] % 16 || (c[4] | c[5] | c[6] | c[7]) || !in_act(&M, c[2], n) ||
                !in_act(&M, c[3], 16)) {
                status = (int)i + 1;
                break;
            }
            unsigned best = 0;
            for (unsigned e = 1; e < n; ++e)
                if (M.act[c[2] + e] > M.act[c[2] + best]) best = e;
            const float mx = M.act[c[2] + best];
            memcpy(&M.act[c[3]], &best, 4);
            M.act[c[3] + 1] = mx;
        } else if (op == 14) { /* GET_ROW extension: row act[idx_off] (uint32 bits) of a matrix, dequantized */
            const unsigned fmt = c[1], cols = c[2];
            const uint64_t h = (uint64_t)c[3] | ((uint64_t)c[4] << 32);
            const orc_weight *w = find_w(M.ws, M.nw, h);
            uint32_t row = 0;
            if (in_act(&M, c[5], 1)) memcpy(&row, &M.act[c[5]], 4);
            if ((fmt != 2 && fmt != 8) || cols == 0 || cols % 32 || c[5] % 16 || c[6] % 16 || c[7] || !w ||
                w->format != fmt || w->cols != cols || !in_act(&M, c[5], 1) || row >= w->rows ||
                !in_act(&M, c[6], cols)) {
                status = (int)i + 1;
                break;
            }
            orc_dequantize_row(w->data + (size_t)row * orc_row_bytes(cols, fmt), cols, fmt, M.act + c[6]);
        } else if (op == 17) { /* GEMV_BATCH extension: y_m = W x_m (+ y_m) for m < batch, as batch GEMV commands */
            const unsigned fmt = c[1] & 0xffu, fl = c[1] & 0xff00u, batch = ((c[1] >> 16) & 0xffffu) + 1u;
            const unsigned rows = c[2], cols = c[3], ys = (rows + 15u) / 16u * 16u;
            const uint64_t h = (uint64_t)c[4] | ((uint64_t)c[5] << 32);
            const orc_weight *w = find_w(M.ws, M.nw, h);
            const size_t xn = (size_t)batch * cols, yn = (size_t)batch * ys;
            if ((fmt != 2 && fmt != 3 && fmt != 8) || (fl != 0 && fl != 0x400u) || rows == 0 || rows > 65536 || cols == 0 || cols > 16384 || cols % 128 || c[6] % 16 || c[7] % 16 ||
                !in_act(&M, c[6], xn) || !in_act(&M, c[7], yn) || (c[6] < c[7] + yn && c[7] < c[6] + xn) || !w ||
                w->format != fmt || w->cols != cols || w->rows != rows) {
                status = (int)i + 1;
                break;
            }
            float *tmp = (float *)malloc(sizeof(float) * rows);
            for (unsigned m = 0; m < batch; ++m) {
                float *y = M.act + c[7] + (size_t)m * ys;
                orc_gemv(w->data, M.act + c[6] + (size_t)m * cols, rows, cols, fmt, tmp, NULL);
                for (unsigned r = 0; r < rows; ++r) y[r] = fl ? tmp[r] + y[r] : tmp[r];
                for (unsigned r = rows; r < ys; ++r) y[r] = 0.0f;
            }
            free(tmp);
        } else if (op == 15 || op == 16) { /* ALLREDUCE / ALLGATHER extensions, one rank: y = x (a test that runs
                                             * several ranks' lists performs the collectives itself, between lists) */
            const unsigned n = c[1];
            const size_t x = c[2], y = c[3];
            int ok = n != 0 && n % 16 == 0 && x % 16 == 0 && y % 16 == 0 && (c[4] | c[5] | c[6] | c[7]) == 0 &&
                     in_act(&M, c[2], n) && in_act(&M, c[3], n);
            if (ok && (x != y)) ok = x + n <= y || y + n <= x;
            if (!ok) {
                status = (int)i + 1;
                break;
            }
            memmove(M.act + y, M.act + x, sizeof(float) * n);
        } else {
            status = (int)i + 1;
            break;
        }
        i += adv;
    }
    free(M.nd_row);
    return status;
}
