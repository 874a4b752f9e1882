// C entry points over the reference's own CPU arithmetic — TEST INFRASTRUCTURE ONLY (the checker of the oracle
// restatement, and the timed "reference" CPU baseline of bench.py).
//
// Compiled by oracle/Makefile from the reference's sources where they lie (fpga/src/gemvq_ref.h by include path;
// nothing is copied) into oracle/_ref/libgemvq_ref.so. Each function forwards to one gemvq_ref:: function:
//   ref_gemv           -> gemvq_ref::reference          (gemvq_ref.h:231-265; Q4_0/Q8_0/Q4_1/Q5_K/Q6_K)
//   ref_gemv_rows_omp  -> the same on row slices, OpenMP over slices (rows are independent; CPU baseline)
//   ref_quantize_q8_k  -> gemvq_ref::quantize_q8_k      (gemvq_ref.h:62-81)
//   ref_half/float     -> half_to_float / float_to_half (gemvq_ref.h:16-52)
//   ref_rownorm        -> gemvq_ref::rownorm            (gemvq_ref.h:309-324)
//   ref_rmsnorm        -> gemvq_ref::rmsnorm            (gemvq_ref.h:286-295)
//   ref_silu_mul/unary/conv/add/mul -> gemvq_ref.h:297-358
//   ref_gdn            -> gemvq_ref::gdn                (gemvq_ref.h:360-397)
//   ref_within_*       -> the reference's tolerances    (gemvq_ref.h:267-284, 399-402)
#include "gemvq_ref.h"
#include <cstring>

#define REF_API extern "C" __attribute__((visibility("default")))

REF_API float ref_half_to_float(uint16_t h) { return gemvq_ref::half_to_float(h); }
REF_API uint16_t ref_float_to_half(float f) { return gemvq_ref::float_to_half(f); }

REF_API int ref_gemv(const uint8_t *w, const float *x, unsigned rows, unsigned cols, unsigned format, float *y,
                     double *mag) {
    std::vector<double> m;
    const std::vector<float> r = gemvq_ref::reference(w, x, rows, cols, format, m);
    std::memcpy(y, r.data(), sizeof(float) * rows);
    if (mag) std::memcpy(mag, m.data(), sizeof(double) * rows);
    return 0;
}

static size_t ref_row_bytes(unsigned cols, unsigned format) {
    switch (format) {
    case 2: return size_t(cols / 32) * 18;
    case 3: return size_t(cols / 32) * 20;
    case 8: return size_t(cols / 32) * 34;
    case 13: return size_t(cols / 256) * 176;
    case 14: return size_t(cols / 256) * 210;
    default: return 0;
    }
}

// The same GEMV split into `slices` row ranges run in parallel (each slice re-quantizes x, as the reference's
// function does per call).
REF_API int ref_gemv_rows_omp(const uint8_t *w, const float *x, unsigned rows, unsigned cols, unsigned format,
                              float *y, int slices) {
    const size_t rb = ref_row_bytes(cols, format);
    if (rb == 0 || slices < 1) return -1;
#pragma omp parallel for schedule(static)
    for (int s = 0; s < slices; ++s) {
        const unsigned r0 = unsigned(uint64_t(rows) * s / slices), r1 = unsigned(uint64_t(rows) * (s + 1) / slices);
        if (r1 <= r0) continue;
        std::vector<double> m;
        const std::vector<float> r = gemvq_ref::reference(w + size_t(r0) * rb, x, r1 - r0, cols, format, m);
        std::memcpy(y + r0, r.data(), sizeof(float) * (r1 - r0));
    }
    return 0;
}

REF_API void ref_quantize_q8_k(const float *x, unsigned n, int8_t *q, float *d) {
    std::vector<int8_t> qq;
    std::vector<float> dd;
    gemvq_ref::quantize_q8_k(x, n, qq, dd);
    std::memcpy(q, qq.data(), n);
    std::memcpy(d, dd.data(), sizeof(float) * (n / 256));
}

REF_API void ref_rownorm(const float *x, const float *w, unsigned n, unsigned rows, float eps, unsigned flags,
                         float *y) {
    const std::vector<float> r = gemvq_ref::rownorm(x, w, n, rows, eps, flags);
    std::memcpy(y, r.data(), sizeof(float) * size_t(n) * rows);
}

REF_API void ref_rmsnorm(const float *x, const float *w, unsigned n, float eps, float *y) {
    const std::vector<float> r = gemvq_ref::rmsnorm(x, w, n, eps);
    std::memcpy(y, r.data(), sizeof(float) * n);
}

REF_API void ref_silu_mul(const float *g, const float *u, unsigned n, float *y) {
    const std::vector<float> r = gemvq_ref::silu_mul(g, u, n);
    std::memcpy(y, r.data(), sizeof(float) * n);
}

REF_API void ref_unary(const float *x, unsigned n, unsigned kind, float *y) {
    const std::vector<float> r = gemvq_ref::unary(x, n, kind);
    std::memcpy(y, r.data(), sizeof(float) * n);
}

REF_API void ref_add(const float *a, const float *b, unsigned n, float *y) {
    const std::vector<float> r = gemvq_ref::add(a, b, n);
    std::memcpy(y, r.data(), sizeof(float) * n);
}

REF_API void ref_mul(const float *a, const float *b, unsigned n, float *y) {
    const std::vector<float> r = gemvq_ref::mul(a, b, n);
    std::memcpy(y, r.data(), sizeof(float) * n);
}

REF_API void ref_conv(const float *state, const float *x, const float *w, unsigned ch, int silu, float *y,
                      float *new_state) {
    std::vector<float> ns;
    const std::vector<float> r = gemvq_ref::conv(state, x, w, ch, silu != 0, ns);
    std::memcpy(y, r.data(), sizeof(float) * ch);
    std::memcpy(new_state, ns.data(), sizeof(float) * ch * 3);
}

REF_API void ref_gdn(float *state, const float *q, const float *k, const float *v, const float *g,
                     const float *beta, unsigned hv, unsigned hk, float scale, float *y, double *y_mag,
                     double *s_mag) {
    std::vector<float> st(state, state + size_t(hv) * 128 * 128);
    std::vector<double> ym, sm;
    const std::vector<float> r = gemvq_ref::gdn(st, q, k, v, g, beta, hv, hk, scale, ym, sm);
    std::memcpy(state, st.data(), sizeof(float) * st.size());
    std::memcpy(y, r.data(), sizeof(float) * r.size());
    if (y_mag) std::memcpy(y_mag, ym.data(), sizeof(double) * ym.size());
    if (s_mag) std::memcpy(s_mag, sm.data(), sizeof(double) * sm.size());
}

REF_API int ref_within_tolerance(float got, float ref, double magnitude) {
    return gemvq_ref::within_tolerance(got, ref, magnitude) ? 1 : 0;
}
REF_API int ref_within_elementwise(float got, float ref) { return gemvq_ref::within_elementwise(got, ref) ? 1 : 0; }
