// Device helpers shared by the b200q kernels (sm_100a).
//
// Rounding: every FP32 operation that must match the CPU reference bit for bit is written with the _rn
// intrinsics, so nvcc cannot contract a*b+c into one FMA (the reference's C++ rounds twice). exp/log: the reference
// calls glibc expf/logf; here they are computed in double precision and rounded once to FP32, which gives the
// correctly rounded FP32 value (glibc's results agree with it except in rare near-halfway cases; the tests use the
// reference's element-wise tolerance there).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace b200q {

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

__device__ __forceinline__ float exp_f32(float x) { return __double2float_rn(exp(double(x))); }
__device__ __forceinline__ float log_f32(float x) { return __double2float_rn(log(double(x))); }

// silu(g) = g / (1 + exp(-g)) in the reference's order (gemvq_ref.h:303-307)
__device__ __forceinline__ float silu_f32(float g) { return fdiv(g, fadd(1.0f, exp_f32(-g))); }
__device__ __forceinline__ float sigmoid_f32(float g) { return fdiv(1.0f, fadd(1.0f, exp_f32(-g))); }
// ggml softplus: x > 20 ? x : log(1 + exp(x)) (gemvq_ref.h:332-342)
__device__ __forceinline__ float softplus_f32(float x) { return x > 20.0f ? x : log_f32(fadd(1.0f, exp_f32(x))); }

__device__ __forceinline__ float half_bits_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t float_to_half_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

// 16-byte streaming load that skips L1 (weights are read once per pass).
__device__ __forceinline__ uint4 ldg_stream16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldg_stream4(const void *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ldg_stream2(const void *p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// Programmatic dependent launch: a kernel launched with the PDL attribute may start while the previous kernel in
// the stream still runs; it must call pdl_wait() before it reads anything the previous kernel writes. Weights are
// never written by a list, so they can be read before the wait.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace b200q
