// ALLREDUCE of explicit (tensor-parallel) lists without NCCL: one kernel that pushes this rank's part over NVLink into
// every rank's receive buffer (CUDA IPC mappings) and adds the ranks' parts in rank order, so every rank gets the same
// bits. No fence and no flag word: every value travels as one 8-byte word {value bits, launch number} (an aligned
// 8-byte store is seen whole or not at all), and a reader waits (bounded) until each word it needs carries this
// launch's number — the exchange costs one NVLink write latency instead of a write, a system-scope fence and a flag
// round trip.
//
// Buffers (per collective slot, one slot per ALLREDUCE of a list; every rank runs the same lists, so slot s means
// the same collective on every rank): recv [2 parities][world][kCollMaxN] words of 8 bytes in each rank's memory, and
// in this rank's memory alone one launch counter per CTA of the slot. Launch k of a slot uses parity k & 1. Reuse is
// safe with two parities: a rank writes launch k + 2 into a peer only after its own launch k + 1 completed, which
// needed that peer's launch k + 1 words, which the peer wrote only after its launch k (the last reader of this
// parity) had completed.
//
// Roofline: latency (a few KB per rank); the bytes are world x n x 8 over NVLink out and in per rank.
#include "common.cuh"
#include "launch.h"
#include "peer.cuh"

namespace b200q {

__device__ __forceinline__ void st_word_sys(uint2 *p, uint32_t v, uint32_t k) {
    asm volatile("st.relaxed.sys.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(v), "r"(k) : "memory");
}
__device__ __forceinline__ uint2 ld_word_sys(const uint2 *p) {
    uint2 w;
    asm volatile("ld.relaxed.sys.global.v2.u32 {%0, %1}, [%2];" : "=r"(w.x), "=r"(w.y) : "l"(p) : "memory");
    return w;
}

// Bounded wait until the word carries launch number k; its value, or false after kWaitLimitNs.
__device__ __forceinline__ bool wait_word(const uint2 *p, uint32_t k, float &v) {
    unsigned long long t0 = 0;
    for (unsigned i = 0;; ++i) {
        const uint2 w = ld_word_sys(p);
        if (w.y == k) {
            v = __uint_as_float(w.x);
            return true;
        }
        if ((i & 255u) == 255u) {
            const unsigned long long now = global_ns();
            if (t0 == 0) t0 = now;
            else if (now - t0 > kWaitLimitNs) return false;
        }
    }
}

__global__ void __launch_bounds__(kCollChunk / 4) allreduce_peer_kernel(const __grid_constant__ CollArgs a) {
    const unsigned c = blockIdx.x, t = threadIdx.x;
    const unsigned off = c * kCollChunk + t * 4;  // this thread's 4 values
    const bool live = off < a.n;
    pdl_launch_dependents();
    pdl_wait();
    // this CTA's launch counter of the slot (this rank's memory, written by this CTA in the slot's previous launch)
    const unsigned k = *reinterpret_cast<volatile unsigned *>(a.flag_local + c) + 1u;
    const unsigned par = k & 1u;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) v = __ldcg(reinterpret_cast<const float4 *>(a.x + off));
    const float mine[4] = {v.x, v.y, v.z, v.w};
    if (live) {
        const size_t dst = (size_t(par) * a.world + a.rank) * kCollMaxN + off;
#pragma unroll 1
        for (unsigned r = 0; r < a.world; ++r) {
            if (r == a.rank) continue;
#pragma unroll
            for (unsigned e = 0; e < 4; ++e) st_word_sys(a.recv[r] + dst + e, __float_as_uint(mine[e]), k);
        }
    }
    // the parts in rank order (this rank's own from registers)
    bool ok = true;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    if (live) {
        const uint2 *base = a.recv[a.rank] + size_t(par) * a.world * kCollMaxN + off;
        for (unsigned r = 0; r < a.world && ok; ++r) {
#pragma unroll
            for (unsigned e = 0; e < 4; ++e) {
                float p = mine[e];
                if (r != a.rank) ok = wait_word(base + size_t(r) * kCollMaxN + e, k, p) && ok;
                s[e] = r == 0 ? p : fadd(s[e], p);
            }
        }
    }
    if (!ok && a.err) atomicExch(a.err, 1u);
    if (live && ok) *reinterpret_cast<float4 *>(a.y + off) = make_float4(s[0], s[1], s[2], s[3]);
    __syncthreads();  // every thread read k before the counter moves on
    if (t == 0) *reinterpret_cast<volatile unsigned *>(a.flag_local + c) = k;
}

cudaError_t launch_allreduce_peer(const CollArgs &a, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.n + kCollChunk - 1) / kCollChunk);
    cfg.blockDim = dim3(kCollChunk / 4);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, allreduce_peer_kernel, a);
}

}  // namespace b200q
