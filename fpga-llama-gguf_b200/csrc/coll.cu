// ALLREDUCE of explicit (tensor-parallel) lists without NCCL: one kernel that pushes this rank's part over NVLink into
// every rank's receive buffer (CUDA IPC mappings), raises a flag word per chunk in every rank, waits (bounded) for the
// flags of the other ranks and adds the parts in rank order. Every rank adds the same parts in the same order, so
// every rank gets the same bits.
//
// Buffers (per collective slot, one slot per ALLREDUCE of a list; every rank runs the same lists, so slot s means
// the same collective on every rank): recv [2 parities][world][kCollMaxN] floats and flags [world][kCollMaxCtas]
// words in each rank's memory. Launch k of a slot (counted by the flag word this CTA wrote for itself in launch k - 1)
// uses parity k & 1. Reuse is safe with two parities: a rank pushes launch k only after its own launch k - 1 of the
// slot completed (stream order), which needed every peer's push of launch k - 1, which each peer made only after its
// launch k - 2 (the last reader of this parity) had completed.
//
// Roofline: latency (a few KB per rank); the bytes are world x n x 4 over NVLink out and in per rank.
#include "common.cuh"
#include "launch.h"
#include "peer.cuh"

namespace b200q {

__global__ void __launch_bounds__(kCollChunk / 4) allreduce_peer_kernel(const __grid_constant__ CollArgs a) {
    const unsigned c = blockIdx.x, t = threadIdx.x;
    const unsigned off = c * kCollChunk + t * 4;  // this thread's 4 floats
    const bool live = off < a.n;
    pdl_launch_dependents();
    pdl_wait();
    // this CTA's own flag word in this rank's memory holds the slot's previous launch count (written by this CTA)
    const unsigned k = ld_acquire_sys(a.flag_local + a.rank * kCollMaxCtas + c) + 1u;
    const unsigned par = k & 1u;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) v = __ldcg(reinterpret_cast<const float4 *>(a.x + off));
    const size_t dst = (size_t(par) * a.world + a.rank) * kCollMaxN + off;
    if (live) {
#pragma unroll 1
        for (unsigned r = 0; r < a.world; ++r) *reinterpret_cast<float4 *>(a.recv[r] + dst) = v;
    }
    // every thread's pushes are visible system-wide before any flag of this CTA
    __threadfence_system();
    __syncthreads();
    if (t < a.world) st_release_sys(a.flags[t] + a.rank * kCollMaxCtas + c, k);
    bool ok = true;
    if (t < a.world && t != a.rank) ok = wait_reached(a.flag_local + t * kCollMaxCtas + c, k);
    if (!ok && a.err) atomicExch(a.err, 1u);
    if (__syncthreads_or(!ok)) return;
    if (live) {
        // volatile loads (no stale L1 lines of the parity's previous use), parts added in rank order
        const float *base = a.recv[a.rank] + size_t(par) * a.world * kCollMaxN + off;
        float4 s = __ldcv(reinterpret_cast<const float4 *>(base));
        for (unsigned r = 1; r < a.world; ++r) {
            const float4 p = __ldcv(reinterpret_cast<const float4 *>(base + size_t(r) * kCollMaxN));
            s.x = fadd(s.x, p.x);
            s.y = fadd(s.y, p.y);
            s.z = fadd(s.z, p.z);
            s.w = fadd(s.w, p.w);
        }
        *reinterpret_cast<float4 *>(a.y + off) = s;
    }
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
