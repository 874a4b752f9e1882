// Decode attention over an F16 KV cache (extension opcode 12). The reference leaves the attention core on the CPU
// (ggml F16 path); this kernel runs it on the GPU so a whole token stays on the device: the token's k and v are
// stored into the cache (F16, round to nearest even) at position pos (read from act, so a replayed graph serves
// every token; outside the slot: nothing is written and the status word says so), then per query head
// scores_t = (q . k_t) * scale over t = 0..pos, softmax with the maximum subtracted, y = sum_t p_t v_t / sum_t p_t.
// GQA: query head h reads KV head h / (n_head / n_kv_head). One CTA per query head; FP32 sums (tolerance-checked
// against the CPU oracle, which sums in FP64).
#include "launch.h"
#include "quant.cuh"

namespace b200q {

constexpr unsigned kAttnThreads = 256;

__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnArgs a) {
    extern __shared__ float sm[];
    float *qsh = sm;               // head_dim
    float *p = sm + a.head_dim;    // pos + 1 scores (room for kv_ctx)
    __shared__ float redf[32];
    pdl_wait();
    const unsigned pos = __float_as_uint(*a.pos);
    if (pos >= a.kv_ctx) {
        if (blockIdx.x == 0 && threadIdx.x == 0 && a.status) atomicOr(a.status, 2u);
        return;
    }
    const unsigned h = blockIdx.x, group = a.n_head / a.n_kv_head, kvh = h / group, hd = a.head_dim;
    const unsigned T = pos + 1, warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = kAttnThreads / 32;
    const size_t kv_row = (size_t(kvh) * a.kv_ctx + pos) * hd;
    for (unsigned e = threadIdx.x; e < hd; e += kAttnThreads) {
        qsh[e] = a.q[size_t(h) * hd + e];
        if (h % group == 0) {
            a.kcache[kv_row + e] = float_to_half_bits(a.k[size_t(kvh) * hd + e]);
            a.vcache[kv_row + e] = float_to_half_bits(a.v[size_t(kvh) * hd + e]);
        }
    }
    __syncthreads();
    const uint16_t *kc = a.kcache + size_t(kvh) * a.kv_ctx * hd;
    const uint16_t *vc = a.vcache + size_t(kvh) * a.kv_ctx * hd;
    for (unsigned t = warp; t < T; t += nw) {
        float s = 0.0f;
        for (unsigned e = lane; e < hd; e += 32) {
            const float kv = t == pos ? half_bits_to_float(float_to_half_bits(a.k[size_t(kvh) * hd + e]))
                                        : half_bits_to_float(kc[size_t(t) * hd + e]);
            s = fmaf(qsh[e], kv, s);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) p[t] = s * a.scale;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (unsigned t = threadIdx.x; t < T; t += kAttnThreads) mx = fmaxf(mx, p[t]);
    mx = warp_max(mx);
    if (lane == 0) redf[warp] = mx;
    __syncthreads();
    mx = redf[0];
    for (unsigned w = 1; w < nw; ++w) mx = fmaxf(mx, redf[w]);
    __syncthreads();
    float sum = 0.0f;
    for (unsigned t = threadIdx.x; t < T; t += kAttnThreads) {
        const float e = expf(p[t] - mx);
        p[t] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) redf[warp] = sum;
    __syncthreads();
    sum = 0.0f;
    for (unsigned w = 0; w < nw; ++w) sum += redf[w];
    const float inv = 1.0f / sum;
    for (unsigned e = threadIdx.x; e < hd; e += kAttnThreads) {
        float acc = 0.0f;
        for (unsigned t = 0; t < T; ++t) {
            const float vv = t == pos ? half_bits_to_float(float_to_half_bits(a.v[size_t(kvh) * hd + e]))
                                        : half_bits_to_float(vc[size_t(t) * hd + e]);
            acc = fmaf(p[t], vv, acc);
        }
        a.y[size_t(h) * hd + e] = acc * inv;
    }
}

cudaError_t launch_attn(const AttnArgs &a, cudaStream_t st, bool pdl) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_head);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = sizeof(float) * (a.head_dim + a.kv_ctx);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_kernel, a);
}

// ---- TRACE: one timestamp per event (global nanosecond timer) and the log writer --------------------------------
__global__ void trace_stamp_kernel(unsigned long long *slot) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    *slot = t;
}

// Log layout of the reference's TRACE opcode (gemvqc16.h:92-98): a header word (float lane 0: stored events,
// lane 1: all events), then 8 events per 16-float word as 64-bit entries: bits 31:0 the time since the list started
// (here nanoseconds of the GPU timer instead of kernel cycles), bits 47:32 the command index, bits 49:48 the kind.
__global__ void trace_write_kernel(const unsigned long long *stamps, const uint32_t *tags, unsigned n, float *log) {
    const unsigned stored = n < 512 ? n : 512;
    for (unsigned i = threadIdx.x; i < 16; i += blockDim.x)
        reinterpret_cast<uint32_t *>(log)[i] = i == 0 ? stored : (i == 1 ? n : 0u);
    const unsigned words = (stored + 7) / 8;
    uint32_t *ev = reinterpret_cast<uint32_t *>(log + 16);
    for (unsigned i = threadIdx.x; i < words * 8; i += blockDim.x) {
        uint32_t lo = 0, hi = 0;
        if (i < stored) {
            lo = uint32_t(stamps[i] - stamps[0]);
            hi = tags[i];
        }
        ev[2 * i] = lo;
        ev[2 * i + 1] = hi;
    }
}

cudaError_t launch_trace_stamp(unsigned long long *slot, cudaStream_t st) {
    trace_stamp_kernel<<<1, 1, 0, st>>>(slot);
    return cudaGetLastError();
}

cudaError_t launch_trace_write(const unsigned long long *stamps, const uint32_t *tags, unsigned n, float *log,
                               cudaStream_t st) {
    trace_write_kernel<<<1, 256, 0, st>>>(stamps, tags, n, log);
    return cudaGetLastError();
}

}  // namespace b200q
