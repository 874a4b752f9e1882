// Decode attention over an F16 KV cache (extension opcode 12). The reference leaves the attention core on the CPU
// (ggml F16 path); this kernel runs it on the GPU so a whole token stays on the device: the token's k and v are
// stored into the cache (F16, round to nearest even) at position pos (read from act, so a replayed graph serves
// every token; outside the slot: nothing is written and the status word says so), then per query head
// scores_t = (q . k_t) * scale over t = 0..pos, softmax with the maximum subtracted, y = sum_t p_t v_t / sum_t p_t.
// GQA: query head h reads KV head h / (n_head / n_kv_head).
//
// Split over positions (flash decoding): CTA (chunk, kv head) takes positions [chunk * C, chunk * C + C) for all G
// query heads of its KV head, so each K/V row is read once per token. The chunk's K and V rows are contiguous in the
// cache: two bulk copies bring them into shared memory. The CTA writes its chunk's maximum m, sum l and unnormalised
// output o per query head; the last CTA of a KV head to finish (counter in the sync words, reset by that CTA) merges
// the chunks: y = sum_c w_c o_c with w_c = e^(m_c - M) / sum_c e^(m_c - M) l_c. Chunks past pos exit at once. Only
// the CTA that holds pos touches row pos: it uses the token's k / v (rounded to F16) for it and stores them after
// its copies landed. FP32 sums (tolerance-checked against the CPU oracle, which sums in FP64).
#include "launch.h"
#include "peer.cuh"
#include "pipeline.cuh"
#include "quant.cuh"

namespace b200q {

constexpr unsigned kAttnThreads = 256, kAttnWarps = kAttnThreads / 32, kAttnMaxGroup = 16;
constexpr unsigned kMergeBatch = 24;  // chunk partials a merging thread holds in registers at once

__device__ __forceinline__ void half8_to_float(uint4 u, float *f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = half_bits_to_float(uint16_t(w[i] & 0xffffu));
        f[2 * i + 1] = half_bits_to_float(uint16_t(w[i] >> 16));
    }
}

struct AttnSmem {
    uint16_t *k, *v;  // [C][hd] F16 rows of the chunk
    float *q;         // [G][hd]
    float *p;         // [G][C] scores, then probabilities
    float *ml;        // [G][2] chunk maximum and sum
    float *w;         // [G][max_chunks] merge weights (last CTA)
};

__device__ __forceinline__ AttnSmem attn_smem(unsigned char *base, unsigned G, unsigned hd, unsigned C,
                                              unsigned max_chunks) {
    AttnSmem S;
    S.k = reinterpret_cast<uint16_t *>(base);
    S.v = S.k + size_t(C) * hd;
    S.q = reinterpret_cast<float *>(S.v + size_t(C) * hd);
    S.p = S.q + G * hd;
    S.ml = S.p + G * C;
    S.w = S.ml + 2 * G;
    (void)max_chunks;
    return S;
}

__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnArgs a) {
    extern __shared__ __align__(128) unsigned char attn_sm[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ unsigned last_s, ok_s;
    const unsigned G = a.n_head / a.n_kv_head, hd = a.head_dim, C = a.chunk, nvec = hd / 8;
    const AttnSmem S = attn_smem(attn_sm, G, hd, C, a.max_chunks);
    const unsigned chunk = blockIdx.x, kvh = blockIdx.y, c0 = chunk * C;
    const size_t row0 = size_t(kvh) * a.kv_ctx + c0;  // first cache row of the chunk
    // The cache rows the token attends to in this chunk, [c0, pos) (row pos is the token's own k / v), come in before
    // the wait on the previous kernel: only ATTN itself writes the cache (the row at pos, which this CTA replaces
    // after the copy), so the copy overlaps the previous kernel's end. The position is read before the wait too; it
    // is read again after the wait, and in the rare case that it changed in between (an earlier kernel of the stream
    // wrote it), the rows are copied again for the position read after the wait. Any value read early gives a copy
    // inside the slot; rows past pos are never copied, so the bytes follow the position, not the slot length.
    auto rows_for = [&](unsigned p) -> unsigned {
        if (p >= a.kv_ctx || p <= c0) return 0u;
        const unsigned r = p - c0;
        return r < C ? r : C;  // (c0 + C <= kv_ctx whenever p - c0 >= C, as p < kv_ctx)
    };
    unsigned copied = 0;  // thread 0: rows of the early copy (phase 0 of bar when non-zero)
    const uint64_t pol = evict_first_policy();
    auto issue = [&](unsigned rows) {
        const unsigned bytes = rows * hd * 2;
        mbar_expect_tx(&bar, 2 * bytes);
        bulk_copy(S.k, a.kcache + row0 * hd, bytes, &bar, pol);
        bulk_copy(S.v, a.vcache + row0 * hd, bytes, &bar, pol);
    };
    // thread 0: bounded wait for phase `parity`; after a timeout one more bounded wait, so that a copy still in
    // flight lands before the CTA exits
    auto land = [&](unsigned parity) -> bool {
        if (mbar_wait(&bar, parity)) return true;
        mbar_wait(&bar, parity);
        return false;
    };
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
        copied = rows_for(__float_as_uint(*reinterpret_cast<const volatile float *>(a.pos)));
        if (copied) issue(copied);
    }
    pdl_wait();
    pdl_launch_dependents();  // the next kernel may stage its weights while this one runs
    peer_wait_rows_cta(a.pw);
    const unsigned pos = __float_as_uint(*a.pos);
    const unsigned T = pos + 1;
    const bool active = pos < a.kv_ctx && c0 < T;
    if (!active) {  // outside the slot, or a chunk past pos: let the copies land, then leave
        if (pos >= a.kv_ctx && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && a.status)
            atomicOr(a.status, 2u);
        if (threadIdx.x == 0 && copied && !land(0u) && a.err) atomicExch(a.err, 1u);
        return;
    }
    const unsigned n_chunks = (T + C - 1) / C, cn = T - c0 < C ? T - c0 : C;
    const unsigned warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    for (unsigned e = threadIdx.x; e < G * hd; e += kAttnThreads) S.q[e] = a.q[size_t(kvh) * G * hd + e];
    if (threadIdx.x == 0) {
        const unsigned need = rows_for(pos);
        ok_s = copied == 0 || land(0u);
        if (ok_s && need > copied) {  // the position changed after the early read: copy its rows again
            issue(need);
            ok_s = land(copied ? 1u : 0u);
        }
        if (!ok_s && a.err) atomicExch(a.err, 1u);
    }
    __syncthreads();
    if (!ok_s) return;
    if (pos < c0 + cn) {  // this CTA holds the new row: use it, then store it in the cache
        const size_t r = size_t(pos - c0) * hd;
        for (unsigned e = threadIdx.x; e < hd; e += kAttnThreads) {
            const uint16_t kb = float_to_half_bits(a.k[size_t(kvh) * hd + e]);
            const uint16_t vb = float_to_half_bits(a.v[size_t(kvh) * hd + e]);
            S.k[r + e] = kb;
            S.v[r + e] = vb;
            a.kcache[(row0 + pos - c0) * hd + e] = kb;
            a.vcache[(row0 + pos - c0) * hd + e] = vb;
        }
    }
    __syncthreads();
    // scores: warp w takes rows w, w + 8, ...; lanes split the row in 8-value vectors
    for (unsigned i = warp; i < cn; i += kAttnWarps) {
        float acc[kAttnMaxGroup];
#pragma unroll
        for (unsigned g = 0; g < kAttnMaxGroup; ++g) acc[g] = 0.0f;
        for (unsigned vec = lane; vec < nvec; vec += 32) {
            float k8[8];
            half8_to_float(reinterpret_cast<const uint4 *>(S.k + size_t(i) * hd)[vec], k8);
#pragma unroll
            for (unsigned g = 0; g < kAttnMaxGroup; ++g) {
                if (g < G) {
                    const float4 qa = reinterpret_cast<const float4 *>(S.q + g * hd)[2 * vec];
                    const float4 qb = reinterpret_cast<const float4 *>(S.q + g * hd)[2 * vec + 1];
                    acc[g] = fmaf(qa.x, k8[0], acc[g]);
                    acc[g] = fmaf(qa.y, k8[1], acc[g]);
                    acc[g] = fmaf(qa.z, k8[2], acc[g]);
                    acc[g] = fmaf(qa.w, k8[3], acc[g]);
                    acc[g] = fmaf(qb.x, k8[4], acc[g]);
                    acc[g] = fmaf(qb.y, k8[5], acc[g]);
                    acc[g] = fmaf(qb.z, k8[6], acc[g]);
                    acc[g] = fmaf(qb.w, k8[7], acc[g]);
                }
            }
        }
#pragma unroll
        for (unsigned g = 0; g < kAttnMaxGroup; ++g) {
            if (g < G) {
                float s = acc[g];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (lane == 0) S.p[g * C + i] = s * a.scale;
            }
        }
    }
    __syncthreads();
    // chunk softmax statistics: warp w takes query heads w, w + 8, ...
    for (unsigned g = warp; g < G; g += kAttnWarps) {
        float mx = -INFINITY;
        for (unsigned i = lane; i < cn; i += 32) mx = fmaxf(mx, S.p[g * C + i]);
        mx = warp_max(mx);
        float sum = 0.0f;
        for (unsigned i = lane; i < cn; i += 32) {
            const float e = expf(S.p[g * C + i] - mx);
            S.p[g * C + i] = e;
            sum += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            S.ml[2 * g] = mx;
            S.ml[2 * g + 1] = sum;
        }
    }
    __syncthreads();
    // unnormalised chunk output: item (g, vec) per thread
    const size_t part_stride = size_t(hd) + 4;  // hd outputs, maximum, sum, 2 pad (16-byte aligned records)
    for (unsigned it = threadIdx.x; it < G * nvec; it += kAttnThreads) {
        const unsigned g = it / nvec, vec = it % nvec;
        float o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll 4
        for (unsigned i = 0; i < cn; ++i) {
            float v8[8];
            half8_to_float(reinterpret_cast<const uint4 *>(S.v + size_t(i) * hd)[vec], v8);
            const float p = S.p[g * C + i];
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = fmaf(p, v8[j], o[j]);
        }
        float *dst = a.part + (size_t(kvh * G + g) * a.max_chunks + chunk) * part_stride;
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[vec * 8 + j] = o[j];
        if (vec == 0) {
            dst[hd] = S.ml[2 * g];
            dst[hd + 1] = S.ml[2 * g + 1];
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned done = atomicAdd(a.counters + kvh, 1u);
        last_s = done == n_chunks - 1;
        if (last_s) a.counters[kvh] = 0;  // every other chunk has counted: ready for the next launch
    }
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    // the chunks' partial outputs of this thread's first item, requested now so that they arrive with the chunk
    // statistics read below (one round trip for both)
    const unsigned nv4 = hd / 4;
    float4 pv[kMergeBatch];
    if (threadIdx.x < G * nv4) {
        const unsigned g = threadIdx.x / nv4, e4 = threadIdx.x % nv4;
        const float *base = a.part + size_t(kvh * G + g) * a.max_chunks * part_stride + 4 * e4;
#pragma unroll
        for (unsigned u = 0; u < kMergeBatch; ++u)
            if (u < n_chunks) pv[u] = __ldcg(reinterpret_cast<const float4 *>(base + u * part_stride));
    }
    // merge weights per (query head, chunk): warp g reduces over the chunks
    for (unsigned g = warp; g < G; g += kAttnWarps) {
        const float *base = a.part + size_t(kvh * G + g) * a.max_chunks * part_stride;
        float M = -INFINITY;
        for (unsigned c = lane; c < n_chunks; c += 32) M = fmaxf(M, __ldcg(base + c * part_stride + hd));
        M = warp_max(M);
        float L = 0.0f;
        for (unsigned c = lane; c < n_chunks; c += 32) {
            const float e = expf(__ldcg(base + c * part_stride + hd) - M);
            S.w[g * a.max_chunks + c] = e;
            L = fmaf(e, __ldcg(base + c * part_stride + hd + 1), L);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        const float inv = 1.0f / L;
        for (unsigned c = lane; c < n_chunks; c += 32) S.w[g * a.max_chunks + c] *= inv;
    }
    __syncthreads();
    // four outputs per thread: one 16-byte load per chunk, a batch of chunks' loads in flight before their sums (in
    // chunk order); the first batch of the first item is already here
    for (unsigned it = threadIdx.x; it < G * nv4; it += kAttnThreads) {
        const unsigned g = it / nv4, e4 = it % nv4;
        const float *base = a.part + size_t(kvh * G + g) * a.max_chunks * part_stride + 4 * e4;
        const float *w = S.w + g * a.max_chunks;
        float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
        for (unsigned c0m = 0; c0m < n_chunks; c0m += kMergeBatch) {
            if (c0m > 0 || it != threadIdx.x) {
#pragma unroll
                for (unsigned u = 0; u < kMergeBatch; ++u)
                    if (c0m + u < n_chunks)
                        pv[u] = __ldcg(reinterpret_cast<const float4 *>(base + (c0m + u) * part_stride));
            }
#pragma unroll
            for (unsigned u = 0; u < kMergeBatch; ++u) {
                if (c0m + u < n_chunks) {
                    const float wc = w[c0m + u];
                    y.x = fmaf(wc, pv[u].x, y.x);
                    y.y = fmaf(wc, pv[u].y, y.y);
                    y.z = fmaf(wc, pv[u].z, y.z);
                    y.w = fmaf(wc, pv[u].w, y.w);
                }
            }
        }
        const size_t o = size_t(kvh * G + g) * hd + 4 * e4;
        const float yv[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
        for (unsigned q = 0; q < 4; ++q) {
            a.y[o + q] = yv[q];
            if (a.gate_y) {  // the fused SILU_MUL (sigmoid) on this output element
                const size_t gi = size_t((o + q) / a.gate_row) * a.gate_stride + (o + q) % a.gate_row;
                a.gate_y[o + q] = fmul(sigmoid_f32(a.gate_g[gi]), yv[q]);
            }
        }
    }
}

unsigned attn_chunk(unsigned kv_ctx, unsigned n_kv_head, unsigned sms) {
    // about one CTA per SM over the whole slot, at least 16 positions per CTA
    const unsigned per = (kv_ctx * n_kv_head + sms - 1) / sms;
    return per <= 16 ? 16u : (per + 15) / 16 * 16;
}

size_t attn_smem_bytes(unsigned n_head, unsigned n_kv_head, unsigned head_dim, unsigned chunk, unsigned max_chunks) {
    const size_t G = n_head / n_kv_head;
    return 2 * size_t(chunk) * head_dim * 2 + sizeof(float) * (G * head_dim + G * chunk + 2 * G + G * max_chunks);
}

cudaError_t launch_attn(const AttnArgs &a, cudaStream_t st, bool pdl) {
    const cudaError_t e = ensure_smem_attr(reinterpret_cast<const void *>(attn_kernel), 200 * 1024);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.max_chunks, a.n_kv_head);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = attn_smem_bytes(a.n_head, a.n_kv_head, a.head_dim, a.chunk, a.max_chunks);
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
