// Kernel launchers (host side of the .cu files), called by the executor in api.cpp. Every launcher takes the
// context stream; `pdl` launches with programmatic stream serialization so the kernel may start while the
// previous one drains (each kernel calls griddepcontrol.wait before reading what earlier kernels wrote).
#pragma once
#include <cuda_runtime.h>

#include <mutex>
#include <set>
#include <utility>

#include "kernel_args.h"
#include "plan.h"

namespace b200q {

// Raise a kernel's dynamic shared-memory limit once per device (the attribute is per device and function). Callers
// hold the current device; safe from several threads.
inline cudaError_t ensure_smem_attr(const void *func, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<int, const void *>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({dev, func})) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.insert({dev, func});
    return e;
}

struct EwArgs {
    unsigned op = 0;      // 3 ADD, 4 SILU_MUL, 5 MUL, 6 UNARY
    unsigned n = 0;
    const float *a = nullptr;
    const float *b = nullptr;
    float *y = nullptr;
    unsigned row = 0, stride = 0;  // strided a (UNARY x / SILU_MUL g): rows of `row` floats every `stride` floats
    unsigned kind = 0;    // UNARY kind
    unsigned sigmoid = 0; // SILU_MUL sigmoid flag
    PeerWait pw;
};

struct GdnArgs {
    unsigned hv = 0, hk = 0;
    const float *q = nullptr, *k = nullptr, *v = nullptr, *g = nullptr, *beta = nullptr;
    const float *dt = nullptr, *a = nullptr;  // gates (null: g, beta used as they are)
    const float *z = nullptr, *wn = nullptr;  // gated RMS norm (null: plain y)
    const float *state_in = nullptr;
    float *state_out = nullptr;
    float *y = nullptr;
    float scale = 0.0f, l2_eps = 0.0f, rms_eps = 0.0f;
    unsigned l2 = 0;
    uint8_t *img = nullptr;  // when set: y also as the quantized x image of the next GEMV (one Q8_0 / Q8_1 block per CTA)
    unsigned img_act = 0;
    PeerWait pw;
};

struct AttnArgs {
    unsigned n_head = 0, n_kv_head = 0, head_dim = 0, kv_ctx = 0;
    const float *pos = nullptr;                     // the token position (uint32 bits)
    unsigned *status = nullptr;                     // bit 1 set when the position is outside the slot
    const float *q = nullptr, *k = nullptr, *v = nullptr;
    float *y = nullptr;
    uint16_t *kcache = nullptr, *vcache = nullptr;  // [n_kv_head][kv_ctx][head_dim] F16 each
    float scale = 0.0f;
    unsigned chunk = 16, max_chunks = 0;            // positions per CTA; CTAs per KV head (kv_ctx / chunk)
    float *part = nullptr;      // [n_head][max_chunks][head_dim + 4] chunk outputs, maximum, sum, pad
    unsigned *counters = nullptr;  // [n_kv_head] finished chunks (zero between launches)
    unsigned *err = nullptr;       // set when a bounded wait for the chunk copies ran out
    PeerWait pw;
    // fused gate (SILU_MUL with the sigmoid flag on y): yg[e] = sigmoid(g[(e / row) * stride + e % row]) * y[e]
    const float *gate_g = nullptr;
    float *gate_y = nullptr;
    unsigned gate_row = 0, gate_stride = 0;
};

// A run of RMSNORM (stored) / ROPE commands in one launch: one CTA per row of a job; a job is a norm, a ROPE, or a
// norm followed by the ROPE of the rows it stored.
struct RowJobArgs {
    const float *x = nullptr, *w = nullptr;  // norm input rows (xstride floats apart), weight (null: none)
    float *y = nullptr;                      // norm output rows (n floats apart)
    unsigned n = 0, xstride = 0, flags = 0;  // RMSNORM flags bits 0..1
    float eps = 0.0f;
    const float *rx = nullptr, *cs = nullptr;  // ROPE input rows (the norm's output when both), cos/sin row
    float *ry = nullptr;
    unsigned nd = 0, ne0 = 0;                // ROPE dims (0: no ROPE), row length
    unsigned rows = 0, row0 = 0;             // rows of the job, its first CTA
    bool norm = false;
};
struct RowOpsArgs {
    RowJobArgs job[kMaxRowJobs];
    unsigned n_jobs = 0, total_rows = 0;
    PeerWait pw;
};

// fill in the shared-memory plan of a pass (stages, result buffers) and return its dynamic shared memory
void plan_gemv_q8(GemvArgs &a, size_t &smem);
unsigned gemv_q8_warps_per_cta();
bool gemv_q8_supported(unsigned fa, unsigned fb);
unsigned gemv_q8_resident_ctas(unsigned fa, unsigned fb, size_t smem, cudaStream_t st);
unsigned gemv_q8_cluster();
void plan_gemv_kq(GemvArgs &a, size_t &smem);
cudaError_t launch_gemv_q8(const GemvArgs &a, unsigned fa, unsigned fb, unsigned grid, size_t smem, cudaStream_t st,
                           bool pdl);
cudaError_t launch_gemv_kq(const GemvArgs &a, unsigned grid, size_t smem, cudaStream_t st, bool pdl);
cudaError_t launch_quantize(const QuantArgs &a, cudaStream_t st);
// GEMV_BATCH: activation rows one launch of gemv_batch_kernel takes (0: the matrix's panels do not fit), and the
// launches of one command (the quantizer, then one or more batch launches)
unsigned gemv_batch_rows_per_launch(const MatrixView &w, unsigned cols);
cudaError_t launch_gemv_batch(const BatchArgs &a, unsigned sms, cudaStream_t st, bool pdl);
// GEMV_BATCH of more than kBatchMax rows: bytes of the quantized-token image, and the two launches (quantizer,
// tensor-core GEMM); a.xq must hold gemm_image_bytes(a.cols, a.tokens) bytes.
size_t gemm_image_bytes(unsigned cols, unsigned tokens);
cudaError_t launch_gemm(GemmArgs a, cudaStream_t st, bool pdl);
cudaError_t launch_rmsnorm(const float *x, const float *w, float *y, unsigned n, unsigned rows, unsigned stride,
                           float eps, unsigned flags, const PeerWait &pw, cudaStream_t st, bool pdl);
cudaError_t launch_ew(const EwArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_conv(const float *x, const float *w, float *y, const float *s_src, float *s_dst, unsigned ch,
                        unsigned use_silu, const PeerWait &pw, cudaStream_t st, bool pdl);
cudaError_t launch_rope(const float *x, const float *cs, float *y, unsigned n_dims, unsigned ne0, unsigned rows,
                        const PeerWait &pw, cudaStream_t st, bool pdl);
cudaError_t launch_argmax(const float *x, unsigned n, float *y, unsigned long long *slot, unsigned *counter,
                          const PeerWait &pw, cudaStream_t st, bool pdl);
cudaError_t launch_get_row(const MatrixView &w, unsigned cols, const float *idx, float *y, unsigned *status,
                           const PeerWait &pw, cudaStream_t st, bool pdl);
cudaError_t launch_gdn(const GdnArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_peer_wait(const PeerWait &pw, cudaStream_t st, bool pdl);
cudaError_t launch_rowops(const RowOpsArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_attn(const AttnArgs &a, cudaStream_t st, bool pdl);
unsigned attn_chunk(unsigned kv_ctx, unsigned n_kv_head, unsigned sms);
size_t attn_smem_bytes(unsigned n_head, unsigned n_kv_head, unsigned head_dim, unsigned chunk, unsigned max_chunks);
cudaError_t launch_allreduce_peer(const CollArgs &a, cudaStream_t st, bool pdl);
// the chain's shared-memory plan (stages, term buffers, x image); false when a pass does not fit
bool plan_gemv_chain(ChainArgs &a, size_t &smem);
cudaError_t launch_gemv_chain(const ChainArgs &a, unsigned grid, size_t smem, cudaStream_t st, bool pdl);
cudaError_t launch_trace_stamp(unsigned long long *slot, cudaStream_t st);
cudaError_t launch_trace_write(const unsigned long long *stamps, const uint32_t *tags, unsigned n_events,
                               float *log, cudaStream_t st);

}  // namespace b200q
