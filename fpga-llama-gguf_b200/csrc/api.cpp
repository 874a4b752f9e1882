// C ABI of b200q (include/b200q.h): the context, the one-time weight upload, the executor that turns a planned
// command list into kernel launches on the context stream, CUDA Graph capture of whole lists, the bit-exactness
// check entry points and the NCCL row sharding.
//
// Reference counterparts: the XRT backend's device plumbing in llama.cpp/overlay/ggml/src/ggml-xrt/ggml-xrt.cpp —
// context init (:2794-2983), weight upload (:735-765), act input/output copies (:1136-1143, :1428-1451), state
// I/O (:455-500), launch + wait (:1241-1280), feature probe (:1284-1300), disable after failure (:2761-2770).
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/b200q.h"
#include "launch.h"
#include "layout.h"
#include "plan.h"

using namespace b200q;

namespace {

// ---- NCCL, loaded on first use (the library has no link-time dependency on it) ---------------------------------
typedef int nccl_result;
typedef void *nccl_comm;
struct NcclUniqueId { char internal[128]; };
struct NcclApi {
    bool loaded = false;
    void *h = nullptr;
    nccl_result (*get_unique_id)(NcclUniqueId *) = nullptr;
    nccl_result (*comm_init_rank)(nccl_comm *, int, NcclUniqueId, int) = nullptr;
    nccl_result (*all_gather)(const void *, void *, size_t, int, nccl_comm, cudaStream_t) = nullptr;
    nccl_result (*all_reduce)(const void *, void *, size_t, int, int, nccl_comm, cudaStream_t) = nullptr;
    nccl_result (*comm_destroy)(nccl_comm) = nullptr;
    const char *(*get_error_string)(nccl_result) = nullptr;
};
NcclApi g_nccl;
std::mutex g_nccl_mu;
constexpr int kNcclFloat32 = 7, kNcclSum = 0;

bool load_nccl(std::string &err) {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (g_nccl.loaded) return true;
    const char *names[] = {"libnccl.so.2", "libnccl.so"};
    for (const char *n : names) {
        g_nccl.h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
        if (g_nccl.h) break;
    }
    if (!g_nccl.h) {
        err = "libnccl.so.2 not found";
        return false;
    }
    g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(dlsym(g_nccl.h, "ncclGetUniqueId"));
    g_nccl.comm_init_rank = reinterpret_cast<decltype(g_nccl.comm_init_rank)>(dlsym(g_nccl.h, "ncclCommInitRank"));
    g_nccl.all_gather = reinterpret_cast<decltype(g_nccl.all_gather)>(dlsym(g_nccl.h, "ncclAllGather"));
    g_nccl.all_reduce = reinterpret_cast<decltype(g_nccl.all_reduce)>(dlsym(g_nccl.h, "ncclAllReduce"));
    g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(dlsym(g_nccl.h, "ncclCommDestroy"));
    g_nccl.get_error_string = reinterpret_cast<decltype(g_nccl.get_error_string)>(dlsym(g_nccl.h, "ncclGetErrorString"));
    if (!g_nccl.get_unique_id || !g_nccl.comm_init_rank || !g_nccl.all_gather || !g_nccl.all_reduce ||
        !g_nccl.comm_destroy) {
        err = "libnccl.so.2 lacks an entry point";
        return false;
    }
    g_nccl.loaded = true;
    return true;
}

constexpr size_t kSnapFloats = size_t(1) << 20;  // snapshot scratch (overlapping in/out ranges)
constexpr unsigned kMaxTraceEvents = 4096;
// device words after the status words: per-KV-head chunk counters of ATTN, the ARGMAX combine slot
constexpr unsigned kSyncAttnWord = 256, kSyncArgmaxWord = 512;
constexpr size_t kAttnPartFloats = size_t(1) << 22;  // ATTN chunk outputs (16 MiB)

// B200Q_FEATURE_MASK bits that switch the executor's fusions off (include/b200q.h): the reference's feature bits
// of the fused forms this library also fuses internally, then this library's own
constexpr uint32_t kMaskGroups = 1u << 3, kMaskDeferNorm = 1u << 9, kMaskGdnOut = 1u << 15;
constexpr uint32_t kMaskImage = 1u << 16, kMaskNsq = 1u << 17, kMaskPdl = 1u << 18, kMaskRowOps = 1u << 19,
                   kMaskAttnGate = 1u << 20, kMaskChains = 1u << 21;
constexpr unsigned kMaxChains = 64;  // persistent GEMV chains per list (each has its own counter block)
// every fusion on but the persistent chains: measured slower than the chained passes' own kernels (one CTA per SM
// cannot hide the x preparation and the uneven end of each pass; 171 vs 139 us per 6-layer stack step)
constexpr uint32_t kDefaultFeatureMask = 0xFFFFFFFFu & ~kMaskChains;
// feature bits a mask never hides: the weight formats and the Q6_K layout (reference ggml-xrt.cpp:1298)
constexpr uint32_t kFeatureKeep = 0xFFFF0000u | 1u | 2u | 4u | (1u << 13);

}  // namespace

struct b200q_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int sms = 148;
    uint8_t *warena = nullptr;
    size_t wbytes = 0, wused = 0;
    float *act = nullptr;
    size_t act_floats = 0;
    float *state = nullptr;
    size_t state_rows = 0;
    uint16_t *kv = nullptr;
    size_t kv_bytes = 0;
    unsigned kv_ctx = 0;
    // scratch: pre-quantized x, the stored deferred norm row, snapshots, debug outputs, trace stamps
    int8_t *xq = nullptr;
    float *xd = nullptr, *xs = nullptr;
    int32_t *xb = nullptr;
    uint16_t *xd16 = nullptr;
    float *ndrow = nullptr;
    // quantized x images handed from a GEMV pass to the next (Q8_0 / Q8_1 of the output, in the GEMV shared-memory
    // layout), two alternating buffers
    uint8_t *qimg[2] = {nullptr, nullptr};
    double *nsq[2] = {nullptr, nullptr};  // per-panel sums of squares handed to a deferred norm (alternating)
    // quantized tokens of GEMV_BATCH commands of more than kBatchMax rows (the tensor-core GEMM's image), sized
    // before a list runs or is captured; a buffer replaced by a larger one stays allocated until the context ends
    // (captured graphs may still use it)
    uint8_t *gemm_img = nullptr;
    size_t gemm_img_bytes = 0;
    std::vector<uint8_t *> gemm_img_old;
    int32_t *gemm_sums = nullptr;  // debug: where the next GEMM stores its first block's integer sums
    float *snap = nullptr;
    size_t snap_used = 0;
    unsigned *dstatus = nullptr;
    float *attn_part = nullptr;
    unsigned long long *tstamps = nullptr;
    uint32_t *ttags = nullptr;
    std::vector<uint32_t> host_tags;
    unsigned n_events = 0;
    std::vector<WeightInfo> weights;
    bool disabled = false;
    std::string err;
    int world = 1, rank = 0;
    nccl_comm comm = nullptr;
    // row-sharded passes without a collective: the peers' act and sync words (IPC-mapped), this rank's sync words,
    // the next free sync slot of the list and the wait not yet handed to a kernel
    bool peer_ok = false;
    float *peer_act[kMaxPeers] = {};
    unsigned *peer_sync[kMaxPeers] = {};
    unsigned *sync = nullptr;  // kSyncWords: ready and data words per (slot, rank), CTA and launch counts per slot
    unsigned slot_next = 0;
    PeerWait pending;          // sharded launches whose rows no kernel has waited for yet
    // explicit (tensor-parallel) lists: the caller's own slices, exchanges only by ALLREDUCE / ALLGATHER commands;
    // with coll_peer, ALLREDUCE runs as the peer kernel (coll.cu) on these buffers, one slot per ALLREDUCE of a list
    bool explicit_comm = false, coll_peer = false;
    uint2 *coll_recv = nullptr;          // kCollSlots x [2][world][kCollMaxN] words, mapped into every peer
    unsigned *coll_flags = nullptr;      // kCollSlots x kCollMaxCtas launch counters (this rank only)
    uint2 *peer_coll_recv[kMaxPeers] = {};
    unsigned coll_slot_next = 0;
    unsigned *chain_counters = nullptr;  // kMaxChains x kChainCounters words, zero between launches
    unsigned chain_next = 0;             // the next chain's counter block in the list being executed
    bool pdl = true;
    bool pdl_env = true;       // B200Q_NO_PDL=1 turns programmatic dependent launch off for the context's life
    uint32_t feature_mask = 0xFFFFFFFFu;  // B200Q_FEATURE_MASK (b200q_set_feature_mask), set at create
    // runtime verification of the first verify_left lists against the caller's checker (b200q_set_verify)
    b200q_verify_fn verify_fn = nullptr;
    void *verify_user = nullptr;
    int verify_left = 0;
    unsigned launches = 0;  // kernels launched by the last executed list
    std::mutex mu;
};

struct b200q_graph {
    b200q_ctx *ctx = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    unsigned kernels = 0;
    std::vector<uint32_t> cmds;  // the list, for runtime verification of its launches
};

namespace {

int set_err(b200q_ctx *c, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    c->err = buf;
    if (code == B200Q_ERR_CUDA) c->disabled = true;
    return code;
}

#define CUDA_TRY(c, expr)                                                                                          \
    do {                                                                                                           \
        cudaError_t e_ = (expr);                                                                                   \
        if (e_ != cudaSuccess) return set_err((c), B200Q_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_));       \
    } while (0)

const WeightInfo *find_w(const b200q_ctx *c, uint64_t h) {
    for (const WeightInfo &w : c->weights)
        if (w.handle == h) return &w;
    return nullptr;
}

MatrixView view_of(const b200q_ctx *c, const WeightInfo &w) {
    MatrixView v;
    v.base = c->warena + w.base_off;
    v.format = w.format;
    v.rows = w.row_end - w.row_begin;
    v.row0 = w.row_begin;
    v.rt = w.rt;
    v.ct = w.ct;
    v.kc = w.kc;
    v.n_rt = w.n_rt;
    v.tile_bytes = w.tile_bytes;
    v.qs_part = w.qs_part;
    v.dm_part = w.dm_part;
    return v;
}

bool meet(const float *a, size_t an, const float *b, size_t bn) { return a < b + bn && b < a + an; }

struct Range {
    const float *p;
    size_t n;
};

// The wait for the peers' rows of the last sharded pass, handed to the next kernel launched (which waits for them
// after its wait on the previous kernel); every kernel after it is ordered behind it.
PeerWait take_wait(b200q_ctx *c) {
    PeerWait w = c->pending;
    c->pending.n = 0;
    return w;
}
// ... or as a kernel of its own, before a copy (or the end of the list) that no kernel covers
int flush_wait(b200q_ctx *c) {
    if (c->pending.n == 0) return 0;
    CUDA_TRY(c, launch_peer_wait(take_wait(c), c->stream, c->pdl));
    ++c->launches;
    return 0;
}

// An input that a kernel of the same launch writes with a different element mapping: copy it first.
const float *snap_if(b200q_ctx *c, const float *in, size_t n, const std::vector<Range> &writes, const float *same_ok,
                     int &rc) {
    bool hit = false;
    for (const Range &w : writes) {
        if (!meet(in, n, w.p, w.n)) continue;
        if (same_ok && in == same_ok && w.p == same_ok) continue;  // element-aligned in place
        hit = true;
    }
    if (!hit) return in;
    if ((rc = flush_wait(c))) return in;
    if (c->snap_used + n > kSnapFloats) {
        rc = set_err(c, B200Q_ERR_NOMEM, "snapshot scratch full");
        return in;
    }
    float *dst = c->snap + c->snap_used;
    c->snap_used += (n + 63) / 64 * 64;
    cudaError_t e = cudaMemcpyAsync(dst, in, n * sizeof(float), cudaMemcpyDeviceToDevice, c->stream);
    if (e != cudaSuccess) rc = set_err(c, B200Q_ERR_CUDA, "snapshot copy: %s", cudaGetErrorString(e));
    return dst;
}

int all_gather_rows(b200q_ctx *c, float *base, size_t per_rank) {
    if (c->world <= 1) return 0;
    const int r = g_nccl.all_gather(base + per_rank * c->rank, base, per_rank, kNcclFloat32, c->comm, c->stream);
    if (r != 0) return set_err(c, B200Q_ERR_COMM, "ncclAllGather: %s", g_nccl.get_error_string ? g_nccl.get_error_string(r) : "?");
    return 0;
}

// ---- one GEMV group ------------------------------------------------------------------------------------------------
// A GEMV pass's output handed to the next GEMV pass as its quantized x image (see link_image).
struct ImageLink {
    uint8_t *out = nullptr;      // this pass writes the image of member out_member's y here
    unsigned out_member = 0;
    unsigned out_act = 0;        // activation type of the next pass (0 Q8_0, 1 Q8_1)
    const uint8_t *in = nullptr;  // this pass reads its x image from here
    double *nsq_out = nullptr;    // this pass writes member nsq_member's per-panel sums of squares here (nsq_out_n)
    unsigned nsq_member = 0, nsq_out_n = 0;
    const double *nsq_in = nullptr;  // this pass's deferred norm reads nsq_n such partials instead of its whole x
    unsigned nsq_n = 0;
};

int exec_gemv(b200q_ctx *c, const Member *mem, unsigned nm, unsigned x_off, unsigned cols, bool from_nd,
              const DeferredNorm &nd, bool prequant, const float *x_override, int32_t *dbg,
              const ImageLink &link = ImageLink()) {
    GemvArgs a;
    a.cols = cols;
    const unsigned act = act_type(mem[0].format);
    const bool kq = act == 2;
    if (x_override) {
        a.x = x_override;
    } else if (from_nd && nd.materialize) {
        a.x = c->ndrow;
    } else if (from_nd) {
        a.x = c->act + nd.x_off;
        a.norm_w = c->act + nd.w_off;
        a.norm_eps = nd.eps;
        a.norm_mode = 8u | nd.flags;
    } else {
        a.x = c->act + x_off;
    }
    int rc = 0;
    std::vector<Range> writes;
    bool shard = false;
    for (unsigned i = 0; i < nm; ++i) {
        const Member &m = mem[i];
        const WeightInfo *w = m.w ? m.w : find_w(c, m.handle);
        if (!w) return set_err(c, B200Q_ERR_ARG, "unknown weight handle");
        GemvMemberArgs &g = a.m[i];
        g.w = view_of(c, *w);
        shard |= g.w.rows != w->rows;
        g.epi = m.epi;
        g.total_rows = m.rows;
        g.y = c->act + m.y_off;
        if (m.epi == EpiAdd) g.res = c->act + m.r_off;
        if (m.epi == EpiConv) {
            g.cw = c->act + m.c_w;
            g.cs = c->act + m.c_src;
            g.cd = c->act + m.c_dst;
            g.csilu = m.c_silu;
        }
        if (m.epi != EpiSwigluG) {
            writes.push_back({g.y, (m.epi == EpiConv || m.epi == EpiAdd) ? m.rows : round16(m.rows)});
            if (m.epi == EpiConv) writes.push_back({g.cd, size_t(3) * m.rows});
        }
    }
    a.n_members = nm;
    // inputs read per row by the thread that writes the row: in place is fine, other overlaps are copied first
    for (unsigned i = 0; i < nm; ++i) {
        GemvMemberArgs &g = a.m[i];
        if (g.res) g.res = snap_if(c, g.res, mem[i].rows, writes, g.y, rc);
        if (g.cs) g.cs = snap_if(c, g.cs, size_t(3) * mem[i].rows, writes, g.cd, rc);
        if (g.cw) g.cw = snap_if(c, g.cw, size_t(4) * mem[i].rows, writes, nullptr, rc);
    }
    if (rc) return rc;
    if (dbg) a.dbg = dbg;
    // x read by every CTA while others write: quantize it first when a member's output overlaps it
    bool xhit = false;
    for (const Range &w : writes) xhit |= meet(a.x, cols, w.p, w.n);
    if (a.norm_w) for (const Range &w : writes) xhit |= meet(a.norm_w, cols, w.p, w.n);
    const bool use_image = link.in && !dbg && !(prequant || xhit);
    if (use_image) a.qin = link.in;
    if (link.out && !dbg) {
        a.qout = link.out;
        a.qout_member = link.out_member;
        a.qout_act = link.out_act;
    }
    if (link.nsq_out && !dbg && !kq) {
        a.nsq_out = link.nsq_out;
        a.nsq_member = link.nsq_member;
    }
    if (link.nsq_in && !dbg && !kq && from_nd && !nd.materialize && !prequant && !xhit) {
        a.nsq_in = link.nsq_in;
        a.nsq_n = link.nsq_n;
    }
    if ((prequant || xhit) && !dbg) {
        QuantArgs q;
        q.x = a.x;
        q.n = cols;
        q.act = act;
        q.norm_w = a.norm_w;
        q.norm_eps = a.norm_eps;
        q.norm_mode = a.norm_mode;
        q.q = c->xq;
        q.d = c->xd;
        q.s = c->xs;
        q.b = c->xb;
        q.pw = take_wait(c);
        CUDA_TRY(c, launch_quantize(q, c->stream));
        ++c->launches;
        a.xq = c->xq;
        a.xd = c->xd;
        a.xs = c->xs;
        a.xb = c->xb;
    }
    // work units (a member, or a SwiGLU pair) and their row tiles
    unsigned u = 0, items = 0;
    for (unsigned i = 0; i < nm; ++i) {
        const bool pair = mem[i].epi == EpiSwigluG && i + 1 < nm;
        a.unit_member[u] = i;
        a.unit_pair[u] = pair ? int(i + 1) : -1;
        a.item_start[u] = items;
        items += a.m[i].w.n_rt;
        ++u;
        if (pair) ++i;
    }
    a.n_units = u;
    a.item_start[u] = items;
    a.err = c->dstatus + 1;
    const unsigned slot0 = c->slot_next;
    // a launch with sharded members takes a sync slot (peer stores, ready / data flags)
    auto take_slot = [&](GemvArgs &g) -> int {
        if (!shard || dbg || !c->peer_ok) return 0;
        bool any = false;
        for (unsigned k = 0; k < g.n_units; ++k) {
            const int pk = g.unit_pair[k];
            const GemvMemberArgs &out = g.m[pk >= 0 ? unsigned(pk) : g.unit_member[k]];
            any = any || out.w.rows != out.total_rows;
        }
        if (!any) return 0;
        if (c->slot_next >= kSyncSlots) return set_err(c, B200Q_ERR_ARG, "too many sharded GEMV launches in a list");
        PeerSync &ps = g.ps;
        ps.act = c->act;
        for (int r = 0; r < c->world; ++r) {
            ps.peer_act[r] = c->peer_act[r];
            ps.peer_sync[r] = c->peer_sync[r];
        }
        ps.sync = c->sync;
        ps.world = unsigned(c->world);
        ps.rank = unsigned(c->rank);
        ps.slot = c->slot_next++;
        return 0;
    };
    size_t smem = 0;
    if (kq) {
        plan_gemv_kq(a, smem);
        const unsigned grid = std::min(items, unsigned(c->sms) * (smem <= 113 * 1024 ? 2u : 1u));
        if ((rc = take_slot(a))) return rc;
        a.pw = take_wait(c);
        CUDA_TRY(c, launch_gemv_kq(a, grid, smem, c->stream, c->pdl));
        ++c->launches;
    } else {
        // one launch per format combination of the units (a member alone, or a SwiGLU g/u pair); one panel per
        // CTA when a launch's panels fit on the GPU at once, else every CTA loops over panels
        plan_gemv_q8(a, smem);
        bool done[kMaxUnits] = {};
        for (unsigned i = 0; i < a.n_units; ++i) {
            if (done[i]) continue;
            const int pr = a.unit_pair[i];
            const unsigned fa = a.m[a.unit_member[i]].w.format, fb = pr >= 0 ? a.m[pr].w.format : 0u;
            GemvArgs g = a;
            unsigned gu = 0, gi = 0;
            const bool one_unit = !(c->feature_mask & kMaskGroups);  // multi-output passes off: a launch per unit
            for (unsigned k = i; k < a.n_units; ++k) {
                const int pk = a.unit_pair[k];
                const unsigned ka = a.m[a.unit_member[k]].w.format, kb = pk >= 0 ? a.m[pk].w.format : 0u;
                if (done[k] || ka != fa || kb != fb || (one_unit && k != i)) continue;
                if (pk >= 0) {
                    const MatrixView &gw = a.m[a.unit_member[k]].w, &uw = a.m[pk].w;
                    if (gw.rt != uw.rt || gw.kc != uw.kc || gw.rows != uw.rows)
                        return set_err(c, B200Q_ERR_ARG, "SwiGLU g and u weights have different panel shapes");
                }
                done[k] = true;
                g.unit_member[gu] = a.unit_member[k];
                g.unit_pair[gu] = pk;
                g.item_start[gu] = gi;
                gi += a.item_start[k + 1] - a.item_start[k];
                ++gu;
            }
            g.n_units = gu;
            g.item_start[gu] = gi;
            if (!gemv_q8_supported(fa, fb)) return set_err(c, B200Q_ERR_ARG, "unsupported GEMV format combination");
            // whole clusters (the x preparation is split over a cluster's CTAs)
            const unsigned cl = gemv_q8_cluster();
            const unsigned grid = std::min((gi + cl - 1) / cl * cl, gemv_q8_resident_ctas(fa, fb, smem, c->stream));
            if ((rc = take_slot(g))) return rc;
            g.pw = take_wait(c);
            CUDA_TRY(c, launch_gemv_q8(g, fa, fb, grid, smem, c->stream, c->pdl));
            ++c->launches;
        }
    }
    if (shard && !dbg && c->peer_ok) {
        // every launch stored its sharded rows into the peers: the next kernel waits for theirs
        c->pending.sync = c->sync;
        c->pending.slot0 = slot0;
        c->pending.n = c->slot_next - slot0;
        c->pending.world = unsigned(c->world);
        c->pending.rank = unsigned(c->rank);
        c->pending.err = c->dstatus + 1;
    } else if (shard && !dbg) {
        for (unsigned i = 0; i < nm; ++i) {
            const GemvMemberArgs &g = a.m[i];
            if (g.epi == EpiSwigluG || g.w.rows == mem[i].rows) continue;
            const size_t per = g.w.rows;
            if ((rc = all_gather_rows(c, g.y, per))) return rc;
            if (g.epi == EpiConv && (rc = all_gather_rows(c, g.cd, 3 * per))) return rc;
        }
    }
    return 0;
}

int exec_elementwise(b200q_ctx *c, const Pass &p) {
    const uint32_t *cmd = p.cmd[0];
    float *A = c->act;
    int rc = 0;
    switch (p.op) {
    case 2: {  // RMSNORM stored
        const unsigned n = cmd[1], rows = cmd[6] ? cmd[6] : 1u, stride = (cmd[7] >> 8) & 0xffffu;
        const unsigned xs = stride ? stride * 16 : n;
        float *y = A + cmd[4];
        std::vector<Range> w{{y, size_t(rows) * n}};
        const float *x = snap_if(c, A + cmd[2], size_t(rows - 1) * xs + n, w, xs == n ? y : nullptr, rc);
        const float *wt = (cmd[7] & 2u) ? nullptr : snap_if(c, A + cmd[3], n, w, nullptr, rc);
        if (rc) return rc;
        CUDA_TRY(c, launch_rmsnorm(x, wt, y, n, rows, xs, *reinterpret_cast<const float *>(&cmd[5]), cmd[7] & 3u,
                                   take_wait(c),
                                   c->stream, c->pdl));
        break;
    }
    case 3: case 4: case 5: case 6: {
        EwArgs e;
        e.op = p.op;
        e.n = cmd[1];
        e.y = A + cmd[4];
        const bool unary = p.op == 6;
        e.row = unary ? cmd[5] : (p.op == 4 ? cmd[6] : 0u);
        e.stride = unary ? cmd[6] : cmd[7];
        e.kind = unary ? cmd[3] : 0u;
        e.sigmoid = p.op == 4 ? (cmd[5] & 1u) : 0u;
        std::vector<Range> w{{e.y, e.n}};
        const size_t span = e.row ? size_t(e.n / e.row - 1) * e.stride + e.row : e.n;
        e.a = snap_if(c, A + cmd[2], span, w, e.row ? nullptr : e.y, rc);
        if (!unary) e.b = snap_if(c, A + cmd[3], e.n, w, e.y, rc);
        if (rc) return rc;
        e.pw = take_wait(c);
        CUDA_TRY(c, launch_ew(e, c->stream, c->pdl));
        break;
    }
    case 8: {  // CONV
        const unsigned ch = cmd[1];
        float *y = A + cmd[4], *sd = A + cmd[6];
        std::vector<Range> w{{y, ch}, {sd, size_t(3) * ch}};
        const float *x = snap_if(c, A + cmd[2], ch, w, y, rc);
        const float *wt = snap_if(c, A + cmd[3], size_t(4) * ch, w, nullptr, rc);
        const float *ss = snap_if(c, A + cmd[5], size_t(3) * ch, w, sd, rc);
        if (rc) return rc;
        CUDA_TRY(c, launch_conv(x, wt, y, ss, sd, ch, cmd[7] & 1u, take_wait(c), c->stream, c->pdl));
        break;
    }
    case 10: {  // ROPE
        const unsigned nd = cmd[1], ne0 = cmd[5], rows = cmd[6];
        float *y = A + cmd[4];
        std::vector<Range> w{{y, size_t(ne0) * rows}};
        const float *x = snap_if(c, A + cmd[2], size_t(ne0) * rows, w, y, rc);
        const float *cs = snap_if(c, A + cmd[3], nd, w, nullptr, rc);
        if (rc) return rc;
        CUDA_TRY(c, launch_rope(x, cs, y, nd, ne0, rows, take_wait(c), c->stream, c->pdl));
        break;
    }
    default: return set_err(c, B200Q_ERR_ARG, "unexpected element-wise opcode %u", p.op);
    }
    ++c->launches;
    return 0;
}

int exec_rowops(b200q_ctx *c, const Pass &p) {
    RowOpsArgs a;
    float *A = c->act;
    unsigned row0 = 0;
    for (const auto &jb : p.rowjobs) {
        RowJobArgs &J = a.job[a.n_jobs++];
        const uint32_t *nc = jb.data(), *rc = jb.data() + 8;
        J.row0 = row0;
        if (nc[0] == 2) {
            J.norm = true;
            J.n = nc[1];
            J.x = A + nc[2];
            J.w = (nc[7] & 2u) ? nullptr : A + nc[3];
            J.y = A + nc[4];
            J.eps = *reinterpret_cast<const float *>(&nc[5]);
            J.rows = nc[6] ? nc[6] : 1u;
            const unsigned stride = (nc[7] >> 8) & 0xffffu;
            J.xstride = stride ? stride * 16 : nc[1];
            J.flags = nc[7] & 3u;
        }
        if (rc[0] == 10) {
            J.nd = rc[1];
            J.rx = A + rc[2];
            J.cs = A + rc[3];
            J.ry = A + rc[4];
            J.ne0 = rc[5];
            J.rows = rc[6];
        }
        row0 += J.rows;
    }
    a.total_rows = row0;
    a.pw = take_wait(c);
    CUDA_TRY(c, launch_rowops(a, c->stream, c->pdl));
    ++c->launches;
    return 0;
}

int exec_gdn(b200q_ctx *c, const Pass &p, const ImageLink &nsq_link) {
    const uint32_t *cmd = p.cmd[0], *ext = p.cmd[1], *ext2 = p.cmd[2];
    float *A = c->act;
    GdnArgs g;
    g.hv = cmd[1] & 0xffffu;
    g.hk = cmd[1] >> 16;
    const unsigned fl = ext[3], S = 128;
    g.y = A + cmd[7];
    std::vector<Range> w{{g.y, size_t(g.hv) * S}};
    int rc = 0;
    g.q = snap_if(c, A + cmd[2], size_t(g.hk) * S, w, nullptr, rc);
    g.k = snap_if(c, A + cmd[3], size_t(g.hk) * S, w, nullptr, rc);
    g.v = snap_if(c, A + cmd[4], size_t(g.hv) * S, w, g.y, rc);
    g.g = snap_if(c, A + cmd[5], g.hv, w, nullptr, rc);
    g.beta = snap_if(c, A + cmd[6], g.hv, w, nullptr, rc);
    g.state_in = c->state + size_t(ext[0]) * S;
    g.state_out = c->state + size_t(ext[1]) * S;
    g.scale = *reinterpret_cast<const float *>(&ext[2]);
    g.l2 = (fl & 2u) ? 1u : 0u;
    g.l2_eps = *reinterpret_cast<const float *>(&ext[4]);
    g.rms_eps = *reinterpret_cast<const float *>(&ext[5]);
    if (fl & 4u) {
        g.wn = snap_if(c, A + ext[6], S, w, nullptr, rc);
        g.z = snap_if(c, A + ext[7], size_t(g.hv) * S, w, g.y, rc);
    }
    if (fl & 8u) {
        g.dt = snap_if(c, A + ext2[0], g.hv, w, nullptr, rc);
        g.a = snap_if(c, A + ext2[1], g.hv, w, nullptr, rc);
    }
    if (rc) return rc;
    // the ssm_out GEMV of a WITH_OUT step reads y: the GDN kernel hands it over quantized (Q8_0 / Q8_1 formats)
    ImageLink out_link;
    if (p.gdn_with_out && act_type(p.gdn_out.format) != 2 && p.gdn_out.cols == g.hv * S &&
        size_t(g.hv) * S * 3 / 2 <= kQImageBytes && (c->feature_mask & kMaskGdnOut)) {
        g.img = c->qimg[0];
        g.img_act = act_type(p.gdn_out.format);
        out_link.in = c->qimg[0];
    }
    out_link.nsq_out = nsq_link.nsq_out;  // the next pass's deferred-norm partials, from the ssm_out rows
    out_link.nsq_member = 0;
    g.pw = take_wait(c);
    CUDA_TRY(c, launch_gdn(g, c->stream, c->pdl));
    ++c->launches;
    DeferredNorm none;
    if (p.gdn_with_gemv) {
        if ((rc = exec_gemv(c, &p.gdn_gemv, 1, p.gdn_gemv.x_off, p.gdn_gemv.cols, false, none, false, nullptr,
                            nullptr)))
            return rc;
    }
    if (p.gdn_with_out) {
        if ((rc = exec_gemv(c, &p.gdn_out, 1, cmd[7], p.gdn_out.cols, false, none, false, nullptr, nullptr,
                            out_link)))
            return rc;
    }
    return 0;
}

int exec_ext(b200q_ctx *c, const Pass &p) {
    const uint32_t *cmd = p.cmd[0];
    float *A = c->act;
    int rc = 0;
    if (p.op == 12) {
        AttnArgs t;
        t.n_head = cmd[1] & 0xffu;
        t.n_kv_head = (cmd[1] >> 8) & 0xffu;
        t.head_dim = (cmd[1] >> 16) * 16u;
        t.kv_ctx = c->kv_ctx;
        t.y = A + cmd[5];
        t.status = c->dstatus;
        std::vector<Range> w{{t.y, size_t(t.n_head) * t.head_dim}};
        t.pos = snap_if(c, A + cmd[6], 1, w, nullptr, rc);
        t.q = snap_if(c, A + cmd[2], size_t(t.n_head) * t.head_dim, w, nullptr, rc);
        t.k = snap_if(c, A + cmd[3], size_t(t.n_kv_head) * t.head_dim, w, nullptr, rc);
        t.v = snap_if(c, A + cmd[4], size_t(t.n_kv_head) * t.head_dim, w, nullptr, rc);
        if (rc) return rc;
        const size_t slot_elems = size_t(t.n_kv_head) * c->kv_ctx * t.head_dim;
        t.kcache = c->kv + size_t(cmd[7]) * slot_elems * 2;
        t.vcache = t.kcache + slot_elems;
        t.scale = 1.0f / std::sqrt(float(t.head_dim));
        t.chunk = attn_chunk(c->kv_ctx, t.n_kv_head, unsigned(c->sms));
        t.max_chunks = (c->kv_ctx + t.chunk - 1) / t.chunk;
        if (size_t(t.n_head) * t.max_chunks * (t.head_dim + 4) > kAttnPartFloats)
            return set_err(c, B200Q_ERR_ARG, "ATTN: n_head x kv_ctx x head_dim too large for the chunk buffer");
        if (attn_smem_bytes(t.n_head, t.n_kv_head, t.head_dim, t.chunk, t.max_chunks) > 200 * 1024)
            return set_err(c, B200Q_ERR_ARG, "ATTN: the chunk does not fit in shared memory");
        t.part = c->attn_part;
        t.counters = c->dstatus + kSyncAttnWord;
        t.err = c->dstatus + 1;
        if (p.attn_gate) {  // SILU_MUL (sigmoid) of the output, applied in the merge (row 0: contiguous g)
            const uint32_t *g = p.gate;
            t.gate_g = A + g[2];
            t.gate_y = A + g[4];
            t.gate_row = g[6] ? g[6] : g[1];
            t.gate_stride = g[6] ? g[7] : g[1];
        }
        t.pw = take_wait(c);
        CUDA_TRY(c, launch_attn(t, c->stream, c->pdl));
    } else if (p.op == 13) {
        std::vector<Range> w{{A + cmd[3], 2}};
        const float *x = snap_if(c, A + cmd[2], cmd[1], w, nullptr, rc);
        if (rc) return rc;
        CUDA_TRY(c, launch_argmax(x, cmd[1], A + cmd[3],
                                  reinterpret_cast<unsigned long long *>(c->dstatus + kSyncArgmaxWord),
                                  c->dstatus + kSyncArgmaxWord + 2, take_wait(c), c->stream, c->pdl));
    } else if (p.op == 14) {
        const WeightInfo *w = find_w(c, uint64_t(cmd[3]) | (uint64_t(cmd[4]) << 32));
        if (!w) return set_err(c, B200Q_ERR_ARG, "GET_ROW: unknown weight");
        float *y = A + cmd[6];
        std::vector<Range> wr{{y, cmd[2]}};
        const float *idx = snap_if(c, A + cmd[5], 1, wr, nullptr, rc);
        if (rc) return rc;
        CUDA_TRY(c, launch_get_row(view_of(c, *w), cmd[2], idx, y, c->dstatus, take_wait(c), c->stream, c->pdl));
    } else if (p.op == 17) {
        const WeightInfo *w = find_w(c, uint64_t(cmd[4]) | (uint64_t(cmd[5]) << 32));
        if (!w) return set_err(c, B200Q_ERR_ARG, "GEMV_BATCH: unknown weight");
        if (c->world > 1 && !c->explicit_comm)
            return set_err(c, B200Q_ERR_ARG, "GEMV_BATCH: not in a row-sharded context (its matrices hold a row slice)");
        const unsigned batch = ((cmd[1] >> 16) & 0xffffu) + 1u;
        if (batch > kBatchMax) {  // prefill: the tokens quantized once, then the tensor-core GEMM
            GemmArgs g;
            g.w = view_of(c, *w);
            g.x = A + cmd[6];
            g.cols = cmd[3];
            g.tokens = batch;
            g.act = (cmd[1] & 0xffu) == 3u ? 1u : 0u;
            g.xq = c->gemm_img;
            g.y = A + cmd[7];
            g.ystride = (cmd[2] + 15u) & ~15u;
            g.add = (cmd[1] & B200Q_GEMV_ADD) != 0;
            g.err = c->dstatus + 1;
            g.sums = c->gemm_sums;
            if (!g.xq || c->gemm_img_bytes < gemm_image_bytes(g.cols, batch))
                return set_err(c, B200Q_ERR_STATE, "GEMV_BATCH: token image not prepared");
            if ((rc = flush_wait(c))) return rc;
            CUDA_TRY(c, launch_gemm(g, c->stream, c->pdl));
            c->launches += 2;  // the quantizer and the GEMM
            return 0;
        }
        BatchArgs a;
        a.w = view_of(c, *w);
        a.cols = cmd[3];
        a.batch = batch;
        a.act = (cmd[1] & 0xffu) == 3u ? 1u : 0u;
        a.x = A + cmd[6];
        a.y = A + cmd[7];
        a.ystride = (cmd[2] + 15u) & ~15u;
        a.add = (cmd[1] & B200Q_GEMV_ADD) != 0;
        a.err = c->dstatus + 1;
        const unsigned per = gemv_batch_rows_per_launch(a.w, a.cols);
        if (per == 0) return set_err(c, B200Q_ERR_ARG, "GEMV_BATCH: the matrix's panels do not fit shared memory");
        if ((rc = flush_wait(c))) return rc;  // the kernel's producer warp runs apart: no in-kernel peer wait
        CUDA_TRY(c, launch_gemv_batch(a, unsigned(c->sms), c->stream, c->pdl));
        c->launches += (a.batch + per - 1) / per - 1;  // launches past the first (counted below)
    } else if (p.op == 15 || p.op == 16) {
        const size_t n = cmd[1];
        const float *x = A + cmd[2];
        float *y = A + cmd[3];
        if (c->world <= 1) {  // one rank: y = x
            if (x != y) CUDA_TRY(c, cudaMemcpyAsync(y, x, n * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
            return 0;
        }
        if ((rc = flush_wait(c))) return rc;
        if (p.op == 15 && c->coll_peer && n <= kCollMaxN) {
            if (c->coll_slot_next >= kCollSlots)
                return set_err(c, B200Q_ERR_ARG, "more than %u peer ALLREDUCE commands in a list", kCollSlots);
            const unsigned slot = c->coll_slot_next++;
            CollArgs a;
            a.x = x;
            a.y = y;
            a.n = unsigned(n);
            a.world = unsigned(c->world);
            a.rank = unsigned(c->rank);
            const size_t rs = size_t(2) * c->world * kCollMaxN;
            for (int r = 0; r < c->world; ++r)
                a.recv[r] = (r == c->rank ? c->coll_recv : c->peer_coll_recv[r]) + slot * rs;
            a.flag_local = c->coll_flags + size_t(slot) * kCollMaxCtas;
            a.err = c->dstatus + 1;
            CUDA_TRY(c, launch_allreduce_peer(a, c->stream, c->pdl));
        } else {
            const int r = p.op == 15 ? g_nccl.all_reduce(x, y, n, kNcclFloat32, kNcclSum, c->comm, c->stream)
                                     : g_nccl.all_gather(x, y, n, kNcclFloat32, c->comm, c->stream);
            if (r != 0)
                return set_err(c, B200Q_ERR_COMM, "%s: %s", p.op == 15 ? "ncclAllReduce" : "ncclAllGather",
                               g_nccl.get_error_string ? g_nccl.get_error_string(r) : "?");
            return 0;  // not one of this library's kernels
        }
    }
    ++c->launches;
    return 0;
}

int stamp(b200q_ctx *c, bool on, unsigned cmd, unsigned kind) {
    if (!on || c->n_events >= kMaxTraceEvents) return 0;
    c->host_tags.push_back((cmd & 0xffffu) | (kind << 16));
    CUDA_TRY(c, launch_trace_stamp(c->tstamps + c->n_events, c->stream));
    ++c->n_events;
    return 0;
}

// Pass p's GEMV output that pass q (the next pass that launches work) reads as its whole x: pass p writes q's
// quantized x image itself, one block per 32-row panel from the values its fold warps store, so q skips its x
// preparation. Needs: q a Q8_0-family GEMV pass without a deferred norm, reading exactly one member's y; that member
// (and its SwiGLU partner) unsharded, in 32-row panels, with a plain / SwiGLU / residual-ADD writer. (For a deferred
// norm the scale needs the whole y first; quantizing it at the end of p costs p's tail more than q's own x
// preparation, which overlaps q's weight staging.) Returns the member index or -1.
int link_image(const b200q_ctx *c, const Pass &p, const Pass &q, ImageLink &link) {
    if (p.kind != PassKind::Gemv || q.kind != PassKind::Gemv || q.prequant || q.from_nd) return -1;
    if (act_type(q.m[0].format) == 2) return -1;
    for (unsigned i = 0; i < p.n_members; ++i) {
        const Member &m = p.m[i];
        if (m.epi == EpiSwigluG || m.epi == EpiConv) continue;
        if (m.y_off != q.x_off || m.rows != q.cols || act_type(m.format) == 2) continue;
        if (m.rows % 32) return -1;
        for (unsigned k = 0; k < p.n_members; ++k) {  // the member and its SwiGLU partner
            if (k != i && !(m.epi == EpiSwigluU && k + 1 == i)) continue;
            const WeightInfo *w = p.m[k].w ? p.m[k].w : find_w(c, p.m[k].handle);
            if (!w || w->rt != 32 || w->row_begin != 0 || w->row_end != w->rows || act_type(w->format) == 2)
                return -1;
        }
        link.out_member = i;
        link.out_act = act_type(q.m[0].format);
        return int(i);
    }
    return -1;
}

// Pass p's GEMV output that pass q (the next pass that launches work) normalizes as its deferred RMSNORM's x: p sums
// the squares of that member's stored values per panel and q adds those partials instead of reading all of x.
// Needs: q a Q4_0 / Q4_1 GEMV pass on a live deferred norm (not stored), p's member a Q8_0-family matrix whose
// y is exactly the norm's x, unsharded, with a plain or residual-ADD writer. Returns the member index or -1.
// (Measured on one box: the 4B-like Q4_0 decode 706 -> 718 tokens/s; for a Q8_0 consumer, whose x preparation
// overlaps twice the weight bytes, the producer's extra tail cost more than it saved: 140.2 -> 140.7 us per stack
// step, so Q8_0 consumers read x as before.)
// 1: member m (index i of its pass) writes q's deferred-norm x and can hand q its partials; 0: it does not; -1: it
// writes that x but cannot.
static int nsq_member_ok(const b200q_ctx *c, const Member &m, unsigned i, const Pass &q, ImageLink &link) {
    if ((m.epi != EpiNone && m.epi != EpiAdd) || m.y_off != q.nd.x_off || m.rows != q.nd.n) return 0;
    const WeightInfo *w = m.w ? m.w : find_w(c, m.handle);
    if (!w || act_type(w->format) == 2 || w->row_begin != 0 || w->row_end != w->rows || w->n_rt > kMaxNsqPanels)
        return -1;
    link.nsq_member = i;
    link.nsq_out_n = w->n_rt;
    return 1;
}

static bool nsq_consumer(const Pass &q) {
    return q.kind == PassKind::Gemv && q.from_nd && !q.nd.materialize && !q.prequant &&
           act_type(q.m[0].format) != 2 && q.m[0].format != B200Q_Q8_0;
}

int link_nsq(const b200q_ctx *c, const Pass &p, const Pass &q, ImageLink &link) {
    if (!nsq_consumer(q)) return -1;
    if (p.kind == PassKind::Gdn) {  // the step's WITH_OUT GEMV (ssm_out + residual) as the producer
        return p.gdn_with_out && nsq_member_ok(c, p.gdn_out, 0, q, link) == 1 ? 0 : -1;
    }
    if (p.kind != PassKind::Gemv) return -1;
    for (unsigned i = 0; i < p.n_members; ++i) {
        const int r = nsq_member_ok(c, p.m[i], i, q, link);
        if (r) return r > 0 ? int(i) : -1;
    }
    return -1;
}

// ---- persistent GEMV chains ----------------------------------------------------------------------------------------
// Pass p as one pass of a chain (gemv_chain_kernel), after `prev` (null: the chain's first pass). Chainable: a GEMV
// pass of one Q4_0 / Q8_0 matrix or a SwiGLU pair of two, its output plain or residual-ADD, unsharded, x not
// quantized ahead (prequant), no output overlapping the pass's own inputs (x, norm weight, residual other than in
// place). Its x: the previous pass's image when it reads exactly that output (32-row panels), a deferred norm, or
// act x.
bool chain_pass(const b200q_ctx *c, const Pass &p, const ChainPass *prev, ChainPass &cp) {
    if (p.kind != PassKind::Gemv || p.prequant || (p.from_nd && p.nd.materialize)) return false;
    const bool pair = p.n_members == 2 && p.m[0].epi == EpiSwigluG && p.m[1].epi == EpiSwigluU;
    if (!(p.n_members == 1 || pair)) return false;
    const Member &mo = p.m[p.n_members - 1];
    if (!pair && mo.epi != EpiNone && mo.epi != EpiAdd) return false;
    const unsigned fmt = p.m[0].format;
    if ((fmt != B200Q_Q4_0 && fmt != B200Q_Q8_0) || (pair && p.m[1].format != fmt)) return false;
    const WeightInfo *wa = p.m[0].w ? p.m[0].w : find_w(c, p.m[0].handle);
    const WeightInfo *wb = pair ? (p.m[1].w ? p.m[1].w : find_w(c, p.m[1].handle)) : nullptr;
    if (!wa || wa->row_begin != 0 || wa->row_end != wa->rows) return false;
    if (pair && (!wb || wb->row_begin != 0 || wb->row_end != wb->rows || wb->rt != wa->rt || wb->kc != wa->kc ||
                 wb->rows != wa->rows))
        return false;
    cp = ChainPass();
    cp.wa = view_of(c, *wa);
    if (pair) cp.wb = view_of(c, *wb);
    cp.fmt = fmt;
    cp.pair = pair ? 1u : 0u;
    cp.cols = p.cols;
    GemvMemberArgs &o = cp.out;
    o.w = cp.wa;
    o.epi = mo.epi;
    o.total_rows = mo.rows;
    o.y = c->act + mo.y_off;
    if (mo.epi == EpiAdd) o.res = c->act + mo.r_off;
    const size_t yn = mo.epi == EpiAdd ? mo.rows : round16(mo.rows);
    if (p.from_nd) {
        cp.x_kind = 1;
        cp.x = c->act + p.nd.x_off;
        cp.norm_w = c->act + p.nd.w_off;
        cp.norm_eps = p.nd.eps;
        cp.norm_mode = 8u | p.nd.flags;
    } else if (prev && prev->out.y == c->act + p.x_off && prev->out.total_rows == p.cols && prev->wa.rt == 32 &&
               p.cols % 32 == 0 && (c->feature_mask & kMaskImage)) {
        cp.x_kind = 2;
    } else {
        cp.x_kind = 0;
        cp.x = c->act + p.x_off;
    }
    // the pass's output does not meet its own inputs (a residual read in place, row by row, is fine)
    if (cp.x_kind != 2 && meet(cp.x, p.cols, o.y, yn)) return false;
    if (cp.x_kind == 1 && !(p.nd.flags & 2u) && meet(cp.norm_w, p.cols, o.y, yn)) return false;
    if (o.res && o.res != o.y && meet(o.res, mo.rows, o.y, yn)) return false;
    return true;
}

// The run of passes from plan.passes[pi] that one chain launch executes (>= 2 GEMV passes, skipping deferred-norm
// markers that launch nothing); returns the index after the run, or pi when no chain starts here.
size_t build_chain(b200q_ctx *c, const Plan &plan, size_t pi, ChainArgs &a) {
    if (!(c->feature_mask & kMaskChains) || plan.has_trace || c->pending.n || c->chain_next >= kMaxChains ||
        (c->world > 1 && !c->explicit_comm))
        return pi;
    a = ChainArgs();
    size_t qi = pi, end = pi;
    unsigned items = 0;
    while (qi < plan.passes.size() && a.n_passes < kMaxChainPasses) {
        const Pass &p = plan.passes[qi];
        if (p.kind == PassKind::Nop && !p.nd_store && p.op == 2) {  // a deferred norm's marker: no launch
            ++qi;
            continue;
        }
        ChainPass &cp = a.p[a.n_passes];
        if (!chain_pass(c, p, a.n_passes ? &a.p[a.n_passes - 1] : nullptr, cp)) break;
        cp.item0 = items;
        items += cp.wa.n_rt;
        ++a.n_passes;
        end = ++qi;
    }
    if (a.n_passes < 2) return pi;
    // a pass whose successor reads its output as an image writes one (alternating buffers)
    for (unsigned k = 0; k + 1 < a.n_passes; ++k) {
        if (a.p[k + 1].x_kind != 2) continue;
        a.p[k].qout = c->qimg[k & 1u];
        a.p[k].qout_act = 0;
        a.p[k + 1].qin = c->qimg[k & 1u];
    }
    a.total_items = items;
    return end;
}

int exec_chain(b200q_ctx *c, ChainArgs &a) {
    size_t smem = 0;
    if (!plan_gemv_chain(a, smem)) return set_err(c, B200Q_ERR_ARG, "GEMV chain: shared-memory plan failed");
    a.counters = c->chain_counters + size_t(c->chain_next++) * kChainCounters;
    a.err = c->dstatus + 1;
    CUDA_TRY(c, launch_gemv_chain(a, unsigned(c->sms), smem, c->stream, c->pdl));
    ++c->launches;
    return 0;
}

// The image of the quantized tokens that the list's GEMV_BATCH commands of more than kBatchMax rows need, allocated
// before the list runs or is captured (no allocation inside a capture).
int prepare_gemm_image(b200q_ctx *c, const Plan &plan) {
    size_t need = 0;
    for (const Pass &p : plan.passes) {
        if (p.op != 17 || p.kind != PassKind::Ext) continue;
        const unsigned batch = ((p.cmd[0][1] >> 16) & 0xffffu) + 1u;
        if (batch > kBatchMax) need = std::max(need, gemm_image_bytes(p.cmd[0][3], batch));
    }
    if (need <= c->gemm_img_bytes) return 0;
    // at least double the old size, so that a caller whose prompts grow a little at a time retires O(log) buffers;
    // exactly the need when the doubled size does not fit
    uint8_t *img = nullptr;
    size_t bytes = std::max(need, 2 * c->gemm_img_bytes);
    cudaError_t e = cudaMalloc(&img, bytes);
    if (e != cudaSuccess && bytes > need) {
        cudaGetLastError();
        bytes = need;
        e = cudaMalloc(&img, bytes);
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_err(c, B200Q_ERR_NOMEM, "GEMV_BATCH token image (%zu bytes): %s", need, cudaGetErrorString(e));
    }
    if (c->gemm_img) c->gemm_img_old.push_back(c->gemm_img);
    c->gemm_img = img;
    c->gemm_img_bytes = bytes;
    return 0;
}

// Executes the passes of a plan on the context stream (no synchronization).
int exec_plan(b200q_ctx *c, const Plan &plan, unsigned n_cmds) {
    c->snap_used = 0;
    c->launches = 0;
    c->slot_next = 0;
    c->coll_slot_next = 0;
    c->chain_next = 0;
    c->pending.n = 0;
    c->n_events = 0;
    c->host_tags.clear();
    const bool tr = plan.has_trace;
    int rc = 0;
    const uint8_t *img_in = nullptr;  // the image the previous GEMV pass wrote for this one
    unsigned img_turn = 0;
    const double *nsq_in = nullptr;   // the norm partials the previous GEMV pass wrote for this one
    unsigned nsq_in_n = 0, nsq_turn = 0;
    for (size_t pi = 0; pi < plan.passes.size(); ++pi) {
        const Pass &p = plan.passes[pi];
        if (p.kind != PassKind::Gemv && !(p.kind == PassKind::Nop && !p.nd_store)) {
            img_in = nullptr;
            nsq_in = nullptr;
        }
        if ((rc = stamp(c, tr, p.first, 0))) return rc;
        const bool is_pass = p.kind == PassKind::Gemv || p.kind == PassKind::Gdn;
        if (is_pass && (rc = stamp(c, tr, p.first, 1))) return rc;
        if (p.kind == PassKind::Gemv && !tr) {
            ChainArgs ca;
            const size_t end = build_chain(c, plan, pi, ca);
            if (end > pi) {
                if ((rc = exec_chain(c, ca))) return rc;
                img_in = nullptr;
                nsq_in = nullptr;
                pi = end - 1;
                continue;
            }
        }
        switch (p.kind) {
        case PassKind::Gemv:
        {
            ImageLink link;
            if (img_in) link.in = img_in;
            img_in = nullptr;
            if (nsq_in) {
                link.nsq_in = nsq_in;
                link.nsq_n = nsq_in_n;
            }
            nsq_in = nullptr;
            size_t qi = pi + 1;  // the next pass that launches work (a deferred RMSNORM's own pass launches none)
            while (qi < plan.passes.size() && plan.passes[qi].kind == PassKind::Nop && !plan.passes[qi].nd_store) ++qi;
            if (qi < plan.passes.size() && (c->feature_mask & kMaskImage) && link_image(c, p, plan.passes[qi], link) >= 0) {
                link.out = c->qimg[img_turn];
                img_in = c->qimg[img_turn];
                img_turn ^= 1u;
            }
            if (qi < plan.passes.size() && (c->feature_mask & kMaskNsq) && link_nsq(c, p, plan.passes[qi], link) >= 0) {
                link.nsq_out = c->nsq[nsq_turn];
                nsq_in = c->nsq[nsq_turn];
                nsq_in_n = link.nsq_out_n;
                nsq_turn ^= 1u;
            }
            rc = exec_gemv(c, p.m, p.n_members, p.x_off, p.cols, p.from_nd, p.nd, p.prequant, nullptr, nullptr, link);
        }
            break;
        case PassKind::Elementwise: rc = exec_elementwise(c, p); break;
        case PassKind::Gdn:
        {
            ImageLink nl;
            size_t qi = pi + 1;
            while (qi < plan.passes.size() && plan.passes[qi].kind == PassKind::Nop && !plan.passes[qi].nd_store) ++qi;
            if (qi < plan.passes.size() && (c->feature_mask & kMaskNsq) && link_nsq(c, p, plan.passes[qi], nl) >= 0) {
                nl.nsq_out = c->nsq[nsq_turn];
                nsq_in = c->nsq[nsq_turn];
                nsq_in_n = nl.nsq_out_n;
                nsq_turn ^= 1u;
            }
            rc = exec_gdn(c, p, nl);
        }
            break;
        case PassKind::Ext: rc = exec_ext(c, p); break;
        case PassKind::RowOps: rc = exec_rowops(c, p); break;
        case PassKind::Nop:
            if (p.nd_store) {  // a deferred RMSNORM whose x or weight changes before its GEMVs: store its row now
                const DeferredNorm &nd = p.nd;
                CUDA_TRY(c, launch_rmsnorm(c->act + nd.x_off, c->act + nd.w_off, c->ndrow, nd.n, 1, nd.n, nd.eps,
                                           nd.flags, take_wait(c), c->stream, c->pdl));
                ++c->launches;
            }
            break;
        }
        if (rc) return rc;
        if (is_pass && (rc = stamp(c, tr, p.first, 2))) return rc;
    }
    // the last sharded pass's rows from the peers are in act before the list ends
    if ((rc = flush_wait(c))) return rc;
    if (tr) {
        const unsigned end_c = plan.status ? unsigned(plan.status - 1) : n_cmds;
        if ((rc = stamp(c, tr, end_c, 0))) return rc;
        if ((rc = stamp(c, tr, end_c + 1, 3))) return rc;
        CUDA_TRY(c, cudaMemcpyAsync(c->ttags, c->host_tags.data(), sizeof(uint32_t) * c->n_events,
                                    cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(c, launch_trace_write(c->tstamps, c->ttags, c->n_events, c->act + plan.trace_off, c->stream));
        c->launches += c->n_events + 1;
    }
    return 0;
}

Limits limits_of(const b200q_ctx *c) {
    Limits L;
    L.act_floats = c->act_floats;
    L.state_rows = c->state_rows;
    L.kv_bytes = c->kv_bytes;
    L.kv_ctx = c->kv_ctx;
    L.check_weights = true;
    L.weights = &c->weights;
    L.defer_norms = (c->feature_mask & kMaskDeferNorm) != 0;
    L.fuse_rowops = (c->feature_mask & kMaskRowOps) != 0;
    L.fuse_attn_gate = (c->feature_mask & kMaskAttnGate) != 0;
    L.world = unsigned(c->world);
    return L;
}

// A pass whose bounded wait ran out sets the device error word (dstatus[1]); read and clear it after a sync.
int check_device_status(b200q_ctx *c) {
    unsigned st[2] = {0, 0};
    CUDA_TRY(c, cudaMemcpy(st, c->dstatus, sizeof(st), cudaMemcpyDeviceToHost));
    if (st[0] | st[1]) {
        const unsigned zero[2] = {0, 0};
        CUDA_TRY(c, cudaMemcpy(c->dstatus, zero, sizeof(zero), cudaMemcpyHostToDevice));
        if (st[1]) return set_err(c, B200Q_ERR_TIMEOUT, "a bounded wait ran out (weight tiles, or a peer GPU's rows)");
        if (st[0] & 2u) return set_err(c, B200Q_ERR_ARG, "ATTN: the position in act is outside the KV slot");
        return set_err(c, B200Q_ERR_ARG, "GET_ROW: the row index in act is outside the matrix");
    }
    return 0;
}

int check_ctx(b200q_ctx *c) {
    if (!c) return B200Q_ERR_ARG;
    if (c->disabled) return B200Q_ERR_DISABLED;
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return set_err(c, B200Q_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    return 0;
}

}  // namespace

// =================================================================================================================
extern "C" {

void b200q_features(uint32_t out[3]) {
    out[0] = B200Q_FEATURES;
    out[1] = B200Q_FEATURES2;
    out[2] = B200Q_FEATURES3;
}

int b200q_create(const b200q_config *cfg, b200q_ctx **out) {
    if (!cfg || !out) return B200Q_ERR_ARG;
    *out = nullptr;
    if (cfg->act_floats < 16 || cfg->act_floats % 16) return B200Q_ERR_ARG;
    b200q_ctx *c = new b200q_ctx();
    c->device = cfg->device;
    auto fail = [&](cudaError_t e, const char *what) {
        fprintf(stderr, "b200q_create: %s: %s\n", what, cudaGetErrorString(e));
        b200q_destroy(c);
        return B200Q_ERR_CUDA;
    };
    cudaError_t e;
    if ((e = cudaSetDevice(cfg->device)) != cudaSuccess) return fail(e, "cudaSetDevice");
    cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, cfg->device);
    if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess) return fail(e, "stream");
    c->wbytes = cfg->weight_bytes;
    if (c->wbytes && (e = cudaMalloc(&c->warena, c->wbytes)) != cudaSuccess) return fail(e, "weight arena");
    c->act_floats = cfg->act_floats;
    if ((e = cudaMalloc(&c->act, c->act_floats * sizeof(float))) != cudaSuccess) return fail(e, "act");
    cudaMemset(c->act, 0, c->act_floats * sizeof(float));
    c->state_rows = cfg->state_rows;
    if (c->state_rows) {
        if ((e = cudaMalloc(&c->state, c->state_rows * 128 * sizeof(float))) != cudaSuccess) return fail(e, "state");
        cudaMemset(c->state, 0, c->state_rows * 128 * sizeof(float));
    }
    c->kv_bytes = cfg->kv_bytes;
    c->kv_ctx = cfg->kv_ctx;
    if (c->kv_bytes) {
        if ((e = cudaMalloc(&c->kv, c->kv_bytes)) != cudaSuccess) return fail(e, "kv");
        cudaMemset(c->kv, 0, c->kv_bytes);
        if ((e = cudaMalloc(&c->attn_part, kAttnPartFloats * sizeof(float))) != cudaSuccess) return fail(e, "attn");
    }
    const size_t scratch = kMaxCols + 4 * (kMaxCols / 16) * 4 + kMaxCols * 4 + kSnapFloats * 4 + 4096 +
                           kMaxTraceEvents * 12;
    uint8_t *s = nullptr;
    if ((e = cudaMalloc(&s, scratch)) != cudaSuccess) return fail(e, "scratch");
    cudaMemset(s, 0, scratch);
    c->xq = reinterpret_cast<int8_t *>(s);
    s += kMaxCols;
    c->xd = reinterpret_cast<float *>(s);
    s += kMaxCols / 16 * 4;
    c->xs = reinterpret_cast<float *>(s);
    s += kMaxCols / 16 * 4;
    c->xb = reinterpret_cast<int32_t *>(s);
    s += kMaxCols / 16 * 4;
    c->xd16 = reinterpret_cast<uint16_t *>(s);
    s += kMaxCols / 16 * 4;
    c->ndrow = reinterpret_cast<float *>(s);
    s += kMaxCols * 4;
    c->snap = reinterpret_cast<float *>(s);
    s += kSnapFloats * 4;
    c->dstatus = reinterpret_cast<unsigned *>(s);
    s += 4096;
    c->tstamps = reinterpret_cast<unsigned long long *>(s);
    s += kMaxTraceEvents * 8;
    c->ttags = reinterpret_cast<uint32_t *>(s);
    uint8_t *qi = nullptr;
    if ((e = cudaMalloc(&qi, 2 * kQImageBytes)) != cudaSuccess) return fail(e, "image scratch");
    c->qimg[0] = qi;
    c->qimg[1] = qi + kQImageBytes;
    double *nq = nullptr;
    if ((e = cudaMalloc(&nq, 2 * kMaxNsqPanels * sizeof(double))) != cudaSuccess) return fail(e, "norm partials");
    c->nsq[0] = nq;
    c->nsq[1] = nq + kMaxNsqPanels;
    if ((e = cudaMalloc(&c->chain_counters, kMaxChains * kChainCounters * sizeof(unsigned))) != cudaSuccess)
        return fail(e, "chain counters");
    cudaMemset(c->chain_counters, 0, kMaxChains * kChainCounters * sizeof(unsigned));
    const char *pdl = getenv("B200Q_NO_PDL");
    c->pdl_env = !(pdl && pdl[0] == '1');
    const char *mask = getenv("B200Q_FEATURE_MASK");
    c->feature_mask = mask && mask[0] ? uint32_t(strtoul(mask, nullptr, 0)) : kDefaultFeatureMask;
    c->pdl = c->pdl_env && (c->feature_mask & kMaskPdl);
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return fail(e, "init");
    *out = c;
    return 0;
}

void b200q_destroy(b200q_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (unsigned p = 0; p < kMaxPeers; ++p) {
        if (c->peer_act[p]) cudaIpcCloseMemHandle(c->peer_act[p]);
        if (c->peer_sync[p]) cudaIpcCloseMemHandle(c->peer_sync[p]);
        if (c->peer_coll_recv[p]) cudaIpcCloseMemHandle(c->peer_coll_recv[p]);
    }
    cudaFree(c->sync);
    cudaFree(c->coll_recv);
    cudaFree(c->coll_flags);
    if (c->comm && g_nccl.comm_destroy) g_nccl.comm_destroy(c->comm);
    cudaFree(c->warena);
    cudaFree(c->qimg[0]);
    cudaFree(c->nsq[0]);
    cudaFree(c->chain_counters);
    cudaFree(c->act);
    cudaFree(c->state);
    cudaFree(c->kv);
    cudaFree(c->attn_part);
    cudaFree(c->xq);
    cudaFree(c->gemm_img);
    for (uint8_t *p : c->gemm_img_old) cudaFree(p);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

const char *b200q_last_error(const b200q_ctx *c) { return c ? c->err.c_str() : "null context"; }
void *b200q_stream(b200q_ctx *c) { return c ? c->stream : nullptr; }
void *b200q_act_device_ptr(b200q_ctx *c) { return c ? c->act : nullptr; }
void *b200q_state_device_ptr(b200q_ctx *c) { return c ? c->state : nullptr; }
void *b200q_kv_device_ptr(b200q_ctx *c) { return c ? c->kv : nullptr; }

int b200q_synchronize(b200q_ctx *c) {
    int rc = check_ctx(c);
    if (rc) return rc;
    CUDA_TRY(c, cudaStreamSynchronize(c->stream));
    return check_device_status(c);
}

size_t b200q_gguf_row_bytes(unsigned cols, unsigned format) { return gguf_row_bytes(cols, format); }

size_t b200q_weight_device_bytes(unsigned rows, unsigned cols, unsigned format) {
    return b200q_weight_device_bytes_ex(rows, cols, format, 0);
}

size_t b200q_weight_device_bytes_ex(unsigned rows, unsigned cols, unsigned format, unsigned flags) {
    if (!format_supported(format)) return 0;
    return device_layout(rows, cols, format, 148, flags >> 8).total;
}

int b200q_row_slice(unsigned rows, unsigned flags, int world, int rank, unsigned *r0, unsigned *r1) {
    if (!r0 || !r1 || world < 1 || rank < 0 || rank >= world) return B200Q_ERR_ARG;
    *r0 = 0;
    *r1 = rows;
    if (world > 1 && !(flags & B200Q_UPLOAD_REPLICATE) && rows % (16u * unsigned(world)) == 0) {
        const unsigned per = rows / unsigned(world);
        *r0 = per * unsigned(rank);
        *r1 = *r0 + per;
    }
    return 0;
}

int b200q_upload_weight_ex(b200q_ctx *c, const void *gguf, unsigned rows, unsigned cols, unsigned format,
                           unsigned block_cols, unsigned flags, uint64_t *w_off) {
    int rc = check_ctx(c);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(c->mu);
    if (!gguf || !w_off || !format_supported(format) || rows == 0 || rows > 1u << 20 || cols == 0 ||
        cols > kMaxCols || cols % ((format == 13 || format == 14) ? 256u : 32u) != 0 ||
        (block_cols != 0 && block_cols != 256))
        return set_err(c, B200Q_ERR_ARG, "upload: bad shape or format");
    unsigned r0 = 0, r1 = rows;
    if (!c->explicit_comm) b200q_row_slice(rows, flags, c->world, c->rank, &r0, &r1);
    // the pass hint, scaled to this rank's share when the matrix is sharded
    const unsigned pass_rows = unsigned(uint64_t(flags >> 8) * (r1 - r0) / rows);
    const DeviceLayout L = device_layout(r1 - r0, cols, format, unsigned(c->sms), pass_rows);
    if (c->wused + L.total > c->wbytes) return set_err(c, B200Q_ERR_NOMEM, "weight arena full");
    const uint8_t *src = static_cast<const uint8_t *>(gguf);
    std::vector<uint8_t> rows_q40;
    if (flags & B200Q_UPLOAD_SRC_Q4_0X8) {  // CPU_REPACK source: back to GGUF rows first (ggml-xrt.cpp:675-710)
        if (format != B200Q_Q4_0 || rows % 8) return set_err(c, B200Q_ERR_ARG, "upload: Q4_0x8 source needs Q4_0, rows % 8 == 0");
        rows_q40.resize(size_t(rows) * (cols / 32) * 18);
        b200q_q4_0x8_to_q4_0(gguf, rows, cols, rows_q40.data());
        src = rows_q40.data();
    }
    std::vector<uint8_t> host(L.total);
    repack_rows(src, r0, r1, L, host.data());
    CUDA_TRY(c, cudaMemcpy(c->warena + c->wused, host.data(), L.total, cudaMemcpyHostToDevice));
    WeightInfo w;
    w.handle = c->wused;
    w.format = format;
    w.rows = rows;
    w.cols = cols;
    w.row_begin = r0;
    w.row_end = r1;
    w.base_off = c->wused;
    w.rt = L.rt;
    w.ct = L.ct;
    w.kc = L.kc;
    w.n_rt = L.n_rt;
    w.tile_bytes = L.tile_bytes;
    w.qs_part = L.qs_part;
    w.dm_part = L.dm_part;
    c->weights.push_back(w);
    *w_off = w.handle;
    c->wused += (L.total + 255) & ~size_t(255);
    return 0;
}

int b200q_upload_weight(b200q_ctx *c, const void *gguf, unsigned rows, unsigned cols, unsigned format,
                        unsigned block_cols, uint64_t *w_off) {
    return b200q_upload_weight_ex(c, gguf, rows, cols, format, block_cols, 0, w_off);
}

int b200q_weights_reset(b200q_ctx *c) {
    int rc = check_ctx(c);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(c->mu);
    CUDA_TRY(c, cudaStreamSynchronize(c->stream));
    c->weights.clear();
    c->wused = 0;
    return 0;
}

int b200q_act_write(b200q_ctx *c, size_t off, const float *src, size_t n) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!src || off > c->act_floats || n > c->act_floats - off) return set_err(c, B200Q_ERR_ARG, "act_write range");
    CUDA_TRY(c, cudaMemcpyAsync(c->act + off, src, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(c, cudaStreamSynchronize(c->stream));
    return 0;
}

int b200q_act_read(b200q_ctx *c, size_t off, float *dst, size_t n) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!dst || off > c->act_floats || n > c->act_floats - off) return set_err(c, B200Q_ERR_ARG, "act_read range");
    CUDA_TRY(c, cudaMemcpyAsync(dst, c->act + off, n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(c, cudaStreamSynchronize(c->stream));
    return 0;
}

int b200q_act_write_async(b200q_ctx *c, size_t off, const float *src, size_t n) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!src || off > c->act_floats || n > c->act_floats - off) return set_err(c, B200Q_ERR_ARG, "act_write range");
    CUDA_TRY(c, cudaMemcpyAsync(c->act + off, src, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    return 0;
}

int b200q_act_read_async(b200q_ctx *c, size_t off, float *dst, size_t n) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!dst || off > c->act_floats || n > c->act_floats - off) return set_err(c, B200Q_ERR_ARG, "act_read range");
    CUDA_TRY(c, cudaMemcpyAsync(dst, c->act + off, n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    return 0;
}

int b200q_act_fill(b200q_ctx *c, size_t off, float value, size_t n) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (off > c->act_floats || n > c->act_floats - off) return set_err(c, B200Q_ERR_ARG, "act_fill range");
    std::vector<float> v(n, value);
    CUDA_TRY(c, cudaMemcpyAsync(c->act + off, v.data(), n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(c, cudaStreamSynchronize(c->stream));
    return 0;
}

int b200q_state_write(b200q_ctx *c, size_t row, const float *src, size_t rows) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!src || row > c->state_rows || rows > c->state_rows - row) return set_err(c, B200Q_ERR_ARG, "state range");
    CUDA_TRY(c, cudaMemcpy(c->state + row * 128, src, rows * 128 * sizeof(float), cudaMemcpyHostToDevice));
    return 0;
}

int b200q_state_read(b200q_ctx *c, size_t row, float *dst, size_t rows) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!dst || row > c->state_rows || rows > c->state_rows - row) return set_err(c, B200Q_ERR_ARG, "state range");
    CUDA_TRY(c, cudaStreamSynchronize(c->stream));
    CUDA_TRY(c, cudaMemcpy(dst, c->state + row * 128, rows * 128 * sizeof(float), cudaMemcpyDeviceToHost));
    return 0;
}

int b200q_kv_write(b200q_ctx *c, size_t byte_off, const void *src, size_t bytes) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!src || byte_off > c->kv_bytes || bytes > c->kv_bytes - byte_off) return set_err(c, B200Q_ERR_ARG, "kv range");
    CUDA_TRY(c, cudaMemcpy(reinterpret_cast<uint8_t *>(c->kv) + byte_off, src, bytes, cudaMemcpyHostToDevice));
    return 0;
}

int b200q_run_async(b200q_ctx *c, const uint32_t *cmds, unsigned n_cmds) {
    int rc = check_ctx(c);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(c->mu);
    if (n_cmds == 0) {  // feature probe (gemvqc16.h:124-134); the mask hides fused forms (ggml-xrt.cpp:1294-1299)
        uint32_t f[3];
        b200q_features(f);
        f[0] &= c->feature_mask | kFeatureKeep;
        CUDA_TRY(c, cudaMemcpyAsync(c->act, f, sizeof(f), cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(c, cudaStreamSynchronize(c->stream));
        return 0;
    }
    if (!cmds) return B200Q_ERR_ARG;
    const Plan plan = plan_list(cmds, n_cmds, limits_of(c));
    if (plan.status == 129) return 129;
    if ((rc = prepare_gemm_image(c, plan))) return rc;
    if ((rc = exec_plan(c, plan, n_cmds))) return rc;
    if (plan.status) c->err = plan.error;
    return plan.status;
}

namespace {
// Host copies of the device buffers a list reads and writes (runtime verification).
struct HostSnap {
    std::vector<float> act, state;
    std::vector<uint8_t> kv;
};

bool verifying(const b200q_ctx *c) { return c && !c->disabled && c->verify_fn && c->verify_left > 0; }

int snapshot(b200q_ctx *c, HostSnap &s) {
    CUDA_TRY(c, cudaStreamSynchronize(c->stream));
    s.act.resize(c->act_floats);
    CUDA_TRY(c, cudaMemcpy(s.act.data(), c->act, c->act_floats * sizeof(float), cudaMemcpyDeviceToHost));
    s.state.resize(c->state_rows * 128);
    if (c->state_rows)
        CUDA_TRY(c, cudaMemcpy(s.state.data(), c->state, s.state.size() * sizeof(float), cudaMemcpyDeviceToHost));
    s.kv.resize(c->kv_bytes);
    if (c->kv_bytes) CUDA_TRY(c, cudaMemcpy(s.kv.data(), c->kv, c->kv_bytes, cudaMemcpyDeviceToHost));
    return 0;
}

// After a verified list ran (and the stream was synchronized): hands the buffers before and after to the caller's
// checker, which recomputes the list on the host (reference: GGML_XRT_VERIFY_CALLS, ggml-xrt.cpp:1153-1202). A
// disagreement disables the context, as the reference backend disables itself when a check throws.
int verify_after(b200q_ctx *c, const uint32_t *cmds, unsigned n_cmds, int status, const HostSnap &before) {
    HostSnap after;
    int rc = snapshot(c, after);
    if (rc) return rc;
    b200q_verify_view v;
    v.cmds = cmds;
    v.n_cmds = n_cmds;
    v.status = status;
    v.act_before = before.act.data();
    v.act_after = after.act.data();
    v.act_floats = c->act_floats;
    v.state_before = before.state.data();
    v.state_after = after.state.data();
    v.state_rows = c->state_rows;
    v.kv_before = before.kv.data();
    v.kv_after = after.kv.data();
    v.kv_bytes = c->kv_bytes;
    v.kv_ctx = c->kv_ctx;
    --c->verify_left;
    char msg[512] = "";
    if (c->verify_fn(c->verify_user, &v, msg, sizeof(msg)) != 0) {
        c->disabled = true;
        return set_err(c, B200Q_ERR_VERIFY, "verify: the list's results differ from the checker's: %s", msg);
    }
    return 0;
}
}  // namespace

int b200q_set_verify(b200q_ctx *c, b200q_verify_fn fn, void *user, int n_calls) {
    if (!c) return B200Q_ERR_ARG;
    std::lock_guard<std::mutex> lock(c->mu);
    if (n_calls < 0) {
        const char *v = getenv("B200Q_VERIFY_CALLS");
        n_calls = v && v[0] ? std::max(0, atoi(v)) : 0;
    }
    c->verify_fn = fn;
    c->verify_user = user;
    c->verify_left = fn ? n_calls : 0;
    return 0;
}

int b200q_set_feature_mask(b200q_ctx *c, uint32_t mask) {
    if (!c) return B200Q_ERR_ARG;
    std::lock_guard<std::mutex> lock(c->mu);
    c->feature_mask = mask;
    c->pdl = c->pdl_env && (mask & kMaskPdl);
    return 0;
}

uint32_t b200q_feature_mask(const b200q_ctx *c) { return c ? c->feature_mask : 0u; }

int b200q_run(b200q_ctx *c, const uint32_t *cmds, unsigned n_cmds) {
    const bool verify = verifying(c) && n_cmds > 0 && cmds;
    HostSnap before;
    if (verify) {
        int rc = check_ctx(c);
        if (rc || (rc = snapshot(c, before))) return rc;
    }
    const int status = b200q_run_async(c, cmds, n_cmds);
    if (status < 0) return status;
    int rc = check_ctx(c);
    if (rc) return rc;
    CUDA_TRY(c, cudaStreamSynchronize(c->stream));
    if ((rc = check_device_status(c))) return rc;
    if (verify && (rc = verify_after(c, cmds, n_cmds, status, before))) return rc;
    return status;
}

int b200q_graph_create(b200q_ctx *c, const uint32_t *cmds, unsigned n_cmds, b200q_graph **out) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!out || (!cmds && n_cmds)) return B200Q_ERR_ARG;
    *out = nullptr;
    std::lock_guard<std::mutex> lock(c->mu);
    const Plan plan = plan_list(cmds, n_cmds, limits_of(c));
    if (plan.status) {
        c->err = plan.error;
        return plan.status;
    }
    if ((rc = prepare_gemm_image(c, plan))) return rc;
    b200q_graph *g = new b200q_graph();
    g->ctx = c;
    CUDA_TRY(c, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    rc = exec_plan(c, plan, n_cmds);
    cudaGraph_t graph = nullptr;
    const cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
    if (rc || e != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        delete g;
        return rc ? rc : set_err(c, B200Q_ERR_CUDA, "capture: %s", cudaGetErrorString(e));
    }
    g->graph = graph;
    g->kernels = c->launches;
    g->cmds.assign(cmds, cmds + size_t(n_cmds) * B200Q_CMD_WORDS);
    const cudaError_t ie = cudaGraphInstantiate(&g->exec, graph, 0);
    if (ie != cudaSuccess) {
        cudaGraphDestroy(graph);
        delete g;
        return set_err(c, B200Q_ERR_CUDA, "instantiate: %s", cudaGetErrorString(ie));
    }
    *out = g;
    return 0;
}

namespace {
// One replay; under runtime verification a synchronous one, checked like b200q_run.
int launch_one(b200q_ctx *c, b200q_graph *g) {
    if (!verifying(c)) {
        CUDA_TRY(c, cudaGraphLaunch(g->exec, c->stream));
        return 0;
    }
    HostSnap before;
    int rc = snapshot(c, before);
    if (rc) return rc;
    CUDA_TRY(c, cudaGraphLaunch(g->exec, c->stream));
    CUDA_TRY(c, cudaStreamSynchronize(c->stream));
    if ((rc = check_device_status(c))) return rc;
    return verify_after(c, g->cmds.data(), unsigned(g->cmds.size() / B200Q_CMD_WORDS), 0, before);
}
}  // namespace

int b200q_graph_launch(b200q_ctx *c, b200q_graph *g) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!g || g->ctx != c) return B200Q_ERR_STATE;
    return launch_one(c, g);
}

int b200q_graph_launch_many(b200q_ctx *c, b200q_graph *const *graphs, unsigned n_graphs, unsigned launches) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!graphs || n_graphs == 0) return B200Q_ERR_ARG;
    for (unsigned i = 0; i < n_graphs; ++i)
        if (!graphs[i] || graphs[i]->ctx != c) return B200Q_ERR_STATE;
    for (unsigned i = 0; i < launches; ++i)
        if ((rc = launch_one(c, graphs[i % n_graphs]))) return rc;
    return 0;
}

void b200q_graph_destroy(b200q_graph *g) {
    if (!g) return;
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    delete g;
}

unsigned b200q_graph_kernel_count(const b200q_graph *g) { return g ? g->kernels : 0; }

int b200q_plan(const uint32_t *cmds, unsigned n_cmds, b200q_pass_info *passes, unsigned max_passes,
               unsigned *n_passes) {
    if (n_passes) *n_passes = 0;
    if (n_cmds == 0) return 0;
    if (!cmds) return B200Q_ERR_ARG;
    Limits L;
    L.kv_ctx = 1u << 30;
    const Plan plan = plan_list(cmds, n_cmds, L);
    unsigned k = 0;
    for (const Pass &p : plan.passes) {
        if (passes && k < max_passes) {
            b200q_pass_info &o = passes[k];
            o.first_cmd = p.first;
            o.n_cmds = p.count;
            o.kind = p.kind == PassKind::RowOps ? uint32_t(PassKind::Elementwise) : uint32_t(p.kind);
            o.n_members = p.kind == PassKind::Gemv ? p.n_members
                                                   : (p.kind == PassKind::Gdn ? unsigned(p.gdn_with_gemv) + unsigned(p.gdn_with_out) : 0u);
            o.fused_norm = p.from_nd ? (p.nd.materialize ? 2u : 1u) : 0u;
        }
        ++k;
    }
    if (n_passes) *n_passes = k;
    return plan.status;
}

int b200q_debug_quantize(b200q_ctx *c, unsigned format, size_t x_off, unsigned n, uint32_t norm_w_off,
                         float norm_eps, unsigned norm_flags, int8_t *q, void *scales, int32_t *bsums) {
    int rc = check_ctx(c);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(c->mu);
    const unsigned act = act_type(format);
    if (!format_supported(format) || n == 0 || n > kMaxCols || n % (act == 2 ? 256u : 32u) || x_off % 16 ||
        x_off + n > c->act_floats || (norm_w_off != UINT32_MAX && norm_w_off + size_t(n) > c->act_floats))
        return set_err(c, B200Q_ERR_ARG, "debug_quantize: bad arguments");
    QuantArgs a;
    a.x = c->act + x_off;
    a.n = n;
    a.act = act;
    if (norm_w_off != UINT32_MAX) {
        a.norm_w = c->act + norm_w_off;
        a.norm_eps = norm_eps;
        a.norm_mode = 8u | (norm_flags & 3u);
    }
    a.q = c->xq;
    a.d = c->xd;
    a.s = c->xs;
    a.b = c->xb;
    a.d16 = c->xd16;
    CUDA_TRY(c, launch_quantize(a, c->stream));
    CUDA_TRY(c, cudaStreamSynchronize(c->stream));
    if (q) CUDA_TRY(c, cudaMemcpy(q, c->xq, n, cudaMemcpyDeviceToHost));
    if (scales) {
        if (act == 0) CUDA_TRY(c, cudaMemcpy(scales, c->xd16, n / 32 * 2, cudaMemcpyDeviceToHost));
        else if (act == 1) CUDA_TRY(c, cudaMemcpy(scales, c->xd16, n / 32 * 4, cudaMemcpyDeviceToHost));
        else CUDA_TRY(c, cudaMemcpy(scales, c->xd, n / 256 * 4, cudaMemcpyDeviceToHost));
    }
    if (bsums) CUDA_TRY(c, cudaMemcpy(bsums, c->xb, (act == 2 ? n / 16 : n / 32) * 4, cudaMemcpyDeviceToHost));
    return 0;
}

int b200q_debug_block_sums(b200q_ctx *c, const uint32_t cmd[8], int32_t *out) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!cmd || !out) return B200Q_ERR_ARG;
    std::lock_guard<std::mutex> lock(c->mu);
    if (cmd[0] == 17u && ((cmd[1] >> 16) & 0xffffu) + 1u > kBatchMax) {
        // the tensor-core GEMM of a GEMV_BATCH command: the int32 sums of block 0 for rows and tokens 0..127
        const Plan plan = plan_list(cmd, 1, limits_of(c));
        if (plan.status) return set_err(c, B200Q_ERR_ARG, "debug_block_sums: invalid GEMV_BATCH (%s)", plan.error.c_str());
        const size_t count = size_t(kGemmRows) * kGemmTokens;
        int32_t *d = nullptr;
        CUDA_TRY(c, cudaMalloc(&d, count * 4));
        cudaMemset(d, 0, count * 4);
        c->gemm_sums = d;
        rc = prepare_gemm_image(c, plan);
        if (!rc) rc = exec_plan(c, plan, 1);
        c->gemm_sums = nullptr;
        cudaError_t e = cudaStreamSynchronize(c->stream);
        if (!rc && e == cudaSuccess) e = cudaMemcpy(out, d, count * 4, cudaMemcpyDeviceToHost);
        cudaFree(d);
        if (rc) return rc;
        if (e != cudaSuccess) return set_err(c, B200Q_ERR_CUDA, "debug_block_sums: %s", cudaGetErrorString(e));
        return check_device_status(c);
    }
    uint32_t one[8];
    std::memcpy(one, cmd, sizeof(one));
    one[1] &= 0xffu;  // no epilogue
    const Plan plan = plan_list(one, 1, limits_of(c));
    if (plan.status || plan.passes.size() != 1 || plan.passes[0].kind != PassKind::Gemv)
        return set_err(c, B200Q_ERR_ARG, "debug_block_sums: invalid GEMV (%s)", plan.error.c_str());
    const Member &m = plan.passes[0].m[0];
    const bool kq = act_type(m.format) == 2;
    const size_t count = kq ? size_t(m.rows) * (m.cols / 256) * 9 : size_t(m.rows) * (m.cols / 32);
    int32_t *d = nullptr;
    CUDA_TRY(c, cudaMalloc(&d, count * 4));
    cudaMemset(d, 0, count * 4);
    DeferredNorm none;
    rc = exec_gemv(c, &m, 1, one[6], m.cols, false, none, false, nullptr, d);
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (!rc && e == cudaSuccess) e = cudaMemcpy(out, d, count * 4, cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (rc) return rc;
    if (e != cudaSuccess) return set_err(c, B200Q_ERR_CUDA, "debug_block_sums: %s", cudaGetErrorString(e));
    return 0;
}

int b200q_layout(unsigned rows, unsigned cols, unsigned format, unsigned sms, b200q_layout_info *out) {
    return b200q_layout_ex(rows, cols, format, sms, 0, out);
}

int b200q_layout_ex(unsigned rows, unsigned cols, unsigned format, unsigned sms, unsigned flags,
                    b200q_layout_info *out) {
    if (!out || !format_supported(format) || rows == 0 || cols == 0) return B200Q_ERR_ARG;
    const DeviceLayout L = device_layout(rows, cols, format, sms, flags >> 8);
    if (L.blocks == 0) return B200Q_ERR_ARG;
    out->rows_per_tile = L.rt;
    out->blocks_per_tile = L.ct;
    out->tiles_per_row_tile = L.kc;
    out->row_tiles = L.n_rt;
    out->tile_bytes = L.tile_bytes;
    out->total_bytes = L.total;
    return 0;
}

int b200q_repack_host(const void *gguf, unsigned rows, unsigned cols, unsigned format, unsigned sms, void *dst) {
    if (!gguf || !dst || !format_supported(format) || rows == 0) return B200Q_ERR_ARG;
    const DeviceLayout L = device_layout(rows, cols, format, sms);
    if (L.blocks == 0) return B200Q_ERR_ARG;
    repack_rows(static_cast<const uint8_t *>(gguf), 0, rows, L, static_cast<uint8_t *>(dst));
    return 0;
}

int b200q_unpack_row_host(const void *dev, unsigned rows, unsigned cols, unsigned format, unsigned sms, unsigned row,
                          void *gguf_row) {
    if (!dev || !gguf_row || !format_supported(format) || row >= rows) return B200Q_ERR_ARG;
    const DeviceLayout L = device_layout(rows, cols, format, sms);
    if (L.blocks == 0) return B200Q_ERR_ARG;
    unpack_row(static_cast<const uint8_t *>(dev), L, row, static_cast<uint8_t *>(gguf_row));
    return 0;
}

namespace {
// Map every peer's act and flag words into this process (CUDA IPC; the handles travel through one NCCL all-gather).
int setup_peers(b200q_ctx *c) {
    const size_t words = kSyncWords;
    CUDA_TRY(c, cudaMalloc(&c->sync, words * sizeof(unsigned)));
    CUDA_TRY(c, cudaMemset(c->sync, 0, words * sizeof(unsigned)));
    cudaIpcMemHandle_t mine[2];
    CUDA_TRY(c, cudaIpcGetMemHandle(&mine[0], c->act));
    CUDA_TRY(c, cudaIpcGetMemHandle(&mine[1], c->sync));
    static_assert(sizeof(mine) % sizeof(float) == 0, "handles travel as floats");
    const size_t n = sizeof(mine) / (sizeof(float));
    float *dev = nullptr;
    CUDA_TRY(c, cudaMalloc(&dev, sizeof(mine) * (size_t(c->world) + 1)));
    CUDA_TRY(c, cudaMemcpy(dev, mine, sizeof(mine), cudaMemcpyHostToDevice));
    const int r = g_nccl.all_gather(dev, dev + n, n, kNcclFloat32, c->comm, c->stream);
    std::vector<cudaIpcMemHandle_t> all(2 * size_t(c->world));
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), dev + n, sizeof(mine) * size_t(c->world), cudaMemcpyDeviceToHost);
    cudaFree(dev);
    if (r != 0) return set_err(c, B200Q_ERR_COMM, "ncclAllGather of the IPC handles: %d", r);
    if (e != cudaSuccess) return set_err(c, B200Q_ERR_CUDA, "IPC handle exchange: %s", cudaGetErrorString(e));
    for (int p = 0; p < c->world; ++p) {
        if (p == c->rank) continue;
        void *pa = nullptr, *pf = nullptr;
        CUDA_TRY(c, cudaIpcOpenMemHandle(&pa, all[2 * size_t(p)], cudaIpcMemLazyEnablePeerAccess));
        CUDA_TRY(c, cudaIpcOpenMemHandle(&pf, all[2 * size_t(p) + 1], cudaIpcMemLazyEnablePeerAccess));
        c->peer_act[p] = static_cast<float *>(pa);
        c->peer_sync[p] = static_cast<unsigned *>(pf);
    }
    c->peer_ok = true;
    return 0;
}

// Receive buffers of the peer ALLREDUCE (coll.cu), mapped into every peer (CUDA IPC; the handles travel through one
// NCCL all-gather), and this rank's launch counters.
int setup_coll_peers(b200q_ctx *c) {
    const size_t recv_bytes = size_t(kCollSlots) * 2 * c->world * kCollMaxN * sizeof(uint2);
    const size_t flag_bytes = size_t(kCollSlots) * kCollMaxCtas * sizeof(unsigned);
    CUDA_TRY(c, cudaMalloc(&c->coll_recv, recv_bytes));
    CUDA_TRY(c, cudaMalloc(&c->coll_flags, flag_bytes));
    // zeroed in stream order before the handle exchange: a peer's all-gather completes only after this rank's ran,
    // so no peer writes into these words before they are zero (launch number 0 never matches a launch)
    CUDA_TRY(c, cudaMemsetAsync(c->coll_recv, 0, recv_bytes, c->stream));
    CUDA_TRY(c, cudaMemsetAsync(c->coll_flags, 0, flag_bytes, c->stream));
    cudaIpcMemHandle_t mine;
    CUDA_TRY(c, cudaIpcGetMemHandle(&mine, c->coll_recv));
    static_assert(sizeof(mine) % sizeof(float) == 0, "handles travel as floats");
    const size_t n = sizeof(mine) / (sizeof(float));
    float *dev = nullptr;
    CUDA_TRY(c, cudaMalloc(&dev, sizeof(mine) * (size_t(c->world) + 1)));
    CUDA_TRY(c, cudaMemcpy(dev, &mine, sizeof(mine), cudaMemcpyHostToDevice));
    const int r = g_nccl.all_gather(dev, dev + n, n, kNcclFloat32, c->comm, c->stream);
    std::vector<cudaIpcMemHandle_t> all(size_t(c->world));
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), dev + n, sizeof(mine) * size_t(c->world), cudaMemcpyDeviceToHost);
    cudaFree(dev);
    if (r != 0) return set_err(c, B200Q_ERR_COMM, "ncclAllGather of the IPC handles: %d", r);
    if (e != cudaSuccess) return set_err(c, B200Q_ERR_CUDA, "IPC handle exchange: %s", cudaGetErrorString(e));
    for (int p = 0; p < c->world; ++p) {
        if (p == c->rank) continue;
        void *pr = nullptr;
        CUDA_TRY(c, cudaIpcOpenMemHandle(&pr, all[size_t(p)], cudaIpcMemLazyEnablePeerAccess));
        c->peer_coll_recv[p] = static_cast<uint2 *>(pr);
    }
    CUDA_TRY(c, cudaDeviceSynchronize());
    c->coll_peer = true;
    return 0;
}
}  // namespace

int b200q_comm_unique_id(uint8_t id[B200Q_UNIQUE_ID_BYTES]) {
    std::string err;
    if (!id || !load_nccl(err)) return B200Q_ERR_COMM;
    NcclUniqueId u;
    if (g_nccl.get_unique_id(&u) != 0) return B200Q_ERR_COMM;
    std::memcpy(id, u.internal, B200Q_UNIQUE_ID_BYTES);
    return 0;
}

int b200q_comm_init(b200q_ctx *c, int world, int rank, const uint8_t id[B200Q_UNIQUE_ID_BYTES]) {
    return b200q_comm_init_ex(c, world, rank, id, 0);
}

int b200q_comm_init_ex(b200q_ctx *c, int world, int rank, const uint8_t id[B200Q_UNIQUE_ID_BYTES], unsigned flags) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (world < 1 || rank < 0 || rank >= world || !id) return B200Q_ERR_ARG;
    if (!c->weights.empty()) return set_err(c, B200Q_ERR_STATE, "comm_init after uploads");
    if (world == 1) return 0;
    std::string err;
    if (!load_nccl(err)) return set_err(c, B200Q_ERR_COMM, "%s", err.c_str());
    NcclUniqueId u;
    std::memcpy(u.internal, id, B200Q_UNIQUE_ID_BYTES);
    const int r = g_nccl.comm_init_rank(&c->comm, world, u, rank);
    if (r != 0) return set_err(c, B200Q_ERR_COMM, "ncclCommInitRank: %d", r);
    c->world = world;
    c->rank = rank;
    c->explicit_comm = (flags & B200Q_COMM_EXPLICIT) != 0;
    // row-sharded lists: outputs exchanged by peer stores (B200Q_PEER=1) or by an NCCL all-gather per sharded member
    // (default: the peer path's per-pass synchronisation costs more than the all-gather); explicit lists: ALLREDUCE by
    // the peer kernel (default: 3.8 us per 2560 floats on 2 GPUs against 10.3 us for ncclAllReduce in a graph) or by
    // NCCL (B200Q_PEER=0)
    const char *pe = getenv("B200Q_PEER");
    if (c->explicit_comm) {
        const bool peer = world <= int(kMaxPeers) && !(pe && pe[0] == '0');
        return peer ? setup_coll_peers(c) : 0;
    }
    if (world <= int(kMaxPeers) && pe && pe[0] == '1') return setup_peers(c);
    return 0;
}

int b200q_comm_world(const b200q_ctx *c) { return c ? c->world : 0; }

}  // extern "C"
