// Graph lowering (host only): a model's op graph, as an array of b200q_node in execution order, to command lists of
// the reference ISA with every tensor placed in act. The counterpart of the reference backend's plan / fusion
// analysis and list emission (ggml-xrt.cpp:1815-2188 and :2190-2745), restated over this library's own node type
// instead of ggml tensors:
//   1. readers: which nodes read each tensor, directly or through a VIEW of it;
//   2. fusions, each behind its feature bit (the reference's feature word, ggml-xrt.cpp:342-363): SwiGLU GEMV pairs,
//      ADD / CONV epilogues of a GEMV, weighted and deferred RMSNORMs, the DeltaNet step's L2 q/k, gates, gated
//      output norm and the GEMV that joins its pass, SILU / SIGMOID folded into a MUL;
//   3. placement: INPUT and PARAM tensors and every tensor a command writes get 16-float aligned act regions in node
//      order (a node with `dst` writes into the region of an earlier INPUT instead);
//   4. emission in node order, commands of a fused group at the position the reference emits them; segments
//      (B200Q_NODE_SEGMENT_END) packed into lists of at most 128 commands.
// Every check a list would fail in the planner (plan.cpp) is made here first, so a lowering either fails with the
// node named or gives lists the device accepts.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/b200q.h"
#include "plan.h"

namespace {

using b200q::kAddRows;
using b200q::kBufWords;
using b200q::kHead;
using b200q::kMaxBlockedRows;
using b200q::kMaxConvChannels;
using b200q::kMaxHeads;
using b200q::kMaxNormRows;
using b200q::kMaxRopeDims;
using b200q::kMaxRows;
using b200q::kMaxCols;
using b200q::kNxFloats;
using b200q::kPairRows;
using b200q::kStateUnits;

constexpr size_t kNone = SIZE_MAX;
constexpr unsigned kMaxListCmds = 128;

// feature bits of the reference's feature word (ggml-xrt.cpp:346-363)
constexpr uint32_t kFeatSwiglu = 1u << 3, kFeatConvEpi = 1u << 6, kFeatGdnNorms = 1u << 7, kFeatAddEpi = 1u << 8,
                   kFeatNormDefer = 1u << 9, kFeatGdnGates = 1u << 10, kFeatGdnOut = 1u << 15,
                   kFeatSigmoidMul = 1u << 16;

unsigned round16(unsigned n) { return (n + 15u) & ~15u; }
uint32_t fbits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
unsigned act_type(unsigned fmt) { return fmt == 13 || fmt == 14 ? 2u : (fmt == 3 ? 1u : 0u); }

struct GdnFuse {
    bool l2 = false, gated = false, gates = false;
    int qn = -1, kn = -1;                 // the L2_NORM nodes
    float l2_eps = 0.0f, rms_eps = 0.0f;
    int out = -1, norm = -1, wmul = -1, silu = -1, w = -1, z = -1;  // gated output chain
    int alpha = -1, beta = -1, dt = -1, a = -1, sig = -1, gmul = -1, sp = -1, gadd = -1;
    int with_out = -1;                    // the GEMV of the step's pass
};

struct Lowering {
    const b200q_node *nd = nullptr;
    unsigned n = 0;
    uint32_t feat = 0;
    std::string err;
    std::vector<std::vector<int>> users;  // direct users (VIEW nodes included)
    std::vector<int> seg;
    std::vector<char> seg_list_end;  // the list ends after this segment
    // fusion roles
    std::vector<char> silent;   // emits nothing at its own position
    std::vector<char> storage;  // holds floats in act
    std::vector<int> pair_g, pair_u, add_epi, conv_epi, wnorm, fold_unary;
    std::vector<int> emit_at;   // the node whose position a node's command is emitted at (itself, or a pair's SWIGLU)
    std::vector<char> deferred;
    std::map<int, GdnFuse> gdn;
    std::vector<char> done;     // emitted already (the GEMV of a GDN pass)
    // placement and output
    std::vector<size_t> off;
    size_t act = 0;
    std::vector<std::vector<uint32_t>> seg_cmds;
    std::vector<std::vector<uint32_t>> lists;

    bool fail(int i, const char *fmt, ...) {
        char buf[256];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        char head[64];
        snprintf(head, sizeof(head), "node %d (op %u): ", i, i >= 0 && unsigned(i) < n ? nd[i].op : 0u);
        err = std::string(head) + buf;
        return false;
    }
    int src(int i, int k) const { return nd[i].src[k]; }
    bool is(int i, uint32_t op) const { return i >= 0 && nd[i].op == op; }
    // a MUL_MAT of one activation row (a GEMV, which the fusions may join); one of several rows (u[0] > 1) is a
    // GEMV_BATCH of its own
    bool gemv_mm(int i) const { return is(i, B200Q_NODE_MUL_MAT) && nd[i].u[0] <= 1; }
    bool output(int i) const { return (nd[i].flags & B200Q_NODE_OUTPUT) != 0; }
    // the non-VIEW nodes that read i, directly or through views of it
    void real_readers(int i, std::vector<int> &out) const {
        for (int u : users[size_t(i)]) {
            if (nd[u].op == B200Q_NODE_VIEW) real_readers(u, out);
            else out.push_back(u);
        }
    }
    bool only_reader(int i, int r) const {
        std::vector<int> rr;
        real_readers(i, rr);
        for (int x : rr)
            if (x != r) return false;
        return !rr.empty() && !output(i);
    }
    // the base (non-VIEW) node of i and i's first float, row length, stride and rows relative to the base
    int base(int i) const { return nd[i].op == B200Q_NODE_VIEW ? nd[i].src[0] : i; }
    bool contiguous(int i) const {
        const b200q_node &v = nd[i];
        return v.op != B200Q_NODE_VIEW || v.u[3] <= 1 || v.u[1] == v.u[2];
    }
    size_t at(int i) const {
        if (nd[i].op == B200Q_NODE_VIEW) {
            const size_t b = off[size_t(nd[i].src[0])];
            return b == kNone ? kNone : b + nd[i].u[0];
        }
        return off[size_t(i)];
    }
    uint32_t o32(int i) const { return uint32_t(at(i)); }

    bool validate();
    void fuse();
    bool place();
    bool emit();
    void push(int i, std::initializer_list<uint32_t> w) {
        std::vector<uint32_t> &c = seg_cmds[size_t(seg[size_t(i)])];
        size_t k = 0;
        for (uint32_t x : w) c.push_back(x), ++k;
        for (; k < 8; ++k) c.push_back(0u);
    }
    void gemv(int m, uint32_t flags, uint32_t x, uint32_t y, int at_node) {
        const b200q_node &g = nd[m];
        push(at_node, {1u, g.fmt | flags, g.rows, g.cols, uint32_t(g.weight), uint32_t(g.weight >> 32), x, y});
    }
    void emit_gemv_with_epilogue(int m, int at_node);
};

bool Lowering::validate() {
    users.assign(n, {});
    seg.assign(n, 0);
    seg_list_end.assign(1, 0);
    int s = 0;
    for (unsigned i = 0; i < n; ++i) {
        const b200q_node &d = nd[i];
        seg[i] = s;
        if (d.flags & B200Q_NODE_LIST_END) seg_list_end[size_t(s)] = 1;
        if (d.flags & B200Q_NODE_SEGMENT_END) {
            ++s;
            seg_list_end.push_back(0);
        }
        for (unsigned k = 0; k < B200Q_NODE_SRCS; ++k) {
            const int r = d.src[k];
            if (r < -1 || r >= int(i)) return fail(int(i), "operand %u is not an earlier node", k);
            if (r >= 0) users[size_t(r)].push_back(int(i));
        }
        if (d.dst < -1 || d.dst >= int(i)) return fail(int(i), "dst is not an earlier node");
        if (d.op < B200Q_NODE_INPUT || d.op > B200Q_NODE_ALLGATHER) return fail(int(i), "unknown op");
        if (d.n == 0) return fail(int(i), "no floats");
        // operands every op needs (the fusion analysis reads them without further checks)
        static const unsigned kArity[] = {0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 1, 3, 5, 2, 4, 1, 1, 1, 1};
        for (unsigned k = 0; k < kArity[d.op]; ++k)
            if (d.src[k] < 0) return fail(int(i), "operand %u missing", k);
        if (d.op == B200Q_NODE_VIEW) {
            const int b = d.src[0];
            if (b < 0 || nd[b].op == B200Q_NODE_VIEW) return fail(int(i), "a VIEW views one non-VIEW node");
            const unsigned rows = d.u[3] ? d.u[3] : 1u;
            if (d.u[0] % 16 || d.u[1] == 0 || d.n != d.u[1] * rows || (rows > 1 && d.u[2] < d.u[1]) ||
                size_t(d.u[0]) + size_t(rows - 1) * d.u[2] + d.u[1] > round16(nd[b].n))
                return fail(int(i), "VIEW outside its node or not 16-float aligned");
        }
        if (d.dst >= 0) {
            const int t = d.dst, tb = nd[t].op == B200Q_NODE_VIEW ? nd[t].src[0] : t;
            if (nd[tb].op != B200Q_NODE_INPUT || !contiguous(t) || nd[t].n < d.n)
                return fail(int(i), "dst must be a contiguous INPUT region of at least n floats");
            if (d.op == B200Q_NODE_MUL_MAT && d.u[0] <= 1 && d.rows % 16 && nd[t].n < round16(d.rows))
                return fail(int(i), "a GEMV pads its output to 16 floats: dst needs that room");
            if (d.op == B200Q_NODE_ARGMAX && nd[t].n < 16) return fail(int(i), "ARGMAX writes into 16 floats of dst");
        }
    }
    seg_cmds.assign(size_t(s) + 1, {});
    return true;
}

void Lowering::fuse() {
    silent.assign(n, 0);
    storage.assign(n, 1);
    pair_g.assign(n, -1);
    pair_u.assign(n, -1);
    add_epi.assign(n, -1);
    conv_epi.assign(n, -1);
    wnorm.assign(n, -1);
    fold_unary.assign(n, -1);
    deferred.assign(n, 0);
    done.assign(n, 0);
    emit_at.resize(n);
    for (unsigned i = 0; i < n; ++i) emit_at[i] = int(i);
    for (unsigned i = 0; i < n; ++i)
        if (nd[i].op == B200Q_NODE_VIEW) storage[i] = 0;
    const auto plain_mm = [&](int m, int reader) {
        return gemv_mm(m) && !silent[size_t(m)] && only_reader(m, reader) && add_epi[size_t(m)] < 0 &&
               conv_epi[size_t(m)] < 0;
    };
    // ---- the DeltaNet step's folds first (their nodes are then not fused otherwise)
    for (unsigned gi = 0; gi < n; ++gi) {
        if (nd[gi].op != B200Q_NODE_GDN) continue;
        const int G = int(gi);
        const unsigned hv = nd[gi].u[0], hk = nd[gi].u[1];
        GdnFuse f;
        const int q = src(G, 0), k = src(G, 1);
        if ((feat & kFeatGdnNorms) && is(q, B200Q_NODE_L2_NORM) && is(k, B200Q_NODE_L2_NORM) && only_reader(q, G) &&
            only_reader(k, G) && nd[q].rows == hk && nd[k].rows == hk && nd[q].eps == nd[k].eps &&
            contiguous(src(q, 0)) && contiguous(src(k, 0))) {
            f.l2 = true;
            f.qn = q;
            f.kn = k;
            f.l2_eps = nd[q].eps;
        }
        // gated output: RMS_NORM (rows of 128) -> MUL by a 128-float weight -> MUL by SILU(z)
        std::vector<int> rr;
        real_readers(G, rr);
        if ((feat & kFeatGdnNorms) && rr.size() == 1 && !output(G) && is(rr[0], B200Q_NODE_RMS_NORM) &&
            src(rr[0], 0) == G && nd[rr[0]].rows == hv && nd[rr[0]].n == hv * kHead) {
            const int R = rr[0];
            std::vector<int> r1;
            real_readers(R, r1);
            const int M1 = r1.size() == 1 && !output(R) ? r1[0] : -1;
            if (M1 >= 0 && is(M1, B200Q_NODE_MUL) && src(M1, 0) == R && nd[src(M1, 1)].n == kHead &&
                contiguous(src(M1, 1))) {
                std::vector<int> r2;
                real_readers(M1, r2);
                const int M2 = r2.size() == 1 && !output(M1) ? r2[0] : -1;
                if (M2 >= 0 && is(M2, B200Q_NODE_MUL) && nd[M2].n == hv * kHead) {
                    const int S = src(M2, 0) == M1 ? src(M2, 1) : (src(M2, 1) == M1 ? src(M2, 0) : -1);
                    if (S >= 0 && is(S, B200Q_NODE_UNARY) && nd[S].u[0] == B200Q_UNARY_SILU && only_reader(S, M2) &&
                        nd[src(S, 0)].n == hv * kHead && contiguous(src(S, 0))) {
                        f.gated = true;
                        f.norm = R;
                        f.wmul = M1;
                        f.silu = S;
                        f.out = M2;
                        f.w = src(M1, 1);
                        f.z = src(S, 0);
                        f.rms_eps = nd[R].eps;
                    }
                }
            }
        }
        // gates: beta = SIGMOID(beta_raw), g = MUL(SOFTPLUS(ADD(alpha_raw, dt)), a)
        const int B = src(G, 4), Gm = src(G, 3);
        if ((feat & kFeatGdnGates) && is(B, B200Q_NODE_UNARY) && nd[B].u[0] == B200Q_UNARY_SIGMOID &&
            only_reader(B, G) && is(Gm, B200Q_NODE_MUL) && only_reader(Gm, G) && contiguous(src(B, 0))) {
            const int s0 = src(Gm, 0), s1 = src(Gm, 1);
            const int SP = is(s0, B200Q_NODE_UNARY) ? s0 : s1, A = SP == s0 ? s1 : s0;
            if (is(SP, B200Q_NODE_UNARY) && nd[SP].u[0] == B200Q_UNARY_SOFTPLUS && only_reader(SP, Gm) &&
                is(base(A), B200Q_NODE_PARAM) && contiguous(A) && nd[A].n == hv) {
                const int AD = src(SP, 0);
                if (is(AD, B200Q_NODE_ADD) && only_reader(AD, SP)) {
                    const int a0 = src(AD, 0), a1 = src(AD, 1);
                    const int DT = is(base(a1), B200Q_NODE_PARAM) ? a1 : (is(base(a0), B200Q_NODE_PARAM) ? a0 : -1);
                    const int AL = DT == a1 ? a0 : a1;
                    if (DT >= 0 && contiguous(DT) && contiguous(AL) && nd[DT].n == hv && nd[AL].n == hv) {
                        f.gates = true;
                        f.sig = B;
                        f.beta = src(B, 0);
                        f.gmul = Gm;
                        f.sp = SP;
                        f.gadd = AD;
                        f.alpha = AL;
                        f.dt = DT;
                        f.a = A;
                    }
                }
            }
        }
        if (f.l2) silent[size_t(f.qn)] = silent[size_t(f.kn)] = 1, storage[size_t(f.qn)] = storage[size_t(f.kn)] = 0;
        if (f.gated) {
            for (int x : {f.norm, f.wmul, f.silu}) silent[size_t(x)] = 1, storage[size_t(x)] = 0;
            silent[size_t(f.out)] = 1;      // written by the step
            storage[size_t(G)] = 0;         // the plain y is never in act
        }
        if (f.gates)
            for (int x : {f.sig, f.gmul, f.sp, f.gadd}) silent[size_t(x)] = 1, storage[size_t(x)] = 0;
        gdn[G] = f;
    }
    // ---- SwiGLU GEMV pairs
    for (unsigned i = 0; i < n && (feat & kFeatSwiglu); ++i) {
        if (nd[i].op != B200Q_NODE_SWIGLU || silent[i]) continue;
        const int g = src(int(i), 0), u = src(int(i), 1);
        if (g != u && plain_mm(g, int(i)) && plain_mm(u, int(i)) && src(g, 0) == src(u, 0) &&
            nd[g].rows == nd[u].rows && nd[g].rows <= kPairRows && act_type(nd[g].fmt) == act_type(nd[u].fmt) &&
            nd[i].n == nd[g].rows) {
            pair_g[i] = g;
            pair_u[i] = u;
            emit_at[size_t(g)] = emit_at[size_t(u)] = int(i);
            silent[size_t(g)] = silent[size_t(u)] = 1;
            storage[size_t(g)] = storage[size_t(u)] = 0;
        }
    }
    // ---- CONV epilogues
    for (unsigned i = 0; i < n && (feat & kFeatConvEpi); ++i) {
        if (nd[i].op != B200Q_NODE_CONV || silent[i]) continue;
        const int m = src(int(i), 0);
        if (plain_mm(m, int(i)) && nd[m].rows == nd[i].n) {
            conv_epi[size_t(m)] = int(i);
            silent[i] = 1;
        }
    }
    // ---- ADD epilogues: the residual operand exists before the GEMV (the reference keeps short adds out, 256 rows)
    for (unsigned i = 0; i < n && (feat & kFeatAddEpi); ++i) {
        if (nd[i].op != B200Q_NODE_ADD || silent[i]) continue;
        for (int k = 0; k < 2; ++k) {
            const int m = src(int(i), k), r = src(int(i), 1 - k);
            if (plain_mm(m, int(i)) && nd[m].rows == nd[i].n && nd[m].rows % 16 == 0 && nd[m].rows <= kAddRows &&
                nd[m].rows >= 256 && base(r) < m && m != r) {
                add_epi[size_t(m)] = int(i);
                silent[i] = 1;
                break;
            }
        }
    }
    // ---- weighted norms: RMS_NORM / L2_NORM read only by a MUL with a row-long weight
    for (unsigned i = 0; i < n; ++i) {
        if (nd[i].op != B200Q_NODE_MUL || silent[i]) continue;
        for (int k = 0; k < 2; ++k) {
            const int nm = src(int(i), k), w = src(int(i), 1 - k);
            if ((is(nm, B200Q_NODE_RMS_NORM) || is(nm, B200Q_NODE_L2_NORM)) && !silent[size_t(nm)] &&
                only_reader(nm, int(i)) && nd[w].n == nd[nm].n / (nd[nm].rows ? nd[nm].rows : 1u) && contiguous(w) &&
                nd[i].n == nd[nm].n) {
                wnorm[i] = nm;
                silent[size_t(nm)] = 1;
                storage[size_t(nm)] = 0;
                break;
            }
        }
    }
    // ---- deferred norms: a single-row norm (weighted or not) read only by MUL_MATs of its segment
    for (unsigned i = 0; i < n && (feat & kFeatNormDefer); ++i) {
        const int nm = wnorm[i] >= 0 ? wnorm[i] : ((is(int(i), B200Q_NODE_RMS_NORM) || is(int(i), B200Q_NODE_L2_NORM)) &&
                                                   !silent[i] ? int(i) : -1);
        if (nm < 0 || (nd[nm].rows > 1) || !contiguous(src(nm, 0)) || nd[i].n % 16 || nd[i].n > kNxFloats ||
            output(int(i)))
            continue;
        std::vector<int> rr;
        real_readers(int(i), rr);
        bool ok = !rr.empty();
        for (int r : rr)
            ok = ok && gemv_mm(r) && src(r, 0) == int(i) && seg[size_t(emit_at[size_t(r)])] == seg[i];
        if (ok) deferred[i] = 1;
    }
    // ---- SILU / SIGMOID folded into the MUL that reads them
    for (unsigned i = 0; i < n; ++i) {
        if (nd[i].op != B200Q_NODE_MUL || silent[i] || wnorm[i] >= 0) continue;
        for (int k = 0; k < 2; ++k) {
            const int un = src(int(i), k);
            if (!is(un, B200Q_NODE_UNARY) || silent[size_t(un)] || !only_reader(un, int(i)) || nd[un].n != nd[i].n)
                continue;
            const bool silu = nd[un].u[0] == B200Q_UNARY_SILU && contiguous(src(un, 0));
            const bool sig = nd[un].u[0] == B200Q_UNARY_SIGMOID && (feat & kFeatSigmoidMul);
            if (silu || sig) {
                fold_unary[i] = un;
                silent[size_t(un)] = 1;
                storage[size_t(un)] = 0;
                break;
            }
        }
    }
    // ---- the GEMV that joins a DeltaNet step's pass: the next command-emitting node reads the step's output
    for (auto &e : gdn) {
        const int G = e.first;
        GdnFuse &f = e.second;
        if (!(feat & kFeatGdnOut)) break;
        const int y = f.gated ? f.out : G;
        const unsigned hv = nd[G].u[0];
        int m = -1;
        for (unsigned j = unsigned(G) + 1; j < n; ++j) {
            if (nd[j].op == B200Q_NODE_VIEW || nd[j].op == B200Q_NODE_INPUT || nd[j].op == B200Q_NODE_PARAM || silent[j])
                continue;
            m = int(j);
            break;
        }
        if (m >= 0 && gemv_mm(m) && src(m, 0) == y && nd[m].cols == hv * kHead &&
            (hv * kHead) % 256 == 0 && nd[m].rows <= kMaxBlockedRows && conv_epi[size_t(m)] < 0 &&
            seg[size_t(m)] == seg[size_t(G)]) {
            f.with_out = m;
        }
    }
}

bool Lowering::place() {
    off.assign(n, kNone);
    act = 0;
    for (unsigned i = 0; i < n; ++i) {
        if (!storage[i] || nd[i].op == B200Q_NODE_VIEW) continue;
        if (nd[i].dst >= 0) {
            off[i] = at(nd[i].dst);
            continue;
        }
        off[i] = act;
        act += round16(nd[i].n);
    }
    // the stored norm a deferred RMSNORM names needs its region too (kept above); GEMV ys of epilogue members as well
    return true;
}

void Lowering::emit_gemv_with_epilogue(int m, int at_node) {
    const b200q_node &g = nd[m];
    const uint32_t x = o32(src(m, 0)), y = o32(m);
    if (add_epi[size_t(m)] >= 0) {
        const int a = add_epi[size_t(m)];
        const int r = src(a, 0) == m ? src(a, 1) : src(a, 0);
        gemv(m, B200Q_GEMV_ADD, x, y, at_node);
        push(at_node, {3u, g.rows, y, o32(r), o32(a)});
    } else if (conv_epi[size_t(m)] >= 0) {
        const int c = conv_epi[size_t(m)];
        gemv(m, B200Q_GEMV_CONV, x, y, at_node);
        push(at_node, {8u, g.rows, y, o32(src(c, 1)), o32(c), o32(src(c, 2)), o32(src(c, 2)), nd[c].u[0] ? 1u : 0u});
    } else {
        gemv(m, 0u, x, y, at_node);
    }
}

bool Lowering::emit() {
    for (unsigned ii = 0; ii < n; ++ii) {
        const int i = int(ii);
        const b200q_node &d = nd[i];
        if (d.op == B200Q_NODE_INPUT || d.op == B200Q_NODE_PARAM || d.op == B200Q_NODE_VIEW || silent[ii] || done[ii])
            continue;
        // a node that emits a command must fit the command's limits (nodes folded into another command need not)
        if (!b200q_node_supported(nd, ii)) return fail(i, "not supported (operands, sizes or format)");
        switch (d.op) {
        case B200Q_NODE_MUL_MAT:
            if (d.u[0] > 1) {  // several activation rows, cols floats apart: one GEMV_BATCH command
                if (!contiguous(src(i, 0))) return fail(i, "the activation rows of a batched MUL_MAT must be contiguous");
                push(i, {17u, d.fmt | ((d.u[0] - 1u) << 16), d.rows, d.cols, uint32_t(d.weight),
                         uint32_t(d.weight >> 32), o32(src(i, 0)), o32(i)});
            } else {
                emit_gemv_with_epilogue(i, i);
            }
            break;
        case B200Q_NODE_SWIGLU:
            if (pair_g[ii] >= 0) {
                if (!b200q_node_supported(nd, unsigned(pair_g[ii])) || !b200q_node_supported(nd, unsigned(pair_u[ii])))
                    return fail(i, "a SwiGLU member is not supported");
                const uint32_t x = o32(src(pair_g[ii], 0));
                gemv(pair_g[ii], B200Q_GEMV_SWIGLU, x, o32(i), i);
                gemv(pair_u[ii], 0u, x, o32(i), i);
            } else {
                push(i, {4u, d.n, o32(src(i, 0)), o32(src(i, 1)), o32(i)});
            }
            break;
        case B200Q_NODE_RMS_NORM:
        case B200Q_NODE_L2_NORM:
        case B200Q_NODE_MUL: {
            int nm = i, w = -1;
            if (d.op == B200Q_NODE_MUL && wnorm[ii] >= 0) {
                nm = wnorm[ii];
                w = src(i, 0) == nm ? src(i, 1) : src(i, 0);
            }
            if (nd[nm].op == B200Q_NODE_MUL) {  // a plain product, or SILU_MUL with the unary folded in
                const int un = fold_unary[ii];
                if (un < 0) {
                    if (nd[src(i, 0)].n != d.n || nd[src(i, 1)].n != d.n)
                        return fail(i, "a MUL by one row is only supported as the weight of the norm before it");
                    push(i, {5u, d.n, o32(src(i, 0)), o32(src(i, 1)), o32(i)});
                } else {
                    const int u = src(i, 0) == un ? src(i, 1) : src(i, 0), g = src(un, 0);
                    const bool sig = nd[un].u[0] == B200Q_UNARY_SIGMOID;
                    const unsigned row = contiguous(g) ? 0u : nd[g].u[1], stride = contiguous(g) ? 0u : nd[g].u[2];
                    if (row % 16 || stride % 16 || nd[u].n != d.n)
                        return fail(i, "SILU_MUL operands: 16-float rows and stride, equal lengths");
                    push(i, {4u, d.n, o32(g), o32(u), o32(i), sig ? 1u : 0u, row, stride});
                }
                break;
            }
            const b200q_node &N = nd[nm];
            const int x = src(nm, 0);
            const unsigned rows = N.rows ? N.rows : 1u, row = N.n / rows;
            if (!contiguous(x) && (nd[x].u[2] % 16 || nd[x].u[1] != row || (nd[x].u[3] ? nd[x].u[3] : 1u) != rows))
                return fail(i, "a norm's strided input must be its rows, 16-float strided");
            const unsigned stride_words = contiguous(x) ? 0u : nd[x].u[2] / 16u;
            uint32_t flags = (N.op == B200Q_NODE_L2_NORM ? B200Q_NORM_L2 : 0u) | (w < 0 ? B200Q_NORM_NO_WEIGHT : 0u);
            if (deferred[ii]) flags |= B200Q_NORM_DEFER;
            push(i, {2u, row, o32(x), w < 0 ? 0u : o32(w), o32(i), fbits(N.eps), N.rows, flags | (stride_words << 8)});
            break;
        }
        case B200Q_NODE_ADD:
            push(i, {3u, d.n, o32(src(i, 0)), o32(src(i, 1)), o32(i)});
            break;
        case B200Q_NODE_UNARY: {
            const int x = src(i, 0);
            const unsigned row = contiguous(x) ? 0u : nd[x].u[1], stride = contiguous(x) ? 0u : nd[x].u[2];
            if (row % 16 || stride % 16) return fail(i, "a strided input needs 16-float rows and stride");
            push(i, {6u, d.n, o32(x), d.u[0], o32(i), row, stride});
            break;
        }
        case B200Q_NODE_CONV:
            push(i, {8u, d.n, o32(src(i, 0)), o32(src(i, 1)), o32(i), o32(src(i, 2)), o32(src(i, 2)), d.u[0] ? 1u : 0u});
            break;
        case B200Q_NODE_GDN: {
            const GdnFuse &f = gdn[i];
            const unsigned hv = d.u[0], hk = d.u[1];
            const uint32_t q = f.l2 ? o32(src(f.qn, 0)) : o32(src(i, 0)), k = f.l2 ? o32(src(f.kn, 0)) : o32(src(i, 1));
            const uint32_t g = f.gates ? o32(f.alpha) : o32(src(i, 3)), beta = f.gates ? o32(f.beta) : o32(src(i, 4));
            const uint32_t y = f.gated ? o32(f.out) : o32(i);
            uint32_t flags = (f.l2 ? B200Q_GDN_L2_QK : 0u) | (f.gated ? B200Q_GDN_GATED : 0u) |
                             (f.gates ? B200Q_GDN_GATES : 0u) | (f.with_out >= 0 ? B200Q_GDN_WITH_OUT : 0u);
            push(i, {7u, hv | (hk << 16), q, k, o32(src(i, 2)), g, beta, y});
            push(i, {d.u[2], d.u[2], fbits(d.eps), flags, fbits(f.l2 ? f.l2_eps : 1e-6f),
                     fbits(f.gated ? f.rms_eps : 1e-6f), f.gated ? o32(f.w) : 0u, f.gated ? o32(f.z) : 0u});
            if (f.gates) push(i, {o32(f.dt), o32(f.a)});
            if (f.with_out >= 0) {
                if (!b200q_node_supported(nd, unsigned(f.with_out))) return fail(f.with_out, "not supported");
                emit_gemv_with_epilogue(f.with_out, i);
                done[size_t(f.with_out)] = 1;
            }
            break;
        }
        case B200Q_NODE_ROPE:
            push(i, {10u, d.u[0], o32(src(i, 0)), o32(src(i, 1)), o32(i), d.u[1], d.u[2]});
            break;
        case B200Q_NODE_ATTN:
            push(i, {12u, d.u[0] | (d.u[1] << 8) | ((d.u[2] / 16u) << 16), o32(src(i, 0)), o32(src(i, 1)),
                     o32(src(i, 2)), o32(i), o32(src(i, 3)), d.u[3]});
            break;
        case B200Q_NODE_GET_ROWS:
            push(i, {14u, d.fmt, d.cols, uint32_t(d.weight), uint32_t(d.weight >> 32), o32(src(i, 0)), o32(i)});
            break;
        case B200Q_NODE_ARGMAX:
            push(i, {13u, nd[src(i, 0)].n, o32(src(i, 0)), o32(i)});
            break;
        case B200Q_NODE_ALLREDUCE:
        case B200Q_NODE_ALLGATHER:
            push(i, {d.op == B200Q_NODE_ALLREDUCE ? 15u : 16u, nd[src(i, 0)].n, o32(src(i, 0)), o32(i)});
            break;
        default:
            return fail(i, "no command for this op");
        }
    }
    // pack segments into lists
    std::vector<uint32_t> cur;
    for (size_t s = 0; s < seg_cmds.size(); ++s) {
        const std::vector<uint32_t> &c = seg_cmds[s];
        if (c.empty()) continue;
        if (c.size() / 8 > kMaxListCmds) {
            char buf[96];
            snprintf(buf, sizeof(buf), "segment %zu has %zu commands (a list holds %u)", s, c.size() / 8, kMaxListCmds);
            err = buf;
            return false;
        }
        if ((cur.size() + c.size()) / 8 > kMaxListCmds) {
            lists.push_back(cur);
            cur.clear();
        }
        cur.insert(cur.end(), c.begin(), c.end());
        if (seg_list_end[s]) {
            lists.push_back(cur);
            cur.clear();
        }
    }
    if (!cur.empty()) lists.push_back(cur);
    return true;
}

}  // namespace

struct b200q_lowering {
    std::vector<std::vector<uint32_t>> lists;
    std::vector<size_t> off;
    size_t act = 0;
};

extern "C" {

int b200q_node_supported(const b200q_node *nodes, unsigned i) {
    if (!nodes) return 0;
    const b200q_node &d = nodes[i];
    const auto n_of = [&](int k) -> unsigned { return d.src[k] >= 0 && d.src[k] < int(i) ? nodes[d.src[k]].n : 0u; };
    const auto has = [&](int k) { return d.src[k] >= 0 && d.src[k] < int(i); };
    switch (d.op) {
    case B200Q_NODE_INPUT:
    case B200Q_NODE_PARAM:
    case B200Q_NODE_VIEW:
        return 1;
    case B200Q_NODE_MUL_MAT: {
        if (d.u[0] > 1)  // batched: GEMV_BATCH (Q8_0 family), y rows round16(rows) floats apart
            return (d.fmt == 2 || d.fmt == 3 || d.fmt == 8) && d.rows >= 1 && d.rows <= kMaxRows && d.cols >= 1 &&
                   d.cols <= kMaxCols && d.cols % 128 == 0 && d.u[0] <= 65536u &&
                   size_t(d.n) == size_t(d.u[0]) * round16(d.rows) && has(0) &&
                   size_t(n_of(0)) == size_t(d.u[0]) * d.cols;
        const bool kq = d.fmt == 13 || d.fmt == 14;
        return (d.fmt == 2 || d.fmt == 3 || d.fmt == 8 || kq) && d.rows >= 1 && d.rows <= kMaxRows && d.cols >= 1 &&
               d.cols <= kMaxCols && d.cols % (kq ? 256u : 128u) == 0 && d.n == d.rows && has(0) && n_of(0) == d.cols;
    }
    case B200Q_NODE_RMS_NORM:
    case B200Q_NODE_L2_NORM: {
        const unsigned rows = d.rows ? d.rows : 1u;
        if (!has(0) || d.n % rows) return 0;
        const unsigned row = d.n / rows;
        return row % 16 == 0 && rows <= kMaxNormRows && (row / 16) * rows <= kBufWords && n_of(0) == d.n;
    }
    case B200Q_NODE_MUL:
    case B200Q_NODE_ADD:
    case B200Q_NODE_SWIGLU:
        // a MUL whose second operand is one row (the weight of the norm before it) is checked by the lowering
        return has(0) && has(1) && d.n % 16 == 0 && d.n <= kBufWords * 16 && n_of(0) == d.n &&
               (n_of(1) == d.n || (d.op == B200Q_NODE_MUL && n_of(1) != 0 && d.n % n_of(1) == 0) ||
                (d.op == B200Q_NODE_MUL && n_of(0) != 0 && n_of(1) == d.n));
    case B200Q_NODE_UNARY:
        return has(0) && d.u[0] >= 1 && d.u[0] <= 4 && d.n % 16 == 0 && d.n <= kBufWords * 16 && n_of(0) == d.n;
    case B200Q_NODE_CONV:
        return has(0) && has(1) && has(2) && d.n % 16 == 0 && d.n <= kMaxConvChannels && n_of(0) == d.n &&
               n_of(1) == 4 * d.n && n_of(2) == 3 * d.n && d.u[0] <= 1;
    case B200Q_NODE_GDN: {
        const unsigned hv = d.u[0], hk = d.u[1];
        return hv >= 1 && hv <= kMaxHeads && hk >= 1 && hk <= hv && hv % hk == 0 && d.u[2] % kStateUnits == 0 &&
               d.n == hv * kHead && has(0) && has(1) && has(2) && has(3) && has(4) && n_of(0) == hk * kHead &&
               n_of(1) == hk * kHead && n_of(2) == hv * kHead && n_of(3) == hv && n_of(4) == hv;
    }
    case B200Q_NODE_ROPE: {
        const unsigned dims = d.u[0], row = d.u[1], rows = d.u[2];
        return has(0) && has(1) && dims >= 32 && dims % 32 == 0 && dims <= kMaxRopeDims && dims <= row &&
               row % 16 == 0 && rows >= 1 && (row / 16) * rows <= kBufWords && d.n == row * rows && n_of(0) == d.n &&
               n_of(1) >= dims;
    }
    case B200Q_NODE_ATTN: {
        const unsigned nh = d.u[0], nkv = d.u[1], hd = d.u[2];
        return has(0) && has(1) && has(2) && has(3) && nh >= 1 && nh < 256 && nkv >= 1 && nkv < 256 && nh % nkv == 0 &&
               nh / nkv <= 16 && hd >= 16 && hd % 16 == 0 && hd <= 512 && d.n == nh * hd && n_of(0) == nh * hd &&
               n_of(1) == nkv * hd && n_of(2) == nkv * hd;
    }
    case B200Q_NODE_GET_ROWS:
        return has(0) && (d.fmt == 2 || d.fmt == 8) && d.cols >= 32 && d.cols % 32 == 0 && d.cols <= kMaxCols &&
               d.n == d.cols;
    case B200Q_NODE_ARGMAX:
        return has(0) && d.n == 2;
    case B200Q_NODE_ALLREDUCE:
        return has(0) && d.n == n_of(0) && d.n % 16 == 0;
    case B200Q_NODE_ALLGATHER:
        return has(0) && n_of(0) % 16 == 0 && d.n % n_of(0) == 0 && d.n / n_of(0) <= b200q::kMaxRanks;
    default:
        return 0;
    }
}

int b200q_lower(const b200q_node *nodes, unsigned n_nodes, uint32_t features, b200q_lowering **out, char *err,
                unsigned err_len) {
    if (err && err_len) err[0] = '\0';
    if (!nodes || !out || n_nodes == 0) return B200Q_ERR_ARG;
    *out = nullptr;
    Lowering L;
    L.nd = nodes;
    L.n = n_nodes;
    L.feat = features;
    bool ok = L.validate();
    if (ok) {
        L.fuse();
        ok = L.place() && L.emit();
    }
    if (!ok) {
        if (err && err_len) snprintf(err, err_len, "%s", L.err.c_str());
        return B200Q_ERR_ARG;
    }
    b200q_lowering *r = new b200q_lowering;
    r->lists = std::move(L.lists);
    r->off = std::move(L.off);
    for (unsigned i = 0; i < n_nodes; ++i)  // views report their first float
        if (nodes[i].op == B200Q_NODE_VIEW && r->off[size_t(nodes[i].src[0])] != kNone)
            r->off[i] = r->off[size_t(nodes[i].src[0])] + nodes[i].u[0];
    r->act = L.act;
    *out = r;
    return 0;
}

void b200q_lowering_free(b200q_lowering *l) { delete l; }

unsigned b200q_lowering_lists(const b200q_lowering *l) { return l ? unsigned(l->lists.size()) : 0u; }

const uint32_t *b200q_lowering_list(const b200q_lowering *l, unsigned i, unsigned *n_cmds) {
    if (!l || i >= l->lists.size()) {
        if (n_cmds) *n_cmds = 0;
        return nullptr;
    }
    if (n_cmds) *n_cmds = unsigned(l->lists[i].size() / 8);
    return l->lists[i].data();
}

size_t b200q_lowering_offset(const b200q_lowering *l, unsigned node) {
    return l && node < l->off.size() ? l->off[node] : SIZE_MAX;
}

size_t b200q_lowering_act_floats(const b200q_lowering *l) { return l ? l->act : 0u; }

}  // extern "C"
