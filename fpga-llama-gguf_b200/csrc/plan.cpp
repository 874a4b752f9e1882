// Command-list planner (see plan.h). Mirrors the control flow of the reference command processor
// (fpga/src/gemvqc16.cpp:553-958) and adds range checks against the device buffers.
#include "plan.h"

#include <cstring>

namespace b200q {
namespace {

float bits_to_float(uint32_t b) {
    float f;
    std::memcpy(&f, &b, 4);
    return f;
}

const uint32_t kZero[8] = {0, 0, 0, 0, 0, 0, 0, 0};

struct Ctx {
    const uint32_t *cmds;
    unsigned n;
    const Limits &lim;
    Plan &plan;
    const uint32_t *at(unsigned i) const { return i < n ? cmds + size_t(i) * 8 : kZero; }
    bool act(size_t off, size_t len) const { return off <= lim.act_floats && len <= lim.act_floats - off; }
};

// gemv_valid of the reference (gemvqc16.cpp:455-466): opcode, one flag bit at most, rows/cols limits, cols a
// multiple of 128 (256 for K-quants), a known format, x and y 16-aligned.
bool gemv_valid(const uint32_t *c) {
    const unsigned fmt = c[1] & 0xffu, rows = c[2], cols = c[3], flags = c[1] & ~0xffu;
    const bool kq = fmt == 13 || fmt == 14;
    return c[0] == 1 && (flags & ~(0x100u | 0x200u | 0x400u)) == 0 && (flags & (flags - 1u)) == 0 && rows != 0 &&
           rows <= kMaxRows && cols != 0 && cols <= kMaxCols && cols % (kq ? 256u : 128u) == 0 &&
           (fmt == 2 || fmt == 3 || fmt == 8 || kq) && c[6] % 16 == 0 && c[7] % 16 == 0;
}

Member member_of(unsigned idx, const uint32_t *c) {
    Member m;
    m.cmd = idx;
    m.format = c[1] & 0xffu;
    m.rows = c[2];
    m.cols = c[3];
    m.x_off = c[6];
    m.handle = uint64_t(c[4]) | (uint64_t(c[5]) << 32);
    m.y_off = c[7];
    const unsigned fl = c[1] & ~0xffu;
    m.epi = (fl & 0x100u) ? EpiSwigluG : (fl & 0x200u) ? EpiConv : (fl & 0x400u) ? EpiAdd : EpiNone;
    return m;
}

// attach_conv (gemvqc16.cpp:488-499): the CONV behind a conv member takes all its rows as channels.
bool attach_conv(Member &m, const uint32_t *cv) {
    const bool ok = cv[0] == 8 && cv[1] == m.rows && cv[2] == m.y_off && cv[1] % 16 == 0 &&
                    cv[1] <= kMaxConvChannels && cv[3] % 16 == 0 && cv[4] % 16 == 0 && cv[5] % 16 == 0 &&
                    cv[6] % 16 == 0 && cv[7] <= 1u;
    m.c_w = cv[3];
    m.y_off = cv[4];
    m.c_src = cv[5];
    m.c_dst = cv[6];
    m.c_silu = cv[7] & 1u;
    return ok;
}

// attach_add (gemvqc16.cpp:476-485): one ADD operand is the member's output, the other the residual.
bool attach_add(Member &m, const uint32_t *ad) {
    const bool ok = ad[0] == 3 && ad[1] == m.rows && (ad[2] == m.y_off || ad[3] == m.y_off) && m.rows % 16 == 0 &&
                    m.rows <= kAddRows && ad[2] % 16 == 0 && ad[3] % 16 == 0 && ad[4] % 16 == 0;
    m.r_off = ad[2] == m.y_off ? ad[3] : ad[2];
    m.y_off = ad[4];
    return ok;
}

// overlaps_x (gemvqc16.cpp:468-474)
bool overlaps_x(const Member &m, unsigned x_off, unsigned cols) {
    const unsigned yr = round16(m.rows);
    return (m.y_off < x_off + cols && x_off < m.y_off + yr) ||
           (m.epi == EpiConv && m.c_dst < x_off + cols && x_off < m.c_dst + 3u * m.rows);
}

const WeightInfo *find_weight(const Limits &lim, uint64_t h) {
    if (!lim.weights) return nullptr;
    for (const WeightInfo &w : *lim.weights)
        if (w.handle == h) return &w;
    return nullptr;
}

// Buffer checks of one member (not in the reference, whose engines would read or write past the buffers).
bool member_ranges_ok(const Ctx &c, Member &m, unsigned x_off, bool allow_missing_weight) {
    if (!c.act(x_off, m.cols)) return false;
    if (c.lim.check_weights) {
        m.w = find_weight(c.lim, m.handle);
        if (!m.w || m.w->format != m.format || m.w->cols != m.cols || m.w->rows != m.rows) return false;
    } else if (!allow_missing_weight) {
        return false;
    }
    switch (m.epi) {
    case EpiSwigluG: return true;  // not written
    case EpiConv:
        return c.act(m.y_off, m.rows) && c.act(m.c_w, size_t(4) * m.rows) && c.act(m.c_src, size_t(3) * m.rows) &&
               c.act(m.c_dst, size_t(3) * m.rows);
    case EpiAdd: return c.act(m.y_off, m.rows) && c.act(m.r_off, m.rows);
    default: return c.act(m.y_off, round16(m.rows));
    }
}

bool ranges_meet(size_t a, size_t an, size_t b, size_t bn) { return a < b + bn && b < a + an; }

// Act ranges a pass writes (for the deferred-norm check).
void pass_writes(const Pass &p, std::vector<std::pair<size_t, size_t>> &w) {
    w.clear();
    const uint32_t *c = p.cmd[0];
    auto add_member = [&](const Member &m) {
        if (m.epi == EpiSwigluG) return;
        w.push_back({m.y_off, m.epi == EpiConv || m.epi == EpiAdd ? m.rows : round16(m.rows)});
        if (m.epi == EpiConv) w.push_back({m.c_dst, size_t(3) * m.rows});
    };
    switch (p.kind) {
    case PassKind::Gemv:
        for (unsigned i = 0; i < p.n_members; ++i) add_member(p.m[i]);
        break;
    case PassKind::Elementwise:
        if (p.op == 2) w.push_back({c[4], size_t(c[1]) * (c[6] ? c[6] : 1u)});
        else if (p.op == 8) { w.push_back({c[4], c[1]}); w.push_back({c[6], size_t(3) * c[1]}); }
        else if (p.op == 10) w.push_back({c[4], size_t(c[5]) * c[6]});
        else w.push_back({c[4], c[1]});
        break;
    case PassKind::Gdn:
        w.push_back({c[7], size_t(c[1] & 0xffffu) * kHead});
        if (p.gdn_with_gemv) add_member(p.gdn_gemv);
        if (p.gdn_with_out) add_member(p.gdn_out);
        break;
    case PassKind::Ext:
        if (p.op == 12) w.push_back({c[5], size_t(c[1] & 0xffu) * ((c[1] >> 16) * 16u)});
        else if (p.op == 13) w.push_back({c[3], 2});
        else if (p.op == 14) w.push_back({c[6], c[2]});
        else if (p.op == 15) w.push_back({c[3], c[1]});
        else if (p.op == 16) w.push_back({c[3], size_t(c[1]) * kMaxRanks});
        else if (p.op == 17) w.push_back({c[7], size_t((c[1] >> 16 & 0xffffu) + 1u) * round16(c[2])});
        break;
    default: break;
    }
}

}  // namespace

// ---- fusions of consecutive small passes (same results as running them one by one) --------------------------------
struct Span {
    size_t off, n;
};
bool spans_meet(const Span &a, const Span &b) { return a.n && b.n && ranges_meet(a.off, a.n, b.off, b.n); }

// Reads and writes (act floats) of a stored RMSNORM / a ROPE command.
void norm_spans(const uint32_t *c, std::vector<Span> &rd, std::vector<Span> &wr) {
    const unsigned n = c[1], rows = c[6] ? c[6] : 1u, stride = (c[7] >> 8) & 0xffffu;
    rd.push_back({c[2], stride ? size_t(rows - 1) * stride * 16 + n : size_t(rows) * n});
    if ((c[7] & 2u) == 0) rd.push_back({c[3], n});
    wr.push_back({c[4], size_t(rows) * n});
}
void rope_spans(const uint32_t *c, std::vector<Span> &rd, std::vector<Span> &wr) {
    rd.push_back({c[2], size_t(c[5]) * c[6]});
    rd.push_back({c[3], c[1]});
    wr.push_back({c[4], size_t(c[5]) * c[6]});
}
bool is_rowop(const Pass &p) {
    return p.kind == PassKind::Elementwise && (p.op == 10 || (p.op == 2 && (p.cmd[0][7] & 4u) == 0));
}

// Runs of RMSNORM / ROPE passes become one RowOps pass: a ROPE whose x is exactly the rows an earlier RMSNORM of the
// run stored joins that norm's job; all jobs must be independent (no job writes what another reads or writes).
void fuse_rowops(std::vector<Pass> &passes) {
    std::vector<Pass> out;
    size_t i = 0;
    while (i < passes.size()) {
        if (!is_rowop(passes[i])) {
            out.push_back(passes[i++]);
            continue;
        }
        std::vector<std::array<uint32_t, 16>> jobs;
        std::vector<std::vector<Span>> jrd, jwr;
        size_t j = i;
        for (; j < passes.size() && is_rowop(passes[j]); ++j) {
            const uint32_t *c = passes[j].cmd[0];
            std::vector<Span> rd, wr;
            int link = -1;
            if (passes[j].op == 10) {
                rope_spans(c, rd, wr);
                for (size_t k = 0; k < jobs.size(); ++k) {
                    const uint32_t *nc = jobs[k].data();
                    if (nc[0] == 2 && jobs[k][8] == 0 && nc[4] == c[2] && (nc[6] ? nc[6] : 1u) == c[6] &&
                        nc[1] == c[5])
                        link = int(k);
                }
            } else {
                norm_spans(c, rd, wr);
            }
            // independence from the other jobs (the linked norm's stored rows are this ROPE's own input)
            bool ok = true;
            for (size_t k = 0; k < jobs.size() && ok; ++k) {
                for (const Span &w : wr) {
                    for (const Span &r : jrd[k]) ok = ok && !spans_meet(w, r);
                    for (const Span &x : jwr[k]) ok = ok && !spans_meet(w, x);
                }
                for (const Span &r : rd)
                    for (const Span &x : jwr[k])
                        if (!(int(k) == link && r.off == x.off && r.n == x.n)) ok = ok && !spans_meet(r, x);
            }
            if (link >= 0) {  // within the job: the ROPE writes nothing the norm reads
                for (const Span &w : wr)
                    for (const Span &r : jrd[size_t(link)]) ok = ok && !spans_meet(w, r);
            }
            if (link < 0 && jobs.size() == kMaxRowJobs) ok = false;  // one launch holds at most kMaxRowJobs jobs
            if (!ok) break;
            if (link >= 0) {
                std::memcpy(jobs[size_t(link)].data() + 8, c, 32);
                for (const Span &r : rd) jrd[size_t(link)].push_back(r);
                for (const Span &w : wr) jwr[size_t(link)].push_back(w);
            } else {
                std::array<uint32_t, 16> jb{};
                std::memcpy(jb.data() + (passes[j].op == 10 ? 8 : 0), c, 32);
                jobs.push_back(jb);
                jrd.push_back(rd);
                jwr.push_back(wr);
            }
        }
        if (j - i < 2) {
            out.push_back(passes[i++]);
            continue;
        }
        Pass f = passes[i];
        f.kind = PassKind::RowOps;
        f.count = passes[j - 1].first + passes[j - 1].count - passes[i].first;
        f.rowjobs = jobs;
        out.push_back(f);
        i = j;
    }
    passes.swap(out);
}

// ATTN followed by a sigmoid SILU_MUL of its output (the gated attention output): the gate is applied in the
// attention merge. Its g rows must not meet the attention output or the gated output; the gated output is the
// attention output itself or apart from it.
void fuse_attn_gate(std::vector<Pass> &passes) {
    std::vector<Pass> out;
    for (size_t i = 0; i < passes.size(); ++i) {
        Pass p = passes[i];
        if (p.kind == PassKind::Ext && p.op == 12 && i + 1 < passes.size() &&
            passes[i + 1].kind == PassKind::Elementwise && passes[i + 1].op == 4) {
            const uint32_t *a = p.cmd[0], *g = passes[i + 1].cmd[0];
            const unsigned nh = a[1] & 0xffu, hd = (a[1] >> 16) * 16u, n = g[1], row = g[6], stride = g[7];
            const Span ya{a[5], size_t(nh) * hd}, yg{g[4], n};
            const Span gs{g[2], row ? size_t(n / row - 1) * stride + row : n};
            const bool ok = (g[5] & 1u) && g[3] == a[5] && n == nh * hd && !spans_meet(gs, ya) && !spans_meet(gs, yg) &&
                            (yg.off == ya.off || !spans_meet(yg, ya));
            if (ok) {
                p.attn_gate = true;
                std::memcpy(p.gate, g, 32);
                p.count += passes[i + 1].count;
                out.push_back(p);
                ++i;
                continue;
            }
        }
        out.push_back(p);
    }
    passes.swap(out);
}

Plan plan_list(const uint32_t *cmds, unsigned n_cmds, const Limits &lim) {
    Plan plan;
    if (n_cmds > 128) {
        plan.status = 129;
        plan.error = "more than 128 commands";
        return plan;
    }
    Ctx C{cmds, n_cmds, lim, plan};
    DeferredNorm nd;
    int nd_pass = -1;          // index of the deferred RMSNORM's Nop pass
    bool nd_dirty = false;     // a pass after the deferred RMSNORM wrote its x or weight
    std::vector<std::pair<size_t, size_t>> writes;
    unsigned c = 0;
    auto reject = [&](unsigned idx, const char *why) {
        plan.status = int(idx) + 1;
        plan.error = std::string("command ") + std::to_string(idx) + ": " + why;
    };
    while (c < n_cmds && plan.status == 0) {
        const uint32_t *cmd = C.at(c);
        const uint32_t op = cmd[0];
        Pass p;
        p.first = c;
        p.op = op;
        std::memcpy(p.cmd[0], cmd, 32);
        unsigned advance = 1;
        if (op == 1) {
            // ---- GEMV group (gemvqc16.cpp:646-733)
            const unsigned cols = cmd[3], x_off = cmd[6];
            Member mem[4];
            unsigned end[4];
            mem[0] = member_of(c, cmd);
            unsigned next_at = c + 1;
            bool bad_epilog = false;
            if (mem[0].epi == EpiConv) {
                bad_epilog = !attach_conv(mem[0], C.at(next_at));
                ++next_at;
            } else if (mem[0].epi == EpiAdd) {
                bad_epilog = !attach_add(mem[0], C.at(next_at));
                ++next_at;
            }
            end[0] = next_at;
            unsigned nm = 1;
            bool open = !bad_epilog && !overlaps_x(mem[0], x_off, cols);
            for (unsigned k = 1; k < 4; ++k) {
                if (!open || next_at >= n_cmds) break;
                const uint32_t *nx = C.at(next_at);
                if (!gemv_valid(nx) || nx[3] != cols || nx[6] != x_off || act_type(nx[1] & 0xffu) != act_type(mem[0].format))
                    break;
                Member m = member_of(next_at, nx);
                if (m.epi == EpiAdd) break;  // an add member starts its own group
                unsigned after = next_at + 1;
                if (m.epi == EpiConv) {
                    if (next_at + 1 >= n_cmds) break;
                    if (!attach_conv(m, C.at(next_at + 1))) break;
                    after = next_at + 2;
                }
                // range checks of a later member: a failing member starts the next group (and is rejected there)
                if (!member_ranges_ok(C, m, x_off, true)) break;
                next_at = after;
                mem[k] = m;
                end[k] = next_at;
                nm = k + 1;
                open = !overlaps_x(m, x_off, cols);
            }
            // SwiGLU pairing (gemvqc16.cpp:702-716)
            bool bad_pair = false;
            unsigned i = 0;
            while (i < nm) {
                if (mem[i].epi != EpiSwigluG) {
                    ++i;
                } else if (i + 1 < nm && mem[i + 1].rows == mem[i].rows && mem[i + 1].epi == EpiNone &&
                           mem[i].rows <= kPairRows) {
                    mem[i + 1].epi = EpiSwigluU;
                    i += 2;
                } else {
                    bad_pair = i == 0;
                    nm = i;
                }
            }
            if (!gemv_valid(cmd)) { reject(c, "invalid GEMV"); break; }
            if (bad_epilog) { reject(c, "invalid CONV/ADD epilogue"); break; }
            if (bad_pair) { reject(c, "SwiGLU g without its u"); break; }
            if (!member_ranges_ok(C, mem[0], x_off, !lim.check_weights)) { reject(c, "GEMV outside the buffers or unknown weight"); break; }
            p.kind = PassKind::Gemv;
            p.x_off = x_off;
            p.cols = cols;
            p.n_members = nm;
            for (unsigned k = 0; k < nm; ++k) p.m[k] = mem[k];
            advance = end[nm - 1] - c;
            if (nd.valid && x_off == nd.y_off && cols == nd.n) {
                p.from_nd = true;
                p.nd = nd;
            }
            for (unsigned k = 0; k < nm; ++k)
                if (overlaps_x(mem[k], x_off, cols)) p.prequant = true;
        } else if (op == 2) {
            // ---- RMSNORM (gemvqc16.cpp:737-757)
            const unsigned nn = cmd[1], xo = cmd[2], wo = cmd[3], yo = cmd[4], flags = cmd[7];
            const unsigned rows = cmd[6] == 0 ? 1u : cmd[6];
            const bool defer = (flags & 4u) != 0;
            const unsigned stride = (flags >> 8) & 0xffffu;
            if (nn == 0 || nn % 16 || rows > kMaxNormRows || (nn / 16) * rows > kBufWords || xo % 16 || wo % 16 ||
                yo % 16 || (flags & 0xff0000f8u) || (stride != 0 && stride < nn / 16) ||
                (defer && (rows != 1 || nn > kNxFloats))) {
                reject(c, "invalid RMSNORM");
                break;
            }
            const size_t span = stride ? size_t(rows - 1) * stride * 16 + nn : size_t(rows) * nn;
            if (!C.act(xo, span) || ((flags & 2u) == 0 && !C.act(wo, nn)) || !C.act(yo, size_t(rows) * nn)) {
                reject(c, "RMSNORM outside act");
                break;
            }
            if (defer) {
                p.kind = PassKind::Nop;
                nd = DeferredNorm{};
                nd.valid = true;
                nd.x_off = xo;
                nd.w_off = wo;
                nd.y_off = yo;
                nd.n = nn;
                nd.flags = flags & 3u;
                nd.eps = bits_to_float(cmd[5]);
                nd.cmd = c;
                nd_pass = int(plan.passes.size());
                nd_dirty = false;
            } else {
                p.kind = PassKind::Elementwise;
            }
        } else if (op == 3 || op == 4 || op == 5 || op == 6) {
            // ---- ADD / SILU_MUL / MUL / UNARY (gemvqc16.cpp:758-773)
            const unsigned nn = cmd[1], a = cmd[2], b = cmd[3], yo = cmd[4];
            const bool unary = op == 6, sm = op == 4;
            const unsigned row = unary ? cmd[5] : (sm ? cmd[6] : 0u), stride = unary ? cmd[6] : cmd[7];
            if (nn == 0 || nn > kBufWords * 16 || nn % 16 || a % 16 || yo % 16 ||
                (unary ? (b == 0 || b > 4) : (b % 16 != 0)) || (sm && (cmd[5] & ~1u)) ||
                (row != 0 && (row % 16 || nn % row || stride % 16 || stride < row))) {
                reject(c, "invalid element-wise command");
                break;
            }
            const size_t span = row ? size_t(nn / row - 1) * stride + row : nn;
            if (!C.act(a, span) || (!unary && !C.act(b, nn)) || !C.act(yo, nn)) {
                reject(c, "element-wise command outside act");
                break;
            }
            p.kind = PassKind::Elementwise;
        } else if (op == 10) {
            // ---- ROPE (gemvqc16.cpp:774-782)
            const unsigned nd_ = cmd[1], xo = cmd[2], cs = cmd[3], yo = cmd[4], ne0 = cmd[5], rows = cmd[6];
            if (nd_ == 0 || nd_ % 32 || nd_ > kMaxRopeDims || nd_ > ne0 || ne0 % 16 || rows == 0 ||
                (ne0 / 16) * rows > kBufWords || xo % 16 || cs % 16 || yo % 16 || cmd[7] != 0) {
                reject(c, "invalid ROPE");
                break;
            }
            if (!C.act(xo, size_t(ne0) * rows) || !C.act(cs, nd_) || !C.act(yo, size_t(ne0) * rows)) {
                reject(c, "ROPE outside act");
                break;
            }
            p.kind = PassKind::Elementwise;
        } else if (op == 11) {
            // ---- TRACE (gemvqc16.cpp:783-790)
            if (cmd[1] % 16 || (cmd[2] | cmd[3] | cmd[4] | cmd[5] | cmd[6] | cmd[7]) != 0) {
                reject(c, "invalid TRACE");
                break;
            }
            if (!C.act(cmd[1], kTraceFloats)) {
                reject(c, "TRACE log outside act");
                break;
            }
            plan.has_trace = true;
            plan.trace_off = cmd[1];
            p.kind = PassKind::Nop;
        } else if (op == 8) {
            // ---- CONV (gemvqc16.cpp:791-800)
            const unsigned ch = cmd[1];
            if (ch == 0 || ch > kMaxConvChannels || ch % 16 || cmd[2] % 16 || cmd[3] % 16 || cmd[4] % 16 ||
                cmd[5] % 16 || cmd[6] % 16 || cmd[7] > 1u) {
                reject(c, "invalid CONV");
                break;
            }
            if (!C.act(cmd[2], ch) || !C.act(cmd[3], size_t(4) * ch) || !C.act(cmd[4], ch) ||
                !C.act(cmd[5], size_t(3) * ch) || !C.act(cmd[6], size_t(3) * ch)) {
                reject(c, "CONV outside act");
                break;
            }
            p.kind = PassKind::Elementwise;
        } else if (op == 7) {
            // ---- GDN (gemvqc16.cpp:801-904)
            const unsigned hv = cmd[1] & 0xffffu, hk = cmd[1] >> 16;
            const uint32_t *ext = C.at(c + 1);
            const bool gates = (ext[3] & 8u) != 0;
            const unsigned slots = gates ? 3u : 2u;
            const uint32_t *ext2 = C.at(c + 2);
            if (c + slots > n_cmds || hv == 0 || hv > kMaxHeads || hk == 0 || hk > hv || hv % hk || cmd[2] % 16 ||
                cmd[3] % 16 || cmd[4] % 16 || cmd[5] % 16 || cmd[6] % 16 || cmd[7] % 16 || ext[0] % kStateUnits ||
                ext[1] % kStateUnits || ext[3] > 31u || ((ext[3] & 4u) && (ext[6] % 16 || ext[7] % 16)) ||
                (gates && (ext2[0] % 16 || ext2[1] % 16))) {
                reject(c, "invalid GDN");
                break;
            }
            const unsigned S = kHead, rows = hv * S;
            const unsigned fl = ext[3];
            bool ok = size_t(ext[0]) + rows <= lim.state_rows && size_t(ext[1]) + rows <= lim.state_rows &&
                      C.act(cmd[2], size_t(hk) * S) && C.act(cmd[3], size_t(hk) * S) && C.act(cmd[4], rows) &&
                      C.act(cmd[5], hv) && C.act(cmd[6], hv) && C.act(cmd[7], rows);
            if (fl & 4u) ok = ok && C.act(ext[6], S) && C.act(ext[7], rows);
            if (gates) ok = ok && C.act(ext2[0], hv) && C.act(ext2[1], hv);
            // partly overlapping state rows (neither equal nor disjoint) would make one head's rows clobber another's
            if (ext[0] != ext[1] && ranges_meet(ext[0], rows, ext[1], rows)) ok = false;
            if (!ok) {
                reject(c, "GDN outside act/state");
                break;
            }
            p.kind = PassKind::Gdn;
            std::memcpy(p.cmd[1], ext, 32);
            if (gates) std::memcpy(p.cmd[2], ext2, 32);
            advance = slots;
            const unsigned step_y = cmd[7];
            if ((fl & 1u) && c + slots < n_cmds) {
                const uint32_t *nx = C.at(c + slots);
                Member m = member_of(c + slots, nx);
                const unsigned yr = round16(m.rows);
                if (gemv_valid(nx) && m.epi == EpiNone && !(nx[6] < step_y + rows && step_y < nx[6] + nx[3]) &&
                    !(m.y_off < step_y + rows && step_y < m.y_off + yr) && member_ranges_ok(C, m, nx[6], !lim.check_weights)) {
                    p.gdn_with_gemv = true;
                    p.gdn_gemv = m;
                    advance = slots + 1;
                }
            }
            if (fl & 16u) {
                const uint32_t *nx = C.at(c + slots), *ad = C.at(c + slots + 1);
                Member m = member_of(c + slots, nx);
                bool wok = (fl & 1u) == 0 && gemv_valid(nx) && m.epi != EpiSwigluG && m.epi != EpiConv &&
                           nx[6] == step_y && nx[3] == rows && rows % 256 == 0 && m.rows <= kMaxBlockedRows &&
                           c + slots < n_cmds;
                if (wok && m.epi == EpiAdd) {
                    wok = c + slots + 1 < n_cmds && attach_add(m, ad) &&
                          !(m.r_off < step_y + rows && step_y < m.r_off + m.rows);
                }
                if (wok) wok = member_ranges_ok(C, m, step_y, !lim.check_weights);
                if (!wok) {
                    reject(c, "invalid GDN_WITH_OUT GEMV");
                    break;
                }
                p.gdn_with_out = true;
                p.gdn_out = m;
                advance = slots + (m.epi == EpiAdd ? 2u : 1u);
            }
        } else if (op == 9) {
            // ---- STATE_LOAD (gemvqc16.cpp:905-913): a prefetch hint; the step reads its state itself
            if (cmd[1] == 0 || cmd[1] > kMaxHeads || cmd[2] % kStateUnits) {
                reject(c, "invalid STATE_LOAD");
                break;
            }
            p.kind = PassKind::Nop;
        } else if (op == 12) {
            // ---- ATTN extension
            const unsigned nh = cmd[1] & 0xffu, nkv = (cmd[1] >> 8) & 0xffu, hd = (cmd[1] >> 16) * 16u;
            const unsigned slot = cmd[7];
            const size_t slot_bytes = size_t(nkv) * lim.kv_ctx * hd * 2 * 2;
            if (nh == 0 || nkv == 0 || nh % nkv || nh / nkv > 16 || hd == 0 || hd > 512 || cmd[2] % 16 || cmd[3] % 16 || cmd[4] % 16 ||
                cmd[5] % 16 || cmd[6] % 16 || lim.kv_ctx == 0 || !C.act(cmd[6], 1) ||
                !C.act(cmd[2], size_t(nh) * hd) || !C.act(cmd[3], size_t(nkv) * hd) ||
                !C.act(cmd[4], size_t(nkv) * hd) || !C.act(cmd[5], size_t(nh) * hd) ||
                (size_t(slot) + 1) * slot_bytes > lim.kv_bytes) {
                reject(c, "invalid ATTN");
                break;
            }
            p.kind = PassKind::Ext;
        } else if (op == 13) {
            // ---- ARGMAX extension
            if (cmd[1] == 0 || cmd[2] % 16 || cmd[3] % 16 || (cmd[4] | cmd[5] | cmd[6] | cmd[7]) ||
                !C.act(cmd[2], cmd[1]) || !C.act(cmd[3], 16)) {
                reject(c, "invalid ARGMAX");
                break;
            }
            p.kind = PassKind::Ext;
        } else if (op == 14) {
            // ---- GET_ROW extension
            const unsigned fmt = cmd[1], cols = cmd[2];
            const uint64_t h = uint64_t(cmd[3]) | (uint64_t(cmd[4]) << 32);
            bool ok = (fmt == 2 || fmt == 8) && cols != 0 && cols % 32 == 0 && cols <= kMaxCols && cmd[5] % 16 == 0 &&
                      cmd[6] % 16 == 0 && cmd[7] == 0 && C.act(cmd[5], 1) && C.act(cmd[6], cols);
            if (ok && lim.check_weights) {
                const WeightInfo *w = find_weight(lim, h);
                ok = w && w->format == fmt && w->cols == cols;
            }
            if (!ok) {
                reject(c, "invalid GET_ROW");
                break;
            }
            p.kind = PassKind::Ext;
        } else if (op == 15 || op == 16) {
            // ---- ALLREDUCE / ALLGATHER extensions: y = sum of the ranks' x / y = the ranks' x side by side
            const size_t n = cmd[1], yn = op == 15 ? n : n * lim.world;
            const size_t x = cmd[2], y = cmd[3];
            bool ok = n != 0 && n % 16 == 0 && x % 16 == 0 && y % 16 == 0 && (cmd[4] | cmd[5] | cmd[6] | cmd[7]) == 0 &&
                      C.act(x, n) && C.act(y, yn);
            if (ok && op == 15) ok = x == y || !ranges_meet(x, n, y, n);
            if (ok && op == 16) ok = !ranges_meet(x, n, y, yn) || (x >= y && (x - y) % n == 0 && x + n <= y + yn);
            if (!ok) {
                reject(c, op == 15 ? "invalid ALLREDUCE" : "invalid ALLGATHER");
                break;
            }
            p.kind = PassKind::Ext;
        } else if (op == 17) {
            // ---- GEMV_BATCH extension: y_m = W x_m (+ y_m) for m < batch, x rows cols apart, y rows round16(rows)
            const unsigned fmt = cmd[1] & 0xffu, fl = cmd[1] & 0xff00u, batch = ((cmd[1] >> 16) & 0xffffu) + 1u;
            const unsigned rows = cmd[2], cols = cmd[3];
            const uint64_t h = uint64_t(cmd[4]) | (uint64_t(cmd[5]) << 32);
            const size_t xs = size_t(batch) * cols, ys = size_t(batch) * round16(rows);
            bool ok = (fmt == 2 || fmt == 3 || fmt == 8) && (fl == 0 || fl == 0x400u) && batch <= kBatchRows &&
                      rows != 0 && rows <= kMaxRows && cols != 0 && cols <= kMaxCols &&
                      cols % 128 == 0 && cmd[6] % 16 == 0 && cmd[7] % 16 == 0 && C.act(cmd[6], xs) &&
                      C.act(cmd[7], ys) && !ranges_meet(cmd[6], xs, cmd[7], ys);
            if (ok && lim.check_weights) {
                const WeightInfo *w = find_weight(lim, h);
                ok = w && w->format == fmt && w->cols == cols && w->rows == rows;
            }
            if (!ok) {
                reject(c, "invalid GEMV_BATCH");
                break;
            }
            p.kind = PassKind::Ext;
        } else {
            reject(c, "unknown opcode");
            break;
        }
        p.count = advance;
        // A consumer of the deferred norm computes it from x and the weight as they are when it runs. When x or the
        // weight changes between the RMSNORM and a consumer (a write by an earlier pass, or by the consumer itself,
        // whose CTAs write while others still read), the norm is stored at its command and consumers read that row.
        // Writes after the last consumer cost nothing.
        if (nd.valid && nd_pass >= 0 && p.kind != PassKind::Nop) {
            pass_writes(p, writes);
            bool hits = false;
            for (const auto &w : writes)
                hits = hits || ranges_meet(w.first, w.second, nd.x_off, nd.n) ||
                       ((nd.flags & 2u) == 0 && ranges_meet(w.first, w.second, nd.w_off, nd.n));
            if (p.kind == PassKind::Gemv && p.from_nd && (nd_dirty || hits || !lim.defer_norms)) {
                nd.materialize = true;
                plan.passes[size_t(nd_pass)].nd_store = true;
                plan.passes[size_t(nd_pass)].nd = nd;
            }
            nd_dirty = nd_dirty || hits;
        }
        if (p.kind == PassKind::Nop && op == 2) p.nd = nd;
        plan.passes.push_back(p);
        c += advance;
    }
    // consumers of a stored deferred norm read the stored row
    for (Pass &p : plan.passes) {
        if (p.kind == PassKind::Gemv && p.from_nd) {
            for (const Pass &q : plan.passes)
                if (q.kind == PassKind::Nop && q.op == 2 && q.nd.cmd == p.nd.cmd && q.nd_store) p.nd.materialize = true;
        }
    }
    if (lim.fuse_rowops) fuse_rowops(plan.passes);
    if (lim.fuse_attn_gate) fuse_attn_gate(plan.passes);
    return plan;
}

}  // namespace b200q
