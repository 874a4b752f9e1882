// Host-side command-list planner: validates a list of the reference ISA and cuts it into passes, the units the
// device executes (one or a few kernel launches each). Pure C++ (no CUDA), so it runs and is tested without a GPU.
//
// The control flow mirrors the reference's on-chip command processor (fpga/src/gemvqc16.cpp:553-958, run_list):
// the same GEMV group collection (<= 4 GEMVs on one x, gemvqc16.cpp:646-733), SwiGLU pairing (:702-716), CONV/ADD
// epilogue attachment (:474-499), deferred RMSNORM (:737-757), GDN slots with WITH_GEMV / WITH_OUT (:801-904) and the
// same 1-based status of the first invalid command. On top of the reference's checks, every offset is checked
// against the device buffers (act, state, KV, weight table), so a list can never make a kernel read or write
// outside them.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <array>
#include <vector>

namespace b200q {

constexpr unsigned kMaxRows = 65536, kMaxCols = 16384, kPairRows = 16384, kAddRows = 16384;
constexpr unsigned kBatchRows = 65536;  // GEMV_BATCH: activation rows per command (the 16-bit batch field)
constexpr unsigned kBufWords = 4096, kMaxNormRows = 4096, kMaxConvChannels = 16384, kNxFloats = 16384;
constexpr unsigned kMaxHeads = 32, kStateUnits = 4, kHead = 128, kMaxBlockedRows = 512 * 20;
constexpr unsigned kMaxRopeDims = 128;
constexpr unsigned kMaxRanks = 8;  // ranks of a communicator (ALLREDUCE / ALLGATHER)
// TRACE log: a 16-float header word and up to 512 events of 64 bits (8 per 16-float word)
constexpr unsigned kTraceEntries = 512, kTraceFloats = 16 + kTraceEntries * 2;

// One weight matrix in the device arena, found by its handle (GEMV words 4/5).
struct WeightInfo {
    uint64_t handle = 0;
    unsigned format = 0, rows = 0, cols = 0;  // rows: full matrix rows
    unsigned row_begin = 0, row_end = 0;      // rows held on this rank (row sharding)
    uint64_t base_off = 0;                    // byte offset of the first tile in the arena
    unsigned rt = 1, ct = 1, kc = 1, n_rt = 0;  // tiling (layout.h)
    unsigned tile_bytes = 0, qs_part = 0, dm_part = 0;
};

struct Limits {
    size_t act_floats = SIZE_MAX;
    size_t state_rows = SIZE_MAX;
    size_t kv_bytes = SIZE_MAX;
    unsigned kv_ctx = 0;
    bool check_weights = false;                // planning without a context: no weight table
    const std::vector<WeightInfo> *weights = nullptr;
    // executor fusions that a feature mask can switch off (results are the same either way): deferred norms
    // computed in the consumers' prologue (off: stored at the RMSNORM command), runs of RMSNORM / ROPE in one launch,
    // the attention gate applied in the attention merge
    bool defer_norms = true, fuse_rowops = true, fuse_attn_gate = true;
    unsigned world = 1;                        // ranks of the communicator (ALLGATHER's output is n x world floats)
};

constexpr unsigned kMaxRowJobs = 8;  // jobs of one RowOps launch

enum class PassKind : uint32_t {
    Gemv = 1,       // GEMV group (1..4 members) with epilogues
    Elementwise,    // RMSNORM (stored), ADD, MUL, SILU_MUL, UNARY, CONV, ROPE
    Gdn,            // GDN step (+ WITH_GEMV GEMV, + WITH_OUT GEMV with ADD)
    Nop,            // STATE_LOAD, TRACE, deferred RMSNORM (no launch of its own)
    Ext,            // ATTN, ARGMAX, GET_ROW, ALLREDUCE, ALLGATHER
    RowOps,         // consecutive RMSNORM (stored) / ROPE commands run as one launch (reported as Elementwise)
};

enum Epi : uint32_t { EpiNone = 0, EpiSwigluG = 1, EpiSwigluU = 2, EpiConv = 3, EpiAdd = 4 };

struct Member {
    unsigned cmd = 0;            // command index of the GEMV
    unsigned format = 0, rows = 0, cols = 0, x_off = 0;
    uint64_t handle = 0;
    const WeightInfo *w = nullptr;
    unsigned y_off = 0;          // where the member's result goes (epilogue command's y for CONV/ADD)
    Epi epi = EpiNone;
    unsigned r_off = 0;          // ADD residual
    unsigned c_w = 0, c_src = 0, c_dst = 0, c_silu = 0;  // CONV epilogue
};

// Deferred RMSNORM kept for the GEMVs that read its y (reference gemvqc16.h:49-51).
struct DeferredNorm {
    bool valid = false;
    unsigned x_off = 0, w_off = 0, y_off = 0, n = 0, flags = 0;
    float eps = 0.0f;
    bool materialize = false;    // x or w changed before a consumer ran: the norm is stored to a private row
    unsigned cmd = 0;            // the RMSNORM command
};

struct Pass {
    PassKind kind = PassKind::Nop;
    unsigned first = 0, count = 1;  // commands consumed
    uint32_t op = 0;                // opcode of the first command
    uint32_t cmd[3][8] = {};        // raw words of up to three slots (GDN uses 2-3)
    // GEMV group
    unsigned x_off = 0, cols = 0, n_members = 0;
    Member m[4];
    bool from_nd = false;           // x is the deferred norm's row
    DeferredNorm nd;                // the norm the group reads (when from_nd)
    bool prequant = false;          // quantize x before any member writes (a member's y overlaps x)
    // GDN
    bool gdn_with_gemv = false, gdn_with_out = false;
    Member gdn_gemv;                // WITH_GEMV member
    Member gdn_out;                 // WITH_OUT member (epi None or Add)
    // deferred RMSNORM that must be stored now (materialize) — kind Nop with this set
    bool nd_store = false;
    // an input range that a kernel of this pass also writes: copied to scratch first
    bool snapshot = false;
    // RowOps: jobs of one launch, each an RMSNORM (stored) and/or the ROPE of its output (op word 0: absent)
    std::vector<std::array<uint32_t, 16>> rowjobs;
    // ATTN followed by SILU_MUL (sigmoid) of its output: the gate command, applied in the attention merge
    bool attn_gate = false;
    uint32_t gate[8] = {};
};

struct Plan {
    std::vector<Pass> passes;
    int status = 0;                 // 0, or 1-based index of the first invalid command, or 129
    bool has_trace = false;
    unsigned trace_off = 0;
    std::string error;              // reason of a rejection (diagnostics)
};

// Plans a list. The returned plan holds the passes of the valid prefix (they run before the status is returned).
Plan plan_list(const uint32_t *cmds, unsigned n_cmds, const Limits &lim);

// Activation type of a weight format: 0 Q8_0 (Q4_0, Q8_0), 1 Q8_1 (Q4_1), 2 Q8_K (Q5_K, Q6_K).
inline unsigned act_type(unsigned format) { return (format == 13 || format == 14) ? 2u : (format == 3 ? 1u : 0u); }
#if defined(__CUDACC__)
__host__ __device__
#endif
inline unsigned round16(unsigned n) { return (n + 15u) / 16u * 16u; }

}  // namespace b200q
