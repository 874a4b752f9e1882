// Launch argument blocks shared by the host executor (api.cpp) and the kernels. Plain structs of device pointers
// and sizes, passed by value as kernel parameters.
#pragma once
#include <cstdint>
#include <vector_types.h>

namespace b200q {

// One weight matrix in the device arena: the tiled layout of layout.h (tile (t, k) = R rows x C blocks, one
// contiguous run of tile_bytes: quants, then scales, then the K-quant d/dmin part).
struct MatrixView {
    const uint8_t *base = nullptr;
    unsigned format = 0;
    unsigned rows = 0;            // rows held here (the local row slice)
    unsigned row0 = 0;            // global index of the first local row
    unsigned rt = 1, ct = 1, kc = 1, n_rt = 0;
    unsigned tile_bytes = 0, qs_part = 0, dm_part = 0;
};

struct GemvMemberArgs {
    MatrixView w;
    float *y = nullptr;           // act + y_off (the member's output, global row indexing)
    unsigned epi = 0;             // Epi (plan.h)
    unsigned total_rows = 0;      // rows of the full matrix (zero padding of y up to a multiple of 16)
    const float *res = nullptr;   // ADD residual (global row indexing)
    const float *cw = nullptr;    // CONV kernel [4 x channels]
    const float *cs = nullptr;    // CONV state in [3 x channels]
    float *cd = nullptr;          // CONV state out
    unsigned csilu = 0;
};

// Row-sharded multi-GPU passes without a collective: every rank stores its output rows into its own act and, over
// NVLink, into the same offsets of every peer's act (IPC-mapped). Each sharded launch of a list has a sync slot. Per
// slot and rank, a rank counts its own launches of the slot (`mine`, raised by the launch's last CTA); a launch k of
// the slot announces in every peer that it has reached the slot (ready = k: its earlier work, which read those rows,
// is complete) and raises its data word to k once all its rows are in every peer. Words only grow, so nothing is
// cleared between lists; all ranks run the same launches in the same order.
constexpr unsigned kMaxPeers = 8;
constexpr unsigned kSyncSlots = 512;
__host__ __device__ inline unsigned ready_word(unsigned slot, unsigned rank) { return slot * kMaxPeers + rank; }
__host__ __device__ inline unsigned data_word(unsigned slot, unsigned rank) {
    return kSyncSlots * kMaxPeers + slot * kMaxPeers + rank;
}
constexpr unsigned kSyncCountWord = 2 * kSyncSlots * kMaxPeers;    // [slot] CTAs of the running launch
constexpr unsigned kSyncMineWord = kSyncCountWord + kSyncSlots;    // [slot] launches of the slot completed here
constexpr unsigned kSyncWords = kSyncMineWord + kSyncSlots;

struct PeerSync {
    float *act = nullptr;              // this rank's act (offsets of peer stores are taken against it)
    float *peer_act[kMaxPeers] = {};   // peers' act; null for this rank
    unsigned *peer_sync[kMaxPeers] = {};  // peers' sync words (IPC-mapped)
    unsigned *sync = nullptr;          // this rank's sync words
    unsigned world = 1, rank = 0, slot = 0;
};

// A kernel that reads rows of sharded launches first waits for the peers' data words of slots [slot0, slot0 + n)
// (n = 0: nothing to wait for).
struct PeerWait {
    const unsigned *sync = nullptr;
    unsigned slot0 = 0, n = 0, world = 1, rank = 0;
    unsigned *err = nullptr;
};

// ALLREDUCE of explicit lists over NVLink peer memory (coll.cu): one slot per ALLREDUCE of a list; per slot and rank
// a receive buffer [2 parities][world][kCollMaxN] 8-byte words {value, launch number}, and per slot this rank's launch
// counters, one per CTA (a CTA per chunk of kCollChunk values).
constexpr unsigned kCollMaxN = 4096, kCollChunk = 512, kCollMaxCtas = kCollMaxN / kCollChunk, kCollSlots = 64;
struct CollArgs {
    const float *x = nullptr;
    float *y = nullptr;
    unsigned n = 0;                      // floats, a multiple of 16, at most kCollMaxN
    uint2 *recv[kMaxPeers] = {};         // per rank: that rank's receive buffer of the slot (this rank's own included)
    unsigned *flag_local = nullptr;      // this rank's launch counters of the slot, one per CTA
    unsigned world = 1, rank = 0;
    unsigned *err = nullptr;             // set when a bounded wait runs out
};

constexpr unsigned kMaxUnits = 4;
// bytes of a quantized x image of up to 16384 values (quants + meta words)
constexpr unsigned kQImageBytes = 16384 + 16384 / 32 * 16;
constexpr unsigned kMaxNsqPanels = 4096;  // per-panel partial sums of squares a pass hands to the next

struct GemvArgs {
    const float *x = nullptr;     // act + x_off (or the deferred norm's x)
    unsigned cols = 0;
    // fused deferred RMSNORM (norm_mode bit 3 set: active; bits 0..1 the RMSNORM flags L2 / no weight)
    const float *norm_w = nullptr;
    float norm_eps = 0.0f;
    unsigned norm_mode = 0;
    // quantized x prepared by a separate launch (when a member's y overlaps x); null: quantize in the prologue
    const int8_t *xq = nullptr;
    const float *xd = nullptr;    // per 32-block scale (Q8_0: FP16 value as float; Q8_1: d) / per 256 (Q8_K)
    const float *xs = nullptr;    // Q8_1: FP16 s as float
    const int32_t *xb = nullptr;  // per-block sums of q (Q8_0/Q8_1) / per 16 (Q8_K)
    GemvMemberArgs m[4];
    unsigned n_members = 0;
    // work units: a member alone, or a SwiGLU pair (g = unit_member, u = unit_pair); a work item is one row tile
    // of a unit, streamed as the unit's kc tiles (pairs: the g and u tiles of the same rows in one stage)
    unsigned n_units = 0;
    unsigned unit_member[kMaxUnits] = {};
    int unit_pair[kMaxUnits] = {-1, -1, -1, -1};
    unsigned item_start[kMaxUnits + 1] = {};   // prefix sums of the units' row tiles
    // shared-memory plan (host-computed): stages of stage_bytes, per-stage compute results, x image
    unsigned n_stages = 0, stage_bytes = 0, res_bytes = 0;
    unsigned wraw = 0;            // the norm weight is staged in shared memory next to x
    unsigned *err = nullptr;      // set when a bounded wait runs out
    int32_t *dbg = nullptr;       // debug: per-block integer sums of member 0 (no y written)
    // Q8_0-family pass: bytes of one matrix's block terms of a panel in shared memory (steps x 32 floats)
    unsigned term_bytes = 0;
    // quantized x images in the GEMV shared-memory layout ([quants: two runs of 16-byte halves][one 16-byte meta
    // word per 32-block]): qin, this pass's x (written by the previous pass); qout, the image of member
    // qout_member's y for the next pass (32-row panels: one block per panel)
    const uint8_t *qin = nullptr;
    uint8_t *qout = nullptr;
    unsigned qout_member = 0;
    unsigned qout_act = 0;        // 0 Q8_0, 1 Q8_1 (the next pass's activation type)
    // the deferred norm's sum of squares from the pass that wrote x: nsq_in holds one FP64 partial per panel of that
    // pass (nsq_n of them), read instead of the whole x; nsq_out: this pass writes those partials for member
    // nsq_member's y (its squares summed per panel)
    const double *nsq_in = nullptr;
    unsigned nsq_n = 0;
    double *nsq_out = nullptr;
    unsigned nsq_member = 0;
    PeerSync ps;                  // world > 1: sharded members' rows also go to the peers
    PeerWait pw;                  // rows of earlier sharded launches this pass reads
};

// A run of consecutive Q4_0 / Q8_0 GEMV passes executed by one persistent kernel (gemv_q8.cu, gemv_chain_kernel):
// each pass a single matrix or a SwiGLU pair, its output a plain or residual-ADD row writer, its x from act (quantized
// in the kernel), a deferred RMSNORM of act, or the quantized image the previous pass of the chain wrote.
constexpr unsigned kMaxChainPasses = 16;
struct ChainPass {
    MatrixView wa, wb;            // wa: the matrix (a pair's g); wb: a pair's u (base null otherwise)
    GemvMemberArgs out;           // the output member (a pair: the u member, epilogue SwiGLU)
    unsigned fmt = 0;             // 2 Q4_0 or 8 Q8_0 (a pair's two matrices alike)
    unsigned pair = 0;
    unsigned cols = 0;
    unsigned x_kind = 0;          // 0: quantize act x; 1: deferred RMSNORM of act x; 2: the image in qin
    const float *x = nullptr;
    const float *norm_w = nullptr;
    float norm_eps = 0.0f;
    unsigned norm_mode = 0;       // 8 | RMSNORM flags (x_kind 1)
    const uint8_t *qin = nullptr; // x_kind 2: written by the previous pass
    uint8_t *qout = nullptr;      // this pass's output, quantized for the next pass (32-row panels), or null
    unsigned qout_act = 0;
    unsigned item0 = 0;           // the pass's first item (row panel) in the chain's item numbering
};
struct ChainArgs {
    ChainPass p[kMaxChainPasses];
    unsigned n_passes = 0, total_items = 0;
    // [0] the next item to take, [1] CTAs finished, [2 + k] items of pass k finished; zero at the launch, left zero
    // by the launch's last CTA
    unsigned *counters = nullptr;
    unsigned *err = nullptr;      // set when a bounded wait runs out
    unsigned n_stages = 0, stage_bytes = 0, term_bytes = 0, ximg_bytes = 0;
};
constexpr unsigned kChainCounters = 2 + kMaxChainPasses;

// Quantize x (optionally through the RMSNORM arithmetic) to scratch: the same device code as the GEMV prologue.
struct QuantArgs {
    const float *x = nullptr;
    unsigned n = 0;
    unsigned act = 0;             // 0 Q8_0, 1 Q8_1, 2 Q8_K
    const float *norm_w = nullptr;
    float norm_eps = 0.0f;
    unsigned norm_mode = 0;
    int8_t *q = nullptr;
    float *d = nullptr;
    float *s = nullptr;
    int32_t *b = nullptr;
    uint16_t *d16 = nullptr;      // optional FP16 bits of the scales (Q8_0: d, Q8_1: d and s interleaved)
    PeerWait pw;
};

// GEMV_BATCH: y_m = W x_m (+ y_m) for the m < batch activation rows of one command, one read of W per launch. Each
// CTA holds the quantized rows in shared memory: per row and 32-value block 48 bytes, the quants of values 0..15,
// those of values 16..31, then {d, s, sum of q, 0} (the XBlock fields of a GEMV pass).
constexpr unsigned kBatchMax = 8;
constexpr unsigned kBatchImgBlockBytes = 48;
struct BatchArgs {
    MatrixView w;
    const float *x = nullptr;     // row m at x + m * cols
    unsigned cols = 0, batch = 0;
    unsigned m0 = 0, mn = 0;      // the rows of this launch: [m0, m0 + mn)
    unsigned act = 0;             // 0 Q8_0 (Q4_0, Q8_0 weights), 1 Q8_1 (Q4_1)
    float *y = nullptr;           // row m at y + m * ystride
    unsigned ystride = 0, add = 0;
    unsigned n_stages = 0, stage_bytes = 0;  // the weight ring of gemv_batch_kernel (host-planned)
    unsigned *err = nullptr;      // set when a bounded wait runs out
};

// GEMV_BATCH of more than kBatchMax rows (prefill): the rows ("tokens") quantized once into an image in global
// memory, then Y = W X on the tensor cores. Image layout for `tpad` tokens (a multiple of kGemmTokens, the tokens past
// `tokens` zero): the 32 quants of (block b, token t) at xq + (b tpad + t) 32 (values 0..15, then 16..31), d and s of
// Q8_0 / Q8_1 at xd / xs + b tpad + t (FP32 holding the FP16-rounded values).
constexpr unsigned kGemmRows = 128;    // weight rows per tile (the MMA's M)
constexpr unsigned kGemmTokens = 128;  // tokens per tile (the MMA's N)
struct GemmArgs {
    MatrixView w;
    const float *x = nullptr;     // token t at x + t * cols
    unsigned cols = 0, tokens = 0, tpad = 0;
    unsigned act = 0;             // 0 Q8_0 (Q4_0, Q8_0 weights), 1 Q8_1 (Q4_1)
    uint8_t *xq = nullptr;        // the image (device scratch, gemm_image_bytes)
    float *xd = nullptr, *xs = nullptr;
    float *y = nullptr;           // token t at y + t * ystride
    unsigned ystride = 0, add = 0;
    unsigned *err = nullptr;      // set when a bounded wait runs out
    int32_t *sums = nullptr;      // optional: the integer block sums of block 0 of tile (0, 0), [128 rows][128 tokens]
};

}  // namespace b200q
