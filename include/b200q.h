/*
 * b200q — B200-native decode hot path for GGUF-quantized models, behind a plain C ABI.
 *
 * This header is the drop-in boundary. It replaces what the reference's llama.cpp backend binds on its device side:
 *   - the kernel entry point gemvqc16(w0..w19, act, cmds, n_cmds, st0..st3, act_rd)
 *     (reference: fpga/src/gemvqc16.h:122-149), here b200q_run();
 *   - the one-time repack + upload of each GGUF weight tensor (reference: ggml-xrt.cpp:735-765 with
 *     fpga/src/gemvqw_layout.h:137-152), here b200q_upload_weight();
 *   - host<->device copies of the activation buffer act (reference: ggml-xrt.cpp:1136-1143, 1428-1451), here
 *     b200q_act_write() / b200q_act_read();
 *   - the recurrent-state buffer I/O (reference: ggml-xrt.cpp:455-500, xrt_rs_io), here b200q_state_write() /
 *     b200q_state_read();
 *   - the feature probe, a launch with zero commands (reference: ggml-xrt.cpp:1284-1300, gemvqc16.h:124-134);
 *   - the direct-register start + poll with timeout (reference: ggml-xrt.cpp:1241-1280), here one CUDA Graph per
 *     command list (b200q_graph_create / b200q_graph_launch).
 *
 * Command list: B200Q_CMD_WORDS (8) uint32 words per command, at most B200Q_MAX_CMDS (128) commands per list. The
 * words, opcodes, flag bits and validity rules are those of the reference command ISA (fpga/src/gemvqc16.h:24-121),
 * so a list built by the reference backend runs unchanged. Two differences, both invisible to a list builder:
 *   - GEMV words 4/5 (w_off lo/hi) carry the 64-bit handle that b200q_upload_weight() returned (a byte offset into
 *     the device weight arena) instead of a word offset into 20 engine arenas;
 *   - GDN state rows are 512-byte rows of one device buffer (row r at byte 512 r) instead of rows striped over four
 *     HBM ports.
 * Opcodes 12 and up are extensions of this library (decode attention, argmax, embedding row); the reference rejects
 * them, and their feature bits tell a builder whether they exist.
 *
 * All functions return 0 on success. b200q_run() returns a positive 1-based command index when that command is
 * invalid (the commands before it ran, none after it), B200Q_MAX_CMDS + 1 for a list that is too long, and a
 * negative B200Q_ERR_* for host or CUDA failures. After a CUDA failure the context refuses further work
 * (B200Q_ERR_DISABLED), as the reference backend does after a failed launch (ggml-xrt.cpp:2761-2770).
 * No function throws; no torch or CUDA types appear in the signatures (streams are passed as void *).
 */
#ifndef B200Q_H
#define B200Q_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B200Q_API __attribute__((visibility("default")))
#else
#define B200Q_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- command ISA (reference fpga/src/gemvqc16.h:100-135) ---------------------------------------------------- */
#define B200Q_CMD_WORDS 8u
#define B200Q_MAX_CMDS 128u
#define B200Q_OP_GEMV 1u
#define B200Q_OP_RMSNORM 2u
#define B200Q_OP_ADD 3u
#define B200Q_OP_SILU_MUL 4u
#define B200Q_OP_MUL 5u
#define B200Q_OP_UNARY 6u
#define B200Q_OP_GDN 7u
#define B200Q_OP_CONV 8u
#define B200Q_OP_STATE_LOAD 9u
#define B200Q_OP_ROPE 10u
#define B200Q_OP_TRACE 11u
/* extensions (no reference counterpart; see the feature word 3 bits below) */
/* [12, n_head | n_kv_head << 8 | (head_dim / 16) << 16, q_off, k_off, v_off, y_off, pos_off, slot]: pos = act[pos_off]
 * (uint32 bits, so a replayed graph reads each token's position from act); stores this token's k, v (F16) at
 * position pos of KV slot `slot`, then y = softmax(q K^T / sqrt(head_dim)) V over positions 0..pos. A pos outside the
 * slot writes nothing and makes b200q_run / b200q_synchronize return B200Q_ERR_ARG. At most 16 query heads per KV
 * head, head_dim <= 512. */
#define B200Q_OP_ATTN 12u
/* [13, n, x_off, y_off, 0, 0, 0, 0]: y[0] = first index of the maximum (uint32 bits), y[1] = the maximum */
#define B200Q_OP_ARGMAX 13u
/* [14, format (Q4_0 / Q8_0), cols, w_off lo, w_off hi, idx_off, y_off, 0]: y = dequantized row act[idx_off]
 * (uint32 bits) of the matrix, as ggml get_rows */
#define B200Q_OP_GET_ROW 14u
/* [15, n, x_off, y_off, 0, 0, 0, 0]: y = the sum over the ranks of a communicator of their x (n floats; every rank runs
 * the command; the ranks' x are added in rank order, so every rank gets the same bits). Without a communicator, or
 * with one rank: y = x. x and y are the same range or disjoint. For lists built per rank (tensor parallel: each
 * rank multiplies its own column slice of a matrix and the partial outputs are summed), with b200q_comm_init_ex and
 * B200Q_COMM_EXPLICIT. */
#define B200Q_OP_ALLREDUCE 15u
/* [16, n, x_off, y_off, 0, 0, 0, 0]: y[r n .. r n + n) = x of rank r, for every rank r (y: n x world floats); with one
 * rank y = x. x and y are disjoint, or x is rank r's own part of y. */
#define B200Q_OP_ALLGATHER 16u
/* [17, format | flags | (batch - 1) << 16, rows, cols, w_off lo, w_off hi, x_off, y_off]: y_m = W x_m for m < batch
 * (1 to 65536), x_m the cols floats at x_off + m cols, y_m the rows floats at y_off + m round16(rows) (zero padding
 * up to a multiple of 16, as a GEMV's y); flags 0 or B200Q_GEMV_ADD (y_m = W x_m + y_m). Formats Q4_0, Q8_0, Q4_1;
 * cols a multiple of 128; the x and y ranges disjoint; not in a row-sharded context. Every y_m has the bits of the
 * GEMV command on x_m. Up to 8 rows: one kernel reads the weights once for all rows (when the rows' quantized images
 * and term buffers do not fit one CTA's shared memory, once per group of rows). More rows (prefill): the rows are
 * quantized once into a device image the context allocates (before the list runs or is captured), then a tensor-core
 * GEMM (int8 MMA per 32-value block, FP32 block terms in block order) takes tiles of 128 weight rows x 128 rows.
 * A GEMV_BATCH does not consume a deferred RMSNORM: it reads x as act holds it. The batch path of the reference's
 * roadmap (docs/ROADMAP.md:80-96, P2), and the prompt's matrix products. */
#define B200Q_OP_GEMV_BATCH 17u

#define B200Q_GEMV_SWIGLU 0x100u
#define B200Q_GEMV_CONV 0x200u
#define B200Q_GEMV_ADD 0x400u
#define B200Q_GROUP 4u
#define B200Q_GDN_WITH_GEMV 1u
#define B200Q_GDN_L2_QK 2u
#define B200Q_GDN_GATED 4u
#define B200Q_GDN_GATES 8u
#define B200Q_GDN_WITH_OUT 16u
#define B200Q_SILU_MUL_SIGMOID 1u
#define B200Q_NORM_L2 1u
#define B200Q_NORM_NO_WEIGHT 2u
#define B200Q_NORM_DEFER 4u
#define B200Q_UNARY_SILU 1u
#define B200Q_UNARY_SIGMOID 2u
#define B200Q_UNARY_SOFTPLUS 3u
#define B200Q_UNARY_COPY 4u
#define B200Q_TRACE_ENTRIES 512u

/* ggml type ids of the weight formats (reference fpga/src/gemvqw.h:5-11) */
#define B200Q_Q4_0 2u
#define B200Q_Q4_1 3u
#define B200Q_Q8_0 8u
#define B200Q_Q5_K 13u
#define B200Q_Q6_K 14u
#define B200Q_F16 1u /* only for B200Q_OP_GET_ROW and the KV cache */
#define B200Q_MAX_ROWS 65536u
#define B200Q_MAX_COLS 16384u

/* feature words written by a zero-command b200q_run() into act[0], act[1] (reference gemvqc16.h:126-134): the
 * reference's marker and bit meanings, all bits set (Q5_K, Q6_K, Q4_1, every fusion, ROPE, TRACE). act[2] holds
 * this library's own word: marker 0x6B53 in the high half, bit 0 ATTN, bit 1 ARGMAX, bit 2 GET_ROW, bit 3
 * row-sharded multi-GPU lists, bit 4 ALLREDUCE / ALLGATHER, bit 5 GEMV_BATCH, bit 6 GEMV_BATCH of more than 8
 * rows (the 16-bit batch field; the tensor-core prefill GEMM). */
#define B200Q_FEATURES 0x6B51FFFFu
#define B200Q_FEATURES2 0x6B520001u
#define B200Q_FEATURES3 0x6B53007Fu

/* ---- status codes ------------------------------------------------------------------------------------------ */
#define B200Q_OK 0
#define B200Q_ERR_ARG (-1)      /* bad argument (null pointer, range outside a buffer, unknown format) */
#define B200Q_ERR_CUDA (-2)     /* a CUDA call failed; see b200q_last_error(); the context is disabled */
#define B200Q_ERR_NOMEM (-3)    /* the weight arena or a device allocation is full */
#define B200Q_ERR_DISABLED (-4) /* an earlier CUDA failure disabled the context */
#define B200Q_ERR_COMM (-5)     /* NCCL failure or missing communicator */
#define B200Q_ERR_STATE (-6)    /* call out of order (e.g. graph launch on another context) */
#define B200Q_ERR_TIMEOUT (-7)  /* a kernel's bounded wait ran out (reported by b200q_run / b200q_synchronize) */
#define B200Q_ERR_VERIFY (-8)   /* runtime verification: the caller's checker disagreed; the context is disabled */

typedef struct b200q_ctx b200q_ctx;
typedef struct b200q_graph b200q_graph;

typedef struct b200q_config {
    int device;            /* CUDA device ordinal */
    size_t weight_bytes;   /* device weight arena (bump allocated by b200q_upload_weight) */
    size_t act_floats;     /* activation buffer act, in floats (reference: 64 MiB act BO) */
    size_t state_rows;     /* DeltaNet state rows of 128 floats (reference: 4 state BOs) */
    size_t kv_bytes;       /* F16 KV cache of the ATTN extension (0: none) */
    unsigned kv_ctx;       /* tokens per KV slot of the ATTN extension */
} b200q_config;

/* Context: one device, one stream, one weight arena, act, state, scratch. Thread-safe for one caller at a time. */
B200Q_API int b200q_create(const b200q_config *cfg, b200q_ctx **out);
B200Q_API void b200q_destroy(b200q_ctx *ctx);
B200Q_API const char *b200q_last_error(const b200q_ctx *ctx);
/* the context's CUDA stream (a cudaStream_t), for callers that time or order work around it */
B200Q_API void *b200q_stream(b200q_ctx *ctx);
B200Q_API int b200q_synchronize(b200q_ctx *ctx);
/* device addresses of the buffers (for callers that keep inputs resident in HBM) */
B200Q_API void *b200q_act_device_ptr(b200q_ctx *ctx);
B200Q_API void *b200q_state_device_ptr(b200q_ctx *ctx);
B200Q_API void *b200q_kv_device_ptr(b200q_ctx *ctx);

/* Feature words (the three words a zero-command b200q_run writes into act[0..2]), without a launch. */
B200Q_API void b200q_features(uint32_t out[3]);

/* One-time repack + upload of a GGUF matrix (rows x cols, row-major GGUF blocks; format a B200Q_Q* id). The bits
 * of every scale and quant stay as they are; only their arrangement changes: Q4_0 / Q4_1 / Q8_0 rows are cut into
 * panels of P rows (P from the matrix shape) whose quants are interleaved 16 bytes per (row, block) step and whose
 * scales follow each 32-block tile; Q5_K / Q6_K matrices are cut into tiles of R rows x up to 16384 columns with
 * the quant fields permuted within each super-block. b200q_layout() reports the arrangement.
 * block_cols: 0, or 256 for a matrix that a GDN_WITH_OUT step consumes (accepted for list compatibility; the
 * device layout is the same). *w_off receives the handle for GEMV words 4/5. In a row-sharded context (after
 * b200q_comm_init) only this rank's row slice is kept. */
B200Q_API int b200q_upload_weight(b200q_ctx *ctx, const void *gguf, unsigned rows, unsigned cols, unsigned format,
                        unsigned block_cols, uint64_t *w_off);
/* As b200q_upload_weight; flags B200Q_UPLOAD_REPLICATE keeps all rows on every rank of a row-sharded context
 * (for matrices read by GET_ROW, such as the token embedding). B200Q_UPLOAD_PASS_ROWS(n) tells a Q4_0 / Q8_0 / Q4_1
 * matrix that its GEMVs share a multi-output pass of n rows in all (say q, k and v on one x): the panel height is
 * then chosen for the whole pass, so that the members' panels make one wave of CTAs rather than two (a layout
 * choice only; results are the same either way). */
#define B200Q_UPLOAD_REPLICATE 1u
#define B200Q_UPLOAD_PASS_ROWS(n) ((unsigned)(n) << 8)
/* the source is a Q4_0 matrix in ggml's CPU_REPACK block_q4_0x8 layout (rows a multiple of 8): it is read back to
 * GGUF rows first (b200q_q4_0x8_to_q4_0), as the reference backend does for tensors of a CPU_REPACK buffer */
#define B200Q_UPLOAD_SRC_Q4_0X8 2u
B200Q_API int b200q_upload_weight_ex(b200q_ctx *ctx, const void *gguf, unsigned rows, unsigned cols, unsigned format,
                           unsigned block_cols, unsigned flags, uint64_t *w_off);
/* Device bytes one matrix takes in the arena (all rows, one rank); _ex: uploaded with these flags. */
B200Q_API size_t b200q_weight_device_bytes(unsigned rows, unsigned cols, unsigned format);
B200Q_API size_t b200q_weight_device_bytes_ex(unsigned rows, unsigned cols, unsigned format, unsigned flags);
/* Bytes of one GGUF row of the format (0 for an unknown format). */
B200Q_API size_t b200q_gguf_row_bytes(unsigned cols, unsigned format);
/* Reset the bump allocator of the weight arena (all handles become invalid). */
B200Q_API int b200q_weights_reset(b200q_ctx *ctx);

/* act and state I/O (synchronous; offsets in floats / rows). */
B200Q_API int b200q_act_write(b200q_ctx *ctx, size_t off, const float *src, size_t n);
B200Q_API int b200q_act_read(b200q_ctx *ctx, size_t off, float *dst, size_t n);
B200Q_API int b200q_act_fill(b200q_ctx *ctx, size_t off, float value, size_t n);
B200Q_API int b200q_state_write(b200q_ctx *ctx, size_t row, const float *src, size_t rows);
B200Q_API int b200q_state_read(b200q_ctx *ctx, size_t row, float *dst, size_t rows);
B200Q_API int b200q_kv_write(b200q_ctx *ctx, size_t byte_off, const void *src, size_t bytes);
/* Stream-ordered act copies for a per-token loop: enqueued on the context stream behind the lists already launched,
 * no wait. The host buffer must stay untouched (write) or unread (read) until b200q_synchronize() returns; page-locked
 * host memory makes the copy asynchronous, pageable memory may make the call wait. */
B200Q_API int b200q_act_write_async(b200q_ctx *ctx, size_t off, const float *src, size_t n);
B200Q_API int b200q_act_read_async(b200q_ctx *ctx, size_t off, float *dst, size_t n);

/* Run one command list (reference gemvqc16 contract, see the top of this header); synchronous: returns once the
 * GPU finished the list. n_cmds = 0 writes the feature words into act[0..2]. */
B200Q_API int b200q_run(b200q_ctx *ctx, const uint32_t *cmds, unsigned n_cmds);
/* Same, asynchronous on the context stream (validation still on the host, before any launch). */
B200Q_API int b200q_run_async(b200q_ctx *ctx, const uint32_t *cmds, unsigned n_cmds);

/* A valid list captured once as a CUDA Graph (one per token in a decode loop); launch replays it on the context
 * stream. Returns the list's status (a rejected list makes no graph). */
B200Q_API int b200q_graph_create(b200q_ctx *ctx, const uint32_t *cmds, unsigned n_cmds, b200q_graph **out);
B200Q_API int b200q_graph_launch(b200q_ctx *ctx, b200q_graph *graph);
B200Q_API void b200q_graph_destroy(b200q_graph *graph);
/* Launches graphs[i % n_graphs] for i = 0 .. launches - 1 on the context stream (a token loop without host
 * round trips between launches). */
B200Q_API int b200q_graph_launch_many(b200q_ctx *ctx, b200q_graph *const *graphs, unsigned n_graphs,
                                      unsigned launches);
/* kernels one replay of the graph launches */
B200Q_API unsigned b200q_graph_kernel_count(const b200q_graph *graph);

/* ---- diagnostics: feature mask and runtime verification ------------------------------------------------------
 * Feature mask (reference: GGML_XRT_FEATURE_MASK, ggml-xrt.cpp:1294-1299). The environment variable
 * B200Q_FEATURE_MASK=<bits> (read at b200q_create) or b200q_set_feature_mask sets it; by default all bits are set but
 * bit 21 (B200Q_DEFAULT_FEATURE_MASK).
 *   bits 0..15: the reference feature word. A cleared bit hides that fused form from the feature probe (a zero-command
 *     b200q_run), so a list builder emits the plain command sequence instead; the weight-format and layout bits
 *     (0, 1, 2, 13) always stay. Where this library also fuses internally, the cleared bit turns that off too:
 *     bit 3 multi-output passes (each GEMV or SwiGLU pair of a group then runs as its own launch), bit 9 deferred
 *     RMSNORM in the GEMV prologue (the norm row is then stored at its command), bit 15 the DeltaNet step handing
 *     its ssm_out GEMV the quantized y.
 *   bits 16..21: this library's own fusions: 16 a GEMV pass handing the next pass its quantized x, 17 per-panel
 *     sums of squares handed to the next deferred norm, 18 programmatic dependent launch, 19 runs of RMSNORM / ROPE
 *     in one launch, 20 the attention gate applied in the attention merge, 21 runs of Q4_0 / Q8_0 GEMV passes
 *     (single matrices or SwiGLU pairs, plain or residual-ADD writers) executed by one persistent kernel.
 * Every fused form gives the same values as its plain form, so results do not depend on the mask (bit for bit, but
 * for the deferred norm's FP64 sum of squares, which is added in a different fixed order when stored; both round to
 * the same FP32 scale unless the exact sum lies within ~1e-13, relative, of an FP32 rounding boundary). The mask is
 * for A/B measurements and for checking exactly that. Graphs keep the mask they were captured with. */
#define B200Q_MASK_GROUPS (1u << 3)
#define B200Q_MASK_DEFER_NORM (1u << 9)
#define B200Q_MASK_GDN_OUT (1u << 15)
#define B200Q_MASK_X_IMAGE (1u << 16)
#define B200Q_MASK_NORM_PARTIALS (1u << 17)
#define B200Q_MASK_PDL (1u << 18)
#define B200Q_MASK_ROW_OPS (1u << 19)
#define B200Q_MASK_ATTN_GATE (1u << 20)
#define B200Q_MASK_CHAINS (1u << 21) /* off by default: measured slower than the passes' own kernels */
#define B200Q_DEFAULT_FEATURE_MASK (0xFFFFFFFFu & ~B200Q_MASK_CHAINS)
B200Q_API int b200q_set_feature_mask(b200q_ctx *ctx, uint32_t mask);
B200Q_API uint32_t b200q_feature_mask(const b200q_ctx *ctx);

/* Runtime verification (reference: GGML_XRT_VERIFY_CALLS=<n>, ggml-xrt.cpp:62-66, 1153-1202): the next n_calls lists
 * run by b200q_run or replayed by b200q_graph_launch(_many) run synchronously, with act, the state rows and the KV
 * cache copied to host memory before and after; the checker gets both copies and the list and returns 0 when the
 * results agree with its own computation of the list (the library links no checker of its own; a caller supplies
 * the CPU reference). A non-zero return makes the call return B200Q_ERR_VERIFY with the checker's message and
 * disables the context, as the reference backend disables itself. n_calls < 0: the count is taken from the
 * environment variable B200Q_VERIFY_CALLS (0 when unset); fn NULL turns verification off. */
typedef struct b200q_verify_view {
    const uint32_t *cmds;
    unsigned n_cmds;
    int status;                 /* the list's status (0, or the 1-based index of its first invalid command) */
    const float *act_before, *act_after;
    size_t act_floats;
    const float *state_before, *state_after;
    size_t state_rows;
    const void *kv_before, *kv_after;
    size_t kv_bytes;
    unsigned kv_ctx;
} b200q_verify_view;
typedef int (*b200q_verify_fn)(void *user, const b200q_verify_view *view, char *msg, unsigned msg_len);
B200Q_API int b200q_set_verify(b200q_ctx *ctx, b200q_verify_fn fn, void *user, int n_calls);

/* ---- host-only planning (no GPU needed) ---------------------------------------------------------------------- */
typedef struct b200q_pass_info {
    uint32_t first_cmd;   /* index of the first command of the pass */
    uint32_t n_cmds;      /* commands the pass consumes */
    uint32_t kind;        /* B200Q_PASS_* */
    uint32_t n_members;   /* GEMVs in the pass */
    uint32_t fused_norm;  /* 1: the GEMVs quantize a deferred RMSNORM's row, computed in the pass; 2: the row stored at
                           * the RMSNORM command (its x or weight changes before this pass) */
} b200q_pass_info;
#define B200Q_PASS_GEMV 1u
#define B200Q_PASS_ELEMENTWISE 2u
#define B200Q_PASS_GDN 3u
#define B200Q_PASS_NOP 4u
#define B200Q_PASS_EXT 5u
/* Validate a list and return its pass structure as the device run would execute it; the return value is the one
 * b200q_run would give (0 or the 1-based index of the first invalid command). */
B200Q_API int b200q_plan(const uint32_t *cmds, unsigned n_cmds, b200q_pass_info *passes, unsigned max_passes,
               unsigned *n_passes);

/* ---- host-only layout (no GPU): the device layout of a matrix, its repack and the inverse, for tests ---------- */
typedef struct b200q_layout_info {
    uint32_t rows_per_tile, blocks_per_tile, tiles_per_row_tile, row_tiles, tile_bytes;
    uint64_t total_bytes;
} b200q_layout_info;
B200Q_API int b200q_layout(unsigned rows, unsigned cols, unsigned format, unsigned sms, b200q_layout_info *out);
/* As b200q_layout for a matrix uploaded with `flags` (B200Q_UPLOAD_PASS_ROWS). */
B200Q_API int b200q_layout_ex(unsigned rows, unsigned cols, unsigned format, unsigned sms, unsigned flags,
                              b200q_layout_info *out);
/* Repack all rows (dst: total_bytes of the layout for `sms`), and the inverse of one row back to GGUF bytes. */
B200Q_API int b200q_repack_host(const void *gguf, unsigned rows, unsigned cols, unsigned format, unsigned sms,
                                void *dst);
B200Q_API int b200q_unpack_row_host(const void *dev, unsigned rows, unsigned cols, unsigned format, unsigned sms,
                                    unsigned row, void *gguf_row);

/* ---- checks of the bit-exact intermediate values (same device code as the GEMV passes) ---------------------- */
/* Quantize act[x_off .. x_off + n) as a GEMV pass of format `format` would (Q8_0 for Q4_0/Q8_0, Q8_K for
 * Q5_K/Q6_K, Q8_1 for Q4_1), optionally through a deferred RMSNORM (norm_w_off = UINT32_MAX: none; else the
 * RMSNORM's w_off, eps, flags). Outputs: q (n int8), scales (Q8_0: n/32 uint16 FP16 bits; Q8_K: n/256 floats;
 * Q8_1: n/32 pairs of uint16), bsums (Q8_0/Q8_1: n/32 int32 block sums of q; Q8_K: n/16 int32). */
B200Q_API int b200q_debug_quantize(b200q_ctx *ctx, unsigned format, size_t x_off, unsigned n, uint32_t norm_w_off,
                         float norm_eps, unsigned norm_flags, int8_t *q, void *scales, int32_t *bsums);
/* Per-block integer dot products of one GEMV command (Q4_0/Q8_0: rows x cols/32 int32 sumi, the ints that scale
 * into each FP32 term; Q5_K/Q6_K: rows x cols/256 x 9 int32: the 8 lane sums of the scaled products, then the
 * mins sum (0 for Q6_K); Q4_1: rows x cols/32). For a GEMV_BATCH command of more than 8 rows (the tensor-core
 * GEMM, which it runs): the 128 x 128 int32 sums of block 0 of weight rows 0..127 and batch rows 0..127, row-major
 * by weight row (entries of batch rows past the batch: 0). */
B200Q_API int b200q_debug_block_sums(b200q_ctx *ctx, const uint32_t cmd[8], int32_t *out);

/* ---- the activation quantizer without a context and without allocation -------------------------------------
 * No counterpart in the reference (its quantizer runs inside the FPGA kernel, gemvqc16.cpp).
 * b200q_quantize_noalloc quantizes n device floats exactly as b200q_debug_quantize does (the same kernel and
 * arithmetic, the same output layout in host memory), for callers that hold no b200q context and may not allocate
 * device memory: a host runtime whose device memory is all reserved up front by its own pool, or a diagnostic path
 * that runs after an allocation failed. It allocates nothing. Its scratch is a fixed array in device memory carried
 * by the library (one per device), so n is limited to B200Q_NOALLOC_MAX_N; larger n is rejected with B200Q_ERR_ARG.
 *   x, norm_w: device (or managed) memory of `device`, 4-byte aligned, each holding n floats inside its allocation
 *   (norm_w NULL: no deferred RMSNORM; else eps and norm_flags as in RMSNORM) — checked on the host before the
 *   launch, so a host pointer, another device's pointer, a misaligned pointer or a range past the allocation's end
 *   returns B200Q_ERR_ARG and never reaches the GPU; stream: a cudaStream_t of that device (NULL: the legacy default
 *   stream; a stream of another device is rejected), synchronized before the call returns; q / scales / bsums: host
 *   memory as in b200q_debug_quantize (NULL: not copied); err_msg: receives the reason of a failure (may be NULL).
 * The first call on a device looks up the scratch address (cudaGetSymbolAddress, which may initialize the CUDA
 * context): make it before any stream capture. The address is kept per device and looked up again when the device's
 * context changed (after cudaDeviceReset). Nothing in the scratch needs to start at zero. Calls on the same device
 * that overlap (from other threads, or on other streams before the previous one returned) share the scratch and
 * race: the library serializes calls within one process, other processes must not share a device this way. */
#define B200Q_NOALLOC_MAX_N 16384
B200Q_API int b200q_quantize_noalloc(int device, const float *x, unsigned n, unsigned format, const float *norm_w,
                                     float norm_eps, unsigned norm_flags, void *stream, int8_t *q, void *scales,
                                     int32_t *bsums, char *err_msg, unsigned err_len);

/* ---- GGUF files and the CPU backend's Q4_0x8 layout (host only) ------------------------------------------------
 * For callers that load weights without llama.cpp. The reference backend receives its weights from llama.cpp's GGUF
 * loader as ggml tensors (ggml-xrt.cpp:642-653 keys them by tensor, data pointer, type, shape and bytes) and reads
 * their rows back to GGUF blocks before its own repack (xrt_gguf, ggml-xrt.cpp:675-710); these functions give the
 * same GGUF rows straight from a file.
 * b200q_gguf_open maps the file read-only and parses the header, metadata and tensor table (GGUF v2 / v3); every
 * length and offset is checked against the file size, and a truncated or corrupt file returns B200Q_ERR_ARG with the
 * reason in err. Pointers handed out (names, keys, values, tensor data) stay valid until b200q_gguf_close. */
typedef struct b200q_gguf b200q_gguf;
typedef struct b200q_gguf_tensor_info {
    const char *name;    /* NUL-terminated */
    uint32_t type;       /* ggml type id (B200Q_Q4_0, ..., 0 F32, 1 F16) */
    uint32_t n_dims;
    uint64_t ne[4];      /* ne[0] elements per row (columns), ne[1] rows; 1 past n_dims */
    uint64_t offset;     /* byte offset of the data in the file */
    uint64_t bytes;      /* bytes of the data (0 for a type this reader does not size) */
    const void *data;    /* the data in the read-only mapping (NULL when bytes is 0) */
} b200q_gguf_tensor_info;
typedef struct b200q_gguf_kv_info {
    const char *key;
    uint32_t type;        /* GGUF value type: 0 u8, 1 i8, 2 u16, 3 i16, 4 u32, 5 i32, 6 f32, 7 bool, 8 string,
                           * 9 array, 10 u64, 11 i64, 12 f64 */
    uint32_t array_type;  /* arrays: the element type */
    uint64_t count;       /* arrays: elements; else 1 */
    const void *value;    /* scalars: the value's bytes; strings: the bytes (str_len of them, not NUL-terminated);
                           * arrays of scalars: the first element; arrays of strings: the first string's 8-byte length */
    uint64_t str_len;
} b200q_gguf_kv_info;
B200Q_API int b200q_gguf_open(const char *path, b200q_gguf **out, char *err, unsigned err_len);
B200Q_API void b200q_gguf_close(b200q_gguf *g);
B200Q_API uint32_t b200q_gguf_version(const b200q_gguf *g);
B200Q_API uint64_t b200q_gguf_n_tensors(const b200q_gguf *g);
B200Q_API uint64_t b200q_gguf_n_kv(const b200q_gguf *g);
B200Q_API int b200q_gguf_tensor(const b200q_gguf *g, uint64_t index, b200q_gguf_tensor_info *out);
B200Q_API int b200q_gguf_find_tensor(const b200q_gguf *g, const char *name, uint64_t *index);
B200Q_API int b200q_gguf_kv(const b200q_gguf *g, uint64_t index, b200q_gguf_kv_info *out);
B200Q_API int b200q_gguf_find_kv(const b200q_gguf *g, const char *key, uint64_t *index);
/* integer (any integer or bool type) / floating (f32, f64 or an integer) metadata value of `key` */
B200Q_API int b200q_gguf_get_int(const b200q_gguf *g, const char *key, int64_t *value);
B200Q_API int b200q_gguf_get_float(const b200q_gguf *g, const char *key, double *value);
/* b200q_upload_weight_ex of tensor `index` (a 2-D matrix: ne[0] columns, ne[1] rows) straight from the mapping. */
B200Q_API int b200q_upload_gguf_tensor(b200q_ctx *ctx, const b200q_gguf *g, uint64_t index, unsigned block_cols,
                                       unsigned flags, uint64_t *w_off);
/* Q4_0 rows back from ggml's CPU_REPACK block_q4_0x8 layout (rows a multiple of 8, cols of 32), bit for bit the
 * original GGUF rows (reference: ggml-xrt.cpp:675-710, xrt_gguf). dst: rows x cols / 32 x 18 bytes. */
B200Q_API int b200q_q4_0x8_to_q4_0(const void *src, unsigned rows, unsigned cols, void *dst);

/* ---- multi-GPU (one process per GPU, NCCL over NVLink) ------------------------------------------------------- */
#define B200Q_UNIQUE_ID_BYTES 128
B200Q_API int b200q_comm_unique_id(uint8_t id[B200Q_UNIQUE_ID_BYTES]);
/* Join a communicator of world ranks; from then on uploads keep only this rank's row slice of each shardable
 * matrix (rows divisible by 16 x world) and every pass gathers its GEMV outputs so all ranks hold the full act, as
 * with one GPU (results bit-identical to one GPU). The gather is an NCCL all-gather per sharded output, or with the
 * environment variable B200Q_PEER=1 the GEMV kernels store their rows straight into every peer's act over NVLink
 * (CUDA IPC mappings made here) and the next kernel waits for the peers' flags (bounded waits). */
B200Q_API int b200q_comm_init(b200q_ctx *ctx, int world, int rank, const uint8_t id[B200Q_UNIQUE_ID_BYTES]);
/* As b200q_comm_init; flags B200Q_COMM_EXPLICIT: the caller builds each rank's own lists (tensor parallel: its own
 * row or column slices of the matrices, uploaded as they are, and ALLREDUCE / ALLGATHER commands where partial
 * results meet). Uploads then keep all rows and no pass gathers anything by itself. ALLREDUCE runs as one kernel that
 * writes this rank's part into every peer's receive buffer over NVLink (CUDA IPC mappings made here; each value with
 * its launch number in one 8-byte word, so no fence or flag is needed) and adds the parts in rank order after bounded
 * waits (up to 8 ranks and 4096 floats; larger ones, ALLGATHER, and everything with the environment variable
 * B200Q_PEER=0 run on NCCL). */
#define B200Q_COMM_EXPLICIT 1u
B200Q_API int b200q_comm_init_ex(b200q_ctx *ctx, int world, int rank, const uint8_t id[B200Q_UNIQUE_ID_BYTES],
                                 unsigned flags);
/* The rows [*r0, *r1) of a rows-row matrix that rank `rank` of `world` keeps at upload (host only): a slice of
 * rows / world when rows divide by 16 x world and flags has no B200Q_UPLOAD_REPLICATE, else all rows. */
B200Q_API int b200q_row_slice(unsigned rows, unsigned flags, int world, int rank, unsigned *r0, unsigned *r1);
B200Q_API int b200q_comm_world(const b200q_ctx *ctx);

/* ---- graph lowering (host only): a model's op graph to command lists ------------------------------------------
 * The reference's backend walks a ggml graph, finds the fusions the kernel supports and emits 8-word command lists
 * with the operands placed in act (plan and fusion analysis: ggml-xrt.cpp:1815-2188; emission: :2190-2745;
 * supports_op: :2998-3015). This is that step for callers that hold their graph in another form: an array of nodes in
 * execution order, each naming its operands by index. The lowering
 *   - places every tensor in act (16-float aligned; INPUT tensors, which the caller writes, and PARAM tensors, which
 *     stay resident, too) and reports the offsets;
 *   - fuses what the command ISA can fuse, each fusion kept only when its feature bit is set (the reference's
 *     feature-word bits): a SWIGLU of two MUL_MATs on one x read only by it becomes a SwiGLU GEMV pair (bit 3); an
 *     ADD of a MUL_MAT read only by it and an operand computed before the MUL_MAT becomes the GEMV's ADD epilogue
 *     (bit 8); a CONV of a MUL_MAT read only by it becomes the GEMV's CONV epilogue (bit 6); an RMS_NORM, with its
 *     weight MUL, read only by MUL_MATs of the same segment becomes a deferred RMSNORM (bit 9); an RMS_NORM followed
 *     by a MUL by a PARAM row becomes one weighted RMSNORM; L2_NORMs of a GDN's q and k and the gated output
 *     MUL(MUL(RMS_NORM(y), w), SILU(z)) fold into the GDN command (bit 7), the gates SIGMOID(beta) and
 *     MUL(SOFTPLUS(ADD(alpha, dt)), a) too (bit 10), and a MUL_MAT on the GDN output right behind it joins the step's
 *     pass (bit 15); MUL by SILU(g) becomes SILU_MUL, MUL by SIGMOID(g) (g possibly strided rows) SILU_MUL with the
 *     sigmoid flag (word 1 bit 0);
 *   - packs the commands of consecutive segments (a node with B200Q_NODE_SEGMENT_END closes one, e.g. a layer)
 *     into lists of at most 128 commands, never splitting a segment, and ends a list after a segment holding a node
 *     flagged B200Q_NODE_LIST_END.
 * No counterpart type in the reference: it stands for the ggml_cgraph the reference's backend receives. */
#define B200Q_NODE_INPUT 1u     /* n floats the caller writes before the lists run (or a buffer commands fill) */
#define B200Q_NODE_PARAM 2u     /* n resident floats the caller writes once (norm weights, conv kernels, states) */
#define B200Q_NODE_VIEW 3u      /* rows u[3] of u[1] floats every u[2] floats of src[0], from float u[0]; no command */
#define B200Q_NODE_MUL_MAT 4u   /* y[rows] = W x: src[0] x (cols floats), weight handle, fmt, rows, cols; u[0] > 1:
                                 * u[0] rows of x (u[0] cols floats) into u[0] rows of round16(rows) floats (n), one
                                 * GEMV_BATCH command (Q4_0 / Q8_0 / Q4_1; joins no fusion) */
#define B200Q_NODE_RMS_NORM 5u  /* rows of n / rows floats of src[0] (eps) */
#define B200Q_NODE_L2_NORM 6u   /* as RMS_NORM with the L2 scale */
#define B200Q_NODE_MUL 7u       /* src[0] * src[1] (src[1] of one row's length: the same row for every row) */
#define B200Q_NODE_ADD 8u       /* src[0] + src[1] */
#define B200Q_NODE_SWIGLU 9u    /* silu(src[0]) * src[1] */
#define B200Q_NODE_UNARY 10u    /* u[0]: B200Q_UNARY_SILU / SIGMOID / SOFTPLUS / COPY of src[0] */
#define B200Q_NODE_CONV 11u     /* causal conv (k = 4) of src[0] (channels) with kernel PARAM src[1] [4 x ch] and state
                                 * PARAM src[2] [3 x ch], updated in place; u[0] 1: SiLU of the result */
#define B200Q_NODE_GDN 12u      /* DeltaNet step: src[0] q, [1] k, [2] v, [3] g, [4] beta; u[0] value heads, u[1] key
                                 * heads, u[2] the first state row; eps = the q scale; y = hv x 128 floats */
#define B200Q_NODE_ROPE 13u     /* NEOX rotation of src[0] by the cos/sin row src[1]: u[0] dims, u[1] row length, u[2] rows */
#define B200Q_NODE_ATTN 14u     /* src[0] q, [1] k, [2] v, [3] position (uint32 bits); u[0] heads, u[1] KV heads,
                                 * u[2] head size, u[3] KV slot */
#define B200Q_NODE_GET_ROWS 15u /* row act[src[0]] (uint32 bits) of a Q4_0 / Q8_0 matrix (weight, fmt, cols) */
#define B200Q_NODE_ARGMAX 16u   /* {first index of the maximum (uint32 bits), maximum} of src[0] */
#define B200Q_NODE_ALLREDUCE 17u /* the sum over the communicator's ranks of src[0] (tensor-parallel lists) */
#define B200Q_NODE_ALLGATHER 18u /* the ranks' src[0] side by side (n = their floats x ranks); src[0] may be this rank's
                                  * own part of dst */
#define B200Q_NODE_SEGMENT_END 1u  /* flags: the last node of a segment (lists are cut between segments) */
#define B200Q_NODE_OUTPUT 2u       /* flags: the caller reads the tensor after the lists (it is kept, not fused away) */
#define B200Q_NODE_LIST_END 4u     /* flags: the list ends with this node's segment (tensor-parallel ranks whose
                                    * segments differ in length cut their lists at the same segments this way, so
                                    * their lists hold the same collectives) */
#define B200Q_NODE_SRCS 6u
typedef struct b200q_node {
    uint32_t op, flags;
    int32_t src[B200Q_NODE_SRCS]; /* operand nodes (earlier indices), -1 for none */
    int32_t dst;                  /* -1, or an earlier node (INPUT or VIEW of one) whose floats this output overwrites */
    uint32_t n;                   /* output floats */
    uint32_t fmt, rows, cols;     /* MUL_MAT / GET_ROWS weight; norms: rows */
    uint64_t weight;              /* weight handle (b200q_upload_weight) */
    float eps;
    uint32_t u[4];
} b200q_node;
typedef struct b200q_lowering b200q_lowering;
/* Lower nodes[0..n_nodes) with `features` (the feature word of b200q_features / a zero-command run: bits 0..15 of
 * word 0, bit 16 = word 1 bit 0). 0 on success; else B200Q_ERR_ARG with the reason in err, naming the node. */
B200Q_API int b200q_lower(const b200q_node *nodes, unsigned n_nodes, uint32_t features, b200q_lowering **out,
                          char *err, unsigned err_len);
B200Q_API void b200q_lowering_free(b200q_lowering *l);
B200Q_API unsigned b200q_lowering_lists(const b200q_lowering *l);
/* the commands of list i (8 words each); NULL past the last list */
B200Q_API const uint32_t *b200q_lowering_list(const b200q_lowering *l, unsigned i, unsigned *n_cmds);
/* act offset of node i's floats (SIZE_MAX for a tensor folded into a command, which act never holds) */
B200Q_API size_t b200q_lowering_offset(const b200q_lowering *l, unsigned node);
/* act floats the lowered lists use (the context's act_floats must be at least this) */
B200Q_API size_t b200q_lowering_act_floats(const b200q_lowering *l);
/* 1 if node i (with its operands) can run on this library, else 0 (the reference backend's supports_op) */
B200Q_API int b200q_node_supported(const b200q_node *nodes, unsigned i);

#ifdef __cplusplus
}
#endif
#endif /* B200Q_H */
