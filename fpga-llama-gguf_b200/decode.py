"""Synthetic hybrid decoder (Qwen3.5-like: Gated DeltaNet layers with a gated GQA attention layer every fourth layer)
expressed as b200q command lists, one token per replay.

This is the caller side of the hot path: the lists a ggml backend emits for one decode token of such a model
(reference: the XRT backend's graph walk, ggml-xrt.cpp:2190-2745, with GATED_DELTA_NET at :2607-2727 and the output
head cut into GEMVs of at most 65536 rows at :133-139 / :1536-1554), written with this library's builders. The head
pieces here are multiples of 128 rows (the reference cuts 65520-row pieces), so that every piece row-shards over
2, 4 or 8 GPUs. The reference runs the
attention core on the CPU; here it is the ATTN extension, so a whole token is device work and consecutive tokens
chain on the device: ARGMAX writes the next token's id where the next token's GET_ROW reads it.

Per token the host writes one record (the position as uint32 bits and the RoPE cos/sin row); everything else is
resident. Weights are seeded synthetic GGUF blocks (Q4_0 layers, Q6_K head, Q4_0 embedding table); no model file is
read. A list holds at most 128 commands, so a token is several lists, cut at layer boundaries.

Layer i is an attention layer when i % attn_every == attn_every - 1, else a Gated DeltaNet layer:

  GDN layer        RMSNORM(defer) -> {qkv GEMV + CONV epilogue, z, beta, alpha} one group
                   -> GDN step (L2 q/k, gates, gated norm * silu(z)) with ssm_out GEMV + residual ADD fused
  attention layer  RMSNORM(defer) -> {q|gate, k, v} one group -> per-head RMSNORM of q and k -> NEOX RoPE
                   -> ATTN over the F16 KV slot -> sigmoid(gate) * attention -> o GEMV + residual ADD
  both             RMSNORM(defer) -> gate + up GEMV pair with SwiGLU -> down GEMV + residual ADD
  head             RMSNORM(defer) -> Q6_K GEMV pieces (one group) -> ARGMAX
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import (CMD_WORDS, GDN_GATED, GDN_GATES, GDN_L2_QK, GDN_WITH_OUT, GEMV_ADD, GEMV_CONV, GEMV_SWIGLU, MAX_CMDS, NORM_DEFER,
               Q4_0, Q6_K, UPLOAD_PASS_ROWS, UPLOAD_REPLICATE, add, argmax, attn, cmd_list, conv, gdn, gemv, get_row, gguf_row_bytes,
               rmsnorm, rope, silu_mul)
from . import synth

GDN_DIM = 128  # DeltaNet head size of the command ISA (state rows of 128 floats)
RECORD = 16 + 128  # per-token host record: position bits, then the cos/sin row (up to 128 floats)


@dataclass(frozen=True)
class Shape:
    hidden: int = 2560
    ffn: int = 9216
    n_layers: int = 32
    attn_every: int = 4
    vocab: int = 151936
    gdn_heads: int = 16         # value heads = key heads, head size 128
    n_head: int = 16
    n_kv_head: int = 4
    head_dim: int = 256
    rope_dims: int = 64         # partial rotary: the first 64 of 256 dims of each head
    rope_theta: float = 1e7
    kv_ctx: int = 640           # KV slot length: 512 prefilled + 128 decoded tokens
    prefill: int = 512
    eps: float = 1e-6
    head_piece: int = 50688     # output-head rows per GEMV (<= 65536; a multiple of 128 so it shards up to 8 GPUs)

    def is_attn(self, layer: int) -> bool:
        return layer % self.attn_every == self.attn_every - 1

    @property
    def n_attn(self) -> int:
        return sum(self.is_attn(i) for i in range(self.n_layers))

    @property
    def n_gdn(self) -> int:
        return self.n_layers - self.n_attn

    @property
    def gdn_rows(self) -> int:   # state rows of one GDN layer
        return self.gdn_heads * GDN_DIM

    @property
    def kv_slot_bytes(self) -> int:  # K then V, [n_kv_head][kv_ctx][head_dim] F16 each
        return 2 * self.n_kv_head * self.kv_ctx * self.head_dim * 2

    def head_pieces(self):
        out, r0 = [], 0
        while r0 < self.vocab:
            n = min(self.head_piece, self.vocab - r0)
            out.append((r0, n))
            r0 += n
        return out

    def bytes_per_token(self, pos: int | None = None) -> int:
        """Algorithmic HBM bytes of one token: every weight byte of the layers and the head (GGUF bits), the KV rows
        read at position pos (default: the prefill length), and the DeltaNet state read + written."""
        p = self.prefill if pos is None else pos
        H, F, d = self.hidden, self.ffn, self.gdn_rows
        q4 = lambda rows, cols: rows * gguf_row_bytes(cols, Q4_0)
        ffn = q4(F, H) * 2 + q4(H, F)
        gdn_l = q4(3 * d, H) + q4(d, H) + 2 * q4(self.gdn_heads, H) + q4(H, d)
        att = self.n_head * self.head_dim
        attn_l = q4(2 * att, H) + 2 * q4(self.n_kv_head * self.head_dim, H) + q4(H, att)
        layers = self.n_layers * ffn + self.n_gdn * gdn_l + self.n_attn * attn_l
        head = self.vocab * gguf_row_bytes(H, Q6_K)
        kv = self.n_attn * 2 * self.n_kv_head * p * self.head_dim * 2
        state = self.n_gdn * 2 * d * GDN_DIM * 4
        return layers + head + kv + state


SHAPE_4B = Shape()
SHAPE_9B = Shape(hidden=4096, ffn=12288)


class ActLayout:
    """Float offsets into act (16-float aligned): shared scratch first, then each layer's resident parameters."""

    def __init__(self, s: Shape):
        self.top = 0
        H, d = s.hidden, s.gdn_rows
        att, kvd = s.n_head * s.head_dim, s.n_kv_head * s.head_dim
        self.REC = self._take(RECORD)
        self.POS, self.CS = self.REC, self.REC + 16
        self.TOK = self._take(16)
        self.X, self.XN, self.OUT = self._take(H), self._take(H), self._take(H)
        self.QKV, self.QKVC, self.Z = self._take(3 * d), self._take(3 * d), self._take(d)
        self.BETA, self.ALPHA, self.Y = self._take(s.gdn_heads), self._take(s.gdn_heads), self._take(d)
        self.QG, self.K, self.V = self._take(2 * att), self._take(kvd), self._take(kvd)
        self.QN, self.KN, self.QR, self.KR = self._take(att), self._take(kvd), self._take(att), self._take(kvd)
        self.YA, self.YG = self._take(att), self._take(att)
        self.FF = self._take(s.ffn)
        self.LOGITS = self._take(s.vocab)
        self.ONORM = self._take(H)
        self.layer = []
        for i in range(s.n_layers):
            p = {"attn_norm": self._take(H), "ffn_norm": self._take(H)}
            if s.is_attn(i):
                p.update(q_norm=self._take(s.head_dim), k_norm=self._take(s.head_dim))
            else:
                p.update(conv_w=self._take(4 * 3 * d), conv_hist=self._take(3 * 3 * d), dt=self._take(s.gdn_heads),
                         a=self._take(s.gdn_heads), gdn_norm=self._take(GDN_DIM))
            self.layer.append(p)
        self.size = self.top

    def _take(self, n: int) -> int:
        off = self.top
        self.top += (n + 15) // 16 * 16
        return off


class HybridDecoder:
    """The synthetic model: seeded weights and resident parameters, the per-token lists and host records."""

    def __init__(self, shape: Shape = SHAPE_4B, seed: int = 4, first_token: int = 1):
        self.s = shape
        self.seed = seed
        self.first_token = first_token
        self.L = ActLayout(shape)
        self.handles: dict = {}

    # ---- weights -------------------------------------------------------------------------------------------------
    def matrices(self):
        """(name, fmt, rows, cols, block_cols, flags, generator) for every matrix, in upload order; the generator
        draws the GGUF bytes from a stream seeded by (seed, matrix index), so each rank of a sharded run sees the
        same model."""
        s = self.s
        H, F, d = s.hidden, s.ffn, s.gdn_rows
        att, kvd = s.n_head * s.head_dim, s.n_kv_head * s.head_dim
        # members of one multi-output pass are told the pass's rows, so their panels make one wave of CTAs
        qkv_pass = UPLOAD_PASS_ROWS(2 * att + 2 * kvd)
        gdn_pass = UPLOAD_PASS_ROWS(4 * d + 2 * s.gdn_heads)
        out = [("tok_embd", Q4_0, s.vocab, H, 0, UPLOAD_REPLICATE)]
        for i in range(s.n_layers):
            if s.is_attn(i):
                out += [(f"{i}.wq_gate", Q4_0, 2 * att, H, 0, qkv_pass), (f"{i}.wk", Q4_0, kvd, H, 0, qkv_pass),
                        (f"{i}.wv", Q4_0, kvd, H, 0, qkv_pass), (f"{i}.wo", Q4_0, H, att, 0, 0)]
            else:
                out += [(f"{i}.wqkv", Q4_0, 3 * d, H, 0, gdn_pass), (f"{i}.wz", Q4_0, d, H, 0, gdn_pass),
                        (f"{i}.wbeta", Q4_0, s.gdn_heads, H, 0, gdn_pass),
                        (f"{i}.walpha", Q4_0, s.gdn_heads, H, 0, gdn_pass), (f"{i}.ssm_out", Q4_0, H, d, 256, 0)]
            out += [(f"{i}.gate", Q4_0, F, H, 0, 0), (f"{i}.up", Q4_0, F, H, 0, 0), (f"{i}.down", Q4_0, H, F, 0, 0)]
        for j, (r0, n) in enumerate(s.head_pieces()):
            out.append((f"output.{j}", Q6_K, n, H, 0, 0))
        return [(name, fmt, rows, cols, bc, fl, self._gen(k, fmt, rows, cols))
                for k, (name, fmt, rows, cols, bc, fl) in enumerate(out)]

    def _gen(self, k: int, fmt: int, rows: int, cols: int):
        return lambda: synth.matrix(fmt, np.random.default_rng([synth.SEED, 40, self.seed, k]), rows, cols)

    def upload(self, upload_fn, keep: dict | None = None) -> None:
        """upload_fn(gguf, rows, cols, fmt, block_cols, flags) -> handle. keep: filled {handle: (gguf, rows, cols,
        fmt)} for a checker."""
        for name, fmt, rows, cols, bc, fl, gen in self.matrices():
            g = gen()
            h = upload_fn(g, rows, cols, fmt, bc, fl)
            self.handles[name] = h
            if keep is not None:
                keep[h] = (g.reshape(-1), rows, cols, fmt)

    # ---- resident state ------------------------------------------------------------------------------------------
    def initial_act(self) -> np.ndarray:
        s, L = self.s, self.L
        r = np.random.default_rng([synth.SEED, 41, self.seed])
        act = np.zeros(L.size, np.float32)
        act[L.TOK] = np.array([self.first_token], np.uint32).view(np.float32)[0]
        act[L.ONORM:L.ONORM + s.hidden] = r.normal(1, 0.1, s.hidden)
        for i, p in enumerate(L.layer):
            for key in ("attn_norm", "ffn_norm"):
                act[p[key]:p[key] + s.hidden] = r.normal(1, 0.1, s.hidden)
            if s.is_attn(i):
                for key in ("q_norm", "k_norm"):
                    act[p[key]:p[key] + s.head_dim] = r.normal(1, 0.1, s.head_dim)
            else:
                ch = 3 * s.gdn_rows
                act[p["conv_w"]:p["conv_w"] + 4 * ch] = r.normal(0, 0.5, 4 * ch)
                act[p["conv_hist"]:p["conv_hist"] + 3 * ch] = r.normal(0, 1, 3 * ch)
                act[p["dt"]:p["dt"] + s.gdn_heads] = r.normal(0, 1, s.gdn_heads)
                act[p["a"]:p["a"] + s.gdn_heads] = -np.exp(r.normal(0, 0.5, s.gdn_heads))
                act[p["gdn_norm"]:p["gdn_norm"] + GDN_DIM] = r.normal(1, 0.1, GDN_DIM)
        return act

    def initial_state(self) -> np.ndarray:
        """DeltaNet state of every GDN layer, fp32 N(0, 0.1), rows of 128 floats (layer j at row j * gdn_rows)."""
        r = np.random.default_rng([synth.SEED, 42, self.seed])
        return r.normal(0, 0.1, self.s.n_gdn * self.s.gdn_rows * GDN_DIM).astype(np.float32)

    def initial_kv(self) -> np.ndarray:
        """F16 KV slots of the attention layers, positions below the prefill length N(0, 1), the rest zero."""
        s = self.s
        r = np.random.default_rng([synth.SEED, 43, self.seed])
        kv = np.zeros((s.n_attn, 2, s.n_kv_head, s.kv_ctx, s.head_dim), np.float16)
        kv[..., :s.prefill, :] = r.normal(0, 1, kv[..., :s.prefill, :].shape).astype(np.float16)
        return kv.view(np.uint16).reshape(-1)

    def record(self, pos: int) -> np.ndarray:
        """Host record of the token at position pos: the position (uint32 bits) and the NEOX RoPE cos/sin row
        (cs[2i], cs[2i+1] = cos, sin of pos * theta^(-2i / rope_dims))."""
        s = self.s
        rec = np.zeros(RECORD, np.float32)
        rec[0] = np.array([pos], np.uint32).view(np.float32)[0]
        i = np.arange(s.rope_dims // 2, dtype=np.float64)
        ang = pos * s.rope_theta ** (-2.0 * i / s.rope_dims)
        rec[16:16 + s.rope_dims:2] = np.cos(ang)
        rec[17:17 + s.rope_dims:2] = np.sin(ang)
        return rec

    # ---- command lists -------------------------------------------------------------------------------------------
    def _gdn_layer(self, i: int, j: int):
        s, L, h = self.s, self.L, self.handles
        H, d = s.hidden, s.gdn_rows
        p = L.layer[i]
        return [
            rmsnorm(H, L.X, p["attn_norm"], L.XN, s.eps, flags=NORM_DEFER),
            gemv(Q4_0, 3 * d, H, h[f"{i}.wqkv"], L.XN, L.QKV, GEMV_CONV),
            conv(3 * d, L.QKV, p["conv_w"], L.QKVC, p["conv_hist"], p["conv_hist"], True),
            gemv(Q4_0, d, H, h[f"{i}.wz"], L.XN, L.Z),
            gemv(Q4_0, s.gdn_heads, H, h[f"{i}.wbeta"], L.XN, L.BETA),
            gemv(Q4_0, s.gdn_heads, H, h[f"{i}.walpha"], L.XN, L.ALPHA),
            gdn(s.gdn_heads, s.gdn_heads, L.QKVC, L.QKVC + d, L.QKVC + 2 * d, L.ALPHA, L.BETA, L.Y,
                j * d, j * d, GDN_DIM ** -0.5, flags=GDN_L2_QK | GDN_GATED | GDN_GATES | GDN_WITH_OUT,
                l2_eps=s.eps, rms_eps=s.eps, w_off=p["gdn_norm"], z_off=L.Z, dt_off=p["dt"], a_off=p["a"]),
            gemv(Q4_0, H, d, h[f"{i}.ssm_out"], L.Y, L.OUT, GEMV_ADD), add(H, L.OUT, L.X, L.X),
        ] + self._ffn(i)

    def _attn_layer(self, i: int, slot: int):
        s, L, h = self.s, self.L, self.handles
        H, hd = s.hidden, s.head_dim
        att, kvd = s.n_head * hd, s.n_kv_head * hd
        p = L.layer[i]
        return [
            rmsnorm(H, L.X, p["attn_norm"], L.XN, s.eps, flags=NORM_DEFER),
            gemv(Q4_0, 2 * att, H, h[f"{i}.wq_gate"], L.XN, L.QG),
            gemv(Q4_0, kvd, H, h[f"{i}.wk"], L.XN, L.K),
            gemv(Q4_0, kvd, H, h[f"{i}.wv"], L.XN, L.V),
            rmsnorm(hd, L.QG, p["q_norm"], L.QN, s.eps, rows=s.n_head, stride_words=2 * hd // 16),
            rmsnorm(hd, L.K, p["k_norm"], L.KN, s.eps, rows=s.n_kv_head),
            rope(s.rope_dims, L.QN, L.CS, L.QR, hd, s.n_head),
            rope(s.rope_dims, L.KN, L.CS, L.KR, hd, s.n_kv_head),
            attn(s.n_head, s.n_kv_head, hd, L.QR, L.KR, L.V, L.YA, L.POS, slot),
            silu_mul(att, L.QG + hd, L.YA, L.YG, sigmoid=True, row=hd, stride=2 * hd),
            gemv(Q4_0, H, att, h[f"{i}.wo"], L.YG, L.OUT, GEMV_ADD), add(H, L.OUT, L.X, L.X),
        ] + self._ffn(i)

    def _ffn(self, i: int):
        s, L, h = self.s, self.L, self.handles
        H, F = s.hidden, s.ffn
        return [
            rmsnorm(H, L.X, L.layer[i]["ffn_norm"], L.XN, s.eps, flags=NORM_DEFER),
            gemv(Q4_0, F, H, h[f"{i}.gate"], L.XN, L.FF, GEMV_SWIGLU), gemv(Q4_0, F, H, h[f"{i}.up"], L.XN, L.FF),
            gemv(Q4_0, H, F, h[f"{i}.down"], L.FF, L.OUT, GEMV_ADD), add(H, L.OUT, L.X, L.X),
        ]

    def _head(self):
        s, L, h = self.s, self.L, self.handles
        H = s.hidden
        cmds = [rmsnorm(H, L.X, L.ONORM, L.XN, s.eps, flags=NORM_DEFER)]
        for j, (r0, n) in enumerate(s.head_pieces()):
            cmds.append(gemv(Q6_K, n, H, h[f"output.{j}"], L.XN, L.LOGITS + r0))
        cmds.append(argmax(s.vocab, L.LOGITS, L.TOK))
        return cmds

    def token_lists(self):
        """The lists of one token, each at most 128 commands, cut at layer boundaries."""
        s, L = self.s, self.L
        blocks = [[get_row(Q4_0, s.hidden, self.handles["tok_embd"], L.TOK, L.X)]]
        j = slot = 0
        for i in range(s.n_layers):
            if s.is_attn(i):
                blocks.append(self._attn_layer(i, slot))
                slot += 1
            else:
                blocks.append(self._gdn_layer(i, j))
                j += 1
        blocks.append(self._head())
        lists, cur = [], []
        for b in blocks:
            block = cmd_list(*b)
            if cur and sum(c.size for c in cur) + block.size > MAX_CMDS * CMD_WORDS:
                lists.append(cmd_list(*cur))
                cur = []
            cur.append(block)
        lists.append(cmd_list(*cur))
        return lists

    # ---- running on a context ------------------------------------------------------------------------------------
    def context_config(self, world: int = 1) -> dict:
        """Context arguments that fit this model on one rank of a world-way row-sharded run."""
        s = self.s
        from . import row_slice, weight_device_bytes
        wb = 0
        for name, fmt, rows, cols, bc, fl, _ in self.matrices():
            r0, r1 = row_slice(rows, world, 0, fl)
            fl_rank = (fl & 0xFF) | UPLOAD_PASS_ROWS((fl >> 8) * (r1 - r0) // rows)  # the hint as the upload scales it
            wb += (weight_device_bytes(r1 - r0, cols, fmt, fl_rank) + 255) // 256 * 256
        return dict(weight_bytes=wb + (64 << 20), act_floats=self.L.size, state_rows=s.n_gdn * s.gdn_rows,
                    kv_bytes=s.n_attn * s.kv_slot_bytes, kv_ctx=s.kv_ctx)

    def load(self, ctx, keep: dict | None = None) -> None:
        """Uploads the weights and writes act, the DeltaNet states and the KV cache."""
        self.upload(lambda g, rows, cols, fmt, bc, fl: ctx.upload(g, rows, cols, fmt, block_cols=bc, flags=fl), keep)
        self.load_resident(ctx)

    def load_gguf(self, ctx, gguf_file) -> None:
        """As load, with every matrix read from an open GGUF file (GgufFile) by name instead of generated: the
        library's reader hands the tensor's GGUF bytes from the file mapping straight to the upload."""
        for name, fmt, rows, cols, bc, fl, _ in self.matrices():
            t = gguf_file.tensor(gguf_file.find(name))
            if t["type"] != fmt or t["ne"][:2] != [cols, rows]:
                raise ValueError(f"GGUF tensor {name}: type {t['type']} shape {t['ne']}, expected {fmt} {[cols, rows]}")
            self.handles[name] = ctx.upload_gguf(gguf_file, name, block_cols=bc, flags=fl)
        self.load_resident(ctx)

    def load_resident(self, ctx) -> None:
        """Writes act (norm weights, conv kernels and histories, gates' parameters), the DeltaNet states and the KV
        cache."""
        ctx.write(0, self.initial_act())
        ctx.write_state(0, self.initial_state())
        ctx.write_kv(0, self.initial_kv())

