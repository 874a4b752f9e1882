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

from dataclasses import dataclass, replace

import numpy as np

from . import (CMD_WORDS, GDN_GATED, GDN_GATES, GDN_L2_QK, GDN_WITH_OUT, GEMV_ADD, GEMV_CONV, GEMV_SWIGLU, MAX_CMDS, NORM_DEFER,
               Q4_0, Q6_K, UPLOAD_PASS_ROWS, UPLOAD_REPLICATE, add, allgather, allreduce, argmax, attn, cmd_list, conv, gdn,
               gemv, get_row, gguf_row_bytes, rmsnorm, rope, silu_mul)
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


def local_shape(s: Shape, world: int) -> Shape:
    """The dimensions one rank of a world-way tensor-parallel run holds: DeltaNet heads, query heads, FFN rows and
    vocabulary rows divided by world (KV heads too, or one KV head shared by world / n_kv_head ranks); the hidden size
    and the full vocabulary (the gathered logits) stay."""
    if world == 1:
        return s
    ok = (s.gdn_heads % world == 0 and s.n_head % world == 0 and s.ffn % (128 * world) == 0 and
          s.vocab % (16 * world) == 0 and (s.n_kv_head % world == 0 or world % s.n_kv_head == 0) and
          (s.n_head // world) * s.head_dim % 128 == 0 and (s.gdn_heads // world) * GDN_DIM % 256 == 0)
    if not ok:
        raise ValueError(f"shape does not split over {world} ranks")
    return replace(s, ffn=s.ffn // world, gdn_heads=s.gdn_heads // world, n_head=s.n_head // world,
                   n_kv_head=max(1, s.n_kv_head // world))


def _rows(g: np.ndarray, rows: int, idx) -> np.ndarray:
    return g.reshape(rows, -1)[idx]


def _cols(g: np.ndarray, rows: int, cols: int, fmt: int, c0: int, c1: int) -> np.ndarray:
    """Columns [c0, c1) (multiples of 32) of a Q4_0 / Q8_0 / Q4_1 matrix: a byte range of every GGUF row."""
    bs = gguf_row_bytes(32, fmt)
    return np.ascontiguousarray(g.reshape(rows, cols // 32, bs)[:, c0 // 32:c1 // 32]).reshape(rows, -1)


class HybridDecoder:
    """The synthetic model: seeded weights and resident parameters, the per-token lists and host records.

    world > 1: rank `rank` of a tensor-parallel run (a context joined with COMM_EXPLICIT). The rank holds its own
    slices of the one model every rank generates from the same seeds: DeltaNet heads (their qkv / z / beta / alpha
    rows, conv channels and states), query heads and their KV heads (K / V rows and KV cache), FFN rows, and
    vocabulary rows of the head; the projections back to the hidden size (ssm_out, wo, down) are split by columns, so
    each rank produces a partial hidden vector, rank 0 adds the residual, and one ALLREDUCE per projection sums them
    into the residual stream (two per layer). The head's logits meet in one ALLGATHER before ARGMAX."""

    def __init__(self, shape: Shape = SHAPE_4B, seed: int = 4, first_token: int = 1, world: int = 1, rank: int = 0):
        self.s = shape
        self.seed = seed
        self.first_token = first_token
        self.world, self.rank = world, rank
        self.ls = local_shape(shape, world)
        self.L = ActLayout(self.ls)
        self.handles: dict = {}

    # ---- this rank's slices --------------------------------------------------------------------------------------
    def _gdn_heads(self):
        h = self.ls.gdn_heads
        return self.rank * h, (self.rank + 1) * h

    def _qkv_channels(self) -> np.ndarray:
        """Rows of the qkv projection (= conv channels) of this rank's DeltaNet heads: its q, k and v rows."""
        h0, h1 = self._gdn_heads()
        d = self.s.gdn_rows
        one = np.arange(h0 * GDN_DIM, h1 * GDN_DIM)
        return np.concatenate([one, d + one, 2 * d + one])

    def _kv_head0(self) -> int:
        """The first KV head of this rank's query heads."""
        return self.rank * self.ls.n_head // (self.s.n_head // self.s.n_kv_head)

    def head_pieces(self):
        """(first row within this rank's vocabulary slice, rows) of each head GEMV."""
        v_l = self.s.vocab // self.world
        out, r0 = [], 0
        while r0 < v_l:
            n = min(self.s.head_piece, v_l - r0)
            out.append((r0, n))
            r0 += n
        return out

    # ---- weights -------------------------------------------------------------------------------------------------
    def matrices(self):
        """(name, fmt, rows, cols, block_cols, flags, generator) for every matrix this rank uploads, in upload order;
        the generator draws the full matrix's GGUF bytes from a stream seeded by (seed, matrix index) and returns
        this rank's slice of it, so every rank holds slices of the same model."""
        s, ls, r = self.s, self.ls, self.rank
        H, F, d = s.hidden, s.ffn, s.gdn_rows
        att, kvd = s.n_head * s.head_dim, s.n_kv_head * s.head_dim
        att_l, kvd_l, d_l, F_l = ls.n_head * s.head_dim, ls.n_kv_head * s.head_dim, ls.gdn_rows, ls.ffn
        tp = self.world > 1
        # members of one multi-output pass are told the pass's rows, so their panels make one wave of CTAs
        qkv_pass = UPLOAD_PASS_ROWS(2 * att_l + 2 * kvd_l)
        gdn_pass = UPLOAD_PASS_ROWS(4 * d_l + 2 * ls.gdn_heads)
        h0, h1 = self._gdn_heads()
        q0 = r * att_l  # this rank's query heads start at q|gate row 2 q0 ([q; gate] row pairs per head)
        kv0 = self._kv_head0() * s.head_dim
        full = [("tok_embd", Q4_0, s.vocab, H, 0, UPLOAD_REPLICATE, None)]
        for i in range(s.n_layers):
            if s.is_attn(i):
                full += [(f"{i}.wq_gate", Q4_0, 2 * att, H, 0, qkv_pass, ("rows", slice(2 * q0, 2 * q0 + 2 * att_l))),
                         (f"{i}.wk", Q4_0, kvd, H, 0, qkv_pass, ("rows", slice(kv0, kv0 + kvd_l))),
                         (f"{i}.wv", Q4_0, kvd, H, 0, qkv_pass, ("rows", slice(kv0, kv0 + kvd_l))),
                         (f"{i}.wo", Q4_0, H, att, 0, 0, ("cols", r * att_l, (r + 1) * att_l))]
            else:
                full += [(f"{i}.wqkv", Q4_0, 3 * d, H, 0, gdn_pass, ("rows", self._qkv_channels())),
                         (f"{i}.wz", Q4_0, d, H, 0, gdn_pass, ("rows", slice(h0 * GDN_DIM, h1 * GDN_DIM))),
                         (f"{i}.wbeta", Q4_0, s.gdn_heads, H, 0, gdn_pass, ("rows", slice(h0, h1))),
                         (f"{i}.walpha", Q4_0, s.gdn_heads, H, 0, gdn_pass, ("rows", slice(h0, h1))),
                         (f"{i}.ssm_out", Q4_0, H, d, 256, 0, ("cols", h0 * GDN_DIM, h1 * GDN_DIM))]
            full += [(f"{i}.gate", Q4_0, F, H, 0, 0, ("rows", slice(r * F_l, (r + 1) * F_l))),
                     (f"{i}.up", Q4_0, F, H, 0, 0, ("rows", slice(r * F_l, (r + 1) * F_l))),
                     (f"{i}.down", Q4_0, H, F, 0, 0, ("cols", r * F_l, (r + 1) * F_l))]
        v0 = r * (s.vocab // self.world)
        full_pieces = [(v0 + a, n) for a, n in self.head_pieces()] if tp else s.head_pieces()
        for j, (a, n) in enumerate(full_pieces):
            full.append((f"output.{j}", Q6_K, n, H, 0, 0, ("head", a, n)))
        out = []
        for k, (name, fmt, rows, cols, bc, fl, cut) in enumerate(full):
            if name.startswith("output."):
                k = len(full)  # the head: one matrix [vocab x hidden], sliced into pieces
                rows_l, cols_l, gen = self._head_piece(cut[1], cut[2], cols)
            elif not tp or cut is None:
                rows_l, cols_l, gen = rows, cols, self._gen(k, fmt, rows, cols)
            elif cut[0] == "rows":
                rows_l = len(np.arange(rows)[cut[1]])
                cols_l, gen = cols, self._sliced(k, fmt, rows, cols, lambda g, rr=rows, c=cut[1]: _rows(g, rr, c))
            else:
                rows_l, cols_l = rows, cut[2] - cut[1]
                gen = self._sliced(k, fmt, rows, cols,
                                   lambda g, rr=rows, cc=cols, f=fmt, c=cut: _cols(g, rr, cc, f, c[1], c[2]))
            out.append((name, fmt, rows_l, cols_l, bc, fl, gen))
        return out

    def _gen(self, k: int, fmt: int, rows: int, cols: int):
        return lambda: synth.matrix(fmt, np.random.default_rng([synth.SEED, 40, self.seed, k]), rows, cols)

    def _sliced(self, k: int, fmt: int, rows: int, cols: int, cut):
        full = self._gen(k, fmt, rows, cols)
        return lambda: np.ascontiguousarray(cut(full()))

    def _head_piece(self, r0: int, n: int, cols: int):
        """Rows [r0, r0 + n) of the Q6_K head. Each piece of the one-rank model is generated on its own (seeded by its
        place in the upload order), so a rank's piece is cut from the one-rank pieces it overlaps."""
        pieces = self.s.head_pieces()
        n_before = 1 + self.s.n_layers * 3 + self.s.n_attn * 4 + self.s.n_gdn * 5  # matrices before the head

        def gen():
            parts = []
            for j, (a, m) in enumerate(pieces):
                lo, hi = max(a, r0), min(a + m, r0 + n)
                if lo < hi:
                    g = self._gen(n_before + j, Q6_K, m, cols)()
                    parts.append(g.reshape(m, -1)[lo - a:hi - a])
            return np.ascontiguousarray(np.concatenate(parts))
        return n, cols, gen

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
        """act of this rank: the norm weights (whole), and this rank's conv channels and gate parameters; drawn in the
        one-rank order from the full model's values."""
        s, L = self.s, self.L
        r = np.random.default_rng([synth.SEED, 41, self.seed])
        act = np.zeros(L.size, np.float32)
        act[L.TOK] = np.array([self.first_token], np.uint32).view(np.float32)[0]
        act[L.ONORM:L.ONORM + s.hidden] = r.normal(1, 0.1, s.hidden)
        ch_idx = self._qkv_channels() if self.world > 1 else slice(None)
        h0, h1 = self._gdn_heads()
        for i, p in enumerate(L.layer):
            for key in ("attn_norm", "ffn_norm"):
                act[p[key]:p[key] + s.hidden] = r.normal(1, 0.1, s.hidden)
            if s.is_attn(i):
                for key in ("q_norm", "k_norm"):
                    act[p[key]:p[key] + s.head_dim] = r.normal(1, 0.1, s.head_dim)
            else:
                ch = 3 * s.gdn_rows
                cw = r.normal(0, 0.5, 4 * ch).reshape(ch, 4)[ch_idx].reshape(-1)
                hist = r.normal(0, 1, 3 * ch).reshape(ch, 3)[ch_idx].reshape(-1)
                dt = r.normal(0, 1, s.gdn_heads)[h0:h1]
                a = -np.exp(r.normal(0, 0.5, s.gdn_heads))[h0:h1]
                act[p["conv_w"]:p["conv_w"] + cw.size] = cw
                act[p["conv_hist"]:p["conv_hist"] + hist.size] = hist
                act[p["dt"]:p["dt"] + dt.size] = dt
                act[p["a"]:p["a"] + a.size] = a
                act[p["gdn_norm"]:p["gdn_norm"] + GDN_DIM] = r.normal(1, 0.1, GDN_DIM)
        return act

    def initial_state(self) -> np.ndarray:
        """DeltaNet state of this rank's heads of every GDN layer, fp32 N(0, 0.1), rows of 128 floats (layer j at row
        j * local rows)."""
        r = np.random.default_rng([synth.SEED, 42, self.seed])
        st = r.normal(0, 0.1, self.s.n_gdn * self.s.gdn_rows * GDN_DIM).astype(np.float32)
        if self.world == 1:
            return st
        h0, h1 = self._gdn_heads()
        st = st.reshape(self.s.n_gdn, self.s.gdn_heads, GDN_DIM * GDN_DIM)[:, h0:h1]
        return np.ascontiguousarray(st).reshape(-1)

    def initial_kv(self) -> np.ndarray:
        """F16 KV slots of the attention layers (this rank's KV heads), positions below the prefill length N(0, 1),
        the rest zero."""
        s = self.s
        r = np.random.default_rng([synth.SEED, 43, self.seed])
        kv = np.zeros((s.n_attn, 2, s.n_kv_head, s.kv_ctx, s.head_dim), np.float16)
        kv[..., :s.prefill, :] = r.normal(0, 1, kv[..., :s.prefill, :].shape).astype(np.float16)
        if self.world > 1:
            k0 = self._kv_head0()
            kv = np.ascontiguousarray(kv[:, :, k0:k0 + self.ls.n_kv_head])
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
    def _project_out(self, fmt: int, cols: int, w: int, x_off: int, flags_extra=0):
        """The projection back to the hidden size with the residual: one rank adds it in the GEMV's epilogue
        (X += W x); tensor parallel: each rank's column slice gives a partial, rank 0 adds the residual, and one
        ALLREDUCE sums the partials into X."""
        s, L = self.s, self.L
        H = s.hidden
        if self.world == 1:
            return [gemv(fmt, H, cols, w, x_off, L.OUT, GEMV_ADD), add(H, L.OUT, L.X, L.X)]
        if self.rank == 0:
            head = [gemv(fmt, H, cols, w, x_off, L.OUT, GEMV_ADD), add(H, L.OUT, L.X, L.OUT)]
        else:
            head = [gemv(fmt, H, cols, w, x_off, L.OUT)]
        return head + [allreduce(H, L.OUT, L.X)]

    def _gdn_layer(self, i: int, j: int):
        s, ls, L, h = self.s, self.ls, self.L, self.handles
        H, d = s.hidden, ls.gdn_rows
        p = L.layer[i]
        return [
            rmsnorm(H, L.X, p["attn_norm"], L.XN, s.eps, flags=NORM_DEFER),
            gemv(Q4_0, 3 * d, H, h[f"{i}.wqkv"], L.XN, L.QKV, GEMV_CONV),
            conv(3 * d, L.QKV, p["conv_w"], L.QKVC, p["conv_hist"], p["conv_hist"], True),
            gemv(Q4_0, d, H, h[f"{i}.wz"], L.XN, L.Z),
            gemv(Q4_0, ls.gdn_heads, H, h[f"{i}.wbeta"], L.XN, L.BETA),
            gemv(Q4_0, ls.gdn_heads, H, h[f"{i}.walpha"], L.XN, L.ALPHA),
            gdn(ls.gdn_heads, ls.gdn_heads, L.QKVC, L.QKVC + d, L.QKVC + 2 * d, L.ALPHA, L.BETA, L.Y,
                j * d, j * d, GDN_DIM ** -0.5, flags=GDN_L2_QK | GDN_GATED | GDN_GATES | GDN_WITH_OUT,
                l2_eps=s.eps, rms_eps=s.eps, w_off=p["gdn_norm"], z_off=L.Z, dt_off=p["dt"], a_off=p["a"]),
        ] + self._project_out(Q4_0, d, h[f"{i}.ssm_out"], L.Y) + self._ffn(i)

    def _attn_layer(self, i: int, slot: int):
        s, ls, L, h = self.s, self.ls, self.L, self.handles
        H, hd = s.hidden, s.head_dim
        att, kvd = ls.n_head * hd, ls.n_kv_head * hd
        p = L.layer[i]
        return [
            rmsnorm(H, L.X, p["attn_norm"], L.XN, s.eps, flags=NORM_DEFER),
            gemv(Q4_0, 2 * att, H, h[f"{i}.wq_gate"], L.XN, L.QG),
            gemv(Q4_0, kvd, H, h[f"{i}.wk"], L.XN, L.K),
            gemv(Q4_0, kvd, H, h[f"{i}.wv"], L.XN, L.V),
            rmsnorm(hd, L.QG, p["q_norm"], L.QN, s.eps, rows=ls.n_head, stride_words=2 * hd // 16),
            rmsnorm(hd, L.K, p["k_norm"], L.KN, s.eps, rows=ls.n_kv_head),
            rope(s.rope_dims, L.QN, L.CS, L.QR, hd, ls.n_head),
            rope(s.rope_dims, L.KN, L.CS, L.KR, hd, ls.n_kv_head),
            attn(ls.n_head, ls.n_kv_head, hd, L.QR, L.KR, L.V, L.YA, L.POS, slot),
            silu_mul(att, L.QG + hd, L.YA, L.YG, sigmoid=True, row=hd, stride=2 * hd),
        ] + self._project_out(Q4_0, att, h[f"{i}.wo"], L.YG) + self._ffn(i)

    def _ffn(self, i: int):
        s, ls, L, h = self.s, self.ls, self.L, self.handles
        H, F = s.hidden, ls.ffn
        return [
            rmsnorm(H, L.X, L.layer[i]["ffn_norm"], L.XN, s.eps, flags=NORM_DEFER),
            gemv(Q4_0, F, H, h[f"{i}.gate"], L.XN, L.FF, GEMV_SWIGLU), gemv(Q4_0, F, H, h[f"{i}.up"], L.XN, L.FF),
        ] + self._project_out(Q4_0, F, h[f"{i}.down"], L.FF)

    def _head(self):
        s, L, h = self.s, self.L, self.handles
        H = s.hidden
        v_l = s.vocab // self.world
        base = L.LOGITS + self.rank * v_l  # this rank's vocabulary rows (all rows for one rank)
        pieces = self.head_pieces() if self.world > 1 else s.head_pieces()
        cmds = [rmsnorm(H, L.X, L.ONORM, L.XN, s.eps, flags=NORM_DEFER)]
        for j, (r0, n) in enumerate(pieces):
            cmds.append(gemv(Q6_K, n, H, h[f"output.{j}"], L.XN, base + r0))
        if self.world > 1:
            cmds.append(allgather(v_l, base, L.LOGITS))
        cmds.append(argmax(s.vocab, L.LOGITS, L.TOK))
        return cmds

    def _blocks(self):
        """The token's command blocks: the embedding row, one per layer, the head."""
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
        return [cmd_list(*b) for b in blocks]

    def list_ends(self):
        """Indices of the blocks that end a list: as many blocks per list as fit 128 commands. Tensor parallel, every
        rank cuts where rank 0 (whose blocks also hold the residual ADDs) cuts, so the ranks' lists hold the same
        collectives (a collective's slot is its place in its list)."""
        ref = self
        if self.world > 1 and self.rank != 0:
            import copy
            ref = copy.copy(self)
            ref.rank = 0
        ends, n = [], 0
        sizes = [b.size for b in ref._blocks()]
        for k, sz in enumerate(sizes):
            if n and n + sz > MAX_CMDS * CMD_WORDS:
                ends.append(k - 1)
                n = 0
            n += sz
        ends.append(len(sizes) - 1)
        return ends

    def token_lists(self):
        """The lists of one token, each at most 128 commands, cut at layer boundaries (list_ends)."""
        blocks, lists, start = self._blocks(), [], 0
        for e in self.list_ends():
            lists.append(cmd_list(*blocks[start:e + 1]))
            start = e + 1
        return lists

    # ---- the same token as an op graph, for the lowering -----------------------------------------------------------
    def token_graph(self):
        """One token as an op graph (graph.Graph) computing what token_lists computes, for b200q_lower to fuse and
        place: the embedding row, the layers (norms as RMS_NORM and MUL by the weight, the DeltaNet gates and gated
        norm as the ops they are made of, the attention q / gate rows as strided views), the head pieces writing into
        one logits buffer and ARGMAX writing the next token's id; tensor parallel (world > 1), this rank's slices with
        ALLREDUCE after each projection back to the hidden size and ALLGATHER of the logits. Returns (graph, names):
        names maps "rec", "tok", "logits", "onorm" and (layer, parameter) to the node ids of the INPUT / PARAM
        tensors."""
        from .graph import Graph
        from . import UNARY_SIGMOID, UNARY_SILU, UNARY_SOFTPLUS
        s, ls, h = self.s, self.ls, self.handles
        H, F, d, hd, hv = s.hidden, ls.ffn, ls.gdn_rows, s.head_dim, ls.gdn_heads
        att, kvd, nh, nkv = ls.n_head * hd, ls.n_kv_head * hd, ls.n_head, ls.n_kv_head
        g = Graph()
        names = {"rec": g.input(RECORD), "tok": g.input(16), "logits": g.input(s.vocab), "onorm": g.param(H)}
        pos, cs = g.view(names["rec"], 0, 16), g.view(names["rec"], 16, 128)
        ends = set(self.list_ends())  # blocks that end a list: 0 the embedding row, 1 + i layer i, then the head
        x = g.get_rows(names["tok"], h["tok_embd"], Q4_0, H)
        g.end_list() if 0 in ends else g.end_segment()

        def param(i, key, n):
            names[(i, key)] = g.param(n)
            return names[(i, key)]

        def project_out(i, yy, cols, name, x):
            part = g.mul_mat(yy, h[f"{i}.{name}"], Q4_0, H, cols)
            if self.world == 1:
                return g.add(part, x)
            return g.allreduce(g.add(part, x) if self.rank == 0 else part)

        j = slot = 0
        for i in range(s.n_layers):
            xn = g.mul(g.rms_norm(x, s.eps), param(i, "attn_norm", H))
            if s.is_attn(i):
                qg = g.mul_mat(xn, h[f"{i}.wq_gate"], Q4_0, 2 * att, H)
                kk = g.mul_mat(xn, h[f"{i}.wk"], Q4_0, kvd, H)
                vv = g.mul_mat(xn, h[f"{i}.wv"], Q4_0, kvd, H)
                qn = g.mul(g.rms_norm(g.view(qg, 0, hd, 2 * hd, nh), s.eps, rows=nh), param(i, "q_norm", hd))
                kn = g.mul(g.rms_norm(kk, s.eps, rows=nkv), param(i, "k_norm", hd))
                qr = g.rope(qn, cs, s.rope_dims, hd, nh)
                kr = g.rope(kn, cs, s.rope_dims, hd, nkv)
                ya = g.attn(qr, kr, vv, pos, nh, nkv, hd, slot)
                yg = g.mul(ya, g.unary(g.view(qg, hd, hd, 2 * hd, nh), UNARY_SIGMOID))
                x = project_out(i, yg, att, "wo", x)
                slot += 1
            else:
                qkv = g.mul_mat(xn, h[f"{i}.wqkv"], Q4_0, 3 * d, H)
                qkvc = g.conv(qkv, param(i, "conv_w", 4 * 3 * d), param(i, "conv_hist", 3 * 3 * d))
                z = g.mul_mat(xn, h[f"{i}.wz"], Q4_0, d, H)
                beta_raw = g.mul_mat(xn, h[f"{i}.wbeta"], Q4_0, hv, H)
                alpha_raw = g.mul_mat(xn, h[f"{i}.walpha"], Q4_0, hv, H)
                q = g.l2_norm(g.view(qkvc, 0, d), s.eps, rows=hv)
                k = g.l2_norm(g.view(qkvc, d, d), s.eps, rows=hv)
                gate = g.mul(g.unary(g.add(alpha_raw, param(i, "dt", hv)), UNARY_SOFTPLUS), param(i, "a", hv))
                y = g.gdn(q, k, g.view(qkvc, 2 * d, d), gate, g.unary(beta_raw, UNARY_SIGMOID), hv, hv, j * d,
                          GDN_DIM ** -0.5)
                yn = g.mul(g.mul(g.rms_norm(y, s.eps, rows=hv), param(i, "gdn_norm", GDN_DIM)), g.unary(z, UNARY_SILU))
                x = project_out(i, yn, d, "ssm_out", x)
                j += 1
            xn = g.mul(g.rms_norm(x, s.eps), param(i, "ffn_norm", H))
            ff = g.swiglu(g.mul_mat(xn, h[f"{i}.gate"], Q4_0, F, H), g.mul_mat(xn, h[f"{i}.up"], Q4_0, F, H))
            x = project_out(i, ff, F, "down", x)
            g.end_list() if 1 + i in ends else g.end_segment()
        xn = g.mul(g.rms_norm(x, s.eps), names["onorm"])
        v_l = s.vocab // self.world
        base = self.rank * v_l  # this rank's vocabulary rows (all rows for one rank)
        pieces = self.head_pieces() if self.world > 1 else s.head_pieces()
        for jj, (r0, n) in enumerate(pieces):
            g.mul_mat(xn, h[f"output.{jj}"], Q6_K, n, H, dst=g.view(names["logits"], base + r0, n))
        if self.world > 1:
            g.allgather(g.view(names["logits"], base, v_l), self.world, dst=names["logits"])
        g.argmax(names["logits"], dst=names["tok"])
        g.end_list()
        return g, names

    def graph_act(self, names, low) -> np.ndarray:
        """act for lowered lists: the resident values of initial_act() at the lowering's offsets."""
        L, a0 = self.L, self.initial_act()
        act = np.zeros(low.act_floats, np.float32)
        act[low.offset(names["tok"]):low.offset(names["tok"]) + 16] = a0[L.TOK:L.TOK + 16]
        act[low.offset(names["onorm"]):low.offset(names["onorm"]) + self.s.hidden] = a0[L.ONORM:L.ONORM + self.s.hidden]
        for key, node in names.items():
            if isinstance(key, tuple):
                i, name = key
                src = L.layer[i][name]
                n = low.offset(node), self._param_len(name)
                act[n[0]:n[0] + n[1]] = a0[src:src + n[1]]
        return act

    def _param_len(self, name: str) -> int:
        s = self.ls
        return {"attn_norm": s.hidden, "ffn_norm": s.hidden, "q_norm": s.head_dim, "k_norm": s.head_dim,
                "conv_w": 4 * 3 * s.gdn_rows, "conv_hist": 3 * 3 * s.gdn_rows, "dt": s.gdn_heads, "a": s.gdn_heads,
                "gdn_norm": GDN_DIM}[name]

    # ---- running on a context ------------------------------------------------------------------------------------
    def context_config(self, world: int = 1) -> dict:
        """Context arguments that fit this model on one rank: of a world-way row-sharded run (the library shards
        the one-rank model's uploads), or of this tensor-parallel rank (its own slices)."""
        s, ls = self.s, self.ls
        from . import row_slice, weight_device_bytes
        wb = 0
        for name, fmt, rows, cols, bc, fl, _ in self.matrices():
            r0, r1 = row_slice(rows, world, 0, fl) if self.world == 1 else (0, rows)
            fl_rank = (fl & 0xFF) | UPLOAD_PASS_ROWS((fl >> 8) * (r1 - r0) // rows)  # the hint as the upload scales it
            wb += (weight_device_bytes(r1 - r0, cols, fmt, fl_rank) + 255) // 256 * 256
        return dict(weight_bytes=wb + (64 << 20), act_floats=self.L.size, state_rows=s.n_gdn * ls.gdn_rows,
                    kv_bytes=s.n_attn * ls.kv_slot_bytes, kv_ctx=s.kv_ctx)

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

