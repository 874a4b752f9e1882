"""Second, independent restatement in FP64 numpy of the paths whose reference versions are HLS-only (they need Vitis
headers that are absent here, so no reference build can produce fixtures for them): NEOX RoPE, the Gated DeltaNet
step with its input stage (L2 of q / k, the gates) and gated output norm, the causal conv1d, and decode attention
over an F16 KV cache. Written from the formulas, not from oracle/oracle.c: every value is computed in float64 from
the float32 inputs, with no float32 rounding in between, so the CPU oracle and the GPU kernels (both float32) are
each compared with the exact arithmetic, and their agreement with each other does not rest on one shared author's
reading of the reference.

Formulas (reference file:line they are read from):
  RoPE NEOX (fpga/src/gemvqc_ops.h:275-312): for i < n_dims/2, x0 = x[i], x1 = x[i + n_dims/2], c = cs[2i],
      s = cs[2i + 1]: y[i] = x0 c - x1 s, y[i + n_dims/2] = x0 s + x1 c; floats from n_dims on are copied.
  GDN input stage (fpga/src/gemvqc_gdn.h:223-281): q, k L2-normalized per key head (x / max(||x||, eps));
      gates: beta = sigmoid(beta_raw), g = softplus(g_raw + dt) * a (softplus(v) = v for v > 20, else log(1 + e^v)).
  GDN step (gemvq_ref.h:360-397; ggml GATED_DELTA_NET, one token): value head h reads key head h % hk;
      S <- S e^g; delta = (v - S k) beta; S <- S + k (x) delta; y = (S q) scale, with state row j of head h holding
      column j of S (y[j] = sum_i S[j, i] q[i]).
  Gated output norm (fpga/src/gemvqc_gdn.h:283-346): per head y * (1 / sqrt(mean(y^2) + eps)) * w * silu(z).
  conv1d (gemvq_ref.h:344-358): window [state[3c], state[3c+1], state[3c+2], x[c]], y[c] = silu(sum_t win[t] w[4c+t]),
      new state = window[1..3].
  Decode attention (ggml's F16 attention path): scores = q . k / sqrt(head_dim) over positions 0..pos (k, v widened
      from F16), softmax, y = sum p v; GQA: query head h reads KV head h / (n_head / n_kv_head).
TEST INFRASTRUCTURE ONLY."""
from __future__ import annotations

import numpy as np


def rope_neox(x: np.ndarray, cs: np.ndarray, n_dims: int, ne0: int, rows: int):
    """(y, magnitude): y in FP64; magnitude |x0 c| + |x1 s| per rotated element (|x| for copied ones)."""
    x = np.asarray(x, np.float64).reshape(rows, ne0)
    c, s = np.asarray(cs, np.float64)[0:n_dims:2], np.asarray(cs, np.float64)[1:n_dims:2]
    half = n_dims // 2
    y, mag = x.copy(), np.abs(x)
    x0, x1 = x[:, :half], x[:, half:n_dims]
    y[:, :half] = x0 * c - x1 * s
    y[:, half:n_dims] = x0 * s + x1 * c
    mag[:, :half] = np.abs(x0 * c) + np.abs(x1 * s)
    mag[:, half:n_dims] = np.abs(x0 * s) + np.abs(x1 * c)
    return y.reshape(-1), mag.reshape(-1)


def softplus(v):
    v = np.asarray(v, np.float64)
    return np.where(v > 20.0, v, np.log1p(np.exp(np.minimum(v, 20.0))))


def sigmoid(v):
    return 1.0 / (1.0 + np.exp(-np.asarray(v, np.float64)))


def silu(v):
    v = np.asarray(v, np.float64)
    return v * sigmoid(v)


def l2_rows(x: np.ndarray, rows: int, eps: float) -> np.ndarray:
    x = np.asarray(x, np.float64).reshape(rows, -1)
    return (x / np.maximum(np.sqrt((x * x).sum(axis=1, keepdims=True)), eps)).reshape(-1)


def gdn_inputs(q, k, g_raw, beta_raw, hk: int, l2: bool, l2_eps: float, gates: bool, dt=None, a=None):
    """The step's q, k, g (log decay) and beta after the input stage, in FP64."""
    q, k = np.asarray(q, np.float64), np.asarray(k, np.float64)
    if l2:
        q, k = l2_rows(q, hk, l2_eps), l2_rows(k, hk, l2_eps)
    g, beta = np.asarray(g_raw, np.float64), np.asarray(beta_raw, np.float64)
    if gates:
        g = softplus(g + np.asarray(dt, np.float64)) * np.asarray(a, np.float64)
        beta = sigmoid(beta)
    return q, k, g, beta


def gdn_step(state: np.ndarray, q, k, v, g, beta, hv: int, hk: int, scale: float):
    """One DeltaNet step in FP64 on inputs after the input stage. state: [hv * 128 rows][128] (row j of head h holds
    column j of S). Returns (new state, y, state magnitude, y magnitude); the magnitudes are the FP64 sums of |terms|
    an FP32 computation rounds, the scale its errors are measured against."""
    S = 128
    st = np.asarray(state, np.float64).reshape(hv, S, S)
    q, k = np.asarray(q, np.float64).reshape(hk, S), np.asarray(k, np.float64).reshape(hk, S)
    v = np.asarray(v, np.float64).reshape(hv, S)
    out, y = np.empty_like(st), np.empty((hv, S))
    smag, ymag = np.empty_like(st), np.empty((hv, S))
    for h in range(hv):
        qh, kh = q[h % hk], k[h % hk]
        sd = st[h] * np.exp(g[h])
        dot = sd @ kh
        delta = (v[h] - dot) * beta[h]
        dmag = (np.abs(v[h]) + np.abs(sd) @ np.abs(kh)) * abs(beta[h])
        out[h] = sd + delta[:, None] * kh[None, :]
        smag[h] = np.abs(sd) + dmag[:, None] * np.abs(kh)[None, :]
        y[h] = (out[h] @ qh) * scale
        ymag[h] = (smag[h] @ np.abs(qh)) * scale
    return out.reshape(-1, S), y.reshape(-1), smag.reshape(-1, S), ymag.reshape(-1)


def gated_norm(y, z, w, hv: int, eps: float):
    """Per head y / sqrt(mean(y^2) + eps) * w * silu(z), FP64."""
    y = np.asarray(y, np.float64).reshape(hv, -1)
    scale = 1.0 / np.sqrt((y * y).mean(axis=1, keepdims=True) + eps)
    return (y * scale * np.asarray(w, np.float64)[None, :] * silu(np.asarray(z, np.float64).reshape(hv, -1))).reshape(-1)


def conv1d(state, x, w, ch: int, use_silu: bool = True):
    """(y, new state) of the causal conv1d, kernel 4, in FP64."""
    st = np.asarray(state, np.float64).reshape(ch, 3)
    win = np.concatenate([st, np.asarray(x, np.float64).reshape(ch, 1)], axis=1)
    y = (win * np.asarray(w, np.float64).reshape(ch, 4)).sum(axis=1)
    return (silu(y) if use_silu else y), win[:, 1:].reshape(-1)


def attention(q, kcache, vcache, n_head: int, n_kv: int, head_dim: int, n_past: int):
    """(y, magnitude) of decode attention over positions 0..n_past-1 of F16 caches [n_kv][ctx][head_dim]; magnitude =
    the softmax-weighted mean of |v| per output element."""
    kc = np.asarray(kcache).view(np.float16).astype(np.float64).reshape(n_kv, -1, head_dim)[:, :n_past]
    vc = np.asarray(vcache).view(np.float16).astype(np.float64).reshape(n_kv, -1, head_dim)[:, :n_past]
    q = np.asarray(q, np.float64).reshape(n_head, head_dim)
    group = n_head // n_kv
    y, mag = np.empty((n_head, head_dim)), np.empty((n_head, head_dim))
    for h in range(n_head):
        sc = kc[h // group] @ q[h] / np.sqrt(head_dim)
        p = np.exp(sc - sc.max())
        p /= p.sum()
        y[h] = p @ vc[h // group]
        mag[h] = p @ np.abs(vc[h // group])
    return y.reshape(-1), mag.reshape(-1)
