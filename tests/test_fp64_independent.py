"""The CPU oracle against a second, independent FP64 restatement (tests/fp64_ref.py) on the paths no reference build
can pin (their reference code is HLS-only): NEOX RoPE, the DeltaNet input stage (L2 of q / k, gates), step and gated
output norm, the conv1d, and decode attention, on the config-3 / config-4 shapes. The GPU kernels are checked against
the same FP64 restatement in tests/test_gpu_fp64.py, with these case builders.

Tolerance: every FP32 result within 1e-6 of its FP64 term magnitude (the sum of the absolute values of the terms the
FP32 arithmetic rounds, e.g. |x0 c| + |x1 s| for a rotated pair), single steps from identical FP32 inputs. The
128-step DeltaNet recurrence, where each side feeds its own rounded state forward, is held to 1e-4 relative error with
a 1e-3 floor (1% of the state's initial standard deviation) and 1e-3 of the step's term magnitude; the unfloored
relative error is printed beside them."""
import numpy as np
import pytest

import fp64_ref as F
from conftest import rng

S = 128
TOL = 1e-6


def rope_case(seed: int, pos: int, n_head: int = 16, head_dim: int = 256, n_dims: int = 64, theta: float = 1e7):
    """act with q rows at 0 and the cos/sin row at CS; command list; expected (y, mag) at Y."""
    import fpga_llama_gguf_b200 as b2
    r = rng(80, seed, pos)
    CS, Y = n_head * head_dim, n_head * head_dim + 128
    act = np.zeros(Y + n_head * head_dim + 16, np.float32)
    act[:n_head * head_dim] = r.normal(0, 1, n_head * head_dim)
    ang = pos * theta ** (-2.0 * np.arange(n_dims // 2) / n_dims)
    act[CS:CS + n_dims:2], act[CS + 1:CS + n_dims:2] = np.cos(ang), np.sin(ang)
    cl = b2.cmd_list(b2.rope(n_dims, 0, CS, Y, head_dim, n_head))
    y, mag = F.rope_neox(act[:n_head * head_dim], act[CS:CS + n_dims], n_dims, head_dim, n_head)
    return act, cl, (Y, y, mag)


GDN_OFF = dict(Q=0, K=2048, V=4096, G=6144, B=6160, DT=6176, A=6192, Z=6208, WN=8256, Y=8384)


def gdn_case(seed: int, gated: bool, hv: int = 16, hk: int = 16):
    """One DeltaNet step with L2 q / k and gates from raw projections (and the gated norm): act, state, list, and the
    FP64 expectation (state, state mag, y, y mag) from the same FP32 inputs."""
    import fpga_llama_gguf_b200 as b2
    o = GDN_OFF
    r = rng(81, seed, int(gated))
    state = r.normal(0, 0.1, hv * S * S).astype(np.float32)
    act = np.zeros(16384, np.float32)
    act[o["Q"]:o["Q"] + hk * S] = r.normal(0, 1, hk * S)
    act[o["K"]:o["K"] + hk * S] = r.normal(0, 1, hk * S)
    act[o["V"]:o["V"] + hv * S] = r.normal(0, 1, hv * S)
    act[o["G"]:o["G"] + hv] = r.normal(0, 1, hv)
    act[o["B"]:o["B"] + hv] = r.normal(0, 1, hv)
    act[o["DT"]:o["DT"] + hv] = r.normal(0, 1, hv)
    act[o["A"]:o["A"] + hv] = -np.exp(r.normal(0, 0.5, hv))
    act[o["Z"]:o["Z"] + hv * S] = r.normal(0, 1, hv * S)
    act[o["WN"]:o["WN"] + S] = r.normal(1, 0.1, S)
    flags = b2.GDN_L2_QK | b2.GDN_GATES | (b2.GDN_GATED if gated else 0)
    cl = b2.gdn(hv, hk, o["Q"], o["K"], o["V"], o["G"], o["B"], o["Y"], 0, 0, S ** -0.5, flags=flags, w_off=o["WN"],
                z_off=o["Z"], dt_off=o["DT"], a_off=o["A"])
    q, k, g, beta = F.gdn_inputs(act[o["Q"]:o["Q"] + hk * S], act[o["K"]:o["K"] + hk * S], act[o["G"]:o["G"] + hv],
                                 act[o["B"]:o["B"] + hv], hk, True, 1e-6, True, act[o["DT"]:o["DT"] + hv],
                                 act[o["A"]:o["A"] + hv])
    st, y, smag, ymag = F.gdn_step(state, q, k, act[o["V"]:o["V"] + hv * S], g, beta, hv, hk, S ** -0.5)
    if gated:
        z, w = act[o["Z"]:o["Z"] + hv * S], act[o["WN"]:o["WN"] + S]
        yg = F.gated_norm(y, z, w, hv, 1e-6)
        yr = y.reshape(hv, S)
        sc = 1.0 / np.sqrt((yr * yr).mean(axis=1, keepdims=True) + 1e-6)
        gmag = (ymag.reshape(hv, S) * sc * np.abs(w)[None, :] *
                np.abs(F.silu(z.astype(np.float64))).reshape(hv, S)).reshape(-1) + np.abs(yg)
        y, ymag = yg, gmag
    return act, state, cl, (st, smag, y, ymag)


def conv_case(seed: int, ch: int = 6144):
    import fpga_llama_gguf_b200 as b2
    r = rng(82, seed)
    X, W, SS, Y, SD = 0, ch, 5 * ch, 8 * ch, 9 * ch
    act = np.zeros(12 * ch, np.float32)
    act[X:X + ch] = r.normal(0, 1, ch)
    act[W:W + 4 * ch] = r.normal(0, 0.5, 4 * ch)
    act[SS:SS + 3 * ch] = r.normal(0, 1, 3 * ch)
    cl = b2.cmd_list(b2.conv(ch, X, W, Y, SS, SD, True))
    y, new_state = F.conv1d(act[SS:SS + 3 * ch], act[X:X + ch], act[W:W + 4 * ch], ch)
    win = np.concatenate([act[SS:SS + 3 * ch].reshape(ch, 3), act[X:X + ch].reshape(ch, 1)], axis=1)
    pre_mag = (np.abs(win.astype(np.float64)) * np.abs(act[W:W + 4 * ch].reshape(ch, 4))).sum(axis=1)
    # silu(s) = s sigmoid(s): an error e in the sum moves the output by at most ~1.1 e
    return act, cl, (Y, y, 1.1 * pre_mag + np.abs(y), SD, new_state)


def attn_case(seed: int, pos: int, nh: int = 16, nkv: int = 4, hd: int = 256, kv_ctx: int = 640):
    """ATTN at position pos of a prefilled F16 slot: act, kv, list, and the FP64 expectation after this token's k / v
    row is stored."""
    import fpga_llama_gguf_b200 as b2
    r = rng(83, seed, pos)
    Q, K, V, Y, POS = 0, nh * hd, nh * hd + nkv * hd, nh * hd + 2 * nkv * hd, 2 * nh * hd + 2 * nkv * hd
    act = np.zeros(POS + 16, np.float32)
    act[Q:Q + nh * hd] = r.normal(0, 1, nh * hd)
    act[K:K + nkv * hd] = r.normal(0, 1, nkv * hd)
    act[V:V + nkv * hd] = r.normal(0, 1, nkv * hd)
    act[POS] = np.array([pos], np.uint32).view(np.float32)[0]
    pre = r.normal(0, 1, (2, nkv, kv_ctx, hd)).astype(np.float16)
    pre[:, :, pos:, :] = 0
    kv = pre.view(np.uint16).reshape(-1).copy()
    cl = b2.cmd_list(b2.attn(nh, nkv, hd, Q, K, V, Y, POS, 0))
    after = pre.copy()
    after[0, :, pos] = act[K:K + nkv * hd].reshape(nkv, hd).astype(np.float16)
    after[1, :, pos] = act[V:V + nkv * hd].reshape(nkv, hd).astype(np.float16)
    y, mag = F.attention(act[Q:Q + nh * hd], after[0].view(np.uint16), after[1].view(np.uint16), nh, nkv, hd, pos + 1)
    return act, kv, cl, kv_ctx, (Y, y, mag)


def config3_inputs(r, hv: int = 16):
    """The fixed part of the config-3 act (conv kernel and state, gates' dt / a, norm weight)."""
    act = np.zeros(65536, np.float32)
    act[6144:6144 + 4 * 6144] = r.normal(0, 0.5, 4 * 6144)
    act[30720:30720 + 3 * 6144] = r.normal(0, 1, 3 * 6144)
    act[55328:55328 + hv] = r.normal(0, 1, hv)
    act[55344:55344 + hv] = -np.exp(r.normal(0, 0.5, hv))
    act[57408:57408 + 128] = r.normal(1, 0.1, 128)
    return act


def config3_list(b2, hv: int = 16):
    """conv1d over the qkv input, then the DeltaNet step with every option but WITH_OUT."""
    return b2.cmd_list(
        b2.conv(6144, 0, 6144, 49152, 30720, 30720, True),
        b2.gdn(hv, hv, 49152, 49152 + 2048, 49152 + 4096, 55296, 55312, 57536, 0, 0, S ** -0.5,
               flags=b2.GDN_L2_QK | b2.GDN_GATED | b2.GDN_GATES, w_off=57408, z_off=55360, dt_off=55328, a_off=55344))


class Config3Fp64:
    """The FP64 recurrence of the config-3 step (conv1d state and DeltaNet state carried in FP64)."""

    def __init__(self, act, state, hv: int = 16):
        self.hv = hv
        self.cs = act[30720:30720 + 3 * 6144].astype(np.float64)
        self.st = state.astype(np.float64).reshape(-1, S)
        self.cw, self.dt, self.a, self.wn = (act[o:o + n].copy() for o, n in ((6144, 4 * 6144), (55328, hv),
                                                                             (55344, hv), (57408, 128)))

    def step(self, x, gb, z):
        hv = self.hv
        c, self.cs = F.conv1d(self.cs, x, self.cw, 6144)
        q, k, g, beta = F.gdn_inputs(c[:2048], c[2048:4096], gb[:hv], gb[hv:2 * hv], hv, True, 1e-6, True, self.dt,
                                     self.a)
        self.st, y, self.smag, _ = F.gdn_step(self.st, q, k, c[4096:6144], g, beta, hv, hv, S ** -0.5)
        return F.gated_norm(y, z, self.wn, hv, 1e-6)


def config3_step_inputs(r):
    return r.normal(0, 1, 6144).astype(np.float32), r.normal(0, 1, 32).astype(np.float32), \
        r.normal(0, 1, 2048).astype(np.float32)


def set_step_inputs(act, x, gb, z):
    act[0:6144], act[55296:55328], act[55360:55360 + 2048] = x, gb, z


# ---- the oracle against the FP64 restatement ------------------------------------------------------------------------
@pytest.mark.parametrize("pos", [0, 1, 517, 639])
def test_oracle_rope_vs_fp64(orc, b2, pos):
    act, cl, (Y, y, mag) = rope_case(0, pos)
    assert orc.run_list(act, cl, {}) == 0
    err = np.abs(act[Y:Y + y.size] - y) / np.maximum(mag, 1e-30)
    assert err.max() <= TOL, err.max()


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_gdn_step_input_stage_and_gated_norm_vs_fp64(orc, b2, seed, gated):
    act, state, cl, (st, smag, y, ymag) = gdn_case(seed, gated)
    assert orc.run_list(act, cl, {}, state=state) == 0
    es = np.abs(state.reshape(-1, S) - st) / smag
    Y = GDN_OFF["Y"]
    ey = np.abs(act[Y:Y + y.size] - y) / ymag
    assert es.max() <= TOL and ey.max() <= TOL, (es.max(), ey.max())


def test_oracle_conv_vs_fp64(orc, b2):
    act, cl, (Y, y, mag, SD, ns) = conv_case(0)
    assert orc.run_list(act, cl, {}) == 0
    assert (np.abs(act[Y:Y + y.size] - y) / mag).max() <= TOL
    assert np.array_equal(act[SD:SD + ns.size], ns.astype(np.float32))


@pytest.mark.parametrize("pos", [0, 31, 512])
def test_oracle_attention_vs_fp64(orc, b2, pos):
    act, kv, cl, kv_ctx, (Y, y, mag) = attn_case(0, pos)
    assert orc.run_list(act, cl, {}, kv=kv, kv_ctx=kv_ctx) == 0
    err = np.abs(act[Y:Y + y.size] - y) / mag
    assert err.max() <= TOL, err.max()


def test_oracle_config3_128_steps_vs_fp64_recurrence(orc, b2):
    r = rng(84)
    act = config3_inputs(r)
    state = r.normal(0, 0.1, 16 * S * S).astype(np.float32)
    ref = Config3Fp64(act, state)
    cl = config3_list(b2)
    worst = run_config3_vs_fp64(lambda: orc.run_list(act, cl, {}, state=state) == 0, lambda: state, act, ref, r)
    print(f"oracle vs FP64, 128 steps: {worst}")
    assert worst["floored"] <= RECURRENCE_REL and worst["per_mag"] <= RECURRENCE_MAG


def run_config3_vs_fp64(run_step, read_state, act, ref, r, steps: int = 128):
    """Runs `steps` config-3 steps through run_step (after writing the step's inputs into act) and the FP64
    recurrence; returns the worst state errors: per FP64 term magnitude of the step, relative with a 1e-3 floor
    (1% of the state's initial standard deviation), and relative without a floor."""
    worst = {"per_mag": 0.0, "floored": 0.0, "unfloored": 0.0}
    for step in range(steps):
        x, gb, z = config3_step_inputs(r)
        set_step_inputs(act, x, gb, z)
        assert run_step()
        ref.step(x, gb, z)
        if step % 16 == 15 or step == 0:
            d = np.abs(read_state().reshape(-1, S) - ref.st)
            worst["per_mag"] = max(worst["per_mag"], float((d / ref.smag).max()))
            worst["floored"] = max(worst["floored"], float((d / np.maximum(np.abs(ref.st), 1e-3)).max()))
            worst["unfloored"] = max(worst["unfloored"], float((d / np.abs(ref.st)).max()))
    return worst


# the recurrence: each side feeds its own rounded state forward for 128 steps
RECURRENCE_REL = 1e-4   # relative, floor 1e-3
RECURRENCE_MAG = 1e-3   # per FP64 term magnitude of the step
