"""The GPU kernels against the independent FP64 restatement (tests/fp64_ref.py) on the paths that no reference build
can pin: NEOX RoPE, the DeltaNet step with its input stage and gated norm, the conv1d, decode attention, and the
128-step config-3 recurrence. Same cases and tolerances as tests/test_fp64_independent.py, which holds the CPU
oracle to them (attention: 1e-5 of the weighted mean of |v|, the GPU kernel's FP32 scores and exponentials)."""
import numpy as np
import pytest

from conftest import rng
from test_fp64_independent import (GDN_OFF, RECURRENCE_MAG, RECURRENCE_REL, S, TOL, Config3Fp64, attn_case,
                                   config3_inputs, config3_list, conv_case, gdn_case, rope_case, run_config3_vs_fp64)

pytestmark = pytest.mark.gpu

ATTN_TOL = 1e-5


def _run(ctx, act, cl, state=None):
    ctx.write(0, act)
    if state is not None:
        ctx.write_state(0, state)
    assert ctx.run(cl) == 0, ctx.last_error()
    return ctx.read(0, act.size)


@pytest.mark.parametrize("pos", [0, 1, 517, 639])
def test_gpu_rope_vs_fp64(ctx, b2, pos):
    act, cl, (Y, y, mag) = rope_case(0, pos)
    got = _run(ctx, act, cl)
    err = np.abs(got[Y:Y + y.size] - y) / np.maximum(mag, 1e-30)
    assert err.max() <= TOL, err.max()


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("seed", [0, 1])
def test_gpu_gdn_step_input_stage_and_gated_norm_vs_fp64(ctx, b2, seed, gated):
    act, state, cl, (st, smag, y, ymag) = gdn_case(seed, gated)
    got = _run(ctx, act, cl, state)
    gs = ctx.read_state(0, state.size // S)
    es = np.abs(gs.reshape(-1, S) - st) / smag
    Y = GDN_OFF["Y"]
    ey = np.abs(got[Y:Y + y.size] - y) / ymag
    assert es.max() <= TOL and ey.max() <= TOL, (es.max(), ey.max())


def test_gpu_conv_vs_fp64(ctx, b2):
    act, cl, (Y, y, mag, SD, ns) = conv_case(0)
    got = _run(ctx, act, cl)
    assert (np.abs(got[Y:Y + y.size] - y) / mag).max() <= TOL
    assert np.array_equal(got[SD:SD + ns.size], ns.astype(np.float32))


@pytest.mark.parametrize("pos", [0, 31, 512])
def test_gpu_attention_vs_fp64(ctx, b2, pos):
    act, kv, cl, kv_ctx, (Y, y, mag) = attn_case(0, pos)
    assert kv_ctx == ctx.kv_ctx
    ctx.write_kv(0, kv)
    got = _run(ctx, act, cl)
    err = np.abs(got[Y:Y + y.size] - y) / mag
    print(f"attention at position {pos}: max error {err.max():.2e} of the weighted mean of |v|")
    assert err.max() <= ATTN_TOL, err.max()


def test_gpu_config3_128_steps_vs_fp64_recurrence(ctx, b2):
    r = rng(84)
    act = config3_inputs(r)
    state = r.normal(0, 0.1, 16 * S * S).astype(np.float32)
    ref = Config3Fp64(act, state)
    ctx.write(0, act)
    ctx.write_state(0, state)
    cl = config3_list(b2)

    def step():
        ctx.write(0, act[0:6144])
        ctx.write(55296, act[55296:55328])
        ctx.write(55360, act[55360:55360 + 2048])
        return ctx.run(cl) == 0

    worst = run_config3_vs_fp64(step, lambda: ctx.read_state(0, 16 * S), act, ref, r)
    print(f"GPU vs FP64, 128 steps: {worst}")
    assert worst["floored"] <= RECURRENCE_REL and worst["per_mag"] <= RECURRENCE_MAG
