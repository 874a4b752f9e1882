"""b200q_quantize_noalloc (the activation quantizer without a context and without device allocation) against the
context entry point b200q_debug_quantize: the same quants, scales and block sums, two calls in a row on different
inputs, for the three activation types (Q8_0, Q8_1, Q8_K), with and without the deferred RMSNORM. Named to be
collected last: it must pass alone and after the other GPU tests."""
import numpy as np
import pytest

from conftest import rng

pytestmark = pytest.mark.gpu

X_OFF, W_OFF = 0, 32768


@pytest.mark.parametrize("fmt", [2, 3, 14])
@pytest.mark.parametrize("norm", [False, True])
def test_matches_the_context_quantizer_two_calls_in_a_row(ctx, b2, synth, fmt, norm):
    n = 2560 if fmt != 3 else 9216
    for call in range(2):
        r = rng(60, fmt, int(norm), call)
        x = synth.activation(r, n) * (1.0 + call)
        ctx.write(X_OFF, x)
        ctx.write(W_OFF, r.normal(1, 0.1, n).astype(np.float32))
        base = ctx.act_ptr
        w_off = W_OFF if norm else None
        want = ctx.debug_quantize(fmt, X_OFF, n, w_off, 1e-6, 0)
        got = b2.quantize_noalloc(0, base + 4 * X_OFF, n, fmt, base + 4 * W_OFF if norm else None, 1e-6, 0)
        for g, w, what in zip(got, want, ("quants", "scales", "block sums")):
            assert np.array_equal(g, w), f"call {call}: {what} differ"


def test_rejects_more_than_the_fixed_scratch_holds(ctx, b2):
    with pytest.raises(b2.B200QError, match="B200Q_NOALLOC_MAX_N"):
        b2.quantize_noalloc(0, ctx.act_ptr, b2.NOALLOC_MAX_N + 32, 2)
    with pytest.raises(b2.B200QError, match="multiple of 256"):
        b2.quantize_noalloc(0, ctx.act_ptr, 2560 + 32, 14)
