"""b200q_quantize_noalloc: the activation quantizer for callers that hold no b200q context and may not allocate device
memory (a runtime whose device memory is all reserved by its own pool, or a diagnostic path after an allocation
failed). Checked through the C ABI against the context entry point b200q_debug_quantize and against the CPU oracle:
the same quants, scales and block sums, on two calls in a row with different inputs, for the three activation types
(Q8_0, Q8_1, Q8_K), with and without the deferred RMSNORM, up to B200Q_NOALLOC_MAX_N values, on the legacy default
stream and on a stream of the caller's. Pointers that are not device memory of the device, misaligned, or shorter than
n floats are refused on the host. Named to be collected last: it must pass alone and after the other GPU tests."""
import numpy as np
import pytest

from conftest import rng

pytestmark = pytest.mark.gpu

X_OFF, W_OFF = 0, 32768
EPS = 1e-6


def _oracle(orc, fmt, x, w):
    """Quants, scales (in the layout b200q returns) and block sums of the CPU restatement."""
    xn = orc.rownorm(x, w, x.size, 1, EPS, 0) if w is not None else x
    if fmt == 14:
        return orc.quantize_q8_k(xn)
    if fmt == 3:
        return orc.quantize_q8_1(xn)
    return orc.quantize_q8_0(xn)


def _check(got, want, what):
    for g, w, name in zip(got, want, ("quants", "scales", "block sums")):
        assert np.array_equal(np.asarray(g), np.asarray(w)), f"{what}: {name} differ"


@pytest.mark.parametrize("fmt,n", [(2, 2560), (3, 9216), (14, 2560), (3, 16384), (14, 16384), (2, 16384)])
@pytest.mark.parametrize("norm", [False, True])
def test_matches_the_context_quantizer_and_the_oracle_two_calls_in_a_row(ctx, b2, orc, synth, fmt, n, norm):
    for call in range(2):
        r = rng(60, fmt, n, int(norm), call)
        x = synth.activation(r, n) * (1.0 + call)
        w = r.normal(1, 0.1, n).astype(np.float32)
        ctx.write(X_OFF, x)
        ctx.write(W_OFF, w)
        base = ctx.act_ptr
        want = ctx.debug_quantize(fmt, X_OFF, n, W_OFF if norm else None, EPS, 0)
        got = b2.quantize_noalloc(0, base + 4 * X_OFF, n, fmt, base + 4 * W_OFF if norm else None, EPS, 0)
        _check(got, want, f"call {call} vs the context entry point")
        _check(got, _oracle(orc, fmt, x, w if norm else None), f"call {call} vs the oracle")


def test_on_a_stream_of_the_caller(ctx, b2, orc, synth):
    import torch
    s = torch.cuda.Stream(device=0)
    n = 4096
    for call in range(2):
        x = synth.activation(rng(61, call), n)
        ctx.write(X_OFF, x)
        got = b2.quantize_noalloc(0, ctx.act_ptr + 4 * X_OFF, n, 2, stream=s.cuda_stream)
        _check(got, _oracle(orc, 2, x, None), f"call {call} on a caller stream")


def test_rejects_more_than_the_fixed_scratch_holds(ctx, b2):
    with pytest.raises(b2.B200QError, match="B200Q_NOALLOC_MAX_N"):
        b2.quantize_noalloc(0, ctx.act_ptr, b2.NOALLOC_MAX_N + 32, 2)
    with pytest.raises(b2.B200QError, match="multiple of 256"):
        b2.quantize_noalloc(0, ctx.act_ptr, 2560 + 32, 14)


def test_rejects_pointers_that_are_not_n_device_floats(ctx, b2):
    host = np.zeros(2560, np.float32)
    with pytest.raises(b2.B200QError, match="not device memory"):
        b2.quantize_noalloc(0, host.ctypes.data, 2560, 2)
    with pytest.raises(b2.B200QError, match="norm_w is not device memory"):
        b2.quantize_noalloc(0, ctx.act_ptr, 2560, 2, host.ctypes.data, EPS, 0)
    with pytest.raises(b2.B200QError, match="4-byte aligned"):
        b2.quantize_noalloc(0, ctx.act_ptr + 2, 2560, 2)
    end = ctx.act_ptr + 4 * ctx.act_floats
    with pytest.raises(b2.B200QError, match="past the end"):
        b2.quantize_noalloc(0, end - 4 * 1024, 2560, 2)
    # a valid call afterwards still works (the refusals launched nothing)
    q, _, _ = b2.quantize_noalloc(0, ctx.act_ptr, 2560, 2)
    assert q.size == 2560
