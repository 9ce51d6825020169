"""owsm_dec_step_static (fixed scratch, no device allocation) against owsm_dec_step (plan scratch), both
through the C ABI, on two decoder calls in a row: logits, argmax, new K/V and the written caches must be
bit-identical (same kernel, same schedule; only where the scratch lives differs). The file sorts last so it
also runs after every other GPU test has used the library; it needs nothing from them."""

import pytest
import torch

from owsm_trt_b200.synthetic import TEST_CFG, decoder_state_dict

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(scope="module")
def kern():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA GPU")
    from owsm_trt_b200.decoder import B200Decoder

    k = B200Decoder.from_state_dict(decoder_state_dict(TEST_CFG, 0, True), TEST_CFG.H, DEV)
    k.set_path(1)  # the fixed-scratch call is a variant of the grid-stage kernel's call: compare with that one
    return k


def _inputs(R, S, Cc, T, seed):
    d = TEST_CFG
    g = torch.Generator().manual_seed(seed)
    tokens = torch.randint(0, d.V, (R, S), generator=g).to(DEV)
    offset = torch.randint(0, Cc - 2 * S, (R,), generator=g).to(DEV)
    kc = (torch.randn(d.L, R, d.H, Cc, d.dk, generator=g) * 0.5).half().to(DEV)
    vc = (torch.randn(d.L, R, d.H, Cc, d.dk, generator=g) * 0.5).half().to(DEV)
    ck = (torch.randn(d.L, R, d.H, T, d.dk, generator=g) * 0.5).half().to(DEV)
    cv = (torch.randn(d.L, R, d.H, T, d.dk, generator=g) * 0.5).half().to(DEV)
    return tokens, offset, kc, vc, ck, cv


def _outputs(R, S):
    d = TEST_CFG
    logits = torch.full((R, S, d.V), float("nan"), device=DEV)
    new_kv = torch.zeros(d.L, 2, R, d.H, S, d.dk, device=DEV, dtype=torch.float16)
    pred = torch.full((R, S), -1, dtype=torch.long, device=DEV)
    return logits, new_kv, pred


def _two_calls(kern, R, S, Cc, T, static: bool, side_stream=None):
    """Two calls in a row: the second feeds the first's argmax at the next offsets, on the updated cache.
    side_stream: a torch.cuda.Stream (non-blocking against the legacy stream) to launch the calls on."""
    from owsm_trt_b200 import _lib

    lib = _lib.lib()
    tokens, offset, kc, vc, ck, cv = _inputs(R, S, Cc, T, 7)
    if side_stream is not None:
        side_stream.wait_stream(torch.cuda.current_stream(DEV))
    stream = (side_stream or torch.cuda.current_stream(DEV)).cuda_stream
    plan = None if static else kern._plan(R, S, Cc, T, 1, 0)
    outs = []
    for _ in range(2):
        logits, new_kv, pred = _outputs(R, S)
        ptrs = (tokens.data_ptr(), tokens.stride(0), offset.data_ptr(), offset.stride(0), kc.data_ptr(),
                vc.data_ptr(), ck.data_ptr(), cv.data_ptr(), None, logits.data_ptr(), new_kv.data_ptr(),
                pred.data_ptr(), None, 0, -1)  # fmt: skip
        if static:
            rc = lib.owsm_dec_step_static(kern._h, stream, R, S, Cc, T, *ptrs)
        else:
            rc = lib.owsm_dec_step(plan, stream, *ptrs)
        _lib.check(rc, "step")
        torch.cuda.synchronize()
        kern.check()
        outs.append((logits, new_kv, pred))
        tokens = pred[:, -1:].expand(R, S).contiguous()
        offset = offset + S
    return outs, kc, vc


def _same(ref, got):
    (ref, kc_ref, vc_ref), (got, kc_got, vc_got) = ref, got
    for (l0, n0, p0), (l1, n1, p1) in zip(ref, got):
        assert bool(torch.isfinite(l1).all())
        assert torch.equal(l0, l1)
        assert torch.equal(n0, n1)
        assert torch.equal(p0, p1)
    assert torch.equal(kc_ref, kc_got) and torch.equal(vc_ref, vc_got)


@pytest.mark.parametrize("R,S", [(1, 1), (2, 3), (8, 1)])
def test_static_scratch_call_equals_plan_call(kern, R, S):
    Cc, T = 32, 96
    _same(_two_calls(kern, R, S, Cc, T, static=False), _two_calls(kern, R, S, Cc, T, static=True))


def test_static_scratch_on_a_side_stream(kern):
    """The first fixed-scratch call of a new shape (its set-up) followed at once by launches on a non-blocking
    stream: the set-up's uploads must have landed before the kernel reads them."""
    Cc, T = 40, 80
    side = torch.cuda.Stream(DEV)
    ref = _two_calls(kern, 3, 2, Cc, T, static=False)
    got = _two_calls(kern, 3, 2, Cc, T, static=True, side_stream=side)
    torch.cuda.synchronize()
    _same(ref, got)


def test_static_scratch_alternating_shapes(kern):
    """One handle, shapes R = 2 then R = 1 then R = 2 again: each change re-lays the array out."""
    Cc, T = 32, 96
    ref = {R: _two_calls(kern, R, 1, Cc, T, static=False) for R in (2, 1)}
    for R in (2, 1, 2):
        _same(ref[R], _two_calls(kern, R, 1, Cc, T, static=True))


def test_static_scratch_rejects_oversize_calls(kern):
    """More than 8 tokens per call is refused with a message; nothing is launched."""
    from owsm_trt_b200 import _lib

    lib = _lib.lib()
    R, S, Cc, T = 3, 3, 32, 96
    tokens, offset, kc, vc, ck, cv = _inputs(R, S, Cc, T, 3)
    logits, new_kv, pred = _outputs(R, S)
    rc = lib.owsm_dec_step_static(kern._h, None, R, S, Cc, T, tokens.data_ptr(), tokens.stride(0),
                                  offset.data_ptr(), offset.stride(0), kc.data_ptr(), vc.data_ptr(), ck.data_ptr(),
                                  cv.data_ptr(), None, logits.data_ptr(), new_kv.data_ptr(), pred.data_ptr(), None,
                                  0, -1)  # fmt: skip
    assert rc == _lib.ERR_LIMIT
    assert b"at most 8 tokens" in lib.owsm_dec_last_error()
    assert bool(torch.isnan(logits).all())
