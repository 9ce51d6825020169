"""Verify calls in one launch (``B200Decoder.verify_fn`` -> ``owsm_dec_step_verify``): the decoder call on the
session's input rows, the argmax of every window position under ESPnet's timestamp rules and the drafted tokens
accepted, on every kernel (cluster, cluster row slices, dense, dense row slices, grid-stage).

The rule decisions and the accepted counts are integer work: they must equal the oracle's restatement of
``_Verify.predict`` / ``_Verify.accept`` (pinned to owsm-trt's own outputs in tests/test_oracle.py) applied to the
kernel's own logits, bit for bit. The logits must equal those of a plain ``step_fn`` call on the same tokens."""

import pytest
import torch

import cases
from oracle import decoder as ref
from owsm_trt_b200.synthetic import TEST_CFG, decoder_state_dict

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
C_CACHE, T_ENC = 64, 37


def _rules():
    rl = cases.VERIFY_RULES
    return ref.TimestampRules(rl["notime"], rl["first_time"], rl["last_time"], rl["eos"], rl["vocab"])


@pytest.fixture(scope="module")
def kern():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA GPU")
    from owsm_trt_b200.decoder import B200Decoder

    return B200Decoder.from_state_dict(decoder_state_dict(TEST_CFG, 0, True), TEST_CFG.H, DEV)


def _inputs(R, W, seed):
    d = TEST_CFG
    _, inp, notime = cases.verify_inputs(R, W, seed)
    g = torch.Generator().manual_seed(seed + 1000)
    kc = torch.randn(d.L, R, d.H, C_CACHE, d.dk, generator=g).half().to(DEV)
    vc = torch.randn(d.L, R, d.H, C_CACHE, d.dk, generator=g).half().to(DEV)
    ck = torch.randn(d.L, R, d.H, T_ENC, d.dk, generator=g).half().to(DEV)
    cv = torch.randn(d.L, R, d.H, T_ENC, d.dk, generator=g).half().to(DEV)
    return inp, notime, kc, vc, ck, cv


def _verify(k, inp, notime, kc, vc, ck, cv, rules=True, res=True):
    d = TEST_CFG
    R, W = inp.shape[0], inp.shape[1] - 4
    logits = torch.full((R, W, d.V), float("nan"), device=DEV)
    new_kv = torch.zeros(d.L, 2, R, d.H, W, d.dk, device=DEV, dtype=torch.float16)
    pred = torch.full((R, W), -1, dtype=torch.long, device=DEV)
    out = torch.full((R, 2), -7, dtype=torch.long, device=DEV) if res else None
    rl = cases.VERIFY_RULES
    run = k.verify_fn(inp.to(DEV), kc.clone(), vc.clone(), ck, cv, logits, new_kv, pred,
                      rules=(rl["first_time"], rl["last_time"], rl["eos"]) if rules else None,
                      notime=notime.to(DEV), res=out, eos=rl["eos"])  # fmt: skip
    assert run.writes_cache and run.writes_pred and run.reads_inp and run.writes_res == res
    run()
    torch.cuda.synchronize()
    k.check()
    return logits.cpu(), pred.cpu(), None if out is None else out.cpu(), run


def _agreeing_drafts(k, inp, notime, kc, vc, ck, cv):
    """Drafts that the decoder accepts in part: for two rows in three, token i + 1 is set to the argmax after
    position i (one call per position, since the argmax at i depends on the tokens up to i); the third row of
    each three keeps its random drafts."""
    R, W = inp.shape[0], inp.shape[1] - 4
    inp = inp.clone()
    for i in range(W - 1):
        _, pred, _, _ = _verify(k, inp, notime, kc, vc, ck, cv, res=False)
        for r in range(R):
            if r % 3 != 2:
                inp[r, i + 1] = pred[r, i]
    return inp


# (rows, window, seed, kernel) -- the kernel the shape selects by default, or the grid-stage kernel forced
SHAPES = [(3, 3, 41, "cluster"), (8, 1, 42, "cluster"), (5, 4, 43, "cluster"), (6, 8, 44, "dense"),
          (16, 3, 45, "dense"), (24, 4, 46, "dense"), (5, 4, 47, "grid")]  # fmt: skip


@pytest.mark.parametrize("R,W,seed,kernel", SHAPES)
def test_verify_rules_and_accept_exact(kern, R, W, seed, kernel):
    inp, notime, kc, vc, ck, cv = _inputs(R, W, seed)
    kern.set_path(1 if kernel == "grid" else 0)
    try:
        inp = _agreeing_drafts(kern, inp, notime, kc, vc, ck, cv)
        logits, pred, res, run = _verify(kern, inp, notime, kc, vc, ck, cv)
        assert kern.plan_kernel(run) == kernel
        assert bool(torch.isfinite(logits).all())
        rules = _rules()
        want = ref.verify_predict(logits, inp, notime, rules)
        assert torch.equal(pred, want), f"rule argmax differs at {(pred != want).nonzero().tolist()[:8]}"
        assert torch.equal(res, ref.verify_accept(pred, inp, rules.eos))
        # the same call with plain argmax, and as step_fn on the same tokens: identical logits
        logits2, pred2, _, _ = _verify(kern, inp, notime, kc, vc, ck, cv, rules=False, res=False)
        assert torch.equal(logits2, logits)
        assert torch.equal(pred2, ref.argmax_first(logits))
        d = TEST_CFG
        lg3 = torch.full((R, W, d.V), float("nan"), device=DEV)
        kv3 = torch.zeros(d.L, 2, R, d.H, W, d.dk, device=DEV, dtype=torch.float16)
        kern.step_fn(inp[:, :W].to(DEV), inp[:, W].contiguous().to(DEV), kc.clone(), vc.clone(), ck, cv, lg3, kv3)()
        torch.cuda.synchronize()
        assert torch.equal(lg3.cpu(), logits)
    finally:
        kern.set_path(0)


def test_verify_accepts_drafts(kern):
    """The agreeing drafts are accepted: every row whose drafts follow the argmax (and hold no <eos>) accepts all
    of them, and the fixture mix accepts between 0 and W - 1 drafts over the rows."""
    R, W = 9, 5
    inp, notime, kc, vc, ck, cv = _inputs(R, W, 48)
    inp = _agreeing_drafts(kern, inp, notime, kc, vc, ck, cv)
    _, pred, res, _ = _verify(kern, inp, notime, kc, vc, ck, cv)
    eos = cases.VERIFY_RULES["eos"]
    for r in range(R):
        s = max(int(inp[r, W + 3]), 0)
        if r % 3 != 2 and eos not in inp[r, s + 1 : W].tolist():
            assert int(res[r, 0]) == W - 1 - s, (r, res[r].tolist(), inp[r].tolist())
    assert int(res[:, 0].max()) >= 2


def test_verify_rejects_bad_buffers(kern):
    inp, notime, kc, vc, ck, cv = _inputs(2, 3, 49)
    d = TEST_CFG
    logits = torch.zeros(2, 3, d.V, device=DEV)
    new_kv = torch.zeros(d.L, 2, 2, d.H, 3, d.dk, device=DEV, dtype=torch.float16)
    pred = torch.zeros(2, 3, dtype=torch.long, device=DEV)
    with pytest.raises(ValueError):  # res without an <eos> id
        kern.verify_fn(inp.to(DEV), kc, vc, ck, cv, logits, new_kv, pred, res=torch.zeros(2, 2, dtype=torch.long,
                                                                                              device=DEV))  # fmt: skip
    with pytest.raises(ValueError):
        kern.verify_fn(inp.to(DEV), kc, vc, ck, cv, logits, new_kv, pred[:, :2].contiguous(), rules=(500, 900, 1))
    with pytest.raises(TypeError):
        kern.verify_fn(inp.to(DEV).int(), kc, vc, ck, cv, logits, new_kv, pred, rules=(500, 900, 1))
