"""Parity at the shapes and bounds of the north star, teacher-forced (oracle/parity.py), on the B200.

Every comparison is against the fp32 oracle (owsm-trt's ``Decoder.step`` semantics, src/owsm_trt/modeling.py:501-560,
pinned to the reference's own outputs by tests/test_oracle.py) on the same seeded weights (plain N(0, 0.02),
fp16-rounded) and encoder memory (N(0, 1) through the decoder's fp32 K/V projections; the kernel reads them in fp16).
Both decoders are fed the oracle's tokens at every step and keep their own caches.

Bounds, written here as the tests assert them:
  * logits max-abs <= 3e-2 over all V logits at every compared step (``parity.TOL``);
  * argmax bit-exact except where the oracle's top-two gap is below 1e-3 (near-ties, counted and printed);
  * beam: parents and tokens bit-exact against the oracle's selection on the kernel's own logits, and against the
    oracle's fp32 run except at near-ties (candidate gap < 1e-3, counted); scores within 1e-2.

Cases: (a) configs[0] 1B b1, 4-token prefix + 64 greedy steps; (b) configs[1] 1B b16, masked encoder lengths,
16 steps from cache position 140; (c) configs[2] 1B beam 5 x 3, 20 steps; (d) configs[3] the 6 x 768 model at
b1 (32 steps) and b64 (4 steps); (e) one 64-row call of the 1B model.
"""

from __future__ import annotations

import os

import pytest
import torch

from oracle import decoder as ref
from oracle import parity
from owsm_trt_b200.synthetic import MEDIUM_1B, SMALL, cross_kv, decoder_state_dict, sinusoidal_positions

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
DEV = torch.device("cuda")
T_ENC = 750
_MODELS: dict = {}


@pytest.fixture(scope="module", autouse=True)
def _all_threads():
    n = torch.get_num_threads()
    torch.set_num_threads(os.cpu_count() or 1)
    yield
    torch.set_num_threads(n)


def _model(d):
    """(state dict, kernel) of the plain seed-0 model of shape d, built once per session."""
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA GPU")
    if d not in _MODELS:
        from owsm_trt_b200.decoder import B200Decoder

        sd = decoder_state_dict(d, 0, False)
        _MODELS[d] = (sd, B200Decoder.from_state_dict(sd, d.H, DEV))
    return _MODELS[d]


def _encoder(sd, d, U: int, seed: int):
    """Cross K/V of U utterances of encoder memory N(0,1) [U, 750, D]: fp32 on the CPU (oracle), fp16 on the GPU."""
    g = torch.Generator().manual_seed(seed)
    enc = torch.randn(U, T_ENC, d.D, generator=g).to(DEV)
    sdd = {k: v.to(DEV) for k, v in sd.items() if ".src_attn.linear_k." in k or ".src_attn.linear_v." in k}
    with torch.no_grad():
        kv = cross_kv(sdd, d, enc)  # fp32 on the GPU (no TF32: torch's default for fp32 matmul)
    ck16, cv16 = kv[:, 0].half().contiguous(), kv[:, 1].half().contiguous()
    ck32, cv32 = kv[:, 0].cpu(), kv[:, 1].cpu()
    return ck32, cv32, ck16, cv16


class _Greedy:
    """The kernel's greedy call on its own fp16 cache, as parity.greedy's ``step``."""

    def __init__(self, k, d, R, C, ck16, cv16, enc_len, kc16=None, vc16=None):
        self.k, self.d, self.ck, self.cv = k, d, ck16, cv16
        self.kc = kc16 if kc16 is not None else torch.zeros(d.L, R, d.H, C, d.dk, device=DEV, dtype=torch.float16)
        self.vc = vc16 if vc16 is not None else torch.zeros_like(self.kc)
        self.el = None if enc_len is None else enc_len.to(torch.int32).to(DEV)
        self.kernels = set()

    def __call__(self, tok, off):
        d = self.d
        R, S = tok.shape
        logits = torch.full((R, S, d.V), float("nan"), device=DEV)
        new_kv = torch.zeros(d.L, 2, R, d.H, S, d.dk, device=DEV, dtype=torch.float16)
        pred = torch.full((R, S), -1, dtype=torch.long, device=DEV)
        run = self.k.step_fn(tok.to(DEV), off.to(DEV), self.kc, self.vc, self.ck, self.cv, logits, new_kv, pred=pred,
                             enc_len=self.el)  # fmt: skip
        run()
        torch.cuda.synchronize()
        self.k.check()
        self.kernels.add(self.k.plan_kernel(run))
        return logits.cpu(), pred.cpu()


def _report(name, tally, extra=None):
    s = tally.summary()
    if extra:
        s.update(extra)
    print(f"\nPARITY {name}: {s}")
    return s


def _assert(tally, name):
    assert tally.max_err <= parity.TOL, f"{name}: logits max-abs {tally.max_err} > {parity.TOL}"
    assert tally.mismatches == 0, f"{name}: argmax differs outside near-ties: {tally.summary()['mismatch_detail']}"


def test_a_1b_b1_64_teacher_forced_steps():
    """batch 1, a 4-token prefix U[0, V), 64 greedy steps, every step compared."""
    d = MEDIUM_1B
    sd, k = _model(d)
    ck32, cv32, ck16, cv16 = _encoder(sd, d, 1, 100)
    g = torch.Generator().manual_seed(101)
    prefix = torch.randint(0, d.V, (1, 4), generator=g)
    C = 72
    kc32 = torch.zeros(d.L, 1, d.H, C, d.dk)
    vc32 = torch.zeros_like(kc32)
    dut = _Greedy(k, d, 1, C, ck16, cv16, None)
    t = parity.greedy(dut, sd, d.H, prefix, torch.zeros(1, dtype=torch.long), ck32, cv32, None, 64, kc32, vc32,
                      sinusoidal_positions(C + 1, d.D))  # fmt: skip
    _report("1B b1 64 steps", t, {"kernels": sorted(dut.kernels)})
    assert t.steps == 4 + 64
    _assert(t, "1B b1")


def test_b_1b_b16_masked_from_position_140():
    """16 rows, encoder lengths U[300, 750] (key-padding mask), 140 cached positions (the oracle's
    prefill of random prefixes; the kernel's cache is its fp16 rounding), then 16 steps to position 155."""
    d = MEDIUM_1B
    sd, k = _model(d)
    R, C, P = 16, 160, 140
    ck32, cv32, ck16, cv16 = _encoder(sd, d, R, 200)
    g = torch.Generator().manual_seed(201)
    enc_len = torch.randint(300, T_ENC + 1, (R,), generator=g)
    prefix = torch.randint(0, d.V, (R, P), generator=g)
    pe = sinusoidal_positions(C + 1, d.D)
    kc32 = torch.zeros(d.L, R, d.H, C, d.dk)
    vc32 = torch.zeros_like(kc32)
    with torch.no_grad():
        lo, kvo = ref.decoder_step(sd, d.H, prefix, torch.zeros(R, dtype=torch.long), kc32, vc32, ck32, cv32,
                                   enc_len=enc_len, pe=pe)  # fmt: skip
        ref.write_kv(kvo, kc32, vc32, torch.zeros(R, dtype=torch.long))
    dut = _Greedy(k, d, R, C, ck16, cv16, enc_len, kc32.half().to(DEV), vc32.half().to(DEV))
    first = ref.argmax_first(lo[:, -1])[:, None]
    t = parity.greedy(dut, sd, d.H, first, torch.full((R,), P, dtype=torch.long), ck32, cv32, enc_len, 15, kc32,
                      vc32, pe)  # fmt: skip
    _report("1B b16 masked pos 140-155", t, {"kernels": sorted(dut.kernels)})
    assert t.steps == 16
    _assert(t, "1B b16")


def test_c_1b_beam_5x3_20_steps():
    """beam 5 over 3 utterances (15 rows, the utterance's cross K/V read once by its 5 hypotheses),
    4-token primers, the first selection on the prefill logits, then 20 fused beam steps (decoder call + log-softmax
    + top-5 of 5 x V + cache reorder), teacher-forced with the oracle's picks."""
    d = MEDIUM_1B
    sd, k = _model(d)
    B, K, P, C, steps = 3, 5, 4, 32, 20
    N = B * K
    ck32, cv32, ck16, cv16 = _encoder(sd, d, B, 300)
    g = torch.Generator().manual_seed(301)
    primer = torch.randint(0, d.V, (B, P), generator=g)
    pe = sinusoidal_positions(C + 1, d.D)
    rows = torch.arange(N) // K
    # prefill per utterance (oracle), copied to the 5 slots of each utterance (BeamSession.decode, runtime.py:1465-1472)
    kb = torch.zeros(d.L, B, d.H, C, d.dk)
    vb = torch.zeros_like(kb)
    with torch.no_grad():
        lo, kvo = ref.decoder_step(sd, d.H, primer, torch.zeros(B, dtype=torch.long), kb, vb, ck32, cv32, pe=pe)
    ref.write_kv(kvo, kb, vb, torch.zeros(B, dtype=torch.long))
    kc32, vc32 = kb[:, rows].clone(), vb[:, rows].clone()
    kc16, vc16 = kc32.half().to(DEV), vc32.half().to(DEV)
    score = torch.zeros(N)
    active = torch.zeros(N, dtype=torch.bool)
    active[::K] = True
    score, parent, token = ref.beam_topk(lo[:, -1][rows], score, active, B, K)
    active[:] = True
    tally = parity.Tally()
    score_err = 0.0
    for j in range(steps):
        off = torch.full((N,), P + j, dtype=torch.long)
        tok = token[:, None]
        with torch.no_grad():
            lo, kvo = ref.decoder_step(sd, d.H, tok, off, kc32, vc32, ck32, cv32, cross_row=rows, pe=pe)
        ref.write_kv(kvo, kc32, vc32, off)
        logp = torch.log_softmax(lo[:, 0].float(), -1)
        cand = (score[:, None] + logp).view(B, K * d.V)
        gap = parity.beam_gap(cand.sort(-1, descending=True).values, K)
        o_score, o_par, o_tok = ref.beam_topk(lo[:, 0], score, active, B, K)
        # the kernel's fused step on its own cache
        kc_pre, vc_pre = kc16.clone(), vc16.clone()
        logits = torch.zeros(N, 1, d.V, device=DEV)
        new_kv = torch.zeros(d.L, 2, N, d.H, 1, d.dk, device=DEV, dtype=torch.float16)
        sc = score.to(DEV).clone()
        par = torch.zeros(N, dtype=torch.long, device=DEV)
        tk = torch.zeros(N, dtype=torch.long, device=DEV)
        run = k.beam_fn(tok.to(DEV), off.to(DEV), kc16, vc16, ck16, cv16, logits, new_kv, sc,
                        active.to(torch.uint8).to(DEV), par, tk, beam=K)  # fmt: skip
        run()
        torch.cuda.synchronize()
        k.check()
        lg = logits[:, 0].cpu()
        # the fused select against the oracle's select on the kernel's own logits: exact
        s_own, p_own, t_own = ref.beam_topk(lg, score, active, B, K)
        assert torch.equal(par.cpu(), p_own) and torch.equal(tk.cpu(), t_own), f"step {j}: fused select"
        score_err = max(score_err, float((sc.cpu() - s_own).abs().max()))
        # against the fp32 oracle run
        err = float((lg - lo[:, 0]).abs().max())
        tally.errs.append(err)
        tally.max_err = max(tally.max_err, err)
        tally.steps += 1
        tally.rows += N
        same = (par.cpu() == o_par) & (tk.cpu() == o_tok)
        for b in range(B):
            ok = bool(same[b * K : (b + 1) * K].all())
            tie = float(gap[b]) < parity.TIE
            tally.near_ties += tie
            tally.tie_flips += tie and not ok
            if not ok and not tie:
                tally.mismatches += 1
                tally.mismatch_gaps.append((j, b, float(gap[b]), err))
        if not bool(same.all()):  # follow the oracle: the kernel's cache as the oracle's picks would have left it
            ref.write_kv(new_kv, kc_pre, vc_pre, off.to(DEV))
            kc16 = ref.reorder_cache(kc_pre, o_par.to(DEV)).contiguous()
            vc16 = ref.reorder_cache(vc_pre, o_par.to(DEV)).contiguous()
        kc32, vc32 = ref.reorder_cache(kc32, o_par), ref.reorder_cache(vc32, o_par)
        score, token = o_score, o_tok
    tally.score_err = score_err
    _report("1B beam 5x3 20 steps", tally, {"kernel": k.plan_kernel(run)})
    assert score_err <= parity.SCORE_TOL, score_err
    _assert(tally, "1B beam")


@pytest.mark.parametrize("R,steps", [(1, 32), (64, 4)])
def test_d_small_model(R, steps):
    """the 6-layer d=768, 12-head decoder at batch 1 and batch 64 (a 4-token prefix, then greedy
    steps), encoder memory 750 frames, every row compared."""
    d = SMALL
    sd, k = _model(d)
    ck32, cv32, ck16, cv16 = _encoder(sd, d, R, 400 + R)
    g = torch.Generator().manual_seed(401 + R)
    prefix = torch.randint(0, d.V, (R, 4), generator=g)
    C = 48
    kc32 = torch.zeros(d.L, R, d.H, C, d.dk)
    vc32 = torch.zeros_like(kc32)
    dut = _Greedy(k, d, R, C, ck16, cv16, None)
    t = parity.greedy(dut, sd, d.H, prefix[:, :1] if R > 16 else prefix, torch.zeros(R, dtype=torch.long), ck32,
                      cv32, None, steps, kc32, vc32, sinusoidal_positions(C + 1, d.D))  # fmt: skip
    _report(f"small b{R} {steps} steps", t, {"kernels": sorted(dut.kernels)})
    _assert(t, f"small b{R}")


def test_e_1b_64_rows_against_oracle():
    """One call of 64 one-token rows on the 1B model (the box-scale shard), masked lengths, cached positions
    up to 100 (random fp16 cache contents): logits, new K/V and argmax against the oracle."""
    d = MEDIUM_1B
    sd, k = _model(d)
    R, C = 64, 128
    ck32, cv32, ck16, cv16 = _encoder(sd, d, R, 500)
    g = torch.Generator().manual_seed(501)
    enc_len = torch.randint(300, T_ENC + 1, (R,), generator=g)
    tokens = torch.randint(0, d.V, (R, 1), generator=g)
    offset = torch.randint(0, 101, (R,), generator=g)
    kc = (torch.randn(d.L, R, d.H, C, d.dk, generator=g) * 0.5).half()
    vc = (torch.randn(d.L, R, d.H, C, d.dk, generator=g) * 0.5).half()
    with torch.no_grad():
        lo, kvo = ref.decoder_step(sd, d.H, tokens, offset, kc.float(), vc.float(), ck32, cv32, enc_len=enc_len,
                                   pe=sinusoidal_positions(C + 1, d.D))  # fmt: skip
    dut = _Greedy(k, d, R, C, ck16, cv16, enc_len, kc.to(DEV), vc.to(DEV))
    lg, pred = dut(tokens, offset)
    t = parity.Tally()
    t.add_greedy(lo[:, 0], lg[:, 0], pred[:, 0])
    _report("1B 64 rows", t, {"kernels": sorted(dut.kernels)})
    _assert(t, "1B 64 rows")
    assert torch.equal(pred[:, 0], ref.argmax_first(lg[:, 0]))
