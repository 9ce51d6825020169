"""The CPU oracle against the golden vectors owsm-trt itself produced (tests/golden/make_golden.py).

These pin the restatement in ``oracle/decoder.py`` before any CUDA result is compared with it."""

import numpy as np
import pytest
import torch

import cases
from oracle import decoder as ref
from owsm_trt_b200.synthetic import MEDIUM_1B, TEST_CFG, cross_kv, decoder_state_dict, sinusoidal_positions

GOLD = cases.__file__.rsplit("/", 1)[0]


@pytest.fixture(scope="module")
def sd():
    return decoder_state_dict(TEST_CFG, 0, True)


@pytest.mark.parametrize("name", list(cases.STEP_CASES))
def test_step_matches_reference(sd, name):
    d = TEST_CFG
    R, S, C, T, seed, enc_len = cases.STEP_CASES[name]
    tokens, offset, k, v, ck, cv = cases.step_inputs(d, R, S, C, T, seed)
    gold = np.load(f"{GOLD}/step_{name}.npz")
    el = None if enc_len is None else torch.tensor(enc_len, dtype=torch.int32)
    logits, new_kv = ref.decoder_step(sd, d.H, tokens, offset, k.float(), v.float(), ck.float(), cv.float(), enc_len=el)
    torch.testing.assert_close(logits, torch.from_numpy(gold["logits"]), rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(new_kv, torch.from_numpy(gold["new_kv"]), rtol=1e-4, atol=1e-5)


def test_cross_row_sharing_equals_duplication(sd):
    """cross_row (rows reading their utterance's K/V) == the reference layout that repeats K/V per row."""
    d = TEST_CFG
    tokens, offset, k, v, ck, cv = cases.step_inputs(d, 4, 1, 32, 20, 9)
    rows = torch.tensor([0, 0, 1, 1])
    a, akv = ref.decoder_step(sd, d.H, tokens, offset, k.float(), v.float(), ck[:, rows].float(), cv[:, rows].float())
    b, bkv = ref.decoder_step(sd, d.H, tokens, offset, k.float(), v.float(), ck[:, :2].float(), cv[:, :2].float(),
                              cross_row=rows)  # fmt: skip
    torch.testing.assert_close(a, b)
    torch.testing.assert_close(akv, bkv)


def test_beam_select_matches_reference():
    d = TEST_CFG
    logits, score, active, k0, v0 = cases.beam_inputs(d)
    gold = np.load(f"{GOLD}/beam.npz")
    B, K = cases.BEAM["B"], cases.BEAM["K"]
    top, parent, token = ref.beam_topk(logits, score, active, B, K)
    torch.testing.assert_close(top, torch.from_numpy(gold["score"]), rtol=1e-6, atol=1e-6)
    assert torch.equal(parent, torch.from_numpy(gold["parent"]))
    assert torch.equal(token, torch.from_numpy(gold["token"]))
    k = ref.reorder_cache(k0, parent)
    assert torch.equal(k[:, 3], k0[:, int(gold["parent"][3])])


def test_greedy_decode_matches_reference_session(sd):
    """Teacher-free greedy decoding with the oracle step == GreedySession.decode (TorchBackend, fp32)."""
    d = TEST_CFG
    G = cases.GREEDY
    ck, cv = cases.greedy_inputs(d)
    gold = np.load(f"{GOLD}/greedy.npz")["out"]
    B, C = G["B"], G["C"]
    primer = torch.tensor(G["primer"])
    p = primer.shape[1]
    k = torch.zeros(d.L, B, d.H, C, d.dk)
    v = torch.zeros(d.L, B, d.H, C, d.dk)
    logits, new_kv = ref.decoder_step(sd, d.H, primer, torch.zeros(B, dtype=torch.long), k, v, ck.float(), cv.float())
    ref.write_kv(new_kv, k, v, torch.zeros(B, dtype=torch.long))
    nxt = ref.argmax_first(logits[:, -1])
    outs = [[] for _ in range(B)]
    done = [False] * B
    pos = p
    for _ in range(G["steps"]):
        for b in range(B):
            if not done[b]:
                if int(nxt[b]) == G["eos"]:
                    done[b] = True
                else:
                    outs[b].append(int(nxt[b]))
        if all(done):
            break
        offs = torch.full((B,), pos, dtype=torch.long)
        logits, new_kv = ref.decoder_step(sd, d.H, nxt[:, None], offs, k, v, ck.float(), cv.float())
        ref.write_kv(new_kv, k, v, offs)
        nxt = ref.argmax_first(logits[:, -1])
        pos += 1
    for b in range(B):
        want = [t for t in gold[b] if t >= 0]
        assert outs[b] == want[: len(outs[b])] and len(outs[b]) == len(want)


@pytest.mark.slow
def test_medium_step_matches_reference():
    """One step of the 18-layer d=1024 decoder (plain weights, b1, T=750): top-32 logits and checksums."""
    d = MEDIUM_1B
    sd = decoder_state_dict(d, 0, False)
    tokens, offset, k, v, enc = cases.medium_inputs(d)
    kv = cross_kv(sd, d, enc).half()
    gold = np.load(f"{GOLD}/medium_step.npz")
    assert abs(float(kv.double().sum()) - float(gold["cross_sum"])) < 1e-3 * float(kv.double().abs().sum()) / kv.numel() ** 0.5 + 1.0
    logits, new_kv = ref.decoder_step(sd, d.H, tokens, offset, k.float(), v.float(), kv[:, 0].float(), kv[:, 1].float(),
                                      pe=sinusoidal_positions(64, d.D))  # fmt: skip
    lg = logits[0, 0]
    top = lg.topk(32)
    assert torch.equal(top.indices, torch.from_numpy(gold["top_idx"]))
    torch.testing.assert_close(top.values, torch.from_numpy(gold["top_val"]), rtol=1e-4, atol=1e-4)
    assert abs(float(lg.double().sum()) - float(gold["sum"])) < 1e-2
    assert abs(float((lg.double() ** 2).sum()) - float(gold["sumsq"])) < 1e-3 * float(gold["sumsq"])


def _verify_rules():
    rl = cases.VERIFY_RULES
    return ref.TimestampRules(rl["notime"], rl["first_time"], rl["last_time"], rl["eos"], rl["vocab"])


@pytest.mark.parametrize("name", list(cases.VERIFY_CASES))
def test_verify_predict_accept_match_reference(name):
    """_Verify.predict (timestamp rules per window position) and _Verify.accept, bit-exact."""
    R, W, seed = cases.VERIFY_CASES[name]
    logits, inp, notime = cases.verify_inputs(R, W, seed)
    gold = np.load(f"{GOLD}/verify.npz")
    rules = _verify_rules()
    pred = ref.verify_predict(logits, inp, notime, rules)
    assert torch.equal(pred, torch.from_numpy(gold[f"{name}_pred"]))
    assert torch.equal(ref.verify_accept(pred, inp, rules.eos), torch.from_numpy(gold[f"{name}_res"]))
    assert torch.equal(ref.verify_predict(logits, inp, notime, None), torch.from_numpy(gold[f"{name}_plain"]))


def test_verify_cases_cover_every_rule_branch():
    """The verify fixtures reach every branch of TimestampRules.forbidden that decides an argmax (no-time row,
    first position, open pair, after an end time, neither) and accepted counts of 0 and more."""
    rl = cases.VERIFY_RULES
    seen, accepted = set(), set()
    for R, W, seed in cases.VERIFY_CASES.values():
        logits, inp, notime = cases.verify_inputs(R, W, seed)
        for r in range(R):
            count, last = int(inp[r, W + 1]), int(inp[r, W + 2])
            for i in range(W):
                t = int(inp[r, i])
                if i > 0 and rl["first_time"] <= t <= rl["last_time"]:
                    count += 1
                prev_time = rl["first_time"] <= t <= rl["last_time"]
                if notime[r]:
                    seen.add("notime")
                elif int(inp[r, W + 3]) == i:
                    seen.add("first")
                elif count % 2 == 1:
                    seen.add("open")
                elif prev_time:
                    seen.add("after_end")
                else:
                    seen.add("closed")
        pred = ref.verify_predict(logits, inp, notime, _verify_rules())
        accepted |= set(ref.verify_accept(pred, inp, rl["eos"])[:, 0].tolist())
    assert seen == {"notime", "first", "open", "after_end", "closed"}
    assert 0 in accepted and max(accepted) >= 2
