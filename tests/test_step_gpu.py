"""The CUDA decoder call (libowsmdec.so through the C ABI) against the CPU oracle and owsm-trt's golden vectors.

Tolerances follow owsm-trt's own kernel tests (tests/test_megakernel.py:76-85): logits max-abs < 0.02 x
max|ref| on the perturbed test model (its output weight is scaled x8), new K/V assert_close(atol 0.05,
rtol 0.02), and the cache after the in-kernel write bit-equal to a scatter of new_kv. On the plain-weight
1B-shaped model the north-star bound applies: logits max-abs 3e-2 against the fp32 reference. Argmax is
bit-exact against the kernel's own logits and equal to the reference's except at near-ties (top-2 gap < 1e-3).
"""

import numpy as np
import pytest
import torch

import cases
from oracle import decoder as ref
from owsm_trt_b200.synthetic import SMALL, TEST_CFG, TEST_CFG384, decoder_state_dict, sinusoidal_positions

pytestmark = pytest.mark.gpu
GOLD = cases.__file__.rsplit("/", 1)[0]
DEV = torch.device("cuda")


def _gpu():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA GPU")


@pytest.fixture(scope="module")
def sd():
    return decoder_state_dict(TEST_CFG, 0, True)


@pytest.fixture(scope="module")
def kern(sd):
    _gpu()
    from owsm_trt_b200.decoder import B200Decoder

    return B200Decoder.from_state_dict(sd, TEST_CFG.H, DEV)


def _run_step(k, d, tokens, offset, kc, vc, ck, cv, enc_len=None, rows_per_utt=1, pred=True, notime=None):
    R, S = tokens.shape
    logits = torch.full((R, S, d.V), float("nan"), device=DEV)
    new_kv = torch.zeros(d.L, 2, R, d.H, S, d.dk, device=DEV, dtype=torch.float16)
    kc2, vc2 = kc.clone(), vc.clone()
    p = torch.full((R, S), -1, dtype=torch.long, device=DEV) if pred else None
    el = None if enc_len is None else torch.tensor(enc_len, dtype=torch.int32, device=DEV)
    run = k.step_fn(tokens.to(DEV), offset.to(DEV), kc2, vc2, ck.to(DEV), cv.to(DEV), logits, new_kv, pred=p,
                    notime=notime, enc_len=el, rows_per_utt=rows_per_utt)  # fmt: skip
    assert run.writes_cache and run.writes_pred == pred
    run()
    torch.cuda.synchronize()
    k.check()
    return logits, new_kv, kc2, vc2, p


def _check_cache(kc, vc, kc2, vc2, new_kv, offset):
    k, v = kc.clone(), vc.clone()
    ref.write_kv(new_kv, k, v, offset.to(DEV))
    assert torch.equal(kc2, k) and torch.equal(vc2, v)  # the new keys/values at each row's offset, nothing else


def _argmax_ok(logits_ref, logits, pred):
    """pred == argmax of our logits (bit-exact); == the reference's except at its near-ties."""
    assert torch.equal(pred.cpu(), ref.argmax_first(logits.cpu()))
    top2 = logits_ref.topk(2, dim=-1).values
    tie = (top2[..., 0] - top2[..., 1]) < 1e-3
    agree = pred.cpu() == logits_ref.argmax(-1)
    assert bool((agree | tie).all()), f"argmax differs outside near-ties: {(~agree & ~tie).sum()}"


@pytest.mark.parametrize("name", list(cases.STEP_CASES))
def test_step_matches_golden(kern, name):
    d = TEST_CFG
    R, S, C, T, seed, enc_len = cases.STEP_CASES[name]
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, S, C, T, seed)
    gold = np.load(f"{GOLD}/step_{name}.npz")
    kcd, vcd = kc.to(DEV), vc.to(DEV)
    logits, new_kv, kc2, vc2, pred = _run_step(kern, d, tokens, offset, kcd, vcd, ck, cv, enc_len=enc_len)
    gl = torch.from_numpy(gold["logits"])
    err = (logits.cpu() - gl).abs().max().item()
    assert err < 0.02 * gl.abs().max().item(), err
    torch.testing.assert_close(new_kv.float().cpu(), torch.from_numpy(gold["new_kv"]), atol=0.05, rtol=0.02)
    _check_cache(kcd, vcd, kc2, vc2, new_kv, offset)
    _argmax_ok(gl, logits, pred)


def test_step_is_deterministic(kern):
    """Two calls on the same inputs give bitwise the same logits (fixed reduction orders)."""
    d = TEST_CFG
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, 4, 1, 64, 37, 401)
    a = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv)
    b = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_rows_per_utt_equals_duplicated_cross(kern, sd):
    """Rows reading their utterance's cross K/V once (rows_per_utt) == owsm-trt's layout duplicating it."""
    d = TEST_CFG
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, 6, 1, 32, 41, 17)
    u = torch.tensor([0, 0, 0, 1, 1, 1])
    dup = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck[:, u], cv[:, u])
    shared = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck[:, :2], cv[:, :2], rows_per_utt=3)
    # the two layouts split the frames differently over the CTAs: same sums, other rounding
    assert (shared[0] - dup[0]).abs().max().item() < 2e-3 * dup[0].abs().max().item()
    lo, _ = ref.decoder_step(sd, d.H, tokens, offset, kc.float(), vc.float(), ck[:, :2].float(), cv[:, :2].float(),
                             cross_row=u)  # fmt: skip
    assert (shared[0].cpu() - lo).abs().max().item() < 0.02 * lo.abs().max().item()


@pytest.mark.parametrize("R,S", [(1, 1), (2, 5), (1, 16), (8, 8), (64, 1), (16, 4), (1, 32), (2, 32)])
def test_step_shapes_match_oracle(kern, sd, R, S):
    """Rows x window shapes up to the kernel's 64 tokens, against the oracle (reference: test_step_matches_decoder)."""
    d = TEST_CFG
    C, T = 64, 37
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, S, C, T, 1000 + R * 10 + S)
    lo, kvo = ref.decoder_step(sd, d.H, tokens, offset, kc.float(), vc.float(), ck.float(), cv.float())
    logits, new_kv, kc2, vc2, pred = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv)
    assert (logits.cpu() - lo).abs().max().item() < 0.02 * lo.abs().max().item()
    torch.testing.assert_close(new_kv.float().cpu(), kvo, atol=0.05, rtol=0.02)
    _check_cache(kc.to(DEV), vc.to(DEV), kc2, vc2, new_kv, offset)
    _argmax_ok(lo, logits, pred)


@pytest.mark.parametrize("R,S", [(1, 1), (16, 1), (2, 5), (32, 1), (8, 8)])
def test_kernel_choice_and_agreement(sd, R, S):
    """Calls of up to 16 tokens run on the cluster kernel, up to 32 as row slices of it, more on the dense kernel;
    that kernel and the grid-stage kernel agree on the same call (logits and new K/V within the oracle
    tolerances)."""
    _gpu()
    from owsm_trt_b200.decoder import B200Decoder

    d = TEST_CFG
    C, T = 64, 37
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, S, C, T, 77 + R * 10 + S)
    outs = {}
    for path in (0, 1):
        k = B200Decoder.from_state_dict(sd, d.H, DEV)
        k.set_path(path)
        logits = torch.zeros(R, S, d.V, device=DEV)
        new_kv = torch.zeros(d.L, 2, R, d.H, S, d.dk, device=DEV, dtype=torch.float16)
        kc2, vc2 = kc.clone().to(DEV), vc.clone().to(DEV)
        pred = torch.zeros(R, S, dtype=torch.long, device=DEV)
        run = k.step_fn(tokens.to(DEV), offset.to(DEV), kc2, vc2, ck.to(DEV), cv.to(DEV), logits, new_kv, pred=pred)
        run()
        torch.cuda.synchronize()
        k.check()
        outs[path] = (k.plan_kernel(run), logits.cpu(), new_kv.float().cpu())
        k.close()
    assert outs[0][0] == ("dense" if R * S > 32 else "cluster") and outs[1][0] == "grid"
    lg0, lg1 = outs[0][1], outs[1][1]
    assert (lg0 - lg1).abs().max().item() < 0.02 * lg1.abs().max().item()
    torch.testing.assert_close(outs[0][2], outs[1][2], atol=0.05, rtol=0.02)


def test_masked_lengths_match_oracle(kern, sd):
    """Per-utterance enc_len (key-padding mask) == the oracle's masked cross-attention, several lengths."""
    d = TEST_CFG
    R, C, T = 5, 64, 300
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, 1, C, T, 55)
    lens = [300, 1, 17, 150, 299]
    lo, _ = ref.decoder_step(sd, d.H, tokens, offset, kc.float(), vc.float(), ck.float(), cv.float(),
                             enc_len=torch.tensor(lens))  # fmt: skip
    logits = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv, enc_len=lens)[0]
    assert (logits.cpu() - lo).abs().max().item() < 0.02 * lo.abs().max().item()


@pytest.mark.parametrize("masked", [False, True])
def test_wide_steps_match_oracle(kern, sd, masked):
    """32 one-token rows over 300 encoder frames: with 4 heads the cluster kernel gives each cross-attention
    unit a whole utterance, so units of 256 frames or more take the wide (32-position) steps and shorter
    masked ones the 8-position steps, both within the oracle tolerance."""
    d = TEST_CFG
    R, C, T = 32, 64, 300
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, 1, C, T, 66)
    lens = [300, 256, 299, 255, 1, 40, 280, 150] * 4 if masked else None
    el = None if lens is None else torch.tensor(lens)
    lo, _ = ref.decoder_step(sd, d.H, tokens, offset, kc.float(), vc.float(), ck.float(), cv.float(), enc_len=el)
    logits, _, _, _, pred = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv, enc_len=lens)
    assert (logits.cpu() - lo).abs().max().item() < 0.02 * lo.abs().max().item()
    assert torch.equal(pred.cpu(), ref.argmax_first(logits.cpu()))


def test_argmax_without_timestamps(kern):
    """Rows flagged <notimestamps> get the argmax over the other ids (megakernel_ring's NOTIME)."""
    d = TEST_CFG
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, 2, 4, 64, 37, 11)
    flags = torch.tensor([True, False], device=DEV)
    ft, lt = 500, 990
    logits, _, _, _, pred = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv, notime=(flags, ft, lt))
    want = ref.argmax_notime(logits.cpu(), flags.cpu(), ft, lt)
    assert torch.equal(pred.cpu(), want)


def test_non_power_of_two_width():
    """d=384, 6 heads (owsm_v4 base/small widths are not powers of 2)."""
    _gpu()
    from owsm_trt_b200.decoder import B200Decoder

    d = TEST_CFG384
    sd = decoder_state_dict(d, 3, True)
    k = B200Decoder.from_state_dict(sd, d.H, DEV)
    for R, S in ((1, 1), (3, 2)):
        tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, S, 32, 29, 7 + R)
        lo, _ = ref.decoder_step(sd, d.H, tokens, offset, kc.float(), vc.float(), ck.float(), cv.float())
        logits = _run_step(k, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv)[0]
        assert (logits.cpu() - lo).abs().max().item() < 0.02 * lo.abs().max().item()


def test_greedy_decode_matches_reference_session(kern, sd):
    """Greedy decoding with the kernel's fused argmax == GreedySession.decode with TorchBackend (fp32)."""
    d = TEST_CFG
    G = cases.GREEDY
    ck, cv = (t.to(DEV) for t in cases.greedy_inputs(d))
    gold = np.load(f"{GOLD}/greedy.npz")["out"]
    B, Cc = G["B"], G["C"]
    primer = torch.tensor(G["primer"], device=DEV)
    p = primer.shape[1]
    kc = torch.zeros(d.L, B, d.H, Cc, d.dk, device=DEV, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    logits = torch.zeros(B, p, d.V, device=DEV)
    new_kv = torch.zeros(d.L, 2, B, d.H, p, d.dk, device=DEV, dtype=torch.float16)
    pred = torch.zeros(B, p, dtype=torch.long, device=DEV)
    zero = torch.zeros(B, dtype=torch.long, device=DEV)
    kern.step_fn(primer, zero, kc, vc, ck, cv, logits, new_kv, pred=pred)()  # prefill in the kernel too
    tok = torch.zeros(B, 1, dtype=torch.long, device=DEV)
    offs = torch.zeros(B, dtype=torch.long, device=DEV)
    lg1 = torch.zeros(B, 1, d.V, device=DEV)
    kv1 = torch.zeros(d.L, 2, B, d.H, 1, d.dk, device=DEV, dtype=torch.float16)
    pr1 = torch.zeros(B, 1, dtype=torch.long, device=DEV)
    run = kern.step_fn(tok, offs, kc, vc, ck, cv, lg1, kv1, pred=pr1)
    nxt = pred[:, -1].clone()
    outs = [[] for _ in range(B)]
    done = [False] * B
    for i in range(G["steps"]):
        for b in range(B):
            if not done[b]:
                if int(nxt[b]) == G["eos"]:
                    done[b] = True
                else:
                    outs[b].append(int(nxt[b]))
        if all(done):
            break
        tok[:, 0] = nxt
        offs.fill_(p + i)
        run()
        nxt = pr1[:, 0].clone()
    torch.cuda.synchronize()
    kern.check()
    for b in range(B):
        want = [t for t in gold[b] if t >= 0]
        assert outs[b] == want


@pytest.mark.parametrize("path", [0, 1])
def test_beam_step_matches_oracle(kern, path):
    """Fused beam step: parents/tokens bit-exact vs BeamSession._select step 1 (oracle) on the kernel's own
    logits, scores within 1e-2, the cache rows replaced by their parents' (bit-exact); on the cluster kernel
    (path 0) and the grid-stage kernel (path 1)."""
    kern.set_path(path)
    try:
        _beam_step_case(kern, "cluster" if path == 0 else "grid")
    finally:
        kern.set_path(0)


def _beam_step_case(kern, kernel):
    d = TEST_CFG
    B, K, C, T = 3, 5, 32, 37
    N = B * K
    g = torch.Generator().manual_seed(21)
    tokens = torch.randint(0, d.V, (N, 1), generator=g)
    offset = torch.full((N,), 9, dtype=torch.long)
    kc = torch.randn(d.L, N, d.H, C, d.dk, generator=g).half()
    vc = torch.randn(d.L, N, d.H, C, d.dk, generator=g).half()
    ck = torch.randn(d.L, B, d.H, T, d.dk, generator=g).half()
    cv = torch.randn(d.L, B, d.H, T, d.dk, generator=g).half()
    score = (torch.randn(N, generator=g) * 2 - 5).float()
    active = torch.rand(N, generator=g) < 0.7
    active[::K] = True
    active[K : 2 * K] = False  # a finished utterance: LOG_ZERO candidates only
    kcd, vcd = kc.to(DEV), vc.to(DEV)
    logits = torch.zeros(N, 1, d.V, device=DEV)
    new_kv = torch.zeros(d.L, 2, N, d.H, 1, d.dk, device=DEV, dtype=torch.float16)
    sc = score.to(DEV)
    act = active.to(torch.uint8).to(DEV)
    parent = torch.zeros(N, dtype=torch.long, device=DEV)
    token = torch.zeros(N, dtype=torch.long, device=DEV)
    run = kern.beam_fn(tokens.to(DEV), offset.to(DEV), kcd, vcd, ck.to(DEV), cv.to(DEV), logits, new_kv, sc, act,
                       parent, token, beam=K)  # fmt: skip
    assert kern.plan_kernel(run) == kernel
    run()
    torch.cuda.synchronize()
    kern.check()
    top, par, tok = ref.beam_topk(logits[:, 0].cpu(), score, active, B, K)
    live = torch.ones(N, dtype=torch.bool)
    live[K : 2 * K] = False  # the finished utterance's picks are ties of LOG_ZERO; order by flat index
    assert torch.equal(parent.cpu(), par) and torch.equal(token.cpu(), tok)
    torch.testing.assert_close(sc.cpu(), top, atol=1e-2, rtol=0)
    # cache: rows after the step's own write, then index_select by parent
    kw, vw = kc.to(DEV).clone(), vc.to(DEV).clone()
    ref.write_kv(new_kv, kw, vw, offset.to(DEV))
    ek, ev = ref.reorder_cache(kw, parent), ref.reorder_cache(vw, parent)
    n = 10  # slots 0 .. offset (the reorder copies the written slots only)
    assert torch.equal(kcd[..., :n, :], ek[..., :n, :]) and torch.equal(vcd[..., :n, :], ev[..., :n, :])


def test_timeout_sets_error_and_recovers(kern):
    """A wait limit of one poll makes the grid barriers give up: the call returns, check() raises, and the
    next call with the default limit is correct again (failure detection without a GPU fault)."""
    d = TEST_CFG
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, 2, 1, 64, 37, 5)
    good = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv)[0]
    kern.set_max_spin(1)
    try:
        logits = torch.zeros(2, 1, d.V, device=DEV)
        new_kv = torch.zeros(d.L, 2, 2, d.H, 1, d.dk, device=DEV, dtype=torch.float16)
        kern.step_fn(tokens.to(DEV), offset.to(DEV), kc.to(DEV), vc.to(DEV), ck.to(DEV), cv.to(DEV), logits, new_kv)()
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="timed out"):
            kern.check()
    finally:
        kern.set_max_spin(0)
    again = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv)[0]
    assert torch.equal(again, good)


def test_cuda_graph_replay(kern):
    """run() captured in a CUDA graph and replayed gives the eager results (fixed buffers, no host sync)."""
    d = TEST_CFG
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, 3, 1, 64, 37, 8)
    eager = _run_step(kern, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv)[0]
    tok, off = tokens.to(DEV), offset.to(DEV)
    kcd, vcd, ckd, cvd = kc.to(DEV), vc.to(DEV), ck.to(DEV), cv.to(DEV)
    logits = torch.zeros(3, 1, d.V, device=DEV)
    new_kv = torch.zeros(d.L, 2, 3, d.H, 1, d.dk, device=DEV, dtype=torch.float16)
    run = kern.step_fn(tok, off, kcd, vcd, ckd, cvd, logits, new_kv)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    logits.zero_()
    graph.replay()
    torch.cuda.synchronize()
    kern.check()
    assert torch.equal(logits, eager)


_MEDIUM = []


def _medium():
    """The 1B-shaped test model (plain weights, seed 0) and its kernel, built once per session."""
    _gpu()
    from owsm_trt_b200.decoder import B200Decoder
    from owsm_trt_b200.synthetic import MEDIUM_1B

    if not _MEDIUM:
        sd = decoder_state_dict(MEDIUM_1B, 0, False)
        _MEDIUM.append((sd, B200Decoder.from_state_dict(sd, MEDIUM_1B.H, DEV)))
    return _MEDIUM[0]


@pytest.mark.slow
def test_medium_step_matches_reference_golden():
    """The 18-layer d=1024 decoder (plain weights, b1, T=750) against owsm-trt's own fp32 step:
    top-32 ids, max-abs 3e-2 on those logits."""
    _gpu()
    from owsm_trt_b200.decoder import B200Decoder
    from owsm_trt_b200.synthetic import MEDIUM_1B, cross_kv

    d = MEDIUM_1B
    sd, k = _medium()
    tokens, offset, kc, vc, enc = cases.medium_inputs(d)
    kv = cross_kv(sd, d, enc).half()
    gold = np.load(f"{GOLD}/medium_step.npz")
    logits, new_kv, kc2, vc2, pred = _run_step(k, d, tokens, offset, kc.to(DEV), vc.to(DEV), kv[:, 0].contiguous(),
                                                kv[:, 1].contiguous())  # fmt: skip
    lg = logits[0, 0].cpu()
    idx = torch.from_numpy(gold["top_idx"])
    err = (lg[idx] - torch.from_numpy(gold["top_val"])).abs().max().item()
    assert err < 3e-2, err
    assert int(pred[0, 0]) == int(idx[0]) or float(gold["top_val"][0] - gold["top_val"][1]) < 1e-3
    assert abs(float(lg.double().sum()) - float(gold["sum"])) < 3e-2 * d.V ** 0.5


@pytest.mark.slow
def test_medium_batch16_matches_oracle():
    """The benchmark's call shape on the 1B-shaped model (16 one-token rows, two token tiles, LayerNorm split
    over each cluster, wide cross-attention steps for the units of 256 frames or more) against the oracle:
    logits within the oracle tolerance, argmax bit-exact outside near-ties, new K/V and cache."""
    from owsm_trt_b200.synthetic import MEDIUM_1B

    d = MEDIUM_1B
    sd, k = _medium()
    R, C, T = 16, 64, 300
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, 1, C, T, 4242)
    lens = [300, 256, 299, 255, 17, 280, 150, 300, 1, 270, 290, 120, 260, 300, 64, 257]
    lo, kvo = ref.decoder_step(sd, d.H, tokens, offset, kc.float(), vc.float(), ck.float(), cv.float(),
                               enc_len=torch.tensor(lens))  # fmt: skip
    logits, new_kv, kc2, vc2, pred = _run_step(k, d, tokens, offset, kc.to(DEV), vc.to(DEV), ck, cv, enc_len=lens)
    assert k.plan_kernel(k.step_fn(tokens.to(DEV), offset.to(DEV), kc2, vc2, ck.to(DEV), cv.to(DEV), logits,
                                   new_kv)) == "cluster"  # fmt: skip
    assert (logits.cpu() - lo).abs().max().item() < 0.02 * lo.abs().max().item()
    torch.testing.assert_close(new_kv.float().cpu(), kvo, atol=0.05, rtol=0.02)
    _check_cache(kc.to(DEV), vc.to(DEV), kc2, vc2, new_kv, offset)
    _argmax_ok(lo, logits, pred)


@pytest.mark.slow
@pytest.mark.parametrize("R,S", [(16, 4), (64, 1), (1, 16), (15, 1), (1, 32)])
def test_medium_row_counts_plan_and_run(R, S):
    """Every row count the benchmarks use on the 1B-shaped model (prefill of 16 x 4, 64 rows, 16- and
    32-token windows, 15 beam rows) gets a plan within shared memory and runs: finite logits, argmax bit-exact
    against them, the cache written at each row's offset."""
    from owsm_trt_b200.synthetic import MEDIUM_1B

    d = MEDIUM_1B
    _, k = _medium()
    g = torch.Generator().manual_seed(R * 100 + S)
    gd = torch.Generator(device=DEV).manual_seed(R * 100 + S)
    C, T = 64, 192
    tokens = torch.randint(0, d.V, (R, S), generator=g)
    offset = torch.randint(0, C - S, (R,), generator=g)

    def rnd(*shape):
        return (torch.randn(*shape, generator=gd, device=DEV) * 0.5).half()

    kc, vc = rnd(d.L, R, d.H, C, d.dk), rnd(d.L, R, d.H, C, d.dk)
    ck, cv = rnd(d.L, R, d.H, T, d.dk), rnd(d.L, R, d.H, T, d.dk)
    logits, new_kv, kc2, vc2, pred = _run_step(k, d, tokens, offset, kc, vc, ck, cv)
    assert bool(torch.isfinite(logits).all())
    assert torch.equal(pred.cpu(), ref.argmax_first(logits.cpu()))
    _check_cache(kc, vc, kc2, vc2, new_kv, offset)


@pytest.mark.parametrize("path", [0, 1])
def test_beam_shared_prefix_matches_full_reorder(kern, path):
    """Eight consecutive fused beam steps with the record of common cache slots (`shared`: a row copies only its
    parent's slots past what the two hold in common) against the same steps copying every slot: identical
    selections and scores, and identical caches over the written slots, step after step; on the cluster kernel
    (path 0) and the grid-stage kernel (path 1)."""
    kern.set_path(path)
    try:
        _shared_prefix_case(kern)
    finally:
        kern.set_path(0)


def _shared_prefix_case(kern):
    d = TEST_CFG
    B, K, C, T, P0 = 2, 4, 32, 37, 6
    N = B * K
    g = torch.Generator().manual_seed(33)
    # the rows of an utterance start from the same prompt: equal keys / values in slots 0 .. P0 - 1
    kc = torch.randn(d.L, B, d.H, C, d.dk, generator=g).half().repeat_interleave(K, dim=1)
    vc = torch.randn(d.L, B, d.H, C, d.dk, generator=g).half().repeat_interleave(K, dim=1)
    ck = torch.randn(d.L, B, d.H, T, d.dk, generator=g).half().to(DEV)
    cv = torch.randn(d.L, B, d.H, T, d.dk, generator=g).half().to(DEV)
    tok0 = torch.randint(0, d.V, (N, 1), generator=g)
    states = []
    for use_shared in (False, True):
        st = {"kc": kc.clone().to(DEV), "vc": vc.clone().to(DEV), "tok": tok0.clone().to(DEV),
              "off": torch.full((N,), P0, dtype=torch.long, device=DEV), "score": torch.zeros(N, device=DEV),
              "active": torch.ones(N, dtype=torch.uint8, device=DEV), "parent": torch.zeros(N, dtype=torch.long, device=DEV),
              "logits": torch.zeros(N, 1, d.V, device=DEV),
              "new_kv": torch.zeros(d.L, 2, N, d.H, 1, d.dk, device=DEV, dtype=torch.float16),
              "shared": torch.full((B, K, K), P0, dtype=torch.int32, device=DEV) if use_shared else None}  # fmt: skip
        st["token"] = st["tok"][:, 0]
        st["run"] = kern.beam_fn(st["tok"], st["off"], st["kc"], st["vc"], ck, cv, st["logits"], st["new_kv"],
                                 st["score"], st["active"], st["parent"], st["token"], beam=K, shared=st["shared"])  # fmt: skip
        states.append(st)
    for step in range(8):
        for st in states:
            st["run"]()
        torch.cuda.synchronize()
        kern.check()
        a, b = states
        assert torch.equal(a["parent"], b["parent"]) and torch.equal(a["token"], b["token"]), step
        assert torch.equal(a["score"], b["score"]), step
        n = P0 + step + 1  # slots written so far
        assert torch.equal(a["kc"][..., :n, :], b["kc"][..., :n, :]), step
        assert torch.equal(a["vc"][..., :n, :], b["vc"][..., :n, :]), step
        for st in states:
            st["off"] += 1
