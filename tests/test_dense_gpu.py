"""The dense kernel (greedy calls of 33 to 64 tokens per launch, row slices beyond; tcgen05 tensor-core GEMMs
with the fp32 accumulator in TMEM) against the CPU oracle (owsm-trt's Decoder.step, src/owsm_trt/modeling.py:501-560).

Tolerances as the other kernel tests (owsm-trt's tests/test_megakernel.py:76-85): logits max-abs < 0.02 x max|ref|
on the perturbed test models, new K/V assert_close(atol 0.05, rtol 0.02), the cache after the in-kernel write
bit-equal to a scatter of new_kv, argmax bit-exact against the kernel's own logits and equal to the oracle's except
at near-ties (top-2 gap < 1e-3)."""

import pytest
import torch

import cases
from oracle import decoder as ref
from owsm_trt_b200.synthetic import TEST_CFG, TEST_CFG384, decoder_state_dict

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _kernel(d, seed, path):
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA GPU")
    from owsm_trt_b200.decoder import B200Decoder

    sd = decoder_state_dict(d, seed, True)
    k = B200Decoder.from_state_dict(sd, d.H, DEV)
    k.set_path(path)
    return sd, k


def _call(k, d, tokens, offset, kc, vc, ck, cv, enc_len=None, rows_per_utt=1):
    R, S = tokens.shape
    logits = torch.full((R, S, d.V), float("nan"), device=DEV)
    new_kv = torch.zeros(d.L, 2, R, d.H, S, d.dk, device=DEV, dtype=torch.float16)
    pred = torch.full((R, S), -1, dtype=torch.long, device=DEV)
    kc2, vc2 = kc.clone().to(DEV), vc.clone().to(DEV)
    el = None if enc_len is None else torch.tensor(enc_len, dtype=torch.int32, device=DEV)
    run = k.step_fn(tokens.to(DEV), offset.to(DEV), kc2, vc2, ck.to(DEV), cv.to(DEV), logits, new_kv, pred=pred,
                    enc_len=el, rows_per_utt=rows_per_utt)  # fmt: skip
    run()
    torch.cuda.synchronize()
    k.check()
    return k.plan_kernel(run), k.launches(run), logits, new_kv, kc2, vc2, pred


def _check(sd, d, tokens, offset, kc, vc, ck, cv, out, enc_len=None, cross_row=None):
    _, _, logits, new_kv, kc2, vc2, pred = out
    lo, kvo = ref.decoder_step(sd, d.H, tokens, offset, kc.float(), vc.float(), ck.float(), cv.float(),
                               enc_len=None if enc_len is None else torch.tensor(enc_len), cross_row=cross_row)  # fmt: skip
    assert bool(torch.isfinite(logits).all())
    err = (logits.cpu() - lo).abs().max().item()
    assert err < 0.02 * lo.abs().max().item(), err
    torch.testing.assert_close(new_kv.float().cpu(), kvo, atol=0.05, rtol=0.02)
    k, v = kc.clone().to(DEV), vc.clone().to(DEV)
    ref.write_kv(new_kv, k, v, offset.to(DEV))
    assert torch.equal(kc2, k) and torch.equal(vc2, v)
    assert torch.equal(pred.cpu(), ref.argmax_first(logits.cpu()))
    top2 = lo.topk(2, dim=-1).values
    tie = (top2[..., 0] - top2[..., 1]) < 1e-3
    assert bool(((pred.cpu() == lo.argmax(-1)) | tie).all())


@pytest.mark.parametrize("R,S", [(64, 1), (33, 1), (8, 8), (4, 16), (1, 1), (16, 2)])
def test_dense_matches_oracle(R, S):
    """Shapes on the dense kernel (forced for the small ones): one-query units (wide cross-attention steps) and
    windows of up to 16 queries."""
    d = TEST_CFG
    sd, k = _kernel(d, 0, 3)
    C, T = 64, 300
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, S, C, T, 3000 + R * 10 + S)
    out = _call(k, d, tokens, offset, kc, vc, ck, cv)
    assert out[0] == "dense" and out[1] == 1
    _check(sd, d, tokens, offset, kc, vc, ck, cv, out)


def test_dense_masked_lengths_and_default_choice():
    """48 rows with per-utterance encoder lengths; the default path picks the dense kernel above 32 tokens."""
    d = TEST_CFG
    sd, k = _kernel(d, 1, 0)
    R, C, T = 48, 64, 300
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, 1, C, T, 4801)
    lens = [300, 1, 17, 150, 299, 256, 255, 40] * 6
    out = _call(k, d, tokens, offset, kc, vc, ck, cv, enc_len=lens)
    assert out[0] == "dense"
    _check(sd, d, tokens, offset, kc, vc, ck, cv, out, enc_len=lens)


def test_dense_row_slices_beyond_64_tokens():
    """150 rows: three launches of up to 64 tokens on the caller's buffers (the 64-token cap of one call lifted)."""
    d = TEST_CFG
    sd, k = _kernel(d, 2, 0)
    R, C, T = 150, 32, 40
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, 1, C, T, 15001)
    out = _call(k, d, tokens, offset, kc, vc, ck, cv)
    assert out[0] == "dense" and out[1] == 3
    _check(sd, d, tokens, offset, kc, vc, ck, cv, out)


def test_dense_shared_cross_rows():
    """rows_per_utt = 4: an utterance's cross K/V read once for its 4 rows (16 utterances x 4 rows)."""
    d = TEST_CFG
    sd, k = _kernel(d, 3, 0)
    R, C, T = 64, 32, 60
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, 1, C, T, 6401)
    u = torch.arange(R) // 4
    out = _call(k, d, tokens, offset, kc, vc, ck[:, ::4].contiguous(), cv[:, ::4].contiguous(), rows_per_utt=4)
    assert out[0] == "dense"
    _check(sd, d, tokens, offset, kc, vc, ck[:, ::4].contiguous(), cv[:, ::4].contiguous(), out, cross_row=u)


def test_dense_width_384_and_determinism():
    """d = 384 (one K range of 384 per tile, FFN K split in two): against the oracle, and two calls bit-identical."""
    d = TEST_CFG384
    sd, k = _kernel(d, 4, 3)
    R, S, C, T = 40, 1, 32, 29
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, S, C, T, 3841)
    a = _call(k, d, tokens, offset, kc, vc, ck, cv)
    _check(sd, d, tokens, offset, kc, vc, ck, cv, a)
    b = _call(k, d, tokens, offset, kc, vc, ck, cv)
    assert torch.equal(a[2], b[2]) and torch.equal(a[3], b[3])


def test_dense_cuda_graph_replay():
    """run() captured in a CUDA graph and replayed gives the eager logits."""
    d = TEST_CFG
    _, k = _kernel(d, 5, 0)
    R, C, T = 64, 32, 37
    tokens, offset, kc, vc, ck, cv = cases.step_inputs(d, R, 1, C, T, 777)
    eager = _call(k, d, tokens, offset, kc, vc, ck, cv)[2]
    tok, off = tokens.to(DEV), offset.to(DEV)
    kcd, vcd, ckd, cvd = kc.to(DEV), vc.to(DEV), ck.to(DEV), cv.to(DEV)
    logits = torch.zeros(R, 1, d.V, device=DEV)
    new_kv = torch.zeros(d.L, 2, R, d.H, 1, d.dk, device=DEV, dtype=torch.float16)
    run = k.step_fn(tok, off, kcd, vcd, ckd, cvd, logits, new_kv)
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
    k.check()
    assert torch.equal(logits, eager)
