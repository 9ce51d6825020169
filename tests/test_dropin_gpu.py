"""The drop-in, exercised through owsm-trt's own callers: ``GreedySession`` (plain steps, drafted verify windows,
timestamp rules) over ``MegaBackend`` (src/owsm_trt/megakernel.py:688-767) with :class:`B200Decoder` as its
kernel must give the tokens of the same session over ``TorchBackend`` -- the reference's
``test_greedy_session_matches_torch`` / ``test_ring_session_with_rules`` (tests/test_megakernel.py:95-119,
:372-392) with this build's kernel in place of the Triton / Gluon one.

This covers what the unit tests of the C ABI cannot: ``MegaBackend.step_fn``'s remap of ``inp`` into strided
``tokens = rows[:, :w]`` / ``offset = rows[:, w]`` views (megakernel.py:743-745), ``kind="verify"`` windows, the
``pred`` / ``notime`` keywords and the sessions' CUDA-graph capture of ``run()``.

The reference package is the pip-installed copy under ``baseline/_ref`` (unmodified sources; git-ignored); these
tests skip when it is absent."""

from __future__ import annotations

import copy
import dataclasses
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _reference():
    if not torch.cuda.is_available():
        pytest.fail("these tests need a CUDA GPU")
    if not (REF / "owsm_trt").is_dir():
        pytest.skip("the reference package is not installed under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.append(str(REF))
    from owsm_trt import megakernel, runtime
    from owsm_trt.config import OWSMConfig
    from owsm_trt.modeling import OWSMModel

    return megakernel, runtime, OWSMConfig, OWSMModel


@pytest.fixture(scope="module")
def ref_model():
    """The reference tests' model: TINY widened to d=256, 4 heads, 3 layers, V=1000, seeded weights with
    non-trivial LayerNorms and biases and the output weight x8 (tests/test_megakernel.py:20-40)."""
    megakernel, runtime, OWSMConfig, OWSMModel = _reference()
    tiny = OWSMConfig(
        vocab_size=50, d_model=32, n_heads=4, enc_layers=2, enc_ffn=64, cgmlp_units=64, cgmlp_kernel=5,
        merge_kernel=3, subsample="conv2d8", dec_layers=2, dec_ffn=64, dec_heads=4, n_mels=16, n_fft=64,
        win_length=48, hop_length=32, sample_rate=1600, speech_seconds=2.0, time_resolution=0.02,
    )  # fmt: skip
    cfg = dataclasses.replace(tiny, d_model=256, n_heads=4, dec_heads=4, dec_ffn=512, dec_layers=3, vocab_size=1000)
    torch.manual_seed(0)
    m = OWSMModel(cfg).eval().requires_grad_(False)
    m.frontend.melmat.uniform_(0, 1)
    for name, p in m.decoder.named_parameters():
        if "norm" in name:
            p.add_(0.2 * torch.randn_like(p))
        elif name.endswith("bias"):
            p.copy_(0.2 * torch.randn_like(p))
    m.decoder.output_layer.weight.mul_(8.0)
    m.fuse_projections()
    return cfg, m.cuda()


def _session(runtime, cfg, backend, batch, windows=(), rules=None):
    return runtime.GreedySession(
        backend, cfg, batch, 64, eos=1, dtype=torch.float16, device=torch.device("cuda"), buckets=[16, 32, 64],
        draft_windows=windows, rules=rules,
    )  # fmt: skip


@pytest.mark.parametrize("drafted", [False, True], ids=["steps", "drafted"])
@pytest.mark.parametrize("batch", [1, 3])
def test_greedy_session_through_megabackend(ref_model, drafted, batch):
    megakernel, runtime, _, _ = _reference()
    from owsm_trt_b200.decoder import B200Decoder

    cfg, model = ref_model
    m16 = copy.deepcopy(model).half()
    m16.frontend.float()
    kern = B200Decoder(model.decoder, torch.device("cuda"))
    be = megakernel.MegaBackend(runtime.TorchBackend(m16), kern, max_tokens=64, trial=True)
    assert be.argmax
    torch.manual_seed(batch)
    feats = m16.frontend(torch.randn(batch, cfg.num_samples, device="cuda"))
    primer = torch.tensor([[2, 3, 4]] * batch, device="cuda")
    drafts = [[5, 6, 7, 8, 9, 10], [11, 12], []][:batch]
    outs = []
    for b in (runtime.TorchBackend(m16), be):
        sess = _session(runtime, cfg, b, batch, (2, 4, 8) if drafted else ())
        sess.encode(feats)
        out = sess.decode_drafted(primer, drafts, 20)[0] if drafted else sess.decode(primer, 20)
        outs.append(out)
    assert not be.failed, "the B200 kernel's trial call failed and MegaBackend fell back to TorchBackend"
    assert outs[0] == outs[1]


@pytest.mark.parametrize("primer", [[2, 3, 999], [2, 3, 4]], ids=["notimestamps", "timestamps"])
def test_session_with_timestamp_rules(ref_model, primer):
    """Under the timestamp rules: the kernel's fused argmax for <notimestamps> rows, kernels.choose for the others
    (tests/test_megakernel.py:372-392)."""
    megakernel, runtime, _, _ = _reference()
    from owsm_trt_b200.decoder import B200Decoder

    cfg, model = ref_model
    m16 = copy.deepcopy(model).half()
    m16.frontend.float()
    kern = B200Decoder(model.decoder, torch.device("cuda"))
    be = megakernel.MegaBackend(runtime.TorchBackend(m16), kern, 32, 8, trial=True)
    rules = runtime.TimestampRules(999, 900, 998, 1, cfg.vocab_size, torch.device("cuda"))
    torch.manual_seed(7)
    feats = m16.frontend(torch.randn(1, cfg.num_samples, device="cuda"))
    outs = []
    for b in (runtime.TorchBackend(m16), be):
        sess = _session(runtime, cfg, b, 1, (2, 4, 8), rules)
        sess.encode(feats)
        out, _ = sess.decode_drafted(torch.tensor([primer], device="cuda"), [[5, 6, 7, 8]], 20)
        outs.append(out)
    assert not be.failed
    assert outs[0] == outs[1]


def _beam_session(runtime, cls, cfg, backend, batch, beam, **kw):
    return cls(backend, cfg, batch, beam, 64, eos=1, dtype=torch.float16, device=torch.device("cuda"),
               buckets=[16, 32, 64], **kw)  # fmt: skip


@pytest.mark.parametrize("batch,beam", [(1, 4), (3, 5)])
def test_beam_session_with_fused_step(ref_model, batch, beam):
    """owsm-trt's BeamSession with each search step as one fused beam_fn launch (decoder call, log-softmax, top-K,
    parents / tokens, cache reorder; owsm_trt_b200.beam.fused_beam_session) gives the hypotheses of the same
    session run unfused over MegaBackend (the kernel's step_fn for the decoder call, torch's selection and cache
    reorder on its logits): the same logits, the same selection. (Against TorchBackend's fp32 search the fp16
    logits may break near-ties between hypotheses' cumulative scores the other way, which beam search carries on
    into different hypotheses; the teacher-forced beam test of the 1B decoder counts those near-ties instead.)"""
    megakernel, runtime, _, _ = _reference()
    from owsm_trt_b200.beam import fused_beam_session
    from owsm_trt_b200.decoder import B200Decoder

    cfg, model = ref_model
    m16 = copy.deepcopy(model).half()
    m16.frontend.float()
    kern = B200Decoder(model.decoder, torch.device("cuda"))
    be = megakernel.MegaBackend(runtime.TorchBackend(m16), kern, max_tokens=64, trial=True)
    torch.manual_seed(100 + batch)
    feats = m16.frontend(torch.randn(batch, cfg.num_samples, device="cuda"))
    primer = torch.tensor([[2, 3, 4]] * batch, device="cuda")
    fused = fused_beam_session(runtime)
    outs = []
    for cls, kw in ((runtime.BeamSession, {}), (fused, {"kernel": kern})):
        sess = _beam_session(runtime, cls, cfg, be, batch, beam, **kw)
        sess.encode(feats)
        outs.append(sess.decode(primer, 24))
    assert not be.failed
    assert outs[1] == outs[0], "fused beam step differs from the same kernel's logits with torch's selection"
