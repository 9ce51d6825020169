"""The host side of the fused beam search (owsm_trt_b200.beam.fused_beam_session) on the CPU: owsm-trt's BeamSession
over TorchBackend against the fused-step subclass, whose kernel is replaced here by a stand-in that does on the CPU
what B200Decoder.beam_fn does on the GPU -- the reference's own decoder step (TorchBackend.step_fn), the new keys and
values written at the rows' offsets, BeamSession._select step 1 and the cache reorder (the oracle's restatements,
runtime.py:1399-1413). Equal hypotheses mean the subclass's own part is right: the step's bookkeeping after the
selection (token histories, finished hypotheses, end_detect; runtime.py:1410-1446), the first selection after the
prompt, the cross K/V read once per utterance. With `record`, the stand-in also keeps the session's record of the
cache slots each pair of an utterance's hypotheses holds in common and copies only a row's slots past it, as the
kernel's select and reorder stages do (select_stage / reorder_stage, owsm_trt_b200/csrc/decoder.cu), and checks after
every step that the record holds: equal hypotheses and the check pin the record's update rule on the CPU. The
reference package is the pip-installed copy under baseline/_ref; the test skips when it is absent."""

from __future__ import annotations

import dataclasses
import sys
from pathlib import Path

import pytest
import torch

from oracle import decoder as ref

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _reference():
    if not (REF / "owsm_trt").is_dir():
        pytest.skip("the reference package is not installed under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.append(str(REF))
    from owsm_trt import runtime
    from owsm_trt.config import OWSMConfig
    from owsm_trt.modeling import OWSMModel

    return runtime, OWSMConfig, OWSMModel


def _record_step(shared, parent, offset, S, beam):
    """The select stage's use of the record D [utterances][beam][beam] (slots each pair of rows holds in common before
    this step's write): row i copies its parent's slots from D[i][parent(i)] on (its first slot to copy, returned per
    row); afterwards two rows hold in common all offset(parent) + S slots of a parent they share, else what their
    parents held in common (D updated in place)."""
    B = shared.shape[0]
    u = torch.arange(B)[:, None]
    pl = parent.view(B, beam) - u * beam  # each row's parent, as an index in its utterance
    first = shared[u, torch.arange(beam)[None, :], pl]
    length = offset.view(B, beam).gather(1, pl) + S
    same = pl[:, :, None] == pl[:, None, :]
    held = shared[u[:, :, None], pl[:, :, None], pl[:, None, :]]
    shared.copy_(torch.where(same, length[:, :, None].expand(B, beam, beam).to(shared.dtype), held))
    return first.reshape(-1)


def _partial_reorder(buf, parent, offset, S, first):
    """The reorder stage in place: a row whose parent is another row takes the parent's slots first .. offset + S - 1
    (the slots before `first` are already the same), every read before any write."""
    src = buf.clone()
    for r in range(buf.shape[1]):
        p = int(parent[r])
        if p == r:
            continue
        lp = int(offset[p]) + S
        cs = min(max(int(first[r]), 0), lp)
        buf[:, r, :, cs:lp] = src[:, p, :, cs:lp]


class _CpuFusedStep:
    """beam_fn's contract on the CPU (see the module docstring); with `record` False, `shared` is left alone and
    the whole cache is reordered."""

    def __init__(self, backend, record):
        self.backend, self.record = backend, record

    def beam_fn(self, tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv, score, active, parent, token,
                *, beam, enc_len=None, shared=None):  # fmt: skip
        def run() -> None:
            ck, cv = cross_k.repeat_interleave(beam, dim=1), cross_v.repeat_interleave(beam, dim=1)
            self.backend.step_fn(tokens, offset, self_k, self_v, ck, cv, logits, new_kv)()
            ref.write_kv(new_kv, self_k, self_v, offset)
            sc, par, tok = ref.beam_topk(logits[:, -1], score, active.bool(), tokens.shape[0] // beam, beam)
            score.copy_(sc)
            parent.copy_(par)
            token.copy_(tok)
            if not self.record:
                self_k.copy_(ref.reorder_cache(self_k, parent))
                self_v.copy_(ref.reorder_cache(self_v, parent))
                return
            S = tokens.shape[1]
            first = _record_step(shared, parent, offset, S, beam)
            _partial_reorder(self_k, parent, offset, S, first)
            _partial_reorder(self_v, parent, offset, S, first)
            for u in range(shared.shape[0]):  # the record holds
                for i in range(beam):
                    for j in range(beam):
                        n = int(shared[u, i, j])
                        for buf in (self_k, self_v):
                            assert torch.equal(buf[:, u * beam + i, :, :n], buf[:, u * beam + j, :, :n]), (u, i, j, n)

        return run


# eos ids picked so that hypotheses end early: at 17 tokens for (1, 3); at 7 tokens for one utterance of (2, 4)
# while the other runs to the length limit
@pytest.mark.parametrize("record", [False, True])
@pytest.mark.parametrize("batch,beam,eos", [(1, 3, 37), (2, 4, 19)])
def test_fused_beam_session_matches_beam_session(batch, beam, eos, record):
    runtime, OWSMConfig, OWSMModel = _reference()
    from owsm_trt_b200.beam import fused_beam_session

    tiny = OWSMConfig(
        vocab_size=50, d_model=32, n_heads=4, enc_layers=2, enc_ffn=64, cgmlp_units=64, cgmlp_kernel=5,
        merge_kernel=3, subsample="conv2d8", dec_layers=2, dec_ffn=64, dec_heads=4, n_mels=16, n_fft=64,
        win_length=48, hop_length=32, sample_rate=1600, speech_seconds=2.0, time_resolution=0.02,
    )  # fmt: skip
    cfg = dataclasses.replace(tiny, vocab_size=200)
    torch.manual_seed(3)
    model = OWSMModel(cfg).eval().requires_grad_(False)
    model.frontend.melmat.uniform_(0, 1)
    model.decoder.output_layer.weight.mul_(8.0)  # sharper distributions: hypotheses finish and diverge
    backend = runtime.TorchBackend(model)
    feats = model.frontend(torch.randn(batch, cfg.num_samples))
    primer = torch.tensor([[2, 3, 4]] * batch)
    kw = dict(eos=eos, dtype=torch.float32, device=torch.device("cpu"), use_cuda_graph=False, buckets=[16, 32, 64])
    outs = []
    for sess in (runtime.BeamSession(backend, cfg, batch, beam, 64, **kw),
                 fused_beam_session(runtime)(backend, cfg, batch, beam, 64, kernel=_CpuFusedStep(backend, record), **kw)):  # fmt: skip
        with torch.no_grad():
            sess.encode(feats)
            outs.append(sess.decode(primer, 30))
    assert outs[1] == outs[0]
    lens = [len(h) for h in outs[0]]
    assert all(0 < n for n in lens) and min(lens) < 30, lens
