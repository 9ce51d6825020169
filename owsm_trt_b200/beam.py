"""Beam search over the fused beam step: owsm-trt's ``BeamSession`` (src/owsm_trt/runtime.py:1340-1492) with each
search step's decoder call and the first part of its selection -- log-softmax, score + log-probability, top-K per
utterance, parents / tokens and the cache reorder (``_select`` step 1, runtime.py:1403-1413) -- done by one
``B200Decoder.beam_fn`` launch. The rest of the step (the hypotheses' token history, finished hypotheses and
ESPnet's ``end_detect``, runtime.py:1410-1446) stays in torch, inside the session's CUDA graph as before.

``fused_beam_session(runtime)`` takes the reference's ``owsm_trt.runtime`` module and returns the subclass; the
reference needs no other change (``INTEGRATION.md`` shows where ``transcribe`` would pick it). What differs from
the reference's session:
  * the decoder reads each utterance's cross K/V once for its ``beam`` hypotheses (``cross_kb`` / ``cross_vb``),
    so ``encode`` no longer copies them to every hypothesis row;
  * the session keeps, per utterance, how many leading cache slots each pair of hypotheses holds in common
    (``shared``: the prompt's after the first selection, then updated by every step), so a hypothesis copies only
    its parent's slots past that instead of its whole cache;
  * the timestamp rules are not fused: a session with ``rules`` raises ``ValueError`` (use ``BeamSession``).
The first selection after the prompt (from the prefill logits) is the reference's own eager ``_select``."""

from __future__ import annotations

import torch


def fused_beam_session(runtime):
    """The fused-step subclass of ``runtime.BeamSession`` (``runtime`` = the reference's ``owsm_trt.runtime``)."""

    class FusedBeamSession(runtime.BeamSession):
        """``BeamSession`` whose search steps run ``kernel.beam_fn`` (a :class:`B200Decoder`); same constructor
        plus ``kernel``. The backend still serves the encoder and the prompt."""

        def __init__(self, backend, cfg, batch, beam, capacity, eos, dtype, device, kernel, use_cuda_graph=True,
                     chunk=4, buckets=None, rules=None):  # fmt: skip
            if rules is not None:
                raise ValueError("the fused beam step has no timestamp rules: use BeamSession")
            self.kernel = kernel
            super().__init__(backend, cfg, batch, beam, capacity, eos, dtype, device, use_cuda_graph, chunk, buckets,
                             rules)  # fmt: skip

        def _capture_all(self) -> None:
            # (BeamSession.__init__ ends here, every buffer made: the fused step of each cache bucket first)
            self.parent = torch.zeros(self.rows, dtype=torch.long, device=self.device)
            self.token = torch.zeros(self.rows, dtype=torch.long, device=self.device)
            active = self.active.view(torch.uint8)  # (bool and uint8 share the byte layout)
            self.shared = torch.zeros(self.batch, self.beam, self.beam, dtype=torch.int32, device=self.device)
            self._fused = {
                c: self.kernel.beam_fn(self.tok, self.offs, k, v, self.cross_kb, self.cross_vb, self.logits,
                                       self.new_kv, self.score, active, self.parent, self.token, beam=self.beam,
                                       shared=self.shared)
                for c, (k, v) in self.caches.items()
            }  # fmt: skip
            super()._capture_all()

        def _select(self, c: int) -> None:
            # (called eagerly once per decode, on the prompt's logits: BeamSession's own selection) every row of an
            # utterance then holds the prompt's keys and values, slots 0 .. pos - 1
            super()._select(c)
            self.shared.copy_(self.pos.to(torch.int32).expand(self.batch, self.beam, self.beam))

        def encode(self, feats: torch.Tensor) -> torch.Tensor:
            return self._encoder(feats, self.cross_kb, self.cross_vb, self.ctc_ids)

        def _body(self, c: int) -> None:
            # _feed + _select step 1: one launch (decoder call at pos, selection, scores, cache reorder)
            self.offs.copy_(self.pos.expand(self.rows))
            self._fused[c]()
            self.pos += 1
            self.step += 1
            self._after_select(self.parent, self.token)

        def _after_select(self, parent: torch.Tensor, token: torch.Tensor) -> None:
            """The selection's bookkeeping once scores, parents and tokens are known (runtime.py:1410-1446)."""
            B, K = self.batch, self.beam
            # the hypotheses' histories follow their parents; the new token goes at pos
            self.seq.copy_(self.seq.index_select(0, parent))
            self.seq.index_copy_(1, self.pos, token.unsqueeze(1))
            # finished hypotheses: an extension ending in <eos>, or every live one at the length limit (which
            # then gets an <eos> appended, so its length counts one more)
            live = ~self.done.repeat_interleave(K)
            limit = self.step == self.last_step
            ended = live & ((token == self.eos) | limit)
            length = self.pos + 1 + limit.long()
            fin = torch.where(ended, self.score, float("-inf")).view(B, K)
            best, k_best = fin.max(dim=-1)  # (the first of equal scores)
            better = best > self.best_score
            self.best_score.copy_(torch.where(better, best, self.best_score))
            rows = self.row_base + k_best
            self.best_seq.copy_(torch.where(better.unsqueeze(1), self.seq.index_select(0, rows), self.best_seq))
            self.best_end.copy_(torch.where(better, self.pos + 1, self.best_end))
            by_len = self.ended_by_len.index_select(1, length)
            self.ended_by_len.index_copy_(1, length, torch.maximum(by_len, best.unsqueeze(1)))
            # end_detect: for each of the last M lengths some hypothesis of that length finished, and the best of
            # them lies more than D below the best finished score
            hits = torch.zeros(B, dtype=torch.long, device=self.device)
            for m in range(runtime.END_DETECT_M):
                n = self.step - m
                s = self.ended_by_len.index_select(1, n.clamp(min=0)).squeeze(1)
                hits += ((n >= 0) & (s > float("-inf")) & (s - self.best_score < runtime.END_DETECT_D)).long()
            still = (live & (token != self.eos)).view(B, K)
            done = self.done | limit | ~still.any(dim=-1) | (hits == runtime.END_DETECT_M)
            self.done.copy_(done)
            self.active.copy_((still & ~done.unsqueeze(1)).view(-1))
            self.tok.copy_(token.unsqueeze(1))

    return FusedBeamSession
