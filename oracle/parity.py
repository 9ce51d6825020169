"""Teacher-forced comparison of a decoder under test against the fp32 oracle, step by step.

TEST INFRASTRUCTURE ONLY (the checker): used by ``tests/`` and by ``bench.py``'s CPU-baseline leg. The
decoder under test is given as a callable; this module never imports the product package.

Protocol (the north star of the build: owsm-trt's torch decoder on identical seeded weights and encoder memory,
teacher-forced token prefixes so that every step is compared):

* both decoders see the same tokens at every step -- the oracle's own argmax (greedy) or the oracle's beam
  choices (beam) -- and each keeps its own KV cache (the oracle's fp32, the tested one's fp16);
* per step: logits max-abs error over all V logits against the fp32 oracle;
* argmax: bit-exact except where the oracle's top-two gap is below ``TIE`` (near-ties, counted);
* beam: parents and tokens bit-exact except where the oracle's candidate scores around the cut-off are closer
  than ``TIE`` (counted); scores within 1e-2.

The oracle steps are ``oracle.decoder.decoder_step`` (owsm-trt ``Decoder.step``, src/owsm_trt/modeling.py:501-560)
and ``beam_topk`` / ``reorder_cache`` (``BeamSession._select``, src/owsm_trt/runtime.py:1399-1413).
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from . import decoder as ref

TOL = 3e-2  # logits max-abs against fp32 (north star)
TIE = 1e-3  # near-tie: the oracle's top-two logit gap (or beam candidate gap) below this
SCORE_TOL = 1e-2  # beam scores


@dataclass
class Tally:
    """Per-step results of a teacher-forced run."""

    steps: int = 0
    rows: int = 0  # row-steps compared
    max_err: float = 0.0
    errs: list = field(default_factory=list)  # per-step max-abs logits error
    near_ties: int = 0  # row-steps whose oracle top-two gap < TIE
    tie_flips: int = 0  # of those, where the tested argmax differs
    mismatches: int = 0  # argmax (or beam pick) differs although the oracle's gap >= TIE
    mismatch_gaps: list = field(default_factory=list)  # (step, row, oracle gap, step max-abs error)
    score_err: float = 0.0
    oracle_s: float = 0.0  # seconds spent in the oracle

    def add_greedy(self, lo: torch.Tensor, lg: torch.Tensor, pred: torch.Tensor) -> None:
        """lo, lg [R, V] (oracle, tested) logits of the step's last position; pred [R] the tested argmax."""
        err = float((lg - lo).abs().max())
        self.errs.append(err)
        self.max_err = max(self.max_err, err)
        top2 = lo.topk(2, dim=-1).values
        gap = top2[:, 0] - top2[:, 1]
        want = ref.argmax_first(lo)
        for r in range(lo.shape[0]):
            tie = float(gap[r]) < TIE
            same = int(pred[r]) == int(want[r])
            self.near_ties += tie
            self.tie_flips += tie and not same
            if not tie and not same:
                self.mismatches += 1
                self.mismatch_gaps.append((self.steps, r, float(gap[r]), err))
        self.steps += 1
        self.rows += lo.shape[0]

    def summary(self) -> dict:
        return {
            "steps": self.steps, "row_steps": self.rows, "logits_max_abs": round(self.max_err, 5),
            "logits_max_abs_median_step": round(sorted(self.errs)[len(self.errs) // 2], 5) if self.errs else None,
            "bound": TOL, "near_ties": self.near_ties, "near_tie_flips": self.tie_flips,
            "mismatches_outside_near_ties": self.mismatches,
            "mismatch_detail": [[s, r, round(g, 5), round(e, 5)] for s, r, g, e in self.mismatch_gaps[:8]],
            "score_max_abs": round(self.score_err, 5) if self.score_err else None,
        }  # fmt: skip


def greedy(step, sd: dict, heads: int, prefix: torch.Tensor, offset0: torch.Tensor, ck32, cv32, enc_len, steps: int,
           kc32: torch.Tensor, vc32: torch.Tensor, pe: torch.Tensor, tally: Tally | None = None,
           compare_prefix: bool = True) -> Tally:  # fmt: skip
    """Teacher-forced greedy run. ``step(tokens [R, S] int64 CPU, offset [R] int64 CPU)`` runs the tested decoder's
    call on its own cache and returns (logits [R, S, V], pred [R, S]) on the CPU.

    The prefix [R, P] is fed first at ``offset0`` (one call each), then ``steps`` one-token calls, each fed the
    oracle's argmax of the call before. kc32 / vc32: the oracle's fp32 caches [L, R, H, C, dk], updated in place."""
    t = tally or Tally()
    R, P = prefix.shape
    tok, off = prefix, offset0.clone()
    for j in range(steps + 1):
        if j == 0 and P == 0:
            continue
        t0 = time.perf_counter()
        with torch.no_grad():
            lo, kvo = ref.decoder_step(sd, heads, tok, off, kc32, vc32, ck32, cv32, enc_len=enc_len, pe=pe)
            ref.write_kv(kvo, kc32, vc32, off)
        t.oracle_s += time.perf_counter() - t0
        lg, pred = step(tok, off)
        if j > 0 or compare_prefix:
            if j == 0:  # every position of the prefix call
                for s in range(tok.shape[1]):
                    t.add_greedy(lo[:, s], lg[:, s], pred[:, s])
            else:
                t.add_greedy(lo[:, -1], lg[:, -1], pred[:, -1])
        off = off + tok.shape[1]
        tok = ref.argmax_first(lo[:, -1])[:, None]
    return t


def beam_gap(cand_sorted: torch.Tensor, beam: int) -> torch.Tensor:
    """Per utterance: the smallest gap between neighbours among the top beam + 1 sorted candidates (an order
    or membership flip of the top-K needs two candidates that close)."""
    top = cand_sorted[:, : beam + 1]
    return (top[:, :-1] - top[:, 1:]).min(-1).values
