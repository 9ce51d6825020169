"""Seeded inputs of the golden cases, shared by ``make_golden.py`` (which runs owsm-trt on them) and the
tests (which rebuild them to check the oracle and the CUDA path against the stored outputs). The CPU
generator makes them bit-identical on every machine."""

from __future__ import annotations

import torch

from owsm_trt_b200.synthetic import DecoderDims

# name -> (rows, window, cache C, frames T, seed, enc_len or None)
STEP_CASES = {
    "r1s1": (1, 1, 64, 37, 101, None),
    "r2s5": (2, 5, 64, 37, 205, None),
    "r4s1": (4, 1, 64, 37, 401, None),
    "r3s3": (3, 3, 32, 50, 303, None),
    "masked": (3, 1, 64, 40, 77, [40, 13, 27]),
}


def step_inputs(d: DecoderDims, R: int, S: int, C: int, T: int, seed: int):
    """tokens [R,S] i64, offset [R] i64 (row 0 at an empty cache), self K/V [L,R,H,C,dk] fp16,
    cross K/V [L,R,H,T,dk] fp16."""
    g = torch.Generator().manual_seed(seed)
    tokens = torch.randint(0, d.V, (R, S), generator=g)
    offset = torch.randint(0, C - S + 1, (R,), generator=g)
    offset[0] = 0

    def half(*s):
        return torch.randn(*s, generator=g).half()

    k, v = half(d.L, R, d.H, C, d.dk), half(d.L, R, d.H, C, d.dk)
    ck, cv = half(d.L, R, d.H, T, d.dk), half(d.L, R, d.H, T, d.dk)
    return tokens, offset, k, v, ck, cv


BEAM = {"B": 3, "K": 5, "C": 16, "pos": 6, "seed": 7}


def beam_inputs(d: DecoderDims):
    """logits [N,V], score [N], active [N] bool, caches k0/v0 [L,N,H,C,dk] fp32 for N = B*K."""
    B, K, C = BEAM["B"], BEAM["K"], BEAM["C"]
    g = torch.Generator().manual_seed(BEAM["seed"])
    N = B * K
    logits = torch.randn(N, d.V, generator=g) * 3.0
    score = torch.randn(N, generator=g) * 2.0 - 5.0
    active = torch.rand(N, generator=g) < 0.7
    active[::K] = True
    k0 = torch.randn(d.L, N, d.H, C, d.dk, generator=g)
    v0 = torch.randn(d.L, N, d.H, C, d.dk, generator=g)
    return logits, score, active, k0, v0


GREEDY = {"B": 2, "C": 64, "T": 11, "seed": 11, "steps": 24, "primer": [[2, 3, 4], [2, 5, 4]], "eos": 1}


def greedy_inputs(d: DecoderDims):
    """cross K/V [L,B,H,T,dk] fp16 of the greedy-session case."""
    g = torch.Generator().manual_seed(GREEDY["seed"])
    B, T = GREEDY["B"], GREEDY["T"]
    ck = torch.randn(d.L, B, d.H, T, d.dk, generator=g).half()
    cv = torch.randn(d.L, B, d.H, T, d.dk, generator=g).half()
    return ck, cv


MEDIUM = {"seed": 5, "C": 64, "T": 750, "offset": 17}


def medium_inputs(d: DecoderDims):
    """tokens [1,1], offset [1], self K/V fp16 [L,1,H,C,dk], encoder output [1,T,D] fp32."""
    g = torch.Generator().manual_seed(MEDIUM["seed"])
    C, T = MEDIUM["C"], MEDIUM["T"]
    tokens = torch.randint(0, d.V, (1, 1), generator=g)
    offset = torch.tensor([MEDIUM["offset"]])
    k = torch.randn(d.L, 1, d.H, C, d.dk, generator=g).half()
    v = torch.randn(d.L, 1, d.H, C, d.dk, generator=g).half()
    enc = torch.randn(1, T, d.D, generator=g)
    return tokens, offset, k, v, enc


# Verify calls of the speculative greedy session: timestamp ids 500..900, <eos> 1, <notimestamps> 3 in a
# vocabulary of 1000; name -> (rows, window, seed).
VERIFY_RULES = {"notime": 3, "first_time": 500, "last_time": 900, "eos": 1, "vocab": 1000}
VERIFY_CASES = {"r5w4": (5, 4, 31), "r8w1": (8, 1, 32), "r6w8": (6, 8, 33), "r16w3": (16, 3, 34)}


def verify_inputs(R: int, W: int, seed: int):
    """logits [R, W, V] fp32, inp [R, W + 4] int64 (W tokens, offset, timestamps so far, last timestamp, first
    generated position), notime [R] bool. The drafted tokens mostly follow the timestamp grammar (a start time
    first, text, an end time at or after it, then a start time or <eos>), sometimes not; the logits favour the
    next drafted token at most positions (so drafts get accepted), timestamps and <eos> elsewhere (so every
    branch of the rules decides some argmax)."""
    rl = VERIFY_RULES
    V, ft, lt, eos = rl["vocab"], rl["first_time"], rl["last_time"], rl["eos"]
    g = torch.Generator().manual_seed(seed)

    def rnd(lo, hi):  # uniform integer in [lo, hi]
        return int(torch.randint(lo, hi + 1, (1,), generator=g))

    def u():
        return float(torch.rand(1, generator=g))

    inp = torch.zeros(R, W + 4, dtype=torch.long)
    notime = torch.rand(R, generator=g) < 0.25
    for r in range(R):
        first = rnd(-1, W - 1)
        count, last = rnd(0, 6), (rnd(ft, lt - 100) if u() < 0.8 else -1)
        inp[r, W:] = torch.tensor([rnd(0, 40), count, last, first])
        toks = [rnd(10, ft - 1) if u() < 0.5 else rnd(ft, lt)]
        for i in range(W - 1):  # token i + 1, chosen in the state after position i
            is_t = lambda t: ft <= t <= lt  # noqa: E731
            if i > 0 and is_t(toks[i]):
                count, last = count + 1, max(last, toks[i])
            x = u()
            if x < 0.15:
                t = rnd(0, V - 1)
            elif notime[r]:
                t = rnd(10, ft - 1) if x < 0.9 else eos
            elif i == first:
                t = rnd(ft, lt)
            elif count % 2 == 1:
                t = rnd(10, ft - 1) if x < 0.6 else rnd(min(max(last + 1, ft), lt), lt)
            elif is_t(toks[i]):
                t = eos if x < 0.3 else rnd(min(max(last, ft), lt), lt)
            else:
                t = rnd(ft, lt)
            toks.append(t)
        inp[r, :W] = torch.tensor(toks)
    logits = torch.randn(R, W, V, generator=g) * 2.0
    logits[:, :, ft : lt + 1] += 1.5 * torch.rand(R, W, 1, generator=g)
    logits[:, :, eos] += 3.0 * torch.rand(R, W, generator=g)
    tok = inp[:, :W]
    nxt = torch.cat([tok[:, 1:], tok[:, -1:]], 1)
    boost = (torch.rand(R, W, generator=g) < 0.8).float() * 12.0
    logits.scatter_add_(2, nxt[:, :, None], boost[:, :, None])
    return logits, inp, notime
