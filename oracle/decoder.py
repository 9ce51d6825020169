"""CPU fp32 restatement of owsm-trt's decoder call and of the selections around it.

TEST INFRASTRUCTURE ONLY. This module is the parity checker: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg may import it. The product path (``owsm_trt_b200``) never calls it and
has no CPU fallback.

Each function restates one reference function (owsm-trt, ``src/owsm_trt/...``), written from its
semantics in torch fp32 on the CPU. The restatement is pinned against vectors the reference itself
produced (``tests/golden/make_golden.py`` → ``tests/golden/*.npz``, checked by ``tests/test_oracle.py``).

Weights are a state dict in the reference's naming (see ``owsm_trt_b200.synthetic``).
Cache / cross layouts follow the sessions: ``self_k/self_v`` [L, R, H, C, dk], ``cross_k/cross_v``
[L, U, H, T, dk] (U = R unless ``cross_row`` maps rows to utterances).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

LN_EPS = 1e-12  # ESPnet LayerNorm eps, src/owsm_trt/modeling.py:25
LOG_ZERO = -1.0e10  # src/owsm_trt/runtime.py:1336


def _ln(x: torch.Tensor, g: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """LayerNorm over the last dim, eps 1e-12 (modeling.py:38-54)."""
    return F.layer_norm(x, (x.shape[-1],), g, b, LN_EPS)


def _lin(sd: dict, name: str, x: torch.Tensor) -> torch.Tensor:
    return x @ sd[name + ".weight"].t() + sd[name + ".bias"]


def decoder_step(
    sd: dict,
    heads: int,
    tokens: torch.Tensor,
    offset: torch.Tensor,
    self_k: torch.Tensor,
    self_v: torch.Tensor,
    cross_k: torch.Tensor,
    cross_v: torch.Tensor,
    enc_len: torch.Tensor | None = None,
    cross_row: torch.Tensor | None = None,
    pe: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """One decoder call: ``Decoder.step`` (src/owsm_trt/modeling.py:501-560).

    tokens [R, S] int64 at positions offset[r] .. offset[r]+S-1; the row attends to its cache slots
    < offset[r] and causally to its S new tokens (modeling.py:527-531, cached_attention :191-209).
    Cross-attention of row r reads utterance ``cross_row[r]`` (default r) and, with ``enc_len``, only its
    first ``enc_len[u]`` frames: the reference's ``Decoder.step`` on ``cross_k[..., :len, :]`` (its T is
    the tensor's length, modeling.py:549-555). Token ids are clamped to [0, V) as the megakernels do
    (src/owsm_trt/megakernel.py:267).

    Returns logits [R, S, V] fp32 and new keys/values [L, 2, R, H, S, dk] (modeling.py:559-560).
    """
    f32 = torch.float32
    R, S = tokens.shape
    L, _, H, C, dk = self_k.shape
    emb = sd["embed.0.weight"].float()
    V, D = emb.shape
    if pe is None:
        from owsm_trt_b200.synthetic import sinusoidal_positions

        pe = sinusoidal_positions(int(offset.max()) + S + 1, D)
    xscale = math.sqrt(D)
    pos = offset[:, None] + torch.arange(S)
    x = emb[tokens.clamp(0, V - 1)] * xscale + pe[pos].to(f32)  # modeling.py:525
    slot = torch.arange(C)
    cache_ok = (slot[None, :] < offset[:, None])[:, None, None, :].expand(R, 1, S, C)
    new_ok = (torch.arange(S)[None, :] <= torch.arange(S)[:, None]).expand(R, 1, S, S)
    mask = torch.cat([cache_ok, new_ok], -1)  # [R, 1, S, C + S]
    rows = torch.arange(R) if cross_row is None else cross_row.long()
    T = cross_k.shape[3]
    if enc_len is None:
        xmask = torch.ones(R, 1, 1, T, dtype=torch.bool)
    else:
        lens = enc_len.long()[rows]
        xmask = (torch.arange(T)[None, :] < lens[:, None])[:, None, None, :]
    new_kv = []
    for i in range(L):
        p = f"decoders.{i}."
        h = _ln(x, sd[p + "norm1.weight"], sd[p + "norm1.bias"])
        q = _lin(sd, p + "self_attn.linear_q", h)
        k = _lin(sd, p + "self_attn.linear_k", h)
        v = _lin(sd, p + "self_attn.linear_v", h)
        q, k, v = (t.reshape(R, S, H, dk).transpose(1, 2) for t in (q, k, v))  # [R, H, S, dk]
        new_kv.append(torch.stack([k, v]))
        qs = q * dk**-0.5
        sc = torch.cat([qs @ self_k[i].float().transpose(-1, -2), qs @ k.transpose(-1, -2)], -1)
        pr = sc.masked_fill(~mask, float("-inf")).softmax(-1)
        o = pr[..., :C] @ self_v[i].float() + pr[..., C:] @ v  # [R, H, S, dk]
        x = x + _lin(sd, p + "self_attn.linear_out", o.transpose(1, 2).reshape(R, S, D))

        h = _ln(x, sd[p + "norm2.weight"], sd[p + "norm2.bias"])
        q2 = _lin(sd, p + "src_attn.linear_q", h).reshape(R, S, H, dk).transpose(1, 2)
        ck, cv = cross_k[i].float()[rows], cross_v[i].float()[rows]  # [R, H, T, dk]
        sc = (q2 * dk**-0.5) @ ck.transpose(-1, -2)
        pr = sc.masked_fill(~xmask, float("-inf")).softmax(-1)
        o2 = pr @ cv
        x = x + _lin(sd, p + "src_attn.linear_out", o2.transpose(1, 2).reshape(R, S, D))

        h = _ln(x, sd[p + "norm3.weight"], sd[p + "norm3.bias"])
        x = x + _lin(sd, p + "feed_forward.w_2", torch.relu(_lin(sd, p + "feed_forward.w_1", h)))
    logits = _lin(sd, "output_layer", _ln(x, sd["after_norm.weight"], sd["after_norm.bias"]))
    return logits.float(), torch.stack(new_kv)


def write_kv(new_kv: torch.Tensor, k: torch.Tensor, v: torch.Tensor, offset: torch.Tensor) -> None:
    """new_kv [L, 2, R, H, S, dk] into caches k/v [L, R, H, C, dk] at slots offset[r] + s, in place
    (``kernels._write_kv``, src/owsm_trt/kernels.py:69-86; ``_Bound.body``'s scatter, runtime.py:1300-1304)."""
    L, _, R, H, S, dk = new_kv.shape
    slots = (offset[:, None] + torch.arange(S, device=offset.device))[None, :, None, :, None].expand(L, R, H, S, dk)
    k.scatter_(3, slots, new_kv[:, 0].to(k.dtype))
    v.scatter_(3, slots, new_kv[:, 1].to(v.dtype))


def argmax_first(logits: torch.Tensor) -> torch.Tensor:
    """Index of the maximum along the last dim, the first one on ties (``torch.argmax``, as
    ``GreedySession._select`` uses, runtime.py:792-797)."""
    mx = logits.max(-1, keepdim=True).values
    V = logits.shape[-1]
    idx = torch.arange(V).expand_as(logits)
    return torch.where(logits == mx, idx, V).min(-1).values


def argmax_notime(logits: torch.Tensor, flags: torch.Tensor, first_time: int, last_time: int) -> torch.Tensor:
    """Argmax over [R, S, V] with ids first_time..last_time excluded in rows whose flag is set (the
    <notimestamps> rows of the ring kernel's fused argmax, src/owsm_trt/megakernel_ring.py:466-470)."""
    masked = logits.clone()
    V = logits.shape[-1]
    ids = torch.arange(V)
    bad = (ids >= first_time) & (ids <= last_time)
    masked[flags.bool()] = masked[flags.bool()].masked_fill(bad, float("-inf"))
    return argmax_first(masked)


def beam_topk(
    logits: torch.Tensor, score: torch.Tensor, active: torch.Tensor, batch: int, beam: int
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Step 1 of ``BeamSession._select`` (src/owsm_trt/runtime.py:1399-1411): fp32 log-softmax over V,
    add the running score, inactive slots LOG_ZERO, top-K over K*V per utterance (rows utterance-major).

    logits [N, V], score [N], active [N] bool -> (new score [N], parent row [N], token [N]). Ties of equal
    candidates go to the lower flat index (k * V + v), the order of a stable sort."""
    N, V = logits.shape
    logp = torch.log_softmax(logits.float(), -1)
    cand = (score[:, None] + logp).masked_fill(~active.bool()[:, None], LOG_ZERO)
    flat = cand.view(batch, beam * V)
    order = torch.sort(flat, dim=-1, descending=True, stable=True)
    top = order.values[:, :beam]
    idx = order.indices[:, :beam]
    row_base = torch.arange(batch)[:, None] * beam
    parent = (idx // V + row_base).reshape(-1)
    token = (idx % V).reshape(-1)
    return top.reshape(-1), parent, token


def reorder_cache(buf: torch.Tensor, parent: torch.Tensor) -> torch.Tensor:
    """``buf.index_select(1, parent)`` on a cache [L, N, H, C, dk] (runtime.py:1412-1413)."""
    return buf.index_select(1, parent.long())


class TimestampRules:
    """ESPnet's timestamp filter, as ``TimestampRules.forbidden`` (src/owsm_trt/runtime.py:457-492)."""

    def __init__(self, notime: int, first_time: int, last_time: int, eos: int, vocab: int):
        self.notime, self.first_time, self.last_time, self.eos = notime, first_time, last_time, eos
        self.ar = torch.arange(vocab)
        self.time = (self.ar >= first_time) & (self.ar <= last_time)

    def is_time(self, t: torch.Tensor) -> torch.Tensor:
        return (t >= self.first_time) & (t <= self.last_time)

    def forbidden(self, notime, first, count, last, prev) -> torch.Tensor:
        ar, time = self.ar, self.time
        last = last[:, None]
        open_pair = (ar == self.eos) | (time & (ar <= last))
        after_end = ((ar < last) | (ar > self.last_time)) & (ar != self.eos)
        closed = torch.where(self.is_time(prev)[:, None], after_end, torch.ones_like(after_end))
        timed = torch.where((count % 2 == 1)[:, None], open_pair, closed)
        timed = torch.where(first[:, None], ~time, timed)
        return torch.where(notime[:, None], time, timed)


def verify_predict(logits: torch.Tensor, inp: torch.Tensor, notime: torch.Tensor | None, rules) -> torch.Tensor:
    """``_Verify.predict`` (src/owsm_trt/runtime.py:1251-1267): the argmax after each window position of
    logits [R, W, V] under the timestamp rules (``rules`` None: plain argmax). ``inp`` [R, W + 4] int64 =
    W tokens, offset, timestamps so far, last timestamp, first generated position; ``notime`` [R] the rows
    whose primer holds <notimestamps>. Restated position by position: the rule state of position i takes the
    row's count / last timestamp and the timestamps the window's own tokens 1 .. i add."""
    if rules is None:
        return argmax_first(logits)
    R, W, V = logits.shape
    flags = torch.zeros(R, dtype=torch.bool) if notime is None else notime.bool()
    st_notime, st_first, st_count, st_last, st_prev = [], [], [], [], []
    for r in range(R):
        row = [int(t) for t in inp[r]]
        count, last = row[W + 1], max(row[W + 2], -1)
        for i in range(W):
            if i > 0 and rules.first_time <= row[i] <= rules.last_time:
                count += 1
                last = max(last, row[i])
            st_notime.append(bool(flags[r]))
            st_first.append(row[W + 3] == i)
            st_count.append(count)
            st_last.append(last)
            st_prev.append(row[i])
    bad = rules.forbidden(
        torch.tensor(st_notime), torch.tensor(st_first), torch.tensor(st_count), torch.tensor(st_last),
        torch.tensor(st_prev),
    )
    return argmax_first(logits.reshape(R * W, V).masked_fill(bad, float("-inf"))).view(R, W)


def verify_accept(pred: torch.Tensor, inp: torch.Tensor, eos: int) -> torch.Tensor:
    """``_Verify.accept`` (src/owsm_trt/runtime.py:1269-1278) per row: positions before the head's end s
    (inp's first-position column, at least 0) count as accepted; then drafted token i + 1 is accepted while it
    equals the argmax after position i and is not <eos>. Returns [R, 2] = (drafted tokens accepted, the argmax
    after the last accepted position)."""
    R, W = pred.shape
    out = torch.zeros(R, 2, dtype=torch.long)
    for r in range(R):
        s = max(int(inp[r, W + 3]), 0)
        end = 0
        while end < W - 1 and (end < s or (int(pred[r, end]) == int(inp[r, end + 1]) and int(inp[r, end + 1]) != eos)):
            end += 1
        out[r, 0] = end - s
        out[r, 1] = pred[r, end]
    return out
