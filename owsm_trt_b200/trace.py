"""Per-stage timing of one decoder call from the kernel's %globaltimer stamps (opt-in, profiling only).

The stages are those of the persistent kernel: embedding; per layer QKV, self-attention, out-projection,
cross-Q, cross-attention, cross-out, FFN1, FFN2; output layer; for beam calls select and the cache reorder.
``profile(kernel, run)`` runs ``run`` once with stamps on and returns them; ``summary`` averages them per
stage kind: the stage's span between consecutive grid-barrier releases, the slowest CTA's work, and the
mean time CTAs spend in the barrier."""

from __future__ import annotations

import torch

from . import _lib

KINDS = ["QKV", "SATT", "WO", "CQ", "XATT", "WCO", "F1", "F2"]


def stage_names(L: int, beam: bool, cluster: bool = False) -> list[str]:
    """Stage names of a call: the grid-stage kernel's eight per layer, or the cluster kernel's three."""
    if cluster:
        names = ["EMBED"] + [("S1", "S2", "S3")[i % 3] for i in range(3 * L)] + ["OUT"]
    else:
        names = ["EMBED"] + [KINDS[i % 8] for i in range(8 * L)] + ["OUT"]
    return names + (["SELECT", "REORDER"] if beam else [])


def profile(kernel, run) -> torch.Tensor:
    """Stamps [stages, programs, 4] (start, end, barrier exit, ns waiting for ring slots) of one call of `run`."""
    lib = _lib.lib()
    n = lib.owsm_dec_plan_stages(run.plan, int(run.beam))
    P = kernel._plan_info(run.plan)[0]
    # stage stamps [n, P, 4], then an event log of 128 stamps per CTA
    ts = torch.zeros(n * P * 4 + P * 128, dtype=torch.int64, device=kernel.device)
    _lib.check(lib.owsm_dec_plan_trace(run.plan, ts.data_ptr()), "owsm_dec_plan_trace")
    try:
        run()
        torch.cuda.synchronize(kernel.device)
    finally:
        _lib.check(lib.owsm_dec_plan_trace(run.plan, None), "owsm_dec_plan_trace")
    kernel.check()
    ts = ts.cpu()
    stages = ts[: n * P * 4].view(n, P, 4)
    stages.events = ts[n * P * 4 :].view(P, 128)
    return stages


def summary(ts: torch.Tensor, L: int, beam: bool = False) -> dict[str, dict[str, float]]:
    """Per stage kind, in microseconds: span (barrier release to barrier release), work (slowest CTA's stage
    time), wait (mean barrier time), ring (the most a CTA waited for its data in the stage), count."""
    names = stage_names(L, beam, cluster=ts.shape[0] == 3 * L + 2 + (2 if beam else 0))
    t = ts.double()
    start, end, exit_ = t[..., 0], t[..., 1], t[..., 2]
    t0 = start.min()
    out: dict[str, dict[str, float]] = {}
    prev = start[0].min()
    for g, name in enumerate(names):
        rel = exit_[g].max() if g < len(names) - 1 else end[g].max()
        span = float(rel - prev) / 1e3
        work = float((end[g] - start[g]).max()) / 1e3
        wait = float((exit_[g] - end[g]).mean()) / 1e3 if g < len(names) - 1 else 0.0
        prev = rel
        ring = float(t[g, :, 3].max()) / 1e3
        d = out.setdefault(name, {"count": 0, "span_us": 0.0, "work_us": 0.0, "wait_us": 0.0, "ring_us": 0.0})
        d["count"] += 1
        d["span_us"] += span
        d["work_us"] += work
        d["wait_us"] += wait
        d["ring_us"] += ring
    for d in out.values():
        for k in ("span_us", "work_us", "wait_us", "ring_us"):
            d[k] = round(d[k] / d["count"], 3)
    out["_total_us"] = {"count": 1, "span_us": round(float(end[-1].max() - t0) / 1e3, 2), "work_us": 0.0, "wait_us": 0.0}
    return out


def main() -> None:
    """``python -m owsm_trt_b200.trace [--batch B] [--path 0|1]``: the stage table of one greedy call of the
    1B-shaped decoder (seeded weights, the benchmark's synthetic encoder lengths, cache position 100)."""
    import argparse
    import json

    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--path", type=int, default=0, help="0: cluster kernel where it applies, 1: grid-stage kernel")
    ap.add_argument("--events", type=int, nargs="*", default=[], help="CTAs whose event log to print")
    ap.add_argument("--beam", type=int, default=0, help="beam width: a beam call of --batch utterances x beam rows")
    ap.add_argument("--from-stage", type=int, default=0, help="the stage at which the event logs start")
    args = ap.parse_args()
    from .decoder import B200Decoder
    from .synthetic import MEDIUM_1B, decoder_state_dict, make_workload

    d, dev, K = MEDIUM_1B, torch.device("cuda", 0), max(args.beam, 1)
    B = args.batch * K
    sd = decoder_state_dict(d, 0, False)
    k = B200Decoder.from_state_dict(sd, d.H, dev)
    k.set_path(args.path)
    ck, cv, enc_len, prefix, kc, vc = make_workload(d, sd, dev, B, 5, rows_per_utt=K)
    tok = prefix[:, -1:].to(dev).contiguous()
    off = torch.full((B,), 100, dtype=torch.long, device=dev)
    logits = torch.zeros(B, 1, d.V, device=dev)
    new_kv = torch.zeros(d.L, 2, B, d.H, 1, d.dk, device=dev, dtype=torch.float16)
    if args.beam:  # (every utterance at the full 750 frames, as the benchmark's beam line)
        el = torch.full((args.batch,), ck.shape[3], dtype=torch.int32, device=dev)
        score = torch.zeros(B, device=dev)
        active = torch.ones(B, dtype=torch.uint8, device=dev)
        parent = torch.zeros(B, dtype=torch.long, device=dev)
        run = k.beam_fn(tok, off, kc, vc, ck, cv, logits, new_kv, score, active, parent, tok[:, 0].clone(),
                        beam=K, enc_len=el)  # fmt: skip
    else:
        run = k.step_fn(tok, off, kc, vc, ck, cv, logits, new_kv, pred=tok, enc_len=enc_len.to(dev))
    for _ in range(3):
        run()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        run()
    e1.record()
    torch.cuda.synchronize(dev)
    _lib.check(_lib.lib().owsm_dec_plan_trace_from(run.plan, args.from_stage), "owsm_dec_plan_trace_from")
    ts = profile(k, run)
    s = summary(ts, d.L, beam=bool(args.beam))
    programs, slots, scratch = k._plan_info(run.plan)
    print(json.dumps({"kernel": k.plan_kernel(run), "programs": programs, "ring_slots": slots, "batch": B, "beam": args.beam, "us_per_call": round(e0.elapsed_time(e1) / 20 * 1e3, 1),
                      "stages": s}, indent=1))  # fmt: skip
    for c in args.events:
        print(json.dumps({"cta": c, "events": event_log(ts, c)}))


def event_log(ts: torch.Tensor, c: int) -> list[list[float]]:
    """CTA c's event log as [tag, µs since the kernel's first stage start] in the order recorded (the first 64
    events of the call: tags 21, 22, 20, 23 inside a LayerNorm (entry, padding zeroed, a row's loads done,
    a team's first barrier passed), 50-57 the steps of an attention stage, 60-63 of
    an FFN stage, 70-72 of the output stage, 80-82 inside an attention unit: queries ready, cached positions
    done, new positions done, 90-93 inside a split projection chunk: data ready, partial product done, team
    barrier passed, epilogue done)."""
    ev = ts.events[c]
    t0 = int(ts[0, :, 0].min())
    out = []
    for i in range(0, ev.numel() - 1, 2):
        t, tag = int(ev[i]), int(ev[i + 1]) & 0xFF
        if t == 0:
            break
        out.append([tag, round((t - t0) / 1e3, 3)])
    return out


if __name__ == "__main__":
    main()
