"""Per-stage timing of one decoder call from the kernel's %globaltimer stamps (opt-in, profiling only).

The stages are those of the persistent kernel: embedding; per layer QKV, self-attention, out-projection,
cross-Q, cross-attention, cross-out, FFN1, FFN2; output layer; for beam calls select and two reorder stages.
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
    return names + (["SELECT", "REORD_A", "REORD_B"] if beam else [])


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
    names = stage_names(L, beam, cluster=ts.shape[0] == 3 * L + 2 + (3 if beam else 0))
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
