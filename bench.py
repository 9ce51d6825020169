"""Decoder-step throughput on B200: decoded tokens/s and us/step against the HBM roofline.

Headline: the 18-layer d=1024 OWSM-v4-medium-shaped decoder, fp16, greedy, 16
utterances per GPU, 200 decoder steps each (a 4-token prefix at positions 0-3, then positions 4..203, the KV cache
growing to 204 slots in a 256-slot buffer), encoder memory N(0,1) [16, 750, 1024] projected to cross K/V once,
encoder lengths uniform in [300, 750] (key-padding mask). Weights: seeded synthetic N(0,0.02) (no checkpoints
here). A *step* is one decoder call over the batch (one launch of the persistent kernel); the greedy argmax feeds
back on the device (the pred buffer is the next call's token buffer). ``--steps K`` timed steps sample the 200
positions evenly (step i at position 4 + i*200//K for K < 200, whole passes otherwise), so any K measures the
configuration's position mix; the algorithmic bytes are those of the timed positions.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched by torchrun, one process per GPU; every rank decodes its own 16 utterances (weak scaling, no
collective on the data path); the timed region is bracketed by barriers and the max over ranks is reported.
``box_scale`` adds configs[4] at every N: 1024 utterances in all, 64 per GPU per batch, 200 steps each, as
sequential batches per rank (strong scaling), device-timed, max over ranks.
On one GPU, ``secondary`` adds batch 1 (configs[0]'s shape, the roofline target), beam 5 x 3,
batch 64, and the 6-layer d=768 model at batch 1 and 64; ``cpu_baseline`` times the reference
algorithm's fp32 CPU restatement on a bounded sample of the headline workload and ``parity`` compares the
kernel's logits with it on those steps (teacher-forced).
``--impl reference`` times the reference's own CPU path (owsm-trt's ``Decoder.step`` from the pip-installed copy
under baseline/_ref, fp32, all host cores; the oracle restatement when that is absent) on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from owsm_trt_b200.synthetic import CACHE, PREFIX, T_ENC, make_workload  # noqa: E402

METRIC = "decoded tokens/s (greedy decoder step, 1B OWSM decoder, batch 16 per GPU)"
UNIT = "tokens/s"
BATCH, STEPS_PER_UTT = 16, 200
BOX_UTTS, BOX_BATCH = 1024, 64
FALLBACK_HBM_GBS = 6650.0
REF_DIR = ROOT / "baseline" / "_ref"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-box-scale", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    return ap.parse_args()


def positions(K: int) -> list[int]:
    """Cache positions of K timed steps: the 200 decode positions 4..203 sampled evenly (whole passes when
    K >= 200)."""
    if K >= STEPS_PER_UTT:
        return [PREFIX + i % STEPS_PER_UTT for i in range(K)]
    return [PREFIX + (i * STEPS_PER_UTT) // K for i in range(K)]


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:  # noqa: BLE001
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(batch: int) -> int | None:
    """DRAM bytes (read + write) of one decoder launch of this workload, from the committed ncu summary of
    the same command (profiles/decoder_cl_kernel_b16_full.md); None for other batch sizes or if absent."""
    p = ROOT / "profiles" / "decoder_cl_kernel_b16_full.md"
    if batch != BATCH or not p.exists():
        return None
    m = re.search(r"^traffic_bytes_per_launch:\s*(\d+)", p.read_text(), re.M)
    return int(m.group(1)) if m else None


def step_bytes(d, batch: int, pos: int, enc_lens: list[int], rows_per_utt: int = 1) -> int:
    """Algorithmic bytes of one decoder call: fp16 weights once, fp32 biases, each utterance's cross K/V
    frames once, each row's self-KV slots < pos, its new K/V, logits (fp32), embedding (fp16) and
    positional (fp32) rows."""
    L, D, F, V = d.L, d.D, d.F, d.V
    p_w = L * (6 * D * D + 2 * D * F) + V * D
    p_bias = L * (7 * D + F) + V
    cross = sum(2 * L * 2 * n * D for n in enc_lens)
    rows = batch * (2 * L * 2 * D * pos + 2 * L * 2 * D + 4 * V + 2 * D + 4 * D)
    return 2 * p_w + 4 * p_bias + cross + rows


class Clocks:
    """nvidia-smi samples of this GPU's clocks and throttle reasons while a region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap,pci.bus_id")  # fmt: skip

    def __init__(self, dev: torch.device):
        props = torch.cuda.get_device_properties(dev)
        self.bus = getattr(props, "pci_bus_id", None)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )  # fmt: skip
        except OSError:
            self.proc = None
        time.sleep(0.2)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def summary(self) -> dict:
        """Median SM clock under load, max clock and the throttle reasons seen, for this process's GPU
        (matched by PCI bus; if that fails, the GPU with the highest median power draw)."""
        by_bus: dict[str, list] = {}
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                row = (float(f[0]), float(f[1]), float(f[2]) if f[2] not in ("[N/A]", "N/A") else 0.0, f[4:8])
            except ValueError:
                continue
            by_bus.setdefault(f[8].lower(), []).append(row)
        if not by_bus:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sel = None
        if self.bus is not None:
            want = f"{int(self.bus):02x}:00.0"
            for bus, rows in by_bus.items():
                if bus.endswith(want):
                    sel = rows
        if sel is None:
            sel = max(by_bus.values(), key=lambda rs: statistics.median(r[2] for r in rs))
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in sel for n, v in zip(names, r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in sel), "sm_max_mhz": max(r[1] for r in sel),
                "reasons": reasons, "samples": len(sel)}  # fmt: skip


def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))  # fmt: skip
        else:  # host-only runs of the rank logic (tests)
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        dist.barrier()


class Greedy:
    """One greedy batch on the kernel: the prefix call (untimed) and one closure per decode position, the argmax
    of each call feeding the next (the pred buffer is the token buffer)."""

    def __init__(self, kern, d, dev, B: int, seed: int, rows_per_utt: int = 1, enc_len_mode: str = "uniform",
                 sd=None, steps: int = STEPS_PER_UTT):  # fmt: skip
        self.d, self.B = d, B
        ck, cv, enc_len, prefix, kc, vc = make_workload(d, sd, dev, B, seed, rows_per_utt)
        if enc_len_mode == "full":  # the reference pads to 30 s: every frame attended (no mask)
            enc_len = torch.full_like(enc_len, T_ENC)
        self.ck, self.cv, self.enc_len, self.prefix, self.kc, self.vc = ck, cv, enc_len, prefix, kc, vc
        self.enc_len_d = enc_len.to(dev)
        # the prefix in one call, or one position per call where rows x 4 exceeds what a call takes
        S = PREFIX if B * PREFIX <= 64 else 1
        lg_p = torch.zeros(B, S, d.V, device=dev)
        kv_p = torch.zeros(d.L, 2, B, d.H, S, d.dk, device=dev, dtype=torch.float16)
        pr_p = torch.zeros(B, S, dtype=torch.long, device=dev)
        pre = prefix.to(dev)
        for p0 in range(0, PREFIX, S):
            off = torch.full((B,), p0, dtype=torch.long, device=dev)
            kern.step_fn(pre[:, p0 : p0 + S].contiguous(), off, kc, vc, ck, cv, lg_p, kv_p, pred=pr_p,
                         enc_len=self.enc_len_d)()  # fmt: skip
        self.tok = pr_p[:, -1:].clone()
        offs = (PREFIX + torch.arange(steps, device=dev))[:, None].expand(steps, B).contiguous()
        self.offs = offs
        self.logits = torch.zeros(B, 1, d.V, device=dev)
        self.new_kv = torch.zeros(d.L, 2, B, d.H, 1, d.dk, device=dev, dtype=torch.float16)
        self.runs = [kern.step_fn(self.tok, offs[j], kc, vc, ck, cv, self.logits, self.new_kv, pred=self.tok,
                                  enc_len=self.enc_len_d) for j in range(steps)]  # fmt: skip
        self.launches = kern.launches(self.runs[0])

    def run_at(self, pos: int) -> None:
        self.runs[pos - PREFIX]()

    def bytes_at(self, pos: int) -> int:
        return step_bytes(self.d, self.B, pos, self.enc_len.tolist())


def timed(fn, n: int, dev) -> float:
    """ms of n calls of fn(i) on the current stream (CUDA events, synchronised on both sides)."""
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    s.record()
    for i in range(n):
        fn(i)
    e.record()
    torch.cuda.synchronize(dev)
    return s.elapsed_time(e)


def run_ours(args, world, rank, local) -> dict | None:
    from owsm_trt_b200.build import build
    from owsm_trt_b200.decoder import B200Decoder
    from owsm_trt_b200.synthetic import MEDIUM_1B, decoder_state_dict

    if rank == 0:
        build()
    barrier(world)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    d = MEDIUM_1B
    sd = decoder_state_dict(d, 0, False)
    kern = B200Decoder.from_state_dict(sd, d.H, dev)
    B = args.batch
    wl = Greedy(kern, d, dev, B, 1000 + rank, sd=sd)
    K, W = args.steps, max(3, args.warmup)
    order = positions(K)
    for i in range(W):
        wl.run_at(order[i % K])
    torch.cuda.synchronize(dev)
    kern.check()
    barrier(world)
    with Clocks(dev) as clk:
        ms = timed(lambda i: wl.run_at(order[i]), K, dev)
    kern.check()
    barrier(world)
    ms_max = max_over_ranks(ms, world, dev)
    per_step_ms = ms_max / K
    value = B * K * world / (ms_max / 1e3)

    # end to end through the public API: tokens and offsets from pinned host memory each step, the argmax back
    # to the host each step (greedy feedback through the host, as a caller without on-device decoding does)
    h_tok = torch.zeros(B, 1, dtype=torch.long).pin_memory()
    h_off = torch.zeros(B, dtype=torch.long).pin_memory()
    h_pred = torch.zeros(B, 1, dtype=torch.long).pin_memory()
    d_tok = torch.zeros(B, 1, dtype=torch.long, device=dev)
    d_off = torch.zeros(B, dtype=torch.long, device=dev)
    d_pred = torch.zeros(B, 1, dtype=torch.long, device=dev)
    run_e2e = kern.step_fn(d_tok, d_off, wl.kc, wl.vc, wl.ck, wl.cv, wl.logits, wl.new_kv, pred=d_pred,
                           enc_len=wl.enc_len_d)  # fmt: skip
    h_tok.copy_(wl.tok.cpu())
    K2 = min(K, 400)
    order2 = positions(K2)
    stream = torch.cuda.current_stream(dev)

    def e2e_steps(n, order_):
        for i in range(n):
            h_off.fill_(order_[i % len(order_)])
            d_tok.copy_(h_tok, non_blocking=True)
            d_off.copy_(h_off, non_blocking=True)
            run_e2e()
            h_pred.copy_(d_pred, non_blocking=True)
            stream.synchronize()
            h_tok.copy_(h_pred)

    e2e_steps(W, order2)
    barrier(world)
    t0 = time.perf_counter()
    e2e_steps(K2, order2)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world, dev)
    e2e_value = B * K2 * world / e2e_s

    hbm, hbm_src = peaks()
    avg_bytes = sum(wl.bytes_at(p) for p in order) / K
    achieved = avg_bytes / (per_step_ms / 1e3) / 1e9  # per GPU (each GPU's step moves avg_bytes)
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(per_step_ms, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) encoder memory)",
        "config": {"workload": "BASELINE configs[1]: 1B decoder greedy, 16 utterances/GPU, 200 steps, enc_len U[300,750]",
                   "global_batch": B * world, "seq_len": PREFIX + STEPS_PER_UTT, "parallelism": f"dp{world} (utterance shards, no collective)",
                   "cache_slots": CACHE, "enc_frames": T_ENC,
                   "timed_positions": f"{order[0]}..{max(order)} ({K} steps, evenly over the 200 decode positions)",
                   "l2": "inputs larger than L2 (631 MB of weights per step > 126 MB)"},  # fmt: skip
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": 2 * B * 8,
                "d2h_bytes_per_step": B * 8, "steps": K2},  # fmt: skip
        "gpu_launches": K * wl.launches,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": profiled_traffic(B), "peak_source": hbm_src,
                     "algorithmic_bytes_per_step": int(avg_bytes)},  # fmt: skip
        "clocks": clk.summary(),
        "us_per_step": round(per_step_ms * 1e3, 2),
    }
    if not args.no_box_scale:
        result["box_scale"] = box_scale(kern, d, dev, world, rank, hbm, sd)
    if rank == 0 and world == 1 and not args.no_secondary:
        result["secondary"] = secondary(kern, sd, d, dev, hbm)
    if rank == 0 and world == 1:
        result["cpu_baseline"], result["parity"] = cpu_baseline(kern, sd, d, wl, dev, args.cpu_seconds)
    kern.close()
    return result if rank == 0 else None


def box_scale(kern, d, dev, world: int, rank: int, hbm: float, sd) -> dict:
    """1024 utterances in all, 64 per batch on each GPU, 200 greedy steps per batch, batches run one
    after another on a rank (1024 / N / 64 of them; every batch reuses one set of buffers: the work of a step does
    not depend on the values). Device-timed (CUDA events around all of a rank's steps), max over ranks."""
    per_rank = BOX_UTTS // world
    nb = max(1, per_rank // BOX_BATCH)
    wl = Greedy(kern, d, dev, BOX_BATCH, 2000 + rank, sd=sd)
    for p in range(PREFIX, PREFIX + 5):
        wl.run_at(p)
    torch.cuda.synchronize(dev)
    kern.check()
    barrier(world)
    n = nb * STEPS_PER_UTT
    ms = timed(lambda i: wl.run_at(PREFIX + i % STEPS_PER_UTT), n, dev)
    kern.check()
    ms_max = max_over_ranks(ms, world, dev)
    avg = statistics.mean(wl.bytes_at(PREFIX + j) for j in range(STEPS_PER_UTT))
    us = ms_max * 1e3 / n
    gbs = avg / (us * 1e-6) / 1e9
    return {"workload": "BASELINE configs[4]: 1024 utterances, 64 per GPU per batch, 200 steps each, enc_len U[300,750]",
            "value": round(nb * BOX_BATCH * STEPS_PER_UTT * world / (ms_max / 1e3), 1), "unit": UNIT,
            "scaling": "strong (1024 utterances in all)", "batches_per_gpu": nb, "us_per_step": round(us, 2),
            "achieved_gbs": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 4), "algorithmic_bytes_per_step": int(avg),
            "gpu_launches_per_step": wl.launches}  # fmt: skip


def _greedy_line(kern, d, dev, hbm, B, seed, sd, enc_len_mode="uniform") -> dict:
    wl = Greedy(kern, d, dev, B, seed, enc_len_mode=enc_len_mode, sd=sd)
    for p in range(PREFIX, PREFIX + 10):
        wl.run_at(p)
    ms = timed(lambda i: wl.run_at(PREFIX + i), STEPS_PER_UTT, dev)
    kern.check()
    us = ms * 1e3 / STEPS_PER_UTT
    avg = statistics.mean(wl.bytes_at(PREFIX + j) for j in range(STEPS_PER_UTT))
    gbs = avg / (us * 1e-6) / 1e9
    return {"us_per_step": round(us, 2), "tokens_per_s": round(B / (us * 1e-6), 1), "achieved_gbs": round(gbs, 1),
            "frac_of_hbm": round(gbs / hbm, 4), "algorithmic_bytes_per_step": int(avg), "kernel": kern.plan_kernel(wl.runs[0]),
            "gpu_launches_per_step": wl.launches, "steps": STEPS_PER_UTT, "enc_len": enc_len_mode}  # fmt: skip


def secondary(kern, sd, d, dev, hbm) -> dict:
    """The other BASELINE shapes on one GPU (us/step, roofline fraction): greedy b1 (configs[0]'s shape, the
    headline roofline target; the reference pads to 30 s, so all 750 frames), beam 5 x batch 3 (configs[2]: fused
    select + reorder), greedy b64 (configs[4]'s per-GPU batch), and the small model at b1 and b64."""
    from owsm_trt_b200.decoder import B200Decoder
    from owsm_trt_b200.synthetic import SMALL, decoder_state_dict

    out = {"greedy_b1": _greedy_line(kern, d, dev, hbm, 1, 77, sd, "full")}
    # beam 5 x 3 utterances, 150 steps, cross K/V once per utterance
    Bu, Kb = 3, 5
    N = Bu * Kb
    ck, cv, enc_len, prefix, kc, vc = make_workload(d, sd, dev, N, 91, rows_per_utt=Kb)
    el = torch.full((Bu,), T_ENC, dtype=torch.int32, device=dev)
    tok = prefix[:, -1:].to(dev).contiguous()
    offs = (PREFIX + torch.arange(150, device=dev))[:, None].expand(150, N).contiguous()
    logits = torch.zeros(N, 1, d.V, device=dev)
    new_kv = torch.zeros(d.L, 2, N, d.H, 1, d.dk, device=dev, dtype=torch.float16)
    score = torch.zeros(N, device=dev)
    active = torch.ones(N, dtype=torch.uint8, device=dev)
    parent = torch.zeros(N, dtype=torch.long, device=dev)
    token = tok[:, 0]
    # the hypotheses' record of common cache slots (the session keeps it so): all PREFIX slots at the start
    shared = torch.full((Bu, Kb, Kb), PREFIX, dtype=torch.int32, device=dev)
    runs = [kern.beam_fn(tok, offs[j], kc, vc, ck, cv, logits, new_kv, score, active, parent, token, beam=Kb,
                         enc_len=el, shared=shared) for j in range(150)]  # fmt: skip
    for i in range(5):
        runs[i]()
    shared.fill_(PREFIX)  # (the timed steps restart at slot PREFIX: the rows' later slots are rewritten)
    ms = timed(lambda i: runs[i](), 150, dev)
    kern.check()
    us = ms * 1e3 / 150
    avg = statistics.mean(step_bytes(d, N, PREFIX + j, [T_ENC] * Bu) for j in range(150))
    gbs = avg / (us * 1e-6) / 1e9
    out["beam5_batch3"] = {"us_per_step": round(us, 2), "tokens_per_s": round(N / (us * 1e-6), 1),
                           "achieved_gbs": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 4),
                           "algorithmic_bytes_per_step": int(avg), "kernel": kern.plan_kernel(runs[0])}  # fmt: skip
    del runs, ck, cv, kc, vc
    out["greedy_b64"] = _greedy_line(kern, d, dev, hbm, 64, 78, sd)
    sds = decoder_state_dict(SMALL, 0, False)
    ks = B200Decoder.from_state_dict(sds, SMALL.H, dev)
    out["small_b1"] = _greedy_line(ks, SMALL, dev, hbm, 1, 79, sds, "full")
    out["small_b64"] = _greedy_line(ks, SMALL, dev, hbm, 64, 80, sds, "full")
    ks.close()
    return out


def cpu_baseline(kern, sd, d, wl: Greedy, dev, seconds: float) -> tuple[dict, dict]:
    """The reference algorithm's fp32 CPU path (the oracle restatement of Decoder.step, all host cores) on a
    bounded sample of the headline workload: its prefix call and then decode steps until ``seconds`` of oracle
    time have passed. The same calls run on the kernel (its own fp16 cache, fed the oracle's tokens: teacher-forced)
    and oracle.parity tallies the logits' max-abs error and the argmax agreement (near-ties counted).
    Returns (cpu_baseline, parity)."""
    from oracle import parity
    from owsm_trt_b200.synthetic import sinusoidal_positions

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    B = wl.B
    ck32, cv32 = wl.ck.float().cpu(), wl.cv.float().cpu()
    pe = sinusoidal_positions(CACHE + 1, d.D)
    kc32 = torch.zeros(d.L, B, d.H, CACHE, d.dk)
    vc32 = torch.zeros_like(kc32)
    kc16 = torch.zeros(d.L, B, d.H, CACHE, d.dk, device=dev, dtype=torch.float16)
    vc16 = torch.zeros_like(kc16)
    enc_len = wl.enc_len.long()

    def gpu_step(tok, off):
        R, S = tok.shape
        logits = torch.zeros(R, S, d.V, device=dev)
        new_kv = torch.zeros(d.L, 2, R, d.H, S, d.dk, device=dev, dtype=torch.float16)
        pred = torch.zeros(R, S, dtype=torch.long, device=dev)
        kern.step_fn(tok.to(dev), off.to(dev), kc16, vc16, wl.ck, wl.cv, logits, new_kv, pred=pred,
                     enc_len=wl.enc_len_d)()  # fmt: skip
        torch.cuda.synchronize(dev)
        kern.check()
        return logits.cpu(), pred.cpu()

    from oracle import decoder as ref

    tally = parity.Tally()
    tok, off = wl.prefix, torch.zeros(B, dtype=torch.long)
    n_dec, t_dec = 0, 0.0
    while True:
        t0 = time.perf_counter()
        with torch.no_grad():
            lo, kvo = ref.decoder_step(sd, d.H, tok, off, kc32, vc32, ck32, cv32, enc_len=enc_len, pe=pe)
            ref.write_kv(kvo, kc32, vc32, off)
        dt = time.perf_counter() - t0
        tally.oracle_s += dt
        lg, pred = gpu_step(tok, off)
        if tok.shape[1] > 1:  # the prefix call: every position compared
            for s_ in range(tok.shape[1]):
                tally.add_greedy(lo[:, s_], lg[:, s_], pred[:, s_])
        else:
            tally.add_greedy(lo[:, -1], lg[:, -1], pred[:, -1])
            n_dec += 1
            t_dec += dt
        off = off + tok.shape[1]
        tok = ref.argmax_first(lo[:, -1])[:, None]
        if tally.oracle_s > seconds or int(off[0]) >= PREFIX + STEPS_PER_UTT:
            break
    el = tally.oracle_s
    base = {"value": round(B * n_dec / t_dec, 2) if n_dec else None, "unit": UNIT,
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"the prefix call and {n_dec} decode calls of batch {B} (positions {PREFIX}..{PREFIX + n_dec - 1}) "
                      f"of the headline workload, 1B decoder, fp32, oracle restatement of owsm-trt Decoder.step; "
                      f"value = decode tokens / decode-call seconds ({el:.1f} s of oracle time in all)"}  # fmt: skip
    par = tally.summary()
    par["workload"] = "headline (b16, masked enc_len), teacher-forced: both fed the oracle's argmax"
    return base, par


def _ref_decoder(d, sd):
    """owsm-trt's own ``Decoder`` (src/owsm_trt/modeling.py:471-560) from the pip-installed copy under
    baseline/_ref with the synthetic weights, or None if that copy is absent."""
    if not (REF_DIR / "owsm_trt").is_dir():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.append(str(REF_DIR))
    from owsm_trt.config import OWSMConfig
    from owsm_trt.modeling import Decoder

    cfg = OWSMConfig(vocab_size=d.V, d_model=d.D, n_heads=d.H, enc_layers=0, enc_ffn=d.F, cgmlp_units=d.F,
                     cgmlp_kernel=31, merge_kernel=31, subsample="conv2d", dec_layers=d.L, dec_ffn=d.F, dec_heads=d.H,
                     n_mels=128, n_fft=512, win_length=400, hop_length=160, sample_rate=16000, speech_seconds=30.0,
                     time_resolution=0.02)  # fmt: skip
    dec = Decoder(cfg).eval().requires_grad_(False)
    dec.load_state_dict(sd, strict=True)
    return dec


def run_reference(args, world, rank) -> dict | None:
    """The reference's CPU path on the host cores, same metric / config / timed positions as the GPU arm; rank 0
    only. owsm-trt's own ``Decoder.step`` (fp32, the path of TorchBackend, src/owsm_trt/runtime.py:93-115) from
    baseline/_ref; without it, the oracle restatement (oracle/decoder.py)."""
    if rank != 0:
        return None
    from owsm_trt_b200.synthetic import MEDIUM_1B, decoder_state_dict

    d = MEDIUM_1B
    B = args.batch
    sd = decoder_state_dict(d, 0, False)
    torch.set_num_threads(os.cpu_count() or 1)
    K = max(1, args.steps)
    order = positions(K)
    if K > 60:  # a bounded sample of the same positions (about 10 s a step at most)
        order = order[:: (K + 59) // 60]
    warm = 3  # the timing rules' minimum of warm-up steps
    g = torch.Generator().manual_seed(5)
    kc = torch.zeros(d.L, B, d.H, CACHE, d.dk)
    vc = torch.zeros_like(kc)
    ck = torch.randn(d.L, B, d.H, T_ENC, d.dk, generator=g).half().float()
    cv = torch.randn(d.L, B, d.H, T_ENC, d.dk, generator=g).half().float()
    tok = torch.randint(0, d.V, (B, 1), generator=g)
    dec = _ref_decoder(d, sd)
    if dec is not None:
        kind, how = "reference", "owsm-trt Decoder.step (baseline/_ref, unmodified), fp32, all 750 frames (no mask: the reference pads to 30 s)"
        sk, sv = [kc[i] for i in range(d.L)], [vc[i] for i in range(d.L)]
        xk, xv = [ck[i] for i in range(d.L)], [cv[i] for i in range(d.L)]

        def one(pos):
            nonlocal tok
            off = torch.full((B,), pos, dtype=torch.long)
            lg, kv = dec.step(tok, off, sk, sv, xk, xv)
            for i in range(d.L):  # the session's cache write (runtime.py:608-616)
                sk[i].index_copy_(2, off[:1], kv[i, 0])
                sv[i].index_copy_(2, off[:1], kv[i, 1])
            tok = lg[:, -1].argmax(-1)[:, None]
    else:
        from oracle import decoder as ref
        from owsm_trt_b200.synthetic import sinusoidal_positions

        kind, how = "port", "oracle restatement of owsm-trt Decoder.step (baseline/_ref absent), fp32, enc_len U[300,750]"
        enc_len = torch.randint(300, T_ENC + 1, (B,), generator=g)
        pe = sinusoidal_positions(CACHE + 1, d.D)

        def one(pos):
            nonlocal tok
            off = torch.full((B,), pos, dtype=torch.long)
            lg, kv = ref.decoder_step(sd, d.H, tok, off, kc, vc, ck, cv, enc_len=enc_len, pe=pe)
            ref.write_kv(kv, kc, vc, off)
            tok = ref.argmax_first(lg[:, -1])[:, None]

    with torch.no_grad():
        for i in range(warm):
            one(order[i % len(order)])
        t0 = time.perf_counter()
        for p in order:
            one(p)
        el = time.perf_counter() - t0
    steps = len(order)
    value = B * steps / el
    return {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": warm,
        "ms_per_step": round(el / steps * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": "BASELINE configs[1]: 1B decoder greedy, 16 utterances/GPU, 200 steps, enc_len U[300,750]",
                   "global_batch": B, "seq_len": PREFIX + STEPS_PER_UTT, "parallelism": "cpu (host cores)",
                   "cache_slots": CACHE, "enc_frames": T_ENC,
                   "timed_positions": f"{order[0]}..{max(order)} ({steps} steps of the GPU arm's {K})"},  # fmt: skip
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": torch.get_num_threads(), "kind": kind,
                         "sample": f"{steps} timed decoder calls of batch {B} at the GPU arm's positions after {warm} warm-up, {how}"},  # fmt: skip
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    if args.impl == "reference":
        # the reference arm is one CPU run on rank 0; the other ranks exit 0 without work (no process group,
        # so nobody waits on a collective while rank 0 computes)
        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        res = run_reference(args, world, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    world, rank, local = setup_dist()
    try:
        res = run_ours(args, world, rank, local)
        if res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
