"""Decoder-step throughput on B200: decoded tokens/s and us/step against the HBM roofline.

Workload: the 18-layer d=1024 OWSM-v4-medium-shaped decoder, fp16, greedy,
16 utterances per GPU, 200 decoder steps each (a 4-token prefix at positions 0-3, then positions 4..203, the
KV cache growing to 204 slots in a 256-slot buffer), encoder memory N(0,1) [16, 750, 1024] projected to
cross K/V once, encoder lengths uniform in [300, 750] (key-padding mask). Weights: seeded synthetic N(0,0.02)
(no checkpoints here). A *step* is one decoder call over the batch (one launch of the persistent kernel);
the greedy argmax feeds back on the device (the pred buffer is the next call's token buffer).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched by torchrun, one process per GPU; every rank decodes its own 16 utterances (weak
scaling, no collective on the data path); the timed region is bracketed by barriers and the max over ranks
is reported. ``--impl reference`` times the reference algorithm's CPU path (the fp32 torch restatement in
oracle/, owsm-trt's TorchBackend semantics) on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
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

METRIC = "decoded tokens/s (greedy decoder step, 1B OWSM decoder, batch 16 per GPU)"
UNIT = "tokens/s"
BATCH, PREFIX, STEPS_PER_UTT, T_ENC, CACHE = 16, 4, 200, 750, 256
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    return ap.parse_args()


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
    p = Path(__file__).resolve().parent / "profiles" / "decoder_cl_kernel_b16_full.md"
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


def make_workload(d, sd, dev, batch: int, seed: int, rows_per_utt: int = 1):
    """Cross K/V of `batch / rows_per_utt` utterances (encoder memory N(0,1) through the decoder's K/V
    projections), encoder lengths U[300, 750], prefix tokens, caches."""
    from owsm_trt_b200.synthetic import cross_kv

    g = torch.Generator().manual_seed(seed)
    U = batch // rows_per_utt
    enc = torch.randn(U, T_ENC, d.D, generator=g).to(dev)
    sd_dev = {k: v.to(dev) for k, v in sd.items() if ".src_attn.linear_k." in k or ".src_attn.linear_v." in k}
    with torch.no_grad():
        kv = cross_kv(sd_dev, d, enc).half()  # [L, 2, U, H, T, dk]
    ck, cv = kv[:, 0].contiguous(), kv[:, 1].contiguous()
    del kv, enc, sd_dev
    enc_len = torch.randint(300, T_ENC + 1, (U,), generator=g).to(torch.int32)
    prefix = torch.randint(0, d.V, (batch, PREFIX), generator=g)
    kc = torch.zeros(d.L, batch, d.H, CACHE, d.dk, device=dev, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    return ck, cv, enc_len, prefix, kc, vc


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
    ck, cv, enc_len, prefix, kc, vc = make_workload(d, sd, dev, B, 1000 + rank)
    enc_len_d = enc_len.to(dev)
    # prefill (4 tokens per row) in the kernel itself, untimed
    lg_p = torch.zeros(B, PREFIX, d.V, device=dev)
    kv_p = torch.zeros(d.L, 2, B, d.H, PREFIX, d.dk, device=dev, dtype=torch.float16)
    pr_p = torch.zeros(B, PREFIX, dtype=torch.long, device=dev)
    zero = torch.zeros(B, dtype=torch.long, device=dev)
    kern.step_fn(prefix.to(dev), zero, kc, vc, ck, cv, lg_p, kv_p, pred=pr_p, enc_len=enc_len_d)()
    # decode steps: offsets PREFIX + j; tokens = the previous call's argmax (same buffer)
    tok = pr_p[:, -1:].clone()
    offs = (PREFIX + torch.arange(STEPS_PER_UTT, device=dev))[:, None].expand(STEPS_PER_UTT, B).contiguous()
    logits = torch.zeros(B, 1, d.V, device=dev)
    new_kv = torch.zeros(d.L, 2, B, d.H, 1, d.dk, device=dev, dtype=torch.float16)
    runs = [kern.step_fn(tok, offs[j], kc, vc, ck, cv, logits, new_kv, pred=tok, enc_len=enc_len_d)
            for j in range(STEPS_PER_UTT)]  # fmt: skip
    K, W = args.steps, max(3, args.warmup)
    for i in range(W):
        runs[i % STEPS_PER_UTT]()
    torch.cuda.synchronize(dev)
    kern.check()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev) as clk:
        torch.cuda.synchronize(dev)
        start.record()
        for i in range(K):
            runs[i % STEPS_PER_UTT]()
        end.record()
        torch.cuda.synchronize(dev)
    kern.check()
    barrier(world)
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ms, world, dev)
    per_step_ms = ms_max / K
    tokens_total = B * K * world
    value = tokens_total / (ms_max / 1e3)

    # end to end through the public API: tokens and offsets from pinned host memory each step, the argmax back
    # to the host each step (greedy feedback through the host, as a caller without on-device decoding does)
    h_tok = torch.zeros(B, 1, dtype=torch.long).pin_memory()
    h_off = torch.zeros(B, dtype=torch.long).pin_memory()
    h_pred = torch.zeros(B, 1, dtype=torch.long).pin_memory()
    d_tok = torch.zeros(B, 1, dtype=torch.long, device=dev)
    d_off = torch.zeros(B, dtype=torch.long, device=dev)
    d_pred = torch.zeros(B, 1, dtype=torch.long, device=dev)
    run_e2e = kern.step_fn(d_tok, d_off, kc, vc, ck, cv, logits, new_kv, pred=d_pred, enc_len=enc_len_d)
    h_tok.copy_(tok.cpu())
    K2 = min(K, 400)
    stream = torch.cuda.current_stream(dev)

    def e2e_steps(n):
        for i in range(n):
            h_off.fill_(PREFIX + i % STEPS_PER_UTT)
            d_tok.copy_(h_tok, non_blocking=True)
            d_off.copy_(h_off, non_blocking=True)
            run_e2e()
            h_pred.copy_(d_pred, non_blocking=True)
            stream.synchronize()
            h_tok.copy_(h_pred)

    e2e_steps(W)
    barrier(world)
    t0 = time.perf_counter()
    e2e_steps(K2)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world, dev)
    e2e_value = B * K2 * world / e2e_s

    hbm, hbm_src = peaks()
    lens = enc_len.tolist()
    avg_bytes = statistics.mean(step_bytes(d, B, PREFIX + j, lens) for j in range(STEPS_PER_UTT))
    # the timed steps cycle through positions: weight the step bytes by how often each position ran
    counts = [K // STEPS_PER_UTT + (1 if j < K % STEPS_PER_UTT else 0) for j in range(STEPS_PER_UTT)]
    avg_bytes = sum(c * step_bytes(d, B, PREFIX + j, lens) for j, c in enumerate(counts)) / K
    achieved = avg_bytes / (per_step_ms / 1e3) / 1e9  # per GPU (each GPU's step moves avg_bytes)
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(per_step_ms, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) encoder memory)",
        "config": {"workload": "BASELINE configs[1]: 1B decoder greedy, 16 utterances/GPU, 200 steps, enc_len U[300,750]",
                   "global_batch": B * world, "seq_len": PREFIX + STEPS_PER_UTT, "parallelism": f"dp{world} (utterance shards, no collective)",
                   "cache_slots": CACHE, "enc_frames": T_ENC,
                   "l2": "inputs larger than L2 (631 MB of weights per step > 126 MB)"},  # fmt: skip
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": 2 * B * 8,
                "d2h_bytes_per_step": B * 8, "steps": K2},  # fmt: skip
        "gpu_launches": K,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": profiled_traffic(B), "peak_source": hbm_src,
                     "algorithmic_bytes_per_step": int(avg_bytes)},  # fmt: skip
        "clocks": clk.summary(),
        "us_per_step": round(per_step_ms * 1e3, 2),
    }
    if rank == 0 and world == 1 and not args.no_secondary:
        result["secondary"] = secondary(kern, sd, d, dev, hbm)
    if rank == 0 and world == 1:
        result["cpu_baseline"] = cpu_baseline(sd, d, B, args.cpu_seconds)
    kern.close()
    return result if rank == 0 else None


def secondary(kern, sd, d, dev, hbm) -> dict:
    """The other BASELINE shapes on one GPU (us/step, roofline fraction): greedy b1 (the headline roofline
    target) and beam 5 x batch 3 (fused select + reorder)."""
    out = {}
    for B in (1,):
        ck, cv, enc_len, prefix, kc, vc = make_workload(d, sd, dev, B, 77)
        el = torch.full_like(enc_len, T_ENC).to(dev)  # b1: the reference pads to 30 s (no mask)
        tok = prefix[:, -1:].to(dev).contiguous()
        offs = (PREFIX + torch.arange(STEPS_PER_UTT, device=dev))[:, None].expand(STEPS_PER_UTT, B).contiguous()
        logits = torch.zeros(B, 1, d.V, device=dev)
        new_kv = torch.zeros(d.L, 2, B, d.H, 1, d.dk, device=dev, dtype=torch.float16)
        runs = [kern.step_fn(tok, offs[j], kc, vc, ck, cv, logits, new_kv, pred=tok, enc_len=el) for j in range(STEPS_PER_UTT)]
        for i in range(10):
            runs[i]()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for i in range(STEPS_PER_UTT):
            runs[i]()
        e.record()
        torch.cuda.synchronize()
        kern.check()
        us = s.elapsed_time(e) * 1e3 / STEPS_PER_UTT
        avg = statistics.mean(step_bytes(d, B, PREFIX + j, [T_ENC]) for j in range(STEPS_PER_UTT))
        gbs = avg / (us * 1e-6) / 1e9
        out[f"greedy_b{B}"] = {"us_per_step": round(us, 2), "tokens_per_s": round(B / (us * 1e-6), 1),
                               "achieved_gbs": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 4),
                               "algorithmic_bytes_per_step": int(avg)}  # fmt: skip
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
    runs = [kern.beam_fn(tok, offs[j], kc, vc, ck, cv, logits, new_kv, score, active, parent, token, beam=Kb,
                         enc_len=el) for j in range(150)]  # fmt: skip
    for i in range(5):
        runs[i]()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for i in range(150):
        runs[i]()
    e.record()
    torch.cuda.synchronize()
    kern.check()
    us = s.elapsed_time(e) * 1e3 / 150
    avg = statistics.mean(step_bytes(d, N, PREFIX + j, [T_ENC] * Bu) for j in range(150))
    gbs = avg / (us * 1e-6) / 1e9
    out["beam5_batch3"] = {"us_per_step": round(us, 2), "tokens_per_s": round(N / (us * 1e-6), 1),
                           "achieved_gbs": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 4),
                           "algorithmic_bytes_per_step": int(avg)}  # fmt: skip
    return out


def cpu_baseline(sd, d, B: int, seconds: float) -> dict:
    """The reference algorithm's fp32 CPU path (oracle/ restatement of Decoder.step) on a bounded sample:
    decoder calls of the same batch at growing positions until `seconds` have passed."""
    from oracle import decoder as ref
    from owsm_trt_b200.synthetic import sinusoidal_positions

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(5)
    C = 64
    kc = torch.zeros(d.L, B, d.H, C, d.dk)
    vc = torch.zeros_like(kc)
    ck = torch.randn(d.L, B, d.H, T_ENC, d.dk, generator=g).half().float()
    cv = torch.randn(d.L, B, d.H, T_ENC, d.dk, generator=g).half().float()
    enc_len = torch.randint(300, T_ENC + 1, (B,), generator=g)
    pe = sinusoidal_positions(C + 8, d.D)
    tok = torch.randint(0, d.V, (B, 1), generator=g)
    n, t0 = 0, time.perf_counter()
    with torch.no_grad():
        while True:
            off = torch.full((B,), PREFIX + n, dtype=torch.long)
            lg, kv = ref.decoder_step(sd, d.H, tok, off, kc, vc, ck, cv, enc_len=enc_len, pe=pe)
            ref.write_kv(kv, kc, vc, off)
            tok = ref.argmax_first(lg[:, -1])[:, None]
            n += 1
            el = time.perf_counter() - t0
            if el > seconds or PREFIX + n >= C:
                break
    return {"value": round(B * n / el, 2), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} decoder calls of batch {B} (positions {PREFIX}..{PREFIX + n - 1}), 1B decoder, fp32, "
                      f"oracle restatement of owsm-trt Decoder.step (TorchBackend semantics), {el:.1f} s"}  # fmt: skip


def run_reference(args, world, rank) -> dict | None:
    """The reference's CPU path (oracle port) on the host cores, same metric / config; rank 0 only."""
    if rank != 0:
        return None
    from owsm_trt_b200.synthetic import MEDIUM_1B, decoder_state_dict

    d = MEDIUM_1B
    B = args.batch
    sd = decoder_state_dict(d, 0, False)
    steps = max(1, min(args.steps, 12))
    warm = 3  # the timing rules' minimum of warm-up steps (more would only add CPU seconds)
    from oracle import decoder as ref
    from owsm_trt_b200.synthetic import sinusoidal_positions

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(5)
    C = 64
    kc = torch.zeros(d.L, B, d.H, C, d.dk)
    vc = torch.zeros_like(kc)
    ck = torch.randn(d.L, B, d.H, T_ENC, d.dk, generator=g).half().float()
    cv = torch.randn(d.L, B, d.H, T_ENC, d.dk, generator=g).half().float()
    enc_len = torch.randint(300, T_ENC + 1, (B,), generator=g)
    pe = sinusoidal_positions(C + 8, d.D)
    tok = torch.randint(0, d.V, (B, 1), generator=g)

    def one(i):
        nonlocal tok
        off = torch.full((B,), PREFIX + i, dtype=torch.long)
        lg, kv = ref.decoder_step(sd, d.H, tok, off, kc, vc, ck, cv, enc_len=enc_len, pe=pe)
        ref.write_kv(kv, kc, vc, off)
        tok = ref.argmax_first(lg[:, -1])[:, None]

    with torch.no_grad():
        for i in range(warm):
            one(i)
        t0 = time.perf_counter()
        for i in range(steps):
            one(warm + i)
        el = time.perf_counter() - t0
    value = B * steps / el
    return {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": warm,
        "ms_per_step": round(el / steps * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": "BASELINE configs[1] (sampled): 1B decoder greedy, batch 16, enc_len U[300,750]",
                   "global_batch": B, "seq_len": PREFIX + steps + warm, "parallelism": "cpu"},  # fmt: skip
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{steps} timed decoder calls (of the 200-step workload) after {warm} warm-up, "
                                   "oracle restatement of owsm-trt Decoder.step, fp32"},  # fmt: skip
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
