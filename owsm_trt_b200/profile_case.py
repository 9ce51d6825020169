"""Small fixed cases for an ncu capture (profiling only): ``python -m owsm_trt_b200.profile_case dense|xkv|beam``.

dense: the 6-layer d=768 model at batch 64, greedy, cache position 100, 750 encoder frames:
four calls of the dense (tcgen05) kernel, the last one the one to capture (``-s 3 -c 1``).
xkv: the 1B model's cross-attention K/V projection of 4 utterances x 750 frames, four launches.
beam: the 1B model's fused beam step, beam 5 over 3 utterances, cache position 100, 750
frames: four calls of the cluster kernel (set OWSM_DEC_NO_COOP=1 under the profiler), the last one to capture.
About 1.5 GB on the device each."""

from __future__ import annotations

import sys

import torch

from .decoder import B200Decoder
from .synthetic import MEDIUM_1B, SMALL, decoder_state_dict, make_workload


def main() -> None:
    what = sys.argv[1] if len(sys.argv) > 1 else "dense"
    dev = torch.device("cuda", 0)
    if what == "dense":
        d, B = SMALL, 64
        sd = decoder_state_dict(d, 0, False)
        k = B200Decoder.from_state_dict(sd, d.H, dev)
        ck, cv, enc_len, prefix, kc, vc = make_workload(d, sd, dev, B, 5)
        tok = prefix[:, -1:].to(dev).contiguous()
        off = torch.full((B,), 100, dtype=torch.long, device=dev)
        logits = torch.zeros(B, 1, d.V, device=dev)
        new_kv = torch.zeros(d.L, 2, B, d.H, 1, d.dk, device=dev, dtype=torch.float16)
        run = k.step_fn(tok, off, kc, vc, ck, cv, logits, new_kv, pred=tok, enc_len=torch.full_like(enc_len, 750).to(dev))
        assert k.plan_kernel(run) == "dense"
        for _ in range(4):
            run()
        torch.cuda.synchronize()
        k.check()
    elif what == "beam":
        d, B, K = MEDIUM_1B, 3, 5
        N = B * K
        sd = decoder_state_dict(d, 0, False)
        k = B200Decoder.from_state_dict(sd, d.H, dev)
        ck, cv, _, prefix, kc, vc = make_workload(d, sd, dev, N, 5, rows_per_utt=K)
        tok = prefix[:, -1:].to(dev).contiguous()
        off = torch.full((N,), 100, dtype=torch.long, device=dev)
        logits = torch.zeros(N, 1, d.V, device=dev)
        new_kv = torch.zeros(d.L, 2, N, d.H, 1, d.dk, device=dev, dtype=torch.float16)
        score = torch.zeros(N, device=dev)
        active = torch.ones(N, dtype=torch.uint8, device=dev)
        parent = torch.zeros(N, dtype=torch.long, device=dev)
        token = torch.zeros(N, dtype=torch.long, device=dev)
        run = k.beam_fn(tok, off, kc, vc, ck, cv, logits, new_kv, score, active, parent, token, beam=K)
        assert k.plan_kernel(run) == "cluster"
        for _ in range(4):
            run()
        torch.cuda.synchronize()
        k.check()
    else:
        d, U = MEDIUM_1B, 4
        sd = decoder_state_dict(d, 0, False)
        k = B200Decoder.from_state_dict(sd, d.H, dev)
        enc = torch.randn(U, 750, d.D, device=dev).half()
        ck = torch.empty(d.L, U, d.H, 750, 64, device=dev, dtype=torch.float16)
        cv = torch.empty_like(ck)
        run = k.cross_kv_fn(enc, ck, cv)
        for _ in range(4):
            run()
        torch.cuda.synchronize()
        k.check_cross_kv()
    print(f"profile case {what}: ok")


if __name__ == "__main__":
    main()
