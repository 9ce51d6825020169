"""Generate the golden vectors that pin the CPU oracle (``oracle/decoder.py``) to owsm-trt itself.

Run in a container where the owsm-trt sources are importable (``OWSM_TRT_SRC`` = its ``src`` directory);
the GPU box never runs this script, it only reads the ``.npz`` files written next to it.

    OWSM_TRT_SRC=/path/to/owsm-trt/src python tests/golden/make_golden.py

Weights are not stored: both this script and the tests rebuild them from a seed with
``owsm_trt_b200.synthetic.decoder_state_dict`` (deterministic on the CPU). The fixtures hold the
reference's inputs and outputs:

* ``step_*.npz`` -- ``Decoder.step`` (src/owsm_trt/modeling.py:501-560) on the reference kernel-test shape
  (d=256, 4 heads, FFN 512, 3 layers, V=1000; tests/test_megakernel.py:20-22), perturbed weights, for
  several (rows, window, offsets); ``masked`` runs each row alone on cross K/V sliced to its length
  (the exact meaning of a key-padding mask, since ``step`` takes T from the tensor shape).
* ``beam.npz`` -- ``BeamSession._select`` (src/owsm_trt/runtime.py:1399-1446) on given logits / scores /
  active slots / caches: new scores, tokens, and the reordered caches.
* ``greedy.npz`` -- ``GreedySession.decode`` (runtime.py:804-828) with ``TorchBackend`` (fp32, CPU).
* ``verify.npz`` -- ``_Verify.predict`` / ``_Verify.accept`` (runtime.py:1251-1278): the argmax of every window
  position under the timestamp rules and the drafted tokens accepted, on given logits and input rows.
* ``medium_step.npz`` -- one ``Decoder.step`` of the 18-layer d=1024 model (plain weights), b1: the
  top-32 logits, their ids and checksums.
"""

from __future__ import annotations

import dataclasses
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, os.environ.get("OWSM_TRT_SRC", "/root/reference/src"))

from owsm_trt.config import OWSMConfig  # noqa: E402
from owsm_trt.modeling import Decoder, OWSMModel  # noqa: E402
from owsm_trt.runtime import BeamSession, GreedySession, TorchBackend  # noqa: E402

from owsm_trt_b200.synthetic import MEDIUM_1B, TEST_CFG, DecoderDims, decoder_state_dict  # noqa: E402

sys.path.insert(0, str(HERE))
import cases  # noqa: E402

# owsm-trt's TINY test config (tests/test_model.py:11-15) widened to the kernel-test shape.
TINY = OWSMConfig(
    vocab_size=50, d_model=32, n_heads=4, enc_layers=2, enc_ffn=64, cgmlp_units=64, cgmlp_kernel=5,
    merge_kernel=3, subsample="conv2d8", dec_layers=2, dec_ffn=64, dec_heads=4, n_mels=16, n_fft=64,
    win_length=48, hop_length=32, sample_rate=1600, speech_seconds=2.0, time_resolution=0.02,
)  # fmt: skip


def cfg_for(d: DecoderDims) -> OWSMConfig:
    return dataclasses.replace(
        TINY, vocab_size=d.V, d_model=d.D, n_heads=d.H, dec_heads=d.H, dec_ffn=d.F, dec_layers=d.L
    )


def ref_decoder(d: DecoderDims, seed: int, perturbed: bool) -> Decoder:
    dec = Decoder(cfg_for(d)).eval().requires_grad_(False)
    dec.load_state_dict(decoder_state_dict(d, seed, perturbed), strict=True)
    return dec


def step_case(dec: Decoder, d: DecoderDims, name: str) -> None:
    R, S, C, T, seed, enc_len = cases.STEP_CASES[name]
    tokens, offset, k, v, ck, cv = cases.step_inputs(d, R, S, C, T, seed)
    with torch.no_grad():
        if enc_len is None:
            logits, new_kv = dec.step(tokens, offset, list(k.float()), list(v.float()), list(ck.float()),
                                      list(cv.float()))  # fmt: skip
        else:
            outs = []
            for r in range(R):
                rb = slice(r, r + 1)
                n = enc_len[r]
                outs.append(dec.step(tokens[rb], offset[rb], list(k[:, rb].float()), list(v[:, rb].float()),
                                     list(ck[:, rb, :, :n].float()), list(cv[:, rb, :, :n].float())))  # fmt: skip
            logits = torch.cat([o[0] for o in outs], 0)
            new_kv = torch.cat([o[1] for o in outs], 2)
    np.savez_compressed(HERE / f"step_{name}.npz", logits=logits.numpy(), new_kv=new_kv.numpy())
    print(name, logits.shape, float(logits.abs().max()))


def beam_case(d: DecoderDims) -> None:
    """BeamSession._select on a session built around a model with the kernel-test decoder."""
    cfg = cfg_for(d)
    torch.manual_seed(0)
    model = OWSMModel(cfg).eval().requires_grad_(False)
    model.decoder.load_state_dict(decoder_state_dict(d, 0, True), strict=True)
    B, K, C, p = cases.BEAM["B"], cases.BEAM["K"], cases.BEAM["C"], cases.BEAM["pos"]
    sess = BeamSession(TorchBackend(model), cfg, B, K, C, eos=1, dtype=torch.float32, device=torch.device("cpu"),
                       use_cuda_graph=False, buckets=[C])  # fmt: skip
    logits, score, active, k0, v0 = cases.beam_inputs(d)
    sess.logits[:, -1] = logits
    sess.score.copy_(score)
    sess.active.copy_(active)
    sess.caches[C][0].copy_(k0)
    sess.caches[C][1].copy_(v0)
    sess.pos.fill_(p)
    sess.step.fill_(1)
    sess.last_step.fill_(50)
    sess.best_score.fill_(float("-inf"))
    sess.ended_by_len.fill_(float("-inf"))
    sess.done.zero_()
    sess._select(C)
    k, v = sess.caches[C]
    # the row each new slot's cache came from (the reorder ``index_select(1, parent)``)
    parent = []
    for r in range(B * K):
        match = [q for q in range(B * K) if torch.equal(k[:, r], k0[:, q]) and torch.equal(v[:, r], v0[:, q])]
        assert len(match) == 1
        parent.append(match[0])
    np.savez_compressed(HERE / "beam.npz", score=sess.score.numpy(), token=sess.tok[:, 0].numpy(),
                        parent=np.array(parent, dtype=np.int64), active=sess.active.numpy())  # fmt: skip
    print("beam", sess.score[:5], sess.tok[:5, 0], parent)


def greedy_case(d: DecoderDims) -> None:
    """GreedySession.decode with TorchBackend (fp32, CPU) from given cross K/V."""
    G = cases.GREEDY
    cfg = cfg_for(d)
    assert cfg.enc_frames == G["T"]
    torch.manual_seed(0)
    model = OWSMModel(cfg).eval().requires_grad_(False)
    model.decoder.load_state_dict(decoder_state_dict(d, 0, True), strict=True)
    B = G["B"]
    sess = GreedySession(TorchBackend(model), cfg, B, G["C"], eos=G["eos"], dtype=torch.float32,
                         device=torch.device("cpu"), use_cuda_graph=False, buckets=[16, 32, 64])  # fmt: skip
    ck, cv = cases.greedy_inputs(d)
    sess.cross_k.copy_(ck.float())
    sess.cross_v.copy_(cv.float())
    out = sess.decode(torch.tensor(G["primer"]), G["steps"])
    seqs = np.full((B, G["steps"]), -1, dtype=np.int64)
    for b, o in enumerate(out):
        seqs[b, : len(o)] = o
    np.savez_compressed(HERE / "greedy.npz", out=seqs)
    print("greedy", out)


def medium_case() -> None:
    d = MEDIUM_1B
    dec = ref_decoder(d, 0, False)
    tokens, offset, k, v, enc = cases.medium_inputs(d)
    with torch.no_grad():
        kv = dec.cross_kv(enc).half()  # [L, 2, R, H, T, dk]
        logits, new_kv = dec.step(tokens, offset, list(k.float()), list(v.float()), list(kv[:, 0].float()),
                                  list(kv[:, 1].float()))  # fmt: skip
    lg = logits[0, 0]
    top = lg.topk(32)
    np.savez_compressed(
        HERE / "medium_step.npz", top_val=top.values.numpy(), top_idx=top.indices.numpy(),
        sum=float(lg.double().sum()), sumsq=float((lg.double() ** 2).sum()), kv_sum=float(new_kv.double().sum()),
        kv_abs=float(new_kv.double().abs().sum()), cross_sum=float(kv.double().sum()),
    )  # fmt: skip
    print("medium", top.values[:4], top.indices[:4])


def verify_case() -> None:
    """_Verify.predict / _Verify.accept (runtime.py:1251-1278) on given logits and input rows, CPU buffers."""
    from owsm_trt.runtime import TimestampRules, _Verify

    rl = cases.VERIFY_RULES
    out = {}
    for name, (R, W, seed) in cases.VERIFY_CASES.items():
        logits, inp, notime = cases.verify_inputs(R, W, seed)
        cfg = dataclasses.replace(TINY, vocab_size=rl["vocab"])
        rules = TimestampRules(rl["notime"], rl["first_time"], rl["last_time"], rl["eos"], rl["vocab"],
                               torch.device("cpu"))  # fmt: skip
        bufs = _Verify(cfg, R, W, {"device": torch.device("cpu"), "dtype": torch.float32}, rules, notime, rl["eos"])
        bufs.inp.copy_(inp)
        bufs.tok.copy_(inp[:, :W])
        bufs.logits.copy_(logits)
        bufs.pred.copy_(bufs.predict())
        out[f"{name}_pred"] = bufs.pred.numpy().copy()
        out[f"{name}_res"] = bufs.accept().numpy().copy()
        plain = _Verify(cfg, R, W, {"device": torch.device("cpu"), "dtype": torch.float32}, None, notime, rl["eos"])
        plain.logits.copy_(logits)
        out[f"{name}_plain"] = plain.predict().numpy().copy()
        print("verify", name, out[f"{name}_res"].tolist())
    np.savez_compressed(HERE / "verify.npz", **out)


def main() -> None:
    torch.set_num_threads(os.cpu_count() or 1)
    d = TEST_CFG
    dec = ref_decoder(d, 0, True)
    for name in cases.STEP_CASES:
        step_case(dec, d, name)
    beam_case(d)
    greedy_case(d)
    medium_case()
    verify_case()


if __name__ == "__main__":
    main()
