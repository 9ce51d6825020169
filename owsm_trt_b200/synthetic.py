"""Seeded synthetic decoder weights and inputs in the reference's parameter naming.

The state dict uses the names of ``owsm_trt.modeling.Decoder`` (``src/owsm_trt/modeling.py:471-488``):
``embed.0.weight``, ``decoders.{i}.self_attn.linear_{q,k,v,out}.{weight,bias}``,
``decoders.{i}.src_attn.linear_{q,k,v,out}.*``, ``decoders.{i}.feed_forward.w_{1,2}.*``,
``decoders.{i}.norm{1,2,3}.*``, ``after_norm.*``, ``output_layer.*``. Such a dict loads into the
reference module with ``load_state_dict`` and into :class:`owsm_trt_b200.decoder.B200Decoder`.

Two variants:

* ``plain`` (benchmarks): every Linear/Embedding weight N(0, 0.02), LayerNorm gamma = 1, beta = 0,
  biases 0. Weights are rounded to fp16 and back, so fp32 and fp16 computations see the same values.
* ``perturbed`` (tests): LayerNorm gamma/beta and every bias get + 0.2 * N(0, 1), and the output
  weight is scaled by 8, as the reference's kernel tests do (``tests/test_megakernel.py:29-40``):
  the LayerNorm folding is exercised and argmax margins are clear.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class DecoderDims:
    """Shapes of a Transformer decoder (``OWSMConfig`` fields ``dec_layers``, ``d_model``, ``dec_heads``,
    ``dec_ffn``, ``vocab_size``; ``src/owsm_trt/config.py:15-30``)."""

    L: int
    D: int
    H: int
    F: int
    V: int
    max_pos: int = 5000

    @property
    def dk(self) -> int:
        return self.D // self.H


# OWSM v4 medium (1B) decoder and the small-model path of the benchmark configurations.
MEDIUM_1B = DecoderDims(L=18, D=1024, H=16, F=4096, V=50000)
SMALL = DecoderDims(L=6, D=768, H=12, F=3072, V=50000)
# The reference's kernel-test model (tests/test_megakernel.py:20-22) and its non-power-of-2 width (:26).
TEST_CFG = DecoderDims(L=3, D=256, H=4, F=512, V=1000)
TEST_CFG384 = DecoderDims(L=2, D=384, H=6, F=768, V=1000)


def sinusoidal_positions(n: int, d: int) -> torch.Tensor:
    """[n, d] sinusoidal table, the function of ``src/owsm_trt/modeling.py:28-35``."""
    pos = torch.arange(n, dtype=torch.float32)[:, None]
    div = torch.exp(torch.arange(0, d, 2, dtype=torch.float32) * (-math.log(10000.0) / d))
    pe = torch.zeros(n, d)
    pe[:, 0::2] = torch.sin(pos * div)
    pe[:, 1::2] = torch.cos(pos * div)
    return pe


def decoder_state_dict(dims: DecoderDims, seed: int = 0, perturbed: bool = False) -> dict[str, torch.Tensor]:
    """fp32 CPU tensors named as the reference ``Decoder``'s parameters (see the module docstring)."""
    g = torch.Generator().manual_seed(seed)
    D, F, V = dims.D, dims.F, dims.V

    def w(*shape):
        return (torch.randn(*shape, generator=g) * 0.02).half().float()

    def vec(n, base):
        t = torch.full((n,), float(base))
        if perturbed:
            t = t + 0.2 * torch.randn(n, generator=g)
        return t.half().float()

    sd: dict[str, torch.Tensor] = {"embed.0.weight": w(V, D)}
    for i in range(dims.L):
        p = f"decoders.{i}."
        for att in ("self_attn", "src_attn"):
            for lin in ("linear_q", "linear_k", "linear_v", "linear_out"):
                sd[f"{p}{att}.{lin}.weight"] = w(D, D)
                sd[f"{p}{att}.{lin}.bias"] = vec(D, 0.0)
        sd[p + "feed_forward.w_1.weight"] = w(F, D)
        sd[p + "feed_forward.w_1.bias"] = vec(F, 0.0)
        sd[p + "feed_forward.w_2.weight"] = w(D, F)
        sd[p + "feed_forward.w_2.bias"] = vec(D, 0.0)
        for n in ("norm1", "norm2", "norm3"):
            sd[f"{p}{n}.weight"] = vec(D, 1.0)
            sd[f"{p}{n}.bias"] = vec(D, 0.0)
    sd["after_norm.weight"] = vec(D, 1.0)
    sd["after_norm.bias"] = vec(D, 0.0)
    wout = w(V, D)
    if perturbed:
        wout = (wout * 8.0).half().float()
    sd["output_layer.weight"] = wout
    sd["output_layer.bias"] = vec(V, 0.0)
    return sd


def dims_of(sd: dict[str, torch.Tensor], heads: int) -> DecoderDims:
    """The shapes of a decoder state dict (reference naming); ``heads`` is not stored in the weights."""
    V, D = sd["embed.0.weight"].shape
    L = 1 + max(int(k.split(".")[1]) for k in sd if k.startswith("decoders."))
    F = sd["decoders.0.feed_forward.w_1.weight"].shape[0]
    return DecoderDims(L=L, D=D, H=heads, F=F, V=V)


def cross_kv(sd: dict[str, torch.Tensor], dims: DecoderDims, enc: torch.Tensor) -> torch.Tensor:
    """Every layer's cross-attention keys/values of encoder output ``enc`` [B, T, D]:
    [L, 2, B, H, T, dk], the projection of ``Decoder.cross_kv`` (``src/owsm_trt/modeling.py:490-499``)."""
    B, T, _ = enc.shape
    out = []
    for i in range(dims.L):
        p = f"decoders.{i}.src_attn."
        kv = []
        for lin in ("linear_k", "linear_v"):
            y = enc @ sd[p + lin + ".weight"].t().to(enc.dtype) + sd[p + lin + ".bias"].to(enc.dtype)
            kv.append(y.reshape(B, T, dims.H, dims.dk).transpose(1, 2))
        out.append(torch.stack(kv))
    return torch.stack(out)


# The benchmark workload's fixed shapes: a 4-token prefix, 750 encoder frames, 256 cache slots.
PREFIX, T_ENC, CACHE = 4, 750, 256


def make_workload(d: DecoderDims, sd: dict[str, torch.Tensor], dev: torch.device, batch: int, seed: int,
                  rows_per_utt: int = 1, enc_lo: int = 300):
    """Inputs of one benchmark batch: cross K/V of ``batch / rows_per_utt`` utterances (encoder memory N(0,1)
    [U, 750, D] through the decoder's K/V projections, :func:`cross_kv`), encoder lengths U[enc_lo, 750],
    a 4-token prefix per row, and zeroed fp16 caches of 256 slots.
    Returns (cross_k, cross_v, enc_len int32 (CPU), prefix int64 (CPU), self_k, self_v)."""
    g = torch.Generator().manual_seed(seed)
    U = batch // rows_per_utt
    enc = torch.randn(U, T_ENC, d.D, generator=g).to(dev)
    sd_dev = {k: v.to(dev) for k, v in sd.items() if ".src_attn.linear_k." in k or ".src_attn.linear_v." in k}
    with torch.no_grad():
        kv = cross_kv(sd_dev, d, enc).half()  # [L, 2, U, H, T, dk]
    ck, cv = kv[:, 0].contiguous(), kv[:, 1].contiguous()
    del kv, enc, sd_dev
    enc_len = torch.randint(enc_lo, T_ENC + 1, (U,), generator=g).to(torch.int32)
    prefix = torch.randint(0, d.V, (batch, PREFIX), generator=g)
    kc = torch.zeros(d.L, batch, d.H, CACHE, d.dk, device=dev, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    return ck, cv, enc_len, prefix, kc, vc
