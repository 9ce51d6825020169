"""B200Decoder's argument checks on the CPU: a malformed buffer is refused with TypeError / ValueError before any
library call, and a well-formed call gets through to the plan. The decoder object is built without its device state
(the checks read only the model's dims and device); its plan step is replaced by a stub that records the call."""

from __future__ import annotations

import pytest
import torch

from owsm_trt_b200.decoder import B200Decoder

L, H, V, D, DK = 2, 4, 100, 256, 64


class _Reached(Exception):
    pass


def _kernel() -> B200Decoder:
    k = B200Decoder.__new__(B200Decoder)
    k.L, k.H, k.V, k.D, k.device = L, H, V, D, torch.device("cpu")

    def plan(*args):
        raise _Reached(args)

    k._plan = plan
    return k


def _greedy(R=2, S=1, C=16, T=8, G=1):
    f16 = dict(dtype=torch.float16)
    return dict(tokens=torch.zeros(R, S, dtype=torch.long), offset=torch.zeros(R, dtype=torch.long),
                self_k=torch.zeros(L, R, H, C, DK, **f16), self_v=torch.zeros(L, R, H, C, DK, **f16),
                cross_k=torch.zeros(L, R // G, H, T, DK, **f16), cross_v=torch.zeros(L, R // G, H, T, DK, **f16),
                logits=torch.zeros(R, S, V), new_kv=torch.zeros(L, 2, R, H, S, DK, **f16))  # fmt: skip


def _beam(B=2, K=2):
    R = B * K
    buf = _greedy(R=R, G=K)
    buf.update(score=torch.zeros(R), active=torch.ones(R, dtype=torch.uint8), parent=torch.zeros(R, dtype=torch.long),
               token=torch.zeros(R, dtype=torch.long))  # fmt: skip
    return buf


def _step(k, buf, **kw):
    names = ("tokens", "offset", "self_k", "self_v", "cross_k", "cross_v", "logits", "new_kv")
    return k.step_fn(*(buf[n] for n in names), **kw)


def _beam_step(k, buf, **kw):
    names = ("tokens", "offset", "self_k", "self_v", "cross_k", "cross_v", "logits", "new_kv", "score", "active",
             "parent", "token")  # fmt: skip
    return k.beam_fn(*(buf[n] for n in names), beam=2, **kw)


def test_well_formed_calls_reach_the_plan():
    k = _kernel()
    with pytest.raises(_Reached):
        _step(k, _greedy(), pred=torch.zeros(2, 1, dtype=torch.long), enc_len=torch.full((2,), 8, dtype=torch.int32))
    with pytest.raises(_Reached):
        _step(k, _greedy(R=4, G=2), rows_per_utt=2, enc_len=torch.full((2,), 8, dtype=torch.int32))
    with pytest.raises(_Reached):
        _beam_step(k, _beam(), enc_len=torch.full((2,), 8, dtype=torch.int32),
                   shared=torch.zeros(2, 2, 2, dtype=torch.int32))  # fmt: skip


STEP_CASES = {
    "tokens int32": (TypeError, lambda b: b.update(tokens=b["tokens"].int()), {}),
    "offset int32": (TypeError, lambda b: b.update(offset=b["offset"].int()), {}),
    "cache fp32": (TypeError, lambda b: b.update(self_k=b["self_k"].float()), {}),
    "cache not contiguous": (TypeError, lambda b: b.update(self_v=b["self_v"].transpose(3, 4)), {}),
    "logits fp16": (TypeError, lambda b: b.update(logits=b["logits"].half()), {}),
    "cache rows": (ValueError, lambda b: b.update(self_k=b["self_k"][:, :1].contiguous()), {}),
    "cross rows": (ValueError, lambda b: None, {"rows_per_utt": 2}),
    "logits vocab": (ValueError, lambda b: b.update(logits=b["logits"][..., :50].contiguous()), {}),
    "pred int32": (ValueError, lambda b: None, {"pred": torch.zeros(2, 1, dtype=torch.int32)}),
    "notime float": (TypeError, lambda b: None, {"pred": torch.zeros(2, 1, dtype=torch.long),
                                                 "notime": (torch.zeros(2), 5, 9)}),
    "enc_len int64": (ValueError, lambda b: None, {"enc_len": torch.full((2,), 8, dtype=torch.long)}),
    "enc_len count": (ValueError, lambda b: None, {"enc_len": torch.full((3,), 8, dtype=torch.int32)}),
}


@pytest.mark.parametrize("case", sorted(STEP_CASES))
def test_step_refuses_malformed_buffers(case):
    err, edit, kw = STEP_CASES[case]
    buf = _greedy()
    edit(buf)
    with pytest.raises(err):
        _step(_kernel(), buf, **kw)


BEAM_CASES = {
    "two tokens per row": (ValueError, lambda b: b.update(tokens=torch.zeros(4, 2, dtype=torch.long),
                                                          logits=torch.zeros(4, 2, V),
                                                          new_kv=torch.zeros(L, 2, 4, H, 2, DK, dtype=torch.float16)),
                           {}),
    "score fp64": (TypeError, lambda b: b.update(score=b["score"].double()), {}),
    "active bool": (TypeError, lambda b: b.update(active=b["active"].bool()), {}),
    "parent int32": (TypeError, lambda b: b.update(parent=b["parent"].int()), {}),
    "shared int64": (TypeError, lambda b: None, {"shared": torch.zeros(2, 2, 2, dtype=torch.long)}),
    "shared shape": (TypeError, lambda b: None, {"shared": torch.zeros(4, 2, 2, dtype=torch.int32)}),
    "enc_len per row": (ValueError, lambda b: None, {"enc_len": torch.full((4,), 8, dtype=torch.int32)}),
    "enc_len int64": (ValueError, lambda b: None, {"enc_len": torch.full((2,), 8, dtype=torch.long)}),
}  # fmt: skip


@pytest.mark.parametrize("case", sorted(BEAM_CASES))
def test_beam_step_refuses_malformed_buffers(case):
    err, edit, kw = BEAM_CASES[case]
    buf = _beam()
    edit(buf)
    with pytest.raises(err):
        _beam_step(_kernel(), buf, **kw)


def _verify(k, R=2, W=3, edit=None, **kw):
    buf = _greedy(R=R, S=W)
    buf.update(inp=torch.zeros(R, W + 4, dtype=torch.long), pred=torch.zeros(R, W, dtype=torch.long))
    if edit is not None:
        edit(buf)
    return k.verify_fn(buf["inp"], buf["self_k"], buf["self_v"], buf["cross_k"], buf["cross_v"], buf["logits"],
                       buf["new_kv"], buf["pred"], **kw)  # fmt: skip


def test_well_formed_verify_calls_reach_the_plan():
    k = _kernel()
    with pytest.raises(_Reached):
        _verify(k, res=torch.zeros(2, 2, dtype=torch.long), eos=1)
    with pytest.raises(_Reached):  # the rules' <eos> serves the accepted-prefix output
        _verify(k, res=torch.zeros(2, 2, dtype=torch.long), rules=(50, 90, 1), notime=torch.zeros(2, dtype=torch.bool))


VERIFY_CASES = {
    "inp int32": (TypeError, lambda b: b.update(inp=b["inp"].int()), {}),
    "inp without tokens": (ValueError, lambda b: b.update(inp=b["inp"][:, :4].contiguous()), {}),
    "pred window": (ValueError, lambda b: b.update(pred=b["pred"][:, :2].contiguous()), {}),
    "res int32": (ValueError, None, {"res": torch.zeros(2, 2, dtype=torch.int32), "eos": 1}),
    "res without eos": (ValueError, None, {"res": torch.zeros(2, 2, dtype=torch.long)}),
    "notime float": (TypeError, None, {"notime": torch.zeros(2)}),
    "enc_len count": (ValueError, None, {"enc_len": torch.full((1,), 8, dtype=torch.int32)}),
}


@pytest.mark.parametrize("case", sorted(VERIFY_CASES))
def test_verify_refuses_malformed_buffers(case):
    err, edit, kw = VERIFY_CASES[case]
    with pytest.raises(err):
        _verify(_kernel(), edit=edit, **kw)


def _cross_kv(k, U=2, T=8, Tc=8, edit=None):
    buf = dict(enc=torch.zeros(U, T, D, dtype=torch.float16),
               cross_k=torch.zeros(L, U, H, Tc, DK, dtype=torch.float16),
               cross_v=torch.zeros(L, U, H, Tc, DK, dtype=torch.float16))  # fmt: skip
    if edit is not None:
        edit(buf)

    def handle():
        raise _Reached()

    k._xkv_handle = handle
    return k.cross_kv_fn(buf["enc"], buf["cross_k"], buf["cross_v"])


def test_cross_kv_checks():
    with pytest.raises(_Reached):
        _cross_kv(_kernel(), Tc=12)  # (cache frames past T are left alone)
    with pytest.raises(TypeError):
        _cross_kv(_kernel(), edit=lambda b: b.update(enc=b["enc"].float()))
    with pytest.raises(TypeError):
        _cross_kv(_kernel(), edit=lambda b: b.update(enc=b["enc"][..., :128].contiguous()))
    with pytest.raises(TypeError):
        _cross_kv(_kernel(), edit=lambda b: b.update(cross_v=b["cross_v"][:, :1].contiguous()))
    with pytest.raises(ValueError):
        _cross_kv(_kernel(), Tc=4)
    k = _kernel()
    k.device = torch.device("cuda", 0)  # buffers elsewhere than the kernel's device
    with pytest.raises(ValueError):
        _cross_kv(k)


def test_buffers_elsewhere_than_the_kernels_device_are_refused():
    k = _kernel()
    k.device = torch.device("cuda", 0)
    with pytest.raises(ValueError):
        _step(k, _greedy())
    with pytest.raises(ValueError):
        _beam_step(k, _beam())
    with pytest.raises(ValueError):
        _verify(k)


def test_outputs_on_the_host_are_refused():
    # an output buffer (one the kernel writes) on another device than the kernel's: here a meta tensor
    with pytest.raises(ValueError):
        _step(_kernel(), _greedy(), pred=torch.zeros(2, 1, dtype=torch.long, device="meta"))
    for name in ("score", "active", "parent", "token"):
        buf = _beam()
        buf[name] = buf[name].to("meta")
        with pytest.raises(ValueError):
            _beam_step(_kernel(), buf)
    with pytest.raises(ValueError):
        _beam_step(_kernel(), _beam(), shared=torch.zeros(2, 2, 2, dtype=torch.int32, device="meta"))
