"""The decoder-step kernel behind owsm-trt's megakernel launcher interface.

:class:`B200Decoder` has the contract of ``MegaDecoder`` / ``RingDecoder`` (src/owsm_trt/megakernel.py:537-685,
src/owsm_trt/megakernel_ring.py:737-861): built from a ``Decoder`` module, ``step_fn(tokens, offset, self_k,
self_v, cross_k, cross_v, logits, new_kv, kind="decode", pred=None, solo=False, notime=None)`` returns a
graph-capturable ``run()`` that fills ``logits`` and ``new_kv``, writes the new keys/values into the cache
(``run.writes_cache``) and, with ``pred``, the argmax (``run.writes_pred``). So ``MegaBackend``, the
sessions and ``OWSM.from_pretrained(..., decoder_kernel=...)`` can use it unchanged.

Additions (keyword-only, optional): ``enc_len`` (int32 [U] frames per utterance: a key-padding mask),
``rows_per_utt`` (rows sharing one utterance's cross K/V, e.g. the beam), :meth:`B200Decoder.verify_fn` (a
verify call of the speculative greedy session: the call on its input rows + the argmax under the timestamp rules
+ the drafted tokens accepted, in one launch) and :meth:`B200Decoder.beam_fn` (the call + BeamSession._select's
top-K + the cache reorder in one launch).

All compute runs in ``libowsmdec.so`` (CUDA, sm_100a), called through ctypes with raw device pointers.
"""

from __future__ import annotations

import ctypes as C
import logging
import math

import torch

from . import _lib
from .synthetic import sinusoidal_positions

log = logging.getLogger(__name__)


def _state_of(decoder) -> tuple[dict, int, torch.Tensor | None, float]:
    """(state dict in the reference naming, heads, positional table or None, LayerNorm eps)."""
    if isinstance(decoder, dict):
        raise TypeError("give (state_dict, heads) as B200Decoder.from_state_dict")
    sd = {k: v for k, v in decoder.state_dict().items()}
    heads = decoder.decoders[0].self_attn.h
    pe = getattr(decoder, "pe", None)
    eps = float(decoder.after_norm.eps)
    return sd, heads, pe, eps


class B200Decoder:
    """The decoder of an encoder-decoder OWSM model as one persistent sm_100a kernel per call."""

    name = "b200-megakernel"
    argmax = True  # step_fn takes pred
    max_tokens = 4096  # rows x window of one call (larger greedy calls run as row slices of up to 64 tokens)
    solo_differs = False  # a single-row call is the same call with or without an encoder alongside

    @torch.no_grad()
    def __init__(self, decoder, device: torch.device | str = "cuda", programs: int | None = None, **opts):
        sd, heads, pe, eps = _state_of(decoder)
        self._init(sd, heads, torch.device(device), programs, pe=pe, eps=eps, **opts)

    @classmethod
    def from_state_dict(cls, sd: dict, heads: int, device="cuda", programs: int | None = None, pe=None,
                        eps: float = 1e-12, **opts) -> "B200Decoder":  # fmt: skip
        obj = cls.__new__(cls)
        obj._init(sd, heads, torch.device(device), programs, pe=pe, eps=eps, **opts)
        return obj

    @torch.no_grad()
    def _init(self, sd: dict, heads: int, device: torch.device, programs, pe=None, eps=1e-12, max_pos=5000,
              weight_dtype=torch.float32):  # fmt: skip
        if device.type != "cuda":
            raise ValueError("B200Decoder needs a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        lib = _lib.lib()
        self.device = device
        V, D = sd["embed.0.weight"].shape
        L = 1 + max(int(k.split(".")[1]) for k in sd if k.startswith("decoders."))
        pre = "decoders.0."
        F = sd[pre + "feed_forward.w_1.weight"].shape[0]
        self.L, self.D, self.H, self.F, self.V = L, D, heads, F, V
        if pe is None:
            pe = sinusoidal_positions(max_pos, D)
        fdt = weight_dtype
        keep = []  # device copies alive during create

        def dev(t, dt=torch.float32):
            t = t.detach().to(device=device, dtype=dt).contiguous()
            keep.append(t)
            return t.data_ptr()

        layers = (_lib.Layer * L)()
        for i in range(L):
            p = f"decoders.{i}."
            ly = layers[i]
            sa, xa, ff = p + "self_attn.", p + "src_attn.", p + "feed_forward."
            if sa + "linear_qkv.weight" in sd:
                ly.wq = dev(sd[sa + "linear_qkv.weight"], fdt)
                ly.bq = dev(sd[sa + "linear_qkv.bias"])
                ly.wk = ly.wv = ly.bk = ly.bv = None
            else:
                ly.wq, ly.wk, ly.wv = (dev(sd[sa + f"linear_{n}.weight"], fdt) for n in "qkv")
                ly.bq, ly.bk, ly.bv = (dev(sd[sa + f"linear_{n}.bias"]) for n in "qkv")
            ly.wo, ly.bo = dev(sd[sa + "linear_out.weight"], fdt), dev(sd[sa + "linear_out.bias"])
            ly.wcq, ly.bcq = dev(sd[xa + "linear_q.weight"], fdt), dev(sd[xa + "linear_q.bias"])
            ly.wco, ly.bco = dev(sd[xa + "linear_out.weight"], fdt), dev(sd[xa + "linear_out.bias"])
            ly.w1, ly.b1 = dev(sd[ff + "w_1.weight"], fdt), dev(sd[ff + "w_1.bias"])
            ly.w2, ly.b2 = dev(sd[ff + "w_2.weight"], fdt), dev(sd[ff + "w_2.bias"])
            for n in (1, 2, 3):
                setattr(ly, f"ln{n}_g", dev(sd[p + f"norm{n}.weight"]))
                setattr(ly, f"ln{n}_b", dev(sd[p + f"norm{n}.bias"]))
        w = _lib.Weights()
        w.weight_dtype = _lib.F32 if fdt == torch.float32 else _lib.F16
        w.emb = dev(sd["embed.0.weight"], fdt)
        w.pe = dev(pe)
        w.layers = C.cast(layers, C.POINTER(_lib.Layer))
        w.lnf_g, w.lnf_b = dev(sd["after_norm.weight"]), dev(sd["after_norm.bias"])
        w.wout, w.bout = dev(sd["output_layer.weight"], fdt), dev(sd["output_layer.bias"])
        dims = _lib.Dims(L, D, heads, F, V, pe.shape[0], float(eps), float(math.sqrt(D)))
        h = C.c_void_p()
        with torch.cuda.device(device):
            _lib.check(lib.owsm_dec_create(C.byref(dims), C.byref(w), device.index or 0, programs or 0, C.byref(h)),
                       "owsm_dec_create")  # fmt: skip
        del keep
        self._h = h
        self._xkv = None  # the K/V projection handle, made on first use (cross_kv_fn)
        self._xkv_src = {k: v for k, v in sd.items() if ".src_attn.linear_k." in k or ".src_attn.linear_v." in k}
        self._plans: dict[tuple, C.c_void_p] = {}
        self.programs = self._plan_info(self._plan(1, 1, 16, 16, 1, 0))[0]
        self.max_pos = pe.shape[0]

    # ------------------------------------------------------------------ plans
    def _plan(self, R: int, S: int, Cc: int, T: int, G: int, beam: int) -> C.c_void_p:
        key = (R, S, Cc, T, G, beam)
        if key not in self._plans:
            p = C.c_void_p()
            with torch.cuda.device(self.device):
                _lib.check(_lib.lib().owsm_dec_plan(self._h, R, S, Cc, T, G, beam, C.byref(p)), "owsm_dec_plan")
            self._plans[key] = p
        return self._plans[key]

    @staticmethod
    def _plan_info(p) -> tuple[int, int, int]:
        a, b, c = C.c_int(), C.c_int(), C.c_int64()
        _lib.check(_lib.lib().owsm_dec_plan_info(p, C.byref(a), C.byref(b), C.byref(c)), "owsm_dec_plan_info")
        return a.value, b.value, c.value

    def close(self) -> None:
        if getattr(self, "_xkv", None):
            _lib.lib().owsm_xkv_destroy(self._xkv)
            self._xkv = None
        if getattr(self, "_h", None):
            lib = _lib.lib()
            for p in self._plans.values():
                lib.owsm_dec_plan_destroy(p)
            self._plans.clear()
            lib.owsm_dec_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 (interpreter shutdown)
            pass

    # ------------------------------------------------------------------ errors
    def check(self) -> None:
        """Raise if a bounded in-kernel wait of an earlier call gave up (its results were garbage);
        resets the plans' counters (``MegaDecoder.check``, src/owsm_trt/megakernel.py:616-622)."""
        code = _lib.lib().owsm_dec_get_error(self._h)
        if code != _lib.OK:
            for p in self._plans.values():
                _lib.lib().owsm_dec_plan_reset(p)
            raise RuntimeError("the decoder kernel timed out at a grid barrier (were all its CTAs resident?)")

    def set_path(self, path: int) -> None:
        """Which kernel later calls use: 0 the default (the dense tcgen05 kernel for greedy calls of more than 32
        tokens, the cluster kernel for the others where it applies), 1 the grid-stage kernel, 2 the cluster kernel
        or an error, 3 the dense kernel or an error. Drops the cached plans."""
        _lib.check(_lib.lib().owsm_dec_set_path(self._h, int(path)), "owsm_dec_set_path")
        for p in self._plans.values():
            _lib.lib().owsm_dec_plan_destroy(p)
        self._plans.clear()

    def plan_kernel(self, run) -> str:
        """"cluster", "grid" or "dense": the kernel behind a step_fn / beam_fn closure."""
        return {1: "grid", 2: "cluster", 3: "dense"}[_lib.lib().owsm_dec_plan_kernel(run.plan)]

    def launches(self, run) -> int:
        """Kernel launches of one call of a step_fn / beam_fn closure (1, or its row slices)."""
        return int(_lib.lib().owsm_dec_plan_launches(run.plan))

    def set_max_spin(self, polls: int) -> None:
        """Testing hook: the in-kernel wait limit of later calls (0: the default)."""
        _lib.check(_lib.lib().owsm_dec_set_max_spin(self._h, polls), "owsm_dec_set_max_spin")

    # ------------------------------------------------------------------ cross K/V
    def _xkv_handle(self):
        if self._xkv is None:
            keep = []

            def dev(t, dt=torch.float32):
                t = t.detach().to(device=self.device, dtype=dt).contiguous()
                keep.append(t)
                return t.data_ptr()

            layers = (_lib.XkvLayer * self.L)()
            for i in range(self.L):
                p = f"decoders.{i}.src_attn."
                ly = layers[i]
                ly.wk, ly.wv = dev(self._xkv_src[p + "linear_k.weight"]), dev(self._xkv_src[p + "linear_v.weight"])
                ly.bk, ly.bv = dev(self._xkv_src[p + "linear_k.bias"]), dev(self._xkv_src[p + "linear_v.bias"])
            h = C.c_void_p()
            with torch.cuda.device(self.device):
                _lib.check(_lib.lib().owsm_xkv_create(self.L, self.D, self.H, _lib.F32, layers, self.device.index or 0,
                                                      C.byref(h)), "owsm_xkv_create")  # fmt: skip
            self._xkv = h
        return self._xkv

    def cross_kv_fn(self, enc: torch.Tensor, cross_k: torch.Tensor, cross_v: torch.Tensor):
        """Every layer's cross-attention keys / values of encoder output ``enc`` [U, T, D] (fp16) into ``cross_k`` /
        ``cross_v`` [L, U, H, T', 64] (fp16, T' >= T; frames T.. untouched): ``Decoder.cross_kv``
        (src/owsm_trt/modeling.py:490-499) as one tcgen05 GEMM. Returns a graph-capturable ``run()``."""
        U, T, D = enc.shape
        if enc.dtype != torch.float16 or not enc.is_contiguous() or D != self.D:
            raise TypeError(f"enc must be contiguous fp16 [U, T, {self.D}]")
        for t in (cross_k, cross_v):
            if t.dtype != torch.float16 or not t.is_contiguous() or t.shape[:3] != (self.L, U, self.H) or t.shape[4] != 64:
                raise TypeError(f"cross_k / cross_v must be contiguous fp16 [{self.L}, {U}, {self.H}, T', 64]")
        t_cap = cross_k.shape[3]
        if t_cap < T or cross_v.shape != cross_k.shape:
            raise ValueError("cross_k / cross_v need at least T frames")
        for t in (enc, cross_k, cross_v):
            if t.device != self.device:
                raise ValueError(f"enc, cross_k and cross_v must be on {self.device}")
        h = self._xkv_handle()
        fn, dev = _lib.lib().owsm_xkv_run, self.device

        def run() -> None:
            _lib.check(fn(h, torch.cuda.current_stream(dev).cuda_stream, enc.data_ptr(), U, T, t_cap,
                          cross_k.data_ptr(), cross_v.data_ptr()), "owsm_xkv_run")  # fmt: skip

        run.buffers = (enc, cross_k, cross_v)
        return run

    def cross_kv(self, enc: torch.Tensor) -> torch.Tensor:
        """``Decoder.cross_kv`` with its return layout: [L, 2, U, H, T, 64] fp16 (allocates)."""
        U, T, _ = enc.shape
        kv = torch.empty(2, self.L, U, self.H, T, 64, device=self.device, dtype=torch.float16)
        self.cross_kv_fn(enc.to(self.device, torch.float16).contiguous(), kv[0], kv[1])()
        return kv.transpose(0, 1)

    def check_cross_kv(self) -> None:
        """Raise if a bounded wait of an earlier K/V projection gave up."""
        if self._xkv is not None and _lib.lib().owsm_xkv_get_error(self._xkv) != _lib.OK:
            raise RuntimeError("the K/V projection kernel timed out")

    # ------------------------------------------------------------------ calls
    def _validate(self, tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv, G):
        R, S = tokens.shape
        L, H, dk = self.L, self.H, 64
        if tokens.dtype != torch.int64 or offset.dtype != torch.int64:
            raise TypeError("tokens and offset must be int64")
        if tokens.stride(1) != 1:
            raise ValueError("tokens must be contiguous along the window")
        for name, t in (("self_k", self_k), ("self_v", self_v), ("cross_k", cross_k), ("cross_v", cross_v),
                        ("new_kv", new_kv)):  # fmt: skip
            if t.dtype != torch.float16 or not t.is_contiguous():
                raise TypeError(f"{name} must be contiguous fp16")
        if logits.dtype != torch.float32 or not logits.is_contiguous():
            raise TypeError("logits must be contiguous fp32")
        Cc = self_k.shape[3]
        T = cross_k.shape[3]
        if self_k.shape != (L, R, H, Cc, dk) or self_v.shape != self_k.shape:
            raise ValueError(f"self_k/self_v must be [L, R, H, C, 64] = {(L, R, H, Cc, dk)}, got {tuple(self_k.shape)}")
        if cross_k.shape != (L, R // G, H, T, dk) or cross_v.shape != cross_k.shape:
            raise ValueError(f"cross_k/cross_v must be [L, R/rows_per_utt, H, T, 64], got {tuple(cross_k.shape)}")
        if logits.shape != (R, S, self.V) or new_kv.shape != (L, 2, R, H, S, dk):
            raise ValueError("logits [R, S, V] / new_kv [L, 2, R, H, S, 64] shape mismatch")
        for t in (tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv):
            if t.device != self.device:
                raise ValueError(f"all buffers must be on {self.device}")
        return R, S, Cc, T

    def _check_enc_len(self, enc_len, n: int) -> None:
        """The frames per utterance, if given: contiguous int32 [n] on the kernel's device (the kernel reads n)."""
        if enc_len is not None and (enc_len.dtype != torch.int32 or enc_len.numel() != n
                                    or not enc_len.is_contiguous() or enc_len.device != self.device):  # fmt: skip
            raise ValueError(f"enc_len must be contiguous int32 [R / rows_per_utt] = [{n}] on {self.device}")

    def step_fn(self, tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv, kind="decode", pred=None,
                solo=False, notime=None, *, enc_len=None, rows_per_utt: int = 1):  # fmt: skip
        """The call on these buffers (see the module docstring). ``notime`` = (flags [R] bool, first timestamp
        token, last one): the argmax of flagged rows leaves those ids out."""
        G = int(rows_per_utt)
        R, S, Cc, T = self._validate(tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv, G)
        if pred is not None and (pred.dtype != torch.int64 or pred.shape != (R, S) or not pred.is_contiguous()):
            raise ValueError("pred must be contiguous int64 [R, S]")
        if pred is not None and pred.device != self.device:
            raise ValueError(f"pred must be on {self.device}")
        ntm, ft, lt = None, 0, -1
        if notime is not None and pred is not None:
            flags, ft, lt = notime
            # the kernel reads the caller's flags at every run (sessions set them in place after building their
            # calls, runtime.py:579-584): one byte per row, bool or uint8, no copy
            if flags.dtype not in (torch.bool, torch.uint8) or not flags.is_contiguous() or flags.shape != (R,):
                raise TypeError("notime flags must be a contiguous bool or uint8 tensor [R]")
            if flags.device != self.device:
                raise ValueError(f"notime flags must be on {self.device}")
            ntm = flags
        self._check_enc_len(enc_len, R // G)
        plan = self._plan(R, S, Cc, T, G, 0)
        lib = _lib.lib()
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        args = (plan, None, ptr(tokens), tokens.stride(0), ptr(offset), offset.stride(0), ptr(self_k), ptr(self_v),
                ptr(cross_k), ptr(cross_v), ptr(enc_len), ptr(logits), ptr(new_kv), ptr(pred), ptr(ntm), int(ft),
                int(lt))  # fmt: skip
        fn = lib.owsm_dec_step
        dev = self.device

        def run() -> None:
            stream = torch.cuda.current_stream(dev).cuda_stream
            _lib.check(fn(args[0], stream, *args[2:]), "owsm_dec_step")

        run.writes_cache = True
        run.writes_pred = pred is not None
        run.plan = plan
        run.beam = False
        run.buffers = (tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv, pred, ntm, enc_len)
        run.programs = self._plan_info(plan)[0]
        run.kernel = self
        return run

    def verify_fn(self, inp, self_k, self_v, cross_k, cross_v, logits, new_kv, pred, *, rules=None, notime=None,
                  res=None, eos=None, enc_len=None, rows_per_utt: int = 1):  # fmt: skip
        """A verify call of the speculative greedy session in one launch (_Bound.body, runtime.py:1292-1316):
        the decoder call on the tokens and offsets of ``inp`` (int64 [R, W + 4] = W tokens, offset, timestamps
        so far, last timestamp, first generated position), the argmax after every position into ``pred``
        [R, W] -- under ``rules`` (the session's TimestampRules, or (first_time, last_time, eos)) with
        ``notime`` [R] bool the rows whose primer holds <notimestamps> (_Verify.predict, runtime.py:1251-1267)
        -- and, with ``res`` int64 [R, 2], the drafted tokens accepted and the argmax after them
        (_Verify.accept, runtime.py:1269-1278; ``eos`` defaults to the rules'). ``run.writes_res``: the
        session's kernels.choose and kernels.accept have nothing left to do."""
        if inp.dtype != torch.int64 or inp.dim() != 2 or inp.stride(1) != 1:
            raise TypeError("inp must be int64 [R, W + 4], contiguous along a row")
        R, W = inp.shape[0], inp.shape[1] - 4
        if W < 1:
            raise ValueError("inp rows are [W tokens, offset, #timestamps, last timestamp, first position]")
        G = int(rows_per_utt)
        tokens, offset = inp[:, :W], inp[:, W]
        R, S, Cc, T = self._validate(tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv, G)
        if pred.dtype != torch.int64 or pred.shape != (R, S) or not pred.is_contiguous():
            raise ValueError("pred must be contiguous int64 [R, W]")
        if res is not None and (res.dtype != torch.int64 or res.shape != (R, 2) or not res.is_contiguous()):
            raise ValueError("res must be contiguous int64 [R, 2]")
        ft, lt, on = 0, -1, 0
        if rules is not None:
            ft, lt, r_eos = (rules.first_time, rules.last_time, rules.eos) if hasattr(rules, "eos") else rules
            eos = r_eos if eos is None else eos
            on = 1
        if res is not None and eos is None:
            raise ValueError("res needs the <eos> id: pass eos= or the session's TimestampRules")
        eos = -1 if eos is None else eos
        ntm = None
        if notime is not None:
            if notime.dtype not in (torch.bool, torch.uint8) or not notime.is_contiguous() or notime.shape != (R,):
                raise TypeError("notime must be a contiguous bool or uint8 tensor [R]")
            ntm = notime
        for t in (pred, res, ntm, enc_len):
            if t is not None and t.device != self.device:
                raise ValueError(f"all buffers must be on {self.device}")
        self._check_enc_len(enc_len, R // G)
        plan = self._plan(R, S, Cc, T, G, 0)
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        args = (ptr(inp), inp.stride(0), ptr(self_k), ptr(self_v), ptr(cross_k), ptr(cross_v), ptr(enc_len),
                ptr(logits), ptr(new_kv), ptr(pred), ptr(ntm), on, int(ft), int(lt), int(eos), ptr(res))  # fmt: skip
        fn = _lib.lib().owsm_dec_step_verify
        dev = self.device

        def run() -> None:
            _lib.check(fn(plan, torch.cuda.current_stream(dev).cuda_stream, *args), "owsm_dec_step_verify")

        run.writes_cache = True
        run.writes_pred = True
        run.writes_res = res is not None
        run.reads_inp = True
        run.plan = plan
        run.beam = False
        run.buffers = (inp, self_k, self_v, cross_k, cross_v, logits, new_kv, pred, ntm, res, enc_len)
        run.programs = self._plan_info(plan)[0]
        run.kernel = self
        return run

    def beam_fn(self, tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv, score, active, parent,
                token, *, beam: int, enc_len=None, shared=None):  # fmt: skip
        """One beam step (S = 1, rows = batch x beam, utterance-major, cross K/V one per utterance): the decoder
        call, then BeamSession._select step 1 (runtime.py:1399-1411) -- ``score`` [R] fp32 is replaced by the new
        scores, ``parent`` / ``token`` [R] int64 written -- and the cache rows replaced by their parents'.
        ``shared`` (int32 [R / beam, beam, beam], optional): per utterance, how many leading cache slots each pair
        of its rows holds in common; with it a row copies only its parent's slots past that (the call keeps the
        record up to date). Fill it with the prompt length when the rows start from the same prompt."""
        R, S, Cc, T = self._validate(tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv, beam)
        if S != 1:
            raise ValueError("beam steps feed one token per row")
        for name, t, dt in (("score", score, torch.float32), ("active", active, torch.uint8),
                            ("parent", parent, torch.int64), ("token", token, torch.int64)):  # fmt: skip
            if t.dtype != dt or t.shape != (R,) or not t.is_contiguous():
                raise TypeError(f"{name} must be contiguous {dt} [R]")
            if t.device != self.device:
                raise ValueError(f"{name} must be on {self.device}")
        if shared is not None and (shared.dtype != torch.int32 or shared.shape != (R // beam, beam, beam)
                                   or not shared.is_contiguous()):  # fmt: skip
            raise TypeError("shared must be contiguous int32 [R / beam, beam, beam]")
        if shared is not None and shared.device != self.device:
            raise ValueError(f"shared must be on {self.device}")
        self._check_enc_len(enc_len, R // beam)
        plan = self._plan(R, S, Cc, T, beam, beam)
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        args = (ptr(tokens), tokens.stride(0), ptr(offset), offset.stride(0), ptr(self_k), ptr(self_v), ptr(cross_k),
                ptr(cross_v), ptr(enc_len), ptr(logits), ptr(new_kv), ptr(score), ptr(active), ptr(parent),
                ptr(token), ptr(shared))  # fmt: skip
        fn = _lib.lib().owsm_dec_beam_step
        dev = self.device

        def run() -> None:
            _lib.check(fn(plan, torch.cuda.current_stream(dev).cuda_stream, *args), "owsm_dec_beam_step")

        run.writes_cache = True
        run.plan = plan
        run.beam = True
        run.buffers = (tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv, score, active, parent, token,
                       shared, enc_len)  # fmt: skip
        return run
