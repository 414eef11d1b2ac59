"""The whole decoder (the reference's LlamaModel forward with greedy sampling) through
the C++ host layer's C interface (flashmlx_b200/host/fmh.h, libflashmoe_host.so).

The forward loop itself is C++ (host/decoder.cpp): every op a libflashmoe call on one
stream.  This module binds it for Python callers (the tests and the bench): weights are
torch tensors on the device in MLX's layout, from numpy arrays (synthetic.make_decoder)
or generated on the device (device_decoder_weights), or a model directory is opened.
Importing it fails loudly when the libraries have not been built.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

from . import _lib, ops

HOST_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libflashmoe_host.so")


class DecoderConfig(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("vocab", C.c_int), ("intermediate", C.c_int), ("rope_theta", C.c_float),
                ("rms_eps", C.c_float), ("group_size", C.c_int), ("bits", C.c_int),
                ("tie_word_embeddings", C.c_int), ("moe", _lib.MoEConfig)]


class Layer(C.Structure):
    _fields_ = [("in_norm", C.c_void_p), ("post_norm", C.c_void_p), ("q", _lib.QWeight), ("k", _lib.QWeight),
                ("v", _lib.QWeight), ("o", _lib.QWeight), ("q_bias", C.c_void_p), ("k_bias", C.c_void_p),
                ("v_bias", C.c_void_p), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("is_moe", C.c_int),
                ("moe", _lib.MoEWeights), ("gate", _lib.QWeight),
                ("up", _lib.QWeight), ("down", _lib.QWeight)]


class Weights(C.Structure):
    _fields_ = [("embed_table", C.c_void_p), ("embed_q", _lib.QWeight), ("norm", C.c_void_p),
                ("lm_head", _lib.QWeight), ("layers", C.POINTER(Layer))]


_p, _i = C.c_void_p, C.c_int
SIGNATURES = {
    "fmh_decoder_create": (_i, [C.POINTER(DecoderConfig), C.POINTER(Weights), _i, _i, _i, _p, C.POINTER(_p)]),
    "fmh_decoder_open": (_i, [C.c_char_p, _i, _i, _i, _p, C.POINTER(_p)]),
    "fmh_decoder_close": (None, [_p]),
    "fmh_last_error": (C.c_char_p, [_p]),
    "fmh_decoder_forward": (_i, [_p, _p, _i, _i, _p]),
    "fmh_decoder_logits": (_p, [_p]),
    "fmh_decoder_copy_logits": (_i, [_p, _p, _i]),
    "fmh_decoder_offset": (_i, [_p]),
    "fmh_decoder_reset": (_i, [_p]),
    "fmh_decoder_sync": (_i, [_p]),
    "fmh_decoder_generate": (_i, [_p, _p, _i, _i, _i, _p]),
    "fmh_decoder_handle": (_p, [_p]),
}

_host = None


def load() -> C.CDLL:
    global _host
    if _host is not None:
        return _host
    if not os.path.exists(HOST_LIB_PATH):
        raise ImportError(f"libflashmoe_host is not built ({HOST_LIB_PATH} missing); run `python -m flashmlx_b200.build`")
    _lib.load()  # libflashmoe first (the host library links it)
    lib = C.CDLL(HOST_LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype, f.argtypes = res, args
    _host = lib
    return lib


def _index(dev: torch.device) -> int:
    return dev.index if dev.index is not None else torch.cuda.current_device()


def _q(t):
    return _lib.QWeight(*(x.data_ptr() if x is not None else None for x in t)) if t is not None else _lib.QWeight()


def _moe_config(m) -> _lib.MoEConfig:
    return _lib.MoEConfig(m.hidden, m.inter, m.num_experts, m.top_k, m.group_size, m.bits, int(m.norm_topk_prob),
                          m.shared_inter, 0, 0)


def config_of(shape) -> DecoderConfig:
    """The C description of a synthetic.DecoderShape."""
    return DecoderConfig(shape.hidden, shape.layers, shape.n_heads, shape.n_kv_heads, shape.head_dim, shape.vocab,
                         shape.intermediate,
                         float(shape.rope_theta), float(shape.rms_eps), shape.group_size, shape.bits,
                         int(shape.tie_word_embeddings), _moe_config(shape.moe))


def upload_weights(w: dict, device) -> dict:
    """numpy weights (synthetic.make_decoder layout) -> the same dict of device tensors."""
    def q(t):
        return tuple(None if a is None else (ops.u32_from_numpy(a, device) if i == 0 else ops.bf16_from_numpy(a, device))
                     for i, a in enumerate(t))

    def moe(m):
        d = {"router_w": ops.bf16_from_numpy(m["router_w"], device)}
        for k in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down"):
            if k in m:
                d[k] = q(m[k])
        if "shared_expert_gate_w" in m:
            d["shared_expert_gate_w"] = ops.bf16_from_numpy(m["shared_expert_gate_w"], device)
        return d

    out = {"embed": q(w["embed"]), "norm": ops.bf16_from_numpy(w["norm"], device), "layers": []}
    if "lm_head" in w:
        out["lm_head"] = q(w["lm_head"])
    for lw in w["layers"]:
        d = {k: ops.bf16_from_numpy(lw[k], device) for k in ("in_norm", "post_norm")}
        for k in ("q", "k", "v", "o"):
            d[k] = q(lw[k])
        for k in ("q_bias", "k_bias", "v_bias", "q_norm", "k_norm"):
            if lw.get(k) is not None:
                d[k] = ops.bf16_from_numpy(lw[k], device)
        if "moe" in lw:
            d["moe"] = moe(lw["moe"])
        else:
            d["mlp"] = {k: q(lw["mlp"][k]) for k in ("gate", "up", "down")}
        out["layers"].append(d)
    return out


def device_decoder_weights(shape, seed: int, device) -> dict:
    """Random-init weights generated on the device (the distributions of
    synthetic.make_decoder, not its values): codes uniform, scales |N(0, 0.02)| (0.1 for
    the embedding), biases -8 scale, norms 1 + 0.1 N, attention biases 0.02 N."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    dev = torch.device(device)
    gs = shape.group_size

    def qm(n, k, std=0.02):
        w = torch.randint(-2 ** 31, 2 ** 31, (n, k // 8), dtype=torch.int32, device=dev, generator=g)
        s = (torch.randn(n, k // gs, device=dev, generator=g).abs() * std).to(torch.bfloat16)
        return w, s, (s.float() * -8.0).to(torch.bfloat16)

    def vec(n, mean, std):
        return (mean + std * torch.randn(n, device=dev, generator=g)).to(torch.bfloat16)

    m = shape.moe
    H, nh, nkv, d = shape.hidden, shape.n_heads, shape.n_kv_heads, shape.head_dim
    out = {"embed": qm(shape.vocab, H, 0.1), "norm": vec(H, 1.0, 0.1), "layers": []}
    if not shape.tie_word_embeddings:
        out["lm_head"] = qm(shape.vocab, H)
    for li in range(shape.layers):
        lw = {"in_norm": vec(H, 1.0, 0.1), "post_norm": vec(H, 1.0, 0.1), "q": qm(nh * d, H), "k": qm(nkv * d, H),
              "v": qm(nkv * d, H), "o": qm(H, nh * d)}
        if shape.attn_bias:
            lw["q_bias"], lw["k_bias"], lw["v_bias"] = vec(nh * d, 0, 0.02), vec(nkv * d, 0, 0.02), vec(nkv * d, 0, 0.02)
        if shape.qk_norm:
            lw["q_norm"], lw["k_norm"] = vec(d, 1.0, 0.1), vec(d, 1.0, 0.1)
        if li in shape.dense_layers:
            I = shape.intermediate
            lw["mlp"] = {"gate": qm(I, H), "up": qm(I, H), "down": qm(H, I)}
            out["layers"].append(lw)
            continue
        E, I = m.num_experts, m.inter
        mo = {"router_w": vec(E * H, 0, 0.02).view(E, H)}
        gw, gsc, gb = qm(E * I, H)
        uw, usc, ub = qm(E * I, H)
        dw, dsc, db = qm(E * H, I)
        mo["gate"] = (gw.view(E, I, -1), gsc.view(E, I, -1), gb.view(E, I, -1))
        mo["up"] = (uw.view(E, I, -1), usc.view(E, I, -1), ub.view(E, I, -1))
        mo["down"] = (dw.view(E, H, -1), dsc.view(E, H, -1), db.view(E, H, -1))
        if m.shared_inter:
            mo["shared_gate"], mo["shared_up"] = qm(m.shared_inter, H), qm(m.shared_inter, H)
            mo["shared_down"] = qm(H, m.shared_inter)
            mo["shared_expert_gate_w"] = vec(H, 0, 0.02).view(1, H)
        lw["moe"] = mo
        out["layers"].append(lw)
    return out


class Decoder:
    """A C++ Decoder (host/decoder.cpp) over device weights, on torch's current stream of
    `device` at creation.  forward(ids [B, L] int32) -> next ids [B]; generate(prompt,
    steps) -> [B, steps]."""

    def __init__(self, ptr, keep=None, stream=None):
        self._d = ptr
        self._keep = keep  # device tensors the C++ side points at
        self._stream = stream
        self.lib = load()

    @classmethod
    def from_weights(cls, shape, weights: dict, device, max_batch: int, max_len: int):
        lib = load()
        dev = torch.device(device)
        layers = (Layer * shape.layers)()
        for i, lw in enumerate(weights["layers"]):
            L = layers[i]
            L.in_norm, L.post_norm = lw["in_norm"].data_ptr(), lw["post_norm"].data_ptr()
            L.q, L.k, L.v, L.o = _q(lw["q"]), _q(lw["k"]), _q(lw["v"]), _q(lw["o"])
            for k in ("q_bias", "k_bias", "v_bias", "q_norm", "k_norm"):
                setattr(L, k, lw[k].data_ptr() if lw.get(k) is not None else None)
            if "mlp" in lw:  # a dense SwiGLU layer
                L.is_moe = 0
                L.gate, L.up, L.down = _q(lw["mlp"]["gate"]), _q(lw["mlp"]["up"]), _q(lw["mlp"]["down"])
                continue
            L.is_moe = 1
            mo = lw["moe"]
            W = _lib.MoEWeights()
            W.router_w = mo["router_w"].data_ptr()
            for k in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down"):
                if k in mo:
                    setattr(W, k, _q(mo[k]))
            if "shared_expert_gate_w" in mo:
                W.shared_expert_gate_w = mo["shared_expert_gate_w"].data_ptr()
            L.moe = W
        table = ops.dequantize(*weights["embed"], group_size=shape.group_size, bits=shape.bits)
        wt = Weights()
        wt.embed_table = table.data_ptr()
        wt.embed_q = _q(weights["embed"])
        wt.norm = weights["norm"].data_ptr()
        if "lm_head" in weights:
            wt.lm_head = _q(weights["lm_head"])
        wt.layers = C.cast(layers, C.POINTER(Layer))
        cfg = config_of(shape)
        stream = torch.cuda.current_stream(dev)
        out = C.c_void_p()
        torch.cuda.synchronize(dev)  # the dequantized table is ready before another stream may read it
        rc = lib.fmh_decoder_create(C.byref(cfg), C.byref(wt), _index(dev), max_batch, max_len,
                                    C.c_void_p(stream.cuda_stream), C.byref(out))
        if rc != 0:
            raise _lib.FlashMoEError(rc, f"fmh_decoder_create: status {rc}")
        return cls(out, keep=(weights, table, layers), stream=stream)

    @classmethod
    def open(cls, model_dir: str, device, max_batch: int, max_len: int):
        lib = load()
        dev = torch.device(device)
        stream = torch.cuda.current_stream(dev)
        out = C.c_void_p()
        rc = lib.fmh_decoder_open(model_dir.encode(), _index(dev), max_batch, max_len,
                                  C.c_void_p(stream.cuda_stream), C.byref(out))
        if rc != 0:
            raise _lib.FlashMoEError(rc, f"fmh_decoder_open: status {rc}")
        return cls(out, stream=stream)

    def _check(self, rc):
        if rc != 0:
            raise _lib.FlashMoEError(rc, self.lib.fmh_last_error(self._d).decode(errors="replace"))

    def forward(self, ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if ids.dtype != torch.int32 or ids.dim() != 2 or not ids.is_contiguous():
            raise ValueError("ids must be a contiguous int32 [B, L] tensor")
        B, L = ids.shape
        nxt = out if out is not None else torch.empty(B, dtype=torch.int32, device=ids.device)
        self._check(self.lib.fmh_decoder_forward(self._d, C.c_void_p(ids.data_ptr()), B, L,
                                                 C.c_void_p(nxt.data_ptr())))
        return nxt

    def logits(self, B: int, vocab: int, device) -> torch.Tensor:
        t = torch.empty(B, vocab, dtype=torch.bfloat16, device=device)
        self._check(self.lib.fmh_decoder_copy_logits(self._d, C.c_void_p(t.data_ptr()), B))
        return t

    @property
    def offset(self) -> int:
        return self.lib.fmh_decoder_offset(self._d)

    def reset(self):
        self._check(self.lib.fmh_decoder_reset(self._d))

    def sync(self):
        self._check(self.lib.fmh_decoder_sync(self._d))

    def generate(self, prompt, steps: int):
        import numpy as np
        p = np.ascontiguousarray(prompt, np.int32)
        B, L = p.shape
        out = np.empty((B, steps), np.int32)
        self._check(self.lib.fmh_decoder_generate(self._d, p.ctypes.data_as(C.c_void_p), B, L, steps,
                                                  out.ctypes.data_as(C.c_void_p)))
        return out

    def handle(self) -> "ops.Handle":
        """The decoder's libflashmoe handle as an ops.Handle view (not owned: for
        profile() / profile_report() / sync())."""
        h = ops.Handle.__new__(ops.Handle)
        h.lib = _lib.load()
        h.h = C.c_void_p(self.lib.fmh_decoder_handle(self._d))
        h.device = torch.cuda.current_device()
        h._borrowed = True
        return h

    def close(self):
        if self._d:
            self.lib.fmh_decoder_close(self._d)
            self._d = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
