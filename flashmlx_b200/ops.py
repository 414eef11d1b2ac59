"""Python mirror of the reference's operator calls, running on libflashmoe.

Same names, argument meaning and error behaviour as the MLX calls the reference makes
(server/src/model.cpp):

    quantized_matmul(x, w, scales, biases, transpose=True, group_size=64, bits=4)
        <- mx::quantized_matmul                                   model.cpp:476-480
    gather_qmm(x, w, scales, biases, lhs_indices, rhs_indices, transpose=True,
               group_size=64, bits=4, sorted_indices=False)
        <- mx::gather_qmm                                         model.cpp:703-721
    MoEBlock(config, weights)(x)
        <- LlamaModel::moe_block                                  model.cpp:750-807

Tensors are torch CUDA tensors used only as device buffers: bf16 activations,
uint32 (or int32) packed weights, bf16 scales / biases.  Work is queued on torch's
current stream.  Unsupported arguments raise ValueError / NotImplementedError before
any launch, like MLX's argument checks; device-side failures raise FlashMoEError at
the next `synchronize()`.
"""
from __future__ import annotations

import ctypes as C
import threading
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import FlashMoEError, MoEConfig, MoEOutputs, MoEWeights, QWeight

__all__ = ["Handle", "default_handle", "quantized_matmul", "gather_qmm", "MoEConfig", "MoEWeightsT", "MoEBlock",
           "FlashMoEError", "synchronize", "bf16_from_numpy", "u32_from_numpy", "bf16_to_numpy"]

_tls = threading.local()


class Handle:
    """One libflashmoe handle (device workspace + stream binding)."""

    def __init__(self, device: int | None = None):
        self.lib = _lib.load()
        if device is None:
            device = torch.cuda.current_device()
        self.device = device
        h = C.c_void_p()
        with torch.cuda.device(device):
            st = self.lib.fm_create(C.byref(h), device, C.c_void_p(torch.cuda.current_stream().cuda_stream))
        if st != _lib.FM_OK:
            raise FlashMoEError(st, "fm_create failed: " + self.lib.fm_status_string(st).decode())
        self.h = h

    def close(self):
        if self.h and not getattr(self, "_borrowed", False):  # a borrowed view never destroys
            self.lib.fm_destroy(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, st: int):
        if st != _lib.FM_OK:
            raise FlashMoEError(st, self.lib.fm_last_error(self.h).decode())

    def bind_stream(self, stream: torch.cuda.Stream | None = None):
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        self.check(self.lib.fm_set_stream(self.h, C.c_void_p(s.cuda_stream)))

    def set_path(self, path: int):
        self.check(self.lib.fm_set_path(self.h, path))

    def last_path(self) -> int:
        """FM_PATH_GEMV (1) or FM_PATH_TCGEN05 (2): the expert-product path of the
        handle's last call, i.e. which of MLX's two arithmetic forms it followed."""
        return int(self.lib.fm_last_path(self.h))

    def set_route_mode(self, mode: int):
        """FM_ROUTE_GRID (cooperative, grid barriers) or FM_ROUTE_LAST_BLOCK (batches of
        at most 128 tokens: top-k, sort and planning in the block that finishes the router
        GEMV last); FM_ROUTE_AUTO is the grid form."""
        self.check(self.lib.fm_set_route_mode(self.h, mode))

    def sync(self):
        self.check(self.lib.fm_sync_status(self.h))

    def workspace_bytes(self) -> int:
        return int(self.lib.fm_workspace_bytes(self.h))

    def profile(self, on: bool = True):
        self.check(self.lib.fm_profile_enable(self.h, int(on)))

    def profile_report(self, reset: bool = True) -> dict:
        """{kernel name: (launches, total device ms)} since the last reset."""
        buf = (_lib.KernelTime * 32)()
        n = C.c_int(0)
        self.check(self.lib.fm_profile_report(self.h, buf, 32, C.byref(n), int(reset)))
        return {buf[i].name.decode(): (int(buf[i].launches), float(buf[i].total_ms)) for i in range(min(n.value, 32))}


def default_handle(device: int | None = None) -> Handle:
    if device is None:
        device = torch.cuda.current_device()
    hs = getattr(_tls, "handles", None)
    if hs is None:
        hs = _tls.handles = {}
    if device not in hs:
        hs[device] = Handle(device)
    return hs[device]


def synchronize(device: int | None = None):
    default_handle(device).sync()


def bf16_from_numpy(a, device="cuda") -> torch.Tensor:
    """bf16 bit patterns (numpy uint16) -> torch bf16 tensor on `device`."""
    import numpy as np
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device).view(torch.bfloat16)


def u32_from_numpy(a, device="cuda") -> torch.Tensor:
    """packed uint32 words (numpy) -> torch int32 tensor with the same bits on `device`."""
    import numpy as np
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32)).to(device)


def bf16_to_numpy(t: torch.Tensor):
    import numpy as np
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _ptr(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def _need(t, name, dtypes, device):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch tensor")
    if t.device.type != "cuda" or (device is not None and t.device != device):
        raise ValueError(f"{name} must live on {device}")
    if t.dtype not in dtypes:
        raise ValueError(f"{name} has dtype {t.dtype}, expected one of {dtypes}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


_U32 = (torch.uint32, torch.int32)


def quantized_matmul(x, w, scales, biases=None, transpose=True, group_size=64, bits=4, handle=None):
    """x [..., K] bf16 @ dequant(w)^T -> [..., N] bf16 (mx::quantized_matmul, transpose=True)."""
    if not transpose:
        raise NotImplementedError("transpose=False is not implemented")
    _need(x, "x", (torch.bfloat16,), None)
    dev = x.device
    _need(w, "w", _U32, dev)
    _need(scales, "scales", (torch.bfloat16,), dev)
    if biases is not None:
        _need(biases, "biases", (torch.bfloat16,), dev)
    K = x.shape[-1]
    if w.dim() != 2 or w.shape[1] * 32 // bits != K:
        raise ValueError(f"w of shape {tuple(w.shape)} does not match K={K} at {bits} bits")
    N = w.shape[0]
    if scales.shape != (N, K // group_size) or (biases is not None and biases.shape != scales.shape):
        raise ValueError("scales / biases shape mismatch")
    M = x.numel() // K
    out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=dev)
    h = handle or default_handle(dev.index)
    h.bind_stream()
    h.check(h.lib.fm_quantized_matmul(h.h, _ptr(x), M, K, _ptr(w), _ptr(scales), _ptr(biases), N, int(transpose),
                                      group_size, bits, _ptr(out)))
    return out


def linear(x, w, scales, biases=None, group_size=64, bits=4, handle=None):
    """fm_linear: the quantized_matmul of a dense layer (LlamaModel::linear_fast), without
    the routing kernel; x [..., K] bf16 -> [..., N] bf16."""
    _need(x, "x", (torch.bfloat16,), None)
    dev = x.device
    _need(w, "w", _U32, dev)
    _need(scales, "scales", (torch.bfloat16,), dev)
    if biases is not None:
        _need(biases, "biases", (torch.bfloat16,), dev)
    K = x.shape[-1]
    if w.dim() != 2 or w.shape[1] * 32 // bits != K:
        raise ValueError(f"w of shape {tuple(w.shape)} does not match K={K} at {bits} bits")
    N = w.shape[0]
    if scales.shape != (N, K // group_size) or (biases is not None and biases.shape != scales.shape):
        raise ValueError("scales / biases shape mismatch")
    out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=dev)
    h = handle or default_handle(dev.index)
    h.bind_stream()
    h.check(h.lib.fm_linear(h.h, _ptr(x), x.numel() // K, K, _ptr(w), _ptr(scales), _ptr(biases), N, group_size,
                            bits, _ptr(out)))
    return out


def gather_qmm(x, w, scales, biases=None, lhs_indices=None, rhs_indices=None, transpose=True, group_size=64,
               bits=4, sorted_indices=False, handle=None):
    """mx::gather_qmm: out[i] = x[lhs(i)] @ dequant(w[rhs[i]])^T, shape batch(idx) + [M, N]."""
    if not transpose:
        raise NotImplementedError("transpose=False is not implemented")
    _need(x, "x", (torch.bfloat16,), None)
    dev = x.device
    _need(w, "w", _U32, dev)
    _need(scales, "scales", (torch.bfloat16,), dev)
    if biases is not None:
        _need(biases, "biases", (torch.bfloat16,), dev)
    if x.dim() < 2 or w.dim() != 3:
        raise ValueError("x must be [..., M, K] and w [E, N, K*bits/32]")
    M, K = x.shape[-2], x.shape[-1]
    E, N = w.shape[0], w.shape[1]
    if w.shape[2] * 32 // bits != K:
        raise ValueError("w does not match K")
    if rhs_indices is None:
        raise ValueError("rhs_indices is required")
    _need(rhs_indices, "rhs_indices", _U32, dev)
    x_batch = tuple(x.shape[:-2])
    xb = 1
    for d in x_batch:
        xb *= d
    if lhs_indices is not None:
        _need(lhs_indices, "lhs_indices", _U32, dev)
        if lhs_indices.shape != rhs_indices.shape:
            raise ValueError("lhs_indices and rhs_indices must have the same shape")
        out_batch = tuple(rhs_indices.shape)
    else:
        out_batch = tuple(torch.broadcast_shapes(x_batch, tuple(rhs_indices.shape)))
        if tuple(rhs_indices.shape) != out_batch:
            raise NotImplementedError("rhs_indices must carry the full broadcast batch shape")
        # x batch index i*xb/B is exact for x batch shapes that broadcast as a prefix
        B = rhs_indices.numel()
        if B % xb:
            raise NotImplementedError("x batch does not broadcast as a prefix of the index batch")
    B = rhs_indices.numel()
    out = torch.empty(*out_batch, M, N, dtype=torch.bfloat16, device=dev)
    h = handle or default_handle(dev.index)
    h.bind_stream()
    h.check(h.lib.fm_gather_qmm(h.h, _ptr(x), xb, M, K, _ptr(w), _ptr(scales), _ptr(biases), E, N,
                                _ptr(lhs_indices), _ptr(rhs_indices), B, int(transpose), group_size, bits,
                                int(sorted_indices), _ptr(out)))
    return out


@dataclass
class MoEWeightsT:
    """Stacked MoE-layer weights as torch CUDA tensors (MoEWeights, model.h:56-72)."""
    router_w: torch.Tensor
    gate: tuple
    up: tuple
    down: tuple
    shared_gate: tuple | None = None
    shared_up: tuple | None = None
    shared_down: tuple | None = None
    shared_expert_gate_w: torch.Tensor | None = None
    router_bias: torch.Tensor | None = None

    @staticmethod
    def from_numpy(d: dict, device) -> "MoEWeightsT":
        def bf(a):
            return bf16_from_numpy(a, device)

        def q(t):
            w, s, b = t
            return (u32_from_numpy(w, device), bf(s), bf(b) if b is not None else None)

        return MoEWeightsT(
            router_w=bf(d["router_w"]), gate=q(d["gate"]), up=q(d["up"]), down=q(d["down"]),
            shared_gate=q(d["shared_gate"]) if "shared_gate" in d else None,
            shared_up=q(d["shared_up"]) if "shared_up" in d else None,
            shared_down=q(d["shared_down"]) if "shared_down" in d else None,
            shared_expert_gate_w=bf(d["shared_expert_gate_w"]) if "shared_expert_gate_w" in d else None,
            router_bias=bf(d["router_bias"]) if "router_bias" in d else None)


def _qw(t):
    if t is None:
        return QWeight(None, None, None)
    w, s, b = t
    return QWeight(w.data_ptr(), s.data_ptr(), b.data_ptr() if b is not None else None)


class MoEBlock:
    """LlamaModel::moe_block on libflashmoe.  cfg: synthetic.MoEShape-like object."""

    def __init__(self, shape, weights: MoEWeightsT, handle: Handle | None = None):
        self.shape = shape
        self.weights = weights
        self.handle = handle
        c = MoEConfig()
        c.hidden, c.inter, c.num_experts, c.top_k = shape.hidden, shape.inter, shape.num_experts, shape.top_k
        c.group_size, c.bits = shape.group_size, shape.bits
        c.norm_topk_prob = int(shape.norm_topk_prob)
        c.shared_inter = shape.shared_inter
        c.router_quantized = 0
        c.shared_gate_quantized = 0
        self.cfg = c
        W = MoEWeights()
        W.router_w = weights.router_w.data_ptr()
        W.gate, W.up, W.down = _qw(weights.gate), _qw(weights.up), _qw(weights.down)
        W.shared_gate, W.shared_up, W.shared_down = (_qw(weights.shared_gate), _qw(weights.shared_up),
                                                     _qw(weights.shared_down))
        if weights.shared_expert_gate_w is not None:
            W.shared_expert_gate_w = weights.shared_expert_gate_w.data_ptr()
        if weights.router_bias is not None:
            W.router_bias = weights.router_bias.data_ptr()
        self.W = W

    def _h(self, device):
        return self.handle or default_handle(device.index)

    def reserve(self, max_tokens: int, device=None):
        h = self._h(device or self.weights.router_w.device)
        h.check(h.lib.fm_reserve(h.h, C.byref(self.cfg), max_tokens))

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None, return_routing: bool = False):
        _need(x, "x", (torch.bfloat16,), self.weights.router_w.device)
        if x.shape[-1] != self.shape.hidden:
            raise ValueError("x last dim must equal hidden size")
        T = x.numel() // self.shape.hidden
        y = out if out is not None else torch.empty_like(x)
        outs = MoEOutputs()
        routing = None
        if return_routing:
            k, E = self.shape.top_k, self.shape.num_experts
            routing = {
                "topk_ids": torch.empty(T, k, dtype=torch.int32, device=x.device),
                "topk_scores": torch.empty(T, k, dtype=torch.bfloat16, device=x.device),
                "sorted_token": torch.empty(T * k, dtype=torch.int32, device=x.device),
                "expert_offsets": torch.empty(E + 1, dtype=torch.int32, device=x.device),
            }
            for n, t in routing.items():
                setattr(outs, n, t.data_ptr())
        h = self._h(x.device)
        h.bind_stream()
        h.check(h.lib.fm_moe_block(h.h, C.byref(self.cfg), C.byref(self.W), _ptr(x), T, _ptr(y), C.byref(outs)))
        return (y, routing) if return_routing else y
class MoEBlockVariant:
    """fm_moe_block_variant: the MoE block with another routing / expert form, e.g.
    NemotronHModel::moe_block (server/src/nemotron_h.cpp:1010-1106): sigmoid routing with
    an e_score_correction_bias and group-limited top-k, fp32 scores times
    routed_scaling_factor, ungated relu^2 experts (fc1 as weights.up, fc2 as weights.down)
    and an ungated shared expert (shared_up, shared_down).  Runs the GEMV expert path."""

    def __init__(self, shape, weights: MoEWeightsT, score_func: int = _lib.FM_SCORE_SIGMOID,
                 expert_act: int = _lib.FM_ACT_RELU2, shared_ungated: bool = True, n_group: int = 1,
                 topk_group: int = 1, routed_scaling_factor: float = 1.0,
                 correction_bias: torch.Tensor | None = None, handle: Handle | None = None):
        self.block = MoEBlock(shape, weights, handle)
        self.shape = shape
        if correction_bias is not None:
            _need(correction_bias, "correction_bias", (torch.float32,), weights.router_w.device)
        self.correction_bias = correction_bias
        v = _lib.MoEVariant()
        v.score_func, v.expert_act, v.shared_ungated = score_func, expert_act, int(shared_ungated)
        v.n_group, v.topk_group, v.routed_scaling_factor = n_group, topk_group, routed_scaling_factor
        v.correction_bias = correction_bias.data_ptr() if correction_bias is not None else None
        self.variant = v

    @staticmethod
    def sigmoid_from_numpy(shape, layer: dict, device, n_group: int = 1, topk_group: int = 1,
                           routed_scaling_factor: float = 1.0, handle: Handle | None = None) -> "MoEBlockVariant":
        """The Nemotron-H form from a synthetic.make_sigmoid_layer-style dict."""
        import numpy as np

        def q(t):
            w, sc, b = t
            return (u32_from_numpy(w, device), bf16_from_numpy(sc, device),
                    bf16_from_numpy(b, device) if b is not None else None)
        W = MoEWeightsT(router_w=bf16_from_numpy(layer["router_w"], device), gate=None, up=q(layer["fc1"]),
                        down=q(layer["fc2"]),
                        shared_up=q(layer["shared_up"]) if "shared_up" in layer else None,
                        shared_down=q(layer["shared_down"]) if "shared_down" in layer else None)
        cb = layer.get("correction_bias")
        cbt = torch.from_numpy(np.ascontiguousarray(cb, np.float32)).to(device) if cb is not None else None
        return MoEBlockVariant(shape, W, n_group=n_group, topk_group=topk_group,
                               routed_scaling_factor=routed_scaling_factor, correction_bias=cbt, handle=handle)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None, return_routing: bool = False):
        w = self.block.weights
        _need(x, "x", (torch.bfloat16,), w.router_w.device)
        if x.shape[-1] != self.shape.hidden:
            raise ValueError("x last dim must equal hidden size")
        T = x.numel() // self.shape.hidden
        y = out if out is not None else torch.empty_like(x)
        outs = MoEOutputs()
        routing = None
        self.variant.topk_scores_f32 = None
        if return_routing:
            k = self.shape.top_k
            routing = {"topk_ids": torch.empty(T, k, dtype=torch.int32, device=x.device),
                       "topk_scores_f32": torch.empty(T, k, dtype=torch.float32, device=x.device)}
            outs.topk_ids = routing["topk_ids"].data_ptr()
            self.variant.topk_scores_f32 = routing["topk_scores_f32"].data_ptr()
        h = self.block._h(x.device)
        h.bind_stream()
        h.check(h.lib.fm_moe_block_variant(h.h, C.byref(self.block.cfg), C.byref(self.variant), C.byref(self.block.W),
                                           _ptr(x), T, _ptr(y), C.byref(outs)))
        return (y, routing) if return_routing else y




# ---------------------------------------------------------------- decoder ops
# The rest of the reference's decoder layer (model.cpp:486-656, sampling.cpp:5-7) on the
# same handle and stream as the MoE calls.

def dequantize(w, scales, biases=None, group_size=64, bits=4, handle=None) -> torch.Tensor:
    """mx::dequantize: [N, K*bits/32] codes -> [N, K] bf16 (bf16(fma(s, q, b)))."""
    _need(w, "w", _U32, None)
    dev = w.device
    _need(scales, "scales", (torch.bfloat16,), dev)
    if biases is not None:
        _need(biases, "biases", (torch.bfloat16,), dev)
    N, K = w.shape[0], w.shape[1] * 32 // bits
    if scales.shape != (N, K // group_size) or (biases is not None and biases.shape != scales.shape):
        raise ValueError("scales / biases shape mismatch")
    out = torch.empty(N, K, dtype=torch.bfloat16, device=dev)
    h = handle or default_handle(dev.index)
    h.bind_stream()
    h.check(h.lib.fm_dequantize(h.h, _ptr(w), _ptr(scales), _ptr(biases), N, K, group_size, bits, _ptr(out)))
    return out


def embed(table, ids, handle=None) -> torch.Tensor:
    """mx::take(table, ids, 0): table [V, H] bf16, ids int32 [...] -> [..., H]."""
    _need(table, "table", (torch.bfloat16,), None)
    dev = table.device
    _need(ids, "ids", (torch.int32,), dev)
    V, H = table.shape
    out = torch.empty(*ids.shape, H, dtype=torch.bfloat16, device=dev)
    h = handle or default_handle(dev.index)
    h.bind_stream()
    h.check(h.lib.fm_embed(h.h, _ptr(table), V, H, _ptr(ids), ids.numel(), _ptr(out)))
    return out


def rms_norm(x, weight, eps, residual=None, h_out=None, handle=None) -> torch.Tensor:
    """mx::fast::rms_norm(x + residual, weight, eps) over the last axis; x + residual (bf16)
    is also written to h_out when given (it may be x)."""
    _need(x, "x", (torch.bfloat16,), None)
    dev = x.device
    _need(weight, "weight", (torch.bfloat16,), dev)
    H = x.shape[-1]
    if weight.numel() != H:
        raise ValueError("weight size differs from the last axis")
    for t, n in ((residual, "residual"), (h_out, "h_out")):
        if t is not None:
            _need(t, n, (torch.bfloat16,), dev)
            if t.shape != x.shape:
                raise ValueError(f"{n} shape differs from x")
    y = torch.empty_like(x)
    h = handle or default_handle(dev.index)
    h.bind_stream()
    h.check(h.lib.fm_rms_norm(h.h, _ptr(x), _ptr(residual), _ptr(weight), x.numel() // H, H, float(eps),
                              _ptr(h_out), _ptr(y)))
    return y


def attention(q, k, v, cache_k, cache_v, B, L, offset, rope_theta, q_bias=None, k_bias=None, v_bias=None,
              scale=0.0, q_norm=None, k_norm=None, norm_eps=1e-6, handle=None) -> torch.Tensor:
    """The attention step after the q/k/v projections (model.cpp:560-635): bias adds, the
    optional per-head q / k RMSNorm (QK-norm weights [d]), RoPE at offset + l, k / v into
    the caches [B, n_kv, max_len, d] at [offset, offset+L), causal SDPA.  q [B*L, nh*d] is
    rotated in place; returns [B*L, nh*d] bf16."""
    _need(q, "q", (torch.bfloat16,), None)
    dev = q.device
    for t, n in ((k, "k"), (v, "v"), (cache_k, "cache_k"), (cache_v, "cache_v")):
        _need(t, n, (torch.bfloat16,), dev)
    for t, n in ((q_bias, "q_bias"), (k_bias, "k_bias"), (v_bias, "v_bias"), (q_norm, "q_norm"), (k_norm, "k_norm")):
        if t is not None:
            _need(t, n, (torch.bfloat16,), dev)
    if cache_k.dim() != 4 or cache_v.shape != cache_k.shape or cache_k.shape[0] < B:
        raise ValueError("caches must be [>= B, n_kv, max_len, d] and alike")
    _, nkv, max_len, d = cache_k.shape
    nh = q.shape[-1] // d
    if q.numel() != B * L * nh * d or k.numel() != B * L * nkv * d or v.numel() != k.numel():
        raise ValueError("q / k / v sizes do not match B, L and the cache heads")
    cfg = _lib.AttnConfig(nh, nkv, d, max_len, float(rope_theta), float(scale), float(norm_eps))
    out = torch.empty(B * L, nh * d, dtype=torch.bfloat16, device=dev)
    h = handle or default_handle(dev.index)
    h.bind_stream()
    h.check(h.lib.fm_attention(h.h, C.byref(cfg), _ptr(q), _ptr(k), _ptr(v), _ptr(q_bias), _ptr(k_bias),
                               _ptr(v_bias), _ptr(q_norm), _ptr(k_norm), _ptr(cache_k), _ptr(cache_v), B, L, offset,
                               _ptr(out)))
    return out


def attention_qkv(qkv, cache_k, cache_v, B, L, offset, rope_theta, q_bias=None, k_bias=None, v_bias=None,
                  scale=0.0, q_norm=None, k_norm=None, norm_eps=1e-6, handle=None) -> torch.Tensor:
    """attention() on the output of a fused q|k|v projection: qkv [B*L, (nh + 2 n_kv) * d]
    holds q, k and v side by side in each row (fm_attn_config.qkv_ld); its q columns are
    rotated in place.  Returns [B*L, nh*d] bf16."""
    _need(qkv, "qkv", (torch.bfloat16,), None)
    dev = qkv.device
    for t, n in ((cache_k, "cache_k"), (cache_v, "cache_v")):
        _need(t, n, (torch.bfloat16,), dev)
    for t, n in ((q_bias, "q_bias"), (k_bias, "k_bias"), (v_bias, "v_bias"), (q_norm, "q_norm"), (k_norm, "k_norm")):
        if t is not None:
            _need(t, n, (torch.bfloat16,), dev)
    if cache_k.dim() != 4 or cache_v.shape != cache_k.shape or cache_k.shape[0] < B:
        raise ValueError("caches must be [>= B, n_kv, max_len, d] and alike")
    _, nkv, max_len, d = cache_k.shape
    W = qkv.shape[-1]
    nh = W // d - 2 * nkv
    if qkv.numel() != B * L * W or W % d or nh <= 0:
        raise ValueError("qkv must be [B*L, (n_heads + 2 n_kv) * d]")
    cfg = _lib.AttnConfig(nh, nkv, d, max_len, float(rope_theta), float(scale), float(norm_eps), W)
    out = torch.empty(B * L, nh * d, dtype=torch.bfloat16, device=dev)
    h = handle or default_handle(dev.index)
    h.bind_stream()
    base = qkv.data_ptr()
    h.check(h.lib.fm_attention(h.h, C.byref(cfg), C.c_void_p(base), C.c_void_p(base + 2 * nh * d),
                               C.c_void_p(base + 2 * (nh + nkv) * d), _ptr(q_bias), _ptr(k_bias), _ptr(v_bias),
                               _ptr(q_norm), _ptr(k_norm), _ptr(cache_k), _ptr(cache_v), B, L, offset, _ptr(out)))
    return out


def swiglu(gate, up, handle=None) -> torch.Tensor:
    """The compiled swiglu of model.cpp:14-25 (silu(g) * u, bf16 after every op)."""
    _need(gate, "gate", (torch.bfloat16,), None)
    _need(up, "up", (torch.bfloat16,), gate.device)
    if up.shape != gate.shape:
        raise ValueError("gate and up shapes differ")
    out = torch.empty_like(gate)
    h = handle or default_handle(gate.device.index)
    h.bind_stream()
    h.check(h.lib.fm_swiglu(h.h, _ptr(gate), _ptr(up), gate.numel(), _ptr(out)))
    return out


def argmax(logits, handle=None) -> torch.Tensor:
    """Greedy sampling: the first index of the largest value along the last axis (int32)."""
    _need(logits, "logits", (torch.bfloat16,), None)
    V = logits.shape[-1]
    out = torch.empty(logits.shape[:-1], dtype=torch.int32, device=logits.device)
    h = handle or default_handle(logits.device.index)
    h.bind_stream()
    h.check(h.lib.fm_argmax(h.h, _ptr(logits), logits.numel() // V, V, _ptr(out)))
    return out
