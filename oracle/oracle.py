"""ctypes front end of the CPU oracle (oracle/oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the CPU
baseline leg of bench.py.  The product library never imports it.

PARITY UNPINNED: MLX (the library holding the reference path's arithmetic) is not
available, and the reference ships no MoE golden vectors; see oracle.cpp's header.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "liboracle.so")
_lib = None


def build(force: bool = False) -> str:
    src = os.path.join(_HERE, "oracle.cpp")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


class QWeight(C.Structure):
    _fields_ = [("w", C.c_void_p), ("s", C.c_void_p), ("b", C.c_void_p)]


class MoEConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "hidden", "inter", "num_experts", "top_k", "group_size", "bits", "norm_topk_prob",
        "shared_inter", "router_quantized", "shared_gate_quantized")]


class MoEWeights(C.Structure):
    _fields_ = [
        ("router_w", C.c_void_p), ("router_s", C.c_void_p), ("router_b", C.c_void_p),
        ("gate", QWeight), ("up", QWeight), ("down", QWeight),
        ("shared_gate", QWeight), ("shared_up", QWeight), ("shared_down", QWeight),
        ("shared_expert_gate_w", C.c_void_p), ("shared_expert_gate_s", C.c_void_p),
        ("shared_expert_gate_b", C.c_void_p), ("router_bias", C.c_void_p),
    ]


class SigConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "hidden", "inter", "num_experts", "top_k", "group_size", "bits", "norm_topk_prob", "shared_inter",
        "n_group", "topk_group")] + [("routed_scaling_factor", C.c_float)]


class SigWeights(C.Structure):
    _fields_ = [("router_w", C.c_void_p), ("correction_bias", C.c_void_p), ("fc1", QWeight), ("fc2", QWeight),
                ("shared_up", QWeight), ("shared_down", QWeight)]


def lib():
    global _lib
    if _lib is None:
        build()  # (re)builds when the library is missing or older than oracle.cpp
        L = C.CDLL(_LIB_PATH)
        p, i, i64 = C.c_void_p, C.c_int, C.c_int64
        L.orc_quantized_matmul.argtypes = [p, i64, i, p, p, p, i, i, i, p, i]
        L.orc_gather_qmm.argtypes = [p, i64, i, i, p, p, p, i, i, p, p, i64, i, i, p, i]
        L.orc_route.argtypes = [p, i64, i, p, p, p, i, p, i, i, i, i, i, p, p, p, p, i]
        L.orc_sort_pairs.argtypes = [p, i64, i, i, p, p, p]
        L.orc_moe_block.argtypes = [C.POINTER(MoEConfig), C.POINTER(MoEWeights), p, i64, p, p, p, p, p, i]
        L.orc_set_weight_rounding.argtypes = [i]
        L.orc_route_sigmoid.argtypes = [p, i64, i, p, p, i, i, i, i, i, C.c_float, p, p, i]
        L.orc_moe_block_sigmoid.argtypes = [C.POINTER(SigConfig), C.POINTER(SigWeights), p, i64, p, p, p, p, p, i]
        L.orc_version.restype = C.c_int
        if L.orc_version() < 2:
            raise ImportError("liboracle.so is stale; rebuild it (python -m oracle.oracle or make -C oracle)")
        for f in ("orc_quantized_matmul", "orc_gather_qmm", "orc_route", "orc_sort_pairs", "orc_moe_block",
                  "orc_set_weight_rounding", "orc_route_sigmoid", "orc_moe_block_sigmoid"):
            getattr(L, f).restype = C.c_int
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dt):
    return None if a is None else np.ascontiguousarray(a, dtype=dt)


NTHREADS = os.cpu_count() or 1

EXACT, BF16_WEIGHTS = 0, 1


class weight_rounding:
    """Context manager: evaluate the oracle with exact (default) or bf16-rounded
    dequantized weights."""

    def __init__(self, mode: int):
        self.mode = mode

    def __enter__(self):
        lib().orc_set_weight_rounding(self.mode)
        return self

    def __exit__(self, *exc):
        lib().orc_set_weight_rounding(EXACT)
        return False


def quantized_matmul(x, w, s, b, group_size=64, bits=4, nthreads=None):
    """x [M, K] bf16 bits; w [N, K/pf]; s, b [N, K/gs] -> [M, N] bf16 bits."""
    x = _c(x, np.uint16); w = _c(w, np.uint32); s = _c(s, np.uint16); b = _c(b, np.uint16)
    M, K = x.shape
    N = w.shape[0]
    out = np.empty((M, N), np.uint16)
    rc = lib().orc_quantized_matmul(_p(x), M, K, _p(w), _p(s), _p(b), N, group_size, bits, _p(out),
                                    nthreads or NTHREADS)
    if rc:
        raise ValueError("orc_quantized_matmul: invalid arguments")
    return out


def gather_qmm(x, w, s, b, lhs_indices, rhs_indices, group_size=64, bits=4, nthreads=None):
    """x [xb, M, K]; w [E, N, K/pf]; rhs [B] -> out [B, M, N] (bf16 bits)."""
    x = _c(x, np.uint16); w = _c(w, np.uint32); s = _c(s, np.uint16); b = _c(b, np.uint16)
    rhs = _c(rhs_indices, np.uint32).reshape(-1)
    lhs = None if lhs_indices is None else _c(lhs_indices, np.uint32).reshape(-1)
    xb, M, K = x.shape
    E, N = w.shape[0], w.shape[1]
    B = rhs.shape[0]
    out = np.empty((B, M, N), np.uint16)
    rc = lib().orc_gather_qmm(_p(x), xb, M, K, _p(w), _p(s), _p(b), E, N, _p(lhs), _p(rhs), B,
                              group_size, bits, _p(out), nthreads or NTHREADS)
    if rc:
        raise ValueError("orc_gather_qmm: invalid arguments")
    return out


def route(x, router_w, top_k, norm_topk=False, router_s=None, router_b=None, router_bias=None,
          group_size=64, bits=4, nthreads=None):
    """Returns ids [T, k] int32, scores [T, k] bf16, logits [T, E] bf16, probs [T, E] bf16."""
    x = _c(x, np.uint16)
    T, H = x.shape
    quant = router_s is not None
    rw = _c(router_w, np.uint32 if quant else np.uint16)
    rs = _c(router_s, np.uint16); rb = _c(router_b, np.uint16); bias = _c(router_bias, np.uint16)
    E = rw.shape[0]
    ids = np.empty((T, top_k), np.int32)
    sc = np.empty((T, top_k), np.uint16)
    lg = np.empty((T, E), np.uint16)
    pr = np.empty((T, E), np.uint16)
    rc = lib().orc_route(_p(x), T, H, _p(rw), _p(rs), _p(rb), int(quant), _p(bias), E, top_k,
                         int(norm_topk), group_size, bits, _p(ids), _p(sc), _p(lg), _p(pr),
                         nthreads or NTHREADS)
    if rc:
        raise ValueError("orc_route: invalid arguments")
    return ids, sc, lg, pr


def sort_pairs(ids, num_experts):
    ids = _c(ids, np.int32)
    T, k = ids.shape
    st = np.empty(T * k, np.int32); sf = np.empty(T * k, np.int32); off = np.empty(num_experts + 1, np.int32)
    if lib().orc_sort_pairs(_p(ids), T, k, num_experts, _p(st), _p(sf), _p(off)):
        raise ValueError("orc_sort_pairs: expert id out of range")
    return st, sf, off


class Layer:
    """Keeps the numpy arrays of one MoE layer alive and exposes ctypes structs."""

    def __init__(self, shape, weights: dict):
        self.shape = shape
        self.arrays = []
        w = weights
        cfg = MoEConfig()
        cfg.hidden, cfg.inter, cfg.num_experts, cfg.top_k = shape.hidden, shape.inter, shape.num_experts, shape.top_k
        cfg.group_size, cfg.bits = shape.group_size, shape.bits
        cfg.norm_topk_prob = int(shape.norm_topk_prob)
        cfg.shared_inter = shape.shared_inter
        cfg.router_quantized = 0
        cfg.shared_gate_quantized = 0
        self.cfg = cfg
        W = MoEWeights()
        W.router_w = self._keep(w["router_w"], np.uint16)
        for name in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down"):
            if name in w:
                qw, qs, qb = w[name]
                setattr(W, name, QWeight(self._keep(qw, np.uint32), self._keep(qs, np.uint16),
                                         self._keep(qb, np.uint16)))
        if "shared_expert_gate_w" in w:
            W.shared_expert_gate_w = self._keep(w["shared_expert_gate_w"], np.uint16)
        if "router_bias" in w:
            W.router_bias = self._keep(w["router_bias"], np.uint16)
        self.weights = W

    def _keep(self, a, dt):
        a = np.ascontiguousarray(a, dtype=dt)
        self.arrays.append(a)
        return a.ctypes.data

    def moe_block(self, x, forced_ids=None, forced_scores=None, nthreads=None):
        """y [T, H] bf16 bits, ids [T, k], scores [T, k] (bf16 bits)."""
        x = _c(x, np.uint16)
        T = x.shape[0]
        k = self.shape.top_k
        y = np.empty_like(x)
        ids = np.empty((T, k), np.int32)
        sc = np.empty((T, k), np.uint16)
        fi = _c(forced_ids, np.int32)
        fs = _c(forced_scores, np.uint16)
        rc = lib().orc_moe_block(C.byref(self.cfg), C.byref(self.weights), _p(x), T, _p(fi), _p(fs),
                                 _p(y), _p(ids), _p(sc), nthreads or NTHREADS)
        if rc:
            raise ValueError("orc_moe_block: invalid arguments")
        return y, ids, sc


class SigmoidLayer:
    """One layer of the sigmoid-routed variant (Nemotron-H / DeepSeek style, see
    oracle.cpp): `shape` is a synthetic.MoEShape (inter = the experts' fc1 rows,
    shared_inter = the ungated shared expert's up rows, norm_topk_prob), `routing` a dict
    with n_group, topk_group, routed_scaling_factor; weights: router_w [E, H] bf16,
    correction_bias [E] fp32 (optional), fc1 / fc2 / shared_up / shared_down as
    (w, s, b) tuples."""

    def __init__(self, shape, weights: dict, routing: dict):
        self.shape = shape
        self.arrays = []
        cfg = SigConfig()
        cfg.hidden, cfg.inter, cfg.num_experts, cfg.top_k = shape.hidden, shape.inter, shape.num_experts, shape.top_k
        cfg.group_size, cfg.bits = shape.group_size, shape.bits
        cfg.norm_topk_prob = int(shape.norm_topk_prob)
        cfg.shared_inter = shape.shared_inter
        cfg.n_group = int(routing.get("n_group", 1))
        cfg.topk_group = int(routing.get("topk_group", 1))
        cfg.routed_scaling_factor = float(routing.get("routed_scaling_factor", 1.0))
        self.cfg = cfg
        W = SigWeights()
        W.router_w = self._keep(weights["router_w"], np.uint16)
        if weights.get("correction_bias") is not None:
            W.correction_bias = self._keep(weights["correction_bias"], np.float32)
        for name in ("fc1", "fc2", "shared_up", "shared_down"):
            if name in weights:
                qw, qs, qb = weights[name]
                setattr(W, name, QWeight(self._keep(qw, np.uint32), self._keep(qs, np.uint16),
                                         None if qb is None else self._keep(qb, np.uint16)))
        self.weights = W

    def _keep(self, a, dt):
        a = np.ascontiguousarray(a, dtype=dt)
        self.arrays.append(a)
        return a.ctypes.data

    def route(self, x, nthreads=None):
        """ids [T, k] in selection order, scores [T, k] fp32."""
        x = _c(x, np.uint16)
        T, k = x.shape[0], self.shape.top_k
        ids = np.empty((T, k), np.int32)
        sc = np.empty((T, k), np.float32)
        c, W = self.cfg, self.weights
        rc = lib().orc_route_sigmoid(_p(x), T, c.hidden, W.router_w, W.correction_bias, c.num_experts, k,
                                     c.n_group, c.topk_group, c.norm_topk_prob, c.routed_scaling_factor,
                                     _p(ids), _p(sc), nthreads or NTHREADS)
        if rc:
            raise ValueError("orc_route_sigmoid: invalid arguments")
        return ids, sc

    def moe_block(self, x, forced_ids=None, forced_scores=None, nthreads=None):
        """y [T, H] bf16 bits, ids [T, k], scores [T, k] fp32."""
        x = _c(x, np.uint16)
        T, k = x.shape[0], self.shape.top_k
        y = np.empty_like(x)
        ids = np.empty((T, k), np.int32)
        sc = np.empty((T, k), np.float32)
        rc = lib().orc_moe_block_sigmoid(C.byref(self.cfg), C.byref(self.weights), _p(x), T,
                                         _p(_c(forced_ids, np.int32)), _p(_c(forced_scores, np.float32)),
                                         _p(y), _p(ids), _p(sc), nthreads or NTHREADS)
        if rc:
            raise ValueError("orc_moe_block_sigmoid: invalid arguments")
        return y, ids, sc
