"""ctypes binding of libflashmoe's C ABI (include/flashmoe.h).

This module is the reference-side binding a Python caller would write; a C++ caller
includes include/flashmoe.h and links lib/libflashmoe.so directly.  Importing it fails
loudly when the library has not been built: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libflashmoe.so")

FM_OK, FM_EINVAL, FM_EUNSUPPORTED, FM_ECUDA, FM_ENCCL, FM_ETIMEOUT, FM_EDEVICE, FM_ENOMEM, FM_ETOOLARGE = range(9)
FM_PATH_AUTO, FM_PATH_GEMV, FM_PATH_TCGEN05 = 0, 1, 2
FM_ROUTE_AUTO, FM_ROUTE_GRID, FM_ROUTE_LAST_BLOCK, FM_ROUTE_CLUSTER = 0, 1, 2, 3

# every function include/flashmoe.h declares: name -> (restype, argtypes)
_p, _i, _i64, _sz, _s = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_char_p


class QWeight(C.Structure):
    _fields_ = [("w", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p)]


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


class MoEOutputs(C.Structure):
    _fields_ = [("topk_ids", C.c_void_p), ("topk_scores", C.c_void_p), ("sorted_token", C.c_void_p),
                ("expert_offsets", C.c_void_p)]


class MoEVariant(C.Structure):
    _fields_ = [("score_func", C.c_int), ("n_group", C.c_int), ("topk_group", C.c_int),
                ("routed_scaling_factor", C.c_float), ("expert_act", C.c_int), ("shared_ungated", C.c_int),
                ("correction_bias", C.c_void_p), ("topk_scores_f32", C.c_void_p)]


FM_SCORE_SOFTMAX, FM_SCORE_SIGMOID = 0, 1
FM_ACT_SWIGLU, FM_ACT_RELU2 = 0, 1


class AttnConfig(C.Structure):
    _fields_ = [("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("max_len", C.c_int),
                ("rope_theta", C.c_float), ("scale", C.c_float), ("norm_eps", C.c_float), ("qkv_ld", C.c_int)]


class KernelTime(C.Structure):
    _fields_ = [("name", C.c_char_p), ("launches", C.c_int64), ("total_ms", C.c_double)]


SIGNATURES = {
    "fm_create": (_i, [C.POINTER(C.c_void_p), _i, _p]),
    "fm_destroy": (_i, [_p]),
    "fm_set_stream": (_i, [_p, _p]),
    "fm_last_error": (_s, [_p]),
    "fm_status_string": (_s, [_i]),
    "fm_sync_status": (_i, [_p]),
    "fm_reserve": (_i, [_p, C.POINTER(MoEConfig), _i64]),
    "fm_workspace_bytes": (_sz, [_p]),
    "fm_workspace_size": (_sz, [C.POINTER(MoEConfig), _i64]),
    "fm_set_path": (_i, [_p, _i]),
    "fm_last_path": (_i, [_p]),
    "fm_set_route_mode": (_i, [_p, _i]),
    "fm_profile_enable": (_i, [_p, _i]),
    "fm_profile_report": (_i, [_p, C.POINTER(KernelTime), _i, C.POINTER(C.c_int), _i]),
    "fm_quantized_matmul": (_i, [_p, _p, _i64, _i, _p, _p, _p, _i, _i, _i, _i, _p]),
    "fm_linear": (_i, [_p, _p, _i64, _i, _p, _p, _p, _i, _i, _i, _p]),
    "fm_gather_qmm": (_i, [_p, _p, _i64, _i, _i, _p, _p, _p, _i, _i, _p, _p, _i64, _i, _i, _i, _i, _p]),
    "fm_moe_block": (_i, [_p, C.POINTER(MoEConfig), C.POINTER(MoEWeights), _p, _i64, _p,
                          C.POINTER(MoEOutputs)]),
    "fm_moe_block_noalloc": (_i, [_i, _p, C.POINTER(MoEConfig), C.POINTER(MoEWeights), _p, _i64, _p]),
    "fm_moe_block_variant": (_i, [_p, C.POINTER(MoEConfig), C.POINTER(MoEVariant), C.POINTER(MoEWeights), _p, _i64,
                                  _p, C.POINTER(MoEOutputs)]),
    "fm_ep_range": (_i, [_i, _i, _i, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "fm_ep_set": (_i, [_p, _i, _i]),
    "fm_ep_dispatch": (_i, [_p, C.POINTER(MoEConfig), C.POINTER(MoEWeights), _p, _i64, C.POINTER(C.c_int32),
                            C.POINTER(C.c_void_p)]),
    "fm_ep_experts": (_i, [_p, C.POINTER(MoEConfig), C.POINTER(MoEWeights), _p, C.POINTER(C.c_int32), _p]),
    "fm_ep_combine": (_i, [_p, C.POINTER(MoEConfig), _p, _p]),
    "fm_ep_p2p_alloc": (_i, [_p, C.POINTER(MoEConfig), _i64, _p]),
    "fm_ep_p2p_open": (_i, [_p, _p]),
    "fm_ep_p2p_forward": (_i, [_p, C.POINTER(MoEConfig), C.POINTER(MoEWeights), _p, _i64, _p]),
    "fm_ep_p2p_close": (_i, [_p]),
    "fm_dequantize": (_i, [_p, _p, _p, _p, _i64, _i, _i, _i, _p]),
    "fm_embed": (_i, [_p, _p, _i64, _i, _p, _i64, _p]),
    "fm_rms_norm": (_i, [_p, _p, _p, _p, _i64, _i, C.c_float, _p, _p]),
    "fm_attention": (_i, [_p, C.POINTER(AttnConfig), _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _p]),
    "fm_swiglu": (_i, [_p, _p, _p, _i64, _p]),
    "fm_argmax": (_i, [_p, _p, _i64, _i64, _p]),
}

_lib = None


def load() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libflashmoe is not built ({LIB_PATH} missing); run `python -m flashmlx_b200.build`")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class FlashMoEError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"libflashmoe status {status}: {message}")
        self.status = status
