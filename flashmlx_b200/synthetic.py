"""Seeded synthetic MoE-layer workloads in MLX's on-device layout.

The benchmark configurations are synthetic: there is no checkpoint and no dataset.
Every tensor is drawn from its own sub-stream, keyed by (seed, tensor name), so that
the GPU path, the CPU oracle and the CPU baseline see bit-identical inputs.

Layout (model.h:56-72, model.cpp:397-423):
  expert weights  [E, N, K/8] uint32 (8 nibbles per word, element j at bits 4*(j%8))
  scales / biases [E, N, K/64] bf16   (biases = -8 * scale, exact in bf16)
  router          [E, H] bf16
  shared expert   [Is, H/8], [H, Is/8] uint32 + [.., K/64] bf16
  shared gate     [1, H] bf16
bf16 tensors are carried as uint16 bit patterns in numpy.
"""
from __future__ import annotations

import dataclasses
import zlib

import numpy as np

__all__ = [
    "MoEShape", "CONFIGS", "f32_to_bf16", "bf16_to_f32", "make_layer", "make_x",
    "make_qmatrix", "zipf_router_bias", "layer_weight_bytes", "routed_flops",
]


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (NaN stays NaN)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = (u + (0x7FFF + ((u >> 16) & 1))) >> 16
    r = np.where(nan, (u >> 16) | 0x40, r)
    return r.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclasses.dataclass(frozen=True)
class MoEShape:
    name: str
    hidden: int
    inter: int
    num_experts: int
    top_k: int
    tokens: int
    norm_topk_prob: bool = False
    shared_inter: int = 0
    zipf_s: float = 0.0          # >0: additive per-expert router-logit bias (load skew)
    group_size: int = 64
    bits: int = 4

    def with_tokens(self, t: int) -> "MoEShape":
        return dataclasses.replace(self, tokens=t)


# BASELINE.json configs.  cfg2 (the full 24-layer decoder) is not a single-layer
# workload and is not listed here.
CONFIGS = {
    "qwen15_decode": MoEShape("qwen15_decode", 2048, 1408, 60, 4, 32, False, 5632),       # configs[0]
    "qwen15_prefill": MoEShape("qwen15_prefill", 2048, 1408, 60, 4, 4096, False, 5632),   # configs[1]
    "qwen3_decode": MoEShape("qwen3_decode", 2048, 768, 128, 8, 256, True, 0),            # configs[3]
    "qwen3_prefill": MoEShape("qwen3_prefill", 2048, 768, 128, 8, 16384, True, 0),        # configs[3]
    "mixtral_prefill": MoEShape("mixtral_prefill", 4096, 14336, 8, 2, 8192, True, 0, 1.2),  # configs[4]
}


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def make_x(shape: MoEShape, seed: int, tokens: int | None = None) -> np.ndarray:
    t = shape.tokens if tokens is None else tokens
    return f32_to_bf16(_rng(seed, "x").standard_normal((t, shape.hidden), dtype=np.float32))


def make_qmatrix(seed: int, name: str, lead: tuple, n: int, k: int, group_size: int = 64,
                 bits: int = 4, scale_std: float = 0.02):
    """Codes uniform over 0..2^bits-1, scales |N(0, scale_std)|, biases = -2^(bits-1)*scale."""
    pf = 32 // bits
    rng = _rng(seed, name)
    w = rng.integers(0, 2**32, size=lead + (n, k // pf), dtype=np.uint32)
    s = f32_to_bf16(np.abs(rng.standard_normal(lead + (n, k // group_size), dtype=np.float32)) * scale_std)
    b = f32_to_bf16(-float(2 ** (bits - 1)) * bf16_to_f32(s))
    return w, s, b


def zipf_router_bias(seed: int, num_experts: int, s: float) -> np.ndarray:
    """bias_e = ln(r_e^-s / sum_r r^-s) over a seeded random rank permutation r (bf16)."""
    ranks = _rng(seed, "zipf_rank").permutation(num_experts) + 1
    p = ranks.astype(np.float64) ** (-s)
    return f32_to_bf16(np.log(p / p.sum()).astype(np.float32))


def make_layer(shape: MoEShape, seed: int) -> dict:
    """All weights of one MoE layer as numpy arrays (bf16 as uint16)."""
    H, I, E = shape.hidden, shape.inter, shape.num_experts
    gs, bits = shape.group_size, shape.bits
    d = {}
    d["router_w"] = f32_to_bf16(_rng(seed, "router").standard_normal((E, H), dtype=np.float32) * 0.02)
    d["gate"] = make_qmatrix(seed, "gate", (E,), I, H, gs, bits)
    d["up"] = make_qmatrix(seed, "up", (E,), I, H, gs, bits)
    d["down"] = make_qmatrix(seed, "down", (E,), H, I, gs, bits)
    if shape.shared_inter:
        Is = shape.shared_inter
        d["shared_gate"] = make_qmatrix(seed, "shared_gate", (), Is, H, gs, bits)
        d["shared_up"] = make_qmatrix(seed, "shared_up", (), Is, H, gs, bits)
        d["shared_down"] = make_qmatrix(seed, "shared_down", (), H, Is, gs, bits)
        d["shared_expert_gate_w"] = f32_to_bf16(
            _rng(seed, "shared_expert_gate").standard_normal((1, H), dtype=np.float32) * 0.02)
    if shape.zipf_s > 0:
        d["router_bias"] = zipf_router_bias(seed, E, shape.zipf_s)
    return d


# The sigmoid-routed variant (fm_moe_block_variant), shaped like Nemotron-3-Nano's MoE
# layers (hidden 2688, 128 experts, top-6, expert width 1856, shared 3712,
# routed_scaling_factor 2.5, renormalised).  Single-GPU bench workloads, not BASELINE
# configs.
VARIANT_CONFIGS = {
    "nemotron_decode": (MoEShape("nemotron_decode", 2688, 1856, 128, 6, 32, True, 3712),
                        {"n_group": 1, "topk_group": 1, "routed_scaling_factor": 2.5}),
}


def make_sigmoid_layer(shape: MoEShape, seed: int, correction_bias: bool = True) -> dict:
    """One layer of the sigmoid-routed variant (Nemotron-H / DeepSeek style): router
    [E, H] bf16, e_score_correction_bias [E] fp32, ungated experts fc1 [E, I, H] and
    fc2 [E, H, I], ungated shared expert up [Is, H] / down [H, Is] (when shared_inter)."""
    H, I, E = shape.hidden, shape.inter, shape.num_experts
    gs, bits = shape.group_size, shape.bits
    d = {"router_w": f32_to_bf16(_rng(seed, "router").standard_normal((E, H), dtype=np.float32) * 0.05)}
    if correction_bias:
        d["correction_bias"] = (_rng(seed, "correction").standard_normal(E) * 0.05).astype(np.float32)
    d["fc1"] = make_qmatrix(seed, "fc1", (E,), I, H, gs, bits)
    d["fc2"] = make_qmatrix(seed, "fc2", (E,), H, I, gs, bits)
    if shape.shared_inter:
        Is = shape.shared_inter
        d["shared_up"] = make_qmatrix(seed, "shared_up", (), Is, H, gs, bits)
        d["shared_down"] = make_qmatrix(seed, "shared_down", (), H, Is, gs, bits)
    return d


def layer_weight_bytes(shape: MoEShape) -> dict:
    """Bytes of one expert / the shared expert / the router in the packed layout."""
    H, I = shape.hidden, shape.inter
    per_w = shape.bits / 8.0                      # 4-bit: 0.5 B per weight
    per_g = 2 * 2 / shape.group_size              # bf16 scale + bias per group
    per = per_w + per_g
    expert = 3 * H * I * per
    shared = 3 * H * shape.shared_inter * per if shape.shared_inter else 0.0
    return {"expert": int(round(expert)), "shared": int(round(shared)),
            "router": shape.num_experts * H * 2, "per_weight": per}


def routed_flops(shape: MoEShape, tokens: int | None = None) -> float:
    t = shape.tokens if tokens is None else tokens
    H, I, E, k = shape.hidden, shape.inter, shape.num_experts, shape.top_k
    f = 2.0 * t * k * H * I * 3 + 2.0 * t * H * E
    if shape.shared_inter:
        f += 2.0 * t * H * shape.shared_inter * 3 + 2.0 * t * H
    return f

