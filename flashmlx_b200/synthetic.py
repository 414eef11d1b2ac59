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


@dataclasses.dataclass(frozen=True)
class DecoderShape:
    """A full decoder (LlamaModel with MoE layers): attention shape, vocabulary, norms,
    and the MoE layer shape of every layer (tokens unused)."""
    name: str
    hidden: int
    layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    rope_theta: float
    rms_eps: float
    moe: MoEShape
    attn_bias: bool = True            # q/k/v biases (Qwen2-MoE), model.cpp:560-566
    tie_word_embeddings: bool = False
    group_size: int = 64
    bits: int = 4
    dense_layers: tuple = ()          # layers with a dense SwiGLU MLP instead of an MoE block
    intermediate: int = 0             # their intermediate_size
    qk_norm: bool = False             # per-head q / k RMSNorm (Qwen3), model.cpp:573-581


# the 24-layer Qwen1.5-MoE-A2.7B-shaped decoder, every MoE block as configs[0];
# and a Qwen3-30B-A3B-shaped decoder (48 layers, 32 query / 4 KV heads of 128, QK-norm, no
# attention biases, every MoE block as configs[3]) -- not a BASELINE config
DECODER_CONFIGS = {
    "qwen15_decoder": DecoderShape("qwen15_decoder", 2048, 24, 16, 16, 128, 151936, 1e6, 1e-6,
                                   MoEShape("qwen15_moe", 2048, 1408, 60, 4, 0, False, 5632)),
    "qwen3_decoder": DecoderShape("qwen3_decoder", 2048, 48, 32, 4, 128, 151936, 1e6, 1e-6,
                                  MoEShape("qwen3_moe", 2048, 768, 128, 8, 0, True, 0),
                                  attn_bias=False, qk_norm=True),
}


def make_decoder(shape: DecoderShape, seed: int) -> dict:
    """Random-init weights of a decoder (numpy, bf16 as uint16): the 4-bit embedding
    `embed` (w, s, b) [V, H]; per layer `in_norm`, `post_norm` [H], 4-bit `q`, `k`, `v`, `o`,
    bf16 `q_bias`, `k_bias`, `v_bias`, and the MoE layer `moe` (make_layer) or, for the
    shape's dense layers, the 4-bit SwiGLU MLP `mlp` {gate, up, down}; `norm` [H] and the
    4-bit `lm_head` [V, H] unless the embeddings are tied."""
    H, nh, nkv, d = shape.hidden, shape.n_heads, shape.n_kv_heads, shape.head_dim
    gs, bits = shape.group_size, shape.bits

    def norm_w(name):  # around 1, as trained RMSNorm weights are
        return f32_to_bf16(1.0 + 0.1 * _rng(seed, name).standard_normal(H, dtype=np.float32))

    def bias(name, n):
        return f32_to_bf16(0.02 * _rng(seed, name).standard_normal(n, dtype=np.float32))

    w = {"embed": make_qmatrix(seed, "embed", (), shape.vocab, H, gs, bits, scale_std=0.1),
         "norm": norm_w("norm"), "layers": []}
    if not shape.tie_word_embeddings:
        w["lm_head"] = make_qmatrix(seed, "lm_head", (), shape.vocab, H, gs, bits)
    for li in range(shape.layers):
        p = f"layers.{li}."
        lw = {"in_norm": norm_w(p + "in_norm"), "post_norm": norm_w(p + "post_norm"),
              "q": make_qmatrix(seed, p + "q", (), nh * d, H, gs, bits),
              "k": make_qmatrix(seed, p + "k", (), nkv * d, H, gs, bits),
              "v": make_qmatrix(seed, p + "v", (), nkv * d, H, gs, bits),
              "o": make_qmatrix(seed, p + "o", (), H, nh * d, gs, bits)}
        if li in shape.dense_layers:
            I = shape.intermediate
            lw["mlp"] = {"gate": make_qmatrix(seed, p + "mlp.gate", (), I, H, gs, bits),
                         "up": make_qmatrix(seed, p + "mlp.up", (), I, H, gs, bits),
                         "down": make_qmatrix(seed, p + "mlp.down", (), H, I, gs, bits)}
        else:
            lw["moe"] = make_layer(shape.moe, seed * 1000 + li)
        if shape.attn_bias:
            lw["q_bias"], lw["k_bias"], lw["v_bias"] = bias(p + "qb", nh * d), bias(p + "kb", nkv * d), bias(
                p + "vb", nkv * d)
        if shape.qk_norm:
            lw["q_norm"] = f32_to_bf16(1.0 + 0.1 * _rng(seed, p + "qn").standard_normal(d, dtype=np.float32))
            lw["k_norm"] = f32_to_bf16(1.0 + 0.1 * _rng(seed, p + "kn").standard_normal(d, dtype=np.float32))
        w["layers"].append(lw)
    return w


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

