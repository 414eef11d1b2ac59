"""Helpers for the decoder tests: an MLX-format checkpoint directory written from the
weights of synthetic.make_decoder, under the key names the reference's LlamaModel loads
(model.cpp:148-184, 486-520, 542-660) and the Qwen config keys of load_config (105-142)."""
from __future__ import annotations

import json
import os

from flashmlx_b200 import checkpoint as CK
from tests.test_checkpoint import _layer_tensors


def write_decoder_checkpoint(path, shape, w, shards: int = 2) -> None:
    m = shape.moe
    cfg = {"hidden_size": shape.hidden, "num_hidden_layers": shape.layers, "num_attention_heads": shape.n_heads,
           "num_key_value_heads": shape.n_kv_heads, "head_dim": shape.head_dim, "vocab_size": shape.vocab,
           "rms_norm_eps": shape.rms_eps, "rope_theta": shape.rope_theta,
           "tie_word_embeddings": shape.tie_word_embeddings, "num_experts": m.num_experts,
           "num_experts_per_tok": m.top_k, "moe_intermediate_size": m.inter,
           "shared_expert_intermediate_size": m.shared_inter, "norm_topk_prob": m.norm_topk_prob,
           "quantization": {"group_size": shape.group_size, "bits": shape.bits},
           "intermediate_size": shape.intermediate or 14336}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    t = {}

    def q(prefix, qm):
        t[prefix + ".weight"], t[prefix + ".scales"], t[prefix + ".biases"] = qm

    q("model.embed_tokens", w["embed"])
    t["model.norm.weight"] = w["norm"]
    if "lm_head" in w:
        q("lm_head", w["lm_head"])
    for li, lw in enumerate(w["layers"]):
        p = f"model.layers.{li}"
        t[p + ".input_layernorm.weight"] = lw["in_norm"]
        t[p + ".post_attention_layernorm.weight"] = lw["post_norm"]
        for proj in ("q", "k", "v", "o"):
            q(f"{p}.self_attn.{proj}_proj", lw[proj])
        for proj in ("q", "k", "v"):
            if lw.get(proj + "_bias") is not None:
                t[f"{p}.self_attn.{proj}_proj.bias"] = lw[proj + "_bias"]
        for proj in ("q", "k"):
            if lw.get(proj + "_norm") is not None:
                t[f"{p}.self_attn.{proj}_norm.weight"] = lw[proj + "_norm"]
        if "moe" in lw:
            t.update(_layer_tensors(lw["moe"], li, stacked=True))
        else:
            for proj in ("gate", "up", "down"):
                q(f"{p}.mlp.{proj}_proj", lw["mlp"][proj])
    names = sorted(t)
    per = (len(names) + shards - 1) // shards
    for i in range(shards):
        part = {n: t[n] for n in names[i * per:(i + 1) * per]}
        CK.write_safetensors(os.path.join(path, f"model-{i + 1:05d}-of-{shards:05d}.safetensors"), part)
