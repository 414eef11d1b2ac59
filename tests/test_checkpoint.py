"""MLX-format checkpoint loading (flashmlx_b200.checkpoint): the safetensors reader and
writer, config.json with the reference's defaults (server/src/model.cpp:105-142), and the
per-layer expert stacking of build_moe_weight_cache (model.cpp:368-470) checked against
the arrays the checkpoint was written from."""
from __future__ import annotations

import json
import os
import struct

import numpy as np
import pytest

from flashmlx_b200 import checkpoint as CK
from flashmlx_b200 import synthetic as S

SHAPE = S.MoEShape("ckpt", 256, 128, 4, 2, 8, True, 256)


def _config(path, shape=SHAPE, layers=2, **extra):
    c = {"hidden_size": shape.hidden, "num_hidden_layers": layers, "num_experts": shape.num_experts,
         "num_experts_per_tok": shape.top_k, "moe_intermediate_size": shape.inter,
         "shared_expert_intermediate_size": shape.shared_inter, "norm_topk_prob": shape.norm_topk_prob,
         "quantization": {"group_size": shape.group_size, "bits": shape.bits}}
    c.update(extra)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(c, f)


def _layer_tensors(layer, li, stacked=False, prefix="model."):
    """The MoE tensors of one layer under the checkpoint's key names."""
    t = {}
    mlp = f"{prefix}layers.{li}.mlp"
    t[f"{mlp}.gate.weight"] = layer["router_w"]
    for proj, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
        w, s, b = layer[key]
        if stacked:
            t[f"{mlp}.switch_mlp.{proj}.weight"], t[f"{mlp}.switch_mlp.{proj}.scales"] = w, s
            t[f"{mlp}.switch_mlp.{proj}.biases"] = b
        else:
            for e in range(w.shape[0]):
                t[f"{mlp}.experts.{e}.{proj}.weight"] = w[e]
                t[f"{mlp}.experts.{e}.{proj}.scales"] = s[e]
                t[f"{mlp}.experts.{e}.{proj}.biases"] = b[e]
    for proj, key in (("gate_proj", "shared_gate"), ("up_proj", "shared_up"), ("down_proj", "shared_down")):
        w, s, b = layer[key]
        t[f"{mlp}.shared_expert.{proj}.weight"], t[f"{mlp}.shared_expert.{proj}.scales"] = w, s
        t[f"{mlp}.shared_expert.{proj}.biases"] = b
    t[f"{mlp}.shared_expert_gate.weight"] = layer["shared_expert_gate_w"]
    return t


def _write_model(path, layer, stacked=False):
    """Layer 0 is the MoE layer, split over two shards; layer 1 is dense (no router)."""
    _config(path)
    t = _layer_tensors(layer, 0, stacked)
    names = sorted(t)
    CK.write_safetensors(os.path.join(path, "model-00001-of-00002.safetensors"),
                         {n: t[n] for n in names[: len(names) // 2]}, {"format": "mlx"})
    rest = {n: t[n] for n in names[len(names) // 2:]}
    rest["model.layers.1.mlp.gate_proj.weight"] = np.zeros((SHAPE.inter, SHAPE.hidden // 8), np.uint32)
    rest["model.embed_tokens.weight"] = ("F32", np.ones((4, 8), np.float32))
    CK.write_safetensors(os.path.join(path, "model-00002-of-00002.safetensors"), rest)


def _same(a, b):
    for key in ("router_w", "shared_expert_gate_w"):
        np.testing.assert_array_equal(a[key], b[key])
    for key in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down"):
        for x, y in zip(a[key], b[key]):
            np.testing.assert_array_equal(x, y)


def test_safetensors_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    t = {"a": rng.integers(0, 2**32, (3, 5), dtype=np.uint32), "b": rng.integers(0, 2**16, (7,), dtype=np.uint16),
         "c": ("F32", rng.standard_normal((2, 2, 2)).astype(np.float32)), "d": np.zeros((0, 4), np.int32),
         "e": ("U16", np.arange(6, dtype=np.uint16))}
    p = str(tmp_path / "t.safetensors")
    CK.write_safetensors(p, t, {"k": "v"})
    with open(p, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
    assert (8 + n) % 8 == 0  # data 8-byte aligned
    got, meta = CK.read_safetensors(p)
    assert meta == {"k": "v"}
    assert got["b"][0] == "BF16" and got["e"][0] == "U16" and got["c"][0] == "F32"
    for k, v in t.items():
        arr = v[1] if isinstance(v, tuple) else v
        np.testing.assert_array_equal(got[k][1], arr)
        assert got[k][1].dtype == arr.dtype and got[k][1].shape == arr.shape


def test_safetensors_rejects_bad_files(tmp_path):
    p = str(tmp_path / "bad.safetensors")
    with open(p, "wb") as f:
        f.write(b"\x01\x00")
    with pytest.raises(ValueError):
        CK.read_safetensors(p)
    h = json.dumps({"x": {"dtype": "U32", "shape": [4], "data_offsets": [0, 8]}}).encode()
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"\x00" * 8)
    with pytest.raises(ValueError, match="data_offsets"):
        CK.read_safetensors(p)
    h = json.dumps({"x": {"dtype": "C64", "shape": [1], "data_offsets": [0, 8]}}).encode()
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"\x00" * 8)
    with pytest.raises(ValueError, match="dtype"):
        CK.read_safetensors(p)


def test_config_defaults(tmp_path):
    with open(tmp_path / "config.json", "w") as f:
        json.dump({"hidden_size": 2048, "num_experts": 60}, f)
    c = CK.load_config(str(tmp_path))
    assert (c.hidden, c.num_layers, c.num_experts, c.top_k, c.inter, c.shared_inter) == (2048, 32, 60, 0, 0, 0)
    assert (c.norm_topk_prob, c.bits, c.group_size) == (False, 0, 64)


@pytest.mark.parametrize("stacked", [False, True])
def test_moe_layer_stacking(tmp_path, stacked):
    layer = S.make_layer(SHAPE, 3)
    _write_model(str(tmp_path), layer, stacked)
    ck = CK.Checkpoint(str(tmp_path))
    assert ck.moe_layers() == [0]
    assert ck.config.shape(8, "ckpt") == SHAPE.with_tokens(8)
    assert ck.has("embed_tokens.weight")  # the "model." prefix is stripped
    _same(ck.moe_layer(0), layer)
    with pytest.raises(KeyError):
        ck.moe_layer(1)


def test_later_shards_override(tmp_path):
    layer = S.make_layer(SHAPE, 4)
    _write_model(str(tmp_path), layer)
    other = S.f32_to_bf16(np.ones((SHAPE.num_experts, SHAPE.hidden), np.float32))
    CK.write_safetensors(str(tmp_path / "model-00003-extra.safetensors"), {"layers.0.mlp.gate.weight": other})
    np.testing.assert_array_equal(CK.Checkpoint(str(tmp_path)).moe_layer(0)["router_w"], other)


def test_moe_layer_errors(tmp_path):
    layer = S.make_layer(SHAPE, 5)
    _config(str(tmp_path))
    t = _layer_tensors(layer, 0)
    bad = dict(t)
    bad["model.layers.0.mlp.gate.scales"] = np.zeros((SHAPE.num_experts, SHAPE.hidden // 64), np.uint16)
    CK.write_safetensors(str(tmp_path / "a.safetensors"), bad)
    with pytest.raises(NotImplementedError, match="quantized router"):
        CK.Checkpoint(str(tmp_path)).moe_layer(0)
    os.remove(tmp_path / "a.safetensors")
    missing = {k: v for k, v in t.items() if ".experts.3.up_proj.weight" not in k}
    CK.write_safetensors(str(tmp_path / "a.safetensors"), missing)
    with pytest.raises(KeyError, match="experts.3.up_proj.weight"):
        CK.Checkpoint(str(tmp_path)).moe_layer(0)
    os.remove(tmp_path / "a.safetensors")
    CK.write_safetensors(str(tmp_path / "a.safetensors"), t)
    _config(str(tmp_path), moe_intermediate_size=SHAPE.inter * 2)
    with pytest.raises(ValueError, match="config gives"):
        CK.Checkpoint(str(tmp_path)).moe_layer(0)
    os.remove(tmp_path / "a.safetensors")
    with pytest.raises(FileNotFoundError):
        CK.Checkpoint(str(tmp_path))


def test_loaded_layer_through_the_oracle(tmp_path):
    """The oracle's MoE block over the loaded layer equals it over the source arrays."""
    from oracle import oracle as O
    layer = S.make_layer(SHAPE, 6)
    _write_model(str(tmp_path), layer)
    loaded = CK.Checkpoint(str(tmp_path)).moe_layer(0)
    x = S.make_x(SHAPE, 6)
    ya = O.Layer(SHAPE, layer).moe_block(x)[0]
    yb = O.Layer(SHAPE, loaded).moe_block(x)[0]
    np.testing.assert_array_equal(ya, yb)


def test_moe_model_layer_discovery(tmp_path):
    """MoEModel finds the layers with a router and rejects the others (no device work)."""
    from flashmlx_b200.model import MoEModel
    layer = S.make_layer(SHAPE, 7)
    _write_model(str(tmp_path), layer)
    m = MoEModel(str(tmp_path), device="cpu")
    assert m.is_moe(0) and not m.is_moe(1)
    assert m.shape.hidden == SHAPE.hidden and m.shape.num_experts == SHAPE.num_experts
    with pytest.raises(KeyError):
        MoEModel(str(tmp_path), device="cpu", layers=[1])


NEMO = S.MoEShape("nemo", 256, 128, 8, 2, 8, True, 256)


def _write_nemotron(path, layer):
    """A 4-layer Nemotron-H model 'ME*E' whose two MoE layers are written from `layer`."""
    c = {"hidden_size": NEMO.hidden, "num_hidden_layers": 4, "hybrid_override_pattern": "ME*E",
         "n_routed_experts": NEMO.num_experts, "num_experts_per_tok": NEMO.top_k,
         "moe_intermediate_size": NEMO.inter, "moe_shared_expert_intermediate_size": NEMO.shared_inter,
         "n_shared_experts": 1, "n_group": 2, "topk_group": 1, "routed_scaling_factor": 2.5,
         "norm_topk_prob": True, "quantization": {"group_size": 64, "bits": 4}}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(c, f)
    t = {}
    for li in (1, 3):
        mx = f"backbone.layers.{li}.mixer"
        t[f"{mx}.gate.weight"] = layer["router_w"]
        t[f"{mx}.gate.e_score_correction_bias"] = ("F32", layer["correction_bias"])
        for key, name in (("fc1", "switch_mlp.fc1"), ("fc2", "switch_mlp.fc2"),
                          ("shared_up", "shared_experts.up_proj"), ("shared_down", "shared_experts.down_proj")):
            w, s, b = layer[key]
            t[f"{mx}.{name}.weight"], t[f"{mx}.{name}.scales"], t[f"{mx}.{name}.biases"] = w, s, b
    t["backbone.layers.0.mixer.A_log"] = ("F32", np.zeros(4, np.float32))
    CK.write_safetensors(os.path.join(path, "model.safetensors"), t)


def test_nemotron_checkpoint(tmp_path):
    layer = S.make_sigmoid_layer(NEMO, 13)
    _write_nemotron(str(tmp_path), layer)
    ck = CK.Checkpoint(str(tmp_path))
    c = ck.config
    assert c.sigmoid_routed and ck.moe_layers() == [1, 3]
    assert (c.num_experts, c.shared_inter) == (NEMO.num_experts, NEMO.shared_inter)
    assert c.routing() == {"n_group": 2, "topk_group": 1, "routed_scaling_factor": 2.5}
    assert ck.has("layers.0.mixer.A_log")  # "backbone." stripped
    got = ck.sigmoid_moe_layer(3)
    np.testing.assert_array_equal(got["router_w"], layer["router_w"])
    np.testing.assert_array_equal(got["correction_bias"], layer["correction_bias"])
    for key in ("fc1", "fc2", "shared_up", "shared_down"):
        for x, y in zip(got[key], layer[key]):
            np.testing.assert_array_equal(x, y)
    with pytest.raises(KeyError):
        ck.sigmoid_moe_layer(2)


def test_nemotron_checkpoint_through_the_oracle(tmp_path):
    """The oracle's variant block over the loaded layer equals it over the source arrays."""
    from oracle import oracle as O
    layer = S.make_sigmoid_layer(NEMO, 14)
    _write_nemotron(str(tmp_path), layer)
    ck = CK.Checkpoint(str(tmp_path))
    x = S.make_x(NEMO, 14)
    ya = O.SigmoidLayer(NEMO, layer, ck.config.routing()).moe_block(x)[0]
    yb = O.SigmoidLayer(NEMO, ck.sigmoid_moe_layer(1), ck.config.routing()).moe_block(x)[0]
    np.testing.assert_array_equal(ya, yb)
