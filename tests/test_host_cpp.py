"""The C++ host layer (flashmlx_b200/host: checkpoint.cpp, moe_model.cpp, driven by the
fm_host program) against the Python loader: config.json with the reference's defaults
(server/src/model.cpp:105-142), the MoE layer list, and the stacked arrays of
build_moe_weight_cache (model.cpp:368-470) / the Nemotron-H 'E' layers
(nemotron_h.cpp:444-468), bit for bit; malformed checkpoints are rejected with a message.
Runs without a GPU (the loading half); the device half is in test_gpu_host_cpp.py."""
from __future__ import annotations

import json
import os
import struct
import subprocess

import numpy as np
import pytest
import torch

from flashmlx_b200 import checkpoint as CK
from flashmlx_b200 import synthetic as S
from tests.test_checkpoint import NEMO, SHAPE, _config, _layer_tensors, _write_model, _write_nemotron


@pytest.fixture(scope="module")
def fm_host():
    from flashmlx_b200 import build as fb
    return fb.build_host()


def _run(exe, *args, check=True):
    r = subprocess.run([exe, *map(str, args)], capture_output=True, text=True, timeout=300)
    if check and r.returncode != 0:
        raise AssertionError(f"fm_host {args[0]} exited {r.returncode}: {r.stderr}")
    return r


def _inspect(exe, path):
    return json.loads(_run(exe, "inspect", path).stdout)


_DT = {"BF16": np.uint16, "U32": np.uint32, "F32": np.float32}


def _dump(exe, path, layer, out):
    os.makedirs(out, exist_ok=True)
    _run(exe, "dump", path, layer, out)
    with open(os.path.join(out, "manifest.json")) as f:
        man = json.load(f)
    arrays = {}
    for name, info in man["arrays"].items():
        a = np.fromfile(os.path.join(out, name + ".bin"), dtype=_DT[info["dtype"]])
        arrays[name] = a.reshape(info["shape"])
    return man["sigmoid"], arrays


def _same_q(arrays, name, q):
    w, s, b = q
    np.testing.assert_array_equal(arrays[name + ".w"], w)
    np.testing.assert_array_equal(arrays[name + ".s"], s)
    if b is None:
        assert name + ".b" not in arrays
    else:
        np.testing.assert_array_equal(arrays[name + ".b"], b)


@pytest.mark.parametrize("stacked", [False, True])
def test_llama_checkpoint(tmp_path, fm_host, stacked):
    layer = S.make_layer(SHAPE, 31)
    _write_model(str(tmp_path), layer, stacked=stacked)
    ck = CK.Checkpoint(str(tmp_path))
    got = _inspect(fm_host, tmp_path)
    c = ck.config
    want = {"hidden": c.hidden, "num_layers": c.num_layers, "num_experts": c.num_experts, "top_k": c.top_k,
            "inter": c.inter, "shared_inter": c.shared_inter, "norm_topk_prob": c.norm_topk_prob,
            "bits": c.bits, "group_size": c.group_size, "n_group": 1, "topk_group": 1,
            "routed_scaling_factor": 1, "sigmoid_routed": False, "moe_layers": ck.moe_layers()}
    assert {k: got[k] for k in want} == want
    # decoder keys absent from this config take LlamaModel::load_config's defaults
    assert (got["n_heads"], got["n_kv_heads"], got["vocab"], got["tie_word_embeddings"]) == (32, 8, 128256, True)
    assert got["head_dim"] == c.hidden // 32 and got["rope_theta"] == 10000 and got["rms_eps"] == pytest.approx(1e-5)
    sig, arrays = _dump(fm_host, tmp_path, 0, tmp_path / "dump")
    assert not sig
    ref = ck.moe_layer(0)
    np.testing.assert_array_equal(arrays["router_w"], ref["router_w"])
    np.testing.assert_array_equal(arrays["shared_expert_gate_w"], ref["shared_expert_gate_w"])
    for key in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down"):
        _same_q(arrays, key, ref[key])


def test_nemotron_checkpoint(tmp_path, fm_host):
    layer = S.make_sigmoid_layer(NEMO, 32)
    _write_nemotron(str(tmp_path), layer)
    got = _inspect(fm_host, tmp_path)
    assert got["sigmoid_routed"] and got["moe_layers"] == [1, 3]
    assert (got["num_experts"], got["shared_inter"], got["n_group"], got["topk_group"]) == (NEMO.num_experts,
                                                                                           NEMO.shared_inter, 2, 1)
    assert got["routed_scaling_factor"] == pytest.approx(2.5)
    sig, arrays = _dump(fm_host, tmp_path, 3, tmp_path / "dump")
    assert sig
    np.testing.assert_array_equal(arrays["router_w"], layer["router_w"])
    np.testing.assert_array_equal(arrays["correction_bias"], layer["correction_bias"])
    for key in ("fc1", "fc2", "shared_up", "shared_down"):
        _same_q(arrays, key, layer[key])


def test_nemotron_bf16_correction_bias(tmp_path, fm_host):
    """A BF16 e_score_correction_bias is widened to fp32 exactly (as the Python loader does)."""
    layer = S.make_sigmoid_layer(NEMO, 33)
    _write_nemotron(str(tmp_path), layer)
    path = os.path.join(str(tmp_path), "model.safetensors")
    t, _ = CK.read_safetensors(path)
    t = {k: (dt, np.array(a)) for k, (dt, a) in t.items()}
    bias16 = (layer["correction_bias"].view(np.uint32) >> 16).astype(np.uint16)
    for li in (1, 3):
        t[f"backbone.layers.{li}.mixer.gate.e_score_correction_bias"] = ("BF16", bias16)
    CK.write_safetensors(path, t)
    _, arrays = _dump(fm_host, tmp_path, 1, tmp_path / "dump")
    np.testing.assert_array_equal(arrays["correction_bias"], CK.Checkpoint(str(tmp_path)).sigmoid_moe_layer(1)
                                  ["correction_bias"])


def test_config_defaults(tmp_path, fm_host):
    """Absent keys take LlamaModel::load_config's defaults (hidden 4096, 32 layers, no
    quantization) -- the same as the Python loader."""
    with open(tmp_path / "config.json", "w") as f:
        json.dump({"num_experts": 4}, f)
    CK.write_safetensors(str(tmp_path / "m.safetensors"), {"x": np.zeros(2, np.uint16)})
    got = _inspect(fm_host, tmp_path)
    c = CK.load_config(str(tmp_path))
    assert (got["hidden"], got["num_layers"], got["bits"], got["group_size"]) == (c.hidden, c.num_layers, c.bits,
                                                                                  c.group_size) == (4096, 32, 0, 64)
    assert got["moe_layers"] == []


def test_later_shard_overrides(tmp_path, fm_host):
    """Keys of a later file (sorted order) replace an earlier file's (load_weights)."""
    layer = S.make_layer(SHAPE, 34)
    _write_model(str(tmp_path), layer)
    other = S.make_layer(SHAPE, 35)
    CK.write_safetensors(str(tmp_path / "model-00003-of-00003.safetensors"),
                         {"model.layers.0.mlp.gate.weight": other["router_w"]})
    _, arrays = _dump(fm_host, tmp_path, 0, tmp_path / "dump")
    np.testing.assert_array_equal(arrays["router_w"], other["router_w"])


def _expect_error(exe, path, *args, match):
    r = _run(exe, *args, path, check=False) if not args else _run(exe, args[0], path, *args[1:], check=False)
    assert r.returncode == 4, (r.returncode, r.stderr)
    assert match in r.stderr, r.stderr


def test_rejects_malformed(tmp_path, fm_host):
    layer = S.make_layer(SHAPE, 36)
    # quantized router
    d = tmp_path / "qrouter"
    d.mkdir()
    _config(str(d), layers=1)
    t = _layer_tensors(layer, 0)
    t["model.layers.0.mlp.gate.scales"] = np.zeros((SHAPE.num_experts, SHAPE.hidden // 64), np.uint16)
    CK.write_safetensors(str(d / "m.safetensors"), t)
    _expect_error(fm_host, d, "dump", 0, str(tmp_path), match="quantized router")
    # config shape mismatch
    d = tmp_path / "shape"
    d.mkdir()
    _config(str(d), layers=1, moe_intermediate_size=SHAPE.inter * 2)
    CK.write_safetensors(str(d / "m.safetensors"), _layer_tensors(layer, 0))
    _expect_error(fm_host, d, "dump", 0, str(tmp_path), match="config gives")
    # not 4-bit
    d = tmp_path / "bits"
    d.mkdir()
    _config(str(d), layers=1, quantization={"bits": 8, "group_size": 64})
    CK.write_safetensors(str(d / "m.safetensors"), _layer_tensors(layer, 0))
    _expect_error(fm_host, d, "dump", 0, str(tmp_path), match="only 4-bit")
    # shared expert in the config, none in the file
    d = tmp_path / "noshared"
    d.mkdir()
    _config(str(d), layers=1)
    t = {k: v for k, v in _layer_tensors(layer, 0).items() if "shared_expert" not in k}
    CK.write_safetensors(str(d / "m.safetensors"), t)
    _expect_error(fm_host, d, "dump", 0, str(tmp_path), match="has none")
    # a header length past the end of the file, and a header that is not JSON
    d = tmp_path / "badfile"
    d.mkdir()
    _config(str(d), layers=1)
    with open(d / "m.safetensors", "wb") as f:
        f.write(struct.pack("<Q", 1 << 20) + b"{}")
    _expect_error(fm_host, d, "inspect", match="exceeds the file")
    with open(d / "m.safetensors", "wb") as f:
        f.write(struct.pack("<Q", 5) + b"{oops")
    _expect_error(fm_host, d, "inspect", match="json")
    # data_offsets that do not hold the declared shape
    hdr = json.dumps({"w": {"dtype": "U32", "shape": [4], "data_offsets": [0, 8]}}).encode()
    with open(d / "m.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 16)
    _expect_error(fm_host, d, "inspect", match="data_offsets")


def test_nemotron_pattern_length(tmp_path, fm_host):
    layer = S.make_sigmoid_layer(NEMO, 37)
    _write_nemotron(str(tmp_path), layer)
    with open(tmp_path / "config.json") as f:
        c = json.load(f)
    c["hybrid_override_pattern"] = "ME*"
    with open(tmp_path / "config.json", "w") as f:
        json.dump(c, f)
    _expect_error(fm_host, tmp_path, "inspect", match="hybrid_override_pattern length")


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device error path")
def test_run_without_a_device_fails_loudly(tmp_path, fm_host):
    """No GPU: the run command reports the CUDA status, it does not compute on the CPU."""
    layer = S.make_layer(SHAPE, 38)
    _write_model(str(tmp_path), layer)
    S.make_x(SHAPE.with_tokens(4), 38).tofile(tmp_path / "x.bin")
    r = _run(fm_host, "run", tmp_path, 0, tmp_path / "x.bin", 4, tmp_path / "y.bin", check=False)
    assert r.returncode == 3, (r.returncode, r.stderr)
    assert r.stderr.startswith("fm_status 3"), r.stderr
    assert not os.path.exists(tmp_path / "y.bin")


# ---------------------------------------------------------------- the decoder's loader
from tests.decoder_util import write_decoder_checkpoint  # noqa: E402

DEC = S.DecoderShape("dec_ckpt", 256, 2, 4, 2, 64, 320, 1e6, 1e-6, S.MoEShape("dec_moe", 256, 128, 4, 2, 0, False, 256))


def test_decoder_checkpoint_layout(tmp_path, fm_host):
    w = S.make_decoder(DEC, 51)
    write_decoder_checkpoint(str(tmp_path), DEC, w)
    got = json.loads(_run(fm_host, "check-decoder", tmp_path).stdout)
    assert got == {"layers": 2, "moe_layers": [0, 1], "attn_bias": True, "qk_norm": False, "embed_quantized": True,
                   "tie_word_embeddings": False, "head_dim": 64, "vocab": 320}
    info = _inspect(fm_host, tmp_path)
    assert (info["n_heads"], info["n_kv_heads"], info["rope_theta"]) == (4, 2, 1e6)


def test_decoder_checkpoint_rejects_misshapen(tmp_path, fm_host):
    w = S.make_decoder(DEC, 52)
    write_decoder_checkpoint(str(tmp_path), DEC, w)
    with open(tmp_path / "config.json") as f:
        c = json.load(f)
    c["num_key_value_heads"] = 4  # k/v projections were written for 2 heads
    with open(tmp_path / "config.json", "w") as f:
        json.dump(c, f)
    _expect_error(fm_host, tmp_path, "check-decoder", match="self_attn.k_proj: shape differs")


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device error path")
def test_generate_without_a_device_fails_loudly(tmp_path, fm_host):
    w = S.make_decoder(DEC, 53)
    write_decoder_checkpoint(str(tmp_path), DEC, w)
    np.zeros((1, 4), np.int32).tofile(tmp_path / "p.bin")
    r = _run(fm_host, "generate", tmp_path, tmp_path / "p.bin", 1, 4, 3, tmp_path / "o.bin", check=False)
    assert r.returncode == 3 and r.stderr.startswith("fm_status 3"), (r.returncode, r.stderr)


def test_fmh_binding_matches_header_and_exports(fm_host):
    """Every function fmh.h declares is exported by libflashmoe_host.so and bound by
    flashmlx_b200.decoder (and nothing else is)."""
    import re
    from flashmlx_b200 import decoder as DEC
    hdr = open(os.path.join(os.path.dirname(DEC.__file__), "host", "fmh.h")).read()
    declared = set(re.findall(r"\b(fmh_\w+)\s*\(", hdr))
    assert declared == set(DEC.SIGNATURES), declared ^ set(DEC.SIGNATURES)
    lib = DEC.load()
    for name in declared:
        assert hasattr(lib, name), name


def test_json_reader(tmp_path):
    """The C++ JSON reader's own unit tests (tests/cpp/test_json.cpp), built with g++."""
    import shutil
    here = os.path.dirname(os.path.abspath(__file__))
    exe = str(tmp_path / "test_json")
    subprocess.check_call([shutil.which("g++") or "g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
                           "-I", os.path.join(os.path.dirname(here), "flashmlx_b200", "host"),
                           os.path.join(here, "cpp", "test_json.cpp"), "-o", exe])
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr


def test_decoder_checkpoint_with_a_dense_layer(tmp_path, fm_host):
    shape = S.DecoderShape("dec_mixed", 256, 3, 4, 2, 64, 320, 1e6, 1e-6,
                           S.MoEShape("dec_moe", 256, 128, 4, 2, 0, False, 256), dense_layers=(0,), intermediate=384)
    write_decoder_checkpoint(str(tmp_path), shape, S.make_decoder(shape, 54))
    got = json.loads(_run(fm_host, "check-decoder", tmp_path).stdout)
    assert got["moe_layers"] == [1, 2] and got["layers"] == 3
    assert _inspect(fm_host, tmp_path)["intermediate"] == 384


def test_decoder_checkpoint_with_qk_norm(tmp_path, fm_host):
    shape = S.DecoderShape("dec_qkn", 256, 2, 4, 2, 64, 320, 1e6, 1e-6,
                           S.MoEShape("dec_moe", 256, 128, 4, 2, 0, False, 256), attn_bias=False, qk_norm=True)
    write_decoder_checkpoint(str(tmp_path), shape, S.make_decoder(shape, 55))
    got = json.loads(_run(fm_host, "check-decoder", tmp_path).stdout)
    assert got["qk_norm"] and not got["attn_bias"]
