"""MLX-format checkpoints of an MoE model (config.json + safetensors shards), read into the
stacked per-layer arrays libflashmoe takes.

Follows the reference's loader for the MoE layers:
  load_config            LlamaModel::load_config (server/src/model.cpp:105-142): hidden_size,
                         num_hidden_layers, num_experts, num_experts_per_tok,
                         moe_intermediate_size, shared_expert_intermediate_size,
                         norm_topk_prob and the nested "quantization" {bits, group_size},
                         with the same defaults
  Checkpoint             LlamaModel::load_weights (148-184): every *.safetensors file of the
                         directory in sorted order, later files overriding earlier keys,
                         a leading "model." (or Nemotron-H's "backbone.") stripped from
                         every key
  Checkpoint.moe_layer   build_moe_weight_cache (368-470): a layer is MoE when it has
                         layers.N.mlp.gate.weight; the experts'
                         experts.E.{gate,up,down}_proj.{weight,scales,biases} are stacked
                         along a new leading expert axis (biases optional), the shared
                         expert is shared_expert.{gate,up,down}_proj.* and its gate
                         shared_expert_gate.weight
Checkpoints written by mlx-lm keep the experts pre-stacked as
layers.N.mlp.switch_mlp.{gate,up,down}_proj.*; those are taken as they are.

Nemotron-H checkpoints (NemotronHModel, server/src/nemotron_h.cpp: config 244-261,
pattern 272-285, MoE weights 444-468) mark their MoE layers 'E' in
hybrid_override_pattern and keep them under layers.N.mixer: gate.weight,
gate.e_score_correction_bias, switch_mlp.fc1 / fc2 (stacked), shared_experts.up_proj /
down_proj; Checkpoint.sigmoid_moe_layer() reads one into the layout of
synthetic.make_sigmoid_layer for ops.MoEBlockVariant.

The result of moe_layer() has the layout of synthetic.make_layer (bf16 as uint16 bits,
packed codes as uint32; arrays the layer owns), so ops.MoEWeightsT.from_numpy(layer,
device) uploads it.  Tensors are memory-mapped, not read, until a layer is stacked.  A
quantized router or shared-expert gate (gate.scales / shared_expert_gate.scales present)
raises NotImplementedError, as the C ABI returns FM_EUNSUPPORTED for it.
"""
from __future__ import annotations

import dataclasses
import glob
import json
import os
import struct

import numpy as np

from .synthetic import MoEShape

__all__ = ["read_safetensors", "write_safetensors", "MoEModelConfig", "load_config", "Checkpoint"]

# safetensors dtype names -> numpy storage (bf16 is kept as its uint16 bit pattern)
_DTYPES = {
    "BOOL": np.bool_, "U8": np.uint8, "I8": np.int8, "U16": np.uint16, "I16": np.int16,
    "U32": np.uint32, "I32": np.int32, "U64": np.uint64, "I64": np.int64,
    "F16": np.float16, "BF16": np.uint16, "F32": np.float32, "F64": np.float64,
}
_NAMES = {np.dtype(np.bool_): "BOOL", np.dtype(np.uint8): "U8", np.dtype(np.int8): "I8",
          np.dtype(np.int16): "I16", np.dtype(np.uint32): "U32", np.dtype(np.int32): "I32",
          np.dtype(np.uint64): "U64", np.dtype(np.int64): "I64", np.dtype(np.float16): "F16",
          np.dtype(np.float32): "F32", np.dtype(np.float64): "F64"}


def read_safetensors(path: str) -> tuple[dict[str, tuple[str, np.ndarray]], dict]:
    """{name: (safetensors dtype, array)} memory-mapped from the file, and its metadata.
    The format: an 8-byte little-endian header length, a JSON header mapping each name
    to {dtype, shape, data_offsets [begin, end)} relative to the data that follows."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file (short header)")
        n = struct.unpack("<Q", raw)[0]
        if n > size - 8:
            raise ValueError(f"{path}: header length {n} exceeds the file")
        header = json.loads(f.read(n))
    data_size = size - 8 - n
    mm = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n, shape=(data_size,)) if data_size else None
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = info["dtype"]
        if dt not in _DTYPES:
            raise ValueError(f"{path}: {name}: unsupported dtype {dt}")
        beg, end = info["data_offsets"]
        shape = tuple(int(v) for v in info["shape"])
        nbytes = int(np.prod(shape, dtype=np.int64)) * np.dtype(_DTYPES[dt]).itemsize
        if not 0 <= beg <= end <= data_size or end - beg != nbytes:
            raise ValueError(f"{path}: {name}: data_offsets {beg}..{end} do not hold {dt}{list(shape)}")
        arr = mm[beg:end].view(_DTYPES[dt]).reshape(shape) if nbytes else np.zeros(shape, _DTYPES[dt])
        out[name] = (dt, arr)
    return out, header.get("__metadata__", {})


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Writes {name: array or (safetensors dtype, array)}; a bare uint16 array is
    written as BF16 (bf16 bit patterns are this library's uint16 arrays)."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        v = tensors[name]
        dt, arr = v if isinstance(v, tuple) else (None, v)
        arr = np.ascontiguousarray(arr)
        if dt is None:
            dt = "BF16" if arr.dtype == np.uint16 else _NAMES.get(arr.dtype)
            if dt is None:
                raise ValueError(f"{name}: no safetensors dtype for {arr.dtype}")
        if np.dtype(_DTYPES[dt]).itemsize != arr.dtype.itemsize:
            raise ValueError(f"{name}: {dt} does not match an array of {arr.dtype}")
        b = arr.tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)  # the data starts 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


@dataclasses.dataclass(frozen=True)
class MoEModelConfig:
    hidden: int
    num_layers: int
    num_experts: int
    top_k: int
    inter: int
    shared_inter: int
    norm_topk_prob: bool
    bits: int
    group_size: int
    # Nemotron-H / DeepSeek-style routing (defaults: off)
    n_group: int = 1
    topk_group: int = 1
    routed_scaling_factor: float = 1.0
    hybrid_override_pattern: str = ""

    @property
    def sigmoid_routed(self) -> bool:
        """A Nemotron-H model (MoE layers marked 'E' in hybrid_override_pattern)."""
        return "E" in self.hybrid_override_pattern

    def routing(self) -> dict:
        """The variant's routing parameters (ops.MoEBlockVariant keyword arguments)."""
        return {"n_group": self.n_group, "topk_group": self.topk_group,
                "routed_scaling_factor": self.routed_scaling_factor}

    def shape(self, tokens: int, name: str = "checkpoint") -> MoEShape:
        """The layer shape for a batch of `tokens` (the MoEBlock / bench description)."""
        return MoEShape(name, self.hidden, self.inter, self.num_experts, self.top_k, tokens, self.norm_topk_prob,
                        self.shared_inter, 0.0, self.group_size, self.bits)


def load_config(model_dir: str) -> MoEModelConfig:
    """config.json of the model directory, with the reference's defaults for absent keys."""
    with open(os.path.join(model_dir, "config.json")) as f:
        c = json.load(f)
    q = c.get("quantization")
    if not isinstance(q, dict):
        q = {}
    pattern = c.get("hybrid_override_pattern") or ""
    return MoEModelConfig(
        hidden=int(c.get("hidden_size", 4096)),
        num_layers=int(c.get("num_hidden_layers", 32)),
        num_experts=int(c.get("num_experts", 0) or c.get("n_routed_experts", 0)),
        top_k=int(c.get("num_experts_per_tok", 0)),
        inter=int(c.get("moe_intermediate_size", 0)),
        shared_inter=int(c.get("shared_expert_intermediate_size", 0) or
                         (c.get("moe_shared_expert_intermediate_size", 0) if c.get("n_shared_experts", 1) else 0)),
        norm_topk_prob=bool(c.get("norm_topk_prob", False)),
        bits=int(q.get("bits", 0)),
        group_size=int(q.get("group_size", 64)),
        n_group=int(c.get("n_group", 1)),
        topk_group=int(c.get("topk_group", 1)),
        routed_scaling_factor=float(c.get("routed_scaling_factor", 1.0)),
        hybrid_override_pattern=str(pattern),
    )


class Checkpoint:
    """The tensors of every *.safetensors file in a model directory (memory-mapped)."""

    def __init__(self, model_dir: str):
        self.dir = model_dir
        self.config = load_config(model_dir)
        files = sorted(glob.glob(os.path.join(model_dir, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no .safetensors files in {model_dir}")
        self.tensors: dict[str, tuple[str, np.ndarray]] = {}
        for path in files:
            t, _ = read_safetensors(path)
            for key, v in t.items():
                # "model." (LlamaModel::load_weights) or "backbone." (NemotronHModel, 333-337)
                for pre in ("model.", "backbone."):
                    if key.startswith(pre):
                        key = key[len(pre):]
                        break
                self.tensors[key] = v

    def has(self, key: str) -> bool:
        return key in self.tensors

    def get(self, key: str, dtype: str | None = None) -> np.ndarray:
        if key not in self.tensors:
            raise KeyError(f"{self.dir}: tensor {key} missing")
        dt, arr = self.tensors[key]
        if dtype is not None and dt != dtype:
            raise ValueError(f"{key}: {dt}, expected {dtype}")
        return arr

    def moe_layers(self) -> list[int]:
        """Indices of the layers with a router: layers.N.mlp.gate.weight, or for a
        Nemotron-H model the 'E' layers of hybrid_override_pattern (layers.N.mixer)."""
        c = self.config
        if c.sigmoid_routed:
            if len(c.hybrid_override_pattern) != c.num_layers:
                raise ValueError("hybrid_override_pattern length differs from num_hidden_layers")
            return [i for i, b in enumerate(c.hybrid_override_pattern) if b == "E"]
        return [i for i in range(c.num_layers) if self.has(f"layers.{i}.mlp.gate.weight")]

    def sigmoid_moe_layer(self, i: int) -> dict:
        """Nemotron-H MoE layer i in the layout of synthetic.make_sigmoid_layer."""
        c = self.config
        mx = f"layers.{i}.mixer"
        if not self.has(mx + ".gate.weight"):
            raise KeyError(f"layer {i} has no router ({mx}.gate.weight)")
        if self.has(mx + ".gate.scales"):
            raise NotImplementedError(f"{mx}.gate is quantized: a quantized router is not implemented")
        if c.bits != 4:
            raise NotImplementedError(f"quantization bits = {c.bits}: only 4-bit affine weights are implemented")
        d = {"router_w": np.array(self.get(mx + ".gate.weight", "BF16"))}
        if self.has(mx + ".gate.e_score_correction_bias"):
            dt, arr = self.tensors[mx + ".gate.e_score_correction_bias"]
            if dt == "F32":
                d["correction_bias"] = np.array(arr, np.float32)
            elif dt == "BF16":
                d["correction_bias"] = (np.asarray(arr, np.uint32) << 16).view(np.float32).copy()
            else:
                raise ValueError(f"{mx}.gate.e_score_correction_bias: {dt}, expected F32 or BF16")
        d["fc1"] = self._qmatrix(mx + ".switch_mlp.fc1")
        d["fc2"] = self._qmatrix(mx + ".switch_mlp.fc2")
        if self.has(mx + ".shared_experts.up_proj.weight"):
            d["shared_up"] = self._qmatrix(mx + ".shared_experts.up_proj")
            d["shared_down"] = self._qmatrix(mx + ".shared_experts.down_proj")
        E, H, I, Is, gs, pw = c.num_experts, c.hidden, c.inter, c.shared_inter, c.group_size, 32 // c.bits
        shapes = {"router_w": (E, H), "fc1": (E, I, H), "fc2": (E, H, I), "shared_up": (Is, H), "shared_down": (H, Is)}
        for key, shp in shapes.items():
            if key not in d:
                if key.startswith("shared") and Is:
                    raise ValueError(f"layer {i}: config has a shared expert ({Is}) but the checkpoint has none")
                continue
            if key == "router_w":
                got, want = d[key].shape, shp
            else:
                got = d[key][0].shape + d[key][1].shape[-1:]
                want = shp[:-1] + (shp[-1] // pw, shp[-1] // gs)
            if tuple(got) != tuple(want):
                raise ValueError(f"layer {i} {key}: shape {tuple(got)}, config gives {tuple(want)}")
        if "correction_bias" in d and d["correction_bias"].shape != (E,):
            raise ValueError(f"layer {i} correction bias: shape {d['correction_bias'].shape}, config gives ({E},)")
        return d

    def _qmatrix(self, prefix: str) -> tuple[np.ndarray, np.ndarray, np.ndarray | None]:
        # copies: a stacked layer owns its arrays (the mapped file stays read-only)
        w = np.array(self.get(prefix + ".weight", "U32"))
        s = np.array(self.get(prefix + ".scales", "BF16"))
        b = np.array(self.get(prefix + ".biases", "BF16")) if self.has(prefix + ".biases") else None
        return w, s, b

    def _stacked(self, mlp: str, proj: str) -> tuple[np.ndarray, np.ndarray, np.ndarray | None]:
        pre = f"{mlp}.switch_mlp.{proj}"
        if self.has(pre + ".weight"):  # mlx-lm layout: already [E, ...]
            return self._qmatrix(pre)
        E = self.config.num_experts
        parts = [self._qmatrix(f"{mlp}.experts.{e}.{proj}") for e in range(E)]
        if any((p[2] is None) != (parts[0][2] is None) for p in parts):
            raise ValueError(f"{mlp}.experts.*.{proj}: biases present for some experts only")
        w = np.stack([p[0] for p in parts])
        s = np.stack([p[1] for p in parts])
        b = np.stack([p[2] for p in parts]) if parts[0][2] is not None else None
        return w, s, b

    def moe_layer(self, i: int) -> dict:
        """Layer i's MoE weights in the layout of synthetic.make_layer."""
        c = self.config
        mlp = f"layers.{i}.mlp"
        if not self.has(mlp + ".gate.weight"):
            raise KeyError(f"layer {i} has no router ({mlp}.gate.weight): not an MoE layer")
        if self.has(mlp + ".gate.scales"):
            raise NotImplementedError(f"{mlp}.gate is quantized: a quantized router is not implemented")
        if c.bits != 4:
            raise NotImplementedError(f"quantization bits = {c.bits}: only 4-bit affine weights are implemented")
        d = {"router_w": np.array(self.get(mlp + ".gate.weight", "BF16"))}
        for proj, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
            d[key] = self._stacked(mlp, proj)
        if self.has(mlp + ".shared_expert.gate_proj.weight"):
            for proj, key in (("gate_proj", "shared_gate"), ("up_proj", "shared_up"), ("down_proj", "shared_down")):
                d[key] = self._qmatrix(f"{mlp}.shared_expert.{proj}")
            if self.has(mlp + ".shared_expert_gate.scales"):
                raise NotImplementedError(f"{mlp}.shared_expert_gate is quantized: not implemented")
            d["shared_expert_gate_w"] = np.array(self.get(mlp + ".shared_expert_gate.weight", "BF16")).reshape(1, -1)
        self._check(i, d)
        return d

    def _check(self, i: int, d: dict) -> None:
        c = self.config
        E, H, I, Is, gs = c.num_experts, c.hidden, c.inter, c.shared_inter, c.group_size
        per_word = 32 // c.bits

        def want(name, arr, shape):
            if tuple(arr.shape) != tuple(shape):
                raise ValueError(f"layer {i} {name}: shape {tuple(arr.shape)}, config gives {tuple(shape)}")

        want("router", d["router_w"], (E, H))
        for key, n, k in (("gate", I, H), ("up", I, H), ("down", H, I)):
            w, s, b = d[key]
            want(key + ".weight", w, (E, n, k // per_word))
            want(key + ".scales", s, (E, n, k // gs))
            if b is not None:
                want(key + ".biases", b, (E, n, k // gs))
        if "shared_gate" in d:
            for key, n, k in (("shared_gate", Is, H), ("shared_up", Is, H), ("shared_down", H, Is)):
                w, s, b = d[key]
                want(key + ".weight", w, (n, k // per_word))
                want(key + ".scales", s, (n, k // gs))
            want("shared_expert_gate", d["shared_expert_gate_w"], (1, H))
        elif Is:
            raise ValueError(f"layer {i}: config has a shared expert ({Is}) but the checkpoint has none")
