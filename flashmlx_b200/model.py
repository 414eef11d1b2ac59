"""The MoE layers of an MLX-format checkpoint on one GPU, called the way the reference's
decoder layer calls them (LlamaModel, and NemotronHModel's 'E' layers through the
sigmoid-routed variant).

LlamaModel's layer (server/src/model.cpp:825-839) normalises the attention output and
dispatches the MLP: moe_block(normed, layer) when the layer has a router
(layer_is_moe_, model.cpp:253-266), else the dense mlp.  MoEModel holds every MoE layer's
weights on the device (stacked by checkpoint.Checkpoint) and answers that call through
libflashmoe's fm_moe_block; the attention, norms and dense MLP stay with the caller.
"""
from __future__ import annotations

import torch

from . import ops
from .checkpoint import Checkpoint

__all__ = ["MoEModel"]


class MoEModel:
    """MoE blocks of a checkpoint directory.  `max_tokens` (optional) sizes the handle's
    workspace once, so later calls up to that many tokens do not allocate."""

    def __init__(self, model_dir: str, device: str | torch.device = "cuda", max_tokens: int | None = None,
                 layers: list[int] | None = None, handle: ops.Handle | None = None):
        self.checkpoint = Checkpoint(model_dir)
        self.config = self.checkpoint.config
        self.device = torch.device(device)
        moe = self.checkpoint.moe_layers()
        if layers is not None:
            missing = sorted(set(layers) - set(moe))
            if missing:
                raise KeyError(f"layers {missing} are not MoE layers of {model_dir}")
            moe = sorted(layers)
        self.shape = self.config.shape(max_tokens or 1, name=model_dir)
        if self.config.sigmoid_routed:  # Nemotron-H: NemotronHModel::moe_block through fm_moe_block_variant
            self.blocks = {i: ops.MoEBlockVariant.sigmoid_from_numpy(self.shape, self.checkpoint.sigmoid_moe_layer(i),
                                                                     self.device, handle=handle,
                                                                     **self.config.routing())
                           for i in moe}
        else:
            self.blocks = {i: ops.MoEBlock(self.shape,
                                           ops.MoEWeightsT.from_numpy(self.checkpoint.moe_layer(i), self.device), handle)
                           for i in moe}
        if max_tokens and self.blocks:
            first = next(iter(self.blocks.values()))
            (first.block if isinstance(first, ops.MoEBlockVariant) else first).reserve(max_tokens, self.device)

    def is_moe(self, layer: int) -> bool:
        """layer_is_moe_[layer]: the layer has a router and its experts are loaded."""
        return layer in self.blocks

    def moe_block(self, x: torch.Tensor, layer: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """LlamaModel::moe_block(x, layer): x [..., hidden] bf16 on the device -> same shape."""
        if layer not in self.blocks:
            raise KeyError(f"layer {layer} is not an MoE layer")
        lead = x.shape[:-1]
        y = self.blocks[layer](x.reshape(-1, x.shape[-1]), out=None if out is None else out.reshape(-1, x.shape[-1]))
        return y.reshape(*lead, x.shape[-1])
