"""An MoE layer loaded from an MLX-format checkpoint runs on the device exactly as the
same arrays uploaded directly (fm_moe_block, both expert paths), and the model shim's
output matches the CPU oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from flashmlx_b200 import checkpoint as CK
from flashmlx_b200 import synthetic as S
from tests.test_checkpoint import SHAPE, _write_model

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("path", [1, 2])  # FM_PATH_GEMV, FM_PATH_TCGEN05
def test_checkpoint_layer_on_device(tmp_path, path):
    from flashmlx_b200 import ops
    layer = S.make_layer(SHAPE, 11)
    _write_model(str(tmp_path), layer)
    ck = CK.Checkpoint(str(tmp_path))
    shape = ck.config.shape(48)
    x = ops.bf16_from_numpy(S.make_x(shape, 11), "cuda")
    h = ops.default_handle(torch.cuda.current_device())
    h.set_path(path)
    try:
        ya = ops.MoEBlock(shape, ops.MoEWeightsT.from_numpy(layer, "cuda"))(x)
        yb = ops.MoEBlock(shape, ops.MoEWeightsT.from_numpy(ck.moe_layer(0), "cuda"))(x)
        torch.cuda.synchronize()
    finally:
        h.set_path(0)
    np.testing.assert_array_equal(ops.bf16_to_numpy(ya), ops.bf16_to_numpy(yb))


def test_moe_model_forward(tmp_path):
    """MoEModel.moe_block(x, layer) over a [B, L, H] batch matches the CPU oracle of the
    layer (model.cpp:750-807) and equals fm_moe_block on the same arrays uploaded directly."""
    from flashmlx_b200 import ops
    from flashmlx_b200.model import MoEModel
    from tests.gpu_util import check_layer_vs_oracle, form_of
    layer = S.make_layer(SHAPE, 12)
    _write_model(str(tmp_path), layer)
    m = MoEModel(str(tmp_path), device="cuda", max_tokens=64)
    x_np = S.make_x(SHAPE.with_tokens(48), 12)
    x = ops.bf16_from_numpy(x_np, "cuda")
    y = m.moe_block(x.view(2, 24, SHAPE.hidden), 0)
    assert y.shape == (2, 24, SHAPE.hidden)
    y_np = ops.bf16_to_numpy(y.reshape(48, -1))
    ref, r = ops.MoEBlock(SHAPE, ops.MoEWeightsT.from_numpy(layer, "cuda"))(x, return_routing=True)
    torch.cuda.synchronize()
    form = form_of(ops.default_handle(torch.cuda.current_device()))  # same T, same path rule
    check_layer_vs_oracle(y_np, SHAPE, layer, x_np, r, form, "MoEModel.moe_block")
    np.testing.assert_array_equal(y_np, ops.bf16_to_numpy(ref))
