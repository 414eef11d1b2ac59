"""The C++ host layer on the device: fm_host run (MoEModel::moe_block over a checkpoint
directory, C++ all the way to libflashmoe's C ABI) gives the same bf16 output as the same
layer's arrays run through the Python binding, for a Llama-family layer (fm_moe_block)
and a Nemotron-H 'E' layer (fm_moe_block_variant), and that output matches the CPU
oracle of the layer.  Top-2 layers: the fp32 sums of two routed rows do not depend on the
order the kernels add them in, so equality is exact."""
from __future__ import annotations

import subprocess

import numpy as np
import pytest
import torch

from flashmlx_b200 import synthetic as S
from tests.gpu_util import check_layer_vs_oracle, form_of
from tests.test_checkpoint import NEMO, SHAPE, _write_model, _write_nemotron

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fm_host():
    from flashmlx_b200 import build as fb
    return fb.build_host()


def _run_host(exe, model_dir, layer, x, out_dir):
    xp, yp = out_dir / "x.bin", out_dir / "y.bin"
    x.tofile(xp)
    r = subprocess.run([exe, "run", str(model_dir), str(layer), str(xp), str(x.shape[0]), str(yp),
                        str(torch.cuda.current_device())], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return np.fromfile(yp, dtype=np.uint16).reshape(x.shape)


@pytest.mark.parametrize("tokens", [5, 48])
def test_llama_layer(tmp_path, fm_host, tokens):
    from flashmlx_b200 import ops
    layer = S.make_layer(SHAPE, 41)
    (tmp_path / "m").mkdir()
    _write_model(str(tmp_path / "m"), layer)
    shape = SHAPE.with_tokens(tokens)
    x = S.make_x(shape, 41)
    y = _run_host(fm_host, tmp_path / "m", 0, x, tmp_path)
    ref, r = ops.MoEBlock(shape, ops.MoEWeightsT.from_numpy(layer, "cuda"))(ops.bf16_from_numpy(x, "cuda"),
                                                                          return_routing=True)
    torch.cuda.synchronize()
    form = form_of(ops.default_handle(torch.cuda.current_device()))  # same T, same path rule
    check_layer_vs_oracle(y, shape, layer, x, r, form, f"fm_host run T={tokens}")
    np.testing.assert_array_equal(y, ops.bf16_to_numpy(ref))


@pytest.mark.parametrize("tokens", [3, 40])
def test_nemotron_layer(tmp_path, fm_host, tokens):
    from flashmlx_b200 import ops
    layer = S.make_sigmoid_layer(NEMO, 42)
    (tmp_path / "m").mkdir()
    _write_nemotron(str(tmp_path / "m"), layer)
    shape = NEMO.with_tokens(tokens)
    x = S.make_x(shape, 42)
    y = _run_host(fm_host, tmp_path / "m", 3, x, tmp_path)
    routing = {"n_group": 2, "topk_group": 1, "routed_scaling_factor": 2.5}
    blk = ops.MoEBlockVariant.sigmoid_from_numpy(shape, layer, "cuda", **routing)
    ref, r = blk(ops.bf16_from_numpy(x, "cuda"), return_routing=True)
    torch.cuda.synchronize()
    form = form_of(ops.default_handle(torch.cuda.current_device()))
    check_layer_vs_oracle(y, shape, layer, x, r, form, f"fm_host run (Nemotron-H) T={tokens}",
                          sigmoid_routing=routing)
    np.testing.assert_array_equal(y, ops.bf16_to_numpy(ref))
