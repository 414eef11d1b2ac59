"""The Nemotron-H / DeepSeek-style block (fm_moe_block_variant: sigmoid routing with a
correction bias and group-limited top-k, fp32 scaled scores, ungated relu^2 experts and
shared expert; server/src/nemotron_h.cpp:1010-1106) on the device against the CPU
oracle's restatement: the routing against the oracle's own routing where no near-tie
decides a pick, the block against the oracle under the device's routing."""
from __future__ import annotations


import numpy as np
import pytest
import torch

from flashmlx_b200 import synthetic as S
from oracle import oracle as O
from tests import numpy_ref as R
from tests.gpu_util import check_vs_oracle, form_of, host_bf16

pytestmark = pytest.mark.gpu


def _shape(tokens, shared):
    return S.MoEShape("sig", 512, 256, 32, 4, tokens, True, shared)


@pytest.mark.parametrize("tokens", [1, 7, 48, 300])
@pytest.mark.parametrize("groups", [(1, 1), (4, 2)])
@pytest.mark.parametrize("shared", [0, 256])
def test_sigmoid_block_vs_oracle(tokens, groups, shared):
    _check_sigmoid(_shape(tokens, shared), groups, 21)


@pytest.mark.parametrize("tokens", [1, 9, 300])
@pytest.mark.parametrize("widths", [(320, 0), (192, 448), (1856, 3712)])
def test_sigmoid_block_half_chunk_widths(tokens, widths):
    """Expert widths that are multiples of 64 but not 128 (Nemotron-3-Nano's 1856): the
    down matrices' K ends in a 64-wide half chunk with an odd number of quant groups
    per row; (192, 448) also splits the shared down's K over two work units."""
    inter, shared = widths
    _check_sigmoid(S.MoEShape("sig64", 512, inter, 32, 4, tokens, True, shared), (4, 2), 23)


def _check_sigmoid(shape, groups, seed):
    from flashmlx_b200 import ops
    tokens, shared = shape.tokens, shape.shared_inter
    layer = S.make_sigmoid_layer(shape, seed)
    x_np = S.make_x(shape, seed)
    routing = {"n_group": groups[0], "topk_group": groups[1], "routed_scaling_factor": 2.5}
    blk = ops.MoEBlockVariant.sigmoid_from_numpy(shape, layer, "cuda", **routing)
    x_dev = ops.bf16_from_numpy(x_np, "cuda")
    y, r = blk(x_dev, return_routing=True)
    torch.cuda.synchronize()
    ids = r["topk_ids"].cpu().numpy()
    sc = r["topk_scores_f32"].cpu().numpy()
    L = O.SigmoidLayer(shape, layer, routing)
    # routing: the same picks (as sets) and scores where the k-th pick is clear of the next
    oid, osc = L.route(x_np)
    _, _, sel = R.sigmoid_route(x_np, layer["router_w"], layer["correction_bias"], shape.top_k, groups[0],
                                groups[1], True, 2.5)
    srt = np.sort(sel, axis=-1)[:, ::-1]
    clear = np.abs(srt[:, shape.top_k - 1] - srt[:, shape.top_k]) > 5e-3
    assert clear.mean() > 0.6
    for t in np.nonzero(clear)[0]:
        assert set(ids[t]) == set(oid[t]), (t, ids[t], oid[t])
        dev = dict(zip(ids[t].tolist(), sc[t].tolist()))
        for e, s in zip(oid[t].tolist(), osc[t].tolist()):
            assert abs(dev[e] - s) <= 2e-2 * abs(s) + 1e-6, (t, e, dev[e], s)
    # the block under the device's routing (ids and fp32 scores as applied)
    check_vs_oracle(host_bf16(y), lambda: L.moe_block(x_np, forced_ids=ids, forced_scores=sc),
                    f"sigmoid block T={tokens} groups={groups} shared={shared}", form_of(blk.block._h(x_dev.device)))


def test_variant_rejects_bad_arguments():
    from flashmlx_b200 import ops
    from flashmlx_b200._lib import FlashMoEError
    shape = _shape(4, 0)
    layer = S.make_sigmoid_layer(shape, 22)
    x = ops.bf16_from_numpy(S.make_x(shape, 22), "cuda")
    with pytest.raises(FlashMoEError):  # 32 experts in 3 groups
        ops.MoEBlockVariant.sigmoid_from_numpy(shape, layer, "cuda", n_group=3, topk_group=1)(x)
    with pytest.raises(FlashMoEError):  # more groups kept than exist
        ops.MoEBlockVariant.sigmoid_from_numpy(shape, layer, "cuda", n_group=4, topk_group=5)(x)
    blk = ops.MoEBlockVariant.sigmoid_from_numpy(shape, layer, "cuda")
    blk.block.W.router_bias = blk.block.weights.router_w.data_ptr()  # a softmax-only logit bias
    with pytest.raises(FlashMoEError):
        blk(x)


@pytest.mark.parametrize("tokens", [48, 700])
@pytest.mark.parametrize("shared", [0, 256])
def test_sigmoid_block_tcgen05_path(tokens, shared):
    """The variant on the tcgen05 expert path (FM_PATH_TCGEN05): the relu^2 epilogue of
    the 2-CTA GEMM, bf16(d) per routed pair, the fp32-score combine."""
    from flashmlx_b200 import _lib, ops
    shape = _shape(tokens, shared)
    layer = S.make_sigmoid_layer(shape, 24)
    x_np = S.make_x(shape, 24)
    routing = {"n_group": 4, "topk_group": 2, "routed_scaling_factor": 2.5}
    blk = ops.MoEBlockVariant.sigmoid_from_numpy(shape, layer, "cuda", **routing)
    h = blk.block._h(torch.device("cuda"))
    h.set_path(_lib.FM_PATH_TCGEN05)
    try:
        y, r = blk(ops.bf16_from_numpy(x_np, "cuda"), return_routing=True)
        torch.cuda.synchronize()
    finally:
        h.set_path(_lib.FM_PATH_AUTO)
    L = O.SigmoidLayer(shape, layer, routing)
    ids, sc = r["topk_ids"].cpu().numpy(), r["topk_scores_f32"].cpu().numpy()
    assert form_of(h) == "bf16", "FM_PATH_TCGEN05 must run the tcgen05 expert path"
    check_vs_oracle(host_bf16(y), lambda: L.moe_block(x_np, forced_ids=ids, forced_scores=sc),
                    f"sigmoid block tcgen05 T={tokens} shared={shared}", "bf16")
