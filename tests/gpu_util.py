"""Helpers for the GPU tests: numpy <-> torch device buffers, oracle comparisons."""
from __future__ import annotations

import numpy as np
import torch

from flashmlx_b200 import synthetic as S
from oracle import oracle as O
from tests._parity import EXACT_FLOOR, TIGHT, assert_close, near_tie_tokens, same_sets


FORM_OF_PATH = {1: "exact", 2: "bf16"}  # FM_PATH_GEMV, FM_PATH_TCGEN05


def form_of(handle) -> str:
    """The arithmetic form the handle's last expert-product call followed (fm_last_path)."""
    p = handle.last_path()
    assert p in FORM_OF_PATH, f"fm_last_path returned {p}"
    return FORM_OF_PATH[p]


def check_vs_oracle(y_bits, oracle_fn, what, form, tight=None):
    """MLX has two arithmetic forms for a 4-bit product: qmm (large batches) rounds the
    dequantized weights to bf16 tiles, qmv (small batches) keeps them exact (affine split
    s*sum(q x) + b*sum(x) in fp32).  The tcgen05 path follows the first ("bf16"), the
    GEMV path the second ("exact").  The result must match the form its path follows
    within TIGHT (north-star max_rel 1e-2, mae_rel 1e-3) and the other form within
    EXACT_FLOOR (the documented gap between the forms).  Prints both comparisons with the
    absolute MAE.  Returns (bf16-weights metrics, exact metrics)."""
    assert form in ("exact", "bf16"), form
    with O.weight_rounding(O.BF16_WEIGHTS):
        yt = oracle_fn()
    yt = yt[0] if isinstance(yt, tuple) else yt
    ye = oracle_fn()
    ye = ye[0] if isinstance(ye, tuple) else ye
    own, other = (ye, yt) if form == "exact" else (yt, ye)
    mo = assert_close(y_bits, own, what + f" [oracle, {form} form, tight]", **(tight or TIGHT))
    mx = assert_close(y_bits, other, what + " [oracle, other form]", **EXACT_FLOOR)
    print(f"PARITY {what} | form={form} max_rel={mo['max_rel']:.3e} mae={mo['mae']:.3e} "
          f"mae_rel={mo['mae_rel']:.3e} max_rel_elem={mo['max_rel_elem']:.3e} | other form "
          f"max_rel={mx['max_rel']:.3e} mae={mx['mae']:.3e}")
    return (mo, mx) if form == "bf16" else (mx, mo)


def check_layer_vs_oracle(y_bits, shape, layer_np, x_np, routing, form, what, sigmoid_routing=None):
    """A layer output produced outside GpuLayer (the model shim, the C++ host program)
    against the oracle: the device's routing (from a return_routing call on the same x)
    against the oracle's own (id sets, near-ties excluded), then y against the oracle
    evaluated on the device's ids and scores in `form`.  sigmoid_routing: the variant's
    routing dict (n_group, topk_group, routed_scaling_factor) for a Nemotron-H layer."""
    ids = routing["topk_ids"].cpu().numpy()
    if sigmoid_routing is None:
        sc = host_bf16(routing["topk_scores"])
        oids, _, _, pr = O.route(x_np, layer_np["router_w"], shape.top_k, norm_topk=shape.norm_topk_prob,
                                 router_bias=layer_np.get("router_bias"))
        ties = near_tie_tokens(pr, shape.top_k)
        assert (same_sets(ids, oids) | ties).all(), f"{what}: routing differs from the oracle"
        fn = lambda: O.Layer(shape, layer_np).moe_block(x_np, forced_ids=ids, forced_scores=sc)  # noqa: E731
    else:
        sc = routing["topk_scores_f32"].cpu().numpy()
        L = O.SigmoidLayer(shape, layer_np, sigmoid_routing)
        fn = lambda: L.moe_block(x_np, forced_ids=ids, forced_scores=sc)  # noqa: E731
    return check_vs_oracle(y_bits, fn, what, form)


def dev_bf16(a: np.ndarray, device="cuda") -> torch.Tensor:
    from flashmlx_b200.ops import bf16_from_numpy
    return bf16_from_numpy(a, device)


def dev_u32(a: np.ndarray, device="cuda") -> torch.Tensor:
    from flashmlx_b200.ops import u32_from_numpy
    return u32_from_numpy(a, device)


def host_bf16(t: torch.Tensor) -> np.ndarray:
    from flashmlx_b200.ops import bf16_to_numpy
    return bf16_to_numpy(t)


class GpuLayer:
    """A synthetic MoE layer resident on the GPU plus its oracle twin."""

    def __init__(self, shape, seed, device="cuda"):
        from flashmlx_b200 import ops
        self.shape = shape
        self.np = S.make_layer(shape, seed)
        self.weights = ops.MoEWeightsT.from_numpy(self.np, device)
        self.block = ops.MoEBlock(shape, self.weights)
        self.oracle = O.Layer(shape, self.np)

    def run(self, x_np: np.ndarray):
        x = dev_bf16(x_np)
        y, r = self.block(x, return_routing=True)
        torch.cuda.synchronize()
        from flashmlx_b200 import ops
        ops.synchronize()
        self.last_form = form_of(self.block._h(x.device))
        return host_bf16(y), {k: (host_bf16(v) if v.dtype == torch.bfloat16 else v.cpu().numpy())
                              for k, v in r.items()}

    def check(self, x_np: np.ndarray, what: str, sample: np.ndarray | None = None, tight: dict | None = None):
        """Routing vs the oracle (sets, near-ties excluded), permutation vs the oracle's
        stable sort of the same ids (exact), activations vs the oracle evaluated on the
        device's routing (all tokens, or a sample of rows)."""
        shape = self.shape
        y, r = self.run(x_np)
        k, E = shape.top_k, shape.num_experts
        ids, sc, lg, pr = O.route(x_np, self.np["router_w"], k, norm_topk=shape.norm_topk_prob,
                                  router_bias=self.np.get("router_bias"))
        ties = near_tie_tokens(pr, k)
        agree = same_sets(r["topk_ids"], ids)
        bad = ~agree & ~ties
        assert not bad.any(), f"{what}: {bad.sum()} tokens routed differently (near-ties excluded: {ties.sum()})"
        # ids in the same order (descending score, ties to the lower id) where the sets agree;
        # scores bit-exact except for the rare token whose fp32 router dot product (tensor-
        # core order vs CPU order) rounds one bf16 logit differently: <= 0.1% of tokens,
        # within 8 bf16 ulps (one logit ulp moves every renormalised top-8 score)
        ok = agree & ~ties
        np.testing.assert_array_equal(r["topk_ids"][ok], ids[ok])
        ds = np.abs(r["topk_scores"][ok].astype(np.int64) - sc[ok].astype(np.int64))
        off_tokens = np.count_nonzero(ds.max(axis=1) > 0) if ds.size else 0
        assert off_tokens <= max(1, int(1e-3 * ok.sum())), f"{what}: {off_tokens} tokens with different scores"
        assert ds.size == 0 or ds.max() <= 8, f"{what}: score differs by {ds.max()} ulps"
        # permutation: canonical stable expert-major order of the device's own ids
        st, sf, off = O.sort_pairs(r["topk_ids"], E)
        np.testing.assert_array_equal(r["expert_offsets"], off)
        np.testing.assert_array_equal(r["sorted_token"], st)
        rows = np.arange(x_np.shape[0]) if sample is None else sample
        m = check_vs_oracle(y[rows], lambda: self.oracle.moe_block(
            x_np[rows], forced_ids=r["topk_ids"][rows], forced_scores=r["topk_scores"][rows]), what,
            form=self.last_form, tight=tight)
        return m, int(ties.sum())
