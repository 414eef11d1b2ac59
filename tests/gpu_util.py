"""Helpers for the GPU tests: numpy <-> torch device buffers, oracle comparisons."""
from __future__ import annotations

import numpy as np
import torch

from flashmlx_b200 import synthetic as S
from oracle import oracle as O
from tests._parity import EXACT_FLOOR, TIGHT, assert_close, near_tie_tokens, same_sets


def check_vs_oracle(y_bits, oracle_fn, what):
    """MLX has two arithmetic forms for a 4-bit product: qmm (large batches) rounds the
    dequantized weights to bf16 tiles, qmv (small batches) keeps them exact (affine split
    s*sum(q x) + b*sum(x) in fp32).  The tcgen05 path follows the first, the GEMV path the
    second.  The result must match one form within TIGHT and both within EXACT_FLOOR
    (the documented gap between the forms).  Returns (bf16-weights metrics, exact metrics)."""
    with O.weight_rounding(O.BF16_WEIGHTS):
        yt = oracle_fn()
    yt = yt[0] if isinstance(yt, tuple) else yt
    ye = oracle_fn()
    ye = ye[0] if isinstance(ye, tuple) else ye
    mt = assert_close(y_bits, yt, what + " [oracle, bf16 weights]", **EXACT_FLOOR)
    me = assert_close(y_bits, ye, what + " [oracle, exact weights]", **EXACT_FLOOR)
    best = min((mt, "bf16 weights"), (me, "exact weights"), key=lambda m: m[0]["mae_rel"])
    assert_close(y_bits, yt if best[1] == "bf16 weights" else ye, what + f" [oracle, {best[1]}, tight]", **TIGHT)
    return mt, me


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
        return host_bf16(y), {k: (host_bf16(v) if v.dtype == torch.bfloat16 else v.cpu().numpy())
                              for k, v in r.items()}

    def check(self, x_np: np.ndarray, what: str, sample: np.ndarray | None = None):
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
            x_np[rows], forced_ids=r["topk_ids"][rows], forced_scores=r["topk_scores"][rows]), what)
        return m, int(ties.sum())
