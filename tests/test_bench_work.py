"""The algorithmic work bench.py divides by a kernel's time for its roofline fraction,
against the figures derived independently for the BASELINE configs: configs[1] (the
4096-token Qwen1.5-MoE prefill layer) is 567,959,093,248 FLOP per layer call (routed
gate/up/down 283.47 G, shared expert 283.47 G, router and shared-expert gate 1.02 G), and a
Qwen1.5-MoE expert is 3 x 2048 x 1408 4-bit weights with bf16 scale and bias per 64 =
4,866,048 bytes."""
from __future__ import annotations

import numpy as np

import bench
from flashmlx_b200 import synthetic as S


def test_prefill_flops_match_the_layer_total():
    shape = S.CONFIGS["qwen15_prefill"]
    T = shape.tokens
    counts = np.full(shape.num_experts, T * shape.top_k // shape.num_experts)
    work, active = bench.kernel_work(shape, T, counts)
    assert active == shape.num_experts
    total = work["qgemm_tc_gateup"][0] + work["qgemm_tc_down"][0] + work["route"][0]
    assert total == 567_959_093_248
    assert work["qgemm_tc_gateup"][0] == 2 * work["qgemm_tc_down"][0]  # two matrices against one


def test_decode_bytes_count_the_active_experts_once():
    shape = S.CONFIGS["qwen15_decode"]
    T, H, I, Is = shape.tokens, shape.hidden, shape.inter, shape.shared_inter
    per_expert = 3 * H * I * (0.5 + 2 * 2 / 64)
    assert per_expert == 4_866_048
    for active in (1, 31, 53, 60):
        counts = np.zeros(shape.num_experts, int)
        counts[:active] = 1
        work, got = bench.kernel_work(shape, T, counts)
        assert got == active
        weights = work["qgemv_gateup"][1] + work["qgemv_down"][1]
        acts = (T * H * 2 + T * shape.top_k * I * 2 + T * Is * 2) + (T * shape.top_k * I * 2 + T * Is * 2 + T * H * 8)
        assert weights - acts == active * per_expert + 3 * H * Is * (0.5 + 2 * 2 / 64)


def test_decoder_step_bytes_grow_with_batch_and_position():
    shape = S.DECODER_CONFIGS["qwen15_decoder"]
    b1, b32 = bench.decoder_step_bytes(shape, 1, 600), bench.decoder_step_bytes(shape, 32, 600)
    assert b1 < b32 and bench.decoder_step_bytes(shape, 32, 100) < b32
    # batch 1 reads the attention projections, ~4 experts + the shared expert and router of
    # every layer, and the lm_head: between 1.3 and 1.6 GB
    assert 1.3e9 < b1 < 1.6e9


def test_expert_parallel_work_splits_the_layer():
    """Summed over ranks, the owner-side expert work of an expert-parallel step is the
    single-GPU layer's routed work plus one shared expert per rank (each rank runs it
    over its own tokens)."""
    shape = S.CONFIGS["qwen15_prefill"]
    T, k, E, world = shape.tokens, shape.top_k, shape.num_experts, 4
    per_rank_experts = E // world
    routed_rows = T * k  # every rank routes T tokens; rows spread evenly over the owners
    f_gu = f_dn = 0.0
    for _ in range(world):
        counts = np.full(world * per_rank_experts, routed_rows // (world * per_rank_experts))
        counts[: routed_rows - int(counts.sum())] += 1  # every owner receives T * k rows
        counts = counts.reshape(world, per_rank_experts)
        work, active = bench.ep_kernel_work(shape, T, int(counts.sum()), counts.ravel(), per_rank_experts)
        assert active == per_rank_experts
        f_gu += work["qgemm_tc_gateup"][0]
        f_dn += work["qgemm_tc_down"][0]
    single, _ = bench.kernel_work(shape, T, np.full(E, routed_rows // E))
    H, I, Is = shape.hidden, shape.inter, shape.shared_inter
    # world ranks x T tokens each: world x the single-GPU routed rows and shared expert
    assert f_gu == world * single["qgemm_tc_gateup"][0]
    assert f_dn == world * single["qgemm_tc_down"][0]
    assert single["qgemm_tc_down"][0] == 2.0 * T * k * I * H + 2.0 * T * Is * H


def test_layer_roofline_bound_and_work():
    """The whole-layer roofline: configs[1] prefill is tensor-bound on its 567,959,093,248
    FLOPs; configs[0] decode is HBM-bound on the bytes of the experts that receive tokens
    (4,866,048 B each), the shared expert, router, shared gate, x and y."""
    peaks = {"hbm_gbs": 6000.0, "bf16_tflops": 1500.0}
    pre = S.CONFIGS["qwen15_prefill"]
    r = bench.layer_roofline(pre, pre.tokens, np.full(pre.num_experts, 273), 1.0, peaks, "test")
    assert r["bound"] == "tensor" and r["algorithmic"] == 567_959_093_248
    assert abs(r["frac"] - 567_959_093_248 / 1.5e15 / 1e-3) < 1e-9
    dec = S.CONFIGS["qwen15_decode"]
    counts = np.zeros(dec.num_experts, int)
    counts[:53] = 2
    r = bench.layer_roofline(dec, dec.tokens, counts, 0.1, peaks, "test")
    want = 53 * 4_866_048 + 19_464_192 + 245_760 + 4_096 + 2 * 32 * 2048 * 2
    assert r["bound"] == "hbm" and r["algorithmic"] == want and r["active_experts"] == 53
    assert abs(r["achieved"] - want / 1e-4 / 1e9) < 1e-6
