"""GPU parity of the operator entry points (fm_quantized_matmul, fm_gather_qmm) against
the CPU oracle, through the C ABI, on both expert-product paths."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from flashmlx_b200 import synthetic as S
from oracle import oracle as O
from tests.gpu_util import check_vs_oracle, dev_bf16, dev_u32, form_of, host_bf16

pytestmark = pytest.mark.gpu
KAT = np.load(os.path.join(os.path.dirname(__file__), "golden", "kat.npz"))
PATHS = {"gemv": 1, "tcgen05": 2}


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from flashmlx_b200 import ops as _ops
    return _ops


def run_qmm(ops, path, x, w, s, b, gs=64):
    h = ops.default_handle()
    h.set_path(path)
    try:
        y = ops.quantized_matmul(dev_bf16(x), dev_u32(w), dev_bf16(s), dev_bf16(b) if b is not None else None,
                                 group_size=gs)
        h.sync()
        return host_bf16(y)
    finally:
        h.set_path(0)


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
def test_kat_quantized_matmul(ops, path):
    for name in ("nibble_order", "group_bias"):
        x, w, s, b = (KAT[f"{name}_{k}"] for k in "xwsb")
        N = w.shape[0]
        if path == "gemv" and x.shape[1] % 128:
            continue  # the GEMV path works in 128-wide K chunks; K=64 runs on tcgen05
        # pad N to 16 rows is already the case (N = 16)
        y = run_qmm(ops, PATHS[path], x, w, s, b)
        np.testing.assert_array_equal(y, KAT[f"{name}_y"], err_msg=name)


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
@pytest.mark.parametrize("M,K,N,gs", [
    (1, 2048, 1408, 64), (7, 2048, 1408, 64), (32, 1408, 2048, 64), (33, 2048, 5632, 64),
    (300, 2048, 1408, 64), (513, 1408, 2048, 64), (64, 2048, 256, 32), (100, 2048, 384, 128),
    (100, 1408, 256, 128),  # 11 quant groups per row: the odd-count scale staging
])
def test_quantized_matmul_parity(ops, path, M, K, N, gs):
    rng = np.random.default_rng(M + K + N + gs)
    x = S.f32_to_bf16(rng.standard_normal((M, K), dtype=np.float32))
    w, s, b = S.make_qmatrix(M, f"qmm{K}{N}", (), N, K, gs)
    y = run_qmm(ops, PATHS[path], x, w, s, b, gs)
    mt, me = check_vs_oracle(y, lambda: O.quantized_matmul(x, w, s, b, group_size=gs),
                             f"quantized_matmul {path} M={M} K={K} N={N} gs={gs}", form_of(ops.default_handle()))
    print(f"qmm {path} M={M} K={K} N={N} gs={gs}: bf16-weights {mt} exact {me}")


@pytest.mark.parametrize("M,K,N,gs", [
    (1, 2048, 2048, 64),    # one decode row: 16 output units
    (4, 2048, 2560, 64),    # q|k|v-shaped
    (2, 1408, 2048, 128),   # K % 256 == 128: the last stage holds one 128-wide half
    (32, 2048, 1408, 64),   # 11 units x 2 row chunks
    (300, 2048, 1408, 64),
])
def test_linear_parity(ops, M, K, N, gs):
    """fm_linear (the decoder's dense projections, without the routing kernel) on the GEMV
    path against the oracle's quantized_matmul."""
    rng = np.random.default_rng(M * 7 + K + N + gs)
    x = S.f32_to_bf16(rng.standard_normal((M, K), dtype=np.float32))
    w, s, b = S.make_qmatrix(M, f"lin{K}{N}", (), N, K, gs)
    h = ops.default_handle()
    h.set_path(PATHS["gemv"])
    try:
        y = host_bf16(ops.linear(dev_bf16(x), dev_u32(w), dev_bf16(s), dev_bf16(b), group_size=gs))
        h.sync()
        check_vs_oracle(y, lambda: O.quantized_matmul(x, w, s, b, group_size=gs), f"linear M={M} K={K} N={N} gs={gs}",
                        form_of(h))
    finally:
        h.set_path(0)


def test_quantized_matmul_without_biases(ops):
    rng = np.random.default_rng(1)
    x = S.f32_to_bf16(rng.standard_normal((40, 1024), dtype=np.float32))
    w, s, _ = S.make_qmatrix(1, "nobias", (), 256, 1024)
    for path in PATHS.values():
        y = run_qmm(ops, path, x, w, s, None)
        check_vs_oracle(y, lambda: O.quantized_matmul(x, w, s, None), f"no-bias path {path}",
                        form_of(ops.default_handle()))


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
def test_kat_gather_qmm(ops, path):
    h = ops.default_handle()
    h.set_path(PATHS[path])
    try:
        x, w, s, b = (KAT[k] for k in ("gather_x", "gather_w", "gather_s", "gather_b"))
        rhs = KAT["gather_rhs"].reshape(4, 2)
        y = ops.gather_qmm(dev_bf16(x).view(4, 1, 1, 64), dev_u32(w), dev_bf16(s), dev_bf16(b),
                           rhs_indices=dev_u32(rhs))
        h.sync()
        np.testing.assert_array_equal(host_bf16(y).reshape(8, 1, 16), KAT["gather_y_bcast"])
        y = ops.gather_qmm(dev_bf16(x), dev_u32(w), dev_bf16(s), dev_bf16(b),
                           lhs_indices=dev_u32(KAT["gather_lhs"]), rhs_indices=dev_u32(KAT["gather_rhs"]))
        h.sync()
        np.testing.assert_array_equal(host_bf16(y), KAT["gather_y_lhs"])
    finally:
        h.set_path(0)


@pytest.mark.parametrize("path", ["gemv", "tcgen05"])
@pytest.mark.parametrize("T,k,sorted_idx", [(5, 4, False), (40, 4, True), (300, 2, True)])
def test_gather_qmm_parity(ops, path, T, k, sorted_idx):
    E, N, K = 8, 1408, 2048
    rng = np.random.default_rng(T * k)
    w, s, b = S.make_qmatrix(T, "gq", (E,), N, K)
    x = S.f32_to_bf16(rng.standard_normal((T, 1, 1, K), dtype=np.float32))
    rhs = rng.integers(0, E, size=(T, k)).astype(np.uint32)
    h = ops.default_handle()
    h.set_path(PATHS[path])
    try:
        if sorted_idx:  # the sorted call of switch_mlp: x gathered by order // k, rhs ascending
            order = np.argsort(rhs.ravel(), kind="stable")
            xs = x.reshape(T, 1, K)[order // k]
            rs = rhs.ravel()[order]
            y = ops.gather_qmm(dev_bf16(xs), dev_u32(w), dev_bf16(s), dev_bf16(b), rhs_indices=dev_u32(rs),
                               sorted_indices=True)
            h.sync()
            check_vs_oracle(host_bf16(y), lambda: O.gather_qmm(xs, w, s, b, None, rs), f"gather sorted {path}",
                            form_of(h))
        else:
            y = ops.gather_qmm(dev_bf16(x), dev_u32(w), dev_bf16(s), dev_bf16(b), rhs_indices=dev_u32(rhs))
            h.sync()
            assert tuple(y.shape) == (T, k, 1, N)
            check_vs_oracle(host_bf16(y).reshape(T * k, 1, N),
                            lambda: O.gather_qmm(x.reshape(T, 1, K), w, s, b, None, rhs.ravel()),
                            f"gather unsorted {path}", form_of(h))
    finally:
        h.set_path(0)


def test_argument_errors(ops):
    x = torch.zeros(4, 128, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(16, 16, dtype=torch.int32, device="cuda")
    s = torch.zeros(16, 2, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(NotImplementedError):
        ops.quantized_matmul(x, w, s, None, transpose=False)
    with pytest.raises(ValueError):
        ops.quantized_matmul(x.float(), w, s, None)
    with pytest.raises(ops.FlashMoEError) as ei:  # 8-bit is valid MLX but not implemented
        ops.quantized_matmul(x, torch.zeros(16, 32, dtype=torch.int32, device="cuda"), s, None, bits=8)
    assert ei.value.status == 2
