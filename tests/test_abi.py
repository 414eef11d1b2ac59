"""CPU tests of the C ABI boundary: the library loads without a GPU, exports every
function include/flashmoe.h declares, and the ctypes struct layouts match the C
compiler's layout of the header's structs.  No compute call is made here."""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

from flashmlx_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flashmoe.h")


def header_functions():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"FM_API\s+[\w\s\*]+?\b(fm_\w+)\s*\(", txt)))


@pytest.fixture(scope="module")
def lib():
    from flashmlx_b200 import build
    build.build()  # no-op when up to date
    return _lib.load()


def test_header_declares_the_bound_functions():
    assert set(header_functions()) == set(_lib.SIGNATURES), (header_functions(), sorted(_lib.SIGNATURES))


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s(fm_\w+)$", out, re.M))
    missing = set(header_functions()) - exported
    assert not missing, missing
    # nothing beyond the ABI leaks out
    assert exported == set(header_functions()), exported - set(header_functions())


def test_enum_constants_match_the_header():
    """The Python constants of the header's enums (status codes, paths, routing forms)."""
    txt = open(HEADER).read()
    consts = dict((k, int(v)) for k, v in re.findall(r"\b(FM_[A-Z0-9_]+)\s*=\s*(\d+)", txt))
    for name in ("FM_PATH_AUTO", "FM_PATH_GEMV", "FM_PATH_TCGEN05", "FM_ROUTE_AUTO", "FM_ROUTE_GRID",
                 "FM_ROUTE_LAST_BLOCK", "FM_ROUTE_CLUSTER", "FM_OK", "FM_EINVAL"):
        assert consts[name] == getattr(_lib, name), name


def test_route_mode_is_checked_without_a_gpu(lib):
    assert lib.fm_set_route_mode(None, _lib.FM_ROUTE_LAST_BLOCK) == _lib.FM_EINVAL


def test_status_strings(lib):
    assert lib.fm_status_string(0) == b"ok"
    assert lib.fm_status_string(5) == b"device wait timed out"
    assert lib.fm_status_string(99) == b"unknown status"


def test_null_handle_is_rejected_without_a_gpu(lib):
    assert lib.fm_destroy(None) == _lib.FM_EINVAL
    assert lib.fm_sync_status(None) == _lib.FM_EINVAL
    assert lib.fm_moe_block(None, None, None, None, 0, None, None) == _lib.FM_EINVAL
    assert lib.fm_last_error(None) == b"null handle"


def test_struct_layout_matches_c_compiler():
    prog = r"""
#include <stdio.h>
#include <stddef.h>
#include "flashmoe.h"
int main(void) {
  printf("%zu %zu %zu %zu\n", sizeof(fm_qweight), sizeof(fm_moe_config), sizeof(fm_moe_weights), sizeof(fm_moe_outputs));
  printf("%zu %zu %zu %zu\n", offsetof(fm_moe_weights, gate), offsetof(fm_moe_weights, shared_down),
         offsetof(fm_moe_weights, shared_expert_gate_w), offsetof(fm_moe_weights, router_bias));
  printf("%zu %zu\n", offsetof(fm_moe_config, shared_inter), offsetof(fm_moe_outputs, expert_offsets));
  printf("%zu %zu\n", sizeof(fm_attn_config), offsetof(fm_attn_config, qkv_ld));
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "l.c"), os.path.join(d, "l")
        open(src, "w").write(prog)
        subprocess.check_call(["gcc", "-I", os.path.join(ROOT, "include"), src, "-o", exe])
        got = subprocess.run([exe], capture_output=True, text=True).stdout.split()
    got = [int(v) for v in got]
    want = [C.sizeof(_lib.QWeight), C.sizeof(_lib.MoEConfig), C.sizeof(_lib.MoEWeights), C.sizeof(_lib.MoEOutputs),
            _lib.MoEWeights.gate.offset, _lib.MoEWeights.shared_down.offset,
            _lib.MoEWeights.shared_expert_gate_w.offset, _lib.MoEWeights.router_bias.offset,
            _lib.MoEConfig.shared_inter.offset, _lib.MoEOutputs.expert_offsets.offset,
            C.sizeof(_lib.AttnConfig), _lib.AttnConfig.qkv_ld.offset]
    assert got == want


def test_oracle_structs_mirror_the_abi():
    from oracle import oracle as O
    assert [f[0] for f in O.MoEConfig._fields_] == [f[0] for f in _lib.MoEConfig._fields_]
    assert C.sizeof(O.MoEWeights) == C.sizeof(_lib.MoEWeights)


def test_workspace_size_is_a_host_query():
    """fm_workspace_size needs no device: it grows with the batch, covers both expert
    paths, and rejects invalid configs with 0."""
    import ctypes as C
    from flashmlx_b200 import _lib
    lib = _lib.load()
    cfg = _lib.MoEConfig(2048, 1408, 60, 4, 64, 4, 0, 5632, 0, 0)
    sizes = [lib.fm_workspace_size(C.byref(cfg), t) for t in (0, 1, 32, 4096, 16384)]
    assert all(s > 0 for s in sizes) and sizes == sorted(sizes) and sizes[-1] > sizes[0]
    assert all(s % (1 << 20) == 0 for s in sizes)  # whole MiB, as the handle allocates
    # 4096 tokens: at least the bf16 activations of every pair (y_pairs, P x H) are held
    assert sizes[3] >= 4096 * 4 * 2048 * 2
    bad = _lib.MoEConfig(0, 1408, 60, 4, 64, 4, 0, 5632, 0, 0)
    assert lib.fm_workspace_size(C.byref(bad), 32) == 0
    assert lib.fm_workspace_size(C.byref(cfg), -1) == 0
