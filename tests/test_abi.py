"""CPU-side checks of the C ABI and the host logic (no compute calls)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import pisa_oracle as O

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "pisa_b200.h").read_text()
    return sorted(set(re.findall(r"PISA_API\s+[\w\s\*]+?\b(pisa_\w+)\(", text)))


def test_library_exports_every_header_symbol():
    from nlogn_pisa_b200 import _lib

    lib = _lib.lib()
    symbols = header_symbols()
    assert len(symbols) >= 10
    for name in symbols:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(symbols)
    assert lib.pisa_version() >= 100


def test_workspace_sizes_are_pure_host_functions():
    from nlogn_pisa_b200 import _lib

    lib = _lib.lib()
    n = lib.pisa_select_workspace_bytes(1, 32768, 32, 8, 128, 32768, 1, 2, 64, 2, 32, 4, 32, 0, 1)
    assert n >= 1 * (512 + 256 + 128 + 64 + 32) * 8 * 128 * 2 + 32768 * 8 * 64 * 9
    assert lib.pisa_select_workspace_bytes(1, 1, 32, 8, 128, 4096, 1, 2, 64, 2, 32, 1, 32, 1, 0) == 256
    assert lib.pisa_sparse_attn_bwd_workspace_bytes(1, 4, 4, 2, 64, 64, 100) >= 2 * 100 * 2 * 64 * 4


def test_invalid_arguments_report_status_without_gpu():
    """Argument checks run before any device work and map to ValueError."""
    from nlogn_pisa_b200 import _lib

    lib = _lib.lib()
    # topk 12 is outside {8,16,32,64}
    rc = lib.pisa_select_blocks(None, 0, 0, 0, None, 0, 0, 0, None, 0, None, None, 0, None, 0, 1, 1, 64,
                                4, 1, 64, 4096, 2, 64, 2, 12, 1, 1, 0, 16, 0, None, None, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED
    assert "topk" in _lib.lib().pisa_last_error().decode()
    with pytest.raises(ValueError):
        _lib.check(rc)


@pytest.mark.parametrize("blocks,topk,branching", [(64, 16, 2), (512, 32, 2), (4096, 32, 2), (20, 16, 2),
                                                   (512, 32, 4), (4096, 32, 4), (1000, 64, 2), (7, 8, 2)])
def test_routing_geometry_matches_oracle(blocks, topk, branching):
    from nlogn_pisa_b200.selection import routing_geometry

    assert routing_geometry(blocks, topk, branching) == O.routing_geometry(blocks, topk, branching)


def test_operators_reject_cpu_tensors():
    import nlogn_pisa_b200 as P

    q = torch.randn(1, 64, 4, 64)
    k = torch.randn(1, 64, 2, 64)
    with pytest.raises(ValueError, match="CUDA"):
        P.select_blocks(q, k, topk=8, block_size=16, force_recent=1)
    with pytest.raises(ValueError, match="CUDA"):
        P.sparse_attention(q, k, k, torch.zeros(1, 64, 2, 8, dtype=torch.long), block_size=16)
    with pytest.raises(ValueError, match="CUDA"):
        P.build_pyramid(k, 16)


def test_validation_contract():
    import nlogn_pisa_b200 as P

    q = torch.randn(1, 64, 3, 64)
    k = torch.randn(1, 64, 2, 64)
    with pytest.raises(ValueError, match="whole number"):
        P.select_blocks(q, k)
    q = torch.randn(1, 64, 4, 64)
    with pytest.raises(ValueError, match="method"):
        P.select_blocks(q, k, method="nope")
    with pytest.raises(ValueError, match="force_recent"):
        P.select_blocks(q, k, force_recent=0)
    with pytest.raises(ValueError, match="leaf_tile"):
        P.select_blocks(q, k, leaf_tile=3)
    with pytest.raises(ValueError, match="indices"):
        P.sparse_attention(q, k, k, torch.zeros(1, 64, 2, dtype=torch.long))


def test_cu_seqlens_contract():
    from nlogn_pisa_b200.validation import packed_queries, sequence_slices

    assert sequence_slices(torch.tensor([0, 5, 9]), 9) == [(0, 5), (5, 9)]
    with pytest.raises(ValueError):
        sequence_slices(torch.tensor([0, 5, 5, 9]), 9)
    q = torch.zeros(1, 2, 4, 8)
    k = torch.zeros(1, 9, 2, 8)
    assert list(packed_queries(q, k, torch.tensor([0, 5, 9]))) == [(0, 1, 0, 5, 4), (1, 2, 5, 9, 3)]


def test_kernel_timer_without_launches():
    """Reading a kernel timer that recorded nothing needs no device."""
    from nlogn_pisa_b200 import _lib

    assert _lib.kernel_time("attn_tiles") == (0.0, 0)
    lib = _lib.lib()
    assert lib.pisa_kernel_time(7, None, None) == _lib.ERR_INVALID
    _lib.kernel_timing(False)


def test_caller_pyramid_tables_are_validated_without_gpu():
    """Level tables that do not describe the keys' pyramid (another branching,
    other keys, too shallow) are rejected before any device work."""
    from nlogn_pisa_b200 import _lib

    lib = _lib.lib()
    N, C, K = 4096, 64, 16                      # 64 leaves: top 2 (b=2), 1 (b=4)
    binary = [64, 32, 16, 8, 4, 2, 1]
    offsets = np.cumsum([0] + binary[:-1]).tolist()

    def call(sizes, branching, top, first_width):
        rc = lib.pisa_select_blocks(
            None, 0, 0, 0, None, 0, 0, 0, ctypes.c_void_p(256), 0, _lib.int64_array(offsets),
            _lib.int64_array(sizes), len(sizes), None, 0, 1, 1, 64, 4, 1, 64, N, 2, C, branching, K, 1, 1,
            top, first_width, 0, ctypes.c_void_p(256), None, 0, None)
        return rc, _lib.lib().pisa_last_error().decode()

    # a binary pyramid read with branching 4
    rc, msg = call(binary, 4, 1, 16)
    assert rc == _lib.ERR_INVALID and "level sizes" in msg
    # sizes of other keys
    rc, msg = call([63, 32, 16, 8, 4, 2, 1], 2, 2, 16)
    assert rc == _lib.ERR_INVALID and "level sizes" in msg
    # shallower than the routing depth without reaching a single node
    rc, msg = call([64, 32], 2, 2, 16)
    assert rc == _lib.ERR_INVALID and "fewer levels" in msg


def test_bsa_entry_checks_run_on_the_host():
    """pisa_bsa_select rejects bad arguments before any device work; workspace is the leaf means."""
    from nlogn_pisa_b200 import _lib

    lib = _lib.lib()
    assert lib.pisa_bsa_workspace_bytes(1, 4096, 4, 64, _lib.BF16, 64, 0) == 64 * 4 * 64 * 2
    assert lib.pisa_bsa_workspace_bytes(1, 4096, 4, 64, _lib.BF16, 64, 1) == 0
    assert lib.pisa_bsa_workspace_bytes(0, 4096, 4, 64, _lib.BF16, 64, 0) == -1
    # 32 query heads per KV head exceed the 16-row warp tile
    rc = lib.pisa_bsa_select(None, 0, 0, 0, None, 0, 0, 0, None, 0, None, 0, _lib.BF16, 1, 64, 32, 1, 64, 64,
                             16, 8, 1, 2, None, None, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED and "16 query heads" in lib.pisa_last_error().decode()
    # last row (position 4095, block 255) needs block 0 plus 9 recent blocks: more than topk 8
    rc = lib.pisa_bsa_select(None, 0, 0, 0, None, 0, 0, 0, None, 0, None, 0, _lib.BF16, 1, 4096, 4, 4, 64,
                             4096, 16, 8, 1, 9, None, None, 0, None)
    assert rc == _lib.ERR_INVALID and "required" in lib.pisa_last_error().decode()


def test_bsa_required_block_count_matches_oracle():
    import numpy as np

    from nlogn_pisa_b200.selection import bsa_required_blocks

    for pos in (0, 15, 16, 47, 48, 1000):
        for ff in (True, False):
            for fr in (0, 1, 2, 3, 5):
                assert bsa_required_blocks(pos, 16, ff, fr) == O.bsa_required(np.array([[pos]]), 16, ff, fr)
