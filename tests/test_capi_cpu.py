"""CPU-side checks of the C ABI and the host layer (no GPU needed, no compute launched).

* the shared library loads and exports every function ``include/sparse_ai_b200.h`` declares;
* argument validation in the library returns SA_EINVAL with a message before any launch;
* the Python surface raises the reference's ValueErrors (block_list.py:199-206,1007-1029)
  and refuses CPU tensors instead of falling back.
"""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from ultrametric import _native as nat
from ultrametric import block_list_attention, build_block_lists, ultrametric_decode
from ultrametric.block_list import BlockLists

HEADER = Path(__file__).resolve().parent.parent / "include" / "sparse_ai_b200.h"


def declared_symbols():
    return sorted(set(re.findall(r"SA_API\s+[\w\s\*]+?\b(sa_\w+)\s*\(", HEADER.read_text())))


def test_header_symbols_exported():
    lib = nat.lib()
    syms = declared_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in the header but not exported"
    assert sorted(nat.exported_symbols()) == syms


def test_abi_version_and_workspace_sizes():
    lib = nat.lib()
    assert lib.sa_abi_version() == 3
    ws = lib.sa_block_list_attention_bwd_workspace_bytes(1, 32, 8, 8192, 128, 128)
    assert lib.sa_block_list_attention_fwd_workspace_bytes(1, 32, 8192, 128, 128) > 0
    NB = 64
    assert ws >= 32 * 8192 * 4 + 2 * 32 * NB * NB * 4
    assert lib.sa_ultrametric_decode_workspace_bytes(64, 32, 8, 128, 512) > 0
    assert lib.sa_ultrametric_decode_workspace_bytes(0, 32, 8, 128, 512) == 0


def test_library_rejects_bad_arguments_without_launch():
    lib = nat.lib()
    st = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    rc = lib.sa_build_block_lists(None, nat.SA_I32, st, 1, 1, 4, 2, None, 2, 1, 0, 0, 0, None, 4,
                                  None, None)
    assert rc == nat.SA_EINVAL
    assert b"null" in lib.sa_last_error()
    rc = lib.sa_block_list_attention_fwd(nat.SA_BF16, 1, 3, 2, 128, 64, 128, None, st, None, st,
                                         None, st, None, st, None, None, 0, None, None, 0, None, 0,
                                         1.0, None, 0, None)
    assert rc == nat.SA_EINVAL and b"multiple" in lib.sa_last_error()
    rc = lib.sa_block_list_attention_fwd(nat.SA_BF16, 1, 2, 2, 128, 48, 128, None, st, None, st,
                                         None, st, None, st, None, None, 0, None, None, 0, None, 0,
                                         1.0, None, 0, None)
    assert rc == nat.SA_EINVAL and b"power of two" in lib.sa_last_error()


def test_python_validation_matches_reference_errors():
    with pytest.raises(ValueError, match="router_indices must be"):
        build_block_lists(torch.zeros(2, 3, 4, dtype=torch.int32), 1)
    q = torch.zeros(1, 2, 64, 32)
    k = torch.zeros(1, 2, 48, 32)
    bl = BlockLists(torch.zeros(1, 2, 1, 1, dtype=torch.int32), torch.ones(1, 2, 1, dtype=torch.int32), 1)
    with pytest.raises(ValueError, match="must share shape"):
        block_list_attention(q, k, k, bl, route_block=64)
    with pytest.raises(ValueError, match="must share dtype"):
        block_list_attention(q, q.half(), q, bl, route_block=64)
    with pytest.raises(ValueError, match="head_dim must be a power of two"):
        block_list_attention(torch.zeros(1, 2, 64, 24), torch.zeros(1, 2, 64, 24),
                             torch.zeros(1, 2, 64, 24), bl, route_block=64)
    with pytest.raises(ValueError, match="route_block must be a power of two"):
        block_list_attention(q, q, q, bl, route_block=48)
    with pytest.raises(ValueError, match="block_lists built for"):
        block_list_attention(q, q, q, bl, route_block=32)
    with pytest.raises(ValueError, match="soft_block_bias must have shape"):
        block_list_attention(q, q, q, bl, route_block=64, soft_block_bias=torch.zeros(1, 2, 1, 2))


def test_no_cpu_fallback():
    q = torch.zeros(1, 2, 64, 32)
    bl = BlockLists(torch.zeros(1, 2, 1, 1, dtype=torch.int32), torch.ones(1, 2, 1, dtype=torch.int32), 1)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        block_list_attention(q, q, q, bl, route_block=64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        build_block_lists(torch.zeros(1, 1, 4, 2, dtype=torch.int32), 1, arity=2)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ultrametric_decode(torch.zeros(1, 2, 16), torch.zeros(2, 2, 4, 16), torch.zeros(2, 2, 4, 16),
                           torch.zeros(1, 2, dtype=torch.int32), torch.ones(1, dtype=torch.int32),
                           torch.zeros(2, 2, 3, dtype=torch.int32), torch.zeros(1, 2, 3, dtype=torch.int32), 1)


def test_invalid_depth_raises_before_launch():
    r = torch.zeros(1, 2, 4, 3, dtype=torch.int32)
    from ultrametric.block_list import _depth_list
    with pytest.raises(ValueError):
        _depth_list(4, 2, 3)
    with pytest.raises(ValueError):
        _depth_list([1, 2, 3], 2, 3)
    assert _depth_list([0, 3], 2, 3) == [0, 3]
