"""The legacy surface of sparse-ai's ``src/ultrametric/kernel.py`` that needs no GPU:
``routing_to_block_indices`` (kernel.py:152-191 there; each block is represented by its
FIRST token's argmax branch, whatever its docstring says about a majority vote) and the
refusal of ``CurriculumSparseAttention`` without the sparse backend (kernel.py:583-604)."""

import pytest
import torch

from ultrametric.kernel import CurriculumSparseAttention, routing_to_block_indices


def _one_hot_routes(B, H, S, L, p, seed):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, p, (B, H, S, L), generator=g)
    return ids, torch.nn.functional.one_hot(ids, p).float()


@pytest.mark.parametrize("S,block", [(512, 128), (200, 64), (64, 128), (130, 32)])
def test_routing_to_block_indices_takes_first_token(S, block):
    B, H, L, p = 2, 3, 5, 3
    ids, assign = _one_hot_routes(B, H, S, L, p, seed=S + block)
    got = routing_to_block_indices(assign, S, block)
    nb = -(-S // block)
    assert got.shape == (B, H, nb, L) and got.dtype == torch.int32
    for i in range(nb):
        assert torch.equal(got[:, :, i], ids[:, :, i * block].to(torch.int32))


def test_routing_to_block_indices_soft_assignments_use_argmax():
    g = torch.Generator().manual_seed(7)
    assign = torch.softmax(torch.randn(1, 2, 256, 4, 2, generator=g), dim=-1)
    got = routing_to_block_indices(assign, 256, 128)
    want = assign.argmax(-1)[:, :, ::128].to(torch.int32)
    assert torch.equal(got, want)


def test_routing_to_block_indices_pads_short_sequences_with_branch_zero():
    # S shorter than seq_len: the missing tokens are padded with branch 0 (kernel.py:179-181)
    ids, assign = _one_hot_routes(1, 1, 100, 2, 2, seed=3)
    got = routing_to_block_indices(assign, 300, 128)
    assert got.shape == (1, 1, 3, 2)
    assert torch.equal(got[0, 0, 0], ids[0, 0, 0].to(torch.int32))
    assert (got[0, 0, 1:] == 0).all()


def test_curriculum_without_sparse_backend_raises():
    q = torch.randn(1, 1, 16, 16)
    r = torch.zeros(1, 1, 1, 2, dtype=torch.int32)
    with pytest.raises(NotImplementedError):
        CurriculumSparseAttention.apply(q, q, q, r, 1, 2, False)
