"""Surgery routing -> block routes oracle (numpy on CPU; TEST INFRASTRUCTURE ONLY).

Restates the glue of sparse-ai's ``SurgicalLlamaAttention._block_list_prefill``
(src/llama_surgery/surgery.py:533-547) that turns router outputs into per-block routes:

* token-level assignments (B, H, S, levels, p): each token's branch per level is the argmax
  over p (first maximum wins); a route block's branch per level is the majority of its
  tokens' branches, ties going to the lowest branch id (argmax of the one-hot vote sums);
  tokens at or past S do not vote (the zero padding of surgery.py:545-546);
* block-level assignments (B, H, NB, levels, p) (surgery.py:533-538): the argmax per level.

Only the first ``r`` levels are used.  The lists then follow from ``block_list_oracle.
build_block_lists(routes, r, is_causal=True, sink_block=True, local_blocks, arity=p)``.
"""

from __future__ import annotations

import numpy as np


def token_branches(assign: np.ndarray, r: int) -> np.ndarray:
    """(B, H, S, levels, p) floats -> (B, H, S, r) argmax branch ids (first maximum)."""
    a = np.asarray(assign)[..., :r, :]
    return np.argmax(a, axis=-1).astype(np.int64)


def majority_routes(assign: np.ndarray, r: int, route_block: int, seq_len: int | None = None) -> np.ndarray:
    """Per-block majority vote of the token branches: (B, H, NB, r) int32."""
    B, H, S_all, _, p = np.asarray(assign).shape
    S = S_all if seq_len is None else seq_len
    idx = token_branches(np.asarray(assign)[:, :, :S], r)
    nb = -(-S // route_block)
    out = np.zeros((B, H, nb, r), dtype=np.int32)
    for i in range(nb):
        seg = idx[:, :, i * route_block:(i + 1) * route_block]          # (B, H, len, r)
        votes = np.stack([(seg == c).sum(axis=2) for c in range(p)], -1)  # (B, H, r, p)
        out[:, :, i] = np.argmax(votes, axis=-1)                         # ties -> lowest id
    return out


def block_level_routes(block_assign: np.ndarray, r: int) -> np.ndarray:
    """Block-level assignments (B, H, NB, levels, p) -> (B, H, NB, r) int32 argmax."""
    return token_branches(block_assign, r).astype(np.int32)
