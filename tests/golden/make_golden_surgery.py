"""Generate tests/golden/surgery_routing.npz by running the sparse-ai reference itself.

    TRITON_INTERPRET=1 python tests/golden/make_golden_surgery.py <reference-root>

It builds the reference's ``SurgicalLlamaAttention`` (the configuration of its own test,
tests/test_surgery_block_list.py:30-38 there) and calls ``_block_list_prefill``
(src/llama_surgery/surgery.py:520-598) on seeded router outputs, with
``ultrametric.block_list.build_block_lists`` wrapped so that the block routes the surgery
glue computed (the per-block majority vote of surgery.py:543-547, or the argmax of
block-level assignments, :533-538) and the lists the builder returned are recorded.  The
reference's Triton kernels run on the CPU under the interpreter.  Cases cover partial last
blocks, exact vote ties (resolved to the lowest branch id), three-way branches, block-level
assignments and several route depths.  Nothing at test time reads the reference.
"""

from __future__ import annotations

import math
import os
import sys
from types import SimpleNamespace

import numpy as np


def main(ref_root: str, out_path: str) -> None:
    assert os.environ.get("TRITON_INTERPRET") == "1", "run with TRITON_INTERPRET=1"
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    import ultrametric.block_list as bl_mod
    from llama_surgery.surgery import SurgicalLlamaAttention

    captured = {}
    real_build = bl_mod.build_block_lists

    def spy(router_indices, req_depth, **kw):
        out = real_build(router_indices, req_depth, **kw)
        captured.update(route=router_indices.clone(), depth=req_depth, kw=dict(kw), bl=out)
        return out

    bl_mod.build_block_lists = spy

    def make_attn(route_block, local_window, p):
        cfg = SimpleNamespace(
            hidden_size=64, num_attention_heads=2, num_key_value_heads=2, head_dim=32,
            max_position_embeddings=4096, surgical_p=p, surgical_init_mode="random",
            surgical_route_block=route_block, surgical_local_window=local_window,
            surgical_attention_backend="block_list", surgical_collect_stats=False,
        )
        return SurgicalLlamaAttention(cfg, layer_idx=0)

    out = {}
    cases = [
        # S, route_block, local_window, r, p, kind
        (200, 32, 16, 2, 2, "soft"),      # partial last block (8 tokens)
        (256, 64, 0, 3, 2, "soft"),
        (96, 32, 40, 1, 2, "soft"),
        (256, 32, 0, 4, 2, "tie"),        # every vote of level 1 ties 16:16
        (160, 32, 0, 3, 3, "soft"),       # three branches
        (192, 64, 64, 2, 3, "tie3"),      # three-way ties
        (384, 128, 16, 5, 2, "soft"),
        (320, 64, 0, 2, 2, "block"),      # block-level assignments (NB entries)
    ]
    for ci, (S, rb, lw, r, p, kind) in enumerate(cases):
        torch.manual_seed(1000 + ci)
        attn = make_attn(rb, lw, p)
        B, H, D = 1, 2, 32
        L = attn.router.levels
        q, k, v = (torch.randn(B, H, S, D) for _ in range(3))
        NB = -(-S // rb)
        g = torch.Generator().manual_seed(2000 + ci)
        if kind == "block":
            assign = torch.softmax(torch.randn(B, H, NB, L, p, generator=g), dim=-1)
        else:
            assign = torch.softmax(torch.randn(B, H, S, L, p, generator=g), dim=-1)
        if kind == "tie":
            # level 1: the first half of every block votes branch 0, the second half branch 1
            pos = torch.arange(S) % rb
            one = (pos >= rb // 2).long()
            assign[:, :, :, 1, :] = torch.nn.functional.one_hot(one, p).float().view(1, 1, S, p)
        if kind == "tie3":
            pos = torch.arange(S) % rb
            br = torch.where(pos < 21, 2, torch.where(pos < 42, 1, 0))  # 21 : 21 : 22 -> 0 wins
            br[(torch.arange(S) // rb) % 2 == 1] = torch.where(pos < 32, 1, 2)[(torch.arange(S) // rb) % 2 == 1]
            assign[:, :, :, 0, :] = torch.nn.functional.one_hot(br, p).float().view(1, 1, S, p)
        captured.clear()
        with torch.no_grad():
            if kind == "block":
                attn._block_list_prefill(q, k, v, assign.repeat_interleave(rb, dim=2)[:, :, :S], r,
                                         block_assignments=assign)
            else:
                attn._block_list_prefill(q, k, v, assign, r)
        key = f"s{ci:02d}"
        kw = captured["kw"]
        out[key + "_assign"] = assign.numpy().astype(np.float32)
        out[key + "_meta"] = np.array([S, rb, r, p, int(kw["local_blocks"]), int(kw["is_causal"]),
                                       int(kw["sink_block"]), int(kw["arity"]),
                                       1 if kind == "block" else 0], dtype=np.int64)
        out[key + "_route"] = captured["route"].numpy().astype(np.int32)
        out[key + "_lists"] = captured["bl"].lists.numpy().astype(np.int32)
        out[key + "_counts"] = captured["bl"].counts.numpy().astype(np.int32)
        print(key, S, rb, r, p, kind, "kept", int(captured["bl"].counts.sum()))
    np.savez_compressed(out_path, **out)


if __name__ == "__main__":
    here = os.path.dirname(os.path.abspath(__file__))
    main(sys.argv[1], os.path.join(here, "surgery_routing.npz"))
