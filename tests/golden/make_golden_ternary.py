"""Generate tests/golden/ternary.npz by running the sparse-ai reference itself.

    TRITON_INTERPRET=1 python tests/golden/make_golden_ternary.py <reference-root>

Records, for seeded inputs: the reference's ``TernaryQuantize`` forward and ``pack_ternary`` /
``unpack_ternary`` (src/llama_surgery/surgery.py:15-75), and the output of its
``ternary_ultrametric_attention_triton`` (src/llama_surgery/kernel.py:348-418, kernel
:147-249) -- the Triton kernel itself, run on the CPU by the interpreter -- on packed K/V
with per-token scales.  Nothing at test time reads the reference.
"""

from __future__ import annotations

import os
import sys

import numpy as np


def main(ref_root: str, out_path: str) -> None:
    assert os.environ.get("TRITON_INTERPRET") == "1", "run with TRITON_INTERPRET=1"
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    from llama_surgery.kernel import ternary_ultrametric_attention_triton
    from llama_surgery.surgery import TernaryQuantize, pack_ternary, unpack_ternary

    out = {}
    # quantisation + packing
    g = torch.Generator().manual_seed(7)
    x = torch.randn(3, 5, 64, generator=g)
    xq = TernaryQuantize.apply(x)
    gamma = x.abs().mean(-1, keepdim=True)
    xt = torch.round(xq / gamma)
    packed = pack_ternary(xt)
    out["q_x"] = x.numpy()
    out["q_xq"] = xq.numpy()
    out["q_packed"] = packed.numpy()
    out["q_unpacked"] = unpack_ternary(packed, tuple(xt.shape)).numpy()

    cases = [
        # Z, H, N, D, local_window, req_depth, TD
        (1, 2, 256, 64, 128, 1, 3),
        (1, 2, 384, 64, 0, 2, 4),
        (2, 1, 200, 32, 64, 1, 3),
    ]
    for ci, (Z, H, N, D, lw, rd, TD) in enumerate(cases):
        g = torch.Generator().manual_seed(100 + ci)
        q = torch.randn(Z, H, N, D, generator=g).half()
        kf = torch.randn(Z, H, N, D, generator=g)
        vf = torch.randn(Z, H, N, D, generator=g)
        ks = kf.abs().mean(-1)
        vs = vf.abs().mean(-1)
        kt = torch.round(TernaryQuantize.apply(kf) / ks.unsqueeze(-1))
        vt = torch.round(TernaryQuantize.apply(vf) / vs.unsqueeze(-1))
        kp, vp = pack_ternary(kt), pack_ternary(vt)
        BM = min(128, N)
        nb = -(-N // BM)
        router = torch.randint(0, 2, (Z, H, nb, TD), generator=g, dtype=torch.int32)
        o = ternary_ultrametric_attention_triton(q, kp, vp, ks.float(), vs.float(), router,
                                                 local_window=lw, req_depth=rd)
        key = f"t{ci:02d}"
        out[key + "_meta"] = np.array([Z, H, N, D, lw, rd, TD], dtype=np.int64)
        out[key + "_q"] = q.numpy()
        out[key + "_kp"] = kp.numpy()
        out[key + "_vp"] = vp.numpy()
        out[key + "_ks"] = ks.float().numpy()
        out[key + "_vs"] = vs.float().numpy()
        out[key + "_router"] = router.numpy()
        out[key + "_out"] = o.float().numpy()
        print(key, Z, H, N, D, lw, rd, float(o.float().abs().mean()))
    np.savez_compressed(out_path, **out)


if __name__ == "__main__":
    here = os.path.dirname(os.path.abspath(__file__))
    main(sys.argv[1], os.path.join(here, "ternary.npz"))
