"""The ternary oracle against the reference's own outputs (tests/golden/ternary.npz, made by
tests/golden/make_golden_ternary.py running sparse-ai's TernaryQuantize, pack_ternary,
unpack_ternary and its ternary Triton kernel under the CPU interpreter)."""

import numpy as np

from oracle import ternary_oracle as to


def test_quantize_pack_unpack_match_reference(golden):
    g = golden("ternary")
    codes, scale = to.quantize(g["q_x"])
    assert np.allclose(codes * scale[..., None], g["q_xq"], rtol=0, atol=1e-6)
    assert np.array_equal(to.pack(codes), g["q_packed"])
    assert np.array_equal(to.unpack(g["q_packed"]), g["q_unpacked"])


def test_ternary_attention_oracle_matches_reference_kernel(golden):
    g = golden("ternary")
    for i in range(3):
        key = f"t{i:02d}"
        Z, H, N, D, lw, rd, TD = (int(x) for x in g[key + "_meta"])
        out = to.ternary_attention(g[key + "_q"].astype(np.float32), g[key + "_kp"], g[key + "_vp"],
                                   g[key + "_ks"], g[key + "_vs"], g[key + "_router"], lw, rd)
        # the reference kernel rounds P to fp16 before P V and stores fp16 outputs
        assert np.abs(out.numpy() - g[key + "_out"]).max() < 2e-2, key
