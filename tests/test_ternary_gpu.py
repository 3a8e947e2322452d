"""GPU checks of the ternary K/V path: quantise + pack and unpack + dequantise kernels
(integer codes bit-exact against the oracle; a value within 1e-5 relative of its threshold
may fall either way, since the fp32 mean |x| is summed in another order), and the ternary
prefill against the reference's outputs (tests/golden/ternary.npz) and the oracle at fp16
tolerance (2e-2 abs + 1e-2 rel)."""

import numpy as np
import pytest
import torch

from helpers import assert_half_close
from oracle import ternary_oracle as to
from ultrametric import _native as nat
from ultrametric.ternary import (TernaryQuantize, dequantize_ternary, pack_ternary,
                                 quantize_pack_ternary, ternary_ultrametric_attention_triton,
                                 unpack_ternary)

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_quantize_pack_matches_oracle(dtype):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(4, 33, 128, generator=g).to(dtype)
    packed, scale = quantize_pack_ternary(x.to(DEV))
    codes, ref_scale = to.quantize(x.float().numpy())
    assert np.allclose(scale.cpu().numpy(), ref_scale, rtol=1e-6, atol=0)
    got = to.unpack(packed.cpu().numpy())
    xf = np.abs(x.float().numpy())
    near = np.abs(xf - 0.5 * ref_scale[..., None]) <= 1e-5 * ref_scale[..., None]
    assert np.array_equal(got[~near], codes[~near])
    deq = dequantize_ternary(packed, scale, torch.float32).cpu().numpy()
    assert np.allclose(deq, got * scale.cpu().numpy()[..., None], rtol=0, atol=0)
    assert nat.read_device_status() == 0


def test_pack_unpack_roundtrip_and_quantize_matches_reference(golden):
    g = golden("ternary")
    codes = torch.from_numpy(g["q_unpacked"]).to(DEV)
    assert np.array_equal(pack_ternary(codes).cpu().numpy(), g["q_packed"])
    assert np.array_equal(unpack_ternary(torch.from_numpy(g["q_packed"]).to(DEV), codes.shape).cpu().numpy(),
                          g["q_unpacked"])
    xq = TernaryQuantize.apply(torch.from_numpy(g["q_x"]).to(DEV)).cpu().numpy()
    assert np.allclose(xq, g["q_xq"], rtol=0, atol=1e-6)


def test_ternary_attention_matches_reference(golden):
    g = golden("ternary")
    for i in range(3):
        key = f"t{i:02d}"
        Z, H, N, D, lw, rd, TD = (int(x) for x in g[key + "_meta"])
        t = {n: torch.from_numpy(g[f"{key}_{n}"]).to(DEV) for n in ("q", "kp", "vp", "ks", "vs", "router")}
        out = ternary_ultrametric_attention_triton(t["q"], t["kp"], t["vp"], t["ks"], t["vs"], t["router"],
                                                   local_window=lw, req_depth=rd)
        assert out.dtype == torch.float16 and out.shape == (Z, H, N, D)
        ref = to.ternary_attention(g[key + "_q"].astype(np.float32), g[key + "_kp"], g[key + "_vp"],
                                   g[key + "_ks"], g[key + "_vs"], g[key + "_router"], lw, rd)
        assert_half_close(out, ref, f"ternary {key} vs oracle")
        assert_half_close(out, torch.from_numpy(g[key + "_out"]).double(), f"ternary {key} vs reference")


def test_ternary_shift_is_rejected():
    q = torch.zeros(1, 1, 128, 64, dtype=torch.float16, device=DEV)
    kp = torch.zeros(1, 1, 128, 4, dtype=torch.int32, device=DEV)
    s = torch.ones(1, 1, 128, device=DEV)
    r = torch.zeros(1, 1, 1, 2, dtype=torch.int32, device=DEV)
    with pytest.raises(NotImplementedError):
        ternary_ultrametric_attention_triton(q, kp, kp, s, s, r, shift_size=64)
